// Plain-old-data argument blocks shared by the host launchers and the
// kernels.  Everything is passed by value as kernel parameters.
#pragma once

#include <cstdint>

namespace kvs {

constexpr int kMaxHeads = 16;   // KV heads per rank handled by one launch
constexpr int kHeadDim = 128;   // the fused kernels are specialised for D=128
constexpr int kTileRows = 128;  // tokens per tile

// Paged KV source/destination: element (block, slot, head, d) of plane kv
// lives at base + block*block_stride + kv*kv_stride + (slot*H + head)*D + d
// (element units, bf16).  Covers [2, nb, bs, H, D] (FlashAttention) and
// [nb, 2, bs, H, D] (FlashInfer) layouts.
struct PagedKV {
  const void* base;
  long long block_stride;
  long long kv_stride;
  int num_blocks;
  int block_size;
};

// Per-request tables of one launch (all device pointers).
struct ReqTable {
  const int32_t* block_table;  // concatenated physical block ids
  const int32_t* bt_off;       // [R] first entry of request r
  const int32_t* n_tokens;     // [R] valid tokens (statistics, written rows)
  const int32_t* n_rows;       // [R] rows = blocks * block_size
  const int32_t* tile_prefix;  // [R+1] cumulative 128-row tiles
  const long long* code_off;   // [R] byte offset of the request's code region
  const long long* meta_off;   // [R] byte offset of the request's fp16 metadata
  int num_req;
};

// Per-layer quantizer description.
struct LayerParams {
  int H;          // local KV heads
  int n_groups;   // distinct value level counts
  float key_levels[kMaxHeads];
  float value_levels[kMaxHeads];
  int key_bits[kMaxHeads];    // bits per code in the code region (8 = plain u8)
  int value_bits[kMaxHeads];
  int group_of_head[kMaxHeads];
  // seg_prefix[s] = sum over segments < s of bytes-per-row, segment s = kv*H + h;
  // a request with n rows stores segment s at code_off + n*seg_prefix[s].
  int seg_prefix[2 * kMaxHeads + 1];
  uint32_t sign_bits[kMaxHeads][4];  // bit d set <=> sign of channel d is -1
  int clamp_top;                     // 1: codes <= levels-1 ; 0: codes <= levels
  int transform;                     // 1: randomized Hadamard ; 0: identity
  float out_scale;                   // 1/sqrt(128) with the Hadamard, else 1
};

// One launch of a fused layer stage (producer or consumer side).
struct LayerLaunch {
  PagedKV kv;            // paged source (producer) or destination (consumer)
  ReqTable rt;
  LayerParams lp;
  const uint8_t* bmat;   // [H][32768] swizzled bf16 transform images
  uint8_t* codes;        // code region base (written by producer, read by consumer)
  uint16_t* meta;        // fp16 metadata base
  uint32_t* kstat;       // [R][H][128][2] order-mapped key min/max (producer)
  uint32_t* err;         // device error word
  int total_tiles;
  int engine;            // 0: tcgen05 + TMA ; 1: SIMT (in-register FWHT)
  void* stream;          // cudaStream_t
};

}  // namespace kvs
