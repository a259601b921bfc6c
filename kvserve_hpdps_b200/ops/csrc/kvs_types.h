// Plain-old-data argument blocks shared by the host launchers and the
// kernels.  LayerLaunch is passed by value; the per-slot arrays it points
// to live in device memory.
#pragma once

#include <cstdint>

namespace kvs {

constexpr int kMaxHeads = 16;   // KV heads per rank handled by one launch
constexpr int kHeadDim = 128;   // the fused kernels are specialised for D=128
constexpr int kTileRows = 128;  // tokens per tile

// Paged KV source/destination: element (block, slot, head, d) of plane kv
// lives at base + block*block_stride + kv*kv_stride + slot*slot_stride +
// head*head_stride + d (element units, bf16).  Covers the [2, nb, bs, H, D]
// (FlashAttention) and [nb, 2, bs, H, D] (FlashInfer) block orders, each with
// the (slot, head) plane token-major (NHD: slot_stride = H*D, head_stride = D)
// or head-major (HND: head_stride = bs*D, slot_stride = D, hnd = 1).
struct PagedKV {
  const void* base;
  long long block_stride;
  long long kv_stride;
  long long slot_stride;
  long long head_stride;
  int num_blocks;
  int block_size;
  int hnd;
  int pad_;
};

// Work items of one launch.  An item is one (layer, request) pair: its
// layer slot selects the paged tensor, tensor maps, quantizer parameters and
// transform images; its block table rows select the request's blocks.
struct ReqTable {
  const int32_t* block_table;  // concatenated physical block ids
  const int32_t* bt_off;       // [R] first entry of item r
  const int32_t* n_tokens;     // [R] valid tokens (statistics, written rows)
  const int32_t* n_rows;       // [R] rows = blocks * block_size
  const int32_t* tile_prefix;  // [R+1] cumulative 128-row tiles
  const int32_t* slot;         // [R] layer slot of item r
  const long long* code_off;   // [R] byte offset of the item's code region
  const long long* meta_off;   // [R] byte offset of the item's fp16 metadata
  const long long* row_off;    // [R] prefix of n_rows (value row-stat scratch)
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
  // an item with n rows stores segment s at code_off + n*seg_prefix[s].
  int seg_prefix[2 * kMaxHeads + 1];
  uint32_t sign_bits[kMaxHeads][4];  // bit d set <=> sign of channel d is -1
  int clamp_top;                     // 1: codes <= levels-1 ; 0: codes <= levels
  int transform;                     // 1: randomized Hadamard ; 0: identity
  float out_scale;                   // 1/sqrt(128) with the Hadamard, else 1
};

// One launch of a fused stage over many items.
struct LayerLaunch {
  const PagedKV* kvs;      // [slots] paged source (producer) / destination (consumer)
  const void* maps;        // [slots][2] CUtensorMap (64-B aligned), K and V planes
  const LayerParams* lps;  // [slots]
  ReqTable rt;
  const uint8_t* bmat;     // [slots][H][32768] swizzled bf16 transform images
  long long bmat_stride;   // bytes per slot in bmat
  uint8_t* codes;          // code region base (written by producer, read by consumer)
  uint16_t* meta;          // fp16 metadata base
  uint32_t* kstat;         // [R][H][128][2] order-mapped key min/max (producer)
  float* vstat;            // [sum rows][H][2] per-row value min/max (producer)
  uint32_t* err;           // device error word
  int total_tiles;
  int num_heads;           // H (identical for every slot of a launch)
  int engine;              // 0: warp-specialized tcgen05 + TMA ; 1: SIMT ; 2: tcgen05 per tile ; 3: persistent tcgen05
  void* stream;            // cudaStream_t
  // Optional device trace (nullptr = off): globaltimer stamps
  // trace[(cta * trace_jobs + job) * 8 + event] for CTAs < kTraceCtas.
  unsigned long long* trace;
  int trace_jobs;
  // Per-row value group (min, 1/scale), [sum rows][H][2] indexed by group
  // like vstat by head; written by k_value_params before the
  // warp-specialized quantize kernel, which reads it (engine 0 only).
  float* vparam;
  // Optional message checksum of the code stores (engine 0 quantize only):
  // the quantize kernel adds the checksum of every code byte it writes,
  // weighted by its message offset ck_off + (address - codes), into ck[2]
  // (used when `codes` is a peer GPU's receive ring; common.cuh defines
  // the checksum).  nullptr = off.
  unsigned long long* ck;
  long long ck_off;
};
constexpr int kTraceCtas = 8;

}  // namespace kvs
