// Fused randomized-Hadamard + hybrid min-max quantization (producer side)
// and dequantization + inverse Hadamard + paged scatter (consumer side).
//
// Semantics follow the reference's compress_v3 / decompress_v3
// (kvserve_v1/tilelang_ops/kv_hadamard_quant.py:1307-1486): keys use
// per-(head, channel) min/max over all tokens of the request layer, values
// use per-token min/max over the heads that share a level count.  The CPU
// oracle is kvserve_hpdps_b200/compression/oracle.py.
//
// Two engines with identical inputs/outputs:
//  * engine 0 (default): 128-token tiles are fetched from the paged cache by
//    TMA (one box per 16-row group and 64-channel half, no multicast), the
//    128-point transform is a tcgen05.mma (bf16 x bf16 -> fp32 in TMEM)
//    against a +-1 Hadamard matrix with the Rademacher signs folded in, and
//    the epilogue reads the accumulator back with tcgen05.ld;
//  * engine 1: thread-per-row loads and an in-register fp32 butterfly.
//
// Launch shapes (one launch covers every request of a layer):
//  key stats / key quant : grid (tiles, H), 128 threads
//  value quant           : grid (tiles),    128 threads, loops over heads
//  dequant + inverse     : grid (tiles, H, 2), 128 threads
#include "common.cuh"
#include "kvs_types.h"

#include <cstdio>

namespace kvs {

constexpr float kRangeEps = 1e-5f;

KVS_DEV uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Request owning global tile `tile` (largest r with tile_prefix[r] <= tile).
KVS_DEV int find_request(const int32_t* tile_prefix, int num_req, int tile) {
  int lo = 0, hi = num_req - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (tile_prefix[mid] <= tile) lo = mid; else hi = mid - 1;
  }
  return lo;
}

struct TileCtx {
  int r, row0, rows, ntok;
};

KVS_DEV TileCtx tile_ctx(const ReqTable& rt, int tile) {
  TileCtx c;
  c.r = find_request(rt.tile_prefix, rt.num_req, tile);
  c.row0 = (tile - rt.tile_prefix[c.r]) * kTileRows;
  c.rows = rt.n_rows[c.r];
  c.ntok = rt.n_tokens[c.r];
  return c;
}

KVS_DEV int phys_block(const ReqTable& rt, int r, int row, int bs) {
  return rt.block_table[rt.bt_off[r] + row / bs];
}

KVS_DEV const __nv_bfloat16* src_row(const PagedKV& kv, int plane, int phys, int slot, int H, int h) {
  return reinterpret_cast<const __nv_bfloat16*>(kv.base) + phys * kv.block_stride +
         plane * kv.kv_stride + (static_cast<long long>(slot) * H + h) * kHeadDim;
}

KVS_DEV __nv_bfloat16* dst_row(const PagedKV& kv, int plane, int phys, int slot, int H, int h) {
  return const_cast<__nv_bfloat16*>(reinterpret_cast<const __nv_bfloat16*>(kv.base)) +
         phys * kv.block_stride + plane * kv.kv_stride +
         (static_cast<long long>(slot) * H + h) * kHeadDim;
}

// Byte address of this request's code row for segment (kv, h).
KVS_DEV uint8_t* code_row(const LayerLaunch& L, const TileCtx& c, int kv, int h, int row) {
  const int bits = kv == 0 ? L.lp.key_bits[h] : L.lp.value_bits[h];
  return L.codes + L.rt.code_off[c.r] +
         static_cast<long long>(c.rows) * L.lp.seg_prefix[kv * L.lp.H + h] +
         static_cast<long long>(row) * 16 * bits;
}

// fp16 metadata of a request: [kmin H*128][kscale H*128][vmin G*rows][vscale G*rows]
KVS_DEV __half* meta_base(const LayerLaunch& L, int r) {
  return reinterpret_cast<__half*>(reinterpret_cast<uint8_t*>(L.meta) + L.rt.meta_off[r]);
}

// ------------------------------------------------------- code (un)packing
template <int W>
KVS_DEV void store_chunk_w(uint8_t* row, int c, const uint32_t (&codes)[32]) {
  uint32_t w[8];
  pack32<W>(codes, w);
  uint32_t* d = reinterpret_cast<uint32_t*>(row + c * 4 * W);
#pragma unroll
  for (int i = 0; i < W; ++i) d[i] = w[i];
}
KVS_DEV void store_chunk(uint8_t* row, int c, int bits, const uint32_t (&codes)[32]) {
  switch (bits) {
    case 1: store_chunk_w<1>(row, c, codes); break;
    case 2: store_chunk_w<2>(row, c, codes); break;
    case 3: store_chunk_w<3>(row, c, codes); break;
    case 4: store_chunk_w<4>(row, c, codes); break;
    case 5: store_chunk_w<5>(row, c, codes); break;
    case 6: store_chunk_w<6>(row, c, codes); break;
    case 7: store_chunk_w<7>(row, c, codes); break;
    default: store_chunk_w<8>(row, c, codes); break;
  }
}
template <int W>
KVS_DEV void load_chunk_w(const uint8_t* row, int c, uint32_t (&codes)[32]) {
  uint32_t w[8];
  const uint32_t* s = reinterpret_cast<const uint32_t*>(row + c * 4 * W);
#pragma unroll
  for (int i = 0; i < W; ++i) w[i] = s[i];
  unpack32<W>(w, codes);
}
KVS_DEV void load_chunk(const uint8_t* row, int c, int bits, uint32_t (&codes)[32]) {
  switch (bits) {
    case 1: load_chunk_w<1>(row, c, codes); break;
    case 2: load_chunk_w<2>(row, c, codes); break;
    case 3: load_chunk_w<3>(row, c, codes); break;
    case 4: load_chunk_w<4>(row, c, codes); break;
    case 5: load_chunk_w<5>(row, c, codes); break;
    case 6: load_chunk_w<6>(row, c, codes); break;
    case 7: load_chunk_w<7>(row, c, codes); break;
    default: load_chunk_w<8>(row, c, codes); break;
  }
}

// ------------------------------------------------------------- SIMT engine
KVS_DEV void load_row_f32(const __nv_bfloat16* p, float (&v)[128]) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint4 u = q[i];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[i * 8 + 2 * j] = __uint_as_float(w[j] << 16);
      v[i * 8 + 2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
    }
  }
}

KVS_DEV void apply_signs(float (&v)[128], const uint32_t (&sb)[4]) {
#pragma unroll
  for (int d = 0; d < 128; ++d)
    v[d] = __uint_as_float(__float_as_uint(v[d]) ^ (((sb[d >> 5] >> (d & 31)) & 1u) << 31));
}

KVS_DEV void fwht128(float (&v)[128]) {
#pragma unroll
  for (int s = 1; s < 128; s <<= 1) {
#pragma unroll
    for (int i = 0; i < 128; ++i) {
      if ((i & s) == 0) {
        const float a = v[i], b = v[i + s];
        v[i] = a + b;
        v[i + s] = a - b;
      }
    }
  }
}

// Forward transform of one source row (SIMT engine): signs, butterfly, scale.
KVS_DEV void simt_forward_row(const LayerLaunch& L, int plane, int phys, int slot, int h,
                              float (&v)[128]) {
  load_row_f32(src_row(L.kv, plane, phys, slot, L.lp.H, h), v);
  if (L.lp.transform) {
    const uint32_t sb[4] = {L.lp.sign_bits[h][0], L.lp.sign_bits[h][1], L.lp.sign_bits[h][2],
                            L.lp.sign_bits[h][3]};
    apply_signs(v, sb);
    fwht128(v);
  }
#pragma unroll
  for (int d = 0; d < 128; ++d) v[d] *= L.lp.out_scale;
}

// ================================================================ key stats
__global__ void __launch_bounds__(128) k_key_stats_simt(LayerLaunch L) {
  extern __shared__ float buf[];  // [128][129]
  const int tid = threadIdx.x, h = blockIdx.y;
  const TileCtx c = tile_ctx(L.rt, blockIdx.x);
  const int nvalid = min(kTileRows, c.ntok - c.row0);
  if (nvalid <= 0) return;
  const int row = c.row0 + tid;
  if (tid < nvalid) {
    float v[128];
    const int bs = L.kv.block_size;
    simt_forward_row(L, 0, phys_block(L.rt, c.r, row, bs), row % bs, h, v);
#pragma unroll
    for (int d = 0; d < 128; ++d) buf[tid * 129 + d] = v[d];
  }
  __syncthreads();
  float mn = INFINITY, mx = -INFINITY;
  for (int t = 0; t < nvalid; ++t) {
    const float x = buf[t * 129 + tid];
    mn = fminf(mn, x);
    mx = fmaxf(mx, x);
  }
  uint32_t* ks = L.kstat + (static_cast<size_t>(c.r * L.lp.H + h) * 128 + tid) * 2;
  atomicMin(ks, float_to_ordered(mn));
  atomicMax(ks + 1, float_to_ordered(mx));
}

// Issue the TMA loads of one 128-row tile of head h (plane chosen by the
// map) into a 2 x 16 KB SW128 tile; returns the number of bytes expected.
KVS_DEV uint32_t issue_tile_loads(const CUtensorMap* map, const ReqTable& rt, const TileCtx& c,
                                  int bs, int h, uint8_t* tile, uint64_t* bar, bool arrive,
                                  uint32_t extra_tx) {
  int nload = 0;
#pragma unroll 1
  for (int g = 0; g < 8; ++g)
    if (c.row0 + g * 16 < c.rows) ++nload;
  const uint32_t tx = extra_tx + static_cast<uint32_t>(nload) * 4096u;
  if (arrive) mbar_arrive_expect_tx(bar, tx);
#pragma unroll 1
  for (int g = 0; g < 8; ++g) {
    const int rr = c.row0 + g * 16;
    if (rr >= c.rows) break;
    const int phys = phys_block(rt, c.r, rr, bs);
    const int slot = rr % bs;
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(tile + g * 2048)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(h), "r"(slot), "r"(phys),
        "r"(smem_u32(bar))
        : "memory");
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(tile + 16384 + g * 2048)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(64), "r"(h), "r"(slot), "r"(phys),
        "r"(smem_u32(bar))
        : "memory");
  }
  return tx;
}

constexpr int kSmemPair = 65536 + 1024 + 256;  // B image + tile + barriers + align slack

__global__ void __launch_bounds__(128) k_key_stats_mma(const __grid_constant__ CUtensorMap kmap,
                                                       LayerLaunch L) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sB = smem;          // A operand: signed Hadamard image of head h
  uint8_t* sT = smem + 32768;  // B operand: key tile [token][channel]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 65536);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + 65536 + 32);
  const int tid = threadIdx.x, warp = tid >> 5, h = blockIdx.y;
  const TileCtx c = tile_ctx(L.rt, blockIdx.x);
  const int nvalid = min(kTileRows, c.ntok - c.row0);
  if (nvalid <= 0) return;  // uniform across the CTA, before any barrier
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tslot, 128);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  if (tid == 0) {
    issue_tile_loads(&kmap, L.rt, c, L.kv.block_size, h, sT, &bars[0], true, 32768u);
    bulk_load(sB, L.bmat + static_cast<size_t>(h) * 32768, 32768, &bars[0]);
    if (mbar_wait(&bars[0], 0, L.err, ERR_MBAR_TIMEOUT)) {
      tc_fence_after();
      // D[n][t] = sum_k Bf[n][k] * K[t][k]: lane n = output channel.
      umma_tile_128x128x128(tmem, smem_u32(sB), smem_u32(sT));
    } else {
      mbar_wait(&bars[0], 0, nullptr, 0);  // drain copies still in flight
    }
    umma_commit(&bars[1]);
  }
  mbar_wait(&bars[1], 0, L.err, ERR_MBAR_TIMEOUT);
  tc_fence_after();
  float mn = INFINITY, mx = -INFINITY;
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
    float v[32];
    tmem_ld32(tmem + lane_base + cc * 32, v);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (cc * 32 + j < nvalid) {
        const float x = v[j] * L.lp.out_scale;
        mn = fminf(mn, x);
        mx = fmaxf(mx, x);
      }
    }
  }
  uint32_t* ks = L.kstat + (static_cast<size_t>(c.r * L.lp.H + h) * 128 + tid) * 2;
  atomicMin(ks, float_to_ordered(mn));
  atomicMax(ks + 1, float_to_ordered(mx));
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 128);
}

// Per-channel key min / reciprocal scale of (request r, head h) into smem;
// tile 0 of the request also publishes the fp16 metadata.
KVS_DEV void key_channel_params(const LayerLaunch& L, const TileCtx& c, int h, bool publish,
                                float* s_min, float* s_rcp) {
  const int n = threadIdx.x;
  const uint32_t* ks = L.kstat + (static_cast<size_t>(c.r * L.lp.H + h) * 128 + n) * 2;
  float kmin = 0.f, kmax = 0.f;
  if (c.ntok > 0) {
    kmin = ordered_to_float(ks[0]);
    kmax = ordered_to_float(ks[1]);
  }
  const float lev = L.lp.key_levels[h];
  const float scale = __fdiv_rn(fmaxf(__fsub_rn(kmax, kmin), kRangeEps), lev - 1.0f);
  s_min[n] = kmin;
  s_rcp[n] = __frcp_rn(scale);
  if (publish) {
    __half* m = meta_base(L, c.r);
    m[h * 128 + n] = __float2half_rn(kmin);
    m[L.lp.H * 128 + h * 128 + n] = __float2half_rn(scale);
  }
}

// ================================================================ key quant
__global__ void __launch_bounds__(128) k_quant_k_simt(LayerLaunch L) {
  __shared__ float s_min[128], s_rcp[128];
  const int tid = threadIdx.x, h = blockIdx.y;
  const TileCtx c = tile_ctx(L.rt, blockIdx.x);
  key_channel_params(L, c, h, c.row0 == 0, s_min, s_rcp);
  __syncthreads();
  const int row = c.row0 + tid;
  if (row >= c.rows) return;
  const int bs = L.kv.block_size;
  float v[128];
  simt_forward_row(L, 0, phys_block(L.rt, c.r, row, bs), row % bs, h, v);
  const float lev = L.lp.key_levels[h];
  const float top = L.lp.clamp_top ? lev - 1.0f : lev;
  const bool valid = row < c.ntok;
  uint8_t* out = code_row(L, c, 0, h, row);
  const int bits = L.lp.key_bits[h];
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
    uint32_t q[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int n = cc * 32 + j;
      const float val = valid ? bf16_round(v[n]) : 0.0f;
      q[j] = quantize_one(val, s_min[n], s_rcp[n], top);
    }
    store_chunk(out, cc, bits, q);
  }
}

__global__ void __launch_bounds__(128) k_quant_k_mma(const __grid_constant__ CUtensorMap kmap,
                                                     LayerLaunch L) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sB = smem;
  uint8_t* sT = smem + 32768;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 65536);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + 65536 + 32);
  float* s_min = reinterpret_cast<float*>(smem + 65536 + 64);
  float* s_rcp = s_min + 128;
  const int tid = threadIdx.x, warp = tid >> 5, h = blockIdx.y;
  const TileCtx c = tile_ctx(L.rt, blockIdx.x);
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tslot, 128);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  if (tid == 0) {
    issue_tile_loads(&kmap, L.rt, c, L.kv.block_size, h, sT, &bars[0], true, 32768u);
    bulk_load(sB, L.bmat + static_cast<size_t>(h) * 32768, 32768, &bars[0]);
  }
  key_channel_params(L, c, h, c.row0 == 0, s_min, s_rcp);
  if (tid == 0) {
    if (mbar_wait(&bars[0], 0, L.err, ERR_MBAR_TIMEOUT)) {
      tc_fence_after();
      // D[t][n] = sum_k K[t][k] * Bf[n][k]: lane t = token row.
      umma_tile_128x128x128(tmem, smem_u32(sT), smem_u32(sB));
    } else {
      mbar_wait(&bars[0], 0, nullptr, 0);
    }
    umma_commit(&bars[1]);
  }
  __syncthreads();  // s_min / s_rcp visible
  mbar_wait(&bars[1], 0, L.err, ERR_MBAR_TIMEOUT);
  tc_fence_after();
  const int row = c.row0 + tid;
  const bool exists = row < c.rows, valid = row < c.ntok;
  const float lev = L.lp.key_levels[h];
  const float top = L.lp.clamp_top ? lev - 1.0f : lev;
  uint8_t* out = exists ? code_row(L, c, 0, h, row) : nullptr;
  const int bits = L.lp.key_bits[h];
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
    float v[32];
    tmem_ld32(tmem + lane_base + cc * 32, v);
    uint32_t q[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int n = cc * 32 + j;
      const float val = valid ? bf16_round(v[j] * L.lp.out_scale) : 0.0f;
      q[j] = quantize_one(val, s_min[n], s_rcp[n], top);
    }
    if (exists) store_chunk(out, cc, bits, q);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 128);
}

// ============================================================== value quant
// Per-row group statistics from the per-head row min/max in smem; the
// thread owning row t computes and publishes its own entries.
KVS_DEV void value_group_params(const LayerLaunch& L, const TileCtx& c, const float* rmin,
                                const float* rmax, float* g_min, float* g_rcp) {
  const int t = threadIdx.x, H = L.lp.H, G = L.lp.n_groups;
  const int row = c.row0 + t;
  __half* m = meta_base(L, c.r);
  for (int g = 0; g < G; ++g) {
    float mn = INFINITY, mx = -INFINITY, lev = 2.0f;
    for (int h = 0; h < H; ++h) {
      if (L.lp.group_of_head[h] != g) continue;
      mn = fminf(mn, rmin[h * 128 + t]);
      mx = fmaxf(mx, rmax[h * 128 + t]);
      lev = L.lp.value_levels[h];
    }
    const float scale = __fdiv_rn(fmaxf(__fsub_rn(mx, mn), kRangeEps), lev - 1.0f);
    g_min[g * 128 + t] = mn;
    g_rcp[g * 128 + t] = __frcp_rn(scale);
    if (row < c.rows) {
      m[2 * H * 128 + g * c.rows + row] = __float2half_rn(mn);
      m[2 * H * 128 + G * c.rows + g * c.rows + row] = __float2half_rn(scale);
    }
  }
}

__global__ void __launch_bounds__(128) k_quant_v_simt(LayerLaunch L) {
  extern __shared__ float vsm[];  // rmin[16*128] rmax[16*128] gmin[16*128] grcp[16*128]
  float* rmin = vsm;
  float* rmax = vsm + kMaxHeads * 128;
  float* gmin = vsm + 2 * kMaxHeads * 128;
  float* grcp = vsm + 3 * kMaxHeads * 128;
  const int tid = threadIdx.x, H = L.lp.H;
  const TileCtx c = tile_ctx(L.rt, blockIdx.x);
  const int row = c.row0 + tid;
  const bool exists = row < c.rows, valid = row < c.ntok;
  const int bs = L.kv.block_size;
  const int phys = exists ? phys_block(L.rt, c.r, row, bs) : 0;
  for (int h = 0; h < H; ++h) {
    float mn = 0.f, mx = 0.f;
    if (exists && valid) {
      float v[128];
      simt_forward_row(L, 1, phys, row % bs, h, v);
      mn = INFINITY;
      mx = -INFINITY;
#pragma unroll
      for (int d = 0; d < 128; ++d) {
        mn = fminf(mn, v[d]);
        mx = fmaxf(mx, v[d]);
      }
    }
    rmin[h * 128 + tid] = mn;
    rmax[h * 128 + tid] = mx;
  }
  value_group_params(L, c, rmin, rmax, gmin, grcp);
  if (!exists) return;
  for (int h = 0; h < H; ++h) {
    float v[128];
    if (valid) {
      simt_forward_row(L, 1, phys, row % bs, h, v);
    } else {
#pragma unroll
      for (int d = 0; d < 128; ++d) v[d] = 0.f;
    }
    const int g = L.lp.group_of_head[h];
    const float mn = gmin[g * 128 + tid], rcp = grcp[g * 128 + tid];
    const float lev = L.lp.value_levels[h];
    const float top = L.lp.clamp_top ? lev - 1.0f : lev;
    uint8_t* out = code_row(L, c, 1, h, row);
    const int bits = L.lp.value_bits[h];
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      uint32_t q[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) q[j] = quantize_one(bf16_round(v[cc * 32 + j]), mn, rcp, top);
      store_chunk(out, cc, bits, q);
    }
  }
}

constexpr int kSmemValue = 2 * 65536 + 4 * kMaxHeads * 128 * 4 + 256 + 1024;

__global__ void __launch_bounds__(128, 1) k_quant_v_mma(const __grid_constant__ CUtensorMap vmap,
                                                        LayerLaunch L) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sB[2] = {smem, smem + 65536};
  uint8_t* sA[2] = {smem + 32768, smem + 65536 + 32768};
  float* rmin = reinterpret_cast<float*>(smem + 131072);
  float* rmax = rmin + kMaxHeads * 128;
  float* gmin = rmin + 2 * kMaxHeads * 128;
  float* grcp = rmin + 3 * kMaxHeads * 128;
  uint64_t* lbar = reinterpret_cast<uint64_t*>(smem + 131072 + 4 * kMaxHeads * 128 * 4);
  uint64_t* mbar = lbar + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(lbar + 4);
  const int tid = threadIdx.x, warp = tid >> 5, H = L.lp.H;
  const TileCtx c = tile_ctx(L.rt, blockIdx.x);
  const uint32_t ncols = H <= 1 ? 128u : (H == 2 ? 256u : 512u);
  const bool recompute = H > 4;
  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&lbar[i], 1);
      mbar_init(&mbar[i], 1);
    }
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tslot, ncols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
  const int row = c.row0 + tid;
  const bool exists = row < c.rows, valid = row < c.ntok;
  const int bs = L.kv.block_size;
  uint32_t use[2] = {0u, 0u};

  auto issue = [&](int hh, int st) {
    issue_tile_loads(&vmap, L.rt, c, bs, hh, sA[st], &lbar[st], true, 32768u);
    bulk_load(sB[st], L.bmat + static_cast<size_t>(hh) * 32768, 32768, &lbar[st]);
  };
  auto quant_head = [&](int hh) {
    const int g = L.lp.group_of_head[hh];
    const float mn = gmin[g * 128 + tid], rcp = grcp[g * 128 + tid];
    const float lev = L.lp.value_levels[hh];
    const float top = L.lp.clamp_top ? lev - 1.0f : lev;
    uint8_t* out = exists ? code_row(L, c, 1, hh, row) : nullptr;
    const int bits = L.lp.value_bits[hh];
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      float v[32];
      tmem_ld32(tmem + lane_base + (hh & 3) * 128 + cc * 32, v);
      uint32_t q[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float val = valid ? bf16_round(v[j] * L.lp.out_scale) : 0.0f;
        q[j] = quantize_one(val, mn, rcp, top);
      }
      if (exists) store_chunk(out, cc, bits, q);
    }
  };
  // mode 0: row statistics; mode 1: quantize (used when heads are recomputed)
  auto run_pass = [&](int mode) {
    if (tid == 0) {
      issue(0, 0);
      if (H > 1) issue(1, 1);
    }
    for (int hh = 0; hh < H; ++hh) {
      const int st = hh & 1;
      const uint32_t par = use[st] & 1u;
      if (tid == 0) {
        if (mbar_wait(&lbar[st], par, L.err, ERR_MBAR_TIMEOUT)) {
          tc_fence_after();
          umma_tile_128x128x128(tmem + (hh & 3) * 128, smem_u32(sA[st]), smem_u32(sB[st]));
        } else {
          mbar_wait(&lbar[st], par, nullptr, 0);
        }
        umma_commit(&mbar[st]);
      }
      mbar_wait(&mbar[st], par, L.err, ERR_MBAR_TIMEOUT);
      use[st]++;
      tc_fence_after();
      if (tid == 0 && hh + 2 < H) issue(hh + 2, st);
      if (mode == 0) {
        float mn = INFINITY, mx = -INFINITY;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          float v[32];
          tmem_ld32(tmem + lane_base + (hh & 3) * 128 + cc * 32, v);
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float x = v[j] * L.lp.out_scale;
            mn = fminf(mn, x);
            mx = fmaxf(mx, x);
          }
        }
        if (!valid) mn = mx = 0.f;
        rmin[hh * 128 + tid] = mn;
        rmax[hh * 128 + tid] = mx;
      } else {
        quant_head(hh);
      }
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
    }
  };

  run_pass(0);
  value_group_params(L, c, rmin, rmax, gmin, grcp);
  if (recompute) {
    run_pass(1);
  } else {
    for (int hh = 0; hh < H; ++hh) quant_head(hh);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, ncols);
}

// ========================================================== dequant+inverse
// Dequantize one code row into 128 floats (bf16-valued).
KVS_DEV void dequant_row(const LayerLaunch& L, const TileCtx& c, int kv, int h, int row,
                         const float* kmin_bf, const float* ksc_bf, float (&v)[128]) {
  const uint8_t* src = code_row(L, c, kv, h, row);
  const int bits = kv == 0 ? L.lp.key_bits[h] : L.lp.value_bits[h];
  float vmn = 0.f, vsc = 0.f;
  if (kv == 1) {
    const __half* m = meta_base(L, c.r);
    const int H = L.lp.H, G = L.lp.n_groups, g = L.lp.group_of_head[h];
    vmn = bf16_round(__half2float(m[2 * H * 128 + g * c.rows + row]));
    vsc = bf16_round(__half2float(m[2 * H * 128 + G * c.rows + g * c.rows + row]));
  }
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
    uint32_t q[32];
    load_chunk(src, cc, bits, q);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int n = cc * 32 + j;
      v[n] = kv == 0 ? dequant_bf16(q[j], ksc_bf[n], kmin_bf[n]) : dequant_bf16(q[j], vsc, vmn);
    }
  }
}

KVS_DEV void load_key_meta_bf(const LayerLaunch& L, int r, int h, float* kmin_bf, float* ksc_bf) {
  const int n = threadIdx.x;
  const __half* m = meta_base(L, r);
  kmin_bf[n] = bf16_round(__half2float(m[h * 128 + n]));
  ksc_bf[n] = bf16_round(__half2float(m[L.lp.H * 128 + h * 128 + n]));
}

KVS_DEV void store_row_bf16(__nv_bfloat16* dst, const float (&v)[128]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const __nv_bfloat162 p = __floats2bfloat162_rn(v[i * 8 + 2 * j], v[i * 8 + 2 * j + 1]);
      w[j] = *reinterpret_cast<const uint32_t*>(&p);
    }
    d[i] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

__global__ void __launch_bounds__(128) k_dequant_inverse_simt(LayerLaunch L) {
  __shared__ float kmin_bf[128], ksc_bf[128];
  const int tid = threadIdx.x, h = blockIdx.y, kv = blockIdx.z;
  const TileCtx c = tile_ctx(L.rt, blockIdx.x);
  if (kv == 0) load_key_meta_bf(L, c.r, h, kmin_bf, ksc_bf);
  __syncthreads();
  const int row = c.row0 + tid;
  if (row >= c.ntok || row >= c.rows) return;
  float v[128];
  dequant_row(L, c, kv, h, row, kmin_bf, ksc_bf, v);
  if (L.lp.transform) {
    fwht128(v);
    const uint32_t sb[4] = {L.lp.sign_bits[h][0], L.lp.sign_bits[h][1], L.lp.sign_bits[h][2],
                            L.lp.sign_bits[h][3]};
#pragma unroll
    for (int d = 0; d < 128; ++d) v[d] = bf16_round(v[d] * L.lp.out_scale);
    apply_signs(v, sb);
  }
  const int bs = L.kv.block_size;
  store_row_bf16(dst_row(L.kv, kv, phys_block(L.rt, c.r, row, bs), row % bs, L.lp.H, h), v);
}

// Byte offset of element n of row t in a 2 x 16 KB K-major SW128 tile.
KVS_DEV uint32_t sw128_offset(int t, int n) {
  const int hb = n >> 6;
  const int byte = (n & 63) * 2;
  const int chunk = (byte >> 4) ^ (t & 7);
  return static_cast<uint32_t>(hb * 16384 + (t >> 3) * 1024 + (t & 7) * 128 + chunk * 16 +
                               (byte & 15));
}

__global__ void __launch_bounds__(128) k_dequant_inverse_mma(LayerLaunch L) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sB = smem;          // inverse image of head h
  uint8_t* sA = smem + 32768;  // dequantized tile [token][channel]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 65536);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + 65536 + 32);
  float* kmin_bf = reinterpret_cast<float*>(smem + 65536 + 64);
  float* ksc_bf = kmin_bf + 128;
  const int tid = threadIdx.x, warp = tid >> 5, h = blockIdx.y, kv = blockIdx.z;
  const TileCtx c = tile_ctx(L.rt, blockIdx.x);
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(&bars[0], 32768u);
    bulk_load(sB, L.bmat + static_cast<size_t>(h) * 32768, 32768, &bars[0]);
  }
  if (warp == 0) tmem_alloc(tslot, 128);
  if (kv == 0) load_key_meta_bf(L, c.r, h, kmin_bf, ksc_bf);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const int row = c.row0 + tid;
  const bool valid = row < c.ntok && row < c.rows;
  {
    float v[128];
    if (valid) {
      dequant_row(L, c, kv, h, row, kmin_bf, ksc_bf, v);
    } else {
#pragma unroll
      for (int d = 0; d < 128; ++d) v[d] = 0.f;
    }
    // 16-byte chunks: 8 consecutive channels per chunk.
#pragma unroll
    for (int ch = 0; ch < 16; ++ch) {
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __nv_bfloat162 p = __floats2bfloat162_rn(v[ch * 8 + 2 * j], v[ch * 8 + 2 * j + 1]);
        w[j] = *reinterpret_cast<const uint32_t*>(&p);
      }
      *reinterpret_cast<uint4*>(sA + sw128_offset(tid, ch * 8)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
  fence_proxy_async_smem();
  __syncthreads();
  if (tid == 0) {
    if (mbar_wait(&bars[0], 0, L.err, ERR_MBAR_TIMEOUT)) {
      tc_fence_after();
      // D[t][k] = sum_n Y[t][n] * Bi[k][n], Bi[k][n] = s[k] H[k][n].
      umma_tile_128x128x128(tmem, smem_u32(sA), smem_u32(sB));
    } else {
      mbar_wait(&bars[0], 0, nullptr, 0);
    }
    umma_commit(&bars[1]);
  }
  mbar_wait(&bars[1], 0, L.err, ERR_MBAR_TIMEOUT);
  tc_fence_after();
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
  const int bs = L.kv.block_size;
  __nv_bfloat16* dst =
      valid ? dst_row(L.kv, kv, phys_block(L.rt, c.r, row, bs), row % bs, L.lp.H, h) : nullptr;
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
    float v[32];
    tmem_ld32(tmem + lane_base + cc * 32, v);
    if (valid) {
      uint32_t w[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const __nv_bfloat162 p =
            __floats2bfloat162_rn(v[2 * j] * L.lp.out_scale, v[2 * j + 1] * L.lp.out_scale);
        w[j] = *reinterpret_cast<const uint32_t*>(&p);
      }
      uint4* d = reinterpret_cast<uint4*>(dst + cc * 32);
#pragma unroll
      for (int i = 0; i < 4; ++i) d[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 128);
}

__global__ void k_init_key_stats(uint32_t* kstat, long long n_pairs) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n_pairs;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    kstat[2 * i] = 0xFFFFFFFFu;
    kstat[2 * i + 1] = 0u;
  }
}

// ----------------------------------------------------------------- host
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 4-D map over one KV plane: (d=128, head, slot, block), box (64, 1, 16, 1).
static int make_plane_map(const PagedKV& kv, int plane, int H, CUtensorMap* map) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return -100;
  void* base = const_cast<void*>(reinterpret_cast<const void*>(
      reinterpret_cast<const __nv_bfloat16*>(kv.base) + plane * kv.kv_stride));
  cuuint64_t dims[4] = {128, static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(kv.block_size),
                        static_cast<cuuint64_t>(kv.num_blocks)};
  cuuint64_t strides[3] = {256, static_cast<cuuint64_t>(H) * 256,
                           static_cast<cuuint64_t>(kv.block_stride) * 2};
  cuuint32_t box[4] = {64, 1, 16, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, base, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -101;
}

template <typename K>
static int set_smem(K kernel, int bytes) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) ==
                 cudaSuccess
             ? 0
             : -102;
}

static int mma_supported(const LayerLaunch& L) {
  return L.kv.block_size % 16 == 0 && L.lp.H <= kMaxHeads;
}

}  // namespace kvs

using namespace kvs;

extern "C" {

int kvs_init_key_stats(uint32_t* kstat, long long n_pairs, void* stream) {
  if (n_pairs <= 0) return 0;
  const int blocks = static_cast<int>(min(1024LL, (n_pairs + 255) / 256));
  k_init_key_stats<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(kstat, n_pairs);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int kvs_key_stats(const LayerLaunch* Lp) {
  const LayerLaunch& L = *Lp;
  if (L.total_tiles <= 0) return 0;
  cudaStream_t s = static_cast<cudaStream_t>(L.stream);
  dim3 grid(L.total_tiles, L.lp.H);
  if (L.engine == 0 && mma_supported(L)) {
    CUtensorMap map;
    int rc = make_plane_map(L.kv, 0, L.lp.H, &map);
    if (rc) return rc;
    if (int rc = set_smem(k_key_stats_mma, kSmemPair)) return rc;
    k_key_stats_mma<<<grid, 128, kSmemPair, s>>>(map, L);
  } else {
    if (int rc = set_smem(k_key_stats_simt, 128 * 129 * 4)) return rc;
    k_key_stats_simt<<<grid, 128, 128 * 129 * 4, s>>>(L);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int kvs_quant_k(const LayerLaunch* Lp) {
  const LayerLaunch& L = *Lp;
  if (L.total_tiles <= 0) return 0;
  cudaStream_t s = static_cast<cudaStream_t>(L.stream);
  dim3 grid(L.total_tiles, L.lp.H);
  if (L.engine == 0 && mma_supported(L)) {
    CUtensorMap map;
    int rc = make_plane_map(L.kv, 0, L.lp.H, &map);
    if (rc) return rc;
    if (int rc = set_smem(k_quant_k_mma, kSmemPair + 1024)) return rc;
    k_quant_k_mma<<<grid, 128, kSmemPair + 1024, s>>>(map, L);
  } else {
    k_quant_k_simt<<<grid, 128, 0, s>>>(L);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int kvs_quant_v(const LayerLaunch* Lp) {
  const LayerLaunch& L = *Lp;
  if (L.total_tiles <= 0) return 0;
  cudaStream_t s = static_cast<cudaStream_t>(L.stream);
  if (L.engine == 0 && mma_supported(L)) {
    CUtensorMap map;
    int rc = make_plane_map(L.kv, 1, L.lp.H, &map);
    if (rc) return rc;
    if (int rc = set_smem(k_quant_v_mma, kSmemValue)) return rc;
    k_quant_v_mma<<<L.total_tiles, 128, kSmemValue, s>>>(map, L);
  } else {
    const int bytes = 4 * kMaxHeads * 128 * 4;
    if (int rc = set_smem(k_quant_v_simt, bytes)) return rc;
    k_quant_v_simt<<<L.total_tiles, 128, bytes, s>>>(L);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int kvs_dequant_inverse(const LayerLaunch* Lp) {
  const LayerLaunch& L = *Lp;
  if (L.total_tiles <= 0) return 0;
  cudaStream_t s = static_cast<cudaStream_t>(L.stream);
  dim3 grid(L.total_tiles, L.lp.H, 2);
  if (L.engine == 0 && mma_supported(L)) {
    if (int rc = set_smem(k_dequant_inverse_mma, kSmemPair + 1024)) return rc;
    k_dequant_inverse_mma<<<grid, 128, kSmemPair + 1024, s>>>(L);
  } else {
    k_dequant_inverse_simt<<<grid, 128, 0, s>>>(L);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int kvs_layer_launch_size(void) { return static_cast<int>(sizeof(LayerLaunch)); }

}  // extern "C"
