// Fused randomized-Hadamard + hybrid min-max quantization (producer side)
// and dequantization + inverse Hadamard + paged scatter (consumer side).
//
// Semantics follow the reference's compress_v3 / decompress_v3
// (kvserve_v1/tilelang_ops/kv_hadamard_quant.py:1307-1486): keys use
// per-(head, channel) min/max over all tokens of the request layer, values
// use per-token min/max over the heads that share a level count.  The CPU
// oracle is kvserve_hpdps_b200/compression/oracle.py.
//
// One launch covers many work items, an item being a (layer, request) pair
// (kvs_types.h).  The producer is three launches:
//   k_init_key_stats                      reset the key min/max accumulators;
//   k_stats_*   grid (tiles, H, 2)        plane 0: per-channel key min/max
//                                         (atomics); plane 1: per-row value
//                                         min/max (stores);
//   k_quant_*   grid (tiles, H, 2)        codes + fp16 metadata of K and V.
// The consumer is one launch: k_dequant_inverse_* grid (tiles, H, 2).
//
// Two engines with identical inputs/outputs:
//  * engine 0 (default): 128-token tiles are fetched from the paged cache by
//    TMA (one box per 16-row group and 64-channel half, no multicast), the
//    128-point transform is a tcgen05.mma (bf16 x bf16 -> fp32 in TMEM)
//    against a +-1 Hadamard matrix with the Rademacher signs folded in, and
//    the epilogue reads the accumulator back with tcgen05.ld;
//  * engine 1: thread-per-row loads and an in-register fp32 butterfly.
#include "common.cuh"
#include "kvs_types.h"

namespace kvs {

constexpr float kRangeEps = 1e-5f;

KVS_DEV uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Item owning global tile `tile` (largest r with tile_prefix[r] <= tile).
KVS_DEV int find_item(const int32_t* tile_prefix, int num_req, int tile) {
  int lo = 0, hi = num_req - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (tile_prefix[mid] <= tile) lo = mid; else hi = mid - 1;
  }
  return lo;
}

struct ItemCtx {
  int r, slot, row0, rows, ntok;
  const LayerParams* lp;
  PagedKV kv;
};

KVS_DEV ItemCtx item_ctx(const LayerLaunch& L, int tile) {
  ItemCtx c;
  c.r = find_item(L.rt.tile_prefix, L.rt.num_req, tile);
  c.slot = L.rt.slot[c.r];
  c.row0 = (tile - L.rt.tile_prefix[c.r]) * kTileRows;
  c.rows = L.rt.n_rows[c.r];
  c.ntok = L.rt.n_tokens[c.r];
  c.lp = L.lps + c.slot;
  c.kv = L.kvs[c.slot];
  return c;
}

KVS_DEV int phys_block(const LayerLaunch& L, const ItemCtx& c, int row) {
  return L.rt.block_table[L.rt.bt_off[c.r] + row / c.kv.block_size];
}

KVS_DEV __nv_bfloat16* kv_row(const ItemCtx& c, int plane, int phys, int slot, int h) {
  return const_cast<__nv_bfloat16*>(reinterpret_cast<const __nv_bfloat16*>(c.kv.base)) +
         phys * c.kv.block_stride + plane * c.kv.kv_stride +
         (static_cast<long long>(slot) * c.lp->H + h) * kHeadDim;
}

KVS_DEV int seg_bits(const ItemCtx& c, int kv, int h) {
  return kv == 0 ? c.lp->key_bits[h] : c.lp->value_bits[h];
}

// Byte address of an item's code row for segment (kv, h).
KVS_DEV uint8_t* code_row(const LayerLaunch& L, const ItemCtx& c, int kv, int h, int row) {
  return L.codes + L.rt.code_off[c.r] +
         static_cast<long long>(c.rows) * c.lp->seg_prefix[kv * c.lp->H + h] +
         static_cast<long long>(row) * 16 * seg_bits(c, kv, h);
}

// fp16 metadata of an item: [kmin H*128][kscale H*128][vmin G*rows][vscale G*rows]
KVS_DEV __half* meta_base(const LayerLaunch& L, int r) {
  return reinterpret_cast<__half*>(reinterpret_cast<uint8_t*>(L.meta) + L.rt.meta_off[r]);
}

KVS_DEV float* vstat_entry(const LayerLaunch& L, const ItemCtx& c, int h, int row) {
  return L.vstat + (L.rt.row_off[c.r] * c.lp->H + static_cast<long long>(h) * c.rows + row) * 2;
}

KVS_DEV const uint8_t* bmat_of(const LayerLaunch& L, int slot, int h) {
  return L.bmat + slot * L.bmat_stride + static_cast<long long>(h) * 32768;
}

KVS_DEV const CUtensorMap* map_of(const LayerLaunch& L, int slot, int plane) {
  return reinterpret_cast<const CUtensorMap*>(L.maps) + slot * 2 + plane;
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

KVS_DEV void apply_signs(float (&v)[128], const uint32_t* sb) {
  uint32_t s[4] = {sb[0], sb[1], sb[2], sb[3]};
#pragma unroll
  for (int d = 0; d < 128; ++d)
    v[d] = __uint_as_float(__float_as_uint(v[d]) ^ (((s[d >> 5] >> (d & 31)) & 1u) << 31));
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
KVS_DEV void simt_forward_row(const ItemCtx& c, int plane, int phys, int slot, int h,
                              float (&v)[128]) {
  load_row_f32(kv_row(c, plane, phys, slot, h), v);
  if (c.lp->transform) {
    apply_signs(v, c.lp->sign_bits[h]);
    fwht128(v);
  }
  const float sc = c.lp->out_scale;
#pragma unroll
  for (int d = 0; d < 128; ++d) v[d] *= sc;
}

// ------------------------------------------------------- shared prologues
// Issue the TMA loads of one 128-row tile of head h (plane chosen by the
// map) into a 2 x 16 KB SW128 tile, arriving on `bar` with the expected
// byte count (plus `extra_tx` for other copies on the same barrier).
KVS_DEV void issue_tile_loads(const LayerLaunch& L, const ItemCtx& c, const CUtensorMap* map,
                              int h, uint8_t* tile, uint64_t* bar, uint32_t extra_tx) {
  int nload = 0;
  for (int g = 0; g < 8; ++g)
    if (c.row0 + g * 16 < c.rows) ++nload;
  mbar_arrive_expect_tx(bar, extra_tx + static_cast<uint32_t>(nload) * 4096u);
  for (int g = 0; g < 8; ++g) {
    const int rr = c.row0 + g * 16;
    if (rr >= c.rows) break;
    const int phys = phys_block(L, c, rr);
    const int slot = rr % c.kv.block_size;
#pragma unroll
    for (int hb = 0; hb < 2; ++hb) {
      asm volatile(
          "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
          " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(tile + hb * 16384 + g * 2048)),
          "l"(reinterpret_cast<uint64_t>(map)), "r"(hb * 64), "r"(h), "r"(slot), "r"(phys),
          "r"(smem_u32(bar))
          : "memory");
    }
  }
}

// Key channel min / reciprocal scale of (item, head h) into smem; tile 0 of
// the item publishes the fp16 metadata.
KVS_DEV void key_channel_params(const LayerLaunch& L, const ItemCtx& c, int h, float* s_min,
                                float* s_rcp) {
  const int n = threadIdx.x;
  const uint32_t* ks = L.kstat + (static_cast<size_t>(c.r * c.lp->H + h) * 128 + n) * 2;
  float kmin = 0.f, kmax = 0.f;
  if (c.ntok > 0) {
    kmin = ordered_to_float(ks[0]);
    kmax = ordered_to_float(ks[1]);
  }
  const float lev = c.lp->key_levels[h];
  const float scale = __fdiv_rn(fmaxf(__fsub_rn(kmax, kmin), kRangeEps), lev - 1.0f);
  s_min[n] = kmin;
  s_rcp[n] = __frcp_rn(scale);
  if (c.row0 == 0) {
    __half* m = meta_base(L, c.r);
    m[h * 128 + n] = __float2half_rn(kmin);
    m[c.lp->H * 128 + h * 128 + n] = __float2half_rn(scale);
  }
}

// Value group min / reciprocal scale of row `row` for head h; the first
// head of the group publishes the fp16 metadata.
KVS_DEV void value_row_params(const LayerLaunch& L, const ItemCtx& c, int h, int row,
                              float* out_min, float* out_rcp) {
  const LayerParams* lp = c.lp;
  const int g = lp->group_of_head[h];
  float mn = INFINITY, mx = -INFINITY;
  int first = -1;
  for (int hh = 0; hh < lp->H; ++hh) {
    if (lp->group_of_head[hh] != g) continue;
    if (first < 0) first = hh;
    const float* e = vstat_entry(L, c, hh, row);
    mn = fminf(mn, e[0]);
    mx = fmaxf(mx, e[1]);
  }
  const float scale = __fdiv_rn(fmaxf(__fsub_rn(mx, mn), kRangeEps), lp->value_levels[h] - 1.0f);
  *out_min = mn;
  *out_rcp = __frcp_rn(scale);
  if (h == first) {
    __half* m = meta_base(L, c.r);
    const int H = lp->H, G = lp->n_groups;
    m[2 * H * 128 + g * c.rows + row] = __float2half_rn(mn);
    m[2 * H * 128 + G * c.rows + g * c.rows + row] = __float2half_rn(scale);
  }
}

// Epilogue of the MMA quant kernel: read this thread's row (its TMEM lane),
// quantize, pack to W bits and stage the 16*W-byte row in shared memory with
// an odd pitch of (W|1) 16-byte chunks, so the 8 threads sharing a bank
// group write different groups.
struct QuantArgs {
  uint32_t taddr;  // TMEM address of this warp's lanes
  float out_scale, top;
  bool valid;
  int plane;
  float vmin, vrcp;
  const float* s_min;
  const float* s_rcp;
  uint8_t* stage;
};

template <int W>
KVS_DEV void quant_epilogue(const QuantArgs& a) {
  uint32_t words[4 * W];
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
    float v[32];
    tmem_ld32(a.taddr + cc * 32, v);
    uint32_t q[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int n = cc * 32 + j;
      const float val = a.valid ? bf16_round(v[j] * a.out_scale) : 0.0f;
      q[j] = a.plane == 0 ? quantize_one(val, a.s_min[n], a.s_rcp[n], a.top)
                          : quantize_one(val, a.vmin, a.vrcp, a.top);
    }
    uint32_t w[8];
    pack32<W>(q, w);
#pragma unroll
    for (int i = 0; i < W; ++i) words[cc * W + i] = w[i];
  }
  constexpr int P = W | 1;
  uint8_t* dst = a.stage + threadIdx.x * P * 16;
#pragma unroll
  for (int k = 0; k < W; ++k)
    *reinterpret_cast<uint4*>(dst + k * 16) =
        make_uint4(words[4 * k], words[4 * k + 1], words[4 * k + 2], words[4 * k + 3]);
}

// ================================================================== stats
__global__ void __launch_bounds__(128) k_stats_simt(LayerLaunch L) {
  extern __shared__ float buf[];  // [128][129] (keys only)
  const int tid = threadIdx.x, h = blockIdx.y, plane = blockIdx.z;
  const ItemCtx c = item_ctx(L, blockIdx.x);
  const int row = c.row0 + tid;
  if (plane == 1) {
    if (row >= c.rows) return;
    float mn = 0.f, mx = 0.f;
    if (row < c.ntok) {
      float v[128];
      simt_forward_row(c, 1, phys_block(L, c, row), row % c.kv.block_size, h, v);
      mn = INFINITY;
      mx = -INFINITY;
#pragma unroll
      for (int d = 0; d < 128; ++d) {
        mn = fminf(mn, v[d]);
        mx = fmaxf(mx, v[d]);
      }
    }
    float* e = vstat_entry(L, c, h, row);
    e[0] = mn;
    e[1] = mx;
    return;
  }
  const int nvalid = min(kTileRows, c.ntok - c.row0);
  if (nvalid <= 0) return;
  if (tid < nvalid) {
    float v[128];
    simt_forward_row(c, 0, phys_block(L, c, row), row % c.kv.block_size, h, v);
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
  uint32_t* ks = L.kstat + (static_cast<size_t>(c.r * c.lp->H + h) * 128 + tid) * 2;
  atomicMin(ks, float_to_ordered(mn));
  atomicMax(ks + 1, float_to_ordered(mx));
}

constexpr int kSmemTile = 65536 + 2048 + 1024;  // B image + tile + scratch + align slack

__global__ void __launch_bounds__(128) k_stats_mma(LayerLaunch L) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sB = smem;          // transform image of head h
  uint8_t* sT = smem + 32768;  // data tile [token][channel]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 65536);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + 65536 + 32);
  const int tid = threadIdx.x, warp = tid >> 5, h = blockIdx.y, plane = blockIdx.z;
  const ItemCtx c = item_ctx(L, blockIdx.x);
  const int nvalid = min(kTileRows, c.ntok - c.row0);
  if (plane == 0 && nvalid <= 0) return;  // uniform across the CTA, before any barrier
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
    issue_tile_loads(L, c, map_of(L, c.slot, plane), h, sT, &bars[0], 32768u);
    bulk_load(sB, bmat_of(L, c.slot, h), 32768, &bars[0]);
    if (mbar_wait(&bars[0], 0, L.err, ERR_MBAR_TIMEOUT)) {
      tc_fence_after();
      if (plane == 0) {
        // D[n][t] = sum_k Bf[n][k] K[t][k]: lane = output channel n.
        umma_tile_128x128x128(tmem, smem_u32(sB), smem_u32(sT));
      } else {
        // D[t][n] = sum_k V[t][k] Bf[n][k]: lane = token row t.
        umma_tile_128x128x128(tmem, smem_u32(sT), smem_u32(sB));
      }
    } else {
      mbar_wait(&bars[0], 0, nullptr, 0);  // drain copies still in flight
    }
    umma_commit(&bars[1]);
  }
  mbar_wait(&bars[1], 0, L.err, ERR_MBAR_TIMEOUT);
  tc_fence_after();
  const float sc = c.lp->out_scale;
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
  float mn = INFINITY, mx = -INFINITY;
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
    float v[32];
    tmem_ld32(tmem + lane_base + cc * 32, v);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (plane == 1 || cc * 32 + j < nvalid) {
        const float x = v[j] * sc;
        mn = fminf(mn, x);
        mx = fmaxf(mx, x);
      }
    }
  }
  if (plane == 0) {
    uint32_t* ks = L.kstat + (static_cast<size_t>(c.r * c.lp->H + h) * 128 + tid) * 2;
    atomicMin(ks, float_to_ordered(mn));
    atomicMax(ks + 1, float_to_ordered(mx));
  } else {
    const int row = c.row0 + tid;
    if (row < c.rows) {
      if (row >= c.ntok) mn = mx = 0.f;
      float* e = vstat_entry(L, c, h, row);
      e[0] = mn;
      e[1] = mx;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 128);
}

// ================================================================== quant
__global__ void __launch_bounds__(128) k_quant_simt(LayerLaunch L) {
  __shared__ float s_min[128], s_rcp[128];
  const int tid = threadIdx.x, h = blockIdx.y, plane = blockIdx.z;
  const ItemCtx c = item_ctx(L, blockIdx.x);
  if (plane == 0) key_channel_params(L, c, h, s_min, s_rcp);
  __syncthreads();
  const int row = c.row0 + tid;
  if (row >= c.rows) return;
  float vmin = 0.f, vrcp = 0.f;
  if (plane == 1) value_row_params(L, c, h, row, &vmin, &vrcp);
  float v[128];
  const bool valid = row < c.ntok;
  if (valid) {
    simt_forward_row(c, plane, phys_block(L, c, row), row % c.kv.block_size, h, v);
  } else {
#pragma unroll
    for (int d = 0; d < 128; ++d) v[d] = 0.f;
  }
  const float lev = plane == 0 ? c.lp->key_levels[h] : c.lp->value_levels[h];
  const float top = c.lp->clamp_top ? lev - 1.0f : lev;
  uint8_t* out = code_row(L, c, plane, h, row);
  const int bits = seg_bits(c, plane, h);
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
    uint32_t q[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int n = cc * 32 + j;
      const float val = bf16_round(v[n]);
      q[j] = plane == 0 ? quantize_one(val, s_min[n], s_rcp[n], top)
                        : quantize_one(val, vmin, vrcp, top);
    }
    store_chunk(out, cc, bits, q);
  }
}

__global__ void __launch_bounds__(128) k_quant_mma(LayerLaunch L) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sB = smem;
  uint8_t* sT = smem + 32768;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 65536);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + 65536 + 32);
  float* s_min = reinterpret_cast<float*>(smem + 65536 + 64);
  float* s_rcp = s_min + 128;
  const int tid = threadIdx.x, warp = tid >> 5, h = blockIdx.y, plane = blockIdx.z;
  const ItemCtx c = item_ctx(L, blockIdx.x);
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
    issue_tile_loads(L, c, map_of(L, c.slot, plane), h, sT, &bars[0], 32768u);
    bulk_load(sB, bmat_of(L, c.slot, h), 32768, &bars[0]);
  }
  const int row = c.row0 + tid;
  const bool exists = row < c.rows, valid = row < c.ntok;
  float vmin = 0.f, vrcp = 0.f;
  if (plane == 0) {
    key_channel_params(L, c, h, s_min, s_rcp);
  } else if (exists) {
    value_row_params(L, c, h, row, &vmin, &vrcp);
  }
  if (tid == 0) {
    if (mbar_wait(&bars[0], 0, L.err, ERR_MBAR_TIMEOUT)) {
      tc_fence_after();
      // D[t][n] = sum_k X[t][k] Bf[n][k]: lane = token row t.
      umma_tile_128x128x128(tmem, smem_u32(sT), smem_u32(sB));
    } else {
      mbar_wait(&bars[0], 0, nullptr, 0);
    }
    umma_commit(&bars[1]);
  }
  __syncthreads();  // s_min / s_rcp visible
  mbar_wait(&bars[1], 0, L.err, ERR_MBAR_TIMEOUT);
  tc_fence_after();
  const float lev = plane == 0 ? c.lp->key_levels[h] : c.lp->value_levels[h];
  const float top = c.lp->clamp_top ? lev - 1.0f : lev;
  const QuantArgs qa{tmem + (static_cast<uint32_t>(warp * 32) << 16), c.lp->out_scale, top, valid,
                     plane, vmin, vrcp, s_min, s_rcp, sT};
  // sT (the data tile) is free: the MMA that read it has completed.
  switch (seg_bits(c, plane, h)) {
    case 1: quant_epilogue<1>(qa); break;
    case 2: quant_epilogue<2>(qa); break;
    case 3: quant_epilogue<3>(qa); break;
    case 4: quant_epilogue<4>(qa); break;
    case 5: quant_epilogue<5>(qa); break;
    case 6: quant_epilogue<6>(qa); break;
    case 7: quant_epilogue<7>(qa); break;
    default: quant_epilogue<8>(qa); break;
  }
  tc_fence_before();
  __syncthreads();
  // Coalesced copy of the tile's contiguous code region.
  const int bits = seg_bits(c, plane, h);
  const int nrows = min(kTileRows, c.rows - c.row0);
  uint8_t* dst0 = code_row(L, c, plane, h, c.row0);
  const int P = bits | 1;  // staging pitch in 16-byte chunks (odd: bank-conflict free)
  for (int k = tid; k < nrows * bits; k += 128) {
    const int r = k / bits, col = k - r * bits;
    *reinterpret_cast<uint4*>(dst0 + static_cast<long long>(k) * 16) =
        *reinterpret_cast<const uint4*>(sT + (r * P + col) * 16);
  }
  if (warp == 0) tmem_dealloc(tmem, 128);
}

// ========================================================== dequant+inverse
// Dequantize one code row into 128 floats (bf16-valued).
KVS_DEV void dequant_row(const LayerLaunch& L, const ItemCtx& c, int kv, int h, int row,
                         const float* kmin_bf, const float* ksc_bf, float (&v)[128]) {
  const uint8_t* src = code_row(L, c, kv, h, row);
  const int bits = seg_bits(c, kv, h);
  float vmn = 0.f, vsc = 0.f;
  if (kv == 1) {
    const __half* m = meta_base(L, c.r);
    const int H = c.lp->H, G = c.lp->n_groups, g = c.lp->group_of_head[h];
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

KVS_DEV void load_key_meta_bf(const LayerLaunch& L, const ItemCtx& c, int h, float* kmin_bf,
                              float* ksc_bf) {
  const int n = threadIdx.x;
  const __half* m = meta_base(L, c.r);
  kmin_bf[n] = bf16_round(__half2float(m[h * 128 + n]));
  ksc_bf[n] = bf16_round(__half2float(m[c.lp->H * 128 + h * 128 + n]));
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
  const ItemCtx c = item_ctx(L, blockIdx.x);
  if (kv == 0) load_key_meta_bf(L, c, h, kmin_bf, ksc_bf);
  __syncthreads();
  const int row = c.row0 + tid;
  if (row >= c.ntok || row >= c.rows) return;
  float v[128];
  dequant_row(L, c, kv, h, row, kmin_bf, ksc_bf, v);
  if (c.lp->transform) {
    fwht128(v);
    const float sc = c.lp->out_scale;
#pragma unroll
    for (int d = 0; d < 128; ++d) v[d] = bf16_round(v[d] * sc);
    apply_signs(v, c.lp->sign_bits[h]);
  }
  store_row_bf16(kv_row(c, kv, phys_block(L, c, row), row % c.kv.block_size, h), v);
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
  const ItemCtx c = item_ctx(L, blockIdx.x);
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(&bars[0], 32768u);
    bulk_load(sB, bmat_of(L, c.slot, h), 32768, &bars[0]);
  }
  if (warp == 0) tmem_alloc(tslot, 128);
  if (kv == 0) load_key_meta_bf(L, c, h, kmin_bf, ksc_bf);
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
#pragma unroll
    for (int ch = 0; ch < 16; ++ch) {
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __nv_bfloat162 p = __floats2bfloat162_rn(v[ch * 8 + 2 * j], v[ch * 8 + 2 * j + 1]);
        w[j] = *reinterpret_cast<const uint32_t*>(&p);
      }
      *reinterpret_cast<uint4*>(sA + sw128_offset(tid, ch * 8)) =
          make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
  fence_proxy_async_smem();
  __syncthreads();
  if (tid == 0) {
    if (mbar_wait(&bars[0], 0, L.err, ERR_MBAR_TIMEOUT)) {
      tc_fence_after();
      // D[t][k] = sum_n Y[t][n] Bi[k][n], Bi[k][n] = s[k] H[k][n].
      umma_tile_128x128x128(tmem, smem_u32(sA), smem_u32(sB));
    } else {
      mbar_wait(&bars[0], 0, nullptr, 0);
    }
    umma_commit(&bars[1]);
  }
  mbar_wait(&bars[1], 0, L.err, ERR_MBAR_TIMEOUT);
  tc_fence_after();
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
  const float sc = c.lp->out_scale;
  // The dequantized tile sA was consumed by the MMA: reuse it to stage the
  // bf16 output in the 128-byte swizzled layout of the destination map.
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
    float v[32];
    tmem_ld32(tmem + lane_base + cc * 32, v);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __nv_bfloat162 p =
            __floats2bfloat162_rn(v[8 * q + 2 * j] * sc, v[8 * q + 2 * j + 1] * sc);
        w[j] = *reinterpret_cast<const uint32_t*>(&p);
      }
      *reinterpret_cast<uint4*>(sA + sw128_offset(tid, cc * 32 + q * 8)) =
          make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  if (tid == 0) {
    // One TMA tensor store per 16-row group and 64-channel half (full
    // 128-byte lines into the paged cache; the groups never straddle blocks).
    const CUtensorMap* map = map_of(L, c.slot, kv);
    for (int g = 0; g < 8; ++g) {
      const int rr = c.row0 + g * 16;
      if (rr >= c.rows) break;
      const int phys = phys_block(L, c, rr);
      const int slot = rr % c.kv.block_size;
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {
        asm volatile(
            "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%1, %2, %3, %4}], [%5];" ::
                "l"(reinterpret_cast<uint64_t>(map)),
            "r"(hb * 64), "r"(h), "r"(slot), "r"(phys), "r"(smem_u32(sA + hb * 16384 + g * 2048))
            : "memory");
      }
    }
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
  }
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

template <typename K>
static int set_smem(K kernel, int bytes) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) ==
                 cudaSuccess
             ? 0
             : -102;
}

}  // namespace kvs

using namespace kvs;

extern "C" {

int kvs_layer_launch_size(void) { return static_cast<int>(sizeof(LayerLaunch)); }
int kvs_layer_params_size(void) { return static_cast<int>(sizeof(LayerParams)); }
int kvs_paged_kv_size(void) { return static_cast<int>(sizeof(PagedKV)); }

// Encode the K and V plane maps of one paged layer into out[0..1] (host
// memory, 128 bytes each): 4-D (d=128, head, slot, block), box (64,1,16,1),
// 128-byte swizzle, no OOB fill.
int kvs_make_plane_maps(const PagedKV* kv, int H, void* out) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return -100;
  CUtensorMap* maps = static_cast<CUtensorMap*>(out);
  for (int plane = 0; plane < 2; ++plane) {
    void* base = const_cast<void*>(reinterpret_cast<const void*>(
        reinterpret_cast<const __nv_bfloat16*>(kv->base) + plane * kv->kv_stride));
    cuuint64_t dims[4] = {128, static_cast<cuuint64_t>(H),
                          static_cast<cuuint64_t>(kv->block_size),
                          static_cast<cuuint64_t>(kv->num_blocks)};
    cuuint64_t strides[3] = {256, static_cast<cuuint64_t>(H) * 256,
                             static_cast<cuuint64_t>(kv->block_stride) * 2};
    cuuint32_t box[4] = {64, 1, 16, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = fn(&maps[plane], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, base, dims, strides, box,
                    estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return -101;
  }
  return 0;
}

int kvs_init_key_stats(uint32_t* kstat, long long n_pairs, void* stream) {
  if (n_pairs <= 0) return 0;
  const int blocks = static_cast<int>(min(1024LL, (n_pairs + 255) / 256));
  k_init_key_stats<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(kstat, n_pairs);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int kvs_stats(const LayerLaunch* Lp) {
  const LayerLaunch& L = *Lp;
  if (L.total_tiles <= 0) return 0;
  cudaStream_t s = static_cast<cudaStream_t>(L.stream);
  dim3 grid(L.total_tiles, L.num_heads, 2);
  if (L.engine == 0) {
    if (int rc = set_smem(k_stats_mma, kSmemTile)) return rc;
    k_stats_mma<<<grid, 128, kSmemTile, s>>>(L);
  } else {
    if (int rc = set_smem(k_stats_simt, 128 * 129 * 4)) return rc;
    k_stats_simt<<<grid, 128, 128 * 129 * 4, s>>>(L);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int kvs_quant(const LayerLaunch* Lp) {
  const LayerLaunch& L = *Lp;
  if (L.total_tiles <= 0) return 0;
  cudaStream_t s = static_cast<cudaStream_t>(L.stream);
  dim3 grid(L.total_tiles, L.num_heads, 2);
  if (L.engine == 0) {
    if (int rc = set_smem(k_quant_mma, kSmemTile)) return rc;
    k_quant_mma<<<grid, 128, kSmemTile, s>>>(L);
  } else {
    k_quant_simt<<<grid, 128, 0, s>>>(L);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int kvs_dequant_inverse(const LayerLaunch* Lp) {
  const LayerLaunch& L = *Lp;
  if (L.total_tiles <= 0) return 0;
  cudaStream_t s = static_cast<cudaStream_t>(L.stream);
  dim3 grid(L.total_tiles, L.num_heads, 2);
  if (L.engine == 0) {
    if (int rc = set_smem(k_dequant_inverse_mma, kSmemTile)) return rc;
    k_dequant_inverse_mma<<<grid, 128, kSmemTile, s>>>(L);
  } else {
    k_dequant_inverse_simt<<<grid, 128, 0, s>>>(L);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // extern "C"
