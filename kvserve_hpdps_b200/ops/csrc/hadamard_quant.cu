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
// Three engines with identical inputs/outputs:
//  * engine 0 (default): persistent tcgen05 kernels (k_*_tc): 128-token
//    tiles are fetched from the paged cache by TMA (one box per 16-row group
//    and 64-channel half, no multicast), the 128-point transform is a
//    tcgen05.mma (bf16 x bf16 -> fp32 in TMEM) against a +-1 Hadamard matrix
//    with the Rademacher signs folded in, the epilogue reads the accumulator
//    back with tcgen05.ld; each CTA pipelines a contiguous range of tiles;
//    (k_stats_ws / k_quant_ws are warp-specialized: a load warp issues the
//    TMA boxes, an MMA warp issues the MMAs, two epilogue groups of 8 warps
//    alternate jobs;
//    k_dequant_ws: unpack warps, a control warp and epilogue warps);
//  * engine 3: the persistent kernels without warp specialization (k_*_tc);
//  * engine 2: the same math with one CTA per tile (k_*_mma);
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

// Physical block holding an item row.  A block id outside the paged cache
// (a corrupt or mismatched block table) records ERR_BOUNDS and returns -1:
// loads then read block 0 (`load_block`) and stores skip the access, so a
// bad table never makes a kernel touch memory outside the cache.
KVS_DEV int phys_block(const LayerLaunch& L, const ItemCtx& c, int row) {
  const int p = L.rt.block_table[L.rt.bt_off[c.r] + row / c.kv.block_size];
  if (static_cast<unsigned>(p) >= static_cast<unsigned>(c.kv.num_blocks)) {
    record_error(L.err, ERR_BOUNDS);
    return -1;
  }
  return p;
}
KVS_DEV int load_block(const LayerLaunch& L, const ItemCtx& c, int row) {
  return max(0, phys_block(L, c, row));
}
// Block-table entry without the check, for callers that validate it later
// (when the value is used) so that the read's latency is not waited on now.
KVS_DEV int raw_block(const LayerLaunch& L, const ItemCtx& c, int row) {
  return L.rt.block_table[L.rt.bt_off[c.r] + row / c.kv.block_size];
}

KVS_DEV __nv_bfloat16* kv_row(const ItemCtx& c, int plane, int phys, int slot, int h) {
  return const_cast<__nv_bfloat16*>(reinterpret_cast<const __nv_bfloat16*>(c.kv.base)) +
         phys * c.kv.block_stride + plane * c.kv.kv_stride +
         static_cast<long long>(slot) * c.kv.slot_stride +
         static_cast<long long>(h) * c.kv.head_stride;
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

// TMA coordinates (y, z) of (head, slot) in a plane map: the maps order
// their middle dimensions by stride (head then slot for NHD, slot then head
// for HND), so a 16-slot box is 16 rows of 128 bytes either way.
KVS_DEV int tma_y(const PagedKV& kv, int h, int slot) { return kv.hnd ? slot : h; }
KVS_DEV int tma_z(const PagedKV& kv, int h, int slot) { return kv.hnd ? h : slot; }

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
    const int phys = load_block(L, c, rr);
    const int slot = rr % c.kv.block_size;
#pragma unroll
    for (int hb = 0; hb < 2; ++hb) {
      asm volatile(
          "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
          " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(tile + hb * 16384 + g * 2048)),
          "l"(reinterpret_cast<uint64_t>(map)), "r"(hb * 64), "r"(tma_y(c.kv, h, slot)),
          "r"(tma_z(c.kv, h, slot)), "r"(phys), "r"(smem_u32(bar))
          : "memory");
    }
  }
}

// Key channel min / reciprocal scale of (item, head h) into smem; tile 0 of
// the item publishes the fp16 metadata.
KVS_DEV void key_channel_params(const LayerLaunch& L, const ItemCtx& c, int h, float* s_min,
                                float* s_rcp, int stride = 1, int n = -1, bool pairs = false) {
  if (n < 0) n = threadIdx.x;
  const uint32_t* ks = L.kstat + (static_cast<size_t>(c.r * c.lp->H + h) * 128 + n) * 2;
  float kmin = 0.f, kmax = 0.f;
  if (c.ntok > 0) {
    kmin = ordered_to_float(ks[0]);
    kmax = ordered_to_float(ks[1]);
  }
  const float lev = c.lp->key_levels[h];
  const float scale = __fdiv_rn(fmaxf(__fsub_rn(kmax, kmin), kRangeEps), lev - 1.0f);
  if (pairs) {  // [min(2p), min(2p+1), rcp(2p), rcp(2p+1)] per channel pair p
    s_min[4 * (n >> 1) + (n & 1)] = kmin;
    s_min[4 * (n >> 1) + 2 + (n & 1)] = __frcp_rn(scale);
  } else {
    s_min[n * stride] = kmin;
    s_rcp[n * stride] = __frcp_rn(scale);
  }
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

// Value parameters of every (item, row, group) in one pass, for the
// warp-specialized quantize kernel: the same operations as value_row_params
// (min / max over the group's heads, scale = max(range, eps) / (levels - 1),
// its reciprocal), written to L.vparam and, as fp16, to the metadata.  Grid
// (ceil(max rows / 256), items).
__global__ void __launch_bounds__(256) k_value_params(LayerLaunch L) {
  const int r = blockIdx.y;
  const int row = blockIdx.x * 256 + threadIdx.x;
  const int rows = L.rt.n_rows[r];
  if (row >= rows) return;
  const LayerParams* lp = L.lps + L.rt.slot[r];
  const int H = lp->H, G = lp->n_groups;
  const long long base = L.rt.row_off[r] * H;
  __half* m = meta_base(L, r);
  for (int g = 0; g < G; ++g) {
    float mn = INFINITY, mx = -INFINITY;
    int first = -1;
    for (int hh = 0; hh < H; ++hh) {
      if (lp->group_of_head[hh] != g) continue;
      if (first < 0) first = hh;
      const float* e = L.vstat + (base + static_cast<long long>(hh) * rows + row) * 2;
      mn = fminf(mn, e[0]);
      mx = fmaxf(mx, e[1]);
    }
    if (first < 0) continue;
    const float scale =
        __fdiv_rn(fmaxf(__fsub_rn(mx, mn), kRangeEps), lp->value_levels[first] - 1.0f);
    reinterpret_cast<float2*>(L.vparam)[base + static_cast<long long>(g) * rows + row] =
        make_float2(mn, __frcp_rn(scale));
    m[2 * H * 128 + g * rows + row] = __float2half_rn(mn);
    m[2 * H * 128 + G * rows + g * rows + row] = __float2half_rn(scale);
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
      simt_forward_row(c, 1, load_block(L, c, row), row % c.kv.block_size, h, v);
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
    simt_forward_row(c, 0, load_block(L, c, row), row % c.kv.block_size, h, v);
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
    simt_forward_row(c, plane, load_block(L, c, row), row % c.kv.block_size, h, v);
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
  const int phys = phys_block(L, c, row);
  if (phys < 0) return;
  store_row_bf16(kv_row(c, kv, phys, row % c.kv.block_size, h), v);
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
      if (phys < 0) continue;  // bad block id: recorded, box skipped
      const int slot = rr % c.kv.block_size;
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {
        asm volatile(
            "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%1, %2, %3, %4}], [%5];" ::
                "l"(reinterpret_cast<uint64_t>(map)),
            "r"(hb * 64), "r"(tma_y(c.kv, h, slot)), "r"(tma_z(c.kv, h, slot)), "r"(phys),
            "r"(smem_u32(sA + hb * 16384 + g * 2048))
            : "memory");
      }
    }
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
  }
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 128);
}

// ============================================= persistent tcgen05 engine
// One CTA per half SM (2 CTAs/SM, 256 threads each) walks a contiguous range
// of jobs; job j = (plane, head, tile) with the tile index fastest, so
// consecutive jobs of a CTA share the transform image (reloaded only when
// the (layer slot, head) changes) and the key-statistics accumulators.
// Shared memory: transform image (32 KB) + two 32 KB tile stages; TMEM: two
// 128-column fp32 accumulators (quant/stats) or one (dequant).  The TMA
// load of job i+1 is in flight while job i runs its MMA and epilogue.
//
// Warp w of the 8 reads TMEM lanes 32*(w%4).. (its quadrant) and the
// column half w/4 of the accumulator.
constexpr int kPThreads = 256;
// image + 2 stages + barriers/scalars (64 B) + f0,f1 (2 KB) + red (2 KB) + 1 KB alignment slack
constexpr int kPSmem = 3 * 32768 + 64 + 2048 + 2048 + 1024;

struct PJob {
  int plane, h, tile;
};
KVS_DEV PJob pjob(int j, int H, int T) {
  PJob o;
  const int q = j / T;
  o.tile = j - q * T;
  o.h = q % H;
  o.plane = q / H;
  return o;
}

struct PSmem;
KVS_DEV uint8_t* pstage(const PSmem& S, int k);

struct PSmem {
  uint8_t* img;     // stage k follows at img + 32768 * (k + 1)
  uint64_t* full;   // [2] tile stage loaded
  uint64_t* mma;    // [2] accumulator ready
  uint64_t* imgb;   // image loaded
  uint32_t* tslot;
  int* abort_flag;
  float* f0;        // 256 floats
  float* f1;        // 256 floats
  float* red;       // 512 floats (cross-half reductions)
};

KVS_DEV PSmem psmem(uint8_t* raw) {
  uint8_t* s = align1024(raw);
  PSmem p;
  p.img = s;
  uint8_t* m = s + 98304;
  p.full = reinterpret_cast<uint64_t*>(m);
  p.mma = p.full + 2;
  p.imgb = p.full + 4;
  p.tslot = reinterpret_cast<uint32_t*>(m + 48);
  p.abort_flag = reinterpret_cast<int*>(m + 52);
  p.f0 = reinterpret_cast<float*>(m + 64);
  p.f1 = p.f0 + 256;
  p.red = reinterpret_cast<float*>(m + 64 + 2048);
  return p;
}

// Jobs [j0, j1) of this CTA (the host keeps 2*H*T below 2^31).
KVS_DEV uint8_t* pstage(const PSmem& S, int k) { return S.img + 32768 * (k + 1); }

KVS_DEV void pjob_range(int J, int& j0, int& j1) {
  j0 = static_cast<int>(static_cast<long long>(blockIdx.x) * J / gridDim.x);
  j1 = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * J / gridDim.x);
}

// Thread 0: issue the tile loads of job j into `stage` (phase completes on `bar`).
KVS_DEV void p_issue_job(const LayerLaunch& L, int j, uint8_t* stage, uint64_t* bar) {
  const PJob jb = pjob(j, L.num_heads, L.total_tiles);
  const ItemCtx c = item_ctx(L, jb.tile);
  issue_tile_loads(L, c, map_of(L, c.slot, jb.plane), jb.h, stage, bar, 0u);
}

// Thread 0 after an abort: wait (bounded, no error recording) for loads
// issued for local jobs [from, to) so that no copy is in flight at exit.
// The abort flag is written only by thread 0 before a __syncthreads and read
// by every thread right after it, so all threads leave the loop together.
KVS_DEV void p_drain(const PSmem& S, int from, int to) {
  for (int k = from; k < to; ++k)
    mbar_wait(&S.full[k & 1], static_cast<uint32_t>((k >> 1) & 1), nullptr, 0);
}

// ------------------------------------------------------------------ stats
__global__ void __launch_bounds__(kPThreads, 2) k_stats_tc(LayerLaunch L) {
  extern __shared__ uint8_t smem_raw[];
  const PSmem S = psmem(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, half = warp >> 2;
  const int H = L.num_heads, T = L.total_tiles;
  int j0, j1;
  pjob_range(2 * H * T, j0, j1);
  const int n = j1 - j0;
  if (n <= 0) return;
  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&S.full[i], 1);
      mbar_init(&S.mma[i], 1);
    }
    mbar_init(S.imgb, 1);
    *S.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(S.tslot, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *S.tslot;
  int issued = 0;
  if (tid == 0) {
    for (; issued < 2 && issued < n; ++issued)
      p_issue_job(L, j0 + issued, pstage(S, issued & 1), &S.full[issued & 1]);
  }
  int cur_img = -1;
  uint32_t img_phase = 0;
  // running key min/max of this thread's channel over consecutive jobs of
  // the same (item, head)
  float run_mn = INFINITY, run_mx = -INFINITY;
  int run_key = -1;  // r * H + h of the running accumulation, -1 = none
  const int lane_id = quad * 32 + lane;  // TMEM lane = channel (keys) or row (values)
  for (int i = 0; i < n; ++i) {
    const int s = static_cast<int>(i & 1);
    const uint32_t ph = static_cast<uint32_t>((i >> 1) & 1);
    const PJob jb = pjob(j0 + i, H, T);
    const ItemCtx c = item_ctx(L, jb.tile);
    const int img_key = c.slot * H + jb.h;
    const uint32_t acc = tmem + static_cast<uint32_t>(s * 128);
    if (tid == 0) {
      bool ok = true;
      if (img_key != cur_img) {
        mbar_arrive_expect_tx(S.imgb, 32768u);
        bulk_load(S.img, bmat_of(L, c.slot, jb.h), 32768, S.imgb);
        ok = mbar_wait(S.imgb, img_phase, L.err, ERR_MBAR_TIMEOUT);
        img_phase ^= 1u;
      }
      ok = ok && mbar_wait(&S.full[s], ph, L.err, ERR_MBAR_TIMEOUT);
      if (ok) {
        tc_fence_after();
        if (jb.plane == 0) {
          umma_tile_128x128x128(acc, smem_u32(S.img), smem_u32(pstage(S, s)));  // lane = channel
        } else {
          umma_tile_128x128x128(acc, smem_u32(pstage(S, s)), smem_u32(S.img));  // lane = row
        }
      }
      umma_commit(&S.mma[s]);
      if (!ok) *S.abort_flag = 1;
    }
    cur_img = img_key;
    __syncthreads();
    if (*S.abort_flag) {
      if (tid == 0) p_drain(S, i, issued);
      break;
    }
    mbar_wait(&S.mma[s], ph, L.err, ERR_MBAR_TIMEOUT);  // a timeout is recorded in L.err
    tc_fence_after();
    if (tid == 0 && issued < n) {  // stage s is free: the MMA that read it is done
      p_issue_job(L, j0 + issued, pstage(S, s), &S.full[s]);
      ++issued;
    }
    const float sc = c.lp->out_scale;
    const uint32_t taddr = acc + (static_cast<uint32_t>(quad * 32) << 16) + half * 64;
    float mn = INFINITY, mx = -INFINITY;
    if (jb.plane == 0) {
      const int nvalid = min(kTileRows, c.ntok - c.row0);
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        float v[32];
        tmem_ld32(taddr + cc * 32, v);
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          if (half * 64 + cc * 32 + k < nvalid) {
            mn = fminf(mn, v[k]);
            mx = fmaxf(mx, v[k]);
          }
        }
      }
      // fl(x*sc) is non-decreasing in x for sc > 0, so min/max commute with
      // the scaling: one multiply per thread instead of one per element.
      if (mn <= mx) {
        mn *= sc;
        mx *= sc;
      }
      const int key = c.r * H + jb.h;
      if (key != run_key) {
        if (run_key >= 0 && run_mn <= run_mx) {
          uint32_t* ks = L.kstat + (static_cast<size_t>(run_key) * 128 + lane_id) * 2;
          atomicMin(ks, float_to_ordered(run_mn));
          atomicMax(ks + 1, float_to_ordered(run_mx));
        }
        run_key = key;
        run_mn = INFINITY;
        run_mx = -INFINITY;
      }
      run_mn = fminf(run_mn, mn);
      run_mx = fmaxf(run_mx, mx);
    } else {
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        float v[32];
        tmem_ld32(taddr + cc * 32, v);
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          mn = fminf(mn, v[k]);
          mx = fmaxf(mx, v[k]);
        }
      }
      mn *= sc;
      mx *= sc;
      if (half == 1) {
        S.red[lane_id * 2] = mn;
        S.red[lane_id * 2 + 1] = mx;
      }
    }
    tc_fence_before();
    __syncthreads();
    if (jb.plane == 1 && half == 0) {
      mn = fminf(mn, S.red[lane_id * 2]);
      mx = fmaxf(mx, S.red[lane_id * 2 + 1]);
      const int row = c.row0 + lane_id;
      if (row < c.rows) {
        if (row >= c.ntok) mn = mx = 0.f;
        float* e = vstat_entry(L, c, jb.h, row);
        e[0] = mn;
        e[1] = mx;
      }
    }
    __syncthreads();  // S.red reusable
  }
  if (run_key >= 0 && run_mn <= run_mx) {
    uint32_t* ks = L.kstat + (static_cast<size_t>(run_key) * 128 + lane_id) * 2;
    atomicMin(ks, float_to_ordered(run_mn));
    atomicMax(ks + 1, float_to_ordered(run_mx));
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

// ------------------------------------------------------------------ quant
// Epilogue of one half row: 64 values -> two 32-code groups of W bits,
// staged at the row's pitch (W|1)*16 bytes, groups 2*half and 2*half+1.
// Codes of 32 consecutive columns (raw bits of 2^23 + code) -> W-bit
// packed words.  For W = 8 the code byte is the low byte of the bits.
template <int W>
KVS_DEV void pack_code_bits(const uint32_t (&b)[32], uint32_t (&w)[8]) {
  if constexpr (W == 8) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t lo = __byte_perm(b[4 * i], b[4 * i + 1], 0x0040);
      const uint32_t hi = __byte_perm(b[4 * i + 2], b[4 * i + 3], 0x0040);
      w[i] = __byte_perm(lo, hi, 0x5410);
    }
  } else {
    uint32_t q[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) q[k] = b[k] & ((1u << W) - 1u);
    pack32<W>(q, w);
  }
}

// Epilogue of one half row: 64 values -> two 32-code groups of W bits,
// staged at the row's pitch, groups 2*half and 2*half+1.  kp holds the key
// (min, rcp) pairs per column, interleaved.
template <int W>
KVS_DEV void p_quant_half(uint32_t taddr, float sc, float top, bool valid, int plane,
                          float vmin, float vrcp, const float* kp, int half,
                          uint8_t* row_stage) {
#pragma unroll
  for (int cc = 0; cc < 2; ++cc) {
    float v[32];
    tmem_ld32(taddr + cc * 32, v);
    uint32_t b[32];
#pragma unroll
    for (int k = 0; k < 32; k += 2) {
      const uint32_t pr = valid ? cvt_bf16x2(v[k] * sc, v[k + 1] * sc) : 0u;
      const float x0 = bf16lo_to_float(pr), x1 = bf16hi_to_float(pr);
      if (plane == 0) {
        const float4 m = *reinterpret_cast<const float4*>(kp + 2 * (half * 64 + cc * 32 + k));
        b[k] = quantize_bits(x0, m.x, m.y, top);
        b[k + 1] = quantize_bits(x1, m.z, m.w, top);
      } else {
        b[k] = quantize_bits(x0, vmin, vrcp, top);
        b[k + 1] = quantize_bits(x1, vmin, vrcp, top);
      }
    }
    uint32_t w[8];
    pack_code_bits<W>(b, w);
    uint32_t* dst = reinterpret_cast<uint32_t*>(row_stage + (2 * half + cc) * 4 * W);
#pragma unroll
    for (int k = 0; k < W; ++k) dst[k] = w[k];
  }
}

// Warp-specialized form of p_quant_half: values go through the quantizer in
// pairs (f32x2 arithmetic), key parameters are read in the pair layout
// [min(2p), min(2p+1), rcp(2p), rcp(2p+1)], and 4-bit codes are packed two
// per byte with one shift-add (the low bytes of the biased bits are the
// codes) and gathered four bytes per word with byte permutes.  Codes are
// identical to p_quant_half's.
template <int W>
KVS_DEV void ws_quant_half(uint32_t taddr, float sc, float top, bool valid, int plane,
                           float vmin, float vrcp, const float* kp, int half,
                           uint8_t* row_stage) {
  const f32x2_t sc2 = f2_pack(sc, sc);
  const f32x2_t vmn2 = f2_pack(vmin, vmin), vrcp2 = f2_pack(vrcp, vrcp);
#pragma unroll
  for (int cc = 0; cc < 2; ++cc) {
    float v[32];
    tmem_ld32(taddr + cc * 32, v);
    uint32_t w[8];
    uint32_t b[32];
    uint32_t nib[16];
#pragma unroll
    for (int k = 0; k < 32; k += 2) {
      float y0, y1;
      f2_unpack(f2_mul(f2_pack(v[k], v[k + 1]), sc2), y0, y1);
      const uint32_t pr = valid ? cvt_bf16x2(y0, y1) : 0u;
      const float x0 = bf16lo_to_float(pr), x1 = bf16hi_to_float(pr);
      f32x2_t mn2 = vmn2, rcp2 = vrcp2;
      if (plane == 0) {
        const float4 m = *reinterpret_cast<const float4*>(kp + 2 * (half * 64 + cc * 32 + k));
        mn2 = f2_pack(m.x, m.y);
        rcp2 = f2_pack(m.z, m.w);
      }
      if constexpr (W == 4 || W == 8) {
        uint32_t b0, b1;
        quantize_bits2(x0, x1, mn2, rcp2, top, b0, b1);
        if constexpr (W == 4)
          nib[k >> 1] = b0 + (b1 << 4);  // low byte: code k | code k+1 << 4
        else
          nib[k >> 1] = __byte_perm(b0, b1, 0x0040);  // low half: code k | code k+1 << 8
      } else {  // scalar form (fewer live registers for the odd widths)
        float m0, m1, r0, r1;
        f2_unpack(mn2, m0, m1);
        f2_unpack(rcp2, r0, r1);
        b[k] = quantize_bits(x0, m0, r0, top);
        b[k + 1] = quantize_bits(x1, m1, r1, top);
      }
    }
    if constexpr (W == 4) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t lo = __byte_perm(nib[4 * i], nib[4 * i + 1], 0x0040);
        const uint32_t hi = __byte_perm(nib[4 * i + 2], nib[4 * i + 3], 0x0040);
        w[i] = __byte_perm(lo, hi, 0x5410);
      }
    } else if constexpr (W == 8) {
#pragma unroll
      for (int i = 0; i < 8; ++i) w[i] = __byte_perm(nib[2 * i], nib[2 * i + 1], 0x5410);
    } else {
      pack_code_bits<W>(b, w);
    }
    uint32_t* dst = reinterpret_cast<uint32_t*>(row_stage + (2 * half + cc) * 4 * W);
    if constexpr (W == 4 || W == 8) {  // 16-byte stores: the row pitch is an odd multiple of 16
#pragma unroll
      for (int k = 0; k < W; k += 4)
        *reinterpret_cast<uint4*>(dst + k) = make_uint4(w[k], w[k + 1], w[k + 2], w[k + 3]);
    } else {
#pragma unroll
      for (int k = 0; k < W; ++k) dst[k] = w[k];
    }
  }
}

__global__ void __launch_bounds__(kPThreads, 2) k_quant_tc(LayerLaunch L) {
  extern __shared__ uint8_t smem_raw[];
  const PSmem S = psmem(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, half = warp >> 2;
  const int H = L.num_heads, T = L.total_tiles;
  int j0, j1;
  pjob_range(2 * H * T, j0, j1);
  const int n = j1 - j0;
  if (n <= 0) return;
  float* kp = S.f0;  // [128][2] key (min, rcp), f0 and f1 contiguous
  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&S.full[i], 1);
      mbar_init(&S.mma[i], 1);
    }
    mbar_init(S.imgb, 1);
    *S.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(S.tslot, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *S.tslot;
  int issued = 0;
  if (tid == 0) {
    for (; issued < 2 && issued < n; ++issued)
      p_issue_job(L, j0 + issued, pstage(S, issued & 1), &S.full[issued & 1]);
  }
  int cur_img = -1;
  uint32_t img_phase = 0;
  const int lane_id = quad * 32 + lane;  // TMEM lane = tile row
  for (int i = 0; i < n; ++i) {
    const int s = static_cast<int>(i & 1);
    const uint32_t ph = static_cast<uint32_t>((i >> 1) & 1);
    const PJob jb = pjob(j0 + i, H, T);
    const ItemCtx c = item_ctx(L, jb.tile);
    const int img_key = c.slot * H + jb.h;
    const uint32_t acc = tmem + static_cast<uint32_t>(s * 128);
    if (tid == 0) {
      bool ok = true;
      if (img_key != cur_img) {
        mbar_arrive_expect_tx(S.imgb, 32768u);
        bulk_load(S.img, bmat_of(L, c.slot, jb.h), 32768, S.imgb);
        ok = mbar_wait(S.imgb, img_phase, L.err, ERR_MBAR_TIMEOUT);
        img_phase ^= 1u;
      }
      ok = ok && mbar_wait(&S.full[s], ph, L.err, ERR_MBAR_TIMEOUT);
      if (ok) {
        tc_fence_after();
        umma_tile_128x128x128(acc, smem_u32(pstage(S, s)), smem_u32(S.img));  // lane = row
      }
      umma_commit(&S.mma[s]);
      if (!ok) *S.abort_flag = 1;
    }
    cur_img = img_key;
    if (jb.plane == 0 && tid < 128) key_channel_params(L, c, jb.h, kp, kp + 1, 2);
    const int row = c.row0 + lane_id;
    const bool exists = row < c.rows, valid = row < c.ntok;
    float vmin = 0.f, vrcp = 0.f;
    if (jb.plane == 1 && exists) {
      if (half == 0) {
        value_row_params(L, c, jb.h, row, &vmin, &vrcp);
        S.red[lane_id * 2] = vmin;
        S.red[lane_id * 2 + 1] = vrcp;
      }
    }
    __syncthreads();  // key params, value params, abort flag visible
    if (*S.abort_flag) {
      if (tid == 0) p_drain(S, i, issued);
      break;
    }
    if (jb.plane == 1 && half == 1 && exists) {
      vmin = S.red[lane_id * 2];
      vrcp = S.red[lane_id * 2 + 1];
    }
    mbar_wait(&S.mma[s], ph, L.err, ERR_MBAR_TIMEOUT);  // a timeout is recorded in L.err
    tc_fence_after();
    const float lev = jb.plane == 0 ? c.lp->key_levels[jb.h] : c.lp->value_levels[jb.h];
    const float top = c.lp->clamp_top ? lev - 1.0f : lev;
    const int bits = seg_bits(c, jb.plane, jb.h);
    const int P = (bits | 1) * 16;  // odd multiple of 16 B: spreads rows over bank groups
    uint8_t* stage = pstage(S, s);    // the MMA that read this tile has completed
    uint8_t* row_stage = stage + lane_id * P;
    const uint32_t taddr = acc + (static_cast<uint32_t>(quad * 32) << 16) + half * 64;
    const float sc = c.lp->out_scale;
    switch (bits) {
      case 1: p_quant_half<1>(taddr, sc, top, valid, jb.plane, vmin, vrcp, kp, half, row_stage); break;
      case 2: p_quant_half<2>(taddr, sc, top, valid, jb.plane, vmin, vrcp, kp, half, row_stage); break;
      case 3: p_quant_half<3>(taddr, sc, top, valid, jb.plane, vmin, vrcp, kp, half, row_stage); break;
      case 4: p_quant_half<4>(taddr, sc, top, valid, jb.plane, vmin, vrcp, kp, half, row_stage); break;
      case 5: p_quant_half<5>(taddr, sc, top, valid, jb.plane, vmin, vrcp, kp, half, row_stage); break;
      case 6: p_quant_half<6>(taddr, sc, top, valid, jb.plane, vmin, vrcp, kp, half, row_stage); break;
      case 7: p_quant_half<7>(taddr, sc, top, valid, jb.plane, vmin, vrcp, kp, half, row_stage); break;
      default: p_quant_half<8>(taddr, sc, top, valid, jb.plane, vmin, vrcp, kp, half, row_stage); break;
    }
    tc_fence_before();
    __syncthreads();
    // Coalesced 16-byte copy of the tile's contiguous code region.
    const int nrows = min(kTileRows, c.rows - c.row0);
    uint8_t* dst0 = code_row(L, c, jb.plane, jb.h, c.row0);
    for (int k = tid; k < nrows * bits; k += kPThreads) {
      const int r = k / bits, col = k - r * bits;
      *reinterpret_cast<uint4*>(dst0 + static_cast<long long>(k) * 16) =
          *reinterpret_cast<const uint4*>(stage + r * P + col * 16);
    }
    fence_proxy_async_smem();  // generic accesses of the stage precede the next TMA write
    __syncthreads();
    if (tid == 0 && issued < n) {
      p_issue_job(L, j0 + issued, pstage(S, s), &S.full[s]);
      ++issued;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 256);
}



// Item context kept in registers across consecutive jobs: refreshed only
// when the tile leaves [t0, t1), the current item's tile range.
struct ItemCursor {
  ItemCtx c;
  int t0, t1;
};
KVS_DEV void cursor_init(ItemCursor& k) {
  k.t0 = 1;
  k.t1 = 0;  // empty range: the first seek loads
}
KVS_DEV void cursor_seek(const LayerLaunch& L, ItemCursor& k, int tile) {
  if (tile < k.t0 || tile >= k.t1) {
    int r;
    if (tile >= k.t1 && k.t1 > k.t0 && k.c.r + 1 < L.rt.num_req && tile < L.rt.tile_prefix[k.c.r + 2])
      r = k.c.r + 1;  // the next item (the common case when walking tiles)
    else
      r = find_item(L.rt.tile_prefix, L.rt.num_req, tile);
    k.t0 = L.rt.tile_prefix[r];
    k.t1 = L.rt.tile_prefix[r + 1];
    k.c.r = r;
    k.c.slot = L.rt.slot[r];
    k.c.rows = L.rt.n_rows[r];
    k.c.ntok = L.rt.n_tokens[r];
    k.c.lp = L.lps + k.c.slot;
    k.c.kv = L.kvs[k.c.slot];
  }
  k.c.row0 = (tile - k.t0) * kTileRows;
}

// Control warp: issue the TMA loads of one tile (16 boxes: 8 row groups x
// 2 channel halves) with lanes 0-15 in parallel, so the block-table reads
// overlap; lane 0 registers the byte count first.
KVS_DEV void issue_tile_loads_warp(const LayerLaunch& L, const ItemCtx& c, const CUtensorMap* map,
                                   int h, uint8_t* tile, uint64_t* bar) {
  const int lane = threadIdx.x & 31;
  const int nload = min(8, (c.rows - c.row0 + 15) / 16);
  if (lane == 0) mbar_arrive_expect_tx(bar, static_cast<uint32_t>(nload) * 4096u);
  __syncwarp();
  if (lane < 2 * nload) {
    const int g = lane >> 1, hb = lane & 1;
    const int rr = c.row0 + g * 16;
    const int phys = load_block(L, c, rr);
    const int slot = rr % c.kv.block_size;
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(tile + hb * 16384 + g * 2048)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(hb * 64), "r"(tma_y(c.kv, h, slot)),
        "r"(tma_z(c.kv, h, slot)), "r"(phys), "r"(smem_u32(bar))
        : "memory");
  }
  __syncwarp();
}

// ====================================== warp-specialized tcgen05 engine
// One CTA per SM: a control warp (lane 0 issues every TMA load into a
// 3-stage ring and every MMA into four 128-column TMEM accumulators) and two
// epilogue groups of 8 warps that take alternate jobs of the CTA's range.
// Epilogue warps wait only on mbarriers (accumulator ready) and on their
// group's named barrier, never on the control thread's loads, so the MMA of
// job k+1 and the loads of jobs k+1..k+2 run while job k's epilogue runs.
//
// Barrier phases (job k of the CTA, acc a(k) = 2*(k&1) + ((k>>1)&1), used
// by jobs k = a's residue mod 4, use index u = k>>2):
//   full[k%3]   completes once per load (parity (k/3)&1);
//   sfree[k%3]  tcgen05.commit after MMA k (stage reusable, old image free);
//   mma[a]      tcgen05.commit after MMA k (parity u&1);
//   afree[a]    8 warp arrivals after the epilogue read accumulator a (u&1).
constexpr int kWsGroups = 2;
constexpr int kWsGroupWarps = 8;
constexpr int kWsGroupThreads = kWsGroupWarps * 32;
constexpr int kWsCtrlWarp = kWsGroups * kWsGroupWarps;  // warp 16: MMAs (dequant: loads too)
constexpr int kWsThreads = (kWsCtrlWarp + 1) * 32;       // 544 (dequantize kernel)
constexpr int kWsLoadWarp = kWsCtrlWarp + 1;             // warp 17: TMA loads (stats, quant)
constexpr int kWsProdThreads = (kWsLoadWarp + 1) * 32;   // 576 (quantize kernel)
constexpr int kWsLoadWarp2 = kWsLoadWarp + 1;            // warp 18: second TMA load warp (stats)
constexpr int kWsStatsThreads = (kWsLoadWarp2 + 1) * 32;  // 608 (stats kernel)
constexpr int kWsMaxStages = 5;
constexpr int kWsStagingBytes = 128 * 144;  // 128 rows x (W|1)*16 B for W <= 8
// Layout from the 1024-aligned base: image | NS stages | staging (quant) |
// barriers | kp | red.  NS = 5 for stats (no staging), 4 for quant.
template <int NS, bool kStaging>
struct WsLayout {
  static constexpr int kOffStages = 32768;
  static constexpr int kOffStaging = kOffStages + NS * 32768;
  static constexpr int kOffBars = kOffStaging + (kStaging ? kWsGroups * kWsStagingBytes : 0);
  static constexpr int kOffKp = kOffBars + 256;
  static constexpr int kOffRed = kOffKp + kWsGroups * 256 * 4;
  static constexpr int kUsed = kOffRed + kWsGroups * 2 * 256 * 4;
  static constexpr int kSmem = kUsed + 1024;  // + alignment slack
  static_assert(kSmem <= 227 * 1024, "warp-specialized shared memory");
};
using WsStatsLayout = WsLayout<5, false>;
using WsQuantLayout = WsLayout<4, true>;

struct WsSmem {
  uint8_t* base;
  int off_staging, off_kp, off_red;
  uint64_t* full;   // [NS]
  uint64_t* sfree;  // [NS]
  uint64_t* mma;    // [4]
  uint64_t* afree;  // [4]
  uint64_t* imgb;
  uint32_t* tslot;
};
template <class LY>
KVS_DEV WsSmem ws_smem(uint8_t* raw) {
  WsSmem w;
  w.base = align1024(raw);
  w.off_staging = LY::kOffStaging;
  w.off_kp = LY::kOffKp;
  w.off_red = LY::kOffRed;
  uint64_t* b = reinterpret_cast<uint64_t*>(w.base + LY::kOffBars);
  w.full = b;
  w.sfree = b + kWsMaxStages;
  w.mma = b + 2 * kWsMaxStages;
  w.afree = b + 2 * kWsMaxStages + 4;
  w.imgb = b + 2 * kWsMaxStages + 8;
  w.tslot = reinterpret_cast<uint32_t*>(b + 2 * kWsMaxStages + 9);
  return w;
}
KVS_DEV uint8_t* ws_img(const WsSmem& S) { return S.base; }
KVS_DEV uint8_t* ws_stage(const WsSmem& S, int k) { return S.base + 32768 + 32768 * k; }
KVS_DEV uint8_t* ws_staging(const WsSmem& S, int g) {
  return S.base + S.off_staging + kWsStagingBytes * g;
}
KVS_DEV float* ws_kp(const WsSmem& S, int g) {
  return reinterpret_cast<float*>(S.base + S.off_kp) + 256 * g;
}
KVS_DEV float* ws_red(const WsSmem& S, int g, int k) {
  return reinterpret_cast<float*>(S.base + S.off_red) + 256 * (2 * g + ((k >> 1) & 1));
}
KVS_DEV int ws_acc(int k) { return 2 * (k & 1) + ((k >> 1) & 1); }
KVS_DEV void group_sync(int g) {
  asm volatile("bar.sync %0, %1;" ::"r"(1 + g), "r"(kWsGroupThreads) : "memory");
}

KVS_DEV void ws_init(const WsSmem& S, int NS) {
  for (int i = 0; i < NS; ++i) {
    mbar_init(&S.full[i], 1);
    mbar_init(&S.sfree[i], 1);
  }
  for (int i = 0; i < 4; ++i) {
    mbar_init(&S.mma[i], 1);
    mbar_init(&S.afree[i], kWsGroupWarps);
  }
  mbar_init(S.imgb, 1);
  fence_mbar_init();
}


KVS_DEV void trace_mark(const LayerLaunch& L, int k, int ev) {
  if (L.trace != nullptr && blockIdx.x < kTraceCtas && k < L.trace_jobs)
    L.trace[(static_cast<long long>(blockIdx.x) * L.trace_jobs + k) * 8 + ev] = globaltimer();
}


// Job mapping of the warp-specialized kernels: the grid is 2*H*R CTAs; CTA b
// owns (plane, head) = (b % (2H)) and tile range r = b / (2H) of R equal
// ranges.  The CTAs of one range (all heads, both planes) run concurrently
// and stream the same tiles, so the heads' 256-byte pieces of each 1 KB
// token row reach DRAM together (row-buffer locality); each CTA's transform
// image changes only at layer boundaries.  Job k of a CTA is tile t0 + k.
struct WsMap {
  int plane, h, t0, n;
};
KVS_DEV WsMap ws_map(const LayerLaunch& L) {
  const int PH = 2 * L.num_heads;
  const int R = gridDim.x / PH;
  const int b = blockIdx.x, ph = b % PH, r = b / PH;
  WsMap m;
  m.plane = ph / L.num_heads;
  m.h = ph % L.num_heads;
  m.t0 = static_cast<int>(static_cast<long long>(r) * L.total_tiles / R);
  m.n = static_cast<int>(static_cast<long long>(r + 1) * L.total_tiles / R) - m.t0;
  return m;
}
KVS_DEV PJob ws_job(const WsMap& m, int k) {
  PJob j;
  j.plane = m.plane;
  j.h = m.h;
  j.tile = m.t0 + k;
  return j;
}

// One job's TMA boxes as seen by one control-warp lane: lane l < 16 owns
// box (row group l/2, channel half l%2).  The block-table read is done when
// the descriptor is prepared, one job before the loads are issued, so the
// issue itself never waits on memory.
struct BoxDesc {
  const CUtensorMap* map;
  int y, z, phys, nload;  // y, z: TMA coordinates of (head, slot)
  int num_blocks;         // phys is checked against it when the box is issued
  bool mine;
};
KVS_DEV BoxDesc box_desc(const LayerLaunch& L, ItemCursor& cur, const PJob& jb) {
  const int lane = threadIdx.x & 31;
  cursor_seek(L, cur, jb.tile);
  const ItemCtx& c = cur.c;
  BoxDesc d;
  d.map = map_of(L, c.slot, jb.plane);
  d.nload = min(8, (c.rows - c.row0 + 15) / 16);
  d.mine = lane < 2 * d.nload;
  d.num_blocks = c.kv.num_blocks;
  d.y = d.z = d.phys = 0;
  if (d.mine) {
    const int rr = c.row0 + (lane >> 1) * 16;
    const int slot = rr % c.kv.block_size;
    d.phys = raw_block(L, c, rr);
    d.y = tma_y(c.kv, jb.h, slot);
    d.z = tma_z(c.kv, jb.h, slot);
  }
  return d;
}
KVS_DEV void issue_boxes(const BoxDesc& d, uint8_t* tile, uint64_t* bar, uint32_t* err) {
  const int lane = threadIdx.x & 31;
  if (lane == 0) mbar_arrive_expect_tx(bar, static_cast<uint32_t>(d.nload) * 4096u);
  __syncwarp();
  if (d.mine) {
    int phys = d.phys;
    if (static_cast<unsigned>(phys) >= static_cast<unsigned>(d.num_blocks)) {
      record_error(err, ERR_BOUNDS);  // outside the cache: read block 0 instead
      phys = 0;
    }
    const int g = lane >> 1, hb = lane & 1;
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(tile + hb * 16384 + g * 2048)),
        "l"(reinterpret_cast<uint64_t>(d.map)), "r"(hb * 64), "r"(d.y), "r"(d.z), "r"(phys),
        "r"(smem_u32(bar))
        : "memory");
  }
  __syncwarp();
}

// Load warps: TMA loads of local jobs [0, n) into the NS-stage ring.  Job j
// goes into stage j % NS as soon as the MMA of job j - NS (the stage's
// previous user) has retired.  With `nl` load warps, warp `first` takes jobs
// first, first + nl, ...: issuing a tile's 16 boxes (lanes 0-15, one box
// each) and reading the block ids of its jobs take a warp about a
// microsecond, so the warps' issues overlap.  A warp reads the block ids of
// its job three issues ahead (the loop is unrolled by three and each
// descriptor is refilled in place after its boxes are issued), so a read's
// latency stays off the loop.  Lane 0 waits on barriers.  After a failed wait
// a warp stops issuing; before returning it waits (bounded) for the copies
// it issued into the ring's last stages.
template <int NS, bool kTraceLoader = false>
KVS_DEV void ws_loader(const LayerLaunch& L, const WsSmem& S, const WsMap& M, int first = 0,
                       int nl = 1) {
  const int n = M.n;
  const int lane = threadIdx.x & 31;
  ItemCursor ld;
  cursor_init(ld);
  auto wait0 = [&](uint64_t* bar, uint32_t parity) -> bool {
    bool r = true;
    if (lane == 0) r = mbar_wait(bar, parity, L.err, ERR_MBAR_TIMEOUT);
    return __shfl_sync(0xFFFFFFFFu, r ? 1 : 0, 0) != 0;
  };
  int job = first;  // the next job this warp issues
  BoxDesc q0 = box_desc(L, ld, ws_job(M, min(job, n - 1)));
  BoxDesc q1 = job + nl < n ? box_desc(L, ld, ws_job(M, job + nl)) : q0;
  BoxDesc q2 = job + 2 * nl < n ? box_desc(L, ld, ws_job(M, job + 2 * nl)) : q0;
  auto step = [&](BoxDesc& q) -> bool {  // issue `job` from q, refill q
    const int st = job % NS;
    if (job >= NS && !wait0(&S.sfree[st], static_cast<uint32_t>((job / NS - 1) & 1)))
      return false;
    if (lane == 0 && kTraceLoader) trace_mark(L, job, 6);
    issue_boxes(q, ws_stage(S, st), &S.full[st], L.err);
    if (lane == 0) trace_mark(L, job, 2);
    if (job + 3 * nl < n) q = box_desc(L, ld, ws_job(M, job + 3 * nl));
    if (lane == 0 && kTraceLoader) trace_mark(L, job, 7);
    job += nl;
    return true;
  };
  while (job < n) {
    if (!step(q0) || job >= n) break;
    if (!step(q1) || job >= n) break;
    if (!step(q2)) break;
  }
  // This warp's copies among the last NS jobs landed (every earlier job's
  // had landed before its stage was refilled; a stage whose phase moved on
  // twice must not be waited on with the old parity).
  if (lane == 0)
    for (int j = job - nl; j >= first && j >= n - NS; j -= nl)
      mbar_wait(&S.full[j % NS], static_cast<uint32_t>((j / NS) & 1), nullptr, 0);
}

// MMA warp: for local jobs [0, n), wait for the job's tile and a free
// accumulator, issue its 128x128x128 MMA and commit the accumulator and the
// stage.  The transform image is reloaded when the (layer slot, head)
// changes, after the previous MMA has retired.  Lane 0 waits and issues.
// After a failed wait it stops waiting and issuing but keeps committing, so
// every epilogue and load barrier still completes.
template <bool kStats, int NS>
KVS_DEV void ws_mma(const LayerLaunch& L, const WsSmem& S, uint32_t tmem, const WsMap& M) {
  const int H = L.num_heads;
  const int n = M.n;
  const int lane = threadIdx.x & 31;
  ItemCursor mm;
  cursor_init(mm);
  auto wait0 = [&](uint64_t* bar, uint32_t parity) -> bool {
    bool r = true;
    if (lane == 0) r = mbar_wait(bar, parity, L.err, ERR_MBAR_TIMEOUT);
    return __shfl_sync(0xFFFFFFFFu, r ? 1 : 0, 0) != 0;
  };
  int cur_img = -1;
  uint32_t img_phase = 0;
  bool ok = true;
  for (int k = 0; k < n; ++k) {
    const int st = k % NS;
    const int a = ws_acc(k);
    const PJob jb = ws_job(M, k);
    cursor_seek(L, mm, jb.tile);
    const int img_key = mm.c.slot * H + jb.h;
    if (ok && img_key != cur_img) {
      if (k >= 1)  // MMA k-1 done: the old image is no longer read
        ok = wait0(&S.sfree[(k - 1) % NS], static_cast<uint32_t>(((k - 1) / NS) & 1));
      if (ok) {
        if (lane == 0) {
          mbar_arrive_expect_tx(S.imgb, 32768u);
          bulk_load(ws_img(S), bmat_of(L, mm.c.slot, jb.h), 32768, S.imgb);
        }
        ok = wait0(S.imgb, img_phase);
        img_phase ^= 1u;
      }
      cur_img = img_key;
    }
    if (ok) ok = wait0(&S.full[st], static_cast<uint32_t>((k / NS) & 1));
    if (lane == 0) trace_mark(L, k, 0);
    if (ok && k >= 4) ok = wait0(&S.afree[a], static_cast<uint32_t>(((k >> 2) - 1) & 1));
    if (lane == 0) trace_mark(L, k, 5);
    if (lane == 0) {
      if (ok) {
        tc_fence_after();
        const uint32_t acc = tmem + static_cast<uint32_t>(a * 128);
        if (kStats && jb.plane == 0) {
          umma_tile_128x128x128(acc, smem_u32(ws_img(S)), smem_u32(ws_stage(S, st)));  // lane = channel
        } else {
          umma_tile_128x128x128(acc, smem_u32(ws_stage(S, st)), smem_u32(ws_img(S)));  // lane = row
        }
      }
      umma_commit(&S.mma[a]);
      umma_commit(&S.sfree[st]);
      trace_mark(L, k, 1);
    }
    __syncwarp();
  }
}

// ------------------------------------------------------------ stats (ws)
__global__ void __launch_bounds__(kWsStatsThreads, 1) k_stats_ws(LayerLaunch L) {
  extern __shared__ uint8_t smem_raw[];
  constexpr int NS = 5;
  const WsSmem S = ws_smem<WsStatsLayout>(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int H = L.num_heads;
  const WsMap M = ws_map(L);
  const int n = M.n;
  if (n <= 0) return;
  if (tid == 0) ws_init(S, NS);
  if (warp == kWsCtrlWarp) tmem_alloc(S.tslot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *S.tslot;
  if (warp == kWsCtrlWarp) {
    ws_mma<true, NS>(L, S, tmem, M);
  } else if (warp == kWsLoadWarp || warp == kWsLoadWarp2) {
    ws_loader<NS>(L, S, M, warp - kWsLoadWarp, 2);
  } else {
    const int g = warp / kWsGroupWarps, gw = warp % kWsGroupWarps;
    const int quad = gw & 3, half = gw >> 2;
    const int lane_id = quad * 32 + lane;  // TMEM lane = channel (keys) or row (values)
    float run_mn = INFINITY, run_mx = -INFINITY;
    int run_key = -1;
    ItemCursor cur;
    cursor_init(cur);
    for (int k = g; k < n; k += kWsGroups) {
      const PJob jb = ws_job(M, k);
      cursor_seek(L, cur, jb.tile);
      const ItemCtx& c = cur.c;
      const int a = ws_acc(k);
      mbar_wait(&S.mma[a], static_cast<uint32_t>((k >> 2) & 1), L.err, ERR_MBAR_TIMEOUT);
      if (gw == 0 && lane == 0) trace_mark(L, k, 3);
      tc_fence_after();
      const uint32_t taddr = tmem + static_cast<uint32_t>(a * 128) +
                             (static_cast<uint32_t>(quad * 32) << 16) + half * 64;
      float mn = INFINITY, mx = -INFINITY;
      const int nvalid = jb.plane == 0 ? min(kTileRows, c.ntok - c.row0) : kTileRows;
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        float v[32];
        tmem_ld32(taddr + cc * 32, v);
#pragma unroll
        for (int q = 0; q < 32; ++q) {
          if (half * 64 + cc * 32 + q < nvalid) {
            mn = fminf(mn, v[q]);
            mx = fmaxf(mx, v[q]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.afree[a]);
      // fl(x*sc) is non-decreasing in x for sc > 0: scale the extremes once.
      const float sc = c.lp->out_scale;
      if (mn <= mx) {
        mn *= sc;
        mx *= sc;
      }
      float* red = ws_red(S, g, k);
      if (jb.plane == 0) {
        const int key = c.r * H + jb.h;
        if (key != run_key) {
          if (run_key >= 0 && run_mn <= run_mx) {
            uint32_t* ks = L.kstat + (static_cast<size_t>(run_key) * 128 + lane_id) * 2;
            atomicMin(ks, float_to_ordered(run_mn));
            atomicMax(ks + 1, float_to_ordered(run_mx));
          }
          run_key = key;
          run_mn = INFINITY;
          run_mx = -INFINITY;
        }
        run_mn = fminf(run_mn, mn);
        run_mx = fmaxf(run_mx, mx);
      } else if (half == 1) {
        red[lane_id * 2] = mn;
        red[lane_id * 2 + 1] = mx;
      }
      group_sync(g);
      if (jb.plane == 1 && half == 0) {
        mn = fminf(mn, red[lane_id * 2]);
        mx = fmaxf(mx, red[lane_id * 2 + 1]);
        const int row = c.row0 + lane_id;
        if (row < c.rows) {
          if (row >= c.ntok) mn = mx = 0.f;
          float* e = vstat_entry(L, c, jb.h, row);
          e[0] = mn;
          e[1] = mx;
        }
      }
      if (gw == 0 && lane == 0) trace_mark(L, k, 4);
    }
    if (run_key >= 0 && run_mn <= run_mx) {
      uint32_t* ks = L.kstat + (static_cast<size_t>(run_key) * 128 + lane_id) * 2;
      atomicMin(ks, float_to_ordered(run_mn));
      atomicMax(ks + 1, float_to_ordered(run_mx));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kWsCtrlWarp) tmem_dealloc(tmem, 512);
}

// ------------------------------------------------------------ quant (ws)
__global__ void __launch_bounds__(kWsProdThreads, 1) k_quant_ws(LayerLaunch L) {
  extern __shared__ uint8_t smem_raw[];
  constexpr int NS = 4;
  const WsSmem S = ws_smem<WsQuantLayout>(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int H = L.num_heads;
  const WsMap M = ws_map(L);
  const int n = M.n;
  if (n <= 0) return;
  if (tid == 0) ws_init(S, NS);
  if (warp == kWsCtrlWarp) tmem_alloc(S.tslot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *S.tslot;
  if (warp == kWsCtrlWarp) {
    ws_mma<false, NS>(L, S, tmem, M);
  } else if (warp == kWsLoadWarp) {
    ws_loader<NS>(L, S, M);
  } else {
    const int g = warp / kWsGroupWarps, gw = warp % kWsGroupWarps;
    const int gtid = tid - g * kWsGroupThreads;
    const int quad = gw & 3, half = gw >> 2;
    const int lane_id = quad * 32 + lane;  // TMEM lane = tile row
    float* kp = ws_kp(S, g);  // key (min, min, rcp, rcp) per channel pair
    uint8_t* stage = ws_staging(S, g);
    ItemCursor cur;
    cursor_init(cur);
    int kp_key = -1;  // (item, head) whose key parameters kp holds
    // Value (min, 1/scale) of this thread's row in job kk (k_value_params
    // computed them); loaded one job of the group ahead, so the load's
    // latency hides behind the current job.  The plane is the CTA's; the
    // item of job kk is tracked by (pr, tiles [pt0, pt1)) only.
    int pr = 0, pt0 = 0, pt1 = 0;
    auto load_vp = [&](int kk) -> float2 {
      if (M.plane != 1 || kk >= n) return make_float2(0.f, 0.f);
      const int tile = ws_job(M, kk).tile;
      if (tile < pt0 || tile >= pt1) {
        pr = find_item(L.rt.tile_prefix, L.rt.num_req, tile);
        pt0 = L.rt.tile_prefix[pr];
        pt1 = L.rt.tile_prefix[pr + 1];
      }
      const int rows = L.rt.n_rows[pr];
      const int prow = (tile - pt0) * kTileRows + lane_id;
      if (prow >= rows) return make_float2(0.f, 0.f);
      const int grp = L.lps[L.rt.slot[pr]].group_of_head[M.h];
      return reinterpret_cast<const float2*>(L.vparam)[L.rt.row_off[pr] * H +
                                                       static_cast<long long>(grp) * rows + prow];
    };
    float2 vp_next = load_vp(g);
    unsigned long long ck1 = 0, ck2 = 0;  // message checksum of this thread's code stores
    for (int k = g; k < n; k += kWsGroups) {
      const PJob jb = ws_job(M, k);
      cursor_seek(L, cur, jb.tile);
      const ItemCtx& c = cur.c;
      const int pk = c.r * H + jb.h;
      const int row = c.row0 + lane_id;
      const bool valid = row < c.ntok;
      const float2 vp = vp_next;
      vp_next = load_vp(k + kWsGroups);
      const float vmin = vp.x, vrcp = vp.y;
      if (jb.plane == 0 && (pk != kp_key || c.row0 == 0)) {  // row0 == 0 publishes the metadata
        // kp's readers of an earlier job finished before that job's staging
        // barrier, which this thread has passed
        if (gtid < 128) key_channel_params(L, c, jb.h, kp, kp, 0, gtid, true);
        kp_key = pk;
      }
      // key parameters visible; every thread finished copying out the
      // group's previous job, so the staging buffer is free
      group_sync(g);
      const int a = ws_acc(k);
      mbar_wait(&S.mma[a], static_cast<uint32_t>((k >> 2) & 1), L.err, ERR_MBAR_TIMEOUT);
      if (gw == 0 && lane == 0) trace_mark(L, k, 3);
      tc_fence_after();
      const float lev = jb.plane == 0 ? c.lp->key_levels[jb.h] : c.lp->value_levels[jb.h];
      const float top = c.lp->clamp_top ? lev - 1.0f : lev;
      const int bits = seg_bits(c, jb.plane, jb.h);
      const int P = (bits | 1) * 16;  // odd multiple of 16 B: spreads rows over bank groups
      uint8_t* row_stage = stage + lane_id * P;
      const uint32_t taddr = tmem + static_cast<uint32_t>(a * 128) +
                             (static_cast<uint32_t>(quad * 32) << 16) + half * 64;
      const float sc = c.lp->out_scale;
      switch (bits) {
        case 1: ws_quant_half<1>(taddr, sc, top, valid, jb.plane, vmin, vrcp, kp, half, row_stage); break;
        case 2: ws_quant_half<2>(taddr, sc, top, valid, jb.plane, vmin, vrcp, kp, half, row_stage); break;
        case 3: ws_quant_half<3>(taddr, sc, top, valid, jb.plane, vmin, vrcp, kp, half, row_stage); break;
        case 4: ws_quant_half<4>(taddr, sc, top, valid, jb.plane, vmin, vrcp, kp, half, row_stage); break;
        case 5: ws_quant_half<5>(taddr, sc, top, valid, jb.plane, vmin, vrcp, kp, half, row_stage); break;
        case 6: ws_quant_half<6>(taddr, sc, top, valid, jb.plane, vmin, vrcp, kp, half, row_stage); break;
        case 7: ws_quant_half<7>(taddr, sc, top, valid, jb.plane, vmin, vrcp, kp, half, row_stage); break;
        default: ws_quant_half<8>(taddr, sc, top, valid, jb.plane, vmin, vrcp, kp, half, row_stage); break;
      }
      if (gw == 0 && lane == 0) trace_mark(L, k, 6);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.afree[a]);
      group_sync(g);  // staging complete
      if (gw == 0 && lane == 0) trace_mark(L, k, 7);
      // Coalesced 16-byte copy of the tile's contiguous code region (the
      // region may be a peer GPU's receive ring: NVLink stores).
      const int nrows = min(kTileRows, c.rows - c.row0);
      uint8_t* dst0 = code_row(L, c, jb.plane, jb.h, c.row0);
      const long long dst_msg = L.ck_off + (dst0 - L.codes);
      const int total = nrows * bits;
      const int sh = (bits & (bits - 1)) == 0 ? __ffs(bits) - 1 : -1;  // log2(bits) or -1
      for (int q = gtid; q < total; q += kWsGroupThreads) {
        const int r = sh >= 0 ? (q >> sh) : q / bits, col = q - r * bits;
        const uint4 v = *reinterpret_cast<const uint4*>(stage + r * P + col * 16);
        *reinterpret_cast<uint4*>(dst0 + static_cast<long long>(q) * 16) = v;
        if (L.ck != nullptr) ck_word4(v, dst_msg + 16ll * q, ck1, ck2);
      }
      if (gw == 0 && lane == 0) trace_mark(L, k, 4);
    }
    if (L.ck != nullptr) ck_flush(L.ck, ck1, ck2);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kWsCtrlWarp) tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------- dequant
// Unpack one 32-code group of a row into bf16 and store it into the
// swizzled A tile (row t, channels 32*part..+31).
// Unpack one 32-code group of a row into bf16 and store it into the
// swizzled A tile (row t, channels 32*part..+31).  Each code becomes the
// float 2^23 + q (one byte permute for 8-bit codes), then
// bf16(bf16(q*scale) + min) with the exact-product FMA and paired
// conversions.  kp holds the key (min, scale, -2^23*scale, 0) per column.
template <int W>
KVS_DEV void p_unpack_group(const uint8_t* src, int t, int part, int kv, const float* kp,
                            float vmn, float vsc, uint8_t* sA) {
  uint32_t w[8];
  if constexpr (W == 8 || W == 4) {  // 4W-byte groups are 16-byte aligned
    const uint4* s128 = reinterpret_cast<const uint4*>(src);
#pragma unroll
    for (int k = 0; k < W / 4; ++k) {
      const uint4 u = __ldg(s128 + k);
      w[4 * k] = u.x;
      w[4 * k + 1] = u.y;
      w[4 * k + 2] = u.z;
      w[4 * k + 3] = u.w;
    }
  } else {
    const uint32_t* s32 = reinterpret_cast<const uint32_t*>(src);
#pragma unroll
    for (int k = 0; k < W; ++k) w[k] = __ldg(s32 + k);
  }
  uint32_t fb[32];  // bits of 2^23 + q
  if constexpr (W == 8) {
#pragma unroll
    for (int k = 0; k < 32; ++k)
      fb[k] = __byte_perm(w[k >> 2], 0x4B000000u, 0x7650u | (k & 3));
  } else {
    uint32_t q[32];
    unpack32<W>(w, q);
#pragma unroll
    for (int k = 0; k < 32; ++k) fb[k] = q[k] | 0x4B000000u;
  }
  const float vneg = -8388608.0f * vsc;
#pragma unroll
  for (int c8 = 0; c8 < 4; ++c8) {
    uint32_t o[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const int k = c8 * 8 + 2 * p;
      float a, b, ma, mb;
      if (kv == 0) {
        const float4 m0 = *reinterpret_cast<const float4*>(kp + 4 * (part * 32 + k));
        const float4 m1 = *reinterpret_cast<const float4*>(kp + 4 * (part * 32 + k + 1));
        a = code_times_scale(fb[k], m0.y, m0.z);
        b = code_times_scale(fb[k + 1], m1.y, m1.z);
        ma = m0.x;
        mb = m1.x;
      } else {
        a = code_times_scale(fb[k], vsc, vneg);
        b = code_times_scale(fb[k + 1], vsc, vneg);
        ma = mb = vmn;
      }
      const uint32_t prod = cvt_bf16x2(a, b);
      o[p] = cvt_bf16x2(__fadd_rn(bf16lo_to_float(prod), ma), __fadd_rn(bf16hi_to_float(prod), mb));
    }
    *reinterpret_cast<uint4*>(sA + sw128_offset(t, part * 32 + c8 * 8)) =
        make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Position of key parameter pair P (channels 2P, 2P+1 of the head) in the
// dequantize kernel's shared table of 16-byte entries (scale(2P) and
// scale(2P+1) as floats, then min(2P) | min(2P+1) << 16 as bf16 bits, then
// padding).  The XOR moves P's 16-byte column by its 128-byte row, so that
// the eight (part, chunk) pairs one quarter-warp reads in ws_unpack_group
// lie in eight different columns.
KVS_DEV int kp_pos(int P) { return P ^ ((P >> 3) & 7); }

// Warp-specialized form of p_unpack_group: codes come from the job's code
// tile in shared memory (staged by a bulk copy), q*scale runs on value pairs
// (f32x2) and the min is added to the bf16 products in bf16x2 (one rounding,
// the same value as rounding the fp32 sum).  Results are identical to
// p_unpack_group's.
template <int W>
KVS_DEV void ws_unpack_group(const uint8_t* src, int t, int part, int m, int kv,
                             const float4* kp, float vmn, float vsc, uint8_t* sA) {
  uint32_t w[8];
  if constexpr (W == 8) {  // 32-byte group: two 16-byte halves, read in rotated order
    const uint4* s = reinterpret_cast<const uint4*>(src);
    const uint4 u0 = s[m], u1 = s[m ^ 1];
    w[0] = u0.x; w[1] = u0.y; w[2] = u0.z; w[3] = u0.w;
    w[4] = u1.x; w[5] = u1.y; w[6] = u1.z; w[7] = u1.w;
  } else if constexpr (W == 4) {  // one word per chunk
    const uint4 u = *reinterpret_cast<const uint4*>(src);
    w[0] = m ? u.z : u.x;
    w[1] = m ? u.w : u.y;
    w[2] = m ? u.x : u.z;
    w[3] = m ? u.y : u.w;
  } else {  // codes straddle words: rotate the 32W-bit group by its half, 16W bits
    uint32_t v[W];
#pragma unroll
    for (int k = 0; k < W; ++k) v[k] = reinterpret_cast<const uint32_t*>(src)[k];
#pragma unroll
    for (int k = 0; k < W; ++k) {
      const uint32_t r = (W & 1) ? __funnelshift_r(v[(k + W / 2) % W], v[(k + W / 2 + 1) % W], 16)
                                 : v[(k + W / 2) % W];
      w[k] = m ? r : v[k];
    }
  }
  uint32_t fb[32];  // bits of 2^23 + q
  if constexpr (W == 8) {
#pragma unroll
    for (int k = 0; k < 32; ++k)
      fb[k] = __byte_perm(w[k >> 2], 0x4B000000u, 0x7650u | (k & 3));
  } else {
    unpack32<W>(w, fb);
#pragma unroll
    for (int k = 0; k < 32; ++k) fb[k] |= 0x4B000000u;
  }
  const f32x2_t vsc2 = f2_pack(vsc, vsc), vneg2 = f2_pack(-8388608.0f * vsc, -8388608.0f * vsc);
  const f32x2_t big2 = f2_pack(-8388608.0f, -8388608.0f);
  const uint32_t vmn2 = bf16x2_splat(vmn);
#pragma unroll
  for (int cs = 0; cs < 4; ++cs) {
    const int c8 = cs ^ (2 * m);  // channel chunk of register chunk cs
    uint32_t o[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const int k = cs * 8 + 2 * p;
      f32x2_t sc2 = vsc2, neg2 = vneg2;
      uint32_t mn2 = vmn2;
      if (kv == 0) {
        const float4 e = kp[kp_pos(part * 16 + c8 * 4 + p)];
        sc2 = f2_pack(e.x, e.y);
        neg2 = f2_mul(sc2, big2);  // exact: a power-of-two multiple
        mn2 = __float_as_uint(e.z);
      }
      float a, b;
      f2_unpack(f2_fma(f2_pack(__uint_as_float(fb[k]), __uint_as_float(fb[k + 1])), sc2, neg2),
                a, b);
      o[p] = bf16x2_add(cvt_bf16x2(a, b), mn2);
    }
    *reinterpret_cast<uint4*>(sA + sw128_offset(t, part * 32 + c8 * 8)) =
        make_uint4(o[0], o[1], o[2], o[3]);
  }
}

__global__ void __launch_bounds__(kPThreads, 2) k_dequant_tc(LayerLaunch L) {
  extern __shared__ uint8_t smem_raw[];
  const PSmem S = psmem(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int quad = warp & 3, half = warp >> 2;
  const int H = L.num_heads, T = L.total_tiles;
  int j0, j1;
  pjob_range(2 * H * T, j0, j1);
  const int n = j1 - j0;
  if (n <= 0) return;
  float* kp = S.f0;  // [128][4] key (min, scale, -2^23*scale, 0): f0 and f1 are contiguous
  if (tid == 0) {
    mbar_init(&S.mma[0], 1);
    mbar_init(S.imgb, 1);
    *S.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(S.tslot, 128);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *S.tslot;
  int cur_img = -1;
  uint32_t img_phase = 0;
  const int lane_id = (warp & 3) * 32 + (tid & 31);
  if (tid == 0) {  // warm L2 with the first two jobs' code regions
    for (int k = 0; k < 2 && k < n; ++k) {
      const PJob jb = pjob(j0 + k, H, T);
      const ItemCtx c = item_ctx(L, jb.tile);
      const int nrows = min(kTileRows, c.rows - c.row0);
      const uint32_t bytes = static_cast<uint32_t>(nrows * 16 * seg_bits(c, jb.plane, jb.h));
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(
                       code_row(L, c, jb.plane, jb.h, c.row0)),
                   "r"(bytes)
                   : "memory");
    }
  }
  for (int i = 0; i < n; ++i) {
    const int s = static_cast<int>(i & 1);
    const PJob jb = pjob(j0 + i, H, T);
    const ItemCtx c = item_ctx(L, jb.tile);
    const int img_key = c.slot * H + jb.h;
    uint8_t* sA = pstage(S, s);
    if (jb.plane == 0 && tid < 128) {
      const __half* m = meta_base(L, c.r);
      const float mn = bf16_round(__half2float(m[jb.h * 128 + tid]));
      const float sc = bf16_round(__half2float(m[c.lp->H * 128 + jb.h * 128 + tid]));
      *reinterpret_cast<float4*>(kp + 4 * tid) = make_float4(mn, sc, -8388608.0f * sc, 0.f);
    }
    if (tid == 0) {
      // the TMA store that read sA two jobs ago must have finished reading
      asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
      if (i + 2 < n) {  // prefetch the code region two jobs ahead into L2
        const PJob jn = pjob(j0 + i + 2, H, T);
        const ItemCtx cn = item_ctx(L, jn.tile);
        const int nrows = min(kTileRows, cn.rows - cn.row0);
        const uint32_t bytes = static_cast<uint32_t>(nrows * 16 * seg_bits(cn, jn.plane, jn.h));
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(
                         code_row(L, cn, jn.plane, jn.h, cn.row0)),
                     "r"(bytes)
                     : "memory");
      }
    }
    __syncthreads();  // key meta visible; sA free
    // Unpack: 4 groups of 32 codes per row, 2 groups per thread.
    const int bits = seg_bits(c, jb.plane, jb.h);
    const int nrows = min(kTileRows, c.rows - c.row0);
    const uint8_t* src0 = code_row(L, c, jb.plane, jb.h, c.row0);
    const __half* meta = meta_base(L, c.r);
    const int Hh = c.lp->H, G = c.lp->n_groups, grp = c.lp->group_of_head[jb.h];
    for (int g = tid; g < kTileRows * 4; g += kPThreads) {
      // lanes of a warp share `part` (broadcast key-parameter loads) and
      // take consecutive rows (conflict-free swizzled stores)
      const int t = g & (kTileRows - 1), part = g >> 7;
      const int row = c.row0 + t;
      if (t < nrows && row < c.ntok) {
        float vmn = 0.f, vsc = 0.f;
        if (jb.plane == 1) {
          vmn = bf16_round(__half2float(meta[2 * Hh * 128 + grp * c.rows + row]));
          vsc = bf16_round(__half2float(meta[2 * Hh * 128 + G * c.rows + grp * c.rows + row]));
        }
        const uint8_t* src = src0 + static_cast<long long>(t) * 16 * bits + part * 4 * bits;
        switch (bits) {
          case 1: p_unpack_group<1>(src, t, part, jb.plane, kp, vmn, vsc, sA); break;
          case 2: p_unpack_group<2>(src, t, part, jb.plane, kp, vmn, vsc, sA); break;
          case 3: p_unpack_group<3>(src, t, part, jb.plane, kp, vmn, vsc, sA); break;
          case 4: p_unpack_group<4>(src, t, part, jb.plane, kp, vmn, vsc, sA); break;
          case 5: p_unpack_group<5>(src, t, part, jb.plane, kp, vmn, vsc, sA); break;
          case 6: p_unpack_group<6>(src, t, part, jb.plane, kp, vmn, vsc, sA); break;
          case 7: p_unpack_group<7>(src, t, part, jb.plane, kp, vmn, vsc, sA); break;
          default: p_unpack_group<8>(src, t, part, jb.plane, kp, vmn, vsc, sA); break;
        }
      } else {
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8)
          *reinterpret_cast<uint4*>(sA + sw128_offset(t, part * 32 + c8 * 8)) =
              make_uint4(0, 0, 0, 0);
      }
    }
    fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) {
      bool ok = true;
      if (img_key != cur_img) {
        mbar_arrive_expect_tx(S.imgb, 32768u);
        bulk_load(S.img, bmat_of(L, c.slot, jb.h), 32768, S.imgb);
        ok = mbar_wait(S.imgb, img_phase, L.err, ERR_MBAR_TIMEOUT);
        img_phase ^= 1u;
      }
      if (ok) {
        tc_fence_after();
        // D[t][k] = sum_n Y[t][n] Bi[k][n]
        umma_tile_128x128x128(tmem, smem_u32(sA), smem_u32(S.img));
      }
      umma_commit(&S.mma[0]);
      if (!ok) *S.abort_flag = 1;
    }
    cur_img = img_key;
    mbar_wait(&S.mma[0], static_cast<uint32_t>(i & 1), L.err, ERR_MBAR_TIMEOUT);
    tc_fence_after();
    // Epilogue: this thread's row half -> bf16 -> swizzled sA (consumed by the MMA).
    const uint32_t taddr = tmem + (static_cast<uint32_t>(quad * 32) << 16) + half * 64;
    const float sc = c.lp->out_scale;
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      float v[32];
      tmem_ld32(taddr + cc * 32, v);
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        uint32_t w[4];
#pragma unroll
        for (int p = 0; p < 4; ++p)
          w[p] = cvt_bf16x2(v[8 * q4 + 2 * p] * sc, v[8 * q4 + 2 * p + 1] * sc);
        *reinterpret_cast<uint4*>(sA + sw128_offset(lane_id, half * 64 + cc * 32 + q4 * 8)) =
            make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (*S.abort_flag) break;
    if (tid == 0) {
      const CUtensorMap* map = map_of(L, c.slot, jb.plane);
      const int nst = min(kTileRows, c.ntok - c.row0);  // rows holding tokens
      for (int g = 0; g < 8; ++g) {
        const int rr = c.row0 + g * 16;
        if (g * 16 >= nst) break;
        const int phys = phys_block(L, c, rr);
        if (phys < 0) continue;  // bad block id: recorded, box skipped
        const int slot = rr % c.kv.block_size;
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {
          asm volatile(
              "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%1, %2, %3, %4}], [%5];" ::
                  "l"(reinterpret_cast<uint64_t>(map)),
              "r"(hb * 64), "r"(tma_y(c.kv, jb.h, slot)), "r"(tma_z(c.kv, jb.h, slot)), "r"(phys),
              "r"(smem_u32(sA + hb * 16384 + g * 2048))
              : "memory");
        }
      }
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
  }
  if (tid == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 128);
}


// ------------------------------------------------------- dequant (ws)
// Warp-specialized dequantize + inverse transform + paged store.  Warps
// 0-7 unpack codes into one of two A tiles, warp 16 issues the MMAs into one
// of two TMEM accumulators, warps 8-15 convert the accumulator to bf16 into
// one of two output tiles and issue the TMA stores.  Unpack of job k+1, the
// MMA of job k and the epilogue and store of job k-1 overlap.  Barriers
// (job k uses buffers b = k & 1, use index u = k >> 1):
//   afull[b]   8 unpack-warp arrivals: A tile b holds job k;
//   afree[b]   tcgen05.commit after MMA k: A tile b and the image are free;
//   dmma[b]    tcgen05.commit after MMA k: accumulator b holds job k;
//   accfree[b] 8 epilogue-warp arrivals: accumulator b has been read.
// Code tiles rotate through kDqCodeBufs buffers (job k: buffer k % 3), so a
// tile's bulk load is issued two unpack periods before it is needed:
//   cfull[c]   the code tile (and value rows) of job k landed in buffer c;
//   cfree[c]   8 unpack-warp arrivals: job k's unpack finished reading it.
// image | A tiles [2] | output tiles [2] | code tiles [3] (128 rows x 128 B
// at most) | value (min, scale) rows [3] | barriers | key parameters
constexpr int kDqCodeBufs = 3;
constexpr int kDqOffA = 32768;
constexpr int kDqOffO = kDqOffA + 2 * 32768;
constexpr int kDqOffC = kDqOffO + 2 * 32768;
constexpr int kDqOffVm = kDqOffC + kDqCodeBufs * 16384;
constexpr int kDqOffBars = kDqOffVm + kDqCodeBufs * 512;
constexpr int kDqOffKp = kDqOffBars + 256;
constexpr int kDqSmem = kDqOffKp + 64 * 16 + 1024;
static_assert(kDqSmem <= 227 * 1024, "dequant ws shared memory");

__global__ void __launch_bounds__(kWsThreads, 1) k_dequant_ws(LayerLaunch L) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = align1024(smem_raw);
  uint8_t* img = base;
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + kDqOffBars);
  uint64_t* afull = bars;        // [2]
  uint64_t* afree = bars + 2;    // [2]
  uint64_t* dmma = bars + 4;     // [2]
  uint64_t* accfree = bars + 6;  // [2]
  uint64_t* imgb = bars + 8;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 9);
  uint64_t* cfull = bars + 10;   // [kDqCodeBufs] code tile (and value rows) landed
  uint64_t* cfree = bars + 10 + kDqCodeBufs;  // [kDqCodeBufs] unpack finished reading them
  float4* kp = reinterpret_cast<float4*>(base + kDqOffKp);  // [64] key pairs, at kp_pos
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int H = L.num_heads;
  const WsMap M = ws_map(L);
  const int n = M.n;
  if (n <= 0) return;
  if (tid == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&afull[b], kWsGroupWarps);
      mbar_init(&afree[b], 1);
      mbar_init(&dmma[b], 1);
      mbar_init(&accfree[b], kWsGroupWarps);
    }
    for (int c = 0; c < kDqCodeBufs; ++c) {
      mbar_init(&cfull[c], 1);
      mbar_init(&cfree[c], kWsGroupWarps);
    }
    mbar_init(imgb, 1);
    fence_mbar_init();
  }
  if (warp == kWsCtrlWarp) tmem_alloc(tslot, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  auto abuf = [&](int b) { return base + kDqOffA + 32768 * b; };
  auto obuf = [&](int b) { return base + kDqOffO + 32768 * b; };
  auto cbuf = [&](int b) { return base + kDqOffC + 16384 * b; };
  auto vmbuf = [&](int b) { return reinterpret_cast<__half*>(base + kDqOffVm + 512 * b); };

  if (warp < kWsGroupWarps) {
    // ------------------------------------------------------------ unpack
    ItemCursor cur;
    cursor_init(cur);
    int kp_key = -1;
    for (int k = 0; k < n; ++k) {
      const int b = k & 1;
      const PJob jb = ws_job(M, k);
      cursor_seek(L, cur, jb.tile);
      const ItemCtx& c = cur.c;
      if (k >= 2)  // MMA k-2 finished reading A tile b
        mbar_wait(&afree[b], static_cast<uint32_t>(((k >> 1) - 1) & 1), L.err, ERR_MBAR_TIMEOUT);
      group_sync(0);  // every unpack thread finished job k-1 (kp may change)
      if (tid == 0) trace_mark(L, k, 0);
      const int pk = c.r * H + jb.h;
      if (jb.plane == 0 && pk != kp_key) {
        if (tid < 128) {
          const __half* m = meta_base(L, c.r);
          const float mn = bf16_round(__half2float(m[jb.h * 128 + tid]));
          const float sc = bf16_round(__half2float(m[c.lp->H * 128 + jb.h * 128 + tid]));
          float* e = reinterpret_cast<float*>(kp + kp_pos(tid >> 1));
          e[tid & 1] = sc;
          reinterpret_cast<uint16_t*>(e + 2)[tid & 1] =
              static_cast<uint16_t>(__float_as_uint(mn) >> 16);  // mn is a bf16 value
        }
        kp_key = pk;
        group_sync(0);  // key parameters visible
      }
      uint8_t* sA = abuf(b);
      const int bits = seg_bits(c, jb.plane, jb.h);
      const int nrows = min(kTileRows, c.rows - c.row0);
      const int cb = k % kDqCodeBufs;
      const uint8_t* src0 = cbuf(cb);
      const __half* vm = vmbuf(cb);  // [0, 128): group min of the tile's rows, [128, 256): scale
      mbar_wait(&cfull[cb], static_cast<uint32_t>((k / kDqCodeBufs) & 1), L.err, ERR_MBAR_TIMEOUT);
      if (tid == 0) trace_mark(L, k, 6);
      for (int g = tid; g < kTileRows * 4; g += kWsGroupThreads) {
        const int t = g >> 2, part = g & 3;  // a warp: 8 rows x 4 parts
        const int m = (t & 1) ^ (part >> 1);
        const int row = c.row0 + t;
        if (t < nrows && row < c.ntok) {
          float vmn = 0.f, vsc = 0.f;
          if (jb.plane == 1) {
            vmn = bf16_round(__half2float(vm[t]));
            vsc = bf16_round(__half2float(vm[128 + t]));
          }
          const uint8_t* src = src0 + t * 16 * bits + part * 4 * bits;
          switch (bits) {
            case 1: ws_unpack_group<1>(src, t, part, m, jb.plane, kp, vmn, vsc, sA); break;
            case 2: ws_unpack_group<2>(src, t, part, m, jb.plane, kp, vmn, vsc, sA); break;
            case 3: ws_unpack_group<3>(src, t, part, m, jb.plane, kp, vmn, vsc, sA); break;
            case 4: ws_unpack_group<4>(src, t, part, m, jb.plane, kp, vmn, vsc, sA); break;
            case 5: ws_unpack_group<5>(src, t, part, m, jb.plane, kp, vmn, vsc, sA); break;
            case 6: ws_unpack_group<6>(src, t, part, m, jb.plane, kp, vmn, vsc, sA); break;
            case 7: ws_unpack_group<7>(src, t, part, m, jb.plane, kp, vmn, vsc, sA); break;
            default: ws_unpack_group<8>(src, t, part, m, jb.plane, kp, vmn, vsc, sA); break;
          }
        } else {
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8)
            *reinterpret_cast<uint4*>(sA + sw128_offset(t, part * 32 + c8 * 8)) =
                make_uint4(0, 0, 0, 0);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&cfree[cb]);  // code tile cb may be refilled
      fence_proxy_async_smem();  // generic writes of A tile b before the MMA reads it
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[b]);
      if (tid == 0) trace_mark(L, k, 1);
    }
  } else if (warp < kWsCtrlWarp) {
    // ---------------------------------------------------------- epilogue
    const int ew = warp - kWsGroupWarps;
    const int quad = ew & 3, half = ew >> 2;
    const int lane_id = quad * 32 + lane;
    ItemCursor cur;
    cursor_init(cur);
    for (int k = 0; k < n; ++k) {
      const int b = k & 1;
      const PJob jb = ws_job(M, k);
      cursor_seek(L, cur, jb.tile);
      const ItemCtx& c = cur.c;
      // lane l < 16 of warp 0 stores box (row group l/2, channel half l%2);
      // its block-table entry is read now so the load overlaps the epilogue
      const int nst = min(kTileRows, c.ntok - c.row0);  // rows holding tokens
      const int sg = lane >> 1, shb = lane & 1;
      const int srow = c.row0 + sg * 16;
      const bool sbox = ew == 0 && lane < 16 && sg * 16 < nst;
      const int sphys = sbox ? raw_block(L, c, srow) : 0;
      if (ew == 0)  // the stores that read output tile b (job k-2) have finished reading
        asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
      group_sync(1);
      mbar_wait(&dmma[b], static_cast<uint32_t>((k >> 1) & 1), L.err, ERR_MBAR_TIMEOUT);
      if (ew == 0 && lane == 0) trace_mark(L, k, 3);
      tc_fence_after();
      uint8_t* sO = obuf(b);
      const uint32_t taddr = tmem + static_cast<uint32_t>(b * 128) +
                             (static_cast<uint32_t>(quad * 32) << 16) + half * 64;
      const float sc = c.lp->out_scale;
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        float v[32];
        tmem_ld32(taddr + cc * 32, v);
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          uint32_t w[4];
#pragma unroll
          for (int p = 0; p < 4; ++p)
            w[p] = cvt_bf16x2(v[8 * q4 + 2 * p] * sc, v[8 * q4 + 2 * p + 1] * sc);
          *reinterpret_cast<uint4*>(sO + sw128_offset(lane_id, half * 64 + cc * 32 + q4 * 8)) =
              make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&accfree[b]);
      fence_proxy_async_smem();  // generic writes of output tile b before the TMA store
      group_sync(1);
      if (ew == 0) {
        // every lane commits its own (possibly empty) bulk group
        if (sbox && static_cast<unsigned>(sphys) >= static_cast<unsigned>(c.kv.num_blocks)) {
          record_error(L.err, ERR_BOUNDS);  // outside the cache: the box is skipped
        } else if (sbox) {
          const CUtensorMap* map = map_of(L, c.slot, jb.plane);
          const int slot = srow % c.kv.block_size;
          asm volatile(
              "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%1, %2, %3, %4}], [%5];" ::
                  "l"(reinterpret_cast<uint64_t>(map)),
              "r"(shb * 64), "r"(tma_y(c.kv, jb.h, slot)), "r"(tma_z(c.kv, jb.h, slot)),
              "r"(sphys), "r"(smem_u32(sO + shb * 16384 + sg * 2048))
              : "memory");
        }
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        if (lane == 0) trace_mark(L, k, 4);
      }
    }
    if (ew == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  } else {
    // ----------------------------------------------------------- control
    ItemCursor cur;
    cursor_init(cur);
    int cur_img = -1;
    uint32_t img_phase = 0;
    bool ok = true;
    auto wait0 = [&](uint64_t* bar, uint32_t parity) -> bool {
      bool r = true;
      if (lane == 0) r = mbar_wait(bar, parity, L.err, ERR_MBAR_TIMEOUT);
      return __shfl_sync(0xFFFFFFFFu, r ? 1 : 0, 0) != 0;
    };
    auto prefetch = [&](int k) {  // the code region of job k into L2
      ItemCursor pc = cur;
      const PJob jn = ws_job(M, k);
      cursor_seek(L, pc, jn.tile);
      const ItemCtx& c = pc.c;
      const int nrows = min(kTileRows, c.rows - c.row0);
      const uint32_t bytes = static_cast<uint32_t>(nrows * 16 * seg_bits(c, jn.plane, jn.h));
      if (lane == 0)
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(
                         code_row(L, c, jn.plane, jn.h, c.row0)),
                     "r"(bytes)
                     : "memory");
    };
    ItemCursor ccur;
    cursor_init(ccur);
    // Code tile of job kk (and, for values, the group min / scale of its
    // rows) into buffer kk % kDqCodeBufs.  After a failed wait only the arrival is
    // made, so the unpack warps never wait past their limit.
    auto issue_codes = [&](int kk) {
      const int cb = kk % kDqCodeBufs;
      const PJob jn = ws_job(M, kk);
      cursor_seek(L, ccur, jn.tile);
      const ItemCtx& c = ccur.c;
      if (lane != 0) return;
      if (!ok) {
        mbar_arrive(&cfull[cb]);
        return;
      }
      const int nrows = min(kTileRows, c.rows - c.row0);
      const uint32_t cbytes = static_cast<uint32_t>(nrows * 16 * seg_bits(c, jn.plane, jn.h));
      const uint32_t vbytes = jn.plane == 1 ? static_cast<uint32_t>(nrows * 2) : 0u;
      mbar_arrive_expect_tx(&cfull[cb], cbytes + 2 * vbytes);
      trace_mark(L, kk, 7);
      bulk_load(cbuf(cb), code_row(L, c, jn.plane, jn.h, c.row0), cbytes, &cfull[cb]);
      if (vbytes) {
        const __half* meta = meta_base(L, c.r) + 2 * c.lp->H * 128;
        const int G = c.lp->n_groups, grp = c.lp->group_of_head[jn.h];
        bulk_load(vmbuf(cb), meta + grp * c.rows + c.row0, vbytes, &cfull[cb]);
        bulk_load(vmbuf(cb) + 128, meta + (G + grp) * c.rows + c.row0, vbytes, &cfull[cb]);
      }
    };
    constexpr int kPrefetchAhead = 6;  // jobs whose code regions are pulled into L2
    for (int k = 0; k < kPrefetchAhead && k < n; ++k) prefetch(k);
    for (int k = 0; k < kDqCodeBufs && k < n; ++k) issue_codes(k);
    for (int k = 0; k < n; ++k) {
      const int b = k & 1;
      const PJob jb = ws_job(M, k);
      cursor_seek(L, cur, jb.tile);
      if (k + kPrefetchAhead < n) prefetch(k + kPrefetchAhead);
      const int img_key = cur.c.slot * H + jb.h;
      if (ok && img_key != cur_img) {
        if (k >= 1)  // MMA k-1 finished reading the old image
          ok = wait0(&afree[(k - 1) & 1], static_cast<uint32_t>(((k - 1) >> 1) & 1));
        if (ok) {
          if (lane == 0) {
            mbar_arrive_expect_tx(imgb, 32768u);
            bulk_load(img, bmat_of(L, cur.c.slot, jb.h), 32768, imgb);
          }
          ok = wait0(imgb, img_phase);
          img_phase ^= 1u;
        }
        cur_img = img_key;
      }
      if (ok) ok = wait0(&afull[b], static_cast<uint32_t>((k >> 1) & 1));
      if (lane == 0) trace_mark(L, k, 5);
      if (ok && k >= 2) ok = wait0(&accfree[b], static_cast<uint32_t>(((k >> 1) - 1) & 1));
      if (lane == 0) {
        if (ok) {
          tc_fence_after();
          // D[t][k] = sum_n Y[t][n] Bi[k][n]
          umma_tile_128x128x128(tmem + static_cast<uint32_t>(b * 128), smem_u32(abuf(b)),
                                smem_u32(img));
        }
        umma_commit(&dmma[b]);
        umma_commit(&afree[b]);
        trace_mark(L, k, 2);
      }
      __syncwarp();
      if (k + kDqCodeBufs < n) {  // job k's unpack has read its code buffer: refill it
        if (ok)
          ok = wait0(&cfree[k % kDqCodeBufs], static_cast<uint32_t>((k / kDqCodeBufs) & 1));
        issue_codes(k + kDqCodeBufs);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kWsCtrlWarp) tmem_dealloc(tmem, 256);
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

// Persistent grid: two CTAs per SM (the shared-memory limit), never more
// CTAs than jobs.
static int persistent_grid(const LayerLaunch& L) {
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    sms = 148;
  const long long jobs = 2LL * L.num_heads * L.total_tiles;
  return static_cast<int>(jobs < 2LL * sms ? jobs : 2LL * sms);  // jobs < 2^31: checked by the caller
}

// Warp-specialized grid: 2*H*R CTAs (at most one per SM), R tile ranges
// of at least one tile each.
static int ws_grid(const LayerLaunch& L) {
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    sms = 148;
  const int PH = 2 * L.num_heads;
  int R = sms / PH;
  if (R < 1) R = 1;
  if (R > L.total_tiles) R = L.total_tiles;
  return PH * R;
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
// memory, 128 bytes each): 4-D (d=128, head, slot, block) with box
// (64,1,16,1) for NHD blocks, (d, slot, head, block) with box (64,16,1,1) for
// HND blocks; 128-byte swizzle, no OOB fill.
int kvs_make_plane_maps(const PagedKV* kv, int H, void* out) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return -100;
  CUtensorMap* maps = static_cast<CUtensorMap*>(out);
  for (int plane = 0; plane < 2; ++plane) {
    void* base = const_cast<void*>(reinterpret_cast<const void*>(
        reinterpret_cast<const __nv_bfloat16*>(kv->base) + plane * kv->kv_stride));
    // (d, head, slot, block) for NHD, (d, slot, head, block) for HND: the
    // middle dimensions in increasing stride order
    const cuuint64_t hd = static_cast<cuuint64_t>(H), sl = static_cast<cuuint64_t>(kv->block_size);
    cuuint64_t dims[4] = {128, kv->hnd ? sl : hd, kv->hnd ? hd : sl,
                          static_cast<cuuint64_t>(kv->num_blocks)};
    const cuuint64_t hs = static_cast<cuuint64_t>(kv->head_stride) * 2;
    const cuuint64_t ss = static_cast<cuuint64_t>(kv->slot_stride) * 2;
    cuuint64_t strides[3] = {kv->hnd ? ss : hs, kv->hnd ? hs : ss,
                             static_cast<cuuint64_t>(kv->block_stride) * 2};
    cuuint32_t box[4] = {64, kv->hnd ? 16u : 1u, kv->hnd ? 1u : 16u, 1};
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
  if (2LL * L.num_heads * L.total_tiles >= (1LL << 31)) return -103;  // job index is 32-bit
  cudaStream_t s = static_cast<cudaStream_t>(L.stream);
  dim3 grid(L.total_tiles, L.num_heads, 2);
  if (L.engine == 0) {
    if (int rc = set_smem(k_stats_ws, WsStatsLayout::kSmem)) return rc;
    k_stats_ws<<<ws_grid(L), kWsStatsThreads, WsStatsLayout::kSmem, s>>>(L);
  } else if (L.engine == 3) {
    if (int rc = set_smem(k_stats_tc, kPSmem)) return rc;
    k_stats_tc<<<persistent_grid(L), kPThreads, kPSmem, s>>>(L);
  } else if (L.engine == 2) {
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
  if (2LL * L.num_heads * L.total_tiles >= (1LL << 31)) return -103;  // job index is 32-bit
  if (L.ck != nullptr && L.engine != 0) return -2;  // the code-store checksum is engine 0's
  cudaStream_t s = static_cast<cudaStream_t>(L.stream);
  dim3 grid(L.total_tiles, L.num_heads, 2);
  if (L.engine == 0) {
    if (int rc = set_smem(k_quant_ws, WsQuantLayout::kSmem)) return rc;
    k_quant_ws<<<ws_grid(L), kWsProdThreads, WsQuantLayout::kSmem, s>>>(L);
  } else if (L.engine == 3) {
    if (int rc = set_smem(k_quant_tc, kPSmem)) return rc;
    k_quant_tc<<<persistent_grid(L), kPThreads, kPSmem, s>>>(L);
  } else if (L.engine == 2) {
    if (int rc = set_smem(k_quant_mma, kSmemTile)) return rc;
    k_quant_mma<<<grid, 128, kSmemTile, s>>>(L);
  } else {
    k_quant_simt<<<grid, 128, 0, s>>>(L);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// Value parameters for the warp-specialized quantize kernel (engine 0),
// after the stats kernel; max_rows = the largest item's row count.
int kvs_value_params(const LayerLaunch* Lp, int max_rows) {
  const LayerLaunch& L = *Lp;
  if (L.rt.num_req <= 0 || max_rows <= 0) return 0;
  if (L.vparam == nullptr) return -2;
  dim3 grid((max_rows + 255) / 256, L.rt.num_req);
  k_value_params<<<grid, 256, 0, static_cast<cudaStream_t>(L.stream)>>>(L);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int kvs_dequant_inverse(const LayerLaunch* Lp) {
  const LayerLaunch& L = *Lp;
  if (L.total_tiles <= 0) return 0;
  if (2LL * L.num_heads * L.total_tiles >= (1LL << 31)) return -103;  // job index is 32-bit
  cudaStream_t s = static_cast<cudaStream_t>(L.stream);
  dim3 grid(L.total_tiles, L.num_heads, 2);
  // k_dequant_ws bulk-copies code tiles and metadata rows: their bases must
  // be 16-byte aligned (item offsets are); otherwise the persistent kernel runs
  const bool aligned = ((reinterpret_cast<uintptr_t>(L.codes) |
                         reinterpret_cast<uintptr_t>(L.meta)) & 15) == 0;
  if (L.engine == 0 && aligned) {
    if (int rc = set_smem(k_dequant_ws, kDqSmem)) return rc;
    k_dequant_ws<<<ws_grid(L), kWsThreads, kDqSmem, s>>>(L);
  } else if (L.engine == 3 || L.engine == 0) {
    if (int rc = set_smem(k_dequant_tc, kPSmem)) return rc;
    k_dequant_tc<<<persistent_grid(L), kPThreads, kPSmem, s>>>(L);
  } else if (L.engine == 2) {
    if (int rc = set_smem(k_dequant_inverse_mma, kSmemTile)) return rc;
    k_dequant_inverse_mma<<<grid, 128, kSmemTile, s>>>(L);
  } else {
    k_dequant_inverse_simt<<<grid, 128, 0, s>>>(L);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // extern "C"
