// LC-style lossless codec: BIT_2 then RZE_1, after the LC compression
// framework of Burtscher et al. (component names as in the reference's
// `codec_type: "lc"`, kvserve_v1/compression/codec/lc_codec.py:46-110, which
// calls an external closed library; this is an independent implementation
// of the two published stages with its own stream format).
//
// Per 16 KB chunk of input bytes:
//   BIT_2  the chunk as little-endian 16-bit words (zero padded to a multiple
//          of 32 words) is transposed into 16 bit planes: plane b, group g
//          is the u32 whose bit i is bit b of word 32g+i; planes are stored
//          plane-major ([16][G] u32), so planes that are zero everywhere
//          (the high bits of small codes) become long zero runs;
//   RZE_1  a bitmap of the non-zero bytes of the shuffled chunk (bit j, LSB
//          first, for byte j) followed by those bytes in order.
// A chunk whose record would not be smaller than its input is stored raw.
//
// Stream: [u32 'LCB2'][u32 chunk bytes][u64 n][u32 chunks][u32 0]
//         [(chunks + 1) x u32 record offsets from the records start, padded
//          to 16 B][records];
// record: [u32 kind (1 coded, 0 raw)][u32 non-zero count or raw bytes]
//         [u32 0][u32 0][bitmap | raw bytes][non-zero bytes], padded to 16 B.
//
// Encode = three launches (records into per-chunk staging slots, a
// single-CTA directory scan, a compaction copy); decode = one CTA per chunk.
#include <cstdint>

#include "common.cuh"

namespace kvs {

constexpr uint32_t kLcMagic = 0x3242434Cu;  // "LCB2"
constexpr int kLcChunk = 16384;             // input bytes per chunk
constexpr int kLcThreads = 256;
constexpr int kLcMaxShuffled = kLcChunk;    // 16 planes x 256 groups x 4 B
// staging slot: record header + bitmap + every byte non-zero
constexpr int kLcSlot = 16 + kLcMaxShuffled / 8 + kLcMaxShuffled;

KVS_DEV uint32_t lc_pad16(uint32_t x) { return (x + 15u) & ~15u; }

// Bytes of the shuffled chunk for `cb` input bytes: 16 planes x G u32.
KVS_DEV uint32_t lc_shuffled_bytes(uint32_t cb) {
  const uint32_t words = (cb + 1) / 2;
  const uint32_t groups = (words + 31) / 32;
  return 16u * groups * 4u;
}

// Exclusive block scan of one value per thread (kLcThreads threads).
KVS_DEV uint32_t lc_block_scan(uint32_t v, uint32_t* warp_sums, uint32_t& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    uint32_t s = lane < kLcThreads / 32 ? warp_sums[lane] : 0u;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, s, o);
      if (lane >= o) s += y;
    }
    if (lane < kLcThreads / 32) warp_sums[lane] = s;  // inclusive
  }
  __syncthreads();
  total = warp_sums[kLcThreads / 32 - 1];
  const uint32_t before = warp == 0 ? 0u : warp_sums[warp - 1];
  __syncthreads();  // warp_sums may be reused by the caller
  return before + x - v;
}

// One CTA per chunk: record into the chunk's staging slot, its length into
// rec_len[chunk].
__global__ void __launch_bounds__(kLcThreads) k_lc_encode(const uint8_t* __restrict__ in,
                                                          uint64_t n, uint8_t* __restrict__ staging,
                                                          uint32_t* __restrict__ rec_len) {
  __shared__ __align__(16) uint32_t sh[kLcMaxShuffled / 4];  // shuffled chunk
  __shared__ __align__(16) uint16_t words[kLcChunk / 2];
  __shared__ uint32_t warp_sums[kLcThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t c = blockIdx.x;
  const uint64_t start = static_cast<uint64_t>(c) * kLcChunk;
  const uint32_t cb = static_cast<uint32_t>(min(static_cast<uint64_t>(kLcChunk), n - start));
  const uint8_t* src = in + start;
  const uint32_t nwords = (cb + 1) / 2;
  const uint32_t groups = (nwords + 31) / 32;
  const uint32_t S = 16u * groups * 4u;
  uint8_t* slot = staging + static_cast<uint64_t>(c) * kLcSlot;

  // input bytes -> words (zero padded)
  for (uint32_t w = tid; w < groups * 32; w += kLcThreads) {
    const uint32_t b0 = 2 * w, b1 = 2 * w + 1;
    const uint32_t lo = b0 < cb ? src[b0] : 0u, hi = b1 < cb ? src[b1] : 0u;
    words[w] = static_cast<uint16_t>(lo | (hi << 8));
  }
  __syncthreads();
  // BIT_2: one ballot per (group, plane); lane b keeps plane b's word
  for (uint32_t g = warp; g < groups; g += kLcThreads / 32) {
    const uint32_t w = words[32 * g + lane];
    uint32_t mine = 0;
#pragma unroll
    for (int b = 0; b < 16; ++b) {
      const uint32_t plane = __ballot_sync(0xFFFFFFFFu, (w >> b) & 1u);
      if (lane == b) mine = plane;
    }
    if (lane < 16) sh[lane * groups + g] = mine;
  }
  __syncthreads();
  // RZE_1: thread t owns shuffled bytes [t*per, (t+1)*per), per a multiple of 64
  const uint32_t per = ((S + kLcThreads - 1) / kLcThreads + 63) & ~63u;
  const uint32_t lo = min(S, tid * per), hi = min(S, lo + per);
  const uint8_t* sb = reinterpret_cast<const uint8_t*>(sh);
  uint32_t cnt = 0;
  for (uint32_t j = lo; j < hi; ++j) cnt += sb[j] != 0;
  uint32_t nz = 0;
  const uint32_t off = lc_block_scan(cnt, warp_sums, nz);
  const uint32_t coded = 16u + S / 8 + nz;
  const bool raw = coded >= 16u + lc_pad16(cb);
  if (raw) {
    for (uint32_t j = tid; j < cb; j += kLcThreads) slot[16 + j] = src[j];
    for (uint32_t j = cb + tid; j < lc_pad16(cb); j += kLcThreads) slot[16 + j] = 0;
    if (tid == 0) {
      reinterpret_cast<uint4*>(slot)[0] = make_uint4(0u, cb, 0u, 0u);
      rec_len[c] = 16u + lc_pad16(cb);
    }
    return;
  }
  uint8_t* bitmap = slot + 16;
  uint8_t* vals = slot + 16 + S / 8;
  uint32_t k = off;
  for (uint32_t j0 = lo; j0 < hi; j0 += 8) {  // one bitmap byte per 8 shuffled bytes
    uint32_t bits = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint8_t v = sb[j0 + q];
      if (v != 0) {
        bits |= 1u << q;
        vals[k++] = v;
      }
    }
    bitmap[j0 / 8] = static_cast<uint8_t>(bits);
  }
  const uint32_t len = lc_pad16(coded);
  for (uint32_t j = coded + tid; j < len; j += kLcThreads) slot[j] = 0;
  if (tid == 0) {
    reinterpret_cast<uint4*>(slot)[0] = make_uint4(1u, nz, 0u, 0u);
    rec_len[c] = len;
  }
}

// Single CTA: stream header and exclusive scan of the record lengths.
__global__ void __launch_bounds__(1024) k_lc_directory(const uint32_t* __restrict__ rec_len,
                                                       uint32_t nc, uint64_t n,
                                                       uint8_t* __restrict__ out,
                                                       uint64_t* total_out) {
  __shared__ uint32_t carry;
  __shared__ uint32_t ws[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t* dir = reinterpret_cast<uint32_t*>(out + 24);
  if (tid == 0) {
    uint32_t* h = reinterpret_cast<uint32_t*>(out);
    h[0] = kLcMagic;
    h[1] = kLcChunk;
    *reinterpret_cast<uint64_t*>(out + 8) = n;
    h[4] = nc;
    h[5] = 0;
    carry = 0;
  }
  __syncthreads();
  for (uint32_t base = 0; base < nc; base += 1024) {
    const uint32_t i = base + tid;
    const uint32_t v = i < nc ? rec_len[i] : 0u;
    uint32_t x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) ws[warp] = x;
    __syncthreads();
    if (warp == 0) {
      uint32_t s = ws[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, s, o);
        if (lane >= o) s += y;
      }
      ws[lane] = s;
    }
    __syncthreads();
    const uint32_t excl = carry + (warp ? ws[warp - 1] : 0u) + x - v;
    if (i < nc) dir[i] = excl;
    __syncthreads();
    if (tid == 0) carry += ws[31];
    __syncthreads();
  }
  if (tid == 0) {
    dir[nc] = carry;
    const uint64_t head = lc_pad16(24u + 4u * (nc + 1));
    for (uint64_t p = 24u + 4u * (nc + 1); p < head; ++p) out[p] = 0;
    *total_out = head + carry;
  }
}

// One warp per record: staging slot -> its place in the stream.
__global__ void __launch_bounds__(256) k_lc_copy(const uint8_t* __restrict__ staging,
                                                 const uint32_t* __restrict__ rec_len,
                                                 uint32_t nc, uint8_t* __restrict__ out) {
  const uint32_t c = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (c >= nc) return;
  const uint32_t* dir = reinterpret_cast<const uint32_t*>(out + 24);
  const uint64_t head = lc_pad16(24u + 4u * (nc + 1));
  const uint4* s = reinterpret_cast<const uint4*>(staging + static_cast<uint64_t>(c) * kLcSlot);
  uint4* d = reinterpret_cast<uint4*>(out + head + dir[c]);
  for (uint32_t i = lane; i < rec_len[c] / 16; i += 32) d[i] = s[i];
}

// One CTA per chunk: records -> bytes.
// Every offset read from the stream is checked against its length `len`:
// a corrupt stream records ERR_CORRUPT and its chunk is skipped.
__global__ void __launch_bounds__(kLcThreads) k_lc_decode(const uint8_t* __restrict__ stream,
                                                          uint64_t len, uint64_t n,
                                                          uint8_t* __restrict__ out,
                                                          uint32_t* err) {
  __shared__ __align__(16) uint32_t sh[kLcMaxShuffled / 4];
  __shared__ uint32_t warp_sums[kLcThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t c = blockIdx.x;
  const uint32_t nc = static_cast<uint32_t>((n + kLcChunk - 1) / kLcChunk);
  const uint64_t head = lc_pad16(24u + 4u * (nc + 1));
  const uint32_t* h = reinterpret_cast<const uint32_t*>(stream);
  bool bad = len < head || h[0] != kLcMagic || h[4] != nc ||
             *reinterpret_cast<const uint64_t*>(stream + 8) != n;
  const uint32_t* dir = reinterpret_cast<const uint32_t*>(stream + 24);
  const uint64_t roff = bad ? 0 : head + dir[c];
  const uint64_t rend = bad ? 0 : head + dir[c + 1];
  bad = bad || rend > len || roff + 16 > rend;
  const uint8_t* rec = stream + roff;
  const uint64_t start = static_cast<uint64_t>(c) * kLcChunk;
  const uint32_t cb = static_cast<uint32_t>(min(static_cast<uint64_t>(kLcChunk), n - start));
  const uint32_t nwords = (cb + 1) / 2;
  const uint32_t groups = (nwords + 31) / 32;
  const uint32_t S = 16u * groups * 4u;
  const uint32_t kind = bad ? 2u : reinterpret_cast<const uint32_t*>(rec)[0];
  const uint32_t nz = bad ? 0u : reinterpret_cast<const uint32_t*>(rec)[1];
  bad = bad || kind > 1 || (kind == 0 && roff + 16 + cb > rend) ||
        (kind == 1 && (nz > S || roff + 16 + S / 8 + nz > rend));
  if (bad) {
    if (tid == 0) record_error(err, ERR_CORRUPT);
    return;
  }
  uint8_t* dst = out + start;
  if (kind == 0) {
    for (uint32_t j = tid; j < cb; j += kLcThreads) dst[j] = rec[16 + j];
    return;
  }
  const uint8_t* bitmap = rec + 16;
  const uint8_t* vals = rec + 16 + S / 8;
  const uint32_t per = ((S + kLcThreads - 1) / kLcThreads + 63) & ~63u;
  const uint32_t lo = min(S, tid * per), hi = min(S, lo + per);
  uint32_t cnt = 0;
  for (uint32_t j0 = lo; j0 < hi; j0 += 8) cnt += __popc(bitmap[j0 / 8]);
  uint32_t total = 0;
  uint32_t k = lc_block_scan(cnt, warp_sums, total);
  if (total != nz) {
    if (tid == 0) record_error(err, ERR_CORRUPT);
    return;
  }
  uint8_t* sb = reinterpret_cast<uint8_t*>(sh);
  for (uint32_t j0 = lo; j0 < hi; j0 += 8) {
    const uint32_t bits = bitmap[j0 / 8];
#pragma unroll
    for (int q = 0; q < 8; ++q) sb[j0 + q] = (bits >> q) & 1u ? vals[k++] : 0;
  }
  __syncthreads();
  // inverse BIT_2: lane i rebuilds word 32g+i from the group's 16 plane words
  for (uint32_t g = warp; g < groups; g += kLcThreads / 32) {
    uint32_t w = 0;
#pragma unroll
    for (int b = 0; b < 16; ++b) w |= ((sh[b * groups + g] >> lane) & 1u) << b;
    const uint32_t b0 = 2 * (32 * g + lane);
    if (b0 < cb) dst[b0] = static_cast<uint8_t>(w & 0xFFu);
    if (b0 + 1 < cb) dst[b0 + 1] = static_cast<uint8_t>(w >> 8);
  }
}

}  // namespace kvs

using namespace kvs;

extern "C" {

uint64_t kvs_lc_max_bytes(uint64_t n) {
  const uint64_t nc = (n + kLcChunk - 1) / kLcChunk;
  return ((24 + 4 * (nc + 1) + 15) & ~15ull) + nc * (16 + ((kLcChunk + 15) & ~15ull));
}

uint64_t kvs_lc_staging_bytes(uint64_t n) {
  return ((n + kLcChunk - 1) / kLcChunk) * static_cast<uint64_t>(kLcSlot);
}

// Encode n bytes (n > 0) into `out` (capacity kvs_lc_max_bytes(n)); the
// stream size goes to *total_out (device).  `staging` holds
// kvs_lc_staging_bytes(n) bytes, `rec_len` one u32 per chunk.
int kvs_lc_encode(const uint8_t* in, uint64_t n, uint8_t* staging, uint32_t* rec_len, uint8_t* out,
                  uint64_t* total_out, void* stream) {
  if (n == 0) return -2;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint32_t nc = static_cast<uint32_t>((n + kLcChunk - 1) / kLcChunk);
  k_lc_encode<<<nc, kLcThreads, 0, s>>>(in, n, staging, rec_len);
  k_lc_directory<<<1, 1024, 0, s>>>(rec_len, nc, n, out, total_out);
  k_lc_copy<<<(nc + 7) / 8, 256, 0, s>>>(staging, rec_len, nc, out);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// Decode the stream of `len` bytes into n bytes at `out`.
int kvs_lc_decode(const uint8_t* stream_buf, uint64_t len, uint8_t* out, uint64_t n,
                  uint32_t* err, void* stream) {
  if (n == 0) return -2;
  const uint32_t nc = static_cast<uint32_t>((n + kLcChunk - 1) / kLcChunk);
  k_lc_decode<<<nc, kLcThreads, 0, static_cast<cudaStream_t>(stream)>>>(stream_buf, len, n, out,
                                                                        err);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // extern "C"
