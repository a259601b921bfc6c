// Device encoder / decoder of the interleaved rANS stream (format: rans.cuh).
//
// Encode = three launches on one stream:
//   k_rans_encode    one warp per chunk: histogram, normalisation, reverse
//                    encode of the chunk's two interleaved streams into a
//                    per-chunk staging slot (raw fallback when the coded record
//                    would not be smaller than the input);
//   k_rans_directory one CTA: exclusive scan of record sizes, header + dir;
//   k_rans_copy      one warp per chunk: compacts each record's three pieces
//                    (prefix, word blocks of the two streams) into the output,
//                    which may be a peer GPU's buffer (NVLink stores); the last
//                    CTA can publish a release flag for the consumer.
// Decode = k_rans_decode, one warp per chunk, symbols written in place.
#include "common.cuh"
#include "rans.cuh"

namespace kvs {
namespace rans {

// Occupancy: a chunk is one warp's work, so a launch finishes in one wave
// only if every chunk's warp is resident at once.  Seven 4-warp CTAs per SM
// (28 warps, at most 73 registers a thread and 32 KB of shared memory per
// CTA) keep a 28-layer 8-request step (3585 chunks) in one wave.
constexpr int kEncWarps = 4;
constexpr int kCtasPerSm = 7;
// Histogram copies: lane l counts into copy l % kHistCopies.  A copy holds
// two 16-bit counts per word (symbol s in word s / 2, half s & 1; a copy
// sees at most cs / kHistCopies symbols, below 2^16) and is padded to
// kHistStride words, so the same symbol in different copies falls in
// different banks.
constexpr int kHistCopies = 8;
constexpr int kHistStride = 129;  // 128 words + 1 (129 mod 32 = 1)
constexpr int kDecWarps = 4;
constexpr int kRing = 512;  // words of one stream's shared-memory ring in the decoder
constexpr int kDecWarpSmem = 4096 + 1024 + kStreams * kRing * 2;
static_assert(kDecWarps * kDecWarpSmem <= 32 * 1024, "decoder shared memory per CTA");

// Encoder table entry packed into 8 bytes (one 64-bit shared-memory load a
// step): the reciprocal, and bias (13 bits) | f - 1 (12 bits) | shift (4 bits)
// of the EncSym it stands for (rans.cuh: make_enc).
struct EncPacked {
  uint32_t rcp;
  uint32_t w;
};
KVS_DEV EncPacked pack_enc(const EncSym& e) {
  const uint32_t f = kProbScale - (e.cmpl_shift & 0xFFFFu);
  return EncPacked{e.rcp, e.bias | ((f - 1) << 13) | ((e.cmpl_shift >> 16) << 25)};
}

// Where an encoded stream goes inside a transfer message (all optional).
struct RansMsg {
  uint32_t prefix[4];           // 16-byte container header stored just before the stream
  int has_prefix;
  int pad_;
  long long msg_off;            // message offset of the stream's first byte (multiple of 16)
  unsigned long long* ck;       // message checksum accumulators (zeroed by the caller)
  unsigned long long* trailer;  // receives the finished checksum (may be peer memory)
  uint32_t* counter;            // completion counter (zero) for the flag publish
  uint32_t* flag;               // ready flag (may be peer memory)
  uint32_t flag_value;
  int pad2_;
};

KVS_DEV uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// The 32 symbols of lane `lane` in super-step `ss` (zero padded past n_sym),
// as two 16-byte words.
struct Syms32 {
  uint4 lo, hi;
};
KVS_DEV Syms32 load_syms(const uint8_t* src, uint32_t ss, int lane, uint32_t n_sym) {
  const uint32_t off = ss * kSuper + lane * kSub;
  Syms32 r;
  if (off + kSub <= n_sym) {
    r.lo = *reinterpret_cast<const uint4*>(src + off);
    r.hi = *reinterpret_cast<const uint4*>(src + off + 16);
    return r;
  }
  uint32_t w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (uint32_t i = 0; i < kSub; ++i)
    if (off + i < n_sym) w[i >> 2] |= static_cast<uint32_t>(src[off + i]) << ((i & 3) * 8);
  r.lo = make_uint4(w[0], w[1], w[2], w[3]);
  r.hi = make_uint4(w[4], w[5], w[6], w[7]);
  return r;
}

KVS_DEV void syms_words(const Syms32& v, uint32_t (&w)[8]) {
  w[0] = v.lo.x; w[1] = v.lo.y; w[2] = v.lo.z; w[3] = v.lo.w;
  w[4] = v.hi.x; w[5] = v.hi.y; w[6] = v.hi.z; w[7] = v.hi.w;
}


// Warp-parallel form of normalize_counts (rans.cuh) with identical integer
// results: lanes compute the scaled frequencies of symbols lane, lane+32,
// ...; the sum and the first symbol with the largest count are reduced
// across the warp; lane 0 applies the (rare, short) correction loop.
KVS_DEV void normalize_counts_warp(const uint32_t* cnt, uint32_t A, uint64_t total, uint32_t* freq,
                                   int lane) {
  uint32_t sum = 0, best = 0xFFFFFFFFu, best_cnt = 0;
  for (uint32_t s = lane; s < A; s += 32) {
    uint32_t f = 0;
    const uint32_t c = cnt[s];
    if (c > 0) {
      f = static_cast<uint32_t>((static_cast<uint64_t>(c) * kProbScale) / total);
      if (f < 1) f = 1;
      if (c > best_cnt) {
        best_cnt = c;
        best = s;
      }
    }
    freq[s] = f;
    sum += f;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
    const uint32_t oc = __shfl_xor_sync(0xFFFFFFFFu, best_cnt, o);
    const uint32_t ob = __shfl_xor_sync(0xFFFFFFFFu, best, o);
    if (oc > best_cnt || (oc == best_cnt && ob < best)) {
      best_cnt = oc;
      best = ob;
    }
  }
  __syncwarp();
  if (lane == 0) {
    int64_t diff = static_cast<int64_t>(kProbScale) - static_cast<int64_t>(sum);
    while (diff != 0) {
      if (diff > 0) {
        freq[best] += static_cast<uint32_t>(diff);
        diff = 0;
      } else {
        uint32_t s_max = 0, f_max = 0;
        for (uint32_t s = 0; s < A; ++s)
          if (freq[s] > f_max) {
            f_max = freq[s];
            s_max = s;
          }
        int64_t take = -diff;
        if (take > static_cast<int64_t>(f_max) - 1) take = static_cast<int64_t>(f_max) - 1;
        freq[s_max] -= static_cast<uint32_t>(take);
        diff += take;
      }
    }
  }
  __syncwarp();
}

// Encoder table from frequencies: lane l owns the contiguous symbols
// [l*per, (l+1)*per); cumulative frequencies come from a warp scan.
KVS_DEV void build_enc_warp(const uint32_t* freq, uint32_t A, EncPacked* enc, int lane) {
  const uint32_t per = (A + 31) / 32;
  const uint32_t b = lane * per, e = min(A, b + per);
  uint32_t local = 0;
  for (uint32_t s = b; s < e; ++s) local += freq[s];
  uint32_t incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t v = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += v;
  }
  uint32_t cum = incl - local;
  for (uint32_t s = b; s < e; ++s) {
    const uint32_t f = freq[s];
    if (f > 0) enc[s] = pack_enc(make_enc(f, cum));
    cum += f;
  }
  __syncwarp();
}

// One warp per chunk.  desc[chunk * kDescWords + k] receives: the record
// length, the prefix length (header + frequencies + states, or the whole raw
// record), the byte length of each stream's word block and the staging
// offset of each word block (see rans.cuh).
__global__ void __launch_bounds__(kEncWarps * 32, kCtasPerSm) k_rans_encode(
    const uint8_t* __restrict__ in, uint64_t n, uint32_t cs, uint8_t* __restrict__ staging,
    uint32_t* __restrict__ desc, uint32_t n_chunks) {
  // a warp's histogram (4 x 256 counts) is dead once its frequencies are
  // normalised, so its encoder table (256 x 8 B) reuses its first 2 KB
  __shared__ __align__(16) uint32_t hist[kEncWarps][kHistCopies * kHistStride + 4];
  __shared__ uint32_t freq_s[kEncWarps][256];
  static_assert(sizeof(EncPacked) * 256 <= sizeof(uint32_t) * kHistCopies * kHistStride,
                "table aliasing");
  static_assert(kMaxChunkSyms / kHistCopies < 65536, "16-bit histogram counts");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t chunk = blockIdx.x * kEncWarps + warp;
  if (chunk >= n_chunks) return;  // warp-uniform
  const uint64_t start = static_cast<uint64_t>(chunk) * cs;
  const uint32_t n_sym = static_cast<uint32_t>(min(static_cast<uint64_t>(cs), n - start));
  const uint32_t n_ss = (n_sym + kSuper - 1) / kSuper;
  const uint8_t* src = in + start;
  uint8_t* slot = staging + static_cast<uint64_t>(chunk) * slot_bytes(cs);
  uint32_t* d = desc + static_cast<uint64_t>(chunk) * kDescWords;

  uint32_t* h = hist[warp];
  for (int i = lane; i < kHistCopies * kHistStride; i += 32) h[i] = 0;
  __syncwarp();
  // Histogram in lane-interleaved copies: spreads the atomic traffic of
  // skewed symbol distributions over kHistCopies addresses in distinct banks.
  uint32_t* hc = h + (lane & (kHistCopies - 1)) * kHistStride;
  // the next super-step's symbols are loaded while this one is counted
  Syms32 nxt = load_syms(src, 0, lane, n_sym);
  for (uint32_t ss = 0; ss < n_ss; ++ss) {
    uint32_t w[8];
    syms_words(nxt, w);
    if (ss + 1 < n_ss) nxt = load_syms(src, ss + 1, lane, n_sym);
#pragma unroll
    for (int i = 0; i < kSub; ++i) {
      const uint32_t sym = (w[i >> 2] >> ((i & 3) * 8)) & 0xFFu;
      atomicAdd(&hc[sym >> 1], 1u << ((sym & 1u) * 16));
    }
  }
  __syncwarp();
  int top = -1;
  uint32_t tot[8];  // this lane's symbols lane*8 .. lane*8+7 (words lane*4 .. lane*4+3)
#pragma unroll
  for (int k = 0; k < 8; k += 2) {
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int cp = 0; cp < kHistCopies; ++cp) {
      const uint32_t v = h[cp * kHistStride + lane * 4 + (k >> 1)];
      lo += v & 0xFFFFu;
      hi += v >> 16;
    }
    tot[k] = lo;
    tot[k + 1] = hi;
  }
  __syncwarp();  // every lane read its words before the totals overwrite them
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    h[lane * 8 + k] = tot[k];  // words 0..255 now hold the 32-bit totals
    if (tot[k] > 0) top = lane * 8 + k;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) top = max(top, __shfl_xor_sync(0xFFFFFFFFu, top, o));
  const uint32_t A = static_cast<uint32_t>(top + 1);
  __syncwarp();
  normalize_counts_warp(h, A, static_cast<uint64_t>(n_ss) * kSuper, freq_s[warp], lane);
  EncPacked* enc = reinterpret_cast<EncPacked*>(hist[warp]);
  build_enc_warp(freq_s[warp], A, enc, lane);

  // Words of stream k grow backwards from the end of region k.
  const int cap = static_cast<int>(region_bytes(cs) / 2);
  uint16_t* words0 = reinterpret_cast<uint16_t*>(slot + kPrefixArea);
  uint16_t* words1 = reinterpret_cast<uint16_t*>(slot + kPrefixArea + region_bytes(cs));
  const uint64_t prefix = coded_prefix_bytes(A);
  const uint64_t raw_len = raw_record_bytes(n_sym);
  int wpos0 = cap, wpos1 = cap;
  uint32_t x0 = kStateLow, x1 = kStateLow;
  bool overflow = false;
  const uint32_t lt = lanemask_lt();
  Syms32 pre = load_syms(src, n_ss - 1, lane, n_sym);  // prefetched one super-step ahead
  for (int ss = static_cast<int>(n_ss) - 1; ss >= 0; --ss) {
    // a super-step emits at most one word per symbol; stop (raw record) as
    // soon as the coded record could reach the raw one's size (two blocks of
    // padding included)
    const int used = (cap - wpos0) + (cap - wpos1);
    if (prefix + 2ull * static_cast<uint64_t>(used + kSuper + 16) >= raw_len) {
      overflow = true;
      break;
    }
    uint32_t w[8];
    syms_words(pre, w);
    if (ss > 0) pre = load_syms(src, ss - 1, lane, n_sym);
    // sub-steps in decreasing order; even ones update stream 0, odd ones
    // stream 1, so consecutive steps are independent chains
#pragma unroll
    for (int m = kSub - 1; m >= 0; --m) {
      const uint32_t s = (w[m >> 2] >> ((m & 3) * 8)) & 0xFFu;
      const EncPacked e = enc[s];
      const uint32_t f = ((e.w >> 13) & 0xFFFu) + 1;
      uint32_t& x = (m & 1) ? x1 : x0;
      int& wpos = (m & 1) ? wpos1 : wpos0;
      uint16_t* words = (m & 1) ? words1 : words0;
      const bool emit = x >= (f << kXmaxShift);
      const uint32_t mask = __ballot_sync(0xFFFFFFFFu, emit);
      const int cnt = __popc(mask);
      if (emit) {
        words[wpos - cnt + __popc(mask & lt)] = static_cast<uint16_t>(x & 0xFFFFu);
        x >>= 16;
      }
      wpos -= cnt;
      const uint32_t q = __umulhi(x, e.rcp) >> (e.w >> 25);
      x = x + (e.w & 0x1FFFu) + q * (kProbScale - f);
    }
  }
  if (!overflow) {
    const int nw0 = cap - wpos0, nw1 = cap - wpos1;
    const int np0 = (8 - (nw0 & 7)) & 7, np1 = (8 - (nw1 & 7)) & 7;
    if (lane < np0) words0[wpos0 - np0 + lane] = 0;
    if (lane < np1) words1[wpos1 - np1 + lane] = 0;
    const uint32_t fpad = static_cast<uint32_t>(pad16(2ull * A));
    if (lane == 0) {
      // ChunkHeader {n_sym, A, n_words[2], n_pad[2], 0, 0} as two 16-byte stores
      reinterpret_cast<uint4*>(slot)[0] =
          make_uint4(n_sym, A, static_cast<uint32_t>(nw0), static_cast<uint32_t>(nw1));
      reinterpret_cast<uint4*>(slot)[1] =
          make_uint4(static_cast<uint32_t>(np0), static_cast<uint32_t>(np1), 0u, 0u);
      const uint32_t len0 = static_cast<uint32_t>(2 * (nw0 + np0));
      const uint32_t len1 = static_cast<uint32_t>(2 * (nw1 + np1));
      d[0] = static_cast<uint32_t>(prefix) + len0 + len1;
      d[1] = static_cast<uint32_t>(prefix);
      d[2] = len0;
      d[3] = len1;
      d[4] = static_cast<uint32_t>(kPrefixArea + 2 * (wpos0 - np0));
      d[5] = static_cast<uint32_t>(kPrefixArea + region_bytes(cs) + 2 * (wpos1 - np1));
    }
    uint16_t* fr = reinterpret_cast<uint16_t*>(slot + sizeof(ChunkHeader));
    for (uint32_t s = lane; s < fpad / 2; s += 32)
      fr[s] = static_cast<uint16_t>(s < A ? freq_s[warp][s] : 0u);
    uint32_t* st = reinterpret_cast<uint32_t*>(slot + sizeof(ChunkHeader) + fpad);
    st[lane] = x0;
    st[kLanes + lane] = x1;
  } else {
    if (lane == 0) {
      reinterpret_cast<uint4*>(slot)[0] = make_uint4(n_sym, 0u, 0u, 0u);  // raw record header
      reinterpret_cast<uint4*>(slot)[1] = make_uint4(0u, 0u, 0u, 0u);
      d[0] = static_cast<uint32_t>(raw_len);
      d[1] = static_cast<uint32_t>(raw_len);
      d[2] = d[3] = d[4] = d[5] = 0;
    }
    for (uint32_t ss = 0; ss < n_ss; ++ss) {
      const Syms32 v = load_syms(src, ss, lane, n_sym);
      const uint32_t off = ss * kSuper + lane * kSub;
      uint8_t* dst = slot + sizeof(ChunkHeader) + off;
      if (off < pad16(n_sym)) *reinterpret_cast<uint4*>(dst) = v.lo;
      if (off + 16 < pad16(n_sym)) *reinterpret_cast<uint4*>(dst + 16) = v.hi;
    }
  }
}

// Single CTA: header, exclusive scan of record lengths, directory.  The
// record offsets also go to `dst_off` (local memory) for k_rans_copy, which
// therefore never reads `out` (it may be a peer GPU's buffer).  With
// m.has_prefix the 16-byte container header m.prefix is written just before
// the stream; with m.ck the checksum of everything this kernel writes is
// added (message offset of out[0] = m.msg_off, a multiple of 16).
__global__ void __launch_bounds__(1024) k_rans_directory(const uint32_t* __restrict__ desc,
                                                         uint32_t n_chunks, uint64_t n,
                                                         uint32_t cs, uint8_t* __restrict__ out,
                                                         uint64_t* __restrict__ total_out,
                                                         uint64_t* __restrict__ dst_off,
                                                         const RansMsg m) {
  __shared__ uint64_t part[1024];
  const int tid = threadIdx.x;
  const uint32_t per = (n_chunks + 1023) / 1024;
  const uint32_t b = tid * per, e = min(n_chunks, b + per);
  uint64_t s = 0;
  for (uint32_t i = b; i < e; ++i) s += desc[static_cast<uint64_t>(i) * kDescWords];
  part[tid] = s;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {
    const uint64_t v = tid >= o ? part[tid - o] : 0;
    __syncthreads();
    part[tid] += v;
    __syncthreads();
  }
  const uint64_t base = pad16(directory_bytes(n_chunks));
  uint64_t* dir = reinterpret_cast<uint64_t*>(out + sizeof(StreamHeader));
  uint64_t run = base + (tid > 0 ? part[tid - 1] : 0);
  unsigned long long s1 = 0, s2 = 0;
  // one 64-bit value at stream byte offset `off`: two words of the checksum
  auto ck64 = [&](uint64_t v, uint64_t off) {
    const unsigned long long w = static_cast<unsigned long long>((m.msg_off + off) >> 2) + 1;
    const unsigned long long lo = v & 0xFFFFFFFFull, hi = v >> 32;
    s1 += lo + hi;
    s2 += w * lo + (w + 1) * hi;
  };
  for (uint32_t i = b; i < e; ++i) {
    dir[i] = run;
    dst_off[i] = run;
    if (m.ck != nullptr) ck64(run, sizeof(StreamHeader) + 8ull * i);
    run += desc[static_cast<uint64_t>(i) * kDescWords];
  }
  if (tid == 0) {
    for (uint64_t i = sizeof(StreamHeader) + 8ull * (n_chunks + 1); i < base; ++i) out[i] = 0;
    if (m.has_prefix) {
      uint4 pre = make_uint4(m.prefix[0], m.prefix[1], m.prefix[2], m.prefix[3]);
      *reinterpret_cast<uint4*>(out - 16) = pre;
      if (m.ck != nullptr) ck_word4(pre, m.msg_off - 16, s1, s2);
    }
  }
  if (tid == 1023) {
    const uint64_t total = base + part[1023];
    dir[n_chunks] = total;
    StreamHeader hd{kMagic, n_chunks, n, cs, static_cast<uint32_t>(kProbBits), total};
    *reinterpret_cast<StreamHeader*>(out) = hd;
    if (total_out) *total_out = total;
    if (m.ck != nullptr) {
      ck64(total, sizeof(StreamHeader) + 8ull * n_chunks);
      const uint64_t* hw = reinterpret_cast<const uint64_t*>(&hd);
      for (int k = 0; k < 4; ++k) ck64(hw[k], 8ull * k);
    }
  }
  if (m.ck != nullptr) ck_flush(m.ck, s1, s2);
  __threadfence_system();
}

// One warp per record: compact its pieces (prefix, then the word blocks of
// the two streams) from staging into out (out may be a peer buffer), at the
// offsets the directory kernel left in `dst_off`.  With m.ck the checksum of
// the records is added; with m.counter the last CTA stores the finished
// checksum to m.trailer (when set) and publishes m.flag_value into m.flag
// with release semantics after a system-scope fence.
__global__ void __launch_bounds__(256) k_rans_copy(
    const uint8_t* __restrict__ staging, const uint32_t* __restrict__ desc,
    const uint64_t* __restrict__ dst_off, uint32_t n_chunks, uint32_t cs, uint8_t* out,
    const RansMsg m) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t chunk = blockIdx.x * 8 + warp;
  unsigned long long s1 = 0, s2 = 0;
  if (chunk < n_chunks) {
    const uint32_t* d = desc + static_cast<uint64_t>(chunk) * kDescWords;
    const uint8_t* slot = staging + static_cast<uint64_t>(chunk) * slot_bytes(cs);
    uint64_t doff = dst_off[chunk];
    const uint32_t len[3] = {d[1], d[2], d[3]};
    const uint32_t src_off[3] = {0u, d[4], d[5]};
#pragma unroll
    for (int piece = 0; piece < 3; ++piece) {
      const uint4* sp = reinterpret_cast<const uint4*>(slot + src_off[piece]);
      uint4* dp = reinterpret_cast<uint4*>(out + doff);
      const uint32_t n16 = len[piece] / 16;
      for (uint32_t i = lane; i < n16; i += 32) {
        const uint4 v = sp[i];
        dp[i] = v;
        if (m.ck != nullptr) ck_word4(v, m.msg_off + static_cast<long long>(doff) + 16ll * i, s1, s2);
      }
      doff += len[piece];
    }
  }
  if (m.ck != nullptr) ck_flush(m.ck, s1, s2);
  if (m.counter != nullptr) {
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0)
      last_cta_publish(m.counter, gridDim.x, m.ck, m.trailer, m.flag, m.flag_value);
  }
}

// Every length and offset read from the stream is checked against the
// expected geometry (n symbols in chunks of cs) and the stream length `len`
// (~0 when unknown: then against the header's own total): a corrupt stream
// records ERR_CORRUPT and its chunks are skipped, nothing is read or written
// outside the buffers.
//
// Each stream's words reach shared memory through its own ring of kRing
// (512) words, filled with asynchronous 16-byte copies (128 words a group) a
// quarter super-step ahead: at the start of each quarter (8 sub-steps, at most
// 128 words of a stream) the copies issued at the previous quarter's start
// are waited for, then groups are issued while they fit before (read pointer
// + kRing).  The previous quarter left the ring filled beyond its read
// pointer + 384 and advanced that pointer by at most 128, so every word of
// the current quarter has landed, and no copy overwrites a word not yet read.
__global__ void __launch_bounds__(kDecWarps * 32, kCtasPerSm) k_rans_decode(const uint8_t* __restrict__ stream,
                                                               uint64_t len,
                                                               uint8_t* __restrict__ out,
                                                               uint64_t n_expected, uint32_t cs,
                                                               uint32_t* err) {
  extern __shared__ uint8_t dsm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* lut = dsm + warp * kDecWarpSmem;
  uint32_t* fc = reinterpret_cast<uint32_t*>(lut + 4096);
  uint16_t* ring0 = reinterpret_cast<uint16_t*>(lut + 4096 + 1024);
  uint16_t* ring1 = ring0 + kRing;
  const uint32_t nc = num_chunks(n_expected, cs);
  if (len < sizeof(StreamHeader)) {
    if (threadIdx.x == 0 && blockIdx.x == 0) record_error(err, ERR_CORRUPT);
    return;
  }
  const StreamHeader hd = *reinterpret_cast<const StreamHeader*>(stream);
  const uint64_t dir_end = sizeof(StreamHeader) + 8ull * (nc + 1);
  if (hd.magic != kMagic || hd.n_symbols != n_expected || hd.prob_bits != kProbBits ||
      hd.chunk_symbols != cs || hd.n_chunks != nc || hd.total_bytes > len || hd.total_bytes < dir_end) {
    if (threadIdx.x == 0 && blockIdx.x == 0) record_error(err, ERR_CORRUPT);
    return;
  }
  const uint32_t chunk = blockIdx.x * kDecWarps + warp;
  if (chunk >= nc) return;
  const uint64_t* dir = reinterpret_cast<const uint64_t*>(stream + sizeof(StreamHeader));
  const uint64_t roff = dir[chunk];
  const uint64_t expect = min(static_cast<uint64_t>(cs), n_expected - static_cast<uint64_t>(chunk) * cs);
  if (roff < dir_end || roff + sizeof(ChunkHeader) > hd.total_bytes || (roff & 15) != 0) {
    if (lane == 0) record_error(err, ERR_CORRUPT);
    return;
  }
  const uint8_t* rec = stream + roff;
  const ChunkHeader ch = *reinterpret_cast<const ChunkHeader*>(rec);
  uint8_t* dst = out + static_cast<uint64_t>(chunk) * cs;
  const uint64_t room = hd.total_bytes - roff;  // record bytes available in the stream
  const uint64_t words0 = static_cast<uint64_t>(ch.n_pad[0]) + ch.n_words[0];
  const uint64_t words1 = static_cast<uint64_t>(ch.n_pad[1]) + ch.n_words[1];
  const bool bad = ch.n_sym != expect || ch.alphabet > 256 ||
                   (ch.alphabet == 0 && raw_record_bytes(ch.n_sym) > room) ||
                   (ch.alphabet != 0 &&
                    (coded_prefix_bytes(ch.alphabet) + 2 * (words0 + words1) > room ||
                     (words0 & 7) != 0 || (words1 & 7) != 0));
  if (bad) {
    if (lane == 0) record_error(err, ERR_CORRUPT);
    return;
  }
  const uint32_t n_ss = (ch.n_sym + kSuper - 1) / kSuper;
  if (ch.alphabet == 0) {
    for (uint32_t i = lane; i < ch.n_sym; i += 32) dst[i] = rec[sizeof(ChunkHeader) + i];
    return;
  }
  const uint32_t A = ch.alphabet;
  const uint16_t* freq = reinterpret_cast<const uint16_t*>(rec + sizeof(ChunkHeader));
  const uint32_t fpad = static_cast<uint32_t>(pad16(2ull * A));
  const uint32_t* states = reinterpret_cast<const uint32_t*>(rec + sizeof(ChunkHeader) + fpad);
  const uint16_t* wsrc0 = reinterpret_cast<const uint16_t*>(rec + coded_prefix_bytes(A));
  const uint16_t* wsrc1 = wsrc0 + words0;
  if (lane == 0) {
    uint32_t cum = 0;
    for (uint32_t s = 0; s < A; ++s) {
      const uint32_t f = freq[s];
      fc[s] = f | (cum << 16);
      cum += f;
    }
    if (cum != kProbScale) record_error(err, ERR_CORRUPT);
  }
  __syncwarp();
  for (uint32_t s = 0; s < A; ++s) {
    const uint32_t f = fc[s] & 0xFFFFu, c = fc[s] >> 16;
    for (uint32_t k = lane; k < f; k += 32)
      if (c + k < kProbScale) lut[c + k] = static_cast<uint8_t>(s);
  }
  uint32_t x0 = states[lane], x1 = states[kLanes + lane];
  uint32_t rp0 = ch.n_pad[0], rp1 = ch.n_pad[1];
  uint32_t ld0 = 0, ld1 = 0;  // words of each stream issued to its ring
  const uint32_t lt = lanemask_lt();
  auto refill = [&](uint16_t* ring, const uint16_t* src, uint32_t& loaded, uint32_t rptr,
                    uint64_t total) {
    while (loaded + 128 <= rptr + kRing && loaded < total) {
      const uint32_t idx = loaded + lane * 4;  // 8 bytes a lane, 128 words a group
      if (idx < total)
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(
                         smem_u32(ring + (idx & (kRing - 1)))),
                     "l"(src + idx)
                     : "memory");
      loaded += 128;
    }
  };
  auto refill_both = [&]() {
    refill(ring0, wsrc0, ld0, rp0, words0);
    refill(ring1, wsrc1, ld1, rp1, words1);
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  __syncwarp();
  refill_both();
  for (uint32_t ss = 0; ss < n_ss; ++ss) {
    uint32_t o[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int quarter = 0; quarter < 4; ++quarter) {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
      __syncwarp();
      refill_both();  // the next quarter's words, in flight during this one
#pragma unroll
      for (int mm = 0; mm < kSub / 4; ++mm) {
        const int m = quarter * (kSub / 4) + mm;
        uint32_t& x = (m & 1) ? x1 : x0;
        uint32_t& rp = (m & 1) ? rp1 : rp0;
        const uint16_t* ring = (m & 1) ? ring1 : ring0;
        const uint32_t sl = x & (kProbScale - 1);
        const uint32_t s = lut[sl];
        const uint32_t e = fc[s];
        x = (e & 0xFFFFu) * (x >> kProbBits) + sl - (e >> 16);
        const bool need = x < kStateLow;
        const uint32_t mask = __ballot_sync(0xFFFFFFFFu, need);
        if (need) x = (x << 16) | ring[(rp + __popc(mask & lt)) & (kRing - 1)];
        rp += __popc(mask);
        o[m >> 2] |= s << ((m & 3) * 8);
      }
    }
    const uint32_t off = ss * kSuper + lane * kSub;
    if (off + kSub <= ch.n_sym) {
      *reinterpret_cast<uint4*>(dst + off) = make_uint4(o[0], o[1], o[2], o[3]);
      *reinterpret_cast<uint4*>(dst + off + 16) = make_uint4(o[4], o[5], o[6], o[7]);
    } else {
      for (uint32_t i = 0; i < kSub; ++i)
        if (off + i < ch.n_sym) dst[off + i] = static_cast<uint8_t>(o[i >> 2] >> ((i & 3) * 8));
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  if (x0 != kStateLow || x1 != kStateLow || rp0 != words0 || rp1 != words1)
    record_error(err, ERR_CORRUPT);
}

}  // namespace rans
}  // namespace kvs

using namespace kvs;
using namespace kvs::rans;

extern "C" {

uint64_t kvs_rans_max_bytes(uint64_t n, uint32_t cs) { return max_stream_bytes(n, cs); }
uint64_t kvs_rans_staging_bytes(uint64_t n, uint32_t cs) {
  return static_cast<uint64_t>(num_chunks(n, cs)) * slot_bytes(cs);
}

// Encode n bytes into `out` (capacity kvs_rans_max_bytes).  `sizes` holds
// kvs_rans_sizes_words(n, cs) uint32 (per-chunk record descriptors and the
// 64-bit output offsets).  The stream size is written to *total_out
// (device).  `msg` (host pointer, may be null) places the stream inside a
// transfer message: container header, checksum, and the ready flag published
// by the last CTA.
int kvs_rans_encode(const uint8_t* in, uint64_t n, uint32_t cs, uint8_t* staging, uint32_t* sizes,
                    uint8_t* out, uint64_t* total_out, const RansMsg* msg, void* stream) {
  if (n == 0 || cs == 0 || cs % kSuper != 0 || cs > kMaxChunkSyms) return -2;
  // the kernels move 16-byte words: input, output and scratch must be aligned
  if (((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out) |
        reinterpret_cast<uintptr_t>(staging) | reinterpret_cast<uintptr_t>(sizes)) & 15) != 0)
    return -3;
  RansMsg m{};
  if (msg != nullptr) m = *msg;
  if ((m.msg_off & 15) != 0) return -2;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint32_t nc = num_chunks(n, cs);
  uint32_t* desc = sizes;
  // 6 words per chunk keep the 64-bit offsets 8-byte aligned for any nc
  uint64_t* dst_off = reinterpret_cast<uint64_t*>(sizes + kDescWords * static_cast<uint64_t>(nc));
  k_rans_encode<<<(nc + kEncWarps - 1) / kEncWarps, kEncWarps * 32, 0, s>>>(in, n, cs, staging,
                                                                            desc, nc);
  k_rans_directory<<<1, 1024, 0, s>>>(desc, nc, n, cs, out, total_out, dst_off, m);
  k_rans_copy<<<(nc + 7) / 8, 256, 0, s>>>(staging, desc, dst_off, nc, cs, out, m);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int kvs_rans_msg_size(void) { return static_cast<int>(sizeof(RansMsg)); }
// uint32 words of the `sizes` scratch for n bytes in chunks of cs.
uint64_t kvs_rans_sizes_words(uint64_t n, uint32_t cs) {
  const uint64_t nc = num_chunks(n, cs);
  return (kDescWords + 2) * nc;
}

// Decode n bytes from a stream of `len` bytes (~0: unknown, the header's
// total bounds the reads).
int kvs_rans_decode(const uint8_t* stream_buf, uint64_t len, uint8_t* out, uint64_t n, uint32_t cs,
                    uint32_t* err, void* stream) {
  if (n == 0 || cs == 0) return -2;
  if (((reinterpret_cast<uintptr_t>(stream_buf) | reinterpret_cast<uintptr_t>(out)) & 15) != 0)
    return -3;  // 16-byte loads and stores
  const uint32_t nc = num_chunks(n, cs);
  const int smem = kDecWarps * kDecWarpSmem;
  cudaFuncSetAttribute(k_rans_decode, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  k_rans_decode<<<(nc + kDecWarps - 1) / kDecWarps, kDecWarps * 32, smem,
                  static_cast<cudaStream_t>(stream)>>>(stream_buf, len, out, n, cs, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // extern "C"

// ===================================================================
// No-allocation variant of the encoder (declared in kvs_noalloc.h; no
// counterpart in the reference).  Same kernels as kvs_rans_encode; the
// staging slots, record sizes and total live in the file-scope device
// arrays below instead of caller-provided buffers.
// ===================================================================
#include <cstdio>
#include <mutex>
#include <utility>

#include "kvs_noalloc.h"

namespace kvs {
namespace rans {

constexpr uint64_t kNoAllocMaxSymbols = 16ull << 20;  // 16 MiB of input
constexpr uint32_t kNoAllocChunk = kChunkSymbols;
constexpr uint32_t kNoAllocMaxChunks =
    static_cast<uint32_t>((kNoAllocMaxSymbols + kNoAllocChunk - 1) / kNoAllocChunk);

static __device__ __align__(256) uint8_t g_noalloc_staging[kNoAllocMaxChunks *
                                                           slot_bytes(kNoAllocChunk)];
// record descriptors and 64-bit output offsets (kvs_rans_encode's layout)
static __device__ __align__(256) uint32_t g_noalloc_sizes[(kDescWords + 2) * kNoAllocMaxChunks];
static __device__ __align__(256) uint64_t g_noalloc_total[2];

// Device addresses of the scratch arrays, looked up with the context that
// is current at the call (host code may not pass the array names
// themselves: on the host they are stand-ins, not device addresses).  The
// arrays live in the library's module, which is loaded once per context, so
// the cache is keyed on the context's unique id: a new context on the same
// device (after cudaDeviceReset, or a driver-API context made current by
// the caller) gets its own lookup instead of a stale address.
struct NoAllocScratch {
  uint8_t* staging;
  uint32_t* sizes;
  uint64_t* total;
};
constexpr int kNoAllocMaxDevices = 64;
static NoAllocScratch g_noalloc_addr[kNoAllocMaxDevices];
static unsigned long long g_noalloc_ctx[kNoAllocMaxDevices];  // context id of the entry, 0 = none
static std::mutex g_noalloc_mu;

typedef int (*CtxGetCurrentFn)(void**);
typedef int (*CtxGetIdFn)(void*, unsigned long long*);

// Unique id of the current context (0 when it cannot be read).  Driver entry
// points are fetched through the runtime, so the library keeps no link-time
// dependency on libcuda.
static unsigned long long current_context_id() {
  static CtxGetCurrentFn get_cur = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static bool tried = false;
  if (!tried) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_cur = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
    tried = true;
  }
  void* ctx = nullptr;
  unsigned long long id = 0;
  if (get_cur == nullptr || get_id == nullptr || get_cur(&ctx) != 0 || ctx == nullptr ||
      get_id(ctx, &id) != 0)
    return 0;
  return id;
}

static int noalloc_scratch(NoAllocScratch* out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices)
    return KVS_NOALLOC_NO_DEVICE;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  const unsigned long long ctx = current_context_id();
  if (ctx == 0 || g_noalloc_ctx[dev] != ctx) {
    NoAllocScratch s{nullptr, nullptr, nullptr};
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&s.staging), g_noalloc_staging) !=
            cudaSuccess ||
        cudaGetSymbolAddress(reinterpret_cast<void**>(&s.sizes), g_noalloc_sizes) !=
            cudaSuccess ||
        cudaGetSymbolAddress(reinterpret_cast<void**>(&s.total), g_noalloc_total) !=
            cudaSuccess) {
      cudaGetLastError();  // the failed lookup's own error
      return KVS_NOALLOC_SYMBOL;
    }
    g_noalloc_addr[dev] = s;
    // the lookup made the device's primary context current if no context
    // was; an id that cannot be read (0) means a new lookup on every call
    g_noalloc_ctx[dev] = current_context_id();
  }
  *out = g_noalloc_addr[dev];
  return KVS_NOALLOC_OK;
}

// One launch whose own error is returned (cudaLaunchKernelEx reports the
// error of this launch; an unrelated earlier error stays where it is).
template <typename... KArgs, typename... Args>
static cudaError_t noalloc_launch(void (*kernel)(KArgs...), unsigned grid, unsigned block,
                                  cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cfg.attrs = nullptr;
  cfg.numAttrs = 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace rans
}  // namespace kvs

extern "C" {

uint64_t kvs_rans_encode_noalloc_max_symbols(void) { return kvs::rans::kNoAllocMaxSymbols; }

int kvs_rans_encode_noalloc(const uint8_t* in, uint64_t n, uint8_t* out, uint64_t out_capacity,
                            void* stream) {
  using namespace kvs::rans;
  if (n == 0) return KVS_NOALLOC_EMPTY;
  if (n > kNoAllocMaxSymbols) {
    std::fprintf(stderr,
                 "kvs_rans_encode_noalloc: input of %llu bytes exceeds the fixed scratch limit "
                 "of %llu bytes; use kvs_rans_encode with caller-provided buffers\n",
                 static_cast<unsigned long long>(n),
                 static_cast<unsigned long long>(kNoAllocMaxSymbols));
    return KVS_NOALLOC_TOO_LARGE;
  }
  if (out_capacity < max_stream_bytes(n, kNoAllocChunk)) return KVS_NOALLOC_OUT_TOO_SMALL;
  if (((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15) != 0)
    return KVS_NOALLOC_UNALIGNED;
  NoAllocScratch s;
  if (int rc = noalloc_scratch(&s)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint32_t nc = num_chunks(n, kNoAllocChunk);
  uint32_t* desc = s.sizes;
  uint64_t* dst_off = reinterpret_cast<uint64_t*>(s.sizes + kDescWords * static_cast<uint64_t>(nc));
  const RansMsg none{};
  cudaError_t e = noalloc_launch(k_rans_encode, (nc + kEncWarps - 1) / kEncWarps, kEncWarps * 32,
                                 st, in, n, kNoAllocChunk, s.staging, desc, nc);
  if (e == cudaSuccess)
    e = noalloc_launch(k_rans_directory, 1, 1024, st, desc, nc, n, kNoAllocChunk, out, s.total,
                       dst_off, none);
  if (e == cudaSuccess)
    e = noalloc_launch(k_rans_copy, (nc + 7) / 8, 256, st, s.staging, desc, dst_off, nc,
                       kNoAllocChunk, out, none);
  if (e != cudaSuccess) {
    cudaGetLastError();  // this call's launch error, reported through the return code
    return KVS_NOALLOC_LAUNCH;
  }
  return KVS_NOALLOC_OK;
}

const char* kvs_noalloc_strerror(int code) {
  switch (code) {
    case KVS_NOALLOC_OK: return "ok";
    case KVS_NOALLOC_EMPTY: return "empty input";
    case KVS_NOALLOC_TOO_LARGE: return "input exceeds the no-alloc scratch limit";
    case KVS_NOALLOC_OUT_TOO_SMALL: return "output buffer smaller than kvs_rans_max_bytes(n)";
    case KVS_NOALLOC_NO_DEVICE: return "no current CUDA device";
    case KVS_NOALLOC_SYMBOL: return "cudaGetSymbolAddress of the scratch arrays failed";
    case KVS_NOALLOC_LAUNCH: return "kernel launch failed";
    case KVS_NOALLOC_UNALIGNED: return "input or output not 16-byte aligned";
    default: return "unknown error";
  }
}

}  // extern "C"
