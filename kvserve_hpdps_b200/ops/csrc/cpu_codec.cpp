// CPU implementation of the interleaved rANS stream (format: rans.cuh) and
// of the fixed-width bit packing used by the fused kernels.
//
// The encoder emulates the 32 warp lanes (two interleaved streams) of the
// device encoder step by step, so for the same input it produces the same
// bytes as k_rans_encode + k_rans_directory + k_rans_copy.  It is the oracle of the device codec and
// the codec of CPU-only round trips.
//
// Chunks are independent, so both directions run them on a pool of host
// threads (``KVS_CPU_THREADS`` caps the count; default: the hardware
// concurrency): the encoder writes each chunk's record, then places the
// records at their prefix-sum offsets, so the stream is the same bytes for any
// thread count; the decoder reports the error of the lowest failing chunk,
// as a chunk-by-chunk loop would.
#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <system_error>
#include <thread>
#include <vector>

#include "rans.cuh"

using namespace kvs::rans;

namespace {

inline uint32_t umulhi32(uint32_t a, uint32_t b) {
  return static_cast<uint32_t>((static_cast<uint64_t>(a) * b) >> 32);
}

inline uint32_t sym_at(const uint8_t* src, uint32_t n_sym, uint32_t idx) {
  return idx < n_sym ? src[idx] : 0u;
}

// One coding step of the 32 lanes of stream k at symbol offset `base` of the
// super-step (lane l codes symbol base + l * kSub): the words that leave the
// lanes go out in reverse lane order (the device writes a step's words in lane
// order just below the previous ones; emitted in reverse, a step's block is
// reversed too), then every lane's state takes its symbol.
template <bool kTail>
inline void encode_step(const uint8_t* src, uint32_t n_sym, uint32_t base, const EncSym* enc,
                        uint32_t* x, uint16_t* out, uint32_t& n_out) {
  uint32_t sym[kLanes];
  for (int l = 0; l < kLanes; ++l)
    sym[l] = kTail ? sym_at(src, n_sym, base + l * kSub) : src[base + l * kSub];
  for (int l = kLanes - 1; l >= 0; --l) {
    if (x[l] >= enc[sym[l]].x_max) {
      out[n_out++] = static_cast<uint16_t>(x[l] & 0xFFFFu);
      x[l] >>= 16;
    }
  }
  for (int l = 0; l < kLanes; ++l) {
    const EncSym& e = enc[sym[l]];
    const uint32_t q = umulhi32(x[l], e.rcp) >> (e.cmpl_shift >> 16);
    x[l] = x[l] + e.bias + q * (e.cmpl_shift & 0xFFFFu);
  }
}

// Encode one chunk; returns its record (the bytes k_rans_copy would place).
std::vector<uint8_t> encode_chunk(const uint8_t* src, uint32_t n_sym, uint32_t cs) {
  (void)cs;
  const uint32_t n_ss = (n_sym + kSuper - 1) / kSuper;
  // symbols past n_sym up to the last super-step are coded as zeros
  uint64_t hist[256] = {0};
  for (uint32_t i = 0; i < n_sym; ++i) hist[src[i]]++;
  hist[0] += static_cast<uint64_t>(n_ss) * kSuper - n_sym;
  int top = -1;
  for (int s = 0; s < 256; ++s)
    if (hist[s]) top = s;
  const uint32_t A = static_cast<uint32_t>(top + 1);
  uint32_t freq[256] = {0};
  normalize_counts(hist, A, static_cast<uint64_t>(n_ss) * kSuper, freq);
  EncSym enc[256];
  uint32_t cum = 0;
  for (uint32_t s = 0; s < A; ++s) {
    if (freq[s]) enc[s] = make_enc(freq[s], cum);
    cum += freq[s];
  }
  const uint64_t prefix = coded_prefix_bytes(A);
  const uint64_t raw_len = raw_record_bytes(n_sym);
  // words of each stream in emission order (reversed at the end); a symbol
  // sends at most one word out of its state, so half a chunk bounds a stream
  thread_local std::vector<uint16_t> emitted[kStreams];
  const uint32_t cap = n_ss * kSuper / kStreams;
  uint32_t n_emit[kStreams] = {0, 0};
  for (int k = 0; k < kStreams; ++k)
    if (emitted[k].size() < cap) emitted[k].resize(cap);
  uint32_t x[kStreams][kLanes];
  for (int k = 0; k < kStreams; ++k)
    for (int l = 0; l < kLanes; ++l) x[k][l] = kStateLow;
  bool overflow = false;
  for (int ss = static_cast<int>(n_ss) - 1; ss >= 0; --ss) {
    const uint64_t used = n_emit[0] + n_emit[1];
    if (prefix + 2 * (used + kSuper + 16) >= raw_len) {
      overflow = true;
      break;
    }
    const uint32_t base = static_cast<uint32_t>(ss) * kSuper;
    const bool tail = base + kSuper > n_sym;
    for (int m = kSub - 1; m >= 0; --m) {
      const int k = m & 1;
      if (tail)
        encode_step<true>(src, n_sym, base + m, enc, x[k], emitted[k].data(), n_emit[k]);
      else
        encode_step<false>(src, n_sym, base + m, enc, x[k], emitted[k].data(), n_emit[k]);
    }
  }
  if (overflow) {
    std::vector<uint8_t> rec(raw_len, 0);
    const uint32_t hd[8] = {n_sym, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
    std::memcpy(rec.data(), hd, sizeof(hd));
    std::memcpy(rec.data() + sizeof(ChunkHeader), src, n_sym);
    return rec;
  }
  uint32_t nw[kStreams], np[kStreams];
  for (int k = 0; k < kStreams; ++k) {
    nw[k] = n_emit[k];
    np[k] = (8 - (nw[k] & 7)) & 7;
  }
  std::vector<uint8_t> rec(prefix + 2ull * (np[0] + nw[0] + np[1] + nw[1]), 0);
  const uint32_t hd[8] = {n_sym, A, nw[0], nw[1], np[0], np[1], 0u, 0u};
  std::memcpy(rec.data(), hd, sizeof(hd));
  const uint32_t fpad = static_cast<uint32_t>(pad16(2ull * A));
  uint16_t* fr = reinterpret_cast<uint16_t*>(rec.data() + sizeof(ChunkHeader));
  for (uint32_t s = 0; s < A; ++s) fr[s] = static_cast<uint16_t>(freq[s]);
  std::memcpy(rec.data() + sizeof(ChunkHeader) + fpad, x, sizeof(x));
  uint16_t* w = reinterpret_cast<uint16_t*>(rec.data() + prefix);
  for (int k = 0; k < kStreams; ++k) {
    w += np[k];  // leading zero padding
    const uint16_t* e = emitted[k].data();
    for (uint32_t i = 0; i < nw[k]; ++i) w[i] = e[nw[k] - 1 - i];
    w += nw[k];
  }
  return rec;
}

// Runs fn(i) for every i in [0, n) on up to hardware-concurrency threads,
// the calling thread included; returns when all are done.
template <class F>
void parallel_for(uint32_t n, F&& fn) {
  unsigned t = std::thread::hardware_concurrency();
  if (t == 0) t = 1;
  if (const char* e = std::getenv("KVS_CPU_THREADS")) {
    const int v = std::atoi(e);
    if (v > 0) t = std::min<unsigned>(t, static_cast<unsigned>(v));
  }
  t = std::min<unsigned>(t, n);
  if (t <= 1) {
    for (uint32_t i = 0; i < n; ++i) fn(i);
    return;
  }
  std::atomic<uint32_t> next{0};
  auto work = [&] {
    for (uint32_t i = next.fetch_add(1); i < n; i = next.fetch_add(1)) fn(i);
  };
  std::vector<std::thread> pool;
  pool.reserve(t - 1);
  for (unsigned k = 1; k < t; ++k) {
    try {
      pool.emplace_back(work);
    } catch (const std::system_error&) {
      break;  // fewer threads: the others take the remaining items
    }
  }
  work();
  for (auto& th : pool) th.join();
}

// Decode chunk c of a validated stream header; 0 or a negative error code.
int decode_chunk(const uint8_t* stream, uint64_t stream_bytes, const uint64_t* dir,
                 const StreamHeader& hd, uint32_t c, uint8_t* out, uint64_t n) {
  if (dir[c] > stream_bytes || stream_bytes - dir[c] < sizeof(ChunkHeader)) return -4;
  const uint8_t* rec = stream + dir[c];
  const uint64_t room = stream_bytes - dir[c];  // bytes of the record and after it
  ChunkHeader ch;
  std::memcpy(&ch, rec, sizeof(ch));
  const uint64_t first = static_cast<uint64_t>(c) * hd.chunk_symbols;
  if (ch.n_sym > hd.chunk_symbols || ch.alphabet > 256 || ch.n_sym > n - first) return -5;
  uint8_t* dst = out + first;
  if (ch.alphabet == 0) {
    if (raw_record_bytes(ch.n_sym) > room) return -4;
    std::memcpy(dst, rec + sizeof(ChunkHeader), ch.n_sym);
    return 0;
  }
  const uint32_t A = ch.alphabet;
  const uint16_t* freq = reinterpret_cast<const uint16_t*>(rec + sizeof(ChunkHeader));
  const uint32_t fpad = static_cast<uint32_t>(pad16(2ull * A));
  uint64_t total_words[kStreams];
  for (int k = 0; k < kStreams; ++k)
    total_words[k] = static_cast<uint64_t>(ch.n_pad[k]) + ch.n_words[k];
  if (coded_prefix_bytes(A) + 2 * (total_words[0] + total_words[1]) > room) return -4;
  uint32_t x[kStreams][kLanes];
  std::memcpy(x, rec + sizeof(ChunkHeader) + fpad, sizeof(x));
  const uint16_t* words[kStreams];
  words[0] = reinterpret_cast<const uint16_t*>(rec + coded_prefix_bytes(A));
  words[1] = words[0] + total_words[0];
  uint32_t fc[256];
  thread_local std::vector<uint8_t> lut;
  lut.assign(kProbScale, 0);
  uint32_t cum = 0;
  for (uint32_t s = 0; s < A; ++s) {
    fc[s] = freq[s] | (cum << 16);
    for (uint32_t k = 0; k < freq[s] && cum + k < kProbScale; ++k)
      lut[cum + k] = static_cast<uint8_t>(s);
    cum += freq[s];
  }
  if (cum != kProbScale) return -6;
  uint64_t rptr[kStreams] = {ch.n_pad[0], ch.n_pad[1]};
  const uint32_t n_ss = (ch.n_sym + kSuper - 1) / kSuper;
  const uint8_t* lt = lut.data();
  for (uint32_t ss = 0; ss < n_ss; ++ss) {
    const uint32_t base = ss * kSuper;
    // the last super-step of a chunk decodes into a scratch block: its
    // symbols past n_sym are coded zeros that must not be stored
    uint8_t tail_buf[kSuper];
    const bool tail = base + kSuper > ch.n_sym;
    uint8_t* blk = tail ? tail_buf : dst + base;
    for (int m = 0; m < kSub; ++m) {
      const int k = m & 1;
      uint32_t* xk = x[k];
      const uint16_t* wk = words[k];
      uint64_t r = rptr[k];
      // a step takes at most one word per lane
      if (r + kLanes > total_words[k]) {
        for (int l = 0; l < kLanes; ++l) {
          const uint32_t sl = xk[l] & (kProbScale - 1);
          const uint32_t s = lt[sl];
          xk[l] = (fc[s] & 0xFFFFu) * (xk[l] >> kProbBits) + sl - (fc[s] >> 16);
          if (xk[l] < kStateLow) {
            if (r >= total_words[k]) return -7;
            xk[l] = (xk[l] << 16) | wk[r++];
          }
          blk[l * kSub + m] = static_cast<uint8_t>(s);
        }
      } else {
        for (int l = 0; l < kLanes; ++l) {
          const uint32_t sl = xk[l] & (kProbScale - 1);
          const uint32_t s = lt[sl];
          xk[l] = (fc[s] & 0xFFFFu) * (xk[l] >> kProbBits) + sl - (fc[s] >> 16);
          if (xk[l] < kStateLow) xk[l] = (xk[l] << 16) | wk[r++];
          blk[l * kSub + m] = static_cast<uint8_t>(s);
        }
      }
      rptr[k] = r;
    }
    if (tail) std::memcpy(dst + base, tail_buf, ch.n_sym - base);
  }
  for (int k = 0; k < kStreams; ++k) {
    for (int l = 0; l < kLanes; ++l)
      if (x[k][l] != kStateLow) return -8;
    if (rptr[k] != total_words[k]) return -9;
  }
  return 0;
}

// ---- LC (BIT_2 + RZE_1), the format of lc_codec.cu and compression/lc.py:
// header {magic "LCB2", chunk 16384, n (u64), n_chunks, 0, u32 offsets[n_chunks + 1]
// relative to the 16-byte aligned end of the header}; per chunk either a raw record
// {0, cb, 0, 0, bytes} or {1, nz, 0, 0, bitmap of the shuffled chunk's nonzero bytes,
// those bytes}, each padded to 16 bytes.  The shuffle views the chunk (zero padded to
// groups * 64 bytes) as groups of 32 little-endian 16-bit words and stores, plane-major,
// the 32-bit word whose bit l is bit b of word l, for b = 0..15.
constexpr uint32_t kLcMagic = 0x3242434Cu;
constexpr uint32_t kLcChunk = 16384;

inline uint32_t lc_groups(uint32_t cb) { return ((cb + 1) / 2 + 31) / 32; }
inline uint64_t lc_head(uint32_t nc) { return pad16(24 + 4ull * (nc + 1)); }

void lc_shuffle(const uint8_t* chunk, uint32_t cb, uint8_t* sb) {
  const uint32_t G = lc_groups(cb);
  for (uint32_t g = 0; g < G; ++g) {
    uint32_t w[32];
    for (uint32_t l = 0; l < 32; ++l) {
      const uint64_t i = 2ull * (g * 32 + l);
      w[l] = (i < cb ? chunk[i] : 0u) | ((i + 1 < cb ? chunk[i + 1] : 0u) << 8);
    }
    for (uint32_t bit = 0; bit < 16; ++bit) {
      uint32_t plane = 0;
      for (uint32_t l = 0; l < 32; ++l) plane |= ((w[l] >> bit) & 1u) << l;
      std::memcpy(sb + 4ull * (bit * G + g), &plane, 4);
    }
  }
}

void lc_unshuffle(const uint8_t* sb, uint32_t cb, uint8_t* chunk) {
  const uint32_t G = lc_groups(cb);
  for (uint32_t g = 0; g < G; ++g) {
    uint32_t plane[16];
    for (uint32_t bit = 0; bit < 16; ++bit) std::memcpy(&plane[bit], sb + 4ull * (bit * G + g), 4);
    for (uint32_t l = 0; l < 32; ++l) {
      uint32_t w = 0;
      for (uint32_t bit = 0; bit < 16; ++bit) w |= ((plane[bit] >> l) & 1u) << bit;
      const uint64_t i = 2ull * (g * 32 + l);
      if (i < cb) chunk[i] = static_cast<uint8_t>(w);
      if (i + 1 < cb) chunk[i + 1] = static_cast<uint8_t>(w >> 8);
    }
  }
}

// One record (padded to 16 bytes) for a chunk of cb bytes.
std::vector<uint8_t> lc_record(const uint8_t* chunk, uint32_t cb) {
  const uint32_t S = lc_groups(cb) * 64;
  std::vector<uint8_t> sb(S);
  lc_shuffle(chunk, cb, sb.data());
  uint32_t nz = 0;
  for (uint32_t i = 0; i < S; ++i) nz += sb[i] != 0;
  const uint64_t coded = 16ull + S / 8 + nz;
  if (coded >= 16 + pad16(cb)) {
    std::vector<uint8_t> rec(16 + pad16(cb), 0);
    const uint32_t hd[4] = {0u, cb, 0u, 0u};
    std::memcpy(rec.data(), hd, 16);
    std::memcpy(rec.data() + 16, chunk, cb);
    return rec;
  }
  std::vector<uint8_t> rec(pad16(coded), 0);
  const uint32_t hd[4] = {1u, nz, 0u, 0u};
  std::memcpy(rec.data(), hd, 16);
  uint8_t* bitmap = rec.data() + 16;
  uint8_t* vals = bitmap + S / 8;
  for (uint32_t i = 0; i < S; ++i) {
    if (sb[i]) {
      bitmap[i >> 3] |= static_cast<uint8_t>(1u << (i & 7));
      *vals++ = sb[i];
    }
  }
  return rec;
}

// Decode record c into out; 0 or a negative error code.
int lc_decode_chunk(const uint8_t* rec, uint64_t rec_len, uint32_t cb, uint8_t* out) {
  if (rec_len < 16) return -4;
  uint32_t hd[4];
  std::memcpy(hd, rec, 16);
  if (hd[0] == 0) {
    if (hd[1] != cb || 16ull + cb > rec_len) return -5;
    std::memcpy(out, rec + 16, cb);
    return 0;
  }
  if (hd[0] != 1) return -5;
  const uint32_t S = lc_groups(cb) * 64;
  const uint32_t nz = hd[1];
  if (nz > S || 16ull + S / 8 + nz > rec_len) return -5;
  const uint8_t* bitmap = rec + 16;
  const uint8_t* vals = bitmap + S / 8;
  std::vector<uint8_t> sb(S, 0);
  uint32_t k = 0;
  for (uint32_t i = 0; i < S; ++i) {
    if (bitmap[i >> 3] >> (i & 7) & 1u) {
      if (k >= nz) return -6;
      sb[i] = vals[k++];
    }
  }
  if (k != nz) return -6;
  lc_unshuffle(sb.data(), cb, out);
  return 0;
}

}  // namespace

extern "C" {

uint64_t kvs_cpu_rans_max_bytes(uint64_t n, uint32_t cs) { return max_stream_bytes(n, cs); }

// Encode n bytes; returns the stream size or 0 on error.
uint64_t kvs_cpu_rans_encode(const uint8_t* in, uint64_t n, uint32_t cs, uint8_t* out,
                             uint64_t out_cap) {
  if (n == 0 || cs == 0 || cs % kSuper != 0) return 0;
  const uint32_t nc = num_chunks(n, cs);
  std::vector<std::vector<uint8_t>> recs(nc);
  parallel_for(nc, [&](uint32_t c) {
    const uint64_t start = static_cast<uint64_t>(c) * cs;
    const uint32_t n_sym = static_cast<uint32_t>(std::min<uint64_t>(cs, n - start));
    recs[c] = encode_chunk(in + start, n_sym, cs);
  });
  const uint64_t base = pad16(directory_bytes(nc));
  std::vector<uint64_t> dir(nc + 1);
  uint64_t run = base;
  for (uint32_t c = 0; c < nc; ++c) {
    dir[c] = run;
    run += recs[c].size();
  }
  dir[nc] = run;
  if (run > out_cap) return 0;
  parallel_for(nc, [&](uint32_t c) { std::memcpy(out + dir[c], recs[c].data(), recs[c].size()); });
  std::memset(out + sizeof(StreamHeader) + 8ull * (nc + 1), 0,
              base - sizeof(StreamHeader) - 8ull * (nc + 1));
  StreamHeader hd{kMagic, nc, n, cs, static_cast<uint32_t>(kProbBits), run};
  std::memcpy(out, &hd, sizeof(hd));
  std::memcpy(out + sizeof(StreamHeader), dir.data(), 8ull * (nc + 1));
  return run;
}

// Decode a stream into n bytes; returns 0 on success, negative on error.  The
// header, the directory and every record are checked against the stream
// length and n before anything is read or written through them.
int kvs_cpu_rans_decode(const uint8_t* stream, uint64_t stream_bytes, uint8_t* out, uint64_t n) {
  if (stream_bytes < sizeof(StreamHeader)) return -1;
  StreamHeader hd;
  std::memcpy(&hd, stream, sizeof(hd));
  if (hd.magic != kMagic || hd.n_symbols != n || hd.prob_bits != kProbBits) return -2;
  if (hd.total_bytes > stream_bytes) return -3;
  if (hd.chunk_symbols == 0 || hd.n_chunks != num_chunks(n, hd.chunk_symbols)) return -2;
  if (directory_bytes(hd.n_chunks) > stream_bytes) return -4;
  std::vector<uint64_t> dir(hd.n_chunks + 1);
  std::memcpy(dir.data(), stream + sizeof(StreamHeader), 8ull * (hd.n_chunks + 1));
  std::vector<int> rc(hd.n_chunks, 0);
  parallel_for(hd.n_chunks, [&](uint32_t c) {
    rc[c] = decode_chunk(stream, stream_bytes, dir.data(), hd, c, out, n);
  });
  for (uint32_t c = 0; c < hd.n_chunks; ++c)
    if (rc[c] != 0) return rc[c];
  return 0;
}

uint64_t kvs_cpu_lc_max_bytes(uint64_t n) {
  const uint32_t nc = static_cast<uint32_t>((n + kLcChunk - 1) / kLcChunk);
  return lc_head(nc) + nc * (16 + pad16(kLcChunk));
}

// LC stream of n bytes (chunks on host threads); returns its size or 0.
uint64_t kvs_cpu_lc_encode(const uint8_t* in, uint64_t n, uint8_t* out, uint64_t out_cap) {
  if (n == 0) return 0;
  const uint32_t nc = static_cast<uint32_t>((n + kLcChunk - 1) / kLcChunk);
  std::vector<std::vector<uint8_t>> recs(nc);
  parallel_for(nc, [&](uint32_t c) {
    const uint64_t first = static_cast<uint64_t>(c) * kLcChunk;
    recs[c] = lc_record(in + first, static_cast<uint32_t>(std::min<uint64_t>(kLcChunk, n - first)));
  });
  const uint64_t head = lc_head(nc);
  std::vector<uint32_t> offs(nc + 1);
  uint64_t run = 0;
  for (uint32_t c = 0; c < nc; ++c) {
    offs[c] = static_cast<uint32_t>(run);
    run += recs[c].size();
  }
  offs[nc] = static_cast<uint32_t>(run);
  if (head + run > out_cap || run > 0xFFFFFFFFull) return 0;
  std::memset(out, 0, head);
  const uint32_t h0[2] = {kLcMagic, kLcChunk};
  std::memcpy(out, h0, 8);
  std::memcpy(out + 8, &n, 8);
  const uint32_t h2[2] = {nc, 0u};
  std::memcpy(out + 16, h2, 8);
  std::memcpy(out + 24, offs.data(), 4ull * (nc + 1));
  parallel_for(nc, [&](uint32_t c) {
    std::memcpy(out + head + offs[c], recs[c].data(), recs[c].size());
  });
  return head + run;
}

// Decode an LC stream into n bytes; 0 or a negative error code (the lowest
// failing chunk's).  Offsets and records are checked against the stream.
int kvs_cpu_lc_decode(const uint8_t* stream, uint64_t len, uint8_t* out, uint64_t n) {
  const uint32_t nc = static_cast<uint32_t>((n + kLcChunk - 1) / kLcChunk);
  const uint64_t head = lc_head(nc);
  if (n == 0 || len < head) return -1;
  uint32_t h0[2], h2[2];
  uint64_t hn;
  std::memcpy(h0, stream, 8);
  std::memcpy(&hn, stream + 8, 8);
  std::memcpy(h2, stream + 16, 8);
  if (h0[0] != kLcMagic || h0[1] != kLcChunk || hn != n || h2[0] != nc) return -2;
  std::vector<uint32_t> offs(nc + 1);
  std::memcpy(offs.data(), stream + 24, 4ull * (nc + 1));
  for (uint32_t c = 0; c < nc; ++c)
    if (offs[c] > offs[c + 1]) return -3;
  if (head + offs[nc] > len) return -3;
  std::vector<int> rc(nc, 0);
  parallel_for(nc, [&](uint32_t c) {
    const uint64_t first = static_cast<uint64_t>(c) * kLcChunk;
    rc[c] = lc_decode_chunk(stream + head + offs[c], offs[c + 1] - offs[c],
                            static_cast<uint32_t>(std::min<uint64_t>(kLcChunk, n - first)),
                            out + first);
  });
  for (uint32_t c = 0; c < nc; ++c)
    if (rc[c] != 0) return rc[c];
  return 0;
}

// Fixed-width packing of rows of 128 codes (code j of a 32-code group at
// bits [j*W, j*W+W) of W little-endian 32-bit words); the device kernels
// read and write the same layout.
void kvs_cpu_bitpack(const uint8_t* codes, uint64_t n_rows, int bits, uint8_t* out) {
  for (uint64_t r = 0; r < n_rows; ++r) {
    const uint8_t* c = codes + r * 128;
    uint32_t* w = reinterpret_cast<uint32_t*>(out + r * 16ull * bits);
    std::memset(w, 0, 16ull * bits);
    for (int g = 0; g < 4; ++g) {
      uint32_t* wg = w + g * bits;
      for (int j = 0; j < 32; ++j) {
        const uint32_t v = c[g * 32 + j] & ((1u << bits) - 1u);
        const int bit = j * bits, wi = bit >> 5, bo = bit & 31;
        wg[wi] |= v << bo;
        if (bo + bits > 32) wg[wi + 1] |= v >> (32 - bo);
      }
    }
  }
}

void kvs_cpu_bitunpack(const uint8_t* packed, uint64_t n_rows, int bits, uint8_t* codes) {
  const uint32_t mask = bits >= 32 ? 0xFFFFFFFFu : ((1u << bits) - 1u);
  for (uint64_t r = 0; r < n_rows; ++r) {
    const uint32_t* w = reinterpret_cast<const uint32_t*>(packed + r * 16ull * bits);
    uint8_t* c = codes + r * 128;
    for (int g = 0; g < 4; ++g) {
      const uint32_t* wg = w + g * bits;
      for (int j = 0; j < 32; ++j) {
        const int bit = j * bits, wi = bit >> 5, bo = bit & 31;
        uint32_t v = wg[wi] >> bo;
        if (bo + bits > 32) v |= wg[wi + 1] << (32 - bo);
        c[g * 32 + j] = static_cast<uint8_t>(v & mask);
      }
    }
  }
}

}  // extern "C"
