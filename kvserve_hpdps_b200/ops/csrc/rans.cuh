// Stream format and constants of the interleaved rANS codec shared by the
// device kernels (rans.cu) and the CPU implementation (cpu_codec.cpp).
//
// Method: range-variant asymmetric numeral systems (J. Duda, "Asymmetric
// numeral systems", 2013) with 32 interleaved states per chunk (F. Giesen,
// "Interleaved entropy coders", 2014), 32-bit states in [2^15, 2^31),
// 16-bit renormalisation and 12-bit probabilities.  Division by a symbol
// frequency in the encoder uses a precomputed reciprocal (T. Granlund and
// P. Montgomery, "Division by invariant integers using multiplication",
// 1994): for f >= 2, s = ceil(log2 f), rcp = ceil(2^(31+s) / f) and
// x / f = umulhi(x, rcp) >> (s-1), exact for x < 2^31.
//
// Stream layout (all offsets in bytes, little endian):
//   StreamHeader (32 B)
//   uint64 dir[n_chunks + 1]      record offsets from the stream start
//   records, each 16-byte aligned:
//     ChunkHeader (32 B) {n_sym, alphabet A (0 = raw), n_words[2], n_pad[2], 0, 0}
//     A > 0: uint16 freq[A] (padded to 16 B), uint32 state[2][32],
//            uint16 words0[n_pad[0] + n_words[0]], uint16 words1[n_pad[1] + n_words[1]]
//            (the first n_pad[k] words of each block are padding; every block is a
//            multiple of 8 words)
//     A = 0: n_sym raw bytes (padded to 16 B)
// Chunk c covers symbols [c*chunk_symbols, min((c+1)*chunk_symbols, n)).
// A chunk holds two interleaved rANS streams that share its frequency table:
// every lane owns one state of each.  Symbol j of a chunk (after zero padding
// to a multiple of 1024) belongs to super-step j/1024, lane (j%1024)/32,
// sub-step j%32 and stream j%2.  Decoding runs super-steps and sub-steps in
// increasing order; at each sub-step the lanes whose state of that sub-step's
// stream fell below 2^15 read one word each from that stream's words, in lane
// order.  Consecutive sub-steps therefore update independent states, which
// gives each lane two dependency chains to interleave.
#pragma once

#include <cstdint>

namespace kvs {
namespace rans {

constexpr uint32_t kMagic = 0x3252564Bu;  // "KVR2"
constexpr int kLanes = 32;
constexpr int kStreams = 2;                           // rANS streams per chunk (states per lane)
constexpr int kSub = 32;                              // symbols per lane per super-step
constexpr int kSuper = kLanes * kSub;                 // 1024 symbols per super-step
constexpr uint32_t kChunkSymbols = 32768;             // default chunk size
constexpr uint32_t kMaxChunkSyms = 1u << 18;          // largest chunk the GPU encoder takes
constexpr int kProbBits = 12;
constexpr uint32_t kProbScale = 1u << kProbBits;      // M = 4096
constexpr uint32_t kStateLow = 1u << 15;              // L
constexpr uint32_t kXmaxShift = 19;                   // ((L >> kProbBits) << 16) == 1 << 19

struct StreamHeader {
  uint32_t magic;
  uint32_t n_chunks;
  uint64_t n_symbols;
  uint32_t chunk_symbols;
  uint32_t prob_bits;
  uint64_t total_bytes;
};
static_assert(sizeof(StreamHeader) == 32, "header size");

struct ChunkHeader {
  uint32_t n_sym;
  uint32_t alphabet;
  uint32_t n_words[kStreams];
  uint32_t n_pad[kStreams];
  uint32_t reserved[2];
};
static_assert(sizeof(ChunkHeader) == 32, "chunk header size");

inline constexpr uint64_t pad16(uint64_t x) { return (x + 15) & ~uint64_t(15); }

// Bytes of a raw (uncoded) record of n symbols: the largest record.
inline constexpr uint64_t raw_record_bytes(uint64_t n) { return sizeof(ChunkHeader) + pad16(n); }

// Bytes before the word blocks of a coded record with alphabet A.
inline constexpr uint64_t coded_prefix_bytes(uint32_t A) {
  return sizeof(ChunkHeader) + pad16(2ull * A) + 4ull * kStreams * kLanes;
}

// Staging slot of one chunk (encoder): the record prefix (header,
// frequencies, states; or the whole raw record) from the slot start, then one
// region per stream whose words are written backwards from the region's end.
constexpr uint64_t kPrefixArea = 1024;
static_assert(kPrefixArea >= sizeof(ChunkHeader) + 512 + 4 * kStreams * kLanes, "prefix area");
inline constexpr uint64_t region_bytes(uint32_t cs) { return pad16(cs) + 16; }
inline constexpr uint64_t slot_bytes(uint32_t cs) { return kPrefixArea + kStreams * region_bytes(cs); }

inline constexpr uint64_t directory_bytes(uint32_t n_chunks) {
  return sizeof(StreamHeader) + 8ull * (n_chunks + 1);
}

inline constexpr uint32_t num_chunks(uint64_t n, uint32_t cs) {
  return static_cast<uint32_t>((n + cs - 1) / cs);
}

// Upper bound of an encoded stream (every chunk raw).
inline constexpr uint64_t max_stream_bytes(uint64_t n, uint32_t cs) {
  return pad16(directory_bytes(num_chunks(n, cs))) + num_chunks(n, cs) * raw_record_bytes(cs);
}

// Per chunk of the encoder's scratch (uint32 words): record length, prefix
// length, byte length of each word block, staging offset of each word block.
constexpr int kDescWords = 6;
static_assert(kDescWords % 2 == 0, "the 64-bit output offsets after the descriptors stay aligned");

// Per-symbol encoder entry.
struct EncSym {
  uint32_t rcp;
  uint32_t x_max;
  uint32_t bias;
  uint32_t cmpl_shift;  // (M - f) | (rshift << 16)
};

// Normalise counts (sum = total > 0) to frequencies summing to M, every
// present symbol >= 1; deterministic integer procedure shared by CPU and GPU
// (the GPU runs it on one lane).
template <typename CountT>
inline
#ifdef __CUDACC__
__host__ __device__
#endif
    uint32_t normalize_counts(const CountT* cnt, uint32_t alphabet, uint64_t total,
                              uint32_t* freq) {
  int64_t sum = 0;
  uint32_t best = 0;
  CountT best_cnt = 0;
  for (uint32_t s = 0; s < alphabet; ++s) {
    uint32_t f = 0;
    if (cnt[s] > 0) {
      f = static_cast<uint32_t>((static_cast<uint64_t>(cnt[s]) * kProbScale) / total);
      if (f < 1) f = 1;
      if (cnt[s] > best_cnt) {
        best_cnt = cnt[s];
        best = s;
      }
    }
    freq[s] = f;
    sum += f;
  }
  int64_t diff = static_cast<int64_t>(kProbScale) - sum;
  while (diff != 0) {
    if (diff > 0) {
      freq[best] += static_cast<uint32_t>(diff);
      diff = 0;
    } else {
      uint32_t s_max = 0, f_max = 0;
      for (uint32_t s = 0; s < alphabet; ++s)
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
  return best;
}

inline
#ifdef __CUDACC__
__host__ __device__
#endif
    EncSym make_enc(uint32_t f, uint32_t cum) {
  EncSym e;
  e.x_max = f << kXmaxShift;
  if (f >= 2) {
    uint32_t s = 0;
    while ((1u << s) < f) ++s;
    e.rcp = static_cast<uint32_t>(((1ull << (31 + s)) + f - 1) / f);
    e.bias = cum;
    e.cmpl_shift = (kProbScale - f) | ((s - 1) << 16);
  } else {
    e.rcp = 0xFFFFFFFFu;
    e.bias = cum + kProbScale - 1;
    e.cmpl_shift = (kProbScale - f);
  }
  return e;
}

}  // namespace rans
}  // namespace kvs
