// Corrupt-stream harness for the CPU decoders of cpu_codec.cpp (rANS and LC).
// Built with AddressSanitizer by tests/test_native_codecs_cpu.py: every
// corrupted copy of a valid stream sits in an allocation of exactly its size,
// so any read past the stream or write past the output is reported.  Each
// decode must return 0 or a negative error code.
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <vector>

extern "C" {
uint64_t kvs_cpu_rans_max_bytes(uint64_t n, uint32_t cs);
uint64_t kvs_cpu_rans_encode(const uint8_t* in, uint64_t n, uint32_t cs, uint8_t* out,
                             uint64_t cap);
int kvs_cpu_rans_decode(const uint8_t* stream, uint64_t stream_bytes, uint8_t* out, uint64_t n);
uint64_t kvs_cpu_lc_max_bytes(uint64_t n);
uint64_t kvs_cpu_lc_encode(const uint8_t* in, uint64_t n, uint8_t* out, uint64_t cap);
int kvs_cpu_lc_decode(const uint8_t* stream, uint64_t len, uint8_t* out, uint64_t n);
}

namespace {

std::vector<uint8_t> sample(std::mt19937_64& rng, uint64_t n) {
  std::vector<uint8_t> x(n);
  for (auto& v : x) v = (rng() % 100 < 88) ? static_cast<uint8_t>(rng() % 6)
                                            : static_cast<uint8_t>(rng());
  for (uint64_t i = n / 3; i < std::min<uint64_t>(n, n / 3 + 33000); ++i)
    x[i] = static_cast<uint8_t>(rng());  // incompressible chunks: raw records
  return x;
}

template <class Decode>
int fuzz(const char* name, std::mt19937_64& rng, const std::vector<uint8_t>& s, uint64_t n,
         int iters, Decode decode) {
  int accepted = 0, rejected = 0;
  for (int it = 0; it < iters; ++it) {
    uint64_t len = s.size();
    if (it % 4 == 0) len = rng() % (len + 1);  // truncated
    uint8_t* b = static_cast<uint8_t*>(std::malloc(len ? len : 1));
    std::memcpy(b, s.data(), len);
    if (it % 4 == 1)  // bit flips anywhere
      for (int k = 0; k < 1 + static_cast<int>(rng() % 8); ++k) b[rng() % len] ^= 1u << (rng() % 8);
    if (it % 4 >= 2 && len > 0)  // header, directory and early record bytes
      b[rng() % std::min<uint64_t>(len, it % 4 == 2 ? 64 : 512)] = static_cast<uint8_t>(rng());
    std::vector<uint8_t> out(n);
    const int rc = decode(b, len, out.data(), n);
    std::free(b);
    if (rc > 0) {
      std::printf("%s: positive return %d\n", name, rc);
      return 1;
    }
    (rc == 0 ? accepted : rejected)++;
  }
  std::printf("%s: %d decoded, %d rejected\n", name, accepted, rejected);
  return rejected > 0 ? 0 : 1;
}

}  // namespace

int main(int argc, char** argv) {
  const int iters = argc > 1 ? std::atoi(argv[1]) : 4000;
  std::mt19937_64 rng(7);
  const uint64_t n = 120001;
  const std::vector<uint8_t> x = sample(rng, n);
  std::vector<uint8_t> y(n);

  std::vector<uint8_t> rs(kvs_cpu_rans_max_bytes(n, 32768));
  rs.resize(kvs_cpu_rans_encode(x.data(), n, 32768, rs.data(), rs.size()));
  if (rs.empty() || kvs_cpu_rans_decode(rs.data(), rs.size(), y.data(), n) != 0 || y != x) {
    std::puts("rans: baseline round trip failed");
    return 1;
  }
  std::vector<uint8_t> ls(kvs_cpu_lc_max_bytes(n));
  ls.resize(kvs_cpu_lc_encode(x.data(), n, ls.data(), ls.size()));
  if (ls.empty() || kvs_cpu_lc_decode(ls.data(), ls.size(), y.data(), n) != 0 || y != x) {
    std::puts("lc: baseline round trip failed");
    return 1;
  }
  int bad = fuzz("rans", rng, rs, n, iters, kvs_cpu_rans_decode);
  bad |= fuzz("lc", rng, ls, n, iters, kvs_cpu_lc_decode);
  return bad;
}
