// Shared device helpers for the sm_100a kernels of kvserve_hpdps_b200.
//
// Everything here is hand-written inline PTX for Blackwell (sm_100a):
// mbarriers, TMA tiled loads (no multicast anywhere: these kernels run on
// multi-GPU jobs), bulk copies, tcgen05 tensor-memory allocation, UMMA
// (tcgen05.mma kind::f16) issue/commit and TMEM loads, plus bounded waits
// that record an error code instead of spinning forever.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#define KVS_DEV __device__ __forceinline__

namespace kvs {

// Error codes written (first writer wins) into a device error word.
enum : uint32_t {
  ERR_NONE = 0,
  ERR_MBAR_TIMEOUT = 1,   // a local mbarrier wait ran out of time
  ERR_FLAG_TIMEOUT = 2,   // a cross-GPU ready flag never arrived
  ERR_BOUNDS = 3,         // an index failed a bounds check
  ERR_CORRUPT = 4,        // a stream header or checksum did not validate
  ERR_OVERFLOW = 5,       // an output region was too small
};

constexpr uint64_t kLocalWaitNs = 2000000000ull;  // 2 s for on-chip waits

KVS_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

KVS_DEV uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

KVS_DEV void record_error(uint32_t* err, uint32_t code) {
  if (err != nullptr) atomicCAS(err, 0u, code);
}

// ---------------------------------------------------------------- mbarrier
KVS_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
KVS_DEV void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
KVS_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t tx) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(tx)
               : "memory");
}
KVS_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
KVS_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait that may suspend the thread for up to `hint_ns` while the phase
// is incomplete (it resumes when the phase completes): waiting warps then
// stop competing for issue slots with the warps doing the work.
KVS_DEV bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
// Bounded wait on a phase of an mbarrier.  Returns false (and records
// `code`) when the phase does not complete within `timeout_ns`.
KVS_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err, uint32_t code,
                       uint64_t timeout_ns = kLocalWaitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try_wait_suspend(bar, parity, 100000u)) return true;  // 100 us per suspension
    if (globaltimer() - t0 > timeout_ns) {
      record_error(err, code);
      return false;
    }
  }
}

// ------------------------------------------------------------ async copies
// Generic-proxy smem writes must be fenced before the async proxy (UMMA,
// TMA store) reads them.
KVS_DEV void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// TMA tiled 3-D load of one box into shared memory (no multicast).
KVS_DEV void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

// Untiled bulk copy global -> shared (16-byte aligned, size multiple of 16).
KVS_DEV void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ------------------------------------------------------------------ tcgen05
// Allocate `ncols` TMEM columns (power of two >= 32); executed by a whole warp.
KVS_DEV void tmem_alloc(uint32_t* slot_in_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(slot_in_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
KVS_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
KVS_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
KVS_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Instruction descriptor: bf16 x bf16 -> f32, A and B K-major, M=128, N=128.
//   bits [4,6) c_format=1 (F32); [7,10) a_format=1 (BF16); [10,13) b_format=1;
//   bit 15/16 a/b major = 0 (K); [17,23) N>>3; [24,29) M>>4.
constexpr uint32_t kIdescBf16M128N128 =
    (1u << 4) | (1u << 7) | (1u << 10) | ((128u >> 3) << 17) | ((128u >> 4) << 24);

// Shared-memory matrix descriptor of a K-major operand in the 128-byte
// swizzled canonical layout: 8-row groups 1024 B apart (SBO), rows 128 B
// apart, 16-byte chunks XOR-swizzled by (row % 8).  The tile base must be
// 1024-byte aligned; stepping along K inside the 128-byte row adds the byte
// offset to the start address.
KVS_DEV uint64_t sw128_kmajor_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);  // start address
  d |= static_cast<uint64_t>(1u) << 16;                 // LBO (unused when swizzled)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;         // SBO = 1024 B
  d |= static_cast<uint64_t>(1u) << 46;                 // descriptor version (sm100)
  d |= static_cast<uint64_t>(2u) << 61;                 // SWIZZLE_128B
  return d;
}

KVS_DEV void umma_bf16_f32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every previously issued tcgen05.mma of this thread
// has completed.
KVS_DEV void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// One 128x128x128 product: D[tmem] = A(128xK) * B(128xK)^T over K=128 bf16.
// Both operands are K-major SW128 tiles of 2 x 16 KB (k 0-63, k 64-127).
KVS_DEV void umma_tile_128x128x128(uint32_t d_tmem, uint32_t a_base, uint32_t b_base) {
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    const uint32_t off = static_cast<uint32_t>((ks >> 2) * 16384 + (ks & 3) * 32);
    umma_bf16_f32(d_tmem, sw128_kmajor_desc(a_base + off), sw128_kmajor_desc(b_base + off),
                  kIdescBf16M128N128, ks > 0 ? 1u : 0u);
  }
}

// Load 32 consecutive fp32 columns of this thread's TMEM lane.
KVS_DEV void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// ------------------------------------------------------- system-scope flags
KVS_DEV uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
KVS_DEV void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
KVS_DEV uint64_t ld_acquire_sys64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
KVS_DEV void st_release_sys64(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// --------------------------------------------------------- float helpers
// Order-preserving map float -> uint32 for atomicMin/atomicMax on floats.
KVS_DEV uint32_t float_to_ordered(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
KVS_DEV float ordered_to_float(uint32_t u) {
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u);
}
KVS_DEV float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Quantize one value: floor((v - mn) * rcp + 0.5) clamped to [0, top],
// with explicit round-to-nearest steps (no FMA contraction) so the device
// matches the CPU oracle bit for bit.
KVS_DEV uint32_t quantize_one(float v, float mn, float rcp, float top) {
  float q = floorf(__fadd_rn(__fmul_rn(__fsub_rn(v, mn), rcp), 0.5f));
  q = fminf(fmaxf(q, 0.0f), top);
  return static_cast<uint32_t>(q);
}

// bf16 dequantization as PyTorch evaluates q_bf16 * scale_bf16 + min_bf16:
// each operation is computed in fp32 and rounded to bf16.
KVS_DEV float dequant_bf16(uint32_t q, float scale_bf, float min_bf) {
  const float prod = bf16_round(__fmul_rn(static_cast<float>(q), scale_bf));
  return bf16_round(__fadd_rn(prod, min_bf));
}

// ---- integer/FMA-pipe forms of the same roundings (no XU conversions) ----
// The conversions above (cvt to bf16, floor, float<->int) issue on the
// quarter-rate XU pipe, which bounds the epilogues; these equivalents use
// integer and FMA-pipe instructions only and give identical results for
// finite inputs.

// Round-to-nearest-even to bf16 of a finite float, by integer arithmetic:
// add 0x7FFF plus the lowest kept bit, then truncate (IEEE RNE at bit 16).
KVS_DEV uint32_t bf16_rne_bits(float x) {
  const uint32_t u = __float_as_uint(x);
  return u + 0x7FFFu + ((u >> 16) & 1u);  // bf16 in the high half; low half is garbage
}
KVS_DEV float bf16_round_fast(float x) { return __uint_as_float(bf16_rne_bits(x) & 0xFFFF0000u); }

// Two bf16 (high halves of a, b) -> packed bf16x2 {lo = a, hi = b}.
KVS_DEV uint32_t pack_bf16_hi(uint32_t a, uint32_t b) { return __byte_perm(a, b, 0x7632); }

// Exact float of a small unsigned integer (< 2^23): place it in the
// mantissa of 2^23 and subtract 2^23.
KVS_DEV float small_uint_to_float(uint32_t q) {
  return __fsub_rn(__uint_as_float(q | 0x4B000000u), 8388608.0f);
}

// quantize_one without XU instructions: clamp t to [0, top] first (floor is
// monotone and top is an integer, so clamp-then-floor == floor-then-clamp),
// then floor by adding 2^23 with round-down: the sum's mantissa holds
// floor(t) exactly for 0 <= t < 2^23.
KVS_DEV uint32_t quantize_fast(float v, float mn, float rcp, float top) {
  float t = __fadd_rn(__fmul_rn(__fsub_rn(v, mn), rcp), 0.5f);
  t = fminf(fmaxf(t, 0.0f), top);
  return __float_as_uint(__fadd_rd(t, 8388608.0f)) - 0x4B000000u;
}

// Two floats -> packed bf16x2 {lo, hi}, round-to-nearest-even (one
// conversion instruction for the pair).
KVS_DEV uint32_t cvt_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
KVS_DEV float bf16lo_to_float(uint32_t p) { return __uint_as_float(p << 16); }
KVS_DEV float bf16hi_to_float(uint32_t p) { return __uint_as_float(p & 0xFFFF0000u); }
// Two bf16 sums, each rounded once to bf16.  For bf16 operands this equals
// rounding their fp32 sum to bf16: the fp32 sum is exact unless the
// exponents differ by 16 or more, and then both results are the larger
// operand, the smaller being far below half a bf16 ulp of it.
KVS_DEV uint32_t bf16x2_add(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
// bf16 bits of a float that is already a bf16 value, in both halves.
KVS_DEV uint32_t bf16x2_splat(float x) {
  const uint32_t h = __float_as_uint(x) >> 16;
  return h | (h << 16);
}

// Packed fp32 pairs (sm_100 f32x2 arithmetic): each instruction performs the
// two IEEE operations of its scalar form, rounded the same way, so results
// are bit-identical to the scalar code.
typedef unsigned long long f32x2_t;
KVS_DEV f32x2_t f2_pack(float lo, float hi) {
  f32x2_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
KVS_DEV void f2_unpack(f32x2_t p, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(p));
}
KVS_DEV f32x2_t f2_sub(f32x2_t a, f32x2_t b) {
  f32x2_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
KVS_DEV f32x2_t f2_mul(f32x2_t a, f32x2_t b) {
  f32x2_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
KVS_DEV f32x2_t f2_add(f32x2_t a, f32x2_t b) {
  f32x2_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
KVS_DEV f32x2_t f2_fma(f32x2_t a, f32x2_t b, f32x2_t c) {
  f32x2_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
KVS_DEV f32x2_t f2_add_rd(f32x2_t a, f32x2_t b) {
  f32x2_t r;
  asm("add.rm.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// quantize_bits on a pair of values with their own (min, rcp) pairs: the
// biased bits 2^23 + code of both, by the same operations in the same order.
KVS_DEV void quantize_bits2(float x0, float x1, f32x2_t mn2, f32x2_t rcp2, float top,
                            uint32_t& b0, uint32_t& b1) {
  const f32x2_t t = f2_add(f2_mul(f2_sub(f2_pack(x0, x1), mn2), rcp2), f2_pack(0.5f, 0.5f));
  float t0, t1;
  f2_unpack(t, t0, t1);
  t0 = fminf(fmaxf(t0, 0.0f), top);
  t1 = fminf(fmaxf(t1, 0.0f), top);
  float r0, r1;
  f2_unpack(f2_add_rd(f2_pack(t0, t1), f2_pack(8388608.0f, 8388608.0f)), r0, r1);
  b0 = __float_as_uint(r0);
  b1 = __float_as_uint(r1);
}

// quantize_fast returning the raw bits of 2^23 + code (code in the low
// mantissa bits): callers that pack codes take the bits they need directly.
KVS_DEV uint32_t quantize_bits(float v, float mn, float rcp, float top) {
  float t = __fadd_rn(__fmul_rn(__fsub_rn(v, mn), rcp), 0.5f);
  t = fminf(fmaxf(t, 0.0f), top);
  return __float_as_uint(__fadd_rd(t, 8388608.0f));
}

// q * scale rounded once, from f = float(2^23 + q) (bits 0x4B000000 | q):
// fma(f, scale, -2^23*scale) is exact before its single rounding because
// 2^23*scale is exact and (2^23 + q)*scale - 2^23*scale == q*scale.
KVS_DEV float code_times_scale(uint32_t biased_bits, float scale, float neg_2p23_scale) {
  return __fmaf_rn(__uint_as_float(biased_bits), scale, neg_2p23_scale);
}

KVS_DEV float dequant_fast(uint32_t q, float scale_bf, float min_bf) {
  const float prod = bf16_round_fast(__fmul_rn(small_uint_to_float(q), scale_bf));
  return bf16_round_fast(__fadd_rn(prod, min_bf));
}

// Pack 32 codes of `W` bits each (code j at bits [j*W, j*W+W) of a
// little-endian bit stream) into W 32-bit words.
template <int W>
KVS_DEV void pack32(const uint32_t (&c)[32], uint32_t (&w)[8]) {
#pragma unroll
  for (int i = 0; i < W; ++i) w[i] = 0;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int bit = j * W;
    const int wi = bit >> 5, bo = bit & 31;
    w[wi] |= c[j] << bo;
    if (bo + W > 32) w[wi + 1] |= c[j] >> (32 - bo);
  }
}
template <int W>
KVS_DEV void unpack32(const uint32_t (&w)[8], uint32_t (&c)[32]) {
  constexpr uint32_t mask = (W == 32) ? 0xFFFFFFFFu : ((1u << W) - 1u);
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int bit = j * W;
    const int wi = bit >> 5, bo = bit & 31;
    uint32_t v = w[wi] >> bo;
    if (bo + W > 32) v |= w[wi + 1] << (32 - bo);
    c[j] = v & mask;
  }
}

// ------------------------------------------------------ message checksum
// Message checksum (producer and consumer compute it the same way): over
// the bytes b_p of a message (p = offset inside the message),
// S1 = sum_p b_p * 2^(8*(p%4)) and S2 = sum_p (p/4 + 1) * b_p * 2^(8*(p%4)),
// both mod 2^64 -- the plain and the position-weighted sums of the message's
// little-endian 32-bit words.  Integer sums are order-independent, so any
// grid, and any split of a message over several kernels adding into the
// same two accumulators, gives the same value.
KVS_DEV void ck_byte(uint8_t b, long long p, unsigned long long& s1, unsigned long long& s2) {
  const unsigned long long v = static_cast<unsigned long long>(b) << (8 * (p & 3));
  s1 += v;
  s2 += static_cast<unsigned long long>((p >> 2) + 1) * v;
}

// Four words at message offset `off` (a multiple of 16).
KVS_DEV void ck_word4(const uint4& v, long long off, unsigned long long& s1,
                      unsigned long long& s2) {
  const unsigned long long w = static_cast<unsigned long long>((off >> 2) + 1);
  s1 += static_cast<unsigned long long>(v.x) + v.y + v.z + v.w;
  s2 += w * v.x + (w + 1) * v.y + (w + 2) * v.z + (w + 3) * v.w;
}

// Warp reduction of a thread's partial sums into the accumulators.
KVS_DEV void ck_flush(unsigned long long* ck, unsigned long long s1, unsigned long long s2) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    s1 += __shfl_xor_sync(0xFFFFFFFFu, s1, o);
    s2 += __shfl_xor_sync(0xFFFFFFFFu, s2, o);
  }
  if ((threadIdx.x & 31) == 0 && (s1 | s2)) {
    atomicAdd(ck, s1);
    atomicAdd(ck + 1, s2);
  }
}

// Called by thread 0 of every CTA after its stores and its checksum sums
// (fenced at system scope by the caller): the last CTA of `total_ctas`
// stores the finished sums to `trailer` (may be peer memory), fences at
// system scope and publishes `flag_value` with release semantics.
KVS_DEV void last_cta_publish(uint32_t* counter, uint32_t total_ctas, unsigned long long* ck,
                              unsigned long long* trailer, uint32_t* flag, uint32_t flag_value) {
  const uint32_t done = atomicAdd(counter, 1u);
  if (done == total_ctas - 1) {
    __threadfence();
    if (trailer != nullptr && ck != nullptr) {
      trailer[0] = atomicAdd(ck, 0ull);  // coherent reads of the finished sums
      trailer[1] = atomicAdd(ck + 1, 0ull);
    }
    __threadfence_system();
    if (flag != nullptr) st_release_sys(flag, flag_value);
    *counter = 0;
  }
}

}  // namespace kvs
