// Fused error-metric reductions for the offline profile search and the
// round-trip checks (reference: cosine / MSE of tests/test_v3_roundtrip.py:44
// and the accuracy evaluators of kvserve_v1/offline_search).
//
// k_kv_error: one pass over two bf16 tensors accumulating, in fp64,
//   sum (a-r)^2, sum r^2, sum a^2, sum a*r and max |a-r|.
// k_logit_agreement: one CTA per row of two [rows, vocab] fp32 logit
//   matrices: argmax of each, and KL(softmax(ref) || softmax(approx)).
#include "common.cuh"

namespace kvs {

KVS_DEV double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}
KVS_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}

__global__ void __launch_bounds__(256) k_kv_error(const __nv_bfloat16* __restrict__ ref,
                                                  const __nv_bfloat16* __restrict__ approx,
                                                  long long n, double* acc, uint32_t* maxabs) {
  double sd = 0, sr = 0, sa = 0, sx = 0;
  float mx = 0.f;
  const long long n8 = n / 8;
  const uint4* r8 = reinterpret_cast<const uint4*>(ref);
  const uint4* a8 = reinterpret_cast<const uint4*>(approx);
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n8; i += stride) {
    const uint4 ru = r8[i], au = a8[i];
    const uint32_t rw[4] = {ru.x, ru.y, ru.z, ru.w}, aw[4] = {au.x, au.y, au.z, au.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const float r = __uint_as_float(k ? (rw[j] & 0xFFFF0000u) : (rw[j] << 16));
        const float a = __uint_as_float(k ? (aw[j] & 0xFFFF0000u) : (aw[j] << 16));
        const double d = static_cast<double>(a) - r;
        sd += d * d;
        sr += static_cast<double>(r) * r;
        sa += static_cast<double>(a) * a;
        sx += static_cast<double>(a) * r;
        mx = fmaxf(mx, fabsf(a - r));
      }
    }
  }
  for (long long i = n8 * 8 + blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n; i += stride) {
    const float r = __bfloat162float(ref[i]), a = __bfloat162float(approx[i]);
    const double d = static_cast<double>(a) - r;
    sd += d * d;
    sr += static_cast<double>(r) * r;
    sa += static_cast<double>(a) * a;
    sx += static_cast<double>(a) * r;
    mx = fmaxf(mx, fabsf(a - r));
  }
  sd = warp_sum(sd);
  sr = warp_sum(sr);
  sa = warp_sum(sa);
  sx = warp_sum(sx);
  mx = warp_max(mx);
  if ((threadIdx.x & 31) == 0) {
    atomicAdd(&acc[0], sd);
    atomicAdd(&acc[1], sr);
    atomicAdd(&acc[2], sa);
    atomicAdd(&acc[3], sx);
    atomicMax(maxabs, __float_as_uint(mx));  // non-negative floats order as uints
  }
}

// out[row] = {argmax(ref), argmax(approx), KL(ref || approx)}
__global__ void __launch_bounds__(256) k_logit_agreement(const float* __restrict__ ref,
                                                         const float* __restrict__ approx,
                                                         int vocab, float* out) {
  __shared__ float s_val[8];
  __shared__ int s_idx[8];
  __shared__ double s_d[8];
  const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* r = ref + static_cast<long long>(row) * vocab;
  const float* a = approx + static_cast<long long>(row) * vocab;
  float res[3];
  float mr = -INFINITY, ma = -INFINITY;
  int ir = 0, ia = 0;
  for (int v = tid; v < vocab; v += blockDim.x) {
    if (r[v] > mr) { mr = r[v]; ir = v; }
    if (a[v] > ma) { ma = a[v]; ia = v; }
  }
  // block argmax (ties -> smallest index), twice
  for (int pass = 0; pass < 2; ++pass) {
    float m = pass ? ma : mr;
    int idx = pass ? ia : ir;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float om = __shfl_xor_sync(0xFFFFFFFFu, m, o);
      const int oi = __shfl_xor_sync(0xFFFFFFFFu, idx, o);
      if (om > m || (om == m && oi < idx)) { m = om; idx = oi; }
    }
    if (lane == 0) { s_val[warp] = m; s_idx[warp] = idx; }
    __syncthreads();
    if (tid == 0) {
      float bm = s_val[0];
      int bi = s_idx[0];
      for (int w = 1; w < static_cast<int>(blockDim.x) / 32; ++w)
        if (s_val[w] > bm || (s_val[w] == bm && s_idx[w] < bi)) { bm = s_val[w]; bi = s_idx[w]; }
      s_val[0] = bm;
      s_idx[0] = bi;
    }
    __syncthreads();
    if (pass == 0) { mr = s_val[0]; res[0] = static_cast<float>(s_idx[0]); }
    else { ma = s_val[0]; res[1] = static_cast<float>(s_idx[0]); }
    __syncthreads();
  }
  // log-sum-exp of both rows and sum p_r * (log p_r - log p_a)
  double zr = 0, za = 0;
  for (int v = tid; v < vocab; v += blockDim.x) {
    zr += exp(static_cast<double>(r[v]) - mr);
    za += exp(static_cast<double>(a[v]) - ma);
  }
  double sums[2] = {zr, za};
  for (int k = 0; k < 2; ++k) {
    double x = warp_sum(sums[k]);
    if (lane == 0) s_d[warp] = x;
    __syncthreads();
    if (tid == 0) {
      double t = 0;
      for (int w = 0; w < static_cast<int>(blockDim.x) / 32; ++w) t += s_d[w];
      s_d[0] = t;
    }
    __syncthreads();
    sums[k] = s_d[0];
    __syncthreads();
  }
  const double lzr = log(sums[0]) + mr, lza = log(sums[1]) + ma;
  double kl = 0;
  for (int v = tid; v < vocab; v += blockDim.x) {
    const double lpr = static_cast<double>(r[v]) - lzr;
    const double lpa = static_cast<double>(a[v]) - lza;
    kl += exp(lpr) * (lpr - lpa);
  }
  kl = warp_sum(kl);
  if (lane == 0) s_d[warp] = kl;
  __syncthreads();
  if (tid == 0) {
    double t = 0;
    for (int w = 0; w < static_cast<int>(blockDim.x) / 32; ++w) t += s_d[w];
    out[3 * row + 0] = res[0];
    out[3 * row + 1] = res[1];
    out[3 * row + 2] = static_cast<float>(t);
  }
}

}  // namespace kvs

using namespace kvs;

extern "C" {

// acc: 4 doubles (zeroed by the caller), maxabs: one uint32 (zeroed).
int kvs_kv_error(const void* ref, const void* approx, long long n, double* acc, uint32_t* maxabs,
                 void* stream) {
  if (n <= 0) return 0;
  long long blocks = (n / 8 + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks < 1) blocks = 1;
  k_kv_error<<<static_cast<int>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(ref), static_cast<const __nv_bfloat16*>(approx), n, acc,
      maxabs);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int kvs_logit_agreement(const float* ref, const float* approx, int rows, int vocab, float* out,
                        void* stream) {
  if (rows <= 0) return 0;
  k_logit_agreement<<<rows, 256, 0, static_cast<cudaStream_t>(stream)>>>(ref, approx, vocab, out);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // extern "C"
