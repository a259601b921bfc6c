// Data-movement kernels of the transfer path:
//  * raw paged-block gather / scatter (compression off), where the gather
//    destination may be a peer GPU's receive ring (NVLink stores);
//  * contiguous device-to-device / device-to-peer copies with an optional
//    release flag published by the last CTA;
//  * a bounded wait on a ready flag that records ERR_FLAG_TIMEOUT instead of
//    spinning forever;
//  * the NVLink bandwidth probe: a timed push of N bytes into a peer buffer,
//    with start/end taken from %globaltimer on the device (no host clock).
//
// Raw transfers use the reference's raw layout per layer,
// [2, nblocks, block_size, H, D] (kvserve_v1/utils/kv_utils.py:59-80).
#include "common.cuh"
#include "kvs_types.h"

namespace kvs {

// Copies `nblocks` blocks of both planes between a paged cache and a
// contiguous [2, nblocks, block_elems] buffer. dir 0: paged -> flat (gather),
// dir 1: flat -> paged (scatter).  grid (nblocks, 2), block 256.
__global__ void __launch_bounds__(256) k_block_copy(PagedKV kv, const int32_t* __restrict__ blocks,
                                                    int nblocks, long long block_elems,
                                                    uint8_t* flat, int dir, uint32_t* counter,
                                                    uint32_t* flag, uint32_t flag_value) {
  const int b = blockIdx.x, plane = blockIdx.y;
  const long long bytes = block_elems * 2;
  uint8_t* paged = const_cast<uint8_t*>(reinterpret_cast<const uint8_t*>(kv.base)) +
                   (static_cast<long long>(blocks[b]) * kv.block_stride + plane * kv.kv_stride) * 2;
  uint8_t* lin = flat + (static_cast<long long>(plane) * nblocks + b) * bytes;
  const uint4* s = reinterpret_cast<const uint4*>(dir == 0 ? paged : lin);
  uint4* d = reinterpret_cast<uint4*>(dir == 0 ? lin : paged);
  for (long long i = threadIdx.x; i < bytes / 16; i += blockDim.x) d[i] = s[i];
  if (counter != nullptr) {
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
      const uint32_t done = atomicAdd(counter, 1u);
      if (done == gridDim.x * gridDim.y - 1) {
        __threadfence_system();
        st_release_sys(flag, flag_value);
        *counter = 0;
      }
    }
  }
}

// Vectorised copy of `bytes` (multiple of 16) with an optional flag.
__global__ void __launch_bounds__(256) k_copy16(const uint4* __restrict__ src, uint4* dst,
                                                long long n16, uint32_t* counter, uint32_t* flag,
                                                uint32_t flag_value) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n16;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    dst[i] = src[i];
  if (counter != nullptr) {
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
      const uint32_t done = atomicAdd(counter, 1u);
      if (done == gridDim.x - 1) {
        __threadfence_system();
        st_release_sys(flag, flag_value);
        *counter = 0;
      }
    }
  }
}

// Gather-copy of several byte ranges (any sizes and 16-byte aligned
// destinations) in one launch: grid.y = segment.  The last CTA to finish
// publishes `flag_value` into `flag` after a system-scope fence, so a
// consumer on another GPU that observes the flag sees every segment.
struct CopySeg {
  const uint8_t* src;
  uint8_t* dst;
  long long bytes;
};

__global__ void __launch_bounds__(256) k_copy_segments(const CopySeg* __restrict__ segs,
                                                       uint32_t* counter, uint32_t* flag,
                                                       uint32_t flag_value) {
  const CopySeg sg = segs[blockIdx.y];
  const bool aligned = ((reinterpret_cast<uintptr_t>(sg.src) | reinterpret_cast<uintptr_t>(sg.dst)) & 15) == 0;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long tid = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (aligned) {
    const long long n16 = sg.bytes / 16;
    for (long long i = tid; i < n16; i += stride)
      reinterpret_cast<uint4*>(sg.dst)[i] = reinterpret_cast<const uint4*>(sg.src)[i];
    for (long long i = n16 * 16 + tid; i < sg.bytes; i += stride) sg.dst[i] = sg.src[i];
  } else {
    for (long long i = tid; i < sg.bytes; i += stride) sg.dst[i] = sg.src[i];
  }
  __threadfence_system();
  if (counter != nullptr) {
    __syncthreads();
    if (threadIdx.x == 0) {
      const uint32_t done = atomicAdd(counter, 1u);
      if (done == gridDim.x * gridDim.y - 1) {
        __threadfence_system();
        st_release_sys(flag, flag_value);
        *counter = 0;
      }
    }
  }
}

// Wait (bounded) until *flag == expected.  One thread spins; on timeout
// the error word records ERR_FLAG_TIMEOUT and the kernel returns.
__global__ void k_wait_flag(const uint32_t* flag, uint32_t expected, uint64_t timeout_ns,
                            uint32_t* err, uint64_t* waited_ns) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (ld_acquire_sys(flag) == expected) break;
    if (globaltimer() - t0 > timeout_ns) {
      record_error(err, ERR_FLAG_TIMEOUT);
      break;
    }
    __nanosleep(200);
  }
  if (waited_ns) *waited_ns = globaltimer() - t0;
}

__global__ void k_set_flag(uint32_t* flag, uint32_t value) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    __threadfence_system();
    st_release_sys(flag, value);
  }
}

// Timed push: every CTA stamps its first/last %globaltimer; the result is
// [min start, max end] in stamps[0..1] (initialised by the host to
// (UINT64_MAX, 0)).
__global__ void __launch_bounds__(512) k_probe_push(const uint4* __restrict__ src, uint4* dst,
                                                    long long n16, unsigned long long* stamps) {
  __shared__ unsigned long long t_start;
  if (threadIdx.x == 0) t_start = globaltimer();
  __syncthreads();
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n16;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    dst[i] = src[i];
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    atomicMin(&stamps[0], t_start);
    atomicMax(&stamps[1], static_cast<unsigned long long>(globaltimer()));
  }
}


// Message checksum: over the bytes b_p of a message (p = offset inside the
// message), S1 = sum_p b_p * 2^(8*(p%4)) and S2 = sum_p (p/4 + 1) * b_p *
// 2^(8*(p%4)), both mod 2^64 -- i.e. the plain and the position-weighted sums
// of the message's little-endian 32-bit words.  Integer sums are
// order-independent, so any grid computes the same value.  A segment is
// (src, message offset, bytes).
struct CkSeg {
  const uint8_t* src;
  long long off;
  long long bytes;
};

KVS_DEV void ck_byte(uint8_t b, long long p, unsigned long long& s1, unsigned long long& s2) {
  const unsigned long long v = static_cast<unsigned long long>(b) << (8 * (p & 3));
  s1 += v;
  s2 += static_cast<unsigned long long>((p >> 2) + 1) * v;
}

__global__ void __launch_bounds__(256) k_checksum(const CkSeg* __restrict__ segs,
                                                  unsigned long long* out) {
  const CkSeg sg = segs[blockIdx.y];
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long tid = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  unsigned long long s1 = 0, s2 = 0;
  if (((reinterpret_cast<uintptr_t>(sg.src) | static_cast<uintptr_t>(sg.off)) & 15) == 0) {
    const long long n16 = sg.bytes / 16;
    for (long long i = tid; i < n16; i += stride) {
      const uint4 v = reinterpret_cast<const uint4*>(sg.src)[i];
      const unsigned long long w = static_cast<unsigned long long>((sg.off >> 2) + 4 * i + 1);
      s1 += static_cast<unsigned long long>(v.x) + v.y + v.z + v.w;
      s2 += w * v.x + (w + 1) * v.y + (w + 2) * v.z + (w + 3) * v.w;
    }
    for (long long i = n16 * 16 + tid; i < sg.bytes; i += stride) ck_byte(sg.src[i], sg.off + i, s1, s2);
  } else {
    for (long long i = tid; i < sg.bytes; i += stride) ck_byte(sg.src[i], sg.off + i, s1, s2);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    s1 += __shfl_xor_sync(0xFFFFFFFFu, s1, o);
    s2 += __shfl_xor_sync(0xFFFFFFFFu, s2, o);
  }
  if ((threadIdx.x & 31) == 0 && (s1 | s2)) {
    atomicAdd(out, s1);
    atomicAdd(out + 1, s2);
  }
}

__global__ void k_zero2(unsigned long long* p) {
  if (threadIdx.x < 2) p[threadIdx.x] = 0;
}

__global__ void k_checksum_compare(const unsigned long long* got,
                                   const unsigned long long* expected, uint32_t* err) {
  if (threadIdx.x == 0 && (got[0] != expected[0] || got[1] != expected[1]))
    record_error(err, ERR_CORRUPT);
}

}  // namespace kvs

using namespace kvs;

extern "C" {

int kvs_block_copy(const PagedKV* kv, const int32_t* blocks, int nblocks, long long block_elems,
                   uint8_t* flat, int dir, uint32_t* counter, uint32_t* flag, uint32_t flag_value,
                   void* stream) {
  if (nblocks <= 0) return 0;
  if ((block_elems * 2) % 16 != 0) return -2;
  k_block_copy<<<dim3(nblocks, 2), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      *kv, blocks, nblocks, block_elems, flat, dir, counter, flag, flag_value);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int kvs_copy16(const void* src, void* dst, long long bytes, uint32_t* counter, uint32_t* flag,
               uint32_t flag_value, int max_blocks, void* stream) {
  if (bytes % 16 != 0) return -2;
  const long long n16 = bytes / 16;
  long long blocks = (n16 + 255) / 256;
  if (blocks > max_blocks) blocks = max_blocks;
  if (blocks < 1) blocks = 1;
  k_copy16<<<static_cast<int>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), static_cast<uint4*>(dst), n16, counter, flag, flag_value);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// segs: device array of n CopySeg {src, dst, bytes}.

// Checksum of `n` segments (device array of CkSeg) into out[2] (device).
int kvs_checksum(const void* segs, int n, unsigned long long* out, int blocks_per_seg,
                 void* stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  k_zero2<<<1, 32, 0, s>>>(out);
  if (n > 0)
    k_checksum<<<dim3(blocks_per_seg, n), 256, 0, s>>>(static_cast<const CkSeg*>(segs), out);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// Recompute the checksum of `segs` into scratch[2] and record ERR_CORRUPT in
// *err when it differs from expected[2] (all device memory; no host wait).
int kvs_checksum_verify(const void* segs, int n, const unsigned long long* expected,
                        unsigned long long* scratch, uint32_t* err, int blocks_per_seg,
                        void* stream) {
  if (int rc = kvs_checksum(segs, n, scratch, blocks_per_seg, stream)) return rc;
  k_checksum_compare<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(scratch, expected, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int kvs_copy_segments(const void* segs, int n, int blocks_per_seg, uint32_t* counter,
                      uint32_t* flag, uint32_t flag_value, void* stream) {
  if (n <= 0) return 0;
  k_copy_segments<<<dim3(blocks_per_seg, n), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const CopySeg*>(segs), counter, flag, flag_value);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int kvs_wait_flag(const uint32_t* flag, uint32_t expected, uint64_t timeout_ns, uint32_t* err,
                  uint64_t* waited_ns, void* stream) {
  k_wait_flag<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(flag, expected, timeout_ns, err,
                                                               waited_ns);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int kvs_set_flag(uint32_t* flag, uint32_t value, void* stream) {
  k_set_flag<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(flag, value);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int kvs_probe_push(const void* src, void* dst, long long bytes, unsigned long long* stamps,
                   int blocks, void* stream) {
  if (bytes % 16 != 0) return -2;
  k_probe_push<<<blocks, 512, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), static_cast<uint4*>(dst), bytes / 16, stamps);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // extern "C"
