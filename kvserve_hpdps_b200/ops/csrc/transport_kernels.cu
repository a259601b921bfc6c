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
                                                    uint32_t* flag, uint32_t flag_value,
                                                    uint32_t* err) {
  const int b = blockIdx.x, plane = blockIdx.y;
  const long long bytes = block_elems * 2;
  const int phys = blocks[b];
  if (static_cast<unsigned>(phys) < static_cast<unsigned>(kv.num_blocks)) {
    uint8_t* paged = const_cast<uint8_t*>(reinterpret_cast<const uint8_t*>(kv.base)) +
                     (static_cast<long long>(phys) * kv.block_stride + plane * kv.kv_stride) * 2;
    uint8_t* lin = flat + (static_cast<long long>(plane) * nblocks + b) * bytes;
    const uint4* s = reinterpret_cast<const uint4*>(dir == 0 ? paged : lin);
    uint4* d = reinterpret_cast<uint4*>(dir == 0 ? lin : paged);
    for (long long i = threadIdx.x; i < bytes / 16; i += blockDim.x) d[i] = s[i];
  } else if (threadIdx.x == 0) {
    record_error(err, ERR_BOUNDS);  // block id outside the cache: nothing copied
  }
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
// consumer on another GPU that observes the flag sees every segment.  With
// `ck` the copy also sums the message checksum of what it writes (segment
// bytes at message offset msg_off, as defined in common.cuh), and
// the last CTA stores the finished sums to `trailer` before the flag.
struct CopySeg {
  const uint8_t* src;
  uint8_t* dst;
  long long bytes;
  long long msg_off;  // message offset of dst[0] (checksum weights)
};

__global__ void __launch_bounds__(256) k_copy_segments(const CopySeg* __restrict__ segs,
                                                       uint32_t* counter, uint32_t* flag,
                                                       uint32_t flag_value, unsigned long long* ck,
                                                       unsigned long long* trailer) {
  const CopySeg sg = segs[blockIdx.y];
  const bool aligned = ((reinterpret_cast<uintptr_t>(sg.src) | reinterpret_cast<uintptr_t>(sg.dst) |
                         static_cast<uintptr_t>(sg.msg_off)) & 15) == 0;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long tid = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  unsigned long long s1 = 0, s2 = 0;
  if (aligned) {
    const long long n16 = sg.bytes / 16;
    for (long long i = tid; i < n16; i += stride) {
      const uint4 v = reinterpret_cast<const uint4*>(sg.src)[i];
      reinterpret_cast<uint4*>(sg.dst)[i] = v;
      if (ck != nullptr) ck_word4(v, sg.msg_off + 16 * i, s1, s2);
    }
    for (long long i = n16 * 16 + tid; i < sg.bytes; i += stride) {
      sg.dst[i] = sg.src[i];
      if (ck != nullptr) ck_byte(sg.src[i], sg.msg_off + i, s1, s2);
    }
  } else {
    for (long long i = tid; i < sg.bytes; i += stride) {
      sg.dst[i] = sg.src[i];
      if (ck != nullptr) ck_byte(sg.src[i], sg.msg_off + i, s1, s2);
    }
  }
  if (ck != nullptr) ck_flush(ck, s1, s2);
  __threadfence_system();
  if (counter != nullptr) {
    __syncthreads();
    if (threadIdx.x == 0)
      last_cta_publish(counter, gridDim.x * gridDim.y, ck, trailer, flag, flag_value);
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


// Segment of a message checksum (the definition is in common.cuh):
// (src, message offset, bytes); with `len_ptr` set the length is
// min(bytes, *len_ptr + len_add), read on the device (a coded stream whose
// size is recorded in its own header).
struct CkSeg {
  const uint8_t* src;
  long long off;
  long long bytes;
  const unsigned long long* len_ptr;
  long long len_add;
};

__global__ void __launch_bounds__(256) k_checksum(const CkSeg* __restrict__ segs,
                                                  unsigned long long* out) {
  const CkSeg sg = segs[blockIdx.y];
  long long bytes = sg.bytes;
  if (sg.len_ptr != nullptr) {
    const unsigned long long dyn = *sg.len_ptr + static_cast<unsigned long long>(sg.len_add);
    if (dyn < static_cast<unsigned long long>(bytes)) bytes = static_cast<long long>(dyn);
  }
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long tid = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  unsigned long long s1 = 0, s2 = 0;
  if (((reinterpret_cast<uintptr_t>(sg.src) | static_cast<uintptr_t>(sg.off)) & 15) == 0) {
    const long long n16 = bytes / 16;
    for (long long i = tid; i < n16; i += stride)
      ck_word4(reinterpret_cast<const uint4*>(sg.src)[i], sg.off + 16 * i, s1, s2);
    for (long long i = n16 * 16 + tid; i < bytes; i += stride) ck_byte(sg.src[i], sg.off + i, s1, s2);
  } else {
    for (long long i = tid; i < bytes; i += stride) ck_byte(sg.src[i], sg.off + i, s1, s2);
  }
  ck_flush(out, s1, s2);
}

// ------------------------------------------------------- raw paged transfer
// Uncompressed transfer of whole paged blocks for many (layer slot, block
// list) items in one launch.  The flat side holds the items back to back,
// item r at flat_off as [2][nblocks][block bytes] -- per layer, the
// reference's raw layout [2, nblocks, block_size, H, D]
// (kvserve_v1/utils/kv_utils.py:59-80); a request's L layer items in order
// form its stacked [L, 2, nblocks, ...] tensor.  dir 0 gathers paged -> flat
// (the flat side may be a peer GPU's receive ring: NVLink stores), dir 1
// scatters flat -> paged.  A unit is one (item, plane, block); CTAs stride
// over units.  Block ids outside a slot's cache record ERR_BOUNDS and the
// unit is skipped.  With `ck` the gather also sums the message checksum of
// the flat bytes (the definition of k_checksum, message offset = flat
// offset); with `flag` the last CTA stores the checksum to `trailer`, fences
// at system scope and publishes `flag_value`.
struct RawItem {
  long long bt_off;    // first block-table entry of the item
  long long flat_off;  // byte offset of the item in the flat buffer
  int slot;            // index into kvs[]
  int nblocks;
};

struct RawLaunch {
  const PagedKV* kvs;
  const RawItem* items;
  const long long* unit_prefix;  // [n_items + 1] units before item r
  const int32_t* block_table;
  uint8_t* flat;
  uint32_t* err;
  unsigned long long* ck;       // [2] checksum accumulators or null
  unsigned long long* trailer;  // [2] checksum destination (may be peer memory) or null
  uint32_t* counter;            // completion counter (zero before the launch) or null
  uint32_t* flag;
  long long n_units;
  int n_items;
  int dir;
  int block_bytes;
  int elem_bytes;
  uint32_t flag_value;
  int pad_;
};

__global__ void __launch_bounds__(256) k_paged_raw(const RawLaunch a) {
  unsigned long long s1 = 0, s2 = 0;
  const int n16 = a.block_bytes >> 4;
  for (long long u = blockIdx.x; u < a.n_units; u += gridDim.x) {
    int lo = 0, hi = a.n_items - 1;  // last item whose first unit is <= u
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (a.unit_prefix[mid] <= u) lo = mid; else hi = mid - 1;
    }
    const RawItem it = a.items[lo];
    const int local = static_cast<int>(u - a.unit_prefix[lo]);
    const int plane = local >= it.nblocks ? 1 : 0;
    const int b = local - plane * it.nblocks;
    const PagedKV kv = a.kvs[it.slot];
    const int phys = a.block_table[it.bt_off + b];
    if (static_cast<unsigned>(phys) >= static_cast<unsigned>(kv.num_blocks)) {
      if (threadIdx.x == 0) record_error(a.err, ERR_BOUNDS);
      continue;
    }
    uint8_t* paged = const_cast<uint8_t*>(reinterpret_cast<const uint8_t*>(kv.base)) +
                     (static_cast<long long>(phys) * kv.block_stride + plane * kv.kv_stride) *
                         a.elem_bytes;
    const long long foff = it.flat_off + static_cast<long long>(local) * a.block_bytes;
    uint8_t* lin = a.flat + foff;
    const uint4* src = reinterpret_cast<const uint4*>(a.dir == 0 ? paged : lin);
    uint4* dst = reinterpret_cast<uint4*>(a.dir == 0 ? lin : paged);
    for (int i0 = threadIdx.x; i0 < n16; i0 += 4 * blockDim.x) {
      uint4 v[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int i = i0 + k * blockDim.x;
        if (i < n16) v[k] = __ldcs(src + i);  // read once: do not keep in L2
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int i = i0 + k * blockDim.x;
        if (i < n16) {
          dst[i] = v[k];
          if (a.ck != nullptr) ck_word4(v[k], foff + 16ll * i, s1, s2);
        }
      }
    }
  }
  if (a.ck != nullptr) ck_flush(a.ck, s1, s2);
  if (a.counter != nullptr) {
    __threadfence_system();  // this thread's stores (peer ones included) and sums first
    __syncthreads();
    if (threadIdx.x == 0)
      last_cta_publish(a.counter, gridDim.x, a.ck, a.trailer, a.flag, a.flag_value);
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
                   uint32_t* err, void* stream) {
  if (nblocks <= 0) return 0;
  if ((block_elems * 2) % 16 != 0) return -2;
  k_block_copy<<<dim3(nblocks, 2), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      *kv, blocks, nblocks, block_elems, flat, dir, counter, flag, flag_value, err);
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

// segs: device array of n CopySeg {src, dst, bytes, msg_off}.  With `ck`
// (int64[2] accumulators, zeroed by the caller) the copy adds the checksum
// of the written bytes; `trailer` then receives the finished sums from the
// last CTA before it publishes the flag.
int kvs_copy_segments(const void* segs, int n, int blocks_per_seg, uint32_t* counter,
                      uint32_t* flag, uint32_t flag_value, unsigned long long* ck,
                      unsigned long long* trailer, void* stream) {
  if (n <= 0) return 0;
  k_copy_segments<<<dim3(blocks_per_seg, n), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const CopySeg*>(segs), counter, flag, flag_value, ck, trailer);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// Zero two int64 accumulators (checksum) on the stream.
int kvs_zero2(unsigned long long* p, void* stream) {
  k_zero2<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(p);
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

int kvs_raw_launch_size() { return static_cast<int>(sizeof(RawLaunch)); }
int kvs_raw_item_size() { return static_cast<int>(sizeof(RawItem)); }

// Raw paged transfer (see k_paged_raw).  Zeroes the checksum accumulators
// first when `ck` is set.  Grid: min(units, max_ctas), at least one CTA so
// that a requested flag is published even for an empty transfer.
int kvs_paged_raw(const RawLaunch* a, int max_ctas, void* stream) {
  if (a->block_bytes <= 0 || a->block_bytes % 16 != 0 || a->n_items <= 0) return -2;
  if ((reinterpret_cast<uintptr_t>(a->flat) & 15) != 0) return -2;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a->ck != nullptr) k_zero2<<<1, 32, 0, s>>>(a->ck);
  long long grid = a->n_units < max_ctas ? a->n_units : max_ctas;
  if (grid < 1) grid = 1;
  k_paged_raw<<<static_cast<int>(grid), 256, 0, s>>>(*a);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // extern "C"
