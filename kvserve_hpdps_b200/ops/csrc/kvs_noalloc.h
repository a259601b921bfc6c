// No-allocation entry point of the rANS encoder.
//
// This entry point has no counterpart in the reference implementation; it is
// an addition of this library.
//
// Who needs it: callers that cannot allocate device memory at the time they
// encode.  A serving engine typically reserves most of the GPU's memory up
// front for its KV cache (vLLM takes a fixed fraction at start-up), so a
// cudaMalloc issued from inside one of its workers can fail, or stall the
// worker while the driver searches for free memory; embedders that run under
// a fixed memory budget, or that hand this library pointers from their own
// pool and have no allocator to offer it, are in the same position.  The
// regular entry point (kvs_rans_encode) needs caller-provided staging and
// size buffers; this variant needs none.
//
// How: its scratch lives in file-scope __device__ arrays of fixed size
// (about 34 MB of staging plus 16 KB of record descriptors).  Every GPU that
// loads the library holds that memory until the process exits.  The caller
// still passes the input and the output buffers.
//
// Contract:
//  * `in` and `out` must be 16-byte aligned (KVS_NOALLOC_UNALIGNED otherwise);
//  * n must be between 1 and kvs_rans_encode_noalloc_max_symbols() bytes;
//    larger inputs are rejected with KVS_NOALLOC_TOO_LARGE before anything
//    is launched, and out_capacity must be at least kvs_rans_max_bytes(n,
//    32768);
//  * the stream is byte-identical to the one kvs_rans_encode writes for the
//    same input with 32768-symbol chunks; its total size is stored in the
//    stream header (bytes 24..31, little endian);
//  * the first call in a CUDA context looks up the device address of the
//    scratch arrays with that context current (the arrays belong to the
//    library's module, loaded once per context; the lookup is kept per device
//    and redone when the current context differs, e.g. after cudaDeviceReset
//    or under a driver-API context of the caller's); make that first call
//    before any CUDA stream capture in the context;
//  * a launch error of this call is returned as KVS_NOALLOC_LAUNCH; an error
//    left pending by unrelated earlier work is neither reported nor cleared;
//  * all calls share one scratch area per device and it keeps the previous
//    call's contents (every byte the encoder reads is written earlier in the
//    same call, so nothing needs clearing); calls whose work overlaps on the
//    GPU race on the scratch, so callers must order them (same stream, or
//    events between streams).
#pragma once

#include <cstdint>

#define KVS_NOALLOC_OK 0
#define KVS_NOALLOC_EMPTY (-2)
#define KVS_NOALLOC_TOO_LARGE (-3)
#define KVS_NOALLOC_OUT_TOO_SMALL (-4)
#define KVS_NOALLOC_NO_DEVICE (-5)
#define KVS_NOALLOC_SYMBOL (-6)
#define KVS_NOALLOC_LAUNCH (-7)
#define KVS_NOALLOC_UNALIGNED (-8)

extern "C" {

// Largest input (bytes) the no-allocation encoder accepts.
uint64_t kvs_rans_encode_noalloc_max_symbols(void);

// Encode n bytes at `in` (device) into `out` (device, capacity
// out_capacity) on `stream`; returns KVS_NOALLOC_OK or a negative code.
int kvs_rans_encode_noalloc(const uint8_t* in, uint64_t n, uint8_t* out, uint64_t out_capacity,
                            void* stream);

// Human-readable text for a return code of kvs_rans_encode_noalloc.
const char* kvs_noalloc_strerror(int code);

}  // extern "C"
