// Allocation-free C entry point for KV-cache decode attention.
//
// This entry point has no counterpart in the reference implementation; it is
// an addition of this library.
//
// Who needs it: callers that cannot allocate device memory while they decode.
// Examples are C or ctypes hosts that load this library without PyTorch (so
// there is no caching allocator to borrow from), and serving processes that
// reserve their whole memory budget at start-up and must not grow it per
// request, or that cannot afford the device-wide synchronisation that a
// cudaMalloc / cudaFree pair implies in the middle of a latency-sensitive
// token loop.  The regular `decode_attn` binding takes its split-K scratch from
// PyTorch's allocator on every call; this one uses a fixed scratch array
// compiled into the library instead.
//
// Contract:
//   * The caller passes device pointers for every input and for the output:
//       q        [B, Sq, Hq, D]   bf16, contiguous
//       k_cache  [B, Smax, Hk, D] bf16, contiguous
//       v_cache  [B, Smax, Hk, D] bf16, contiguous
//       cache_len[B] int32  valid cache rows per sequence (new rows included)
//       q_start  [B] int32  absolute position of query row 0
//       out      [B, Sq, Hq, D]   bf16
//     with D in {64, 128} and (Hq / Hk) * Sq <= 32.
//   * Scratch lives in one file-scope device array of
//     NQ_DECODE_NOALLOC_SCRATCH_BYTES bytes (8 MiB).  Every GPU that loads
//     the library holds that array until the process exits.  A call needs
//     B * Hq * Sq * splits * (D + 2) * 4 bytes of it, where splits is the
//     split-K factor the library picks from the cache length (at most
//     ceil(Smax / 256)); calls that would need more are rejected with an
//     error, never truncated.
//   * The first call on a device (with that device current) looks up the
//     array's device address with cudaGetSymbolAddress and caches it; make
//     that first call before any stream capture begins on the device.
//   * All calls share the one array, and each call overwrites what the last
//     one left there (every scratch element a call reads was written earlier
//     in the same call, so nothing has to start at zero).  Calls whose kernels
//     overlap on the GPU -- on different streams without ordering between
//     them, or from different host threads -- race on the scratch and corrupt
//     each other's results; serialise them.
//   * Nothing is allocated or freed: no cudaMalloc, cudaFree or allocating
//     library routine is called on any path.
//
// Returns 0 on success.  On failure returns a non-zero code and, when `err`
// is non-null, writes a NUL-terminated message of at most err_len bytes.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

#define NQ_DECODE_NOALLOC_SCRATCH_BYTES (8u << 20)

#ifdef __cplusplus
extern "C" {
#endif

enum {
  NQ_NOALLOC_OK = 0,
  NQ_NOALLOC_BAD_ARG = 1,
  NQ_NOALLOC_TOO_LARGE = 2,
  NQ_NOALLOC_CUDA_ERROR = 3,
};

__attribute__((visibility("default"))) int nq_decode_attn_noalloc(
    const void* q, const void* k_cache, const void* v_cache, const int* cache_len,
    const int* q_start, void* out, int B, int Sq, int Hq, int Hk, int D, int Smax, float scale,
    cudaStream_t stream, char* err, int err_len);

#ifdef __cplusplus
}
#endif
