// Allocation-free entry point of the tcgen05 bf16 GEMM.
//
// This entry point has no counterpart in the reference (vectie/lunaflux has no
// GPU kernels of its own).  It exists for callers that cannot allocate device
// memory: code running inside a memory-pool-restricted host application or an
// embedding runtime that owns every device allocation, code that runs where a
// cudaMalloc would implicitly synchronise the device or fail under a strict
// memory cap, and plugins loaded into processes that forbid allocation after
// start-up.  Such a caller passes its own inputs and outputs; the split-K
// scratch the GEMM needs for skinny shapes lives in a fixed-size array that is
// part of the loaded library instead of being allocated per call.
//
// Scratch: a file-scope __device__ array of LF_GEMM_NOALLOC_SCRATCH_FLOATS
// floats (16 MiB).  Every GPU that loads the library holds this array until
// the process exits.  All calls on a device share it and it keeps the last
// call's contents; every element a call reads is first written by that same
// call, so nothing has to start at zero.  Calls whose execution overlaps on
// the GPU (concurrent streams, or graphs replayed concurrently) race on the
// scratch and produce wrong results: serialise them.
//
// Set-up: the first call on each device, made with that device current,
// resolves the scratch array's device address (cudaGetSymbolAddress) and sets
// the kernels' shared-memory limits.  Make that first call before any stream
// capture on that device.  A set-up that fails returns
// LF_NOALLOC_SETUP_FAILED and is retried by the next call.
//
// Semantics: D[M, N] = A[M, K] . B[N, K]^T with bf16 A/B (row strides lda,
// ldb in elements) and, by `epi`: 0 bf16 D, 1 fp32 D, 2 SwiGLU (B's rows are
// gate/up interleaved in groups of 32 rows; D is bf16 [M, N/2]).  Skinny
// shapes are split over K into fp32 slabs in the scratch array and summed by
// a second kernel, a different plan from the allocating entry point's (which
// reduces split partials in distributed shared memory): the two agree within
// bf16 rounding, not bitwise.
#pragma once
#include <stdint.h>

#define LF_GEMM_NOALLOC_SCRATCH_FLOATS (4u * 1024u * 1024u)

// Return codes.
#define LF_NOALLOC_OK 0
#define LF_NOALLOC_BAD_ARGUMENT 1     // shape, stride, alignment or epi not supported
#define LF_NOALLOC_TOO_LARGE 2        // the split-K plan needs more scratch than the array holds
#define LF_NOALLOC_SETUP_FAILED 3     // cudaGetSymbolAddress / attribute set-up failed
#define LF_NOALLOC_LAUNCH_FAILED 4    // a kernel launch reported an error

#ifdef __cplusplus
extern "C" {
#endif

// `stream` is a cudaStream_t (0 = the legacy default stream).  Returns one of
// the LF_NOALLOC_* codes; nothing is launched (and D is untouched) unless it
// returns LF_NOALLOC_OK or LF_NOALLOC_LAUNCH_FAILED.  Each launch's own return
// code decides LF_NOALLOC_LAUNCH_FAILED: errors left by the caller's earlier
// CUDA calls are neither reported nor cleared.
int lf_gemm_bf16_noalloc(const void* A, const void* B, void* D, int M, int N, int K, int64_t lda, int64_t ldb,
                         int64_t ldd, int epi, void* stream);

#ifdef __cplusplus
}
#endif
