// Allocation-free split-K bf16 GEMM: C entry point (implementation: gemm_noalloc.cu).
//
// No counterpart in the reference: this library adds it for callers that cannot
// allocate device memory where they call it (a host program that fixes the
// memory budget at start-up, a plugin running inside another runtime's
// allocator, or a path where cudaMalloc/cudaFree and their synchronisation are
// not allowed).  Its workspace is a 4 MiB static device array inside the
// library, so splits * m * n must not exceed 1,048,576 floats; larger requests
// return -5 and launch nothing.  The first call on a device resolves the
// array's address (make that first call before timing-critical use), all calls
// on a device share the array, and calls that overlap on the GPU race on it.
#pragma once
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

// out[m][n] = x[m][k] . w[n][k]^T (bf16 in/out, fp32 accumulation), K split
// `splits` ways (2 <= splits <= k/64), n % 128 == 0, k % 64 == 0.  `status` is a
// caller-owned device int that receives device-side error bits (1 = a bounded
// pipeline wait gave up, 8 = tensor-memory allocation failed); zero it before the
// call and read it after the stream reaches the call.
// Returns 0, -2 (bad shape or null pointer), -5 (exceeds the static scratch) or a
// CUDA error code.
int rkt_gemm_bf16_splitk_noalloc(const void* w, const void* x, void* out, int n, int k, int m, int splits,
                                 int* status, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
