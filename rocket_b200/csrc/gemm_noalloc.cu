// Allocation-free entry point of the split-K bf16 GEMM.
//
// This entry point has no counterpart in the reference: it is an addition of
// this library for callers that cannot allocate device memory.
//
// Who needs it: code that must not call cudaMalloc / cudaFree (or any
// allocating library routine, torch's caching allocator included) at the point
// where it runs -- for example a host that hands this library a fixed memory
// budget and forbids growth after start-up, a plugin running inside another
// runtime whose allocator it does not own, or a latency-critical path where an
// allocation (and the device synchronisation cudaFree implies) is not allowed.
// The regular entry point (gemm_launch with splits > 1) needs a caller-provided
// fp32 workspace; this one takes its workspace from a fixed device array that
// is part of the library image instead.
//
// Contract:
//   rkt_gemm_bf16_splitk_noalloc(w, x, out, n, k, m, splits, status, stream)
//     out[m][n] (bf16) = x[m][k] (bf16) . w[n][k] (bf16)^T, fp32 accumulation,
//     K split `splits` ways; partial sums go to kNoAllocScratchFloats floats of
//     static device memory and are summed in a fixed order (deterministic).
//     `status` is a caller-owned device int (an output, like `out`): the kernel
//     ORs error bits into it (1 = a pipeline wait gave up after its bounded spin,
//     8 = tensor-memory allocation failed), so a device-side failure is reported
//     instead of dropped.  The caller zeroes it and reads it once the stream has
//     reached the call; the return code covers only what the host can check.
//   Limits: splits * m * n <= kNoAllocScratchFloats (4 MiB of fp32), n % 128 == 0,
//     k % 64 == 0, k / 64 >= splits; otherwise it returns an error code and
//     launches nothing.
//   Set-up: the first call on a device (with that device current) resolves the
//     scratch array's device address with cudaGetSymbolAddress and caches it per
//     device; call it once on every device before timing-critical use or stream
//     capture so that set-up does not happen there.
//   Sharing: every call on a device uses the same scratch.  Two calls whose
//     kernels overlap on the GPU (different streams without ordering) race on it;
//     order them on one stream or with events.  Every partial that the reduce
//     reads is written by the same call first, so no clearing is needed.
//   Memory: every GPU that loads this library holds the 4 MiB array until exit.
#include <cuda_runtime.h>
#include <stdint.h>

#include "gemm_noalloc.h"
#include "gemm_sm100.h"

namespace {

constexpr size_t kNoAllocScratchFloats = 1u << 20;  // 4 MiB of fp32 partial sums

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

constexpr int kMaxDevices = 64;
float* g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of the scratch array for the current device (resolved once).
int scratch_for_current_device(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= kMaxDevices) return -10;
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return (int)e;
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return 0;
}

}  // namespace

// Returns 0 on success; -2 for unsupported shapes or a null pointer; -5 when splits * m * n exceeds
// the static scratch (kNoAllocScratchFloats floats); a CUDA error code otherwise.
extern "C" __attribute__((visibility("default"))) int rkt_gemm_bf16_splitk_noalloc(
    const void* w, const void* x, void* out, int n, int k, int m, int splits, int* status, cudaStream_t stream) {
  if (!w || !x || !out || !status || n <= 0 || k <= 0 || m <= 0 || splits < 2) return -2;
  if (n % 128 || k % 64 || k / 64 < splits) return -2;
  if ((size_t)splits * (size_t)m * (size_t)n > kNoAllocScratchFloats) return -5;
  float* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc) return rc;
  rkt::GemmArgs p;
  p.nvf4 = 0;
  p.n_w = n;
  p.k = k;
  p.m_tokens = m;
  p.ldb_bytes = (uint64_t)k * 2;
  p.epi = rkt::EPI_STORE_BF16;
  p.out = out;
  p.ldo = n;
  p.splits = splits;
  p.ws = scratch;
  p.ws_rows = m;
  p.err = status;
  const int bn = m <= 32 ? 32 : (m <= 128 ? 128 : 256);
  const int grid_y = (m + bn - 1) / bn;
  return rkt::gemm_launch(p, w, x, m, grid_y, bn, stream);
}
