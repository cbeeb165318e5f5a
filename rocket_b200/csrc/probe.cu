// Device clock stamps and memory-bandwidth microbenchmark kernels.
//
//   stamp_kernel    writes %globaltimer (ns) into a slot: bracketing a region on the
//                   launching stream gives its device-side duration without events
//                   (multi-GPU timing takes the max of these over ranks)
//   bw_copy / bw_read / bw_triad / bw_gather
//                   STREAM-style kernels: 16-byte vector accesses, grid-stride loops
//                   over a grid of (SMs x resident blocks); the gather reads 64-byte
//                   rows at random indices (the access pattern of paged KV / expert
//                   row gathers)
//
// Counterparts of the reference's hardware microbenchmarks (scripts/hardware/mem-bw.cu,
// mem-bw-sweep.cu, mem-gather.cu) and its device timing notes; written for sm_100a.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"

namespace rkt {

namespace {

__global__ void stamp_kernel(unsigned long long* out, int slot) {
  if (threadIdx.x == 0) out[slot] = globaltimer();
}

__global__ void bw_copy_kernel(const uint4* __restrict__ a, uint4* __restrict__ b, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    b[i] = a[i];
}

__global__ void bw_read_kernel(const uint4* __restrict__ a, size_t n, unsigned* __restrict__ sink) {
  unsigned acc = 0;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const uint4 v = a[i];
    acc ^= v.x ^ v.y ^ v.z ^ v.w;
  }
  if (acc == 0x9e3779b9u) sink[0] = acc;  // keeps the loads live; practically never taken
}

__global__ void bw_triad_kernel(float4* __restrict__ a, const float4* __restrict__ b, const float4* __restrict__ c,
                                float s, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float4 x = b[i], y = c[i];
    a[i] = make_float4(x.x + s * y.x, x.y + s * y.y, x.z + s * y.z, x.w + s * y.w);
  }
}

// 64-byte rows: 4 threads per row, one uint4 each
__global__ void bw_gather_kernel(const uint4* __restrict__ src, const int* __restrict__ idx, uint4* __restrict__ dst,
                                 size_t rows) {
  for (size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x; t < rows * 4; t += (size_t)gridDim.x * blockDim.x) {
    const size_t r = t >> 2, q = t & 3;
    dst[t] = src[(size_t)idx[r] * 4 + q];
  }
}

int grid_for(int threads) {
  int dev = 0, sms = 148, per = 1;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int maxthr = 2048;
  cudaDeviceGetAttribute(&maxthr, cudaDevAttrMaxThreadsPerMultiProcessor, dev);
  per = maxthr / threads;
  return sms * (per > 0 ? per : 1);
}

}  // namespace

int launch_stamp(unsigned long long* out, int slot, cudaStream_t st) {
  stamp_kernel<<<1, 32, 0, st>>>(out, slot);
  return (int)cudaGetLastError();
}

int launch_bw(int kind, void* a, const void* b, const void* c, const int* idx, size_t bytes, cudaStream_t st) {
  const int threads = 512;
  const int grid = grid_for(threads);
  switch (kind) {
    case 0: bw_copy_kernel<<<grid, threads, 0, st>>>((const uint4*)b, (uint4*)a, bytes / 16); break;
    case 1: bw_read_kernel<<<grid, threads, 0, st>>>((const uint4*)b, bytes / 16, (unsigned*)a); break;
    case 2: bw_triad_kernel<<<grid, threads, 0, st>>>((float4*)a, (const float4*)b, (const float4*)c, 3.f, bytes / 16);
      break;
    case 3: bw_gather_kernel<<<grid, threads, 0, st>>>((const uint4*)b, idx, (uint4*)a, bytes / 64); break;
    default: return -2;
  }
  return (int)cudaGetLastError();
}

}  // namespace rkt
