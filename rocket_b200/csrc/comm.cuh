// Device-side primitives for collectives fused into compute kernels over
// NVLink peer memory (CUDA IPC mappings of every rank's symmetric buffer).
//
// Signalling uses epochs instead of resettable flags so it works under CUDA
// graph replay: every signalling site s has a local launch counter; a producer
// launch publishes epoch e = ++counter into flags[s][my_rank] on each
// destination with a system-scope release store after its data stores, and a
// consumer launch waits (bounded, acquire) until flags[s][src] >= its own
// ++counter for every source.  All ranks launch the same sequence of sites,
// so the epochs agree.  Waits give up after kWaitLimitNs, OR kErrPeerTimeout
// into the status word and return false; nothing traps.
//
// Only plain ld/st (and atomics) touch peer memory here: no TMA, and never a
// multicast load, reads another GPU's memory.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

#include "comm_types.h"

namespace rkt {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t* flag_ptr(const PeerPtrs& pp, int rank, int site, int src) {
  return reinterpret_cast<uint32_t*>(pp.base[rank] + pp.flag_off) + site * kMaxRanks + src;
}

// Counter layout (this rank's local int array, zeroed once):
//   [0, kSites)            producer epochs
//   [kSites, 2*kSites)     consumer epochs
//   [2*kSites, 3*kSites)   last-CTA arrival counters
__device__ __forceinline__ uint32_t consumer_epoch(const PeerPtrs& pp, int site) {
  return pp.counters[kSites + site] + 1;
}
__device__ __forceinline__ void consumer_commit(const PeerPtrs& pp, int site, uint32_t e) {
  pp.counters[kSites + site] = e;
}
__device__ __forceinline__ unsigned int* arrival_counter(const PeerPtrs& pp, int site) {
  return pp.counters + 2 * kSites + site;
}

// Called by exactly one thread of the launch after all of its peer stores are
// globally visible (see last_block_done): publish the next epoch of `site`
// to every rank in `dst_mask`.
__device__ __forceinline__ void signal_peers(const PeerPtrs& pp, int site, uint32_t dst_mask = 0xffffffffu) {
  const uint32_t e = pp.counters[site] + 1;
  pp.counters[site] = e;
  __threadfence_system();
  for (int r = 0; r < pp.world; ++r)
    if (dst_mask >> r & 1) st_release_sys(flag_ptr(pp, r, site, pp.rank), e);
}

// One thread: wait until every source in `src_mask` has published epoch >= e of
// `site`.  Returns false (and sets the error bit) on timeout.  Every CTA of a
// consumer launch may wait on the same epoch; the launch's last CTA then calls
// consumer_commit once.
__device__ __forceinline__ bool wait_peers(const PeerPtrs& pp, int site, uint32_t e, int* err,
                                           uint32_t src_mask = 0xffffffffu) {
  const unsigned long long t0 = globaltimer();
  for (int r = 0; r < pp.world; ++r) {
    if (!(src_mask >> r & 1)) continue;
    const uint32_t* f = flag_ptr(pp, pp.rank, site, r);
    while ((int)(ld_acquire_sys(f) - e) < 0) {
      if (globaltimer() - t0 > kWaitLimitNs) {
        if (err) atomicOr(err, kErrPeerTimeout);
        return false;
      }
    }
  }
  // peers' generic-proxy stores must be visible to this CTA's TMA (async proxy) reads too
  asm volatile("fence.proxy.async.global;" ::: "memory");
  return true;
}

// Grid-wide completion: every CTA calls this once after its stores (all threads
// of the CTA); exactly one CTA -- the last to arrive -- gets true.  `ctr` is a
// zero-initialised global counter that the last CTA resets.
__device__ __forceinline__ bool last_block_done(unsigned int* ctr) {
  // all threads of the CTA call this
  __shared__ bool last;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int prev = atomicAdd(ctr, 1u);
    last = prev == gridDim.x * gridDim.y * gridDim.z - 1;
    if (last) {
      __threadfence();
      *ctr = 0;
    }
  }
  __syncthreads();
  return last;
}

}  // namespace rkt
