// Device side of the tensor-parallel exchange (the region layout is in
// fk_kernels.h): a producer grid writes its partial rows into every rank's
// region, then its last block releases the buffer's next epoch into every
// rank's flags; a consumer waits, with a bound, until every rank's flag in
// its own region has reached its own epoch, then reads the partials locally.
#pragma once

#include "fk_common.cuh"
#include "fk_kernels.h"

namespace fk {

constexpr long long kPeerWaitCycles = 4000000000LL;  // ~2 s

__device__ __forceinline__ uint32_t* xflags(char* base) { return reinterpret_cast<uint32_t*>(base); }
__device__ __forceinline__ uint32_t* xepoch(char* base) { return reinterpret_cast<uint32_t*>(base + 128); }
__device__ __forceinline__ uint32_t* xcounter(char* base) { return reinterpret_cast<uint32_t*>(base + 160); }
__device__ __forceinline__ float* xdata(char* base, uint32_t buf, uint32_t src) {
  return reinterpret_cast<float*>(base + 256) + ((size_t)buf * FK_MAX_PEERS + src) * FK_XSLOT;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Every thread of every block of the producer calls this after its last
// write into the peers' regions.
__device__ __forceinline__ void peers_signal(const FkPeers& P, uint32_t buf) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    char* me = P.base[P.rank];
    const uint32_t done = atomicAdd(xcounter(me) + buf, 1u);
    if (done == gridDim.x - 1) {
      xcounter(me)[buf] = 0;
      const uint32_t e = xepoch(me)[buf] + 1;
      xepoch(me)[buf] = e;
      __threadfence_system();
      for (uint32_t q = 0; q < P.world; ++q) st_release_sys(xflags(P.base[q]) + buf * FK_MAX_PEERS + P.rank, e);
    }
  }
}

// Every thread of a consumer block calls this; thread 0 waits. False when
// a rank's signal did not come within the bound (recorded in *err).
__device__ __forceinline__ bool peers_wait(const FkPeers& P, uint32_t buf, int* err) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    char* me = P.base[P.rank];
    const uint32_t e = *reinterpret_cast<volatile uint32_t*>(xepoch(me) + buf);
    ok = 1;
    for (uint32_t q = 0; q < P.world && ok; ++q) {
      const long long t0 = clock64();
      while (ld_acquire_sys(xflags(me) + buf * FK_MAX_PEERS + q) < e) {
        if (clock64() - t0 > kPeerWaitCycles) {
          if (err) atomicCAS(err, 0, 10 + (int)buf);
          ok = 0;
          break;
        }
      }
    }
  }
  __syncthreads();
  return ok != 0;
}

}  // namespace fk
