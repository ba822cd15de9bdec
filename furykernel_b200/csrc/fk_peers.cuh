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

// A flag store after the caller's own system-scope fence: relaxed, so that
// a thread storing to several ranks does not pay one release fence a rank.
__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// Every thread of every block of the producer calls this after its last
// write into the peers' regions; `wrote` says whether this thread wrote
// (only writers need the system-scope fence before the block's barrier).
__device__ __forceinline__ void peers_signal(const FkPeers& P, uint32_t buf, bool wrote = true) {
  if (wrote) __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    char* me = P.base[P.rank];
    const uint32_t done = atomicAdd(xcounter(me) + buf, 1u);
    if (done == gridDim.x - 1) {
      xcounter(me)[buf] = 0;
      const uint32_t e = xepoch(me)[buf] + 1;
      xepoch(me)[buf] = e;
      fence_acq_rel_sys();  // one fence, then the flags (a release each would fence again)
      for (uint32_t q = 0; q < P.world; ++q) st_relaxed_sys(xflags(P.base[q]) + buf * FK_MAX_PEERS + P.rank, e);
    }
  }
}

// The producer's broadcast of a partial it has written into its own slot
// of its own region (m_n floats, 16-byte aligned): every block of the grid
// calls this once its part of the slot is written. Blocks fence at GPU
// scope and count themselves in; the last one in copies the whole slot
// into this rank's slot of every other rank's region with 128-bit stores,
// fences at system scope and releases the buffer's next epoch into every
// rank's flags. One block, not every writer, pays for system scope.
__device__ __forceinline__ void peers_broadcast(const FkPeers& P, uint32_t buf, uint32_t count, bool wrote) {
  __shared__ uint32_t last;
  if (wrote) __threadfence();
  __syncthreads();
  char* me = P.base[P.rank];
  if (threadIdx.x == 0) last = atomicAdd(xcounter(me) + buf, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  const float4* src = reinterpret_cast<const float4*>(xdata(me, buf, P.rank));
  const uint32_t n4 = (count + 3) / 4;
  for (uint32_t q = 0; q < P.world; ++q) {
    if (q == P.rank) continue;
    float4* dst = reinterpret_cast<float4*>(xdata(P.base[q], buf, P.rank));
    for (uint32_t i = threadIdx.x; i < n4; i += blockDim.x) dst[i] = __ldcg(src + i);
  }
  fence_acq_rel_sys();
  __syncthreads();
  // Thread q stores rank q's flag: one fence above, no fence a flag.
  const uint32_t e = xepoch(me)[buf] + 1;
  if (threadIdx.x < P.world) {
    fence_acq_rel_sys();  // orders the block's copies (seen through the barrier) before the flag
    st_relaxed_sys(xflags(P.base[threadIdx.x]) + buf * FK_MAX_PEERS + P.rank, e);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    xcounter(me)[buf] = 0;
    xepoch(me)[buf] = e;
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
