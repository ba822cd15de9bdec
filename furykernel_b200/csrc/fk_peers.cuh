// Device side of the tensor-parallel exchange (the region layout is in
// fk_kernels.h). Buffers 0 and 1 (the row-parallel partials) use counted
// rows: producer blocks write their rows into every rank's region and add
// the rows to that rank's count for them, a consumer waits until every
// rank's count reaches the rows of all uses so far. Buffer 2 (the greedy
// candidates) uses epochs: the producer's last block releases the buffer's
// next epoch into every rank's flags, a consumer waits for its own epoch.
// Every wait is bounded and records why it gave up.
#pragma once

#include "fk_common.cuh"
#include "fk_kernels.h"

namespace fk {

// A wait's bound when the context gives none: about 2 s at the B200's clock.
constexpr long long kPeerWaitCycles = 4000000000LL;
__device__ __forceinline__ long long wait_bound(const FkPeers& P) {
  return P.wait_cycles > 0 ? P.wait_cycles : kPeerWaitCycles;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// With statistics on, the time a block's wait took, added to the context's
// totals (nanoseconds, and one wait).
__device__ __forceinline__ void wait_stats_add(const FkPeers& P, unsigned long long t0) {
  if (P.stats) {
    atomicAdd(P.stats, global_ns() - t0);
    atomicAdd(P.stats + 1, 1ull);
  }
}

__device__ __forceinline__ uint32_t* xflags(char* base) { return reinterpret_cast<uint32_t*>(base); }
__device__ __forceinline__ uint32_t* xepoch(char* base) { return reinterpret_cast<uint32_t*>(base + 128); }
__device__ __forceinline__ uint32_t* xcounter(char* base) { return reinterpret_cast<uint32_t*>(base + 160); }
__device__ __forceinline__ float* xdata(char* base, uint32_t buf, uint32_t src) {
  return reinterpret_cast<float*>(base + 256) + ((size_t)buf * FK_MAX_PEERS + src) * FK_XSLOT;
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

// The counted exchange of the row-parallel partials (buffers 0 and 1): a
// buffer's flag word for rank q counts the rows rank q has written into its
// slot of this region, all uses of the buffer together (u32, compared
// modulo 2^32). Every producer block writes its run of rows straight into
// every rank's slot, then counts itself in at GPU scope: thread 0's
// acquire-release add on this rank's block counter, after the block's
// barrier (so it releases every thread's writes). The last block to count
// in has acquired them all; it bumps this rank's use count of the buffer
// (local), then one system-scope fence and a relaxed add of the launch's
// rows to each rank's flag word publish every block's rows at once. (A
// release is cumulative, so the other GPUs see the whole grid's writes
// once they see the count. A system-scope release by every block instead
// cost about 6 us a launch, measured on a B200: the dominant cost of the
// exchange.)
__device__ __forceinline__ void red_relaxed_sys_add(uint32_t* p, uint32_t v) {
  asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ void peers_count_rows(const FkPeers& P, uint32_t buf, uint32_t launch_rows) {
  __syncthreads();
  if (threadIdx.x == 0) {
    char* me = P.base[P.rank];
    if (atom_add_acq_rel_gpu(xcounter(me) + buf, 1u) == gridDim.x - 1) {
      xcounter(me)[buf] = 0;
      xepoch(me)[buf] += 1;
      fence_acq_rel_sys();
      for (uint32_t q = 0; q < P.world; ++q) red_relaxed_sys_add(xflags(P.base[q]) + buf * FK_MAX_PEERS + P.rank, launch_rows);
    }
  }
}

// The consumer side: thread 0 waits, with a bound, until every rank's count
// has reached (uses so far) x (rows a use). False when one did not come
// within the bound (recorded in *err as 10 + buf).
__device__ __forceinline__ bool peers_wait_rows(const FkPeers& P, uint32_t buf, uint32_t rows, int* err) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    char* me = P.base[P.rank];
    const uint32_t target = *reinterpret_cast<volatile uint32_t*>(xepoch(me) + buf) * rows;
    const unsigned long long w0 = P.stats ? global_ns() : 0ull;
    ok = 1;
    for (uint32_t q = 0; q < P.world && ok; ++q) {
      const long long t0 = clock64();
      while ((int32_t)(ld_acquire_sys(xflags(me) + buf * FK_MAX_PEERS + q) - target) < 0) {
        if (clock64() - t0 > wait_bound(P)) {
          if (err) atomicCAS(err, 0, 10 + (int)buf);
          ok = 0;
          break;
        }
      }
    }
    wait_stats_add(P, w0);
  }
  __syncthreads();
  return ok != 0;
}

// Every thread of a consumer block calls this; thread 0 waits. False when
// a rank's signal did not come within the bound (recorded in *err).
__device__ __forceinline__ bool peers_wait(const FkPeers& P, uint32_t buf, int* err) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    char* me = P.base[P.rank];
    const uint32_t e = *reinterpret_cast<volatile uint32_t*>(xepoch(me) + buf);
    const unsigned long long w0 = P.stats ? global_ns() : 0ull;
    ok = 1;
    for (uint32_t q = 0; q < P.world && ok; ++q) {
      const long long t0 = clock64();
      while (ld_acquire_sys(xflags(me) + buf * FK_MAX_PEERS + q) < e) {
        if (clock64() - t0 > wait_bound(P)) {
          if (err) atomicCAS(err, 0, 10 + (int)buf);
          ok = 0;
          break;
        }
      }
    }
    wait_stats_add(P, w0);
  }
  __syncthreads();
  return ok != 0;
}

}  // namespace fk
