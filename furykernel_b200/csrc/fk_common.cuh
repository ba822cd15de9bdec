// Shared device helpers of the furykernel-cuda kernels (sm_100a).
//
// Every kernel here computes what the reference's CPU target computes for
// the same spec kernel: binary32 arithmetic with one rounding per operation
// (the library builds with --fmad=false; FuryKernel's Strict math,
// src/FuryKernel/Backend.hs:179-200), SIMD-group reductions pairwise with
// neighbours first (src/FuryKernel/Cpu.hs:469-505), threadgroup reductions
// in the order of src/FuryKernel/Reduce.hs:59-85, and Rsqrt/Exp computed in
// binary64 and rounded once (Cpu.hs:639-660).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace fk {

constexpr int kWarp = 32;

// IEEE 754-2019 maximumNumber, as the CPU target's fk_max (Cpu.hs:157-170).
__device__ __forceinline__ float max_number(float a, float b) {
  if (isnan(a)) return isnan(b) ? __int_as_float(0x7fc00000) : b;
  if (isnan(b) || a > b) return a;
  if (b > a) return b;
  return __int_as_float(__float_as_int(a) & __float_as_int(b));
}

// A SIMD group's sum, pairwise with neighbours first: the butterfly over
// lane offsets 1, 2, 4, 8, 16 adds exactly the pairs the CPU target adds
// (binary32 addition commutes), and leaves the total in every lane.
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 1; o < kWarp; o <<= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 1; o < kWarp; o <<= 1) v = max_number(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// tgReduceSum over 8 SIMD groups (256 threads), given each group's sum:
// lane l < 8 of the first group adds slot l to -0, the rest hold -0, and
// the pairwise sum of those 32 lanes is ((s0+s1)+(s2+s3))+((s4+s5)+(s6+s7))
// (adding -0 changes nothing).
__device__ __forceinline__ float tg_sum8(const float* s) {
  return __fadd_rn(__fadd_rn(__fadd_rn(s[0], s[1]), __fadd_rn(s[2], s[3])),
                   __fadd_rn(__fadd_rn(s[4], s[5]), __fadd_rn(s[6], s[7])));
}

// tgReduceMax over 8 SIMD groups: lane l < 8 of the first group takes the
// maximum of -inf and slot l (a NaN slot gives -inf there), then the
// pairwise tree; over NaNs alone the result is -inf, the identity.
__device__ __forceinline__ float tg_max8(const float* s) {
  float a[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) a[i] = max_number(-INFINITY, s[i]);
  return max_number(max_number(max_number(a[0], a[1]), max_number(a[2], a[3])),
                    max_number(max_number(a[4], a[5]), max_number(a[6], a[7])));
}

// Rsqrt and Exp of the CPU target: binary64, rounded once to binary32.
__device__ __forceinline__ float rsqrt_rounded(float v) {
  return (float)(1.0 / sqrt((double)v));
}
__device__ __forceinline__ float exp_rounded(float v) { return (float)exp((double)v); }

// One pack's chain of the GEMV order contract (test/Test/FuryKernel/Gemv.hs:19-20):
// ((x0 w0 + x1 w1) + (x2 w2 + x3 w3)).
__device__ __forceinline__ float pack_dot(float4 x, float4 w) {
  return __fadd_rn(__fadd_rn(__fmul_rn(x.x, w.x), __fmul_rn(x.y, w.y)),
                   __fadd_rn(__fmul_rn(x.z, w.z), __fmul_rn(x.w, w.w)));
}

// Streaming loads of data read once: no L1 allocation.
__device__ __forceinline__ float4 ld_stream(const float4* p) {
  float4 v;
  asm("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}

// A bulk prefetch of [p, p + bytes) into L2 by the copy engine, in pieces of
// at most 32 KiB: p 16-byte aligned, bytes a multiple of 16. Nothing waits
// for it; a later load of those lines finds them in L2.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  const char* c = static_cast<const char*>(p);
  for (uint32_t off = 0; off < bytes; off += 32768u) {
    const uint32_t n = bytes - off < 32768u ? bytes - off : 32768u;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(c + off), "r"(n) : "memory");
  }
}

// This block's slice of [p, p + bytes) brought toward L2 by one thread (p
// 16-byte aligned, bytes a multiple of 16; the slices of all blocks of the
// grid cover the range once). Null p: nothing.
__device__ __forceinline__ void prefetch_l2_slice(const void* p, unsigned long long bytes) {
  if (!p || threadIdx.x != 0) return;
  const unsigned long long per = ((bytes + gridDim.x - 1) / gridDim.x + 15) & ~15ull;
  const unsigned long long off = (unsigned long long)blockIdx.x * per;
  if (off >= bytes) return;
  const unsigned long long n = bytes - off < per ? bytes - off : per;
  for (unsigned long long done = 0; done < n; done += 0x40000000ull) {
    const unsigned long long piece = n - done < 0x40000000ull ? n - done : 0x40000000ull;
    prefetch_l2_bulk(static_cast<const char*>(p) + off + done, (uint32_t)piece);
  }
}

// Programmatic dependent launch: wait for the grids this one depends on,
// and let the next one be scheduled.
__device__ __forceinline__ void grid_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

}  // namespace fk
