// The tree reduction of config 1 for callers that cannot allocate device
// memory: the same two kernels as reduce_groups / reduce_final, with their
// scratch (the groups' partials, the final pass's chain sums and its
// completion counter) in one static device array instead of memory from
// cudaMalloc. Nothing here allocates.
#include <cuda_runtime.h>
#include <stdio.h>

#include <mutex>
#include <string>

#include "../../include/furykernel_cuda.h"
#include "fk_kernels.h"

namespace {

// The largest input: 2^26 floats (256 MiB of input), 2^18 group partials.
constexpr uint64_t kMaxElements = 1ull << 26;
constexpr uint32_t kMaxGroups = (uint32_t)(kMaxElements / 256);
constexpr uint32_t kChains = 256;
// partials [kMaxGroups] | chains [kChains] | counter (one word, padded)
constexpr size_t kScratchFloats = (size_t)kMaxGroups + kChains + 64;

constexpr int kMaxDevices = 64;
void* g_scratch[kMaxDevices] = {};
int g_sms[kMaxDevices] = {};
std::mutex g_setup;

}  // namespace

// Shared by every call on a device, for the life of the process
// (kScratchFloats * 4 bytes, just over 1 MiB, on each GPU that loads the library).
static __device__ __align__(256) float fk_noalloc_scratch[kScratchFloats];

extern int fkc_noalloc_fail(int code, const char* msg);

// The device address of this device's scratch, found once per device with
// the device current. Host code must not use the array's name as an
// address: on the host it names a stand-in, not device memory.
static int scratch_of(int device, float** out, int* sms) {
  std::lock_guard<std::mutex> lock(g_setup);
  if (!g_scratch[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, fk_noalloc_scratch);
    if (e != cudaSuccess) {
      std::string m = std::string("fkc_reduce_sum_f32_noalloc: cudaGetSymbolAddress: ") + cudaGetErrorString(e);
      return fkc_noalloc_fail(FKC_ERR_CUDA, m.c_str());
    }
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
    if (e != cudaSuccess) {
      std::string m = std::string("fkc_reduce_sum_f32_noalloc: cudaDeviceGetAttribute: ") + cudaGetErrorString(e);
      return fkc_noalloc_fail(FKC_ERR_CUDA, m.c_str());
    }
    g_sms[device] = n;
    g_scratch[device] = p;
  }
  *out = (float*)g_scratch[device];
  *sms = g_sms[device];
  return FKC_OK;
}

extern "C" int fkc_reduce_sum_f32_noalloc(const void* x, uint64_t n, void* y, void* stream) {
  if (!x || !y) return fkc_noalloc_fail(FKC_ERR_ARGUMENT, "fkc_reduce_sum_f32_noalloc: null argument.");
  if (n == 0 || n > kMaxElements) {
    char buf[256];
    snprintf(buf, sizeof buf,
             "fkc_reduce_sum_f32_noalloc: n is %llu, outside 1..%llu, the most its static scratch holds.",
             (unsigned long long)n, (unsigned long long)kMaxElements);
    return fkc_noalloc_fail(FKC_ERR_ARGUMENT, buf);
  }
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return fkc_noalloc_fail(FKC_ERR_CUDA, "fkc_reduce_sum_f32_noalloc: cudaGetDevice failed.");
  if (device < 0 || device >= kMaxDevices)
    return fkc_noalloc_fail(FKC_ERR_ARGUMENT, "fkc_reduce_sum_f32_noalloc: device index past 63.");
  float* scratch = nullptr;
  int sms = 0;
  int rc = scratch_of(device, &scratch, &sms);
  if (rc != FKC_OK) return rc;
  float* partials = scratch;
  float* chains = scratch + kMaxGroups;
  unsigned int* done = reinterpret_cast<unsigned int*>(scratch + kMaxGroups + kChains);
  cudaStream_t s = (cudaStream_t)stream;
  const uint32_t groups = (uint32_t)((n + 255) / 256);
  // The final pass counts finished blocks from zero; the last call may have
  // left anything there.
  e = cudaMemsetAsync(done, 0, sizeof(unsigned int), s);
  if (e == cudaSuccess) e = fk_launch_reduce_groups((const float*)x, n, partials, sms, s);
  if (e == cudaSuccess) e = fk_launch_reduce_final(partials, groups, chains, done, (float*)y, s);
  if (e != cudaSuccess) {
    std::string m = std::string("fkc_reduce_sum_f32_noalloc: ") + cudaGetErrorString(e);
    return fkc_noalloc_fail(FKC_ERR_CUDA, m.c_str());
  }
  return FKC_OK;
}
