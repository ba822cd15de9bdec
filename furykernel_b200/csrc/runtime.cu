// The C ABI of furykernel-cuda (include/furykernel_cuda.h): contexts,
// device memory, the kernel table with its ABI texts and hashes, checked
// launches, CUDA-graph capture of a plan's launches, and NCCL.
#include <cuda_runtime.h>
#include <math.h>
#include <nccl.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <string>
#include <unordered_set>
#include <vector>

#include "../../include/furykernel_cuda.h"
#include "fk_kernels.h"

// ---------------------------------------------------------------------------
// Errors

static thread_local std::string g_last_error;

static int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

static int cuda_fail(cudaError_t e, const char* what) {
  return fail(FKC_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

#define FKC_CUDA(call, what)                   \
  do {                                         \
    cudaError_t e_ = (call);                   \
    if (e_ != cudaSuccess) return cuda_fail(e_, what); \
  } while (0)

extern "C" const char* fkc_last_error(void) { return g_last_error.c_str(); }

// The no-allocation reduction's failures, reported through fkc_last_error.
int fkc_noalloc_fail(int code, const char* msg) {
  g_last_error = msg;
  return code;
}
extern "C" int fkc_version(void) { return 1; }

// ---------------------------------------------------------------------------
// Contexts

struct fkc_ctx {
  int device = 0;
  int sms = 0;
  cudaStream_t stream = nullptr;
  bool pdl = false;
  bool capturing = false;
  // Scratch of reduce_final: the 256 chains' sums and a completion counter.
  float* red_chains = nullptr;
  unsigned int* red_done = nullptr;
  // Where kernels with bounded waits record why they gave up (0: nothing).
  int* status = nullptr;
  std::unordered_set<void*> allocs;
  ncclComm_t comm = nullptr;
  int nranks = 1, rank = 0;
  // The peer set: every rank's exchange region, this rank's own included,
  // by rank (fkc_peer_set).
  FkPeers peers = {};
  std::unordered_set<void*> opened;  // peers' regions mapped here
  unsigned long long* wait_stats = nullptr;  // fkc_set_wait_stats: [ns waited, waits]
  size_t prefetch = 0;  // fkc_set_prefetch: the streaming GEMVs' L2 prefetch budget
  const void* l2pf = nullptr;  // fkc_set_l2_prefetch: a range the attention launches prefetch
  unsigned long long l2pf_bytes = 0;
  unsigned gemm_tm = 0, gemm_parts = 1;  // fkc_set_gemm_tile: tm 0 = the shape's own pick
};

struct fkc_graph {
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  int device = 0;
};

extern "C" int fkc_open(int device, fkc_ctx** out) {
  if (!out) return fail(FKC_ERR_ARGUMENT, "fkc_open: no place for the context.");
  int count = 0;
  FKC_CUDA(cudaGetDeviceCount(&count), "fkc_open: cudaGetDeviceCount");
  if (device < 0 || device >= count)
    return fail(FKC_ERR_ARGUMENT, "fkc_open: device %d is not one of the %d devices.", device, count);
  FKC_CUDA(cudaSetDevice(device), "fkc_open: cudaSetDevice");
  cudaDeviceProp prop;
  FKC_CUDA(cudaGetDeviceProperties(&prop, device), "fkc_open: cudaGetDeviceProperties");
  if (prop.major != 10)
    return fail(FKC_ERR_ARGUMENT, "fkc_open: device %d is sm_%d%d; this library is built for sm_100a.", device,
                prop.major, prop.minor);
  fkc_ctx* c = new fkc_ctx;
  c->device = device;
  c->sms = prop.multiProcessorCount;
  cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMalloc(&c->red_chains, 256 * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&c->red_done, sizeof(unsigned int));
  if (e == cudaSuccess) e = cudaMemset(c->red_done, 0, sizeof(unsigned int));
  if (e == cudaSuccess) e = cudaMalloc(&c->status, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(c->status, 0, sizeof(int));
  if (e != cudaSuccess) {
    fkc_close(c);
    return cuda_fail(e, "fkc_open");
  }
  *out = c;
  return FKC_OK;
}

extern "C" int fkc_close(fkc_ctx* c) {
  if (!c) return FKC_OK;
  cudaSetDevice(c->device);
  if (c->stream) cudaStreamSynchronize(c->stream);
  if (c->comm) ncclCommDestroy(c->comm);
  for (void* p : c->opened) cudaIpcCloseMemHandle(p);
  for (void* p : c->allocs) cudaFree(p);
  if (c->red_chains) cudaFree(c->red_chains);
  if (c->red_done) cudaFree(c->red_done);
  if (c->status) cudaFree(c->status);
  if (c->wait_stats) cudaFree(c->wait_stats);
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
  return FKC_OK;
}

extern "C" int fkc_stream(fkc_ctx* c, void** s) {
  if (!c || !s) return fail(FKC_ERR_ARGUMENT, "fkc_stream: null argument.");
  *s = (void*)c->stream;
  return FKC_OK;
}

extern "C" int fkc_sm_count(fkc_ctx* c, int* sms) {
  if (!c || !sms) return fail(FKC_ERR_ARGUMENT, "fkc_sm_count: null argument.");
  *sms = c->sms;
  return FKC_OK;
}

extern "C" int fkc_set_pdl(fkc_ctx* c, int enabled) {
  if (!c) return fail(FKC_ERR_ARGUMENT, "fkc_set_pdl: null context.");
  c->pdl = enabled != 0;
  return FKC_OK;
}

extern "C" int fkc_set_wait_limit(fkc_ctx* c, unsigned microseconds) {
  if (!c) return fail(FKC_ERR_ARGUMENT, "fkc_set_wait_limit: null context.");
  int khz = 0;
  FKC_CUDA(cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, c->device), "fkc_set_wait_limit");
  c->peers.wait_cycles = (long long)microseconds * (long long)khz / 1000;
  return FKC_OK;
}

extern "C" int fkc_set_prefetch(fkc_ctx* c, unsigned long long bytes) {
  if (!c) return fail(FKC_ERR_ARGUMENT, "fkc_set_prefetch: null context.");
  c->prefetch = (size_t)bytes;
  return FKC_OK;
}

extern "C" int fkc_set_l2_prefetch(fkc_ctx* c, const void* p, unsigned long long bytes) {
  if (!c) return fail(FKC_ERR_ARGUMENT, "fkc_set_l2_prefetch: null context.");
  if (p && (((uintptr_t)p & 15) || bytes % 16))
    return fail(FKC_ERR_ARGUMENT, "fkc_set_l2_prefetch: the range must start on a 16-byte boundary and hold whole "
                                  "16 bytes.");
  c->l2pf = bytes ? p : nullptr;
  c->l2pf_bytes = p ? bytes : 0;
  return FKC_OK;
}

extern "C" int fkc_set_gemm_tile(fkc_ctx* c, unsigned tm, unsigned parts) {
  if (!c) return fail(FKC_ERR_ARGUMENT, "fkc_set_gemm_tile: null context.");
  if (tm != 0 && (tm > 256 || tm % 16 != 0))
    return fail(FKC_ERR_ARGUMENT, "fkc_set_gemm_tile: tm %u is not a multiple of 16 in 16..256.", tm);
  if (parts > 2) return fail(FKC_ERR_ARGUMENT, "fkc_set_gemm_tile: parts %u is not 0, 1 or 2.", parts);
  c->gemm_tm = tm;
  c->gemm_parts = parts;
  return FKC_OK;
}

extern "C" int fkc_set_wait_stats(fkc_ctx* c, int enabled) {
  if (!c) return fail(FKC_ERR_ARGUMENT, "fkc_set_wait_stats: null context.");
  if (c->capturing) return fail(FKC_ERR_STATE, "fkc_set_wait_stats: not during a capture.");
  cudaSetDevice(c->device);
  if (enabled && !c->wait_stats) {
    FKC_CUDA(cudaMalloc(&c->wait_stats, 2 * sizeof(unsigned long long)), "fkc_set_wait_stats");
    FKC_CUDA(cudaMemset(c->wait_stats, 0, 2 * sizeof(unsigned long long)), "fkc_set_wait_stats");
  }
  c->peers.stats = enabled ? c->wait_stats : nullptr;
  return FKC_OK;
}

extern "C" int fkc_read_wait_stats(fkc_ctx* c, unsigned long long* ns_waited, unsigned long long* waits) {
  if (!c || !ns_waited || !waits) return fail(FKC_ERR_ARGUMENT, "fkc_read_wait_stats: null argument.");
  *ns_waited = 0, *waits = 0;
  if (!c->wait_stats) return FKC_OK;
  cudaSetDevice(c->device);
  unsigned long long h[2];
  FKC_CUDA(cudaStreamSynchronize(c->stream), "fkc_read_wait_stats");
  FKC_CUDA(cudaMemcpy(h, c->wait_stats, sizeof h, cudaMemcpyDeviceToHost), "fkc_read_wait_stats");
  FKC_CUDA(cudaMemset(c->wait_stats, 0, sizeof h), "fkc_read_wait_stats");
  *ns_waited = h[0], *waits = h[1];
  return FKC_OK;
}

extern "C" int fkc_sync(fkc_ctx* c) {
  if (!c) return fail(FKC_ERR_ARGUMENT, "fkc_sync: null context.");
  cudaSetDevice(c->device);
  FKC_CUDA(cudaStreamSynchronize(c->stream), "fkc_sync");
  return FKC_OK;
}

extern "C" int fkc_status(fkc_ctx* c, int* code) {
  if (!c || !code) return fail(FKC_ERR_ARGUMENT, "fkc_status: null argument.");
  cudaSetDevice(c->device);
  FKC_CUDA(cudaStreamSynchronize(c->stream), "fkc_status");
  FKC_CUDA(cudaMemcpy(code, c->status, sizeof(int), cudaMemcpyDeviceToHost), "fkc_status");
  FKC_CUDA(cudaMemset(c->status, 0, sizeof(int)), "fkc_status");
  return FKC_OK;
}

// ---------------------------------------------------------------------------
// Memory

extern "C" int fkc_buf_alloc(fkc_ctx* c, size_t bytes, void** dptr) {
  if (!c || !dptr) return fail(FKC_ERR_ARGUMENT, "fkc_buf_alloc: null argument.");
  cudaSetDevice(c->device);
  void* p = nullptr;
  FKC_CUDA(cudaMalloc(&p, bytes ? bytes : 16), "fkc_buf_alloc");
  c->allocs.insert(p);
  *dptr = p;
  return FKC_OK;
}

extern "C" int fkc_buf_free(fkc_ctx* c, void* dptr) {
  if (!c) return fail(FKC_ERR_ARGUMENT, "fkc_buf_free: null context.");
  if (!dptr) return FKC_OK;
  auto it = c->allocs.find(dptr);
  if (it == c->allocs.end()) return fail(FKC_ERR_ARGUMENT, "fkc_buf_free: %p is not a buffer of this context.", dptr);
  cudaSetDevice(c->device);
  c->allocs.erase(it);
  FKC_CUDA(cudaFree(dptr), "fkc_buf_free");
  return FKC_OK;
}

extern "C" int fkc_buf_zero(fkc_ctx* c, void* dptr, size_t bytes) {
  if (!c || (!dptr && bytes)) return fail(FKC_ERR_ARGUMENT, "fkc_buf_zero: null argument.");
  cudaSetDevice(c->device);
  FKC_CUDA(cudaMemsetAsync(dptr, 0, bytes, c->stream), "fkc_buf_zero");
  return FKC_OK;
}

extern "C" int fkc_buf_upload(fkc_ctx* c, void* dptr, const void* host, size_t bytes) {
  if (!c || (bytes && (!dptr || !host))) return fail(FKC_ERR_ARGUMENT, "fkc_buf_upload: null argument.");
  cudaSetDevice(c->device);
  FKC_CUDA(cudaMemcpyAsync(dptr, host, bytes, cudaMemcpyHostToDevice, c->stream), "fkc_buf_upload");
  if (!c->capturing) FKC_CUDA(cudaStreamSynchronize(c->stream), "fkc_buf_upload");
  return FKC_OK;
}

extern "C" int fkc_buf_download(fkc_ctx* c, void* host, const void* dptr, size_t bytes) {
  if (!c || (bytes && (!dptr || !host))) return fail(FKC_ERR_ARGUMENT, "fkc_buf_download: null argument.");
  cudaSetDevice(c->device);
  FKC_CUDA(cudaMemcpyAsync(host, dptr, bytes, cudaMemcpyDeviceToHost, c->stream), "fkc_buf_download");
  if (!c->capturing) FKC_CUDA(cudaStreamSynchronize(c->stream), "fkc_buf_download");
  return FKC_OK;
}

extern "C" int fkc_host_alloc(size_t bytes, void** host) {
  if (!host) return fail(FKC_ERR_ARGUMENT, "fkc_host_alloc: null argument.");
  FKC_CUDA(cudaHostAlloc(host, bytes ? bytes : 16, cudaHostAllocDefault), "fkc_host_alloc");
  return FKC_OK;
}

extern "C" int fkc_host_free(void* host) {
  if (host) FKC_CUDA(cudaFreeHost(host), "fkc_host_free");
  return FKC_OK;
}

extern "C" int fkc_kv_arena(fkc_ctx* c, uint32_t layers, uint32_t slots, uint32_t kv_heads, uint32_t length,
                            uint32_t head_dim, void** k_base, void** v_base) {
  if (!c || !k_base || !v_base) return fail(FKC_ERR_ARGUMENT, "fkc_kv_arena: null argument.");
  const size_t per = (size_t)slots * kv_heads * length * head_dim * sizeof(float);
  const size_t total = per * layers;
  int rc = fkc_buf_alloc(c, total, k_base);
  if (rc) return rc;
  rc = fkc_buf_alloc(c, total, v_base);
  if (rc) return rc;
  rc = fkc_buf_zero(c, *k_base, total);
  if (rc) return rc;
  return fkc_buf_zero(c, *v_base, total);
}

extern "C" int fkc_kv_arena_elem(fkc_ctx* c, uint32_t layers, uint32_t slots, uint32_t kv_heads, uint32_t length,
                                 uint32_t head_dim, uint32_t elem_bytes, void** k_base, void** v_base) {
  if (!c || !k_base || !v_base) return fail(FKC_ERR_ARGUMENT, "fkc_kv_arena_elem: null argument.");
  if (elem_bytes != 2 && elem_bytes != 4)
    return fail(FKC_ERR_ARGUMENT, "fkc_kv_arena_elem: elements of %u bytes; a cache holds 2 (bf16, f16) or 4 (f32).",
                elem_bytes);
  const size_t per = (size_t)slots * kv_heads * length * head_dim * elem_bytes;
  const size_t total = per * layers;
  int rc = fkc_buf_alloc(c, total, k_base);
  if (rc) return rc;
  rc = fkc_buf_alloc(c, total, v_base);
  if (rc) return rc;
  rc = fkc_buf_zero(c, *k_base, total);
  if (rc) return rc;
  return fkc_buf_zero(c, *v_base, total);
}

extern "C" int fkc_rope_tables(fkc_ctx* c, double theta, uint32_t d, uint32_t rotated, uint32_t positions,
                               void** cos_t, void** sin_t) {
  if (!c || !cos_t || !sin_t || d == 0) return fail(FKC_ERR_ARGUMENT, "fkc_rope_tables: bad argument.");
  const size_t n = (size_t)positions * rotated;
  std::vector<float> hc(n), hs(n);
  for (uint32_t p = 0; p < positions; ++p)
    for (uint32_t i = 0; i < rotated; ++i) {
      const double angle = (double)p * pow(theta, -((double)(2 * i) / (double)d));
      hc[(size_t)p * rotated + i] = (float)cos(angle);
      hs[(size_t)p * rotated + i] = (float)sin(angle);
    }
  int rc = fkc_buf_alloc(c, n * sizeof(float), cos_t);
  if (rc) return rc;
  rc = fkc_buf_alloc(c, n * sizeof(float), sin_t);
  if (rc) return rc;
  rc = fkc_buf_upload(c, *cos_t, hc.data(), n * sizeof(float));
  if (rc) return rc;
  return fkc_buf_upload(c, *sin_t, hs.data(), n * sizeof(float));
}

extern "C" int fkc_fill_normal(fkc_ctx* c, void* dptr, uint64_t n, uint64_t seed, double mu, double sigma) {
  if (!c || (n && !dptr)) return fail(FKC_ERR_ARGUMENT, "fkc_fill_normal: null argument.");
  cudaSetDevice(c->device);
  FKC_CUDA(fk_launch_fill_normal((float*)dptr, n, seed, mu, sigma, c->stream), "fkc_fill_normal");
  return FKC_OK;
}

extern "C" int fkc_fill_normal_bf16(fkc_ctx* c, void* dptr, uint64_t n, uint64_t seed, double mu, double sigma) {
  if (!c || (n && !dptr)) return fail(FKC_ERR_ARGUMENT, "fkc_fill_normal_bf16: null argument.");
  cudaSetDevice(c->device);
  FKC_CUDA(fk_launch_fill_normal_w16(FK_BF16, (uint16_t*)dptr, n, seed, mu, sigma, c->stream), "fkc_fill_normal_bf16");
  return FKC_OK;
}

extern "C" int fkc_fill_normal_f16(fkc_ctx* c, void* dptr, uint64_t n, uint64_t seed, double mu, double sigma) {
  if (!c || (n && !dptr)) return fail(FKC_ERR_ARGUMENT, "fkc_fill_normal_f16: null argument.");
  cudaSetDevice(c->device);
  FKC_CUDA(fk_launch_fill_normal_w16(FK_F16, (uint16_t*)dptr, n, seed, mu, sigma, c->stream), "fkc_fill_normal_f16");
  return FKC_OK;
}

extern "C" int fkc_fill_uniform(fkc_ctx* c, void* dptr, uint64_t n, uint64_t seed, double a, double b) {
  if (!c || (n && !dptr)) return fail(FKC_ERR_ARGUMENT, "fkc_fill_uniform: null argument.");
  cudaSetDevice(c->device);
  FKC_CUDA(fk_launch_fill_uniform((float*)dptr, n, seed, a, b, c->stream), "fkc_fill_uniform");
  return FKC_OK;
}

// ---------------------------------------------------------------------------
// The kernel table

namespace {

struct BufSpec {
  const char* name;
  const char* access;  // read, write, read_write
  const char* type;    // f32, u32
};

struct ParamSpec {
  const char* name;
  const char* type;  // u32 or f32
  bool dim;
  uint32_t lo, hi, mult;
};

struct Params {
  const unsigned char* bytes;
  const std::vector<uint32_t>* offsets;
  uint32_t u(int i) const {
    uint32_t v;
    memcpy(&v, bytes + (*offsets)[i], 4);
    return v;
  }
  float f(int i) const {
    float v;
    memcpy(&v, bytes + (*offsets)[i], 4);
    return v;
  }
};

typedef int (*LaunchFn)(fkc_ctx*, const Params&, void* const*);

struct KernelSpec {
  const char* name;
  uint32_t threads;
  std::vector<BufSpec> bufs;
  std::vector<ParamSpec> params;
  LaunchFn launch;
  // Derived: the C layout, the ABI text and its hash.
  std::vector<uint32_t> offsets;
  uint32_t params_size = 0;
  std::string abi;
  uint64_t hash = 0;
  // Tables of device addresses, bound after the buffers (IR.hs:400-429):
  // each entry the start of an array of the table's type.
  std::vector<BufSpec> tables = {};
};

uint64_t fnv1a(const void* p, size_t n) {
  const unsigned char* b = (const unsigned char*)p;
  uint64_t h = 0xcbf29ce484222325ULL;
  for (size_t i = 0; i < n; ++i) {
    h ^= b[i];
    h *= 0x100000001b3ULL;
  }
  return h;
}

int launched(cudaError_t e, const char* name) {
  if (e == cudaErrorInvalidValue)
    return fail(FKC_ERR_ARGUMENT, "%s: the launch's shape is not one this kernel takes.", name);
  if (e != cudaSuccess) return cuda_fail(e, name);
  return FKC_OK;
}

#define F(i) ((float*)bufs[i])
#define CF(i) ((const float*)bufs[i])
#define CU(i) ((const uint32_t*)bufs[i])
#define U(i) ((uint32_t*)bufs[i])

int l_reduce_groups(fkc_ctx* c, const Params& p, void* const* bufs) {
  return launched(fk_launch_reduce_groups(CF(0), p.u(0), F(1), c->sms, c->stream), "reduce_groups");
}

int l_reduce_final(fkc_ctx* c, const Params& p, void* const* bufs) {
  return launched(fk_launch_reduce_final(CF(0), p.u(0), c->red_chains, c->red_done, F(1), c->stream),
                  "reduce_final");
}

int l_rmsnorm_rows(fkc_ctx* c, const Params& p, void* const* bufs) {
  return launched(fk_launch_rmsnorm_rows(CF(0), CF(1), F(2), p.u(0), p.u(1), p.f(2), p.f(3), c->stream),
                  "rmsnorm_rows");
}

int l_softmax_rows(fkc_ctx* c, const Params& p, void* const* bufs) {
  return launched(fk_launch_softmax_rows(CF(0), F(1), p.u(0), p.u(1), c->stream), "softmax_rows");
}

// Decode batches of up to 4 rows stream through the persistent kernel; larger
// batches take the chunked one. Both keep the GEMV order contract.
cudaError_t run_gemv(fkc_ctx* c, const FkGemv& g0) {
  FkGemv g = g0;
  g.prefetch = c->prefetch;
  if (fk_gemv_streams(g)) return fk_launch_gemv_stream(g, c->sms, c->stream);
  if (fk_gemv_batches(g)) return fk_launch_gemv_batch(g, c->sms, c->stream);
  return fk_launch_gemv(g, c->stream);
}

FkGemv gemv_base(fkc_ctx* c, const Params& p) {
  FkGemv g = {};
  g.n = p.u(0);
  g.k = p.u(1);
  g.m = p.u(2);
  g.split = p.u(3);
  g.ldx = p.u(4);
  g.ldy = p.u(5);
  g.factor = 1.0f;
  g.pdl = c->pdl;
  return g;
}

// gemv: w, x, y | n k m split ldx ldy
int l_gemv(fkc_ctx* c, const Params& p, void* const* bufs) {
  FkGemv g = gemv_base(c, p);
  g.w = CF(0), g.x = CF(1), g.y = F(2);
  g.prologue = FK_PRO_NONE;
  return launched(run_gemv(c, g), "gemv");
}
// gemv_add: w, x, r, y | n k m split ldx ldy ldr
int l_gemv_add(fkc_ctx* c, const Params& p, void* const* bufs) {
  FkGemv g = gemv_base(c, p);
  g.w = CF(0), g.x = CF(1), g.r = CF(2), g.y = F(3);
  g.ldr = p.u(6);
  g.prologue = FK_PRO_NONE;
  return launched(run_gemv(c, g), "gemv_add");
}
// gemv_rmsnorm: w, x, gamma, y | n k m split ldx ldy eps factor
int l_gemv_rmsnorm(fkc_ctx* c, const Params& p, void* const* bufs) {
  FkGemv g = gemv_base(c, p);
  g.w = CF(0), g.x = CF(1), g.gamma = CF(2), g.y = F(3);
  g.eps = p.f(6);
  g.factor = p.f(7);
  g.prologue = FK_PRO_RMSNORM;
  return launched(run_gemv(c, g), "gemv_rmsnorm");
}
// gemv_rmsnorm_silu: w, x, gamma, y | n k m split ldx ldy eps factor; rows
// interleave gate and up, y gets n / 2 columns.
int l_gemv_rmsnorm_silu(fkc_ctx* c, const Params& p, void* const* bufs) {
  FkGemv g = gemv_base(c, p);
  g.w = CF(0), g.x = CF(1), g.gamma = CF(2), g.y = F(3);
  g.eps = p.f(6);
  g.factor = p.f(7);
  g.prologue = FK_PRO_RMSNORM;
  g.silu_pair = true;
  if (g.n % 2 != 0) return fail(FKC_ERR_ARGUMENT, "gemv_rmsnorm_silu: n %u is not a whole number of row pairs.", g.n);
  if (!fk_gemv_streams(g) && !fk_gemv_batches(g))
    return fail(FKC_ERR_ARGUMENT,
                "gemv_rmsnorm_silu: m %u, k %u and split %u are past what the row-pair kernels take (m at most 64, "
                "split 1 past m 4).",
                g.m, g.k, g.split);
  return launched(run_gemv(c, g), "gemv_rmsnorm_silu");
}

// gemv_silu: w, x, y | n k m split ldx ldy up_off
int l_gemv_silu(fkc_ctx* c, const Params& p, void* const* bufs) {
  FkGemv g = gemv_base(c, p);
  g.w = CF(0), g.x = CF(1), g.y = F(2);
  g.up_off = p.u(6);
  g.prologue = FK_PRO_SILU;
  return launched(run_gemv(c, g), "gemv_silu");
}
// gemv_silu_add: w, x, r, y | n k m split ldx ldy ldr up_off
int l_gemv_silu_add(fkc_ctx* c, const Params& p, void* const* bufs) {
  FkGemv g = gemv_base(c, p);
  g.w = CF(0), g.x = CF(1), g.r = CF(2), g.y = F(3);
  g.ldr = p.u(6);
  g.up_off = p.u(7);
  g.prologue = FK_PRO_SILU;
  return launched(run_gemv(c, g), "gemv_silu_add");
}

// kv_store_ring: qkv cos sin pos slot k_cache v_cache | m kv_heads d length rotated ldq k_off v_off
int l_kv_store(fkc_ctx* c, const Params& p, void* const* bufs) {
  FkKvStore a = {};
  a.qkv = CF(0), a.cos_t = CF(1), a.sin_t = CF(2), a.pos = CU(3), a.slot = CU(4), a.kc = F(5), a.vc = F(6);
  a.m = p.u(0), a.kv_heads = p.u(1), a.d = p.u(2), a.length = p.u(3), a.rotated = p.u(4);
  a.ldq = p.u(5), a.k_off = p.u(6), a.v_off = p.u(7);
  a.pdl = c->pdl;
  if (a.rotated > a.d / 2) return fail(FKC_ERR_ARGUMENT, "kv_store_ring: rotated %u is more than d/2.", a.rotated);
  return launched(fk_launch_kv_store(a, c->stream), "kv_store_ring");
}

// attend_split: qkv cos sin pos slot k_cache v_cache part_m part_l part_acc
//   | m heads kv_heads d length rotated chunk max_splits ldq q_off scale
int l_attend(fkc_ctx* c, const Params& p, void* const* bufs) {
  FkAttend a = {};
  a.qkv = CF(0), a.cos_t = CF(1), a.sin_t = CF(2), a.pos = CU(3), a.slot = CU(4), a.kc = CF(5), a.vc = CF(6);
  a.part_m = F(7), a.part_l = F(8), a.part_acc = F(9);
  a.m = p.u(0), a.heads = p.u(1), a.kv_heads = p.u(2), a.d = p.u(3), a.length = p.u(4), a.rotated = p.u(5);
  a.chunk = p.u(6), a.max_splits = p.u(7), a.ldq = p.u(8), a.q_off = p.u(9);
  a.scale = p.f(10);
  a.pdl = c->pdl;
  a.pf = c->l2pf, a.pf_bytes = c->l2pf_bytes;
  if (a.kv_heads == 0 || a.heads % a.kv_heads != 0)
    return fail(FKC_ERR_ARGUMENT, "attend_split: %u heads do not share %u KV heads in groups.", a.heads, a.kv_heads);
  return launched(fk_launch_attend(a, c->stream), "attend_split");
}

// attend_decode: qkv cos sin pos slot k_cache v_cache part_m part_l part_acc
//   | m heads kv_heads d length rotated chunk max_splits ldq q_off k_off v_off scale
// The KV store and attention steps of a decode step whose rows sit in
// distinct slots, in one launch (attend_combine follows).
int l_attend_decode(fkc_ctx* c, const Params& p, void* const* bufs) {
  FkAttendDecode f = {};
  FkAttend& a = f.a;
  a.qkv = CF(0), a.cos_t = CF(1), a.sin_t = CF(2), a.pos = CU(3), a.slot = CU(4), a.kc = CF(5), a.vc = CF(6);
  a.part_m = F(7), a.part_l = F(8), a.part_acc = F(9);
  f.kc_w = F(5), f.vc_w = F(6);
  a.m = p.u(0), a.heads = p.u(1), a.kv_heads = p.u(2), a.d = p.u(3), a.length = p.u(4), a.rotated = p.u(5);
  a.chunk = p.u(6), a.max_splits = p.u(7), a.ldq = p.u(8), a.q_off = p.u(9);
  f.k_off = p.u(10), f.v_off = p.u(11);
  a.scale = p.f(12);
  a.pdl = c->pdl;
  a.pf = c->l2pf, a.pf_bytes = c->l2pf_bytes;
  if (a.kv_heads == 0 || a.heads % a.kv_heads != 0)
    return fail(FKC_ERR_ARGUMENT, "attend_decode: %u heads do not share %u KV heads in groups.", a.heads, a.kv_heads);
  if (a.rotated > a.d / 2) return fail(FKC_ERR_ARGUMENT, "attend_decode: rotated %u is more than d/2.", a.rotated);
  return launched(fk_launch_attend_decode(f, c->stream), "attend_decode");
}

// attend_prompt: qkv cos sin pos slot k_cache v_cache out
//   | m heads kv_heads d length rotated ldq q_off ldo max_pos scale
// A prompt's rows in one slot (slot[0]), positions <= max_pos < length.
int l_attend_prompt(fkc_ctx* c, const Params& p, void* const* bufs) {
  FkAttend a = {};
  a.qkv = CF(0), a.cos_t = CF(1), a.sin_t = CF(2), a.pos = CU(3), a.slot = CU(4), a.kc = CF(5), a.vc = CF(6);
  a.m = p.u(0), a.heads = p.u(1), a.kv_heads = p.u(2), a.d = p.u(3), a.length = p.u(4), a.rotated = p.u(5);
  a.ldq = p.u(6), a.q_off = p.u(7);
  a.scale = p.f(10);
  a.pdl = c->pdl;
  if (a.kv_heads == 0 || a.heads % a.kv_heads != 0)
    return fail(FKC_ERR_ARGUMENT, "attend_prompt: %u heads do not share %u KV heads in groups.", a.heads, a.kv_heads);
  if (a.rotated > a.d / 2) return fail(FKC_ERR_ARGUMENT, "attend_prompt: rotated %u is more than d/2.", a.rotated);
  if (p.u(9) >= a.length)
    return fail(FKC_ERR_ARGUMENT, "attend_prompt: max_pos %u is not within the ring's length %u.", p.u(9), a.length);
  return launched(fk_launch_attend_prompt(a, F(7), p.u(8), p.u(9), c->stream), "attend_prompt");
}

// attend_combine: part_m part_l part_acc pos out | m heads d chunk max_splits ldo
int l_combine(fkc_ctx* c, const Params& p, void* const* bufs) {
  FkCombine a = {};
  a.part_m = CF(0), a.part_l = CF(1), a.part_acc = CF(2), a.pos = CU(3), a.out = F(4);
  a.m = p.u(0), a.heads = p.u(1), a.d = p.u(2), a.chunk = p.u(3), a.max_splits = p.u(4), a.ldo = p.u(5);
  a.pdl = c->pdl;
  return launched(fk_launch_combine(a, c->stream), "attend_combine");
}

// gather: table tokens y | width m factor
int l_gather(fkc_ctx* c, const Params& p, void* const* bufs) {
  return launched(fk_launch_gather(CF(0), p.u(0), CU(1), p.u(1), p.f(2), F(2), c->pdl, c->stream), "gather");
}

// argmax: x ids | m n ldx
int l_argmax(fkc_ctx* c, const Params& p, void* const* bufs) {
  return launched(fk_launch_argmax(CF(0), p.u(0), p.u(1), p.u(2), U(1), c->pdl, c->stream), "argmax");
}

// rope: x pos cos sin y | m heads d rotated ldx ldy
int l_rope(fkc_ctx* c, const Params& p, void* const* bufs) {
  if (p.u(3) > p.u(2) / 2) return fail(FKC_ERR_ARGUMENT, "rope: rotated %u is more than d/2.", p.u(3));
  return launched(
      fk_launch_rope(CF(0), p.u(0), p.u(1), p.u(2), p.u(3), p.u(4), CU(1), CF(2), CF(3), F(4), p.u(5), c->stream),
      "rope");
}

// split_tf32: x hi lo | n
int l_split_tf32(fkc_ctx* c, const Params& p, void* const* bufs) {
  return launched(fk_launch_split_tf32(CF(0), F(1), F(2), p.u(0), c->stream), "split_tf32");
}

// gemm_tf32x3: a a_hi a_lo w_hi w_lo c | M N K ldc. A is split into the
// caller's a_hi / a_lo first; W comes split (split_tf32, once).
int l_gemm_tf32x3(fkc_ctx* c, const Params& p, void* const* bufs) {
  const uint32_t M = p.u(0), N = p.u(1), K = p.u(2), ldc = p.u(3);
  if (ldc < N) return fail(FKC_ERR_ARGUMENT, "gemm_tf32x3: ldc %u is less than N %u.", ldc, N);
  cudaError_t e = fk_launch_split_tf32(CF(0), F(1), F(2), (uint64_t)M * K, c->stream);
  if (e == cudaSuccess) e = fk_launch_gemm_tf32x3(CF(1), CF(2), CF(3), CF(4), F(5), M, N, K, ldc, c->status, c->stream);
  return launched(e, "gemm_tf32x3");
}

// gemm_tf32x3w: a a_hi a_lo w c | M N K ldc. A is split into the caller's
// a_hi / a_lo first; W (f32, as the weight arena holds it) is split inside
// the kernel. The tile is the shape's (fk_gemm_tf32x3w_tile), or the one
// fkc_set_gemm_tile set.
int l_gemm_tf32x3w(fkc_ctx* c, const Params& p, void* const* bufs) {
  const uint32_t M = p.u(0), N = p.u(1), K = p.u(2), ldc = p.u(3);
  if (ldc < N) return fail(FKC_ERR_ARGUMENT, "gemm_tf32x3w: ldc %u is less than N %u.", ldc, N);
  FkGemmTile tile = fk_gemm_tf32x3w_tile(M, N, K, c->sms);
  if (c->gemm_tm) {
    const uint64_t tiles = (uint64_t)((N + 127) / 128) * ((M + c->gemm_tm - 1) / c->gemm_tm);
    const uint64_t g = c->gemm_parts == 1 ? tiles : c->gemm_parts == 2 ? 2 * tiles
                                                                       : std::min<uint64_t>(tiles, c->sms);
    if (g > 0x7fffffffull) return fail(FKC_ERR_ARGUMENT, "gemm_tf32x3w: %llu CTAs for the set tile.", (unsigned long long)g);
    tile = {c->gemm_tm, (uint32_t)g};
  }
  cudaError_t e = fk_launch_split_tf32(CF(0), F(1), F(2), (uint64_t)M * K, c->stream);
  if (e == cudaSuccess)
    e = fk_launch_gemm_tf32x3w(CF(1), CF(2), CF(3), F(4), M, N, K, ldc, tile, c->peers.wait_cycles, c->status,
                               c->stream);
  return launched(e, "gemm_tf32x3w");
}

// argmax_pairs: x pairs | m n ldx offset
int l_argmax_pairs(fkc_ctx* c, const Params& p, void* const* bufs) {
  return launched(fk_launch_argmax_pairs(CF(0), p.u(0), p.u(1), p.u(2), p.u(3), U(1), nullptr, c->pdl, c->stream),
                  "argmax_pairs");
}

bool have_peers(fkc_ctx* c) { return c->peers.world >= 1 && c->peers.base[0] != nullptr; }

// argmax_scatter: x | m n ldx offset: the candidates into every rank's buffer 2.
int l_argmax_scatter(fkc_ctx* c, const Params& p, void* const* bufs) {
  if (!have_peers(c)) return fail(FKC_ERR_STATE, "argmax_scatter: the context has no peer set.");
  return launched(fk_launch_argmax_pairs(CF(0), p.u(0), p.u(1), p.u(2), p.u(3), nullptr, &c->peers, c->pdl,
                                         c->stream),
                  "argmax_scatter");
}

// argmax_gather_pick: ids | m: the ranks' candidates from this rank's buffer 2.
int l_argmax_gather_pick(fkc_ctx* c, const Params& p, void* const* bufs) {
  if (!have_peers(c)) return fail(FKC_ERR_STATE, "argmax_gather_pick: the context has no peer set.");
  return launched(fk_launch_argmax_pick(nullptr, c->peers.world, p.u(0), U(0), &c->peers, c->status, c->pdl,
                                        c->stream),
                  "argmax_gather_pick");
}

// gemv_scatter: w x | n k m split ldx xbuf: this rank's partial rows into
// every rank's exchange buffer xbuf.
int l_gemv_scatter(fkc_ctx* c, const Params& p, void* const* bufs) {
  if (!have_peers(c)) return fail(FKC_ERR_STATE, "gemv_scatter: the context has no peer set.");
  FkGemv g = {};
  g.w = CF(0), g.x = CF(1);
  g.n = p.u(0), g.k = p.u(1), g.m = p.u(2), g.split = p.u(3), g.ldx = p.u(4), g.xbuf = p.u(5);
  g.factor = 1.0f;
  g.pdl = c->pdl;
  g.prologue = FK_PRO_NONE;
  g.scatter = true;
  g.peers = c->peers;
  g.err = c->status;
  if (!fk_gemv_streams(g)) return fail(FKC_ERR_ARGUMENT, "gemv_scatter: m %u is past the streaming kernel's 4.", g.m);
  g.prefetch = c->prefetch;
  return launched(fk_launch_gemv_stream(g, c->sms, c->stream), "gemv_scatter");
}

// gemv_reduce_rmsnorm(_silu): w r gamma xout y | n k m split ldr ldy eps factor
// xbuf: x = r + the ranks' partials in buffer xbuf, in rank order, stored to
// xout; then RMSNorm and the GEMV (SiLU-gate of row pairs for _silu).
int reduce_gemv(fkc_ctx* c, const Params& p, void* const* bufs, bool silu, const char* name) {
  if (!have_peers(c)) return fail(FKC_ERR_STATE, "%s: the context has no peer set.", name);
  FkGemv g = {};
  g.w = CF(0), g.x = CF(1), g.gamma = CF(2), g.xout = F(3), g.y = F(4);
  g.n = p.u(0), g.k = p.u(1), g.m = p.u(2), g.split = p.u(3), g.ldx = p.u(4), g.ldy = p.u(5);
  g.eps = p.f(6), g.factor = p.f(7), g.xbuf = p.u(8);
  g.pdl = c->pdl;
  g.prologue = FK_PRO_REDUCE_RMSNORM;
  g.silu_pair = silu;
  g.peers = c->peers;
  g.err = c->status;
  if (g.ldx != g.k) return fail(FKC_ERR_ARGUMENT, "%s: the residual rows must be whole (ldr %u, k %u).", name, g.ldx, g.k);
  if (!fk_gemv_streams(g)) return fail(FKC_ERR_ARGUMENT, "%s: m %u is past the streaming kernel's 4.", name, g.m);
  g.prefetch = c->prefetch;
  return launched(fk_launch_gemv_stream(g, c->sms, c->stream), name);
}
int l_gemv_reduce_rmsnorm(fkc_ctx* c, const Params& p, void* const* bufs) {
  return reduce_gemv(c, p, bufs, false, "gemv_reduce_rmsnorm");
}
int l_gemv_reduce_rmsnorm_silu(fkc_ctx* c, const Params& p, void* const* bufs) {
  return reduce_gemv(c, p, bufs, true, "gemv_reduce_rmsnorm_silu");
}

// argmax_pick: pairs ids | shards m
int l_argmax_pick(fkc_ctx* c, const Params& p, void* const* bufs) {
  return launched(fk_launch_argmax_pick(CU(0), p.u(0), p.u(1), U(1), nullptr, nullptr, c->pdl, c->stream),
                  "argmax_pick");
}

// advance: ids tokens pos | m
int l_advance(fkc_ctx* c, const Params& p, void* const* bufs) {
  return launched(fk_launch_advance(CU(0), U(1), U(2), p.u(0), c->pdl, c->stream), "advance");
}

int l_add(fkc_ctx* c, const Params& p, void* const* bufs) {
  return launched(fk_launch_add(CF(0), CF(1), F(2), p.u(0), c->stream), "add");
}

int l_silu_mul(fkc_ctx* c, const Params& p, void* const* bufs) {
  return launched(fk_launch_silu_mul(CF(0), CF(1), F(2), p.u(0), c->stream), "silu_mul");
}
// gemv_bf16: w x y | n k m pack split ldx ldy: the reference's bf16 GEMV
// family (test/Test/FuryKernel/Gemv.hs), pack width 4, 8 or 16.
int l_gemv_bf16(fkc_ctx* c, const Params& p, void* const* bufs) {
  const uint32_t pack = p.u(3);
  if (pack != 4 && pack != 8 && pack != 16)
    return fail(FKC_ERR_ARGUMENT, "gemv_bf16: the pack width %u is not 4, 8 or 16.", pack);
  if (p.u(1) % pack != 0 || p.u(5) % pack != 0)
    return fail(FKC_ERR_ARGUMENT, "gemv_bf16: k %u and ldx %u are not multiples of the pack width %u.", p.u(1),
                p.u(5), pack);
  return launched(fk_launch_gemv_bf16((const uint16_t*)bufs[0], (const uint16_t*)bufs[1], (uint16_t*)bufs[2], p.u(0),
                                      p.u(1), p.u(2), pack, p.u(4), p.u(5), p.u(6), c->sms, c->pdl, c->stream),
                  "gemv_bf16");
}

// silu_pairs: x y | n: y[i] = silu(x[2i]) * x[2i + 1].
int l_silu_pairs(fkc_ctx* c, const Params& p, void* const* bufs) {
  return launched(fk_launch_silu_pairs(CF(0), F(1), p.u(0), c->stream), "silu_pairs");
}

// ---- 16-bit weights (the entries' `w`, `gamma`, `table` buffers are bf16 or
// f16, EL) and 16-bit KV caches (`k_cache`, `v_cache`) ----
#define W16(i) ((const uint16_t*)bufs[i])
#define M16(i) ((uint16_t*)bufs[i])
// An entry's name: a 16-bit weights form (WN) or KV cache form (KN) of base.
#define WN(base) (EL == FK_F16 ? base "_wf16" : base "_wbf16")
#define KN(base) (EL == FK_F16 ? base "_kvf16" : base "_kvbf16")

template <FkElem EL>
int gemv_w16(fkc_ctx* c, const FkGemv& g0, const uint16_t* w, const uint16_t* gamma, const char* name) {
  FkGemv g = g0;
  g.prefetch = c->prefetch;
  return launched(fk_launch_gemv_w16(g, EL, w, gamma, c->sms, c->stream), name);
}
template <FkElem EL>
int l_gemv_w16(fkc_ctx* c, const Params& p, void* const* bufs) {
  FkGemv g = gemv_base(c, p);
  g.x = CF(1), g.y = F(2);
  g.prologue = FK_PRO_NONE;
  return gemv_w16<EL>(c, g, W16(0), nullptr, WN("gemv"));
}
template <FkElem EL>
int l_gemv_add_w16(fkc_ctx* c, const Params& p, void* const* bufs) {
  FkGemv g = gemv_base(c, p);
  g.x = CF(1), g.r = CF(2), g.y = F(3);
  g.ldr = p.u(6);
  g.prologue = FK_PRO_NONE;
  return gemv_w16<EL>(c, g, W16(0), nullptr, WN("gemv_add"));
}
template <FkElem EL>
int l_gemv_rmsnorm_w16(fkc_ctx* c, const Params& p, void* const* bufs) {
  FkGemv g = gemv_base(c, p);
  g.x = CF(1), g.y = F(3);
  g.eps = p.f(6);
  g.factor = p.f(7);
  g.prologue = FK_PRO_RMSNORM;
  return gemv_w16<EL>(c, g, W16(0), W16(2), WN("gemv_rmsnorm"));
}
template <FkElem EL>
int l_gemv_rmsnorm_silu_w16(fkc_ctx* c, const Params& p, void* const* bufs) {
  FkGemv g = gemv_base(c, p);
  g.x = CF(1), g.y = F(3);
  g.eps = p.f(6);
  g.factor = p.f(7);
  g.prologue = FK_PRO_RMSNORM;
  g.silu_pair = true;
  if (g.n % 2 != 0)
    return fail(FKC_ERR_ARGUMENT, "%s: n %u is not a whole number of row pairs.", WN("gemv_rmsnorm_silu"), g.n);
  if (!fk_gemv_streams(g) && !fk_gemv_w16_batches(g, W16(0)))
    return fail(FKC_ERR_ARGUMENT,
                "%s: m %u, k %u and split %u are past what the row-pair kernels take (m at most 64, split 1 past m "
                "4).",
                WN("gemv_rmsnorm_silu"), g.m, g.k, g.split);
  return gemv_w16<EL>(c, g, W16(0), W16(2), WN("gemv_rmsnorm_silu"));
}
template <FkElem EL>
int l_gemv_silu_w16(fkc_ctx* c, const Params& p, void* const* bufs) {
  FkGemv g = gemv_base(c, p);
  g.x = CF(1), g.y = F(2);
  g.up_off = p.u(6);
  g.prologue = FK_PRO_SILU;
  return gemv_w16<EL>(c, g, W16(0), nullptr, WN("gemv_silu"));
}
template <FkElem EL>
int l_gemv_silu_add_w16(fkc_ctx* c, const Params& p, void* const* bufs) {
  FkGemv g = gemv_base(c, p);
  g.x = CF(1), g.r = CF(2), g.y = F(3);
  g.ldr = p.u(6);
  g.up_off = p.u(7);
  g.prologue = FK_PRO_SILU;
  return gemv_w16<EL>(c, g, W16(0), nullptr, WN("gemv_silu_add"));
}
template <FkElem EL>
int l_gemv_scatter_w16(fkc_ctx* c, const Params& p, void* const* bufs) {
  if (!have_peers(c)) return fail(FKC_ERR_STATE, "%s: the context has no peer set.", WN("gemv_scatter"));
  FkGemv g = {};
  g.x = CF(1);
  g.n = p.u(0), g.k = p.u(1), g.m = p.u(2), g.split = p.u(3), g.ldx = p.u(4), g.xbuf = p.u(5);
  g.factor = 1.0f;
  g.pdl = c->pdl;
  g.prologue = FK_PRO_NONE;
  g.scatter = true;
  g.peers = c->peers;
  g.err = c->status;
  if (!fk_gemv_streams(g))
    return fail(FKC_ERR_ARGUMENT, "%s: m %u is past the streaming kernel's 4.", WN("gemv_scatter"), g.m);
  return gemv_w16<EL>(c, g, W16(0), nullptr, WN("gemv_scatter"));
}
template <FkElem EL>
int reduce_gemv_w16(fkc_ctx* c, const Params& p, void* const* bufs, bool silu, const char* name) {
  if (!have_peers(c)) return fail(FKC_ERR_STATE, "%s: the context has no peer set.", name);
  FkGemv g = {};
  g.x = CF(1), g.xout = F(3), g.y = F(4);
  g.n = p.u(0), g.k = p.u(1), g.m = p.u(2), g.split = p.u(3), g.ldx = p.u(4), g.ldy = p.u(5);
  g.eps = p.f(6), g.factor = p.f(7), g.xbuf = p.u(8);
  g.pdl = c->pdl;
  g.prologue = FK_PRO_REDUCE_RMSNORM;
  g.silu_pair = silu;
  g.peers = c->peers;
  g.err = c->status;
  if (g.ldx != g.k) return fail(FKC_ERR_ARGUMENT, "%s: the residual rows must be whole (ldr %u, k %u).", name, g.ldx, g.k);
  if (!fk_gemv_streams(g)) return fail(FKC_ERR_ARGUMENT, "%s: m %u is past the streaming kernel's 4.", name, g.m);
  return gemv_w16<EL>(c, g, W16(0), W16(2), name);
}
template <FkElem EL>
int l_gemv_reduce_rmsnorm_w16(fkc_ctx* c, const Params& p, void* const* bufs) {
  return reduce_gemv_w16<EL>(c, p, bufs, false, WN("gemv_reduce_rmsnorm"));
}
template <FkElem EL>
int l_gemv_reduce_rmsnorm_silu_w16(fkc_ctx* c, const Params& p, void* const* bufs) {
  return reduce_gemv_w16<EL>(c, p, bufs, true, WN("gemv_reduce_rmsnorm_silu"));
}
template <FkElem EL>
int l_gather_w16(fkc_ctx* c, const Params& p, void* const* bufs) {
  return launched(fk_launch_gather_w16(EL, W16(0), p.u(0), CU(1), p.u(1), p.f(2), F(2), c->pdl, c->stream),
                  WN("gather"));
}
template <FkElem EL>
int l_rmsnorm_rows_w16(fkc_ctx* c, const Params& p, void* const* bufs) {
  return launched(fk_launch_rmsnorm_rows_w16(EL, CF(0), W16(1), F(2), p.u(0), p.u(1), p.f(2), p.f(3), c->stream),
                  WN("rmsnorm_rows"));
}
template <FkElem EL>
int l_split_tf32_w16(fkc_ctx* c, const Params& p, void* const* bufs) {
  return launched(fk_launch_split_tf32_w16(EL, W16(0), F(1), F(2), p.u(0), c->stream), WN("split_tf32"));
}

template <FkElem EL>
int l_kv_store_kv16(fkc_ctx* c, const Params& p, void* const* bufs) {
  FkKvStore a = {};
  a.qkv = CF(0), a.cos_t = CF(1), a.sin_t = CF(2), a.pos = CU(3), a.slot = CU(4);
  a.m = p.u(0), a.kv_heads = p.u(1), a.d = p.u(2), a.length = p.u(3), a.rotated = p.u(4);
  a.ldq = p.u(5), a.k_off = p.u(6), a.v_off = p.u(7);
  a.pdl = c->pdl;
  if (a.rotated > a.d / 2) return fail(FKC_ERR_ARGUMENT, "%s: rotated %u is more than d/2.", KN("kv_store_ring"), a.rotated);
  return launched(fk_launch_kv_store16(a, EL, M16(5), M16(6), c->stream), KN("kv_store_ring"));
}
FkAttend attend_base(fkc_ctx* c, const Params& p, void* const* bufs) {
  FkAttend a = {};
  a.qkv = CF(0), a.cos_t = CF(1), a.sin_t = CF(2), a.pos = CU(3), a.slot = CU(4);
  a.m = p.u(0), a.heads = p.u(1), a.kv_heads = p.u(2), a.d = p.u(3), a.length = p.u(4), a.rotated = p.u(5);
  a.pdl = c->pdl;
  a.pf = c->l2pf, a.pf_bytes = c->l2pf_bytes;
  return a;
}
template <FkElem EL>
int l_attend_kv16(fkc_ctx* c, const Params& p, void* const* bufs) {
  FkAttend a = attend_base(c, p, bufs);
  a.part_m = F(7), a.part_l = F(8), a.part_acc = F(9);
  a.chunk = p.u(6), a.max_splits = p.u(7), a.ldq = p.u(8), a.q_off = p.u(9);
  a.scale = p.f(10);
  if (a.kv_heads == 0 || a.heads % a.kv_heads != 0)
    return fail(FKC_ERR_ARGUMENT, "%s: %u heads do not share %u KV heads in groups.", KN("attend_split"), a.heads,
                a.kv_heads);
  return launched(fk_launch_attend16(a, EL, W16(5), W16(6), c->stream), KN("attend_split"));
}
template <FkElem EL>
int l_attend_decode_kv16(fkc_ctx* c, const Params& p, void* const* bufs) {
  FkAttend a = attend_base(c, p, bufs);
  a.part_m = F(7), a.part_l = F(8), a.part_acc = F(9);
  a.chunk = p.u(6), a.max_splits = p.u(7), a.ldq = p.u(8), a.q_off = p.u(9);
  a.scale = p.f(12);
  if (a.kv_heads == 0 || a.heads % a.kv_heads != 0)
    return fail(FKC_ERR_ARGUMENT, "%s: %u heads do not share %u KV heads in groups.", KN("attend_decode"), a.heads,
                a.kv_heads);
  if (a.rotated > a.d / 2) return fail(FKC_ERR_ARGUMENT, "%s: rotated %u is more than d/2.", KN("attend_decode"), a.rotated);
  return launched(fk_launch_attend_decode16(a, EL, p.u(10), p.u(11), M16(5), M16(6), c->stream), KN("attend_decode"));
}
template <FkElem EL>
int l_attend_prompt_kv16(fkc_ctx* c, const Params& p, void* const* bufs) {
  FkAttend a = attend_base(c, p, bufs);
  a.ldq = p.u(6), a.q_off = p.u(7);
  a.scale = p.f(10);
  if (a.kv_heads == 0 || a.heads % a.kv_heads != 0)
    return fail(FKC_ERR_ARGUMENT, "%s: %u heads do not share %u KV heads in groups.", KN("attend_prompt"), a.heads,
                a.kv_heads);
  if (a.rotated > a.d / 2) return fail(FKC_ERR_ARGUMENT, "%s: rotated %u is more than d/2.", KN("attend_prompt"), a.rotated);
  if (p.u(9) >= a.length)
    return fail(FKC_ERR_ARGUMENT, "%s: max_pos %u is not within the ring's length %u.", KN("attend_prompt"), p.u(9),
                a.length);
  return launched(fk_launch_attend_prompt16(a, EL, W16(5), W16(6), F(7), p.u(8), p.u(9), c->stream),
                  KN("attend_prompt"));
}

// ---- routed experts ------------------------------------------------------
// route_topk: x ids ws | m n k ldx; route_topk_scaled: x scale ids ws | m n k ldx
int l_route_topk(fkc_ctx* c, const Params& p, void* const* bufs) {
  return launched(fk_launch_route_topk(CF(0), p.u(0), p.u(1), p.u(2), p.u(3), nullptr, FK_F32, U(1), F(2), c->pdl,
                                       c->stream),
                  "route_topk");
}
int l_route_topk_scaled(fkc_ctx* c, const Params& p, void* const* bufs) {
  return launched(fk_launch_route_topk(CF(0), p.u(0), p.u(1), p.u(2), p.u(3), bufs[1], FK_F32, U(2), F(3), c->pdl,
                                       c->stream),
                  "route_topk_scaled");
}
// gemv_routed: table ids x y | entries n kk m k split ldx ldy per_rank
int gemv_routed(fkc_ctx* c, const Params& p, void* const* bufs, FkElem el, const char* name) {
  if (p.u(8) > 1) return fail(FKC_ERR_ARGUMENT, "%s: per_rank is %u, not 0 or 1.", name, p.u(8));
  return launched(fk_launch_gemv_routed(bufs[0], el, p.u(0), p.u(1), p.u(2), CU(1), p.u(3), p.u(4), CF(2), p.u(6),
                                        p.u(8) != 0, p.u(5), F(3), p.u(7), c->pdl, c->stream),
                  name);
}
int l_gemv_routed(fkc_ctx* c, const Params& p, void* const* bufs) {
  return gemv_routed(c, p, bufs, FK_F32, "gemv_routed");
}
// route_topk_scaled with 16-bit expert scales (the model's weights' type).
template <FkElem EL>
int l_route_topk_scaled_w16(fkc_ctx* c, const Params& p, void* const* bufs) {
  return launched(fk_launch_route_topk(CF(0), p.u(0), p.u(1), p.u(2), p.u(3), bufs[1], EL, U(2), F(3), c->pdl,
                                       c->stream),
                  WN("route_topk_scaled"));
}
template <FkElem EL>
int l_gemv_routed_w16(fkc_ctx* c, const Params& p, void* const* bufs) {
  return gemv_routed(c, p, bufs, EL, WN("gemv_routed"));
}
// gated_gelu: x y | segments f
int l_gated_gelu(fkc_ctx* c, const Params& p, void* const* bufs) {
  return launched(fk_launch_gated_gelu(CF(0), p.u(0), p.u(1), F(1), c->pdl, c->stream), "gated_gelu");
}
// combine_ranks_add: r ws segs y | m k d
int l_combine_ranks_add(fkc_ctx* c, const Params& p, void* const* bufs) {
  return launched(fk_launch_combine_ranks_add(CF(0), CF(1), CF(2), p.u(0), p.u(1), p.u(2), F(3), c->pdl, c->stream),
                  "combine_ranks_add");
}

// ---- paged KV caches: each row's block table (indices), the blocks reached
// through the caches' tables of block addresses (bound after the buffers,
// as the reference's ABI orders tables: Abi.hs:136-159) -------------------
// kv_store_paged: qkv cos sin pos table | tables k_cache v_cache
//   | m kv_heads d block_size table_len blocks rotated ldq k_off v_off
int kv_store_paged(fkc_ctx* c, const Params& p, void* const* bufs, FkElem el, const char* name) {
  FkKvStore a = {};
  a.qkv = CF(0), a.cos_t = CF(1), a.sin_t = CF(2), a.pos = CU(3);
  a.m = p.u(0), a.kv_heads = p.u(1), a.d = p.u(2), a.rotated = p.u(6);
  a.ldq = p.u(7), a.k_off = p.u(8), a.v_off = p.u(9);
  a.pdl = c->pdl;
  const FkPaged pg = {CU(4), p.u(3), p.u(4), p.u(5)};
  if (a.rotated > a.d / 2) return fail(FKC_ERR_ARGUMENT, "%s: rotated %u is more than d/2.", name, a.rotated);
  return launched(fk_launch_kv_store_paged(a, pg, bufs[5], bufs[6], el, c->stream), name);
}
int l_kv_store_paged(fkc_ctx* c, const Params& p, void* const* bufs) {
  return kv_store_paged(c, p, bufs, FK_F32, "kv_store_paged");
}
template <FkElem EL>
int l_kv_store_paged_kv16(fkc_ctx* c, const Params& p, void* const* bufs) {
  return kv_store_paged(c, p, bufs, EL, KN("kv_store_paged"));
}
// attend_split_paged: qkv cos sin pos table part_m part_l part_acc | tables k_cache v_cache
//   | m heads kv_heads d block_size table_len blocks rotated chunk max_splits ldq q_off scale
int attend_paged(fkc_ctx* c, const Params& p, void* const* bufs, FkElem el, const char* name) {
  FkAttend a = {};
  a.qkv = CF(0), a.cos_t = CF(1), a.sin_t = CF(2), a.pos = CU(3);
  a.part_m = F(5), a.part_l = F(6), a.part_acc = F(7);
  a.m = p.u(0), a.heads = p.u(1), a.kv_heads = p.u(2), a.d = p.u(3), a.rotated = p.u(7);
  a.chunk = p.u(8), a.max_splits = p.u(9), a.ldq = p.u(10), a.q_off = p.u(11);
  a.scale = p.f(12);
  a.pdl = c->pdl;
  a.pf = c->l2pf, a.pf_bytes = c->l2pf_bytes;
  const FkPaged pg = {CU(4), p.u(4), p.u(5), p.u(6)};
  if (a.kv_heads == 0 || a.heads % a.kv_heads != 0)
    return fail(FKC_ERR_ARGUMENT, "%s: %u heads do not share %u KV heads in groups.", name, a.heads, a.kv_heads);
  if (a.rotated > a.d / 2) return fail(FKC_ERR_ARGUMENT, "%s: rotated %u is more than d/2.", name, a.rotated);
  return launched(fk_launch_attend_paged(a, pg, bufs[8], bufs[9], el, c->stream), name);
}
int l_attend_paged(fkc_ctx* c, const Params& p, void* const* bufs) {
  return attend_paged(c, p, bufs, FK_F32, "attend_split_paged");
}
template <FkElem EL>
int l_attend_paged_kv16(fkc_ctx* c, const Params& p, void* const* bufs) {
  return attend_paged(c, p, bufs, EL, KN("attend_split_paged"));
}
// attend_decode_paged: qkv cos sin pos table part_m part_l part_acc | tables k_cache v_cache
//   | m heads kv_heads d block_size table_len blocks rotated chunk max_splits ldq q_off k_off v_off scale
// The KV store folded into the split attention; every block-table entry
// distinct (no row reads what another row stores).
int attend_decode_paged(fkc_ctx* c, const Params& p, void* const* bufs, FkElem el, const char* name) {
  FkAttend a = {};
  a.qkv = CF(0), a.cos_t = CF(1), a.sin_t = CF(2), a.pos = CU(3);
  a.part_m = F(5), a.part_l = F(6), a.part_acc = F(7);
  a.m = p.u(0), a.heads = p.u(1), a.kv_heads = p.u(2), a.d = p.u(3), a.rotated = p.u(7);
  a.chunk = p.u(8), a.max_splits = p.u(9), a.ldq = p.u(10), a.q_off = p.u(11);
  a.scale = p.f(14);
  a.pdl = c->pdl;
  a.pf = c->l2pf, a.pf_bytes = c->l2pf_bytes;
  const FkPaged pg = {CU(4), p.u(4), p.u(5), p.u(6)};
  if (a.kv_heads == 0 || a.heads % a.kv_heads != 0)
    return fail(FKC_ERR_ARGUMENT, "%s: %u heads do not share %u KV heads in groups.", name, a.heads, a.kv_heads);
  if (a.rotated > a.d / 2) return fail(FKC_ERR_ARGUMENT, "%s: rotated %u is more than d/2.", name, a.rotated);
  return launched(fk_launch_attend_decode_paged(a, pg, bufs[8], bufs[9], el, p.u(12), p.u(13), c->stream), name);
}
int l_attend_decode_paged(fkc_ctx* c, const Params& p, void* const* bufs) {
  return attend_decode_paged(c, p, bufs, FK_F32, "attend_decode_paged");
}
template <FkElem EL>
int l_attend_decode_paged_kv16(fkc_ctx* c, const Params& p, void* const* bufs) {
  return attend_decode_paged(c, p, bufs, EL, KN("attend_decode_paged"));
}
// attend_prompt_paged: qkv cos sin pos table out | tables k_cache v_cache
//   | m heads kv_heads d block_size table_len blocks rotated ldq q_off ldo max_pos scale
// A prompt's rows of one sequence: row 0's block table serves them all.
int attend_prompt_paged(fkc_ctx* c, const Params& p, void* const* bufs, FkElem el, const char* name) {
  FkAttend a = {};
  a.qkv = CF(0), a.cos_t = CF(1), a.sin_t = CF(2), a.pos = CU(3);
  a.m = p.u(0), a.heads = p.u(1), a.kv_heads = p.u(2), a.d = p.u(3), a.rotated = p.u(7);
  a.ldq = p.u(8), a.q_off = p.u(9);
  a.scale = p.f(12);
  a.pdl = c->pdl;
  const FkPaged pg = {CU(4), p.u(4), p.u(5), p.u(6)};
  if (a.kv_heads == 0 || a.heads % a.kv_heads != 0)
    return fail(FKC_ERR_ARGUMENT, "%s: %u heads do not share %u KV heads in groups.", name, a.heads, a.kv_heads);
  if (a.rotated > a.d / 2) return fail(FKC_ERR_ARGUMENT, "%s: rotated %u is more than d/2.", name, a.rotated);
  if ((uint64_t)p.u(11) >= (uint64_t)pg.table_len * pg.block_size)
    return fail(FKC_ERR_ARGUMENT, "%s: max_pos %u is past the block table's %u positions.", name, p.u(11),
                pg.table_len * pg.block_size);
  return launched(fk_launch_attend_prompt_paged(a, pg, bufs[6], bufs[7], el, F(5), p.u(10), p.u(11), c->stream),
                  name);
}
int l_attend_prompt_paged(fkc_ctx* c, const Params& p, void* const* bufs) {
  return attend_prompt_paged(c, p, bufs, FK_F32, "attend_prompt_paged");
}
template <FkElem EL>
int l_attend_prompt_paged_kv16(fkc_ctx* c, const Params& p, void* const* bufs) {
  return attend_prompt_paged(c, p, bufs, EL, KN("attend_prompt_paged"));
}

#undef W16
#undef M16
#undef WN
#undef KN

#undef F
#undef CF
#undef CU
#undef U

constexpr uint32_t kMax = 4294967295u;

ParamSpec dim(const char* n, uint32_t lo, uint32_t hi, uint32_t mult = 1) { return {n, "u32", true, lo, hi, mult}; }
ParamSpec u32(const char* n) { return {n, "u32", false, 0, 0, 0}; }
ParamSpec f32(const char* n) { return {n, "f32", false, 0, 0, 0}; }

std::vector<KernelSpec> make_table() {
  std::vector<KernelSpec> t;
  // m: any batch; the launchers take up to 4 rows streaming, up to 64 in the
  // packed batched kernel, and past that 32 rows a launch of the chunked one.
  auto gemv_dims = std::vector<ParamSpec>{dim("n", 1, 1048576), dim("k", 4, 65536, 4), dim("m", 1, 65535),
                                          dim("split", 1, 8),   u32("ldx"),           u32("ldy")};
  auto with = [](std::vector<ParamSpec> a, std::initializer_list<ParamSpec> b) {
    a.insert(a.end(), b.begin(), b.end());
    return a;
  };
  t.push_back({"reduce_groups", 256, {{"x", "read", "f32"}, {"partials", "write", "f32"}}, {dim("n", 1, 2147483648u)},
               l_reduce_groups});
  t.push_back({"reduce_final", 256, {{"partials", "read", "f32"}, {"y", "write", "f32"}}, {dim("count", 1, 16777216)},
               l_reduce_final});
  t.push_back({"rmsnorm_rows",
               256,
               {{"x", "read", "f32"}, {"gamma", "read", "f32"}, {"y", "write", "f32"}},
               {dim("rows", 1, 1048576), dim("h", 4, 16384, 4), f32("eps"), f32("factor")},
               l_rmsnorm_rows});
  t.push_back({"softmax_rows",
               256,
               {{"x", "read", "f32"}, {"y", "write", "f32"}},
               {dim("rows", 1, 1048576), dim("h", 4, 16384, 4)},
               l_softmax_rows});
  t.push_back({"gemv", 256, {{"w", "read", "f32"}, {"x", "read", "f32"}, {"y", "write", "f32"}}, gemv_dims, l_gemv});
  t.push_back({"gemv_add",
               256,
               {{"w", "read", "f32"}, {"x", "read", "f32"}, {"r", "read", "f32"}, {"y", "write", "f32"}},
               with(gemv_dims, {u32("ldr")}),
               l_gemv_add});
  t.push_back({"gemv_rmsnorm",
               256,
               {{"w", "read", "f32"}, {"x", "read", "f32"}, {"gamma", "read", "f32"}, {"y", "write", "f32"}},
               with(gemv_dims, {f32("eps"), f32("factor")}),
               l_gemv_rmsnorm});
  t.push_back({"gemv_rmsnorm_silu",
               512,
               {{"w", "read", "f32"}, {"x", "read", "f32"}, {"gamma", "read", "f32"}, {"y", "write", "f32"}},
               with(gemv_dims, {f32("eps"), f32("factor")}),
               l_gemv_rmsnorm_silu});
  t.push_back({"gemv_silu",
               256,
               {{"w", "read", "f32"}, {"x", "read", "f32"}, {"y", "write", "f32"}},
               with(gemv_dims, {u32("up_off")}),
               l_gemv_silu});
  t.push_back({"gemv_silu_add",
               256,
               {{"w", "read", "f32"}, {"x", "read", "f32"}, {"r", "read", "f32"}, {"y", "write", "f32"}},
               with(gemv_dims, {u32("ldr"), u32("up_off")}),
               l_gemv_silu_add});
  t.push_back({"kv_store_ring",
               64,
               {{"qkv", "read", "f32"},
                {"cos", "read", "f32"},
                {"sin", "read", "f32"},
                {"pos", "read", "u32"},
                {"slot", "read", "u32"},
                {"k_cache", "read_write", "f32"},
                {"v_cache", "read_write", "f32"}},
               {dim("m", 1, 65535), dim("kv_heads", 1, 1024), dim("d", 2, 2048, 2), dim("length", 1, kMax),
                u32("rotated"), u32("ldq"), u32("k_off"), u32("v_off")},
               l_kv_store});
  t.push_back({"attend_split",
               128,
               {{"qkv", "read", "f32"},
                {"cos", "read", "f32"},
                {"sin", "read", "f32"},
                {"pos", "read", "u32"},
                {"slot", "read", "u32"},
                {"k_cache", "read", "f32"},
                {"v_cache", "read", "f32"},
                {"part_m", "write", "f32"},
                {"part_l", "write", "f32"},
                {"part_acc", "write", "f32"}},
               {dim("m", 1, 16384), dim("heads", 1, 1024), dim("kv_heads", 1, 1024), dim("d", 128, 128),
                dim("length", 1, kMax), u32("rotated"), dim("chunk", 1, 256), dim("max_splits", 1, 65535), u32("ldq"),
                u32("q_off"), f32("scale")},
               l_attend});
  t.push_back({"attend_decode",
               128,
               {{"qkv", "read", "f32"},
                {"cos", "read", "f32"},
                {"sin", "read", "f32"},
                {"pos", "read", "u32"},
                {"slot", "read", "u32"},
                {"k_cache", "read_write", "f32"},
                {"v_cache", "read_write", "f32"},
                {"part_m", "write", "f32"},
                {"part_l", "write", "f32"},
                {"part_acc", "write", "f32"}},
               {dim("m", 1, 64), dim("heads", 1, 1024), dim("kv_heads", 1, 1024), dim("d", 128, 128),
                dim("length", 1, kMax), u32("rotated"), dim("chunk", 1, 256), dim("max_splits", 1, 65535), u32("ldq"),
                u32("q_off"), u32("k_off"), u32("v_off"), f32("scale")},
               l_attend_decode});
  t.push_back({"attend_prompt",
               256,
               {{"qkv", "read", "f32"},
                {"cos", "read", "f32"},
                {"sin", "read", "f32"},
                {"pos", "read", "u32"},
                {"slot", "read", "u32"},
                {"k_cache", "read", "f32"},
                {"v_cache", "read", "f32"},
                {"out", "write", "f32"}},
               {dim("m", 1, 65535), dim("heads", 1, 1024), dim("kv_heads", 1, 1024), dim("d", 128, 128),
                dim("length", 1, kMax), u32("rotated"), u32("ldq"), u32("q_off"), u32("ldo"), dim("max_pos", 0, kMax - 1),
                f32("scale")},
               l_attend_prompt});
  t.push_back({"attend_combine",
               128,
               {{"part_m", "read", "f32"},
                {"part_l", "read", "f32"},
                {"part_acc", "read", "f32"},
                {"pos", "read", "u32"},
                {"out", "write", "f32"}},
               {dim("m", 1, 65535), dim("heads", 1, 1024), dim("d", 1, 1024), dim("chunk", 1, 256),
                dim("max_splits", 1, 65535), u32("ldo")},
               l_combine});
  t.push_back({"gather",
               256,
               {{"table", "read", "f32"}, {"tokens", "read", "u32"}, {"y", "write", "f32"}},
               {dim("width", 4, 1048576, 4), dim("m", 1, 65535), f32("factor")},
               l_gather});
  t.push_back({"argmax",
               1024,
               {{"x", "read", "f32"}, {"ids", "write", "u32"}},
               {dim("m", 1, 65535), dim("n", 1, kMax), u32("ldx")},
               l_argmax});
  t.push_back({"rope",
               64,
               {{"x", "read", "f32"}, {"pos", "read", "u32"}, {"cos", "read", "f32"}, {"sin", "read", "f32"},
                {"y", "write", "f32"}},
               {dim("m", 1, 65535), dim("heads", 1, 65535), dim("d", 2, 2048, 2), u32("rotated"), u32("ldx"),
                u32("ldy")},
               l_rope});
  t.push_back({"split_tf32",
               256,
               {{"x", "read", "f32"}, {"hi", "write", "f32"}, {"lo", "write", "f32"}},
               {dim("n", 1, kMax)},
               l_split_tf32});
  t.push_back({"gemm_tf32x3",
               192,
               {{"a", "read", "f32"},
                {"a_hi", "read_write", "f32"},
                {"a_lo", "read_write", "f32"},
                {"w_hi", "read", "f32"},
                {"w_lo", "read", "f32"},
                {"c", "write", "f32"}},
               {dim("M", 1, 1048576), dim("N", 1, 1048576), dim("K", 32, 1048576, 32), u32("ldc")},
               l_gemm_tf32x3});
  t.push_back({"gemm_tf32x3w",
               192,
               {{"a", "read", "f32"},
                {"a_hi", "read_write", "f32"},
                {"a_lo", "read_write", "f32"},
                {"w", "read", "f32"},
                {"c", "write", "f32"}},
               {dim("M", 1, 1048576), dim("N", 1, 1048576), dim("K", 16, 1048576, 16), u32("ldc")},
               l_gemm_tf32x3w});
  t.push_back({"argmax_pairs",
               1024,
               {{"x", "read", "f32"}, {"pairs", "write", "u32"}},
               {dim("m", 1, 65535), dim("n", 1, kMax), u32("ldx"), u32("offset")},
               l_argmax_pairs});
  t.push_back({"argmax_pick",
               256,
               {{"pairs", "read", "u32"}, {"ids", "write", "u32"}},
               {dim("shards", 1, 64), dim("m", 1, 65535)},
               l_argmax_pick});
  t.push_back({"argmax_scatter",
               1024,
               {{"x", "read", "f32"}},
               {dim("m", 1, 4), dim("n", 1, kMax), u32("ldx"), u32("offset")},
               l_argmax_scatter});
  t.push_back({"argmax_gather_pick", 256, {{"ids", "write", "u32"}}, {dim("m", 1, 4)}, l_argmax_gather_pick});
  t.push_back({"gemv_scatter",
               512,
               {{"w", "read", "f32"}, {"x", "read", "f32"}},
               {dim("n", 1, 65536), dim("k", 4, 65536, 4), dim("m", 1, 4), dim("split", 1, 8), u32("ldx"),
                dim("xbuf", 0, 1)},
               l_gemv_scatter});
  for (int silu = 0; silu < 2; ++silu)
    t.push_back({silu ? "gemv_reduce_rmsnorm_silu" : "gemv_reduce_rmsnorm",
                 512,
                 {{"w", "read", "f32"},
                  {"r", "read", "f32"},
                  {"gamma", "read", "f32"},
                  {"xout", "write", "f32"},
                  {"y", "write", "f32"}},
                 {dim("n", 1, 1048576), dim("k", 4, 16384, 4), dim("m", 1, 4), dim("split", 1, 8), u32("ldr"),
                  u32("ldy"), f32("eps"), f32("factor"), dim("xbuf", 0, 1)},
                 silu ? l_gemv_reduce_rmsnorm_silu : l_gemv_reduce_rmsnorm});
  t.push_back({"advance",
               256,
               {{"ids", "read", "u32"}, {"tokens", "write", "u32"}, {"pos", "read_write", "u32"}},
               {dim("m", 1, 65535)},
               l_advance});
  t.push_back({"add",
               256,
               {{"a", "read", "f32"}, {"b", "read", "f32"}, {"y", "write", "f32"}},
               {dim("n", 1, kMax)},
               l_add});
  t.push_back({"silu_mul",
               256,
               {{"a", "read", "f32"}, {"b", "read", "f32"}, {"y", "write", "f32"}},
               {dim("n", 1, kMax)},
               l_silu_mul});
  t.push_back({"silu_pairs", 256, {{"x", "read", "f32"}, {"y", "write", "f32"}}, {dim("n", 1, kMax)}, l_silu_pairs});
  t.push_back({"gemv_bf16",
               512,
               {{"w", "read", "bf16"}, {"x", "read", "bf16"}, {"y", "write", "bf16"}},
               {dim("n", 1, 1048576), dim("k", 4, 65536, 4), dim("m", 1, 16), dim("pack", 4, 16, 4), dim("split", 1, 16),
                u32("ldx"), u32("ldy")},
               l_gemv_bf16});
  // Paged caches (Graph.hs:144-152): a row's block table instead of its slot.
  t.push_back({"kv_store_paged",
               64,
               {{"qkv", "read", "f32"},
                {"cos", "read", "f32"},
                {"sin", "read", "f32"},
                {"pos", "read", "u32"},
                {"table", "read", "u32"}},
               {dim("m", 1, 65535), dim("kv_heads", 1, 1024), dim("d", 2, 2048, 2), dim("block_size", 1, 65536),
                dim("table_len", 1, kMax), dim("blocks", 1, kMax), u32("rotated"), u32("ldq"), u32("k_off"),
                u32("v_off")},
               l_kv_store_paged});
  t.back().tables = {{"k_cache", "read_write", "f32"}, {"v_cache", "read_write", "f32"}};
  t.push_back({"attend_split_paged",
               128,
               {{"qkv", "read", "f32"},
                {"cos", "read", "f32"},
                {"sin", "read", "f32"},
                {"pos", "read", "u32"},
                {"table", "read", "u32"},
                {"part_m", "write", "f32"},
                {"part_l", "write", "f32"},
                {"part_acc", "write", "f32"}},
               {dim("m", 1, 16384), dim("heads", 1, 1024), dim("kv_heads", 1, 1024), dim("d", 128, 128),
                dim("block_size", 1, 65536), dim("table_len", 1, kMax), dim("blocks", 1, kMax), u32("rotated"),
                dim("chunk", 1, 256), dim("max_splits", 1, 65535), u32("ldq"), u32("q_off"), f32("scale")},
               l_attend_paged});
  t.back().tables = {{"k_cache", "read", "f32"}, {"v_cache", "read", "f32"}};
  t.push_back({"attend_decode_paged",
               128,
               {{"qkv", "read", "f32"},
                {"cos", "read", "f32"},
                {"sin", "read", "f32"},
                {"pos", "read", "u32"},
                {"table", "read", "u32"},
                {"part_m", "write", "f32"},
                {"part_l", "write", "f32"},
                {"part_acc", "write", "f32"}},
               {dim("m", 1, 64), dim("heads", 1, 1024), dim("kv_heads", 1, 1024), dim("d", 128, 128),
                dim("block_size", 1, 65536), dim("table_len", 1, kMax), dim("blocks", 1, kMax), u32("rotated"),
                dim("chunk", 1, 256), dim("max_splits", 1, 65535), u32("ldq"), u32("q_off"), u32("k_off"),
                u32("v_off"), f32("scale")},
               l_attend_decode_paged});
  t.back().tables = {{"k_cache", "read_write", "f32"}, {"v_cache", "read_write", "f32"}};
  t.push_back({"attend_prompt_paged",
               256,
               {{"qkv", "read", "f32"},
                {"cos", "read", "f32"},
                {"sin", "read", "f32"},
                {"pos", "read", "u32"},
                {"table", "read", "u32"},
                {"out", "write", "f32"}},
               {dim("m", 1, 65535), dim("heads", 1, 1024), dim("kv_heads", 1, 1024), dim("d", 128, 128),
                dim("block_size", 1, 65536), dim("table_len", 1, kMax), dim("blocks", 1, kMax), u32("rotated"),
                u32("ldq"), u32("q_off"), u32("ldo"), dim("max_pos", 0, kMax - 1), f32("scale")},
               l_attend_prompt_paged});
  t.back().tables = {{"k_cache", "read", "f32"}, {"v_cache", "read", "f32"}};
  // Routed experts (Graph.hs:306-340).
  t.push_back({"route_topk",
               32,
               {{"x", "read", "f32"}, {"ids", "write", "u32"}, {"ws", "write", "f32"}},
               {dim("m", 1, 65535), dim("n", 1, 1024), dim("k", 1, 8), u32("ldx")},
               l_route_topk});
  t.push_back({"route_topk_scaled",
               32,
               {{"x", "read", "f32"}, {"scale", "read", "f32"}, {"ids", "write", "u32"}, {"ws", "write", "f32"}},
               {dim("m", 1, 65535), dim("n", 1, 1024), dim("k", 1, 8), u32("ldx")},
               l_route_topk_scaled});
  t.push_back({"gemv_routed",
               256,
               {{"table", "read", "f32"}, {"ids", "read", "u32"}, {"x", "read", "f32"}, {"y", "write", "f32"}},
               {dim("entries", 1, 4096), dim("n", 1, 1048576), dim("kk", 4, 65536, 4), dim("m", 1, 65535),
                dim("k", 1, 8), dim("split", 1, 8), u32("ldx"), u32("ldy"), u32("per_rank")},
               l_gemv_routed});
  t.push_back({"gated_gelu", 256, {{"x", "read", "f32"}, {"y", "write", "f32"}},
               {dim("segments", 1, kMax), dim("f", 1, kMax)}, l_gated_gelu});
  t.push_back({"combine_ranks_add",
               256,
               {{"r", "read", "f32"}, {"ws", "read", "f32"}, {"segs", "read", "f32"}, {"y", "write", "f32"}},
               {dim("m", 1, 65535), dim("k", 1, 8), dim("d", 1, kMax)},
               l_combine_ranks_add});
  // The 16-bit forms: an f32 entry's parameters with some buffers bf16 or
  // f16 (the model's weights, or its KV caches) and their own launchers.
  struct Variant {
    const char* base;
    const char* name;
    std::vector<const char*> retyped;
    LaunchFn launch;
    const char* type;
  };
#define W_FORMS(base, fn, ...)                                       \
  {base, base "_wbf16", {__VA_ARGS__}, fn<FK_BF16>, "bf16"}, {       \
    base, base "_wf16", {__VA_ARGS__}, fn<FK_F16>, "f16"             \
  }
#define KV_FORMS(base, fn)                                                        \
  {base, base "_kvbf16", {"k_cache", "v_cache"}, fn<FK_BF16>, "bf16"}, {          \
    base, base "_kvf16", {"k_cache", "v_cache"}, fn<FK_F16>, "f16"                \
  }
  const std::vector<Variant> variants = {
      W_FORMS("gemv", l_gemv_w16, "w"),
      W_FORMS("gemv_add", l_gemv_add_w16, "w"),
      W_FORMS("gemv_rmsnorm", l_gemv_rmsnorm_w16, "w", "gamma"),
      W_FORMS("gemv_rmsnorm_silu", l_gemv_rmsnorm_silu_w16, "w", "gamma"),
      W_FORMS("gemv_silu", l_gemv_silu_w16, "w"),
      W_FORMS("gemv_silu_add", l_gemv_silu_add_w16, "w"),
      W_FORMS("gemv_scatter", l_gemv_scatter_w16, "w"),
      W_FORMS("gemv_reduce_rmsnorm", l_gemv_reduce_rmsnorm_w16, "w", "gamma"),
      W_FORMS("gemv_reduce_rmsnorm_silu", l_gemv_reduce_rmsnorm_silu_w16, "w", "gamma"),
      W_FORMS("gather", l_gather_w16, "table"),
      W_FORMS("rmsnorm_rows", l_rmsnorm_rows_w16, "gamma"),
      W_FORMS("split_tf32", l_split_tf32_w16, "x"),
      W_FORMS("gemv_routed", l_gemv_routed_w16, "table"),
      W_FORMS("route_topk_scaled", l_route_topk_scaled_w16, "scale"),
      KV_FORMS("kv_store_ring", l_kv_store_kv16),
      KV_FORMS("attend_split", l_attend_kv16),
      KV_FORMS("attend_decode", l_attend_decode_kv16),
      KV_FORMS("attend_prompt", l_attend_prompt_kv16),
      KV_FORMS("kv_store_paged", l_kv_store_paged_kv16),
      KV_FORMS("attend_split_paged", l_attend_paged_kv16),
      KV_FORMS("attend_decode_paged", l_attend_decode_paged_kv16),
      KV_FORMS("attend_prompt_paged", l_attend_prompt_paged_kv16),
  };
#undef W_FORMS
#undef KV_FORMS
  for (const Variant& v : variants) {
    KernelSpec k;
    bool found = false;
    for (const KernelSpec& b : t)
      if (strcmp(b.name, v.base) == 0) {
        k = b;
        found = true;
      }
    if (!found) continue;
    k.name = v.name;
    k.launch = v.launch;
    for (std::vector<BufSpec>* list : {&k.bufs, &k.tables})
      for (BufSpec& b : *list)
        for (const char* r : v.retyped)
          if (strcmp(b.name, r) == 0) b.type = v.type;
    t.push_back(k);
  }
  // The C layout (Abi.hs:113-133) and the canonical text (Abi.hs:136-159).
  for (auto& k : t) {
    uint32_t off = 0, align = 1;
    for (auto& p : k.params) {
      const uint32_t size = 4;
      off = (off + size - 1) / size * size;
      k.offsets.push_back(off);
      off += size;
      if (size > align) align = size;
    }
    k.params_size = k.params.empty() ? 0 : (off + align - 1) / align * align;
    std::string a = "abi 1\n";
    for (auto& b : k.bufs) a += std::string("buffer ") + b.name + " " + b.access + " " + b.type + " align 16\n";
    // A read-only table's line names no access (Abi.hs:143-152).
    for (auto& b : k.tables)
      a += std::string("table ") + b.name + (strcmp(b.access, "read") == 0 ? "" : std::string(" ") + b.access) + " " +
           b.type + " align 16\n";
    for (size_t i = 0; i < k.params.size(); ++i)
      a += std::string("param ") + k.params[i].name + " " + k.params[i].type + " at " + std::to_string(k.offsets[i]) +
           "\n";
    a += "params size " + std::to_string(k.params_size) + "\n";
    k.abi = a;
    k.hash = fnv1a(a.data(), a.size());
  }
  return t;
}

const std::vector<KernelSpec>& table() {
  static std::vector<KernelSpec> t = make_table();
  return t;
}

std::string range_text(const ParamSpec& p) {
  std::string s = std::to_string(p.lo) + ".." + std::to_string(p.hi);
  if (p.mult > 1) s += " multiple of " + std::to_string(p.mult);
  return s;
}

}  // namespace

extern "C" uint64_t fkc_fnv1a64(const void* bytes, size_t n) { return fnv1a(bytes, n); }

extern "C" int fkc_kernel_count(void) { return (int)table().size(); }

extern "C" int fkc_kernel_describe(int id, const char** name, const char** abi, uint64_t* hash, uint32_t* threads,
                                   uint32_t* params_size, uint32_t* buffers) {
  const auto& t = table();
  if (id < 0 || id >= (int)t.size()) return fail(FKC_ERR_ARGUMENT, "fkc_kernel_describe: no kernel %d.", id);
  const KernelSpec& k = t[id];
  if (name) *name = k.name;
  if (abi) *abi = k.abi.c_str();
  if (hash) *hash = k.hash;
  if (threads) *threads = k.threads;
  if (params_size) *params_size = k.params_size;
  if (buffers) *buffers = (uint32_t)(k.bufs.size() + k.tables.size());
  return FKC_OK;
}

extern "C" int fkc_kernel_find(const char* name, uint64_t abi_hash, int* id) {
  if (!name || !id) return fail(FKC_ERR_ARGUMENT, "fkc_kernel_find: null argument.");
  const auto& t = table();
  for (size_t i = 0; i < t.size(); ++i) {
    if (strcmp(t[i].name, name) != 0) continue;
    if (t[i].hash != abi_hash)
      return fail(FKC_ERR_ARGUMENT,
                  "The kernel %s has another ABI than the target's %s: hash 0x%016llx where the target has "
                  "0x%016llx.",
                  name, t[i].name, (unsigned long long)abi_hash, (unsigned long long)t[i].hash);
    *id = (int)i;
    return FKC_OK;
  }
  return fail(FKC_ERR_ARGUMENT, "The target has no kernel %s.", name);
}

extern "C" int fkc_launch(fkc_ctx* c, int kernel, const void* params, size_t params_len, void* const* bufs,
                          int nbufs) {
  if (!c) return fail(FKC_ERR_ARGUMENT, "fkc_launch: null context.");
  const auto& t = table();
  if (kernel < 0 || kernel >= (int)t.size()) return fail(FKC_ERR_ARGUMENT, "fkc_launch: no kernel %d.", kernel);
  const KernelSpec& k = t[kernel];
  if (params_len != k.params_size)
    return fail(FKC_ERR_ARGUMENT, "%s: the parameter struct is %zu bytes, not %u.", k.name, params_len,
                k.params_size);
  const int nb = (int)k.bufs.size(), nt = (int)k.tables.size();
  if (nbufs != nb + nt) {
    if (nt) return fail(FKC_ERR_ARGUMENT, "%s: %d bindings, not %d buffers and %d tables.", k.name, nbufs, nb, nt);
    return fail(FKC_ERR_ARGUMENT, "%s: %d buffers bound, not %d.", k.name, nbufs, nb);
  }
  for (int i = 0; i < nb; ++i)
    if (!bufs[i] || ((uintptr_t)bufs[i] & 15u))
      return fail(FKC_ERR_ARGUMENT, "%s: buffer %s is %s.", k.name, k.bufs[i].name,
                  bufs[i] ? "not aligned to 16 bytes" : "null");
  for (int i = 0; i < nt; ++i)  // a table is an array of 8-byte addresses
    if (!bufs[nb + i] || ((uintptr_t)bufs[nb + i] & 7u))
      return fail(FKC_ERR_ARGUMENT, "%s: table %s is %s.", k.name, k.tables[i].name,
                  bufs[nb + i] ? "not aligned to 8 bytes" : "null");
  Params p{(const unsigned char*)params, &k.offsets};
  // The dimensions' ranges first, as the CPU target's asserts (Emit/Rust.hs:94-104).
  for (size_t i = 0; i < k.params.size(); ++i) {
    const ParamSpec& s = k.params[i];
    if (!s.dim) continue;
    const uint32_t v = p.u((int)i);
    if (v < s.lo || v > s.hi || (s.mult > 1 && v % s.mult != 0))
      return fail(FKC_ERR_ARGUMENT, "%s: the dimension %s is %u, outside its range %s.", k.name, s.name, v,
                  range_text(s).c_str());
  }
  cudaSetDevice(c->device);
  return k.launch(c, p, bufs);
}

// ---------------------------------------------------------------------------
// Graphs

extern "C" int fkc_capture_begin(fkc_ctx* c) {
  if (!c) return fail(FKC_ERR_ARGUMENT, "fkc_capture_begin: null context.");
  if (c->capturing) return fail(FKC_ERR_STATE, "fkc_capture_begin: a capture is open.");
  cudaSetDevice(c->device);
  FKC_CUDA(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeRelaxed), "fkc_capture_begin");
  c->capturing = true;
  return FKC_OK;
}

extern "C" int fkc_capture_end(fkc_ctx* c, fkc_graph** out) {
  if (!c || !out) return fail(FKC_ERR_ARGUMENT, "fkc_capture_end: null argument.");
  if (!c->capturing) return fail(FKC_ERR_STATE, "fkc_capture_end: no capture is open.");
  cudaSetDevice(c->device);
  c->capturing = false;
  fkc_graph* g = new fkc_graph;
  g->device = c->device;
  cudaError_t e = cudaStreamEndCapture(c->stream, &g->graph);
  if (e == cudaSuccess) e = cudaGraphInstantiate(&g->exec, g->graph, 0);
  if (e == cudaSuccess) e = cudaGraphUpload(g->exec, c->stream);
  if (e != cudaSuccess) {
    fkc_graph_destroy(g);
    return cuda_fail(e, "fkc_capture_end");
  }
  *out = g;
  return FKC_OK;
}

extern "C" int fkc_graph_launch(fkc_ctx* c, fkc_graph* g) {
  if (!c || !g) return fail(FKC_ERR_ARGUMENT, "fkc_graph_launch: null argument.");
  cudaSetDevice(c->device);
  FKC_CUDA(cudaGraphLaunch(g->exec, c->stream), "fkc_graph_launch");
  return FKC_OK;
}

extern "C" int fkc_graph_destroy(fkc_graph* g) {
  if (!g) return FKC_OK;
  cudaSetDevice(g->device);
  if (g->exec) cudaGraphExecDestroy(g->exec);
  if (g->graph) cudaGraphDestroy(g->graph);
  delete g;
  return FKC_OK;
}

extern "C" int fkc_step(fkc_ctx* c, fkc_graph* g, const void* host_in, void* dev_in, size_t in_bytes,
                        void* host_out, const void* dev_out, size_t out_bytes) {
  if (!c || !g) return fail(FKC_ERR_ARGUMENT, "fkc_step: null argument.");
  cudaSetDevice(c->device);
  if (in_bytes) FKC_CUDA(cudaMemcpyAsync(dev_in, host_in, in_bytes, cudaMemcpyHostToDevice, c->stream), "fkc_step: in");
  FKC_CUDA(cudaGraphLaunch(g->exec, c->stream), "fkc_step: replay");
  if (out_bytes)
    FKC_CUDA(cudaMemcpyAsync(host_out, dev_out, out_bytes, cudaMemcpyDeviceToHost, c->stream), "fkc_step: out");
  FKC_CUDA(cudaStreamSynchronize(c->stream), "fkc_step: sync");
  return FKC_OK;
}

extern "C" int fkc_time_graph(fkc_ctx* c, fkc_graph* g, int warmup, int iters, float* ms) {
  if (!c || !g || !ms || iters <= 0) return fail(FKC_ERR_ARGUMENT, "fkc_time_graph: bad argument.");
  cudaSetDevice(c->device);
  for (int i = 0; i < warmup; ++i) FKC_CUDA(cudaGraphLaunch(g->exec, c->stream), "fkc_time_graph");
  cudaEvent_t a, b;
  FKC_CUDA(cudaEventCreate(&a), "fkc_time_graph");
  FKC_CUDA(cudaEventCreate(&b), "fkc_time_graph");
  FKC_CUDA(cudaStreamSynchronize(c->stream), "fkc_time_graph");
  cudaEventRecord(a, c->stream);
  for (int i = 0; i < iters; ++i) FKC_CUDA(cudaGraphLaunch(g->exec, c->stream), "fkc_time_graph");
  cudaEventRecord(b, c->stream);
  cudaError_t e = cudaEventSynchronize(b);
  if (e == cudaSuccess) e = cudaEventElapsedTime(ms, a, b);
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  if (e != cudaSuccess) return cuda_fail(e, "fkc_time_graph");
  return FKC_OK;
}

// ---------------------------------------------------------------------------
// NCCL

static int nccl_fail(ncclResult_t r, const char* what) {
  return fail(FKC_ERR_NCCL, "%s: %s", what, ncclGetErrorString(r));
}

extern "C" int fkc_comm_unique_id(void* id128) {
  if (!id128) return fail(FKC_ERR_ARGUMENT, "fkc_comm_unique_id: null argument.");
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  ncclUniqueId id;
  ncclResult_t r = ncclGetUniqueId(&id);
  if (r != ncclSuccess) return nccl_fail(r, "fkc_comm_unique_id");
  memcpy(id128, &id, sizeof id);
  return FKC_OK;
}

extern "C" int fkc_comm_init(fkc_ctx* c, int nranks, int rank, const void* id128) {
  if (!c || !id128 || nranks < 1 || rank < 0 || rank >= nranks)
    return fail(FKC_ERR_ARGUMENT, "fkc_comm_init: bad argument.");
  if (c->comm) return fail(FKC_ERR_STATE, "fkc_comm_init: the context has a communicator.");
  cudaSetDevice(c->device);
  ncclUniqueId id;
  memcpy(&id, id128, sizeof id);
  ncclResult_t r = ncclCommInitRank(&c->comm, nranks, id, rank);
  if (r != ncclSuccess) {
    c->comm = nullptr;
    return nccl_fail(r, "fkc_comm_init");
  }
  c->nranks = nranks;
  c->rank = rank;
  return FKC_OK;
}

extern "C" int fkc_allreduce_sum_f32(fkc_ctx* c, void* dptr, size_t count) {
  if (!c || (count && !dptr)) return fail(FKC_ERR_ARGUMENT, "fkc_allreduce_sum_f32: null argument.");
  if (!c->comm) return fail(FKC_ERR_STATE, "fkc_allreduce_sum_f32: no communicator.");
  cudaSetDevice(c->device);
  ncclResult_t r = ncclAllReduce(dptr, dptr, count, ncclFloat32, ncclSum, c->comm, c->stream);
  if (r != ncclSuccess) return nccl_fail(r, "fkc_allreduce_sum_f32");
  return FKC_OK;
}

extern "C" int fkc_allgather_u32(fkc_ctx* c, const void* send, void* recv, size_t count) {
  if (!c || (count && (!send || !recv))) return fail(FKC_ERR_ARGUMENT, "fkc_allgather_u32: null argument.");
  if (!c->comm) return fail(FKC_ERR_STATE, "fkc_allgather_u32: no communicator.");
  cudaSetDevice(c->device);
  ncclResult_t r = ncclAllGather(send, recv, count, ncclUint32, c->comm, c->stream);
  if (r != ncclSuccess) return nccl_fail(r, "fkc_allgather_u32");
  return FKC_OK;
}

extern "C" int fkc_comm_rank(fkc_ctx* c, int* rank, int* nranks) {
  if (!c || !rank || !nranks) return fail(FKC_ERR_ARGUMENT, "fkc_comm_rank: null argument.");
  *rank = c->rank;
  *nranks = c->nranks;
  return FKC_OK;
}

// ---------------------------------------------------------------------------
// Peer memory over NVLink: exchange regions mapped between the processes

extern "C" size_t fkc_peer_region_bytes(void) { return FK_XREGION; }

extern "C" int fkc_peer_alloc(fkc_ctx* c, size_t bytes, void** local, void* handle64) {
  if (!c || !local || !handle64) return fail(FKC_ERR_ARGUMENT, "fkc_peer_alloc: null argument.");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "an IPC handle is 64 bytes");
  int rc = fkc_buf_alloc(c, bytes, local);
  if (rc) return rc;
  rc = fkc_buf_zero(c, *local, bytes);
  if (rc) return rc;
  FKC_CUDA(cudaStreamSynchronize(c->stream), "fkc_peer_alloc");
  cudaIpcMemHandle_t h;
  FKC_CUDA(cudaIpcGetMemHandle(&h, *local), "fkc_peer_alloc: cudaIpcGetMemHandle");
  memcpy(handle64, &h, sizeof h);
  return FKC_OK;
}

extern "C" int fkc_peer_open(fkc_ctx* c, const void* handle64, void** peer) {
  if (!c || !handle64 || !peer) return fail(FKC_ERR_ARGUMENT, "fkc_peer_open: null argument.");
  cudaSetDevice(c->device);
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof h);
  void* p = nullptr;
  FKC_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "fkc_peer_open: cudaIpcOpenMemHandle");
  c->opened.insert(p);
  *peer = p;
  return FKC_OK;
}

extern "C" int fkc_peer_set(fkc_ctx* c, int world, int rank, void* const* regions) {
  if (!c || !regions || world < 1 || world > FK_MAX_PEERS || rank < 0 || rank >= world)
    return fail(FKC_ERR_ARGUMENT, "fkc_peer_set: %d ranks (at most %d), rank %d.", world, FK_MAX_PEERS, rank);
  for (int q = 0; q < world; ++q) {
    if (!regions[q]) return fail(FKC_ERR_ARGUMENT, "fkc_peer_set: no region for rank %d.", q);
    c->peers.base[q] = (char*)regions[q];
  }
  c->peers.world = (uint32_t)world;
  c->peers.rank = (uint32_t)rank;
  return FKC_OK;
}

extern "C" int fkc_comm_destroy(fkc_ctx* c) {
  if (!c) return fail(FKC_ERR_ARGUMENT, "fkc_comm_destroy: null context.");
  if (c->comm) {
    ncclResult_t r = ncclCommDestroy(c->comm);
    c->comm = nullptr;
    if (r != ncclSuccess) return nccl_fail(r, "fkc_comm_destroy");
  }
  return FKC_OK;
}
