// Error plumbing, identity and small diagnostic entry points of the C ABI.
#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"

namespace glm53 {

static thread_local char g_last_error[512] = "";

constexpr unsigned long long kDefaultWaitNs = 2000000000ull;
static std::atomic<unsigned long long> g_wait_limit_ns{kDefaultWaitNs};

unsigned long long ep_wait_limit_ns() { return g_wait_limit_ns.load(std::memory_order_relaxed); }

void set_last_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int check_launch(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    set_last_error("%s: %s", what, cudaGetErrorString(err));
    return GLM53_ERR_CUDA;
  }
  return GLM53_OK;
}

int sm_count() {
  static thread_local int cached_dev = -1;
  static thread_local int cached = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kNumSMs;
  if (dev != cached_dev) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = kNumSMs;
    cached = n;
    cached_dev = dev;
  }
  return cached;
}

int ensure_max_smem(const void* func, size_t bytes) {
  // cudaFuncSetAttribute once per (kernel, device, size): repeated calls are
  // avoided so launches can be recorded into CUDA graphs.
  struct Entry { const void* f; int dev; size_t bytes; };
  static Entry table[256];
  static int used = 0;
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (table[i].f == func && table[i].dev == dev && table[i].bytes >= bytes) return GLM53_OK;
  cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess) {
    set_last_error("cudaFuncSetAttribute(%zu bytes): %s", bytes, cudaGetErrorString(e));
    return GLM53_ERR_CUDA;
  }
  if (used < 256) table[used++] = Entry{func, dev, bytes};
  return GLM53_OK;
}

__global__ void sigmoid_bf16_kernel(const uint16_t* __restrict__ g, int64_t n,
                                    uint16_t* __restrict__ out) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = f32_to_bf16_bits(sigmoid_bf16(g[i]));
}

}  // namespace glm53

using namespace glm53;

extern "C" const char* glm53_kernel_abi(void) {
  return "glm53-b200-sm100a-v1"
         "-e4m3lut480-block128"
         "-gemv-splitrow-f32"
         "-packed-decode-exact-bf16-swiglu"
         "-grouped-bf16mma-scalefold";
}

extern "C" const char* glm53_last_error(void) { return g_last_error; }

namespace glm53 {

// 16-byte copy between device memory and pinned (device-mapped) host memory.
// A programmatic dependent (the router of a host decode step) may launch at
// once; it waits for this grid before it reads the copy.
// With `status` and `mirror` set, thread 0 of block 0 also copies the device
// status word into the mapped host word `mirror` (the work before this grid
// on the stream has finished, so the word holds every earlier call's bits).
// Launched as a programmatic dependent (pdl), the copy may run while the
// previous kernel still does; the status word is read only after
// griddepcontrol.wait, when that kernel has finished (a no-op otherwise).
__global__ void __launch_bounds__(256) copy16_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                                     size_t n16, const uint32_t* __restrict__ status,
                                                     volatile uint32_t* mirror) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (size_t)gridDim.x * blockDim.x)
    dst[i] = src[i];
  if (mirror && blockIdx.x == 0 && threadIdx.x == 0) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    *mirror = *(const volatile uint32_t*)status;
  }
}

__global__ void status_mirror_kernel(const uint32_t* __restrict__ status, volatile uint32_t* mirror) {
  *mirror = *(const volatile uint32_t*)status;
}

void* mapped_host(const void* p) {
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return at.type == cudaMemoryTypeHost ? at.devicePointer : nullptr;  // null when not device-mapped
}

// Small host <-> device copy: a kernel over the pinned buffer's device
// mapping (a copy-engine transfer of a few KB costs 7-10 us of stream time
// on B200, the kernel about 2), else cudaMemcpyAsync.
cudaError_t small_copy(void* dst, const void* src, size_t bytes, bool to_device, cudaStream_t st, bool* by_kernel,
                       const uint32_t* status, uint32_t* status_mirror, bool pdl) {
  const void* host = to_device ? src : dst;
  void* mapped = (bytes % 16 == 0 && ((uintptr_t)src | (uintptr_t)dst) % 16 == 0) ? mapped_host(host) : nullptr;
  if (by_kernel) *by_kernel = mapped != nullptr;
  if (!mapped)
    return cudaMemcpyAsync(dst, src, bytes, to_device ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToHost, st);
  const size_t n16 = bytes / 16;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)std::min<size_t>((n16 + 255) / 256, 64));
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaLaunchKernelEx(&cfg, copy16_kernel, (const uint4*)(to_device ? mapped : src), (uint4*)(to_device ? dst : mapped),
                     n16, status, status ? status_mirror : (uint32_t*)nullptr);
  return cudaGetLastError();
}

int mirror_status(const uint32_t* status, uint32_t* host_word, cudaStream_t st, const char* fn) {
  void* mapped = (status && host_word && ((uintptr_t)host_word & 3) == 0) ? mapped_host(host_word) : nullptr;
  if (!mapped) {
    set_last_error("%s: the status mirror must be a 4-byte aligned word of pinned (device-mapped) host memory", fn);
    return GLM53_ERR_INVALID;
  }
  status_mirror_kernel<<<1, 1, 0, st>>>(status, (volatile uint32_t*)mapped);
  return check_launch(fn);
}

}  // namespace glm53

extern "C" int glm53_graph_step(void* graph_exec, const void* x_host, void* x_dev, size_t x_bytes, const void* out_dev,
                                void* out_host, size_t out_bytes, void* stream) {
  if (!graph_exec || (x_bytes && (!x_host || !x_dev)) || (out_host && (!out_dev || !out_bytes))) {
    set_last_error("glm53_graph_step: invalid arguments");
    return GLM53_ERR_INVALID;
  }
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = x_bytes ? small_copy(x_dev, x_host, x_bytes, true, st, nullptr) : cudaSuccess;
  if (e == cudaSuccess) e = cudaGraphLaunch((cudaGraphExec_t)graph_exec, st);
  if (e == cudaSuccess && out_host) e = small_copy(out_host, out_dev, out_bytes, false, st, nullptr);
  if (e != cudaSuccess) {
    set_last_error("glm53_graph_step: %s", cudaGetErrorString(e));
    return GLM53_ERR_CUDA;
  }
  return GLM53_OK;
}

extern "C" int glm53_set_wait_limit_ns(unsigned long long ns) {
  if (ns != 0 && (ns < 1000000ull || ns > 60000000000ull)) {
    set_last_error("glm53_set_wait_limit_ns: %llu ns is outside [1 ms, 60 s] (0 restores the default)", ns);
    return GLM53_ERR_INVALID;
  }
  g_wait_limit_ns.store(ns ? ns : kDefaultWaitNs, std::memory_order_relaxed);
  return GLM53_OK;
}

extern "C" int glm53_status_mirror(const uint32_t* status, uint32_t* host_word, void* stream) {
  return mirror_status(status, host_word, (cudaStream_t)stream, "glm53_status_mirror");
}

extern "C" int glm53_sigmoid_bf16(const void* gate, int64_t n, void* out, void* stream) {
  if (n < 0 || (n > 0 && (!gate || !out))) {
    set_last_error("glm53_sigmoid_bf16: invalid arguments");
    return GLM53_ERR_INVALID;
  }
  if (n == 0) return GLM53_OK;
  int64_t blocks = (n + 255) / 256;
  sigmoid_bf16_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
      (const uint16_t*)gate, n, (uint16_t*)out);
  return check_launch("glm53_sigmoid_bf16");
}
