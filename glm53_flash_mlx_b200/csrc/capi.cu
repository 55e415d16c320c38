// Error plumbing, identity and small diagnostic entry points of the C ABI.
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "common.cuh"

namespace glm53 {

static thread_local char g_last_error[512] = "";

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
