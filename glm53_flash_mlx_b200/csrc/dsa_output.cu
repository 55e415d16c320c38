// Layout step of the sparse-attention output projection: the head-major
// attention result [heads, rows, dim] becomes the row-major o_proj input
// [rows, heads * dim] (glm53_native_prefill_dsa_head_to_row_bfloat16,
// native_execution/native_indexer_plan.metal:2290-2304, run by
// NativePrefillDSAOutputPlan::execute, native_prefill_dsa_output_plan.cpp:68-106).
// Every (head, row) run of dim values is contiguous on both sides, so each
// thread moves one 16-byte piece of a run: reads and writes are coalesced.
#include "common.cuh"

namespace glm53 {
namespace {

__global__ void __launch_bounds__(256) head_to_rows_kernel(const uint4* __restrict__ head_major, int64_t heads,
                                                            int64_t rows, int64_t pieces_per_run,
                                                            uint4* __restrict__ row_major) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= heads * rows * pieces_per_run) return;
  const int64_t piece = i % pieces_per_run;
  const int64_t run = i / pieces_per_run;  // head * rows + row
  const int64_t row = run % rows, head = run / rows;
  row_major[(row * heads + head) * pieces_per_run + piece] = ldg_stream(head_major + i);
}

}  // namespace
}  // namespace glm53

using namespace glm53;

extern "C" int glm53_head_major_to_rows(const void* head_major, int64_t heads, int64_t rows, int64_t dim,
                                        void* row_major, void* stream) {
  if (heads < 0 || rows < 0 || dim <= 0 || dim % 8 != 0) {
    set_last_error("glm53_head_major_to_rows: dim %lld must be a positive multiple of 8", (long long)dim);
    return GLM53_ERR_INVALID;
  }
  const int64_t n = heads * rows * (dim / 8);
  if (n == 0) return GLM53_OK;
  if (!head_major || !row_major || (((uintptr_t)head_major | (uintptr_t)row_major) & 15)) {
    set_last_error("glm53_head_major_to_rows: tensors must be non-NULL and 16-byte aligned");
    return GLM53_ERR_INVALID;
  }
  head_to_rows_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      (const uint4*)head_major, heads, rows, dim / 8, (uint4*)row_major);
  return check_launch("head_to_rows_kernel");
}
