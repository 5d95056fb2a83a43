// Test infrastructure only (a checker and comparator, never the product): a C ABI over
// kernel-lab's own C++ launchers, so tests can call kernel-lab's CUDA kernels built from its
// unmodified sources (csrc/paged_attention.cu, csrc/rmsnorm.cu) with ctypes.
//
// kernel_lab.h (kernel-lab csrc/kernel_lab.h:12-33: DType order, launcher argument lists) is
// found through the build recipe's -I of kernel-lab's csrc directory; nothing of it is copied.
#include <cstdint>

#include <cuda_runtime.h>

#include "kernel_lab.h"

extern "C" {

// kernel_lab::launch_paged_decode_attention (kernel_lab.h:27-33); dtype 0/1/2 = f32/f16/bf16.
int klref_paged_decode_attention(int dtype, void* out, const void* q, const void* k_cache, const void* v_cache,
                                 const int32_t* block_table, const int32_t* seq_lens, int batch, int num_q_heads,
                                 int num_kv_heads, int head_dim, int page_size, int64_t block_table_stride,
                                 float scale, void* stream) {
  return static_cast<int>(kernel_lab::launch_paged_decode_attention(
      static_cast<kernel_lab::DType>(dtype), out, q, k_cache, v_cache, block_table, seq_lens, batch, num_q_heads,
      num_kv_heads, head_dim, page_size, block_table_stride, scale, static_cast<cudaStream_t>(stream)));
}

// kernel_lab::launch_rms_norm (kernel_lab.h:17-19); residual may be null (plain RMSNorm).
int klref_rms_norm(int dtype, void* out, const void* x, void* residual, const void* weight, int rows, int hidden,
                   int64_t x_row_stride, float eps, void* stream) {
  return static_cast<int>(kernel_lab::launch_rms_norm(static_cast<kernel_lab::DType>(dtype), out, x, residual,
                                                      weight, rows, hidden, x_row_stride, eps,
                                                      static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
