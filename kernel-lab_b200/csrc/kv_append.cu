// Paged KV append for sm_100a: the write side of the paged cache (16-bit and e4m3 caches).
// Each sequence's new token's K and V rows go into its page pool at token position positions[b]:
//   page = block_table[b, pos / page_size], slot = pos % page_size,
//   k_cache[page, slot, :, :] = k_new[b], v_cache[page, slot, :, :] = v_new[b]
// in kernel-lab's NHD layout (csrc/kernel_lab.h:21-26: [num_pages, page_size, num_kv_heads,
// head_dim], contiguous). kernel-lab has no append kernel (its fixtures build the pool on the
// host, kernel_lab/kv_cache.py:33-80); this is the step of a decode loop that feeds the decode
// kernel its next token.
//
// HBM-bound and tiny (2 * batch * num_kv_heads * head_dim elements): one block per sequence,
// 16-byte copies, the block-table entry read once per block. k_new / v_new rows may be strided
// (a view of a fused QKV projection output) but each row's heads are contiguous. A negative
// position skips the sequence (padding); a position past the block-table width or a page id
// outside [0, num_pages) skips it and sets KL_STATUS_BAD_PAGE in the caller's status word.
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "kernel_lab_b200.h"

namespace klb {
namespace {

constexpr int kAppendThreads = 128;

struct AppendArgs {
  void* k_cache;
  void* v_cache;
  const void* k_new;
  const void* v_new;
  const int32_t* block_table;
  const int32_t* positions;
  int64_t bt_stride;
  int64_t new_stride;  // elements between consecutive sequences' rows of k_new / v_new
  int64_t num_pages;   // < 0: unknown, page ids not range-checked
  int max_pages;
  int page_size;
  int row_elems;       // num_kv_heads * head_dim
  int elem_bytes;
  uint32_t* status;    // may be null
};

// 16-byte path: every row start and the row length are 16-byte aligned.
__global__ void __launch_bounds__(kAppendThreads) kv_append_vec16(const AppendArgs a) {
  wait_prior_grid();
  allow_next_grid();
  const int b = blockIdx.x;
  const int pos = a.positions[b];
  if (pos < 0) return;
  const int pidx = pos / a.page_size;
  int64_t page = -1;
  if (pidx < a.max_pages) page = a.block_table[static_cast<int64_t>(b) * a.bt_stride + pidx];
  if (page < 0 || (a.num_pages >= 0 && page >= a.num_pages)) {
    if (threadIdx.x == 0 && a.status) atomicOr(a.status, kStatusBadPage);
    return;
  }
  const int64_t row_bytes = static_cast<int64_t>(a.row_elems) * a.elem_bytes;
  const int64_t dst_row = page * a.page_size + (pos - pidx * a.page_size);
  const int64_t src = static_cast<int64_t>(b) * a.new_stride * a.elem_bytes;
  const int n16 = static_cast<int>(row_bytes / 16);
  const uint4* ks = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.k_new) + src);
  const uint4* vs = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.v_new) + src);
  uint4* kd = reinterpret_cast<uint4*>(static_cast<uint8_t*>(a.k_cache) + dst_row * row_bytes);
  uint4* vd = reinterpret_cast<uint4*>(static_cast<uint8_t*>(a.v_cache) + dst_row * row_bytes);
  for (int i = threadIdx.x; i < n16; i += blockDim.x) {
    const uint4 k = __ldg(ks + i);
    const uint4 v = __ldg(vs + i);
    kd[i] = k;
    vd[i] = v;
  }
}

// Element path for anything else (odd head_dim, misaligned views).
template <typename E>
__global__ void __launch_bounds__(kAppendThreads) kv_append_scalar(const AppendArgs a) {
  wait_prior_grid();
  allow_next_grid();
  const int b = blockIdx.x;
  const int pos = a.positions[b];
  if (pos < 0) return;
  const int pidx = pos / a.page_size;
  int64_t page = -1;
  if (pidx < a.max_pages) page = a.block_table[static_cast<int64_t>(b) * a.bt_stride + pidx];
  if (page < 0 || (a.num_pages >= 0 && page >= a.num_pages)) {
    if (threadIdx.x == 0 && a.status) atomicOr(a.status, kStatusBadPage);
    return;
  }
  const int64_t dst_row = page * a.page_size + (pos - pidx * a.page_size);
  const E* ks = static_cast<const E*>(a.k_new) + static_cast<int64_t>(b) * a.new_stride;
  const E* vs = static_cast<const E*>(a.v_new) + static_cast<int64_t>(b) * a.new_stride;
  E* kd = static_cast<E*>(a.k_cache) + dst_row * a.row_elems;
  E* vd = static_cast<E*>(a.v_cache) + dst_row * a.row_elems;
  for (int i = threadIdx.x; i < a.row_elems; i += blockDim.x) {
    kd[i] = ks[i];
    vd[i] = vs[i];
  }
}

// e4m3 cache: each new row is quantised per KV head, e4m3(x / scale) with an IEEE float
// division, rounding to nearest-even and saturating to +-448 (NaN stays NaN).
template <typename E>
__global__ void __launch_bounds__(kAppendThreads) kv_append_e4m3(const AppendArgs a, const float* k_scale,
                                                                  const float* v_scale, int head_dim) {
  wait_prior_grid();
  allow_next_grid();
  const int b = blockIdx.x;
  const int pos = a.positions[b];
  if (pos < 0) return;
  const int pidx = pos / a.page_size;
  int64_t page = -1;
  if (pidx < a.max_pages) page = a.block_table[static_cast<int64_t>(b) * a.bt_stride + pidx];
  if (page < 0 || (a.num_pages >= 0 && page >= a.num_pages)) {
    if (threadIdx.x == 0 && a.status) atomicOr(a.status, kStatusBadPage);
    return;
  }
  const int64_t dst_row = page * a.page_size + (pos - pidx * a.page_size);
  const E* ks = static_cast<const E*>(a.k_new) + static_cast<int64_t>(b) * a.new_stride;
  const E* vs = static_cast<const E*>(a.v_new) + static_cast<int64_t>(b) * a.new_stride;
  uint8_t* kd = static_cast<uint8_t*>(a.k_cache) + dst_row * a.row_elems;
  uint8_t* vd = static_cast<uint8_t*>(a.v_cache) + dst_row * a.row_elems;
  for (int i = 2 * threadIdx.x; i < a.row_elems; i += 2 * blockDim.x) {  // head_dim is even
    const int h = i / head_dim;
    const float kq = k_scale[h], vq = v_scale[h];
    const float2 kx = make_float2(Storage<E>::load(ks[i]) / kq, Storage<E>::load(ks[i + 1]) / kq);
    const float2 vx = make_float2(Storage<E>::load(vs[i]) / vq, Storage<E>::load(vs[i + 1]) / vq);
    *reinterpret_cast<__nv_fp8x2_storage_t*>(kd + i) = __nv_cvt_float2_to_fp8x2(kx, __NV_SATFINITE, __NV_E4M3);
    *reinterpret_cast<__nv_fp8x2_storage_t*>(vd + i) = __nv_cvt_float2_to_fp8x2(vx, __NV_SATFINITE, __NV_E4M3);
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Launched with programmatic stream serialization (KL_APPEND_PDL=0: without, read once). Each
// block waits for the previous kernel before its first global access and at once lets the next
// kernel (normally the decode that reads these rows, which waits for this grid's completion
// before its own first global access) start launching into the SMs beside it.
bool append_pdl() {
  static const bool on = env_switch_on("KL_APPEND_PDL");
  return on;
}

template <typename... Params, typename... Args>
cudaError_t launch_rows(void (*kernel)(Params...), int batch, cudaStream_t st, const Args&... args) {
  return launch_kernel(append_pdl(), kernel, dim3(static_cast<unsigned>(batch)), dim3(kAppendThreads), 0, st, args...);
}

}  // namespace
}  // namespace klb

extern "C" int kl_paged_kv_append(int dtype, void* k_cache, void* v_cache, const void* k_new, const void* v_new,
                                  const int32_t* block_table, const int32_t* positions, int batch,
                                  int num_kv_heads, int head_dim, int page_size, int64_t block_table_stride,
                                  int max_pages_per_seq, int64_t num_pages, int64_t new_row_stride,
                                  uint32_t* status, void* stream) {
  using namespace klb;
  if (batch == 0) return 0;
  if (batch < 0 || num_kv_heads <= 0 || head_dim <= 0 || page_size <= 0 || max_pages_per_seq < 0 ||
      block_table_stride < max_pages_per_seq || !k_cache || !v_cache || !k_new || !v_new || !block_table ||
      !positions) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  if (dtype != KL_FLOAT32 && dtype != KL_FLOAT16 && dtype != KL_BFLOAT16) return static_cast<int>(cudaErrorInvalidValue);
  const int64_t row_elems = static_cast<int64_t>(num_kv_heads) * head_dim;
  if (row_elems > (1 << 24) || new_row_stride < row_elems) return static_cast<int>(cudaErrorInvalidValue);
  AppendArgs a{};
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.k_new = k_new;
  a.v_new = v_new;
  a.block_table = block_table;
  a.positions = positions;
  a.bt_stride = block_table_stride;
  a.new_stride = new_row_stride;
  a.num_pages = num_pages;
  a.max_pages = max_pages_per_seq;
  a.page_size = page_size;
  a.row_elems = static_cast<int>(row_elems);
  a.elem_bytes = dtype == KL_FLOAT32 ? 4 : 2;
  a.status = status;
  const auto st = static_cast<cudaStream_t>(stream);
  const int64_t row_bytes = row_elems * a.elem_bytes;
  const bool vec = row_bytes % 16 == 0 && (new_row_stride * a.elem_bytes) % 16 == 0 && aligned16(k_cache) &&
                   aligned16(v_cache) && aligned16(k_new) && aligned16(v_new);
  cudaError_t e;
  if (vec) {
    e = launch_rows(kv_append_vec16, batch, st, a);
  } else if (a.elem_bytes == 4) {
    e = launch_rows(kv_append_scalar<float>, batch, st, a);
  } else {
    e = launch_rows(kv_append_scalar<uint16_t>, batch, st, a);
  }
  return static_cast<int>(e);
}

extern "C" int kl_paged_kv_append_fp8(int dtype, void* k_cache, void* v_cache, const void* k_new, const void* v_new,
                                      const float* k_scale, const float* v_scale, const int32_t* block_table,
                                      const int32_t* positions, int batch, int num_kv_heads, int head_dim,
                                      int page_size, int64_t block_table_stride, int max_pages_per_seq,
                                      int64_t num_pages, int64_t new_row_stride, uint32_t* status, void* stream) {
  using namespace klb;
  if (batch == 0) return 0;
  if (batch < 0 || num_kv_heads <= 0 || head_dim <= 0 || head_dim % 2 != 0 || page_size <= 0 ||
      max_pages_per_seq < 0 || block_table_stride < max_pages_per_seq || !k_cache || !v_cache || !k_new || !v_new ||
      !k_scale || !v_scale || !block_table || !positions) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  if (dtype != KL_FLOAT32 && dtype != KL_FLOAT16 && dtype != KL_BFLOAT16) return static_cast<int>(cudaErrorInvalidValue);
  const int64_t row_elems = static_cast<int64_t>(num_kv_heads) * head_dim;
  if (row_elems > (1 << 24) || new_row_stride < row_elems) return static_cast<int>(cudaErrorInvalidValue);
  AppendArgs a{};
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.k_new = k_new;
  a.v_new = v_new;
  a.block_table = block_table;
  a.positions = positions;
  a.bt_stride = block_table_stride;
  a.new_stride = new_row_stride;
  a.num_pages = num_pages;
  a.max_pages = max_pages_per_seq;
  a.page_size = page_size;
  a.row_elems = static_cast<int>(row_elems);
  a.elem_bytes = 1;
  a.status = status;
  const auto st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  switch (dtype) {
    case KL_FLOAT32: e = launch_rows(kv_append_e4m3<float>, batch, st, a, k_scale, v_scale, head_dim); break;
    case KL_FLOAT16: e = launch_rows(kv_append_e4m3<__half>, batch, st, a, k_scale, v_scale, head_dim); break;
    default: e = launch_rows(kv_append_e4m3<__nv_bfloat16>, batch, st, a, k_scale, v_scale, head_dim); break;
  }
  return static_cast<int>(e);
}
