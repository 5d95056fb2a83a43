// PyTorch operators torch.ops.kernel_lab.* over the C ABI in kernel_lab_b200.h.
//
// Registers the same TORCH_LIBRARY(kernel_lab) schemas as kernel-lab
// (csrc/torch_bindings.cpp:107-119 there), so `import kernel_lab._C` is a drop-in:
//   rms_norm(Tensor! out, Tensor x, Tensor weight, float eps) -> ()
//   fused_add_rms_norm(Tensor! out, Tensor x, Tensor! residual, Tensor weight, float eps) -> ()
//   paged_decode_attention(Tensor! out, Tensor q, Tensor k_cache, Tensor v_cache,
//                          Tensor block_table, Tensor seq_lens, float scale) -> ()
// plus one extension op that forces the number of KV splits:
//   paged_decode_attention_splits(..., float scale, int num_splits) -> ()
// Validation mirrors kernel-lab's (TORCH_CHECK -> RuntimeError); a non-zero status from
// the C ABI becomes "kernel_lab: <op> failed: <reason>". Meta kernels (no-ops: the ops
// only mutate their outputs) let torch.compile(fullgraph=True) trace the ops.
//
// Decode scratch (split partials and arrival counters) is owned here, one pair of
// buffers per (device, stream), allocated through PyTorch's caching allocator and grown
// on demand. The counters are zeroed once at allocation; every call leaves them zero.
// Entries live as long as the process (a stream that is destroyed keeps its entry, so a
// host that creates streams per request should reuse a pool of them).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <map>
#include <mutex>
#include <utility>

#include "kernel_lab_b200.h"

namespace {

int to_dtype(at::ScalarType t) {
  switch (t) {
    case at::kFloat:
      return KL_FLOAT32;
    case at::kHalf:
      return KL_FLOAT16;
    case at::kBFloat16:
      return KL_BFLOAT16;
    default:
      TORCH_CHECK(false, "kernel_lab: unsupported dtype ", t);
  }
}

void check_status(int rc, const char* what) {
  TORCH_CHECK(rc == 0, "kernel_lab: ", what, " failed: ", kl_status_string(rc));
}

void rms_norm_impl(at::Tensor& out, const at::Tensor& x, at::Tensor* residual, const at::Tensor& weight,
                   double eps, const char* what) {
  TORCH_CHECK(x.is_cuda() && weight.is_cuda() && out.is_cuda(), "tensors must be on CUDA");
  TORCH_CHECK(x.dim() >= 1 && x.stride(-1) == 1, "x must have a contiguous last dimension");
  TORCH_CHECK(out.is_contiguous() && weight.is_contiguous(), "out and weight must be contiguous");
  const int64_t hidden = x.size(-1);
  TORCH_CHECK(weight.numel() == hidden, "weight size ", weight.numel(), " != hidden ", hidden);
  TORCH_CHECK(out.sizes() == x.sizes(), "out must match x");
  TORCH_CHECK(x.scalar_type() == weight.scalar_type() && x.scalar_type() == out.scalar_type(),
              "x, weight and out must share a dtype");
  TORCH_CHECK(weight.device() == x.device() && out.device() == x.device(), "tensors must be on one device");
  const at::Tensor x2 = x.dim() == 2 ? x : x.reshape({-1, hidden});
  TORCH_CHECK(x2.stride(-1) == 1, "x cannot be viewed as rows with a contiguous last dim");
  void* res_ptr = nullptr;
  if (residual != nullptr) {
    TORCH_CHECK(residual->is_contiguous() && residual->sizes() == x.sizes() &&
                    residual->scalar_type() == x.scalar_type() && residual->device() == x.device(),
                "residual must be contiguous, same shape and dtype as x");
    res_ptr = residual->data_ptr();
  }
  const c10::cuda::CUDAGuard guard(x.device());
  check_status(kl_rms_norm(to_dtype(x.scalar_type()), out.data_ptr(), x2.data_ptr(), res_ptr, weight.data_ptr(),
                           static_cast<int>(x2.size(0)), static_cast<int>(hidden), x2.stride(0),
                           static_cast<float>(eps), at::cuda::getCurrentCUDAStream().stream()),
               what);
}

void rms_norm(at::Tensor& out, const at::Tensor& x, const at::Tensor& weight, double eps) {
  rms_norm_impl(out, x, nullptr, weight, eps, "rms_norm");
}

void fused_add_rms_norm(at::Tensor& out, const at::Tensor& x, at::Tensor& residual, const at::Tensor& weight,
                        double eps) {
  rms_norm_impl(out, x, &residual, weight, eps, "fused_add_rms_norm");
}

struct Scratch {
  at::Tensor partials;  // uint8, no initialisation needed
  at::Tensor sync;      // uint8, zero at rest
};

std::mutex g_scratch_mu;
std::map<std::pair<int, cudaStream_t>, Scratch> g_scratch;

Scratch& scratch_for(const at::Device& dev, cudaStream_t stream, size_t partial_bytes, size_t sync_bytes) {
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  Scratch& s = g_scratch[{dev.index(), stream}];
  const auto opts = at::TensorOptions().dtype(at::kByte).device(dev);
  if (!s.partials.defined() || static_cast<size_t>(s.partials.numel()) < partial_bytes) {
    s.partials = at::empty({static_cast<int64_t>(std::max<size_t>(partial_bytes, 256) * 5 / 4)}, opts);
  }
  if (!s.sync.defined() || static_cast<size_t>(s.sync.numel()) < sync_bytes) {
    at::Tensor grown = at::zeros({static_cast<int64_t>(std::max<size_t>(sync_bytes, 256) * 5 / 4)}, opts);
    // Status word 0 is sticky until decode_status(clear=True): carry it into the larger buffer
    // (stream-ordered after every earlier call on this stream; the counters are zero at rest).
    if (s.sync.defined()) grown.narrow(0, 0, 4).copy_(s.sync.narrow(0, 0, 4), /*non_blocking=*/true);
    s.sync = grown;
  }
  return s;
}

void paged_decode_impl(at::Tensor& out, const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                       const at::Tensor& block_table, const at::Tensor& seq_lens, double scale, int64_t num_splits) {
  TORCH_CHECK(q.is_cuda() && k_cache.is_cuda() && v_cache.is_cuda(), "tensors must be on CUDA");
  TORCH_CHECK(q.dim() == 3 && k_cache.dim() == 4, "q is [batch, heads, dim]; caches are 4-D");
  TORCH_CHECK(q.is_contiguous() && out.is_contiguous() && k_cache.is_contiguous() && v_cache.is_contiguous(),
              "q, out and both caches must be contiguous");
  TORCH_CHECK(k_cache.sizes() == v_cache.sizes(), "k_cache and v_cache shapes differ");
  TORCH_CHECK(block_table.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt,
              "block_table and seq_lens must be int32");
  TORCH_CHECK(block_table.dim() == 2 && block_table.stride(-1) == 1 && seq_lens.is_contiguous(),
              "block_table rows and seq_lens must be contiguous");
  TORCH_CHECK(q.scalar_type() == k_cache.scalar_type() && q.scalar_type() == v_cache.scalar_type() &&
                  q.scalar_type() == out.scalar_type(),
              "q, caches and out must share a dtype");
  TORCH_CHECK(out.sizes() == q.sizes(), "out must match q");
  TORCH_CHECK(k_cache.device() == q.device() && v_cache.device() == q.device() && out.device() == q.device() &&
                  block_table.device() == q.device() && seq_lens.device() == q.device(),
              "tensors must be on one device");
  TORCH_CHECK(num_splits >= 0 && num_splits <= (1 << 20), "num_splits must be >= 0");

  const int batch = static_cast<int>(q.size(0));
  const int num_q_heads = static_cast<int>(q.size(1));
  const int head_dim = static_cast<int>(q.size(2));
  const int page_size = static_cast<int>(k_cache.size(1));
  const int num_kv_heads = static_cast<int>(k_cache.size(2));
  TORCH_CHECK(k_cache.size(3) == head_dim, "cache head_dim differs from q");
  TORCH_CHECK(num_kv_heads > 0 && num_q_heads % num_kv_heads == 0,
              "num_q_heads must be a multiple of num_kv_heads");
  TORCH_CHECK(seq_lens.numel() == batch && block_table.size(0) == batch,
              "block_table and seq_lens need one row / entry per sequence");
  if (batch == 0) return;

  const int dtype = to_dtype(q.scalar_type());
  const int max_pages = static_cast<int>(block_table.size(1));
  const c10::cuda::CUDAGuard guard(q.device());
  const cudaStream_t stream = at::cuda::getCurrentCUDAStream().stream();
  size_t partial_bytes = 0, sync_bytes = 0;
  check_status(kl_paged_decode_workspace_size(dtype, batch, num_q_heads, num_kv_heads, head_dim, page_size,
                                              max_pages, static_cast<int>(num_splits), &partial_bytes,
                                              &sync_bytes),
               "paged_decode_attention (workspace)");
  Scratch& s = scratch_for(q.device(), stream, partial_bytes, sync_bytes);
  check_status(kl_paged_decode(dtype, out.data_ptr(), q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                               block_table.data_ptr<int32_t>(), seq_lens.data_ptr<int32_t>(), batch, num_q_heads,
                               num_kv_heads, head_dim, page_size, block_table.stride(0), max_pages,
                               k_cache.size(0), static_cast<float>(scale), static_cast<int>(num_splits),
                               s.partials.data_ptr(), static_cast<size_t>(s.partials.numel()), s.sync.data_ptr(),
                               static_cast<size_t>(s.sync.numel()), stream),
               "paged_decode_attention");
}

void paged_decode_attention(at::Tensor& out, const at::Tensor& q, const at::Tensor& k_cache,
                            const at::Tensor& v_cache, const at::Tensor& block_table, const at::Tensor& seq_lens,
                            double scale) {
  paged_decode_impl(out, q, k_cache, v_cache, block_table, seq_lens, scale, 0);
}

void paged_decode_attention_splits(at::Tensor& out, const at::Tensor& q, const at::Tensor& k_cache,
                                   const at::Tensor& v_cache, const at::Tensor& block_table,
                                   const at::Tensor& seq_lens, double scale, int64_t num_splits) {
  paged_decode_impl(out, q, k_cache, v_cache, block_table, seq_lens, scale, num_splits);
}

// Write each sequence's new token's K/V rows into its pages (kl_paged_kv_append); bad page
// ids are skipped and flagged in the same status word as the decode calls of this stream.
void paged_kv_append(at::Tensor& k_cache, at::Tensor& v_cache, const at::Tensor& k_new, const at::Tensor& v_new,
                     const at::Tensor& block_table, const at::Tensor& positions) {
  TORCH_CHECK(k_cache.is_cuda() && v_cache.is_cuda() && k_new.is_cuda() && v_new.is_cuda(),
              "tensors must be on CUDA");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.is_contiguous() && v_cache.is_contiguous() &&
                  k_cache.sizes() == v_cache.sizes(),
              "caches are contiguous [num_pages, page_size, num_kv_heads, head_dim] of one shape");
  const int64_t num_kv_heads = k_cache.size(2), head_dim = k_cache.size(3);
  TORCH_CHECK(k_new.sizes() == v_new.sizes() && k_new.strides() == v_new.strides(),
              "k_new and v_new must have one shape and layout");
  TORCH_CHECK((k_new.dim() == 3 && k_new.size(1) == num_kv_heads && k_new.size(2) == head_dim &&
               k_new.stride(2) == 1 && k_new.stride(1) == head_dim) ||
                  (k_new.dim() == 2 && k_new.size(1) == num_kv_heads * head_dim && k_new.stride(1) == 1),
              "k_new is [batch, num_kv_heads, head_dim] (or [batch, num_kv_heads*head_dim]) with contiguous rows");
  TORCH_CHECK(k_new.scalar_type() == k_cache.scalar_type() && v_new.scalar_type() == k_cache.scalar_type() &&
                  v_cache.scalar_type() == k_cache.scalar_type(),
              "new rows and caches must share a dtype");
  TORCH_CHECK(block_table.scalar_type() == at::kInt && positions.scalar_type() == at::kInt,
              "block_table and positions must be int32");
  TORCH_CHECK(block_table.dim() == 2 && block_table.stride(-1) == 1 && positions.is_contiguous(),
              "block_table rows and positions must be contiguous");
  const int64_t batch = k_new.size(0);
  TORCH_CHECK(positions.numel() == batch && block_table.size(0) == batch,
              "block_table and positions need one row / entry per sequence");
  TORCH_CHECK(k_cache.device() == k_new.device() && v_cache.device() == k_new.device() &&
                  v_new.device() == k_new.device() && block_table.device() == k_new.device() &&
                  positions.device() == k_new.device(),
              "tensors must be on one device");
  if (batch == 0) return;
  const c10::cuda::CUDAGuard guard(k_new.device());
  const cudaStream_t stream = at::cuda::getCurrentCUDAStream().stream();
  Scratch& s = scratch_for(k_new.device(), stream, 0, 4);
  check_status(kl_paged_kv_append(to_dtype(k_cache.scalar_type()), k_cache.data_ptr(), v_cache.data_ptr(),
                                  k_new.data_ptr(), v_new.data_ptr(), block_table.data_ptr<int32_t>(),
                                  positions.data_ptr<int32_t>(), static_cast<int>(batch),
                                  static_cast<int>(num_kv_heads), static_cast<int>(head_dim),
                                  static_cast<int>(k_cache.size(1)), block_table.stride(0),
                                  static_cast<int>(block_table.size(1)), k_cache.size(0), k_new.stride(0),
                                  static_cast<uint32_t*>(s.sync.data_ptr()), stream),
               "paged_kv_append");
}

bool is_e4m3(const at::Tensor& t) { return t.scalar_type() == at::kFloat8_e4m3fn || t.scalar_type() == at::kByte; }

void check_scales(const at::Tensor& k_scale, const at::Tensor& v_scale, int64_t num_kv_heads, const at::Device& dev) {
  TORCH_CHECK(k_scale.scalar_type() == at::kFloat && v_scale.scalar_type() == at::kFloat &&
                  k_scale.is_contiguous() && v_scale.is_contiguous() && k_scale.numel() == num_kv_heads &&
                  v_scale.numel() == num_kv_heads && k_scale.device() == dev && v_scale.device() == dev,
              "k_scale and v_scale are contiguous float32 [num_kv_heads] on the caches' device");
}

// Decode over an e4m3 cache with per-KV-head scales (kl_paged_decode_fp8).
void paged_decode_attention_fp8(at::Tensor& out, const at::Tensor& q, const at::Tensor& k_cache,
                                const at::Tensor& v_cache, const at::Tensor& k_scale, const at::Tensor& v_scale,
                                const at::Tensor& block_table, const at::Tensor& seq_lens, double scale) {
  TORCH_CHECK(q.is_cuda() && k_cache.is_cuda() && v_cache.is_cuda(), "tensors must be on CUDA");
  TORCH_CHECK(q.dim() == 3 && k_cache.dim() == 4, "q is [batch, heads, dim]; caches are 4-D");
  TORCH_CHECK(q.is_contiguous() && out.is_contiguous() && k_cache.is_contiguous() && v_cache.is_contiguous(),
              "q, out and both caches must be contiguous");
  TORCH_CHECK(k_cache.sizes() == v_cache.sizes(), "k_cache and v_cache shapes differ");
  TORCH_CHECK(is_e4m3(k_cache) && is_e4m3(v_cache), "caches must be float8_e4m3fn (or uint8 e4m3 codes)");
  TORCH_CHECK((q.scalar_type() == at::kHalf || q.scalar_type() == at::kBFloat16) &&
                  out.scalar_type() == q.scalar_type() && out.sizes() == q.sizes(),
              "q and out are fp16 or bf16 of one shape");
  TORCH_CHECK(block_table.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt &&
                  block_table.dim() == 2 && block_table.stride(-1) == 1 && seq_lens.is_contiguous(),
              "block_table rows and seq_lens must be contiguous int32");
  TORCH_CHECK(k_cache.device() == q.device() && v_cache.device() == q.device() && out.device() == q.device() &&
                  block_table.device() == q.device() && seq_lens.device() == q.device(),
              "tensors must be on one device");
  const int batch = static_cast<int>(q.size(0));
  const int num_q_heads = static_cast<int>(q.size(1));
  const int head_dim = static_cast<int>(q.size(2));
  const int page_size = static_cast<int>(k_cache.size(1));
  const int num_kv_heads = static_cast<int>(k_cache.size(2));
  TORCH_CHECK(k_cache.size(3) == head_dim, "cache head_dim differs from q");
  TORCH_CHECK(num_kv_heads > 0 && num_q_heads % num_kv_heads == 0, "num_q_heads must be a multiple of num_kv_heads");
  TORCH_CHECK(seq_lens.numel() == batch && block_table.size(0) == batch,
              "block_table and seq_lens need one row / entry per sequence");
  check_scales(k_scale, v_scale, num_kv_heads, q.device());
  if (batch == 0) return;
  const int dtype = to_dtype(q.scalar_type());
  const int max_pages = static_cast<int>(block_table.size(1));
  const c10::cuda::CUDAGuard guard(q.device());
  const cudaStream_t stream = at::cuda::getCurrentCUDAStream().stream();
  size_t partial_bytes = 0, sync_bytes = 0;
  check_status(kl_paged_decode_workspace_size(dtype, batch, num_q_heads, num_kv_heads, head_dim, page_size,
                                              max_pages, 0, &partial_bytes, &sync_bytes),
               "paged_decode_attention_fp8 (workspace)");
  Scratch& s = scratch_for(q.device(), stream, partial_bytes, sync_bytes);
  check_status(kl_paged_decode_fp8(dtype, out.data_ptr(), q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                                   k_scale.data_ptr<float>(), v_scale.data_ptr<float>(),
                                   block_table.data_ptr<int32_t>(), seq_lens.data_ptr<int32_t>(), batch,
                                   num_q_heads, num_kv_heads, head_dim, page_size, block_table.stride(0), max_pages,
                                   k_cache.size(0), static_cast<float>(scale), 0, s.partials.data_ptr(),
                                   static_cast<size_t>(s.partials.numel()), s.sync.data_ptr(),
                                   static_cast<size_t>(s.sync.numel()), stream),
               "paged_decode_attention_fp8");
}

// Quantising append into an e4m3 cache (kl_paged_kv_append_fp8).
void paged_kv_append_fp8(at::Tensor& k_cache, at::Tensor& v_cache, const at::Tensor& k_new, const at::Tensor& v_new,
                         const at::Tensor& k_scale, const at::Tensor& v_scale, const at::Tensor& block_table,
                         const at::Tensor& positions) {
  TORCH_CHECK(k_cache.is_cuda() && v_cache.is_cuda() && k_new.is_cuda() && v_new.is_cuda(),
              "tensors must be on CUDA");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.is_contiguous() && v_cache.is_contiguous() &&
                  k_cache.sizes() == v_cache.sizes() && is_e4m3(k_cache) && is_e4m3(v_cache),
              "caches are contiguous e4m3 [num_pages, page_size, num_kv_heads, head_dim] of one shape");
  const int64_t num_kv_heads = k_cache.size(2), head_dim = k_cache.size(3);
  TORCH_CHECK(k_new.sizes() == v_new.sizes() && k_new.strides() == v_new.strides() &&
                  k_new.scalar_type() == v_new.scalar_type(),
              "k_new and v_new must have one shape, layout and dtype");
  TORCH_CHECK((k_new.dim() == 3 && k_new.size(1) == num_kv_heads && k_new.size(2) == head_dim &&
               k_new.stride(2) == 1 && k_new.stride(1) == head_dim) ||
                  (k_new.dim() == 2 && k_new.size(1) == num_kv_heads * head_dim && k_new.stride(1) == 1),
              "k_new is [batch, num_kv_heads, head_dim] (or [batch, num_kv_heads*head_dim]) with contiguous rows");
  TORCH_CHECK(block_table.scalar_type() == at::kInt && positions.scalar_type() == at::kInt &&
                  block_table.dim() == 2 && block_table.stride(-1) == 1 && positions.is_contiguous(),
              "block_table rows and positions must be contiguous int32");
  const int64_t batch = k_new.size(0);
  TORCH_CHECK(positions.numel() == batch && block_table.size(0) == batch,
              "block_table and positions need one row / entry per sequence");
  TORCH_CHECK(v_cache.device() == k_cache.device() && k_new.device() == k_cache.device() &&
                  v_new.device() == k_cache.device() && block_table.device() == k_cache.device() &&
                  positions.device() == k_cache.device(),
              "tensors must be on one device");
  check_scales(k_scale, v_scale, num_kv_heads, k_cache.device());
  if (batch == 0) return;
  const c10::cuda::CUDAGuard guard(k_new.device());
  const cudaStream_t stream = at::cuda::getCurrentCUDAStream().stream();
  Scratch& s = scratch_for(k_new.device(), stream, 0, 4);
  check_status(kl_paged_kv_append_fp8(to_dtype(k_new.scalar_type()), k_cache.data_ptr(), v_cache.data_ptr(),
                                      k_new.data_ptr(), v_new.data_ptr(), k_scale.data_ptr<float>(),
                                      v_scale.data_ptr<float>(), block_table.data_ptr<int32_t>(),
                                      positions.data_ptr<int32_t>(), static_cast<int>(batch),
                                      static_cast<int>(num_kv_heads), static_cast<int>(head_dim),
                                      static_cast<int>(k_cache.size(1)), block_table.stride(0),
                                      static_cast<int>(block_table.size(1)), k_cache.size(0), k_new.stride(0),
                                      static_cast<uint32_t*>(s.sync.data_ptr()), stream),
               "paged_kv_append_fp8");
}

// Cascade (shared-prefix) decode (kl_paged_decode_cascade): the sequences of group p,
// [prefix_indptr[p], prefix_indptr[p+1]), attend to the prefix_lens[p] tokens in the pages of
// prefix_block_table row p and then to their own. The caches are q's dtype, or e4m3 with
// per-KV-head scales when k_scale / v_scale are given.
void paged_decode_attention_cascade(at::Tensor& out, const at::Tensor& q, const at::Tensor& k_cache,
                                    const at::Tensor& v_cache, const at::Tensor& prefix_block_table,
                                    const at::Tensor& prefix_lens, const at::Tensor& prefix_indptr,
                                    const at::Tensor& block_table, const at::Tensor& seq_lens, double scale,
                                    const std::optional<at::Tensor>& k_scale, const std::optional<at::Tensor>& v_scale) {
  TORCH_CHECK(q.is_cuda() && k_cache.is_cuda() && v_cache.is_cuda(), "tensors must be on CUDA");
  TORCH_CHECK(q.dim() == 3 && k_cache.dim() == 4, "q is [batch, heads, dim]; caches are 4-D");
  TORCH_CHECK(q.is_contiguous() && out.is_contiguous() && k_cache.is_contiguous() && v_cache.is_contiguous(),
              "q, out and both caches must be contiguous");
  TORCH_CHECK(k_cache.sizes() == v_cache.sizes() && k_cache.scalar_type() == v_cache.scalar_type(),
              "k_cache and v_cache differ in shape or dtype");
  TORCH_CHECK(k_scale.has_value() == v_scale.has_value(), "give both k_scale and v_scale, or neither");
  const bool fp8 = k_scale.has_value();
  if (fp8) {
    TORCH_CHECK(is_e4m3(k_cache), "with scales the caches must be float8_e4m3fn (or uint8 e4m3 codes)");
    TORCH_CHECK(q.scalar_type() == at::kHalf || q.scalar_type() == at::kBFloat16, "q is fp16 or bf16");
  } else {
    TORCH_CHECK(q.scalar_type() == k_cache.scalar_type(), "q and caches must share a dtype");
  }
  TORCH_CHECK(out.scalar_type() == q.scalar_type() && out.sizes() == q.sizes(), "out must match q");
  for (const at::Tensor* t : {&prefix_block_table, &prefix_lens, &prefix_indptr, &block_table, &seq_lens}) {
    TORCH_CHECK(t->scalar_type() == at::kInt && t->device() == q.device(),
                "block tables, lengths and prefix_indptr must be int32 on q's device");
  }
  TORCH_CHECK(block_table.dim() == 2 && block_table.stride(-1) == 1 && prefix_block_table.dim() == 2 &&
                  prefix_block_table.stride(-1) == 1 && seq_lens.is_contiguous() && prefix_lens.is_contiguous() &&
                  prefix_indptr.is_contiguous(),
              "block-table rows, lengths and prefix_indptr must be contiguous");
  TORCH_CHECK(k_cache.device() == q.device() && v_cache.device() == q.device() && out.device() == q.device(),
              "tensors must be on one device");
  const int batch = static_cast<int>(q.size(0));
  const int num_q_heads = static_cast<int>(q.size(1));
  const int head_dim = static_cast<int>(q.size(2));
  const int page_size = static_cast<int>(k_cache.size(1));
  const int num_kv_heads = static_cast<int>(k_cache.size(2));
  TORCH_CHECK(k_cache.size(3) == head_dim, "cache head_dim differs from q");
  TORCH_CHECK(num_kv_heads > 0 && num_q_heads % num_kv_heads == 0, "num_q_heads must be a multiple of num_kv_heads");
  TORCH_CHECK(seq_lens.numel() == batch && block_table.size(0) == batch,
              "block_table and seq_lens need one row / entry per sequence");
  const int64_t groups = prefix_lens.numel();
  TORCH_CHECK(prefix_block_table.size(0) == groups && prefix_indptr.numel() == groups + 1,
              "prefix_block_table needs one row and prefix_indptr groups + 1 entries per prefix group");
  if (fp8) check_scales(*k_scale, *v_scale, num_kv_heads, q.device());
  if (batch == 0) return;
  const int dtype = to_dtype(q.scalar_type());
  const int max_pages = static_cast<int>(block_table.size(1));
  const int max_prefix_pages = static_cast<int>(prefix_block_table.size(1));
  const c10::cuda::CUDAGuard guard(q.device());
  const cudaStream_t stream = at::cuda::getCurrentCUDAStream().stream();
  size_t partial_bytes = 0, sync_bytes = 0;
  check_status(kl_paged_decode_cascade_workspace_size(dtype, batch, static_cast<int>(groups), num_q_heads,
                                                      num_kv_heads, head_dim, page_size, max_pages, max_prefix_pages,
                                                      &partial_bytes, &sync_bytes),
               "paged_decode_attention_cascade (workspace)");
  Scratch& s = scratch_for(q.device(), stream, partial_bytes, sync_bytes);
  check_status(
      kl_paged_decode_cascade(dtype, out.data_ptr(), q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                              fp8 ? k_scale->data_ptr<float>() : nullptr, fp8 ? v_scale->data_ptr<float>() : nullptr,
                              prefix_block_table.data_ptr<int32_t>(), prefix_lens.data_ptr<int32_t>(),
                              prefix_indptr.data_ptr<int32_t>(), static_cast<int>(groups), prefix_block_table.stride(0),
                              max_prefix_pages, block_table.data_ptr<int32_t>(), seq_lens.data_ptr<int32_t>(), batch,
                              num_q_heads, num_kv_heads, head_dim, page_size, block_table.stride(0), max_pages,
                              k_cache.size(0), static_cast<float>(scale), s.partials.data_ptr(),
                              static_cast<size_t>(s.partials.numel()), s.sync.data_ptr(),
                              static_cast<size_t>(s.sync.numel()), stream),
      "paged_decode_attention_cascade");
}

// Status bits (KL_STATUS_*) left by decode calls on the current device and stream.
int64_t decode_status(bool clear) {
  const at::Device dev(at::kCUDA, c10::cuda::current_device());
  const cudaStream_t stream = at::cuda::getCurrentCUDAStream().stream();
  at::Tensor sync;
  {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    auto it = g_scratch.find({dev.index(), stream});
    if (it == g_scratch.end() || !it->second.sync.defined()) return 0;
    sync = it->second.sync;
  }
  uint32_t status = 0;
  check_status(kl_paged_decode_read_status(sync.data_ptr(), &status, clear ? 1 : 0, stream), "decode_status");
  return status;
}

void noop_rms_norm(at::Tensor&, const at::Tensor&, const at::Tensor&, double) {}
void noop_fused(at::Tensor&, const at::Tensor&, at::Tensor&, const at::Tensor&, double) {}
void noop_decode(at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&,
                 const at::Tensor&, double) {}
void noop_decode_splits(at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&,
                        const at::Tensor&, double, int64_t) {}
void noop_append(at::Tensor&, at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&,
                 const at::Tensor&) {}
void noop_decode_fp8(at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&,
                     const at::Tensor&, const at::Tensor&, const at::Tensor&, double) {}
void noop_append_fp8(at::Tensor&, at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&,
                     const at::Tensor&, const at::Tensor&, const at::Tensor&) {}
void noop_cascade(at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&,
                  const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&, double,
                  const std::optional<at::Tensor>&, const std::optional<at::Tensor>&) {}

}  // namespace

TORCH_LIBRARY(kernel_lab, m) {
  m.def("rms_norm(Tensor! out, Tensor x, Tensor weight, float eps) -> ()");
  m.def("fused_add_rms_norm(Tensor! out, Tensor x, Tensor! residual, Tensor weight, float eps) -> ()");
  m.def(
      "paged_decode_attention(Tensor! out, Tensor q, Tensor k_cache, Tensor v_cache, "
      "Tensor block_table, Tensor seq_lens, float scale) -> ()");
  m.def(
      "paged_decode_attention_splits(Tensor! out, Tensor q, Tensor k_cache, Tensor v_cache, "
      "Tensor block_table, Tensor seq_lens, float scale, int num_splits) -> ()");
  m.def(
      "paged_kv_append(Tensor! k_cache, Tensor! v_cache, Tensor k_new, Tensor v_new, "
      "Tensor block_table, Tensor positions) -> ()");
  m.def(
      "paged_decode_attention_fp8(Tensor! out, Tensor q, Tensor k_cache, Tensor v_cache, Tensor k_scale, "
      "Tensor v_scale, Tensor block_table, Tensor seq_lens, float scale) -> ()");
  m.def(
      "paged_kv_append_fp8(Tensor! k_cache, Tensor! v_cache, Tensor k_new, Tensor v_new, Tensor k_scale, "
      "Tensor v_scale, Tensor block_table, Tensor positions) -> ()");
  m.def(
      "paged_decode_attention_cascade(Tensor! out, Tensor q, Tensor k_cache, Tensor v_cache, "
      "Tensor prefix_block_table, Tensor prefix_lens, Tensor prefix_indptr, Tensor block_table, "
      "Tensor seq_lens, float scale, Tensor? k_scale=None, Tensor? v_scale=None) -> ()");
}

TORCH_LIBRARY_IMPL(kernel_lab, CUDA, m) {
  m.impl("rms_norm", &rms_norm);
  m.impl("fused_add_rms_norm", &fused_add_rms_norm);
  m.impl("paged_decode_attention", &paged_decode_attention);
  m.impl("paged_decode_attention_splits", &paged_decode_attention_splits);
  m.impl("paged_kv_append", &paged_kv_append);
  m.impl("paged_decode_attention_fp8", &paged_decode_attention_fp8);
  m.impl("paged_kv_append_fp8", &paged_kv_append_fp8);
  m.impl("paged_decode_attention_cascade", &paged_decode_attention_cascade);
}

TORCH_LIBRARY_IMPL(kernel_lab, Meta, m) {
  m.impl("rms_norm", &noop_rms_norm);
  m.impl("fused_add_rms_norm", &noop_fused);
  m.impl("paged_decode_attention", &noop_decode);
  m.impl("paged_decode_attention_splits", &noop_decode_splits);
  m.impl("paged_kv_append", &noop_append);
  m.impl("paged_decode_attention_fp8", &noop_decode_fp8);
  m.impl("paged_kv_append_fp8", &noop_append_fp8);
  m.impl("paged_decode_attention_cascade", &noop_cascade);
}

// Importing kernel_lab._C runs the registrations above.
PYBIND11_MODULE(_C, m) {
  m.def("decode_status", &decode_status, pybind11::arg("clear") = false,
        "Status bits left by paged_decode_attention on the current device and stream.");
  m.attr("version") = kl_version();
}
