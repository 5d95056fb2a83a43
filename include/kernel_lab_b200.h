/*
 * kernel_lab_b200.h -- C ABI of the B200 (sm_100a) kernels for kernel-lab's two hot paths:
 * fused residual-add + RMSNorm, and paged-KV single-token decode attention.
 *
 * Shared library: libkernel_lab_b200.so. Plain C types only: device pointers are
 * `void*`, a stream is a `cudaStream_t` passed as `void*` (NULL = legacy default
 * stream). Every entry point returns 0 on success or a `cudaError_t` code (as int);
 * nothing throws across the ABI. Work is enqueued on the given stream; no call
 * synchronises the host except kl_paged_decode_read_status.
 *
 * Layouts (all row-major, contiguous unless a stride is given):
 *   x, residual, out   [rows, hidden]   (x rows are x_row_stride elements apart)
 *   weight             [hidden]
 *   q, out             [batch, num_q_heads, head_dim]
 *   k_cache, v_cache   [num_pages, page_size, num_kv_heads, head_dim]        ("NHD")
 *   block_table        [batch, >= max_pages_per_seq] int32, rows block_table_stride apart
 *   seq_lens           [batch] int32
 * Query head h attends with KV head h / (num_q_heads / num_kv_heads) (GQA / MQA).
 */
#ifndef KERNEL_LAB_B200_H_
#define KERNEL_LAB_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Storage dtypes; same order as kernel_lab::DType (csrc/kernel_lab.h:12 in kernel-lab). */
enum {
  KL_FLOAT32 = 0,
  KL_FLOAT16 = 1,
  KL_BFLOAT16 = 2
};

/* Status bits a decode call leaves in word 0 of its sync buffer (sticky; see
 * kl_paged_decode_read_status). */
enum {
  KL_STATUS_BAD_PAGE = 1,     /* a block-table entry outside [0, num_pages): that page was skipped */
  KL_STATUS_LEN_CLAMPED = 2,  /* a sequence longer than max_pages_per_seq * page_size was clamped */
  KL_STATUS_WAIT_TIMEOUT = 4,  /* an internal pipeline wait exceeded its time limit; output is invalid */
  KL_STATUS_BAD_PREFIX_GROUPS = 8, /* cascade: prefix_indptr is not a partition of the batch; prefixes ignored */
  KL_STATUS_PEER_TIMEOUT = 16      /* head gather: another rank's arrival did not come in time */
};

/* Library version string, e.g. "kernel_lab_b200 0.1.0 sm_100a". */
const char* kl_version(void);

/* Human-readable text for a status code returned by any kl_* call. */
const char* kl_status_string(int status);

/*
 * RMSNorm over rows of length `hidden`. With `residual` non-NULL this is the fused
 * pre-norm step: residual <- dtype(x + residual) (in place, bit-exact), then
 * out <- dtype(residual * rsqrt(mean(residual^2) + eps) * weight). With `residual`
 * NULL: out <- rmsnorm(x). fp32 math. rows == 0 is a no-op.
 *
 * Replaces kernel_lab::launch_rms_norm (csrc/kernel_lab.h:14-19 in kernel-lab), same
 * arguments; called by the torch ops rms_norm / fused_add_rms_norm
 * (csrc/torch_bindings.cpp:31-69).
 */
int kl_rms_norm(int dtype, void* out, const void* x, void* residual, const void* weight, int rows,
                int hidden, int64_t x_row_stride, float eps, void* stream);

/*
 * Scratch needed by kl_paged_decode for this problem on the current device:
 *   *partial_bytes: per-split partial outputs (no initialisation needed);
 *   *sync_bytes:    status word + one arrival counter per (sequence, KV head); must
 *                   be zero before its first use (cudaMemset), and every call leaves
 *                   the counters zero again, so one buffer serves any later call that
 *                   fits in it.
 * num_splits: 0 = load-balanced planner; > 0 = force that many KV splits per sequence
 * (the kernel-lab Triton semantics: pages_per_split = ceil(max_pages_per_seq / num_splits)).
 */
int kl_paged_decode_workspace_size(int dtype, int batch, int num_q_heads, int num_kv_heads, int head_dim,
                                   int page_size, int max_pages_per_seq, int num_splits,
                                   size_t* partial_bytes, size_t* sync_bytes);

/*
 * Single-token decode attention over a paged KV cache, split-KV with an exact
 * log-sum-exp merge:  out[b, h] = softmax(scale * q[b, h] . K_b^T) V_b.
 * Only the first ceil(seq_lens[b] / page_size) block-table entries of row b are read.
 * seq_lens[b] == 0 yields zeros. num_pages bounds valid page ids (entries outside
 * [0, num_pages) are skipped and flagged KL_STATUS_BAD_PAGE). The scratch buffers come
 * from kl_paged_decode_workspace_size; calls that overlap on the GPU need separate
 * buffers. batch == 0 is a no-op.
 *
 * Superset of kernel_lab::launch_paged_decode_attention (csrc/kernel_lab.h:21-33 in
 * kernel-lab), which is the torch op paged_decode_attention's backend
 * (csrc/torch_bindings.cpp:71-103): adds the block-table width, the pool size, the
 * split override and caller-owned scratch. Any head_dim, group size and page size are
 * accepted (fp16/bf16 with head_dim 64/128/256 run on the tensor-core path).
 */
int kl_paged_decode(int dtype, void* out, const void* q, const void* k_cache, const void* v_cache,
                    const int32_t* block_table, const int32_t* seq_lens, int batch, int num_q_heads,
                    int num_kv_heads, int head_dim, int page_size, int64_t block_table_stride,
                    int max_pages_per_seq, int64_t num_pages, float scale, int num_splits, void* partials,
                    size_t partial_bytes, void* sync, size_t sync_bytes, void* stream);

/*
 * Exactly the argument list of kernel_lab::launch_paged_decode_attention
 * (csrc/kernel_lab.h:27-33 in kernel-lab). The block-table width is taken to be
 * block_table_stride and page ids are not range-checked (the pool size is unknown), as
 * in kernel-lab. Scratch comes from cudaMallocAsync on `stream` and is freed on it.
 */
int kl_paged_decode_attention(int dtype, void* out, const void* q, const void* k_cache, const void* v_cache,
                              const int32_t* block_table, const int32_t* seq_lens, int batch,
                              int num_q_heads, int num_kv_heads, int head_dim, int page_size,
                              int64_t block_table_stride, float scale, void* stream);

/*
 * Synchronise `stream`, copy status word 0 of a decode sync buffer to *status and,
 * if clear != 0, reset it to zero.
 */
int kl_paged_decode_read_status(void* sync, uint32_t* status, int clear, void* stream);

/*
 * Multi-GPU decode sharded by KV head (tensor parallel; one process per GPU of one node), with
 * the head gather fused into the decode kernel. Rank r of N holds KV heads [r*Hkv, (r+1)*Hkv)
 * of the pool (its own contiguous NHD pool of Hkv heads) and their query heads
 * [r*Hq, (r+1)*Hq) of q; num_q_heads / num_kv_heads below are these per-rank counts. Every
 * rank's output is the whole [batch, N*num_q_heads, head_dim]: the kernel stores each final row
 * into this rank's output and, with plain stores over NVLink, into every other rank's, at this
 * rank's head offset. The last CTA to finish on a GPU then publishes the call's epoch into every
 * rank's flags and waits until all N ranks have published it, so when the call completes on a
 * rank's stream that rank's output holds every head. No NCCL call, no copy, no multicast.
 *
 * Buffers: out[r] and flags[r] are rank r's output and flags as mapped in this process (through
 * kl_ipc_open for r != rank); flags[r] is uint32[N], done is one uint32 of this rank; both start
 * at zero (kl_ipc_alloc zeroes its memory). epoch must be the same on every rank for the same
 * call, start at 1 and grow by one per call. Ranks must be on distinct GPUs (they wait on one
 * another) and make the same calls in the same order. Peers write a rank's output while that
 * rank may still be reading an earlier call's: call e + 1 of a peer can run once every rank has
 * arrived at call e. Alternate the output regions by epoch: two regions when every reader of a
 * call's output is stream-ordered before the rank's next call, three when a reader (a copy on
 * another stream, say) only has to finish before the call after next. A rank whose peers do not
 * arrive within timeout_ms (0: 10 s) sets KL_STATUS_PEER_TIMEOUT in `sync` and returns (its
 * output then lacks the late ranks' heads; its own heads are stored).
 * num_ranks == 1: plain kl_paged_decode into out[0].
 *
 * Tensor-core shapes only (fp16/bf16, head_dim 64/128/256, page size 8 or a multiple of 16, the
 * pointers 16-byte aligned); other calls return cudaErrorNotSupported. Scratch as for
 * kl_paged_decode with the per-rank shape. No counterpart in kernel-lab (single-GPU).
 */
#define KL_GATHER_MAX_RANKS 8
#define KL_IPC_HANDLE_BYTES 64

typedef struct kl_head_gather {
  int num_ranks;
  int rank;
  uint32_t epoch;
  void* out[KL_GATHER_MAX_RANKS];
  uint32_t* flags[KL_GATHER_MAX_RANKS];
  uint32_t* done;
  uint32_t timeout_ms; /* wait for the peers' arrivals; 0: 10 s */
} kl_head_gather_t;

int kl_paged_decode_gather(int dtype, const kl_head_gather_t* gather, const void* q, const void* k_cache,
                           const void* v_cache, const int32_t* block_table, const int32_t* seq_lens, int batch,
                           int num_q_heads, int num_kv_heads, int head_dim, int page_size,
                           int64_t block_table_stride, int max_pages_per_seq, int64_t num_pages, float scale,
                           void* partials, size_t partial_bytes, void* sync, size_t sync_bytes, void* stream);

/*
 * Device memory another process of this node can map (CUDA IPC; plain peer mappings, no
 * multicast): kl_ipc_alloc allocates `bytes` on the current device, zeroes them and writes the
 * KL_IPC_HANDLE_BYTES-byte handle a peer passes to kl_ipc_open to map them (on its own current
 * device, peer access enabled). kl_ipc_close unmaps a peer's buffer; kl_ipc_free frees one's own.
 * These are set-up calls (they synchronise); no counterpart in kernel-lab.
 */
int kl_ipc_alloc(size_t bytes, void** ptr, void* handle);
int kl_ipc_open(const void* handle, void** ptr);
int kl_ipc_close(void* ptr);
int kl_ipc_free(void* ptr);

/* Bytes of device memory the library reserves per GPU for kl_paged_decode_noalloc. */
#define KL_NOALLOC_SCRATCH_BYTES ((16u << 20) + (256u << 10))

/*
 * kl_paged_decode for callers that cannot allocate device memory when they call it: a
 * server whose GPU memory was handed out to its own pools at start-up, a runtime that has
 * reserved every free byte for the KV cache, or a step loop that must never call
 * cudaMalloc. It allocates nothing; the caller passes inputs and outputs only. Scratch is
 * one fixed array in this library's device memory, KL_NOALLOC_SCRATCH_BYTES per GPU
 * (16 MiB of split partials + 256 KiB of counters), held until process exit.
 *
 * - CUDA reserves the array on a GPU when it loads this library's device code there. With
 *   lazy module loading (CUDA's default) that is the first kernel launch or symbol lookup on
 *   that GPU, not dlopen. A host that hands all free memory to its own pools at start-up must
 *   therefore make one call (or any kl_* launch) on each GPU first, or run with
 *   CUDA_MODULE_LOADING=EAGER; otherwise that first call can fail with an out-of-memory error.
 * - A problem whose scratch (kl_paged_decode_workspace_size) exceeds that array is rejected
 *   with cudaErrorMemoryAllocation before anything is launched (batch 64, context 4096,
 *   32/8 heads of 128 fit with room to spare).
 * - The first call on a device looks up the array's device address (cudaGetSymbolAddress)
 *   with that device current; make that first call before capturing any stream.
 * - Every call on a device shares the one array and leaves its contents behind; each call
 *   zeroes the counters and the status word (a cudaMemsetAsync on `stream`) before its
 *   kernel. Calls that overlap on the GPU (other streams, other host threads) race on the
 *   array: run them in one stream order.
 * - The status bits of kl_paged_decode (KL_STATUS_*) go to word 0 of the array; read them with
 *   kl_paged_decode_noalloc_read_status before the next call on the device clears them.
 * Arguments and results are otherwise those of kl_paged_decode without the scratch buffers.
 * No counterpart in kernel-lab.
 */
int kl_paged_decode_noalloc(int dtype, void* out, const void* q, const void* k_cache, const void* v_cache,
                            const int32_t* block_table, const int32_t* seq_lens, int batch, int num_q_heads,
                            int num_kv_heads, int head_dim, int page_size, int64_t block_table_stride,
                            int max_pages_per_seq, int64_t num_pages, float scale, int num_splits, void* stream);

/*
 * Status bits (KL_STATUS_*) left by the last kl_paged_decode_noalloc call on the current device:
 * synchronises `stream`, copies word 0 of the library's array to *status and, if clear != 0,
 * resets it. Call it after the decode and before the next kl_paged_decode_noalloc on this
 * device, which clears the word. Allocates nothing. No counterpart in kernel-lab.
 */
int kl_paged_decode_noalloc_read_status(uint32_t* status, int clear, void* stream);

/*
 * Paged KV append: write each sequence's new token's K and V rows into its pages.
 *   k_cache, v_cache    [num_pages, page_size, num_kv_heads, head_dim]   (NHD, contiguous)
 *   k_new, v_new        [batch][num_kv_heads * head_dim], rows new_row_stride elements apart
 *                       (a view of a fused QKV output needs no copy)
 *   block_table         [batch, block_table_stride] int32, max_pages_per_seq entries used
 *   positions           [batch] int32: token index written (the length before the append);
 *                       negative = skip the sequence
 * Token p of sequence b goes to page block_table[b, p / page_size], slot p % page_size. A
 * position past max_pages_per_seq * page_size or a page id outside [0, num_pages) (num_pages < 0:
 * unchecked) skips that sequence and ORs KL_STATUS_BAD_PAGE into *status (if non-null, a
 * device word). Stream-ordered, no allocation. No counterpart in kernel-lab (its pools are
 * built on the host); the layout is that of kernel-lab's csrc/kernel_lab.h:21-26.
 */
int kl_paged_kv_append(int dtype, void* k_cache, void* v_cache, const void* k_new, const void* v_new,
                       const int32_t* block_table, const int32_t* positions, int batch, int num_kv_heads,
                       int head_dim, int page_size, int64_t block_table_stride, int max_pages_per_seq,
                       int64_t num_pages, int64_t new_row_stride, uint32_t* status, void* stream);

/*
 * FP8 KV cache (the roadmap item of kernel-lab's README.md:98): k_cache / v_cache hold e4m3
 * codes (one byte per element, same NHD layout), dequantised as code value * k_scale[h] (or
 * v_scale[h]) for KV head h; k_scale, v_scale are [num_kv_heads] fp32 device arrays. q and out
 * are fp16 or bf16 (dtype). Otherwise exactly kl_paged_decode, including the scratch from
 * kl_paged_decode_workspace_size (same dtype and shape arguments). head_dim 128 or 256, page
 * size 8 or a multiple of 16; other shapes return cudaErrorInvalidValue. The MMAs run in f16
 * (e4m3 -> f16 is exact; q is rounded to f16, probabilities to f16), accumulating in fp32.
 * No counterpart in kernel-lab.
 */
int kl_paged_decode_fp8(int dtype, void* out, const void* q, const void* k_cache, const void* v_cache,
                        const float* k_scale, const float* v_scale, const int32_t* block_table,
                        const int32_t* seq_lens, int batch, int num_q_heads, int num_kv_heads, int head_dim,
                        int page_size, int64_t block_table_stride, int max_pages_per_seq, int64_t num_pages,
                        float scale, int num_splits, void* partials, size_t partial_bytes, void* sync,
                        size_t sync_bytes, void* stream);

/*
 * kl_paged_kv_append into an e4m3 cache: each new row (dtype fp32, fp16 or bf16) is quantised
 * per KV head as e4m3(x / scale[h]) (float32 division, round to nearest-even, saturating to
 * +-448; NaN stays NaN) and written like kl_paged_kv_append. head_dim must be even.
 * No counterpart in kernel-lab.
 */
int kl_paged_kv_append_fp8(int dtype, void* k_cache, void* v_cache, const void* k_new, const void* v_new,
                           const float* k_scale, const float* v_scale, const int32_t* block_table,
                           const int32_t* positions, int batch, int num_kv_heads, int head_dim, int page_size,
                           int64_t block_table_stride, int max_pages_per_seq, int64_t num_pages,
                           int64_t new_row_stride, uint32_t* status, void* stream);

/*
 * Cascade (shared-prefix) decode: the sequences of group p, [prefix_indptr[p], prefix_indptr[p+1]),
 * share the prefix_lens[p] tokens held in the pages of row p of prefix_block_table
 * ([num_prefixes, >= max_prefix_pages] int32, rows prefix_block_table_stride apart, pages of the
 * same pools). Sequence b attends to its group's prefix tokens and then to its own
 * seq_lens[b] tokens (block_table row b):
 *   out[b, h] = softmax(scale * q[b, h] . [K_prefix(b); K_b]^T) [V_prefix(b); V_b].
 * A prefix's pages are read once per block of sequences of its group (the block's query rows
 * share each tensor-core MMA), not once per sequence, and the two parts are merged exactly by
 * their log-sum-exp in the same launch. prefix_indptr must partition the batch (entry 0 = 0,
 * non-decreasing, entry num_prefixes = batch); otherwise the prefixes are ignored and
 * KL_STATUS_BAD_PREFIX_GROUPS is set. num_prefixes == 0 is plain kl_paged_decode. k_scale and
 * v_scale both NULL: caches of `dtype`; both given: e4m3 caches as in kl_paged_decode_fp8.
 * Tensor-core shapes only (fp16/bf16, head_dim 64/128/256, page size 8 or a multiple of 16);
 * other shapes return cudaErrorInvalidValue. Scratch from
 * kl_paged_decode_cascade_workspace_size, with the same rules as kl_paged_decode's.
 * Mirrors FlashInfer's two-level cascade (shared prefix + unique suffix), which kernel-lab names
 * as a next step (docs/design.md:96-102); no counterpart in kernel-lab.
 */
int kl_paged_decode_cascade_workspace_size(int dtype, int batch, int num_prefixes, int num_q_heads,
                                           int num_kv_heads, int head_dim, int page_size, int max_pages_per_seq,
                                           int max_prefix_pages, size_t* partial_bytes, size_t* sync_bytes);

int kl_paged_decode_cascade(int dtype, void* out, const void* q, const void* k_cache, const void* v_cache,
                            const float* k_scale, const float* v_scale, const int32_t* prefix_block_table,
                            const int32_t* prefix_lens, const int32_t* prefix_indptr, int num_prefixes,
                            int64_t prefix_block_table_stride, int max_prefix_pages, const int32_t* block_table,
                            const int32_t* seq_lens, int batch, int num_q_heads, int num_kv_heads, int head_dim,
                            int page_size, int64_t block_table_stride, int max_pages_per_seq, int64_t num_pages,
                            float scale, void* partials, size_t partial_bytes, void* sync, size_t sync_bytes,
                            void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KERNEL_LAB_B200_H_ */
