// Paged-KV single-token decode attention for sm_100a: split-KV with an exact
// log-sum-exp merge, GQA head packing, TMA page staging and a load-balanced planner.
//
// What it replaces: kernel-lab's warp-per-token CUDA kernel (csrc/paged_attention.cu:27-128),
// with the split/merge semantics of its Triton kernel
// (kernel_lab/triton_kernels/paged_attention.py:37-173): partial outputs are normalised,
// carry a base-2 LSE, and an empty split has lse = -inf and zero weight.
//
// Work decomposition. The unit of work is a 16-token "tile" of one (sequence, KV head).
// Every CTA computes the same plan from seq_lens (no host sync): the tiles of all
// (sequence, KV head) pairs are laid end to end, and CTA c takes the contiguous range
// [c*R, (c+1)*R) with R = max(min_tiles, ceil(total / grid)). Every CTA therefore streams
// the same number of KV bytes whatever the length distribution (ragged batches included).
// A (sequence, KV head) that a range boundary cuts is a "chunk": the CTA writes a
// normalised fp32 partial and its LSE to scratch and bumps an arrival counter; the CTA
// that arrives last merges all chunks (no waiting on other CTAs) and resets the counter.
// A forced split count (num_splits > 0) instead gives every sequence exactly
// ceil(max_pages / pages_per_split) splits, including empty ones, like the Triton kernel.
//
// Tensor-core kernel (fp16/bf16, head_dim 64/128/256, page size 8 or a multiple of 16):
// one producer warp walks the plan and issues 2-D TMA loads of each tile's K and V rows
// (block-table indirection, 128-byte swizzle, L2 evict-first) into a ring of shared-memory
// stages guarded by mbarriers; four consumer warps take tiles round-robin. A consumer warp
// computes S = K.Q^T with mma.m16n8k16 (M = 16 tokens, N = 8 query heads of the group,
// K = head_dim), does the online softmax in base 2 on the fp32 fragments, turns P into
// the B operand with movmatrix, and accumulates O^T += V^T.P^T (V^T via ldmatrix.trans).
// Partial results of the consumer warps are combined through shared memory.
//
// Generic kernel (fp32, other head_dims / page sizes / groups): same plan and merge, CUDA
// cores, 32-token chunks staged through shared memory.
//
// Safety: pages outside [0, num_pages) are skipped and flagged; every mbarrier wait is
// bounded in time and flags a timeout; the producer lets all its copies land before exit.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"
#include "kernel_lab_b200.h"

namespace klb {

constexpr int kTile = 16;          // tokens per tile: the MMA's M
constexpr int kCW = 4;             // consumer warps (tensor-core kernel)
constexpr int kTCThreads = 32 * (kCW + 1);
constexpr int kGenThreads = 128;
constexpr int kGenChunk = 32;      // tokens per step of the generic kernel
constexpr int kMaxBatch = 16384;   // the plan lives in shared memory
constexpr uint64_t kWaitLimitNs = 1000000000ull;

struct DecodeArgs {
  void* out;
  const void* q;
  const void* k_cache;
  const void* v_cache;
  const int32_t* block_table;
  const int32_t* seq_lens;
  int batch, num_q_heads, num_kv_heads, group, head_dim, page_size;
  int64_t bt_stride;
  int max_pages;
  int64_t num_pages;  // < 0: unknown, page ids not range-checked
  float scale_log2;
  int splits;           // 0: balanced plan; > 0: forced splits per sequence
  int pages_per_split;  // forced mode
  int min_tiles;        // balanced mode: minimum tiles per CTA
  uint32_t* sync;       // [0] status, [1 + b * Hkv + kvh] arrival counters
  float* part_o;        // [slot][group][head_dim]
  float* part_lse;      // [slot][group]
};

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ------------------------------------------------------------------------- plan

struct Seg {
  int b, kvh;
  int tok_begin, tok_end;  // token range; empty when tok_end <= tok_begin
  int slot;                // partial slot of this chunk (unused when whole)
  int nchunks;             // chunks of this (sequence, KV head)
  int c_first;             // balanced mode: CTA holding the first chunk
  bool first_aligned;      // balanced mode: first chunk starts its CTA's range
  bool whole;
};

struct Walk {
  int t, t1, R;     // balanced
  int item, items;  // forced
};

__device__ __forceinline__ int clamp_len(const DecodeArgs& a, int b, bool report) {
  int len = a.seq_lens[b];
  const int cap = a.max_pages * a.page_size;
  if (len > cap) {
    if (report) atomicOr(a.sync, kStatusLenClamped);
    len = cap;
  }
  return len < 0 ? 0 : len;
}

// All threads of the block. lens[b] = clamped length; prefix[b] = tiles of sequences
// before b (balanced mode); misc[0] = total tiles over all KV heads, misc[1] = R.
// misc[4..35] is scan scratch. Ends with a block barrier.
__device__ void plan_build(const DecodeArgs& a, int* lens, int* prefix, int* misc) {
  const int B = a.batch;
  const int nt = blockDim.x;
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5, nw = nt >> 5;
  const int per = (B + nt - 1) / nt;
  const int lo = min(B, tid * per), hi = min(B, lo + per);
  int local = 0;
  for (int i = lo; i < hi; ++i) {
    const int len = clamp_len(a, i, blockIdx.x == 0);
    lens[i] = len;
    local += (len + kTile - 1) / kTile;
  }
  // Block-wide exclusive scan of `local`.
  int inc = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += v;
  }
  int* wtot = misc + 4;
  if (lane == 31) wtot[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    const int v = lane < nw ? wtot[lane] : 0;
    int vi = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, vi, o);
      if (lane >= o) vi += u;
    }
    if (lane < nw) wtot[lane] = vi - v;
    if (lane == 31) misc[2] = vi;  // total tiles of one KV head
  }
  __syncthreads();
  int run = wtot[warp] + inc - local;
  for (int i = lo; i < hi; ++i) {
    prefix[i] = run;
    run += (lens[i] + kTile - 1) / kTile;
  }
  if (tid == 0) {
    const int per_head = misc[2];
    prefix[B] = per_head;
    const int total = per_head * a.num_kv_heads;
    misc[0] = total;
    misc[1] = max(a.min_tiles, (total + (int)gridDim.x - 1) / (int)gridDim.x);
    misc[2] = 0;  // abort flag from here on
    misc[3] = 0;  // "last arrival" flag
  }
  __syncthreads();
}

__device__ __forceinline__ void walk_init(const DecodeArgs& a, const int* misc, Walk& w) {
  if (a.splits == 0) {
    const int total = misc[0];
    w.R = misc[1];
    const int64_t t0 = static_cast<int64_t>(blockIdx.x) * w.R;
    w.t = static_cast<int>(min(t0, static_cast<int64_t>(total)));
    w.t1 = static_cast<int>(min(t0 + w.R, static_cast<int64_t>(total)));
  } else {
    w.item = blockIdx.x;
    w.items = a.batch * a.num_kv_heads * a.splits;
  }
}

__device__ __forceinline__ bool walk_next(const DecodeArgs& a, const int* lens, const int* prefix, Walk& w,
                                          Seg& s) {
  const int H = a.num_kv_heads;
  if (a.splits == 0) {
    if (w.t >= w.t1) return false;
    int lo = 0, hi = a.batch - 1;  // largest b with H * prefix[b] <= t
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (static_cast<int64_t>(H) * prefix[mid] <= w.t) lo = mid; else hi = mid - 1;
    }
    const int b = lo;
    const int n = prefix[b + 1] - prefix[b];
    const int seq0 = H * prefix[b];
    const int off = w.t - seq0;
    const int kvh = off / n, tile = off - kvh * n;
    const int len = min(n - tile, w.t1 - w.t);
    const int s_begin = seq0 + kvh * n;
    const int s_end = s_begin + n;
    s.b = b;
    s.kvh = kvh;
    s.tok_begin = tile * kTile;
    s.tok_end = min(lens[b], (tile + len) * kTile);
    s.c_first = s_begin / w.R;
    s.nchunks = (s_end - 1) / w.R - s.c_first + 1;
    s.first_aligned = s_begin == s.c_first * w.R;
    s.whole = s.nchunks == 1;
    s.slot = w.t == static_cast<int>(blockIdx.x) * w.R ? 2 * blockIdx.x : 2 * blockIdx.x + 1;
    w.t += len;
    return true;
  }
  if (w.item >= w.items) return false;
  const int i = w.item;
  const int S = a.splits;
  s.kvh = i % H;
  const int sp = (i / H) % S;
  s.b = i / (H * S);
  const int span = a.pages_per_split * a.page_size;
  s.tok_begin = sp * span;
  s.tok_end = max(s.tok_begin, min(lens[s.b], s.tok_begin + span));
  s.slot = i;
  s.nchunks = S;
  s.c_first = 0;
  s.first_aligned = true;
  s.whole = S == 1;
  w.item += gridDim.x;
  return true;
}

__device__ __forceinline__ int chunk_slot(const DecodeArgs& a, const Seg& s, int k) {
  if (a.splits == 0) {
    const int c = s.c_first + k;
    return (k == 0 && !s.first_aligned) ? 2 * c + 1 : 2 * c;
  }
  return (s.b * a.splits + k) * a.num_kv_heads + s.kvh;
}

// ------------------------------------------------------------------------- emit / merge

// One output element of a segment: O / L is the normalised value, M (base 2) its max.
template <typename T>
__device__ __forceinline__ void emit_value(const DecodeArgs& a, const Seg& s, int h, int d, float O, float L,
                                           float M) {
  const int G = a.group, D = a.head_dim;
  const float o = L > 0.0f ? O / L : 0.0f;
  if (s.whole) {
    T* out = static_cast<T*>(a.out);
    out[(static_cast<int64_t>(s.b) * a.num_q_heads + s.kvh * G + h) * D + d] = Storage<T>::store(o);
  } else {
    a.part_o[(static_cast<int64_t>(s.slot) * G + h) * D + d] = o;
    if (d == 0) a.part_lse[static_cast<int64_t>(s.slot) * G + h] = L > 0.0f ? M + __log2f(L) : -INFINITY;
  }
}

// Called by the `nthr` threads that emitted this segment. The chunk's partial is
// published; the last chunk to arrive for its (sequence, KV head) merges them all.
template <typename T, typename Sync>
__device__ __forceinline__ void merge_if_last(const DecodeArgs& a, const Seg& s, int ctid, int nthr,
                                              volatile int* flag, Sync sync) {
  if (s.whole) return;
  __threadfence();
  sync();
  uint32_t* counter = a.sync + 1 + s.b * a.num_kv_heads + s.kvh;
  if (ctid == 0) {
    const uint32_t old = atomicAdd(counter, 1u);
    *flag = old == static_cast<uint32_t>(s.nchunks - 1);
  }
  sync();
  if (*flag) {
    __threadfence();
    const int G = a.group, D = a.head_dim;
    T* out = static_cast<T*>(a.out);
    for (int idx = ctid; idx < G * D; idx += nthr) {
      const int h = idx / D, d = idx - h * D;
      float M = -INFINITY;
      for (int k = 0; k < s.nchunks; ++k) {
        M = fmaxf(M, __ldcg(a.part_lse + static_cast<int64_t>(chunk_slot(a, s, k)) * G + h));
      }
      float W = 0.0f, O = 0.0f;
      if (M > -INFINITY) {
        for (int k = 0; k < s.nchunks; ++k) {
          const int64_t slot = chunk_slot(a, s, k);
          const float lse = __ldcg(a.part_lse + slot * G + h);
          if (lse > -INFINITY) {
            const float wk = fast_exp2(lse - M);
            W += wk;
            O += wk * __ldcg(a.part_o + (slot * G + h) * D + d);
          }
        }
      }
      out[(static_cast<int64_t>(s.b) * a.num_q_heads + s.kvh * G + h) * D + d] =
          Storage<T>::store(W > 0.0f ? O / W : 0.0f);
    }
    if (ctid == 0) atomicExch(counter, 0u);
  }
}

// Zero the outputs of empty sequences (balanced mode has no work item for them).
template <typename T>
__device__ __forceinline__ void zero_empty_sequences(const DecodeArgs& a, const int* lens, int ctid, int nthr) {
  if (a.splits != 0) return;
  T* out = static_cast<T*>(a.out);
  const int n = a.num_q_heads * a.head_dim;
  for (int b = blockIdx.x; b < a.batch; b += gridDim.x) {
    if (lens[b] != 0) continue;
    for (int i = ctid; i < n; i += nthr) out[static_cast<int64_t>(b) * n + i] = Storage<T>::store(0.0f);
  }
}

// ------------------------------------------------------------------------- tensor-core kernel

struct TcLayout {
  uint32_t stage_bytes, ring, bars, red_m, red_l, red_acc, misc, prefix, lens, total;
};

__host__ __device__ constexpr uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

__host__ __device__ inline TcLayout tc_layout(int D, int NT, int nstage, int batch) {
  TcLayout L{};
  L.stage_bytes = 2u * kTile * D * 2u;
  uint32_t off = 0;
  L.ring = off;
  off += nstage * L.stage_bytes;
  L.bars = off;
  off += 2u * nstage * 8u;
  L.red_m = off;
  off += kCW * 8u * NT * 4u;
  L.red_l = off;
  off += kCW * 8u * NT * 4u;
  L.red_acc = off;
  off += kCW * 8u * NT * (D + 4u) * 4u;
  L.misc = off;
  off += 64u * 4u;
  L.prefix = off;
  off += (batch + 1u) * 4u;
  L.lens = off;
  off += batch * 4u;
  L.total = align_up(off, 16) + 1024u;  // slack to align the base to 1024 B (swizzle atom)
  return L;
}

template <typename T, int D, int NT>
__global__ void __launch_bounds__(kTCThreads) decode_tc_kernel(const __grid_constant__ CUtensorMap tmk,
                                                               const __grid_constant__ CUtensorMap tmv,
                                                               const DecodeArgs a, const int nstage,
                                                               const int p_rows, const int hg_count) {
  constexpr int KS = D / 16;   // k-steps of K.Q^T, m-tiles of V^T.P^T
  constexpr int NCH = D / 64;  // 128-byte chunks of one token row of one head
  constexpr int HPW = 8 * NT;  // query heads per consumer warp
  constexpr uint32_t kHalf = kTile * D * 2;  // bytes of the K (or V) half of a stage
  constexpr uint32_t kChunkBytes = kTile * 128;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const TcLayout L = tc_layout(D, NT, nstage, a.batch);
  const uint32_t ring = smem_u32(smem + L.ring);
  const uint32_t bars = smem_u32(smem + L.bars);
  float* red_m = reinterpret_cast<float*>(smem + L.red_m);
  float* red_l = reinterpret_cast<float*>(smem + L.red_l);
  float* red_acc = reinterpret_cast<float*>(smem + L.red_acc);
  int* misc = reinterpret_cast<int*>(smem + L.misc);
  int* prefix = reinterpret_cast<int*>(smem + L.prefix);
  int* lens = reinterpret_cast<int*>(smem + L.lens);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int HG = hg_count, TW = kCW / hg_count;

  if (threadIdx.x == 0) {
    for (int s = 0; s < nstage; ++s) {
      mbar_init(bars + 8u * s, 1);                    // full: the producer's expect_tx arrival
      mbar_init(bars + 8u * (nstage + s), hg_count);  // empty: one arrival per consuming warp
    }
    fence_barrier_init();
  }
  if (warp == kCW && lane == 0) {
    tma_prefetch_descriptor(&tmk);
    tma_prefetch_descriptor(&tmv);
  }
  plan_build(a, lens, prefix, misc);
  volatile int* abort_flag = misc + 2;

  if (warp == kCW) {
    // ---------------- producer warp
    Walk w;
    walk_init(a, misc, w);
    Seg s;
    uint32_t gt = 0;
    const uint64_t policy = l2_policy_evict_first();
    const int nsub = kTile / p_rows;
    const uint32_t sub_bytes = 2u * NCH * p_rows * 128u;
    bool ok = true;
    while (ok && walk_next(a, lens, prefix, w, s)) {
      const int ntok = s.tok_end - s.tok_begin;
      if (ntok <= 0) continue;
      const int ntiles = (ntok + kTile - 1) / kTile;
      const int32_t* bt_row = a.block_table + static_cast<int64_t>(s.b) * a.bt_stride;
      const int last_page = (s.tok_end - 1) / a.page_size;
      // The warp caches 32 consecutive block-table entries (one per lane) and
      // prefetches the next 32, so page lookups never stall the TMA issue.
      int cur_base = INT_MIN / 2, nxt_base = INT_MIN / 2;
      int32_t cur = 0, nxt = 0;
      for (int j = 0; j < ntiles; ++j, ++gt) {
        const int stage = static_cast<int>(gt % nstage);
        const uint32_t full = bars + 8u * stage;
        const uint32_t empty = bars + 8u * (nstage + stage);
        if (*abort_flag || !mbar_wait_bounded(empty, ((gt / nstage) & 1u) ^ 1u, a.sync, kWaitLimitNs)) {
          *abort_flag = 1;
          ok = false;
          break;
        }
        const int t0 = s.tok_begin + j * kTile;
        uint32_t bytes = 0;
        int ys[2] = {0, 0};
        bool vs[2] = {false, false};
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          if (r >= nsub) break;
          const int tok = t0 + r * p_rows;
          if (tok >= s.tok_end) break;
          const int pidx = tok / a.page_size;
          if (pidx < cur_base || pidx >= cur_base + 32) {
            if (pidx == nxt_base) {
              cur = nxt;
              cur_base = nxt_base;
            } else {
              cur_base = pidx;
              cur = pidx + lane <= last_page ? __ldg(bt_row + pidx + lane) : 0;
            }
            nxt_base = cur_base + 32;
            nxt = nxt_base + lane <= last_page ? __ldg(bt_row + nxt_base + lane) : 0;
          }
          const int page = __shfl_sync(0xffffffffu, cur, pidx - cur_base);
          if (page < 0 || (a.num_pages >= 0 && page >= a.num_pages)) {
            if (lane == 0) atomicOr(a.sync, kStatusBadPage);
          } else {
            vs[r] = true;
            ys[r] = page * a.page_size + (tok - pidx * a.page_size);
            bytes += sub_bytes;
          }
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(full, bytes);
          const uint32_t sk = ring + stage * L.stage_bytes;
          const uint32_t sv = sk + kHalf;
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            if (!vs[r]) continue;
#pragma unroll
            for (int c = 0; c < NCH; ++c) {
              const uint32_t dst = c * kChunkBytes + r * p_rows * 128u;
              const int x = s.kvh * D + c * 64;
              tma_load_2d(sk + dst, &tmk, x, ys[r], full, policy);
              tma_load_2d(sv + dst, &tmv, x, ys[r], full, policy);
            }
          }
        }
        __syncwarp();
      }
    }
    // Let every copy this CTA issued land before the CTA may exit.
    const uint32_t inflight = min(gt, static_cast<uint32_t>(nstage));
    for (uint32_t k = gt - inflight; k < gt; ++k) {
      mbar_wait_bounded(bars + 8u * (k % nstage), (k / nstage) & 1u, a.sync, kWaitLimitNs);
    }
    return;
  }

  // ---------------- consumer warps (threads 0..127)
  const int ctid = threadIdx.x;
  zero_empty_sequences<T>(a, lens, ctid, kCW * 32);
  const int hg = warp % HG, tw = warp / HG;
  const int g = lane >> 2, t4 = lane & 3;
  const int mi = lane >> 3, r8 = lane & 7;
  // ldmatrix row addresses: K (A operand of S = K.Q^T) and V (A operand of O^T = V^T.P^T, transposed).
  const uint32_t k_row = (r8 + 8 * (mi & 1)) * 128u;
  const int k_half = mi >> 1;
  const uint32_t v_row = (r8 + 8 * (mi >> 1)) * 128u;
  const int v_half = mi & 1;
  const float sl = a.scale_log2;
  const auto csync = [] { named_barrier(1, kCW * 32); };

  Walk w;
  walk_init(a, misc, w);
  Seg s;
  uint32_t gt = 0;
  while (walk_next(a, lens, prefix, w, s)) {
    const int ntok = max(0, s.tok_end - s.tok_begin);
    const int ntiles = (ntok + kTile - 1) / kTile;

    // Q^T as the B operand: lane holds q[head g][2t4, 2t4+1] and [2t4+8, 2t4+9] of each k-step.
    uint32_t qf[KS][NT][2];
    const T* qb = static_cast<const T*>(a.q) + (static_cast<int64_t>(s.b) * a.num_q_heads + s.kvh * a.group) * D;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int h = hg * HPW + nt * 8 + g;
      const bool hv = h < a.group;
      const uint32_t* qrow = reinterpret_cast<const uint32_t*>(qb + static_cast<int64_t>(hv ? h : 0) * D);
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        qf[ks][nt][0] = hv ? __ldg(qrow + ks * 8 + t4) : 0u;
        qf[ks][nt][1] = hv ? __ldg(qrow + ks * 8 + 4 + t4) : 0u;
      }
    }

    float m_run[NT][2], l_run[NT][2], acc[KS][NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      m_run[nt][0] = m_run[nt][1] = -INFINITY;
      l_run[nt][0] = l_run[nt][1] = 0.0f;
#pragma unroll
      for (int mt = 0; mt < KS; ++mt) acc[mt][nt][0] = acc[mt][nt][1] = acc[mt][nt][2] = acc[mt][nt][3] = 0.0f;
    }

    for (int j = tw; j < ntiles; j += TW) {
      const uint32_t gj = gt + j;
      const int stage = static_cast<int>(gj % nstage);
      if (*abort_flag) break;
      if (!mbar_wait_bounded(bars + 8u * stage, (gj / nstage) & 1u, a.sync, kWaitLimitNs)) {
        *abort_flag = 1;
        break;
      }
      const int valid = min(kTile, ntok - j * kTile);
      const uint32_t sk = ring + stage * L.stage_bytes;
      const uint32_t sv = sk + kHalf;

      // S = K . Q^T : [16 tokens x 8 heads] per n-tile.
      float sc[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.0f;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(sk + (ks >> 2) * kChunkBytes + k_row + (((((2 * ks) & 7) + k_half) ^ r8) << 4), a0, a1, a2, a3);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) Mma<T>::run(sc[nt], a0, a1, a2, a3, qf[ks][nt][0], qf[ks][nt][1]);
      }

      // Online softmax in base 2. Lane holds tokens g and g+8 of heads 2*t4 and 2*t4+1.
      const bool row0 = g < valid, row1 = g + 8 < valid;
      uint32_t pb[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[nt][e] *= sl;
        if (!row0) sc[nt][0] = sc[nt][1] = -INFINITY;
        if (!row1) sc[nt][2] = sc[nt][3] = -INFINITY;
        float alpha[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float mx = fmaxf(sc[nt][e], sc[nt][2 + e]);
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
          const float mn = fmaxf(m_run[nt][e], mx);
          alpha[e] = fast_exp2(m_run[nt][e] - mn);
          m_run[nt][e] = mn;
        }
        const uint32_t p01 =
            Storage<T>::pack2(fast_exp2(sc[nt][0] - m_run[nt][0]), fast_exp2(sc[nt][1] - m_run[nt][1]));
        const uint32_t p23 =
            Storage<T>::pack2(fast_exp2(sc[nt][2] - m_run[nt][0]), fast_exp2(sc[nt][3] - m_run[nt][1]));
        // The normaliser sums the rounded probabilities the MMA actually uses.
        const float2 f01 = Storage<T>::unpack2(p01), f23 = Storage<T>::unpack2(p23);
        l_run[nt][0] = l_run[nt][0] * alpha[0] + (f01.x + f23.x);
        l_run[nt][1] = l_run[nt][1] * alpha[1] + (f01.y + f23.y);
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
          acc[mt][nt][0] *= alpha[0];
          acc[mt][nt][1] *= alpha[1];
          acc[mt][nt][2] *= alpha[0];
          acc[mt][nt][3] *= alpha[1];
        }
        // P (tokens x heads, C layout) -> P^T as the B operand of the PV product.
        pb[nt][0] = movmatrix_trans(p01);
        pb[nt][1] = movmatrix_trans(p23);
      }

      // O^T += V^T . P^T ; rows of V past the valid tokens are zeroed, never multiplied.
      uint32_t m01 = 0xffffffffu, m23 = 0xffffffffu;
      if (valid < kTile) {
        m01 = (2 * t4 < valid ? 0x0000ffffu : 0u) | (2 * t4 + 1 < valid ? 0xffff0000u : 0u);
        m23 = (2 * t4 + 8 < valid ? 0x0000ffffu : 0u) | (2 * t4 + 9 < valid ? 0xffff0000u : 0u);
      }
#pragma unroll
      for (int mt = 0; mt < KS; ++mt) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4_trans(sv + (mt >> 2) * kChunkBytes + v_row + (((((2 * mt) & 7) + v_half) ^ r8) << 4), a0, a1, a2,
                      a3);
        a0 &= m01;
        a1 &= m01;
        a2 &= m23;
        a3 &= m23;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) Mma<T>::run(acc[mt][nt], a0, a1, a2, a3, pb[nt][0], pb[nt][1]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bars + 8u * (nstage + stage));
    }
    gt += ntiles;

    // Publish this warp's (m, l, acc) and combine the tile-parallel warps of each head group.
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float l = l_run[nt][e];
        l += __shfl_xor_sync(0xffffffffu, l, 4);
        l += __shfl_xor_sync(0xffffffffu, l, 8);
        l += __shfl_xor_sync(0xffffffffu, l, 16);
        l_run[nt][e] = l;
      }
    }
    float* rm = red_m + warp * HPW;
    float* rl = red_l + warp * HPW;
    float* ra = red_acc + warp * HPW * (D + 4);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int hl = nt * 8 + 2 * t4 + e;
        if (g == 0) {
          rm[hl] = m_run[nt][e];
          rl[hl] = l_run[nt][e];
        }
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
          ra[hl * (D + 4) + mt * 16 + g] = acc[mt][nt][e];
          ra[hl * (D + 4) + mt * 16 + g + 8] = acc[mt][nt][2 + e];
        }
      }
    }
    csync();
    for (int idx = ctid; idx < a.group * D; idx += kCW * 32) {
      const int h = idx / D, d = idx - h * D;
      const int hgi = h / HPW, hl = h - hgi * HPW;
      float M = -INFINITY;
      for (int tw2 = 0; tw2 < TW; ++tw2) M = fmaxf(M, red_m[(tw2 * HG + hgi) * HPW + hl]);
      float O = 0.0f, Ls = 0.0f;
      if (M > -INFINITY) {
        for (int tw2 = 0; tw2 < TW; ++tw2) {
          const int wi = tw2 * HG + hgi;
          const float mw = red_m[wi * HPW + hl];
          if (mw > -INFINITY) {
            const float f = fast_exp2(mw - M);
            Ls += red_l[wi * HPW + hl] * f;
            O += red_acc[(wi * HPW + hl) * (D + 4) + d] * f;
          }
        }
      }
      emit_value<T>(a, s, h, d, O, Ls, M);
    }
    merge_if_last<T>(a, s, ctid, kCW * 32, misc + 3, csync);
    csync();
  }
}

// ------------------------------------------------------------------------- generic kernel

struct GenLayout {
  uint32_t q, acc, p, m, l, alpha, rows, misc, prefix, lens, total;
};

__host__ __device__ inline GenLayout gen_layout(int G, int D, int batch) {
  GenLayout L{};
  uint32_t off = 0;
  L.q = off;
  off += G * D * 4u;
  L.acc = off;
  off += G * D * 4u;
  L.p = off;
  off += kGenChunk * G * 4u;
  L.m = off;
  off += G * 4u;
  L.l = off;
  off += G * 4u;
  L.alpha = off;
  off += G * 4u;
  off = align_up(off, 8);
  L.rows = off;
  off += kGenChunk * 8u;
  L.misc = off;
  off += 64u * 4u;
  L.prefix = off;
  off += (batch + 1u) * 4u;
  L.lens = off;
  off += batch * 4u;
  L.total = align_up(off, 16);
  return L;
}

template <typename T>
__global__ void __launch_bounds__(kGenThreads) decode_generic_kernel(const DecodeArgs a) {
  extern __shared__ __align__(16) uint8_t gsmem[];
  const int G = a.group, D = a.head_dim, H = a.num_kv_heads;
  const GenLayout L = gen_layout(G, D, a.batch);
  float* q_s = reinterpret_cast<float*>(gsmem + L.q);
  float* acc_s = reinterpret_cast<float*>(gsmem + L.acc);
  float* p_s = reinterpret_cast<float*>(gsmem + L.p);
  float* m_s = reinterpret_cast<float*>(gsmem + L.m);
  float* l_s = reinterpret_cast<float*>(gsmem + L.l);
  float* al_s = reinterpret_cast<float*>(gsmem + L.alpha);
  int64_t* row_s = reinterpret_cast<int64_t*>(gsmem + L.rows);
  int* misc = reinterpret_cast<int*>(gsmem + L.misc);
  int* prefix = reinterpret_cast<int*>(gsmem + L.prefix);
  int* lens = reinterpret_cast<int*>(gsmem + L.lens);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  plan_build(a, lens, prefix, misc);
  zero_empty_sequences<T>(a, lens, tid, kGenThreads);
  const auto bsync = [] { __syncthreads(); };
  const int64_t tok_stride = static_cast<int64_t>(H) * D;

  Walk w;
  walk_init(a, misc, w);
  Seg s;
  while (walk_next(a, lens, prefix, w, s)) {
    const T* qb = static_cast<const T*>(a.q) + (static_cast<int64_t>(s.b) * a.num_q_heads + s.kvh * G) * D;
    for (int i = tid; i < G * D; i += kGenThreads) {
      q_s[i] = Storage<T>::load(qb[i]);
      acc_s[i] = 0.0f;
    }
    if (tid < G) {
      m_s[tid] = -INFINITY;
      l_s[tid] = 0.0f;
    }
    const T* kc = static_cast<const T*>(a.k_cache) + s.kvh * D;
    const T* vc = static_cast<const T*>(a.v_cache) + s.kvh * D;
    const int32_t* bt_row = a.block_table + static_cast<int64_t>(s.b) * a.bt_stride;
    __syncthreads();
    for (int base = s.tok_begin; base < s.tok_end; base += kGenChunk) {
      const int n = min(kGenChunk, s.tok_end - base);
      if (tid < n) {
        const int tok = base + tid;
        const int pidx = tok / a.page_size;
        const int page = bt_row[pidx];
        int64_t row = -1;
        if (page < 0 || (a.num_pages >= 0 && page >= a.num_pages)) {
          atomicOr(a.sync, kStatusBadPage);
        } else {
          row = (static_cast<int64_t>(page) * a.page_size + (tok - pidx * a.page_size)) * tok_stride;
        }
        row_s[tid] = row;
      }
      __syncthreads();
      for (int j = warp; j < n; j += kGenThreads / 32) {
        const int64_t row = row_s[j];
        for (int gi = 0; gi < G; ++gi) {
          float part = 0.0f;
          if (row >= 0) {
            for (int d = lane; d < D; d += 32) part = fmaf(q_s[gi * D + d], Storage<T>::load(kc[row + d]), part);
          }
          part = warp_allreduce_sum(part);
          if (lane == 0) p_s[j * G + gi] = row >= 0 ? part * a.scale_log2 : -INFINITY;
        }
      }
      __syncthreads();
      if (tid < G) {
        float mx = -INFINITY;
        for (int j = 0; j < n; ++j) mx = fmaxf(mx, p_s[j * G + tid]);
        const float mo = m_s[tid];
        const float mn = fmaxf(mo, mx);
        float sum = 0.0f;
        float alpha = 1.0f;
        if (mn > -INFINITY) {
          alpha = fast_exp2(mo - mn);
          for (int j = 0; j < n; ++j) {
            const float e = fast_exp2(p_s[j * G + tid] - mn);
            p_s[j * G + tid] = e;
            sum += e;
          }
        } else {
          for (int j = 0; j < n; ++j) p_s[j * G + tid] = 0.0f;
        }
        l_s[tid] = l_s[tid] * alpha + sum;
        m_s[tid] = mn;
        al_s[tid] = alpha;
      }
      __syncthreads();
      for (int idx = tid; idx < G * D; idx += kGenThreads) {
        const int gi = idx / D, d = idx - gi * D;
        float v = acc_s[idx] * al_s[gi];
        for (int j = 0; j < n; ++j) {
          const int64_t row = row_s[j];
          if (row >= 0) v = fmaf(p_s[j * G + gi], Storage<T>::load(vc[row + d]), v);
        }
        acc_s[idx] = v;
      }
      __syncthreads();
    }
    for (int idx = tid; idx < G * D; idx += kGenThreads) {
      const int h = idx / D, d = idx - h * D;
      emit_value<T>(a, s, h, d, acc_s[idx], l_s[h], m_s[h]);
    }
    merge_if_last<T>(a, s, tid, kGenThreads, misc + 3, bsync);
    __syncthreads();
  }
}

// ------------------------------------------------------------------------- host side

namespace {

struct Plan {
  bool tc = false;
  int D = 0, NT = 1, HG = 1, nstage = 0, p_rows = 16;
  size_t smem = 0;
  int grid = 0;
  int splits = 0, pps = 0;
  int slots = 0;
  size_t part_bytes = 0, sync_bytes = 0;
  const void* fn = nullptr;
};

std::mutex g_mu;

int device_sms(int dev) {
  static int cache[64] = {0};
  if (dev < 0 || dev >= 64) return 0;
  std::lock_guard<std::mutex> lock(g_mu);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    cache[dev] = n;
  }
  return cache[dev];
}

// Blocks per SM for `fn` at `smem` dynamic bytes; also raises the kernel's
// dynamic shared-memory limit on first use on this device.
int blocks_per_sm(int dev, const void* fn, int threads, size_t smem) {
  static std::map<std::tuple<int, const void*, size_t>, int> occ;
  static std::map<std::pair<int, const void*>, bool> attr;
  std::lock_guard<std::mutex> lock(g_mu);
  auto key = std::make_tuple(dev, fn, smem);
  auto it = occ.find(key);
  if (it != occ.end()) return it->second;
  if (!attr[{dev, fn}]) {
    int max_optin = 0;
    cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, max_optin) != cudaSuccess) return 0;
    attr[{dev, fn}] = true;
  }
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, threads, smem) != cudaSuccess) n = 0;
  occ[key] = n;
  return n;
}

template <typename T>
const void* tc_fn(int D, int NT) {
  if (D == 64) return NT == 1 ? (const void*)decode_tc_kernel<T, 64, 1> : (const void*)decode_tc_kernel<T, 64, 2>;
  if (D == 128) return NT == 1 ? (const void*)decode_tc_kernel<T, 128, 1> : (const void*)decode_tc_kernel<T, 128, 2>;
  return (const void*)decode_tc_kernel<T, 256, 1>;
}

const void* gen_fn(int dtype) {
  switch (dtype) {
    case KL_FLOAT32: return (const void*)decode_generic_kernel<float>;
    case KL_FLOAT16: return (const void*)decode_generic_kernel<__half>;
    default: return (const void*)decode_generic_kernel<__nv_bfloat16>;
  }
}

constexpr int kMinTilesPerCta = 4;
constexpr uint32_t kSmemTarget = 112 * 1024;  // two CTAs per SM

// Partial outputs [slots][G][D] fp32 first, then their LSEs [slots][G], 256-byte aligned.
size_t lse_offset(int slots, int G, int D) {
  return (static_cast<size_t>(slots) * G * D * 4 + 255) / 256 * 256;
}

// Launch shape and scratch sizes of one decode call. `generic` forces the CUDA-core kernel.
int make_plan(int dtype, int batch, int Hq, int Hkv, int D, int P, int max_pages, int num_splits, bool generic,
              Plan& p) {
  if (batch <= 0 || batch > kMaxBatch || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0 || D <= 0 || P <= 0 ||
      max_pages < 0 || num_splits < 0) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  if (dtype != KL_FLOAT32 && dtype != KL_FLOAT16 && dtype != KL_BFLOAT16) return static_cast<int>(cudaErrorInvalidValue);
  const int G = Hq / Hkv;
  const int64_t max_tokens = static_cast<int64_t>(max_pages) * P;
  if (max_tokens > INT_MAX / 2) return static_cast<int>(cudaErrorInvalidValue);
  const int64_t total_tiles = static_cast<int64_t>(batch) * ((max_tokens + kTile - 1) / kTile) * Hkv;
  if (total_tiles > INT_MAX / 2) return static_cast<int>(cudaErrorInvalidValue);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return static_cast<int>(cudaErrorNoDevice);
  const int sms = device_sms(dev);
  if (sms <= 0) return static_cast<int>(cudaErrorNoDevice);

  p.D = D;
  p.tc = !generic && dtype != KL_FLOAT32 && (D == 64 || D == 128 || D == 256) && (P == 8 || P % 16 == 0) &&
         (D == 256 ? G <= 32 : G <= 64);
  int threads;
  if (p.tc) {
    p.NT = (G > 8 && D <= 128) ? 2 : 1;
    const int need = (G + 8 * p.NT - 1) / (8 * p.NT);
    p.HG = need <= 1 ? 1 : need <= 2 ? 2 : 4;
    p.p_rows = P < 16 ? P : 16;
    const TcLayout base = tc_layout(D, p.NT, 0, batch);
    const uint32_t stage = 2u * kTile * D * 2u + 16u;
    int ns = base.total < kSmemTarget ? static_cast<int>((kSmemTarget - base.total) / stage) : 0;
    ns = std::min(16, ns);
    if (ns < 4) ns = 4;  // one CTA per SM then
    p.nstage = ns;
    p.smem = tc_layout(D, p.NT, ns, batch).total;
    p.fn = dtype == KL_FLOAT16 ? tc_fn<__half>(D, p.NT) : tc_fn<__nv_bfloat16>(D, p.NT);
    threads = kTCThreads;
  } else {
    if (static_cast<int64_t>(G) * D > 8192) return static_cast<int>(cudaErrorInvalidValue);
    p.smem = gen_layout(G, D, batch).total;
    p.fn = gen_fn(dtype);
    threads = kGenThreads;
  }
  int max_optin = 0;
  cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (p.smem > static_cast<size_t>(max_optin)) return static_cast<int>(cudaErrorInvalidValue);
  const int per_sm = blocks_per_sm(dev, p.fn, threads, p.smem);
  if (per_sm <= 0) return static_cast<int>(cudaErrorInvalidConfiguration);

  if (num_splits > 0) {
    const int mp = std::max(1, max_pages);
    p.pps = (mp + num_splits - 1) / num_splits;
    p.splits = (mp + p.pps - 1) / p.pps;
    const int64_t items = static_cast<int64_t>(batch) * Hkv * p.splits;
    if (items > INT_MAX / 2) return static_cast<int>(cudaErrorInvalidValue);
    p.slots = static_cast<int>(items);
    p.grid = static_cast<int>(std::min<int64_t>(items, static_cast<int64_t>(sms) * per_sm));
  } else {
    p.splits = 0;
    p.grid = sms * per_sm;
    p.slots = 2 * p.grid;
  }
  p.part_bytes = lse_offset(p.slots, G, D) + static_cast<size_t>(p.slots) * G * 4;
  p.sync_bytes = (1 + static_cast<size_t>(batch) * Hkv) * 4;
  return 0;
}

std::once_flag g_encode_once;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  });
  return g_encode;
}

// 2-D view of one cache: rows = every token slot of the pool, columns = Hkv*D elements.
// Box = 64 columns (128 bytes) x p_rows rows, 128-byte swizzle.
bool encode_kv_map(CUtensorMap* map, const void* base, int dtype, int64_t pool_tokens, int Hkv, int D, int p_rows) {
  auto enc = encoder();
  if (!enc) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(Hkv) * D, static_cast<cuuint64_t>(pool_tokens)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(Hkv) * D * 2};
  const cuuint32_t box[2] = {64u, static_cast<cuuint32_t>(p_rows)};
  const cuuint32_t estr[2] = {1u, 1u};
  const CUtensorMapDataType dt =
      dtype == KL_FLOAT16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

template <typename T>
cudaError_t launch_tc(const Plan& p, const CUtensorMap& tmk, const CUtensorMap& tmv, const DecodeArgs& a,
                      cudaStream_t st) {
  const int hg = p.HG;
  switch (p.D) {
    case 64:
      if (p.NT == 1) decode_tc_kernel<T, 64, 1><<<p.grid, kTCThreads, p.smem, st>>>(tmk, tmv, a, p.nstage, p.p_rows, hg);
      else decode_tc_kernel<T, 64, 2><<<p.grid, kTCThreads, p.smem, st>>>(tmk, tmv, a, p.nstage, p.p_rows, hg);
      break;
    case 128:
      if (p.NT == 1) decode_tc_kernel<T, 128, 1><<<p.grid, kTCThreads, p.smem, st>>>(tmk, tmv, a, p.nstage, p.p_rows, hg);
      else decode_tc_kernel<T, 128, 2><<<p.grid, kTCThreads, p.smem, st>>>(tmk, tmv, a, p.nstage, p.p_rows, hg);
      break;
    default:
      decode_tc_kernel<T, 256, 1><<<p.grid, kTCThreads, p.smem, st>>>(tmk, tmv, a, p.nstage, p.p_rows, hg);
      break;
  }
  return cudaGetLastError();
}

int decode_impl(int dtype, void* out, const void* q, const void* k_cache, const void* v_cache,
                const int32_t* block_table, const int32_t* seq_lens, int batch, int Hq, int Hkv, int D, int P,
                int64_t bt_stride, int max_pages, int64_t num_pages, float scale, int num_splits, void* partials,
                size_t partial_bytes, void* sync, size_t sync_bytes, cudaStream_t st) {
  if (batch == 0) return 0;
  if (!out || !q || !k_cache || !v_cache || !block_table || !seq_lens || !sync) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  if (bt_stride < 0 || (batch > 1 && bt_stride < max_pages)) return static_cast<int>(cudaErrorInvalidValue);
  Plan p;
  if (const int rc = make_plan(dtype, batch, Hq, Hkv, D, P, max_pages, num_splits, false, p)) return rc;
  // The tensor-core path needs 16-byte aligned caches (TMA), 4-byte aligned q and
  // TMA row coordinates that fit in int32; otherwise take the generic kernel.
  const bool tc_ok = p.tc && aligned(k_cache, 16) && aligned(v_cache, 16) && aligned(q, 4) &&
                     (num_pages < 0 || num_pages * P <= INT_MAX);
  CUtensorMap tmk, tmv;
  bool use_tc = false;
  if (tc_ok) {
    const int64_t pool_tokens = num_pages >= 0 ? std::max<int64_t>(num_pages, 1) * P : (int64_t(1) << 31) - 1;
    use_tc = encode_kv_map(&tmk, k_cache, dtype, pool_tokens, Hkv, D, p.p_rows) &&
             encode_kv_map(&tmv, v_cache, dtype, pool_tokens, Hkv, D, p.p_rows);
  }
  if (!use_tc && p.tc) {
    if (const int rc = make_plan(dtype, batch, Hq, Hkv, D, P, max_pages, num_splits, true, p)) return rc;
  }
  if (partial_bytes < p.part_bytes || sync_bytes < p.sync_bytes || !partials) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  const int G = Hq / Hkv;
  DecodeArgs a{};
  a.out = out;
  a.q = q;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.block_table = block_table;
  a.seq_lens = seq_lens;
  a.batch = batch;
  a.num_q_heads = Hq;
  a.num_kv_heads = Hkv;
  a.group = G;
  a.head_dim = D;
  a.page_size = P;
  a.bt_stride = bt_stride;
  a.max_pages = max_pages;
  a.num_pages = num_pages;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.splits = p.splits;
  a.pages_per_split = p.pps;
  a.min_tiles = kMinTilesPerCta;
  a.sync = static_cast<uint32_t*>(sync);
  a.part_o = static_cast<float*>(partials);
  a.part_lse = reinterpret_cast<float*>(static_cast<uint8_t*>(partials) + lse_offset(p.slots, G, D));

  if (use_tc) {
    const cudaError_t e = dtype == KL_FLOAT16 ? launch_tc<__half>(p, tmk, tmv, a, st)
                                              : launch_tc<__nv_bfloat16>(p, tmk, tmv, a, st);
    return static_cast<int>(e);
  }
  switch (dtype) {
    case KL_FLOAT32: decode_generic_kernel<float><<<p.grid, kGenThreads, p.smem, st>>>(a); break;
    case KL_FLOAT16: decode_generic_kernel<__half><<<p.grid, kGenThreads, p.smem, st>>>(a); break;
    default: decode_generic_kernel<__nv_bfloat16><<<p.grid, kGenThreads, p.smem, st>>>(a); break;
  }
  return static_cast<int>(cudaGetLastError());
}

}  // namespace
}  // namespace klb

extern "C" {

const char* kl_version(void) { return "kernel_lab_b200 0.1.0 sm_100a"; }

const char* kl_status_string(int status) {
  return status == 0 ? "success" : cudaGetErrorString(static_cast<cudaError_t>(status));
}

int kl_paged_decode_workspace_size(int dtype, int batch, int num_q_heads, int num_kv_heads, int head_dim,
                                   int page_size, int max_pages_per_seq, int num_splits, size_t* partial_bytes,
                                   size_t* sync_bytes) {
  if (!partial_bytes || !sync_bytes) return static_cast<int>(cudaErrorInvalidValue);
  *partial_bytes = 0;
  *sync_bytes = 4;
  if (batch == 0) return 0;
  klb::Plan p;
  if (const int rc = klb::make_plan(dtype, batch, num_q_heads, num_kv_heads, head_dim, page_size,
                                    max_pages_per_seq, num_splits, false, p)) {
    return rc;
  }
  // A misaligned call falls back to the generic kernel, whose grid may differ: size for both.
  klb::Plan g;
  if (p.tc && klb::make_plan(dtype, batch, num_q_heads, num_kv_heads, head_dim, page_size, max_pages_per_seq,
                             num_splits, true, g) == 0) {
    p.part_bytes = std::max(p.part_bytes, g.part_bytes);
  }
  *partial_bytes = p.part_bytes;
  *sync_bytes = p.sync_bytes;
  return 0;
}

int kl_paged_decode(int dtype, void* out, const void* q, const void* k_cache, const void* v_cache,
                    const int32_t* block_table, const int32_t* seq_lens, int batch, int num_q_heads,
                    int num_kv_heads, int head_dim, int page_size, int64_t block_table_stride, int max_pages_per_seq,
                    int64_t num_pages, float scale, int num_splits, void* partials, size_t partial_bytes, void* sync,
                    size_t sync_bytes, void* stream) {
  return klb::decode_impl(dtype, out, q, k_cache, v_cache, block_table, seq_lens, batch, num_q_heads, num_kv_heads,
                          head_dim, page_size, block_table_stride, max_pages_per_seq, num_pages, scale, num_splits,
                          partials, partial_bytes, sync, sync_bytes, static_cast<cudaStream_t>(stream));
}

int kl_paged_decode_attention(int dtype, void* out, const void* q, const void* k_cache, const void* v_cache,
                              const int32_t* block_table, const int32_t* seq_lens, int batch, int num_q_heads,
                              int num_kv_heads, int head_dim, int page_size, int64_t block_table_stride, float scale,
                              void* stream) {
  if (batch == 0) return 0;
  if (block_table_stride <= 0 || block_table_stride > INT_MAX) return static_cast<int>(cudaErrorInvalidValue);
  const int max_pages = static_cast<int>(block_table_stride);
  size_t pb = 0, sb = 0;
  if (const int rc = kl_paged_decode_workspace_size(dtype, batch, num_q_heads, num_kv_heads, head_dim, page_size,
                                                    max_pages, 0, &pb, &sb)) {
    return rc;
  }
  auto st = static_cast<cudaStream_t>(stream);
  void* buf = nullptr;
  const size_t sync_off = (pb + 255) / 256 * 256;
  cudaError_t e = cudaMallocAsync(&buf, sync_off + sb, st);
  if (e != cudaSuccess) return static_cast<int>(e);
  e = cudaMemsetAsync(static_cast<uint8_t*>(buf) + sync_off, 0, sb, st);
  int rc = static_cast<int>(e);
  if (rc == 0) {
    rc = kl_paged_decode(dtype, out, q, k_cache, v_cache, block_table, seq_lens, batch, num_q_heads, num_kv_heads,
                         head_dim, page_size, block_table_stride, max_pages, -1, scale, 0, buf, pb,
                         static_cast<uint8_t*>(buf) + sync_off, sb, stream);
  }
  const cudaError_t f = cudaFreeAsync(buf, st);
  return rc != 0 ? rc : static_cast<int>(f);
}

int kl_paged_decode_read_status(void* sync, uint32_t* status, int clear, void* stream) {
  if (!sync || !status) return static_cast<int>(cudaErrorInvalidValue);
  auto st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(status, sync, sizeof(uint32_t), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess && clear) {
    e = cudaMemsetAsync(sync, 0, sizeof(uint32_t), st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  }
  return static_cast<int>(e);
}

}  // extern "C"
