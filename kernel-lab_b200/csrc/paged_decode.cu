// Paged-KV single-token decode attention for sm_100a: split-KV with an exact
// log-sum-exp merge, GQA head packing, TMA page staging and a load-balanced planner.
//
// What it replaces: kernel-lab's warp-per-token CUDA kernel (csrc/paged_attention.cu:27-128),
// with the split/merge semantics of its Triton kernel
// (kernel_lab/triton_kernels/paged_attention.py:37-173): partial outputs are normalised,
// carry a base-2 LSE, and an empty split has lse = -inf and zero weight.
//
// Work decomposition. A "tile" is 16 tokens of one sequence for one "unit" of heads: a
// block of HT consecutive KV heads in the tensor-core kernel, one KV head in the generic
// one. Every CTA computes the same plan from seq_lens (no host sync): the (sequence, unit)
// items are laid end to end, each costing its tiles plus a fixed per-item charge (the time
// a CTA spends starting an item), and CTA c takes the cost range [c*R, (c+1)*R),
// R = max(min_tiles, ceil(total / grid)), so every CTA streams about the same number of KV
// bytes whatever the length distribution (ragged batches included). An item that a range
// boundary cuts is split into "chunks". A chunk reads its item's arrival counter when it
// starts; if every sibling has already published, it merges their partials with its own
// registers at the end; otherwise it writes a normalised fp32 partial and base-2 LSE,
// bumps the counter, and the chunk that completes the count merges. The merge always
// runs in chunk order, so the result does not depend on arrival order, and it resets the
// counter to zero; nobody waits on another CTA. A forced split count (num_splits > 0)
// instead gives every sequence exactly ceil(max_pages / pages_per_split) chunks,
// including empty ones, like the Triton kernel.
//
// Tensor-core kernel (fp16/bf16, head_dim 64/128/256, page size 8 or a multiple of 16).
// A stage holds the K and V rows of one tile for HT KV heads: with Llama-3-8B's 8 KV
// heads that is one whole 16-token page, 32 KB of K and 32 KB of V read contiguously,
// instead of 256-byte per-head rows scattered over the page. One producer warp walks the
// plan and issues one 3-D TMA box per tensor per tile (128-byte swizzle, L2 evict-first)
// into a ring of shared-memory stages guarded by mbarriers. Eight consumer warps: warp
// (ht, hg, tw) owns KV head ht of the stage and query-head group hg (8*NT query heads of
// that KV head's GQA group); when a unit has fewer heads than warps, TW warps split the
// tiles and combine through shared memory. A consumer computes S = K.Q^T with
// mma.m16n8k16 (M = 16 tokens, N = 8 query heads, K = head_dim), the online softmax in
// base 2 on the fp32 fragments, turns P into the B operand with movmatrix, and
// accumulates O^T += V^T.P^T. K and V fragments come from plain 16-byte shared loads in a
// permuted contraction / output-row order, so no ldmatrix is needed.
//
// Generic kernel (fp32, other head_dims / page sizes / groups): same plan, CUDA cores,
// 32-token chunks staged through shared memory; every chunk publishes its partial and the
// one that completes the count merges them all from scratch, in chunk order.
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
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <type_traits>

#include "common.cuh"
#include "kernel_lab_b200.h"

namespace klb {

constexpr int kTile = 16;
constexpr uint32_t kBatchStageBytes = 32 * 1024;  // producer issues tiles in batches up to this stage size
constexpr int kRegisterMergeChunks = 4;  // splits of at most this many chunks merge from registers         // tokens per tile: the MMA's M
constexpr int kCW = 8;            // consumer warps of the tensor-core kernel
constexpr int kTCThreads = 32 * (kCW + 1);
constexpr int kGenThreads = 128;
constexpr int kGenChunk = 32;     // tokens per step of the generic kernel
constexpr int kMaxBatch = 16384;  // the plan lives in shared memory
constexpr int kMaxHeadGroups = 4; // query-head groups per KV head (counter stride)
constexpr uint64_t kWaitLimit = 2000000000ull;  // SM cycles: about one second at 1.9 GHz
constexpr int kMaxRanks = KL_GATHER_MAX_RANKS;   // GPUs of one head gather
constexpr uint64_t kPeerWaitNs = 10000000000ull; // default wait (10 s) of a rank for its peers' arrivals

// Head gather over NVLink (ranks > 1): every final output row is stored to this rank's output
// and, with plain peer stores, to the same place in every other rank's (out[r]: rank r's output
// as mapped in this process, at this rank's head offset). The launch then ends with one
// cross-GPU arrival: the last CTA to finish on this GPU publishes `epoch` in every rank's flags
// and waits (bounded) until every rank has published it in this rank's flags.
struct Gather {
  int ranks;  // 0 or 1: no gather
  int rank;
  uint32_t epoch;
  void* out[kMaxRanks];
  uint32_t* flags[kMaxRanks];  // rank r's arrival flags [ranks]
  uint32_t* done;              // this rank's count of finished CTAs (zero at rest)
  uint64_t wait_ns;            // how long the last CTA waits for the peers' arrivals
};

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
  int64_t num_pages;    // < 0: unknown, page ids not range-checked
  float scale_log2;
  int units;            // work units per sequence (head blocks or KV heads)
  int splits;           // 0: balanced plan; > 0: forced splits per sequence
  int pages_per_split;  // forced mode
  int min_tiles;        // balanced mode: minimum tiles per CTA
  int seg_cost;         // balanced mode: tiles' worth of time charged for starting a (sequence, unit)
  uint32_t* sync;       // [0] status, [1 + (b*Hkv + kvh)*kMaxHeadGroups + hg] arrival counters
  float* part_o;        // [slot][slot_heads][head_dim]
  float* part_lse;      // [slot][slot_heads]
  const float* k_scale;  // e4m3 cache: per-KV-head dequantisation scales (null otherwise)
  const float* v_scale;
  // Cascade (shared-prefix) decode; off when num_prefixes == 0. The sequences of group p,
  // [prefix_indptr[p], prefix_indptr[p+1]), share prefix_lens[p] tokens held in the pages of row p
  // of prefix_bt; each sequence attends to them and to its own tokens (block_table, seq_lens).
  const int32_t* prefix_bt;
  const int32_t* prefix_lens;
  const int32_t* prefix_indptr;
  int num_prefixes;
  int64_t prefix_bt_stride;
  int prefix_max_pages;
  int members;    // sequences whose query rows one prefix item packs (a "member block")
  // Prefix chunks of prefix_chunk tokens computed by the tensor-core prefix kernel (0: the
  // prefix items are entries of this kernel's plan, one chunk each). A sequence's state is merged
  // from nch = ceil(prefix length / prefix_chunk) prefix planes (plane c: chunk c) and its own
  // plane (cas_planes), by whichever of the nch + 1 arrivals comes last.
  int prefix_chunk;
  int cas_planes;
  int cas_hpw;    // query rows per counter group (the decode kernel's heads per warp)
  float* cas_o;   // [cas_planes + 1][batch * num_q_heads][head_dim]: normalised partial outputs
  float* cas_lse; // [cas_planes + 1][batch * num_q_heads]: their base-2 LSEs
  // Output placement: sequence b's query head h at out + b * out_seq_stride + h * head_dim
  // (out_seq_stride = num_q_heads * head_dim unless out is this rank's head slice of a wider
  // output), and the head gather (tensor-core kernel, plain decode only).
  int64_t out_seq_stride;
  Gather gat;
};

struct TcShape {
  int nstage;  // ring stages
  int p_rows;  // rows of one TMA box: min(page_size, 16)
  int ht;      // KV heads per tile
  int hg;      // query-head groups (of 8*NT heads) per KV head
  int tw;      // warps splitting the tiles of one (head, group)
  int ns;      // streams: TW when each warp walks its own range (one (head, group) a tile), else 1
};

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ------------------------------------------------------------------------- plan

// Plan entries: without a cascade, entry b is sequence b. With one, entries [0, V) are prefix
// items (member blocks: up to `members` consecutive sequences of one group, whose query rows
// share each MMA) and entry V + b is sequence b's own tokens.
struct Seg {
  int b, u;                // plan entry, unit
  int tok_begin, tok_end;  // token range; empty when tok_end <= tok_begin
  int chunk;               // chunk id of this piece (partial slots derive from it)
  int nchunks;             // chunks of this (entry, unit)
  int c_first;             // balanced mode: CTA holding the first chunk
  bool first_aligned;      // balanced mode: the first chunk starts its CTA's range
  bool whole;
  int seq;                 // first sequence whose query rows the entry serves
  int nmem;                // sequences it serves (1 unless a prefix item)
  int grp;                 // prefix group of a prefix item, -1 for a sequence's own tokens
  int cb;                  // arrival-counter block: seq for own tokens, batch + entry for prefix items
};

struct Walk {
  int t, t1, R;     // balanced
  bool first;       // balanced: no segment produced yet
  int item, items;  // forced
  int n, V;         // plan entries, prefix items among them
  int vidx, vgrid;  // the walker's range: range vidx of vgrid (a CTA, or one stream of a CTA)
};

// Shared-memory plan arrays. lens/prefix have one slot per entry (+1 for prefix); hp and vstart
// exist only for a cascade: hp[b] = clamped prefix length of sequence b's group, vstart[p] = first
// entry of group p (vstart[num_prefixes] = V).
struct PlanSmem {
  int* lens;
  int* prefix;
  int* misc;
  int* hp;
  int* vstart;
};

// misc[]: 0 total cost, 1 R, 2 abort flag, 3 spare, 8..40 scan scratch, 48 V, 49 entries.
constexpr int kMiscScan = 8, kMiscV = 48, kMiscEntries = 49;

__device__ __forceinline__ int clamp_len(const DecodeArgs& a, int b, bool report) {
  int len = a.seq_lens[b];
  const int cap = a.max_pages * a.page_size;
  if (len > cap) {
    if (report) atomicOr(a.sync, kStatusLenClamped);
    len = cap;
  }
  return len < 0 ? 0 : len;
}

__device__ __forceinline__ int clamp_prefix_len(const DecodeArgs& a, int p, bool report) {
  int len = a.prefix_lens[p];
  const int cap = a.prefix_max_pages * a.page_size;
  if (len > cap) {
    if (report) atomicOr(a.sync, kStatusLenClamped);
    len = cap;
  }
  return len < 0 ? 0 : len;
}

// Exclusive prefix sum of f(i) over i in [0, n) into out[0..n] (out[n] = total), by every thread
// of the block; returns the total. Each thread scans a contiguous range, then one warp scans the
// warps' sums. scratch: 33 ints. Ends with a block barrier.
template <typename F>
__device__ __forceinline__ int block_scan(int n, F f, int* out, int* scratch) {
  const int nt = blockDim.x, tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5, nw = nt >> 5;
  const int per = (n + nt - 1) / nt;
  const int lo = min(n, tid * per), hi = min(n, lo + per);
  int local = 0;
  for (int i = lo; i < hi; ++i) local += f(i);
  int inc = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += v;
  }
  if (lane == 31) scratch[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    const int v = lane < nw ? scratch[lane] : 0;
    int vi = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, vi, o);
      if (lane >= o) vi += u;
    }
    if (lane < nw) scratch[lane] = vi - v;
    if (lane == 31) scratch[32] = vi;
  }
  __syncthreads();
  int run = scratch[warp] + inc - local;
  for (int i = lo; i < hi; ++i) {
    out[i] = run;
    run += f(i);
  }
  const int total = scratch[32];
  if (tid == 0) out[n] = total;
  __syncthreads();
  return total;
}

// Group of prefix item e (< V): the last group whose first entry is <= e.
__device__ __forceinline__ int group_of_entry(const int* vstart, int P, int e) {
  int lo = 0, hi = P - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (vstart[mid] <= e) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// All threads of the block. Builds the plan's entries: lens[e] = clamped token count, prefix[e] =
// cost of one unit of every entry before e, where a non-empty entry costs its tiles plus seg_cost
// (the time a CTA spends starting an (entry, unit): Q loads, partial write and count, merge);
// misc[0] = total cost over all units, misc[1] = R, misc[2] (abort flag) and misc[3] zeroed,
// misc[kMiscV] = V, misc[kMiscEntries] = entries. For a cascade, also hp and vstart; a group
// table that is not a partition of the batch (indptr[0] = 0, non-decreasing, indptr[P] = batch)
// turns the prefixes off and sets KL_STATUS_BAD_PREFIX_GROUPS. Ends with a block barrier.
// `streams`: ranges per CTA (the plan is cut into gridDim.x * streams ranges).
// The kernels' helpers are all force-inlined: the decode kernels run at their register cap, where a
// helper compiled as a real call (with a stack frame) costs spills.
__device__ __forceinline__ void plan_build(const DecodeArgs& a, const PlanSmem& ps, int streams = 1) {
  const int B = a.batch;
  const int nt = blockDim.x, tid = threadIdx.x;
  const bool report = blockIdx.x == 0;
  int* misc = ps.misc;
  int V = 0;
  if (a.num_prefixes > 0) {
    const int P = a.num_prefixes, Mb = a.members;
    bool bad = false;
    for (int p = tid; p < P; p += nt) {
      const int lo = __ldg(a.prefix_indptr + p), hi = __ldg(a.prefix_indptr + p + 1);
      bad |= lo > hi || (p == 0 && lo != 0) || (p == P - 1 && hi != B);
    }
    bad = __syncthreads_or(bad);
    if (bad && report && tid == 0) atomicOr(a.sync, kStatusBadPrefixGroups);
    V = block_scan(
        P,
        [&](int p) {
          if (bad) return 0;
          const int m = __ldg(a.prefix_indptr + p + 1) - __ldg(a.prefix_indptr + p);
          return (m + Mb - 1) / Mb;
        },
        ps.vstart, misc + kMiscScan);
    for (int b = tid; b < B; b += nt) {
      int len = 0;
      if (!bad) {
        int lo = 0, hi = P - 1;  // last group starting at or before b
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (__ldg(a.prefix_indptr + mid) <= b) lo = mid; else hi = mid - 1;
        }
        len = clamp_prefix_len(a, lo, false);
      }
      ps.hp[b] = len;
    }
    if (report) {
      for (int p = tid; p < P; p += nt) clamp_prefix_len(a, p, true);
    }
  }
  if (a.prefix_chunk > 0) V = 0;  // the prefix chunks run in the tensor-core prefix kernel
  const int n = V + B;
  for (int e = tid; e < n; e += nt) {
    ps.lens[e] = e < V ? clamp_prefix_len(a, group_of_entry(ps.vstart, a.num_prefixes, e), false)
                       : clamp_len(a, e - V, report);
  }
  __syncthreads();
  const int* lens = ps.lens;
  const int per_unit = block_scan(
      n, [&](int e) { return lens[e] > 0 ? (lens[e] + kTile - 1) / kTile + a.seg_cost : 0; }, ps.prefix,
      misc + kMiscScan);
  if (tid == 0) {
    const int total = per_unit * a.units;
    misc[0] = total;
    const int vgrid = static_cast<int>(gridDim.x) * streams;
    misc[1] = max(a.min_tiles, (total + vgrid - 1) / vgrid);
    misc[2] = 0;
    misc[3] = 0;
    misc[kMiscV] = V;
    misc[kMiscEntries] = n;
  }
  __syncthreads();
}

// Range vidx of vgrid (default: this CTA's of the grid's); plan_build must have cut the plan into
// vgrid ranges.
__device__ __forceinline__ void walk_init(const DecodeArgs& a, const int* misc, Walk& w, int vidx = -1,
                                          int vgrid = -1) {
  w.vidx = vidx >= 0 ? vidx : static_cast<int>(blockIdx.x);
  w.vgrid = vgrid > 0 ? vgrid : static_cast<int>(gridDim.x);
  w.V = misc[kMiscV];
  w.n = misc[kMiscEntries];
  if (a.splits == 0) {
    const int total = misc[0];
    w.R = misc[1];
    const int64_t t0 = static_cast<int64_t>(w.vidx) * w.R;
    w.t = static_cast<int>(min(t0, static_cast<int64_t>(total)));
    w.t1 = static_cast<int>(min(t0 + w.R, static_cast<int64_t>(total)));
    w.first = true;
  } else {
    w.item = w.vidx;
    w.items = a.batch * a.units * a.splits;
  }
}

// Who entry b serves: a prefix item's member block, or sequence b - V. CAS: the launch is a
// cascade (otherwise entries are sequences, known at compile time).
template <bool CAS>
__device__ __forceinline__ void entry_members(const DecodeArgs& a, const PlanSmem& ps, const Walk& w, Seg& s) {
  if (!CAS) {
    s.seq = s.b;
    s.nmem = 1;
    s.grp = -1;
    s.cb = s.b;
  } else if (s.b < w.V) {
    const int p = group_of_entry(ps.vstart, a.num_prefixes, s.b);
    const int first = __ldg(a.prefix_indptr + p), end = __ldg(a.prefix_indptr + p + 1);
    s.seq = first + (s.b - ps.vstart[p]) * a.members;
    s.nmem = min(a.members, end - s.seq);
    s.grp = p;
    s.cb = a.batch + s.b;
  } else {
    s.seq = s.b - w.V;
    s.nmem = 1;
    s.grp = -1;
    s.cb = s.seq;
  }
}

template <bool CAS = false>
__device__ __forceinline__ bool walk_next(const DecodeArgs& a, const PlanSmem& ps, Walk& w, Seg& s) {
  const int U = a.units;
  const int* lens = ps.lens;
  const int* prefix = ps.prefix;
  if (a.splits == 0) {
    if (w.t >= w.t1) return false;
    int lo = 0, hi = w.n - 1;  // largest entry b with U * prefix[b] <= t
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (static_cast<int64_t>(U) * prefix[mid] <= w.t) lo = mid; else hi = mid - 1;
    }
    // b is never empty here: an empty entry has the same prefix as the next one.
    const int b = lo;
    const int nc = prefix[b + 1] - prefix[b];      // cost of one unit: seg_cost, then the tiles
    const int n = (lens[b] + kTile - 1) / kTile;  // tiles of one unit
    const int seq0 = U * prefix[b];
    const int u = (w.t - seq0) / nc;
    const int s_begin = seq0 + u * nc;  // the item's cost range [s_begin, s_end) ends with its tiles
    const int s_end = s_begin + nc;
    const int ts = s_end - n;
    if (w.t1 <= ts) return false;  // this range ends before the item's first tile
    const int from = max(w.t, ts);
    const int tile = from - ts;
    const int len = min(s_end, w.t1) - from;
    s.b = b;
    s.u = u;
    s.tok_begin = tile * kTile;
    s.tok_end = min(lens[b], (tile + len) * kTile);
    s.c_first = ts / w.R;
    s.nchunks = (s_end - 1) / w.R - s.c_first + 1;
    // The first chunk is its CTA's first segment iff that CTA's range holds no earlier tiles.
    s.first_aligned = s.c_first * w.R >= s_begin;
    s.whole = s.nchunks == 1;
    s.chunk = w.first ? 2 * w.vidx : 2 * w.vidx + 1;
    w.first = false;
    w.t = from + len;
    entry_members<CAS>(a, ps, w, s);
    return true;
  }
  if (w.item >= w.items) return false;
  const int i = w.item;
  const int S = a.splits;
  s.u = i % U;
  const int sp = (i / U) % S;
  s.b = i / (U * S);
  const int span = a.pages_per_split * a.page_size;
  s.tok_begin = sp * span;
  s.tok_end = max(s.tok_begin, min(lens[s.b], s.tok_begin + span));
  s.chunk = i;
  s.nchunks = S;
  s.c_first = 0;
  s.first_aligned = true;
  s.whole = S == 1;
  w.item += w.vgrid;
  entry_members<CAS>(a, ps, w, s);
  return true;
}

// Chunk id of the k-th chunk of segment s's (entry, unit).
__device__ __forceinline__ int chunk_id(const DecodeArgs& a, const Seg& s, int k) {
  if (a.splits == 0) {
    const int c = s.c_first + k;
    return (k == 0 && !s.first_aligned) ? 2 * c + 1 : 2 * c;
  }
  return (s.b * a.splits + k) * a.units + s.u;
}

// Arrival counters: block cb in [0, batch) for sequences' own tokens, [batch, 2 batch) for
// prefix items; a cascade's per-sequence side counters follow at 2 batch + b.
__device__ __forceinline__ uint32_t* counter_of(const DecodeArgs& a, int cb, int kvh, int hg) {
  return a.sync + 1 + (static_cast<int64_t>(cb) * a.num_kv_heads + kvh) * kMaxHeadGroups + hg;
}

// Stores one vector of final output at element offset `off`: to this call's output and, in a
// head gather, to the same place in every other rank's output (plain stores over NVLink).
template <typename T, bool GATHER, typename V>
__device__ __forceinline__ void store_out(const DecodeArgs& a, int64_t off, const V& v) {
  *reinterpret_cast<V*>(static_cast<T*>(a.out) + off) = v;
  if (GATHER) {
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r) {
      if (r < a.gat.ranks && r != a.gat.rank) *reinterpret_cast<V*>(static_cast<T*>(a.gat.out[r]) + off) = v;
    }
  }
}

// Zero the outputs of sequences with no token at all (balanced mode has no work for them).
// seq_len_s[b] = sequence b's own clamped length; hp (cascade only) its group's prefix length.
template <typename T, bool GATHER>
__device__ __forceinline__ void zero_empty_sequences(const DecodeArgs& a, const int* seq_len_s, const int* hp,
                                                     int ctid, int nthr) {
  if (a.splits != 0) return;
  const int n = a.num_q_heads * a.head_dim;
  const T zero = Storage<T>::store(0.0f);
  for (int b = blockIdx.x; b < a.batch; b += gridDim.x) {
    if (seq_len_s[b] != 0 || (hp != nullptr && hp[b] != 0)) continue;
    for (int i = ctid; i < n; i += nthr) store_out<T, GATHER>(a, static_cast<int64_t>(b) * (GATHER ? a.out_seq_stride : n) + i, zero);
  }
}

// Where a warp's final rows go. Row hl of the warp is query row r = row0 + hl of its entry:
// member m = r / group, query head kvh * group + r % group of sequence seq + m (rows with
// m >= nmem are padding). Members whose bit is set in `cas` are one side of a cascade: their rows
// go, normalised, to that side's fp32 state with their LSE; the other rows are final outputs.
struct RowSink {
  int seq, nmem, kvh, row0, side;
  uint32_t cas;
};

template <bool CAS>
__device__ __forceinline__ int64_t sink_row(const DecodeArgs& a, const RowSink& k, int hl, int& m) {
  const int r = k.row0 + hl;
  m = CAS ? r / a.group : 0;  // without a cascade every row < nh belongs to member 0
  return static_cast<int64_t>(k.seq + m) * a.num_q_heads + k.kvh * a.group + (r - m * a.group);
}

// Element offset of row hl's final output (member m of the sink, as sink_row gives it). Without a
// gather the output rows are contiguous ([batch, num_q_heads, head_dim]).
template <bool CAS, bool GATHER>
__device__ __forceinline__ int64_t sink_out(const DecodeArgs& a, const RowSink& k, int hl, int m) {
  const int r = k.row0 + hl;
  const int head = k.kvh * a.group + (r - m * a.group);
  if (!GATHER) return (static_cast<int64_t>(k.seq + m) * a.num_q_heads + head) * a.head_dim;
  return static_cast<int64_t>(k.seq + m) * a.out_seq_stride + static_cast<int64_t>(head) * a.head_dim;
}


// Row offset of a cascade side's plane: the (single) prefix plane of an in-plan prefix item, or
// the sequence's own plane after the prefix chunk planes.
__device__ __forceinline__ int64_t side_offset(const DecodeArgs& a, int side) {
  return static_cast<int64_t>(side == 0 ? 0 : a.cas_planes) * a.batch * a.num_q_heads;
}

// Prefix planes of sequence b's cascade, from its group's clamped prefix length.
__device__ __forceinline__ int prefix_planes(const DecodeArgs& a, int prefix_len) {
  return a.prefix_chunk > 0 ? (prefix_len + a.prefix_chunk - 1) / a.prefix_chunk : 1;
}

// Merge of a split (entry, unit, query-head group) by one warp, every chunk's normalised
// partial and base-2 LSE being in scratch. Lane k reads chunk k's LSEs (32 chunks a round);
// the per-head max M and weight sum W come from fixed-order warp reductions. Then lane L owns
// float4 i = L + 32*j (j < NE) of the nh x D outputs and accumulates sum_k 2^(lse_k - M) * o_k
// in chunk order, with KB chunks' loads in flight at a time and each weight shuffled from its
// chunk's lane. The result depends only on the partials, never on which chunk merges; it is
// written as out = sum / W (zero where every chunk was empty). kernel-lab's merge formula
// (triton_kernels/paged_attention.py:150-166).
template <typename T, int D, int HPW, int NE, int KB, bool CAS, bool GATHER>
__device__ __forceinline__ void merge_chunks_impl(const DecodeArgs& a, const Seg& s, int slots_per_chunk, int mu,
                                                  int nh, const RowSink& sink, int lane) {
  constexpr int Q = D / 4;  // float4 per head row
  const int n4 = nh * Q;
  const int nchunks = s.nchunks;
  auto part_row = [&](int k) {  // first element (in heads) of chunk k's partial rows for this group
    return (static_cast<int64_t>(chunk_id(a, s, k)) * slots_per_chunk + mu) * HPW;
  };
  auto load_lse = [&](int k, float (&l)[HPW]) {
#pragma unroll
    for (int h = 0; h < HPW; ++h) l[h] = -INFINITY;
    if (k < nchunks) {
      const float4* p = reinterpret_cast<const float4*>(a.part_lse + part_row(k));
#pragma unroll
      for (int h4 = 0; h4 < HPW / 4; ++h4) {
        const float4 v = __ldcg(p + h4);
        l[4 * h4 + 0] = 4 * h4 + 0 < nh ? v.x : -INFINITY;
        l[4 * h4 + 1] = 4 * h4 + 1 < nh ? v.y : -INFINITY;
        l[4 * h4 + 2] = 4 * h4 + 2 < nh ? v.z : -INFINITY;
        l[4 * h4 + 3] = 4 * h4 + 3 < nh ? v.w : -INFINITY;
      }
    }
  };
  float4 x[KB][NE];
  auto load_batch = [&](int k0) {
#pragma unroll
    for (int q = 0; q < KB; ++q) {
      const bool kv = k0 + q < nchunks;
      const float4* p = reinterpret_cast<const float4*>(a.part_o + (kv ? part_row(k0 + q) : 0) * D);
#pragma unroll
      for (int j = 0; j < NE; ++j) {
        const int i = lane + 32 * j;
        x[q][j] = kv && i < n4 ? __ldcg(p + i) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
    }
  };
  auto weigh = [&](float (&f)[HPW], const float (&M)[HPW], float (&W)[HPW]) {
#pragma unroll
    for (int h = 0; h < HPW; ++h) {
      f[h] = f[h] > -INFINITY ? fast_exp2(f[h] - M[h]) : 0.0f;
      W[h] += warp_allreduce_sum(f[h]);
    }
  };
  load_batch(0);  // in flight while the LSEs are read and reduced

  float M[HPW], W[HPW], f[HPW];
#pragma unroll
  for (int h = 0; h < HPW; ++h) {
    M[h] = -INFINITY;
    W[h] = 0.0f;
  }
  for (int k0 = 0; k0 < nchunks; k0 += 32) {
    load_lse(k0 + lane, f);
#pragma unroll
    for (int h = 0; h < HPW; ++h) M[h] = fmaxf(M[h], warp_allreduce_max(f[h]));
  }
  if (nchunks <= 32) weigh(f, M, W);  // f still holds the only round's LSEs
  float4 o[NE];
#pragma unroll
  for (int j = 0; j < NE; ++j) o[j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  for (int k0 = 0; k0 < nchunks; k0 += 32) {
    if (nchunks > 32) {
      load_lse(k0 + lane, f);
      weigh(f, M, W);
    }
    const int kn = min(32, nchunks - k0);
    for (int kb = 0; kb < kn; kb += KB) {
      if (k0 + kb > 0) load_batch(k0 + kb);
#pragma unroll
      for (int q = 0; q < KB; ++q) {
        if (kb + q >= kn) break;
#pragma unroll
        for (int j = 0; j < NE; ++j) {
          // Lane L's head in slot j is (L + 32j) / Q: at most two heads across the warp.
          const int h_lo = (32 * j) / Q, h_hi = min(HPW - 1, (32 * j + 31) / Q);
          const int h = (lane + 32 * j) / Q;
          float w = 0.0f;
#pragma unroll
          for (int hh = h_lo; hh <= h_hi; ++hh) {
            const float v = __shfl_sync(0xffffffffu, f[hh], kb + q);
            if (h == hh) w = v;
          }
          o[j].x += w * x[q][j].x;
          o[j].y += w * x[q][j].y;
          o[j].z += w * x[q][j].z;
          o[j].w += w * x[q][j].w;
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < NE; ++j) {
    const int i = lane + 32 * j;
    if (i >= n4) continue;
    const int h_lo = (32 * j) / Q, h_hi = min(HPW - 1, (32 * j + 31) / Q);
    const int h = i / Q;
    float wsum = 0.0f, mh = -INFINITY;
#pragma unroll
    for (int hh = h_lo; hh <= h_hi; ++hh) {
      if (h == hh) {
        wsum = W[hh];
        mh = M[hh];
      }
    }
    const float inv = wsum > 0.0f ? 1.0f / wsum : 0.0f;
    const int c4 = i - h * Q;
    int m;
    const int64_t row = sink_row<CAS>(a, sink, h, m);
    if (CAS && ((sink.cas >> m) & 1u)) {
      const int64_t srow = side_offset(a, sink.side) + row;
      reinterpret_cast<float4*>(a.cas_o + srow * D)[c4] =
          make_float4(o[j].x * inv, o[j].y * inv, o[j].z * inv, o[j].w * inv);
      if (c4 == 0) a.cas_lse[srow] = wsum > 0.0f ? mh + __log2f(wsum) : -INFINITY;
    } else {
      uint2 pk;
      pk.x = Storage<T>::pack2(o[j].x * inv, o[j].y * inv);
      pk.y = Storage<T>::pack2(o[j].z * inv, o[j].w * inv);
      store_out<T, GATHER>(a, sink_out<CAS, GATHER>(a, sink, h, m) + 4 * c4, pk);
    }
  }
}

// Picks the per-lane slot count for the group's nh x D outputs: 4, 8 or 16 float4 per lane
// per chunk, with 4, 2 or 1 chunks' loads in flight (64 registers of loads in each case).
template <typename T, int D, int HPW, bool CAS, bool GATHER>
__device__ __forceinline__ void merge_chunks(const DecodeArgs& a, const Seg& s, int slots_per_chunk, int mu, int nh,
                                             const RowSink& sink, int lane) {
  constexpr int Q = D / 4;
  const int n4 = nh * Q;
  if (n4 <= 128) {
    merge_chunks_impl<T, D, HPW, 4, 4, CAS, GATHER>(a, s, slots_per_chunk, mu, nh, sink, lane);
  } else if (HPW * Q > 128 && n4 <= 256) {
    merge_chunks_impl<T, D, HPW, (HPW * Q > 128 ? 8 : 4), 1, CAS, GATHER>(a, s, slots_per_chunk, mu, nh, sink, lane);
  } else if (HPW * Q > 256) {
    merge_chunks_impl<T, D, HPW, (HPW * Q > 256 ? 16 : 4), 1, CAS, GATHER>(a, s, slots_per_chunk, mu, nh, sink, lane);
  }
}

// Final output of sequence b's query heads kvh * group + row0 .. + nh in a cascade, once every
// part has stored its normalised output and LSE: the nch prefix planes (chunks of its group's
// shared prefix) and, if `own`, its own plane. One pass in plane order with a running maximum,
// out = sum_k 2^(lse_k - M) o_k / sum_k 2^(lse_k - M): the same arithmetic whichever part arrives
// last. One warp: lane L owns float4 columns L + 32 j of the nh x head_dim rows, and four planes'
// loads are in flight at a time.
template <typename T, int D, int NE>
__device__ __forceinline__ void cascade_merge_impl(const DecodeArgs& a, int b, int kvh, int row0, int nh, int nch,
                                                   bool own, int lane) {
  constexpr int Q = D / 4;
  constexpr int KB = 4;
  const int n4 = nh * Q;
  const int np = nch + (own ? 1 : 0);
  const int64_t plane = static_cast<int64_t>(a.batch) * a.num_q_heads;
  const int64_t r0 = static_cast<int64_t>(b) * a.num_q_heads + kvh * a.group + row0;
  float m[NE], wsum[NE];
  float4 acc[NE];
#pragma unroll
  for (int j = 0; j < NE; ++j) {
    m[j] = -INFINITY;
    wsum[j] = 0.0f;
    acc[j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  }
  for (int k0 = 0; k0 < np; k0 += KB) {
    float l[KB][NE];
    float4 x[KB][NE];
#pragma unroll
    for (int q = 0; q < KB; ++q) {
      const int k = k0 + q;
      const int64_t off = static_cast<int64_t>(k < nch ? k : a.cas_planes) * plane;
#pragma unroll
      for (int j = 0; j < NE; ++j) {
        const int i = lane + 32 * j;
        const bool ld = k < np && i < n4;
        const int h = i / Q;
        l[q][j] = ld ? __ldcg(a.cas_lse + off + r0 + h) : -INFINITY;
        x[q][j] = ld ? __ldcg(reinterpret_cast<const float4*>(a.cas_o + (off + r0 + h) * D) + (i - h * Q))
                     : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
    }
#pragma unroll
    for (int q = 0; q < KB; ++q) {
#pragma unroll
      for (int j = 0; j < NE; ++j) {
        const float mn = fmaxf(m[j], l[q][j]);
        if (mn == -INFINITY) continue;
        const float fa = fast_exp2(m[j] - mn), fb = fast_exp2(l[q][j] - mn);
        m[j] = mn;
        wsum[j] = wsum[j] * fa + fb;
        acc[j].x = acc[j].x * fa + fb * x[q][j].x;
        acc[j].y = acc[j].y * fa + fb * x[q][j].y;
        acc[j].z = acc[j].z * fa + fb * x[q][j].z;
        acc[j].w = acc[j].w * fa + fb * x[q][j].w;
      }
    }
  }
  T* out = static_cast<T*>(a.out);
#pragma unroll
  for (int j = 0; j < NE; ++j) {
    const int i = lane + 32 * j;
    if (i >= n4) continue;
    const int h = i / Q;
    const float inv = wsum[j] > 0.0f ? 1.0f / wsum[j] : 0.0f;
    uint2 pk;
    pk.x = Storage<T>::pack2(acc[j].x * inv, acc[j].y * inv);
    pk.y = Storage<T>::pack2(acc[j].z * inv, acc[j].w * inv);
    *reinterpret_cast<uint2*>(out + (r0 + h) * D + 4 * (i - h * Q)) = pk;
  }
}

template <typename T, int D>
__device__ __forceinline__ void cascade_merge(const DecodeArgs& a, int b, int kvh, int row0, int nh, int nch,
                                              bool own, int lane) {
  constexpr int Q = D / 4;
  if (nh * Q <= 128) {
    cascade_merge_impl<T, D, 4>(a, b, kvh, row0, nh, nch, own, lane);
  } else if (nh * Q <= 256) {
    cascade_merge_impl<T, D, 8>(a, b, kvh, row0, nh, nch, own, lane);
  } else {
    for (int r = 0; r < nh; r += 256 / Q) {  // 256 float4 at a time
      cascade_merge_impl<T, D, 8>(a, b, kvh, row0 + r, min(256 / Q, nh - r), nch, own, lane);
    }
  }
}

// After a warp has stored one side of a cascade for the members in sink.cas: each such member's
// lane counts the side's arrival (a release of the warp's stores); the second side to arrive
// (acquire) merges the member's rows and returns its counter to zero. `hg` is the query-head
// group of the counter: a member's rows in it are its query heads grow0 .. grow0 + nh of the KV
// head's group (grow0 = hg * heads per warp; a packed prefix item has one group).
template <typename T, int D>
__device__ __forceinline__ void cascade_arrive(const DecodeArgs& a, const RowSink& sink, int hg,
                                               int grow0, int nh, int lane) {
  __syncwarp();
  bool last = false;
  if (lane < sink.nmem && ((sink.cas >> lane) & 1u)) {
    // The tensor-core prefix kernels ran before this launch: the prefix state is complete in
    // plane 0 and this side is the last. Otherwise two sides count.
    last = a.prefix_chunk > 0 ||
           atom_add_acq_rel_gpu(counter_of(a, 2 * a.batch + sink.seq + lane, sink.kvh, hg), 1u) == 1u;
  }
  uint32_t todo = __ballot_sync(0xffffffffu, last);
  while (todo != 0u) {
    const int m = __ffs(todo) - 1;
    todo &= todo - 1u;
    __syncwarp();
    cascade_merge<T, D>(a, sink.seq + m, sink.kvh, grow0, nh, 1, true, lane);
    if (lane == m && a.prefix_chunk == 0) {
      *reinterpret_cast<volatile uint32_t*>(counter_of(a, 2 * a.batch + sink.seq + m, sink.kvh, hg)) = 0u;
    }
  }
}

// End of a head-gather launch, by every consumer thread of every CTA. The CTA meets at a barrier
// (its rows, local and over NVLink, are stored), and one thread counts the CTA with a GPU-scope
// releasing atomic. The CTA that completes the count acquires every CTA's rows through it, fences
// at system scope and publishes this launch's epoch in every rank's flags with system-scope
// releases: a peer that acquires its flag sees every row this GPU stored (release and acquire are
// cumulative along the chain barrier, GPU-scope count, system-scope flag). It then waits until
// every rank's epoch has arrived in this rank's flags (an epoch at or past this launch's also
// counts: a peer may already be one launch ahead), for at most g.wait_ns; on timeout it sets
// kStatusPeerTimeout and leaves. It returns the count to zero for the next launch. One system-scope
// fence per launch instead of one per thread: measured 176 against 188 us at two GPUs.
__device__ __forceinline__ void gather_finish(const DecodeArgs& a, int nthreads) {
  named_barrier(15, nthreads);
  if (threadIdx.x != 0) return;
  const Gather& g = a.gat;
  if (atom_add_acq_rel_gpu(g.done, 1u) != gridDim.x - 1) return;
  fence_acq_rel_sys();
  for (int r = 0; r < g.ranks; ++r) st_release_sys(g.flags[r] + g.rank, g.epoch);
  const uint32_t* own = g.flags[g.rank];
  const uint64_t t0 = globaltimer_ns();
  bool late = false;
  for (int r = 0; r < g.ranks && !late; ++r) {
    while (static_cast<int32_t>(ld_acquire_sys(own + r) - g.epoch) < 0) {
      if (globaltimer_ns() - t0 > g.wait_ns) {
        atomicOr(a.sync, kStatusPeerTimeout);
        late = true;
        break;
      }
      __nanosleep(128);
    }
  }
  *reinterpret_cast<volatile uint32_t*>(g.done) = 0u;
}

// ------------------------------------------------------------------------- tensor-core kernel

struct TcLayout {
  uint32_t head_bytes, half, stage_bytes, ring, bars, red_m, red_l, red_acc, misc, prefix, lens, hp, vstart, total;
};

__host__ __device__ constexpr uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

// groups > 0: a cascade over that many prefix groups (plan entries for prefix items as well).
// streams > 1: each warp walks its own range (no combine slots).
__host__ __device__ __forceinline__ TcLayout tc_layout(int D, int NT, int TW, int streams, int nstage, int batch, int eb = 2,
                                              int groups = 0, int HT = 1) {
  TcLayout L{};
  L.head_bytes = kTile * D * eb;  // one head's K (or V) rows of a tile (eb bytes per element)
  L.half = HT * L.head_bytes;
  L.stage_bytes = 2u * L.half;
  uint32_t off = 0;
  L.ring = off;
  off += nstage * L.stage_bytes;
  L.bars = off;
  off += 2u * nstage * 8u;
  // Shared ring with TW > 1: combine slots for the warps that hand their (m, l, acc) to a tw == 0
  // warp (all but kCW / TW). Streams need none.
  const uint32_t red_warps = TW > 1 && streams == 1 ? kCW - kCW / TW : 0;
  L.red_m = off;
  off += red_warps * 8u * NT * 4u;
  L.red_l = off;
  off += red_warps * 8u * NT * 4u;
  L.red_acc = off;
  off += red_warps * 8u * NT * (D + 4u) * 4u;
  L.misc = off;
  off += 64u * 4u;
  const uint32_t entries = groups > 0 ? 2u * batch : static_cast<uint32_t>(batch);
  L.prefix = off;
  off += (entries + 1u) * 4u;
  L.lens = off;
  off += entries * 4u;
  L.hp = off;
  off += groups > 0 ? batch * 4u : 0u;
  L.vstart = off;
  off += groups > 0 ? (groups + 1u) * 4u : 0u;
  L.total = align_up(off, 16) + 1024u;  // slack to align the base to 1024 B (swizzle atom)
  return L;
}

// Stores a warp's final rows held in the MMA fragment layout: lane (g, t4) owns, for row
// hl = nt*8 + 2*t4 + e and piece c, output d = 8*OW*c + OW*g + k (k < OW), the value
// X[c*OW/2 + k/2][nt][e + 2*(k & 1)] * f[nt][e]. Rows hl >= nh are padding. A cascade member's
// rows go to its side's fp32 state (with lse), the others to out as T.
template <typename T, int D, int NT, int OW, bool CAS, bool GATHER>
__device__ __forceinline__ void store_rows(const DecodeArgs& a, const RowSink& sink, const float (&X)[D / 16][NT][4],
                                           const float (&f)[NT][2], const float (&lse)[NT][2], int g, int t4,
                                           int nh) {
  constexpr int NCH = D / (8 * OW);
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int hl = nt * 8 + 2 * t4 + e;
      if (hl >= nh) continue;
      int m;
      const int64_t row = sink_row<CAS>(a, sink, hl, m);
      const float x = f[nt][e];
      if (CAS && ((sink.cas >> m) & 1u)) {
        const int64_t srow = side_offset(a, sink.side) + row;
        float* dst = a.cas_o + srow * D;
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
#pragma unroll
          for (int h = 0; h < OW / 4; ++h) {
            const int m0 = c * (OW / 2) + 2 * h;
            *reinterpret_cast<float4*>(dst + c * 8 * OW + OW * g + 4 * h) =
                make_float4(X[m0][nt][e] * x, X[m0][nt][e + 2] * x, X[m0 + 1][nt][e] * x, X[m0 + 1][nt][e + 2] * x);
          }
        }
        if (g == 0) a.cas_lse[srow] = lse[nt][e];
      } else {
        const int64_t orow = sink_out<CAS, GATHER>(a, sink, hl, m);
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
#pragma unroll
          for (int h = 0; h < OW / 8; ++h) {
            const int m0 = c * (OW / 2) + 4 * h;
            uint4 pk;
            pk.x = Storage<T>::pack2(X[m0 + 0][nt][e] * x, X[m0 + 0][nt][e + 2] * x);
            pk.y = Storage<T>::pack2(X[m0 + 1][nt][e] * x, X[m0 + 1][nt][e + 2] * x);
            pk.z = Storage<T>::pack2(X[m0 + 2][nt][e] * x, X[m0 + 2][nt][e + 2] * x);
            pk.w = Storage<T>::pack2(X[m0 + 3][nt][e] * x, X[m0 + 3][nt][e + 2] * x);
            store_out<T, GATHER>(a, orow + c * 8 * OW + OW * g + 8 * h, pk);
          }
        }
      }
    }
  }
}

template <typename T, int D, int NT, bool KV8, bool CAS, bool GATHER>
__global__ void __launch_bounds__(kTCThreads, 1) decode_tc_kernel(const __grid_constant__ CUtensorMap tmk,
                                                                  const __grid_constant__ CUtensorMap tmv,
                                                                  const __grid_constant__ DecodeArgs a, const TcShape cfg) {
  // KV8: the cache holds e4m3 (one byte per element, per-KV-head scales) and the MMAs run in
  // f16 (e4m3 converts to f16 exactly); otherwise the cache and the MMAs use T.
  using MT = typename std::conditional<KV8, __half, T>::type;
  constexpr int EB = KV8 ? 1 : 2;     // cache bytes per element
  constexpr int NCH = D * EB / 128;   // 128-byte pieces of one head's row of K (or V)
  constexpr int KS = D / 16;          // k-steps of K.Q^T, and m-tiles of V^T.P^T
  constexpr int HPW = 8 * NT;         // query heads per consumer warp
  constexpr int OW = 128 / (8 * EB);  // consecutive output values a lane owns per piece (8 or 16)

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int HT = cfg.ht, HG = cfg.hg, TW = cfg.tw, nstage = cfg.nstage;
  // Streams exist only in the one-n-tile kernels; the others see the constant 1.
  const int NS = NT == 1 ? cfg.ns : 1;  // streams (ranges) of this CTA
  const TcLayout L = tc_layout(D, NT, TW, NS, nstage, a.batch, EB, a.num_prefixes, HT);
  const uint32_t ring = smem_u32(smem + L.ring);
  const uint32_t bars = smem_u32(smem + L.bars);
  float* red_m = reinterpret_cast<float*>(smem + L.red_m);
  float* red_l = reinterpret_cast<float*>(smem + L.red_l);
  float* red_acc = reinterpret_cast<float*>(smem + L.red_acc);
  PlanSmem ps;
  ps.misc = reinterpret_cast<int*>(smem + L.misc);
  ps.prefix = reinterpret_cast<int*>(smem + L.prefix);
  ps.lens = reinterpret_cast<int*>(smem + L.lens);
  ps.hp = a.num_prefixes > 0 ? reinterpret_cast<int*>(smem + L.hp) : nullptr;
  ps.vstart = a.num_prefixes > 0 ? reinterpret_cast<int*>(smem + L.vstart) : nullptr;
  int* misc = ps.misc;
  // A stage half holds the tile as rows of 128 bytes, row r = token * HT * NCH + piece with
  // piece = head * NCH + c over the tile's HT heads, in the TMA's 128-byte swizzle: 16-byte unit
  // u of row r sits at unit u ^ (r & 7).
  const int rows_per_tok = HT * NCH;
  auto stage_row = [&](int tok, int piece) { return tok * rows_per_tok + piece; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // Streams: when a tile holds one (head, group) pair (HT * HG == 1, TW == 8), warp t is stream t:
  // it walks its own range of the plan (range CTA * TW + t) and reads its own ring stages t,
  // t + TW, t + 2 TW, ... (SPS of them); no warp waits for another, and the producer feeds every
  // stream. Otherwise (NS == 1) the CTA has one range and one ring: the HT * HG warps of a tile
  // read every stage, and with TW > 1 the TW warps of a (head, group) take its tiles in turn and
  // combine at the end of a segment. Streams measured 205.5 -> 186.2 us at 512 sequences x 4096
  // tokens of one KV head (Llama-3-8B heads sharded 8 ways), and slower than the shared ring with
  // two or four warps a stream (their ranges cut the plan 2-4 times finer: more split merges).
  const int SPS = nstage / NS;  // stages per stream (nstage is a multiple of TW)
  if (threadIdx.x == 0) {
    for (int s = 0; s < nstage; ++s) {
      mbar_init(bars + 8u * s, 1);                   // full: the producer's expect_tx arrival
      mbar_init(bars + 8u * (nstage + s), HT * HG);  // empty: every warp of the stream reads the stage
    }
    fence_barrier_init();
  }
  if (warp == kCW && lane == 0) {
    tma_prefetch_descriptor(&tmk);
    tma_prefetch_descriptor(&tmv);
  }
  // Launched with programmatic stream serialization: the prologue above overlaps the previous
  // kernel's tail; nothing global (inputs, status word, scratch shared with the previous call) is
  // touched before that kernel has completed. The next call may start launching right away: its
  // CTAs can only take an SM this grid has left.
  wait_prior_grid();
  allow_next_grid();
  plan_build(a, ps, NS);
  volatile int* abort_flag = misc + 2;

  if (warp == kCW) {
    // ---------------- producer warp: one 3-D TMA box per tensor per tile (per page for page size 8).
    // Lane-parallel issue for small stages: each pass finds how many of the next tiles have a
    // free ring stage (lane t tests tile t's stage without blocking) and lane t issues tile t.
    // One producer pass is a serial chain of ~1300 cycles, so one tile a pass caps an SM at a
    // tile per ~0.66 us (12 GB/s with 8 KB tiles); batched, the ring fills at once at start-up
    // and whenever consumers free several stages together. Only when the next stage is busy does
    // the warp block, on that stage alone.
    Walk w;
    walk_init(a, misc, w);
    Seg s;
    uint32_t gt = 0;
    // Pages read once are streamed (evict first); a shared prefix's pages are read again by the
    // group's other member blocks, so they keep the normal priority.
    const uint64_t policy_stream = l2_policy_evict_first();
    const uint64_t policy_shared = l2_policy_evict_normal();
    const int p_rows = cfg.p_rows;
    const int nsub = kTile / p_rows;
    const uint32_t sub_bytes = 2u * p_rows * rows_per_tok * 128u;
    if (NT == 1 && NS > 1) {
      // Stream mode: lane t < NS feeds stream t. It walks the stream's range, looks each tile's
      // page(s) up one tile ahead (a plain load whose latency hides behind the stream's stages) and
      // issues the tile as soon as the stream's next stage is free; no lane waits for another, so a
      // stream whose warps are busy with a segment's end holds back only its own stages.
      const bool mine = lane < NS;
      Walk sw;
      Seg ss;
      if (mine) walk_init(a, misc, sw, static_cast<int>(blockIdx.x) * NS + lane, static_cast<int>(gridDim.x) * NS);
      bool done = !mine, live = false;
      int j = 0, ntiles = 0, piece0 = 0;
      uint32_t k = 0;  // tiles issued on this stream
      const int32_t* bt_row = nullptr;
      uint64_t policy = policy_stream;
      bool pv[2] = {false, false};
      int py[2] = {0, 0};
      auto lookup = [&](int jj) {  // tile jj's page pieces: TMA row coordinate, or invalid
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int tok = ss.tok_begin + jj * kTile + r * p_rows;
          pv[r] = false;
          py[r] = 0;
          if (r < nsub && tok < ss.tok_end) {
            const int pidx = tok / a.page_size;
            const int page = __ldg(bt_row + pidx);
            const bool good = page >= 0 && (a.num_pages < 0 || page < a.num_pages);
            if (!good) atomicOr(a.sync, kStatusBadPage);
            pv[r] = good;
            py[r] = good ? page * a.page_size + (tok - pidx * a.page_size) : 0;
          }
        }
      };
      uint64_t idle_since = clock64();
      while (__any_sync(0xffffffffu, !done)) {
        if (*abort_flag) break;
        bool progressed = false;
        if (!done && !live) {
          bool got = walk_next<CAS>(a, ps, sw, ss);
          while (got && ss.tok_end <= ss.tok_begin) got = walk_next<CAS>(a, ps, sw, ss);  // empty splits
          if (!got) {
            done = true;
          } else {
            live = true;
            j = 0;
            ntiles = (ss.tok_end - ss.tok_begin + kTile - 1) / kTile;
            const bool shared = CAS && ss.grp >= 0;
            bt_row = shared ? a.prefix_bt + static_cast<int64_t>(ss.grp) * a.prefix_bt_stride
                            : a.block_table + static_cast<int64_t>(ss.seq) * a.bt_stride;
            policy = shared ? policy_shared : policy_stream;
            piece0 = ss.u * rows_per_tok;
            lookup(0);
          }
        }
        if (live) {
          const uint32_t stage = static_cast<uint32_t>(lane) + NS * (k % SPS);
          if (mbar_test_wait(bars + 8u * (nstage + stage), ((k / SPS) & 1u) ^ 1u)) {
            const uint32_t full = bars + 8u * stage;
            mbar_arrive_expect_tx(full, (pv[0] ? sub_bytes : 0u) + (pv[1] ? sub_bytes : 0u));
            const uint32_t sbase = ring + stage * L.stage_bytes;
            if (pv[0]) {
              tma_load_3d(sbase, &tmk, 0, piece0, py[0], full, policy);
              tma_load_3d(sbase + L.half, &tmv, 0, piece0, py[0], full, policy);
            }
            if (pv[1]) {
              const uint32_t off = p_rows * rows_per_tok * 128u;
              tma_load_3d(sbase + off, &tmk, 0, piece0, py[1], full, policy);
              tma_load_3d(sbase + L.half + off, &tmv, 0, piece0, py[1], full, policy);
            }
            ++k;
            progressed = true;
            if (++j < ntiles) {
              lookup(j);
            } else {
              live = false;
            }
          }
        }
        if (__any_sync(0xffffffffu, progressed)) {
          idle_since = clock64();
        } else {
          if (static_cast<uint64_t>(clock64()) - idle_since > kWaitLimit) {
            if (lane == 0) atomicOr(a.sync, kStatusWaitTimeout);
            *abort_flag = 1;
            break;
          }
          __nanosleep(32);
        }
      }
      // Let every copy this stream issued land before the CTA may exit.
      if (mine) {
        for (uint32_t kk = k > static_cast<uint32_t>(SPS) ? k - SPS : 0u; kk < k; ++kk) {
          mbar_wait_bounded(bars + 8u * (lane + NS * (kk % SPS)), (kk / SPS) & 1u, a.sync, kWaitLimit);
        }
      }
      return;
    }
    // Batched issue pays off for stages up to 32 KB (4 heads or fewer per tile); with 64 KB
    // stages a tile takes longer to arrive than a producer pass, and single-tile passes
    // measured faster (batch 256 x 8192 tokens, 70B heads).
    const int batch_max = L.stage_bytes <= kBatchStageBytes ? min(32, nstage) : 1;
    bool ok = true;
    while (ok && walk_next<CAS>(a, ps, w, s)) {
      const int ntok = s.tok_end - s.tok_begin;
      if (ntok <= 0) continue;
      const int ntiles = (ntok + kTile - 1) / kTile;
      const bool shared = CAS && s.grp >= 0;
      const int32_t* bt_row = shared ? a.prefix_bt + static_cast<int64_t>(s.grp) * a.prefix_bt_stride
                                     : a.block_table + static_cast<int64_t>(s.seq) * a.bt_stride;
      const uint64_t policy = shared ? policy_shared : policy_stream;
      const int last_page = (s.tok_end - 1) / a.page_size;
      const int piece0 = s.u * rows_per_tok;
      // Block-table window [wbase, wbase + 64): entry wbase + lane in cur, wbase + 32 + lane in nxt.
      int wbase = s.tok_begin / a.page_size;
      int32_t cur = wbase + lane <= last_page ? __ldg(bt_row + wbase + lane) : 0;
      int32_t nxt = wbase + 32 + lane <= last_page ? __ldg(bt_row + wbase + 32 + lane) : 0;
      int j0 = 0;
      while (j0 < ntiles) {
        if (*abort_flag) {
          ok = false;
          break;
        }
        const int tok_first = s.tok_begin + j0 * kTile;
        if (tok_first / a.page_size >= wbase + 32) {
          wbase += 32;
          cur = nxt;
          nxt = wbase + 32 + lane <= last_page ? __ldg(bt_row + wbase + 32 + lane) : 0;
        }
        // Tiles whose pages all lie in the window (at least 16: page size >= 8, and the window
        // reaches 32 pages past the first tile's page).
        const int in_window = ((wbase + 64) * a.page_size - tok_first) / kTile;
        const int want = min(min(ntiles - j0, batch_max), in_window);
        // Lane t < want: the page(s) of tile j0 + t, looked up in the window by shuffles that
        // every lane joins (other lanes look up a dummy entry). Done before any wait, so a
        // freed stage is refilled with nothing but the copies' issue in between.
        const int t0 = tok_first + lane * kTile;
        bool v[2] = {false, false};
        int y[2] = {0, 0};
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int tok = t0 + r * p_rows;
          const bool live = lane < want && r < nsub && tok < s.tok_end;
          const int pidx = live ? tok / a.page_size : wbase;
          const int src = pidx - wbase;
          const int32_t from_cur = __shfl_sync(0xffffffffu, cur, src & 31);
          const int32_t from_nxt = __shfl_sync(0xffffffffu, nxt, src & 31);
          const int page = src < 32 ? from_cur : from_nxt;
          const bool good = page >= 0 && (a.num_pages < 0 || page < a.num_pages);
          if (live && !good) atomicOr(a.sync, kStatusBadPage);  // idempotent if looked up again
          v[r] = live && good;
          y[r] = v[r] ? page * a.page_size + (tok - pidx * a.page_size) : 0;
        }
        const uint32_t g = gt + lane;
        const uint32_t stage = g % static_cast<uint32_t>(nstage);
        const bool is_free = lane < want && mbar_test_wait(bars + 8u * (nstage + stage), ((g / nstage) & 1u) ^ 1u);
        const uint32_t freed = __ballot_sync(0xffffffffu, is_free);
        int nb = freed == 0xffffffffu ? 32 : __ffs(~freed) - 1;  // leading free stages
        // The CTA's first tile goes out alone, a pass ahead of the rest of the ring: at
        // launch every SM requests its whole ring at once, and a first tile queued behind its
        // siblings lands late and holds the consumers back (measured: ~1-2 us at batch 64).
        if (gt == 0) nb = min(nb, 1);
        if (nb == 0) {
          const uint32_t e0 = bars + 8u * (nstage + gt % static_cast<uint32_t>(nstage));
          if (!mbar_wait_bounded(e0, ((gt / nstage) & 1u) ^ 1u, a.sync, kWaitLimit)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          nb = 1;
        }
        if (lane < nb) {
          const uint32_t full = bars + 8u * stage;
          mbar_arrive_expect_tx(full, (v[0] ? sub_bytes : 0u) + (v[1] ? sub_bytes : 0u));
          const uint32_t sbase = ring + stage * L.stage_bytes;
          if (v[0]) {
            tma_load_3d(sbase, &tmk, 0, piece0, y[0], full, policy);
            tma_load_3d(sbase + L.half, &tmv, 0, piece0, y[0], full, policy);
          }
          if (v[1]) {
            const uint32_t off = p_rows * rows_per_tok * 128u;
            tma_load_3d(sbase + off, &tmk, 0, piece0, y[1], full, policy);
            tma_load_3d(sbase + L.half + off, &tmv, 0, piece0, y[1], full, policy);
          }
        }
        __syncwarp();
        gt += nb;
        j0 += nb;
      }
    }
    // Let every copy this CTA issued land before the CTA may exit.
    const uint32_t inflight = min(gt, static_cast<uint32_t>(nstage));
    for (uint32_t k = gt - inflight; k < gt; ++k) {
      mbar_wait_bounded(bars + 8u * (k % nstage), (k / nstage) & 1u, a.sync, kWaitLimit);
    }
    return;
  }

  // ---------------- consumer warps (threads 0..255)
  //
  // Fragments come from plain 16-byte shared loads. The contraction index of S = K.Q^T is
  // permuted (identically for K and Q): k-step j = 2*kk + jj covers, for lane (g, t4),
  // d = 32*kk + 8*t4 + 4*jj + {0,1} (cols 2t4, 2t4+1) and + {2,3} (cols 2t4+8, 2t4+9), so a
  // lane's 16 contiguous bytes of a K row feed two k-steps. The output-row index of
  // O^T = V^T.P^T is permuted too: m-tile 4*c + mt, row g holds d = 64*c + 8*g + 2*mt and
  // row g+8 holds d + 1, so a lane reads one 16-byte unit of V per token and ends up owning
  // 8 consecutive output values per head. Within a quarter-warp the K loads meet 2-way and
  // the V loads 4-way shared-memory bank conflicts (every token of a (head, piece) has the
  // same swizzle phase); a piece-major stage with permuted token rows removes them but measured
  // no faster, the kernel being bound by HBM, not shared memory.
  zero_empty_sequences<T, GATHER>(a, ps.lens + misc[kMiscV], ps.hp, threadIdx.x, kCW * 32);
  const int ht = warp % HT;
  const int hg = (warp / HT) % HG;
  const int tw = warp / (HT * HG);
  const int mu = ht * HG + hg;  // (head, group) within the unit: slot and barrier index
  const int g = lane >> 2, t4 = lane & 3;
  const float sl = a.scale_log2;
  const int G = a.group;

  // A stream walks range CTA * NS + tw and takes every tile of its segments; in the shared ring the
  // TW warps of a (head, group) take tiles tw, tw + TW, ... of the CTA's segments.
  const int st = NS > 1 ? tw : 0;
  const int j_first = NS > 1 ? 0 : tw, j_step = NS > 1 ? 1 : TW;
  Walk w;
  walk_init(a, misc, w, static_cast<int>(blockIdx.x) * NS + st, static_cast<int>(gridDim.x) * NS);
  Seg s;
  uint32_t gt = 0;  // tiles of this ring (the stream's, or the CTA's) before the segment
  while (walk_next<CAS>(a, ps, w, s)) {
    const int ntok = max(0, s.tok_end - s.tok_begin);
    const int ntiles = (ntok + kTile - 1) / kTile;
    const int kvh = s.u * HT + ht;

    // A split chunk reads how many of its sibling chunks have published already; the load's
    // latency hides behind this segment's tiles. If all of them have, this chunk is the last
    // one and merges straight from its registers at the end of the segment.
    uint32_t published = 0;
    if (!s.whole && (NS > 1 || tw == 0) && lane == 0) published = ld_relaxed_gpu(counter_of(a, s.cb, kvh, hg));

    // Q^T as the B operand, in the permuted contraction order of the K loads: one 16-byte load
    // per 32 d (16-bit cache) or two per 64 d (e4m3 cache, converted to f16).
    uint32_t qf[KS][NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      // Query row r of the entry: member r / G (a prefix item packs several sequences' rows into
      // the MMA's N columns), query head r % G of KV head kvh's group.
      const int r = hg * HPW + nt * 8 + g;
      const int m = CAS ? r / G : (r < G ? 0 : 1);
      const bool hv = m < s.nmem;
      const uint4* qrow = reinterpret_cast<const uint4*>(
          static_cast<const T*>(a.q) +
          (static_cast<int64_t>(s.seq + (hv ? m : 0)) * a.num_q_heads + kvh * G + (hv ? r - m * G : 0)) * D);
      if constexpr (!KV8) {
#pragma unroll
        for (int kk = 0; kk < D / 32; ++kk) {
          const uint4 v = hv ? __ldg(qrow + kk * 4 + t4) : make_uint4(0u, 0u, 0u, 0u);
          qf[2 * kk][nt][0] = v.x;
          qf[2 * kk][nt][1] = v.y;
          qf[2 * kk + 1][nt][0] = v.z;
          qf[2 * kk + 1][nt][1] = v.w;
        }
      } else {
#pragma unroll
        for (int kk = 0; kk < D / 64; ++kk) {  // d = 64kk + 16t4 + 0..15 feed k-steps 4kk..4kk+3
          const uint4 v0 = hv ? __ldg(qrow + kk * 8 + 2 * t4) : make_uint4(0u, 0u, 0u, 0u);
          const uint4 v1 = hv ? __ldg(qrow + kk * 8 + 2 * t4 + 1) : make_uint4(0u, 0u, 0u, 0u);
          const uint32_t wq[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            qf[4 * kk + jj][nt][0] = to_f16x2<T>(wq[2 * jj]);
            qf[4 * kk + jj][nt][1] = to_f16x2<T>(wq[2 * jj + 1]);
          }
        }
      }
    }
    // e4m3 cache: the K scale folds into the softmax multiplier, the V scale into the output.
    const float sl_h = KV8 ? sl * __ldg(a.k_scale + kvh) : sl;
    const float v_scale = KV8 ? __ldg(a.v_scale + kvh) : 1.0f;

    float m_run[NT][2], l_run[NT][2], acc[KS][NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      m_run[nt][0] = m_run[nt][1] = -INFINITY;
      l_run[nt][0] = l_run[nt][1] = 0.0f;
#pragma unroll
      for (int mt = 0; mt < KS; ++mt) acc[mt][nt][0] = acc[mt][nt][1] = acc[mt][nt][2] = acc[mt][nt][3] = 0.0f;
    }

    for (int j = j_first; j < ntiles; j += j_step) {
      const uint32_t gj = gt + j;
      const int stage = st + NS * static_cast<int>(gj % SPS);
      if (*abort_flag) break;
      if (!mbar_wait_bounded(bars + 8u * stage, (gj / SPS) & 1u, a.sync, kWaitLimit)) {
        *abort_flag = 1;
        break;
      }
      const int valid = min(kTile, ntok - j * kTile);
      const uint32_t sk = ring + stage * L.stage_bytes;
      const uint32_t sv = sk + L.half;

      // V rows of this tile for piece c: tokens 2t4, 2t4+1, 2t4+8, 2t4+9 (zero past the valid ones).
      auto load_v = [&](int c, uint4 (&v)[4]) {
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const int tok = 2 * t4 + (q4 & 1) + 8 * (q4 >> 1);
          const int r = stage_row(tok, ht * NCH + c);
          v[q4] = lds128(sv + r * 128 + ((g ^ (r & 7)) << 4));
          if (tok >= valid) v[q4] = make_uint4(0u, 0u, 0u, 0u);
        }
      };
      // e4m3 with one piece (outside a cascade, whose kernel has no registers to spare): the V
      // rows are read before the score product, so their shared-memory latency overlaps the
      // MMAs and the softmax instead of following them, and the score product sums its k-steps
      // into two accumulators (even and odd), halving its chain of dependent MMAs.
      constexpr bool kEarlyV = KV8 && NCH == 1 && !CAS;
      // The 16-bit kernel splits its score chain the same way where it has registers to spare
      // (one n-tile, head_dim <= 128, outside a cascade).
      constexpr bool kTwoAcc = kEarlyV || (!KV8 && !CAS && NT == 1 && D <= 128);
      uint4 v_early[4];
      if constexpr (kEarlyV) load_v(0, v_early);

      // S = K . Q^T : [16 tokens x 8 heads] per n-tile.
      float sc[NT][4], sc_odd[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[nt][e] = sc_odd[nt][e] = 0.0f;
      }
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        const int ra = stage_row(g, ht * NCH + c);      // token g
        const int rb = stage_row(g + 8, ht * NCH + c);  // token g + 8
#pragma unroll
        for (int par = 0; par < 2; ++par) {
          const int u = par * 4 + t4;
          const uint4 x = lds128(sk + ra * 128 + ((u ^ (ra & 7)) << 4));
          const uint4 y = lds128(sk + rb * 128 + ((u ^ (rb & 7)) << 4));
          if constexpr (!KV8) {
            const int j0 = 4 * c + 2 * par;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              Mma<MT>::run(sc[nt], x.x, y.x, x.y, y.y, qf[j0][nt][0], qf[j0][nt][1]);
              Mma<MT>::run(kTwoAcc ? sc_odd[nt] : sc[nt], x.z, y.z, x.w, y.w, qf[j0 + 1][nt][0], qf[j0 + 1][nt][1]);
            }
          } else {
            // 16 e4m3 of d = 128c + 64par + 16t4 + 4jj + {0,1 | 2,3} feed k-step 8c + 4par + jj.
            const uint32_t xw[4] = {x.x, x.y, x.z, x.w}, yw[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
              const uint32_t a0 = e4m3x2_lo_to_f16x2(xw[jj]), a2 = e4m3x2_hi_to_f16x2(xw[jj]);
              const uint32_t a1 = e4m3x2_lo_to_f16x2(yw[jj]), a3 = e4m3x2_hi_to_f16x2(yw[jj]);
              const int j = 8 * c + 4 * par + jj;
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) {
                Mma<MT>::run((kTwoAcc && (jj & 1)) ? sc_odd[nt] : sc[nt], a0, a1, a2, a3, qf[j][nt][0], qf[j][nt][1]);
              }
            }
          }
        }
      }
      if constexpr (kTwoAcc) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
          for (int e = 0; e < 4; ++e) sc[nt][e] += sc_odd[nt][e];
        }
      }

      // Online softmax in base 2. Lane holds tokens g and g+8 of heads 2*t4 and 2*t4+1.
      const bool row0 = g < valid, row1 = g + 8 < valid;
      uint32_t pb[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[nt][e] *= sl_h;
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
            Storage<MT>::pack2(fast_exp2(sc[nt][0] - m_run[nt][0]), fast_exp2(sc[nt][1] - m_run[nt][1]));
        const uint32_t p23 =
            Storage<MT>::pack2(fast_exp2(sc[nt][2] - m_run[nt][0]), fast_exp2(sc[nt][3] - m_run[nt][1]));
        // The normaliser sums the rounded probabilities the MMA actually uses.
        const float2 f01 = Storage<MT>::unpack2(p01), f23 = Storage<MT>::unpack2(p23);
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

      // O^T += V^T . P^T ; V rows past the valid tokens are zeroed, never multiplied.
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        uint4 v[4];
        if constexpr (kEarlyV) {
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) v[q4] = v_early[q4];
        } else {
          load_v(c, v);
        }
        const uint32_t va[4] = {v[0].x, v[0].y, v[0].z, v[0].w};
        const uint32_t vb[4] = {v[1].x, v[1].y, v[1].z, v[1].w};
        const uint32_t vc[4] = {v[2].x, v[2].y, v[2].z, v[2].w};
        const uint32_t vd[4] = {v[3].x, v[3].y, v[3].z, v[3].w};
#pragma unroll
        for (int mt = 0; mt < OW / 2; ++mt) {
          // m-tile c*OW/2 + mt: row g holds d = 8*OW*c + OW*g + 2mt (the lane's output value 2mt
          // of piece c), row g + 8 holds d + 1; columns are tokens 2t4, 2t4+1, 2t4+8, 2t4+9.
          uint32_t a0, a1, a2, a3;
          if constexpr (!KV8) {
            a0 = __byte_perm(va[mt], vb[mt], 0x5410);
            a1 = __byte_perm(va[mt], vb[mt], 0x7632);
            a2 = __byte_perm(vc[mt], vd[mt], 0x5410);
            a3 = __byte_perm(vc[mt], vd[mt], 0x7632);
          } else {
            // Pair the two tokens' bytes first, (tok0 d, tok1 d, tok0 d+1, tok1 d+1); one
            // conversion per register then yields the fragment.
            const uint32_t sel = (mt & 1) ? 0x7362u : 0x5140u;
            const uint32_t x01 = __byte_perm(va[mt >> 1], vb[mt >> 1], sel);
            const uint32_t x23 = __byte_perm(vc[mt >> 1], vd[mt >> 1], sel);
            a0 = e4m3x2_lo_to_f16x2(x01);
            a1 = e4m3x2_hi_to_f16x2(x01);
            a2 = e4m3x2_lo_to_f16x2(x23);
            a3 = e4m3x2_hi_to_f16x2(x23);
          }
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            Mma<MT>::run(acc[c * (OW / 2) + mt][nt], a0, a1, a2, a3, pb[nt][0], pb[nt][1]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bars + 8u * (nstage + stage));
    }
    gt += ntiles;

    // Per-head normaliser over the 8 token-row groups of the fragments.
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

    // Lane (g, t4) owns, for head hl = nt*8 + 2*t4 + e and piece c, output d = 8*OW*c + OW*g + k,
    // k = 0..OW-1, held in acc[c*OW/2 + k/2][nt][e + 2*(k & 1)].
    // Shared ring with TW > 1: the warps that split the tiles of one (head, group) combine into
    // the tw == 0 warp.
    if (NS == 1 && TW > 1) {
      if (tw != 0) {
        const int slot_w = warp - HT * HG;  // warps with tw >= 1, in order
        float* rm = red_m + slot_w * HPW;
        float* rl = red_l + slot_w * HPW;
        float* ra = red_acc + slot_w * HPW * (D + 4);
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
            for (int c = 0; c < NCH; ++c) {
              float* dst = ra + hl * (D + 4) + c * 8 * OW + OW * g;
#pragma unroll
              for (int k = 0; k < OW; ++k) dst[k] = acc[c * (OW / 2) + (k >> 1)][nt][e + 2 * (k & 1)];
            }
          }
        }
      }
      named_barrier(1 + mu, TW * 32);
      if (tw == 0) {
        // The combine slot of warp (ht, hg, t2 >= 1) is its warp index less HT * HG, i.e.
        // (hg * HT + ht) + HT * HG * (t2 - 1): the (head, group) order of the warp index, which is
        // not mu's (ht * HG + hg) when a tile has two or more heads and two or more groups.
        const int wl = warp % (HT * HG);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int hl = nt * 8 + 2 * t4 + e;
            float M = m_run[nt][e];
            for (int t2 = 1; t2 < TW; ++t2) M = fmaxf(M, red_m[(wl + HT * HG * (t2 - 1)) * HPW + hl]);
            if (M == -INFINITY) continue;
            const float f0 = fast_exp2(m_run[nt][e] - M);
            float l = l_run[nt][e] * f0;
#pragma unroll
            for (int mt = 0; mt < KS; ++mt) {
              acc[mt][nt][e] *= f0;
              acc[mt][nt][2 + e] *= f0;
            }
            for (int t2 = 1; t2 < TW; ++t2) {
              const int w2 = wl + HT * HG * (t2 - 1);  // combine slot of warp (ht, hg, t2)
              const float m2 = red_m[w2 * HPW + hl];
              if (m2 == -INFINITY) continue;
              const float f = fast_exp2(m2 - M);
              l += red_l[w2 * HPW + hl] * f;
              const float* src = red_acc + (w2 * HPW + hl) * (D + 4);
#pragma unroll
              for (int c = 0; c < NCH; ++c) {
#pragma unroll
                for (int k = 0; k < OW; ++k) {
                  acc[c * (OW / 2) + (k >> 1)][nt][e + 2 * (k & 1)] += src[c * 8 * OW + OW * g + k] * f;
                }
              }
            }
            m_run[nt][e] = M;
            l_run[nt][e] = l;
          }
        }
      }
      named_barrier(1 + mu, TW * 32);
      if (tw != 0) continue;
    }

    // ---- emit: the final output, or this chunk's partial and (if last) the merge.
    RowSink sink;
    sink.seq = s.seq;
    sink.nmem = s.nmem;
    sink.kvh = kvh;
    sink.row0 = hg * HPW;
    sink.side = s.grp >= 0 ? 0 : 1;
    sink.cas = 0u;
    if (CAS) {
      // Members with both a shared prefix and tokens of their own: this entry is one side of
      // their cascade, merged with the other side by whichever finishes second.
      const bool both = lane < s.nmem && (s.grp >= 0 ? ps.lens[w.V + s.seq + lane] > 0 : ps.hp[s.seq] > 0);
      sink.cas = __ballot_sync(0xffffffffu, both);
    }
    const int nh_warp = min(HPW, s.nmem * G - hg * HPW);  // this warp's rows that are not padding
    const int nh_member = min(HPW, G - hg * HPW);         // one member's rows in this warp's group
    if (s.whole) {
      float inv[NT][2], lse[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float l = l_run[nt][e];
          inv[nt][e] = l > 0.0f ? v_scale / l : 0.0f;
          lse[nt][e] = l > 0.0f ? m_run[nt][e] + __log2f(l) : -INFINITY;
        }
      }
      store_rows<T, D, NT, OW, CAS, GATHER>(a, sink, acc, inv, lse, g, t4, nh_warp);
      if (CAS && sink.cas != 0u) cascade_arrive<T, D>(a, sink, hg, hg * HPW, nh_member, lane);
      continue;
    }
    // This chunk's normalised partial and base-2 LSE, in the fragment layout; padding heads of
    // the last query-head group are never written nor read.
    float lse_own[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float l = l_run[nt][e];
        const float inv = l > 0.0f ? v_scale / l : 0.0f;
        lse_own[nt][e] = l > 0.0f ? m_run[nt][e] + __log2f(l) : -INFINITY;
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
          acc[mt][nt][e] *= inv;
          acc[mt][nt][e + 2] *= inv;
        }
      }
    }
    // Few chunks: the last one merges from its registers (written only if it must publish).
    // Many: every chunk writes its partial and the last merges them all with the flat merge.
    const bool flat = s.nchunks > kRegisterMergeChunks;
    uint32_t* counter = counter_of(a, s.cb, kvh, hg);
    const uint32_t siblings = static_cast<uint32_t>(s.nchunks - 1);
    bool last = __shfl_sync(0xffffffffu, published, 0) == siblings;
    if (flat || !last) {
      const int64_t slot = static_cast<int64_t>(s.chunk) * (HT * HG) + mu;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int hl = nt * 8 + 2 * t4 + e;
          if (hl >= nh_warp) continue;
          float* po = a.part_o + (slot * HPW + hl) * D;
#pragma unroll
          for (int c = 0; c < NCH; ++c) {
            float4* dst = reinterpret_cast<float4*>(po + c * 8 * OW + OW * g);
#pragma unroll
            for (int h = 0; h < OW / 4; ++h) {
              const int m0 = c * (OW / 2) + 2 * h;
              dst[h] = make_float4(acc[m0][nt][e], acc[m0][nt][e + 2], acc[m0 + 1][nt][e], acc[m0 + 1][nt][e + 2]);
            }
          }
          if (g == 0) a.part_lse[slot * HPW + hl] = lse_own[nt][e];
        }
      }
      // The warp barrier orders every lane's stores before what follows: the flat merge's
      // reads by this warp, and lane 0's count (a release) otherwise.
      __syncwarp();
    }
    if (!last) {
      uint32_t before = 0;
      if (lane == 0) before = atom_add_acq_rel_gpu(counter, 1u);  // publish; acquire if last
      last = __shfl_sync(0xffffffffu, before, 0) == siblings;
      if (!last) continue;
    } else if (lane == 0) {
      fence_acq_rel_gpu();  // acquire what the siblings published before the count was read
    }
    __syncwarp();
    if (flat) {
      merge_chunks<T, D, HPW, CAS, GATHER>(a, s, HT * HG, mu, nh_warp, sink, lane);
    } else {
      // Merge in chunk order with a running max, this chunk's own term from its registers (the
      // values it would have stored), so the result does not depend on which chunk merges; a
      // sibling's loads are all issued before any of its arithmetic.
      float m_acc[NT][2], w_acc[NT][2], o_acc[KS][NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        m_acc[nt][0] = m_acc[nt][1] = -INFINITY;
        w_acc[nt][0] = w_acc[nt][1] = 0.0f;
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) o_acc[mt][nt][0] = o_acc[mt][nt][1] = o_acc[mt][nt][2] = o_acc[mt][nt][3] = 0.0f;
      }
      for (int k = 0; k < s.nchunks; ++k) {
        const int ck = chunk_id(a, s, k);
        const bool own = ck == s.chunk;
        const int64_t slot2 = static_cast<int64_t>(ck) * (HT * HG) + mu;
        // Heads whose loads are in flight together: both of a lane's heads when registers allow.
        constexpr int EG = NT * NCH <= 2 ? 2 : 1;
#pragma unroll
        for (int ne = 0; ne < NT * 2; ne += EG) {
          const int nt = ne / 2;
          float lse[EG];
          float4 x[EG][NCH][OW / 4];
#pragma unroll
          for (int ei = 0; ei < EG; ++ei) {
            const int e = ne % 2 + ei;
            const int hl = nt * 8 + 2 * t4 + e;
            const bool ld = !own && hl < nh_warp;
            const float* po = a.part_o + (slot2 * HPW + hl) * D;
            lse[ei] = own ? lse_own[nt][e] : ld ? __ldcg(a.part_lse + slot2 * HPW + hl) : -INFINITY;
#pragma unroll
            for (int c = 0; c < NCH; ++c) {
#pragma unroll
              for (int h = 0; h < OW / 4; ++h) {
                const float* lo = &acc[c * (OW / 2) + 2 * h][nt][0];
                const float* hi = &acc[c * (OW / 2) + 2 * h + 1][nt][0];
                x[ei][c][h] = own ? make_float4(lo[e], lo[e + 2], hi[e], hi[e + 2])
                            : ld  ? __ldcg(reinterpret_cast<const float4*>(po + c * 8 * OW + OW * g + 4 * h))
                                  : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
              }
            }
          }
#pragma unroll
          for (int ei = 0; ei < EG; ++ei) {
            const int e = ne % 2 + ei;
            const float mn = fmaxf(m_acc[nt][e], lse[ei]);
            if (mn == -INFINITY) continue;
            const float fa = fast_exp2(m_acc[nt][e] - mn), fb = fast_exp2(lse[ei] - mn);
            m_acc[nt][e] = mn;
            w_acc[nt][e] = w_acc[nt][e] * fa + fb;
#pragma unroll
            for (int c = 0; c < NCH; ++c) {
#pragma unroll
              for (int h = 0; h < OW / 4; ++h) {
                float* lo = &o_acc[c * (OW / 2) + 2 * h][nt][0];
                float* hi = &o_acc[c * (OW / 2) + 2 * h + 1][nt][0];
                lo[e] = lo[e] * fa + fb * x[ei][c][h].x;
                lo[e + 2] = lo[e + 2] * fa + fb * x[ei][c][h].y;
                hi[e] = hi[e] * fa + fb * x[ei][c][h].z;
                hi[e + 2] = hi[e + 2] * fa + fb * x[ei][c][h].w;
              }
            }
          }
        }
      }
      float inv[NT][2], lse[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float wsum = w_acc[nt][e];
          inv[nt][e] = wsum > 0.0f ? 1.0f / wsum : 0.0f;
          lse[nt][e] = wsum > 0.0f ? m_acc[nt][e] + __log2f(wsum) : -INFINITY;
        }
      }
      store_rows<T, D, NT, OW, CAS, GATHER>(a, sink, o_acc, inv, lse, g, t4, nh_warp);
    }
    if (CAS && sink.cas != 0u) cascade_arrive<T, D>(a, sink, hg, hg * HPW, nh_member, lane);
    // Every sibling has counted (or none needed to): nobody else touches the counter in this
    // launch, so a plain store returns it to zero for the next one.
    if (lane == 0) *reinterpret_cast<volatile uint32_t*>(counter) = 0u;
  }
  if constexpr (GATHER) gather_finish(a, kCW * 32);
}

// ------------------------------------------------------------------------- tensor-core prefix kernel
//
// The shared-prefix half of a cascade on the 5th-generation tensor cores. A prefix's keys are
// read by every sequence of its group, so its attention is a real matrix product: 128 query rows
// (128 / group sequences of one group, all query heads of one KV head) against the prefix's keys.
// One CTA takes one segment: (member block of 128 rows, KV head, up to kPrefixChunksMax
// consecutive chunks of kPrefixTokens tokens). Q is loaded once; K and V of the chunks stream
// through two shared-memory stages, the next chunk's loads in flight during the current chunk's
// work. Per chunk:
//   one thread issues S = Q.K^T (M = 128 rows, N = 128 tokens, K = head_dim) into TMEM;
//   two warpgroups split every row (TMEM lane) by columns, one thread per half row: the chunk's
//   row maximum (the halves exchange theirs), the online softmax with a lazy rescale (O in TMEM is
//   rescaled only when a row's maximum grows by more than 2^8, so the exponentials stay below 2^8
//   otherwise), P written to shared memory as the next A operand;
//   one thread issues O += P.V (N = head_dim, K = chunk tokens; V as an MN-major operand).
// tcgen05 operations of one thread complete in issue order, so once S of chunk j has completed,
// O += P.V of chunk j-1 has too: the rescale and the reuse of its stage need no further wait.
// Each row is then normalised and stored, with its base-2 LSE, as prefix plane `segment` of the
// row's sequence; cascade_prefix_reduce_kernel collapses a prefix's planes.

constexpr int kPrefixTokens = 128;    // tokens of one chunk: the N of S = Q.K^T, the K of O = P.V
constexpr int kPrefixThreads = 256;   // two warpgroups: each row's columns split between them
constexpr int kPrefixChunksMax = 8;   // chunks of one CTA's segment, at most
constexpr float kLazyRescale = 8.0f;  // log2 headroom before O is rescaled

struct PrefixLayout {
  uint32_t q, k[2], v[2], p[2], bars, tptr, ints, total;
};

// Q [NH][128 rows x 128 B]; stage s: K and V [NH][128 tokens x 128 B]. P (128 rows x 128 tokens)
// overwrites its stage's K once S has been computed when it fits (head_dim 128), otherwise it
// has its own buffer per stage.
__host__ __device__ __forceinline__ PrefixLayout prefix_layout(int D) {
  constexpr uint32_t CT = kPrefixTokens;
  const uint32_t nh = D / 64;
  const uint32_t kv = nh * CT * 128u;
  const uint32_t pbytes = 128u * CT * 2u;
  PrefixLayout L{};
  uint32_t off = nh * 128u * 128u;
  L.q = 0;
  for (int s = 0; s < 2; ++s) {
    L.k[s] = off;
    off += kv;
    L.v[s] = off;
    off += kv;
  }
  for (int s = 0; s < 2; ++s) {
    if (kv >= pbytes) {
      L.p[s] = L.k[s];
    } else {
      L.p[s] = off;
      off += pbytes;
    }
  }
  L.bars = off;
  L.tptr = off + 64u;
  L.ints = off + 128u;
  L.total = L.ints + 1536u * 4u + 1024u;  // + slack to align the base to 1024 B
  return L;
}

template <typename T, int D>
__global__ void __launch_bounds__(kPrefixThreads, 1) cascade_prefix_kernel(const __grid_constant__ CUtensorMap tmq,
                                                                           const __grid_constant__ CUtensorMap tmk,
                                                                           const __grid_constant__ CUtensorMap tmv,
                                                                           const __grid_constant__ DecodeArgs a) {
  constexpr int CT = kPrefixTokens;
  constexpr int NH = D / 64;                  // 128-byte column blocks of a head row
  constexpr uint32_t QH = 128u * 128u;        // one column block of Q: 128 rows
  constexpr uint32_t KH = CT * 128u;          // one column block of K or V: CT token rows
  constexpr uint32_t PH = 128u * 128u;        // one 64-token column block of P: 128 rows
  constexpr uint32_t NCOL = 256u;             // S: columns 0..127, O: 128..128+D-1
  static_assert(CT + D <= 256, "S and O share 256 TMEM columns");
  constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t IDESC_S = umma_idesc_f16(BF16, 128, CT, false);
  constexpr uint32_t IDESC_O = umma_idesc_f16(BF16, 128, D, true);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const PrefixLayout L = prefix_layout(D);
  const uint32_t base = smem_u32(smem);
  const uint32_t sq = base + L.q;
  const uint32_t bq = base + L.bars, bs = bq + 8, bo = bq + 16;  // Q landed, S done, O += P.V done
  auto bk = [&](int s) { return bq + 24u + 8u * s; };           // stage s: K landed
  auto bv = [&](int s) { return bq + 40u + 8u * s; };           // stage s: V landed
  int* ints = reinterpret_cast<int*>(smem + L.ints);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = a.group, B = a.batch, P = a.page_size;
  const int Mb = 128 / G;
  const int seg = blockIdx.x, kvh = blockIdx.y;
  const int nseg_chunks = a.prefix_chunk / CT;  // chunks per segment

  // Launched with programmatic stream serialization: nothing global is touched before the
  // previous kernel in the stream (possibly the previous call, which shares the prefix planes)
  // has completed.
  wait_prior_grid();
  // ---- member block blockIdx.z: its group (a block scan over the groups' block counts)
  {
    const int ngrp = a.num_prefixes;
    const int per = (ngrp + kPrefixThreads - 1) / kPrefixThreads;
    const int lo = min(ngrp, tid * per), hi = min(ngrp, lo + per);
    int local = 0;
    bool bad = false;
    for (int p = lo; p < hi; ++p) {
      const int i0 = __ldg(a.prefix_indptr + p), i1 = __ldg(a.prefix_indptr + p + 1);
      bad |= i0 > i1 || (p == 0 && i0 != 0) || (p == ngrp - 1 && i1 != B);
      local += i1 > i0 ? (i1 - i0 + Mb - 1) / Mb : 0;
    }
    if (__syncthreads_or(bad)) return;  // the decode kernel reports it and ignores the prefixes
    ints[tid] = local;
    if (tid == 0) ints[560] = -1;
    __syncthreads();
    block_scan(kPrefixThreads, [&](int i) { return ints[i]; }, ints + 256, ints + 520);
    const int first = ints[256 + tid];
    const int z = blockIdx.z;
    if (z >= first && z < first + local) {
      int acc = first;
      for (int p = lo; p < hi; ++p) {
        const int i0 = __ldg(a.prefix_indptr + p), i1 = __ldg(a.prefix_indptr + p + 1);
        const int nb = i1 > i0 ? (i1 - i0 + Mb - 1) / Mb : 0;
        if (z < acc + nb) {
          const int b0 = i0 + (z - acc) * Mb;
          ints[560] = p;
          ints[561] = b0;
          ints[562] = min(Mb, i1 - b0);
          break;
        }
        acc += nb;
      }
    }
    __syncthreads();
  }
  const int grp = ints[560];
  if (grp < 0) return;
  const int b0 = ints[561], nmem = ints[562];
  const int plen = clamp_prefix_len(a, grp, false);
  const int tok_seg = seg * nseg_chunks * CT;
  if (tok_seg >= plen) return;
  const int seg_tokens = min(nseg_chunks * CT, plen - tok_seg);
  const int nchunk = (seg_tokens + CT - 1) / CT;
  const int nplanes = prefix_planes(a, plen);
  const int npg = (seg_tokens + P - 1) / P;  // pages of the segment (CT is a multiple of the page size)
  const int pages_per_chunk = CT / P;

  // One parallel round of small loads: the segment's page ids (-1: outside the pool) and the
  // block's sequences' own lengths.
  int* s_own = ints + 576;   // up to 128 lengths: 576..703
  int* s_page = ints + 704;  // up to kPrefixChunksMax * CT / 8 = 128 pages: 704..831
  float* s_half = reinterpret_cast<float*>(ints + 832);  // [2 halves][128 rows]: chunk max, then row sum
  for (int i = tid; i < npg; i += kPrefixThreads) {
    const int page = __ldg(a.prefix_bt + static_cast<int64_t>(grp) * a.prefix_bt_stride + tok_seg / P + i);
    s_page[i] = (page < 0 || (a.num_pages >= 0 && page >= a.num_pages)) ? -1 : page;
  }
  if (tid < nmem) s_own[tid] = clamp_len(a, b0 + tid, false);
  if (tid == 0) {
    mbar_init(bq, 1);
    mbar_init(bs, 1);
    mbar_init(bo, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(bk(s), 1);
      mbar_init(bv(s), 1);
    }
    fence_barrier_init();
  }
  __syncwarp();  // tcgen05.alloc is .sync.aligned: the whole warp, converged
  if (warp == 0) {
    tmem_alloc(base + L.tptr, NCOL);
    tmem_relinquish();
  }
  tcgen05_fence_before();
  __syncthreads();
  tcgen05_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + L.tptr);
  const uint32_t tS = tmem, tO = tmem + CT;
  // Pages outside the pool are skipped (flagged). Their rows would hold whatever the stage held
  // before, so when the segment has any, both stages start zeroed.
  bool anybad = false;
  for (int i = tid; i < npg; i += kPrefixThreads) anybad |= s_page[i] < 0;
  if (__syncthreads_or(anybad)) {
    if (tid == 0) atomicOr(a.sync, kStatusBadPage);
    for (int s = 0; s < 2; ++s) {
      for (uint32_t off = tid * 16u; off < NH * KH; off += kPrefixThreads * 16u) {
        sts128(base + L.k[s] + off, make_uint4(0u, 0u, 0u, 0u));
        sts128(base + L.v[s] + off, make_uint4(0u, 0u, 0u, 0u));
      }
    }
    fence_proxy_async_smem();
    __syncthreads();
  }

  // Warp 0 issues chunk j's loads into stage j & 1: lane i takes the chunk's page i.
  const uint64_t pol = l2_policy_evict_normal();
  auto issue_chunk = [&](int j) {
    const int s = j & 1;
    const int pg = j * pages_per_chunk + lane;
    const int page = lane < pages_per_chunk && pg < npg ? s_page[pg] : -1;
    const uint32_t nvalid = static_cast<uint32_t>(__popc(__ballot_sync(0xffffffffu, page >= 0)));
    if (lane == 0) {
      mbar_arrive_expect_tx(bk(s), nvalid * NH * P * 128u);
      mbar_arrive_expect_tx(bv(s), nvalid * NH * P * 128u);
    }
    __syncwarp();
    if (page >= 0) {
#pragma unroll
      for (int h = 0; h < NH; ++h) {
        tma_load_3d(base + L.k[s] + h * KH + lane * P * 128u, &tmk, 0, kvh * NH + h, page * P, bk(s), pol);
      }
#pragma unroll
      for (int h = 0; h < NH; ++h) {
        tma_load_3d(base + L.v[s] + h * KH + lane * P * 128u, &tmv, 0, kvh * NH + h, page * P, bv(s), pol);
      }
    }
  };
  if (warp == 0) {
    if (lane == 0) mbar_arrive_expect_tx(bq, NH * QH);
    __syncwarp();
    if (lane < NH) tma_load_3d(sq + lane * QH, &tmq, lane * 64, kvh * G, b0, bq, pol);
    issue_chunk(0);
  }

  // Thread tid works on row rw = tid % 128 (TMEM lane; warp w reads lanes 32 * (w % 4) ..) and
  // on half hf = tid / 128 of that row's columns: S columns hf * CT/2 .., P's 64-token block hf,
  // O columns hf * D/2 ... The halves share the chunk maximum (so both make the same rescale
  // decision) and add their row sums at the end.
  const int rw = tid & 127, hf = tid >> 7;
  constexpr int SC = CT / 2, OC = D / 2;  // S and O columns per half
  static_assert(SC == 64, "a half's S columns are one 64-token block of P");
  const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
  const float sl = a.scale_log2;
  float m_used = -INFINITY, lsum = 0.0f;
  bool ok = true;
  int j_last = 0;  // the last chunk whose loads were issued and waited for
  // A wait that runs out (thread 0's Q or K, anyone's S, V or O) flags the launch. Every copy
  // already issued is still waited for (bounded) before the CTA may leave: no wait is skipped
  // after a failure, thread 0 issues no further chunk once one of its waits failed, and the CTA
  // leaves the loop, by one verdict, after that chunk's V has landed.
#pragma unroll 1
  for (int j = 0; j < nchunk; ++j) {
    const int s = j & 1;
    const int ntok = min(CT, seg_tokens - j * CT);
    j_last = j;
    if (tid == 0) {
      const bool gq = j > 0 || mbar_wait_bounded(bq, 0, a.sync, kWaitLimit);
      const bool gk = mbar_wait_bounded(bk(s), (j >> 1) & 1, a.sync, kWaitLimit);
      ok = ok && gq && gk;
      if (ok) {
        tcgen05_fence_after();
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t off = (ks % 4) * 32u;
          const uint64_t ad = umma_desc_sw128(sq + (ks / 4) * QH + off, 16u, 1024u);
          const uint64_t bd = umma_desc_sw128(base + L.k[s] + (ks / 4) * KH + off, 16u, 1024u);
          umma_f16(tS, ad, bd, IDESC_S, ks > 0 ? 1u : 0u);
        }
      }
      umma_commit(bs);
    }
    // The other stage is free once O += P.V of chunk j - 1 has completed, which the completion of
    // S of chunk j implies; warp 0 then starts chunk j + 1's loads.
    ok = mbar_wait_bounded(bs, j & 1, a.sync, kWaitLimit) && ok;
    tcgen05_fence_after();
    if (warp == 0) {
      const bool lead_ok = __shfl_sync(0xffffffffu, ok, 0);  // thread 0's waits so far
      if (j + 1 < nchunk && lead_ok) issue_chunk(j + 1);
    }

    // ---- this thread's half row of S: the chunk's maximum, a lazy rescale, P
    uint32_t sr[SC / 32][32];
    __syncwarp();  // tcgen05.ld is .sync.aligned
#pragma unroll
    for (int cc = 0; cc < SC / 32; ++cc) tmem_ld32(tS + lane_base + hf * SC + cc * 32, sr[cc]);
    tmem_wait_ld();
    // Every chunk but a prefix's last is full: its softmax runs without the per-column masks.
    // The operations are the same; the compiler may fuse a multiply and a subtraction
    // differently in the two bodies, so the outputs can differ in the last bit.
    const bool full = ntok == CT;
    auto half_max = [&](auto all_valid) {
      float m = -INFINITY;
#pragma unroll
      for (int cc = 0; cc < SC / 32; ++cc) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if (decltype(all_valid)::value || hf * SC + cc * 32 + i < ntok) m = fmaxf(m, __uint_as_float(sr[cc][i]) * sl);
        }
      }
      return m;
    };
    float mc = full ? half_max(std::true_type{}) : half_max(std::false_type{});
    s_half[hf * 128 + rw] = mc;
    // One verdict for the CTA: thread 0's ok is the one warp 0 used to decide on chunk j + 1.
    const bool stop = __syncthreads_or(tid == 0 && !ok);
    mc = fmaxf(s_half[rw], s_half[128 + rw]);
    float alpha = 1.0f;
    if (mc > m_used + kLazyRescale) {  // also the first chunk, where m_used = -inf
      alpha = m_used == -INFINITY ? 0.0f : fast_exp2(m_used - mc);
      m_used = mc;
      lsum *= alpha;
    }
    if (j > 0 && __any_sync(0xffffffffu, alpha < 1.0f)) {
      // O (complete up to chunk j - 1) *= alpha for this warp's rows and half, through registers.
#pragma unroll 1
      for (int cc = 0; cc < OC / 32; ++cc) {
        uint32_t r[32];
        tmem_ld32(tO + lane_base + hf * OC + cc * 32, r);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
        tmem_st32(tO + lane_base + hf * OC + cc * 32, r);
      }
      tmem_wait_st();
    }
    const uint32_t sp = base + L.p[s];
    auto write_p = [&](auto all_valid) {
      constexpr bool kAll = decltype(all_valid)::value;
      float l_even = 0.0f, l_odd = 0.0f;  // the chunk's even and odd columns, summed apart
#pragma unroll
      for (int cc = 0; cc < SC / 32; ++cc) {
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {  // 8 tokens: one 16-byte unit of P's row
          uint32_t w[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int t0 = hf * SC + cc * 32 + q8 * 8 + 2 * u;
            const float s0 = __uint_as_float(sr[cc][q8 * 8 + 2 * u]) * sl;
            const float s1 = __uint_as_float(sr[cc][q8 * 8 + 2 * u + 1]) * sl;
            const float p0 = (kAll || t0 < ntok) ? fast_exp2(s0 - m_used) : 0.0f;
            const float p1 = (kAll || t0 + 1 < ntok) ? fast_exp2(s1 - m_used) : 0.0f;
            w[u] = Storage<T>::pack2(p0, p1);
            add_pair_to<T>(w[u], l_even, l_odd);  // the normaliser sums what the MMA uses
          }
          const uint32_t unit = static_cast<uint32_t>(cc * 4 + q8) ^ static_cast<uint32_t>(rw & 7);
          sts128(sp + hf * PH + rw * 128u + (unit << 4), make_uint4(w[0], w[1], w[2], w[3]));
        }
      }
      lsum += l_even + l_odd;
    };
    if (full) {
      write_p(std::true_type{});
    } else {
      write_p(std::false_type{});
    }
    // V rows past the chunk's tokens (a page's tail) are zeroed: P is zero there, but 0 * NaN is not.
    ok = mbar_wait_bounded(bv(s), (j >> 1) & 1, a.sync, kWaitLimit) && ok;
    for (int i = tid; i < NH * (CT - ntok) * 8; i += kPrefixThreads) {
      const int h = i / ((CT - ntok) * 8), r = ntok + (i / 8) % (CT - ntok), u = i % 8;
      sts128(base + L.v[s] + h * KH + r * 128u + u * 16u, make_uint4(0u, 0u, 0u, 0u));
    }
    fence_proxy_async_smem();
    tcgen05_fence_before();
    __syncthreads();
    if (tid == 0) {
      tcgen05_fence_after();
      if (ok) {
        // O += P . V: K = chunk tokens in steps of 16; A = P (K-major, 64-token column blocks),
        // B = V as an MN-major operand (rows = tokens, 64-element column blocks KH bytes apart).
#pragma unroll
        for (int ks = 0; ks < CT / 16; ++ks) {
          const uint64_t ad = umma_desc_sw128(sp + (ks / 4) * PH + (ks % 4) * 32u, 16u, 1024u);
          const uint64_t bd = umma_desc_sw128(base + L.v[s] + ks * 16u * 128u, KH, 1024u);
          umma_f16(tO, ad, bd, IDESC_O, (j > 0 || ks > 0) ? 1u : 0u);
        }
      }
      umma_commit(bo);
    }
    if (stop) break;  // chunk j + 1 was not issued
  }
  ok = mbar_wait_bounded(bo, j_last & 1, a.sync, kWaitLimit) && ok;
  s_half[hf * 128 + rw] = lsum;
  ok = __syncthreads_and(ok);  // one verdict for the CTA (only thread 0 waited on the loads)
  lsum = s_half[rw] + s_half[128 + rw];  // the two halves' sums, in a fixed order
  tcgen05_fence_after();
  allow_next_grid();  // the reduce kernel may start launching (it waits for this grid's stores)

  // ---- epilogue: row tid = member m, query head gi of KV head kvh. A sequence whose prefix is
  // this one segment and that has no tokens of its own gets its final output here; otherwise the
  // row becomes prefix plane `seg` (collapsed by cascade_prefix_reduce_kernel when the prefix has
  // several, merged with the sequence's own tokens by the decode kernel).
  const int m = rw / G, gi = rw - m * G;
  const bool valid = ok && m < nmem;
  const bool direct = valid && nplanes == 1 && s_own[m] == 0;
  const int64_t row = static_cast<int64_t>(b0 + m) * a.num_q_heads + kvh * G + gi;
  const float inv = lsum > 0.0f ? 1.0f / lsum : 0.0f;
  const float lse = lsum > 0.0f ? m_used + __log2f(lsum) : -INFINITY;
  uint32_t orr[OC / 32][32];
  __syncwarp();  // tcgen05.ld is .sync.aligned
#pragma unroll
  for (int cc = 0; cc < OC / 32; ++cc) tmem_ld32(tO + lane_base + hf * OC + cc * 32, orr[cc]);
  tmem_wait_ld();
#pragma unroll
  for (int cc = 0; cc < OC / 32; ++cc) {
    const uint32_t(&r)[32] = orr[cc];
    if (!valid) continue;
    if (direct) {
      T* dst = static_cast<T*>(a.out) + row * D + hf * OC + cc * 32;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 pk;
        pk.x = Storage<T>::pack2(__uint_as_float(r[8 * q + 0]) * inv, __uint_as_float(r[8 * q + 1]) * inv);
        pk.y = Storage<T>::pack2(__uint_as_float(r[8 * q + 2]) * inv, __uint_as_float(r[8 * q + 3]) * inv);
        pk.z = Storage<T>::pack2(__uint_as_float(r[8 * q + 4]) * inv, __uint_as_float(r[8 * q + 5]) * inv);
        pk.w = Storage<T>::pack2(__uint_as_float(r[8 * q + 6]) * inv, __uint_as_float(r[8 * q + 7]) * inv);
        reinterpret_cast<uint4*>(dst)[q] = pk;
      }
    } else {
      float4* dst = reinterpret_cast<float4*>(
          a.cas_o + (static_cast<int64_t>(seg) * B * a.num_q_heads + row) * D + hf * OC + cc * 32);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        dst[q] = make_float4(__uint_as_float(r[4 * q]) * inv, __uint_as_float(r[4 * q + 1]) * inv,
                             __uint_as_float(r[4 * q + 2]) * inv, __uint_as_float(r[4 * q + 3]) * inv);
      }
    }
  }
  if (valid && !direct && hf == 0) a.cas_lse[static_cast<int64_t>(seg) * B * a.num_q_heads + row] = lse;
  tcgen05_fence_before();
  __syncthreads();  // every TMEM read done
  if (warp == 0) {
    __syncwarp();
    tmem_dealloc(tmem, NCOL);
  }
}

// Collapses the prefix planes (segments) of every sequence whose group's prefix has several into
// plane 0 (output and LSE); a sequence without tokens of its own gets its final output instead.
// Runs between the prefix kernel and the decode kernel. A thread owns one float4 column of one
// query row (head_dim / 4 threads a row, all in one warp) and walks the planes in order with a
// running maximum, eight planes' loads in flight; the row's threads have read every LSE before its
// one writer replaces plane 0's.
constexpr int kReduceThreads = 256;

template <typename T, int D>
__global__ void __launch_bounds__(kReduceThreads) cascade_prefix_reduce_kernel(const __grid_constant__ DecodeArgs a) {
  constexpr int Q = D / 4;
  static_assert(32 % Q == 0, "a query row's columns must sit in one warp");
  constexpr int KB = 8;
  wait_prior_grid();  // the prefix kernel's planes are complete and visible
  const int64_t rows = static_cast<int64_t>(a.batch) * a.num_q_heads;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * kReduceThreads + threadIdx.x;
  const int64_t row = min(i / Q, rows - 1);
  const int c4 = static_cast<int>(i % Q);
  const int b = static_cast<int>(row / a.num_q_heads);
  int lo = 0, hi = a.num_prefixes - 1;  // last group starting at or before b
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(a.prefix_indptr + mid) <= b) lo = mid; else hi = mid - 1;
  }
  const int nch = prefix_planes(a, clamp_prefix_len(a, lo, false));
  const bool work = i < rows * Q && nch > 1;
  const int64_t plane = rows;
  float mx = -INFINITY, wsum = 0.0f;
  float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  for (int k0 = 0; work && k0 < nch; k0 += KB) {
    float l[KB];
    float4 x[KB];
#pragma unroll
    for (int q = 0; q < KB; ++q) {
      const int k = k0 + q;
      l[q] = k < nch ? __ldcg(a.cas_lse + k * plane + row) : -INFINITY;
      x[q] = k < nch ? __ldcg(reinterpret_cast<const float4*>(a.cas_o + (k * plane + row) * D) + c4)
                     : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
#pragma unroll
    for (int q = 0; q < KB; ++q) {
      const float mn = fmaxf(mx, l[q]);
      if (mn == -INFINITY) continue;
      const float fa = fast_exp2(mx - mn), fb = fast_exp2(l[q] - mn);
      mx = mn;
      wsum = wsum * fa + fb;
      acc.x = acc.x * fa + fb * x[q].x;
      acc.y = acc.y * fa + fb * x[q].y;
      acc.z = acc.z * fa + fb * x[q].z;
      acc.w = acc.w * fa + fb * x[q].w;
    }
  }
  __syncwarp();  // every reader of the row's LSEs is done before its writer replaces plane 0's
  if (!work) return;
  const float inv = wsum > 0.0f ? 1.0f / wsum : 0.0f;
  if (clamp_len(a, b, false) == 0) {
    uint2 pk;
    pk.x = Storage<T>::pack2(acc.x * inv, acc.y * inv);
    pk.y = Storage<T>::pack2(acc.z * inv, acc.w * inv);
    *reinterpret_cast<uint2*>(static_cast<T*>(a.out) + row * D + 4 * c4) = pk;
    return;
  }
  reinterpret_cast<float4*>(a.cas_o + row * D)[c4] = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
  if (c4 == 0) a.cas_lse[row] = wsum > 0.0f ? mx + __log2f(wsum) : -INFINITY;
}

// ------------------------------------------------------------------------- generic kernel

struct GenLayout {
  uint32_t q, acc, p, m, l, alpha, rows, misc, prefix, lens, total;
};

__host__ __device__ __forceinline__ GenLayout gen_layout(int G, int D, int batch) {
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

// One CTA of 128 threads handles one (sequence, KV head) chunk at a time.
template <typename T>
__global__ void __launch_bounds__(kGenThreads) decode_generic_kernel(const __grid_constant__ DecodeArgs a) {
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
  PlanSmem ps;
  ps.misc = reinterpret_cast<int*>(gsmem + L.misc);
  ps.prefix = reinterpret_cast<int*>(gsmem + L.prefix);
  ps.lens = reinterpret_cast<int*>(gsmem + L.lens);
  ps.hp = nullptr;  // no cascade on this kernel
  ps.vstart = nullptr;
  int* misc = ps.misc;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  plan_build(a, ps);
  zero_empty_sequences<T, false>(a, ps.lens, nullptr, tid, kGenThreads);
  const int64_t tok_stride = static_cast<int64_t>(H) * D;
  T* out = static_cast<T*>(a.out);

  Walk w;
  walk_init(a, misc, w);
  Seg s;
  while (walk_next(a, ps, w, s)) {
    const int kvh = s.u;
    const T* qb = static_cast<const T*>(a.q) + (static_cast<int64_t>(s.seq) * a.num_q_heads + kvh * G) * D;
    for (int i = tid; i < G * D; i += kGenThreads) {
      q_s[i] = Storage<T>::load(qb[i]);
      acc_s[i] = 0.0f;
    }
    if (tid < G) {
      m_s[tid] = -INFINITY;
      l_s[tid] = 0.0f;
    }
    const T* kc = static_cast<const T*>(a.k_cache) + kvh * D;
    const T* vc = static_cast<const T*>(a.v_cache) + kvh * D;
    const int32_t* bt_row = a.block_table + static_cast<int64_t>(s.seq) * a.bt_stride;
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

    const int64_t out_row0 = static_cast<int64_t>(s.seq) * a.num_q_heads + kvh * G;
    if (s.whole) {
      for (int idx = tid; idx < G * D; idx += kGenThreads) {
        const int h = idx / D;
        const float l = l_s[h];
        out[out_row0 * D + idx] = Storage<T>::store(l > 0.0f ? acc_s[idx] / l : 0.0f);
      }
      __syncthreads();
      continue;
    }
    const int64_t slot = s.chunk;
    for (int idx = tid; idx < G * D; idx += kGenThreads) {
      const int h = idx / D, d = idx - h * D;
      const float l = l_s[h];
      a.part_o[(slot * G + h) * D + d] = l > 0.0f ? acc_s[idx] / l : 0.0f;
      if (d == 0) a.part_lse[slot * G + h] = l > 0.0f ? m_s[h] + __log2f(l) : -INFINITY;
    }
    // The block barrier orders every thread's stores before thread 0's count (a release);
    // the count's acquire and the second barrier order the merge's reads after the siblings'.
    __syncthreads();
    uint32_t* counter = counter_of(a, s.cb, kvh, 0);
    if (tid == 0) misc[3] = atom_add_acq_rel_gpu(counter, 1u) == static_cast<uint32_t>(s.nchunks - 1);
    __syncthreads();
    if (misc[3]) {
      for (int idx = tid; idx < G * D; idx += kGenThreads) {
        const int h = idx / D, d = idx - h * D;
        float M = -INFINITY;
        for (int k = 0; k < s.nchunks; ++k) {
          M = fmaxf(M, __ldcg(a.part_lse + static_cast<int64_t>(chunk_id(a, s, k)) * G + h));
        }
        float W = 0.0f, O = 0.0f;
        if (M > -INFINITY) {
          for (int k = 0; k < s.nchunks; ++k) {
            const int64_t sk2 = chunk_id(a, s, k);
            const float lse = __ldcg(a.part_lse + sk2 * G + h);
            if (lse == -INFINITY) continue;
            const float f = fast_exp2(lse - M);
            W += f;
            O += f * __ldcg(a.part_o + (sk2 * G + h) * D + d);
          }
        }
        out[out_row0 * D + idx] = Storage<T>::store(W > 0.0f ? O / W : 0.0f);
      }
      if (tid == 0) atomicExch(counter, 0u);
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------------- host side

namespace {

constexpr int kMinTilesPerCta = 4;  // balanced plan: fewest tiles a CTA takes, by default

struct Plan {
  bool tc = false;
  int D = 0, NT = 1;
  TcShape shape{};
  size_t smem = 0;
  int grid = 0;
  int units = 0;
  int splits = 0, pps = 0;
  int slots = 0, slot_heads = 0;
  int seg_cost = 0;
  int min_tiles = kMinTilesPerCta;
  bool kv8 = false;
  int groups = 0;   // cascade: prefix groups (0: plain decode)
  bool gather = false;  // the kernel stores its rows into other GPUs' outputs too
  int members = 1;  // cascade: sequences packed into one prefix item
  int prefix_chunk = 0;  // cascade: tokens per tensor-core prefix chunk (0: prefix items in the plan)
  int cas_planes = 1;    // cascade: prefix planes per sequence (chunks of the longest prefix)
  size_t prefix_smem = 0;
  size_t cas_o_off = 0, cas_lse_off = 0;  // cascade: side states within the partials buffer
  size_t part_bytes = 0, sync_bytes = 0;
  const void* fn = nullptr;
};

// Shared-prefix groups of a cascade call (groups == 0: none).
struct CascadeIn {
  const int32_t* bt = nullptr;
  const int32_t* lens = nullptr;
  const int32_t* indptr = nullptr;
  int groups = 0;
  int64_t bt_stride = 0;
  int max_pages = 0;
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

// Blocks per SM for `fn` at `smem` dynamic bytes; also raises the kernel's dynamic
// shared-memory limit on first use on this device.
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

// Every tensor-core kernel instantiation has this signature.
using TcKernel = void (*)(CUtensorMap, CUtensorMap, DecodeArgs, TcShape);

// The instantiation for a plan: cascades have no gather, and the gather exists for 16-bit caches only.
template <typename T, int D, int NT, bool KV8>
TcKernel tc_kernel_one(bool cas, bool gather) {
  if (cas) return decode_tc_kernel<T, D, NT, KV8, true, false>;
  if constexpr (!KV8) {
    if (gather) return decode_tc_kernel<T, D, NT, false, false, true>;
  }
  return decode_tc_kernel<T, D, NT, KV8, false, false>;
}

template <typename T>
TcKernel tc_kernel(int D, int NT, bool kv8, bool cas, bool gather) {
  if (kv8) {
    if (D == 128) return NT == 1 ? tc_kernel_one<T, 128, 1, true>(cas, false) : tc_kernel_one<T, 128, 2, true>(cas, false);
    return tc_kernel_one<T, 256, 1, true>(cas, false);
  }
  if (D == 64) return NT == 1 ? tc_kernel_one<T, 64, 1, false>(cas, gather) : tc_kernel_one<T, 64, 2, false>(cas, gather);
  if (D == 128) return NT == 1 ? tc_kernel_one<T, 128, 1, false>(cas, gather) : tc_kernel_one<T, 128, 2, false>(cas, gather);
  return tc_kernel_one<T, 256, 1, false>(cas, gather);
}

const void* gen_fn(int dtype) {
  switch (dtype) {
    case KL_FLOAT32: return (const void*)decode_generic_kernel<float>;
    case KL_FLOAT16: return (const void*)decode_generic_kernel<__half>;
    default: return (const void*)decode_generic_kernel<__nv_bfloat16>;
  }
}

constexpr uint32_t kTcSmemBudget = 225 * 1024;  // one tensor-core CTA per SM (227 KB is the limit)
constexpr int kMaxStages = 24;
// Balanced plan: tiles' worth of time a tensor-core CTA loses per (sequence, head block) it
// starts (Q loads, partial write and count). Charging 4 (sweep of 2..8, one box): batch 64 x 512
// tokens 29.0 us against 31.1 us with 2, batch 8 x 512 16.7 against 18.8; batch 64 x 4096,
// 256 x 512 and the 70B shape within 1 us of the cost-2 plan.
constexpr int kTcSegmentCost = 4;

// Optional tuning overrides read from the environment on each call:
//   KL_DECODE_HEADS_PER_TILE (1/2/4/8), KL_DECODE_STAGES (2..24), KL_DECODE_SEGMENT_COST
//   (tiles charged per (sequence, unit) start by the balanced plan; negative: none),
//   KL_DECODE_MIN_TILES (fewest tiles a CTA of the balanced plan takes), KL_DECODE_NT (1/2:
//   8 or 16 query heads per warp, where the group allows). 0 = automatic.
int env_int(const char* name) {
  const char* v = std::getenv(name);
  return v ? std::atoi(v) : 0;
}

// Partial outputs [slots][slot_heads][D] fp32 first, then their LSEs, 256-byte aligned.
size_t lse_offset(int slots, int slot_heads, int D) {
  return (static_cast<size_t>(slots) * slot_heads * D * 4 + 255) / 256 * 256;
}

// Launch shape and scratch sizes of one decode call. `generic` forces the CUDA-core kernel.
// kv8: e4m3 cache (tensor-core kernel only: head_dim 128 or 256, q/out fp16 or bf16).
// groups > 0: a cascade over that many shared-prefix groups of at most prefix_max_pages pages
// (tensor-core kernel and balanced plan only).
int make_plan(int dtype, int batch, int Hq, int Hkv, int D, int P, int max_pages, int num_splits, bool generic,
              Plan& p, bool kv8 = false, int groups = 0, int prefix_max_pages = 0, bool gather = false) {
  if (batch <= 0 || batch > kMaxBatch || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0 || D <= 0 || P <= 0 ||
      max_pages < 0 || num_splits < 0 || groups < 0 || groups > kMaxBatch || prefix_max_pages < 0) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  const bool cascade = groups > 0;
  if (cascade && (generic || num_splits != 0)) return static_cast<int>(cudaErrorInvalidValue);
  // A cascade runs on the tensor-core kernel only: reject other shapes before any device query.
  if (cascade && (dtype == KL_FLOAT32 || !(D == 64 || D == 128 || D == 256) || !(P == 8 || P % 16 == 0))) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  if (dtype != KL_FLOAT32 && dtype != KL_FLOAT16 && dtype != KL_BFLOAT16) return static_cast<int>(cudaErrorInvalidValue);
  const int G = Hq / Hkv;
  const int64_t max_tokens = static_cast<int64_t>(max_pages) * P;
  if (max_tokens > INT_MAX / 2) return static_cast<int>(cudaErrorInvalidValue);
  const int64_t max_tiles = (max_tokens + kTile - 1) / kTile;
  if (static_cast<int64_t>(batch) * max_tiles * Hkv > INT_MAX / 2) return static_cast<int>(cudaErrorInvalidValue);
  const int64_t prefix_tokens = cascade ? static_cast<int64_t>(prefix_max_pages) * P : 0;
  if (prefix_tokens > INT_MAX / 2) return static_cast<int>(cudaErrorInvalidValue);
  const int64_t prefix_tiles = (prefix_tokens + kTile - 1) / kTile;  // per prefix item (at most batch of them)
  if (static_cast<int64_t>(batch) * prefix_tiles * Hkv > INT_MAX / 2) return static_cast<int>(cudaErrorInvalidValue);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return static_cast<int>(cudaErrorNoDevice);
  const int sms = device_sms(dev);
  if (sms <= 0) return static_cast<int>(cudaErrorNoDevice);

  p.D = D;
  int NT = (G > 8 && D <= 128) ? 2 : 1;
  // Groups of 9-32 query heads on small problems: 8 heads per warp (up to 4 warp groups a KV
  // head) rather than 16. Each warp's tile work is shorter, which is what a problem of few tiles
  // per SM is bound by. Measured at head_dim 128, bf16 (us, 16 against 8 heads a warp): MQA 32/1
  // 4 x 4096 48.5 / 31.7, 8 x 4096 41.4 / 27.3, 32 x 4096 46.2 / 41.5 (55 tiles per SM),
  // 1 x 32768 141.4 / 91.4; 32/2 16 x 4096 41.2 / 32.8; 64/4 8 x 4096 44.1 / 35.4. From about 110
  // tiles per SM on, 16 heads a warp is faster (MQA 64 x 4096 58.5 / 62.9, 64/4 64 x 4096
  // 105.6 / 125.1, config 4's ragged MQA 294 / 424). The table width stands in for the lengths.
  if (NT == 2 && !cascade && !kv8 && D == 128 && (G + 7) / 8 <= kMaxHeadGroups &&
      static_cast<int64_t>(batch) * max_tiles * Hkv < 64LL * sms) {
    NT = 1;
  }
  // KL_DECODE_NT=1 / 2 forces the query columns per warp (8 or 16 heads) where the shape allows.
  const int forced_nt = env_int("KL_DECODE_NT");
  if (forced_nt == 1 && (G + 7) / 8 <= kMaxHeadGroups) NT = 1;
  if (forced_nt == 2 && D <= 128) NT = 2;
  // A cascade may widen the warps' query columns so that a prefix item packs more sequences
  // (KL_DECODE_CASCADE_NT=2; head_dim <= 128).
  if (cascade && env_int("KL_DECODE_CASCADE_NT") == 2 && D <= 128) NT = 2;
  const int hg_need = (G + 8 * NT - 1) / (8 * NT);
  const int HG = hg_need <= 1 ? 1 : hg_need <= 2 ? 2 : hg_need <= 4 ? 4 : 0;
  p.tc = !generic && dtype != KL_FLOAT32 && (D == (kv8 ? 128 : 64) || D == 128 || D == 256) &&
         (P == 8 || P % 16 == 0) && HG > 0;
  if (kv8 && !p.tc) return static_cast<int>(cudaErrorInvalidValue);
  // Cascade prefixes on the tensor-core prefix kernel when its shapes fit (16-bit cache, head_dim
  // 64 or 128, a group size that divides the 128 rows of an MMA, pages that tile a chunk) and it
  // pays: groups that fill half an MMA tile on average, and prefix tables at least twice as wide
  // as the sequences' own (otherwise the prefix items ride in the decode kernel's balanced plan,
  // measured faster: 8 groups of 8 sequences, 65 us against 84 us; 4 groups of 64 with equal
  // prefix and own lengths, 215 us against 244 us). KL_DECODE_CASCADE_TC=1 / 0 forces either.
  if (cascade) {
    const char* tc_env = std::getenv("KL_DECODE_CASCADE_TC");
    const bool fits = !kv8 && (D == 64 || D == 128) && 128 % G == 0 && P <= kPrefixTokens && kPrefixTokens % P == 0;
    const bool pays = static_cast<int64_t>(batch) * 2 * G >= static_cast<int64_t>(groups) * 128 &&
                      prefix_max_pages >= 2 * static_cast<int64_t>(max_pages);
    const bool tc_prefix = fits && (tc_env ? std::atoi(tc_env) != 0 : pays);
    p.prefix_chunk = 0;
    p.cas_planes = 1;
    if (tc_prefix) {
      // Segments of consecutive chunks, sized so that (member blocks x KV heads x segments) is
      // about one CTA per SM (the member blocks estimated from the batch and the group count).
      const int64_t chunks = std::max<int64_t>(1, (prefix_tokens + kPrefixTokens - 1) / kPrefixTokens);
      const int64_t blocks = std::min<int64_t>(batch, (batch + 128 / G - 1) / (128 / G) + groups - 1);
      const int64_t segs_per_pair = std::max<int64_t>(1, sms / std::max<int64_t>(1, blocks * Hkv));
      const int64_t ncpc = std::min<int64_t>(kPrefixChunksMax, (chunks + segs_per_pair - 1) / segs_per_pair);
      p.prefix_chunk = static_cast<int>(ncpc) * kPrefixTokens;
      p.cas_planes = static_cast<int>((chunks + ncpc - 1) / ncpc);
    }
  }
  const int64_t plan_prefix_tiles = p.prefix_chunk > 0 ? 0 : prefix_tiles;  // prefix tiles in the decode plan
  p.kv8 = kv8;
  const int eb = kv8 ? 1 : 2;
  int threads;
  if (p.tc) {
    p.NT = NT;
    // Heads per tile: a power of two dividing Hkv, at most 8 / HG warps' worth, a stage of
    // at most 64 KB, and enough (sequence, head-block) tiles to keep every SM busy.
    int ht = 1;
    while (ht * 2 <= 8 / HG && Hkv % (ht * 2) == 0 && ht * 2 * D <= 1024) ht *= 2;
    const int64_t tiles = static_cast<int64_t>(batch) * (max_tiles + plan_prefix_tiles);
    while (ht > 1 && tiles * (Hkv / ht) < 4LL * sms) ht /= 2;
    const int forced_ht = env_int("KL_DECODE_HEADS_PER_TILE");
    if (forced_ht > 0 && forced_ht <= 8 / HG && Hkv % forced_ht == 0 && (forced_ht & (forced_ht - 1)) == 0 &&
        forced_ht * D <= 1024) {
      ht = forced_ht;
    }
    p.shape.ht = ht;
    p.shape.hg = HG;
    p.shape.tw = kCW / (ht * HG);
    p.shape.p_rows = P < 16 ? P : 16;
    // Streams (one warp a stream) when a tile holds one (head, group) pair, the kernel has one
    // n-tile (the two-n-tile kernels have no registers to spare for the stream producer) and the
    // ring holds at least two stages a stream; otherwise one shared ring.
    const int forced_ns = env_int("KL_DECODE_STAGES");
    auto ring_stages = [&](int streams) {
      const TcLayout base = tc_layout(D, NT, p.shape.tw, streams, 0, batch, eb, groups, ht);
      const uint32_t stage = base.stage_bytes + 16u;
      int n = base.total < kTcSmemBudget ? static_cast<int>((kTcSmemBudget - base.total) / stage) : 0;
      n = std::min(kMaxStages, n);
      if (forced_ns >= 2) n = std::min(n, forced_ns);
      return n / p.shape.tw * p.shape.tw;
    };
    int streams = ht * HG == 1 && NT == 1 ? p.shape.tw : 1;
    int ns = ring_stages(streams);
    if (streams > 1 && ns < 2 * streams) {
      streams = 1;
      ns = ring_stages(1);
    }
    // The stage count is a multiple of TW. Streams: stream t owns stages t, t + TW, ..., at least
    // two. Shared ring: stage s is consumed only by the warps with tw == s % TW, in order, so a
    // warp never waits on a stage whose previous phase belongs to another warp (with a stage
    // count that is not a multiple of TW, a wait for phase k could be satisfied by phase k-2, of
    // the same parity, and the ring would fall out of step).
    if (ns < std::max(2, p.shape.tw) || ns < 2 * streams) return static_cast<int>(cudaErrorInvalidValue);
    p.shape.nstage = ns;
    p.shape.ns = streams;
    p.smem = tc_layout(D, NT, p.shape.tw, streams, ns, batch, eb, groups, ht).total;
    p.fn = reinterpret_cast<const void*>(
        dtype == KL_FLOAT16 ? tc_kernel<__half>(D, NT, kv8, cascade, gather)
                            : tc_kernel<__nv_bfloat16>(D, NT, kv8, cascade, gather));
    p.gather = gather;
    p.units = Hkv / ht;
    p.slot_heads = 8 * NT;
    p.groups = groups;
    p.members = HG * 8 * NT / G > 1 ? HG * 8 * NT / G : 1;
    threads = kTCThreads;
  } else {
    if (cascade) return static_cast<int>(cudaErrorInvalidValue);
    if (static_cast<int64_t>(G) * D > 8192) return static_cast<int>(cudaErrorInvalidValue);
    p.smem = gen_layout(G, D, batch).total;
    p.fn = gen_fn(dtype);
    p.units = Hkv;
    p.slot_heads = G;
    threads = kGenThreads;
  }
  int max_optin = 0;
  cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (p.smem > static_cast<size_t>(max_optin)) return static_cast<int>(cudaErrorInvalidValue);
  const int per_sm = blocks_per_sm(dev, p.fn, threads, p.smem);
  if (per_sm <= 0) return static_cast<int>(cudaErrorInvalidConfiguration);

  const int slots_per_chunk = p.tc ? p.shape.ht * p.shape.hg : 1;
  int64_t chunks;
  if (num_splits > 0) {
    const int mp = std::max(1, max_pages);
    p.pps = (mp + num_splits - 1) / num_splits;
    p.splits = (mp + p.pps - 1) / p.pps;
    chunks = static_cast<int64_t>(batch) * p.units * p.splits;
    // Every stream of a CTA walks its own items.
    const int streams = p.tc ? p.shape.ns : 1;
    p.grid = static_cast<int>(std::min<int64_t>((chunks + streams - 1) / streams, static_cast<int64_t>(sms) * per_sm));
  } else {
    p.splits = 0;
    p.grid = sms * per_sm;
    // Two chunk ids per range: the plan is cut into grid * streams ranges.
    chunks = 2LL * p.grid * (p.tc ? p.shape.ns : 1);
  }
  if (chunks * slots_per_chunk > INT_MAX / 2) return static_cast<int>(cudaErrorInvalidValue);
  const int forced_min = env_int("KL_DECODE_MIN_TILES");
  if (forced_min > 0) p.min_tiles = std::min(forced_min, 1 << 20);
  const int forced_cost = env_int("KL_DECODE_SEGMENT_COST");
  p.seg_cost = forced_cost < 0 ? 0 : forced_cost > 0 ? std::min(forced_cost, 64) : p.tc ? kTcSegmentCost : 0;
  const int64_t cost = static_cast<int64_t>(batch) * (max_tiles + p.seg_cost) +
                       (cascade ? static_cast<int64_t>(batch) * (plan_prefix_tiles + p.seg_cost) : 0);
  if (cost * p.units > INT_MAX / 2) return static_cast<int>(cudaErrorInvalidValue);
  p.slots = static_cast<int>(chunks * slots_per_chunk);
  p.part_bytes = lse_offset(p.slots, p.slot_heads, D) + static_cast<size_t>(p.slots) * p.slot_heads * 4;
  // Counter blocks: sequences' own tokens, then (cascade) prefix items and the per-sequence sides.
  p.sync_bytes = (1 + static_cast<size_t>(cascade ? 3 : 1) * batch * Hkv * kMaxHeadGroups) * 4;
  if (cascade) {
    const size_t rows = static_cast<size_t>(batch) * Hq;
    const size_t planes = static_cast<size_t>(p.cas_planes) + 1;  // prefix planes + the sequences' own
    p.cas_o_off = (p.part_bytes + 255) / 256 * 256;
    p.cas_lse_off = p.cas_o_off + planes * rows * D * 4;
    p.part_bytes = p.cas_lse_off + planes * rows * 4;
    if (p.prefix_chunk > 0) {
      p.prefix_smem = prefix_layout(D).total;
      const void* pf = dtype == KL_FLOAT16 ? (D == 64 ? (const void*)cascade_prefix_kernel<__half, 64>
                                                      : (const void*)cascade_prefix_kernel<__half, 128>)
                                           : (D == 64 ? (const void*)cascade_prefix_kernel<__nv_bfloat16, 64>
                                                      : (const void*)cascade_prefix_kernel<__nv_bfloat16, 128>);
      if (blocks_per_sm(dev, pf, kPrefixThreads, p.prefix_smem) <= 0) return static_cast<int>(cudaErrorInvalidConfiguration);
    }
  }
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

// 3-D view of one cache: (64 elements = 128 bytes) x (Hkv*D/64 pieces of a token row, 128 B
// apart) x (every token slot of the pool, Hkv*D*2 bytes apart). A box of HT*D/64 pieces x
// p_rows tokens is one tile (or half of one, for page size 8) of a head block: for HT == Hkv a
// whole page, read front to back.
bool encode_kv_map(CUtensorMap* map, const void* base, int dtype, int64_t pool_tokens, int Hkv, int D, int HT,
                   int p_rows, bool kv8, int box_pieces = 0) {
  auto enc = encoder();
  if (!enc) return false;
  // 128-byte pieces: 64 two-byte elements, or 128 e4m3 bytes (moved as uint8).
  const int per_piece = kv8 ? 128 : 64;
  const int row_bytes = Hkv * D * (kv8 ? 1 : 2);
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(per_piece), static_cast<cuuint64_t>(row_bytes / 128),
                              static_cast<cuuint64_t>(pool_tokens)};
  const cuuint64_t strides[2] = {128u, static_cast<cuuint64_t>(row_bytes)};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(per_piece), static_cast<cuuint32_t>(box_pieces > 0 ? box_pieces : HT * D * (kv8 ? 1 : 2) / 128),
                             static_cast<cuuint32_t>(p_rows)};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  const CUtensorMapDataType dt = kv8                  ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                 : dtype == KL_FLOAT16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                       : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const CUresult r = enc(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// q as the A operand of the prefix kernel: (64 elements = 128 bytes) x (query heads) x (sequences);
// a box of 64 x group x 128/group is one 128-byte column block of a member block's 128 rows.
bool encode_q_map(CUtensorMap* map, const void* q, int dtype, int batch, int Hq, int D, int G) {
  auto enc = encoder();
  if (!enc) return false;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(Hq), static_cast<cuuint64_t>(batch)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * 2u, static_cast<cuuint64_t>(Hq) * D * 2u};
  const cuuint32_t box[3] = {64u, static_cast<cuuint32_t>(G), static_cast<cuuint32_t>(128 / G)};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  const CUresult r = enc(map, dtype == KL_FLOAT16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                         const_cast<void*>(q), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// Launch with programmatic stream serialization (KL_DECODE_PDL=0: without, read once): the kernel
// may begin while the previous kernel in the stream finishes; every kernel launched this way calls
// wait_prior_grid() before touching global memory.
bool decode_pdl() {
  static const bool on = env_switch_on("KL_DECODE_PDL");
  return on;
}

template <typename... Params, typename... Args>
cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, int threads, size_t smem, cudaStream_t st,
                       const Args&... args) {
  return launch_kernel(decode_pdl(), kernel, grid, dim3(static_cast<unsigned>(threads)), smem, st, args...);
}

// The plan's kernel instantiation (p.fn), launched with programmatic stream serialization: its
// prologue may overlap the previous kernel in the stream (see decode_tc_kernel).
cudaError_t launch_tc(const Plan& p, const CUtensorMap& tmk, const CUtensorMap& tmv, const DecodeArgs& a,
                      cudaStream_t st) {
  const TcKernel kernel = reinterpret_cast<TcKernel>(const_cast<void*>(p.fn));
  return launch_pdl(kernel, dim3(static_cast<unsigned>(p.grid)), kTCThreads, p.smem, st, tmk, tmv, a, p.shape);
}

// The kernel one call takes, and its plan: the tensor-core kernel where the shape allows it, the
// buffers are aligned for it (16-byte caches for TMA, q and out for vector loads and stores), TMA
// row coordinates fit in int32 and both tensor maps encode; otherwise the generic kernel, which
// has no e4m3 or cascade form (those calls get cudaErrorInvalidValue). On success *use_tc says
// which, and for the tensor-core kernel *tmk / *tmv hold the caches' tensor maps. Every entry
// point that launches a decode, or sizes scratch for one it will launch, decides here.
int choose_kernel(int dtype, const void* out, const void* q, const void* k_cache, const void* v_cache, int batch,
                  int Hq, int Hkv, int D, int P, int max_pages, int64_t num_pages, int num_splits, bool kv8,
                  const CascadeIn& cas, Plan& p, CUtensorMap* tmk, CUtensorMap* tmv, bool* use_tc,
                  bool gather = false) {
  *use_tc = false;
  if (const int rc = make_plan(dtype, batch, Hq, Hkv, D, P, max_pages, num_splits, false, p, kv8, cas.groups,
                               cas.max_pages, gather)) {
    return rc;
  }
  const bool tc_ok = p.tc && aligned(k_cache, 16) && aligned(v_cache, 16) && aligned(q, 16) && aligned(out, 16) &&
                     (num_pages < 0 || num_pages * P <= INT_MAX);
  if (tc_ok) {
    const int64_t pool_tokens = num_pages >= 0 ? std::max<int64_t>(num_pages, 1) * P : (int64_t(1) << 31) - 1;
    *use_tc = encode_kv_map(tmk, k_cache, dtype, pool_tokens, Hkv, D, p.shape.ht, p.shape.p_rows, kv8) &&
              encode_kv_map(tmv, v_cache, dtype, pool_tokens, Hkv, D, p.shape.ht, p.shape.p_rows, kv8);
  }
  if ((kv8 || cas.groups > 0) && !*use_tc) return static_cast<int>(cudaErrorInvalidValue);
  if (!*use_tc && p.tc) return make_plan(dtype, batch, Hq, Hkv, D, P, max_pages, num_splits, true, p);
  return 0;
}

// k_scale / v_scale non-null: the caches hold e4m3 (tensor-core kernel only, no fallback).
int decode_impl(int dtype, void* out, const void* q, const void* k_cache, const void* v_cache,
                const int32_t* block_table, const int32_t* seq_lens, int batch, int Hq, int Hkv, int D, int P,
                int64_t bt_stride, int max_pages, int64_t num_pages, float scale, int num_splits, void* partials,
                size_t partial_bytes, void* sync, size_t sync_bytes, cudaStream_t st,
                const float* k_scale = nullptr, const float* v_scale = nullptr, const CascadeIn& cas = CascadeIn{},
                const kl_head_gather_t* gather = nullptr) {
  if (batch == 0) return 0;
  if (!out || !q || !k_cache || !v_cache || !block_table || !seq_lens || !sync) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  const bool cascade = cas.groups > 0;
  if (cascade && (!cas.bt || !cas.lens || !cas.indptr || cas.bt_stride < 0 ||
                  (cas.groups > 1 && cas.bt_stride < cas.max_pages))) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  const bool kv8 = k_scale != nullptr || v_scale != nullptr;
  if (kv8 && (!k_scale || !v_scale)) return static_cast<int>(cudaErrorInvalidValue);
  if (bt_stride < 0 || (batch > 1 && bt_stride < max_pages)) return static_cast<int>(cudaErrorInvalidValue);
  // A head gather runs on the tensor-core kernel of plain decode only.
  const bool gathering = gather != nullptr && gather->num_ranks > 1;
  Plan p;
  CUtensorMap tmk, tmv;
  bool use_tc = false;
  if (const int rc = choose_kernel(dtype, out, q, k_cache, v_cache, batch, Hq, Hkv, D, P, max_pages, num_pages,
                                   num_splits, kv8, cas, p, &tmk, &tmv, &use_tc, gathering && !cascade && !kv8)) {
    return rc;
  }
  if (partial_bytes < p.part_bytes || sync_bytes < p.sync_bytes || !partials) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  if (gathering && (!use_tc || cascade || kv8 || !p.gather)) return static_cast<int>(cudaErrorNotSupported);
  DecodeArgs a{};
  a.out = out;
  a.out_seq_stride = static_cast<int64_t>(Hq) * D;
  if (gather != nullptr) {
    // This rank's heads [rank * Hq, (rank + 1) * Hq) of every rank's [batch, ranks * Hq, D] output.
    const size_t eb = dtype == KL_FLOAT32 ? 4 : 2;
    const size_t head_off = static_cast<size_t>(gather->rank) * Hq * D * eb;
    a.out_seq_stride = static_cast<int64_t>(gather->num_ranks) * Hq * D;
    a.out = static_cast<uint8_t*>(gather->out[gather->rank]) + head_off;
    if (gathering) {
      a.gat.ranks = gather->num_ranks;
      a.gat.rank = gather->rank;
      a.gat.epoch = gather->epoch;
      a.gat.done = gather->done;
      a.gat.wait_ns = gather->timeout_ms ? gather->timeout_ms * 1000000ull : kPeerWaitNs;
      for (int r = 0; r < gather->num_ranks; ++r) {
        a.gat.out[r] = static_cast<uint8_t*>(gather->out[r]) + head_off;
        a.gat.flags[r] = gather->flags[r];
      }
    }
  }
  a.q = q;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.block_table = block_table;
  a.seq_lens = seq_lens;
  a.batch = batch;
  a.num_q_heads = Hq;
  a.num_kv_heads = Hkv;
  a.group = Hq / Hkv;
  a.head_dim = D;
  a.page_size = P;
  a.bt_stride = bt_stride;
  a.max_pages = max_pages;
  a.num_pages = num_pages;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.units = p.units;
  a.splits = p.splits;
  a.pages_per_split = p.pps;
  a.min_tiles = p.min_tiles;
  a.seg_cost = p.seg_cost;
  a.sync = static_cast<uint32_t*>(sync);
  a.part_o = static_cast<float*>(partials);
  a.part_lse = reinterpret_cast<float*>(static_cast<uint8_t*>(partials) + lse_offset(p.slots, p.slot_heads, D));
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  a.prefix_bt = cas.bt;
  a.prefix_lens = cas.lens;
  a.prefix_indptr = cas.indptr;
  a.num_prefixes = cascade ? cas.groups : 0;
  a.prefix_bt_stride = cas.bt_stride;
  a.prefix_max_pages = cas.max_pages;
  a.members = p.members;
  a.prefix_chunk = p.prefix_chunk;
  a.cas_planes = p.cas_planes;
  a.cas_hpw = 8 * p.NT;
  if (cascade) {
    a.cas_o = reinterpret_cast<float*>(static_cast<uint8_t*>(partials) + p.cas_o_off);
    a.cas_lse = reinterpret_cast<float*>(static_cast<uint8_t*>(partials) + p.cas_lse_off);
  }

  if (use_tc && p.prefix_chunk > 0) {
    // The shared prefixes first, on the tensor-core prefix kernel (one CTA per member block, KV
    // head and chunk; CTAs past the real ones exit at once), then the sequences' own tokens.
    CUtensorMap tmq, tpk, tpv;
    const int64_t pool_tokens = num_pages >= 0 ? std::max<int64_t>(num_pages, 1) * P : (int64_t(1) << 31) - 1;
    const int G = Hq / Hkv;
    if (!encode_q_map(&tmq, q, dtype, batch, Hq, D, G) ||
        !encode_kv_map(&tpk, k_cache, dtype, pool_tokens, Hkv, D, 1, P, false, 1) ||
        !encode_kv_map(&tpv, v_cache, dtype, pool_tokens, Hkv, D, 1, P, false, 1)) {
      return static_cast<int>(cudaErrorInvalidValue);
    }
    const dim3 grid(p.cas_planes, Hkv, (batch + 128 / G - 1) / (128 / G) + cas.groups);
    cudaError_t e;
    if (dtype == KL_FLOAT16) {
      e = D == 64 ? launch_pdl(cascade_prefix_kernel<__half, 64>, grid, kPrefixThreads, p.prefix_smem, st, tmq, tpk, tpv, a)
                  : launch_pdl(cascade_prefix_kernel<__half, 128>, grid, kPrefixThreads, p.prefix_smem, st, tmq, tpk, tpv, a);
    } else {
      e = D == 64 ? launch_pdl(cascade_prefix_kernel<__nv_bfloat16, 64>, grid, kPrefixThreads, p.prefix_smem, st, tmq, tpk, tpv, a)
                  : launch_pdl(cascade_prefix_kernel<__nv_bfloat16, 128>, grid, kPrefixThreads, p.prefix_smem, st, tmq, tpk, tpv, a);
    }
    if (e != cudaSuccess) return static_cast<int>(e);
    if (p.cas_planes > 1) {
      const int64_t threads = static_cast<int64_t>(batch) * Hq * (D / 4);  // one per float4 column
      const dim3 blocks(static_cast<unsigned>((threads + kReduceThreads - 1) / kReduceThreads));
      if (dtype == KL_FLOAT16) {
        e = D == 64 ? launch_pdl(cascade_prefix_reduce_kernel<__half, 64>, blocks, kReduceThreads, 0, st, a)
                    : launch_pdl(cascade_prefix_reduce_kernel<__half, 128>, blocks, kReduceThreads, 0, st, a);
      } else {
        e = D == 64 ? launch_pdl(cascade_prefix_reduce_kernel<__nv_bfloat16, 64>, blocks, kReduceThreads, 0, st, a)
                    : launch_pdl(cascade_prefix_reduce_kernel<__nv_bfloat16, 128>, blocks, kReduceThreads, 0, st, a);
      }
      if (e != cudaSuccess) return static_cast<int>(e);
    }
  }

  if (use_tc) {
    const cudaError_t e = launch_tc(p, tmk, tmv, a, st);
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

const char* kl_version(void) { return "kernel_lab_b200 0.2.0 sm_100a"; }

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
  // A misaligned call falls back to the generic kernel, whose shape differs: size for both.
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

int kl_paged_decode_fp8(int dtype, void* out, const void* q, const void* k_cache, const void* v_cache,
                        const float* k_scale, const float* v_scale, const int32_t* block_table,
                        const int32_t* seq_lens, int batch, int num_q_heads, int num_kv_heads, int head_dim,
                        int page_size, int64_t block_table_stride, int max_pages_per_seq, int64_t num_pages,
                        float scale, int num_splits, void* partials, size_t partial_bytes, void* sync,
                        size_t sync_bytes, void* stream) {
  if (batch != 0 && (!k_scale || !v_scale)) return static_cast<int>(cudaErrorInvalidValue);
  return klb::decode_impl(dtype, out, q, k_cache, v_cache, block_table, seq_lens, batch, num_q_heads, num_kv_heads,
                          head_dim, page_size, block_table_stride, max_pages_per_seq, num_pages, scale, num_splits,
                          partials, partial_bytes, sync, sync_bytes, static_cast<cudaStream_t>(stream), k_scale,
                          v_scale);
}

int kl_paged_decode_cascade_workspace_size(int dtype, int batch, int num_prefixes, int num_q_heads,
                                           int num_kv_heads, int head_dim, int page_size, int max_pages_per_seq,
                                           int max_prefix_pages, size_t* partial_bytes, size_t* sync_bytes) {
  if (!partial_bytes || !sync_bytes) return static_cast<int>(cudaErrorInvalidValue);
  *partial_bytes = 0;
  *sync_bytes = 4;
  if (batch == 0) return 0;
  if (num_prefixes == 0) {
    return kl_paged_decode_workspace_size(dtype, batch, num_q_heads, num_kv_heads, head_dim, page_size,
                                          max_pages_per_seq, 0, partial_bytes, sync_bytes);
  }
  klb::Plan p;
  if (const int rc = klb::make_plan(dtype, batch, num_q_heads, num_kv_heads, head_dim, page_size, max_pages_per_seq,
                                    0, false, p, false, num_prefixes, max_prefix_pages)) {
    return rc;
  }
  *partial_bytes = p.part_bytes;
  *sync_bytes = p.sync_bytes;
  return 0;
}

int kl_paged_decode_cascade(int dtype, void* out, const void* q, const void* k_cache, const void* v_cache,
                            const float* k_scale, const float* v_scale, const int32_t* prefix_block_table,
                            const int32_t* prefix_lens, const int32_t* prefix_indptr, int num_prefixes,
                            int64_t prefix_block_table_stride, int max_prefix_pages, const int32_t* block_table,
                            const int32_t* seq_lens, int batch, int num_q_heads, int num_kv_heads, int head_dim,
                            int page_size, int64_t block_table_stride, int max_pages_per_seq, int64_t num_pages,
                            float scale, void* partials, size_t partial_bytes, void* sync, size_t sync_bytes,
                            void* stream) {
  if (num_prefixes < 0 || ((k_scale == nullptr) != (v_scale == nullptr))) return static_cast<int>(cudaErrorInvalidValue);
  klb::CascadeIn cas;
  cas.bt = prefix_block_table;
  cas.lens = prefix_lens;
  cas.indptr = prefix_indptr;
  cas.groups = num_prefixes;
  cas.bt_stride = prefix_block_table_stride;
  cas.max_pages = max_prefix_pages;
  return klb::decode_impl(dtype, out, q, k_cache, v_cache, block_table, seq_lens, batch, num_q_heads, num_kv_heads,
                          head_dim, page_size, block_table_stride, max_pages_per_seq, num_pages, scale, 0, partials,
                          partial_bytes, sync, sync_bytes, static_cast<cudaStream_t>(stream), k_scale, v_scale, cas);
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

int kl_paged_decode_gather(int dtype, const kl_head_gather_t* gather, const void* q, const void* k_cache,
                           const void* v_cache, const int32_t* block_table, const int32_t* seq_lens, int batch,
                           int num_q_heads, int num_kv_heads, int head_dim, int page_size,
                           int64_t block_table_stride, int max_pages_per_seq, int64_t num_pages, float scale,
                           void* partials, size_t partial_bytes, void* sync, size_t sync_bytes, void* stream) {
  if (!gather || gather->num_ranks < 1 || gather->num_ranks > KL_GATHER_MAX_RANKS || gather->rank < 0 ||
      gather->rank >= gather->num_ranks) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  for (int r = 0; r < gather->num_ranks; ++r) {
    if (!gather->out[r] || (gather->num_ranks > 1 && !gather->flags[r])) return static_cast<int>(cudaErrorInvalidValue);
  }
  if (gather->num_ranks > 1 && (!gather->done || gather->epoch == 0u)) return static_cast<int>(cudaErrorInvalidValue);
  if (batch == 0) return 0;
  return klb::decode_impl(dtype, gather->out[gather->rank], q, k_cache, v_cache, block_table, seq_lens, batch,
                          num_q_heads, num_kv_heads, head_dim, page_size, block_table_stride, max_pages_per_seq,
                          num_pages, scale, 0, partials, partial_bytes, sync, sync_bytes,
                          static_cast<cudaStream_t>(stream), nullptr, nullptr, klb::CascadeIn{}, gather);
}

int kl_ipc_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return static_cast<int>(cudaErrorInvalidValue);
  *ptr = nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return static_cast<int>(e);
  e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h{};
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return static_cast<int>(e);
  }
  static_assert(sizeof(h) == KL_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return 0;
}

int kl_ipc_open(const void* handle, void** ptr) {
  if (!ptr || !handle) return static_cast<int>(cudaErrorInvalidValue);
  cudaIpcMemHandle_t h{};
  std::memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  return static_cast<int>(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

int kl_ipc_close(void* ptr) { return ptr ? static_cast<int>(cudaIpcCloseMemHandle(ptr)) : 0; }

int kl_ipc_free(void* ptr) { return ptr ? static_cast<int>(cudaFree(ptr)) : 0; }

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

// ------------------------------------------------------------------------- no-allocation entry point
//
// Decode with scratch that lives in this library's own device memory, for callers that
// cannot allocate device memory at call time: an inference server whose memory is carved
// up and owned by its pool at start-up, a runtime that has already reserved every free
// byte for the KV cache, or code that must not call cudaMalloc (or wait on the caching
// allocator) from inside its step loop. The scratch is one fixed array per GPU. CUDA reserves
// it when this library's device code is loaded on that GPU (with lazy module loading, the
// default, at the first launch or symbol lookup there, not at dlopen) and holds it until the
// process exits.

namespace klb {
namespace {

constexpr size_t kNoAllocPartialBytes = size_t(16) << 20;  // split partials
constexpr size_t kNoAllocSyncBytes = size_t(256) << 10;    // status word + arrival counters
static_assert(kNoAllocPartialBytes + kNoAllocSyncBytes == KL_NOALLOC_SCRATCH_BYTES, "header and library disagree");

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocPartialBytes + kNoAllocSyncBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {};

// Device address of g_noalloc_scratch on the current device, looked up on first use there.
cudaError_t noalloc_scratch(void** ptr) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_noalloc_ptr[dev] = p;
  }
  *ptr = g_noalloc_ptr[dev];
  return cudaSuccess;
}

}  // namespace
}  // namespace klb

extern "C" int kl_paged_decode_noalloc(int dtype, void* out, const void* q, const void* k_cache,
                                       const void* v_cache, const int32_t* block_table, const int32_t* seq_lens,
                                       int batch, int num_q_heads, int num_kv_heads, int head_dim, int page_size,
                                       int64_t block_table_stride, int max_pages_per_seq, int64_t num_pages,
                                       float scale, int num_splits, void* stream) {
  if (batch == 0) return 0;
  // Size the scratch of the kernel kl_paged_decode will launch for these pointers: the same
  // choice (tensor-core or generic kernel, tensor maps included) that the launch makes.
  klb::Plan plan;
  CUtensorMap tmk, tmv;
  bool use_tc = false;
  if (const int rc = klb::choose_kernel(dtype, out, q, k_cache, v_cache, batch, num_q_heads, num_kv_heads, head_dim,
                                        page_size, max_pages_per_seq, num_pages, num_splits, false, klb::CascadeIn{},
                                        plan, &tmk, &tmv, &use_tc)) {
    return rc;
  }
  const size_t sync_bytes = plan.sync_bytes;
  if (plan.part_bytes > klb::kNoAllocPartialBytes || sync_bytes > klb::kNoAllocSyncBytes) {
    return static_cast<int>(cudaErrorMemoryAllocation);  // does not fit the fixed scratch
  }
  void* base = nullptr;
  if (const cudaError_t e = klb::noalloc_scratch(&base)) return static_cast<int>(e);
  uint8_t* partials = static_cast<uint8_t*>(base);
  uint8_t* sync = partials + klb::kNoAllocPartialBytes;
  auto st = static_cast<cudaStream_t>(stream);
  // The array keeps whatever the previous call left: start from zeroed counters and status.
  if (const cudaError_t e = cudaMemsetAsync(sync, 0, sync_bytes, st)) return static_cast<int>(e);
  return kl_paged_decode(dtype, out, q, k_cache, v_cache, block_table, seq_lens, batch, num_q_heads, num_kv_heads,
                         head_dim, page_size, block_table_stride, max_pages_per_seq, num_pages, scale, num_splits,
                         partials, klb::kNoAllocPartialBytes, sync, klb::kNoAllocSyncBytes, stream);
}

extern "C" int kl_paged_decode_noalloc_read_status(uint32_t* status, int clear, void* stream) {
  if (!status) return static_cast<int>(cudaErrorInvalidValue);
  void* base = nullptr;
  if (const cudaError_t e = klb::noalloc_scratch(&base)) return static_cast<int>(e);
  return kl_paged_decode_read_status(static_cast<uint8_t*>(base) + klb::kNoAllocPartialBytes, status, clear, stream);
}
