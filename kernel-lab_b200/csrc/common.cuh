// Device helpers for the sm_100a kernels: storage-type traits, 16-byte packs,
// reductions, and thin inline-PTX wrappers for mbarriers, TMA tensor loads,
// ldmatrix / movmatrix and the m16n8k16 tensor-core MMA.
//
// Every wait on an mbarrier is bounded (by the SM cycle counter): a wait that runs
// out records an error bit in the caller's status word and returns false, so a
// kernel can stop cleanly instead of hanging the GPU.
#pragma once

#include <cstdint>
#include <cstdlib>

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

namespace klb {

// ----------------------------------------------------------------- storage types

template <typename T>
struct Storage;

template <>
struct Storage<float> {
  static __device__ __forceinline__ float load(float v) { return v; }
  static __device__ __forceinline__ float store(float v) { return v; }
};

template <>
struct Storage<__half> {
  static __device__ __forceinline__ float load(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half store(float v) { return __float2half_rn(v); }
  // Two floats -> one 32-bit register holding (lo, hi) as f16.
  static __device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  static __device__ __forceinline__ float2 unpack2(uint32_t v) {
    return __half22float2(*reinterpret_cast<const __half2*>(&v));
  }
};

template <>
struct Storage<__nv_bfloat16> {
  static __device__ __forceinline__ float load(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 store(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  static __device__ __forceinline__ float2 unpack2(uint32_t v) {
    return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
  }
};

// N storage elements moved as one naturally aligned vector (16 bytes at most).
template <typename T, int N>
struct alignas(sizeof(T) * N) Vec {
  T v[N];
};

// Two e4m3 values -> f16x2 (low half first); exact, e4m3 being a subset of f16. The pair is the
// low (e4m3x2_lo_to_f16x2) or high (e4m3x2_hi_to_f16x2) 16 bits of a word, low byte first; the
// half is taken as a register half, with no mask or shift.
__device__ __forceinline__ uint32_t e4m3x2_lo_to_f16x2(uint32_t word) {
  uint32_t r;
  asm("{\n.reg .b16 lo, hi;\nmov.b32 {lo, hi}, %1;\ncvt.rn.f16x2.e4m3x2 %0, lo;\n}" : "=r"(r) : "r"(word));
  return r;
}
__device__ __forceinline__ uint32_t e4m3x2_hi_to_f16x2(uint32_t word) {
  uint32_t r;
  asm("{\n.reg .b16 lo, hi;\nmov.b32 {lo, hi}, %1;\ncvt.rn.f16x2.e4m3x2 %0, hi;\n}" : "=r"(r) : "r"(word));
  return r;
}

// lo += the low element, hi += the high element of a packed 16-bit pair, each widened exactly and
// added with one mixed-precision add (no unpacking into two floats first).
template <typename T>
__device__ __forceinline__ void add_pair_to(uint32_t w, float& lo, float& hi);
template <>
__device__ __forceinline__ void add_pair_to<__nv_bfloat16>(uint32_t w, float& lo, float& hi) {
  asm("{\n.reg .b16 l, h;\nmov.b32 {l, h}, %2;\nadd.rn.f32.bf16 %0, l, %0;\nadd.rn.f32.bf16 %1, h, %1;\n}"
      : "+f"(lo), "+f"(hi)
      : "r"(w));
}
template <>
__device__ __forceinline__ void add_pair_to<__half>(uint32_t w, float& lo, float& hi) {
  asm("{\n.reg .b16 l, h;\nmov.b32 {l, h}, %2;\nadd.rn.f32.f16 %0, l, %0;\nadd.rn.f32.f16 %1, h, %1;\n}"
      : "+f"(lo), "+f"(hi)
      : "r"(w));
}

// A packed pair of the storage type -> f16x2 (the operand type of the fp8-cache MMAs).
template <typename T>
__device__ __forceinline__ uint32_t to_f16x2(uint32_t v);
template <>
__device__ __forceinline__ uint32_t to_f16x2<__half>(uint32_t v) { return v; }
template <>
__device__ __forceinline__ uint32_t to_f16x2<__nv_bfloat16>(uint32_t v) {
  return Storage<__half>::pack2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
}

// ----------------------------------------------------------------- reductions

__device__ __forceinline__ float warp_allreduce_sum(float v) {
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  return v;
}

__device__ __forceinline__ float warp_allreduce_max(float v) {
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, m));
  return v;
}

// Barrier over a subset of the block's warps (named barrier `id`, `threads` threads).
__device__ __forceinline__ void named_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ----------------------------------------------------------------- status bits

// Bits of the status word a decode call leaves in its sync buffer (word 0).
enum StatusBits : uint32_t {
  kStatusBadPage = 1u,       // a block-table entry outside [0, num_pages): that page was skipped
  kStatusLenClamped = 2u,    // a sequence longer than max_pages * page_size was clamped
  kStatusWaitTimeout = 4u,   // an mbarrier wait ran out of time; the kernel stopped early
  kStatusBadPrefixGroups = 8u,  // cascade groups do not partition the batch: prefixes were ignored
  kStatusPeerTimeout = 16u,     // head gather: a rank's arrival did not come within the time limit
};

// ----------------------------------------------------------------- programmatic dependent launch

// For kernels launched with cudaLaunchAttributeProgrammaticStreamSerialization: wait until the
// previous kernel in the stream has completed and its writes are visible (returns at once when it
// already has, or when this kernel was launched without the attribute); let the next kernel in
// the stream start launching.
__device__ __forceinline__ void wait_prior_grid() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void allow_next_grid() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// An on/off switch read from the environment: unset or anything but "0" is on.
inline bool env_switch_on(const char* name) {
  const char* v = std::getenv(name);
  return !(v && std::atoi(v) == 0);
}

// Host side: launch `kernel` on `st`, with programmatic stream serialization when `pdl` is set.
// A kernel launched this way must call wait_prior_grid() before it touches global memory.
template <typename... Params, typename... Args>
inline cudaError_t launch_kernel(bool pdl, void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                                 cudaStream_t st, const Args&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// ----------------------------------------------------------------- shared-memory addresses

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ----------------------------------------------------------------- mbarriers

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// Make barrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile(
      "{\n"
      ".reg .b64 st;\n"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n"
      "}\n" ::"r"(bar)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile(
      "{\n"
      ".reg .b64 st;\n"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n"
      "}\n" ::"r"(bar),
      "r"(bytes)
      : "memory");
}

// Non-blocking test: has the phase with the given parity completed?
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

// Wait for the phase with the given parity to complete, for at most `limit_cycles` SM
// clock cycles (about a second at B200 clocks). The bound is kept with the SM's own cycle
// counter, which is cheap to read, and only checked every 256 polls. On timeout: set
// kStatusWaitTimeout in *status (if non-null) and return false.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, uint32_t* status,
                                                  uint64_t limit_cycles) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = clock64();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 256; ++i) {
      if (mbar_try_wait(bar, parity)) return true;
    }
    if (static_cast<uint64_t>(clock64()) - start > limit_cycles) {
      if (status) atomicOr(status, kStatusWaitTimeout);
      return false;
    }
  }
}

// Relaxed GPU-scope load of a flag another CTA updates. Followed by fence_acq_rel_gpu() once
// the value is seen, it forms an acquire (the fence-based acquire pattern of the PTX memory model).
// Not ordered against earlier memory operations, so it can be issued well before its use.
__device__ __forceinline__ uint32_t ld_relaxed_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// GPU-scope release/acquire without a sequentially consistent fence (which costs
// microseconds when many SMs issue it at once):
// - atom_add_acq_rel_gpu publishes every write ordered before it (the issuing thread's, and
//   its warp's through a preceding __syncwarp) and acquires what the previous holders of the
//   counter published;
// - fence_acq_rel_gpu after a relaxed load that saw another thread's count acquires that
//   thread's writes (the fence-based acquire pattern).
__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// System-scope forms, for flags that other GPUs read or write over NVLink (peer memory mapped
// into this process): a fence that orders this thread's earlier stores (local and remote) before
// its later ones, a releasing store and an acquiring load.
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Nanoseconds of the GPU's global timer (wall-clock time limits for waits on other GPUs).
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ----------------------------------------------------------------- TMA

// L2 eviction-priority policy for streamed-once data.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// L2 policy for data that other CTAs read again soon (a shared prefix's pages).
__device__ __forceinline__ uint64_t l2_policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void tma_prefetch_descriptor(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// 2-D tiled TMA load of one box into shared memory, completing on `bar` (no multicast).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, int x, int y, uint32_t bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(bar), "l"(policy)
      : "memory");
}

// 3-D tiled TMA load of one box into shared memory, completing on `bar` (no multicast).
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* tmap, int x, int y, int z, uint32_t bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(bar), "l"(policy)
      : "memory");
}

// ----------------------------------------------------------------- tcgen05 (5th-generation tensor cores)
//
// One thread issues tcgen05.mma for the CTA; operands A and B come from shared memory through
// 64-bit matrix descriptors, the fp32 accumulator lives in tensor memory (TMEM: 128 lanes x 512
// 32-bit columns per SM), and completion is signalled on an mbarrier by tcgen05.commit. TMEM
// addresses are (lane << 16) | column; a warp reads only lanes 32 * (warp % 4) .. + 31.

// Allocates `ncols` TMEM columns (a power of two >= 32) for this CTA; the whole warp executes
// it and the base address lands in shared memory at `dst`.
__device__ __forceinline__ void tmem_alloc(uint32_t dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tcgen05_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tcgen05_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Orders this thread's generic-proxy shared-memory writes before later async-proxy reads
// (tensor-core operands written by threads).
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Shared-memory matrix descriptor for a tile in the 128-byte swizzle layout (the layout TMA
// writes with CU_TENSOR_MAP_SWIZZLE_128B; tile bases 1024-byte aligned). Fields: start address,
// leading- and stride-dimension byte offsets (all >> 4), version 1, layout type 2 (128B swizzle).
// K-major operand: lbo = 16 (unused), sbo = byte distance between groups of 8 rows of 128 bytes.
// MN-major operand: lbo = byte distance between 64-element column blocks, sbo = between groups of
// 8 rows along K.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// Instruction descriptor of tcgen05.mma kind::f16 with an fp32 accumulator: A and B both f16 or
// both bf16, A K-major, B K-major or MN-major, M x N.
__host__ __device__ constexpr uint32_t umma_idesc_f16(bool bf16, int M, int N, bool b_mn_major) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// D[tmem] (+)= A[smem] . B[smem]; accumulate = 0 overwrites D. Issued by one thread.
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  const uint32_t mask0 = 0u, mask1 = 0u, mask2 = 0u, mask3 = 0u;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(mask0), "r"(mask1), "r"(mask2), "r"(mask3)
      : "memory");
}

// Arrives once on `bar` when every tcgen05.mma this thread issued before it has completed.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// 32 consecutive 32-bit columns of this thread's TMEM lane (shape 32x32b, x32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 consecutive 32-bit columns into this thread's TMEM lane (shape 32x32b, x32).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// ----------------------------------------------------------------- shared-memory vectors

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// ----------------------------------------------------------------- ldmatrix / movmatrix / mma

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr)
               : "memory");
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                              uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr)
               : "memory");
}

// Transpose an 8x8 matrix of 16-bit values held one row-pair per lane.
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}

template <typename T>
struct Mma;

// D = A(16x16, row) * B(16x8, col) + C, fp32 accumulate.
template <>
struct Mma<__nv_bfloat16> {
  static __device__ __forceinline__ void run(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
};

template <>
struct Mma<__half> {
  static __device__ __forceinline__ void run(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
};

}  // namespace klb
