// Device helpers shared by the sm_100a kernels: bounded mbarrier waits, TMA
// tile loads, tcgen05 (TMEM / UMMA) wrappers, and the activation math of the
// policy-sampling path.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace feb {

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  A kernel launched by launch_pdl may start
// while the kernel before it in the stream is still running; it calls
// griddep_wait() before it reads anything an earlier kernel wrote (the wait
// returns once the previous grid completed and its writes are visible; it is a
// no-op for a normal launch).  griddep_launch() lets the next kernel start.
// Every thread of a PDL kernel passes griddep_wait() before it exits, so the
// previous grid's completion carries over to the kernels after this one.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
  cudaLaunchAttribute attr{};
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ---------------------------------------------------------------------------
// error flags written by device code (never a trap): the host reads them after
// the launch and turns them into FE_STATUS_RESOURCE_EXHAUSTED.
enum DeviceError : int {
  kErrNone = 0,
  kErrWaitTimeoutProducer = 1,
  kErrWaitTimeoutMma = 2,
  kErrWaitTimeoutEpilogue = 3,
  kErrTmemAlloc = 4,
  kErrGridBarrierTimeout = 5,
  kErrProgramLayout = 6,
  kErrDependencyTimeout = 7,
  kErrStageTimeout = 8,
};

// Every mbarrier wait gives up after kWaitNs of wall time (read from the
// global nanosecond timer), far above any legitimate stall (one tile's K loop
// takes tens of microseconds).  kSpinLimit bounds the drain waits that run
// after an abort.
constexpr uint64_t kWaitNs = 1000000000ull;
constexpr uint32_t kSpinLimit = 1u << 20;

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* ptr) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(ptr));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait that may suspend the thread for up to `hint_ns` (it resumes as
// soon as the phase completes), so a waiting role does not take issue slots
// from the warps that share its scheduler.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Bulk copy of `bytes` (a multiple of 16; both addresses 16-byte aligned)
// from global to this CTA's shared memory, completing on `bar`'s tx count.
__device__ __forceinline__ void bulk_load_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Bounded wait: returns false (and never hangs) once kWaitNs elapsed or
// another role raised `abort_flag`.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_ns();
  for (uint32_t spin = 1;; ++spin) {
    if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
    if ((spin & 63u) == 0u) {
      if (*abort_flag) return false;
      if (global_ns() - start > kWaitNs) return false;
    }
  }
}

// ---------------------------------------------------------------------------
// thread-block clusters: distributed shared memory between the CTAs of a
// cluster (plain remote stores and remote mbarrier arrivals only)

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_index() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_count() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}

// Address in CTA `rank` of the cluster of the shared variable at `addr` here.
__device__ __forceinline__ uint32_t cluster_map(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void st_cluster_f64x2(uint32_t addr, double a, double b) {
  asm volatile("st.shared::cluster.v2.f64 [%0], {%1, %2};" ::"r"(addr), "d"(a), "d"(b) : "memory");
}

__device__ __forceinline__ void fence_acq_rel_cluster() { asm volatile("fence.acq_rel.cluster;" ::: "memory"); }

// Arrive (release, cluster scope) on an mbarrier of another CTA of the cluster.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t remote_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote_addr) : "memory");
}

// All threads of all CTAs of the cluster.  Used only where every thread of
// both CTAs is known to arrive: right after set-up and at kernel exit.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Bounded wait with cluster-scope acquire, for phases completed by another CTA.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  const uint64_t start = global_ns();
  for (uint32_t spin = 0;; ++spin) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;"
        "\n\tselp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(20000u)
        : "memory");
    if (ok != 0) return true;
    if ((spin & 63u) == 63u) {
      if (*abort_flag) return false;
      if (global_ns() - start > kWaitNs) return false;
    }
  }
}

// Named barrier whose result is the AND of every participant's predicate, so
// that a decision (e.g. "a wait timed out") is the same in all of them.
__device__ __forceinline__ bool bar_and(int id, int threads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, %2, %3, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(threads)
      : "memory");
  return r != 0;
}

// ---------------------------------------------------------------------------
// TMA: plain tiled loads, each CTA fetching its own tiles

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// L2 policy that keeps lines past streaming traffic (weights reused by every
// N tile of a GEMM), and the 2-D load that carries it as a cache hint.
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, %3}], "
      "[%4], %5;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 in, fp32 accumulate).
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every tcgen05.mma issued so far by this thread completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Shared-memory matrix descriptor, K-major operand, 128-byte swizzle: rows of
// 128 B, 8-row core groups 1024 B apart (SBO), LBO unused for swizzled K-major,
// descriptor version 1 (sm_100), layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr) {
  uint64_t desc = 0;
  desc |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  desc |= static_cast<uint64_t>(1) << 16;            // LBO (ignored)
  desc |= static_cast<uint64_t>(1024 >> 4) << 32;    // SBO
  desc |= static_cast<uint64_t>(1) << 46;            // version
  desc |= static_cast<uint64_t>(2) << 61;            // SWIZZLE_128B
  return desc;
}

// Instruction descriptor: BF16 x BF16 -> F32, both operands K-major.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int m, int n) {
  return (1u << 4)                                 // D = F32
         | (1u << 7)                               // A = BF16
         | (1u << 10)                              // B = BF16
         | (static_cast<uint32_t>(n >> 3) << 17)   // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);  // M / 16
}

// Instruction descriptor: F16 x F16 -> F32, both operands K-major.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int m, int n) {
  return (1u << 4)                                 // D = F32
         | (static_cast<uint32_t>(n >> 3) << 17)   // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);  // M / 16
}

// 32 lanes x 32 columns of 32-bit TMEM data into registers (one row per lane).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 16 columns (one row per lane).  The wait names the destination
// registers as operands, so no use of them can be scheduled before it.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15])::"memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 8 columns (one row per lane).
// 16 columns of this warp's TMEM lanes without the wait: registers hold the
// values only after tmem_wait_ld(), so several loads can be in flight at once.
__device__ __forceinline__ void tmem_ld16_async(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// Waits for this thread's TMEM loads; the registers are tied to the wait so
// that no use is scheduled above it.
template <int N>
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[N]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void named_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ bool elect_lane0() { return (threadIdx.x & 31) == 0; }

// ---------------------------------------------------------------------------
// activation math

// mish(x) = x * tanh(softplus(x)).  With e = exp(x), tanh(log(1 + e)) =
// ((1+e)^2 - 1) / ((1+e)^2 + 1) = n / (n + 2) where n = e * (e + 2); this
// identity needs one exponential and one division and has no cancellation for
// negative x (n -> 2e).  For x > 20, tanh(softplus(x)) == 1 in fp32.
__device__ __forceinline__ float mish_f(float x) {
  if (x > 20.0f) return x;
  const float e = expf(x);
  const float n = e * (e + 2.0f);
  return x * (n / (n + 2.0f));
}

// Mish with the fast exponential and division, for values rounded to fp16
// right afterwards (relative error ~1e-6, far below the fp16 step of 2^-11).
__device__ __forceinline__ float mish_fast(float x) {
  if (x > 20.0f) return x;
  const float e = __expf(x);
  const float n = e * (e + 2.0f);
  return x * __fdividef(n, n + 2.0f);
}

// mish_fast without a branch: the exponent is clamped at 20 and the ratio
// replaced by 1 above it, so the result equals mish_fast's for every input.
__device__ __forceinline__ float mish_sel(float x) {
  const float e = __expf(fminf(x, 20.0f));
  const float n = e * (e + 2.0f);
  const float r = __fdividef(n, n + 2.0f);
  return x * (x > 20.0f ? 1.0f : r);
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

// SiLU with the fast exponential and division, for the tensor path (its
// outputs are rounded to 16 bits; relative error ~1e-6).  For x < -87 the
// exponential overflows to inf and the quotient is -0, the limit of silu.
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// Grid barrier of a cooperative launch (every CTA resident) on a monotonic
// arrival counter sync[0]: barrier number `epoch` (from 1) passes once the
// counter reaches epoch * gridDim.x.  Thread 0 arrives with a GPU-scope
// release and polls with a GPU-scope acquire, between two CTA barriers.  The
// wait is bounded: after kWaitNs it records kErrGridBarrierTimeout and sets
// the abort word sync[2]; every CTA returns false at its next barrier once
// the abort word is set.  sync[0] and sync[2] start at zero for each launch.
__device__ inline bool coop_grid_sync(unsigned* sync, int* err, unsigned& epoch) {
  __shared__ int s_ok;
  __syncthreads();
  ++epoch;
  if (threadIdx.x == 0) {
    volatile unsigned* abort_flag = sync + 2;
    int ok = *abort_flag == 0u;
    if (ok) {
      const unsigned target = epoch * gridDim.x;
      asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(sync) : "memory");
      const uint64_t t0 = global_ns();
      for (uint32_t spin = 0;; ++spin) {
        unsigned v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(sync) : "memory");
        if (v >= target) break;
        if ((spin & 15u) == 15u) {
          if (*abort_flag != 0u) {
            ok = 0;
            break;
          }
          if (global_ns() - t0 > kWaitNs) {
            atomicCAS(err, 0, kErrGridBarrierTimeout);
            atomicExch(sync + 2, 1u);
            ok = 0;
            break;
          }
        }
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

// 2^x by the hardware approximation (MUFU.EX2, flush-to-zero)
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// 2^x for a pair of x <= 126 on the FMA pipe, so that a kernel bound by the
// MUFU unit can move some of its exponentials off it.  Range reduction
// x = k + r, k = round(x), r in [-0.5, 0.5], by the 1.5 * 2^23 rounding
// constant (its low mantissa bits then hold k); 2^r by the degree-5
// Chebyshev interpolant of 2^r on [-0.5, 0.5] in monomial form (nodes of
// degree 5, coefficients rounded to fp32; max relative error 2.4e-7 over the
// interval in fp32 Horner evaluation, against ex2.approx's 2^-22); 2^k added
// to the exponent field.  x is clamped at -125 so the exponent stays normal;
// 2^-125 stands in for the flushed-to-zero values of ex2.approx.ftz below it.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  x.x = fmaxf(x.x, -125.0f);
  x.y = fmaxf(x.y, -125.0f);
  const float2 t = __fadd2_rn(x, make_float2(kRound, kRound));
  const float2 k = __fadd2_rn(t, make_float2(-kRound, -kRound));
  const float2 r = __ffma2_rn(k, make_float2(-1.0f, -1.0f), x);
  float2 p = __ffma2_rn(make_float2(1.3390863e-3f, 1.3390863e-3f), r, make_float2(9.6760318e-3f, 9.6760318e-3f));
  p = __ffma2_rn(p, r, make_float2(5.5503570e-2f, 5.5503570e-2f));
  p = __ffma2_rn(p, r, make_float2(2.4022107e-1f, 2.4022107e-1f));
  p = __ffma2_rn(p, r, make_float2(6.9314718e-1f, 6.9314718e-1f));
  p = __ffma2_rn(p, r, make_float2(1.0000001f, 1.0000001f));
  // the low 9 bits of kRound's encoding are zero, so t's bits shifted by 23
  // are k in the exponent field
  return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23)));
}

// SiLU of a pair with one MUFU operation per element: x / (1 + 2^(-x log2 e)),
// the power by exp2_poly2 on the FMA pipe (argument clamped at 126: for
// x < -87 silu(x) is -0 to fp32 precision, and 1 + 2^126 keeps the reciprocal
// finite), the reciprocal by rcp.approx.  For values rounded to fp16 right
// afterwards (relative error ~1e-6).
__device__ __forceinline__ float2 silu2_fma(float2 x) {
  constexpr float kLog2e = 1.4426950408889634f;
  const float2 e = exp2_poly2(make_float2(fminf(-x.x * kLog2e, 126.0f), fminf(-x.y * kLog2e, 126.0f)));
  const float2 d = __fadd2_rn(e, make_float2(1.0f, 1.0f));
  float2 r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r.x) : "f"(d.x));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r.y) : "f"(d.y));
  return __fmul2_rn(x, r);
}

__device__ __forceinline__ float softplus_f(float x) { return fmaxf(x, 0.0f) + log1pf(expf(-fabsf(x))); }

__device__ __forceinline__ float half_lo(uint32_t packed) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(packed & 0xFFFFu)));
}
__device__ __forceinline__ float half_hi(uint32_t packed) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(packed >> 16)));
}

__device__ __forceinline__ float bf16_lo(uint32_t packed) { return __uint_as_float(packed << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t packed) { return __uint_as_float(packed & 0xFFFF0000u); }

// fp16 operand storage saturates at the largest finite value (never inf)
__device__ __forceinline__ __half to_half_sat(float v) { return __float2half_rn(fminf(fmaxf(v, -65504.0f), 65504.0f)); }

// fp16 of v with saturation at +-65504 in one conversion (cvt.rn.satfinite)
__device__ __forceinline__ __half half_satfinite(float v) {
  unsigned short r;
  asm("cvt.rn.satfinite.f16.f32 %0, %1;" : "=h"(r) : "f"(v));
  return __ushort_as_half(r);
}

// fp16 pair {lo, hi} with saturation at +-65504 (cvt.rn.satfinite; NaN stays NaN)
__device__ __forceinline__ uint32_t pack_half2_sat(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// Mish of a pair, x * n / (n + 2) with n = e (e + 2), e = 2^(min(x, 20) log2 e)
// by the hardware ex2 and reciprocal approximations; above 20 the quotient
// rounds to 1 in fp32, so the clamp changes nothing.  For values rounded to
// fp16 right afterwards (relative error ~1e-6).
__device__ __forceinline__ float2 mish2(float2 x) {
  constexpr float kLog2e = 1.4426950408889634f;
  const float2 t = __fmul2_rn(make_float2(fminf(x.x, 20.0f), fminf(x.y, 20.0f)), make_float2(kLog2e, kLog2e));
  const float2 e = make_float2(ex2_approx(t.x), ex2_approx(t.y));
  const float2 n = __fmul2_rn(e, __fadd2_rn(e, make_float2(2.0f, 2.0f)));
  const float2 d = __fadd2_rn(n, make_float2(2.0f, 2.0f));
  float2 r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r.x) : "f"(d.x));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r.y) : "f"(d.y));
  return __fmul2_rn(x, __fmul2_rn(n, r));
}

__device__ __forceinline__ uint32_t pack_half(float lo, float hi) {
  __half2 v = __halves2half2(to_half_sat(lo), to_half_sat(hi));
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

}  // namespace feb
