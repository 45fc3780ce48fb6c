// Persistent U-Net sampling program for small token counts (batch x horizon
// <= 16), sm_100a.
//
// One cooperative launch runs a whole DDIM / DDPM sampling call as a dataflow
// program: the FiLM condition GEMV once, then for every denoising step the
// convolutions of the forward in program order and the scheduler update.
// Every CTA (one per SM, 16 warps) walks the same op list and there is no grid
// barrier: an op waits only for the ops whose outputs it reads, on their
// completion counters, and a conv issues its first weight copies before that
// wait, so HBM keeps streaming weights while a dependency resolves.  At these
// sizes a forward is a stream of weights (0.5 GB per denoising step for the
// PushT-shaped model in bf16).
//
//  * Convolutions are split-K GEMVs on the warp-level tensor cores
//    (mma.sync m16n8k16, fp16 operands, fp32 accumulators) over units of 16
//    output rows x 16 K values (512 bytes of fp16 weights per plane, stored
//    fragment-ordered at load so each lane reads one 16-byte vector).  The
//    rows x K units are split evenly over the CTAs in row-major order, so a
//    CTA's units are one contiguous byte range, which one lane streams by
//    cp.async.bulk through a shared-memory ring; 15 warps consume it.
//  * A conv's output stays as its split-K partial segments: per row block one
//    segment per CTA whose units meet it.  Whoever reads the output adds the
//    bias, then the segments in segment order, so results are deterministic.
//    After writing its segments a CTA adds 1 to the conv's completion counter
//    (release); a consumer waits (acquire) until every CTA of the conv did.
//  * GroupNorm + Mish + FiLM / residual run in the consumer, while it stages
//    its input: every CTA sums the producer's segments into shared memory,
//    reduces the per-(sample, group) statistics itself (double, fixed order)
//    and stages the normalised activation as an fp16 pair hi + lo
//    (hi = fp16(x), lo = fp16(x - hi), ~22 bits of x; fp32-weight models also
//    add the W_lo * x_hi product).
//  * A block output (GroupNorm + Mish + residual) has several consumers: the
//    next block, a residual, a skip connection.  Its first consumer also
//    writes it to global memory (each CTA a slice); later consumers read that
//    copy once the first consumer's counter says it is complete.
//  * Counters are monotonic over the call: a step-s consumer waits for
//    (s + 1) x the producer's CTA count.  A conv of step s + 1 rewrites its
//    buffers only after everything of step s that read them completed, as
//    every op feeds the scheduler update that the next step's first convs
//    wait on.  While a conv runs, each CTA asks the L2 to prefetch its share
//    of the next conv's weights.
//
// Every wait is bounded (global timer); a timeout sets the device error word
// and a shared abort flag, after which every CTA leaves at its next wait.
// Data written inside the launch is read with ld.global.cg (L2), as L1 is not
// coherent across SMs.
#pragma once

#include "simt.cuh"

namespace feb {
namespace sp {

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kComputeWarps = kWarps - 1;  // warp 0 streams the weights
constexpr int kMaxTok = 16;    // tokens of one conv output
constexpr int kMaxSlots = 64;  // row blocks one CTA may touch per conv
constexpr int kRowPad = 8;     // fp16 padding per staged row (spreads banks)
constexpr int kMaxTaps = 5;
constexpr int kChunk = kComputeWarps * 2048;  // bytes of one weight copy (cp.async.bulk): a group per compute warp
constexpr int kMinStages = 2;
constexpr int kMaxStages = 8;
constexpr int kMaxSeg = 8;       // partial segments of a row block
constexpr int kMaxDeps = 6;      // counters one op waits on
constexpr int kGnQuads = 4;      // 4-channel quads (tokens) per thread when staging a normalised input
constexpr int kMaxStats = 256;   // (sample, group) pairs of a normalised input
// Trace stamps per (op, CTA): op start, dependencies met, normalised input
// loaded, input staged, compute warp 1 done, producer done, segments
// written, normalised input's statistics, normalised input transformed (by
// thread 0), op done.
constexpr int kTracePhases = 11;

enum OpKind : int { kOpConv = 0, kOpReduce = 1, kOpUpdate = 2 };

// Wait until *ctr >= base + per_step * step.
struct Dep {
  const unsigned* ctr;
  unsigned base, per_step;
};

// A conv output as its split-K segments: value(n, m) = bias[m] + the
// segments of row block m / 16 in order.
struct RawSrc {
  const float* P;     // [rbs][seg_max][T][16]
  const int* nseg;    // [rbs] segments of each row block
  const float* bias;  // [M] or null
  int seg_max;
  int T;              // tokens of the conv output
};

enum SrcKind : int { kSrcNone = 0, kSrcMat = 1, kSrcRaw = 2, kSrcGn = 3 };

// One channel range of a conv input.
//  kSrcMat: an fp32 tensor [T_in][C].
//  kSrcRaw: a conv output, or two phase convs interleaved in time (a
//           transposed conv: token b*2L + 2t + ph is phase ph's token b*L + t).
//  kSrcGn:  mish(GroupNorm(raw[0])), then FiLM (z = fs * z + fh, the rows
//           film_off (scale) and film_off + C (shift) of the condition and time
//           tables) or a residual (a conv output `res`, or the tensor `mat`).
struct StageSrc {
  int kind;
  int C;     // channels of the tensor
  int Cpad;  // channels it takes in the staged rows (C rounded up to 64; the rest are zero)
  const float* mat;
  RawSrc raw[2];
  int phases;
  int res_kind;  // kSrcGn: 0 none, 1 `res`, 2 `mat`
  RawSrc res;
  const float* gamma;
  const float* beta;
  int groups;
  int film;
  int film_off;
  float* materialize;  // kSrcGn: the activation is also written here ([T_in][C]), a slice per CTA
};

struct ConvOp {
  const uint4* w;  // [rb][ks][planes][32 lanes], fragment order
  int planes;      // 1: fp16 weights, 2: fp16 hi + lo
  int rbs, ks;
  int ic_pad;      // channels of the concatenated input; K = ntaps * ic_pad
  StageSrc src[2];  // channels [0, src[0].Cpad) and [src[0].Cpad, ic_pad); src[1].kind == kSrcNone: one source
  int samples, L_in, L_out, stride;
  int ntaps;
  int tap_off[kMaxTaps];  // input time = t * stride + tap_off
  int halo_lo, rows;      // staged rows per sample (input time + halo_lo)
  float* P;
  int seg_max;
  int T;
  int nct;         // CTAs the units are split over (every one of them has units)
  int cta0;        // the first of them: CTA cta0 + r (mod the grid) takes the r-th unit range
  int nslots;      // row blocks one CTA touches at most (slots per compute warp)
  int slots_off;   // shared-memory offset of the warp slots (after the staged input)
  int ring_off;    // shared-memory offset of the weight ring
  int stages;      // ring stages of kChunk bytes
  unsigned* done;  // completion counter
  // weights of the next conv in program order (L2 prefetch), or null
  const uint4* next_w;
  long long next_units;
  int next_planes;
};

// out[n][m] = value(n, m) of a conv output, n < T, m < M (all CTAs, grid-stride)
struct ReduceOp {
  RawSrc y;
  int M, T;
  float* out;
  unsigned* done;
};

// One CTA: eps[n][a] = y[n][a]; x = scheduler(x, eps); x_master and the next input
struct UpdateOp {
  RawSrc y;
  int cta;  // the CTA that runs it
  int A, H, Cin, samples;
  float* x_master;  // [T][A]
  float* x_in;      // [T][Cin] fp32
  const uint64_t* seeds;
  unsigned* done;
};

struct alignas(16) Op {
  int kind;
  int ndeps;
  Dep deps[kMaxDeps];
  union {
    ConvOp conv;
    ReduceOp reduce;
    UpdateOp update;
  };
};
static_assert(sizeof(Op) % 16 == 0, "ops are copied to shared memory in 16-byte pieces");

struct Program {
  const Op* ops;
  int n_pre;                   // ops run once, before the steps
  int n_step;                  // ops run at every step
  int steps;
  const int* step_t;           // [steps] timestep of each step (FiLM time row)
  const StepScalars* scalars;  // [steps]
  const float* film_cond;      // [samples][film_F], written by the pre ops
  const float* film_time;      // [timesteps][film_F]
  int film_F;
  unsigned* sync;              // [2] abort
  int* err;
  // null, or [executed op][CTA][kTracePhases] global-timer stamps of the call
  unsigned long long* trace;
};

// ---------------------------------------------------------------------------
// Shared-memory state of the program kernel, at namespace scope so that every
// function of the kernel names it directly: its fields are read with
// shared-memory instructions, never through pointers or copies in local
// memory (which, with nearly all of L1 given to shared memory, would cost L2
// round trips).

extern __shared__ __align__(128) uint8_t sp_smem[];  // staged input, warp slots, weight ring
__shared__ Program sp_pg;                            // the launch's parameters
__shared__ Op sp_op;                                 // the op being run
__shared__ int sp_uses[kMaxStages];                  // phases each ring buffer went through
__shared__ __align__(8) uint64_t sp_full[kMaxStages];   // ring buffer s: its copy landed
__shared__ __align__(8) uint64_t sp_empty[kMaxStages];  // ring buffer s: every compute warp is done with it
__shared__ float2 sp_stat[kMaxStats];                // GroupNorm (mean, 1 / std) per (sample, group)
__shared__ int sp_flag;                              // a CTA-wide decision of thread 0

// ---------------------------------------------------------------------------
// helpers

__device__ __forceinline__ void mma16816(float (&d)[4], const uint4& a, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}

// CTA whose range [U c / NC, U (c + 1) / NC) holds item u
__device__ __forceinline__ int cta_of(long long u, long long U, int NC) {
  int c = static_cast<int>((u * NC) / U);
  while (c + 1 < NC && (U * (c + 1)) / NC <= u) ++c;
  while (c > 0 && (U * c) / NC > u) --c;
  return c;
}

// Value of a conv output: the bias, then the segments in order.  Every row
// block has seg_max segment slots; the slots past its own segment count are
// never written and hold zeros, so all seg_max slots are requested at once
// (no wait for the count) and adding the zeros changes no sum.
__device__ __forceinline__ float y_at(const RawSrc& y, int n, int m) {
  const int rb = m >> 4;
  float v = y.bias != nullptr ? __ldg(y.bias + m) : 0.0f;
  const float* p = y.P + ((static_cast<long long>(rb) * y.seg_max) * y.T + n) * 16 + (m & 15);
  const long long stride = static_cast<long long>(y.T) * 16;
  float t[kMaxSeg];
#pragma unroll
  for (int s = 0; s < kMaxSeg; ++s) t[s] = s < y.seg_max ? __ldcg(p + s * stride) : 0.0f;
#pragma unroll
  for (int s = 0; s < kMaxSeg; ++s)
    if (s < y.seg_max) v += t[s];
  return v;
}

// The bias quad of channels m .. m + 3 (zeros without a bias).
__device__ __forceinline__ float4 bias_quad(const RawSrc& y, int m) {
  return y.bias != nullptr ? __ldg(reinterpret_cast<const float4*>(y.bias + m)) : make_float4(0.f, 0.f, 0.f, 0.f);
}

// The same for the four channels m .. m + 3 (m a multiple of 4), starting
// from the bias quad `v`: the segment layout keeps them in one 16-byte
// vector; the sums are y_at's, per channel.
template <int SEG>
__device__ __forceinline__ float4 y_quad_from(const RawSrc& y, int n, int m, float4 v) {
  const int rb = m >> 4;
  const float* p = y.P + ((static_cast<long long>(rb) * y.seg_max) * y.T + n) * 16 + (m & 15);
  const long long stride = static_cast<long long>(y.T) * 16;
  float4 t[SEG];
#pragma unroll
  for (int s = 0; s < SEG; ++s)
    t[s] = s < y.seg_max ? __ldcg(reinterpret_cast<const float4*>(p + s * stride)) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int s = 0; s < SEG; ++s)
    if (s < y.seg_max) {
      v.x += t[s].x;
      v.y += t[s].y;
      v.z += t[s].z;
      v.w += t[s].w;
    }
  return v;
}

template <int SEG>
__device__ __forceinline__ float4 y_quad(const RawSrc& y, int n, int m) {
  return y_quad_from<SEG>(y, n, m, bias_quad(y, m));
}

// Trace stamp `phase` of the executed op `exec` (FLOWEDGE_PROGRAM_TRACE)
__device__ __forceinline__ void trace_stamp(int exec, int phase) {
  if (sp_pg.trace != nullptr)
    sp_pg.trace[(static_cast<long long>(exec) * gridDim.x + blockIdx.x) * kTracePhases + phase] = global_ns();
}

__device__ __forceinline__ void release_add(unsigned* ctr) {
  asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
}

__device__ __forceinline__ volatile unsigned* abort_word() { return sp_pg.sync + 2; }

__device__ __forceinline__ void raise_abort(int code) {
  atomicCAS(sp_pg.err, 0, code);
  atomicExch(sp_pg.sync + 2, 1u);
}

// Thread 0: bounded wait for the current op's dependencies at `step`.  On a
// timeout it records kErrDependencyTimeout and sets the abort word; false once
// aborted.
__device__ bool wait_deps(int step) {
  const uint64_t t0 = global_ns();
  for (int i = 0; i < sp_op.ndeps; ++i) {
    const unsigned* ctr = sp_op.deps[i].ctr;
    const unsigned target = sp_op.deps[i].base + sp_op.deps[i].per_step * static_cast<unsigned>(step);
    for (uint32_t spin = 0;; ++spin) {
      unsigned v;
      asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
      if (v >= target) break;
      if (spin >= 4) __nanosleep(64);  // many CTAs poll one counter: back off after a few tries
      if ((spin & 15u) == 15u) {
        if (*abort_word() != 0u) return false;
        if (global_ns() - t0 > kWaitNs) {
          raise_abort(kErrDependencyTimeout);
          return false;
        }
      }
    }
  }
  // the relaxed reads that saw every counter, then one acquire fence (an abort
  // raised meanwhile is seen at the next wait)
  asm volatile("fence.acq_rel.gpu;" ::: "memory");
  return true;
}

__device__ __forceinline__ void store_pair(__half* xh, __half* xl, int off, const float4& v) {
  const __half h0 = __float2half_rn(v.x), h1 = __float2half_rn(v.y), h2 = __float2half_rn(v.z),
               h3 = __float2half_rn(v.w);
  __half2* dh = reinterpret_cast<__half2*>(xh + off);
  __half2* dl = reinterpret_cast<__half2*>(xl + off);
  dh[0] = __halves2half2(h0, h1);
  dh[1] = __halves2half2(h2, h3);
  dl[0] = __halves2half2(__float2half_rn(v.x - __half2float(h0)), __float2half_rn(v.y - __half2float(h1)));
  dl[1] = __halves2half2(__float2half_rn(v.z - __half2float(h2)), __float2half_rn(v.w - __half2float(h3)));
}

// The staged input: fp16 hi / lo rows [sample][time + halo_lo] of rs halfs,
// one zero row last.
__device__ __forceinline__ int staged_rs() { return sp_op.conv.ic_pad + kRowPad; }
__device__ __forceinline__ __half* staged_hi() { return reinterpret_cast<__half*>(sp_smem); }
__device__ __forceinline__ __half* staged_lo() {
  return staged_hi() + (sp_op.conv.samples * sp_op.conv.rows + 1) * staged_rs();
}

// ---------------------------------------------------------------------------
// staging of a conv input

// Segments a source's conv outputs have at most (1 when no row block is split
// over CTAs).
__device__ __forceinline__ int src_segments(const StageSrc& s) {
  if (s.kind == kSrcMat || s.kind == kSrcNone) return 1;
  int m = s.raw[0].seg_max;
  if (s.kind == kSrcRaw && s.phases == 2) m = max(m, s.raw[1].seg_max);
  if (s.kind == kSrcGn && s.res_kind == 1) m = max(m, s.res.seg_max);
  return m;
}

// Channel quad (token n of the input tensor, channels c .. c + 3) of a Mat or
// Raw source.
template <int SEG>
__device__ __forceinline__ float4 src_quad(const StageSrc& s, int n, int c, int L) {
  if (s.kind == kSrcMat) return __ldcg(reinterpret_cast<const float4*>(s.mat + static_cast<long long>(n) * s.C + c));
  if (s.phases == 2) {
    const int b = n / L, t = n - b * L;
    return y_quad<SEG>(s.raw[t & 1], b * (L >> 1) + (t >> 1), c);
  }
  return y_quad<SEG>(s.raw[0], n, c);
}

// Source `si` (a Mat / Raw source) into channels [off, off + Cpad), every
// staged row (rows outside the sequence, the last row and the channels past C
// are zero).  Loads in batches of BATCH quads per thread so their latencies
// overlap.
template <int BATCH, int SEG>
__device__ __noinline__ void stage_plain(int si, int off) {
  const ConvOp& op = sp_op.conv;
  const StageSrc& s = op.src[si];
  __half* xh = staged_hi();
  __half* xl = staged_lo();
  const int rs = staged_rs();
  const int nrows = op.samples * op.rows;
  const int q4 = s.Cpad / 4;
  const int items = (nrows + 1) * q4;
  for (int base = 0; base < items; base += BATCH * kThreads) {
    float4 v[BATCH];
#pragma unroll
    for (int j = 0; j < BATCH; ++j) {
      const int i = base + j * kThreads + static_cast<int>(threadIdx.x);
      v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i < items) {
        const int r = i / q4;
        const int c = (i - r * q4) * 4;
        if (r < nrows && c < s.C) {
          const int b = r / op.rows;
          const int t_in = r - b * op.rows - op.halo_lo;
          if (t_in >= 0 && t_in < op.L_in) v[j] = src_quad<SEG>(s, b * op.L_in + t_in, c, op.L_in);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < BATCH; ++j) {
      const int i = base + j * kThreads + static_cast<int>(threadIdx.x);
      if (i < items) {
        const int r = i / q4;
        const int c = (i - r * q4) * 4;
        store_pair(xh, xl, r * rs + off + c, v[j]);
      }
    }
  }
}

// Source `si` (kSrcGn) into channels [off, off + Cpad) (the channels past C
// are zero).  Thread t owns the
// channel quad c = 4 (t % (C / 4)) of the tokens t / (C / 4) + j kThreads /
// (C / 4) (the host requires C / 4 to divide kThreads and the tokens to fit
// kGnQuads per thread), so every load - the conv values, the residual, gamma
// / beta and the FiLM rows - goes out in one round (ROUND quads at a time for
// split conv outputs).  Each thread sums its quads (double) into shared
// memory, aliasing the staged rows (dead until they are written), where one
// warp per (sample, group) adds them in a fixed order; then every thread
// normalises its quads.  Sums match the reference GroupNorm: biased variance
// E[x^2] - E[x]^2 in double, clamped at 0, eps 1e-5.
template <int SEG, int ROUND>
__device__ __noinline__ void stage_gn(int si, int off, int step, int rel, int exec) {
  const ConvOp& op = sp_op.conv;
  const StageSrc& s = op.src[si];
  float* temp = reinterpret_cast<float*>(sp_smem);
  const int C = s.C, q4 = C / 4, L = op.L_in;
  const int T_in = op.samples * L;
  const int tid = static_cast<int>(threadIdx.x);
  const int c = (tid % q4) * 4;
  const int n0 = tid / q4, dn = kThreads / q4;
  const int F = sp_pg.film_F;
  const float* ft = s.film ? sp_pg.film_time + static_cast<long long>(sp_pg.step_t[step]) * F + s.film_off : nullptr;
  const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);
  const float4 ga = __ldg(reinterpret_cast<const float4*>(s.gamma + c));
  const float4 be = __ldg(reinterpret_cast<const float4*>(s.beta + c));
  const float4 ts = s.film ? __ldg(reinterpret_cast<const float4*>(ft + c)) : zero4;
  const float4 th = s.film ? __ldg(reinterpret_cast<const float4*>(ft + C + c)) : zero4;
  // the thread's channel quad is the same for all its tokens: its bias, and
  // (batch 1) its FiLM condition rows, are loaded once
  const float4 yb = bias_quad(s.raw[0], c);
  const float4 rb = s.res_kind == 1 ? bias_quad(s.res, c) : zero4;
  const bool one_sample = op.samples == 1;
  const float* fc0 = s.film ? sp_pg.film_cond + s.film_off : nullptr;
  const float4 fs0 = s.film && one_sample ? __ldcg(reinterpret_cast<const float4*>(fc0 + c)) : zero4;
  const float4 fh0 = s.film && one_sample ? __ldcg(reinterpret_cast<const float4*>(fc0 + C + c)) : zero4;
  // y: conv values; a1 / a2: the FiLM condition rows (scale / shift), or a1 the residual
  float4 y[kGnQuads], a1[kGnQuads], a2[kGnQuads];
#pragma unroll
  for (int j0 = 0; j0 < kGnQuads; j0 += ROUND) {
#pragma unroll
    for (int j = j0; j < j0 + ROUND; ++j) {
      const int n = n0 + j * dn;
      y[j] = a1[j] = a2[j] = zero4;
      if (n < T_in) {
        y[j] = y_quad_from<SEG>(s.raw[0], n, c, yb);
        if (s.film) {
          if (one_sample) {
            a1[j] = fs0;
            a2[j] = fh0;
          } else {
            const float* fc = fc0 + static_cast<long long>(n / L) * F;
            a1[j] = __ldcg(reinterpret_cast<const float4*>(fc + c));
            a2[j] = __ldcg(reinterpret_cast<const float4*>(fc + C + c));
          }
        } else if (s.res_kind == 1) {
          a1[j] = y_quad_from<SEG>(s.res, n, c, rb);
        } else if (s.res_kind == 2) {
          a1[j] = __ldcg(reinterpret_cast<const float4*>(s.mat + static_cast<long long>(n) * C + c));
        }
      }
    }
  }
  // per-quad partial sums (double, fixed order) of the thread's own values
  double2* part = reinterpret_cast<double2*>(temp);  // [T_in][C / 4]
#pragma unroll
  for (int j = 0; j < kGnQuads; ++j) {
    const int n = n0 + j * dn;
    if (n < T_in) {
      const double x0 = y[j].x, x1 = y[j].y, x2 = y[j].z, x3 = y[j].w;
      part[n * q4 + (c >> 2)] = make_double2(((x0 + x1) + x2) + x3, ((x0 * x0 + x1 * x1) + x2 * x2) + x3 * x3);
    }
  }
  __syncthreads();
  if (tid == 0) trace_stamp(exec, 2);
  // one warp per (sample, group): its L x cpg / 4 quad sums, in a fixed order
  const int warp = tid >> 5, lane = tid & 31;
  const int cpg = C / s.groups, qpg = cpg / 4;
  for (int item = warp; item < op.samples * s.groups; item += kWarps) {
    const int b = item / s.groups, g = item - b * s.groups;
    double s1 = 0.0, s2 = 0.0;
    const double2* base = part + b * L * q4 + g * qpg;
    for (int e = lane; e < L * qpg; e += 32) {
      const int t = e / qpg;
      const double2 v = base[t * q4 + (e - t * qpg)];
      s1 += v.x;
      s2 += v.y;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
      s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    }
    if (lane == 0) {
      const double cnt = static_cast<double>(cpg) * L;
      const double mean = s1 / cnt;
      const double var = fmax(0.0, s2 / cnt - mean * mean);
      sp_stat[item] = make_float2(static_cast<float>(mean), static_cast<float>(1.0 / sqrt(var + 1e-5)));
    }
  }
  __syncthreads();
  if (tid == 0) trace_stamp(exec, 8);
  __half* xh = staged_hi();
  __half* xl = staged_lo();
  const int rs = staged_rs();
  const int gq = c / cpg;
  const float gv[4] = {ga.x, ga.y, ga.z, ga.w}, bv[4] = {be.x, be.y, be.z, be.w};
  const float tsv[4] = {ts.x, ts.y, ts.z, ts.w}, thv[4] = {th.x, th.y, th.z, th.w};
  // quad j of this thread is quad tid + j * kThreads of the tensor; the CTA at
  // place (quad mod nct) writes it out
  const int step_mod = kThreads % op.nct;
  int slice = tid % op.nct;
#pragma unroll
  for (int j = 0; j < kGnQuads; ++j, slice = (slice + step_mod) % op.nct) {
    const int n = n0 + j * dn;
    if (n < T_in) {
      const int b = n / L, t = n - b * L;
      const float2 st = sp_stat[b * s.groups + gq];
      const float z0[4] = {y[j].x, y[j].y, y[j].z, y[j].w};
      const float v1[4] = {a1[j].x, a1[j].y, a1[j].z, a1[j].w}, v2[4] = {a2[j].x, a2[j].y, a2[j].z, a2[j].w};
      float z[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        // fast exponential and division: ~1e-6 relative, below the fp16 hi / lo staging of any step after
        const float v = mish_fast((z0[q] - st.x) * (st.y * gv[q]) + bv[q]);
        // FiLM: (condition + time scale) * v + (condition + time shift); else v + residual
        z[q] = s.film ? (v1[q] + tsv[q]) * v + (v2[q] + thv[q]) : v + v1[q];
      }
      const float4 out = make_float4(z[0], z[1], z[2], z[3]);
      if (s.materialize != nullptr && slice == rel)
        *reinterpret_cast<float4*>(s.materialize + static_cast<long long>(n) * C + c) = out;
      store_pair(xh, xl, (b * op.rows + t + op.halo_lo) * rs + off + c, out);
    }
  }
  if (tid == 0) trace_stamp(exec, 9);
  // rows of this channel range outside the sequence (halo_lo before and
  // rows - L - halo_lo after each sample's), and the last row, are zero
  const int pad_rows = op.rows - L;
  const int zrows = op.samples * pad_rows + 1;
  for (int i = tid; i < zrows * q4; i += kThreads) {
    const int z = i / q4;
    const int b = z / max(pad_rows, 1), k = z - b * max(pad_rows, 1);
    const int rr = z == zrows - 1 ? op.samples * op.rows : b * op.rows + (k < op.halo_lo ? k : L + k);
    store_pair(xh, xl, rr * rs + off + (i - z * q4) * 4, zero4);
  }
  // and so are the padding channels [C, Cpad) of every row
  const int pq = (s.Cpad - C) / 4;
  for (int i = tid; i < (op.samples * op.rows + 1) * pq; i += kThreads) {
    const int rr = i / pq;
    store_pair(xh, xl, rr * rs + off + C + (i - rr * pq) * 4, zero4);
  }
}

// ---------------------------------------------------------------------------
// convolution (split-K GEMV on mma.sync)

// Units are consumed in groups of kGroupBytes (4 units of fp16 weights, or 2
// units of hi + lo planes): a group never crosses a tap or a row block, so its
// position is computed once and its units are independent MMAs.  A CTA's
// range is a whole number of groups: CTA r of the conv takes groups
// [Ug r / nct, Ug (r + 1) / nct) of the Ug = rbs * ks / G groups.
constexpr int kGroupBytes = 2048;

// Weights reach shared memory by cp.async.bulk: a CTA's units are one
// contiguous byte range, copied in kChunk pieces (one group per compute warp)
// through a ring of `stages` buffers by warp 0 (lane 0); compute warp w takes
// group w - 1 of every chunk, reads its A fragments from the ring (16 bytes
// per lane, conflict-free) and releases the buffer on its "empty" mbarrier.
// Per-warp partial sums of each row block go to a (warp, row block) slot and
// are combined in warp order.  The mbarriers are initialised once per launch;
// sp_uses[s] counts the phases ring buffer s went through in earlier convs of
// the launch, so chunk c of this conv waits on parity
// (sp_uses[c % stages] + c / stages) & 1.  The ring runs to its end even
// after an abort (the MMAs are skipped then), so no copy is left in flight;
// its waits are bounded by time only.

// Conv geometry of this CTA, recomputed from sp_op where needed.
struct ConvRange {
  long long cu0, cu1;  // unit range
  int cta;             // place among the conv's CTAs
};

template <int PLANES>
__device__ __forceinline__ ConvRange conv_range() {
  constexpr int G = kGroupBytes / (PLANES * 512);
  const ConvOp& op = sp_op.conv;
  ConvRange r;
  // consecutive convs use rotated CTA ranges, so a conv's CTAs are free to
  // fetch its weights while the previous conv still runs
  r.cta = (static_cast<int>(blockIdx.x) - op.cta0 + static_cast<int>(gridDim.x)) % static_cast<int>(gridDim.x);
  const long long Ug = static_cast<long long>(op.rbs) * (op.ks / G);
  r.cu0 = r.cta < op.nct ? G * (Ug * r.cta / op.nct) : 0;
  r.cu1 = r.cta < op.nct ? G * (Ug * (r.cta + 1) / op.nct) : 0;
  return r;
}

// Copy chunk c of this CTA's range into its ring buffer (lane 0 of warp 0).
template <int PLANES>
__device__ __forceinline__ void issue_chunk(int c, long long cu0, int ngroups) {
  const ConvOp& op = sp_op.conv;
  const int st = c % op.stages;
  const int g0 = c * kComputeWarps;
  const int ng = ngroups - g0 < kComputeWarps ? ngroups - g0 : kComputeWarps;
  const unsigned bytes = static_cast<unsigned>(ng) * kGroupBytes;
  const char* src = reinterpret_cast<const char*>(op.w) + cu0 * (PLANES * 512) + static_cast<long long>(g0) * kGroupBytes;
  mbar_arrive_expect_tx(&sp_full[st], bytes);
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(sp_smem + op.ring_off + st * kChunk)),
      "l"(src), "r"(bytes), "r"(smem_u32(&sp_full[st]))
      : "memory");
}

// A compute warp: group (warp - 1) of every ring chunk.  PACKED (<= 4
// tokens): one n = 8 tile holds x_hi (columns 0-3) and x_lo (columns 4-7) of
// the tokens, so W * (x_hi + x_lo) is one MMA and the halves are added at
// flush.  Returns false once the ring failed (warp-uniform).  An abort raised
// by another CTA is not polled here (that would put an L2 round trip on every
// conv): the ring waits are time-bounded and the next dependency wait sees it.
template <int PLANES, bool PACKED>
__device__ __noinline__ bool consume(long long cu0, int ngroups, int nchunks, int rb_lo, bool ok) {
  constexpr int kUnitBytes = PLANES * 512;
  constexpr int G = kGroupBytes / kUnitBytes;
  constexpr int NB = PACKED ? 1 : 2;  // n blocks of 8 tokens
  const ConvOp& op = sp_op.conv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cw = warp - 1;
  const int g = lane >> 2, t4 = lane & 3;
  const int T = op.T;
  const bool two_nb = T > 8;
  const int nrows = op.samples * op.rows;
  const int rs = staged_rs();
  const __half* xh = staged_hi();
  const __half* xl = staged_lo();
  const int nslots = op.nslots;
  const int stages = op.stages;
  float* slots = reinterpret_cast<float*>(sp_smem + op.slots_off);
  int* touched = reinterpret_cast<int*>(slots + kComputeWarps * nslots * 16 * T);
  const uint8_t* ring = sp_smem + op.ring_off;
  int no_abort = 0;
  volatile int* ring_abort = &no_abort;
  int tap_row[NB][kMaxTaps];  // staged row of this lane's token for every tap (nrows: zero row)
#pragma unroll
  for (int nb = 0; nb < NB; ++nb) {
    const int n = PACKED ? (g & 3) : nb * 8 + g;
    int base = -1;
    if (n < T) {
      const int b = n / op.L_out;
      const int t = n - b * op.L_out;
      base = b * op.rows + t * op.stride + op.halo_lo;
    }
#pragma unroll
    for (int j = 0; j < kMaxTaps; ++j) tap_row[nb][j] = (base >= 0 && j < op.ntaps) ? base + op.tap_off[j] : nrows;
  }
  const int ks = op.ks, ic_pad = op.ic_pad;
  // accumulator chains: [unit parity][n block][x hi / x lo]
  float acc[2][NB][2][4];
  auto zero = [&]() {
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int hl = 0; hl < 2; ++hl)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[u][nb][hl][i] = 0.0f;
  };
  auto total = [&](int nb, int i) {
    return (acc[0][nb][0][i] + acc[1][nb][0][i]) + (acc[0][nb][1][i] + acc[1][nb][1][i]);
  };
  zero();
  int cur = -1;  // row block of the accumulators, or -1
  auto flush = [&]() {
    const int sidx = cur - rb_lo;
    if (sidx >= 0 && sidx < nslots) {
      float* sl = slots + (cw * nslots + sidx) * (16 * T);
      if constexpr (PACKED) {
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = total(0, i);
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] += __shfl_xor_sync(0xffffffffu, v[i], 2);  // hi column + lo column
        const int n0 = 2 * t4;
        if (t4 < 2 && n0 < T) {
          sl[g * T + n0] = v[0];
          sl[(g + 8) * T + n0] = v[2];
        }
        if (t4 < 2 && n0 + 1 < T) {
          sl[g * T + n0 + 1] = v[1];
          sl[(g + 8) * T + n0 + 1] = v[3];
        }
      } else {
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
          const int n0 = nb * 8 + 2 * t4;
          if (n0 < T) {
            sl[g * T + n0] = total(nb, 0);
            sl[(g + 8) * T + n0] = total(nb, 2);
          }
          if (n0 + 1 < T) {
            sl[g * T + n0 + 1] = total(nb, 1);
            sl[(g + 8) * T + n0 + 1] = total(nb, 3);
          }
        }
      }
      if (lane == 0) touched[warp * nslots + sidx] = 1;
    } else if (lane == 0) {
      atomicCAS(sp_pg.err, 0, kErrProgramLayout);  // the host bounds the row blocks of a CTA; never expected
    }
  };
  bool ring_ok = true;
  for (int c = 0; c < nchunks && ring_ok; ++c) {
    const int st = c % stages;
    ring_ok = __all_sync(0xffffffffu, mbar_wait(&sp_full[st], (sp_uses[st] + c / stages) & 1, ring_abort));
    if (!ring_ok && lane == 0) raise_abort(kErrWaitTimeoutMma);
    ok = ok && ring_ok;  // warp-uniform: the MMAs below are warp-collective
    const int gi = c * kComputeWarps + cw;
    if (ok && gi < ngroups) {
      const long long q = cu0 + static_cast<long long>(gi) * G;  // first unit of the group
      const int rb = static_cast<int>(q / ks);
      const int k = static_cast<int>(q - static_cast<long long>(rb) * ks);
      const int tap = (k * 16) / ic_pad;
      const int ch = k * 16 - tap * ic_pad;
      if (rb != cur) {
        if (cur >= 0) flush();
        zero();
        cur = rb;
      }
      const uint8_t* abuf = ring + st * kChunk + cw * kGroupBytes + lane * 16;
      if constexpr (PACKED) {
        int r = nrows;
#pragma unroll
        for (int j = 0; j < kMaxTaps; ++j)
          if (j == tap) r = tap_row[0][j];
        const uint32_t* px = reinterpret_cast<const uint32_t*>((g < 4 ? xh : xl) + r * rs + ch + 2 * t4);
#pragma unroll
        for (int j = 0; j < G; ++j) {
          uint4 a[PLANES];
#pragma unroll
          for (int pl = 0; pl < PLANES; ++pl) a[pl] = *reinterpret_cast<const uint4*>(abuf + j * kUnitBytes + pl * 512);
          const uint32_t b0 = px[8 * j], b1 = px[8 * j + 4];
          mma16816(acc[j & 1][0][0], a[0], b0, b1);
          if constexpr (PLANES == 2) mma16816(acc[j & 1][0][1], a[1], g < 4 ? b0 : 0u, g < 4 ? b1 : 0u);
        }
      } else {
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
          if (nb == 0 || two_nb) {
            int r = nrows;
#pragma unroll
            for (int j = 0; j < kMaxTaps; ++j)
              if (j == tap) r = tap_row[nb][j];
            const int off = r * rs + ch + 2 * t4;
            const uint32_t* ph = reinterpret_cast<const uint32_t*>(xh + off);
            const uint32_t* pl = reinterpret_cast<const uint32_t*>(xl + off);
#pragma unroll
            for (int j = 0; j < G; ++j) {
              uint4 a[PLANES];
#pragma unroll
              for (int p2 = 0; p2 < PLANES; ++p2) a[p2] = *reinterpret_cast<const uint4*>(abuf + j * kUnitBytes + p2 * 512);
              const uint32_t b0h = ph[8 * j], b1h = ph[8 * j + 4];  // channels +0 / +8
              const uint32_t b0l = pl[8 * j], b1l = pl[8 * j + 4];
              mma16816(acc[j & 1][nb][0], a[0], b0h, b1h);
              mma16816(acc[j & 1][nb][1], a[0], b0l, b1l);
              if constexpr (PLANES == 2) mma16816(acc[j & 1][nb][1], a[1], b0h, b1h);
            }
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sp_empty[st]);
  }
  if (ok && cur >= 0) flush();
  return ok;
}

template <int PLANES>
__device__ __noinline__ bool run_conv(int step, int exec) {
  constexpr int kUnitBytes = PLANES * 512;
  constexpr int G = kGroupBytes / kUnitBytes;
  const ConvOp& op = sp_op.conv;
  const ConvRange rg = conv_range<PLANES>();
  if (rg.cu0 == rg.cu1) return true;  // uniform across the CTA (an abort is seen at the next wait)
  const int cta = rg.cta;
  const long long cu0 = rg.cu0;
  const int NC = op.nct;
  const long long gpr = op.ks / G;
  const long long Ug = static_cast<long long>(op.rbs) * gpr;
  const int stages = op.stages;
  const int ngroups = static_cast<int>((rg.cu1 - cu0) / G);
  const int nchunks = (ngroups + kComputeWarps - 1) / kComputeWarps;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    // the first copies go out before the dependency wait: weights do not
    // depend on the activations (earlier ops wrote this shared memory through
    // the generic proxy)
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    for (int c = 0; c < stages && c < nchunks; ++c) issue_chunk<PLANES>(c, cu0, ngroups);
    // the rest of this CTA's weights into L2 (the ring refills then come from there)
    const char* wsrc = reinterpret_cast<const char*>(op.w) + cu0 * kUnitBytes;
    const long long ring_bytes = static_cast<long long>(stages) * kChunk;
    const long long my_bytes = static_cast<long long>(ngroups) * kGroupBytes;
    for (long long o = ring_bytes; o < my_bytes; o += 65536) {
      const unsigned chunk = static_cast<unsigned>(my_bytes - o < 65536 ? my_bytes - o : 65536);
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(wsrc + o), "r"(chunk) : "memory");
    }
    // a 1 / nct share of the next conv's weights into L2
    if (op.next_w != nullptr) {
      const long long nu0 = op.next_units * cta / NC, nu1 = op.next_units * (cta + 1) / NC;
      const char* base = reinterpret_cast<const char*>(op.next_w) + nu0 * op.next_planes * 512;
      const long long bytes = (nu1 - nu0) * op.next_planes * 512;
      for (long long o = 0; o < bytes; o += 65536) {
        const unsigned chunk = static_cast<unsigned>(bytes - o < 65536 ? bytes - o : 65536);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(base + o), "r"(chunk) : "memory");
      }
    }
    sp_flag = wait_deps(step) ? 1 : 0;
    trace_stamp(exec, 1);
  }
  __syncthreads();
  bool ok = sp_flag != 0;

  // stage the input: a normalised source first (its buffer aliases the
  // staged rows), then a plain one
  if (ok) {
    int off = 0;
    for (int si = 0; si < 2; ++si) {
      const StageSrc& s = op.src[si];
      if (s.kind == kSrcGn) {
        const int nseg = src_segments(s);
        if (nseg == 1) stage_gn<1, 4>(si, off, step, cta, exec);
        else if (nseg == 2) stage_gn<2, 2>(si, off, step, cta, exec);
        else if (nseg <= 4) stage_gn<4, 1>(si, off, step, cta, exec);
        else stage_gn<kMaxSeg, 1>(si, off, step, cta, exec);
      }
      off += s.kind == kSrcNone ? 0 : s.Cpad;
    }
    off = 0;
    for (int si = 0; si < 2; ++si) {
      const StageSrc& s = op.src[si];
      const int nseg = src_segments(s);
      if (s.kind == kSrcMat || (s.kind == kSrcRaw && nseg == 1)) stage_plain<8, 1>(si, off);
      else if (s.kind == kSrcRaw && nseg <= 4) stage_plain<4, 4>(si, off);
      else if (s.kind == kSrcRaw) stage_plain<2, kMaxSeg>(si, off);
      off += s.kind == kSrcNone ? 0 : s.Cpad;
    }
  }
  const int nslots = op.nslots;
  const int T = op.T;
  float* slots = reinterpret_cast<float*>(sp_smem + op.slots_off);
  int* touched = reinterpret_cast<int*>(slots + kComputeWarps * nslots * 16 * T);
  for (int i = threadIdx.x; i < kWarps * nslots; i += kThreads) touched[i] = 0;
  __syncthreads();
  if (threadIdx.x == 0) trace_stamp(exec, 3);

  const int rb_lo = static_cast<int>(cu0 / op.ks);
  if (warp == 0) {
    // producer: refill each buffer once every compute warp released it
    if (lane == 0) {
      int no_abort = 0;
      volatile int* ring_abort = &no_abort;
      bool pok = true;
      for (int c = stages; c < nchunks && pok; ++c) {
        const int st = c % stages;
        pok = mbar_wait(&sp_empty[st], (sp_uses[st] + (c / stages) - 1) & 1, ring_abort);
        if (pok) issue_chunk<PLANES>(c, cu0, ngroups);
      }
      if (!pok) raise_abort(kErrWaitTimeoutProducer);
      trace_stamp(exec, 5);
    }
  } else {
    if (T <= 4) ok = consume<PLANES, true>(cu0, ngroups, nchunks, rb_lo, ok);
    else ok = consume<PLANES, false>(cu0, ngroups, nchunks, rb_lo, ok);
    if (warp == 1 && lane == 0) trace_stamp(exec, 4);
  }
  // every warp saw no failure: the CTA goes on together either way
  const bool all_ok = __syncthreads_and(ok ? 1 : 0) != 0;
  // phases each ring buffer went through in this conv (every chunk completes
  // one phase of its `full` and of its `empty` barrier)
  if (threadIdx.x < stages) sp_uses[threadIdx.x] += (nchunks - static_cast<int>(threadIdx.x) + stages - 1) / stages;
  if (!all_ok) return false;

  // combine the warps' slots per row block (warp order) and write this CTA's segment
  const int slot_floats = 16 * T;
  const int rb_hi = static_cast<int>((rg.cu1 - 1) / op.ks);
  const int total_f = (rb_hi - rb_lo + 1) * slot_floats;
  for (int i = threadIdx.x; i < total_f; i += kThreads) {
    const int rbi = i / slot_floats;
    const int e = i - rbi * slot_floats;
    const int rb = rb_lo + rbi;
    float v = 0.0f;
    if (rbi < nslots)
      for (int w = 1; w < kWarps; ++w)
        if (touched[w * nslots + rbi]) v += slots[((w - 1) * nslots + rbi) * slot_floats + e];
    const int seg = op.seg_max == 1 ? 0 : cta - cta_of(static_cast<long long>(rb) * gpr, Ug, NC);
    const int m = e / T, n = e - m * T;
    op.P[((static_cast<long long>(rb) * op.seg_max + seg) * T + n) * 16 + m] = v;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    trace_stamp(exec, 6);
    release_add(op.done);
  }
  return true;
}

// out[n][m] = value(n, m) (every CTA, grid-stride)
__device__ __noinline__ bool run_reduce(int step) {
  const ReduceOp& op = sp_op.reduce;
  if (threadIdx.x == 0) sp_flag = wait_deps(step) ? 1 : 0;
  __syncthreads();
  if (sp_flag == 0) return false;
  const long long total = static_cast<long long>(op.T) * op.M;
  for (long long i = blockIdx.x * static_cast<long long>(kThreads) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * kThreads) {
    const int n = static_cast<int>(i / op.M);
    const int m = static_cast<int>(i - static_cast<long long>(n) * op.M);
    op.out[i] = y_at(op.y, n, m);
  }
  __syncthreads();
  if (threadIdx.x == 0) release_add(op.done);
  return true;
}

// The scheduler update, on one CTA (the others go on to the next step's
// convs, which wait on this op's counter)
__device__ __noinline__ bool run_update(int step) {
  const UpdateOp& op = sp_op.update;
  if (static_cast<int>(blockIdx.x) != op.cta) return true;
  if (threadIdx.x == 0) sp_flag = wait_deps(step) ? 1 : 0;
  __syncthreads();
  if (sp_flag == 0) return false;
  const StepScalars& s = sp_pg.scalars[step];
  const int total = op.samples * op.H * op.A;
  for (int i = threadIdx.x; i < total; i += kThreads) {
    const int n = i / op.A;
    const int a = i - n * op.A;
    const int b = n / op.H;
    const int t = n - b * op.H;
    const float eps = y_at(op.y, n, a);
    const float x = scheduler_update(s, __ldcg(op.x_master + i), eps, op.seeds != nullptr ? op.seeds[b] : 0,
                                     static_cast<uint64_t>(t) * op.A + a, op.H * op.A);
    op.x_master[i] = x;
    op.x_in[static_cast<long long>(n) * op.Cin + a] = x;
  }
  __syncthreads();
  if (threadIdx.x == 0) release_add(op.done);
  return true;
}

template <int PLANES>
static __global__ void __launch_bounds__(kThreads, 1) unet_program_kernel(const Program pg) {
  if (threadIdx.x == 0) {
    sp_pg = pg;
    for (int st = 0; st < kMaxStages; ++st) {
      mbar_init(&sp_full[st], 1);              // full: the copy landed
      mbar_init(&sp_empty[st], kComputeWarps);  // empty: every compute warp is done with it
      sp_uses[st] = 0;
    }
    fence_mbar_init();
  }
  int executed = 0;
  auto run = [&](const Op* src, int step) {
    __syncthreads();  // the previous op is done with sp_op (and sp_pg is set)
    constexpr int kPieces = static_cast<int>(sizeof(Op) / 16);
    for (int i = threadIdx.x; i < kPieces; i += kThreads)
      reinterpret_cast<uint4*>(&sp_op)[i] = __ldg(reinterpret_cast<const uint4*>(src) + i);
    __syncthreads();
    if (threadIdx.x == 0) trace_stamp(executed, 0);
    bool ok = true;
    switch (sp_op.kind) {
      case kOpConv:
        ok = run_conv<PLANES>(step, executed);
        break;
      case kOpReduce:
        ok = run_reduce(step);
        break;
      case kOpUpdate:
        ok = run_update(step);
        break;
      default:
        break;
    }
    if (threadIdx.x == 0) trace_stamp(executed, kTracePhases - 1);
    ++executed;
    return ok;
  };
  for (int i = 0; i < pg.n_pre; ++i)
    if (!run(pg.ops + i, 0)) return;
  for (int s = 0; s < pg.steps; ++s)
    for (int i = 0; i < pg.n_step; ++i)
      if (!run(pg.ops + pg.n_pre + i, s)) return;
}

}  // namespace sp
}  // namespace feb
