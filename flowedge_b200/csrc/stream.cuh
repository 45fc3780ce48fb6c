// Persistent U-Net sampling program for small token counts (batch x horizon
// <= 16), sm_100a.
//
// One cooperative launch runs a whole DDIM / DDPM sampling call: the FiLM
// condition GEMV once, then for every denoising step every convolution,
// GroupNorm + Mish + FiLM / residual, down / up-sampling reduction, the output
// 1x1 conv and the scheduler update.  Ops run in program order on all CTAs (one
// per SM, 16 warps) separated by a grid barrier.  At these sizes a forward is a
// stream of weights (0.5 GB per denoising step for the PushT-shaped model in
// bf16), so the design goal is to keep HBM busy:
//
//  * Convolutions are split-K GEMVs on the warp-level tensor cores
//    (mma.sync m16n8k16, fp16 operands, fp32 accumulators).  A conv is cut
//    into units of 16 output rows x 16 K values (512 bytes of fp16 weights,
//    stored fragment-ordered at load so each lane issues one coalesced 16-byte
//    load per unit).  The rows x K units are split evenly over all warps of
//    the grid, in row-major order, so any conv shape balances; each warp walks
//    a contiguous weight range with loads several units ahead.
//  * Activations stay fp32 in global memory.  Each CTA stages the conv input
//    in shared memory as an fp16 pair hi + lo (hi = fp16(x), lo = fp16(x - hi)),
//    so a product W * x costs two MMAs and keeps ~22 bits of x.  fp32-weight
//    models store W the same way and add the W_lo * x_hi product (3 MMAs).
//  * Partial sums of a row block are combined inside the CTA in warp order and
//    written once per (row block, CTA); a consumer adds the <= few segments in
//    segment order, so results are deterministic.
//  * While a conv runs, each CTA asks the L2 to prefetch its share of the next
//    conv's weights, so HBM keeps streaming across barriers and norm ops.
//
// Every barrier wait is bounded (global timer); a timeout sets the device error
// word and a shared abort flag, after which every CTA leaves at its next
// barrier.  Data written inside the launch is read with ld.global.cg (L2), as
// L1 is not coherent across SMs.
#pragma once

#include "simt.cuh"

namespace feb {
namespace sp {

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kComputeWarps = kWarps - 1;  // warp 0 streams the weights
constexpr int kMaxTok = 16;   // tokens of one conv output
constexpr int kMaxSlots = 64;  // row blocks one CTA may touch per conv
constexpr int kRowPad = 8;    // fp16 padding per staged row (spreads banks)
constexpr int kMaxTaps = 5;
constexpr int kChunk = 16384;  // bytes of one weight copy (cp.async.bulk)
constexpr int kMinStages = 3;
constexpr int kMaxStages = 8;
constexpr int kGnPerThread = 4;  // GroupNorm elements per thread (group * L <= 2048)
constexpr int kMaxSeg = 8;       // partial segments of a row block

enum OpKind : int { kOpConv = 0, kOpGn = 1, kOpReduce = 2, kOpUpdate = 3 };

// Conv output y[n][m] = bias[m] + sum of the partial segments of row block
// m / 16.  Segment s of row block r was written by the s-th CTA whose unit
// range meets r (units r * ks .. r * ks + ks - 1).
struct YSrc {
  const float* P;     // [rbs][seg_max][T][16]
  const int* nseg;    // [rbs] segments of each row block
  const float* bias;  // [M] or null
  int ks;             // 16-wide K steps per row block
  long long units;    // rbs * ks
  int seg_max;
  int T;              // tokens (samples * L_out)
};

struct ConvOp {
  const uint4* w;  // [rb][ks][planes][32 lanes], fragment order
  int planes;      // 1: fp16 weights, 2: fp16 hi + lo
  int rbs, ks;
  int ic_pad;      // channels of the concatenated input; K = ntaps * ic_pad
  const float* src0;
  int c0;          // fp32 [samples][L_in][c0]
  const float* src1;
  int c1;          // concatenated second source, or null
  int samples, L_in, L_out, stride;
  int ntaps;
  int tap_off[kMaxTaps];  // input time = t * stride + tap_off
  int halo_lo, rows;      // staged rows per sample (input time + halo_lo)
  float* P;
  int seg_max;
  int T;
  int nct;         // CTAs the units are split over (<= gridDim.x; tiny convs use fewer)
  int nslots;      // row blocks one CTA touches at most (slots per compute warp)
  int ring_off;    // shared-memory offset of the weight ring (after the staged input, slots and flags)
  int stages;      // ring stages of kChunk bytes
  // weights of the next conv in program order (L2 prefetch), or null
  const uint4* next_w;
  long long next_units;
  int next_planes;
};

struct GnOp {
  YSrc y;
  int C, groups, samples, L;
  const float* gamma;
  const float* beta;
  int film;                 // z = (fc + ft) * z + (fc' + ft'), fc from film_cond, ft the step's time row
  const float* film_cond;   // [samples][film_F]
  const float* film_time;   // [timesteps][film_F]
  int film_F, film_off;
  int res_mode;             // 0 none, 1 conv output (res), 2 fp32 tensor
  YSrc res;
  const float* res_tensor;  // [T][C]
  float* out;               // [T][C]
};

// out[(n / L * L * tmul) + (n % L) * tmul + tadd][m] = y[n][m] for m < M
struct ReduceOp {
  YSrc y;
  int M, L, tmul, tadd;
  float* out;
};

// eps[n][a] = y[n][a]; x = scheduler(x, eps); x_master and the next input
struct UpdateOp {
  YSrc y;
  int A, H, Cin, samples;
  float* x_master;  // [T][A]
  float* x_in;      // [T][Cin] fp32
  const uint64_t* seeds;
};

struct Op {
  int kind;
  int barrier_after;
  union {
    ConvOp conv;
    GnOp gn;
    ReduceOp reduce;
    UpdateOp update;
  };
};

struct Program {
  const Op* ops;
  int n_pre;                   // ops run once, before the steps
  int n_step;                  // ops run at every step
  int steps;
  const int* step_t;           // [steps] timestep of each step (FiLM time row)
  const StepScalars* scalars;  // [steps]
  unsigned* sync;              // [0] arrivals (monotonic), [2] abort
  int* err;
  unsigned long long* trace;   // null, or one global-timer stamp per executed op (CTA 0)
};

// ---------------------------------------------------------------------------
// helpers

// volatile: issued where written (the ring below relies on loads being in
// flight several units before their use; a pure asm could be sunk to its use)
__device__ __forceinline__ uint4 ld_weights(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p));
  return v;
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint4& a, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}

// CTA whose unit range [U c / NC, U (c + 1) / NC) holds unit u
__device__ __forceinline__ int cta_of(long long u, long long U, int NC) {
  int c = static_cast<int>((u * NC) / U);
  while (c + 1 < NC && (U * (c + 1)) / NC <= u) ++c;
  while (c > 0 && (U * c) / NC > u) --c;
  return c;
}

// All segments are requested at once (static bound kMaxSeg), then added in
// segment order.
__device__ __forceinline__ float y_at(const YSrc& y, int n, int m) {
  const int rb = m >> 4;
  const int nseg = __ldg(y.nseg + rb);
  float v = y.bias != nullptr ? __ldg(y.bias + m) : 0.0f;
  const float* p = y.P + ((static_cast<long long>(rb) * y.seg_max) * y.T + n) * 16 + (m & 15);
  const long long stride = static_cast<long long>(y.T) * 16;
  float t[kMaxSeg];
#pragma unroll
  for (int s = 0; s < kMaxSeg; ++s) t[s] = s < nseg ? __ldcg(p + s * stride) : 0.0f;
#pragma unroll
  for (int s = 0; s < kMaxSeg; ++s)
    if (s < nseg) v += t[s];
  return v;
}

// Grid barrier on a monotonic arrival counter: barrier number k (from 1) is
// passed once the counter reaches k * gridDim.x.  The arrival is a release
// and the poll an acquire at GPU scope, so every CTA's writes before the
// barrier are visible to every CTA after it (with __syncthreads on both sides
// for the CTA's other threads).  Bounded wait; returns false once the program
// is aborted.
__device__ bool grid_sync(const Program& pg, unsigned& epoch) {
  __shared__ int s_ok;
  __syncthreads();
  ++epoch;
  if (threadIdx.x == 0) {
    volatile unsigned* abort_flag = pg.sync + 2;
    int ok = *abort_flag == 0u;
    if (ok) {
      const unsigned target = epoch * gridDim.x;
      asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(pg.sync) : "memory");
      const uint64_t t0 = global_ns();
      for (uint32_t spin = 0;; ++spin) {
        unsigned v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(pg.sync) : "memory");
        if (v >= target) break;
        if ((spin & 15u) == 15u) {
          if (*abort_flag != 0u) {
            ok = 0;
            break;
          }
          if (global_ns() - t0 > kWaitNs) {
            atomicCAS(pg.err, 0, kErrGridBarrierTimeout);
            atomicExch(pg.sync + 2, 1u);
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

// ---------------------------------------------------------------------------
// convolution (split-K GEMV on mma.sync)

// Weights reach shared memory by cp.async.bulk: a CTA's units are one
// contiguous byte range, copied in kChunk pieces through a ring of `stages`
// buffers by warp 0 (lane 0); the other warps take the units of each chunk in
// turn, read their A fragments from the ring (16 bytes per lane, conflict-free)
// and release the buffer on an "empty" mbarrier.  Per-warp partial sums of each
// row block go to a (warp, row block) slot and are combined in warp order.
// `full` / `empty` are initialised once per launch; `uses[s]` counts the
// phases ring buffer s went through in earlier convs of the launch, so chunk c
// of this conv waits on parity (uses[c % stages] + c / stages) & 1.
template <int PLANES>
__device__ __noinline__ void run_conv(const ConvOp& op_in, uint8_t* smem, uint64_t* full, uint64_t* empty, int* uses,
                                      volatile unsigned* abort_flag, int* err) {
  const ConvOp op = op_in;  // one batch of independent loads instead of a chain of field reads
  const int NC = op.nct;
  const int cta = blockIdx.x;
  const long long U = static_cast<long long>(op.rbs) * op.ks;
  const long long cu0 = cta < NC ? U * cta / NC : U, cu1 = cta < NC ? U * (cta + 1) / NC : U;

  // L2 prefetch of a 1 / gridDim.x share of the next conv's weights (issued
  // after this conv's own first copies)
  auto prefetch_next = [&]() {
    if (op.next_w == nullptr) return;
    const long long nu0 = op.next_units * cta / gridDim.x, nu1 = op.next_units * (cta + 1) / gridDim.x;
    const char* base = reinterpret_cast<const char*>(op.next_w) + nu0 * op.next_planes * 512;
    const long long bytes = (nu1 - nu0) * op.next_planes * 512;
    for (long long off = 0; off < bytes; off += 65536) {
      const unsigned chunk = static_cast<unsigned>(bytes - off < 65536 ? bytes - off : 65536);
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(base + off), "r"(chunk) : "memory");
    }
  };
  if (cu0 == cu1) {  // uniform across the CTA
    if (threadIdx.x == 0) prefetch_next();
    return;
  }

  constexpr int kUnitBytes = PLANES * 512;
  constexpr int kUnitsPerChunk = kChunk / kUnitBytes;
  const int stages = op.stages;
  const long long nunits = cu1 - cu0;
  const int nchunks = static_cast<int>((nunits + kUnitsPerChunk - 1) / kUnitsPerChunk);
  const char* wsrc = reinterpret_cast<const char*>(op.w) + cu0 * kUnitBytes;
  uint8_t* ring = smem + op.ring_off;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // first copies go out before the staging
  auto issue = [&](int c) {
    const int st = c % stages;
    const long long u0 = static_cast<long long>(c) * kUnitsPerChunk;
    const long long nu = nunits - u0 < kUnitsPerChunk ? nunits - u0 : kUnitsPerChunk;
    const unsigned bytes = static_cast<unsigned>(nu * kUnitBytes);
    mbar_arrive_expect_tx(&full[st], bytes);
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(ring + st * kChunk)),
        "l"(wsrc + u0 * kUnitBytes), "r"(bytes), "r"(smem_u32(&full[st]))
        : "memory");
  };
  if (threadIdx.x == 0) {
    // earlier ops wrote this shared memory through the generic proxy
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    for (int c = 0; c < stages && c < nchunks; ++c) issue(c);
    prefetch_next();
  }

  // stage the input as fp16 hi / lo: rows [sample][time + halo_lo], one zero
  // row last; loads in batches of 8 per thread so their latencies overlap
  const int rs = op.ic_pad + kRowPad;  // halfs per staged row
  const int nrows = op.samples * op.rows;
  __half* xh = reinterpret_cast<__half*>(smem);
  __half* xl = xh + static_cast<long long>(nrows + 1) * rs;
  float* slots = reinterpret_cast<float*>(xl + static_cast<long long>(nrows + 1) * rs);
  const int nslots = op.nslots;
  int* touched = reinterpret_cast<int*>(slots + static_cast<long long>(kComputeWarps) * nslots * 16 * op.T);
  const int q4 = op.ic_pad / 4;
  const int items = (nrows + 1) * q4;
  constexpr int kBatch = 8;
  constexpr int kStagers = kComputeWarps * 32;  // warp 0 issues the copies meanwhile
  const int sid = threadIdx.x - 32;
  for (int base = 0; warp > 0 && base < items; base += kBatch * kStagers) {
    float4 v[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int i = base + j * kStagers + sid;
      v[j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      if (i < items) {
        const int r = i / q4;
        const int ch = (i - r * q4) * 4;
        if (r < nrows) {
          const int b = r / op.rows;
          const int t_in = r - b * op.rows - op.halo_lo;
          if (t_in >= 0 && t_in < op.L_in) {
            const float* src = ch < op.c0
                                   ? op.src0 + (static_cast<long long>(b) * op.L_in + t_in) * op.c0 + ch
                                   : op.src1 + (static_cast<long long>(b) * op.L_in + t_in) * op.c1 + (ch - op.c0);
            v[j] = __ldcg(reinterpret_cast<const float4*>(src));
          }
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int i = base + j * kStagers + sid;
      if (i < items) {
        const int r = i / q4;
        const int ch = (i - r * q4) * 4;
        const __half h0 = __float2half_rn(v[j].x), h1 = __float2half_rn(v[j].y), h2 = __float2half_rn(v[j].z),
                     h3 = __float2half_rn(v[j].w);
        __half2* dh = reinterpret_cast<__half2*>(xh + static_cast<long long>(r) * rs + ch);
        __half2* dl = reinterpret_cast<__half2*>(xl + static_cast<long long>(r) * rs + ch);
        dh[0] = __halves2half2(h0, h1);
        dh[1] = __halves2half2(h2, h3);
        dl[0] = __halves2half2(__float2half_rn(v[j].x - __half2float(h0)), __float2half_rn(v[j].y - __half2float(h1)));
        dl[1] = __halves2half2(__float2half_rn(v[j].z - __half2float(h2)), __float2half_rn(v[j].w - __half2float(h3)));
      }
    }
  }
  for (int i = sid; warp > 0 && i < kWarps * nslots; i += kStagers) touched[i] = 0;
  // the compute warps wait for each other's staging only: warp 0 may still be
  // issuing copies (an issue can stall while earlier copies are in flight)
  if (warp > 0) named_barrier(1, kStagers);

  const int T = op.T;
  const int slot_floats = 16 * T;
  const int rb_lo = static_cast<int>(cu0 / op.ks);
  bool ok = true;
  if (warp == 0) {
    // producer: refill each buffer once every compute warp released it
    if (lane == 0) {
      for (int c = stages; c < nchunks && ok; ++c) {
        const int st = c % stages;
        ok = mbar_wait(&empty[st], (uses[st] + (c / stages) - 1) & 1, reinterpret_cast<volatile int*>(abort_flag));
        if (ok) issue(c);
      }
      if (!ok) {
        atomicCAS(err, 0, kErrWaitTimeoutProducer);
        atomicExch(const_cast<unsigned*>(abort_flag), 1u);
      }
    }
  } else {
    // compute warp cw takes units cu0 + cw, cu0 + cw + 15, ... in order; the
    // unit's (row block, K step, tap, channel) advance incrementally
    const int cw = warp - 1;
    const int g = lane >> 2, t4 = lane & 3;
    const bool two_nb = T > 8;
    // T <= 4: one n=8 tile holds x_hi (columns 0-3) and x_lo (columns 4-7) of
    // the tokens, so W * (x_hi + x_lo) is one MMA; the halves are added at flush
    const bool packed = T <= 4;
    int tap_row[2][kMaxTaps];  // staged row of this lane's token for every tap (nrows: zero row)
#pragma unroll
    for (int nb = 0; nb < 2; ++nb) {
      const int n = packed ? (g & 3) : nb * 8 + g;
      int base = -1;
      if (n < T) {
        const int b = n / op.L_out;
        const int t = n - b * op.L_out;
        base = b * op.rows + t * op.stride + op.halo_lo;
      }
#pragma unroll
      for (int j = 0; j < kMaxTaps; ++j)
        tap_row[nb][j] = (base >= 0 && j < op.ntaps) ? base + op.tap_off[j] : nrows;
    }
    const int ks = op.ks, ic_pad = op.ic_pad;
    // independent accumulator chains: [n block][x hi / x lo]
    float acc[2][2][4];
    auto zero = [&]() {
#pragma unroll
      for (int nb = 0; nb < 2; ++nb)
#pragma unroll
        for (int hl = 0; hl < 2; ++hl)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[nb][hl][i] = 0.0f;
    };
    zero();
    int cur = -1;  // row block of the accumulators, or -1
    auto flush = [&]() {
      const int sidx = cur - rb_lo;
      if (sidx >= 0 && sidx < nslots) {
        float* sl = slots + static_cast<long long>(cw * nslots + sidx) * slot_floats;
        if (packed) {
          float v[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) v[i] = acc[0][0][i] + acc[0][1][i];
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
          if (lane == 0) touched[warp * nslots + sidx] = 1;
          return;
        }
#pragma unroll
        for (int nb = 0; nb < 2; ++nb) {
          const int n0 = nb * 8 + 2 * t4;
          if (n0 < T) {
            sl[g * T + n0] = acc[nb][0][0] + acc[nb][1][0];
            sl[(g + 8) * T + n0] = acc[nb][0][2] + acc[nb][1][2];
          }
          if (n0 + 1 < T) {
            sl[g * T + n0 + 1] = acc[nb][0][1] + acc[nb][1][1];
            sl[(g + 8) * T + n0 + 1] = acc[nb][0][3] + acc[nb][1][3];
          }
        }
        if (lane == 0) touched[warp * nslots + sidx] = 1;
      } else if (lane == 0) {
        atomicCAS(err, 0, kErrProgramLayout);  // the host bounds the row blocks of a CTA; never expected
      }
    };
    // position of this warp's next unit (offset from cu0)
    int next = cw;
    int rb = 0, k = 0, tap = 0, ch = 0;
    bool pos_valid = false;
    for (int c = 0; c < nchunks && ok; ++c) {
      const int st = c % stages;
      ok = mbar_wait(&full[st], (uses[st] + c / stages) & 1, reinterpret_cast<volatile int*>(abort_flag));
      if (!ok) {
        if (lane == 0) {
          atomicCAS(err, 0, kErrWaitTimeoutMma);
          atomicExch(const_cast<unsigned*>(abort_flag), 1u);
        }
        break;
      }
      const int c0 = c * kUnitsPerChunk;
      const int c1 = static_cast<int>(nunits - c0 < kUnitsPerChunk ? nunits : c0 + kUnitsPerChunk);
      const uint8_t* buf = ring + st * kChunk;
      for (; next < c1; next += kComputeWarps) {
        if (!pos_valid) {
          const long long q = cu0 + next;
          rb = static_cast<int>(q / ks);
          k = static_cast<int>(q - static_cast<long long>(rb) * ks);
          tap = (k * 16) / ic_pad;
          ch = k * 16 - tap * ic_pad;
          pos_valid = true;
        }
        if (rb != cur) {
          if (cur >= 0) flush();
          zero();
          cur = rb;
        }
        uint4 a[PLANES];
#pragma unroll
        for (int pl = 0; pl < PLANES; ++pl)
          a[pl] = *reinterpret_cast<const uint4*>(buf + (next - c0) * kUnitBytes + pl * 512 + lane * 16);
        if (packed) {
          int r = nrows;
#pragma unroll
          for (int j = 0; j < kMaxTaps; ++j)
            if (j == tap) r = tap_row[0][j];
          const long long off = static_cast<long long>(r) * rs + ch + 2 * t4;
          const uint32_t* px = reinterpret_cast<const uint32_t*>((g < 4 ? xh : xl) + off);
          const uint32_t b0 = px[0], b1 = px[4];
          mma16816(acc[0][0], a[0], b0, b1);
          if constexpr (PLANES == 2) mma16816(acc[0][1], a[1], g < 4 ? b0 : 0u, g < 4 ? b1 : 0u);
        } else {
#pragma unroll
        for (int nb = 0; nb < 2; ++nb) {
          if (nb == 0 || two_nb) {
            int r = nrows;
#pragma unroll
            for (int j = 0; j < kMaxTaps; ++j)
              if (j == tap) r = tap_row[nb][j];
            const long long off = static_cast<long long>(r) * rs + ch + 2 * t4;
            const uint32_t* ph = reinterpret_cast<const uint32_t*>(xh + off);
            const uint32_t* pl = reinterpret_cast<const uint32_t*>(xl + off);
            const uint32_t b0h = ph[0], b1h = ph[4];  // channels +0 / +8
            const uint32_t b0l = pl[0], b1l = pl[4];
            mma16816(acc[nb][0], a[0], b0h, b1h);
            mma16816(acc[nb][1], a[0], b0l, b1l);
            if constexpr (PLANES == 2) mma16816(acc[nb][1], a[1], b0h, b1h);
          }
        }
        }
        // advance by kComputeWarps units
        k += kComputeWarps;
        if (k >= ks) {
          pos_valid = false;  // next row block(s): recompute from the unit index
        } else {
          ch += 16 * kComputeWarps;
          while (ch >= ic_pad) {
            ch -= ic_pad;
            ++tap;
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
    if (cur >= 0) flush();
  }
  __syncthreads();
  // phases each ring buffer went through in this conv (every chunk completes
  // one phase of its `full` and of its `empty` barrier)
  if (threadIdx.x < stages) uses[threadIdx.x] += (nchunks - static_cast<int>(threadIdx.x) + stages - 1) / stages;

  // combine the warps' slots per row block (warp order) and write this CTA's segment
  const int rb_hi = static_cast<int>((cu1 - 1) / op.ks);
  const int total = (rb_hi - rb_lo + 1) * slot_floats;
  for (int i = threadIdx.x; i < total; i += kThreads) {
    const int rbi = i / slot_floats;
    const int e = i - rbi * slot_floats;
    const int rb = rb_lo + rbi;
    float v = 0.0f;
    if (rbi < nslots)
      for (int w = 1; w < kWarps; ++w)
        if (touched[w * nslots + rbi]) v += slots[static_cast<long long>((w - 1) * nslots + rbi) * slot_floats + e];
    const int seg = cta - cta_of(static_cast<long long>(rb) * op.ks, U, NC);
    const int m = e / T, n = e - m * T;
    op.P[((static_cast<long long>(rb) * op.seg_max + seg) * T + n) * 16 + m] = v;
  }
}

// ---------------------------------------------------------------------------
// GroupNorm + Mish (+ FiLM or residual): one CTA per (sample, group)

// The head of a conv output point (token n, channel m): its segment count,
// its bias (the start of the sum) and the address of its first segment.
__device__ __forceinline__ void y_head(const YSrc& y, int n, int m, int& nseg, float& v, const float*& p) {
  const int rb = m >> 4;
  nseg = __ldg(y.nseg + rb);
  v = y.bias != nullptr ? __ldg(y.bias + m) : 0.0f;
  p = y.P + ((static_cast<long long>(rb) * y.seg_max) * y.T + n) * 16 + (m & 15);
}

// Each CTA takes whole (sample, group) items; E elements of the group per
// thread (E * kThreads >= channels per group * L).  With two elements per
// thread the loads go out in two dependent rounds: first everything that
// depends on nothing else (segment counts and biases of the conv output and of
// a conv residual, the affine and FiLM terms, an fp32 residual), then every
// segment of both conv outputs.  With four, the values in flight would not fit
// the registers, so the residual and the affine / FiLM terms follow in later
// rounds.  Sums keep y_at's order: bias, then the segments in order.
template <int E>
__device__ __forceinline__ void run_gn_items(const GnOp& op, int step, const int* step_t) {
  constexpr bool kEarly = E <= 2;  // residual, affine and FiLM loads in the first round
  __shared__ double red[2][kWarps];
  __shared__ float stat[2];
  const int NC = gridDim.x;
  const int cpg = op.C / op.groups;
  const int cnt = cpg * op.L;
  const int items = op.samples * op.groups;
  const bool res_conv = op.res_mode == 1;
  const float* ft = op.film ? op.film_time + static_cast<long long>(step_t[step]) * op.film_F + op.film_off : nullptr;
  const long long sy = static_cast<long long>(op.y.T) * 16;
  const long long sr = static_cast<long long>(op.res.T) * 16;
  for (int item = blockIdx.x; item < items; item += NC) {
    const int b = item / op.groups;
    const int gi = item - b * op.groups;
    const float* fc = op.film ? op.film_cond + static_cast<long long>(b) * op.film_F + op.film_off : nullptr;
    int n[E], c[E];
    bool ok[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const int i = threadIdx.x + e * kThreads;
      ok[e] = i < cnt;
      const int t = ok[e] ? i / cpg : 0;
      c[e] = ok[e] ? gi * cpg + (i - t * cpg) : 0;
      n[e] = b * op.L + t;
    }
    // the residual (conv output or fp32 tensor): heads or values
    auto res_heads = [&](int (&nr)[E], float (&r)[E], const float* (&pr)[E]) {
#pragma unroll
      for (int e = 0; e < E; ++e) {
        nr[e] = 0;
        r[e] = 0.0f;
        pr[e] = op.res.P;
        if (ok[e]) {
          if (res_conv) y_head(op.res, n[e], c[e], nr[e], r[e], pr[e]);
          else if (op.res_mode == 2) r[e] = __ldcg(op.res_tensor + static_cast<long long>(n[e]) * op.C + c[e]);
        }
      }
    };
    // gamma, beta and the FiLM scale / shift (condition row + time row)
    auto affine = [&](int e, float& ga, float& be, float& fs, float& fh) {
      ga = __ldg(op.gamma + c[e]);
      be = __ldg(op.beta + c[e]);
      fs = fh = 0.0f;
      if (op.film) {
        fs = __ldcg(fc + c[e]) + __ldg(ft + c[e]);
        fh = __ldcg(fc + op.C + c[e]) + __ldg(ft + op.C + c[e]);
      }
    };
    int ny[E], nr[E];
    const float* py[E];
    const float* pr[E];
    float v[E], r[E], ga[E], be[E], fs[E], fh[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
      ny[e] = 0;
      v[e] = 0.0f;
      py[e] = op.y.P;
      if (ok[e]) y_head(op.y, n[e], c[e], ny[e], v[e], py[e]);
    }
    if constexpr (kEarly) {
      res_heads(nr, r, pr);
#pragma unroll
      for (int e = 0; e < E; ++e)
        if (ok[e]) affine(e, ga[e], be[e], fs[e], fh[e]);
      float ty[E][kMaxSeg], tr[E][kMaxSeg];
#pragma unroll
      for (int e = 0; e < E; ++e)
#pragma unroll
        for (int s = 0; s < kMaxSeg; ++s) {
          ty[e][s] = s < ny[e] ? __ldcg(py[e] + s * sy) : 0.0f;
          tr[e][s] = s < nr[e] ? __ldcg(pr[e] + s * sr) : 0.0f;
        }
#pragma unroll
      for (int e = 0; e < E; ++e)
#pragma unroll
        for (int s = 0; s < kMaxSeg; ++s) {
          if (s < ny[e]) v[e] += ty[e][s];
          if (s < nr[e]) r[e] += tr[e][s];
        }
    } else {
      float t[E][kMaxSeg];
#pragma unroll
      for (int e = 0; e < E; ++e)
#pragma unroll
        for (int s = 0; s < kMaxSeg; ++s) t[e][s] = s < ny[e] ? __ldcg(py[e] + s * sy) : 0.0f;
#pragma unroll
      for (int e = 0; e < E; ++e)
#pragma unroll
        for (int s = 0; s < kMaxSeg; ++s)
          if (s < ny[e]) v[e] += t[e][s];
      res_heads(nr, r, pr);
#pragma unroll
      for (int e = 0; e < E; ++e)
#pragma unroll
        for (int s = 0; s < kMaxSeg; ++s) t[e][s] = s < nr[e] ? __ldcg(pr[e] + s * sr) : 0.0f;
#pragma unroll
      for (int e = 0; e < E; ++e)
#pragma unroll
        for (int s = 0; s < kMaxSeg; ++s)
          if (s < nr[e]) r[e] += t[e][s];
    }
    double s1 = 0.0, s2 = 0.0;
#pragma unroll
    for (int e = 0; e < E; ++e)
      if (ok[e]) {
        s1 += v[e];
        s2 += static_cast<double>(v[e]) * v[e];
      }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      s1 += __shfl_xor_sync(0xffffffffu, s1, off);
      s2 += __shfl_xor_sync(0xffffffffu, s2, off);
    }
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) {
      red[0][warp] = s1;
      red[1][warp] = s2;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      double t1 = 0.0, t2 = 0.0;
      for (int w = 0; w < kWarps; ++w) {
        t1 += red[0][w];
        t2 += red[1][w];
      }
      // biased variance E[x^2] - E[x]^2 clamped at 0, eps 1e-5, in double
      const double mean = t1 / cnt;
      const double var = fmax(0.0, t2 / cnt - mean * mean);
      stat[0] = static_cast<float>(mean);
      stat[1] = static_cast<float>(1.0 / sqrt(var + 1e-5));
    }
    __syncthreads();
    const float mean = stat[0], inv = stat[1];
#pragma unroll
    for (int e = 0; e < E; ++e) {
      if (ok[e]) {
        if constexpr (!kEarly) affine(e, ga[e], be[e], fs[e], fh[e]);
        float z = (v[e] - mean) * (inv * ga[e]) + be[e];
        z = mish_f(z);
        if (op.film) z = fs[e] * z + fh[e];
        op.out[static_cast<long long>(n[e]) * op.C + c[e]] = z + r[e];
      }
    }
    __syncthreads();
  }
}

// GroupNorm + Mish (+ FiLM or residual): two elements per thread when a group
// holds at most 2 * kThreads of them (every PushT-shaped layer), else four.
__device__ __noinline__ void run_gn(const GnOp& op, int step, const int* step_t) {
  static_assert(kGnPerThread == 4, "run_gn instantiates 2 and 4 elements per thread");
  if ((op.C / op.groups) * op.L <= 2 * kThreads) run_gn_items<2>(op, step, step_t);
  else run_gn_items<4>(op, step, step_t);
}

__device__ void run_reduce(const ReduceOp& op) {
  const int NC = gridDim.x;
  const long long total = static_cast<long long>(op.y.T) * op.M;
  for (long long i = blockIdx.x * static_cast<long long>(kThreads) + threadIdx.x; i < total;
       i += static_cast<long long>(NC) * kThreads) {
    const int n = static_cast<int>(i / op.M);
    const int m = static_cast<int>(i - static_cast<long long>(n) * op.M);
    const int b = n / op.L, t = n - b * op.L;
    const long long row = static_cast<long long>(b) * op.L * op.tmul + static_cast<long long>(t) * op.tmul + op.tadd;
    op.out[row * op.M + m] = y_at(op.y, n, m);
  }
}

__device__ void run_update(const UpdateOp& op, const StepScalars& s) {
  const int NC = gridDim.x;
  const int total = op.samples * op.H * op.A;
  for (int i = blockIdx.x * kThreads + threadIdx.x; i < total; i += NC * kThreads) {
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
}

template <int PLANES>
__device__ __forceinline__ bool run_op(const Program& pg, const Op& op, int step, uint8_t* smem, uint64_t* bars,
                                       int* uses, unsigned& epoch) {
  switch (op.kind) {
    case kOpConv:
      run_conv<PLANES>(op.conv, smem, bars, bars + kMaxStages, uses, pg.sync + 2, pg.err);
      break;
    case kOpGn:
      run_gn(op.gn, step, pg.step_t);
      break;
    case kOpReduce:
      run_reduce(op.reduce);
      break;
    case kOpUpdate:
      run_update(op.update, pg.scalars[step]);
      break;
    default:
      break;
  }
  return op.barrier_after ? grid_sync(pg, epoch) : true;
}

template <int PLANES>
static __global__ void __launch_bounds__(kThreads, 1) unet_program_kernel(const Program pg) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ int uses[kMaxStages];  // phases each ring buffer went through
  __shared__ __align__(8) uint64_t bars[2 * kMaxStages];
  if (threadIdx.x == 0) {
    for (int st = 0; st < kMaxStages; ++st) {
      mbar_init(&bars[st], 1);                          // full: the copy landed
      mbar_init(&bars[kMaxStages + st], kComputeWarps);  // empty: every compute warp is done with it
      uses[st] = 0;
    }
    fence_mbar_init();
  }
  __syncthreads();
  int executed = 0;
  unsigned epoch = 0;
  auto stamp = [&]() {
    if (pg.trace != nullptr && blockIdx.x == 0 && threadIdx.x == 0) pg.trace[executed] = global_ns();
    ++executed;
  };
  stamp();
  for (int i = 0; i < pg.n_pre; ++i) {
    if (!run_op<PLANES>(pg, pg.ops[i], 0, smem, bars, uses, epoch)) return;
    stamp();
  }
  for (int s = 0; s < pg.steps; ++s)
    for (int i = 0; i < pg.n_step; ++i) {
      if (!run_op<PLANES>(pg, pg.ops[pg.n_pre + i], s, smem, bars, uses, epoch)) return;
      stamp();
    }
}

}  // namespace sp
}  // namespace feb
