// Persistent tcgen05 implicit-GEMM for sm_100a.
//
//   out[token][m] = epilogue( sum_seg sum_c A[m][seg.a_k + c] * B_seg[token](c) )
//
// A is a K-major 16-bit weight matrix [M_total][K_total] (bf16 or fp16, the
// same format as B).  B is gathered per "segment": a TMA box of 64 channels
// from a 16-bit activation tensor laid out
// [samples][length][channels], read at a time offset `t_off` and channel
// offset `ch_off`.  A 1-D convolution with k taps is k segments (one per tap,
// t_off = tap - pad); a channel concatenation is one segment per source; a
// stride-2 convolution reads a [samples][length/2][2*channels] view of its
// input.  TMA zero-fills rows whose time index falls outside [0, length) and
// samples beyond the batch, which is exactly the convolution's zero padding.
//
// Tile: 128 (M) x 256 (N tokens) x 64 (K) per stage, 4 stages, fp32
// accumulators double-buffered in TMEM (2 x 256 columns).  Warp roles:
//   warp 0: TMA producer (one lane)
//   warp 1: TMEM allocator + MMA issuer (one lane)
//   warps 2..: epilogue (TMEM -> registers -> global), one accumulator row
//              (= one output channel) per thread; EPI_PARTS warps per TMEM
//              lane quadrant, each taking EPI_COLS of the tile's 256 columns.
// Every mbarrier wait is bounded; a timeout sets an error code, raises a
// shared abort flag, drains in-flight copies/MMAs with bounded waits, frees
// TMEM and returns.
#pragma once

#include "common.cuh"

namespace feb {
namespace tc {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN * BK * 2;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int MAX_SEGS = 12;
constexpr int MAX_TILE_SAMPLES = 64;  // samples per N tile when GN statistics are gathered
constexpr int EPI_WARPS = 16;
constexpr int EPI_THREADS = EPI_WARPS * 32;
constexpr int EPI_PARTS = EPI_WARPS / 4;    // epilogue warps per TMEM lane quadrant
constexpr int EPI_COLS = BN / EPI_PARTS;    // tile columns per epilogue warp
constexpr int THREADS = 64 + EPI_THREADS;
constexpr int TMEM_COLS = 512;
constexpr int MAX_TILE_GROUPS = 4;   // groups of >= 32 channels inside a 128-row tile
constexpr int BP_SAMPLES = 32;       // samples of a tile in the per-slice statistics (L >= 8)
static_assert(2 * 16 * BP_SAMPLES <= 4 * 4 * MAX_TILE_SAMPLES, "per-slice partials fit the partials buffer");
constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + 256 + 4 * EPI_PARTS * MAX_TILE_SAMPLES * 16 +
                           MAX_TILE_SAMPLES * MAX_TILE_GROUPS * 8 + 3 * MAX_TILE_SAMPLES * 16;
static_assert(SMEM_BYTES <= 232448, "shared memory above the 227 KB per-CTA limit");

// kActSwiGLU: accumulator rows interleave gate (even row 2f) and up (odd row
// 2f + 1) of feature f; the output holds bf16(bf16(up) * SiLU(bf16(gate))) at
// channel f (bf16 output, plain epilogue; SiLU by the fast exponential and
// division, whose ~1e-6 relative error is far below the bf16 step).
enum Act : int { kActNone = 0, kActSilu = 1, kActSoftplus = 2, kActSwiGLU = 3 };

struct Seg {
  int src;      // which B tensor map (0..2)
  int t_off;    // time offset of the tap
  int ch_off;   // first channel within the source
  int kblocks;  // number of 64-channel blocks
  int a_k;      // K offset of this segment in A
};

struct Params {
  int n_tiles_m, n_tiles_n, total_tiles;
  int L;            // tokens per sample inside an N tile (TMA box length, power of 2)
  int L_shift;      // log2(L)
  int tile_samples; // BN / L
  int n_samples;    // valid samples (tokens of samples >= this are skipped)
  int m_valid;      // rows >= m_valid are not stored
  int nseg;
  Seg seg[MAX_SEGS];
  // epilogue
  const float* bias;      // [m] or null
  const float* add_vec;   // [m] or null
  const float* add_tok;   // fp32 or null: element add_base + token * add_cs + m
  long long add_base;
  int add_cs;
  int act;
  int fp16;               // operand format (and 16-bit output format): 1 fp16, 0 bf16
  int out_f32;            // 1: fp32 output, 0: 16-bit
  int out_accumulate;     // fp32 output only: out += value
  void* out;              // element out_base + token * out_cs + m, token = sample * L + t
  long long out_base;
  int out_cs;
  int n_tokens;           // n_samples * L
  int out_bf16;           // 16-bit output as bf16 even with fp16 operands
  int out_lo_off;         // fp16 16-bit output only, nonzero: also store the rounding
                          // remainder y - half(y) at element offset out_lo_off
  // GroupNorm partial statistics (sum, sum of squares) per (sample, group, part)
  double* stats;          // null: no statistics
  int group_ch;           // channels per group (multiple of 32)
  int groups;             // groups of the layer
  int parts;              // max(1, group_ch / 128)
  // GroupNorm applied in the epilogue (groups of <= 128 channels lie inside
  // one tile): z = mish(GN(y)) then FiLM, or + residual; z goes to `out`
  // (16-bit) and optionally to the fp32 copy `out_twin`.
  int gn_fuse;
  const float* gamma;
  const float* beta;
  const float* film_cond;  // [sample][film_F]: scale at film_off + m, shift at film_off + film_C + m
  const float* film_time;  // [film_F] time part, added to both
  int film_F, film_off, film_C;
  const float* res_f32;    // residual rows laid out like the output, or null
  const void* res16;       // 16-bit residual (used when res_f32 is null), or null
  float* out_twin;         // fp32 copy of z, or null
  // causal depthwise conv of 4 taps over each sequence's tokens, then SiLU,
  // for the rows < conv_rows (kEpiConv; the Mamba in-projection's x half):
  // u = SiLU(conv_b[m] + sum_j conv_w[m][j] y[t - 3 + j]), taps before the
  // sequence's first token zero, stored fp32 to conv_u (when not null) and
  // fp16 to conv_u16 at element token * conv_ld + m; rows >= conv_rows take
  // the plain store.
  // Sequences of conv_seq tokens (a power of two dividing BN) tile the tokens.
  const float* conv_w;     // [conv_rows][4]
  const float* conv_b;
  float* conv_u;
  __half* conv_u16;
  int conv_rows, conv_seq, conv_ld;
  int* err;
};

// Epilogue modes (one kernel instantiation each, so each carries only its
// own code):
//   kEpiPlain: bias (+ add terms, activation), fp32 or 16-bit store
//   kEpiStats: as plain, plus GroupNorm partial sums to p.stats
//   kEpiFused: GroupNorm + Mish (+ FiLM / residual) applied in the epilogue
//   kEpiConv:  plain fp32, with the causal conv + SiLU of Params::conv_* on
//              the rows below conv_rows
enum EpiMode : int { kEpiPlain = 0, kEpiStats = 1, kEpiFused = 2, kEpiConv = 3 };

// kEpiConv rows: the causal conv and SiLU over this warp's EPI_COLS tokens,
// straight from the accumulator (tbase: the warp's first column), in the
// reference's order (kernels_scalar.cc:10-27): the bias, then the taps oldest
// to newest, each one fused multiply-add; the SiLU with one MUFU operation
// per element (silu2_fma, ~1e-6 relative, far below the fp16 rounding of the
// u that the x-projection and the scan read).  A sequence that began in an
// earlier column slice of the tile takes its last three inputs from the
// TMEM columns before this slice (the accumulator is released only after
// every epilogue warp is done with it).
static __device__ __noinline__ void epi_conv(const Params& p, uint32_t tbase, int m, bool m_ok, int tok0, int lim) {
  constexpr int CH = 16;
  const int mm = m_ok ? m : 0;
  const float4 w = *reinterpret_cast<const float4*>(p.conv_w + static_cast<long long>(mm) * 4);
  const float cb = p.conv_b[mm];
  const int smask = p.conv_seq - 1;
  float x1 = 0.0f, x2 = 0.0f, x3 = 0.0f;  // inputs of steps t - 1, t - 2, t - 3
  const int r = tok0 & smask;              // the same for the whole warp
  if (r != 0) {
    float pv[CH];
    tmem_ld16(tbase - CH, pv);
    x1 = pv[CH - 1];
    x2 = r >= 2 ? pv[CH - 2] : 0.0f;
    x3 = r >= 3 ? pv[CH - 3] : 0.0f;
  }
  const long long ld = p.conv_ld;
  float* ou = p.conv_u != nullptr ? p.conv_u + static_cast<long long>(tok0) * ld + m : nullptr;
  __half* oh = p.conv_u16 + static_cast<long long>(tok0) * ld + m;
#pragma unroll 1
  for (int c = 0; c < EPI_COLS; c += CH) {
    float v[CH];
    tmem_ld16(tbase + c, v);
    // tok0 + c is a multiple of CH: sequences of >= CH tokens begin only at
    // a chunk's first column, shorter ones anywhere in it
    if (smask >= CH - 1) {
      if (((tok0 + c) & smask) == 0) x1 = x2 = x3 = 0.0f;
#pragma unroll
      for (int j = 0; j < CH; ++j) {
        float a = fmaf(w.x, x3, cb);
        a = fmaf(w.y, x2, a);
        a = fmaf(w.z, x1, a);
        a = fmaf(w.w, v[j], a);
        x3 = x2;
        x2 = x1;
        x1 = v[j];
        v[j] = a;
      }
    } else {
#pragma unroll
      for (int j = 0; j < CH; ++j) {
        if (((tok0 + c + j) & smask) == 0) x1 = x2 = x3 = 0.0f;
        float a = fmaf(w.x, x3, cb);
        a = fmaf(w.y, x2, a);
        a = fmaf(w.z, x1, a);
        a = fmaf(w.w, v[j], a);
        x3 = x2;
        x2 = x1;
        x1 = v[j];
        v[j] = a;
      }
    }
#pragma unroll
    for (int j = 0; j < CH; j += 2) {
      const float2 sj = silu2_fma(make_float2(v[j], v[j + 1]));
      v[j] = sj.x;
      v[j + 1] = sj.y;
    }
    const long long oc = static_cast<long long>(c) * ld;
#pragma unroll
    for (int j = 0; j < CH; ++j)
      if (c + j < lim) {
        if (ou != nullptr) ou[oc + j * ld] = v[j];
        oh[oc + j * ld] = to_half_sat(v[j]);
      }
  }
}

// PAIR (fused mode, GroupNorm groups of 256 channels): the kernel runs as
// clusters of 2 CTAs.  Both CTAs of a cluster walk the same sequence of tile
// pairs; CTA rank r takes the 128-row tile 2*i + r of a 256-row group, so a
// group's two halves are computed side by side.  After pass 1 each CTA stores
// its per-sample partial sums into the other's shared memory and arrives on
// the other's mbarrier (release, cluster scope); each then waits (bounded) for
// the other's partials and normalises with the whole group's statistics.
//
// TOKM (fused mode only, no PAIR): tokens on the accumulator rows.  The
// activation tile (128 tokens x 64 channels, box {64, L, 128 / L}) is the MMA's
// A operand and the weight tile (256 output channels x 64) its B operand, in
// the same stage buffers (16 KB + 32 KB) and with the same UMMA shape and TMEM
// footprint; tile t covers channel tile t % n_tiles_n of token tile
// t / n_tiles_n, so the CTAs running at once share token tiles in L2.  An
// epilogue thread then owns one token and 64 consecutive output channels:
// GroupNorm groups of up to 256 channels lie inside one tile, and the
// per-channel work runs on packed fp32 pairs with 16-byte loads and stores.
template <int MODE, bool PAIR = false, bool TOKM = false>
static __global__ void __launch_bounds__(THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB0,
                   const __grid_constant__ CUtensorMap tmB1, const __grid_constant__ CUtensorMap tmB2,
                   const __grid_constant__ Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* xfull = drain + 1;  // [2]: the other CTA's GroupNorm partials arrived (PAIR)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xfull + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  double2* red = reinterpret_cast<double2*>(smem + STAGES * STAGE_BYTES + 256);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], EPI_THREADS);
    }
    mbar_init(drain, 1);
    mbar_init(&xfull[0], 1);
    mbar_init(&xfull[1], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB0);
    prefetch_tmap(&tmB1);
    prefetch_tmap(&tmB2);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // the other CTA's barriers are initialised before anyone arrives on them
  if constexpr (PAIR) cluster_sync_all();
  // Programmatic dependent launch: the set-up above (barriers, tensor-map
  // prefetch, TMEM allocation; no global memory) may overlap the previous
  // kernel's tail.  Nothing below touches global memory before the previous
  // grid has completed.  Only one CTA of this kernel fits an SM (shared
  // memory), and no other kernel allocates TMEM, so the early allocation
  // never waits on another grid.
  griddep_wait();
  griddep_launch();

  // Tile walk.  Plain: tiles blockIdx.x, +gridDim.x, ...  PAIR: tile pairs
  // (cluster index, +clusters, ...), of which this CTA takes row block
  // 2 * (pair % (n_tiles_m / 2)) + rank.
  const int rank = PAIR ? static_cast<int>(cluster_rank()) : 0;
  const int walk_first = PAIR ? static_cast<int>(cluster_index()) : static_cast<int>(blockIdx.x);
  const int walk_stride = PAIR ? static_cast<int>(cluster_count()) : static_cast<int>(gridDim.x);
  const int walk_count = PAIR ? p.total_tiles / 2 : p.total_tiles;
  static_assert(!TOKM || (MODE == kEpiFused && !PAIR), "tokens on the rows: fused GroupNorm epilogue, unpaired");
  auto tile_mn = [&](int t, int& m_blk, int& n_blk) {
    if constexpr (TOKM) {
      n_blk = t % p.n_tiles_n;
      m_blk = t / p.n_tiles_n;
    } else if constexpr (PAIR) {
      const int npm = p.n_tiles_m >> 1;
      m_blk = (t % npm) * 2 + rank;
      n_blk = t / npm;
    } else {
      m_blk = t % p.n_tiles_m;
      n_blk = t / p.n_tiles_m;
    }
  };

  const int total_kb = [&] {
    int n = 0;
    for (int s = 0; s < p.nseg; ++s) n += p.seg[s].kblocks;
    return n;
  }();

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      // the weights (A) are read by every N tile: keep them in L2 past the
      // streaming activations and residuals
      const uint64_t keep_a = l2_policy_evict_last();
      uint32_t kb_iter = 0;
      uint32_t armed = 0, armed_phase = 0;  // per-stage bits: armed at least once / parity of its last arm
      bool ok = true;
      for (int tile = walk_first; tile < walk_count && ok; tile += walk_stride) {
        int m_blk, n_blk;
        tile_mn(tile, m_blk, n_blk);
        for (int s = 0; s < p.nseg && ok; ++s) {
          const Seg sg = p.seg[s];
          const CUtensorMap* mapB = sg.src == 0 ? &tmB0 : (sg.src == 1 ? &tmB1 : &tmB2);
          for (int kb = 0; kb < sg.kblocks; ++kb, ++kb_iter) {
            const int stage = kb_iter % STAGES;
            const uint32_t phase = (kb_iter / STAGES) & 1;
            if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) {
              ok = false;
              break;
            }
            uint8_t* a_dst = smem + stage * STAGE_BYTES;
            uint8_t* b_dst = a_dst + A_BYTES;
            mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
            armed |= 1u << stage;
            armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
            if constexpr (TOKM) {
              tma_load_3d(a_dst, mapB, sg.ch_off + kb * BK, sg.t_off, m_blk * p.tile_samples, &full[stage]);
              tma_load_2d_hint(b_dst, &tmA, sg.a_k + kb * BK, n_blk * BN, &full[stage], keep_a);
            } else {
              tma_load_2d_hint(a_dst, &tmA, sg.a_k + kb * BK, m_blk * BM, &full[stage], keep_a);
              tma_load_3d(b_dst, mapB, sg.ch_off + kb * BK, sg.t_off, n_blk * p.tile_samples, &full[stage]);
            }
          }
        }
      }
      if (!ok) {
        atomicCAS(p.err, 0, kErrWaitTimeoutProducer);
        *abort_flag = 1;
        for (int s = 0; s < STAGES; ++s)
          if (armed & (1u << s)) {
            const uint32_t ph = (armed_phase >> s) & 1u;
            for (uint32_t spin = 0; spin < kSpinLimit && !mbar_try_wait(&full[s], ph); ++spin) {
            }
          }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = p.fp16 ? idesc_f16_f32(BM, BN) : idesc_bf16_f32(BM, BN);
      uint32_t kb_iter = 0;
      uint32_t acc_iter = 0;
      bool ok = true;
      for (int tile = walk_first; tile < walk_count && ok; tile += walk_stride, ++acc_iter) {
        const int acc = acc_iter & 1;
        const uint32_t acc_phase = (acc_iter >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < total_kb; ++kb, ++kb_iter) {
          const int stage = kb_iter % STAGES;
          const uint32_t phase = (kb_iter / STAGES) & 1;
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            umma_bf16(d_tmem, sw128_desc(a_addr + k * 32), sw128_desc(b_addr + k * 32), idesc,
                      (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
      }
      if (!ok) {
        atomicCAS(p.err, 0, kErrWaitTimeoutMma);
        *abort_flag = 1;
      }
      // Make sure every issued MMA finished before TMEM is released.
      umma_commit(drain);
      for (uint32_t spin = 0; spin < kSpinLimit && !mbar_try_wait(drain, 0); ++spin) {
      }
    }
  } else if constexpr (TOKM) {
    // ---------------- epilogue, tokens on the accumulator rows ----------------
    // Thread (quadrant q, lane) owns token row q*32 + lane of the tile and the
    // 64 channel columns [64 part, 64 part + 64).  Pass 1 sums y = acc + bias
    // over the thread's channels of each GroupNorm group (fp32), then over the
    // sample's lanes (double, shuffles); one double2 per (warp, sample of the
    // warp, group piece) goes to shared memory, buffered by accumulator parity,
    // and after one epilogue barrier every thread adds up the entries of its
    // (sample, group) in a fixed order.  Pass 2: z = Mish(GN(y)), then FiLM or
    // + residual, stored as fp16 (and fp32 when out_twin is set).
    const int q = warp & 3;
    const int part = (warp - 2) >> 2;
    const int row = q * 32 + lane;
    const int col0 = part * EPI_COLS;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    const int lps = p.L < 32 ? p.L : 32;                 // lanes of one sample in a warp (L >= 8)
    const int qps = p.L > 32 ? p.L >> 5 : 1;             // quadrants of one sample
    const int pieces = p.group_ch < EPI_COLS ? EPI_COLS / p.group_ch : 1;  // groups in the slice (1 or 2)
    const int ppg = p.group_ch > EPI_COLS ? p.group_ch / EPI_COLS : 1;    // slices of one group
    const double inv_cnt = 1.0 / (static_cast<double>(p.group_ch) * p.L);
    const bool film = p.film_cond != nullptr;
    // [acc][warp slot q * EPI_PARTS + part][sample of the warp][piece]
    auto red_at = [&](int a, int qq, int pp, int siw, int pc) -> double2& {
      return red[((a * EPI_WARPS + qq * EPI_PARTS + pp) * 4 + siw) * 2 + pc];
    };
    uint32_t acc_iter = 0;
    for (int tile = walk_first; tile < walk_count; tile += walk_stride, ++acc_iter) {
      int m_blk, n_blk;
      tile_mn(tile, m_blk, n_blk);
      const int acc = acc_iter & 1;
      const uint32_t acc_phase = (acc_iter >> 1) & 1;
      const bool waited = bar_and(2, EPI_THREADS, mbar_wait(&tfull[acc], acc_phase, abort_flag));
      if (!waited) {
        atomicCAS(p.err, 0, kErrWaitTimeoutEpilogue);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int tok = m_blk * BM + row;
      const int smp = tok >> p.L_shift;
      const bool tok_ok = smp < p.n_samples;
      const int smp_c = tok_ok ? smp : p.n_samples - 1;  // in-range sample for the FiLM loads
      const int ch0 = n_blk * BN + col0;                 // output channel of this slice's column 0
      const int nval = min(max(p.m_valid - ch0, 0), EPI_COLS);
      const uint32_t tbase = tmem_base + lane_base + acc * BN + col0;

      // pass 1: per-piece sums of y over this thread's channels (piece 1 is
      // channels 32-63 when a group has 32 channels)
      float2 s1[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
      float2 s2[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
#pragma unroll 1
      for (int c = 0; c < EPI_COLS / 16; ++c) {
        float v[16];
        tmem_ld16(tbase + c * 16, v);
        float2 c1 = make_float2(0.0f, 0.0f), c2 = make_float2(0.0f, 0.0f);
        if (c * 16 + 16 <= nval) {
          const float4* b4 = reinterpret_cast<const float4*>(p.bias + ch0 + c * 16);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float4 b = b4[k];
            const float2 y0 = __fadd2_rn(make_float2(v[4 * k], v[4 * k + 1]), make_float2(b.x, b.y));
            const float2 y1 = __fadd2_rn(make_float2(v[4 * k + 2], v[4 * k + 3]), make_float2(b.z, b.w));
            c1 = __fadd2_rn(c1, __fadd2_rn(y0, y1));
            c2 = __ffma2_rn(y0, y0, c2);
            c2 = __ffma2_rn(y1, y1, c2);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 16; j += 2) {
            const float y0 = c * 16 + j < nval ? v[j] + p.bias[ch0 + c * 16 + j] : 0.0f;
            const float y1 = c * 16 + j + 1 < nval ? v[j + 1] + p.bias[ch0 + c * 16 + j + 1] : 0.0f;
            c1 = __fadd2_rn(c1, make_float2(y0, y1));
            c2 = __ffma2_rn(make_float2(y0, y1), make_float2(y0, y1), c2);
          }
        }
        if (c >= 2 && pieces == 2) {
          s1[1] = __fadd2_rn(s1[1], c1);
          s2[1] = __fadd2_rn(s2[1], c2);
        } else {
          s1[0] = __fadd2_rn(s1[0], c1);
          s2[0] = __fadd2_rn(s2[0], c2);
        }
      }
      const int siw = p.L < 32 ? lane / lps : 0;  // sample of this lane within the warp
#pragma unroll
      for (int pc = 0; pc < 2; ++pc) {
        if (pc < pieces) {
          double d1 = static_cast<double>(s1[pc].x) + static_cast<double>(s1[pc].y);
          double d2 = static_cast<double>(s2[pc].x) + static_cast<double>(s2[pc].y);
          for (int off = 1; off < lps; off <<= 1) {
            d1 += __shfl_xor_sync(0xffffffffu, d1, off);
            d2 += __shfl_xor_sync(0xffffffffu, d2, off);
          }
          if ((lane & (lps - 1)) == 0) red_at(acc, q, part, siw, pc) = make_double2(d1, d2);
        }
      }
      named_barrier(1, EPI_THREADS);
      // statistics of this thread's (sample, group) per piece: the sample's
      // quadrants, then the group's slices, in that order
      float2 st[2];
#pragma unroll
      for (int pc = 0; pc < 2; ++pc) {
        st[pc] = make_float2(0.0f, 1.0f);
        if (pc < pieces) {
          const int qs0 = p.L > 32 ? ((row >> p.L_shift) << p.L_shift) >> 5 : q;
          const int pg0 = ppg > 1 ? (part / ppg) * ppg : part;
          const int ppc = pieces == 2 ? pc : 0;
          double d1 = 0.0, d2 = 0.0;
          for (int qq = qs0; qq < qs0 + qps; ++qq)
            for (int pp = pg0; pp < pg0 + ppg; ++pp) {
              const double2 r = red_at(acc, qq, pp, siw, ppc);
              d1 += r.x;
              d2 += r.y;
            }
          const double mean = d1 * inv_cnt;
          const double var = fmax(0.0, d2 * inv_cnt - mean * mean);
          st[pc] = make_float2(static_cast<float>(mean), rsqrtf(static_cast<float>(var + 1e-5)));
        }
      }

      // pass 2, eight channels at a time
      const long long o_tok = static_cast<long long>(tok) * p.out_cs + p.out_base + ch0;
      const float* fcs = film ? p.film_cond + (static_cast<long long>(smp_c) * p.film_F + p.film_off + ch0) : nullptr;
      const float* fts = film ? p.film_time + (p.film_off + ch0) : nullptr;
      const float* rf = p.res_f32 != nullptr ? p.res_f32 + o_tok : nullptr;
      __half* o16 = static_cast<__half*>(p.out) + o_tok;
      float* tw = p.out_twin != nullptr ? p.out_twin + o_tok : nullptr;
#pragma unroll 1
      for (int cb = 0; cb < EPI_COLS; cb += 8) {
        float v[8];
        tmem_ld8(tbase + cb, v);
        const float2 sg = (pieces == 2 && cb >= 32) ? st[1] : st[0];
        if (tok_ok && cb + 8 <= nval) {
          const float2 inv2 = make_float2(sg.y, sg.y), nmean2 = make_float2(-sg.x, -sg.x);
          uint32_t h[4];
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const float4 b = reinterpret_cast<const float4*>(p.bias + ch0 + cb)[k];
            const float4 g = reinterpret_cast<const float4*>(p.gamma + ch0 + cb)[k];
            const float4 be = reinterpret_cast<const float4*>(p.beta + ch0 + cb)[k];
            // GN(y) = y * sc + of with sc = inv * gamma, of = (bias - mean) * sc + beta
            const float2 sc0 = __fmul2_rn(inv2, make_float2(g.x, g.y));
            const float2 sc1 = __fmul2_rn(inv2, make_float2(g.z, g.w));
            const float2 of0 = __ffma2_rn(__fadd2_rn(make_float2(b.x, b.y), nmean2), sc0, make_float2(be.x, be.y));
            const float2 of1 = __ffma2_rn(__fadd2_rn(make_float2(b.z, b.w), nmean2), sc1, make_float2(be.z, be.w));
            float2 z0 = mish2(__ffma2_rn(make_float2(v[4 * k], v[4 * k + 1]), sc0, of0));
            float2 z1 = mish2(__ffma2_rn(make_float2(v[4 * k + 2], v[4 * k + 3]), sc1, of1));
            if (film) {
              const float4 cs4 = reinterpret_cast<const float4*>(fcs + cb)[k];
              const float4 ts4 = reinterpret_cast<const float4*>(fts + cb)[k];
              const float4 ch4 = reinterpret_cast<const float4*>(fcs + p.film_C + cb)[k];
              const float4 th4 = reinterpret_cast<const float4*>(fts + p.film_C + cb)[k];
              z0 = __ffma2_rn(__fadd2_rn(make_float2(cs4.x, cs4.y), make_float2(ts4.x, ts4.y)), z0,
                              __fadd2_rn(make_float2(ch4.x, ch4.y), make_float2(th4.x, th4.y)));
              z1 = __ffma2_rn(__fadd2_rn(make_float2(cs4.z, cs4.w), make_float2(ts4.z, ts4.w)), z1,
                              __fadd2_rn(make_float2(ch4.z, ch4.w), make_float2(th4.z, th4.w)));
            }
            if (rf != nullptr) {
              const float4 r = __ldcs(reinterpret_cast<const float4*>(rf + cb) + k);
              z0 = __fadd2_rn(z0, make_float2(r.x, r.y));
              z1 = __fadd2_rn(z1, make_float2(r.z, r.w));
            }
            if (tw != nullptr) reinterpret_cast<float4*>(tw + cb)[k] = make_float4(z0.x, z0.y, z1.x, z1.y);
            h[2 * k] = pack_half2_sat(z0.x, z0.y);
            h[2 * k + 1] = pack_half2_sat(z1.x, z1.y);
          }
          *reinterpret_cast<uint4*>(o16 + cb) = make_uint4(h[0], h[1], h[2], h[3]);
        } else if (tok_ok) {
          // ragged channel slice (fewer than 8 valid channels left): scalar, masked
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int ch = cb + j;
            if (ch < nval) {
              const float sc = sg.y * p.gamma[ch0 + ch];
              const float of = fmaf(p.bias[ch0 + ch] - sg.x, sc, p.beta[ch0 + ch]);
              const float m = mish_sel(fmaf(v[j], sc, of));
              const float fsc = film ? fcs[ch] + fts[ch] : 1.0f;
              const float fsh = film ? fcs[p.film_C + ch] + fts[p.film_C + ch] : 0.0f;
              const float z = fmaf(fsc, m, fsh) + (rf != nullptr ? rf[ch] : 0.0f);
              o16[ch] = to_half_sat(z);
              if (tw != nullptr) tw[ch] = z;
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
  } else {
    // ---------------- epilogue (warps 2 .. 2 + EPI_WARPS - 1) ----------------
    // Thread (quadrant q, lane) owns accumulator row q*32 + lane (one output
    // channel) and COLS consecutive tile columns (tokens).  A tile covers BN
    // consecutive global tokens, and output rows are affine in the global
    // token, so column c of this warp lives at element o0 + c * out_cs.  Each
    // TMEM load brings CH columns; all per-element work is branch-free and
    // the only branches are per chunk and uniform across the warp.
    constexpr bool kStats = MODE == kEpiStats || MODE == kEpiFused;
    constexpr int CH = 16;
    const int q = warp & 3;                    // TMEM lane quadrant this warp may access
    const int part = (warp - 2) >> 2;          // which COLS-wide slice of the tile's columns
    const int row = q * 32 + lane;
    const int col0 = part * EPI_COLS;
    float2* stat = reinterpret_cast<float2*>(red + 4 * EPI_PARTS * MAX_TILE_SAMPLES);  // [sample][group] (mean, inv)
    // PAIR: [2][sample] partials written by the other CTA (by accumulator
    // parity), then [sample] this CTA's own
    double2* xbuf = reinterpret_cast<double2*>(stat + MAX_TILE_SAMPLES * MAX_TILE_GROUPS);
    double2* xbuf_own = xbuf + 2 * MAX_TILE_SAMPLES;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    const int lmask = p.L - 1;
    const int cs = p.out_cs;
    // Fused, unpaired, every sample inside one column slice (L <= EPI_COLS):
    // the GroupNorm statistics of a slice's samples come from that slice's
    // four warps (one per TMEM lane quadrant) only, so each slice combines
    // them behind its own 128-thread named barrier (3 + part) and the slices
    // run independently of one another.
    const bool by_part = MODE == kEpiFused && !PAIR && p.L <= EPI_COLS;
    const int bp_wpg = p.group_ch >= BM ? 4 : p.group_ch / 32;  // quadrants (warps) of one group
    const double bp_inv_cnt = 1.0 / (static_cast<double>(p.group_ch) * p.L);
    uint32_t acc_iter = 0;
    for (int tile = walk_first; tile < walk_count; tile += walk_stride, ++acc_iter) {
      int m_blk, n_blk;
      tile_mn(tile, m_blk, n_blk);
      const int acc = acc_iter & 1;
      const uint32_t acc_phase = (acc_iter >> 1) & 1;
      bool waited = mbar_wait(&tfull[acc], acc_phase, abort_flag);
      // modes with named barriers below take the same decision in every thread
      // that shares them: the whole epilogue, or one column slice (by_part)
      if constexpr (kStats) waited = by_part ? bar_and(3 + part, 128, waited) : bar_and(2, EPI_THREADS, waited);
      if (!waited) {
        atomicCAS(p.err, 0, kErrWaitTimeoutEpilogue);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int m = m_blk * BM + row;
      const bool m_ok = m < p.m_valid;
      const int mm = m_ok ? m : 0;  // in-range index for per-channel loads
      const float bb = m_ok ? ((p.bias != nullptr ? p.bias[m] : 0.0f) + (p.add_vec != nullptr ? p.add_vec[m] : 0.0f))
                            : 0.0f;
      const int tok0 = n_blk * BN + col0;  // global token of this warp's first column
      // columns [0, lim) of this warp are stored (0 for padding rows)
      const int lim = m_ok ? min(max(p.n_tokens - tok0, 0), EPI_COLS) : 0;
      const long long o0 = static_cast<long long>(tok0) * cs + p.out_base + m;
      const int sample0 = n_blk * p.tile_samples;
      const uint32_t tbase = tmem_base + lane_base + acc * BN + col0;

      bool conv_rows = false;
      if constexpr (MODE == kEpiConv) {
        conv_rows = m_blk * BM < p.conv_rows;  // whole tiles: conv_rows % BM == 0
        if (conv_rows) epi_conv(p, tbase, m, m_ok, tok0, lim);
      }

      // pass 1: GroupNorm partial sums (stats / fused) and the plain store
      float s1 = 0.0f, s2 = 0.0f;
#pragma unroll 1
      for (int c = 0; c < (conv_rows ? 0 : EPI_COLS); c += CH) {
        float v[CH];
        tmem_ld16(tbase + c, v);
        if constexpr (kStats) {
          // sums of v per row; the bias is folded in once per run of columns
#pragma unroll
          for (int j = 0; j < CH; ++j) {
            s1 += v[j];
            s2 = fmaf(v[j], v[j], s2);
            if ((j & 3) == 3) {  // samples span >= 4 columns, so runs end only here
              const int col = col0 + c + j;
              if (((col + 1) & lmask) == 0 || col + 1 == col0 + EPI_COLS) {
                const double n = static_cast<double>(min(p.L, EPI_COLS));
                const double db = bb;
                double d1 = static_cast<double>(s1) + n * db;
                double d2 = static_cast<double>(s2) + 2.0 * db * static_cast<double>(s1) + n * db * db;
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) {
                  d1 += __shfl_xor_sync(0xffffffffu, d1, off);
                  d2 += __shfl_xor_sync(0xffffffffu, d2, off);
                }
                if (lane == 0) {
                  // by_part: [acc][warp][sample of the tile], so the next
                  // tile's partials never overwrite ones still being read
                  const int slot = by_part ? ((acc * EPI_WARPS + q * EPI_PARTS + part) * BP_SAMPLES + (col >> p.L_shift))
                                           : (q * EPI_PARTS + part) * MAX_TILE_SAMPLES + (col >> p.L_shift);
                  red[slot] = make_double2(d1, d2);
                }
                s1 = 0.0f;
                s2 = 0.0f;
              }
            }
          }
        }
        if constexpr (MODE != kEpiFused) {
          float y[CH];
#pragma unroll
          for (int j = 0; j < CH; ++j) y[j] = v[j] + bb;
          if (p.add_tok != nullptr) {
            const float* a = p.add_tok + (static_cast<long long>(tok0 + c) * p.add_cs + p.add_base + mm);
#pragma unroll
            for (int j = 0; j < CH; ++j)
              if (c + j < lim) y[j] += a[j * p.add_cs];
          }
          if (p.act == kActSilu) {
#pragma unroll
            for (int j = 0; j < CH; ++j) y[j] = silu_fast(y[j]);
          } else if (p.act == kActSoftplus) {
#pragma unroll
            for (int j = 0; j < CH; ++j) y[j] = softplus_f(y[j]);
          }
          const long long oc = o0 + static_cast<long long>(c) * cs;
          if (p.act == kActSwiGLU) {
            // the gate lane (even row) takes the up value of the next lane
            __nv_bfloat16* o = static_cast<__nv_bfloat16*>(p.out) + (oc - m + (m >> 1));
#pragma unroll
            for (int j = 0; j < CH; ++j) {
              const float r = __bfloat162float(__float2bfloat16_rn(y[j]));
              const float up = __shfl_xor_sync(0xffffffffu, r, 1);
              if ((lane & 1) == 0 && c + j < lim) o[j * cs] = __float2bfloat16_rn(up * silu_fast(r));
            }
          } else if (p.out_f32) {
            float* o = static_cast<float*>(p.out) + oc;
            if (p.out_accumulate) {
              // the chunk's previous values all requested before its first
              // store (in place, the compiler cannot tell the rows apart, so
              // `o[j * cs] += y[j]` would wait out one round trip per element)
              float prev[CH];
#pragma unroll
              for (int j = 0; j < CH; ++j) prev[j] = c + j < lim ? o[j * cs] : 0.0f;
#pragma unroll
              for (int j = 0; j < CH; ++j)
                if (c + j < lim) o[j * cs] = prev[j] + y[j];
            } else {
#pragma unroll
              for (int j = 0; j < CH; ++j)
                if (c + j < lim) o[j * cs] = y[j];
            }
          } else if (p.fp16 && !p.out_bf16) {
            __half* o = static_cast<__half*>(p.out) + oc;
            if (p.out_lo_off != 0) {
#pragma unroll
              for (int j = 0; j < CH; ++j)
                if (c + j < lim) {
                  const __half hi = to_half_sat(y[j]);
                  o[j * cs] = hi;
                  o[j * cs + p.out_lo_off] = __float2half_rn(y[j] - __half2float(hi));
                }
            } else {
#pragma unroll
              for (int j = 0; j < CH; ++j)
                if (c + j < lim) o[j * cs] = to_half_sat(y[j]);
            }
          } else {
            __nv_bfloat16* o = static_cast<__nv_bfloat16*>(p.out) + oc;
#pragma unroll
            for (int j = 0; j < CH; ++j)
              if (c + j < lim) o[j * cs] = __float2bfloat16_rn(y[j]);
          }
        }
      }
      if constexpr (MODE != kEpiFused) {
        // TMEM buffer may be overwritten by the next tile's MMAs from here on.
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
      }
      // by_part: a warp's 32 channels lie in one group, so lane i combines the
      // partials of the slice's sample i (the group's quadrants in quadrant
      // order; E[y^2] - E[y]^2 in double, clamped at 0, eps 1e-5) and pass 2
      // takes them by shuffle: one barrier of the slice's four warps is all
      // the statistics take
      float2 st_lane = make_float2(0.0f, 1.0f);
      if (kStats && by_part) {
        named_barrier(3 + part, 128);
        const int gw = (q * 32) / p.group_ch;  // this warp's group within the tile
        if (lane < (EPI_COLS >> p.L_shift)) {
          const int ls = (col0 >> p.L_shift) + lane;
          double d1 = 0.0, d2 = 0.0;
          for (int w = 0; w < bp_wpg; ++w) {
            const double2 r = red[(acc * EPI_WARPS + (gw * bp_wpg + w) * EPI_PARTS + part) * BP_SAMPLES + ls];
            d1 += r.x;
            d2 += r.y;
          }
          const double mean = d1 * bp_inv_cnt;
          const double var = fmax(0.0, fma(-mean, mean, d2 * bp_inv_cnt));
          st_lane = make_float2(static_cast<float>(mean), rsqrtf(static_cast<float>(var) + 1e-5f));
        }
      } else if constexpr (kStats) {
        named_barrier(1, EPI_THREADS);
        // combine the partials of the quadrants (and column slices) of each
        // (sample, group) of the tile
        const int tid = threadIdx.x - 64;
        const int warps_per_group = p.group_ch >= BM ? 4 : p.group_ch / 32;
        const int groups_in_tile = BM / (warps_per_group * 32);
        const int items = p.tile_samples * groups_in_tile;
        for (int it = tid; it < items; it += EPI_THREADS) {
          const int ls = it / groups_in_tile;
          const int gl = it - ls * groups_in_tile;
          const int b = sample0 + ls;
          const int p_lo = (ls * p.L) / EPI_COLS;
          const int p_hi = ((ls + 1) * p.L - 1) / EPI_COLS;
          double d1 = 0.0, d2 = 0.0;
          for (int w = 0; w < warps_per_group; ++w)
            for (int pp = p_lo; pp <= p_hi; ++pp) {
              const double2 r = red[((gl * warps_per_group + w) * EPI_PARTS + pp) * MAX_TILE_SAMPLES + ls];
              d1 += r.x;
              d2 += r.y;
            }
          if constexpr (PAIR) {
            // this CTA's half of the group: keep it, and send it to the other CTA
            xbuf_own[ls] = make_double2(d1, d2);
            st_cluster_f64x2(cluster_map(smem_u32(&xbuf[acc * MAX_TILE_SAMPLES + ls]), rank ^ 1), d1, d2);
          } else if constexpr (MODE == kEpiFused) {
            // biased variance E[y^2] - E[y]^2 clamped at 0, eps 1e-5, in double
            const double cnt = static_cast<double>(p.group_ch) * p.L;
            const double mean = d1 / cnt;
            const double var = fmax(0.0, d2 / cnt - mean * mean);
            stat[ls * MAX_TILE_GROUPS + gl] =
                make_float2(static_cast<float>(mean), static_cast<float>(1.0 / sqrt(var + 1e-5)));
          } else {
            if (b < p.n_samples) {
              const int row0 = m_blk * BM + gl * warps_per_group * 32;
              const int g = row0 / p.group_ch;
              const int gpart = (row0 % p.group_ch) / BM;
              double* dst = p.stats + (((static_cast<long long>(b) * p.groups + g) * p.parts + gpart) * 2);
              dst[0] = d1;
              dst[1] = d2;
            }
          }
        }
        named_barrier(1, EPI_THREADS);
        if constexpr (PAIR) {
          if (tid == 0) {
            fence_acq_rel_cluster();
            mbar_arrive_cluster(cluster_map(smem_u32(&xfull[acc]), rank ^ 1));
          }
          const bool got = bar_and(2, EPI_THREADS, mbar_wait_cluster(&xfull[acc], acc_phase, abort_flag));
          if (!got) {
            atomicCAS(p.err, 0, kErrWaitTimeoutEpilogue);
            *abort_flag = 1;
            break;
          }
          for (int ls = tid; ls < p.tile_samples; ls += EPI_THREADS) {
            const double2 a = xbuf_own[ls];
            const double2 o = xbuf[acc * MAX_TILE_SAMPLES + ls];
            const double cnt = static_cast<double>(p.group_ch) * p.L;
            const double mean = (a.x + o.x) / cnt;
            const double var = fmax(0.0, (a.y + o.y) / cnt - mean * mean);
            stat[ls * MAX_TILE_GROUPS] = make_float2(static_cast<float>(mean), static_cast<float>(1.0 / sqrt(var + 1e-5)));
          }
          named_barrier(1, EPI_THREADS);
        }
      }
      if constexpr (MODE == kEpiFused) {
        // pass 2: z = mish((y - mean) * inv * gamma + beta), then FiLM or + residual.
        // Samples span >= 8 columns, so each 8-column half chunk has one sample.
        const int gl = row / p.group_ch;
        const float gam = m_ok ? p.gamma[m] : 0.0f;
        const float bet = m_ok ? p.beta[m] : 0.0f;
        const bool film = p.film_cond != nullptr;
        const float ft_s = film ? p.film_time[p.film_off + mm] : 0.0f;
        const float ft_h = film ? p.film_time[p.film_off + p.film_C + mm] : 0.0f;
        const float* rf = p.res_f32 != nullptr ? p.res_f32 + o0 : nullptr;
        const __half* rh = (rf == nullptr && p.res16 != nullptr) ? static_cast<const __half*>(p.res16) + o0 : nullptr;
        __half* o16 = static_cast<__half*>(p.out) + o0;
        float* tw = p.out_twin != nullptr ? p.out_twin + o0 : nullptr;
        // FiLM (scale, shift) of each 8-column half chunk and the residual run
        // one chunk ahead of their use, so their latency overlaps the math
        auto load_film = [&](int c, float2 (&f)[CH / 8]) {
#pragma unroll
          for (int h = 0; h < CH / 8; ++h) {
            f[h] = make_float2(1.0f, 0.0f);
            if (film) {
              const int b = min(sample0 + ((col0 + c + 8 * h) >> p.L_shift), p.n_samples - 1);
              const float* fc = p.film_cond + (static_cast<long long>(b) * p.film_F + p.film_off + mm);
              f[h] = make_float2(fc[0] + ft_s, fc[p.film_C] + ft_h);
            }
          }
        };
        // all EPI_COLS columns stored (every full tile): running pointers, no
        // per-element predicates
        const bool full = lim == EPI_COLS;
        auto load_res = [&](int c, float (&r)[CH]) {
          if (rf != nullptr && full) {
            const float* rp = rf + static_cast<long long>(c) * cs;
#pragma unroll
            for (int j = 0; j < CH; ++j, rp += cs) r[j] = *rp;
          } else if (rf != nullptr) {
#pragma unroll
            for (int j = 0; j < CH; ++j) r[j] = c + j < lim ? rf[static_cast<long long>(c + j) * cs] : 0.0f;
          } else if (rh != nullptr) {
#pragma unroll
            for (int j = 0; j < CH; ++j)
              r[j] = c + j < lim ? __half2float(rh[static_cast<long long>(c + j) * cs]) : 0.0f;
          } else {
#pragma unroll
            for (int j = 0; j < CH; ++j) r[j] = 0.0f;
          }
        };
        float2 f_cur[CH / 8], f_nxt[CH / 8];
        float r_cur[CH], r_nxt[CH];
        load_film(0, f_cur);
        load_res(0, r_cur);
#pragma unroll 1
        for (int c = 0; c < EPI_COLS; c += CH) {
          const int cn = c + CH < EPI_COLS ? c + CH : c;  // the last chunk re-reads its own values
          load_film(cn, f_nxt);
          load_res(cn, r_nxt);
          float v[CH];
          tmem_ld16(tbase + c, v);
          float z[CH];
          // consecutive columns (tokens) of this channel in packed pairs
#pragma unroll
          for (int h = 0; h < CH / 8; ++h) {
            const int ls = (col0 + c + 8 * h) >> p.L_shift;
            float2 st;
            if (by_part) {
              st.x = __shfl_sync(0xffffffffu, st_lane.x, ls - (col0 >> p.L_shift));
              st.y = __shfl_sync(0xffffffffu, st_lane.y, ls - (col0 >> p.L_shift));
            } else {
              st = stat[ls * MAX_TILE_GROUPS + gl];
            }
            const float sc = st.y * gam;
            const float of = fmaf(bb - st.x, sc, bet);
            const float2 sc2 = make_float2(sc, sc), of2 = make_float2(of, of);
            const float2 fs2 = make_float2(f_cur[h].x, f_cur[h].x), fh2 = make_float2(f_cur[h].y, f_cur[h].y);
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
              const int i = 8 * h + j;
              const float2 mz = mish2(__ffma2_rn(make_float2(v[i], v[i + 1]), sc2, of2));
              const float2 zz = __fadd2_rn(__ffma2_rn(fs2, mz, fh2), make_float2(r_cur[i], r_cur[i + 1]));
              z[i] = zz.x;
              z[i + 1] = zz.y;
            }
          }
          if (full) {
            __half* o = o16 + static_cast<long long>(c) * cs;
#pragma unroll
            for (int j = 0; j < CH; ++j, o += cs) *o = half_satfinite(z[j]);
            if (tw != nullptr) {
              float* t = tw + static_cast<long long>(c) * cs;
#pragma unroll
              for (int j = 0; j < CH; ++j, t += cs) *t = z[j];
            }
          } else {
            __half* o = o16 + static_cast<long long>(c) * cs;
#pragma unroll
            for (int j = 0; j < CH; ++j)
              if (c + j < lim) o[j * cs] = half_satfinite(z[j]);
            if (tw != nullptr) {
              float* t = tw + static_cast<long long>(c) * cs;
#pragma unroll
              for (int j = 0; j < CH; ++j)
                if (c + j < lim) t[j * cs] = z[j];
            }
          }
#pragma unroll
          for (int h = 0; h < CH / 8; ++h) f_cur[h] = f_nxt[h];
#pragma unroll
          for (int j = 0; j < CH; ++j) r_cur[j] = r_nxt[j];
        }
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, TMEM_COLS);
  // no CTA leaves while the other may still write into its shared memory
  if constexpr (PAIR) cluster_sync_all();
}

}  // namespace tc
}  // namespace feb
