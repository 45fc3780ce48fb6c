// The flow head's velocity evaluations of a whole solve as one persistent
// tcgen05 program (reference: src/core/heads/flow/flow.cc:152-184 for the
// MLP, flow.cc:210-323 and span_ops.h:33-56 for the solver stages).
//
// Every GEMM of every evaluation (input projection + time / condition terms,
// the hidden layers, the output projection) is one "layer" of a table in
// device memory; the layers' 128 x 128 output tiles form one sequence
// (layer-major, row tiles fastest) that each CTA walks with stride gridDim.x.
// A layer reads the previous layer's output, so its tile (m, n) may start
// once all row tiles of token block n of the previous layer are stored:
// ctr[layer][n] counts them (GPU-scope release by the epilogue after the
// block's stores, acquire by the TMA producer before it loads the block).
// Tiles depend only on tiles earlier in the sequence and every CTA walks the
// sequence in order, so the program always progresses; each wait is bounded
// and sets the error word and the abort flag when it runs out.
//
// The output projection applies the ODE stage update of the solver in its
// epilogue (the expressions of the separate stage kernel, in its order): it
// writes the state (x or the probe), the stage slope where a later stage
// reads it, and the next evaluation's fp16 input, which the next layer's
// producer loads after the counter says the block is done.
//
// Warp roles are those of tc_gemm_kernel: warp 0 TMA producer, warp 1 TMEM
// allocator + MMA issuer, warps 2-17 epilogue; 6 stages of 128 x 64
// (weights) + 128 x 64 (activations) fp16, fp32 accumulators of 128 x 128
// double-buffered in TMEM.
#pragma once

#include "tc_gemm.cuh"

namespace feb {
namespace fp {

using tc::A_BYTES;
using tc::BK;
using tc::BM;
using tc::EPI_PARTS;
using tc::EPI_THREADS;
using tc::THREADS;

// 128-token tiles: a layer of 4096 tokens is 8 x 32 tiles, about two per SM,
// so one tile's epilogue overlaps the next tile's MMAs on the same SM, and a
// token block's chain of layers has half a tile's latency per layer
constexpr int BN = 128;
constexpr int B_BYTES = BN * BK * 2;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int STAGES = 6;
constexpr int TMEM_COLS = 2 * BN;         // two accumulators
constexpr int EPI_COLS = BN / EPI_PARTS;  // tokens per epilogue warp

constexpr int kMaxSegs = 3;
constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + 256;

struct alignas(64) Layer {
  CUtensorMap a;  // weights [rows_pad][K] fp16, box {64, 128}
  CUtensorMap b;  // input activations [rows][width] fp16, box {64, 128}
  int tiles_m, tiles_n, tile0, kb_total;
  int nseg;
  int seg_kb[kMaxSegs], seg_bcol[kMaxSegs], seg_acol[kMaxSegs];
  int dep, dep_target;  // producing layer (-1: none) and its row tiles
  int m_valid, n_tokens;
  int act;                // tc::kActNone or tc::kActSilu
  const float* add_vec;   // [m] or null
  const float* add_tok;   // [token][add_ld] or null
  int add_ld;
  __half* out;            // fp16 [token][out_ld]; out_lo != 0: the rounding remainder out_lo elements after
  int out_ld, out_lo;
  // output projection: the ODE stage update instead of a store
  int ode, method, stage, steps;
  float* x;
  float* probe;
  float* k[4];
  int ld;                 // row stride of x, probe and k
  __half* next_in;
  int ld_in;
  int next_mode;          // 1: fp16 [b][ld_in]; 2: hi at [b][a], lo at [b][ld_in + a] (row stride 2 ld_in)
};

// Solver fields of the output projection, copied out of the layer table once
// per tile so that the stores below cannot alias them.
struct Ode {
  int method, stage, ld, ld_in, next_mode;
  float dt;
  float* __restrict__ x;
  float* __restrict__ probe;
  float* __restrict__ k0;
  float* __restrict__ k1;
  float* __restrict__ k2;
  __half* __restrict__ next_in;
};

// The stage update of n consecutive tokens b0 .. b0 + n - 1 of action a with
// velocities v (the separate stage kernel's expressions, with k[stage] = v):
// every load of the chunk is issued before its first store.
template <int N>
__device__ __forceinline__ void ode_chunk(const Ode& o, int b0, int n, int a, const float (&v)[N]) {
  float xs[N], ka[N], kb[N], kc[N];
#pragma unroll
  for (int j = 0; j < N; ++j) {
    const long long i = static_cast<long long>(b0 + j) * o.ld + a;
    xs[j] = j < n ? o.x[i] : 0.0f;
    ka[j] = (j < n && o.stage > 0) ? o.k0[i] : 0.0f;
    kb[j] = (j < n && o.method == 2 && o.stage > 1) ? o.k1[i] : 0.0f;
    kc[j] = (j < n && o.method == 2 && o.stage > 2) ? o.k2[i] : 0.0f;
  }
  const float dt = o.dt, half = 0.5f * dt;
#pragma unroll
  for (int j = 0; j < N; ++j) {
    if (j >= n) continue;
    const long long i = static_cast<long long>(b0 + j) * o.ld + a;
    float nxt;
    if (o.method == 0) {
      nxt = xs[j] + dt * v[j];
      o.x[i] = nxt;
    } else if (o.method == 1) {
      if (o.stage == 0) {
        o.k0[i] = v[j];
        nxt = xs[j] + (dt * v[j]);
        o.probe[i] = nxt;
      } else {
        nxt = xs[j] + 0.5f * dt * (ka[j] + v[j]);
        o.x[i] = nxt;
      }
    } else {
      if (o.stage == 0) {
        o.k0[i] = v[j];
        nxt = xs[j] + (half * v[j]);
        o.probe[i] = nxt;
      } else if (o.stage == 1) {
        o.k1[i] = v[j];
        nxt = xs[j] + (half * v[j]);
        o.probe[i] = nxt;
      } else if (o.stage == 2) {
        o.k2[i] = v[j];
        nxt = xs[j] + (dt * v[j]);
        o.probe[i] = nxt;
      } else {
        nxt = xs[j] + (dt / 6.0f) * (ka[j] + (2.0f * kb[j]) + (2.0f * kc[j]) + v[j]);
        o.x[i] = nxt;
      }
    }
    const __half hi = to_half_sat(nxt);
    if (o.next_mode == 2) {
      const long long ii = static_cast<long long>(b0 + j) * 2 * o.ld_in + a;
      o.next_in[ii] = hi;
      o.next_in[ii + o.ld_in] = __float2half_rn(nxt - __half2float(hi));
    } else {
      o.next_in[static_cast<long long>(b0 + j) * o.ld_in + a] = hi;
    }
  }
}

// Epilogue of one tile, one function per kind of layer: each allocates its
// own registers, so the output projection's state and the input projection's
// condition-row prefetch do not spill the hidden layers' loop.  Chunks of 16
// columns: the next chunk's global loads (condition rows, or the ODE state)
// are in flight while this chunk is computed, and this chunk's TMEM load
// overlaps them; the layer's fields are read into registers first (the
// stores cannot alias them).

// The solver fields of an output projection tile.
__device__ __forceinline__ Ode ode_fields(const Layer& L) {
  Ode ode{};
  ode.method = L.method;
  ode.stage = L.stage;
  ode.ld = L.ld;
  ode.ld_in = L.ld_in;
  ode.next_mode = L.next_mode;
  ode.dt = 1.0f / static_cast<float>(L.steps);
  ode.x = L.x;
  ode.probe = L.probe;
  ode.k0 = L.k[0];
  ode.k1 = L.k[1];
  ode.k2 = L.k[2];
  ode.next_in = L.next_in;
  return ode;
}

// Euler: x += dt v, the next input from x.
__device__ __noinline__ void epi_euler(const Layer& L, int m, int tok0, int lim, uint32_t tbase) {
  const Ode ode = ode_fields(L);
  float g_cur[16], g_nxt[16];
  auto load_x = [&](int c, float (&g)[16]) {
    const int n = min(max(lim - c, 0), 16);
#pragma unroll
    for (int j = 0; j < 16; ++j) g[j] = j < n ? ode.x[static_cast<long long>(tok0 + c + j) * ode.ld + m] : 0.0f;
  };
  load_x(0, g_cur);
#pragma unroll 1
  for (int c = 0; c < EPI_COLS; c += 16) {
    uint32_t r[16];
    tmem_ld16_async(tbase + c, r);
    if (c + 16 < EPI_COLS) load_x(c + 16, g_nxt);
    const int n = min(max(lim - c, 0), 16);
    tmem_wait_ld(r);
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (j < n) {
        const int b = tok0 + c + j;
        const float nxt = g_cur[j] + ode.dt * __uint_as_float(r[j]);
        ode.x[static_cast<long long>(b) * ode.ld + m] = nxt;
        const __half hi = to_half_sat(nxt);
        if (ode.next_mode == 2) {
          const long long ii = static_cast<long long>(b) * 2 * ode.ld_in + m;
          ode.next_in[ii] = hi;
          ode.next_in[ii + ode.ld_in] = __float2half_rn(nxt - __half2float(hi));
        } else {
          ode.next_in[static_cast<long long>(b) * ode.ld_in + m] = hi;
        }
      }
#pragma unroll
    for (int j = 0; j < 16; ++j) g_cur[j] = g_nxt[j];
  }
}

// Heun and RK4 stages, eight tokens at a time.
__device__ __noinline__ void epi_stage(const Layer& L, int m, bool m_ok, int tok0, int lim, uint32_t tbase) {
  const Ode ode = ode_fields(L);
#pragma unroll 1
  for (int c = 0; c < EPI_COLS; c += 8) {
    float v[8];
    tmem_ld8(tbase + c, v);
    if (m_ok) ode_chunk<8>(ode, tok0 + c, min(max(lim - c, 0), 8), m, v);
  }
}

// Hidden layers, and with TOK the input projection (+ the condition rows).
template <bool TOK>
__device__ __noinline__ void epi_plain(const Layer& L, int m, int mm, int tok0, int lim, uint32_t tbase) {
  const float addv = L.add_vec != nullptr ? L.add_vec[mm] : 0.0f;
  const float* __restrict__ add_tok = L.add_tok;
  const int add_ld = L.add_ld, out_ld = L.out_ld, out_lo = L.out_lo;
  const bool silu = L.act == tc::kActSilu;
  __half* __restrict__ out = L.out;
  // the condition rows (input projection only) one chunk ahead
  float g_cur[16], g_nxt[16];
  constexpr bool has_tok = TOK;
  auto load_g = [&](int c, float (&g)[16]) {
    const int n = min(max(lim - c, 0), 16);
    const float* ap = add_tok + (static_cast<long long>(tok0 + c) * add_ld + mm);
#pragma unroll
    for (int j = 0; j < 16; ++j) g[j] = j < n ? ap[static_cast<long long>(j) * add_ld] : 0.0f;
  };
  if constexpr (has_tok) load_g(0, g_cur);
#pragma unroll 1
  for (int c = 0; c < EPI_COLS; c += 16) {
    uint32_t r[16];
    tmem_ld16_async(tbase + c, r);
    if (has_tok && c + 16 < EPI_COLS) load_g(c + 16, g_nxt);
    const int n = min(max(lim - c, 0), 16);
    tmem_wait_ld(r);
    float y[16];
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      float2 v2 = make_float2(__uint_as_float(r[j]) + addv, __uint_as_float(r[j + 1]) + addv);
      if (has_tok) v2 = __fadd2_rn(v2, make_float2(g_cur[j], g_cur[j + 1]));
      if (silu) v2 = silu2_fma(v2);  // one MUFU operation per element (the epilogue's bound otherwise)
      y[j] = v2.x;
      y[j + 1] = v2.y;
    }
    __half* o = out + (static_cast<long long>(tok0 + c) * out_ld + m);
    if (n == 16) {
      if (out_lo != 0) {
#pragma unroll
        for (int j = 0; j < 16; ++j, o += out_ld) {
          const __half hi = to_half_sat(y[j]);
          o[0] = hi;
          o[out_lo] = __float2half_rn(y[j] - __half2float(hi));
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j, o += out_ld) *o = half_satfinite(y[j]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (j < n) {
          const __half hi = to_half_sat(y[j]);
          o[static_cast<long long>(j) * out_ld] = hi;
          if (out_lo != 0) o[static_cast<long long>(j) * out_ld + out_lo] = __float2half_rn(y[j] - __half2float(hi));
        }
    }
    if (has_tok)
#pragma unroll
      for (int j = 0; j < 16; ++j) g_cur[j] = g_nxt[j];
  }
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Per-tile global-timer stamps when `trace` is set: [tile][kTraceStamps] =
// producer start, dependency met, last MMA issued, epilogue start (the
// accumulator is ready), block published.
constexpr int kTraceStamps = 5;

__global__ void __launch_bounds__(THREADS, 1)
    flow_program_kernel(const Layer* __restrict__ layers, int n_layers, int total_tiles, int* ctr, int ctr_ld,
                        int* err, unsigned long long* trace) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

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
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();
  griddep_launch();

  // layer of a tile (tiles are visited in increasing order)
  auto advance_layer = [&](int tile, int li) {
    while (li + 1 < n_layers && tile >= layers[li + 1].tile0) ++li;
    return li;
  };

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const uint64_t keep_a = l2_policy_evict_last();
      uint32_t kb_iter = 0;
      uint32_t armed = 0, armed_phase = 0;
      bool ok = true;
      int li = 0, code = kErrWaitTimeoutProducer;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        li = advance_layer(tile, li);
        const Layer& L = layers[li];
        const int t = tile - L.tile0;
        const int m_blk = t % L.tiles_m, n_blk = t / L.tiles_m;
        if (trace != nullptr) trace[static_cast<long long>(tile) * kTraceStamps] = global_ns();
        // the weights depend on nothing: the first stages' weight tiles go out
        // before the dependency wait, their activation tiles after it
        const int early = L.kb_total < STAGES ? L.kb_total : STAGES;
        auto stage_of = [&](int k, int& s_, int& kb_) {
          s_ = 0;
          kb_ = k;
          while (kb_ >= L.seg_kb[s_]) {
            kb_ -= L.seg_kb[s_];
            ++s_;
          }
        };
        for (int k = 0; k < early && ok; ++k) {
          const uint32_t it = kb_iter + k;
          const int stage = it % STAGES;
          const uint32_t phase = (it / STAGES) & 1;
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          int s_, kb_;
          stage_of(k, s_, kb_);
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          armed |= 1u << stage;
          armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
          tma_load_2d_hint(smem + stage * STAGE_BYTES, &L.a, L.seg_acol[s_] + kb_ * BK, m_blk * BM, &full[stage],
                           keep_a);
        }
        if (ok && L.dep >= 0) {
          // the producing layer's row tiles of this token block are stored
          const int* c = ctr + L.dep * ctr_ld + n_blk;
          const uint64_t t0 = global_ns();
          for (uint32_t spin = 0;; ++spin) {
            int v;
            asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(c) : "memory");
            if (v >= L.dep_target) break;
            __nanosleep(64);
            if ((spin & 63u) == 63u && (*abort_flag != 0 || global_ns() - t0 > kWaitNs)) {
              ok = false;
              code = kErrDependencyTimeout;
              break;
            }
          }
          if (ok) fence_proxy_async_global();
        }
        if (trace != nullptr) trace[static_cast<long long>(tile) * kTraceStamps + 1] = global_ns();
        for (int k = 0; k < early && ok; ++k) {
          const int stage = (kb_iter + k) % STAGES;
          int s_, kb_;
          stage_of(k, s_, kb_);
          tma_load_2d(smem + stage * STAGE_BYTES + A_BYTES, &L.b, L.seg_bcol[s_] + kb_ * BK, n_blk * BN, &full[stage]);
        }
        kb_iter += early;
        for (int k = early; k < L.kb_total && ok; ++k, ++kb_iter) {
          const int stage = kb_iter % STAGES;
          const uint32_t phase = (kb_iter / STAGES) & 1;
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          int s_, kb_;
          stage_of(k, s_, kb_);
          uint8_t* a_dst = smem + stage * STAGE_BYTES;
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          armed |= 1u << stage;
          armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
          tma_load_2d_hint(a_dst, &L.a, L.seg_acol[s_] + kb_ * BK, m_blk * BM, &full[stage], keep_a);
          tma_load_2d(a_dst + A_BYTES, &L.b, L.seg_bcol[s_] + kb_ * BK, n_blk * BN, &full[stage]);
        }
      }
      if (!ok) {
        atomicCAS(err, 0, code);
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
      const uint32_t idesc = idesc_f16_f32(BM, BN);
      uint32_t kb_iter = 0, acc_iter = 0;
      bool ok = true;
      int li = 0;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x, ++acc_iter) {
        li = advance_layer(tile, li);
        const int kb_total = layers[li].kb_total;
        const int acc = acc_iter & 1;
        const uint32_t acc_phase = (acc_iter >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < kb_total; ++kb, ++kb_iter) {
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
          for (int k = 0; k < BK / 16; ++k)
            umma_bf16(d_tmem, sw128_desc(a_addr + k * 32), sw128_desc(b_addr + k * 32), idesc,
                      (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit(&empty[stage]);
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        if (trace != nullptr) trace[static_cast<long long>(tile) * kTraceStamps + 2] = global_ns();
      }
      if (!ok) {
        atomicCAS(err, 0, kErrWaitTimeoutMma);
        *abort_flag = 1;
      }
      umma_commit(drain);
      for (uint32_t spin = 0; spin < kSpinLimit && !mbar_try_wait(drain, 0); ++spin) {
      }
    }
  } else {
    // ---------------- epilogue (warps 2 .. 17) ----------------
    // Thread (quadrant q, lane) owns accumulator row q*32 + lane (one output
    // feature) and EPI_COLS consecutive tokens of the tile.
    const int q = warp & 3;
    const int part = (warp - 2) >> 2;
    const int row = q * 32 + lane;
    const int col0 = part * EPI_COLS;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    uint32_t acc_iter = 0;
    int li = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, ++acc_iter) {
      li = advance_layer(tile, li);
      const Layer& L = layers[li];
      const int t = tile - L.tile0;
      const int m_blk = t % L.tiles_m, n_blk = t / L.tiles_m;
      const int acc = acc_iter & 1;
      const uint32_t acc_phase = (acc_iter >> 1) & 1;
      const bool waited = bar_and(2, EPI_THREADS, mbar_wait(&tfull[acc], acc_phase, abort_flag));
      if (!waited) {
        atomicCAS(err, 0, kErrWaitTimeoutEpilogue);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      if (trace != nullptr && threadIdx.x == 64) trace[static_cast<long long>(tile) * kTraceStamps + 3] = global_ns();
      const int m = m_blk * BM + row;
      const bool m_ok = m < L.m_valid;
      const int mm = m_ok ? m : 0;
      const int tok0 = n_blk * BN + col0;
      const int lim = m_ok ? min(max(L.n_tokens - tok0, 0), EPI_COLS) : 0;
      const uint32_t tbase = tmem_base + lane_base + acc * BN + col0;
      if (L.ode != 0 && L.method == 0) {
        epi_euler(L, m, tok0, lim, tbase);
      } else if (L.ode != 0) {
        epi_stage(L, m, m_ok, tok0, lim, tbase);
      } else if (L.add_tok != nullptr) {
        epi_plain<true>(L, m, mm, tok0, lim, tbase);
      } else {
        epi_plain<false>(L, m, mm, tok0, lim, tbase);
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      // publish the token block once every epilogue thread's stores are done:
      // the barrier orders them before this thread's GPU-scope fence and
      // release (cumulative), which the consumer's acquire pairs with
      named_barrier(1, EPI_THREADS);
      if (threadIdx.x == 64) {
        __threadfence();
        fence_proxy_async_global();
        asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(ctr + li * ctr_ld + n_blk) : "memory");
        if (trace != nullptr) trace[static_cast<long long>(tile) * kTraceStamps + 4] = global_ns();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, TMEM_COLS);
}

}  // namespace fp
}  // namespace feb
