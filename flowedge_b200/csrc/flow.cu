// Device-resident flow-matching head: velocity MLP integrated with Euler /
// Heun / RK4 (reference: src/core/heads/flow/flow.cc:64-323).
//
//   h = SiLU(W_in x + W_t [sin(t f) | cos(t f)] + c_emb),  c_emb = W_c cond
//   h = SiLU(W_l h)  (mlp_layers times),  v = W_out h        (no biases)
//
// Rows of a batch are independent samples sharing the weights.  One ODE step
// (1, 2 or 4 velocity evaluations) is captured as a CUDA graph per (batch,
// method, path); the step index lives in device memory and is advanced by the
// graph itself, so a resumable solve replays the same graph.  Small batches
// use the weight-streaming CUDA-core GEMV (fp32 or bf16 weights); batches of
// 128+ rows in bf16 mode use the tcgen05 GEMM with SiLU / time / condition
// terms in its epilogue.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "flow_program.cuh"
#include "runtime.cuh"
#include "simt.cuh"

namespace feb {
namespace {

constexpr int kTcMinRows = 128;


struct Mat {
  int rows = 0, rows_pad = 0, cols = 0, cols_pad = 0;
  void* w = nullptr;  // [rows_pad][cols_pad]
  // fp32 engines, tensor-core path: fp16 [rows_pad][3 * cols_pad] rows
  // [hi(W) | hi(W) | lo(W)], lo = W - hi rounded to fp16, so that one GEMM
  // over the activations split the same way, [hi(x) | lo(x)] against
  // [hi | hi | lo] with the x segments hi, lo, hi, gives
  // hi(W) hi(x) + hi(W) lo(x) + lo(W) hi(x), W x to about 2^-21 relative
  void* w3 = nullptr;
  SimtSlice* slices = nullptr;
  int nslices = 0;
};

// t of velocity evaluation `stage` within step `step` (flow.cc:275-300)
__device__ __forceinline__ float stage_time(int step, int steps, int method, int stage) {
  const float dt = 1.0f / static_cast<float>(steps);
  const float t = static_cast<float>(step) * dt;
  if (method == 1) return stage == 0 ? t : t + dt;
  if (method == 2) {
    const float half = 0.5f * dt;
    return stage == 0 ? t : (stage == 3 ? t + dt : t + half);
  }
  return t;
}

// tp[h] = sum_j Wt[h][j] * [sin(t f) | cos(t f)]_j; one warp per row h, the
// lanes stride the row (coalesced) and a shuffle tree adds their sums
constexpr int kTimeProjRowsPerBlock = 8;
__global__ void time_proj_kernel(const int* step_idx, int steps, int method, int stage, const float* freqs, int half,
                                 const float* wt, int H, float* tp) {
  griddep_wait();
  griddep_launch();
  extern __shared__ float sinu[];
  const float t = stage_time(*step_idx, steps, method, stage);
  for (int j = threadIdx.x; j < half; j += blockDim.x) {
    sinu[j] = sinf(t * freqs[j]);
    sinu[half + j] = cosf(t * freqs[j]);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  for (int h = blockIdx.x * warps + warp; h < H; h += gridDim.x * warps) {
    const float* w = wt + static_cast<long long>(h) * 2 * half;
    float acc = 0.0f;
    for (int j = lane; j < 2 * half; j += 32) acc = fmaf(w[j], sinu[j], acc);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) tp[h] = acc;
  }
}

// time_proj_kernel for every evaluation of steps first .. first + count - 1
// at once (blockIdx.y = evaluation e = (step - first) * stages + stage), into
// tp[e][h], for the persistent tensor-core solve
__global__ void time_proj_all_kernel(int first, int steps, int method, int stages, const float* freqs, int half,
                                     const float* wt, int H, float* tp) {
  extern __shared__ float sinu[];
  const int e = blockIdx.y;
  const float t = stage_time(first + e / stages, steps, method, e % stages);
  for (int j = threadIdx.x; j < half; j += blockDim.x) {
    sinu[j] = sinf(t * freqs[j]);
    sinu[half + j] = cosf(t * freqs[j]);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  float* out = tp + static_cast<long long>(e) * H;
  for (int h = blockIdx.x * warps + warp; h < H; h += gridDim.x * warps) {
    const float* w = wt + static_cast<long long>(h) * 2 * half;
    float acc = 0.0f;
    for (int j = lane; j < 2 * half; j += 32) acc = fmaf(w[j], sinu[j], acc);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) out[h] = acc;
  }
}

// ODE stage update after velocity evaluation `stage` wrote k[stage]
// (span_ops.h:33-56 expression order).  Writes the next evaluation's input
// (probe or x) into `next_in` (fp32 or bf16, padded width ld_in).
struct OdeParams {
  int B, A, ld;  // rows, action dim, row stride of the fp32 state buffers
  int method, stage, steps;
  const int* step_idx;
  int* step_out;  // incremented after the last stage (null: no increment)
  float* x;
  float* probe;
  const float* k[4];
  void* next_in;
  int ld_in;
  int next_mode;  // 0 fp32, 1 fp16, 2 fp16 hi at a and lo at ld_in + a (row stride 2 ld_in)
};

__global__ void ode_stage_kernel(const OdeParams p) {
  griddep_wait();
  griddep_launch();
  const float dt = 1.0f / static_cast<float>(p.steps);
  const long long total = static_cast<long long>(p.B) * p.A;
  const int last = p.method == 0 ? 0 : (p.method == 1 ? 1 : 3);
  const bool narrow = total < (1LL << 31);  // 32-bit index division (uniform branch)
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    int b, a;
    if (narrow) {
      const int ii = static_cast<int>(i);
      b = ii / p.A;
      a = ii - b * p.A;
    } else {
      b = static_cast<int>(i / p.A);
      a = static_cast<int>(i - static_cast<long long>(b) * p.A);
    }
    const long long o = static_cast<long long>(b) * p.ld + a;
    float nxt;
    if (p.method == 0) {
      nxt = p.x[o] + dt * p.k[0][o];
      p.x[o] = nxt;
    } else if (p.method == 1) {
      if (p.stage == 0) {
        nxt = p.x[o] + (dt * p.k[0][o]);
        p.probe[o] = nxt;
      } else {
        nxt = p.x[o] + 0.5f * dt * (p.k[0][o] + p.k[1][o]);
        p.x[o] = nxt;
      }
    } else {
      const float half = 0.5f * dt;
      if (p.stage == 0) {
        nxt = p.x[o] + (half * p.k[0][o]);
        p.probe[o] = nxt;
      } else if (p.stage == 1) {
        nxt = p.x[o] + (half * p.k[1][o]);
        p.probe[o] = nxt;
      } else if (p.stage == 2) {
        nxt = p.x[o] + (dt * p.k[2][o]);
        p.probe[o] = nxt;
      } else {
        nxt = p.x[o] + (dt / 6.0f) * (p.k[0][o] + (2.0f * p.k[1][o]) + (2.0f * p.k[2][o]) + p.k[3][o]);
        p.x[o] = nxt;
      }
    }
    if (p.next_mode == 2) {
      const long long ii = static_cast<long long>(b) * 2 * p.ld_in + a;
      const __half hi = to_half_sat(nxt);
      static_cast<__half*>(p.next_in)[ii] = hi;
      static_cast<__half*>(p.next_in)[ii + p.ld_in] = __float2half_rn(nxt - __half2float(hi));
    } else {
      const long long ii = static_cast<long long>(b) * p.ld_in + a;
      if (p.next_mode == 1) static_cast<__half*>(p.next_in)[ii] = to_half_sat(nxt);
      else static_cast<float*>(p.next_in)[ii] = nxt;
    }
  }
  if (p.step_out != nullptr && p.stage == last && blockIdx.x == 0 && threadIdx.x == 0) *p.step_out = *p.step_idx + 1;
}

// fp32 [B][A] (dense) -> padded fp32 state and padded next-input buffer;
// in_mode as OdeParams::next_mode
__global__ void load_rows_kernel(const float* src, int B, int A, float* dst, int ld, void* in, int ld_in, int in_mode) {
  const long long total = static_cast<long long>(B) * ld_in;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int b = static_cast<int>(i / ld_in);
    const int a = static_cast<int>(i - static_cast<long long>(b) * ld_in);
    const float v = a < A ? src[static_cast<long long>(b) * A + a] : 0.0f;
    if (dst != nullptr && a < ld) dst[static_cast<long long>(b) * ld + a] = v;
    if (in_mode == 2) {
      const long long ii = static_cast<long long>(b) * 2 * ld_in + a;
      const __half hi = to_half_sat(v);
      static_cast<__half*>(in)[ii] = hi;
      static_cast<__half*>(in)[ii + ld_in] = __float2half_rn(v - __half2float(hi));
    } else if (in_mode == 1) {
      static_cast<__half*>(in)[i] = to_half_sat(v);
    } else {
      static_cast<float*>(in)[i] = v;
    }
  }
}

__global__ void store_rows_kernel(const float* src, int B, int A, int ld, float* dst) {
  const long long total = static_cast<long long>(B) * A;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int b = static_cast<int>(i / A);
    const int a = static_cast<int>(i - static_cast<long long>(b) * A);
    dst[i] = src[static_cast<long long>(b) * ld + a];
  }
}

// ---------------------------------------------------------------------------
// Fused small-batch solve: one cooperative launch runs `count` ODE steps
// (flow.cc:152-184, 210-323).  Every CTA is resident; per velocity evaluation
//   P1  sinusoid of t (each CTA), then per hidden row h (one warp per row,
//       lanes stride K): tp = W_t[h] . sinu, h0 = SiLU(W_in[h] . x + tp + c_emb)
//   P2  hidden layers h = SiLU(W_l h), one phase each
//   P3  v = W_out h; the warp of output element a then applies the ODE stage
//       update of ode_stage_kernel to (b, a) and writes the next input
// separated by bounded grid barriers (coop_grid_sync).  Rows are spread
// CTA-first so short phases still use every SM; inputs written inside the
// launch are staged into shared memory through L2 (ld.global.cg).
constexpr int kFlowThreads = 512;
constexpr int kFlowWarps = kFlowThreads / 32;
constexpr int kFuseMaxBatch = 8;
constexpr int kFuseMaxLayers = 8;

struct FlowFusedParams {
  int B, A, H, half, layers, steps, method, first, count;
  const float* freqs;  // [half]
  const float* wt;     // [H][2 half] fp32
  const void* w_in;    // [H][ld_in], fp32 or fp16
  int ld_in;
  const void* w_l[kFuseMaxLayers];  // [H][ld_l]
  int ld_l;
  const void* w_out;  // [A][ld_out]
  int ld_out;
  const float* cemb;  // [B][H]
  float* x;           // [B][ld_a] state
  float* probe;
  float* k[4];
  float* xin;         // [B][ld_a] current evaluation input (fp32)
  int ld_a;
  float* h0;
  float* h1;  // [B][H]
  unsigned* sync;
  int* err;
};

// dot products of one weight row with nb staged vectors (row stride ldv);
// lane l takes pairs (k, k + 1), k = 2 l + 64 j, and issues up to
// kFlowPairs of its weight loads before the first multiply
constexpr int kFlowPairs = 16;
template <bool HALF>
__device__ __forceinline__ void flow_dots(const void* w, long long row, int ld, int n, const float* v, int ldv,
                                          int nb, float (&acc)[kFuseMaxBatch]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int b = 0; b < kFuseMaxBatch; ++b) acc[b] = 0.0f;
  for (int k0 = 2 * lane; k0 < n; k0 += 64 * kFlowPairs) {
    float2 wv[kFlowPairs];
#pragma unroll
    for (int u = 0; u < kFlowPairs; ++u) {
      const int k = k0 + 64 * u;
      wv[u] = make_float2(0.0f, 0.0f);
      if (k < n) {
        if constexpr (HALF) {
          wv[u] = __half22float2(*reinterpret_cast<const __half2*>(static_cast<const __half*>(w) + row * ld + k));
        } else {
          wv[u] = *reinterpret_cast<const float2*>(static_cast<const float*>(w) + row * ld + k);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kFlowPairs; ++u) {
      const int k = k0 + 64 * u;
      if (k < n) {
        const bool two = k + 1 < n;
#pragma unroll
        for (int b = 0; b < kFuseMaxBatch; ++b)
          if (b < nb) {
            acc[b] = fmaf(wv[u].x, v[b * ldv + k], acc[b]);
            if (two) acc[b] = fmaf(wv[u].y, v[b * ldv + k + 1], acc[b]);
          }
      }
    }
  }
#pragma unroll
  for (int b = 0; b < kFuseMaxBatch; ++b)
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc[b] += __shfl_xor_sync(0xffffffffu, acc[b], off);
}

template <bool HALF>
__global__ void __launch_bounds__(kFlowThreads, 1) flow_fused_kernel(const FlowFusedParams p) {
  extern __shared__ float sv[];  // [B][max(H, ld_a)] staged vectors, then [2 half] sinusoid
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gwarp = warp * gridDim.x + blockIdx.x, nwarps = gridDim.x * kFlowWarps;
  const int B = p.B, A = p.A, H = p.H;
  const int ldv = H > p.ld_a ? H : p.ld_a;
  float* sinu = sv + B * ldv;
  const int stages = p.method == 0 ? 1 : (p.method == 1 ? 2 : 4);
  const int last = stages - 1;
  const float dt = 1.0f / static_cast<float>(p.steps);
  unsigned epoch = 0;
  for (int step = p.first; step < p.first + p.count; ++step) {
    for (int s = 0; s < stages; ++s) {
      // P1: time projection and input layer
      const float t = stage_time(step, p.steps, p.method, s);
      for (int j = threadIdx.x; j < p.half; j += blockDim.x) {
        sinu[j] = sinf(t * p.freqs[j]);
        sinu[p.half + j] = cosf(t * p.freqs[j]);
      }
      for (int i = threadIdx.x; i < B * p.ld_a; i += blockDim.x) {
        const int b = i / p.ld_a, a = i - b * p.ld_a;
        sv[b * ldv + a] = __ldcg(p.xin + i);
      }
      __syncthreads();
      for (int h = gwarp; h < H; h += nwarps) {
        const float* w = p.wt + static_cast<long long>(h) * 2 * p.half;
        float tp = 0.0f;
        for (int j = lane; j < 2 * p.half; j += 32) tp = fmaf(w[j], sinu[j], tp);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) tp += __shfl_xor_sync(0xffffffffu, tp, off);
        float acc[kFuseMaxBatch];
        flow_dots<HALF>(p.w_in, h, p.ld_in, A, sv, ldv, B, acc);
        if (lane == 0) {
#pragma unroll
          for (int b = 0; b < kFuseMaxBatch; ++b)
            if (b < B)
              p.h0[static_cast<long long>(b) * H + h] =
                  silu_f((acc[b] + tp) + p.cemb[static_cast<long long>(b) * H + h]);
        }
      }
      if (!coop_grid_sync(p.sync, p.err, epoch)) return;
      // P2: hidden layers
      float* hin = p.h0;
      float* hout = p.h1;
      for (int l = 0; l < p.layers; ++l) {
        for (int i = threadIdx.x; i < B * H; i += blockDim.x) {
          const int b = i / H, c = i - b * H;
          sv[b * ldv + c] = __ldcg(hin + i);
        }
        __syncthreads();
        for (int r = gwarp; r < H; r += nwarps) {
          float acc[kFuseMaxBatch];
          flow_dots<HALF>(p.w_l[l], r, p.ld_l, H, sv, ldv, B, acc);
          if (lane == 0) {
#pragma unroll
            for (int b = 0; b < kFuseMaxBatch; ++b)
              if (b < B) hout[static_cast<long long>(b) * H + r] = silu_f(acc[b]);
          }
        }
        if (!coop_grid_sync(p.sync, p.err, epoch)) return;
        float* tmp = hin;
        hin = hout;
        hout = tmp;
      }
      // P3: output layer and the ODE stage update (span_ops.h:33-56 order)
      for (int i = threadIdx.x; i < B * H; i += blockDim.x) {
        const int b = i / H, c = i - b * H;
        sv[b * ldv + c] = __ldcg(hin + i);
      }
      __syncthreads();
      for (int a = gwarp; a < A; a += nwarps) {
        float acc[kFuseMaxBatch];
        flow_dots<HALF>(p.w_out, a, p.ld_out, H, sv, ldv, B, acc);
        if (lane == 0)
#pragma unroll
          for (int b = 0; b < kFuseMaxBatch; ++b) {
            if (b >= B) continue;
            const long long o = static_cast<long long>(b) * p.ld_a + a;
            p.k[s][o] = acc[b];
            const float x = __ldcg(p.x + o);
            float nxt;
            if (p.method == 0) {
              nxt = x + dt * acc[b];
              p.x[o] = nxt;
            } else if (p.method == 1) {
              if (s == 0) {
                nxt = x + (dt * acc[b]);
                p.probe[o] = nxt;
              } else {
                nxt = x + 0.5f * dt * (__ldcg(p.k[0] + o) + acc[b]);
                p.x[o] = nxt;
              }
            } else {
              const float hf = 0.5f * dt;
              if (s == 0) {
                nxt = x + (hf * acc[b]);
                p.probe[o] = nxt;
              } else if (s == 1) {
                nxt = x + (hf * acc[b]);
                p.probe[o] = nxt;
              } else if (s == 2) {
                nxt = x + (dt * acc[b]);
                p.probe[o] = nxt;
              } else {
                nxt = x + (dt / 6.0f) * (__ldcg(p.k[0] + o) + (2.0f * __ldcg(p.k[1] + o)) +
                                         (2.0f * __ldcg(p.k[2] + o)) + acc[b]);
                p.x[o] = nxt;
              }
            }
            p.xin[o] = nxt;
          }
      }
      if (!coop_grid_sync(p.sync, p.err, epoch)) return;
      (void)last;
    }
  }
}

class Flow final : public FlowDevice {
 public:
  Flow(std::shared_ptr<DeviceContext> ctx, Precision prec) : ctx_(std::move(ctx)), prec_(prec) {}
  ~Flow() override {
    for (auto& [k, g] : graphs_) cudaGraphExecDestroy(g);
    for (auto& [k, pr] : programs_) {
      cudaFree(pr.table);
      cudaFree(pr.ctr);
      cudaFree(pr.tp);
      cudaFree(pr.trace);
    }
    if (pinned_ != nullptr) cudaFreeHost(pinned_);
  }
  bool load(const TensorTable& t, std::string& err);
  const FlowConfig& config() const noexcept override { return cfg_; }
  std::size_t capacity() const noexcept override { return cap_; }
  int reserve(std::size_t batch, std::string& err) noexcept override;
  int begin(const float* condition, const float* x0, std::size_t batch, std::size_t steps, int method,
            bool condition_on_device, std::string& err) noexcept override;
  int advance(std::size_t first, std::size_t count, float* out, std::string& err) noexcept override;
  int sample_device(const float* condition, const float* x0, std::size_t batch, std::size_t steps, int method,
                    float* out, void* stream, std::string& err) noexcept override;
  int sample_static(const float* condition, const float* x0, std::size_t batch, std::size_t steps, int method,
                    float* out, void* stream, std::string& err) noexcept override;

 private:
  bool use_tc(std::size_t batch) const { return tc_ok_ && static_cast<int>(batch) >= kTcMinRows; }
  // fp32 engines run the tensor-core path on hi / lo fp16 splits
  bool split() const { return prec_ != Precision::kBF16; }
  int in_mode(bool tc) const { return tc ? (split() ? 2 : 1) : 0; }
  bool gemm(const Mat& m, const void* in, int in_ld, std::size_t batch, float* out_f32, void* out_half, int out_ld,
            const float* add_vec, const float* add_tok, int act, bool tc, cudaStream_t st, std::string& err);
  bool record_step(std::size_t batch, int method, bool tc, cudaStream_t st, std::string& err);
  bool prepare(const float* condition, const float* x0, std::size_t batch, bool cond_device, bool x_device,
               cudaStream_t st, std::string& err);

  std::shared_ptr<DeviceContext> ctx_;
  Precision prec_;
  FlowConfig cfg_{};
  int a_pad_ = 0, c_pad_ = 0;
  bool tc_ok_ = false;
  DeviceArena wts_;
  Mat in_, cond_, out_;
  std::vector<Mat> layers_;
  float* wt_ = nullptr;     // [H][td] fp32
  float* freqs_ = nullptr;  // [td/2]
  DeviceArena ws_;
  std::size_t cap_ = 0, cap_rows_ = 0;
  float *x_ = nullptr, *probe_ = nullptr, *k_[4] = {}, *cemb_ = nullptr, *tp_ = nullptr, *part_ = nullptr;
  float* in_cond_ = nullptr;
  void *xin_ = nullptr, *h0_ = nullptr, *h1_ = nullptr, *cin_ = nullptr;
  int* step_ = nullptr;
  std::size_t part_elems_ = 0;
  float* pinned_ = nullptr;
  std::size_t batch_ = 0, steps_ = 0;
  int method_ = 0;
  std::map<std::tuple<std::size_t, int, bool, std::size_t>, cudaGraphExec_t> graphs_;
  unsigned* fsync_ = nullptr;  // grid-barrier words of the fused small-batch solve
  // persistent tensor-core solve (flow_program_kernel): one layer table per
  // (batch, first step, steps run, method, total steps), its block counters
  // and the time projections of its evaluations
  struct Program {
    fp::Layer* table = nullptr;
    int* ctr = nullptr;
    float* tp = nullptr;
    unsigned long long* trace = nullptr;  // FLOWEDGE_FLOW_TRACE=<file>: per-tile stamps of the last call
    int n_layers = 0, total_tiles = 0, tiles_n = 0, n_evals = 0;
    std::vector<int> tiles_m;             // per layer
  };
  std::map<std::tuple<std::size_t, std::size_t, std::size_t, int, std::size_t>, Program> programs_;
  bool program_solve(std::size_t first, std::size_t count, cudaStream_t st, std::string& err, bool& used);
  // one cooperative launch for `count` steps of a small batch, or false when
  // the batch / shape does not take the fused kernel
  bool fused_advance(std::size_t first, std::size_t count, cudaStream_t st, std::string& err, bool& used);
};

bool Flow::load(const TensorTable& t, std::string& err) {
  const HostTensor* in = t.find("flow.in_proj.weight");
  const HostTensor* tp = t.find("flow.time_proj.weight");
  const HostTensor* cp = t.find("flow.cond_proj.weight");
  const HostTensor* op = t.find("flow.out_proj.weight");
  if (in == nullptr || tp == nullptr || cp == nullptr || op == nullptr || in->ndim != 2 || tp->ndim != 2 ||
      cp->ndim != 2 || op->ndim != 2) {
    err = "flow.* projections missing";
    return false;
  }
  cfg_.hidden = in->shape[0];
  cfg_.action_dim = in->shape[1];
  cfg_.time_dim = tp->shape[1];
  cfg_.cond_dim = cp->shape[1];
  if (cfg_.hidden == 0 || cfg_.action_dim == 0 || cfg_.time_dim == 0 || cfg_.cond_dim == 0 ||
      cfg_.time_dim % 2 != 0 || tp->shape[0] != cfg_.hidden || cp->shape[0] != cfg_.hidden ||
      op->shape[0] != cfg_.action_dim || op->shape[1] != cfg_.hidden) {
    err = "flow.* projection shapes are inconsistent";
    return false;
  }
  std::vector<const HostTensor*> layer_t;
  for (std::size_t n = 0; n < 8; ++n) {
    const HostTensor* lw = t.find("flow.layers." + std::to_string(n) + ".weight");
    if (lw == nullptr) break;
    if (lw->ndim != 2 || lw->shape[0] != cfg_.hidden || lw->shape[1] != cfg_.hidden) {
      err = "flow layer shape mismatch";
      return false;
    }
    layer_t.push_back(lw);
  }
  cfg_.mlp_layers = layer_t.size();
  const int H = static_cast<int>(cfg_.hidden);
  a_pad_ = static_cast<int>((cfg_.action_dim + 63) / 64 * 64);
  c_pad_ = static_cast<int>((cfg_.cond_dim + 63) / 64 * 64);
  if (H % 8 != 0) {
    err = "flow hidden width must be a multiple of 8";
    return false;
  }
  tc_ok_ = H % 64 == 0 &&
           cudaFuncSetAttribute(fp::flow_program_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                fp::SMEM_BYTES) == cudaSuccess;
  const bool bf = prec_ == Precision::kBF16;
  // every projection but the time projection (fp32 on the device) is held in fp16
  {
    std::vector<std::pair<const HostTensor*, std::string>> planes = {
        {in, "flow.in_proj.weight"}, {cp, "flow.cond_proj.weight"}, {op, "flow.out_proj.weight"}};
    for (std::size_t n = 0; n < layer_t.size(); ++n)
      planes.emplace_back(layer_t[n], "flow.layers." + std::to_string(n) + ".weight");
    for (const auto& [tensor, name] : planes) {
      const auto w = widen_f32(*tensor);
      if (!check_fp16_storable(name, w.data(), w.size(), bf, err)) return false;
    }
  }
  ArenaPlan plan;
  auto plan_mat = [&](int rows, int cols) {
    const int rp = (rows + 127) / 128 * 128;
    const int cp2 = (cols + 63) / 64 * 64;
    plan.add(static_cast<std::size_t>(rp) * cp2 * (bf ? 2 : 4));
    if (!bf && tc_ok_) plan.add(static_cast<std::size_t>(rp) * cp2 * 3 * 2);
    plan.add_n<SimtSlice>(static_cast<std::size_t>((cp2 + 255) / 256));
  };
  plan_mat(H, static_cast<int>(cfg_.action_dim));
  plan_mat(H, static_cast<int>(cfg_.cond_dim));
  plan_mat(static_cast<int>(cfg_.action_dim), H);
  for (std::size_t i = 0; i < cfg_.mlp_layers; ++i) plan_mat(H, H);
  plan.add_n<float>(cfg_.hidden * cfg_.time_dim + cfg_.time_dim);
  if (!wts_.init(plan.total(), err)) return false;
  auto put_mat = [&](const HostTensor* src, Mat& m) {
    m.rows = static_cast<int>(src->shape[0]);
    m.cols = static_cast<int>(src->shape[1]);
    m.rows_pad = (m.rows + 127) / 128 * 128;
    m.cols_pad = (m.cols + 63) / 64 * 64;
    const auto w = widen_f32(*src);  // bf16 files widen exactly (flow.cc:41-58)
    std::vector<float> padded(static_cast<std::size_t>(m.rows_pad) * m.cols_pad, 0.0f);
    for (int r = 0; r < m.rows; ++r)
      std::memcpy(&padded[static_cast<std::size_t>(r) * m.cols_pad], &w[static_cast<std::size_t>(r) * m.cols],
                  static_cast<std::size_t>(m.cols) * 4);
    if (bf) {
      std::vector<std::uint16_t> h(padded.size());
      for (std::size_t i = 0; i < h.size(); ++i) h[i] = fp16_bits_of_bf16_rounded(padded[i]);
      m.w = wts_.take(h.size() * 2);
      cudaMemcpy(m.w, h.data(), h.size() * 2, cudaMemcpyHostToDevice);
    } else {
      m.w = wts_.take(padded.size() * 4);
      cudaMemcpy(m.w, padded.data(), padded.size() * 4, cudaMemcpyHostToDevice);
      if (tc_ok_) {
        const std::size_t cp = static_cast<std::size_t>(m.cols_pad);
        std::vector<std::uint16_t> h3(padded.size() * 3);
        for (int r = 0; r < m.rows_pad; ++r)
          for (std::size_t c = 0; c < cp; ++c) {
            const float v = padded[static_cast<std::size_t>(r) * cp + c];
            const __half hi = __float2half_rn(v);
            std::uint16_t* row = &h3[static_cast<std::size_t>(r) * 3 * cp];
            row[c] = __half_as_ushort(hi);
            row[cp + c] = __half_as_ushort(hi);
            row[2 * cp + c] = __half_as_ushort(__float2half_rn(v - __half2float(hi)));
          }
        m.w3 = wts_.take(h3.size() * 2);
        cudaMemcpy(m.w3, h3.data(), h3.size() * 2, cudaMemcpyHostToDevice);
      }
    }
    std::vector<SimtSlice> sl;
    for (int c = 0; c < m.cols_pad; c += 256) sl.push_back(SimtSlice{0, 0, c, std::min(256, m.cols_pad - c), c});
    m.nslices = static_cast<int>(sl.size());
    m.slices = wts_.take_n<SimtSlice>(sl.size());
    cudaMemcpy(m.slices, sl.data(), sl.size() * sizeof(SimtSlice), cudaMemcpyHostToDevice);
  };
  put_mat(in, in_);
  put_mat(cp, cond_);
  put_mat(op, out_);
  layers_.resize(cfg_.mlp_layers);
  for (std::size_t i = 0; i < cfg_.mlp_layers; ++i) put_mat(layer_t[i], layers_[i]);
  const auto wt = widen_f32(*tp);
  wt_ = wts_.take_n<float>(wt.size());
  cudaMemcpy(wt_, wt.data(), wt.size() * 4, cudaMemcpyHostToDevice);
  // f_j = 10000^(-j / half) in float pow (flow.cc:104)
  const std::size_t half = cfg_.time_dim / 2;
  std::vector<float> f(half);
  for (std::size_t j = 0; j < half; ++j)
    f[j] = std::pow(10000.0f, -static_cast<float>(j) / static_cast<float>(half));
  freqs_ = wts_.take_n<float>(half);
  if (wts_.overflowed()) {
    err = "internal error: flow weight arena too small";
    return false;
  }
  cudaMemcpy(freqs_, f.data(), half * 4, cudaMemcpyHostToDevice);
  if (cudaDeviceSynchronize() != cudaSuccess) {
    err = "flow weight upload failed";
    return false;
  }
  return true;
}

int Flow::reserve(std::size_t batch, std::string& err) noexcept {
  if (batch == 0) batch = 1;
  if (batch <= cap_) return 0;
  for (auto& [k, g] : graphs_) cudaGraphExecDestroy(g);
  graphs_.clear();
  const std::size_t rows = (batch + 255) / 256 * 256;
  const std::size_t H = cfg_.hidden;
  const std::size_t nsl = static_cast<std::size_t>(std::max({in_.nslices, cond_.nslices, out_.nslices,
                                                             layers_.empty() ? 1 : layers_[0].nslices}));
  part_elems_ = nsl * batch * std::max<std::size_t>(H, static_cast<std::size_t>(out_.rows_pad));
  ArenaPlan plan;
  for (int i = 0; i < 6; ++i) plan.add_n<float>(rows * static_cast<std::size_t>(a_pad_));
  plan.add_n<float>(rows * H);           // c_emb
  plan.add_n<float>(H);                  // tp
  plan.add_n<float>(part_elems_);
  plan.add_n<float>(rows * static_cast<std::size_t>(c_pad_));
  plan.add_n<float>(rows * static_cast<std::size_t>(a_pad_));  // xin
  plan.add_n<float>(rows * H);                                 // h0
  plan.add_n<float>(rows * H);                                 // h1
  plan.add_n<float>(rows * static_cast<std::size_t>(c_pad_));  // cin
  plan.add_n<int>(4);
  plan.add_n<unsigned>(4);
  ws_.release();
  if (!ws_.init(plan.total(), err)) {
    cap_ = 0;
    return 2;
  }
  x_ = ws_.take_n<float>(rows * a_pad_);
  probe_ = ws_.take_n<float>(rows * a_pad_);
  for (auto& k : k_) k = ws_.take_n<float>(rows * a_pad_);
  cemb_ = ws_.take_n<float>(rows * H);
  tp_ = ws_.take_n<float>(H);
  part_ = ws_.take_n<float>(part_elems_);
  in_cond_ = ws_.take_n<float>(rows * c_pad_);
  xin_ = ws_.take(rows * a_pad_ * 4);
  h0_ = ws_.take(rows * H * 4);
  h1_ = ws_.take(rows * H * 4);
  cin_ = ws_.take(rows * c_pad_ * 4);
  step_ = ws_.take_n<int>(4);
  fsync_ = ws_.take_n<unsigned>(4);
  if (ws_.overflowed()) {
    err = "internal error: flow workspace arena too small";
    cap_ = 0;
    return 2;
  }
  cudaMemset(x_, 0, ws_.used());
  if (pinned_ != nullptr) cudaFreeHost(pinned_);
  pinned_ = nullptr;
  if (counted_host_malloc(reinterpret_cast<void**>(&pinned_), batch * (cfg_.cond_dim + 2 * cfg_.action_dim) * 4) !=
      cudaSuccess) {
    err = "pinned host allocation failed";
    return 2;
  }
  cap_ = batch;
  cap_rows_ = rows;
  return cudaDeviceSynchronize() == cudaSuccess ? 0 : 2;
}

bool Flow::gemm(const Mat& m, const void* in, int in_ld, std::size_t batch, float* out_f32, void* out_half, int out_ld,
                const float* add_vec, const float* add_tok, int act, bool tc, cudaStream_t st, std::string& err) {
  if (tc) {
    TcLaunch l;
    l.fp16 = true;
    l.M_rows = m.rows_pad;
    l.L = 1;
    l.n_samples = static_cast<int>(batch);
    l.m_valid = m.rows;
    const int kb = m.cols_pad / 64;
    if (split()) {
      l.A = m.w3;
      l.K = 3 * m.cols_pad;
      l.src[0] = TcSource{in, 2 * in_ld, 1, static_cast<int>(cap_rows_)};
      l.segs = {tc::Seg{0, 0, 0, kb, 0}, tc::Seg{0, 0, in_ld, kb, m.cols_pad}, tc::Seg{0, 0, 0, kb, 2 * m.cols_pad}};
      if (out_f32 == nullptr) {
        l.out_lo_off = out_ld;
        out_ld *= 2;
      }
    } else {
      l.A = m.w;
      l.K = m.cols_pad;
      l.src[0] = TcSource{in, in_ld, 1, static_cast<int>(cap_rows_)};
      l.segs = {tc::Seg{0, 0, 0, kb, 0}};
    }
    l.add_vec = add_vec;
    l.add_tok = add_tok;
    l.add_ld = static_cast<int>(cfg_.hidden);
    l.act = act;
    l.out_f32 = out_f32 != nullptr;
    l.out = out_f32 != nullptr ? static_cast<void*>(out_f32) : out_half;
    l.out_ld = out_ld;
    return tc_gemm(l, *ctx_, st, err) == cudaSuccess;
  }
  SimtConvParams p{};
  p.W = m.w;
  p.M = m.rows;
  p.K = m.cols_pad;
  p.src[0] = SimtSource{static_cast<const float*>(in), in_ld, 1};
  p.stride = 1;
  p.L_out = 1;
  p.n_tokens = static_cast<int>(batch);
  p.slices = m.slices;
  p.partial = part_;
  const int nt = p.n_tokens >= 16 ? 16 : (p.n_tokens >= 8 ? 8 : 4);
  const dim3 grid(static_cast<unsigned>(m.nslices), static_cast<unsigned>((m.rows + 127) / 128),
                  static_cast<unsigned>((p.n_tokens + nt - 1) / nt));
  const bool bf = prec_ == Precision::kBF16;
  if (nt == 16) bf ? simt_conv_kernel<16, true><<<grid, 128, 0, st>>>(p) : simt_conv_kernel<16, false><<<grid, 128, 0, st>>>(p);
  else if (nt == 8) bf ? simt_conv_kernel<8, true><<<grid, 128, 0, st>>>(p) : simt_conv_kernel<8, false><<<grid, 128, 0, st>>>(p);
  else bf ? simt_conv_kernel<4, true><<<grid, 128, 0, st>>>(p) : simt_conv_kernel<4, false><<<grid, 128, 0, st>>>(p);
  ReduceParams r{};
  r.partial = part_;
  r.nslices = m.nslices;
  r.n_tokens = static_cast<int>(batch);
  r.M = m.rows;
  r.add_vec = add_vec;
  r.add_tok = add_tok;
  r.act = act;
  r.out = out_f32 != nullptr ? out_f32 : static_cast<float*>(out_half);
  r.out_ld = out_ld;
  reduce_partials_kernel<<<ew_grid(static_cast<long long>(batch) * m.rows, 256, *ctx_), 256, 0, st>>>(r);
  return cudaGetLastError() == cudaSuccess;
}

bool Flow::record_step(std::size_t batch, int method, bool tc, cudaStream_t st, std::string& err) {
  const int H = static_cast<int>(cfg_.hidden);
  const int A = static_cast<int>(cfg_.action_dim);
  const int half = static_cast<int>(cfg_.time_dim / 2);
  const int stages = method == 0 ? 1 : (method == 1 ? 2 : 4);
  for (int s = 0; s < stages; ++s) {
    // later stages follow ode_stage_kernel: a programmatic dependent launch
    // (the first stage follows the step-index copy, a plain dependency)
    const dim3 tgrid((H + kTimeProjRowsPerBlock - 1) / kTimeProjRowsPerBlock), tblock(32 * kTimeProjRowsPerBlock);
    const std::size_t tsmem = static_cast<std::size_t>(2 * half) * 4;
    if (s > 0)
      launch_pdl(time_proj_kernel, tgrid, tblock, tsmem, st, static_cast<const int*>(step_), static_cast<int>(steps_),
                 method, s, static_cast<const float*>(freqs_), half, static_cast<const float*>(wt_), H, tp_);
    else
      time_proj_kernel<<<tgrid, tblock, tsmem, st>>>(step_, static_cast<int>(steps_), method, s, freqs_, half, wt_, H,
                                                     tp_);
    // h = SiLU(W_in x + tp + c_emb)
    void* hin = h0_;
    void* hout = h1_;
    if (!gemm(in_, xin_, a_pad_, batch, tc ? nullptr : static_cast<float*>(hin), tc ? hin : nullptr, H, tp_, cemb_,
              tc::kActSilu, tc, st, err))
      return false;
    for (const Mat& l : layers_) {
      if (!gemm(l, hin, H, batch, tc ? nullptr : static_cast<float*>(hout), tc ? hout : nullptr, H, nullptr, nullptr,
                tc::kActSilu, tc, st, err))
        return false;
      std::swap(hin, hout);
    }
    if (!gemm(out_, hin, H, batch, k_[s], nullptr, a_pad_, nullptr, nullptr, tc::kActNone, tc, st, err)) return false;
    OdeParams p{};
    p.B = static_cast<int>(batch);
    p.A = A;
    p.ld = a_pad_;
    p.method = method;
    p.stage = s;
    p.steps = static_cast<int>(steps_);
    p.step_idx = step_;
    p.step_out = s == stages - 1 ? step_ + 1 : nullptr;
    p.x = x_;
    p.probe = probe_;
    for (int i = 0; i < 4; ++i) p.k[i] = k_[i];
    p.next_in = xin_;
    p.ld_in = a_pad_;
    p.next_mode = in_mode(tc);
    launch_pdl(ode_stage_kernel, dim3(ew_grid(static_cast<long long>(batch) * A, 256, *ctx_)), dim3(256), 0, st, p);
  }
  // step_[0] <- step_[1] (next step index) for the next replay
  cudaMemcpyAsync(step_, step_ + 1, sizeof(int), cudaMemcpyDeviceToDevice, st);
  return cudaGetLastError() == cudaSuccess;
}

bool Flow::prepare(const float* condition, const float* x0, std::size_t batch, bool cond_device, bool x_device,
                   cudaStream_t st, std::string& err) {
  const bool tc = use_tc(batch);
  const int C = static_cast<int>(cfg_.cond_dim), A = static_cast<int>(cfg_.action_dim);
  float* pc = pinned_;
  float* px = pinned_ + batch * cfg_.cond_dim;
  const float* dcond = condition;
  const float* dx = x0;
  float* staging = k_[3];  // dense [B][A] staging for x0 (reused, overwritten by the solve)
  if (!cond_device) {
    std::memcpy(pc, condition, batch * C * 4);
    cudaMemcpyAsync(probe_, pc, batch * C * 4, cudaMemcpyHostToDevice, st);
    dcond = probe_;  // probe_ holds >= rows * a_pad floats; cond fits when C <= a_pad (else use part_)
    if (static_cast<std::size_t>(C) > static_cast<std::size_t>(a_pad_)) {
      cudaMemcpyAsync(part_, pc, batch * C * 4, cudaMemcpyHostToDevice, st);
      dcond = part_;
    }
  }
  if (!x_device) {
    std::memcpy(px, x0, batch * A * 4);
    cudaMemcpyAsync(staging, px, batch * A * 4, cudaMemcpyHostToDevice, st);
    dx = staging;
  }
  // condition -> padded input (fp32 or bf16), then c_emb = W_c cond (flow.cc:256)
  load_rows_kernel<<<ew_grid(static_cast<long long>(batch) * c_pad_, 256, *ctx_), 256, 0, st>>>(
      dcond, static_cast<int>(batch), C, nullptr, 0, tc ? cin_ : static_cast<void*>(in_cond_), c_pad_, in_mode(tc));
  if (!gemm(cond_, tc ? cin_ : static_cast<void*>(in_cond_), c_pad_, batch, cemb_, nullptr,
            static_cast<int>(cfg_.hidden), nullptr, nullptr, tc::kActNone, tc, st, err))
    return false;
  load_rows_kernel<<<ew_grid(static_cast<long long>(batch) * a_pad_, 256, *ctx_), 256, 0, st>>>(
      dx, static_cast<int>(batch), A, x_, a_pad_, xin_, a_pad_, in_mode(tc));
  cudaMemsetAsync(step_, 0, 2 * sizeof(int), st);
  return cudaGetLastError() == cudaSuccess;
}

int Flow::begin(const float* condition, const float* x0, std::size_t batch, std::size_t steps, int method,
                bool condition_on_device, std::string& err) noexcept {
  if (batch == 0 || steps == 0 || method < 0 || method > 2) {
    err = "invalid flow arguments";
    return 1;
  }
  if (batch > cap_ && reserve(batch, err) != 0) return 2;
  cudaSetDevice(ctx_->device);
  batch_ = batch;
  steps_ = steps;
  method_ = method;
  if (!prepare(condition, x0, batch, condition_on_device, false, ctx_->stream, err)) return 2;
  return 0;
}

bool Flow::fused_advance(std::size_t first, std::size_t count, cudaStream_t st, std::string& err, bool& used) {
  used = false;
  const int H = static_cast<int>(cfg_.hidden);
  if (batch_ > static_cast<std::size_t>(kFuseMaxBatch) || use_tc(batch_) ||
      layers_.size() > static_cast<std::size_t>(kFuseMaxLayers) || H % 2 != 0)
    return true;
  const int ldv = std::max(H, a_pad_);
  const std::size_t smem = (static_cast<std::size_t>(batch_) * ldv + cfg_.time_dim) * sizeof(float);
  const bool half = prec_ == Precision::kBF16;
  const void* fn = half ? reinterpret_cast<const void*>(flow_fused_kernel<true>)
                        : reinterpret_cast<const void*>(flow_fused_kernel<false>);
  int per_sm = 0;
  if (smem > 227 * 1024 || cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                static_cast<int>(smem)) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kFlowThreads, smem) != cudaSuccess || per_sm < 1) {
    cudaGetLastError();
    return true;  // not fused: the per-kernel graph runs instead
  }
  FlowFusedParams p{};
  p.B = static_cast<int>(batch_);
  p.A = static_cast<int>(cfg_.action_dim);
  p.H = H;
  p.half = static_cast<int>(cfg_.time_dim / 2);
  p.layers = static_cast<int>(layers_.size());
  p.steps = static_cast<int>(steps_);
  p.method = method_;
  p.first = static_cast<int>(first);
  p.count = static_cast<int>(count);
  p.freqs = freqs_;
  p.wt = wt_;
  p.w_in = in_.w;
  p.ld_in = in_.cols_pad;
  for (std::size_t i = 0; i < layers_.size(); ++i) p.w_l[i] = layers_[i].w;
  p.ld_l = layers_.empty() ? 0 : layers_[0].cols_pad;
  p.w_out = out_.w;
  p.ld_out = out_.cols_pad;
  p.cemb = cemb_;
  p.x = x_;
  p.probe = probe_;
  for (int i = 0; i < 4; ++i) p.k[i] = k_[i];
  p.xin = static_cast<float*>(xin_);
  p.ld_a = a_pad_;
  p.h0 = static_cast<float*>(h0_);
  p.h1 = static_cast<float*>(h1_);
  p.sync = fsync_;
  p.err = ctx_->d_err;
  cudaMemsetAsync(fsync_, 0, 4 * sizeof(unsigned), st);
  cudaLaunchAttribute attr{};
  attr.id = cudaLaunchAttributeCooperative;
  attr.val.cooperative = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(ctx_->sm_count));
  cfg.blockDim = dim3(kFlowThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  const cudaError_t rc = half ? cudaLaunchKernelEx(&cfg, flow_fused_kernel<true>, p)
                              : cudaLaunchKernelEx(&cfg, flow_fused_kernel<false>, p);
  if (rc != cudaSuccess) {
    err = std::string("fused flow launch: ") + cudaGetErrorString(rc);
    return false;
  }
  used = true;
  return true;
}

bool Flow::program_solve(std::size_t first, std::size_t count, cudaStream_t st, std::string& err, bool& used) {
  used = false;
  // bf16 mode only: with the fp32 engines' hi / lo splits every GEMM has three
  // times the K blocks, each tile's operand stream from L2 is the bound, and
  // the per-launch graph (256-token tiles, one wave per GEMM) measured faster
  if (!use_tc(batch_) || split() || count == 0 || first + count > steps_) return true;
  const int H = static_cast<int>(cfg_.hidden);
  const int stages = method_ == 0 ? 1 : (method_ == 1 ? 2 : 4);
  const auto key = std::make_tuple(batch_, first, count, method_, steps_);
  auto it = programs_.find(key);
  if (it == programs_.end()) {
    Program pr;
    pr.n_evals = static_cast<int>(count) * stages;
    pr.tiles_n = static_cast<int>((batch_ + fp::BN - 1) / fp::BN);
    const bool sp = split();
    std::vector<fp::Layer> host;
    int tiles = 0;
    // one GEMM layer reading `in` (row width in_ld, hi / lo halves when split)
    auto add_layer = [&](const Mat& m, const void* in, int in_ld, fp::Layer& L) -> bool {
      L.tiles_m = m.rows_pad / fp::BM;
      L.tiles_n = pr.tiles_n;
      L.tile0 = tiles;
      const int kb = m.cols_pad / fp::BK;
      if (sp) {
        L.nseg = 3;
        const int bcol[3] = {0, in_ld, 0}, acol[3] = {0, m.cols_pad, 2 * m.cols_pad};
        for (int i = 0; i < 3; ++i) {
          L.seg_kb[i] = kb;
          L.seg_bcol[i] = bcol[i];
          L.seg_acol[i] = acol[i];
        }
      } else {
        L.nseg = 1;
        L.seg_kb[0] = kb;
        L.seg_bcol[0] = 0;
        L.seg_acol[0] = 0;
      }
      L.kb_total = L.nseg * kb;
      L.m_valid = m.rows;
      L.n_tokens = static_cast<int>(batch_);
      L.dep = host.empty() ? -1 : static_cast<int>(host.size()) - 1;
      L.dep_target = host.empty() ? 0 : host.back().tiles_m;
      tiles += L.tiles_m * L.tiles_n;
      const std::uint64_t a_cols = static_cast<std::uint64_t>(sp ? 3 * m.cols_pad : m.cols_pad);
      const std::uint64_t b_cols = static_cast<std::uint64_t>(sp ? 2 * in_ld : in_ld);
      return encode_tmap_2d(&L.a, sp ? m.w3 : m.w, a_cols, static_cast<std::uint64_t>(m.rows_pad), fp::BK, fp::BM,
                            true, err) &&
             encode_tmap_2d(&L.b, in, b_cols, static_cast<std::uint64_t>(cap_rows_), fp::BK, fp::BN, true, err);
    };
    const int hld = sp ? 2 * H : H;
    for (int e = 0; e < pr.n_evals; ++e) {
      void* hin = h0_;
      void* hout = h1_;
      fp::Layer L{};
      if (!add_layer(in_, xin_, a_pad_, L)) return false;
      L.act = tc::kActSilu;
      L.add_tok = cemb_;
      L.add_ld = H;
      L.out = static_cast<__half*>(hin);
      L.out_ld = hld;
      L.out_lo = sp ? H : 0;
      host.push_back(L);
      L.add_vec = nullptr;  // set once the time-projection buffer exists
      for (const Mat& m : layers_) {
        fp::Layer Lh{};
        if (!add_layer(m, hin, H, Lh)) return false;
        Lh.act = tc::kActSilu;
        Lh.out = static_cast<__half*>(hout);
        Lh.out_ld = hld;
        Lh.out_lo = sp ? H : 0;
        host.push_back(Lh);
        std::swap(hin, hout);
      }
      fp::Layer Lo{};
      if (!add_layer(out_, hin, H, Lo)) return false;
      Lo.ode = 1;
      Lo.method = method_;
      Lo.stage = e % stages;
      Lo.steps = static_cast<int>(steps_);
      Lo.x = x_;
      Lo.probe = probe_;
      for (int i = 0; i < 4; ++i) Lo.k[i] = k_[i];
      Lo.ld = a_pad_;
      Lo.next_in = static_cast<__half*>(xin_);
      Lo.ld_in = a_pad_;
      Lo.next_mode = in_mode(true);
      host.push_back(Lo);
    }
    pr.n_layers = static_cast<int>(host.size());
    pr.total_tiles = tiles;
    for (const fp::Layer& L : host) pr.tiles_m.push_back(L.tiles_m);
    if (std::getenv("FLOWEDGE_FLOW_TRACE") != nullptr &&
        counted_malloc(reinterpret_cast<void**>(&pr.trace),
                       static_cast<std::size_t>(tiles) * fp::kTraceStamps * sizeof(unsigned long long)) != cudaSuccess)
      pr.trace = nullptr;
    if (counted_malloc(reinterpret_cast<void**>(&pr.table), host.size() * sizeof(fp::Layer)) != cudaSuccess ||
        counted_malloc(reinterpret_cast<void**>(&pr.ctr), host.size() * pr.tiles_n * sizeof(int)) != cudaSuccess ||
        counted_malloc(reinterpret_cast<void**>(&pr.tp), static_cast<std::size_t>(pr.n_evals) * H * sizeof(float)) !=
            cudaSuccess) {
      cudaFree(pr.table);
      cudaFree(pr.ctr);
      err = "device allocation failed (flow program)";
      return false;
    }
    const std::size_t per_eval = layers_.size() + 2;
    for (int e = 0; e < pr.n_evals; ++e) host[static_cast<std::size_t>(e) * per_eval].add_vec = pr.tp + static_cast<std::size_t>(e) * H;
    if (cudaMemcpy(pr.table, host.data(), host.size() * sizeof(fp::Layer), cudaMemcpyHostToDevice) != cudaSuccess) {
      err = "flow program upload failed";
      return false;
    }
    it = programs_.emplace(key, pr).first;
  }
  const Program& pr = it->second;
  const int half = static_cast<int>(cfg_.time_dim / 2);
  time_proj_all_kernel<<<dim3((H + kTimeProjRowsPerBlock - 1) / kTimeProjRowsPerBlock, pr.n_evals),
                         32 * kTimeProjRowsPerBlock, static_cast<std::size_t>(2 * half) * 4, st>>>(
      static_cast<int>(first), static_cast<int>(steps_), method_, stages, freqs_, half, wt_, H, pr.tp);
  cudaMemsetAsync(pr.ctr, 0, static_cast<std::size_t>(pr.n_layers) * pr.tiles_n * sizeof(int), st);
  const int grid = std::min(pr.total_tiles, ctx_->sm_count);
  if (pr.trace != nullptr)
    cudaMemsetAsync(pr.trace, 0, static_cast<std::size_t>(pr.total_tiles) * fp::kTraceStamps * 8, st);
  fp::flow_program_kernel<<<grid, fp::THREADS, fp::SMEM_BYTES, st>>>(pr.table, pr.n_layers, pr.total_tiles, pr.ctr,
                                                                      pr.tiles_n, ctx_->d_err, pr.trace);
  if (cudaGetLastError() != cudaSuccess) {
    err = "flow program launch failed";
    return false;
  }
  if (pr.trace != nullptr) {
    // profiling only: wait for the call and write "tile layer m n" and the
    // five stamps (ns from the first producer start) per line
    std::vector<unsigned long long> h(static_cast<std::size_t>(pr.total_tiles) * fp::kTraceStamps);
    cudaStreamSynchronize(st);
    cudaMemcpy(h.data(), pr.trace, h.size() * 8, cudaMemcpyDeviceToHost);
    unsigned long long t0 = ~0ull;
    for (std::size_t i = 0; i < h.size(); i += fp::kTraceStamps)
      if (h[i] != 0) t0 = std::min(t0, h[i]);
    if (FILE* f = std::fopen(std::getenv("FLOWEDGE_FLOW_TRACE"), "w")) {
      std::fprintf(f, "tile layer m n start dep_met mma_issued epi_start published\n");
      int layer = 0, base = 0;
      for (int t = 0; t < pr.total_tiles; ++t) {
        while (layer + 1 < pr.n_layers && t >= base + pr.tiles_m[static_cast<std::size_t>(layer)] * pr.tiles_n) {
          base += pr.tiles_m[static_cast<std::size_t>(layer)] * pr.tiles_n;
          ++layer;
        }
        const int tm = pr.tiles_m[static_cast<std::size_t>(layer)];
        std::fprintf(f, "%d %d %d %d", t, layer, (t - base) % tm, (t - base) / tm);
        for (int k = 0; k < fp::kTraceStamps; ++k) {
          const unsigned long long v = h[static_cast<std::size_t>(t) * fp::kTraceStamps + k];
          std::fprintf(f, " %lld", v == 0 ? -1LL : static_cast<long long>(v - t0));
        }
        std::fprintf(f, "\n");
      }
      std::fclose(f);
    }
  }
  used = true;
  return true;
}

int Flow::advance(std::size_t first, std::size_t count, float* out, std::string& err) noexcept {
  cudaSetDevice(ctx_->device);
  cudaStream_t st = ctx_->stream;
  const bool tc = use_tc(batch_);
  bool fused = false;
  if (count > 0 && !fused_advance(first, count, st, err, fused)) return 2;
  if (count > 0 && !fused && !program_solve(first, count, st, err, fused)) return 2;
  if (count > 0 && !fused) {
    const auto key = std::make_tuple(batch_, method_, tc, steps_);
    auto it = graphs_.find(key);
    if (it == graphs_.end()) {
      cudaStream_t cap = nullptr;
      cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking);
      cudaStreamSynchronize(st);
      cudaGraph_t graph = nullptr;
      cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal);
      const bool ok = record_step(batch_, method_, tc, cap, err);
      const cudaError_t end = cudaStreamEndCapture(cap, &graph);
      cudaStreamDestroy(cap);
      if (!ok || end != cudaSuccess) {
        if (graph != nullptr) cudaGraphDestroy(graph);
        if (err.empty()) err = "flow graph capture failed";
        cudaGetLastError();
        return 2;
      }
      cudaGraphExec_t exec = nullptr;
      const cudaError_t inst = cudaGraphInstantiate(&exec, graph, 0);
      cudaGraphDestroy(graph);
      if (inst != cudaSuccess) {
        err = "flow graph instantiation failed";
        return 2;
      }
      it = graphs_.emplace(key, exec).first;
    }
    const int first_i = static_cast<int>(first);
    cudaMemcpyAsync(step_, &first_i, sizeof(int), cudaMemcpyHostToDevice, st);
    for (std::size_t i = 0; i < count; ++i)
      if (cudaGraphLaunch(it->second, st) != cudaSuccess) {
        err = "flow graph launch failed";
        return 2;
      }
  }
  if (out != nullptr) {
    const int A = static_cast<int>(cfg_.action_dim);
    float* stage = k_[3];
    store_rows_kernel<<<ew_grid(static_cast<long long>(batch_) * A, 256, *ctx_), 256, 0, st>>>(
        x_, static_cast<int>(batch_), A, a_pad_, stage);
    float* px = pinned_ + batch_ * cfg_.cond_dim;
    cudaMemcpyAsync(px, stage, batch_ * A * 4, cudaMemcpyDeviceToHost, st);
    if (cudaStreamSynchronize(st) != cudaSuccess) {
      err = std::string("flow solve failed: ") + cudaGetErrorString(cudaGetLastError());
      return 2;
    }
    if (take_device_error(*ctx_, st) != 0) {
      err = "a device pipeline wait timed out";
      return 2;
    }
    std::memcpy(out, px, batch_ * A * 4);
  }
  return 0;
}

int Flow::sample_device(const float* condition, const float* x0, std::size_t batch, std::size_t steps, int method,
                        float* out, void* stream, std::string& err) noexcept {
  if (batch == 0 || steps == 0 || method < 0 || method > 2) {
    err = "invalid flow arguments";
    return 1;
  }
  if (batch > cap_) {
    err = "batch exceeds the reserved capacity (call fe_engine_reserve_batch first)";
    return 2;
  }
  cudaSetDevice(ctx_->device);
  cudaStream_t st = stream != nullptr ? static_cast<cudaStream_t>(stream) : ctx_->stream;
  batch_ = batch;
  steps_ = steps;
  method_ = method;
  if (!prepare(condition, x0, batch, true, true, st, err)) return 2;
  const bool tc = use_tc(batch);
  bool programmed = false;
  if (!program_solve(0, steps, st, err, programmed)) return 2;
  if (programmed) {
    store_rows_kernel<<<ew_grid(static_cast<long long>(batch) * cfg_.action_dim, 256, *ctx_), 256, 0, st>>>(
        x_, static_cast<int>(batch), static_cast<int>(cfg_.action_dim), a_pad_, out);
    return cudaGetLastError() == cudaSuccess ? 0 : 2;
  }
  const auto key = std::make_tuple(batch, method, tc, steps);
  auto it = graphs_.find(key);
  if (it == graphs_.end()) {
    // record on the caller's stream ordering: capture on a private stream
    cudaStream_t cap = nullptr;
    cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking);
    cudaStreamSynchronize(st);
    cudaGraph_t graph = nullptr;
    cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal);
    const bool ok = record_step(batch, method, tc, cap, err);
    cudaStreamEndCapture(cap, &graph);
    cudaStreamDestroy(cap);
    if (!ok || graph == nullptr) {
      if (graph != nullptr) cudaGraphDestroy(graph);
      return 2;
    }
    cudaGraphExec_t exec = nullptr;
    cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    it = graphs_.emplace(key, exec).first;
  }
  for (std::size_t i = 0; i < steps; ++i) cudaGraphLaunch(it->second, st);
  store_rows_kernel<<<ew_grid(static_cast<long long>(batch) * cfg_.action_dim, 256, *ctx_), 256, 0, st>>>(
      x_, static_cast<int>(batch), static_cast<int>(cfg_.action_dim), a_pad_, out);
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

// ---------------------------------------------------------------------------
// Allocation-free flow solve (fe_engine_sample_condition_static).
//
// Some callers cannot call cudaMalloc when they sample: a fixed-period
// control loop, where cudaMalloc may block and synchronise the device and so
// miss the period, or a host process whose device memory another runtime's
// pool allocator claimed at start-up.  The resident-engine
// entry points grow the engine's workspace with cudaMalloc when a batch
// exceeds the reserved capacity; this variant never allocates: its scratch
// (solver state, stage slopes, hidden activations, split-K partial sums) is
// the file-scope array below, which every GPU that loads this library holds
// for the life of the process.
//
// * Limit: kStaticScratchBytes (4 MiB); a request whose scratch would not fit
//   is rejected with FE_STATUS_RESOURCE_EXHAUSTED and a message naming it.
// * The first call on a device looks up the array's device address with
//   cudaGetSymbolAddress while that device is current; make that first call
//   before capturing any stream.
// * Every call shares the array and it keeps the last call's contents: the
//   padded columns are rewritten by every call, the step counter is cleared
//   by every call.  Calls that overlap on the GPU (different streams, or
//   engines on the same device used concurrently) race on the array.
// * It always runs the weight-streaming CUDA-core kernels (the same kernels,
//   in the same order, as the engine's small-batch path).
constexpr std::size_t kStaticScratchBytes = std::size_t(4) << 20;
static __device__ __align__(256) unsigned char g_flow_static_scratch[kStaticScratchBytes];

void* static_scratch_address(int device, std::string& err) {
  static std::mutex mu;
  static void* addr[64] = {};
  if (device < 0 || device >= 64) {
    err = "device index out of range for the static scratch table";
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (addr[device] == nullptr) {
    void* p = nullptr;
    const cudaError_t rc = cudaGetSymbolAddress(&p, g_flow_static_scratch);
    if (rc != cudaSuccess || p == nullptr) {
      err = std::string("cudaGetSymbolAddress(static scratch) failed: ") + cudaGetErrorString(rc);
      return nullptr;
    }
    addr[device] = p;
  }
  return addr[device];
}

int Flow::sample_static(const float* condition, const float* x0, std::size_t batch, std::size_t steps, int method,
                        float* out, void* stream, std::string& err) noexcept {
  if (batch == 0 || steps == 0 || method < 0 || method > 2 || condition == nullptr || x0 == nullptr ||
      out == nullptr) {
    err = "invalid flow arguments";
    return 1;
  }
  const int H = static_cast<int>(cfg_.hidden), A = static_cast<int>(cfg_.action_dim);
  const int C = static_cast<int>(cfg_.cond_dim), half = static_cast<int>(cfg_.time_dim / 2);
  // every row needs at least one full-width fp32 row of scratch: reject batches
  // that cannot fit before any size arithmetic (which then cannot wrap)
  const std::size_t widest = std::max({static_cast<std::size_t>(a_pad_), static_cast<std::size_t>(H),
                                       static_cast<std::size_t>(c_pad_)});
  if (batch > kStaticScratchBytes / (4 * widest)) {
    err = "batch of " + std::to_string(batch) + " rows cannot fit the " + std::to_string(kStaticScratchBytes) +
          "-byte static array (use fewer rows)";
    return 2;
  }
  const std::size_t rows = batch;
  const std::size_t nsl = static_cast<std::size_t>(std::max({in_.nslices, cond_.nslices, out_.nslices,
                                                             layers_.empty() ? 1 : layers_[0].nslices}));
  // carve the static array (256-byte aligned pieces) and check it fits
  std::size_t need = 0;
  auto piece = [&](std::size_t floats) {
    const std::size_t off = need;
    need += (floats * 4 + 255) & ~std::size_t(255);
    return off;
  };
  const std::size_t o_x = piece(rows * a_pad_), o_probe = piece(rows * a_pad_);
  std::size_t o_k[4];
  for (auto& o : o_k) o = piece(rows * a_pad_);
  const std::size_t o_cemb = piece(rows * H), o_tp = piece(H);
  const std::size_t o_part = piece(nsl * rows * std::max<std::size_t>(H, static_cast<std::size_t>(out_.rows_pad)));
  const std::size_t o_cin = piece(rows * c_pad_), o_xin = piece(rows * a_pad_);
  const std::size_t o_h0 = piece(rows * H), o_h1 = piece(rows * H), o_step = piece(4);
  if (need > kStaticScratchBytes) {
    err = "request needs " + std::to_string(need) + " bytes of scratch, above the " +
          std::to_string(kStaticScratchBytes) + "-byte static array (use fewer rows)";
    return 2;
  }
  // the caller's current device is restored on every return; errors left
  // pending on this thread by earlier calls are cleared so that the status
  // below reports this call's launches only
  int caller_device = -1;
  cudaGetDevice(&caller_device);
  struct RestoreDevice {
    int device;
    ~RestoreDevice() {
      if (device >= 0) cudaSetDevice(device);
    }
  } restore{caller_device};
  cudaSetDevice(ctx_->device);
  cudaGetLastError();
  auto* base = static_cast<unsigned char*>(static_scratch_address(ctx_->device, err));
  if (base == nullptr) {
    cudaGetLastError();
    return 2;
  }
  auto F = [&](std::size_t off) { return reinterpret_cast<float*>(base + off); };
  float *x = F(o_x), *probe = F(o_probe), *cemb = F(o_cemb), *tp = F(o_tp), *part = F(o_part);
  float *cin = F(o_cin), *xin = F(o_xin), *h0 = F(o_h0), *h1 = F(o_h1);
  float* k[4] = {F(o_k[0]), F(o_k[1]), F(o_k[2]), F(o_k[3])};
  int* step = reinterpret_cast<int*>(base + o_step);
  cudaStream_t st = stream != nullptr ? static_cast<cudaStream_t>(stream) : ctx_->stream;
  const bool bf = prec_ == Precision::kBF16;
  auto linear = [&](const Mat& m, const float* in, int in_ld, float* dst, int dst_ld, const float* add_vec,
                    const float* add_tok, int act) {
    SimtConvParams p{};
    p.W = m.w;
    p.M = m.rows;
    p.K = m.cols_pad;
    p.src[0] = SimtSource{in, in_ld, 1};
    p.stride = 1;
    p.L_out = 1;
    p.n_tokens = static_cast<int>(rows);
    p.slices = m.slices;
    p.partial = part;
    const int nt = p.n_tokens >= 16 ? 16 : (p.n_tokens >= 8 ? 8 : 4);
    const dim3 grid(static_cast<unsigned>(m.nslices), static_cast<unsigned>((m.rows + 127) / 128),
                    static_cast<unsigned>((p.n_tokens + nt - 1) / nt));
    if (nt == 16) bf ? simt_conv_kernel<16, true><<<grid, 128, 0, st>>>(p) : simt_conv_kernel<16, false><<<grid, 128, 0, st>>>(p);
    else if (nt == 8) bf ? simt_conv_kernel<8, true><<<grid, 128, 0, st>>>(p) : simt_conv_kernel<8, false><<<grid, 128, 0, st>>>(p);
    else bf ? simt_conv_kernel<4, true><<<grid, 128, 0, st>>>(p) : simt_conv_kernel<4, false><<<grid, 128, 0, st>>>(p);
    ReduceParams r{};
    r.partial = part;
    r.nslices = m.nslices;
    r.n_tokens = static_cast<int>(rows);
    r.M = m.rows;
    r.add_vec = add_vec;
    r.add_tok = add_tok;
    r.act = act;
    r.out = dst;
    r.out_ld = dst_ld;
    reduce_partials_kernel<<<ew_grid(static_cast<long long>(rows) * m.rows, 256, *ctx_), 256, 0, st>>>(r);
  };
  // c_emb = W_c cond; x = x0 (padded copies rewrite every padding column)
  load_rows_kernel<<<ew_grid(static_cast<long long>(rows) * c_pad_, 256, *ctx_), 256, 0, st>>>(
      condition, static_cast<int>(rows), C, nullptr, 0, cin, c_pad_, 0);
  linear(cond_, cin, c_pad_, cemb, H, nullptr, nullptr, tc::kActNone);
  load_rows_kernel<<<ew_grid(static_cast<long long>(rows) * a_pad_, 256, *ctx_), 256, 0, st>>>(
      x0, static_cast<int>(rows), A, x, a_pad_, xin, a_pad_, 0);
  if (const cudaError_t rc = cudaMemsetAsync(step, 0, 2 * sizeof(int), st); rc != cudaSuccess) {
    err = std::string("clearing the static step counter failed: ") + cudaGetErrorString(rc);
    cudaGetLastError();
    return 2;
  }
  const int stages = method == 0 ? 1 : (method == 1 ? 2 : 4);
  for (std::size_t i = 0; i < steps; ++i) {
    for (int s = 0; s < stages; ++s) {
      time_proj_kernel<<<(H + kTimeProjRowsPerBlock - 1) / kTimeProjRowsPerBlock, 32 * kTimeProjRowsPerBlock, static_cast<std::size_t>(2 * half) * 4, st>>>(
          step, static_cast<int>(steps), method, s, freqs_, half, wt_, H, tp);
      float* hin = h0;
      float* hout = h1;
      linear(in_, xin, a_pad_, hin, H, tp, cemb, tc::kActSilu);
      for (const Mat& l : layers_) {
        linear(l, hin, H, hout, H, nullptr, nullptr, tc::kActSilu);
        std::swap(hin, hout);
      }
      linear(out_, hin, H, k[s], a_pad_, nullptr, nullptr, tc::kActNone);
      OdeParams p{};
      p.B = static_cast<int>(rows);
      p.A = A;
      p.ld = a_pad_;
      p.method = method;
      p.stage = s;
      p.steps = static_cast<int>(steps);
      p.step_idx = step;
      p.step_out = s == stages - 1 ? step + 1 : nullptr;
      p.x = x;
      p.probe = probe;
      for (int j = 0; j < 4; ++j) p.k[j] = k[j];
      p.next_in = xin;
      p.ld_in = a_pad_;
      p.next_mode = 0;
      ode_stage_kernel<<<ew_grid(static_cast<long long>(rows) * A, 256, *ctx_), 256, 0, st>>>(p);
    }
    if (const cudaError_t rc = cudaMemcpyAsync(step, step + 1, sizeof(int), cudaMemcpyDeviceToDevice, st);
        rc != cudaSuccess) {
      err = std::string("advancing the static step counter failed: ") + cudaGetErrorString(rc);
      cudaGetLastError();
      return 2;
    }
  }
  store_rows_kernel<<<ew_grid(static_cast<long long>(rows) * A, 256, *ctx_), 256, 0, st>>>(
      x, static_cast<int>(rows), A, a_pad_, out);
  const cudaError_t rc = cudaGetLastError();
  if (rc != cudaSuccess) {
    err = std::string("static flow solve launch failed: ") + cudaGetErrorString(rc);
    return 2;
  }
  return 0;
}

}  // namespace

std::unique_ptr<FlowDevice> make_flow_device(const TensorTable& tensors, std::shared_ptr<DeviceContext> ctx,
                                             Precision precision, std::string& err) {
  cudaSetDevice(ctx->device);
  auto f = std::make_unique<Flow>(std::move(ctx), precision);
  if (!f->load(tensors, err)) return nullptr;
  if (f->reserve(1, err) != 0) return nullptr;
  return f;
}

}  // namespace feb
