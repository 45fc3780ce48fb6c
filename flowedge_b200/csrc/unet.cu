// Device-resident Diffusion Policy ConditionalUnet1D with the DDIM / DDPM
// sampler (reference: src/core/heads/diffusion/diffusion.cc:383-1035).
//
// Two execution paths share one weight layout (tap-major packed GEMM rows,
// [out][tap][in], input channels padded to 64):
//   * tensor path (bf16 weights, batch * horizon >= kTcMinTokens): every conv
//     is one tcgen05 implicit GEMM whose epilogue adds the bias and gathers
//     GroupNorm statistics; GroupNorm + Mish + FiLM / residual is one bf16
//     elementwise pass; the output 1x1 conv is fused with the DDIM / DDPM
//     update.
//   * weight-streaming path (fp32 or bf16 weights, small batch): split-K
//     CUDA-core convolution whose partial sums are reduced inside the
//     GroupNorm kernel (fixed order, deterministic).
// FiLM is split as W_t * mish(temb(t)) + W_c * mish(cond) + b: the time part
// is tabulated for every training timestep at load, the condition part is
// computed once per sample call.  The whole sampling loop of one call is
// captured as one CUDA graph per (batch, steps, scheduler).
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <map>
#include <numbers>
#include <tuple>

#include "runtime.cuh"
#include "simt.cuh"
#include "stream.cuh"

namespace feb {
namespace {

constexpr int kSliceCh = 256;
constexpr long long kTcMinTokens = 512;
// The weight-streaming path runs the batch in chunks of at most this many
// tokens (its split-K partial buffers scale with the chunk, not the batch).
constexpr std::size_t kSimtChunkTokens = 1024;
constexpr std::size_t kFinalNormGroups = 8;


struct Part {
  int channels;  // actual input channels of this concatenated part
  int padded;    // channels in the activation tensor (multiple of 64)
};

enum class ConvKind { kSame, kDown, kUp0, kUp1, kPoint };

struct ConvDev {
  ConvKind kind{};
  int oc = 0, oc_rows = 0, K = 0, ic_total = 0, taps = 0;
  void* w = nullptr;  // [oc_rows][K] (weight dtype)
  float* bias = nullptr;
  SimtSlice* slices = nullptr;
  int nslices = 0;
  std::vector<tc::Seg> segs;
  int stride = 1;
  std::vector<int> tap_off;  // input time offset of each tap
  // small-batch program: rows in mma.sync fragment order (see stream_pack)
  void* sw = nullptr;
  int s_rbs = 0, s_ks = 0;
  // host staging before upload
  std::vector<float> host_w;
  std::vector<float> host_b;
  std::vector<SimtSlice> host_slices;
};

struct BlockDev {
  ConvDev c1, c2, res;
  bool has_res = false;
  float *g1 = nullptr, *b1 = nullptr, *g2 = nullptr, *b2 = nullptr;
  std::vector<float> hg1, hb1, hg2, hb2;
  int oc = 0;
  int film_off = 0;
};

// tap list: (kernel index into the stored weight, time offset)
std::vector<std::pair<int, int>> taps_for(ConvKind kind, int k) {
  std::vector<std::pair<int, int>> taps;
  switch (kind) {
    case ConvKind::kSame:
      for (int j = 0; j < k; ++j) taps.emplace_back(j, j - k / 2);
      break;
    case ConvKind::kDown:  // k3 s2 p1: input t = 2*t_out + j - 1
      for (int j = 0; j < 3; ++j) taps.emplace_back(j, j - 1);
      break;
    case ConvKind::kUp0:  // convT k4 s2 p1, even outputs 2s: x[s] * W1 + x[s-1] * W3
      taps = {{1, 0}, {3, -1}};
      break;
    case ConvKind::kUp1:  // odd outputs 2s+1: x[s+1] * W0 + x[s] * W2
      taps = {{0, 1}, {2, 0}};
      break;
    case ConvKind::kPoint:
      taps = {{0, 0}};
      break;
  }
  return taps;
}

// Pack one convolution.  `w` is [oc][ic][k] (conv) or [ic][oc][4] (convT).
void pack_conv(ConvDev& c, ConvKind kind, const std::vector<float>& w, const std::vector<float>& b, int oc,
               const std::vector<Part>& parts, int k) {
  c.kind = kind;
  c.oc = oc;
  c.oc_rows = (oc + 127) / 128 * 128;
  int ic_actual = 0, ic_pad = 0;
  for (const Part& p : parts) {
    ic_actual += p.channels;
    ic_pad += p.padded;
  }
  c.ic_total = ic_pad;
  const auto taps = taps_for(kind, k);
  c.taps = static_cast<int>(taps.size());
  c.K = c.taps * ic_pad;
  c.host_w.assign(static_cast<std::size_t>(c.oc_rows) * c.K, 0.0f);
  const bool transposed = kind == ConvKind::kUp0 || kind == ConvKind::kUp1;
  for (int o = 0; o < oc; ++o)
    for (int j = 0; j < c.taps; ++j) {
      const int kk = taps[static_cast<std::size_t>(j)].first;
      int src_ic = 0, dst = 0;
      for (const Part& p : parts) {
        for (int i = 0; i < p.channels; ++i) {
          const int ic = src_ic + i;
          const float v = transposed ? w[(static_cast<std::size_t>(ic) * oc + o) * 4 + kk]
                                     : w[(static_cast<std::size_t>(o) * ic_actual + ic) * k + kk];
          c.host_w[static_cast<std::size_t>(o) * c.K + static_cast<std::size_t>(j) * ic_pad + dst + i] = v;
        }
        src_ic += p.channels;
        dst += p.padded;
      }
    }
  c.host_b = b;
  c.stride = kind == ConvKind::kDown ? 2 : 1;
  c.tap_off.clear();
  for (const auto& tp : taps) c.tap_off.push_back(tp.second);
  // weight-streaming slices and tensor-core segments
  for (int j = 0; j < c.taps; ++j) {
    const int t_off = taps[static_cast<std::size_t>(j)].second;
    int off = 0;
    for (int q = 0; q < static_cast<int>(parts.size()); ++q) {
      const int pc = parts[static_cast<std::size_t>(q)].padded;
      for (int ch = 0; ch < pc; ch += kSliceCh)
        c.host_slices.push_back(SimtSlice{q, t_off, ch, std::min(kSliceCh, pc - ch), j * ic_pad + off + ch});
      if (kind == ConvKind::kDown) {
        // [B][L/2][2C] pair view: x[2s + d] = view[s][d * C + c]
        const int pair_t = j == 0 ? -1 : 0;
        const int ch_off = j == 1 ? 0 : pc;
        c.segs.push_back(tc::Seg{0, pair_t, ch_off, pc / 64, j * ic_pad + off});
      } else {
        c.segs.push_back(tc::Seg{q, t_off, 0, pc / 64, j * ic_pad + off});
      }
      off += pc;
    }
  }
  c.nslices = static_cast<int>(c.host_slices.size());
}

// Rows of a [rows][K] weight matrix in the order the small-batch program's
// mma.sync m16n8k16 A fragments are loaded: for row block rb and K step k,
// plane p, lane l = 4g + t holds the 32-bit pairs
//   {W[16rb+g][16k+2t..+1], W[16rb+g+8][16k+2t..+1], W[16rb+g][16k+2t+8..+9], W[16rb+g+8][16k+2t+8..+9]}
// (lower column in the low half).  bf16 weights: one plane, the bf16-rounded
// value as fp16.  fp32 weights: planes hi = fp16(w) and lo = fp16(w - hi).
int stream_planes(bool bf16) { return bf16 ? 1 : 2; }

std::size_t stream_bytes(int rows, int K, bool bf16) {
  return static_cast<std::size_t>((rows + 15) / 16) * static_cast<std::size_t>(K / 16) *
         static_cast<std::size_t>(stream_planes(bf16)) * 512;
}

void stream_pack(const float* w, int rows, int K, bool bf16, std::vector<std::uint32_t>& out) {
  const int rbs = (rows + 15) / 16, ks = K / 16, planes = stream_planes(bf16);
  out.assign(static_cast<std::size_t>(rbs) * ks * planes * 128, 0u);
  auto bits = [&](int r, int k, int plane) -> std::uint32_t {
    if (r >= rows) return 0u;
    const float v = w[static_cast<std::size_t>(r) * K + k];
    if (bf16) return fp16_bits_of_bf16_rounded(v);
    const __half hi = __float2half_rn(v);
    return plane == 0 ? __half_as_ushort(hi) : __half_as_ushort(__float2half_rn(v - __half2float(hi)));
  };
  auto pair = [&](int r, int k, int plane) { return bits(r, k, plane) | (bits(r, k + 1, plane) << 16); };
  std::size_t i = 0;
  for (int rb = 0; rb < rbs; ++rb)
    for (int k = 0; k < ks; ++k)
      for (int pl = 0; pl < planes; ++pl)
        for (int lane = 0; lane < 32; ++lane) {
          const int r0 = rb * 16 + (lane >> 2), c0 = k * 16 + 2 * (lane & 3);
          out[i++] = pair(r0, c0, pl);
          out[i++] = pair(r0 + 8, c0, pl);
          out[i++] = pair(r0, c0 + 8, pl);
          out[i++] = pair(r0 + 8, c0 + 8, pl);
        }
}

struct Act {
  void* p = nullptr;
  int C = 0;
  int L = 0;
};

struct StepPlan {
  int timestep;
  int previous;
  StepScalars scalars;
};

class Unet final : public UnetDevice {
 public:
  Unet(std::shared_ptr<DeviceContext> ctx, Precision prec) : ctx_(std::move(ctx)), prec_(prec) {}
  ~Unet() override {
    write_trace();
    if (trace_ != nullptr) cudaFree(trace_);
    for (auto& [key, g] : graphs_) {
      cudaGraphExecDestroy(g.exec);
      if (g.tables != nullptr) cudaFree(g.tables);
    }
    drop_streams();
    if (pinned_ != nullptr) cudaFreeHost(pinned_);
  }

  bool load(const TensorTable& t, std::string& err);

  const DiffusionConfig& config() const noexcept override { return cfg_; }
  Precision precision() const noexcept override { return prec_; }
  std::size_t capacity() const noexcept override { return cap_; }
  std::uint64_t kernel_launches() const noexcept override { return launches_; }
  int reserve(std::size_t batch, std::string& err) noexcept override;
  int denoise(const float* condition, const float* sample, float timestep, float* eps, std::size_t batch,
              std::string& err) noexcept override;
  int sample(const float* condition, const float* noise, std::size_t batch, std::size_t steps, int scheduler,
             std::uint64_t seed, float* action, std::string& err) noexcept override;
  int sample_device(const float* condition, const float* noise, std::size_t batch, std::size_t steps,
                    int scheduler, std::uint64_t seed, float* action, void* stream,
                    std::string& err) noexcept override;

 private:
  bool use_tc(std::size_t batch) const {
    return prec_ == Precision::kBF16 && tc_ok_ &&
           static_cast<long long>(batch) * static_cast<long long>(cfg_.horizon) >= kTcMinTokens;
  }
  bool bf16_weights() const { return prec_ == Precision::kBF16; }
  void upload_conv(ConvDev& c);
  bool build_plan(std::string& err);
  std::vector<StepPlan> plan_steps(std::size_t steps, int scheduler) const;
  bool record_sample(std::size_t batch, const std::vector<StepPlan>& plan, cudaStream_t st, std::string& err);
  bool record_forward(std::size_t batch, bool tc, const float* film_time_row, cudaStream_t st, std::string& err);
  bool record_film_cond(std::size_t batch, bool tc, cudaStream_t st, std::string& err);
  bool simt_conv(const ConvDev& c, const std::vector<Act>& srcs, int L_out, std::size_t batch, float* partial,
                 cudaStream_t st, std::string& err);
  void simt_reduce(const ConvDev& c, const float* partial, std::size_t batch, int L_tok, Act out, int rps, int tmul,
                   int tadd, cudaStream_t st);
  void simt_gn(const ConvDev& c, const float* partial, std::size_t batch, int L, const float* gamma,
               const float* beta, int groups, const BlockDev* film_block, const float* film_time_row,
               const float* res_tensor, const ConvDev* res_conv, const float* res_partial, Act out, cudaStream_t st);
  // GroupNorm + Mish (+ FiLM / residual) fused into a conv's epilogue
  struct Fuse {
    const float* gamma = nullptr;
    const float* beta = nullptr;
    const BlockDev* film_block = nullptr;
    const float* film_time_row = nullptr;
    const float* res_f32 = nullptr;
    const void* res16 = nullptr;
    float* out_twin = nullptr;
    int groups = 0;
  };
  bool tc_conv(const ConvDev& c, const std::vector<Act>& srcs, int L_out, std::size_t batch, void* out,
               long long out_ld, int rps, int tmul, int tadd, bool stats, int groups, bool out_f32, cudaStream_t st,
               std::string& err, const Fuse* fuse = nullptr);
  // GroupNorm fits the conv epilogue: samples of at least 8 tokens, and
  // groups of 32..128 channels inside one 128-row tile, or groups of 256
  // channels over the two tiles of a 2-CTA cluster
  bool fusable(int channels, int groups, int L) const {
    const int gc = channels / groups;
    if (gc < 32 || L < 8) return false;
    if (gc <= 128) return 128 % gc == 0;
    return gc == 256 && channels % 256 == 0 && ctx_->pair_clusters > 0;
  }
  void tc_gn(const Act& y, std::size_t batch, int groups, int parts, const float* gamma, const float* beta,
             const BlockDev* film_block, const float* film_time_row, const float* res_f32, const void* res_half,
             Act out, float* out_f32, cudaStream_t st);
  // `in_f32` / `out_f32`: fp32 residual-stream copies of the block input /
  // output on the tensor path (null when absent)
  bool block(const BlockDev& blk, const std::vector<Act>& in, int L, std::size_t batch, bool tc,
             const float* film_time_row, Act out, cudaStream_t st, std::string& err, const float* in_f32 = nullptr,
             float* out_f32 = nullptr);
  template <typename Kernel, typename... Args>
  void launch(Kernel k, dim3 grid, dim3 block, std::size_t smem, cudaStream_t st, Args... args) {
    k<<<grid, block, smem, st>>>(args...);
    ++recorded_;
  }
  // fp32 pointer to sample b0_ of a [samples][per_sample] buffer (the
  // weight-streaming path processes the batch chunk by chunk; b0_ = 0 on the
  // tensor path)
  float* at_sample(void* base, std::size_t per_sample) const { return static_cast<float*>(base) + b0_ * per_sample; }
  std::size_t chunk_samples(std::size_t batch, bool tc) const {
    return tc ? batch : std::max<std::size_t>(1, kSimtChunkTokens / cfg_.horizon);
  }
  bool record_update(std::size_t nb, bool tc, const StepScalars* step, float* eps_out, cudaStream_t st);

  std::shared_ptr<DeviceContext> ctx_;
  Precision prec_;
  DiffusionConfig cfg_{};
  bool tc_ok_ = false;
  int cin_pad_ = 64, cond_pad_ = 64, F_ = 0;
  std::vector<float> alphas_;
  // weights
  DeviceArena wts_;
  std::vector<std::array<BlockDev, 2>> down_;
  std::vector<ConvDev> ds_;
  std::array<BlockDev, 2> mid_;
  std::vector<std::array<BlockDev, 2>> up_;
  std::vector<std::array<ConvDev, 2>> us_;
  ConvDev fc_;
  float *fn_g_ = nullptr, *fn_b_ = nullptr, *fo_w_ = nullptr, *fo_b_ = nullptr;
  ConvDev fo_s_;  // output 1x1 conv in the small-batch program's layout
  // output 1x1 conv for the tensor path: fp16 rows [hi(w) | lo(w)] padded to
  // 128 rows, and the bias of the high rows
  void* fo16_ = nullptr;
  float* fo_b128_ = nullptr;
  std::vector<float> h_fn_g_, h_fn_b_, h_fo_w_, h_fo_b_;
  ConvDev film_;  // W_c of every block's FiLM, [F][cond_pad]
  float* film_time_ = nullptr;  // [T][F]
  float *te1_w_ = nullptr, *te1_b_ = nullptr, *te2_w_ = nullptr, *te2_b_ = nullptr, *wt_ = nullptr;
  float *amin_ = nullptr, *amax_ = nullptr;
  // workspace (reserve)
  DeviceArena ws_;
  std::size_t cap_ = 0;
  std::size_t cap_tc_ = 0;  // capacity rounded for TMA boxes
  float* in_cond_ = nullptr;   // [cap][C]
  float* in_noise_ = nullptr;  // [cap][H][A]
  float* out_action_ = nullptr;
  float* x_master_ = nullptr;
  float* eps_ = nullptr;
  std::uint64_t* seeds_ = nullptr;
  std::uint64_t* seed0_ = nullptr;
  float* tstep_ = nullptr;  // timestep scalar for denoise()
  float* tm_row_ = nullptr;
  float* ft_row_ = nullptr;  // film_time row for denoise()
  void* mcond_ = nullptr;
  float* film_cond_ = nullptr;
  void* x_in_ = nullptr;
  std::vector<void*> acts_;    // per-layer outputs
  std::vector<float*> acts32_;  // fp32 residual-stream copies (tensor path)
  void* h1_ = nullptr;
  void* y1_ = nullptr;
  void* y2_ = nullptr;
  void* yr_ = nullptr;
  float *p1_ = nullptr, *p2_ = nullptr, *p3_ = nullptr;
  double* stats_ = nullptr;
  std::size_t act_elems_ = 0;   // elements per activation buffer
  std::size_t part_elems_ = 0;  // elements per partial buffer
  float* pinned_ = nullptr;
  std::size_t pinned_floats_ = 0;
  struct Graph {
    cudaGraphExec_t exec = nullptr;
    std::uint64_t launches = 0;
    void* tables = nullptr;  // small-batch program: per-step timestep and scheduler scalars
  };
  // small-batch persistent program (stream.cuh), one per batch size
  struct StreamProg {
    void* dev = nullptr;  // ops, partial-sum buffers, segment tables, barrier words
    const sp::Op* ops = nullptr;
    unsigned* sync = nullptr;  // abort word and completion counters, zeroed at every call
    std::size_t sync_words = 0;
    int n_pre = 0, n_step = 0;
    std::size_t smem = 0;
    bool ok = false;
  };
  std::map<std::size_t, StreamProg> progs_;
  // FLOWEDGE_PROGRAM_TRACE=<file>: op timeline of the last program call
  // (mapped host memory, CTA 0's global-timer stamps), written at close
  unsigned long long* trace_ = nullptr;  // device stamps (FLOWEDGE_PROGRAM_TRACE)
  std::size_t trace_bytes_ = 0;
  std::vector<int> trace_kinds_;
  void write_trace() noexcept;
  bool use_stream(std::size_t batch);
  bool build_stream(std::size_t batch, StreamProg& out);
  bool record_stream(std::size_t batch, std::size_t steps, const void* tables, cudaStream_t st, std::string& err);
  void drop_streams() noexcept;
  std::map<std::tuple<std::size_t, std::size_t, int, bool>, Graph> graphs_;
  std::uint64_t launches_ = 0;
  std::uint64_t recorded_ = 0;
  std::size_t b0_ = 0;
  // profiling (fe_engine_profile_diffusion): events around each tensor-core conv
  bool profiling_ = false;
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> prof_events_;
  double prof_flops_ = 0;
 public:
  int profile(std::size_t batch, double* metrics, std::string& err) noexcept override;
};

bool Unet::load(const TensorTable& t, std::string& err) {
  const HostTensor* meta = t.find("dp.meta");
  const HostTensor* dims = t.find("dp.dims");
  if (meta == nullptr || dims == nullptr || meta->dtype != DType::F32 || meta->numel() != 16 ||
      dims->dtype != DType::F32) {
    err = "dp.meta / dp.dims missing or malformed";
    return false;
  }
  const auto mv = widen_f32(*meta);
  auto sz = [&](int i) { return static_cast<std::size_t>(mv[static_cast<std::size_t>(i)]); };
  for (int i : {0, 1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 15}) {
    const float v = mv[static_cast<std::size_t>(i)];
    if (!std::isfinite(v) || v < 0 || std::floor(v) != v) {
      err = "dp.meta holds a non-integer size";
      return false;
    }
  }
  cfg_.action_dim = sz(1);
  cfg_.horizon = sz(2);
  cfg_.action_steps = sz(3);
  cfg_.observation_steps = sz(4);
  cfg_.condition_dim = sz(5);
  cfg_.stages = sz(6);
  cfg_.kernel = sz(7);
  cfg_.groups = sz(8);
  cfg_.timestep_dim = sz(9);
  cfg_.train_timesteps = sz(10);
  cfg_.clip_sample = sz(13) != 0;
  cfg_.clip_sample_range = mv[14];
  // same validation as DiffusionHead::DiffusionHead (diffusion.cc:383-426)
  if (sz(0) != 1 || sz(11) != 0 || sz(12) != 0 || sz(15) != 0 || sz(13) > 1 || cfg_.action_dim == 0 ||
      cfg_.horizon == 0 || cfg_.action_steps == 0 || cfg_.observation_steps == 0 ||
      cfg_.observation_steps > cfg_.horizon || cfg_.action_steps > cfg_.horizon - cfg_.observation_steps + 1 ||
      cfg_.condition_dim == 0 || cfg_.stages < 2 || cfg_.stages > 8 || cfg_.kernel == 0 || cfg_.kernel % 2 == 0 ||
      cfg_.groups == 0 || cfg_.timestep_dim < 4 || cfg_.timestep_dim % 2 != 0 || cfg_.train_timesteps == 0 ||
      dims->numel() != cfg_.stages || !std::isfinite(cfg_.clip_sample_range) || cfg_.clip_sample_range <= 0) {
    err = "dp.meta describes an unsupported Diffusion Policy configuration";
    return false;
  }
  const auto dv = widen_f32(*dims);
  for (float d : dv) {
    if (!(d > 0) || std::floor(d) != d || static_cast<std::size_t>(d) % cfg_.groups != 0) {
      err = "dp.dims entries must be positive multiples of the group count";
      return false;
    }
    cfg_.dims.push_back(static_cast<std::size_t>(d));
  }
  if (cfg_.dims[0] % kFinalNormGroups != 0 || cfg_.horizon % (std::size_t(1) << (cfg_.stages - 1)) != 0) {
    err = "U-Net geometry does not match the horizon";
    return false;
  }
  const int A = static_cast<int>(cfg_.action_dim);
  const int Cd = static_cast<int>(cfg_.condition_dim);
  const int td = static_cast<int>(cfg_.timestep_dim);
  const int k = static_cast<int>(cfg_.kernel);
  cin_pad_ = (A + 63) / 64 * 64;
  cond_pad_ = (Cd + 63) / 64 * 64;

  auto get = [&](const std::string& name, std::initializer_list<std::size_t> shape, bool allow_bf16,
                 std::vector<float>& out) {
    const HostTensor* h = t.find(name);
    if (h == nullptr) {
      err = "missing tensor " + name;
      return false;
    }
    if (h->ndim != static_cast<int>(shape.size()) || (!allow_bf16 && h->dtype != DType::F32)) {
      err = "tensor " + name + " has an unsupported shape or dtype";
      return false;
    }
    int i = 0;
    for (std::size_t s : shape)
      if (h->shape[static_cast<std::size_t>(i++)] != s) {
        err = "tensor " + name + " has an unexpected shape";
        return false;
      }
    out = widen_f32(*h);
    // conv and FiLM weights live on the device in fp16 planes (the time MLP
    // stays fp32: it is tabulated at load)
    if (allow_bf16 && shape.size() >= 2 && name.rfind("dp.te", 0) != 0 &&
        !check_fp16_storable(name, out.data(), out.size(), bf16_weights(), err))
      return false;
    return true;
  };
  // Conv weights: the reference accepts F32 only; BF16 convs are this build's
  // added precision mode.
  auto conv_t = [&](const std::string& pfx, int oc, int ic, int kk, std::vector<float>& w, std::vector<float>& b) {
    return get(pfx + ".w", {static_cast<std::size_t>(oc), static_cast<std::size_t>(ic), static_cast<std::size_t>(kk)},
               true, w) &&
           get(pfx + ".b", {static_cast<std::size_t>(oc)}, false, b);
  };
  std::vector<float> te1w, te1b, te2w, te2b, amin, amax;
  if (!get("dp.te1.w", {static_cast<std::size_t>(4 * td), static_cast<std::size_t>(td)}, true, te1w) ||
      !get("dp.te1.b", {static_cast<std::size_t>(4 * td)}, false, te1b) ||
      !get("dp.te2.w", {static_cast<std::size_t>(td), static_cast<std::size_t>(4 * td)}, true, te2w) ||
      !get("dp.te2.b", {static_cast<std::size_t>(td)}, false, te2b) ||
      !get("dp.action_min", {static_cast<std::size_t>(A)}, false, amin) ||
      !get("dp.action_max", {static_cast<std::size_t>(A)}, false, amax))
    return false;
  for (int a = 0; a < A; ++a)
    if (!std::isfinite(amin[a]) || !std::isfinite(amax[a]) || !(amax[a] > amin[a])) {
      err = "action normalisation statistics are invalid";
      return false;
    }

  std::vector<float> wt_all, wc_all, fb_all;  // FiLM: [F][td], [F][cond_pad], [F]
  F_ = 0;
  auto load_block = [&](BlockDev& blk, const std::string& pfx, std::vector<Part> in_parts, int oc) {
    int ic = 0;
    for (const Part& p : in_parts) ic += p.channels;
    std::vector<float> w, b;
    blk.oc = oc;
    if (!conv_t(pfx + ".c1", oc, ic, k, w, b)) return false;
    pack_conv(blk.c1, ConvKind::kSame, w, b, oc, in_parts, k);
    if (!get(pfx + ".n1.w", {static_cast<std::size_t>(oc)}, false, blk.hg1) ||
        !get(pfx + ".n1.b", {static_cast<std::size_t>(oc)}, false, blk.hb1))
      return false;
    std::vector<float> fw, fbias;
    if (!get(pfx + ".film.w", {static_cast<std::size_t>(2 * oc), static_cast<std::size_t>(td + Cd)}, true, fw) ||
        !get(pfx + ".film.b", {static_cast<std::size_t>(2 * oc)}, false, fbias))
      return false;
    blk.film_off = F_;
    for (int r = 0; r < 2 * oc; ++r) {
      for (int j = 0; j < td; ++j) wt_all.push_back(fw[static_cast<std::size_t>(r) * (td + Cd) + j]);
      for (int j = 0; j < cond_pad_; ++j)
        wc_all.push_back(j < Cd ? fw[static_cast<std::size_t>(r) * (td + Cd) + td + j] : 0.0f);
      fb_all.push_back(fbias[static_cast<std::size_t>(r)]);
    }
    F_ += 2 * oc;
    if (!conv_t(pfx + ".c2", oc, oc, k, w, b)) return false;
    pack_conv(blk.c2, ConvKind::kSame, w, b, oc, {{oc, oc}}, k);
    if (!get(pfx + ".n2.w", {static_cast<std::size_t>(oc)}, false, blk.hg2) ||
        !get(pfx + ".n2.b", {static_cast<std::size_t>(oc)}, false, blk.hb2))
      return false;
    blk.has_res = ic != oc;
    if (blk.has_res) {
      if (!conv_t(pfx + ".res", oc, ic, 1, w, b)) return false;
      pack_conv(blk.res, ConvKind::kPoint, w, b, oc, in_parts, 1);
    }
    return true;
  };

  const int S = static_cast<int>(cfg_.stages);
  down_.resize(static_cast<std::size_t>(S));
  ds_.resize(static_cast<std::size_t>(S));
  for (int s = 0; s < S; ++s) {
    const int oc = static_cast<int>(cfg_.dims[static_cast<std::size_t>(s)]);
    const std::vector<Part> in0 = s == 0 ? std::vector<Part>{{A, cin_pad_}}
                                         : std::vector<Part>{{static_cast<int>(cfg_.dims[s - 1]),
                                                              static_cast<int>(cfg_.dims[s - 1])}};
    if (!load_block(down_[s][0], "dp.d" + std::to_string(s) + ".r0", in0, oc) ||
        !load_block(down_[s][1], "dp.d" + std::to_string(s) + ".r1", {{oc, oc}}, oc))
      return false;
    if (s + 1 < S) {
      std::vector<float> w, b;
      if (!conv_t("dp.d" + std::to_string(s) + ".ds", oc, oc, 3, w, b)) return false;
      pack_conv(ds_[s], ConvKind::kDown, w, b, oc, {{oc, oc}}, 3);
    }
  }
  const int top = static_cast<int>(cfg_.dims.back());
  for (int m = 0; m < 2; ++m)
    if (!load_block(mid_[m], "dp.m" + std::to_string(m), {{top, top}}, top)) return false;
  up_.resize(static_cast<std::size_t>(S - 1));
  us_.resize(static_cast<std::size_t>(S - 1));
  for (int s = 0; s + 1 < S; ++s) {
    const int high = static_cast<int>(cfg_.dims[static_cast<std::size_t>(S - 1 - s)]);
    const int low = static_cast<int>(cfg_.dims[static_cast<std::size_t>(S - 2 - s)]);
    if (!load_block(up_[s][0], "dp.u" + std::to_string(s) + ".r0", {{high, high}, {high, high}}, low) ||
        !load_block(up_[s][1], "dp.u" + std::to_string(s) + ".r1", {{low, low}}, low))
      return false;
    std::vector<float> w, b;
    if (!get("dp.u" + std::to_string(s) + ".us.w",
             {static_cast<std::size_t>(low), static_cast<std::size_t>(low), 4}, true, w) ||
        !get("dp.u" + std::to_string(s) + ".us.b", {static_cast<std::size_t>(low)}, false, b))
      return false;
    pack_conv(us_[s][0], ConvKind::kUp0, w, b, low, {{low, low}}, 4);
    pack_conv(us_[s][1], ConvKind::kUp1, w, b, low, {{low, low}}, 4);
  }
  const int c0 = static_cast<int>(cfg_.dims[0]);
  {
    std::vector<float> w, b;
    if (!conv_t("dp.f.c", c0, c0, k, w, b)) return false;
    pack_conv(fc_, ConvKind::kSame, w, b, c0, {{c0, c0}}, k);
    if (!get("dp.f.n.w", {static_cast<std::size_t>(c0)}, false, h_fn_g_) ||
        !get("dp.f.n.b", {static_cast<std::size_t>(c0)}, false, h_fn_b_) ||
        !conv_t("dp.f.o", A, c0, 1, h_fo_w_, h_fo_b_))
      return false;
  }
  // FiLM condition projection as one GEMM over all blocks
  film_.kind = ConvKind::kPoint;
  film_.oc = F_;
  film_.oc_rows = (F_ + 127) / 128 * 128;
  film_.K = cond_pad_;
  film_.taps = 1;
  film_.ic_total = cond_pad_;
  film_.host_w.assign(static_cast<std::size_t>(film_.oc_rows) * cond_pad_, 0.0f);
  std::copy(wc_all.begin(), wc_all.end(), film_.host_w.begin());
  film_.host_b = fb_all;
  for (int ch = 0; ch < cond_pad_; ch += kSliceCh)
    film_.host_slices.push_back(SimtSlice{0, 0, ch, std::min(kSliceCh, cond_pad_ - ch), ch});
  film_.nslices = static_cast<int>(film_.host_slices.size());
  film_.segs.push_back(tc::Seg{0, 0, 0, cond_pad_ / 64, 0});
  film_.tap_off = {0};

  // alphas_cumprod: squaredcos_cap_v2 betas in double, cumulative product in
  // float (diffusion.cc:186-191, 529-541)
  auto alpha_bar = [](double time) {
    const double c = std::cos(((time + 0.008) / 1.008) * (std::numbers::pi / 2.0));
    return c * c;
  };
  float cumulative = 1.0f;
  const std::size_t T = cfg_.train_timesteps;
  for (std::size_t s = 0; s < T; ++s) {
    const double begin = static_cast<double>(s) / static_cast<double>(T);
    const double end = static_cast<double>(s + 1) / static_cast<double>(T);
    const float beta = static_cast<float>(std::min(1.0 - (alpha_bar(end) / alpha_bar(begin)), 0.999));
    cumulative *= 1.0f - beta;
    alphas_.push_back(cumulative);
  }

  // tensor-path geometry: 64-multiple channels, whole groups per 128-row tile,
  // L >= 4 at the deepest stage.
  tc_ok_ = true;
  for (std::size_t d : cfg_.dims) {
    const std::size_t gc = d / cfg_.groups;
    if (d % 128 != 0 || gc % 32 != 0 || (gc < 128 && 128 % gc != 0) || (gc > 128 && gc % 128 != 0)) tc_ok_ = false;
  }
  if ((cfg_.dims[0] / kFinalNormGroups) % 32 != 0 || cfg_.horizon > 256 || 2 * cfg_.action_dim > tc::BM ||
      (cfg_.horizon & (cfg_.horizon - 1)) != 0 || (cfg_.horizon >> (cfg_.stages - 1)) < 4)
    tc_ok_ = false;

  // ---- upload everything into one arena
  ArenaPlan plan;
  const std::size_t wbytes = bf16_weights() ? 2 : 4;
  auto plan_conv = [&](const ConvDev& c) {
    plan.add(c.host_w.size() * wbytes);
    plan.add(stream_bytes(c.oc, c.K, bf16_weights()));
    plan.add_n<float>(c.host_b.size());
    plan.add_n<SimtSlice>(c.host_slices.size());
  };
  auto plan_block = [&](const BlockDev& b) {
    plan_conv(b.c1);
    plan_conv(b.c2);
    if (b.has_res) plan_conv(b.res);
    plan.add_n<float>(4 * static_cast<std::size_t>(b.oc));
  };
  for (auto& st : down_) plan_block(st[0]), plan_block(st[1]);
  for (auto& c : ds_) plan_conv(c);
  plan_block(mid_[0]);
  plan_block(mid_[1]);
  for (auto& st : up_) plan_block(st[0]), plan_block(st[1]);
  for (auto& pr : us_) plan_conv(pr[0]), plan_conv(pr[1]);
  plan_conv(fc_);
  plan_conv(film_);
  plan.add_n<float>(2 * c0 + A * c0 + A + 2 * A);
  plan.add(static_cast<std::size_t>(tc::BM) * c0 * 2);
  plan.add_n<float>(tc::BM);
  plan.add(stream_bytes(A, c0, bf16_weights()));
  plan.add_n<float>(T * static_cast<std::size_t>(F_));
  plan.add_n<float>(te1w.size() + te1b.size() + te2w.size() + te2b.size() + wt_all.size());
  plan.add_n<float>(T + T * td);
  if (!wts_.init(plan.total(), err)) return false;

  cudaStream_t st = ctx_->stream;
  auto put = [&](const std::vector<float>& h) -> float* {
    float* d = wts_.take_n<float>(h.size());
    cudaMemcpyAsync(d, h.data(), h.size() * sizeof(float), cudaMemcpyHostToDevice, st);
    return d;
  };
  std::vector<std::uint16_t> bf_stage;
  std::vector<std::uint32_t> sw_stage;
  auto put_stream = [&](ConvDev& c, const float* w, int rows) {
    stream_pack(w, rows, c.K, bf16_weights(), sw_stage);
    c.sw = wts_.take(sw_stage.size() * 4);
    if (c.sw != nullptr) cudaMemcpy(c.sw, sw_stage.data(), sw_stage.size() * 4, cudaMemcpyHostToDevice);
    c.s_rbs = (rows + 15) / 16;
    c.s_ks = c.K / 16;
  };
  auto put_conv = [&](ConvDev& c) {
    put_stream(c, c.host_w.data(), c.oc);
    if (bf16_weights()) {
      bf_stage.resize(c.host_w.size());
      for (std::size_t i = 0; i < c.host_w.size(); ++i) bf_stage[i] = fp16_bits_of_bf16_rounded(c.host_w[i]);
      c.w = wts_.take(bf_stage.size() * 2);
      cudaMemcpy(c.w, bf_stage.data(), bf_stage.size() * 2, cudaMemcpyHostToDevice);
    } else {
      c.w = put(c.host_w);
    }
    c.bias = put(c.host_b);
    c.slices = wts_.take_n<SimtSlice>(c.host_slices.size());
    cudaMemcpyAsync(c.slices, c.host_slices.data(), c.host_slices.size() * sizeof(SimtSlice), cudaMemcpyHostToDevice,
                    st);
    cudaStreamSynchronize(st);
    std::vector<float>().swap(c.host_w);
  };
  auto put_block = [&](BlockDev& b) {
    put_conv(b.c1);
    put_conv(b.c2);
    if (b.has_res) put_conv(b.res);
    b.g1 = put(b.hg1);
    b.b1 = put(b.hb1);
    b.g2 = put(b.hg2);
    b.b2 = put(b.hb2);
  };
  for (auto& stg : down_) put_block(stg[0]), put_block(stg[1]);
  for (int s = 0; s + 1 < S; ++s) put_conv(ds_[s]);
  put_block(mid_[0]);
  put_block(mid_[1]);
  for (auto& stg : up_) put_block(stg[0]), put_block(stg[1]);
  for (auto& pr : us_) put_conv(pr[0]), put_conv(pr[1]);
  put_conv(fc_);
  put_conv(film_);
  fn_g_ = put(h_fn_g_);
  fn_b_ = put(h_fn_b_);
  fo_w_ = put(h_fo_w_);
  fo_b_ = put(h_fo_b_);
  // output 1x1 conv as a program conv (A rows x c0)
  fo_s_.kind = ConvKind::kPoint;
  fo_s_.oc = A;
  fo_s_.K = c0;
  fo_s_.ic_total = c0;
  fo_s_.taps = 1;
  fo_s_.tap_off = {0};
  fo_s_.bias = fo_b_;
  put_stream(fo_s_, h_fo_w_.data(), A);
  if (tc_ok_) {
    // w = hi + lo with hi = fp16(w), lo = fp16(w - hi): the pair carries the
    // fp32 weight to about 2^-22 relative, and the tensor cores accumulate in fp32
    std::vector<std::uint16_t> w16(static_cast<std::size_t>(tc::BM) * c0, 0);
    std::vector<float> b128(tc::BM, 0.0f);
    for (int a = 0; a < A; ++a) {
      for (int c = 0; c < c0; ++c) {
        const float w = h_fo_w_[static_cast<std::size_t>(a) * c0 + c];
        const __half hi = __float2half_rn(w);
        const __half lo = __float2half_rn(w - __half2float(hi));
        w16[static_cast<std::size_t>(a) * c0 + c] = __half_as_ushort(hi);
        w16[static_cast<std::size_t>(A + a) * c0 + c] = __half_as_ushort(lo);
      }
      b128[static_cast<std::size_t>(a)] = h_fo_b_[static_cast<std::size_t>(a)];
    }
    fo16_ = wts_.take(w16.size() * 2);
    if (fo16_ != nullptr) cudaMemcpy(fo16_, w16.data(), w16.size() * 2, cudaMemcpyHostToDevice);
    fo_b128_ = put(b128);
  }
  amin_ = put(amin);
  amax_ = put(amax);
  film_time_ = wts_.take_n<float>(T * static_cast<std::size_t>(F_));
  te1_w_ = put(te1w);
  te1_b_ = put(te1b);
  te2_w_ = put(te2w);
  te2_b_ = put(te2b);
  wt_ = put(wt_all);
  std::vector<float> ts(T);
  for (std::size_t i = 0; i < T; ++i) ts[i] = static_cast<float>(i);
  float* d_ts = put(ts);
  float* d_tm = wts_.take_n<float>(T * static_cast<std::size_t>(td));
  if (wts_.overflowed()) {
    err = "internal error: U-Net weight arena too small";
    return false;
  }
  temb_kernel<<<static_cast<unsigned>(T), 128, static_cast<std::size_t>(5 * td) * sizeof(float), st>>>(
      d_ts, static_cast<int>(T), td, te1_w_, te1_b_, te2_w_, te2_b_, d_tm);
  film_time_kernel<<<ew_grid(static_cast<long long>(T) * F_, 256, *ctx_), 256, 0, st>>>(d_tm, static_cast<int>(T), td,
                                                                                        wt_, F_, film_time_);
  if (cudaStreamSynchronize(st) != cudaSuccess) {
    err = std::string("weight upload failed: ") + cudaGetErrorString(cudaGetLastError());
    return false;
  }
  return true;
}

int Unet::reserve(std::size_t batch, std::string& err) noexcept {
  if (batch == 0) batch = 1;
  if (batch <= cap_) return 0;
  // drop graphs and programs recorded against the old workspace
  for (auto& [key, g] : graphs_) {
    cudaGraphExecDestroy(g.exec);
    if (g.tables != nullptr) cudaFree(g.tables);
  }
  graphs_.clear();
  drop_streams();
  const std::size_t H = cfg_.horizon, A = cfg_.action_dim;
  const std::size_t cap_tc = (batch + 255) / 256 * 256;
  std::size_t max_c = 0;
  for (std::size_t d : cfg_.dims) max_c = std::max(max_c, d);
  // largest activation: C * L at any stage is at most max(dims[s] * H >> s), plus concat (2 * high * L)
  std::size_t per_sample = static_cast<std::size_t>(cin_pad_) * H;
  for (std::size_t s = 0; s < cfg_.stages; ++s) {
    per_sample = std::max(per_sample, cfg_.dims[s] * (H >> s));
  }
  act_elems_ = per_sample * cap_tc;
  // split-K partials: nslices * n_tokens * M for the largest conv, for one
  // chunk of the weight-streaming path
  std::size_t part = 0;
  const std::size_t simt_batch = std::min(batch, chunk_samples(batch, false));
  auto pc = [&](const ConvDev& c, std::size_t L) {
    part = std::max(part, static_cast<std::size_t>(c.nslices) * simt_batch * L * static_cast<std::size_t>(c.oc));
  };
  for (std::size_t s = 0; s < cfg_.stages; ++s) {
    const std::size_t L = H >> s;
    for (auto& b : down_[s]) {
      pc(b.c1, L), pc(b.c2, L);
      if (b.has_res) pc(b.res, L);
    }
    if (s + 1 < cfg_.stages) pc(ds_[s], L / 2);
  }
  const std::size_t Lm = H >> (cfg_.stages - 1);
  for (auto& b : mid_) pc(b.c1, Lm), pc(b.c2, Lm);
  for (std::size_t s = 0; s + 1 < cfg_.stages; ++s) {
    const std::size_t L = H >> (cfg_.stages - 1 - s);
    for (auto& b : up_[s]) {
      pc(b.c1, L), pc(b.c2, L);
      if (b.has_res) pc(b.res, L);
    }
    pc(us_[s][0], L), pc(us_[s][1], L);
  }
  pc(fc_, H);
  pc(film_, 1);
  part_elems_ = part;
  // outputs: 3 per down stage (r0, r1, downsample), 2 middle, 3 per up stage
  const std::size_t n_layers = 6 * cfg_.stages;
  const std::size_t ebytes = 4;  // activation buffers sized for fp32 (bf16 uses half)
  ArenaPlan plan;
  plan.add_n<float>(batch * cfg_.condition_dim);
  plan.add_n<float>(batch * H * A);
  plan.add_n<float>(batch * H * A);
  plan.add_n<float>(batch * H * A);
  plan.add_n<float>(batch * H * A);
  plan.add_n<std::uint64_t>(batch);
  plan.add_n<std::uint64_t>(1);
  plan.add_n<float>(1);
  plan.add_n<float>(cfg_.timestep_dim);
  plan.add_n<float>(static_cast<std::size_t>(F_));
  plan.add(cap_tc * static_cast<std::size_t>(cond_pad_) * ebytes);
  plan.add_n<float>(batch * static_cast<std::size_t>(F_));
  plan.add(cap_tc * H * static_cast<std::size_t>(cin_pad_) * ebytes);
  const bool twins = prec_ == Precision::kBF16 && tc_ok_;
  for (std::size_t i = 0; i < n_layers + 4 + (twins ? n_layers : 0); ++i) plan.add(act_elems_ * ebytes);
  for (int i = 0; i < 3; ++i) plan.add_n<float>(part_elems_);
  plan.add_n<double>(cap_tc * 8 * 2 * 2 + 64);
  ws_.release();
  if (!ws_.init(plan.total(), err)) {
    cap_ = 0;
    return 2;
  }
  in_cond_ = ws_.take_n<float>(batch * cfg_.condition_dim);
  in_noise_ = ws_.take_n<float>(batch * H * A);
  out_action_ = ws_.take_n<float>(batch * H * A);
  x_master_ = ws_.take_n<float>(batch * H * A);
  eps_ = ws_.take_n<float>(batch * H * A);
  seeds_ = ws_.take_n<std::uint64_t>(batch);
  seed0_ = ws_.take_n<std::uint64_t>(1);
  tstep_ = ws_.take_n<float>(1);
  tm_row_ = ws_.take_n<float>(cfg_.timestep_dim);
  ft_row_ = ws_.take_n<float>(static_cast<std::size_t>(F_));
  mcond_ = ws_.take(cap_tc * static_cast<std::size_t>(cond_pad_) * ebytes);
  film_cond_ = ws_.take_n<float>(batch * static_cast<std::size_t>(F_));
  x_in_ = ws_.take(cap_tc * H * static_cast<std::size_t>(cin_pad_) * ebytes);
  acts_.clear();
  for (std::size_t i = 0; i < n_layers; ++i) acts_.push_back(ws_.take(act_elems_ * ebytes));
  acts32_.assign(n_layers, nullptr);
  if (twins)
    for (std::size_t i = 0; i < n_layers; ++i) acts32_[i] = ws_.take_n<float>(act_elems_);
  h1_ = ws_.take(act_elems_ * ebytes);
  y1_ = ws_.take(act_elems_ * ebytes);
  y2_ = ws_.take(act_elems_ * ebytes);
  yr_ = ws_.take(act_elems_ * ebytes);
  p1_ = ws_.take_n<float>(part_elems_);
  p2_ = ws_.take_n<float>(part_elems_);
  p3_ = ws_.take_n<float>(part_elems_);
  stats_ = ws_.take_n<double>(cap_tc * 8 * 2 * 2 + 64);
  if (ws_.overflowed()) {
    err = "internal error: U-Net workspace arena too small";
    cap_ = 0;
    return 2;
  }
  // zero everything once so padded channels / padded samples read as zeros
  cudaMemsetAsync(in_cond_, 0, ws_.used(), ctx_->stream);
  // pinned staging for host calls
  const std::size_t need = batch * (cfg_.condition_dim + 2 * H * A);
  if (pinned_floats_ < need) {
    if (pinned_ != nullptr) cudaFreeHost(pinned_);
    pinned_ = nullptr;
    if (counted_host_malloc(reinterpret_cast<void**>(&pinned_), need * sizeof(float)) != cudaSuccess) {
      err = "pinned host allocation failed";
      pinned_floats_ = 0;
      return 2;
    }
    pinned_floats_ = need;
  }
  if (cudaStreamSynchronize(ctx_->stream) != cudaSuccess) {
    err = "workspace initialisation failed";
    return 2;
  }
  cap_ = batch;
  cap_tc_ = cap_tc;
  return 0;
}

bool Unet::simt_conv(const ConvDev& c, const std::vector<Act>& srcs, int L_out, std::size_t batch, float* partial,
                     cudaStream_t st, std::string& err) {
  SimtConvParams p{};
  p.W = c.w;
  p.M = c.oc;
  p.K = c.K;
  for (std::size_t i = 0; i < srcs.size() && i < 3; ++i)
    p.src[i] = SimtSource{static_cast<const float*>(srcs[i].p), srcs[i].C, srcs[i].L};
  p.stride = c.stride;
  p.L_out = L_out;
  p.n_tokens = static_cast<int>(batch) * L_out;
  p.slices = c.slices;
  p.partial = partial;
  const int nt = p.n_tokens >= 16 ? 16 : (p.n_tokens >= 8 ? 8 : 4);
  const dim3 grid(static_cast<unsigned>(c.nslices), static_cast<unsigned>((c.oc + 127) / 128),
                  static_cast<unsigned>((p.n_tokens + nt - 1) / nt));
  const bool bf = bf16_weights();
  if (nt == 16) {
    if (bf) launch(simt_conv_kernel<16, true>, grid, dim3(128), 0, st, p);
    else launch(simt_conv_kernel<16, false>, grid, dim3(128), 0, st, p);
  } else if (nt == 8) {
    if (bf) launch(simt_conv_kernel<8, true>, grid, dim3(128), 0, st, p);
    else launch(simt_conv_kernel<8, false>, grid, dim3(128), 0, st, p);
  } else {
    if (bf) launch(simt_conv_kernel<4, true>, grid, dim3(128), 0, st, p);
    else launch(simt_conv_kernel<4, false>, grid, dim3(128), 0, st, p);
  }
  (void)err;
  return true;
}

void Unet::simt_reduce(const ConvDev& c, const float* partial, std::size_t batch, int L_tok, Act out, int rps,
                       int tmul, int tadd, cudaStream_t st) {
  // generic reduce with a row mapping: token (b, t) -> out row b * rps + t * tmul + tadd
  ReduceParams p{};
  p.partial = partial;
  p.nslices = c.nslices;
  p.n_tokens = static_cast<int>(batch) * L_tok;
  p.M = c.oc;
  p.bias = c.bias;
  p.act = 0;
  p.accumulate = 0;
  if (rps == L_tok && tmul == 1 && tadd == 0) {
    p.out = static_cast<float*>(out.p);
    p.out_ld = out.C;
    launch(reduce_partials_kernel, dim3(ew_grid(static_cast<long long>(p.n_tokens) * p.M, 256, *ctx_)), dim3(256), 0,
           st, p);
    return;
  }
  // strided rows (conv-transpose phases): one launch per sample row pattern via out_ld trick:
  // out row for (b, t) = b * rps + t * tmul + tadd; with rps == L_tok * tmul this is
  // (b * L_tok + t) * tmul + tadd, i.e. a fixed stride of tmul rows.
  p.out = static_cast<float*>(out.p) + static_cast<long long>(tadd) * out.C;
  p.out_ld = out.C * tmul;
  launch(reduce_partials_kernel, dim3(ew_grid(static_cast<long long>(p.n_tokens) * p.M, 256, *ctx_)), dim3(256), 0,
         st, p);
}

void Unet::simt_gn(const ConvDev& c, const float* partial, std::size_t batch, int L, const float* gamma,
                   const float* beta, int groups, const BlockDev* film_block, const float* film_time_row,
                   const float* res_tensor, const ConvDev* res_conv, const float* res_partial, Act out,
                   cudaStream_t st) {
  GnParams p{};
  p.partial = partial;
  p.nslices = c.nslices;
  p.n_tokens = static_cast<int>(batch) * L;
  p.C = c.oc;
  p.L = L;
  p.bias = c.bias;
  p.gamma = gamma;
  p.beta = beta;
  p.groups = groups;
  p.mish = 1;
  if (film_block != nullptr) {
    p.film_cond = film_cond_ + b0_ * static_cast<std::size_t>(F_);
    p.film_time = film_time_row;
    p.film_F = F_;
    p.film_off = film_block->film_off;
  }
  p.res = res_tensor;
  if (res_conv != nullptr) {
    p.res_partial = res_partial;
    p.res_nslices = res_conv->nslices;
    p.res_bias = res_conv->bias;
  }
  p.out = static_cast<float*>(out.p);
  launch(gn_partials_kernel, dim3(static_cast<unsigned>(batch), static_cast<unsigned>(groups)), dim3(256), 0, st, p);
}

bool Unet::tc_conv(const ConvDev& c, const std::vector<Act>& srcs, int L_out, std::size_t batch, void* out,
                   long long out_ld, int rps, int tmul, int tadd, bool stats, int groups, bool out_f32,
                   cudaStream_t st, std::string& err, const Fuse* fuse) {
  TcLaunch l;
  l.fp16 = true;
  l.A = c.w;
  l.M_rows = c.oc_rows;
  l.K = c.K;
  for (std::size_t i = 0; i < srcs.size() && i < 3; ++i) {
    l.src[i].ptr = srcs[i].p;
    l.src[i].channels = srcs[i].C;
    l.src[i].length = srcs[i].L;
    l.src[i].samples = static_cast<int>(cap_tc_);
  }
  if (c.kind == ConvKind::kDown) {  // pair view of the input
    l.src[0].channels = srcs[0].C * 2;
    l.src[0].length = srcs[0].L / 2;
  }
  l.L = L_out;
  l.n_samples = static_cast<int>(batch);
  l.m_valid = c.oc;
  l.segs = c.segs;
  l.bias = c.bias;
  l.out = out;
  l.out_ld = out_ld;
  l.out_rps = rps;
  l.out_tmul = tmul;
  l.out_tadd = tadd;
  l.out_f32 = out_f32;
  if (stats) {
    l.stats = stats_;
    l.groups = groups;
    l.group_ch = c.oc / groups;
  }
  if (fuse != nullptr) {
    l.gn_fuse = true;
    l.groups = fuse->groups;
    l.group_ch = c.oc / fuse->groups;
    l.gamma = fuse->gamma;
    l.beta = fuse->beta;
    if (fuse->film_block != nullptr) {
      l.film_cond = film_cond_;
      l.film_time = fuse->film_time_row;
      l.film_F = F_;
      l.film_off = fuse->film_block->film_off;
      l.film_C = c.oc;
    }
    l.res_f32 = fuse->res_f32;
    l.res16 = fuse->res16;
    l.out_twin = fuse->out_twin;
  }
  ++recorded_;
  if (!profiling_) return tc_gemm(l, *ctx_, st, err) == cudaSuccess;
  // algorithmic FLOPs: 2 * out channels * (taps * real input channels) * tokens
  int ic_real = 0;
  for (const tc::Seg& sg : c.segs) ic_real += sg.kblocks * 64;
  if (c.kind == ConvKind::kSame && c.ic_total == cin_pad_) ic_real = static_cast<int>(cfg_.action_dim) * c.taps;
  prof_flops_ += 2.0 * c.oc * ic_real * static_cast<double>(batch) * L_out;
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  cudaEventRecord(a, st);
  const bool ok = tc_gemm(l, *ctx_, st, err) == cudaSuccess;
  cudaEventRecord(b, st);
  prof_events_.emplace_back(a, b);
  return ok;
}

void Unet::tc_gn(const Act& y, std::size_t batch, int groups, int parts, const float* gamma, const float* beta,
                 const BlockDev* film_block, const float* film_time_row, const float* res_f32, const void* res_half,
                 Act out, float* out_f32, cudaStream_t st) {
  GnTcParams p{};
  p.y = static_cast<const float*>(y.p);
  p.n_tokens = static_cast<long long>(batch) * y.L;
  p.C = y.C;
  p.L = y.L;
  p.groups = groups;
  p.parts = parts;
  p.stats = stats_;
  p.gamma = gamma;
  p.beta = beta;
  if (film_block != nullptr) {
    p.film_cond = film_cond_;
    p.film_time = film_time_row;
    p.film_F = F_;
    p.film_off = film_block->film_off;
  }
  p.res_f32 = res_f32;
  p.res_half = res_f32 == nullptr ? static_cast<const __half*>(res_half) : nullptr;
  p.out = static_cast<__half*>(out.p);
  p.out_f32 = out_f32;
  launch(gn_tc_kernel, dim3(ew_grid(p.n_tokens * (p.C / 8), 256, *ctx_)), dim3(256), 0, st, p);
}

bool Unet::block(const BlockDev& blk, const std::vector<Act>& in, int L, std::size_t batch, bool tc,
                 const float* film_time_row, Act out, cudaStream_t st, std::string& err, const float* in_f32,
                 float* out_f32) {
  const int G = static_cast<int>(cfg_.groups);
  const int oc = blk.oc;
  Act h1{at_sample(h1_, static_cast<std::size_t>(oc) * L), oc, L};
  if (!tc) {
    if (!simt_conv(blk.c1, in, L, batch, p1_, st, err)) return false;
    simt_gn(blk.c1, p1_, batch, L, blk.g1, blk.b1, G, &blk, film_time_row, nullptr, nullptr, nullptr, h1, st);
    if (!simt_conv(blk.c2, {h1}, L, batch, p2_, st, err)) return false;
    if (blk.has_res) {
      if (!simt_conv(blk.res, in, L, batch, p3_, st, err)) return false;
      simt_gn(blk.c2, p2_, batch, L, blk.g2, blk.b2, G, nullptr, nullptr, nullptr, &blk.res, p3_, out, st);
    } else {
      simt_gn(blk.c2, p2_, batch, L, blk.g2, blk.b2, G, nullptr, nullptr, static_cast<const float*>(in[0].p), nullptr,
              nullptr, out, st);
    }
    return true;
  }
  if (fusable(oc, G, L)) {
    // GroupNorm + Mish + FiLM / residual in the conv epilogues
    Fuse f1;
    f1.gamma = blk.g1;
    f1.beta = blk.b1;
    f1.film_block = &blk;
    f1.film_time_row = film_time_row;
    f1.groups = G;
    if (!tc_conv(blk.c1, in, L, batch, h1.p, oc, L, 1, 0, false, 0, false, st, err, &f1)) return false;
    Fuse f2;
    f2.gamma = blk.g2;
    f2.beta = blk.b2;
    f2.groups = G;
    f2.out_twin = out_f32;
    if (blk.has_res) {
      if (!tc_conv(blk.res, in, L, batch, yr_, oc, L, 1, 0, false, 0, true, st, err)) return false;
      f2.res_f32 = static_cast<const float*>(yr_);
    } else {
      f2.res_f32 = in_f32;
      f2.res16 = in_f32 == nullptr ? in[0].p : nullptr;
    }
    return tc_conv(blk.c2, {h1}, L, batch, out.p, oc, L, 1, 0, false, 0, false, st, err, &f2);
  }
  // conv outputs (pre-norm y, 1x1 residual) stay fp32; only GEMM operands are 16-bit
  const int parts = (oc / G) > 128 ? (oc / G) / 128 : 1;
  Act y1{y1_, oc, L}, y2{y2_, oc, L};
  if (!tc_conv(blk.c1, in, L, batch, y1_, oc, L, 1, 0, true, G, true, st, err)) return false;
  tc_gn(y1, batch, G, parts, blk.g1, blk.b1, &blk, film_time_row, nullptr, nullptr, h1, nullptr, st);
  if (!tc_conv(blk.c2, {h1}, L, batch, y2_, oc, L, 1, 0, true, G, true, st, err)) return false;
  const float* res_f32 = in_f32;
  const void* res_half = in[0].p;
  if (blk.has_res) {
    if (!tc_conv(blk.res, in, L, batch, yr_, oc, L, 1, 0, false, 0, true, st, err)) return false;
    res_f32 = static_cast<const float*>(yr_);
  }
  tc_gn(y2, batch, G, parts, blk.g2, blk.b2, nullptr, nullptr, res_f32, res_half, out, out_f32, st);
  return true;
}

bool Unet::record_film_cond(std::size_t batch, bool tc, cudaStream_t st, std::string& err) {
  launch(prep_cond_kernel, dim3(ew_grid(static_cast<long long>(batch) * cond_pad_, 256, *ctx_)), dim3(256), 0, st,
         static_cast<const float*>(in_cond_ + b0_ * cfg_.condition_dim), static_cast<int>(batch),
         static_cast<int>(cfg_.condition_dim), static_cast<void*>(at_sample(mcond_, cond_pad_)), cond_pad_, tc ? 1 : 0);
  Act mc{at_sample(mcond_, cond_pad_), cond_pad_, 1};
  if (tc) return tc_conv(film_, {mc}, 1, batch, film_cond_, F_, 1, 1, 0, false, 0, true, st, err);
  if (!simt_conv(film_, {mc}, 1, batch, p1_, st, err)) return false;
  simt_reduce(film_, p1_, batch, 1, Act{film_cond_ + b0_ * static_cast<std::size_t>(F_), F_, 1}, 1, 1, 0, st);
  return true;
}

bool Unet::record_forward(std::size_t batch, bool tc, const float* ft_row, cudaStream_t st, std::string& err) {
  const std::size_t S = cfg_.stages;
  const int H = static_cast<int>(cfg_.horizon);
  std::size_t li = 0;
  Act x{at_sample(x_in_, static_cast<std::size_t>(cin_pad_) * H), cin_pad_, H};
  float* x_f32 = nullptr;  // fp32 residual-stream copy of x (tensor path)
  std::vector<Act> skips(S);
  int L = H;
  for (std::size_t s = 0; s < S; ++s) {
    const int oc = static_cast<int>(cfg_.dims[s]);
    const std::size_t per = static_cast<std::size_t>(oc) * L;
    Act o0{at_sample(acts_[li], per), oc, L}, o1{at_sample(acts_[li + 1], per), oc, L};
    float* t0 = tc ? acts32_[li] : nullptr;
    float* t1 = tc ? acts32_[li + 1] : nullptr;
    li += 2;
    if (!block(down_[s][0], {x}, L, batch, tc, ft_row, o0, st, err, nullptr, t0)) return false;
    if (!block(down_[s][1], {o0}, L, batch, tc, ft_row, o1, st, err, t0, t1)) return false;
    x_f32 = t1;
    skips[s] = o1;
    x = o1;
    if (s + 1 < S) {
      Act d{at_sample(acts_[li++], per / 2), oc, L / 2};
      if (tc) {
        if (!tc_conv(ds_[s], {x}, L / 2, batch, d.p, oc, L / 2, 1, 0, false, 0, false, st, err)) return false;
      } else {
        if (!simt_conv(ds_[s], {x}, L / 2, batch, p1_, st, err)) return false;
        simt_reduce(ds_[s], p1_, batch, L / 2, d, L / 2, 1, 0, st);
      }
      x = d;
      x_f32 = nullptr;
      L /= 2;
    } else {
      ++li;
    }
  }
  for (int m = 0; m < 2; ++m) {
    float* tm = tc ? acts32_[li] : nullptr;
    Act o{at_sample(acts_[li++], static_cast<std::size_t>(x.C) * L), x.C, L};
    if (!block(mid_[m], {x}, L, batch, tc, ft_row, o, st, err, x_f32, tm)) return false;
    x = o;
    x_f32 = tm;
  }
  for (std::size_t s = 0; s + 1 < S; ++s) {
    const Act skip = skips[S - 1 - s];
    const int low = static_cast<int>(cfg_.dims[S - 2 - s]);
    const std::size_t per = static_cast<std::size_t>(low) * L;
    Act o0{at_sample(acts_[li], per), low, L}, o1{at_sample(acts_[li + 1], per), low, L};
    float* t0 = tc ? acts32_[li] : nullptr;
    li += 2;
    if (!block(up_[s][0], {x, skip}, L, batch, tc, ft_row, o0, st, err, nullptr, t0)) return false;
    if (!block(up_[s][1], {o0}, L, batch, tc, ft_row, o1, st, err, t0, nullptr)) return false;
    Act u{at_sample(acts_[li++], 2 * per), low, 2 * L};
    for (int ph = 0; ph < 2; ++ph) {
      if (tc) {
        if (!tc_conv(us_[s][ph], {o1}, L, batch, u.p, low, 2 * L, 2, ph, false, 0, false, st, err)) return false;
      } else {
        if (!simt_conv(us_[s][ph], {o1}, L, batch, p1_, st, err)) return false;
        simt_reduce(us_[s][ph], p1_, batch, L, u, 2 * L, 2, ph, st);
      }
    }
    x = u;
    L *= 2;
  }
  // final conv -> GN(8) + Mish -> z in h1_
  const int c0 = static_cast<int>(cfg_.dims[0]);
  Act z{at_sample(h1_, static_cast<std::size_t>(c0) * H), c0, H};
  if (tc) {
    if (fusable(c0, static_cast<int>(kFinalNormGroups), H)) {
      Fuse f;
      f.gamma = fn_g_;
      f.beta = fn_b_;
      f.groups = static_cast<int>(kFinalNormGroups);
      if (!tc_conv(fc_, {x}, H, batch, z.p, c0, H, 1, 0, false, 0, false, st, err, &f)) return false;
    } else {
      if (!tc_conv(fc_, {x}, H, batch, y1_, c0, H, 1, 0, true, static_cast<int>(kFinalNormGroups), true, st, err))
        return false;
      tc_gn(Act{y1_, c0, H}, batch, static_cast<int>(kFinalNormGroups), 1, fn_g_, fn_b_, nullptr, nullptr, nullptr,
            nullptr, z, nullptr, st);
    }
  } else {
    if (!simt_conv(fc_, {x}, H, batch, p1_, st, err)) return false;
    simt_gn(fc_, p1_, batch, H, fn_g_, fn_b_, static_cast<int>(kFinalNormGroups), nullptr, nullptr, nullptr, nullptr,
            nullptr, z, st);
  }
  return true;
}

std::vector<StepPlan> Unet::plan_steps(std::size_t steps, int scheduler) const {
  std::vector<StepPlan> plan;
  const std::size_t ratio = cfg_.train_timesteps / steps;
  for (std::size_t i = 0; i < steps; ++i) {
    const std::size_t timestep = (steps - 1 - i) * ratio;
    const long long previous = static_cast<long long>(timestep) - static_cast<long long>(ratio);
    // scalar arithmetic exactly as DiffusionHead::sample (diffusion.cc:997-1024)
    const float alpha_t = alphas_[timestep];
    const float alpha_prev = previous >= 0 ? alphas_[static_cast<std::size_t>(previous)] : 1.0f;
    const float beta_t = 1.0f - alpha_t;
    StepScalars s{};
    s.sqrt_alpha = std::sqrt(alpha_t);
    s.sqrt_beta = std::sqrt(beta_t);
    s.sqrt_alpha_prev = std::sqrt(alpha_prev);
    s.sqrt_one_minus_prev = std::sqrt(1.0f - alpha_prev);
    s.clip = cfg_.clip_sample ? 1 : 0;
    s.clip_range = cfg_.clip_sample_range;
    s.ddpm = scheduler == 1 ? 1 : 0;
    if (s.ddpm) {
      const float current_alpha = alpha_t / alpha_prev;
      const float current_beta = 1.0f - current_alpha;
      s.orig_coef = std::sqrt(alpha_prev) * current_beta / std::max(beta_t, 1e-20f);
      s.sample_coef = std::sqrt(current_alpha) * (1.0f - alpha_prev) / std::max(beta_t, 1e-20f);
      const float variance = ((1.0f - alpha_prev) / std::max(beta_t, 1e-20f)) * current_beta;
      s.noise_std = std::sqrt(std::max(variance, 1e-20f));
      s.add_noise = previous >= 0 ? 1 : 0;
      s.noise_draw = static_cast<int>(i);
    }
    plan.push_back(StepPlan{static_cast<int>(timestep), static_cast<int>(previous), s});
  }
  return plan;
}

__global__ void seeds_kernel(const std::uint64_t* seed0, std::uint64_t* seeds, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) seeds[i] = *seed0 + static_cast<std::uint64_t>(i);
}

bool Unet::record_update(std::size_t nb, bool tc, const StepScalars* step, float* eps_out, cudaStream_t st) {
  const int H = static_cast<int>(cfg_.horizon), A = static_cast<int>(cfg_.action_dim);
  const int c0 = static_cast<int>(cfg_.dims[0]);
  const int n_tokens = static_cast<int>(nb) * H;
  const unsigned blocks = static_cast<unsigned>((n_tokens * 32 + 255) / 256);
  const std::size_t xa = b0_ * static_cast<std::size_t>(H * A);
  auto fill = [&](auto& p) {
    p.C = c0, p.A = A, p.H = H, p.n_tokens = n_tokens;
    p.W = fo_w_, p.bias = fo_b_, p.x_master = x_master_ + xa;
    p.eps_out = eps_out != nullptr ? eps_out + xa : nullptr;
    p.update = step != nullptr ? 1 : 0;
    if (step != nullptr) p.step = *step;
    p.seeds = seeds_ + b0_;
    p.Cin = cin_pad_;
  };
  if (tc) {
    // eps pairs [token][2A] on the tensor cores, then the elementwise update
    TcLaunch l;
    l.fp16 = true;
    l.A = fo16_;
    l.M_rows = tc::BM;
    l.K = c0;
    l.src[0] = TcSource{h1_, c0, H, static_cast<int>(cap_tc_)};
    l.L = H;
    l.n_samples = static_cast<int>(nb);
    l.m_valid = 2 * A;
    l.segs = {tc::Seg{0, 0, 0, c0 / 64, 0}};
    l.bias = fo_b128_;
    l.out = yr_;
    l.out_ld = 2 * A;
    l.out_rps = H;
    l.out_f32 = true;
    std::string err;
    ++recorded_;
    if (tc_gemm(l, *ctx_, st, err) != cudaSuccess) return false;
    EpsUpdateParams p{};
    p.t = static_cast<const float*>(yr_);
    p.A = A, p.H = H, p.n_tokens = n_tokens;
    p.x_master = x_master_ + xa;
    p.eps_out = eps_out != nullptr ? eps_out + xa : nullptr;
    p.update = step != nullptr ? 1 : 0;
    if (step != nullptr) p.step = *step;
    p.seeds = seeds_ + b0_;
    p.x_in = static_cast<__half*>(x_in_);
    p.Cin = cin_pad_;
    launch(eps_update_kernel, dim3(ew_grid(static_cast<long long>(n_tokens) * A, 256, *ctx_)), dim3(256), 0, st, p);
  } else {
    OutParams<float> p{};
    fill(p);
    p.z = at_sample(h1_, static_cast<std::size_t>(c0) * H);
    p.x_in = at_sample(x_in_, static_cast<std::size_t>(cin_pad_) * H);
    p.x_in_half = 0;
    if (A <= 16) launch(out_update_kernel<float, 16>, dim3(blocks), dim3(256), 0, st, p);
    else launch(out_update_kernel<float, 64>, dim3(blocks), dim3(256), 0, st, p);
  }
  return cudaPeekAtLastError() == cudaSuccess;
}

bool Unet::record_sample(std::size_t batch, const std::vector<StepPlan>& plan, cudaStream_t st, std::string& err) {
  const bool tc = use_tc(batch);
  const int H = static_cast<int>(cfg_.horizon), A = static_cast<int>(cfg_.action_dim);
  const int n_tokens = static_cast<int>(batch) * H;
  const std::size_t chunk = chunk_samples(batch, tc);
  b0_ = 0;
  launch(seeds_kernel, dim3((static_cast<unsigned>(batch) + 255) / 256), dim3(256), 0, st,
         static_cast<const std::uint64_t*>(seed0_), seeds_, static_cast<int>(batch));
  launch(prep_sample_kernel, dim3(ew_grid(static_cast<long long>(n_tokens) * cin_pad_, 256, *ctx_)), dim3(256), 0, st,
         static_cast<const float*>(in_noise_), n_tokens, A, x_master_, x_in_, cin_pad_, tc ? 1 : 0);
  for (b0_ = 0; b0_ < batch; b0_ += chunk)
    if (!record_film_cond(std::min(chunk, batch - b0_), tc, st, err)) return false;
  for (const StepPlan& sp : plan) {
    const float* ft_row = film_time_ + static_cast<std::size_t>(sp.timestep) * static_cast<std::size_t>(F_);
    for (b0_ = 0; b0_ < batch; b0_ += chunk) {
      const std::size_t nb = std::min(chunk, batch - b0_);
      if (!record_forward(nb, tc, ft_row, st, err) || !record_update(nb, tc, &sp.scalars, nullptr, st)) {
        b0_ = 0;
        return false;
      }
    }
  }
  b0_ = 0;
  launch(unnormalize_kernel, dim3(ew_grid(static_cast<long long>(n_tokens) * A, 256, *ctx_)), dim3(256), 0, st,
         static_cast<const float*>(x_master_), n_tokens, A, static_cast<const float*>(amin_),
         static_cast<const float*>(amax_), out_action_);
  return true;
}

// ---------------------------------------------------------------------------
// small-batch persistent program (stream.cuh)

namespace {
// per-step tables of a recorded program: int timestep[steps], then StepScalars[steps]
std::size_t stream_table_off(std::size_t steps) { return (steps * sizeof(int) + 255) & ~std::size_t(255); }

// CTA whose range [U c / NC, U (c + 1) / NC) holds item u (host twin of sp::cta_of)
int cta_of_host(long long u, long long U, int NC) {
  int c = static_cast<int>((u * NC) / U);
  while (c + 1 < NC && (U * (c + 1)) / NC <= u) ++c;
  while (c > 0 && (U * c) / NC > u) --c;
  return c;
}
}  // namespace

// One line per (executed op, CTA) of the last traced call: op index, kind
// (10 + kind for the once-per-call ops), CTA, then the sp::kTracePhases stamps
// of stream.cuh in ns from the call's first stamp (-1: the CTA had no such
// phase in that op).
void Unet::write_trace() noexcept {
  const char* path = std::getenv("FLOWEDGE_PROGRAM_TRACE");
  if (trace_ == nullptr || path == nullptr) return;
  const std::size_t grid = static_cast<std::size_t>(ctx_->sm_count);
  constexpr std::size_t kPh = sp::kTracePhases;
  std::vector<unsigned long long> h(trace_kinds_.size() * grid * kPh);
  if (cudaMemcpy(h.data(), trace_, h.size() * sizeof(unsigned long long), cudaMemcpyDeviceToHost) != cudaSuccess)
    return;
  unsigned long long t0 = ~0ull;
  for (unsigned long long v : h)
    if (v != 0) t0 = std::min(t0, v);
  if (std::FILE* f = std::fopen(path, "w")) {
    for (std::size_t i = 0; i < trace_kinds_.size(); ++i) {
      if (h[(i * grid) * kPh + kPh - 1] == 0) break;  // past the last executed op
      for (std::size_t c = 0; c < grid; ++c) {
        std::fprintf(f, "%zu %d %zu", i, trace_kinds_[i], c);
        for (std::size_t ph = 0; ph < kPh; ++ph) {
          const unsigned long long v = h[(i * grid + c) * kPh + ph];
          std::fprintf(f, " %lld", v == 0 ? -1ll : static_cast<long long>(v - t0));
        }
        std::fprintf(f, "\n");
      }
    }
    std::fclose(f);
  }
}

void Unet::drop_streams() noexcept {
  for (auto& [b, pg] : progs_)
    if (pg.dev != nullptr) cudaFree(pg.dev);
  progs_.clear();
}

bool Unet::use_stream(std::size_t batch) {
  if (use_tc(batch) || batch * cfg_.horizon > static_cast<std::size_t>(sp::kMaxTok) || fo_s_.sw == nullptr)
    return false;
  auto it = progs_.find(batch);
  if (it == progs_.end()) {
    StreamProg pg;
    if (!build_stream(batch, pg)) {
      if (pg.dev != nullptr) cudaFree(pg.dev);
      pg = StreamProg{};
    }
    it = progs_.emplace(batch, pg).first;
  }
  return it->second.ok;
}

// Builds the op list of one sampling call for `batch` samples (the dataflow
// program of stream.cuh): the forward of the weight-streaming path conv by
// conv, with GroupNorm + Mish + FiLM / residual folded into the staging of the
// conv that reads them.  Two passes over the same emission code: the first
// sizes the device buffer, the second fills in its addresses.
bool Unet::build_stream(std::size_t batch, StreamProg& out) {
  const int NC = ctx_->sm_count;
  const int planes = stream_planes(bf16_weights());
  const int S = static_cast<int>(cfg_.stages);
  const int H = static_cast<int>(cfg_.horizon), A = static_cast<int>(cfg_.action_dim);
  const int G = static_cast<int>(cfg_.groups);
  const int B = static_cast<int>(batch);
  int dev_smem_max = 0;
  cudaDeviceGetAttribute(&dev_smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, ctx_->device);
  std::size_t total = 0;
  // a tensor as the convs that read it stage it, and what they wait on
  struct VT {
    sp::StageSrc src{};
    std::vector<sp::Dep> deps;
  };
  auto add_deps = [](std::vector<sp::Dep>& into, const std::vector<sp::Dep>& from) {
    for (const sp::Dep& d : from) {
      bool have = false;
      for (sp::Dep& e : into)
        if (e.ctr == d.ctr) {
          e.base = std::max(e.base, d.base);
          e.per_step = std::max(e.per_step, d.per_step);
          have = true;
        }
      if (!have) into.push_back(d);
    }
  };
  for (int pass = 0; pass < 2; ++pass) {
    const std::uintptr_t base = reinterpret_cast<std::uintptr_t>(out.dev);
    std::size_t used = 0;
    bool fits = true;
    std::size_t smem = 0;
    std::vector<std::pair<std::size_t, std::vector<int>>> tables;
    auto take = [&](std::size_t bytes) {
      used = (used + 255) & ~std::size_t(255);
      const std::size_t off = used;
      used += bytes;
      return off;
    };
    auto at = [&](std::size_t off) { return base + off; };
    // completion counters: one block, zeroed at every call (index 2 is the abort word)
    constexpr int kCtrBase = 4;
    constexpr int kMaxCtrs = 252;
    const std::size_t ctr_off = take((kCtrBase + kMaxCtrs) * sizeof(unsigned));
    int n_ctrs = 0;
    auto counter = [&]() {
      if (n_ctrs >= kMaxCtrs) fits = false;
      const int i = std::min(n_ctrs++, kMaxCtrs - 1);
      return reinterpret_cast<unsigned*>(at(ctr_off)) + kCtrBase + i;
    };
    std::vector<sp::Op> pre, step;
    std::vector<sp::Op>* cur = &pre;
    bool in_step = false;
    int next_cta = 0;  // first CTA of the next conv (rotating)
    unsigned* upd_ctr = counter();
    unsigned* film_ctr = counter();
    auto done_dep = [&](unsigned* ctr, int per) {
      return sp::Dep{ctr, static_cast<unsigned>(per), in_step ? static_cast<unsigned>(per) : 0u};
    };
    auto set_deps = [&](sp::Op& op, const std::vector<sp::Dep>& deps) {
      if (deps.size() > static_cast<std::size_t>(sp::kMaxDeps)) fits = false;
      op.ndeps = static_cast<int>(std::min<std::size_t>(deps.size(), sp::kMaxDeps));
      for (int i = 0; i < op.ndeps; ++i) op.deps[i] = deps[static_cast<std::size_t>(i)];
    };

    auto conv = [&](const ConvDev& c, const std::vector<VT*>& ins, int L_in, int L_out) {
      sp::Op op{};
      op.kind = sp::kOpConv;
      sp::ConvOp& o = op.conv;
      o.w = static_cast<const uint4*>(c.sw);
      o.planes = planes;
      o.rbs = c.s_rbs;
      o.ks = c.s_ks;
      o.ic_pad = c.ic_total;
      std::vector<sp::Dep> deps;
      int csum = 0, gn_c = 0;
      if (ins.empty() || ins.size() > 2) fits = false;
      for (std::size_t k = 0; k < ins.size() && k < 2; ++k) {
        const int C = ins[k]->src.C;
        if (C < 4 || C % 4 != 0 || ins[k]->src.kind == sp::kSrcNone) {  // also a conv that did not fit
          fits = false;
          return VT{};
        }
        o.src[k] = ins[k]->src;
        o.src[k].Cpad = (C + 63) / 64 * 64;  // the staged rows keep the activations' 64-channel padding
        csum += o.src[k].Cpad;
        add_deps(deps, ins[k]->deps);
        if (ins[k]->src.kind == sp::kSrcGn) {
          // one normalised source, first: its buffer aliases the staged rows
          if (k != 0) fits = false;
          gn_c = C;
          const int groups = ins[k]->src.groups;
          // stage_gn: a thread owns one channel quad of kGnQuads tokens
          if (groups < 1 || gn_c % groups != 0 || (gn_c / groups) % 4 != 0 || B * groups > sp::kMaxStats ||
              gn_c / 4 > sp::kThreads || sp::kThreads % (gn_c / 4) != 0 ||
              B * L_in > sp::kGnQuads * (sp::kThreads / (gn_c / 4)))
            fits = false;
        }
        if (ins[k]->src.kind == sp::kSrcRaw && ins[k]->src.phases == 2 && L_in % 2 != 0) fits = false;
      }
      if (csum != o.ic_pad || c.tap_off.empty() || c.tap_off.size() > static_cast<std::size_t>(sp::kMaxTaps) ||
          o.ic_pad % 16 != 0 || o.ks < 1 || o.rbs < 1 || c.sw == nullptr) {
        fits = false;
        return VT{};
      }
      o.samples = B;
      o.L_in = L_in;
      o.L_out = L_out;
      o.stride = c.stride;
      o.ntaps = static_cast<int>(c.tap_off.size());
      int lo = 0, hi = 0;
      for (int j = 0; j < o.ntaps && j < sp::kMaxTaps; ++j) {
        o.tap_off[j] = c.tap_off[static_cast<std::size_t>(j)];
        lo = std::min(lo, o.tap_off[j]);
        hi = std::max(hi, o.tap_off[j]);
      }
      o.halo_lo = -lo;
      o.rows = L_in + o.halo_lo + std::max(0, (L_out - 1) * o.stride + hi - (L_in - 1));
      o.T = B * L_out;
      if (o.T > sp::kMaxTok) fits = false;
      // units are taken in groups of sp::kGroupBytes (that never cross a tap
      // or a row block)
      const int G = sp::kGroupBytes / (planes * 512);
      if (o.ks % G != 0 || o.ic_pad % (16 * G) != 0) fits = false;
      const long long gpr = std::max(1, o.ks / G);
      const long long Ug = static_cast<long long>(o.rbs) * gpr;
      // CTAs the groups are split over.  With at most as many row blocks as
      // CTAs, each row block's K goes to s CTAs (s segments), s the smallest
      // factor that brings a CTA's weights down to what its ring holds or
      // the largest that keeps s * rbs CTAs (other CTAs stay free to fetch
      // the next convs' weights); a conv that still leaves a CTA more than its
      // ring goes to all CTAs.  With more row blocks than CTAs, the largest
      // divisor of the row blocks up to the CTA count (no row block split),
      // else all CTAs.
      const std::size_t row_block_bytes = static_cast<std::size_t>(o.ks) * planes * 512;
      constexpr std::size_t kRingTarget = std::size_t(4) * sp::kChunk;
      int nct = o.rbs;
      if (o.rbs <= NC) {
        int split = 1;
        while (o.rbs * (split + 1) <= NC && row_block_bytes / split > kRingTarget && split < static_cast<int>(gpr))
          ++split;
        nct = o.rbs * split;
        // still more than a ring per CTA: every CTA streams a share (row blocks
        // then meet up to two or three CTAs)
        if (row_block_bytes / split > kRingTarget && nct < NC) nct = NC;
      } else {
        nct = NC;
        for (int d = NC; d >= NC / 2; --d)
          if (o.rbs % d == 0) {
            nct = d;
            break;
          }
      }
      nct = static_cast<int>(std::min<long long>(nct, Ug));
      o.nct = nct;
      o.cta0 = next_cta;
      next_cta = (next_cta + nct) % NC;
      std::vector<int> nseg(static_cast<std::size_t>(o.rbs));
      int seg_max = 1;
      for (int rb = 0; rb < o.rbs; ++rb) {
        const long long g0 = static_cast<long long>(rb) * gpr;
        nseg[static_cast<std::size_t>(rb)] = cta_of_host(g0 + gpr - 1, Ug, nct) - cta_of_host(g0, Ug, nct) + 1;
        seg_max = std::max(seg_max, nseg[static_cast<std::size_t>(rb)]);
      }
      // row blocks one CTA's groups meet (a slot per compute warp each)
      int nslots = 1;
      for (int ci = 0; ci < nct; ++ci) {
        const long long a = (Ug * ci) / nct, b = (Ug * (ci + 1)) / nct;
        if (b > a) nslots = std::max(nslots, static_cast<int>((b - 1) / gpr - a / gpr + 1));
      }
      if (nslots > sp::kMaxSlots) fits = false;
      o.nslots = nslots;
      if (seg_max > sp::kMaxSeg) fits = false;
      o.seg_max = seg_max;
      const std::size_t poff = take(static_cast<std::size_t>(o.rbs) * seg_max * o.T * 16 * sizeof(float));
      const std::size_t noff = take(static_cast<std::size_t>(o.rbs) * sizeof(int));
      tables.emplace_back(noff, std::move(nseg));
      o.P = reinterpret_cast<float*>(at(poff));
      o.done = counter();
      // shared memory: staged input (fp16 hi / lo; a normalised source's fp32
      // values alias it), per-warp slots, then the weight ring
      const std::size_t staged = static_cast<std::size_t>(2) * (B * o.rows + 1) * (o.ic_pad + sp::kRowPad) * 2;
      // a normalised source's per-quad (double2) sums take as much as its fp32 values
      const std::size_t temp = static_cast<std::size_t>(B) * L_in * gn_c * sizeof(float);
      o.slots_off = static_cast<int>((std::max(staged, temp) + 127) & ~std::size_t(127));
      const std::size_t head = static_cast<std::size_t>(o.slots_off) +
                               static_cast<std::size_t>(sp::kComputeWarps) * nslots * 16 * o.T * sizeof(float) +
                               static_cast<std::size_t>(sp::kWarps) * nslots * sizeof(int);
      o.ring_off = static_cast<int>((head + 127) & ~std::size_t(127));
      smem = std::max(smem, static_cast<std::size_t>(o.ring_off) + sp::kMinStages * sp::kChunk);
      // as many stages as the launch's shared memory (sized in the first pass) leaves
      o.stages = pass == 0 ? sp::kMinStages
                           : static_cast<int>(std::min<std::size_t>(sp::kMaxStages, (out.smem - o.ring_off) / sp::kChunk));
      set_deps(op, deps);
      cur->push_back(op);
      const sp::Dep mine = done_dep(o.done, nct);
      // a block output is written out by its first consumer; later ones read that copy
      for (VT* in : ins)
        if (in->src.kind == sp::kSrcGn && in->src.materialize != nullptr) {
          VT m;
          m.src.kind = sp::kSrcMat;
          m.src.C = in->src.C;
          m.src.mat = in->src.materialize;
          m.deps = {mine};
          *in = m;
        }
      VT y;
      y.src.kind = sp::kSrcRaw;
      y.src.C = c.oc;
      y.src.phases = 1;
      y.src.raw[0] = sp::RawSrc{o.P, reinterpret_cast<const int*>(at(noff)), c.bias, seg_max, o.T};
      y.deps = {mine};
      return y;
    };
    // mish(GroupNorm(y)) with FiLM or a residual, as its consumer stages it
    auto gn = [&](const VT& y, const float* gamma, const float* beta, int groups, const BlockDev* film_blk,
                  const VT* res, void* materialize) {
      VT v;
      v.src.kind = sp::kSrcGn;
      v.src.C = y.src.C;
      v.src.raw[0] = y.src.raw[0];
      v.src.gamma = gamma;
      v.src.beta = beta;
      v.src.groups = groups;
      v.deps = y.deps;
      if (y.src.kind != sp::kSrcRaw || y.src.phases != 1) fits = false;
      if (film_blk != nullptr) {
        v.src.film = 1;
        v.src.film_off = film_blk->film_off;
        add_deps(v.deps, {sp::Dep{film_ctr, static_cast<unsigned>(NC), 0u}});
      }
      if (res != nullptr) {
        if (res->src.kind == sp::kSrcRaw && res->src.phases == 1) {
          v.src.res_kind = 1;
          v.src.res = res->src.raw[0];
        } else if (res->src.kind == sp::kSrcMat) {
          v.src.res_kind = 2;
          v.src.mat = res->src.mat;
        } else {
          fits = false;
        }
        if (res->src.C != v.src.C) fits = false;
        add_deps(v.deps, res->deps);
      }
      v.src.materialize = static_cast<float*>(materialize);
      return v;
    };
    auto block = [&](const BlockDev& blk, const std::vector<VT*>& in, int L, void* dst) {
      const VT y1 = conv(blk.c1, in, L, L);
      VT yr;
      if (blk.has_res) yr = conv(blk.res, in, L, L);
      VT h1 = gn(y1, blk.g1, blk.b1, G, &blk, nullptr, nullptr);
      const VT y2 = conv(blk.c2, {&h1}, L, L);
      if (!blk.has_res && in.size() != 1) fits = false;
      return gn(y2, blk.g2, blk.b2, G, nullptr, blk.has_res ? &yr : in[0], dst);
    };

    // once per call: FiLM condition part W_c * mish(cond) + b -> film_cond_
    {
      VT mc;
      mc.src.kind = sp::kSrcMat;
      mc.src.C = cond_pad_;
      mc.src.mat = static_cast<const float*>(mcond_);
      const VT yf = conv(film_, {&mc}, 1, 1);
      sp::Op op{};
      op.kind = sp::kOpReduce;
      op.reduce.y = yf.src.raw[0];
      op.reduce.M = F_;
      op.reduce.T = B;
      op.reduce.out = film_cond_;
      op.reduce.done = film_ctr;
      set_deps(op, yf.deps);
      pre.push_back(op);
    }
    // every step: the forward and the update
    cur = &step;
    in_step = true;
    std::deque<VT> keep;  // tensors referred to later (skips), at stable addresses
    std::size_t li = 0;
    int L = H;
    keep.emplace_back();
    keep.back().src.kind = sp::kSrcMat;
    keep.back().src.C = cin_pad_;
    keep.back().src.mat = static_cast<const float*>(x_in_);
    keep.back().deps = {sp::Dep{upd_ctr, 0u, 1u}};  // step s reads the input the update of step s - 1 wrote
    VT* x = &keep.back();
    std::vector<VT*> skips(static_cast<std::size_t>(S));
    for (int st = 0; st < S; ++st) {
      keep.push_back(block(down_[static_cast<std::size_t>(st)][0], {x}, L, acts_[li]));
      VT* o0 = &keep.back();
      keep.push_back(block(down_[static_cast<std::size_t>(st)][1], {o0}, L, acts_[li + 1]));
      li += 2;
      skips[static_cast<std::size_t>(st)] = x = &keep.back();
      if (st + 1 < S) {
        keep.push_back(conv(ds_[static_cast<std::size_t>(st)], {x}, L, L / 2));
        x = &keep.back();
        ++li;
        L /= 2;
      } else {
        ++li;
      }
    }
    for (int m = 0; m < 2; ++m) {
      keep.push_back(block(mid_[static_cast<std::size_t>(m)], {x}, L, acts_[li++]));
      x = &keep.back();
    }
    for (int st = 0; st + 1 < S; ++st) {
      VT* skip = skips[static_cast<std::size_t>(S - 1 - st)];
      keep.push_back(block(up_[static_cast<std::size_t>(st)][0], {x, skip}, L, acts_[li]));
      VT* o0 = &keep.back();
      keep.push_back(block(up_[static_cast<std::size_t>(st)][1], {o0}, L, acts_[li + 1]));
      VT* o1 = &keep.back();
      li += 3;
      const VT y0 = conv(us_[static_cast<std::size_t>(st)][0], {o1}, L, L);
      const VT y1 = conv(us_[static_cast<std::size_t>(st)][1], {o1}, L, L);
      keep.emplace_back();
      VT& u = keep.back();
      u.src.kind = sp::kSrcRaw;
      u.src.C = y0.src.C;
      u.src.phases = 2;
      u.src.raw[0] = y0.src.raw[0];
      u.src.raw[1] = y1.src.raw[0];
      u.deps = y0.deps;
      add_deps(u.deps, y1.deps);
      x = &u;
      L *= 2;
    }
    const VT yc = conv(fc_, {x}, H, H);
    VT hf = gn(yc, fn_g_, fn_b_, static_cast<int>(kFinalNormGroups), nullptr, nullptr, nullptr);
    const VT ye = conv(fo_s_, {&hf}, H, H);
    {
      sp::Op op{};
      op.kind = sp::kOpUpdate;
      op.update.y = ye.src.raw[0];
      op.update.cta = next_cta;  // a CTA outside the output conv's
      op.update.A = A;
      op.update.H = H;
      op.update.Cin = cin_pad_;
      op.update.samples = B;
      op.update.x_master = x_master_;
      op.update.x_in = static_cast<float*>(x_in_);
      op.update.seeds = seeds_;
      op.update.done = upd_ctr;
      set_deps(op, ye.deps);
      step.push_back(op);
    }
    // L2 prefetch chain: each conv names the next conv's weights (the last
    // conv of a step names the first conv of the next step)
    std::vector<sp::ConvOp*> convs;
    for (auto& op : pre)
      if (op.kind == sp::kOpConv) convs.push_back(&op.conv);
    const std::size_t first_step = convs.size();
    for (auto& op : step)
      if (op.kind == sp::kOpConv) convs.push_back(&op.conv);
    for (std::size_t i = 0; i < convs.size(); ++i) {
      const sp::ConvOp* nx = convs[i + 1 < convs.size() ? i + 1 : first_step];
      convs[i]->next_w = nx->w;
      convs[i]->next_units = static_cast<long long>(nx->rbs) * nx->ks;
      convs[i]->next_planes = nx->planes;
    }
    const std::size_t n_ops = pre.size() + step.size();
    const std::size_t ops_off = take(n_ops * sizeof(sp::Op));
    if (pass == 0) {
      // use all the shared memory a CTA may have: deeper rings for the smaller convs
      constexpr std::size_t kStaticSmem = 4096;  // the kernel's static shared memory (2.8 KB), with margin
      if (!fits || smem > static_cast<std::size_t>(dev_smem_max) - kStaticSmem) return false;
      smem = std::max(smem, static_cast<std::size_t>(dev_smem_max) - kStaticSmem);
      total = used;
      if (counted_malloc(&out.dev, total) != cudaSuccess) {
        cudaGetLastError();
        out.dev = nullptr;
        return false;
      }
      cudaMemset(out.dev, 0, total);
      out.smem = smem;
      continue;
    }
    std::vector<sp::Op> all(pre);
    all.insert(all.end(), step.begin(), step.end());
    char* dev = static_cast<char*>(out.dev);
    cudaMemcpy(dev + ops_off, all.data(), n_ops * sizeof(sp::Op), cudaMemcpyHostToDevice);
    for (const auto& [off, tab] : tables) cudaMemcpy(dev + off, tab.data(), tab.size() * sizeof(int), cudaMemcpyHostToDevice);
    out.ops = reinterpret_cast<const sp::Op*>(dev + ops_off);
    if (std::getenv("FLOWEDGE_PROGRAM_TRACE") != nullptr && trace_ == nullptr) {
      // stamps per (op, CTA) of a call of up to train_timesteps steps
      const std::size_t n =
          (pre.size() + cfg_.train_timesteps * step.size()) * static_cast<std::size_t>(NC) * sp::kTracePhases;
      trace_bytes_ = n * sizeof(unsigned long long);
      if (cudaMalloc(reinterpret_cast<void**>(&trace_), trace_bytes_) != cudaSuccess) {
        cudaGetLastError();
        trace_ = nullptr;
      }
      trace_kinds_.clear();
      for (const auto& op : pre) trace_kinds_.push_back(10 + op.kind);
      for (std::size_t r = 0; r < cfg_.train_timesteps; ++r)
        for (const auto& op : step) trace_kinds_.push_back(op.kind);
    }
    out.sync = reinterpret_cast<unsigned*>(dev + ctr_off);
    out.sync_words = static_cast<std::size_t>(kCtrBase + n_ctrs);
    out.n_pre = static_cast<int>(pre.size());
    out.n_step = static_cast<int>(step.size());
  }
  // the whole grid must be resident at once (cooperative launch)
  auto kernel = planes == 1 ? sp::unet_program_kernel<1> : sp::unet_program_kernel<2>;
  int per_sm = 0;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(out.smem)) !=
          cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, sp::kThreads, out.smem) != cudaSuccess ||
      per_sm < 1 || cudaDeviceSynchronize() != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  out.ok = true;
  return true;
}

bool Unet::record_stream(std::size_t batch, std::size_t steps, const void* tables, cudaStream_t st,
                         std::string& err) {
  const StreamProg& pg = progs_.at(batch);
  const int H = static_cast<int>(cfg_.horizon), A = static_cast<int>(cfg_.action_dim);
  const int n_tokens = static_cast<int>(batch) * H;
  b0_ = 0;
  launch(seeds_kernel, dim3((static_cast<unsigned>(batch) + 255) / 256), dim3(256), 0, st,
         static_cast<const std::uint64_t*>(seed0_), seeds_, static_cast<int>(batch));
  launch(prep_sample_kernel, dim3(ew_grid(static_cast<long long>(n_tokens) * cin_pad_, 256, *ctx_)), dim3(256), 0, st,
         static_cast<const float*>(in_noise_), n_tokens, A, x_master_, x_in_, cin_pad_, 0);
  launch(prep_cond_kernel, dim3(ew_grid(static_cast<long long>(batch) * cond_pad_, 256, *ctx_)), dim3(256), 0, st,
         static_cast<const float*>(in_cond_), static_cast<int>(batch), static_cast<int>(cfg_.condition_dim),
         mcond_, cond_pad_, 0);
  cudaMemsetAsync(pg.sync, 0, pg.sync_words * sizeof(unsigned), st);
  sp::Program prog{};
  prog.ops = pg.ops;
  prog.n_pre = pg.n_pre;
  prog.n_step = pg.n_step;
  prog.steps = static_cast<int>(steps);
  prog.step_t = static_cast<const int*>(tables);
  prog.scalars = reinterpret_cast<const StepScalars*>(static_cast<const char*>(tables) + stream_table_off(steps));
  prog.film_cond = film_cond_;
  prog.film_time = film_time_;
  prog.film_F = F_;
  prog.sync = pg.sync;
  prog.err = ctx_->d_err;
  prog.trace = trace_;
  if (trace_ != nullptr) cudaMemsetAsync(trace_, 0, trace_bytes_, st);
  cudaLaunchAttribute attr{};
  attr.id = cudaLaunchAttributeCooperative;
  attr.val.cooperative = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(ctx_->sm_count));
  cfg.blockDim = dim3(sp::kThreads);
  cfg.dynamicSmemBytes = pg.smem;
  cfg.stream = st;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  const cudaError_t rc = bf16_weights() ? cudaLaunchKernelEx(&cfg, sp::unet_program_kernel<1>, prog)
                                        : cudaLaunchKernelEx(&cfg, sp::unet_program_kernel<2>, prog);
  ++recorded_;
  if (rc != cudaSuccess) {
    err = std::string("program launch: ") + cudaGetErrorString(rc);
    return false;
  }
  launch(unnormalize_kernel, dim3(ew_grid(static_cast<long long>(n_tokens) * A, 256, *ctx_)), dim3(256), 0, st,
         static_cast<const float*>(x_master_), n_tokens, A, static_cast<const float*>(amin_),
         static_cast<const float*>(amax_), out_action_);
  return true;
}

int Unet::sample_device(const float* condition, const float* noise, std::size_t batch, std::size_t steps,
                        int scheduler, std::uint64_t seed, float* action, void* stream, std::string& err) noexcept {
  if (batch == 0 || steps == 0 || steps > cfg_.train_timesteps || (scheduler != 0 && scheduler != 1)) {
    err = "invalid diffusion sampling arguments";
    return 1;
  }
  if (batch > cap_) {
    err = "batch exceeds the reserved capacity (call fe_engine_reserve_batch first)";
    return 2;
  }
  cudaSetDevice(ctx_->device);
  cudaStream_t st = stream != nullptr ? static_cast<cudaStream_t>(stream) : ctx_->stream;
  const std::size_t H = cfg_.horizon, A = cfg_.action_dim;
  if (condition != in_cond_)
    cudaMemcpyAsync(in_cond_, condition, batch * cfg_.condition_dim * sizeof(float), cudaMemcpyDeviceToDevice, st);
  if (noise != in_noise_)
    cudaMemcpyAsync(in_noise_, noise, batch * H * A * sizeof(float), cudaMemcpyDeviceToDevice, st);
  cudaMemcpyAsync(seed0_, &seed, sizeof(seed), cudaMemcpyHostToDevice, st);
  const auto key = std::make_tuple(batch, steps, scheduler, use_tc(batch));
  auto it = graphs_.find(key);
  if (it == graphs_.end()) {
    // record once per (batch, steps, scheduler) on a private capture stream
    cudaStream_t cap = nullptr;
    cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking);
    cudaStreamSynchronize(st);
    cudaGraph_t graph = nullptr;
    recorded_ = 0;
    // small batches: one persistent program launch; its per-step tables are
    // uploaded before the capture
    const bool stream = use_stream(batch);
    const std::vector<StepPlan> plan = plan_steps(steps, scheduler);
    void* tables = nullptr;
    if (stream) {
      std::vector<char> host(stream_table_off(steps) + steps * sizeof(StepScalars));
      for (std::size_t i = 0; i < steps; ++i) {
        std::memcpy(host.data() + i * sizeof(int), &plan[i].timestep, sizeof(int));
        std::memcpy(host.data() + stream_table_off(steps) + i * sizeof(StepScalars), &plan[i].scalars,
                    sizeof(StepScalars));
      }
      if (counted_malloc(&tables, host.size()) != cudaSuccess ||
          cudaMemcpy(tables, host.data(), host.size(), cudaMemcpyHostToDevice) != cudaSuccess) {
        err = "device allocation of the program tables failed";
        if (tables != nullptr) cudaFree(tables);
        cudaStreamDestroy(cap);
        return 2;
      }
    }
    if (cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
      err = "cudaStreamBeginCapture failed";
      if (tables != nullptr) cudaFree(tables);
      cudaStreamDestroy(cap);
      return 2;
    }
    const bool ok = stream ? record_stream(batch, steps, tables, cap, err) : record_sample(batch, plan, cap, err);
    const cudaError_t end = cudaStreamEndCapture(cap, &graph);
    cudaStreamDestroy(cap);
    if (!ok || end != cudaSuccess || graph == nullptr) {
      if (graph != nullptr) cudaGraphDestroy(graph);
      if (tables != nullptr) cudaFree(tables);
      if (err.empty()) err = std::string("graph capture failed: ") + cudaGetErrorString(end);
      cudaGetLastError();
      return 2;
    }
    Graph g;
    const cudaError_t inst = cudaGraphInstantiate(&g.exec, graph, 0);
    cudaGraphDestroy(graph);
    if (inst != cudaSuccess) {
      err = std::string("cudaGraphInstantiate failed: ") + cudaGetErrorString(inst);
      if (tables != nullptr) cudaFree(tables);
      return 2;
    }
    g.launches = recorded_;
    g.tables = tables;
    it = graphs_.emplace(key, g).first;
  }
  if (cudaGraphLaunch(it->second.exec, st) != cudaSuccess) {
    err = "cudaGraphLaunch failed";
    return 2;
  }
  launches_ += it->second.launches;
  if (action != out_action_)
    cudaMemcpyAsync(action, out_action_, batch * H * A * sizeof(float), cudaMemcpyDeviceToDevice, st);
  return 0;
}

int Unet::sample(const float* condition, const float* noise, std::size_t batch, std::size_t steps, int scheduler,
                 std::uint64_t seed, float* action, std::string& err) noexcept {
  if (batch > cap_) {
    const int rc = reserve(batch, err);
    if (rc != 0) return rc;
  }
  cudaSetDevice(ctx_->device);
  cudaStream_t st = ctx_->stream;
  const std::size_t H = cfg_.horizon, A = cfg_.action_dim, Cd = cfg_.condition_dim;
  float* pc = pinned_;
  float* pn = pinned_ + batch * Cd;
  float* pa = pn + batch * H * A;
  std::memcpy(pc, condition, batch * Cd * sizeof(float));
  std::memcpy(pn, noise, batch * H * A * sizeof(float));
  cudaMemcpyAsync(in_cond_, pc, batch * Cd * sizeof(float), cudaMemcpyHostToDevice, st);
  cudaMemcpyAsync(in_noise_, pn, batch * H * A * sizeof(float), cudaMemcpyHostToDevice, st);
  const int rc = sample_device(in_cond_, in_noise_, batch, steps, scheduler, seed, out_action_, st, err);
  if (rc != 0) return rc;
  cudaMemcpyAsync(pa, out_action_, batch * H * A * sizeof(float), cudaMemcpyDeviceToHost, st);
  if (cudaStreamSynchronize(st) != cudaSuccess) {
    err = std::string("diffusion sampling failed on the device: ") + cudaGetErrorString(cudaGetLastError());
    return 2;
  }
  if (const int code = take_device_error(*ctx_, st); code != 0) {
    err = device_error_text(code);
    return 2;
  }
  std::memcpy(action, pa, batch * H * A * sizeof(float));
  return 0;
}

int Unet::denoise(const float* condition, const float* sample, float timestep, float* eps, std::size_t batch,
                  std::string& err) noexcept {
  if (!std::isfinite(timestep) || batch == 0) {
    err = "invalid denoise arguments";
    return 1;
  }
  if (batch > cap_) {
    const int rc = reserve(batch, err);
    if (rc != 0) return rc;
  }
  cudaSetDevice(ctx_->device);
  cudaStream_t st = ctx_->stream;
  const std::size_t H = cfg_.horizon, A = cfg_.action_dim, Cd = cfg_.condition_dim;
  const bool tc = use_tc(batch);
  const std::size_t chunk = chunk_samples(batch, tc);
  const int n_tokens = static_cast<int>(batch * H);
  float* pc = pinned_;
  float* pn = pinned_ + batch * Cd;
  std::memcpy(pc, condition, batch * Cd * sizeof(float));
  std::memcpy(pn, sample, batch * H * A * sizeof(float));
  cudaMemcpyAsync(in_cond_, pc, batch * Cd * sizeof(float), cudaMemcpyHostToDevice, st);
  cudaMemcpyAsync(in_noise_, pn, batch * H * A * sizeof(float), cudaMemcpyHostToDevice, st);
  cudaMemcpyAsync(tstep_, &timestep, sizeof(float), cudaMemcpyHostToDevice, st);
  const int td = static_cast<int>(cfg_.timestep_dim);
  temb_kernel<<<1, 128, static_cast<std::size_t>(5 * td) * sizeof(float), st>>>(tstep_, 1, td, te1_w_, te1_b_,
                                                                                 te2_w_, te2_b_, tm_row_);
  film_time_kernel<<<ew_grid(F_, 256, *ctx_), 256, 0, st>>>(tm_row_, 1, td, wt_, F_, ft_row_);
  prep_sample_kernel<<<ew_grid(static_cast<long long>(n_tokens) * cin_pad_, 256, *ctx_), 256, 0, st>>>(
      in_noise_, n_tokens, static_cast<int>(A), x_master_, x_in_, cin_pad_, tc ? 1 : 0);
  bool ok = true;
  for (b0_ = 0; ok && b0_ < batch; b0_ += chunk) {
    const std::size_t nb = std::min(chunk, batch - b0_);
    ok = record_film_cond(nb, tc, st, err) && record_forward(nb, tc, ft_row_, st, err) &&
         record_update(nb, tc, nullptr, eps_, st);
  }
  b0_ = 0;
  if (!ok) return 2;
  float* pe = pinned_;
  cudaMemcpyAsync(pe, eps_, batch * H * A * sizeof(float), cudaMemcpyDeviceToHost, st);
  if (cudaStreamSynchronize(st) != cudaSuccess) {
    err = std::string("diffusion denoise failed on the device: ") + cudaGetErrorString(cudaGetLastError());
    return 2;
  }
  if (const int code = take_device_error(*ctx_, st); code != 0) {
    err = device_error_text(code);
    return 2;
  }
  std::memcpy(eps, pe, batch * H * A * sizeof(float));
  return 0;
}

// One forward of `batch` samples (timestep 0 row of the FiLM table), run
// directly on the engine stream with a CUDA event pair around every
// tensor-core convolution.  metrics[0] = summed conv kernel ms, [1] = conv
// launches, [2] = algorithmic conv FLOPs, [3] = whole-forward ms.
int Unet::profile(std::size_t batch, double* metrics, std::string& err) noexcept {
  if (!use_tc(batch)) {
    err = "profiling covers the tensor-core path (bf16 mode, batch * horizon >= 512)";
    return 1;
  }
  if (batch > cap_) {
    err = "batch exceeds the reserved capacity";
    return 2;
  }
  cudaSetDevice(ctx_->device);
  cudaStream_t st = ctx_->stream;
  prof_events_.clear();
  prof_flops_ = 0;
  profiling_ = true;
  cudaEvent_t all0, all1;
  cudaEventCreate(&all0);
  cudaEventCreate(&all1);
  cudaEventRecord(all0, st);
  const bool ok = record_forward(batch, true, film_time_, st, err);
  cudaEventRecord(all1, st);
  profiling_ = false;
  if (!ok || cudaStreamSynchronize(st) != cudaSuccess) {
    if (err.empty()) err = "profiling forward failed";
    return 2;
  }
  double conv_ms = 0;
  for (auto& [a, b] : prof_events_) {
    float ms = 0;
    cudaEventElapsedTime(&ms, a, b);
    conv_ms += ms;
    cudaEventDestroy(a);
    cudaEventDestroy(b);
  }
  float all_ms = 0;
  cudaEventElapsedTime(&all_ms, all0, all1);
  cudaEventDestroy(all0);
  cudaEventDestroy(all1);
  metrics[0] = conv_ms;
  metrics[1] = static_cast<double>(prof_events_.size());
  metrics[2] = prof_flops_;
  metrics[3] = all_ms;
  prof_events_.clear();
  return take_device_error(*ctx_, st) == 0 ? 0 : 2;
}

}  // namespace

std::unique_ptr<UnetDevice> make_unet_device(const TensorTable& tensors, std::shared_ptr<DeviceContext> ctx,
                                             Precision precision, std::string& err) {
  auto unet = std::make_unique<Unet>(std::move(ctx), precision);
  if (!unet->load(tensors, err)) return nullptr;
  if (unet->reserve(1, err) != 0) return nullptr;
  return unet;
}

}  // namespace feb
