// CUDA-side runtime shared by the head modules: device context, counted
// allocations, a bump arena over one allocation, TMA descriptor encoding and
// the launcher of the tcgen05 GEMM.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

#include "device.h"
#include "tc_gemm.cuh"

namespace feb {

struct DeviceContext {
  int device = 0;
  cudaStream_t stream = nullptr;
  int sm_count = 0;
  int* d_err = nullptr;  // device error word written by kernels (never trapped)
  int pair_clusters = 0;  // co-resident 2-CTA clusters of the paired GroupNorm GEMM (0: unavailable)
  ~DeviceContext();
};

// cudaMalloc / cudaFree with the allocation counter.
cudaError_t counted_malloc(void** ptr, std::size_t bytes);
cudaError_t counted_host_malloc(void** ptr, std::size_t bytes);

// One device allocation carved by a bump pointer (256-byte aligned pieces).
class DeviceArena {
 public:
  DeviceArena() = default;
  DeviceArena(const DeviceArena&) = delete;
  DeviceArena& operator=(const DeviceArena&) = delete;
  ~DeviceArena();
  bool init(std::size_t bytes, std::string& err);
  void* take(std::size_t bytes);
  template <typename T>
  T* take_n(std::size_t n) {
    return static_cast<T*>(take(n * sizeof(T)));
  }
  [[nodiscard]] std::size_t used() const noexcept { return used_; }
  [[nodiscard]] std::size_t size() const noexcept { return size_; }
  // True once a take() did not fit (it returned null); callers check this
  // before launching anything on the carved buffers.
  [[nodiscard]] bool overflowed() const noexcept { return overflowed_; }
  void reset() noexcept { used_ = 0; }
  void release() noexcept;

 private:
  char* base_ = nullptr;
  std::size_t size_ = 0;
  std::size_t used_ = 0;
  bool overflowed_ = false;
};

// Sizing pass for a DeviceArena.  Every add() rounds up like take(); the
// total carries 64 KiB of slack for the rounding of takes that a plan lumps
// into one add().
class ArenaPlan {
 public:
  void add(std::size_t bytes) { total_ += (bytes + 255) & ~std::size_t(255); }
  template <typename T>
  void add_n(std::size_t n) {
    add(n * sizeof(T));
  }
  [[nodiscard]] std::size_t total() const noexcept { return total_ + (std::size_t(1) << 16); }

 private:
  std::size_t total_ = 0;
};

// --- tcgen05 GEMM launch ----------------------------------------------------

struct TcSource {
  const void* ptr = nullptr;  // bf16 [samples][length][channels]
  int channels = 0;
  int length = 0;
  int samples = 0;  // extent of the buffer (>= tile samples)
};

struct TcLaunch {
  bool fp16 = false;        // operand format of A, B and 16-bit outputs: fp16 (true) or bf16
  const void* A = nullptr;  // [M_rows][K] 16-bit, M_rows multiple of 128, K multiple of 64
  int M_rows = 0;
  int K = 0;
  TcSource src[3];
  int L = 1;          // tokens per sample in the N tile (power of two <= 256)
  int n_samples = 0;  // valid samples
  int m_valid = 0;
  std::vector<tc::Seg> segs;
  const float* bias = nullptr;
  const float* add_vec = nullptr;
  const float* add_tok = nullptr;
  int add_ld = 0;
  int act = tc::kActNone;
  bool out_f32 = false;
  bool out_accumulate = false;
  void* out = nullptr;
  long long out_ld = 0;
  int out_rps = 1, out_tmul = 1, out_tadd = 0, out_ch_off = 0;
  // fp16 output only, nonzero: the rounding remainder y - half(y) of each
  // output element is also stored, out_lo_off elements after it
  long long out_lo_off = 0;
  // plain epilogue with fp16 operands: store the 16-bit output as bf16
  bool out_bf16 = false;
  double* stats = nullptr;
  int group_ch = 0, groups = 0;
  // GroupNorm + Mish (+ FiLM or residual) applied in the epilogue; `out` is
  // then the 16-bit normalised activation (see tc::Params::gn_fuse)
  bool gn_fuse = false;
  const float* gamma = nullptr;
  const float* beta = nullptr;
  const float* film_cond = nullptr;
  const float* film_time = nullptr;
  int film_F = 0, film_off = 0, film_C = 0;
  const float* res_f32 = nullptr;
  const void* res16 = nullptr;
  float* out_twin = nullptr;
  // causal conv + SiLU epilogue on the rows < conv_rows (see
  // tc::Params::conv_w): plain fp32 GEMM, L = 1, sequences of conv_seq
  // tokens; conv_u may be null (only the fp16 copy is stored)
  const float* conv_w = nullptr;
  const float* conv_b = nullptr;
  float* conv_u = nullptr;
  __half* conv_u16 = nullptr;
  int conv_rows = 0, conv_seq = 0, conv_ld = 0;
};

cudaError_t tc_gemm(const TcLaunch& launch, DeviceContext& ctx, cudaStream_t stream, std::string& err);

// 2-D tensor map of a 16-bit row-major matrix [outer][inner] (128-byte
// swizzle, box {box_inner, box_outer}), for kernels that keep their maps in
// device memory.
bool encode_tmap_2d(CUtensorMap* map, const void* ptr, std::uint64_t inner, std::uint64_t outer,
                    std::uint32_t box_inner, std::uint32_t box_outer, bool fp16, std::string& err);

// grid size for grid-stride elementwise kernels
inline int ew_grid(long long total, int threads, const DeviceContext& ctx) {
  long long blocks = (total + threads - 1) / threads;
  const long long cap = static_cast<long long>(ctx.sm_count) * 8;
  if (blocks > cap) blocks = cap;
  return static_cast<int>(blocks < 1 ? 1 : blocks);
}

// Reads and clears the device error word; non-zero means a bounded wait in a
// kernel gave up.
int take_device_error(DeviceContext& ctx, cudaStream_t stream);
// Message for a device error word value.
const char* device_error_text(int code) noexcept;

std::vector<float> widen_f32(const HostTensor& t);

// bf16 mode: a weight is rounded to bf16 (nearest even) and stored on the
// device as fp16, which holds every bf16 value of magnitude >= 2^-17 exactly
// (smaller ones round to the fp16 subnormal grid, error < 2^-25).  fp16
// operands let the activations keep 3 more mantissa bits at the same tensor
// throughput.
std::uint16_t fp16_bits_of_bf16_rounded(float v);

// Load-time range check of a weight tensor that the device holds in fp16:
// bf16 mode stores fp16(bf16(w)); fp32 mode stores the pair hi = fp16(w),
// lo = fp16(w - hi), which is within max(2^-22 |w|, 2^-25) of w.  Fails with a
// message naming the tensor when a value cannot be stored (|w| beyond the fp16
// range 65504, or not finite), or when the stored values miss the intended
// ones (bf16(w), or w) by more than 2^-9 (bf16 mode) or 2^-16 (fp32 mode) of
// the tensor's largest magnitude; that happens only for a tensor whose values
// all lie far below 1 (under about 2^-16 in bf16 mode, 2^-9 in fp32 mode),
// where fp16's subnormal spacing 2^-24 is no longer small against them.
bool check_fp16_storable(const std::string& name, const float* w, std::size_t n, bool bf16_mode, std::string& err);

}  // namespace feb
