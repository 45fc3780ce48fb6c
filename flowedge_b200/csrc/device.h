// Host-side interfaces of the device-resident heads.  No CUDA types appear
// here, so the C++23 runtime (engine.cc) and the CUDA translation units share
// it.  All device memory of a head is taken from one allocation made at load
// (weights) and one made by reserve() (workspace for a batch capacity); no
// call after that allocates.
#pragma once

#include <array>
#include <atomic>
#include <cstddef>
#include <cstdint>
#include <memory>
#include <string>
#include <string_view>
#include <vector>

namespace feb {

enum class DType : std::uint8_t { F32 = 0, BF16 = 1 };

struct HostTensor {
  std::string name;
  DType dtype{};
  int ndim{};
  std::array<std::size_t, 4> shape{};
  const void* data{};
  std::size_t bytes{};
  [[nodiscard]] std::size_t numel() const noexcept {
    std::size_t n = 1;
    for (int i = 0; i < ndim; ++i) n *= shape[static_cast<std::size_t>(i)];
    return n;
  }
};

struct TensorTable {
  std::vector<HostTensor> tensors;
  [[nodiscard]] const HostTensor* find(std::string_view name) const noexcept {
    for (const auto& t : tensors)
      if (t.name == name) return &t;
    return nullptr;
  }
};

// Arithmetic of the GEMM / conv weights on the device.
enum class Precision : int { kAuto = 0, kF32 = 1, kBF16 = 2 };

// Process-wide counters of device and pinned-host allocations made by this
// library (asserted flat after warmup by the tests).
std::uint64_t device_malloc_count() noexcept;
std::uint64_t host_malloc_count() noexcept;

// Opaque per-engine device context: device index, one CUDA stream, SM count.
struct DeviceContext;
std::shared_ptr<DeviceContext> make_device_context(int device, std::string& err);
int context_device(const DeviceContext& ctx) noexcept;
// Waits for all work on the context's stream; non-zero on a device error.
int synchronize_context(DeviceContext& ctx) noexcept;

struct DiffusionConfig {
  std::size_t action_dim{}, horizon{}, action_steps{}, observation_steps{}, condition_dim{};
  std::size_t stages{}, kernel{}, groups{}, timestep_dim{}, train_timesteps{};
  bool clip_sample{};
  float clip_sample_range{};
  std::vector<std::size_t> dims;
};

class UnetDevice {
 public:
  virtual ~UnetDevice() = default;
  [[nodiscard]] virtual const DiffusionConfig& config() const noexcept = 0;
  [[nodiscard]] virtual Precision precision() const noexcept = 0;
  [[nodiscard]] virtual std::size_t capacity() const noexcept = 0;
  virtual int reserve(std::size_t batch, std::string& err) noexcept = 0;
  // Host buffers; synchronous.  condition [B][C], sample/noise [B][H][A].
  virtual int denoise(const float* condition, const float* sample, float timestep, float* eps, std::size_t batch,
                      std::string& err) noexcept = 0;
  virtual int sample(const float* condition, const float* noise, std::size_t batch, std::size_t steps,
                     int scheduler, std::uint64_t seed, float* action, std::string& err) noexcept = 0;
  // Device buffers; asynchronous on `stream` (cudaStream_t, null = the head's stream).
  virtual int sample_device(const float* condition, const float* noise, std::size_t batch, std::size_t steps,
                            int scheduler, std::uint64_t seed, float* action, void* stream,
                            std::string& err) noexcept = 0;
  [[nodiscard]] virtual std::uint64_t kernel_launches() const noexcept = 0;
  // One forward with CUDA events around each tensor-core conv (see unet.cu).
  virtual int profile(std::size_t batch, double* metrics, std::string& err) noexcept = 0;
};

std::unique_ptr<UnetDevice> make_unet_device(const TensorTable& tensors, std::shared_ptr<DeviceContext> ctx,
                                             Precision precision, std::string& err);

struct FlowConfig {
  std::size_t action_dim{}, cond_dim{}, hidden{}, time_dim{}, mlp_layers{};
};

class FlowDevice {
 public:
  virtual ~FlowDevice() = default;
  [[nodiscard]] virtual const FlowConfig& config() const noexcept = 0;
  [[nodiscard]] virtual std::size_t capacity() const noexcept = 0;
  virtual int reserve(std::size_t batch, std::string& err) noexcept = 0;
  // Resumable solve over `batch` rows held on the device between calls.
  virtual int begin(const float* condition, const float* x0, std::size_t batch, std::size_t steps, int method,
                    bool condition_on_device, std::string& err) noexcept = 0;
  // Runs up to `budget` ODE steps starting at step `first`; copies x to `out`.
  virtual int advance(std::size_t first, std::size_t count, float* out, std::string& err) noexcept = 0;
  virtual int sample_device(const float* condition, const float* x0, std::size_t batch, std::size_t steps,
                            int method, float* out, void* stream, std::string& err) noexcept = 0;
  // As sample_device, but every scratch buffer lives in a fixed static
  // device array (no allocation, no use of the reserved workspace).
  virtual int sample_static(const float* condition, const float* x0, std::size_t batch, std::size_t steps, int method,
                            float* out, void* stream, std::string& err) noexcept = 0;
};

std::unique_ptr<FlowDevice> make_flow_device(const TensorTable& tensors, std::shared_ptr<DeviceContext> ctx,
                                             Precision precision, std::string& err);

struct MambaConfig {
  std::size_t vocab{}, d_model{}, n_layers{}, d_inner{}, d_state{}, d_conv{}, dt_rank{};
};

class MambaDevice {
 public:
  virtual ~MambaDevice() = default;
  [[nodiscard]] virtual const MambaConfig& config() const noexcept = 0;
  [[nodiscard]] virtual std::size_t capacity() const noexcept = 0;
  virtual int reserve(std::size_t batch, std::size_t max_len, std::string& err) noexcept = 0;
  // tokens [B][L] -> hidden [B][L][d_model] (host) ; `last_only` copies only
  // the last position of each sequence.
  virtual int forward(const std::int32_t* tokens, std::size_t batch, std::size_t len, float* hidden, bool last_only,
                      std::string& err) noexcept = 0;
  // Device pointer to the last-position hidden states of the latest forward.
  [[nodiscard]] virtual const float* last_hidden_device() const noexcept = 0;
  virtual int forward_device(const std::int32_t* tokens, std::size_t batch, std::size_t len, float* last_hidden,
                             void* stream, std::string& err) noexcept = 0;
  // Streaming decode: state lives on the device; snapshot copies it out / in.
  virtual int step(std::int32_t token, float* out, std::string& err) noexcept = 0;
  virtual void reset() noexcept = 0;
  [[nodiscard]] virtual std::size_t state_floats() const noexcept = 0;
  virtual int read_state(float* dst, std::string& err) noexcept = 0;
  virtual int write_state(const float* src, std::string& err) noexcept = 0;
};

std::unique_ptr<MambaDevice> make_mamba_device(const TensorTable& tensors, std::shared_ptr<DeviceContext> ctx,
                                               Precision precision, std::string& err);

struct SmolVLAConfig {
  std::size_t expert_width{}, action_dim{}, vlm_width{}, state_dim{}, layers{};
  std::size_t heads{}, kv_heads{}, head_width{}, mlp_width{}, cache_width{};
};

// SmolVLA-shaped flow action expert (smolvla_action_expert.h:31-124).  The
// batch-one entries mirror the reference's; sample() also takes a batch of
// independent chunks with per-sample or shared prefix caches.
class SmolVLADevice {
 public:
  virtual ~SmolVLADevice() = default;
  [[nodiscard]] virtual const SmolVLAConfig& config() const noexcept = 0;
  // Host buffers, synchronous.  Return 0, or the reference runtime's codes:
  // 1 for sizes outside the limits, 3 when the expert could not run (an
  // invalid mask), 2 for device failures.
  virtual int embed_suffix(const float* noisy, std::size_t chunk, float timestep, float* out,
                           std::string& err) noexcept = 0;
  virtual int run_expert(const float* suffix, std::size_t chunk, const float* keys, const float* values,
                         const std::uint8_t* mask, std::size_t prefix, float* out, std::string& err) noexcept = 0;
  virtual int project_actions(const float* hidden, std::size_t chunk, float* out, std::string& err) noexcept = 0;
  virtual int denoise(const float* noisy, std::size_t chunk, float timestep, const float* keys, const float* values,
                      const std::uint8_t* mask, std::size_t prefix, float* out, std::string& err) noexcept = 0;
  // noise / out [batch][chunk][action_dim]; keys / values [batch or 1][layers][prefix][cache_width];
  // mask [batch or 1][prefix] (1 = shared_prefix).  `on_device`: every pointer is a device
  // pointer and the work is enqueued on `stream` without a final synchronisation.
  virtual int sample(const float* noise, std::size_t batch, std::size_t chunk, std::size_t steps, const float* keys,
                     const float* values, const std::uint8_t* mask, std::size_t prefix, bool shared_prefix,
                     float* out, bool on_device, void* stream, std::string& err) noexcept = 0;
  // Workspace for `batch` chunks of `chunk` tokens and prefixes of `prefix` slots.
  virtual int reserve(std::size_t batch, std::size_t chunk, std::size_t prefix, bool shared_prefix,
                      std::string& err) noexcept = 0;
  [[nodiscard]] virtual std::uint64_t kernel_launches() const noexcept = 0;
};

std::unique_ptr<SmolVLADevice> make_smolvla_device(const TensorTable& tensors, std::shared_ptr<DeviceContext> ctx,
                                                   std::string& err);

}  // namespace feb
