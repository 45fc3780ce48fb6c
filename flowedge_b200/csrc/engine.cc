// The C ABI (include/flowedge_b200.h) over the device-resident heads.
//
// Argument checks, status codes and last-error strings follow the reference
// (src/core/api/engine.cc, src/core/runtime/engine_runtime.cc); the work runs
// in UnetDevice / FlowDevice / MambaDevice.  Host C++23, no CUDA headers.
#include <algorithm>
#include <atomic>
#include <charconv>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <limits>
#include <memory>
#include <mutex>
#include <optional>
#include <string>
#include <string_view>
#include <vector>

#include "../../include/flowedge_b200.h"
#include "device.h"
#include "loader.h"

static_assert(sizeof(fe_model_digest) == 16);
static_assert(sizeof(fe_model_metadata) == 96);
static_assert(sizeof(fe_condition_metadata) == 88);
static_assert(sizeof(fe_action_metadata) == 80);

namespace {

constexpr unsigned kMaxThreads = 8;
constexpr std::size_t kMaxPrefill = 512;  // engine_runtime.cc:22
constexpr std::size_t kSnapshotHeader = 96;

// Thread-local last error; the pointed-to text stays valid until the next call
// on this thread (engine.cc:22-26).
std::string& error_text() {
  thread_local std::string text;
  return text;
}
const char*& last_error() {
  thread_local const char* ptr = "";
  return ptr;
}
void clear_error() { last_error() = ""; }
void set_error(const char* message) { last_error() = message; }
void set_error(std::string message) {
  error_text() = std::move(message);
  last_error() = error_text().c_str();
}

bool env_flag(const char* name) {
  const char* v = std::getenv(name);
  return v != nullptr && v[0] == '1' && v[1] == '\0';
}

std::optional<std::uint64_t> env_uint(const char* name) {
  const char* v = std::getenv(name);
  if (v == nullptr || v[0] == '\0') return std::nullopt;
  std::uint64_t out = 0;
  const std::string_view s(v);
  const auto [p, ec] = std::from_chars(s.data(), s.data() + s.size(), out);
  if (ec != std::errc{} || p != s.data() + s.size()) return std::nullopt;
  return out;
}

std::uint64_t nfe_for(std::size_t steps, int method) {
  const std::uint64_t per = method == FE_SOLVER_RK4 ? 4u : (method == FE_SOLVER_HEUN ? 2u : 1u);
  return steps > std::numeric_limits<std::uint64_t>::max() / per ? std::numeric_limits<std::uint64_t>::max()
                                                                  : static_cast<std::uint64_t>(steps) * per;
}

template <typename T>
void write_le(std::byte* dst, std::size_t off, T v) {
  for (std::size_t i = 0; i < sizeof(T); ++i) dst[off + i] = static_cast<std::byte>((static_cast<std::uint64_t>(v) >> (8 * i)) & 0xFF);
}
template <typename T>
T read_le(const std::byte* src, std::size_t off) {
  std::uint64_t v = 0;
  for (std::size_t i = 0; i < sizeof(T); ++i) v |= static_cast<std::uint64_t>(std::to_integer<std::uint8_t>(src[off + i])) << (8 * i);
  return static_cast<T>(v);
}

}  // namespace

struct FeWeights {
  std::shared_ptr<const feb::ModelWeights> value;
};

struct FlowRequest {
  std::uint64_t timestamp_ns = 0;
  std::uint64_t deadline_ns = 0;
  std::uint64_t generation = 0;
  std::size_t steps = 0;
  int method = FE_SOLVER_EULER;
  bool tracking = false;
};

struct FeEngine {
  std::shared_ptr<const feb::ModelWeights> weights;
  std::shared_ptr<feb::DeviceContext> ctx;
  std::unique_ptr<feb::UnetDevice> unet;
  std::unique_ptr<feb::FlowDevice> flow;
  std::unique_ptr<feb::MambaDevice> mamba;
  std::unique_ptr<feb::SmolVLADevice> smolvla;
  unsigned threads = 0;
  std::uint32_t architecture = FE_ARCH_UNKNOWN;
  std::uint64_t d_model = 0, n_layers = 0, d_inner = 0, d_state = 0, d_conv = 0;
  std::uint64_t action_dim = 0, condition_dim = 0;
  // resumable flow solve (FlowHead::SamplerState, flow.h:37-58)
  FlowRequest request;
  std::size_t next_step = 0;
  bool flow_active = false;
  bool flow_cancelled = false;
  std::atomic<std::uint64_t> latest_generation{0};
  std::vector<float> scratch;  // host staging for copies (sized at load)

  [[nodiscard]] std::size_t remaining() const { return next_step < request.steps ? request.steps - next_step : 0; }
  [[nodiscard]] std::size_t state_bytes() const {
    return mamba ? kSnapshotHeader + mamba->state_floats() * sizeof(float) : 0;
  }
};

namespace {

fe_engine* create_engine(std::shared_ptr<const feb::ModelWeights> weights, const fe_engine_options& opt) {
  if (opt.worker_threads > kMaxThreads) {
    set_error("Worker thread count must be from 0 through 8");
    return nullptr;
  }
  if (!weights) {
    set_error("Invalid null model weights");
    return nullptr;
  }
  if (env_flag("FLOWEDGE_CUDA_FORCE_HOST")) {
    set_error("FLOWEDGE_CUDA_FORCE_HOST=1 is not supported: this library has no host kernels");
    return nullptr;
  }
  try {
    auto engine = std::make_unique<FeEngine>();
    engine->weights = weights;
    engine->threads = opt.worker_threads;
    int device = opt.device;
    if (device < 0) device = static_cast<int>(env_uint("FLOWEDGE_DEVICE").value_or(0));
    std::string err;
    engine->ctx = feb::make_device_context(device, err);
    if (!engine->ctx) {
      set_error("CUDA device unavailable: " + err);
      return nullptr;
    }
    feb::Precision precision = static_cast<feb::Precision>(opt.precision);
    if (opt.precision == FE_PRECISION_MODE_AUTO) {
      const char* env = std::getenv("FLOWEDGE_PRECISION");
      if (env != nullptr && std::string_view(env) == "bf16") precision = feb::Precision::kBF16;
      else if (env != nullptr && std::string_view(env) == "fp32") precision = feb::Precision::kF32;
      else precision = weights->precision() == FE_PRECISION_F32 ? feb::Precision::kF32 : feb::Precision::kBF16;
    }
    if (precision != feb::Precision::kF32 && precision != feb::Precision::kBF16) {
      set_error("Invalid precision mode");
      return nullptr;
    }
    std::size_t max_batch = opt.max_batch;
    if (max_batch == 0) max_batch = env_uint("FLOWEDGE_MAX_BATCH").value_or(0);
    if (max_batch == 0) max_batch = std::max<std::size_t>(weights->default_max_batch(), 1);
    std::size_t max_seq = opt.max_sequence == 0 ? kMaxPrefill : opt.max_sequence;
    const feb::TensorTable& t = weights->table();
    if (t.find("dp.meta") != nullptr) {
      engine->unet = feb::make_unet_device(t, engine->ctx, precision, err);
      if (!engine->unet) {
        set_error("Diffusion Policy head failed to load: " + err);
        return nullptr;
      }
    }
    if (t.find("flow.in_proj.weight") != nullptr) {
      engine->flow = feb::make_flow_device(t, engine->ctx, precision, err);
      if (!engine->flow) {
        set_error("Flow head failed to load: " + err);
        return nullptr;
      }
    }
    // engine_runtime.cc:76-83: a SmolVLA expert is recognised by its action / state projections
    if (t.find("model.action_in_proj.weight") != nullptr && t.find("model.state_proj.weight") != nullptr) {
      engine->smolvla = feb::make_smolvla_device(t, engine->ctx, err);
      if (!engine->smolvla) {
        set_error("SmolVLA action expert failed to load: " + err);
        return nullptr;
      }
    }
    if (t.find("backbone.embeddings.weight") != nullptr) {
      engine->mamba = feb::make_mamba_device(t, engine->ctx, precision, err);
      if (!engine->mamba) {
        set_error("Mamba backbone failed to load: " + err);
        return nullptr;
      }
    }
    // architecture (engine_runtime.cc:167-176, Transformer not built)
    engine->architecture = engine->unet               ? FE_ARCH_DIFFUSION_HEAD
                           : engine->mamba && engine->flow ? FE_ARCH_MAMBA_FLOW
                           : engine->mamba            ? FE_ARCH_MAMBA
                           : engine->smolvla          ? FE_ARCH_SMOLVLA_ACTION_EXPERT
                           : engine->flow             ? FE_ARCH_FLOW_HEAD
                                                      : FE_ARCH_UNKNOWN;
    if (engine->architecture == FE_ARCH_UNKNOWN) {
      set_error("Model architecture initialization failed");
      return nullptr;
    }
    if (engine->mamba) {
      const auto& c = engine->mamba->config();
      engine->d_model = c.d_model;
      engine->n_layers = c.n_layers;
      engine->d_inner = c.d_inner;
      engine->d_state = c.d_state;
      engine->d_conv = c.d_conv;
      if (engine->mamba->reserve(std::max<std::size_t>(max_batch, 1), max_seq, err) != 0) {
        set_error("Mamba workspace: " + err);
        return nullptr;
      }
    }
    if (engine->flow) {
      engine->action_dim = engine->flow->config().action_dim;
      engine->condition_dim = engine->flow->config().cond_dim;
      if (engine->flow->reserve(std::max<std::size_t>(max_batch, 1), err) != 0) {
        set_error("Flow workspace: " + err);
        return nullptr;
      }
    }
    if (engine->smolvla) {
      // engine_runtime.cc:192-198
      const auto& c = engine->smolvla->config();
      engine->d_model = c.vlm_width;
      engine->n_layers = c.layers;
      engine->d_inner = c.expert_width;
      engine->action_dim = c.action_dim;
    }
    if (engine->unet) {
      engine->action_dim = engine->unet->config().action_dim;
      engine->condition_dim = engine->unet->config().condition_dim;
      if (engine->unet->reserve(std::max<std::size_t>(max_batch, 1), err) != 0) {
        set_error("Diffusion workspace: " + err);
        return nullptr;
      }
    }
    return engine.release();
  } catch (const std::exception&) {
    set_error("Exception during engine load (likely OOM)");
    return nullptr;
  }
}

fe_engine_options default_options(unsigned threads) {
  fe_engine_options o{};
  o.struct_size = sizeof(o);
  o.worker_threads = threads;
  o.device = -1;
  o.precision = FE_PRECISION_MODE_AUTO;
  return o;
}

std::optional<unsigned> environment_threads() {
  const char* v = std::getenv("FLOWEDGE_THREADS");
  if (v == nullptr || v[0] == '\0') return 0u;
  const auto parsed = env_uint("FLOWEDGE_THREADS");
  if (!parsed || *parsed > kMaxThreads) {
    set_error("FLOWEDGE_THREADS must be an integer from 0 through 8");
    return std::nullopt;
  }
  return static_cast<unsigned>(*parsed);
}

fe_engine* load_path(const char* path, const fe_engine_options& opt) {
  if (path == nullptr) {
    set_error("Invalid null model path");
    return nullptr;
  }
  std::string err;
  auto weights = feb::ModelWeights::open(path, err);
  if (!weights) {
    set_error(err);
    return nullptr;
  }
  return create_engine(std::move(weights), opt);
}

int flow_begin_impl(fe_engine* e, const float* condition, const float* noise, const FlowRequest& req,
                    std::size_t batch = 1, bool condition_on_device = false) {
  if (!e->flow) {
    set_error("Model has no flow head to sample from");
    return FE_STATUS_UNSUPPORTED_MODEL;
  }
  e->request = req;
  if (req.tracking) {
    std::uint64_t observed = e->latest_generation.load(std::memory_order_relaxed);
    while (observed < req.generation &&
           !e->latest_generation.compare_exchange_weak(observed, req.generation, std::memory_order_release,
                                                       std::memory_order_relaxed)) {
    }
  }
  e->flow_active = false;
  e->flow_cancelled = false;
  std::string err;
  if (e->flow->begin(condition, noise, batch, req.steps, req.method, condition_on_device, err) != 0) {
    set_error("Failed to initialize resumable flow sampler: " + err);
    return FE_STATUS_RESOURCE_EXHAUSTED;
  }
  e->next_step = 0;
  e->flow_active = true;
  return FE_STATUS_OK;
}

bool cancelled(const fe_engine* e) {
  return e->request.tracking && e->latest_generation.load(std::memory_order_acquire) > e->request.generation;
}

// FlowHead::sampler_advance, device branch (flow.cc:260-300): with generation
// tracking the solve advances one step per device call so cancellation is
// observed between steps.
int flow_advance_impl(fe_engine* e, std::size_t budget, float* action, std::size_t& remaining) {
  if (e->flow_cancelled) {
    set_error("Flow solve was cancelled by a newer generation");
    remaining = e->remaining();
    return FE_STATUS_CANCELLED;
  }
  if (!e->flow_active) {
    set_error("No resumable flow sample is active");
    return FE_STATUS_NO_ACTIVE_OPERATION;
  }
  const std::size_t todo = std::min(budget, e->remaining());
  std::size_t done = 0;
  std::string err;
  while (done < todo) {
    if (cancelled(e)) {
      e->flow_cancelled = true;
      e->flow_active = false;
      break;
    }
    const std::size_t chunk = e->request.tracking ? 1 : todo - done;
    if (e->flow->advance(e->next_step, chunk, nullptr, err) != 0) {
      set_error("Flow solve failed on the device: " + err);
      return FE_STATUS_RESOURCE_EXHAUSTED;
    }
    e->next_step += chunk;
    done += chunk;
  }
  if (e->flow->advance(e->next_step, 0, action, err) != 0) {
    set_error("Flow solve failed on the device: " + err);
    return FE_STATUS_RESOURCE_EXHAUSTED;
  }
  remaining = e->remaining();
  if (e->flow_cancelled) {
    set_error("Flow solve was cancelled by a newer generation");
    return FE_STATUS_CANCELLED;
  }
  return FE_STATUS_OK;
}

bool valid_solver(int method) { return method >= FE_SOLVER_EULER && method <= FE_SOLVER_RK4; }

int check_tokens(const fe_engine* e, const std::int32_t* tokens, std::size_t n) {
  const std::uint64_t vocab = e->mamba->config().vocab;
  for (std::size_t i = 0; i < n; ++i)
    if (tokens[i] < 0 || static_cast<std::uint64_t>(tokens[i]) >= vocab) {
      set_error("Token ID out of vocabulary range");
      return FE_STATUS_TOKEN_OUT_OF_RANGE;
    }
  return FE_STATUS_OK;
}

}  // namespace

extern "C" {

const char* fe_engine_last_error(void) { return last_error(); }

fe_engine* fe_engine_load(const char* path) {
  clear_error();
  const auto threads = environment_threads();
  if (!threads) return nullptr;
  return load_path(path, default_options(*threads));
}

fe_engine* fe_engine_load_with_threads(const char* path, unsigned worker_threads) {
  clear_error();
  return load_path(path, default_options(worker_threads));
}

fe_engine* fe_engine_load_with_options(const char* path, const fe_engine_options* options) {
  clear_error();
  if (options == nullptr || options->struct_size < sizeof(fe_engine_options)) {
    set_error("Invalid engine options");
    return nullptr;
  }
  return load_path(path, *options);
}

fe_weights* fe_weights_load(const char* path) {
  clear_error();
  if (path == nullptr) {
    set_error("Invalid null model path");
    return nullptr;
  }
  std::string err;
  auto w = feb::ModelWeights::open(path, err);
  if (!w) {
    set_error(err);
    return nullptr;
  }
  try {
    return new FeWeights{std::move(w)};
  } catch (const std::exception&) {
    set_error("Exception creating immutable weight handle (likely OOM)");
    return nullptr;
  }
}

size_t fe_weights_size_bytes(const fe_weights* weights) {
  return weights != nullptr && weights->value ? weights->value->weight_bytes() : 0;
}

void fe_weights_free(fe_weights* weights) { delete weights; }

fe_engine* fe_engine_create_from_weights(const fe_weights* weights, unsigned worker_threads) {
  clear_error();
  if (weights == nullptr) {
    set_error("Invalid null model weights");
    return nullptr;
  }
  return create_engine(weights->value, default_options(worker_threads));
}

fe_engine* fe_engine_create_from_weights_auto(const fe_weights* weights) {
  clear_error();
  if (weights == nullptr) {
    set_error("Invalid null model weights");
    return nullptr;
  }
  const auto threads = environment_threads();
  if (!threads) return nullptr;
  return create_engine(weights->value, default_options(*threads));
}

fe_engine* fe_engine_create_from_weights_with_options(const fe_weights* weights, const fe_engine_options* options) {
  clear_error();
  if (weights == nullptr || options == nullptr || options->struct_size < sizeof(fe_engine_options)) {
    set_error("Invalid arguments to fe_engine_create_from_weights_with_options");
    return nullptr;
  }
  return create_engine(weights->value, *options);
}

void fe_engine_free(fe_engine* engine) { delete engine; }

void fe_engine_dims(const fe_engine* engine, size_t* d_model, size_t* n_layers) {
  if (engine == nullptr) return;
  if (d_model != nullptr) *d_model = engine->d_model;
  if (n_layers != nullptr) *n_layers = engine->n_layers;
}

unsigned fe_engine_thread_count(const fe_engine* engine) { return engine != nullptr ? engine->threads : 0u; }

int fe_engine_cuda_resident(const fe_engine* engine) { return engine != nullptr ? 1 : 0; }

int fe_engine_model_metadata(const fe_engine* engine, fe_model_metadata* metadata) {
  clear_error();
  if (engine == nullptr || metadata == nullptr) {
    set_error("Invalid arguments to fe_engine_model_metadata");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  fe_model_metadata r{};
  r.struct_size = sizeof(r);
  r.protocol_version = FE_PROTOCOL_VERSION;
  r.architecture = engine->architecture;
  r.precision = engine->weights->precision();
  std::memcpy(r.model_digest.bytes, engine->weights->digest().data(), 16);
  r.d_model = engine->d_model;
  r.n_layers = engine->n_layers;
  r.d_inner = engine->d_inner;
  r.d_state = engine->d_state;
  r.d_conv = engine->d_conv;
  r.action_dim = engine->action_dim;
  r.condition_dim = engine->condition_dim;
  r.decode_snapshot_bytes = engine->state_bytes();
  *metadata = r;
  return FE_STATUS_OK;
}

int fe_engine_deployment_profile(const fe_engine* engine, fe_deployment_profile* profile) {
  clear_error();
  if (engine == nullptr || profile == nullptr) {
    set_error("Invalid arguments to fe_engine_deployment_profile");
    return 1;
  }
  const feb::DeploymentProfile* p = engine->weights->profile();
  if (p == nullptr) {
    set_error("Checkpoint has no deployment profile");
    return 2;
  }
  fe_deployment_profile r{};
  r.struct_size = sizeof(r);
  r.profile_version = p->profile_version;
  r.model_compatibility_version = p->model_compatibility_version;
  r.action_units = static_cast<std::uint32_t>(p->action_units);
  r.normalization_type = static_cast<std::uint32_t>(p->normalization_type);
  r.solver_default = static_cast<std::uint32_t>(p->solver_default);
  r.observation_schema_hash = p->observation_schema_hash.c_str();
  r.action_dim = p->action_dim;
  r.action_horizon = p->action_horizon;
  r.normalization_count = p->normalization_min.size();
  r.normalization_min = p->normalization_min.empty() ? nullptr : p->normalization_min.data();
  r.normalization_max = p->normalization_max.empty() ? nullptr : p->normalization_max.data();
  r.solver_min_steps = p->solver_min_steps;
  r.solver_max_steps = p->solver_max_steps;
  *profile = r;
  return 0;
}

size_t fe_engine_action_dim(const fe_engine* engine) { return engine != nullptr ? engine->action_dim : 0; }

size_t fe_engine_action_horizon(const fe_engine* engine) {
  if (engine == nullptr) return 0;
  if (engine->unet) return engine->unet->config().horizon;
  if (engine->flow) return 1;
  return engine->smolvla ? 50 : 0;  // engine_runtime.cc:322-327
}

size_t fe_engine_condition_dim(const fe_engine* engine) { return engine != nullptr ? engine->condition_dim : 0; }

int fe_engine_diffusion_metadata(const fe_engine* engine, fe_diffusion_metadata* metadata) {
  clear_error();
  if (engine == nullptr || metadata == nullptr) {
    set_error("Invalid arguments to fe_engine_diffusion_metadata");
    return 1;
  }
  if (!engine->unet) {
    set_error("Model has no Diffusion Policy head");
    return 4;
  }
  const auto& c = engine->unet->config();
  fe_diffusion_metadata r{};
  r.struct_size = sizeof(r);
  r.protocol_version = FE_PROTOCOL_VERSION;
  r.clip_sample = c.clip_sample ? 1u : 0u;
  r.action_dim = c.action_dim;
  r.condition_dim = c.condition_dim;
  r.horizon = c.horizon;
  r.action_steps = c.action_steps;
  r.observation_steps = c.observation_steps;
  r.train_timesteps = c.train_timesteps;
  r.clip_sample_range = c.clip_sample_range;
  *metadata = r;
  return 0;
}

// ---- Diffusion Policy ------------------------------------------------------

int fe_engine_sample_diffusion_batch(fe_engine* engine, const float* condition, const float* noise, size_t batch,
                                     size_t steps, int scheduler, uint64_t seed, float* action) {
  clear_error();
  if (engine == nullptr || condition == nullptr || noise == nullptr || action == nullptr || steps == 0 ||
      batch == 0) {
    set_error("Invalid arguments to fe_engine_sample_diffusion");
    return 1;
  }
  if (scheduler != FE_DIFFUSION_DDIM && scheduler != FE_DIFFUSION_DDPM) {
    set_error("Diffusion scheduler must be FE_DIFFUSION_DDIM or FE_DIFFUSION_DDPM");
    return 5;
  }
  if (!engine->unet) {
    set_error("Model has no Diffusion Policy head to sample from");
    return 4;
  }
  if (steps > engine->unet->config().train_timesteps) {
    set_error("Diffusion inference steps must be between 1 and the training timestep count");
    return 1;
  }
  std::string err;
  const int rc = engine->unet->sample(condition, noise, batch, steps, scheduler, seed, action, err);
  if (rc != 0) {
    set_error("Diffusion sampling failed: " + err);
    return rc;
  }
  return 0;
}

int fe_engine_sample_diffusion(fe_engine* engine, const float* condition, const float* noise, size_t steps,
                               int scheduler, uint64_t seed, float* action) {
  return fe_engine_sample_diffusion_batch(engine, condition, noise, 1, steps, scheduler, seed, action);
}

int fe_engine_sample_diffusion_device(fe_engine* engine, const float* condition, const float* noise, size_t batch,
                                      size_t steps, int scheduler, uint64_t seed, float* action, void* stream) {
  clear_error();
  if (engine == nullptr || condition == nullptr || noise == nullptr || action == nullptr || steps == 0 ||
      batch == 0) {
    set_error("Invalid arguments to fe_engine_sample_diffusion_device");
    return 1;
  }
  if (scheduler != FE_DIFFUSION_DDIM && scheduler != FE_DIFFUSION_DDPM) {
    set_error("Diffusion scheduler must be FE_DIFFUSION_DDIM or FE_DIFFUSION_DDPM");
    return 5;
  }
  if (!engine->unet) {
    set_error("Model has no Diffusion Policy head to sample from");
    return 4;
  }
  std::string err;
  const int rc = engine->unet->sample_device(condition, noise, batch, steps, scheduler, seed, action, stream, err);
  if (rc != 0) set_error("Diffusion sampling failed: " + err);
  return rc;
}

int fe_engine_diffusion_denoise_batch(fe_engine* engine, const float* condition, const float* normalized_sample,
                                      size_t batch, float timestep, float* predicted_noise) {
  clear_error();
  if (engine == nullptr || condition == nullptr || normalized_sample == nullptr || predicted_noise == nullptr ||
      !std::isfinite(timestep) || batch == 0) {
    set_error("Invalid arguments to fe_engine_diffusion_denoise");
    return 1;
  }
  if (!engine->unet) {
    set_error("Model has no Diffusion Policy head");
    return 4;
  }
  std::string err;
  const int rc = engine->unet->denoise(condition, normalized_sample, timestep, predicted_noise, batch, err);
  if (rc != 0) {
    set_error("Diffusion denoiser execution failed: " + err);
    return 2;
  }
  return 0;
}

int fe_engine_diffusion_denoise(fe_engine* engine, const float* condition, const float* normalized_sample,
                                float timestep, float* predicted_noise) {
  return fe_engine_diffusion_denoise_batch(engine, condition, normalized_sample, 1, timestep, predicted_noise);
}

int fe_engine_reserve_batch(fe_engine* engine, size_t max_batch) {
  clear_error();
  if (engine == nullptr || max_batch == 0) {
    set_error("Invalid arguments to fe_engine_reserve_batch");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  std::string err;
  if (engine->unet && engine->unet->reserve(max_batch, err) != 0) {
    set_error("Diffusion workspace: " + err);
    return FE_STATUS_RESOURCE_EXHAUSTED;
  }
  if (engine->flow && engine->flow->reserve(max_batch, err) != 0) {
    set_error("Flow workspace: " + err);
    return FE_STATUS_RESOURCE_EXHAUSTED;
  }
  if (engine->mamba && engine->mamba->reserve(max_batch, kMaxPrefill, err) != 0) {
    set_error("Mamba workspace: " + err);
    return FE_STATUS_RESOURCE_EXHAUSTED;
  }
  return FE_STATUS_OK;
}

// ---- flow head ---------------------------------------------------------------

int fe_engine_sample_condition(fe_engine* engine, const float* condition, const float* noise, size_t steps,
                               int method, float* action) {
  clear_error();
  if (engine == nullptr || condition == nullptr || noise == nullptr || action == nullptr || steps == 0) {
    set_error("Invalid arguments to fe_engine_sample_condition");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  if (!valid_solver(method)) {
    set_error("Invalid solver method");
    return FE_STATUS_INVALID_SOLVER;
  }
  FlowRequest req;
  req.steps = steps;
  req.method = method;
  int rc = flow_begin_impl(engine, condition, noise, req);
  if (rc != 0) return rc;
  std::size_t remaining = steps;
  return flow_advance_impl(engine, steps, action, remaining);
}

int fe_engine_sample_condition_batch(fe_engine* engine, const float* condition, const float* noise, size_t batch,
                                     size_t steps, int method, float* action) {
  clear_error();
  if (engine == nullptr || condition == nullptr || noise == nullptr || action == nullptr || steps == 0 ||
      batch == 0) {
    set_error("Invalid arguments to fe_engine_sample_condition_batch");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  if (!valid_solver(method)) {
    set_error("Invalid solver method");
    return FE_STATUS_INVALID_SOLVER;
  }
  FlowRequest req;
  req.steps = steps;
  req.method = method;
  int rc = flow_begin_impl(engine, condition, noise, req, batch);
  if (rc != 0) return rc;
  std::size_t remaining = steps;
  return flow_advance_impl(engine, steps, action, remaining);
}

int fe_engine_sample_condition_device(fe_engine* engine, const float* condition, const float* noise, size_t batch,
                                      size_t steps, int method, float* action, void* stream) {
  clear_error();
  if (engine == nullptr || condition == nullptr || noise == nullptr || action == nullptr || steps == 0 ||
      batch == 0) {
    set_error("Invalid arguments to fe_engine_sample_condition_device");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  if (!valid_solver(method)) {
    set_error("Invalid solver method");
    return FE_STATUS_INVALID_SOLVER;
  }
  if (!engine->flow) {
    set_error("Model has no flow head to sample from");
    return FE_STATUS_UNSUPPORTED_MODEL;
  }
  std::string err;
  const int rc = engine->flow->sample_device(condition, noise, batch, steps, method, action, stream, err);
  if (rc != 0) set_error("Flow sampling failed: " + err);
  return rc;
}

int fe_engine_sample_condition_static(fe_engine* engine, const float* condition, const float* noise, size_t batch,
                                      size_t steps, int method, float* action, void* stream) {
  clear_error();
  if (engine == nullptr || condition == nullptr || noise == nullptr || action == nullptr || steps == 0 ||
      batch == 0) {
    set_error("Invalid arguments to fe_engine_sample_condition_static");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  if (!valid_solver(method)) {
    set_error("Invalid solver method");
    return FE_STATUS_INVALID_SOLVER;
  }
  if (!engine->flow) {
    set_error("Model has no flow head to sample from");
    return FE_STATUS_UNSUPPORTED_MODEL;
  }
  std::string err;
  const int rc = engine->flow->sample_static(condition, noise, batch, steps, method, action, stream, err);
  if (rc != 0) set_error("Static-scratch flow sampling failed: " + err);
  return rc;
}

int fe_engine_flow_begin(fe_engine* engine, const float* condition, const float* noise, size_t steps, int method) {
  clear_error();
  if (engine == nullptr || condition == nullptr || noise == nullptr || steps == 0) {
    set_error("Invalid arguments to fe_engine_flow_begin");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  if (!valid_solver(method)) {
    set_error("Invalid solver method");
    return FE_STATUS_INVALID_SOLVER;
  }
  FlowRequest req;
  req.steps = steps;
  req.method = method;
  return flow_begin_impl(engine, condition, noise, req);
}

int fe_engine_make_condition_metadata(const fe_engine* engine, uint64_t timestamp_ns, uint64_t deadline_ns,
                                      uint64_t generation, size_t steps, int method,
                                      fe_condition_metadata* metadata) {
  clear_error();
  if (engine == nullptr || metadata == nullptr || steps == 0 || (deadline_ns != 0 && deadline_ns < timestamp_ns)) {
    set_error("Invalid arguments to fe_engine_make_condition_metadata");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  if (!valid_solver(method)) {
    set_error("Invalid solver method");
    return FE_STATUS_INVALID_SOLVER;
  }
  fe_condition_metadata r{};
  r.struct_size = sizeof(r);
  r.protocol_version = FE_PROTOCOL_VERSION;
  r.solver = static_cast<std::uint32_t>(method);
  std::memcpy(r.model_digest.bytes, engine->weights->digest().data(), 16);
  r.timestamp_ns = timestamp_ns;
  r.deadline_ns = deadline_ns;
  r.generation = generation;
  r.condition_dim = engine->condition_dim;
  r.action_dim = engine->action_dim;
  r.solver_steps = steps;
  r.remaining_nfe = nfe_for(steps, method);
  *metadata = r;
  return 0;
}

int fe_engine_flow_begin_request(fe_engine* engine, const float* condition, const float* noise,
                                 const fe_condition_metadata* metadata) {
  clear_error();
  if (engine == nullptr || condition == nullptr || noise == nullptr || metadata == nullptr ||
      metadata->struct_size < sizeof(*metadata) || metadata->protocol_version != FE_PROTOCOL_VERSION ||
      metadata->reserved != 0 || metadata->solver_steps == 0) {
    set_error("Invalid versioned flow request metadata");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  if (!valid_solver(static_cast<int>(metadata->solver))) {
    set_error("Invalid solver method in flow request metadata");
    return FE_STATUS_INVALID_SOLVER;
  }
  const int method = static_cast<int>(metadata->solver);
  if (std::memcmp(metadata->model_digest.bytes, engine->weights->digest().data(), 16) != 0 ||
      metadata->condition_dim != engine->condition_dim || metadata->action_dim != engine->action_dim ||
      metadata->remaining_nfe != nfe_for(metadata->solver_steps, method) ||
      (metadata->deadline_ns != 0 && metadata->deadline_ns < metadata->timestamp_ns)) {
    set_error("Flow request metadata is incompatible with this model");
    return FE_STATUS_INCOMPATIBLE_STATE;
  }
  FlowRequest req;
  req.timestamp_ns = metadata->timestamp_ns;
  req.deadline_ns = metadata->deadline_ns;
  req.generation = metadata->generation;
  req.steps = static_cast<std::size_t>(metadata->solver_steps);
  req.method = method;
  req.tracking = true;
  return flow_begin_impl(engine, condition, noise, req);
}

void fe_engine_cancel_before(fe_engine* engine, uint64_t generation) {
  if (engine == nullptr) return;
  std::uint64_t observed = engine->latest_generation.load(std::memory_order_relaxed);
  while (observed < generation &&
         !engine->latest_generation.compare_exchange_weak(observed, generation, std::memory_order_release,
                                                          std::memory_order_relaxed)) {
  }
}

int fe_engine_flow_advance(fe_engine* engine, size_t step_budget, float* action, size_t* steps_remaining) {
  clear_error();
  if (engine == nullptr || action == nullptr || step_budget == 0) {
    set_error("Invalid arguments to fe_engine_flow_advance");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  std::size_t remaining = 0;
  const int rc = flow_advance_impl(engine, step_budget, action, remaining);
  if ((rc == 0 || rc == FE_STATUS_CANCELLED) && steps_remaining != nullptr) *steps_remaining = remaining;
  return rc;
}

int fe_engine_flow_action_metadata(const fe_engine* engine, fe_action_metadata* metadata) {
  clear_error();
  if (engine == nullptr || metadata == nullptr) {
    set_error("Invalid arguments to fe_engine_flow_action_metadata");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  fe_action_metadata r{};
  r.struct_size = sizeof(r);
  r.protocol_version = FE_PROTOCOL_VERSION;
  r.solver = static_cast<std::uint32_t>(engine->request.method);
  r.status = engine->flow_cancelled ? FE_ACTION_CANCELLED
             : !engine->flow_active ? FE_ACTION_FAILED
             : engine->remaining() == 0 ? FE_ACTION_COMPLETE
                                        : FE_ACTION_RUNNING;
  std::memcpy(r.model_digest.bytes, engine->weights->digest().data(), 16);
  r.timestamp_ns = engine->request.timestamp_ns;
  r.deadline_ns = engine->request.deadline_ns;
  r.generation = engine->request.generation;
  r.condition_dim = engine->condition_dim;
  r.action_dim = engine->action_dim;
  r.remaining_nfe = nfe_for(engine->remaining(), engine->request.method);
  *metadata = r;
  return 0;
}

// ---- Mamba backbone ------------------------------------------------------------

int fe_engine_run_batch(fe_engine* engine, const int32_t* tokens, size_t batch, size_t seq_len, float* out) {
  clear_error();
  if (engine == nullptr || tokens == nullptr || out == nullptr || seq_len == 0 || batch == 0) {
    set_error("Invalid arguments to fe_engine_run");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  if (!engine->mamba) {
    set_error("Model has no backbone");
    return FE_STATUS_UNSUPPORTED_MODEL;
  }
  if (seq_len > kMaxPrefill) {
    set_error("Token sequence length is outside the configured prefill limit");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  if (const int rc = check_tokens(engine, tokens, batch * seq_len); rc != 0) return rc;
  std::string err;
  if (engine->mamba->forward(tokens, batch, seq_len, out, false, err) != 0) {
    set_error("Mamba forward failed: " + err);
    return FE_STATUS_RESOURCE_EXHAUSTED;
  }
  return FE_STATUS_OK;
}

int fe_engine_run(fe_engine* engine, const int32_t* tokens, size_t seq_len, float* out) {
  return fe_engine_run_batch(engine, tokens, 1, seq_len, out);
}

int fe_engine_run_device(fe_engine* engine, const int32_t* tokens, size_t batch, size_t seq_len, float* last_hidden,
                         void* stream) {
  clear_error();
  if (engine == nullptr || tokens == nullptr || last_hidden == nullptr || seq_len == 0 || batch == 0) {
    set_error("Invalid arguments to fe_engine_run_device");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  if (!engine->mamba) {
    set_error("Model has no backbone");
    return FE_STATUS_UNSUPPORTED_MODEL;
  }
  std::string err;
  if (engine->mamba->forward_device(tokens, batch, seq_len, last_hidden, stream, err) != 0) {
    set_error("Mamba forward failed: " + err);
    return FE_STATUS_RESOURCE_EXHAUSTED;
  }
  return FE_STATUS_OK;
}

int fe_engine_sample_batch(fe_engine* engine, const int32_t* tokens, size_t batch, size_t seq_len,
                           const float* noise, size_t steps, int method, float* action) {
  clear_error();
  if (engine == nullptr || tokens == nullptr || noise == nullptr || action == nullptr || seq_len == 0 ||
      steps == 0 || batch == 0) {
    set_error("Invalid arguments to fe_engine_sample");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  if (!valid_solver(method)) {
    set_error("Invalid solver method");
    return FE_STATUS_INVALID_SOLVER;
  }
  if (!engine->flow) {
    set_error("Model has no flow head to sample from");
    return FE_STATUS_UNSUPPORTED_MODEL;
  }
  if (!engine->mamba) {
    set_error("Model has no backbone for token-conditioned sampling");
    return FE_STATUS_UNSUPPORTED_MODEL;
  }
  if (engine->flow->config().cond_dim != engine->d_model) {
    set_error("Flow conditioning dimension does not match the backbone");
    return FE_STATUS_UNSUPPORTED_MODEL;
  }
  if (seq_len > kMaxPrefill) {
    set_error("Token sequence exceeds the configured prefill limit");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  if (const int rc = check_tokens(engine, tokens, batch * seq_len); rc != 0) return rc;
  std::string err;
  if (engine->mamba->forward(tokens, batch, seq_len, nullptr, true, err) != 0) {
    set_error("Mamba forward failed: " + err);
    return FE_STATUS_RESOURCE_EXHAUSTED;
  }
  FlowRequest req;
  req.steps = steps;
  req.method = method;
  int rc = flow_begin_impl(engine, engine->mamba->last_hidden_device(), noise, req, batch, true);
  if (rc != 0) return rc;
  std::size_t remaining = steps;
  return flow_advance_impl(engine, steps, action, remaining);
}

int fe_engine_sample(fe_engine* engine, const int32_t* tokens, size_t seq_len, const float* noise, size_t steps,
                     int method, float* action) {
  return fe_engine_sample_batch(engine, tokens, 1, seq_len, noise, steps, method, action);
}

int fe_engine_step(fe_engine* engine, int32_t token, float* out) {
  clear_error();
  if (engine == nullptr || out == nullptr) {
    set_error("Invalid null arguments to fe_engine_step");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  if (!engine->mamba) {
    set_error("Model has no streaming state initialized");
    return FE_STATUS_RESOURCE_EXHAUSTED;
  }
  if (token < 0 || static_cast<std::uint64_t>(token) >= engine->mamba->config().vocab) {
    set_error("Token ID out of vocabulary range");
    return FE_STATUS_TOKEN_OUT_OF_RANGE;
  }
  std::string err;
  if (engine->mamba->step(token, out, err) != 0) {
    set_error("Mamba decode step failed: " + err);
    return FE_STATUS_RESOURCE_EXHAUSTED;
  }
  return FE_STATUS_OK;
}

void fe_engine_reset(fe_engine* engine) {
  if (engine != nullptr && engine->mamba) engine->mamba->reset();
}

size_t fe_engine_decode_state_bytes(const fe_engine* engine) {
  return engine != nullptr ? engine->state_bytes() : 0;
}

// Snapshot layout (src/core/protocol/snapshot.cc:24-58): "FESNAP01", u16
// version 1, u16 header 96, u32 flags 0, u32 architecture, u32 precision,
// 16-byte digest, u64 d_model / n_layers / d_inner / d_state / d_conv,
// u64 payload bytes, u64 payload checksum, then the fp32 state.
int fe_engine_export_decode_state(const fe_engine* engine, void* destination, size_t bytes) {
  clear_error();
  if (engine == nullptr || destination == nullptr) {
    set_error("Invalid arguments to fe_engine_export_decode_state");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  const std::size_t required = engine->state_bytes();
  if (required != 0 && bytes < required) {
    set_error("Decode snapshot destination is too small");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  if (!engine->mamba) {
    set_error("Model has no streaming decode state");
    return FE_STATUS_STATE_UNAVAILABLE;
  }
  std::vector<float> state(engine->mamba->state_floats());
  std::string err;
  if (const_cast<fe_engine*>(engine)->mamba->read_state(state.data(), err) != 0) {
    set_error("Decode state read failed: " + err);
    return FE_STATUS_RESOURCE_EXHAUSTED;
  }
  auto* dst = static_cast<std::byte*>(destination);
  std::memset(dst, 0, required);
  std::memcpy(dst, "FESNAP01", 8);
  write_le<std::uint16_t>(dst, 8, 1);
  write_le<std::uint16_t>(dst, 10, static_cast<std::uint16_t>(kSnapshotHeader));
  write_le<std::uint32_t>(dst, 12, 0);
  write_le<std::uint32_t>(dst, 16, engine->architecture);
  write_le<std::uint32_t>(dst, 20, engine->weights->precision());
  std::memcpy(dst + 24, engine->weights->digest().data(), 16);
  write_le<std::uint64_t>(dst, 40, engine->d_model);
  write_le<std::uint64_t>(dst, 48, engine->n_layers);
  write_le<std::uint64_t>(dst, 56, engine->d_inner);
  write_le<std::uint64_t>(dst, 64, engine->d_state);
  write_le<std::uint64_t>(dst, 72, engine->d_conv);
  const std::size_t payload = state.size() * sizeof(float);
  write_le<std::uint64_t>(dst, 80, payload);
  const feb::Digest check = feb::fingerprint_bytes(state.data(), payload);
  std::uint64_t checksum = 0;
  for (int i = 0; i < 8; ++i) checksum |= static_cast<std::uint64_t>(check[static_cast<std::size_t>(i)]) << (8 * i);
  write_le<std::uint64_t>(dst, 88, checksum);
  std::memcpy(dst + kSnapshotHeader, state.data(), payload);
  return FE_STATUS_OK;
}

int fe_engine_import_decode_state(fe_engine* engine, const void* source, size_t bytes) {
  clear_error();
  if (engine == nullptr || source == nullptr) {
    set_error("Invalid arguments to fe_engine_import_decode_state");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  const std::size_t required = engine->state_bytes();
  if (required != 0 && bytes != required) {
    set_error(bytes < required ? "Decode snapshot source is truncated" : "Decode snapshot source size is incompatible");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  if (!engine->mamba) {
    set_error("Model has no streaming decode state");
    return FE_STATUS_STATE_UNAVAILABLE;
  }
  const auto* src = static_cast<const std::byte*>(source);
  if (std::memcmp(src, "FESNAP01", 8) != 0) {
    set_error("Decode snapshot magic is invalid");
    return FE_STATUS_CORRUPT_STATE;
  }
  if (read_le<std::uint16_t>(src, 8) != 1 || read_le<std::uint16_t>(src, 10) != kSnapshotHeader) {
    set_error("Decode snapshot version is unsupported");
    return FE_STATUS_INCOMPATIBLE_STATE;
  }
  if (read_le<std::uint32_t>(src, 12) != 0) {
    set_error("Decode snapshot header flags are invalid");
    return FE_STATUS_CORRUPT_STATE;
  }
  const std::size_t payload = engine->mamba->state_floats() * sizeof(float);
  if (read_le<std::uint64_t>(src, 80) != payload) {
    set_error("Decode snapshot size is incompatible or truncated");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  const bool compatible = read_le<std::uint32_t>(src, 16) == engine->architecture &&
                          read_le<std::uint32_t>(src, 20) == engine->weights->precision() &&
                          std::memcmp(src + 24, engine->weights->digest().data(), 16) == 0 &&
                          read_le<std::uint64_t>(src, 40) == engine->d_model &&
                          read_le<std::uint64_t>(src, 48) == engine->n_layers &&
                          read_le<std::uint64_t>(src, 56) == engine->d_inner &&
                          read_le<std::uint64_t>(src, 64) == engine->d_state &&
                          read_le<std::uint64_t>(src, 72) == engine->d_conv;
  if (!compatible) {
    set_error("Decode snapshot belongs to an incompatible model");
    return FE_STATUS_INCOMPATIBLE_STATE;
  }
  const feb::Digest check = feb::fingerprint_bytes(src + kSnapshotHeader, payload);
  std::uint64_t checksum = 0;
  for (int i = 0; i < 8; ++i) checksum |= static_cast<std::uint64_t>(check[static_cast<std::size_t>(i)]) << (8 * i);
  if (read_le<std::uint64_t>(src, 88) != checksum) {
    set_error("Decode snapshot checksum mismatch");
    return FE_STATUS_CORRUPT_STATE;
  }
  std::vector<float> state(engine->mamba->state_floats());
  std::memcpy(state.data(), src + kSnapshotHeader, payload);
  std::string err;
  if (engine->mamba->write_state(state.data(), err) != 0) {
    set_error("Decode state write failed: " + err);
    return FE_STATUS_RESOURCE_EXHAUSTED;
  }
  return FE_STATUS_OK;
}

// ---- families this build does not implement ------------------------------------

int fe_engine_run_embeddings(fe_engine* engine, const float* embeddings, size_t seq_len, float* out) {
  clear_error();
  if (engine == nullptr || embeddings == nullptr || out == nullptr || seq_len == 0) {
    set_error("Invalid arguments to fe_engine_run_embeddings");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  set_error("Model has no Transformer backbone for external embeddings");
  return FE_STATUS_UNSUPPORTED_MODEL;
}

int fe_engine_run_embeddings_masked(fe_engine* engine, const float* embeddings, const uint8_t* attention_mask,
                                    size_t seq_len, float* out) {
  clear_error();
  if (engine == nullptr || embeddings == nullptr || attention_mask == nullptr || out == nullptr || seq_len == 0) {
    set_error("Invalid arguments to fe_engine_run_embeddings_masked");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  set_error("Model has no Transformer backbone for external embeddings");
  return FE_STATUS_UNSUPPORTED_MODEL;
}

int fe_engine_smolvla_embed_suffix(fe_engine* engine, const float* noisy_actions, size_t chunk_size, float timestep,
                                   float* out) {
  clear_error();
  if (engine == nullptr || noisy_actions == nullptr || out == nullptr || chunk_size == 0 ||
      !std::isfinite(timestep)) {
    set_error("Invalid arguments to fe_engine_smolvla_embed_suffix");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  if (!engine->smolvla) {
    set_error("Model has no SmolVLA action-expert projection boundary");
    return FE_STATUS_UNSUPPORTED_MODEL;
  }
  std::string err;
  const int rc = engine->smolvla->embed_suffix(noisy_actions, chunk_size, timestep, out, err);
  if (rc != 0) set_error(err);
  return rc;
}

int fe_engine_smolvla_run_expert(fe_engine* engine, const float* suffix, size_t chunk_size,
                                 const float* prefix_keys, const float* prefix_values, const uint8_t* prefix_mask,
                                 size_t prefix_length, float* out) {
  clear_error();
  if (engine == nullptr || suffix == nullptr || chunk_size == 0 || prefix_keys == nullptr ||
      prefix_values == nullptr || prefix_mask == nullptr || prefix_length == 0 || out == nullptr) {
    set_error("Invalid arguments to fe_engine_smolvla_run_expert");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  if (!engine->smolvla) {
    set_error("Model has no SmolVLA action expert");
    return FE_STATUS_UNSUPPORTED_MODEL;
  }
  std::string err;
  const int rc = engine->smolvla->run_expert(suffix, chunk_size, prefix_keys, prefix_values, prefix_mask,
                                             prefix_length, out, err);
  if (rc != 0) set_error(err);
  return rc;
}

int fe_engine_smolvla_project_actions(fe_engine* engine, const float* hidden, size_t chunk_size, float* out) {
  clear_error();
  if (engine == nullptr || hidden == nullptr || chunk_size == 0 || out == nullptr) {
    set_error("Invalid arguments to fe_engine_smolvla_project_actions");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  if (!engine->smolvla) {
    set_error("Model has no SmolVLA action expert");
    return FE_STATUS_UNSUPPORTED_MODEL;
  }
  std::string err;
  const int rc = engine->smolvla->project_actions(hidden, chunk_size, out, err);
  if (rc != 0) set_error(err);
  return rc;
}

int fe_engine_smolvla_denoise(fe_engine* engine, const float* noisy_actions, size_t chunk_size, float timestep,
                              const float* prefix_keys, const float* prefix_values, const uint8_t* prefix_mask,
                              size_t prefix_length, float* out) {
  clear_error();
  if (engine == nullptr || noisy_actions == nullptr || chunk_size == 0 || !std::isfinite(timestep) ||
      prefix_keys == nullptr || prefix_values == nullptr || prefix_mask == nullptr || prefix_length == 0 ||
      out == nullptr) {
    set_error("Invalid arguments to fe_engine_smolvla_denoise");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  if (!engine->smolvla) {
    set_error("Model has no SmolVLA action expert");
    return FE_STATUS_UNSUPPORTED_MODEL;
  }
  std::string err;
  const int rc = engine->smolvla->denoise(noisy_actions, chunk_size, timestep, prefix_keys, prefix_values,
                                          prefix_mask, prefix_length, out, err);
  if (rc != 0) set_error(err);
  return rc;
}

int fe_engine_smolvla_sample(fe_engine* engine, const float* initial_noise, size_t chunk_size, size_t steps,
                             const float* prefix_keys, const float* prefix_values, const uint8_t* prefix_mask,
                             size_t prefix_length, float* out) {
  clear_error();
  if (engine == nullptr || initial_noise == nullptr || chunk_size == 0 || steps == 0 || prefix_keys == nullptr ||
      prefix_values == nullptr || prefix_mask == nullptr || prefix_length == 0 || out == nullptr) {
    set_error("Invalid arguments to fe_engine_smolvla_sample");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  if (!engine->smolvla) {
    set_error("Model has no SmolVLA action expert");
    return FE_STATUS_UNSUPPORTED_MODEL;
  }
  std::string err;
  // `out` may alias `initial_noise` (engine.h:187-193): the noise is copied to the device first
  const int rc = engine->smolvla->sample(initial_noise, 1, chunk_size, steps, prefix_keys, prefix_values,
                                         prefix_mask, prefix_length, true, out, false, nullptr, err);
  if (rc != 0) set_error(err);
  return rc;
}

int fe_engine_smolvla_sample_batch(fe_engine* engine, const float* initial_noise, size_t batch, size_t chunk_size,
                                   size_t steps, const float* prefix_keys, const float* prefix_values,
                                   const uint8_t* prefix_mask, size_t prefix_length, int shared_prefix, float* out) {
  clear_error();
  if (engine == nullptr || initial_noise == nullptr || batch == 0 || chunk_size == 0 || steps == 0 ||
      prefix_keys == nullptr || prefix_values == nullptr || prefix_mask == nullptr || prefix_length == 0 ||
      out == nullptr) {
    set_error("Invalid arguments to fe_engine_smolvla_sample_batch");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  if (!engine->smolvla) {
    set_error("Model has no SmolVLA action expert");
    return FE_STATUS_UNSUPPORTED_MODEL;
  }
  std::string err;
  const int rc = engine->smolvla->sample(initial_noise, batch, chunk_size, steps, prefix_keys, prefix_values,
                                         prefix_mask, prefix_length, shared_prefix != 0, out, false, nullptr, err);
  if (rc != 0) set_error(err);
  return rc;
}

int fe_engine_smolvla_sample_device(fe_engine* engine, const float* initial_noise, size_t batch, size_t chunk_size,
                                    size_t steps, const float* prefix_keys, const float* prefix_values,
                                    const uint8_t* prefix_mask, size_t prefix_length, int shared_prefix, float* out,
                                    void* stream) {
  clear_error();
  if (engine == nullptr || initial_noise == nullptr || batch == 0 || chunk_size == 0 || steps == 0 ||
      prefix_keys == nullptr || prefix_values == nullptr || prefix_mask == nullptr || prefix_length == 0 ||
      out == nullptr) {
    set_error("Invalid arguments to fe_engine_smolvla_sample_device");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  if (!engine->smolvla) {
    set_error("Model has no SmolVLA action expert");
    return FE_STATUS_UNSUPPORTED_MODEL;
  }
  std::string err;
  const int rc = engine->smolvla->sample(initial_noise, batch, chunk_size, steps, prefix_keys, prefix_values,
                                         prefix_mask, prefix_length, shared_prefix != 0, out, true, stream, err);
  if (rc != 0) set_error(err);
  return rc;
}

int fe_engine_smolvla_reserve(fe_engine* engine, size_t batch, size_t chunk_size, size_t prefix_length,
                              int shared_prefix) {
  clear_error();
  if (engine == nullptr || batch == 0 || chunk_size == 0 || prefix_length == 0) {
    set_error("Invalid arguments to fe_engine_smolvla_reserve");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  if (!engine->smolvla) {
    set_error("Model has no SmolVLA action expert");
    return FE_STATUS_UNSUPPORTED_MODEL;
  }
  std::string err;
  if (engine->smolvla->reserve(batch, chunk_size, prefix_length, shared_prefix != 0, err) != 0) {
    set_error("SmolVLA workspace: " + err);
    return FE_STATUS_RESOURCE_EXHAUSTED;
  }
  return FE_STATUS_OK;
}

// ---- counters ---------------------------------------------------------------------

uint64_t fe_device_malloc_count(void) { return feb::device_malloc_count(); }
uint64_t fe_host_malloc_count(void) { return feb::host_malloc_count(); }

int fe_engine_profile_diffusion(fe_engine* engine, size_t batch, double* metrics) {
  clear_error();
  if (engine == nullptr || metrics == nullptr || batch == 0) {
    set_error("Invalid arguments to fe_engine_profile_diffusion");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  if (!engine->unet) {
    set_error("Model has no Diffusion Policy head");
    return FE_STATUS_UNSUPPORTED_MODEL;
  }
  std::string err;
  const int rc = engine->unet->profile(batch, metrics, err);
  if (rc != 0) set_error("Diffusion profiling failed: " + err);
  return rc;
}

int fe_engine_synchronize(fe_engine* engine) {
  clear_error();
  if (engine == nullptr) {
    set_error("Invalid null engine");
    return FE_STATUS_INVALID_ARGUMENT;
  }
  if (feb::synchronize_context(*engine->ctx) != 0) {
    set_error("Device work failed");
    return FE_STATUS_RESOURCE_EXHAUSTED;
  }
  return FE_STATUS_OK;
}

uint64_t fe_engine_kernel_launches(const fe_engine* engine) {
  if (engine == nullptr) return 0;
  return (engine->unet ? engine->unet->kernel_launches() : 0) +
         (engine->smolvla ? engine->smolvla->kernel_launches() : 0);
}

}  // extern "C"
