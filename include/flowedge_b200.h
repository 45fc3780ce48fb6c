/*
 * flowedge_b200 - B200 (sm_100a) implementation of FlowEdge's policy-sampling
 * hot path behind FlowEdge's own C ABI.
 *
 * Part 1 declares the reference ABI unchanged: same names, argument meaning,
 * status codes, struct layouts and error behaviour.  Each declaration cites
 * the reference declaration it replaces (paths inside the FlowEdge repository:
 * src/core/api/engine.h and src/core/protocol/contracts.h).  A program built
 * against the reference header links against libflowedge_b200.so unchanged.
 *
 * Part 2 adds what the reference has no equivalent for: batched entry points
 * (the reference is batch-1 only), device-pointer entry points, load options,
 * capacity reservation and allocation / launch counters.
 *
 * All work runs on a B200; there is no CPU fallback.  Loading fails with a
 * message when no sm_100 device is present.
 */
#ifndef FLOWEDGE_B200_H
#define FLOWEDGE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* ------------------------------------------------------------------------- */
/* contracts (src/core/protocol/contracts.h:11-121)                           */

enum { FE_PROTOCOL_VERSION = 1, FE_MODEL_DIGEST_BYTES = 16 };

enum {
  FE_ARCH_UNKNOWN = 0,
  FE_ARCH_MAMBA = 1,
  FE_ARCH_FLOW_HEAD = 2,
  FE_ARCH_MAMBA_FLOW = 3,
  FE_ARCH_DIFFUSION_HEAD = 4,
  FE_ARCH_TRANSFORMER = 5,
  FE_ARCH_TRANSFORMER_FLOW = 6,
  FE_ARCH_SMOLVLA_ACTION_EXPERT = 7,
};

enum { FE_PRECISION_UNKNOWN = 0, FE_PRECISION_F32 = 1, FE_PRECISION_BF16 = 2, FE_PRECISION_MIXED = 3 };

enum { FE_ACTION_RUNNING = 0, FE_ACTION_COMPLETE = 1, FE_ACTION_CANCELLED = 2, FE_ACTION_FAILED = 3 };

enum { FE_ACTION_UNITS_NORMALIZED = 0, FE_ACTION_UNITS_PHYSICAL = 1 };

enum { FE_NORMALIZATION_NONE = 0, FE_NORMALIZATION_MINMAX = 1 };

enum { FE_PROFILE_SOLVER_EULER = 0, FE_PROFILE_SOLVER_HEUN = 1, FE_PROFILE_SOLVER_RK4 = 2 };

typedef struct fe_model_digest {
  uint8_t bytes[FE_MODEL_DIGEST_BYTES];
} fe_model_digest;

typedef struct fe_model_metadata {
  uint32_t struct_size;
  uint32_t protocol_version;
  uint32_t architecture;
  uint32_t precision;
  fe_model_digest model_digest;
  uint64_t d_model;
  uint64_t n_layers;
  uint64_t d_inner;
  uint64_t d_state;
  uint64_t d_conv;
  uint64_t action_dim;
  uint64_t condition_dim;
  uint64_t decode_snapshot_bytes;
} fe_model_metadata;

typedef struct fe_deployment_profile {
  uint32_t struct_size;
  uint32_t profile_version;
  uint32_t model_compatibility_version;
  uint32_t action_units;
  uint32_t normalization_type;
  uint32_t solver_default;
  uint32_t reserved;
  const char* observation_schema_hash;
  const float* normalization_min;
  const float* normalization_max;
  uint64_t action_dim;
  uint64_t action_horizon;
  uint64_t normalization_count;
  uint64_t solver_min_steps;
  uint64_t solver_max_steps;
} fe_deployment_profile;

typedef struct fe_condition_metadata {
  uint32_t struct_size;
  uint32_t protocol_version;
  uint32_t solver;
  uint32_t reserved;
  fe_model_digest model_digest;
  uint64_t timestamp_ns;
  uint64_t deadline_ns;
  uint64_t generation;
  uint64_t condition_dim;
  uint64_t action_dim;
  uint64_t solver_steps;
  uint64_t remaining_nfe;
} fe_condition_metadata;

typedef struct fe_action_metadata {
  uint32_t struct_size;
  uint32_t protocol_version;
  uint32_t solver;
  uint32_t status;
  fe_model_digest model_digest;
  uint64_t timestamp_ns;
  uint64_t deadline_ns;
  uint64_t generation;
  uint64_t condition_dim;
  uint64_t action_dim;
  uint64_t remaining_nfe;
} fe_action_metadata;

/* ------------------------------------------------------------------------- */
/* Part 1: the reference C ABI (src/core/api/engine.h)                        */

typedef struct FeEngine fe_engine;
typedef struct FeWeights fe_weights;

enum { FE_SOLVER_EULER = 0, FE_SOLVER_HEUN = 1, FE_SOLVER_RK4 = 2 }; /* engine.h:16-21 */

enum { FE_DIFFUSION_DDIM = 0, FE_DIFFUSION_DDPM = 1 }; /* engine.h:23-27 */

typedef struct fe_diffusion_metadata { /* engine.h:29-44 */
  uint32_t struct_size;
  uint32_t protocol_version;
  uint32_t clip_sample;
  uint32_t reserved;
  uint64_t action_dim;
  uint64_t condition_dim;
  uint64_t horizon;
  uint64_t action_steps;
  uint64_t observation_steps;
  uint64_t train_timesteps;
  float clip_sample_range;
  float reserved_float;
} fe_diffusion_metadata;

enum { /* engine.h:46-59 */
  FE_STATUS_OK = 0,
  FE_STATUS_INVALID_ARGUMENT = 1,
  FE_STATUS_RESOURCE_EXHAUSTED = 2,
  FE_STATUS_TOKEN_OUT_OF_RANGE = 3,
  FE_STATUS_UNSUPPORTED_MODEL = 4,
  FE_STATUS_INVALID_SOLVER = 5,
  FE_STATUS_NO_ACTIVE_OPERATION = 6,
  FE_STATUS_STATE_UNAVAILABLE = 7,
  FE_STATUS_CANCELLED = 8,
  FE_STATUS_INCOMPATIBLE_STATE = 9,
  FE_STATUS_CORRUPT_STATE = 10,
};

/* engine.h:60-63: last error of this thread, valid until the next call, never NULL */
const char* fe_engine_last_error(void);

/* engine.h:65-71: load with FLOWEDGE_THREADS (0..8). FLOWEDGE_CUDA_FORCE_HOST=1
 * is a load error here (no host kernels exist); FLOWEDGE_CUDA_REQUIRED=1 is
 * always satisfied by a successful load. */
fe_engine* fe_engine_load(const char* path);
/* engine.h:73-82: worker_threads above 8 are rejected */
fe_engine* fe_engine_load_with_threads(const char* path, unsigned worker_threads);
/* engine.h:84-85 */
fe_weights* fe_weights_load(const char* path);
/* engine.h:87-88 */
size_t fe_weights_size_bytes(const fe_weights* weights);
/* engine.h:90-91 */
void fe_weights_free(fe_weights* weights);
/* engine.h:93-94 */
fe_engine* fe_engine_create_from_weights(const fe_weights* weights, unsigned worker_threads);
/* engine.h:96-97 */
fe_engine* fe_engine_create_from_weights_auto(const fe_weights* weights);
/* engine.h:99-105 */
void fe_engine_dims(const fe_engine* engine, size_t* d_model, size_t* n_layers);
/* engine.h:107-114: Mamba prefill, out [seq_len][d_model] */
int fe_engine_run(fe_engine* engine, const int32_t* tokens, size_t seq_len, float* out);
/* engine.h:116-124: Transformer backbone (not built: FE_STATUS_UNSUPPORTED_MODEL) */
int fe_engine_run_embeddings(fe_engine* engine, const float* embeddings, size_t seq_len, float* out);
/* engine.h:126-134 (not built: FE_STATUS_UNSUPPORTED_MODEL) */
int fe_engine_run_embeddings_masked(fe_engine* engine, const float* embeddings, const uint8_t* attention_mask,
                                    size_t seq_len, float* out);
/* engine.h:136-146: SmolVLA suffix embedding, out [chunk_size][expert_width] */
int fe_engine_smolvla_embed_suffix(fe_engine* engine, const float* noisy_actions, size_t chunk_size,
                                   float timestep, float* out);
/* engine.h:148-161: the expert's layers over a caller-supplied prefix cache
 * [expert_layers][prefix_length][cache_width] (cache_width = the K / V width in
 * the reference's layout; this build also accepts a wider cache that the
 * cross-attention layers project, e.g. a 960-wide prefix for 12 heads of 60) */
int fe_engine_smolvla_run_expert(fe_engine* engine, const float* suffix, size_t chunk_size,
                                 const float* prefix_keys, const float* prefix_values, const uint8_t* prefix_mask,
                                 size_t prefix_length, float* out);
/* engine.h:163-171 */
int fe_engine_smolvla_project_actions(fe_engine* engine, const float* hidden, size_t chunk_size, float* out);
/* engine.h:173-183 */
int fe_engine_smolvla_denoise(fe_engine* engine, const float* noisy_actions, size_t chunk_size, float timestep,
                              const float* prefix_keys, const float* prefix_values, const uint8_t* prefix_mask,
                              size_t prefix_length, float* out);
/* engine.h:185-196: Euler sample, t = 1 - step / steps */
int fe_engine_smolvla_sample(fe_engine* engine, const float* initial_noise, size_t chunk_size, size_t steps,
                             const float* prefix_keys, const float* prefix_values, const uint8_t* prefix_mask,
                             size_t prefix_length, float* out);
/* engine.h:198-205: streaming Mamba decode of one token, out [d_model] */
int fe_engine_step(fe_engine* engine, int32_t token, float* out);
/* engine.h:207-211 */
void fe_engine_reset(fe_engine* engine);
/* engine.h:213-218 */
unsigned fe_engine_thread_count(const fe_engine* engine);
/* engine.h:220-228: always 1 for a loaded engine (weights are device-resident) */
int fe_engine_cuda_resident(const fe_engine* engine);
/* engine.h:230-231 */
int fe_engine_model_metadata(const fe_engine* engine, fe_model_metadata* metadata);
/* engine.h:233-239: returns 2 when the checkpoint has no deployment profile */
int fe_engine_deployment_profile(const fe_engine* engine, fe_deployment_profile* profile);
/* engine.h:241-246 */
size_t fe_engine_action_dim(const fe_engine* engine);
/* engine.h:248-251 */
size_t fe_engine_action_horizon(const fe_engine* engine);
/* engine.h:253-254 */
int fe_engine_diffusion_metadata(const fe_engine* engine, fe_diffusion_metadata* metadata);
/* engine.h:256-261 */
size_t fe_engine_condition_dim(const fe_engine* engine);
/* engine.h:263-279: DDIM (eta 0) / DDPM sample, action in original units */
int fe_engine_sample_diffusion(fe_engine* engine, const float* condition, const float* noise, size_t steps,
                               int scheduler, uint64_t seed, float* action);
/* engine.h:281-284: one epsilon prediction in normalized action space */
int fe_engine_diffusion_denoise(fe_engine* engine, const float* condition, const float* normalized_sample,
                                float timestep, float* predicted_noise);
/* engine.h:286-303: Mamba condition from tokens, then the flow ODE */
int fe_engine_sample(fe_engine* engine, const int32_t* tokens, size_t seq_len, const float* noise, size_t steps,
                     int method, float* action);
/* engine.h:305-322 */
int fe_engine_sample_condition(fe_engine* engine, const float* condition, const float* noise, size_t steps,
                               int method, float* action);
/* engine.h:324-333 */
int fe_engine_flow_begin(fe_engine* engine, const float* condition, const float* noise, size_t steps, int method);
/* engine.h:335-341 */
int fe_engine_make_condition_metadata(const fe_engine* engine, uint64_t timestamp_ns, uint64_t deadline_ns,
                                      uint64_t generation, size_t steps, int method,
                                      fe_condition_metadata* metadata);
/* engine.h:343-345 */
int fe_engine_flow_begin_request(fe_engine* engine, const float* condition, const float* noise,
                                 const fe_condition_metadata* metadata);
/* engine.h:347-351: the one call that is safe concurrently with fe_engine_flow_advance */
void fe_engine_cancel_before(fe_engine* engine, uint64_t generation);
/* engine.h:353-365 */
int fe_engine_flow_advance(fe_engine* engine, size_t step_budget, float* action, size_t* steps_remaining);
/* engine.h:367-368 */
int fe_engine_flow_action_metadata(const fe_engine* engine, fe_action_metadata* metadata);
/* engine.h:370-375: 96-byte header + decode state */
size_t fe_engine_decode_state_bytes(const fe_engine* engine);
/* engine.h:377-383 */
int fe_engine_export_decode_state(const fe_engine* engine, void* destination, size_t bytes);
/* engine.h:385-391 */
int fe_engine_import_decode_state(fe_engine* engine, const void* source, size_t bytes);
/* engine.h:393-397 */
void fe_engine_free(fe_engine* engine);

/* ------------------------------------------------------------------------- */
/* Part 2: extensions (no counterpart in the reference, which is batch 1)     */

enum { FE_PRECISION_MODE_AUTO = 0, FE_PRECISION_MODE_F32 = 1, FE_PRECISION_MODE_BF16 = 2 };

typedef struct fe_engine_options {
  uint32_t struct_size;    /* sizeof(fe_engine_options) */
  uint32_t worker_threads; /* 0..8, kept for fe_engine_thread_count */
  int32_t device;          /* CUDA device index; -1 = FLOWEDGE_DEVICE or 0 */
  uint32_t precision;      /* FE_PRECISION_MODE_*; AUTO = bf16 if the file stores bf16 weights */
  uint64_t max_batch;      /* batch capacity reserved at load (0 = FLOWEDGE_MAX_BATCH or 1) */
  uint64_t max_sequence;   /* Mamba prefill capacity in tokens (0 = 512) */
} fe_engine_options;

/* Load with explicit options (device, precision, batch capacity). */
fe_engine* fe_engine_load_with_options(const char* path, const fe_engine_options* options);
/* Shared-weight variant of fe_engine_load_with_options. */
fe_engine* fe_engine_create_from_weights_with_options(const fe_weights* weights, const fe_engine_options* options);

/* Grow the device workspace to hold `max_batch` independent samples.  This is
 * the only call besides loading that allocates device memory; calls with
 * batch <= the reserved capacity never allocate. */
int fe_engine_reserve_batch(fe_engine* engine, size_t max_batch);

/* Batched fe_engine_sample_diffusion: condition [batch][C], noise and action
 * [batch][H][A].  Sample b uses DDPM seed `seed + b`. */
int fe_engine_sample_diffusion_batch(fe_engine* engine, const float* condition, const float* noise, size_t batch,
                                     size_t steps, int scheduler, uint64_t seed, float* action);
/* Batched fe_engine_diffusion_denoise. */
int fe_engine_diffusion_denoise_batch(fe_engine* engine, const float* condition, const float* normalized_sample,
                                      size_t batch, float timestep, float* predicted_noise);
/* As fe_engine_sample_diffusion_batch with DEVICE pointers, enqueued on
 * `stream` (a cudaStream_t, NULL = the engine's stream); returns before the
 * work completes. */
int fe_engine_sample_diffusion_device(fe_engine* engine, const float* condition, const float* noise, size_t batch,
                                      size_t steps, int scheduler, uint64_t seed, float* action, void* stream);
/* Batched fe_engine_sample_condition: condition [batch][C], noise/action [batch][A]. */
int fe_engine_sample_condition_batch(fe_engine* engine, const float* condition, const float* noise, size_t batch,
                                     size_t steps, int method, float* action);
/* Device-pointer variant of fe_engine_sample_condition_batch. */
int fe_engine_sample_condition_device(fe_engine* engine, const float* condition, const float* noise, size_t batch,
                                      size_t steps, int method, float* action, void* stream);
/* Allocation-free variant of fe_engine_sample_condition_device (no
 * counterpart in the reference ABI).  For callers that cannot call cudaMalloc
 * while they sample - a fixed-period control loop, where cudaMalloc may block
 * and synchronise the device, or a host process whose device memory another
 * runtime's pool allocator claimed at start-up - it runs the flow ODE solve on caller device buffers (condition [batch][C],
 * noise / action [batch][A], enqueued on `stream`) with its scratch in a
 * fixed 4 MiB static device array that every GPU loading the library holds
 * until exit, never touching the engine's reserved workspace.  Requests whose
 * scratch exceeds 4 MiB are rejected with FE_STATUS_RESOURCE_EXHAUSTED.  The
 * first call on a device looks up the array's address; make it before any
 * stream capture.  Calls share the array: calls that overlap on the GPU race. */
int fe_engine_sample_condition_static(fe_engine* engine, const float* condition, const float* noise, size_t batch,
                                      size_t steps, int method, float* action, void* stream);
/* Batched Mamba prefill: tokens [batch][seq_len], out [batch][seq_len][d_model]. */
int fe_engine_run_batch(fe_engine* engine, const int32_t* tokens, size_t batch, size_t seq_len, float* out);
/* Mamba prefill on DEVICE buffers, enqueued on `stream` (NULL = the engine's
 * stream): tokens [batch][seq_len] (ids are not range-checked on the host),
 * last_hidden [batch][d_model] = the final-normed hidden state of each
 * sequence's last position (the flow condition).  Returns before the work
 * completes; batch * seq_len must fit the reserved capacity. */
int fe_engine_run_device(fe_engine* engine, const int32_t* tokens, size_t batch, size_t seq_len, float* last_hidden,
                         void* stream);
/* Batched fe_engine_sample: tokens [batch][seq_len], noise/action [batch][A]. */
int fe_engine_sample_batch(fe_engine* engine, const int32_t* tokens, size_t batch, size_t seq_len,
                           const float* noise, size_t steps, int method, float* action);
/* Batched fe_engine_smolvla_sample: initial_noise / out [batch][chunk_size][max_action_dim];
 * prefix_keys / prefix_values [batch][expert_layers][prefix_length][cache_width] and
 * prefix_mask [batch][prefix_length], or one prefix for every sample when
 * shared_prefix != 0. */
int fe_engine_smolvla_sample_batch(fe_engine* engine, const float* initial_noise, size_t batch, size_t chunk_size,
                                   size_t steps, const float* prefix_keys, const float* prefix_values,
                                   const uint8_t* prefix_mask, size_t prefix_length, int shared_prefix, float* out);
/* As fe_engine_smolvla_sample_batch with DEVICE pointers, enqueued on `stream`
 * (NULL = the engine's stream); returns before the work completes.  The mask is
 * not validated on the host. */
int fe_engine_smolvla_sample_device(fe_engine* engine, const float* initial_noise, size_t batch, size_t chunk_size,
                                    size_t steps, const float* prefix_keys, const float* prefix_values,
                                    const uint8_t* prefix_mask, size_t prefix_length, int shared_prefix, float* out,
                                    void* stream);
/* Reserve the SmolVLA workspace for `batch` chunks of `chunk_size` tokens and
 * prefixes of `prefix_length` slots (the only SmolVLA call besides the first
 * sample of a larger shape that allocates device memory). */
int fe_engine_smolvla_reserve(fe_engine* engine, size_t batch, size_t chunk_size, size_t prefix_length,
                              int shared_prefix);
/* Wait for all work enqueued by this engine. */
int fe_engine_synchronize(fe_engine* engine);

/* Profile one U-Net forward of `batch` samples on the tensor-core path with
 * CUDA events around every convolution GEMM: metrics[0] = summed GEMM kernel
 * milliseconds, [1] = GEMM launches, [2] = algorithmic GEMM FLOPs,
 * [3] = whole forward milliseconds.  The batch must be within the reserved
 * capacity and use the tensor-core path (bf16 mode). */
int fe_engine_profile_diffusion(fe_engine* engine, size_t batch, double* metrics);

/* Process-wide counts of device / pinned-host allocations made by this library. */
uint64_t fe_device_malloc_count(void);
uint64_t fe_host_malloc_count(void);
/* Kernel launches issued by this engine so far (graph replays counted per node). */
uint64_t fe_engine_kernel_launches(const fe_engine* engine);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* FLOWEDGE_B200_H */
