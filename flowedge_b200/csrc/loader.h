// Checkpoint loading (host, C++23): safetensors container, deployment
// profile metadata, model identity (digest / precision).
#pragma once

#include <array>
#include <cstddef>
#include <cstdint>
#include <memory>
#include <optional>
#include <string>
#include <vector>

#include "device.h"

namespace feb {

using Digest = std::array<std::uint8_t, 16>;

struct DeploymentProfile {
  std::uint32_t profile_version{};
  std::uint32_t model_compatibility_version{};
  std::string observation_schema_hash;
  std::size_t action_dim{};
  std::size_t action_horizon{};
  int action_units{};        // 0 normalized, 1 physical
  int normalization_type{};  // 0 none, 1 minmax
  std::vector<float> normalization_min, normalization_max;
  int solver_default{};      // 0 euler, 1 heun, 2 rk4
  std::size_t solver_min_steps{}, solver_max_steps{};
};

// One immutable, shareable checkpoint store (the fe_weights handle).
class ModelWeights {
 public:
  // Reads and validates `path`; on failure returns null and sets `error`.
  static std::shared_ptr<const ModelWeights> open(const char* path, std::string& error);

  [[nodiscard]] const TensorTable& table() const noexcept { return table_; }
  [[nodiscard]] std::size_t weight_bytes() const noexcept { return weight_bytes_; }
  [[nodiscard]] const DeploymentProfile* profile() const noexcept { return profile_ ? &*profile_ : nullptr; }
  [[nodiscard]] const Digest& digest() const noexcept { return digest_; }
  [[nodiscard]] std::uint32_t precision() const noexcept { return precision_; }
  // Batch capacity written into the file by flowedge_b200.checkpoint
  // (metadata key "flowedge.max_batch"; 0 = none): the default reservation of
  // engines created from this store when their options and FLOWEDGE_MAX_BATCH
  // name none.
  [[nodiscard]] std::size_t default_max_batch() const noexcept { return default_max_batch_; }

 private:
  std::vector<std::byte> storage_;
  TensorTable table_;
  std::size_t weight_bytes_{};
  std::optional<DeploymentProfile> profile_;
  Digest digest_{};
  std::uint32_t precision_{};
  std::size_t default_max_batch_{};
};

// XXH64 of a byte range (the published xxHash 64-bit algorithm).
std::uint64_t xxh64(const void* data, std::size_t size, std::uint64_t seed) noexcept;
// 16-byte digest of a byte range (snapshot payload checksum).
Digest fingerprint_bytes(const void* data, std::size_t size) noexcept;

}  // namespace feb
