// safetensors reader, deployment-profile parser and model identity.
//
// Container rules follow the reference loader (src/core/loader/safetensors.cc):
// u64 little-endian header length, JSON header, F32 / BF16 tensors kept as
// stored (other dtypes are skipped), at most 4 dimensions, data ranges inside
// the file and non-overlapping, element count x element size == byte length.
// Tensors keep the header's textual order, which the model digest depends on.
#include "loader.h"

#include <algorithm>
#include <bit>
#include <charconv>
#include <cmath>
#include <cstring>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <limits>
#include <map>
#include <string_view>
#include <utility>
#include <variant>

namespace feb {
namespace {

// ---------------------------------------------------------------------------
// minimal JSON (objects keep insertion order)

struct Json;
using JsonObject = std::vector<std::pair<std::string, Json>>;
using JsonArray = std::vector<Json>;

struct Json {
  std::variant<std::nullptr_t, bool, double, std::string, JsonArray, JsonObject> v;
  [[nodiscard]] const JsonObject* object() const { return std::get_if<JsonObject>(&v); }
  [[nodiscard]] const JsonArray* array() const { return std::get_if<JsonArray>(&v); }
  [[nodiscard]] const std::string* string() const { return std::get_if<std::string>(&v); }
  [[nodiscard]] const double* number() const { return std::get_if<double>(&v); }
  [[nodiscard]] const Json* get(std::string_view key) const {
    if (const auto* o = object())
      for (const auto& [k, val] : *o)
        if (k == key) return &val;
    return nullptr;
  }
};

class JsonParser {
 public:
  explicit JsonParser(std::string_view text) : s_(text) {}
  bool parse(Json& out) {
    if (!value(out, 0)) return false;
    ws();
    return pos_ == s_.size();
  }

 private:
  void ws() {
    while (pos_ < s_.size() && (s_[pos_] == ' ' || s_[pos_] == '\n' || s_[pos_] == '\r' || s_[pos_] == '\t')) ++pos_;
  }
  bool literal(std::string_view lit) {
    if (s_.substr(pos_, lit.size()) != lit) return false;
    pos_ += lit.size();
    return true;
  }
  bool str(std::string& out) {
    if (pos_ >= s_.size() || s_[pos_] != '"') return false;
    ++pos_;
    while (pos_ < s_.size()) {
      const char c = s_[pos_++];
      if (c == '"') return true;
      if (c != '\\') {
        out.push_back(c);
        continue;
      }
      if (pos_ >= s_.size()) return false;
      const char e = s_[pos_++];
      switch (e) {
        case '"': out.push_back('"'); break;
        case '\\': out.push_back('\\'); break;
        case '/': out.push_back('/'); break;
        case 'b': out.push_back('\b'); break;
        case 'f': out.push_back('\f'); break;
        case 'n': out.push_back('\n'); break;
        case 'r': out.push_back('\r'); break;
        case 't': out.push_back('\t'); break;
        case 'u': {
          if (pos_ + 4 > s_.size()) return false;
          unsigned code = 0;
          const auto [p, ec] = std::from_chars(s_.data() + pos_, s_.data() + pos_ + 4, code, 16);
          if (ec != std::errc{} || p != s_.data() + pos_ + 4) return false;
          pos_ += 4;
          if (code < 0x80) out.push_back(static_cast<char>(code));
          else out.push_back('?');
          break;
        }
        default: return false;
      }
    }
    return false;
  }
  bool value(Json& out, int depth) {
    if (depth > 32) return false;
    ws();
    if (pos_ >= s_.size()) return false;
    const char c = s_[pos_];
    if (c == '{') {
      ++pos_;
      JsonObject obj;
      ws();
      if (pos_ < s_.size() && s_[pos_] == '}') {
        ++pos_;
        out.v = std::move(obj);
        return true;
      }
      while (true) {
        ws();
        std::string key;
        if (!str(key)) return false;
        ws();
        if (pos_ >= s_.size() || s_[pos_++] != ':') return false;
        Json val;
        if (!value(val, depth + 1)) return false;
        obj.emplace_back(std::move(key), std::move(val));
        ws();
        if (pos_ >= s_.size()) return false;
        if (s_[pos_] == ',') {
          ++pos_;
          continue;
        }
        if (s_[pos_] == '}') {
          ++pos_;
          break;
        }
        return false;
      }
      out.v = std::move(obj);
      return true;
    }
    if (c == '[') {
      ++pos_;
      JsonArray arr;
      ws();
      if (pos_ < s_.size() && s_[pos_] == ']') {
        ++pos_;
        out.v = std::move(arr);
        return true;
      }
      while (true) {
        Json val;
        if (!value(val, depth + 1)) return false;
        arr.push_back(std::move(val));
        ws();
        if (pos_ >= s_.size()) return false;
        if (s_[pos_] == ',') {
          ++pos_;
          continue;
        }
        if (s_[pos_] == ']') {
          ++pos_;
          break;
        }
        return false;
      }
      out.v = std::move(arr);
      return true;
    }
    if (c == '"') {
      std::string s;
      if (!str(s)) return false;
      out.v = std::move(s);
      return true;
    }
    if (literal("true")) {
      out.v = true;
      return true;
    }
    if (literal("false")) {
      out.v = false;
      return true;
    }
    if (literal("null")) {
      out.v = nullptr;
      return true;
    }
    const std::size_t start = pos_;
    while (pos_ < s_.size() && (std::isdigit(static_cast<unsigned char>(s_[pos_])) || s_[pos_] == '-' ||
                                s_[pos_] == '+' || s_[pos_] == '.' || s_[pos_] == 'e' || s_[pos_] == 'E'))
      ++pos_;
    if (start == pos_) return false;
    double d = 0;
    const auto [p, ec] = std::from_chars(s_.data() + start, s_.data() + pos_, d);
    if (ec != std::errc{} || p != s_.data() + pos_) return false;
    out.v = d;
    return true;
  }
  std::string_view s_;
  std::size_t pos_ = 0;
};

bool as_uint(const Json* j, std::uint64_t& out) {
  if (j == nullptr || j->number() == nullptr) return false;
  const double d = *j->number();
  if (!(d >= 0) || std::floor(d) != d || d > 9.007199254740992e15) return false;
  out = static_cast<std::uint64_t>(d);
  return true;
}

// ---------------------------------------------------------------------------
// deployment profile (fields and limits of src/core/protocol/deployment_profile.cc)

bool valid_hash(const std::string& v) {
  if (v.size() != 71 || !v.starts_with("sha256:")) return false;
  return std::all_of(v.begin() + 7, v.end(), [](char c) { return std::isxdigit(static_cast<unsigned char>(c)); });
}

bool parse_profile(const std::string& text, DeploymentProfile& p, std::string& error) {
  Json root;
  if (!JsonParser(text).parse(root) || root.object() == nullptr) {
    error = "deployment profile JSON is invalid";
    return false;
  }
  std::uint64_t u = 0;
  const char* missing = "deployment profile field is missing";
  for (const char* key : {"profile_version", "model_compatibility_version", "observation_schema_hash", "action_dim",
                          "action_horizon", "action_units", "normalization_type", "normalization_parameters",
                          "solver_default", "solver_min_steps", "solver_max_steps"})
    if (root.get(key) == nullptr) {
      error = missing;
      return false;
    }
  if (!as_uint(root.get("profile_version"), u) || u != 1) {
    error = "deployment profile version is unsupported";
    return false;
  }
  p.profile_version = 1;
  if (!as_uint(root.get("model_compatibility_version"), u) || u != 1) {
    error = "model compatibility version is unsupported";
    return false;
  }
  p.model_compatibility_version = 1;
  const std::string* hash = root.get("observation_schema_hash")->string();
  if (hash == nullptr || !valid_hash(*hash)) {
    error = "observation_schema_hash must be sha256 followed by 64 hex digits";
    return false;
  }
  p.observation_schema_hash = *hash;
  if (!as_uint(root.get("action_dim"), u) || u == 0 || u > 65536) {
    error = "action_dim must be between 1 and 65536";
    return false;
  }
  p.action_dim = u;
  if (!as_uint(root.get("action_horizon"), u) || u == 0 || u > 4096) {
    error = "action_horizon must be between 1 and 4096";
    return false;
  }
  p.action_horizon = u;
  const std::string* units = root.get("action_units")->string();
  if (units == nullptr || (*units != "normalized" && *units != "physical")) {
    error = "action_units must be normalized or physical";
    return false;
  }
  p.action_units = *units == "physical" ? 1 : 0;
  const std::string* norm = root.get("normalization_type")->string();
  if (norm == nullptr || (*norm != "none" && *norm != "minmax")) {
    error = "normalization_type must be none or minmax";
    return false;
  }
  p.normalization_type = *norm == "minmax" ? 1 : 0;
  const Json* params = root.get("normalization_parameters");
  const char* bad_params = "normalization_parameters must contain finite min/max arrays matching action_dim";
  if (params->object() == nullptr) {
    error = bad_params;
    return false;
  }
  const Json* mn = params->get("min");
  const Json* mx = params->get("max");
  if (p.normalization_type == 1) {
    if (mn == nullptr || mx == nullptr || mn->array() == nullptr || mx->array() == nullptr ||
        mn->array()->size() != p.action_dim || mx->array()->size() != p.action_dim) {
      error = bad_params;
      return false;
    }
    for (std::size_t i = 0; i < p.action_dim; ++i) {
      const double* a = (*mn->array())[i].number();
      const double* b = (*mx->array())[i].number();
      if (a == nullptr || b == nullptr || !std::isfinite(*a) || !std::isfinite(*b) ||
          static_cast<float>(*a) >= static_cast<float>(*b)) {
        error = bad_params;
        return false;
      }
      p.normalization_min.push_back(static_cast<float>(*a));
      p.normalization_max.push_back(static_cast<float>(*b));
    }
  } else if (mn != nullptr || mx != nullptr) {
    error = bad_params;
    return false;
  }
  const std::string* solver = root.get("solver_default")->string();
  if (solver == nullptr || (*solver != "euler" && *solver != "heun" && *solver != "rk4")) {
    error = "solver_default must be euler, heun, or rk4";
    return false;
  }
  p.solver_default = *solver == "euler" ? 0 : (*solver == "heun" ? 1 : 2);
  std::uint64_t lo = 0, hi = 0;
  if (!as_uint(root.get("solver_min_steps"), lo) || !as_uint(root.get("solver_max_steps"), hi) || lo == 0 ||
      hi == 0 || lo > hi || hi > 4096) {
    error = "solver_min_steps and solver_max_steps must be between 1 and 4096";
    return false;
  }
  p.solver_min_steps = lo;
  p.solver_max_steps = hi;
  return true;
}

// ---------------------------------------------------------------------------
// XXH64 (published algorithm) and the reference's tensor-table digest

constexpr std::uint64_t P1 = 11400714785074694791ULL;
constexpr std::uint64_t P2 = 14029467366897019727ULL;
constexpr std::uint64_t P3 = 1609587929392839161ULL;
constexpr std::uint64_t P4 = 9650029242287828579ULL;
constexpr std::uint64_t P5 = 2870177450012600261ULL;

std::uint64_t rd64(const std::uint8_t* p) {
  std::uint64_t v;
  std::memcpy(&v, p, 8);
  return v;
}
std::uint32_t rd32(const std::uint8_t* p) {
  std::uint32_t v;
  std::memcpy(&v, p, 4);
  return v;
}
constexpr std::uint64_t xround(std::uint64_t acc, std::uint64_t in) { return std::rotl(acc + in * P2, 31) * P1; }
constexpr std::uint64_t avalanche(std::uint64_t h) {
  h ^= h >> 33;
  h *= P2;
  h ^= h >> 29;
  h *= P3;
  return h ^ (h >> 32);
}
// Accumulator used by the model digest: (rotl(acc ^ round(0, v), 27) * P1) + P4
// (src/core/protocol/model_identity.cc:100-104); kept identical so digests,
// decode snapshots and request metadata interoperate with the reference.
constexpr std::uint64_t combine(std::uint64_t acc, std::uint64_t v) {
  return (std::rotl(acc ^ xround(0, v), 27) * P1) + P4;
}

Digest make_digest(std::uint64_t a, std::uint64_t b) {
  Digest d{};
  for (int i = 0; i < 8; ++i) {
    d[static_cast<std::size_t>(i)] = static_cast<std::uint8_t>(a >> (8 * i));
    d[static_cast<std::size_t>(8 + i)] = static_cast<std::uint8_t>(b >> (8 * i));
  }
  return d;
}

Digest fingerprint_table(const TensorTable& table) {
  std::uint64_t first = combine(0x243f6a8885a308d3ULL, table.tensors.size());
  std::uint64_t second = combine(0x13198a2e03707344ULL, table.tensors.size());
  for (const HostTensor& t : table.tensors) {
    const std::uint64_t nh = xxh64(t.name.data(), t.name.size(), P3);
    first = combine(first, nh);
    second = combine(second, std::rotl(nh, 17));
    // dtype code as in the reference TensorView (F32 = 0, BF16 = 1)
    const std::uint64_t format = static_cast<std::uint64_t>(t.dtype) | (static_cast<std::uint64_t>(t.ndim) << 8);
    first = combine(first, format);
    second = combine(second, format ^ t.bytes);
    for (int i = 0; i < t.ndim; ++i) {
      first = combine(first, t.shape[static_cast<std::size_t>(i)]);
      second = combine(second, std::rotl(static_cast<std::uint64_t>(t.shape[static_cast<std::size_t>(i)]), 23));
    }
    const std::uint64_t content = xxh64(t.data, t.bytes, P5);
    first = combine(first, content);
    second = combine(second, std::rotl(content, 31) ^ t.bytes);
  }
  return make_digest(avalanche(first), avalanche(second));
}

struct Mapped {
  const std::uint8_t* data = nullptr;
  std::size_t size = 0;
  ~Mapped() {
    if (data != nullptr) munmap(const_cast<std::uint8_t*>(data), size);
  }
};

}  // namespace

std::uint64_t xxh64(const void* data, std::size_t size, std::uint64_t seed) noexcept {
  const auto* p = static_cast<const std::uint8_t*>(data);
  const std::uint8_t* const end = p + size;
  std::uint64_t h;
  if (size >= 32) {
    std::uint64_t v1 = seed + P1 + P2, v2 = seed + P2, v3 = seed, v4 = seed - P1;
    const std::uint8_t* const limit = end - 32;
    do {
      v1 = xround(v1, rd64(p));
      v2 = xround(v2, rd64(p + 8));
      v3 = xround(v3, rd64(p + 16));
      v4 = xround(v4, rd64(p + 24));
      p += 32;
    } while (p <= limit);
    h = std::rotl(v1, 1) + std::rotl(v2, 7) + std::rotl(v3, 12) + std::rotl(v4, 18);
    for (const std::uint64_t v : {v1, v2, v3, v4}) {
      h ^= xround(0, v);
      h = h * P1 + P4;
    }
  } else {
    h = seed + P5;
  }
  h += size;
  while (p + 8 <= end) {
    h ^= xround(0, rd64(p));
    h = std::rotl(h, 27) * P1 + P4;
    p += 8;
  }
  if (p + 4 <= end) {
    h ^= static_cast<std::uint64_t>(rd32(p)) * P1;
    h = std::rotl(h, 23) * P2 + P3;
    p += 4;
  }
  while (p < end) {
    h ^= static_cast<std::uint64_t>(*p) * P5;
    h = std::rotl(h, 11) * P1;
    ++p;
  }
  return avalanche(h);
}

Digest fingerprint_bytes(const void* data, std::size_t size) noexcept {
  const std::uint64_t first = xxh64(data, size, 0x243f6a8885a308d3ULL);
  const std::uint64_t second = avalanche(first ^ static_cast<std::uint64_t>(size) ^ 0x13198a2e03707344ULL);
  return make_digest(first, second);
}

std::shared_ptr<const ModelWeights> ModelWeights::open(const char* path, std::string& error) {
  const int fd = ::open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) {
    error = "Failed to open safetensors file";
    return nullptr;
  }
  struct stat st {};
  if (fstat(fd, &st) != 0 || st.st_size < 8) {
    ::close(fd);
    error = "File too small";
    return nullptr;
  }
  Mapped m;
  m.size = static_cast<std::size_t>(st.st_size);
  void* addr = mmap(nullptr, m.size, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (addr == MAP_FAILED) {
    error = "Failed to mmap safetensors file";
    return nullptr;
  }
  m.data = static_cast<const std::uint8_t*>(addr);
  std::uint64_t header_len = 0;
  std::memcpy(&header_len, m.data, 8);
  if (header_len > m.size - 8) {
    error = "Invalid header length";
    return nullptr;
  }
  const std::string_view header(reinterpret_cast<const char*>(m.data + 8), header_len);
  Json root;
  if (!JsonParser(header).parse(root) || root.object() == nullptr) {
    error = "Invalid safetensors header JSON";
    return nullptr;
  }
  const std::uint8_t* const base = m.data + 8 + header_len;
  const std::uint64_t data_size = m.size - 8 - header_len;

  auto weights = std::shared_ptr<ModelWeights>(new ModelWeights());
  struct Pending {
    std::string name;
    DType dtype;
    int ndim;
    std::array<std::size_t, 4> shape;
    std::uint64_t begin, end;
  };
  std::vector<Pending> pending;
  std::vector<std::pair<std::uint64_t, std::uint64_t>> spans;
  std::size_t total = 0;
  for (const auto& [name, entry] : *root.object()) {
    if (name == "__metadata__") {
      const Json* profile = entry.get("flowedge.deployment_profile");
      if (profile != nullptr) {
        if (profile->string() == nullptr) {
          error = "Invalid safetensors metadata value";
          return nullptr;
        }
        DeploymentProfile p;
        if (!parse_profile(*profile->string(), p, error)) return nullptr;
        weights->profile_ = std::move(p);
      }
      if (const Json* mb = entry.get("flowedge.max_batch"); mb != nullptr) {
        const std::string* text = mb->string();
        std::size_t value = 0;
        const char* first = text != nullptr ? text->data() : nullptr;
        const auto parsed = text != nullptr ? std::from_chars(first, first + text->size(), value)
                                            : std::from_chars_result{nullptr, std::errc::invalid_argument};
        if (text == nullptr || parsed.ec != std::errc() || parsed.ptr != first + text->size() || value == 0 ||
            value > (std::size_t(1) << 24)) {
          error = "Invalid flowedge.max_batch metadata (a batch count from 1 to 16777216)";
          return nullptr;
        }
        weights->default_max_batch_ = value;
      }
      continue;
    }
    const Json* dtype = entry.get("dtype");
    if (dtype == nullptr || dtype->string() == nullptr) {
      error = "Failed during tensor iteration or out of bounds";
      return nullptr;
    }
    const bool f32 = *dtype->string() == "F32", bf16 = *dtype->string() == "BF16";
    if (!f32 && !bf16) continue;  // unsupported dtypes are skipped, as the reference does
    const Json* shape = entry.get("shape");
    const Json* offsets = entry.get("data_offsets");
    if (shape == nullptr || shape->array() == nullptr || shape->array()->size() > 4 || offsets == nullptr ||
        offsets->array() == nullptr || offsets->array()->size() != 2) {
      error = "Failed during tensor iteration or out of bounds";
      return nullptr;
    }
    Pending pt{name, bf16 ? DType::BF16 : DType::F32, static_cast<int>(shape->array()->size()), {}, 0, 0};
    std::uint64_t elements = 1;
    for (std::size_t i = 0; i < shape->array()->size(); ++i) {
      std::uint64_t d = 0;
      if (!as_uint(&(*shape->array())[i], d) || (d != 0 && elements > std::numeric_limits<std::uint64_t>::max() / d)) {
        error = "Failed during tensor iteration or out of bounds";
        return nullptr;
      }
      pt.shape[i] = d;
      elements *= d;
    }
    if (!as_uint(&(*offsets->array())[0], pt.begin) || !as_uint(&(*offsets->array())[1], pt.end) ||
        pt.end < pt.begin || pt.end > data_size || elements * (bf16 ? 2 : 4) != pt.end - pt.begin) {
      error = "Failed during tensor iteration or out of bounds";
      return nullptr;
    }
    for (const auto& [b, e] : spans)
      if (pt.begin < e && b < pt.end) {
        error = "Failed during tensor iteration or out of bounds";
        return nullptr;
      }
    spans.emplace_back(pt.begin, pt.end);
    total += pt.end - pt.begin;
    pending.push_back(std::move(pt));
  }
  if (pending.empty()) {
    error = "Failed to load safetensors file or find supported tensors";
    return nullptr;
  }
  // one immutable store, 64-byte aligned tensors
  std::size_t padded = 0;
  for (const Pending& p : pending) padded += (p.end - p.begin + 63) / 64 * 64;
  weights->storage_.resize(padded + 64);
  auto* cursor = reinterpret_cast<std::uint8_t*>((reinterpret_cast<std::uintptr_t>(weights->storage_.data()) + 63) &
                                                 ~std::uintptr_t(63));
  bool f32_seen = false, bf16_seen = false;
  for (const Pending& p : pending) {
    const std::size_t bytes = p.end - p.begin;
    std::memcpy(cursor, base + p.begin, bytes);
    HostTensor t;
    t.name = p.name;
    t.dtype = p.dtype;
    t.ndim = p.ndim;
    t.shape = p.shape;
    t.data = cursor;
    t.bytes = bytes;
    weights->table_.tensors.push_back(std::move(t));
    cursor += (bytes + 63) / 64 * 64;
    (p.dtype == DType::F32 ? f32_seen : bf16_seen) = true;
  }
  weights->weight_bytes_ = total;
  weights->digest_ = fingerprint_table(weights->table_);
  weights->precision_ = f32_seen && bf16_seen ? 3u : (bf16_seen ? 2u : 1u);
  return weights;
}

}  // namespace feb
