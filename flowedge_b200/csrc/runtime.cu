#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>

#include "runtime.cuh"

namespace feb {
namespace {

std::atomic<std::uint64_t> g_device_mallocs{0};
std::atomic<std::uint64_t> g_host_mallocs{0};

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
  static EncodeTiled fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult status{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &status) != cudaSuccess ||
        status != cudaDriverEntryPointSuccess)
      ptr = nullptr;
    return reinterpret_cast<EncodeTiled>(ptr);
  }();
  return fn;
}

bool encode_2d(CUtensorMap* map, const void* ptr, std::uint64_t inner, std::uint64_t outer, std::uint32_t box_inner,
               std::uint32_t box_outer, CUtensorMapDataType dtype, std::string& err) {
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {inner * 2};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult rc = encode_fn()(map, dtype, 2, const_cast<void*>(ptr), dims, strides,
                                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (rc != CUDA_SUCCESS) {
    err = "cuTensorMapEncodeTiled (weights) failed: " + std::to_string(static_cast<int>(rc));
    return false;
  }
  return true;
}

bool encode_3d(CUtensorMap* map, const TcSource& s, std::uint32_t box_l, std::uint32_t box_s, CUtensorMapDataType dtype,
               std::string& err) {
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(s.channels), static_cast<cuuint64_t>(s.length),
                              static_cast<cuuint64_t>(s.samples)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(s.channels) * 2,
                                 static_cast<cuuint64_t>(s.channels) * s.length * 2};
  const cuuint32_t box[3] = {64, box_l, box_s};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult rc = encode_fn()(map, dtype, 3, const_cast<void*>(s.ptr), dims, strides,
                                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (rc != CUDA_SUCCESS) {
    err = "cuTensorMapEncodeTiled (activations) failed: " + std::to_string(static_cast<int>(rc));
    return false;
  }
  return true;
}

}  // namespace

bool encode_tmap_2d(CUtensorMap* map, const void* ptr, std::uint64_t inner, std::uint64_t outer,
                    std::uint32_t box_inner, std::uint32_t box_outer, bool fp16, std::string& err) {
  return encode_2d(map, ptr, inner, outer, box_inner, box_outer,
                   fp16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, err);
}

std::uint64_t device_malloc_count() noexcept { return g_device_mallocs.load(); }
std::uint64_t host_malloc_count() noexcept { return g_host_mallocs.load(); }

cudaError_t counted_malloc(void** ptr, std::size_t bytes) {
  g_device_mallocs.fetch_add(1);
  return cudaMalloc(ptr, bytes);
}

cudaError_t counted_host_malloc(void** ptr, std::size_t bytes) {
  g_host_mallocs.fetch_add(1);
  return cudaMallocHost(ptr, bytes);
}

DeviceContext::~DeviceContext() {
  if (stream != nullptr) {
    cudaSetDevice(device);
    cudaStreamSynchronize(stream);
    cudaStreamDestroy(stream);
  }
  if (d_err != nullptr) cudaFree(d_err);
}

std::shared_ptr<DeviceContext> make_device_context(int device, std::string& err) {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    cudaGetLastError();
    err = "no CUDA device is available (this library has no CPU fallback)";
    return nullptr;
  }
  if (device < 0 || device >= count) {
    err = "FLOWEDGE_DEVICE is out of range";
    return nullptr;
  }
  cudaDeviceProp prop{};
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) {
    err = "cudaGetDeviceProperties failed";
    return nullptr;
  }
  if (prop.major != 10 || prop.minor != 0) {
    err = "this library is built for sm_100a (B200); found compute capability " + std::to_string(prop.major) + "." +
          std::to_string(prop.minor);
    return nullptr;
  }
  if (encode_fn() == nullptr) {
    err = "driver entry point cuTensorMapEncodeTiled is unavailable";
    return nullptr;
  }
  auto ctx = std::make_shared<DeviceContext>();
  ctx->device = device;
  ctx->sm_count = prop.multiProcessorCount;
  cudaSetDevice(device);
  if (cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess) {
    err = "cudaStreamCreate failed";
    return nullptr;
  }
  if (counted_malloc(reinterpret_cast<void**>(&ctx->d_err), 256) != cudaSuccess ||
      cudaMemset(ctx->d_err, 0, 256) != cudaSuccess) {
    err = "device allocation failed";
    return nullptr;
  }
  if (cudaFuncSetAttribute(tc::tc_gemm_kernel<tc::kEpiPlain>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           tc::SMEM_BYTES) != cudaSuccess ||
      cudaFuncSetAttribute(tc::tc_gemm_kernel<tc::kEpiStats>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           tc::SMEM_BYTES) != cudaSuccess ||
      cudaFuncSetAttribute(tc::tc_gemm_kernel<tc::kEpiFused>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           tc::SMEM_BYTES) != cudaSuccess ||
      cudaFuncSetAttribute(tc::tc_gemm_kernel<tc::kEpiConv>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           tc::SMEM_BYTES) != cudaSuccess ||
      cudaFuncSetAttribute(tc::tc_gemm_kernel<tc::kEpiFused, false, true>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, tc::SMEM_BYTES) != cudaSuccess) {
    err = "cannot enable the tensor-core kernel's shared memory";
    return nullptr;
  }
  // 2-CTA clusters for GroupNorm groups that span two 128-row tiles: launch
  // only as many clusters as can be resident at once (the kernel is persistent)
  {
    cudaLaunchAttribute attr{};
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(ctx->sm_count & ~1));
    cfg.blockDim = dim3(tc::THREADS);
    cfg.dynamicSmemBytes = tc::SMEM_BYTES;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaFuncSetAttribute(tc::tc_gemm_kernel<tc::kEpiFused, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             tc::SMEM_BYTES) == cudaSuccess &&
        cudaOccupancyMaxActiveClusters(&clusters, tc::tc_gemm_kernel<tc::kEpiFused, true>, &cfg) == cudaSuccess)
      ctx->pair_clusters = clusters;
    else
      cudaGetLastError();
  }
  return ctx;
}

int context_device(const DeviceContext& ctx) noexcept { return ctx.device; }

int synchronize_context(DeviceContext& ctx) noexcept {
  cudaSetDevice(ctx.device);
  if (cudaStreamSynchronize(ctx.stream) != cudaSuccess) return 2;
  return take_device_error(ctx, ctx.stream) == 0 ? 0 : 2;
}

const char* device_error_text(int code) noexcept {
  switch (code) {
    case kErrWaitTimeoutProducer: return "a device pipeline wait timed out (copy producer)";
    case kErrWaitTimeoutMma: return "a device pipeline wait timed out (tensor-core consumer)";
    case kErrWaitTimeoutEpilogue: return "a device pipeline wait timed out (epilogue)";
    case kErrTmemAlloc: return "tensor memory allocation failed";
    case kErrGridBarrierTimeout: return "a device grid barrier timed out";
    case kErrProgramLayout: return "internal error: small-batch program layout check failed";
    case kErrDependencyTimeout: return "a program dependency wait timed out (small-batch U-Net or tensor-core flow solve)";
    case kErrStageTimeout: return "a staged-input wait of the selective scan timed out";
    default: return "a device pipeline wait timed out";
  }
}

int take_device_error(DeviceContext& ctx, cudaStream_t stream) {
  int host = 0;
  if (cudaMemcpyAsync(&host, ctx.d_err, sizeof(int), cudaMemcpyDeviceToHost, stream) != cudaSuccess) return -1;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return -1;
  if (host != 0) cudaMemsetAsync(ctx.d_err, 0, sizeof(int), stream);
  return host;
}

DeviceArena::~DeviceArena() { release(); }

bool DeviceArena::init(std::size_t bytes, std::string& err) {
  release();
  if (bytes == 0) bytes = 256;
  if (counted_malloc(reinterpret_cast<void**>(&base_), bytes) != cudaSuccess) {
    cudaGetLastError();
    base_ = nullptr;
    err = "device allocation of " + std::to_string(bytes >> 20) + " MiB failed";
    return false;
  }
  size_ = bytes;
  used_ = 0;
  overflowed_ = false;
  return true;
}

void* DeviceArena::take(std::size_t bytes) {
  const std::size_t aligned = (bytes + 255) & ~std::size_t(255);
  if (base_ == nullptr || used_ + aligned > size_) {
    overflowed_ = true;
    return nullptr;
  }
  void* p = base_ + used_;
  used_ += aligned;
  return p;
}

void DeviceArena::release() noexcept {
  if (base_ != nullptr) cudaFree(base_);
  base_ = nullptr;
  size_ = used_ = 0;
}

std::vector<float> widen_f32(const HostTensor& t) {
  std::vector<float> out(t.numel());
  if (t.dtype == DType::F32) {
    std::memcpy(out.data(), t.data, out.size() * sizeof(float));
  } else {
    const auto* bits = static_cast<const std::uint16_t*>(t.data);
    for (std::size_t i = 0; i < out.size(); ++i) {
      const std::uint32_t w = static_cast<std::uint32_t>(bits[i]) << 16;
      std::memcpy(&out[i], &w, sizeof(float));
    }
  }
  return out;
}

std::uint16_t fp16_bits_of_bf16_rounded(float v) {
  std::uint32_t u;
  std::memcpy(&u, &v, 4);
  if ((u & 0x7FFFFFFFu) <= 0x7F800000u) {
    u += 0x7FFFu + ((u >> 16) & 1u);
    u &= 0xFFFF0000u;
  }
  float r;
  std::memcpy(&r, &u, 4);
  const __half h = __float2half_rn(r);
  return __half_as_ushort(h);
}

bool check_fp16_storable(const std::string& name, const float* w, std::size_t n, bool bf16_mode, std::string& err) {
  double max_abs = 0.0, max_err = 0.0;
  for (std::size_t i = 0; i < n; ++i) {
    const float v = w[i];
    if (!std::isfinite(v)) {
      err = "tensor " + name + " holds a non-finite value at element " + std::to_string(i);
      return false;
    }
    double target, stored;
    if (bf16_mode) {
      const std::uint16_t h = fp16_bits_of_bf16_rounded(v);
      std::uint32_t u;
      std::memcpy(&u, &v, 4);
      u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
      float r;
      std::memcpy(&r, &u, 4);
      target = r;
      stored = __half2float(__ushort_as_half(h));
    } else {
      const __half hi = __float2half_rn(v);
      const float hf = __half2float(hi);
      target = v;
      stored = static_cast<double>(hf) + static_cast<double>(__half2float(__float2half_rn(v - hf)));
    }
    if (!std::isfinite(stored)) {
      err = "tensor " + name + " holds " + std::to_string(v) + " at element " + std::to_string(i) +
            ", beyond the fp16 range (65504) of this build's " + (bf16_mode ? "bf16" : "fp32") +
            " weight storage";
      return false;
    }
    max_abs = std::max(max_abs, std::fabs(target));
    max_err = std::max(max_err, std::fabs(stored - target));
  }
  const double bound = bf16_mode ? 1.0 / 512.0 : 1.0 / 65536.0;
  if (max_err > bound * max_abs) {
    err = "tensor " + name + " cannot be stored in fp16 to " + (bf16_mode ? "2^-9" : "2^-16") +
          " of its largest magnitude " + std::to_string(max_abs) + " (fp16 subnormal range); largest error " +
          std::to_string(max_err);
    return false;
  }
  return true;
}

cudaError_t tc_gemm(const TcLaunch& l, DeviceContext& ctx, cudaStream_t stream, std::string& err) {
  if (l.M_rows % tc::BM != 0 || l.K % tc::BK != 0 || l.L < 1 || l.L > tc::BN || (l.L & (l.L - 1)) != 0 ||
      l.segs.empty() || static_cast<int>(l.segs.size()) > tc::MAX_SEGS) {
    err = "tc_gemm: unsupported geometry";
    return cudaErrorInvalidValue;
  }
  tc::Params p{};
  p.L = l.L;
  p.L_shift = 0;
  while ((1 << p.L_shift) < l.L) ++p.L_shift;
  p.fp16 = l.fp16 ? 1 : 0;
  const CUtensorMapDataType dtype = l.fp16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  p.tile_samples = tc::BN / l.L;
  if (l.stats != nullptr && (p.tile_samples > tc::MAX_TILE_SAMPLES || l.group_ch % 32 != 0 ||
                             (l.group_ch > tc::BM && l.group_ch % tc::BM != 0) ||
                             (l.group_ch < tc::BM && tc::BM % l.group_ch != 0))) {
    err = "tc_gemm: unsupported GroupNorm geometry";
    return cudaErrorInvalidValue;
  }
  p.n_tiles_m = l.M_rows / tc::BM;
  p.n_tiles_n = (l.n_samples + p.tile_samples - 1) / p.tile_samples;
  p.total_tiles = p.n_tiles_m * p.n_tiles_n;
  p.n_samples = l.n_samples;
  p.m_valid = l.m_valid;
  p.nseg = static_cast<int>(l.segs.size());
  for (int i = 0; i < p.nseg; ++i) {
    p.seg[i] = l.segs[static_cast<std::size_t>(i)];
    const TcSource& s = l.src[p.seg[i].src];
    if (s.ptr == nullptr || s.channels % 64 != 0 || s.length != l.L || s.samples < p.tile_samples ||
        p.seg[i].ch_off % 64 != 0 || p.seg[i].ch_off + p.seg[i].kblocks * 64 > s.channels ||
        p.seg[i].a_k + p.seg[i].kblocks * 64 > l.K) {
      err = "tc_gemm: segment does not fit its source";
      return cudaErrorInvalidValue;
    }
  }
  // Output row of token (b, t) is b * rps + t * tmul + tadd; the epilogue
  // needs it affine in the global token b * L + t, i.e. rps == L * tmul.
  const long long cs = static_cast<long long>(l.out_tmul) * l.out_ld;
  const long long acs = static_cast<long long>(l.out_tmul) * l.add_ld;
  if (l.out_rps != l.L * l.out_tmul || l.out_tmul < 1 || l.out_tadd < 0 || l.out_tadd >= l.out_tmul ||
      cs * tc::BN >= (1LL << 31) || acs * tc::BN >= (1LL << 31)) {
    err = "tc_gemm: unsupported output row mapping";
    return cudaErrorInvalidValue;
  }
  if (l.stats != nullptr && (l.act != tc::kActNone || l.add_tok != nullptr)) {
    err = "tc_gemm: GroupNorm statistics need a linear epilogue";
    return cudaErrorInvalidValue;
  }
  p.bias = l.bias;
  p.add_vec = l.add_vec;
  p.add_tok = l.add_tok;
  p.add_cs = static_cast<int>(acs);
  p.add_base = static_cast<long long>(l.out_tadd) * l.add_ld;
  p.act = l.act;
  p.out_f32 = l.out_f32 ? 1 : 0;
  p.out_accumulate = l.out_accumulate ? 1 : 0;
  p.out = l.out;
  p.out_cs = static_cast<int>(cs);
  p.out_base = static_cast<long long>(l.out_tadd) * l.out_ld + l.out_ch_off;
  p.n_tokens = l.n_samples * l.L;
  if (l.out_lo_off != 0) {
    if (!l.fp16 || l.out_f32 || l.gn_fuse || l.stats != nullptr) {
      err = "tc_gemm: a hi/lo output needs a plain fp16 epilogue";
      return cudaErrorInvalidValue;
    }
    p.out_lo_off = static_cast<int>(l.out_lo_off);
  }
  if (l.act == tc::kActSwiGLU &&
      (l.out_f32 || (l.fp16 && !l.out_bf16) || l.out_lo_off != 0 || l.gn_fuse || l.stats != nullptr ||
       l.m_valid % 2 != 0 || l.add_tok != nullptr)) {
    err = "tc_gemm: the SwiGLU epilogue needs interleaved rows and a plain bf16 output";
    return cudaErrorInvalidValue;
  }
  if (l.conv_w != nullptr) {
    if (!l.out_f32 || l.out_accumulate || l.act != tc::kActNone || l.bias != nullptr || l.add_vec != nullptr ||
        l.add_tok != nullptr || l.stats != nullptr || l.gn_fuse || l.L != 1 || l.conv_b == nullptr ||
        l.conv_u16 == nullptr || l.conv_rows % tc::BM != 0 || l.conv_seq < 1 ||
        l.conv_seq > tc::BN || tc::BN % l.conv_seq != 0 || l.n_samples % l.conv_seq != 0 ||
        static_cast<long long>(l.conv_ld) * tc::BN >= (1LL << 31)) {
      err = "tc_gemm: the conv epilogue needs a plain fp32 GEMM over whole sequences that tile the token blocks";
      return cudaErrorInvalidValue;
    }
    p.conv_w = l.conv_w;
    p.conv_b = l.conv_b;
    p.conv_u = l.conv_u;
    p.conv_u16 = l.conv_u16;
    p.conv_rows = l.conv_rows;
    p.conv_seq = l.conv_seq;
    p.conv_ld = l.conv_ld;
  }
  if (l.out_bf16) {
    if (l.out_f32 || l.gn_fuse || l.stats != nullptr || l.out_lo_off != 0) {
      err = "tc_gemm: a bf16 output needs a plain 16-bit epilogue";
      return cudaErrorInvalidValue;
    }
    p.out_bf16 = 1;
  }
  p.stats = l.stats;
  p.group_ch = l.group_ch;
  p.groups = l.groups;
  p.parts = l.group_ch > tc::BM ? l.group_ch / tc::BM : 1;
  p.err = ctx.d_err;
  // Fused GroupNorm convs run with tokens on the accumulator rows (TOKM)
  // when the layout allows its 16-byte accesses: 128-token tiles (L in
  // [8, 128]), groups inside a 256-channel tile, bias without add terms, an
  // fp32 residual (or none), and every per-channel vector, row stride and base
  // 16-byte aligned.
  const auto al16 = [](const void* ptr) { return (reinterpret_cast<std::uintptr_t>(ptr) & 15u) == 0; };
  // Only the convs whose groups span 256 channels take it (they would
  // otherwise run as 2-CTA pairs) and only without an fp32 residual or twin:
  // with tokens on the lanes each 16-byte access of a warp lands in a
  // different token row, four to eight times the L1 line requests of the
  // channel-per-lane layout, which the fp32 residual stream makes the bound.
  const bool tokm =
      l.gn_fuse && l.L >= 8 && l.L <= tc::BM && l.group_ch == 256 && l.res_f32 == nullptr &&
      l.res16 == nullptr && l.out_twin == nullptr &&
      l.M_rows >= tc::BN && l.bias != nullptr && l.add_vec == nullptr && p.out_cs % 8 == 0 && p.out_base % 8 == 0 &&
      al16(l.out) && al16(l.bias) && al16(l.gamma) && al16(l.beta) && al16(l.out_twin) && al16(l.res_f32) &&
      (l.res16 == nullptr || l.res_f32 != nullptr) &&
      (l.film_cond == nullptr || (al16(l.film_cond) && al16(l.film_time) && l.film_F % 4 == 0 &&
                                  l.film_off % 4 == 0 && l.film_C % 4 == 0)) &&
      [&] {
        for (int i = 0; i < 3; ++i)
          if (l.src[i].ptr != nullptr && l.src[i].samples < tc::BM / l.L) return false;
        return true;
      }();
  if (l.gn_fuse) {
    const bool in_tile = l.group_ch >= 32 && l.group_ch <= tc::BM && tc::BM % l.group_ch == 0 &&
                         tc::BM / l.group_ch <= tc::MAX_TILE_GROUPS;
    const bool paired = l.group_ch == 2 * tc::BM && p.n_tiles_m % 2 == 0 && ctx.pair_clusters > 0;
    if (l.stats != nullptr || l.out_f32 || !(in_tile || paired || tokm) || p.tile_samples > tc::MAX_TILE_SAMPLES || l.L < 8 ||
        l.gamma == nullptr ||
        l.beta == nullptr || l.act != tc::kActNone || l.add_tok != nullptr || !l.fp16) {
      err = "tc_gemm: unsupported fused GroupNorm geometry";
      return cudaErrorInvalidValue;
    }
    p.gn_fuse = 1;
    p.group_ch = l.group_ch;
    p.gamma = l.gamma;
    p.beta = l.beta;
    p.film_cond = l.film_cond;
    p.film_time = l.film_time;
    p.film_F = l.film_F;
    p.film_off = l.film_off;
    p.film_C = l.film_C;
    p.res_f32 = l.res_f32;
    p.res16 = l.res16;
    p.out_twin = l.out_twin;
  }

  if (tokm) {
    p.tile_samples = tc::BM / l.L;
    p.n_tiles_m = (l.n_samples + p.tile_samples - 1) / p.tile_samples;
    p.n_tiles_n = (l.M_rows + tc::BN - 1) / tc::BN;
    p.total_tiles = p.n_tiles_m * p.n_tiles_n;
  }

  CUtensorMap ta{}, tb[3]{};
  if (!encode_2d(&ta, l.A, static_cast<std::uint64_t>(l.K), static_cast<std::uint64_t>(l.M_rows), 64,
                 tokm ? tc::BN : tc::BM, dtype, err))
    return cudaErrorInvalidValue;
  for (int i = 0; i < 3; ++i) {
    const TcSource& s = l.src[i].ptr != nullptr ? l.src[i] : l.src[0];
    if (!encode_3d(&tb[i], s, static_cast<std::uint32_t>(l.L), static_cast<std::uint32_t>(p.tile_samples), dtype, err))
      return cudaErrorInvalidValue;
  }
  // Launched as a programmatic dependent of the previous kernel in the stream
  // (the kernel waits for that grid before its first global access).
  cudaLaunchAttribute attrs[2]{};
  attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.blockDim = dim3(tc::THREADS);
  cfg.dynamicSmemBytes = tc::SMEM_BYTES;
  cfg.stream = stream;
  cfg.attrs = attrs;
  cfg.numAttrs = 1;
  if (tokm) {
    cfg.gridDim = dim3(static_cast<unsigned>(p.total_tiles < ctx.sm_count ? p.total_tiles : ctx.sm_count));
    const cudaError_t rc =
        cudaLaunchKernelEx(&cfg, tc::tc_gemm_kernel<tc::kEpiFused, false, true>, ta, tb[0], tb[1], tb[2], p);
    if (rc != cudaSuccess) err = std::string("tc_gemm launch: ") + cudaGetErrorString(rc);
    return rc;
  }
  if (p.gn_fuse && l.group_ch == 2 * tc::BM) {
    attrs[1].id = cudaLaunchAttributeClusterDimension;
    attrs[1].val.clusterDim.x = 2;
    attrs[1].val.clusterDim.y = 1;
    attrs[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
    cfg.gridDim = dim3(static_cast<unsigned>(2 * std::min(p.total_tiles / 2, ctx.pair_clusters)));
    const cudaError_t rc =
        cudaLaunchKernelEx(&cfg, tc::tc_gemm_kernel<tc::kEpiFused, true>, ta, tb[0], tb[1], tb[2], p);
    if (rc != cudaSuccess) err = std::string("tc_gemm cluster launch: ") + cudaGetErrorString(rc);
    return rc;
  }
  cfg.gridDim = dim3(static_cast<unsigned>(p.total_tiles < ctx.sm_count ? p.total_tiles : ctx.sm_count));
  cudaError_t rc;
  if (p.gn_fuse)
    rc = cudaLaunchKernelEx(&cfg, tc::tc_gemm_kernel<tc::kEpiFused>, ta, tb[0], tb[1], tb[2], p);
  else if (p.stats != nullptr)
    rc = cudaLaunchKernelEx(&cfg, tc::tc_gemm_kernel<tc::kEpiStats>, ta, tb[0], tb[1], tb[2], p);
  else if (p.conv_w != nullptr)
    rc = cudaLaunchKernelEx(&cfg, tc::tc_gemm_kernel<tc::kEpiConv>, ta, tb[0], tb[1], tb[2], p);
  else
    rc = cudaLaunchKernelEx(&cfg, tc::tc_gemm_kernel<tc::kEpiPlain>, ta, tb[0], tb[1], tb[2], p);
  if (rc != cudaSuccess) err = std::string("tc_gemm launch: ") + cudaGetErrorString(rc);
  return rc;
}

}  // namespace feb
