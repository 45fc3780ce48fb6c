// Test hooks (include/flowedge_b200_testing.h): one tcgen05 GEMM / conv on
// host buffers, for kernel-level numerics tests.
#include <algorithm>
#include <cstring>
#include <vector>

#include "../../include/flowedge_b200_testing.h"
#include "runtime.cuh"

namespace {

int fail(void* a, void* b, void* c) {
  cudaFree(a);
  cudaFree(b);
  cudaFree(c);
  return 2;
}

}  // namespace

extern "C" int febtest_gemm_16(const uint16_t* A, int M, int K, const uint16_t* B, int N, float* C, int fp16) {
  std::string err;
  auto ctx = feb::make_device_context(0, err);
  if (!ctx) return 1;
  const int Mp = (M + 127) / 128 * 128, Kp = (K + 63) / 64 * 64, Np = (N + 255) / 256 * 256;
  std::vector<uint16_t> a(static_cast<size_t>(Mp) * Kp, 0), b(static_cast<size_t>(Np) * Kp, 0);
  for (int m = 0; m < M; ++m) std::memcpy(&a[static_cast<size_t>(m) * Kp], A + static_cast<size_t>(m) * K, K * 2);
  for (int n = 0; n < N; ++n) std::memcpy(&b[static_cast<size_t>(n) * Kp], B + static_cast<size_t>(n) * K, K * 2);
  void *da = nullptr, *db = nullptr, *dc = nullptr;
  if (cudaMalloc(&da, a.size() * 2) != cudaSuccess || cudaMalloc(&db, b.size() * 2) != cudaSuccess ||
      cudaMalloc(&dc, static_cast<size_t>(N) * M * 4) != cudaSuccess)
    return fail(da, db, dc);
  cudaMemcpy(da, a.data(), a.size() * 2, cudaMemcpyHostToDevice);
  cudaMemcpy(db, b.data(), b.size() * 2, cudaMemcpyHostToDevice);
  feb::TcLaunch l;
  l.fp16 = fp16 != 0;
  l.A = da;
  l.M_rows = Mp;
  l.K = Kp;
  l.src[0] = feb::TcSource{db, Kp, 1, Np};
  l.L = 1;
  l.n_samples = N;
  l.m_valid = M;
  l.segs = {feb::tc::Seg{0, 0, 0, Kp / 64, 0}};
  l.out_f32 = true;
  l.out = dc;
  l.out_ld = M;
  if (feb::tc_gemm(l, *ctx, ctx->stream, err) != cudaSuccess) return fail(da, db, dc);
  if (cudaStreamSynchronize(ctx->stream) != cudaSuccess) return fail(da, db, dc);
  const int dev_err = feb::take_device_error(*ctx, ctx->stream);
  cudaMemcpy(C, dc, static_cast<size_t>(N) * M * 4, cudaMemcpyDeviceToHost);
  cudaFree(da);
  cudaFree(db);
  cudaFree(dc);
  return dev_err == 0 ? 0 : 3;
}

extern "C" int febtest_conv_16(const uint16_t* x, int B, int L, int C, const uint16_t* W, const float* bias, int OC,
                               int k, int group_ch, float* y, double* stats, int fp16) {
  std::string err;
  auto ctx = feb::make_device_context(0, err);
  if (!ctx) return 1;
  if (C % 64 != 0) return 1;
  const int OCp = (OC + 127) / 128 * 128, K = k * C;
  const int tile_samples = 256 / L;
  const int Bp = (B + tile_samples - 1) / tile_samples * tile_samples;
  // pack W [OC][C][k] -> [OCp][k][C]
  std::vector<uint16_t> a(static_cast<size_t>(OCp) * K, 0);
  for (int o = 0; o < OC; ++o)
    for (int c = 0; c < C; ++c)
      for (int j = 0; j < k; ++j)
        a[static_cast<size_t>(o) * K + static_cast<size_t>(j) * C + c] = W[(static_cast<size_t>(o) * C + c) * k + j];
  void *da = nullptr, *dx = nullptr, *dy = nullptr, *dbias = nullptr, *dst = nullptr;
  const int groups = group_ch > 0 ? OC / group_ch : 0;
  cudaMalloc(&da, a.size() * 2);
  cudaMalloc(&dx, static_cast<size_t>(Bp) * L * C * 2);
  cudaMalloc(&dy, static_cast<size_t>(B) * L * OC * 2);
  cudaMalloc(&dbias, static_cast<size_t>(OC) * 4);
  const int parts = group_ch > 128 ? group_ch / 128 : 1;
  cudaMalloc(&dst, static_cast<size_t>(B) * (groups > 0 ? groups : 1) * parts * 2 * 8);
  cudaMemset(dx, 0, static_cast<size_t>(Bp) * L * C * 2);
  cudaMemcpy(da, a.data(), a.size() * 2, cudaMemcpyHostToDevice);
  cudaMemcpy(dx, x, static_cast<size_t>(B) * L * C * 2, cudaMemcpyHostToDevice);
  cudaMemcpy(dbias, bias, static_cast<size_t>(OC) * 4, cudaMemcpyHostToDevice);
  feb::TcLaunch l;
  l.fp16 = fp16 != 0;
  l.A = da;
  l.M_rows = OCp;
  l.K = K;
  l.src[0] = feb::TcSource{dx, C, L, Bp};
  l.L = L;
  l.n_samples = B;
  l.m_valid = OC;
  for (int j = 0; j < k; ++j) l.segs.push_back(feb::tc::Seg{0, j - k / 2, 0, C / 64, j * C});
  l.bias = static_cast<const float*>(dbias);
  l.out = dy;
  l.out_ld = OC;
  l.out_rps = L;
  if (groups > 0) {
    l.stats = static_cast<double*>(dst);
    l.groups = groups;
    l.group_ch = group_ch;
  }
  int rc = 0;
  if (feb::tc_gemm(l, *ctx, ctx->stream, err) != cudaSuccess || cudaStreamSynchronize(ctx->stream) != cudaSuccess)
    rc = 2;
  if (rc == 0 && feb::take_device_error(*ctx, ctx->stream) != 0) rc = 3;
  if (rc == 0) {
    std::vector<uint16_t> yb(static_cast<size_t>(B) * L * OC);
    cudaMemcpy(yb.data(), dy, yb.size() * 2, cudaMemcpyDeviceToHost);
    for (size_t i = 0; i < yb.size(); ++i) {
      if (fp16) {
        y[i] = __half2float(__ushort_as_half(yb[i]));
      } else {
        const uint32_t bits = static_cast<uint32_t>(yb[i]) << 16;
        std::memcpy(&y[i], &bits, 4);
      }
    }
    if (groups > 0 && stats != nullptr) {
      std::vector<double> s(static_cast<size_t>(B) * groups * parts * 2);
      cudaMemcpy(s.data(), dst, s.size() * 8, cudaMemcpyDeviceToHost);
      for (int b = 0; b < B; ++b)
        for (int g = 0; g < groups; ++g) {
          double s1 = 0, s2 = 0;
          for (int p = 0; p < parts; ++p) {
            s1 += s[((static_cast<size_t>(b) * groups + g) * parts + p) * 2];
            s2 += s[((static_cast<size_t>(b) * groups + g) * parts + p) * 2 + 1];
          }
          stats[(static_cast<size_t>(b) * groups + g) * 2] = s1;
          stats[(static_cast<size_t>(b) * groups + g) * 2 + 1] = s2;
        }
    }
  }
  cudaFree(da);
  cudaFree(dx);
  cudaFree(dy);
  cudaFree(dbias);
  cudaFree(dst);
  return rc;
}

extern "C" int febtest_check_fp16_storable(const char* name, const float* w, size_t n, int bf16_mode, char* message,
                                           size_t message_len) {
  std::string err;
  const bool ok = feb::check_fp16_storable(name != nullptr ? name : "", w, n, bf16_mode != 0, err);
  if (message != nullptr && message_len > 0) {
    const size_t len = std::min(err.size(), message_len - 1);
    std::memcpy(message, err.data(), len);
    message[len] = '\0';
  }
  return ok ? 0 : 1;
}
