// Device-resident Mamba encoder (reference: src/core/models/mamba/mamba.cc).
//
// Per layer, tokens of all sequences at once (token-major [B*L][width]):
//   normed = RMSNorm(hidden)                     rmsnorm_kernel
//   [x | z] = normed W_in^T                      GEMM (fp32 out)
//   u = SiLU(causal depthwise conv(x) + b)       causal_conv_kernel, or the
//                                                in-projection's epilogue
//                                                (bf16 tensor path, sequences
//                                                that tile its token blocks)
//   [dt_in | B | C] = u W_x^T                    GEMM (fp32 out)
//   scan: dt = softplus(dt_in W_dt^T + b_dt) fused into the selective scan,
//         y = (D u + sum_n h_n C_n) * SiLU(z)   scan_kernel
//   hidden += y W_out^T                          GEMM (fp32 accumulate)
// then a final RMSNorm.  GEMMs use the weight-streaming CUDA-core kernel for
// short token counts and the tcgen05 GEMM (bf16 operands) for long ones in
// bf16 mode.  Streaming decode keeps the per-layer conv window and SSM state
// on the device in the reference's snapshot layout ([di][dc] window, newest
// last, then [ds][di] state).
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <map>
#include <tuple>

#include "runtime.cuh"
#include "simt.cuh"

namespace feb {
namespace {

constexpr int kTcMinTokens = 128;
constexpr int kMaxState = 16;
constexpr int kMaxRank = 64;
constexpr int kMaxConv = 8;  // causal conv width limit (register window)

std::uint16_t bf16_of(float v) {
  std::uint32_t u;
  std::memcpy(&u, &v, 4);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FC0;
  u += 0x7FFFu + ((u >> 16) & 1u);
  return static_cast<std::uint16_t>(u >> 16);
}

struct Mat {
  int rows = 0, rows_pad = 0, cols = 0, cols_pad = 0;
  void* w = nullptr;
  void* w3 = nullptr;  // fp32 engines: fp16 [rows_pad][3 cols_pad] = [hi | hi | lo] for the tensor path
  SimtSlice* slices = nullptr;
  int nslices = 0;
};

struct Layer {
  float* norm = nullptr;
  Mat in_proj, x_proj, out_proj;
  float* conv_w = nullptr;  // [di][dc]
  float* conv_b = nullptr;
  float* dt_w = nullptr;    // [di][dr] fp32 (widened)
  float* dt_b = nullptr;
  float* a_neg = nullptr;   // [ds][di] = -exp(A_log)^T (mamba.cc:167-176)
  float* d = nullptr;
};

// 16-bit GEMM operand of an activation: fp16(v) at [row][c] of a [rows][ld]
// matrix, or with split = 1 the pair hi = fp16(v) at [row][c], lo = fp16(v - hi)
// at [row][ld + c] of a [rows][2 ld] matrix (fp32 engines on the tensor cores)
__device__ __forceinline__ void store_act16(__half* base, long long row, int ld, int c, float v, int split) {
  const __half hi = to_half_sat(v);
  if (split) {
    base[row * 2 * ld + c] = hi;
    base[row * 2 * ld + ld + c] = __float2half_rn(v - __half2float(hi));
  } else {
    base[row * ld + c] = hi;
  }
}

// one warp per row; RMSNorm with eps 1e-5 (kernels_scalar.cc:48-60); optional
// 16-bit copy for the tensor-core GEMM (store_act16)
__global__ void rmsnorm_kernel(const float* in, const float* w, int rows, int dim, float* out, __half* out_bf,
                               int split) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* x = in + static_cast<long long>(row) * dim;
  float ss = 0.0f;
  for (int i = lane; i < dim; i += 32) ss = fmaf(x[i], x[i], ss);
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float scale = 1.0f / sqrtf((ss / static_cast<float>(dim)) + 1e-5f);
  for (int i = lane; i < dim; i += 32) {
    const float v = x[i] * scale * w[i];
    if (out != nullptr) out[static_cast<long long>(row) * dim + i] = v;
    if (out_bf != nullptr) store_act16(out_bf, row, dim, i, v, split);
  }
}

// rmsnorm_kernel for rows of 128 * NV floats: lane l holds the float4s at
// columns 4 l + 128 k of its row, all requested before the sum of squares
// (the per-lane partial sums run over k, then the warp reduction; the same
// value up to the order of that sum), and the 16-bit copy goes out 4 halves
// per store.
template <int NV>
__global__ void __launch_bounds__(256) rmsnorm_vec_kernel(const float* __restrict__ in, const float* __restrict__ w,
                                                          int rows, float* __restrict__ out,
                                                          __half* __restrict__ out_bf, int split) {
  constexpr int kDim = 128 * NV;
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float4* x = reinterpret_cast<const float4*>(in + static_cast<long long>(row) * kDim) + lane;
  float4 v[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) v[k] = x[32 * k];
  float ss = 0.0f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    ss = fmaf(v[k].x, v[k].x, ss);
    ss = fmaf(v[k].y, v[k].y, ss);
    ss = fmaf(v[k].z, v[k].z, ss);
    ss = fmaf(v[k].w, v[k].w, ss);
  }
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float scale = 1.0f / sqrtf((ss / static_cast<float>(kDim)) + 1e-5f);
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int c = 4 * (lane + 32 * k);
    const float4 wk = *reinterpret_cast<const float4*>(w + c);
    const float4 r = make_float4(v[k].x * scale * wk.x, v[k].y * scale * wk.y, v[k].z * scale * wk.z,
                                 v[k].w * scale * wk.w);
    if (out != nullptr) *reinterpret_cast<float4*>(out + static_cast<long long>(row) * kDim + c) = r;
    if (out_bf != nullptr) {
      const __half h0 = to_half_sat(r.x), h1 = to_half_sat(r.y), h2 = to_half_sat(r.z), h3 = to_half_sat(r.w);
      const __half2 p01 = __halves2half2(h0, h1), p23 = __halves2half2(h2, h3);
      const long long ob = split ? static_cast<long long>(row) * 2 * kDim + c : static_cast<long long>(row) * kDim + c;
      *reinterpret_cast<uint2*>(out_bf + ob) =
          make_uint2(*reinterpret_cast<const uint32_t*>(&p01), *reinterpret_cast<const uint32_t*>(&p23));
      if (split) {
        const __half2 l01 = __floats2half2_rn(r.x - __half2float(h0), r.y - __half2float(h1));
        const __half2 l23 = __floats2half2_rn(r.z - __half2float(h2), r.w - __half2float(h3));
        *reinterpret_cast<uint2*>(out_bf + ob + kDim) =
            make_uint2(*reinterpret_cast<const uint32_t*>(&l01), *reinterpret_cast<const uint32_t*>(&l23));
      }
    }
  }
}

// RMSNorm of many rows: the vector kernel for widths 128, 256, 512 and 1024
// (all pointers 16-byte aligned), else rmsnorm_kernel
void launch_rmsnorm(const float* in, const float* w, long long rows, int dim, float* out, __half* out_bf, int split,
                    cudaStream_t st) {
  const unsigned grid = static_cast<unsigned>((rows * 32 + 255) / 256);
  const bool al = (reinterpret_cast<std::uintptr_t>(in) | reinterpret_cast<std::uintptr_t>(w) |
                   reinterpret_cast<std::uintptr_t>(out) | reinterpret_cast<std::uintptr_t>(out_bf)) % 16 == 0;
  const int r = static_cast<int>(rows);
  if (al && dim == 512)
    rmsnorm_vec_kernel<4><<<grid, 256, 0, st>>>(in, w, r, out, out_bf, split);
  else if (al && dim == 1024)
    rmsnorm_vec_kernel<8><<<grid, 256, 0, st>>>(in, w, r, out, out_bf, split);
  else if (al && dim == 256)
    rmsnorm_vec_kernel<2><<<grid, 256, 0, st>>>(in, w, r, out, out_bf, split);
  else if (al && dim == 128)
    rmsnorm_vec_kernel<1><<<grid, 256, 0, st>>>(in, w, r, out, out_bf, split);
  else
    rmsnorm_kernel<<<grid, 256, 0, st>>>(in, w, r, dim, out, out_bf, split);
}

// u[b][t][c] = SiLU(bias[c] + sum_k w[c][k] * x[b][t - (dc-1) + k][c]), x is the
// first di columns of xz (row stride 2*di) (kernels_scalar.cc:10-27).
//
// Many sequences: one thread per (sequence, 4 channels) walks t with the last
// dc inputs in a register window (float4 loads and stores, each input read
// once).  The window is right-aligned in kMaxConv slots so every index is a
// compile-time constant; slots before the first step hold zeros, which the
// taps that reach before t = 0 multiply (the reference skips them: same sum).
__global__ void causal_conv_kernel(const float* __restrict__ xz, int B, int L, int di, int dc,
                                   const float* __restrict__ w, const float* __restrict__ bias, float* __restrict__ u,
                                   __half* __restrict__ u_bf, int split) {
  const int q = di >> 2;
  const long long total = static_cast<long long>(B) * q;
  const int first = kMaxConv - dc;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int b = static_cast<int>(i / q);
    const int c = static_cast<int>(i - static_cast<long long>(b) * q) * 4;
    float wk[4][kMaxConv];
#pragma unroll
    for (int j = 0; j < kMaxConv; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) wk[e][j] = j >= first ? w[(c + e) * dc + (j - first)] : 0.0f;
    const float4 bv = *reinterpret_cast<const float4*>(bias + c);
    float4 win[kMaxConv];
#pragma unroll
    for (int j = 0; j < kMaxConv; ++j) win[j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const long long tok0 = static_cast<long long>(b) * L;
    // the next step's input is requested one step ahead
    float4 ahead = __ldg(reinterpret_cast<const float4*>(xz + tok0 * 2 * di + c));
    for (int t = 0; t < L; ++t) {
#pragma unroll
      for (int j = 0; j + 1 < kMaxConv; ++j) win[j] = win[j + 1];
      win[kMaxConv - 1] = ahead;
      if (t + 1 < L) ahead = __ldg(reinterpret_cast<const float4*>(xz + (tok0 + t + 1) * 2 * di + c));
      float a0 = bv.x, a1 = bv.y, a2 = bv.z, a3 = bv.w;
#pragma unroll
      for (int j = 0; j < kMaxConv; ++j)
        if (j >= first) {
          a0 += wk[0][j] * win[j].x;
          a1 += wk[1][j] * win[j].y;
          a2 += wk[2][j] * win[j].z;
          a3 += wk[3][j] * win[j].w;
        }
      const float4 v = make_float4(silu_f(a0), silu_f(a1), silu_f(a2), silu_f(a3));
      const long long o = (tok0 + t) * di + c;
      *reinterpret_cast<float4*>(u + o) = v;
      if (u_bf != nullptr) {
        const __half h0 = to_half_sat(v.x), h1 = to_half_sat(v.y), h2 = to_half_sat(v.z), h3 = to_half_sat(v.w);
        const __half2 p01 = __halves2half2(h0, h1);
        const __half2 p23 = __halves2half2(h2, h3);
        const long long ob = split ? (tok0 + t) * 2 * di + c : o;
        *reinterpret_cast<uint2*>(u_bf + ob) =
            make_uint2(*reinterpret_cast<const uint32_t*>(&p01), *reinterpret_cast<const uint32_t*>(&p23));
        if (split) {
          const __half2 l01 = __floats2half2_rn(v.x - __half2float(h0), v.y - __half2float(h1));
          const __half2 l23 = __floats2half2_rn(v.z - __half2float(h2), v.w - __half2float(h3));
          *reinterpret_cast<uint2*>(u_bf + ob + di) =
              make_uint2(*reinterpret_cast<const uint32_t*>(&l01), *reinterpret_cast<const uint32_t*>(&l23));
        }
      }
    }
  }
}

// causal_conv_kernel for a compile-time width DC (4 for the encoders here):
// the window and weights take DC instead of kMaxConv registers, and each
// thread keeps its next kConvAhead inputs in flight (a ring of registers, the
// step loop unrolled by kConvAhead), so more threads per SM each with more
// loads outstanding.  Same expressions in the same order as
// causal_conv_kernel (window oldest to newest against weights 0 .. DC - 1).
constexpr int kConvAhead = 4;
template <int DC>
__global__ void __launch_bounds__(256) causal_conv_fixed_kernel(const float* __restrict__ xz, int B, int L, int di,
                                                                const float* __restrict__ w,
                                                                const float* __restrict__ bias, float* __restrict__ u,
                                                                __half* __restrict__ u_bf, int split) {
  const int q = di >> 2;
  const long long total = static_cast<long long>(B) * q;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int b = static_cast<int>(i / q);
    const int c = static_cast<int>(i - static_cast<long long>(b) * q) * 4;
    float wk[4][DC];
#pragma unroll
    for (int j = 0; j < DC; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) wk[e][j] = w[(c + e) * DC + j];
    const float4 bv = *reinterpret_cast<const float4*>(bias + c);
    float4 win[DC];
#pragma unroll
    for (int j = 0; j < DC; ++j) win[j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const long long tok0 = static_cast<long long>(b) * L;
    const float* src = xz + tok0 * 2 * di + c;
    float4 ahead[kConvAhead];
#pragma unroll
    for (int k = 0; k < kConvAhead; ++k)
      ahead[k] = k < L ? __ldg(reinterpret_cast<const float4*>(src + static_cast<long long>(k) * 2 * di))
                       : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (int t0 = 0; t0 < L; t0 += kConvAhead) {
#pragma unroll
      for (int k = 0; k < kConvAhead; ++k) {
        const int t = t0 + k;
        if (t >= L) break;
#pragma unroll
        for (int j = 0; j + 1 < DC; ++j) win[j] = win[j + 1];
        win[DC - 1] = ahead[k];
        if (t + kConvAhead < L)
          ahead[k] = __ldg(reinterpret_cast<const float4*>(src + static_cast<long long>(t + kConvAhead) * 2 * di));
        float a0 = bv.x, a1 = bv.y, a2 = bv.z, a3 = bv.w;
#pragma unroll
        for (int j = 0; j < DC; ++j) {
          a0 += wk[0][j] * win[j].x;
          a1 += wk[1][j] * win[j].y;
          a2 += wk[2][j] * win[j].z;
          a3 += wk[3][j] * win[j].w;
        }
        const float4 v = make_float4(silu_f(a0), silu_f(a1), silu_f(a2), silu_f(a3));
        const long long o = (tok0 + t) * di + c;
        *reinterpret_cast<float4*>(u + o) = v;
        if (u_bf != nullptr) {
          const __half h0 = to_half_sat(v.x), h1 = to_half_sat(v.y), h2 = to_half_sat(v.z), h3 = to_half_sat(v.w);
          const __half2 p01 = __halves2half2(h0, h1);
          const __half2 p23 = __halves2half2(h2, h3);
          const long long ob = split ? (tok0 + t) * 2 * di + c : o;
          *reinterpret_cast<uint2*>(u_bf + ob) =
              make_uint2(*reinterpret_cast<const uint32_t*>(&p01), *reinterpret_cast<const uint32_t*>(&p23));
          if (split) {
            const __half2 l01 = __floats2half2_rn(v.x - __half2float(h0), v.y - __half2float(h1));
            const __half2 l23 = __floats2half2_rn(v.z - __half2float(h2), v.w - __half2float(h3));
            *reinterpret_cast<uint2*>(u_bf + ob + di) =
                make_uint2(*reinterpret_cast<const uint32_t*>(&l01), *reinterpret_cast<const uint32_t*>(&l23));
          }
        }
      }
    }
  }
}

// Few sequences: one thread per (token, channel), the dc inputs re-read
__global__ void causal_conv_tok_kernel(const float* xz, int B, int L, int di, int dc, const float* w,
                                       const float* bias, float* u, __half* u_bf, int split) {
  const long long total = static_cast<long long>(B) * L * di;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long tok = i / di;
    const int c = static_cast<int>(i - tok * di);
    const int t = static_cast<int>(tok % L);
    float acc = bias[c];
    for (int k = 0; k < dc; ++k) {
      const int ti = t - (dc - 1) + k;
      if (ti >= 0) acc += w[c * dc + k] * xz[(tok - t + ti) * 2 * di + c];
    }
    const float v = silu_f(acc);
    u[i] = v;
    if (u_bf != nullptr) store_act16(u_bf, tok, di, c, v, split);
  }
}

// Selective scan with the dt projection fused in.  One thread per (sequence,
// channel), states in registers, sequential over t (kernels_scalar.cc:133-169):
//   dt = softplus(b_dt[c] + sum_r W_dt[c][r] dbl[t][r])
//   h_n = exp(dt A_n) h_n + dt B_n u ;  y = (D u + sum_n h_n C_n) * SiLU(z)
// dbl rows of the block's sequence are staged in shared memory.
// FAST (the bf16-activation path): exp(dt A) as 2^(dt A log2 e) by the
// hardware ex2 approximation with A pre-scaled, softplus and the SiLU gate
// through the fast exp / log intrinsics
template <int DS, int DR, bool FAST>
__global__ void __launch_bounds__(256) scan_kernel(const float* dbl, int wd, const float* u, const float* xz, int L,
                                                   int di, const float* dt_w, const float* dt_b, const float* a_neg,
                                                   const float* dsk, float* state, float* y, __half* y_bf,
                                                   int split) {
  static_assert(DR % 4 == 0 && DS % 4 == 0, "rows of [dt_in | B | C] are read as float4");
  extern __shared__ __align__(16) float sdbl[];  // [L][wd], wd = DR + 2 DS
  const int b = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  {
    // the sequence's rows as 16-byte copies, eight loads in flight per thread
    // (wd is a multiple of 4 and dbl 16-byte aligned)
    const float4* src = reinterpret_cast<const float4*>(dbl + static_cast<long long>(b) * L * wd);
    float4* dst = reinterpret_cast<float4*>(sdbl);
    const int n4 = L * wd / 4;
    constexpr int kBatch = 8;
    for (int i0 = threadIdx.x; i0 < n4; i0 += kBatch * blockDim.x) {
      float4 v[kBatch];
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        const int i = i0 + j * blockDim.x;
        if (i < n4) v[j] = __ldg(src + i);
      }
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        const int i = i0 + j * blockDim.x;
        if (i < n4) dst[i] = v[j];
      }
    }
  }
  __syncthreads();
  if (c >= di) return;
  float wdt[DR], an[DS], h[DS];
#pragma unroll
  for (int r = 0; r < DR; ++r) wdt[r] = dt_w[c * DR + r];
#pragma unroll
  for (int n = 0; n < DS; ++n) {
    an[n] = FAST ? a_neg[n * di + c] * 1.4426950408889634f : a_neg[n * di + c];
    h[n] = state != nullptr ? state[(static_cast<long long>(b) * DS + n) * di + c] : 0.0f;
  }
  const float bdt = dt_b[c], dk = dsk[c];
  // u and z of step t are requested kScanAhead steps earlier: the loop is
  // unrolled by kScanAhead, so slot j holds the values of steps t = j mod
  // kScanAhead and each load has kScanAhead steps of recurrence to complete
  constexpr int kScanAhead = 4;
  const long long tok0 = static_cast<long long>(b) * L;
  float u_ahead[kScanAhead], z_ahead[kScanAhead];
#pragma unroll
  for (int j = 0; j < kScanAhead; ++j) {
    u_ahead[j] = j < L ? u[(tok0 + j) * di + c] : 0.0f;
    z_ahead[j] = j < L ? xz[(tok0 + j) * 2 * di + di + c] : 0.0f;
  }
  for (int t0 = 0; t0 < L; t0 += kScanAhead) {
#pragma unroll
    for (int j = 0; j < kScanAhead; ++j) {
      const int t = t0 + j;
      if (t >= L) break;
      const float uv = u_ahead[j], zv = z_ahead[j];
      if (t + kScanAhead < L) {
        u_ahead[j] = u[(tok0 + t + kScanAhead) * di + c];
        z_ahead[j] = xz[(tok0 + t + kScanAhead) * 2 * di + di + c];
      }
      // the row as 16-byte shared-memory reads (same sums, same order)
      const float4* row4 = reinterpret_cast<const float4*>(sdbl + t * wd);
      float acc = 0.0f;
#pragma unroll
      for (int r = 0; r < DR / 4; ++r) {
        const float4 v = row4[r];
        acc += v.x * wdt[4 * r];
        acc += v.y * wdt[4 * r + 1];
        acc += v.z * wdt[4 * r + 2];
        acc += v.w * wdt[4 * r + 3];
      }
      const float pre = acc + bdt;
      const float dt = FAST ? fmaxf(pre, 0.0f) + __logf(1.0f + __expf(-fabsf(pre))) : softplus_f(pre);
      const long long tok = tok0 + t;
      float yv = dk * uv;
#pragma unroll
      for (int n4 = 0; n4 < DS / 4; ++n4) {
        const float4 bq = row4[DR / 4 + n4], cq = row4[(DR + DS) / 4 + n4];
        const float bn[4] = {bq.x, bq.y, bq.z, bq.w}, cn[4] = {cq.x, cq.y, cq.z, cq.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int n = 4 * n4 + i;
          const float da = FAST ? ex2_approx(dt * an[n]) : expf(dt * an[n]);
          const float dbu = dt * bn[i] * uv;
          h[n] = (da * h[n]) + dbu;
          yv += h[n] * cn[i];
        }
      }
      const float out = yv * (FAST ? silu_fast(zv) : (zv / (1.0f + expf(-zv))));
      y[tok * di + c] = out;
      if (y_bf != nullptr) store_act16(y_bf, tok, di, c, out, split);
    }
  }
  if (state != nullptr)
#pragma unroll
    for (int n = 0; n < DS; ++n) state[(static_cast<long long>(b) * DS + n) * di + c] = h[n];
}

// Selective scan for many sequences with staged inputs: one thread per
// (sequence, channel) as in scan_kernel, one CTA per (sequence, kScanThreads
// channels).  The sequence's [dt_in | B | C] rows and the CTA's u and z
// columns arrive by bulk copies in tiles of kScanTile steps, two tiles in
// flight.  A tile runs in two passes per thread:
//   A. for every step of the tile (independent of the state, so the steps
//      overlap): dt = softplus(dt_in . W_dt + b_dt) into the thread's slot of
//      a per-CTA buffer, the gate SiLU(z) over z in the stage;
//   B. the recurrence h_n = exp(dt A_n) h_n + dt B_n u, y = (D u + sum_n h_n
//      C_n) * gate, step after step.
// No CTA barrier per tile: each warp counts itself done with a stage on a
// shared-memory counter, and the warp that completes the count requests the
// stage's next tile.  Every warp waits on every tile's full barrier, so none
// runs more than one tile ahead of the slowest.
// FAST (the bf16 mode) runs on packed fp32 pairs (FFMA2 / FMUL2): the dt dot
// product as two interleaved pair sums, the states two at a time, sum_n h_n
// C_n as two pair sums, dt B u as (dt u) B; POLY of the DS / 2 state pairs take
// their exponential from exp2_poly2 on the FMA pipe rather than the MUFU unit,
// which carries the other 14 state exponentials and the 4 of softplus and
// SiLU per (token, channel).  The fp32 mode (!FAST) evaluates scan_kernel's
// expressions in scan_kernel's order.  y (fp32) is written only when given:
// the tensor-core out-projection reads the 16-bit copy.  U16 (bf16 mode with
// the conv in the in-projection's epilogue) stages u from its fp16 copy, the
// x-projection's operand, so the fp32 u is never written.  A full-barrier wait
// that times out records kErrStageTimeout and ends every warp's loop; the
// CTA waits (bounded) for the copies it issued and returns.
constexpr int kScanTile = 16;
constexpr int kScanThreads = 256;
constexpr int kScanWarps = kScanThreads / 32;
constexpr int kScanPolyPairs = 1;  // state pairs of the 16-state bf16 scan on exp2_poly2

// floats of one stage ([kScanTile][dr + 2 ds] dbl rows, then u and z
// [kScanTile][kScanThreads]), and of the whole dynamic shared memory (two
// stages and the dt buffer [kScanTile][kScanThreads])
__host__ __device__ constexpr int scan_stage_floats(int ds, int dr) {
  return kScanTile * (dr + 2 * ds + 2 * kScanThreads);
}
__host__ __device__ constexpr int scan_smem_floats(int ds, int dr) {
  return 2 * scan_stage_floats(ds, dr) + kScanTile * kScanThreads;
}

template <int DS, int DR, bool FAST, int POLY, bool U16 = false>
__global__ void __launch_bounds__(kScanThreads, 2)
    scan_staged_kernel(const float* __restrict__ dbl, const void* __restrict__ u, const float* __restrict__ xz, int L,
                       int di, const float* __restrict__ dt_w, const float* __restrict__ dt_b,
                       const float* __restrict__ a_neg, const float* __restrict__ dsk, float* __restrict__ y,
                       __half* __restrict__ y_bf, int split, int* err) {
  static_assert(DR % 4 == 0 && DS % 4 == 0 && POLY >= 0 && POLY <= DS / 2, "rows are read as float4");
  static_assert(!U16 || FAST, "the fp16 u belongs to the bf16 mode");
  constexpr int WD = DR + 2 * DS;
  constexpr int kStage = scan_stage_floats(DS, DR);
  extern __shared__ __align__(128) float sst[];
  float* sdt = sst + 2 * kStage;  // [kScanTile][kScanThreads] dt of the current tile, per thread
  __shared__ uint64_t full[2];
  __shared__ int done_warps[2], last_req[2], abort_word, zero_word;
  const int b = blockIdx.y, c0 = blockIdx.x * kScanThreads, tid = threadIdx.x, lane = tid & 31;
  const int nch = min(kScanThreads, di - c0);
  const int c = c0 + tid;
  const long long tok0 = static_cast<long long>(b) * L;
  const int ntiles = (L + kScanTile - 1) / kScanTile;
  if (tid == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    done_warps[0] = done_warps[1] = 0;
    last_req[0] = last_req[1] = -1;
    abort_word = zero_word = 0;
    fence_mbar_init();
  }
  __syncthreads();
  // one warp: tile `tile` into stage tile % 2 (lane 0 the dbl rows, lane j
  // the u and z row slices of step j; 16-byte aligned since di % 4 == 0, and
  // di % 8 == 0 for the fp16 u)
  auto request = [&](int tile) {
    const int s = tile & 1, t0 = tile * kScanTile, n = min(kScanTile, L - t0);
    float* sd = sst + s * kStage;
    float* su = sd + kScanTile * WD;
    float* sz = su + kScanTile * kScanThreads;
    if (lane == 0) {
      last_req[s] = tile;
      mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(n * WD * 4 + n * nch * (U16 ? 6 : 8)));
    }
    __syncwarp();
    if (lane == 0) bulk_load_g2s(sd, dbl + (tok0 + t0) * WD, static_cast<uint32_t>(n * WD * 4), &full[s]);
    if (lane < n) {
      const long long tok = tok0 + t0 + lane;
      if constexpr (U16)
        bulk_load_g2s(reinterpret_cast<__half*>(su) + lane * kScanThreads,
                      static_cast<const __half*>(u) + tok * di + c0, static_cast<uint32_t>(nch * 2), &full[s]);
      else
        bulk_load_g2s(su + lane * kScanThreads, static_cast<const float*>(u) + tok * di + c0,
                      static_cast<uint32_t>(nch * 4), &full[s]);
      bulk_load_g2s(sz + lane * kScanThreads, xz + tok * 2 * di + di + c0, static_cast<uint32_t>(nch * 4), &full[s]);
    }
  };
  if (tid < 32) {
    request(0);
    if (ntiles > 1) request(1);
  }
  const bool active = tid < nch;
  const int cc = active ? c : c0;  // idle threads of a ragged last CTA read channel c0's constants
  float wdt[DR], an[DS], h[DS];
#pragma unroll
  for (int r = 0; r < DR; ++r) wdt[r] = dt_w[cc * DR + r];
#pragma unroll
  for (int n = 0; n < DS; ++n) {
    an[n] = FAST ? a_neg[n * di + cc] * 1.4426950408889634f : a_neg[n * di + cc];
    h[n] = 0.0f;
  }
  const float bdt = dt_b[cc], dk = dsk[cc];
  bool failed = false;
  for (int tile = 0; tile < ntiles; ++tile) {
    const int s = tile & 1, t0 = tile * kScanTile, n = min(kScanTile, L - t0);
    const bool ok = __all_sync(0xffffffffu, mbar_wait(&full[s], static_cast<uint32_t>(tile >> 1) & 1u, &abort_word));
    if (!ok) {
      if (lane == 0) {
        atomicCAS(err, 0, kErrStageTimeout);
        atomicExch(&abort_word, 1);
      }
      failed = true;
      break;
    }
    const float* sd = sst + s * kStage;
    const float* su = sd + kScanTile * WD;
    float* sz = sst + s * kStage + kScanTile * WD + kScanTile * kScanThreads;
    if (active) {
      // A: dt and the gate of every step of the tile
#pragma unroll 4
      for (int j = 0; j < n; ++j) {
        const float4* row4 = reinterpret_cast<const float4*>(sd + j * WD);
        const float zv = sz[j * kScanThreads + tid];
        float dt, gate;
        if constexpr (FAST) {
          float2 acc0 = make_float2(0.0f, 0.0f), acc1 = make_float2(0.0f, 0.0f);
#pragma unroll
          for (int r = 0; r < DR / 4; ++r) {
            const float4 v = row4[r];
            acc0 = __ffma2_rn(make_float2(v.x, v.y), make_float2(wdt[4 * r], wdt[4 * r + 1]), acc0);
            acc1 = __ffma2_rn(make_float2(v.z, v.w), make_float2(wdt[4 * r + 2], wdt[4 * r + 3]), acc1);
          }
          const float pre = ((acc0.x + acc1.x) + (acc0.y + acc1.y)) + bdt;
          dt = fmaxf(pre, 0.0f) + __logf(1.0f + __expf(-fabsf(pre)));
          gate = silu_fast(zv);
        } else {
          float acc = 0.0f;
#pragma unroll
          for (int r = 0; r < DR / 4; ++r) {
            const float4 v = row4[r];
            acc += v.x * wdt[4 * r];
            acc += v.y * wdt[4 * r + 1];
            acc += v.z * wdt[4 * r + 2];
            acc += v.w * wdt[4 * r + 3];
          }
          dt = softplus_f(acc + bdt);
          gate = zv / (1.0f + expf(-zv));
        }
        sdt[j * kScanThreads + tid] = dt;
        sz[j * kScanThreads + tid] = gate;
      }
      // B: the recurrence
#pragma unroll 2
      for (int j = 0; j < n; ++j) {
        const float4* row4 = reinterpret_cast<const float4*>(sd + j * WD);
        const float dt = sdt[j * kScanThreads + tid];
        const float uv = U16 ? __half2float(reinterpret_cast<const __half*>(su)[j * kScanThreads + tid])
                             : su[j * kScanThreads + tid];
        const float gate = sz[j * kScanThreads + tid];
        float out;
        if constexpr (FAST) {
          const float dtu = dt * uv;
          const float2 dt2 = make_float2(dt, dt), dtu2 = make_float2(dtu, dtu);
          float2 y0 = make_float2(dk * uv, 0.0f), y1 = make_float2(0.0f, 0.0f);
#pragma unroll
          for (int q = 0; q < DS / 4; ++q) {
            const float4 bq = row4[DR / 4 + q], cq = row4[(DR + DS) / 4 + q];
#pragma unroll
            for (int half = 0; half < 2; ++half) {
              const int pr = 2 * q + half;  // states 2 pr and 2 pr + 1
              const float2 e = __fmul2_rn(dt2, make_float2(an[2 * pr], an[2 * pr + 1]));
              const float2 da = pr >= DS / 2 - POLY ? exp2_poly2(e) : make_float2(ex2_approx(e.x), ex2_approx(e.y));
              const float2 bn = half ? make_float2(bq.z, bq.w) : make_float2(bq.x, bq.y);
              const float2 cn = half ? make_float2(cq.z, cq.w) : make_float2(cq.x, cq.y);
              const float2 hn = __ffma2_rn(da, make_float2(h[2 * pr], h[2 * pr + 1]), __fmul2_rn(dtu2, bn));
              h[2 * pr] = hn.x;
              h[2 * pr + 1] = hn.y;
              if (half)
                y1 = __ffma2_rn(hn, cn, y1);
              else
                y0 = __ffma2_rn(hn, cn, y0);
            }
          }
          out = ((y0.x + y1.x) + (y0.y + y1.y)) * gate;
        } else {
          float yv = dk * uv;
#pragma unroll
          for (int q = 0; q < DS / 4; ++q) {
            const float4 bq = row4[DR / 4 + q], cq = row4[(DR + DS) / 4 + q];
            const float bn[4] = {bq.x, bq.y, bq.z, bq.w}, cn[4] = {cq.x, cq.y, cq.z, cq.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int st = 4 * q + i;
              const float da = expf(dt * an[st]);
              const float dbu = dt * bn[i] * uv;
              h[st] = (da * h[st]) + dbu;
              yv += h[st] * cn[i];
            }
          }
          out = yv * gate;
        }
        const long long tok = tok0 + t0 + j;
        if (y != nullptr) y[tok * di + c] = out;
        if (y_bf != nullptr) store_act16(y_bf, tok, di, c, out, split);
      }
    }
    // this warp is done with the stage; the warp completing the count requests
    // the stage's next tile (the gates were written into the stage by the
    // generic proxy, the copies write it through the async proxy)
    __syncwarp();
    int last = 0;
    if (lane == 0) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __threadfence_block();
      last = atomicAdd(&done_warps[s], 1) == kScanWarps * ((tile >> 1) + 1) - 1;
      __threadfence_block();
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last && tile + 2 < ntiles) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      request(tile + 2);
    }
  }
  if (__syncthreads_or(failed)) {
    // the copies this CTA issued may still be in flight: wait for each
    // stage's last request (bounded) before the shared memory is released
    if (tid == 0)
      for (int s = 0; s < 2; ++s)
        if (last_req[s] >= 0) mbar_wait(&full[s], static_cast<uint32_t>(last_req[s] >> 1) & 1u, &zero_word);
    __syncthreads();
  }
}

// Chunked selective scan for few sequences (the sequential kernel above runs
// one thread per (sequence, channel), so one sequence is 1024 threads walking
// all L steps).  The recurrence h_t = a_t h_(t-1) + b_t (a_t = exp(dt A),
// b_t = dt B_t u_t) is split into chunks of kScanChunk steps: thread
// (chunk w, channel c) first folds its chunk into (P, Q) = (prod a_t, the
// chunk's h from a zero start), the chunks' (P, Q) are combined in order
// through shared memory into the state entering each chunk, and a second pass
// replays the chunk from that state with scan_kernel's expressions.  State n
// at a time: y_t accumulates D u_t + sum_n h_t[n] C_t[n] in scan_kernel's n
// order.  A CTA holds kScanCh consecutive channels (coalesced loads) and all
// L / kScanChunk chunks; `state` (optional) is read as h_0 and receives h_L.
constexpr int kScanChunk = 8;
constexpr int kScanCh = 8;

template <int DS, int DR, bool FAST>
__global__ void scan_chunked_kernel(const float* dbl, int wd, const float* u, const float* xz, int L, int di,
                                    const float* dt_w, const float* dt_b, const float* a_neg, const float* dsk,
                                    float* state, float* y, __half* y_bf, int split) {
  extern __shared__ __align__(16) float sm[];
  float* sdbl = sm;                  // [L][wd]
  float* red = sdbl + L * wd;        // [2][nch][kScanCh][P, Q]
  const int nch = L / kScanChunk;
  const int b = blockIdx.y;
  const int w = threadIdx.x / kScanCh, sub = threadIdx.x - w * kScanCh;
  const int c = blockIdx.x * kScanCh + sub;
  const float* drow = dbl + static_cast<long long>(b) * L * wd;
  {
    // 16-byte copies, eight in flight per thread (wd is a multiple of 4)
    const int n4 = L * wd / 4;
    const float4* src = reinterpret_cast<const float4*>(drow);
    float4* dst = reinterpret_cast<float4*>(sdbl);
    for (int i0 = threadIdx.x; i0 < n4; i0 += 8 * blockDim.x) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = i0 + u * blockDim.x;
        v[u] = i < n4 ? src[i] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = i0 + u * blockDim.x;
        if (i < n4) dst[i] = v[u];
      }
    }
  }
  __syncthreads();
  const bool live = c < di;
  const int cc = live ? c : 0;
  const int t0 = w * kScanChunk;
  float dt[kScanChunk], uv[kScanChunk], yv[kScanChunk];
  {
    float wdt[DR];
#pragma unroll
    for (int r = 0; r < DR; ++r) wdt[r] = dt_w[cc * DR + r];
    const float bdt = dt_b[cc], dk = dsk[cc];
#pragma unroll
    for (int i = 0; i < kScanChunk; ++i) {
      const float* row = sdbl + (t0 + i) * wd;
      float acc = 0.0f;
#pragma unroll
      for (int r = 0; r < DR; ++r) acc += row[r] * wdt[r];
      const float pre = acc + bdt;
      dt[i] = FAST ? fmaxf(pre, 0.0f) + __logf(1.0f + __expf(-fabsf(pre))) : softplus_f(pre);
      const long long tok = static_cast<long long>(b) * L + t0 + i;
      uv[i] = live ? u[tok * di + cc] : 0.0f;
      yv[i] = dk * uv[i];
    }
  }
  for (int n = 0; n < DS; ++n) {
    const float an = FAST ? a_neg[n * di + cc] * 1.4426950408889634f : a_neg[n * di + cc];
    // pass 1: the chunk from a zero state
    float P = 1.0f, Q = 0.0f;
#pragma unroll
    for (int i = 0; i < kScanChunk; ++i) {
      const float da = FAST ? ex2_approx(dt[i] * an) : expf(dt[i] * an);
      const float dbu = dt[i] * sdbl[(t0 + i) * wd + DR + n] * uv[i];
      P *= da;
      Q = (da * Q) + dbu;
    }
    float* rd = red + (n & 1) * nch * kScanCh * 2;
    rd[(w * kScanCh + sub) * 2] = P;
    rd[(w * kScanCh + sub) * 2 + 1] = Q;
    __syncthreads();
    // state entering this chunk: the earlier chunks in order
    float h = (state != nullptr && live) ? state[(static_cast<long long>(b) * DS + n) * di + cc] : 0.0f;
    for (int v = 0; v < w; ++v) h = (rd[(v * kScanCh + sub) * 2] * h) + rd[(v * kScanCh + sub) * 2 + 1];
    // pass 2: the chunk from that state (scan_kernel's update)
#pragma unroll
    for (int i = 0; i < kScanChunk; ++i) {
      const float da = FAST ? ex2_approx(dt[i] * an) : expf(dt[i] * an);
      const float dbu = dt[i] * sdbl[(t0 + i) * wd + DR + n] * uv[i];
      h = (da * h) + dbu;
      yv[i] += h * sdbl[(t0 + i) * wd + DR + DS + n];
    }
    if (state != nullptr && live && w == nch - 1) state[(static_cast<long long>(b) * DS + n) * di + cc] = h;
  }
  if (!live) return;
#pragma unroll
  for (int i = 0; i < kScanChunk; ++i) {
    const long long tok = static_cast<long long>(b) * L + t0 + i;
    const float zv = xz[tok * 2 * di + di + cc];
    const float out = yv[i] * (FAST ? silu_fast(zv) : (zv / (1.0f + expf(-zv))));
    y[tok * di + cc] = out;
    if (y_bf != nullptr) store_act16(y_bf, tok, di, cc, out, split);
  }
}

// hidden[b][t] = embedding[token[b][t]]
__global__ void embed_kernel(const int* tokens, long long n_tok, const float* emb, int dm, float* hidden) {
  const long long total = n_tok * dm;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long tok = i / dm;
    const int c = static_cast<int>(i - tok * dm);
    hidden[i] = emb[static_cast<long long>(tokens[tok]) * dm + c];
  }
}

// last position of each sequence -> dense [B][dm]
__global__ void gather_last_kernel(const float* hidden, int B, int L, int dm, float* out) {
  const long long total = static_cast<long long>(B) * dm;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long b = i / dm;
    const int c = static_cast<int>(i - b * dm);
    out[i] = hidden[((b * L) + L - 1) * dm + c];
  }
}

// decode: shift the conv window, append x, conv + SiLU (mamba.cc:353-360)
__global__ void conv_step_kernel(const float* xz, int di, int dc, float* window, const float* w, const float* bias,
                                 float* u) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= di) return;
  float* wc = window + c * dc;
  for (int k = 0; k + 1 < dc; ++k) wc[k] = wc[k + 1];
  wc[dc - 1] = xz[c];
  float acc = bias[c];
  for (int k = 0; k < dc; ++k) acc += w[c * dc + k] * wc[k];
  u[c] = silu_f(acc);
}

// ---------------------------------------------------------------------------
// Fused streaming decode: one cooperative launch per token (mamba.cc:317-382).
// Every CTA is resident; phases are separated by a bounded grid barrier
// (monotonic arrival counter, release / acquire at GPU scope).  Per layer:
//   A. RMSNorm of the residual (each CTA computes the scale itself and stages
//      the normed row in shared memory); in_proj rows spread over all warps
//      (one warp per row, lanes stride K); the warp of x row c then steps the
//      conv window of channel c and writes u[c] = SiLU(conv)       | barrier
//   B. x_proj rows ([dt_in | B | C])                                 | barrier
//   C. dt_proj + softplus, selective-scan update and the SiLU(z) gate,
//      one thread per channel (scan_kernel's expression order)      | barrier
//   D. out_proj rows added to the residual                          | barrier
// then the final RMSNorm.  Data written inside the launch is read through L2
// (ld.global.cg); a channel's conv window and scan state are touched only by
// the thread that owns the channel.

constexpr int kDecThreads = 512;
constexpr int kDecWarps = kDecThreads / 32;

struct DecodeLayer {
  const void* w_in;   // [2 di][ld_in], fp32 or fp16
  const void* w_x;    // [dr + 2 ds][ld_x]
  const void* w_out;  // [dm][ld_out]
  int ld_in, ld_x, ld_out;
  const float *norm, *conv_w, *conv_b, *dt_w, *dt_b, *a_neg, *d;
};

struct DecodeParams {
  const DecodeLayer* layers;
  int n_layers, dm, di, ds, dc, dr;
  const int* token;
  const float* emb;
  const float* norm_f;
  float* state;  // [layers][di * (dc + ds)]: window [di][dc], then h [ds][di]
  float *x, *xz, *u, *dbl, *y, *out;
  unsigned* sync;  // [0] arrivals, [2] abort
  int* err;
};

__device__ __forceinline__ bool dec_grid_sync(const DecodeParams& p, unsigned& epoch) {
  return coop_grid_sync(p.sync, p.err, epoch);
}

// sum over a row of `n` weights times the shared / global vector v (one warp)
template <bool HALF>
__device__ __forceinline__ float warp_dot(const void* w, long long row, int ld, int n, const float* v) {
  float acc = 0.0f;
  const int lane = threadIdx.x & 31;
  // lane l takes pairs (k, k + 1), k = 2 l + 64 j; up to 16 pairs (all of a
  // 1024-long row) in flight before the first multiply
  constexpr int kPairs = 16;
  for (int k0 = lane * 2; k0 < n; k0 += 64 * kPairs) {
    float2 f2[kPairs];
#pragma unroll
    for (int u = 0; u < kPairs; ++u) {
      const int k = k0 + 64 * u;
      f2[u] = make_float2(0.0f, 0.0f);
      if (k < n) {
        if constexpr (HALF) {
          f2[u] = __half22float2(*reinterpret_cast<const __half2*>(static_cast<const __half*>(w) + row * ld + k));
        } else {
          f2[u] = *reinterpret_cast<const float2*>(static_cast<const float*>(w) + row * ld + k);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kPairs; ++u) {
      const int k = k0 + 64 * u;
      if (k < n) acc = fmaf(f2[u].x, v[k], acc);
      if (k + 1 < n) acc = fmaf(f2[u].y, v[k + 1], acc);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  return acc;
}

// RMSNorm scale of the residual (read through L2), every CTA on its own
__device__ float dec_rms_scale(const float* x, int dm, float* red) {
  float ss = 0.0f;
  for (int k = threadIdx.x; k < dm; k += blockDim.x) {
    const float v = __ldcg(x + k);
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float t = 0.0f;
  for (int w = 0; w < kDecWarps; ++w) t += red[w];
  __syncthreads();
  return 1.0f / sqrtf((t / static_cast<float>(dm)) + 1e-5f);
}

template <bool HALF>
__global__ void __launch_bounds__(kDecThreads, 1) mamba_decode_kernel(const DecodeParams p) {
  extern __shared__ float sh[];  // [max(dm, di)] staged input vector
  __shared__ float red[kDecWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // index i belongs to CTA i % gridDim.x: short loops still spread over every SM
  const int gwarp = warp * gridDim.x + blockIdx.x, nwarps = gridDim.x * kDecWarps;
  const int gthread = threadIdx.x * gridDim.x + blockIdx.x, nthreads = gridDim.x * blockDim.x;
  const int dm = p.dm, di = p.di, ds = p.ds, dc = p.dc, dr = p.dr, wd = dr + 2 * ds;
  unsigned epoch = 0;
  const int tok = *p.token;
  for (int k = gthread; k < dm; k += nthreads) p.x[k] = p.emb[static_cast<long long>(tok) * dm + k];
  if (!dec_grid_sync(p, epoch)) return;
  const std::size_t per = static_cast<std::size_t>(di) * (dc + ds);
  for (int li = 0; li < p.n_layers; ++li) {
    const DecodeLayer L = p.layers[li];
    float* window = p.state + li * per;
    float* h = window + static_cast<std::size_t>(di) * dc;
    // A. normed row (x * scale * w, kernels_scalar.cc:48-60), in_proj, conv step
    const float scale = dec_rms_scale(p.x, dm, red);
    for (int k = threadIdx.x; k < dm; k += blockDim.x) sh[k] = __ldcg(p.x + k) * scale * L.norm[k];
    __syncthreads();
    for (int r = gwarp; r < 2 * di; r += nwarps) {
      const float v = warp_dot<HALF>(L.w_in, r, L.ld_in, dm, sh);
      if (lane == 0) {
        p.xz[r] = v;
        if (r < di) {  // conv_step_kernel: shift, append, conv + bias, SiLU
          float* wc = window + static_cast<long long>(r) * dc;
          for (int k = 0; k + 1 < dc; ++k) wc[k] = wc[k + 1];
          wc[dc - 1] = v;
          float acc = L.conv_b[r];
          for (int k = 0; k < dc; ++k) acc += L.conv_w[r * dc + k] * wc[k];
          p.u[r] = silu_f(acc);
        }
      }
    }
    if (!dec_grid_sync(p, epoch)) return;
    // B. x_proj
    for (int k = threadIdx.x; k < di; k += blockDim.x) sh[k] = __ldcg(p.u + k);
    __syncthreads();
    for (int r = gwarp; r < wd; r += nwarps) {
      const float v = warp_dot<HALF>(L.w_x, r, L.ld_x, di, sh);
      if (lane == 0) p.dbl[r] = v;
    }
    if (!dec_grid_sync(p, epoch)) return;
    // C. scan step per channel (scan_kernel order, non-FAST)
    for (int k = threadIdx.x; k < wd; k += blockDim.x) sh[k] = __ldcg(p.dbl + k);
    __syncthreads();
    for (int c = gthread; c < di; c += nthreads) {
      float acc = 0.0f;
      for (int r = 0; r < dr; ++r) acc += sh[r] * L.dt_w[c * dr + r];
      const float dt = softplus_f(acc + L.dt_b[c]);
      const float uv = __ldcg(p.u + c);
      float yv = L.d[c] * uv;
      for (int n = 0; n < ds; ++n) {
        const float da = expf(dt * L.a_neg[n * di + c]);
        const float dbu = dt * sh[dr + n] * uv;
        const float hn = (da * h[static_cast<long long>(n) * di + c]) + dbu;
        h[static_cast<long long>(n) * di + c] = hn;
        yv += hn * sh[dr + ds + n];
      }
      const float zv = __ldcg(p.xz + di + c);
      p.y[c] = yv * (zv / (1.0f + expf(-zv)));
    }
    if (!dec_grid_sync(p, epoch)) return;
    // D. out_proj added to the residual
    for (int k = threadIdx.x; k < di; k += blockDim.x) sh[k] = __ldcg(p.y + k);
    __syncthreads();
    for (int r = gwarp; r < dm; r += nwarps) {
      const float v = warp_dot<HALF>(L.w_out, r, L.ld_out, di, sh);
      if (lane == 0) p.x[r] = __ldcg(p.x + r) + v;
    }
    if (!dec_grid_sync(p, epoch)) return;
  }
  // final RMSNorm
  const float scale = dec_rms_scale(p.x, dm, red);
  for (int k = gthread; k < dm; k += nthreads) p.out[k] = __ldcg(p.x + k) * scale * p.norm_f[k];
}

class Mamba final : public MambaDevice {
 public:
  Mamba(std::shared_ptr<DeviceContext> ctx, Precision prec) : ctx_(std::move(ctx)), prec_(prec) {}
  ~Mamba() override {
    if (step_graph_ != nullptr) cudaGraphExecDestroy(step_graph_);
    for (auto& [k, g] : fwd_graphs_) cudaGraphExecDestroy(g);
    if (pinned_ != nullptr) cudaFreeHost(pinned_);
  }
  bool load(const TensorTable& t, std::string& err);
  const MambaConfig& config() const noexcept override { return cfg_; }
  std::size_t capacity() const noexcept override { return cap_tokens_; }
  int reserve(std::size_t batch, std::size_t max_len, std::string& err) noexcept override;
  int forward(const std::int32_t* tokens, std::size_t batch, std::size_t len, float* hidden, bool last_only,
              std::string& err) noexcept override;
  const float* last_hidden_device() const noexcept override { return last_; }
  int forward_device(const std::int32_t* tokens, std::size_t batch, std::size_t len, float* last_hidden, void* stream,
                     std::string& err) noexcept override;
  int step(std::int32_t token, float* out, std::string& err) noexcept override;
  void reset() noexcept override;
  std::size_t state_floats() const noexcept override {
    return cfg_.n_layers * cfg_.d_inner * (cfg_.d_conv + cfg_.d_state);
  }
  int read_state(float* dst, std::string& err) noexcept override;
  int write_state(const float* src, std::string& err) noexcept override;

 private:
  // conv: the layer whose causal conv runs in the epilogue (tensor path,
  // in-projection; sequences of conv_seq tokens; u to u_ (fp32, when
  // conv_u32) and ub_ (fp16))
  bool gemm(const Mat& m, const void* in, int in_ld, long long n_tok, float* out, int out_ld, bool accumulate,
            bool tc, cudaStream_t st, std::string& err, const Layer* conv = nullptr, int conv_seq = 0,
            bool conv_u32 = true);
  bool run_layers(long long n_tok, int B, int L, bool tc, cudaStream_t st, std::string& err);
  // one decode token: the token from pinned_[0], the normed output to pinned_ + 1
  bool record_step(cudaStream_t st, std::string& err);

  std::shared_ptr<DeviceContext> ctx_;
  Precision prec_;
  MambaConfig cfg_{};
  DeviceArena wts_, ws_;
  float* emb_ = nullptr;
  float* norm_f_ = nullptr;
  std::vector<Layer> layers_;
  std::size_t cap_tokens_ = 0, cap_batch_ = 0, cap_rows_ = 0;
  int* tokens_ = nullptr;
  float *hidden_ = nullptr, *xz_ = nullptr, *u_ = nullptr, *dbl_ = nullptr, *y_ = nullptr, *part_ = nullptr;
  float* last_ = nullptr;
  float* out_ = nullptr;
  __half *nb_ = nullptr, *ub_ = nullptr, *yb_ = nullptr;
  float* state_ = nullptr;  // decode state (snapshot layout)
  float* dh_ = nullptr;     // decode scratch
  std::size_t part_elems_ = 0;
  float* pinned_ = nullptr;
  std::size_t pinned_floats_ = 0;
  // the decode step as one graph (token upload, every layer, output download);
  // rebuilt after reserve() moves the buffers
  cudaGraphExec_t step_graph_ = nullptr;
  // prefill kernels (embedding .. last-position gather) as one graph per
  // (batch, length, destination); rebuilt after reserve() moves the buffers
  std::map<std::tuple<std::size_t, std::size_t, const float*>, cudaGraphExec_t> fwd_graphs_;
  // fused decode (one cooperative launch per token) when the whole grid fits
  DecodeLayer* dec_layers_ = nullptr;
  unsigned* dec_sync_ = nullptr;
  bool dec_fused_ = false;
};

bool Mamba::load(const TensorTable& t, std::string& err) {
  const HostTensor* emb = t.find("backbone.embeddings.weight");
  const HostTensor* a0 = t.find("backbone.layers.0.mixer.A_log");
  const HostTensor* cv0 = t.find("backbone.layers.0.mixer.conv1d.weight");
  const HostTensor* xp0 = t.find("backbone.layers.0.mixer.x_proj.weight");
  const HostTensor* nf = t.find("backbone.norm_f.weight");
  if (emb == nullptr || a0 == nullptr || cv0 == nullptr || xp0 == nullptr || nf == nullptr || emb->ndim != 2 ||
      a0->ndim != 2 || cv0->ndim != 3 || xp0->ndim != 2 || emb->dtype != DType::F32 || a0->dtype != DType::F32) {
    err = "backbone.* tensors missing or malformed";
    return false;
  }
  cfg_.vocab = emb->shape[0];
  cfg_.d_model = emb->shape[1];
  cfg_.d_inner = a0->shape[0];
  cfg_.d_state = a0->shape[1];
  cfg_.d_conv = cv0->shape[2];
  if (xp0->shape[0] < 2 * cfg_.d_state) {
    err = "x_proj is narrower than 2 * d_state";
    return false;
  }
  cfg_.dt_rank = xp0->shape[0] - 2 * cfg_.d_state;
  if (cfg_.d_state > static_cast<std::size_t>(kMaxState) || cfg_.dt_rank > static_cast<std::size_t>(kMaxRank) ||
      cfg_.d_model % 8 != 0 || cfg_.d_inner % 8 != 0 || cfg_.d_conv < 1 ||
      cfg_.d_conv > static_cast<std::size_t>(kMaxConv)) {
    err = "Mamba dimensions outside this build's limits (d_state <= 16, dt_rank <= 64, d_conv <= 8)";
    return false;
  }
  const std::size_t dm = cfg_.d_model, di = cfg_.d_inner, ds = cfg_.d_state, dc = cfg_.d_conv, dr = cfg_.dt_rank;
  std::size_t n = 0;
  while (n < 64 && t.find("backbone.layers." + std::to_string(n) + ".norm.weight") != nullptr) ++n;
  cfg_.n_layers = n;
  if (n == 0) {
    err = "no Mamba layers";
    return false;
  }
  const bool bf = prec_ == Precision::kBF16;
  auto mat_bytes = [&](std::size_t rows, std::size_t cols) {
    const std::size_t rp = (rows + 127) / 128 * 128, cp = (cols + 63) / 64 * 64;
    // bf16: 16-bit W; fp32: fp32 W (CUDA cores) and the [hi | hi | lo] fp16 copy
    return rp * cp * (bf ? 2 : 4 + 6) + ((cp + 255) / 256) * sizeof(SimtSlice) + 1024;
  };
  ArenaPlan plan;
  plan.add_n<float>(cfg_.vocab * dm + dm);
  for (std::size_t i = 0; i < n; ++i) {
    plan.add(mat_bytes(2 * di, dm));
    plan.add(mat_bytes(dr + 2 * ds, di));
    plan.add(mat_bytes(dm, di));
    plan.add_n<float>(dm + di * dc + di + di * dr + di + ds * di + di);
  }
  if (!wts_.init(plan.total(), err)) return false;
  auto get = [&](std::size_t layer, const std::string& sub, std::initializer_list<std::size_t> shape,
                 bool allow_bf16, std::vector<float>& out) {
    const std::string name = "backbone.layers." + std::to_string(layer) + "." + sub;
    const HostTensor* h = t.find(name);
    if (h == nullptr || h->ndim != static_cast<int>(shape.size()) || (!allow_bf16 && h->dtype != DType::F32)) {
      err = "tensor " + name + " missing or malformed";
      return false;
    }
    int i = 0;
    for (std::size_t s : shape)
      if (h->shape[static_cast<std::size_t>(i++)] != s) {
        err = "tensor " + name + " has an unexpected shape";
        return false;
      }
    out = widen_f32(*h);
    // the in / x / out projections are held in fp16 (dt_proj stays fp32)
    if (allow_bf16 && sub.find("_proj.weight") != std::string::npos && sub.find("dt_proj") == std::string::npos &&
        !check_fp16_storable(name, out.data(), out.size(), bf, err))
      return false;
    return true;
  };
  auto put = [&](const std::vector<float>& h) {
    float* d = wts_.take_n<float>(h.size());
    cudaMemcpy(d, h.data(), h.size() * 4, cudaMemcpyHostToDevice);
    return d;
  };
  auto put_mat = [&](const std::vector<float>& w, int rows, int cols, Mat& m) {
    m.rows = rows;
    m.cols = cols;
    m.rows_pad = (rows + 127) / 128 * 128;
    m.cols_pad = (cols + 63) / 64 * 64;
    std::vector<float> padded(static_cast<std::size_t>(m.rows_pad) * m.cols_pad, 0.0f);
    for (int r = 0; r < rows; ++r)
      std::memcpy(&padded[static_cast<std::size_t>(r) * m.cols_pad], &w[static_cast<std::size_t>(r) * cols],
                  static_cast<std::size_t>(cols) * 4);
    if (bf) {
      std::vector<std::uint16_t> hb(padded.size());
      for (std::size_t i = 0; i < hb.size(); ++i) hb[i] = fp16_bits_of_bf16_rounded(padded[i]);
      m.w = wts_.take(hb.size() * 2);
      cudaMemcpy(m.w, hb.data(), hb.size() * 2, cudaMemcpyHostToDevice);
    } else {
      m.w = put(padded);
      // [hi | hi | lo] rows for the fp32 tensor path
      const std::size_t cp = static_cast<std::size_t>(m.cols_pad);
      std::vector<std::uint16_t> h3(padded.size() * 3);
      for (std::size_t r = 0; r < static_cast<std::size_t>(m.rows_pad); ++r)
        for (std::size_t c = 0; c < cp; ++c) {
          const float v = padded[r * cp + c];
          const __half hi = __float2half_rn(v);
          h3[r * 3 * cp + c] = __half_as_ushort(hi);
          h3[r * 3 * cp + cp + c] = __half_as_ushort(hi);
          h3[r * 3 * cp + 2 * cp + c] = __half_as_ushort(__float2half_rn(v - __half2float(hi)));
        }
      m.w3 = wts_.take(h3.size() * 2);
      cudaMemcpy(m.w3, h3.data(), h3.size() * 2, cudaMemcpyHostToDevice);
    }
    std::vector<SimtSlice> sl;
    for (int c = 0; c < m.cols_pad; c += 256) sl.push_back(SimtSlice{0, 0, c, std::min(256, m.cols_pad - c), c});
    m.nslices = static_cast<int>(sl.size());
    m.slices = wts_.take_n<SimtSlice>(sl.size());
    cudaMemcpy(m.slices, sl.data(), sl.size() * sizeof(SimtSlice), cudaMemcpyHostToDevice);
  };
  emb_ = put(widen_f32(*emb));
  {
    const HostTensor* nfw = t.find("backbone.norm_f.weight");
    if (nfw->ndim != 1 || nfw->shape[0] != dm || nfw->dtype != DType::F32) {
      err = "backbone.norm_f.weight malformed";
      return false;
    }
    norm_f_ = put(widen_f32(*nfw));
  }
  layers_.resize(n);
  for (std::size_t i = 0; i < n; ++i) {
    Layer& L = layers_[i];
    std::vector<float> v;
    if (!get(i, "norm.weight", {dm}, false, v)) return false;
    L.norm = put(v);
    if (!get(i, "mixer.in_proj.weight", {2 * di, dm}, true, v)) return false;
    put_mat(v, static_cast<int>(2 * di), static_cast<int>(dm), L.in_proj);
    if (!get(i, "mixer.conv1d.weight", {di, 1, dc}, false, v)) return false;
    L.conv_w = put(v);
    if (!get(i, "mixer.conv1d.bias", {di}, false, v)) return false;
    L.conv_b = put(v);
    if (!get(i, "mixer.x_proj.weight", {dr + 2 * ds, di}, true, v)) return false;
    put_mat(v, static_cast<int>(dr + 2 * ds), static_cast<int>(di), L.x_proj);
    if (!get(i, "mixer.dt_proj.weight", {di, dr}, true, v)) return false;
    if (bf) {  // the bf16 mode rounds every projection weight
      for (float& x : v) {
        const std::uint32_t bits = static_cast<std::uint32_t>(bf16_of(x)) << 16;
        std::memcpy(&x, &bits, 4);
      }
    }
    L.dt_w = put(v);
    if (!get(i, "mixer.dt_proj.bias", {di}, false, v)) return false;
    L.dt_b = put(v);
    if (!get(i, "mixer.A_log", {di, ds}, false, v)) return false;
    std::vector<float> an(ds * di);
    for (std::size_t s = 0; s < ds; ++s)
      for (std::size_t c = 0; c < di; ++c) an[s * di + c] = -std::exp(v[c * ds + s]);
    L.a_neg = put(an);
    if (!get(i, "mixer.D", {di}, false, v)) return false;
    L.d = put(v);
    if (!get(i, "mixer.out_proj.weight", {dm, di}, true, v)) return false;
    put_mat(v, static_cast<int>(dm), static_cast<int>(di), L.out_proj);
  }
  if (wts_.overflowed()) {
    err = "internal error: Mamba weight arena too small";
    return false;
  }
  for (const void* k : {reinterpret_cast<const void*>(scan_chunked_kernel<16, 32, false>),
                        reinterpret_cast<const void*>(scan_chunked_kernel<16, 32, true>),
                        reinterpret_cast<const void*>(scan_chunked_kernel<8, 4, false>),
                        reinterpret_cast<const void*>(scan_chunked_kernel<8, 4, true>),
                        reinterpret_cast<const void*>(scan_chunked_kernel<4, 4, false>),
                        reinterpret_cast<const void*>(scan_chunked_kernel<4, 4, true>),
                        reinterpret_cast<const void*>(scan_kernel<16, 32, false>),
                        reinterpret_cast<const void*>(scan_kernel<16, 32, true>),
                        reinterpret_cast<const void*>(scan_kernel<8, 4, false>),
                        reinterpret_cast<const void*>(scan_kernel<8, 4, true>),
                        reinterpret_cast<const void*>(scan_kernel<4, 4, false>),
                        reinterpret_cast<const void*>(scan_kernel<4, 4, true>),
                        reinterpret_cast<const void*>(scan_staged_kernel<16, 32, false, 0>),
                        reinterpret_cast<const void*>(scan_staged_kernel<16, 32, true, kScanPolyPairs>),
                        reinterpret_cast<const void*>(scan_staged_kernel<16, 32, true, kScanPolyPairs, true>),
                        reinterpret_cast<const void*>(scan_staged_kernel<8, 4, true, 0, true>),
                        reinterpret_cast<const void*>(scan_staged_kernel<4, 4, true, 0, true>),
                        reinterpret_cast<const void*>(scan_staged_kernel<8, 4, false, 0>),
                        reinterpret_cast<const void*>(scan_staged_kernel<8, 4, true, 0>),
                        reinterpret_cast<const void*>(scan_staged_kernel<4, 4, false, 0>),
                        reinterpret_cast<const void*>(scan_staged_kernel<4, 4, true, 0>)})
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  if (cudaDeviceSynchronize() != cudaSuccess) {
    err = "Mamba weight upload failed";
    return false;
  }
  return true;
}

int Mamba::reserve(std::size_t batch, std::size_t max_len, std::string& err) noexcept {
  if (batch == 0) batch = 1;
  if (max_len == 0) max_len = 512;
  const std::size_t tokens = batch * max_len;
  if (tokens <= cap_tokens_ && batch <= cap_batch_) return 0;
  if (step_graph_ != nullptr) {
    cudaGraphExecDestroy(step_graph_);
    step_graph_ = nullptr;
  }
  for (auto& [k, g] : fwd_graphs_) cudaGraphExecDestroy(g);
  fwd_graphs_.clear();
  const std::size_t dm = cfg_.d_model, di = cfg_.d_inner, wd = cfg_.dt_rank + 2 * cfg_.d_state;
  const std::size_t rows = (tokens + 255) / 256 * 256;
  std::size_t nsl = 1;
  for (const Layer& L : layers_)
    nsl = std::max({nsl, static_cast<std::size_t>(L.in_proj.nslices), static_cast<std::size_t>(L.x_proj.nslices),
                    static_cast<std::size_t>(L.out_proj.nslices)});
  // split-K partials are only used on the CUDA-core path (short inputs)
  const std::size_t simt_tokens = std::min<std::size_t>(tokens, 4096);
  part_elems_ = nsl * simt_tokens * 2 * di;
  ArenaPlan plan;
  plan.add_n<int>(rows);
  plan.add_n<float>(rows * dm);       // hidden
  plan.add_n<float>(rows * 2 * di);   // xz
  plan.add_n<float>(rows * di);       // u
  plan.add_n<float>(rows * wd);       // dbl
  plan.add_n<float>(rows * di);       // y
  plan.add_n<float>(part_elems_);
  plan.add_n<float>(batch * dm);      // last
  plan.add_n<float>(rows * dm);       // out
  plan.add_n<__half>(rows * 2 * dm);
  plan.add_n<__half>(rows * 2 * di);
  plan.add_n<__half>(rows * 2 * di);
  plan.add_n<float>(state_floats());
  plan.add_n<float>(dm + 2 * di + di + wd + di + di + dm + 64);
  plan.add_n<DecodeLayer>(layers_.size());
  plan.add_n<unsigned>(4);
  // keep the decode state across a re-reserve
  std::vector<float> saved;
  if (state_ != nullptr) {
    saved.resize(state_floats());
    cudaMemcpy(saved.data(), state_, saved.size() * 4, cudaMemcpyDeviceToHost);
  }
  ws_.release();
  if (!ws_.init(plan.total(), err)) {
    cap_tokens_ = 0;
    return 2;
  }
  tokens_ = ws_.take_n<int>(rows);
  hidden_ = ws_.take_n<float>(rows * dm);
  xz_ = ws_.take_n<float>(rows * 2 * di);
  u_ = ws_.take_n<float>(rows * di);
  dbl_ = ws_.take_n<float>(rows * wd);
  y_ = ws_.take_n<float>(rows * di);
  part_ = ws_.take_n<float>(part_elems_);
  last_ = ws_.take_n<float>(batch * dm);
  out_ = ws_.take_n<float>(rows * dm);
  nb_ = ws_.take_n<__half>(rows * 2 * dm);  // room for hi / lo pairs (fp32 engines)
  ub_ = ws_.take_n<__half>(rows * 2 * di);
  yb_ = ws_.take_n<__half>(rows * 2 * di);
  state_ = ws_.take_n<float>(state_floats());
  dh_ = ws_.take_n<float>(dm + 2 * di + di + wd + di + di + dm + 64);
  dec_layers_ = ws_.take_n<DecodeLayer>(layers_.size());
  dec_sync_ = ws_.take_n<unsigned>(4);
  if (ws_.overflowed()) {
    err = "internal error: Mamba workspace arena too small";
    cap_tokens_ = 0;
    return 2;
  }
  cudaMemset(tokens_, 0, ws_.used());
  {
    std::vector<DecodeLayer> dl(layers_.size());
    for (std::size_t i = 0; i < layers_.size(); ++i) {
      const Layer& Ly = layers_[i];
      dl[i] = DecodeLayer{Ly.in_proj.w, Ly.x_proj.w, Ly.out_proj.w, Ly.in_proj.cols_pad, Ly.x_proj.cols_pad,
                          Ly.out_proj.cols_pad, Ly.norm, Ly.conv_w, Ly.conv_b, Ly.dt_w, Ly.dt_b, Ly.a_neg, Ly.d};
    }
    cudaMemcpy(dec_layers_, dl.data(), dl.size() * sizeof(DecodeLayer), cudaMemcpyHostToDevice);
    // the fused decode needs one resident CTA per SM (cooperative launch)
    const std::size_t smem = std::max({dm, di, wd}) * 4;
    int per_sm = 0;
    const bool half = prec_ == Precision::kBF16;
    const cudaError_t oc = half ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, mamba_decode_kernel<true>,
                                                                               kDecThreads, smem)
                                : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, mamba_decode_kernel<false>,
                                                                               kDecThreads, smem);
    dec_fused_ = oc == cudaSuccess && per_sm >= 1;
    cudaGetLastError();
  }
  if (!saved.empty()) cudaMemcpy(state_, saved.data(), saved.size() * 4, cudaMemcpyHostToDevice);
  const std::size_t need = tokens * (dm + 1) + state_floats();
  if (pinned_floats_ < need) {
    if (pinned_ != nullptr) cudaFreeHost(pinned_);
    pinned_ = nullptr;
    if (counted_host_malloc(reinterpret_cast<void**>(&pinned_), need * 4) != cudaSuccess) {
      err = "pinned host allocation failed";
      return 2;
    }
    pinned_floats_ = need;
  }
  cap_tokens_ = tokens;
  cap_batch_ = batch;
  cap_rows_ = rows;
  return cudaDeviceSynchronize() == cudaSuccess ? 0 : 2;
}

bool Mamba::gemm(const Mat& m, const void* in, int in_ld, long long n_tok, float* out, int out_ld, bool accumulate,
                 bool tc, cudaStream_t st, std::string& err, const Layer* conv, int conv_seq, bool conv_u32) {
  if (tc) {
    TcLaunch l;
    l.fp16 = true;
    l.M_rows = m.rows_pad;
    l.L = 1;
    l.n_samples = static_cast<int>(n_tok);
    l.m_valid = m.rows;
    const int kb = m.cols_pad / 64;
    if (prec_ != Precision::kBF16) {
      // fp32 engine: [hi(W) | hi(W) | lo(W)] against [hi(x) | lo(x)] (segments hi, lo, hi)
      l.A = m.w3;
      l.K = 3 * m.cols_pad;
      l.src[0] = TcSource{in, 2 * in_ld, 1, static_cast<int>(cap_rows_)};
      l.segs = {tc::Seg{0, 0, 0, kb, 0}, tc::Seg{0, 0, in_ld, kb, m.cols_pad}, tc::Seg{0, 0, 0, kb, 2 * m.cols_pad}};
    } else {
      l.A = m.w;
      l.K = m.cols_pad;
      l.src[0] = TcSource{in, in_ld, 1, static_cast<int>(cap_rows_)};
      l.segs = {tc::Seg{0, 0, 0, kb, 0}};
    }
    l.out_f32 = true;
    l.out_accumulate = accumulate;
    l.out = out;
    l.out_ld = out_ld;
    if (conv != nullptr) {
      // in-projection with the causal conv in its epilogue: x half -> u (fp32
      // and the fp16 operand of the x-projection), z half -> out
      l.conv_w = conv->conv_w;
      l.conv_b = conv->conv_b;
      l.conv_u = conv_u32 ? u_ : nullptr;
      l.conv_u16 = ub_;
      l.conv_rows = static_cast<int>(cfg_.d_inner);
      l.conv_seq = conv_seq;
      l.conv_ld = static_cast<int>(cfg_.d_inner);
    }
    return tc_gemm(l, *ctx_, st, err) == cudaSuccess;
  }
  // CUDA-core path, chunks of <= 4096 tokens through the partial buffer
  for (long long t0 = 0; t0 < n_tok; t0 += 4096) {
    const long long nt_tok = std::min<long long>(4096, n_tok - t0);
    SimtConvParams p{};
    p.W = m.w;
    p.M = m.rows;
    p.K = m.cols_pad;
    p.src[0] = SimtSource{static_cast<const float*>(in) + t0 * in_ld, in_ld, 1};
    p.stride = 1;
    p.L_out = 1;
    p.n_tokens = static_cast<int>(nt_tok);
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
    r.n_tokens = p.n_tokens;
    r.M = m.rows;
    r.act = 0;
    r.out = out + t0 * out_ld;
    r.out_ld = out_ld;
    r.accumulate = accumulate ? 1 : 0;
    reduce_partials_kernel<<<ew_grid(nt_tok * m.rows, 256, *ctx_), 256, 0, st>>>(r);
  }
  return cudaGetLastError() == cudaSuccess;
}

bool Mamba::run_layers(long long n_tok, int B, int L, bool tc, cudaStream_t st, std::string& err) {
  const int dm = static_cast<int>(cfg_.d_model), di = static_cast<int>(cfg_.d_inner);
  const int ds = static_cast<int>(cfg_.d_state), dc = static_cast<int>(cfg_.d_conv);
  const int dr = static_cast<int>(cfg_.dt_rank), wd = dr + 2 * ds;
  float* normed = out_;  // fp32 normed rows share the output buffer until the final norm
  // tensor path: bf16 engines take fp16 operands, fp32 engines fp16 hi / lo splits;
  // the scan's fast exponentials belong to the bf16 mode only
  const int split = tc && prec_ != Precision::kBF16 ? 1 : 0;
  const bool fast = prec_ == Precision::kBF16;
  // bf16 tensor path with sequences that tile the GEMM's token blocks: the
  // causal conv runs in the in-projection's epilogue, and only z goes to xz
  const bool conv_fused = tc && split == 0 && dc == 4 && di % tc::BM == 0 && L <= tc::BN && tc::BN % L == 0;
  const dim3 grid(static_cast<unsigned>((di + 255) / 256), static_cast<unsigned>(B));
  const std::size_t smem = static_cast<std::size_t>(L) * wd * 4;
  // few sequences: chunks of the sequence in parallel (when L splits into them)
  const dim3 cgrid(static_cast<unsigned>((di + kScanCh - 1) / kScanCh), static_cast<unsigned>(B));
  const unsigned cthreads = static_cast<unsigned>(kScanCh * (L / kScanChunk));
  const std::size_t csmem =
      (static_cast<std::size_t>(L) * wd + 2 * static_cast<std::size_t>(L / kScanChunk) * kScanCh * 2) * 4;
  const bool chunked = L % kScanChunk == 0 && L / kScanChunk <= 64 && static_cast<long long>(B) * di < 32768 &&
                       csmem <= 200 * 1024 && wd % 4 == 0;
  // many sequences: the staged kernel (bulk copies need di % 4 == 0); the
  // fp32 y is read only by the CUDA-core out-projection
  const bool staged = di % 4 == 0;
  const dim3 sgrid(static_cast<unsigned>((di + kScanThreads - 1) / kScanThreads), static_cast<unsigned>(B));
  // with the conv fused, the staged scan reads u from its fp16 copy and the
  // fp32 u is not written
  const bool u16 = conv_fused && !chunked && staged && di % 8 == 0;
  for (const Layer& Ly : layers_) {
    launch_rmsnorm(hidden_, Ly.norm, n_tok, dm, tc ? nullptr : normed, tc ? nb_ : nullptr, split, st);
    if (conv_fused) {
      if (!gemm(Ly.in_proj, nb_, dm, n_tok, xz_, 2 * di, false, tc, st, err, &Ly, L, !u16)) return false;
    } else {
      if (!gemm(Ly.in_proj, tc ? static_cast<const void*>(nb_) : normed, dm, n_tok, xz_, 2 * di, false, tc, st, err))
        return false;
      if (static_cast<long long>(B) * (di / 4) >= 32LL * 32 * ctx_->sm_count && dc == 4)
        causal_conv_fixed_kernel<4><<<ew_grid(static_cast<long long>(B) * (di / 4), 256, *ctx_), 256, 0, st>>>(
            xz_, B, L, di, Ly.conv_w, Ly.conv_b, u_, tc ? ub_ : nullptr, split);
      else if (static_cast<long long>(B) * (di / 4) >= 32LL * 32 * ctx_->sm_count)
        causal_conv_kernel<<<ew_grid(static_cast<long long>(B) * (di / 4), 256, *ctx_), 256, 0, st>>>(
            xz_, B, L, di, dc, Ly.conv_w, Ly.conv_b, u_, tc ? ub_ : nullptr, split);
      else
        causal_conv_tok_kernel<<<ew_grid(n_tok * di, 256, *ctx_), 256, 0, st>>>(xz_, B, L, di, dc, Ly.conv_w,
                                                                              Ly.conv_b, u_, tc ? ub_ : nullptr, split);
    }
    if (!gemm(Ly.x_proj, tc ? static_cast<const void*>(ub_) : u_, di, n_tok, dbl_, wd, false, tc, st, err))
      return false;
    auto scan = [&](auto kernel, auto ckernel, auto skernel, auto skernel16, int sds, int sdr) {
      if (chunked)
        ckernel<<<cgrid, cthreads, csmem, st>>>(dbl_, wd, u_, xz_, L, di, Ly.dt_w, Ly.dt_b, Ly.a_neg, Ly.d, nullptr,
                                                y_, tc ? yb_ : nullptr, split);
      else if (staged)
        (u16 ? skernel16 : skernel)<<<sgrid, kScanThreads, static_cast<std::size_t>(scan_smem_floats(sds, sdr)) * 4,
                                      st>>>(dbl_, u16 ? static_cast<const void*>(ub_) : u_, xz_, L, di, Ly.dt_w,
                                            Ly.dt_b, Ly.a_neg, Ly.d, tc ? nullptr : y_, tc ? yb_ : nullptr, split,
                                            ctx_->d_err);
      else
        kernel<<<grid, 256, smem, st>>>(dbl_, wd, u_, xz_, L, di, Ly.dt_w, Ly.dt_b, Ly.a_neg, Ly.d, nullptr, y_,
                                        tc ? yb_ : nullptr, split);
    };
    // (u16 implies the bf16 mode: the fp32 instantiations pass their own
    // staged kernel twice)
    if (ds == 16 && dr == 32)
      fast ? scan(scan_kernel<16, 32, true>, scan_chunked_kernel<16, 32, true>,
                  scan_staged_kernel<16, 32, true, kScanPolyPairs>, scan_staged_kernel<16, 32, true, kScanPolyPairs, true>,
                  16, 32)
           : scan(scan_kernel<16, 32, false>, scan_chunked_kernel<16, 32, false>, scan_staged_kernel<16, 32, false, 0>,
                  scan_staged_kernel<16, 32, false, 0>, 16, 32);
    else if (ds == 4 && dr == 4)
      fast ? scan(scan_kernel<4, 4, true>, scan_chunked_kernel<4, 4, true>, scan_staged_kernel<4, 4, true, 0>,
                  scan_staged_kernel<4, 4, true, 0, true>, 4, 4)
           : scan(scan_kernel<4, 4, false>, scan_chunked_kernel<4, 4, false>, scan_staged_kernel<4, 4, false, 0>,
                  scan_staged_kernel<4, 4, false, 0>, 4, 4);
    else if (ds == 8 && dr == 4)
      fast ? scan(scan_kernel<8, 4, true>, scan_chunked_kernel<8, 4, true>, scan_staged_kernel<8, 4, true, 0>,
                  scan_staged_kernel<8, 4, true, 0, true>, 8, 4)
           : scan(scan_kernel<8, 4, false>, scan_chunked_kernel<8, 4, false>, scan_staged_kernel<8, 4, false, 0>,
                  scan_staged_kernel<8, 4, false, 0>, 8, 4);
    else {
      err = "no scan instantiation for this (d_state, dt_rank)";
      return false;
    }
    if (!gemm(Ly.out_proj, tc ? static_cast<const void*>(yb_) : y_, di, n_tok, hidden_, dm, true, tc, st, err))
      return false;
  }
  launch_rmsnorm(hidden_, norm_f_, n_tok, dm, out_, nullptr, 0, st);
  return cudaGetLastError() == cudaSuccess;
}

int Mamba::forward_device(const std::int32_t* tokens, std::size_t batch, std::size_t len, float* last_hidden,
                          void* stream, std::string& err) noexcept {
  const long long n_tok = static_cast<long long>(batch * len);
  if (batch * len > cap_tokens_ || batch > cap_batch_) {
    err = "batch * sequence exceeds the reserved capacity";
    return 2;
  }
  cudaSetDevice(ctx_->device);
  cudaStream_t st = stream != nullptr ? static_cast<cudaStream_t>(stream) : ctx_->stream;
  const bool tc = n_tok >= kTcMinTokens;
  if (tokens != tokens_) cudaMemcpyAsync(tokens_, tokens, n_tok * 4, cudaMemcpyDeviceToDevice, st);
  const int dm = static_cast<int>(cfg_.d_model);
  float* dst = last_hidden != nullptr ? last_hidden : last_;
  const auto key = std::make_tuple(batch, len, static_cast<const float*>(dst));
  auto it = fwd_graphs_.find(key);
  if (it == fwd_graphs_.end()) {
    cudaStream_t cap = nullptr;
    cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking);
    cudaStreamSynchronize(st);
    cudaGraph_t graph = nullptr;
    cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal);
    embed_kernel<<<ew_grid(n_tok * dm, 256, *ctx_), 256, 0, cap>>>(tokens_, n_tok, emb_, dm, hidden_);
    const bool ok = run_layers(n_tok, static_cast<int>(batch), static_cast<int>(len), tc, cap, err);
    gather_last_kernel<<<ew_grid(static_cast<long long>(batch) * dm, 256, *ctx_), 256, 0, cap>>>(
        out_, static_cast<int>(batch), static_cast<int>(len), dm, dst);
    const cudaError_t end = cudaStreamEndCapture(cap, &graph);
    cudaStreamDestroy(cap);
    if (!ok || end != cudaSuccess || graph == nullptr) {
      if (graph != nullptr) cudaGraphDestroy(graph);
      if (err.empty()) err = "Mamba prefill graph capture failed";
      cudaGetLastError();
      return 2;
    }
    cudaGraphExec_t exec = nullptr;
    const cudaError_t inst = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (inst != cudaSuccess) {
      err = "Mamba prefill graph instantiation failed";
      return 2;
    }
    it = fwd_graphs_.emplace(key, exec).first;
  }
  return cudaGraphLaunch(it->second, st) == cudaSuccess ? 0 : 2;
}

int Mamba::forward(const std::int32_t* tokens, std::size_t batch, std::size_t len, float* hidden, bool last_only,
                   std::string& err) noexcept {
  if ((batch * len > cap_tokens_ || batch > cap_batch_) && reserve(batch, std::max<std::size_t>(len, 512), err) != 0)
    return 2;
  cudaSetDevice(ctx_->device);
  cudaStream_t st = ctx_->stream;
  const long long n_tok = static_cast<long long>(batch * len);
  auto* ptok = reinterpret_cast<std::int32_t*>(pinned_);
  std::memcpy(ptok, tokens, n_tok * 4);
  cudaMemcpyAsync(tokens_, ptok, n_tok * 4, cudaMemcpyHostToDevice, st);
  if (forward_device(tokens_, batch, len, nullptr, st, err) != 0) return 2;
  const std::size_t dm = cfg_.d_model;
  float* ph = pinned_ + n_tok;
  if (!last_only && hidden != nullptr) cudaMemcpyAsync(ph, out_, n_tok * dm * 4, cudaMemcpyDeviceToHost, st);
  if (cudaStreamSynchronize(st) != cudaSuccess) {
    err = std::string("Mamba forward failed: ") + cudaGetErrorString(cudaGetLastError());
    return 2;
  }
  if (take_device_error(*ctx_, st) != 0) {
    err = "a device pipeline wait timed out";
    return 2;
  }
  if (!last_only && hidden != nullptr) std::memcpy(hidden, ph, n_tok * dm * 4);
  return 0;
}

bool Mamba::record_step(cudaStream_t st, std::string& err) {
  const int dm = static_cast<int>(cfg_.d_model), di = static_cast<int>(cfg_.d_inner);
  if (dec_fused_) {
    float* x = dh_;
    DecodeParams p{};
    p.layers = dec_layers_;
    p.n_layers = static_cast<int>(layers_.size());
    p.dm = dm;
    p.di = di;
    p.ds = static_cast<int>(cfg_.d_state);
    p.dc = static_cast<int>(cfg_.d_conv);
    p.dr = static_cast<int>(cfg_.dt_rank);
    p.token = tokens_;
    p.emb = emb_;
    p.norm_f = norm_f_;
    p.state = state_;
    p.x = x;
    p.xz = x + dm;
    p.u = p.xz + 2 * di;
    p.dbl = p.u + di;
    p.y = p.dbl + (p.dr + 2 * p.ds);
    p.out = p.y + 2 * di;
    p.sync = dec_sync_;
    p.err = ctx_->d_err;
    cudaMemcpyAsync(tokens_, pinned_, 4, cudaMemcpyHostToDevice, st);
    cudaMemsetAsync(dec_sync_, 0, 4 * sizeof(unsigned), st);
    cudaLaunchAttribute attr{};
    attr.id = cudaLaunchAttributeCooperative;
    attr.val.cooperative = 1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(ctx_->sm_count));
    cfg.blockDim = dim3(kDecThreads);
    cfg.dynamicSmemBytes = static_cast<std::size_t>(std::max({dm, di, p.dr + 2 * p.ds})) * 4;
    cfg.stream = st;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    const cudaError_t rc = prec_ == Precision::kBF16 ? cudaLaunchKernelEx(&cfg, mamba_decode_kernel<true>, p)
                                                     : cudaLaunchKernelEx(&cfg, mamba_decode_kernel<false>, p);
    if (rc != cudaSuccess) {
      err = std::string("fused decode launch: ") + cudaGetErrorString(rc);
      return false;
    }
    cudaMemcpyAsync(pinned_ + 1, p.out, dm * 4, cudaMemcpyDeviceToHost, st);
    return cudaGetLastError() == cudaSuccess;
  }
  const int ds = static_cast<int>(cfg_.d_state), dc = static_cast<int>(cfg_.d_conv);
  const int dr = static_cast<int>(cfg_.dt_rank), wd = dr + 2 * ds;
  float* x = dh_;                // [dm] hidden
  float* xz = x + dm;            // [2 di]
  float* u = xz + 2 * di;        // [di]
  float* dbl = u + di;           // [wd]
  float* y = dbl + wd;           // [di]
  float* normed = y + di + di;   // [dm]
  cudaMemcpyAsync(tokens_, pinned_, 4, cudaMemcpyHostToDevice, st);
  embed_kernel<<<1, 256, 0, st>>>(tokens_, 1, emb_, dm, x);
  const std::size_t per = static_cast<std::size_t>(di) * (dc + ds);
  for (std::size_t li = 0; li < layers_.size(); ++li) {
    const Layer& Ly = layers_[li];
    float* window = state_ + li * per;
    float* h = window + static_cast<std::size_t>(di) * dc;
    rmsnorm_kernel<<<1, 32, 0, st>>>(x, Ly.norm, 1, dm, normed, nullptr, 0);
    if (!gemm(Ly.in_proj, normed, dm, 1, xz, 2 * di, false, false, st, err)) return false;
    conv_step_kernel<<<(di + 255) / 256, 256, 0, st>>>(xz, di, dc, window, Ly.conv_w, Ly.conv_b, u);
    if (!gemm(Ly.x_proj, u, di, 1, dbl, wd, false, false, st, err)) return false;
    const dim3 grid(static_cast<unsigned>((di + 255) / 256), 1);
    const std::size_t smem = static_cast<std::size_t>(wd) * 4;
    if (ds == 16 && dr == 32)
      scan_kernel<16, 32, false><<<grid, 256, smem, st>>>(dbl, wd, u, xz, 1, di, Ly.dt_w, Ly.dt_b, Ly.a_neg, Ly.d, h, y, nullptr, 0);
    else if (ds == 4 && dr == 4)
      scan_kernel<4, 4, false><<<grid, 256, smem, st>>>(dbl, wd, u, xz, 1, di, Ly.dt_w, Ly.dt_b, Ly.a_neg, Ly.d, h, y, nullptr, 0);
    else if (ds == 8 && dr == 4)
      scan_kernel<8, 4, false><<<grid, 256, smem, st>>>(dbl, wd, u, xz, 1, di, Ly.dt_w, Ly.dt_b, Ly.a_neg, Ly.d, h, y, nullptr, 0);
    else {
      err = "no scan instantiation for this (d_state, dt_rank)";
      return false;
    }
    if (!gemm(Ly.out_proj, y, di, 1, x, dm, true, false, st, err)) return false;
  }
  rmsnorm_kernel<<<1, 32, 0, st>>>(x, norm_f_, 1, dm, normed, nullptr, 0);
  cudaMemcpyAsync(pinned_ + 1, normed, dm * 4, cudaMemcpyDeviceToHost, st);
  return cudaGetLastError() == cudaSuccess;
}

// Streaming decode of one token (mamba.cc:317-382): the conv window and scan
// state stay on the device; the whole step replays as one CUDA graph.
int Mamba::step(std::int32_t token, float* out, std::string& err) noexcept {
  cudaSetDevice(ctx_->device);
  cudaStream_t st = ctx_->stream;
  if (step_graph_ == nullptr) {
    cudaStream_t cap = nullptr;
    cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking);
    cudaStreamSynchronize(st);
    cudaGraph_t graph = nullptr;
    cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal);
    const bool ok = record_step(cap, err);
    const cudaError_t end = cudaStreamEndCapture(cap, &graph);
    cudaStreamDestroy(cap);
    if (!ok || end != cudaSuccess || graph == nullptr) {
      if (graph != nullptr) cudaGraphDestroy(graph);
      if (err.empty()) err = "Mamba step graph capture failed";
      cudaGetLastError();
      return 2;
    }
    const cudaError_t inst = cudaGraphInstantiate(&step_graph_, graph, 0);
    cudaGraphDestroy(graph);
    if (inst != cudaSuccess) {
      step_graph_ = nullptr;
      err = "Mamba step graph instantiation failed";
      return 2;
    }
  }
  *reinterpret_cast<int*>(pinned_) = token;
  if (cudaGraphLaunch(step_graph_, st) != cudaSuccess || cudaStreamSynchronize(st) != cudaSuccess) {
    err = std::string("Mamba step failed: ") + cudaGetErrorString(cudaGetLastError());
    return 2;
  }
  if (const int code = take_device_error(*ctx_, st); code != 0) {
    err = device_error_text(code);
    return 2;
  }
  std::memcpy(out, pinned_ + 1, cfg_.d_model * 4);
  return 0;
}

void Mamba::reset() noexcept {
  cudaSetDevice(ctx_->device);
  cudaMemsetAsync(state_, 0, state_floats() * 4, ctx_->stream);
  cudaStreamSynchronize(ctx_->stream);
}

int Mamba::read_state(float* dst, std::string& err) noexcept {
  cudaSetDevice(ctx_->device);
  if (cudaMemcpyAsync(pinned_, state_, state_floats() * 4, cudaMemcpyDeviceToHost, ctx_->stream) != cudaSuccess ||
      cudaStreamSynchronize(ctx_->stream) != cudaSuccess) {
    err = "decode state copy failed";
    return 2;
  }
  std::memcpy(dst, pinned_, state_floats() * 4);
  return 0;
}

int Mamba::write_state(const float* src, std::string& err) noexcept {
  cudaSetDevice(ctx_->device);
  std::memcpy(pinned_, src, state_floats() * 4);
  if (cudaMemcpyAsync(state_, pinned_, state_floats() * 4, cudaMemcpyHostToDevice, ctx_->stream) != cudaSuccess ||
      cudaStreamSynchronize(ctx_->stream) != cudaSuccess) {
    err = "decode state copy failed";
    return 2;
  }
  return 0;
}

}  // namespace

std::unique_ptr<MambaDevice> make_mamba_device(const TensorTable& tensors, std::shared_ptr<DeviceContext> ctx,
                                               Precision precision, std::string& err) {
  cudaSetDevice(ctx->device);
  auto m = std::make_unique<Mamba>(std::move(ctx), precision);
  if (!m->load(tensors, err)) return nullptr;
  return m;
}

}  // namespace feb
