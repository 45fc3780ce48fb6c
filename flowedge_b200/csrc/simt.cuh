// CUDA-core kernels of the policy-sampling path: weight-streaming split-K
// convolution for small token counts, GroupNorm + Mish + FiLM / residual
// application, the fused output projection + DDIM / DDPM update, and the
// device replica of the reference's seeded Gaussian stream.
#pragma once

#include "common.cuh"

namespace feb {

// ---------------------------------------------------------------------------
// weight-streaming convolution / GEMV for N <= NT tokens per pass
//
//   partial[slice][n][m] = sum_{c in slice} W[m][slice.k_begin + c] * X_slice(n, c)
//
// X_slice(n, c) = src[b][t * stride + t_off][ch_begin + c] (0 outside the
// sample), n = b * L_out + t.  One CTA = 128 output rows (one per lane of its
// 4 warps) x one K-slice of <= 256 channels staged in shared memory.  Weights
// are read once, 32 contiguous bytes per lane per step.

struct SimtSlice {
  int src;
  int t_off;
  int ch_begin;
  int nch;      // multiple of 8, <= 256
  int k_begin;  // offset of the slice in a weight row
};

struct SimtSource {
  const float* ptr;
  int channels;  // row length of the source tensor
  int length;    // input positions per sample
};

struct SimtConvParams {
  const void* W;  // [M][K] fp32 or fp16
  int M, K;
  SimtSource src[3];
  int stride;     // input time = t * stride + t_off
  int L_out;      // output positions per sample
  int n_tokens;   // B * L_out
  const SimtSlice* slices;
  float* partial; // [nslices][n_tokens][M]
};

template <int NT, bool HALF>
static __global__ void __launch_bounds__(128) simt_conv_kernel(const SimtConvParams p) {
  __shared__ __align__(16) float xs[256 * NT];
  const SimtSlice sl = p.slices[blockIdx.x];
  const SimtSource src = p.src[sl.src];
  const int n0 = blockIdx.z * NT;
  // stage X slice: xs[c][n]
  for (int i = threadIdx.x; i < sl.nch * NT; i += blockDim.x) {
    const int c = i / NT;
    const int n = i - c * NT;
    const int tok = n0 + n;
    float v = 0.0f;
    if (tok < p.n_tokens) {
      const int b = tok / p.L_out;
      const int t = tok - b * p.L_out;
      const int ti = t * p.stride + sl.t_off;
      if (ti >= 0 && ti < src.length)
        v = src.ptr[(static_cast<long long>(b) * src.length + ti) * src.channels + sl.ch_begin + c];
    }
    xs[i] = v;
  }
  __syncthreads();
  const int m = blockIdx.y * 128 + threadIdx.x;
  if (m >= p.M) return;
  float acc[NT];
#pragma unroll
  for (int n = 0; n < NT; ++n) acc[n] = 0.0f;
  if constexpr (HALF) {
    const uint4* wrow = reinterpret_cast<const uint4*>(static_cast<const __half*>(p.W) +
                                                       static_cast<long long>(m) * p.K + sl.k_begin);
    uint4 wnext = __ldg(wrow);
    for (int c = 0; c < sl.nch; c += 8) {
      const uint4 wv = wnext;
      if (c + 8 < sl.nch) wnext = __ldg(wrow + (c + 8) / 8);
      const float w[8] = {half_lo(wv.x), half_hi(wv.x), half_lo(wv.y), half_hi(wv.y),
                          half_lo(wv.z), half_hi(wv.z), half_lo(wv.w), half_hi(wv.w)};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4* xr = reinterpret_cast<const float4*>(xs + (c + i) * NT);
#pragma unroll
        for (int n4 = 0; n4 < NT / 4; ++n4) {
          const float4 x = xr[n4];
          acc[n4 * 4 + 0] = fmaf(w[i], x.x, acc[n4 * 4 + 0]);
          acc[n4 * 4 + 1] = fmaf(w[i], x.y, acc[n4 * 4 + 1]);
          acc[n4 * 4 + 2] = fmaf(w[i], x.z, acc[n4 * 4 + 2]);
          acc[n4 * 4 + 3] = fmaf(w[i], x.w, acc[n4 * 4 + 3]);
        }
      }
    }
  } else {
    const float4* wrow =
        reinterpret_cast<const float4*>(static_cast<const float*>(p.W) + static_cast<long long>(m) * p.K + sl.k_begin);
    float4 wa = __ldg(wrow), wb = __ldg(wrow + 1);
    for (int c = 0; c < sl.nch; c += 8) {
      const float w[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
      if (c + 8 < sl.nch) {
        wa = __ldg(wrow + (c + 8) / 4);
        wb = __ldg(wrow + (c + 8) / 4 + 1);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4* xr = reinterpret_cast<const float4*>(xs + (c + i) * NT);
#pragma unroll
        for (int n4 = 0; n4 < NT / 4; ++n4) {
          const float4 x = xr[n4];
          acc[n4 * 4 + 0] = fmaf(w[i], x.x, acc[n4 * 4 + 0]);
          acc[n4 * 4 + 1] = fmaf(w[i], x.y, acc[n4 * 4 + 1]);
          acc[n4 * 4 + 2] = fmaf(w[i], x.z, acc[n4 * 4 + 2]);
          acc[n4 * 4 + 3] = fmaf(w[i], x.w, acc[n4 * 4 + 3]);
        }
      }
    }
  }
  float* out = p.partial + (static_cast<long long>(blockIdx.x) * p.n_tokens + n0) * p.M + m;
#pragma unroll
  for (int n = 0; n < NT; ++n)
    if (n0 + n < p.n_tokens) out[static_cast<long long>(n) * p.M] = acc[n];
}

// y[n][m] = bias[m] + sum_s partial[s][n][m] (fixed order; deterministic)
__device__ __forceinline__ float sum_partials(const float* partial, int nslices, int n_tokens, int M, int n, int m,
                                              const float* bias) {
  float v = bias != nullptr ? bias[m] : 0.0f;
  const long long stride = static_cast<long long>(n_tokens) * M;
  const float* ptr = partial + static_cast<long long>(n) * M + m;
  for (int s = 0; s < nslices; ++s) v += ptr[s * stride];
  return v;
}

// out[n][m] = act(bias + sum partials (+ add_vec[m]) (+ add_tok[n][m])), optional accumulate
struct ReduceParams {
  const float* partial;
  int nslices, n_tokens, M;
  const float* bias;
  const float* add_vec;
  const float* add_tok;
  int act;  // 0 none, 1 silu, 2 softplus
  float* out;
  int out_ld;
  int accumulate;
};

static __global__ void reduce_partials_kernel(const ReduceParams p) {
  const long long total = static_cast<long long>(p.n_tokens) * p.M;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int n = static_cast<int>(i / p.M);
    const int m = static_cast<int>(i - static_cast<long long>(n) * p.M);
    float v = sum_partials(p.partial, p.nslices, p.n_tokens, p.M, n, m, p.bias);
    if (p.add_vec != nullptr) v += p.add_vec[m];
    if (p.add_tok != nullptr) v += p.add_tok[static_cast<long long>(n) * p.M + m];
    if (p.act == 1) v = silu_f(v);
    else if (p.act == 2) v = softplus_f(v);
    float* o = p.out + static_cast<long long>(n) * p.out_ld + m;
    *o = p.accumulate ? *o + v : v;
  }
}

// ---------------------------------------------------------------------------
// GroupNorm (+ Mish) + FiLM or residual, fp32 token-major, inputs as split-K
// partials.  One CTA per (sample, group).  Statistics in double, biased
// variance E[x^2] - E[x]^2 clamped at 0, eps 1e-5 (as the reference CPU op).

struct GnParams {
  const float* partial;
  int nslices, n_tokens, C, L;
  const float* bias;
  const float* gamma;
  const float* beta;
  int groups;
  int mish;
  // FiLM: z = z * (fc[b][off + c] + ft[off + c]) + (fc[b][off + C + c] + ft[off + C + c])
  const float* film_cond;  // [B][F] or null
  const float* film_time;  // [F] row for the current timestep or null
  int film_F, film_off;
  // residual: z += res (tensor [n][C]) or the sum of its partials + bias
  const float* res;
  const float* res_partial;
  int res_nslices;
  const float* res_bias;
  float* out;  // [n][C]
};

static __global__ void __launch_bounds__(256) gn_partials_kernel(const GnParams p) {
  const int b = blockIdx.x;
  const int g = blockIdx.y;
  const int cpg = p.C / p.groups;
  const int count = cpg * p.L;
  double s1 = 0.0, s2 = 0.0;
  for (int i = threadIdx.x; i < count; i += blockDim.x) {
    const int t = i / cpg;
    const int c = g * cpg + (i - t * cpg);
    const float v = sum_partials(p.partial, p.nslices, p.n_tokens, p.C, b * p.L + t, c, p.bias);
    s1 += v;
    s2 += static_cast<double>(v) * v;
  }
  __shared__ double red1[8], red2[8];
  for (int off = 16; off > 0; off >>= 1) {
    s1 += __shfl_xor_sync(0xffffffffu, s1, off);
    s2 += __shfl_xor_sync(0xffffffffu, s2, off);
  }
  if ((threadIdx.x & 31) == 0) {
    red1[threadIdx.x >> 5] = s1;
    red2[threadIdx.x >> 5] = s2;
  }
  __syncthreads();
  double t1 = 0.0, t2 = 0.0;
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) {
    t1 += red1[w];
    t2 += red2[w];
  }
  const double mean = t1 / count;
  const double var = fmax(0.0, t2 / count - mean * mean);
  const float inv = static_cast<float>(1.0 / sqrt(var + 1e-5));
  const float mean_f = static_cast<float>(mean);
  for (int i = threadIdx.x; i < count; i += blockDim.x) {
    const int t = i / cpg;
    const int c = g * cpg + (i - t * cpg);
    const int n = b * p.L + t;
    const float v = sum_partials(p.partial, p.nslices, p.n_tokens, p.C, n, c, p.bias);
    float z = (v - mean_f) * (inv * p.gamma[c]) + p.beta[c];
    if (p.mish) z = mish_f(z);
    if (p.film_cond != nullptr) {
      const float* fc = p.film_cond + static_cast<long long>(b) * p.film_F + p.film_off;
      const float* ft = p.film_time + p.film_off;
      z = (fc[c] + ft[c]) * z + (fc[p.C + c] + ft[p.C + c]);
    }
    if (p.res != nullptr) z += p.res[static_cast<long long>(n) * p.C + c];
    if (p.res_partial != nullptr) z += sum_partials(p.res_partial, p.res_nslices, p.n_tokens, p.C, n, c, p.res_bias);
    p.out[static_cast<long long>(n) * p.C + c] = z;
  }
}

// ---------------------------------------------------------------------------
// GroupNorm application after the tensor-core conv, whose epilogue produced
// y (fp32, bias included) and per-(sample, group, part) partial sums.
// z = mish(GN(y)) then FiLM, or + residual (fp32 residual stream, or bf16 when
// no fp32 copy exists).  Writes the bf16 GEMM operand and, optionally, the
// fp32 residual-stream copy.  8 channels per thread.

struct GnTcParams {
  const float* y;
  long long n_tokens;
  int C, L, groups, parts;
  const double* stats;
  const float* gamma;
  const float* beta;
  const float* film_cond;
  const float* film_time;
  int film_F, film_off;
  const float* res_f32;           // [n][C] or null
  const __half* res_half;  // [n][C] or null
  __half* out;             // [n][C]
  float* out_f32;                 // [n][C] or null
};

static __global__ void __launch_bounds__(256) gn_tc_kernel(const GnTcParams p) {
  const int vec_per_tok = p.C / 8;
  const long long total = p.n_tokens * vec_per_tok;
  const int cpg = p.C / p.groups;
  const double count = static_cast<double>(cpg) * p.L;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long n = i / vec_per_tok;
    const int c0 = static_cast<int>(i - n * vec_per_tok) * 8;
    const int b = static_cast<int>(n / p.L);
    const int g = c0 / cpg;
    const double* st = p.stats + (static_cast<long long>(b) * p.groups + g) * p.parts * 2;
    double s1 = 0.0, s2 = 0.0;
    for (int part = 0; part < p.parts; ++part) {
      s1 += st[2 * part];
      s2 += st[2 * part + 1];
    }
    const double mean = s1 / count;
    const double var = fmax(0.0, s2 / count - mean * mean);
    const float inv = static_cast<float>(1.0 / sqrt(var + 1e-5));
    const float mean_f = static_cast<float>(mean);
    const float4 ya = *reinterpret_cast<const float4*>(p.y + n * p.C + c0);
    const float4 yb = *reinterpret_cast<const float4*>(p.y + n * p.C + c0 + 4);
    float v[8] = {ya.x, ya.y, ya.z, ya.w, yb.x, yb.y, yb.z, yb.w};
    float r[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (p.res_f32 != nullptr) {
      const float4 ra = *reinterpret_cast<const float4*>(p.res_f32 + n * p.C + c0);
      const float4 rb = *reinterpret_cast<const float4*>(p.res_f32 + n * p.C + c0 + 4);
      r[0] = ra.x; r[1] = ra.y; r[2] = ra.z; r[3] = ra.w; r[4] = rb.x; r[5] = rb.y; r[6] = rb.z; r[7] = rb.w;
    } else if (p.res_half != nullptr) {
      const uint4 rv = *reinterpret_cast<const uint4*>(p.res_half + n * p.C + c0);
      r[0] = half_lo(rv.x); r[1] = half_hi(rv.x); r[2] = half_lo(rv.y); r[3] = half_hi(rv.y);
      r[4] = half_lo(rv.z); r[5] = half_hi(rv.z); r[6] = half_lo(rv.w); r[7] = half_hi(rv.w);
    }
    float gam[8], bet[8], fsc[8], fsh[8];
    {
      const float4 g0 = *reinterpret_cast<const float4*>(p.gamma + c0);
      const float4 g1 = *reinterpret_cast<const float4*>(p.gamma + c0 + 4);
      const float4 b0 = *reinterpret_cast<const float4*>(p.beta + c0);
      const float4 b1 = *reinterpret_cast<const float4*>(p.beta + c0 + 4);
      gam[0] = g0.x; gam[1] = g0.y; gam[2] = g0.z; gam[3] = g0.w; gam[4] = g1.x; gam[5] = g1.y; gam[6] = g1.z; gam[7] = g1.w;
      bet[0] = b0.x; bet[1] = b0.y; bet[2] = b0.z; bet[3] = b0.w; bet[4] = b1.x; bet[5] = b1.y; bet[6] = b1.z; bet[7] = b1.w;
    }
    if (p.film_cond != nullptr) {
      const float* fc = p.film_cond + static_cast<long long>(b) * p.film_F + p.film_off + c0;
      const float* ft = p.film_time + p.film_off + c0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        fsc[j] = fc[j] + ft[j];
        fsh[j] = fc[p.C + j] + ft[p.C + j];
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float z = mish_fast((v[j] - mean_f) * (inv * gam[j]) + bet[j]);
      if (p.film_cond != nullptr) z = fsc[j] * z + fsh[j];
      v[j] = z + r[j];
    }
    uint4 o;
    o.x = pack_half(v[0], v[1]);
    o.y = pack_half(v[2], v[3]);
    o.z = pack_half(v[4], v[5]);
    o.w = pack_half(v[6], v[7]);
    *reinterpret_cast<uint4*>(p.out + n * p.C + c0) = o;
    if (p.out_f32 != nullptr) {
      *reinterpret_cast<float4*>(p.out_f32 + n * p.C + c0) = make_float4(v[0], v[1], v[2], v[3]);
      *reinterpret_cast<float4*>(p.out_f32 + n * p.C + c0 + 4) = make_float4(v[4], v[5], v[6], v[7]);
    }
  }
}

// ---------------------------------------------------------------------------
// seeded Gaussian stream (splitmix64 -> 24-bit uniform -> Box-Muller, cosine
// first), random access by value index: the k-th 64-bit draw of a stream
// seeded with s mixes s + (k + 1) * 0x9e3779b97f4a7c15, so value j uses draws
// 2*(j/2) + 1 and 2*(j/2) + 2.  Same sequence as the host generator of the
// reference DiffusionHead (one value per element per DDPM step).

__device__ __forceinline__ uint64_t splitmix_mix(uint64_t v) {
  v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ULL;
  v = (v ^ (v >> 27)) * 0x94d049bb133111ebULL;
  return v ^ (v >> 31);
}

__device__ __forceinline__ float stream_uniform(uint64_t x) {
  return static_cast<float>((x >> 40) + 1u) / 16777217.0f;
}

__device__ __forceinline__ float gaussian_at(uint64_t seed, uint64_t j) {
  const uint64_t pair = j >> 1;
  const uint64_t golden = 0x9e3779b97f4a7c15ULL;
  const float first = fmaxf(stream_uniform(splitmix_mix(seed + (2 * pair + 2) * golden)), 1.17549435e-38f);
  const float second = stream_uniform(splitmix_mix(seed + (2 * pair + 3) * golden));
  const float radius = sqrtf(-2.0f * logf(first));
  const float angle = 6.28318548f * second;
  return (j & 1) ? radius * sinf(angle) : radius * cosf(angle);
}

// ---------------------------------------------------------------------------
// scheduler update, shared by both paths

struct StepScalars {
  float sqrt_alpha, sqrt_beta;  // of alpha_t
  float sqrt_alpha_prev, sqrt_one_minus_prev;
  float orig_coef, sample_coef, noise_std;
  int ddpm;         // 0 = DDIM (eta 0), 1 = DDPM
  int add_noise;    // DDPM and previous >= 0
  int noise_draw;   // index of this step's draw in the sample's stream
  int clip;
  float clip_range;
};

__device__ __forceinline__ float scheduler_update(const StepScalars& s, float x, float eps, uint64_t seed,
                                                  uint64_t value_index, int values_per_draw) {
  float pred = (x - s.sqrt_beta * eps) / s.sqrt_alpha;
  if (s.clip) pred = fminf(fmaxf(pred, -s.clip_range), s.clip_range);
  if (!s.ddpm) return s.sqrt_alpha_prev * pred + s.sqrt_one_minus_prev * eps;
  float next = s.orig_coef * pred + s.sample_coef * x;
  if (s.add_noise)
    next += s.noise_std *
            gaussian_at(seed, static_cast<uint64_t>(s.noise_draw) * values_per_draw + value_index);
  return next;
}

// ---------------------------------------------------------------------------
// output 1x1 conv (dims[0] -> A) fused with the scheduler update.  One warp
// per token; z is the final GN+Mish activation (fp32 or bf16), x_master the
// fp32 sample [B][H][A].  Writes the next step's network input (x_in, padded
// to Cin channels) and optionally the raw epsilon.

template <typename ZT>
struct OutParams {
  const ZT* z;          // [n][C]
  int C, A, H, n_tokens;
  const float* W;       // [A][C]
  const float* bias;    // [A]
  float* x_master;      // [n][A]
  float* eps_out;       // [n][A] or null
  int update;           // 0: only write eps
  StepScalars step;
  const uint64_t* seeds;  // per-sample seeds (DDPM)
  void* x_in;           // [n][Cin] next input (fp32 or bf16 per x_in_half)
  int Cin;
  int x_in_half;
};

template <typename ZT>
__device__ __forceinline__ float load_act(const ZT* p, long long i);
template <>
__device__ __forceinline__ float load_act<float>(const float* p, long long i) { return p[i]; }
template <>
__device__ __forceinline__ float load_act<__half>(const __half* p, long long i) {
  return __half2float(p[i]);
}

template <typename ZT, int MAXA>
static __global__ void __launch_bounds__(256) out_update_kernel(const OutParams<ZT> p) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= p.n_tokens) return;
  const int n = warp;
  float acc[MAXA];
#pragma unroll
  for (int a = 0; a < MAXA; ++a) acc[a] = 0.0f;
  const ZT* zr = p.z + static_cast<long long>(n) * p.C;
  for (int c = lane; c < p.C; c += 32) {
    const float zv = load_act<ZT>(zr, c);
#pragma unroll
    for (int a = 0; a < MAXA; ++a)
      if (a < p.A) acc[a] = fmaf(p.W[a * p.C + c], zv, acc[a]);
  }
#pragma unroll
  for (int a = 0; a < MAXA; ++a)
    for (int off = 16; off > 0; off >>= 1) acc[a] += __shfl_xor_sync(0xffffffffu, acc[a], off);
  if (lane != 0) return;
  const int b = n / p.H;
  const int t = n - b * p.H;
  for (int a = 0; a < p.A; ++a) {
    const float eps = acc[a] + p.bias[a];
    const long long xi = static_cast<long long>(n) * p.A + a;
    if (p.eps_out != nullptr) p.eps_out[xi] = eps;
    if (!p.update) continue;
    const float x = scheduler_update(p.step, p.x_master[xi], eps, p.seeds != nullptr ? p.seeds[b] : 0,
                                     static_cast<uint64_t>(t) * p.A + a, p.H * p.A);
    p.x_master[xi] = x;
    const long long ii = static_cast<long long>(n) * p.Cin + a;
    if (p.x_in_half) static_cast<__half*>(p.x_in)[ii] = to_half_sat(x);
    else static_cast<float*>(p.x_in)[ii] = x;
  }
}

// Scheduler update after the output 1x1 conv ran on the tensor cores.  The
// conv's weights were split into fp16 high and low rows, so the conv wrote
// 2A values per token: eps[a] = t[n][a] + t[n][A + a].  Elementwise over the
// tokens' A values; writes x_master, the next input x_in (fp16, padded to Cin
// channels) and optionally the raw epsilon.
struct EpsUpdateParams {
  const float* t;       // [n][2A]
  int A, H, n_tokens;
  float* x_master;      // [n][A]
  float* eps_out;       // [n][A] or null
  int update;           // 0: only write eps
  StepScalars step;
  const uint64_t* seeds;
  __half* x_in;         // [n][Cin]
  int Cin;
};

static __global__ void __launch_bounds__(256) eps_update_kernel(const EpsUpdateParams p) {
  const long long total = static_cast<long long>(p.n_tokens) * p.A;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int n = static_cast<int>(i / p.A);
    const int a = static_cast<int>(i - static_cast<long long>(n) * p.A);
    const float* tr = p.t + static_cast<long long>(n) * 2 * p.A;
    const float eps = tr[a] + tr[p.A + a];
    if (p.eps_out != nullptr) p.eps_out[i] = eps;
    if (!p.update) continue;
    const int b = n / p.H;
    const int t = n - b * p.H;
    const float x = scheduler_update(p.step, p.x_master[i], eps, p.seeds != nullptr ? p.seeds[b] : 0,
                                     static_cast<uint64_t>(t) * p.A + a, p.H * p.A);
    p.x_master[i] = x;
    p.x_in[static_cast<long long>(n) * p.Cin + a] = to_half_sat(x);
  }
}

// noise [n][A] -> x_master [n][A] and x_in [n][Cin] (zero padded)
static __global__ void prep_sample_kernel(const float* noise, int n_tokens, int A, float* x_master, void* x_in, int Cin,
                                   int x_in_half) {
  const long long total = static_cast<long long>(n_tokens) * Cin;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long n = i / Cin;
    const int c = static_cast<int>(i - n * Cin);
    float v = 0.0f;
    if (c < A) {
      v = noise[n * A + c];
      if (x_master != nullptr) x_master[n * A + c] = v;
    }
    if (x_in_half) static_cast<__half*>(x_in)[i] = to_half_sat(v);
    else static_cast<float*>(x_in)[i] = v;
  }
}

// mish(cond) [B][Cpad] (zero padded) in fp32 or bf16
static __global__ void prep_cond_kernel(const float* cond, int B, int Cd, void* out, int Cpad, int out_half) {
  const long long total = static_cast<long long>(B) * Cpad;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long b = i / Cpad;
    const int c = static_cast<int>(i - b * Cpad);
    const float v = c < Cd ? mish_f(cond[b * Cd + c]) : 0.0f;
    if (out_half) static_cast<__half*>(out)[i] = to_half_sat(v);
    else static_cast<float*>(out)[i] = v;
  }
}

// x_master [n][A] -> action = (x + 1) / 2 * (max - min) + min
static __global__ void unnormalize_kernel(const float* x, int n_tokens, int A, const float* amin, const float* amax,
                                   float* out) {
  const long long total = static_cast<long long>(n_tokens) * A;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int a = static_cast<int>(i % A);
    out[i] = ((x[i] + 1.0f) * 0.5f * (amax[a] - amin[a])) + amin[a];
  }
}

// ---------------------------------------------------------------------------
// diffusion step embedding -> time MLP -> mish, one CTA per timestep value;
// then film_time[r][f] = sum_j Wt[f][j] * tm[r][j].

static __global__ void temb_kernel(const float* timesteps, int rows, int td, const float* w1, const float* b1,
                            const float* w2, const float* b2, float* tm_out) {
  extern __shared__ float sh[];
  const int r = blockIdx.x;
  if (r >= rows) return;
  float* raw = sh;
  float* hid = sh + td;
  const int half = td / 2;
  const float ts = timesteps[r];
  const float factor = logf(10000.0f) / static_cast<float>(half - 1);
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float phase = ts * expf(-factor * static_cast<float>(i));
    raw[i] = sinf(phase);
    raw[half + i] = cosf(phase);
  }
  __syncthreads();
  for (int o = threadIdx.x; o < 4 * td; o += blockDim.x) {
    float acc = 0.0f;
    for (int j = 0; j < td; ++j) acc = fmaf(w1[o * td + j], raw[j], acc);
    hid[o] = mish_f(acc + b1[o]);
  }
  __syncthreads();
  for (int o = threadIdx.x; o < td; o += blockDim.x) {
    float acc = 0.0f;
    for (int j = 0; j < 4 * td; ++j) acc = fmaf(w2[o * 4 * td + j], hid[j], acc);
    tm_out[r * td + o] = mish_f(acc + b2[o]);
  }
}

static __global__ void film_time_kernel(const float* tm, int rows, int td, const float* wt, int F, float* out) {
  const long long total = static_cast<long long>(rows) * F;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / F);
    const int f = static_cast<int>(i - static_cast<long long>(r) * F);
    float acc = 0.0f;
    for (int j = 0; j < td; ++j) acc = fmaf(wt[static_cast<long long>(f) * td + j], tm[r * td + j], acc);
    out[i] = acc;
  }
}

}  // namespace feb
