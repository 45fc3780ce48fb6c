// SmolVLA-shaped flow action expert on sm_100a (12 heads of 60 over a 960-wide
// prefix, and the reference's own shapes).
//
// The reference runs the expert on the host with bf16 rounding at every
// boundary (src/core/models/smolvla/smolvla_action_expert.cc:209-477).  Here a
// batch of independent action chunks runs as one token matrix of
// rows = batch x chunk:
//
//   * Every projection is a tcgen05 GEMM (tc_gemm.cuh).  The layer
//     projections take bf16 operands: the reference rounds their inputs and
//     weights to bf16, so the tensor cores see the reference's operand values
//     and the products are exact; only the fp32 summation order differs.  The
//     epilogue rounds to bf16 where the reference does (q, k, v, gate, up,
//     o and down) and applies the SwiGLU gate ([Wgate; Wup] rows interleaved).
//     The suffix embedding, the action projection and the cross-attention
//     K / V projections consume fp32 activations (the reference does not round
//     them): they run on fp16 hi / lo splits of the activations against
//     [W | W], which keeps ~22 bits of each activation.
//   * Fused q / k / v rows ([Wq; Wk; Wv], one GEMM) for self-attention layers.
//   * Attention (grouped-query, RoPE, the reference's softmax order: max,
//     exp, 1 / sum, bf16 probabilities) runs on mma.sync with bf16 operands,
//     one CTA per (sample, K / V head) with K and V^T staged in shared memory.
//     RoPE is applied while staging q and k.
//   * The cross-attention K / V of a prefix do not change across Euler steps:
//     they are projected once per call (the reference recomputes them every
//     step; the values are the same).
//   * One Euler step (time embedding ... action projection, update) is
//     captured as a CUDA graph and replayed `steps` times.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "runtime.cuh"

namespace feb {
namespace {

using bf16 = __nv_bfloat16;

constexpr int kHwPad = 64;          // head width padded to the mma k-steps (head width <= 64)
constexpr int kKRow = kHwPad + 8;   // staged q / k row (bf16 elements)
constexpr int kAttnThreads = 128;
constexpr int kMaxChunk = 512;      // engine_runtime.cc:677, :702
constexpr int kMaxPrefix = 512;     // engine_runtime.cc:702
constexpr std::size_t kMaxSteps = 100;  // smolvla_action_expert.h:91

inline int pad(int v, int m) { return (v + m - 1) / m * m; }

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
__device__ __forceinline__ float ldbf(const bf16* p) { return __bfloat162float(*p); }

// ---------------------------------------------------------------------------
// elementwise kernels

// fp32 rows [rows][cols] -> fp16 hi / lo rows [rows][2 * ld_dst]: hi = fp16(v)
// at c, lo = fp16(v - hi) at ld_dst + c; columns cols .. ld_dst - 1 are zero.
// Source row r is at (r / group) * group_stride + (r % group) * ld_src (one
// layer's slots of every sample of a [samples][layers][slots][cols] cache).
__global__ void split_rows_kernel(const float* src, long long rows, int cols, int ld_src, long long group,
                                  long long group_stride, __half* dst, int ld_dst) {
  const long long total = rows * ld_dst;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / ld_dst;
    const int c = static_cast<int>(i - r * ld_dst);
    const long long gi = r / group;
    const float v = c < cols ? src[gi * group_stride + (r - gi * group) * ld_src + c] : 0.0f;
    const __half hi = to_half_sat(v);
    dst[r * 2 * ld_dst + c] = hi;
    dst[r * 2 * ld_dst + ld_dst + c] = __float2half_rn(v - __half2float(hi));
  }
}

// Time half of the suffix embedding (smolvla_action_expert.cc:225-240):
// temb[m] = bias[m] + sum_j Wt[m][j] time_j with time = [sin(w_i t) | cos(w_i t)],
// w_i = 2 pi / period_i precomputed on the host in the reference's float
// expression, t = 1 + step dt, dt = -1 / steps (:464-466), or *t_direct.
// One warp per row m.
__global__ void time_embed_kernel(const int* step_idx, int steps, const float* t_direct, const float* omega, int half,
                                  const float* wt, const float* bias, int W, float* temb) {
  extern __shared__ float tv[];
  float t;
  if (t_direct != nullptr) {
    t = *t_direct;
  } else {
    const float dt = -1.0f / static_cast<float>(steps);
    t = __fadd_rn(1.0f, __fmul_rn(static_cast<float>(*step_idx), dt));
  }
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float a = __fmul_rn(omega[i], t);
    tv[i] = sinf(a);
    tv[half + i] = cosf(a);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int m = blockIdx.x * (blockDim.x >> 5) + warp; m < W; m += gridDim.x * (blockDim.x >> 5)) {
    const float* w = wt + static_cast<long long>(m) * W;
    float acc = 0.0f;
    for (int j = lane; j < W; j += 32) acc = fmaf(w[j], tv[j], acc);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) temb[m] = acc + bias[m];
  }
}

// One warp per row (rmsnorm_bf16, kernels.h:246-265, with the residual of
// smolvla_action_expert.cc:355-358 / :376-379 in front):
//   proj != null: h = bf16(h + proj), stored back (proj: a projection the GEMM
//   epilogue already rounded to bf16)
//   n = bf16(bf16(h * scale) * w), scale = 1 / sqrt(sum(h^2) / W + 1e-5)
// out_mode 0: n as bf16 [rows][ld_out]; 1: fp16 hi / lo [rows][2 ld_out]; 2: fp32 [rows][ld_out].
// Lane l holds elements 4 (l + 32 k) .. + 3 (16-byte loads, W a multiple of 4,
// W <= 128 * kRmsVec); every load of a row is issued before the first use.
constexpr int kRmsVec = 8;
__device__ __forceinline__ float4 bf16x4_to_f4(uint2 u) {
  return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u), __uint_as_float(u.y << 16),
                     __uint_as_float(u.y & 0xFFFF0000u));
}
__global__ void rms_kernel(float* __restrict__ h, int ld_h, const bf16* __restrict__ proj, int ld_p,
                           const float* __restrict__ w, int W, long long rows, int out_mode, void* out, int ld_out) {
  griddep_wait();
  griddep_launch();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long r = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + warp;
  if (r >= rows) return;
  float* hr = h + r * ld_h;
  float4 v[kRmsVec];
#pragma unroll
  for (int k = 0; k < kRmsVec; ++k) {
    const int c = 4 * (lane + 32 * k);
    v[k] = c < W ? *reinterpret_cast<const float4*>(hr + c) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  }
  if (proj != nullptr) {
    uint2 pr[kRmsVec];
#pragma unroll
    for (int k = 0; k < kRmsVec; ++k) {
      const int c = 4 * (lane + 32 * k);
      pr[k] = c < W ? __ldg(reinterpret_cast<const uint2*>(proj + r * ld_p + c)) : make_uint2(0u, 0u);
    }
#pragma unroll
    for (int k = 0; k < kRmsVec; ++k) {
      const int c = 4 * (lane + 32 * k);
      if (c < W) {
        const float4 pf = bf16x4_to_f4(pr[k]);
        v[k] = make_float4(bf16r(__fadd_rn(v[k].x, pf.x)), bf16r(__fadd_rn(v[k].y, pf.y)),
                           bf16r(__fadd_rn(v[k].z, pf.z)), bf16r(__fadd_rn(v[k].w, pf.w)));
        *reinterpret_cast<float4*>(hr + c) = v[k];
      }
    }
  }
  float ss = 0.0f;
#pragma unroll
  for (int k = 0; k < kRmsVec; ++k) {
    ss = fmaf(v[k].x, v[k].x, ss);
    ss = fmaf(v[k].y, v[k].y, ss);
    ss = fmaf(v[k].z, v[k].z, ss);
    ss = fmaf(v[k].w, v[k].w, ss);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float scale = 1.0f / sqrtf(__fadd_rn(ss / static_cast<float>(W), 1e-5f));
  float4 wv[kRmsVec];
#pragma unroll
  for (int k = 0; k < kRmsVec; ++k) {
    const int c = 4 * (lane + 32 * k);
    wv[k] = c < W ? __ldg(reinterpret_cast<const float4*>(w + c)) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  }
  auto norm = [&](float x, float wx) { return bf16r(__fmul_rn(bf16r(__fmul_rn(x, scale)), wx)); };
#pragma unroll
  for (int k = 0; k < kRmsVec; ++k) {
    const int c = 4 * (lane + 32 * k);
    if (c >= W) continue;
    const float4 n = make_float4(norm(v[k].x, wv[k].x), norm(v[k].y, wv[k].y), norm(v[k].z, wv[k].z),
                                 norm(v[k].w, wv[k].w));
    if (out_mode == 0) {
      *reinterpret_cast<uint2*>(static_cast<bf16*>(out) + r * ld_out + c) =
          make_uint2(pack_bf16(n.x, n.y), pack_bf16(n.z, n.w));
    } else if (out_mode == 1) {
      __half* o = static_cast<__half*>(out) + r * 2 * ld_out + c;
      const __half h0 = to_half_sat(n.x), h1 = to_half_sat(n.y), h2 = to_half_sat(n.z), h3 = to_half_sat(n.w);
      const __half2 hi01 = __halves2half2(h0, h1), hi23 = __halves2half2(h2, h3);
      const __half2 lo01 = __floats2half2_rn(n.x - __half2float(h0), n.y - __half2float(h1));
      const __half2 lo23 = __floats2half2_rn(n.z - __half2float(h2), n.w - __half2float(h3));
      *reinterpret_cast<uint2*>(o) = make_uint2(*reinterpret_cast<const uint32_t*>(&hi01),
                                                *reinterpret_cast<const uint32_t*>(&hi23));
      *reinterpret_cast<uint2*>(o + ld_out) = make_uint2(*reinterpret_cast<const uint32_t*>(&lo01),
                                                         *reinterpret_cast<const uint32_t*>(&lo23));
    } else {
      *reinterpret_cast<float4*>(static_cast<float*>(out) + r * ld_out + c) = n;
    }
  }
}

// x = x + dt v (smolvla_action_expert.cc:472-473), the next step's fp16 hi / lo
// input and the step counter.
__global__ void euler_kernel(const float* v, int ld_v, float* x, int A, long long rows, int steps, __half* x2,
                             int ld2, const int* step_idx, int* step_out) {
  griddep_wait();
  griddep_launch();
  const float dt = -1.0f / static_cast<float>(steps);
  const long long total = rows * A;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / A;
    const int a = static_cast<int>(i - r * A);
    const float nx = __fadd_rn(x[i], __fmul_rn(dt, v[r * ld_v + a]));
    x[i] = nx;
    const __half hi = to_half_sat(nx);
    x2[r * 2 * ld2 + a] = hi;
    x2[r * 2 * ld2 + ld2 + a] = __float2half_rn(nx - __half2float(hi));
  }
  if (step_out != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *step_out = *step_idx + 1;
}

// fp32 [rows][ld_src] -> dense [rows][cols]
__global__ void gather_rows_kernel(const float* src, int ld_src, long long rows, int cols, float* dst) {
  const long long total = rows * cols;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / cols;
    dst[i] = src[r * ld_src + (i - r * cols)];
  }
}

// dense fp32 [rows][cols] -> [rows][ld_dst] (padding columns untouched)
__global__ void scatter_rows_kernel(const float* src, long long rows, int cols, float* dst, int ld_dst) {
  const long long total = rows * cols;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / cols;
    dst[r * ld_dst + (i - r * cols)] = src[i];
  }
}

// valid[b] = number of set mask bytes of sample b (RoPE base of self-attention)
__global__ void count_valid_kernel(const uint8_t* mask, int P, int* valid) {
  __shared__ int part[32];
  int n = 0;
  for (int j = threadIdx.x; j < P; j += blockDim.x) n += mask[static_cast<long long>(blockIdx.x) * P + j] != 0;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) n += __shfl_xor_sync(0xffffffffu, n, off);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = n;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += part[w];
    valid[blockIdx.x] = t;
  }
}

// ---------------------------------------------------------------------------
// grouped-query attention (kernels.h:267-336) on mma.sync m16n8k16 (bf16)

struct AttnParams {
  const bf16* qkv;  // [rows][qkv_ld]: q of head h at h * hw; self layers: k at k_off, v at v_off
  int qkv_ld, k_off, v_off;
  const bf16* kvp;  // cross: [samples][P][kvp_ld], k at kvh * hw, v at kv_w + kvh * hw
  int kvp_ld, kv_w;
  long long kvp_b;  // sample stride of kvp in rows (0: shared prefix)
  const float* pk;  // self layers in the reference layout: prefix keys / values [samples][P][p_ld] of this layer
  const float* pv;
  int p_ld;
  long long p_b;    // sample stride in rows (elements / p_ld) of pk / pv, 0 shared
  long long layer_off;  // element offset of this layer inside one sample's cache
  const uint8_t* mask;
  long long mask_b;
  const int* valid;
  int valid_b;
  const float2* rope;  // [position][hw / 2]: (cos, sin) of position / exp(ln(1e4) * 2c / hw)
  int chunk, chunk_pad, P, heads, kv_heads, hw;
  int cross;
  int S, S_pad, npre;  // keys (prefix part first), padded to 16; npre keys precede the action tokens
  float sqrt_hw;
  bf16* out;
  int out_ld;
};

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// (first, second) rotated by the angle whose (cos, sin) is cs (kernels.h:353-358)
__device__ __forceinline__ void rope_pair(float first, float second, float2 cs, float& o0, float& o1) {
  o0 = __fsub_rn(__fmul_rn(first, cs.x), __fmul_rn(second, cs.y));
  o1 = __fadd_rn(__fmul_rn(second, cs.x), __fmul_rn(first, cs.y));
}

// table[pos][c] = (cos, sin)(pos / denom[c]), the angles of apply_rope
// (kernels.h:345-352) for positions 0 .. npos - 1
__global__ void rope_table_kernel(const float* denom, int half, int npos, float2* table) {
  const int total = npos * half;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int pos = i / half, c = i - pos * half;
    float sn, cs;
    sincosf(static_cast<float>(pos) / denom[c], &sn, &cs);
    table[i] = make_float2(cs, sn);
  }
}

__device__ __forceinline__ void ldsm_x4(const void* p, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(const void* p, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ uint2 ld_bf16x4(const bf16* p) { return __ldg(reinterpret_cast<const uint2*>(p)); }

// 4 fp32 cache values -> 4 bf16 (the reference multiplies the fp32 cache; the
// VLM cache is bf16 at the source, so this is exact for bf16-valued caches)
__device__ __forceinline__ uint2 bf16x4_of(const float* p) {
  const float4 v = __ldg(reinterpret_cast<const float4*>(p));
  return make_uint2(pack_bf16(v.x, v.y), pack_bf16(v.z, v.w));
}

constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kStageBatch = 4;  // independent 8-byte loads in flight per thread while staging

// One CTA per (sample, K / V head, task slice): K and V of the head staged
// once per CTA (row-major, 8-byte copies; RoPE of the action-token keys from a
// per-call cos / sin table).  A task is (G query heads of the group, 16 query
// rows): the G heads share every K / V fragment a warp loads (grouped-query
// attention), and the CTA's four warps split the task's keys (blocks of 16,
// round robin):
//   phase 1: scores with an online row max / sum per warp, merged across the
//            warps in warp order (the rescaled sum equals the reference's sum
//            of exp(s - max) up to rounding),
//   phase 2: p = bf16(exp(s - max) / sum) packed as A fragments, O += P V over
//            the warp's keys; the warps' O partials are summed in warp order.
// Fragments come from shared memory by ldmatrix (V transposed on the fly).
// Exponentials are 2^x (ex2.approx) of scores scaled by log2(e) / sqrt(hw).
// gridDim.z slices the tasks so that small batches still fill the GPU.
template <int G>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const AttnParams p) {
  griddep_wait();
  griddep_launch();
  extern __shared__ __align__(16) uint8_t smem[];
  bf16* Ks = reinterpret_cast<bf16*>(smem);                  // [S_pad][kKRow]
  bf16* Vs = Ks + static_cast<long long>(p.S_pad) * kKRow;  // [S_pad][kKRow]
  float* kbias = reinterpret_cast<float*>(Vs + static_cast<long long>(p.S_pad) * kKRow);  // [S_pad]
  float* red = kbias + p.S_pad;                             // [G][warps][16][max, sum]
  float* opart = red + G * kAttnWarps * 16 * 2;             // [warps][16][kHwPad]
  bf16* Qs = reinterpret_cast<bf16*>(opart + kAttnWarps * 16 * kHwPad);  // [G][16][kKRow]
  const int b = blockIdx.x, kvh = blockIdx.y;
  const int tid = threadIdx.x;
  const int hw = p.hw, half = hw / 2, nq = hw / 4;
  const int base = p.cross ? 0 : p.valid[static_cast<long long>(b) * p.valid_b];  // RoPE position of token 0
  const long long tok0 = static_cast<long long>(b) * p.chunk;
  const uint32_t z2 = 0u;

  // zero padding (keys >= S, dims >= hw) and the key bias
  for (int i = tid; i < p.S_pad * (kHwPad / 4); i += kAttnThreads) {
    const int j = i / (kHwPad / 4), q = i - j * (kHwPad / 4);
    if (j >= p.S || q >= nq) {
      *reinterpret_cast<uint2*>(Ks + j * kKRow + 4 * q) = make_uint2(z2, z2);
      *reinterpret_cast<uint2*>(Vs + j * kKRow + 4 * q) = make_uint2(z2, z2);
    }
  }
  for (int i = tid; i < p.S_pad; i += kAttnThreads) {
    float bias = -INFINITY;
    if (i < p.npre) bias = p.mask[static_cast<long long>(b) * p.mask_b + i] != 0 ? 0.0f : -INFINITY;
    else if (i < p.S) bias = 0.0f;
    kbias[i] = bias;
  }
  // K / V rows, 4 dims per item, kStageBatch loads in flight per thread
  const int items = p.S * nq;
  for (int i0 = tid; i0 < items; i0 += kAttnThreads * kStageBatch) {
    uint2 kv[kStageBatch], vv[kStageBatch];
#pragma unroll
    for (int u = 0; u < kStageBatch; ++u) {
      const int i = i0 + u * kAttnThreads;
      kv[u] = make_uint2(z2, z2);
      vv[u] = make_uint2(z2, z2);
      if (i < items) {
        const int j = i / nq, q = i - j * nq;
        const int col = kvh * hw + 4 * q;
        if (p.cross) {
          const bf16* row = p.kvp + (static_cast<long long>(b) * p.kvp_b + j) * p.kvp_ld;
          kv[u] = ld_bf16x4(row + col);
          vv[u] = ld_bf16x4(row + p.kv_w + col);
        } else if (j < p.npre) {
          const long long o = static_cast<long long>(b) * p.p_b * p.p_ld + p.layer_off +
                              static_cast<long long>(j) * p.p_ld + col;
          kv[u] = bf16x4_of(p.pk + o);
          vv[u] = bf16x4_of(p.pv + o);
        } else {
          const bf16* row = p.qkv + (tok0 + j - p.npre) * p.qkv_ld;
          kv[u] = ld_bf16x4(row + p.k_off + col);
          vv[u] = ld_bf16x4(row + p.v_off + col);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kStageBatch; ++u) {
      const int i = i0 + u * kAttnThreads;
      if (i < items) {
        const int j = i / nq, q = i - j * nq;
        *reinterpret_cast<uint2*>(Ks + j * kKRow + 4 * q) = kv[u];
        *reinterpret_cast<uint2*>(Vs + j * kKRow + 4 * q) = vv[u];
      }
    }
  }
  __syncthreads();
  // RoPE of the action-token keys (self-attention), in place
  if (!p.cross) {
    const int n = (p.S - p.npre) * half;
    for (int i = tid; i < n; i += kAttnThreads) {
      const int t = i / half, c = i - t * half;
      bf16* kr = Ks + (p.npre + t) * kKRow;
      float r0, r1;
      rope_pair(__bfloat162float(kr[c]), __bfloat162float(kr[c + half]), p.rope[(base + t) * half + c], r0, r1);
      kr[c] = __float2bfloat16_rn(r0);
      kr[c + half] = __float2bfloat16_rn(r1);
    }
    __syncthreads();
  }

  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int lr = lane & 7, lm = lane >> 3;  // ldmatrix: row within, and index of, the lane's 8x8 matrix
  const int groups = p.heads / p.kv_heads;
  const int hgroups = groups / G;  // tasks per m-tile
  const int n_mt = p.chunk_pad / 16;
  const int tasks = hgroups * n_mt;
  const int t_lo = static_cast<int>((static_cast<long long>(tasks) * blockIdx.z) / gridDim.z);
  const int t_hi = static_cast<int>((static_cast<long long>(tasks) * (blockIdx.z + 1)) / gridDim.z);
  const int nkk = p.S_pad / 16;
  // scores in log2 units: s = (q . k) * log2(e) / sqrt(hw) + bias, probabilities 2^(s - max)
  const float sc = 1.4426950408889634f / p.sqrt_hw;
  auto merge = [](float& m0, float& l0, float m1, float l1) {
    const float mn = fmaxf(m0, m1);
    if (mn != -INFINITY)
      l0 = (m0 == -INFINITY ? 0.0f : l0 * ex2_approx(m0 - mn)) + (m1 == -INFINITY ? 0.0f : l1 * ex2_approx(m1 - mn));
    m0 = mn;
  };
  for (int task = t_lo; task < t_hi; ++task) {
    const int hg = task / n_mt, mt = task - hg * n_mt;
    const int h0 = kvh * groups + hg * G;  // first query head of the task
    // the task's G x 16 query rows with RoPE (position base + row)
    for (int i = tid; i < G * 16 * (kHwPad / 4); i += kAttnThreads) {
      const int gr = i / (kHwPad / 4), q = i - gr * (kHwPad / 4);
      const int gh = gr / 16, r = gr - gh * 16;
      uint2 v = make_uint2(z2, z2);
      if (mt * 16 + r < p.chunk && q < nq)
        v = ld_bf16x4(p.qkv + (tok0 + mt * 16 + r) * p.qkv_ld + (h0 + gh) * hw + 4 * q);
      *reinterpret_cast<uint2*>(Qs + gr * kKRow + 4 * q) = v;
    }
    __syncthreads();
    for (int i = tid; i < G * 16 * half; i += kAttnThreads) {
      const int gr = i / half, c = i - gr * half;
      const int r = gr & 15;
      float r0, r1;
      rope_pair(__bfloat162float(Qs[gr * kKRow + c]), __bfloat162float(Qs[gr * kKRow + c + half]),
                p.rope[(base + mt * 16 + r) * half + c], r0, r1);
      Qs[gr * kKRow + c] = __float2bfloat16_rn(r0);
      Qs[gr * kKRow + c + half] = __float2bfloat16_rn(r1);
    }
    __syncthreads();
    // A fragments: matrices (rows 0-7, k lo), (rows 8-15, k lo), (rows 0-7, k hi), (rows 8-15, k hi)
    uint32_t qa[G][kHwPad / 16][4];
#pragma unroll
    for (int gh = 0; gh < G; ++gh)
#pragma unroll
      for (int ks = 0; ks < kHwPad / 16; ++ks)
        ldsm_x4(Qs + (gh * 16 + (lm & 1) * 8 + lr) * kKRow + ks * 16 + (lm >> 1) * 8, qa[gh][ks]);
    const int row0 = mt * 16 + g, row1 = row0 + 8;
    // scores of the 16 keys of block kk for the G heads (K fragments loaded once)
    auto scores16 = [&](int kk, float (&s)[G][2][4]) {
      // B fragments: matrices (keys 0-7, k lo), (keys 0-7, k hi), (keys 8-15, k lo), (keys 8-15, k hi)
      uint32_t kb[kHwPad / 16][4];
#pragma unroll
      for (int ks = 0; ks < kHwPad / 16; ++ks)
        ldsm_x4(Ks + (kk * 16 + (lm >> 1) * 8 + lr) * kKRow + ks * 16 + (lm & 1) * 8, kb[ks]);
      float acc[G][2][4];
#pragma unroll
      for (int gh = 0; gh < G; ++gh)
#pragma unroll
        for (int x = 0; x < 2; ++x)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[gh][x][e] = 0.0f;
#pragma unroll
      for (int ks = 0; ks < kHwPad / 16; ++ks)
#pragma unroll
        for (int gh = 0; gh < G; ++gh)
#pragma unroll
          for (int x = 0; x < 2; ++x) mma_bf16_16816(acc[gh][x], qa[gh][ks], kb[ks][2 * x], kb[ks][2 * x + 1]);
      float2 bias[2];
#pragma unroll
      for (int x = 0; x < 2; ++x) bias[x] = *reinterpret_cast<const float2*>(kbias + (2 * kk + x) * 8 + 2 * t4);
#pragma unroll
      for (int gh = 0; gh < G; ++gh)
#pragma unroll
        for (int x = 0; x < 2; ++x)
#pragma unroll
          for (int e = 0; e < 4; ++e) s[gh][x][e] = fmaf(acc[gh][x][e], sc, (e & 1) ? bias[x].y : bias[x].x);
      // causal action tokens: only blocks reaching past this m-tile's first row
      if (!p.cross && kk * 16 + 15 - p.npre > mt * 16) {
#pragma unroll
        for (int x = 0; x < 2; ++x)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = (2 * kk + x) * 8 + 2 * t4 + (e & 1);
            if (j >= p.npre && j - p.npre > (e < 2 ? row0 : row1))
#pragma unroll
              for (int gh = 0; gh < G; ++gh) s[gh][x][e] = -INFINITY;
          }
      }
    };
    // phase 1: this warp's key blocks kk = warp, warp + 4, ...: online max / sum
    float m[G][2], l[G][2];
#pragma unroll
    for (int gh = 0; gh < G; ++gh) {
      m[gh][0] = m[gh][1] = -INFINITY;
      l[gh][0] = l[gh][1] = 0.0f;
    }
    for (int kk = warp; kk < nkk; kk += kAttnWarps) {
      float s[G][2][4];
      scores16(kk, s);
#pragma unroll
      for (int gh = 0; gh < G; ++gh)
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          const float tmax = fmaxf(fmaxf(s[gh][0][2 * rr], s[gh][0][2 * rr + 1]),
                                   fmaxf(s[gh][1][2 * rr], s[gh][1][2 * rr + 1]));
          const float mn = fmaxf(m[gh][rr], tmax);
          if (mn != -INFINITY) {
            l[gh][rr] = (m[gh][rr] == -INFINITY ? 0.0f : l[gh][rr] * ex2_approx(m[gh][rr] - mn)) +
                        ex2_approx(s[gh][0][2 * rr] - mn) + ex2_approx(s[gh][0][2 * rr + 1] - mn) +
                        ex2_approx(s[gh][1][2 * rr] - mn) + ex2_approx(s[gh][1][2 * rr + 1] - mn);
            m[gh][rr] = mn;
          }
        }
    }
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1)
#pragma unroll
      for (int gh = 0; gh < G; ++gh)
#pragma unroll
        for (int rr = 0; rr < 2; ++rr)
          merge(m[gh][rr], l[gh][rr], __shfl_xor_sync(0xffffffffu, m[gh][rr], off),
                __shfl_xor_sync(0xffffffffu, l[gh][rr], off));
    if (t4 == 0) {
#pragma unroll
      for (int gh = 0; gh < G; ++gh) {
        float* rd = red + ((gh * kAttnWarps + warp) * 16) * 2;
        rd[g * 2] = m[gh][0];
        rd[g * 2 + 1] = l[gh][0];
        rd[(g + 8) * 2] = m[gh][1];
        rd[(g + 8) * 2 + 1] = l[gh][1];
      }
    }
    __syncthreads();
    // every thread combines the warps' partials of its rows in warp order
    float inv[G][2];
#pragma unroll
    for (int gh = 0; gh < G; ++gh)
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        const int row = g + 8 * rr;
        float mm = -INFINITY, ll = 0.0f;
        for (int w = 0; w < kAttnWarps; ++w) {
          const float* rd = red + ((gh * kAttnWarps + w) * 16 + row) * 2;
          merge(mm, ll, rd[0], rd[1]);
        }
        m[gh][rr] = mm;
        inv[gh][rr] = 1.0f / ll;
      }
    // phase 2: probabilities rounded to bf16 (kernels.h:320-321) times V over this warp's keys
    float o[G][kHwPad / 8][4];
#pragma unroll
    for (int gh = 0; gh < G; ++gh)
#pragma unroll
      for (int dn = 0; dn < kHwPad / 8; ++dn)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[gh][dn][e] = 0.0f;
    for (int kk = warp; kk < nkk; kk += kAttnWarps) {
      float s[G][2][4];
      scores16(kk, s);
      // B fragments of V (transposed): matrices (keys lo, dims dn), (keys hi, dims dn),
      // (keys lo, dims dn + 1), (keys hi, dims dn + 1)
      uint32_t vb[kHwPad / 16][4];
#pragma unroll
      for (int d2 = 0; d2 < kHwPad / 16; ++d2)
        ldsm_x4_t(Vs + (kk * 16 + (lm & 1) * 8 + lr) * kKRow + (2 * d2 + (lm >> 1)) * 8, vb[d2]);
#pragma unroll
      for (int gh = 0; gh < G; ++gh) {
        uint32_t pa[4];
        pa[0] = pack_bf16(ex2_approx(s[gh][0][0] - m[gh][0]) * inv[gh][0],
                          ex2_approx(s[gh][0][1] - m[gh][0]) * inv[gh][0]);
        pa[1] = pack_bf16(ex2_approx(s[gh][0][2] - m[gh][1]) * inv[gh][1],
                          ex2_approx(s[gh][0][3] - m[gh][1]) * inv[gh][1]);
        pa[2] = pack_bf16(ex2_approx(s[gh][1][0] - m[gh][0]) * inv[gh][0],
                          ex2_approx(s[gh][1][1] - m[gh][0]) * inv[gh][0]);
        pa[3] = pack_bf16(ex2_approx(s[gh][1][2] - m[gh][1]) * inv[gh][1],
                          ex2_approx(s[gh][1][3] - m[gh][1]) * inv[gh][1]);
#pragma unroll
        for (int d2 = 0; d2 < kHwPad / 16; ++d2) {
          mma_bf16_16816(o[gh][2 * d2], pa, vb[d2][0], vb[d2][1]);
          mma_bf16_16816(o[gh][2 * d2 + 1], pa, vb[d2][2], vb[d2][3]);
        }
      }
    }
    // partial outputs of the warps, summed in warp order (one head at a time)
#pragma unroll
    for (int gh = 0; gh < G; ++gh) {
#pragma unroll
      for (int dn = 0; dn < kHwPad / 8; ++dn) {
        const int c = dn * 8 + 2 * t4;
        *reinterpret_cast<float2*>(opart + (warp * 16 + g) * kHwPad + c) = make_float2(o[gh][dn][0], o[gh][dn][1]);
        *reinterpret_cast<float2*>(opart + (warp * 16 + g + 8) * kHwPad + c) = make_float2(o[gh][dn][2], o[gh][dn][3]);
      }
      __syncthreads();
      for (int i = tid; i < 16 * (hw / 2); i += kAttnThreads) {
        const int r = i / (hw / 2), c = 2 * (i - r * (hw / 2));
        if (mt * 16 + r < p.chunk) {
          float a0 = 0.0f, a1 = 0.0f;
          for (int w = 0; w < kAttnWarps; ++w) {
            const float2 v = *reinterpret_cast<const float2*>(opart + (w * 16 + r) * kHwPad + c);
            a0 += v.x;
            a1 += v.y;
          }
          *reinterpret_cast<__nv_bfloat162*>(p.out + (tok0 + mt * 16 + r) * p.out_ld + (h0 + gh) * hw + c) =
              __floats2bfloat162_rn(a0, a1);
        }
      }
      __syncthreads();
    }
  }
}

// Batched variant: one CTA per (sample, K / V head), K and V staged once;
// each warp owns whole tasks (G query heads x 16 rows over every key), so a
// task needs no cross-warp merge and no CTA barrier after the staging.  The
// warp stages its queries with RoPE in its own buffer.  Same arithmetic as
// attention_kernel (online max / sum over the keys in block order, then
// bf16 probabilities times V).
template <int G>
__global__ void __launch_bounds__(kAttnThreads) attention_rows_kernel(const AttnParams p) {
  griddep_wait();
  griddep_launch();
  extern __shared__ __align__(16) uint8_t smem[];
  bf16* Ks = reinterpret_cast<bf16*>(smem);                  // [S_pad][kKRow]
  bf16* Vs = Ks + static_cast<long long>(p.S_pad) * kKRow;  // [S_pad][kKRow]
  float* kbias = reinterpret_cast<float*>(Vs + static_cast<long long>(p.S_pad) * kKRow);  // [S_pad]
  bf16* Qw = reinterpret_cast<bf16*>(kbias + p.S_pad);      // [warps][G][16][kKRow]
  const int b = blockIdx.x, kvh = blockIdx.y;
  const int tid = threadIdx.x;
  const int hw = p.hw, half = hw / 2, nq = hw / 4;
  const int base = p.cross ? 0 : p.valid[static_cast<long long>(b) * p.valid_b];
  const long long tok0 = static_cast<long long>(b) * p.chunk;
  const uint32_t z2 = 0u;
  for (int i = tid; i < p.S_pad * (kHwPad / 4); i += kAttnThreads) {
    const int j = i / (kHwPad / 4), q = i - j * (kHwPad / 4);
    if (j >= p.S || q >= nq) {
      *reinterpret_cast<uint2*>(Ks + j * kKRow + 4 * q) = make_uint2(z2, z2);
      *reinterpret_cast<uint2*>(Vs + j * kKRow + 4 * q) = make_uint2(z2, z2);
    }
  }
  for (int i = tid; i < p.S_pad; i += kAttnThreads) {
    float bias = -INFINITY;
    if (i < p.npre) bias = p.mask[static_cast<long long>(b) * p.mask_b + i] != 0 ? 0.0f : -INFINITY;
    else if (i < p.S) bias = 0.0f;
    kbias[i] = bias;
  }
  const int items = p.S * nq;
  for (int i0 = tid; i0 < items; i0 += kAttnThreads * kStageBatch) {
    uint2 kv[kStageBatch], vv[kStageBatch];
#pragma unroll
    for (int u = 0; u < kStageBatch; ++u) {
      const int i = i0 + u * kAttnThreads;
      kv[u] = make_uint2(z2, z2);
      vv[u] = make_uint2(z2, z2);
      if (i < items) {
        const int j = i / nq, q = i - j * nq;
        const int col = kvh * hw + 4 * q;
        if (p.cross) {
          const bf16* row = p.kvp + (static_cast<long long>(b) * p.kvp_b + j) * p.kvp_ld;
          kv[u] = ld_bf16x4(row + col);
          vv[u] = ld_bf16x4(row + p.kv_w + col);
        } else if (j < p.npre) {
          const long long o = static_cast<long long>(b) * p.p_b * p.p_ld + p.layer_off +
                              static_cast<long long>(j) * p.p_ld + col;
          kv[u] = bf16x4_of(p.pk + o);
          vv[u] = bf16x4_of(p.pv + o);
        } else {
          const bf16* row = p.qkv + (tok0 + j - p.npre) * p.qkv_ld;
          kv[u] = ld_bf16x4(row + p.k_off + col);
          vv[u] = ld_bf16x4(row + p.v_off + col);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kStageBatch; ++u) {
      const int i = i0 + u * kAttnThreads;
      if (i < items) {
        const int j = i / nq, q = i - j * nq;
        *reinterpret_cast<uint2*>(Ks + j * kKRow + 4 * q) = kv[u];
        *reinterpret_cast<uint2*>(Vs + j * kKRow + 4 * q) = vv[u];
      }
    }
  }
  __syncthreads();
  if (!p.cross) {
    const int n = (p.S - p.npre) * half;
    for (int i = tid; i < n; i += kAttnThreads) {
      const int t = i / half, c = i - t * half;
      bf16* kr = Ks + (p.npre + t) * kKRow;
      float r0, r1;
      rope_pair(__bfloat162float(kr[c]), __bfloat162float(kr[c + half]), p.rope[(base + t) * half + c], r0, r1);
      kr[c] = __float2bfloat16_rn(r0);
      kr[c + half] = __float2bfloat16_rn(r1);
    }
    __syncthreads();
  }

  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int lr = lane & 7, lm = lane >> 3;
  const int groups = p.heads / p.kv_heads;
  const int n_mt = p.chunk_pad / 16;
  const int tasks = (groups / G) * n_mt;
  const int nkk = p.S_pad / 16;
  const float sc = 1.4426950408889634f / p.sqrt_hw;
  bf16* Qs = Qw + warp * G * 16 * kKRow;
  for (int task = warp; task < tasks; task += kAttnWarps) {
    const int hg = task / n_mt, mt = task - hg * n_mt;
    const int h0 = kvh * groups + hg * G;
    __syncwarp();
    // raw query rows, then RoPE in place (each lane rotates whole pairs)
    for (int i = lane; i < G * 16 * (kHwPad / 4); i += 32) {
      const int gr = i / (kHwPad / 4), q = i - gr * (kHwPad / 4);
      const int gh = gr / 16, r = gr - gh * 16;
      uint2 v = make_uint2(z2, z2);
      if (mt * 16 + r < p.chunk && q < nq)
        v = ld_bf16x4(p.qkv + (tok0 + mt * 16 + r) * p.qkv_ld + (h0 + gh) * hw + 4 * q);
      *reinterpret_cast<uint2*>(Qs + gr * kKRow + 4 * q) = v;
    }
    __syncwarp();
    for (int i = lane; i < G * 16 * half; i += 32) {
      const int gr = i / half, c = i - gr * half;
      const int r = gr & 15;
      float r0, r1;
      rope_pair(__bfloat162float(Qs[gr * kKRow + c]), __bfloat162float(Qs[gr * kKRow + c + half]),
                p.rope[(base + mt * 16 + r) * half + c], r0, r1);
      Qs[gr * kKRow + c] = __float2bfloat16_rn(r0);
      Qs[gr * kKRow + c + half] = __float2bfloat16_rn(r1);
    }
    __syncwarp();
    uint32_t qa[G][kHwPad / 16][4];
#pragma unroll
    for (int gh = 0; gh < G; ++gh)
#pragma unroll
      for (int ks = 0; ks < kHwPad / 16; ++ks)
        ldsm_x4(Qs + (gh * 16 + (lm & 1) * 8 + lr) * kKRow + ks * 16 + (lm >> 1) * 8, qa[gh][ks]);
    const int row0 = mt * 16 + g, row1 = row0 + 8;
    auto scores16 = [&](int kk, float (&s)[G][2][4]) {
      uint32_t kb[kHwPad / 16][4];
#pragma unroll
      for (int ks = 0; ks < kHwPad / 16; ++ks)
        ldsm_x4(Ks + (kk * 16 + (lm >> 1) * 8 + lr) * kKRow + ks * 16 + (lm & 1) * 8, kb[ks]);
      float acc[G][2][4];
#pragma unroll
      for (int gh = 0; gh < G; ++gh)
#pragma unroll
        for (int x = 0; x < 2; ++x)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[gh][x][e] = 0.0f;
#pragma unroll
      for (int ks = 0; ks < kHwPad / 16; ++ks)
#pragma unroll
        for (int gh = 0; gh < G; ++gh)
#pragma unroll
          for (int x = 0; x < 2; ++x) mma_bf16_16816(acc[gh][x], qa[gh][ks], kb[ks][2 * x], kb[ks][2 * x + 1]);
      float2 bias[2];
#pragma unroll
      for (int x = 0; x < 2; ++x) bias[x] = *reinterpret_cast<const float2*>(kbias + (2 * kk + x) * 8 + 2 * t4);
#pragma unroll
      for (int gh = 0; gh < G; ++gh)
#pragma unroll
        for (int x = 0; x < 2; ++x)
#pragma unroll
          for (int e = 0; e < 4; ++e) s[gh][x][e] = fmaf(acc[gh][x][e], sc, (e & 1) ? bias[x].y : bias[x].x);
      if (!p.cross && kk * 16 + 15 - p.npre > mt * 16) {
#pragma unroll
        for (int x = 0; x < 2; ++x)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = (2 * kk + x) * 8 + 2 * t4 + (e & 1);
            if (j >= p.npre && j - p.npre > (e < 2 ? row0 : row1))
#pragma unroll
              for (int gh = 0; gh < G; ++gh) s[gh][x][e] = -INFINITY;
          }
      }
    };
    float m[G][2], l[G][2];
#pragma unroll
    for (int gh = 0; gh < G; ++gh) {
      m[gh][0] = m[gh][1] = -INFINITY;
      l[gh][0] = l[gh][1] = 0.0f;
    }
    for (int kk = 0; kk < nkk; ++kk) {
      float s[G][2][4];
      scores16(kk, s);
#pragma unroll
      for (int gh = 0; gh < G; ++gh)
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          const float tmax = fmaxf(fmaxf(s[gh][0][2 * rr], s[gh][0][2 * rr + 1]),
                                   fmaxf(s[gh][1][2 * rr], s[gh][1][2 * rr + 1]));
          const float mn = fmaxf(m[gh][rr], tmax);
          if (mn != -INFINITY) {
            l[gh][rr] = (m[gh][rr] == -INFINITY ? 0.0f : l[gh][rr] * ex2_approx(m[gh][rr] - mn)) +
                        ex2_approx(s[gh][0][2 * rr] - mn) + ex2_approx(s[gh][0][2 * rr + 1] - mn) +
                        ex2_approx(s[gh][1][2 * rr] - mn) + ex2_approx(s[gh][1][2 * rr + 1] - mn);
            m[gh][rr] = mn;
          }
        }
    }
    float inv[G][2];
#pragma unroll
    for (int gh = 0; gh < G; ++gh)
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
#pragma unroll
        for (int off = 1; off <= 2; off <<= 1) {
          const float mo = __shfl_xor_sync(0xffffffffu, m[gh][rr], off);
          const float lo = __shfl_xor_sync(0xffffffffu, l[gh][rr], off);
          const float mn = fmaxf(m[gh][rr], mo);
          if (mn != -INFINITY)
            l[gh][rr] = (m[gh][rr] == -INFINITY ? 0.0f : l[gh][rr] * ex2_approx(m[gh][rr] - mn)) +
                        (mo == -INFINITY ? 0.0f : lo * ex2_approx(mo - mn));
          m[gh][rr] = mn;
        }
        inv[gh][rr] = 1.0f / l[gh][rr];
      }
    float o[G][kHwPad / 8][4];
#pragma unroll
    for (int gh = 0; gh < G; ++gh)
#pragma unroll
      for (int dn = 0; dn < kHwPad / 8; ++dn)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[gh][dn][e] = 0.0f;
    for (int kk = 0; kk < nkk; ++kk) {
      float s[G][2][4];
      scores16(kk, s);
      uint32_t vb[kHwPad / 16][4];
#pragma unroll
      for (int d2 = 0; d2 < kHwPad / 16; ++d2)
        ldsm_x4_t(Vs + (kk * 16 + (lm & 1) * 8 + lr) * kKRow + (2 * d2 + (lm >> 1)) * 8, vb[d2]);
#pragma unroll
      for (int gh = 0; gh < G; ++gh) {
        uint32_t pa[4];
        pa[0] = pack_bf16(ex2_approx(s[gh][0][0] - m[gh][0]) * inv[gh][0],
                          ex2_approx(s[gh][0][1] - m[gh][0]) * inv[gh][0]);
        pa[1] = pack_bf16(ex2_approx(s[gh][0][2] - m[gh][1]) * inv[gh][1],
                          ex2_approx(s[gh][0][3] - m[gh][1]) * inv[gh][1]);
        pa[2] = pack_bf16(ex2_approx(s[gh][1][0] - m[gh][0]) * inv[gh][0],
                          ex2_approx(s[gh][1][1] - m[gh][0]) * inv[gh][0]);
        pa[3] = pack_bf16(ex2_approx(s[gh][1][2] - m[gh][1]) * inv[gh][1],
                          ex2_approx(s[gh][1][3] - m[gh][1]) * inv[gh][1]);
#pragma unroll
        for (int d2 = 0; d2 < kHwPad / 16; ++d2) {
          mma_bf16_16816(o[gh][2 * d2], pa, vb[d2][0], vb[d2][1]);
          mma_bf16_16816(o[gh][2 * d2 + 1], pa, vb[d2][2], vb[d2][3]);
        }
      }
    }
#pragma unroll
    for (int gh = 0; gh < G; ++gh)
#pragma unroll
      for (int dn = 0; dn < kHwPad / 8; ++dn) {
        const int c = dn * 8 + 2 * t4;
        if (c < hw) {
          bf16* orow = p.out + (h0 + gh) * hw + c;
          if (row0 < p.chunk)
            *reinterpret_cast<__nv_bfloat162*>(orow + (tok0 + row0) * p.out_ld) =
                __floats2bfloat162_rn(o[gh][dn][0], o[gh][dn][1]);
          if (row1 < p.chunk)
            *reinterpret_cast<__nv_bfloat162*>(orow + (tok0 + row1) * p.out_ld) =
                __floats2bfloat162_rn(o[gh][dn][2], o[gh][dn][3]);
        }
      }
  }
}

// ---------------------------------------------------------------------------
// Small-row GEMM (rows <= kSmallRows tokens, e.g. one 50-token chunk): the
// tcgen05 GEMM would run one 256-row N tile on M / 128 CTAs, so instead the
// K range is split over many CTAs.  CTA (m16, ks) computes a 16-row block of
// W times all rows over K slice ks on mma.sync m16n8k16 (A = weights straight
// from global, B = activations staged in shared memory; bf16 operands, or
// fp16 W against the fp16 hi and lo planes of split activations); the four
// warps take alternate 16-wide K steps and add their tiles in warp order.
// partial[ks][row][m] then goes to small_epilogue_kernel, which adds the
// slices in slice order and applies the tcgen05 GEMM's epilogue.
constexpr int kSmallRows = 64;
constexpr int kSmallK = 128;  // K per CTA
constexpr int kSmallLd = kSmallK + 8;  // staged row (16-bit elements)

struct SmallGemm {
  const void* w;       // [M_pad][ld_w]: bf16, or fp16 [W | W] (split)
  int ld_w, M, kp;     // kp: K (multiple of 64)
  int split;           // 1: fp16 weights and fp16 hi / lo activations [rows][2 kp]
  const void* x;       // activations [rows][ld_x] (16-bit)
  int ld_x, rows;
  float* partial;      // [nks][rows][M_pad16]
  int m_pad;           // M rounded up to 16
};

template <bool SPLIT>
__global__ void __launch_bounds__(128) small_gemm_kernel(const SmallGemm g) {
  // [plane][row][k] staged activations; reused as [warp][16][rows] fp32 tiles
  __shared__ __align__(16) uint16_t xs[2 * kSmallRows * kSmallLd];
  float* red = reinterpret_cast<float*>(xs);
  const int mb = blockIdx.x, ks = blockIdx.y;
  const int k0 = ks * kSmallK;
  const int kn = min(kSmallK, g.kp - k0);  // multiple of 16
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g4 = lane >> 2, t4 = lane & 3;
  // this warp's weight fragments (K steps warp * 16 and warp * 16 + 64) do not
  // depend on the previous kernel: loaded before the dependency wait
  const uint16_t* wrow0 = static_cast<const uint16_t*>(g.w) + static_cast<long long>(mb * 16 + g4) * g.ld_w + k0;
  const uint16_t* wrow1 = wrow0 + 8LL * g.ld_w;
  uint32_t a[kSmallK / 64][4];
#pragma unroll
  for (int j = 0; j < kSmallK / 64; ++j) {
    const int kk = warp * 16 + 64 * j;
    const bool in = kk < kn;
    a[j][0] = in ? __ldg(reinterpret_cast<const uint32_t*>(wrow0 + kk + 2 * t4)) : 0u;
    a[j][1] = in ? __ldg(reinterpret_cast<const uint32_t*>(wrow1 + kk + 2 * t4)) : 0u;
    a[j][2] = in ? __ldg(reinterpret_cast<const uint32_t*>(wrow0 + kk + 2 * t4 + 8)) : 0u;
    a[j][3] = in ? __ldg(reinterpret_cast<const uint32_t*>(wrow1 + kk + 2 * t4 + 8)) : 0u;
  }
  griddep_wait();
  griddep_launch();
  // stage x[rows][k0 .. k0 + kn) (both planes when split); rows >= g.rows are zero
  const int nq = kn / 8;  // 16-byte groups per row and plane
  for (int i = tid; i < (SPLIT ? 2 : 1) * kSmallRows * nq; i += 128) {
    const int pl = i / (kSmallRows * nq);
    const int rem = i - pl * kSmallRows * nq;
    const int r = rem / nq, q = rem - r * nq;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (r < g.rows)
      v = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(g.x) + static_cast<long long>(r) * g.ld_x +
                                               pl * g.kp + k0 + 8 * q));
    *reinterpret_cast<uint4*>(&xs[(pl * kSmallRows + r) * kSmallLd + 8 * q]) = v;
  }
  __syncthreads();
  const int nt = (g.rows + 7) / 8;  // n-tiles of 8 rows
  float acc[SPLIT ? 2 : 1][kSmallRows / 8][4];
#pragma unroll
  for (int pl = 0; pl < (SPLIT ? 2 : 1); ++pl)
#pragma unroll
    for (int n = 0; n < kSmallRows / 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[pl][n][e] = 0.0f;
#pragma unroll
  for (int j = 0; j < kSmallK / 64; ++j) {
    const int kk = warp * 16 + 64 * j;
    if (kk >= kn) break;
    const uint32_t (&a_)[4] = a[j];
#pragma unroll
    for (int n = 0; n < kSmallRows / 8; ++n) {
      if (n < nt) {
#pragma unroll
        for (int pl = 0; pl < (SPLIT ? 2 : 1); ++pl) {
          const uint16_t* xr = &xs[(pl * kSmallRows + n * 8 + g4) * kSmallLd + kk + 2 * t4];
          const uint32_t b0 = *reinterpret_cast<const uint32_t*>(xr);
          const uint32_t b1 = *reinterpret_cast<const uint32_t*>(xr + 8);
          if constexpr (SPLIT) {
            asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                "{%0,%1,%2,%3};"
                : "+f"(acc[pl][n][0]), "+f"(acc[pl][n][1]), "+f"(acc[pl][n][2]), "+f"(acc[pl][n][3])
                : "r"(a_[0]), "r"(a_[1]), "r"(a_[2]), "r"(a_[3]), "r"(b0), "r"(b1));
          } else {
            mma_bf16_16816(acc[pl][n], a_, b0, b1);
          }
        }
      }
    }
  }
  // warp tiles (hi + lo planes) to shared memory, then added in warp order
  __syncthreads();  // every warp is done with the staged activations
#pragma unroll
  for (int n = 0; n < kSmallRows / 8; ++n) {
    if (n < nt) {
      float v[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) v[e] = SPLIT ? acc[0][n][e] + acc[SPLIT ? 1 : 0][n][e] : acc[0][n][e];
      float* rw = red + warp * 16 * kSmallRows;
      rw[g4 * kSmallRows + n * 8 + 2 * t4] = v[0];
      rw[g4 * kSmallRows + n * 8 + 2 * t4 + 1] = v[1];
      rw[(g4 + 8) * kSmallRows + n * 8 + 2 * t4] = v[2];
      rw[(g4 + 8) * kSmallRows + n * 8 + 2 * t4 + 1] = v[3];
    }
  }
  __syncthreads();
  for (int i = tid; i < 16 * g.rows; i += 128) {
    const int r = i / 16, mm = i - r * 16;  // consecutive threads: consecutive output rows m
    const int o = mm * kSmallRows + r;
    const float v = red[o] + red[16 * kSmallRows + o] + red[32 * kSmallRows + o] + red[48 * kSmallRows + o];
    g.partial[(static_cast<long long>(ks) * g.rows + r) * g.m_pad + mb * 16 + mm] = v;
  }
}

struct SmallEpilogue {
  const float* partial;
  int nks, rows, m_valid, m_pad;
  const float* bias;
  const float* add_vec;
  int act;          // tc::kActNone / kActSilu / kActSwiGLU
  int out_kind;     // 0 fp32, 1 bf16, 2 fp16, 3 fp16 hi / lo
  void* out;
  long long out_ld;
  long long lo_off;
  int ch_off;
};

// y = sum of the K slices in slice order + bias + add_vec, then the act and
// the store of the tcgen05 epilogue (SwiGLU: rows 2f / 2f + 1 are gate / up)
__global__ void small_epilogue_kernel(const SmallEpilogue e) {
  griddep_wait();
  griddep_launch();
  const bool swiglu = e.act == tc::kActSwiGLU;
  const int cols = swiglu ? e.m_valid / 2 : e.m_valid;
  const long long total = static_cast<long long>(e.rows) * cols;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / cols), c = static_cast<int>(i - static_cast<long long>(r) * cols);
    auto y_of = [&](int m) {
      float y = 0.0f;
      for (int k = 0; k < e.nks; ++k) y += e.partial[(static_cast<long long>(k) * e.rows + r) * e.m_pad + m];
      if (e.bias != nullptr) y += e.bias[m];
      if (e.add_vec != nullptr) y += e.add_vec[m];
      return y;
    };
    float y;
    if (swiglu) {
      const float gte = bf16r(y_of(2 * c)), up = bf16r(y_of(2 * c + 1));
      y = up * silu_fast(gte);
    } else {
      y = y_of(c);
      if (e.act == tc::kActSilu) y = silu_fast(y);
    }
    const long long o = static_cast<long long>(r) * e.out_ld + e.ch_off + c;
    if (e.out_kind == 0) {
      static_cast<float*>(e.out)[o] = y;
    } else if (e.out_kind == 1) {
      static_cast<bf16*>(e.out)[o] = __float2bfloat16_rn(y);
    } else if (e.out_kind == 2) {
      static_cast<__half*>(e.out)[o] = to_half_sat(y);
    } else {
      const __half hi = to_half_sat(y);
      static_cast<__half*>(e.out)[o] = hi;
      static_cast<__half*>(e.out)[o + e.lo_off] = __float2half_rn(y - __half2float(hi));
    }
  }
}

// ---------------------------------------------------------------------------

struct Mat {
  void* w = nullptr;
  int rows = 0, rows_pad = 0, kp = 0;  // kp: padded input width (split GEMMs read 2 kp)
  bool split = false;                  // fp16 [rows_pad][2 kp] = [W | W] against hi / lo activations
};

struct Layer {
  bool cross = false;
  float* in_norm = nullptr;
  float* post_norm = nullptr;
  Mat qkv;   // self: [Wq; Wk; Wv]; cross: Wq
  Mat k, v;  // cross: split Wk / Wv over the cache width
  Mat o, gu, down;
};

class SmolVLA final : public SmolVLADevice {
 public:
  SmolVLA(std::shared_ptr<DeviceContext> ctx) : ctx_(std::move(ctx)) {}
  ~SmolVLA() override {
    for (auto& [k, g] : graphs_) cudaGraphExecDestroy(g.first);
  }
  bool load(const TensorTable& t, std::string& err);
  const SmolVLAConfig& config() const noexcept override { return cfg_; }
  int embed_suffix(const float* noisy, std::size_t chunk, float timestep, float* out, std::string& err) noexcept override;
  int run_expert(const float* suffix, std::size_t chunk, const float* keys, const float* values,
                 const std::uint8_t* mask, std::size_t prefix, float* out, std::string& err) noexcept override;
  int project_actions(const float* hidden, std::size_t chunk, float* out, std::string& err) noexcept override;
  int denoise(const float* noisy, std::size_t chunk, float timestep, const float* keys, const float* values,
              const std::uint8_t* mask, std::size_t prefix, float* out, std::string& err) noexcept override;
  int sample(const float* noise, std::size_t batch, std::size_t chunk, std::size_t steps, const float* keys,
             const float* values, const std::uint8_t* mask, std::size_t prefix, bool shared_prefix, float* out,
             bool on_device, void* stream, std::string& err) noexcept override;
  int reserve(std::size_t batch, std::size_t chunk, std::size_t prefix, bool shared_prefix,
              std::string& err) noexcept override;
  std::uint64_t kernel_launches() const noexcept override { return launches_; }

 private:
  // largest split-K partial buffer of any small-row GEMM: K slices x rows x M
  std::size_t small_part_floats() const {
    const std::size_t kmax = static_cast<std::size_t>(std::max({Wp_, attn_p_, mlp_p_, Cp_, Ap_}));
    const std::size_t mmax = static_cast<std::size_t>(std::max({qkv_ld_, 2 * mlp_, Wp_, kvp_ld_, Ap_ + 128}));
    return (kmax + kSmallK - 1) / kSmallK * kSmallRows * mmax;
  }
  bool gemm(const Mat& m, const void* src, long long rows, void* out, int out_ld, bool out_f32, long long lo_off,
            const float* bias, const float* add_vec, int act, cudaStream_t st, std::string& err,
            long long src_rows = 0, int out_ch_off = 0, bool out_bf16 = false);
  int check_prefix(const std::uint8_t* mask, std::size_t prefix, std::size_t chunk, std::string& err) const;
  // cache upload (host or device pointers), valid counts and the cross K / V projections
  bool prepare_prefix(const float* keys, const float* values, const std::uint8_t* mask, std::size_t samples,
                      std::size_t prefix, bool device_ptrs, cudaStream_t st, std::string& err);
  // suffix embedding of rows x2_ -> h_ (time from the step counter or *t_direct)
  bool record_embed(long long rows, const float* t_direct, int steps, cudaStream_t st, std::string& err);
  // layers + final norm on h_; final output as split fp16 (mode 1) or fp32 (mode 2)
  bool record_layers(std::size_t batch, std::size_t chunk, bool shared, int final_mode, cudaStream_t st,
                     std::string& err);
  bool record_step(std::size_t batch, std::size_t chunk, std::size_t steps, bool shared, cudaStream_t st,
                   std::string& err);
  bool attention(const Layer& L, std::size_t li, std::size_t batch, std::size_t chunk, bool shared, cudaStream_t st,
                 std::string& err);
  int finish(cudaStream_t st, std::string& err);
  // heads per attention task: 3 (the reference's 15 / 5 and the SmolVLA-shaped
  // expert's 12 / 4) when the batch fills the GPU, else 1 (more, smaller CTAs)
  int attn_g(std::size_t batch) const {
    return cfg_.heads / cfg_.kv_heads % 3 == 0 && batch * cfg_.kv_heads >= static_cast<std::size_t>(ctx_->sm_count)
               ? 3
               : 1;
  }
  static std::size_t attn_rows_smem(int S_pad, int G) {
    return static_cast<std::size_t>(S_pad) * kKRow * 2 * 2 + static_cast<std::size_t>(S_pad) * 4 +
           static_cast<std::size_t>(kAttnWarps) * G * 16 * kKRow * 2;
  }
  std::size_t attn_smem(int S_pad, int G) const {
    return static_cast<std::size_t>(S_pad) * kKRow * 2 * 2 + static_cast<std::size_t>(S_pad) * 4 + static_cast<std::size_t>(G) * kAttnWarps * 16 * 2 * 4 +
           static_cast<std::size_t>(kAttnWarps) * 16 * kHwPad * 4 + static_cast<std::size_t>(G) * 16 * kKRow * 2;
  }

  std::shared_ptr<DeviceContext> ctx_;
  SmolVLAConfig cfg_{};
  int W_ = 0, Wp_ = 0, A_ = 0, Ap_ = 0, attn_ = 0, attn_p_ = 0, kvw_ = 0, mlp_ = 0, mlp_p_ = 0, Cw_ = 0, Cp_ = 0;
  int qkv_ld_ = 0, kvp_ld_ = 0;
  bool ref_layout_ = false;  // cache width == K / V width: self layers attend over the cache too
  DeviceArena wts_;
  std::vector<Layer> layers_;
  Mat in_, tin_, tout_, out_;
  float *b_in_ = nullptr, *b_tout_ = nullptr, *b_out_ = nullptr, *b_tin_ = nullptr, *wt_ = nullptr;
  float *omega_ = nullptr, *rope_ = nullptr, *final_norm_ = nullptr;
  // workspace
  DeviceArena ws_;
  std::size_t cap_rows_ = 0, cap_chunk_ = 0, cap_prefix_ = 0, cap_psamples_ = 0, cap_batch_ = 0;
  long long rows_alloc_ = 0, prow_alloc_ = 0;  // rows of the activation / prefix-row buffers
  float *x_ = nullptr, *h_ = nullptr, *v_ = nullptr, *temb_ = nullptr, *tval_ = nullptr;
  bf16* proj_ = nullptr;  // bf16 output projection (o / down), added to h by the next norm
  float *kcache_ = nullptr, *vcache_ = nullptr, *io_ = nullptr;
  float2* rope_tab_ = nullptr;  // [prefix + chunk][head_width / 2] (cos, sin), rebuilt by every call
  float* small_part_ = nullptr;  // split-K partials of the small-row GEMM
  __half *x2_ = nullptr, *a2_ = nullptr, *h12_ = nullptr, *fin2_ = nullptr, *c2_ = nullptr;
  bf16 *nb_ = nullptr, *qkv_ = nullptr, *att_ = nullptr, *act_ = nullptr, *kvp_ = nullptr;
  std::uint8_t* mask_ = nullptr;
  int *valid_ = nullptr, *step_ = nullptr;
  std::size_t prefix_ = 0;
  std::uint64_t launches_ = 0;
  // graph of one Euler step and the kernels it launches
  std::map<std::tuple<std::size_t, std::size_t, std::size_t, std::size_t, bool>,
           std::pair<cudaGraphExec_t, std::uint64_t>>
      graphs_;
};

bool SmolVLA::load(const TensorTable& t, std::string& err) {
  const HostTensor* ain = t.find("model.action_in_proj.weight");
  const HostTensor* aout = t.find("model.action_out_proj.weight");
  const HostTensor* tin = t.find("model.action_time_mlp_in.weight");
  const HostTensor* tout = t.find("model.action_time_mlp_out.weight");
  const HostTensor* st = t.find("model.state_proj.weight");
  if (ain == nullptr || aout == nullptr || tin == nullptr || tout == nullptr || st == nullptr || ain->ndim != 2 ||
      aout->ndim != 2 || tin->ndim != 2 || tout->ndim != 2 || st->ndim != 2) {
    err = "SmolVLA action-expert projections missing";
    return false;
  }
  cfg_.expert_width = ain->shape[0];
  cfg_.action_dim = ain->shape[1];
  cfg_.vlm_width = st->shape[0];
  cfg_.state_dim = st->shape[1];
  const std::size_t W = cfg_.expert_width, A = cfg_.action_dim;
  // smolvla_action_expert.cc:84-96
  if (W == 0 || W > 4096 || A == 0 || A > 256 || cfg_.vlm_width == 0 || cfg_.vlm_width > 4096 ||
      cfg_.state_dim == 0 || cfg_.state_dim > 256 || W % 2 != 0 || aout->shape[0] != A || aout->shape[1] != W ||
      tin->shape[0] != W || tin->shape[1] != 2 * W || tout->shape[0] != W || tout->shape[1] != W) {
    err = "SmolVLA projection shapes are inconsistent";
    return false;
  }
  auto vec = [&](const char* name, std::size_t n, bool f32_only) -> const HostTensor* {
    const HostTensor* v = t.find(name);
    if (v == nullptr || v->ndim != 1 || v->shape[0] != n || (f32_only && v->dtype != DType::F32)) return nullptr;
    return v;
  };
  const HostTensor* bin = vec("model.action_in_proj.bias", W, true);
  const HostTensor* bout = vec("model.action_out_proj.bias", A, true);
  const HostTensor* btin = vec("model.action_time_mlp_in.bias", W, true);
  const HostTensor* btout = vec("model.action_time_mlp_out.bias", W, true);
  const HostTensor* fnorm = vec("model.vlm_with_expert.lm_expert.norm.weight", W, false);
  if (bin == nullptr || bout == nullptr || btin == nullptr || btout == nullptr ||
      vec("model.state_proj.bias", cfg_.vlm_width, true) == nullptr || fnorm == nullptr) {
    err = "SmolVLA biases or final norm missing";
    return false;
  }
  const std::string pre = "model.vlm_with_expert.lm_expert.layers.";
  auto lt = [&](std::size_t l, const char* s) { return t.find(pre + std::to_string(l) + "." + s); };
  const HostTensor* q0 = lt(0, "self_attn.q_proj.weight");
  const HostTensor* k0 = lt(0, "self_attn.k_proj.weight");
  const HostTensor* g0 = lt(0, "mlp.gate_proj.weight");
  if (q0 == nullptr || k0 == nullptr || g0 == nullptr || q0->ndim != 2 || k0->ndim != 2 || g0->ndim != 2) {
    err = "SmolVLA layer 0 missing";
    return false;
  }
  const std::size_t attn = q0->shape[0], kvw = k0->shape[0], mlp = g0->shape[0];
  // head width: the reference fixes 64 (smolvla_action_expert.cc:120-128); this build also
  // reads flowedge.smolvla.head_width
  std::size_t hw = 64;
  if (const HostTensor* h = t.find("flowedge.smolvla.head_width"); h != nullptr) {
    const auto v = widen_f32(*h);
    if (v.size() != 1 || !(v[0] >= 2.0f) || v[0] != std::floor(v[0])) {
      err = "flowedge.smolvla.head_width must be one positive integer";
      return false;
    }
    hw = static_cast<std::size_t>(v[0]);
  }
  if (hw % 4 != 0 || hw > kHwPad || attn % hw != 0 || kvw % hw != 0 || kvw == 0 || (attn / hw) % (kvw / hw) != 0 ||
      mlp % 2 != 0 || W % 4 != 0 || W > 128 * static_cast<std::size_t>(kRmsVec)) {
    err = "SmolVLA geometry unsupported by this build (head width a multiple of 4 and <= 64, query heads a "
          "multiple of K/V heads, expert width a multiple of 4 and <= 1024)";
    return false;
  }
  std::vector<std::size_t> kv_in;
  std::size_t n = 0;
  for (; n < 48; ++n) {
    if (lt(n, "self_attn.q_proj.weight") == nullptr) break;
    const bool cross = n % 2 == 1;
    const HostTensor* k = lt(n, "self_attn.k_proj.weight");
    if (k == nullptr || k->ndim != 2) break;
    kv_in.push_back(k->shape[1]);
    (void)cross;
  }
  if (n == 0) {
    err = "no SmolVLA expert layers";
    return false;
  }
  cfg_.layers = n;
  cfg_.head_width = hw;
  cfg_.heads = attn / hw;
  cfg_.kv_heads = kvw / hw;
  cfg_.mlp_width = mlp;
  cfg_.cache_width = n > 1 ? kv_in[1] : kvw;
  W_ = static_cast<int>(W);
  Wp_ = pad(W_, 64);
  A_ = static_cast<int>(A);
  Ap_ = pad(A_, 64);
  attn_ = static_cast<int>(attn);
  attn_p_ = pad(attn_, 64);
  kvw_ = static_cast<int>(kvw);
  mlp_ = static_cast<int>(mlp);
  mlp_p_ = pad(mlp_, 64);
  Cw_ = static_cast<int>(cfg_.cache_width);
  Cp_ = pad(Cw_, 64);
  ref_layout_ = Cw_ == kvw_;
  qkv_ld_ = pad(attn_ + 2 * kvw_, 128);
  kvp_ld_ = pad(2 * kvw_, 128);

  // weights: validate all layers, then one arena
  struct Src {
    std::vector<float> in_norm, post_norm, q, k, v, o, g, u, d;
  };
  std::vector<Src> src(n);
  auto mat = [&](std::size_t l, const char* s, std::size_t rows, std::size_t cols, std::vector<float>& dst) {
    const HostTensor* m = lt(l, s);
    if (m == nullptr || m->ndim != 2 || m->shape[0] != rows || m->shape[1] != cols) return false;
    dst = widen_f32(*m);
    return true;
  };
  auto nvec = [&](std::size_t l, const char* s, std::vector<float>& dst) {
    const HostTensor* m = lt(l, s);
    if (m == nullptr || m->ndim != 1 || m->shape[0] != W) return false;
    dst = widen_f32(*m);
    return true;
  };
  for (std::size_t l = 0; l < n; ++l) {
    const bool cross = l % 2 == 1;
    const std::size_t kin = cross ? cfg_.cache_width : W;
    Src& s = src[l];
    if (!nvec(l, "input_layernorm.weight", s.in_norm) || !nvec(l, "post_attention_layernorm.weight", s.post_norm) ||
        !mat(l, "self_attn.q_proj.weight", attn, W, s.q) || !mat(l, "self_attn.k_proj.weight", kvw, kin, s.k) ||
        !mat(l, "self_attn.v_proj.weight", kvw, kin, s.v) || !mat(l, "self_attn.o_proj.weight", W, attn, s.o) ||
        !mat(l, "mlp.gate_proj.weight", mlp, W, s.g) || !mat(l, "mlp.up_proj.weight", mlp, W, s.u) ||
        !mat(l, "mlp.down_proj.weight", W, mlp, s.d)) {
      err = "SmolVLA layer " + std::to_string(l) + " tensors missing or mis-shaped";
      return false;
    }
  }

  ArenaPlan plan;
  auto plan_mat = [&](int rows, int cols, bool split) {
    plan.add(static_cast<std::size_t>(pad(rows, 128)) * pad(cols, 64) * (split ? 4 : 2));
  };
  for (std::size_t l = 0; l < n; ++l) {
    const bool cross = l % 2 == 1;
    plan_mat(cross ? attn_ : attn_ + 2 * kvw_, W_, false);
    if (cross) {
      plan_mat(kvw_, Cw_, true);
      plan_mat(kvw_, Cw_, true);
    }
    plan_mat(W_, attn_, false);
    plan_mat(2 * mlp_, W_, false);
    plan_mat(W_, mlp_, false);
    plan.add_n<float>(2 * W);
  }
  plan_mat(W_, A_, true);
  plan_mat(W_, W_, true);
  plan_mat(W_, W_, true);
  plan_mat(A_, W_, true);
  plan.add_n<float>(W * W + 6 * W + A + hw);
  if (!wts_.init(plan.total(), err)) return false;

  // bf16 [rows_pad][kp] or split fp16 [rows_pad][2 kp] from row blocks (each [rows][cols])
  // split matrices hold fp16(bf16(w)): check their range first
  bool planes_ok = true;
  auto put_mat = [&](Mat& m, const std::vector<const std::vector<float>*>& blocks, int cols, bool split,
                     const std::string& name = std::string()) {
    if (split && planes_ok)
      for (const auto* b : blocks)
        if (!check_fp16_storable(name, b->data(), b->size(), true, err)) {
          planes_ok = false;
          return;
        }
    int rows = 0;
    for (const auto* b : blocks) rows += static_cast<int>(b->size() / static_cast<std::size_t>(cols));
    m.rows = rows;
    m.rows_pad = pad(rows, 128);
    m.kp = pad(cols, 64);
    m.split = split;
    const std::size_t ld = static_cast<std::size_t>(split ? 2 * m.kp : m.kp);
    std::vector<std::uint16_t> h(static_cast<std::size_t>(m.rows_pad) * ld, 0);
    std::size_t r = 0;
    for (const auto* b : blocks) {
      const std::size_t br = b->size() / static_cast<std::size_t>(cols);
      for (std::size_t i = 0; i < br; ++i, ++r)
        for (int c = 0; c < cols; ++c) {
          const float v = (*b)[i * static_cast<std::size_t>(cols) + static_cast<std::size_t>(c)];
          if (split) {
            const std::uint16_t f = fp16_bits_of_bf16_rounded(v);
            h[r * ld + static_cast<std::size_t>(c)] = f;
            h[r * ld + static_cast<std::size_t>(m.kp + c)] = f;
          } else {
            h[r * ld + static_cast<std::size_t>(c)] = __bfloat16_as_ushort(__float2bfloat16_rn(v));
          }
        }
    }
    m.w = wts_.take(h.size() * 2);
    if (m.w != nullptr) cudaMemcpy(m.w, h.data(), h.size() * 2, cudaMemcpyHostToDevice);
  };
  auto put_vec = [&](const std::vector<float>& v) {
    float* d = wts_.take_n<float>(v.size());
    if (d != nullptr) cudaMemcpy(d, v.data(), v.size() * 4, cudaMemcpyHostToDevice);
    return d;
  };
  layers_.resize(n);
  for (std::size_t l = 0; l < n; ++l) {
    Layer& L = layers_[l];
    Src& s = src[l];
    L.cross = l % 2 == 1;
    if (L.cross) {
      put_mat(L.qkv, {&s.q}, W_, false);
      put_mat(L.k, {&s.k}, Cw_, true, pre + std::to_string(l) + ".self_attn.k_proj.weight");
      put_mat(L.v, {&s.v}, Cw_, true, pre + std::to_string(l) + ".self_attn.v_proj.weight");
    } else {
      put_mat(L.qkv, {&s.q, &s.k, &s.v}, W_, false);
    }
    put_mat(L.o, {&s.o}, attn_, false);
    // rows interleaved gate / up (gate f at 2f, up f at 2f + 1) for the SwiGLU epilogue
    std::vector<float> gu(static_cast<std::size_t>(2) * mlp * W);
    for (std::size_t f = 0; f < mlp; ++f) {
      std::memcpy(&gu[(2 * f) * W], &s.g[f * W], W * 4);
      std::memcpy(&gu[(2 * f + 1) * W], &s.u[f * W], W * 4);
    }
    put_mat(L.gu, {&gu}, W_, false);
    put_mat(L.down, {&s.d}, mlp_, false);
    L.in_norm = put_vec(s.in_norm);
    L.post_norm = put_vec(s.post_norm);
  }
  const auto win = widen_f32(*ain), wtin = widen_f32(*tin), wtout = widen_f32(*tout), wout = widen_f32(*aout);
  std::vector<float> wa(W * W), wt(W * W);
  for (std::size_t m = 0; m < W; ++m)
    for (std::size_t j = 0; j < W; ++j) {
      wa[m * W + j] = wtin[m * 2 * W + j];
      wt[m * W + j] = wtin[m * 2 * W + W + j];
    }
  put_mat(in_, {&win}, A_, true, "model.action_in_proj.weight");
  put_mat(tin_, {&wa}, W_, true, "model.action_time_mlp_in.weight");
  put_mat(tout_, {&wtout}, W_, true, "model.action_time_mlp_out.weight");
  put_mat(out_, {&wout}, W_, true, "model.action_out_proj.weight");
  if (!planes_ok) return false;
  wt_ = put_vec(wt);
  b_in_ = put_vec(widen_f32(*bin));
  b_tin_ = put_vec(widen_f32(*btin));
  b_tout_ = put_vec(widen_f32(*btout));
  b_out_ = put_vec(widen_f32(*bout));
  final_norm_ = put_vec(widen_f32(*fnorm));
  // w_i = 2 pi / period_i, period_i = 0.004 * (4 / 0.004)^(i / (half - 1)) (smolvla_action_expert.cc:230-236)
  const std::size_t half = W / 2;
  std::vector<float> om(half);
  for (std::size_t i = 0; i < half; ++i) {
    const float fraction = half > 1 ? static_cast<float>(i) / static_cast<float>(half - 1) : 0.0f;
    const float period = 0.004F * std::pow(4.0F / 0.004F, fraction);
    constexpr float kPi = 3.14159265358979323846F;
    om[i] = 2.0F * kPi / period;
  }
  omega_ = put_vec(om);
  // RoPE denominators exp(ln(1e4) * 2c / hw) (kernels.h:345-352)
  std::vector<float> rd(hw / 2);
  for (std::size_t c = 0; c < hw / 2; ++c) {
    const float exponent = (2.0F * static_cast<float>(c)) / static_cast<float>(hw);
    rd[c] = std::exp(9.210340371976184F * exponent);
  }
  rope_ = put_vec(rd);
  if (wts_.overflowed()) {
    err = "internal error: SmolVLA weight arena too small";
    return false;
  }
  cudaFuncSetAttribute(attention_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  cudaFuncSetAttribute(attention_kernel<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  cudaFuncSetAttribute(attention_rows_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  cudaFuncSetAttribute(attention_rows_kernel<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  if (cudaDeviceSynchronize() != cudaSuccess) {
    err = "SmolVLA weight upload failed";
    return false;
  }
  return true;
}

int SmolVLA::reserve(std::size_t batch, std::size_t chunk, std::size_t prefix, bool shared_prefix,
                     std::string& err) noexcept {
  batch = std::max<std::size_t>(batch, 1);
  chunk = std::max<std::size_t>(chunk, 1);
  prefix = std::max<std::size_t>(prefix, 1);
  const std::size_t psamples = shared_prefix ? 1 : batch;
  const std::size_t rows = batch * chunk;
  if (rows <= cap_rows_ && chunk <= cap_chunk_ && prefix <= cap_prefix_ && psamples <= cap_psamples_ &&
      batch <= cap_batch_)
    return 0;
  for (auto& [k, g] : graphs_) cudaGraphExecDestroy(g.first);
  graphs_.clear();
  const std::size_t R = std::max(rows, cap_rows_);
  const std::size_t Bc = std::max(batch, cap_batch_);
  const std::size_t Cc = std::max(chunk, cap_chunk_);
  const std::size_t Pc = std::max(prefix, cap_prefix_);
  const std::size_t Sc = std::max(psamples, cap_psamples_);
  const std::size_t ra = (R + 255) / 256 * 256;  // TMA sources hold >= one 256-row tile
  const std::size_t prow = (Sc * Pc + 255) / 256 * 256;
  const std::size_t Wp = static_cast<std::size_t>(Wp_), L = cfg_.layers;
  ArenaPlan plan;
  plan.add_n<float>(ra * A_);                        // x
  plan.add_n<float>(ra * Wp);                        // h
  plan.add_n<bf16>(ra * Wp);                         // proj
  plan.add_n<float>(ra * Ap_);                       // v
  plan.add_n<float>(Wp + 4);                         // temb, t
  plan.add_n<float>(2 * Sc * L * Pc * Cw_);          // caches
  plan.add_n<float>(std::max(ra * Wp, ra * static_cast<std::size_t>(Ap_)));  // host I/O staging
  plan.add_n<__half>(ra * 2 * Ap_);                  // x2
  plan.add_n<__half>(ra * 2 * Wp);                   // a2
  plan.add_n<__half>(ra * 2 * Wp);                   // h12
  plan.add_n<__half>(ra * 2 * Wp);                   // fin2
  plan.add_n<__half>(prow * 2 * Cp_);                // c2
  plan.add_n<bf16>(ra * Wp);                         // nb
  plan.add_n<bf16>(ra * qkv_ld_);                    // qkv
  plan.add_n<bf16>(ra * attn_p_);                    // att
  plan.add_n<bf16>(ra * mlp_p_);                     // act
  plan.add_n<bf16>(L * prow * kvp_ld_);              // kvp
  plan.add_n<float2>((Pc + Cc) * cfg_.head_width / 2);
  plan.add_n<float>(small_part_floats());
  plan.add_n<std::uint8_t>(Sc * Pc);
  plan.add_n<int>(Sc + 4);
  ws_.release();
  if (!ws_.init(plan.total(), err)) {
    cap_rows_ = 0;
    return 2;
  }
  x_ = ws_.take_n<float>(ra * A_);
  h_ = ws_.take_n<float>(ra * Wp);
  proj_ = ws_.take_n<bf16>(ra * Wp);
  v_ = ws_.take_n<float>(ra * Ap_);
  temb_ = ws_.take_n<float>(Wp + 4);
  tval_ = temb_ + Wp;
  kcache_ = ws_.take_n<float>(Sc * L * Pc * Cw_);
  vcache_ = ws_.take_n<float>(Sc * L * Pc * Cw_);
  io_ = ws_.take_n<float>(std::max(ra * Wp, ra * static_cast<std::size_t>(Ap_)));
  x2_ = ws_.take_n<__half>(ra * 2 * Ap_);
  a2_ = ws_.take_n<__half>(ra * 2 * Wp);
  h12_ = ws_.take_n<__half>(ra * 2 * Wp);
  fin2_ = ws_.take_n<__half>(ra * 2 * Wp);
  c2_ = ws_.take_n<__half>(prow * 2 * Cp_);
  nb_ = ws_.take_n<bf16>(ra * Wp);
  qkv_ = ws_.take_n<bf16>(ra * qkv_ld_);
  att_ = ws_.take_n<bf16>(ra * attn_p_);
  act_ = ws_.take_n<bf16>(ra * mlp_p_);
  kvp_ = ws_.take_n<bf16>(L * prow * kvp_ld_);
  rope_tab_ = ws_.take_n<float2>((Pc + Cc) * cfg_.head_width / 2);
  small_part_ = ws_.take_n<float>(small_part_floats());
  mask_ = ws_.take_n<std::uint8_t>(Sc * Pc);
  valid_ = ws_.take_n<int>(Sc + 4);
  step_ = valid_ + Sc;
  if (ws_.overflowed()) {
    err = "internal error: SmolVLA workspace arena too small";
    cap_rows_ = 0;
    return 2;
  }
  // padding columns of every GEMM operand must read as zero
  cudaMemset(x_, 0, ws_.used());
  rows_alloc_ = static_cast<long long>(ra);
  prow_alloc_ = static_cast<long long>(prow);
  cap_rows_ = R;
  cap_batch_ = Bc;
  cap_chunk_ = Cc;
  cap_prefix_ = Pc;
  cap_psamples_ = Sc;
  return cudaDeviceSynchronize() == cudaSuccess ? 0 : 2;
}

bool SmolVLA::gemm(const Mat& m, const void* src, long long rows, void* out, int out_ld, bool out_f32,
                   long long lo_off, const float* bias, const float* add_vec, int act, cudaStream_t st,
                   std::string& err, long long src_rows, int out_ch_off, bool out_bf16) {
  if (src_rows == 0) src_rows = rows_alloc_;
  if (rows <= kSmallRows) {
    // split-K mma.sync tiles + a fixed-order reduction with the same epilogue
    SmallGemm g{};
    g.w = m.w;
    g.ld_w = m.split ? 2 * m.kp : m.kp;
    g.M = m.rows;
    g.kp = m.kp;
    g.split = m.split ? 1 : 0;
    g.x = src;
    g.ld_x = m.split ? 2 * m.kp : m.kp;
    g.rows = static_cast<int>(rows);
    g.partial = small_part_;
    g.m_pad = pad(m.rows, 16);
    const int nks = (m.kp + kSmallK - 1) / kSmallK;
    const dim3 grid(static_cast<unsigned>(g.m_pad / 16), static_cast<unsigned>(nks));
    if (m.split) launch_pdl(small_gemm_kernel<true>, grid, dim3(128), 0, st, g);
    else launch_pdl(small_gemm_kernel<false>, grid, dim3(128), 0, st, g);
    SmallEpilogue e{};
    e.partial = small_part_;
    e.nks = nks;
    e.rows = g.rows;
    e.m_valid = m.rows;
    e.m_pad = g.m_pad;
    e.bias = bias;
    e.add_vec = add_vec;
    e.act = act;
    e.out_kind = out_f32 ? 0 : (!m.split || out_bf16) ? 1 : (lo_off != 0 ? 3 : 2);
    e.out = out;
    e.out_ld = out_ld;
    e.lo_off = lo_off;
    e.ch_off = out_ch_off;
    const long long cols = act == tc::kActSwiGLU ? m.rows / 2 : m.rows;
    launch_pdl(small_epilogue_kernel, dim3(ew_grid(rows * cols, 256, *ctx_)), dim3(256), 0, st, e);
    launches_ += 2;
    return cudaGetLastError() == cudaSuccess;
  }
  TcLaunch l;
  l.fp16 = m.split;
  l.A = m.w;
  l.M_rows = m.rows_pad;
  l.m_valid = m.rows;
  l.L = 1;
  l.n_samples = static_cast<int>(rows);
  const int kb = m.kp / 64;
  if (m.split) {
    l.K = 2 * m.kp;
    l.src[0] = TcSource{src, 2 * m.kp, 1, static_cast<int>(src_rows)};
    l.segs = {tc::Seg{0, 0, 0, kb, 0}, tc::Seg{0, 0, m.kp, kb, m.kp}};
  } else {
    l.K = m.kp;
    l.src[0] = TcSource{src, m.kp, 1, static_cast<int>(src_rows)};
    l.segs = {tc::Seg{0, 0, 0, kb, 0}};
  }
  l.bias = bias;
  l.add_vec = add_vec;
  l.act = act;
  l.out_f32 = out_f32;
  l.out = out;
  l.out_ld = out_ld;
  l.out_lo_off = lo_off;
  l.out_ch_off = out_ch_off;
  l.out_bf16 = out_bf16;
  ++launches_;
  return tc_gemm(l, *ctx_, st, err) == cudaSuccess;
}

int SmolVLA::check_prefix(const std::uint8_t* mask, std::size_t prefix, std::size_t chunk, std::string& err) const {
  if (chunk == 0 || chunk > static_cast<std::size_t>(kMaxChunk) || prefix == 0 ||
      prefix > static_cast<std::size_t>(kMaxPrefix)) {
    err = "SmolVLA expert chunk or prefix length is outside the fixed execution limit";
    return 1;
  }
  const int S = static_cast<int>(ref_layout_ ? prefix + chunk : std::max(prefix, chunk));
  if (std::max(attn_smem(pad(S, 16), 3), attn_rows_smem(pad(S, 16), 3)) > 227 * 1024) {
    err = "SmolVLA prefix + chunk exceeds this build's attention tile (shared memory)";
    return 1;
  }
  if (mask != nullptr) {
    std::size_t valid = 0;
    for (std::size_t i = 0; i < prefix; ++i) {
      if (mask[i] > 1) {
        err = "SmolVLA cached-VLM action expert could not be executed";
        return 3;
      }
      valid += mask[i];
    }
    if (valid == 0) {
      err = "SmolVLA cached-VLM action expert could not be executed";
      return 3;
    }
  }
  return 0;
}

bool SmolVLA::prepare_prefix(const float* keys, const float* values, const std::uint8_t* mask, std::size_t samples,
                             std::size_t prefix, bool device_ptrs, cudaStream_t st, std::string& err) {
  const std::size_t L = cfg_.layers;
  const std::size_t per = L * prefix * static_cast<std::size_t>(Cw_);
  const cudaMemcpyKind kind = device_ptrs ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  cudaMemcpyAsync(kcache_, keys, samples * per * 4, kind, st);
  cudaMemcpyAsync(vcache_, values, samples * per * 4, kind, st);
  cudaMemcpyAsync(mask_, mask, samples * prefix, kind, st);
  count_valid_kernel<<<static_cast<unsigned>(samples), 256, 0, st>>>(mask_, static_cast<int>(prefix), valid_);
  ++launches_;
  // RoPE angles of every position a call can reach (valid prefix slots + action tokens)
  {
    const int half = static_cast<int>(cfg_.head_width / 2);
    const int npos = static_cast<int>(prefix + cap_chunk_);
    rope_table_kernel<<<ew_grid(static_cast<long long>(npos) * half, 256, *ctx_), 256, 0, st>>>(rope_, half, npos,
                                                                                                rope_tab_);
    ++launches_;
  }
  prefix_ = prefix;
  const long long prow = static_cast<long long>(samples * prefix);
  for (std::size_t l = 0; l < L; ++l) {
    const Layer& Ly = layers_[l];
    if (!Ly.cross) continue;
    // K = bf16(keys W_k^T) at columns [0, kv), V = bf16(values W_v^T) at [kv, 2 kv)
    // of this layer's prefix rows (smolvla_action_expert.cc:311-323)
    bf16* dst = kvp_ + l * static_cast<std::size_t>(prow_alloc_) * kvp_ld_;
    for (int sel = 0; sel < 2; ++sel) {
      const float* cache = (sel == 0 ? kcache_ : vcache_) + l * prefix * static_cast<std::size_t>(Cw_);
      split_rows_kernel<<<ew_grid(prow * Cp_, 256, *ctx_), 256, 0, st>>>(
          cache, prow, Cw_, Cw_, static_cast<long long>(prefix), static_cast<long long>(per), c2_, Cp_);
      ++launches_;
      if (!gemm(sel == 0 ? Ly.k : Ly.v, c2_, prow, dst, kvp_ld_, false, 0, nullptr, nullptr, tc::kActNone, st, err,
                prow_alloc_, sel == 0 ? 0 : kvw_, true))
        return false;
    }
  }
  return cudaGetLastError() == cudaSuccess;
}

bool SmolVLA::record_embed(long long rows, const float* t_direct, int steps, cudaStream_t st, std::string& err) {
  const int half = W_ / 2;
  time_embed_kernel<<<(W_ + 7) / 8, 256, static_cast<std::size_t>(W_) * 4, st>>>(
      step_, steps, t_direct, omega_, half, wt_, b_tin_, W_, temb_);
  ++launches_;
  // a = W_in x + b_in (fp32 activations: hi / lo split), h1 = SiLU(W_a a + temb), h = W_out h1 + b
  if (!gemm(in_, x2_, rows, a2_, 2 * Wp_, false, Wp_, b_in_, nullptr, tc::kActNone, st, err)) return false;
  if (!gemm(tin_, a2_, rows, h12_, 2 * Wp_, false, Wp_, nullptr, temb_, tc::kActSilu, st, err)) return false;
  return gemm(tout_, h12_, rows, h_, Wp_, true, 0, b_tout_, nullptr, tc::kActNone, st, err);
}

bool SmolVLA::attention(const Layer& Ly, std::size_t li, std::size_t batch, std::size_t chunk, bool shared,
                        cudaStream_t st, std::string& err) {
  AttnParams p{};
  const int P = static_cast<int>(prefix_);
  p.qkv = qkv_;
  p.qkv_ld = qkv_ld_;
  p.k_off = attn_;
  p.v_off = attn_ + kvw_;
  p.kvp = kvp_ + li * static_cast<std::size_t>(prow_alloc_) * kvp_ld_;
  p.kvp_ld = kvp_ld_;
  p.kv_w = kvw_;
  p.kvp_b = shared ? 0 : P;
  p.pk = kcache_;
  p.pv = vcache_;
  p.p_ld = Cw_;
  p.p_b = shared ? 0 : static_cast<long long>(cfg_.layers) * P;
  p.layer_off = static_cast<long long>(li) * P * Cw_;
  p.mask = mask_;
  p.mask_b = shared ? 0 : P;
  p.valid = valid_;
  p.valid_b = shared ? 0 : 1;
  p.rope = rope_tab_;
  p.chunk = static_cast<int>(chunk);
  p.chunk_pad = pad(p.chunk, 16);
  p.P = P;
  p.heads = static_cast<int>(cfg_.heads);
  p.kv_heads = static_cast<int>(cfg_.kv_heads);
  p.hw = static_cast<int>(cfg_.head_width);
  p.cross = Ly.cross ? 1 : 0;
  p.npre = Ly.cross ? P : (ref_layout_ ? P : 0);
  p.S = Ly.cross ? P : p.npre + p.chunk;
  p.S_pad = pad(p.S, 16);
  p.sqrt_hw = std::sqrt(static_cast<float>(cfg_.head_width));
  p.out = att_;
  p.out_ld = attn_p_;
  const int G = attn_g(batch);
  if (static_cast<long long>(batch) * p.kv_heads >= 2LL * ctx_->sm_count) {
    // enough (sample, head) CTAs to fill the GPU: warps own whole tasks
    const dim3 grid(static_cast<unsigned>(batch), static_cast<unsigned>(cfg_.kv_heads));
    const std::size_t rsmem = attn_rows_smem(p.S_pad, G);
    if (G == 3) launch_pdl(attention_rows_kernel<3>, grid, dim3(kAttnThreads), rsmem, st, p);
    else launch_pdl(attention_rows_kernel<1>, grid, dim3(kAttnThreads), rsmem, st, p);
    ++launches_;
    if (cudaGetLastError() != cudaSuccess) {
      err = "SmolVLA attention launch failed";
      return false;
    }
    return true;
  }
  const std::size_t smem = attn_smem(p.S_pad, G);
  // tasks of a K / V head: (G query heads of its group, 16 query rows), all
  // four warps on each; one CTA per task while the (sample, head) CTAs alone
  // leave SMs idle, else every task of the head in one CTA (K / V staged once)
  const int tasks = (p.heads / p.kv_heads / G) * (p.chunk_pad / 16);
  const int slices = static_cast<long long>(batch) * p.kv_heads < 2LL * ctx_->sm_count ? tasks : 1;
  const dim3 grid(static_cast<unsigned>(batch), static_cast<unsigned>(cfg_.kv_heads), static_cast<unsigned>(slices));
  if (G == 3) launch_pdl(attention_kernel<3>, grid, dim3(kAttnThreads), smem, st, p);
  else launch_pdl(attention_kernel<1>, grid, dim3(kAttnThreads), smem, st, p);
  ++launches_;
  if (cudaGetLastError() != cudaSuccess) {
    err = "SmolVLA attention launch failed";
    return false;
  }
  return true;
}

bool SmolVLA::record_layers(std::size_t batch, std::size_t chunk, bool shared, int final_mode, cudaStream_t st,
                            std::string& err) {
  const long long rows = static_cast<long long>(batch * chunk);
  const unsigned rgrid = static_cast<unsigned>((rows + 7) / 8);
  const bf16* pending = nullptr;  // residual projection not yet added to h
  for (std::size_t li = 0; li < layers_.size(); ++li) {
    const Layer& L = layers_[li];
    launch_pdl(rms_kernel, dim3(rgrid), dim3(256), 0, st, h_, Wp_, pending, Wp_, L.in_norm, W_, rows, 0, nb_, Wp_);
    ++launches_;
    if (!gemm(L.qkv, nb_, rows, qkv_, qkv_ld_, false, 0, nullptr, nullptr, tc::kActNone, st, err)) return false;
    if (!attention(L, li, batch, chunk, shared, st, err)) return false;
    if (!gemm(L.o, att_, rows, proj_, Wp_, false, 0, nullptr, nullptr, tc::kActNone, st, err)) return false;
    launch_pdl(rms_kernel, dim3(rgrid), dim3(256), 0, st, h_, Wp_, proj_, Wp_, L.post_norm, W_, rows, 0, nb_, Wp_);
    ++launches_;
    // act = bf16(bf16(up) * SiLU(bf16(gate))) straight from the GEMM epilogue
    // (gate_silu, kernels_scalar.cc:61-67, smolvla_action_expert.cc:366-372)
    if (!gemm(L.gu, nb_, rows, act_, mlp_p_, false, 0, nullptr, nullptr, tc::kActSwiGLU, st, err)) return false;
    if (!gemm(L.down, act_, rows, proj_, Wp_, false, 0, nullptr, nullptr, tc::kActNone, st, err)) return false;
    pending = proj_;
  }
  if (final_mode == 1)
    launch_pdl(rms_kernel, dim3(rgrid), dim3(256), 0, st, h_, Wp_, pending, Wp_, final_norm_, W_, rows, 1, fin2_, Wp_);
  else
    launch_pdl(rms_kernel, dim3(rgrid), dim3(256), 0, st, h_, Wp_, pending, Wp_, final_norm_, W_, rows, 2, io_, W_);
  ++launches_;
  return cudaGetLastError() == cudaSuccess;
}

bool SmolVLA::record_step(std::size_t batch, std::size_t chunk, std::size_t steps, bool shared, cudaStream_t st,
                          std::string& err) {
  const long long rows = static_cast<long long>(batch * chunk);
  if (!record_embed(rows, nullptr, static_cast<int>(steps), st, err)) return false;
  if (!record_layers(batch, chunk, shared, 1, st, err)) return false;
  if (!gemm(out_, fin2_, rows, v_, Ap_, true, 0, b_out_, nullptr, tc::kActNone, st, err)) return false;
  launch_pdl(euler_kernel, dim3(ew_grid(rows * A_, 256, *ctx_)), dim3(256), 0, st, v_, Ap_, x_, A_, rows,
             static_cast<int>(steps), x2_, Ap_, step_, step_ + 1);
  ++launches_;
  // step_[0] <- step_[1] for the next replay
  cudaMemcpyAsync(step_, step_ + 1, sizeof(int), cudaMemcpyDeviceToDevice, st);
  return cudaGetLastError() == cudaSuccess;
}

int SmolVLA::finish(cudaStream_t st, std::string& err) {
  if (cudaStreamSynchronize(st) != cudaSuccess) {
    err = std::string("SmolVLA expert failed: ") + cudaGetErrorString(cudaGetLastError());
    return 2;
  }
  if (const int code = take_device_error(*ctx_, st); code != 0) {
    err = device_error_text(code);
    return 2;
  }
  return 0;
}

int SmolVLA::embed_suffix(const float* noisy, std::size_t chunk, float timestep, float* out, std::string& err) noexcept {
  if (chunk == 0 || chunk > static_cast<std::size_t>(kMaxChunk)) {
    err = "SmolVLA chunk size is outside the fixed projection limit";
    return 1;
  }
  if (reserve(1, chunk, 1, true, err) != 0) return 2;
  cudaSetDevice(ctx_->device);
  cudaStream_t st = ctx_->stream;
  const long long rows = static_cast<long long>(chunk);
  cudaMemcpyAsync(io_, noisy, chunk * A_ * 4, cudaMemcpyHostToDevice, st);
  split_rows_kernel<<<ew_grid(rows * Ap_, 256, *ctx_), 256, 0, st>>>(io_, rows, A_, A_, rows, 0, x2_, Ap_);
  cudaMemcpyAsync(tval_, &timestep, 4, cudaMemcpyHostToDevice, st);
  if (!record_embed(rows, tval_, 1, st, err)) return 2;
  gather_rows_kernel<<<ew_grid(rows * W_, 256, *ctx_), 256, 0, st>>>(h_, Wp_, rows, W_, io_);
  cudaMemcpyAsync(out, io_, chunk * W_ * 4, cudaMemcpyDeviceToHost, st);
  return finish(st, err);
}

int SmolVLA::run_expert(const float* suffix, std::size_t chunk, const float* keys, const float* values,
                        const std::uint8_t* mask, std::size_t prefix, float* out, std::string& err) noexcept {
  if (const int rc = check_prefix(mask, prefix, chunk, err); rc != 0) return rc;
  if (reserve(1, chunk, prefix, true, err) != 0) return 2;
  cudaSetDevice(ctx_->device);
  cudaStream_t st = ctx_->stream;
  const long long rows = static_cast<long long>(chunk);
  if (!prepare_prefix(keys, values, mask, 1, prefix, false, st, err)) return 2;
  cudaMemcpyAsync(io_, suffix, chunk * W_ * 4, cudaMemcpyHostToDevice, st);
  scatter_rows_kernel<<<ew_grid(rows * W_, 256, *ctx_), 256, 0, st>>>(io_, rows, W_, h_, Wp_);
  if (!record_layers(1, chunk, true, 2, st, err)) return 2;
  cudaMemcpyAsync(out, io_, chunk * W_ * 4, cudaMemcpyDeviceToHost, st);
  return finish(st, err);
}

int SmolVLA::project_actions(const float* hidden, std::size_t chunk, float* out, std::string& err) noexcept {
  if (chunk == 0 || chunk > static_cast<std::size_t>(kMaxChunk)) {
    err = "SmolVLA action chunk size is outside the fixed projection limit";
    return 1;
  }
  if (reserve(1, chunk, 1, true, err) != 0) return 2;
  cudaSetDevice(ctx_->device);
  cudaStream_t st = ctx_->stream;
  const long long rows = static_cast<long long>(chunk);
  cudaMemcpyAsync(io_, hidden, chunk * W_ * 4, cudaMemcpyHostToDevice, st);
  split_rows_kernel<<<ew_grid(rows * Wp_, 256, *ctx_), 256, 0, st>>>(io_, rows, W_, W_, rows, 0, fin2_, Wp_);
  if (!gemm(out_, fin2_, rows, v_, Ap_, true, 0, b_out_, nullptr, tc::kActNone, st, err)) return 2;
  gather_rows_kernel<<<ew_grid(rows * A_, 256, *ctx_), 256, 0, st>>>(v_, Ap_, rows, A_, io_);
  cudaMemcpyAsync(out, io_, chunk * A_ * 4, cudaMemcpyDeviceToHost, st);
  return finish(st, err);
}

int SmolVLA::denoise(const float* noisy, std::size_t chunk, float timestep, const float* keys, const float* values,
                     const std::uint8_t* mask, std::size_t prefix, float* out, std::string& err) noexcept {
  if (const int rc = check_prefix(mask, prefix, chunk, err); rc != 0) return rc;
  if (reserve(1, chunk, prefix, true, err) != 0) return 2;
  cudaSetDevice(ctx_->device);
  cudaStream_t st = ctx_->stream;
  const long long rows = static_cast<long long>(chunk);
  if (!prepare_prefix(keys, values, mask, 1, prefix, false, st, err)) return 2;
  cudaMemcpyAsync(io_, noisy, chunk * A_ * 4, cudaMemcpyHostToDevice, st);
  split_rows_kernel<<<ew_grid(rows * Ap_, 256, *ctx_), 256, 0, st>>>(io_, rows, A_, A_, rows, 0, x2_, Ap_);
  cudaMemcpyAsync(tval_, &timestep, 4, cudaMemcpyHostToDevice, st);
  if (!record_embed(rows, tval_, 1, st, err)) return 2;
  if (!record_layers(1, chunk, true, 1, st, err)) return 2;
  if (!gemm(out_, fin2_, rows, v_, Ap_, true, 0, b_out_, nullptr, tc::kActNone, st, err)) return 2;
  gather_rows_kernel<<<ew_grid(rows * A_, 256, *ctx_), 256, 0, st>>>(v_, Ap_, rows, A_, io_);
  cudaMemcpyAsync(out, io_, chunk * A_ * 4, cudaMemcpyDeviceToHost, st);
  return finish(st, err);
}

int SmolVLA::sample(const float* noise, std::size_t batch, std::size_t chunk, std::size_t steps, const float* keys,
                    const float* values, const std::uint8_t* mask, std::size_t prefix, bool shared_prefix,
                    float* out, bool on_device, void* stream, std::string& err) noexcept {
  if (batch == 0 || steps == 0 || steps > kMaxSteps) {
    err = "SmolVLA Euler sample dimensions or step count are outside the fixed execution limit";
    return 1;
  }
  if (const int rc = check_prefix(nullptr, prefix, chunk, err); rc != 0) return rc;
  if (!on_device) {
    const std::size_t ms = shared_prefix ? 1 : batch;
    for (std::size_t s = 0; s < ms; ++s)
      if (const int rc = check_prefix(mask + s * prefix, prefix, chunk, err); rc != 0) return rc;
  }
  if (reserve(batch, chunk, prefix, shared_prefix, err) != 0) return 2;
  cudaSetDevice(ctx_->device);
  cudaStream_t st = stream != nullptr ? static_cast<cudaStream_t>(stream) : ctx_->stream;
  const long long rows = static_cast<long long>(batch * chunk);
  const std::size_t samples = shared_prefix ? 1 : batch;
  if (!prepare_prefix(keys, values, mask, samples, prefix, on_device, st, err)) return 2;
  // x = noise (dense [rows][A]); its hi / lo split feeds the first step
  cudaMemcpyAsync(x_, noise, static_cast<std::size_t>(rows) * A_ * 4,
                  on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, st);
  split_rows_kernel<<<ew_grid(rows * Ap_, 256, *ctx_), 256, 0, st>>>(x_, rows, A_, A_, rows, 0, x2_, Ap_);
  ++launches_;
  cudaMemsetAsync(step_, 0, 2 * sizeof(int), st);
  const auto key = std::make_tuple(batch, chunk, steps, prefix, shared_prefix);
  auto it = graphs_.find(key);
  if (it == graphs_.end()) {
    cudaStream_t cap = nullptr;
    cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking);
    cudaStreamSynchronize(st);
    cudaGraph_t graph = nullptr;
    const std::uint64_t before = launches_;
    cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal);
    const bool ok = record_step(batch, chunk, steps, shared_prefix, cap, err);
    const cudaError_t end = cudaStreamEndCapture(cap, &graph);
    cudaStreamDestroy(cap);
    const std::uint64_t per_step = launches_ - before;
    launches_ = before;
    if (!ok || end != cudaSuccess || graph == nullptr) {
      if (graph != nullptr) cudaGraphDestroy(graph);
      if (err.empty()) err = "SmolVLA graph capture failed";
      cudaGetLastError();
      return 2;
    }
    cudaGraphExec_t exec = nullptr;
    const cudaError_t inst = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (inst != cudaSuccess) {
      err = "SmolVLA graph instantiation failed";
      return 2;
    }
    it = graphs_.emplace(key, std::make_pair(exec, per_step)).first;
  }
  for (std::size_t i = 0; i < steps; ++i)
    if (cudaGraphLaunch(it->second.first, st) != cudaSuccess) {
      err = "SmolVLA graph launch failed";
      return 2;
    }
  launches_ += it->second.second * steps;
  if (on_device) {
    cudaMemcpyAsync(out, x_, static_cast<std::size_t>(rows) * A_ * 4, cudaMemcpyDeviceToDevice, st);
    return cudaGetLastError() == cudaSuccess ? 0 : 2;
  }
  cudaMemcpyAsync(out, x_, static_cast<std::size_t>(rows) * A_ * 4, cudaMemcpyDeviceToHost, st);
  return finish(st, err);
}

}  // namespace

std::unique_ptr<SmolVLADevice> make_smolvla_device(const TensorTable& tensors, std::shared_ptr<DeviceContext> ctx,
                                                   std::string& err) {
  cudaSetDevice(ctx->device);
  auto m = std::make_unique<SmolVLA>(std::move(ctx));
  if (!m->load(tensors, err)) return nullptr;
  return m;
}

}  // namespace feb
