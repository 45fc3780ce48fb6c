/*
 * Test hooks of libflowedge_b200.so: single kernels on host buffers, used by
 * the numerics tests to compare one device kernel with a PyTorch fp32
 * reference of the same op.  No counterpart in the reference ABI; not part of
 * the drop-in surface.  Each call allocates and frees its own device buffers.
 */
#ifndef FLOWEDGE_B200_TESTING_H
#define FLOWEDGE_B200_TESTING_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* C[N][M] = A[M][K] . B[N][K]^T with 16-bit operands (raw bits; fp16 when
 * `fp16` != 0, else bf16) and fp32 output, on the tcgen05 GEMM.  M, K any
 * positive size (padded internally). */
int febtest_gemm_16(const uint16_t* A, int M, int K, const uint16_t* B, int N, float* C, int fp16);

/* y[b][t][o] = bias[o] + sum_{c,j} W[o][c][j] * x[b][t + j - k/2][c] (zero
 * padded), 16-bit x / W (fp16 when `fp16` != 0, else bf16), y rounded to the
 * same 16-bit format and returned as fp32, on the tcgen05 implicit-GEMM
 * convolution.
 * Also returns the per-(sample, group) GroupNorm sums the epilogue gathers
 * in stats[b][g][2] (sum, sum of squares of the fp32 outputs before their
 * bf16 rounding), groups = OC / group_ch (group_ch = 0: no statistics). */
int febtest_conv_16(const uint16_t* x, int B, int L, int C, const uint16_t* W, const float* bias, int OC, int k,
                    int group_ch, float* y, double* stats, int fp16);

/* The load-time range check applied to every weight tensor that the device
 * holds in fp16 (bf16 mode when `bf16_mode` != 0, else the fp32 hi / lo
 * split).  Returns 0 when `w` can be stored, else 1 with the loader's message
 * (naming `name`) in `message` (NUL-terminated, truncated to `message_len`).
 * Host only: needs no GPU. */
int febtest_check_fp16_storable(const char* name, const float* w, size_t n, int bf16_mode, char* message,
                                size_t message_len);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* FLOWEDGE_B200_TESTING_H */
