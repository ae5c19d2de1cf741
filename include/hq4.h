/* hq4 -- B200 (sm_100a) int4 GEMV / dequant kernels behind a C ABI.
 *
 * Drop-in device-side replacement for the reference's native kernel,
 * hetero-infer kernel/q4gemv.c, which its NumPy backend binds through ctypes
 * (hetero/cpu_model.py:33-45).  Plain pointers and sizes only: every pointer
 * argument is a CUDA device pointer unless stated otherwise, `stream` is a
 * cudaStream_t passed as void*, and every call is asynchronous on it.
 *
 * Weight layout (identical to the reference, kernel/q4gemv.c:7-11):
 *   w       [n_out][n_in/8]   uint32, eight 4-bit values, low nibble first
 *   scales  [n_out][n_in/gs]  IEEE fp16 bits
 *   biases  [n_out][n_in/gs]  IEEE fp16 bits
 *   value = q * scale + bias
 *
 * Return codes follow the reference convention (0 ok, -1 bad shape) with
 * further negative codes for the device side.
 */
#ifndef HQ4_H
#define HQ4_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HQ4_OK 0
#define HQ4_ERR_SHAPE (-1)     /* n_in % gs, unsupported gs, n_out/n_in/m <= 0 */
#define HQ4_ERR_ALIGN (-2)     /* w not 32-byte aligned, x not 16-byte, out not 4-byte */
#define HQ4_ERR_LAUNCH (-4)    /* a CUDA launch failed (cudaGetLastError) */
#define HQ4_ERR_DEVICE (-5)    /* current device is not sm_100 */

/* Library version, (major << 16) | minor. */
int hq4_version(void);

/* Device status word of the current device (synchronising): bit 0 is set
 * when a kernel's bounded wait on its cluster x-image exchange ran out (the
 * kernel then wrote no output).  Non-zero `clear` resets it.  Has no
 * counterpart in the reference, whose CPU kernel cannot stall this way. */
int hq4_device_status(int clear);

/* out[m][n_out] = x[m][n_in] . W^T with W dequantised on the fly.
 * Replaces  int q4_gemv(w, scales, biases, x, out, n_out, n_in, gs, nthreads)
 * (kernel/q4gemv.c:232-233): same pointer order and shape arguments; the
 * host thread count becomes the token count m and the CUDA stream.
 * x and out are fp32 row-major.  Supported gs: 32, and 64 * 2^k.
 * Needs no workspace; the x row must fit one CTA's shared memory
 * (n_in up to ~64K values).
 * Arithmetic: exact nibble dequantisation, products exact in fp32, per-group
 * fp32 scale and bias as the reference's float path (kernel/q4gemv.c:113-139,
 * 177-181): results match it to fp32 summation-order rounding. */
int hq4_gemv(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
             const float* x, float* out, int n_out, int n_in, int gs, int m, void* stream);

/* hq4_gemv with the projection's epilogue fused into the store:
 *   out[i][r] = (x[i] . W[r]) + row_add[r] + residual[i][r]
 * row_add (length n_out, e.g. the q/k/v bias of hetero/cpu_model.py:156-157)
 * and residual ([m][n_out], the decoder's residual stream,
 * hetero/cpu_model.py:305-306) may each be NULL.  out may alias residual. */
int hq4_gemv_fused(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                   const float* x, float* out, int n_out, int n_in, int gs, int m,
                   const float* row_add, const float* residual, void* stream);

/* Rows [row0,row1) of W expanded to fp32 into out [row1-row0][n_in].
 * Replaces  int q4_dequant(w, scales, biases, out, row0, row1, n_in, gs,
 * nthreads)  (kernel/q4gemv.c:359-360).  Bit-exact with the reference. */
int hq4_dequant(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                float* out, int row0, int row1, int n_in, int gs, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HQ4_H */
