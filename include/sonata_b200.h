/*
 * sonata_b200 -- C ABI of the B200 (sm_100a) hot-path kernels.
 *
 * Every entry point takes plain device pointers, integer shapes / strides and
 * a cudaStream_t passed as void*.  None of them allocates, synchronises or
 * aborts: they validate their arguments on the host, enqueue work on the given
 * stream and return SN_OK or a negative SN_ERR_* code.  They are therefore
 * safe to call while a CUDA graph is being captured on that stream.  The
 * caller owns every buffer.  Strides are in elements.
 *
 * Reference interfaces replaced (paths are inside Vishal-Padia/Sonata):
 *   kernels/gemv.py   skinny_gemv{,_coalesced,_splitk_m1,_splitk_m2} launchers
 *                     (gemv.py:38-54, 169-193) and _run (gemv.py:199-212)
 *   scripts/fake_quant.py fake_quantize_weights (fake_quant.py:16-42)
 *   kernels/bmm.py    launch_bmm (bmm.py:96-117)
 *   kernels/fused_snake_conv.py _launch_fused_snake_conv1d (:89-131) via
 *                     fused_snake_conv1d (:134-199)
 */
#ifndef SONATA_B200_H_
#define SONATA_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---- */
#define SN_OK 0
#define SN_ERR_INVALID_ARGUMENT (-1) /* null pointer, non-positive or inconsistent shape */
#define SN_ERR_MISALIGNED (-2)       /* pointer / stride alignment a kernel requires */
#define SN_ERR_UNSUPPORTED (-3)      /* shape outside what the kernels implement */
#define SN_ERR_LAUNCH (-4)           /* the CUDA launch itself failed */
#define SN_ERR_DEVICE (-5)           /* current device is not sm_100 */
#define SN_ERR_TIMEOUT (-6)          /* a bounded device-side wait ran out */

/* ---- dtype codes for outputs ---- */
#define SN_DTYPE_BF16 0
#define SN_DTYPE_F32 1

/* ---- flags ---- */
/* Programmatic dependent launch: the kernel may start while the previous
 * kernel on the stream is still running and begins streaming its weights
 * before waiting for it.  Only valid when the previous kernel does not write
 * the weight (or scale) buffer -- e.g. frozen nn.Linear weights. */
#define SN_FLAG_PDL 1u

/* Library version (major * 10000 + minor * 100 + patch). */
int sn_version(void);
/* Static description of a status code. */
const char *sn_status_string(int status);

/*
 * bf16 skinny GEMV: y[m, n] = sum_k x[m, k] * W[n, k], fp32 accumulation.
 * W: bf16 [N, K] row stride ldw (nn.Linear weight layout); x: bf16 [M, K]
 * row stride ldx; y: [M, N] row stride ldy, bf16 (rounded to nearest even)
 * or fp32 per y_dtype.  1 <= M <= 4.
 * Replaces kernels/gemv.py:179-193 (skinny_gemv_splitk_m1 / _m2) and every
 * other launcher of that file (gemv.py:38-54, 169-175), same contract.
 */
int sn_gemv_bf16(const void *W, int64_t ldw, const void *x, int64_t ldx, void *y, int64_t ldy,
                 int M, int N, int K, int y_dtype, unsigned flags, void *stream);

/*
 * Weight-only int8 GEMV with the dequantisation fused:
 *   y[m, n] = scale[n] * sum_k x[m, k] * q[n, k]
 * q: int8 [N, K] row stride ldq; scale: fp32 [N] (per output channel).
 * Equals "dequantise to fp32 then matmul" of scripts/fake_quant.py:16-42
 * (bits=8, group_size=None) up to fp32 summation order.
 */
int sn_gemv_int8(const int8_t *q, int64_t ldq, const float *scale, const void *x, int64_t ldx,
                 void *y, int64_t ldy, int M, int N, int K, int y_dtype, unsigned flags,
                 void *stream);

/* Same with float8 e4m3 (fn) codes: y[m, n] = scale[n] * sum_k x[m, k] * e4m3(q[n, k]). */
int sn_gemv_fp8e4m3(const uint8_t *q, int64_t ldq, const float *scale, const void *x, int64_t ldx,
                    void *y, int64_t ldy, int M, int N, int K, int y_dtype, unsigned flags,
                    void *stream);

/*
 * Per-output-channel weight quantisation on the device (bit-identical to
 * scripts/fake_quant.py:37-40 for int8):
 *   scale[n] = max(max_k |W[n, k]|, 1e-8) / 127   (int8)   or / 448 (e4m3)
 *   q[n, k]  = round_half_even(W[n, k] / scale[n])       (int8, clamped to +-127)
 *            = e4m3_rn(W[n, k] / scale[n])                (e4m3)
 * W: bf16 [N, K] row stride ldw; q: [N, K] row stride ldq.
 */
int sn_quantize_rows_int8(const void *W, int64_t ldw, int N, int K, int8_t *q, int64_t ldq,
                          float *scale, void *stream);
int sn_quantize_rows_fp8e4m3(const void *W, int64_t ldw, int N, int K, uint8_t *q, int64_t ldq,
                             float *scale, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* SONATA_B200_H_ */
