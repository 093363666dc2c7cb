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

#include <stddef.h>
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
#define SN_ERR_SCRATCH_LIMIT (-7)    /* needs more scratch than the allocation-free entry point holds */
#define SN_ERR_SCRATCH_ADDRESS (-8)  /* the allocation-free entry point could not look up its array's address */

/* ---- dtype codes for outputs ---- */
#define SN_DTYPE_BF16 0
#define SN_DTYPE_F32 1

/* ---- flags ---- */
/* Programmatic dependent launch: the kernel may start while the previous
 * kernel on the stream is still running and begins streaming its weights
 * before waiting for it.  Only valid when the previous kernel does not write
 * the weight (or scale) buffer -- e.g. frozen nn.Linear weights. */
#define SN_FLAG_PDL 1u
/* sn_snake_conv1d_ex / sn_snake_conv_transpose1d: the workspace already holds
 * the weights packed by sn_snake_conv1d_pack / sn_snake_conv_transpose1d_pack
 * (same W and shape), so the call does not pack them again. */
#define SN_FLAG_PREPACKED 2u

/* ---- weight kinds of sn_gemv_ex ---- */
#define SN_WEIGHT_BF16 0
#define SN_WEIGHT_INT8 1
#define SN_WEIGHT_E4M3 2

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
 * Any of the three GEMVs above (w_kind SN_WEIGHT_*; scale ignored for bf16)
 * with a prefetch hint for the decode chain: next_W (kind next_kind, [next_N,
 * next_K], row stride next_ldw elements) is the weight of the GEMV that
 * follows on the stream.  When each CTA's own weight reads have landed, it
 * prefetches the first bytes of the matching CTA ranges of that launch into
 * L2 (8 MB in all), so that HBM keeps streaming across the kernel boundary.  The result is identical with or without the hint; next_W == NULL
 * gives the plain call.  A next weight whose rows a bulk prefetch cannot
 * address (not 16-byte aligned) is not prefetched.  Same decode-chain role as
 * the back-to-back GEMV launches of kernels/patch.py:54-66 under a CUDA graph
 * (no counterpart in the reference).
 */
int sn_gemv_ex(int w_kind, const void *W, int64_t ldw, const float *scale, const void *x, int64_t ldx,
               void *y, int64_t ldy, int M, int N, int K, int y_dtype, unsigned flags, void *stream,
               int next_kind, const void *next_W, int64_t next_ldw, int next_N, int next_K);

/*
 * bf16 GEMV with the normalisation before it fused into the x staging (the
 * Zonos decode step's gated RMSNorm -> out_proj and add + LayerNorm ->
 * in_proj / qkv / fc1; no counterpart in the reference, where the norm is a
 * separate kernel).  Every CTA normalises the x rows it stages:
 *   SN_NORM_RMS_GATED: x' = (x * SiLU(aux)) / rms(x * SiLU(aux)) * norm_w
 *                      (aux = z, may be NULL: no gate; the whole row is one
 *                      group), as sn_rmsnorm_gated with norm_before_gate 0;
 *   SN_NORM_ADD_LAYER: h = x + aux (aux = residual or NULL),
 *                      x' = LayerNorm(h) * norm_w (+ norm_b), and
 *                      residual_out (or NULL) = h in bf16, as
 *                      sn_layer_norm_fused with bf16 residuals;
 * then y = x' W^T as sn_gemv_ex (next-weight hint as there).  x, aux,
 * residual_out: contiguous bf16 [M, K], 16-byte aligned; M <= 4, K a
 * multiple of 1024 up to 4096; SN_ERR_UNSUPPORTED for shapes the tensor-core
 * kernel does not take (the caller then runs the two kernels).  The row sums
 * are taken in another order than the standalone norm kernels', so x' may
 * differ from theirs by one bf16 rounding step.
 */
#define SN_NORM_RMS_GATED 1
#define SN_NORM_ADD_LAYER 2
int sn_gemv_bf16_norm(int norm_kind, const void *W, int64_t ldw, const void *x, const void *aux, const void *norm_w,
                      const void *norm_b, void *residual_out, float eps, void *y, int64_t ldy, int M, int N, int K,
                      int y_dtype, unsigned flags, void *stream, int next_kind, const void *next_W,
                      int64_t next_ldw, int next_N, int next_K);

/*
 * GEMV chain: a list of bf16 decode GEMVs y_j = x_j W_j^T (e.g. the per-token
 * projection set of a Zonos-hybrid decode step) run by ONE persistent
 * launch instead of one launch per GEMV.  Every CTA streams the jobs' weight
 * rows in order through one ring, so HBM keeps reading the next job's
 * weights while the current job finishes; only a job's x waits, inside the
 * kernel, for the job named by `dep` (an earlier job, or -1: x is ready when
 * the launch starts).  dep = j - 1 for every job gives the ordering of
 * back-to-back launches on one stream.  bf16 and int8 results are
 * bit-identical to sn_gemv_bf16 / sn_gemv_int8 on the same job (same
 * tensor-core arithmetic and order); e4m3 accumulates each row in one fp32
 * accumulator, so it matches sn_gemv_fp8e4m3 within fp32 summation order.
 * Same role as a CUDA graph of patched nn.Linear calls (kernels/patch.py:54-66,
 * kernels/bench_gemv_graph.py:30-63); no counterpart in the reference.
 *
 * Every job of a chain has the same weight kind w_kind (SN_WEIGHT_*): bf16,
 * or the fused-dequant int8 / e4m3 codes with per-row scales (same
 * arithmetic as sn_gemv_int8 / sn_gemv_fp8e4m3).  Job: W [N, ldw], x bf16
 * [M, ldx], y [M, ldy] in y_dtype; W and x 16-byte aligned, row strides of
 * 16 bytes; K within the tensor-core GEMV's rules (K * element size a
 * multiple of 512).  M (1 or 2) is common to the chain.
 * No job may write a weight or another job's y, nor x of a job that does not
 * wait for it (through its dep, its dep's dep, ...); x and y of a job must
 * not overlap.  Violations: SN_ERR_INVALID_ARGUMENT.
 *
 * sn_gemv_chain_plan validates the jobs on the host, writes the device job
 * table and zeroed completion counters into `workspace` (device memory of
 * sn_gemv_chain_workspace_size(njobs) bytes, 16-byte aligned) and fills
 * *info; it synchronises `stream` (set-up, not for capture).
 * sn_gemv_chain_launch enqueues the chain (capturable; flags 0 or
 * SN_FLAG_PDL).  One launch per workspace at a time: the counters live there.
 */
typedef struct sn_gemv_job {
  const void *W;       /* bf16 [N, ldw], or 8-bit codes [N, ldw] (sn_quantize_rows_*) */
  const void *x;       /* bf16 [M, ldx] */
  void *y;             /* [M, ldy] in y_dtype */
  const float *scale;  /* 8-bit kinds: per-row scales [N]; ignored for bf16 */
  int64_t ldw, ldx, ldy; /* elements */
  int N, K;
  int dep;     /* earlier job whose outputs x waits for, -1: none */
  int y_dtype; /* SN_DTYPE_BF16 or SN_DTYPE_F32 */
} sn_gemv_job;

typedef struct sn_gemv_chain_info { /* filled by sn_gemv_chain_plan */
  int njobs, M;
  int w_kind;                    /* SN_WEIGHT_* of every job */
  int x_buffers;                 /* x staging buffers (x is staged this many jobs ahead) */
  uint32_t tile_bytes_max;       /* largest weight tile (16 / S whole rows) */
  uint32_t ring_bytes, xbuf_bytes; /* shared-memory weight ring, one x buffer */
  uint32_t accumulators;         /* TMEM accumulators */
  uint32_t accumulator_cols;     /* TMEM columns per accumulator */
  uint32_t grid;                 /* CTAs (one per SM of the planning device) */
  uint64_t workspace_bytes;
} sn_gemv_chain_info;

size_t sn_gemv_chain_workspace_size(int njobs);
int sn_gemv_chain_plan(int w_kind, const sn_gemv_job *jobs, int njobs, int M, void *workspace,
                       size_t workspace_bytes, sn_gemv_chain_info *info, void *stream);
int sn_gemv_chain_launch(const sn_gemv_chain_info *info, void *workspace, unsigned flags, void *stream);

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

/*
 * Status recorded on the device by kernels whose bounded waits ran out
 * (SN_ERR_TIMEOUT), SN_OK if none.  reset != 0 clears it.  Unlike every other
 * entry point this one synchronises `stream` (it copies the status words back),
 * so it must not be called while the stream is being captured.
 * No counterpart in the reference (its kernels have no device-side waits).
 */
int sn_device_status(int reset, void *stream);

/*
 * Failure-detection check: launches one thread that waits, with the same
 * bounded mbarrier wait every kernel here uses, on a barrier nothing arrives
 * on.  After limit_ns nanoseconds (1 us .. 1 s) the wait gives up, the kernel
 * records SN_ERR_TIMEOUT and returns, so a following sn_device_status reports
 * SN_ERR_TIMEOUT and the context stays usable.  No counterpart in the
 * reference (its kernels have no device-side waits).
 */
int sn_diag_bounded_wait(uint64_t limit_ns, void *stream);

/*
 * Multi-codebook logit head, BASELINE config 4 (no kernel exists in the
 * reference; it is the per-codebook bmm its decode step runs on the 9 heads):
 *   logits[cb, b, n] = sum_k hidden[cb, b, k] * W[cb, k, n]
 * sn_codebook_head_pack transposes W [ncb, K, N] (bf16) once into Wt
 * [ncb, N, K]; sn_codebook_head_bmm reads hidden [ncb, B, K] (bf16,
 * contiguous) and Wt, and writes fp32 logits [ncb, B, N].  B <= 4 runs the
 * decode GEMV, B >= 5 the tcgen05 contraction (K a multiple of 64).  flags:
 * 0 or SN_FLAG_PDL (programmatic dependent launch: the head starts and
 * streams its first weights while the previous kernel on the stream is still
 * running, and reads hidden / writes logits only after it has finished).
 */
int sn_codebook_head_pack(const void *W, int ncb, int K, int N, void *Wt, void *stream);
int sn_codebook_head_bmm(const void *hidden, const void *Wt, float *logits, int ncb, int B, int K, int N,
                         unsigned flags, void *stream);

/*
 * Mamba2 SSD chunk product, replaces launch_bmm (kernels/bmm.py:96-117):
 *   CB[b, c, g, i, j] = sum_d C[b, c*CHUNK+i, g, d] * B[b, c*CHUNK+j, g, d]
 * C, B: bf16 [BATCH, >= SEQLEN, NGROUPS, DSTATE] with element strides
 * (s*b, s*t, s*g) and unit stride over d; CB_out: fp32 contiguous
 * [BATCH, NCHUNKS, NGROUPS, CHUNK, CHUNK].  Positions >= SEQLEN count as zero
 * (the masked semantics of kernels/bmm.py:205-212), so the ragged last chunk
 * is exact.  NCHUNKS * CHUNK must cover SEQLEN.
 */
int sn_ssd_chunk_bmm(const void *C, const void *B, int64_t sCb, int64_t sCt, int64_t sCg, int64_t sBb,
                     int64_t sBt, int64_t sBg, int batch, int seqlen, int ngroups, int dstate, int chunk,
                     int nchunks, float *CB_out, void *stream);

/*
 * Fused Snake + Conv1d, replaces fused_snake_conv1d / _launch_fused_snake_conv1d
 * (kernels/fused_snake_conv.py:89-199):
 *   y[b, o, t] = bias[o] + sum_{i,k} W[o, i, k] * snake(x[b, i, t*stride - padding + k*dilation])
 *   snake(v) = v + sin(alpha[i] * v)^2 / (alpha[i] + eps), zero outside [0, T)
 * x: fp32 [B, Cin, T]; alpha: fp32 [Cin]; W: fp32 [Cout, Cin, K]; bias: fp32
 * [Cout] or NULL; y: fp32 [B, Cout, Tout], Tout = sn_snake_conv1d_output_length
 * (kernels/fused_snake_conv.py:13-26).  All contiguous.  With a workspace of
 * at least sn_snake_conv1d_workspace_size(Cin, Cout, K) bytes (16-byte
 * aligned; the packed bf16 hi/lo weights go there) shapes with stride 1,
 * K <= 7, (K-1)*dilation <= 72 and Cin, Cout multiples of 16 run on the
 * tensor cores; everything else runs the per-output fallback.
 */
int64_t sn_snake_conv1d_output_length(int64_t T, int K, int stride, int padding, int dilation);
size_t sn_snake_conv1d_workspace_size(int Cin, int Cout, int K);
int sn_snake_conv1d(const float *x, const float *alpha, const float *W, const float *bias, float *y, int B,
                    int Cin, int Cout, int T, int K, int stride, int padding, int dilation, float eps,
                    void *workspace, size_t workspace_bytes, void *stream);

/*
 * The DAC decoder's other Snake -> conv edges (the HF transformers DacDecoder
 * the reference decodes with, modeling_dac.py DacResidualUnit / DacDecoder;
 * edge list in docs/dac_architecture.md:137-168, 306-314).
 *
 * sn_snake_conv1d_ex: sn_snake_conv1d plus
 *   act      SN_ACT_SNAKE (as sn_snake_conv1d) or SN_ACT_NONE (no activation:
 *            the decoder's stem conv1; alpha may be NULL),
 *   residual fp32 [B, Cout, Tout] added after the bias (the residual unit's
 *            "hidden_state + conv2(snake2(...))"), or NULL,
 *   post     SN_POST_NONE or SN_POST_TANH (the decoder's final tanh), applied last.
 * residual must not alias y.  flags: 0 or SN_FLAG_PREPACKED (workspace holds
 * sn_snake_conv1d_pack(W) output; W is still read by the fallback path).
 */
#define SN_ACT_SNAKE 0
#define SN_ACT_NONE 1
#define SN_ACT_SILU 2 /* sn_causal_conv1d_update only */
#define SN_POST_NONE 0
#define SN_POST_TANH 1
int sn_snake_conv1d_ex(const float *x, const float *alpha, const float *W, const float *bias,
                       const float *residual, float *y, int B, int Cin, int Cout, int T, int K, int stride,
                       int padding, int dilation, float eps, int act, int post, unsigned flags, void *workspace,
                       size_t workspace_bytes, void *stream);
/* Pack W [Cout, Cin, K] once into the tensor-core layout (packed_bytes >=
 * sn_snake_conv1d_workspace_size(Cin, Cout, K), 16-byte aligned), for calls
 * with SN_FLAG_PREPACKED: a decoder packs its weights at load time. */
int sn_snake_conv1d_pack(const float *W, int Cin, int Cout, int K, void *packed, size_t packed_bytes,
                         void *stream);

/*
 * Snake1d on its own, elementwise over x [B, C, T] (contiguous):
 *   y[b, c, t] = x + sin(alpha[c] * x)^2 / (alpha[c] + eps)
 * with the same device arithmetic as the fused kernels' activation (sin^2
 * after a Cody-Waite reduction modulo pi, accurate for any |alpha * x|).
 * y may equal x.  The Snake of kernels/fused_snake_conv.py:264-286
 * (reference_snake_conv1d) and of transformers' Snake1d, which the reference's
 * DAC decoder runs before each conv (docs/dac_architecture.md:46-51).
 */
int sn_snake1d(const float *x, const float *alpha, float *y, int B, int C, int64_t T, float eps, void *stream);

/*
 * Fused Snake + ConvTranspose1d (the DacDecoderBlock's snake1 -> conv_t1):
 *   y[b, o, t] = bias[o] + sum over (i, k, j) with t = j*stride - padding + k of
 *                snake(x[b, i, j]) * W[i, o, k]
 * x: fp32 [B, Cin, T]; W: fp32 [Cin, Cout, K] (torch ConvTranspose1d layout,
 * groups 1, dilation 1, output_padding 0); y: fp32 [B, Cout, Ty], Ty =
 * sn_snake_conv_transpose1d_output_length.  Workspace as sn_snake_conv1d
 * (sn_snake_conv1d_workspace_size(Cin, Cout, K) bytes).  K a multiple of
 * stride with Cin and Cout * stride multiples of 16 runs on the tensor cores
 * as a polyphase GEMM (K / stride taps, one GEMM column per (o, phase));
 * other shapes run a per-output fallback.
 */
int64_t sn_snake_conv_transpose1d_output_length(int64_t T, int K, int stride, int padding);
int sn_snake_conv_transpose1d(const float *x, const float *alpha, const float *W, const float *bias, float *y,
                              int B, int Cin, int Cout, int T, int K, int stride, int padding, float eps,
                              unsigned flags, void *workspace, size_t workspace_bytes, void *stream);
/* Pack W [Cin, Cout, K] into the polyphase planes for SN_FLAG_PREPACKED calls;
 * SN_ERR_UNSUPPORTED when K is not a multiple of stride (no polyphase GEMM). */
int sn_snake_conv_transpose1d_pack(const float *W, int Cin, int Cout, int K, int stride, void *packed,
                                   size_t packed_bytes, void *stream);

/*
 * Strided variants for a streaming (cached-convolution) decoder, whose
 * per-layer inputs and outputs are windows of larger buffers: x, y and
 * residual take a batch stride (*_bs) and a channel-row stride (*_ld), in
 * elements, with time contiguous (ld >= the row's length; batches must not
 * overlap).  y must not overlap x or residual.  Otherwise
 * sn_snake_conv1d_strided is sn_snake_conv1d_ex.
 * sn_snake_conv_transpose1d_strided writes samples [0, Ty) of the transposed
 * convolution with the given padding, for any 1 <= Ty <= (T - 1) * stride -
 * padding + K: a streaming decoder passes [previous input frame | new frames]
 * with padding = stride (+ the layer's own padding on the first chunk) and Ty
 * = the samples whose input frames have all arrived.  No counterpart in the
 * reference, which vocodes a stream by re-decoding overlapping windows
 * (scripts/streaming.py:191-238); these replace that re-decode with
 * per-convolution left-history caches (docs/dac_profile.md:42,86).
 */
int sn_snake_conv1d_strided(const float *x, int64_t x_bs, int64_t x_ld, const float *alpha, const float *W,
                            const float *bias, const float *residual, int64_t r_bs, int64_t r_ld, float *y,
                            int64_t y_bs, int64_t y_ld, int B, int Cin, int Cout, int T, int K, int stride,
                            int padding, int dilation, float eps, int act, int post, unsigned flags, void *workspace,
                            size_t workspace_bytes, void *stream);
int sn_snake_conv_transpose1d_strided(const float *x, int64_t x_bs, int64_t x_ld, const float *alpha, const float *W,
                                      const float *bias, float *y, int64_t y_bs, int64_t y_ld, int B, int Cin,
                                      int Cout, int T, int K, int stride, int padding, int Ty, float eps,
                                      unsigned flags, void *workspace, size_t workspace_bytes, void *stream);

/*
 * History move of a streaming decoder, for up to SN_SHIFT_MAX_DESCS layer
 * buffers in one launch: in every row (batch b, channel c) of entry i,
 * samples [src, src + len) move to [0, len) (len <= SN_SHIFT_MAX_LEN;
 * overlapping ranges are fine).  The table is read on the host and passed by
 * value, so it may be reused or freed as soon as the call returns.
 */
#define SN_SHIFT_MAX_DESCS 48
#define SN_SHIFT_MAX_LEN 64
typedef struct sn_shift_desc {
  float *buf;
  int64_t batch_stride, row_stride; /* elements */
  int batches, rows;
  int src, len;
} sn_shift_desc;
int sn_stream_shift(const sn_shift_desc *descs, int n, void *stream);

/*
 * Allocation-free Snake + Conv1d.  No counterpart in the reference.
 *
 * For callers that must not allocate device memory at all: a host that runs
 * the vocoder from a real-time audio callback (cudaMalloc can block and
 * synchronise the whole device), or an application that loads this library
 * through the C ABI from another runtime that gives it no CUDA allocator.
 * Same computation and arguments as sn_snake_conv1d minus the workspace: the
 * packed weights go to a static device array of
 * SN_SNAKE_CONV1D_NOALLOC_MAX_SCRATCH bytes (16 MiB, enough for the largest
 * DAC unit, Cin = Cout = 768, K = 7) that every GPU loading the library keeps
 * until the process exits.
 *
 * Limit: only shapes that run on the tensor cores use the array (stride 1,
 * K <= 7, (K-1)*dilation <= 72, Cin and Cout multiples of 16); among those,
 * problems whose packed weights (Cin * Cout * K * 4 bytes) exceed the array
 * return SN_ERR_SCRATCH_LIMIT.  Every other shape runs the per-output kernel,
 * which reads W directly, needs no scratch and has no size limit.
 *
 * The function calls no cudaMalloc / cudaFree.  It looks the array's device
 * address up (cudaGetSymbolAddress, with the caller's device current) on
 * every call; SN_ERR_SCRATCH_ADDRESS means that lookup failed.  The first
 * call into this library on a device (this one or any other entry point)
 * loads the library's device code on that device, which reserves the 16 MiB
 * and may block or synchronise: make it outside the real-time thread and
 * before capturing any stream (or load eagerly with CUDA_MODULE_LOADING=EAGER).
 * All calls share the one array and it keeps the last call's weights: calls
 * that may overlap on the GPU (other streams, other threads) race on it and
 * must be ordered by the caller.
 */
#define SN_SNAKE_CONV1D_NOALLOC_MAX_SCRATCH (16u * 1024u * 1024u)
int sn_snake_conv1d_noalloc(const float *x, const float *alpha, const float *W, const float *bias, float *y,
                            int B, int Cin, int Cout, int T, int K, int stride, int padding, int dilation,
                            float eps, void *stream);

/*
 * Mamba2 decode-step ops (bf16 tensors, fp32 arithmetic, bf16 outputs), the
 * semantics of the libraries the reference's frozen goldens were made with
 * (scripts/validation_harness.py:39,58-115,140-171: causal_conv1d
 * 1.6.2.post1, mamba_ssm 2.3.2.post1).  All tensors contiguous.  Each op
 * is launched with programmatic dependent launch and waits for the previous
 * kernel in the stream before its first memory access (same results as a
 * plain launch; its start overlaps that kernel's tail), and lets the next
 * one start early.
 *
 * sn_causal_conv1d_update (causal_conv1d_update): conv_state [B, D, W]
 * (W <= 8) shifts one step left and takes x [B, D] as its newest column, in
 * place; y [B, D] = act(sum_w state[b, d, w] * weight[d, w] + bias[d]),
 * activation SN_ACT_NONE or SN_ACT_SILU; bias may be NULL.
 */
int sn_causal_conv1d_update(const void *x, void *conv_state, const void *weight, const void *bias, void *y, int B,
                            int D, int W, int activation, void *stream);
/*
 * sn_selective_state_update (mamba_ssm selective_state_update): state
 * [batch, nheads, headdim, dstate] (dstate <= 256) updated in place;
 * dt' = dt + dt_bias, softplus(dt') when dt_softplus (threshold 20);
 * state = state * exp(dt' * A) + dt' * B * x;
 * y = sum_dstate(state * C) + D * x, times SiLU(z).  x, dt, z, y [batch,
 * nheads, headdim]; A fp32 [nheads, headdim, dstate]; B, C [batch, ngroups,
 * dstate] (nheads / ngroups heads per group); D, dt_bias [nheads, headdim];
 * D, z, dt_bias may be NULL.
 */
int sn_selective_state_update(void *state, const void *x, const void *dt, const float *A, const void *B,
                              const void *C, const void *D, const void *z, const void *dt_bias, void *y, int batch,
                              int nheads, int headdim, int dstate, int ngroups, int dt_softplus, void *stream);
/*
 * sn_rmsnorm_gated (mamba_ssm layernorm_gated rmsnorm_fn): rows x [rows, N]
 * normalised per group of group_size columns (N % group_size == 0,
 * group_size <= 8192): norm_before_gate 0: y = rms(x * SiLU(z)) * weight
 * (+ bias); 1: y = rms(x) * weight (+ bias) * SiLU(z).  z, bias may be NULL.
 */
int sn_rmsnorm_gated(const void *x, const void *weight, const void *bias, const void *z, void *y, int rows, int N,
                     int group_size, float eps, int norm_before_gate, void *stream);
/*
 * sn_layer_norm_fused (mamba_ssm layer_norm_fn, prenorm add + norm): h = x +
 * residual (residual bf16, or fp32 when residual_f32; may be NULL) in fp32;
 * residual_out (may be NULL; bf16, or fp32 when residual_out_f32) = h; out =
 * LayerNorm(h) (RMSNorm when is_rms_norm) * weight (+ bias), from the
 * unrounded h.  x, out [rows, N], N <= 8192.
 */
int sn_layer_norm_fused(const void *x, const void *residual, int residual_f32, const void *weight,
                        const void *bias, void *out, void *residual_out, int residual_out_f32, int rows, int N,
                        float eps, int is_rms_norm, void *stream);

/*
 * Decode-step glue of the Zonos hybrid (no counterpart kernels in the
 * reference, where torch slices, broadcasts and elementwise ops run between
 * the library calls; each of these is one launch in place of several).
 *
 * sn_mamba2_split_conv: from the Mamba2 in_proj output zxbcdt [batch, ld]
 * (= [z (d_inner) | xBC (d_inner + 2 ngroups d_state) | dt (nheads)], ld >=
 * that width) writes z [batch, d_inner]; causal_conv1d_update with SiLU of
 * xBC (conv_state [batch, conv_dim, d_conv] updated in place, weight
 * [conv_dim, d_conv], bias or NULL) split into x [batch, d_inner], B and C
 * [batch, ngroups * d_state]; and dt broadcast over headdim [batch, nheads,
 * headdim] (nheads * headdim == d_inner).  Same values as the separate
 * sn_causal_conv1d_update on the contiguous slices.
 * sn_rotary_kv_append: qkv [batch, (nheads + 2 nheads_kv) head_dim] -> q
 * [batch, nheads, head_dim] with non-interleaved rotary (cos / sin fp32
 * [head_dim / 2] of the position), k rotated and v written at position pos
 * of k_cache / v_cache [batch, nheads_kv, max_seqlen, head_dim].
 * sn_swiglu: h [batch, 2d] -> y [batch, d] = h[:, :d] * SiLU(h[:, d:]).
 * All bf16 and contiguous.
 */
int sn_mamba2_split_conv(const void *zxbcdt, int64_t ld, void *conv_state, const void *conv_weight,
                         const void *conv_bias, void *z, void *x, void *B, void *C, void *dt, int batch, int d_inner,
                         int ngroups, int d_state, int nheads, int headdim, int d_conv, void *stream);
/*
 * sn_mamba2_conv_ssu: sn_mamba2_split_conv followed by
 * sn_selective_state_update with dt softplus, in one launch (the Mamba2
 * step between in_proj and the gated norm: mamba_ssm Mamba2.step, as the
 * two calls above restate it).  zxbcdt, conv_state, conv_weight,
 * conv_bias as in sn_mamba2_split_conv; ssm_state [batch, nheads, headdim,
 * d_state] updated in place; A fp32 [nheads], D and dt_bias bf16 [nheads]
 * (NULL for none): the per-head values those two calls take broadcast over
 * headdim and d_state.  Writes z [batch, d_inner] and y [batch, nheads,
 * headdim], equal bit for bit to the two-call path.  sync: batch * ngroups
 * unsigned counters, zero before the first call and left zero by each call
 * (one set per stream of calls: calls that share it must not overlap).
 * SN_ERR_UNSUPPORTED unless d_state is 128 or 256, headdim a multiple of 16
 * and ssm_state 16-byte aligned (the two-call path serves the rest).
 */
int sn_mamba2_conv_ssu(const void *zxbcdt, int64_t ld, void *conv_state, const void *conv_weight,
                       const void *conv_bias, void *ssm_state, const float *A, const void *D, const void *dt_bias,
                       void *z, void *y, unsigned *sync, int batch, int d_inner, int ngroups, int d_state, int nheads,
                       int headdim, int d_conv, void *stream);
int sn_rotary_kv_append(const void *qkv, void *q, void *k_cache, void *v_cache, const float *cos, const float *sin,
                        int batch, int nheads, int nheads_kv, int head_dim, int max_seqlen, int pos, void *stream);
int sn_swiglu(const void *h, void *y, int batch, int d, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* SONATA_B200_H_ */
