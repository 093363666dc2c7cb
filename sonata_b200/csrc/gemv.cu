// Decode (batch 1-4) GEMV for B200: y[m, n] = scale[n] * sum_k x[m, k] * W[n, k].
//
// Replaces the CuTe-DSL skinny GEMVs of kernels/gemv.py (12-193) and adds the
// fused-dequant weight-only int8 / e4m3 variants that scripts/fake_quant.py
// only simulates.  The path is HBM-bound: the weight is streamed once, x and y
// are a few KB.
//
// bf16 fast path (gemv_mma_kernel): one CTA per SM owns an equal contiguous
// range of weight rows.  A producer lane streams 32 KB slots of whole rows
// (cp.async.bulk, L2 evict-first) into a shared-memory ring before
// griddepcontrol.wait, so under programmatic dependent launch the next GEMV of
// a decode step streams its weights while this one drains.  The dot products
// run on the tensor core (tcgen05.mma, fp32 accumulation in TMEM): each row is
// cut into segments that form the 8-row groups of an M = 128 operand, x is
// the matching B operand, and the epilogue sums the diagonal partial products
// with a warp-shuffle reduction.  A slot is released the moment its MMAs
// retire, and the CUDA cores issue a few instructions per 32 KB.
//
// 8-bit weights and batched calls (gemv_bulk_kernel): the same ring, with
// eight consumer warps reducing one row each with packed f32x2 FMAs (FFMA2)
// against x staged as bf16 in shared memory.
//
// Measured on B200: the 156-GEMV decode chain of BASELINE config 2 runs about
// 1.6x faster than cuBLAS in the same graph; what remains is the latency of
// each kernel boundary (waiting for the producer of x, then loading x), not
// the arithmetic.
//
// Fallbacks: gemv_vec_kernel (16-byte register loads; rows whose length is not
// a multiple of 16 bytes or longer than 64 KB) and gemv_scalar_kernel (rows
// that are not 16-byte aligned).
#include "tc.cuh"

#include <algorithm>
#include <climits>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>
#include <vector>

namespace sn {
namespace {

enum WKind : int { W_BF16 = 0, W_INT8 = 1, W_E4M3 = 2 };

template <int WK>
struct WT {
  static constexpr int EPC = (WK == W_BF16) ? 8 : 16;  // elements per 16-byte chunk
  static constexpr int ESZ = (WK == W_BF16) ? 2 : 1;   // bytes per element
};

struct GemvParams {
  const uint8_t* W;  // weight base (bytes)
  int64_t ldw;       // row stride, elements
  int64_t sW;        // batch stride, elements
  const float* scale;
  int64_t sS;
  const __nv_bfloat16* x;
  int64_t ldx, sx;
  void* y;
  int64_t ldy, sy;
  int M, N, K;
  int Kp;     // padded fp32 row stride of x in shared memory
  int y_f32;
  int x_vec;  // x rows are 16-byte aligned and K % 8 == 0
  // Next-weight L2 prefetch (tensor-core GEMV only; pf == nullptr: none).
  // The next GEMV's pf_rows rows (pf_row_bytes each, pf_ld bytes apart) are
  // cut into pf_parts equal ranges, one per CTA of its launch; the first
  // pf_part_bytes of every range are prefetched once this GEMV has issued
  // all of its own weight copies.
  const uint8_t* pf;
  int64_t pf_ld;
  int pf_rows, pf_parts;
  int pf_q, pf_rem;  // the next launch's rows per CTA: pf_q, one more for its first pf_rem CTAs
  uint32_t pf_row_bytes, pf_part_bytes;
  int x_rot;    // x row copies start at a CTA-dependent 128-byte piece
  int pf_lead;  // issue once all but this many of the CTA's own tiles have landed (< 0: at once)
  // Normalisation fused into the x staging of the bf16 tensor-core GEMV
  // (sn_gemv_bf16_norm): every CTA normalises the x rows it stages.
  int xn;                       // 0 none, SN_NORM_RMS_GATED, SN_NORM_ADD_LAYER
  const __nv_bfloat16* xn_aux;  // gate z (RMS) or residual (LayerNorm, may be null), [M][K] row stride ldx
  const __nv_bfloat16* xn_w;    // norm weight [K]
  const __nv_bfloat16* xn_b;    // LayerNorm bias [K] or null
  __nv_bfloat16* xn_rout;       // LayerNorm: x + residual [M][K] (row stride ldx), written by CTA (0, 0), or null
  float xn_eps;
};

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

// Stage x[0:M, 0:K] (bf16, global) as fp32 rows of stride Kp in shared memory;
// rows M..MT-1 are zero.
template <int MT>
__device__ __forceinline__ void stage_x(const GemvParams& p, const __nv_bfloat16* xb, float* xs) {
  if (p.x_vec) {
    const int cpr = p.K >> 3;  // 8-element chunks per row
    for (int i = threadIdx.x; i < MT * cpr; i += kThreads) {
      const int m = i / cpr, c = i - m * cpr;
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
      if (m < p.M) {
        const uint4 u = *reinterpret_cast<const uint4*>(xb + m * p.ldx + c * 8);
        a = make_float4(bf16lo(u.x), bf16hi(u.x), bf16lo(u.y), bf16hi(u.y));
        b = make_float4(bf16lo(u.z), bf16hi(u.z), bf16lo(u.w), bf16hi(u.w));
      }
      float4* dst = reinterpret_cast<float4*>(xs + m * p.Kp + c * 8);
      dst[0] = a;
      dst[1] = b;
    }
  } else {
    for (int i = threadIdx.x; i < MT * p.K; i += kThreads) {
      const int m = i / p.K, k = i - m * p.K;
      xs[m * p.Kp + k] = (m < p.M) ? __bfloat162float(xb[m * p.ldx + k]) : 0.f;
    }
  }
}

// 16 one-byte codes -> 16 exact fp32 values (as 8 float2 pairs).
template <int WK>
__device__ __forceinline__ void dequant16(const uint4& w, float2 (&v)[8]) {
  if constexpr (WK == W_INT8) {
    // Signed byte q -> fp32 exactly: bias to u = q + 128, splice u into the
    // mantissa of 2^23 (0x4B0000uu == 2^23 + u), subtract 2^23 + 128.
    const float2 off = make_float2(-8388736.0f, -8388736.0f);
    const uint32_t words[4] = {w.x ^ 0x80808080u, w.y ^ 0x80808080u, w.z ^ 0x80808080u, w.w ^ 0x80808080u};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float f0 = __uint_as_float(__byte_perm(words[j], 0x4B000000u, 0x7440));
      const float f1 = __uint_as_float(__byte_perm(words[j], 0x4B000000u, 0x7441));
      const float f2 = __uint_as_float(__byte_perm(words[j], 0x4B000000u, 0x7442));
      const float f3 = __uint_as_float(__byte_perm(words[j], 0x4B000000u, 0x7443));
      v[2 * j] = __fadd2_rn(make_float2(f0, f1), off);
      v[2 * j + 1] = __fadd2_rn(make_float2(f2, f3), off);
    }
  } else {
    // e4m3 pairs -> f16x2 (hardware cvt, exact) -> fp32 pairs (exact).
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const __half2_raw h01 =
          __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(words[j] & 0xFFFFu), __NV_E4M3);
      const __half2_raw h23 =
          __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(words[j] >> 16), __NV_E4M3);
      v[2 * j] = __half22float2(*reinterpret_cast<const __half2*>(&h01));
      v[2 * j + 1] = __half22float2(*reinterpret_cast<const __half2*>(&h23));
    }
  }
}

// acc[m] += dot(16-byte weight chunk, x[m, k0 : k0 + EPC])
template <int WK, int MT>
__device__ __forceinline__ void chunk_fma(const uint4& w, const float* __restrict__ xs, int Kp, int k0,
                                          float2 (&acc)[MT]) {
  if constexpr (WK == W_BF16) {
    const float2 w0 = make_float2(bf16lo(w.x), bf16hi(w.x));
    const float2 w1 = make_float2(bf16lo(w.y), bf16hi(w.y));
    const float2 w2 = make_float2(bf16lo(w.z), bf16hi(w.z));
    const float2 w3 = make_float2(bf16lo(w.w), bf16hi(w.w));
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const float4 xa = *reinterpret_cast<const float4*>(xs + m * Kp + k0);
      const float4 xb = *reinterpret_cast<const float4*>(xs + m * Kp + k0 + 4);
      acc[m] = __ffma2_rn(w0, make_float2(xa.x, xa.y), acc[m]);
      acc[m] = __ffma2_rn(w1, make_float2(xa.z, xa.w), acc[m]);
      acc[m] = __ffma2_rn(w2, make_float2(xb.x, xb.y), acc[m]);
      acc[m] = __ffma2_rn(w3, make_float2(xb.z, xb.w), acc[m]);
    }
  } else {
    float2 v[8];
    dequant16<WK>(w, v);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const float4* xr = reinterpret_cast<const float4*>(xs + m * Kp + k0);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 xv = xr[q];
        acc[m] = __ffma2_rn(v[2 * q], make_float2(xv.x, xv.y), acc[m]);
        acc[m] = __ffma2_rn(v[2 * q + 1], make_float2(xv.z, xv.w), acc[m]);
      }
    }
  }
}

// acc[m] += dot(16-byte weight chunk, xr[m][o : o + EPC]) with x in registers.
template <int WK, int MT, int XN>
__device__ __forceinline__ void chunk_fma_regs(const uint4& w, const float (&xr)[MT][XN], int o,
                                               float2 (&acc)[MT]) {
  if constexpr (WK == W_BF16) {
    const float2 wv[4] = {make_float2(bf16lo(w.x), bf16hi(w.x)), make_float2(bf16lo(w.y), bf16hi(w.y)),
                          make_float2(bf16lo(w.z), bf16hi(w.z)), make_float2(bf16lo(w.w), bf16hi(w.w))};
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int j = 0; j < 4; ++j)
        acc[m] = __ffma2_rn(wv[j], make_float2(xr[m][o + 2 * j], xr[m][o + 2 * j + 1]), acc[m]);
  } else {
    float2 v[8];
    dequant16<WK>(w, v);
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int j = 0; j < 8; ++j)
        acc[m] = __ffma2_rn(v[j], make_float2(xr[m][o + 2 * j], xr[m][o + 2 * j + 1]), acc[m]);
  }
}

template <int WK>
__device__ __forceinline__ float load_weight_scalar(const uint8_t* row, int k) {
  if constexpr (WK == W_BF16) {
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(row)[k]);
  } else if constexpr (WK == W_INT8) {
    return static_cast<float>(reinterpret_cast<const int8_t*>(row)[k]);
  } else {
    const __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(row[k]), __NV_E4M3);
    return __half2float(*reinterpret_cast<const __half*>(&h));
  }
}

template <int MT>
__device__ __forceinline__ void store_row(const GemvParams& p, void* yb, int n, int m, float v) {
  if (m >= p.M) return;
  if (p.y_f32)
    reinterpret_cast<float*>(yb)[m * p.ldy + n] = v;
  else
    reinterpret_cast<__nv_bfloat16*>(yb)[m * p.ldy + n] = __float2bfloat16_rn(v);
}

// Vectorised kernel: weight rows are 16-byte aligned.
template <int WK, int MT, int R, int CPL>
__global__ void __launch_bounds__(kThreads) gemv_vec_kernel(const GemvParams p) {
  constexpr int EPC = WT<WK>::EPC;
  constexpr int ESZ = WT<WK>::ESZ;
  extern __shared__ __align__(16) float xs[];
  pdl_launch_dependents();

  const int b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = (blockIdx.x * kWarps + warp) * R;
  const int nck = p.K / EPC;  // whole 16-byte chunks per row
  const uint8_t* Wb = p.W + (int64_t)b * p.sW * ESZ;

  const uint4* rowp[R];
  bool live[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    live[r] = (row0 + r) < p.N;
    rowp[r] = reinterpret_cast<const uint4*>(Wb + (int64_t)(live[r] ? row0 + r : 0) * p.ldw * ESZ);
  }

  uint4 wv[R][CPL];
  auto issue = [&](int base) {
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        const int idx = base + c * 32 + lane;
        wv[r][c] = (live[r] && idx < nck) ? ld_stream_v4(rowp[r] + idx) : make_uint4(0, 0, 0, 0);
      }
  };

  issue(0);           // weights are independent of the previous kernel
  pdl_wait();         // x (and y) may be produced / consumed by it
  stage_x<MT>(p, p.x + (int64_t)b * p.sx, xs);
  __syncthreads();

  float2 acc[R][MT];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[r][m] = make_float2(0.f, 0.f);

  for (int base = 0; base < nck; base += CPL * 32) {
    if (base) issue(base);
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
      const int idx = base + c * 32 + lane;
      if (idx < nck) {
#pragma unroll
        for (int r = 0; r < R; ++r) chunk_fma<WK, MT>(wv[r][c], xs, p.Kp, idx * EPC, acc[r]);
      }
    }
  }

  // K tail that does not fill a 16-byte chunk
  const int k_tail = nck * EPC;
  if (k_tail < p.K) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (!live[r]) continue;
      const uint8_t* row = reinterpret_cast<const uint8_t*>(rowp[r]);
      for (int k = k_tail + lane; k < p.K; k += 32) {
        const float wk = load_weight_scalar<WK>(row, k);
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[r][m].x = fmaf(wk, xs[m * p.Kp + k], acc[r][m].x);
      }
    }
  }

  void* yb = reinterpret_cast<uint8_t*>(p.y) + (int64_t)b * p.sy * (p.y_f32 ? 4 : 2);
#pragma unroll
  for (int r = 0; r < R; ++r) {
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const float s = warp_sum(acc[r][m].x + acc[r][m].y);
      if (lane == 0 && live[r]) {
        float v = s;
        if constexpr (WK != W_BF16) v *= p.scale[(int64_t)b * p.sS + row0 + r];
        store_row<MT>(p, yb, row0 + r, m, v);
      }
    }
  }
}

// Fallback for weight rows that are not 16-byte aligned: one warp per row,
// element loads.  Correct for any stride; not the fast path.
template <int WK, int MT>
__global__ void __launch_bounds__(kThreads) gemv_scalar_kernel(const GemvParams p) {
  constexpr int ESZ = WT<WK>::ESZ;
  extern __shared__ __align__(16) float xs[];
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.y;
  stage_x<MT>(p, p.x + (int64_t)b * p.sx, xs);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x * kWarps + warp;
  if (n >= p.N) return;
  const uint8_t* row = p.W + ((int64_t)b * p.sW + (int64_t)n * p.ldw) * ESZ;
  float acc[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) acc[m] = 0.f;
  for (int k = lane; k < p.K; k += 32) {
    const float wk = load_weight_scalar<WK>(row, k);
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = fmaf(wk, xs[m * p.Kp + k], acc[m]);
  }
  void* yb = reinterpret_cast<uint8_t*>(p.y) + (int64_t)b * p.sy * (p.y_f32 ? 4 : 2);
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    const float s = warp_sum(acc[m]);
    if (lane == 0) {
      float v = s;
      if constexpr (WK != W_BF16) v *= p.scale[(int64_t)b * p.sS + n];
      store_row<MT>(p, yb, n, m, v);
    }
  }
}

// ---------------------------------------------------------------------------
// TMA bulk-copy kernel (the fast path).
//
// Grid: one CTA per SM.  CTA c owns the contiguous row range
// [c*R/G, (c+1)*R/G) of the flattened (batch x N) rows, so every SM streams
// the same number of bytes.  Warp 8 lane 0 streams chunks of `rs` whole rows
// (~32 KB, one cp.async.bulk when the rows are adjacent) global -> shared into
// a ring of `ns` slots with a full/empty mbarrier pair per slot; warps 0-7
// consume.  x is staged once as bf16 in shared memory.
//
// Resource use is kept to about half an SM (<= 112 registers per thread,
// ~110 KB of shared memory) so that under programmatic dependent launch the
// next GEMV's CTA fits beside this one and streams its weights (issued before
// griddepcontrol.wait) while this one drains: the HBM pipe stays full across
// the kernel boundaries of a decode step.
// ---------------------------------------------------------------------------
constexpr int kBulkWarps = 8;  // consumer warps; +1 producer warp
constexpr int kBulkThreads = (kBulkWarps + 1) * 32;

__host__ __device__ constexpr uint32_t round_up_u32(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

struct BulkShape {
  int ns;              // ring slots
  int rs;              // weight rows per slot (<= kBulkWarps: one row per consumer warp)
  uint32_t slot_bytes;
  uint32_t bar_bytes;
  uint32_t xs_bytes;   // x area: span * MT rows of Kp (fp32 for bf16 weights, bf16 planes for 8-bit)
  int total_rows;      // batch * N (< 2^31, checked on the host)
  int contiguous;      // rows of consecutive index are adjacent in memory
};

// x is staged in shared memory as bf16 (half the shared-memory traffic of
// fp32, which measured slower in the decode chain).  Next to bf16 weights a
// row is plain; next to 8-bit weights it is stored as two planes of Kp/2, the
// h-th plane holding the h-th 8-element half of every 16-element chunk, so
// that both 16-byte x loads of a warp are contiguous.
template <int WK>
struct XStage {
  static constexpr int BYTES = 2;
};

// acc[m][*] += dot(16-byte weight chunk idx, x[m]); two FFMA2 chains per row.
template <int WK, int MT>
__device__ __forceinline__ void chunk_fma2(const uint4& w, const __nv_bfloat16* __restrict__ xs, int Kp, int idx,
                                           float2 (&acc)[MT][2]) {
  if constexpr (WK == W_BF16) {
    const float2 w0 = make_float2(bf16lo(w.x), bf16hi(w.x));
    const float2 w1 = make_float2(bf16lo(w.y), bf16hi(w.y));
    const float2 w2 = make_float2(bf16lo(w.z), bf16hi(w.z));
    const float2 w3 = make_float2(bf16lo(w.w), bf16hi(w.w));
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const uint4 xv = *reinterpret_cast<const uint4*>(xs + m * Kp + idx * 8);
      acc[m][0] = __ffma2_rn(w0, make_float2(bf16lo(xv.x), bf16hi(xv.x)), acc[m][0]);
      acc[m][1] = __ffma2_rn(w1, make_float2(bf16lo(xv.y), bf16hi(xv.y)), acc[m][1]);
      acc[m][0] = __ffma2_rn(w2, make_float2(bf16lo(xv.z), bf16hi(xv.z)), acc[m][0]);
      acc[m][1] = __ffma2_rn(w3, make_float2(bf16lo(xv.w), bf16hi(xv.w)), acc[m][1]);
    }
  } else {
    float2 v[8];
    dequant16<WK>(w, v);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const uint4 xa = *reinterpret_cast<const uint4*>(xs + m * Kp + idx * 8);
      const uint4 xb = *reinterpret_cast<const uint4*>(xs + m * Kp + (Kp >> 1) + idx * 8);
      acc[m][0] = __ffma2_rn(v[0], make_float2(bf16lo(xa.x), bf16hi(xa.x)), acc[m][0]);
      acc[m][1] = __ffma2_rn(v[1], make_float2(bf16lo(xa.y), bf16hi(xa.y)), acc[m][1]);
      acc[m][0] = __ffma2_rn(v[2], make_float2(bf16lo(xa.z), bf16hi(xa.z)), acc[m][0]);
      acc[m][1] = __ffma2_rn(v[3], make_float2(bf16lo(xa.w), bf16hi(xa.w)), acc[m][1]);
      acc[m][0] = __ffma2_rn(v[4], make_float2(bf16lo(xb.x), bf16hi(xb.x)), acc[m][0]);
      acc[m][1] = __ffma2_rn(v[5], make_float2(bf16lo(xb.y), bf16hi(xb.y)), acc[m][1]);
      acc[m][0] = __ffma2_rn(v[6], make_float2(bf16lo(xb.z), bf16hi(xb.z)), acc[m][0]);
      acc[m][1] = __ffma2_rn(v[7], make_float2(bf16lo(xb.w), bf16hi(xb.w)), acc[m][1]);
    }
  }
}

// Same as chunk_fma2 with the x words already in registers: xv[m][0] holds
// the 16 bytes of x at chunk idx (bf16 weights), xv[m][0..1] the two planes'
// halves (8-bit weights).
template <int WK, int MT>
__device__ __forceinline__ void chunk_fma2_x(const uint4& w, const uint4 (&xv)[MT][2], float2 (&acc)[MT][2]) {
  if constexpr (WK == W_BF16) {
    const float2 w0 = make_float2(bf16lo(w.x), bf16hi(w.x));
    const float2 w1 = make_float2(bf16lo(w.y), bf16hi(w.y));
    const float2 w2 = make_float2(bf16lo(w.z), bf16hi(w.z));
    const float2 w3 = make_float2(bf16lo(w.w), bf16hi(w.w));
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const uint4& x = xv[m][0];
      acc[m][0] = __ffma2_rn(w0, make_float2(bf16lo(x.x), bf16hi(x.x)), acc[m][0]);
      acc[m][1] = __ffma2_rn(w1, make_float2(bf16lo(x.y), bf16hi(x.y)), acc[m][1]);
      acc[m][0] = __ffma2_rn(w2, make_float2(bf16lo(x.z), bf16hi(x.z)), acc[m][0]);
      acc[m][1] = __ffma2_rn(w3, make_float2(bf16lo(x.w), bf16hi(x.w)), acc[m][1]);
    }
  } else {
    float2 v[8];
    dequant16<WK>(w, v);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const uint4& xa = xv[m][0];
      const uint4& xb = xv[m][1];
      acc[m][0] = __ffma2_rn(v[0], make_float2(bf16lo(xa.x), bf16hi(xa.x)), acc[m][0]);
      acc[m][1] = __ffma2_rn(v[1], make_float2(bf16lo(xa.y), bf16hi(xa.y)), acc[m][1]);
      acc[m][0] = __ffma2_rn(v[2], make_float2(bf16lo(xa.z), bf16hi(xa.z)), acc[m][0]);
      acc[m][1] = __ffma2_rn(v[3], make_float2(bf16lo(xa.w), bf16hi(xa.w)), acc[m][1]);
      acc[m][0] = __ffma2_rn(v[4], make_float2(bf16lo(xb.x), bf16hi(xb.x)), acc[m][0]);
      acc[m][1] = __ffma2_rn(v[5], make_float2(bf16lo(xb.y), bf16hi(xb.y)), acc[m][1]);
      acc[m][0] = __ffma2_rn(v[6], make_float2(bf16lo(xb.z), bf16hi(xb.z)), acc[m][0]);
      acc[m][1] = __ffma2_rn(v[7], make_float2(bf16lo(xb.w), bf16hi(xb.w)), acc[m][1]);
    }
  }
}

// Chunks a consumer lane loads before its first FMA: as many independent
// 16-byte shared-memory loads in flight as the register budget allows.
template <int WK, int MT>
struct Batch {
  static constexpr int XW = (WK == W_BF16) ? 1 : 2;  // 16-byte x words per chunk and row
  static constexpr int U = (8 / (MT * XW)) < 1 ? 1 : (8 / (MT * XW));
};

template <int WK, int MT>
__global__ void __launch_bounds__(kBulkThreads, 2) gemv_bulk_kernel(const GemvParams p, const BulkShape sh) {
  constexpr int EPC = WT<WK>::EPC;
  constexpr int ESZ = WT<WK>::ESZ;
  extern __shared__ __align__(128) uint8_t smem[];
  const int ns = sh.ns, rs = sh.rs;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + ns;
  uint8_t* xs = smem + sh.bar_bytes;
  uint8_t* slots = smem + sh.bar_bytes + sh.xs_bytes;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = static_cast<int>(static_cast<int64_t>(sh.total_rows) * blockIdx.x / gridDim.x);
  const int r1 = static_cast<int>(static_cast<int64_t>(sh.total_rows) * (blockIdx.x + 1) / gridDim.x);
  const int nrows = r1 - r0;
  const uint32_t row_bytes = static_cast<uint32_t>(p.K) * ESZ;
  const int nchunks = (nrows + rs - 1) / rs;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ns; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, kBulkWarps);  // every consumer warp releases every chunk
    }
    fence_barrier_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kBulkWarps) {
    // ---------------- producer: weights only, so no griddepcontrol.wait ----
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      int c = 0;
      for (; c < nchunks; ++c) {
        const int s = c % ns, k = c / ns;
        if (k > 0 && !mbar_wait_bounded(empty + s, (k - 1) & 1)) {
          record_status(SN_ERR_TIMEOUT);
          break;
        }
        const int first = r0 + c * rs;
        const int cnt = min(rs, r1 - first);
        uint8_t* dst = slots + static_cast<size_t>(s) * sh.slot_bytes;
        mbar_arrive_expect_tx(full + s, static_cast<uint32_t>(cnt) * row_bytes);
        if (sh.contiguous) {
          const int b = first / p.N, n = first - b * p.N;
          bulk_g2s(dst, p.W + (static_cast<int64_t>(b) * p.sW + static_cast<int64_t>(n) * p.ldw) * ESZ,
                   static_cast<uint32_t>(cnt) * row_bytes, full + s, pol);
        } else {
          for (int r = 0; r < cnt; ++r) {
            const int row = first + r;
            const int b = row / p.N, n = row - b * p.N;
            bulk_g2s(dst + static_cast<size_t>(r) * row_bytes,
                     p.W + (static_cast<int64_t>(b) * p.sW + static_cast<int64_t>(n) * p.ldw) * ESZ, row_bytes,
                     full + s, pol);
          }
        }
      }
      if (c < nchunks) {  // error path: let the copies in flight land before exit
        for (int j = (c > ns ? c - ns : 0); j < c; ++j) mbar_wait_bounded(full + j % ns, (j / ns) & 1);
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  pdl_wait();  // x and y belong to the previous kernel from here on
  const int nck = p.K / EPC;
  const int b0 = r0 / p.N;
  const int nb = (r1 - 1) / p.N - b0 + 1;  // batch entries touched by this CTA
  {
    const int cpr = p.Kp >> 3;  // 8-element groups per staged row
    for (int i = threadIdx.x; i < nb * MT * cpr; i += kBulkWarps * 32) {
      const int bm = i / cpr, c = i - bm * cpr;
      const int bb = bm / MT, m = bm - bb * MT;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (m < p.M && c * 8 < p.K) {
        const __nv_bfloat16* src = p.x + static_cast<int64_t>(b0 + bb) * p.sx + m * p.ldx + c * 8;
        if (p.x_vec) {
          v = *reinterpret_cast<const uint4*>(src);
        } else {
          __align__(16) __nv_bfloat16 t[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) t[e] = (c * 8 + e < p.K) ? src[e] : __float2bfloat16_rn(0.f);
          v = *reinterpret_cast<const uint4*>(t);
        }
      }
      const int dst = (WK == W_BF16) ? c * 8 : (c & 1) * (p.Kp >> 1) + (c >> 1) * 8;
      *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(xs) + bm * p.Kp + dst) = v;
    }
  }
  named_bar_sync(1, kBulkWarps * 32);

  // Every consumer warp waits on every chunk in ring order and arrives once on
  // its empty barrier, so no warp can ever test a slot's parity two phases
  // ahead.  Warp w reduces row w of the chunk.
  for (int ch = 0; ch < nchunks; ++ch) {
    const int s = ch % ns, k = ch / ns;
    if (!mbar_wait_bounded(full + s, k & 1)) {
      record_status(SN_ERR_TIMEOUT);
      break;
    }
    const int cnt = min(rs, nrows - ch * rs);
    const bool has_row = warp < cnt;
    const uint4* wr = reinterpret_cast<const uint4*>(slots + static_cast<size_t>(s) * sh.slot_bytes +
                                                     static_cast<size_t>(warp) * row_bytes);
    const int row = r0 + ch * rs + warp;
    const int b = row / p.N, n = row - b * p.N;
    const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(xs) + static_cast<size_t>(b - b0) * MT * p.Kp;
    float2 acc[MT][2];
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m][0] = acc[m][1] = make_float2(0.f, 0.f);
    if (has_row) {
      constexpr int U = Batch<WK, MT>::U;
      for (int base = lane; base < nck; base += 32 * U) {
        // issue every load of the batch, then the arithmetic
        uint4 wv[U];
        uint4 xv[U][MT][2];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int idx = base + 32 * u;
          const bool ok = idx < nck;
          wv[u] = ok ? wr[idx] : make_uint4(0, 0, 0, 0);
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            xv[u][m][0] = ok ? *reinterpret_cast<const uint4*>(xb + m * p.Kp + idx * 8) : make_uint4(0, 0, 0, 0);
            if constexpr (Batch<WK, MT>::XW == 2)
              xv[u][m][1] = ok ? *reinterpret_cast<const uint4*>(xb + m * p.Kp + (p.Kp >> 1) + idx * 8)
                               : make_uint4(0, 0, 0, 0);
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) chunk_fma2_x<WK, MT>(wv[u], xv[u], acc);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty + s);
    if (has_row) {
      void* yb = reinterpret_cast<uint8_t*>(p.y) + static_cast<int64_t>(b) * p.sy * (p.y_f32 ? 4 : 2);
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        const float v = warp_sum((acc[m][0].x + acc[m][1].x) + (acc[m][0].y + acc[m][1].y));
        if (lane == 0) {
          float o = v;
          if constexpr (WK != W_BF16) o *= p.scale[static_cast<int64_t>(b) * p.sS + n];
          store_row<MT>(p, yb, n, m, o);
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Tensor-core decode GEMV (bf16, int8 or e4m3 weights; grid.y = batch entry).
//
// The same bulk-copy ring as gemv_bulk_kernel, but the tensor core does the
// dot products, so the CUDA cores issue almost nothing per weight byte and a
// ring slot is released as soon as its MMAs retire.
//
// A slot holds R whole weight rows back to back (row r at r * K * esz bytes).
// Each row is cut into S segments of L = K * esz / S bytes, and the R * S = 16
// segments are the sixteen 8-row groups of an M = 128 A operand in the
// no-swizzle K-major layout: group g = r * S + s starts at g * L bytes
// (stride byte offset = L), and inside a group the eight 16-byte "rows" are
// eight consecutive 16-byte pieces of the segment, the second K half of each
// MMA 128 bytes further on (leading byte offset).  One MMA (K = 16 bf16 or
// K = 32 int8) therefore consumes 256 consecutive bytes of every segment, and
// L / 256 MMAs consume the slot.
//
// x is the B operand, laid out the same way: B group G = (d * MT + m) * S + s
// is segment s of x row m (digit plane d for int8).  Then
//   D[lane 8g + j][column 8G + j] = sum over that segment piece of W * x
// whenever g and G name the same segment s; y[row r, m] is the sum of those
// entries over (s, j).  The epilogue reads them with one TMEM load per x row
// and digit (lane l of the warp takes column l mod 8S) and a shuffle
// reduction over the 8S lanes of a weight row.  The MMA computes
// N = 8 * S * MT * digits columns where MT * digits are needed; the tensor
// core has room for that at HBM speed.
//
// bf16: x staged once by one bulk copy per row, kind::f16, fp32 in TMEM.
// int8: the int8 codes feed kind::i8 directly (no conversion on the CUDA
// cores).  x row m is rounded once to the integer X = rint(x * 2^e_m) with
// max|X| in [2^21, 2^22) and split into three signed base-256 digits, each an
// int8 plane of B; TMEM holds three exact s32 partial sums per row, combined
// in 64-bit integers: y = (sum_k q_k X_k) * 2^-e_m * scale_row.  The only
// approximation is the rounding of x to 22 significant bits (absolute error
// at most 2^-23 of max|x| per element).
// e4m3: the codes feed kind::f8f6f4 directly.  x row m is scaled by 2^e_m
// (max in [2^7, 2^8)) and written as the sum of two e4m3 terms t1 = rn(x),
// t2 = rn(x - t1): exact for every element of at least 2^-2 (bf16 has 8
// significant bits, e4m3 4), absolute error at most 2^-10 below that (2^-17
// of max|x|).  Two B planes, products exact, fp32 accumulation in TMEM.
// An x row holding inf or NaN gives NaN outputs on both 8-bit paths.
//
// Warps: 0 = weight producer (no griddepcontrol.wait: weights are frozen),
// 1 = TMEM owner and MMA issuer (bf16: also the x copy), 2..5 = epilogue
// (TMEM lane quarter = warp % 4; int8: also the x digits).  Up to four
// accumulators in TMEM let the epilogue lag the MMAs by several slots.
// ---------------------------------------------------------------------------
constexpr int kMmaGemvThreads = 192;
constexpr int kAccMax = 4;  // TMEM accumulators: the MMAs of slot t wait for the epilogue of slot t - nacc

struct MmaShape {
  int ns;              // ring slots
  int N;               // MMA N = 8 * S * MT * digits
  int acc_log2;        // log2 of the TMEM accumulators (0, 1 or 2)
  uint32_t slot_bytes; // R * K * esz
  uint32_t xs_off;     // byte offset of the B operand (x, or x digits)
  uint32_t xraw_off;   // int8: byte offset of x as copied (bf16 [MT][K])
  uint32_t ring_off;   // byte offset of slot 0
  uint32_t tcols;      // TMEM columns allocated
  int q, rem;          // rows per CTA: q, one more for the first rem CTAs of grid.x
};

// v[idx] for a lane-dependent idx without local-memory indexing.
template <int W>
__device__ __forceinline__ float pick(const float (&v)[W], int idx) {
  float t[W];
#pragma unroll
  for (int i = 0; i < W; ++i) t[i] = v[i];
#pragma unroll
  for (int w = W / 2; w >= 1; w >>= 1) {
    const bool hi = (idx & w) != 0;
#pragma unroll
    for (int i = 0; i < w; ++i) t[i] = hi ? t[i + w] : t[i];
  }
  return t[0];
}

// This lane's diagonal entry of the 8S TMEM columns starting at taddr.
template <int S>
__device__ __forceinline__ float diag_entry(uint32_t taddr, int lane) {
  if constexpr (S == 2) {
    float t[16];
    tc::tmem_ld16(taddr, t);
    return pick<16>(t, lane & 15);
  } else {
    float t[32];
    tc::tmem_ld32(taddr, t);
    return pick<32>(t, lane);
  }
}

// This lane's diagonal entries of ND blocks of 8S TMEM columns (one per B
// plane, starting at ta[d]), with the ND loads in flight together and one wait.
template <int S, int ND>
__device__ __forceinline__ void diag_entries(const uint32_t (&ta)[ND], int lane, float (&out)[ND]) {
  constexpr int W = 8 * S;
  uint32_t r[ND][W];
#pragma unroll
  for (int d = 0; d < ND; ++d) {
    if constexpr (S == 1)
      tc::tmem_ld8_async(ta[d], r[d]);
    else if constexpr (S == 2)
      tc::tmem_ld16_async(ta[d], r[d]);
    else
      tc::tmem_ld32_async(ta[d], r[d]);
  }
  tc::tmem_wait_ld();
#pragma unroll
  for (int d = 0; d < ND; ++d) {
    float t[W];
#pragma unroll
    for (int i = 0; i < W; ++i) {
      tc::tmem_reg_fence(r[d][i]);
      t[i] = __uint_as_float(r[d][i]);
    }
    out[d] = pick<W>(t, lane & (W - 1));
  }
}

// The next GEMV's weights are frozen too: while this kernel's last weight
// copies are in flight, HBM reads the first bytes of every CTA range of the
// next launch into L2, so that the next kernel's first ring fills hit L2 and
// HBM is not idle across the kernel boundary.  One thread per CTA; ranges
// are dealt out round-robin over this launch's CTAs.
__device__ __forceinline__ void prefetch_next_weights(const GemvParams& p) {
  constexpr uint32_t kPiece = 32 * 1024;
  const int nblk = static_cast<int>(gridDim.x * gridDim.y);
  for (int j = static_cast<int>(blockIdx.y * gridDim.x + blockIdx.x); j < p.pf_parts; j += nblk) {
    // the next launch's CTA j owns rows [a, b) (its division-free split)
    const int64_t a = static_cast<int64_t>(j) * p.pf_q + min(j, p.pf_rem);
    const int64_t b = a + p.pf_q + (j < p.pf_rem ? 1 : 0);
    const int64_t bytes = min(static_cast<int64_t>(p.pf_part_bytes), (b - a) * p.pf_row_bytes);
    if (p.pf_ld == static_cast<int64_t>(p.pf_row_bytes)) {
      const uint8_t* src = p.pf + a * p.pf_ld;
      for (int64_t o = 0; o < bytes; o += kPiece)
        bulk_prefetch_l2(src + o, static_cast<uint32_t>(min(static_cast<int64_t>(kPiece), bytes - o)));
    } else {
      for (int64_t r = a, left = bytes; left > 0; ++r, left -= p.pf_row_bytes)
        bulk_prefetch_l2(p.pf + r * p.pf_ld, static_cast<uint32_t>(min(static_cast<int64_t>(p.pf_row_bytes), left)));
    }
  }
}

// 16-byte x pieces an 8-bit kernel's staging thread may hold in registers
// (then no shared-memory copy of x: K <= 1024 * kXRegs / MT).
constexpr int kXRegs = 8;

// 16-byte load cached in L2 only: x is written by the previous kernel, and
// this SM's L1 may hold lines of the same buffer from an earlier launch.
__device__ __forceinline__ uint4 ld_cg_v4(const void* ptr) {
  uint4 r;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(ptr));
  return r;
}

// One x row that every CTA of the launch copies at the same moment (when
// the dependency resolves): CTA c starts at 128-byte piece `rot` of the row
// and wraps around, so the CTAs' requests spread over the L2 slices instead
// of queuing on the same lines in the same order.  src, dst and bytes are
// multiples of 16.  Used where an 8-bit kernel stages x through shared
// memory (K * M beyond the staging registers): measured when every 8-bit x
// row went that way, int8 / e4m3 in_proj chains -1.5% / -2%.  The bf16
// kernel keeps one copy per row (the second copy cost it +0.8%, config 2
// +0.7%).
__device__ __forceinline__ void bulk_g2s_rot(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol,
                                             uint32_t rot) {
  const uint32_t pieces = bytes / 128;
  const uint32_t off = (bytes % 128 == 0 && pieces > 1) ? (rot % pieces) * 128 : 0;
  if (off == 0) {
    bulk_g2s(dst, src, bytes, bar, pol);
    return;
  }
  bulk_g2s(static_cast<uint8_t*>(dst) + off, static_cast<const uint8_t*>(src) + off, bytes - off, bar, pol);
  bulk_g2s(dst, src, off, bar, pol);
}

// ---- x staging of the 8-bit kinds (shared by gemv_mma_kernel's staging
// threads and the chain's x loader) ----
// max |x| of a 16-byte bf16 piece, as a bit pattern (non-negative bf16 values
// order like their patterns)
__device__ __forceinline__ uint32_t x8_piece_max(uint4 v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t mx = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) mx = max(mx, max(w[j] & 0x7FFFu, (w[j] >> 16) & 0x7FFFu));
  return mx;
}
// Scale of an x row with max |x| pattern mx: max|x| < 2^(E+1), E = biased
// exponent - 127 (subnormal rows too: E = -127); 2^e with e = 21 - E (int8)
// or 7 - E (e4m3), returned as two exact power-of-two factors (e in
// [-107, 148]); INT_MIN for a row holding inf or NaN.
template <int WK>
__device__ __forceinline__ int x8_row_scale(uint32_t mx, float& up1, float& up2) {
  const int ebits = static_cast<int>(mx >> 7);
  const int e = (WK == W_INT8 ? 21 : 7) - (ebits - 127);
  up1 = __uint_as_float(static_cast<uint32_t>(127 + e / 2) << 23);
  up2 = __uint_as_float(static_cast<uint32_t>(127 + (e - e / 2)) << 23);
  return (ebits == 255) ? INT_MIN : e;
}
// The ND B-operand planes of 16-byte piece c of x row m (planes[(d * MT + m)
// * K + 8c ...]): three signed base-256 digits of rint(x * 2^e) (int8), or
// the two e4m3 terms t1 = rn(x 2^e), t2 = rn(x 2^e - t1).
template <int WK, int MT>
__device__ __forceinline__ void x8_emit(uint8_t* planes, int K, int m, int c, uint4 v, float up1, float up2) {
  constexpr int ND = (WK == W_INT8) ? 3 : 2;
  uint32_t dg[ND][2] = {};
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const uint32_t h = w[e >> 1];
    const float xf = (e & 1) ? bf16hi(h) : bf16lo(h);
    const float xsc = (xf * up1) * up2;
    uint32_t b[ND];
    if constexpr (WK == W_INT8) {
      int X = __float2int_rn(xsc);  // |X| < 2^22
      const int d0 = static_cast<int8_t>(X & 0xFF);
      X = (X - d0) >> 8;
      const int d1 = static_cast<int8_t>(X & 0xFF);
      const int d2 = (X - d1) >> 8;  // |d2| <= 64
      b[0] = static_cast<uint32_t>(d0) & 0xFFu;
      b[1] = static_cast<uint32_t>(d1) & 0xFFu;
      b[2] = static_cast<uint32_t>(d2) & 0xFFu;
    } else {
      // |xsc| < 2^8: no saturation; t1 + t2 reproduces xsc to 2^-10
      const __nv_fp8_storage_t t1 = __nv_cvt_float_to_fp8(xsc, __NV_SATFINITE, __NV_E4M3);
      const float r = xsc - __half2float(__half(__nv_cvt_fp8_to_halfraw(t1, __NV_E4M3)));
      const __nv_fp8_storage_t t2 = __nv_cvt_float_to_fp8(r, __NV_SATFINITE, __NV_E4M3);
      b[0] = t1;
      b[1] = t2;
    }
#pragma unroll
    for (int d = 0; d < ND; ++d) dg[d][e >> 2] |= b[d] << (8 * (e & 3));
  }
#pragma unroll
  for (int d = 0; d < ND; ++d)
    *reinterpret_cast<uint2*>(planes + (static_cast<size_t>(d) * MT + m) * K + c * 8) = make_uint2(dg[d][0], dg[d][1]);
}
// x_m . w of an 8-bit row from its TMEM sums: int8 -- the three digit sums
// combined exactly in 64 bits, times 2^-e in double, rounded once to fp32;
// e4m3 -- the fp32 sum (v[0]) times 2^-e.  NaN when x row m was non-finite.
template <int WK, int ND>
__device__ __forceinline__ float x8_dot(const int (&v)[ND], int e) {
  if (e == INT_MIN) return __int_as_float(0x7FC00000);
  const double inv = __longlong_as_double(static_cast<long long>(1023 - e) << 52);
  if constexpr (WK == W_INT8) {
    const long long acc = static_cast<long long>(v[0]) + (static_cast<long long>(v[1]) << 8) +
                          (static_cast<long long>(v[2]) << 16);
    return static_cast<float>(static_cast<double>(acc) * inv);
  } else {
    return static_cast<float>(static_cast<double>(__int_as_float(v[0])) * inv);
  }
}

// Fused normalisation of the bf16 GEMV's x rows (the decode step's gated
// RMSNorm before out_proj and add + LayerNorm before in_proj / qkv / fc1):
// the 128 staging threads of every CTA load the row(s) (16-byte pieces from
// L2), reduce over the row through shared memory and write the normalised
// bf16 row where the plain kernel's bulk copy would have put x.  Same
// arithmetic as rmsnorm_gated_kernel / layer_norm_kernel (fp32, one bf16
// rounding); only the order of the row sums differs.  K % 1024 == 0,
// K <= 4096 (host-checked).
template <int MT>
__device__ __forceinline__ void stage_x_norm(const GemvParams& p, const __nv_bfloat16* xb, uint8_t* xs, float* red) {
  constexpr int kMaxPieces = 4;  // 16-byte pieces a thread holds per row (K <= 4096)
  const int xt = threadIdx.x - 64;  // 0..127 (warps 2-5)
  const int wq = xt >> 5, ln = xt & 31;
  const int np = p.K / 1024;       // pieces per thread
  const bool writer = p.xn_rout != nullptr && blockIdx.x == 0 && blockIdx.y == 0;
  auto block_sum = [&](float v) {
    v = warp_sum(v);
    if (ln == 0) red[wq] = v;
    named_bar_sync(3, 128);
    const float t = red[0] + red[1] + red[2] + red[3];
    named_bar_sync(3, 128);  // red reusable
    return t;
  };
  for (int m = 0; m < MT; ++m) {
    uint4* dst = reinterpret_cast<uint4*>(xs + static_cast<size_t>(m) * p.K * 2);
    if (m >= p.M) {
      for (int c = xt; c < p.K / 8; c += 128) dst[c] = make_uint4(0, 0, 0, 0);
      continue;
    }
    float t[kMaxPieces][8];
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxPieces; ++j) {
      if (j >= np) break;
      const int c = xt + 128 * j;
      const uint4 xv = ld_cg_v4(xb + m * p.ldx + c * 8);
      uint4 av = make_uint4(0, 0, 0, 0);
      if (p.xn_aux) av = ld_cg_v4(p.xn_aux + m * p.ldx + c * 8);
      const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w}, aw[4] = {av.x, av.y, av.z, av.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float xf = (e & 1) ? bf16hi(xw[e >> 1]) : bf16lo(xw[e >> 1]);
        const float af = (e & 1) ? bf16hi(aw[e >> 1]) : bf16lo(aw[e >> 1]);
        float v;
        if (p.xn == SN_NORM_RMS_GATED) {
          v = p.xn_aux ? xf * (af / (1.0f + expf(-af))) : xf;
          acc = fmaf(v, v, acc);
        } else {
          v = xf + af;
          acc += v;
        }
        t[j][e] = v;
      }
      if (writer) {
        uint32_t o[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(t[j][2 * q]));
          const uint32_t hi = __bfloat16_as_ushort(__float2bfloat16_rn(t[j][2 * q + 1]));
          o[q] = lo | (hi << 16);
        }
        *reinterpret_cast<uint4*>(p.xn_rout + m * p.ldx + c * 8) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    float mean = 0.f, r;
    if (p.xn == SN_NORM_RMS_GATED) {
      r = rsqrtf(block_sum(acc) / p.K + p.xn_eps);
    } else {
      mean = block_sum(acc) / p.K;
      float sq = 0.f;
#pragma unroll
      for (int j = 0; j < kMaxPieces; ++j) {
        if (j >= np) break;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float d = t[j][e] - mean;
          sq = fmaf(d, d, sq);
        }
      }
      r = rsqrtf(block_sum(sq) / p.K + p.xn_eps);
    }
#pragma unroll
    for (int j = 0; j < kMaxPieces; ++j) {
      if (j >= np) break;
      const int c = xt + 128 * j;
      const uint4 wv = *reinterpret_cast<const uint4*>(p.xn_w + c * 8);
      uint4 bv = make_uint4(0, 0, 0, 0);
      if (p.xn_b) bv = *reinterpret_cast<const uint4*>(p.xn_b + c * 8);
      const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w}, bw[4] = {bv.x, bv.y, bv.z, bv.w};
      uint32_t o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float f[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int e = 2 * q + h;
          const float wf = h ? bf16hi(ww[q]) : bf16lo(ww[q]);
          float o1 = (p.xn == SN_NORM_RMS_GATED) ? t[j][e] * r * wf : (t[j][e] - mean) * r * wf;
          if (p.xn_b) o1 += h ? bf16hi(bw[q]) : bf16lo(bw[q]);
          f[h] = o1;
        }
        o[q] = static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(f[0]))) |
               (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(f[1]))) << 16);
      }
      dst[c] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

template <int WK, int MT, int S>
__global__ void __launch_bounds__(kMmaGemvThreads, 2) gemv_mma_kernel(const GemvParams p, const MmaShape sh) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int R = 16 / S;
  constexpr int G = 8 * S;  // TMEM lanes (and columns) per weight row
  constexpr int ESZ = WT<WK>::ESZ;
  constexpr int ND = (WK == W_INT8) ? 3 : (WK == W_E4M3) ? 2 : 1;  // B planes per x row
  const int ns = sh.ns;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + ns;
  uint64_t* tfull = empty + ns;
  uint64_t* tempty = tfull + kAccMax;
  uint64_t* done = tempty + kAccMax;
  uint64_t* xbar = done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xbar + 1);
  uint32_t* xmax = tmem_slot + 1;            // int8: [MT] max |x| (bf16 bit patterns)
  int* xexp = reinterpret_cast<int*>(xmax + MT);  // int8: [MT] e_m (x row m scaled by 2^e_m)
  uint8_t* xs = smem + sh.xs_off;
  uint8_t* ring = smem + sh.ring_off;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // batch entry blockIdx.y (independent W, x, y, scale); rows split over blockIdx.x
  const uint8_t* Wb = p.W + static_cast<int64_t>(blockIdx.y) * p.sW * ESZ;
  const __nv_bfloat16* xb = p.x + static_cast<int64_t>(blockIdx.y) * p.sx;
  void* yb = reinterpret_cast<uint8_t*>(p.y) + static_cast<int64_t>(blockIdx.y) * p.sy * (p.y_f32 ? 4 : 2);
  const float* sb = (WK != W_BF16) ? p.scale + static_cast<int64_t>(blockIdx.y) * p.sS : nullptr;
  // rows of this CTA without a division (a run-time division costs the
  // single-threaded producer and MMA issuer ~0.1 us each at launch)
  const int bx = static_cast<int>(blockIdx.x);
  const int r0 = bx * sh.q + min(bx, sh.rem);
  const int r1 = r0 + sh.q + (bx < sh.rem ? 1 : 0);
  const int nrows = r1 - r0;
  const uint32_t row_bytes = static_cast<uint32_t>(p.K) * ESZ;
  const int ntiles = (nrows + R - 1) / R;
  const int nacc = 1 << sh.acc_log2;
  uint32_t tmem = 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ns; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);  // released by the MMA commit
    }
    for (int b = 0; b < kAccMax; ++b) {
      mbar_init(tfull + b, 1);
      mbar_init(tempty + b, 4);  // one arrive per epilogue warp
    }
    mbar_init(done, 1);
    mbar_init(xbar, 1);
    for (int m = 0; m < MT; ++m) xmax[m] = 0;
    fence_barrier_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == 0) {
    // ---------------- producer: weights only, so no griddepcontrol.wait ----
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      if (p.pf != nullptr && p.pf_lead <= -2) prefetch_next_weights(p);  // before this CTA's own copies
      int t = 0, s = 0, k = 0;  // tile, its slot (t mod ns) and round (t / ns), kept incrementally
      for (; t < ntiles; ++t, s = (s + 1 == ns) ? 0 : s + 1, k += (s == 0)) {
        if (k > 0 && !mbar_wait_bounded(empty + s, (k - 1) & 1)) {
          record_status(SN_ERR_TIMEOUT);
          break;
        }
        const int first = r0 + t * R;
        const int cnt = min(R, r1 - first);
        uint8_t* dst = ring + static_cast<size_t>(s) * sh.slot_bytes;
        mbar_arrive_expect_tx(full + s, static_cast<uint32_t>(cnt) * row_bytes);
        if (p.ldw == p.K) {
          bulk_g2s(dst, Wb + static_cast<int64_t>(first) * p.ldw * ESZ, static_cast<uint32_t>(cnt) * row_bytes,
                   full + s, pol);
        } else {
          for (int r = 0; r < cnt; ++r)
            bulk_g2s(dst + static_cast<size_t>(r) * row_bytes, Wb + static_cast<int64_t>(first + r) * p.ldw * ESZ,
                     row_bytes, full + s, pol);
        }
      }
      if (t < ntiles) {  // error path: let the copies in flight land before exit
        for (int j = (t > ns ? t - ns : 0); j < t; ++j) mbar_wait_bounded(full + j % ns, (j / ns) & 1);
      } else if (p.pf != nullptr && p.pf_lead > -2) {
        // once this CTA's own reads are (nearly) all served: wait until tile
        // ntiles - 1 - lead has landed (lead < ns, so its slot was not reused)
        const int lead = min(p.pf_lead, ns - 1);
        const int j = ntiles - 1 - lead;
        if (lead < 0 || j < 0 || mbar_wait_bounded(full + j % ns, (j / ns) & 1)) prefetch_next_weights(p);
      }
    }
  } else {
    // TMEM (warp 1) and the x staging overlap the first weight copies; the
    // producer never waits for either.
    if (warp == 1) tc::tmem_alloc(tmem_slot, sh.tcols);
    pdl_wait();  // x and y belong to the previous kernel from here on
    const int cpr = p.K >> 3;  // 16-byte pieces of a bf16 x row
    if constexpr (WK == W_BF16) {
      if (p.xn != 0) {
        // x rows normalised by the staging warps; one arrival completes xbar
        if (warp >= 2) {
          stage_x_norm<MT>(p, xb, xs, reinterpret_cast<float*>(smem + 768));
          tc::fence_proxy_async_smem();
          named_bar_sync(3, 128);
          if (threadIdx.x == 64) mbar_arrive(xbar);
        }
      } else if (warp == 1) {
        // x rows by bulk copy (one L2 round trip); padding rows zeroed meanwhile
        if (lane == 0) {
          const uint64_t pol = l2_policy_evict_normal();
          mbar_arrive_expect_tx(xbar, static_cast<uint32_t>(p.M) * row_bytes);
          for (int m = 0; m < p.M; ++m)
            bulk_g2s(xs + static_cast<size_t>(m) * row_bytes, xb + m * p.ldx, row_bytes, xbar, pol);
        }
      } else if (MT > 1) {
        for (int i = threadIdx.x - 64 + p.M * cpr; i < MT * cpr; i += 128)
          reinterpret_cast<uint4*>(xs)[i] = make_uint4(0, 0, 0, 0);
        tc::fence_proxy_async_smem();
      }
    } else {
      // x rows, then the B planes of x * 2^e_m: three int8 digits of
      // rint(x * 2^e_m), or two e4m3 terms.  When every 16-byte piece a
      // staging thread needs fits in kXRegs registers, the pieces are loaded
      // straight into registers (no staging copy in shared memory, which
      // leaves room for one more ring slot); otherwise one bulk copy per row.
      if (warp >= 2) {
        const int xt = threadIdx.x - 64;  // 0..127
        auto row_max = [&](int m, uint32_t mx) {
          mx = __reduce_max_sync(0xffffffffu, mx);
          if (lane == 0) atomicMax(xmax + m, mx);
        };
        auto row_scale = [&](int m, float& up1, float& up2) {
          const int e = x8_row_scale<WK>(xmax[m], up1, up2);
          if (xt == 0) xexp[m] = e;
        };
        auto emit = [&](int m, int c, uint4 v, float up1, float up2) { x8_emit<WK, MT>(xs, p.K, m, c, v, up1, up2); };
        auto piece_max = [](uint4 v) { return x8_piece_max(v); };
        if (sh.xraw_off == 0) {
          constexpr int PPR = kXRegs / MT;  // pieces per row a thread holds (host: cpr <= 128 * PPR)
          uint4 xv[MT][PPR];
#pragma unroll
          for (int m = 0; m < MT; ++m)
#pragma unroll
            for (int j = 0; j < PPR; ++j) {
              const int c = xt + 128 * j;
              xv[m][j] = (m < p.M && c < cpr) ? ld_cg_v4(xb + m * p.ldx + c * 8) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            uint32_t mx = 0;
#pragma unroll
            for (int j = 0; j < PPR; ++j) mx = max(mx, piece_max(xv[m][j]));
            row_max(m, mx);
          }
          named_bar_sync(2, 128);
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            float up1, up2;
            row_scale(m, up1, up2);
#pragma unroll
            for (int j = 0; j < PPR; ++j)
              if (xt + 128 * j < cpr) emit(m, xt + 128 * j, xv[m][j], up1, up2);
          }
        } else {
          const __nv_bfloat16* xraw = reinterpret_cast<const __nv_bfloat16*>(smem + sh.xraw_off);
          if (xt == 0) {
            const uint64_t pol = l2_policy_evict_normal();
            mbar_arrive_expect_tx(xbar, static_cast<uint32_t>(p.M) * p.K * 2);
            for (int m = 0; m < p.M; ++m)
              bulk_g2s_rot(const_cast<__nv_bfloat16*>(xraw) + m * p.K, xb + m * p.ldx, p.K * 2, xbar, pol,
                           p.x_rot ? blockIdx.x + m : 0);
          }
          if (!__all_sync(0xffffffffu, mbar_wait_bounded(xbar, 0))) record_status(SN_ERR_TIMEOUT);
          const uint4* xr = reinterpret_cast<const uint4*>(xraw);
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            uint32_t mx = 0;
            if (m < p.M)
              for (int c = xt; c < cpr; c += 128) mx = max(mx, piece_max(xr[m * cpr + c]));
            row_max(m, mx);
          }
          named_bar_sync(2, 128);
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            float up1, up2;
            row_scale(m, up1, up2);
            for (int c = xt; c < cpr; c += 128)
              emit(m, c, m < p.M ? xr[m * cpr + c] : make_uint4(0, 0, 0, 0), up1, up2);
          }
        }
        tc::fence_proxy_async_smem();
      }
    }
    tc::fence_before_sync();
    named_bar_sync(1, 160);  // warps 1..5: TMEM allocated, x staged (bf16: copy issued)
    tc::fence_after_sync();
    tmem = *tmem_slot;

    const uint32_t L = row_bytes / S;  // segment bytes = stride between 8-row groups
    const uint32_t nk = L / 256;       // MMAs per slot
    if (warp == 1) {
      // ---------------- MMA issuer ----------------
      if (lane == 0) {
        const uint32_t idesc = (WK == W_INT8)   ? tc::idesc_s8_s32(128, sh.N)
                               : (WK == W_E4M3) ? tc::idesc_e4m3_f32(128, sh.N)
                                                : tc::idesc_bf16_f32(128, sh.N);
        const uint64_t db0 = tc::smem_desc_noswz(xs, 128, L);
        bool x_ok = true;
        if constexpr (WK == W_BF16) x_ok = mbar_wait_bounded(xbar, 0);
        if (!x_ok) record_status(SN_ERR_TIMEOUT);
        for (int t = 0, s = 0, ph = 0; t < ntiles && x_ok; ++t, s = (s + 1 == ns) ? 0 : s + 1, ph ^= (s == 0)) {
          const int b = t & (nacc - 1);
          if (!mbar_wait_bounded(full + s, ph) ||
              (t >= nacc && !mbar_wait_bounded(tempty + b, ((t >> sh.acc_log2) - 1) & 1))) {
            record_status(SN_ERR_TIMEOUT);
            break;
          }
          tc::fence_after_sync();
          const uint64_t da0 = tc::smem_desc_noswz(ring + static_cast<size_t>(s) * sh.slot_bytes, 128, L);
          const uint32_t d = tmem + static_cast<uint32_t>(b * sh.N);
          for (uint32_t k = 0; k < nk; ++k) {  // 256 bytes of every segment per MMA
            if constexpr (WK == W_INT8)
              tc::mma_s8(d, da0 + 16 * k, db0 + 16 * k, idesc, k != 0);
            else if constexpr (WK == W_E4M3)
              tc::mma_e4m3(d, da0 + 16 * k, db0 + 16 * k, idesc, k != 0);
            else
              tc::mma_bf16(d, da0 + 16 * k, db0 + 16 * k, idesc, k != 0);
          }
          tc::mma_commit(empty + s);
          tc::mma_commit(tfull + b);
        }
        tc::mma_commit(done);
        if (!mbar_wait_bounded(done, 0)) record_status(SN_ERR_TIMEOUT);
      }
      __syncwarp();
    } else {
      // ---------------- epilogue ----------------
      const int q = warp & 3;
      const int i = q * 32 + lane;  // A row = TMEM lane
      const int r = i / G;          // weight row inside the slot
      // 8-bit row scales are frozen weights: fetch slot t + 1's while slot t computes
      float rs_next = 0.f;
      if constexpr (WK != W_BF16) rs_next = (r < min(R, nrows)) ? sb[r0 + r] : 0.f;
      for (int t = 0; t < ntiles; ++t) {
        const int b = t & (nacc - 1);
        const int first = r0 + t * R;
        const int cnt = min(R, r1 - first);
        float rs = 0.f;
        if constexpr (WK != W_BF16) {
          rs = rs_next;
          if (t + 1 < ntiles) rs_next = (r < min(R, nrows - (t + 1) * R)) ? sb[first + R + r] : 0.f;
        }
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(tfull + b, (t >> sh.acc_log2) & 1))) {
          record_status(SN_ERR_TIMEOUT);
          break;
        }
        tc::fence_after_sync();
        const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) + b * sh.N;
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          if constexpr (WK == W_BF16) {
            float v = diag_entry<S>(taddr + m * G, lane);
#pragma unroll
            for (int o = G / 2; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if ((lane & (G - 1)) == 0 && r < cnt) store_row<MT>(p, yb, first + r, m, v);
          } else if constexpr (WK == W_E4M3) {
            float v = 0.f;
#pragma unroll
            for (int d = 0; d < ND; ++d) v += diag_entry<S>(taddr + (d * MT + m) * G, lane);
#pragma unroll
            for (int o = G / 2; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if ((lane & (G - 1)) == 0 && r < cnt) {
              const int e = xexp[m];
              const float dot = (e == INT_MIN) ? __int_as_float(0x7FC00000)
                                               : static_cast<float>(static_cast<double>(v) *
                                                                    __longlong_as_double(static_cast<long long>(1023 - e) << 52));
              store_row<MT>(p, yb, first + r, m, dot * rs);
            }
          } else {
            int v[3];
#pragma unroll
            for (int d = 0; d < 3; ++d) {
              v[d] = __float_as_int(diag_entry<S>(taddr + (d * MT + m) * G, lane));
#pragma unroll
              for (int o = G / 2; o >= 1; o >>= 1) v[d] += __shfl_xor_sync(0xffffffffu, v[d], o);
            }
            if ((lane & (G - 1)) == 0 && r < cnt) {
              const long long acc = static_cast<long long>(v[0]) + (static_cast<long long>(v[1]) << 8) +
                                    (static_cast<long long>(v[2]) << 16);
              const int e = xexp[m];
              // sum_k q_k X_k exactly, times 2^-e (exact in double), rounded once to fp32
              const float dot = (e == INT_MIN)
                                    ? __int_as_float(0x7FC00000)
                                    : static_cast<float>(static_cast<double>(acc) *
                                                         __longlong_as_double(static_cast<long long>(1023 - e) << 52));
              store_row<MT>(p, yb, first + r, m, dot * rs);
            }
          }
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty + b);
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) tc::tmem_dealloc(tmem, sh.tcols);
}

// Opt a kernel into more than 48 KB of dynamic shared memory, once per
// (kernel, device); the table is keyed by the kernel's address.
inline bool ensure_smem(const void* kern, size_t bytes) {
  if (bytes <= 48 * 1024) return true;
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, size_t> done;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  std::lock_guard<std::mutex> lock(mu);
  auto key = std::make_pair(kern, dev);
  auto it = done.find(key);
  if (it != done.end() && it->second >= bytes) return true;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)) !=
      cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  // carve the unified L1/shared array for shared memory, so that two CTAs
  // (this kernel's and the next PDL-launched one's) can be resident per SM
  if (cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
    cudaGetLastError();
  done[key] = bytes;
  return true;
}

// Kernel selection override for measurement:
// SONATA_GEMV_KERNEL = mma (default) | bulk | regs.
int gemv_kernel_choice() {
  static int v = [] {
    const char* e = getenv("SONATA_GEMV_KERNEL");
    if (e && strcmp(e, "regs") == 0) return 2;
    if (e && strcmp(e, "bulk") == 0) return 1;
    return 0;
  }();
  return v;
}

template <typename Kern>
int launch_gemv(Kern kern, const GemvParams& p, int rows_per_cta, int batch, size_t smem, cudaStream_t st,
                bool pdl) {
  if (!ensure_smem(reinterpret_cast<const void*>(kern), smem)) return SN_ERR_UNSUPPORTED;
  dim3 grid((p.N + rows_per_cta - 1) / rows_per_cta, batch);
  return launch(kern, grid, dim3(kThreads), smem, st, pdl, p);
}

// Shared-memory budget of one bulk-GEMV CTA (override: SONATA_GEMV_SMEM_KB).
// The default leaves room for two CTAs per SM (this GEMV and the next one).
size_t bulk_smem_budget() {
  static size_t v = [] {
    const char* e = getenv("SONATA_GEMV_SMEM_KB");
    long kb = e ? strtol(e, nullptr, 10) : 0;
    if (kb < 32 || kb > 220) kb = 110;
    return static_cast<size_t>(kb) * 1024;
  }();
  return v;
}

// Returns SN_ERR_UNSUPPORTED when the bulk kernel does not apply.
template <int WK, int MT>
int dispatch_bulk(const GemvParams& p, int batch, cudaStream_t st, bool pdl) {
  constexpr int ESZ = WT<WK>::ESZ;
  constexpr int EPC = WT<WK>::EPC;
  const uint32_t row_bytes = static_cast<uint32_t>(p.K) * ESZ;
  if (row_bytes % 16 != 0 || row_bytes > 64 * 1024) return SN_ERR_UNSUPPORTED;
  const int64_t total_rows = static_cast<int64_t>(batch) * p.N;
  if (total_rows >= (int64_t(1) << 31)) return SN_ERR_UNSUPPORTED;
  const int grid = static_cast<int>(std::min<int64_t>(sm_count(), total_rows));
  const int64_t rows_per_cta = (total_rows + grid - 1) / grid;
  BulkShape sh;
  sh.total_rows = static_cast<int>(total_rows);
  sh.contiguous = (p.ldw == p.K) && (batch == 1 || p.sW == static_cast<int64_t>(p.N) * p.ldw);
  // ~32 KB per bulk copy, one row per consumer warp
  sh.rs = static_cast<int>(std::max<uint32_t>(1, std::min<uint32_t>(kBulkWarps, (32u * 1024u) / row_bytes)));
  sh.rs = static_cast<int>(std::min<int64_t>(sh.rs, rows_per_cta));
  sh.slot_bytes = round_up_u32(static_cast<uint32_t>(sh.rs) * row_bytes, 128);
  const int ns_max = 16;
  sh.bar_bytes = round_up_u32(2 * ns_max * 8, 128);
  const int64_t span = std::min<int64_t>(batch, rows_per_cta / p.N + 2);
  sh.xs_bytes = round_up_u32(static_cast<uint32_t>(span * MT * p.Kp * XStage<WK>::BYTES), 128);
  const size_t budget = bulk_smem_budget();
  size_t room = budget > sh.bar_bytes + sh.xs_bytes ? budget - sh.bar_bytes - sh.xs_bytes : 0;
  int ns = static_cast<int>(std::min<size_t>(ns_max, room / sh.slot_bytes));
  const int64_t chunks_per_cta = (rows_per_cta + sh.rs - 1) / sh.rs;
  ns = static_cast<int>(std::min<int64_t>(ns, chunks_per_cta));
  ns = std::max(ns, 2);  // two slots even when that exceeds the budget (one CTA per SM then)
  sh.ns = ns;
  const size_t smem = sh.bar_bytes + sh.xs_bytes + static_cast<size_t>(sh.ns) * sh.slot_bytes;
  if (smem > 220 * 1024) return SN_ERR_UNSUPPORTED;
  auto kern = gemv_bulk_kernel<WK, MT>;
  if (!ensure_smem(reinterpret_cast<const void*>(kern), smem)) return SN_ERR_UNSUPPORTED;
  return launch(kern, dim3(grid), dim3(kBulkThreads), smem, st, pdl, p, sh);
}

// Segments per weight row of the tensor-core GEMV: the smallest S in {2, 4}
// whose segments are whole MMAs (K * esz / S a multiple of 256 bytes), whose
// slot of 16 / S rows stays within 32 KB and whose N = 8 * S * MT * digits
// fits one MMA (<= 256).  SONATA_GEMV_MMA_S forces 2 or 4 where valid.
int mma_segments(int K, int esz, int MT, int nd) {
  static int forced = [] {
    const char* e = getenv("SONATA_GEMV_MMA_S");
    const int v = e ? atoi(e) : 0;
    return (v == 2 || v == 4) ? v : 0;
  }();
  const int64_t row = static_cast<int64_t>(K) * esz;
  auto ok = [&](int S) { return row % (256 * S) == 0 && 8 * S * MT * nd <= 256; };
  auto small = [&](int S) { return (16 / S) * row <= 32 * 1024; };
  if (forced) return ok(forced) ? forced : 0;
  if (ok(2) && small(2)) return 2;
  if (ok(4)) return 4;  // smaller slots than S = 2 even when above 32 KB
  return ok(2) ? 2 : 0;
}

// Launch geometry of the tensor-core GEMV for an [N, K] weight of esz-byte
// elements with nd B planes per x row (MT x rows, `batch` weights along
// grid.y).  False when mma_segments finds no valid S.
struct MmaGrid {
  int S, cps, acc_log2, grid;
};
bool mma_grid(int esz, int nd, int MT, int N, int K, int batch, MmaGrid& g) {
  g.S = mma_segments(K, esz, MT, nd);
  if (g.S == 0) return false;
  const int n_mma = 8 * g.S * MT * nd;
  // CTAs per SM from the weight bytes each SM streams: up to one ring's worth
  // (~96 KB) one CTA, prefetched whole under programmatic dependent launch;
  // up to two rings' worth two CTAs; beyond that three, whose three rings
  // keep more bytes in flight than the next kernel's prefetch would
  // (measured per shape on B200).  SONATA_GEMV_CTAS_PER_SM overrides (1..4).
  static const int cps_env = [] {
    const char* e = getenv("SONATA_GEMV_CTAS_PER_SM");
    const int v = e ? atoi(e) : 0;
    return (v >= 1 && v <= 4) ? v : 0;
  }();
  const int64_t bytes_per_sm = static_cast<int64_t>(N) * K * esz * batch / sm_count();
  int cps = cps_env ? cps_env : bytes_per_sm <= 96 * 1024 ? 1 : bytes_per_sm <= 192 * 1024 ? 2 : 3;
  // TMEM: this kernel's CTAs and the next kernel's (programmatic dependent
  // launch) share an SM's 512 columns, so each CTA takes at most 512 / (2 cps)
  // (a CTA whose allocation does not fit would wait for another to exit)
  auto max_cols = [](int c) { return c == 1 ? 256 : c == 2 ? 128 : 64; };
  while (cps > 1 && static_cast<int>(tc::tmem_cols_for(n_mma)) > max_cols(cps)) --cps;
  auto acc_log2_for = [&](int c) {
    int a = 2;
    while (a > 0 && static_cast<int>(tc::tmem_cols_for(n_mma << a)) > max_cols(c)) --a;
    return a;
  };
  // at least two accumulators (the MMAs of a slot must not wait for the
  // previous slot's epilogue): fewer CTAs per SM rather than one accumulator
  while (cps > 1 && acc_log2_for(cps) == 0) --cps;
  g.cps = cps;
  g.acc_log2 = acc_log2_for(cps);
  g.grid = std::max(1, std::min(N, cps * sm_count() / batch));
  return true;
}

// Returns SN_ERR_UNSUPPORTED when the tensor-core GEMV does not apply
// (16-byte aligned rows, x rows and batch strides; K within mma_segments' rules).
template <int WK, int MT>
int dispatch_mma(const GemvParams& p, int batch, cudaStream_t st, bool pdl) {
  constexpr int ESZ = WT<WK>::ESZ;
  if (batch > 1 && ((p.sW * ESZ) % 16 != 0 || p.sx % 8 != 0)) return SN_ERR_UNSUPPORTED;
  constexpr int ND = (WK == W_INT8) ? 3 : (WK == W_E4M3) ? 2 : 1;
  if (!p.x_vec || (reinterpret_cast<uintptr_t>(p.W) & 15) || (p.ldw * ESZ) % 16 != 0) return SN_ERR_UNSUPPORTED;
  MmaGrid g;
  if (!mma_grid(ESZ, ND, MT, p.N, p.K, batch, g)) return SN_ERR_UNSUPPORTED;
  const int S = g.S, cps = g.cps, grid = g.grid;
  const int R = 16 / S;
  MmaShape sh;
  sh.N = 8 * S * MT * ND;
  sh.slot_bytes = static_cast<uint32_t>(R) * p.K * ESZ;
  sh.acc_log2 = g.acc_log2;
  sh.q = p.N / grid;
  sh.rem = p.N % grid;
  sh.tcols = tc::tmem_cols_for(sh.N << sh.acc_log2);
  const int rows_per_cta = (p.N + grid - 1) / grid;
  const int tiles_per_cta = (rows_per_cta + R - 1) / R;
  const int ns_max = 16;
  sh.xs_off = 1024;  // barriers, TMEM address and x scales below
  sh.xraw_off = round_up_u32(sh.xs_off + static_cast<uint32_t>(MT * ND) * p.K * ESZ, 128);
  sh.ring_off = sh.xraw_off;
  if (WK != W_BF16) {
    if ((p.K >> 3) <= 128 * (kXRegs / MT))
      sh.xraw_off = 0;  // x pieces staged in registers: no shared-memory copy
    else
      sh.ring_off = round_up_u32(sh.xraw_off + static_cast<uint32_t>(MT) * p.K * 2, 128);
  }
  // shared memory: ~half an SM per CTA at one CTA per SM, ~72 KB (two slots)
  // at two or three (SONATA_GEMV_SMEM_KB overrides)
  const size_t budget = getenv("SONATA_GEMV_SMEM_KB") ? bulk_smem_budget() : cps == 1 ? 110 * 1024 : 72 * 1024;
  const size_t room = budget > sh.ring_off ? budget - sh.ring_off : 0;
  int ns = static_cast<int>(std::min<size_t>(ns_max, room / sh.slot_bytes));
  ns = std::min(ns, tiles_per_cta);
  ns = std::max(ns, 2);
  sh.ns = ns;
  const size_t smem = sh.ring_off + static_cast<size_t>(ns) * sh.slot_bytes;
  if (smem > 220 * 1024) return SN_ERR_UNSUPPORTED;
  auto k2 = gemv_mma_kernel<WK, MT, 2>;
  auto k4 = gemv_mma_kernel<WK, MT, 4>;
  const void* kern = S == 2 ? reinterpret_cast<const void*>(k2) : reinterpret_cast<const void*>(k4);
  if (!ensure_smem(kern, smem)) return SN_ERR_UNSUPPORTED;
  if (S == 2) return launch(k2, dim3(grid, batch), dim3(kMmaGemvThreads), smem, st, pdl, p, sh);
  return launch(k4, dim3(grid, batch), dim3(kMmaGemvThreads), smem, st, pdl, p, sh);
}

template <int WK, int MT>
int dispatch_mt(const GemvParams& p, int batch, size_t smem, cudaStream_t st, bool pdl, bool wvec) {
  constexpr int EPC = WT<WK>::EPC;
  if (!wvec) return launch_gemv(gemv_scalar_kernel<WK, MT>, p, kWarps, batch, smem, st, pdl);
  if (gemv_kernel_choice() == 0) {
    const int rc = dispatch_mma<WK, MT>(p, batch, st, pdl);
    if (rc != SN_ERR_UNSUPPORTED) return rc;
  }
  if (gemv_kernel_choice() <= 1) {
    const int rc = dispatch_bulk<WK, MT>(p, batch, st, pdl);
    if (rc != SN_ERR_UNSUPPORTED) return rc;
  }
  const int nck = p.K / EPC;
  const int per_lane = (nck + 31) / 32;
  // Two rows per warp only when there are plenty of rows to fill 148 SMs.
  const bool many_rows = (int64_t)p.N * batch >= 4736;
  if (per_lane <= 4) {
    if (many_rows) return launch_gemv(gemv_vec_kernel<WK, MT, 2, 4>, p, kWarps * 2, batch, smem, st, pdl);
    return launch_gemv(gemv_vec_kernel<WK, MT, 1, 4>, p, kWarps, batch, smem, st, pdl);
  }
  if (per_lane <= 8) {
    if (many_rows) return launch_gemv(gemv_vec_kernel<WK, MT, 2, 8>, p, kWarps * 2, batch, smem, st, pdl);
    return launch_gemv(gemv_vec_kernel<WK, MT, 1, 8>, p, kWarps, batch, smem, st, pdl);
  }
  return launch_gemv(gemv_vec_kernel<WK, MT, 1, 16>, p, kWarps, batch, smem, st, pdl);
}

}  // namespace

int tu_status_gemv(bool reset, cudaStream_t st, int* out) { return read_tu_status(reset, st, out); }

namespace {
// The weight of the GEMV that follows on the stream (L2 prefetch hint).
struct GemvNext {
  int wk;
  const void* W;
  int64_t ldw;
  int N, K;
};

// Bytes of the next weight prefetched into L2: 8 MB, about what HBM moves
// while a launch drains and the next one starts (measured best of 4..48 MB
// on the config-2 chain; SONATA_GEMV_PREFETCH_MB overrides, 0 disables).
// When a CTA issues the prefetch: once all but this many of its own tiles
// have landed (0: the last one; -1: as soon as its last copy is issued,
// which competes with its own reads and measured slower; -2: at the start,
// before its own copies).
// SONATA_GEMV_PREFETCH_LEAD overrides.
int prefetch_lead() {
  static const int v = [] {
    const char* e = getenv("SONATA_GEMV_PREFETCH_LEAD");
    return e ? atoi(e) : 0;
  }();
  return v;
}

// Rotated x row copies (bulk_g2s_rot); SONATA_GEMV_X_ROT=0 turns them off.
int x_rotate() {
  static const int v = [] {
    const char* e = getenv("SONATA_GEMV_X_ROT");
    return e ? (atoi(e) != 0) : 1;
  }();
  return v;
}

int64_t prefetch_budget() {
  static const int64_t v = [] {
    const char* e = getenv("SONATA_GEMV_PREFETCH_MB");
    const long mb = e ? strtol(e, nullptr, 10) : 8;
    return static_cast<int64_t>(std::max(0L, std::min(mb, 96L))) << 20;
  }();
  return v;
}

// At most this percentage of the next weight is prefetched: 25 (measured
// against 35 / 50 / 100 on the config-2 chain, 0.919 -> 0.913 ms, and on
// int8 / e4m3 in_proj chains, -2%; the 8 MB budget already is ~25% of a
// bf16 in_proj); SONATA_GEMV_PREFETCH_PCT overrides (100: budget only).
int prefetch_pct() {
  static const int v = [] {
    const char* e = getenv("SONATA_GEMV_PREFETCH_PCT");
    const int pct = e ? atoi(e) : 25;
    return std::max(0, std::min(pct, 100));
  }();
  return v;
}

int nd_of(int wk) { return wk == W_INT8 ? 3 : wk == W_E4M3 ? 2 : 1; }

// Normalisation fused into the x staging (sn_gemv_bf16_norm).
struct GemvNorm {
  int kind;  // SN_NORM_*
  const void *aux, *w, *b;
  void* rout;
  float eps;
};

int gemv_impl(int wk, const void* W, int64_t ldw, int64_t sW, const float* scale, int64_t sS, const void* x,
              int64_t ldx, int64_t sx, void* y, int64_t ldy, int64_t sy, int M, int N, int K, int batch,
              int y_dtype, unsigned flags, cudaStream_t st, const GemvNext* next, const GemvNorm* norm = nullptr);
}  // namespace

// Shared by the C entry points and the codebook-head BMM (batch > 1).
int gemv_any(int wk, const void* W, int64_t ldw, int64_t sW, const float* scale, int64_t sS,
             const void* x, int64_t ldx, int64_t sx, void* y, int64_t ldy, int64_t sy, int M, int N, int K,
             int batch, int y_dtype, unsigned flags, cudaStream_t st) {
  return gemv_impl(wk, W, ldw, sW, scale, sS, x, ldx, sx, y, ldy, sy, M, N, K, batch, y_dtype, flags, st,
                   nullptr);
}

namespace {
int gemv_impl(int wk, const void* W, int64_t ldw, int64_t sW, const float* scale, int64_t sS, const void* x,
              int64_t ldx, int64_t sx, void* y, int64_t ldy, int64_t sy, int M, int N, int K, int batch,
              int y_dtype, unsigned flags, cudaStream_t st, const GemvNext* next, const GemvNorm* norm) {
  if (!W || !x || !y) return SN_ERR_INVALID_ARGUMENT;
  if (wk != W_BF16 && !scale) return SN_ERR_INVALID_ARGUMENT;
  if (next && next->W &&
      (next->wk < W_BF16 || next->wk > W_E4M3 || next->N < 1 || next->K < 1 || next->ldw < next->K))
    return SN_ERR_INVALID_ARGUMENT;
  if (M < 1 || M > 4 || N < 1 || K < 1 || batch < 1 || batch > 65535) return SN_ERR_INVALID_ARGUMENT;
  if (ldw < K || ldx < K || ldy < N) return SN_ERR_INVALID_ARGUMENT;
  if (y_dtype != SN_DTYPE_BF16 && y_dtype != SN_DTYPE_F32) return SN_ERR_INVALID_ARGUMENT;
  GemvParams p;
  p.W = static_cast<const uint8_t*>(W);
  p.ldw = ldw;
  p.sW = sW;
  p.scale = scale;
  p.sS = sS;
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.ldx = ldx;
  p.sx = sx;
  p.y = y;
  p.ldy = ldy;
  p.sy = sy;
  p.M = M;
  p.N = N;
  p.K = K;
  p.Kp = (K + 15) & ~15;
  p.y_f32 = y_dtype == SN_DTYPE_F32;
  p.x_vec = aligned16(x) && (K % 8 == 0) && (ldx % 8 == 0) && (batch == 1 || sx % 8 == 0);
  const int esz = (wk == W_BF16) ? 2 : 1;
  const bool wvec = aligned16(W) && ((ldw * esz) % 16 == 0) && (batch == 1 || (sW * esz) % 16 == 0);
  const int MT = M == 1 ? 1 : (M == 2 ? 2 : 4);
  p.pf = nullptr;
  p.pf_ld = 0;
  p.pf_rows = p.pf_parts = 0;
  p.pf_q = p.pf_rem = 0;
  p.pf_row_bytes = p.pf_part_bytes = 0;
  p.pf_lead = prefetch_lead();
  p.x_rot = x_rotate();
  p.xn = 0;
  p.xn_aux = p.xn_w = p.xn_b = nullptr;
  p.xn_rout = nullptr;
  p.xn_eps = 0.f;
  if (norm) {
    // the tensor-core bf16 kernel's staging threads normalise the rows: 16-byte
    // pieces, K a multiple of 1024 up to 4096, one weight (batch 1)
    if (norm->kind != SN_NORM_RMS_GATED && norm->kind != SN_NORM_ADD_LAYER) return SN_ERR_INVALID_ARGUMENT;
    if (!norm->w) return SN_ERR_INVALID_ARGUMENT;
    if (wk != W_BF16 || batch != 1 || K % 1024 != 0 || K > 4096) return SN_ERR_UNSUPPORTED;
    if (!p.x_vec || !aligned16(norm->w) || (norm->aux && !aligned16(norm->aux)) || (norm->b && !aligned16(norm->b)) ||
        (norm->rout && !aligned16(norm->rout)))
      return SN_ERR_MISALIGNED;
    p.xn = norm->kind;
    p.xn_aux = static_cast<const __nv_bfloat16*>(norm->aux);
    p.xn_w = static_cast<const __nv_bfloat16*>(norm->w);
    p.xn_b = static_cast<const __nv_bfloat16*>(norm->b);
    p.xn_rout = static_cast<__nv_bfloat16*>(norm->rout);
    p.xn_eps = norm->eps;
  }
  if (next && next->W) {
    const int nesz = (next->wk == W_BF16) ? 2 : 1;
    const int64_t row_b = static_cast<int64_t>(next->K) * nesz;
    const int64_t nbytes = static_cast<int64_t>(next->N) * row_b;
    const int64_t want = std::min(std::min(nbytes, prefetch_budget()), nbytes / 100 * prefetch_pct());
    // a hint: weights a bulk prefetch cannot address (16-byte rules) are skipped
    if (want > 0 && aligned16(next->W) && (next->ldw * nesz) % 16 == 0 && row_b % 16 == 0 && row_b < (1 << 30)) {
      MmaGrid g;
      const int parts = mma_grid(nesz, nd_of(next->wk), MT, next->N, next->K, 1, g) ? g.grid : sm_count();
      p.pf = static_cast<const uint8_t*>(next->W);
      p.pf_ld = next->ldw * nesz;
      p.pf_rows = next->N;
      p.pf_parts = parts;
      p.pf_q = next->N / parts;
      p.pf_rem = next->N % parts;
      p.pf_row_bytes = static_cast<uint32_t>(row_b);
      const int64_t per_part = ((want + parts - 1) / parts + 127) / 128 * 128;  // whole 128-byte lines
      p.pf_part_bytes = static_cast<uint32_t>(std::min<int64_t>(per_part, int64_t(1) << 30));
    }
  }
  const size_t smem = (size_t)MT * p.Kp * sizeof(float);
  if (smem > 200 * 1024) return SN_ERR_UNSUPPORTED;  // x must fit in shared memory
  const bool pdl = (flags & SN_FLAG_PDL) != 0;
  if (p.xn != 0) {  // only the tensor-core bf16 kernel implements the fused normalisation
    if (!wvec) return SN_ERR_UNSUPPORTED;
    switch (MT) {
      case 1: return dispatch_mma<W_BF16, 1>(p, batch, st, pdl);
      case 2: return dispatch_mma<W_BF16, 2>(p, batch, st, pdl);
      default: return dispatch_mma<W_BF16, 4>(p, batch, st, pdl);
    }
  }
#define SN_DISPATCH(WKV)                                                   \
  switch (MT) {                                                            \
    case 1: return dispatch_mt<WKV, 1>(p, batch, smem, st, pdl, wvec);     \
    case 2: return dispatch_mt<WKV, 2>(p, batch, smem, st, pdl, wvec);     \
    default: return dispatch_mt<WKV, 4>(p, batch, smem, st, pdl, wvec);    \
  }
  switch (wk) {
    case W_BF16: SN_DISPATCH(W_BF16)
    case W_INT8: SN_DISPATCH(W_INT8)
    case W_E4M3: SN_DISPATCH(W_E4M3)
    default: return SN_ERR_INVALID_ARGUMENT;
  }
#undef SN_DISPATCH
}
}  // namespace

// ---------------------------------------------------------------------------
// Device-side per-row quantisation (bit-identical to scripts/fake_quant.py:37-40
// for int8; BASELINE's e4m3 rule with torch's RNE float8_e4m3fn conversion).
// One warp per row: max|w| by warp reduction, then q = rne(w / scale).
// ---------------------------------------------------------------------------
namespace {
template <bool E4M3>
__global__ void __launch_bounds__(256) quantize_rows_kernel(const __nv_bfloat16* W, int64_t ldw, int N, int K,
                                                            uint8_t* q, int64_t ldq, float* scale) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x * 8 + warp;
  if (n >= N) return;
  const __nv_bfloat16* row = W + (int64_t)n * ldw;
  float amax = 0.f;
  for (int k = lane; k < K; k += 32) amax = fmaxf(amax, fabsf(__bfloat162float(row[k])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  amax = fmaxf(amax, 1e-8f);
  const float s = amax / (E4M3 ? 448.0f : 127.0f);  // IEEE division (no fast-math)
  if (lane == 0) scale[n] = s;
  uint8_t* qrow = q + (int64_t)n * ldq;
  for (int k = lane; k < K; k += 32) {
    const float v = __bfloat162float(row[k]) / s;
    if (E4M3) {
      // |v| <= 448 * (1 + 2^-23) here, so satfinite and torch's
      // NaN-on-overflow rule give the same code.
      qrow[k] = static_cast<uint8_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
    } else {
      float r = rintf(v);
      r = fminf(fmaxf(r, -127.f), 127.f);
      qrow[k] = static_cast<uint8_t>(static_cast<int8_t>(r));
    }
  }
}
}  // namespace

// ---------------------------------------------------------------------------
// GEMV chain: a list of bf16 decode GEMVs (the per-token projection set of a
// decode step) streamed by ONE persistent launch.
//
// Between two launches of the per-call kernel HBM idles for the kernel
// boundary (~2.2 us per GEMV on B200: the previous grid drains, the next one's
// griddepcontrol.wait returns, x lands, the first MMAs issue), which is what
// holds the 156-GEMV set of a Zonos step below the copy roofline.  Weights are
// frozen, so nothing stops a CTA from streaming the next GEMV's rows into its
// ring while the current GEMV finishes: here every CTA walks the jobs in
// order with the same ring, TMEM accumulators and epilogue as the per-call
// kernel, and only the x of a job waits, in the kernel, for the job that
// produces it.
//
// Ordering between jobs: job j names `dep`, an earlier job whose completion
// its x waits for (-1: x is ready when the launch starts).  Every CTA's
// epilogue, after storing its rows of job j, releases one count on job j's
// completion counter (gpu scope); a job's x loader acquires its dep's counter
// at grid size before it copies x (then a proxy fence, since the copy is a
// bulk copy).  dep = j - 1 for every job is the order of back-to-back
// launches on one stream.  The last CTA to leave zeroes the counters for the
// next launch.  All CTAs are co-resident (cooperative launch), and every wait
// is bounded.
//
// Warps: 0 weight producer (frozen weights, no wait), 1 TMEM owner and MMA
// issuer, 2..5 epilogue (TMEM lane quarter = warp % 4), 6 x loader (and 7,
// for the 8-bit kinds, whose x staging computes digit planes).
// ---------------------------------------------------------------------------
namespace {

struct ChainJob {  // device copy of one job (96 bytes)
  const uint8_t* W;
  const __nv_bfloat16* x;
  void* y;
  const float* scale;  // 8-bit kinds: per-row scales
  int64_t ldw_bytes;
  int ldx, ldy;  // elements
  int N, K;
  int dep;
  int S;      // row segments (1, 2 or 4): 16 / S rows per tile
  int flags;  // kJobF32 (fp32 y), kJobSignal (a later job waits for this one)
  uint32_t tile_bytes;
  int n;      // MMA N: 8 * S * MT * planes, rounded up to 16
  int sl;     // log2 S
  int q, rem; // rows per CTA: q, one more for the first rem CTAs (no division in the kernel)
  int pad[2];
};
static_assert(sizeof(ChainJob) == 96, "ChainJob is 96 bytes");

constexpr int kChainThreads = 256;
constexpr int kXPieces = 16;  // 16-byte x pieces an 8-bit x staging lane holds (rows up to K = 4096)
constexpr int kChainAcc = 8;             // TMEM accumulators (a power of two)
constexpr int kJobF32 = 1, kJobSignal = 2;
constexpr int kChainTiles = 16;          // weight tiles in flight at most (mbarrier pairs)
constexpr int kChainXBufs = 4;           // x buffers at most: x staging runs this many jobs ahead
constexpr int kChainExps = 16;           // 8-bit x exponents in flight (> x buffers + accumulators)
constexpr int kChainCounterStride = 32;  // one 128-byte line per completion counter

struct ChainParams {
  const ChainJob* jobs;
  unsigned* counters;  // [njobs] completions, one line each, then the exit ticket
  int njobs, M;
  uint32_t ring_bytes;   // weight ring (>= every job's tile_bytes)
  uint32_t xbuf_bytes;   // one x buffer: MT rows of the longest K
  uint32_t xs_off, ring_off;
  uint32_t tcols;
  int nxb_log2;       // x buffers in use: 2 or 4 (log2 1 or 2)
  int nacc_log2;      // TMEM accumulators in use: 2, 4 or 8
  uint32_t acc_cols;  // TMEM columns per accumulator: the largest MMA N of the chain
};

// The job table is read-only for the launch.  The loads are volatile so that
// the compiler issues them where they stand (a role loads job j + 1 when it
// starts job j) instead of sinking them to their first use at the job
// boundary, where their latency (~0.5 us under a full HBM stream) stalled
// every role once per job.
__device__ __forceinline__ uint4 ld_nc_v4_early(const void* ptr) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(ptr));
  return r;
}
__device__ __forceinline__ ChainJob load_job(const ChainJob* jobs, int j) {
  union {
    uint4 v[6];
    ChainJob job;
  } u;
  const uint4* src = reinterpret_cast<const uint4*>(jobs + j);
#pragma unroll
  for (int i = 0; i < 6; ++i) u.v[i] = ld_nc_v4_early(src + i);
  return u.job;
}

// Named barrier that also returns the OR of `v` over the participating threads.
__device__ __forceinline__ bool named_bar_or(int id, int threads, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.or.pred q, %2, %3, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "r"(id), "r"(threads)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Rows [r0, r1) of a job with N rows owned by CTA c of G.
// (no division: a job's q and rem come from the plan, whose grid the launch
// uses; integer divisions by run-time values cost the single-threaded roles
// ~0.1 us each at every job boundary)
__device__ __forceinline__ void cta_rows(const ChainJob& job, int c, int& r0, int& r1) {
  r0 = c * job.q + min(c, job.rem);
  r1 = r0 + job.q + (c < job.rem ? 1 : 0);
}

template <int WK, int MT>
__global__ void __launch_bounds__(kChainThreads, 1) gemv_chain_kernel(const ChainParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int ESZ = WT<WK>::ESZ;
  constexpr int ND = (WK == W_INT8) ? 3 : (WK == W_E4M3) ? 2 : 1;  // B planes per x row
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);  // [kChainTiles], tile t uses t % kChainTiles
  uint64_t* empty = full + kChainTiles;
  uint64_t* tfull = empty + kChainTiles;
  uint64_t* tempty = tfull + kChainAcc;
  uint64_t* xfull = tempty + kChainAcc;
  uint64_t* xfree = xfull + kChainXBufs;
  uint64_t* done = xfree + kChainXBufs;
  uint64_t* eready = done + 1;  // 8-bit: [kChainExps], the exponents of x use u are in xexp
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(eready + kChainExps);
  uint32_t* tbeg = tmem_slot + 1;  // producer only: ring range of the tiles in flight
  uint32_t* tend = tbeg + kChainTiles;
  int* xexp = reinterpret_cast<int*>(tend + kChainTiles);  // 8-bit: [use % kChainExps][m] e (x row m scaled by 2^e)
  uint8_t* xs = smem + p.xs_off;
  uint8_t* ring = smem + p.ring_off;
  // accumulators: a power of two, so masks and shifts (not divisions) in the hot loops
  const int nacc = 1 << p.nacc_log2, nl = p.nacc_log2;
  const uint32_t acc_cols = p.acc_cols;
  const int nxb = 1 << p.nxb_log2, xl = p.nxb_log2;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = static_cast<int>(gridDim.x), c = static_cast<int>(blockIdx.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kChainTiles; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < kChainAcc; ++b) {
      mbar_init(tfull + b, 1);
      mbar_init(tempty + b, 4);
    }
    for (int b = 0; b < kChainXBufs; ++b) {
      mbar_init(xfull + b, 1);
      mbar_init(xfree + b, 1);
    }
    mbar_init(done, 1);
    for (int k = 0; k < kChainExps; ++k) mbar_init(eready + k, 1);
    fence_barrier_init();
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, p.tcols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();

  if (warp == 0) {
    // ---------------- producer: every job's weight rows, in job order ------
    // The ring is a byte ring: tile t (tile_bytes of its job) goes right
    // after tile t - 1, or at 0 when it would pass the end, so tiles of
    // different jobs pack without padding; before it is written, the oldest
    // tiles it overlaps (and any beyond kChainTiles in flight) must have
    // been consumed.
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      int t = 0, tail = 0;
      uint32_t off = 0;
      bool ok = true;
      ChainJob job = load_job(p.jobs, 0), nxt;
      for (int j = 0; j < p.njobs && ok; ++j, job = nxt) {
        nxt = load_job(p.jobs, min(j + 1, p.njobs - 1));  // in flight while job j runs
        if (job.tile_bytes > p.ring_bytes) {  // workspace and plan do not match
          record_status(SN_ERR_INVALID_ARGUMENT);
          ok = false;
          break;
        }
        const int R = 16 >> job.sl;
        const uint32_t row_bytes = static_cast<uint32_t>(job.K) * ESZ;
        int r0, r1;
        cta_rows(job, c, r0, r1);
        for (int first = r0; first < r1; first += R, ++t) {
          if (off + job.tile_bytes > p.ring_bytes) off = 0;
          const uint32_t end = off + job.tile_bytes;
          // the youngest tile in flight that the new one overlaps (tiles are
          // consumed in order, so its release implies every older one's)
          // (tiles before t - kChainTiles were released before their pairs
          // were reused, so at most kChainTiles entries are scanned)
          int need = t - kChainTiles;  // the mbarrier pair is reused
          for (int v = max(tail, t - kChainTiles); v < t; ++v) {
            const int q = v % kChainTiles;
            if (tend[q] > off && tbeg[q] < end) need = max(need, v);
          }
          if (need >= tail) {
            if (!mbar_wait_bounded(empty + need % kChainTiles, (need / kChainTiles) & 1)) {
              record_status(SN_ERR_TIMEOUT);
              ok = false;
              break;
            }
            tail = need + 1;
          }
          const int q = t % kChainTiles;
          tbeg[q] = off;
          tend[q] = end;
          const int cnt = min(R, r1 - first);
          uint8_t* dst = ring + off;
          mbar_arrive_expect_tx(full + q, static_cast<uint32_t>(cnt) * row_bytes);
          if (job.ldw_bytes == static_cast<int64_t>(row_bytes)) {
            bulk_g2s(dst, job.W + static_cast<int64_t>(first) * job.ldw_bytes, static_cast<uint32_t>(cnt) * row_bytes,
                     full + q, pol);
          } else {
            for (int r = 0; r < cnt; ++r)
              bulk_g2s(dst + static_cast<size_t>(r) * row_bytes, job.W + static_cast<int64_t>(first + r) * job.ldw_bytes,
                       row_bytes, full + q, pol);
          }
          off = end;
        }
      }
      if (!ok) {
        // let the copies in flight land before the CTA exits
        for (int v = (t > kChainTiles ? t - kChainTiles : 0); v < t; ++v)
          mbar_wait_bounded(full + v % kChainTiles, (v / kChainTiles) & 1);
      }
    }
  } else if (warp == 6 || warp == 7) {
    // ---------------- x loaders: wait for each job's producer --------------
    // bf16: warp 6 alone (one bulk copy per row); 8-bit: warps 6 and 7 take
    // alternate jobs (a warp's row maximum and planes take ~3 us at K = 2048)
    constexpr int kXWarps = (WK == W_BF16) ? 1 : 2;
    const int xw = warp - 6;
    pdl_wait();  // the first jobs' x and the counters belong to earlier kernels
    int u = 0;
    ChainJob job = load_job(p.jobs, 0), nxt;
    for (int j = 0; j < p.njobs && xw < kXWarps; ++j, job = nxt) {
      nxt = load_job(p.jobs, min(j + 1, p.njobs - 1));
      int r0, r1;
      cta_rows(job, c, r0, r1);
      if (r0 == r1) continue;
      if (u % kXWarps != xw) {  // the other warp's job
        ++u;
        continue;
      }
      const int b = u & (nxb - 1);
      const uint32_t row_bytes = static_cast<uint32_t>(job.K) * ESZ;  // x row bytes in the B operand
      if (static_cast<uint32_t>(MT * ND) * row_bytes > p.xbuf_bytes) {
        if (lane == 0) record_status(SN_ERR_INVALID_ARGUMENT);
        break;
      }
      bool w = u < nxb || mbar_wait_bounded(xfree + b, ((u >> xl) - 1) & 1);
      // every lane that reads x acquires its producer's completion itself
      if (w && job.dep >= 0 && (WK != W_BF16 || lane == 0))
        w = wait_counter(p.counters + static_cast<size_t>(job.dep) * kChainCounterStride, static_cast<unsigned>(G));
      if (!__all_sync(0xffffffffu, w)) {
        if (lane == 0) record_status(SN_ERR_TIMEOUT);
        break;
      }
      uint8_t* dst = xs + static_cast<size_t>(b) * p.xbuf_bytes;
      if constexpr (WK == W_BF16) {
        // x rows by bulk copy, completing xfull[b]
        if (lane == 0) {
          if (job.dep >= 0) fence_proxy_async_global();  // acquired generic writes -> the bulk copy below
          mbar_arrive_expect_tx(xfull + b, static_cast<uint32_t>(p.M) * row_bytes);
          for (int m = 0; m < p.M; ++m)
            bulk_g2s(dst + static_cast<size_t>(m) * row_bytes, job.x + static_cast<int64_t>(m) * job.ldx, row_bytes,
                     xfull + b, l2_policy_evict_normal());
        }
      } else {
        // the B planes of x * 2^e_m (8-bit kinds), by the whole warp: the row
        // maximum, then the digits / terms of every element
        const int cpr = job.K / 8;  // 16-byte pieces of a bf16 x row
        for (int m = 0; m < MT; ++m) {
          int e = 0;
          float up1 = 0.f, up2 = 0.f;
          const __nv_bfloat16* xrow = job.x + static_cast<int64_t>(m) * job.ldx;
          if (cpr <= 32 * kXPieces) {
            // rows up to 32 kXPieces pieces: one load of each piece, held in
            // registers between the maximum and the planes
            uint4 v[kXPieces];
            uint32_t mx = 0;
#pragma unroll
            for (int i = 0; i < kXPieces; ++i) {
              const int cc = lane + 32 * i;
              v[i] = (m < p.M && cc < cpr) ? ld_cg_v4(xrow + cc * 8) : make_uint4(0, 0, 0, 0);
              mx = max(mx, x8_piece_max(v[i]));
            }
            mx = __reduce_max_sync(0xffffffffu, mx);
            e = x8_row_scale<WK>(mx, up1, up2);
#pragma unroll
            for (int i = 0; i < kXPieces; ++i) {
              const int cc = lane + 32 * i;
              if (cc < cpr) x8_emit<WK, MT>(dst, job.K, m, cc, v[i], up1, up2);
            }
          } else {
            if (m < p.M) {
              uint32_t mx = 0;
              for (int cc = lane; cc < cpr; cc += 32) mx = max(mx, x8_piece_max(ld_cg_v4(xrow + cc * 8)));
              mx = __reduce_max_sync(0xffffffffu, mx);
              e = x8_row_scale<WK>(mx, up1, up2);
            }
            for (int cc = lane; cc < cpr; cc += 32)
              x8_emit<WK, MT>(dst, job.K, m, cc, m < p.M ? ld_cg_v4(xrow + cc * 8) : make_uint4(0, 0, 0, 0), up1,
                              up2);
          }
          if (lane == 0) xexp[(u % kChainExps) * MT + m] = e;
        }
        tc::fence_proxy_async_smem();  // the plane stores -> the tensor core's reads
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(xfull + b);
          mbar_arrive(eready + u % kChainExps);  // the exponents -> the epilogue
        }
      }
      ++u;
    }
    // the last bulk copies have landed before the CTA can exit (the MMA
    // issuer waits for them too unless it stopped early)
    if (WK == W_BF16 && xw == 0 && lane == 0)
      for (int v = (u > nxb ? u - nxb : 0); v < u; ++v) mbar_wait_bounded(xfull + (v & (nxb - 1)), (v >> xl) & 1);
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int t = 0, u = 0;
      uint32_t off = 0;  // the producer's placement rule, replayed
      bool ok = true;
      ChainJob job = load_job(p.jobs, 0), nxt;
      for (int j = 0; j < p.njobs && ok; ++j, job = nxt) {
        nxt = load_job(p.jobs, min(j + 1, p.njobs - 1));
        int r0, r1;
        cta_rows(job, c, r0, r1);
        if (r0 == r1) continue;
        const int b = u & (nxb - 1);
        if (!mbar_wait_bounded(xfull + b, (u >> xl) & 1)) {
          record_status(SN_ERR_TIMEOUT);
          break;
        }
        const int R = 16 >> job.sl;
        const uint32_t L = (static_cast<uint32_t>(job.K) * ESZ) >> job.sl;  // segment bytes
        const uint32_t nk = L / 256;                                      // MMAs per tile
        const int n = job.n;
        const uint32_t idesc = (WK == W_INT8)   ? tc::idesc_s8_s32(128, n)
                               : (WK == W_E4M3) ? tc::idesc_e4m3_f32(128, n)
                                                : tc::idesc_bf16_f32(128, n);
        const uint64_t db0 = tc::smem_desc_noswz(xs + static_cast<size_t>(b) * p.xbuf_bytes, 128, L);
        for (int first = r0; first < r1; first += R, ++t) {
          if (off + job.tile_bytes > p.ring_bytes) off = 0;
          const int q = t % kChainTiles, a = t & (nacc - 1);
          if (!mbar_wait_bounded(full + q, (t / kChainTiles) & 1) ||
              (t >= nacc && !mbar_wait_bounded(tempty + a, ((t >> nl) - 1) & 1))) {
            record_status(SN_ERR_TIMEOUT);
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint64_t da0 = tc::smem_desc_noswz(ring + off, 128, L);
          const uint32_t d = tmem + static_cast<uint32_t>(a) * acc_cols;
          for (uint32_t k = 0; k < nk; ++k) {  // 256 bytes of every segment per MMA
            if constexpr (WK == W_INT8)
              tc::mma_s8(d, da0 + 16 * k, db0 + 16 * k, idesc, k != 0);
            else if constexpr (WK == W_E4M3)
              tc::mma_e4m3(d, da0 + 16 * k, db0 + 16 * k, idesc, k != 0);
            else
              tc::mma_bf16(d, da0 + 16 * k, db0 + 16 * k, idesc, k != 0);
          }
          tc::mma_commit(empty + q);
          tc::mma_commit(tfull + a);
          off += job.tile_bytes;
        }
        tc::mma_commit(xfree + b);  // x buffer b is free once these MMAs retire
        ++u;
      }
      // every MMA issued has retired before TMEM is released
      tc::mma_commit(done);
      if (!mbar_wait_bounded(done, 0)) record_status(SN_ERR_TIMEOUT);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    pdl_wait();  // y and the counters belong to earlier kernels until here
    const int q = warp & 3;
    const int i = q * 32 + lane;  // A row = TMEM lane
    int t = 0, u = 0;
    bool ok = true;
    ChainJob job = load_job(p.jobs, 0), nxt;
    for (int j = 0; j < p.njobs; ++j, job = nxt) {
      nxt = load_job(p.jobs, min(j + 1, p.njobs - 1));
      int r0, r1;
      cta_rows(job, c, r0, r1);
      const int R = 16 >> job.sl;
      const int Gs = 8 << job.sl;  // TMEM lanes (and columns) per weight row
      const int r = i / Gs;      // weight row inside the tile
      int e[MT];                 // 8-bit: x row m was scaled by 2^e[m]
#pragma unroll
      for (int m = 0; m < MT; ++m) e[m] = 0;
      if (WK != W_BF16 && r0 < r1 && ok) {
        ok = mbar_wait_bounded(eready + u % kChainExps, (u / kChainExps) & 1);
#pragma unroll
        for (int m = 0; m < MT; ++m) e[m] = xexp[(u % kChainExps) * MT + m];
        if (!ok) record_status(SN_ERR_TIMEOUT);
      }
      if (r0 < r1) ++u;
      for (int first = r0; ok && first < r1; first += R, ++t) {
        const int a = t & (nacc - 1);
        const int cnt = min(R, r1 - first);
        // the row scale (frozen weights) is in flight while the MMAs finish
        const float rs = (WK != W_BF16 && r < cnt) ? __ldg(job.scale + first + r) : 0.f;
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(tfull + a, (t >> nl) & 1))) {
          record_status(SN_ERR_TIMEOUT);
          ok = false;
          break;
        }
        tc::fence_after_sync();
        const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(a) * acc_cols;
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          float v;
          if constexpr (WK == W_BF16) {
            v = job.S == 2 ? diag_entry<2>(taddr + m * Gs, lane) : diag_entry<4>(taddr + m * Gs, lane);
            for (int o = Gs / 2; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
          } else {
            // same arithmetic and order as gemv_mma_kernel's epilogue
            int d32[ND];
            uint32_t ta[ND];
            float de[ND];
#pragma unroll
            for (int d = 0; d < ND; ++d) ta[d] = taddr + (d * MT + m) * Gs;
            if (job.S == 1)
              diag_entries<1, ND>(ta, lane, de);
            else if (job.S == 2)
              diag_entries<2, ND>(ta, lane, de);
            else
              diag_entries<4, ND>(ta, lane, de);
            if constexpr (WK == W_INT8) {
#pragma unroll
              for (int d = 0; d < ND; ++d) {  // exact s32 digit sums
                int iv = __float_as_int(de[d]);
                for (int o = Gs / 2; o >= 1; o >>= 1) iv += __shfl_xor_sync(0xffffffffu, iv, o);
                d32[d] = iv;
              }
            } else {
              float f = 0.f;  // the two e4m3 terms' products, summed per lane first
#pragma unroll
              for (int d = 0; d < ND; ++d) f += de[d];
              for (int o = Gs / 2; o >= 1; o >>= 1) f += __shfl_xor_sync(0xffffffffu, f, o);
#pragma unroll
              for (int d = 0; d < ND; ++d) d32[d] = __float_as_int(f);
            }
            v = x8_dot<WK, ND>(d32, e[m]) * rs;
          }
          if ((lane & (Gs - 1)) == 0 && r < cnt && m < p.M) {
            const int64_t off = static_cast<int64_t>(m) * job.ldy + first + r;
            if (job.flags & kJobF32)
              static_cast<float*>(job.y)[off] = v;
            else
              static_cast<__nv_bfloat16*>(job.y)[off] = __float2bfloat16_rn(v);
          }
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty + a);
      }
      // the four epilogue warps agree on whether to go on (a warp whose wait
      // ran out skipped its remaining tiles); then, if a later job waits for
      // job j, one count on its completion: this CTA's rows are stored (the
      // barrier orders the four warps' stores before the release)
      // (a warp that stopped skips the tiles of the jobs without a barrier
      // and leaves at the next one, with the others)
      if (job.flags & kJobSignal) {
        if (named_bar_or(2, 128, !ok)) break;
        if (threadIdx.x == 64) red_release_gpu_add(p.counters + static_cast<size_t>(j) * kChainCounterStride, 1u);
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) tc::tmem_dealloc(tmem, p.tcols);
  if (threadIdx.x == 0) {
    // the last CTA to leave zeroes the counters for the next launch (every
    // other CTA has finished all its waits and counts before taking a ticket)
    unsigned* ticket = p.counters + static_cast<size_t>(p.njobs) * kChainCounterStride;
    __threadfence();
    if (atomicAdd(ticket, 1u) == static_cast<unsigned>(G) - 1) {
      __threadfence();
      for (int j = 0; j < p.njobs; ++j) p.counters[static_cast<size_t>(j) * kChainCounterStride] = 0;
      *ticket = 0;
      __threadfence();
    }
  }
}

}  // namespace

namespace {

constexpr int kChainMaxJobs = 4096;

size_t chain_table_bytes(int njobs) { return (static_cast<size_t>(njobs) * sizeof(ChainJob) + 127) / 128 * 128; }
size_t chain_workspace_bytes(int njobs) {
  return chain_table_bytes(njobs) + static_cast<size_t>(njobs + 1) * kChainCounterStride * sizeof(unsigned);
}

// Dynamic shared memory of one chain CTA: one CTA per SM (a second one would
// halve the ring, and config-2 shapes need two 44 KB tiles plus x in each).
constexpr size_t kChainSmem = 232448;

struct ByteRange {
  uintptr_t lo, hi;  // [lo, hi)
};
ByteRange rows_range(const void* p, int rows, int64_t ld, int64_t len, int esz) {
  const uintptr_t lo = reinterpret_cast<uintptr_t>(p);
  return {lo, lo + static_cast<uintptr_t>(((rows - 1) * ld + len) * esz)};
}
bool overlap(const ByteRange& a, const ByteRange& b) { return a.lo < b.hi && b.lo < a.hi; }

}  // namespace

namespace {
template <int WK, int MT>
int chain_launch(const ChainParams& p, int grid, size_t smem, unsigned flags, cudaStream_t stream) {
  auto kern = gemv_chain_kernel<WK, MT>;
  if (!ensure_smem(reinterpret_cast<const void*>(kern), smem)) return SN_ERR_UNSUPPORTED;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kChainThreads, smem) != cudaSuccess) {
    cudaGetLastError();
    return SN_ERR_LAUNCH;
  }
  if (per_sm < 1) return SN_ERR_UNSUPPORTED;
  // every CTA waits for others (job completions): all must be resident at
  // once, which a cooperative launch guarantees
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kChainThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  int na = 1;
  if (flags & SN_FLAG_PDL) {
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    na = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  if (cudaLaunchKernelEx(&cfg, kern, p) != cudaSuccess) {
    cudaGetLastError();
    return SN_ERR_LAUNCH;
  }
  return SN_OK;
}
}  // namespace

}  // namespace sn

extern "C" {

int sn_gemv_bf16(const void* W, int64_t ldw, const void* x, int64_t ldx, void* y, int64_t ldy, int M, int N,
                 int K, int y_dtype, unsigned flags, void* stream) {
  return sn::gemv_any(sn::W_BF16, W, ldw, 0, nullptr, 0, x, ldx, 0, y, ldy, 0, M, N, K, 1, y_dtype, flags,
                      static_cast<cudaStream_t>(stream));
}

int sn_gemv_int8(const int8_t* q, int64_t ldq, const float* scale, const void* x, int64_t ldx, void* y,
                 int64_t ldy, int M, int N, int K, int y_dtype, unsigned flags, void* stream) {
  return sn::gemv_any(sn::W_INT8, q, ldq, 0, scale, 0, x, ldx, 0, y, ldy, 0, M, N, K, 1, y_dtype, flags,
                      static_cast<cudaStream_t>(stream));
}

int sn_gemv_fp8e4m3(const uint8_t* q, int64_t ldq, const float* scale, const void* x, int64_t ldx, void* y,
                    int64_t ldy, int M, int N, int K, int y_dtype, unsigned flags, void* stream) {
  return sn::gemv_any(sn::W_E4M3, q, ldq, 0, scale, 0, x, ldx, 0, y, ldy, 0, M, N, K, 1, y_dtype, flags,
                      static_cast<cudaStream_t>(stream));
}

int sn_gemv_ex(int w_kind, const void* W, int64_t ldw, const float* scale, const void* x, int64_t ldx, void* y,
               int64_t ldy, int M, int N, int K, int y_dtype, unsigned flags, void* stream, int next_kind,
               const void* next_W, int64_t next_ldw, int next_N, int next_K) {
  if (w_kind < SN_WEIGHT_BF16 || w_kind > SN_WEIGHT_E4M3) return SN_ERR_INVALID_ARGUMENT;
  const sn::GemvNext nx{next_kind, next_W, next_ldw, next_N, next_K};
  return sn::gemv_impl(w_kind, W, ldw, 0, w_kind == SN_WEIGHT_BF16 ? nullptr : scale, 0, x, ldx, 0, y, ldy, 0,
                       M, N, K, 1, y_dtype, flags, static_cast<cudaStream_t>(stream), next_W ? &nx : nullptr);
}

int sn_gemv_bf16_norm(int norm_kind, const void* W, int64_t ldw, const void* x, const void* aux, const void* norm_w,
                      const void* norm_b, void* residual_out, float eps, void* y, int64_t ldy, int M, int N, int K,
                      int y_dtype, unsigned flags, void* stream, int next_kind, const void* next_W,
                      int64_t next_ldw, int next_N, int next_K) {
  if (M > 4) return SN_ERR_INVALID_ARGUMENT;
  const sn::GemvNext nx{next_kind, next_W, next_ldw, next_N, next_K};
  const sn::GemvNorm nm{norm_kind, aux, norm_w, norm_b, residual_out, eps};
  return sn::gemv_impl(SN_WEIGHT_BF16, W, ldw, 0, nullptr, 0, x, K, 0, y, ldy, 0, M, N, K, 1, y_dtype, flags,
                       static_cast<cudaStream_t>(stream), next_W ? &nx : nullptr, &nm);
}

static int quantize_rows(bool e4m3, const void* W, int64_t ldw, int N, int K, void* q, int64_t ldq, float* scale,
                         void* stream) {
  if (!W || !q || !scale) return SN_ERR_INVALID_ARGUMENT;
  if (N < 1 || K < 1 || ldw < K || ldq < K) return SN_ERR_INVALID_ARGUMENT;
  dim3 grid((N + 7) / 8);
  auto k = e4m3 ? sn::quantize_rows_kernel<true> : sn::quantize_rows_kernel<false>;
  return sn::launch(k, grid, dim3(256), 0, static_cast<cudaStream_t>(stream), false,
                    static_cast<const __nv_bfloat16*>(W), ldw, N, K, static_cast<uint8_t*>(q), ldq, scale);
}

int sn_quantize_rows_int8(const void* W, int64_t ldw, int N, int K, int8_t* q, int64_t ldq, float* scale,
                          void* stream) {
  return quantize_rows(false, W, ldw, N, K, q, ldq, scale, stream);
}

int sn_quantize_rows_fp8e4m3(const void* W, int64_t ldw, int N, int K, uint8_t* q, int64_t ldq, float* scale,
                             void* stream) {
  return quantize_rows(true, W, ldw, N, K, q, ldq, scale, stream);
}


size_t sn_gemv_chain_workspace_size(int njobs) {
  if (njobs < 1 || njobs > sn::kChainMaxJobs) return 0;
  return sn::chain_workspace_bytes(njobs);
}

int sn_gemv_chain_plan(int w_kind, const sn_gemv_job* jobs, int njobs, int M, void* workspace,
                       size_t workspace_bytes, sn_gemv_chain_info* info, void* stream) {
  using namespace sn;
  if (!jobs || !workspace || !info || njobs < 1 || njobs > kChainMaxJobs || M < 1 || M > 2)
    return SN_ERR_INVALID_ARGUMENT;
  if (w_kind < SN_WEIGHT_BF16 || w_kind > SN_WEIGHT_E4M3) return SN_ERR_INVALID_ARGUMENT;
  if (workspace_bytes < chain_workspace_bytes(njobs)) return SN_ERR_INVALID_ARGUMENT;
  if (!aligned16(workspace)) return SN_ERR_MISALIGNED;
  const int MT = M;
  const int esz = (w_kind == SN_WEIGHT_BF16) ? 2 : 1;
  const int nd = nd_of(w_kind);
  std::vector<ChainJob> dev(static_cast<size_t>(njobs));
  const int grid = sm_count();  // one CTA per SM; the jobs' row split is for this grid
  std::vector<ByteRange> xr(njobs), yr(njobs), wr(njobs);
  uint32_t tile_max = 0, xbuf_need = 0;
  for (int j = 0; j < njobs; ++j) {
    const sn_gemv_job& a = jobs[j];
    if (!a.W || !a.x || !a.y || a.N < 1 || a.K < 1 || a.ldw < a.K || a.ldx < a.K || a.ldy < a.N)
      return SN_ERR_INVALID_ARGUMENT;
    if (a.N >= (1 << 24)) return SN_ERR_UNSUPPORTED;  // the kernel splits rows in 32-bit arithmetic
    if (esz == 1 && !a.scale) return SN_ERR_INVALID_ARGUMENT;
    if (a.dep < -1 || a.dep >= j) return SN_ERR_INVALID_ARGUMENT;
    if (a.y_dtype != SN_DTYPE_BF16 && a.y_dtype != SN_DTYPE_F32) return SN_ERR_INVALID_ARGUMENT;
    if (!aligned16(a.W) || !aligned16(a.x) || (a.ldw * esz) % 16 != 0 || (a.ldx * 2) % 16 != 0)
      return SN_ERR_MISALIGNED;
    int S = mma_segments(a.K, esz, MT, nd);
    // 8-bit: one segment per row where it fits, so a tile is 16 whole rows
    // (32 KB at K = 2048) and the per-tile costs are paid half as often
    if (esz == 1 && a.K % 256 == 0 && 16 * a.K <= 64 * 1024) S = 1;
    if (S == 0 || a.ldx > INT_MAX || a.ldy > INT_MAX) return SN_ERR_UNSUPPORTED;
    const int n = (8 * S * MT * nd + 15) / 16 * 16;  // MMA N (M = 128 takes multiples of 16)
    if (n > 256) return SN_ERR_UNSUPPORTED;
    const int64_t tile = static_cast<int64_t>(16 / S) * a.K * esz;
    if (tile > 128 * 1024) return SN_ERR_UNSUPPORTED;
    ChainJob& d = dev[j];
    d.W = static_cast<const uint8_t*>(a.W);
    d.x = static_cast<const __nv_bfloat16*>(a.x);
    d.y = a.y;
    d.scale = esz == 1 ? a.scale : nullptr;
    d.ldw_bytes = a.ldw * esz;
    d.ldx = static_cast<int>(a.ldx);
    d.ldy = static_cast<int>(a.ldy);
    d.N = a.N;
    d.K = a.K;
    d.dep = a.dep;
    d.S = S;
    d.flags = (a.y_dtype == SN_DTYPE_F32) ? kJobF32 : 0;
    d.tile_bytes = static_cast<uint32_t>(tile);
    d.n = n;
    d.sl = S == 1 ? 0 : S == 2 ? 1 : 2;
    d.q = a.N / grid;
    d.rem = a.N % grid;
    d.pad[0] = d.pad[1] = 0;
    // the B operand spans n / 8 groups of L = K esz / S bytes
    xbuf_need = std::max<uint32_t>(xbuf_need, static_cast<uint32_t>(n / 8) * static_cast<uint32_t>(a.K * esz / S));
    tile_max = std::max(tile_max, d.tile_bytes);
    xr[j] = rows_range(a.x, M, a.ldx, a.K, 2);
    yr[j] = rows_range(a.y, M, a.ldy, a.N, a.y_dtype == SN_DTYPE_F32 ? 4 : 2);
    wr[j] = rows_range(a.W, a.N, a.ldw, a.K, esz);
  }
  for (int j = 0; j < njobs; ++j)
    if (jobs[j].dep >= 0) dev[jobs[j].dep].flags |= kJobSignal;
  // Buffers: no job writes a weight or another job's output, and a job's x
  // may be written only by a job it waits for (its dep, its dep's dep, ...).
  for (int j = 0; j < njobs; ++j) {
    for (int i = 0; i < njobs; ++i) {
      if (overlap(yr[i], wr[j])) return SN_ERR_INVALID_ARGUMENT;
      if (i != j && overlap(yr[i], yr[j])) return SN_ERR_INVALID_ARGUMENT;
      if (!overlap(yr[i], xr[j])) continue;
      bool waits = false;
      for (int d = jobs[j].dep; d >= 0 && !waits; d = jobs[d].dep) waits = (d == i);
      if (!waits) return SN_ERR_INVALID_ARGUMENT;
    }
  }
  // one x buffer: the largest B operand of the chain (MT bf16 rows, or the
  // nd 8-bit planes of each row; an int8 N rounded up to 16 reads one more
  // plane's bytes, unused)
  const uint32_t xbuf = round_up_u32(xbuf_need, 128);
  // x buffers: up to kChainXBufs while the ring keeps two tiles and 96 KB
  // (deeper rings measured no faster), at least two
  const size_t ring_min = std::max<size_t>(2 * static_cast<size_t>(tile_max), 96 * 1024);
  int nxb = kChainXBufs;  // 4 or 2 (a power of two: masks in the kernel)
  if (kChainSmem < round_up_u32(1024 + nxb * xbuf, 1024) + ring_min) nxb = 2;
  const uint32_t ring_off = round_up_u32(1024 + nxb * xbuf, 1024);
  if (kChainSmem < ring_off + 2 * static_cast<size_t>(tile_max)) return SN_ERR_UNSUPPORTED;  // two tiles in flight
  const uint32_t ring_bytes = static_cast<uint32_t>((kChainSmem - ring_off) / 1024 * 1024);
  // TMEM accumulators: as many (up to kChainAcc, a power of two) as 512 columns hold
  // TMEM accumulators: as many (a power of two up to kChainAcc) as 512
  // columns hold at the chain's largest MMA N
  uint32_t acc_cols = 0;
  for (int j = 0; j < njobs; ++j) acc_cols = std::max(acc_cols, static_cast<uint32_t>(dev[j].n));
  int nacc = kChainAcc;
  while (nacc > 2 && nacc * acc_cols > 512) nacc /= 2;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (cudaMemcpyAsync(ws, dev.data(), dev.size() * sizeof(ChainJob), cudaMemcpyHostToDevice, st) != cudaSuccess ||
      cudaMemsetAsync(ws + chain_table_bytes(njobs), 0,
                      static_cast<size_t>(njobs + 1) * kChainCounterStride * sizeof(unsigned), st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess) {
    cudaGetLastError();
    return SN_ERR_LAUNCH;
  }
  info->njobs = njobs;
  info->M = M;
  info->w_kind = w_kind;
  info->x_buffers = nxb;
  info->tile_bytes_max = tile_max;
  info->ring_bytes = ring_bytes;
  info->xbuf_bytes = xbuf;
  info->accumulators = static_cast<uint32_t>(nacc);
  info->accumulator_cols = acc_cols;
  info->grid = static_cast<uint32_t>(grid);
  info->workspace_bytes = chain_workspace_bytes(njobs);
  return SN_OK;
}


int sn_gemv_chain_launch(const sn_gemv_chain_info* info, void* workspace, unsigned flags, void* stream) {
  using namespace sn;
  if (!info || !workspace) return SN_ERR_INVALID_ARGUMENT;
  const int njobs = info->njobs, M = info->M, wk = info->w_kind;
  const int nd = (wk >= SN_WEIGHT_BF16 && wk <= SN_WEIGHT_E4M3) ? nd_of(wk) : 0;
  if (njobs < 1 || njobs > kChainMaxJobs || M < 1 || M > 2 || nd == 0 || info->x_buffers < 2 ||
      info->x_buffers > kChainXBufs || (info->x_buffers & (info->x_buffers - 1)) != 0 ||
      (info->accumulators != 2 && info->accumulators != 4 && info->accumulators != 8) ||
      info->accumulator_cols == 0 || info->accumulator_cols % 16 != 0 || info->accumulator_cols > 256 ||
      info->accumulators * info->accumulator_cols > 512 ||
      info->tile_bytes_max == 0 || info->tile_bytes_max % 16 != 0 || info->ring_bytes % 1024 != 0 ||
      info->ring_bytes < 2 * info->tile_bytes_max || info->xbuf_bytes % 128 != 0 ||
      info->workspace_bytes != chain_workspace_bytes(njobs))
    return SN_ERR_INVALID_ARGUMENT;
  if ((flags & ~SN_FLAG_PDL) != 0) return SN_ERR_INVALID_ARGUMENT;
  ChainParams p;
  p.jobs = static_cast<const ChainJob*>(workspace);
  p.counters = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(workspace) + chain_table_bytes(njobs));
  p.njobs = njobs;
  p.M = M;
  p.ring_bytes = info->ring_bytes;
  p.xbuf_bytes = info->xbuf_bytes;
  p.nxb_log2 = info->x_buffers == 4 ? 2 : 1;
  p.xs_off = 1024;
  p.ring_off = round_up_u32(1024 + info->x_buffers * p.xbuf_bytes, 1024);
  p.nacc_log2 = info->accumulators == 8 ? 3 : info->accumulators == 4 ? 2 : 1;
  p.acc_cols = info->accumulator_cols;
  p.tcols = tc::tmem_cols_for(info->accumulators * info->accumulator_cols);
  const size_t smem = p.ring_off + static_cast<size_t>(p.ring_bytes);
  if (smem > kChainSmem) return SN_ERR_INVALID_ARGUMENT;
  // the plan split the rows for its device's SM count: one CTA per SM
  const int grid = static_cast<int>(info->grid);
  if (grid < 1 || grid > sm_count()) return SN_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (wk * 2 + (M - 1)) {
    case SN_WEIGHT_BF16 * 2: return chain_launch<W_BF16, 1>(p, grid, smem, flags, st);
    case SN_WEIGHT_BF16 * 2 + 1: return chain_launch<W_BF16, 2>(p, grid, smem, flags, st);
    case SN_WEIGHT_INT8 * 2: return chain_launch<W_INT8, 1>(p, grid, smem, flags, st);
    case SN_WEIGHT_INT8 * 2 + 1: return chain_launch<W_INT8, 2>(p, grid, smem, flags, st);
    case SN_WEIGHT_E4M3 * 2: return chain_launch<W_E4M3, 1>(p, grid, smem, flags, st);
    default: return chain_launch<W_E4M3, 2>(p, grid, smem, flags, st);
  }
}

}  // extern "C"
