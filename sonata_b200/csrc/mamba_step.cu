// Mamba2 decode-step element ops around the decode GEMVs (bf16, B200).
//
// The four ops Mamba2.step() runs between its projections, with the
// semantics of the libraries the reference pins them to
// (scripts/validation_harness.py:39, :58-115, :140-171): causal_conv1d
// 1.6.2.post1 `causal_conv1d_update` and mamba_ssm 2.3.2.post1
// `selective_state_update`, `rmsnorm_fn` (layernorm_gated) and
// `layer_norm_fn`.  All arithmetic in fp32, outputs rounded once to bf16, as
// those kernels do.  Decode shapes are tiny (a few K elements per row, batch
// 1-2), so each op is one launch sized to the rows it has and bounded by
// launch latency and one HBM round trip, not bandwidth.  Each kernel starts
// with griddepcontrol.launch_dependents: the projection GEMV that follows it
// in a decode step (launched with programmatic dependent launch) may then
// start streaming its frozen weights while the op runs; it reads the op's
// output only after griddepcontrol.wait.  The ops themselves are launched
// the same way and execute griddepcontrol.wait before their first memory
// access, so their launch and set-up overlap the tail of the kernel before
// them (a GEMV that produced their input), whatever that kernel is.
#include "common.cuh"

#include <climits>

namespace sn {
namespace {

__device__ __forceinline__ float bf(const __nv_bfloat16* p, int64_t i) { return __bfloat162float(p[i]); }
__device__ __forceinline__ float silu(float v) { return v / (1.0f + expf(-v)); }

// ---------------------------------------------------------------------------
// causal_conv1d_update: state [B, D, W] shifts one step left and takes x
// [B, D] as its newest column; y = SiLU?(sum_w state[w] * weight[d, w] + bias).
// One thread per (b, d).
// ---------------------------------------------------------------------------
constexpr int kMaxConvWidth = 8;

// One channel d of causal_conv1d_update: st (W values) shifts one step left
// and takes xv as its newest value; returns act(sum_w st[w] * w[d, w] + bias).
__device__ __forceinline__ __nv_bfloat16 conv_update_channel(__nv_bfloat16 xv, __nv_bfloat16* st,
                                                             const __nv_bfloat16* __restrict__ w,
                                                             const __nv_bfloat16* __restrict__ bias, int d, int W,
                                                             int act) {
  float s[kMaxConvWidth];
#pragma unroll
  for (int k = 0; k < kMaxConvWidth; ++k) s[k] = (k + 1 < W) ? __bfloat162float(st[k + 1]) : 0.f;
  float acc = bias ? bf(bias, d) : 0.f;
#pragma unroll
  for (int k = 0; k < kMaxConvWidth; ++k) {
    if (k + 1 < W) acc = fmaf(s[k], bf(w, static_cast<int64_t>(d) * W + k), acc);
  }
  acc = fmaf(__bfloat162float(xv), bf(w, static_cast<int64_t>(d) * W + W - 1), acc);
#pragma unroll
  for (int k = 0; k < kMaxConvWidth; ++k)
    if (k + 1 < W) st[k] = __float2bfloat16_rn(s[k]);  // exact: bf16 values moved one slot
  st[W - 1] = xv;
  return __float2bfloat16_rn(act ? silu(acc) : acc);
}

// The same output as conv_update_channel (SiLU), from the state as it is,
// without moving it: for channels whose state another CTA moves on.
__device__ __forceinline__ __nv_bfloat16 conv_peek_channel(__nv_bfloat16 xv, const __nv_bfloat16* st,
                                                           const __nv_bfloat16* __restrict__ w,
                                                           const __nv_bfloat16* __restrict__ bias, int d, int W) {
  float acc = bias ? bf(bias, d) : 0.f;
#pragma unroll
  for (int k = 0; k < kMaxConvWidth; ++k) {
    if (k + 1 < W) acc = fmaf(__bfloat162float(st[k + 1]), bf(w, static_cast<int64_t>(d) * W + k), acc);
  }
  acc = fmaf(__bfloat162float(xv), bf(w, static_cast<int64_t>(d) * W + W - 1), acc);
  return __float2bfloat16_rn(silu(acc));
}

__global__ void __launch_bounds__(256) causal_conv1d_update_kernel(const __nv_bfloat16* __restrict__ x,
                                                                   __nv_bfloat16* __restrict__ state,
                                                                   const __nv_bfloat16* __restrict__ w,
                                                                   const __nv_bfloat16* __restrict__ bias,
                                                                   __nv_bfloat16* __restrict__ y, int B, int D,
                                                                   int W, int act) {
  pdl_launch_dependents();  // a following programmatic-dependent GEMV may start its weight stream
  pdl_wait();               // launched early (programmatic dependent launch): inputs from here on
  const int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (e >= static_cast<int64_t>(B) * D) return;
  const int d = static_cast<int>(e % D);
  y[e] = conv_update_channel(x[e], state + e * W, w, bias, d, W, act);
}

// ---------------------------------------------------------------------------
// selective_state_update: per (batch, head, headdim row), dt (+ dt_bias,
// softplus) is shared by the row; state = state * exp(dt * A) + dt * B * x;
// y = sum(state * C) + D * x, times SiLU(z).  Every load of a row is issued
// before its first state store: the state is written through a pointer the
// compiler cannot prove distinct from A / B / C, so loads interleaved with
// the stores would wait out one HBM round trip each.
// ---------------------------------------------------------------------------
constexpr int kMaxStatePerLane = 8;  // strided kernel: d_state <= 256

struct SsuParams {
  __nv_bfloat16* state;            // [batch, nh, hd, ds]
  const __nv_bfloat16* x;          // [batch, nh, hd]
  const __nv_bfloat16* dt;         // [batch, nh, hd]
  const float* A;                  // [nh, hd, ds]
  const __nv_bfloat16* Bm;         // [batch, ng, ds]
  const __nv_bfloat16* Cm;         // [batch, ng, ds]
  const __nv_bfloat16* D;          // [nh, hd] or nullptr
  const __nv_bfloat16* z;          // [batch, nh, hd] or nullptr
  const __nv_bfloat16* dt_bias;    // [nh, hd] or nullptr
  __nv_bfloat16* y;                // [batch, nh, hd]
  int batch, nh, hd, ds, ng, softplus;
  int hpg;  // heads per group (nh / ng)
};

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const uint32_t a = __bfloat16_as_ushort(__float2bfloat16_rn(lo));
  const uint32_t b = __bfloat16_as_ushort(__float2bfloat16_rn(hi));
  return a | (b << 16);
}

// Indices of one (batch, head, headdim) row into the [batch, nh, hd],
// [nh, hd] and [batch, ng] tensors.
struct SsuRow {
  int64_t row, hrow, bg;  // [batch, nh, hd], [nh, hd] and [batch, ng] indices
};
// Rows number fewer than 2^31 (host-checked), so the split is 32-bit.
__device__ __forceinline__ SsuRow ssu_row(const SsuParams& p, int64_t row) {
  const int ri = static_cast<int>(row);
  const int t = ri / p.hd;
  const int dd = ri - t * p.hd;
  const int b = t / p.nh;
  const int h = t - b * p.nh;
  const int g = h / p.hpg;
  return {row, static_cast<int64_t>(h) * p.hd + dd, static_cast<int64_t>(b) * p.ng + g};
}
// The D and z terms of a row, read before the state update so that their
// loads overlap the others instead of following the reduction.
struct SsuTail {
  float d, z;
};
__device__ __forceinline__ SsuTail ssu_tail(const SsuParams& p, const SsuRow& r) {
  return {p.D ? bf(p.D, r.hrow) : 0.f, p.z ? bf(p.z, r.row) : 0.f};
}
__device__ __forceinline__ void ssu_finish(const SsuParams& p, const SsuRow& r, float acc, float xv,
                                           const SsuTail& tl) {
  float out = acc;
  if (p.D) out = fmaf(xv, tl.d, out);
  if (p.z) out *= silu(tl.z);
  p.y[r.row] = __float2bfloat16_rn(out);
}
__device__ __forceinline__ float ssu_dt(const SsuParams& p, const SsuRow& r) {
  float dt = bf(p.dt, r.row);
  if (p.dt_bias) dt += bf(p.dt_bias, r.hrow);
  if (p.softplus) dt = dt <= 20.f ? log1pf(expf(dt)) : dt;
  return dt;
}

// Vector kernel (d_state = 128 NCH, 16-byte aligned state / B / C / A rows):
// 16 lanes per row, two rows per warp; lane l of a row holds elements
// 128 c + 8 l .. 128 c + 8 l + 7 of chunk c (one 16-byte bf16 load of state,
// B and C, two 16-byte loads of A).  Half the threads of a warp per row keep
// every row of a decode step resident in one wave (8192 rows at the Zonos
// shapes) at this kernel's register count.
template <int NCH>
__global__ void __launch_bounds__(256) selective_state_update_vec_kernel(const SsuParams p) {
  pdl_launch_dependents();
  pdl_wait();
  const int l16 = threadIdx.x & 15;
  const int64_t rows = static_cast<int64_t>(p.batch) * p.nh * p.hd;
  const int64_t row = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 4;
  const bool valid = row < rows;  // no early exit: the half-warp shuffles below need every lane
  const SsuRow r = ssu_row(p, valid ? row : 0);
  __nv_bfloat16* st = p.state + r.row * p.ds;
  const float* Ar = p.A + r.hrow * p.ds;
  const __nv_bfloat16* Br = p.Bm + r.bg * p.ds;
  const __nv_bfloat16* Cr = p.Cm + r.bg * p.ds;
  uint4 sv[NCH], bv[NCH], cv[NCH];
  float4 av[2 * NCH];
  if (valid) {
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int s = 128 * c + 8 * l16;
      sv[c] = *reinterpret_cast<const uint4*>(st + s);
      av[2 * c] = *reinterpret_cast<const float4*>(Ar + s);
      av[2 * c + 1] = *reinterpret_cast<const float4*>(Ar + s + 4);
      bv[c] = *reinterpret_cast<const uint4*>(Br + s);
      cv[c] = *reinterpret_cast<const uint4*>(Cr + s);
    }
  }
  const SsuTail tl = (valid && l16 == 0) ? ssu_tail(p, r) : SsuTail{0.f, 0.f};
  const float dt = valid ? ssu_dt(p, r) : 0.f;
  const float xv = valid ? bf(p.x, r.row) : 0.f;
  const float dtx = dt * xv;
  float acc = 0.f;
  if (valid) {
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const uint32_t su[4] = {sv[c].x, sv[c].y, sv[c].z, sv[c].w};
      const uint32_t bu[4] = {bv[c].x, bv[c].y, bv[c].z, bv[c].w};
      const uint32_t cu[4] = {cv[c].x, cv[c].y, cv[c].z, cv[c].w};
      const float a8[8] = {av[2 * c].x, av[2 * c].y, av[2 * c].z, av[2 * c].w,
                           av[2 * c + 1].x, av[2 * c + 1].y, av[2 * c + 1].z, av[2 * c + 1].w};
      uint32_t o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float n0 = fmaf(bf16lo(su[k]), expf(dt * a8[2 * k]), dtx * bf16lo(bu[k]));
        const float n1 = fmaf(bf16hi(su[k]), expf(dt * a8[2 * k + 1]), dtx * bf16hi(bu[k]));
        acc = fmaf(n0, bf16lo(cu[k]), acc);
        acc = fmaf(n1, bf16hi(cu[k]), acc);
        o[k] = pack_bf16x2(n0, n1);
      }
      *reinterpret_cast<uint4*>(st + 128 * c + 8 * l16) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (valid && l16 == 0) ssu_finish(p, r, acc, xv, tl);
}

// Strided kernel (any d_state <= 256, any alignment): one warp per row,
// lane l holds elements l, l + 32, ...
__global__ void __launch_bounds__(256) selective_state_update_kernel(const SsuParams p) {
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t row = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= static_cast<int64_t>(p.batch) * p.nh * p.hd) return;
  const SsuRow r = ssu_row(p, row);
  __nv_bfloat16* st = p.state + row * p.ds;
  const float* Ar = p.A + r.hrow * p.ds;
  const __nv_bfloat16* Br = p.Bm + r.bg * p.ds;
  const __nv_bfloat16* Cr = p.Cm + r.bg * p.ds;
  float sv[kMaxStatePerLane], av[kMaxStatePerLane], bv[kMaxStatePerLane], cv[kMaxStatePerLane];
#pragma unroll
  for (int i = 0; i < kMaxStatePerLane; ++i) {
    const int s = lane + 32 * i;
    if (s < p.ds) {
      sv[i] = __bfloat162float(st[s]);
      av[i] = Ar[s];
      bv[i] = __bfloat162float(Br[s]);
      cv[i] = __bfloat162float(Cr[s]);
    }
  }
  const SsuTail tl = lane == 0 ? ssu_tail(p, r) : SsuTail{0.f, 0.f};
  const float dt = ssu_dt(p, r);
  const float xv = bf(p.x, row);
  const float dtx = dt * xv;
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxStatePerLane; ++i) {
    const int s = lane + 32 * i;
    if (s < p.ds) {
      const float ns = fmaf(sv[i], expf(dt * av[i]), dtx * bv[i]);
      st[s] = __float2bfloat16_rn(ns);
      acc = fmaf(ns, cv[i], acc);
    }
  }
  acc = warp_sum(acc);
  if (lane == 0) ssu_finish(p, r, acc, xv, tl);
}

// ---------------------------------------------------------------------------
// Row norms.  A decode step normalises 1-2 rows of a few thousand elements:
// one CTA per row leaves the reduction latency-bound on a single SM (each
// warp waits out its own dependent loads and reductions; measured 13 us for
// 2 x 4096).  So each row (rmsnorm_gated: each group) is spread over a
// cluster of CL CTAs of 256 threads, at most kNormPer elements a thread, and
// the row sums are reduced through distributed shared memory: every CTA
// publishes its partial, a cluster barrier, every CTA adds the CL partials in
// rank order (the same order everywhere, so every CTA gets the same sum).
// ---------------------------------------------------------------------------
constexpr int kNormThreads = 256;
constexpr int kNormPer = 4;  // elements per thread: rows up to 8 * 256 * 4 = 8192

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_barrier() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ float ld_cluster_f32(const float* local, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(local)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(a) : "memory");
  return v;
}

// Sum of v over the CL CTAs of the cluster (all threads of every CTA call it;
// slot: this reduction's index, so consecutive reductions use fresh smem).
template <int CL>
__device__ __forceinline__ float cluster_sum(float v, float* red, float* part, int slot) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[slot * 8 + warp] = v;
  __syncthreads();
  if (warp == 0) {
    float t = lane < (kNormThreads >> 5) ? red[slot * 8 + lane] : 0.f;
    t = warp_sum(t);
    if (lane == 0) part[slot] = t;
  }
  if constexpr (CL == 1) {
    __syncthreads();
    return part[slot];
  } else {
    cluster_barrier();  // every CTA's part[slot] is written and visible
    float tot = 0.f;
#pragma unroll
    for (int r = 0; r < CL; ++r) tot += ld_cluster_f32(part + slot, static_cast<uint32_t>(r));
    return tot;
  }
}

// y = rms_normalise(x * SiLU(z)) * w (+ bias) for norm_before_gate == 0;
// rms_normalise(x) * w (+ bias) * SiLU(z) otherwise.  Cluster = one (row, group).
template <int CL>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_gated_kernel(const __nv_bfloat16* __restrict__ x,
                                                                     const __nv_bfloat16* __restrict__ w,
                                                                     const __nv_bfloat16* __restrict__ bias,
                                                                     const __nv_bfloat16* __restrict__ z,
                                                                     __nv_bfloat16* __restrict__ y, int N, int G,
                                                                     float eps, int norm_before_gate) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float red[16];
  __shared__ float part[2];
  const int rank = CL == 1 ? 0 : static_cast<int>(cluster_rank());
  const int64_t base = static_cast<int64_t>(blockIdx.x / CL) * G;  // element offset of this (row, group)
  const int c0 = static_cast<int>(base % N);                       // its first column
  const int span = (G + CL - 1) / CL;                              // columns per CTA
  const int cb = rank * span, ce = min(G, cb + span);
  float v[kNormPer];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kNormPer; ++i) {
    const int c = cb + threadIdx.x + i * kNormThreads;
    float t = 0.f;
    if (c < ce) {
      t = bf(x, base + c);
      if (z && !norm_before_gate) t *= silu(bf(z, base + c));
    }
    v[i] = t;
    ss = fmaf(t, t, ss);
  }
  const float r = rsqrtf(cluster_sum<CL>(ss, red, part, 0) / G + eps);
#pragma unroll
  for (int i = 0; i < kNormPer; ++i) {
    const int c = cb + threadIdx.x + i * kNormThreads;
    if (c < ce) {
      float o = v[i] * r * bf(w, c0 + c);
      if (bias) o += bf(bias, c0 + c);
      if (z && norm_before_gate) o *= silu(bf(z, base + c));
      y[base + c] = __float2bfloat16_rn(o);
    }
  }
  if constexpr (CL > 1) cluster_barrier();  // no CTA leaves while a peer may read its part[]
}

// h = x + residual (fp32); residual_out = h (bf16 or fp32) when asked;
// out = LayerNorm or RMSNorm of h (unrounded) * w + bias.  Cluster = one row.
template <int CL>
__global__ void __launch_bounds__(kNormThreads) layer_norm_kernel(const __nv_bfloat16* __restrict__ x,
                                                                  const void* __restrict__ residual, int res_f32,
                                                                  const __nv_bfloat16* __restrict__ w,
                                                                  const __nv_bfloat16* __restrict__ bias,
                                                                  __nv_bfloat16* __restrict__ out,
                                                                  void* __restrict__ residual_out, int rout_f32,
                                                                  int N, float eps, int rms) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float red[16];
  __shared__ float part[2];
  const int rank = CL == 1 ? 0 : static_cast<int>(cluster_rank());
  const int64_t base = static_cast<int64_t>(blockIdx.x / CL) * N;
  const int span = (N + CL - 1) / CL;
  const int cb = rank * span, ce = min(N, cb + span);
  float v[kNormPer];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < kNormPer; ++i) {
    const int c = cb + threadIdx.x + i * kNormThreads;
    float t = 0.f;
    if (c < ce) {
      t = bf(x, base + c);
      if (residual)
        t += res_f32 ? static_cast<const float*>(residual)[base + c]
                     : bf(static_cast<const __nv_bfloat16*>(residual), base + c);
      if (residual_out) {
        if (rout_f32)
          static_cast<float*>(residual_out)[base + c] = t;
        else
          static_cast<__nv_bfloat16*>(residual_out)[base + c] = __float2bfloat16_rn(t);
      }
    }
    v[i] = t;
    sum += t;
  }
  const float mean = rms ? 0.f : cluster_sum<CL>(sum, red, part, 0) / N;
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < kNormPer; ++i) {
    const int c = cb + threadIdx.x + i * kNormThreads;
    const float d = c < ce ? v[i] - mean : 0.f;
    sq = fmaf(d, d, sq);
  }
  const float r = rsqrtf(cluster_sum<CL>(sq, red, part, 1) / N + eps);
#pragma unroll
  for (int i = 0; i < kNormPer; ++i) {
    const int c = cb + threadIdx.x + i * kNormThreads;
    if (c < ce) {
      float o = (v[i] - mean) * r * bf(w, c);
      if (bias) o += bf(bias, c);
      out[base + c] = __float2bfloat16_rn(o);
    }
  }
  if constexpr (CL > 1) cluster_barrier();
}

// Cluster size for a row of n elements: the fewest CTAs (1, 2, 4, 8) with at
// most one element a thread, 8 at most (then up to kNormPer).  Measured
// against two and four elements a thread: add + LayerNorm over 2 x 2048
// 3.70 / 4.34 -> 3.60 us; gated RMSNorm over 2 x 4096 is at 8 CTAs either way.
inline int norm_cluster(int n) {
  int cl = 1;
  while (cl < 8 && n > cl * kNormThreads) cl *= 2;
  return cl;
}

template <typename Kern, typename... Args>
int launch_cluster(Kern kern, int clusters, int cl, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(clusters * cl));
  cfg.blockDim = dim3(kNormThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(cl);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // the kernels wait (griddepcontrol.wait)
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (cudaLaunchKernelEx(&cfg, kern, args...) != cudaSuccess) {
    cudaGetLastError();
    return SN_ERR_LAUNCH;
  }
  return SN_OK;
}

// ---------------------------------------------------------------------------
// Decode-step glue, fused so that a Zonos decode step launches one kernel
// where torch would launch several (slices made contiguous, broadcasts,
// elementwise products):
//
// mamba2_split_conv: the in_proj output zxbcdt [b, ld] = [z | xBC | dt] of a
//   Mamba2 step -> z [b, di] (copy), causal_conv1d_update + SiLU of xBC (state
//   updated in place) written as x [b, di], B [b, ng*ds], C [b, ng*ds], and
//   dt broadcast over headdim [b, nh, hd] -- the inputs of
//   selective_state_update and the gated RMSNorm, each contiguous.
// rotary_kv_append: the qkv projection [b, (hq + 2 hk) hd] -> q rotated
//   [b, hq, hd]; k rotated and v written at position pos of the KV caches
//   [b, hk, max_seqlen, hd].  Non-interleaved rotary (halves rotate), fp32
//   arithmetic with the products and the difference / sum rounded separately
//   (no fused multiply-add: the same values as the torch expression).
// swiglu: h [b, 2d] -> h[:, :d] * SiLU(h[:, d:]) [b, d], SiLU rounded to
//   bf16 before the product (torch's bf16 ops).
// ---------------------------------------------------------------------------
struct SplitConvParams {
  const __nv_bfloat16* zx;  // [b, ld]
  int64_t ld;
  __nv_bfloat16* conv_state;  // [b, conv_dim, W]
  const __nv_bfloat16* w;     // [conv_dim, W]
  const __nv_bfloat16* bias;  // [conv_dim] or null
  __nv_bfloat16 *z, *x, *Bm, *Cm, *dt;
  int batch, di, gds, nh, hd, W;
};

__global__ void __launch_bounds__(256) mamba2_split_conv_kernel(const SplitConvParams p) {
  pdl_launch_dependents();
  pdl_wait();
  const int conv_dim = p.di + 2 * p.gds;
  const int per_b = conv_dim + p.di + p.nh * p.hd;  // conv channels, z copy, dt broadcast
  const int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (e >= static_cast<int64_t>(p.batch) * per_b) return;
  const int b = static_cast<int>(e / per_b);
  int i = static_cast<int>(e % per_b);
  const __nv_bfloat16* row = p.zx + b * p.ld;
  if (i < conv_dim) {
    const __nv_bfloat16 v = conv_update_channel(row[p.di + i], p.conv_state + (static_cast<int64_t>(b) * conv_dim + i) * p.W,
                                                p.w, p.bias, i, p.W, 1);
    if (i < p.di)
      p.x[static_cast<int64_t>(b) * p.di + i] = v;
    else if (i < p.di + p.gds)
      p.Bm[static_cast<int64_t>(b) * p.gds + i - p.di] = v;
    else
      p.Cm[static_cast<int64_t>(b) * p.gds + i - p.di - p.gds] = v;
    return;
  }
  i -= conv_dim;
  if (i < p.di) {
    p.z[static_cast<int64_t>(b) * p.di + i] = row[i];
    return;
  }
  i -= p.di;  // dt broadcast: head i / hd
  p.dt[static_cast<int64_t>(b) * p.nh * p.hd + i] = row[p.di + conv_dim + i / p.hd];
}

// mamba2_conv_ssu: mamba2_split_conv and selective_state_update (vector
// form, d_state 128 or 256, dt softplus) in one launch, with A, D and
// dt_bias per head.  A CTA is 16 rows (b, h, dd .. dd + 15) of one head, 16
// lanes a row, as in selective_state_update_vec_kernel, with the same
// arithmetic in the same order, so the outputs equal the two-launch path's
// bit for bit.  x channels: lane 0 of a row runs the row's conv update (its
// own channel).  B and C of the head's group: every CTA of the (batch,
// group) computes them into shared memory from the conv state as it is,
// then draws a ticket (sync[b * ngroups + g]) with release semantics; the
// CTA that draws the last ticket, whichever it is, has seen every other
// CTA's reads (acquire) and moves the state on at its end, then resets the
// counter to zero.  No CTA waits for another.
struct ConvSsuParams {
  const __nv_bfloat16* zx;  // [b, ld]
  int64_t ld;
  __nv_bfloat16* conv_state;  // [b, conv_dim, W]
  const __nv_bfloat16* w;     // [conv_dim, W]
  const __nv_bfloat16* bias;  // [conv_dim] or null
  __nv_bfloat16* state;       // [b, nh, hd, ds]
  const float* A;             // [nh]
  const __nv_bfloat16* D;     // [nh] or null
  const __nv_bfloat16* dt_bias;  // [nh] or null
  __nv_bfloat16 *z, *y;       // [b, di], [b, nh, hd]
  unsigned* sync;             // [b * ng]
  int di, gds, ds, ng, nh, hd, hpg, W;
  int bpg;  // CTAs per (batch, group): hpg * hd / 16, the tickets drawn per call
};

// Release pattern (fence, then a relaxed atomic at GPU scope): returns the
// count before this one.
__device__ __forceinline__ unsigned fence_then_ticket(unsigned* c) {
  unsigned old;
  asm volatile("fence.acq_rel.gpu;\n\tatom.relaxed.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(c) : "memory");
  return old;
}

template <int NCH>
__global__ void __launch_bounds__(256) mamba2_conv_ssu_kernel(const ConvSsuParams p) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ __align__(16) __nv_bfloat16 sbc[2 * 128 * NCH];  // B then C of this CTA's (batch, group)
  __shared__ int s_mover;
  const int tid = threadIdx.x, l16 = tid & 15;
  const int rowbase = static_cast<int>(blockIdx.x) * 16;
  const int t = rowbase / p.hd;
  const int b = t / p.nh;
  const int h = t - b * p.nh;
  const int g = h / p.hpg;
  const int dd = rowbase - t * p.hd + (tid >> 4);
  const int conv_dim = p.di + 2 * p.gds;
  const int ds = 128 * NCH;
  const __nv_bfloat16* zx = p.zx + static_cast<int64_t>(b) * p.ld;
  __nv_bfloat16* cs = p.conv_state + static_cast<int64_t>(b) * conv_dim * p.W;
  // every load that needs nothing computed here first: the row's SSM state,
  // dt, A, D (selective_state_update of row (b, h, dd))
  const int64_t row = static_cast<int64_t>(t) * p.hd + dd;
  __nv_bfloat16* st = p.state + row * ds;
  uint4 sv[NCH];
#pragma unroll
  for (int c = 0; c < NCH; ++c) sv[c] = *reinterpret_cast<const uint4*>(st + 128 * c + 8 * l16);
  float dt = __bfloat162float(zx[p.di + conv_dim + h]);
  if (p.dt_bias) dt += bf(p.dt_bias, h);
  const float a = p.A[h];
  const float dval = (p.D && l16 == 0) ? bf(p.D, h) : 0.f;
  // B and C of (b, g), from the group's conv state as it is; each thread
  // keeps its channels' moved-on state (the old values shifted, the new
  // input last) for the CTA that stores it
  __nv_bfloat16 kept[NCH][kMaxConvWidth];
#pragma unroll
  for (int j = 0; j < NCH; ++j) {
    const int k = tid + 256 * j;  // 2 * ds = 256 * NCH channels, one per thread and j
    const int ch = p.di + (k < ds ? g * ds + k : p.gds + g * ds + (k - ds));
    const __nv_bfloat16* cst = cs + static_cast<int64_t>(ch) * p.W;
    const __nv_bfloat16 xin = zx[p.di + ch];
#pragma unroll
    for (int w = 0; w < kMaxConvWidth; ++w) kept[j][w] = (w + 1 < p.W) ? cst[w + 1] : xin;
    sbc[k] = conv_peek_channel(xin, cst, p.w, p.bias, ch, p.W);
  }
  // this row's x channel (owned by this row) and z: read now, stored after
  // the count below, so that the count's release has no global store of
  // this CTA to wait for
  const int ch = h * p.hd + dd;
  __nv_bfloat16* xst = cs + static_cast<int64_t>(ch) * p.W;
  __nv_bfloat16 xkept[kMaxConvWidth];
  __nv_bfloat16 zv = __float2bfloat16_rn(0.f);
  float xv = 0.f;
  if (l16 == 0) {
    const __nv_bfloat16 xin = zx[p.di + ch];
#pragma unroll
    for (int w = 0; w < kMaxConvWidth; ++w) xkept[w] = (w + 1 < p.W) ? xst[w + 1] : xin;
    xv = __bfloat162float(conv_peek_channel(xin, xst, p.w, p.bias, ch, p.W));
  }
  if (l16 == 1) zv = zx[ch];
  __syncthreads();
  // every CTA of the group takes a ticket once all its threads have read
  // the group's B / C state (release: fence, then the atomic; no global
  // store of this CTA is pending yet, so the fence is cheap); the ticket
  // comes back while the SSU below runs, and the CTA that drew the last one
  // moves the state on at the end
  unsigned* cnt = p.sync + b * p.ng + g;
  unsigned ticket = 0;
  if (tid == 0) ticket = fence_then_ticket(cnt);
  if (l16 == 0) {
#pragma unroll
    for (int w = 0; w < kMaxConvWidth; ++w)
      if (w < p.W) xst[w] = xkept[w];
  }
  if (l16 == 1) p.z[static_cast<int64_t>(b) * p.di + ch] = zv;

  xv = __shfl_sync(0xffffffffu, xv, 0, 16);
  dt = dt <= 20.f ? log1pf(expf(dt)) : dt;
  const float ea = expf(dt * a);
  const float dtx = dt * xv;
  float acc = 0.f;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int s = 128 * c + 8 * l16;
    const uint4 bv = *reinterpret_cast<const uint4*>(sbc + s);
    const uint4 cv = *reinterpret_cast<const uint4*>(sbc + ds + s);
    const uint32_t su[4] = {sv[c].x, sv[c].y, sv[c].z, sv[c].w};
    const uint32_t bu[4] = {bv.x, bv.y, bv.z, bv.w};
    const uint32_t cu[4] = {cv.x, cv.y, cv.z, cv.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float n0 = fmaf(bf16lo(su[k]), ea, dtx * bf16lo(bu[k]));
      const float n1 = fmaf(bf16hi(su[k]), ea, dtx * bf16hi(bu[k]));
      acc = fmaf(n0, bf16lo(cu[k]), acc);
      acc = fmaf(n1, bf16hi(cu[k]), acc);
      o[k] = pack_bf16x2(n0, n1);
    }
    *reinterpret_cast<uint4*>(st + s) = make_uint4(o[0], o[1], o[2], o[3]);
  }
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (l16 == 0) {
    float out = acc;
    if (p.D) out = fmaf(xv, dval, out);
    p.y[row] = __float2bfloat16_rn(out);
  }

  // the CTA with the last ticket moves the B / C state on: every other CTA
  // of the group has read it (acquire: the fence after the atomic's result)
  if (tid == 0) {
    s_mover = ticket == static_cast<unsigned>(p.bpg - 1);
    if (s_mover) {
      asm volatile("fence.acq_rel.gpu;" ::: "memory");
      *cnt = 0;  // the next launch starts from zero
    }
  }
  __syncthreads();
  if (s_mover) {
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int k = tid + 256 * j;
      const int c2 = p.di + (k < ds ? g * ds + k : p.gds + g * ds + (k - ds));
      __nv_bfloat16* cst = cs + static_cast<int64_t>(c2) * p.W;
#pragma unroll
      for (int w = 0; w < kMaxConvWidth; ++w)
        if (w < p.W) cst[w] = kept[j][w];
    }
  }
}

struct RotaryParams {
  const __nv_bfloat16* qkv;  // [b, (hq + 2 hk) hd]
  __nv_bfloat16* q;          // [b, hq, hd]
  __nv_bfloat16 *kc, *vc;    // [b, hk, S, hd]
  const float *cos, *sin;    // [hd / 2]
  int batch, hq, hk, hd, S, pos;
};

__global__ void __launch_bounds__(256) rotary_kv_append_kernel(const RotaryParams p) {
  pdl_launch_dependents();
  pdl_wait();
  const int h2 = p.hd / 2;
  const int heads = p.hq + 2 * p.hk;
  const int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;  // (b, head, j < h2)
  if (e >= static_cast<int64_t>(p.batch) * heads * h2) return;
  const int j = static_cast<int>(e % h2);
  const int head = static_cast<int>((e / h2) % heads);
  const int b = static_cast<int>(e / (static_cast<int64_t>(h2) * heads));
  const __nv_bfloat16* src = p.qkv + (static_cast<int64_t>(b) * heads + head) * p.hd;
  const float x1 = __bfloat162float(src[j]), x2 = __bfloat162float(src[j + h2]);
  if (head >= p.hq + p.hk) {  // v: copied into the cache
    __nv_bfloat16* dst = p.vc + ((static_cast<int64_t>(b) * p.hk + head - p.hq - p.hk) * p.S + p.pos) * p.hd;
    dst[j] = src[j];
    dst[j + h2] = src[j + h2];
    return;
  }
  const float c = p.cos[j], s = p.sin[j];
  const float r1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
  const float r2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
  __nv_bfloat16* dst = head < p.hq ? p.q + (static_cast<int64_t>(b) * p.hq + head) * p.hd
                                   : p.kc + ((static_cast<int64_t>(b) * p.hk + head - p.hq) * p.S + p.pos) * p.hd;
  dst[j] = __float2bfloat16_rn(r1);
  dst[j + h2] = __float2bfloat16_rn(r2);
}

__global__ void __launch_bounds__(256) swiglu_kernel(const __nv_bfloat16* __restrict__ h, __nv_bfloat16* __restrict__ y,
                                                     int batch, int d) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (e >= static_cast<int64_t>(batch) * d) return;
  const int64_t b = e / d, i = e % d;
  const float g = __bfloat162float(h[b * 2 * d + d + i]);
  const float sg = __bfloat162float(__float2bfloat16_rn(silu(g)));
  y[e] = __float2bfloat16_rn(__fmul_rn(__bfloat162float(h[b * 2 * d + i]), sg));
}

}  // namespace

}  // namespace sn

extern "C" {

int sn_causal_conv1d_update(const void* x, void* conv_state, const void* weight, const void* bias, void* y, int B,
                            int D, int W, int activation, void* stream) {
  if (!x || !conv_state || !weight || !y || B < 1 || D < 1 || W < 1 || W > sn::kMaxConvWidth)
    return SN_ERR_INVALID_ARGUMENT;
  if (activation != SN_ACT_NONE && activation != SN_ACT_SILU) return SN_ERR_INVALID_ARGUMENT;
  const int64_t n = static_cast<int64_t>(B) * D;
  return sn::launch(sn::causal_conv1d_update_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), true, static_cast<const __nv_bfloat16*>(x),
                    static_cast<__nv_bfloat16*>(conv_state), static_cast<const __nv_bfloat16*>(weight),
                    static_cast<const __nv_bfloat16*>(bias), static_cast<__nv_bfloat16*>(y), B, D, W,
                    activation == SN_ACT_SILU ? 1 : 0);
}

int sn_selective_state_update(void* state, const void* x, const void* dt, const float* A, const void* Bm,
                              const void* Cm, const void* D, const void* z, const void* dt_bias, void* y, int batch,
                              int nheads, int headdim, int dstate, int ngroups, int dt_softplus, void* stream) {
  if (!state || !x || !dt || !A || !Bm || !Cm || !y || batch < 1 || nheads < 1 || headdim < 1 || dstate < 1 ||
      ngroups < 1)
    return SN_ERR_INVALID_ARGUMENT;
  if (nheads % ngroups != 0 || dstate > 32 * sn::kMaxStatePerLane) return SN_ERR_INVALID_ARGUMENT;
  sn::SsuParams p;
  p.state = static_cast<__nv_bfloat16*>(state);
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.dt = static_cast<const __nv_bfloat16*>(dt);
  p.A = A;
  p.Bm = static_cast<const __nv_bfloat16*>(Bm);
  p.Cm = static_cast<const __nv_bfloat16*>(Cm);
  p.D = static_cast<const __nv_bfloat16*>(D);
  p.z = static_cast<const __nv_bfloat16*>(z);
  p.dt_bias = static_cast<const __nv_bfloat16*>(dt_bias);
  p.y = static_cast<__nv_bfloat16*>(y);
  p.batch = batch;
  p.nh = nheads;
  p.hd = headdim;
  p.ds = dstate;
  p.ng = ngroups;
  p.softplus = dt_softplus ? 1 : 0;
  p.hpg = nheads / ngroups;
  const int64_t rows = static_cast<int64_t>(batch) * nheads * headdim;
  if (rows > INT32_MAX / 16) return SN_ERR_UNSUPPORTED;  // 32-bit row split, 16 lanes a row
  const bool vec = (dstate == 128 || dstate == 256) && sn::aligned16(state) && sn::aligned16(Bm) &&
                   sn::aligned16(Cm) && sn::aligned16(A);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (vec) {
    const dim3 grid(static_cast<unsigned>((rows + 15) / 16));  // 16 rows per 256-thread CTA
    return dstate == 128 ? sn::launch(sn::selective_state_update_vec_kernel<1>, grid, dim3(256), 0, st, true, p)
                         : sn::launch(sn::selective_state_update_vec_kernel<2>, grid, dim3(256), 0, st, true, p);
  }
  return sn::launch(sn::selective_state_update_kernel, dim3(static_cast<unsigned>((rows + 7) / 8)), dim3(256), 0, st,
                    true, p);
}

int sn_rmsnorm_gated(const void* x, const void* weight, const void* bias, const void* z, void* y, int rows, int N,
                     int group_size, float eps, int norm_before_gate, void* stream) {
  if (!x || !weight || !y || rows < 1 || N < 1 || group_size < 1 || N % group_size != 0) return SN_ERR_INVALID_ARGUMENT;
  if (group_size > 8 * sn::kNormThreads * sn::kNormPer) return SN_ERR_UNSUPPORTED;
  const int64_t groups = static_cast<int64_t>(rows) * (N / group_size);
  if (groups * 8 > INT32_MAX) return SN_ERR_UNSUPPORTED;
  const int cl = sn::norm_cluster(group_size);
  auto args = [&](auto kern) {
    return sn::launch_cluster(kern, static_cast<int>(groups), cl, static_cast<cudaStream_t>(stream),
                              static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(weight),
                              static_cast<const __nv_bfloat16*>(bias), static_cast<const __nv_bfloat16*>(z),
                              static_cast<__nv_bfloat16*>(y), N, group_size, eps, norm_before_gate ? 1 : 0);
  };
  switch (cl) {
    case 1: return args(sn::rmsnorm_gated_kernel<1>);
    case 2: return args(sn::rmsnorm_gated_kernel<2>);
    case 4: return args(sn::rmsnorm_gated_kernel<4>);
    default: return args(sn::rmsnorm_gated_kernel<8>);
  }
}

int sn_layer_norm_fused(const void* x, const void* residual, int residual_f32, const void* weight, const void* bias,
                        void* out, void* residual_out, int residual_out_f32, int rows, int N, float eps,
                        int is_rms_norm, void* stream) {
  if (!x || !weight || !out || rows < 1 || N < 1) return SN_ERR_INVALID_ARGUMENT;
  if (N > 8 * sn::kNormThreads * sn::kNormPer) return SN_ERR_UNSUPPORTED;
  if (static_cast<int64_t>(rows) * 8 > INT32_MAX) return SN_ERR_UNSUPPORTED;
  const int cl = sn::norm_cluster(N);
  auto args = [&](auto kern) {
    return sn::launch_cluster(kern, rows, cl, static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(x),
                              residual, residual_f32 ? 1 : 0, static_cast<const __nv_bfloat16*>(weight),
                              static_cast<const __nv_bfloat16*>(bias), static_cast<__nv_bfloat16*>(out),
                              residual_out, residual_out_f32 ? 1 : 0, N, eps, is_rms_norm ? 1 : 0);
  };
  switch (cl) {
    case 1: return args(sn::layer_norm_kernel<1>);
    case 2: return args(sn::layer_norm_kernel<2>);
    case 4: return args(sn::layer_norm_kernel<4>);
    default: return args(sn::layer_norm_kernel<8>);
  }
}

int sn_mamba2_split_conv(const void* zxbcdt, int64_t ld, void* conv_state, const void* conv_weight,
                         const void* conv_bias, void* z, void* x, void* B, void* C, void* dt, int batch, int d_inner,
                         int ngroups, int d_state, int nheads, int headdim, int d_conv, void* stream) {
  if (!zxbcdt || !conv_state || !conv_weight || !z || !x || !B || !C || !dt || batch < 1 || d_inner < 1 ||
      ngroups < 1 || d_state < 1 || nheads < 1 || headdim < 1 || d_conv < 1 || d_conv > sn::kMaxConvWidth)
    return SN_ERR_INVALID_ARGUMENT;
  if (static_cast<int64_t>(nheads) * headdim != d_inner) return SN_ERR_INVALID_ARGUMENT;
  const int64_t gds = static_cast<int64_t>(ngroups) * d_state;
  if (ld < 2 * d_inner + 2 * gds + nheads) return SN_ERR_INVALID_ARGUMENT;
  sn::SplitConvParams p;
  p.zx = static_cast<const __nv_bfloat16*>(zxbcdt);
  p.ld = ld;
  p.conv_state = static_cast<__nv_bfloat16*>(conv_state);
  p.w = static_cast<const __nv_bfloat16*>(conv_weight);
  p.bias = static_cast<const __nv_bfloat16*>(conv_bias);
  p.z = static_cast<__nv_bfloat16*>(z);
  p.x = static_cast<__nv_bfloat16*>(x);
  p.Bm = static_cast<__nv_bfloat16*>(B);
  p.Cm = static_cast<__nv_bfloat16*>(C);
  p.dt = static_cast<__nv_bfloat16*>(dt);
  p.batch = batch;
  p.di = d_inner;
  p.gds = static_cast<int>(gds);
  p.nh = nheads;
  p.hd = headdim;
  p.W = d_conv;
  const int64_t n = static_cast<int64_t>(batch) * (2 * d_inner + 2 * gds + static_cast<int64_t>(nheads) * headdim);
  return sn::launch(sn::mamba2_split_conv_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), true, p);
}

int sn_mamba2_conv_ssu(const void* zxbcdt, int64_t ld, void* conv_state, const void* conv_weight,
                       const void* conv_bias, void* ssm_state, const float* A, const void* D, const void* dt_bias,
                       void* z, void* y, unsigned* sync, int batch, int d_inner, int ngroups, int d_state, int nheads,
                       int headdim, int d_conv, void* stream) {
  if (!zxbcdt || !conv_state || !conv_weight || !ssm_state || !A || !z || !y || !sync || batch < 1 || d_inner < 1 ||
      ngroups < 1 || d_state < 1 || nheads < 1 || headdim < 1 || d_conv < 1 || d_conv > sn::kMaxConvWidth)
    return SN_ERR_INVALID_ARGUMENT;
  if (static_cast<int64_t>(nheads) * headdim != d_inner || nheads % ngroups != 0) return SN_ERR_INVALID_ARGUMENT;
  const int64_t gds = static_cast<int64_t>(ngroups) * d_state;
  if (ld < 2 * d_inner + 2 * gds + nheads) return SN_ERR_INVALID_ARGUMENT;
  const int64_t rows = static_cast<int64_t>(batch) * d_inner;
  if ((d_state != 128 && d_state != 256) || headdim % 16 != 0 || !sn::aligned16(ssm_state) ||
      rows > INT32_MAX / 16 || 2 * d_inner + 2 * gds + nheads > INT32_MAX)
    return SN_ERR_UNSUPPORTED;
  sn::ConvSsuParams p;
  p.zx = static_cast<const __nv_bfloat16*>(zxbcdt);
  p.ld = ld;
  p.conv_state = static_cast<__nv_bfloat16*>(conv_state);
  p.w = static_cast<const __nv_bfloat16*>(conv_weight);
  p.bias = static_cast<const __nv_bfloat16*>(conv_bias);
  p.state = static_cast<__nv_bfloat16*>(ssm_state);
  p.A = A;
  p.D = static_cast<const __nv_bfloat16*>(D);
  p.dt_bias = static_cast<const __nv_bfloat16*>(dt_bias);
  p.z = static_cast<__nv_bfloat16*>(z);
  p.y = static_cast<__nv_bfloat16*>(y);
  p.sync = sync;
  p.di = d_inner;
  p.gds = static_cast<int>(gds);
  p.ds = d_state;
  p.ng = ngroups;
  p.nh = nheads;
  p.hd = headdim;
  p.hpg = nheads / ngroups;
  p.W = d_conv;
  p.bpg = p.hpg * headdim / 16;
  const dim3 grid(static_cast<unsigned>(rows / 16));
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  return d_state == 128 ? sn::launch(sn::mamba2_conv_ssu_kernel<1>, grid, dim3(256), 0, st, true, p)
                        : sn::launch(sn::mamba2_conv_ssu_kernel<2>, grid, dim3(256), 0, st, true, p);
}

int sn_rotary_kv_append(const void* qkv, void* q, void* k_cache, void* v_cache, const float* cos, const float* sin,
                        int batch, int nheads, int nheads_kv, int head_dim, int max_seqlen, int pos, void* stream) {
  if (!qkv || !q || !k_cache || !v_cache || !cos || !sin || batch < 1 || nheads < 1 || nheads_kv < 1 ||
      head_dim < 2 || head_dim % 2 != 0 || max_seqlen < 1 || pos < 0 || pos >= max_seqlen)
    return SN_ERR_INVALID_ARGUMENT;
  sn::RotaryParams p;
  p.qkv = static_cast<const __nv_bfloat16*>(qkv);
  p.q = static_cast<__nv_bfloat16*>(q);
  p.kc = static_cast<__nv_bfloat16*>(k_cache);
  p.vc = static_cast<__nv_bfloat16*>(v_cache);
  p.cos = cos;
  p.sin = sin;
  p.batch = batch;
  p.hq = nheads;
  p.hk = nheads_kv;
  p.hd = head_dim;
  p.S = max_seqlen;
  p.pos = pos;
  const int64_t n = static_cast<int64_t>(batch) * (nheads + 2 * nheads_kv) * (head_dim / 2);
  return sn::launch(sn::rotary_kv_append_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), true, p);
}

int sn_swiglu(const void* h, void* y, int batch, int d, void* stream) {
  if (!h || !y || batch < 1 || d < 1) return SN_ERR_INVALID_ARGUMENT;
  const int64_t n = static_cast<int64_t>(batch) * d;
  return sn::launch(sn::swiglu_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), true, static_cast<const __nv_bfloat16*>(h),
                    static_cast<__nv_bfloat16*>(y), batch, d);
}

}  // extern "C"
