// Fused Snake + Conv1d on B200 tensor cores.
//
// Replaces _fused_snake_conv1d_kernel (kernels/fused_snake_conv.py:29-131):
//   y[b, o, t] = bias[o] + sum_{i,k} W[o, i, k] * snake(x[b, i, t*s - p + k*d])
//   snake(v)   = v + sin(alpha_i v)^2 / (alpha_i + eps),   zero outside [0, T)
// The reference evaluates sin once per (output, input, tap); here every input
// element is activated once per CTA tile and reused by all taps and output
// channels of the tile.
//
// Fast path (stride 1, K <= 7, (K-1)*d <= 72, Cin and Cout multiples of 16):
// an implicit GEMM per batch row,  Y[t, o] = sum_k sum_i S[t - p + k*d, i] W_k[o, i]
//   * UMMA M = 128 output times, N = an output-channel tile (<= 256), K = input
//     channels in chunks of 64;
//   * 8 producer warps load x (coalesced along time), apply snake in fp32 and
//     store the activation as K-major bf16 hi/lo pairs in the 128-byte-swizzled
//     layout, (128 + (K-1)*d) rows per chunk; tap k reads the same buffer
//     through a descriptor whose start is k*d rows further (the hardware
//     applies the swizzle to the absolute shared-memory address, so any row
//     offset addresses the rows TMA-style writes left there);
//   * weights are packed once per call into bf16 hi/lo planes [K][2][Cout][Cin]
//     and streamed per tap by TMA;
//   * split-precision products hi*hi + lo*hi + hi*lo (three kind::f16 MMAs)
//     accumulate in fp32 TMEM: about 2^-16 relative error per product, far
//     inside the 2e-3 max-abs gate, at 1.5x the cost of a tf32 MMA;
//   * epilogue: TMEM -> registers, + bias, stores coalesced along time.
// Any other shape runs the fallback: one thread per output, the reference's
// loop order (correct for every stride / padding / dilation / kernel size).
#include "tc.cuh"

#include <algorithm>
#include <climits>
#include <cstring>
#include <cstdlib>
#include <cstdint>

namespace sn {
namespace {

constexpr int kScProducerWarps = 8;
constexpr int kScEpilogueWarps = 8;  // two per TMEM lane quarter, half the columns each
constexpr int kScThreads = (2 + kScProducerWarps + kScEpilogueWarps) * 32;  // TMA, MMA, producers, epilogue
constexpr int kScWStages = 2;
// x tiles by TMA (convolutions without a halo: 128 activation rows): two
// fp32 staging buffers of [64 channels][128 rows], filled by the weight
// producer's thread and read by the snake producers from shared memory
constexpr int kScXStages = 2;
constexpr uint32_t kScXBytes = 64 * 128 * 4;
constexpr int kScPairWStages = 2;  // weight stages in the CTA-pair kernel (4 measured no faster)
constexpr int kMaxTaps = 7;
constexpr int kMaxRowIters = 7;  // activation rows per chunk <= 32 * 7 = 224 ((K-1)*d <= 72)

struct ScParams {
  const float* x;      // [B, Cin, T]
  const float* alpha;  // [Cin]
  const float* bias;   // [Cout] or nullptr
  float* y;            // [B, Cout, Tout]
  int B, Cin, Cout, T, Tout, K, pad, dil;
  float eps;
  int nt;              // output channels per tile (UMMA N, multiple of 32)
  int ntiles_o, ntiles_t, ntiles;
  int rows;            // activation rows per chunk (128 + (K-1)*d, rounded up to 8)
  uint32_t a_bytes;    // one activation plane (rows * 128)
  uint32_t w_bytes;    // one weight plane (nt * 128)
  uint32_t tcols;      // TMEM columns per accumulator buffer
  int ntiles_t2, ntiles2;  // CTA-pair kernel: 256-row time tiles and pair tiles
  // epilogue / activation variants
  const float* res;    // [B, Cout, Tout] added to the output (DAC residual unit), or nullptr
  int act;             // SN_ACT_SNAKE or SN_ACT_NONE (the producers store x itself)
  int post;            // SN_POST_NONE or SN_POST_TANH (applied last)
  // transposed convolution as a polyphase GEMM (up_s > 0): GEMM column
  // o' = o * up_s + r, row q holds y[b, o, up_s * q + r - up_p]; y is
  // [B, Cy, Ty].  up_s == 0: plain convolution, column o, row t of y[b, o, t].
  int up_s, up_p, Cy, Ty;
  int up_sh;  // log2(up_s) when up_s is a power of two (every DAC stride), else -1
  int up_vec;          // widest vector store (1, 2 or 4 floats) the phase runs of y allow
  int x_tma;           // 1: the x tiles arrive by TMA into shared staging (no halo, aligned x)
  // element strides of the batch and channel (row) dimensions; time is
  // contiguous.  Whole tensors: x (Cin * T, T), y and res (Cy * Ty, Ty); a
  // streaming decoder passes windows of larger per-layer buffers.
  int64_t x_bs, x_ld, y_bs, y_ld, r_bs, r_ld;
};

// Pull a tile's residual (GEMM rows t0 .. t0 + 127, columns o0 .. o0 + nt - 1)
// into L2 while its MMAs run, so that the epilogue's reads hit L2: one
// 128-byte line per (channel, 32-row segment), spread over the epilogue
// threads (et = 0 .. 32 * kScEpilogueWarps - 1).
__device__ __forceinline__ void sc_prefetch_res(const ScParams& p, int b, int t0, int o0, int et) {
  if (!p.res || p.up_s != 0) return;
  const float* rb = p.res + static_cast<int64_t>(b) * p.r_bs;
  for (int l = et; l < p.nt * 4; l += 32 * kScEpilogueWarps) {
    const int o = o0 + (l >> 2), t = t0 + 32 * (l & 3);
    if (o < p.Cy && t < p.Tout)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(rb + static_cast<int64_t>(o) * p.r_ld + t));
  }
}

// The epilogue works on 16 GEMM columns of GEMM row t (output time, or
// polyphase row q) at a time: sc_load_bias16 / sc_load_res16 read the chunk's
// bias and residual values, sc_emit16 adds them to the accumulator values,
// applies the post-op and stores to y (plain stores are coalesced along time
// across the warp).  Every read of a chunk is issued before the chunk's first
// store: y may alias the bias and residual as far as the compiler knows, so a
// read placed after a store would wait out its whole latency once per element
// (measured: the epilogue then bounds the kernel for Cout <= 192).
struct ScChunk {
  float bv[16], rv[16];
};

template <bool UP>
__device__ __forceinline__ void sc_load_bias16(const ScParams& p, int o_base, float (&bv)[16]) {
  if constexpr (!UP) {
#pragma unroll
    for (int e = 0; e < 16; ++e) bv[e] = (p.bias && o_base + e < p.Cy) ? __ldg(p.bias + o_base + e) : 0.f;
  } else {
#pragma unroll
    for (int e = 0; e < 16; ++e)
      bv[e] = (p.bias && o_base + e < p.Cout)
                  ? __ldg(p.bias + (p.up_sh >= 0 ? (o_base + e) >> p.up_sh : (o_base + e) / p.up_s))
                  : 0.f;
  }
}

__device__ __forceinline__ void sc_load_res16(const ScParams& p, int b, int t, int o_base, float (&rv)[16]) {
#pragma unroll
  for (int e = 0; e < 16; ++e) rv[e] = 0.f;
  if (p.res && p.up_s == 0 && t < p.Tout) {
    const float* rb = p.res + static_cast<int64_t>(b) * p.r_bs;
#pragma unroll
    for (int e = 0; e < 16; ++e)
      if (o_base + e < p.Cy) rv[e] = __ldg(rb + static_cast<int64_t>(o_base + e) * p.r_ld + t);
  }
}

// Polyphase store for a stride S dividing 16: the chunk covers 16 / S whole
// output channels, whose S phases of row t are S consecutive output times
// starting at S * t - padding, written as up_vec-float vectors away from the
// edges.
template <int S>
__device__ __forceinline__ void sc_emit16_phases(const ScParams& p, float* yb, int t, int o_base,
                                                 const float (&vv)[16], const ScChunk& c) {
  constexpr int G = 16 / S;
  const int o_first = o_base / S;
  const int ty0 = S * t - p.up_p;
  const bool inside = ty0 >= 0 && ty0 + S <= p.Ty;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int o = o_first + g;
    if (o >= p.Cy) break;
    float w[S];
#pragma unroll
    for (int r = 0; r < S; ++r) {
      w[r] = vv[g * S + r] + c.bv[g * S + r];
      if (p.post == SN_POST_TANH) w[r] = tanhf(w[r]);
    }
    float* dst = yb + static_cast<int64_t>(o) * p.y_ld + ty0;
    if constexpr (S % 4 == 0) {
      if (inside && p.up_vec == 4) {
#pragma unroll
        for (int r = 0; r < S; r += 4) *reinterpret_cast<float4*>(dst + r) = make_float4(w[r], w[r + 1], w[r + 2], w[r + 3]);
        continue;
      }
    }
    if constexpr (S % 2 == 0) {
      if (inside && p.up_vec >= 2) {
#pragma unroll
        for (int r = 0; r < S; r += 2) *reinterpret_cast<float2*>(dst + r) = make_float2(w[r], w[r + 1]);
        continue;
      }
    }
#pragma unroll
    for (int r = 0; r < S; ++r)
      if (ty0 + r >= 0 && ty0 + r < p.Ty) dst[r] = w[r];
  }
}

template <bool UP>
__device__ __forceinline__ void sc_emit16(const ScParams& p, int b, int t, int o_base, const float (&vv)[16],
                                          const ScChunk& c) {
  if (t >= p.Tout) return;
  if constexpr (!UP) {
    float* yb = p.y + static_cast<int64_t>(b) * p.y_bs;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const int o = o_base + e;
      if (o < p.Cy) {
        float v = vv[e] + c.bv[e] + c.rv[e];
        if (p.post == SN_POST_TANH) v = tanhf(v);
        yb[static_cast<int64_t>(o) * p.y_ld + t] = v;
      }
    }
  } else {
    float* yb = p.y + static_cast<int64_t>(b) * p.y_bs;
    switch (p.up_s) {  // the DAC strides; o_base is a multiple of 16
      case 2: sc_emit16_phases<2>(p, yb, t, o_base, vv, c); return;
      case 4: sc_emit16_phases<4>(p, yb, t, o_base, vv, c); return;
      case 8: sc_emit16_phases<8>(p, yb, t, o_base, vv, c); return;
      default: break;
    }
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const int oc = o_base + e;
      if (oc < p.Cout) {
        const int o = oc / p.up_s, r = oc - o * p.up_s;
        const int ty = p.up_s * t + r - p.up_p;
        if (ty >= 0 && ty < p.Ty) {
          float v = vv[e] + c.bv[e];
          if (p.post == SN_POST_TANH) v = tanhf(v);
          yb[static_cast<int64_t>(o) * p.y_ld + ty] = v;
        }
      }
    }
  }
}

// One tile's epilogue: this thread's row (its TMEM lane), half of the tile's
// nt accumulator columns.
// With a residual (HBM reads) chunk c + 1's residual is read before chunk c is
// stored; bias reads (L1 hits) go just before their own chunk's stores.
template <bool UP>
__device__ __forceinline__ void sc_epilogue_tile(const ScParams& p, uint32_t base, int b, int t, int o0) {
  ScChunk c;
  float rnext[16];
  const bool res = !UP && p.res;
  // the two warps of a lane quarter take one half of the tile's columns each
  const int half = (threadIdx.x - 32 * (2 + kScProducerWarps)) / (32 * 4);
  const int ccb = half * (p.nt / 2), cce = ccb + p.nt / 2;
  if (res) sc_load_res16(p, b, t, o0 + ccb, rnext);
  for (int cc = ccb; cc < cce; cc += 16) {
    float vv[16];
    tc::tmem_ld16(base + cc, vv);
    if (res) {
#pragma unroll
      for (int e = 0; e < 16; ++e) c.rv[e] = rnext[e];
      if (cc + 16 < cce) sc_load_res16(p, b, t, o0 + cc + 16, rnext);
    } else {
#pragma unroll
      for (int e = 0; e < 16; ++e) c.rv[e] = 0.f;
    }
    sc_load_bias16<UP>(p, o0 + cc, c.bv);
    sc_emit16<UP>(p, b, t, o0 + cc, vv, c);
  }
}

// sin(y)^2 for the Snake activation, accurate for arguments of any size.
// sin^2 has period pi, so y is first reduced to r = y - n*pi, n = rint(y/pi),
// |r| <= pi/2, by Cody and Waite's method (W. J. Cody and W. Waite, Software
// Manual for the Elementary Functions, 1980): pi is split into three fp32
// parts PI_A + PI_B + PI_C (the fp32 value of pi, then the fp32 values of the
// two successive remainders) and each n * part is subtracted with one FMA.
// For n != 0, |y| >= pi/2 > 1, so y is a multiple of 2^-23 and n * PI_A of
// 2^-21: the first difference is exact.  The hardware approximation __sinf
// is then only evaluated on |r| <= pi/2, where its absolute error is about
// 2^-21; applied to a large y directly its error grows with |y|.
__device__ __forceinline__ float snake_sin2(float y) {
  constexpr float kInvPi = 0x1.45f306p-2f;
  constexpr float kPiA = 0x1.921fb6p+1f;
  constexpr float kPiB = -0x1.777a5cp-24f;
  constexpr float kPiC = -0x1.ee59dap-49f;
  const float n = rintf(y * kInvPi);
  float r = fmaf(-n, kPiA, y);
  r = fmaf(-n, kPiB, r);
  r = fmaf(-n, kPiC, r);
  const float sv = __sinf(r);
  return sv * sv;
}

// snake(v) = v + sin(alpha v)^2 / (alpha + eps), with inv = 1 / (alpha + eps)
__device__ __forceinline__ float snake_value(float v, float alpha, float inv) {
  return fmaf(snake_sin2(alpha * v), inv, v);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const uint32_t a = __bfloat16_as_ushort(__float2bfloat16_rn(lo));
  const uint32_t b = __bfloat16_as_ushort(__float2bfloat16_rn(hi));
  return a | (b << 16);
}

// Persistent: CTA c handles tiles c, c + G, c + 2G, ...; every role walks its
// own sequence (tiles x chunks x taps) and every mbarrier phase in order.
//   warp 0      TMA of the weight planes, one (hi, lo) pair per (chunk, tap)
//   warp 1      TMEM owner; lane 0 issues the MMAs into accumulator (j & 1)
//   warps 2-9   snake producers (activation buffer g & 1 for chunk g)
//   warps 10-13 epilogue: drain accumulator (j & 1) while tile j+1 computes
// UP: the polyphase (transposed-convolution) epilogue, compiled separately so
// that the plain convolutions carry none of its code.
template <bool UP>
__global__ void __launch_bounds__(kScThreads, 1)
    snake_conv_mma_kernel(const __grid_constant__ CUtensorMap mapW, const __grid_constant__ CUtensorMap mapX,
                          const ScParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // layout: [A0 hi][A0 lo][A1 hi][A1 lo][W0 hi][W0 lo][W1 hi][W1 lo][X0][X1 (x_tma only)][barriers]
  uint8_t* abuf = smem;
  uint8_t* wbuf = smem + 4 * p.a_bytes;
  uint8_t* xstage = wbuf + 2 * kScWStages * p.w_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(xstage + (p.x_tma ? kScXStages * kScXBytes : 0u));
  uint64_t* a_full = bars;
  uint64_t* a_empty = bars + 2;
  uint64_t* w_full = bars + 4;
  uint64_t* w_empty = w_full + kScWStages;
  uint64_t* t_full = w_empty + kScWStages;
  uint64_t* t_empty = t_full + 2;
  uint64_t* x_full = t_empty + 2;           // [kScXStages]
  uint64_t* x_empty = x_full + kScXStages;  // [kScXStages]: every producer warp has read the tile
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(x_empty + kScXStages);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nchunks = (p.Cin + 63) / 64;
  const int my_tiles = p.ntiles > static_cast<int>(blockIdx.x)
                           ? (p.ntiles - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                           : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(a_full + i, kScProducerWarps);
      mbar_init(a_empty + i, 1);
      mbar_init(t_full + i, 1);
      mbar_init(t_empty + i, kScEpilogueWarps);
    }
    for (int i = 0; i < kScWStages; ++i) {
      mbar_init(w_full + i, 1);
      mbar_init(w_empty + i, 1);
    }
    for (int i = 0; i < kScXStages; ++i) {
      mbar_init(x_full + i, 1);
      mbar_init(x_empty + i, kScProducerWarps);
    }
    fence_barrier_init();
    tc::prefetch_map(&mapW);
    if (p.x_tma) tc::prefetch_map(&mapX);
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, 2 * p.tcols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  auto tile_coords = [&](int j, int& b, int& t0, int& o0) {
    int u = static_cast<int>(blockIdx.x) + j * static_cast<int>(gridDim.x);
    const int ot = u % p.ntiles_o;
    u /= p.ntiles_o;
    const int tt = u % p.ntiles_t;
    b = u / p.ntiles_t;
    t0 = tt * 128;
    o0 = ot * p.nt;
  };

  if (warp == 0) {
    // ---------------- weight TMA ----------------
    if (lane == 0) {
      const int total = my_tiles * nchunks * p.K;
      // (tap, chunk, tile) of stage q, kept incrementally: run-time
      // divisions here cost the single producer thread ~0.1 us each
      int q = 0, tap = 0, c = 0, j = 0, b = 0, t0 = 0, o0 = 0;
      int gx = 0;  // x tiles issued (one per chunk, before the chunk's first weight stage)
      if (total > 0) tile_coords(0, b, t0, o0);
      for (; q < total; ++q) {
        if (p.x_tma && tap == 0) {
          // chunk gx's x tile: 64 channels from c * 64, rows t0 .. t0 + 127 (no
          // halo: the time coordinate is t0, a multiple of 128); channels and
          // times past the tensor read as zero
          const int xs = gx & (kScXStages - 1);
          if (gx >= kScXStages && !mbar_wait_bounded(x_empty + xs, ((gx / kScXStages) - 1) & 1)) {
            record_status(SN_ERR_TIMEOUT);
            break;
          }
          // a tile wholly past T (the odd CTA of a pair at the end) reads the
          // last 128-row block instead: its rows are computed but never stored
          const int tx = t0 < p.T ? t0 : (p.T - 1) / 128 * 128;
          mbar_arrive_expect_tx(x_full + xs, kScXBytes);
          tc::tma_load_3d(xstage + static_cast<size_t>(xs) * kScXBytes, &mapX, tx, c * 64, b, x_full + xs);
          ++gx;
        }
        const int s = q % kScWStages, k = q / kScWStages;
        if (k > 0 && !mbar_wait_bounded(w_empty + s, (k - 1) & 1)) {
          record_status(SN_ERR_TIMEOUT);
          break;
        }
        uint8_t* dst = wbuf + static_cast<size_t>(s) * 2 * p.w_bytes;
        mbar_arrive_expect_tx(w_full + s, 2 * p.w_bytes);
        tc::tma_load_3d(dst, &mapW, c * 64, o0, tap * 2 + 0, w_full + s);
        tc::tma_load_3d(dst + p.w_bytes, &mapW, c * 64, o0, tap * 2 + 1, w_full + s);
        if (++tap == p.K) {
          tap = 0;
          if (++c == nchunks) {
            c = 0;
            if (++j < my_tiles) tile_coords(j, b, t0, o0);
          }
        }
      }
      if (q < total) {  // error path: let issued copies land before exit
        for (int j = (q > kScWStages ? q - kScWStages : 0); j < q; ++j)
          mbar_wait_bounded(w_full + j % kScWStages, (j / kScWStages) & 1);
      }
      // the last x tiles have landed before the CTA can exit (the producers
      // wait for them too unless they stopped early)
      for (int v = (gx > kScXStages ? gx - kScXStages : 0); v < gx; ++v)
        mbar_wait_bounded(x_full + (v & (kScXStages - 1)), (v / kScXStages) & 1);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_bf16_f32(128, p.nt);
      bool ok = true;
      int q = 0, g = 0;
      for (int j = 0; j < my_tiles && ok; ++j) {
        const int tb = j & 1;
        if (j >= 2 && !mbar_wait_bounded(t_empty + tb, ((j >> 1) - 1) & 1)) {
          record_status(SN_ERR_TIMEOUT);
          break;
        }
        tc::fence_after_sync();
        const uint32_t acc_tmem = tmem + static_cast<uint32_t>(tb) * p.tcols;
        for (int c = 0; c < nchunks && ok; ++c, ++g) {
          const int ab = g & 1;
          if (!mbar_wait_bounded(a_full + ab, (g >> 1) & 1)) {
            record_status(SN_ERR_TIMEOUT);
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const int ksteps = min(4, (p.Cin - c * 64) / 16);  // 16-channel MMA steps in this chunk
          const uint64_t a_hi = tc::smem_desc_sw128(abuf + (2 * ab + 0) * p.a_bytes);
          const uint64_t a_lo = tc::smem_desc_sw128(abuf + (2 * ab + 1) * p.a_bytes);
          for (int tap = 0; tap < p.K; ++tap, ++q) {
            const int s = q % kScWStages;
            if (!mbar_wait_bounded(w_full + s, (q / kScWStages) & 1)) {
              record_status(SN_ERR_TIMEOUT);
              ok = false;
              break;
            }
            tc::fence_after_sync();
            const uint8_t* w = wbuf + static_cast<size_t>(s) * 2 * p.w_bytes;
            const uint64_t w_hi = tc::smem_desc_sw128(w), w_lo = tc::smem_desc_sw128(w + p.w_bytes);
            const uint64_t shift = static_cast<uint64_t>(tap * p.dil * 128) >> 4;  // tap rows further on
            for (int kk = 0; kk < ksteps; ++kk) {
              const uint32_t acc0 = (c | tap | kk) != 0;
              tc::mma_bf16(acc_tmem, a_hi + shift + 2 * kk, w_hi + 2 * kk, idesc, acc0);
              tc::mma_bf16(acc_tmem, a_lo + shift + 2 * kk, w_hi + 2 * kk, idesc, 1);
              tc::mma_bf16(acc_tmem, a_hi + shift + 2 * kk, w_lo + 2 * kk, idesc, 1);
            }
            tc::mma_commit(w_empty + s);
          }
          tc::mma_commit(a_empty + ab);
        }
        tc::mma_commit(t_full + tb);
      }
    }
  } else if (warp < 2 + kScProducerWarps) {
    // ---------------- snake producers ----------------
    const int pw = warp - 2;  // the 8-channel group of every chunk this warp fills
    int g = 0;
    for (int j = 0; j < my_tiles; ++j) {
      int b, t0, o0;
      tile_coords(j, b, t0, o0);
      const float* xb = p.x + static_cast<int64_t>(b) * p.x_bs;
      const int tin0 = t0 - p.pad;  // input time of activation row 0
      for (int c = 0; c < nchunks; ++c, ++g) {
        const int ab = g & 1;
        const int i0 = c * 64 + pw * 8;  // first input channel of this warp's group
        float v[kMaxRowIters][8];
        if (p.x_tma) {
          // the chunk's x tile is in staging buffer g mod kScXStages, [channel][row]
          const int xs = g & (kScXStages - 1);
          if (!__all_sync(0xffffffffu, mbar_wait_bounded(x_full + xs, (g / kScXStages) & 1))) {
            record_status(SN_ERR_TIMEOUT);
            j = my_tiles;  // unwind
            break;
          }
          const float* xt = reinterpret_cast<const float*>(xstage + static_cast<size_t>(xs) * kScXBytes);
#pragma unroll
          for (int it = 0; it < kMaxRowIters; ++it) {
            const int r = lane + 32 * it;
#pragma unroll
            for (int e = 0; e < 8; ++e) v[it][e] = (r < 128) ? xt[(pw * 8 + e) * 128 + r] : 0.f;
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(x_empty + xs);  // this warp is done with the staging buffer
        } else {
          {
            // pull the next chunk's x lines (this warp's 8 channels x rows) into L2
            // while this chunk's loads are outstanding: one 128-byte line per lane
            // and (channel, 32-row step) pair
            int nb = b, nt0 = tin0, ni0 = i0 + 64;
            if (c + 1 == nchunks) {
              int t1, o1;
              if (j + 1 < my_tiles) {
                tile_coords(j + 1, nb, t1, o1);
                nt0 = t1 - p.pad;
              }
              ni0 = pw * 8;
            }
            const bool more = (c + 1 < nchunks) || (j + 1 < my_tiles);
            const float* nxb = p.x + static_cast<int64_t>(nb) * p.x_bs;
  #pragma unroll
            for (int k = lane; k < 8 * kMaxRowIters; k += 32) {
              const int e = k & 7, it = k >> 3;
              const int tin = max(nt0 + 32 * it, 0);
              if (more && ni0 + e < p.Cin && 32 * it < p.rows && tin < p.T)
                asm volatile("prefetch.global.L2 [%0];" ::"l"(nxb + static_cast<int64_t>(ni0 + e) * p.x_ld + tin));
            }
          }
          // issue every x load of this chunk before the first use (memory-level
          // parallelism: 8 channels x up to 7 rows per lane in flight)
  #pragma unroll
          for (int it = 0; it < kMaxRowIters; ++it) {
            const int r = lane + 32 * it;
            const int tin = tin0 + r;
            const bool in_t = r < p.rows && tin >= 0 && tin < p.T;
  #pragma unroll
            for (int e = 0; e < 8; ++e)
              v[it][e] = (in_t && i0 + e < p.Cin) ? __ldg(xb + static_cast<int64_t>(i0 + e) * p.x_ld + tin) : 0.f;
          }
        }
        float al[8], inv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          al[e] = (p.act == SN_ACT_SNAKE && i0 + e < p.Cin) ? __ldg(p.alpha + i0 + e) : 0.f;
          inv[e] = 1.0f / (al[e] + p.eps);
        }
        if (g >= 2 && !__all_sync(0xffffffffu, mbar_wait_bounded(a_empty + ab, ((g >> 1) - 1) & 1))) {
          record_status(SN_ERR_TIMEOUT);
          j = my_tiles;  // unwind
          break;
        }
        uint8_t* ahi = abuf + (2 * ab + 0) * p.a_bytes;
        uint8_t* alo = abuf + (2 * ab + 1) * p.a_bytes;
#pragma unroll
        for (int it = 0; it < kMaxRowIters; ++it) {
          const int r = lane + 32 * it;
          if (r < p.rows) {
            float hi[8], lo[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              float s = v[it][e];
              if (p.act == SN_ACT_SNAKE) s = snake_value(s, al[e], inv[e]);  // snake(0) == 0
              hi[e] = __bfloat162float(__float2bfloat16_rn(s));
              lo[e] = s - hi[e];
            }
            // 16-byte chunk pw of row r, XOR-swizzled with the row's low 3 bits
            const uint32_t off =
                static_cast<uint32_t>(r) * 128u + ((static_cast<uint32_t>(pw) ^ (r & 7)) << 4);
            *reinterpret_cast<uint4*>(ahi + off) = make_uint4(pack_bf16x2(hi[0], hi[1]), pack_bf16x2(hi[2], hi[3]),
                                                              pack_bf16x2(hi[4], hi[5]), pack_bf16x2(hi[6], hi[7]));
            *reinterpret_cast<uint4*>(alo + off) = make_uint4(pack_bf16x2(lo[0], lo[1]), pack_bf16x2(lo[2], lo[3]),
                                                              pack_bf16x2(lo[4], lo[5]), pack_bf16x2(lo[6], lo[7]));
          }
        }
        tc::fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core
        __syncwarp();
        if (lane == 0) mbar_arrive(a_full + ab);
      }
    }
  } else {
    // ---------------- epilogue ----------------
    const int q4 = warp & 3;  // a warp may only read TMEM lanes 32*(warp id % 4) ..
    for (int j = 0; j < my_tiles; ++j) {
      const int tb = j & 1;
      {
        int b, t0, o0;
        tile_coords(j, b, t0, o0);
        sc_prefetch_res(p, b, t0, o0, threadIdx.x - 32 * (2 + kScProducerWarps));
      }
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(t_full + tb, (j >> 1) & 1))) {
        record_status(SN_ERR_TIMEOUT);
        break;
      }
      tc::fence_after_sync();
      int b, t0, o0;
      tile_coords(j, b, t0, o0);
      const int t = t0 + q4 * 32 + lane;
      const uint32_t base = tmem + (static_cast<uint32_t>(q4 * 32) << 16) + static_cast<uint32_t>(tb) * p.tcols;
      sc_epilogue_tile<UP>(p, base, b, t, o0);
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(t_empty + tb);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) tc::tmem_dealloc(tmem, 2 * p.tcols);
}

// ---------------------------------------------------------------------------
// CTA-pair variant (cta_group::2).  A cluster of two CTAs computes a tile of
// 256 output times x nt output channels with M = 256 MMAs: CTA r owns time
// rows [128 r, 128 r + 128) of the tile (its own snake producers, activation
// buffers, TMEM accumulator rows and epilogue) and holds nt / 2 rows of each
// weight plane; the even CTA issues the MMAs, which read both CTAs' shared
// memory.  Every weight byte read by the tensor core now feeds 256 rows
// instead of 128, which is what bounds the single-CTA kernel (operand reads).
// Synchronisation: producers and epilogue warps of the odd CTA arrive on the
// even CTA's barriers remotely (release / acquire at cluster scope); weight
// TMA of both CTAs completes on the even CTA's barrier; MMA commits are
// multicast to the same barrier offset in both CTAs.  Every wait is bounded,
// and a cluster barrier at exit keeps each CTA alive while its peer may
// still read its shared memory.
// ---------------------------------------------------------------------------
template <bool UP>
__global__ void __launch_bounds__(kScThreads, 1)
    snake_conv_pair_kernel(const __grid_constant__ CUtensorMap mapW, const __grid_constant__ CUtensorMap mapX,
                           const ScParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // layout: [A0 hi][A0 lo][A1 hi][A1 lo][W0 hi/2][W0 lo/2][W1 hi/2][W1 lo/2][X0][X1 (x_tma only)][barriers]
  const uint32_t wh = p.w_bytes / 2;  // this CTA's half of one weight plane
  uint8_t* abuf = smem;
  uint8_t* wbuf = smem + 4 * p.a_bytes;
  uint8_t* xstage = wbuf + 2 * kScPairWStages * wh;
  uint64_t* bars = reinterpret_cast<uint64_t*>(xstage + (p.x_tma ? kScXStages * kScXBytes : 0u));
  uint64_t* a_full = bars;        // even CTA: both CTAs' producers
  uint64_t* a_empty = bars + 2;   // both CTAs: MMA commit
  uint64_t* w_full = bars + 4;    // even CTA: both CTAs' weight bytes
  uint64_t* w_empty = w_full + kScPairWStages;  // both CTAs: MMA commit
  uint64_t* t_full = w_empty + kScPairWStages;  // both CTAs: MMA commit
  uint64_t* t_empty = t_full + 2;           // even CTA: both CTAs' epilogues
  uint64_t* x_full = t_empty + 2;           // this CTA's x staging (local barriers)
  uint64_t* x_empty = x_full + kScXStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(x_empty + kScXStages);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = tc::cluster_ctarank();
  const int pair = static_cast<int>(blockIdx.x >> 1), npairs = static_cast<int>(gridDim.x >> 1);
  const int nchunks = (p.Cin + 63) / 64;
  const int my_tiles = p.ntiles2 > pair ? (p.ntiles2 - 1 - pair) / npairs + 1 : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(a_full + i, 2 * kScProducerWarps);
      mbar_init(a_empty + i, 1);
      mbar_init(t_full + i, 1);
      mbar_init(t_empty + i, 2 * kScEpilogueWarps);
    }
    for (int i = 0; i < kScPairWStages; ++i) {
      mbar_init(w_full + i, 1);
      mbar_init(w_empty + i, 1);
    }
    for (int i = 0; i < kScXStages; ++i) {
      mbar_init(x_full + i, 1);
      mbar_init(x_empty + i, kScProducerWarps);
    }
    fence_barrier_init();
    tc::prefetch_map(&mapW);
    if (p.x_tma) tc::prefetch_map(&mapX);
  }
  if (warp == 1) tc::tmem_alloc_pair(tmem_slot, 2 * p.tcols);
  tc::fence_before_sync();
  __syncthreads();
  tc::cluster_sync_all();  // both CTAs' barriers and TMEM exist before any remote use
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  // the even CTA's barriers, addressed from either CTA
  const uint32_t a_full0 = tc::mapa_shared(smem_u32(a_full), 0);
  const uint32_t w_full0 = tc::mapa_shared(smem_u32(w_full), 0);
  const uint32_t t_empty0 = tc::mapa_shared(smem_u32(t_empty), 0);

  // pair tile j of this cluster -> batch, first time of THIS CTA's rows, first output channel
  auto tile_coords = [&](int j, int& b, int& t0, int& o0) {
    int u = pair + j * npairs;
    const int ot = u % p.ntiles_o;
    u /= p.ntiles_o;
    const int tt = u % p.ntiles_t2;
    b = u / p.ntiles_t2;
    t0 = tt * 256 + static_cast<int>(rank) * 128;
    o0 = ot * p.nt;
  };

  if (warp == 0) {
    // ---------------- weight TMA: this CTA's half of each (chunk, tap) ----------
    if (lane == 0) {
      const int total = my_tiles * nchunks * p.K;
      // (tap, chunk, tile) of stage q, kept incrementally (no divisions)
      int q = 0, tap = 0, c = 0, j = 0, b = 0, t0 = 0, o0 = 0;
      int gx = 0;  // x tiles issued (one per chunk, before the chunk's first weight stage)
      if (total > 0) tile_coords(0, b, t0, o0);
      for (; q < total; ++q) {
        if (p.x_tma && tap == 0) {
          // chunk gx's x tile for this CTA's 128 rows (t0: a multiple of 128, no halo)
          const int xs = gx & (kScXStages - 1);
          if (gx >= kScXStages && !mbar_wait_bounded(x_empty + xs, ((gx / kScXStages) - 1) & 1)) {
            record_status(SN_ERR_TIMEOUT);
            break;
          }
          // a tile wholly past T (the odd CTA of a pair at the end) reads the
          // last 128-row block instead: its rows are computed but never stored
          const int tx = t0 < p.T ? t0 : (p.T - 1) / 128 * 128;
          mbar_arrive_expect_tx(x_full + xs, kScXBytes);
          tc::tma_load_3d(xstage + static_cast<size_t>(xs) * kScXBytes, &mapX, tx, c * 64, b, x_full + xs);
          ++gx;
        }
        const int s = q % kScPairWStages, k = q / kScPairWStages;
        if (k > 0 && !mbar_wait_bounded(w_empty + s, (k - 1) & 1)) {
          record_status(SN_ERR_TIMEOUT);
          break;
        }
        uint8_t* dst = wbuf + static_cast<size_t>(s) * 2 * wh;
        if (rank == 0) mbar_arrive_expect_tx(w_full + s, 4 * wh);  // both halves of both planes
        const int orow = o0 + static_cast<int>(rank) * (p.nt / 2);
        tc::tma_load_3d_pair(dst, &mapW, c * 64, orow, tap * 2 + 0, w_full0 + 8u * s);
        tc::tma_load_3d_pair(dst + wh, &mapW, c * 64, orow, tap * 2 + 1, w_full0 + 8u * s);
        if (++tap == p.K) {
          tap = 0;
          if (++c == nchunks) {
            c = 0;
            if (++j < my_tiles) tile_coords(j, b, t0, o0);
          }
        }
      }
      for (int v = (gx > kScXStages ? gx - kScXStages : 0); v < gx; ++v)  // the last x tiles have landed
        mbar_wait_bounded(x_full + (v & (kScXStages - 1)), (v / kScXStages) & 1);
      (void)q;
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (even CTA) ----------------
    if (lane == 0 && rank == 0) {
      const uint32_t idesc = tc::idesc_bf16_f32(256, p.nt);
      bool ok = true;
      int q = 0, g = 0;
      for (int j = 0; j < my_tiles && ok; ++j) {
        const int tb = j & 1;
        if (j >= 2 && !tc::mbar_wait_cluster_bounded(t_empty + tb, ((j >> 1) - 1) & 1)) {
          record_status(SN_ERR_TIMEOUT);
          break;
        }
        tc::fence_after_sync();
        const uint32_t acc_tmem = tmem + static_cast<uint32_t>(tb) * p.tcols;
        for (int c = 0; c < nchunks && ok; ++c, ++g) {
          const int ab = g & 1;
          if (!tc::mbar_wait_cluster_bounded(a_full + ab, (g >> 1) & 1)) {
            record_status(SN_ERR_TIMEOUT);
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const int ksteps = min(4, (p.Cin - c * 64) / 16);
          const uint64_t a_hi = tc::smem_desc_sw128(abuf + (2 * ab + 0) * p.a_bytes);
          const uint64_t a_lo = tc::smem_desc_sw128(abuf + (2 * ab + 1) * p.a_bytes);
          for (int tap = 0; tap < p.K; ++tap, ++q) {
            const int s = q % kScPairWStages;
            if (!mbar_wait_bounded(w_full + s, (q / kScPairWStages) & 1)) {
              record_status(SN_ERR_TIMEOUT);
              ok = false;
              break;
            }
            tc::fence_after_sync();
            const uint8_t* w = wbuf + static_cast<size_t>(s) * 2 * wh;
            const uint64_t w_hi = tc::smem_desc_sw128(w), w_lo = tc::smem_desc_sw128(w + wh);
            const uint64_t shift = static_cast<uint64_t>(tap * p.dil * 128) >> 4;
            for (int kk = 0; kk < ksteps; ++kk) {
              const uint32_t acc0 = (c | tap | kk) != 0;
              tc::mma_bf16_pair(acc_tmem, a_hi + shift + 2 * kk, w_hi + 2 * kk, idesc, acc0);
              tc::mma_bf16_pair(acc_tmem, a_lo + shift + 2 * kk, w_hi + 2 * kk, idesc, 1);
              tc::mma_bf16_pair(acc_tmem, a_hi + shift + 2 * kk, w_lo + 2 * kk, idesc, 1);
            }
            tc::mma_commit_pair(w_empty + s);
          }
          tc::mma_commit_pair(a_empty + ab);
        }
        tc::mma_commit_pair(t_full + tb);
      }
    }
  } else if (warp < 2 + kScProducerWarps) {
    // ---------------- snake producers (this CTA's 128 rows + halo) -------------
    const int pw = warp - 2;
    int g = 0;
    for (int j = 0; j < my_tiles; ++j) {
      int b, t0, o0;
      tile_coords(j, b, t0, o0);
      const float* xb = p.x + static_cast<int64_t>(b) * p.x_bs;
      const int tin0 = t0 - p.pad;
      for (int c = 0; c < nchunks; ++c, ++g) {
        const int ab = g & 1;
        const int i0 = c * 64 + pw * 8;
        float v[kMaxRowIters][8];
        if (p.x_tma) {
          // the chunk's x tile is in this CTA's staging buffer g mod kScXStages, [channel][row]
          const int xs = g & (kScXStages - 1);
          if (!__all_sync(0xffffffffu, mbar_wait_bounded(x_full + xs, (g / kScXStages) & 1))) {
            record_status(SN_ERR_TIMEOUT);
            j = my_tiles;
            break;
          }
          const float* xt = reinterpret_cast<const float*>(xstage + static_cast<size_t>(xs) * kScXBytes);
#pragma unroll
          for (int it = 0; it < kMaxRowIters; ++it) {
            const int r = lane + 32 * it;
#pragma unroll
            for (int e = 0; e < 8; ++e) v[it][e] = (r < 128) ? xt[(pw * 8 + e) * 128 + r] : 0.f;
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(x_empty + xs);  // this warp is done with the staging buffer
        } else {
#pragma unroll
          for (int it = 0; it < kMaxRowIters; ++it) {
            const int r = lane + 32 * it;
            const int tin = tin0 + r;
            const bool in_t = r < p.rows && tin >= 0 && tin < p.T;
#pragma unroll
            for (int e = 0; e < 8; ++e)
              v[it][e] = (in_t && i0 + e < p.Cin) ? __ldg(xb + static_cast<int64_t>(i0 + e) * p.x_ld + tin) : 0.f;
          }
        }
        float al[8], inv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          al[e] = (p.act == SN_ACT_SNAKE && i0 + e < p.Cin) ? __ldg(p.alpha + i0 + e) : 0.f;
          inv[e] = 1.0f / (al[e] + p.eps);
        }
        if (g >= 2 && !__all_sync(0xffffffffu, mbar_wait_bounded(a_empty + ab, ((g >> 1) - 1) & 1))) {
          record_status(SN_ERR_TIMEOUT);
          j = my_tiles;
          break;
        }
        uint8_t* ahi = abuf + (2 * ab + 0) * p.a_bytes;
        uint8_t* alo = abuf + (2 * ab + 1) * p.a_bytes;
#pragma unroll
        for (int it = 0; it < kMaxRowIters; ++it) {
          const int r = lane + 32 * it;
          if (r < p.rows) {
            float hi[8], lo[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              float s = v[it][e];
              if (p.act == SN_ACT_SNAKE) s = snake_value(s, al[e], inv[e]);
              hi[e] = __bfloat162float(__float2bfloat16_rn(s));
              lo[e] = s - hi[e];
            }
            const uint32_t off =
                static_cast<uint32_t>(r) * 128u + ((static_cast<uint32_t>(pw) ^ (r & 7)) << 4);
            *reinterpret_cast<uint4*>(ahi + off) = make_uint4(pack_bf16x2(hi[0], hi[1]), pack_bf16x2(hi[2], hi[3]),
                                                              pack_bf16x2(hi[4], hi[5]), pack_bf16x2(hi[6], hi[7]));
            *reinterpret_cast<uint4*>(alo + off) = make_uint4(pack_bf16x2(lo[0], lo[1]), pack_bf16x2(lo[2], lo[3]),
                                                              pack_bf16x2(lo[4], lo[5]), pack_bf16x2(lo[6], lo[7]));
          }
        }
        tc::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive_remote(a_full0 + 8u * ab);  // the even CTA's barrier (own CTA if even)
      }
    }
  } else {
    // ---------------- epilogue: this CTA's 128 time rows ----------------
    const int q4 = warp & 3;
    for (int j = 0; j < my_tiles; ++j) {
      const int tb = j & 1;
      {
        int b, t0, o0;
        tile_coords(j, b, t0, o0);
        sc_prefetch_res(p, b, t0, o0, threadIdx.x - 32 * (2 + kScProducerWarps));
      }
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(t_full + tb, (j >> 1) & 1))) {
        record_status(SN_ERR_TIMEOUT);
        break;
      }
      tc::fence_after_sync();
      int b, t0, o0;
      tile_coords(j, b, t0, o0);
      const int t = t0 + q4 * 32 + lane;
      const uint32_t base = tmem + (static_cast<uint32_t>(q4 * 32) << 16) + static_cast<uint32_t>(tb) * p.tcols;
      sc_epilogue_tile<UP>(p, base, b, t, o0);
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive_remote(t_empty0 + 8u * tb);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::cluster_sync_all();  // neither CTA leaves while the other may read its shared memory or TMEM
  if (warp == 1) tc::tmem_dealloc_pair(tmem, 2 * p.tcols);
}

// W fp32 [Cout, Cin, K] -> bf16 planes Wp[(k*2 + h)][o][i], h = 0 hi, 1 lo,
// o < Cg (the GEMM width, Cout rounded up to 16; rows past Cout are zero).
__global__ void pack_weights_kernel(const float* __restrict__ W, __nv_bfloat16* __restrict__ Wp, int Cout,
                                    int Cin, int K, int Cg) {
  // one thread per (o, i), i fastest: the K taps are one contiguous read, and
  // each tap's plane write is coalesced across the warp
  const int64_t total = static_cast<int64_t>(Cg) * Cin;
  const int64_t plane = static_cast<int64_t>(Cg) * Cin;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(e % Cin);
    const int o = static_cast<int>(e / Cin);
    for (int k = 0; k < K; ++k) {
      const float w = o < Cout ? W[(static_cast<int64_t>(o) * Cin + i) * K + k] : 0.f;
      const __nv_bfloat16 h = __float2bfloat16_rn(w);
      const __nv_bfloat16 l = __float2bfloat16_rn(w - __bfloat162float(h));
      Wp[(static_cast<int64_t>(k) * 2 + 0) * plane + e] = h;
      Wp[(static_cast<int64_t>(k) * 2 + 1) * plane + e] = l;
    }
  }
}

// ConvTranspose1d weight W fp32 [Cin, Cout, K] (K = m * s) -> the polyphase
// GEMM's bf16 planes Wp[(k'*2 + h)][o * s + r][i]: GEMM tap k' (reading input
// q - (m - 1) + k') of phase r uses W[i, o, r + (m - 1 - k') * s].  One thread
// per (o, i), i fastest: coalesced plane writes, K contiguous reads a thread.
__global__ void pack_weights_t_kernel(const float* __restrict__ W, __nv_bfloat16* __restrict__ Wp, int Cin,
                                      int Cout, int K, int s) {
  const int m = K / s;
  const int64_t total = static_cast<int64_t>(Cout) * Cin;
  const int64_t plane = static_cast<int64_t>(Cout) * s * Cin;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(e % Cin);
    const int o = static_cast<int>(e / Cin);
    const float* wr = W + (static_cast<int64_t>(i) * Cout + o) * K;
    for (int k = 0; k < K; ++k) {
      const int r = k % s, kt = m - 1 - k / s;
      const float w = wr[k];
      const __nv_bfloat16 h = __float2bfloat16_rn(w);
      const __nv_bfloat16 l = __float2bfloat16_rn(w - __bfloat162float(h));
      const int64_t col = (static_cast<int64_t>(o) * s + r) * Cin + i;
      Wp[(static_cast<int64_t>(kt) * 2 + 0) * plane + col] = h;
      Wp[(static_cast<int64_t>(kt) * 2 + 1) * plane + col] = l;
    }
  }
}

__device__ __forceinline__ float sc_act(int act, float v, float a, float inv) {
  if (act != SN_ACT_SNAKE) return v;
  const float sv = sinf(a * v);
  return fmaf(sv * sv, inv, v);
}

// Snake1d on its own (transformers' Snake1d, the activation each DAC
// Snake -> conv edge fuses): y = snake(x) elementwise over [rows = B*C, T],
// with the fused kernels' snake_value, so it also shows what their producers
// compute.  Four consecutive times a thread (one 16-byte access when T % 4 == 0
// and both pointers are 16-byte aligned).  y may be x.
__global__ void snake1d_kernel(const float* x, const float* __restrict__ alpha, float* y, int64_t rows, int64_t T,
                               int C, float eps, bool vec) {
  const int64_t groups_per_row = (T + 3) / 4;
  const int64_t total = rows * groups_per_row;
  for (int64_t g = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; g < total;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = g / groups_per_row;
    const int64_t t0 = (g - row * groups_per_row) * 4;
    const float a = __ldg(alpha + row % C);
    const float inv = 1.0f / (a + eps);
    const int64_t base = row * T + t0;
    if (vec) {
      float4 v = *reinterpret_cast<const float4*>(x + base);
      v.x = snake_value(v.x, a, inv);
      v.y = snake_value(v.y, a, inv);
      v.z = snake_value(v.z, a, inv);
      v.w = snake_value(v.w, a, inv);
      *reinterpret_cast<float4*>(y + base) = v;
    } else {
      for (int e = 0; e < 4 && t0 + e < T; ++e) y[base + e] = snake_value(x[base + e], a, inv);
    }
  }
}

// Batch and row (channel) strides, in elements, of the fallback kernels'
// x, y and residual tensors; time is contiguous.
struct ScStrides {
  int64_t x_bs, x_ld, y_bs, y_ld, r_bs, r_ld;
};

// The history move of a streaming decoder: for each table entry, every row
// (batch b, channel c) keeps samples [src, src + len) of its buffer row by
// moving them to [0, len).  One warp per row loads the kept samples into
// registers before storing any, so overlapping ranges move correctly.
struct ShiftTable {
  sn_shift_desc d[SN_SHIFT_MAX_DESCS];
  int64_t first_row[SN_SHIFT_MAX_DESCS];
  int64_t total_rows;
  int n;
};

__global__ void stream_shift_kernel(const __grid_constant__ ShiftTable tab) {
  static_assert(SN_SHIFT_MAX_LEN <= 64, "two samples a lane");
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t row = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); row < tab.total_rows;
       row += warps) {
    int i = 0;
    while (i + 1 < tab.n && tab.first_row[i + 1] <= row) ++i;
    const sn_shift_desc& d = tab.d[i];
    const int64_t r = row - tab.first_row[i];
    const int64_t b = r / d.rows, c = r - b * d.rows;
    float* base = d.buf + b * d.batch_stride + c * d.row_stride;
    const float v0 = lane < d.len ? base[d.src + lane] : 0.f;
    const float v1 = lane + 32 < d.len ? base[d.src + lane + 32] : 0.f;
    __syncwarp();
    if (lane < d.len) base[lane] = v0;
    if (lane + 32 < d.len) base[lane + 32] = v1;
  }
}

// Fallback: one thread per output element, the reference's loop order.
__global__ void snake_conv_simt_kernel(const float* __restrict__ x, const float* __restrict__ alpha,
                                       const float* __restrict__ W, const float* __restrict__ bias,
                                       const float* __restrict__ res, float* __restrict__ y, int B, int Cin,
                                       int Cout, int T, int Tout, int K, int stride, int pad, int dil, float eps,
                                       int act, int post, ScStrides ss) {
  const int64_t total = static_cast<int64_t>(B) * Cout * Tout;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(e % Tout);
    const int64_t r = e / Tout;
    const int o = static_cast<int>(r % Cout);
    const int b = static_cast<int>(r / Cout);
    float acc = bias ? bias[o] : 0.f;
    for (int i = 0; i < Cin; ++i) {
      const float a = act == SN_ACT_SNAKE ? alpha[i] : 0.f;
      const float inv = 1.0f / (a + eps);
      const float* xr = x + b * ss.x_bs + i * ss.x_ld;
      const float* wr = W + (static_cast<int64_t>(o) * Cin + i) * K;
      for (int k = 0; k < K; ++k) {
        const int ti = t * stride - pad + k * dil;
        if (ti < 0 || ti >= T) continue;
        acc = fmaf(sc_act(act, xr[ti], a, inv), wr[k], acc);
      }
    }
    if (res) acc += res[b * ss.r_bs + o * ss.r_ld + t];
    if (post == SN_POST_TANH) acc = tanhf(acc);
    y[b * ss.y_bs + o * ss.y_ld + t] = acc;
  }
}

// Transposed fallback: y[b, o, t] = bias[o] + sum over (i, k) with
// t = j * s - p + k, 0 <= j < T, of snake(x[b, i, j]) * W[i, o, k].
__global__ void snake_convt_simt_kernel(const float* __restrict__ x, const float* __restrict__ alpha,
                                        const float* __restrict__ W, const float* __restrict__ bias,
                                        float* __restrict__ y, int B, int Cin, int Cout, int T, int Tout, int K,
                                        int stride, int pad, float eps, ScStrides ss) {
  const int64_t total = static_cast<int64_t>(B) * Cout * Tout;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(e % Tout);
    const int64_t r = e / Tout;
    const int o = static_cast<int>(r % Cout);
    const int b = static_cast<int>(r / Cout);
    float acc = bias ? bias[o] : 0.f;
    for (int i = 0; i < Cin; ++i) {
      const float a = alpha[i];
      const float inv = 1.0f / (a + eps);
      const float* xr = x + b * ss.x_bs + i * ss.x_ld;
      const float* wr = W + (static_cast<int64_t>(i) * Cout + o) * K;
      for (int k = 0; k < K; ++k) {
        const int num = t + pad - k;  // j * stride
        if (num < 0 || num % stride != 0) continue;
        const int j = num / stride;
        if (j >= T) continue;
        acc = fmaf(sc_act(SN_ACT_SNAKE, xr[j], a, inv), wr[k], acc);
      }
    }
    y[b * ss.y_bs + o * ss.y_ld + t] = acc;
  }
}

// Cout: the GEMM width (a multiple of 16: the plain convolution pads it).
bool fast_path_ok(int Cin, int Cout, int K, int stride, int dil, int Tout) {
  return stride == 1 && K >= 1 && K <= kMaxTaps && dil >= 1 && (K - 1) * dil <= 72 && Cin % 16 == 0 &&
         Cout % 16 == 0 && Tout >= 1;
}

// Output-channel tile (UMMA N, a multiple of 32, <= 256): the width that
// minimises (tiles per SM) x (width + 128) over a persistent grid of `sms`
// CTAs.  The 128 stands for the per-tile cost that does not scale with the
// width (snake re-evaluated for every output tile, prologue, epilogue);
// ties go to the wider tile.  Measured with 32 / 64 / 128 / 192 / 256: the
// DAC decoder 619 -> 615 us per audio-second from 64 to 128 and flat
// beyond; the config-5 units unchanged.
// The CTA-pair kernel (SONATA_SNAKE_PAIR=0 selects the single-CTA kernel).
bool snake_pair_enabled() {
  static bool v = [] {
    const char* e = getenv("SONATA_SNAKE_PAIR");
    return !(e && strcmp(e, "0") == 0);
  }();
  return v;
}

int out_tile(int Cout, int64_t time_tiles, int sms) {
  int best = 32;
  int64_t best_cost = INT64_MAX;
  for (int nt = std::min(256, (Cout + 31) / 32 * 32); nt >= 32; nt -= 32) {
    const int64_t tiles = time_tiles * ((Cout + nt - 1) / nt);
    const int64_t cost = (tiles + sms - 1) / sms * (nt + 128);
    if (cost < best_cost) {
      best_cost = cost;
      best = nt;
    }
  }
  return best;
}

}  // namespace

int tu_status_snake(bool reset, cudaStream_t st, int* out) { return read_tu_status(reset, st, out); }

}  // namespace sn

extern "C" {

int64_t sn_snake_conv1d_output_length(int64_t T, int K, int stride, int padding, int dilation) {
  if (stride < 1 || K < 1 || dilation < 1 || padding < 0) return -1;
  return (T + 2 * static_cast<int64_t>(padding) - static_cast<int64_t>(dilation) * (K - 1) - 1) / stride + 1;
}

size_t sn_snake_conv1d_workspace_size(int Cin, int Cout, int K) {
  if (Cin < 1 || Cout < 1 || K < 1) return 0;
  const size_t cg = (static_cast<size_t>(Cout) + 15) / 16 * 16;  // 64-bit before the round-up
  return static_cast<size_t>(Cin) * cg * static_cast<size_t>(K) * 2 * sizeof(__nv_bfloat16);
}

int sn_snake_conv1d(const float* x, const float* alpha, const float* W, const float* bias, float* y, int B, int Cin,
                    int Cout, int T, int K, int stride, int padding, int dilation, float eps, void* workspace,
                    size_t workspace_bytes, void* stream) {
  return sn_snake_conv1d_ex(x, alpha, W, bias, nullptr, y, B, Cin, Cout, T, K, stride, padding, dilation, eps,
                            SN_ACT_SNAKE, SN_POST_NONE, 0u, workspace, workspace_bytes, stream);
}

}  // extern "C"

namespace sn {
namespace {

// The tensor-core path for a GEMM-shaped problem: p carries B, Cin, Cout (GEMM
// columns), T, Tout (GEMM rows), K (taps), pad, dil, eps and the epilogue
// variant; `pack` writes the bf16 hi/lo planes [K][2][Cout][Cin] into Wp.
// SN_ERR_UNSUPPORTED when the shape or the resources rule the path out.
template <typename Pack>
int snake_fast(ScParams p, __nv_bfloat16* Wp, cudaStream_t st, Pack pack) {
  p.ntiles_t = (p.Tout + 127) / 128;
  const int sms = sm_count();
  p.nt = out_tile(p.Cout, static_cast<int64_t>(p.B) * p.ntiles_t, sms);
  p.ntiles_o = (p.Cout + p.nt - 1) / p.nt;
  p.tcols = tc::tmem_cols_for(p.nt);
  p.rows = (128 + (p.K - 1) * p.dil + 7) / 8 * 8;
  p.a_bytes = static_cast<uint32_t>(p.rows) * 128;
  p.w_bytes = static_cast<uint32_t>(p.nt) * 128;
  // x tiles by TMA where the tile has no halo and x's strides allow a map
  // (the DAC residual units' k1 convolutions): one 32 KB box per chunk
  CUtensorMap mapX = {};
  p.x_tma = 0;
  if (p.rows == 128 && p.pad == 0 && p.x_ld % 4 == 0 && (p.B == 1 || p.x_bs % 4 == 0) && aligned16(p.x)) {
    const uint64_t xdims[3] = {static_cast<uint64_t>(p.T), static_cast<uint64_t>(p.Cin), static_cast<uint64_t>(p.B)};
    const uint64_t xstr[2] = {static_cast<uint64_t>(p.x_ld) * 4,
                              p.B == 1 ? (static_cast<uint64_t>(p.x_ld) * p.Cin * 4 + 15) / 16 * 16
                                       : static_cast<uint64_t>(p.x_bs) * 4};
    const uint32_t xbox[3] = {128, 64, 1};
    p.x_tma = tc::make_map_f32_plain(&mapX, p.x, 3, xdims, xstr, xbox) ? 1 : 0;
  }
  const int x_map_ok = p.x_tma;  // each kernel below also needs room for the staging
  const size_t smem0 = 1024 + 4 * static_cast<size_t>(p.a_bytes) + 2 * kScWStages * static_cast<size_t>(p.w_bytes) +
                       256;
  if (smem0 + static_cast<size_t>(kScXStages) * kScXBytes > 227 * 1024) p.x_tma = 0;  // no room for the staging
  const size_t smem = smem0 + (p.x_tma ? static_cast<size_t>(kScXStages) * kScXBytes : 0);
  const int64_t ntiles64 = static_cast<int64_t>(p.B) * p.ntiles_t * p.ntiles_o;
  p.ntiles = static_cast<int>(std::min<int64_t>(ntiles64, INT32_MAX));
  if (!(smem <= 227 * 1024 && ntiles64 < (int64_t(1) << 31) && p.rows <= 32 * kMaxRowIters && 2 * p.tcols <= 512))
    return SN_ERR_UNSUPPORTED;
  int rc = pack();
  if (rc != SN_OK) return rc;
  auto mma_kern = p.up_s > 0 ? snake_conv_mma_kernel<true> : snake_conv_mma_kernel<false>;
  auto pair_kern = p.up_s > 0 ? snake_conv_pair_kernel<true> : snake_conv_pair_kernel<false>;
  CUtensorMap mapW;
  const uint64_t dims[3] = {static_cast<uint64_t>(p.Cin), static_cast<uint64_t>(p.Cout),
                            static_cast<uint64_t>(2 * p.K)};
  const uint64_t strides[2] = {static_cast<uint64_t>(p.Cin) * 2, static_cast<uint64_t>(p.Cout) * p.Cin * 2};
  // CTA pairs pay off from Cout = 192 up (measured: -3 to -4% at C = 192 and
  // 384, even at 768, +9% at C = 96 where nt / 2 = 48 weight rows per CTA)
  if (snake_pair_enabled() && p.Cout >= 128) {
    // CTA-pair kernel: 256-row time tiles, each CTA holding nt / 2 weight rows
    ScParams q = p;
    q.x_tma = x_map_ok;  // the pair kernel's own room is checked below
    q.ntiles_t2 = (p.Tout + 255) / 256;
    const int npairs = std::max(1, sms / 2);
    q.nt = out_tile(p.Cout, static_cast<int64_t>(p.B) * q.ntiles_t2, npairs);
    q.ntiles_o = (p.Cout + q.nt - 1) / q.nt;
    q.tcols = tc::tmem_cols_for(q.nt);
    q.w_bytes = static_cast<uint32_t>(q.nt) * 128;
    const int64_t nt2 = static_cast<int64_t>(p.B) * q.ntiles_t2 * q.ntiles_o;
    q.ntiles2 = static_cast<int>(std::min<int64_t>(nt2, INT32_MAX));
    const size_t smem20 = 1024 + 4 * static_cast<size_t>(q.a_bytes) + kScPairWStages * static_cast<size_t>(q.w_bytes) +
                          256;
    if (smem20 + static_cast<size_t>(kScXStages) * kScXBytes > 227 * 1024) q.x_tma = 0;  // no room for the staging
    const size_t smem2 = smem20 + (q.x_tma ? static_cast<size_t>(kScXStages) * kScXBytes : 0);
    const uint32_t box2[3] = {64, static_cast<uint32_t>(q.nt / 2), 1};
    if (nt2 < (int64_t(1) << 31) && 2 * q.tcols <= 512 && smem2 <= 227 * 1024 &&
        tc::make_map_bf16_sw128(&mapW, Wp, 3, dims, strides, box2) &&
        cudaFuncSetAttribute(pair_kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem2)) == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2 * std::min(q.ntiles2, npairs));
      cfg.blockDim = dim3(kScThreads);
      cfg.dynamicSmemBytes = smem2;
      cfg.stream = st;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      if (cudaLaunchKernelEx(&cfg, pair_kern, mapW, mapX, q) == cudaSuccess) return SN_OK;
    }
    cudaGetLastError();
  }
  const uint32_t box[3] = {64, static_cast<uint32_t>(p.nt), 1};
  if (tc::make_map_bf16_sw128(&mapW, Wp, 3, dims, strides, box)) {
    if (cudaFuncSetAttribute(mma_kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) == cudaSuccess) {
      const int grid = std::min(p.ntiles, sms);
      return launch(mma_kern, dim3(grid), dim3(kScThreads), smem, st, false, mapW, mapX, p);
    }
    cudaGetLastError();
  }
  return SN_ERR_UNSUPPORTED;
}

ScParams base_params(const float* x, const float* alpha, const float* bias, float* y, int B, int Cin, float eps) {
  ScParams p = {};
  p.x = x;
  p.alpha = alpha;
  p.bias = bias;
  p.y = y;
  p.B = B;
  p.Cin = Cin;
  p.eps = eps;
  p.res = nullptr;
  p.act = SN_ACT_SNAKE;
  p.post = SN_POST_NONE;
  p.up_s = p.up_p = 0;
  p.up_sh = -1;
  p.up_vec = 1;
  return p;
}

int blocks_for(int64_t total, int per_sm) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, int64_t(148) * per_sm)));
}

}  // namespace
}  // namespace sn

extern "C" {

int sn_snake_conv1d_pack(const float* W, int Cin, int Cout, int K, void* packed, size_t packed_bytes,
                         void* stream) {
  if (!W || !packed || Cin < 1 || Cout < 1 || K < 1) return SN_ERR_INVALID_ARGUMENT;
  if (packed_bytes < sn_snake_conv1d_workspace_size(Cin, Cout, K)) return SN_ERR_INVALID_ARGUMENT;
  if (!sn::aligned16(packed)) return SN_ERR_MISALIGNED;
  if (Cout > INT32_MAX - 15) return SN_ERR_INVALID_ARGUMENT;  // the round-up to 16 below stays in int
  const int Cg = (Cout + 15) / 16 * 16;
  const int64_t tot = static_cast<int64_t>(Cg) * Cin;
  return sn::launch(sn::pack_weights_kernel, dim3(sn::blocks_for(tot, 8)), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), false, W, static_cast<__nv_bfloat16*>(packed), Cout, Cin, K,
                    Cg);
}

int sn_snake_conv_transpose1d_pack(const float* W, int Cin, int Cout, int K, int stride, void* packed,
                                   size_t packed_bytes, void* stream) {
  if (!W || !packed || Cin < 1 || Cout < 1 || K < 1 || stride < 1) return SN_ERR_INVALID_ARGUMENT;
  if (K % stride != 0) return SN_ERR_UNSUPPORTED;  // no polyphase GEMM: the fallback reads W itself
  if (packed_bytes < sn_snake_conv1d_workspace_size(Cin, Cout, K)) return SN_ERR_INVALID_ARGUMENT;
  if (!sn::aligned16(packed)) return SN_ERR_MISALIGNED;
  const int64_t tot = static_cast<int64_t>(Cin) * Cout;
  return sn::launch(sn::pack_weights_t_kernel, dim3(sn::blocks_for(tot, 8)), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), false, W, static_cast<__nv_bfloat16*>(packed), Cin, Cout, K,
                    stride);
}

}  // extern "C"

namespace sn {
namespace {

// Row (channel) strides must keep rows apart: ld >= len, and batch strides
// must keep batches apart.
bool strides_ok(int64_t bs, int64_t ld, int B, int C, int64_t len) {
  return ld >= len && (B == 1 || bs >= (static_cast<int64_t>(C) - 1) * ld + len) && bs >= 0;
}

int snake_conv1d_impl(const float* x, int64_t x_bs, int64_t x_ld, const float* alpha, const float* W,
                      const float* bias, const float* residual, int64_t r_bs, int64_t r_ld, float* y, int64_t y_bs,
                      int64_t y_ld, int B, int Cin, int Cout, int T, int K, int stride, int padding, int dilation,
                      float eps, int act, int post, unsigned flags, void* workspace, size_t workspace_bytes,
                      void* stream) {
  if (!x || !W || !y || B < 1 || Cin < 1 || Cout < 1 || T < 1 || K < 1 || stride < 1 || padding < 0 ||
      dilation < 1)
    return SN_ERR_INVALID_ARGUMENT;
  if (flags & ~SN_FLAG_PREPACKED) return SN_ERR_INVALID_ARGUMENT;
  const bool prepacked = (flags & SN_FLAG_PREPACKED) != 0;
  if ((act != SN_ACT_SNAKE && act != SN_ACT_NONE) || (post != SN_POST_NONE && post != SN_POST_TANH))
    return SN_ERR_INVALID_ARGUMENT;
  if (act == SN_ACT_SNAKE && !alpha) return SN_ERR_INVALID_ARGUMENT;
  const int64_t tout64 = sn_snake_conv1d_output_length(T, K, stride, padding, dilation);
  if (tout64 < 1 || tout64 > (int64_t(1) << 31) - 1) return SN_ERR_INVALID_ARGUMENT;
  const int Tout = static_cast<int>(tout64);
  if (!strides_ok(x_bs, x_ld, B, Cin, T) || !strides_ok(y_bs, y_ld, B, Cout, Tout) ||
      (residual && !strides_ok(r_bs, r_ld, B, Cout, Tout)))
    return SN_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (Cout > INT32_MAX - 15) return SN_ERR_INVALID_ARGUMENT;  // the round-up to 16 below stays in int
  const int Cg = (Cout + 15) / 16 * 16;  // GEMM width: zero weight rows past Cout
  if (fast_path_ok(Cin, Cg, K, stride, dilation, Tout) && workspace &&
      workspace_bytes >= sn_snake_conv1d_workspace_size(Cin, Cout, K) && aligned16(workspace)) {
    ScParams p = base_params(x, alpha, bias, y, B, Cin, eps);
    p.Cout = Cg;
    p.T = T;
    p.Tout = Tout;
    p.K = K;
    p.pad = padding;
    p.dil = dilation;
    p.res = residual;
    p.act = act;
    p.post = post;
    p.Cy = Cout;
    p.Ty = Tout;
    p.x_bs = x_bs;
    p.x_ld = x_ld;
    p.y_bs = y_bs;
    p.y_ld = y_ld;
    p.r_bs = r_bs;
    p.r_ld = r_ld;
    __nv_bfloat16* Wp = static_cast<__nv_bfloat16*>(workspace);
    const int rc = snake_fast(p, Wp, st, [&] {
      if (prepacked) return static_cast<int>(SN_OK);
      const int64_t tot = static_cast<int64_t>(Cg) * Cin;
      return launch(pack_weights_kernel, dim3(blocks_for(tot, 8)), dim3(256), 0, st, false, W, Wp, Cout, Cin, K,
                    Cg);
    });
    if (rc != SN_ERR_UNSUPPORTED) return rc;
  }
  const int64_t total = static_cast<int64_t>(B) * Cout * Tout;
  const ScStrides ss = {x_bs, x_ld, y_bs, y_ld, r_bs, r_ld};
  return launch(snake_conv_simt_kernel, dim3(blocks_for(total, 32)), dim3(256), 0, st, false, x, alpha, W, bias,
                residual, y, B, Cin, Cout, T, Tout, K, stride, padding, dilation, eps, act, post, ss);
}

// Transposed convolution writing output samples [0, Ty) of the full
// ConvTranspose1d (whose own length would be (T - 1) * stride - 2 * padding + K):
// Ty may be shorter (a streaming decoder emits only the samples whose inputs
// have all arrived) or longer up to (T - 1) * stride - padding + K.
int snake_convt_impl(const float* x, int64_t x_bs, int64_t x_ld, const float* alpha, const float* W,
                     const float* bias, float* y, int64_t y_bs, int64_t y_ld, int B, int Cin, int Cout, int T, int K,
                     int stride, int padding, int Ty, float eps, unsigned flags, void* workspace,
                     size_t workspace_bytes, void* stream) {
  if (!x || !alpha || !W || !y || B < 1 || Cin < 1 || Cout < 1 || T < 1 || K < 1 || stride < 1 || padding < 0 ||
      Ty < 1)
    return SN_ERR_INVALID_ARGUMENT;
  if (flags & ~SN_FLAG_PREPACKED) return SN_ERR_INVALID_ARGUMENT;
  if (static_cast<int64_t>(Ty) > (static_cast<int64_t>(T) - 1) * stride - padding + K) return SN_ERR_INVALID_ARGUMENT;
  if (!strides_ok(x_bs, x_ld, B, Cin, T) || !strides_ok(y_bs, y_ld, B, Cout, Ty)) return SN_ERR_INVALID_ARGUMENT;
  const bool prepacked = (flags & SN_FLAG_PREPACKED) != 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // polyphase GEMM: m = K / s taps per phase over rows q in [0, T + m - 1);
  // row q holds output samples s * q + r - padding, so rows past the one that
  // holds sample Ty - 1 are not computed
  const int m = (K % stride == 0) ? K / stride : 0;
  const int64_t gcols = static_cast<int64_t>(Cout) * stride;
  const int64_t rows = std::min<int64_t>(static_cast<int64_t>(T) + m - 1,
                                         (static_cast<int64_t>(Ty) - 1 + padding) / stride + 1);
  if (m >= 1 && gcols <= INT32_MAX && rows <= INT32_MAX &&
      fast_path_ok(Cin, static_cast<int>(gcols), m, 1, 1, static_cast<int>(rows)) && workspace &&
      workspace_bytes >= sn_snake_conv1d_workspace_size(Cin, Cout, K) && aligned16(workspace)) {
    ScParams p = base_params(x, alpha, bias, y, B, Cin, eps);
    p.Cout = static_cast<int>(gcols);
    p.T = T;
    p.Tout = static_cast<int>(rows);
    p.K = m;
    p.pad = m - 1;
    p.dil = 1;
    p.up_s = stride;
    p.up_sh = (stride & (stride - 1)) == 0 ? __builtin_ctz(static_cast<unsigned>(stride)) : -1;
    p.up_p = padding;
    p.Cy = Cout;
    p.Ty = Ty;
    p.x_bs = x_bs;
    p.x_ld = x_ld;
    p.y_bs = y_bs;
    p.y_ld = y_ld;
    // phase runs start at stride * q - padding: vector stores when that and
    // every row start keep 16 (8) byte alignment
    const uintptr_t ya = reinterpret_cast<uintptr_t>(y);
    p.up_vec = (stride % 4 == 0 && padding % 4 == 0 && y_ld % 4 == 0 && y_bs % 4 == 0 && ya % 16 == 0)   ? 4
               : (stride % 2 == 0 && padding % 2 == 0 && y_ld % 2 == 0 && y_bs % 2 == 0 && ya % 8 == 0) ? 2
                                                                                                        : 1;
    __nv_bfloat16* Wp = static_cast<__nv_bfloat16*>(workspace);
    const int rc = snake_fast(p, Wp, st, [&] {
      if (prepacked) return static_cast<int>(SN_OK);
      const int64_t tot = static_cast<int64_t>(Cin) * Cout;
      return launch(pack_weights_t_kernel, dim3(blocks_for(tot, 8)), dim3(256), 0, st, false, W, Wp, Cin, Cout, K,
                    stride);
    });
    if (rc != SN_ERR_UNSUPPORTED) return rc;
  }
  const int64_t total = static_cast<int64_t>(B) * Cout * Ty;
  const ScStrides ss = {x_bs, x_ld, y_bs, y_ld, 0, 0};
  return launch(snake_convt_simt_kernel, dim3(blocks_for(total, 32)), dim3(256), 0, st, false, x, alpha, W, bias, y,
                B, Cin, Cout, T, Ty, K, stride, padding, eps, ss);
}

}  // namespace
}  // namespace sn

extern "C" {

int sn_snake_conv1d_ex(const float* x, const float* alpha, const float* W, const float* bias, const float* residual,
                       float* y, int B, int Cin, int Cout, int T, int K, int stride, int padding, int dilation,
                       float eps, int act, int post, unsigned flags, void* workspace, size_t workspace_bytes,
                       void* stream) {
  const int64_t tout = sn_snake_conv1d_output_length(T, K, stride, padding, dilation);
  if (tout < 1 || T < 1 || Cin < 1 || Cout < 1) return SN_ERR_INVALID_ARGUMENT;
  const int64_t xb = static_cast<int64_t>(Cin) * T, yb = static_cast<int64_t>(Cout) * tout;
  return sn::snake_conv1d_impl(x, xb, T, alpha, W, bias, residual, yb, tout, y, yb, tout, B, Cin, Cout, T, K, stride,
                               padding, dilation, eps, act, post, flags, workspace, workspace_bytes, stream);
}

int sn_snake_conv1d_strided(const float* x, int64_t x_bs, int64_t x_ld, const float* alpha, const float* W,
                            const float* bias, const float* residual, int64_t r_bs, int64_t r_ld, float* y,
                            int64_t y_bs, int64_t y_ld, int B, int Cin, int Cout, int T, int K, int stride,
                            int padding, int dilation, float eps, int act, int post, unsigned flags, void* workspace,
                            size_t workspace_bytes, void* stream) {
  return sn::snake_conv1d_impl(x, x_bs, x_ld, alpha, W, bias, residual, r_bs, r_ld, y, y_bs, y_ld, B, Cin, Cout, T, K,
                               stride, padding, dilation, eps, act, post, flags, workspace, workspace_bytes, stream);
}

int64_t sn_snake_conv_transpose1d_output_length(int64_t T, int K, int stride, int padding) {
  if (T < 1 || stride < 1 || K < 1 || padding < 0) return -1;
  return (T - 1) * stride - 2 * static_cast<int64_t>(padding) + K;
}

int sn_snake_conv_transpose1d(const float* x, const float* alpha, const float* W, const float* bias, float* y, int B,
                              int Cin, int Cout, int T, int K, int stride, int padding, float eps, unsigned flags,
                              void* workspace, size_t workspace_bytes, void* stream) {
  const int64_t ty64 = sn_snake_conv_transpose1d_output_length(T, K, stride, padding);
  if (ty64 < 1 || ty64 > (int64_t(1) << 31) - 1 || Cin < 1 || Cout < 1) return SN_ERR_INVALID_ARGUMENT;
  const int64_t xb = static_cast<int64_t>(Cin) * T, yb = static_cast<int64_t>(Cout) * ty64;
  return sn::snake_convt_impl(x, xb, T, alpha, W, bias, y, yb, ty64, B, Cin, Cout, T, K, stride, padding,
                              static_cast<int>(ty64), eps, flags, workspace, workspace_bytes, stream);
}

int sn_snake_conv_transpose1d_strided(const float* x, int64_t x_bs, int64_t x_ld, const float* alpha, const float* W,
                                      const float* bias, float* y, int64_t y_bs, int64_t y_ld, int B, int Cin,
                                      int Cout, int T, int K, int stride, int padding, int Ty, float eps,
                                      unsigned flags, void* workspace, size_t workspace_bytes, void* stream) {
  return sn::snake_convt_impl(x, x_bs, x_ld, alpha, W, bias, y, y_bs, y_ld, B, Cin, Cout, T, K, stride, padding, Ty,
                              eps, flags, workspace, workspace_bytes, stream);
}

int sn_snake1d(const float* x, const float* alpha, float* y, int B, int C, int64_t T, float eps, void* stream) {
  if (!x || !alpha || !y || B < 1 || C < 1 || T < 1) return SN_ERR_INVALID_ARGUMENT;
  const int64_t rows = static_cast<int64_t>(B) * C;
  const bool vec = T % 4 == 0 && sn::aligned16(x) && sn::aligned16(y);
  return sn::launch(sn::snake1d_kernel, dim3(sn::blocks_for(rows * ((T + 3) / 4), 16)), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), false, x, alpha, y, rows, T, C, eps, vec);
}

int sn_stream_shift(const sn_shift_desc* descs, int n, void* stream) {
  if (!descs || n < 1 || n > SN_SHIFT_MAX_DESCS) return SN_ERR_INVALID_ARGUMENT;
  sn::ShiftTable tab = {};
  int64_t rows = 0;
  for (int i = 0; i < n; ++i) {
    const sn_shift_desc& d = descs[i];
    if (!d.buf || d.batches < 1 || d.rows < 1 || d.src < 0 || d.len < 0 || d.len > SN_SHIFT_MAX_LEN ||
        d.row_stride < static_cast<int64_t>(d.src) + d.len ||
        (d.batches > 1 && d.batch_stride < static_cast<int64_t>(d.rows) * d.row_stride))
      return SN_ERR_INVALID_ARGUMENT;
    tab.d[i] = d;
    tab.first_row[i] = rows;
    rows += static_cast<int64_t>(d.batches) * d.rows;
  }
  tab.n = n;
  tab.total_rows = rows;
  const int warps_per_block = 8;
  const int64_t blocks = std::min<int64_t>((rows + warps_per_block - 1) / warps_per_block, 148 * 16);
  return sn::launch(sn::stream_shift_kernel, dim3(static_cast<unsigned>(std::max<int64_t>(blocks, 1))),
                    dim3(32 * warps_per_block), 0, static_cast<cudaStream_t>(stream), false, tab);
}

// ---------------------------------------------------------------------------
// Allocation-free variant.  Its scratch (the packed bf16 hi/lo weights) lives
// in this file-scope device array instead of a caller-provided workspace; the
// array exists once per GPU that loads the library, for the life of the
// process.  Host code cannot use the array's name as a device address: the
// address is looked up with cudaGetSymbolAddress on every call, with the
// caller's device current.  The lookup is a host-side query once the module
// is loaded, and looking it up each time keeps the address right after a
// cudaDeviceReset re-creates the context (the array may then sit elsewhere).
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_snake_noalloc_scratch[SN_SNAKE_CONV1D_NOALLOC_MAX_SCRATCH];

static void* snake_noalloc_scratch() {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_snake_noalloc_scratch) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return p;
}

int sn_snake_conv1d_noalloc(const float* x, const float* alpha, const float* W, const float* bias, float* y, int B,
                            int Cin, int Cout, int T, int K, int stride, int padding, int dilation, float eps,
                            void* stream) {
  if (Cin < 1 || Cout < 1 || K < 1 || T < 1 || stride < 1 || padding < 0 || dilation < 1)
    return SN_ERR_INVALID_ARGUMENT;
  const int64_t tout = sn_snake_conv1d_output_length(T, K, stride, padding, dilation);
  if (tout < 1 || tout > INT32_MAX) return SN_ERR_INVALID_ARGUMENT;
  // Only the tensor-core path packs weights into the scratch; every other
  // shape runs the per-output kernel, which reads W directly and needs none.
  if (Cout > INT32_MAX - 15) return SN_ERR_INVALID_ARGUMENT;  // the round-up to 16 below stays in int
  const int Cg = (Cout + 15) / 16 * 16;
  if (!sn::fast_path_ok(Cin, Cg, K, stride, dilation, static_cast<int>(tout)))
    return sn_snake_conv1d(x, alpha, W, bias, y, B, Cin, Cout, T, K, stride, padding, dilation, eps, nullptr, 0,
                           stream);
  if (sn_snake_conv1d_workspace_size(Cin, Cout, K) > SN_SNAKE_CONV1D_NOALLOC_MAX_SCRATCH)
    return SN_ERR_SCRATCH_LIMIT;
  void* scratch = snake_noalloc_scratch();
  if (!scratch) return SN_ERR_SCRATCH_ADDRESS;
  return sn_snake_conv1d(x, alpha, W, bias, y, B, Cin, Cout, T, K, stride, padding, dilation, eps, scratch,
                         SN_SNAKE_CONV1D_NOALLOC_MAX_SCRATCH, stream);
}

}  // extern "C"
