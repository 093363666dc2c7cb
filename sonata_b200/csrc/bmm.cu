// Batched matrix products on B200 tensor cores (tcgen05 + TMA + TMEM).
//
// 1. Multi-codebook logit head:
//      logits[cb, b, n] = sum_k hidden[cb, b, k] * W[cb, k, n]
//    W is packed once to [cb, n, k] (K-major rows, sn_codebook_head_pack).
//    B <= 4 streams: the decode GEMV (weights streamed once, CUDA cores).
//    B >= 5: a tcgen05 contraction -- tile of 128 weight rows (UMMA M) x the
//    stream batch (UMMA N <= 256) accumulated over K in TMEM; 3-D TMA maps
//    make the rows past N = 1025 and the streams past B read as zero without
//    touching memory.
// 2. Mamba2 SSD chunk product of kernels/bmm.py (launch_bmm, bmm.py:96-117):
//      CB[b, c, g, i, j] = sum_d C[b, c*CH+i, g, d] * B[b, c*CH+j, g, d]
//    with the masked semantics of bmm.py:205-212 (positions >= SEQLEN are
//    zero): the 4-D TMA maps give the sequence dimension the extent SEQLEN, so
//    the ragged tail of the last chunk is filled with zeros by the copy engine.
//    One CTA per 128 x 128 output tile (UMMA M = N = 128).
//
// Roles in the tensor-core kernels: warp 0 lane 0 issues TMA, warp 1 owns TMEM
// and lane 0 of it issues tcgen05.mma, warps 2-5 drain TMEM (32x32b loads, one
// lane quarter each) and store fp32.  All mbarrier waits are bounded.
#include "tc.cuh"

#include <algorithm>
#include <cstdlib>

namespace sn {
int gemv_any(int wk, const void* W, int64_t ldw, int64_t sW, const float* scale, int64_t sS, const void* x,
             int64_t ldx, int64_t sx, void* y, int64_t ldy, int64_t sy, int M, int N, int K, int batch,
             int y_dtype, unsigned flags, cudaStream_t st);

namespace {

constexpr int kTcThreads = 192;  // 6 warps
constexpr int kHeadStages = 4;

// ---------------------------------------------------------------------------
// codebook head
// ---------------------------------------------------------------------------
struct HeadParams {
  float* out;  // [ncb, B, N]
  int ncb, B, K, N;
  int bt;      // streams per tile (UMMA N, multiple of 16, <= 256)
  int nbt;     // stream tiles
  int ntiles;  // 128-row weight tiles per codebook
  uint32_t stage_bytes, a_bytes;
};

__global__ void __launch_bounds__(kTcThreads, 1)
    head_mma_kernel(const __grid_constant__ CUtensorMap mapW, const __grid_constant__ CUtensorMap mapH,
                    const HeadParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kHeadStages * p.stage_bytes);
  uint64_t* empty = full + kHeadStages;
  uint64_t* done = empty + kHeadStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int u = blockIdx.x;
  const int bt = u % p.nbt;
  u /= p.nbt;
  const int nt = u % p.ntiles;
  const int cb = u / p.ntiles;
  const int n0 = nt * 128, b0 = bt * p.bt;
  const int nkb = p.K / 64;
  const uint32_t tcols = tc::tmem_cols_for(p.bt);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kHeadStages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    mbar_init(done, 1);
    fence_barrier_init();
    tc::prefetch_map(&mapW);
    tc::prefetch_map(&mapH);
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, tcols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    int kb = 0;
    for (; kb < nkb; ++kb) {
      const int s = kb % kHeadStages, k = kb / kHeadStages;
      if (k > 0 && !mbar_wait_bounded(empty + s, (k - 1) & 1)) {
        record_status(SN_ERR_TIMEOUT);
        break;
      }
      uint8_t* a = smem + s * p.stage_bytes;
      uint8_t* b = a + p.a_bytes;
      mbar_arrive_expect_tx(full + s, p.stage_bytes);
      tc::tma_load_3d(a, &mapW, kb * 64, n0, cb, full + s);
      tc::tma_load_3d(b, &mapH, kb * 64, b0, cb, full + s);
    }
    if (kb < nkb) {  // error path: let issued copies land before the CTA exits
      for (int j = (kb > kHeadStages ? kb - kHeadStages : 0); j < kb; ++j)
        mbar_wait_bounded(full + j % kHeadStages, (j / kHeadStages) & 1);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    const uint32_t idesc = tc::idesc_bf16_f32(128, p.bt);
    bool ok = true;
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % kHeadStages;
      if (!mbar_wait_bounded(full + s, (kb / kHeadStages) & 1)) {
        record_status(SN_ERR_TIMEOUT);
        ok = false;
        break;
      }
      tc::fence_after_sync();
      const uint8_t* a = smem + s * p.stage_bytes;
      const uint64_t da = tc::smem_desc_sw128(a), db = tc::smem_desc_sw128(a + p.a_bytes);
#pragma unroll
      for (int k = 0; k < 4; ++k)  // 16 bf16 = 32 bytes per step inside the 128-byte swizzle row
        tc::mma_bf16(tmem, da + 2 * k, db + 2 * k, idesc, (kb | k) != 0);
      tc::mma_commit(empty + s);
    }
    (void)ok;
    tc::mma_commit(done);  // fires once every issued MMA has completed
  } else if (warp >= 2) {
    // ---------------- epilogue: TMEM -> fp32 logits ----------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    // the TMEM loads below are warp-collective: take the wait's outcome as a warp
    if (__all_sync(0xffffffffu, mbar_wait_bounded(done, 0))) {
      tc::fence_after_sync();
      const int n = n0 + q * 32 + lane;
      for (int c = 0; c < p.bt; c += 16) {
        float v[16];
        tc::tmem_ld16(tmem + (static_cast<uint32_t>(q * 32) << 16) + c, v);
        if (n < p.N) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int b = b0 + c + j;
            if (b < p.B) p.out[(static_cast<int64_t>(cb) * p.B + b) * p.N + n] = v[j];
          }
        }
      }
    } else {
      record_status(SN_ERR_TIMEOUT);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) tc::tmem_dealloc(tmem, tcols);
}

// ---------------------------------------------------------------------------
// codebook head, K split over a CTA pair (B >= 5)
//
// The 128-row weight tiles x stream tiles are spread over clusters of two
// CTAs (one per SM, 74 clusters on 148 SMs; a cluster loops if there are more
// tiles).  CTA rank r accumulates the K half r of its tile in TMEM.  The pair
// then reduces through distributed shared memory in a fixed order: each CTA
// owns half of the stream columns, sends the other half of its partial tile
// to its peer (st.shared::cluster), and adds the peer's half to its own,
// k-half 0 first, so the result does not depend on timing.  Rows past the
// last full 128-row tile (row 1024 of the 1025-row head) are dot products on
// the CUDA cores of the epilogue warps of every CTA, while the MMAs run.
// ---------------------------------------------------------------------------
constexpr int kSkThreads = 192;
constexpr int kSkStagesMax = 8;

struct HeadSkParams {
  float* out;                    // [ncb, B, N]
  const __nv_bfloat16* hidden;   // [ncb, B, K]
  const __nv_bfloat16* Wt;       // [ncb, N, K]
  int ncb, B, K, N;
  int bt, nbt;                   // stream tile (UMMA N, multiple of 32) and tiles per codebook
  int nrt;                       // full 128-row tiles per codebook
  int ntiles;                    // ncb * nrt * nbt
  int stages;
  uint32_t stage_bytes, a_bytes;
  uint32_t recv_off, bar_off;    // recv: [bt / 2 columns][128 rows] fp32
  int alias_recv;                // one tile per cluster: recv lies over the (then idle) stage ring
};

__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

__global__ void __launch_bounds__(kSkThreads, 1)
    head_splitk_kernel(const __grid_constant__ CUtensorMap mapW, const __grid_constant__ CUtensorMap mapH,
                       const HeadSkParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int ns = p.stages;
  float* recv = reinterpret_cast<float*>(smem + p.recv_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.bar_off);
  uint64_t* empty = full + ns;
  uint64_t* tfull = empty + ns;
  uint64_t* tempty = tfull + 1;
  uint64_t* rfull = tempty + 1;   // peer's half of my columns has landed in recv
  uint64_t* rempty = rfull + 1;   // peer has read my half of its columns (recv reusable)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rempty + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = tc::cluster_ctarank(), peer = rank ^ 1u;
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
  const int nkb = p.K / 64, kb_half = nkb / 2, kb0 = static_cast<int>(rank) * kb_half;
  const uint32_t tcols = tc::tmem_cols_for(p.bt);
  const int half = p.bt / 2;
  const int own_lo = static_cast<int>(rank) * half, peer_lo = static_cast<int>(peer) * half;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ns; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    mbar_init(tfull, 1);
    mbar_init(tempty, 4);
    mbar_init(rfull, 128);   // every epilogue thread of the peer
    mbar_init(rempty, 128);
    fence_barrier_init();
    tc::prefetch_map(&mapW);
    tc::prefetch_map(&mapH);
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, tcols);
  tc::fence_before_sync();
  __syncthreads();
  tc::cluster_sync_all();  // the peer's barriers are initialised before any remote arrive
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  pdl_launch_dependents();
  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer: K half `rank` of each tile ----------------
    auto load_w = [&](uint8_t* a, int kb, int rt, int cb, uint64_t* bar) {
      tc::tma_load_3d(a, &mapW, kb * 64, rt * 128, cb, bar);
    };
    int it = 0;
    bool ok = true;
    // weights are frozen: the first ring's weight boxes go out before the
    // previous kernel (programmatic dependent launch) has finished; hidden,
    // which it may produce, only after griddepcontrol.wait
    const int pre = min(ns, (p.ntiles > cluster ? (p.ntiles - 1 - cluster) / nclusters + 1 : 0) * kb_half);
    {
      int t = cluster, j = 0;
      int rt = (t / p.nbt) % p.nrt, cb = t / (p.nbt * p.nrt);  // per tile, not per stage
      for (int q = 0; q < pre; ++q) {
        mbar_arrive_expect_tx(full + q, p.stage_bytes);
        load_w(smem + q * p.stage_bytes, kb0 + j, rt, cb, full + q);
        if (++j == kb_half) {
          j = 0;
          t += nclusters;
          rt = (t / p.nbt) % p.nrt;
          cb = t / (p.nbt * p.nrt);
        }
      }
    }
    pdl_wait();
    int s = 0, k = 0;  // stage of `it` (it mod ns) and its round (it / ns), kept without divisions
    for (int t = cluster; t < p.ntiles && ok; t += nclusters) {
      const int bti = t % p.nbt, rt = (t / p.nbt) % p.nrt, cb = t / (p.nbt * p.nrt);
      for (int j = 0; j < kb_half; ++j, ++it, k += (++s == ns), s = (s == ns) ? 0 : s) {
        uint8_t* a = smem + s * p.stage_bytes;
        if (it >= pre) {
          if (k > 0 && !mbar_wait_bounded(empty + s, (k - 1) & 1)) {
            record_status(SN_ERR_TIMEOUT);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full + s, p.stage_bytes);
          load_w(a, kb0 + j, rt, cb, full + s);
        }
        tc::tma_load_3d(a + p.a_bytes, &mapH, (kb0 + j) * 64, bti * p.bt, cb, full + s);
      }
    }
    if (!ok) {  // error path: let issued copies land before the CTA exits
      for (int j = (it > ns ? it - ns : 0); j < it; ++j) mbar_wait_bounded(full + j % ns, (j / ns) & 1);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    const uint32_t idesc = tc::idesc_bf16_f32(128, p.bt);
    int it = 0, j = 0, s = 0, ph = 0;  // stage it mod ns and its phase, kept without divisions
    bool ok = true;
    for (int t = cluster; t < p.ntiles && ok; t += nclusters, ++j) {
      if (j > 0 && !mbar_wait_bounded(tempty, (j - 1) & 1)) {
        record_status(SN_ERR_TIMEOUT);
        break;
      }
      tc::fence_after_sync();
      for (int kb = 0; kb < kb_half; ++kb, ++it, ph ^= (++s == ns), s = (s == ns) ? 0 : s) {
        if (!mbar_wait_bounded(full + s, ph)) {
          record_status(SN_ERR_TIMEOUT);
          ok = false;
          break;
        }
        tc::fence_after_sync();
        const uint8_t* a = smem + s * p.stage_bytes;
        const uint64_t da = tc::smem_desc_sw128(a), db = tc::smem_desc_sw128(a + p.a_bytes);
#pragma unroll
        for (int k = 0; k < 4; ++k) tc::mma_bf16(tmem, da + 2 * k, db + 2 * k, idesc, (kb | k) != 0);
        tc::mma_commit(empty + s);
      }
      tc::mma_commit(tfull);
    }
  } else if (warp >= 2) {
    pdl_wait();  // hidden and the logits buffer belong to the previous kernel until here
    // ---- rows past the last full tile (row 1024 of the head): CUDA-core dot
    // products, done while this CTA's MMAs run; all loads of a dot issued first
    {
      const int nx = p.N - p.nrt * 128;
      const int items = p.ncb * p.B * nx;  // < 2^31 (host-checked shapes)
      const int gw = blockIdx.x * 4 + (warp - 2), nw = gridDim.x * 4;
      const int nck = p.K / 8;  // 16-byte chunks per row
      for (int e = gw; e < items; e += nw) {
        const int x = e % nx;
        const int b = (e / nx) % p.B;
        const int cb = e / (nx * p.B);
        const int n = p.nrt * 128 + x;
        const uint4* hr = reinterpret_cast<const uint4*>(p.hidden + (static_cast<int64_t>(cb) * p.B + b) * p.K);
        const uint4* wr = reinterpret_cast<const uint4*>(p.Wt + (static_cast<int64_t>(cb) * p.N + n) * p.K);
        float acc = 0.f;
        for (int i0 = lane; i0 < nck; i0 += 32 * 8) {
          uint4 hv[8], wv[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int i = i0 + 32 * u;
            hv[u] = i < nck ? hr[i] : make_uint4(0, 0, 0, 0);
            wv[u] = i < nck ? wr[i] : make_uint4(0, 0, 0, 0);
          }
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const uint32_t hw[4] = {hv[u].x, hv[u].y, hv[u].z, hv[u].w}, ww[4] = {wv[u].x, wv[u].y, wv[u].z, wv[u].w};
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              acc = fmaf(bf16lo(hw[v]), bf16lo(ww[v]), acc);
              acc = fmaf(bf16hi(hw[v]), bf16hi(ww[v]), acc);
            }
          }
        }
        acc = warp_sum(acc);
        if (lane == 0) p.out[(static_cast<int64_t>(cb) * p.B + b) * p.N + n] = acc;
      }
    }
    // ---------------- epilogue: exchange halves with the peer, add, store ----
    const int q = warp & 3;
    const int row = q * 32 + lane;  // TMEM lane = weight row inside the tile
    const uint32_t tq = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const uint32_t peer_recv = tc::mapa_shared(smem_u32(recv), peer);
    const uint32_t peer_rfull = tc::mapa_shared(smem_u32(rfull), peer);
    const uint32_t peer_rempty = tc::mapa_shared(smem_u32(rempty), peer);
    int j = 0;
    for (int t = cluster; t < p.ntiles; t += nclusters, ++j) {
      const int bti = t % p.nbt, rt = (t / p.nbt) % p.nrt, cb = t / (p.nbt * p.nrt);
      bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(tfull, j & 1));
      if (p.alias_recv) {
        // recv lies over the stage ring: my ring is idle once my MMAs are done,
        // and the peer's once it says so
        tc::fence_before_sync();
        tc::mbar_arrive_remote(peer_rempty);
        if (ok) ok = __all_sync(0xffffffffu, tc::mbar_wait_cluster_bounded(rempty, 0));
      } else if (ok && j > 0) {
        // the peer's recv buffer is free once it has read the previous tile's
        ok = __all_sync(0xffffffffu, tc::mbar_wait_cluster_bounded(rempty, (j - 1) & 1));
      }
      if (!ok) {
        record_status(SN_ERR_TIMEOUT);
        break;
      }
      tc::fence_after_sync();
      for (int c = 0; c < half; c += 16) {  // the peer's columns of my partial -> its recv[c][row]
        float v[16];
        tc::tmem_ld16(tq + peer_lo + c, v);
#pragma unroll
        for (int i = 0; i < 16; ++i) st_cluster_f32(peer_recv + static_cast<uint32_t>(((c + i) * 128 + row) * 4), v[i]);
      }
      tc::mbar_arrive_remote(peer_rfull);
      if (!__all_sync(0xffffffffu, tc::mbar_wait_cluster_bounded(rfull, j & 1))) {
        record_status(SN_ERR_TIMEOUT);
        break;
      }
      const int n = rt * 128 + row;
      float* ob = p.out + (static_cast<int64_t>(cb) * p.B) * p.N + n;
      for (int c = 0; c < half; c += 16) {  // my columns: k-half 0 + k-half 1
        float v[16];
        tc::tmem_ld16(tq + own_lo + c, v);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float r = recv[(c + i) * 128 + row];
          const float y = (rank == 0) ? (v[i] + r) : (r + v[i]);
          const int b = bti * p.bt + own_lo + c + i;
          if (b < p.B) ob[static_cast<int64_t>(b) * p.N] = y;
        }
      }
      if (!p.alias_recv) tc::mbar_arrive_remote(peer_rempty);  // my recv may be refilled
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty);
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  tc::cluster_sync_all();  // no CTA leaves while its peer may still touch its shared memory
  if (warp == 1) tc::tmem_dealloc(tmem, tcols);
}

// W [ncb, K, N] -> Wt [ncb, N, K] (32 x 32 tiles through shared memory)
__global__ void transpose_kn_kernel(const __nv_bfloat16* __restrict__ W, __nv_bfloat16* __restrict__ Wt, int K,
                                    int N) {
  __shared__ __nv_bfloat16 tile[32][33];
  const int cb = blockIdx.z;
  const int k0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
  const __nv_bfloat16* src = W + static_cast<int64_t>(cb) * K * N;
  __nv_bfloat16* dst = Wt + static_cast<int64_t>(cb) * K * N;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int k = k0 + r, n = n0 + threadIdx.x;
    if (k < K && n < N) tile[r][threadIdx.x] = src[static_cast<int64_t>(k) * N + n];
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int n = n0 + r, k = k0 + threadIdx.x;
    if (k < K && n < N) dst[static_cast<int64_t>(n) * K + k] = tile[threadIdx.x][r];
  }
}

// ---------------------------------------------------------------------------
// SSD chunk product
// ---------------------------------------------------------------------------
struct SsdParams {
  float* out;  // [BATCH, NCH, NG, CH, CH]
  int batch, seqlen, ng, dstate, ch, nch;
  int mtiles;  // CH / 128 row tiles
  int ntiles;  // CH / 128 column tiles (UMMA N = 128)
  uint32_t a_bytes, b_bytes;  // per 64-wide K block
};

__global__ void __launch_bounds__(kTcThreads, 1)
    ssd_mma_kernel(const __grid_constant__ CUtensorMap mapC, const __grid_constant__ CUtensorMap mapB,
                   const SsdParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int nkb = p.dstate / 64;
  const uint32_t kb_bytes = p.a_bytes + p.b_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + nkb * kb_bytes);  // one barrier per K block
  uint64_t* done = full + nkb;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int u = blockIdx.x;
  const int nt = u % p.ntiles;
  u /= p.ntiles;
  const int mt = u % p.mtiles;
  u /= p.mtiles;
  const int g = u % p.ng;
  u /= p.ng;
  const int c = u % p.nch;
  const int b = u / p.nch;
  const int i0 = c * p.ch + mt * 128;  // first sequence row of the A tile
  const int j0 = c * p.ch + nt * 128;  // first sequence row of the B tile
  const uint32_t tcols = 128;

  if (threadIdx.x == 0) {
    for (int s = 0; s < nkb; ++s) mbar_init(full + s, 1);
    mbar_init(done, 1);
    fence_barrier_init();
    tc::prefetch_map(&mapC);
    tc::prefetch_map(&mapB);
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, tcols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    for (int kb = 0; kb < nkb; ++kb) {
      uint8_t* a = smem + kb * kb_bytes;
      mbar_arrive_expect_tx(full + kb, kb_bytes);
      tc::tma_load_4d(a, &mapC, kb * 64, g, i0, b, full + kb);
      tc::tma_load_4d(a + p.a_bytes, &mapB, kb * 64, g, j0, b, full + kb);
    }
  } else if (warp == 1 && lane == 0) {
    const uint32_t idesc = tc::idesc_bf16_f32(128, 128);
    for (int kb = 0; kb < nkb; ++kb) {
      if (!mbar_wait_bounded(full + kb, 0)) {
        record_status(SN_ERR_TIMEOUT);
        break;
      }
      tc::fence_after_sync();
      const uint8_t* a = smem + kb * kb_bytes;
      const uint64_t da = tc::smem_desc_sw128(a), db = tc::smem_desc_sw128(a + p.a_bytes);
#pragma unroll
      for (int k = 0; k < 4; ++k) tc::mma_bf16(tmem, da + 2 * k, db + 2 * k, idesc, (kb | k) != 0);
    }
    tc::mma_commit(done);
  } else if (warp >= 2) {
    const int q = warp & 3;
    if (__all_sync(0xffffffffu, mbar_wait_bounded(done, 0))) {
      tc::fence_after_sync();
      // Lane l holds row q * 32 + l of the tile.  Each 32 x 32 block goes
      // through shared memory (the operand buffers are free once the MMAs
      // are done; 36-float rows keep both passes free of bank conflicts) so
      // that every store instruction writes four whole 128-byte row
      // segments, not 32 pieces of 16 bytes in 32 different rows.
      float* stage = reinterpret_cast<float*>(smem) + q * (32 * 36);
      float* tile = p.out +
                    ((((static_cast<int64_t>(b) * p.nch + c) * p.ng + g) * p.ch) + mt * 128 + q * 32) * p.ch +
                    nt * 128;
      for (int j = 0; j < 128; j += 32) {
        float v[32];
        tc::tmem_ld32(tmem + (static_cast<uint32_t>(q * 32) << 16) + j, v);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          *reinterpret_cast<float4*>(stage + lane * 36 + 4 * k) =
              make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
        __syncwarp();
#pragma unroll
        for (int it = 0; it < 8; ++it) {
          const int r = it * 4 + (lane >> 3);
          *reinterpret_cast<float4*>(tile + static_cast<int64_t>(r) * p.ch + j + (lane & 7) * 4) =
              *reinterpret_cast<const float4*>(stage + r * 36 + (lane & 7) * 4);
        }
        __syncwarp();
      }
    } else {
      record_status(SN_ERR_TIMEOUT);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) tc::tmem_dealloc(tmem, tcols);
}

// Any-shape fallback: one thread per output element, masked, fp32 accumulate.
__global__ void ssd_simt_kernel(const __nv_bfloat16* __restrict__ C, const __nv_bfloat16* __restrict__ Bm,
                                int64_t sCb, int64_t sCt, int64_t sCg, int64_t sBb, int64_t sBt, int64_t sBg,
                                SsdParams p) {
  const int64_t total = static_cast<int64_t>(p.batch) * p.nch * p.ng * p.ch * p.ch;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t r = e;
    const int j = static_cast<int>(r % p.ch);
    r /= p.ch;
    const int i = static_cast<int>(r % p.ch);
    r /= p.ch;
    const int g = static_cast<int>(r % p.ng);
    r /= p.ng;
    const int c = static_cast<int>(r % p.nch);
    const int b = static_cast<int>(r / p.nch);
    const int ti = c * p.ch + i, tj = c * p.ch + j;
    float acc = 0.f;
    if (ti < p.seqlen && tj < p.seqlen) {
      const __nv_bfloat16* ci = C + b * sCb + ti * sCt + g * sCg;
      const __nv_bfloat16* bj = Bm + b * sBb + tj * sBt + g * sBg;
      for (int d = 0; d < p.dstate; ++d) acc = fmaf(__bfloat162float(ci[d]), __bfloat162float(bj[d]), acc);
    }
    p.out[e] = acc;
  }
}

}  // namespace

int tu_status_bmm(bool reset, cudaStream_t st, int* out) { return read_tu_status(reset, st, out); }

// Codebook head for B >= 5 with K split over CTA pairs; SN_ERR_UNSUPPORTED when
// the cluster launch or the shared-memory plan does not fit.
int head_splitk(const void* hidden, const void* Wt, float* logits, int ncb, int B, int K, int N, bool pdl,
                cudaStream_t st) {
  // the kernel's CUDA-core tail indexes ncb * B * (N mod 128) items in int
  if (static_cast<int64_t>(ncb) * B * 128 >= (int64_t(1) << 31)) return SN_ERR_UNSUPPORTED;
  HeadSkParams p;
  p.out = logits;
  p.hidden = static_cast<const __nv_bfloat16*>(hidden);
  p.Wt = static_cast<const __nv_bfloat16*>(Wt);
  p.ncb = ncb;
  p.B = B;
  p.K = K;
  p.N = N;
  p.bt = std::min(256, (B + 31) / 32 * 32);  // halves of 16-column chunks
  p.nbt = (B + p.bt - 1) / p.bt;
  p.nrt = N / 128;
  p.ntiles = ncb * p.nrt * p.nbt;
  p.a_bytes = 128 * 64 * 2;
  p.stage_bytes = p.a_bytes + static_cast<uint32_t>(p.bt) * 64 * 2;
  const uint32_t recv_bytes = static_cast<uint32_t>(p.bt / 2) * 128 * 4;
  const size_t cap = 227 * 1024 - 1024 - 256;  // opt-in maximum less the alignment slack and the barriers
  // A ring of at most ~110 KB leaves room for the next kernel's CTA beside
  // this one (programmatic dependent launch overlaps its start and first
  // weight loads with this kernel's tail; measured in a chain of calls with
  // 2..8 stages: B = 8 11.7 -> 10.2 us, B = 64 12.9 -> 11.3 us).  Where that
  // leaves fewer than three stages (B = 256: 48 KB stages) the ring takes up
  // to the whole shared memory instead (2 stages measured 18.2 us, 3..4
  // 17.6 us).  With one tile per cluster the exchange buffer lies over the
  // idle ring.
  const size_t coresident = 110 * 1024 - 1024 - 256;
  const int clusters = std::max(1, sm_count() / 2);
  p.alias_recv = p.ntiles <= clusters;
  static const int stages_env = [] {  // SONATA_HEAD_STAGES caps the ring (2..8)
    const char* e = getenv("SONATA_HEAD_STAGES");
    const int v = e ? atoi(e) : 0;
    return (v >= 2 && v <= kSkStagesMax) ? v : 0;
  }();
  const size_t extra = p.alias_recv ? 0 : recv_bytes;
  int stages;
  if (stages_env) {
    stages = stages_env;
  } else if (coresident > extra && (coresident - extra) / p.stage_bytes >= 3) {
    stages = static_cast<int>(std::min<size_t>(kSkStagesMax, (coresident - extra) / p.stage_bytes));
  } else {
    stages = static_cast<int>(std::min<size_t>(kSkStagesMax, (cap - extra) / p.stage_bytes));
  }
  stages = std::min(stages, K / 128);
  if (p.alias_recv)
    while (static_cast<size_t>(stages) * p.stage_bytes < recv_bytes) ++stages;
  if (stages < 2 || static_cast<size_t>(stages) * p.stage_bytes + extra > cap) return SN_ERR_UNSUPPORTED;
  p.stages = stages;
  p.recv_off = p.alias_recv ? 0 : static_cast<uint32_t>(stages) * p.stage_bytes;
  p.bar_off = p.alias_recv ? static_cast<uint32_t>(stages) * p.stage_bytes : p.recv_off + recv_bytes;
  const size_t smem = 1024 + p.bar_off + 8 * (2 * stages + 4) + 16;
  CUtensorMap mapW, mapH;
  const uint64_t dW[3] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N), static_cast<uint64_t>(ncb)};
  const uint64_t sW[2] = {static_cast<uint64_t>(K) * 2, static_cast<uint64_t>(N) * K * 2};
  const uint32_t bW[3] = {64, 128, 1};
  const uint64_t dH[3] = {static_cast<uint64_t>(K), static_cast<uint64_t>(B), static_cast<uint64_t>(ncb)};
  const uint64_t sH[2] = {static_cast<uint64_t>(K) * 2, static_cast<uint64_t>(B) * K * 2};
  const uint32_t bH[3] = {64, static_cast<uint32_t>(p.bt), 1};
  if (!tc::make_map_bf16_sw128(&mapW, Wt, 3, dW, sW, bW) || !tc::make_map_bf16_sw128(&mapH, hidden, 3, dH, sH, bH))
    return SN_ERR_UNSUPPORTED;
  if (cudaFuncSetAttribute(head_splitk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess) {
    cudaGetLastError();
    return SN_ERR_UNSUPPORTED;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * clusters);
  cfg.blockDim = dim3(kSkThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  if (cudaLaunchKernelEx(&cfg, head_splitk_kernel, mapW, mapH, p) != cudaSuccess) {
    cudaGetLastError();
    return SN_ERR_LAUNCH;
  }
  return SN_OK;
}
}  // namespace sn

extern "C" {

int sn_codebook_head_pack(const void* W, int ncb, int K, int N, void* Wt, void* stream) {
  if (!W || !Wt || ncb < 1 || K < 1 || N < 1 || ncb > 65535) return SN_ERR_INVALID_ARGUMENT;
  dim3 grid((N + 31) / 32, (K + 31) / 32, ncb);
  return sn::launch(sn::transpose_kn_kernel, grid, dim3(32, 8), 0, static_cast<cudaStream_t>(stream), false,
                    static_cast<const __nv_bfloat16*>(W), static_cast<__nv_bfloat16*>(Wt), K, N);
}

int sn_codebook_head_bmm(const void* hidden, const void* Wt, float* logits, int ncb, int B, int K, int N,
                         unsigned flags, void* stream) {
  if (!hidden || !Wt || !logits || ncb < 1 || B < 1 || K < 1 || N < 1) return SN_ERR_INVALID_ARGUMENT;
  if (B > INT32_MAX - 31) return SN_ERR_INVALID_ARGUMENT;  // stream tiles round B up in int
  if (flags & ~SN_FLAG_PDL) return SN_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool tc_ok = (K % 64 == 0) && sn::aligned16(hidden) && sn::aligned16(Wt);
  if (B <= 4 || !tc_ok) {
    // decode GEMV over the (codebook, row) pairs, up to 4 streams per launch
    for (int b0 = 0; b0 < B; b0 += 4) {
      const int m = std::min(4, B - b0);
      const int rc = sn::gemv_any(0, Wt, K, static_cast<int64_t>(N) * K, nullptr, 0,
                                  static_cast<const __nv_bfloat16*>(hidden) + static_cast<int64_t>(b0) * K, K,
                                  static_cast<int64_t>(B) * K, logits + static_cast<int64_t>(b0) * N, N,
                                  static_cast<int64_t>(B) * N, m, N, K, ncb, SN_DTYPE_F32, flags, st);
      if (rc != SN_OK) return rc;
    }
    return SN_OK;
  }
  if (K % 128 == 0 && N >= 128) {
    const int rc = sn::head_splitk(hidden, Wt, logits, ncb, B, K, N, (flags & SN_FLAG_PDL) != 0, st);
    if (rc != SN_ERR_UNSUPPORTED) return rc;
  }
  sn::HeadParams p;
  p.out = logits;
  p.ncb = ncb;
  p.B = B;
  p.K = K;
  p.N = N;
  p.bt = std::min(256, (B + 15) / 16 * 16);
  p.nbt = (B + p.bt - 1) / p.bt;
  p.ntiles = (N + 127) / 128;
  p.a_bytes = 128 * 64 * 2;
  p.stage_bytes = p.a_bytes + static_cast<uint32_t>(p.bt) * 64 * 2;
  CUtensorMap mapW, mapH;
  const uint64_t dW[3] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N), static_cast<uint64_t>(ncb)};
  const uint64_t sW[2] = {static_cast<uint64_t>(K) * 2, static_cast<uint64_t>(N) * K * 2};
  const uint32_t bW[3] = {64, 128, 1};
  const uint64_t dH[3] = {static_cast<uint64_t>(K), static_cast<uint64_t>(B), static_cast<uint64_t>(ncb)};
  const uint64_t sH[2] = {static_cast<uint64_t>(K) * 2, static_cast<uint64_t>(B) * K * 2};
  const uint32_t bH[3] = {64, static_cast<uint32_t>(p.bt), 1};
  if (!sn::tc::make_map_bf16_sw128(&mapW, Wt, 3, dW, sW, bW) ||
      !sn::tc::make_map_bf16_sw128(&mapH, hidden, 3, dH, sH, bH))
    return SN_ERR_UNSUPPORTED;
  const size_t smem = 1024 + sn::kHeadStages * static_cast<size_t>(p.stage_bytes) + 256;
  if (cudaFuncSetAttribute(sn::head_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess) {
    cudaGetLastError();
    return SN_ERR_UNSUPPORTED;
  }
  const int units = ncb * p.ntiles * p.nbt;
  return sn::launch(sn::head_mma_kernel, dim3(units), dim3(sn::kTcThreads), smem, st, false, mapW, mapH, p);
}

int sn_ssd_chunk_bmm(const void* C, const void* Bm, int64_t sCb, int64_t sCt, int64_t sCg, int64_t sBb,
                     int64_t sBt, int64_t sBg, int batch, int seqlen, int ngroups, int dstate, int chunk,
                     int nchunks, float* CB_out, void* stream) {
  if (!C || !Bm || !CB_out || batch < 1 || seqlen < 0 || ngroups < 1 || dstate < 1 || chunk < 1 || nchunks < 0)
    return SN_ERR_INVALID_ARGUMENT;
  if (static_cast<int64_t>(nchunks) * chunk < seqlen) return SN_ERR_INVALID_ARGUMENT;
  if (nchunks == 0) return SN_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  sn::SsdParams p;
  p.out = CB_out;
  p.batch = batch;
  p.seqlen = seqlen;
  p.ng = ngroups;
  p.dstate = dstate;
  p.ch = chunk;
  p.nch = nchunks;
  p.mtiles = chunk / 128;
  p.ntiles = chunk / 128;
  p.a_bytes = 128 * 64 * 2;
  p.b_bytes = 128 * 64 * 2;
  const bool tc_ok = (chunk == 128 || chunk == 256) && dstate % 64 == 0 && dstate <= 256 && seqlen > 0 &&
                     sn::aligned16(C) && sn::aligned16(Bm) && ((sCg * 2) % 16 == 0) && ((sCt * 2) % 16 == 0) &&
                     ((sCb * 2) % 16 == 0) && ((sBg * 2) % 16 == 0) && ((sBt * 2) % 16 == 0) &&
                     ((sBb * 2) % 16 == 0);
  const size_t smem = 1024 + static_cast<size_t>(dstate / 64) * (p.a_bytes + p.b_bytes) + 256;
  if (tc_ok && smem <= 220 * 1024) {
    CUtensorMap mapC, mapB;
    const uint64_t dims[4] = {static_cast<uint64_t>(dstate), static_cast<uint64_t>(ngroups),
                              static_cast<uint64_t>(seqlen), static_cast<uint64_t>(batch)};
    const uint64_t stC[3] = {static_cast<uint64_t>(sCg) * 2, static_cast<uint64_t>(sCt) * 2,
                             static_cast<uint64_t>(sCb) * 2};
    const uint64_t stB[3] = {static_cast<uint64_t>(sBg) * 2, static_cast<uint64_t>(sBt) * 2,
                             static_cast<uint64_t>(sBb) * 2};
    const uint32_t boxC[4] = {64, 1, 128, 1};
    const uint32_t boxB[4] = {64, 1, 128, 1};
    if (sn::tc::make_map_bf16_sw128(&mapC, C, 4, dims, stC, boxC) &&
        sn::tc::make_map_bf16_sw128(&mapB, Bm, 4, dims, stB, boxB)) {
      if (cudaFuncSetAttribute(sn::ssd_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) ==
          cudaSuccess) {
        const int units = batch * nchunks * ngroups * p.mtiles * p.ntiles;
        return sn::launch(sn::ssd_mma_kernel, dim3(units), dim3(sn::kTcThreads), smem, st, false, mapC, mapB, p);
      }
      cudaGetLastError();
    }
  }
  const int64_t total = static_cast<int64_t>(batch) * nchunks * ngroups * chunk * chunk;
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 148 * 16));
  return sn::launch(sn::ssd_simt_kernel, dim3(blocks), dim3(256), 0, st, false,
                    static_cast<const __nv_bfloat16*>(C), static_cast<const __nv_bfloat16*>(Bm), sCb, sCt, sCg,
                    sBb, sBt, sBg, p);
}

}  // extern "C"
