// 3xTF32 projection GEMM for 128 activation rows per CTA (the prefill, and any
// GEMM with more than 64 rows).
//
// Same method as gemm_tc.cu (W split into W_b + W_s in registers and stored to
// tensor memory, X pre-split by its producer, tensor-core accumulation promoted
// into IEEE fp32 registers), but each MMA covers 128 activation rows:
//
//   D[:, 0:256] += W_b . [X_b ; X_s]      (N = 256: 128 rows of X_b, then of X_s)
//   D[:, 0:128] += W_s . X_b              (N = 128)
//
// A tf32 MMA of N <= 128 costs ~60 cycles and one of N = 256 ~130, so twice
// the rows take the same 8 instructions per 32-wide K chunk at ~1.5x the
// tensor time.  The 256-column accumulator leaves room for 2 A stages of two
// chunks but not for a second accumulator, so the MMA issuer waits while the
// promoters drain it (every 8 chunks).
//   warp 0       TMA of the W tile [128 x 32] into a 5-deep ring
//   warp 1       MMA issuer (one wait and one commit per stage of two chunks)
//   warps 2..5   split W rows into the TMEM A stages (one lane quarter each);
//                warp 2 also waits for the stage's activation tiles
//   warps 6..13  promote: two warps per lane quarter, 64 activation rows each
//   warp 14      TMA of [X_b ; X_s] (4 boxes of 64 rows per chunk), 2 stages
// Epilogue: shared-memory tile, every thread stores float4s (tc_epilogue.cuh).
// Every mbarrier wait is bounded.
#include <cuda.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "engine.h"
#include "tc_epilogue.cuh"
#include "tcgen05.cuh"

namespace rtr {

constexpr int TW_THREADS = 480;          // 15 warps
constexpr int TW_KC = 32;
constexpr int TW_WROWS = 128;
constexpr int TW_NTOK = 128;
constexpr int TW_WSTAGES = 5;            // W ring depth (chunks)
constexpr int TW_CPS = 2;                // chunks per A/X stage
constexpr int TW_STAGES = 2;             // A/X stages
constexpr int TW_PROMOTE = 8;            // chunks per promotion
constexpr int TW_GSTAGES = TW_PROMOTE / TW_CPS;
constexpr int TW_W_BYTES = TW_WROWS * 128;        // 16 KB
constexpr int TW_XC_BYTES = 2 * TW_NTOK * 128;    // 32 KB: [X_b ; X_s] of one chunk
constexpr int TW_X_BYTES = TW_CPS * TW_XC_BYTES;  // one stage
constexpr int TW_D_COLS = 2 * TW_NTOK;            // 256
constexpr int TW_AC_COLS = 2 * TW_KC;             // W_b and W_s of one chunk
constexpr int TW_A_COLS = TW_CPS * TW_AC_COLS;    // one stage
constexpr int TW_TMEM_COLS = 512;                 // accumulator + 2 A stages
constexpr int TW_NBARS = 2 * TW_WSTAGES + 3 * TW_STAGES + 3;
constexpr int TW_RING_BYTES = TW_WSTAGES * TW_W_BYTES + TW_STAGES * TW_X_BYTES;
constexpr int TW_SMEM_BYTES = TW_RING_BYTES + 1024 + 8 * TW_NBARS + 16;
constexpr int TW_RLD = TW_WROWS + 4;
static_assert(TW_NTOK * TW_RLD * 4 <= TW_RING_BYTES, "epilogue tile fits in the rings");
static_assert(TW_D_COLS + TW_STAGES * TW_A_COLS <= TW_TMEM_COLS, "tensor memory budget");
static_assert(TW_GSTAGES % TW_STAGES == 0, "a group starts on stage 0");

__global__ void __launch_bounds__(TW_THREADS, 1)
    gemm_tc_wide_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmXb,
                        const __grid_constant__ CUtensorMap tmXs, TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* wring = smem;
  uint8_t* xring = smem + TW_WSTAGES * TW_W_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(xring + TW_STAGES * TW_X_BYTES);
  uint64_t* w_full = bars;
  uint64_t* w_empty = w_full + TW_WSTAGES;
  uint64_t* x_full = w_empty + TW_WSTAGES;  // [TW_STAGES] activation stage landed (TMA)
  uint64_t* a_full = x_full + TW_STAGES;    // [TW_STAGES] split weights stored, activations landed
  uint64_t* s_empty = a_full + TW_STAGES;   // [TW_STAGES] MMAs of the stage done (frees A and X)
  uint64_t* d_full = s_empty + TW_STAGES;
  uint64_t* d_empty = d_full + 1;
  uint64_t* red_bar = d_empty + 1;         // split-K finish: every CTA of the cluster arrived
  volatile int* abort_flag = reinterpret_cast<volatile int*>(red_bar + 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(red_bar + 1) + 1;
  __shared__ int go;                        // this cluster finishes the tile

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tok0 = blockIdx.x * TW_NTOK;
  const int n0 = blockIdx.y * TW_WROWS;
  const int nchunks = (p.K + TW_KC - 1) / TW_KC;
  const int c0 = (int)((long)blockIdx.z * nchunks / p.splits);
  const int c1 = (int)((long)(blockIdx.z + 1) * nchunks / p.splits);
  const int nloc = c1 - c0;
  const int nstages = (nloc + TW_CPS - 1) / TW_CPS;
  const int ngroups = (nloc + TW_PROMOTE - 1) / TW_PROMOTE;

  if (threadIdx.x == 0) {
    for (int s = 0; s < TW_WSTAGES; ++s) { mbar_init(smem_addr(&w_full[s]), 1); mbar_init(smem_addr(&w_empty[s]), 4); }
    for (int s = 0; s < TW_STAGES; ++s) {
      mbar_init(smem_addr(&x_full[s]), 1);
      mbar_init(smem_addr(&a_full[s]), 4);
      mbar_init(smem_addr(&s_empty[s]), 1);
    }
    mbar_init(smem_addr(d_full), 1);
    mbar_init(smem_addr(d_empty), 8);
    mbar_init(smem_addr(red_bar), cluster_ncta());
    go = 0;
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmXb);
    tma_prefetch_desc(&tmXs);
  }
  if (warp == 1) tmem_alloc(smem_addr(tmem_slot), TW_TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  if (cluster_ncta() > 1) cluster_sync_all();  // peers' barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_a = tmem + TW_D_COLS;

  int w_issued = 0, x_issued = 0;
  uint32_t last_bar = 0, last_par = 0;  // MMA thread: barrier and phase of its last commit
  float acc[64];  // live only in the promoter warps

  if (warp == 0) {
    if (lane == 0) {
      // weights do not depend on the previous kernel: no griddepcontrol.wait
      for (int i = 0; i < nloc; ++i) {
        const int s = i % TW_WSTAGES;
        if (!mbar_wait(smem_addr(&w_empty[s]), ((i / TW_WSTAGES) & 1) ^ 1, abort_flag)) break;
        const uint32_t fb = smem_addr(&w_full[s]);
        mbar_expect_tx(fb, TW_W_BYTES);
        tma_load_2d(smem_addr(wring + s * TW_W_BYTES), &tmW, 0, (blockIdx.y * nchunks + c0 + i) * TW_WROWS, fb);
        w_issued = i + 1;
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // MMA issuer: stage indices, descriptors and accumulate flags are
    // compile-time; one wait and one commit per stage of two chunks.
    if (lane == 0) {
      constexpr uint32_t id_cat = idesc_tf32(TW_WROWS, 2 * TW_NTOK);
      constexpr uint32_t id_x = idesc_tf32(TW_WROWS, TW_NTOK);
      const uint64_t bx0 = sw128_desc(smem_addr(xring));
      bool ok = true;
      for (int j = 0; ok && j * TW_GSTAGES < nstages; ++j) {
        // single accumulator: a new group starts once the promoters drained the last one
        if (j >= 1 && !mbar_wait(smem_addr(d_empty), (j - 1) & 1, abort_flag)) break;
#pragma unroll
        for (int u = 0; u < TW_GSTAGES; ++u) {
          const int q = j * TW_GSTAGES + u, s = u % TW_STAGES;
          if (q >= nstages) break;
          if (!mbar_wait(smem_addr(&a_full[s]), (u / TW_STAGES) & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < TW_CPS; ++c) {
            if (c > 0 && q * TW_CPS + c >= nloc) break;
            const uint32_t ab = tmem_a + s * TW_A_COLS + c * TW_AC_COLS;
            const uint64_t bx = bx0 + (uint64_t)((s * TW_X_BYTES + c * TW_XC_BYTES) >> 4);
#pragma unroll
            for (int kk = 0; kk < TW_KC / 8; ++kk) {  // 8 tf32 = 32 bytes along K
              mma_tf32_ts(tmem, ab + kk * 8, bx + 2 * kk, id_cat, (u | c | kk) ? 1u : 0u);
              mma_tf32_ts(tmem, ab + TW_KC + kk * 8, bx + 2 * kk, id_x, 1u);
            }
          }
          mma_commit(smem_addr(&s_empty[s]));
          last_bar = smem_addr(&s_empty[s]);
          last_par = (u / TW_STAGES) & 1;
        }
        if (!ok) break;
        mma_commit(smem_addr(d_full));
        last_bar = smem_addr(d_full);
        last_par = j & 1;
      }
    }
    __syncwarp();
  } else if (warp == 14) {
    pdl_wait();
    if (lane == 0) {
      for (int q = 0; q < nstages; ++q) {
        const int s = q % TW_STAGES;
        if (!mbar_wait(smem_addr(&s_empty[s]), ((q / TW_STAGES) & 1) ^ 1, abort_flag)) break;
        const int nc = nloc - q * TW_CPS < TW_CPS ? nloc - q * TW_CPS : TW_CPS;
        const uint32_t fb = smem_addr(&x_full[s]);
        uint8_t* st = xring + s * TW_X_BYTES;
        mbar_expect_tx(fb, nc * TW_XC_BYTES);
        for (int c = 0; c < nc; ++c) {
          const int kx = (c0 + q * TW_CPS + c) * TW_KC;
          uint8_t* sc = st + c * TW_XC_BYTES;
          tma_load_2d(smem_addr(sc), &tmXb, kx, tok0, fb);
          tma_load_2d(smem_addr(sc + 64 * 128), &tmXb, kx, tok0 + 64, fb);
          tma_load_2d(smem_addr(sc + 128 * 128), &tmXs, kx, tok0, fb);
          tma_load_2d(smem_addr(sc + 192 * 128), &tmXs, kx, tok0 + 64, fb);
        }
        x_issued = q + 1;
      }
    }
    __syncwarp();
  } else if (warp <= 5) {
    // --------------------------- warps 2..5: split W rows into TMEM
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    for (int i = 0; i < nloc; ++i) {
      const int ws = i % TW_WSTAGES, q = i / TW_CPS, c = i % TW_CPS, s = q % TW_STAGES;
      if (!mbar_wait(smem_addr(&w_full[ws]), (i / TW_WSTAGES) & 1, abort_flag)) break;
      const uint8_t* tile = wring + ws * TW_W_BYTES + row * 128;
      uint32_t big[TW_KC], small[TW_KC];
#pragma unroll
      for (int k4 = 0; k4 < TW_KC / 4; ++k4) {  // undo the 128B swizzle: chunk k4 lives at k4 ^ (row % 8)
        const float4 v = *reinterpret_cast<const float4*>(tile + ((k4 ^ (row & 7)) << 4));
        big[4 * k4] = __float_as_uint(v.x); big[4 * k4 + 1] = __float_as_uint(v.y);
        big[4 * k4 + 2] = __float_as_uint(v.z); big[4 * k4 + 3] = __float_as_uint(v.w);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(&w_empty[ws]));
#pragma unroll
      for (int k = 0; k < TW_KC; ++k) {
        const float w = __uint_as_float(big[k]);
        const float bv = tf32_round(w);
        big[k] = __float_as_uint(bv);
        small[k] = __float_as_uint(w - bv);
      }
      if (c == 0 && !mbar_wait(smem_addr(&s_empty[s]), ((q / TW_STAGES) & 1) ^ 1, abort_flag)) break;
      tc_fence_after();
      const uint32_t a = tmem_a + lane_base + s * TW_A_COLS + c * TW_AC_COLS;
      tmem_st32(a, big);
      tmem_st32(a + TW_KC, small);
      if (c == TW_CPS - 1 || i == nloc - 1) {  // the stage is complete
        tmem_st_wait();
        tc_fence_before();
        // one converter also waits for the stage's activation tiles, so the
        // MMA thread waits on a single barrier per stage
        const bool x_ok = warp != 2 || mbar_wait(smem_addr(&x_full[s]), (q / TW_STAGES) & 1, abort_flag);
        __syncwarp();
        if (!x_ok) break;
        if (lane == 0) mbar_arrive(smem_addr(&a_full[s]));
      }
    }
  } else {
    // ------------ warps 6..13: promote (lane quarter warp & 3, rows half * 64 ..)
    pdl_wait();
    const int quarter = warp & 3, half = (warp - 6) >> 2;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
#pragma unroll
    for (int j = 0; j < 64; ++j) acc[j] = 0.f;
    for (int g = 0; g < ngroups; ++g) {
      if (!mbar_wait(smem_addr(d_full), g & 1, abort_flag)) break;
      tc_fence_after();
      const uint32_t d = tmem + lane_base + half * 64;
#pragma unroll
      for (int cb = 0; cb < 64; cb += 16) {
        uint32_t r[16], s[16];
        tmem_ld16(d + cb, r);             // W_b.X_b + W_s.X_b
        tmem_ld16(d + TW_NTOK + cb, s);   // W_b.X_s
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[cb + j] += __uint_as_float(r[j]) + __uint_as_float(s[j]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(d_empty));
    }
  }
  pdl_launch_dependents();
  __syncthreads();  // every role is done waiting: the abort flag is final

  // drain on abort: issued copies and MMAs must land before smem/TMEM go away
  const bool aborted = *abort_flag != 0;
  if (aborted) {
    if (threadIdx.x == 0) atomicOr(p.status, RTR_DEV_TIMEOUT);
    if (warp == 0 && lane == 0) drain_ring(w_full, TW_WSTAGES, w_issued);
    if (warp == 14 && lane == 0) drain_ring(x_full, TW_STAGES, x_issued);
    if (warp == 1 && lane == 0 && last_bar) mbar_drain(last_bar, last_par);  // all MMAs issued
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TW_TMEM_COLS);
  }
  if (aborted) {
    if (p.splits > 1) {
      pdl_wait();  // the tickets are shared with earlier kernels
      int r0, r1;
      splitk_claim(p, smem_addr(red_bar), &go, 0, blockIdx.y * gridDim.x + blockIdx.x, r0, r1, true);
    }
    return;
  }

  const bool have = warp >= 6 && warp <= 13;
  const int quarter = warp & 3, half = (warp - 6) >> 2;
  const int col = quarter * 32 + lane;     // weight row of this thread within the tile
  const int n = n0 + col;
  const int rows = p.M - tok0 < TW_NTOK ? p.M - tok0 : TW_NTOK;
  const int cols4 = (p.N - n0 < TW_WROWS ? p.N - n0 : TW_WROWS) >> 2;
  float4* red4 = reinterpret_cast<float4*>(smem);  // the rings are free now
  if (p.splits > 1) {
    // partial tiles are tile-contiguous: ws[(split * tiles + tile)][row][128]
    const int tile = blockIdx.y * gridDim.x + blockIdx.x;
    const long tstride = (long)gridDim.x * gridDim.y * (TW_NTOK * TW_WROWS);
    if (have && n < p.N) {
      float* w = p.ws + blockIdx.z * tstride + (long)tile * (TW_NTOK * TW_WROWS) + half * 64 * TW_WROWS + col;
#pragma unroll
      for (int j = 0; j < 64; ++j)
        if (half * 64 + j < rows) __stcg(w + j * TW_WROWS, acc[j]);
    }
    __threadfence();
    __syncthreads();
    splitk_finish<TW_THREADS, TW_NTOK>(p, red4, smem_addr(red_bar), &go, tok0, n0, rows, cols4, tile, tstride);
    return;
  }
  if (have && n < p.N) {
    float* red = reinterpret_cast<float*>(smem) + half * 64 * TW_RLD + col;
#pragma unroll
    for (int j = 0; j < 64; ++j)
      if (half * 64 + j < rows) red[j * TW_RLD] = acc[j];
  }
  __syncthreads();
  tile_epilogue<TW_THREADS>(p, red4, TW_RLD / 4, tok0, n0, rows, cols4);
}

cudaError_t gemm_tc_wide_init() {
  return cudaFuncSetAttribute(gemm_tc_wide_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TW_SMEM_BYTES);
}

// Same arguments and checks as gemm_tc(); the activation tensor maps keep
// their 64-row boxes (four loads fill one 128-row stage).
cudaError_t gemm_tc_wide(const TensorMap& tmW, const TensorMap& tmXb, const TensorMap& tmXs, float* C, float* C_big,
                         float* C_small, int ldc, const float* bias, int M, int N, int K, int epi, float* ws,
                         size_t ws_floats, int* tickets, int max_tickets, uint32_t* status, int sms,
                         cudaStream_t stream, bool pdl, const RopeArgs* rope, const NormFold* fold) {
  if (epi == EPI_SWIGLU && (!C_big || !C_small)) return cudaErrorInvalidValue;
  if (epi == EPI_ROPE) {
    if (!rope || !bias || (rope->head_dim != 64 && rope->head_dim != 128) ||
        N != (rope->heads + 2 * rope->kv_heads) * rope->head_dim || (reinterpret_cast<uintptr_t>(bias) & 15))
      return cudaErrorInvalidValue;
  }
  if (epi != EPI_ROPE && (N % 4 || ldc % 4 || (reinterpret_cast<uintptr_t>(C) & 15))) return cudaErrorInvalidValue;
  if (fold && fold->ss_out && (epi != EPI_RESID || !C_big || !C_small || fold->parts * 128 != N)) return cudaErrorInvalidValue;
  if (fold && fold->ss_in && (epi == EPI_RESID || fold->hidden != K)) return cudaErrorInvalidValue;
  const int tt = (M + TW_NTOK - 1) / TW_NTOK, wt = (N + TW_WROWS - 1) / TW_WROWS;
  const int nchunks = (K + TW_KC - 1) / TW_KC;
  int dev = 0;
  cudaGetDevice(&dev);
  const SplitPlan plan = tc_split_plan(tt * wt, nchunks, sms, g_tc_clusters[dev < kMaxDevices ? dev : 0], TC_MAX_CLUSTER,
                                       ws_floats, (long)TW_NTOK * TW_WROWS, max_tickets);
  const int splits = plan.splits, cs = plan.cluster;
  TcParams p{C, C_big, C_small, bias, M, N, K, ldc, epi, splits, ws, tickets, status, {}, {}};
  if (rope) p.rope = *rope;
  if (fold) p.fold = *fold;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tt, wt, splits);
  cfg.blockDim = dim3(TW_THREADS);
  cfg.dynamicSmemBytes = TW_SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = cs;
  cfg.attrs = attr;
  cfg.numAttrs = cs > 1 ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, gemm_tc_wide_kernel, *reinterpret_cast<const CUtensorMap*>(&tmW),
                            *reinterpret_cast<const CUtensorMap*>(&tmXb),
                            *reinterpret_cast<const CUtensorMap*>(&tmXs), p);
}

}  // namespace rtr
