// FP32-accurate projection GEMM from fp16 pairs on the 5th-generation tensor
// cores.
//
//   C[m, n] (+ epilogue) = sum_k X[m, k] * W[n, k]
//
// Both operands are carried as pairs of fp16 values with 22 significant bits
// between them:
//   W = w_hi + w_lo / 2048               (packed once at load, 4 bytes a weight)
//   X = 16 (x_hi + x_lo / 2048)          (written by the activation producers)
// so that, dropping the 2^-22 cross term,
//   X.W = 16 [ x_hi.w_hi + (x_lo.w_hi + x_hi.w_lo) / 2048 ]
// Three fp16 products with fp32 accumulation, all operands straight from
// shared memory: no operand conversion inside the kernel, which is what bounds
// the 3xTF32 kernel (gemm_tc.cu) below the HBM rate (its converter warps'
// TMEM stores and shared-memory reads).
//
// A CTA owns 128 weight rows (MMA M) x NTOK activation rows (64 or 128) for a
// range of K, walked in 64-element chunks (one 128-byte row of fp16):
//   warp 0     TMA of the packed weight block of a chunk: [w_hi 128 rows;
//              w_lo 128 rows] x 64 (32 KB, one box, 128B swizzle)
//   warp 2     TMA of the activation tiles [x_hi NTOK rows; x_lo NTOK rows]
//              both into a ring of one-chunk stages (one full barrier: two
//              arrivals + bytes; one empty barrier)
//   warp 1     MMA issuer: per 16-element step two tcgen05.mma kind::f16,
//                D[0, 2 NTOK)      (+)= w_hi . [x_hi; x_lo]    (N = 2 NTOK)
//                D[NTOK, 2 NTOK)    += w_lo . x_hi             (N = NTOK)
//              one wait and one commit per stage
//   warps 4..  promote the TMEM accumulator (double-buffered) into fp32
//              registers every 4 chunks (K = 256):
//                acc += D[j] + D[NTOK + j] / 2048
// The finished sums are scaled by 16 (exact) and go through the split-K
// cluster finish and the epilogues shared with the 3xTF32 kernels
// (tc_epilogue.cuh).  Every mbarrier wait is bounded.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "engine.h"
#include "tc_epilogue.cuh"
#include "tcgen05.cuh"

namespace rtr {

constexpr int FX_KC = 64;                 // K elements per chunk (128-byte fp16 rows)
constexpr int FX_WROWS = 128;             // MMA M
constexpr int FX_PROMOTE = 4;             // chunks accumulated in TMEM per promotion
constexpr int FX_WPLANE = FX_WROWS * 128; // one plane (hi or lo) of a chunk: 16 KB
constexpr int FX_W_BYTES = 2 * FX_WPLANE; // weight block of a chunk: 32 KB

template <int NTOK> struct FxCfg {
  static constexpr int THREADS = NTOK == 64 ? 256 : 384;     // 4 + NTOK / 16 warps
  static constexpr int PROMOTERS = NTOK / 16;                // warps 4 .. 4 + PROMOTERS
  static constexpr int XPLANE = NTOK * 128;                  // x_hi or x_lo tile of a chunk
  static constexpr int X_BYTES = 2 * XPLANE;
  static constexpr int STAGES = NTOK == 64 ? 4 : 3;          // 192 KB of ring either way
  static constexpr int D_COLS = 2 * NTOK;                    // [hi.hi | hi.lo + lo.hi]
  static constexpr int TMEM_COLS = 2 * D_COLS;               // double-buffered
  static constexpr int NBARS = 2 * STAGES + 5;
  static constexpr int RING = STAGES * (FX_W_BYTES + X_BYTES);
  static constexpr int SMEM = RING + 1024 + 8 * NBARS + 16;
  static constexpr int RLD = FX_WROWS + 4;                   // epilogue tile row stride (floats)
  static_assert(NTOK * RLD * 4 <= RING, "epilogue tile fits in the ring");
  static_assert(TMEM_COLS <= 512, "tensor memory");
};

// Bound of the pipeline waits and the test switch that withholds the
// activation copies (rtr_debug_wait_control); one copy per device.
static __device__ WaitControl g_fx_wait = {kWaitCycles, 0, 0};

template <int NTOK>
__global__ void __launch_bounds__(FxCfg<NTOK>::THREADS, 1)
    gemm_f16x2_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmXh,
                      const __grid_constant__ CUtensorMap tmXl, TcParams p) {
  using Cfg = FxCfg<NTOK>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* wring = smem;
  uint8_t* xring = smem + STAGES * FX_W_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(xring + STAGES * Cfg::X_BYTES);
  uint64_t* s_full = bars;                  // [STAGES] W and X of the stage landed (2 arrivals + bytes)
  uint64_t* s_empty = s_full + STAGES;      // [STAGES] the stage's MMAs are done
  uint64_t* d_full = s_empty + STAGES;      // [2]
  uint64_t* d_empty = d_full + 2;           // [2]
  uint64_t* red_bar = d_empty + 2;          // split-K finish: every CTA of the cluster arrived
  volatile int* abort_flag = reinterpret_cast<volatile int*>(red_bar + 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(red_bar + 1) + 1;
  __shared__ int go;                        // this cluster finishes the tile
  __shared__ int issued[2];                 // copies issued by the W and X producers (abort path)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tok0 = blockIdx.x * NTOK;
  const int n0 = blockIdx.y * FX_WROWS;
  const long long lim = g_fx_wait.wait_cycles;
  const int nchunks = (p.K + FX_KC - 1) / FX_KC;
  const int c0 = (int)((long)blockIdx.z * nchunks / p.splits);
  const int c1 = (int)((long)(blockIdx.z + 1) * nchunks / p.splits);
  const int nloc = c1 - c0;
  const int ngroups = (nloc + FX_PROMOTE - 1) / FX_PROMOTE;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) { mbar_init(smem_addr(&s_full[s]), 2); mbar_init(smem_addr(&s_empty[s]), 1); }
    for (int b = 0; b < 2; ++b) { mbar_init(smem_addr(&d_full[b]), 1); mbar_init(smem_addr(&d_empty[b]), Cfg::PROMOTERS); }
    mbar_init(smem_addr(red_bar), cluster_ncta());
    go = 0;
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmXh);
    tma_prefetch_desc(&tmXl);
  }
  if (warp == 1) tmem_alloc(smem_addr(tmem_slot), Cfg::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  if (cluster_ncta() > 1) cluster_sync_all();  // peers' barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  int w_issued = 0, x_issued = 0;
  uint32_t last_bar = 0, last_par = 0;  // MMA thread: barrier and phase of its last commit
  float acc[64];  // live only in the promoter warps

  if (warp == 0) {
    if (lane == 0) {
      // ----------------------------------------------- weight producer (TMA)
      // weights do not depend on the previous kernel: no griddepcontrol.wait
      for (int q = 0; q < nloc; ++q) {
        const int s = q % STAGES;
        if (!mbar_wait(smem_addr(&s_empty[s]), ((q / STAGES) & 1) ^ 1, abort_flag, lim)) break;
        const uint32_t fb = smem_addr(&s_full[s]);
        mbar_expect_tx(fb, FX_W_BYTES);
        // packed block of (tile, chunk): 256 rows of 128 bytes, contiguous
        tma_load_2d(smem_addr(wring + s * FX_W_BYTES), &tmW, 0, (blockIdx.y * nchunks + c0 + q) * 2 * FX_WROWS, fb);
        w_issued = q + 1;
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ----------------------------------------------------------- MMA issuer
      constexpr uint32_t id_cat = idesc_f16(FX_WROWS, 2 * NTOK);
      constexpr uint32_t id_x = idesc_f16(FX_WROWS, NTOK);
      const uint64_t ad0 = sw128_desc(smem_addr(wring)), bd0 = sw128_desc(smem_addr(xring));
      bool ok = true;
      for (int j = 0; ok && j < ngroups; ++j) {  // one promotion group
        const int b = j & 1;
        if (j >= 2 && !mbar_wait(smem_addr(&d_empty[b]), ((j >> 1) - 1) & 1, abort_flag, lim)) break;
        const uint32_t d = tmem + b * Cfg::D_COLS;
#pragma unroll
        for (int u = 0; u < FX_PROMOTE; ++u) {
          const int q = j * FX_PROMOTE + u;
          if (q < nloc) {
            const int s = q % STAGES;
            if (!mbar_wait(smem_addr(&s_full[s]), (q / STAGES) & 1, abort_flag, lim)) {
              ok = false;
            } else {
              tc_fence_after();
              const uint64_t ah = ad0 + (uint64_t)((s * FX_W_BYTES) >> 4);
              const uint64_t al = ah + (uint64_t)(FX_WPLANE >> 4);
              const uint64_t bx = bd0 + (uint64_t)((s * Cfg::X_BYTES) >> 4);
#pragma unroll
              for (int kk = 0; kk < FX_KC / 16; ++kk) {  // 16 fp16 = 32 bytes along K
                mma_f16_ss(d, ah + 2 * kk, bx + 2 * kk, id_cat, (u | kk) ? 1u : 0u);
                mma_f16_ss(d + NTOK, al + 2 * kk, bx + 2 * kk, id_x, 1u);
              }
              mma_commit(smem_addr(&s_empty[s]));
              last_bar = smem_addr(&s_empty[s]);
              last_par = (q / STAGES) & 1;
            }
          }
          if (!ok) break;
        }
        if (!ok) break;
        mma_commit(smem_addr(&d_full[b]));
        last_bar = smem_addr(&d_full[b]);
        last_par = (j >> 1) & 1;
      }
    }
    __syncwarp();
  } else if (warp == 2) {
    // ------------------------------------------- activation producer (TMA)
    pdl_wait();
    if (lane == 0 && !g_fx_wait.withhold_x) {
      for (int q = 0; q < nloc; ++q) {
        const int s = q % STAGES;
        if (!mbar_wait(smem_addr(&s_empty[s]), ((q / STAGES) & 1) ^ 1, abort_flag, lim)) break;
        const uint32_t fb = smem_addr(&s_full[s]);
        uint8_t* st = xring + s * Cfg::X_BYTES;
        mbar_expect_tx(fb, Cfg::X_BYTES);
        const int kx = (c0 + q) * FX_KC;
#pragma unroll
        for (int h = 0; h < NTOK / 64; ++h) {  // 64-row boxes
          tma_load_2d(smem_addr(st + h * 64 * 128), &tmXh, kx, tok0 + h * 64, fb);
          tma_load_2d(smem_addr(st + Cfg::XPLANE + h * 64 * 128), &tmXl, kx, tok0 + h * 64, fb);
        }
        x_issued = q + 1;
      }
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ----------------------------------- promote the accumulators into fp32
    // TMEM lane quarter = warp % 4 (weight rows); column half (NTOK = 128) =
    // which 64 activation rows
    const int half = (warp - 4) >> 2;
#pragma unroll
    for (int j = 0; j < 64; ++j) acc[j] = 0.f;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    for (int g = 0; g < ngroups; ++g) {
      const int b = g & 1;
      if (!mbar_wait(smem_addr(&d_full[b]), (g >> 1) & 1, abort_flag, lim)) break;
      tc_fence_after();
      const uint32_t d = tmem + lane_base + b * Cfg::D_COLS + half * 64;
#pragma unroll
      for (int cb = 0; cb < 64; cb += 32) {
        uint32_t r[32];
        float hh[32];
        tmem_ld32(d + cb, r);          // x_hi . w_hi
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) hh[j] = __uint_as_float(r[j]);
        tmem_ld32(d + NTOK + cb, r);   // x_lo . w_hi + x_hi . w_lo
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[cb + j] += hh[j] + __uint_as_float(r[j]) * (1.0f / kPairLo);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(&d_empty[b]));
    }
  }
  pdl_launch_dependents();
  if (warp == 0 && lane == 0) issued[0] = w_issued;
  if (warp == 2 && lane == 0) issued[1] = x_issued;
  __syncthreads();  // every role is done waiting: the abort flag is final

  // drain on abort: issued copies and MMAs must land before smem/TMEM go away
  const bool aborted = *abort_flag != 0;
  if (aborted) {
    if (threadIdx.x == 0) {
      atomicOr(p.status, RTR_DEV_TIMEOUT);
      // a stage's full barrier takes one arrival from each producer: stand in
      // for the one that stopped earlier, then wait for the issued copies
      const int wi = issued[0], xi = issued[1];
      ring_stand_in(s_full, STAGES, xi, wi);
      ring_stand_in(s_full, STAGES, wi, xi);
      drain_ring(s_full, STAGES, wi > xi ? wi : xi);
    }
    if (warp == 1 && lane == 0 && last_bar) mbar_drain(last_bar, last_par);  // all MMAs issued
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
  pdl_wait();  // the split-K workspace and the epilogue touch memory of earlier kernels
  const int tile = blockIdx.y * gridDim.x + blockIdx.x;
  if (aborted) {
    if (p.splits > 1) {
      int r0, r1;
      splitk_claim(p, smem_addr(red_bar), &go, 0, tile, r0, r1, true);
    }
    return;
  }

  const bool have = warp >= 4;
  const int quarter = warp & 3, half = (warp - 4) >> 2;
  const int n = n0 + quarter * 32 + lane;  // weight row of this thread
  const int rows = p.M - tok0 < NTOK ? p.M - tok0 : NTOK;
  const int cols4 = (p.N - n0 < FX_WROWS ? p.N - n0 : FX_WROWS) >> 2;
  float4* red4 = reinterpret_cast<float4*>(smem);  // the rings are free now
  if (p.splits > 1) {
    // Partial tiles are tile-contiguous: ws[(split * tiles + tile)][row][128].
    const long tstride = (long)gridDim.x * gridDim.y * (NTOK * FX_WROWS);
    if (have && n < p.N) {
      float* w = p.ws + blockIdx.z * tstride + (long)tile * (NTOK * FX_WROWS) + (half * 64) * FX_WROWS +
                 quarter * 32 + lane;
#pragma unroll
      for (int j = 0; j < 64; ++j)
        if (half * 64 + j < rows) __stcg(w + j * FX_WROWS, acc[j] * kPairScale);
    }
    __threadfence();
    __syncthreads();
    splitk_finish<Cfg::THREADS, NTOK>(p, red4, smem_addr(red_bar), &go, tok0, n0, rows, cols4, tile, tstride);
    return;
  }
  // Stage the finished tile in shared memory ([NTOK][RLD], padded so the
  // float4 reads of consecutive rows spread over the banks); then every
  // thread of the CTA stores float4s.
  if (have && n < p.N) {
    float* red = reinterpret_cast<float*>(smem) + (half * 64) * Cfg::RLD + quarter * 32 + lane;
#pragma unroll
    for (int j = 0; j < 64; ++j)
      if (half * 64 + j < rows) red[j * Cfg::RLD] = acc[j] * kPairScale;
  }
  __syncthreads();
  tile_epilogue<Cfg::THREADS>(p, red4, Cfg::RLD / 4, tok0, n0, rows, cols4);
}

// ---------------------------------------------------------------- host side
// W [N, K] fp32 (times col_scale[k] when given: the folded RMSNorm weight)
// becomes blocks [N/128 tiles][K/64 chunks][hi 128 rows; lo 128 rows][64 fp16]
// (zero padded): w_hi = fp16(w), w_lo = fp16((w - w_hi) * 2048); every TMA
// load of a (tile, chunk) reads 32 KB of contiguous memory.
__global__ void pack_f16x2_kernel(const float* __restrict__ src, int N, int K, int nchunks,
                                  const float* __restrict__ col_scale, __half* __restrict__ dst, long total) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    // i indexes (tile, chunk, row, k) of the hi plane; the lo plane follows it
    const int k = (int)(i & 63);
    const int r = (int)((i >> 6) & 127);
    const long blk = i >> 13;
    const int c = (int)(blk % nchunks);
    const long t = blk / nchunks;
    const long row = t * FX_WROWS + r, col = (long)c * FX_KC + k;
    float w = 0.f;
    if (row < N && col < K) w = col_scale ? src[row * K + col] * col_scale[col] : src[row * K + col];
    const __half hi = __float2half_rn(w);
    const __half lo = __float2half_rn((w - __half2float(hi)) * kPairLo);
    const long o = blk * (2 * FX_WROWS * FX_KC) + r * FX_KC + k;
    dst[o] = hi;
    dst[o + FX_WROWS * FX_KC] = lo;
  }
}

size_t packed_weight_elems_f16x2(int N, int K) {
  return (size_t)((N + FX_WROWS - 1) / FX_WROWS) * ((K + FX_KC - 1) / FX_KC) * 2 * FX_WROWS * FX_KC;
}

cudaError_t pack_weight_tiles_f16x2(const float* src, int N, int K, void* dst, cudaStream_t stream,
                                    const float* col_scale) {
  const long total = (long)packed_weight_elems_f16x2(N, K) / 2;
  pack_f16x2_kernel<<<148 * 8, 256, 0, stream>>>(src, N, K, (K + FX_KC - 1) / FX_KC, col_scale,
                                                 static_cast<__half*>(dst), total);
  return cudaGetLastError();
}

// 2-D fp16 row-major [rows][cols] (row stride ld elements), box [box_rows][64].
bool make_tmap_f16(TensorMap* out, const void* base, long rows, long cols, long ld, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || (ld * 2) % 16 || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)FX_KC, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(reinterpret_cast<CUtensorMap*>(out), CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base),
                  dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_tmap_packed_f16x2(TensorMap* out, const void* packed, int N, int K) {
  const long rows = (long)packed_weight_elems_f16x2(N, K) / FX_KC;
  return make_tmap_f16(out, packed, rows, FX_KC, FX_KC, 2 * FX_WROWS);
}

cudaError_t gemm_f16x2_wait_control(long long wait_cycles, int withhold_x) {
  const WaitControl c{wait_cycles, withhold_x, 0};
  return cudaMemcpyToSymbol(g_fx_wait, &c, sizeof(c));
}

cudaError_t gemm_f16x2_init() {
  cudaError_t e = cudaFuncSetAttribute(gemm_f16x2_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       FxCfg<64>::SMEM);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(gemm_f16x2_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, FxCfg<128>::SMEM);
}

// Same arguments and checks as gemm_tc(); tmXh / tmXl map the activation's
// fp16 hi and lo planes ([rows][K], box [64][64]).  M <= 64 runs 64-row CTAs,
// larger M 128-row CTAs (the weight tile is read once per 128 rows).
cudaError_t gemm_f16x2(const TensorMap& tmW, const TensorMap& tmXh, const TensorMap& tmXl, float* C, float* C_big,
                       float* C_small, int ldc, const float* bias, int M, int N, int K, int epi, float* ws,
                       size_t ws_floats, int* tickets, int max_tickets, uint32_t* status, int sms, cudaStream_t stream,
                       bool pdl, const RopeArgs* rope, const NormFold* fold, float2* lse, int lse_ld) {
  if (epi == EPI_SWIGLU && (!C_big || !C_small)) return cudaErrorInvalidValue;
  if (lse && (epi != EPI_STORE || lse_ld < (N + FX_WROWS - 1) / FX_WROWS)) return cudaErrorInvalidValue;
  if (epi == EPI_ROPE) {
    if (!rope || !bias || (rope->head_dim != 64 && rope->head_dim != 128) ||
        N != (rope->heads + 2 * rope->kv_heads) * rope->head_dim || (reinterpret_cast<uintptr_t>(bias) & 15))
      return cudaErrorInvalidValue;
  }
  if (epi != EPI_ROPE && (N % 4 || ldc % 4 || (reinterpret_cast<uintptr_t>(C) & 15))) return cudaErrorInvalidValue;
  if (fold && fold->ss_out && (epi != EPI_RESID || !C_big || !C_small || fold->parts * 128 != N)) return cudaErrorInvalidValue;
  if (fold && fold->ss_in && (epi == EPI_RESID || fold->hidden != K)) return cudaErrorInvalidValue;
  if (K % 8) return cudaErrorInvalidValue;  // TMA rows of the activations: 16-byte multiples
  const bool wide = M > 64;
  const int ntok = wide ? 128 : 64;
  const int tt = (M + ntok - 1) / ntok, wt = (N + FX_WROWS - 1) / FX_WROWS;
  const int nchunks = (K + FX_KC - 1) / FX_KC;
  int dev = 0;
  cudaGetDevice(&dev);
  // the plan counts 128-byte chunk rows: a 64-element chunk row of the pair is two
  const SplitPlan plan = tc_split_plan(tt * wt, 2 * nchunks, sms, g_tc_clusters[dev < kMaxDevices ? dev : 0],
                                       4, ws_floats, (long)ntok * FX_WROWS, max_tickets, 0.0, true);
  const int splits = plan.splits < nchunks ? plan.splits : nchunks;
  const int cs = splits % plan.cluster ? 1 : plan.cluster;
  TcParams p{C, C_big, C_small, bias, M, N, K, ldc, epi, splits, ws, tickets, status, {}, {}, SPLIT_F16};
  if (rope) p.rope = *rope;
  if (fold) p.fold = *fold;
  p.lse = lse;
  p.lse_ld = lse_ld;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tt, wt, splits);
  cfg.blockDim = dim3(wide ? FxCfg<128>::THREADS : FxCfg<64>::THREADS);
  cfg.dynamicSmemBytes = wide ? FxCfg<128>::SMEM : FxCfg<64>::SMEM;
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
  const CUtensorMap& w = *reinterpret_cast<const CUtensorMap*>(&tmW);
  const CUtensorMap& xh = *reinterpret_cast<const CUtensorMap*>(&tmXh);
  const CUtensorMap& xl = *reinterpret_cast<const CUtensorMap*>(&tmXl);
  return wide ? cudaLaunchKernelEx(&cfg, gemm_f16x2_kernel<128>, w, xh, xl, p)
              : cudaLaunchKernelEx(&cfg, gemm_f16x2_kernel<64>, w, xh, xl, p);
}

}  // namespace rtr
