// FP32 projection GEMM on the 5th-generation tensor cores: error-compensated
// 3xTF32 with tcgen05.mma, TMA-staged operands, A operand and accumulators in
// tensor memory.
//
//   C[m, n] (+ epilogue) = sum_k X[m, k] * W[n, k]        X: activations, W: nn.Linear weight
//
// A CTA owns 128 weight rows (the MMA M side) x 64 activation rows (the MMA
// N side) for a range of K, walked in 32-wide chunks (one 128-byte row):
//   warp 0     TMA of the W tile [128 x 32] into a 6-deep shared ring (128B swizzle)
//   warp 10    TMA of the activation tiles (its own warp, so a wait on the
//              MMA-paced activation ring never stalls the weight stream): the
//              big and small halves of X, which the producing kernels already
//              split (X_b = tf32(X), X_s = X - X_b), stacked per chunk into one
//              [128 x 32] operand [X_b ; X_s]
//   warps 2..5 (one TMEM lane quarter each, thread = weight row) read their row
//              of W, split it in registers (W_b = tf32(W), W_s = W - W_b), store
//              both into tensor memory and free the W stage at once
//   warp 1     MMA (A from TMEM, B from shared memory):
//                D[:, 0:128] += W_b . [X_b ; X_s]     D[:, 0:64] += W_s . X_b
//              so D[:, 0:64] + D[:, 64:128] = W.X up to W_s.X_s (~2^-22 relative)
//   warps 6..9 promote: the tensor core's fp32 accumulation drifts over long K,
//              so every 4 chunks the accumulator (double-buffered in TMEM) is
//              added into IEEE fp32 registers; they also run the epilogue.
// The A operand and the activation tiles move in stages of two chunks: one
// MMA thread issues ~60 cycles of tensor work per instruction, and its own
// waits and commits cost as much again unless they are amortised over a
// stage (16 MMAs per wait pair and commit).
// Every role has its own ring, so loading, splitting, MMA and promotion of
// different chunks overlap.  Small GEMMs split K over CTAs, launched as
// clusters of consecutive splits; the cluster holding the last partial to
// arrive sums the partial tiles in split order (deterministic), each CTA a
// slice of the rows.
// Every mbarrier wait is bounded (~1 s): on expiry the CTA records
// RTR_DEV_TIMEOUT, stops issuing work, drains what it issued and frees TMEM.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>

#include "common.cuh"
#include "engine.h"
#include "tcgen05.cuh"
#include "tc_epilogue.cuh"

namespace rtr {

constexpr int TC_THREADS = 352;          // 11 warps
constexpr int TC_KC = 32;                // fp32 per 128-byte row: one K chunk
constexpr int TC_WROWS = 128;            // MMA M
constexpr int TC_NTOK = 64;              // activation rows per CTA
constexpr int TC_WSTAGES = 5;            // W ring depth (chunks)
constexpr int TC_CPS = 2;                // chunks per stage
constexpr int TC_STAGES = 2;             // TMEM A-operand stages
constexpr int TC_XSTAGES = 4;            // activation stages: X lands ~1 us after it is asked for
constexpr int TC_PROMOTE = 8;            // chunks accumulated in TMEM per promotion (4 stages)
constexpr int TC_W_BYTES = TC_WROWS * 128;
constexpr int TC_XC_BYTES = 2 * TC_NTOK * 128;        // [X_b ; X_s] of one chunk
constexpr int TC_X_BYTES = TC_CPS * TC_XC_BYTES;      // one stage
constexpr int TC_D_COLS = 2 * TC_NTOK;                // one accumulator buffer
constexpr int TC_AC_COLS = 2 * TC_KC;                 // W_b and W_s of one chunk
constexpr int TC_A_COLS = TC_CPS * TC_AC_COLS;        // one stage
constexpr int TC_TMEM_COLS = 512;                     // 2 accumulators + 2 A stages
constexpr int TC_NBARS = 2 * TC_WSTAGES + 2 * TC_XSTAGES + 2 * TC_STAGES + 5;
constexpr int TC_SMEM_BYTES = TC_WSTAGES * TC_W_BYTES + TC_XSTAGES * TC_X_BYTES + 1024 + 8 * TC_NBARS + 16;
static_assert(2 * TC_D_COLS + TC_STAGES * TC_A_COLS <= TC_TMEM_COLS, "tensor memory budget");
constexpr int TC_GSTAGES = TC_PROMOTE / TC_CPS;       // stages per promotion group
static_assert(TC_GSTAGES % TC_STAGES == 0 && TC_GSTAGES % TC_XSTAGES == 0, "a group starts on stage 0");

__global__ void __launch_bounds__(TC_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmXb,
                   const __grid_constant__ CUtensorMap tmXs, TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* wring = smem;
  uint8_t* xring = smem + TC_WSTAGES * TC_W_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(xring + TC_XSTAGES * TC_X_BYTES);
  uint64_t* w_full = bars;
  uint64_t* w_empty = w_full + TC_WSTAGES;
  uint64_t* x_full = w_empty + TC_WSTAGES;  // [TC_XSTAGES] activation stage landed (TMA)
  uint64_t* x_empty = x_full + TC_XSTAGES;  // [TC_XSTAGES] its MMAs are done (relayed by warp 2)
  uint64_t* a_full = x_empty + TC_XSTAGES;  // [TC_STAGES] split weights stored, activations landed
  uint64_t* s_empty = a_full + TC_STAGES;   // [TC_STAGES] MMAs of the stage done (frees A)
  uint64_t* d_full = s_empty + TC_STAGES;   // [2]
  uint64_t* d_empty = d_full + 2;           // [2]
  uint64_t* red_bar = d_empty + 2;         // split-K finish: every CTA of the cluster arrived
  volatile int* abort_flag = reinterpret_cast<volatile int*>(red_bar + 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(red_bar + 1) + 1;
  __shared__ int go;                        // this cluster finishes the tile
  __shared__ float prsc[TC_NTOK];           // persistent launch: row scales of the folded RMSNorm

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tok0 = blockIdx.x * TC_NTOK;
  const int n0 = blockIdx.y * TC_WROWS;
  const int nchunks = (p.K + TC_KC - 1) / TC_KC;
  const int c0 = (int)((long)blockIdx.z * nchunks / p.splits);
  const int c1 = (int)((long)(blockIdx.z + 1) * nchunks / p.splits);
  // Persistent launch (fewer CTAs than weight tiles; one split, whole
  // promotion groups per tile): this CTA runs weight tiles blockIdx.y,
  // blockIdx.y + gridDim.y, ... as one chunk stream, and the promoters store
  // each finished tile while the next one streams.
  const int wtiles = (p.N + TC_WROWS - 1) / TC_WROWS;
  const bool persist = (int)gridDim.y < wtiles;
  const int ntl = persist ? (wtiles - (int)blockIdx.y + (int)gridDim.y - 1) / (int)gridDim.y : 1;
  const int nloc_t = c1 - c0;  // chunks of one tile
  const int nloc = nloc_t * ntl;
  const int nstages = (nloc + TC_CPS - 1) / TC_CPS;
  const int ngroups = (nloc + TC_PROMOTE - 1) / TC_PROMOTE;

  if (threadIdx.x == 0) {
    for (int s = 0; s < TC_WSTAGES; ++s) { mbar_init(smem_addr(&w_full[s]), 1); mbar_init(smem_addr(&w_empty[s]), 4); }
    for (int s = 0; s < TC_XSTAGES; ++s) { mbar_init(smem_addr(&x_full[s]), 1); mbar_init(smem_addr(&x_empty[s]), 1); }
    for (int s = 0; s < TC_STAGES; ++s) { mbar_init(smem_addr(&a_full[s]), 4); mbar_init(smem_addr(&s_empty[s]), 1); }
    for (int b = 0; b < 2; ++b) { mbar_init(smem_addr(&d_full[b]), 1); mbar_init(smem_addr(&d_empty[b]), 4); }
    mbar_init(smem_addr(red_bar), cluster_ncta());
    go = 0;
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmXb);
    tma_prefetch_desc(&tmXs);
  }
  if (warp == 1) tmem_alloc(smem_addr(tmem_slot), TC_TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  if (cluster_ncta() > 1) cluster_sync_all();  // peers' barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_a = tmem + 2 * TC_D_COLS;  // A stages after the two accumulators

  int w_issued = 0, x_issued = 0;
  uint32_t last_bar = 0, last_par = 0;  // MMA thread: barrier and phase of its last commit
  float acc[TC_NTOK];  // live only in the promoter warps (set there)

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------- W producer (TMA)
      // weights do not depend on the previous kernel: no griddepcontrol.wait
      for (int i = 0; i < nloc; ++i) {
        const int s = i % TC_WSTAGES;
        if (!mbar_wait(smem_addr(&w_empty[s]), ((i / TC_WSTAGES) & 1) ^ 1, abort_flag)) break;
        const uint32_t fb = smem_addr(&w_full[s]);
        mbar_expect_tx(fb, TC_W_BYTES);
        // packed weights: the [128 x 32] block of (tile, chunk) is 16 KB contiguous
        const int y = (int)blockIdx.y + (i / nloc_t) * (int)gridDim.y;
        tma_load_2d(smem_addr(wring + s * TC_W_BYTES), &tmW, 0, (y * nchunks + c0 + i % nloc_t) * TC_WROWS, fb);
        w_issued = i + 1;
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    // The issuing thread's own instruction stream bounds the MMA rate, so the
    // loop is unrolled over the stages (stage indices, descriptors and the
    // accumulate flags are compile-time) and a stage of two chunks costs one
    // wait pair and one commit.
    if (lane == 0) {
      constexpr uint32_t id_cat = idesc_tf32(TC_WROWS, 2 * TC_NTOK);
      constexpr uint32_t id_x = idesc_tf32(TC_WROWS, TC_NTOK);
      const uint64_t bx0 = sw128_desc(smem_addr(xring));
      bool ok = true;
      for (int j = 0; ok && j * TC_GSTAGES < nstages; ++j) {  // one promotion group
        const int b = j & 1;
        if (j >= 2 && !mbar_wait(smem_addr(&d_empty[b]), ((j >> 1) - 1) & 1, abort_flag)) break;
        const uint32_t d = tmem + b * TC_D_COLS;
#pragma unroll
        for (int u = 0; u < TC_GSTAGES; ++u) {
          const int q = j * TC_GSTAGES + u, s = u % TC_STAGES;
          if (q >= nstages) break;
          // the converters fold the activation stage's arrival into a_full
          if (!mbar_wait(smem_addr(&a_full[s]), (u / TC_STAGES) & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < TC_CPS; ++c) {
            if (c > 0 && q * TC_CPS + c >= nloc) break;
            const uint32_t ab = tmem_a + s * TC_A_COLS + c * TC_AC_COLS;
            const uint64_t bx = bx0 + (uint64_t)(((u % TC_XSTAGES) * TC_X_BYTES + c * TC_XC_BYTES) >> 4);
#pragma unroll
            for (int kk = 0; kk < TC_KC / 8; ++kk) {  // 8 tf32 = 32 bytes along K
              mma_tf32_ts(d, ab + kk * 8, bx + 2 * kk, id_cat, (u | c | kk) ? 1u : 0u);
              mma_tf32_ts(d, ab + TC_KC + kk * 8, bx + 2 * kk, id_x, 1u);
            }
          }
          mma_commit(smem_addr(&s_empty[s]));
          last_bar = smem_addr(&s_empty[s]);
          last_par = (u / TC_STAGES) & 1;
        }
        if (!ok) break;
        mma_commit(smem_addr(&d_full[b]));
        last_bar = smem_addr(&d_full[b]);
        last_par = (j >> 1) & 1;
      }
    }
    __syncwarp();
  } else if (warp == 10) {
    // --------------------------------------- activation producer (TMA)
    pdl_wait();
    if (lane == 0) {
      for (int q = 0; q < nstages; ++q) {
        const int s = q % TC_XSTAGES;
        if (!mbar_wait(smem_addr(&x_empty[s]), ((q / TC_XSTAGES) & 1) ^ 1, abort_flag)) break;
        const int nc = nloc - q * TC_CPS < TC_CPS ? nloc - q * TC_CPS : TC_CPS;
        const uint32_t fb = smem_addr(&x_full[s]);
        uint8_t* st = xring + s * TC_X_BYTES;
        mbar_expect_tx(fb, nc * TC_XC_BYTES);
        for (int c = 0; c < nc; ++c) {
          const int kx = (c0 + (q * TC_CPS + c) % nloc_t) * TC_KC;
          tma_load_2d(smem_addr(st + c * TC_XC_BYTES), &tmXb, kx, tok0, fb);
          tma_load_2d(smem_addr(st + c * TC_XC_BYTES + TC_XC_BYTES / 2), &tmXs, kx, tok0, fb);
        }
        x_issued = q + 1;
      }
    }
    __syncwarp();
  } else if (warp <= 5) {
    // ------------------------------- warps 2..5: split W rows into TMEM
    // A stage's two chunks are read from shared memory together (16
    // independent loads in flight: the reads queue behind the TMA writes and
    // the MMAs' operand reads), split, and stored once the MMAs of the
    // stage's previous use are done.
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;  // TMEM lane = weight row of the tile
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    for (int q = 0; q < nstages; ++q) {
      const int s = q % TC_STAGES;
      const int nc = nloc - q * TC_CPS < TC_CPS ? nloc - q * TC_CPS : TC_CPS;
      uint32_t v[TC_CPS][TC_KC];
      bool ok = true;
#pragma unroll
      for (int c = 0; c < TC_CPS; ++c) {
        if (c < nc) {
          const int i = q * TC_CPS + c, ws = i % TC_WSTAGES;
          if (!mbar_wait(smem_addr(&w_full[ws]), (i / TC_WSTAGES) & 1, abort_flag)) { ok = false; break; }
          const uint8_t* tile = wring + ws * TC_W_BYTES + row * 128;
#pragma unroll
          for (int k4 = 0; k4 < TC_KC / 4; ++k4) {  // undo the 128B swizzle: chunk k4 lives at k4 ^ (row % 8)
            const float4 f = *reinterpret_cast<const float4*>(tile + ((k4 ^ (row & 7)) << 4));
            v[c][4 * k4] = __float_as_uint(f.x); v[c][4 * k4 + 1] = __float_as_uint(f.y);
            v[c][4 * k4 + 2] = __float_as_uint(f.z); v[c][4 * k4 + 3] = __float_as_uint(f.w);
          }
        }
      }
      if (!ok) break;
      __syncwarp();
      if (lane == 0)  // the rows are in registers
        for (int c = 0; c < nc; ++c) mbar_arrive(smem_addr(&w_empty[(q * TC_CPS + c) % TC_WSTAGES]));
      // the stage waits until the MMAs of its last use are done
      if (!mbar_wait(smem_addr(&s_empty[s]), ((q / TC_STAGES) & 1) ^ 1, abort_flag)) break;
      // the MMAs of stage q - TC_STAGES are done: relay the release of its activation stage
      if (warp == 2 && lane == 0 && q >= TC_STAGES) mbar_arrive(smem_addr(&x_empty[(q - TC_STAGES) % TC_XSTAGES]));
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < TC_CPS; ++c) {
        if (c < nc) {
          uint32_t big[TC_KC];
#pragma unroll
          for (int k = 0; k < TC_KC; ++k) {
            const float w = __uint_as_float(v[c][k]);
            const float bv = tf32_round(w);
            big[k] = __float_as_uint(bv);
            v[c][k] = __float_as_uint(w - bv);
          }
          const uint32_t a = tmem_a + lane_base + s * TC_A_COLS + c * TC_AC_COLS;
          tmem_st32(a, big);
          tmem_st32(a + TC_KC, v[c]);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      // one converter also waits for the stage's activation tiles, so the
      // MMA thread waits on a single barrier per stage
      const bool x_ok = warp != 2 || mbar_wait(smem_addr(&x_full[q % TC_XSTAGES]), (q / TC_XSTAGES) & 1, abort_flag);
      __syncwarp();
      if (!x_ok) break;
      if (lane == 0) mbar_arrive(smem_addr(&a_full[s]));
    }
  } else {
    // ------------------------- warps 6..9: promote accumulators, epilogue
    pdl_wait();
#pragma unroll
    for (int j = 0; j < TC_NTOK; ++j) acc[j] = 0.f;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const int gpt = ngroups / ntl;  // promotion groups per tile
    const int prow = p.M - tok0 < TC_NTOK ? p.M - tok0 : TC_NTOK;
    if (persist && p.fold.ss_in) {
      // the folded RMSNorm's row scales, as tile_epilogue computes them
      const int t = threadIdx.x - 6 * 32;
      if (t < prow) {
        float ss = 0.f;
        for (int k = 0; k < p.fold.parts; ++k) ss += p.fold.ss_in[(long)k * p.fold.ld + tok0 + t];
        prsc[t] = 1.0f / sqrtf(ss / (float)p.fold.hidden + p.fold.eps);
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");  // the four promoter warps
    }
    for (int g = 0; g < ngroups; ++g) {
      const int b = g & 1;
      if (!mbar_wait(smem_addr(&d_full[b]), (g >> 1) & 1, abort_flag)) break;
      tc_fence_after();
      const uint32_t d = tmem + lane_base + b * TC_D_COLS;
      // persistent launch, last group of a tile: store the finished tile from
      // registers (EPI_STORE, the products tile_epilogue forms) and restart
      const bool tile_done = persist && (g + 1) % gpt == 0;
      const int n = ((int)blockIdx.y + (g / gpt) * (int)gridDim.y) * TC_WROWS + (warp & 3) * 32 + lane;
#pragma unroll
      for (int cb = 0; cb < TC_NTOK; cb += 32) {
        uint32_t r[32];
        float part[32];
        tmem_ld32(d + cb, r);             // W_b.X_b + W_s.X_b
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) part[j] = __uint_as_float(r[j]);
        tmem_ld32(d + TC_NTOK + cb, r);   // W_b.X_s
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[cb + j] += part[j] + __uint_as_float(r[j]);
        if (tile_done) {
          float* c = p.C + (long)(tok0 + cb) * p.ldc + n;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (cb + j < prow && n < p.N) *c = p.fold.ss_in ? acc[cb + j] * prsc[cb + j] : acc[cb + j];
            acc[cb + j] = 0.f;
            c += p.ldc;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(&d_empty[b]));
    }
  }
  pdl_launch_dependents();
  __syncthreads();  // every role is done waiting: the abort flag is final

  // drain on abort: issued copies and MMAs must land before smem/TMEM go away
  const bool aborted = *abort_flag != 0;
  if (aborted) {
    if (threadIdx.x == 0) atomicOr(p.status, RTR_DEV_TIMEOUT);
    if (warp == 0 && lane == 0) drain_ring(w_full, TC_WSTAGES, w_issued);
    if (warp == 10 && lane == 0) drain_ring(x_full, TC_XSTAGES, x_issued);
    if (warp == 1 && lane == 0 && last_bar) mbar_drain(last_bar, last_par);  // all MMAs issued
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TC_TMEM_COLS);
  }
  if (aborted && !persist && p.splits > 1) {
    pdl_wait();  // the tickets are shared with earlier kernels
    int r0, r1;
    splitk_claim(p, smem_addr(red_bar), &go, 0, blockIdx.y * gridDim.x + blockIdx.x, r0, r1, true);
  }
  if (aborted || persist) return;

  const bool have = warp >= 6 && warp <= 9;
  const int quarter = warp & 3;
  const int n = n0 + quarter * 32 + lane;  // weight row of this thread
  const int rows = p.M - tok0 < TC_NTOK ? p.M - tok0 : TC_NTOK;  // real activation rows of the tile
  const int cols4 = (p.N - n0 < TC_WROWS ? p.N - n0 : TC_WROWS) >> 2;
  float4* red4 = reinterpret_cast<float4*>(smem);  // the rings are free now
  if (p.splits > 1) {
    // Partial tiles are tile-contiguous: ws[(split * tiles + tile)][row][128].
    const int tile = blockIdx.y * gridDim.x + blockIdx.x;
    const long tstride = (long)gridDim.x * gridDim.y * (TC_NTOK * TC_WROWS);
    if (have && n < p.N) {
      float* w = p.ws + blockIdx.z * tstride + (long)tile * (TC_NTOK * TC_WROWS) + quarter * 32 + lane;
#pragma unroll
      for (int j = 0; j < TC_NTOK; ++j)
        if (j < rows) __stcg(w + j * TC_WROWS, acc[j]);
    }
    __threadfence();
    __syncthreads();
    splitk_finish<TC_THREADS, TC_NTOK>(p, red4, smem_addr(red_bar), &go, tok0, n0, rows, cols4, tile, tstride);
    return;
  }
  // Stage the finished tile in shared memory ([64][TC_WROWS + 4], padded so
  // the float4 reads of consecutive rows spread over the banks); then every
  // thread of the CTA stores float4s.
  constexpr int RLD = TC_WROWS + 4;
  if (have && n < p.N) {
    float* red = reinterpret_cast<float*>(smem) + quarter * 32 + lane;
#pragma unroll
    for (int j = 0; j < TC_NTOK; ++j)
      if (j < rows) red[j * RLD] = acc[j];
  }
  __syncthreads();
  tile_epilogue<TC_THREADS>(p, red4, RLD / 4, tok0, n0, rows, cols4);
}

// ---------------------------------------------------------------- host side
// 2-D fp32 row-major [rows][cols] (row stride ld floats), box [box_rows][32].
bool make_tmap_f32(TensorMap* out, const float* base, long rows, long cols, long ld, int box_rows) {
  static_assert(sizeof(TensorMap) == sizeof(CUtensorMap), "TensorMap size");
  EncodeTiledFn fn = encode_fn();
  if (!fn || (ld * 4) % 16 || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  cuuint32_t box[2] = {(cuuint32_t)TC_KC, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(reinterpret_cast<CUtensorMap*>(out), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base),
                  dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Weight layout for the tensor-core GEMM (optionally with an RMSNorm weight
// folded into the columns: W[n][k] * col_scale[k]): W [N, K] becomes blocks
// [N/128 tiles][K/32 chunks][128 rows][32 floats] (zero padded), so every TMA
// load of a (tile, chunk) reads 16 KB of contiguous memory.
__global__ void pack_tiles_kernel(const float* __restrict__ src, int N, int K, int nchunks, float* __restrict__ dst,
                                  long total, const float* __restrict__ col_scale) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int k = (int)(i & 31);
    const int r = (int)((i >> 5) & 127);
    const long blk = i >> 12;
    const int c = (int)(blk % nchunks);
    const long t = blk / nchunks;
    const long row = t * TC_WROWS + r, col = (long)c * TC_KC + k;
    dst[i] = (row < N && col < K) ? (col_scale ? src[row * K + col] * col_scale[col] : src[row * K + col]) : 0.f;
  }
}

size_t packed_weight_floats(int N, int K) {
  return (size_t)((N + TC_WROWS - 1) / TC_WROWS) * ((K + TC_KC - 1) / TC_KC) * TC_WROWS * TC_KC;
}

cudaError_t pack_weight_tiles(const float* src, int N, int K, float* dst, cudaStream_t stream, const float* col_scale) {
  const long total = (long)packed_weight_floats(N, K);
  pack_tiles_kernel<<<148 * 8, 256, 0, stream>>>(src, N, K, (K + TC_KC - 1) / TC_KC, dst, total, col_scale);
  return cudaGetLastError();
}

bool make_tmap_packed(TensorMap* out, const float* packed, int N, int K) {
  const long rows = (long)packed_weight_floats(N, K) / TC_KC;
  return make_tmap_f32(out, packed, rows, TC_KC, TC_KC, TC_WROWS);
}

int g_tc_clusters[kMaxDevices][TC_MAX_CLUSTER + 1];

cudaError_t gemm_tc_init() {
  cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM_BYTES);
  if (e != cudaSuccess) return e;
  int dev = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if (dev >= kMaxDevices) return cudaErrorInvalidDevice;
  return query_cluster_waves(reinterpret_cast<const void*>(gemm_tc_kernel), TC_THREADS, TC_SMEM_BYTES,
                             g_tc_clusters[dev], TC_MAX_CLUSTER);
}

cudaError_t gemm_tc(const TensorMap& tmW, const TensorMap& tmXb, const TensorMap& tmXs, float* C, float* C_big,
                    float* C_small, int ldc, const float* bias, int M, int N, int K, int epi, float* ws,
                    size_t ws_floats, int* tickets, int max_tickets, uint32_t* status, int sms, cudaStream_t stream,
                    bool pdl, const RopeArgs* rope, const NormFold* fold) {
  if (epi == EPI_SWIGLU && (!C_big || !C_small)) return cudaErrorInvalidValue;
  if (epi == EPI_ROPE) {
    // whole heads per 128-row tile, float4 pairs, q/k/v row layout
    if (!rope || !bias || (rope->head_dim != 64 && rope->head_dim != 128) ||
        N != (rope->heads + 2 * rope->kv_heads) * rope->head_dim || (reinterpret_cast<uintptr_t>(bias) & 15))
      return cudaErrorInvalidValue;
  }
  // float4 epilogue: column counts, row strides and bases in 16-byte units
  if (epi != EPI_ROPE && (N % 4 || ldc % 4 || (reinterpret_cast<uintptr_t>(C) & 15))) return cudaErrorInvalidValue;
  if (fold && fold->ss_out && (epi != EPI_RESID || !C_big || !C_small || fold->parts * 128 != N)) return cudaErrorInvalidValue;
  if (fold && fold->ss_in && (epi == EPI_RESID || fold->hidden != K)) return cudaErrorInvalidValue;
  const int tt = (M + TC_NTOK - 1) / TC_NTOK, wt = (N + TC_WROWS - 1) / TC_WROWS;
  const int nchunks = (K + TC_KC - 1) / TC_KC;
  int dev = 0;
  cudaGetDevice(&dev);
  const SplitPlan plan = tc_split_plan(tt * wt, nchunks, sms, g_tc_clusters[dev < kMaxDevices ? dev : 0], TC_MAX_CLUSTER,
                                       ws_floats, (long)TC_NTOK * TC_WROWS, max_tickets);
  const int splits = plan.splits, cs = plan.cluster;
  TcParams p{C, C_big, C_small, bias, M, N, K, ldc, epi, splits, ws, tickets, status, {}, {}};
  if (rope) p.rope = *rope;
  if (fold) p.fold = *fold;
  // many weight tiles of one row tile (the LM head): one persistent CTA per
  // SM instead of waves of one-tile CTAs (RTR_TC_PERSIST=0 turns it off)
  static const bool persist_on = [] {
    const char* e = getenv("RTR_TC_PERSIST");
    return !(e && e[0] == '0');
  }();
  const bool persist = persist_on && splits == 1 && tt == 1 && epi == EPI_STORE && wt > sms && nchunks % TC_PROMOTE == 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tt, persist ? sms : wt, splits);
  cfg.blockDim = dim3(TC_THREADS);
  cfg.dynamicSmemBytes = TC_SMEM_BYTES;
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
  return cudaLaunchKernelEx(&cfg, gemm_tc_kernel, *reinterpret_cast<const CUtensorMap*>(&tmW),
                            *reinterpret_cast<const CUtensorMap*>(&tmXb), *reinterpret_cast<const CUtensorMap*>(&tmXs),
                            p);
}

}  // namespace rtr
