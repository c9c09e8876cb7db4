// BF16 projection GEMM on the 5th-generation tensor cores (the bf16 mode of
// the engine: weights, activations and KV in bf16, fp32 accumulation).
//
//   C[m, n] (+ epilogue) = sum_k X[m, k] * W[n, k]        X: bf16 activations, W: bf16 weight
//
// A CTA owns 128 weight rows (MMA M) x 64 activation rows (MMA N) for a range
// of K, walked in 64-element chunks (one 128-byte row of bf16); above 64 rows
// gemm_bf16_wide_kernel (further down) owns 128 activation rows:
//   warp 0     TMA of the packed W tiles [128 x 64] (128B swizzle)
//   warp 2     TMA of the activation tiles [64 x 64]
//              both into a 4-deep ring of stages of two chunks; a stage has one
//              full barrier (both producers arrive) and one empty barrier
//   warp 1     MMA issuer: tcgen05.mma kind::f16, A = W, B = X, both from shared
//              memory, 4 instructions (K = 16 each) per chunk; one wait and one
//              commit per stage, stage indices compile-time (the issuing
//              thread's own instruction stream is what bounds the MMA rate)
//   warps 4..7 promote the TMEM accumulator (double-buffered) into fp32
//              registers every 4 chunks, as the 3xTF32 kernel does
// Epilogues round where a bf16 torch model rounds (the reference's
// bf16-experimental mode casts the whole model, benchmark_inference.py:93-98):
// every linear output is rounded to bf16 once (bias included), the residual
// add, SiLU, the SwiGLU product and each RoPE product and sum are rounded
// again; the LM head writes fp32 copies of its bf16 logits (HF upcasts the
// logits before the log-softmax).  Split-K and the shared-memory epilogue are
// the 3xTF32 kernel's.  Every mbarrier wait is bounded.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "engine.h"
#include "tc_epilogue.cuh"
#include "tcgen05.cuh"

namespace rtr {

constexpr int BF_THREADS = 256;          // 8 warps
constexpr int BF_KC = 64;                // bf16 per 128-byte row
constexpr int BF_WROWS = 128;            // MMA M
constexpr int BF_NTOK = 64;              // activation rows per CTA (MMA N)
constexpr int BF_CPS = 2;                // chunks per stage
constexpr int BF_STAGES = 4;             // ring depth in stages
constexpr int BF_PROMOTE = 4;            // chunks per promotion (K = 256: the tensor core's fp32
                                         // accumulation drifts past 1 bf16 ulp at K = 512)
constexpr int BF_GSTAGES = BF_PROMOTE / BF_CPS;
constexpr int BF_WC_BYTES = BF_WROWS * 128;           // one chunk of W
constexpr int BF_XC_BYTES = BF_NTOK * 128;            // one chunk of X
constexpr int BF_W_BYTES = BF_CPS * BF_WC_BYTES;      // one stage
constexpr int BF_X_BYTES = BF_CPS * BF_XC_BYTES;
constexpr int BF_D_COLS = BF_NTOK;
constexpr int BF_TMEM_COLS = 2 * BF_D_COLS;   // 128: double-buffered accumulator
constexpr int BF_NBARS = 2 * BF_STAGES + 5;
constexpr int BF_RING_BYTES = BF_STAGES * (BF_W_BYTES + BF_X_BYTES);
static_assert(2 * BF_GSTAGES == BF_STAGES, "one pass over the ring = both accumulator buffers");
constexpr int BF_SMEM_BYTES = BF_RING_BYTES + 1024 + 8 * BF_NBARS + 16;
constexpr int BF_RLD = BF_WROWS + 4;          // epilogue tile row stride (floats)
static_assert(BF_NTOK * BF_RLD * 4 <= BF_RING_BYTES, "epilogue tile fits in the rings");

struct BfParams {
  void* C;                 // bf16 [M][ldc]; fp32 for EPI_STORE (logits)
  const float* bias;       // bf16 values held in fp32
  int M, N, K, ldc, epi, splits;
  float* ws;
  int* tickets;
  uint32_t* status;
  RopeArgs rope;           // EPI_ROPE: q_out / k_dst / v_dst are bf16
  float2* lse = nullptr;   // EPI_STORE (LM head): per row and 128-column tile, (max, sum exp(x - max))
  int lse_ld = 0;          // tiles per row of the partials (row stride)
};

RTR_DEVICE float rbf(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
RTR_DEVICE __nv_bfloat16* bfp(void* p) { return static_cast<__nv_bfloat16*>(p); }
RTR_DEVICE float4 rbf4(float4 v) { return make_float4(rbf(v.x), rbf(v.y), rbf(v.z), rbf(v.w)); }
RTR_DEVICE void st_bf4(__nv_bfloat16* dst, float4 v) {  // 8-byte store of 4 bf16
  __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&a);
  u.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(dst) = u;
}
RTR_DEVICE float4 ld_bf4(const __nv_bfloat16* src) {
  const uint2 u = *reinterpret_cast<const uint2*>(src);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
RTR_DEVICE float4 bf_mul4(float4 a, float4 b) { return rbf4(make_float4(a.x * b.x, a.y * b.y, a.z * b.z, a.w * b.w)); }
RTR_DEVICE float4 bf_add4(float4 a, float4 b) { return rbf4(make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w)); }

// Epilogue from a [rows][ld4 float4] shared tile of fp32 sums, every thread of
// the CTA, 4 columns at a time.
template <int THREADS>
RTR_DEVICE void bf_tile_epilogue(const BfParams& p, const float4* red4, int ld4, int tok0, int n0, int rows,
                                 int cols4) {
  if (p.epi == EPI_SWIGLU) {
    // packed rows: 32 q + [0,16) gate, 32 q + [16,32) up of intermediate 16 q + [0,16)
    for (int q = threadIdx.x; q < rows * 16; q += THREADS) {
      const int j = q >> 4, blk = (q >> 2) & 3, g4 = q & 3;
      const int c4 = blk * 8 + g4;
      if (c4 + 4 >= cols4) continue;
      const float4 g = rbf4(red4[j * ld4 + c4]), u = rbf4(red4[j * ld4 + c4 + 4]);
      const float4 sg = rbf4(make_float4(silu_f(g.x), silu_f(g.y), silu_f(g.z), silu_f(g.w)));
      const long o = (long)(tok0 + j) * p.ldc + ((n0 + blk * 32) >> 5) * 16 + g4 * 4;
      st_bf4(bfp(p.C) + o, bf_mul4(sg, u));
    }
    return;
  }
  if (p.epi == EPI_ROPE) {
    const RopeArgs& r = p.rope;
    const int D = r.head_dim, half = D >> 1;

    // QB iterations per thread at a time, their global loads in two rounds:
    // the bias columns and the row's position, then the RoPE table rows
    constexpr int QB = 2;
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int q0 = threadIdx.x; q0 < rows * 32; q0 += QB * THREADS) {
      float4 bv[QB], bp[QB], cs[QB], sn[QB];
      int pos[QB];
#pragma unroll
      for (int k = 0; k < QB; ++k) {
        const int q = q0 + k * THREADS, j = q >> 5, c4 = q & 31;
        const bool ok = q < rows * 32 && c4 < cols4;
        const int col = n0 + c4 * 4, m = tok0 + j, h = col / D, d = col % D;
        const bool rot = ok && h < r.heads + r.kv_heads;
        const int pc4 = d < half ? c4 + half / 4 : c4 - half / 4;
        bv[k] = ok ? *reinterpret_cast<const float4*>(p.bias + col) : zero;
        bp[k] = rot ? *reinterpret_cast<const float4*>(p.bias + n0 + pc4 * 4) : zero;
        // decode: position L + slot, L of the row's user in a batched step
        pos[k] = !rot ? 0 : r.slot < 0 ? m : r.L_dev[r.rows_per_user ? m / r.rows_per_user : 0] + r.slot;
      }
#pragma unroll
      for (int k = 0; k < QB; ++k) {
        const int q = q0 + k * THREADS, j = q >> 5, c4 = q & 31;
        const bool ok = q < rows * 32 && c4 < cols4;
        const int col = n0 + c4 * 4, h = col / D, d = col % D;
        cs[k] = sn[k] = zero;
        if (ok && h < r.heads + r.kv_heads) {
          if (pos[k] < 0 || pos[k] >= r.positions) {
            atomicOr(p.status, RTR_DEV_BAD_LENGTH);
            pos[k] = 0;
          }
          cs[k] = *reinterpret_cast<const float4*>(r.cos_t + (long)pos[k] * half + (d % half));
          sn[k] = *reinterpret_cast<const float4*>(r.sin_t + (long)pos[k] * half + (d % half));
        }
      }
#pragma unroll
      for (int k = 0; k < QB; ++k) {
        const int q = q0 + k * THREADS, j = q >> 5, c4 = q & 31;
        if (q >= rows * 32 || c4 >= cols4) continue;
        const int col = n0 + c4 * 4, m = tok0 + j;
        const int h = col / D, d = col % D;
        float4 v = rbf4(f4add(red4[j * ld4 + c4], bv[k]));
        if (h < r.heads + r.kv_heads) {
          const int pc4 = d < half ? c4 + half / 4 : c4 - half / 4;
          const float4 pv = rbf4(f4add(red4[j * ld4 + pc4], bp[k]));
          // q * cos + rotate_half(q) * sin, each product and the sum rounded to bf16
          v = d < half ? bf_add4(bf_mul4(v, cs[k]), bf_mul4(f4neg(pv), sn[k]))
                       : bf_add4(bf_mul4(v, cs[k]), bf_mul4(pv, sn[k]));
        }
        __nv_bfloat16* dst;
        if (h < r.heads) {
          dst = bfp(r.q_out) + ((long)m * r.heads + h) * D + d;
        } else {
          const bool is_k = h < r.heads + r.kv_heads;
          const int g = is_k ? h - r.heads : h - r.heads - r.kv_heads;
          __nv_bfloat16* cache = bfp(is_k ? r.k_dst : r.v_dst);
          dst = r.slot < 0 ? cache + ((long)g * r.prefix_cap + m) * D + d : cache + ((long)m * r.kv_heads + g) * D + d;
        }
        st_bf4(dst, v);
      }
    }
    if (r.slot < 0 && r.vtpair_hi && n0 + FTILE_COLS > (r.heads + r.kv_heads) * D) {
      // prefill: the tile's V columns also transposed ([group][dim][token],
      // the same bf16 values) for the tensor-core prefill attention; a warp
      // takes consecutive tokens of a column, so its stores are contiguous
      const float* red = reinterpret_cast<const float*>(red4);
      for (int q = threadIdx.x; q < rows * cols4 * 4; q += THREADS) {
        const int c = q / rows, j = q % rows;
        const int col = n0 + c, h = col / D, d = col % D;
        if (h < r.heads + r.kv_heads) continue;
        const int g = h - r.heads - r.kv_heads;
        bfp(r.vtpair_hi)[((long)g * D + d) * r.pair_cap + tok0 + j] =
            __float2bfloat16_rn(red[j * ld4 * 4 + c] + p.bias[col]);
      }
    }
    return;
  }
  if (p.epi == EPI_RESID) {
    // x = bf16(x + bf16(y)); QB iterations' residual loads in flight together
    constexpr int QB = 4;
    for (int q0 = threadIdx.x; q0 < rows * 32; q0 += QB * THREADS) {
      float4 x[QB];
#pragma unroll
      for (int k = 0; k < QB; ++k) {
        const int q = q0 + k * THREADS, j = q >> 5, c4 = q & 31;
        x[k] = q < rows * 32 && c4 < cols4 ? ld_bf4(bfp(p.C) + (long)(tok0 + j) * p.ldc + n0 + c4 * 4)
                                           : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int k = 0; k < QB; ++k) {
        const int q = q0 + k * THREADS, j = q >> 5, c4 = q & 31;
        if (q < rows * 32 && c4 < cols4)
          st_bf4(bfp(p.C) + (long)(tok0 + j) * p.ldc + n0 + c4 * 4, f4add(x[k], rbf4(red4[j * ld4 + c4])));
      }
    }
    return;
  }
  for (int q = threadIdx.x; q < rows * 32; q += THREADS) {
    const int j = q >> 5, c4 = q & 31;
    if (c4 >= cols4) continue;
    const int col = n0 + c4 * 4;
    const long o = (long)(tok0 + j) * p.ldc + col;
    float4 v = red4[j * ld4 + c4];
    if (p.epi == EPI_STORE) {  // logits: fp32 copies of the bf16 values
      *reinterpret_cast<float4*>(static_cast<float*>(p.C) + o) = rbf4(v);
    } else if (p.epi == EPI_BIAS) {
      st_bf4(bfp(p.C) + o, f4add(v, *reinterpret_cast<const float4*>(p.bias + col)));
    } else {  // EPI_RESID: x = bf16(x + bf16(y))
      st_bf4(bfp(p.C) + o, f4add(ld_bf4(bfp(p.C) + o), rbf4(v)));
    }
  }
  if (p.lse && p.epi == EPI_STORE) {
    // LM head: every row's (max, sum of exp(x - max)) over the tile's bf16
    // logits, for the first log-softmax (the step tail then reads the logits
    // once).  Warp w takes rows w, w + 8, ... eight at a time (lane = float4
    // column).  The hardware exponential: these partials only set the row's
    // normaliser, whose sum over the vocabulary averages their rounding.
    constexpr int NW = THREADS / 32, G = 8;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int j0 = warp; j0 < rows; j0 += NW * G) {
      float4 v[G];
      float mx[G], e[G];
#pragma unroll
      for (int r = 0; r < G; ++r) {
        const int j = j0 + r * NW;
        const bool ok = j < rows && lane < cols4;
        v[r] = ok ? rbf4(red4[j * ld4 + lane]) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        mx[r] = fmaxf(fmaxf(v[r].x, v[r].y), fmaxf(v[r].z, v[r].w));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int r = 0; r < G; ++r) mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], o));
#pragma unroll
      for (int r = 0; r < G; ++r)
        e[r] = lane < cols4 ? (__expf(v[r].x - mx[r]) + __expf(v[r].y - mx[r])) +
                                  (__expf(v[r].z - mx[r]) + __expf(v[r].w - mx[r]))
                            : 0.f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int r = 0; r < G; ++r) e[r] += __shfl_xor_sync(0xffffffffu, e[r], o);
      if (lane == 0)
#pragma unroll
        for (int r = 0; r < G; ++r) {
          const int j = j0 + r * NW;
          if (j < rows) p.lse[(long)(tok0 + j) * p.lse_ld + (n0 >> 7)] = make_float2(mx[r], e[r]);
        }
    }
  }
}

// Split-K sum (a CTA finishing a tile): rows [row0, row0 + rows) of the
// partials summed in split order into the same rows of a [64][128] shared
// tile.  Each round of loads is one L2 round trip, so the sum takes whichever
// order needs fewer rounds: every split (up to KS_MAX) of two float4 slots per
// thread at once, or every slot two splits at a time.
template <int THREADS, int NTOK>
RTR_DEVICE void bf_splitk_sum(const BfParams& p, float4* red4, int row0, int rows, int cols4, int tile, long tstride) {
  constexpr int SLOTS = (NTOK * BF_WROWS / 4 + THREADS - 1) / THREADS;
  const float4* base = reinterpret_cast<const float4*>(p.ws + (long)tile * (NTOK * BF_WROWS)) + row0 * 32;
  red4 += row0 * 32;
  const long zs = tstride >> 2;
  const int nslots = rows * (BF_WROWS / 4);
  const int active = (nslots + THREADS - 1) / THREADS;  // slots a thread holds
  if (p.splits <= KS_MAX && (active + 1) / 2 < (p.splits + 1) / 2) {
    constexpr int PS = 2;
#pragma unroll 1
    for (int u0 = 0; u0 < SLOTS && u0 * THREADS < nslots; u0 += PS) {
      float4 v[PS][KS_MAX];
#pragma unroll
      for (int u = 0; u < PS; ++u)
#pragma unroll
        for (int z = 0; z < KS_MAX; ++z) {
          const int q = threadIdx.x + (u0 + u) * THREADS;
          const bool ok = u0 + u < SLOTS && z < p.splits && q < nslots && (q & 31) < cols4;
          v[u][z] = ok ? __ldcg(base + z * zs + q) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
      for (int u = 0; u < PS; ++u) {
        const int q = threadIdx.x + (u0 + u) * THREADS;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int z = 0; z < KS_MAX; ++z)
          if (z < p.splits) acc = f4add(acc, v[u][z]);  // split order
        if (u0 + u < SLOTS && q < nslots) red4[q] = acc;
      }
    }
    __syncthreads();
    return;
  }
  float4 s[SLOTS];
#pragma unroll
  for (int u = 0; u < SLOTS; ++u) s[u] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int z = 0; z < p.splits; z += 2) {
    float4 v[2][SLOTS];
#pragma unroll
    for (int dz = 0; dz < 2; ++dz)
#pragma unroll
      for (int u = 0; u < SLOTS; ++u) {
        const int q = threadIdx.x + u * THREADS;
        const bool ok = z + dz < p.splits && q < nslots && (q & 31) < cols4;
        v[dz][u] = ok ? __ldcg(base + (z + dz) * zs + q) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
    for (int dz = 0; dz < 2; ++dz)
#pragma unroll
      for (int u = 0; u < SLOTS; ++u)
        if (z + dz < p.splits) s[u] = f4add(s[u], v[dz][u]);  // split order
  }
#pragma unroll
  for (int u = 0; u < SLOTS; ++u) {
    const int q = threadIdx.x + u * THREADS;
    if (q < nslots) red4[q] = s[u];
  }
  __syncthreads();
}

// Bound of the pipeline waits and the test switch that withholds the
// activation copies (rtr_debug_wait_control); one copy per device.
static __device__ WaitControl g_bf_wait = {kWaitCycles, 0, 0};

__global__ void __launch_bounds__(BF_THREADS, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, BfParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* wring = smem;
  uint8_t* xring = smem + BF_STAGES * BF_W_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(xring + BF_STAGES * BF_X_BYTES);
  uint64_t* s_full = bars;                  // [BF_STAGES] W and X of the stage landed (2 arrivals + bytes)
  uint64_t* s_empty = s_full + BF_STAGES;   // [BF_STAGES] the stage's MMAs are done
  uint64_t* d_full = s_empty + BF_STAGES;   // [2]
  uint64_t* d_empty = d_full + 2;           // [2]
  uint64_t* red_bar = d_empty + 2;         // split-K finish: every CTA of the cluster arrived
  volatile int* abort_flag = reinterpret_cast<volatile int*>(red_bar + 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(red_bar + 1) + 1;
  __shared__ int go;                        // this cluster finishes the tile
  __shared__ int issued[2];                 // stages issued by the W and X producers (abort path)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tok0 = blockIdx.x * BF_NTOK;
  const int n0 = blockIdx.y * BF_WROWS;
  const long long lim = g_bf_wait.wait_cycles;
  const int nchunks = (p.K + BF_KC - 1) / BF_KC;
  const int c0 = (int)((long)blockIdx.z * nchunks / p.splits);
  const int c1 = (int)((long)(blockIdx.z + 1) * nchunks / p.splits);
  const int nloc = c1 - c0;
  const int nstages = (nloc + BF_CPS - 1) / BF_CPS;
  const int ngroups = (nloc + BF_PROMOTE - 1) / BF_PROMOTE;

  if (threadIdx.x == 0) {
    for (int s = 0; s < BF_STAGES; ++s) { mbar_init(smem_addr(&s_full[s]), 2); mbar_init(smem_addr(&s_empty[s]), 1); }
    for (int b = 0; b < 2; ++b) { mbar_init(smem_addr(&d_full[b]), 1); mbar_init(smem_addr(&d_empty[b]), 4); }
    mbar_init(smem_addr(red_bar), cluster_ncta());
    go = 0;
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
  }
  if (warp == 1) tmem_alloc(smem_addr(tmem_slot), BF_TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  if (cluster_ncta() > 1) cluster_sync_all();  // peers' barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  int w_issued = 0, x_issued = 0;
  uint32_t last_bar = 0, last_par = 0;  // MMA thread: barrier and phase of its last commit
  float acc[BF_NTOK];  // live only in the promoter warps

  if (warp == 0) {
    if (lane == 0) {
      // weights do not depend on the previous kernel: no griddepcontrol.wait
      for (int q = 0; q < nstages; ++q) {
        const int s = q % BF_STAGES;
        if (!mbar_wait(smem_addr(&s_empty[s]), ((q / BF_STAGES) & 1) ^ 1, abort_flag, lim)) break;
        const int nc = nloc - q * BF_CPS < BF_CPS ? nloc - q * BF_CPS : BF_CPS;
        const uint32_t fb = smem_addr(&s_full[s]);
        mbar_expect_tx(fb, nc * BF_WC_BYTES);
        for (int c = 0; c < nc; ++c)
          tma_load_2d(smem_addr(wring + s * BF_W_BYTES + c * BF_WC_BYTES), &tmW, 0,
                      (blockIdx.y * nchunks + c0 + q * BF_CPS + c) * BF_WROWS, fb);
        w_issued = q + 1;
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(BF_WROWS, BF_NTOK);
      const uint64_t ad0 = sw128_desc(smem_addr(wring)), bd0 = sw128_desc(smem_addr(xring));
      bool ok = true;
      // one pass over the ring = two promotion groups, one per accumulator buffer
      for (int jj = 0; ok && jj * BF_STAGES < nstages; ++jj) {
#pragma unroll
        for (int b = 0; b < 2; ++b) {
          const int j = 2 * jj + b;  // promotion group
          if (j * BF_GSTAGES >= nstages) break;
          if (j >= 2 && !mbar_wait(smem_addr(&d_empty[b]), (jj - 1) & 1, abort_flag, lim)) {
            ok = false;
            break;
          }
          const uint32_t d = tmem + b * BF_D_COLS;
#pragma unroll
          for (int u = 0; u < BF_GSTAGES; ++u) {
            const int q = j * BF_GSTAGES + u, s = b * BF_GSTAGES + u;
            if (q >= nstages) break;
            if (!mbar_wait(smem_addr(&s_full[s]), jj & 1, abort_flag, lim)) {
              ok = false;
              break;
            }
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < BF_CPS; ++c) {
              if (c > 0 && q * BF_CPS + c >= nloc) break;
              const uint64_t ad = ad0 + (uint64_t)((s * BF_W_BYTES + c * BF_WC_BYTES) >> 4);
              const uint64_t bd = bd0 + (uint64_t)((s * BF_X_BYTES + c * BF_XC_BYTES) >> 4);
#pragma unroll
              for (int kk = 0; kk < BF_KC / 16; ++kk)  // 16 bf16 = 32 bytes along K
                mma_f16_ss(d, ad + 2 * kk, bd + 2 * kk, idesc, (u | c | kk) ? 1u : 0u);
            }
            mma_commit(smem_addr(&s_empty[s]));
            last_bar = smem_addr(&s_empty[s]);
            last_par = jj & 1;
          }
          if (!ok) break;
          mma_commit(smem_addr(&d_full[b]));
          last_bar = smem_addr(&d_full[b]);
          last_par = jj & 1;
        }
      }
    }
    __syncwarp();
  } else if (warp == 2) {
    pdl_wait();
    if (lane == 0 && !g_bf_wait.withhold_x) {
      for (int q = 0; q < nstages; ++q) {
        const int s = q % BF_STAGES;
        if (!mbar_wait(smem_addr(&s_empty[s]), ((q / BF_STAGES) & 1) ^ 1, abort_flag, lim)) break;
        const int nc = nloc - q * BF_CPS < BF_CPS ? nloc - q * BF_CPS : BF_CPS;
        const uint32_t fb = smem_addr(&s_full[s]);
        mbar_expect_tx(fb, nc * BF_XC_BYTES);
        for (int c = 0; c < nc; ++c)
          tma_load_2d(smem_addr(xring + s * BF_X_BYTES + c * BF_XC_BYTES), &tmX, (c0 + q * BF_CPS + c) * BF_KC, tok0, fb);
        x_issued = q + 1;
      }
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------ warps 4..7: promote accumulators
#pragma unroll
    for (int j = 0; j < BF_NTOK; ++j) acc[j] = 0.f;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    for (int g = 0; g < ngroups; ++g) {
      const int b = g & 1;
      if (!mbar_wait(smem_addr(&d_full[b]), (g >> 1) & 1, abort_flag, lim)) break;
      tc_fence_after();
      const uint32_t d = tmem + lane_base + b * BF_D_COLS;
#pragma unroll
      for (int cb = 0; cb < BF_NTOK; cb += 32) {
        uint32_t r[32];
        tmem_ld32(d + cb, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[cb + j] += __uint_as_float(r[j]);
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
      ring_stand_in(s_full, BF_STAGES, xi, wi);
      ring_stand_in(s_full, BF_STAGES, wi, xi);
      drain_ring(s_full, BF_STAGES, wi > xi ? wi : xi);
    }
    if (warp == 1 && lane == 0 && last_bar) mbar_drain(last_bar, last_par);  // all MMAs issued
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, BF_TMEM_COLS);
  }
  pdl_wait();  // the split-K workspace and the epilogue touch memory of earlier kernels
  if (aborted) {
    if (p.splits > 1) {
      int r0, r1;
      splitk_claim(p, smem_addr(red_bar), &go, 0, blockIdx.y * gridDim.x + blockIdx.x, r0, r1, true);
    }
    return;
  }

  const bool have = warp >= 4;
  const int quarter = warp & 3;
  const int n = n0 + quarter * 32 + lane;  // weight row of this thread
  const int rows = p.M - tok0 < BF_NTOK ? p.M - tok0 : BF_NTOK;
  const int cols4 = (p.N - n0 < BF_WROWS ? p.N - n0 : BF_WROWS) >> 2;
  float4* red4 = reinterpret_cast<float4*>(smem);  // the rings are free now
  if (p.splits > 1) {
    const int tile = blockIdx.y * gridDim.x + blockIdx.x;
    const long tstride = (long)gridDim.x * gridDim.y * (BF_NTOK * BF_WROWS);
    if (have && n < p.N) {
      float* w = p.ws + blockIdx.z * tstride + (long)tile * (BF_NTOK * BF_WROWS) + quarter * 32 + lane;
#pragma unroll
      for (int j = 0; j < BF_NTOK; ++j)
        if (j < rows) __stcg(w + j * BF_WROWS, acc[j]);
    }
    __threadfence();
    __syncthreads();
    int r0 = 0, r1 = 0;
    if (!splitk_claim(p, smem_addr(red_bar), &go, rows, tile, r0, r1)) return;
    bf_splitk_sum<BF_THREADS, BF_NTOK>(p, red4, r0, r1 - r0, cols4, tile, tstride);
    bf_tile_epilogue<BF_THREADS>(p, red4 + r0 * 32, BF_WROWS / 4, tok0 + r0, n0, r1 - r0, cols4);
    return;
  }
  if (have && n < p.N) {
    float* red = reinterpret_cast<float*>(smem) + quarter * 32 + lane;
#pragma unroll
    for (int j = 0; j < BF_NTOK; ++j)
      if (j < rows) red[j * BF_RLD] = acc[j];
  }
  __syncthreads();
  bf_tile_epilogue<BF_THREADS>(p, red4, BF_RLD / 4, tok0, n0, rows, cols4);
}

// ------------------------------------------------------- 128-row variant
// More than 64 activation rows (the prefill, batched decode): a CTA owns 128
// weight rows x 128 activation rows, so a weight tile is read once per 128
// rows and each MMA is N = 128.  Stages of one chunk (16 KB of W + 16 KB of
// X, 6 deep), runtime stage indices; warps 4..11 promote (lane quarter x
// 64-row half).  The same promotion groups (4 chunks) and split-K plan as
// the 64-row kernel for the same tiles.
constexpr int BW_NTOK = 128;
constexpr int BW_PROMOTERS = 8;
constexpr int BW_THREADS = 128 + 32 * BW_PROMOTERS;   // 12 warps
constexpr int BW_STAGES = 6;
constexpr int BW_XC_BYTES = BW_NTOK * 128;
constexpr int BW_D_COLS = BW_NTOK;
constexpr int BW_TMEM_COLS = 2 * BW_D_COLS;           // 256: double-buffered accumulator
constexpr int BW_NBARS = 2 * BW_STAGES + 5;
constexpr int BW_RING_BYTES = BW_STAGES * (BF_WC_BYTES + BW_XC_BYTES);
constexpr int BW_SMEM_BYTES = BW_RING_BYTES + 1024 + 8 * BW_NBARS + 16;
static_assert(BW_NTOK * BF_RLD * 4 <= BW_RING_BYTES, "epilogue tile fits in the rings");

__global__ void __launch_bounds__(BW_THREADS, 1)
    gemm_bf16_wide_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                          BfParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* wring = smem;
  uint8_t* xring = smem + BW_STAGES * BF_WC_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(xring + BW_STAGES * BW_XC_BYTES);
  uint64_t* s_full = bars;                  // [BW_STAGES] W and X of the stage landed (2 arrivals + bytes)
  uint64_t* s_empty = s_full + BW_STAGES;   // [BW_STAGES] the stage's MMAs are done
  uint64_t* d_full = s_empty + BW_STAGES;   // [2]
  uint64_t* d_empty = d_full + 2;           // [2]
  uint64_t* red_bar = d_empty + 2;          // split-K finish: every CTA of the cluster arrived
  volatile int* abort_flag = reinterpret_cast<volatile int*>(red_bar + 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(red_bar + 1) + 1;
  __shared__ int go;                        // this cluster finishes the tile
  __shared__ int issued[2];                 // chunks issued by the W and X producers (abort path)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tok0 = blockIdx.x * BW_NTOK;
  const int n0 = blockIdx.y * BF_WROWS;
  const long long lim = g_bf_wait.wait_cycles;
  const int nchunks = (p.K + BF_KC - 1) / BF_KC;
  const int c0 = (int)((long)blockIdx.z * nchunks / p.splits);
  const int c1 = (int)((long)(blockIdx.z + 1) * nchunks / p.splits);
  const int nloc = c1 - c0;
  const int ngroups = (nloc + BF_PROMOTE - 1) / BF_PROMOTE;

  if (threadIdx.x == 0) {
    for (int s = 0; s < BW_STAGES; ++s) { mbar_init(smem_addr(&s_full[s]), 2); mbar_init(smem_addr(&s_empty[s]), 1); }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_addr(&d_full[b]), 1);
      mbar_init(smem_addr(&d_empty[b]), BW_PROMOTERS);
    }
    mbar_init(smem_addr(red_bar), cluster_ncta());
    go = 0;
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
  }
  if (warp == 1) tmem_alloc(smem_addr(tmem_slot), BW_TMEM_COLS);
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
      // weights do not depend on the previous kernel: no griddepcontrol.wait
      for (int q = 0; q < nloc; ++q) {
        const int s = q % BW_STAGES;
        if (!mbar_wait(smem_addr(&s_empty[s]), ((q / BW_STAGES) & 1) ^ 1, abort_flag, lim)) break;
        const uint32_t fb = smem_addr(&s_full[s]);
        mbar_expect_tx(fb, BF_WC_BYTES);
        tma_load_2d(smem_addr(wring + s * BF_WC_BYTES), &tmW, 0, (blockIdx.y * nchunks + c0 + q) * BF_WROWS, fb);
        w_issued = q + 1;
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(BF_WROWS, BW_NTOK);
      const uint64_t ad0 = sw128_desc(smem_addr(wring)), bd0 = sw128_desc(smem_addr(xring));
      bool ok = true;
      for (int j = 0; ok && j < ngroups; ++j) {  // one promotion group
        const int b = j & 1;
        if (j >= 2 && !mbar_wait(smem_addr(&d_empty[b]), ((j >> 1) - 1) & 1, abort_flag, lim)) break;
        const uint32_t d = tmem + b * BW_D_COLS;
#pragma unroll
        for (int u = 0; u < BF_PROMOTE; ++u) {
          const int q = j * BF_PROMOTE + u;
          if (q >= nloc) break;
          const int s = q % BW_STAGES;
          if (!mbar_wait(smem_addr(&s_full[s]), (q / BW_STAGES) & 1, abort_flag, lim)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = ad0 + (uint64_t)((s * BF_WC_BYTES) >> 4);
          const uint64_t bd = bd0 + (uint64_t)((s * BW_XC_BYTES) >> 4);
#pragma unroll
          for (int kk = 0; kk < BF_KC / 16; ++kk)  // 16 bf16 = 32 bytes along K
            mma_f16_ss(d, ad + 2 * kk, bd + 2 * kk, idesc, (u | kk) ? 1u : 0u);
          mma_commit(smem_addr(&s_empty[s]));
          last_bar = smem_addr(&s_empty[s]);
          last_par = (q / BW_STAGES) & 1;
        }
        if (!ok) break;
        mma_commit(smem_addr(&d_full[b]));
        last_bar = smem_addr(&d_full[b]);
        last_par = (j >> 1) & 1;
      }
    }
    __syncwarp();
  } else if (warp == 2) {
    pdl_wait();
    if (lane == 0 && !g_bf_wait.withhold_x) {
      for (int q = 0; q < nloc; ++q) {
        const int s = q % BW_STAGES;
        if (!mbar_wait(smem_addr(&s_empty[s]), ((q / BW_STAGES) & 1) ^ 1, abort_flag, lim)) break;
        const uint32_t fb = smem_addr(&s_full[s]);
        uint8_t* st = xring + s * BW_XC_BYTES;
        mbar_expect_tx(fb, BW_XC_BYTES);
        const int kx = (c0 + q) * BF_KC;
#pragma unroll
        for (int h = 0; h < BW_NTOK / 64; ++h)  // 64-row boxes
          tma_load_2d(smem_addr(st + h * 64 * 128), &tmX, kx, tok0 + h * 64, fb);
        x_issued = q + 1;
      }
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------- warps 4..11: promote (lane quarter = warp % 4, 64-row half)
    const int half = (warp - 4) >> 2;
#pragma unroll
    for (int j = 0; j < 64; ++j) acc[j] = 0.f;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    for (int g = 0; g < ngroups; ++g) {
      const int b = g & 1;
      if (!mbar_wait(smem_addr(&d_full[b]), (g >> 1) & 1, abort_flag, lim)) break;
      tc_fence_after();
      const uint32_t d = tmem + lane_base + b * BW_D_COLS + half * 64;
#pragma unroll
      for (int cb = 0; cb < 64; cb += 32) {
        uint32_t r[32];
        tmem_ld32(d + cb, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[cb + j] += __uint_as_float(r[j]);
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
      ring_stand_in(s_full, BW_STAGES, xi, wi);
      ring_stand_in(s_full, BW_STAGES, wi, xi);
      drain_ring(s_full, BW_STAGES, wi > xi ? wi : xi);
    }
    if (warp == 1 && lane == 0 && last_bar) mbar_drain(last_bar, last_par);  // all MMAs issued
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, BW_TMEM_COLS);
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
  const int rows = p.M - tok0 < BW_NTOK ? p.M - tok0 : BW_NTOK;
  const int cols4 = (p.N - n0 < BF_WROWS ? p.N - n0 : BF_WROWS) >> 2;
  float4* red4 = reinterpret_cast<float4*>(smem);  // the rings are free now
  if (p.splits > 1) {
    // partial tiles are tile-contiguous: ws[(split * tiles + tile)][row][128]
    const long tstride = (long)gridDim.x * gridDim.y * (BW_NTOK * BF_WROWS);
    if (have && n < p.N) {
      float* w = p.ws + blockIdx.z * tstride + (long)tile * (BW_NTOK * BF_WROWS) + (half * 64) * BF_WROWS +
                 quarter * 32 + lane;
#pragma unroll
      for (int j = 0; j < 64; ++j)
        if (half * 64 + j < rows) __stcg(w + j * BF_WROWS, acc[j]);
    }
    __threadfence();
    __syncthreads();
    int r0 = 0, r1 = 0;
    if (!splitk_claim(p, smem_addr(red_bar), &go, rows, tile, r0, r1)) return;
    bf_splitk_sum<BW_THREADS, BW_NTOK>(p, red4, r0, r1 - r0, cols4, tile, tstride);
    bf_tile_epilogue<BW_THREADS>(p, red4 + r0 * 32, BF_WROWS / 4, tok0 + r0, n0, r1 - r0, cols4);
    return;
  }
  if (have && n < p.N) {
    float* red = reinterpret_cast<float*>(smem) + (half * 64) * BF_RLD + quarter * 32 + lane;
#pragma unroll
    for (int j = 0; j < 64; ++j)
      if (half * 64 + j < rows) red[j * BF_RLD] = acc[j];
  }
  __syncthreads();
  bf_tile_epilogue<BW_THREADS>(p, red4, BF_RLD / 4, tok0, n0, rows, cols4);
}

// ---------------------------------------------------------------- host side
// 2-D bf16 row-major [rows][cols] (row stride ld elements), box [box_rows][64].
bool make_tmap_bf16(TensorMap* out, const void* base, long rows, long cols, long ld, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || (ld * 2) % 16 || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)BF_KC, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(reinterpret_cast<CUtensorMap*>(out), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base),
                  dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// W [N, K] (fp32 source, rounded to bf16) becomes blocks
// [N/128 tiles][K/64 chunks][128 rows][64 bf16] (zero padded): every TMA load
// of a (tile, chunk) reads 16 KB of contiguous memory.
__global__ void pack_bf16_kernel(const float* __restrict__ src, int N, int K, int nchunks,
                                 __nv_bfloat16* __restrict__ dst, long total) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int k = (int)(i & 63);
    const int r = (int)((i >> 6) & 127);
    const long blk = i >> 13;
    const int c = (int)(blk % nchunks);
    const long t = blk / nchunks;
    const long row = t * BF_WROWS + r, col = (long)c * BF_KC + k;
    dst[i] = __float2bfloat16_rn((row < N && col < K) ? src[row * K + col] : 0.f);
  }
}

size_t packed_weight_elems_bf16(int N, int K) {
  return (size_t)((N + BF_WROWS - 1) / BF_WROWS) * ((K + BF_KC - 1) / BF_KC) * BF_WROWS * BF_KC;
}

cudaError_t pack_weight_tiles_bf16(const float* src, int N, int K, void* dst, cudaStream_t stream) {
  const long total = (long)packed_weight_elems_bf16(N, K);
  pack_bf16_kernel<<<148 * 8, 256, 0, stream>>>(src, N, K, (K + BF_KC - 1) / BF_KC,
                                                static_cast<__nv_bfloat16*>(dst), total);
  return cudaGetLastError();
}

bool make_tmap_packed_bf16(TensorMap* out, const void* packed, int N, int K) {
  const long rows = (long)packed_weight_elems_bf16(N, K) / BF_KC;
  return make_tmap_bf16(out, packed, rows, BF_KC, BF_KC, BF_WROWS);
}

static int g_bf_clusters[kMaxDevices][TC_MAX_CLUSTER + 1];

cudaError_t gemm_bf16_wait_control(long long wait_cycles, int withhold_x) {
  const WaitControl c{wait_cycles, withhold_x, 0};
  return cudaMemcpyToSymbol(g_bf_wait, &c, sizeof(c));
}

cudaError_t gemm_bf16_init() {
  cudaError_t e = cudaFuncSetAttribute(gemm_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, BF_SMEM_BYTES);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(gemm_bf16_wide_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, BW_SMEM_BYTES);
  if (e != cudaSuccess) return e;
  int dev = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if (dev >= kMaxDevices) return cudaErrorInvalidDevice;
  return query_cluster_waves(reinterpret_cast<const void*>(gemm_bf16_kernel), BF_THREADS, BF_SMEM_BYTES,
                             g_bf_clusters[dev], TC_MAX_CLUSTER);
}

cudaError_t gemm_bf16(const TensorMap& tmW, const TensorMap& tmX, void* C, int ldc, const float* bias, int M, int N,
                      int K, int epi, float* ws, size_t ws_floats, int* tickets, int max_tickets, uint32_t* status,
                      int sms, cudaStream_t stream, bool pdl, const RopeArgs* rope, float2* lse, int lse_ld,
                      bool allow_wide) {
  if (lse && (epi != EPI_STORE || lse_ld < (N + BF_WROWS - 1) / BF_WROWS)) return cudaErrorInvalidValue;
  if (epi == EPI_ROPE) {
    if (!rope || !bias || (rope->head_dim != 64 && rope->head_dim != 128) ||
        N != (rope->heads + 2 * rope->kv_heads) * rope->head_dim || (reinterpret_cast<uintptr_t>(bias) & 15))
      return cudaErrorInvalidValue;
  } else if (N % 4 || ldc % 4 || (reinterpret_cast<uintptr_t>(C) & 15)) {
    return cudaErrorInvalidValue;
  }
  if (epi == EPI_BIAS && (!bias || (reinterpret_cast<uintptr_t>(bias) & 15))) return cudaErrorInvalidValue;
  if (K % 8) return cudaErrorInvalidValue;  // TMA rows of the activations: 16-byte multiples
  // more than 64 rows: 128-row CTAs (the same split plan and promotion order
  // as 64-row CTAs for the same tiles)
  const bool wide = allow_wide && M > BF_NTOK;
  const int ntok = wide ? BW_NTOK : BF_NTOK;
  const int tt = (M + ntok - 1) / ntok, wt = (N + BF_WROWS - 1) / BF_WROWS;
  const int nchunks = (K + BF_KC - 1) / BF_KC;
  // a 64-element bf16 chunk row is 128 bytes, as a 32-element tf32 one: the same plan
  int dev = 0;
  cudaGetDevice(&dev);
  // the fp16-pair kernel's rule: no cost for clusters beyond two, sizes 2 and 4 only
  const SplitPlan plan = tc_split_plan(tt * wt, nchunks, sms, g_bf_clusters[dev < kMaxDevices ? dev : 0], 4,
                                       ws_floats, (long)ntok * BF_WROWS, max_tickets, 0.0, true);
  const int splits = plan.splits, cs = plan.cluster;
  BfParams p{C, bias, M, N, K, ldc, epi, splits, ws, tickets, status, {}};
  if (rope) p.rope = *rope;
  p.lse = lse;
  p.lse_ld = lse_ld;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tt, wt, splits);
  cfg.blockDim = dim3(wide ? BW_THREADS : BF_THREADS);
  cfg.dynamicSmemBytes = wide ? BW_SMEM_BYTES : BF_SMEM_BYTES;
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
  const CUtensorMap& x = *reinterpret_cast<const CUtensorMap*>(&tmX);
  return wide ? cudaLaunchKernelEx(&cfg, gemm_bf16_wide_kernel, w, x, p) : cudaLaunchKernelEx(&cfg, gemm_bf16_kernel, w, x, p);
}

}  // namespace rtr
