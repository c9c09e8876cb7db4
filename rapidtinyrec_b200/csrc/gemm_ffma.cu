// FP32 FFMA GEMM for the Qwen2 projections: C[M,N] = A[M,K] . W[N,K]^T.
//
// A is the activation matrix (row-major, K contiguous), W a weight matrix in
// nn.Linear layout [out_features, in_features].  Tiles of 64 x 128 x 16 are
// staged through a 4-stage cp.async pipeline (16-byte copies, rows padded by 4
// floats so the k-contiguous tiles are read conflict-free); each of the 256
// threads owns a 4 x 8 register tile.  Split-K is deterministic: every split
// writes its partial tile to a workspace, and the last CTA to arrive on the
// tile's ticket sums the partials in split order, so a replay reproduces every
// bit.  Epilogues fuse the Qwen2 element-wise tails:
//   STORE   C = acc                                    (LM head)
//   BIAS    C = acc + bias[n]                          (q/k/v projection)
//   RESID   C = C + acc   (residual + projection)      (o_proj, down_proj)
//   SWIGLU  act[m,i] = silu(gate) * up  on gate/up columns packed in blocks of
//           16 (packed cols 32q..32q+15 = gate 16q.., 32q+16.. = up 16q..)
// The epilogues follow Qwen2DecoderLayer.forward / Qwen2MLP.forward
// (transformers modeling_qwen2.py:46-48, 290-309).
#include "common.cuh"
#include "engine.h"

namespace rtr {

constexpr int BM = 64, BN = 128, BK = 16, STAGES = 4, THREADS = 256;
constexpr int LDS = BK + 4;  // padded smem row (floats)
constexpr int TILE_SMEM = (BM + BN) * LDS;

RTR_DEVICE float silu(float g) { return g / (1.0f + expf(-g)); }

struct GemmParams {
  const float* A; const float* W; float* C;
  const float* bias;
  int M, N, K, lda, ldc;
  int splits;
  float* ws;          // [splits][Mpad][N] partials
  int* tickets;       // one per output tile
  int epi;
};

__global__ void __launch_bounds__(THREADS, 2) gemm_f32_kernel(GemmParams p) {
  extern __shared__ __align__(16) float smem[];
  const int tid = threadIdx.x;
  const int tm = tid >> 4, tn = tid & 15;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int nk = p.K / BK;
  const int kt0 = (int)((long)blockIdx.z * nk / p.splits);
  const int kt1 = (int)((long)(blockIdx.z + 1) * nk / p.splits);
  const int ktiles = kt1 - kt0;

  // loader mapping: A tile = 64 rows x 4 float4, W tile = 128 rows x 4 float4
  const int a_row = tid >> 2, a_col = (tid & 3) * 4;
  const bool a_ok = (m0 + a_row) < p.M;
  const float* a_src = p.A + (long)(a_ok ? m0 + a_row : 0) * p.lda + a_col;
  const int w_row0 = tid >> 2, w_col = (tid & 3) * 4;
  const bool w_ok0 = (n0 + w_row0) < p.N, w_ok1 = (n0 + w_row0 + 64) < p.N;
  const float* w_src0 = p.W + (long)(w_ok0 ? n0 + w_row0 : 0) * p.K + w_col;
  const float* w_src1 = p.W + (long)(w_ok1 ? n0 + w_row0 + 64 : 0) * p.K + w_col;

  pdl_wait();

  auto load_stage = [&](int stage, int kt) {
    float* As = smem + stage * TILE_SMEM;
    float* Ws = As + BM * LDS;
    const long koff = (long)kt * BK;
    cp_async16(As + a_row * LDS + a_col, a_src + koff, a_ok);
    cp_async16(Ws + w_row0 * LDS + w_col, w_src0 + koff, w_ok0);
    cp_async16(Ws + (w_row0 + 64) * LDS + w_col, w_src1 + koff, w_ok1);
  };

  float acc[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

#pragma unroll
  for (int s = 0; s < STAGES - 1; ++s) {
    if (s < ktiles) load_stage(s, kt0 + s);
    cp_async_commit();
  }

  for (int it = 0; it < ktiles; ++it) {
    cp_async_wait<STAGES - 2>();
    __syncthreads();
    const int nxt = it + STAGES - 1;
    if (nxt < ktiles) load_stage(nxt % STAGES, kt0 + nxt);
    cp_async_commit();

    const float* As = smem + (it % STAGES) * TILE_SMEM;
    const float* Ws = As + BM * LDS;
#pragma unroll
    for (int kk = 0; kk < BK; kk += 4) {
      float4 a[4], b[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = *reinterpret_cast<const float4*>(As + (tm + 16 * i) * LDS + kk);
#pragma unroll
      for (int j = 0; j < 8; ++j) b[j] = *reinterpret_cast<const float4*>(Ws + (tn + 16 * j) * LDS + kk);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          acc[i][j] = fmaf(a[i].x, b[j].x, acc[i][j]);
          acc[i][j] = fmaf(a[i].y, b[j].y, acc[i][j]);
          acc[i][j] = fmaf(a[i].z, b[j].z, acc[i][j]);
          acc[i][j] = fmaf(a[i].w, b[j].w, acc[i][j]);
        }
    }
  }
  cp_async_wait<0>();
  pdl_launch_dependents();

  if (p.splits > 1) {
    const long mpad = (long)gridDim.y * BM;
    float* ws = p.ws + (long)blockIdx.z * mpad * p.N;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int m = m0 + tm + 16 * i;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int n = n0 + tn + 16 * j;
        if (n < p.N) __stcg(ws + (long)m * p.N + n, acc[i][j]);
      }
    }
    __threadfence();
    __syncthreads();
    __shared__ int last;
    if (tid == 0) {
      int* t = p.tickets + blockIdx.y * gridDim.x + blockIdx.x;
      last = (atomicAdd(t, 1) == p.splits - 1);
      if (last) *t = 0;  // re-arm for the next launch / graph replay
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
    for (int z = 0; z < p.splits; ++z) {  // split order; 32 independent loads per split
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int m = m0 + tm + 16 * i;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int n = n0 + tn + 16 * j;
          if (n < p.N) acc[i][j] += __ldcg(p.ws + ((long)z * mpad + m) * p.N + n);
        }
      }
    }
  }

  // epilogue
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + tm + 16 * i;
    if (m >= p.M) continue;
    if (p.epi == EPI_SWIGLU) {
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        const int n = n0 + tn + 16 * j;  // gate column of this pair
        if (n >= p.N) continue;
        const int inter = (n >> 5) * 16 + (n & 15);
        const float g = acc[i][j], u = acc[i][j + 1];
        p.C[(long)m * p.ldc + inter] = silu(g) * u;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int n = n0 + tn + 16 * j;
        if (n >= p.N) continue;
        float* c = p.C + (long)m * p.ldc + n;
        if (p.epi == EPI_STORE) *c = acc[i][j];
        else if (p.epi == EPI_BIAS) *c = acc[i][j] + p.bias[n];
        else *c = *c + acc[i][j];
      }
    }
  }
}

static int choose_splits(int tiles, int nk, int sms) {
  if (tiles >= sms) return 1;
  int s = (sms + tiles - 1) / tiles;
  if (s > nk) s = nk;
  if (s > 16) s = 16;
  return s < 1 ? 1 : s;
}

size_t gemm_workspace_floats(int max_m, int max_n, int sms) {
  const int mpad = (max_m + BM - 1) / BM * BM;
  (void)sms;
  return (size_t)16 * mpad * max_n;
}

int gemm_tile_count(int max_m, int max_n) {
  return ((max_m + BM - 1) / BM) * ((max_n + BN - 1) / BN);
}

cudaError_t gemm_f32(const float* A, int lda, const float* W, float* C, int ldc, const float* bias,
                     int M, int N, int K, int epi, float* ws, size_t ws_floats, int* tickets,
                     int sms, cudaStream_t stream, bool pdl) {
  if (K % BK != 0 || M <= 0 || N <= 0) return cudaErrorInvalidValue;
  const int mt = (M + BM - 1) / BM, nt = (N + BN - 1) / BN;
  int splits = choose_splits(mt * nt, K / BK, sms);
  while (splits > 1 && (size_t)splits * mt * BM * N > ws_floats) --splits;
  GemmParams p{A, W, C, bias, M, N, K, lda, ldc, splits, ws, tickets, epi};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nt, mt, splits);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = STAGES * TILE_SMEM * sizeof(float);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemm_f32_kernel, p);
}

cudaError_t gemm_init() {
  return cudaFuncSetAttribute(gemm_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              STAGES * TILE_SMEM * (int)sizeof(float));
}

}  // namespace rtr
