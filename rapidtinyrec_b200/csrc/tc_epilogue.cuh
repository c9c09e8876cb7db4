// Parameters and epilogues shared by the 3xTF32 tensor-core GEMMs (the
// 64-row kernel in gemm_tc.cu and the 128-row kernel in gemm_tc_wide.cu).
#pragma once

#include "common.cuh"
#include "engine.h"
#include "tcgen05.cuh"

namespace rtr {

struct TcParams {
  float* C;
  float* C_big;     // SWIGLU: also write the split halves of the activation
  float* C_small;
  const float* bias;
  int M, N, K, ldc, epi, splits;
  float* ws;
  int* tickets;
  uint32_t* status;
  RopeArgs rope;    // EPI_ROPE only
  NormFold fold;    // ss_in: scale rows by their RMS factor; ss_out: EPI_RESID partials
  int xfmt;         // split written for the next GEMM: SPLIT_TF32 or SPLIT_F16
  float2* lse = nullptr;  // EPI_STORE (LM head): per row and 128-column tile, (max, sum exp(x - max))
  int lse_ld = 0;         // tiles per row of the partials (row stride)
};


// K splits for a grid of `tiles` output tiles: fill the SMs, at least two
// 32-wide chunks per split, at most 16 splits.
inline int tc_split_count(int tiles, int nchunks, int sms) {
  if (tiles >= sms) return 1;
  int s = sms / tiles;
  if (s > nchunks / 2) s = nchunks / 2;
  if (s > 16) s = 16;
  return s < 1 ? 1 : s;
}

// Split-K clusters: at most this many CTAs (consecutive splits of one tile).
constexpr int TC_MAX_CLUSTER = 8;
constexpr int kMaxDevices = 16;

// Clusters of CTAs that one wave of a one-CTA-per-SM kernel holds, per
// cluster size (index), per device; filled by gemm_tc_init() and used by both
// tf32 kernels.
extern int g_tc_clusters[kMaxDevices][TC_MAX_CLUSTER + 1];

// For cluster sizes 2..max_cs: how many clusters of that size one wave of
// `kernel` holds (cudaOccupancyMaxActiveClusters); 0 where it is not known.
inline cudaError_t query_cluster_waves(const void* kernel, int threads, int smem, int* out, int max_cs) {
  out[0] = out[1] = 0;
  for (int cs = 2; cs <= max_cs; ++cs) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, 1, cs);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = cs;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    out[cs] = n;
  }
  return cudaSuccess;
}

// Split-K plan of the tf32 kernels: the split count and the cluster size
// that finishes each tile.  Candidates run from the SM-filling count
// (tc_split_count) down to half of it; each takes every cluster size up to the
// cap (RTR_TC_CLUSTER, default 8) that divides it and whose clusters all fit
// in one wave.  The plan with the least modelled time wins, the model fitted
// to launches timed back to back on B200 at M = 50:
//   weight stream  max(0.1 us per chunk of a split, the tiles' weight bytes
//                  at 6.5 TB/s scaled by the share of SMs the grid uses)
//   finish         3.1 ns per split per row of the slice (64 / cluster rows)
//   clusters       cluster_us per CTA beyond two: 0.5 us for the 3xTF32
//                  kernels (co-scheduling a larger cluster of 11-warp CTAs on
//                  one GPC delayed its start); the fp16-pair and bf16 kernels
//                  take 0 but only cluster sizes 2 and 4 (a sweep of splits x
//                  sizes at M = 50 put 8 x 4 first for o_proj and q/k/v and
//                  12 x 2 for down_proj; 10 x 5 and 8 x 8 were slower)
// Both kernels take the same plan for the same tiles and K (one CTA per SM
// in both, one wave table, 64 nominal rows), so their sums agree bit for bit.
struct SplitPlan {
  int splits, cluster;
};
inline SplitPlan tc_split_plan(int tiles, int nchunks, int sms, const int* waves, int max_cs, size_t ws_floats,
                               long tile_floats, int max_tickets, double cluster_us = 0.5, bool pow2 = false) {
  static const int cap = [] {
    const char* e = getenv("RTR_TC_CLUSTER");
    const int v = e ? atoi(e) : 8;
    return v < 1 ? 1 : v;
  }();
  int s0 = tc_split_count(tiles, nchunks, sms);
  while (s0 > 1 && ((size_t)s0 * tiles * tile_floats > ws_floats || tiles > max_tickets)) --s0;
  SplitPlan best{s0, 1};
  if (s0 < 2) return best;
  const double stream_us = (double)tiles * 128 * nchunks * 32 * 4 / 6.5e6;  // all SMs streaming
  double best_t = 1e30;
  for (int s = s0; s >= 2 && 2 * s >= s0; --s) {
    const double share = (double)tiles * s / sms;
    const double t_main = fmax(0.1 * ((nchunks + s - 1) / s), stream_us / (share < 1.0 ? share : 1.0));
    for (int c = 1; c <= (cap < max_cs ? cap : max_cs); ++c) {
      if (s % c != 0 || (c > 1 && (long)tiles * (s / c) > waves[c]) || (pow2 && (c & (c - 1)))) continue;
      const double t = t_main + 0.0031 * s * ((64 + c - 1) / c) + (c > 2 ? cluster_us * (c - 2) : 0.0);
      if (t < best_t - 1e-9) { best_t = t; best = SplitPlan{s, c}; }
    }
  }
  return best;
}

constexpr int FTILE_COLS = 128;  // output columns of a tensor-core GEMM tile

// Split-K sum, run by every thread of a CTA finishing a tile: rows
// [row0, row0 + rows) of the partial tiles summed in split order into the same
// rows of a [NTOK][128] shared tile.  Each round of loads is one L2 round trip,
// so the sum takes whichever order needs fewer rounds: every split (up to
// KS_MAX) of two float4 slots per thread in flight at once - a decode slice
// (13 or 25 rows, 8 or 12 splits) then takes 1-2 rounds instead of 2-6 - or
// groups of G slots four splits at a time (prefill slices: many slots, few
// splits).
constexpr int KS_MAX = 12;
template <int THREADS, int NTOK>
RTR_DEVICE void splitk_sum(const TcParams& p, float4* red4, int row0, int rows, int cols4, int tile, long tstride) {
  constexpr int SLOTS = (NTOK * 128 / 4 + THREADS - 1) / THREADS;
  constexpr int G = SLOTS < 6 ? SLOTS : 3;
  const float4* base = reinterpret_cast<const float4*>(p.ws + (long)tile * (NTOK * 128)) + row0 * 32;
  red4 += row0 * 32;
  const long zs = tstride >> 2;
  const int nslots = rows * 32;
  const int active = (nslots + THREADS - 1) / THREADS;  // slots a thread holds
  if (NTOK == 64 && p.splits <= KS_MAX && (active + 1) / 2 < (active + G - 1) / G * ((p.splits + 3) / 4)) {
    constexpr int PS = 2;  // slots in flight per thread (registers: 2 x 12 float4)
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
  // slots in groups of G keep four splits of loads in flight without running out of registers
#pragma unroll 1
  for (int u0 = 0; u0 < SLOTS && u0 * THREADS < nslots; u0 += G) {
    float4 acc[G];
#pragma unroll
    for (int u = 0; u < G; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int z = 0; z < p.splits; z += 4) {
      float4 v[4][G];
#pragma unroll
      for (int dz = 0; dz < 4; ++dz)
#pragma unroll
        for (int u = 0; u < G; ++u) {
          const int q = threadIdx.x + (u0 + u) * THREADS;
          const bool ok = u0 + u < SLOTS && z + dz < p.splits && q < nslots && (q & 31) < cols4;
          v[dz][u] = ok ? __ldcg(base + (z + dz) * zs + q) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
      for (int dz = 0; dz < 4; ++dz)
#pragma unroll
        for (int u = 0; u < G; ++u)
          if (z + dz < p.splits) acc[u] = f4add(acc[u], v[dz][u]);  // split order
    }
#pragma unroll
    for (int u = 0; u < G; ++u) {
      const int q = threadIdx.x + (u0 + u) * THREADS;
      if (u0 + u < SLOTS && q < nslots) red4[q] = acc[u];
    }
  }
  __syncthreads();
}

// Epilogue from a [rows][ld4 float4] shared tile of finished sums, run by
// every thread of the CTA with float4 loads and stores (N, ldc and the head
// dimension are multiples of 4; checked by the host).
template <int THREADS>
RTR_DEVICE void tile_epilogue(const TcParams& p, const float4* red4, int ld4, int tok0, int n0, int rows, int cols4) {
  // RMSNorm folded into this GEMM: row scale 1 / sqrt(mean(x^2) + eps) from
  // the producer's partial sums of squares, summed in chunk order
  // (a row's partials are all loaded before the first is added: one L2
  // round trip, not one per chunk)
  __shared__ float rsc[128];
  const bool scaled = p.fold.ss_in != nullptr;
  if (scaled) {
    constexpr int PB = 16;  // partials in flight per round (hidden <= 2048: one round)
    for (int j = threadIdx.x; j < rows; j += THREADS) {
      const float* src = p.fold.ss_in + tok0 + j;
      float ss = 0.f;
      for (int t0 = 0; t0 < p.fold.parts; t0 += PB) {
        float v[PB];
#pragma unroll
        for (int t = 0; t < PB; ++t) v[t] = t0 + t < p.fold.parts ? src[(long)(t0 + t) * p.fold.ld] : 0.f;
#pragma unroll
        for (int t = 0; t < PB; ++t)
          if (t0 + t < p.fold.parts) ss += v[t];  // chunk order
      }
      rsc[j] = 1.0f / sqrtf(ss / (float)p.fold.hidden + p.fold.eps);
    }
    __syncthreads();
  }
  auto row_scale = [&](float4 v, int j) {
    if (!scaled) return v;
    const float r = rsc[j];
    return make_float4(v.x * r, v.y * r, v.z * r, v.w * r);
  };
  if (p.epi == EPI_SWIGLU) {
    // packed rows: 32 q + [0,16) gate, 32 q + [16,32) up of intermediate 16 q + [0,16)
    for (int q = threadIdx.x; q < rows * 16; q += THREADS) {
      const int j = q >> 4, blk = (q >> 2) & 3, g4 = q & 3;
      const int c4 = blk * 8 + g4;
      if (c4 + 4 >= cols4) continue;  // the up half lies past N
      const float4 g = row_scale(red4[j * ld4 + c4], j), u = row_scale(red4[j * ld4 + c4 + 4], j);
      const float4 a = make_float4(silu_f(g.x) * u.x, silu_f(g.y) * u.y, silu_f(g.z) * u.z, silu_f(g.w) * u.w);
      const long o = (long)(tok0 + j) * p.ldc + ((n0 + blk * 32) >> 5) * 16 + g4 * 4;
      *reinterpret_cast<float4*>(p.C + o) = a;
      store_split4(p.C_big, p.C_small, o, a, p.xfmt);
    }
    return;
  }
  if (p.epi == EPI_ROPE) {
    // q/k/v projection + bias, then apply_rotary_pos_emb (modeling_qwen2.py:116-146)
    // on q and k with separately rounded products, as rope_kv() does.  A
    // 128-column tile holds whole heads, so each rotary partner is in the tile.
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
        float4 v = f4add(row_scale(red4[j * ld4 + c4], j), bv[k]);
        if (h < r.heads + r.kv_heads) {
          const int pc4 = d < half ? c4 + half / 4 : c4 - half / 4;
          const float4 pv = f4add(row_scale(red4[j * ld4 + pc4], j), bp[k]);
          v = d < half ? f4add_rn(f4mul(v, cs[k]), f4mul(f4neg(pv), sn[k]))   // x1 cos - x2 sin
                       : f4add_rn(f4mul(v, cs[k]), f4mul(pv, sn[k]));          // x2 cos + x1 sin
        }
        float* dst;
        if (h < r.heads) {
          dst = r.q_out + ((long)m * r.heads + h) * D + d;
        } else {
          const bool is_k = h < r.heads + r.kv_heads;
          const int g = is_k ? h - r.heads : h - r.heads - r.kv_heads;
          float* cache = is_k ? r.k_dst : r.v_dst;
          dst = r.slot < 0 ? cache + ((long)g * r.prefix_cap + m) * D + d : cache + ((long)m * r.kv_heads + g) * D + d;
          if (r.slot < 0 && r.kpair_hi) {
            // the same K / V values as fp16 pairs for the tensor-core attention
            __align__(8) __half hi[4];
            __align__(8) __half lo[4];
            pair_split(v.x, hi[0], lo[0]); pair_split(v.y, hi[1], lo[1]);
            pair_split(v.z, hi[2], lo[2]); pair_split(v.w, hi[3], lo[3]);
            if (is_k) {  // V is written transposed below
              const long o = ((long)g * r.pair_cap + m) * D + d;
              *reinterpret_cast<uint2*>(static_cast<__half*>(r.kpair_hi) + o) = *reinterpret_cast<const uint2*>(hi);
              *reinterpret_cast<uint2*>(static_cast<__half*>(r.kpair_lo) + o) = *reinterpret_cast<const uint2*>(lo);
            }
          }
        }
        *reinterpret_cast<float4*>(dst) = v;
      }
    }
    if (r.slot < 0 && r.vtpair_hi && n0 + FTILE_COLS > (r.heads + r.kv_heads) * D) {
      // the tile's V columns as fp16 pairs, transposed ([group][dim][token]):
      // consecutive threads take consecutive tokens of a column, so the stores
      // of a warp are contiguous
      const float* red = reinterpret_cast<const float*>(red4);
      for (int q = threadIdx.x; q < rows * cols4 * 4; q += THREADS) {
        const int c = q / rows, j = q % rows;
        const int col = n0 + c, h = col / D, d = col % D;
        if (h < r.heads + r.kv_heads) continue;
        const int g = h - r.heads - r.kv_heads;
        float v = red[j * ld4 * 4 + c];
        if (scaled) v *= rsc[j];
        v += p.bias[col];
        __half hi, lo;
        pair_split(v, hi, lo);
        const long o = ((long)g * D + d) * r.pair_cap + tok0 + j;
        static_cast<__half*>(r.vtpair_hi)[o] = hi;
        static_cast<__half*>(r.vtpair_lo)[o] = lo;
      }
    }
    return;
  }
  if (p.epi == EPI_RESID && p.fold.ss_out) {
    // x += y, its split, and the row's sum of squares over this 128-column
    // tile (a warp holds one row: lane = float4 column); every residual value
    // of the thread is loaded before the first is used
    constexpr int QB = 4;  // iterations per thread whose residual loads are in flight together
    for (int q0 = threadIdx.x; q0 < rows * 32; q0 += QB * THREADS) {
      float4 x[QB];
#pragma unroll
      for (int k = 0; k < QB; ++k) {
        const int q = q0 + k * THREADS, j = q >> 5, c4 = q & 31;
        x[k] = q < rows * 32 && c4 < cols4
                   ? *reinterpret_cast<const float4*>(p.C + (long)(tok0 + j) * p.ldc + n0 + c4 * 4)
                   : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int k = 0; k < QB; ++k) {
        const int q = q0 + k * THREADS, j = q >> 5, c4 = q & 31;
        if (q < rows * 32) {  // whole warps: rows * 32 is a multiple of 32
          const bool ok = c4 < cols4;
          const long o = (long)(tok0 + j) * p.ldc + n0 + c4 * 4;
          float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
          if (ok) {
            v = f4add(x[k], red4[j * ld4 + c4]);
            *reinterpret_cast<float4*>(p.C + o) = v;
            store_split4(p.C_big, p.C_small, o, v, p.xfmt);
          }
          const float sq = warp_sum((v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w));
          if (c4 == 0) p.fold.ss_out[(long)(n0 >> 7) * p.fold.ld + tok0 + j] = sq;
        }
      }
    }
    return;
  }
  for (int q = threadIdx.x; q < rows * 32; q += THREADS) {
    const int j = q >> 5, c4 = q & 31;
    if (c4 >= cols4) continue;
    float4 v = row_scale(red4[j * ld4 + c4], j);
    const int col = n0 + c4 * 4;
    float4* c = reinterpret_cast<float4*>(p.C + (long)(tok0 + j) * p.ldc + col);
    if (p.epi == EPI_BIAS) v = f4add(v, *reinterpret_cast<const float4*>(p.bias + col));
    else if (p.epi == EPI_RESID) v = f4add(*c, v);
    *c = v;
  }
  if (p.lse && p.epi == EPI_STORE) {
    // LM head: every row's (max, sum of exp(x - max)) over the tile's columns,
    // for the first log-softmax (the step tail then reads the logits once).
    // Warp w takes rows w, w + W, ... eight at a time (lane = float4 column),
    // so the eight shuffle trees of a group overlap instead of queueing.  The
    // hardware exponential: these partials only set the row's normaliser,
    // whose sum over the vocabulary averages their rounding.
    constexpr int NW = THREADS / 32, G = 8;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int j0 = warp; j0 < rows; j0 += NW * G) {
      float4 v[G];
      float mx[G], e[G];
#pragma unroll
      for (int r = 0; r < G; ++r) {
        const int j = j0 + r * NW;
        const bool ok = j < rows && lane < cols4;
        v[r] = ok ? row_scale(red4[j * ld4 + lane], j) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
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

// Split-K finish, claim step, after every thread of the CTA has stored its
// partial tile (then __threadfence + __syncthreads).  A tile's splits are
// launched as clusters of consecutive splits; the cluster holding the last
// partial to arrive finishes the tile, each of its CTAs summing a slice of the
// rows over all splits in split order (the bits one CTA summing every row
// would get) and running the epilogue on that slice.  Returns whether this
// CTA finishes rows [r0, r1).  `red_bar` (count = cluster size) and `*go` (0)
// were set before the start-up cluster barrier.
//
// A CTA that aborted (a pipeline wait ran out; the status word says so) still
// takes its ticket and arrives on every peer with `skip` set: the ticket count
// stays whole for the next launch, and the CTA stays resident until every
// peer's remote store and arrive on it has happened.  It never finishes rows,
// and when it holds the last ticket no CTA of its cluster does.
template <class P>
RTR_DEVICE bool splitk_claim(const P& p, uint32_t red_bar, int* go, int rows, int tile, int& r0, int& r1,
                             bool skip = false) {
  const uint32_t cs = cluster_ncta();
  if (threadIdx.x == 0) {
    int* tk = p.tickets + tile;
    const bool last = atomicAdd(tk, 1) == p.splits - 1;
    if (last) {
      *tk = 0;  // re-arm for the next launch / graph replay
      __threadfence();
    }
    const bool fin = last && !skip;
    if (cs == 1) {
      *go = fin;
    } else {
      const uint32_t goa = smem_addr(go);
      for (uint32_t r = 0; r < cs; ++r) {
        if (fin) st_cluster_u32(cluster_map(goa, r), 1u);
        mbar_arrive_remote(cluster_map(red_bar, r));
      }
      // every CTA of the cluster has arrived: no remote access to this CTA follows
      if (!mbar_wait_cluster(red_bar, 0)) {
        atomicOr(p.status, RTR_DEV_TIMEOUT);
        *go = 0;
      }
    }
  }
  __syncthreads();
  if (skip || !*reinterpret_cast<volatile int*>(go)) return false;
  __threadfence();
  const int r = (int)cluster_rank();
  r0 = r * rows / (int)cs;
  r1 = (r + 1) * rows / (int)cs;
  return r1 > r0;
}

template <int THREADS, int NTOK>
RTR_DEVICE void splitk_finish(const TcParams& p, float4* red4, uint32_t red_bar, int* go, int tok0, int n0,
                              int rows, int cols4, int tile, long tstride) {
  int r0 = 0, r1 = 0;
  if (!splitk_claim(p, red_bar, go, rows, tile, r0, r1)) return;
  splitk_sum<THREADS, NTOK>(p, red4, r0, r1 - r0, cols4, tile, tstride);
  tile_epilogue<THREADS>(p, red4 + r0 * 32, 32, tok0 + r0, n0, r1 - r0, cols4);
}

}  // namespace rtr
