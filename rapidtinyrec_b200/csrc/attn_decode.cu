// Folded decode attention with the key range split over a thread-block cluster.
//
// The reference folds the query heads that share a KV head into rows
// (rapidtinyrec/folded_attention.py:16-31): q [B, Hq, 1, D] becomes
// [B, Hkv, Hq/Hkv, D], so one SDPA call streams each KV head's keys once for
// all its query heads.  Here the rows of KV group g are (beam b, head j) for
// the 50 beams and the Hq/Hkv heads of the group, and a CTA owns 32 of them:
//
//   cluster of 8 CTAs = one (user, KV group, 32-row tile); CTA rank r of the
//   cluster takes keys [r K, (r + 1) K) of the shared prefix, K = ceil(L / 8)
//   (L is read from device memory, so one captured graph serves every prompt
//   length); the last rank also takes every beam's own suffix keys, found
//   through the ancestry table (the direct-reorder parent gather,
//   prefix_replay.py:95-117, without moving any bytes).
//
// Per 32-key chunk, staged by TMA (cp.async.bulk.tensor, 128-byte swizzle, a
// two-slot ring; this GPU's memory only, no multicast):
//   A  scores: warp w takes head_dim / 8 dimensions; lane = 4 rows x 8 keys
//      (keys lane % 4 + 4 i, so the 8 lanes of a shared-memory phase read 4
//      consecutive keys: distinct swizzled units), q of its rows in registers;
//   B  thread = (row, 4 keys): sums the 8 warps' partial scores in warp
//      order, online softmax of the row across its 8 lanes (shuffles);
//   C  warp w = 4 rows, lane = head_dim / 32 dimensions: O = O corr + P.V.
// The 8 CTAs' partial (m, l, O) meet through distributed shared memory: rank
// r finishes rows 4r .. 4r + 3, summing the ranks in rank order (the same
// bits on every run).
#include <cuda.h>
#include <math.h>

#include "common.cuh"
#include "engine.h"
#include "tcgen05.cuh"

namespace rtr {

constexpr int FD_ROWS = 32;      // (beam, head) rows of a CTA (16 measured slower)
constexpr int FD_KC = 32;        // keys per chunk = TMA box height
constexpr int FD_SPLITS = 8;     // CTAs of a cluster, one key range each
constexpr int FD_WARPS = 8;
constexpr int FD_THREADS = FD_WARPS * 32;
constexpr int FD_PLD = FD_KC + 1;  // partial-score / probability row stride (floats)
constexpr int FD_RL = FD_ROWS / FD_WARPS;          // rows per lane (score phase), per warp (P.V phase)
constexpr int FD_LPR = FD_THREADS / FD_ROWS;       // lanes per row in the softmax phase
constexpr int FD_KPT = FD_KC / FD_LPR;             // keys per thread in the softmax phase
constexpr int FD_RPR = FD_ROWS / FD_SPLITS;        // rows each cluster rank finishes
static_assert(FD_RL * FD_WARPS == FD_ROWS && FD_LPR <= 32 && FD_KPT >= 1 && FD_RPR >= 1, "row tiling");

template <int HD, typename T> struct FdCfg {
  static constexpr int E = 16 / (int)sizeof(T);            // elements per 16-byte unit
  static constexpr int BOXW = 128 / (int)sizeof(T);        // elements per 128-byte box row
  static constexpr int NBOX = HD / BOXW;                   // boxes across a K or V row
  static constexpr int BOX_BYTES = FD_KC * 128;            // one box: 32 keys x 128 bytes
  static constexpr int HALF = NBOX * BOX_BYTES;            // K (or V) of a chunk
  static constexpr int STAGE = 2 * HALF;
  static constexpr int DS = HD / FD_WARPS;                 // score phase: dimensions per warp
  static constexpr int DU = DS / E;                        // 16-byte units per warp slice
  static constexpr int VD = HD / 32;                       // P.V phase: dimensions per lane
  static constexpr int RING = 2 * STAGE;
  static constexpr int PART = FD_WARPS * FD_ROWS * FD_PLD; // floats
  static constexpr int OPART = FD_ROWS * HD;               // floats (aliases the ring)
  static_assert(NBOX >= 1 && DU >= 1 && VD >= 1, "head_dim 64 or 128");
  static_assert(OPART * 4 <= RING, "partial O fits in the ring");
  // ring (at least RING bytes: also the suffix staging) | part | P | corr | ml | bars
  static constexpr int SMEM_REST = 4 * (PART + FD_ROWS * FD_PLD + FD_ROWS + 2 * FD_ROWS) + 64;
};

// Loads from a peer CTA's shared memory (addresses from cluster_map).  Not
// volatile: the cluster barriers around them order them, and the compiler may
// issue them back to back.
RTR_DEVICE float ld_cluster_f32x1(uint32_t addr) {
  float v;
  asm("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}
RTR_DEVICE float2 ld_cluster_f32x2(uint32_t addr) {
  float2 v;
  asm("ld.shared::cluster.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr));
  return v;
}
RTR_DEVICE void cluster_barrier() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// E elements of type T at a 16-byte-aligned shared address, as floats.
template <typename T, int N> RTR_DEVICE void lds_f(const unsigned char* p, float (&x)[N]);
template <> RTR_DEVICE void lds_f<float, 4>(const unsigned char* p, float (&x)[4]) {
  const float4 v = *reinterpret_cast<const float4*>(p);
  x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
}
template <> RTR_DEVICE void lds_f<float, 2>(const unsigned char* p, float (&x)[2]) {
  const float2 v = *reinterpret_cast<const float2*>(p);
  x[0] = v.x; x[1] = v.y;
}
template <> RTR_DEVICE void lds_f<__nv_bfloat16, 8>(const unsigned char* p, float (&x)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
    x[2 * i] = f.x; x[2 * i + 1] = f.y;
  }
}
template <> RTR_DEVICE void lds_f<__nv_bfloat16, 4>(const unsigned char* p, float (&x)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  x[0] = a.x; x[1] = a.y; x[2] = b.x; x[3] = b.y;
}
template <> RTR_DEVICE void lds_f<__nv_bfloat16, 2>(const unsigned char* p, float (&x)[2]) {
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
  x[0] = a.x; x[1] = a.y;
}

// N consecutive elements of global memory as floats (N * sizeof(T) bytes, aligned).
template <typename T, int N> RTR_DEVICE void ldg_f(const T* p, float (&x)[N]) {
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int i = 0; i < N; i += 4) {
      if constexpr (N % 4 == 0) {
        const float4 v = *reinterpret_cast<const float4*>(p + i);
        x[i] = v.x; x[i + 1] = v.y; x[i + 2] = v.z; x[i + 3] = v.w;
      }
    }
    if constexpr (N % 4 != 0) {
#pragma unroll
      for (int i = 0; i < N; i += 2) {
        const float2 v = *reinterpret_cast<const float2*>(p + i);
        x[i] = v.x; x[i + 1] = v.y;
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; i += 2) {
      const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p + i));
      x[i] = v.x; x[i + 1] = v.y;
    }
  }
}

// Byte offset of element (key, d) of a K or V chunk staged as NBOX boxes of
// [32 keys][128 bytes] in the 128-byte swizzle (16-byte unit u of key k sits
// at unit u ^ (k % 8)).
template <int HD, typename T> RTR_DEVICE int fd_off(int key, int d) {
  using C = FdCfg<HD, T>;
  const int gu = d / C::E;
  return (gu >> 3) * C::BOX_BYTES + key * 128 + (((gu & 7) ^ (key & 7)) << 4) + (d % C::E) * (int)sizeof(T);
}

// Shared-memory row stride (elements) of the suffix rows the last rank stages:
// padded by 16 bytes so 8 consecutive rows start in distinct bank groups.
template <int HD, typename T> constexpr int fd_srow() { return HD + 16 / (int)sizeof(T); }
// Beams a 32-row tile touches for hpg query heads per KV head.
__host__ __device__ constexpr int fd_tile_beams(int hpg) { return (FD_ROWS - 1) / hpg + 2; }

// Ring bytes: two chunks, or the last rank's suffix staging (4 slots of K and
// V rows of the tile's beams) when that is larger.
template <int HD, typename T> constexpr int fd_ring_bytes(int hpg) {
  const int staging = 2 * 4 * fd_tile_beams(hpg) * fd_srow<HD, T>() * (int)sizeof(T);
  return staging > FdCfg<HD, T>::RING ? (staging + 1023) / 1024 * 1024 : FdCfg<HD, T>::RING;
}

template <int HD, typename T>
__global__ void __cluster_dims__(FD_SPLITS, 1, 1) __launch_bounds__(FD_THREADS, 2) decode_attn_folded_kernel(
    const __grid_constant__ CUtensorMap arena, long krow0, long vrow0, long user_rows, const T* __restrict__ q,
    const T* __restrict__ ksuf, const T* __restrict__ vsuf, const int32_t* __restrict__ anc,
    const int32_t* __restrict__ L_dev, T* __restrict__ out, float* __restrict__ out_big, float* __restrict__ out_small,
    int beams, int cap, int heads, int kv_heads, int t, float scale, uint32_t* __restrict__ status,
    int anc_user_stride, int xfmt, int ring_bytes) {
  using C = FdCfg<HD, T>;
  constexpr int SROW = fd_srow<HD, T>();
  constexpr int PREFIX_RANKS = FD_SPLITS - 1;  // the last rank takes the suffix
  extern __shared__ __align__(1024) unsigned char fd_smem_raw[];
  // the ring starts on a 1024-byte boundary (the 128-byte swizzle); offset
  // from the shared array itself so the compiler keeps every access a
  // shared-memory one
  unsigned char* ring = fd_smem_raw + ((1024u - (smem_addr(fd_smem_raw) & 1023u)) & 1023u);
  float* part = reinterpret_cast<float*>(ring + ring_bytes);  // [8 warps][32 rows][PLD]
  float* ps = part + C::PART;                                // [32 rows][PLD] probabilities
  float* corr_s = ps + FD_ROWS * FD_PLD;                     // [32]
  float* ml = corr_s + FD_ROWS;                              // [32][2] (m, l) for the cluster combine
  uint64_t* full = reinterpret_cast<uint64_t*>(ml + 2 * FD_ROWS);  // [2] chunk landed
  volatile int* abort_flag = reinterpret_cast<volatile int*>(full + 2);
  float* opart = reinterpret_cast<float*>(ring);             // [32][HD] after the last chunk

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rank = (int)cluster_rank();
  const bool suffix_rank = rank == PREFIX_RANKS;
  const int hpg = heads / kv_heads;
  const int nrows = beams * hpg;                             // rows of one KV group
  const int ug = blockIdx.z, u = ug / kv_heads, g = ug % kv_heads;
  const int rt0 = blockIdx.y * FD_ROWS;
  const int r0 = u * beams, rows_all = gridDim.z / kv_heads * beams;
  const int bfirst = rt0 / hpg;                              // first beam of the tile
  const int nb = fd_tile_beams(hpg);                         // suffix staging: beams per slot
  anc += (long)u * anc_user_stride;

  int L = L_dev[u];  // copied from the host before the request's first kernel
  const bool bad_len = L < 1 || L > cap;
  if (bad_len) L = 0;  // the prefill recorded no valid prefix: attend to the suffix only
  const int kper = (L + PREFIX_RANKS - 1) / PREFIX_RANKS;
  const int kbeg = suffix_rank ? L : (rank * kper < L ? rank * kper : L);
  const int kend = suffix_rank ? L : (kbeg + kper < L ? kbeg + kper : L);
  const int nchunks = (kend - kbeg + FD_KC - 1) / FD_KC;
  const long krow = krow0 + (long)u * user_rows + (long)g * cap + kbeg;
  const long vrow = vrow0 + (long)u * user_rows + (long)g * cap + kbeg;

  auto issue = [&](int c) {  // chunk c into slot c & 1 (thread 0)
    unsigned char* st = ring + (c & 1) * C::STAGE;
    const uint32_t bar = smem_addr(&full[c & 1]);
    mbar_expect_tx(bar, C::STAGE);
#pragma unroll
    for (int b = 0; b < C::NBOX; ++b) {
      tma_load_2d(smem_addr(st + b * C::BOX_BYTES), &arena, b * C::BOXW, (int)(krow + c * FD_KC), bar);
      tma_load_2d(smem_addr(st + C::HALF + b * C::BOX_BYTES), &arena, b * C::BOXW, (int)(vrow + c * FD_KC), bar);
    }
  };
  // suffix staging (last rank): K and V rows of slot sl of the tile's beams,
  // [slot][beam][SROW] each, in the ring
  T* sk = reinterpret_cast<T*>(ring);
  T* sv = sk + 4 * nb * SROW;
  auto stage_suffix = [&](int sl) {
    constexpr int UR = HD / C::E;  // 16-byte units per row
    for (int i = tid; i < nb * UR; i += FD_THREADS) {
      const int bi = i / UR, d = (i % UR) * C::E;
      const int b = bfirst + bi;
      if (b >= beams) continue;
      int row = sl == t - 1 ? b : anc[b * 4 + sl];
      if (row < 0 || row >= beams) {
        if (d == 0) atomicOr(status, RTR_DEV_BAD_PARENT);
        row = b;
      }
      const long off = (((long)sl * rows_all + r0 + row) * kv_heads + g) * HD + d;
      cp_async16(sk + (sl * nb + bi) * SROW + d, ksuf + off, true);
      cp_async16(sv + (sl * nb + bi) * SROW + d, vsuf + off, true);
    }
  };
  if (tid == 0) {
    mbar_init(smem_addr(&full[0]), 1);
    mbar_init(smem_addr(&full[1]), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  pdl_launch_dependents();
  // Every kernel of the chain may let its successor start early, so nothing
  // written by an earlier kernel (not even the prefill's prefix) is read
  // before this wait.
  pdl_wait();
  if (tid == 0) {
    if (bad_len && rank == 0) atomicOr(status, RTR_DEV_BAD_LENGTH);
    if (nchunks > 0) issue(0);
    if (nchunks > 1) issue(1);
  }
  if (suffix_rank) {
    for (int sl = 0; sl < t; ++sl) stage_suffix(sl);
    cp_async_commit();
  }
  __syncthreads();

  // score phase: q of rows 4 rq .. 4 rq + 3, dimensions [warp DS, (warp + 1) DS)
  const int rq = lane >> 2, ko = lane & 3;
  float qr[FD_RL][C::DS];
#pragma unroll
  for (int a = 0; a < FD_RL; ++a) {
    const int rho = rt0 + FD_RL * rq + a;
    if (rho < nrows) {
      const int b = rho / hpg, h = g * hpg + rho % hpg;
      ldg_f<T, C::DS>(q + ((long)(r0 + b) * heads + h) * HD + warp * C::DS, qr[a]);
    } else {
#pragma unroll
      for (int e = 0; e < C::DS; ++e) qr[a][e] = 0.f;
    }
  }
  // softmax state of row tid / 8 (replicated over its 8 lanes)
  const int brow = tid / FD_LPR, bq = tid % FD_LPR;
  float m = -INFINITY, l = 0.f;
  // P.V accumulators: rows 4 warp .. 4 warp + 3, dimensions lane VD ..
  float acc[FD_RL][C::VD];
#pragma unroll
  for (int a = 0; a < FD_RL; ++a)
#pragma unroll
    for (int e = 0; e < C::VD; ++e) acc[a][e] = 0.f;

  // B: row brow's online softmax over scores part[.][brow][0 .. nk) (shared by
  // the prefix chunks and the suffix)
  auto softmax_step = [&](int nk) {
    float sc[FD_KPT], mx = -INFINITY;
#pragma unroll
    for (int cc = 0; cc < FD_KPT; ++cc) {
      const int k = FD_KPT * bq + cc;
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < FD_WARPS; ++w) v += part[(w * FD_ROWS + brow) * FD_PLD + k];
      sc[cc] = k < nk ? v * scale : -INFINITY;
      mx = fmaxf(mx, sc[cc]);
    }
#pragma unroll
    for (int o = 1; o < FD_LPR; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float mn = fmaxf(m, mx);  // finite: at least one key
    const float corr = expf(m - mn);
    float sum = 0.f;
#pragma unroll
    for (int cc = 0; cc < FD_KPT; ++cc) {
      const float p = expf(sc[cc] - mn);
      sum += p;
      ps[brow * FD_PLD + FD_KPT * bq + cc] = p;
    }
#pragma unroll
    for (int o = 1; o < FD_LPR; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    l = l * corr + sum;
    m = mn;
    if (bq == 0) corr_s[brow] = corr;
  };

  int consumed = 0;  // chunks fully used (the ones after it, up to two, may be in flight)
  for (int c = 0; c < nchunks; ++c) {
    const bool landed = mbar_wait(smem_addr(&full[c & 1]), (c >> 1) & 1, abort_flag);
    if (__syncthreads_or(!landed)) break;  // the whole CTA leaves the loop together
    const unsigned char* kst = ring + (c & 1) * C::STAGE;
    const unsigned char* vst = kst + C::HALF;
    const int key0 = kbeg + c * FD_KC;
    const int nk = kend - key0 < FD_KC ? kend - key0 : FD_KC;
    {  // A: partial scores of FD_RL rows x 8 keys over this warp's dimensions, in two halves of 4 keys
      float* pw = part + (warp * FD_ROWS + FD_RL * rq) * FD_PLD + ko;
#pragma unroll
      for (int hk = 0; hk < 2; ++hk) {
        float s[FD_RL][4];
#pragma unroll
        for (int a = 0; a < FD_RL; ++a)
#pragma unroll
          for (int i = 0; i < 4; ++i) s[a][i] = 0.f;
#pragma unroll
        for (int uu = 0; uu < C::DU; ++uu) {
          const int d0 = warp * C::DS + uu * C::E;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float kv[C::E];
            lds_f<T, C::E>(kst + fd_off<HD, T>(ko + 4 * (4 * hk + i), d0), kv);
#pragma unroll
            for (int a = 0; a < FD_RL; ++a)
#pragma unroll
              for (int e = 0; e < C::E; ++e) s[a][i] = fmaf(qr[a][uu * C::E + e], kv[e], s[a][i]);
          }
        }
#pragma unroll
        for (int a = 0; a < FD_RL; ++a)
#pragma unroll
          for (int i = 0; i < 4; ++i) pw[a * FD_PLD + 4 * (4 * hk + i)] = s[a][i];
      }
    }
    __syncthreads();
    softmax_step(nk);  // B
    __syncthreads();
    {  // C: acc = acc corr + P.V over the chunk's valid keys
#pragma unroll
      for (int a = 0; a < FD_RL; ++a) {
        const float cr = corr_s[FD_RL * warp + a];
#pragma unroll
        for (int e = 0; e < C::VD; ++e) acc[a][e] *= cr;
      }
      const float* pr = ps + FD_RL * warp * FD_PLD;
#pragma unroll 4
      for (int k = 0; k < nk; ++k) {
        float v[C::VD];
        lds_f<T, C::VD>(vst + fd_off<HD, T>(k, lane * C::VD), v);
#pragma unroll
        for (int a = 0; a < FD_RL; ++a) {
          const float p = pr[a * FD_PLD + k];
#pragma unroll
          for (int e = 0; e < C::VD; ++e) acc[a][e] = fmaf(p, v[e], acc[a][e]);
        }
      }
    }
    __syncthreads();  // the slot is free: refill it with chunk c + 2
    if (tid == 0 && c + 2 < nchunks) issue(c + 2);
    consumed = c + 1;
  }
  if (consumed < nchunks) {
    // a chunk never landed: record it, let issued copies land before the ring goes away
    if (tid == 0) {
      atomicOr(status, RTR_DEV_TIMEOUT);
      const int issued = nchunks < consumed + 2 ? nchunks : consumed + 2;
      for (int c = consumed; c < issued; ++c) mbar_drain(smem_addr(&full[c & 1]), (c >> 1) & 1);
    }
    __syncthreads();
  }

  // The suffix rank: every row's t suffix keys, its beam's own (slot t - 1 is
  // the beam's row, older slots the rows the ancestry table recorded: the
  // direct-reorder parent gather without moving bytes).
  if (suffix_rank) {
    cp_async_wait<0>();
    __syncthreads();
    {  // A: lane ko takes slot ko of its 4 rows over this warp's dimensions
      float* pw = part + (warp * FD_ROWS + FD_RL * rq) * FD_PLD + ko;
#pragma unroll
      for (int a = 0; a < FD_RL; ++a) {
        const int rho = rt0 + FD_RL * rq + a;
        const int bi = (rho < nrows ? rho / hpg : bfirst) - bfirst;
        float sa = 0.f;
        if (ko < t) {
          const T* kr = sk + (ko * nb + bi) * SROW + warp * C::DS;
#pragma unroll
          for (int uu = 0; uu < C::DU; ++uu) {
            float kv[C::E];
            lds_f<T, C::E>(reinterpret_cast<const unsigned char*>(kr + uu * C::E), kv);
#pragma unroll
            for (int e = 0; e < C::E; ++e) sa = fmaf(qr[a][uu * C::E + e], kv[e], sa);
          }
        }
        pw[a * FD_PLD] = sa;
      }
    }
    __syncthreads();
    softmax_step(t);  // B: keys 0 .. t - 1 are the slots
    __syncthreads();
#pragma unroll
    for (int a = 0; a < FD_RL; ++a) {  // C
      const int rr = FD_RL * warp + a, rho = rt0 + rr;
      const int bi = (rho < nrows ? rho / hpg : bfirst) - bfirst;
      const float cr = corr_s[rr];
#pragma unroll
      for (int e = 0; e < C::VD; ++e) acc[a][e] *= cr;
      for (int sl = 0; sl < t; ++sl) {
        const float p = ps[rr * FD_PLD + sl];
        float v[C::VD];
        lds_f<T, C::VD>(reinterpret_cast<const unsigned char*>(sv + (sl * nb + bi) * SROW + lane * C::VD), v);
#pragma unroll
        for (int e = 0; e < C::VD; ++e) acc[a][e] = fmaf(p, v[e], acc[a][e]);
      }
    }
  }

  // partial (m, l, O) of the 32 rows into shared memory, then the cluster combine
  __syncthreads();  // the ring is free (every chunk consumed or drained, the suffix read)
  if (bq == 0) {
    ml[2 * brow] = m;
    ml[2 * brow + 1] = l;
  }
#pragma unroll
  for (int a = 0; a < FD_RL; ++a)
#pragma unroll
    for (int e = 0; e < C::VD; ++e) opart[(FD_RL * warp + a) * HD + lane * C::VD + e] = acc[a][e];
  cluster_barrier();
  {
    // rank r finishes rows r FD_RPR ..: thread = (row, DPT dimensions); the
    // remote loads of all ranks are issued before any is used
    constexpr int DPT = (HD * FD_RPR + FD_THREADS - 1) / FD_THREADS;
    const bool active = tid < HD * FD_RPR / DPT;
    const int rr = FD_RPR * rank + (active ? tid / (HD / DPT) : 0);
    const int d0 = (tid % (HD / DPT)) * DPT;
    const uint32_t ml_a = smem_addr(ml + 2 * rr), o_a = smem_addr(opart + rr * HD + d0);
    float2 mlj[FD_SPLITS];
    float oj[FD_SPLITS][DPT];
#pragma unroll
    for (int j = 0; j < FD_SPLITS; ++j) {
      mlj[j] = ld_cluster_f32x2(cluster_map(ml_a, j));
      if constexpr (DPT == 2) {
        const float2 v = ld_cluster_f32x2(cluster_map(o_a, j));
        oj[j][0] = v.x;
        oj[j][1] = v.y;
      } else {
        oj[j][0] = ld_cluster_f32x1(cluster_map(o_a, j));
      }
    }
    float M = -INFINITY;
#pragma unroll
    for (int j = 0; j < FD_SPLITS; ++j) M = fmaxf(M, mlj[j].x);
    float Ls = 0.f, o[DPT];
#pragma unroll
    for (int e = 0; e < DPT; ++e) o[e] = 0.f;
#pragma unroll
    for (int j = 0; j < FD_SPLITS; ++j) {  // rank order: the same bits every run
      const float w = expf(mlj[j].x - M);  // 0 for a rank without keys (m = -inf)
      Ls = fmaf(w, mlj[j].y, Ls);
#pragma unroll
      for (int e = 0; e < DPT; ++e) o[e] = fmaf(w, oj[j][e], o[e]);
    }
    const int rho = rt0 + rr;
    if (active && rho < nrows) {
      const int b = rho / hpg, h = g * hpg + rho % hpg;
      const float inv = 1.0f / Ls;
      const long base = ((long)(r0 + b) * heads + h) * HD + d0;
#pragma unroll
      for (int e = 0; e < DPT; ++e) {
        if constexpr (sizeof(T) == 4)
          store_split(reinterpret_cast<float*>(out), out_big, out_small, base + e, o[e] * inv, xfmt);
        else
          reinterpret_cast<__nv_bfloat16*>(out)[base + e] = __float2bfloat16_rn(o[e] * inv);
      }
    }
  }
  cluster_barrier();  // no CTA leaves while a peer still reads its shared memory
}

template <int HD, typename T>
static cudaError_t launch_folded(const TensorMap& arena, long krow0, long vrow0, long user_rows, const void* q,
                                 const void* ks, const void* vs, const int32_t* anc, const int32_t* L_dev, int t,
                                 void* out, float* ob, float* os, int beams, int cap, int heads, int kv_heads,
                                 float scale, uint32_t* status, cudaStream_t stream, const DecodeUsers& du, int xfmt) {
  const int hpg = heads / kv_heads;
  const int ring = fd_ring_bytes<HD, T>(hpg);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(FD_SPLITS, (beams * hpg + FD_ROWS - 1) / FD_ROWS, du.users * kv_heads);
  cfg.blockDim = dim3(FD_THREADS);
  cfg.dynamicSmemBytes = 1024 + ring + FdCfg<HD, T>::SMEM_REST;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_on(PDL_ATTN) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, decode_attn_folded_kernel<HD, T>, *reinterpret_cast<const CUtensorMap*>(&arena),
                            krow0, vrow0, user_rows, static_cast<const T*>(q), static_cast<const T*>(ks),
                            static_cast<const T*>(vs), anc, L_dev, static_cast<T*>(out), ob, os, beams, cap, heads,
                            kv_heads, t, scale, status, du.anc_user_stride, xfmt, ring);
}

cudaError_t attention_decode_folded(const TensorMap& arena, long krow0, long vrow0, long user_rows, const void* q,
                                    const void* k_suffix, const void* v_suffix, const int32_t* anc,
                                    const int32_t* L_dev, int t, void* out, float* out_big, float* out_small,
                                    int beams, int prefix_cap, int heads, int kv_heads, int head_dim, float scale,
                                    uint32_t* status, bool bf16, cudaStream_t stream, const DecodeUsers& du,
                                    int xfmt) {
  if (t < 1 || t > 4 || beams > MAX_BEAMS || du.users < 1 || !attention_folded_supported(heads, kv_heads, head_dim, bf16))
    return cudaErrorInvalidValue;
  if (head_dim == 128)
    return bf16 ? launch_folded<128, __nv_bfloat16>(arena, krow0, vrow0, user_rows, q, k_suffix, v_suffix, anc, L_dev,
                                                    t, out, nullptr, nullptr, beams, prefix_cap, heads, kv_heads, scale,
                                                    status, stream, du, 0)
                : launch_folded<128, float>(arena, krow0, vrow0, user_rows, q, k_suffix, v_suffix, anc, L_dev, t, out,
                                            out_big, out_small, beams, prefix_cap, heads, kv_heads, scale, status,
                                            stream, du, xfmt);
  if (head_dim == 64)
    return bf16 ? launch_folded<64, __nv_bfloat16>(arena, krow0, vrow0, user_rows, q, k_suffix, v_suffix, anc, L_dev,
                                                   t, out, nullptr, nullptr, beams, prefix_cap, heads, kv_heads, scale,
                                                   status, stream, du, 0)
                : launch_folded<64, float>(arena, krow0, vrow0, user_rows, q, k_suffix, v_suffix, anc, L_dev, t, out,
                                           out_big, out_small, beams, prefix_cap, heads, kv_heads, scale, status,
                                           stream, du, xfmt);
  return cudaErrorInvalidValue;
}

bool attention_folded_supported(int heads, int kv_heads, int head_dim, bool bf16) {
  // at least two query heads per KV head: a 32-row tile touches at most 17 beams
  return kv_heads >= 1 && heads % kv_heads == 0 && heads / kv_heads >= 2 && (head_dim == 64 || head_dim == 128);
}

template <int HD, typename T> static cudaError_t folded_set_smem() {
  // the largest ring: two query heads per KV head (17 beams per tile)
  return cudaFuncSetAttribute(decode_attn_folded_kernel<HD, T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              1024 + fd_ring_bytes<HD, T>(2) + FdCfg<HD, T>::SMEM_REST);
}

cudaError_t attention_folded_init() {
  cudaError_t e = folded_set_smem<128, float>();
  if (e == cudaSuccess) e = folded_set_smem<64, float>();
  if (e == cudaSuccess) e = folded_set_smem<128, __nv_bfloat16>();
  if (e == cudaSuccess) e = folded_set_smem<64, __nv_bfloat16>();
  return e;
}

}  // namespace rtr
