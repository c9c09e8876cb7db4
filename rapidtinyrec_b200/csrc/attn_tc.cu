// Attention on the 5th-generation tensor cores: the decode and prefill
// attention of the fp32 mode, fp32-accurate through fp16 pairs (the scheme of
// the projection GEMM, gemm_f16x2.cu), and of the bf16 mode with bf16
// operands.
//
// The reference folds the query heads that share a KV head into rows
// (rapidtinyrec/folded_attention.py:16-31).  Here the rows of KV group g are
// its (beam, head) pairs in decode and its (token, head) pairs in prefill,
// 128 to a tile (the MMA's M).  K and V come by TMA in 64-key chunks (the
// 128-byte swizzle): in fp32 from the fp16-pair copies the prefill's q/k/v
// epilogue writes (K as [key][dim], V transposed as [dim][key], hi and lo
// planes), in bf16 K straight from the prefix arena and V from a transposed
// bf16 copy.  Per chunk, a thread per (row, quarter of the keys / dims):
//   S = q.k^T in TMEM (fp32: q_hi.[k_hi; k_lo]^T (N = 128) + q_lo.k_hi^T
//       (N = 64); bf16: one product);
//   the row's softmax over the chunk from tcgen05.ld, P back to shared memory
//       as a pair (fp16 or bf16 hi / lo);
//   O = P.V in TMEM (fp32: p_hi.[v_hi; v_lo] (N = 2 head_dim) + p_lo.v_hi;
//       bf16: p_hi.v + p_lo.v).
// The dropped lo.lo terms are 2^-22 relative (fp16 pairs).
//
//   decode_attn_tc_kernel (fp32, RTR_ATTN=tc): a thread-block cluster of 8
//       CTAs per (user, group, row tile): ranks 0..6 one 64-key chunk of the
//       shared prefix each (prompts of up to 448 tokens), rank 7 every beam's
//       own suffix keys (at most 4, found through the ancestry table: the
//       direct-reorder parent gather without moving bytes) on the FMA pipe;
//       the 8 partial (m, l, O) meet through distributed shared memory, rank
//       r finishing rows 16 r .. 16 r + 15 in rank order (the same bits every
//       run);
//   decode_attn_tc_bf16_kernel (bf16 default): the same cluster, prefix rank
//       r walking chunks r, r + 7, .. with an online softmax (any prompt the
//       arena holds);
//   prefill_attn_tc_kernel / _bf16_kernel (defaults): one CTA per tile walks
//       the causal key range with an online softmax, the next chunk's scores
//       computed while the threads run the current softmax.
// Every wait is bounded; a wait that runs out sets RTR_DEV_TIMEOUT.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <math.h>

#include "common.cuh"
#include "engine.h"
#include "tcgen05.cuh"

namespace rtr {

constexpr int AT_ROWS = 128;      // MMA M: (beam, head) rows of a tile
constexpr int AT_KEYS = 64;       // keys per chunk (one 128-byte row of fp16)
constexpr int AT_CLUSTER = 8;     // 7 prefix chunks + the suffix rank
constexpr int AT_THREADS = 512;   // thread = (row, quarter of its keys / dimensions)
constexpr int AT_MAX_PREFIX = (AT_CLUSTER - 1) * AT_KEYS;

template <int HD> struct AtCfg {
  static constexpr int NC = HD / 64;                     // 128-byte chunks of a q / k row
  static constexpr int Q_BYTES = 2 * NC * AT_ROWS * 128; // hi / lo planes
  static constexpr int K_BYTES = NC * 2 * AT_KEYS * 128; // per dim chunk: [k_hi 64 keys; k_lo 64 keys]
  static constexpr int V_BYTES = 2 * HD * 128;           // [v_hi^T HD rows; v_lo^T HD rows] x 64 keys
  static constexpr int P_BYTES = 2 * AT_ROWS * 128;      // p_hi, p_lo planes
  static constexpr int Q_OFF = 0, K_OFF = Q_BYTES, V_OFF = K_OFF + K_BYTES, P_OFF = V_OFF + V_BYTES;
  static constexpr int PRE_BYTES = P_OFF + P_BYTES;      // the prefix ranks' operands
  // (m, l) per row, barriers, then [4][128] partials, [4][80] suffix rows, [16][128] partial dots
  static constexpr int TAIL_BYTES = AT_ROWS * 8 + 64 + (4 * AT_ROWS + 4 * 80 + 16 * AT_ROWS) * 4;
  static constexpr int S_COLS = 2 * AT_KEYS;             // [hh | cross]
  static constexpr int O_COLS = 2 * HD;
  static constexpr int TMEM_COLS = S_COLS + O_COLS <= 256 ? 256 : 512;
  static_assert(AT_ROWS * (HD + 4) * 4 <= Q_BYTES + K_BYTES, "the partial O tile fits where q and k were");
};

// Beams a 128-row tile touches for hpg query heads per KV head.
__host__ __device__ constexpr int at_tile_beams(int hpg) { return (AT_ROWS - 1) / hpg + 2; }
// The suffix rank's staging: the tile's q rows ([128][HD + 4] fp32) and the
// K and V rows of 4 slots of its beams ([4][beams][HD + 4] fp32 each; the
// padding spreads rows of different beams over the banks).
template <int HD> constexpr int at_suffix_bytes(int hpg) {
  return (AT_ROWS * (HD + 4) + 2 * 4 * at_tile_beams(hpg) * (HD + 4)) * 4;
}
// Offset of the (m, l) array and the barriers: after the larger of the two uses.
template <int HD> constexpr int at_tail_off(int hpg) {
  const int a = AtCfg<HD>::PRE_BYTES, b = at_suffix_bytes<HD>(hpg);
  return ((a > b ? a : b) + 1023) / 1024 * 1024;
}

RTR_DEVICE float4 ld_cluster_f32x4(uint32_t addr) {
  float4 v;
  asm("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}
RTR_DEVICE float2 ld_cluster_f32x2_tc(uint32_t addr) {
  float2 v;
  asm("ld.shared::cluster.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr));
  return v;
}
RTR_DEVICE void cluster_barrier_tc() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Row r of a 128-byte-row operand in the 128-byte swizzle: 16-byte unit u of
// the row sits at unit u ^ (r % 8) (what TMA writes for a 1024-aligned box).
RTR_DEVICE uint8_t* sw_unit(uint8_t* plane, int r, int u) { return plane + r * 128 + ((u ^ (r & 7)) << 4); }

// Eight fp32 values as fp16 pairs (pair_split: x / 16 = hi + lo / 2048) into
// unit u of row r of the hi and lo planes.
RTR_DEVICE void put_pairs8(uint8_t* hi_plane, uint8_t* lo_plane, int r, int u, const float* x, float pre) {
  __align__(16) __half hi[8];
  __align__(16) __half lo[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float xs = x[e] * pre;
    hi[e] = __float2half_rn(xs);
    lo[e] = __float2half_rn((xs - __half2float(hi[e])) * kPairLo);
  }
  *reinterpret_cast<uint4*>(sw_unit(hi_plane, r, u)) = *reinterpret_cast<const uint4*>(hi);
  *reinterpret_cast<uint4*>(sw_unit(lo_plane, r, u)) = *reinterpret_cast<const uint4*>(lo);
}

// A tile's 128 q rows (fp32) -> fp16 pair planes in the 128-byte swizzle (the
// A operand of S = q.k^T).  Tile row rr reads q[qrow(rr) * HD ..] (qrow < 0:
// zeros); a warp reads whole rows, and every thread issues all of its loads
// before it converts and stores any, so the tile costs one L2 round trip.
template <int HD, typename RowOf>
RTR_DEVICE void load_q_pairs(uint8_t* qs, const float* __restrict__ q, RowOf qrow) {
  constexpr int NC = HD / 64, PER = AT_ROWS * (HD / 4) / AT_THREADS;
  static_assert(AT_ROWS * (HD / 4) % AT_THREADS == 0, "whole float4s per thread");
  float4 v[PER];
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int i = threadIdx.x + k * AT_THREADS, rr = i / (HD / 4), c4 = i % (HD / 4);
    const long row = qrow(rr);
    v[k] = row >= 0 ? *reinterpret_cast<const float4*>(q + row * HD + 4 * c4) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int i = threadIdx.x + k * AT_THREADS, rr = i / (HD / 4), c4 = i % (HD / 4);
    __align__(8) __half hi[4];
    __align__(8) __half lo[4];
    pair_split(v[k].x, hi[0], lo[0]); pair_split(v[k].y, hi[1], lo[1]);
    pair_split(v[k].z, hi[2], lo[2]); pair_split(v[k].w, hi[3], lo[3]);
    const int c = (4 * c4) >> 6, un = ((4 * c4) & 63) >> 3, half8 = (c4 & 1) * 8;
    *reinterpret_cast<uint2*>(sw_unit(qs + c * AT_ROWS * 128, rr, un) + half8) = *reinterpret_cast<const uint2*>(hi);
    *reinterpret_cast<uint2*>(sw_unit(qs + (NC + c) * AT_ROWS * 128, rr, un) + half8) =
        *reinterpret_cast<const uint2*>(lo);
  }
}

template <int HD>
__global__ void __cluster_dims__(AT_CLUSTER, 1, 1) __launch_bounds__(AT_THREADS, 1) decode_attn_tc_kernel(
    const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap, long krow0, long kplane,
    long kuser, long vrow0, long vplane, long vuser, int pair_cap, const float* __restrict__ q,
    const float* __restrict__ ksuf, const float* __restrict__ vsuf, const int32_t* __restrict__ anc,
    const int32_t* __restrict__ L_dev, float* __restrict__ out, float* __restrict__ out_big,
    float* __restrict__ out_small, int beams, int cap, int heads, int kv_heads, int t, float scale,
    uint32_t* __restrict__ status, int anc_user_stride, int xfmt, int tail_off) {
  using C = AtCfg<HD>;
  extern __shared__ __align__(1024) uint8_t at_smem_raw[];
  uint8_t* smem = at_smem_raw + ((1024u - (smem_addr(at_smem_raw) & 1023u)) & 1023u);
  uint8_t* qs = smem + C::Q_OFF;
  uint8_t* ks = smem + C::K_OFF;
  uint8_t* vs = smem + C::V_OFF;
  uint8_t* ps = smem + C::P_OFF;
  float* ml = reinterpret_cast<float*>(smem + tail_off);
  // [128][HD + 4] after the S product (q and k are consumed); the padding
  // spreads the row-per-thread stores over the banks
  constexpr int OLD = HD + 4;
  float* opart = reinterpret_cast<float*>(qs);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + tail_off + AT_ROWS * 8);
  uint64_t* kv_full = bars;       // K and V chunk landed (TMA)
  uint64_t* s_done = bars + 1;    // S product done
  uint64_t* o_done = bars + 2;    // O product done
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 3);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3) + 1;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // thread = (row, quarter): warps w and w + 4, w + 8, w + 12 share TMEM lanes
  // 32 (w % 4) .., each takes a quarter of the row's keys or dimensions
  const int lq = warp & 3, qt = warp >> 2, r = lq * 32 + lane;
  const int rank = (int)cluster_rank();
  const bool suffix_rank = rank == AT_CLUSTER - 1;
  const int hpg = heads / kv_heads;
  const int nrows = beams * hpg;
  const int ug = blockIdx.z, u = ug / kv_heads, g = ug % kv_heads;
  const int rt0 = blockIdx.y * AT_ROWS;
  const int r0 = u * beams, rows_all = gridDim.z / kv_heads * beams;
  anc += (long)u * anc_user_stride;
  float* red = reinterpret_cast<float*>(smem + tail_off + AT_ROWS * 8 + 64);  // [4][128] per-quarter partials

  if (tid == 0) {
    mbar_init(smem_addr(kv_full), 1);
    mbar_init(smem_addr(s_done), 1);
    mbar_init(smem_addr(o_done), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch_desc(&kmap);
    tma_prefetch_desc(&vmap);
  }
  if (warp == 0) tmem_alloc(smem_addr(tmem_slot), C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t s_tmem = tmem, o_tmem = tmem + C::S_COLS;
  const uint32_t lane_base = (uint32_t)(lq * 32) << 16;
  int L = L_dev[u];  // copied in before the request's first kernel: read before the wait
  pdl_launch_dependents();
  pdl_wait();  // q, the suffix rows and the pair copies come from earlier kernels

  if (L < 1 || L > cap || L > AT_MAX_PREFIX) {  // no valid prefix: attend to the suffix only
    if (tid == 0 && rank == 0) atomicOr(status, RTR_DEV_BAD_LENGTH);
    L = 0;
  }
  const int key0 = rank * AT_KEYS;
  const int nk = suffix_rank ? 0 : (L - key0 < 0 ? 0 : (L - key0 < AT_KEYS ? L - key0 : AT_KEYS));

  float m = -INFINITY, l = 0.f;
  bool issued_s = false, issued_o = false;
  if (nk > 0) {
    if (tid == 0) {
      // K chunk: per 64-dim chunk c, [k_hi 64 keys; k_lo 64 keys]; V^T: [v_hi^T; v_lo^T]
      const uint32_t bar = smem_addr(kv_full);
      mbar_expect_tx(bar, C::K_BYTES + C::V_BYTES);
      const long kr = krow0 + (long)u * kuser + (long)g * pair_cap + key0;
      const long vr = vrow0 + (long)u * vuser + (long)g * HD;
#pragma unroll
      for (int c = 0; c < C::NC; ++c) {
        tma_load_2d(smem_addr(ks + c * 2 * AT_KEYS * 128), &kmap, c * 64, (int)kr, bar);
        tma_load_2d(smem_addr(ks + c * 2 * AT_KEYS * 128 + AT_KEYS * 128), &kmap, c * 64, (int)(kr + kplane), bar);
      }
      tma_load_2d(smem_addr(vs), &vmap, key0, (int)vr, bar);
      tma_load_2d(smem_addr(vs + HD * 128), &vmap, key0, (int)(vr + vplane), bar);
    }
    // the tile's q rows -> pair planes (A operand), zeros past the group's rows
    load_q_pairs<HD>(qs, q, [&](int rr) -> long {
      const int rh = rt0 + rr;
      return rh < nrows ? (long)(r0 + rh / hpg) * heads + g * hpg + rh % hpg : -1;
    });
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    if (tid == 32) {
      // S = q_hi.[k_hi; k_lo]^T + q_lo.k_hi^T over head_dim in steps of 16
      if (mbar_wait(smem_addr(kv_full), 0, abort_flag)) {
        tc_fence_after();
        constexpr uint32_t id_cat = idesc_f16(AT_ROWS, 2 * AT_KEYS), id_one = idesc_f16(AT_ROWS, AT_KEYS);
#pragma unroll
        for (int c = 0; c < C::NC; ++c) {
          const uint64_t qh = sw128_desc(smem_addr(qs + c * AT_ROWS * 128));
          const uint64_t ql = sw128_desc(smem_addr(qs + (C::NC + c) * AT_ROWS * 128));
          const uint64_t kk = sw128_desc(smem_addr(ks + c * 2 * AT_KEYS * 128));
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            mma_f16_ss(s_tmem, qh + 2 * k, kk + 2 * k, id_cat, (c | k) ? 1u : 0u);
            mma_f16_ss(s_tmem + AT_KEYS, ql + 2 * k, kk + 2 * k, id_one, 1u);
          }
        }
        mma_commit(smem_addr(s_done));
        issued_s = true;
      }
    }
    const bool s_ok = mbar_wait(smem_addr(s_done), 0, abort_flag);
    if (__syncthreads_or(!s_ok) == 0) {
      tc_fence_after();
      // softmax of row r over the chunk, keys 16 qt .. 16 qt + 15 in this
      // thread: s = 256 (hh + cross / 2048) * scale
      constexpr int KQ = AT_KEYS / 4;
      float sv[KQ];
      {
        uint32_t hh[16], cr[16];
        tmem_ld16(s_tmem + lane_base + qt * KQ, hh);
        tmem_ld16(s_tmem + lane_base + AT_KEYS + qt * KQ, cr);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < KQ; ++j) {
          const float raw = __uint_as_float(hh[j]) + __uint_as_float(cr[j]) * (1.0f / kPairLo);
          sv[j] = qt * KQ + j < nk ? raw * (kPairScale * kPairScale) * scale : -INFINITY;
        }
      }
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < KQ; ++j) mx = fmaxf(mx, sv[j]);
      red[qt * AT_ROWS + r] = mx;
      __syncthreads();
      m = fmaxf(fmaxf(red[r], red[AT_ROWS + r]), fmaxf(red[2 * AT_ROWS + r], red[3 * AT_ROWS + r]));
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < KQ; ++j) {
        sv[j] = __expf(sv[j] - m);  // the hardware exponential: ~2 ulp, the pair's own precision
        sum += sv[j];
      }
#pragma unroll
      for (int un = 0; un < KQ / 8; ++un) put_pairs8(ps, ps + AT_ROWS * 128, r, qt * (KQ / 8) + un, sv + un * 8, 1.0f);
      __syncthreads();  // every max is read before the sums reuse the array
      red[qt * AT_ROWS + r] = sum;
      fence_proxy_async();
      tc_fence_before();
      __syncthreads();
      l = (red[r] + red[AT_ROWS + r]) + (red[2 * AT_ROWS + r] + red[3 * AT_ROWS + r]);
      if (tid == 32) {
        // O = p_hi.[v_hi; v_lo] + p_lo.v_hi over the chunk's keys in steps of 16
        tc_fence_after();
        constexpr uint32_t id_cat = idesc_f16(AT_ROWS, 2 * HD), id_one = idesc_f16(AT_ROWS, HD);
        const uint64_t ph = sw128_desc(smem_addr(ps)), pl = sw128_desc(smem_addr(ps + AT_ROWS * 128));
        const uint64_t vv = sw128_desc(smem_addr(vs));
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          mma_f16_ss(o_tmem, ph + 2 * k, vv + 2 * k, id_cat, k ? 1u : 0u);
          mma_f16_ss(o_tmem + HD, pl + 2 * k, vv + 2 * k, id_one, 1u);
        }
        mma_commit(smem_addr(o_done));
        issued_o = true;
      }
      const bool o_ok = mbar_wait(smem_addr(o_done), 0, abort_flag);
      if (__syncthreads_or(!o_ok) == 0) {
        tc_fence_after();
        // partial O of row r (unnormalised), dimensions qt HD / 4 ..: 16 (hh + cross / 2048)
        constexpr int DQ = HD / 4;
#pragma unroll
        for (int cb = 0; cb < DQ; cb += 16) {
          uint32_t hh[16], cr[16];
          tmem_ld16(o_tmem + lane_base + qt * DQ + cb, hh);
          tmem_ld16(o_tmem + lane_base + HD + qt * DQ + cb, cr);
          tmem_ld_wait();
          float* orow = opart + r * OLD + qt * DQ + cb;
#pragma unroll
          for (int j = 0; j < 16; j += 4) {
            float4 o4;
            o4.x = (__uint_as_float(hh[j]) + __uint_as_float(cr[j]) * (1.0f / kPairLo)) * kPairScale;
            o4.y = (__uint_as_float(hh[j + 1]) + __uint_as_float(cr[j + 1]) * (1.0f / kPairLo)) * kPairScale;
            o4.z = (__uint_as_float(hh[j + 2]) + __uint_as_float(cr[j + 2]) * (1.0f / kPairLo)) * kPairScale;
            o4.w = (__uint_as_float(hh[j + 3]) + __uint_as_float(cr[j + 3]) * (1.0f / kPairLo)) * kPairScale;
            *reinterpret_cast<float4*>(orow + j) = o4;
          }
        }
      }
    }
    if (*abort_flag) {
      // a wait ran out: record it; issued copies and products finish before the memory goes away
      if (tid == 0) {
        atomicOr(status, RTR_DEV_TIMEOUT);
        mbar_drain(smem_addr(kv_full), 0);
      }
      if (tid == 32) {
        if (issued_s) mbar_drain(smem_addr(s_done), 0);
        if (issued_o) mbar_drain(smem_addr(o_done), 0);
      }
      m = -INFINITY;
      l = 0.f;
    }
  } else if (suffix_rank) {
    // every row's t suffix keys of its beam on the FMA pipe, from q rows and
    // the beams' K / V rows staged in shared memory (rows padded to HD + 4
    // floats so the float4 reads of consecutive rows spread over the banks)
    constexpr int QLD = HD + 4;
    const int bfirst = rt0 / hpg, nb = at_tile_beams(hpg);
    float* sq = reinterpret_cast<float*>(smem);   // [128][QLD]
    float* sk = sq + AT_ROWS * QLD;               // [4][nb][QLD]
    float* sv = sk + 4 * nb * QLD;
    int* srows = reinterpret_cast<int*>(red + 4 * AT_ROWS);  // [4][nb <= 80] K / V row of (slot, beam)
    // q rows first: they do not wait for the ancestry rows
    for (int i = tid; i < AT_ROWS * (HD / 4); i += AT_THREADS) {
      const int rr = i / (HD / 4), d = (i % (HD / 4)) * 4, rh = rt0 + rr;
      const bool ok = rh < nrows;
      const int bb = ok ? rh / hpg : 0, hh = g * hpg + (ok ? rh % hpg : 0);
      cp_async16(sq + rr * QLD + d, q + ((long)(r0 + bb) * heads + hh) * HD + d, ok);
    }
    for (int i = tid; i < t * nb; i += AT_THREADS) {
      const int sl = i / nb, bb = bfirst + i % nb;
      int row = bb < beams ? bb : 0;
      if (bb < beams && sl != t - 1) {
        row = anc[bb * 4 + sl];
        if (row < 0 || row >= beams) {
          atomicOr(status, RTR_DEV_BAD_PARENT);
          row = bb;
        }
      }
      srows[i] = row;
    }
    __syncthreads();
    for (int i = tid; i < t * nb * (HD / 4); i += AT_THREADS) {
      const int sl = i / (nb * (HD / 4)), bi = (i / (HD / 4)) % nb, d = (i % (HD / 4)) * 4;
      const bool ok = bfirst + bi < beams;
      const long off = (((long)sl * rows_all + r0 + srows[sl * nb + bi]) * kv_heads + g) * HD + d;
      cp_async16(sk + (sl * nb + bi) * QLD + d, ksuf + off, ok);
      cp_async16(sv + (sl * nb + bi) * QLD + d, vsuf + off, ok);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    // thread (r, qt) takes a quarter of the dimensions of row r; the quarter
    // dot products meet in shared memory
    constexpr int DQ = HD / 4;
    const int rho = rt0 + r;
    const int bi = (rho < nrows ? rho / hpg : bfirst) - bfirst;
    float dots[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int d0 = qt * DQ; d0 < qt * DQ + DQ; d0 += 4) {
      const float4 qv = *reinterpret_cast<const float4*>(sq + r * QLD + d0);
#pragma unroll
      for (int sl = 0; sl < 4; ++sl) {
        if (sl < t) {
          const float4 kv = *reinterpret_cast<const float4*>(sk + (sl * nb + bi) * QLD + d0);
          dots[sl] = fmaf(qv.x, kv.x, fmaf(qv.y, kv.y, fmaf(qv.z, kv.z, fmaf(qv.w, kv.w, dots[sl]))));
        }
      }
    }
    float* sdot = red + 4 * AT_ROWS + 4 * 80;  // [4 quarters][4 slots][128]: past srows
#pragma unroll
    for (int sl = 0; sl < 4; ++sl) sdot[(qt * 4 + sl) * AT_ROWS + r] = dots[sl];
    __syncthreads();  // every q row is read and every partial dot written
    float pr[4];
#pragma unroll
    for (int sl = 0; sl < 4; ++sl) {
      const float dsum = (sdot[sl * AT_ROWS + r] + sdot[(4 + sl) * AT_ROWS + r]) +
                         (sdot[(8 + sl) * AT_ROWS + r] + sdot[(12 + sl) * AT_ROWS + r]);
      dots[sl] = sl < t ? dsum * scale : -INFINITY;
      m = fmaxf(m, dots[sl]);
    }
#pragma unroll
    for (int sl = 0; sl < 4; ++sl) {
      pr[sl] = sl < t ? __expf(dots[sl] - m) : 0.f;
      l += pr[sl];
    }
#pragma unroll
    for (int d0 = qt * DQ; d0 < qt * DQ + DQ; d0 += 4) {
      float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int sl = 0; sl < 4; ++sl) {
        if (sl < t) {
          const float4 vv = *reinterpret_cast<const float4*>(sv + (sl * nb + bi) * QLD + d0);
          o.x = fmaf(pr[sl], vv.x, o.x); o.y = fmaf(pr[sl], vv.y, o.y);
          o.z = fmaf(pr[sl], vv.z, o.z); o.w = fmaf(pr[sl], vv.w, o.w);
        }
      }
      *reinterpret_cast<float4*>(opart + r * OLD + d0) = o;  // row r's own q slots, read above
    }
  } else {
    // no key of the prefix falls to this rank
    for (int d0 = qt * (HD / 4); d0 < (qt + 1) * (HD / 4); d0 += 4)
      *reinterpret_cast<float4*>(opart + r * OLD + d0) = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (qt == 0) {
    ml[2 * r] = m;
    ml[2 * r + 1] = l;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
  cluster_barrier_tc();
  {
    // rank k finishes rows 16 k .. 16 k + 15: 32 threads per row, HD / 32 dims each
    constexpr int DPT = HD / 32;
    const int rr = 16 * rank + (tid >> 5), d0 = lane * DPT;
    const uint32_t ml_a = smem_addr(ml + 2 * rr), o_a = smem_addr(opart + rr * OLD + d0);
    // only ranks that hold keys are read: the first ceil(L / 64) and the suffix rank
    const int nfull = (L + AT_KEYS - 1) / AT_KEYS;
    float2 mine = make_float2(-INFINITY, 0.f);
    if (lane < AT_CLUSTER && (lane < nfull || lane == AT_CLUSTER - 1))
      mine = ld_cluster_f32x2_tc(cluster_map(ml_a, lane));
    float2 mlj[AT_CLUSTER];
    float oj[AT_CLUSTER][DPT];
#pragma unroll
    for (int j = 0; j < AT_CLUSTER; ++j) {
      mlj[j].x = __shfl_sync(0xffffffffu, mine.x, j);
      mlj[j].y = __shfl_sync(0xffffffffu, mine.y, j);
#pragma unroll
      for (int e = 0; e < DPT; ++e) oj[j][e] = 0.f;
      if (j < nfull || j == AT_CLUSTER - 1) {
        if constexpr (DPT == 4) {
          const float4 v = ld_cluster_f32x4(cluster_map(o_a, j));
          oj[j][0] = v.x; oj[j][1] = v.y; oj[j][2] = v.z; oj[j][3] = v.w;
        } else {
          const float2 v = ld_cluster_f32x2_tc(cluster_map(o_a, j));
          oj[j][0] = v.x; oj[j][1] = v.y;
        }
      }
    }
    float M = -INFINITY;
#pragma unroll
    for (int j = 0; j < AT_CLUSTER; ++j) M = fmaxf(M, mlj[j].x);
    float Ls = 0.f;
    float o[DPT];
#pragma unroll
    for (int e = 0; e < DPT; ++e) o[e] = 0.f;
#pragma unroll
    for (int j = 0; j < AT_CLUSTER; ++j) {  // rank order
      const float w = expf(mlj[j].x - M);   // 0 for a rank without keys (m = -inf)
      Ls = fmaf(w, mlj[j].y, Ls);
#pragma unroll
      for (int e = 0; e < DPT; ++e) o[e] = fmaf(w, oj[j][e], o[e]);
    }
    const int rh = rt0 + rr;
    if (rh < nrows) {
      const int bb = rh / hpg, hh = g * hpg + rh % hpg;
      const float inv = 1.0f / Ls;
      const long base = ((long)(r0 + bb) * heads + hh) * HD + d0;
      if constexpr (DPT == 4) {
        const float4 v = make_float4(o[0] * inv, o[1] * inv, o[2] * inv, o[3] * inv);
        *reinterpret_cast<float4*>(out + base) = v;
        if (out_big) store_split4(out_big, out_small, base, v, xfmt);
      } else {
#pragma unroll
        for (int e = 0; e < DPT; ++e) store_split(out, out_big, out_small, base + e, o[e] * inv, xfmt);
      }
    }
  }
  cluster_barrier_tc();  // no CTA leaves while a peer still reads its shared memory
}

// ------------------------------------------------------------------ prefill
// Causal prefill attention of one prompt on the tensor cores, from the same
// pair copies of K and V^T (written by the q/k/v epilogue of the same layer)
// and the same fp16-pair products as the decode kernel above.  A CTA owns 128
// rows of KV group g, row rho = token * hpg + head-in-group (the reference's
// folded layout, rapidtinyrec/folded_attention.py:16-31, applied to the
// prompt), and walks the keys 0 .. last token of its rows in 64-key chunks
// with an online softmax (the causal SDPA of the reference's prefill,
// rapidtinyrec/benchmark_inference.py:134):
//   K chunks double-buffered, loaded two chunks ahead; V^T single-buffered,
//   loaded while the next chunk's scores are computed;
//   S(c + 1) issued as soon as S(c) has landed (two S buffers in TMEM), so the
//   tensor core computes it while the threads run the softmax of chunk c;
//   O(c) = P(c).V(c) into TMEM, folded into the fp32 running output in
//   registers with the softmax rescale: o = o * exp(m_old - m_new) + O(c).
// Thread = (row, quarter): 16 keys of the chunk, HD / 4 output dimensions.
// Every wait is bounded; a wait that runs out sets RTR_DEV_TIMEOUT, the CTA
// drains what it issued and writes nothing.
template <int HD> struct PtCfg {
  static constexpr int NC = HD / 64;
  static constexpr int Q_BYTES = 2 * NC * AT_ROWS * 128;
  static constexpr int K_BYTES = NC * 2 * AT_KEYS * 128;  // one chunk
  static constexpr int V_BYTES = 2 * HD * 128;
  static constexpr int P_BYTES = 2 * AT_ROWS * 128;
  static constexpr int Q_OFF = 0, K_OFF = Q_BYTES, V_OFF = K_OFF + 2 * K_BYTES, P_OFF = V_OFF + V_BYTES;
  static constexpr int TAIL_OFF = P_OFF + P_BYTES;
  static constexpr int TAIL_BYTES = 64 + 2 * 4 * AT_ROWS * 4;  // barriers, [2][4][128] row partials
  static constexpr int SMEM = 1024 + TAIL_OFF + TAIL_BYTES;
  static constexpr int S_COLS = 2 * AT_KEYS;              // one S buffer: [hh | cross]
  static constexpr int O_COLS = 2 * HD;
  static constexpr int TMEM_COLS = 512;                   // 2 S buffers + O
  static_assert(2 * S_COLS + O_COLS <= TMEM_COLS, "tensor memory");
};

template <int HD>
__global__ void __launch_bounds__(AT_THREADS, 1) prefill_attn_tc_kernel(
    const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap, long krow, long kplane,
    long vrow, long vplane, int pair_cap, const float* __restrict__ q, float* __restrict__ out,
    float* __restrict__ out_big, float* __restrict__ out_small, int L, int heads, int kv_heads, float scale,
    uint32_t* __restrict__ status, int xfmt) {
  using C = PtCfg<HD>;
  extern __shared__ __align__(1024) uint8_t pt_smem_raw[];
  uint8_t* smem = pt_smem_raw + ((1024u - (smem_addr(pt_smem_raw) & 1023u)) & 1023u);
  uint8_t* qs = smem + C::Q_OFF;
  uint8_t* kb = smem + C::K_OFF;  // [2] chunks
  uint8_t* vs = smem + C::V_OFF;
  uint8_t* ps = smem + C::P_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::TAIL_OFF);
  uint64_t* k_full = bars;      // [2]
  uint64_t* v_full = bars + 2;
  uint64_t* s_done = bars + 3;  // [2]
  uint64_t* o_done = bars + 5;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 6);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 6) + 1;
  float* red = reinterpret_cast<float*>(smem + C::TAIL_OFF + 64);  // [2][4][128]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int lq = warp & 3, qt = warp >> 2, r = lq * 32 + lane;
  const int hpg = heads / kv_heads, nrows = L * hpg;
  const int g = blockIdx.y, rt0 = blockIdx.x * AT_ROWS;
  const int last_tok = min(L - 1, (rt0 + AT_ROWS - 1) / hpg);
  const int nch = last_tok / AT_KEYS + 1;
  const int rho = rt0 + r;
  const int tok = rho < nrows ? rho / hpg : 0;  // padding rows see key 0 only; never stored
  const long kr0 = krow + (long)g * pair_cap;  // the group's key 0 (hi plane)
  const long vr0 = vrow + (long)g * HD;        // the group's dimension 0 (V^T, hi plane)

  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_addr(&k_full[i]), 1);
      mbar_init(smem_addr(&s_done[i]), 1);
    }
    mbar_init(smem_addr(v_full), 1);
    mbar_init(smem_addr(o_done), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch_desc(&kmap);
    tma_prefetch_desc(&vmap);
  }
  if (warp == 0) tmem_alloc(smem_addr(tmem_slot), C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t o_tmem = tmem + 2 * C::S_COLS;
  const uint32_t lane_base = (uint32_t)(lq * 32) << 16;
  pdl_wait();  // q and the pair copies come from the q/k/v projection

  auto load_k = [&](int c) {
    const uint32_t bar = smem_addr(&k_full[c & 1]);
    uint8_t* dst = kb + (c & 1) * C::K_BYTES;
    mbar_expect_tx(bar, C::K_BYTES);
    const long row = kr0 + (long)c * AT_KEYS;
#pragma unroll
    for (int cc = 0; cc < C::NC; ++cc) {
      tma_load_2d(smem_addr(dst + cc * 2 * AT_KEYS * 128), &kmap, cc * 64, (int)row, bar);
      tma_load_2d(smem_addr(dst + cc * 2 * AT_KEYS * 128 + AT_KEYS * 128), &kmap, cc * 64, (int)(row + kplane), bar);
    }
  };
  auto load_v = [&](int c) {
    const uint32_t bar = smem_addr(v_full);
    mbar_expect_tx(bar, C::V_BYTES);
    tma_load_2d(smem_addr(vs), &vmap, c * AT_KEYS, (int)vr0, bar);
    tma_load_2d(smem_addr(vs + HD * 128), &vmap, c * AT_KEYS, (int)(vr0 + vplane), bar);
  };
  // S(c) = q_hi.[k_hi; k_lo]^T + q_lo.k_hi^T into S buffer c % 2
  auto issue_s = [&](int c) -> bool {
    if (!mbar_wait(smem_addr(&k_full[c & 1]), (c >> 1) & 1, abort_flag)) return false;
    tc_fence_after();
    constexpr uint32_t id_cat = idesc_f16(AT_ROWS, 2 * AT_KEYS), id_one = idesc_f16(AT_ROWS, AT_KEYS);
    const uint32_t st = tmem + (c & 1) * C::S_COLS;
    const uint8_t* kc = kb + (c & 1) * C::K_BYTES;
#pragma unroll
    for (int cc = 0; cc < C::NC; ++cc) {
      const uint64_t qh = sw128_desc(smem_addr(qs + cc * AT_ROWS * 128));
      const uint64_t ql = sw128_desc(smem_addr(qs + (C::NC + cc) * AT_ROWS * 128));
      const uint64_t kk = sw128_desc(smem_addr(kc + cc * 2 * AT_KEYS * 128));
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        mma_f16_ss(st, qh + 2 * k, kk + 2 * k, id_cat, (cc | k) ? 1u : 0u);
        mma_f16_ss(st + AT_KEYS, ql + 2 * k, kk + 2 * k, id_one, 1u);
      }
    }
    mma_commit(smem_addr(&s_done[c & 1]));
    return true;
  };

  int k_issued = 0, v_issued = 0, s_issued = 0, o_issued = 0;  // tid 0: copies; tid 32: products
  if (tid == 0) {
    load_k(0);
    k_issued = 1;
    if (nch > 1) {
      load_k(1);
      k_issued = 2;
    }
    load_v(0);
    v_issued = 1;
  }
  // the tile's q rows -> pair planes (A operand), zeros past the prompt's rows
  load_q_pairs<HD>(qs, q, [&](int rr) -> long {
    const int rh = rt0 + rr;
    return rh < nrows ? (long)(rh / hpg) * heads + g * hpg + rh % hpg : -1;
  });
  fence_proxy_async();
  tc_fence_before();
  __syncthreads();
  if (tid == 32 && issue_s(0)) s_issued = 1;
  pdl_launch_dependents();

  constexpr int KQ = AT_KEYS / 4, DQ = HD / 4;
  float o[DQ];
#pragma unroll
  for (int e = 0; e < DQ; ++e) o[e] = 0.f;
  float m = -INFINITY, l = 0.f;
  bool ok = true;
  for (int c = 0; c < nch; ++c) {
    ok = mbar_wait(smem_addr(&s_done[c & 1]), (c >> 1) & 1, abort_flag);
    if (__syncthreads_or(!ok)) {
      ok = false;
      break;
    }
    tc_fence_after();
    if (tid == 32 && c + 1 < nch && issue_s(c + 1)) s_issued = c + 2;  // overlaps this chunk's softmax
    if (tid == 0 && c + 2 < nch) {
      load_k(c + 2);  // S(c) has read its buffer
      k_issued = c + 3;
    }
    // softmax of row r over the chunk, keys 16 qt .. 16 qt + 15 in this thread
    float sv[KQ];
    {
      uint32_t hh[16], cr[16];
      const uint32_t st = tmem + (c & 1) * C::S_COLS + lane_base + qt * KQ;
      tmem_ld16(st, hh);
      tmem_ld16(st + AT_KEYS, cr);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < KQ; ++j) {
        const float raw = __uint_as_float(hh[j]) + __uint_as_float(cr[j]) * (1.0f / kPairLo);
        sv[j] = c * AT_KEYS + qt * KQ + j <= tok ? raw * (kPairScale * kPairScale) * scale : -INFINITY;
      }
    }
    float* rm = red + (c & 1) * 4 * AT_ROWS;  // alternating halves: one barrier per use
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < KQ; ++j) mx = fmaxf(mx, sv[j]);
    rm[qt * AT_ROWS + r] = mx;
    __syncthreads();
    const float mn = fmaxf(m, fmaxf(fmaxf(rm[r], rm[AT_ROWS + r]), fmaxf(rm[2 * AT_ROWS + r], rm[3 * AT_ROWS + r])));
    const float alpha = __expf(m - mn);  // 0 on the first chunk (m = -inf); mn is finite: key 0 is every row's
    m = mn;
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < KQ; ++j) {
      sv[j] = __expf(sv[j] - mn);
      sum += sv[j];
    }
#pragma unroll
    for (int un = 0; un < KQ / 8; ++un) put_pairs8(ps, ps + AT_ROWS * 128, r, qt * (KQ / 8) + un, sv + un * 8, 1.0f);
    float* rs = red + ((c + 1) & 1) * 4 * AT_ROWS;
    rs[qt * AT_ROWS + r] = sum;
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    l = l * alpha + ((rs[r] + rs[AT_ROWS + r]) + (rs[2 * AT_ROWS + r] + rs[3 * AT_ROWS + r]));
    if (tid == 32) {
      // O(c) = p_hi.[v_hi; v_lo] + p_lo.v_hi over the chunk's keys
      if (mbar_wait(smem_addr(v_full), c & 1, abort_flag)) {
        tc_fence_after();
        constexpr uint32_t id_cat = idesc_f16(AT_ROWS, 2 * HD), id_one = idesc_f16(AT_ROWS, HD);
        const uint64_t ph = sw128_desc(smem_addr(ps)), pl = sw128_desc(smem_addr(ps + AT_ROWS * 128));
        const uint64_t vv = sw128_desc(smem_addr(vs));
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          mma_f16_ss(o_tmem, ph + 2 * k, vv + 2 * k, id_cat, k ? 1u : 0u);
          mma_f16_ss(o_tmem + HD, pl + 2 * k, vv + 2 * k, id_one, 1u);
        }
        mma_commit(smem_addr(o_done));
        o_issued = c + 1;
      }
    }
    ok = mbar_wait(smem_addr(o_done), c & 1, abort_flag);
    if (__syncthreads_or(!ok)) {
      ok = false;
      break;
    }
    tc_fence_after();
    if (tid == 0 && c + 1 < nch) {
      load_v(c + 1);  // O(c) has read the buffer
      v_issued = c + 2;
    }
#pragma unroll
    for (int cb = 0; cb < DQ; cb += 16) {
      uint32_t hh[16], cr[16];
      tmem_ld16(o_tmem + lane_base + qt * DQ + cb, hh);
      tmem_ld16(o_tmem + lane_base + HD + qt * DQ + cb, cr);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 16; ++j)
        o[cb + j] = fmaf(o[cb + j], alpha,
                         (__uint_as_float(hh[j]) + __uint_as_float(cr[j]) * (1.0f / kPairLo)) * kPairScale);
    }
    tc_fence_before();
    __syncthreads();  // O(c) and S(c) are read: the next products may overwrite them
  }
  if (!ok) {
    // a wait ran out: record it; issued copies and products land before the memory goes away
    if (tid == 0) {
      atomicOr(status, RTR_DEV_TIMEOUT);
      for (int c = k_issued > 2 ? k_issued - 2 : 0; c < k_issued; ++c) mbar_drain(smem_addr(&k_full[c & 1]), (c >> 1) & 1);
      if (v_issued) mbar_drain(smem_addr(v_full), (v_issued - 1) & 1);
    }
    if (tid == 32) {
      for (int c = s_issued > 2 ? s_issued - 2 : 0; c < s_issued; ++c) mbar_drain(smem_addr(&s_done[c & 1]), (c >> 1) & 1);
      if (o_issued) mbar_drain(smem_addr(o_done), (o_issued - 1) & 1);
    }
  } else {
    // normalised rows through a shared tile ([128][HD + 4] over the free
    // operand buffers), then a warp stores whole rows (coalesced)
    constexpr int OLD = HD + 4;
    static_assert(AT_ROWS * OLD * 4 <= C::TAIL_OFF, "output tile fits in the operand buffers");
    float* ot = reinterpret_cast<float*>(smem);
    const float inv = 1.0f / l;
#pragma unroll
    for (int e = 0; e < DQ; e += 4)
      *reinterpret_cast<float4*>(ot + r * OLD + qt * DQ + e) =
          make_float4(o[e] * inv, o[e + 1] * inv, o[e + 2] * inv, o[e + 3] * inv);
    __syncthreads();
    for (int i = tid; i < AT_ROWS * (HD / 4); i += AT_THREADS) {
      const int rr = i / (HD / 4), c4 = i % (HD / 4), rh = rt0 + rr;
      if (rh >= nrows) continue;
      const long base = ((long)(rh / hpg) * heads + g * hpg + rh % hpg) * HD + 4 * c4;
      const float4 v = *reinterpret_cast<const float4*>(ot + rr * OLD + 4 * c4);
      *reinterpret_cast<float4*>(out + base) = v;
      if (out_big) store_split4(out_big, out_small, base, v, xfmt);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// The bf16 mode's prefill attention: the structure of prefill_attn_tc_kernel
// with bf16 operands, K read by TMA straight from the prefix arena and V from
// the transposed copy the bf16 q/k/v epilogue writes.  S = q.k^T is one bf16
// product (fp32 accumulation of exact bf16 products, as the FFMA kernel's fp32
// arithmetic on the same bf16 inputs); P is carried as a bf16 pair
// (p_hi + p_lo, 16 significant bits) into O = p_hi.v + p_lo.v; the output is
// rounded to bf16 once, as the FFMA kernel stores it.
template <int HD> struct PbCfg {
  static constexpr int NC = HD / 64;
  static constexpr int Q_BYTES = NC * AT_ROWS * 128;
  static constexpr int K_BYTES = NC * AT_KEYS * 128;  // one chunk
  static constexpr int V_BYTES = HD * 128;
  static constexpr int P_BYTES = 2 * AT_ROWS * 128;
  static constexpr int Q_OFF = 0, K_OFF = Q_BYTES, V_OFF = K_OFF + 2 * K_BYTES, P_OFF = V_OFF + V_BYTES;
  static constexpr int TAIL_OFF = P_OFF + P_BYTES;
  static constexpr int TAIL_BYTES = 64 + 2 * 4 * AT_ROWS * 4;
  static constexpr int SMEM = 1024 + TAIL_OFF + TAIL_BYTES;
  static constexpr int S_COLS = AT_KEYS;
  static constexpr int TMEM_COLS = 256;
  static_assert(2 * S_COLS + HD <= TMEM_COLS, "tensor memory");
  static_assert(AT_ROWS * (HD + 4) * 4 <= TAIL_OFF, "output tile fits in the operand buffers");
};

// Eight fp32 values as bf16 pairs (hi = bf16(x), lo = bf16(x - hi)) into unit
// u of row r of the hi and lo planes.
RTR_DEVICE void put_bf16_pairs8(uint8_t* hi_plane, uint8_t* lo_plane, int r, int u, const float* x) {
  __align__(16) __nv_bfloat16 hi[8];
  __align__(16) __nv_bfloat16 lo[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    hi[e] = __float2bfloat16_rn(x[e]);
    lo[e] = __float2bfloat16_rn(x[e] - __bfloat162float(hi[e]));
  }
  *reinterpret_cast<uint4*>(sw_unit(hi_plane, r, u)) = *reinterpret_cast<const uint4*>(hi);
  *reinterpret_cast<uint4*>(sw_unit(lo_plane, r, u)) = *reinterpret_cast<const uint4*>(lo);
}

template <int HD>
__global__ void __launch_bounds__(AT_THREADS, 1) prefill_attn_tc_bf16_kernel(
    const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap, long krow, int cap, long vrow,
    int pair_cap, const __nv_bfloat16* __restrict__ q, __nv_bfloat16* __restrict__ out, int L, int heads,
    int kv_heads, float scale, uint32_t* __restrict__ status) {
  using C = PbCfg<HD>;
  extern __shared__ __align__(1024) uint8_t pb_smem_raw[];
  uint8_t* smem = pb_smem_raw + ((1024u - (smem_addr(pb_smem_raw) & 1023u)) & 1023u);
  uint8_t* qs = smem + C::Q_OFF;
  uint8_t* kb = smem + C::K_OFF;
  uint8_t* vs = smem + C::V_OFF;
  uint8_t* ps = smem + C::P_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::TAIL_OFF);
  uint64_t* k_full = bars;      // [2]
  uint64_t* v_full = bars + 2;
  uint64_t* s_done = bars + 3;  // [2]
  uint64_t* o_done = bars + 5;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 6);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 6) + 1;
  float* red = reinterpret_cast<float*>(smem + C::TAIL_OFF + 64);  // [2][4][128]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int lq = warp & 3, qt = warp >> 2, r = lq * 32 + lane;
  const int hpg = heads / kv_heads, nrows = L * hpg;
  const int g = blockIdx.y, rt0 = blockIdx.x * AT_ROWS;
  const int last_tok = min(L - 1, (rt0 + AT_ROWS - 1) / hpg);
  const int nch = last_tok / AT_KEYS + 1;
  const int rho = rt0 + r;
  const int tok = rho < nrows ? rho / hpg : 0;  // padding rows see key 0 only; never stored
  const long kr0 = krow + (long)g * cap;        // the group's key 0 in the arena's K plane
  const long vr0 = vrow + (long)g * HD;         // the group's dimension 0 in the V^T copy

  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_addr(&k_full[i]), 1);
      mbar_init(smem_addr(&s_done[i]), 1);
    }
    mbar_init(smem_addr(v_full), 1);
    mbar_init(smem_addr(o_done), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch_desc(&kmap);
    tma_prefetch_desc(&vmap);
  }
  if (warp == 0) tmem_alloc(smem_addr(tmem_slot), C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t o_tmem = tmem + 2 * C::S_COLS;
  const uint32_t lane_base = (uint32_t)(lq * 32) << 16;
  pdl_wait();  // q, the arena rows and the V^T copy come from the q/k/v projection

  auto load_k = [&](int c) {
    const uint32_t bar = smem_addr(&k_full[c & 1]);
    uint8_t* dst = kb + (c & 1) * C::K_BYTES;
    mbar_expect_tx(bar, C::K_BYTES);
#pragma unroll
    for (int cc = 0; cc < C::NC; ++cc)
      tma_load_2d(smem_addr(dst + cc * AT_KEYS * 128), &kmap, cc * 64, (int)(kr0 + (long)c * AT_KEYS), bar);
  };
  auto load_v = [&](int c) {
    const uint32_t bar = smem_addr(v_full);
    mbar_expect_tx(bar, C::V_BYTES);
    tma_load_2d(smem_addr(vs), &vmap, c * AT_KEYS, (int)vr0, bar);
  };
  auto issue_s = [&](int c) -> bool {
    if (!mbar_wait(smem_addr(&k_full[c & 1]), (c >> 1) & 1, abort_flag)) return false;
    tc_fence_after();
    constexpr uint32_t id = idesc_bf16(AT_ROWS, AT_KEYS);
    const uint32_t st = tmem + (c & 1) * C::S_COLS;
    const uint8_t* kc = kb + (c & 1) * C::K_BYTES;
#pragma unroll
    for (int cc = 0; cc < C::NC; ++cc) {
      const uint64_t qd = sw128_desc(smem_addr(qs + cc * AT_ROWS * 128));
      const uint64_t kd = sw128_desc(smem_addr(kc + cc * AT_KEYS * 128));
#pragma unroll
      for (int k = 0; k < 4; ++k) mma_f16_ss(st, qd + 2 * k, kd + 2 * k, id, (cc | k) ? 1u : 0u);
    }
    mma_commit(smem_addr(&s_done[c & 1]));
    return true;
  };

  int k_issued = 0, v_issued = 0, s_issued = 0, o_issued = 0;
  if (tid == 0) {
    load_k(0);
    k_issued = 1;
    if (nch > 1) {
      load_k(1);
      k_issued = 2;
    }
    load_v(0);
    v_issued = 1;
  }
  {
    // the tile's q rows (bf16) -> the A operand, zeros past the prompt's rows:
    // every 16-byte load in flight before any store
    constexpr int UPR = HD / 8, PER = AT_ROWS * UPR / AT_THREADS;
    static_assert(AT_ROWS * UPR % AT_THREADS == 0, "whole units per thread");
    uint4 v[PER];
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int i = tid + k * AT_THREADS, rr = i / UPR, u8 = i % UPR, rh = rt0 + rr;
      v[k] = rh < nrows ? *reinterpret_cast<const uint4*>(q + ((long)(rh / hpg) * heads + g * hpg + rh % hpg) * HD + 8 * u8)
                        : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int i = tid + k * AT_THREADS, rr = i / UPR, u8 = i % UPR;
      *reinterpret_cast<uint4*>(sw_unit(qs + (u8 >> 3) * AT_ROWS * 128, rr, u8 & 7)) = v[k];
    }
  }
  fence_proxy_async();
  tc_fence_before();
  __syncthreads();
  if (tid == 32 && issue_s(0)) s_issued = 1;
  pdl_launch_dependents();

  constexpr int KQ = AT_KEYS / 4, DQ = HD / 4;
  float o[DQ];
#pragma unroll
  for (int e = 0; e < DQ; ++e) o[e] = 0.f;
  float m = -INFINITY, l = 0.f;
  bool ok = true;
  for (int c = 0; c < nch; ++c) {
    ok = mbar_wait(smem_addr(&s_done[c & 1]), (c >> 1) & 1, abort_flag);
    if (__syncthreads_or(!ok)) {
      ok = false;
      break;
    }
    tc_fence_after();
    if (tid == 32 && c + 1 < nch && issue_s(c + 1)) s_issued = c + 2;
    if (tid == 0 && c + 2 < nch) {
      load_k(c + 2);
      k_issued = c + 3;
    }
    float sv[KQ];
    {
      uint32_t sr[16];
      tmem_ld16(tmem + (c & 1) * C::S_COLS + lane_base + qt * KQ, sr);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < KQ; ++j)
        sv[j] = c * AT_KEYS + qt * KQ + j <= tok ? __uint_as_float(sr[j]) * scale : -INFINITY;
    }
    float* rm = red + (c & 1) * 4 * AT_ROWS;
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < KQ; ++j) mx = fmaxf(mx, sv[j]);
    rm[qt * AT_ROWS + r] = mx;
    __syncthreads();
    const float mn = fmaxf(m, fmaxf(fmaxf(rm[r], rm[AT_ROWS + r]), fmaxf(rm[2 * AT_ROWS + r], rm[3 * AT_ROWS + r])));
    const float alpha = __expf(m - mn);
    m = mn;
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < KQ; ++j) {
      sv[j] = __expf(sv[j] - mn);
      sum += sv[j];
    }
#pragma unroll
    for (int un = 0; un < KQ / 8; ++un) put_bf16_pairs8(ps, ps + AT_ROWS * 128, r, qt * (KQ / 8) + un, sv + un * 8);
    float* rs = red + ((c + 1) & 1) * 4 * AT_ROWS;
    rs[qt * AT_ROWS + r] = sum;
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    l = l * alpha + ((rs[r] + rs[AT_ROWS + r]) + (rs[2 * AT_ROWS + r] + rs[3 * AT_ROWS + r]));
    if (tid == 32) {
      if (mbar_wait(smem_addr(v_full), c & 1, abort_flag)) {
        tc_fence_after();
        constexpr uint32_t id = idesc_bf16(AT_ROWS, HD);
        const uint64_t ph = sw128_desc(smem_addr(ps)), pl = sw128_desc(smem_addr(ps + AT_ROWS * 128));
        const uint64_t vv = sw128_desc(smem_addr(vs));
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          mma_f16_ss(o_tmem, ph + 2 * k, vv + 2 * k, id, k ? 1u : 0u);
          mma_f16_ss(o_tmem, pl + 2 * k, vv + 2 * k, id, 1u);
        }
        mma_commit(smem_addr(o_done));
        o_issued = c + 1;
      }
    }
    ok = mbar_wait(smem_addr(o_done), c & 1, abort_flag);
    if (__syncthreads_or(!ok)) {
      ok = false;
      break;
    }
    tc_fence_after();
    if (tid == 0 && c + 1 < nch) {
      load_v(c + 1);
      v_issued = c + 2;
    }
#pragma unroll
    for (int cb = 0; cb < DQ; cb += 16) {
      uint32_t ov[16];
      tmem_ld16(o_tmem + lane_base + qt * DQ + cb, ov);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 16; ++j) o[cb + j] = fmaf(o[cb + j], alpha, __uint_as_float(ov[j]));
    }
    tc_fence_before();
    __syncthreads();
  }
  if (!ok) {
    if (tid == 0) {
      atomicOr(status, RTR_DEV_TIMEOUT);
      for (int c = k_issued > 2 ? k_issued - 2 : 0; c < k_issued; ++c) mbar_drain(smem_addr(&k_full[c & 1]), (c >> 1) & 1);
      if (v_issued) mbar_drain(smem_addr(v_full), (v_issued - 1) & 1);
    }
    if (tid == 32) {
      for (int c = s_issued > 2 ? s_issued - 2 : 0; c < s_issued; ++c) mbar_drain(smem_addr(&s_done[c & 1]), (c >> 1) & 1);
      if (o_issued) mbar_drain(smem_addr(o_done), (o_issued - 1) & 1);
    }
  } else {
    constexpr int OLD = HD + 4;
    float* ot = reinterpret_cast<float*>(smem);
    const float inv = 1.0f / l;
#pragma unroll
    for (int e = 0; e < DQ; e += 4)
      *reinterpret_cast<float4*>(ot + r * OLD + qt * DQ + e) =
          make_float4(o[e] * inv, o[e + 1] * inv, o[e + 2] * inv, o[e + 3] * inv);
    __syncthreads();
    for (int i = tid; i < AT_ROWS * (HD / 4); i += AT_THREADS) {
      const int rr = i / (HD / 4), c4 = i % (HD / 4), rh = rt0 + rr;
      if (rh >= nrows) continue;
      const float4 v = *reinterpret_cast<const float4*>(ot + rr * OLD + 4 * c4);
      const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
      uint2 u;
      u.x = *reinterpret_cast<const uint32_t*>(&a);
      u.y = *reinterpret_cast<const uint32_t*>(&b);
      *reinterpret_cast<uint2*>(out + ((long)(rh / hpg) * heads + g * hpg + rh % hpg) * HD + 4 * c4) = u;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// The bf16 mode's decode attention on the tensor cores, for long prefixes
// too: the cluster layout of decode_attn_tc_kernel (rows = a KV group's
// (beam, head) pairs, 128 to a tile; ranks 0..6 the prefix, rank 7 the beams'
// suffix keys on the FMA pipe; the partial (m, l, O) of the 8 ranks combined
// through distributed shared memory in rank order), with every prefix rank
// walking chunks rank, rank + 7, rank + 14, .. with an online softmax, so
// prompts of any length the arena holds are served.  K comes by TMA straight
// from the bf16 prefix arena, V from the transposed copy of the prefill; S is
// one bf16 product, P a bf16 pair, the output rounded to bf16 once.
template <int HD> struct DbCfg {
  static constexpr int NC = HD / 64;
  static constexpr int Q_BYTES = NC * AT_ROWS * 128;
  static constexpr int K_BYTES = NC * AT_KEYS * 128;
  static constexpr int V_BYTES = HD * 128;
  static constexpr int P_BYTES = 2 * AT_ROWS * 128;
  static constexpr int Q_OFF = 0, K_OFF = Q_BYTES, V_OFF = K_OFF + 2 * K_BYTES, P_OFF = V_OFF + V_BYTES;
  static constexpr int PRE_BYTES = P_OFF + P_BYTES;
  static constexpr int OLD = HD + 4;                     // partial O rows (fp32), over Q / K / V
  static constexpr int SLD = HD + 8;                     // suffix staging rows (bf16)
  static constexpr int S_COLS = AT_KEYS;
  static constexpr int TMEM_COLS = 256;
  // (m, l) per row, barriers, [2][4][128] row partials, [4][80] suffix rows, [16][128] partial dots
  static constexpr int TAIL_BYTES = AT_ROWS * 8 + 64 + (2 * 4 * AT_ROWS + 4 * 80 + 16 * AT_ROWS) * 4;
  static_assert(AT_ROWS * OLD * 4 <= P_OFF, "the partial O tile fits over q, k and v");
  static_assert(2 * S_COLS + HD <= TMEM_COLS, "tensor memory");
};
template <int HD> constexpr int db_suffix_bytes(int hpg) {
  return (AT_ROWS * DbCfg<HD>::SLD + 2 * 4 * at_tile_beams(hpg) * DbCfg<HD>::SLD) * 2;
}
template <int HD> constexpr int db_tail_off(int hpg) {
  const int a = DbCfg<HD>::PRE_BYTES, b = db_suffix_bytes<HD>(hpg);
  return ((a > b ? a : b) + 1023) / 1024 * 1024;
}

RTR_DEVICE float4 bf4_to_f4(uint2 u) {
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

template <int HD>
__global__ void __cluster_dims__(AT_CLUSTER, 1, 1) __launch_bounds__(AT_THREADS, 1) decode_attn_tc_bf16_kernel(
    const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap, long krow, long kuser,
    long vrow, long vuser, int cap, const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ ksuf,
    const __nv_bfloat16* __restrict__ vsuf, const int32_t* __restrict__ anc, const int32_t* __restrict__ L_dev,
    __nv_bfloat16* __restrict__ out, int beams, int heads, int kv_heads, int t, float scale,
    uint32_t* __restrict__ status, int anc_user_stride, int tail_off) {
  using C = DbCfg<HD>;
  constexpr int OLD = C::OLD, SLD = C::SLD;
  extern __shared__ __align__(1024) uint8_t db_smem_raw[];
  uint8_t* smem = db_smem_raw + ((1024u - (smem_addr(db_smem_raw) & 1023u)) & 1023u);
  uint8_t* qs = smem + C::Q_OFF;
  uint8_t* kb = smem + C::K_OFF;  // [2] chunks
  uint8_t* vs = smem + C::V_OFF;
  uint8_t* ps = smem + C::P_OFF;
  float* opart = reinterpret_cast<float*>(smem);  // [128][OLD] after the last product
  float* ml = reinterpret_cast<float*>(smem + tail_off);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + tail_off + AT_ROWS * 8);
  uint64_t* k_full = bars;      // [2]
  uint64_t* v_full = bars + 2;
  uint64_t* s_done = bars + 3;  // [2]
  uint64_t* o_done = bars + 5;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 6);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 6) + 1;
  float* red = reinterpret_cast<float*>(smem + tail_off + AT_ROWS * 8 + 64);  // [2][4][128]
  int* srows = reinterpret_cast<int*>(red + 2 * 4 * AT_ROWS);                // [4][nb <= 80]
  float* sdot = reinterpret_cast<float*>(srows + 4 * 80);                    // [16][128]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int lq = warp & 3, qt = warp >> 2, r = lq * 32 + lane;
  const int rank = (int)cluster_rank();
  const bool suffix_rank = rank == AT_CLUSTER - 1;
  const int hpg = heads / kv_heads;
  const int nrows = beams * hpg;
  const int ug = blockIdx.z, u = ug / kv_heads, g = ug % kv_heads;
  const int rt0 = blockIdx.y * AT_ROWS;
  const int r0 = u * beams, rows_all = gridDim.z / kv_heads * beams;
  anc += (long)u * anc_user_stride;
  const long kr0 = krow + (long)u * kuser + (long)g * cap;
  const long vr0 = vrow + (long)u * vuser + (long)g * HD;

  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_addr(&k_full[i]), 1);
      mbar_init(smem_addr(&s_done[i]), 1);
    }
    mbar_init(smem_addr(v_full), 1);
    mbar_init(smem_addr(o_done), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch_desc(&kmap);
    tma_prefetch_desc(&vmap);
  }
  if (warp == 0) tmem_alloc(smem_addr(tmem_slot), C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t o_tmem = tmem + 2 * C::S_COLS;
  const uint32_t lane_base = (uint32_t)(lq * 32) << 16;
  int L = L_dev[u];  // copied in before the request's first kernel: read before the wait
  pdl_launch_dependents();
  pdl_wait();  // q, the suffix rows and the prefix copies come from earlier kernels

  if (L < 1 || L > cap) {  // no valid prefix: attend to the suffix only
    if (tid == 0 && rank == 0) atomicOr(status, RTR_DEV_BAD_LENGTH);
    L = 0;
  }
  const int nch_all = (L + AT_KEYS - 1) / AT_KEYS;
  const int nmine = suffix_rank || rank >= nch_all ? 0 : (nch_all - rank + AT_CLUSTER - 2) / (AT_CLUSTER - 1);

  float m = -INFINITY, l = 0.f;
  if (nmine > 0) {
    auto chunk = [&](int i) { return rank + i * (AT_CLUSTER - 1); };
    auto load_k = [&](int i) {
      const uint32_t bar = smem_addr(&k_full[i & 1]);
      uint8_t* dst = kb + (i & 1) * C::K_BYTES;
      mbar_expect_tx(bar, C::K_BYTES);
#pragma unroll
      for (int cc = 0; cc < C::NC; ++cc)
        tma_load_2d(smem_addr(dst + cc * AT_KEYS * 128), &kmap, cc * 64, (int)(kr0 + (long)chunk(i) * AT_KEYS), bar);
    };
    auto load_v = [&](int i) {
      const uint32_t bar = smem_addr(v_full);
      mbar_expect_tx(bar, C::V_BYTES);
      tma_load_2d(smem_addr(vs), &vmap, chunk(i) * AT_KEYS, (int)vr0, bar);
    };
    auto issue_s = [&](int i) -> bool {
      if (!mbar_wait(smem_addr(&k_full[i & 1]), (i >> 1) & 1, abort_flag)) return false;
      tc_fence_after();
      constexpr uint32_t id = idesc_bf16(AT_ROWS, AT_KEYS);
      const uint32_t st = tmem + (i & 1) * C::S_COLS;
      const uint8_t* kc = kb + (i & 1) * C::K_BYTES;
#pragma unroll
      for (int cc = 0; cc < C::NC; ++cc) {
        const uint64_t qd = sw128_desc(smem_addr(qs + cc * AT_ROWS * 128));
        const uint64_t kd = sw128_desc(smem_addr(kc + cc * AT_KEYS * 128));
#pragma unroll
        for (int k = 0; k < 4; ++k) mma_f16_ss(st, qd + 2 * k, kd + 2 * k, id, (cc | k) ? 1u : 0u);
      }
      mma_commit(smem_addr(&s_done[i & 1]));
      return true;
    };
    int k_issued = 0, v_issued = 0, s_issued = 0, o_issued = 0;
    if (tid == 0) {
      load_k(0);
      k_issued = 1;
      if (nmine > 1) {
        load_k(1);
        k_issued = 2;
      }
      load_v(0);
      v_issued = 1;
    }
    {
      // the tile's q rows (bf16) -> the A operand, zeros past the group's rows
      constexpr int UPR = HD / 8, PER = AT_ROWS * UPR / AT_THREADS;
      uint4 v[PER];
#pragma unroll
      for (int k = 0; k < PER; ++k) {
        const int i = tid + k * AT_THREADS, rr = i / UPR, u8 = i % UPR, rh = rt0 + rr;
        v[k] = rh < nrows ? *reinterpret_cast<const uint4*>(q + ((long)(r0 + rh / hpg) * heads + g * hpg + rh % hpg) * HD + 8 * u8)
                          : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int k = 0; k < PER; ++k) {
        const int i = tid + k * AT_THREADS, rr = i / UPR, u8 = i % UPR;
        *reinterpret_cast<uint4*>(sw_unit(qs + (u8 >> 3) * AT_ROWS * 128, rr, u8 & 7)) = v[k];
      }
    }
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    if (tid == 32 && issue_s(0)) s_issued = 1;

    constexpr int KQ = AT_KEYS / 4, DQ = HD / 4;
    float o[DQ];
#pragma unroll
    for (int e = 0; e < DQ; ++e) o[e] = 0.f;
    bool ok = true;
    for (int i = 0; i < nmine; ++i) {
      ok = mbar_wait(smem_addr(&s_done[i & 1]), (i >> 1) & 1, abort_flag);
      if (__syncthreads_or(!ok)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (tid == 32 && i + 1 < nmine && issue_s(i + 1)) s_issued = i + 2;
      if (tid == 0 && i + 2 < nmine) {
        load_k(i + 2);
        k_issued = i + 3;
      }
      float sv[KQ];
      {
        uint32_t sr[16];
        tmem_ld16(tmem + (i & 1) * C::S_COLS + lane_base + qt * KQ, sr);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < KQ; ++j)
          sv[j] = chunk(i) * AT_KEYS + qt * KQ + j < L ? __uint_as_float(sr[j]) * scale : -INFINITY;
      }
      float* rm = red + (i & 1) * 4 * AT_ROWS;
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < KQ; ++j) mx = fmaxf(mx, sv[j]);
      rm[qt * AT_ROWS + r] = mx;
      __syncthreads();
      // finite: the rank's first chunk holds key rank * 64 < L for every row
      const float mn = fmaxf(m, fmaxf(fmaxf(rm[r], rm[AT_ROWS + r]), fmaxf(rm[2 * AT_ROWS + r], rm[3 * AT_ROWS + r])));
      const float alpha = __expf(m - mn);
      m = mn;
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < KQ; ++j) {
        sv[j] = __expf(sv[j] - mn);
        sum += sv[j];
      }
#pragma unroll
      for (int un = 0; un < KQ / 8; ++un) put_bf16_pairs8(ps, ps + AT_ROWS * 128, r, qt * (KQ / 8) + un, sv + un * 8);
      float* rs = red + ((i + 1) & 1) * 4 * AT_ROWS;
      rs[qt * AT_ROWS + r] = sum;
      fence_proxy_async();
      tc_fence_before();
      __syncthreads();
      l = l * alpha + ((rs[r] + rs[AT_ROWS + r]) + (rs[2 * AT_ROWS + r] + rs[3 * AT_ROWS + r]));
      if (tid == 32) {
        if (mbar_wait(smem_addr(v_full), i & 1, abort_flag)) {
          tc_fence_after();
          constexpr uint32_t id = idesc_bf16(AT_ROWS, HD);
          const uint64_t ph = sw128_desc(smem_addr(ps)), pl = sw128_desc(smem_addr(ps + AT_ROWS * 128));
          const uint64_t vv = sw128_desc(smem_addr(vs));
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            mma_f16_ss(o_tmem, ph + 2 * k, vv + 2 * k, id, k ? 1u : 0u);
            mma_f16_ss(o_tmem, pl + 2 * k, vv + 2 * k, id, 1u);
          }
          mma_commit(smem_addr(o_done));
          o_issued = i + 1;
        }
      }
      ok = mbar_wait(smem_addr(o_done), i & 1, abort_flag);
      if (__syncthreads_or(!ok)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (tid == 0 && i + 1 < nmine) {
        load_v(i + 1);
        v_issued = i + 2;
      }
#pragma unroll
      for (int cb = 0; cb < DQ; cb += 16) {
        uint32_t ov[16];
        tmem_ld16(o_tmem + lane_base + qt * DQ + cb, ov);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) o[cb + j] = fmaf(o[cb + j], alpha, __uint_as_float(ov[j]));
      }
      tc_fence_before();
      __syncthreads();  // S(i), O(i), the K / V buffers and q are read
    }
    if (!ok) {
      if (tid == 0) {
        atomicOr(status, RTR_DEV_TIMEOUT);
        for (int i = k_issued > 2 ? k_issued - 2 : 0; i < k_issued; ++i)
          mbar_drain(smem_addr(&k_full[i & 1]), (i >> 1) & 1);
        if (v_issued) mbar_drain(smem_addr(v_full), (v_issued - 1) & 1);
      }
      if (tid == 32) {
        for (int i = s_issued > 2 ? s_issued - 2 : 0; i < s_issued; ++i)
          mbar_drain(smem_addr(&s_done[i & 1]), (i >> 1) & 1);
        if (o_issued) mbar_drain(smem_addr(o_done), (o_issued - 1) & 1);
      }
      __syncthreads();
      m = -INFINITY;
      l = 0.f;
    } else {
#pragma unroll
      for (int e = 0; e < DQ; e += 4)
        *reinterpret_cast<float4*>(opart + r * OLD + qt * DQ + e) = make_float4(o[e], o[e + 1], o[e + 2], o[e + 3]);
    }
  } else if (suffix_rank) {
    // every row's t suffix keys of its beam on the FMA pipe, from bf16 q rows
    // and the beams' K / V rows staged in shared memory
    const int bfirst = rt0 / hpg, nb = at_tile_beams(hpg);
    __nv_bfloat16* sq = reinterpret_cast<__nv_bfloat16*>(smem);  // [128][SLD]
    __nv_bfloat16* sk = sq + AT_ROWS * SLD;                      // [4][nb][SLD]
    __nv_bfloat16* sv = sk + 4 * nb * SLD;
    for (int i = tid; i < AT_ROWS * (HD / 8); i += AT_THREADS) {
      const int rr = i / (HD / 8), d = (i % (HD / 8)) * 8, rh = rt0 + rr;
      const bool okr = rh < nrows;
      const int bb = okr ? rh / hpg : 0, hh = g * hpg + (okr ? rh % hpg : 0);
      cp_async16(sq + rr * SLD + d, q + ((long)(r0 + bb) * heads + hh) * HD + d, okr);
    }
    for (int i = tid; i < t * nb; i += AT_THREADS) {
      const int sl = i / nb, bb = bfirst + i % nb;
      int row = bb < beams ? bb : 0;
      if (bb < beams && sl != t - 1) {
        row = anc[bb * 4 + sl];
        if (row < 0 || row >= beams) {
          atomicOr(status, RTR_DEV_BAD_PARENT);
          row = bb;
        }
      }
      srows[i] = row;
    }
    __syncthreads();
    for (int i = tid; i < t * nb * (HD / 8); i += AT_THREADS) {
      const int sl = i / (nb * (HD / 8)), bi = (i / (HD / 8)) % nb, d = (i % (HD / 8)) * 8;
      const bool okb = bfirst + bi < beams;
      const long off = (((long)sl * rows_all + r0 + srows[sl * nb + bi]) * kv_heads + g) * HD + d;
      cp_async16(sk + (sl * nb + bi) * SLD + d, ksuf + off, okb);
      cp_async16(sv + (sl * nb + bi) * SLD + d, vsuf + off, okb);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    constexpr int DQ = HD / 4;
    const int rho = rt0 + r;
    const int bi = (rho < nrows ? rho / hpg : bfirst) - bfirst;
    float dots[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int d0 = qt * DQ; d0 < qt * DQ + DQ; d0 += 4) {
      const float4 qv = bf4_to_f4(*reinterpret_cast<const uint2*>(sq + r * SLD + d0));
#pragma unroll
      for (int sl = 0; sl < 4; ++sl) {
        if (sl < t) {
          const float4 kv = bf4_to_f4(*reinterpret_cast<const uint2*>(sk + (sl * nb + bi) * SLD + d0));
          dots[sl] = fmaf(qv.x, kv.x, fmaf(qv.y, kv.y, fmaf(qv.z, kv.z, fmaf(qv.w, kv.w, dots[sl]))));
        }
      }
    }
#pragma unroll
    for (int sl = 0; sl < 4; ++sl) sdot[(qt * 4 + sl) * AT_ROWS + r] = dots[sl];
    __syncthreads();
    float pr[4];
#pragma unroll
    for (int sl = 0; sl < 4; ++sl) {
      const float dsum = (sdot[sl * AT_ROWS + r] + sdot[(4 + sl) * AT_ROWS + r]) +
                         (sdot[(8 + sl) * AT_ROWS + r] + sdot[(12 + sl) * AT_ROWS + r]);
      dots[sl] = sl < t ? dsum * scale : -INFINITY;
      m = fmaxf(m, dots[sl]);
    }
#pragma unroll
    for (int sl = 0; sl < 4; ++sl) {
      pr[sl] = sl < t ? __expf(dots[sl] - m) : 0.f;
      l += pr[sl];
    }
    float4 ov[DQ / 4];
#pragma unroll
    for (int e = 0; e < DQ / 4; ++e) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int sl = 0; sl < 4; ++sl) {
        if (sl < t) {
          const float4 vv = bf4_to_f4(*reinterpret_cast<const uint2*>(sv + (sl * nb + bi) * SLD + qt * DQ + 4 * e));
          acc.x = fmaf(pr[sl], vv.x, acc.x); acc.y = fmaf(pr[sl], vv.y, acc.y);
          acc.z = fmaf(pr[sl], vv.z, acc.z); acc.w = fmaf(pr[sl], vv.w, acc.w);
        }
      }
      ov[e] = acc;
    }
    __syncthreads();  // the staged rows are read: opart overlays them
#pragma unroll
    for (int e = 0; e < DQ / 4; ++e) *reinterpret_cast<float4*>(opart + r * OLD + qt * DQ + 4 * e) = ov[e];
  }
  if (qt == 0) {
    ml[2 * r] = m;
    ml[2 * r + 1] = l;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
  cluster_barrier_tc();
  {
    // rank k finishes rows 16 k .. 16 k + 15: 32 threads per row, HD / 32 dims each
    constexpr int DPT = HD / 32;
    const int rr = 16 * rank + (tid >> 5), d0 = lane * DPT;
    const uint32_t ml_a = smem_addr(ml + 2 * rr), o_a = smem_addr(opart + rr * OLD + d0);
    const int nfull = nch_all < AT_CLUSTER - 1 ? nch_all : AT_CLUSTER - 1;  // prefix ranks holding keys
    float2 mine = make_float2(-INFINITY, 0.f);
    if (lane < AT_CLUSTER && (lane < nfull || lane == AT_CLUSTER - 1))
      mine = ld_cluster_f32x2_tc(cluster_map(ml_a, lane));
    float2 mlj[AT_CLUSTER];
    float oj[AT_CLUSTER][DPT];
#pragma unroll
    for (int j = 0; j < AT_CLUSTER; ++j) {
      mlj[j].x = __shfl_sync(0xffffffffu, mine.x, j);
      mlj[j].y = __shfl_sync(0xffffffffu, mine.y, j);
#pragma unroll
      for (int e = 0; e < DPT; ++e) oj[j][e] = 0.f;
      if ((j < nfull || j == AT_CLUSTER - 1) && mlj[j].y > 0.f) {
        if constexpr (DPT == 4) {
          const float4 v = ld_cluster_f32x4(cluster_map(o_a, j));
          oj[j][0] = v.x; oj[j][1] = v.y; oj[j][2] = v.z; oj[j][3] = v.w;
        } else {
          const float2 v = ld_cluster_f32x2_tc(cluster_map(o_a, j));
          oj[j][0] = v.x; oj[j][1] = v.y;
        }
      }
    }
    float M = -INFINITY;
#pragma unroll
    for (int j = 0; j < AT_CLUSTER; ++j) M = fmaxf(M, mlj[j].x);
    float Ls = 0.f;
    float o[DPT];
#pragma unroll
    for (int e = 0; e < DPT; ++e) o[e] = 0.f;
#pragma unroll
    for (int j = 0; j < AT_CLUSTER; ++j) {  // rank order
      const float w = mlj[j].y > 0.f ? expf(mlj[j].x - M) : 0.f;
      Ls = fmaf(w, mlj[j].y, Ls);
#pragma unroll
      for (int e = 0; e < DPT; ++e) o[e] = fmaf(w, oj[j][e], o[e]);
    }
    const int rh = rt0 + rr;
    if (rh < nrows) {
      const int bb = rh / hpg, hh = g * hpg + rh % hpg;
      const float inv = 1.0f / Ls;
      __nv_bfloat16* dst = out + ((long)(r0 + bb) * heads + hh) * HD + d0;
      if constexpr (DPT == 4) {
        const __nv_bfloat162 a = __floats2bfloat162_rn(o[0] * inv, o[1] * inv);
        const __nv_bfloat162 b = __floats2bfloat162_rn(o[2] * inv, o[3] * inv);
        uint2 w;
        w.x = *reinterpret_cast<const uint32_t*>(&a);
        w.y = *reinterpret_cast<const uint32_t*>(&b);
        *reinterpret_cast<uint2*>(dst) = w;
      } else {
        *reinterpret_cast<__nv_bfloat162*>(dst) = __floats2bfloat162_rn(o[0] * inv, o[1] * inv);
      }
    }
  }
  cluster_barrier_tc();  // no CTA leaves while a peer still reads its shared memory
}

// Largest dynamic shared memory a CTA may take (227 KB) minus the alignment slack.
constexpr int AT_SMEM_MAX = 227 * 1024 - 1024;

static int at_smem_bytes(int head_dim, int hpg) {
  const int off = head_dim == 128 ? at_tail_off<128>(hpg) : at_tail_off<64>(hpg);
  return off + (head_dim == 128 ? AtCfg<128>::TAIL_BYTES : AtCfg<64>::TAIL_BYTES);
}

bool attention_tc_supported(int heads, int kv_heads, int head_dim, int max_prefix) {
  return kv_heads >= 1 && heads % kv_heads == 0 && (head_dim == 64 || head_dim == 128) &&
         max_prefix <= AT_MAX_PREFIX && at_tile_beams(heads / kv_heads) <= 80 &&
         at_smem_bytes(head_dim, heads / kv_heads) <= AT_SMEM_MAX;
}

template <int HD>
static cudaError_t launch_tc(const AttnPairs& ap, const float* q, const float* ks, const float* vs,
                             const int32_t* anc, const int32_t* L_dev, int t, float* out, float* ob, float* os,
                             int beams, int cap, int heads, int kv_heads, float scale, uint32_t* status,
                             cudaStream_t stream, const DecodeUsers& du, int xfmt) {
  const int hpg = heads / kv_heads;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(AT_CLUSTER, (beams * hpg + AT_ROWS - 1) / AT_ROWS, du.users * kv_heads);
  cfg.blockDim = dim3(AT_THREADS);
  const int tail_off = at_tail_off<HD>(hpg);
  cfg.dynamicSmemBytes = 1024 + tail_off + AtCfg<HD>::TAIL_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_on(PDL_ATTN) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, decode_attn_tc_kernel<HD>, *reinterpret_cast<const CUtensorMap*>(&ap.kmap),
                            *reinterpret_cast<const CUtensorMap*>(&ap.vmap), ap.krow0, ap.kplane, ap.kuser, ap.vrow0,
                            ap.vplane, ap.vuser, ap.pair_cap, q, ks, vs, anc, L_dev, out, ob, os, beams, cap, heads,
                            kv_heads, t, scale, status, du.anc_user_stride, xfmt, tail_off);
}

cudaError_t attention_decode_tc(const AttnPairs& ap, const float* q, const float* k_suffix, const float* v_suffix,
                                const int32_t* anc, const int32_t* L_dev, int t, float* out, float* out_big,
                                float* out_small, int beams, int prefix_cap, int heads, int kv_heads, int head_dim,
                                float scale, uint32_t* status, cudaStream_t stream, const DecodeUsers& du, int xfmt) {
  if (t < 1 || t > 4 || beams > MAX_BEAMS || du.users < 1 ||
      !attention_tc_supported(heads, kv_heads, head_dim, prefix_cap))
    return cudaErrorInvalidValue;
  if (head_dim == 128)
    return launch_tc<128>(ap, q, k_suffix, v_suffix, anc, L_dev, t, out, out_big, out_small, beams, prefix_cap, heads,
                          kv_heads, scale, status, stream, du, xfmt);
  return launch_tc<64>(ap, q, k_suffix, v_suffix, anc, L_dev, t, out, out_big, out_small, beams, prefix_cap, heads,
                       kv_heads, scale, status, stream, du, xfmt);
}

bool attention_prefill_tc_supported(int heads, int kv_heads, int head_dim) {
  return kv_heads >= 1 && heads % kv_heads == 0 && (head_dim == 64 || head_dim == 128);
}

template <int HD>
static cudaError_t launch_prefill_tc(const AttnPairs& ap, int user, const float* q, float* out, float* ob, float* os,
                                     int L, int heads, int kv_heads, float scale, uint32_t* status, cudaStream_t stream,
                                     int xfmt) {
  const int hpg = heads / kv_heads;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((L * hpg + AT_ROWS - 1) / AT_ROWS, kv_heads);
  cfg.blockDim = dim3(AT_THREADS);
  cfg.dynamicSmemBytes = PtCfg<HD>::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_on(PDL_ATTN) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, prefill_attn_tc_kernel<HD>, *reinterpret_cast<const CUtensorMap*>(&ap.kmap),
                            *reinterpret_cast<const CUtensorMap*>(&ap.vmap), ap.krow0 + (long)user * ap.kuser,
                            ap.kplane, ap.vrow0 + (long)user * ap.vuser, ap.vplane, ap.pair_cap, q, out, ob, os, L,
                            heads, kv_heads, scale, status, xfmt);
}

cudaError_t attention_prefill_tc(const AttnPairs& ap, int user, const float* q, float* out, float* out_big,
                                 float* out_small, int L, int heads, int kv_heads, int head_dim, float scale,
                                 uint32_t* status, cudaStream_t stream, int xfmt) {
  if (L < 1 || L > ap.pair_cap || !attention_prefill_tc_supported(heads, kv_heads, head_dim))
    return cudaErrorInvalidValue;
  if (head_dim == 128)
    return launch_prefill_tc<128>(ap, user, q, out, out_big, out_small, L, heads, kv_heads, scale, status, stream,
                                  xfmt);
  return launch_prefill_tc<64>(ap, user, q, out, out_big, out_small, L, heads, kv_heads, scale, status, stream, xfmt);
}

template <int HD>
static cudaError_t launch_prefill_tc_bf16(const BfPrefillMaps& mp, int user, int layer, const void* q, void* out,
                                          int L, int heads, int kv_heads, int cap, float scale, uint32_t* status,
                                          cudaStream_t stream, int layers) {
  const int hpg = heads / kv_heads;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((L * hpg + AT_ROWS - 1) / AT_ROWS, kv_heads);
  cfg.blockDim = dim3(AT_THREADS);
  cfg.dynamicSmemBytes = PbCfg<HD>::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_on(PDL_ATTN) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const long ul = (long)user * layers + layer;
  const long krow = ul * 2 * kv_heads * cap;        // the arena's K plane of (user, layer)
  const long vrow = ul * kv_heads * HD;             // the V^T copy of (user, layer)
  return cudaLaunchKernelEx(&cfg, prefill_attn_tc_bf16_kernel<HD>, *reinterpret_cast<const CUtensorMap*>(&mp.kmap),
                            *reinterpret_cast<const CUtensorMap*>(&mp.vmap), krow, cap, vrow, mp.pair_cap,
                            static_cast<const __nv_bfloat16*>(q), static_cast<__nv_bfloat16*>(out), L, heads, kv_heads,
                            scale, status);
}

cudaError_t attention_prefill_tc_bf16(const BfPrefillMaps& mp, int user, int layer, int layers, const void* q,
                                      void* out, int L, int heads, int kv_heads, int head_dim, int cap, float scale,
                                      uint32_t* status, cudaStream_t stream) {
  if (L < 1 || L > cap || L > mp.pair_cap || !attention_prefill_tc_supported(heads, kv_heads, head_dim))
    return cudaErrorInvalidValue;
  if (head_dim == 128)
    return launch_prefill_tc_bf16<128>(mp, user, layer, q, out, L, heads, kv_heads, cap, scale, status, stream, layers);
  return launch_prefill_tc_bf16<64>(mp, user, layer, q, out, L, heads, kv_heads, cap, scale, status, stream, layers);
}

bool attention_decode_tc_bf16_supported(int heads, int kv_heads, int head_dim) {
  if (kv_heads < 1 || heads % kv_heads || (head_dim != 64 && head_dim != 128)) return false;
  const int hpg = heads / kv_heads;
  if (at_tile_beams(hpg) > 80) return false;
  const int off = head_dim == 128 ? db_tail_off<128>(hpg) : db_tail_off<64>(hpg);
  return off + (head_dim == 128 ? DbCfg<128>::TAIL_BYTES : DbCfg<64>::TAIL_BYTES) <= AT_SMEM_MAX;
}

template <int HD>
static cudaError_t launch_decode_tc_bf16(const BfPrefillMaps& mp, int layer, int layers, const void* q, const void* ks,
                                         const void* vs, const int32_t* anc, const int32_t* L_dev, int t, void* out,
                                         int beams, int cap, int heads, int kv_heads, float scale, uint32_t* status,
                                         cudaStream_t stream, const DecodeUsers& du) {
  const int hpg = heads / kv_heads;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(AT_CLUSTER, (beams * hpg + AT_ROWS - 1) / AT_ROWS, du.users * kv_heads);
  cfg.blockDim = dim3(AT_THREADS);
  const int tail_off = db_tail_off<HD>(hpg);
  cfg.dynamicSmemBytes = 1024 + tail_off + DbCfg<HD>::TAIL_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_on(PDL_ATTN) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const long krow = (long)layer * 2 * kv_heads * cap, kuser = (long)layers * 2 * kv_heads * cap;
  const long vrow = (long)layer * kv_heads * HD, vuser = (long)layers * kv_heads * HD;
  return cudaLaunchKernelEx(&cfg, decode_attn_tc_bf16_kernel<HD>, *reinterpret_cast<const CUtensorMap*>(&mp.kmap),
                            *reinterpret_cast<const CUtensorMap*>(&mp.vmap), krow, kuser, vrow, vuser, cap,
                            static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(ks),
                            static_cast<const __nv_bfloat16*>(vs), anc, L_dev, static_cast<__nv_bfloat16*>(out),
                            beams, heads, kv_heads, t, scale, status, du.anc_user_stride, tail_off);
}

cudaError_t attention_decode_tc_bf16(const BfPrefillMaps& mp, int layer, int layers, const void* q,
                                     const void* k_suffix, const void* v_suffix, const int32_t* anc,
                                     const int32_t* L_dev, int t, void* out, int beams, int prefix_cap, int heads,
                                     int kv_heads, int head_dim, float scale, uint32_t* status, cudaStream_t stream,
                                     const DecodeUsers& du) {
  if (t < 1 || t > 4 || beams > MAX_BEAMS || du.users < 1 || prefix_cap > mp.pair_cap ||
      !attention_decode_tc_bf16_supported(heads, kv_heads, head_dim))
    return cudaErrorInvalidValue;
  if (head_dim == 128)
    return launch_decode_tc_bf16<128>(mp, layer, layers, q, k_suffix, v_suffix, anc, L_dev, t, out, beams, prefix_cap,
                                      heads, kv_heads, scale, status, stream, du);
  return launch_decode_tc_bf16<64>(mp, layer, layers, q, k_suffix, v_suffix, anc, L_dev, t, out, beams, prefix_cap,
                                   heads, kv_heads, scale, status, stream, du);
}

cudaError_t attention_tc_init() {
  // the most a supported launch takes (the suffix staging grows as hpg falls)
  cudaError_t e = cudaFuncSetAttribute(decode_attn_tc_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       AT_SMEM_MAX + 1024);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(decode_attn_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             AT_SMEM_MAX + 1024);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(prefill_attn_tc_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             PtCfg<128>::SMEM);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(prefill_attn_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             PtCfg<64>::SMEM);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(prefill_attn_tc_bf16_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             PbCfg<128>::SMEM);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(prefill_attn_tc_bf16_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             PbCfg<64>::SMEM);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(decode_attn_tc_bf16_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             AT_SMEM_MAX + 1024);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(decode_attn_tc_bf16_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             AT_SMEM_MAX + 1024);
  return e;
}

}  // namespace rtr
