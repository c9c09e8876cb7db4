// Attention kernels for the shared-prefix beam path (FP32, head_dim 64/128).
//
// Prefill: causal GQA attention of one request (sdpa_attention_forward with
// is_causal=True, transformers integrations/sdpa_attention.py:40-104).  A CTA
// owns 16 query positions of one query head; key/value chunks of 32 rows are
// staged in shared memory (keys transposed so lane j scores key j
// conflict-free) and every warp runs an online softmax for its two rows.
//
// Decode: the reference's folded_sdpa (rapidtinyrec/folded_attention.py:16-31)
// maps query head h to KV head h / (Hq/Hkv) and attends over
// cat(prefix.expand(50), suffix) (shared_prefix.py:22-29).  Here the prefix is
// read in place: phase 1 streams each 32-key prefix chunk of a KV head into
// shared memory once and scores it against all 50 beams of one query head,
// writing (max, sum, weighted V) partials; phase 2 merges the partials with the
// beam's own suffix keys, found through the ancestry table instead of a
// physical reorder (the direct_reorder parent gather, prefix_replay.py:95-117).
#include <math.h>

#include "common.cuh"
#include "engine.h"

namespace rtr {

constexpr int KC = 32;     // keys per chunk
constexpr int QB = 16;     // prefill query positions per CTA
constexpr int ATT_THREADS = 256;

template <int HD>
__global__ void __launch_bounds__(ATT_THREADS) prefill_attn_kernel(
    const float* __restrict__ q, const float* __restrict__ kp, const float* __restrict__ vp,
    float* __restrict__ out, float* __restrict__ out_big, float* __restrict__ out_small, int L, int cap, int heads,
    int kv_heads, float scale) {
  constexpr int PER = HD / 32;
  __shared__ float qs[QB][HD];
  __shared__ float ks[HD][KC + 1];
  __shared__ float vs[KC][HD];
  const int h = blockIdx.y, g = h / (heads / kv_heads);
  const int q0 = blockIdx.x * QB;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* kbase = kp + (long)g * cap * HD;
  const float* vbase = vp + (long)g * cap * HD;

  for (int i = threadIdx.x; i < QB * HD; i += ATT_THREADS) {
    const int r = i / HD, d = i % HD;
    qs[r][d] = (q0 + r < L) ? q[((long)(q0 + r) * heads + h) * HD + d] : 0.f;
  }
  constexpr int ROWS = QB / (ATT_THREADS / 32);  // 2 rows per warp
  float m_run[ROWS], l_run[ROWS], acc[ROWS][PER];
#pragma unroll
  for (int r = 0; r < ROWS; ++r) {
    m_run[r] = -INFINITY; l_run[r] = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) acc[r][i] = 0.f;
  }
  const int last = min(L, q0 + QB) - 1;  // highest query position in the block
  for (int c0 = 0; c0 <= last; c0 += KC) {
    __syncthreads();
    for (int i = threadIdx.x; i < KC * HD; i += ATT_THREADS) {
      const int j = i / HD, d = i % HD;
      const bool ok = c0 + j < L;
      ks[d][j] = ok ? kbase[(long)(c0 + j) * HD + d] : 0.f;
      vs[j][d] = ok ? vbase[(long)(c0 + j) * HD + d] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      const int row = warp * ROWS + r;
      const int qpos = q0 + row;
      if (qpos >= L || c0 > qpos) continue;
      float s = 0.f;
#pragma unroll 8
      for (int d = 0; d < HD; ++d) s = fmaf(qs[row][d], ks[d][lane], s);
      s *= scale;
      const int kpos = c0 + lane;
      if (kpos > qpos) s = -INFINITY;
      const float mc = warp_max(s);
      const float mn = fmaxf(m_run[r], mc);
      const float corr = expf(m_run[r] - mn);
      const float p = expf(s - mn);
      l_run[r] = l_run[r] * corr + warp_sum(p);
      m_run[r] = mn;
#pragma unroll
      for (int i = 0; i < PER; ++i) acc[r][i] *= corr;
#pragma unroll 8
      for (int j = 0; j < KC; ++j) {
        const float pj = __shfl_sync(0xffffffffu, p, j);
#pragma unroll
        for (int i = 0; i < PER; ++i) acc[r][i] = fmaf(pj, vs[j][lane + 32 * i], acc[r][i]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < ROWS; ++r) {
    const int qpos = q0 + warp * ROWS + r;
    if (qpos >= L) continue;
    const float inv = 1.0f / l_run[r];
#pragma unroll
    for (int i = 0; i < PER; ++i)
      store_split(out, out_big, out_small, ((long)qpos * heads + h) * HD + lane + 32 * i, acc[r][i] * inv);
  }
}

cudaError_t attention_prefill(const float* q, const float* k_prefix, const float* v_prefix,
                              float* out, float* out_big, float* out_small, int L, int prefix_cap, int heads,
                              int kv_heads, int head_dim, float scale, cudaStream_t stream) {
  dim3 grid((L + QB - 1) / QB, heads);
  if (head_dim == 128)
    prefill_attn_kernel<128><<<grid, ATT_THREADS, 0, stream>>>(q, k_prefix, v_prefix, out, out_big, out_small, L,
                                                               prefix_cap, heads, kv_heads, scale);
  else if (head_dim == 64)
    prefill_attn_kernel<64><<<grid, ATT_THREADS, 0, stream>>>(q, k_prefix, v_prefix, out, out_big, out_small, L,
                                                              prefix_cap, heads, kv_heads, scale);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

// ------------------------------------------------------------------- decode
int attention_decode_chunks(int max_prefix) { return (max_prefix + KC - 1) / KC; }

// Phase 1: grid (chunks, kv_heads, heads_per_group); one query head of the
// group against one prefix chunk, all beams.
template <int HD>
__global__ void __launch_bounds__(ATT_THREADS) decode_prefix_kernel(
    const float* __restrict__ q, const float* __restrict__ kp, const float* __restrict__ vp,
    const int32_t* __restrict__ L_dev, float* __restrict__ part, int beams, int cap, int heads,
    int kv_heads, int nc_max, float scale) {
  constexpr int PER = HD / 32;
  __shared__ float ks[HD][KC + 1];
  __shared__ float vs[KC][HD];
  __shared__ float qrow[ATT_THREADS / 32][HD];
  const int L = *L_dev;
  const int c = blockIdx.x, g = blockIdx.y;
  const int h = g * (heads / kv_heads) + blockIdx.z;
  const int c0 = c * KC;
  if (c0 >= L || L > cap) return;
  const int nkeys = min(KC, L - c0);
  const float* kbase = kp + ((long)g * cap + c0) * HD;
  const float* vbase = vp + ((long)g * cap + c0) * HD;
  for (int i = threadIdx.x; i < KC * HD; i += ATT_THREADS) {
    const int j = i / HD, d = i % HD;
    const bool ok = j < nkeys;
    ks[d][j] = ok ? kbase[(long)j * HD + d] : 0.f;
    vs[j][d] = ok ? vbase[(long)j * HD + d] : 0.f;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int b = warp; b < beams; b += ATT_THREADS / 32) {
    const float* qr = q + ((long)b * heads + h) * HD;
#pragma unroll
    for (int i = 0; i < PER; ++i) qrow[warp][lane + 32 * i] = qr[lane + 32 * i];
    __syncwarp();
    float s = 0.f;
#pragma unroll 8
    for (int d = 0; d < HD; ++d) s = fmaf(qrow[warp][d], ks[d][lane], s);
    s = lane < nkeys ? s * scale : -INFINITY;
    const float m = warp_max(s);
    const float p = expf(s - m);
    const float l = warp_sum(p);
    float acc[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) acc[i] = 0.f;
#pragma unroll 8
    for (int j = 0; j < KC; ++j) {
      const float pj = __shfl_sync(0xffffffffu, p, j);
#pragma unroll
      for (int i = 0; i < PER; ++i) acc[i] = fmaf(pj, vs[j][lane + 32 * i], acc[i]);
    }
    float* dst = part + (((long)b * heads + h) * nc_max + c) * (HD + 2);
    if (lane == 0) { dst[0] = m; dst[1] = l; }
#pragma unroll
    for (int i = 0; i < PER; ++i) dst[2 + lane + 32 * i] = acc[i];
    __syncwarp();
  }
}

// Phase 2: one warp per (beam, query head): merge prefix partials and the
// beam's suffix keys (slots 0..t-1).
template <int HD>
__global__ void decode_combine_kernel(const float* __restrict__ q, const float* __restrict__ ks,
                                      const float* __restrict__ vsuf, const int32_t* __restrict__ anc,
                                      const int32_t* __restrict__ L_dev, const float* __restrict__ part,
                                      float* __restrict__ out, float* __restrict__ out_big,
                                      float* __restrict__ out_small, int beams, int heads, int kv_heads,
                                      int nc_max, int t, float scale) {
  constexpr int PER = HD / 32;
  const int warp_global = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (warp_global >= beams * heads) return;
  const int b = warp_global / heads, h = warp_global % heads;
  const int g = h / (heads / kv_heads);
  const int L = *L_dev;
  const int nc = min((L + KC - 1) / KC, nc_max);
  float qv[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) qv[i] = q[((long)b * heads + h) * HD + lane + 32 * i];
  // suffix scores
  float ss[4];
  int rows[4];
  float M = -INFINITY;
  for (int s = 0; s < t; ++s) {
    int row = (s == t - 1) ? b : anc[b * 4 + s];
    if (row < 0 || row >= beams) row = b;
    rows[s] = row;
    const float* key = ks + (((long)s * beams + row) * kv_heads + g) * HD;
    float d = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) d = fmaf(qv[i], key[lane + 32 * i], d);
    d = warp_sum(d) * scale;
    ss[s] = d;
    M = fmaxf(M, d);
  }
  const float* pb = part + ((long)b * heads + h) * nc_max * (HD + 2);
  for (int c = 0; c < nc; ++c) M = fmaxf(M, pb[c * (HD + 2)]);
  float l = 0.f, acc[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) acc[i] = 0.f;
  for (int c = 0; c < nc; ++c) {
    const float* pc = pb + c * (HD + 2);
    const float w = expf(pc[0] - M);
    l = fmaf(pc[1], w, l);
#pragma unroll
    for (int i = 0; i < PER; ++i) acc[i] = fmaf(pc[2 + lane + 32 * i], w, acc[i]);
  }
  for (int s = 0; s < t; ++s) {
    const float w = expf(ss[s] - M);
    l += w;
    const float* val = vsuf + (((long)s * beams + rows[s]) * kv_heads + g) * HD;
#pragma unroll
    for (int i = 0; i < PER; ++i) acc[i] = fmaf(w, val[lane + 32 * i], acc[i]);
  }
  const float inv = 1.0f / l;
#pragma unroll
  for (int i = 0; i < PER; ++i)
    store_split(out, out_big, out_small, ((long)b * heads + h) * HD + lane + 32 * i, acc[i] * inv);
}

cudaError_t attention_decode(const float* q, const float* k_prefix, const float* v_prefix,
                             const float* k_suffix, const float* v_suffix, const int32_t* anc,
                             const int32_t* L_dev, int t, float* part, float* out, float* out_big,
                             float* out_small, int beams, int prefix_cap, int heads, int kv_heads, int head_dim,
                             float scale, cudaStream_t stream) {
  const int nc_max = attention_decode_chunks(prefix_cap);
  dim3 g1(nc_max, kv_heads, heads / kv_heads);
  const int warps = beams * heads, cb = (warps + 3) / 4;
  if (head_dim == 128) {
    decode_prefix_kernel<128><<<g1, ATT_THREADS, 0, stream>>>(q, k_prefix, v_prefix, L_dev, part, beams, prefix_cap, heads, kv_heads, nc_max, scale);
    decode_combine_kernel<128><<<cb, 128, 0, stream>>>(q, k_suffix, v_suffix, anc, L_dev, part, out, out_big, out_small, beams, heads, kv_heads, nc_max, t, scale);
  } else if (head_dim == 64) {
    decode_prefix_kernel<64><<<g1, ATT_THREADS, 0, stream>>>(q, k_prefix, v_prefix, L_dev, part, beams, prefix_cap, heads, kv_heads, nc_max, scale);
    decode_combine_kernel<64><<<cb, 128, 0, stream>>>(q, k_suffix, v_suffix, anc, L_dev, part, out, out_big, out_small, beams, heads, kv_heads, nc_max, t, scale);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace rtr
