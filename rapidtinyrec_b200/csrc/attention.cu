// Attention kernels for the shared-prefix beam path (FP32, head_dim 64/128).
//
// Prefill: causal GQA attention of one request (sdpa_attention_forward with
// is_causal=True, transformers integrations/sdpa_attention.py:40-104).  A CTA
// owns 16 query positions of one query head, two per warp.
//
// Decode: the reference's folded_sdpa (rapidtinyrec/folded_attention.py:16-31)
// maps query head h to KV head h / (Hq/Hkv) and attends over
// cat(prefix.expand(50), suffix) (shared_prefix.py:22-29).  Here the prefix is
// read in place and never expanded: a CTA owns one query head and 8 beams (one
// warp each); after the prefix, every warp walks its beam's own suffix keys,
// found through the ancestry table instead of a physical reorder (the
// direct_reorder parent gather, prefix_replay.py:95-117).
//
// Both stream the prefix K/V rows of the head's KV group through a
// double-buffered shared ring of 64-key chunks with cp.async (K rows padded by
// four floats so the float4 score reads of 8 consecutive keys hit distinct
// banks), and every warp runs an online softmax over its query rows: lane j
// scores keys j and j + 32 of the chunk, then accumulates P.V over its own
// HD/32 output dimensions.
#include <math.h>

#include "common.cuh"
#include "engine.h"

namespace rtr {

constexpr int AK = 64;         // keys per chunk
constexpr int AWARPS = 8;      // warps per CTA
constexpr int ATHREADS = AWARPS * 32;
constexpr int PQ = 16;         // prefill query positions per CTA (2 per warp)
constexpr int DBEAMS = AWARPS; // decode beams per CTA (1 per warp)

template <int HD> constexpr int kld() { return HD + 4; }
template <int HD> constexpr size_t attn_smem_bytes(int qrows) {
  return (size_t)(2 * AK * kld<HD>() + 2 * AK * HD + qrows * HD) * sizeof(float);
}

// Stage keys [k0, k0 + AK) of one KV group into ring slot `buf` (zero rows
// past `kend`); one cp.async group.
template <int HD>
RTR_DEVICE void load_kv_chunk(float* kbuf, float* vbuf, const float* kbase, const float* vbase, int k0, int kend,
                              int buf) {
  constexpr int V4 = HD / 4;
  float* kd = kbuf + (size_t)buf * AK * kld<HD>();
  float* vd = vbuf + (size_t)buf * AK * HD;
  for (int i = threadIdx.x; i < AK * V4; i += ATHREADS) {
    const int j = i / V4, d = (i % V4) * 4;
    const bool ok = k0 + j < kend;
    const long row = ok ? k0 + j : 0;
    cp_async16(kd + j * kld<HD>() + d, kbase + row * HD + d, ok);
    cp_async16(vd + j * HD + d, vbase + row * HD + d, ok);
  }
  cp_async_commit();
}

// VEC consecutive floats from shared memory as one vector access.
template <int VEC> RTR_DEVICE void load_vec(const float* src, float (&x)[VEC]);
template <> RTR_DEVICE void load_vec<4>(const float* src, float (&x)[4]) {
  const float4 v = *reinterpret_cast<const float4*>(src);
  x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
}
template <> RTR_DEVICE void load_vec<2>(const float* src, float (&x)[2]) {
  const float2 v = *reinterpret_cast<const float2*>(src);
  x[0] = v.x; x[1] = v.y;
}

// One warp, one query row (q in shared memory), one staged chunk of keys
// [k0, k0 + AK): online-softmax update of (m, l, acc) over keys < kend.
template <int HD>
RTR_DEVICE void chunk_update(const float* qrow, const float* kc, const float* vc, int k0, int kend, float scale,
                             float& m, float& l, float (&acc)[HD / 32]) {
  constexpr int VEC = HD / 32;
  const int lane = threadIdx.x & 31;
  const float4* q4 = reinterpret_cast<const float4*>(qrow);
  const float4* ka = reinterpret_cast<const float4*>(kc + lane * kld<HD>());
  const float4* kb = reinterpret_cast<const float4*>(kc + (lane + 32) * kld<HD>());
  float s0 = 0.f, s1 = 0.f;
#pragma unroll 8
  for (int d = 0; d < HD / 4; ++d) {
    const float4 qq = q4[d], a = ka[d], b = kb[d];
    s0 = fmaf(qq.x, a.x, s0); s0 = fmaf(qq.y, a.y, s0); s0 = fmaf(qq.z, a.z, s0); s0 = fmaf(qq.w, a.w, s0);
    s1 = fmaf(qq.x, b.x, s1); s1 = fmaf(qq.y, b.y, s1); s1 = fmaf(qq.z, b.z, s1); s1 = fmaf(qq.w, b.w, s1);
  }
  s0 = k0 + lane < kend ? s0 * scale : -INFINITY;
  s1 = k0 + lane + 32 < kend ? s1 * scale : -INFINITY;
  const float mn = fmaxf(m, warp_max(fmaxf(s0, s1)));  // finite: key k0 is always valid
  const float corr = expf(m - mn);
  const float p0 = expf(s0 - mn), p1 = expf(s1 - mn);
  l = l * corr + warp_sum(p0 + p1);
  m = mn;
#pragma unroll
  for (int i = 0; i < VEC; ++i) acc[i] *= corr;
  const float* va = vc + lane * VEC;
#pragma unroll 4
  for (int j = 0; j < 32; ++j) {
    const float pa = __shfl_sync(0xffffffffu, p0, j), pb = __shfl_sync(0xffffffffu, p1, j);
    float x[VEC], y[VEC];
    load_vec<VEC>(va + j * HD, x);
    load_vec<VEC>(va + (j + 32) * HD, y);
#pragma unroll
    for (int i = 0; i < VEC; ++i) acc[i] = fmaf(pa, x[i], acc[i]);
#pragma unroll
    for (int i = 0; i < VEC; ++i) acc[i] = fmaf(pb, y[i], acc[i]);
  }
}

// ------------------------------------------------------------------ prefill
template <int HD>
__global__ void __launch_bounds__(ATHREADS) prefill_attn_kernel(
    const float* __restrict__ q, const float* __restrict__ kp, const float* __restrict__ vp,
    float* __restrict__ out, float* __restrict__ out_big, float* __restrict__ out_small, int L, int cap, int heads,
    int kv_heads, float scale) {
  constexpr int VEC = HD / 32, ROWS = PQ / AWARPS;
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ __align__(16) float asmem[];
  float* kbuf = asmem;
  float* vbuf = kbuf + 2 * AK * kld<HD>();
  float* qs = vbuf + 2 * AK * HD;  // [PQ][HD]
  const int h = blockIdx.y, g = h / (heads / kv_heads);
  const int q0 = blockIdx.x * PQ;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* kbase = kp + (long)g * cap * HD;
  const float* vbase = vp + (long)g * cap * HD;
  const int kend = min(L, q0 + PQ);  // keys any row of the block may see
  const int nchunks = (kend + AK - 1) / AK;

  load_kv_chunk<HD>(kbuf, vbuf, kbase, vbase, 0, kend, 0);
  for (int i = threadIdx.x; i < PQ * HD / 4; i += ATHREADS) {
    const int r = i / (HD / 4), d = (i % (HD / 4)) * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (q0 + r < L) v = *reinterpret_cast<const float4*>(q + ((long)(q0 + r) * heads + h) * HD + d);
    *reinterpret_cast<float4*>(qs + r * HD + d) = v;
  }
  float m[ROWS], l[ROWS], acc[ROWS][VEC];
#pragma unroll
  for (int r = 0; r < ROWS; ++r) {
    m[r] = -INFINITY; l[r] = 0.f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) acc[r][i] = 0.f;
  }
  for (int c = 0; c < nchunks; ++c) {
    if (c + 1 < nchunks) load_kv_chunk<HD>(kbuf, vbuf, kbase, vbase, (c + 1) * AK, kend, (c + 1) & 1);
    else cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const float* kc = kbuf + (c & 1) * AK * kld<HD>();
    const float* vc = vbuf + (c & 1) * AK * HD;
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      const int row = warp * ROWS + r, qpos = q0 + row;
      if (qpos < L && c * AK <= qpos)
        chunk_update<HD>(qs + row * HD, kc, vc, c * AK, qpos + 1, scale, m[r], l[r], acc[r]);
    }
    __syncthreads();  // the slot is refilled by the next iteration's load
  }
#pragma unroll
  for (int r = 0; r < ROWS; ++r) {
    const int qpos = q0 + warp * ROWS + r;
    if (qpos >= L) continue;
    const float inv = 1.0f / l[r];
#pragma unroll
    for (int i = 0; i < VEC; ++i)
      store_split(out, out_big, out_small, ((long)qpos * heads + h) * HD + lane * VEC + i, acc[r][i] * inv);
  }
}

cudaError_t attention_prefill(const float* q, const float* k_prefix, const float* v_prefix,
                              float* out, float* out_big, float* out_small, int L, int prefix_cap, int heads,
                              int kv_heads, int head_dim, float scale, cudaStream_t stream) {
  if (L <= 0 || L > prefix_cap) return cudaErrorInvalidValue;
  dim3 grid((L + PQ - 1) / PQ, heads);
  if (head_dim == 128)
    return launch_pdl(PDL_ATTN, prefill_attn_kernel<128>, grid, dim3(ATHREADS), attn_smem_bytes<128>(PQ), stream, q, k_prefix,
                      v_prefix, out, out_big, out_small, L, prefix_cap, heads, kv_heads, scale);
  else if (head_dim == 64)
    return launch_pdl(PDL_ATTN, prefill_attn_kernel<64>, grid, dim3(ATHREADS), attn_smem_bytes<64>(PQ), stream, q, k_prefix,
                      v_prefix, out, out_big, out_small, L, prefix_cap, heads, kv_heads, scale);
  return cudaErrorInvalidValue;
}

// ------------------------------------------------------------------- decode
template <int HD>
__global__ void __launch_bounds__(ATHREADS) decode_attn_kernel(
    const float* __restrict__ q, const float* __restrict__ kp, const float* __restrict__ vp,
    const float* __restrict__ ksuf, const float* __restrict__ vsuf, const int32_t* __restrict__ anc,
    const int32_t* __restrict__ L_dev, float* __restrict__ out, float* __restrict__ out_big,
    float* __restrict__ out_small, int beams, int cap, int heads, int kv_heads, int t, float scale,
    uint32_t* __restrict__ status) {
  constexpr int VEC = HD / 32;
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ __align__(16) float asmem[];
  float* kbuf = asmem;
  float* vbuf = kbuf + 2 * AK * kld<HD>();
  float* qs = vbuf + 2 * AK * HD;  // [DBEAMS][HD]
  const int h = blockIdx.x, g = h / (heads / kv_heads);
  const int b0 = blockIdx.y * DBEAMS;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = b0 + warp;
  int L = *L_dev;
  if (L < 1 || L > cap) {  // the prefill recorded no valid prefix: attend to the suffix only
    if (threadIdx.x == 0) atomicOr(status, RTR_DEV_BAD_LENGTH);
    L = 0;
  }
  const float* kbase = kp + (long)g * cap * HD;
  const float* vbase = vp + (long)g * cap * HD;
  const int nchunks = (L + AK - 1) / AK;

  if (nchunks > 0) load_kv_chunk<HD>(kbuf, vbuf, kbase, vbase, 0, L, 0);
  for (int i = threadIdx.x; i < DBEAMS * HD / 4; i += ATHREADS) {
    const int r = i / (HD / 4), d = (i % (HD / 4)) * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (b0 + r < beams) v = *reinterpret_cast<const float4*>(q + ((long)(b0 + r) * heads + h) * HD + d);
    *reinterpret_cast<float4*>(qs + r * HD + d) = v;
  }
  float m = -INFINITY, l = 0.f, acc[VEC];
#pragma unroll
  for (int i = 0; i < VEC; ++i) acc[i] = 0.f;
  for (int c = 0; c < nchunks; ++c) {
    if (c + 1 < nchunks) load_kv_chunk<HD>(kbuf, vbuf, kbase, vbase, (c + 1) * AK, L, (c + 1) & 1);
    else cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (b < beams)
      chunk_update<HD>(qs + warp * HD, kbuf + (c & 1) * AK * kld<HD>(), vbuf + (c & 1) * AK * HD, c * AK, L, scale,
                       m, l, acc);
    __syncthreads();  // the slot is refilled by the next iteration's load
  }
  if (nchunks == 0) __syncthreads();  // q rows staged
  if (b >= beams) return;

  // the beam's suffix: slot s < t - 1 lives in row anc[b][s], slot t - 1 in row b
  const float* qrow = qs + warp * HD + lane * VEC;
  float qv[VEC];
#pragma unroll
  for (int i = 0; i < VEC; ++i) qv[i] = qrow[i];
  for (int s = 0; s < t; ++s) {
    int row = (s == t - 1) ? b : anc[b * 4 + s];
    if (row < 0 || row >= beams) {
      if (lane == 0) atomicOr(status, RTR_DEV_BAD_PARENT);
      row = b;
    }
    const long off = (((long)s * beams + row) * kv_heads + g) * HD + lane * VEC;
    float d = 0.f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) d = fmaf(qv[i], ksuf[off + i], d);
    const float sc = warp_sum(d) * scale;
    const float mn = fmaxf(m, sc);
    const float corr = expf(m - mn);
    const float p = expf(sc - mn);
    l = l * corr + p;
    m = mn;
#pragma unroll
    for (int i = 0; i < VEC; ++i) acc[i] = fmaf(p, vsuf[off + i], acc[i] * corr);
  }
  const float inv = 1.0f / l;
#pragma unroll
  for (int i = 0; i < VEC; ++i)
    store_split(out, out_big, out_small, ((long)b * heads + h) * HD + lane * VEC + i, acc[i] * inv);
}

cudaError_t attention_decode(const float* q, const float* k_prefix, const float* v_prefix,
                             const float* k_suffix, const float* v_suffix, const int32_t* anc,
                             const int32_t* L_dev, int t, float* out, float* out_big, float* out_small, int beams,
                             int prefix_cap, int heads, int kv_heads, int head_dim, float scale, uint32_t* status,
                             cudaStream_t stream) {
  if (t < 1 || t > 4 || beams > MAX_BEAMS) return cudaErrorInvalidValue;
  dim3 grid(heads, (beams + DBEAMS - 1) / DBEAMS);
  if (head_dim == 128)
    return launch_pdl(PDL_ATTN, decode_attn_kernel<128>, grid, dim3(ATHREADS), attn_smem_bytes<128>(DBEAMS), stream, q,
                      k_prefix, v_prefix, k_suffix, v_suffix, anc, L_dev, out, out_big, out_small, beams, prefix_cap,
                      heads, kv_heads, t, scale, status);
  else if (head_dim == 64)
    return launch_pdl(PDL_ATTN, decode_attn_kernel<64>, grid, dim3(ATHREADS), attn_smem_bytes<64>(DBEAMS), stream, q,
                      k_prefix, v_prefix, k_suffix, v_suffix, anc, L_dev, out, out_big, out_small, beams, prefix_cap,
                      heads, kv_heads, t, scale, status);
  return cudaErrorInvalidValue;
}

cudaError_t attention_init() {
  cudaError_t e = cudaFuncSetAttribute(prefill_attn_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)attn_smem_bytes<128>(PQ));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(prefill_attn_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)attn_smem_bytes<64>(PQ));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(decode_attn_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)attn_smem_bytes<128>(DBEAMS));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(decode_attn_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)attn_smem_bytes<64>(DBEAMS));
  return e;
}

}  // namespace rtr
