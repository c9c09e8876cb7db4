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

// Prefix K/V rows are staged in their storage type T (fp32, or bf16 in the
// bf16 mode); K rows are padded so 16-byte copies stay aligned and the score
// reads of consecutive keys spread over the banks.  q lives in fp32.
template <int HD, typename T> __host__ __device__ constexpr int kld() { return HD + 16 / (int)sizeof(T); }
template <int HD, typename T> constexpr size_t attn_smem_bytes(int qrows) {
  return (size_t)(2 * AK * kld<HD, T>() + 2 * AK * HD) * sizeof(T) + (size_t)qrows * HD * sizeof(float);
}

// Four consecutive elements as floats.
RTR_DEVICE float4 ld4f(const float* p) { return *reinterpret_cast<const float4*>(p); }
RTR_DEVICE float4 ld4f(const __nv_bfloat16* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
// Output element i of a row: fp32 rows also get their tf32 split (the 3xTF32
// GEMM operands); bf16 rows are rounded once.
RTR_DEVICE void store_out(float* out, float* big, float* small, long i, float v, int fmt) {
  store_split(out, big, small, i, v, fmt);
}
RTR_DEVICE void store_out(__nv_bfloat16* out, float*, float*, long i, float v, int) { out[i] = __float2bfloat16_rn(v); }

// Stage keys [k0, k0 + AK) of one KV group into ring slot `buf` (zero rows
// past `kend`); one cp.async group.
template <int HD, typename T>
RTR_DEVICE void load_kv_chunk(T* kbuf, T* vbuf, const T* kbase, const T* vbase, int k0, int kend, int buf) {
  constexpr int E = 16 / (int)sizeof(T);  // elements per 16-byte copy
  constexpr int V4 = HD / E;
  T* kd = kbuf + (size_t)buf * AK * kld<HD, T>();
  T* vd = vbuf + (size_t)buf * AK * HD;
  for (int i = threadIdx.x; i < AK * V4; i += ATHREADS) {
    const int j = i / V4, d = (i % V4) * E;
    const bool ok = k0 + j < kend;
    const long row = ok ? k0 + j : 0;
    cp_async16(kd + j * kld<HD, T>() + d, kbase + row * HD + d, ok);
    cp_async16(vd + j * HD + d, vbase + row * HD + d, ok);
  }
  cp_async_commit();
}

// VEC consecutive elements from shared memory as one vector access.
RTR_DEVICE void load_vec(const float* src, float (&x)[4]) {
  const float4 v = *reinterpret_cast<const float4*>(src);
  x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
}
RTR_DEVICE void load_vec(const float* src, float (&x)[2]) {
  const float2 v = *reinterpret_cast<const float2*>(src);
  x[0] = v.x; x[1] = v.y;
}
RTR_DEVICE void load_vec(const __nv_bfloat16* src, float (&x)[4]) {
  const float4 v = ld4f(src);
  x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
}
RTR_DEVICE void load_vec(const __nv_bfloat16* src, float (&x)[2]) {
  const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(src));
  x[0] = v.x; x[1] = v.y;
}

// One warp, one query row (q in shared memory), one staged chunk of keys
// [k0, k0 + AK): online-softmax update of (m, l, acc) over keys < kend.
template <int HD, typename T>
RTR_DEVICE void chunk_update(const float* qrow, const T* kc, const T* vc, int k0, int kend, float scale,
                             float& m, float& l, float (&acc)[HD / 32]) {
  constexpr int VEC = HD / 32;
  const int lane = threadIdx.x & 31;
  const float4* q4 = reinterpret_cast<const float4*>(qrow);
  const T* ka = kc + lane * kld<HD, T>();
  const T* kb = kc + (lane + 32) * kld<HD, T>();
  float s0 = 0.f, s1 = 0.f;
#pragma unroll 8
  for (int d = 0; d < HD / 4; ++d) {
    const float4 qq = q4[d], a = ld4f(ka + 4 * d), b = ld4f(kb + 4 * d);
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
  const T* va = vc + lane * VEC;
#pragma unroll 4
  for (int j = 0; j < 32; ++j) {
    const float pa = __shfl_sync(0xffffffffu, p0, j), pb = __shfl_sync(0xffffffffu, p1, j);
    float x[VEC], y[VEC];
    load_vec(va + j * HD, x);
    load_vec(va + (j + 32) * HD, y);
#pragma unroll
    for (int i = 0; i < VEC; ++i) acc[i] = fmaf(pa, x[i], acc[i]);
#pragma unroll
    for (int i = 0; i < VEC; ++i) acc[i] = fmaf(pb, y[i], acc[i]);
  }
}

// ------------------------------------------------------------------ prefill
template <int HD, typename T>
__global__ void __launch_bounds__(ATHREADS) prefill_attn_kernel(
    const T* __restrict__ q, const T* __restrict__ kp, const T* __restrict__ vp,
    T* __restrict__ out, float* __restrict__ out_big, float* __restrict__ out_small, int L, int cap, int heads,
    int kv_heads, float scale, int xfmt) {
  constexpr int VEC = HD / 32, ROWS = PQ / AWARPS;
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ __align__(16) unsigned char asmem[];
  T* kbuf = reinterpret_cast<T*>(asmem);
  T* vbuf = kbuf + 2 * AK * kld<HD, T>();
  float* qs = reinterpret_cast<float*>(vbuf + 2 * AK * HD);  // [PQ][HD]
  const int h = blockIdx.y, g = h / (heads / kv_heads);
  const int q0 = blockIdx.x * PQ;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const T* kbase = kp + (long)g * cap * HD;
  const T* vbase = vp + (long)g * cap * HD;
  const int kend = min(L, q0 + PQ);  // keys any row of the block may see
  const int nchunks = (kend + AK - 1) / AK;

  load_kv_chunk<HD, T>(kbuf, vbuf, kbase, vbase, 0, kend, 0);
  for (int i = threadIdx.x; i < PQ * HD / 4; i += ATHREADS) {
    const int r = i / (HD / 4), d = (i % (HD / 4)) * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (q0 + r < L) v = ld4f(q + ((long)(q0 + r) * heads + h) * HD + d);
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
    if (c + 1 < nchunks) load_kv_chunk<HD, T>(kbuf, vbuf, kbase, vbase, (c + 1) * AK, kend, (c + 1) & 1);
    else cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const T* kc = kbuf + (c & 1) * AK * kld<HD, T>();
    const T* vc = vbuf + (c & 1) * AK * HD;
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      const int row = warp * ROWS + r, qpos = q0 + row;
      if (qpos < L && c * AK <= qpos)
        chunk_update<HD, T>(qs + row * HD, kc, vc, c * AK, qpos + 1, scale, m[r], l[r], acc[r]);
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
      store_out(out, out_big, out_small, ((long)qpos * heads + h) * HD + lane * VEC + i, acc[r][i] * inv, xfmt);
  }
}

template <int HD, typename T>
static cudaError_t launch_prefill(const void* q, const void* kp, const void* vp, void* out, float* ob, float* os, int L,
                                  int cap, int heads, int kv_heads, float scale, cudaStream_t stream, int xfmt) {
  dim3 grid((L + PQ - 1) / PQ, heads);
  return launch_pdl(PDL_ATTN, prefill_attn_kernel<HD, T>, grid, dim3(ATHREADS), attn_smem_bytes<HD, T>(PQ), stream,
                    static_cast<const T*>(q), static_cast<const T*>(kp), static_cast<const T*>(vp), static_cast<T*>(out),
                    ob, os, L, cap, heads, kv_heads, scale, xfmt);
}

cudaError_t attention_prefill(const void* q, const void* k_prefix, const void* v_prefix, void* out, float* out_big,
                              float* out_small, int L, int prefix_cap, int heads, int kv_heads, int head_dim,
                              float scale, bool bf16, cudaStream_t stream, int xfmt) {
  if (L <= 0 || L > prefix_cap) return cudaErrorInvalidValue;
  if (head_dim == 128)
    return bf16 ? launch_prefill<128, __nv_bfloat16>(q, k_prefix, v_prefix, out, nullptr, nullptr, L, prefix_cap, heads,
                                                     kv_heads, scale, stream, 0)
                : launch_prefill<128, float>(q, k_prefix, v_prefix, out, out_big, out_small, L, prefix_cap, heads,
                                             kv_heads, scale, stream, xfmt);
  if (head_dim == 64)
    return bf16 ? launch_prefill<64, __nv_bfloat16>(q, k_prefix, v_prefix, out, nullptr, nullptr, L, prefix_cap, heads,
                                                    kv_heads, scale, stream, 0)
                : launch_prefill<64, float>(q, k_prefix, v_prefix, out, out_big, out_small, L, prefix_cap, heads,
                                            kv_heads, scale, stream, xfmt);
  return cudaErrorInvalidValue;
}

// ------------------------------------------------------------------- decode
// One CTA per (query head, 8 beams); the prefix's 64-key chunks stream through
// a double-buffered shared ring (cp.async).  Shared-memory wavefronts bound
// this kernel (a 128-bit LDS costs 4 of them whatever its reuse), so each
// phase tiles registers to load every element once per many FMAs:
//   A  scores: warp w takes a slice of head_dim/8 dimensions; lane = 4 beams x
//      4 keys (keys kg, kg+16, kg+32, kg+48), 16 partial dot products;
//   B  warp = beam: sums the 8 warps' partials of its 64 scores, online
//      softmax (m, l stay in this warp's registers);
//   C  warp w takes keys 8w..8w+7; lane = head_dim/32 output dimensions x 8
//      beams, accumulated across chunks and summed over the warps at the end.
// The beams' suffix rows (found through the ancestry table, the direct-reorder
// parent gather) are staged at the start and folded in by warp = beam.
constexpr int DQLD_PAD = 4;           // q rows: float4 columns of 8 beams in distinct banks
constexpr int DSLD = AK + 4;          // partial-score rows: the two beam halves 16 banks apart

template <int HD, typename T>
constexpr size_t decode_smem_bytes() {
  return (size_t)(2 * AK * kld<HD, T>() + 2 * AK * HD + 2 * DBEAMS * 4 * HD) * sizeof(T) +
         (size_t)(DBEAMS * (HD + DQLD_PAD) + AWARPS * DBEAMS * DSLD + DBEAMS * AK + DBEAMS * 8) * sizeof(float);
}

template <int HD, typename T>
__global__ void __launch_bounds__(ATHREADS) decode_attn_kernel(
    const T* __restrict__ q, const T* __restrict__ kp, const T* __restrict__ vp,
    const T* __restrict__ ksuf, const T* __restrict__ vsuf, const int32_t* __restrict__ anc,
    const int32_t* __restrict__ L_dev, T* __restrict__ out, float* __restrict__ out_big,
    float* __restrict__ out_small, int beams, int cap, int heads, int kv_heads, int t, float scale,
    uint32_t* __restrict__ status, int users, long prefix_user_stride, int anc_user_stride, int xfmt) {
  constexpr int VEC = HD / 32, QLD = HD + DQLD_PAD, E = 16 / (int)sizeof(T);
  constexpr int AD4 = HD / 4 / AWARPS;  // float4 columns per warp in phase A
  static_assert(DBEAMS == 8 && AWARPS == 8 && AK == 64, "tiling assumes 8 beams, 8 warps, 64-key chunks");
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ __align__(16) unsigned char asmem[];
  T* kbuf = reinterpret_cast<T*>(asmem);
  T* vbuf = kbuf + 2 * AK * kld<HD, T>();
  T* sufk = vbuf + 2 * AK * HD;                                  // [DBEAMS][4][HD]
  T* sufv = sufk + DBEAMS * 4 * HD;
  float* qs = reinterpret_cast<float*>(sufv + DBEAMS * 4 * HD);  // [DBEAMS][QLD]
  float* part = qs + DBEAMS * QLD;                               // [AWARPS][DBEAMS][DSLD] partial scores
  float* pr = part + AWARPS * DBEAMS * DSLD;                     // [DBEAMS][AK] probabilities
  float* corr_s = pr + DBEAMS * AK;                              // [DBEAMS]
  const int h = blockIdx.x, g = h / (heads / kv_heads);
  // batched decode: user u owns rows u * beams .. (its own prefix, length and ancestry)
  const int gpu = (beams + DBEAMS - 1) / DBEAMS, u = blockIdx.y / gpu;
  const int b0 = (blockIdx.y % gpu) * DBEAMS, r0 = u * beams, rows = users * beams;
  anc += (long)u * anc_user_stride;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int L = L_dev[u];
  if (L < 1 || L > cap) {  // the prefill recorded no valid prefix: attend to the suffix only
    if (threadIdx.x == 0) atomicOr(status, RTR_DEV_BAD_LENGTH);
    L = 0;
  }
  const T* kbase = kp + u * prefix_user_stride + (long)g * cap * HD;
  const T* vbase = vp + u * prefix_user_stride + (long)g * cap * HD;
  const int nchunks = (L + AK - 1) / AK;

  // the suffix rows of the 8 beams (slot s < t - 1: row anc[b][s]; slot t - 1: row b)
  for (int i = threadIdx.x; i < DBEAMS * 4 * (HD / E); i += ATHREADS) {
    const int bb = i / (4 * (HD / E)), sl = (i / (HD / E)) % 4, d = (i % (HD / E)) * E;
    const int b = b0 + bb;
    if (b >= beams || sl >= t) continue;
    int row = (sl == t - 1) ? b : anc[b * 4 + sl];
    if (row < 0 || row >= beams) {
      if (d == 0) atomicOr(status, RTR_DEV_BAD_PARENT);
      row = b;
    }
    const long off = (((long)sl * rows + r0 + row) * kv_heads + g) * HD + d;
    cp_async16(sufk + (bb * 4 + sl) * HD + d, ksuf + off, true);
    cp_async16(sufv + (bb * 4 + sl) * HD + d, vsuf + off, true);
  }
  cp_async_commit();
  if (nchunks > 0) load_kv_chunk<HD, T>(kbuf, vbuf, kbase, vbase, 0, L, 0);
  else cp_async_commit();
  for (int i = threadIdx.x; i < DBEAMS * HD / 4; i += ATHREADS) {
    const int r = i / (HD / 4), d = (i % (HD / 4)) * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (b0 + r < beams) v = ld4f(q + ((long)(r0 + b0 + r) * heads + h) * HD + d);
    *reinterpret_cast<float4*>(qs + r * QLD + d) = v;
  }
  const int abg = lane >> 4, akg = lane & 15;  // phase A: beams 4abg.., keys akg + 16j
  float m = -INFINITY, l = 0.f;                // phase B state of beam `warp`
  float acc[DBEAMS][VEC];                      // phase C: this warp's keys, dimensions lane*VEC..
#pragma unroll
  for (int b = 0; b < DBEAMS; ++b)
#pragma unroll
    for (int i = 0; i < VEC; ++i) acc[b][i] = 0.f;

  for (int c = 0; c < nchunks; ++c) {
    if (c + 1 < nchunks) load_kv_chunk<HD, T>(kbuf, vbuf, kbase, vbase, (c + 1) * AK, L, (c + 1) & 1);
    else cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const T* kc = kbuf + (c & 1) * AK * kld<HD, T>();
    const T* vc = vbuf + (c & 1) * AK * HD;
    {  // A: 4 beams x 4 keys over this warp's dimension slice
      float ps[4][4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) ps[i][j] = 0.f;
#pragma unroll
      for (int u = 0; u < AD4; ++u) {
        const int d = (warp * AD4 + u) * 4;
        float4 qq[4], kk[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) qq[i] = *reinterpret_cast<const float4*>(qs + (4 * abg + i) * QLD + d);
#pragma unroll
        for (int j = 0; j < 4; ++j) kk[j] = ld4f(kc + (akg + 16 * j) * kld<HD, T>() + d);
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            ps[i][j] = fmaf(qq[i].x, kk[j].x, ps[i][j]);
            ps[i][j] = fmaf(qq[i].y, kk[j].y, ps[i][j]);
            ps[i][j] = fmaf(qq[i].z, kk[j].z, ps[i][j]);
            ps[i][j] = fmaf(qq[i].w, kk[j].w, ps[i][j]);
          }
      }
      float* pw = part + warp * DBEAMS * DSLD;
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) pw[(4 * abg + i) * DSLD + akg + 16 * j] = ps[i][j];
    }
    __syncthreads();
    {  // B: beam `warp`, keys lane and lane + 32; partials summed in warp order
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int w = 0; w < AWARPS; ++w) {
        s0 += part[(w * DBEAMS + warp) * DSLD + lane];
        s1 += part[(w * DBEAMS + warp) * DSLD + lane + 32];
      }
      const int k0 = c * AK;
      s0 = k0 + lane < L ? s0 * scale : -INFINITY;
      s1 = k0 + lane + 32 < L ? s1 * scale : -INFINITY;
      const float mn = fmaxf(m, warp_max(fmaxf(s0, s1)));  // finite: key k0 is always valid
      const float corr = expf(m - mn);
      const float p0 = expf(s0 - mn), p1 = expf(s1 - mn);
      l = l * corr + warp_sum(p0 + p1);
      m = mn;
      pr[warp * AK + lane] = p0;
      pr[warp * AK + lane + 32] = p1;
      if (lane == 0) corr_s[warp] = corr;
    }
    __syncthreads();
    {  // C: acc = acc * corr + P.V over keys 8 warp .. 8 warp + 7
#pragma unroll
      for (int b = 0; b < DBEAMS; ++b) {
        const float cr = corr_s[b];
#pragma unroll
        for (int i = 0; i < VEC; ++i) acc[b][i] *= cr;
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int key = warp * 8 + k;
        float x[VEC];
        load_vec(vc + key * HD + lane * VEC, x);
#pragma unroll
        for (int b = 0; b < DBEAMS; ++b) {
          const float p = pr[b * AK + key];  // broadcast
#pragma unroll
          for (int i = 0; i < VEC; ++i) acc[b][i] = fmaf(p, x[i], acc[b][i]);
        }
      }
    }
    __syncthreads();  // the slot is refilled by the next iteration's load
  }
  cp_async_wait<0>();
  // sum the warps' P.V partials (the K ring is free now): beam `warp`, dims lane*VEC..
  float* red = reinterpret_cast<float*>(kbuf);  // [AWARPS][DBEAMS][HD]
#pragma unroll
  for (int b = 0; b < DBEAMS; ++b)
#pragma unroll
    for (int i = 0; i < VEC; ++i) red[(warp * DBEAMS + b) * HD + lane * VEC + i] = acc[b][i];
  __syncthreads();
  float a[VEC];
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < AWARPS; ++w) v += red[(w * DBEAMS + warp) * HD + lane * VEC + i];
    a[i] = v;
  }
  // the beam's suffix keys, then the output
  const int b = b0 + warp;
  float qv[VEC];
#pragma unroll
  for (int i = 0; i < VEC; ++i) qv[i] = qs[warp * QLD + lane * VEC + i];
  for (int sl = 0; sl < t; ++sl) {
    float kx[VEC], vx[VEC];
    load_vec(sufk + (warp * 4 + sl) * HD + lane * VEC, kx);
    load_vec(sufv + (warp * 4 + sl) * HD + lane * VEC, vx);
    float d = 0.f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) d = fmaf(qv[i], kx[i], d);
    const float sk = warp_sum(d) * scale;
    const float mn = fmaxf(m, sk);
    const float corr = expf(m - mn);
    const float p = expf(sk - mn);
    l = l * corr + p;
    m = mn;
#pragma unroll
    for (int i = 0; i < VEC; ++i) a[i] = fmaf(p, vx[i], a[i] * corr);
  }
  if (b < beams) {
    const float inv = 1.0f / l;
#pragma unroll
    for (int i = 0; i < VEC; ++i)
      store_out(out, out_big, out_small, ((long)(r0 + b) * heads + h) * HD + lane * VEC + i, a[i] * inv, xfmt);
  }
}

template <int HD, typename T>
static cudaError_t launch_decode(const void* q, const void* kp, const void* vp, const void* ks, const void* vs,
                                 const int32_t* anc, const int32_t* L_dev, int t, void* out, float* ob, float* os,
                                 int beams, int cap, int heads, int kv_heads, float scale, uint32_t* status,
                                 cudaStream_t stream, const DecodeUsers& du, int xfmt) {
  dim3 grid(heads, du.users * ((beams + DBEAMS - 1) / DBEAMS));
  return launch_pdl(PDL_ATTN, decode_attn_kernel<HD, T>, grid, dim3(ATHREADS), decode_smem_bytes<HD, T>(), stream,
                    static_cast<const T*>(q), static_cast<const T*>(kp), static_cast<const T*>(vp),
                    static_cast<const T*>(ks), static_cast<const T*>(vs), anc, L_dev, static_cast<T*>(out), ob, os,
                    beams, cap, heads, kv_heads, t, scale, status, du.users, du.prefix_user_stride,
                    du.anc_user_stride, xfmt);
}

cudaError_t attention_decode(const void* q, const void* k_prefix, const void* v_prefix, const void* k_suffix,
                             const void* v_suffix, const int32_t* anc, const int32_t* L_dev, int t, void* out,
                             float* out_big, float* out_small, int beams, int prefix_cap, int heads, int kv_heads,
                             int head_dim, float scale, uint32_t* status, bool bf16, cudaStream_t stream,
                             const DecodeUsers& du, int xfmt) {
  if (t < 1 || t > 4 || beams > MAX_BEAMS || du.users < 1) return cudaErrorInvalidValue;
  if (head_dim == 128)
    return bf16 ? launch_decode<128, __nv_bfloat16>(q, k_prefix, v_prefix, k_suffix, v_suffix, anc, L_dev, t, out,
                                                    nullptr, nullptr, beams, prefix_cap, heads, kv_heads, scale, status,
                                                    stream, du, 0)
                : launch_decode<128, float>(q, k_prefix, v_prefix, k_suffix, v_suffix, anc, L_dev, t, out, out_big,
                                            out_small, beams, prefix_cap, heads, kv_heads, scale, status, stream, du,
                                            xfmt);
  if (head_dim == 64)
    return bf16 ? launch_decode<64, __nv_bfloat16>(q, k_prefix, v_prefix, k_suffix, v_suffix, anc, L_dev, t, out,
                                                   nullptr, nullptr, beams, prefix_cap, heads, kv_heads, scale, status,
                                                   stream, du, 0)
                : launch_decode<64, float>(q, k_prefix, v_prefix, k_suffix, v_suffix, anc, L_dev, t, out, out_big,
                                           out_small, beams, prefix_cap, heads, kv_heads, scale, status, stream, du,
                                           xfmt);
  return cudaErrorInvalidValue;
}

template <int HD, typename T>
static cudaError_t attn_set_smem() {
  cudaError_t e = cudaFuncSetAttribute(prefill_attn_kernel<HD, T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)attn_smem_bytes<HD, T>(PQ));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(decode_attn_kernel<HD, T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)decode_smem_bytes<HD, T>());
  return e;
}

cudaError_t attention_init() {
  cudaError_t e = attn_set_smem<128, float>();
  if (e == cudaSuccess) e = attn_set_smem<64, float>();
  if (e == cudaSuccess) e = attn_set_smem<128, __nv_bfloat16>();
  if (e == cudaSuccess) e = attn_set_smem<64, __nv_bfloat16>();
  return e;
}

}  // namespace rtr
