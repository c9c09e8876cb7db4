// Attention kernels for the shared-prefix beam path (FP32, head_dim 64/128).
//
// Prefill: causal GQA attention of one request (sdpa_attention_forward with
// is_causal=True, transformers integrations/sdpa_attention.py:40-104).  A CTA
// owns 32 query positions of one query head, register-tiled (below).
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
// banks), with an online softmax over each query row.
#include <math.h>

#include "common.cuh"
#include "engine.h"

namespace rtr {

constexpr int AK = 64;         // keys per chunk
constexpr int AWARPS = 8;      // warps per CTA
constexpr int ATHREADS = AWARPS * 32;
constexpr int PT_Q = 32;       // prefill query positions per CTA
constexpr int DBEAMS = AWARPS; // decode beams per CTA (1 per warp)

// Prefix K/V rows are staged in their storage type T (fp32, or bf16 in the
// bf16 mode); K rows are padded so 16-byte copies stay aligned and the score
// reads of consecutive keys spread over the banks.  q lives in fp32.
template <int HD, typename T> __host__ __device__ constexpr int kld() { return HD + 16 / (int)sizeof(T); }

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

// ------------------------------------------------------------------ prefill
// Register-tiled causal attention: a CTA owns PT_Q = 32 query rows of one
// query head and walks the keys in staged 64-key chunks.  Thread (ty, tx) =
// (tid / 16, tid % 16) owns rows 2 ty, 2 ty + 1:
//   scores  keys tx + 16 j (j < 4): a 2 x 4 tile, per 4 dimensions two q
//           float4 and four K float4 loads for 32 FMAs (K rows padded so the
//           16 keys of a half-warp hit distinct banks; the other half-warp
//           reads the same keys)
//   softmax online per row across the 16 lanes of the half-warp (shuffles)
//   P.V     P goes through shared memory; dimensions 4 tx .. 4 tx + 3 (and
//           + 64 for head_dim 128): per 4 keys two P float4 and HD / 64 * 4 V
//           float4 loads for HD / 2 FMAs
template <int HD, typename T> constexpr size_t prefill_smem_bytes() {
  return (size_t)(2 * AK * kld<HD, T>() + 2 * AK * HD) * sizeof(T) +
         (size_t)(PT_Q * (HD + 4) + PT_Q * (AK + 4)) * sizeof(float);
}

template <int HD, typename T>
__global__ void __launch_bounds__(ATHREADS, 1) prefill_attn_kernel(
    const T* __restrict__ q, const T* __restrict__ kp, const T* __restrict__ vp,
    T* __restrict__ out, float* __restrict__ out_big, float* __restrict__ out_small, int L, int cap, int heads,
    int kv_heads, float scale, int xfmt) {
  constexpr int QLD = HD + 4, PLD = AK + 4, KLD = kld<HD, T>();
  constexpr int NV = HD / 64;  // float4 column groups of the output per thread
  static_assert(ATHREADS == 256 && PT_Q == 32 && AK == 64, "tiling assumes 256 threads, 32 rows, 64 keys");
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ __align__(16) unsigned char asmem[];
  T* kbuf = reinterpret_cast<T*>(asmem);
  T* vbuf = kbuf + 2 * AK * KLD;
  float* qs = reinterpret_cast<float*>(vbuf + 2 * AK * HD);  // [PT_Q][QLD]
  float* ps = qs + PT_Q * QLD;                                // [PT_Q][PLD]
  const int h = blockIdx.y, g = h / (heads / kv_heads);
  const int q0 = blockIdx.x * PT_Q;
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
  const int r0 = 2 * ty;
  const T* kbase = kp + (long)g * cap * HD;
  const T* vbase = vp + (long)g * cap * HD;
  const int kend = min(L, q0 + PT_Q);  // keys any row of the block may see
  const int nchunks = (kend + AK - 1) / AK;
  // last key of each row (padding rows past L see key 0 only: their values are never stored)
  int klast[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) klast[i] = q0 + r0 + i < L ? q0 + r0 + i : 0;

  load_kv_chunk<HD, T>(kbuf, vbuf, kbase, vbase, 0, kend, 0);
  for (int i = threadIdx.x; i < PT_Q * HD / 4; i += ATHREADS) {
    const int r = i / (HD / 4), d = (i % (HD / 4)) * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (q0 + r < L) v = ld4f(q + ((long)(q0 + r) * heads + h) * HD + d);
    *reinterpret_cast<float4*>(qs + r * QLD + d) = v;
  }
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f}, acc[2][4 * NV];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int e = 0; e < 4 * NV; ++e) acc[i][e] = 0.f;

  for (int c = 0; c < nchunks; ++c) {
    if (c + 1 < nchunks) load_kv_chunk<HD, T>(kbuf, vbuf, kbase, vbase, (c + 1) * AK, kend, (c + 1) & 1);
    else cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const T* kc = kbuf + (c & 1) * AK * KLD;
    const T* vc = vbuf + (c & 1) * AK * HD;
    // ---- scores: rows r0, r0 + 1 x keys tx + 16 j
    float sc[2][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) sc[i][j] = 0.f;
#pragma unroll 4
    for (int d = 0; d < HD; d += 4) {
      const float4 qa = *reinterpret_cast<const float4*>(qs + r0 * QLD + d);
      const float4 qb = *reinterpret_cast<const float4*>(qs + (r0 + 1) * QLD + d);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 k = ld4f(kc + (tx + 16 * j) * KLD + d);
        sc[0][j] = fmaf(qa.x, k.x, sc[0][j]); sc[0][j] = fmaf(qa.y, k.y, sc[0][j]);
        sc[0][j] = fmaf(qa.z, k.z, sc[0][j]); sc[0][j] = fmaf(qa.w, k.w, sc[0][j]);
        sc[1][j] = fmaf(qb.x, k.x, sc[1][j]); sc[1][j] = fmaf(qb.y, k.y, sc[1][j]);
        sc[1][j] = fmaf(qb.z, k.z, sc[1][j]); sc[1][j] = fmaf(qb.w, k.w, sc[1][j]);
      }
    }
    // ---- online softmax per row over the half-warp's 64 keys
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int key = c * AK + tx + 16 * j;
        sc[i][j] = key <= klast[i] ? sc[i][j] * scale : -INFINITY;
        mx = fmaxf(mx, sc[i][j]);
      }
#pragma unroll
      for (int o = 8; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float mn = fmaxf(m[i], mx);  // finite: key 0 is valid for every row
      const float corr = expf(m[i] - mn);
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float pv = expf(sc[i][j] - mn);
        sum += pv;
        ps[(r0 + i) * PLD + tx + 16 * j] = pv;
      }
#pragma unroll
      for (int o = 8; o >= 1; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      l[i] = l[i] * corr + sum;
      m[i] = mn;
#pragma unroll
      for (int e = 0; e < 4 * NV; ++e) acc[i][e] *= corr;
    }
    __syncthreads();  // P of the whole tile is in shared memory
    // ---- P.V: rows r0, r0 + 1 x dimensions 4 tx + 64 n (n < NV)
#pragma unroll 2
    for (int k4 = 0; k4 < AK; k4 += 4) {
      const float4 pa = *reinterpret_cast<const float4*>(ps + r0 * PLD + k4);
      const float4 pb = *reinterpret_cast<const float4*>(ps + (r0 + 1) * PLD + k4);
      const float pav[4] = {pa.x, pa.y, pa.z, pa.w}, pbv[4] = {pb.x, pb.y, pb.z, pb.w};
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
        for (int n = 0; n < NV; ++n) {
          const float4 v = ld4f(vc + (k4 + kk) * HD + n * 64 + 4 * tx);
          acc[0][4 * n] = fmaf(pav[kk], v.x, acc[0][4 * n]);
          acc[0][4 * n + 1] = fmaf(pav[kk], v.y, acc[0][4 * n + 1]);
          acc[0][4 * n + 2] = fmaf(pav[kk], v.z, acc[0][4 * n + 2]);
          acc[0][4 * n + 3] = fmaf(pav[kk], v.w, acc[0][4 * n + 3]);
          acc[1][4 * n] = fmaf(pbv[kk], v.x, acc[1][4 * n]);
          acc[1][4 * n + 1] = fmaf(pbv[kk], v.y, acc[1][4 * n + 1]);
          acc[1][4 * n + 2] = fmaf(pbv[kk], v.z, acc[1][4 * n + 2]);
          acc[1][4 * n + 3] = fmaf(pbv[kk], v.w, acc[1][4 * n + 3]);
        }
      }
    }
    __syncthreads();  // the K/V slot and P are refilled by the next iteration
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int qpos = q0 + r0 + i;
    if (qpos >= L) continue;
    const float inv = 1.0f / l[i];
#pragma unroll
    for (int n = 0; n < NV; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e)
        store_out(out, out_big, out_small, ((long)qpos * heads + h) * HD + n * 64 + 4 * tx + e, acc[i][4 * n + e] * inv,
                  xfmt);
  }
}

template <int HD, typename T>
static cudaError_t launch_prefill(const void* q, const void* kp, const void* vp, void* out, float* ob, float* os, int L,
                                  int cap, int heads, int kv_heads, float scale, cudaStream_t stream, int xfmt) {
  dim3 grid((L + PT_Q - 1) / PT_Q, heads);
  return launch_pdl(PDL_ATTN, prefill_attn_kernel<HD, T>, grid, dim3(ATHREADS), prefill_smem_bytes<HD, T>(), stream,
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
  // batched decode: user u owns rows u * beams .. (its own prefix, length and ancestry)
  const int gpu = (beams + DBEAMS - 1) / DBEAMS, u = blockIdx.y / gpu;
  // the prompt length is copied in before the request's first kernel: read before the wait
  int L = L_dev[u];
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
  const int b0 = (blockIdx.y % gpu) * DBEAMS, r0 = u * beams, rows = users * beams;
  anc += (long)u * anc_user_stride;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
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
                                       (int)prefill_smem_bytes<HD, T>());
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
