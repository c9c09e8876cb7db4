// Row-wise kernels of the Qwen2 forward: embedding gather, RMSNorm, RoPE with
// the KV-cache write, the M=1 LM-head GEMV, and the synthetic weight filler.
#include <thread>
#include <vector>

#include "common.cuh"
#include "engine.h"

namespace rtr {

// ---------------------------------------------------------------- embedding
// Row m's token: ids[(m / grp_rows) * grp_stride + (m % grp_rows) * ids_stride]
// (groups: the users of a batched decode step, each with its own beam state).
__device__ __forceinline__ int row_token(const int32_t* ids, int m, int ids_stride, int grp_rows, long grp_stride) {
  return ids[(long)(m / grp_rows) * grp_stride + (long)(m % grp_rows) * ids_stride];
}

__global__ void embed_kernel(const int32_t* ids, int ids_stride, const float* table, int vocab,
                             int hidden, float* x, uint32_t* status, float* x_big, float* x_small, float* ss,
                             int ss_ld, int grp_rows, long grp_stride, int xfmt) {
  pdl_launch_dependents();
  pdl_wait();
  const int m = blockIdx.x;
  int tok = row_token(ids, m, ids_stride, grp_rows, grp_stride);
  if (tok < 0 || tok >= vocab) {
    if (threadIdx.x == 0) atomicOr(status, RTR_DEV_BAD_TOKEN);
    tok = 0;
  }
  const float4* src = reinterpret_cast<const float4*>(table + (long)tok * hidden);
  float4* dst = reinterpret_cast<float4*>(x + (long)m * hidden);
  if (!x_big) {
    for (int i = threadIdx.x; i < hidden / 4; i += blockDim.x) dst[i] = src[i];
    return;
  }
  // warp w takes 128-column chunks w, w + warps, ...: copy, split and the
  // chunk's sum of squares (lane sums of 4 squares, then a shuffle tree)
  const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
  for (int chunk = threadIdx.x >> 5; chunk < hidden / 128; chunk += warps) {
    const int i = chunk * 32 + lane;
    const float4 v = src[i];
    dst[i] = v;
    store_split4(x_big, x_small, (long)m * hidden + 4 * i, v, xfmt);
    const float sq = warp_sum((v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w));
    if (lane == 0 && ss) ss[(long)chunk * ss_ld + m] = sq;
  }
}

cudaError_t embed_rows(const int32_t* ids, int ids_stride, int M, const float* table, int vocab,
                       int hidden, float* x, uint32_t* status, cudaStream_t stream, float* x_big, float* x_small,
                       float* ss, int ss_ld, int grp_rows, long grp_stride, int xfmt) {
  if (x_big && (hidden % 128 || !x_small)) return cudaErrorInvalidValue;
  if (grp_rows <= 0) grp_rows = M;
  return launch_pdl(PDL_EMBED, embed_kernel, dim3(M), dim3(128), 0, stream, ids, ids_stride, table, vocab, hidden, x,
                    status, x_big, x_small, ss, ss_ld, grp_rows, grp_stride, xfmt);
}

// ------------------------------------------------------------------ RMSNorm
// Qwen2RMSNorm.forward (modeling_qwen2.py:258-263): w * (x * rsqrt(mean(x^2) + eps)).
__global__ void rms_norm_kernel(const float* x, const float* w, float* h, float* h_big, float* h_small, int hidden,
                                float eps, int xfmt) {
  pdl_launch_dependents();
  pdl_wait();
  const int m = blockIdx.x;
  const float4* xr = reinterpret_cast<const float4*>(x + (long)m * hidden);
  float ss = 0.f;
  for (int i = threadIdx.x; i < hidden / 4; i += blockDim.x) {
    float4 v = xr[i];
    ss = fmaf(v.x, v.x, ss); ss = fmaf(v.y, v.y, ss);
    ss = fmaf(v.z, v.z, ss); ss = fmaf(v.w, v.w, ss);
  }
  __shared__ float red[32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float r = 1.0f / sqrtf(red[0] / (float)hidden + eps);
  const float4* wr = reinterpret_cast<const float4*>(w);
  const long row = (long)m * hidden;
  for (int i = threadIdx.x; i < hidden / 4; i += blockDim.x) {
    const float4 v = xr[i], g = wr[i];
    store_split(h, h_big, h_small, row + 4 * i, g.x * (v.x * r), xfmt);
    store_split(h, h_big, h_small, row + 4 * i + 1, g.y * (v.y * r), xfmt);
    store_split(h, h_big, h_small, row + 4 * i + 2, g.z * (v.z * r), xfmt);
    store_split(h, h_big, h_small, row + 4 * i + 3, g.w * (v.w * r), xfmt);
  }
}

cudaError_t rms_norm_rows(const float* x, const float* w, float* h, float* h_big, float* h_small, int M, int hidden,
                          float eps, cudaStream_t stream, int xfmt) {
  return launch_pdl(PDL_NORM, rms_norm_kernel, dim3(M), dim3(256), 0, stream, x, w, h, h_big, h_small, hidden, eps,
                    xfmt);
}

// ------------------------------------------------------------- bf16 mode
// The bf16 model of the reference's bf16-experimental opt-in: embeddings,
// residual stream and norms in bf16, reductions in fp32.
__global__ void embed_bf16_kernel(const int32_t* ids, int ids_stride, const __nv_bfloat16* table, int vocab,
                                  int hidden, __nv_bfloat16* x, uint32_t* status, int grp_rows, long grp_stride) {
  pdl_launch_dependents();
  pdl_wait();
  const int m = blockIdx.x;
  int tok = row_token(ids, m, ids_stride, grp_rows, grp_stride);
  if (tok < 0 || tok >= vocab) {
    if (threadIdx.x == 0) atomicOr(status, RTR_DEV_BAD_TOKEN);
    tok = 0;
  }
  const uint4* src = reinterpret_cast<const uint4*>(table + (long)tok * hidden);
  uint4* dst = reinterpret_cast<uint4*>(x + (long)m * hidden);
  for (int i = threadIdx.x; i < hidden / 8; i += blockDim.x) dst[i] = src[i];
}

cudaError_t embed_rows_bf16(const int32_t* ids, int ids_stride, int M, const void* table, int vocab, int hidden,
                            void* x, uint32_t* status, cudaStream_t stream, int grp_rows, long grp_stride) {
  if (grp_rows <= 0) grp_rows = M;
  return launch_pdl(PDL_EMBED, embed_bf16_kernel, dim3(M), dim3(128), 0, stream, ids, ids_stride,
                    static_cast<const __nv_bfloat16*>(table), vocab, hidden, static_cast<__nv_bfloat16*>(x), status,
                    grp_rows, grp_stride);
}

// Qwen2RMSNorm on a bf16 model (modeling_qwen2.py:258-263): the variance in
// fp32, then weight * bf16(x * rsqrt(var + eps)) rounded to bf16; w holds the
// bf16 norm weights as fp32.
// One CTA (256 threads) per row.  The weights (constants) are loaded before
// the wait for the previous kernel and the row stays in registers, so the
// only dependent global round trips are the row's load and the store; the
// sum of squares runs in the same order for every hidden size.
constexpr int NORM16_THREADS = 256, NORM16_PAIRS = 8;  // hidden <= 2 * 8 * 256 = 4096
__global__ void __launch_bounds__(NORM16_THREADS)
    rms_norm_bf16_kernel(const __nv_bfloat16* x, const float* w, __nv_bfloat16* h, int hidden, float eps) {
  const int npair = hidden / 2;
  float2 wv[NORM16_PAIRS];
#pragma unroll
  for (int t = 0; t < NORM16_PAIRS; ++t) {
    const int i = threadIdx.x + t * NORM16_THREADS;
    wv[t] = i < npair ? make_float2(w[2 * i], w[2 * i + 1]) : make_float2(0.f, 0.f);
  }
  pdl_launch_dependents();
  pdl_wait();
  const int m = blockIdx.x;
  const __nv_bfloat162* xr = reinterpret_cast<const __nv_bfloat162*>(x + (long)m * hidden);
  float2 xv[NORM16_PAIRS];
#pragma unroll
  for (int t = 0; t < NORM16_PAIRS; ++t) {
    const int i = threadIdx.x + t * NORM16_THREADS;
    xv[t] = i < npair ? __bfloat1622float2(xr[i]) : make_float2(0.f, 0.f);
  }
  float ss = 0.f;
#pragma unroll
  for (int t = 0; t < NORM16_PAIRS; ++t) {
    if (threadIdx.x + t * NORM16_THREADS < npair) {
      ss = fmaf(xv[t].x, xv[t].x, ss);
      ss = fmaf(xv[t].y, xv[t].y, ss);
    }
  }
  __shared__ float red[32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (NORM16_THREADS >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float r = 1.0f / sqrtf(red[0] / (float)hidden + eps);
  __nv_bfloat162* hr = reinterpret_cast<__nv_bfloat162*>(h + (long)m * hidden);
#pragma unroll
  for (int t = 0; t < NORM16_PAIRS; ++t) {
    const int i = threadIdx.x + t * NORM16_THREADS;
    if (i < npair) hr[i] = __floats2bfloat162_rn(wv[t].x * bf16_round(xv[t].x * r), wv[t].y * bf16_round(xv[t].y * r));
  }
}

cudaError_t rms_norm_rows_bf16(const void* x, const float* w, void* h, int M, int hidden, float eps,
                               cudaStream_t stream) {
  if (hidden % 2 || hidden > 2 * NORM16_PAIRS * NORM16_THREADS) return cudaErrorInvalidValue;
  return launch_pdl(PDL_NORM16, rms_norm_bf16_kernel, dim3(M), dim3(NORM16_THREADS), 0, stream,
                    static_cast<const __nv_bfloat16*>(x), w, static_cast<__nv_bfloat16*>(h), hidden, eps);
}

// y[n] = float(bf16(dot(x, W[n]))) for the prefill's last-row LM head: bf16
// weights and activations, fp32 accumulation, logits rounded like a bf16 model's.
__global__ void gemv_bf16_kernel(const __nv_bfloat16* x, const __nv_bfloat16* W, float* y, int N, int K) {
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ float xs[];
  for (int i = threadIdx.x; i < K; i += blockDim.x) xs[i] = __bfloat162float(x[i]);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows_per_warp = 4;
  const int n0 = (blockIdx.x * (blockDim.x >> 5) + warp) * rows_per_warp;
#pragma unroll
  for (int r = 0; r < rows_per_warp; ++r) {
    const int n = n0 + r;
    if (n >= N) return;
    const __nv_bfloat162* w = reinterpret_cast<const __nv_bfloat162*>(W + (long)n * K);
    float acc = 0.f;
    for (int k = lane; k < K / 2; k += 32) {
      const float2 a = __bfloat1622float2(w[k]);
      acc = fmaf(a.x, xs[2 * k], acc);
      acc = fmaf(a.y, xs[2 * k + 1], acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) y[n] = bf16_round(acc);
  }
}

cudaError_t gemv_bf16(const void* x, const void* W, float* y, int N, int K, cudaStream_t stream) {
  const int threads = 256, rows_per_block = (threads / 32) * 4;
  return launch_pdl(PDL_GEMV, gemv_bf16_kernel, dim3((N + rows_per_block - 1) / rows_per_block), dim3(threads),
                    K * sizeof(float), stream, static_cast<const __nv_bfloat16*>(x),
                    static_cast<const __nv_bfloat16*>(W), y, N, K);
}

// fp32 -> bf16-rounded fp32 (biases and norm weights of the bf16 mode)
__global__ void round_bf16_kernel(float* v, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    v[i] = bf16_round(v[i]);
}

cudaError_t round_to_bf16(float* v, int64_t n, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  int blocks = (int)((n + 255) / 256);
  if (blocks > 148 * 8) blocks = 148 * 8;
  round_bf16_kernel<<<blocks, 256, 0, stream>>>(v, n);
  return cudaGetLastError();
}

// --------------------------------------------------------------------- RoPE
// apply_rotary_pos_emb (modeling_qwen2.py:116-146): out = x*cos + rotate_half(x)*sin
// with separately rounded products, as the CPU reference evaluates it.
__global__ void rope_kv_kernel(const float* qkv, int heads, int kv_heads, int head_dim,
                               const float* cos_t, const float* sin_t, int rope_positions,
                               float* q_out, float* k_dst, float* v_dst, int prefix_cap, int slot,
                               const int32_t* L_dev, uint32_t* status) {
  pdl_launch_dependents();
  pdl_wait();
  const int m = blockIdx.x;
  const int half = head_dim / 2;
  const int qkv_dim = (heads + 2 * kv_heads) * head_dim;
  int pos = slot < 0 ? m : (*L_dev + slot);
  if (pos < 0 || pos >= rope_positions) {
    if (threadIdx.x == 0) atomicOr(status, RTR_DEV_BAD_LENGTH);
    pos = 0;
  }
  const float* row = qkv + (long)m * qkv_dim;
  const float* c = cos_t + (long)pos * half;
  const float* s = sin_t + (long)pos * half;
  // rotary pairs of q and k heads
  const int pairs = (heads + kv_heads) * half;
  for (int i = threadIdx.x; i < pairs; i += blockDim.x) {
    const int head = i / half, d = i % half;
    const float* src = row + head * head_dim;
    const float x1 = src[d], x2 = src[d + half];
    const float cc = c[d], ss = s[d];
    const float o1 = __fadd_rn(__fmul_rn(x1, cc), __fmul_rn(-x2, ss));
    const float o2 = __fadd_rn(__fmul_rn(x2, cc), __fmul_rn(x1, ss));
    if (head < heads) {
      float* dst = q_out + (long)m * heads * head_dim + head * head_dim;
      dst[d] = o1; dst[d + half] = o2;
    } else {
      const int g = head - heads;
      float* dst = slot < 0 ? k_dst + ((long)g * prefix_cap + m) * head_dim
                            : k_dst + ((long)m * kv_heads + g) * head_dim;
      dst[d] = o1; dst[d + half] = o2;
    }
  }
  const float* vsrc = row + (heads + kv_heads) * head_dim;
  for (int i = threadIdx.x; i < kv_heads * head_dim; i += blockDim.x) {
    const int g = i / head_dim, d = i % head_dim;
    float* dst = slot < 0 ? v_dst + ((long)g * prefix_cap + m) * head_dim
                          : v_dst + ((long)m * kv_heads + g) * head_dim;
    dst[d] = vsrc[i];
  }
}

cudaError_t rope_kv(const float* qkv, int M, int heads, int kv_heads, int head_dim,
                    const float* cos_t, const float* sin_t, int rope_positions,
                    float* q_out, float* k_dst, float* v_dst, int prefix_cap,
                    int slot, const int32_t* L_dev, uint32_t* status, cudaStream_t stream) {
  return launch_pdl(PDL_ROPE, rope_kv_kernel, dim3(M), dim3(256), 0, stream, qkv, heads, kv_heads, head_dim, cos_t, sin_t,
                    rope_positions, q_out, k_dst, v_dst, prefix_cap, slot, L_dev, status);
}

// --------------------------------------------------------------------- GEMV
// y[n] = dot(x, W[n]) for the last-token LM head of the prefill (M = 1).
__global__ void gemv_kernel(const float* x, const float* W, float* y, int N, int K) {
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ float xs[];
  for (int i = threadIdx.x; i < K; i += blockDim.x) xs[i] = x[i];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows_per_warp = 4;
  const int n0 = (blockIdx.x * (blockDim.x >> 5) + warp) * rows_per_warp;
#pragma unroll
  for (int r = 0; r < rows_per_warp; ++r) {
    const int n = n0 + r;
    if (n >= N) return;
    const float4* w = reinterpret_cast<const float4*>(W + (long)n * K);
    float acc = 0.f;
    for (int k = lane; k < K / 4; k += 32) {
      float4 a = w[k];
      acc = fmaf(a.x, xs[4 * k], acc);
      acc = fmaf(a.y, xs[4 * k + 1], acc);
      acc = fmaf(a.z, xs[4 * k + 2], acc);
      acc = fmaf(a.w, xs[4 * k + 3], acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) y[n] = acc;
  }
}

cudaError_t gemv_f32(const float* x, const float* W, float* y, int N, int K, cudaStream_t stream) {
  const int threads = 256, rows_per_block = (threads / 32) * 4;
  return launch_pdl(PDL_GEMV, gemv_kernel, dim3((N + rows_per_block - 1) / rows_per_block), dim3(threads), K * sizeof(float),
                    stream, x, W, y, N, K);
}

// ------------------------------------------------------- synthetic weights
// Counter-based splitmix64 stream; (k - 2^23) * (scale * 2^-23) + offset with
// k the top 24 bits: one exact conversion and two IEEE roundings, identical on
// host and device.
__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}
__host__ __device__ __forceinline__ uint64_t stream_key(uint64_t seed, uint64_t tid) {
  return mix64(seed * 0x9E3779B97F4A7C15ULL + tid * 0xD1B54A32D192ED03ULL + 1ULL);
}

__global__ void synth_kernel(float* dst, int64_t n, uint64_t key, float step, float offset) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t z = mix64(key + (uint64_t)i * 0x9E3779B97F4A7C15ULL);
    const float k = (float)((int32_t)(z >> 40) - (1 << 23));
    dst[i] = __fadd_rn(__fmul_rn(k, step), offset);
  }
}

static float synth_step(float scale) { return scale * (1.0f / 8388608.0f); }

cudaError_t synth_fill_device(float* dst, int64_t n, uint64_t seed, uint64_t tid, float scale,
                              float offset, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  int blocks = (int)((n + 255) / 256);
  if (blocks > 148 * 32) blocks = 148 * 32;
  synth_kernel<<<blocks, 256, 0, stream>>>(dst, n, stream_key(seed, tid), synth_step(scale), offset);
  return cudaGetLastError();
}

void synth_fill_host(float* dst, int64_t n, uint64_t seed, uint64_t tid, float scale, float offset) {
  const uint64_t key = stream_key(seed, tid);
  const float step = synth_step(scale);
  unsigned hw = std::thread::hardware_concurrency();
  int workers = (int)(hw ? hw : 4);
  if (n < (1 << 20)) workers = 1;
  auto work = [&](int64_t lo, int64_t hi) {
    for (int64_t i = lo; i < hi; ++i) {
      const uint64_t z = mix64(key + (uint64_t)i * 0x9E3779B97F4A7C15ULL);
      const float k = (float)((int32_t)(z >> 40) - (1 << 23));
      volatile float prod = k * step;  // keep the two roundings separate
      dst[i] = prod + offset;
    }
  };
  std::vector<std::thread> pool;
  for (int w = 0; w < workers; ++w) {
    const int64_t lo = n * w / workers, hi = n * (w + 1) / workers;
    if (workers == 1) { work(lo, hi); break; }
    pool.emplace_back(work, lo, hi);
  }
  for (auto& t : pool) t.join();
}

__global__ void f32_to_bf16_kernel(const float* src, __nv_bfloat16* dst, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = __float2bfloat16_rn(src[i]);
}

cudaError_t f32_to_bf16(const float* src, void* dst, int64_t n, cudaStream_t stream) {
  int blocks = (int)((n + 255) / 256);
  if (blocks > 148 * 32) blocks = 148 * 32;
  if (blocks < 1) blocks = 1;
  f32_to_bf16_kernel<<<blocks, 256, 0, stream>>>(src, static_cast<__nv_bfloat16*>(dst), n);
  return cudaGetLastError();
}

}  // namespace rtr
