// Test hook: one causal prefill attention (one layer, one user) through a
// chosen kernel on caller-owned fp32 device buffers, so the attention kernels
// can be checked against a plain float64 product at any prompt length,
// including the lengths the workloads never produce (1, 63, 64, 65, ...).  It
// builds the operands each kernel reads in a request - the prefix arena, the
// fp16-pair copies of K and V^T, the bf16 arena and V^T copy - with small
// kernels of its own.  Scratch is allocated and freed per call: not for a hot
// path.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "engine.h"
#include "rtr_b200.h"

namespace rtr {

// k, v [kv][L][D] fp32 -> the arena [K|V][kv][cap][D] (fp32 or bf16), the
// K pair planes [kv][pc][D] and the V^T planes [kv][D][pc] (fp16 pairs, or
// bf16 in `vt_bf`), every copy the kernel under test reads.
__global__ void attn_check_stage_kernel(const float* __restrict__ k, const float* __restrict__ v, int L, int kv,
                                        int D, int cap, int pc, float* arena32, __nv_bfloat16* arena16,
                                        __half* kp_hi, __half* kp_lo, __half* vt_hi, __half* vt_lo,
                                        __nv_bfloat16* vt_bf) {
  const long n = (long)kv * L * D;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const int d = (int)(i % D), key = (int)((i / D) % L), g = (int)(i / ((long)D * L));
    const float kx = k[i], vx = v[i];
    const long ak = ((long)g * cap + key) * D + d, av = ((long)(kv + g) * cap + key) * D + d;
    if (arena32) {
      arena32[ak] = kx;
      arena32[av] = vx;
    }
    if (arena16) {
      arena16[ak] = __float2bfloat16_rn(kx);
      arena16[av] = __float2bfloat16_rn(vx);
    }
    if (kp_hi) {
      __half h, l;
      pair_split(kx, h, l);
      kp_hi[((long)g * pc + key) * D + d] = h;
      kp_lo[((long)g * pc + key) * D + d] = l;
      pair_split(vx, h, l);
      vt_hi[((long)g * D + d) * pc + key] = h;
      vt_lo[((long)g * D + d) * pc + key] = l;
    }
    if (vt_bf) vt_bf[((long)g * D + d) * pc + key] = __float2bfloat16_rn(vx);
  }
}

__global__ void attn_check_to_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, long n) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    y[i] = __float2bfloat16_rn(x[i]);
}
__global__ void attn_check_from_bf16_kernel(const __nv_bfloat16* __restrict__ x, float* __restrict__ y, long n) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    y[i] = __bfloat162float(x[i]);
}

static int attention_check_impl(int device, const float* q, const float* k, const float* v, float* out, int L,
                                int heads, int kv, int D, int kernel) {
  if (!q || !k || !v || !out || L < 1 || heads < 1 || kv < 1 || heads % kv || (D != 64 && D != 128) || kernel < 0 ||
      kernel > 3)
    return RTR_ERR_ARG;
  if ((kernel == 1 || kernel == 3) && !attention_prefill_tc_supported(heads, kv, D)) return RTR_ERR_ARG;
  if (cudaSetDevice(device) != cudaSuccess) return RTR_ERR_CUDA;
  if (attention_init() != cudaSuccess || attention_tc_init() != cudaSuccess) return RTR_ERR_CUDA;
  const bool bf = kernel >= 2, tc = kernel == 1 || kernel == 3;
  const int cap = L, pc = (L + 63) / 64 * 64;
  const long nq = (long)L * heads * D, narena = 2L * kv * cap * D, nplane = (long)kv * pc * D;
  const float scale = (float)(1.0 / sqrt((double)D));
  float* arena32 = nullptr;
  __nv_bfloat16 *arena16 = nullptr, *q16 = nullptr, *o16 = nullptr, *vt_bf = nullptr;
  __half* pairs = nullptr;  // K hi, K lo, V^T hi, V^T lo
  uint32_t* status = nullptr;
  cudaStream_t stream = nullptr;
  int rc = RTR_OK;
  cudaError_t e = cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMalloc(&status, sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMemsetAsync(status, 0, sizeof(uint32_t), stream);
  if (e == cudaSuccess && !bf) e = cudaMalloc(&arena32, narena * sizeof(float));
  if (e == cudaSuccess && bf) e = cudaMalloc(&arena16, narena * sizeof(__nv_bfloat16));
  if (e == cudaSuccess && bf) e = cudaMalloc(&q16, nq * sizeof(__nv_bfloat16));
  if (e == cudaSuccess && bf) e = cudaMalloc(&o16, nq * sizeof(__nv_bfloat16));
  if (e == cudaSuccess && kernel == 1) e = cudaMalloc(&pairs, 4 * nplane * sizeof(__half));
  if (e == cudaSuccess && kernel == 1) e = cudaMemsetAsync(pairs, 0, 4 * nplane * sizeof(__half), stream);
  if (e == cudaSuccess && kernel == 3) e = cudaMalloc(&vt_bf, nplane * sizeof(__nv_bfloat16));
  if (e == cudaSuccess && kernel == 3) e = cudaMemsetAsync(vt_bf, 0, nplane * sizeof(__nv_bfloat16), stream);
  if (e == cudaSuccess) {
    attn_check_stage_kernel<<<256, 256, 0, stream>>>(
        k, v, L, kv, D, cap, pc, arena32, arena16, pairs, pairs ? pairs + nplane : nullptr,
        pairs ? pairs + 2 * nplane : nullptr, pairs ? pairs + 3 * nplane : nullptr, vt_bf);
    if (bf) attn_check_to_bf16_kernel<<<256, 256, 0, stream>>>(q, q16, nq);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) {
    if (kernel == 0) {
      e = attention_prefill(q, arena32, arena32 + (long)kv * cap * D, out, nullptr, nullptr, L, cap, heads, kv, D,
                            scale, false, stream, 0);
    } else if (kernel == 2) {
      e = attention_prefill(q16, arena16, arena16 + (long)kv * cap * D, o16, nullptr, nullptr, L, cap, heads, kv, D,
                            scale, true, stream, 0);
    } else if (kernel == 1) {
      AttnPairs ap = {};
      ap.pair_cap = pc;
      ap.kplane = (long)kv * pc;
      ap.vplane = (long)kv * D;
      if (!make_tmap_f16(&ap.kmap, pairs, 2 * ap.kplane, D, D, 64) ||
          !make_tmap_f16(&ap.vmap, pairs + 2 * nplane, 2 * ap.vplane, pc, pc, D))
        rc = RTR_ERR_CUDA;
      else
        e = attention_prefill_tc(ap, 0, q, out, nullptr, nullptr, L, heads, kv, D, scale, status, stream, 0);
    } else {
      BfPrefillMaps mp = {};
      mp.pair_cap = pc;
      if (!make_tmap_bf16(&mp.kmap, arena16, 2L * kv * cap, D, D, 64) ||
          !make_tmap_bf16(&mp.vmap, vt_bf, (long)kv * D, pc, pc, D))
        rc = RTR_ERR_CUDA;
      else
        e = attention_prefill_tc_bf16(mp, 0, 0, 1, q16, o16, L, heads, kv, D, cap, scale, status, stream);
    }
  }
  if (e == cudaSuccess && rc == RTR_OK && bf) {
    attn_check_from_bf16_kernel<<<256, 256, 0, stream>>>(o16, out, nq);
    e = cudaGetLastError();
  }
  uint32_t st = 0;
  if (e == cudaSuccess && rc == RTR_OK) e = cudaMemcpyAsync(&st, status, sizeof(st), cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) rc = e == cudaErrorInvalidValue ? RTR_ERR_ARG : RTR_ERR_CUDA;
  else if (rc == RTR_OK && st) rc = RTR_ERR_DEVICE;
  cudaFree(arena32);
  cudaFree(arena16);
  cudaFree(q16);
  cudaFree(o16);
  cudaFree(vt_bf);
  cudaFree(pairs);
  cudaFree(status);
  if (stream) cudaStreamDestroy(stream);
  return rc;
}

}  // namespace rtr

extern "C" int rtr_attention_check(int32_t device, const float* q_dev, const float* k_dev, const float* v_dev,
                                   float* out_dev, int32_t L, int32_t heads, int32_t kv_heads, int32_t head_dim,
                                   int32_t kernel) {
  return rtr::attention_check_impl(device, q_dev, k_dev, v_dev, out_dev, L, heads, kv_heads, head_dim, kernel);
}
