// Test hook: one projection GEMM through a chosen kernel on caller-owned
// device buffers, so the kernels' numerics can be checked against a plain
// float64 product at any shape (the engine itself only calls them through its
// layer loop).  Scratch is allocated and freed per call: not for a hot path.
#include <cuda.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "engine.h"
#include "rtr_b200.h"

namespace rtr {

__global__ void split_tf32_kernel(const float* __restrict__ x, float* __restrict__ big, float* __restrict__ small,
                                  long n) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float v = x[i];
    const float b = tf32_round(v);
    big[i] = b;
    small[i] = v - b;
  }
}

__global__ void split_pair_kernel(const float* __restrict__ x, __half* __restrict__ hi, __half* __restrict__ lo,
                                  long n) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    pair_split(x[i], hi[i], lo[i]);
}

static int gemm_check_impl(int device, const float* x, const float* w, float* c, int M, int N, int K, int kernel) {
  if (!x || !w || !c || M < 1 || N < 1 || K < 1 || N % 4 || kernel < 0 || kernel > 5) return RTR_ERR_ARG;
  if (kernel == 4 && K % 32) return RTR_ERR_ARG;  // the FFMA kernel walks K in 32-wide slabs
  if (cudaSetDevice(device) != cudaSuccess) return RTR_ERR_CUDA;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return RTR_ERR_CUDA;
  if (gemm_init() != cudaSuccess || gemm_tc_init() != cudaSuccess || gemm_tc_wide_init() != cudaSuccess ||
      gemm_bf16_init() != cudaSuccess || gemm_f16x2_init() != cudaSuccess)
    return RTR_ERR_CUDA;
  // split-K partials: the tensor-core kernels split only while tiles x splits <= SMs
  const size_t ws_floats = kernel == 4 ? gemm_workspace_floats(M, N, sms) : (size_t)sms * 128 * 128;
  const int tc_tiles = ((M + 63) / 64) * ((N + 127) / 128);
  const int max_tickets = kernel == 4 ? gemm_tile_count(M, N) : tc_tiles;
  float *ws = nullptr, *xb = nullptr, *xs = nullptr, *wp = nullptr;
  void *xh = nullptr, *xh2 = nullptr, *wh = nullptr;
  int* tickets = nullptr;
  uint32_t* status = nullptr;
  cudaStream_t stream = nullptr;
  int rc = RTR_OK;
  cudaError_t e = cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMalloc(&ws, ws_floats * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&tickets, max_tickets * sizeof(int));
  if (e == cudaSuccess) e = cudaMalloc(&status, sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMemsetAsync(tickets, 0, max_tickets * sizeof(int), stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(status, 0, sizeof(uint32_t), stream);
  if (e == cudaSuccess && (kernel == 0 || kernel == 5)) {
    // the fp16-pair kernel (the engine's fp32 GEMM): activations split into
    // (hi, lo) fp16 planes, weights packed into pair blocks
    const long n = (long)M * K;
    e = cudaMalloc(&xh, n * 2);
    if (e == cudaSuccess) e = cudaMalloc(&xh2, n * 2);
    if (e == cudaSuccess) e = cudaMalloc(&wh, packed_weight_elems_f16x2(N, K) * 2);
    if (e == cudaSuccess) {
      split_pair_kernel<<<sms * 4, 256, 0, stream>>>(x, static_cast<__half*>(xh), static_cast<__half*>(xh2), n);
      e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = pack_weight_tiles_f16x2(w, N, K, wh, stream);
    TensorMap tw, txh, txl;
    if (e == cudaSuccess && (!make_tmap_packed_f16x2(&tw, wh, N, K) || !make_tmap_f16(&txh, xh, M, K, K, 64) ||
                             !make_tmap_f16(&txl, xh2, M, K, K, 64)))
      rc = RTR_ERR_ARG;  // K rows must be 16-byte aligned for TMA
    if (e == cudaSuccess && rc == RTR_OK)
      e = gemm_f16x2(tw, txh, txl, c, nullptr, nullptr, N, nullptr, M, N, K, EPI_STORE, ws, ws_floats, tickets,
                     max_tickets, status, sms, stream, false);
  } else if (e == cudaSuccess && (kernel <= 2)) {
    const long n = (long)M * K;
    e = cudaMalloc(&xb, n * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&xs, n * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&wp, packed_weight_floats(N, K) * sizeof(float));
    if (e == cudaSuccess) {
      split_tf32_kernel<<<sms * 4, 256, 0, stream>>>(x, xb, xs, n);
      e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = pack_weight_tiles(w, N, K, wp, stream);
    TensorMap tw, txb, txs;
    if (e == cudaSuccess && (!make_tmap_packed(&tw, wp, N, K) || !make_tmap_f32(&txb, xb, M, K, K, 64) ||
                             !make_tmap_f32(&txs, xs, M, K, K, 64)))
      rc = RTR_ERR_ARG;  // K rows must be 16-byte aligned for TMA
    if (e == cudaSuccess && rc == RTR_OK) {
      const bool wide = kernel == 2;
      e = wide ? gemm_tc_wide(tw, txb, txs, c, nullptr, nullptr, N, nullptr, M, N, K, EPI_STORE, ws, ws_floats,
                              tickets, max_tickets, status, sms, stream, false)
               : gemm_tc(tw, txb, txs, c, nullptr, nullptr, N, nullptr, M, N, K, EPI_STORE, ws, ws_floats, tickets,
                         max_tickets, status, sms, stream, false);
    }
  } else if (e == cudaSuccess && kernel == 3) {
    e = cudaMalloc(&xh, (size_t)M * K * 2);
    if (e == cudaSuccess) e = cudaMalloc(&wh, packed_weight_elems_bf16(N, K) * 2);
    if (e == cudaSuccess) e = f32_to_bf16(x, xh, (int64_t)M * K, stream);
    if (e == cudaSuccess) e = pack_weight_tiles_bf16(w, N, K, wh, stream);
    TensorMap tw, tx;
    if (e == cudaSuccess && (!make_tmap_packed_bf16(&tw, wh, N, K) || !make_tmap_bf16(&tx, xh, M, K, K, 64)))
      rc = RTR_ERR_ARG;
    if (e == cudaSuccess && rc == RTR_OK)
      e = gemm_bf16(tw, tx, c, N, nullptr, M, N, K, EPI_STORE, ws, ws_floats, tickets, max_tickets, status, sms,
                    stream, false);
  } else if (e == cudaSuccess) {
    e = gemm_f32(x, K, w, c, N, nullptr, M, N, K, EPI_STORE, ws, ws_floats, tickets, sms, stream, false);
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  uint32_t st = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&st, status, sizeof(st), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) rc = RTR_ERR_CUDA;
  else if (rc == RTR_OK && st != 0) rc = RTR_ERR_DEVICE;
  cudaFree(ws); cudaFree(tickets); cudaFree(status); cudaFree(xb); cudaFree(xs); cudaFree(wp);
  cudaFree(xh); cudaFree(xh2); cudaFree(wh);
  if (stream) cudaStreamDestroy(stream);
  return rc;
}

}  // namespace rtr

extern "C" int rtr_gemm_check(int32_t device, const float* x_dev, const float* w_dev, float* c_dev, int32_t M,
                              int32_t N, int32_t K, int32_t kernel) {
  return rtr::gemm_check_impl(device, x_dev, w_dev, c_dev, M, N, K, kernel);
}

extern "C" int rtr_debug_wait_control(int32_t device, int64_t wait_cycles, int32_t withhold_activation_copies) {
  if (wait_cycles < 1000 || withhold_activation_copies < 0 || withhold_activation_copies > 1) return RTR_ERR_ARG;
  if (cudaSetDevice(device) != cudaSuccess) return RTR_ERR_CUDA;
  if (rtr::gemm_f16x2_wait_control(wait_cycles, withhold_activation_copies) != cudaSuccess ||
      rtr::gemm_bf16_wait_control(wait_cycles, withhold_activation_copies) != cudaSuccess)
    return RTR_ERR_CUDA;
  return RTR_OK;
}
