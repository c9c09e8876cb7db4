// Shared device helpers for the sm_100a kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <utility>

#define RTR_DEVICE __device__ __forceinline__

// Device-side status bits written to the session's status word.  Kernels
// never trap: a failed bound check records a bit and skips the access.
enum : uint32_t {
  RTR_DEV_BAD_TOKEN = 1u << 0,      // token id outside [0, vocab)
  RTR_DEV_BAD_PARENT = 1u << 1,     // parent index outside [0, beams)
  RTR_DEV_NOT_STOPPED = 1u << 2,    // beam loop would continue after 5 steps
  RTR_DEV_STOPPED_EARLY = 1u << 3,  // beam loop would stop before 5 steps
  RTR_DEV_FEW_FINITE = 1u << 4,     // fewer finite candidates than beams
  RTR_DEV_BAD_LENGTH = 1u << 5,     // prefix length outside the arena
  RTR_DEV_TOO_MANY_CAND = 1u << 6,  // candidate buffer overflow
  RTR_DEV_NAN_SCORE = 1u << 7,      // a NaN score (ranked as -inf)
  RTR_DEV_TIMEOUT = 1u << 8,        // a bounded pipeline wait expired (kernel gave up)
};

RTR_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

RTR_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Order-preserving map float -> uint32 (larger float -> larger key; -0 < +0).
RTR_DEVICE uint32_t float_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

RTR_DEVICE float key_float(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

RTR_DEVICE float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Round to the nearest tf32 value (ties away from zero): the low 13 mantissa
// bits are clear, so a tensor core reads it exactly.
RTR_DEVICE float tf32_round(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// GEMM operand split of an activation, in one of two formats:
//   SPLIT_TF32  big = tf32(x), small = x - big (both exact fp32; the 3xTF32
//               kernels read them from fp32 planes)
//   SPLIT_F16   x = 16 (hi + lo / 2048) with hi = fp16(x / 16) and
//               lo = fp16((x / 16 - hi) * 2048): two fp16 planes (the first
//               half of the big/small allocations) for the fp16-pair kernel.
//               22 significant bits for |x| up to 16 * 65504.
enum : int { SPLIT_TF32 = 0, SPLIT_F16 = 1 };
constexpr float kPairScale = 16.0f;       // activations enter the fp16 pair scaled by 1/16
constexpr float kPairLo = 2048.0f;        // lo carries the remainder scaled by 2^11

RTR_DEVICE void pair_split(float x, __half& hi, __half& lo) {
  const float xs = x * (1.0f / kPairScale);
  hi = __float2half_rn(xs);
  lo = __float2half_rn((xs - __half2float(hi)) * kPairLo);  // xs - hi is exact
}

// Store x and its split when the split outputs are present; the tensor-core
// GEMMs consume the split pair.
RTR_DEVICE void store_split(float* out, float* big, float* small, long i, float x, int fmt = SPLIT_TF32) {
  out[i] = x;
  if (big) {
    if (fmt == SPLIT_F16) {
      __half h, l;
      pair_split(x, h, l);
      reinterpret_cast<__half*>(big)[i] = h;
      reinterpret_cast<__half*>(small)[i] = l;
    } else {
      const float b = tf32_round(x);
      big[i] = b;
      small[i] = x - b;
    }
  }
}

// The split of four consecutive elements [i, i + 4) (i a multiple of 4).
RTR_DEVICE void store_split4(float* big, float* small, long i, float4 v, int fmt) {
  if (fmt == SPLIT_F16) {
    __align__(8) __half h[4];
    __align__(8) __half l[4];
    pair_split(v.x, h[0], l[0]); pair_split(v.y, h[1], l[1]);
    pair_split(v.z, h[2], l[2]); pair_split(v.w, h[3], l[3]);
    *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(big) + i) = *reinterpret_cast<const uint2*>(h);
    *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(small) + i) = *reinterpret_cast<const uint2*>(l);
  } else {
    const float4 b = make_float4(tf32_round(v.x), tf32_round(v.y), tf32_round(v.z), tf32_round(v.w));
    *reinterpret_cast<float4*>(big + i) = b;
    *reinterpret_cast<float4*>(small + i) = make_float4(v.x - b.x, v.y - b.y, v.z - b.z, v.w - b.w);
  }
}

// Element load/store for the two activation/weight types.
template <typename T> RTR_DEVICE float to_f32(T v);
template <> RTR_DEVICE float to_f32<float>(float v) { return v; }
template <> RTR_DEVICE float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T> RTR_DEVICE T from_f32(float v);
template <> RTR_DEVICE float from_f32<float>(float v) { return v; }
template <> RTR_DEVICE __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

RTR_DEVICE void cp_async16(void* smem, const void* gmem, bool pred) {
  unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(n));
}
RTR_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N> RTR_DEVICE void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue, and wait for the previous kernel's memory before reading it.
RTR_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
RTR_DEVICE void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;\n" ::); }

// Programmatic dependent launch (PDL) policy per kernel class.  RTR_PDL is a
// comma-separated list of classes launched with PDL ("gemm", "norm" (fp32
// RMSNorm), "rope", "attn", "embed", "gemv", "tail", "rms16" (the bf16 mode's
// RMSNorm)), "0" for none, "all" for every class.  Read once per process.
// The default leaves the fp32 RMSNorm and RoPE on plain launches: measured on
// the 1.5B decode, PDL on RMSNorm cost 1.9 ms per request (4 ms with 64-thread
// norm CTAs that fit beside a GEMM CTA, so SM co-residency is not the cause),
// on RoPE 0.2 ms, while the GEMM, attention, embedding, GEMV and beam-tail
// launches each gained.
enum PdlClass : unsigned {
  PDL_GEMM = 1u, PDL_NORM = 2u, PDL_ROPE = 4u, PDL_ATTN = 8u, PDL_EMBED = 16u, PDL_GEMV = 32u, PDL_TAIL = 64u,
  PDL_NORM16 = 128u, PDL_ALL = 255u
};
// The bf16 mode's RMSNorm (between its GEMMs) gains from it: decode steps
// 2.09 -> 2.01 ms at 1.5B, 4.06 -> 3.99 ms at 7B (A/B on one box).
constexpr unsigned kPdlDefault = PDL_GEMM | PDL_ATTN | PDL_EMBED | PDL_GEMV | PDL_TAIL | PDL_NORM16;
inline unsigned pdl_mask() {
  static const unsigned mask = [] {
    const char* e = getenv("RTR_PDL");
    if (!e) return kPdlDefault;
    if (strcmp(e, "all") == 0) return (unsigned)PDL_ALL;
    static const struct { const char* name; unsigned bit; } names[] = {
        {"gemm", PDL_GEMM}, {"norm", PDL_NORM}, {"rope", PDL_ROPE}, {"attn", PDL_ATTN},
        {"embed", PDL_EMBED}, {"gemv", PDL_GEMV}, {"tail", PDL_TAIL}, {"rms16", PDL_NORM16}};
    unsigned m = 0;
    for (const auto& n : names)
      if (strstr(e, n.name)) m |= n.bit;
    return m;
  }();
  return mask;
}
inline bool pdl_on(unsigned cls) { return (pdl_mask() & cls) != 0; }

// Launch with programmatic stream serialization: the kernel may be scheduled
// while its predecessor in the stream is still running.  Kernels launched this
// way call pdl_launch_dependents() and then pdl_wait() before touching memory
// (the tensor-core GEMM streams its constant weights before the wait), so
// memory order stays stream order and only launch latency and prologues overlap.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(unsigned cls, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_on(cls) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

