// Shared device helpers for the exploration_b200 sm_100a kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#define EB_DEVICE __device__ __forceinline__
#define EB_HOST_DEVICE __host__ __device__ __forceinline__

#define EB_CUDA_CHECK(expr)                                                          \
  do {                                                                               \
    cudaError_t _err = (expr);                                                       \
    TORCH_CHECK(_err == cudaSuccess, "CUDA error ", cudaGetErrorString(_err), " at ", \
                __FILE__, ":", __LINE__);                                            \
  } while (0)

namespace eb {

// Host-side count of kernels launched by this extension (read by bench.py).
void count_launch(int kernels = 1);

constexpr float kNegInf = -__builtin_huge_valf();

template <typename T>
EB_DEVICE float load_f(const T* p);
template <>
EB_DEVICE float load_f<float>(const float* p) { return *p; }
template <>
EB_DEVICE float load_f<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <>
EB_DEVICE float load_f<__half>(const __half* p) { return __half2float(*p); }

template <typename T>
EB_DEVICE T cast_f(float v);
template <>
EB_DEVICE float cast_f<float>(float v) { return v; }
template <>
EB_DEVICE __nv_bfloat16 cast_f<__nv_bfloat16>(float v) { return __float2bfloat16(v); }
template <>
EB_DEVICE __half cast_f<__half>(float v) { return __float2half(v); }

EB_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

EB_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Hardware base-2 exponential / logarithm (MUFU), used by the bf16 paths.
EB_DEVICE float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

EB_DEVICE float lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

EB_DEVICE float finite_or_zero(float x) { return x == kNegInf ? 0.f : x; }

// log(exp(a) + exp(b)) with -inf handled.
EB_DEVICE float log_add(float a, float b) {
  float m = fmaxf(a, b);
  if (m == kNegInf) return kNegInf;
  return m + logf(expf(a - m) + expf(b - m));
}

EB_HOST_DEVICE int cdiv(int a, int b) { return (a + b - 1) / b; }

}  // namespace eb
