// Flat-buffer AdamW for graph-captured training steps (sm_100a).
//
// All master parameters live in one fp32 buffer (the model's parameters are
// views into it) and their gradients in a second one, so the optimizer is
// one vectorised pass instead of a multi-tensor table built on the host
// every step. Everything that changes from step to step is read from device
// memory, `hyper = [lr, step, max_norm, grad_sq_norm]`, which lets a
// captured CUDA graph replay the update after an in-graph copy from pinned
// host memory refreshes the first three.
//
// * flat_sq_norm: per-CTA partial sums of squares (16-byte loads), then one
//   CTA adds the partials into `hyper[3]` (deterministic two-stage sum; the
//   caller all-reduces it across shards when the state is sharded).
// * flat_adamw: clip coefficient min(1, max_norm / (norm + 1e-6)) and the
//   bias corrections are formed per thread from `hyper` (torch's
//   clip_grad_norm_ and AdamW arithmetic). If the norm or the step's loss is
//   not finite the whole update is skipped, which is what the eager path does
//   by raising before the step. The fp32 master and its bf16 shadow (the
//   GEMM operand copy) are written in the same pass.
//
// The reference updates parameters with torch's AdamW (st/runtime/engine.py:
// 88-119, 179) and clips with clip_grad_norm_.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "../common/util.cuh"

namespace eb {
namespace {

constexpr int kThreads = 256;
constexpr int kNormBlocks = 592;   // 4 per SM

__global__ void __launch_bounds__(kThreads) flat_sq_norm_kernel(const float4* __restrict__ g, int64_t n4,
                                                                float* __restrict__ partial) {
  __shared__ float warp_part[kThreads / 32];
  float acc = 0.f;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const float4 x = g[i];
    acc += x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
  }
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) warp_part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < kThreads / 32 ? warp_part[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) partial[blockIdx.x] = v;
  }
}

__global__ void __launch_bounds__(1024) flat_sum_kernel(const float* __restrict__ partial, int count,
                                                        float* __restrict__ out) {
  __shared__ float warp_part[32];
  float acc = 0.f;
  for (int i = threadIdx.x; i < count; i += blockDim.x) acc += partial[i];
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) warp_part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? warp_part[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) *out = v;
  }
}

EB_DEVICE uint2 pack4_bf16(float a, float b, float c, float d) {
  __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
  return make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
}

__global__ void __launch_bounds__(kThreads)
flat_adamw_kernel(float4* __restrict__ p, const float4* __restrict__ g, float4* __restrict__ m,
                  float4* __restrict__ v, uint2* __restrict__ shadow, int64_t n4, const float* __restrict__ hyper,
                  const float* __restrict__ loss_check, float beta1, float beta2, float eps, float decay) {
  const float lr = hyper[0], step = hyper[1], max_norm = hyper[2], sq = hyper[3];
  const float lc = loss_check != nullptr ? *loss_check : 0.f;
  if (!isfinite(sq) || !isfinite(lc)) return;
  float scale = 1.f;
  if (max_norm > 0.f) scale = fminf(max_norm / (sqrtf(sq) + 1e-6f), 1.f);
  const float bc1 = 1.f - powf(beta1, step);
  const float bc2 = 1.f - powf(beta2, step);
  const float step_size = lr / bc1;
  const float inv_sqrt_bc2 = 1.f / sqrtf(bc2);
  const float keep = 1.f - lr * decay;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    float4 pi = p[i], gi = g[i], mi = m[i], vi = v[i];
    float* pp = &pi.x;
    const float* gg = &gi.x;
    float* mm = &mi.x;
    float* vv = &vi.x;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float gt = gg[t] * scale;
      mm[t] = beta1 * mm[t] + (1.f - beta1) * gt;
      vv[t] = beta2 * vv[t] + (1.f - beta2) * gt * gt;
      pp[t] = pp[t] * keep - step_size * mm[t] / (sqrtf(vv[t]) * inv_sqrt_bc2 + eps);
    }
    p[i] = pi;
    m[i] = mi;
    v[i] = vi;
    if (shadow != nullptr) shadow[i] = pack4_bf16(pi.x, pi.y, pi.z, pi.w);
  }
}

__global__ void __launch_bounds__(kThreads) flat_cast_bf16_kernel(const float4* __restrict__ x,
                                                                  uint2* __restrict__ out, int64_t n4) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const float4 a = x[i];
    out[i] = pack4_bf16(a.x, a.y, a.z, a.w);
  }
}

int grid_for(int64_t n4) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n4 + kThreads - 1) / kThreads, 148 * 8)));
}

void check_flat(const at::Tensor& t, at::ScalarType type, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == type && t.is_contiguous() && t.numel() % 4 == 0 &&
                  reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
              name, ": contiguous 16-byte aligned CUDA tensor with a multiple of 4 elements");
}

}  // namespace

// hyper[3] = sum(g^2) over this buffer (no cross-rank reduction).
void flat_sq_norm(const at::Tensor& grad, at::Tensor& hyper) {
  check_flat(grad, at::kFloat, "grad");
  TORCH_CHECK(hyper.is_cuda() && hyper.scalar_type() == at::kFloat && hyper.numel() >= 4, "hyper [4] fp32");
  const c10::cuda::CUDAGuard guard(grad.device());
  auto partial = at::empty({kNormBlocks}, grad.options());
  auto stream = at::cuda::getCurrentCUDAStream();
  flat_sq_norm_kernel<<<kNormBlocks, kThreads, 0, stream>>>(reinterpret_cast<const float4*>(grad.data_ptr()),
                                                            grad.numel() / 4, partial.data_ptr<float>());
  flat_sum_kernel<<<1, 1024, 0, stream>>>(partial.data_ptr<float>(), kNormBlocks, hyper.data_ptr<float>() + 3);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(2);
}

void flat_adamw(at::Tensor& param, const at::Tensor& grad, at::Tensor& exp_avg, at::Tensor& exp_avg_sq,
                const c10::optional<at::Tensor>& shadow, const at::Tensor& hyper,
                const c10::optional<at::Tensor>& loss_check, double beta1, double beta2, double eps,
                double decay) {
  check_flat(param, at::kFloat, "param");
  check_flat(grad, at::kFloat, "grad");
  check_flat(exp_avg, at::kFloat, "exp_avg");
  check_flat(exp_avg_sq, at::kFloat, "exp_avg_sq");
  const int64_t n = param.numel();
  TORCH_CHECK(grad.numel() == n && exp_avg.numel() == n && exp_avg_sq.numel() == n, "flat_adamw: sizes differ");
  uint2* sh = nullptr;
  if (shadow.has_value() && shadow->defined()) {
    check_flat(*shadow, at::kBFloat16, "shadow");
    TORCH_CHECK(shadow->numel() == n, "flat_adamw: shadow size");
    sh = reinterpret_cast<uint2*>(shadow->data_ptr());
  }
  const float* lc = nullptr;
  if (loss_check.has_value() && loss_check->defined()) {
    TORCH_CHECK(loss_check->is_cuda() && loss_check->scalar_type() == at::kFloat, "loss_check fp32");
    lc = loss_check->data_ptr<float>();
  }
  TORCH_CHECK(hyper.is_cuda() && hyper.scalar_type() == at::kFloat && hyper.numel() >= 4, "hyper [4] fp32");
  const c10::cuda::CUDAGuard guard(param.device());
  const int64_t n4 = n / 4;
  flat_adamw_kernel<<<grid_for(n4), kThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<float4*>(param.data_ptr()), reinterpret_cast<const float4*>(grad.data_ptr()),
      reinterpret_cast<float4*>(exp_avg.data_ptr()), reinterpret_cast<float4*>(exp_avg_sq.data_ptr()), sh, n4,
      hyper.data_ptr<float>(), lc, static_cast<float>(beta1), static_cast<float>(beta2), static_cast<float>(eps),
      static_cast<float>(decay));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(1);
}

void flat_cast_bf16(const at::Tensor& x, at::Tensor& out) {
  check_flat(x, at::kFloat, "x");
  check_flat(out, at::kBFloat16, "out");
  TORCH_CHECK(out.numel() == x.numel(), "flat_cast_bf16: sizes differ");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t n4 = x.numel() / 4;
  flat_cast_bf16_kernel<<<grid_for(n4), kThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const float4*>(x.data_ptr()), reinterpret_cast<uint2*>(out.data_ptr()), n4);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(1);
}

}  // namespace eb
