// LayerNorm (forward/backward) and bias+GELU (forward/backward) for sm_100a.
//
// LayerNorm: one warp per row, fp32 statistics; the output is written
// directly in the matmul dtype (bf16 under autocast), which removes the
// separate cast kernel autocast would run before the next GEMM. The
// backward writes dx per row and reduces dgamma/dbeta per column in a
// second, deterministic pass (no atomics).
//
// GELU is the exact erf form of torch.nn.GELU().
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "../common/util.cuh"

namespace eb {
namespace {

constexpr int kRowWarps = 8;          // rows per CTA for row-wise kernels
constexpr int kColThreads = 256;      // columns per CTA for column reductions
constexpr int kColSplits = 148;       // row splits of column reductions (one wave)

template <typename TIn, typename TOut>
__global__ void __launch_bounds__(kRowWarps * 32)
layer_norm_fwd_kernel(const TIn* __restrict__ x, const float* __restrict__ w,
                      const float* __restrict__ b, TOut* __restrict__ y, float* __restrict__ mean,
                      float* __restrict__ rstd, int rows, int cols, float eps) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kRowWarps + warp;
  if (row >= rows) return;
  const TIn* xr = x + static_cast<int64_t>(row) * cols;
  float sum = 0.f;
  for (int c = lane; c < cols; c += 32) sum += load_f(xr + c);
  const float mu = warp_sum(sum) / cols;
  float sq = 0.f;
  for (int c = lane; c < cols; c += 32) {
    float d = load_f(xr + c) - mu;
    sq += d * d;
  }
  const float rs = rsqrtf(warp_sum(sq) / cols + eps);
  TOut* yr = y + static_cast<int64_t>(row) * cols;
  for (int c = lane; c < cols; c += 32) yr[c] = cast_f<TOut>((load_f(xr + c) - mu) * rs * w[c] + b[c]);
  if (lane == 0) {
    mean[row] = mu;
    rstd[row] = rs;
  }
}

template <typename TIn, typename TGrad>
__global__ void __launch_bounds__(kRowWarps * 32)
layer_norm_bwd_dx_kernel(const TGrad* __restrict__ dy, const TIn* __restrict__ x,
                         const float* __restrict__ w, const float* __restrict__ mean,
                         const float* __restrict__ rstd, TIn* __restrict__ dx, int rows, int cols) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kRowWarps + warp;
  if (row >= rows) return;
  const int64_t base = static_cast<int64_t>(row) * cols;
  const float mu = mean[row], rs = rstd[row];
  float s1 = 0.f, s2 = 0.f;   // sum(dxhat), sum(dxhat * xhat)
  for (int c = lane; c < cols; c += 32) {
    float xh = (load_f(x + base + c) - mu) * rs;
    float g = load_f(dy + base + c) * w[c];
    s1 += g;
    s2 += g * xh;
  }
  s1 = warp_sum(s1) / cols;
  s2 = warp_sum(s2) / cols;
  for (int c = lane; c < cols; c += 32) {
    float xh = (load_f(x + base + c) - mu) * rs;
    float g = load_f(dy + base + c) * w[c];
    dx[base + c] = cast_f<TIn>(rs * (g - s1 - xh * s2));
  }
}

// Column partial sums of dy * xhat and dy over a contiguous range of rows.
template <typename TIn, typename TGrad>
__global__ void __launch_bounds__(kColThreads)
layer_norm_bwd_dwdb_kernel(const TGrad* __restrict__ dy, const TIn* __restrict__ x,
                           const float* __restrict__ mean, const float* __restrict__ rstd,
                           float* __restrict__ part_w, float* __restrict__ part_b, int rows,
                           int cols, int rows_per_split) {
  const int c = blockIdx.x * kColThreads + threadIdx.x;
  const int split = blockIdx.y;
  if (c >= cols) return;
  const int r0 = split * rows_per_split, r1 = min(rows, r0 + rows_per_split);
  float aw = 0.f, ab = 0.f;
  for (int r = r0; r < r1; ++r) {
    const int64_t i = static_cast<int64_t>(r) * cols + c;
    float g = load_f(dy + i);
    aw += g * (load_f(x + i) - mean[r]) * rstd[r];
    ab += g;
  }
  part_w[static_cast<int64_t>(split) * cols + c] = aw;
  part_b[static_cast<int64_t>(split) * cols + c] = ab;
}

// out_p[c] (+)= sum over s of part_p[s][c] for one or two partial arrays
// (p < kParts). A CTA owns 32 columns; its 16 warps each sum a contiguous
// slice of the partial rows (a warp reads 128 contiguous bytes per row), and
// warp 0 adds the 16 slice sums in slice order, so the result does not depend
// on scheduling. `accumulate` adds into the outputs (parameter gradients).
constexpr int kReduceSlices = 16;   // 16 warps: each thread has at most splits / 16 loads in flight

template <int kParts>
__global__ void __launch_bounds__(32 * kReduceSlices)
column_reduce_kernel(const float* __restrict__ part0, const float* __restrict__ part1, float* __restrict__ out0,
                     float* __restrict__ out1, int splits, int cols, int accumulate) {
  __shared__ float slice_sum[kParts][kReduceSlices][32];
  const int lane = threadIdx.x & 31, slice = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  const int per = (splits + kReduceSlices - 1) / kReduceSlices;
  const int s0 = slice * per, s1 = min(splits, s0 + per);
#pragma unroll
  for (int q = 0; q < kParts; ++q) {
    const float* part = q == 0 ? part0 : part1;
    float acc = 0.f;
    if (c < cols) {
#pragma unroll 8
      for (int s = s0; s < s1; ++s) acc += part[static_cast<int64_t>(s) * cols + c];
    }
    slice_sum[q][slice][lane] = acc;
  }
  __syncthreads();
  if (slice == 0 && c < cols) {
#pragma unroll
    for (int q = 0; q < kParts; ++q) {
      float total = 0.f;
#pragma unroll
      for (int k = 0; k < kReduceSlices; ++k) total += slice_sum[q][k][lane];
      float* out = q == 0 ? out0 : out1;
      out[c] = accumulate ? out[c] + total : total;
    }
  }
}

void column_sums(const float* part, float* out, int splits, int cols, bool accumulate, cudaStream_t stream) {
  column_reduce_kernel<1><<<cdiv(cols, 32), 32 * kReduceSlices, 0, stream>>>(part, nullptr, out, nullptr, splits,
                                                                             cols, accumulate ? 1 : 0);
}

void column_sums2(const float* part_w, const float* part_b, float* out_w, float* out_b, int splits, int cols,
                  bool accumulate, cudaStream_t stream) {
  column_reduce_kernel<2><<<cdiv(cols, 32), 32 * kReduceSlices, 0, stream>>>(part_w, part_b, out_w, out_b, splits,
                                                                             cols, accumulate ? 1 : 0);
}

// Gradient of a linear layer's fp32 output: the bf16 copy the GEMMs read and
// the per-CTA column sums (the bias gradient) in one read of the input.
// CTA = kCastRows rows; thread = 4 consecutive columns (grid-stride over cols).
constexpr int kCastRows = 32;

__global__ void __launch_bounds__(256) cast_colsum_kernel(const float4* __restrict__ x, uint2* __restrict__ out,
                                                          float4* __restrict__ part, int rows, int cols4) {
  const int r0 = blockIdx.x * kCastRows, r1 = min(rows, r0 + kCastRows);
  for (int c = threadIdx.x; c < cols4; c += blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
    for (int r = r0; r < r1; ++r) {
      const int64_t i = static_cast<int64_t>(r) * cols4 + c;
      const float4 v = x[i];
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
      __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
      out[i] = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
    }
    part[static_cast<int64_t>(blockIdx.x) * cols4 + c] = acc;
  }
}

// ---------------------------------------------------------------------------
// Register-resident LayerNorm for rows of cols = 128 * V (V float4 per lane):
// one warp per row, the row is read once; the backward also accumulates the
// dgamma/dbeta column partials of its CTA's rows in registers, reduces them
// across the CTA's warps in shared memory and writes one partial row per CTA
// (summed by one more small kernel), so x and dy are each read exactly once.
// ---------------------------------------------------------------------------

constexpr int kVecWarps = 8;
constexpr int kVecRowsPerCta = 64;

template <typename T>
EB_DEVICE void load4(const T* p, float (&v)[4]);
template <>
EB_DEVICE void load4<float>(const float* p, float (&v)[4]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
}
template <>
EB_DEVICE void load4<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}

template <typename T>
EB_DEVICE void store4(T* p, const float (&v)[4]);
template <>
EB_DEVICE void store4<float>(float* p, const float (&v)[4]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}
template <>
EB_DEVICE void store4<__nv_bfloat16>(__nv_bfloat16* p, const float (&v)[4]) {
  __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]), b = __floats2bfloat162_rn(v[2], v[3]);
  *reinterpret_cast<uint2*>(p) = make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
}

template <typename TIn, typename TOut, int V>
__global__ void __launch_bounds__(kVecWarps * 32)
ln_fwd_vec_kernel(const TIn* __restrict__ x, const float* __restrict__ w, const float* __restrict__ b,
                  TOut* __restrict__ y, float* __restrict__ mean, float* __restrict__ rstd, int rows, float eps) {
  constexpr int cols = 128 * V;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kVecWarps + warp;
  if (row >= rows) return;
  const TIn* xr = x + static_cast<int64_t>(row) * cols;
  float v[V][4];
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < V; ++j) {
    load4<TIn>(xr + 128 * j + 4 * lane, v[j]);
    sum += v[j][0] + v[j][1] + v[j][2] + v[j][3];
  }
  const float mu = warp_sum(sum) * (1.f / cols);
  float sq = 0.f;
#pragma unroll
  for (int j = 0; j < V; ++j)
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float d = v[j][t] - mu;
      sq += d * d;
    }
  const float rs = rsqrtf(warp_sum(sq) * (1.f / cols) + eps);
  TOut* yr = y + static_cast<int64_t>(row) * cols;
#pragma unroll
  for (int j = 0; j < V; ++j) {
    const int c = 128 * j + 4 * lane;
    const float4 ww = *reinterpret_cast<const float4*>(w + c);
    const float4 bb = *reinterpret_cast<const float4*>(b + c);
    float o[4] = {(v[j][0] - mu) * rs * ww.x + bb.x, (v[j][1] - mu) * rs * ww.y + bb.y,
                  (v[j][2] - mu) * rs * ww.z + bb.z, (v[j][3] - mu) * rs * ww.w + bb.w};
    store4<TOut>(yr + c, o);
  }
  if (lane == 0) {
    mean[row] = mu;
    rstd[row] = rs;
  }
}

template <typename TIn, typename TGrad, int V>
__global__ void __launch_bounds__(kVecWarps * 32)
ln_bwd_vec_kernel(const TGrad* __restrict__ dy, const TIn* __restrict__ x, const float* __restrict__ w,
                  const float* __restrict__ mean, const float* __restrict__ rstd, TIn* __restrict__ dx,
                  float* __restrict__ part_w, float* __restrict__ part_b, int rows, const float* __restrict__ dres) {
  constexpr int cols = 128 * V;
  extern __shared__ float red[];                       // [kVecWarps][2][cols], then w [cols]
  float* ws = red + kVecWarps * 2 * cols;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int c = threadIdx.x; c < cols; c += kVecWarps * 32) ws[c] = w[c];
  __syncthreads();
  float aw[V][4], ab[V][4];
#pragma unroll
  for (int j = 0; j < V; ++j)
#pragma unroll
    for (int t = 0; t < 4; ++t) aw[j][t] = ab[j][t] = 0.f;
  const int r0 = blockIdx.x * kVecRowsPerCta;
  const int r1 = min(rows, r0 + kVecRowsPerCta);
  for (int row = r0 + warp; row < r1; row += kVecWarps) {
    const int64_t base = static_cast<int64_t>(row) * cols;
    const float mu = mean[row], rs = rstd[row];
    float xh[V][4], dv[V][4];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int j = 0; j < V; ++j) {
      float xv[4];
      load4<TIn>(x + base + 128 * j + 4 * lane, xv);
      load4<TGrad>(dy + base + 128 * j + 4 * lane, dv[j]);
      const float4 ww = *reinterpret_cast<const float4*>(ws + 128 * j + 4 * lane);
      const float wt[4] = {ww.x, ww.y, ww.z, ww.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        xh[j][t] = (xv[t] - mu) * rs;
        const float g = dv[j][t] * wt[t];
        s1 += g;
        s2 += g * xh[j][t];
        aw[j][t] += dv[j][t] * xh[j][t];
        ab[j][t] += dv[j][t];
      }
    }
    s1 = warp_sum(s1) * (1.f / cols);
    s2 = warp_sum(s2) * (1.f / cols);
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const float4 ww = *reinterpret_cast<const float4*>(ws + 128 * j + 4 * lane);
      const float wt[4] = {ww.x, ww.y, ww.z, ww.w};
      float o[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) o[t] = rs * (dv[j][t] * wt[t] - s1 - xh[j][t] * s2);
      if (dres != nullptr) {                             // the residual branch's gradient of x
        const float4 r4 = *reinterpret_cast<const float4*>(dres + base + 128 * j + 4 * lane);
        o[0] += r4.x;
        o[1] += r4.y;
        o[2] += r4.z;
        o[3] += r4.w;
      }
      store4<TIn>(dx + base + 128 * j + 4 * lane, o);
    }
  }
  // CTA column partials: warps -> shared memory -> one row per CTA.
#pragma unroll
  for (int j = 0; j < V; ++j)
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      red[(warp * 2) * cols + 128 * j + 4 * lane + t] = aw[j][t];
      red[(warp * 2 + 1) * cols + 128 * j + 4 * lane + t] = ab[j][t];
    }
  __syncthreads();
  for (int c = threadIdx.x; c < cols; c += kVecWarps * 32) {
    float sw = 0.f, sb = 0.f;
#pragma unroll
    for (int q = 0; q < kVecWarps; ++q) {
      sw += red[(q * 2) * cols + c];
      sb += red[(q * 2 + 1) * cols + c];
    }
    part_w[static_cast<int64_t>(blockIdx.x) * cols + c] = sw;
    part_b[static_cast<int64_t>(blockIdx.x) * cols + c] = sb;
  }
}

#define EB_DISPATCH_V(V_VALUE, NAME, ...)                                   \
  switch (V_VALUE) {                                                        \
    case 1: { constexpr int NAME = 1; __VA_ARGS__(); break; }              \
    case 2: { constexpr int NAME = 2; __VA_ARGS__(); break; }              \
    case 4: { constexpr int NAME = 4; __VA_ARGS__(); break; }              \
    case 6: { constexpr int NAME = 6; __VA_ARGS__(); break; }              \
    case 8: { constexpr int NAME = 8; __VA_ARGS__(); break; }              \
    case 12: { constexpr int NAME = 12; __VA_ARGS__(); break; }            \
    case 16: { constexpr int NAME = 16; __VA_ARGS__(); break; }            \
    default: TORCH_CHECK(false, "unsupported LayerNorm width");            \
  }

#define EB_DISPATCH_V_SMALL(V_VALUE, NAME, ...)                             \
  switch (V_VALUE) {                                                        \
    case 1: { constexpr int NAME = 1; __VA_ARGS__(); break; }              \
    case 2: { constexpr int NAME = 2; __VA_ARGS__(); break; }              \
    case 4: { constexpr int NAME = 4; __VA_ARGS__(); break; }              \
    case 6: { constexpr int NAME = 6; __VA_ARGS__(); break; }              \
    case 8: { constexpr int NAME = 8; __VA_ARGS__(); break; }              \
    default: TORCH_CHECK(false, "unsupported LayerNorm width");            \
  }

bool vec_width(int cols) {
  if (cols % 128) return false;
  const int v = cols / 128;
  return v == 1 || v == 2 || v == 4 || v == 6 || v == 8 || v == 12 || v == 16;
}

EB_DEVICE float gelu(float v) { return 0.5f * v * (1.f + erff(v * 0.70710678118654752f)); }

EB_DEVICE float gelu_grad(float v) {
  const float cdf = 0.5f * (1.f + erff(v * 0.70710678118654752f));
  const float pdf = expf(-0.5f * v * v) * 0.39894228040143268f;
  return cdf + v * pdf;
}

template <typename T>
__global__ void bias_gelu_fwd_kernel(const T* __restrict__ h, const float* __restrict__ bias,
                                     T* __restrict__ out, int64_t total, int cols) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    out[i] = cast_f<T>(gelu(load_f(h + i) + bias[i % cols]));
  }
}

// dh = dout * gelu'(h + bias), written per element; column partials of dh for dbias.
template <typename T>
__global__ void __launch_bounds__(kColThreads)
bias_gelu_bwd_kernel(const T* __restrict__ dout, const T* __restrict__ h,
                     const float* __restrict__ bias, T* __restrict__ dh,
                     float* __restrict__ part, int rows, int cols, int rows_per_split) {
  const int c = blockIdx.x * kColThreads + threadIdx.x;
  const int split = blockIdx.y;
  if (c >= cols) return;
  const int r0 = split * rows_per_split, r1 = min(rows, r0 + rows_per_split);
  const float bc = bias[c];
  float acc = 0.f;
  for (int r = r0; r < r1; ++r) {
    const int64_t i = static_cast<int64_t>(r) * cols + c;
    const float g = load_f(dout + i) * gelu_grad(load_f(h + i) + bc);
    const T q = cast_f<T>(g);
    dh[i] = q;
    acc += g;
  }
  part[static_cast<int64_t>(split) * cols + c] = acc;
}

int row_splits(int rows) { return std::max(1, std::min(kColSplits, rows)); }

}  // namespace

#define EB_DISPATCH_FLOAT_BF16(TYPE, NAME, ...)                                  \
  [&] {                                                                         \
    if ((TYPE) == at::kFloat) {                                                 \
      using NAME = float;                                                       \
      return __VA_ARGS__();                                                     \
    } else if ((TYPE) == at::kBFloat16) {                                       \
      using NAME = __nv_bfloat16;                                               \
      return __VA_ARGS__();                                                     \
    }                                                                           \
    TORCH_CHECK(false, "expected float32 or bfloat16, got ", (TYPE));           \
  }()

std::vector<at::Tensor> layer_norm_fwd(const at::Tensor& x, const at::Tensor& w, const at::Tensor& b,
                                       double eps, at::ScalarType out_dtype) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous(), "x must be contiguous CUDA [T, C]");
  TORCH_CHECK(w.scalar_type() == at::kFloat && b.scalar_type() == at::kFloat, "fp32 affine params");
  const c10::cuda::CUDAGuard guard(x.device());
  const int rows = x.size(0), cols = x.size(1);
  auto y = at::empty({rows, cols}, x.options().dtype(out_dtype));
  auto mean = at::empty({rows}, x.options().dtype(at::kFloat));
  auto rstd = at::empty({rows}, x.options().dtype(at::kFloat));
  if (rows == 0) return {y, mean, rstd};
  auto stream = at::cuda::getCurrentCUDAStream();
  const int grid = cdiv(rows, kRowWarps);
  if (vec_width(cols)) {
    EB_DISPATCH_FLOAT_BF16(x.scalar_type(), TIn, [&] {
      EB_DISPATCH_FLOAT_BF16(out_dtype, TOut, [&] {
        EB_DISPATCH_V(cols / 128, V, [&] {
          ln_fwd_vec_kernel<TIn, TOut, V><<<cdiv(rows, kVecWarps), kVecWarps * 32, 0, stream>>>(
              reinterpret_cast<const TIn*>(x.data_ptr()), w.data_ptr<float>(), b.data_ptr<float>(),
              reinterpret_cast<TOut*>(y.data_ptr()), mean.data_ptr<float>(), rstd.data_ptr<float>(), rows,
              static_cast<float>(eps));
        });
      });
    });
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    count_launch(1);
    return {y, mean, rstd};
  }
  EB_DISPATCH_FLOAT_BF16(x.scalar_type(), TIn, [&] {
    EB_DISPATCH_FLOAT_BF16(out_dtype, TOut, [&] {
      layer_norm_fwd_kernel<TIn, TOut><<<grid, kRowWarps * 32, 0, stream>>>(
          reinterpret_cast<const TIn*>(x.data_ptr()), w.data_ptr<float>(), b.data_ptr<float>(),
          reinterpret_cast<TOut*>(y.data_ptr()), mean.data_ptr<float>(), rstd.data_ptr<float>(),
          rows, cols, static_cast<float>(eps));
    });
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(1);
  return {y, mean, rstd};
}

// dres: optional fp32 gradient of x from another branch, added to dx inside the
// kernel. dw_acc / db_acc: optional fp32 [cols] tensors (parameter gradients)
// the weight and bias gradients are added into instead of being returned fresh.
std::vector<at::Tensor> layer_norm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w,
                                       const at::Tensor& mean, const at::Tensor& rstd,
                                       const c10::optional<at::Tensor>& dres_opt,
                                       const c10::optional<at::Tensor>& dw_acc,
                                       const c10::optional<at::Tensor>& db_acc) {
  TORCH_CHECK(dy.is_contiguous() && x.is_contiguous() && dy.sizes() == x.sizes(), "dy/x mismatch");
  const c10::cuda::CUDAGuard guard(x.device());
  const int rows = x.size(0), cols = x.size(1);
  const bool has_res = dres_opt.has_value() && dres_opt->defined();
  if (has_res)
    TORCH_CHECK(dres_opt->is_contiguous() && dres_opt->scalar_type() == at::kFloat && dres_opt->numel() == x.numel(),
                "layer_norm_bwd: dres must be contiguous fp32 with x's size");
  const bool acc = dw_acc.has_value() && dw_acc->defined();
  if (acc)
    TORCH_CHECK(db_acc.has_value() && db_acc->defined() && dw_acc->is_contiguous() && db_acc->is_contiguous() &&
                    dw_acc->scalar_type() == at::kFloat && db_acc->scalar_type() == at::kFloat &&
                    dw_acc->numel() == cols && db_acc->numel() == cols,
                "layer_norm_bwd: dw_acc/db_acc must be contiguous fp32 [cols]");
  auto dx = at::empty_like(x);
  at::Tensor dw = acc ? *dw_acc : at::zeros({cols}, x.options().dtype(at::kFloat));
  at::Tensor db = acc ? *db_acc : at::zeros({cols}, x.options().dtype(at::kFloat));
  if (rows == 0) return {dx, dw, db};
  auto stream = at::cuda::getCurrentCUDAStream();
  if (vec_width(cols) && cols <= 1024) {
    const int ctas = cdiv(rows, kVecRowsPerCta);
    auto pw = at::empty({ctas, cols}, x.options().dtype(at::kFloat));
    auto pb = at::empty({ctas, cols}, x.options().dtype(at::kFloat));
    const size_t smem = sizeof(float) * (kVecWarps * 2 + 1) * cols;
    EB_DISPATCH_FLOAT_BF16(x.scalar_type(), TIn, [&] {
      EB_DISPATCH_FLOAT_BF16(dy.scalar_type(), TGrad, [&] {
        EB_DISPATCH_V_SMALL(cols / 128, V, [&] {
          auto kernel = ln_bwd_vec_kernel<TIn, TGrad, V>;
          EB_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
          kernel<<<ctas, kVecWarps * 32, smem, stream>>>(
              reinterpret_cast<const TGrad*>(dy.data_ptr()), reinterpret_cast<const TIn*>(x.data_ptr()),
              w.data_ptr<float>(), mean.data_ptr<float>(), rstd.data_ptr<float>(),
              reinterpret_cast<TIn*>(dx.data_ptr()), pw.data_ptr<float>(), pb.data_ptr<float>(), rows,
              has_res ? dres_opt->data_ptr<float>() : nullptr);
        });
      });
    });
    column_sums2(pw.data_ptr<float>(), pb.data_ptr<float>(), dw.data_ptr<float>(), db.data_ptr<float>(), ctas, cols,
                 acc, stream);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    count_launch(2);
    return {dx, dw, db};
  }
  const int splits = row_splits(rows);
  const int per_split = cdiv(rows, splits);
  auto part_w = at::empty({splits, cols}, x.options().dtype(at::kFloat));
  auto part_b = at::empty({splits, cols}, x.options().dtype(at::kFloat));
  EB_DISPATCH_FLOAT_BF16(x.scalar_type(), TIn, [&] {
    EB_DISPATCH_FLOAT_BF16(dy.scalar_type(), TGrad, [&] {
      layer_norm_bwd_dx_kernel<TIn, TGrad><<<cdiv(rows, kRowWarps), kRowWarps * 32, 0, stream>>>(
          reinterpret_cast<const TGrad*>(dy.data_ptr()), reinterpret_cast<const TIn*>(x.data_ptr()),
          w.data_ptr<float>(), mean.data_ptr<float>(), rstd.data_ptr<float>(),
          reinterpret_cast<TIn*>(dx.data_ptr()), rows, cols);
      dim3 grid(cdiv(cols, kColThreads), splits);
      layer_norm_bwd_dwdb_kernel<TIn, TGrad><<<grid, kColThreads, 0, stream>>>(
          reinterpret_cast<const TGrad*>(dy.data_ptr()), reinterpret_cast<const TIn*>(x.data_ptr()),
          mean.data_ptr<float>(), rstd.data_ptr<float>(), part_w.data_ptr<float>(),
          part_b.data_ptr<float>(), rows, cols, per_split);
    });
  });
  // General widths: fresh sums, then the optional accumulations as separate adds.
  at::Tensor dw_f = acc ? at::empty({cols}, x.options().dtype(at::kFloat)) : dw;
  at::Tensor db_f = acc ? at::empty({cols}, x.options().dtype(at::kFloat)) : db;
  column_sums2(part_w.data_ptr<float>(), part_b.data_ptr<float>(), dw_f.data_ptr<float>(), db_f.data_ptr<float>(),
               splits, cols, false, stream);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(3);
  if (acc) {
    dw.add_(dw_f);
    db.add_(db_f);
  }
  if (has_res) dx.add_(dres_opt->view(dx.sizes()));
  return {dx, dw, db};
}

// x fp32 [rows, cols] -> (bf16 copy, column sums). With `sum_acc` (fp32 [cols],
// e.g. a bias gradient) the sums are added into it and it is returned.
std::vector<at::Tensor> cast_colsum(const at::Tensor& x, const c10::optional<at::Tensor>& sum_acc) {
  TORCH_CHECK(x.is_cuda() && x.is_contiguous() && x.dim() == 2 && x.scalar_type() == at::kFloat &&
                  x.size(1) % 4 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0,
              "cast_colsum: contiguous 16-byte aligned fp32 [rows, cols], cols % 4 == 0");
  const c10::cuda::CUDAGuard guard(x.device());
  const int rows = x.size(0), cols = x.size(1);
  const bool acc = sum_acc.has_value() && sum_acc->defined();
  if (acc)
    TORCH_CHECK(sum_acc->is_contiguous() && sum_acc->scalar_type() == at::kFloat && sum_acc->numel() == cols,
                "cast_colsum: sum_acc must be contiguous fp32 [cols]");
  auto out = at::empty({rows, cols}, x.options().dtype(at::kBFloat16));
  at::Tensor sums = acc ? *sum_acc : at::zeros({cols}, x.options());
  if (rows == 0) return {out, sums};
  const int ctas = cdiv(rows, kCastRows);
  auto part = at::empty({ctas, cols}, x.options());
  auto stream = at::cuda::getCurrentCUDAStream();
  cast_colsum_kernel<<<ctas, 256, 0, stream>>>(reinterpret_cast<const float4*>(x.data_ptr()),
                                               reinterpret_cast<uint2*>(out.data_ptr()),
                                               reinterpret_cast<float4*>(part.data_ptr()), rows, cols / 4);
  column_sums(part.data_ptr<float>(), sums.data_ptr<float>(), ctas, cols, acc, stream);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(2);
  return {out, sums};
}

// out (+)= sum over rows of part [splits, cols] (fp32).
at::Tensor column_sum(const at::Tensor& part, const c10::optional<at::Tensor>& sum_acc) {
  TORCH_CHECK(part.is_cuda() && part.is_contiguous() && part.dim() == 2 && part.scalar_type() == at::kFloat,
              "column_sum: contiguous fp32 [splits, cols]");
  const c10::cuda::CUDAGuard guard(part.device());
  const int splits = part.size(0), cols = part.size(1);
  const bool acc = sum_acc.has_value() && sum_acc->defined();
  if (acc)
    TORCH_CHECK(sum_acc->is_contiguous() && sum_acc->scalar_type() == at::kFloat && sum_acc->numel() == cols,
                "column_sum: sum_acc must be contiguous fp32 [cols]");
  at::Tensor sums = acc ? *sum_acc : at::empty({cols}, part.options());
  if (cols == 0) return sums;
  column_sums(part.data_ptr<float>(), sums.data_ptr<float>(), splits, cols, acc, at::cuda::getCurrentCUDAStream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(1);
  return sums;
}

at::Tensor bias_gelu_fwd(const at::Tensor& h, const at::Tensor& bias) {
  TORCH_CHECK(h.is_contiguous() && h.dim() == 2 && bias.scalar_type() == at::kFloat, "bad bias_gelu args");
  const c10::cuda::CUDAGuard guard(h.device());
  auto out = at::empty_like(h);
  const int64_t total = h.numel();
  if (total == 0) return out;
  const int grid = static_cast<int>(std::min<int64_t>(cdiv(total, 256), 148 * 16));
  EB_DISPATCH_FLOAT_BF16(h.scalar_type(), T, [&] {
    bias_gelu_fwd_kernel<T><<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const T*>(h.data_ptr()), bias.data_ptr<float>(),
        reinterpret_cast<T*>(out.data_ptr()), total, static_cast<int>(h.size(1)));
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(1);
  return out;
}

std::vector<at::Tensor> bias_gelu_bwd(const at::Tensor& dout, const at::Tensor& h, const at::Tensor& bias) {
  TORCH_CHECK(dout.sizes() == h.sizes() && dout.is_contiguous() && h.is_contiguous(), "bad shapes");
  TORCH_CHECK(dout.scalar_type() == h.scalar_type(), "dout/h dtype mismatch");
  const c10::cuda::CUDAGuard guard(h.device());
  const int rows = h.size(0), cols = h.size(1);
  auto dh = at::empty_like(h);
  auto dbias = at::zeros({cols}, h.options().dtype(at::kFloat));
  if (rows == 0) return {dh, dbias};
  const int splits = row_splits(rows);
  auto part = at::empty({splits, cols}, h.options().dtype(at::kFloat));
  auto stream = at::cuda::getCurrentCUDAStream();
  EB_DISPATCH_FLOAT_BF16(h.scalar_type(), T, [&] {
    dim3 grid(cdiv(cols, kColThreads), splits);
    bias_gelu_bwd_kernel<T><<<grid, kColThreads, 0, stream>>>(
        reinterpret_cast<const T*>(dout.data_ptr()), reinterpret_cast<const T*>(h.data_ptr()),
        bias.data_ptr<float>(), reinterpret_cast<T*>(dh.data_ptr()), part.data_ptr<float>(), rows,
        cols, cdiv(rows, splits));
  });
  column_sums(part.data_ptr<float>(), dbias.data_ptr<float>(), splits, cols, false, stream);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(2);
  return {dh, dbias};
}

}  // namespace eb
