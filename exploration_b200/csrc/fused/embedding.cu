// Token-embedding gradient without sorting (sm_100a).
//
//   dE[v, :] = sum over tokens t with ids[t] == v of dX[t, :]     (fp32)
//
// The vocabularies of this framework's models are small (bytes and the
// synthetic tasks' alphabets: a few hundred rows) while a training step
// covers thousands of tokens, so the gradient is computed per vocabulary row:
// CTA (v, column block) scans the id list in segments of 8,192 tokens
// (each thread tests 32 consecutive ids, loaded as 16-byte vectors), compacts
// the matching token indices into shared memory in token order (a prefix sum
// of the per-thread counts) and adds those dX rows, 4 columns per thread and
// eight rows in flight, in that order. Every output element is written by
// one thread after a fixed-order sum: deterministic, no atomics, no sort and
// no partial buffers. The id list (8 bytes per token) is re-read by every CTA
// but stays in L2; dX is read once in total.
//
// The reference takes the gradient of nn.Embedding from PyTorch, whose CUDA
// backward sorts the ids first (st/models/stack.py:121-122, the tied
// embedding and LM head).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "../common/util.cuh"

namespace eb {
namespace {

constexpr int kThreads = 256;
constexpr int kColsPerCta = 4 * kThreads;
constexpr int kPerThread = 32;                       // ids scanned per thread and segment
constexpr int kSegment = kThreads * kPerThread;      // 8192 tokens per segment
constexpr int kUnroll = 8;                           // dX rows in flight per thread

__global__ void __launch_bounds__(kThreads)
embedding_bwd_kernel(const int64_t* __restrict__ ids, const float* __restrict__ dx, float* __restrict__ out,
                     int64_t tokens, int cols) {
  __shared__ int picked[kSegment];
  __shared__ int warp_total[kThreads / 32];
  const int64_t v = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.y * kColsPerCta + threadIdx.x * 4;
  const bool live = c < cols;                        // cols is a multiple of 4 (checked on the host)
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int64_t seg = 0; seg < tokens; seg += kSegment) {
    // 1. Thread i tests the contiguous tokens [i * 32, i * 32 + 32) of the
    //    segment (all loads issued before any compare), so a prefix sum of
    //    the per-thread counts over the threads keeps token order.
    const int64_t t0 = seg + static_cast<int64_t>(threadIdx.x) * kPerThread;
    unsigned hits = 0u;
    if (t0 + kPerThread <= tokens) {
      int64_t local[kPerThread];
      const int4* src = reinterpret_cast<const int4*>(ids + t0);
#pragma unroll
      for (int j = 0; j < kPerThread / 2; ++j) {
        const int4 pair = __ldg(src + j);
        local[2 * j] = (static_cast<int64_t>(pair.y) << 32) | static_cast<uint32_t>(pair.x);
        local[2 * j + 1] = (static_cast<int64_t>(pair.w) << 32) | static_cast<uint32_t>(pair.z);
      }
#pragma unroll
      for (int j = 0; j < kPerThread; ++j) hits |= (local[j] == v ? 1u : 0u) << j;
    } else {
      for (int j = 0; j < kPerThread && t0 + j < tokens; ++j) hits |= (ids[t0 + j] == v ? 1u : 0u) << j;
    }
    const int mine = __popc(hits);
    int incl = mine;                                  // inclusive prefix over the warp
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    if (lane == 31) warp_total[warp] = incl;
    __syncthreads();
    int before = incl - mine, total = 0;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) {
      before += w < warp ? warp_total[w] : 0;
      total += warp_total[w];
    }
    for (unsigned m = hits; m; m &= m - 1u) picked[before++] = static_cast<int>(threadIdx.x) * kPerThread + __ffs(m) - 1;
    __syncthreads();
    // 2. Add the matching rows in token order, kUnroll loads in flight.
    if (live) {
      const float* base = dx + seg * cols + c;
      int i = 0;
      for (; i + kUnroll <= total; i += kUnroll) {
        float4 g[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u)
          g[u] = __ldcs(reinterpret_cast<const float4*>(base + static_cast<int64_t>(picked[i + u]) * cols));
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          acc.x += g[u].x;
          acc.y += g[u].y;
          acc.z += g[u].z;
          acc.w += g[u].w;
        }
      }
      for (; i < total; ++i) {
        const float4 g = __ldcs(reinterpret_cast<const float4*>(base + static_cast<int64_t>(picked[i]) * cols));
        acc.x += g.x;
        acc.y += g.y;
        acc.z += g.z;
        acc.w += g.w;
      }
    }
    __syncthreads();                                  // picked / warp_total are rewritten by the next segment
  }
  if (live) *reinterpret_cast<float4*>(out + v * cols + c) = acc;
}

}  // namespace

at::Tensor embedding_bwd(const at::Tensor& ids, const at::Tensor& dx, int64_t vocab) {
  TORCH_CHECK(ids.is_cuda() && dx.is_cuda(), "embedding_bwd: CUDA tensors expected");
  TORCH_CHECK(ids.scalar_type() == at::kLong, "embedding_bwd: int64 ids expected");
  TORCH_CHECK(dx.scalar_type() == at::kFloat, "embedding_bwd: fp32 gradient expected");
  const int64_t cols = dx.size(-1);
  const int64_t tokens = ids.numel();
  TORCH_CHECK(dx.numel() == tokens * cols, "embedding_bwd: gradient shape does not match the ids");
  TORCH_CHECK(cols % 4 == 0, "embedding_bwd: the embedding width must be a multiple of 4");
  TORCH_CHECK(vocab > 0 && vocab <= 65535, "embedding_bwd: vocabulary size out of range");
  const c10::cuda::CUDAGuard guard(dx.device());
  // The kernel reads both with 16-byte vector loads.
  auto ids_c = ids.contiguous();
  if (reinterpret_cast<uintptr_t>(ids_c.data_ptr()) % 16) ids_c = ids_c.clone();
  auto dx_c = dx.contiguous();
  if (reinterpret_cast<uintptr_t>(dx_c.data_ptr()) % 16) dx_c = dx_c.clone();
  auto out = at::empty({vocab, cols}, dx.options());
  const dim3 grid(static_cast<unsigned>(vocab), static_cast<unsigned>((cols + kColsPerCta - 1) / kColsPerCta));
  embedding_bwd_kernel<<<grid, kThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      ids_c.data_ptr<int64_t>(), dx_c.data_ptr<float>(), out.data_ptr<float>(), tokens, static_cast<int>(cols));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(1);
  return out;
}

}  // namespace eb
