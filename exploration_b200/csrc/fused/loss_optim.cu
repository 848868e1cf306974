// Cross-entropy head (loss, argmax hits and the logit gradient in one pass)
// and the multi-tensor AdamW / gradient-norm kernels.
//
// Cross entropy: one warp per row. The gradient softmax(logits) - onehot is
// produced together with the loss, so backward is a single scale. Rows with
// target -100 are ignored (zero loss, zero gradient, counted as hits).
//
// AdamW: one launch updates every tensor of a parameter group. The host
// builds a chunk table (tensor index, first element) so each CTA streams one
// contiguous chunk of one tensor with 16-byte vector accesses.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "../common/util.cuh"

namespace eb {
namespace {

constexpr int kCeWarps = 8;

__global__ void __launch_bounds__(kCeWarps * 32)
cross_entropy_kernel(const float* __restrict__ logits, const int64_t* __restrict__ targets,
                     float* __restrict__ row_loss, bool* __restrict__ hits,
                     float* __restrict__ grad, int rows, int vocab) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kCeWarps + warp;
  if (row >= rows) return;
  const float* lr = logits + static_cast<int64_t>(row) * vocab;
  float* gr = grad + static_cast<int64_t>(row) * vocab;
  const int64_t target = targets[row];
  float best = kNegInf;
  int best_i = vocab;
  for (int c = lane; c < vocab; c += 32) {
    float v = lr[c];
    if (v > best) {   // first index wins among equal values within a lane
      best = v;
      best_i = c;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, best, o);
    int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
    if (ov > best || (ov == best && oi < best_i)) {
      best = ov;
      best_i = oi;
    }
  }
  float sum = 0.f;
  for (int c = lane; c < vocab; c += 32) sum += expf(lr[c] - best);
  sum = warp_sum(sum);
  const float lse = best + logf(sum);
  const bool ignored = target == -100;
  for (int c = lane; c < vocab; c += 32) {
    float p = ignored ? 0.f : expf(lr[c] - lse);
    gr[c] = p - ((!ignored && c == target) ? 1.f : 0.f);
  }
  if (lane == 0) {
    row_loss[row] = ignored ? 0.f : lse - lr[target];
    hits[row] = ignored || best_i == target;
  }
}

struct ChunkRef {
  int tensor;
  int64_t start;
};

constexpr int kAdamChunk = 8192;   // elements per CTA
constexpr int kMaxAdamTensors = 4096;

struct AdamPointers {
  float* param[kMaxAdamTensors];
};

__global__ void __launch_bounds__(256)
adamw_kernel(float* const* __restrict__ params, const float* const* __restrict__ grads,
             float* const* __restrict__ m1, float* const* __restrict__ m2,
             const int64_t* __restrict__ sizes, const ChunkRef* __restrict__ chunks, float lr,
             float beta1, float beta2, float eps, float decay, float inv_bc1, float inv_sqrt_bc2,
             float grad_scale) {
  const ChunkRef ref = chunks[blockIdx.x];
  const int t = ref.tensor;
  const int64_t n = sizes[t];
  const int64_t end = min(n, ref.start + kAdamChunk);
  float* p = params[t];
  const float* g = grads[t];
  float* m = m1[t];
  float* v = m2[t];
  const float keep = 1.f - lr * decay;
  const float step = lr * inv_bc1;
  for (int64_t i = ref.start + threadIdx.x; i < end; i += blockDim.x) {
    const float gi = g[i] * grad_scale;
    const float mi = beta1 * m[i] + (1.f - beta1) * gi;
    const float vi = beta2 * v[i] + (1.f - beta2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    p[i] = p[i] * keep - step * mi / (sqrtf(vi) * inv_sqrt_bc2 + eps);
  }
}

// Partial sums of squares per chunk (deterministic two-stage reduction).
__global__ void __launch_bounds__(256)
sq_norm_kernel(const float* const* __restrict__ tensors, const int64_t* __restrict__ sizes,
               const ChunkRef* __restrict__ chunks, float* __restrict__ partial) {
  __shared__ float warp_part[8];
  const ChunkRef ref = chunks[blockIdx.x];
  const float* x = tensors[ref.tensor];
  const int64_t end = min(sizes[ref.tensor], ref.start + kAdamChunk);
  float acc = 0.f;
  for (int64_t i = ref.start + threadIdx.x; i < end; i += blockDim.x) acc += x[i] * x[i];
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) warp_part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < 8 ? warp_part[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) partial[blockIdx.x] = v;
  }
}

__global__ void sum_kernel(const float* __restrict__ partial, int count, float* __restrict__ out) {
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

// Host-side table of device pointers, chunk references and sizes, uploaded
// in one copy through a pinned staging tensor.
struct TensorTable {
  at::Tensor device;
  int chunks = 0;
  float** ptr_lists[4] = {nullptr, nullptr, nullptr, nullptr};
  int64_t* sizes = nullptr;
  ChunkRef* chunk_refs = nullptr;
};

TensorTable build_table(const std::vector<std::vector<at::Tensor>>& lists) {
  const size_t count = lists[0].size();
  std::vector<ChunkRef> refs;
  for (size_t t = 0; t < count; ++t) {
    const int64_t n = lists[0][t].numel();
    for (int64_t s = 0; s < n; s += kAdamChunk) refs.push_back({static_cast<int>(t), s});
  }
  const size_t ptr_bytes = lists.size() * count * sizeof(void*);
  const size_t size_bytes = count * sizeof(int64_t);
  const size_t ref_bytes = refs.size() * sizeof(ChunkRef);
  const size_t total = ptr_bytes + size_bytes + ref_bytes;
  auto host = at::empty({static_cast<int64_t>(total)}, at::TensorOptions().dtype(at::kByte).pinned_memory(true));
  auto* base = host.data_ptr<uint8_t>();
  auto** ptrs = reinterpret_cast<void**>(base);
  for (size_t l = 0; l < lists.size(); ++l)
    for (size_t t = 0; t < count; ++t) ptrs[l * count + t] = lists[l][t].data_ptr();
  auto* sizes = reinterpret_cast<int64_t*>(base + ptr_bytes);
  for (size_t t = 0; t < count; ++t) sizes[t] = lists[0][t].numel();
  std::memcpy(base + ptr_bytes + size_bytes, refs.data(), ref_bytes);
  TensorTable table;
  table.device = host.to(lists[0][0].device(), /*non_blocking=*/true);
  auto* dev = table.device.data_ptr<uint8_t>();
  for (size_t l = 0; l < lists.size(); ++l)
    table.ptr_lists[l] = reinterpret_cast<float**>(dev) + l * count;
  table.sizes = reinterpret_cast<int64_t*>(dev + ptr_bytes);
  table.chunk_refs = reinterpret_cast<ChunkRef*>(dev + ptr_bytes + size_bytes);
  table.chunks = static_cast<int>(refs.size());
  return table;
}

}  // namespace

std::vector<at::Tensor> cross_entropy_fwd(const at::Tensor& logits, const at::Tensor& targets) {
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == at::kFloat && logits.dim() == 2 &&
                  logits.is_contiguous(), "logits must be contiguous fp32 CUDA [T, V]");
  TORCH_CHECK(targets.scalar_type() == at::kLong && targets.numel() == logits.size(0), "targets [T] int64");
  const c10::cuda::CUDAGuard guard(logits.device());
  const int rows = logits.size(0), vocab = logits.size(1);
  auto row_loss = at::empty({rows}, logits.options());
  auto hits = at::empty({rows}, logits.options().dtype(at::kBool));
  auto grad = at::empty_like(logits);
  if (rows > 0) {
    cross_entropy_kernel<<<cdiv(rows, kCeWarps), kCeWarps * 32, 0, at::cuda::getCurrentCUDAStream()>>>(
        logits.data_ptr<float>(), targets.contiguous().data_ptr<int64_t>(), row_loss.data_ptr<float>(),
        hits.data_ptr<bool>(), grad.data_ptr<float>(), rows, vocab);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    count_launch(1);
  }
  return {row_loss.sum(), hits, grad};
}

void adamw_step(const std::vector<at::Tensor>& params, const std::vector<at::Tensor>& grads,
                const std::vector<at::Tensor>& exp_avg, const std::vector<at::Tensor>& exp_avg_sq,
                double lr, double beta1, double beta2, double eps, double decay, double bc1, double bc2,
                double grad_scale) {
  TORCH_CHECK(!params.empty() && params.size() == grads.size() && params.size() == exp_avg.size() &&
                  params.size() == exp_avg_sq.size(), "AdamW tensor lists differ");
  TORCH_CHECK(params.size() <= static_cast<size_t>(kMaxAdamTensors), "too many tensors in one group");
  for (size_t i = 0; i < params.size(); ++i) {
    TORCH_CHECK(params[i].scalar_type() == at::kFloat && grads[i].scalar_type() == at::kFloat &&
                    params[i].is_contiguous() && grads[i].is_contiguous() &&
                    exp_avg[i].is_contiguous() && exp_avg_sq[i].is_contiguous(),
                "AdamW expects contiguous fp32 tensors");
  }
  const c10::cuda::CUDAGuard guard(params[0].device());
  TensorTable table = build_table({params, grads, exp_avg, exp_avg_sq});
  if (table.chunks == 0) return;
  adamw_kernel<<<table.chunks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      table.ptr_lists[0], const_cast<const float* const*>(table.ptr_lists[1]), table.ptr_lists[2],
      table.ptr_lists[3], table.sizes, table.chunk_refs, static_cast<float>(lr), static_cast<float>(beta1),
      static_cast<float>(beta2), static_cast<float>(eps), static_cast<float>(decay),
      static_cast<float>(1.0 / bc1), static_cast<float>(1.0 / std::sqrt(bc2)), static_cast<float>(grad_scale));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(1);
}

at::Tensor grad_sq_norm(const std::vector<at::Tensor>& tensors) {
  TORCH_CHECK(!tensors.empty(), "no tensors");
  for (const auto& t : tensors)
    TORCH_CHECK(t.scalar_type() == at::kFloat && t.is_contiguous() && t.is_cuda(), "fp32 contiguous CUDA");
  const c10::cuda::CUDAGuard guard(tensors[0].device());
  TensorTable table = build_table({tensors});
  auto out = at::zeros({}, tensors[0].options());
  if (table.chunks == 0) return out;
  auto partial = at::empty({table.chunks}, tensors[0].options());
  auto stream = at::cuda::getCurrentCUDAStream();
  sq_norm_kernel<<<table.chunks, 256, 0, stream>>>(const_cast<const float* const*>(table.ptr_lists[0]),
                                                   table.sizes, table.chunk_refs, partial.data_ptr<float>());
  sum_kernel<<<1, 1024, 0, stream>>>(partial.data_ptr<float>(), table.chunks, out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(2);
  return out;
}

}  // namespace eb
