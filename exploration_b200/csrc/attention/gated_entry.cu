// Gated dense attention entry points: allocate outputs and pick the kernel.
//
// bf16 with head_dim 64 or 128 and a power-of-two block size dividing 128
// runs the tcgen05/TMEM kernels (gated_tc.cu); everything else runs the
// fp32-accumulating CUDA-core kernels (gated_simt.cu).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstdlib>
#include <string>

#include "gated_common.cuh"
#include "../common/tma.cuh"

#include <atomic>
#include <mutex>

namespace eb {

namespace {
std::atomic<long long> launched{0};
}  // namespace

void count_launch(int kernels) { launched.fetch_add(kernels, std::memory_order_relaxed); }

long long launch_count() { return launched.load(std::memory_order_relaxed); }

sm100::ErrorSlot* device_error_slot(int device) {
  static std::mutex lock;
  static sm100::ErrorSlot* slots[64] = {nullptr};
  std::lock_guard<std::mutex> guard(lock);
  TORCH_CHECK(device >= 0 && device < 64, "device index out of range");
  if (slots[device] == nullptr) {
    void* ptr = nullptr;
    TORCH_CHECK(cudaMalloc(&ptr, sizeof(sm100::ErrorSlot)) == cudaSuccess, "error slot allocation failed");
    TORCH_CHECK(cudaMemset(ptr, 0, sizeof(sm100::ErrorSlot)) == cudaSuccess, "error slot init failed");
    slots[device] = static_cast<sm100::ErrorSlot*>(ptr);
  }
  return slots[device];
}

void gated_fwd_simt_launch(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& pos,
                           int64_t block, at::Tensor& out, at::Tensor& rc, at::Tensor& pr, at::Tensor& zr,
                           at::Tensor& lse);
void gated_bwd_simt_launch(const at::Tensor& grad, const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                           const at::Tensor& pos, const at::Tensor& out, const at::Tensor& rc,
                           const at::Tensor& pr, const at::Tensor& zr, const at::Tensor& lse, int64_t block,
                           at::Tensor& dq, at::Tensor& dk, at::Tensor& dv);
bool gated_tc_supported(const at::Tensor& q, int64_t block);
void gated_fwd_tc_launch(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& pos,
                         int64_t block, at::Tensor& out, at::Tensor& rc, at::Tensor& pr, at::Tensor& zr,
                         at::Tensor& lse);
void gated_bwd_tc_launch(const at::Tensor& grad, const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                         const at::Tensor& pos, const at::Tensor& out, const at::Tensor& rc, const at::Tensor& pr,
                         const at::Tensor& zr, const at::Tensor& lse, int64_t block, at::Tensor& dq,
                         at::Tensor& dk, at::Tensor& dv);

namespace {
void check_inputs(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& pos,
                  int64_t block) {
  TORCH_CHECK(q.is_cuda() && k.is_cuda() && v.is_cuda() && pos.is_cuda(), "gated attention: CUDA tensors");
  TORCH_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous() && pos.is_contiguous(),
              "gated attention: contiguous tensors");
  TORCH_CHECK(q.dim() == 4 && k.sizes() == v.sizes() && k.size(0) == q.size(0) && k.size(2) == q.size(2) &&
                  k.size(3) == q.size(3), "gated attention: q[B,Q,H,D], k/v[B,N,H,D]");
  TORCH_CHECK(pos.scalar_type() == at::kInt && pos.size(0) == q.size(0) && pos.size(1) == q.size(1),
              "gated attention: positions [B,Q] int32");
  TORCH_CHECK(q.scalar_type() == k.scalar_type() && q.scalar_type() == v.scalar_type(), "dtype mismatch");
  TORCH_CHECK(q.scalar_type() == at::kFloat || q.scalar_type() == at::kBFloat16, "fp32 or bf16 inputs");
  TORCH_CHECK(block >= 2 && block <= 128 && (block & (block - 1)) == 0, "block size: power of two in [2,128]");
  TORCH_CHECK(q.size(3) <= 256 && q.size(3) % 2 == 0, "head_dim must be even and <= 256");
}
}  // namespace

std::string gated_attention_path(const at::Tensor& q, int64_t block) {
  return gated_tc_supported(q, block) ? "tcgen05" : "cuda_core_fp32";
}

std::vector<at::Tensor> gated_attention_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                            const at::Tensor& pos, int64_t block) {
  check_inputs(q, k, v, pos, block);
  const c10::cuda::CUDAGuard guard(q.device());
  auto out = at::empty_like(q);
  auto rc = at::empty(q.sizes(), q.options().dtype(at::kFloat));
  auto pr = at::empty({q.size(0), q.size(1), q.size(2)}, q.options().dtype(at::kFloat));
  auto zr = at::empty_like(pr);
  auto lse = at::empty_like(pr);
  if (q.numel() == 0) return {out, rc, pr, zr, lse};
  if (gated_tc_supported(q, block))
    gated_fwd_tc_launch(q, k, v, pos, block, out, rc, pr, zr, lse);
  else
    gated_fwd_simt_launch(q, k, v, pos, block, out, rc, pr, zr, lse);
  return {out, rc, pr, zr, lse};
}

std::vector<at::Tensor> gated_attention_bwd(const at::Tensor& grad, const at::Tensor& q, const at::Tensor& k,
                                            const at::Tensor& v, const at::Tensor& pos, const at::Tensor& out,
                                            const at::Tensor& rc, const at::Tensor& pr, const at::Tensor& zr,
                                            const at::Tensor& lse, int64_t block) {
  check_inputs(q, k, v, pos, block);
  TORCH_CHECK(grad.sizes() == q.sizes() && grad.scalar_type() == q.scalar_type() && grad.is_contiguous(),
              "gated attention: grad must match q");
  const c10::cuda::CUDAGuard guard(q.device());
  auto dq = at::empty_like(q);
  auto dk = at::empty_like(k);
  auto dv = at::empty_like(v);
  if (q.numel() == 0) return {dq, dk.zero_(), dv.zero_()};
  if (gated_tc_supported(q, block))
    gated_bwd_tc_launch(grad, q, k, v, pos, out, rc, pr, zr, lse, block, dq, dk, dv);
  else
    gated_bwd_simt_launch(grad, q, k, v, pos, out, rc, pr, zr, lse, block, dq, dk, dv);
  return {dq, dk, dv};
}

}  // namespace eb
