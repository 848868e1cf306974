// Python bindings of the exploration_b200 sm_100a extension.
#include <torch/extension.h>

#include <cuda_runtime.h>

#include <string>
#include <vector>

namespace eb {
namespace sm100 {
struct ErrorSlot {
  int code;
  int block;
};
}  // namespace sm100
sm100::ErrorSlot* device_error_slot(int device);
long long launch_count();

std::vector<at::Tensor> layer_norm_fwd(const at::Tensor& x, const at::Tensor& w, const at::Tensor& b, double eps,
                                       at::ScalarType out_dtype);
std::vector<at::Tensor> layer_norm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w,
                                       const at::Tensor& mean, const at::Tensor& rstd);
at::Tensor bias_gelu_fwd(const at::Tensor& h, const at::Tensor& bias);
std::vector<at::Tensor> bias_gelu_bwd(const at::Tensor& dout, const at::Tensor& h, const at::Tensor& bias);
std::vector<at::Tensor> cross_entropy_fwd(const at::Tensor& logits, const at::Tensor& targets);
void adamw_step(const std::vector<at::Tensor>& params, const std::vector<at::Tensor>& grads,
                const std::vector<at::Tensor>& exp_avg, const std::vector<at::Tensor>& exp_avg_sq, double lr,
                double beta1, double beta2, double eps, double decay, double bc1, double bc2, double grad_scale);
at::Tensor grad_sq_norm(const std::vector<at::Tensor>& tensors);
bool local_attention_supported(int block, int dim);
std::vector<at::Tensor> local_attention_fwd(const at::Tensor& qkv, const c10::optional<at::Tensor>& prev,
                                            int64_t start, int64_t valid_start, int64_t n, int64_t block);
std::vector<at::Tensor> local_attention_bwd(const at::Tensor& dout, const at::Tensor& qkv,
                                            const c10::optional<at::Tensor>& prev, const at::Tensor& out,
                                            const at::Tensor& lse, int64_t start, int64_t valid_start, int64_t n,
                                            int64_t block);
std::string gated_attention_path(const at::Tensor& q, int64_t block);
std::vector<at::Tensor> gated_attention_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                            const at::Tensor& pos, int64_t block);
std::vector<at::Tensor> gated_attention_bwd(const at::Tensor& grad, const at::Tensor& q, const at::Tensor& k,
                                            const at::Tensor& v, const at::Tensor& pos, const at::Tensor& out,
                                            const at::Tensor& rc, const at::Tensor& pr, const at::Tensor& zr,
                                            const at::Tensor& lse, int64_t block);
std::vector<at::Tensor> block_scores_topk(const at::Tensor& q, const at::Tensor& k, const at::Tensor& pos,
                                          int64_t block, int64_t first, int64_t topk);
bool gemm_supported(const at::Tensor& a, bool a_mn, const at::Tensor& b, bool b_mn);
void gemm(const at::Tensor& a, bool a_mn, const at::Tensor& b, bool b_mn, at::Tensor& out, int64_t epilogue,
          double alpha, const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& residual,
          const c10::optional<at::Tensor>& aux, const c10::optional<at::Tensor>& col_partial);
std::vector<at::Tensor> sparse_pop(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                   const at::Tensor& pos, const at::Tensor& ids, const at::Tensor& scores,
                                   const at::Tensor& log_zr, int64_t block, int64_t offset);
}  // namespace eb

namespace {

// Read and clear the bounded-wait error slot of a device: (site id, CTA).
std::pair<int, int> device_errors(int device) {
  eb::sm100::ErrorSlot host{0, 0};
  auto* slot = eb::device_error_slot(device);
  TORCH_CHECK(cudaMemcpy(&host, slot, sizeof(host), cudaMemcpyDeviceToHost) == cudaSuccess, "error slot read");
  TORCH_CHECK(cudaMemset(slot, 0, sizeof(host)) == cudaSuccess, "error slot reset");
  return {host.code, host.block};
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "exploration_b200 sm_100a kernels";
  m.def("layer_norm_fwd", &eb::layer_norm_fwd);
  m.def("layer_norm_bwd", &eb::layer_norm_bwd);
  m.def("bias_gelu_fwd", &eb::bias_gelu_fwd);
  m.def("bias_gelu_bwd", &eb::bias_gelu_bwd);
  m.def("cross_entropy_fwd", &eb::cross_entropy_fwd);
  m.def("adamw_step", &eb::adamw_step);
  m.def("grad_sq_norm", &eb::grad_sq_norm);
  m.def("local_attention_supported", &eb::local_attention_supported);
  m.def("local_attention_fwd", &eb::local_attention_fwd);
  m.def("local_attention_bwd", &eb::local_attention_bwd);
  m.def("gated_attention_path", &eb::gated_attention_path);
  m.def("gated_attention_fwd", &eb::gated_attention_fwd);
  m.def("gated_attention_bwd", &eb::gated_attention_bwd);
  m.def("block_scores_topk", &eb::block_scores_topk);
  m.def("sparse_pop", &eb::sparse_pop);
  m.def("gemm_supported", &eb::gemm_supported);
  m.def("gemm", &eb::gemm, "persistent tcgen05 GEMM with fused epilogues");
  m.def("launch_count", &eb::launch_count, "kernels launched by this extension so far");
  m.def("device_errors", &device_errors, "read and clear (site, cta) of the last bounded-wait timeout");
}
