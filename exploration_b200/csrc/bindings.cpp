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
                                       const at::Tensor& mean, const at::Tensor& rstd,
                                       const c10::optional<at::Tensor>& dres, const c10::optional<at::Tensor>& dw_acc,
                                       const c10::optional<at::Tensor>& db_acc);
at::Tensor bias_gelu_fwd(const at::Tensor& h, const at::Tensor& bias);
std::vector<at::Tensor> cast_colsum(const at::Tensor& x, const c10::optional<at::Tensor>& sum_acc);
at::Tensor column_sum(const at::Tensor& part, const c10::optional<at::Tensor>& sum_acc);
std::vector<at::Tensor> bias_gelu_bwd(const at::Tensor& dout, const at::Tensor& h, const at::Tensor& bias);
std::vector<at::Tensor> cross_entropy_fwd(const at::Tensor& logits, const at::Tensor& targets);
at::Tensor embedding_bwd(const at::Tensor& ids, const at::Tensor& dx, int64_t vocab);
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
int64_t gemm_plain(const at::Tensor& a, bool a_mn, const at::Tensor& b, bool b_mn, at::Tensor& out, bool accumulate,
                   int64_t splits, int64_t shape);
std::vector<int64_t> gemm_plain_plan(int64_t M, int64_t N, int64_t K, int64_t sms);
void gemm(const at::Tensor& a, bool a_mn, const at::Tensor& b, bool b_mn, at::Tensor& out, int64_t epilogue,
          double alpha, const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& residual,
          const c10::optional<at::Tensor>& aux, const c10::optional<at::Tensor>& col_partial, int64_t shape);
void gemm_scatter(const at::Tensor& a, const at::Tensor& b, bool b_mn, const std::vector<int64_t>& dst,
                  int64_t rank, int64_t parts, int64_t batch, int64_t n_local, int64_t C);
void gemm_gather(const std::vector<int64_t>& src, int64_t rank, int64_t parts, int64_t batch, int64_t n_local,
                 int64_t C, const at::Tensor& b, bool b_mn, at::Tensor& out, int64_t epilogue,
                 const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& residual);
int64_t heap_alloc(int64_t bytes, int64_t device);
void heap_free(int64_t ptr, int64_t device);
at::Tensor heap_ipc_handle(int64_t ptr, int64_t device);
int64_t heap_open(const at::Tensor& handle, int64_t device);
void heap_close(int64_t ptr, int64_t device);
at::Tensor heap_tensor(int64_t base, int64_t bytes_offset, at::IntArrayRef sizes, at::ScalarType dtype,
                       int64_t device);
int64_t heap_signal_bytes();
void heap_barrier(const std::vector<int64_t>& bases, int64_t rank, double timeout_s);
void gather_rows(const std::vector<int64_t>& src, int64_t rank, int64_t parts, int64_t batch, int64_t n_local,
                 int64_t C, at::Tensor& out);
void flat_sq_norm(const at::Tensor& grad, at::Tensor& hyper);
void flat_adamw(at::Tensor& param, const at::Tensor& grad, at::Tensor& exp_avg, at::Tensor& exp_avg_sq,
                const c10::optional<at::Tensor>& shadow, const at::Tensor& hyper,
                const c10::optional<at::Tensor>& loss_check, double beta1, double beta2, double eps,
                double decay);
void flat_cast_bf16(const at::Tensor& x, at::Tensor& out);
int64_t grad_flag_bytes();
int64_t grad_reduce_max_buckets();
void grad_reduce_bucket(const std::vector<int64_t>& grads, const std::vector<int64_t>& flags, int64_t rank,
                        int64_t bucket, int64_t lo, int64_t hi, int64_t q, bool all_reduce, double scale,
                        at::Tensor& partial, double timeout_s);
void grad_norm_exchange(const at::Tensor& partial, const std::vector<int64_t>& flags, int64_t rank, at::Tensor& hyper,
                        double timeout_s);
void flat_adamw_peer(at::Tensor& param, const at::Tensor& grad, at::Tensor& exp_avg, at::Tensor& exp_avg_sq,
                     const std::vector<int64_t>& shadows, int64_t rank, const at::Tensor& hyper,
                     const c10::optional<at::Tensor>& loss_check, double beta1, double beta2, double eps,
                     double decay);
bool local_tc_supported(const at::Tensor& qkv, int64_t block);
std::vector<at::Tensor> local_tc_fwd(const at::Tensor& qkv, const c10::optional<at::Tensor>& prev, int64_t start,
                                     int64_t valid_start, int64_t n);
std::vector<at::Tensor> local_tc_bwd(const at::Tensor& dout, const at::Tensor& qkv, const c10::optional<at::Tensor>& prev,
                                     const at::Tensor& out, const at::Tensor& lse, int64_t start, int64_t valid_start,
                                     int64_t n);
bool block_scores_tc_supported(const at::Tensor& q, const at::Tensor& k, int64_t block, int64_t topk);
std::vector<at::Tensor> block_scores_topk_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& pos,
                                             int64_t block, int64_t first, int64_t topk);
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
  m.def("layer_norm_bwd", &eb::layer_norm_bwd, "LayerNorm backward; optional residual-gradient add and "
        "accumulation into parameter gradients", py::arg("dy"), py::arg("x"), py::arg("w"), py::arg("mean"),
        py::arg("rstd"), py::arg("dres") = py::none(), py::arg("dw_acc") = py::none(), py::arg("db_acc") = py::none());
  m.def("bias_gelu_fwd", &eb::bias_gelu_fwd);
  m.def("cast_colsum", &eb::cast_colsum, "fp32 -> (bf16 copy, column sums; optionally added into sum_acc)",
        py::arg("x"), py::arg("sum_acc") = py::none());
  m.def("column_sum", &eb::column_sum, "column sums of fp32 partials (optionally added into sum_acc)",
        py::arg("part"), py::arg("sum_acc") = py::none());
  m.def("bias_gelu_bwd", &eb::bias_gelu_bwd);
  m.def("cross_entropy_fwd", &eb::cross_entropy_fwd);
  m.def("embedding_bwd", &eb::embedding_bwd);
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
  m.def("gemm", &eb::gemm, "persistent tcgen05 GEMM with fused epilogues", py::arg("a"), py::arg("a_mn"),
        py::arg("b"), py::arg("b_mn"), py::arg("out"), py::arg("epilogue"), py::arg("alpha"), py::arg("bias"),
        py::arg("residual"), py::arg("aux"), py::arg("col_partial"), py::arg("shape") = 0);
  m.def("gemm_plain", &eb::gemm_plain, "tcgen05 GEMM without epilogue (store / fp32 accumulate), split-K when few tiles",
        py::arg("a"), py::arg("a_mn"), py::arg("b"), py::arg("b_mn"), py::arg("out"), py::arg("accumulate"),
        py::arg("splits") = 0, py::arg("shape") = 0);
  m.def("gemm_plain_plan", &eb::gemm_plain_plan);
  m.def("gemm_scatter", &eb::gemm_scatter, "projection GEMM whose epilogue stores head shards to their owners");
  m.def("gemm_gather", &eb::gemm_gather, "GEMM whose A operand is read from the owners' head shards");
  m.def("heap_alloc", &eb::heap_alloc);
  m.def("heap_free", &eb::heap_free);
  m.def("heap_ipc_handle", &eb::heap_ipc_handle);
  m.def("heap_open", &eb::heap_open);
  m.def("heap_close", &eb::heap_close);
  m.def("heap_tensor", &eb::heap_tensor);
  m.def("heap_signal_bytes", &eb::heap_signal_bytes);
  m.def("heap_barrier", &eb::heap_barrier, "bounded all-rank barrier over peer signal words");
  m.def("gather_rows", &eb::gather_rows, "sequence-layout copy of rank-sharded head buffers");
  m.def("flat_sq_norm", &eb::flat_sq_norm, "hyper[3] = sum of squares of a flat fp32 buffer");
  m.def("flat_adamw", &eb::flat_adamw, "AdamW over a flat buffer with device-side lr/step/clip");
  m.def("flat_cast_bf16", &eb::flat_cast_bf16);
  m.def("grad_flag_bytes", &eb::grad_flag_bytes);
  m.def("grad_reduce_max_buckets", &eb::grad_reduce_max_buckets);
  m.def("grad_reduce_bucket", &eb::grad_reduce_bucket,
        "reduce one gradient bucket over NVLink peer memory (owned slice; fused norm partials)");
  m.def("grad_norm_exchange", &eb::grad_norm_exchange, "global squared gradient norm; end-of-reduction barrier");
  m.def("flat_adamw_peer", &eb::flat_adamw_peer, "AdamW over an owned slice with the bf16 shadow stored to every rank");
  m.def("local_tc_supported", &eb::local_tc_supported);
  m.def("local_tc_fwd", &eb::local_tc_fwd, "tcgen05 local halo attention forward (block 16, head dim 64, bf16)");
  m.def("local_tc_bwd", &eb::local_tc_bwd, "tcgen05 local halo attention backward (dQ kernel + dK/dV kernel)");
  m.def("block_scores_tc_supported", &eb::block_scores_tc_supported);
  m.def("block_scores_topk_tc", &eb::block_scores_topk_tc,
        "tcgen05 exact block scores with log Z_R and a radix-select top-k per row");
  m.def("launch_count", &eb::launch_count, "kernels launched by this extension so far");
  m.def("device_errors", &device_errors, "read and clear (site, cta) of the last bounded-wait timeout");
}
