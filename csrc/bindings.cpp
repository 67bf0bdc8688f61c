// Python bindings of the nano_train_b200 CUDA extension (module `_C`).
#include <execinfo.h>
#include <signal.h>
#include <unistd.h>

#include <cstdlib>

#include <torch/extension.h>

#include "host_utils.h"

namespace {
// Debug aid (NTB_DEBUG_HOST=1): print the native backtrace of a SIGSEGV before dying.
void segv_backtrace(int sig) {
  void* frames[64];
  const int n = backtrace(frames, 64);
  const char msg[] = "[ntb] native backtrace:\n";
  ssize_t w = write(2, msg, sizeof(msg) - 1);
  (void)w;
  backtrace_symbols_fd(frames, n, 2);
  signal(sig, SIG_DFL);
  raise(sig);
}
}  // namespace

namespace ntb {
// gemm.cu
void gemm_bf16(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, const c10::optional<at::Tensor>& bias,
               bool a_mn, bool b_mn, bool accumulate, double alpha);
void gemm_grouped_bf16(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, const at::Tensor& offsets,
                       int64_t mode, bool b_mn, bool accumulate, int64_t c_group_stride);
// ops.cu
std::vector<at::Tensor> rmsnorm_fwd(const at::Tensor& x, const c10::optional<at::Tensor>& residual,
                                    const at::Tensor& w, double eps);
std::vector<at::Tensor> rmsnorm_bwd(const at::Tensor& dy, const at::Tensor& h, const at::Tensor& w,
                                    const at::Tensor& rstd, const c10::optional<at::Tensor>& dres,
                                    const c10::optional<at::Tensor>& dw_into);
std::vector<at::Tensor> layernorm_fwd(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& b,
                                      double eps);
std::vector<at::Tensor> layernorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w,
                                      const at::Tensor& mean, const at::Tensor& rstd);
void rope_(at::Tensor& x, const c10::optional<at::Tensor>& positions, int64_t off, int64_t R, int64_t seq_len,
           double theta, int64_t mode, bool inverse);
void rope_table_(at::Tensor& x, const at::Tensor& table, int64_t off, int64_t R, int64_t seq_len, int64_t mode,
                 bool inverse);
at::Tensor mla_k_assemble(const at::Tensor& kv, const at::Tensor& kr, const at::Tensor& table, int64_t Dn,
                          int64_t seq_len);
at::Tensor mla_k_assemble_bwd(const at::Tensor& dk, at::Tensor& dkv, const at::Tensor& table, int64_t Dn,
                              int64_t seq_len);
at::Tensor swiglu_fwd(const at::Tensor& gu);
at::Tensor swiglu_bwd(const at::Tensor& dout, const at::Tensor& gu);
at::Tensor gelu_fwd(const at::Tensor& x);
at::Tensor gelu_bwd(const at::Tensor& dy, const at::Tensor& x);
std::vector<at::Tensor> ce_stats(const at::Tensor& logits, const at::Tensor& labels, int64_t vstart,
                                 int64_t ignore_index);
void ce_bwd(const at::Tensor& logits, const at::Tensor& labels, const at::Tensor& lse, const at::Tensor& scale,
            int64_t vstart, int64_t ignore_index, at::Tensor& grad);
at::Tensor embedding_fwd(const at::Tensor& ids, const at::Tensor& W, int64_t vstart);
void embedding_bwd_(const at::Tensor& ids, const at::Tensor& dout, at::Tensor& dW, int64_t vstart);
void adamw_flat_(at::Tensor& p, at::Tensor& m, at::Tensor& v, const at::Tensor& g,
                 const c10::optional<at::Tensor>& p_bf16, double lr, double b1, double b2, double eps, double wd,
                 int64_t step, const c10::optional<at::Tensor>& grad_scale, const c10::optional<at::Tensor>& skip);
void grad_stats_(at::Tensor& g, const c10::optional<at::Tensor>& inv_scale, at::Tensor& out);
// attention.cu
std::vector<at::Tensor> flash_attn_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, double scale,
                                       bool causal);
std::vector<at::Tensor> flash_attn_bwd(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k,
                                       const at::Tensor& v, const at::Tensor& out, const at::Tensor& lse, double scale,
                                       bool causal, const c10::optional<at::Tensor>& dq,
                                       const c10::optional<at::Tensor>& dk, const c10::optional<at::Tensor>& dv);
// attention_tc.cu
std::vector<at::Tensor> flash_attn_fwd_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, double scale,
                                          bool causal);
// gemm_fp8.cu
void gemm_fp8_blockscaled(const at::Tensor& a_q, const at::Tensor& sa, const at::Tensor& b_q, const at::Tensor& sb,
                          at::Tensor& out, const c10::optional<at::Tensor>& bias);
// persistent.cu
std::vector<at::Tensor> persistent_quantize(const at::Tensor& w, bool nf4, bool per_tensor);
at::Tensor persistent_dequantize(const at::Tensor& codes, const at::Tensor& scale, int64_t rows, int64_t cols,
                                 bool nf4, at::ScalarType dtype);
// dropout.cu
at::Tensor dropout_apply(const at::Tensor& x, double p, int64_t seed);
// gemm_fp4.cu
std::vector<at::Tensor> nvfp4_quantize(const at::Tensor& x);
at::Tensor nvfp4_dequantize(const at::Tensor& q, const at::Tensor& sf, const at::Tensor& gs, at::ScalarType dtype);
void gemm_nvfp4(const at::Tensor& a_q, const at::Tensor& sfa, const at::Tensor& gsa, const at::Tensor& b_q,
                const at::Tensor& sfb, const at::Tensor& gsb, at::Tensor& out, const c10::optional<at::Tensor>& bias);
// quant.cu
std::vector<at::Tensor> fp8_quantize(const at::Tensor& x, int64_t block_rows, bool stochastic, int64_t seed);
at::Tensor fp8_quant_dequant(const at::Tensor& x, int64_t block_rows, bool stochastic, int64_t seed);
at::Tensor fp8_quant_dequant_strided(const at::Tensor& src, int64_t groups, int64_t rows_per_group, int64_t cols,
                                     int64_t group_stride);
std::vector<at::Tensor> fp8_quantize_strided(const at::Tensor& src, int64_t groups, int64_t rows_per_group,
                                             int64_t cols, int64_t group_stride);
std::vector<at::Tensor> fp8_quantize_with_dq(const at::Tensor& x, bool stochastic, int64_t seed);
void gemm_fp8_grouped(const at::Tensor& a_q, const at::Tensor& sa, const at::Tensor& b_q, const at::Tensor& sb,
                      at::Tensor& out, const at::Tensor& offsets);
at::Tensor fp8_dequantize(const at::Tensor& q, const at::Tensor& scales, int64_t block_rows, at::ScalarType dtype);
// tp_fused.cu
void ag_gemm(const at::Tensor& x_local, at::Tensor& x_full_out, const at::Tensor& w, at::Tensor& y,
             const c10::optional<at::Tensor>& bias, bool b_mn, std::vector<int64_t> slots, std::vector<int64_t> ready,
             at::Tensor& ctrs, int64_t rank, int64_t epoch, const c10::optional<at::Tensor>& trace);
void gemm_rs(const at::Tensor& x, const at::Tensor& w, at::Tensor& out, const c10::optional<at::Tensor>& bias,
             bool b_mn, std::vector<int64_t> recv, std::vector<int64_t> tctrs, at::Tensor& ctrs, int64_t rank,
             int64_t epoch, const c10::optional<at::Tensor>& trace);
void wait_flag(const at::Tensor& flag, int64_t expect, int64_t limit_ns);
void rs_pull(std::vector<int64_t> parts, at::Tensor& out, const c10::optional<at::Tensor>& bias, int64_t rank,
             int64_t flags_ptr, int64_t epoch);
void gemm_rsp(const at::Tensor& x, const at::Tensor& w, at::Tensor& out, const c10::optional<at::Tensor>& bias,
              bool b_mn, std::vector<int64_t> parts, std::vector<int64_t> rdy, int64_t my_rdy, int64_t tpc_stride,
              at::Tensor& acc, at::Tensor& acc_cnt, at::Tensor& ctrs, int64_t rank, int64_t epoch,
              const c10::optional<at::Tensor>& trace);
void gemm_bf16_publish(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, bool b_mn,
                       std::vector<int64_t> flags, int64_t epoch, at::Tensor& ctr);
// router.cu
std::vector<at::Tensor> router_fwd(const at::Tensor& logits, int64_t K, bool softmax, int64_t n_group,
                                   int64_t topk_group, bool norm_topk, double scale);
at::Tensor router_bwd(const at::Tensor& logits, const at::Tensor& idx, const at::Tensor& dw, const at::Tensor& dpsum,
                      int64_t K, bool softmax, int64_t n_group, int64_t topk_group, bool norm_topk, double scale);
// moe_ep.cu
void ep_dispatch(const at::Tensor& x, const at::Tensor& idx, const at::Tensor& w, at::Tensor& dest_tk,
                 at::Tensor& slot_tk, const at::Tensor& ctr, int64_t epr, std::vector<int64_t> payload,
                 std::vector<int64_t> pscale, std::vector<int64_t> meta, std::vector<int64_t> flag,
                 std::vector<int64_t> info, const at::Tensor& done, int64_t P, int64_t epoch, bool fp8,
                 bool stochastic, int64_t seed);
void ep_recv_keys(int64_t meta_ptr, int64_t info_ptr, at::Tensor& keys, at::Tensor& counts, int64_t P, int64_t n,
                  int64_t epr, int64_t K);
void ep_recv_layout(const at::Tensor& skeys, const at::Tensor& order, int64_t meta_ptr, int64_t info_ptr,
                    const at::Tensor& counts, at::Tensor& offsets, at::Tensor& row_src, at::Tensor& row_slot,
                    at::Tensor& row_tok, at::Tensor& row_w, int64_t rowmap_ptr, at::Tensor& stats, int64_t P,
                    int64_t n, int64_t epr, int64_t K, int64_t E, double capacity_factor, int64_t host_cap);
void ep_wait(int64_t flags_ptr, int64_t n, int64_t epoch, int64_t device);
void ep_signal(std::vector<int64_t> flag, int64_t epoch, int64_t device);
void ep_gather(at::Tensor& out, const at::Tensor& rows_used, const at::Tensor& row_src, const at::Tensor& row_slot,
               int64_t payload_ptr, int64_t scale_ptr, int64_t P, int64_t n, bool fp8);
void ep_quant_rows(const at::Tensor& y, const at::Tensor& rows_used, int64_t q_ptr, int64_t scale_ptr,
                   bool stochastic, int64_t seed);
void ep_pull(at::Tensor& out, const at::Tensor& dest_tk, const at::Tensor& slot_tk,
             const c10::optional<at::Tensor>& w_tk, const c10::optional<at::Tensor>& pos_in,
             std::vector<int64_t> rowmap, std::vector<int64_t> src, std::vector<int64_t> src_scale, int64_t P,
             int64_t rows_cap, bool fp8, const c10::optional<at::Tensor>& y_save,
             const c10::optional<at::Tensor>& pos_out);
void ep_combine_bwd(at::Tensor& dy, const at::Tensor& rows_used, const at::Tensor& row_src, const at::Tensor& row_tok,
                    const at::Tensor& row_w, std::vector<int64_t> dout, int64_t T);
// zero_fused.cu
void zero_reduce_scatter(std::vector<std::vector<int64_t>> grad_ptrs, const std::vector<at::Tensor>& red,
                         std::vector<int64_t> cls, at::Tensor& stats_acc, std::vector<int64_t> stats_slots,
                         std::vector<int64_t> flag_stats, const at::Tensor& done, int64_t me, int64_t epoch,
                         bool publish, int64_t grid);
void zero_adam_allgather(std::vector<std::vector<int64_t>> param_ptrs, const std::vector<at::Tensor>& red,
                         const std::vector<at::Tensor>& master, const std::vector<at::Tensor>& m,
                         const std::vector<at::Tensor>& v, std::vector<double> lr, std::vector<double> wd,
                         int64_t stats_in_ptr, int64_t my_stats_flags_ptr, std::vector<int64_t> flag_params,
                         const at::Tensor& done, int64_t me, int64_t epoch, double b1, double b2, double eps,
                         int64_t step, double inv_dp, double max_norm, at::Tensor& grad_norm, at::Tensor& scale_out);
// symm.cpp
std::tuple<int64_t, py::bytes> symm_alloc(int64_t bytes);
int64_t symm_open(py::bytes handle);
void symm_close(int64_t peer_ptr);
void symm_free(int64_t ptr);
at::Tensor symm_local_view(int64_t ptr, int64_t offset_bytes, std::vector<int64_t> sizes, at::ScalarType dtype,
                           int64_t device);
}  // namespace ntb

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "nano_train_b200 sm_100a kernels";
  if (std::getenv("NTB_DEBUG_HOST")) signal(SIGSEGV, segv_backtrace);
  m.def("gemm_bf16", &ntb::gemm_bf16, "tcgen05 bf16 GEMM", py::arg("a"), py::arg("b"), py::arg("out"),
        py::arg("bias") = py::none(), py::arg("a_mn") = false, py::arg("b_mn") = false, py::arg("accumulate") = false,
        py::arg("alpha") = 1.0);
  m.def("gemm_grouped_bf16", &ntb::gemm_grouped_bf16, "grouped (mixture-of-experts) tcgen05 GEMM", py::arg("a"),
        py::arg("b"), py::arg("out"), py::arg("offsets"), py::arg("mode"), py::arg("b_mn") = false,
        py::arg("accumulate") = false, py::arg("c_group_stride") = 0);
  m.def("rmsnorm_fwd", &ntb::rmsnorm_fwd);
  m.def("rmsnorm_bwd", &ntb::rmsnorm_bwd, py::arg("dy"), py::arg("h"), py::arg("w"), py::arg("rstd"),
        py::arg("dres"), py::arg("dw_into") = py::none());
  m.def("layernorm_fwd", &ntb::layernorm_fwd);
  m.def("layernorm_bwd", &ntb::layernorm_bwd);
  m.def("rope_", &ntb::rope_);
  m.def("rope_table_", &ntb::rope_table_);
  m.def("mla_k_assemble", &ntb::mla_k_assemble, "MLA keys [nope | rope(kr)] per head in one launch");
  m.def("mla_k_assemble_bwd", &ntb::mla_k_assemble_bwd, "dK nope part into dkv, rope part summed over heads");
  m.def("swiglu_fwd", &ntb::swiglu_fwd);
  m.def("swiglu_bwd", &ntb::swiglu_bwd);
  m.def("gelu_fwd", &ntb::gelu_fwd);
  m.def("gelu_bwd", &ntb::gelu_bwd);
  m.def("ce_stats", &ntb::ce_stats);
  m.def("ce_bwd", &ntb::ce_bwd);
  m.def("embedding_fwd", &ntb::embedding_fwd);
  m.def("embedding_bwd_", &ntb::embedding_bwd_);
  m.def("adamw_flat_", &ntb::adamw_flat_);
  m.def("grad_stats_", &ntb::grad_stats_);
  m.def("flash_attn_fwd", &ntb::flash_attn_fwd);
  m.def("flash_attn_bwd", &ntb::flash_attn_bwd, py::arg("dout"), py::arg("q"), py::arg("k"), py::arg("v"),
        py::arg("out"), py::arg("lse"), py::arg("scale"), py::arg("causal"), py::arg("dq") = py::none(),
        py::arg("dk") = py::none(), py::arg("dv") = py::none());
  m.def("flash_attn_fwd_tc", &ntb::flash_attn_fwd_tc);
  m.def("gemm_fp8_blockscaled", &ntb::gemm_fp8_blockscaled, py::arg("a_q"), py::arg("sa"), py::arg("b_q"),
        py::arg("sb"), py::arg("out"), py::arg("bias") = py::none());
  m.def("fp8_quantize", &ntb::fp8_quantize);
  m.def("nvfp4_quantize", &ntb::nvfp4_quantize);
  m.def("dropout_apply", &ntb::dropout_apply);
  m.def("persistent_quantize", &ntb::persistent_quantize);
  m.def("persistent_dequantize", &ntb::persistent_dequantize);
  m.def("nvfp4_dequantize", &ntb::nvfp4_dequantize);
  m.def("gemm_nvfp4", &ntb::gemm_nvfp4, py::arg("a_q"), py::arg("sfa"), py::arg("gsa"), py::arg("b_q"),
        py::arg("sfb"), py::arg("gsb"), py::arg("out"), py::arg("bias") = py::none());
  m.def("fp8_quant_dequant", &ntb::fp8_quant_dequant);
  m.def("fp8_quant_dequant_strided", &ntb::fp8_quant_dequant_strided);
  m.def("fp8_quantize_strided", &ntb::fp8_quantize_strided);
  m.def("fp8_quantize_with_dq", &ntb::fp8_quantize_with_dq);
  m.def("gemm_fp8_grouped", &ntb::gemm_fp8_grouped);
  m.def("fp8_dequantize", &ntb::fp8_dequantize);
  m.def("ag_gemm", &ntb::ag_gemm, py::arg("x_local"), py::arg("x_full_out"), py::arg("w"), py::arg("y"),
        py::arg("bias"), py::arg("b_mn"), py::arg("slots"), py::arg("ready"), py::arg("ctrs"), py::arg("rank"),
        py::arg("epoch"), py::arg("trace") = py::none());
  m.def("gemm_rs", &ntb::gemm_rs, py::arg("x"), py::arg("w"), py::arg("out"), py::arg("bias"), py::arg("b_mn"),
        py::arg("recv"), py::arg("tctrs"), py::arg("ctrs"), py::arg("rank"), py::arg("epoch"),
        py::arg("trace") = py::none());
  m.def("rs_pull", &ntb::rs_pull, py::arg("parts"), py::arg("out"), py::arg("bias"), py::arg("rank"),
        py::arg("flags_ptr") = 0, py::arg("epoch") = 0);
  m.def("gemm_rsp", &ntb::gemm_rsp, "GEMM + reduce-scatter with progressive peer pulls", py::arg("x"),
        py::arg("w"), py::arg("out"), py::arg("bias"), py::arg("b_mn"), py::arg("parts"), py::arg("rdy"),
        py::arg("my_rdy"), py::arg("tpc_stride"), py::arg("acc"), py::arg("acc_cnt"), py::arg("ctrs"),
        py::arg("rank"), py::arg("epoch"), py::arg("trace") = py::none());
  m.def("gemm_bf16_publish", &ntb::gemm_bf16_publish, "tcgen05 bf16 GEMM whose last CTA publishes an epoch",
        py::arg("a"), py::arg("b"), py::arg("out"), py::arg("b_mn"), py::arg("flags"), py::arg("epoch"),
        py::arg("ctr"));
  m.def("wait_flag", &ntb::wait_flag, py::arg("flag"), py::arg("expect"), py::arg("limit_ns"));
  m.def("ep_dispatch", &ntb::ep_dispatch, py::arg("x"), py::arg("idx"), py::arg("w"), py::arg("dest_tk"),
        py::arg("slot_tk"), py::arg("ctr"), py::arg("epr"), py::arg("payload"), py::arg("pscale"), py::arg("meta"),
        py::arg("flag"), py::arg("info"), py::arg("done"), py::arg("P"), py::arg("epoch"), py::arg("fp8"),
        py::arg("stochastic"), py::arg("seed"));
  m.def("ep_recv_keys", &ntb::ep_recv_keys);
  m.def("ep_recv_layout", &ntb::ep_recv_layout);
  m.def("ep_wait", &ntb::ep_wait);
  m.def("router_fwd", &ntb::router_fwd);
  m.def("zero_reduce_scatter", &ntb::zero_reduce_scatter, py::arg("grad_ptrs"), py::arg("red"), py::arg("cls"),
        py::arg("stats_acc"), py::arg("stats_slots"), py::arg("flag_stats"), py::arg("done"), py::arg("me"),
        py::arg("epoch"), py::arg("publish") = true, py::arg("grid") = 0);
  m.def("zero_adam_allgather", &ntb::zero_adam_allgather);
  m.def("router_bwd", &ntb::router_bwd);
  m.def("ep_signal", &ntb::ep_signal);
  m.def("ep_gather", &ntb::ep_gather);
  m.def("ep_quant_rows", &ntb::ep_quant_rows);
  m.def("ep_pull", &ntb::ep_pull, py::arg("out"), py::arg("dest_tk"), py::arg("slot_tk"), py::arg("w_tk"),
        py::arg("pos_in"), py::arg("rowmap"), py::arg("src"), py::arg("src_scale"), py::arg("P"),
        py::arg("rows_cap"), py::arg("fp8"), py::arg("y_save") = py::none(), py::arg("pos_out") = py::none());
  m.def("ep_combine_bwd", &ntb::ep_combine_bwd);
  m.def("symm_alloc", &ntb::symm_alloc);
  m.def("symm_open", &ntb::symm_open);
  m.def("symm_close", &ntb::symm_close);
  m.def("symm_free", &ntb::symm_free);
  m.def("symm_local_view", &ntb::symm_local_view);
  m.def("num_sms", &ntb::num_sms);
  m.def("launch_count", &ntb::launch_count);
  m.def("read_and_clear_status", &ntb::read_and_clear_status);
}
