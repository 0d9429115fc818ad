// Python bindings of the sm_100a kernel library (module nano_qwen_b200._C).
#include <torch/extension.h>

#include <vector>

namespace nq {
// gemm.cu
torch::Tensor gemm_nt(torch::Tensor A, torch::Tensor B);
int64_t gemm_pair_mode(int64_t mode);
void gemm_nt_out(torch::Tensor A, torch::Tensor B, torch::Tensor C);
std::vector<torch::Tensor> gemm_nt_swiglu(torch::Tensor A, torch::Tensor B);
torch::Tensor gemm_nn(torch::Tensor A, torch::Tensor B);
void gemm_nn_out(torch::Tensor A, torch::Tensor B, torch::Tensor C);
void gemm_tn_acc(torch::Tensor A, torch::Tensor B, torch::Tensor C);
torch::Tensor grouped_gemm_nt(torch::Tensor X, torch::Tensor W, torch::Tensor offsets, int64_t, int64_t, int64_t,
                              int64_t, int64_t, int64_t);
torch::Tensor grouped_gemm_nn(torch::Tensor dY, torch::Tensor W, torch::Tensor offsets, int64_t, int64_t, int64_t,
                              int64_t, int64_t, int64_t);
void grouped_gemm_tn_acc(torch::Tensor dY, torch::Tensor X, torch::Tensor dW, torch::Tensor offsets);
// norm.cu
std::vector<torch::Tensor> add_rmsnorm_fwd(torch::Tensor, c10::optional<torch::Tensor>, torch::Tensor, double);
std::vector<torch::Tensor> add_rmsnorm_bwd(torch::Tensor, c10::optional<torch::Tensor>, torch::Tensor,
                                           torch::Tensor, torch::Tensor, c10::optional<torch::Tensor>);
std::vector<torch::Tensor> rmsnorm_fwd(torch::Tensor, torch::Tensor, double, c10::ScalarType);
torch::Tensor rmsnorm_bwd(torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, c10::optional<torch::Tensor>);
std::vector<torch::Tensor> layernorm_fwd(torch::Tensor, torch::Tensor, c10::optional<torch::Tensor>, double, c10::ScalarType);
torch::Tensor layernorm_bwd(torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor,
                            c10::optional<torch::Tensor>, c10::optional<torch::Tensor>);
// rope.cu
std::vector<torch::Tensor> qknorm_rope_fwd(torch::Tensor, c10::optional<torch::Tensor>, c10::optional<torch::Tensor>,
                                           torch::Tensor, torch::Tensor, c10::optional<torch::Tensor>, int64_t,
                                           int64_t, int64_t, int64_t, int64_t, double);
void qknorm_rope_bwd(torch::Tensor, torch::Tensor, c10::optional<torch::Tensor>, c10::optional<torch::Tensor>,
                     torch::Tensor, torch::Tensor, torch::Tensor, c10::optional<torch::Tensor>, torch::Tensor,
                     c10::optional<torch::Tensor>, c10::optional<torch::Tensor>, int64_t, int64_t, int64_t,
                     int64_t, int64_t);
// attention
std::vector<torch::Tensor> attn_fwd(torch::Tensor, torch::Tensor, int64_t, int64_t, int64_t, int64_t, int64_t, bool, double,
                                    c10::optional<torch::Tensor>);
torch::Tensor attn_bwd(torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor,
                       int64_t, int64_t, int64_t, int64_t, int64_t, bool, double, c10::optional<torch::Tensor>);
std::vector<torch::Tensor> attn_fwd_cp(torch::Tensor, torch::Tensor, int64_t, int64_t, int64_t, int64_t, int64_t,
                                       int64_t, int64_t, int64_t, int64_t, double, int64_t, int64_t, int64_t);
std::vector<torch::Tensor> attn_bwd_cp(torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor,
                                       int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                                       int64_t, double, c10::optional<torch::Tensor>);
// cp_comm.cu
int64_t cp_kv_scatter(std::vector<int64_t>, std::vector<int64_t>, int64_t, torch::Tensor, torch::Tensor,
                      torch::Tensor, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, torch::Tensor,
                      int64_t);
void cp_signal(std::vector<int64_t>, std::vector<int64_t>, int64_t, int64_t, int64_t);
torch::Tensor cp_dkv_gather(std::vector<int64_t>, std::vector<int64_t>, int64_t, torch::Tensor, int64_t, int64_t,
                            int64_t, int64_t, int64_t);
torch::Tensor decode_attn(torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, double);
// elementwise.cu
int64_t error_flag_read();
void error_flag_clear();
void wait_limits_set(int64_t, int64_t);
std::vector<int64_t> wait_limits_get();
torch::Tensor swiglu_fwd(torch::Tensor);
torch::Tensor swiglu_bwd(torch::Tensor, torch::Tensor);
torch::Tensor gelu_fwd(torch::Tensor);
torch::Tensor gelu_bwd(torch::Tensor, torch::Tensor);
void scale_inplace(torch::Tensor, torch::Tensor);
void axpy_(torch::Tensor, torch::Tensor, torch::Tensor);
torch::Tensor embedding_fwd(torch::Tensor, torch::Tensor);
void embedding_bwd(torch::Tensor, torch::Tensor, torch::Tensor);
torch::Tensor ce_count_valid(torch::Tensor);
void ce_fused_chunk(torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, bool);
void ce_lse_chunk(torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor);
void ce_grad_chunk(torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor);
torch::Tensor sum_squares(torch::Tensor);
void adamw_flat(torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor,
                int64_t, int64_t, int64_t, int64_t, double, double, double, double, double, double, double, double);
// moe.cu
std::vector<torch::Tensor> router_fwd(torch::Tensor, int64_t, bool);
torch::Tensor router_bwd(torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, bool);
std::vector<torch::Tensor> moe_plan(torch::Tensor, int64_t, int64_t, int64_t);
torch::Tensor moe_gather(torch::Tensor, torch::Tensor);
torch::Tensor moe_combine(torch::Tensor, torch::Tensor, torch::Tensor);
std::vector<torch::Tensor> moe_combine_bwd(torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor);
torch::Tensor moe_scatter_add(torch::Tensor, torch::Tensor, int64_t);
// tensor-parallel fused communication (gemm.cu, tp_comm.cu)
torch::Tensor gemm_ag(torch::Tensor, torch::Tensor, bool, int64_t, int64_t, int64_t);
int64_t gemm_rs(torch::Tensor, torch::Tensor, bool, std::vector<int64_t>, int64_t, torch::Tensor, int64_t,
                std::vector<int64_t>, int64_t, int64_t);
int64_t tp_norm_fwd(torch::Tensor, c10::optional<torch::Tensor>, c10::optional<torch::Tensor>, torch::Tensor,
                    torch::Tensor, torch::Tensor, torch::Tensor, double, std::vector<int64_t>, torch::Tensor,
                    std::vector<int64_t>, int64_t, int64_t, int64_t, int64_t, int64_t, torch::Tensor, int64_t);
int64_t tp_norm_bwd(c10::optional<torch::Tensor>, c10::optional<torch::Tensor>, c10::optional<torch::Tensor>,
                    torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor,
                    c10::optional<torch::Tensor>, std::vector<int64_t>, torch::Tensor, std::vector<int64_t>,
                    int64_t, int64_t, int64_t, int64_t, int64_t, torch::Tensor, int64_t);
// ep_comm.cu
void ep_layout(std::vector<int64_t>, std::vector<int64_t>, int64_t, torch::Tensor, int64_t, int64_t, int64_t,
               torch::Tensor, torch::Tensor, torch::Tensor, int64_t);
int64_t ep_dispatch(std::vector<int64_t>, std::vector<int64_t>, std::vector<int64_t>, int64_t, torch::Tensor,
                    torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor,
                    torch::Tensor, int64_t, int64_t, int64_t, torch::Tensor, int64_t);
void ep_wait(std::vector<int64_t>, std::vector<int64_t>, int64_t, int64_t, int64_t);
void ep_signal(std::vector<int64_t>, std::vector<int64_t>, int64_t, int64_t, int64_t);
void ep_combine(std::vector<int64_t>, std::vector<int64_t>, std::vector<int64_t>, int64_t, torch::Tensor,
                torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, int64_t, int64_t);
int64_t ep_combine_bwd(std::vector<int64_t>, std::vector<int64_t>, std::vector<int64_t>, int64_t, torch::Tensor,
                       torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor, int64_t, int64_t,
                       torch::Tensor, int64_t);
void ep_dispatch_bwd(std::vector<int64_t>, std::vector<int64_t>, std::vector<int64_t>, int64_t, torch::Tensor,
                     torch::Tensor, torch::Tensor, int64_t, int64_t);
// zero_comm.cu
void zero_rs(std::vector<int64_t>, std::vector<int64_t>, std::vector<int64_t>, int64_t, int64_t, int64_t,
             torch::Tensor, int64_t, int64_t, double);
void zero_clip(torch::Tensor, double, torch::Tensor, torch::Tensor);
void zero_adamw_ag(std::vector<int64_t>, std::vector<int64_t>, std::vector<int64_t>, int64_t, torch::Tensor,
                   torch::Tensor, torch::Tensor, torch::Tensor, int64_t, int64_t, int64_t, int64_t, double,
                   double, double, double, double, double, double, double);
void zero_publish(std::vector<int64_t>, std::vector<int64_t>, std::vector<int64_t>, int64_t, int64_t);
}  // namespace nq

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "nano_qwen_b200 sm_100a kernels";
  m.def("gemm_nt", &nq::gemm_nt, "C = A @ B^T (bf16, tcgen05)");
  m.def("gemm_nt_out", &nq::gemm_nt_out);
  m.def("gemm_pair_mode", &nq::gemm_pair_mode,
        "CTA-pair (cta_group::2) GEMMs: 1 on, 0 off, <0 query; returns the previous mode");
  m.def("gemm_nt_swiglu", &nq::gemm_nt_swiglu, "gu = A @ [gate; up]^T, h = silu(g) * u (one GEMM)");
  m.def("gemm_nn", &nq::gemm_nn, "C = A @ B (bf16, tcgen05)");
  m.def("gemm_nn_out", &nq::gemm_nn_out);
  m.def("gemm_tn_acc", &nq::gemm_tn_acc, "C(fp32) += A^T @ B (tcgen05)");
  m.def("grouped_gemm_nt", &nq::grouped_gemm_nt,
        "rows grouped by expert segments: C[r] = X[r] @ W[g(r)]^T; ep_*: wait per source rank for "
        "expert-parallel dispatch flags before loading a tile's rows",
        py::arg("X"), py::arg("W"), py::arg("offsets"), py::arg("ep_counts") = 0, py::arg("ep_flags") = 0,
        py::arg("ep_seq") = 0, py::arg("ep_world") = 0, py::arg("ep_E") = 0, py::arg("ep_expert0") = 0);
  m.def("grouped_gemm_nn", &nq::grouped_gemm_nn,
        "rows grouped by expert segments: C[r] = dY[r] @ W[g(r)]; ep_*: as grouped_gemm_nt",
        py::arg("dY"), py::arg("W"), py::arg("offsets"), py::arg("ep_counts") = 0, py::arg("ep_flags") = 0,
        py::arg("ep_seq") = 0, py::arg("ep_world") = 0, py::arg("ep_E") = 0, py::arg("ep_expert0") = 0);
  m.def("grouped_gemm_tn_acc", &nq::grouped_gemm_tn_acc);
  m.def("add_rmsnorm_fwd", &nq::add_rmsnorm_fwd);
  m.def("add_rmsnorm_bwd", &nq::add_rmsnorm_bwd);
  m.def("rmsnorm_fwd", &nq::rmsnorm_fwd);
  m.def("rmsnorm_bwd", &nq::rmsnorm_bwd);
  m.def("layernorm_fwd", &nq::layernorm_fwd);
  m.def("layernorm_bwd", &nq::layernorm_bwd);
  m.def("qknorm_rope_fwd", &nq::qknorm_rope_fwd);
  m.def("qknorm_rope_bwd", &nq::qknorm_rope_bwd);
  m.def("attn_fwd", &nq::attn_fwd, "causal / full GQA flash attention forward; kv_lo: per-query first visible key",
        py::arg("qk"), py::arg("qkv"), py::arg("B"), py::arg("S"), py::arg("Hq"), py::arg("Hk"), py::arg("D"),
        py::arg("causal"), py::arg("scale"), py::arg("kv_lo") = py::none());
  m.def("attn_bwd", &nq::attn_bwd, "attention backward; q_hi: per-key end of the queries that see it",
        py::arg("dO"), py::arg("qk"), py::arg("qkv"), py::arg("O"), py::arg("lse"), py::arg("dqkv"), py::arg("B"),
        py::arg("S"), py::arg("Hq"), py::arg("Hk"), py::arg("D"), py::arg("causal"), py::arg("scale"),
        py::arg("q_hi") = py::none());
  m.def("attn_fwd_cp", &nq::attn_fwd_cp, "context-parallel attention forward (local queries, gathered keys)");
  m.def("attn_bwd_cp", &nq::attn_bwd_cp, "context-parallel attention backward");
  m.def("cp_kv_scatter", &nq::cp_kv_scatter, "store local k|v rows into every CP rank's gathered buffer (P2P)");
  m.def("cp_signal", &nq::cp_signal);
  m.def("cp_dkv_gather", &nq::cp_dkv_gather, "sum every CP rank's dk|dv partials of the local tokens (P2P)");
  m.def("decode_attn", &nq::decode_attn);
  m.def("error_flag_read", &nq::error_flag_read);
  m.def("error_flag_clear", &nq::error_flag_clear);
  m.def("wait_limits_set", &nq::wait_limits_set,
        "bounded-wait limits of the current device in ns (mbarrier, peer flag); <= 0 keeps a value");
  m.def("wait_limits_get", &nq::wait_limits_get);
  m.def("swiglu_fwd", &nq::swiglu_fwd);
  m.def("swiglu_bwd", &nq::swiglu_bwd);
  m.def("gelu_fwd", &nq::gelu_fwd);
  m.def("gelu_bwd", &nq::gelu_bwd);
  m.def("scale_inplace", &nq::scale_inplace);
  m.def("axpy_", &nq::axpy_);
  m.def("embedding_fwd", &nq::embedding_fwd);
  m.def("embedding_bwd", &nq::embedding_bwd);
  m.def("ce_count_valid", &nq::ce_count_valid);
  m.def("ce_fused_chunk", &nq::ce_fused_chunk);
  m.def("ce_lse_chunk", &nq::ce_lse_chunk);
  m.def("ce_grad_chunk", &nq::ce_grad_chunk);
  m.def("sum_squares", &nq::sum_squares);
  m.def("adamw_flat", &nq::adamw_flat);
  m.def("router_fwd", &nq::router_fwd);
  m.def("router_bwd", &nq::router_bwd);
  m.def("moe_plan", &nq::moe_plan);
  m.def("moe_gather", &nq::moe_gather);
  m.def("moe_combine", &nq::moe_combine);
  m.def("moe_combine_bwd", &nq::moe_combine_bwd);
  m.def("moe_scatter_add", &nq::moe_scatter_add);
  m.def("gemm_ag", &nq::gemm_ag, "GEMM whose A rows arrive from peers (waits on all-gather flags)");
  m.def("gemm_rs", &nq::gemm_rs, "GEMM whose row tiles are stored into their owners' partial buffers");
  m.def("tp_norm_fwd", &nq::tp_norm_fwd, "residual + sum of TP partials + RMSNorm, all-gathered to peers");
  m.def("tp_norm_bwd", &nq::tp_norm_bwd, "RMSNorm backward with TP partial inputs and all-gathered output");
  m.def("ep_layout", &nq::ep_layout, "exchange per-expert counts and compute the dispatch layout");
  m.def("ep_dispatch", &nq::ep_dispatch, "store token rows into the expert owners' receive buffers (P2P)");
  m.def("ep_wait", &nq::ep_wait);
  m.def("ep_signal", &nq::ep_signal);
  m.def("ep_combine", &nq::ep_combine, "pull expert outputs (P2P) and form the weighted top-k sum");
  m.def("ep_combine_bwd", &nq::ep_combine_bwd);
  m.def("ep_dispatch_bwd", &nq::ep_dispatch_bwd);
  m.def("zero_rs", &nq::zero_rs, "peer-memory reduce-scatter of the mean gradient + squared norm");
  m.def("zero_clip", &nq::zero_clip);
  m.def("zero_adamw_ag", &nq::zero_adamw_ag, "sharded AdamW fused with the bf16 all-gather by P2P stores");
  m.def("zero_publish", &nq::zero_publish);
}
