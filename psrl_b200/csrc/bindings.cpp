// Python bindings of the psrl_b200 CUDA kernels (module psrl_b200._C).
#include <torch/extension.h>

namespace psrl {
std::vector<at::Tensor> rmsnorm_fwd(at::Tensor x, c10::optional<at::Tensor> residual, at::Tensor w, double eps);
std::vector<at::Tensor> rmsnorm_bwd(at::Tensor dy, at::Tensor s, at::Tensor w, at::Tensor rstd,
                                    c10::optional<at::Tensor> dres);
at::Tensor head_rmsnorm_(at::Tensor x, at::Tensor w, double eps);
void rope_(at::Tensor qkv, at::Tensor positions, at::Tensor cos_t, at::Tensor sin_t, int64_t nq, int64_t nkv,
           int64_t d, bool inverse, c10::optional<at::Tensor> k_cache, c10::optional<at::Tensor> v_cache,
           c10::optional<at::Tensor> slots);
at::Tensor swiglu_fwd(at::Tensor gu);
at::Tensor swiglu_bwd(at::Tensor gu, at::Tensor dout);
void adamw_(at::Tensor p, at::Tensor g, at::Tensor m, at::Tensor v, c10::optional<at::Tensor> p16, double lr,
            double b1, double b2, double eps, double wd, int64_t step, c10::optional<at::Tensor> gscale_t,
            double gscale);
void sqnorm_accumulate_(at::Tensor x, at::Tensor out, at::Tensor partial);
void clip_coef_(at::Tensor sq, double max_norm, at::Tensor coef, at::Tensor norm_out);
std::vector<at::Tensor> logprob_fwd(at::Tensor logits, at::Tensor labels, double temperature, bool want_entropy);
void logprob_bwd_(at::Tensor logits, at::Tensor labels, double temperature, c10::optional<at::Tensor> glp,
                  c10::optional<at::Tensor> gent, at::Tensor lse, c10::optional<at::Tensor> ent);
std::vector<at::Tensor> sample(at::Tensor logits, c10::optional<at::Tensor> temps, c10::optional<at::Tensor> seeds,
                               c10::optional<at::Tensor> streams);
std::vector<at::Tensor> attn_varlen_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor cu_seqlens,
                                        int64_t max_seqlen, double scale, bool want_lse);
at::Tensor attn_paged_prefill(at::Tensor q, at::Tensor k_cache, at::Tensor v_cache, at::Tensor cu_q,
                              at::Tensor kv_lens, at::Tensor block_table, int64_t max_q_len, double scale);
std::vector<at::Tensor> attn_varlen_bwd(at::Tensor dO, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o,
                                        at::Tensor lse, at::Tensor cu_seqlens, int64_t max_seqlen, double scale);
int64_t decode_num_splits(int64_t batch, int64_t nkv, int64_t max_ctx);
at::Tensor attn_decode(at::Tensor q, at::Tensor k_cache, at::Tensor v_cache, at::Tensor block_table,
                       at::Tensor kv_lens, double scale, int64_t splits, c10::optional<at::Tensor> scratch,
                       int64_t stages);
std::tuple<pybind11::bytes, int64_t> ipc_handle(at::Tensor t);
at::Tensor ipc_open(pybind11::bytes handle, int64_t offset, int64_t numel, at::ScalarType dtype, int64_t src_device);
void enable_peer_access(int64_t peer);
void scatter_segments(at::Tensor src, std::vector<at::Tensor> dsts, std::vector<int64_t> src_offsets_bytes,
                      std::vector<int64_t> lengths_bytes);
void copy_rows(at::Tensor dst, at::Tensor table, at::Tensor start);
void copy_segments(at::Tensor dst, std::vector<at::Tensor> srcs, std::vector<int64_t> dst_offsets_bytes,
                   std::vector<int64_t> src_offsets_bytes, std::vector<int64_t> lengths_bytes);
at::Tensor tc_gemm(at::Tensor a, at::Tensor b, at::Tensor err);
at::Tensor tc_grouped_gemm(at::Tensor a, at::Tensor w, at::Tensor seg, at::Tensor err);
at::Tensor tc_gemm2(at::Tensor a, at::Tensor b, bool a_mn, bool b_mn, c10::optional<at::Tensor> out, int64_t splits,
                    int64_t group_m, c10::optional<at::Tensor> bias, at::Tensor err);
std::vector<at::Tensor> tc_gemm2_swiglu(at::Tensor x, at::Tensor w, int64_t group_m, at::Tensor err);
void tc_gemm2_allreduce2(at::Tensor a, at::Tensor b, bool b_mn, at::Tensor acc_local, at::Tensor acc_peer,
                         int64_t group_m, at::Tensor err);
void peer_barrier(std::vector<at::Tensor> flags_in_peer, std::vector<at::Tensor> own_slots, int64_t epoch,
                  double timeout_s, at::Tensor err);
void acc_finalize(at::Tensor acc, at::Tensor out, c10::optional<at::Tensor> bias);
at::Tensor tc_gemm_skinny(at::Tensor x, at::Tensor w, c10::optional<at::Tensor> bias, bool swiglu, int64_t split,
                          at::Tensor err);
std::vector<at::Tensor> attn_fwd_sm100_kv(at::Tensor q, at::Tensor kv, at::Tensor cu_q, at::Tensor cu_k,
                                          int64_t max_q, int64_t nq, int64_t nkv, double scale, bool want_lse,
                                          at::Tensor err);
std::vector<at::Tensor> attn_bwd_sm100_kv(at::Tensor q, at::Tensor kv, at::Tensor o, at::Tensor dout, at::Tensor lse,
                                          at::Tensor cu_q, at::Tensor cu_k, int64_t max_q, int64_t max_k, int64_t nq,
                                          int64_t nkv, double scale, at::Tensor err);
std::vector<at::Tensor> attn_fwd_sm100(at::Tensor qkv, at::Tensor cu_seqlens, int64_t max_seqlen, int64_t nq,
                                       int64_t nkv, double scale, bool want_lse, at::Tensor err);
at::Tensor attn_bwd_sm100(at::Tensor qkv, at::Tensor o, at::Tensor dout, at::Tensor lse, at::Tensor cu_seqlens,
                          int64_t max_seqlen, int64_t nq, int64_t nkv, double scale, at::Tensor err);
std::vector<at::Tensor> moe_route(at::Tensor logits, c10::optional<at::Tensor> prior, int64_t k, bool renorm);
std::vector<at::Tensor> moe_permute(at::Tensor ids, at::Tensor counts, int64_t bm, int64_t tiles_n);
at::Tensor moe_gather(at::Tensor x, at::Tensor token_of_row);
at::Tensor moe_combine(at::Tensor ys, at::Tensor pos, at::Tensor w);
void peer_reduce(std::vector<at::Tensor> grads, std::vector<at::Tensor> flats, at::Tensor start, at::Tensor src_off,
                 at::Tensor red, at::Tensor sq, at::Tensor partial);
void peer_adamw(std::vector<at::Tensor> grads, std::vector<at::Tensor> flats, at::Tensor start, at::Tensor src_off,
                at::Tensor master, at::Tensor red, at::Tensor m, at::Tensor v, double lr, double b1, double b2,
                double eps, double wd, int64_t step, at::Tensor coef, double gscale);
std::vector<at::Tensor> tc_linear_logprob(at::Tensor h, at::Tensor w, at::Tensor labels, double temperature,
                                          at::Tensor err);
void kv_copy_blocks(at::Tensor src_layers, at::Tensor dst_layers, at::Tensor src_blk, at::Tensor dst_blk,
                    int64_t block_bytes, int64_t src_blocks, int64_t dst_blocks);
bool kernel_checks_enabled();
std::vector<int64_t> kernel_check_status(bool clear);
void register_vmm(pybind11::module& m);
pybind11::dict green_partition(int64_t device, int64_t reserve_sms, int64_t priority);
}  // namespace psrl

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "psrl_b200 sm_100a kernels";
  m.def("rmsnorm_fwd", &psrl::rmsnorm_fwd);
  m.def("rmsnorm_bwd", &psrl::rmsnorm_bwd);
  m.def("head_rmsnorm_", &psrl::head_rmsnorm_);
  m.def("rope_", &psrl::rope_);
  m.def("swiglu_fwd", &psrl::swiglu_fwd);
  m.def("swiglu_bwd", &psrl::swiglu_bwd);
  m.def("adamw_", &psrl::adamw_);
  m.def("sqnorm_accumulate_", &psrl::sqnorm_accumulate_);
  m.def("clip_coef_", &psrl::clip_coef_);
  m.def("logprob_fwd", &psrl::logprob_fwd);
  m.def("logprob_bwd_", &psrl::logprob_bwd_);
  m.def("sample", &psrl::sample);
  m.def("attn_varlen_fwd", &psrl::attn_varlen_fwd);
  m.def("attn_paged_prefill", &psrl::attn_paged_prefill);
  m.def("attn_varlen_bwd", &psrl::attn_varlen_bwd);
  m.def("decode_num_splits", &psrl::decode_num_splits);
  m.def("attn_decode", &psrl::attn_decode, pybind11::arg("q"), pybind11::arg("k_cache"), pybind11::arg("v_cache"),
        pybind11::arg("block_table"), pybind11::arg("kv_lens"), pybind11::arg("scale"), pybind11::arg("splits"), pybind11::arg("scratch"),
        pybind11::arg("stages") = 0);
  m.def("ipc_handle", &psrl::ipc_handle);
  m.def("ipc_open", &psrl::ipc_open);
  m.def("enable_peer_access", &psrl::enable_peer_access);
  m.def("copy_segments", &psrl::copy_segments);
  m.def("scatter_segments", &psrl::scatter_segments);
  m.def("copy_rows", &psrl::copy_rows);
  m.def("tc_gemm", &psrl::tc_gemm);
  m.def("tc_grouped_gemm", &psrl::tc_grouped_gemm);
  m.def("tc_gemm2", &psrl::tc_gemm2);
  m.def("tc_gemm2_swiglu", &psrl::tc_gemm2_swiglu);
  m.def("tc_gemm_skinny", &psrl::tc_gemm_skinny);
  m.def("tc_gemm2_allreduce2", &psrl::tc_gemm2_allreduce2);
  m.def("peer_barrier", &psrl::peer_barrier);
  m.def("acc_finalize", &psrl::acc_finalize);
  m.def("attn_fwd_sm100", &psrl::attn_fwd_sm100);
  m.def("attn_fwd_sm100_kv", &psrl::attn_fwd_sm100_kv);
  m.def("attn_bwd_sm100_kv", &psrl::attn_bwd_sm100_kv);
  m.def("attn_bwd_sm100", &psrl::attn_bwd_sm100);
  m.def("moe_route", &psrl::moe_route);
  m.def("moe_permute", &psrl::moe_permute);
  m.def("moe_gather", &psrl::moe_gather);
  m.def("moe_combine", &psrl::moe_combine);
  m.def("peer_reduce", &psrl::peer_reduce);
  m.def("peer_adamw", &psrl::peer_adamw);
  m.def("tc_linear_logprob", &psrl::tc_linear_logprob);
  m.def("kv_copy_blocks", &psrl::kv_copy_blocks, py::arg("src_layers"), py::arg("dst_layers"), py::arg("src_blk"),
        py::arg("dst_blk"), py::arg("block_bytes"), py::arg("src_blocks") = 0, py::arg("dst_blocks") = 0);
  m.def("kernel_checks_enabled", &psrl::kernel_checks_enabled);
  m.def("kernel_check_status", &psrl::kernel_check_status, py::arg("clear") = true);
  psrl::register_vmm(m);
  m.def("green_partition", &psrl::green_partition);
}
