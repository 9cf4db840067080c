// Python bindings of the sm_100a kernels (module tiny_dsv41_b200._C).
#include <execinfo.h>
#include <signal.h>
#include <torch/extension.h>
#include <unistd.h>

#include <cstdlib>
#include <vector>

namespace {
// Debug aid (TDSV_SEGV_BACKTRACE=1): print the native stack of a crashing thread to stderr.
void segv_handler(int sig) {
  void* frames[64];
  const int n = backtrace(frames, 64);
  const char msg[] = "tiny_dsv41_b200: native backtrace of the faulting thread:\n";
  ssize_t ignored = write(STDERR_FILENO, msg, sizeof(msg) - 1);
  (void)ignored;
  backtrace_symbols_fd(frames, n, STDERR_FILENO);
  signal(sig, SIG_DFL);
  raise(sig);
}
void maybe_install_segv_handler() {
  const char* flag = std::getenv("TDSV_SEGV_BACKTRACE");
  if (flag != nullptr && flag[0] == '1') {
    struct sigaction sa {};
    sa.sa_handler = segv_handler;
    sigemptyset(&sa.sa_mask);
    sigaction(SIGSEGV, &sa, nullptr);
  }
}
}  // namespace

namespace tdsv {
// status
int64_t read_status();
at::Tensor status_word();
void set_peer_wait_limit_ns(int64_t ns);
uint64_t peer_wait_limit_ns();
// norm.cu
std::vector<at::Tensor> moe_route_plan(const at::Tensor& ids, int64_t num_experts, int64_t block,
                                       const c10::optional<at::Tensor>& slab_counts, int64_t slab);
std::vector<at::Tensor> ep_dest_plan(const at::Tensor& ids, int64_t experts_per_rank, int64_t ranks);
at::Tensor fp4_dequant(const at::Tensor& packed, const at::Tensor& scale);
void fp4_grouped_gemm(const at::Tensor& a, const at::Tensor& codes, const at::Tensor& scales,
                      const at::Tensor& group_off, const at::Tensor& group_rows, at::Tensor& out, bool b_mn,
                      int64_t max_rows);
std::vector<at::Tensor> rmsnorm_fwd(const at::Tensor& x, const at::Tensor& w, double eps);
std::vector<at::Tensor> rmsnorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w,
                                    const at::Tensor& rstd, bool need_dw);
at::Tensor column_sum(const at::Tensor& partial);
// rope.cu
std::vector<at::Tensor> qk_norm_rope_fwd(const at::Tensor& qkv, const at::Tensor& wq, const at::Tensor& wk,
                                         const at::Tensor& pos, const at::Tensor& inv_freq, int64_t hq, int64_t hkv,
                                         double eps);
std::vector<at::Tensor> qk_norm_rope_bwd(const at::Tensor& dq, const at::Tensor& dk, const at::Tensor& dv,
                                         const at::Tensor& qkv, const at::Tensor& wq, const at::Tensor& wk,
                                         const at::Tensor& pos, const at::Tensor& inv_freq, int64_t hq, int64_t hkv,
                                         double eps);
at::Tensor rope_interleaved(const at::Tensor& x, const at::Tensor& pos, const at::Tensor& inv_freq, int64_t rope_dim,
                            bool inverse);
// router.cu
std::vector<at::Tensor> router_fwd(const at::Tensor& logits, const c10::optional<at::Tensor>& bias, int64_t k,
                                   int64_t func, bool normalize, double norm_eps, double scale);
at::Tensor router_bwd(const at::Tensor& dweights, const at::Tensor& ids, const at::Tensor& scores,
                      const at::Tensor& logits, const c10::optional<at::Tensor>& aux_coef, int64_t func,
                      bool normalize, double norm_eps, double scale);
// moe_permute.cu
at::Tensor moe_gather(const at::Tensor& x, const at::Tensor& src, const c10::optional<at::Tensor>& row_limit);
at::Tensor moe_combine(const at::Tensor& rows, const at::Tensor& idx, const c10::optional<at::Tensor>& w);
std::vector<at::Tensor> moe_combine_bwd(const at::Tensor& dout, const at::Tensor& rows, const at::Tensor& idx,
                                        const c10::optional<at::Tensor>& w, bool need_dw);
void moe_zero_padding(at::Tensor& buf, const at::Tensor& src, const c10::optional<at::Tensor>& row_limit);
// swiglu.cu
at::Tensor swiglu_fwd(const at::Tensor& gu, const c10::optional<at::Tensor>& w, bool interleaved, double limit,
                      const c10::optional<at::Tensor>& row_limit);
std::vector<at::Tensor> swiglu_bwd(const at::Tensor& dout, const at::Tensor& gu, const c10::optional<at::Tensor>& w,
                                   bool interleaved, double limit, bool need_dw,
                                   const c10::optional<at::Tensor>& row_limit);
// loss.cu
std::vector<at::Tensor> cross_entropy_fused(at::Tensor& logits, const at::Tensor& targets, double scale,
                                            int64_t ignore_index, bool write_grad);
std::vector<at::Tensor> token_logprob_fwd(const at::Tensor& logits, const at::Tensor& targets, double temperature);
at::Tensor token_logprob_bwd(const at::Tensor& logits, const at::Tensor& targets, const at::Tensor& lse,
                             const at::Tensor& dlogp, double temperature);
// optim.cu
void adamw_step(at::Tensor& master, const at::Tensor& grad, at::Tensor& m, at::Tensor& v,
                const c10::optional<at::Tensor>& out, double lr, double beta1, double beta2, double eps,
                double weight_decay, int64_t step, double grad_scale, const c10::optional<at::Tensor>& grad_scale_t,
                const c10::optional<at::Tensor>& step_t, int64_t max_blocks);
void sgd_step(at::Tensor& param, const at::Tensor& grad, const c10::optional<at::Tensor>& out, double lr,
              double grad_scale, const c10::optional<at::Tensor>& nonfinite);
at::Tensor grad_sq_norm(const at::Tensor& g);
// gemm_tc.cu
void gemm(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, bool a_mn, bool b_mn, bool accumulate);
void grouped_gemm_m(const at::Tensor& a, const at::Tensor& b, const at::Tensor& group_off,
                    const at::Tensor& group_rows, at::Tensor& out, bool b_mn, int64_t max_rows);
void grouped_gemm_k(const at::Tensor& a, const at::Tensor& b, const at::Tensor& group_off,
                    const at::Tensor& group_rows, at::Tensor& out, bool accumulate);
// mhc.cu
at::Tensor mhc_sinkhorn_fwd(const at::Tensor& comb, int64_t iters, double eps);
at::Tensor mhc_sinkhorn_bwd(const at::Tensor& comb, const at::Tensor& grad, int64_t iters, double eps);
at::Tensor mhc_collapse_fwd(const at::Tensor& s, const at::Tensor& w);
std::vector<at::Tensor> mhc_collapse_bwd(const at::Tensor& g, const at::Tensor& s, const at::Tensor& w);
at::Tensor mhc_expand_fwd(const at::Tensor& v, const at::Tensor& r, const at::Tensor& post, const at::Tensor& comb);
std::vector<at::Tensor> mhc_expand_bwd(const at::Tensor& g, const at::Tensor& v, const at::Tensor& r,
                                       const at::Tensor& post, const at::Tensor& comb);
// ep_nvlink.cu
void ep_wait(const at::Tensor& flags, int64_t epoch, const c10::optional<at::Tensor>& epoch_base);
void ep_signal(const at::Tensor& peer_flags, const c10::optional<at::Tensor>& peer_counts,
               const c10::optional<at::Tensor>& counts, int64_t my_rank, int64_t epoch,
               const c10::optional<at::Tensor>& epoch_base);
void ep_push_rows(const at::Tensor& x, const at::Tensor& dest_mask, const at::Tensor& slot,
                  const at::Tensor& peer_recv, const c10::optional<at::Tensor>& peer_meta,
                  const c10::optional<at::Tensor>& ids, const c10::optional<at::Tensor>& weights, int64_t t_cap,
                  int64_t e_local, at::Tensor& done_counter, const at::Tensor& peer_flags,
                  const c10::optional<at::Tensor>& peer_counts, const c10::optional<at::Tensor>& counts,
                  int64_t my_rank, int64_t epoch, const c10::optional<at::Tensor>& epoch_base);
void ep_combine_push(const at::Tensor& y, const at::Tensor& route, const c10::optional<at::Tensor>& weights,
                     const at::Tensor& counts, const at::Tensor& peer_ret, const c10::optional<at::Tensor>& row_extra,
                     const c10::optional<at::Tensor>& peer_retw, int64_t t_cap, at::Tensor& done_counter,
                     const at::Tensor& peer_flags, int64_t my_rank, int64_t epoch,
                     const c10::optional<at::Tensor>& epoch_base);
at::Tensor ep_reduce_returned(const at::Tensor& ret, const at::Tensor& dest_mask, const at::Tensor& slot,
                              int64_t tokens);
// peer_optim.cu
void peer_update(const at::Tensor& peer_grad, const at::Tensor& peer_param, const at::Tensor& peer_flags,
                 const at::Tensor& my_flags, int64_t flag_row, int64_t my_rank, int64_t epoch, int64_t offset,
                 at::Tensor& master, const c10::optional<at::Tensor>& m, const c10::optional<at::Tensor>& v,
                 int64_t algo, double lr, double beta1, double beta2, double eps, double weight_decay, int64_t step,
                 double grad_scale, const c10::optional<at::Tensor>& grad_scale_t,
                 const c10::optional<at::Tensor>& nonfinite, int64_t max_blocks,
                 const c10::optional<at::Tensor>& step_t, const c10::optional<at::Tensor>& epoch_base);
// sparse_attention.cu
std::vector<at::Tensor> sparse_attention_fwd(const at::Tensor& q, const at::Tensor& kv, const at::Tensor& win_idx,
                                             const at::Tensor& win_mask, const c10::optional<at::Tensor>& comp,
                                             const c10::optional<at::Tensor>& comp_idx, const at::Tensor& sinks);
std::vector<at::Tensor> sparse_attention_bwd(const at::Tensor& q, const at::Tensor& kv, const at::Tensor& win_idx,
                                             const at::Tensor& win_mask, const c10::optional<at::Tensor>& comp,
                                             const c10::optional<at::Tensor>& comp_idx, const at::Tensor& sinks,
                                             const at::Tensor& out, const at::Tensor& lse, const at::Tensor& dout,
                                             c10::optional<int64_t> ordered_chunk);
// fake_quant.cu
at::Tensor cache_fake_quant(const at::Tensor& x, int64_t kind);
// index_scores.cu
at::Tensor index_scores(const at::Tensor& query, const at::Tensor& keys, const at::Tensor& weights,
                        const at::Tensor& starts, const at::Tensor& ends, int64_t width,
                        const c10::optional<at::Tensor>& candidates);
// attention.cu
std::vector<at::Tensor> attn_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                 const c10::optional<at::Tensor>& trace);
std::vector<at::Tensor> attn_bwd(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k,
                                 const at::Tensor& v, const at::Tensor& out, const at::Tensor& lse,
                                 const c10::optional<at::Tensor>& trace);
std::vector<at::Tensor> attn_fwd_cp(const at::Tensor& q, const std::vector<int64_t>& k_ptrs,
                                    const std::vector<int64_t>& v_ptrs, int64_t chunk, int64_t q_offset,
                                    int64_t kv_heads);
at::Tensor attn_bwd_cp(const at::Tensor& dout, const at::Tensor& q, const std::vector<int64_t>& k_ptrs,
                       const std::vector<int64_t>& v_ptrs, const at::Tensor& out, const at::Tensor& lse, int64_t chunk,
                       int64_t q_offset, int64_t kv_heads, at::Tensor& outbox);
void attn_cp_pull(const at::Tensor& src, at::Tensor& dst, int64_t chunk_bytes);
std::vector<at::Tensor> attn_cp_finalize(const at::Tensor& boxes, int64_t me, int64_t batch, int64_t chunk,
                                         int64_t kv_heads);
}  // namespace tdsv

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "tiny_dsv41_b200 sm_100a kernels";
  maybe_install_segv_handler();
  m.def("read_status", &tdsv::read_status, "read and clear the device pipeline status word");
  m.def("status_word", &tdsv::status_word, "the current device's status word as a 1-element int32 tensor view");
  m.def("set_peer_wait_limit_ns", &tdsv::set_peer_wait_limit_ns, "limit of waits on other ranks' flags (ns)");
  m.def("peer_wait_limit_ns", []() { return static_cast<int64_t>(tdsv::peer_wait_limit_ns()); });
  m.def("moe_route_plan", &tdsv::moe_route_plan, "expert-major routing plan (stable, 128-row segments)",
        py::arg("ids"), py::arg("num_experts"), py::arg("block") = 128, py::arg("slab_counts") = py::none(),
        py::arg("slab") = 1);
  m.def("ep_dest_plan", &tdsv::ep_dest_plan, "per-token destination ranks, receive slots and counts");
  m.def("attn_fwd", &tdsv::attn_fwd, "causal GQA flash attention forward (tcgen05): (out, lse)", py::arg("q"),
        py::arg("k"), py::arg("v"), py::arg("trace") = py::none());
  m.def("attn_bwd", &tdsv::attn_bwd, "causal GQA flash attention backward (tcgen05): (dq, dk, dv)", py::arg("dout"),
        py::arg("q"), py::arg("k"), py::arg("v"), py::arg("out"), py::arg("lse"), py::arg("trace") = py::none());
  m.def("attn_fwd_cp", &tdsv::attn_fwd_cp,
        "context-parallel causal attention forward: keys / values read from each owner's chunk (peer memory)");
  m.def("attn_bwd_cp", &tdsv::attn_bwd_cp,
        "context-parallel attention backward: dq, with per-owner dK / dV partials in the local outbox");
  m.def("attn_cp_pull", &tdsv::attn_cp_pull, "copy other ranks' K / V chunks into this rank's memory (peer loads)");
  m.def("attn_cp_finalize", &tdsv::attn_cp_finalize,
        "this rank's dk / dv: fixed-order sum of its slot in every rank's outbox (peer loads)");
  m.def("cache_fake_quant", &tdsv::cache_fake_quant, "FP8 / FP4 block fake quantization (0 fp8, 1 fp4_index, 2 fp4_kv)");
  m.def("index_scores", &tdsv::index_scores, "DSV4 sparse-indexer scores (tcgen05, fused relu / head reduction)");
  m.def("fp4_dequant", &tdsv::fp4_dequant, "MXFP4 (E2M1 + E8M0 per 32) to bf16");
  m.def("fp4_grouped_gemm", &tdsv::fp4_grouped_gemm, "expert-grouped GEMM against packed MXFP4 weights");
  m.def("rmsnorm_fwd", &tdsv::rmsnorm_fwd);
  m.def("rmsnorm_bwd", &tdsv::rmsnorm_bwd);
  m.def("column_sum", &tdsv::column_sum);
  m.def("qk_norm_rope_fwd", &tdsv::qk_norm_rope_fwd);
  m.def("qk_norm_rope_bwd", &tdsv::qk_norm_rope_bwd);
  m.def("rope_interleaved", &tdsv::rope_interleaved);
  m.def("router_fwd", &tdsv::router_fwd);
  m.def("router_bwd", &tdsv::router_bwd);
  m.def("moe_gather", &tdsv::moe_gather);
  m.def("moe_combine", &tdsv::moe_combine);
  m.def("moe_combine_bwd", &tdsv::moe_combine_bwd);
  m.def("moe_zero_padding", &tdsv::moe_zero_padding);
  m.def("swiglu_fwd", &tdsv::swiglu_fwd);
  m.def("swiglu_bwd", &tdsv::swiglu_bwd);
  m.def("cross_entropy_fused", &tdsv::cross_entropy_fused);
  m.def("token_logprob_fwd", &tdsv::token_logprob_fwd);
  m.def("token_logprob_bwd", &tdsv::token_logprob_bwd);
  m.def("adamw_step", &tdsv::adamw_step, py::arg("master"), py::arg("grad"), py::arg("m"), py::arg("v"),
        py::arg("out"), py::arg("lr"), py::arg("beta1"), py::arg("beta2"), py::arg("eps"), py::arg("weight_decay"),
        py::arg("step"), py::arg("grad_scale"), py::arg("grad_scale_t"), py::arg("step_t") = py::none(),
        py::arg("max_blocks") = 0);
  m.def("sgd_step", &tdsv::sgd_step);
  m.def("grad_sq_norm", &tdsv::grad_sq_norm);
  m.def("gemm", &tdsv::gemm);
  m.def("grouped_gemm_m", &tdsv::grouped_gemm_m);
  m.def("grouped_gemm_k", &tdsv::grouped_gemm_k);
  m.def("mhc_sinkhorn_fwd", &tdsv::mhc_sinkhorn_fwd);
  m.def("mhc_sinkhorn_bwd", &tdsv::mhc_sinkhorn_bwd);
  m.def("mhc_collapse_fwd", &tdsv::mhc_collapse_fwd);
  m.def("mhc_collapse_bwd", &tdsv::mhc_collapse_bwd);
  m.def("mhc_expand_fwd", &tdsv::mhc_expand_fwd);
  m.def("mhc_expand_bwd", &tdsv::mhc_expand_bwd);
  // the trailing epoch_base (device int32 scalar added to the epoch) is optional
  m.def("ep_wait", &tdsv::ep_wait, py::arg("flags"), py::arg("epoch"), py::arg("epoch_base") = py::none());
  m.def("ep_signal", &tdsv::ep_signal, py::arg("peer_flags"), py::arg("peer_counts"), py::arg("counts"),
        py::arg("my_rank"), py::arg("epoch"), py::arg("epoch_base") = py::none());
  m.def("ep_push_rows", &tdsv::ep_push_rows, py::arg("x"), py::arg("dest_mask"), py::arg("slot"), py::arg("peer_recv"),
        py::arg("peer_meta"), py::arg("ids"), py::arg("weights"), py::arg("t_cap"), py::arg("e_local"),
        py::arg("done_counter"), py::arg("peer_flags"), py::arg("peer_counts"), py::arg("counts"), py::arg("my_rank"),
        py::arg("epoch"), py::arg("epoch_base") = py::none());
  m.def("ep_combine_push", &tdsv::ep_combine_push, py::arg("y"), py::arg("route"), py::arg("weights"),
        py::arg("counts"), py::arg("peer_ret"), py::arg("row_extra"), py::arg("peer_retw"), py::arg("t_cap"),
        py::arg("done_counter"), py::arg("peer_flags"), py::arg("my_rank"), py::arg("epoch"),
        py::arg("epoch_base") = py::none());
  m.def("ep_reduce_returned", &tdsv::ep_reduce_returned);
  m.def("peer_update", &tdsv::peer_update, py::arg("peer_grad"), py::arg("peer_param"), py::arg("peer_flags"),
        py::arg("my_flags"), py::arg("flag_row"), py::arg("my_rank"), py::arg("epoch"), py::arg("offset"),
        py::arg("master"), py::arg("m"), py::arg("v"), py::arg("algo"), py::arg("lr"), py::arg("beta1"),
        py::arg("beta2"), py::arg("eps"), py::arg("weight_decay"), py::arg("step"), py::arg("grad_scale"),
        py::arg("grad_scale_t"), py::arg("nonfinite"), py::arg("max_blocks"), py::arg("step_t") = py::none(),
        py::arg("epoch_base") = py::none());
  m.def("sparse_attention_fwd", &tdsv::sparse_attention_fwd);
  m.def("sparse_attention_bwd", &tdsv::sparse_attention_bwd, py::arg("q"), py::arg("kv"), py::arg("win_idx"),
        py::arg("win_mask"), py::arg("comp"), py::arg("comp_idx"), py::arg("sinks"), py::arg("out"), py::arg("lse"),
        py::arg("dout"), py::arg("ordered_chunk") = py::none());
}
