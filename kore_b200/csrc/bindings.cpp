// Python bindings of the kore_b200 native extension (_C).
#include <torch/extension.h>

namespace kore {
void gemm_bf16(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, bool a_mn, bool b_mn,
               double alpha, bool accumulate, const c10::optional<at::Tensor>& residual,
               int64_t max_ctas);
void rmsnorm_fwd(const at::Tensor& x, const at::Tensor& w, at::Tensor& y,
                 const c10::optional<at::Tensor>& rstd, double eps);
void rmsnorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w,
                 const at::Tensor& rstd, const c10::optional<at::Tensor>& dres, at::Tensor& dx,
                 const c10::optional<at::Tensor>& dw);
void qk_norm_rope_fwd(const at::Tensor& qkv, const at::Tensor& qw, const at::Tensor& kw,
                      const at::Tensor& pos, const at::Tensor& cos_t, const at::Tensor& sin_t,
                      at::Tensor& out, const c10::optional<at::Tensor>& rstd, int64_t Hq,
                      int64_t Hkv, double eps);
void qk_norm_rope_bwd(const at::Tensor& dout, const at::Tensor& qkv, const at::Tensor& qw,
                      const at::Tensor& kw, const at::Tensor& pos, const at::Tensor& cos_t,
                      const at::Tensor& sin_t, at::Tensor& dqkv, at::Tensor& dqw, at::Tensor& dkw,
                      int64_t Hq, int64_t Hkv, double eps);
void swiglu_fwd(const at::Tensor& gu, at::Tensor& out);
void swiglu_bwd(const at::Tensor& dout, const at::Tensor& gu, at::Tensor& dgu);
void embed_fwd(const at::Tensor& ids, const at::Tensor& table, at::Tensor& out);
void embed_bwd(const at::Tensor& ids, const at::Tensor& dy, at::Tensor& dtable);
void logprob_fwd_bwd(at::Tensor& logits, const c10::optional<at::Tensor>& targets,
                     double inv_temp, const c10::optional<at::Tensor>& logp,
                     const c10::optional<at::Tensor>& entropy, const c10::optional<at::Tensor>& lse,
                     const c10::optional<at::Tensor>& coef, bool write_grad);
void sumsq_accumulate(const at::Tensor& g, at::Tensor& out);
void adamw_step(at::Tensor& p, const c10::optional<at::Tensor>& master, const at::Tensor& g,
                at::Tensor& m, at::Tensor& v, double lr, double b1, double b2, double eps,
                double wd, int64_t step, double grad_scale, const c10::optional<at::Tensor>& sumsq,
                double max_norm, int64_t seed);
void attn_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
              const at::Tensor& cu_seqlens, int64_t max_seqlen, double scale, at::Tensor& o,
              at::Tensor& lse);
void attn_bwd(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k,
              const at::Tensor& v, const at::Tensor& o, const at::Tensor& lse,
              const at::Tensor& cu_seqlens, int64_t max_seqlen, double scale, at::Tensor& dq,
              at::Tensor& dk, at::Tensor& dv, at::Tensor& dq_acc, at::Tensor& delta);
void kv_append(const at::Tensor& k, const at::Tensor& v, const at::Tensor& slots, at::Tensor& kc,
               at::Tensor& vc);
void paged_attention(const at::Tensor& q, const at::Tensor& kc, const at::Tensor& vc,
                     const at::Tensor& block_table, const at::Tensor& seq_lens,
                     const at::Tensor& q_start, int64_t max_q, int64_t page_size, double scale,
                     int64_t nsplit, at::Tensor& out, const c10::optional<at::Tensor>& part_o,
                     const c10::optional<at::Tensor>& part_ml);
void sample_tokens(const at::Tensor& logits, double temperature, double top_p, int64_t seed,
                   int64_t step, at::Tensor& tokens, at::Tensor& logprobs,
                   const c10::optional<at::Tensor>& step_dev);
int64_t gemm_set_pair_mode(int64_t mode);
void gemm_grouped_dev(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, const at::Tensor& tiles,
                      const at::Tensor& ntiles, bool b_mn, bool accumulate);
void gemm_grouped_wgrad(const at::Tensor& dy, const at::Tensor& x, at::Tensor& out, const at::Tensor& offsets,
                        bool accumulate);
void moe_plan(const at::Tensor& idx, int64_t lo, int64_t hi, at::Tensor& pos, at::Tensor& src_row,
              at::Tensor& offsets, at::Tensor& tiles, at::Tensor& ntiles, at::Tensor& counts);
void moe_gather_rows(const at::Tensor& x, const at::Tensor& src_row, at::Tensor& out);
void moe_ep_plan(const at::Tensor& idx, const at::Tensor& allc, int64_t W, int64_t rank, int64_t cap,
                 at::Tensor& dst_rank, at::Tensor& dst_row, at::Tensor& loc_offsets, at::Tensor& loc_totals,
                 at::Tensor& tiles, at::Tensor& ntiles, at::Tensor& overflow);
void moe_zero_pad_rows(at::Tensor& buf, const at::Tensor& offsets, const at::Tensor& totals, int64_t H);
int64_t symm_heap_create(int64_t bytes, int64_t rank, int64_t world);
at::Tensor symm_heap_handle(int64_t id);
void symm_heap_open(int64_t id, const at::Tensor& handles);
at::Tensor symm_heap_tensor(int64_t id, int64_t offset, const std::vector<int64_t>& shape,
                            at::ScalarType dtype);
void symm_barrier(int64_t id, int64_t sig_offset, int64_t epoch);
void symm_rs_sumsq(int64_t id, int64_t grad_offset, int64_t n, const c10::optional<at::Tensor>& out,
                   at::Tensor& sumsq, double scale);
void symm_scalar_allreduce(int64_t id, int64_t sig_offset, int64_t epoch, const at::Tensor& local,
                           at::Tensor& out);
void symm_adamw_bcast(int64_t id, int64_t param_offset, int64_t grad_offset, int64_t n, double gscale,
                      const c10::optional<at::Tensor>& master, at::Tensor& m, at::Tensor& v, double lr,
                      double b1, double b2, double eps, double wd, int64_t step,
                      const c10::optional<at::Tensor>& sumsq, double max_norm, int64_t seed);
void gemm_grouped_bf16(const at::Tensor& a, const at::Tensor& b, at::Tensor& out,
                       const std::vector<int64_t>& offsets, bool b_mn, bool accumulate);
void moe_route_fwd(const at::Tensor& logits, int64_t k, bool norm, at::Tensor& probs, at::Tensor& idx,
                   at::Tensor& w);
void moe_route_bwd(const at::Tensor& probs, const at::Tensor& idx, const at::Tensor& w, const at::Tensor& dw,
                   bool norm, at::Tensor& dlogits);
void moe_combine(const at::Tensor& src, const at::Tensor& pos, const c10::optional<at::Tensor>& w,
                 const c10::optional<at::Tensor>& resid, at::Tensor& out);
void moe_combine_bwd(const at::Tensor& dy, const at::Tensor& src, const at::Tensor& pos, const at::Tensor& w,
                     at::Tensor& dsrc, at::Tensor& dw);
void symm_ep_scatter(int64_t id, int64_t buf_offset, const at::Tensor& x, const at::Tensor& src_row,
                     const at::Tensor& dst_rank, const at::Tensor& dst_row,
                     const c10::optional<at::Tensor>& scale, int64_t cap);
void symm_ep_gather(int64_t id, int64_t buf_offset, const at::Tensor& rank, const at::Tensor& row,
                    const c10::optional<at::Tensor>& w, const c10::optional<at::Tensor>& resid,
                    at::Tensor& y, const c10::optional<at::Tensor>& g, const c10::optional<at::Tensor>& dw,
                    int64_t H);
void gemm_tp_bf16(const c10::optional<at::Tensor>& a_local, const std::vector<int64_t>& a_peers, int64_t lda,
                  int64_t M, const at::Tensor& b, const c10::optional<at::Tensor>& out,
                  const std::vector<int64_t>& rs_peers, int64_t ldc, int64_t rows, int64_t rank,
                  const c10::optional<at::Tensor>& stage, const c10::optional<at::Tensor>& flags, int64_t epoch);
void tp_reduce_norm(const at::Tensor& slots, int64_t W, int64_t R, at::Tensor& x, const c10::optional<at::Tensor>& g,
                    const c10::optional<at::Tensor>& hn, double eps);
std::vector<int64_t> symm_peer_addrs(int64_t id, int64_t offset);
void symm_ep_index_push(int64_t id, int64_t index_offset, const at::Tensor& dst_rank, const at::Tensor& dst_row,
                        int64_t k, int64_t cap);
void moe_index_pads(at::Tensor& index, const at::Tensor& offsets, const at::Tensor& totals);
void gemm_grouped_dev_pull(at::Tensor& stage, const at::Tensor& b, at::Tensor& out, const at::Tensor& tiles,
                           const at::Tensor& ntiles, const std::vector<int64_t>& tok_peers, int64_t lda,
                           const at::Tensor& index, const at::Tensor& rows_dev, at::Tensor& flags, int64_t epoch,
                           bool b_mn);
void symm_gather_ce(int64_t id, int64_t src_offset, int64_t bytes, at::Tensor& dst);
void nvls_sumsq(int64_t mc_grad, int64_t n, double gscale, at::Tensor& out);
void nvls_adamw(int64_t mc_grad, int64_t mc_param, const at::Tensor& own_param,
                const c10::optional<at::Tensor>& master, at::Tensor& m, at::Tensor& v, int64_t elem0, double gscale,
                double lr, double b1, double b2, double eps, double wd, int64_t step,
                const c10::optional<at::Tensor>& sumsq, double max_norm, int64_t seed);
int64_t device_wait_flag(const at::Tensor& flag, int64_t want, double timeout_s);
int read_and_clear_device_error();
}  // namespace kore

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "kore_b200 sm_100a kernels";
  m.def("gemm_bf16", &kore::gemm_bf16, "tcgen05 bf16 GEMM");
  m.def("gemm_set_pair_mode", &kore::gemm_set_pair_mode,
        "large plain GEMMs on 2-CTA pairs (1) or one CTA per tile (0); returns the previous mode");
  m.def("rmsnorm_fwd", &kore::rmsnorm_fwd);
  m.def("rmsnorm_bwd", &kore::rmsnorm_bwd);
  m.def("qk_norm_rope_fwd", &kore::qk_norm_rope_fwd);
  m.def("qk_norm_rope_bwd", &kore::qk_norm_rope_bwd);
  m.def("swiglu_fwd", &kore::swiglu_fwd);
  m.def("swiglu_bwd", &kore::swiglu_bwd);
  m.def("embed_fwd", &kore::embed_fwd);
  m.def("embed_bwd", &kore::embed_bwd);
  m.def("logprob_fwd_bwd", &kore::logprob_fwd_bwd);
  m.def("sumsq_accumulate", &kore::sumsq_accumulate);
  m.def("adamw_step", &kore::adamw_step);
  m.def("attn_fwd", &kore::attn_fwd, "tcgen05 causal GQA flash attention forward");
  m.def("attn_bwd", &kore::attn_bwd, "tcgen05 causal GQA flash attention backward");
  m.def("kv_append", &kore::kv_append);
  m.def("paged_attention", &kore::paged_attention);
  m.def("sample_tokens", &kore::sample_tokens, "temperature / top-p sampler",
        py::arg("logits"), py::arg("temperature"), py::arg("top_p"), py::arg("seed"), py::arg("step"),
        py::arg("tokens"), py::arg("logprobs"), py::arg("step_dev") = py::none());
  m.def("symm_heap_create", &kore::symm_heap_create);
  m.def("symm_heap_handle", &kore::symm_heap_handle);
  m.def("symm_heap_open", &kore::symm_heap_open);
  m.def("symm_heap_tensor", &kore::symm_heap_tensor);
  m.def("symm_barrier", &kore::symm_barrier);
  m.def("device_wait_flag", &kore::device_wait_flag, "bounded wait on a device flag; 0 seen, 2 timed out");
  m.def("symm_rs_sumsq", &kore::symm_rs_sumsq);
  m.def("symm_scalar_allreduce", &kore::symm_scalar_allreduce);
  m.def("symm_adamw_bcast", &kore::symm_adamw_bcast);
  m.def("gemm_grouped_bf16", &kore::gemm_grouped_bf16, "grouped (MoE) tcgen05 GEMM");
  m.def("moe_route_fwd", &kore::moe_route_fwd);
  m.def("moe_plan", &kore::moe_plan, "device routing plan: counts, padded offsets, positions, tiles");
  m.def("moe_gather_rows", &kore::moe_gather_rows);
  m.def("moe_ep_plan", &kore::moe_ep_plan, "expert-parallel plan from gathered counts (device)");
  m.def("moe_zero_pad_rows", &kore::moe_zero_pad_rows);
  m.def("gemm_grouped_dev", &kore::gemm_grouped_dev, "grouped GEMM over a device tile table");
  m.def("gemm_grouped_dev_pull", &kore::gemm_grouped_dev_pull,
        "grouped GEMM with the expert-parallel pull dispatch staged in its prologue");
  m.def("symm_ep_index_push", &kore::symm_ep_index_push, "pull-dispatch index entries into the owners' heaps");
  m.def("moe_index_pads", &kore::moe_index_pads, "pad entries of the pull-dispatch index");
  m.def("gemm_grouped_wgrad", &kore::gemm_grouped_wgrad, "per-expert weight gradient, device offsets");
  m.def("moe_route_bwd", &kore::moe_route_bwd);
  m.def("moe_combine", &kore::moe_combine);
  m.def("moe_combine_bwd", &kore::moe_combine_bwd);
  m.def("symm_ep_scatter", &kore::symm_ep_scatter, "P2P scatter of rows into owners' buffers",
        py::arg("id"), py::arg("buf_offset"), py::arg("x"), py::arg("src_row"), py::arg("dst_rank"),
        py::arg("dst_row"), py::arg("scale") = py::none(), py::arg("cap") = 0);
  m.def("symm_ep_gather", &kore::symm_ep_gather);
  m.def("gemm_tp_bf16", &kore::gemm_tp_bf16, "tensor-parallel AG->GEMM / GEMM->RS over peer memory",
        py::arg("a_local"), py::arg("a_peers"), py::arg("lda"), py::arg("M"), py::arg("b"), py::arg("out"),
        py::arg("rs_peers"), py::arg("ldc"), py::arg("rows"), py::arg("rank"), py::arg("stage") = py::none(),
        py::arg("flags") = py::none(), py::arg("epoch") = 0);
  m.def("tp_reduce_norm", &kore::tp_reduce_norm);
  m.def("symm_peer_addrs", &kore::symm_peer_addrs);
  m.def("symm_gather_ce", &kore::symm_gather_ce, "all-gather of heap shards on the copy engines");
  m.def("nvls_sumsq", &kore::nvls_sumsq, "sum of squares of the switch-reduced gradient shard (multimem)");
  m.def("nvls_adamw", &kore::nvls_adamw, "AdamW on the switch-reduced gradient shard, multicast parameter store");
  m.def("read_and_clear_device_error", &kore::read_and_clear_device_error);
}
