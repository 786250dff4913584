// Python bindings of the verl_omni_b200 sm_100a kernels (module verl_omni_b200._C).
#include <torch/extension.h>

#include <atomic>
#include <string>
#include <utility>
#include <vector>

namespace vo {
using DcheckReader = unsigned long long (*)(bool reset);
static std::vector<std::pair<std::string, DcheckReader>>& dcheck_table() {
  static std::vector<std::pair<std::string, DcheckReader>> t;
  return t;
}
void dcheck_register(const char* file, DcheckReader fn) { dcheck_table().emplace_back(file, fn); }

// {"enabled": built with VO_DEVICE_CHECKS, "sites": {source file: first failing line}} (cleared with reset)
py::dict device_check_status(bool reset) {
  py::dict out, sites;
#ifdef VO_DEVICE_CHECKS
  out["enabled"] = true;
#else
  out["enabled"] = false;
#endif
  for (auto& e : dcheck_table()) {
    const unsigned long long v = e.second(reset);
    if (v) sites[py::str(e.first)] = (int64_t)v;
  }
  out["sites"] = sites;
  return out;
}

static std::atomic<int64_t> g_launches{0};
void count_launch(int64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
int64_t launch_count() { return g_launches.load(); }
std::vector<torch::Tensor> sde_step_fwd(torch::Tensor x, torch::Tensor v, torch::Tensor sigma, torch::Tensor sigma_prev,
                                        c10::optional<torch::Tensor> prev, c10::optional<torch::Tensor> noise,
                                        double sigma_max, double eta, int64_t type, int64_t seed, int64_t offset,
                                        bool want_logp, bool norm, c10::optional<torch::Tensor> row_seeds);
torch::Tensor normal_fill(torch::Tensor row_seeds, int64_t n, int64_t offset);
torch::Tensor sde_step_bwd(torch::Tensor x, torch::Tensor prev, torch::Tensor mean, torch::Tensor sigma,
                           torch::Tensor sigma_prev, torch::Tensor g_logp, torch::Tensor g_mean, double sigma_max,
                           double eta, int64_t type);
std::vector<torch::Tensor> ppo_clip_fwd(torch::Tensor logp, torch::Tensor old, torch::Tensor adv,
                                        c10::optional<torch::Tensor> w, double clip);
torch::Tensor ppo_clip_bwd(torch::Tensor logp, torch::Tensor old, torch::Tensor adv, c10::optional<torch::Tensor> w,
                           double clip, torch::Tensor g_loss);
std::vector<torch::Tensor> adaln_ln_fwd(torch::Tensor x, c10::optional<torch::Tensor> mod, int64_t shift_off,
                                        int64_t scale_off, c10::optional<torch::Tensor> w,
                                        c10::optional<torch::Tensor> bias, int64_t S, double eps);
std::vector<torch::Tensor> adaln_ln_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor mean, torch::Tensor rstd,
                                        torch::Tensor mod, int64_t shift_off, int64_t scale_off, int64_t S);
std::vector<torch::Tensor> qk_rmsnorm_fwd(torch::Tensor qkv, torch::Tensor wq, torch::Tensor wk,
                                          c10::optional<torch::Tensor> q_, c10::optional<torch::Tensor> k_,
                                          c10::optional<torch::Tensor> v_, int64_t S_seg, int64_t seg_off,
                                          c10::optional<torch::Tensor> rope_cos, c10::optional<torch::Tensor> rope_sin,
                                          double eps, std::vector<int64_t> part_off);
std::vector<torch::Tensor> qk_rmsnorm_bwd(torch::Tensor qkv, torch::Tensor wq, torch::Tensor wk,
                                          c10::optional<torch::Tensor> dq_, c10::optional<torch::Tensor> dk_,
                                          c10::optional<torch::Tensor> dv_, torch::Tensor rq, torch::Tensor rk,
                                          int64_t S_seg, int64_t seg_off, c10::optional<torch::Tensor> rope_cos,
                                          c10::optional<torch::Tensor> rope_sin, std::vector<int64_t> part_off);
torch::Tensor sq_norm(torch::Tensor g);
void adamw_flat(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, c10::optional<torch::Tensor> p16,
                double lr, double b1, double b2, double eps, double wd, int64_t step, double max_norm,
                c10::optional<torch::Tensor> sq_norm_t, double grad_scale);
std::vector<torch::Tensor> gemm_fwd(torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> b, int64_t epi,
                                    c10::optional<torch::Tensor> gate, c10::optional<torch::Tensor> res, int64_t S,
                                    c10::optional<torch::Tensor> ext_a, c10::optional<torch::Tensor> ext_b);
torch::Tensor gemm_dgrad(torch::Tensor dy, torch::Tensor w, c10::optional<torch::Tensor> ext_a,
                         c10::optional<torch::Tensor> ext_b);
void gemm_wgrad(torch::Tensor dy, torch::Tensor x, torch::Tensor out, bool accumulate);
std::vector<torch::Tensor> gemm_fwd_pair(torch::Tensor x0, torch::Tensor w0, c10::optional<torch::Tensor> b0,
                                         c10::optional<torch::Tensor> gate0, c10::optional<torch::Tensor> res0,
                                         int64_t S0, torch::Tensor x1, torch::Tensor w1,
                                         c10::optional<torch::Tensor> b1, c10::optional<torch::Tensor> gate1,
                                         c10::optional<torch::Tensor> res1, int64_t S1, int64_t epi);
void gemm_scatter(torch::Tensor x0, torch::Tensor w0, c10::optional<torch::Tensor> b0, int64_t seg_rows0,
                  int64_t dst_seq0, int64_t row_off0, c10::optional<torch::Tensor> x1, c10::optional<torch::Tensor> w1,
                  c10::optional<torch::Tensor> b1, int64_t seg_rows1, int64_t dst_seq1, int64_t row_off1,
                  std::vector<int64_t> peers, int64_t part_cols, int64_t dst_cols, int64_t dst_ld, int64_t dst_rows);
torch::Tensor moe_gemm_fwd(torch::Tensor x, torch::Tensor w, torch::Tensor tile_expert);
void gemm_tp(c10::optional<torch::Tensor> a, c10::optional<torch::Tensor> b, int64_t M, int64_t N, int64_t K,
             int64_t lda, int64_t ldb, int64_t a_mn, int64_t b_mn, c10::optional<torch::Tensor> out,
             c10::optional<torch::Tensor> out_f32, c10::optional<torch::Tensor> bias, int64_t gather,
             std::vector<int64_t> gather_ptrs, int64_t gather_rows, std::vector<int64_t> red_ptrs,
             int64_t red_rows, int64_t red_slot);
torch::Tensor moe_gemm_dgrad(torch::Tensor dy, torch::Tensor w, torch::Tensor tile_expert);
void moe_gemm_wgrad(torch::Tensor dy, torch::Tensor x, torch::Tensor seg, torch::Tensor out, bool accumulate);
std::vector<torch::Tensor> gemm_dgrad_pair(torch::Tensor dy0, torch::Tensor w0, torch::Tensor dy1, torch::Tensor w1);
void gemm_wgrad_pair(torch::Tensor dy0, torch::Tensor x0, torch::Tensor out0, torch::Tensor dy1, torch::Tensor x1,
                     torch::Tensor out1, bool accumulate);
torch::Tensor gelu_tanh_bwd(torch::Tensor dy, torch::Tensor pre);
int64_t gemm_error(bool reset);
std::vector<torch::Tensor> fmha_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, bool causal, double scale,
                                    int64_t version, int64_t split, c10::optional<torch::Tensor> kv_len);
int64_t fmha_error(bool reset);
void peer_copy(torch::Tensor dst, int64_t src_ptr, int64_t nbytes);
torch::Tensor slot_sum(torch::Tensor slots, int64_t W, c10::optional<torch::Tensor> bias);
void peer_row_copy(torch::Tensor src, torch::Tensor src_idx, torch::Tensor dst_rank, torch::Tensor dst_row,
                   std::vector<int64_t> peers, int64_t dst_rows, c10::optional<torch::Tensor> err);
void vocab_lse_update(torch::Tensor logits, int64_t lo, torch::Tensor targets, double inv_t, torch::Tensor m,
                      torch::Tensor s, torch::Tensor t);
void vocab_lse_grad(torch::Tensor logits, int64_t lo, torch::Tensor targets, double inv_t, torch::Tensor lse,
                    torch::Tensor g);
std::vector<torch::Tensor> rms_norm_fwd(torch::Tensor x, torch::Tensor w, double eps);
torch::Tensor rms_norm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor rstd, torch::Tensor dw,
                           bool accumulate);
torch::Tensor swiglu_fwd(torch::Tensor gu);
torch::Tensor swiglu_bwd(torch::Tensor da, torch::Tensor gu);
std::vector<torch::Tensor> router_topk(torch::Tensor logits, int64_t K);
torch::Tensor head_rmsnorm_rope(torch::Tensor x, int64_t col0, int64_t H, torch::Tensor w, torch::Tensor cos_t,
                                torch::Tensor sin_t, double eps);
torch::Tensor head_rmsnorm_rope_bwd(torch::Tensor dy, torch::Tensor x, int64_t col0, int64_t H, torch::Tensor w,
                                    torch::Tensor cos_t, torch::Tensor sin_t, double eps, torch::Tensor dw);
torch::Tensor sq_dist_fwd(torch::Tensor a, torch::Tensor b);
std::vector<torch::Tensor> sq_dist_bwd(torch::Tensor a, torch::Tensor b, torch::Tensor g, bool want_gb);
int64_t decode_tc_error(bool reset);
torch::Tensor decode_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor lens,
                               double scale, int64_t splits, c10::optional<torch::Tensor> block_table);
void fmha_fwd_peer(torch::Tensor q, torch::Tensor k, torch::Tensor v, std::vector<int64_t> peer_o,
                   std::vector<int64_t> peer_o2, int64_t sl, int64_t si, int64_t htot, int64_t h0, double scale,
                   int64_t version);
std::vector<torch::Tensor> linear_bwd_prep(torch::Tensor dy, c10::optional<torch::Tensor> saved,
                                           c10::optional<torch::Tensor> gate, int64_t S, int64_t mode,
                                           c10::optional<torch::Tensor> db, bool db_accumulate);
torch::Tensor cfg_combine(torch::Tensor pos, torch::Tensor neg, double g, bool renorm);
void peer_push(int64_t src_ptr, torch::Tensor plan, std::vector<int64_t> dst_ptrs);
torch::Tensor group_norm_nhwc(torch::Tensor x, torch::Tensor gamma, torch::Tensor beta, int64_t groups, double eps,
                              bool silu);
int64_t symm_malloc(int64_t nbytes);
void symm_free(int64_t ptr);
torch::Tensor ipc_get_handle(int64_t ptr);
int64_t ipc_open(torch::Tensor handle);
void ipc_close(int64_t ptr);
torch::Tensor tensor_from_ptr(int64_t ptr, int64_t numel, int64_t dtype_code, int64_t device);
void peer_a2a(torch::Tensor jobs, std::vector<int64_t> src_numel, std::vector<int64_t> dst_ptrs, int64_t dst_cap);
torch::Tensor peer_grad_reduce(std::vector<int64_t> grad_ptrs, int64_t lo, int64_t n, double scale, torch::Tensor out);
void peer_adamw_bcast(std::vector<int64_t> flat_ptrs, int64_t lo, int64_t n, torch::Tensor p, torch::Tensor grad,
                      torch::Tensor m, torch::Tensor v, double lr, double b1, double b2, double eps, double wd,
                      int64_t step, double max_norm, torch::Tensor sq_norm);
torch::Tensor fmha_bwd_trace();
std::vector<torch::Tensor> fmha_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o,
                                    torch::Tensor lse, torch::Tensor dO, bool causal, double scale, int64_t version,
                                    c10::optional<torch::Tensor> o2, c10::optional<torch::Tensor> dO2, int64_t split,
                                    c10::optional<torch::Tensor> kv_len);
}  // namespace vo

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "verl_omni_b200 sm_100a kernels";
  m.def("launch_count", &vo::launch_count);
  m.def("device_check_status", &vo::device_check_status, py::arg("reset") = false,
        "first failing VO_DCHECK site per source file (builds with VO_DEVICE_CHECKS=1)");
  m.def("count_launches", &vo::count_launch, "adds n to the launch counter (replayed CUDA graphs of counted kernels)");
  m.def("sde_step_fwd", &vo::sde_step_fwd, py::arg("x"), py::arg("v"), py::arg("sigma"), py::arg("sigma_prev"),
        py::arg("prev"), py::arg("noise"), py::arg("sigma_max"), py::arg("eta"), py::arg("type"), py::arg("seed"),
        py::arg("offset"), py::arg("want_logp"), py::arg("norm"), py::arg("row_seeds") = py::none());
  m.def("normal_fill", &vo::normal_fill);
  m.def("sde_step_bwd", &vo::sde_step_bwd);
  m.def("ppo_clip_fwd", &vo::ppo_clip_fwd);
  m.def("ppo_clip_bwd", &vo::ppo_clip_bwd);
  m.def("sq_dist_fwd", &vo::sq_dist_fwd, "per-sample mean squared distance of two fp32 [B, ...] tensors");
  m.def("sq_dist_bwd", &vo::sq_dist_bwd, "backward of sq_dist_fwd");
  m.def("adaln_ln_fwd", &vo::adaln_ln_fwd);
  m.def("adaln_ln_bwd", &vo::adaln_ln_bwd);
  m.def("qk_rmsnorm_fwd", &vo::qk_rmsnorm_fwd);
  m.def("qk_rmsnorm_bwd", &vo::qk_rmsnorm_bwd);
  m.def("sq_norm", &vo::sq_norm);
  m.def("adamw_flat", &vo::adamw_flat);
  m.def("gemm_fwd", &vo::gemm_fwd, py::arg("x"), py::arg("w"), py::arg("b"), py::arg("epi"), py::arg("gate"),
        py::arg("res"), py::arg("S"), py::arg("ext_a") = py::none(), py::arg("ext_b") = py::none());
  m.def("gemm_dgrad", &vo::gemm_dgrad, py::arg("dy"), py::arg("w"), py::arg("ext_a") = py::none(),
        py::arg("ext_b") = py::none());
  m.def("gemm_wgrad", &vo::gemm_wgrad);
  m.def("gemm_fwd_pair", &vo::gemm_fwd_pair, "two linear forwards in one persistent GEMM launch");
  m.def("gemm_dgrad_pair", &vo::gemm_dgrad_pair);
  m.def("gemm_tp", &vo::gemm_tp, "GEMM with a tensor-parallel operand gather and / or peer reduce-scatter",
        py::arg("a"), py::arg("b"), py::arg("M"), py::arg("N"), py::arg("K"), py::arg("lda"), py::arg("ldb"),
        py::arg("a_mn"), py::arg("b_mn"), py::arg("out"), py::arg("out_f32"), py::arg("bias"), py::arg("gather"),
        py::arg("gather_ptrs"), py::arg("gather_rows"), py::arg("red_ptrs"), py::arg("red_rows"),
        py::arg("red_slot") = -1);
  m.def("moe_gemm_fwd", &vo::moe_gemm_fwd, "expert-grouped GEMM over expert-sorted, 128-padded rows");
  m.def("moe_gemm_dgrad", &vo::moe_gemm_dgrad);
  m.def("moe_gemm_wgrad", &vo::moe_gemm_wgrad);
  m.def("gemm_scatter", &vo::gemm_scatter, "QKV projection with the Ulysses head scatter in the epilogue");
  m.def("gemm_wgrad_pair", &vo::gemm_wgrad_pair);
  m.def("gelu_tanh_bwd", &vo::gelu_tanh_bwd);
  m.def("gemm_error", &vo::gemm_error);
  m.def("fmha_fwd", &vo::fmha_fwd, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("causal"), py::arg("scale"),
        py::arg("version") = 2, py::arg("split") = 0, py::arg("kv_len") = py::none());
  m.def("fmha_error", &vo::fmha_error);
  m.def("peer_copy", &vo::peer_copy, "copy-engine read of a peer buffer into a local tensor");
  m.def("slot_sum", &vo::slot_sum, "sum of W bf16 partial-sum slots (+ bias), fp32 accumulation",
        py::arg("slots"), py::arg("W"), py::arg("bias") = py::none());
  m.def("peer_row_copy", &vo::peer_row_copy, "row copies into peer GPUs' buffers (expert-parallel exchange)",
        py::arg("src"), py::arg("src_idx"), py::arg("dst_rank"), py::arg("dst_row"), py::arg("peers"),
        py::arg("dst_rows"), py::arg("err") = py::none());
  m.def("vocab_lse_update", &vo::vocab_lse_update, "online log-sum-exp + target logit over one vocabulary chunk");
  m.def("vocab_lse_grad", &vo::vocab_lse_grad, "in-place d(log p(target)) / d(logits) over one vocabulary chunk");
  m.def("rms_norm_fwd", &vo::rms_norm_fwd, "row RMSNorm (bf16), returns (y, rstd)");
  m.def("rms_norm_bwd", &vo::rms_norm_bwd, "row RMSNorm backward: dx, weight grad into fp32 dw");
  m.def("swiglu_fwd", &vo::swiglu_fwd, "silu(gate) * up over [M, 2F] (gate | up)");
  m.def("swiglu_bwd", &vo::swiglu_bwd, "SwiGLU backward -> d(gate | up)");
  m.def("router_topk", &vo::router_topk, "softmax router + top-k with renormalised gates");
  m.def("head_rmsnorm_rope", &vo::head_rmsnorm_rope, "per-head RMSNorm + rotate-half RoPE, [B,S,H*Dh] -> [B,H,S,Dh]");
  m.def("head_rmsnorm_rope_bwd", &vo::head_rmsnorm_rope_bwd, "backward of head_rmsnorm_rope");
  m.def("decode_tc_error", &vo::decode_tc_error, "first error code of a bounded wait in the tcgen05 decode kernel");
  m.def("decode_attention", &vo::decode_attention,
        "grouped-query decode attention over a contiguous or paged (block table) KV cache", py::arg("q"),
        py::arg("k_cache"), py::arg("v_cache"), py::arg("lens"), py::arg("scale"), py::arg("splits"),
        py::arg("block_table") = py::none());
  m.def("fmha_fwd_peer", &vo::fmha_fwd_peer, "Ulysses attention writing each output row to its owner rank",
        py::arg("q"), py::arg("k"), py::arg("v"), py::arg("peer_o"), py::arg("peer_o2"), py::arg("sl"), py::arg("si"),
        py::arg("htot"), py::arg("h0"), py::arg("scale"), py::arg("version") = 3);
  m.def("fmha_bwd_trace", &vo::fmha_bwd_trace, "event stamps of the last traced FMHA backward (version 6)");
  m.def("fmha_bwd", &vo::fmha_bwd, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"), py::arg("lse"),
        py::arg("dO"), py::arg("causal"), py::arg("scale"), py::arg("version") = 1, py::arg("o2") = py::none(),
        py::arg("dO2") = py::none(), py::arg("split") = 0, py::arg("kv_len") = py::none());
  m.def("linear_bwd_prep", &vo::linear_bwd_prep);
  m.def("cfg_combine", &vo::cfg_combine);
  m.def("peer_push", &vo::peer_push);
  m.def("group_norm_nhwc", &vo::group_norm_nhwc);
  m.def("symm_malloc", &vo::symm_malloc);
  m.def("symm_free", &vo::symm_free);
  m.def("ipc_get_handle", &vo::ipc_get_handle);
  m.def("ipc_open", &vo::ipc_open);
  m.def("ipc_close", &vo::ipc_close);
  m.def("tensor_from_ptr", &vo::tensor_from_ptr);
  m.def("peer_grad_reduce", &vo::peer_grad_reduce);
  m.def("peer_a2a", &vo::peer_a2a, "all-to-all with layout change over peer memory (Ulysses exchanges)");
  m.def("peer_adamw_bcast", &vo::peer_adamw_bcast);
}
