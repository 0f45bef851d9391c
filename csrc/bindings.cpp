// Python bindings of the thundersync_b200 native kernels.
#include "common.h"

namespace ts {
std::vector<at::Tensor> rms_norm_fwd(const at::Tensor& x, const at::Tensor& w, double eps, bool unit);
std::vector<at::Tensor> rms_norm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w,
                                     const at::Tensor& rstd, bool unit, const c10::optional<at::Tensor>& dres,
                                     const c10::optional<at::Tensor>& dw_acc, double dw_scale);
std::vector<at::Tensor> qk_norm_rope_fwd(const at::Tensor& qkv, const c10::optional<at::Tensor>& qw,
                                         const c10::optional<at::Tensor>& kw, const at::Tensor& pos,
                                         const at::Tensor& inv_freq, int64_t hq, int64_t hkv, int64_t d, double eps,
                                         bool unit, const c10::optional<at::Tensor>& cos_tab,
                                         const c10::optional<at::Tensor>& sin_tab,
                                         const c10::optional<at::Tensor>& k_out,
                                         const c10::optional<at::Tensor>& v_out);
std::vector<c10::optional<at::Tensor>> qk_norm_rope_bwd(const at::Tensor& dq, const at::Tensor& dk,
                                                        const at::Tensor& dv, const at::Tensor& qkv,
                                                        const c10::optional<at::Tensor>& qw,
                                                        const c10::optional<at::Tensor>& kw, const at::Tensor& pos,
                                                        const at::Tensor& inv_freq, int64_t hq, int64_t hkv,
                                                        int64_t d, double eps, bool unit,
                                                        const c10::optional<at::Tensor>& cos_tab,
                                                        const c10::optional<at::Tensor>& sin_tab,
                                                        const c10::optional<at::Tensor>& dqw_acc,
                                                        const c10::optional<at::Tensor>& dkw_acc, double dw_scale);
at::Tensor swiglu_fwd(const at::Tensor& gu);
at::Tensor swiglu_bwd(const at::Tensor& da, const at::Tensor& gu);
void embedding_bwd_accumulate(at::Tensor& target, const at::Tensor& ids, const at::Tensor& dy, double scale);
void fold_stats(const c10::optional<at::Tensor>& g1, at::Tensor& g2, const at::Tensor& src, double r);
void axpby(at::Tensor& out, const at::Tensor& x, const c10::optional<at::Tensor>& y, double a, double b);
void scale(at::Tensor& x, double s);
void reduce_into(at::Tensor& out, const std::vector<at::Tensor>& parts);
std::vector<c10::optional<at::Tensor>> lse_gather(const at::Tensor& logits, const at::Tensor& tgt, bool with_entropy);
at::Tensor logprob_dlogits(const at::Tensor& logits, const at::Tensor& tgt, const at::Tensor& lse,
                           const at::Tensor& g_lp, const c10::optional<at::Tensor>& g_ent,
                           const c10::optional<at::Tensor>& ent, bool out_bf16);
at::Tensor sq_norm(const at::Tensor& x);
std::vector<at::Tensor> clip_coef(const at::Tensor& sq, double max_norm);
void adamw_flat(at::Tensor& master, at::Tensor& param, const at::Tensor& grad, at::Tensor& m, at::Tensor& v,
                double lr, double b1, double b2, double eps, double wd, int64_t step,
                const c10::optional<at::Tensor>& scale_t, double scale, bool maximize);
void symm_barrier(const std::vector<int64_t>& flag_ptrs, int64_t rank, int64_t slot, int64_t epoch,
                  at::Tensor& status, double timeout_s);
at::Tensor symm_reduce(const std::vector<int64_t>& buf_ptrs, int64_t rank, int64_t lo, int64_t hi, double scale,
                       bool write_all, const at::Tensor& like);
void symm_reduce_oneshot(const std::vector<int64_t>& buf_ptrs, int64_t n, double scale, at::Tensor& out);
void symm_norm_put(const at::Tensor& partial, const std::vector<int64_t>& flag_ptrs, int64_t rank,
                   int64_t norm_offset);
void symm_adamw_gather(at::Tensor& master, at::Tensor& m, at::Tensor& v, const at::Tensor& grad,
                       const std::vector<int64_t>& param_ptrs, int64_t lo, double lr, double b1, double b2,
                       double eps, double wd, int64_t step, bool maximize, const at::Tensor& norm_slots,
                       double max_norm, at::Tensor& norm_out);
std::vector<at::Tensor> tc_selftest(const at::Tensor& a, const at::Tensor& bk, const at::Tensor& bm);
std::vector<at::Tensor> attn_fwd_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, double scale,
                                    const c10::optional<at::Tensor>& out);
at::Tensor tc_status(const at::Tensor& like);
std::vector<at::Tensor> attn_bwd_tc(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k,
                                    const at::Tensor& v, const at::Tensor& o, const at::Tensor& lse, double scale,
                                    const c10::optional<at::Tensor>& dq_out, const c10::optional<at::Tensor>& dk_out,
                                    const c10::optional<at::Tensor>& dv_out);
std::vector<at::Tensor> attn_fwd_packed(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                        const at::Tensor& qtab, const at::Tensor& far, double scale,
                                        const c10::optional<at::Tensor>& out);
std::vector<at::Tensor> attn_bwd_packed(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k,
                                        const at::Tensor& v, const at::Tensor& o, const at::Tensor& lse,
                                        const at::Tensor& qtab, const at::Tensor& far, const at::Tensor& ktab,
                                        const at::Tensor& cons, double scale,
                                        const c10::optional<at::Tensor>& dq_out,
                                        const c10::optional<at::Tensor>& dk_out,
                                        const c10::optional<at::Tensor>& dv_out);
void register_ipc(pybind11::module& m);
uint64_t bounds_word_rowops(bool reset);
uint64_t bounds_word_fold(bool reset);
void register_pinned(pybind11::module& m);
void gemm_tc(at::Tensor& out, const at::Tensor& a, const at::Tensor& b, bool a_t, bool b_t, int64_t mode,
             double alpha, const c10::optional<at::Tensor>& residual);
std::vector<at::Tensor> gdn_chunk_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                      const at::Tensor& g, const at::Tensor& beta, const at::Tensor& state);
std::vector<at::Tensor> gdn_chunk_bwd(const at::Tensor& dout, const at::Tensor& dfinal, const at::Tensor& q,
                                      const at::Tensor& k, const at::Tensor& v, const at::Tensor& g,
                                      const at::Tensor& beta, const at::Tensor& starts, const at::Tensor& delta,
                                      const at::Tensor& tsv, const at::Tensor& psv, const at::Tensor& kd,
                                      const at::Tensor& kb);
int64_t gemm_tc_pair(int64_t on);
int64_t gemm_tc_epi8(int64_t mode);
int64_t gemm_tc_wide(int64_t mode);
int64_t gemm_tc_direct(int64_t on);
int64_t gemm_tc_pdl(int64_t on);
void gemm_tc_profile(int64_t on);
at::Tensor gemm_tc_profile_read();
std::vector<at::Tensor> dense_layer_fwd(const at::Tensor& h, const at::Tensor& pos, const at::Tensor& inv_freq,
                                        const at::Tensor& cos_tab, const at::Tensor& sin_tab, const at::Tensor& ln1,
                                        const at::Tensor& wqkv, const c10::optional<at::Tensor>& qn,
                                        const c10::optional<at::Tensor>& kn, const at::Tensor& wo,
                                        const at::Tensor& ln2, const at::Tensor& wgu, const at::Tensor& wd,
                                        const std::vector<at::Tensor>& past_k, const std::vector<at::Tensor>& past_v,
                                        int64_t hq, int64_t hkv, int64_t d, double eps, double scale, int64_t cov,
                                        const std::vector<at::Tensor>& tabs);
std::vector<at::Tensor> dense_layer_bwd(
    const at::Tensor& dout, const c10::optional<at::Tensor>& dk_out, const c10::optional<at::Tensor>& dv_out,
    const at::Tensor& h, const at::Tensor& pos, const at::Tensor& inv_freq, const at::Tensor& cos_tab,
    const at::Tensor& sin_tab, const at::Tensor& ln1, const at::Tensor& wqkv, const c10::optional<at::Tensor>& qn,
    const c10::optional<at::Tensor>& kn, const at::Tensor& wo, const at::Tensor& ln2, const at::Tensor& wgu,
    const at::Tensor& wd, const at::Tensor& k_own, const at::Tensor& v_own, const std::vector<at::Tensor>& past_k,
    const std::vector<at::Tensor>& past_v, const std::vector<at::Tensor>& saved,
    int64_t hq, int64_t hkv, int64_t d, double eps, double scale, int64_t cov, int64_t sp,
    const std::vector<c10::optional<at::Tensor>>& sinks, double sink_scale, int64_t side,
    const std::vector<at::Tensor>& tabs);
void gemm_tc_cat(at::Tensor& out, const at::Tensor& a, const at::Tensor& b, const c10::optional<at::Tensor>& a2,
                 const c10::optional<at::Tensor>& b2, bool a_t, bool b_t, int64_t mode, double alpha,
                 const c10::optional<at::Tensor>& residual);
std::vector<at::Tensor> lmhead_lse_tc(const at::Tensor& h, const at::Tensor& w, const at::Tensor& tgt,
                                      bool with_entropy);
at::Tensor lmhead_dlogits_tc(const at::Tensor& h, const at::Tensor& w, const at::Tensor& tgt, const at::Tensor& lse,
                             const at::Tensor& glp, const c10::optional<at::Tensor>& gent,
                             const c10::optional<at::Tensor>& ent);
std::vector<at::Tensor> conv1d_silu_fwd(const at::Tensor& x, const at::Tensor& w, const at::Tensor& tail);
std::vector<at::Tensor> conv1d_silu_bwd(const at::Tensor& dy, const at::Tensor& dtail_out, const at::Tensor& x,
                                        const at::Tensor& w, const at::Tensor& tail);
std::vector<at::Tensor> gdn_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& g,
                                const at::Tensor& beta, const at::Tensor& state);
std::vector<at::Tensor> gdn_bwd(const at::Tensor& dout, const at::Tensor& dfinal, const at::Tensor& q,
                                const at::Tensor& k, const at::Tensor& v, const at::Tensor& g, const at::Tensor& beta,
                                const at::Tensor& saved);
}  // namespace ts

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "thundersync_b200 native sm_100a kernels";
  ts::register_ipc(m);
  ts::register_pinned(m);
  m.def("rms_norm_fwd", &ts::rms_norm_fwd);
  m.def("rms_norm_bwd", &ts::rms_norm_bwd, pybind11::arg("dy"), pybind11::arg("x"), pybind11::arg("w"),
        pybind11::arg("rstd"), pybind11::arg("unit"), pybind11::arg("dres") = pybind11::none(),
        pybind11::arg("dw_acc") = pybind11::none(), pybind11::arg("dw_scale") = 1.0);
  m.def("qk_norm_rope_fwd", &ts::qk_norm_rope_fwd, pybind11::arg("qkv"), pybind11::arg("qw"), pybind11::arg("kw"),
        pybind11::arg("pos"), pybind11::arg("inv_freq"), pybind11::arg("hq"), pybind11::arg("hkv"), pybind11::arg("d"),
        pybind11::arg("eps"), pybind11::arg("unit"), pybind11::arg("cos_tab") = pybind11::none(),
        pybind11::arg("sin_tab") = pybind11::none(),
        pybind11::arg("k_out") = pybind11::none(), pybind11::arg("v_out") = pybind11::none());
  m.def("qk_norm_rope_bwd", &ts::qk_norm_rope_bwd, pybind11::arg("dq"), pybind11::arg("dk"), pybind11::arg("dv"),
        pybind11::arg("qkv"), pybind11::arg("qw"), pybind11::arg("kw"), pybind11::arg("pos"), pybind11::arg("inv_freq"),
        pybind11::arg("hq"), pybind11::arg("hkv"), pybind11::arg("d"), pybind11::arg("eps"), pybind11::arg("unit"),
        pybind11::arg("cos_tab") = pybind11::none(), pybind11::arg("sin_tab") = pybind11::none(),
        pybind11::arg("dqw_acc") = pybind11::none(), pybind11::arg("dkw_acc") = pybind11::none(),
        pybind11::arg("dw_scale") = 1.0);
  m.def("swiglu_fwd", &ts::swiglu_fwd);
  m.def("swiglu_bwd", &ts::swiglu_bwd);
  m.def("embedding_bwd_accumulate", &ts::embedding_bwd_accumulate);
  m.def("fold_stats", &ts::fold_stats);
  m.def("axpby", &ts::axpby);
  m.def("scale", &ts::scale);
  m.def("reduce_into", &ts::reduce_into);
  m.def("lse_gather", &ts::lse_gather);
  m.def("logprob_dlogits", &ts::logprob_dlogits);
  m.def("sq_norm", &ts::sq_norm);
  m.def("clip_coef", &ts::clip_coef);
  m.def("adamw_flat", &ts::adamw_flat);
  m.def("symm_barrier", &ts::symm_barrier);
  m.def("tc_selftest", &ts::tc_selftest);
  m.def("attn_fwd_tc", &ts::attn_fwd_tc, pybind11::arg("q"), pybind11::arg("k"), pybind11::arg("v"),
        pybind11::arg("scale"), pybind11::arg("out") = pybind11::none());
  m.def("tc_status", &ts::tc_status);
  m.def("attn_bwd_tc", &ts::attn_bwd_tc, pybind11::arg("dout"), pybind11::arg("q"), pybind11::arg("k"),
        pybind11::arg("v"), pybind11::arg("o"), pybind11::arg("lse"), pybind11::arg("scale"),
        pybind11::arg("dq") = pybind11::none(), pybind11::arg("dk") = pybind11::none(),
        pybind11::arg("dv") = pybind11::none());
  m.def("attn_fwd_packed", &ts::attn_fwd_packed, pybind11::arg("q"), pybind11::arg("k"), pybind11::arg("v"),
        pybind11::arg("qtab"), pybind11::arg("far"), pybind11::arg("scale"), pybind11::arg("out") = pybind11::none());
  m.def("attn_bwd_packed", &ts::attn_bwd_packed, pybind11::arg("dout"), pybind11::arg("q"), pybind11::arg("k"),
        pybind11::arg("v"), pybind11::arg("o"), pybind11::arg("lse"), pybind11::arg("qtab"), pybind11::arg("far"),
        pybind11::arg("ktab"), pybind11::arg("cons"), pybind11::arg("scale"), pybind11::arg("dq") = pybind11::none(),
        pybind11::arg("dk") = pybind11::none(), pybind11::arg("dv") = pybind11::none());
  m.def("symm_reduce", &ts::symm_reduce);
  m.def("symm_norm_put", &ts::symm_norm_put);
  m.def("symm_reduce_oneshot", &ts::symm_reduce_oneshot);
  m.def("symm_adamw_gather", &ts::symm_adamw_gather);
  m.def("conv1d_silu_fwd", &ts::conv1d_silu_fwd);
  m.def("conv1d_silu_bwd", &ts::conv1d_silu_bwd);
  m.def("gdn_fwd", &ts::gdn_fwd);
  m.def("gemm_tc", &ts::gemm_tc, pybind11::arg("out"), pybind11::arg("a"), pybind11::arg("b"), pybind11::arg("a_t"),
        pybind11::arg("b_t"), pybind11::arg("mode"), pybind11::arg("alpha"),
        pybind11::arg("residual") = pybind11::none());
  m.def("lmhead_lse_tc", &ts::lmhead_lse_tc);
  m.def("gemm_tc_pair", &ts::gemm_tc_pair);
  m.def("gemm_tc_epi8", &ts::gemm_tc_epi8);
  m.def("gemm_tc_wide", &ts::gemm_tc_wide);
  m.def("gemm_tc_direct", &ts::gemm_tc_direct);
  m.def("gemm_tc_pdl", &ts::gemm_tc_pdl);
  m.def("gemm_tc_profile", &ts::gemm_tc_profile);
  m.def("gemm_tc_profile_read", &ts::gemm_tc_profile_read);
  m.def("dense_layer_fwd", &ts::dense_layer_fwd);
  m.def("dense_layer_bwd", &ts::dense_layer_bwd);
  m.def(
      "bounds_status",
      [](bool reset) {
        // failed index checks per source file: {file: (site, index)}; empty when every check passed
        pybind11::dict out;
        const std::pair<const char*, uint64_t (*)(bool)> units[] = {{"rowops", &ts::bounds_word_rowops},
                                                                   {"fold", &ts::bounds_word_fold}};
        for (const auto& u : units) {
          const uint64_t w = u.second(reset);
          if (w != 0) {
            int64_t idx = (int64_t)(w & 0xFFFFFFFFFFFFull);
            if (idx & (int64_t(1) << 47)) idx -= int64_t(1) << 48;  // sign-extend a negative index
            out[u.first] = pybind11::make_tuple((int)(w >> 48), idx);
          }
        }
        return out;
      },
      pybind11::arg("reset") = true);
  m.def("bounds_checked_build", []() {
#ifdef TS_BOUNDS_CHECK
    return true;
#else
    return false;
#endif
  });
  m.def("gemm_tc_cat", &ts::gemm_tc_cat, pybind11::arg("out"), pybind11::arg("a"), pybind11::arg("b"),
        pybind11::arg("a2"), pybind11::arg("b2"), pybind11::arg("a_t"), pybind11::arg("b_t"), pybind11::arg("mode"),
        pybind11::arg("alpha"), pybind11::arg("residual") = pybind11::none());
  m.def("lmhead_dlogits_tc", &ts::lmhead_dlogits_tc);
  m.def("gdn_bwd", &ts::gdn_bwd);
  m.def("gdn_chunk_fwd", &ts::gdn_chunk_fwd);
  m.def("gdn_chunk_bwd", &ts::gdn_chunk_bwd);
}
