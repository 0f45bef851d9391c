// One Qwen3 decoder layer (forward and backward) issued from C++ (C16, the per-layer executor op).
//
// The same kernels and GEMMs, in the same order and with the same operands,
// as the Python single-segment path of engine/dense_layer.py; what moves to
// C++ is the host work between launches (Python op dispatch, view
// bookkeeping, gradient-sink routing). For packs up to ~2k tokens that host
// work, not the GPU, set the step's pace: about 24 ms per pack of 28 layers.
// Every projection product is this package's tcgen05 GEMM (gemm_tc.cu): the
// residual adds ride its epilogue and the weight gradients are TMA
// reduce-adds into the fp32 gradient sink.
//
// Layer: h1 = h + o_proj(attn(rope(norm(qkv(rmsnorm1(h)))))),
//        out = h1 + down(swiglu(gate_up(rmsnorm2(h1)))).
// Attention reads the ancestors' keys/values and the pack's own from one
// buffer [S_past + t, hkv, d] built for the call (forward and again in the
// backward) from the ancestor chunks and the pack's own rows, which stay
// tensors of their own: descendants keep only those, never a copy of the
// ancestors. Single segment: attention reads the first S_past + cov rows;
// rows [cov, t) are pack padding. A pack of several segments passes its
// packed-attention work tables (`tabs`): the ancestor part then holds each
// unique ancestor chunk once and attention is one packed launch over all
// segments.
#include "common.h"

#include <ATen/cuda/CUDAEvent.h>
#include <c10/cuda/CUDACachingAllocator.h>

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
std::vector<at::Tensor> attn_fwd_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, double scale,
                                    const c10::optional<at::Tensor>& out);
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

void gemm_tc(at::Tensor& out, const at::Tensor& a, const at::Tensor& b, bool a_t, bool b_t, int64_t mode,
             double alpha, const c10::optional<at::Tensor>& residual);

namespace {

// [chunks... | own] along rows, one copy kernel
at::Tensor join_rows(const std::vector<at::Tensor>& chunks, const at::Tensor& own) {
  std::vector<at::Tensor> all(chunks.begin(), chunks.end());
  all.push_back(own);
  return at::cat(all, 0);
}

// x [M, K] · Wᵀ (W [N, K]) [+ residual], bf16
at::Tensor lin(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& residual = c10::nullopt) {
  auto out = at::empty({x.size(0), w.size(0)}, x.options());
  gemm_tc(out, x, w, false, true, 0, 1.0, residual);
  return out;
}

// dy [M, N] · W (W [N, K]), bf16
at::Tensor mm_w(const at::Tensor& dy, const at::Tensor& w) {
  auto out = at::empty({dy.size(0), w.size(1)}, dy.options());
  gemm_tc(out, dy, w, false, false, 0, 1.0, c10::nullopt);
  return out;
}

// dyᵀ x (dy [T, N], x [T, K]) -> [N, K] bf16
at::Tensor mm_tn(const at::Tensor& dy, const at::Tensor& x) {
  auto out = at::empty({dy.size(1), x.size(1)}, dy.options());
  gemm_tc(out, dy, x, true, false, 0, 1.0, c10::nullopt);
  return out;
}

// target += scale · dyᵀ x (fp32 accumulation into a gradient-sink view); with a side stream the GEMM runs
// there after the producing work of the current stream, and the operands' memory is kept until it ends
void deposit(at::Tensor target, const at::Tensor& dy, const at::Tensor& x, double scale, int64_t side) {
  if (side == 0) {
    gemm_tc(target, dy, x, true, false, 2, scale, c10::nullopt);
    return;
  }
  auto main = at::cuda::getCurrentCUDAStream();
  auto st = at::cuda::getStreamFromExternal(reinterpret_cast<cudaStream_t>(side), dy.get_device());
  // one reusable event per device (re-recording moves it to the current point of the main stream)
  static at::cuda::CUDAEvent events[64];
  at::cuda::CUDAEvent& ev = events[dy.get_device() & 63];
  ev.record(main);
  ev.block(st);
  {
    c10::cuda::CUDAStreamGuard guard(st);
    gemm_tc(target, dy, x, true, false, 2, scale, c10::nullopt);
  }
  c10::cuda::CUDACachingAllocator::recordStream(dy.storage().data_ptr(), st);
  c10::cuda::CUDACachingAllocator::recordStream(x.storage().data_ptr(), st);
}

}  // namespace

// Returns {out, k, v, x1, rstd1, qkv, q, o, lse, h1, x2, rstd2, gu, a}; k / v are the pack's own rows.
std::vector<at::Tensor> dense_layer_fwd(const at::Tensor& h, const at::Tensor& pos, const at::Tensor& inv_freq,
                                        const at::Tensor& cos_tab, const at::Tensor& sin_tab, const at::Tensor& ln1,
                                        const at::Tensor& wqkv, const c10::optional<at::Tensor>& qn,
                                        const c10::optional<at::Tensor>& kn, const at::Tensor& wo,
                                        const at::Tensor& ln2, const at::Tensor& wgu, const at::Tensor& wd,
                                        const std::vector<at::Tensor>& past_k, const std::vector<at::Tensor>& past_v,
                                        int64_t hq, int64_t hkv, int64_t d, double eps, double scale, int64_t cov,
                                        const std::vector<at::Tensor>& tabs) {
  check_cuda(h, "h");
  const int64_t t = h.size(0);
  TS_CHECK(cov > 0 && cov <= t && past_k.size() == past_v.size(), "dense_layer_fwd: rows / ancestor chunks");
  const c10::cuda::CUDAGuard guard(h.device());
  auto r1 = rms_norm_fwd(h, ln1, eps, false);
  const at::Tensor& x1 = r1[0];
  auto qkv = lin(x1, wqkv);
  int64_t sp = 0;
  for (const auto& x : past_k) sp += x.size(0);
  auto rr = qk_norm_rope_fwd(qkv, qn, kn, pos, inv_freq, hq, hkv, d, eps, false, cos_tab, sin_tab, c10::nullopt,
                             c10::nullopt);
  const at::Tensor &q = rr[0], &k_own = rr[1], &v_own = rr[2];
  at::Tensor kbuf = k_own, vbuf = v_own;
  if (sp > 0) kbuf = join_rows(past_k, k_own), vbuf = join_rows(past_v, v_own);
  auto o = at::empty({t, hq, d}, h.options());
  std::vector<at::Tensor> att;
  if (tabs.empty()) {
    att = attn_fwd_tc(q.narrow(0, 0, cov), kbuf.narrow(0, 0, sp + cov), vbuf.narrow(0, 0, sp + cov), scale,
                      o.narrow(0, 0, cov));
  } else {
    // several segments: one packed launch over [unique ancestor chunks | own rows]
    att = attn_fwd_packed(q, kbuf, vbuf, tabs[0], tabs[1], scale, o);
  }
  if (cov < t) o.narrow(0, cov, t - cov).zero_();  // pack padding rows: no attention output
  auto h1 = lin(o.view({t, hq * d}), wo, h);
  auto r2 = rms_norm_fwd(h1, ln2, eps, false);
  auto gu = lin(r2[0], wgu);
  auto a = swiglu_fwd(gu);
  auto out = lin(a, wd, h1);
  return {out, k_own, v_own, x1, r1[1], qkv, q, o, att[1], h1, r2[0], r2[1], gu, a};
}

// Sink targets (fp32 views: ln1, qkv span, q-norm, k-norm, o, ln2, gate/up span, down) receive the weight
// gradients when given (scaled by sink_scale); otherwise the gradients come back. side: a CUDA stream
// handle for the projection weight-gradient GEMMs, or 0. saved = {x1, rstd1, qkv, q, o, lse, h1, x2, rstd2,
// gu, a} of dense_layer_fwd. Returns {dh, dkbuf_past, dvbuf_past, g_ln1, g_qkv, g_qn, g_kn, g_o, g_ln2,
// g_gu, g_d} (a gradient is an undefined tensor when it went into the sink).
std::vector<at::Tensor> dense_layer_bwd(
    const at::Tensor& dout, const c10::optional<at::Tensor>& dk_out, const c10::optional<at::Tensor>& dv_out,
    const at::Tensor& h, const at::Tensor& pos, const at::Tensor& inv_freq, const at::Tensor& cos_tab,
    const at::Tensor& sin_tab, const at::Tensor& ln1, const at::Tensor& wqkv, const c10::optional<at::Tensor>& qn,
    const c10::optional<at::Tensor>& kn, const at::Tensor& wo, const at::Tensor& ln2, const at::Tensor& wgu,
    const at::Tensor& wd, const at::Tensor& k_own, const at::Tensor& v_own, const std::vector<at::Tensor>& past_k,
    const std::vector<at::Tensor>& past_v, const std::vector<at::Tensor>& saved,
    int64_t hq, int64_t hkv, int64_t d, double eps, double scale, int64_t cov, int64_t sp,
    const std::vector<c10::optional<at::Tensor>>& sinks, double sink_scale, int64_t side,
    const std::vector<at::Tensor>& tabs) {
  TS_CHECK(saved.size() == 11 && sinks.size() == 8, "dense_layer_bwd: saved / sink lists");
  const c10::cuda::CUDAGuard guard(h.device());
  const at::Tensor &x1 = saved[0], &rstd1 = saved[1], &qkv = saved[2], &q = saved[3], &o = saved[4],
                   &lse = saved[5], &h1 = saved[6], &x2 = saved[7], &rstd2 = saved[8], &gu = saved[9],
                   &a = saved[10];
  const int64_t t = h.size(0);
  const auto &s_ln1 = sinks[0], &s_qkv = sinks[1], &s_qn = sinks[2], &s_kn = sinks[3], &s_o = sinks[4],
             &s_ln2 = sinks[5], &s_gu = sinks[6], &s_d = sinks[7];
  at::Tensor g_ln1, g_qkv, g_qn, g_kn, g_o, g_ln2, g_gu, g_d;
  auto dout_c = dout.contiguous();
  // out = h1 + down(a)
  auto da = mm_w(dout_c, wd);
  if (s_d) deposit(*s_d, dout_c, a, sink_scale, side);
  else g_d = mm_tn(dout_c, a);
  auto dgu = swiglu_bwd(da, gu);
  auto dx2 = mm_w(dgu, wgu);
  if (s_gu) deposit(*s_gu, dgu, x2, sink_scale, side);
  else g_gu = mm_tn(dgu, x2);
  // h1 -> rmsnorm2, plus the residual branch's gradient
  auto r2 = rms_norm_bwd(dx2, h1, ln2, rstd2, false, dout_c, s_ln2, s_ln2 ? sink_scale : 1.0);
  const at::Tensor dh1 = r2[0];
  if (!s_ln2) g_ln2 = r2[1];
  // h1 = h + o_proj(o)
  auto do2 = mm_w(dh1, wo);
  auto o2 = o.view({t, hq * d});
  if (s_o) deposit(*s_o, dh1, o2, sink_scale, side);
  else g_o = mm_tn(dh1, o2);
  auto do3 = do2.view({t, hq, d});
  // attention over [ancestors | own rows] (the buffer is rebuilt here: no event keeps a copy of its
  // ancestors' rows between its forward and backward); gradients land in one buffer of the same layout
  at::Tensor kbuf = k_own, vbuf = v_own;
  if (sp > 0) kbuf = join_rows(past_k, k_own), vbuf = join_rows(past_v, v_own);
  auto dq = at::empty_like(q);
  auto dkbuf = at::empty_like(kbuf);
  auto dvbuf = at::empty_like(vbuf);
  if (cov < t) dq.narrow(0, cov, t - cov).zero_();
  if (tabs.empty()) {
    if (cov < t) {
      dkbuf.narrow(0, sp + cov, t - cov).zero_();
      dvbuf.narrow(0, sp + cov, t - cov).zero_();
    }
    attn_bwd_tc(do3.narrow(0, 0, cov).contiguous(), q.narrow(0, 0, cov), kbuf.narrow(0, 0, sp + cov),
                vbuf.narrow(0, 0, sp + cov), o.narrow(0, 0, cov), lse, scale, dq.narrow(0, 0, cov),
                dkbuf.narrow(0, 0, sp + cov), dvbuf.narrow(0, 0, sp + cov));
  } else {
    // the key items cover every key row (padding rows get zero gradients)
    TS_CHECK(tabs.size() == 4, "dense_layer_bwd: packed attention needs qtab, far, ktab and cons");
    attn_bwd_packed(do3, q, kbuf, vbuf, o, lse, tabs[0], tabs[1], tabs[2], tabs[3], scale, dq, dkbuf, dvbuf);
  }
  auto dk = dkbuf.narrow(0, sp, t), dv = dvbuf.narrow(0, sp, t);
  if (dk_out) dk.add_(*dk_out);
  if (dv_out) dv.add_(*dv_out);
  // qkv -> QK-norm + RoPE
  auto rq = qk_norm_rope_bwd(dq, dk, dv, qkv, qn, kn, pos, inv_freq, hq, hkv, d, eps, false, cos_tab, sin_tab,
                             s_qn, s_kn, sink_scale);
  const at::Tensor dqkv = *rq[0];
  if (qn && !s_qn) g_qn = *rq[1];
  if (kn && !s_kn) g_kn = *rq[2];
  auto dx1 = mm_w(dqkv, wqkv);
  if (s_qkv) deposit(*s_qkv, dqkv, x1, sink_scale, side);
  else g_qkv = mm_tn(dqkv, x1);
  // h -> rmsnorm1, plus the residual gradient dh1
  auto r1 = rms_norm_bwd(dx1, h, ln1, rstd1, false, dh1, s_ln1, s_ln1 ? sink_scale : 1.0);
  if (!s_ln1) g_ln1 = r1[1];
  return {r1[0], dkbuf.narrow(0, 0, sp), dvbuf.narrow(0, 0, sp), g_ln1, g_qkv, g_qn, g_kn, g_o, g_ln2, g_gu, g_d};
}

}  // namespace ts
