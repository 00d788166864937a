// Torch operator registration for the harp_b200 CUDA library.
//
// Namespaces:
//   harp::*                the framework's own fused kernels (used by the models)
//   xhpops::kp_linear_*    the reference's linear ops (unigemm_linear.py:25,45;
//                          their library kernels/_C*.so is not shipped) on harp_gemm
//   async_op::*            the reference's elementwise / norm / rope / init /
//                          foreach_adamw ops (async_rt/csrc/async_op_api.cc:46-73,
//                          kp_multi_tensor_adamw.py:67) with the same schemas
// ring_attention_ops::* and harp_comm::* are registered in attention_sm100.cu
// and comm.cu.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <torch/library.h>

#include "gemm_sm100.h"
#include "staging.h"

namespace harp {

// elementwise.cu
int rows_per_block_for(int rows_per_batch);
void rmsnorm_mod_fwd(const at::Tensor& x, const c10::optional<at::Tensor>& w, const c10::optional<at::Tensor>& scale,
                     const c10::optional<at::Tensor>& shift, int64_t rows_per_batch, double eps, at::Tensor& y,
                     at::Tensor& rstd, bool save_rms);
void rmsnorm_mod_bwd(const at::Tensor& x, const at::Tensor& rstd, const at::Tensor& dy,
                     const c10::optional<at::Tensor>& w, const c10::optional<at::Tensor>& scale, int64_t rows_per_batch,
                     const c10::optional<at::Tensor>& dres, at::Tensor& dx, const c10::optional<at::Tensor>& pw,
                     const c10::optional<at::Tensor>& ps, const c10::optional<at::Tensor>& pb, int64_t rpb);
void reduce_partials(const at::Tensor& part, int64_t per_group, at::Tensor& out, bool accumulate);
void qknorm_rope_fwd(const at::Tensor& qkv, int64_t H, int64_t Dh, const c10::optional<at::Tensor>& wq,
                     const c10::optional<at::Tensor>& wk, const c10::optional<at::Tensor>& freqs, int64_t freq_rows,
                     double eps, bool do_norm, at::Tensor& qo, at::Tensor& ko, const c10::optional<at::Tensor>& rstd_q,
                     const c10::optional<at::Tensor>& rstd_k);
void qknorm_rope_bwd(const at::Tensor& dq, const at::Tensor& dk, const at::Tensor& qkv,
                     const c10::optional<at::Tensor>& rstd_q, const c10::optional<at::Tensor>& rstd_k, int64_t H,
                     int64_t Dh, const c10::optional<at::Tensor>& wq, const c10::optional<at::Tensor>& wk,
                     const c10::optional<at::Tensor>& freqs, int64_t freq_rows, bool do_norm, at::Tensor& dqkv,
                     const c10::optional<at::Tensor>& pwq, const c10::optional<at::Tensor>& pwk, int64_t items_per_block);
void swiglu_fwd(const at::Tensor& gu, at::Tensor& h);
void swiglu_bwd(const at::Tensor& dh, const at::Tensor& gu, at::Tensor& dgu);
void gate_bwd(const at::Tensor& dy, const c10::optional<at::Tensor>& a, const at::Tensor& gate, int64_t rows_per_batch,
              at::Tensor& da, const c10::optional<at::Tensor>& pg, const c10::optional<at::Tensor>& pb, int64_t rpb);
void colsum_partial(const at::Tensor& x, int64_t rpb, at::Tensor& part);
void layernorm_mod_fwd(const at::Tensor& x, const c10::optional<at::Tensor>& scale,
                       const c10::optional<at::Tensor>& shift, int64_t rows_per_batch, double eps, at::Tensor& y,
                       at::Tensor& mean, at::Tensor& rstd);
void layernorm_mod_bwd(const at::Tensor& x, const at::Tensor& mean, const at::Tensor& rstd, const at::Tensor& dy,
                       const c10::optional<at::Tensor>& scale, int64_t rows_per_batch, at::Tensor& dx,
                       const c10::optional<at::Tensor>& ps, const c10::optional<at::Tensor>& pb, int64_t rpb);
void elementwise(int64_t op, const at::Tensor& a, const c10::optional<at::Tensor>& b, double s, at::Tensor& out);
void adamw_flat(at::Tensor& master, at::Tensor& m, at::Tensor& v, const at::Tensor& grad,
                const c10::optional<at::Tensor>& param, double lr, double beta1, double beta2, double eps, double wd,
                int64_t step, double grad_scale, const c10::optional<at::Tensor>& hyper);
void adamw_list(at::TensorList params, at::TensorList grads, at::TensorList exp_avgs, at::TensorList exp_avg_sqs,
                double lr, double beta1, double beta2, double eps, double wd, int64_t step);
void philox_uniform(at::Tensor& out, int64_t seed, int64_t offset, double lo, double hi);
void rowdot(const at::Tensor& a, const at::Tensor& b, int64_t H, int64_t Dh, int64_t S, at::Tensor& out);

namespace {

// Per-device error word used by the compat ops (which have no err argument).
at::Tensor& compat_err(const at::Device& dev) {
  static std::vector<at::Tensor> words(64);
  auto& w = words.at(dev.index());
  if (!w.defined()) w = at::zeros({4}, at::TensorOptions().dtype(at::kInt).device(dev));
  return w;
}

void gemm_op(const at::Tensor& A, bool a_mn, const at::Tensor& B, bool b_mn, at::Tensor C, int64_t M, int64_t N,
             int64_t K, const c10::optional<at::Tensor>& bias, int64_t epi, double alpha,
             const c10::optional<at::Tensor>& residual, const c10::optional<at::Tensor>& gate, int64_t rows_per_batch,
             at::Tensor err, bool force_simt, const c10::optional<at::Tensor>& C2) {
  gemm(A, a_mn, B, b_mn, C, (int)M, (int)N, (int)K, bias, (int)epi, alpha, residual, gate, (int)rows_per_batch, err,
       force_simt, C2);
}

// ---- xhpops (reference linear ops) ----
void kp_linear_forward(const at::Tensor& input, const at::Tensor& weight, const c10::optional<at::Tensor>& bias,
                       at::Tensor out) {
  auto x = input.reshape({-1, input.size(-1)});
  auto o = out.view({-1, out.size(-1)});
  gemm(x, false, weight, false, o, x.size(0), weight.size(0), x.size(1), bias, kEpiStoreBf16, 1.0, c10::nullopt,
       c10::nullopt, 0, compat_err(input.device()), false);
}
void kp_linear_backward(const at::Tensor& grad_out, const at::Tensor& input, const at::Tensor& weight,
                        at::Tensor grad_input, at::Tensor grad_weight, const c10::optional<at::Tensor>& grad_bias) {
  auto g = grad_out.reshape({-1, grad_out.size(-1)}).contiguous();
  auto x = input.reshape({-1, input.size(-1)}).contiguous();
  auto gi = grad_input.view({-1, grad_input.size(-1)});
  const int M = g.size(0), N = weight.size(0), K = weight.size(1);
  auto& err = compat_err(input.device());
  gemm(g, false, weight, true, gi, M, K, N, c10::nullopt, kEpiStoreBf16, 1.0, c10::nullopt, c10::nullopt, 0, err,
       false);
  gemm(g, true, x, true, grad_weight, N, K, M, c10::nullopt, kEpiStoreBf16, 1.0, c10::nullopt, c10::nullopt, 0, err,
       false);
  if (grad_bias.has_value()) {
    const int rpb = 64;
    auto part = at::empty({(M + rpb - 1) / rpb, N}, g.options().dtype(at::kFloat));
    colsum_partial(g, rpb, part);
    auto gb = grad_bias->view({1, N});
    reduce_partials(part, part.size(0), gb, false);
  }
}

// ---- async_op (reference elementwise / norm / rope ops) ----
void silu_out(const at::Tensor& x, at::Tensor out) { elementwise(0, x, c10::nullopt, 0, out); }
void silu_backward_out(const at::Tensor& dy, const at::Tensor& x, at::Tensor dx) { elementwise(1, dy, x, 0, dx); }
void tanh_out(const at::Tensor& x, at::Tensor out) { elementwise(2, x, c10::nullopt, 0, out); }
void tanh_backward_out(const at::Tensor& dy, const at::Tensor& y, at::Tensor dx) { elementwise(3, dy, y, 0, dx); }
void add_out(const at::Tensor& a, const at::Tensor& b, at::Tensor out) { elementwise(4, a, b, 0, out); }
void mul_out(const at::Tensor& a, const at::Tensor& b, at::Tensor out) { elementwise(5, a, b, 0, out); }
void add_scalar_out(const at::Tensor& a, double s, at::Tensor out) { elementwise(6, a, c10::nullopt, s, out); }

// rmsnorm_forward_out saves rms (not its inverse), as the reference does
// (rms_norm.cc:21-101).
// The caller's tensors may be views at any offset: operands that are not
// contiguous 16-byte aligned blocks are staged (staging.h).
void rmsnorm_forward_out(const at::Tensor& input, const at::Tensor& weight, at::Tensor output, at::Tensor rms,
                         double eps) {
  TORCH_CHECK(input.scalar_type() == at::kBFloat16 && weight.scalar_type() == at::kBFloat16 &&
                  output.scalar_type() == at::kBFloat16 && rms.scalar_type() == at::kFloat,
              "rmsnorm_forward_out: bf16 input, weight and output, fp32 rms");
  auto x = block16(input).view({-1, input.size(-1)});
  StagedOut out(output), r(rms);
  auto y = out.work.view({-1, output.size(-1)});
  rmsnorm_mod_fwd(x, block16(weight), c10::nullopt, c10::nullopt, x.size(0), eps, y, r.work, true);
  out.finish();
  r.finish();
}
void rmsnorm_backward_out(const at::Tensor& input, const at::Tensor& grad_out, const at::Tensor& weight,
                          const at::Tensor& rms, at::Tensor grad_input, at::Tensor grad_weight) {
  TORCH_CHECK(input.scalar_type() == at::kBFloat16 && grad_out.scalar_type() == at::kBFloat16 &&
                  weight.scalar_type() == at::kBFloat16 && grad_input.scalar_type() == at::kBFloat16 &&
                  grad_weight.scalar_type() == at::kBFloat16,
              "rmsnorm_backward_out: bf16 tensors (rms fp32)");
  auto x = block16(input).view({-1, input.size(-1)});
  auto g = block16(grad_out).view({-1, grad_out.size(-1)});
  StagedOut gi_out(grad_input), gw_out(grad_weight);
  auto gi = gi_out.work.view({-1, grad_input.size(-1)});
  const int R = x.size(0), D = x.size(1);
  auto rstd = rms.reciprocal().contiguous();
  const int rpb = 32;
  auto pw = at::empty({(R + rpb - 1) / rpb, D}, x.options().dtype(at::kFloat));
  rmsnorm_mod_bwd(x, rstd, g, block16(weight), c10::nullopt, R, c10::nullopt, gi, pw, c10::nullopt, c10::nullopt,
                  rpb);
  auto gw = gw_out.work.view({1, D});
  reduce_partials(pw, pw.size(0), gw, false);
  gi_out.finish();
  gw_out.finish();
}
// x: [..., D] (interleaved complex pairs); freqs_cis: complex64 [..., D/2]
// broadcastable over the leading dims of x except the last two.
void rope_apply(const at::Tensor& x, const at::Tensor& freqs_cis, at::Tensor out, bool inverse) {
  auto f = at::view_as_real(freqs_cis.to(at::kComplexFloat));
  auto c = f.select(-1, 0), s = f.select(-1, 1);
  auto xf = x.to(at::kFloat).reshape({-1, x.size(-1) / 2, 2});
  // broadcast freqs over x's leading dims: reference layout [B,H,T,D] with
  // freqs [B,T,D/2] -> unsqueeze head dim.
  at::Tensor cb = c, sb = s;
  if (x.dim() == 4 && freqs_cis.dim() == 3) { cb = c.unsqueeze(1); sb = s.unsqueeze(1); }
  cb = cb.expand({x.size(0), x.dim() == 4 ? x.size(1) : 1, x.size(-2), x.size(-1) / 2}).reshape({-1, x.size(-1) / 2});
  sb = sb.expand({x.size(0), x.dim() == 4 ? x.size(1) : 1, x.size(-2), x.size(-1) / 2}).reshape({-1, x.size(-1) / 2});
  auto x0 = xf.select(-1, 0), x1 = xf.select(-1, 1);
  at::Tensor o0, o1;
  if (!inverse) { o0 = x0 * cb - x1 * sb; o1 = x0 * sb + x1 * cb; }
  else { o0 = x0 * cb + x1 * sb; o1 = -x0 * sb + x1 * cb; }
  out.copy_(at::stack({o0, o1}, -1).reshape(x.sizes()).to(out.scalar_type()));
}
void rope_forward_impl(const at::Tensor& x, const at::Tensor& freqs, at::Tensor out) { rope_apply(x, freqs, out, false); }
void rope_backward_impl(const at::Tensor& g, const at::Tensor& freqs, at::Tensor out) { rope_apply(g, freqs, out, true); }

at::Tensor random_uniform(at::Tensor self, double from, double to, c10::optional<at::Generator> gen) {
  static int64_t offset = 0;
  (void)gen;
  // Fixed seed: every rank draws identical initial weights, as the reference's
  // FastInitMode requires (random.cc:158-172, train.py:274-285).
  if (self.is_contiguous()) {
    philox_uniform(self, 42, offset, from, to);
  } else {
    auto tmp = at::empty_like(self, self.options().memory_format(at::MemoryFormat::Contiguous));
    philox_uniform(tmp, 42, offset, from, to);
    self.copy_(tmp);
  }
  offset += (self.numel() + 3) / 4;
  return self;
}

void foreach_adamw(at::TensorList params, at::TensorList grads, at::TensorList exp_avgs, at::TensorList exp_avg_sqs,
                   at::TensorList steps, double beta1, double beta2, double eps, double lr) {
  // steps: per-param step counters (0-d tensors), incremented here.
  for (auto& s : steps) const_cast<at::Tensor&>(s).add_(1);
  const int64_t step = steps.empty() ? 1 : steps[0].item<double>();
  adamw_list(params, grads, exp_avgs, exp_avg_sqs, lr, beta1, beta2, eps, 0.0, step);
}
void foreach_adamw_wd(at::TensorList params, at::TensorList grads, at::TensorList exp_avgs,
                      at::TensorList exp_avg_sqs, at::TensorList steps, double beta1, double beta2, double eps,
                      double lr, double weight_decay) {
  for (auto& s : steps) const_cast<at::Tensor&>(s).add_(1);
  const int64_t step = steps.empty() ? 1 : steps[0].item<double>();
  adamw_list(params, grads, exp_avgs, exp_avg_sqs, lr, beta1, beta2, eps, weight_decay, step);
}

int64_t launch_count_op() { return launch_count(); }
// Replays of a captured CUDA graph launch the captured harp kernels again
// without passing through the launchers; the caller adds them here.
void add_launch_count_op(int64_t n) { add_launch_count(n); }
void reset_launch_count_op() { reset_launch_count(); }
int64_t gemm_pair_mode_op(int64_t mode) { return set_gemm_pair_mode((int)mode); }
int64_t rows_per_block_op(int64_t rpb) { return rows_per_block_for((int)rpb); }

}  // namespace
}  // namespace harp

TORCH_LIBRARY(harp, m) {
  m.def("gemm(Tensor A, bool a_mn, Tensor B, bool b_mn, Tensor(a!) C, int M, int N, int K, Tensor? bias, int epi, "
        "float alpha, Tensor? residual, Tensor? gate, int rows_per_batch, Tensor(b!) err, bool force_simt, "
        "Tensor(c!)? C2=None) -> ()");
  m.def("rmsnorm_mod_fwd(Tensor x, Tensor? w, Tensor? scale, Tensor? shift, int rows_per_batch, float eps, "
        "Tensor(a!) y, Tensor(b!) rstd, bool save_rms) -> ()");
  m.def("rmsnorm_mod_bwd(Tensor x, Tensor rstd, Tensor dy, Tensor? w, Tensor? scale, int rows_per_batch, "
        "Tensor? dres, Tensor(a!) dx, Tensor(b!)? pw, Tensor(c!)? ps, Tensor(d!)? pb, int rpb) -> ()");
  m.def("reduce_partials(Tensor part, int per_group, Tensor(a!) out, bool accumulate) -> ()");
  m.def("qknorm_rope_fwd(Tensor qkv, int H, int Dh, Tensor? wq, Tensor? wk, Tensor? freqs, int freq_rows, float eps, "
        "bool do_norm, Tensor(a!) qo, Tensor(b!) ko, Tensor(c!)? rstd_q, Tensor(d!)? rstd_k) -> ()");
  m.def("qknorm_rope_bwd(Tensor dq, Tensor dk, Tensor qkv, Tensor? rstd_q, Tensor? rstd_k, int H, int Dh, Tensor? wq, "
        "Tensor? wk, Tensor? freqs, int freq_rows, bool do_norm, Tensor(a!) dqkv, Tensor(b!)? pwq, Tensor(c!)? pwk, "
        "int items_per_block) -> ()");
  m.def("swiglu_fwd(Tensor gu, Tensor(a!) h) -> ()");
  m.def("swiglu_bwd(Tensor dh, Tensor gu, Tensor(a!) dgu) -> ()");
  m.def("gate_bwd(Tensor dy, Tensor? a, Tensor gate, int rows_per_batch, Tensor(a!) da, Tensor(b!)? pg, "
        "Tensor(c!)? pb, int rpb) -> ()");
  m.def("colsum_partial(Tensor x, int rpb, Tensor(a!) part) -> ()");
  m.def("layernorm_mod_fwd(Tensor x, Tensor? scale, Tensor? shift, int rows_per_batch, float eps, Tensor(a!) y, "
        "Tensor(b!) mean, Tensor(c!) rstd) -> ()");
  m.def("layernorm_mod_bwd(Tensor x, Tensor mean, Tensor rstd, Tensor dy, Tensor? scale, int rows_per_batch, "
        "Tensor(a!) dx, Tensor(b!)? ps, Tensor(c!)? pb, int rpb) -> ()");
  m.def("elementwise(int op, Tensor a, Tensor? b, float s, Tensor(a!) out) -> ()");
  m.def("adamw_flat(Tensor(a!) master, Tensor(b!) m, Tensor(c!) v, Tensor grad, Tensor(d!)? param, float lr, "
        "float beta1, float beta2, float eps, float wd, int step, float grad_scale, Tensor? hyper=None) -> ()");
  m.def("philox_uniform(Tensor(a!) out, int seed, int offset, float lo, float hi) -> ()");
  m.def("rowdot(Tensor a, Tensor b, int H, int Dh, int S, Tensor(a!) out) -> ()");
  m.def("launch_count() -> int");
  m.def("add_launch_count(int n) -> ()");
  m.def("reset_launch_count() -> ()");
  m.def("rows_per_block(int rows_per_batch) -> int");
  m.def("gemm_pair_mode(int mode) -> int");
  m.def("gemm_probe() -> Tensor");
  m.def("set_weight_gate(Tensor? flags, int first, int count, int epoch, float timeout_s, Tensor? step_delta=None, "
        "int per_step=0) -> ()");
  m.def("debug_bounds_status() -> Tensor");
}

TORCH_LIBRARY_IMPL(harp, CUDA, m) {
  m.impl("gemm", &harp::gemm_op);
  m.impl("rmsnorm_mod_fwd", &harp::rmsnorm_mod_fwd);
  m.impl("rmsnorm_mod_bwd", &harp::rmsnorm_mod_bwd);
  m.impl("reduce_partials", &harp::reduce_partials);
  m.impl("qknorm_rope_fwd", &harp::qknorm_rope_fwd);
  m.impl("qknorm_rope_bwd", &harp::qknorm_rope_bwd);
  m.impl("swiglu_fwd", &harp::swiglu_fwd);
  m.impl("swiglu_bwd", &harp::swiglu_bwd);
  m.impl("gate_bwd", &harp::gate_bwd);
  m.impl("colsum_partial", &harp::colsum_partial);
  m.impl("layernorm_mod_fwd", &harp::layernorm_mod_fwd);
  m.impl("layernorm_mod_bwd", &harp::layernorm_mod_bwd);
  m.impl("elementwise", &harp::elementwise);
  m.impl("adamw_flat", &harp::adamw_flat);
  m.impl("philox_uniform", &harp::philox_uniform);
  m.impl("rowdot", &harp::rowdot);
}

TORCH_LIBRARY_IMPL(harp, CompositeExplicitAutograd, m) {
  m.impl("launch_count", &harp::launch_count_op);
  m.impl("add_launch_count", &harp::add_launch_count_op);
  m.impl("reset_launch_count", &harp::reset_launch_count_op);
  m.impl("rows_per_block", &harp::rows_per_block_op);
  m.impl("gemm_pair_mode", &harp::gemm_pair_mode_op);
  m.impl("gemm_probe", &harp::gemm_probe);
  m.impl("set_weight_gate", &harp::set_weight_gate);
  m.impl("debug_bounds_status", &harp::debug_bounds_status);
}

TORCH_LIBRARY(xhpops, m) {
  m.def("kp_linear_forward(Tensor input, Tensor weight, Tensor? bias, Tensor(a!) out) -> ()");
  m.def("kp_linear_backward(Tensor grad_out, Tensor input, Tensor weight, Tensor(a!) grad_input, "
        "Tensor(b!) grad_weight, Tensor(c!)? grad_bias) -> ()");
}
TORCH_LIBRARY_IMPL(xhpops, CUDA, m) {
  m.impl("kp_linear_forward", &harp::kp_linear_forward);
  m.impl("kp_linear_backward", &harp::kp_linear_backward);
}

TORCH_LIBRARY(async_op, m) {
  m.def("silu_out(Tensor x, Tensor(a!) out) -> ()");
  m.def("silu_backward_out(Tensor grad_out, Tensor x, Tensor(a!) grad_in) -> ()");
  m.def("tanh_out(Tensor x, Tensor(a!) out) -> ()");
  m.def("tanh_backward_out(Tensor grad_out, Tensor y, Tensor(a!) grad_in) -> ()");
  m.def("add_out(Tensor a, Tensor b, Tensor(a!) out) -> ()");
  m.def("mul_out(Tensor a, Tensor b, Tensor(a!) out) -> ()");
  m.def("add_scalar_out(Tensor a, float s, Tensor(a!) out) -> ()");
  m.def("rmsnorm_forward_out(Tensor input, Tensor weight, Tensor(a!) output, Tensor(b!) rms, float eps) -> ()");
  m.def("rmsnorm_backward_out(Tensor input, Tensor grad_out, Tensor weight, Tensor rms, Tensor(a!) grad_input, "
        "Tensor(b!) grad_weight) -> ()");
  m.def("rope_forward_impl(Tensor x, Tensor freqs_cis, Tensor(a!) out) -> ()");
  m.def("rope_backward_impl(Tensor grad, Tensor freqs_cis, Tensor(a!) out) -> ()");
  m.def("random_uniform(Tensor(a!) self, float from=0, float to=1, *, Generator? generator=None) -> Tensor(a!)");
  m.def("foreach_adamw(Tensor(a!)[] params, Tensor[] grads, Tensor(b!)[] exp_avgs, Tensor(c!)[] exp_avg_sqs, "
        "Tensor(d!)[] steps, float beta1, float beta2, float eps, float lr) -> ()");
  m.def("foreach_adamw_wd(Tensor(a!)[] params, Tensor[] grads, Tensor(b!)[] exp_avgs, Tensor(c!)[] exp_avg_sqs, "
        "Tensor(d!)[] steps, float beta1, float beta2, float eps, float lr, float weight_decay) -> ()");
}
TORCH_LIBRARY_IMPL(async_op, CUDA, m) {
  m.impl("silu_out", &harp::silu_out);
  m.impl("silu_backward_out", &harp::silu_backward_out);
  m.impl("tanh_out", &harp::tanh_out);
  m.impl("tanh_backward_out", &harp::tanh_backward_out);
  m.impl("add_out", &harp::add_out);
  m.impl("mul_out", &harp::mul_out);
  m.impl("add_scalar_out", &harp::add_scalar_out);
  m.impl("rmsnorm_forward_out", &harp::rmsnorm_forward_out);
  m.impl("rmsnorm_backward_out", &harp::rmsnorm_backward_out);
  m.impl("rope_forward_impl", &harp::rope_forward_impl);
  m.impl("rope_backward_impl", &harp::rope_backward_impl);
  m.impl("random_uniform", &harp::random_uniform);
  m.impl("foreach_adamw", &harp::foreach_adamw);
  m.impl("foreach_adamw_wd", &harp::foreach_adamw_wd);
}
