// Bindings of the SIMT / warp-MMA kernels.  Tensors are validated here; the
// current CUDA stream is used; every launch failure raises.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "kernels_api.h"

namespace k = tn5b::kernels;

namespace {
cudaStream_t cur() { return at::cuda::getCurrentCUDAStream().stream(); }
void ok(int r, const char* what) {
  TORCH_CHECK(r == 0, what, " failed: ", r < 0 ? "bad arguments" : cudaGetErrorString(cudaError_t(r)));
}
void need(const at::Tensor& t, at::ScalarType dt, const char* name, bool contiguous = true) {
  TORCH_CHECK(t.is_cuda(), name, " must be on CUDA");
  TORCH_CHECK(t.scalar_type() == dt, name, " has the wrong dtype");
  if (contiguous) TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}
const void* opt_ptr(const c10::optional<at::Tensor>& t) { return t ? t->data_ptr() : nullptr; }

void taco_encode(const at::Tensor& in, at::Tensor& packet) {
  need(in, at::kBFloat16, "input"); need(packet, at::kByte, "packet");
  TORCH_CHECK(packet.numel() == in.numel() / 128 * 136, "packet size must be elements/128*136");
  const c10::cuda::CUDAGuard g(in.device());
  ok(k::taco_encode(in.data_ptr(), packet.data_ptr(), in.numel(), cur()), "taco_encode");
}
void taco_decode(const at::Tensor& packet, at::Tensor& out) {
  need(out, at::kBFloat16, "out"); need(packet, at::kByte, "packet");
  TORCH_CHECK(packet.numel() == out.numel() / 128 * 136, "packet size must be elements/128*136");
  const c10::cuda::CUDAGuard g(out.device());
  ok(k::taco_decode(packet.data_ptr(), out.data_ptr(), out.numel(), cur()), "taco_decode");
}
void taco_decode_reduce(const at::Tensor& local, const at::Tensor& packets, at::Tensor& out, int64_t rank,
                        int64_t world) {
  need(local, at::kBFloat16, "local"); need(packets, at::kByte, "packets"); need(out, at::kBFloat16, "out");
  TORCH_CHECK(packets.numel() == (world - 1) * (local.numel() / 128 * 136), "packets size");
  const c10::cuda::CUDAGuard g(out.device());
  ok(k::taco_decode_reduce(local.data_ptr(), packets.data_ptr(), out.data_ptr(), local.numel(), int(rank),
                           int(world), cur()), "taco_decode_reduce");
}
void ordered_reduce(const at::Tensor& local, const at::Tensor& remote, at::Tensor& out, int64_t rank,
                    int64_t world) {
  need(local, at::kBFloat16, "local"); need(remote, at::kBFloat16, "remote"); need(out, at::kBFloat16, "out");
  TORCH_CHECK(remote.numel() == (world - 1) * local.numel(), "remote size");
  const c10::cuda::CUDAGuard g(out.device());
  ok(k::ordered_reduce(local.data_ptr(), remote.data_ptr(), out.data_ptr(), local.numel(), int(rank),
                       int(world), cur()), "ordered_reduce");
}
void diagnostic_delay(int64_t cycles) { ok(k::diagnostic_delay(uint64_t(cycles), cur()), "diagnostic_delay"); }

void layernorm_fwd(const at::Tensor& x, const at::Tensor& w, const at::Tensor& b, at::Tensor& y,
                   at::Tensor& mean, at::Tensor& rstd, double eps) {
  need(x, at::kBFloat16, "x", false); need(y, at::kBFloat16, "y", false);
  need(w, at::kBFloat16, "w"); need(b, at::kBFloat16, "b");
  need(mean, at::kFloat, "mean"); need(rstd, at::kFloat, "rstd");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && y.stride(1) == 1);
  const c10::cuda::CUDAGuard g(x.device());
  ok(k::layernorm_fwd(x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(), mean.data_ptr<float>(),
                      rstd.data_ptr<float>(), int(x.size(0)), int(x.size(1)), x.stride(0), y.stride(0),
                      float(eps), cur()), "layernorm_fwd");
}
int64_t layernorm_bwd_workspace(int64_t rows, int64_t H) { return 2 * int64_t(k::layernorm_bwd_parts(int(rows))) * H; }
void layernorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w, const at::Tensor& mean,
                   const at::Tensor& rstd, at::Tensor& dx, at::Tensor& dw, at::Tensor& db,
                   at::Tensor& workspace, const c10::optional<at::Tensor>& dres) {
  need(dy, at::kBFloat16, "dy"); need(x, at::kBFloat16, "x"); need(dx, at::kBFloat16, "dx");
  need(workspace, at::kFloat, "workspace");
  TORCH_CHECK(workspace.numel() >= layernorm_bwd_workspace(x.size(0), x.size(1)), "workspace too small");
  const c10::cuda::CUDAGuard g(x.device());
  ok(k::layernorm_bwd(dy.data_ptr(), x.data_ptr(), w.data_ptr(), mean.data_ptr<float>(),
                      rstd.data_ptr<float>(), dx.data_ptr(), dw.data_ptr(), db.data_ptr(),
                      workspace.data_ptr<float>(), int(x.size(0)), int(x.size(1)), opt_ptr(dres), cur()),
     "layernorm_bwd");
}
void column_sum(const at::Tensor& gm, at::Tensor& out, at::Tensor& workspace) {
  need(gm, at::kBFloat16, "g", false); need(out, at::kBFloat16, "out"); need(workspace, at::kFloat, "ws");
  TORCH_CHECK(gm.dim() == 2 && gm.stride(1) == 1);
  TORCH_CHECK(workspace.numel() >= int64_t(k::layernorm_bwd_parts(int(gm.size(0)))) * gm.size(1));
  const c10::cuda::CUDAGuard g(gm.device());
  ok(k::column_sum(gm.data_ptr(), gm.stride(0), int(gm.size(0)), int(gm.size(1)), out.data_ptr(),
                   workspace.data_ptr<float>(), cur()), "column_sum");
}
void gelu_bwd(const at::Tensor& dy, const at::Tensor& pre, at::Tensor& dx) {
  need(dy, at::kBFloat16, "dy"); need(pre, at::kBFloat16, "pre"); need(dx, at::kBFloat16, "dx");
  const c10::cuda::CUDAGuard g(dy.device());
  ok(k::gelu_bwd(dy.data_ptr(), pre.data_ptr(), dx.data_ptr(), dy.numel(), cur()), "gelu_bwd");
}

void ce_stats(const at::Tensor& logits, const at::Tensor& targets, int64_t start, at::Tensor& rowmax,
              at::Tensor& selected) {
  need(logits, at::kBFloat16, "logits", false); need(targets, at::kLong, "targets");
  const c10::cuda::CUDAGuard g(logits.device());
  ok(k::ce_stats(logits.data_ptr(), logits.stride(0), int(logits.size(0)), int(logits.size(1)),
                 targets.data_ptr<int64_t>(), start, rowmax.data_ptr<float>(), selected.data_ptr<float>(),
                 cur()), "ce_stats");
}
void ce_sumexp(const at::Tensor& logits, const at::Tensor& gmax, at::Tensor& sumexp) {
  const c10::cuda::CUDAGuard g(logits.device());
  ok(k::ce_sumexp(logits.data_ptr(), logits.stride(0), int(logits.size(0)), int(logits.size(1)),
                  gmax.data_ptr<float>(), sumexp.data_ptr<float>(), cur()), "ce_sumexp");
}
void ce_loss(const at::Tensor& gmax, const at::Tensor& sumexp, const at::Tensor& selected,
             const c10::optional<at::Tensor>& row_loss, at::Tensor& mean_loss, double scale) {
  const c10::cuda::CUDAGuard g(gmax.device());
  ok(k::ce_loss(gmax.data_ptr<float>(), sumexp.data_ptr<float>(), selected.data_ptr<float>(),
                int(gmax.numel()), row_loss ? row_loss->data_ptr<float>() : nullptr,
                mean_loss.data_ptr<float>(), float(scale), cur()), "ce_loss");
}
void ce_bwd(at::Tensor& logits, const at::Tensor& targets, int64_t start, const at::Tensor& gmax,
            const at::Tensor& sumexp, double scale, const c10::optional<at::Tensor>& scale_t) {
  need(logits, at::kBFloat16, "logits", false);
  const c10::cuda::CUDAGuard g(logits.device());
  ok(k::ce_bwd(logits.data_ptr(), logits.stride(0), int(logits.size(0)), int(logits.size(1)),
               targets.data_ptr<int64_t>(), start, gmax.data_ptr<float>(), sumexp.data_ptr<float>(),
               float(scale), scale_t ? scale_t->data_ptr<float>() : nullptr, cur()), "ce_bwd");
}

int64_t grad_sqsum_parts(int64_t n) { return k::grad_sqsum_parts(n); }
void grad_sqsum(const at::Tensor& grad, at::Tensor& partial, at::Tensor& out, bool accumulate) {
  TORCH_CHECK(grad.is_cuda() && grad.is_contiguous());
  need(partial, at::kDouble, "partial"); need(out, at::kDouble, "out");
  TORCH_CHECK(partial.numel() >= k::grad_sqsum_parts(grad.numel()), "partial workspace too small");
  const bool fp32 = grad.scalar_type() == at::kFloat;
  TORCH_CHECK(fp32 || grad.scalar_type() == at::kBFloat16);
  const c10::cuda::CUDAGuard g(grad.device());
  ok(k::grad_sqsum(grad.data_ptr(), fp32, grad.numel(), partial.data_ptr<double>(), out.data_ptr<double>(),
                   accumulate, cur()), "grad_sqsum");
}
void adamw_step(at::Tensor& master, at::Tensor& m, at::Tensor& v, const at::Tensor& grad, at::Tensor& param,
                int64_t n_decay, const at::Tensor& norm2, double max_norm, double lr, double wd, double beta1,
                double beta2, double eps, int64_t step, const at::Tensor& status) {
  need(master, at::kFloat, "master"); need(m, at::kFloat, "m"); need(v, at::kFloat, "v");
  need(param, at::kBFloat16, "param"); need(norm2, at::kDouble, "norm2");
  const bool fp32 = grad.scalar_type() == at::kFloat;
  TORCH_CHECK(grad.numel() == master.numel() && param.numel() == master.numel() && m.numel() == master.numel());
  const c10::cuda::CUDAGuard g(master.device());
  ok(k::adamw_step(master.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), grad.data_ptr(), fp32,
                   param.data_ptr(), master.numel(), n_decay, norm2.data_ptr<double>(), float(max_norm),
                   float(lr), float(wd), float(beta1), float(beta2), float(eps), int(step),
                   status.data_ptr<int>(), cur()), "adamw_step");
}

void embed_fwd(const at::Tensor& tok, const at::Tensor& E, at::Tensor& out, int64_t start) {
  need(tok, at::kLong, "tokens"); need(E, at::kBFloat16, "E"); need(out, at::kBFloat16, "out");
  const c10::cuda::CUDAGuard g(E.device());
  ok(k::embed_fwd(tok.data_ptr<int64_t>(), E.data_ptr(), out.data_ptr(), int(tok.numel()), int(E.size(1)),
                  start, E.size(0), cur()), "embed_fwd");
}
void add_position(at::Tensor& x, const at::Tensor& P, int64_t row0) {
  need(x, at::kBFloat16, "x"); need(P, at::kBFloat16, "P");
  const c10::cuda::CUDAGuard g(x.device());
  ok(k::add_position(x.data_ptr(), P.data_ptr(), int(x.size(0)), int(x.size(1)), row0, int(P.size(0)), cur()),
     "add_position");
}
void position_bwd(const at::Tensor& gr, at::Tensor& dP, int64_t row0) {
  need(gr, at::kBFloat16, "g"); need(dP, at::kBFloat16, "dP");
  const c10::cuda::CUDAGuard g(gr.device());
  ok(k::position_bwd(gr.data_ptr(), dP.data_ptr(), int(gr.size(0)), int(gr.size(1)), row0, int(dP.size(0)),
                     cur()), "position_bwd");
}
int64_t embed_bwd_workspace(int64_t M, int64_t V) { return k::embed_bwd_workspace_ints(int(M), V); }
void embed_bwd(const at::Tensor& tok, const at::Tensor& gr, at::Tensor& dE, int64_t start, at::Tensor& ws,
               bool accumulate) {
  need(tok, at::kLong, "tokens"); need(gr, at::kBFloat16, "g"); need(dE, at::kBFloat16, "dE");
  need(ws, at::kInt, "workspace");
  TORCH_CHECK(ws.numel() >= k::embed_bwd_workspace_ints(int(tok.numel()), dE.size(0)));
  const c10::cuda::CUDAGuard g(gr.device());
  ok(k::embed_bwd(tok.data_ptr<int64_t>(), gr.data_ptr(), dE.data_ptr(), int(tok.numel()), int(dE.size(1)),
                  start, dE.size(0), ws.data_ptr<int>(), accumulate, cur()), "embed_bwd");
}

void attention_fwd_tc(const at::Tensor& qkv, at::Tensor& out, at::Tensor& lse, int64_t B, int64_t S, int64_t H,
                      double scale, const at::Tensor& status, int64_t timeout_ns, int64_t trace) {
  need(qkv, at::kBFloat16, "qkv", false); need(out, at::kBFloat16, "out", false); need(lse, at::kFloat, "lse");
  TORCH_CHECK(qkv.stride(1) == 1 && out.stride(1) == 1);
  TORCH_CHECK(qkv.size(0) == B * S && qkv.size(1) == 3 * H * 128 && out.size(1) == H * 128);
  const c10::cuda::CUDAGuard g(qkv.device());
  ok(k::attention_fwd_tc(qkv.data_ptr(), qkv.stride(0), out.data_ptr(), out.stride(0), lse.data_ptr<float>(),
                         int(B), int(S), int(H), float(scale), status.data_ptr<int>(), uint64_t(timeout_ns), cur(),
                         reinterpret_cast<unsigned long long*>(trace)),
     "attention_fwd_tc");
}
// Optional [2, CTAs, 8] int64 cycle counters of the backward kernels (dK/dV, dQ).
unsigned long long* dbg_words(const c10::optional<at::Tensor>& dbg, int kernel, int64_t ctas) {
  if (!dbg) return nullptr;
  TORCH_CHECK(dbg->is_cuda() && dbg->scalar_type() == at::kLong && dbg->is_contiguous() &&
                  dbg->numel() == 2 * ctas * 8,
              "attention debug counters must be a contiguous int64 [2, B*H*S/128, 8] CUDA tensor");
  return reinterpret_cast<unsigned long long*>(dbg->data_ptr<int64_t>()) + kernel * ctas * 8;
}
void attention_bwd_tc(const at::Tensor& qkv, const at::Tensor& out, const at::Tensor& dout, const at::Tensor& lse,
                      at::Tensor& Dvec, at::Tensor& dqkv, int64_t B, int64_t S, int64_t H, double scale,
                      const at::Tensor& status, int64_t timeout_ns, const c10::optional<at::Tensor>& dbg) {
  need(qkv, at::kBFloat16, "qkv", false); need(out, at::kBFloat16, "out", false);
  need(dout, at::kBFloat16, "dout", false); need(dqkv, at::kBFloat16, "dqkv", false);
  need(lse, at::kFloat, "lse"); need(Dvec, at::kFloat, "D");
  TORCH_CHECK(qkv.stride(1) == 1 && dout.stride(1) == 1 && dqkv.stride(1) == 1 && out.stride(1) == 1);
  const c10::cuda::CUDAGuard g(qkv.device());
  ok(k::attention_bwd_pre(out.data_ptr(), out.stride(0), dout.data_ptr(), dout.stride(0), Dvec.data_ptr<float>(),
                          int(B), int(S), int(H), cur()), "attention_bwd_pre");
  ok(k::attention_bwd_tc(qkv.data_ptr(), qkv.stride(0), dout.data_ptr(), dout.stride(0), lse.data_ptr<float>(),
                         Dvec.data_ptr<float>(), dqkv.data_ptr(), dqkv.stride(0), int(B), int(S), int(H), float(scale),
                         status.data_ptr<int>(), uint64_t(timeout_ns), cur(), dbg_words(dbg, 0, B * H * (S / 128)),
                         dbg_words(dbg, 1, B * H * (S / 128))),
     "attention_bwd_tc");
}
}  // namespace

// Launch entry points touch no Python object: the GIL is released while they
// run, so other Python threads (e.g. a stall watchdog) keep running.
using nogil = pybind11::call_guard<pybind11::gil_scoped_release>;

void register_kernels(pybind11::module& m) {
  m.def("taco_encode", &taco_encode, nogil());
  m.def("taco_decode", &taco_decode, nogil());
  m.def("taco_decode_reduce", &taco_decode_reduce, nogil());
  m.def("ordered_reduce", &ordered_reduce, nogil());
  m.def("diagnostic_delay", &diagnostic_delay, nogil());
  m.def("layernorm_fwd", &layernorm_fwd, nogil());
  m.def("layernorm_bwd_workspace", &layernorm_bwd_workspace, nogil());
  m.def("layernorm_bwd", &layernorm_bwd, nogil());
  m.def("column_sum", &column_sum, nogil());
  m.def("gelu_bwd", &gelu_bwd, nogil());
  m.def("ce_stats", &ce_stats, nogil());
  m.def("ce_sumexp", &ce_sumexp, nogil());
  m.def("ce_loss", &ce_loss, nogil());
  m.def("ce_bwd", &ce_bwd, nogil());
  m.def("grad_sqsum_parts", &grad_sqsum_parts, nogil());
  m.def("grad_sqsum", &grad_sqsum, nogil());
  m.def("adamw_step", &adamw_step, nogil());
  m.def("embed_fwd", &embed_fwd, nogil());
  m.def("add_position", &add_position, nogil());
  m.def("position_bwd", &position_bwd, nogil());
  m.def("embed_bwd_workspace", &embed_bwd_workspace, nogil());
  m.def("embed_bwd", &embed_bwd, nogil());
  m.def("attention_fwd_tc", &attention_fwd_tc, pybind11::arg("qkv"), pybind11::arg("out"), pybind11::arg("lse"),
        pybind11::arg("B"), pybind11::arg("S"), pybind11::arg("H"), pybind11::arg("scale"), pybind11::arg("status"),
        pybind11::arg("timeout_ns"), pybind11::arg("trace") = 0, nogil());
  m.def("attention_bwd_tc", &attention_bwd_tc, nogil());
}
