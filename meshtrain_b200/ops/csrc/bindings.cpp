// bindings.cpp -- torch adapters for the meshtrain_b200 sm_100a kernels.
//
// Each function validates dtypes/shapes/alignment, launches on the current
// CUDA stream of the tensor's device and raises a Python error if the launch
// fails.  No function here falls back to a library implementation.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "mt_api.h"

namespace {

using torch::Tensor;

#define MT_CHECK_LAUNCH(expr, what)                                              \
  do {                                                                           \
    int _rc = (expr);                                                            \
    TORCH_CHECK(_rc == 0, "meshtrain_b200 ", what, " failed (code ", _rc, ")"); \
  } while (0)

void check_cuda(const Tensor& t, const char* name, at::ScalarType dt) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == dt, name, " has dtype ", t.scalar_type(), ", expected ", dt);
}
void check_rows(const Tensor& t, const char* name) {
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0, name, " must be 16-byte aligned");
}
cudaStream_t stream_of(const Tensor& t) { return at::cuda::getCurrentCUDAStream(t.get_device()); }

void check_matrix(const Tensor& t, const char* name) {
  check_cuda(t, name, at::kBFloat16);
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1, name, " must be a 2-D row-major matrix");
  TORCH_CHECK(t.stride(0) % 8 == 0 && t.stride(0) >= t.size(1), name,
              " leading dimension must be a multiple of 8 elements and cover a row");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0, name, " must be 16-byte aligned");
}

// D = epi(A x B^T).  a: [M,K] (a_mn=false) or [K,M]; b: [N,K] (b_mn=false) or [K,N].
void gemm(Tensor a, bool a_mn, Tensor b, bool b_mn, Tensor d, int64_t epi, c10::optional<Tensor> bias,
          c10::optional<Tensor> aux, c10::optional<Tensor> d2, double beta) {
  check_matrix(a, "A");
  check_matrix(b, "B");
  const int64_t M = a_mn ? a.size(1) : a.size(0);
  const int64_t K = a_mn ? a.size(0) : a.size(1);
  const int64_t N = b_mn ? b.size(1) : b.size(0);
  TORCH_CHECK((b_mn ? b.size(0) : b.size(1)) == K, "gemm: K mismatch");
  TORCH_CHECK(d.is_cuda() && d.dim() == 2 && d.stride(1) == 1 && d.size(0) == M, "gemm: D must be [M, *] row-major");
  TORCH_CHECK(a.get_device() == b.get_device() && a.get_device() == d.get_device(), "gemm: device mismatch");
  const bool f32 = epi == 4;
  TORCH_CHECK(d.scalar_type() == (f32 ? at::kFloat : at::kBFloat16), "gemm: D dtype does not match the epilogue");
  if (epi == 5) {
    TORCH_CHECK(d.size(1) >= N / 2, "gemm: SwiGLU output too narrow");
  } else {
    TORCH_CHECK(d.size(1) >= N, "gemm: D too narrow");
  }
  c10::cuda::CUDAGuard guard(a.get_device());
  mt::GemmArgs g{};
  g.a = a.data_ptr();
  g.lda = a.stride(0);
  g.a_mn = a_mn;
  g.b = b.data_ptr();
  g.ldb = b.stride(0);
  g.b_mn = b_mn;
  g.M = (int)M;
  g.N = (int)N;
  g.K = (int)K;
  g.epi = (int)epi;
  g.d = d.data_ptr();
  g.ldd = d.stride(0);
  g.beta = (float)beta;
  if (bias) {
    check_cuda(*bias, "bias", at::kBFloat16);
    TORCH_CHECK(bias->is_contiguous() && bias->numel() >= N, "gemm: bias must be contiguous [N]");
    g.bias = bias->data_ptr();
  }
  if (aux) {
    check_cuda(*aux, "aux", at::kBFloat16);
    TORCH_CHECK(aux->dim() == 2 && aux->stride(1) == 1 && aux->size(0) == M && aux->size(1) >= N, "gemm: bad aux");
    g.aux = aux->data_ptr();
    g.ldaux = aux->stride(0);
  }
  if (d2) {
    check_cuda(*d2, "d2", at::kBFloat16);
    TORCH_CHECK(d2->dim() == 2 && d2->stride(1) == 1 && d2->size(0) == M && d2->size(1) >= N, "gemm: bad d2");
    g.d2 = d2->data_ptr();
    g.ldd2 = d2->stride(0);
  }
  if (epi == 1 || epi == 5) TORCH_CHECK(g.d2 != nullptr, "gemm: epilogue needs d2");
  if (epi == 2 || epi == 3) TORCH_CHECK(g.aux != nullptr, "gemm: epilogue needs aux");
  if (epi == 5) TORCH_CHECK(N % 32 == 0, "gemm: SwiGLU needs N % 32 == 0");
  if (M == 0 || N == 0) return;
  if (K == 0) {
    if (f32) {
      if (beta == 0.0) d.narrow(1, 0, N).zero_();
      else if (beta != 1.0) d.narrow(1, 0, N).mul_(beta);
    } else {
      d.narrow(1, 0, epi == 5 ? N / 2 : N).zero_();
    }
    return;
  }
  char err[256] = {0};
  int rc = mt::gemm_launch(g, a.get_device(), stream_of(a), err, sizeof(err));
  TORCH_CHECK(rc == 0, "meshtrain_b200 gemm: ", err);
}

std::vector<Tensor> layernorm_fwd(Tensor x, Tensor gamma, Tensor beta, double eps) {
  check_cuda(x, "x", at::kBFloat16);
  check_rows(x, "x");
  const int64_t d = x.size(-1), T = x.numel() / std::max<int64_t>(d, 1);
  c10::cuda::CUDAGuard guard(x.get_device());
  auto y = torch::empty_like(x);
  auto opts = x.options().dtype(at::kFloat);
  auto mean = torch::empty({T}, opts), rstd = torch::empty({T}, opts);
  MT_CHECK_LAUNCH(mt::layernorm_fwd(x.data_ptr(), gamma.data_ptr(), beta.data_ptr(), y.data_ptr(),
                                    mean.data_ptr<float>(), rstd.data_ptr<float>(), (int)T, (int)d, (float)eps,
                                    stream_of(x)),
                  "layernorm_fwd");
  return {y, mean, rstd};
}

Tensor layernorm_bwd(Tensor dy, Tensor x, Tensor gamma, Tensor mean, Tensor rstd, c10::optional<Tensor> dres,
                     Tensor dgamma, Tensor dbeta) {
  check_cuda(dy, "dy", at::kBFloat16);
  check_rows(dy, "dy");
  check_rows(x, "x");
  check_cuda(dgamma, "dgamma", at::kFloat);
  check_cuda(dbeta, "dbeta", at::kFloat);
  const int64_t d = x.size(-1), T = x.numel() / std::max<int64_t>(d, 1);
  c10::cuda::CUDAGuard guard(x.get_device());
  auto dx = torch::empty_like(x);
  MT_CHECK_LAUNCH(mt::layernorm_bwd(dy.data_ptr(), x.data_ptr(), gamma.data_ptr(), mean.data_ptr<float>(),
                                    rstd.data_ptr<float>(), dres ? dres->data_ptr() : nullptr, dx.data_ptr(),
                                    dgamma.data_ptr<float>(), dbeta.data_ptr<float>(), (int)T, (int)d, stream_of(x)),
                  "layernorm_bwd");
  return dx;
}

std::vector<Tensor> rmsnorm_fwd(Tensor x, Tensor gamma, double eps) {
  check_cuda(x, "x", at::kBFloat16);
  check_rows(x, "x");
  const int64_t d = x.size(-1), T = x.numel() / std::max<int64_t>(d, 1);
  c10::cuda::CUDAGuard guard(x.get_device());
  auto y = torch::empty_like(x);
  auto rstd = torch::empty({T}, x.options().dtype(at::kFloat));
  MT_CHECK_LAUNCH(mt::rmsnorm_fwd(x.data_ptr(), gamma.data_ptr(), y.data_ptr(), rstd.data_ptr<float>(), (int)T,
                                  (int)d, (float)eps, stream_of(x)),
                  "rmsnorm_fwd");
  return {y, rstd};
}

Tensor rmsnorm_bwd(Tensor dy, Tensor x, Tensor gamma, Tensor rstd, c10::optional<Tensor> dres, Tensor dgamma) {
  check_cuda(dy, "dy", at::kBFloat16);
  check_rows(dy, "dy");
  check_rows(x, "x");
  check_cuda(dgamma, "dgamma", at::kFloat);
  const int64_t d = x.size(-1), T = x.numel() / std::max<int64_t>(d, 1);
  c10::cuda::CUDAGuard guard(x.get_device());
  auto dx = torch::empty_like(x);
  MT_CHECK_LAUNCH(mt::rmsnorm_bwd(dy.data_ptr(), x.data_ptr(), gamma.data_ptr(), rstd.data_ptr<float>(),
                                  dres ? dres->data_ptr() : nullptr, dx.data_ptr(), dgamma.data_ptr<float>(), (int)T,
                                  (int)d, stream_of(x)),
                  "rmsnorm_bwd");
  return dx;
}

Tensor embedding_fwd(Tensor ids, Tensor tok, c10::optional<Tensor> pos, int64_t S) {
  check_cuda(ids, "ids", at::kLong);
  check_cuda(tok, "tok", at::kBFloat16);
  const int64_t T = ids.numel(), d = tok.size(1), V = tok.size(0);
  c10::cuda::CUDAGuard guard(tok.get_device());
  auto out = torch::empty({T, d}, tok.options());
  MT_CHECK_LAUNCH(mt::embedding_fwd(ids.contiguous().data_ptr<int64_t>(), tok.data_ptr(),
                                    pos ? pos->data_ptr() : nullptr, out.data_ptr(), (int)T, (int)S, (int)d, (int)V,
                                    stream_of(tok)),
                  "embedding_fwd");
  return out;
}

void embedding_bwd(Tensor ids, Tensor dy, Tensor tok_grad, c10::optional<Tensor> pos_grad, int64_t S) {
  check_cuda(ids, "ids", at::kLong);
  check_cuda(dy, "dy", at::kBFloat16);
  check_rows(dy, "dy");
  check_cuda(tok_grad, "tok_grad", at::kFloat);
  const int64_t T = ids.numel(), d = tok_grad.size(1), V = tok_grad.size(0);
  c10::cuda::CUDAGuard guard(dy.get_device());
  Tensor flat_ids = ids.contiguous();
  if (T <= 32768 && V <= 131072) {  // deterministic: sorted by token id, one writer per row
    Tensor scratch = torch::empty({mt::embedding_bwd_sorted_scratch_ints((int)T)},
                                  torch::dtype(torch::kInt32).device(dy.device()));
    MT_CHECK_LAUNCH(mt::embedding_bwd_sorted(flat_ids.data_ptr<int64_t>(), dy.data_ptr(), tok_grad.data_ptr<float>(),
                                             pos_grad ? pos_grad->data_ptr<float>() : nullptr, (int)T, (int)S, (int)d,
                                             (int)V, scratch.data_ptr<int>(), stream_of(dy)),
                    "embedding_bwd_sorted");
    return;
  }
  MT_CHECK_LAUNCH(mt::embedding_bwd(flat_ids.data_ptr<int64_t>(), dy.data_ptr(), tok_grad.data_ptr<float>(),
                                    pos_grad ? pos_grad->data_ptr<float>() : nullptr, (int)T, (int)S, (int)d, (int)V,
                                    stream_of(dy)),
                  "embedding_bwd");
}

void colsum_(Tensor dy, Tensor out) {
  check_cuda(dy, "dy", at::kBFloat16);
  check_cuda(out, "out", at::kFloat);
  TORCH_CHECK(dy.dim() == 2 && dy.stride(1) == 1, "colsum: dy must be 2-D row-major");
  c10::cuda::CUDAGuard guard(dy.get_device());
  MT_CHECK_LAUNCH(mt::colsum_accumulate(dy.data_ptr(), dy.stride(0), out.data_ptr<float>(), (int)dy.size(0),
                                        (int)dy.size(1), stream_of(dy)),
                  "colsum");
}

Tensor swiglu_bwd(Tensor dout, Tensor raw) {
  check_cuda(dout, "dout", at::kBFloat16);
  check_cuda(raw, "raw", at::kBFloat16);
  check_rows(dout, "dout");
  check_rows(raw, "raw");
  const int64_t F = dout.size(-1), T = dout.numel() / std::max<int64_t>(F, 1);
  c10::cuda::CUDAGuard guard(dout.get_device());
  auto draw = torch::empty_like(raw);
  MT_CHECK_LAUNCH(mt::swiglu_bwd(dout.data_ptr(), raw.data_ptr(), draw.data_ptr(), (int)T, (int)F, stream_of(dout)),
                  "swiglu_bwd");
  return draw;
}

void rope_(Tensor qk, int64_t S, int64_t H, int64_t hd, double theta, bool inverse) {
  check_cuda(qk, "qk", at::kBFloat16);
  TORCH_CHECK(qk.dim() == 2 && qk.stride(1) == 1 && qk.size(1) >= H * hd, "rope: qk must be [T, >=H*hd]");
  c10::cuda::CUDAGuard guard(qk.get_device());
  MT_CHECK_LAUNCH(mt::rope_apply(qk.data_ptr(), qk.stride(0), (int)qk.size(0), (int)S, (int)H, (int)hd, (float)theta,
                                 inverse, stream_of(qk)),
                  "rope");
}

void cross_entropy_(Tensor logits, int64_t V, Tensor targets, Tensor loss_sum, double loss_scale, double grad_scale) {
  check_cuda(logits, "logits", at::kBFloat16);
  check_cuda(targets, "targets", at::kLong);
  check_cuda(loss_sum, "loss_sum", at::kFloat);
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1 && logits.stride(0) % 8 == 0 && logits.size(1) >= V,
              "cross_entropy: logits must be [T, >=V] with a leading dim multiple of 8");
  TORCH_CHECK(targets.numel() == logits.size(0), "cross_entropy: one target per row");
  c10::cuda::CUDAGuard guard(logits.get_device());
  MT_CHECK_LAUNCH(mt::cross_entropy_fwd_bwd(logits.data_ptr(), logits.stride(0), targets.contiguous().data_ptr<int64_t>(),
                                            loss_sum.data_ptr<float>(), (int)logits.size(0), (int)V, (float)loss_scale,
                                            (float)grad_scale, stream_of(logits)),
                  "cross_entropy");
}

void adam_(Tensor p, Tensor g, Tensor m, Tensor v, c10::optional<Tensor> pb, double lr, double beta1, double beta2,
           double eps, double wd, bool decoupled, double bc1, double bc2, double grad_scale) {
  for (auto* t : {&p, &g, &m, &v}) {
    check_cuda(*t, "adam buffer", at::kFloat);
    check_rows(*t, "adam buffer");
    TORCH_CHECK(t->numel() == p.numel(), "adam: buffer sizes differ");
  }
  if (pb) {
    check_cuda(*pb, "param_bf16", at::kBFloat16);
    TORCH_CHECK(pb->is_contiguous() && pb->numel() == p.numel(), "adam: bf16 copy size differs");
    TORCH_CHECK((reinterpret_cast<uintptr_t>(pb->data_ptr()) & 7) == 0, "adam: bf16 copy must be 8-byte aligned");
  }
  c10::cuda::CUDAGuard guard(p.get_device());
  MT_CHECK_LAUNCH(mt::adam_step(p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
                                pb ? pb->data_ptr() : nullptr, p.numel(), (float)lr, (float)beta1, (float)beta2,
                                (float)eps, (float)wd, decoupled, (float)bc1, (float)bc2, (float)grad_scale,
                                stream_of(p)),
                  "adam");
}

void cast_bf16_(Tensor in, Tensor out) {
  check_cuda(in, "in", at::kFloat);
  check_cuda(out, "out", at::kBFloat16);
  check_rows(in, "in");
  check_rows(out, "out");
  TORCH_CHECK(in.numel() == out.numel(), "cast: size mismatch");
  c10::cuda::CUDAGuard guard(in.get_device());
  MT_CHECK_LAUNCH(mt::cast_f32_bf16(in.data_ptr<float>(), out.data_ptr(), in.numel(), stream_of(in)), "cast");
}

void check_bshd(const Tensor& t, const char* name) {
  check_cuda(t, name, at::kBFloat16);
  TORCH_CHECK(t.dim() == 4, name, " must be [B, S, H, hd]");
  TORCH_CHECK(t.stride(3) == 1 && t.stride(2) == t.size(3), name, " must have contiguous heads");
  TORCH_CHECK(t.size(0) == 1 || t.stride(0) == t.size(1) * t.stride(1), name, " batches must be back to back");
  TORCH_CHECK(t.stride(1) % 8 == 0 && (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0, name,
              " rows must be 16-byte aligned");
}

std::vector<Tensor> attention_fwd(Tensor q, Tensor k, Tensor v, bool causal, double scale) {
  check_bshd(q, "q");
  check_bshd(k, "k");
  check_bshd(v, "v");
  const int64_t B = q.size(0), S = q.size(1), Hq = q.size(2), hd = q.size(3), Hk = k.size(2);
  TORCH_CHECK(k.size(0) == B && k.size(1) == S && k.size(3) == hd && v.sizes() == k.sizes(), "attention: k/v shape");
  c10::cuda::CUDAGuard guard(q.get_device());
  auto o = torch::empty({B, S, Hq, hd}, q.options());
  auto lse = torch::empty({B, Hq, S}, q.options().dtype(at::kFloat));
  mt::AttnArgs a{};
  a.q = q.data_ptr();
  a.k = k.data_ptr();
  a.v = v.data_ptr();
  a.ld_q = q.stride(1);
  a.ld_k = k.stride(1);
  a.ld_v = v.stride(1);
  a.o = o.data_ptr();
  a.ld_o = Hq * hd;
  a.lse = lse.data_ptr<float>();
  a.B = (int)B;
  a.S = (int)S;
  a.Hq = (int)Hq;
  a.Hk = (int)Hk;
  a.hd = (int)hd;
  a.scale = (float)scale;
  a.causal = causal;
  char err[256] = {0};
  int rc = mt::attention_fwd(a, q.get_device(), stream_of(q), err, sizeof(err));
  TORCH_CHECK(rc == 0, "meshtrain_b200 ", err);
  return {o, lse};
}

std::vector<Tensor> attention_bwd(Tensor dout, Tensor q, Tensor k, Tensor v, Tensor o, Tensor lse, bool causal,
                                  double scale, c10::optional<Tensor> dq_out, c10::optional<Tensor> dk_out,
                                  c10::optional<Tensor> dv_out) {
  check_bshd(dout, "dout");
  check_bshd(q, "q");
  check_bshd(k, "k");
  check_bshd(v, "v");
  check_bshd(o, "o");
  check_cuda(lse, "lse", at::kFloat);
  TORCH_CHECK(lse.is_contiguous(), "lse must be contiguous [B, Hq, S]");
  const int64_t B = q.size(0), S = q.size(1), Hq = q.size(2), hd = q.size(3), Hk = k.size(2);
  c10::cuda::CUDAGuard guard(q.get_device());
  Tensor dq = dq_out ? *dq_out : torch::empty({B, S, Hq, hd}, q.options());
  Tensor dk = dk_out ? *dk_out : torch::empty({B, S, Hk, hd}, q.options());
  Tensor dv = dv_out ? *dv_out : torch::empty({B, S, Hk, hd}, q.options());
  check_bshd(dq, "dq");
  check_bshd(dk, "dk");
  check_bshd(dv, "dv");
  auto fopts = q.options().dtype(at::kFloat);
  auto dq_accum = torch::empty({B, S, Hq, hd}, fopts);
  auto delta = torch::empty({B, Hq, S}, fopts);
  mt::AttnBwdArgs a{};
  a.f.q = q.data_ptr();
  a.f.k = k.data_ptr();
  a.f.v = v.data_ptr();
  a.f.ld_q = q.stride(1);
  a.f.ld_k = k.stride(1);
  a.f.ld_v = v.stride(1);
  a.f.o = o.data_ptr();
  a.f.ld_o = o.stride(1);
  a.f.lse = lse.data_ptr<float>();
  a.f.B = (int)B;
  a.f.S = (int)S;
  a.f.Hq = (int)Hq;
  a.f.Hk = (int)Hk;
  a.f.hd = (int)hd;
  a.f.scale = (float)scale;
  a.f.causal = causal;
  a.dout = dout.data_ptr();
  a.ld_do = dout.stride(1);
  a.dq = dq.data_ptr();
  a.dk = dk.data_ptr();
  a.dv = dv.data_ptr();
  a.ld_dq = dq.stride(1);
  a.ld_dk = dk.stride(1);
  a.ld_dv = dv.stride(1);
  a.dq_accum = dq_accum.data_ptr<float>();
  a.delta = delta.data_ptr<float>();
  char err[256] = {0};
  int rc = mt::attention_bwd(a, q.get_device(), stream_of(q), err, sizeof(err));
  TORCH_CHECK(rc == 0, "meshtrain_b200 ", err);
  return {dq, dk, dv};
}

int64_t read_status(int64_t device) { return (int64_t)mt::read_and_clear_status((int)device); }
int64_t read_checks() { return (int64_t)mt::read_and_clear_checks(); }

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "meshtrain_b200 hand-written sm_100a kernels";
  m.def("gemm", &gemm, "tcgen05 GEMM with fused epilogue");
  m.def("layernorm_fwd", &layernorm_fwd);
  m.def("layernorm_bwd", &layernorm_bwd);
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("embedding_fwd", &embedding_fwd);
  m.def("embedding_bwd", &embedding_bwd);
  m.def("colsum_", &colsum_);
  m.def("swiglu_bwd", &swiglu_bwd);
  m.def("rope_", &rope_);
  m.def("cross_entropy_", &cross_entropy_);
  m.def("adam_", &adam_);
  m.def("cast_bf16_", &cast_bf16_);
  m.def("attention_fwd", &attention_fwd);
  m.def("attention_bwd", &attention_bwd);
  m.def("read_status", &read_status);
  m.def("read_checks", &read_checks);
  m.def("debug_checks_built", &mt::debug_checks_built);
}
