// PyTorch bindings of the model-side kernels.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "ops_api.h"

namespace nexar {

void count_launch(unsigned long long n);

namespace {
cudaStream_t stream_of(const at::Tensor& t) {
  return at::cuda::getCurrentCUDAStream(t.get_device()).stream();
}
void chk(cudaError_t e, const char* what) {
  TORCH_CHECK(e == cudaSuccess, "nexar_b200: ", what, " failed: ", cudaGetErrorString(e));
}
void need_bf16(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.is_contiguous(), "nexar_b200: ", name,
              " must be a contiguous bf16 CUDA tensor");
}
void need_f32(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kFloat && t.is_contiguous(), "nexar_b200: ", name,
              " must be a contiguous fp32 CUDA tensor");
}
__nv_bfloat16* bf(const at::Tensor& t) { return reinterpret_cast<__nv_bfloat16*>(t.data_ptr()); }
const __nv_bfloat16* bfc(const c10::optional<at::Tensor>& t) {
  return t ? reinterpret_cast<const __nv_bfloat16*>(t->data_ptr()) : nullptr;
}
}  // namespace

// LayerNorm forward; x: [R, C]. Returns nothing; writes y, mean, rstd (and
// sum_out = x + res when res is given).
void op_ln_fwd(const at::Tensor& x, const c10::optional<at::Tensor>& res,
               const c10::optional<at::Tensor>& sum_out, const at::Tensor& w, const at::Tensor& b,
               const at::Tensor& y, const at::Tensor& mean, const at::Tensor& rstd, double eps,
               const c10::optional<at::Tensor>& rbias) {
  need_bf16(x, "x");
  need_bf16(y, "y");
  need_bf16(w, "weight");
  need_bf16(b, "bias");
  need_f32(mean, "mean");
  need_f32(rstd, "rstd");
  const int C = x.size(-1);
  const int R = x.numel() / C;
  TORCH_CHECK(res.has_value() == sum_out.has_value(), "ln_fwd: res and sum_out go together");
  TORCH_CHECK(!rbias || (res && rbias->numel() == C), "ln_fwd: rbias needs res and C elements");
  c10::cuda::CUDAGuard g(x.get_device());
  chk(ln_fwd_ex(bf(x), bfc(res), bfc(rbias), sum_out ? bf(*sum_out) : nullptr, bf(w), bf(b), bf(y),
                mean.data_ptr<float>(), rstd.data_ptr<float>(), R, C, (float)eps, stream_of(x)),
      "ln_fwd");
  count_launch(1);
}

int64_t op_ln_bwd_scratch_floats(int64_t R, int64_t C, bool dsum) {
  return (int64_t)ln_bwd_scratch_floats_ex((int)C, ln_bwd_blocks((int)R), dsum);
}

void op_ln_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& mean, const at::Tensor& rstd,
               const at::Tensor& w, const c10::optional<at::Tensor>& dres, const at::Tensor& dx,
               const at::Tensor& dw, const at::Tensor& db, const at::Tensor& scratch,
               const at::Tensor& counter, const c10::optional<at::Tensor>& dsum) {
  need_bf16(dy, "dy");
  need_bf16(x, "x");
  need_bf16(dx, "dx");
  need_bf16(dw, "dw");
  need_bf16(db, "db");
  need_f32(scratch, "scratch");
  const int C = x.size(-1);
  const int R = x.numel() / C;
  const int blocks = ln_bwd_blocks(R);
  TORCH_CHECK((size_t)scratch.numel() >= ln_bwd_scratch_floats_ex(C, blocks, dsum.has_value()),
              "ln_bwd: scratch too small");
  if (dsum) need_bf16(*dsum, "dsum");
  c10::cuda::CUDAGuard g(x.get_device());
  chk(ln_bwd_ex(bf(dy), bf(x), mean.data_ptr<float>(), rstd.data_ptr<float>(), bf(w), bfc(dres), bf(dx),
                bf(dw), bf(db), dsum ? bf(*dsum) : nullptr, scratch.data_ptr<float>(), R, C, blocks, stream_of(x)),
      "ln_bwd");
  count_launch(2);
}

int64_t op_colsum_scratch_floats(int64_t R, int64_t C) { return (int64_t)colsum_slabs((int)R) * C; }

// out[c] (+)= sum over rows of x[:, c] (bias gradient), fp32 accumulation.
void op_colsum(const at::Tensor& x, const at::Tensor& out, const at::Tensor& scratch, bool accumulate) {
  need_bf16(x, "x");
  need_bf16(out, "out");
  need_f32(scratch, "scratch");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "colsum: 2-D x with contiguous rows");
  const int R = x.size(0), C = x.size(1);
  TORCH_CHECK(out.numel() == C, "colsum: out must have C elements");
  TORCH_CHECK(scratch.numel() >= op_colsum_scratch_floats(R, C), "colsum: scratch too small");
  c10::cuda::CUDAGuard g(x.get_device());
  chk(colsum_bf16(bf(x), x.stride(0), R, C, bf(out), accumulate, scratch.data_ptr<float>(), stream_of(x)), "colsum");
  count_launch(2);
}

void op_gelu_fwd(const at::Tensor& x, const at::Tensor& y) {
  need_bf16(x, "x");
  need_bf16(y, "y");
  c10::cuda::CUDAGuard g(x.get_device());
  chk(gelu_fwd(bf(x), bf(y), x.numel(), stream_of(x)), "gelu_fwd");
  count_launch(1);
}
void op_gelu_bwd(const at::Tensor& x, const at::Tensor& dy, const at::Tensor& dx) {
  need_bf16(x, "x");
  need_bf16(dy, "dy");
  need_bf16(dx, "dx");
  c10::cuda::CUDAGuard g(x.get_device());
  chk(gelu_bwd(bf(x), bf(dy), bf(dx), x.numel(), stream_of(x)), "gelu_bwd");
  count_launch(1);
}
void op_swiglu_fwd(const at::Tensor& gu, const at::Tensor& y) {
  need_bf16(gu, "gu");
  need_bf16(y, "y");
  const int F = y.size(-1);
  const int R = y.numel() / F;
  TORCH_CHECK(gu.numel() == 2LL * R * F, "swiglu: gu must be [R, 2F]");
  c10::cuda::CUDAGuard g(gu.get_device());
  chk(swiglu_fwd(bf(gu), bf(y), R, F, stream_of(gu)), "swiglu_fwd");
  count_launch(1);
}
void op_swiglu_bwd(const at::Tensor& gu, const at::Tensor& dy, const at::Tensor& dgu) {
  need_bf16(gu, "gu");
  need_bf16(dy, "dy");
  need_bf16(dgu, "dgu");
  const int F = dy.size(-1);
  const int R = dy.numel() / F;
  c10::cuda::CUDAGuard g(gu.get_device());
  chk(swiglu_bwd(bf(gu), bf(dy), bf(dgu), R, F, stream_of(gu)), "swiglu_bwd");
  count_launch(1);
}

void op_xent(const at::Tensor& logits, const at::Tensor& targets, const at::Tensor& losses,
             const c10::optional<at::Tensor>& dlogits, int64_t V, double grad_scale) {
  need_bf16(logits, "logits");
  TORCH_CHECK(targets.scalar_type() == at::kLong && targets.is_contiguous(), "xent: targets must be int64");
  need_f32(losses, "losses");
  const int Vp = logits.size(-1);
  const int R = logits.numel() / Vp;
  TORCH_CHECK(targets.numel() == R && losses.numel() == R, "xent: one target/loss per row");
  c10::cuda::CUDAGuard g(logits.get_device());
  chk(xent_fwd_bwd(bf(logits), targets.data_ptr<int64_t>(), losses.data_ptr<float>(),
                   dlogits ? bf(*dlogits) : nullptr, R, (int)V, Vp, (float)grad_scale, stream_of(logits)),
      "xent");
  count_launch(1);
}

void op_embed_fwd(const at::Tensor& tok, const at::Tensor& wte, const at::Tensor& wpe, const at::Tensor& out,
                  int64_t T) {
  TORCH_CHECK(tok.scalar_type() == at::kLong && tok.is_contiguous(), "embed: tokens must be int64");
  need_bf16(wte, "wte");
  need_bf16(wpe, "wpe");
  need_bf16(out, "out");
  const int C = wte.size(-1);
  c10::cuda::CUDAGuard g(wte.get_device());
  chk(embed_fwd(tok.data_ptr<int64_t>(), bf(wte), bf(wpe), bf(out), tok.numel(), (int)T, C, stream_of(wte)),
      "embed_fwd");
  count_launch(1);
}
void op_embed_bwd(const at::Tensor& tok, const at::Tensor& dout, const at::Tensor& dwte, const at::Tensor& dwpe,
                  int64_t B, int64_t T) {
  need_bf16(dout, "dout");
  need_bf16(dwte, "dwte");
  need_bf16(dwpe, "dwpe");
  const int C = dout.size(-1);
  c10::cuda::CUDAGuard g(dout.get_device());
  chk(embed_bwd(tok.data_ptr<int64_t>(), bf(dout), bf(dwte), bf(dwpe), (int)B, (int)T, C, stream_of(dout)),
      "embed_bwd");
  count_launch(2);
}

int64_t op_grad_norm_blocks(int64_t n) { return grad_norm_blocks(n); }
void op_grad_norm_clip(const at::Tensor& g, double max_norm, const at::Tensor& scratch, const at::Tensor& counter,
                       const at::Tensor& norm_out, const at::Tensor& coef) {
  need_bf16(g, "grads");
  const int blocks = grad_norm_blocks(g.numel());
  TORCH_CHECK(scratch.numel() >= blocks, "grad_norm: scratch too small");
  c10::cuda::CUDAGuard gd(g.get_device());
  chk(grad_norm_clip(bf(g), g.numel(), (float)max_norm, scratch.data_ptr<float>(),
                     reinterpret_cast<unsigned int*>(counter.data_ptr()), norm_out.data_ptr<float>(),
                     coef.data_ptr<float>(), blocks, stream_of(g)),
      "grad_norm");
  count_launch(1);
}

void op_adamw(const at::Tensor& p, const at::Tensor& m, const at::Tensor& v, const at::Tensor& g,
              const at::Tensor& pb, int64_t decay_end, double lr, double b1, double b2, double eps, double wd,
              int64_t step, const c10::optional<at::Tensor>& gscale, const c10::optional<at::Tensor>& step_dev,
              const c10::optional<at::Tensor>& lr_dev) {
  need_f32(p, "param");
  need_f32(m, "exp_avg");
  need_f32(v, "exp_avg_sq");
  need_bf16(g, "grad");
  need_bf16(pb, "param_bf16");
  TORCH_CHECK(p.numel() == m.numel() && p.numel() == v.numel() && p.numel() == g.numel() && p.numel() == pb.numel(),
              "adamw: size mismatch");
  c10::cuda::CUDAGuard gd(p.get_device());
  chk(adamw_step(p.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), bf(g), bf(pb), p.numel(),
                 decay_end, (float)lr, (float)b1, (float)b2, (float)eps, (float)wd, (int)step,
                 gscale ? gscale->data_ptr<float>() : nullptr, step_dev ? step_dev->data_ptr<int>() : nullptr,
                 lr_dev ? lr_dev->data_ptr<float>() : nullptr, stream_of(p)),
      "adamw");
  count_launch(1);
}

void register_gemm_ops(py::module& m);
void register_ops(py::module& m) {
  register_gemm_ops(m);
  m.def("ln_fwd", &op_ln_fwd, py::arg("x"), py::arg("res"), py::arg("sum_out"), py::arg("w"), py::arg("b"),
        py::arg("y"), py::arg("mean"), py::arg("rstd"), py::arg("eps"), py::arg("rbias") = py::none());
  m.def("ln_bwd", &op_ln_bwd, py::arg("dy"), py::arg("x"), py::arg("mean"), py::arg("rstd"), py::arg("w"),
        py::arg("dres"), py::arg("dx"), py::arg("dw"), py::arg("db"), py::arg("scratch"), py::arg("counter"),
        py::arg("dsum") = py::none());
  m.def("ln_bwd_scratch_floats", &op_ln_bwd_scratch_floats, py::arg("R"), py::arg("C"), py::arg("dsum") = false);
  m.def("colsum", &op_colsum, py::arg("x"), py::arg("out"), py::arg("scratch"), py::arg("accumulate") = false);
  m.def("colsum_scratch_floats", &op_colsum_scratch_floats);
  m.def("gelu_fwd", &op_gelu_fwd);
  m.def("gelu_bwd", &op_gelu_bwd);
  m.def("swiglu_fwd", &op_swiglu_fwd);
  m.def("swiglu_bwd", &op_swiglu_bwd);
  m.def("xent", &op_xent);
  m.def("embed_fwd", &op_embed_fwd);
  m.def("embed_bwd", &op_embed_bwd);
  m.def("grad_norm_blocks", &op_grad_norm_blocks);
  m.def("grad_norm_clip", &op_grad_norm_clip);
  m.def("adamw", &op_adamw);
}

}  // namespace nexar

// ---------------------------------------------------------------- GEMM (tcgen05)
#include "gemm_api.h"
#include "compress_api.h"
#include "attention_api.h"
namespace nexar {
void op_gemm(const at::Tensor& A, const at::Tensor& B, const at::Tensor& C, const c10::optional<at::Tensor>& bias,
             const c10::optional<at::Tensor>& residual, const c10::optional<at::Tensor>& pre, int64_t act,
             double alpha) {
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && C.is_cuda(), "gemm: CUDA tensors required");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16 && C.scalar_type() == at::kBFloat16,
              "gemm: bf16 operands required");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && C.dim() == 2, "gemm: 2D operands required");
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1 && C.stride(1) == 1, "gemm: inner dimension must be contiguous");
  const int M = A.size(0), K = A.size(1), N = B.size(0);
  TORCH_CHECK(B.size(1) == K && C.size(0) == M && C.size(1) == N, "gemm: shape mismatch");
  c10::cuda::CUDAGuard g(A.get_device());
  const __nv_bfloat16* rp = residual ? reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr()) : nullptr;
  chk(gemm_bf16(reinterpret_cast<const __nv_bfloat16*>(A.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(B.data_ptr()),
                reinterpret_cast<__nv_bfloat16*>(C.data_ptr()), M, N, K, A.stride(0), B.stride(0), C.stride(0),
                bias ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr, rp,
                residual ? residual->stride(0) : 0, pre ? reinterpret_cast<__nv_bfloat16*>(pre->data_ptr()) : nullptr,
                (int)act, (float)alpha, stream_of(A)),
      "gemm");
  count_launch(1);
}
// C[M, N] = act(alpha * opA . opB^T + bias) (+ residual) (+ C if accumulate).
// a_mn: A is given as the stored [K, M] matrix (opA = A^T); b_mn: B is given
// as [K, N] (opB = B^T). ws: optional fp32 split-K workspace.
void op_gemm_ex(const at::Tensor& A, const at::Tensor& B, const at::Tensor& C, bool a_mn, bool b_mn,
                const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& residual,
                const c10::optional<at::Tensor>& pre, int64_t act, double alpha, bool accumulate, int64_t splits,
                const c10::optional<at::Tensor>& ws) {
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && C.is_cuda(), "gemm_ex: CUDA tensors required");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16 && C.scalar_type() == at::kBFloat16,
              "gemm_ex: bf16 operands required");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && C.dim() == 2, "gemm_ex: 2D operands required");
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1 && C.stride(1) == 1, "gemm_ex: inner dimension must be contiguous");
  const int M = a_mn ? A.size(1) : A.size(0);
  const int K = a_mn ? A.size(0) : A.size(1);
  const int N = b_mn ? B.size(1) : B.size(0);
  const int Kb = b_mn ? B.size(0) : B.size(1);
  TORCH_CHECK(Kb == K && C.size(0) == M && C.size(1) == N, "gemm_ex: shape mismatch");
  if (bias) TORCH_CHECK(bias->is_cuda() && bias->numel() == N && bias->scalar_type() == at::kBFloat16, "gemm_ex: bias");
  if (ws) TORCH_CHECK(ws->is_cuda() && ws->scalar_type() == at::kFloat && ws->is_contiguous(), "gemm_ex: fp32 ws");
  c10::cuda::CUDAGuard g(A.get_device());
  int sp = (int)splits;
  if (sp <= 0) sp = gemm_choose_splits(M, N, K);
  const size_t wsb = ws ? (size_t)ws->numel() * 4 : 0;
  if (sp > 1 && wsb < gemm_split_workspace_bytes(M, N, sp)) sp = 1;
  const cudaError_t err = gemm_bf16_ex(
      reinterpret_cast<const __nv_bfloat16*>(A.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(B.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(C.data_ptr()), M, N, K, A.stride(0), B.stride(0), C.stride(0), a_mn, b_mn,
      bias ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr,
      residual ? reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr()) : nullptr,
      residual ? residual->stride(0) : 0, pre ? reinterpret_cast<__nv_bfloat16*>(pre->data_ptr()) : nullptr, (int)act,
      (float)alpha, accumulate, sp, ws ? ws->data_ptr<float>() : nullptr, wsb, stream_of(A));
  const std::string what = std::string("gemm_ex [") + gemm_last_failure() + "; earlier error on this thread: " +
                           gemm_stale_error() + "] M=" + std::to_string(M) + " N=" + std::to_string(N) +
                           " K=" + std::to_string(K) + " a_t=" + std::to_string(a_mn) + " b_t=" + std::to_string(b_mn) +
                           " splits=" + std::to_string(sp);
  chk(err, what.c_str());
  count_launch(sp > 1 ? 2 : 1);
}

// fp8 e4m3 tensors travel as torch.float8_e4m3fn (or uint8) tensors.
static bool is_fp8_bytes(const at::Tensor& t) {
  return t.scalar_type() == at::kFloat8_e4m3fn || t.scalar_type() == at::kByte;
}

void op_quant_fp8_1x128(const at::Tensor& x, const at::Tensor& q, const at::Tensor& s) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1, "x: 2-D bf16");
  TORCH_CHECK(q.is_cuda() && is_fp8_bytes(q) && q.dim() == 2 && q.stride(1) == 1 && q.sizes() == x.sizes(), "q: e4m3 like x");
  const int R = x.size(0), K = x.size(1);
  TORCH_CHECK(s.is_cuda() && s.scalar_type() == at::kFloat && s.is_contiguous() && s.numel() == (int64_t)R * ((K + 127) / 128),
              "s: fp32 [R, ceil(K/128)]");
  c10::cuda::CUDAGuard g(x.get_device());
  chk(quant_fp8_1x128(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
                      reinterpret_cast<uint8_t*>(q.data_ptr()), q.stride(0), s.data_ptr<float>(), R, K, stream_of(x)),
      "quant_fp8_1x128");
  count_launch(1);
}

void op_quant_fp8_128x128(const at::Tensor& w, const at::Tensor& q, const at::Tensor& s) {
  TORCH_CHECK(w.is_cuda() && w.scalar_type() == at::kBFloat16 && w.dim() == 2 && w.stride(1) == 1, "w: 2-D bf16");
  TORCH_CHECK(q.is_cuda() && is_fp8_bytes(q) && q.dim() == 2 && q.stride(1) == 1 && q.sizes() == w.sizes(), "q: e4m3 like w");
  const int N = w.size(0), K = w.size(1);
  TORCH_CHECK(s.is_cuda() && s.scalar_type() == at::kFloat && s.is_contiguous() &&
                  s.numel() == (int64_t)((N + 127) / 128) * ((K + 127) / 128),
              "s: fp32 [ceil(N/128), ceil(K/128)]");
  c10::cuda::CUDAGuard g(w.get_device());
  chk(quant_fp8_128x128(reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), w.stride(0),
                        reinterpret_cast<uint8_t*>(q.data_ptr()), q.stride(0), s.data_ptr<float>(), N, K, stream_of(w)),
      "quant_fp8_128x128");
  count_launch(1);
}

// C[M, N] = act(alpha * blockscaled(A, sa) . blockscaled(B, sb)^T + bias)
void op_gemm_fp8(const at::Tensor& A, const at::Tensor& sa, const at::Tensor& B, const at::Tensor& sb,
                 const at::Tensor& C, const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& pre,
                 int64_t act, double alpha) {
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && C.is_cuda(), "gemm_fp8: CUDA tensors required");
  TORCH_CHECK(is_fp8_bytes(A) && is_fp8_bytes(B) && C.scalar_type() == at::kBFloat16, "gemm_fp8: e4m3 A/B, bf16 C");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && C.dim() == 2 && A.stride(1) == 1 && B.stride(1) == 1 && C.stride(1) == 1,
              "gemm_fp8: 2-D operands with contiguous rows");
  const int M = A.size(0), K = A.size(1), N = B.size(0);
  TORCH_CHECK(B.size(1) == K && C.size(0) == M && C.size(1) == N, "gemm_fp8: shape mismatch");
  const int kb = (K + 127) / 128;
  TORCH_CHECK(sa.scalar_type() == at::kFloat && sa.is_contiguous() && sa.numel() == (int64_t)M * kb, "gemm_fp8: sa [M, ceil(K/128)]");
  TORCH_CHECK(sb.scalar_type() == at::kFloat && sb.is_contiguous() && sb.numel() == (int64_t)((N + 127) / 128) * kb,
              "gemm_fp8: sb [ceil(N/128), ceil(K/128)]");
  c10::cuda::CUDAGuard g(A.get_device());
  chk(gemm_fp8_blockscaled(reinterpret_cast<const uint8_t*>(A.data_ptr()), sa.data_ptr<float>(),
                           reinterpret_cast<const uint8_t*>(B.data_ptr()), sb.data_ptr<float>(),
                           reinterpret_cast<__nv_bfloat16*>(C.data_ptr()), M, N, K, A.stride(0), B.stride(0), C.stride(0),
                           bias ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr, (int)act,
                           pre ? reinterpret_cast<__nv_bfloat16*>(pre->data_ptr()) : nullptr, (float)alpha, stream_of(A)),
      "gemm_fp8");
  count_launch(1);
}

void op_swiglu_quant_fp8(const at::Tensor& gu, const at::Tensor& q, const at::Tensor& s) {
  TORCH_CHECK(gu.is_cuda() && gu.scalar_type() == at::kBFloat16 && gu.dim() == 2 && gu.is_contiguous(), "gu: [R, 2F] bf16");
  const int R = gu.size(0), F = gu.size(1) / 2;
  TORCH_CHECK(q.is_cuda() && is_fp8_bytes(q) && q.is_contiguous() && q.numel() == (int64_t)R * F, "q: e4m3 [R, F]");
  TORCH_CHECK(s.is_cuda() && s.scalar_type() == at::kFloat && s.is_contiguous() && s.numel() == (int64_t)R * ((F + 127) / 128),
              "s: fp32 [R, ceil(F/128)]");
  c10::cuda::CUDAGuard g(gu.get_device());
  chk(swiglu_quant_fp8_1x128(reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()), reinterpret_cast<uint8_t*>(q.data_ptr()),
                             s.data_ptr<float>(), R, F, stream_of(gu)),
      "swiglu_quant_fp8");
  count_launch(1);
}

void register_gemm_ops(py::module& m) {
  m.def("swiglu_quant_fp8", &op_swiglu_quant_fp8);
  m.def("quant_fp8_1x128", &op_quant_fp8_1x128);
  m.def("quant_fp8_128x128", &op_quant_fp8_128x128);
  m.def("gemm_fp8", &op_gemm_fp8, py::arg("A"), py::arg("sa"), py::arg("B"), py::arg("sb"), py::arg("C"),
        py::arg("bias") = py::none(), py::arg("pre") = py::none(), py::arg("act") = 0, py::arg("alpha") = 1.0);
  m.def("gemm_ex", &op_gemm_ex, py::arg("A"), py::arg("B"), py::arg("C"), py::arg("a_t") = false,
        py::arg("b_t") = false, py::arg("bias") = py::none(), py::arg("residual") = py::none(),
        py::arg("pre") = py::none(), py::arg("act") = 0, py::arg("alpha") = 1.0, py::arg("accumulate") = false,
        py::arg("splits") = 1, py::arg("ws") = py::none());
  m.def("gemm_choose_splits", &gemm_choose_splits);
  m.def("gemm_set_2sm", &gemm_set_2sm);
  m.def("gemm_get_2sm", &gemm_get_2sm);
  m.def("gemm_split_workspace_bytes",
        [](int64_t M, int64_t N, int64_t sp) { return (int64_t)gemm_split_workspace_bytes(M, N, sp); });
  m.def("gemm", &op_gemm, py::arg("A"), py::arg("B"), py::arg("C"), py::arg("bias") = py::none(),
        py::arg("residual") = py::none(), py::arg("pre") = py::none(), py::arg("act") = 0, py::arg("alpha") = 1.0);
  m.def("gemm_error_flag", &gemm_error_flag);
  m.def("compress_workspace_bytes", [](int64_t n) { return (int64_t)compress_workspace_bytes(n, nullptr); });
  m.def("compress_blob_bytes", [](int64_t k) { return (int64_t)((compress_blob_bytes(k) + 15) / 16 * 16); });
  m.def("topk_fp8_compress", [](const at::Tensor& grad, const at::Tensor& residual, int64_t k, const at::Tensor& blob,
                                const at::Tensor& ws) {
    TORCH_CHECK(grad.is_cuda() && grad.is_contiguous() && grad.scalar_type() == at::kBFloat16, "grad: contiguous bf16");
    TORCH_CHECK(residual.is_cuda() && residual.is_contiguous() && residual.scalar_type() == at::kFloat &&
                    residual.numel() == grad.numel(), "residual: contiguous fp32 like grad");
    TORCH_CHECK(blob.numel() * blob.element_size() >= (int64_t)compress_blob_bytes(k), "blob too small");
    TORCH_CHECK(ws.numel() * ws.element_size() >= (int64_t)compress_workspace_bytes(grad.numel(), nullptr),
                "workspace too small");
    c10::cuda::CUDAGuard g(grad.get_device());
    chk(topk_fp8_compress(reinterpret_cast<const __nv_bfloat16*>(grad.data_ptr()), residual.data_ptr<float>(),
                          grad.numel(), k, reinterpret_cast<unsigned char*>(blob.data_ptr()), ws.data_ptr(),
                          stream_of(grad)),
        "topk_fp8_compress");
    count_launch(compress_kernel_launches());
  });
  m.def("decompress_accumulate", [](const at::Tensor& blob, int64_t k, const at::Tensor& out, double scale) {
    need_bf16(out, "out");
    c10::cuda::CUDAGuard g(out.get_device());
    chk(decompress_accumulate(reinterpret_cast<const unsigned char*>(blob.data_ptr()), k, bf(out), (float)scale,
                              stream_of(out)),
        "decompress_accumulate");
    count_launch(1);
  });
  // ---- self-attention (head dimension 64, tcgen05): qkv [B*T, 3C] -> y [B*T, C]
  m.def("attn_supported", [](int64_t B, int64_t T, int64_t H, int64_t hd) {
    return attention_supported((int)B, (int)T, (int)H, (int)hd);
  });
  m.def("attn_trace_select", [](int64_t cta) { chk(attention_trace_select((int)cta), "attn_trace_select"); });
  m.def("attn_trace_read", []() {
    at::Tensor out = at::empty({4096}, at::TensorOptions().dtype(at::kLong));
    chk(attention_trace_read(reinterpret_cast<unsigned long long*>(out.data_ptr<int64_t>()), 4096),
        "attn_trace_read");
    return out;
  });
  m.def("attn_bwd_workspace_floats", [](int64_t B, int64_t T, int64_t H) {
    return (int64_t)attention_bwd_workspace_floats((int)B, (int)T, (int)H);
  });
  m.def("attn_fwd", [](const at::Tensor& qkv, const at::Tensor& y, const at::Tensor& lse, int64_t B, int64_t T,
                       int64_t H, bool causal) {
    need_bf16(qkv, "qkv");
    need_bf16(y, "y");
    need_f32(lse, "lse");
    TORCH_CHECK(attention_supported((int)B, (int)T, (int)H, 64), "attn_fwd: needs head dim 64 and T % 128 == 0");
    const int64_t C = H * 64;
    TORCH_CHECK(qkv.numel() == B * T * 3 * C && y.numel() == B * T * C && lse.numel() == B * H * T,
                "attn_fwd: shape mismatch");
    c10::cuda::CUDAGuard g(qkv.get_device());
    chk(attention_fwd(bf(qkv), bf(y), lse.data_ptr<float>(), (int)B, (int)T, (int)H, causal, stream_of(qkv)),
        "attn_fwd");
    count_launch(1);
  });
  m.def("attn_bwd", [](const at::Tensor& qkv, const at::Tensor& y, const at::Tensor& dy, const at::Tensor& lse,
                       const at::Tensor& dqkv, const at::Tensor& ws, int64_t B, int64_t T, int64_t H, bool causal) {
    need_bf16(qkv, "qkv");
    need_bf16(y, "y");
    need_bf16(dy, "dy");
    need_bf16(dqkv, "dqkv");
    need_f32(lse, "lse");
    need_f32(ws, "ws");
    TORCH_CHECK(attention_supported((int)B, (int)T, (int)H, 64), "attn_bwd: needs head dim 64 and T % 128 == 0");
    const int64_t C = H * 64;
    TORCH_CHECK(qkv.numel() == B * T * 3 * C && dqkv.numel() == qkv.numel() && y.numel() == B * T * C &&
                    dy.numel() == y.numel() && lse.numel() == B * H * T,
                "attn_bwd: shape mismatch");
    TORCH_CHECK(ws.numel() >= (int64_t)attention_bwd_workspace_floats((int)B, (int)T, (int)H),
                "attn_bwd: workspace too small");
    c10::cuda::CUDAGuard g(qkv.get_device());
    chk(attention_bwd(bf(qkv), bf(y), bf(dy), lse.data_ptr<float>(), bf(dqkv), ws.data_ptr<float>(), (int)B,
                      (int)T, (int)H, causal, stream_of(qkv)),
        "attn_bwd");
    count_launch(3);
  });
}
}  // namespace nexar
