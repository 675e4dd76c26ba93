// PyTorch bindings of the device runtime (module nexar_b200._cuda).
//
// Every entry point validates shapes and dtypes, splits messages that exceed
// the staging slot into slot-sized pieces, and launches on the caller's
// current CUDA stream.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <atomic>
#include <memory>

#include "coll_api.h"
#include "device_comm.h"
#include "ops_api.h"
#include "gemm_api.h"
#include "moe_api.h"
#include "nvls_api.h"

namespace nexar {

std::atomic<unsigned long long> g_launches{0};
void count_launch(unsigned long long n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

int dtype_code(at::ScalarType t) {
  switch (t) {
    case at::kFloat: return kF32;
    case at::kDouble: return kF64;
    case at::kHalf: return kF16;
    case at::kBFloat16: return kBF16;
    case at::kChar: return kI8;
    case at::kInt: return kI32;
    case at::kLong: return kI64;
    case at::kByte: return kU8;
    case at::kUInt32: return kU32;
    case at::kUInt64: return kU64;
    case at::kFloat8_e4m3fn: return kF8E4M3;
    case at::kFloat8_e5m2: return kF8E5M2;
    default: TORCH_CHECK(false, "nexar_b200: unsupported dtype ", t);
  }
}

at::ScalarType scalar_type_of(int code) {
  switch (code) {
    case kF32: return at::kFloat;
    case kF64: return at::kDouble;
    case kF16: return at::kHalf;
    case kBF16: return at::kBFloat16;
    case kI8: return at::kChar;
    case kI32: return at::kInt;
    case kI64: return at::kLong;
    case kU8: return at::kByte;
    case kU32: return at::kUInt32;
    case kU64: return at::kUInt64;
    case kF8E4M3: return at::kFloat8_e4m3fn;
    case kF8E5M2: return at::kFloat8_e5m2;
    default: TORCH_CHECK(false, "nexar_b200: unknown dtype code ", code);
  }
}

static void check_dev_tensor(const DeviceComm& c, const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), "nexar_b200: ", name, " must be a CUDA tensor");
  TORCH_CHECK(t.get_device() == c.device(), "nexar_b200: ", name, " is on cuda:", t.get_device(),
              " but the communicator is on cuda:", c.device());
  TORCH_CHECK(t.is_contiguous(), "nexar_b200: ", name, " must be contiguous");
}

static void check_launch(cudaError_t e, const char* what) {
  TORCH_CHECK(e == cudaSuccess, "nexar_b200: ", what, " launch failed: ", cudaGetErrorString(e));
}

static cudaStream_t cur_stream(const DeviceComm& c) {
  return at::cuda::getCurrentCUDAStream(c.device()).stream();
}

static unsigned long long round_down(unsigned long long v, unsigned long long m) { return v / m * m; }

using CommPtr = std::shared_ptr<DeviceComm>;

// ---------------------------------------------------------------- collectives
void all_reduce(const CommPtr& c, const at::Tensor& in, const at::Tensor& out, int op, double scale,
                int algo, long long oneshot_max_bytes) {
  check_dev_tensor(*c, in, "input");
  check_dev_tensor(*c, out, "output");
  TORCH_CHECK(in.numel() == out.numel(), "all_reduce: input and output sizes differ");
  TORCH_CHECK(c->connected(), "communicator is not connected");
  c10::cuda::CUDAGuard g(c->device());
  const int dti = dtype_code(in.scalar_type()), dto = dtype_code(out.scalar_type());
  const unsigned long long n = in.numel();
  const int esi = in.element_size(), eso = out.element_size();
  const unsigned long long bytes = n * esi;
  if (n == 0) return;
  cudaStream_t s = cur_stream(*c);
  if (c->world() == 1) {
    // A single rank: the result is the (scaled, cast) input.
    check_launch(launch_all_reduce(c->dev(), in.data_ptr(), out.data_ptr(), dti, dto, op, n,
                                   (float)scale, kAlgoOneShot, -1, c->max_blocks, s), "all_reduce");
    count_launch(1);
    c->last_allreduce_algo = 0;
    return;
  }
  // NVLS (switch-side reduction) for large messages; in place with no staging
  // when the tensor lives in the NVLS region.
  const bool nvls_ok = dti == dto && nvls_can_reduce(c->dev(), dti, op, in.data_ptr(), out.data_ptr(), bytes);
  const long long noff = in.data_ptr() == out.data_ptr() ? c->nvls_offset(in.data_ptr(), bytes) : -1;
  const uint64_t nvls_from = noff >= 0 ? (256ull << 10) : c->nvls_min_bytes;  // in place: no copies to amortise
  if (nvls_ok && (algo == kAlgoNvls || (algo == kAlgoAuto && bytes >= nvls_from))) {
    check_launch(launch_all_reduce_nvls(c->dev(), in.data_ptr(), out.data_ptr(), dti, bytes, (float)scale, noff,
                                        c->max_blocks, s),
                 "all_reduce(nvls)");
    count_launch(1);
    c->last_allreduce_algo = noff >= 0 ? 4 : 3;
    return;
  }
  TORCH_CHECK(algo != kAlgoNvls, "all_reduce: NVLS path unavailable for this message (needs an active NVLS region, "
              "Sum of f32/bf16/f16, 16-byte aligned sizes and pointers)");
  long long sym = -1;
  if (algo == kAlgoAuto) algo = (long long)bytes <= oneshot_max_bytes ? kAlgoOneShot : kAlgoTwoShot;
  // Zero-copy in place only for two-shot: there rank r alone reads and writes
  // chunk r. A one-shot rank would overwrite its input while peers still read
  // it, so one-shot always goes through the staging slot.
  if (in.data_ptr() == out.data_ptr() && dti == dto && algo == kAlgoTwoShot)
    sym = c->symmetric_offset(in.data_ptr(), bytes);
  if (sym >= 0) {
    check_launch(launch_all_reduce(c->dev(), in.data_ptr(), out.data_ptr(), dti, dto, op, n,
                                   (float)scale, algo, sym, c->max_blocks, s), "all_reduce");
    count_launch(1);
    c->last_allreduce_algo = 5;
    return;
  }
  c->last_allreduce_algo = algo == kAlgoOneShot ? 1 : 2;
  const unsigned long long per = round_down(c->slot_bytes() / std::max(esi, eso), 256);
  for (unsigned long long off = 0; off < n; off += per) {
    const unsigned long long m = std::min(per, n - off);
    check_launch(launch_all_reduce(c->dev(), (const char*)in.data_ptr() + off * esi,
                                   (char*)out.data_ptr() + off * eso, dti, dto, op, m, (float)scale,
                                   algo, -1, c->max_blocks, s),
                 "all_reduce");
    count_launch(1);
  }
}

void reduce_scatter(const CommPtr& c, const at::Tensor& in, const at::Tensor& out, int op,
                    double scale) {
  check_dev_tensor(*c, in, "input");
  check_dev_tensor(*c, out, "output");
  const int N = c->world();
  TORCH_CHECK(in.numel() == out.numel() * N, "reduce_scatter: input must hold world_size * output elements");
  c10::cuda::CUDAGuard g(c->device());
  const int dti = dtype_code(in.scalar_type()), dto = dtype_code(out.scalar_type());
  const unsigned long long count = out.numel();
  const int esi = in.element_size(), eso = out.element_size();
  cudaStream_t s = cur_stream(*c);
  const long long in_sym = c->nvls_offset(in.data_ptr(), count * esi * N);
  if (dti == dto && N > 1 && (in_sym >= 0 || count * esi * N >= c->nvls_min_rs_bytes) &&
      nvls_can_reduce(c->dev(), dti, op, in.data_ptr(), out.data_ptr(), count * esi)) {
    check_launch(launch_reduce_scatter_nvls(c->dev(), in.data_ptr(), out.data_ptr(), dti, count * esi, (float)scale,
                                            in_sym, c->max_blocks, s),
                 "reduce_scatter(nvls)");
    count_launch(1);
    return;
  }
  const unsigned long long per = round_down(c->slot_bytes() / ((unsigned long long)N * std::max(esi, eso)), 256);
  for (unsigned long long off = 0; off < count; off += per) {
    const unsigned long long m = std::min(per, count - off);
    check_launch(launch_reduce_scatter(c->dev(), (const char*)in.data_ptr() + off * esi,
                                       (char*)out.data_ptr() + off * eso, dti, dto, op, m, count,
                                       (float)scale, c->max_blocks, s),
                 "reduce_scatter");
    count_launch(1);
  }
}

void all_gather(const CommPtr& c, const at::Tensor& in, const at::Tensor& out) {
  check_dev_tensor(*c, in, "input");
  check_dev_tensor(*c, out, "output");
  const int N = c->world();
  TORCH_CHECK(out.numel() == in.numel() * N, "all_gather: output must hold world_size * input elements");
  TORCH_CHECK(in.scalar_type() == out.scalar_type(), "all_gather: dtype mismatch");
  c10::cuda::CUDAGuard g(c->device());
  const int dt = dtype_code(in.scalar_type());
  const unsigned long long count = in.numel();
  const int es = in.element_size();
  cudaStream_t s = cur_stream(*c);
  const long long out_sym = c->nvls_offset(out.data_ptr(), count * es * N);
  if (N > 1 && (out_sym >= 0 || count * es * N >= c->nvls_min_ag_bytes) &&
      nvls_can_move(c->dev(), in.data_ptr(), out.data_ptr(), count * es)) {
    check_launch(launch_all_gather_nvls(c->dev(), in.data_ptr(), out.data_ptr(), count * es, out_sym, c->max_blocks, s),
                 "all_gather(nvls)");
    count_launch(1);
    return;
  }
  const unsigned long long per = round_down(c->slot_bytes() / es, 256);
  for (unsigned long long off = 0; off < count; off += per) {
    const unsigned long long m = std::min(per, count - off);
    check_launch(launch_all_gather(c->dev(), (const char*)in.data_ptr() + off * es,
                                   (char*)out.data_ptr() + off * es, dt, m, count, c->max_blocks, s),
                 "all_gather");
    count_launch(1);
  }
}

void all_to_all(const CommPtr& c, const at::Tensor& in, const at::Tensor& out) {
  check_dev_tensor(*c, in, "input");
  check_dev_tensor(*c, out, "output");
  const int N = c->world();
  TORCH_CHECK(in.numel() == out.numel() && in.numel() % N == 0,
              "all_to_all: input and output must both hold world_size * count elements");
  TORCH_CHECK(in.scalar_type() == out.scalar_type(), "all_to_all: dtype mismatch");
  c10::cuda::CUDAGuard g(c->device());
  const int dt = dtype_code(in.scalar_type());
  const unsigned long long count = in.numel() / N;
  const int es = in.element_size();
  const unsigned long long per = round_down(c->slot_bytes() / ((unsigned long long)N * es), 256);
  cudaStream_t s = cur_stream(*c);
  for (unsigned long long off = 0; off < count; off += per) {
    const unsigned long long m = std::min(per, count - off);
    check_launch(launch_all_to_all(c->dev(), (const char*)in.data_ptr() + off * es,
                                   (char*)out.data_ptr() + off * es, dt, m, count, count,
                                   c->max_blocks, s),
                 "all_to_all");
    count_launch(1);
  }
}

void broadcast(const CommPtr& c, const at::Tensor& in, const at::Tensor& out, int root) {
  check_dev_tensor(*c, in, "input");
  check_dev_tensor(*c, out, "output");
  TORCH_CHECK(in.numel() == out.numel() && in.scalar_type() == out.scalar_type(), "broadcast: shape/dtype mismatch");
  TORCH_CHECK(root >= 0 && root < c->world(), "broadcast: root out of range");
  c10::cuda::CUDAGuard g(c->device());
  const int dt = dtype_code(in.scalar_type());
  const unsigned long long n = in.numel();
  const int es = in.element_size();
  cudaStream_t s = cur_stream(*c);
  // Every rank must pass an NVLS-resident output, or none (same path on all ranks).
  const long long out_sym = c->nvls_offset(out.data_ptr(), n * es);
  if (c->world() > 1 && (out_sym >= 0 || n * es >= c->nvls_min_bcast_bytes) &&
      nvls_can_move(c->dev(), in.data_ptr(), out.data_ptr(), n * es)) {
    check_launch(launch_broadcast_nvls(c->dev(), in.data_ptr(), out.data_ptr(), n * es, root, out_sym, c->max_blocks, s),
                 "broadcast(nvls)");
    count_launch(1);
    return;
  }
  const unsigned long long per = round_down(c->slot_bytes() / es, 256);
  for (unsigned long long off = 0; off < n; off += per) {
    const unsigned long long m = std::min(per, n - off);
    check_launch(launch_broadcast(c->dev(), (const char*)in.data_ptr() + off * es,
                                  (char*)out.data_ptr() + off * es, dt, m, root, c->max_blocks, s),
                 "broadcast");
    count_launch(1);
  }
}

void reduce(const CommPtr& c, const at::Tensor& in, const at::Tensor& out, int root, int op,
            double scale) {
  check_dev_tensor(*c, in, "input");
  check_dev_tensor(*c, out, "output");
  TORCH_CHECK(in.numel() == out.numel(), "reduce: size mismatch");
  TORCH_CHECK(root >= 0 && root < c->world(), "reduce: root out of range");
  c10::cuda::CUDAGuard g(c->device());
  const int dti = dtype_code(in.scalar_type()), dto = dtype_code(out.scalar_type());
  const unsigned long long n = in.numel();
  const int esi = in.element_size(), eso = out.element_size();
  const unsigned long long per = round_down(c->slot_bytes() / std::max(esi, eso), 256);
  cudaStream_t s = cur_stream(*c);
  for (unsigned long long off = 0; off < n; off += per) {
    const unsigned long long m = std::min(per, n - off);
    check_launch(launch_reduce(c->dev(), (const char*)in.data_ptr() + off * esi,
                               (char*)out.data_ptr() + off * eso, dti, dto, op, m, root,
                               (float)scale, c->max_blocks, s),
                 "reduce");
    count_launch(1);
  }
}

void gather(const CommPtr& c, const at::Tensor& in, const at::Tensor& out, int root) {
  check_dev_tensor(*c, in, "input");
  check_dev_tensor(*c, out, "output");
  const int N = c->world();
  TORCH_CHECK(out.numel() == in.numel() * N, "gather: output must hold world_size * input elements");
  TORCH_CHECK(in.scalar_type() == out.scalar_type(), "gather: dtype mismatch");
  TORCH_CHECK(root >= 0 && root < N, "gather: root out of range");
  c10::cuda::CUDAGuard g(c->device());
  const int dt = dtype_code(in.scalar_type());
  const unsigned long long count = in.numel();
  const int es = in.element_size();
  const unsigned long long per = round_down(c->slot_bytes() / es, 256);
  cudaStream_t s = cur_stream(*c);
  for (unsigned long long off = 0; off < count; off += per) {
    const unsigned long long m = std::min(per, count - off);
    check_launch(launch_gather(c->dev(), (const char*)in.data_ptr() + off * es,
                               (char*)out.data_ptr() + off * es, dt, m, count, root, c->max_blocks, s),
                 "gather");
    count_launch(1);
  }
}

void scatter(const CommPtr& c, const at::Tensor& in, const at::Tensor& out, int root) {
  check_dev_tensor(*c, in, "input");
  check_dev_tensor(*c, out, "output");
  const int N = c->world();
  TORCH_CHECK(in.numel() == out.numel() * N, "scatter: input must hold world_size * output elements");
  TORCH_CHECK(in.scalar_type() == out.scalar_type(), "scatter: dtype mismatch");
  TORCH_CHECK(root >= 0 && root < N, "scatter: root out of range");
  c10::cuda::CUDAGuard g(c->device());
  const int dt = dtype_code(in.scalar_type());
  const unsigned long long count = out.numel();
  const int es = in.element_size();
  const unsigned long long per = round_down(c->slot_bytes() / ((unsigned long long)N * es), 256);
  cudaStream_t s = cur_stream(*c);
  for (unsigned long long off = 0; off < count; off += per) {
    const unsigned long long m = std::min(per, count - off);
    check_launch(launch_scatter(c->dev(), (const char*)in.data_ptr() + off * es,
                                (char*)out.data_ptr() + off * es, dt, m, count, root, c->max_blocks, s),
                 "scatter");
    count_launch(1);
  }
}

void scan(const CommPtr& c, const at::Tensor& in, const at::Tensor& out, int op, bool exclusive) {
  check_dev_tensor(*c, in, "input");
  check_dev_tensor(*c, out, "output");
  TORCH_CHECK(in.numel() == out.numel() && in.scalar_type() == out.scalar_type(), "scan: shape/dtype mismatch");
  c10::cuda::CUDAGuard g(c->device());
  const int dt = dtype_code(in.scalar_type());
  const unsigned long long n = in.numel();
  const int es = in.element_size();
  const unsigned long long per = round_down(c->slot_bytes() / es, 256);
  cudaStream_t s = cur_stream(*c);
  for (unsigned long long off = 0; off < n; off += per) {
    const unsigned long long m = std::min(per, n - off);
    check_launch(launch_scan(c->dev(), (const char*)in.data_ptr() + off * es,
                             (char*)out.data_ptr() + off * es, dt, op, m, exclusive, c->max_blocks, s),
                 "scan");
    count_launch(1);
  }
}

void barrier(const CommPtr& c) {
  c10::cuda::CUDAGuard g(c->device());
  check_launch(launch_barrier(c->dev(), cur_stream(*c)), "barrier");
  count_launch(1);
}

void reduce_inplace(const at::Tensor& dst, const at::Tensor& src, int op) {
  TORCH_CHECK(dst.is_cuda() && src.is_cuda() && dst.is_contiguous() && src.is_contiguous(),
              "reduce_inplace: contiguous CUDA tensors required");
  TORCH_CHECK(dst.numel() == src.numel() && dst.scalar_type() == src.scalar_type(),
              "reduce_inplace: shape/dtype mismatch");
  c10::cuda::CUDAGuard g(dst.get_device());
  check_launch(launch_reduce_inplace(dst.data_ptr(), src.data_ptr(), dtype_code(dst.scalar_type()), op,
                                     dst.numel(), at::cuda::getCurrentCUDAStream().stream()),
               "reduce_inplace");
  count_launch(1);
}

at::Tensor symmetric_tensor(const CommPtr& c, unsigned long long offset, std::vector<int64_t> shape,
                            int dtype) {
  at::ScalarType st = scalar_type_of(dtype);
  int64_t numel = 1;
  for (auto d : shape) numel *= d;
  TORCH_CHECK(offset + numel * c10::elementSize(st) <= c->heap_bytes(), "symmetric_tensor out of heap range");
  CommPtr keep = c;
  auto opts = at::TensorOptions().dtype(st).device(at::kCUDA, c->device());
  return torch::from_blob(c->local_base() + offset, shape, [keep](void*) {}, opts);
}

at::Tensor nvls_tensor(const CommPtr& c, unsigned long long offset, std::vector<int64_t> shape, int dtype) {
  TORCH_CHECK(c->nvls_active(), "nvls_tensor: NVLS region not active");
  at::ScalarType st = scalar_type_of(dtype);
  int64_t numel = 1;
  for (auto d : shape) numel *= d;
  TORCH_CHECK(offset + numel * c10::elementSize(st) <= c->nvls_bytes(), "nvls_tensor out of region range");
  CommPtr keep = c;
  auto opts = at::TensorOptions().dtype(st).device(at::kCUDA, c->device());
  return torch::from_blob(c->nvls_local() + offset, shape, [keep](void*) {}, opts);
}

py::dict status_dict(const CommPtr& c) {
  DeviceStatus s = c->status();
  py::dict d;
  d["code"] = s.code;
  d["rank"] = s.rank;
  d["op"] = s.op;
  d["block"] = s.block;
  d["epoch"] = s.epoch;
  return d;
}

// ---------------------------------------------------------------- fused GEMM + collective
static const __nv_bfloat16* cbf(const at::Tensor& t) { return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr()); }
static __nv_bfloat16* mbf(const at::Tensor& t) { return reinterpret_cast<__nv_bfloat16*>(t.data_ptr()); }
static void need_bf16_2d(const at::Tensor& t, const char* n) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 2 && t.stride(1) == 1, "nexar_b200: ", n,
              " must be a 2D bf16 CUDA tensor with contiguous rows");
}

void gemm_rs(const CommPtr& c, const at::Tensor& A, const at::Tensor& B, const at::Tensor& out,
             const c10::optional<at::Tensor>& bias, double alpha) {
  need_bf16_2d(A, "A");
  need_bf16_2d(B, "B");
  need_bf16_2d(out, "out");
  const int M = A.size(0), K = A.size(1), N = B.size(0);
  TORCH_CHECK(B.size(1) == K && out.size(0) * c->world() == M && out.size(1) == N, "gemm_reduce_scatter: shape mismatch");
  c10::cuda::CUDAGuard g(c->device());
  check_launch(gemm_reduce_scatter(c->dev(), cbf(A), cbf(B), mbf(out), M, N, K, A.stride(0), B.stride(0), out.stride(0),
                                   bias ? cbf(*bias) : nullptr, (float)alpha, c->rs_maps(M, N), cur_stream(*c)),
               "gemm_reduce_scatter");
  count_launch(1);
}

void gemm_fp8_rs(const CommPtr& c, const at::Tensor& A, const at::Tensor& sa, const at::Tensor& B, const at::Tensor& sb,
                 const at::Tensor& out, const c10::optional<at::Tensor>& bias, double alpha) {
  auto fp8 = [](const at::Tensor& t) { return t.scalar_type() == at::kFloat8_e4m3fn || t.scalar_type() == at::kByte; };
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && fp8(A) && fp8(B) && A.dim() == 2 && B.dim() == 2 && A.stride(1) == 1 &&
                  B.stride(1) == 1, "gemm_fp8_reduce_scatter: 2-D e4m3 A and B");
  need_bf16_2d(out, "out");
  const int M = A.size(0), K = A.size(1), N = B.size(0);
  TORCH_CHECK(B.size(1) == K && out.size(0) * c->world() == M && out.size(1) == N, "gemm_fp8_reduce_scatter: shape mismatch");
  const int kb = (K + 127) / 128;
  TORCH_CHECK(sa.scalar_type() == at::kFloat && sa.is_contiguous() && sa.numel() == (int64_t)M * kb, "sa [M, ceil(K/128)]");
  TORCH_CHECK(sb.scalar_type() == at::kFloat && sb.is_contiguous() && sb.numel() == (int64_t)((N + 127) / 128) * kb,
              "sb [ceil(N/128), ceil(K/128)]");
  c10::cuda::CUDAGuard g(c->device());
  check_launch(gemm_fp8_reduce_scatter(c->dev(), reinterpret_cast<const uint8_t*>(A.data_ptr()), sa.data_ptr<float>(),
                                       reinterpret_cast<const uint8_t*>(B.data_ptr()), sb.data_ptr<float>(), mbf(out), M,
                                       N, K, A.stride(0), B.stride(0), out.stride(0), bias ? cbf(*bias) : nullptr,
                                       (float)alpha, c->rs_maps(M, N), cur_stream(*c)),
               "gemm_fp8_reduce_scatter");
  count_launch(1);
}

void ag_gemm(const CommPtr& c, const at::Tensor& x, const at::Tensor& B, const at::Tensor& out, const at::Tensor& afull,
             const at::Tensor& cnt, const c10::optional<at::Tensor>& bias, int act, const c10::optional<at::Tensor>& pre,
             double alpha) {
  need_bf16_2d(x, "x");
  need_bf16_2d(B, "B");
  need_bf16_2d(out, "out");
  TORCH_CHECK(afull.is_cuda() && afull.is_contiguous() && afull.scalar_type() == at::kBFloat16, "afull workspace");
  TORCH_CHECK(cnt.is_cuda() && cnt.is_contiguous() && cnt.element_size() == 4, "cnt workspace");
  const int W = c->world();
  const int M = x.size(0) * W, K = x.size(1), N = B.size(0);
  TORCH_CHECK(B.size(1) == K && out.size(0) == M && out.size(1) == N && afull.numel() >= (int64_t)M * K,
              "all_gather_gemm: shape mismatch");
  TORCH_CHECK(cnt.numel() >= M / 128 + 2, "all_gather_gemm: cnt too small");
  c10::cuda::CUDAGuard g(c->device());
  check_launch(all_gather_gemm(c->dev(), cbf(x), x.stride(0), cbf(B), mbf(out), mbf(afull),
                               reinterpret_cast<unsigned int*>(cnt.data_ptr()), M, N, K, B.stride(0), out.stride(0),
                               bias ? cbf(*bias) : nullptr, act, pre ? mbf(*pre) : nullptr, (float)alpha,
                               cur_stream(*c)),
               "all_gather_gemm");
  count_launch(1);
}

#include "bindings_moe.inc"

void register_ops(py::module& m);

}  // namespace nexar

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  using namespace nexar;
  m.doc() = "nexar_b200 device runtime: symmetric heap, peer-memory collectives, fused kernels (sm_100a)";
  py::class_<DeviceComm, std::shared_ptr<DeviceComm>>(m, "DeviceComm")
      .def(py::init<int, int, int, uint64_t, uint64_t, uint64_t>(), py::arg("rank"), py::arg("world"),
           py::arg("device"), py::arg("heap_bytes"), py::arg("slot_bytes"), py::arg("timeout_us"))
      .def("export_handle", [](const DeviceComm& c) { return py::bytes(c.export_handle()); })
      .def("connect", [](DeviceComm& c, const std::vector<py::bytes>& hs) {
        std::vector<std::string> v;
        for (auto& h : hs) v.push_back(std::string(h));
        c.connect(v);
      })
      .def("alloc_symmetric", &DeviceComm::alloc_symmetric, py::arg("bytes"), py::arg("align") = 256)
      .def("reset_symmetric", &DeviceComm::reset_symmetric)
      .def("symmetric_offset", [](const DeviceComm& c, const at::Tensor& t) {
        return c.symmetric_offset(t.data_ptr(), t.numel() * t.element_size());
      })
      .def("status", &status_dict)
      .def("clear_status", &DeviceComm::clear_status)
      .def_property_readonly("rank", &DeviceComm::rank)
      .def_property_readonly("world", &DeviceComm::world)
      .def_property_readonly("device", &DeviceComm::device)
      .def_property_readonly("heap_bytes", &DeviceComm::heap_bytes)
      .def_property_readonly("slot_bytes", &DeviceComm::slot_bytes)
      .def_property_readonly("user_bytes_free", &DeviceComm::user_bytes_free)
      .def_property_readonly("connected", &DeviceComm::connected)
      .def_property("timeout_us", &DeviceComm::timeout_us, &DeviceComm::set_timeout_us)
      .def_readwrite("max_blocks", &DeviceComm::max_blocks)
      .def_property("checks", &DeviceComm::checks, &DeviceComm::set_checks)
      .def("debug_set_call_counter", &DeviceComm::debug_set_call_counter)
      .def("debug_broadcast_raw_root", [](DeviceComm& c, const at::Tensor& in, const at::Tensor& out, int root) {
        TORCH_CHECK(in.is_cuda() && out.is_cuda() && in.numel() == out.numel() &&
                        in.scalar_type() == out.scalar_type(),
                    "debug_broadcast_raw_root: matching CUDA tensors");
        c10::cuda::CUDAGuard g(c.device());
        c.debug_broadcast_raw_root(in.data_ptr(), out.data_ptr(), dtype_code(in.scalar_type()), in.numel(), root,
                                   at::cuda::getCurrentCUDAStream(c.device()).stream());
      })
      .def_readwrite("nvls_min_bytes", &DeviceComm::nvls_min_bytes)
      .def_readonly("last_allreduce_algo", &DeviceComm::last_allreduce_algo)
      .def_readwrite("nvls_min_rs_bytes", &DeviceComm::nvls_min_rs_bytes)
      .def_readwrite("nvls_min_ag_bytes", &DeviceComm::nvls_min_ag_bytes)
      .def_readwrite("nvls_min_bcast_bytes", &DeviceComm::nvls_min_bcast_bytes)
      .def("nvls_supported", &DeviceComm::nvls_supported)
      .def("nvls_create", &DeviceComm::nvls_create)
      .def("nvls_import", &DeviceComm::nvls_import)
      .def("nvls_add_device", &DeviceComm::nvls_add_device)
      .def("nvls_bind_map", &DeviceComm::nvls_bind_map)
      .def("nvls_active", &DeviceComm::nvls_active)
      .def("nvls_bytes", &DeviceComm::nvls_bytes)
      .def("nvls_alloc", &DeviceComm::nvls_alloc, py::arg("bytes"), py::arg("align") = 256)
      .def("nvls_reset", &DeviceComm::nvls_reset)
      .def("nvls_release", &DeviceComm::nvls_release)
      .def("nvls_offset", [](const DeviceComm& c, const at::Tensor& t) {
        return c.nvls_offset(t.data_ptr(), (uint64_t)t.numel() * t.element_size());
      })
      .def("peer_ptr", [](const DeviceComm& c, int p) { return (uint64_t)c.peer_base(p); })
      .def("local_ptr", [](const DeviceComm& c) { return (uint64_t)c.local_base(); });
  m.def("all_reduce", &all_reduce);
  m.def("reduce_scatter", &reduce_scatter);
  m.def("all_gather", &all_gather);
  m.def("all_to_all", &all_to_all);
  m.def("broadcast", &broadcast);
  m.def("reduce", &reduce);
  m.def("gather", &gather);
  m.def("scatter", &scatter);
  m.def("scan", &scan);
  m.def("barrier", &barrier);
  m.def("reduce_inplace", &reduce_inplace);
  m.def("symmetric_tensor", &symmetric_tensor);
  m.def("nvls_tensor", &nvls_tensor);
  m.def("nvls_stage_bytes", []() { return (unsigned long long)kNvlsStageBytes; });
  m.def("launch_count", []() { return g_launches.load(); });
  m.def("gemm_reduce_scatter", &gemm_rs);
  m.def("moe_route", &moe_route_op);
  m.def("moe_dispatch", &moe_dispatch_op);
  m.def("moe_combine", &moe_combine_op);
  m.def("moe_dispatch_rows", &moe_dispatch_rows_op, py::arg("comm"), py::arg("g"), py::arg("slot_expert"),
        py::arg("slot_pos"), py::arg("slot_scale"), py::arg("dst"), py::arg("ticket"));
  m.def("all_gather_gemm", &ag_gemm);
  m.def("gemm_fp8_reduce_scatter", &gemm_fp8_rs);
  register_ops(m);
}
