// torch.ops.b200 registration of the dense tcgen05 GEMM and its fused all-reduce.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

extern "C" {
void b200_gemm_workspace(int T, int N, int K, int max_splits, int64_t* ws_floats, int64_t* n_counters);
int b200_gemm_bf16(void* y, int ldy, int out_f32, const void* x, int ldx, const void* w, const void* bias, int T,
                   int N, int K, float* ws, int64_t ws_floats, int* counters, int64_t n_counters, int max_splits,
                   int* status, cudaStream_t s);
void b200_gemm_force_nt(int nt);
void b200_gemm_plan(int T, int N, int K, int max_splits, int sms, int* out);
int b200_gemm_bf16_scatter(void* const* dst, int n_dst, int ldd, const void* x, int ldx, const void* w, int T, int N,
                           int K, float* ws, int64_t ws_floats, int* counters, int64_t n_counters, int max_splits,
                           int* status, cudaStream_t s);
int b200_gemm_fp8(void* y, int ldy, int out_f32, const void* x, int ldx, const void* w, const void* bias,
                  const float* alpha, int alpha_n, int T, int N, int K, float* ws, int64_t ws_floats, int* counters,
                  int64_t n_counters, int max_splits, int* status, cudaStream_t s);
int b200_fp8_quant(void* q, int ldq, const void* x, int ldx, int rows, int H, const float* scale, unsigned* amax_ws,
                   const float* w_scale, float* alpha, int alpha_n, cudaStream_t s);
int b200_rms_norm_fp8(void* q, const void* x, void* residual, const float* w, int rows, int H, float eps,
                      const float* scale, cudaStream_t s);
size_t b200_red_region_bytes(int T_cap, int H_cap);
void b200_gemm_set_trace(void* buf);
int b200_gemm_bf16_allreduce(const void* x, int ldx, const void* w, int T, int N, int K, void* red_uc, void* red_mc,
                             int T_cap, int H_cap, int max_splits, int* items, int* status, cudaStream_t s);
int b200_allreduce_finish(void* red_uc, int T_cap, int H_cap, int expected, void* out, void* residual,
                          const void* bias, const float* w, float eps, int T, int H, int num_blocks,
                          unsigned long long wait_ns, int* status, cudaStream_t s);
}

namespace {
using at::Tensor;

void check_x_w(const Tensor& x, const Tensor& w) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda(), "gemm: CUDA tensors required");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16, "gemm: bf16 x and w");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1), "gemm: x [T, K], w [N, K]");
  TORCH_CHECK(x.stride(1) == 1 && w.is_contiguous(), "gemm: x rows and w must be contiguous");
}

std::vector<int64_t> gemm_workspace(int64_t T, int64_t N, int64_t K, int64_t max_splits) {
  int64_t ws = 0, nc = 0;
  b200_gemm_workspace(T, N, K, max_splits, &ws, &nc);
  return {ws, nc};
}

void gemm_bf16(Tensor y, Tensor x, Tensor w, c10::optional<Tensor> bias, Tensor ws, Tensor counters,
               int64_t max_splits, c10::optional<Tensor> status) {
  check_x_w(x, w);
  const int T = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK((y.scalar_type() == at::kBFloat16 || y.scalar_type() == at::kFloat) && y.dim() == 2 &&
                  y.size(0) == T && y.size(1) == N && y.stride(1) == 1,
              "gemm: y [T, N] bf16 or fp32 with contiguous rows");
  if (bias.has_value())
    TORCH_CHECK(bias->scalar_type() == at::kBFloat16 && bias->numel() == N && bias->is_contiguous(), "gemm: bias");
  TORCH_CHECK(ws.scalar_type() == at::kFloat && counters.scalar_type() == at::kInt, "gemm: workspace dtypes");
  c10::cuda::CUDAGuard g(x.device());
  const int rc = b200_gemm_bf16(y.data_ptr(), y.stride(0), y.scalar_type() == at::kFloat, x.data_ptr(),
                                x.stride(0), w.data_ptr(),
                                bias.has_value() ? bias->data_ptr() : nullptr, T, N, K, ws.data_ptr<float>(),
                                ws.numel(), counters.data_ptr<int>(), counters.numel(), max_splits,
                                status.has_value() ? status->data_ptr<int>() : nullptr,
                                at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(rc == 0, "b200::gemm_bf16 failed with code ", rc);
}

// Y = X . W^T with row block q (T / len(dst) rows) stored at the device address dst[q] (rows of
// ldd elements): the producer side of a sequence-parallel reduce-scatter.
void gemm_scatter(at::IntArrayRef dst, int64_t ldd, Tensor x, Tensor w, Tensor ws, Tensor counters,
                  int64_t max_splits, c10::optional<Tensor> status) {
  check_x_w(x, w);
  const int T = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(dst.size() >= 1 && dst.size() <= 8, "gemm_scatter: 1..8 destinations");
  TORCH_CHECK(ws.scalar_type() == at::kFloat && counters.scalar_type() == at::kInt, "gemm: workspace dtypes");
  void* ptrs[8];
  for (size_t i = 0; i < dst.size(); ++i) ptrs[i] = reinterpret_cast<void*>(dst[i]);
  c10::cuda::CUDAGuard g(x.device());
  const int rc = b200_gemm_bf16_scatter(ptrs, dst.size(), ldd, x.data_ptr(), x.stride(0), w.data_ptr(), T, N, K,
                                        ws.data_ptr<float>(), ws.numel(), counters.data_ptr<int>(), counters.numel(),
                                        max_splits, status.has_value() ? status->data_ptr<int>() : nullptr,
                                        at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(rc == 0, "b200::gemm_scatter failed with code ", rc);
}

void gemm_force_nt(int64_t nt) { b200_gemm_force_nt((int)nt); }

// The planner's decision: [token tile width, output tiles, K splits, cluster split, k stages per split].
std::vector<int64_t> gemm_plan(int64_t T, int64_t N, int64_t K, int64_t max_splits, int64_t sms) {
  int o[5];
  b200_gemm_plan(T, N, K, max_splits, sms, o);
  return {o[0], o[1], o[2], o[3], o[4]};
}

void gemm_fp8(Tensor y, Tensor x, Tensor w, c10::optional<Tensor> bias, Tensor alpha, Tensor ws, Tensor counters,
              int64_t max_splits, c10::optional<Tensor> status) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda(), "gemm_fp8: CUDA tensors required");
  TORCH_CHECK(x.scalar_type() == at::kFloat8_e4m3fn && w.scalar_type() == at::kFloat8_e4m3fn, "gemm_fp8: e4m3 x and w");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1), "gemm_fp8: x [T, K], w [N, K]");
  TORCH_CHECK(x.stride(1) == 1 && w.is_contiguous(), "gemm_fp8: x rows and w must be contiguous");
  const int T = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK((y.scalar_type() == at::kBFloat16 || y.scalar_type() == at::kFloat) && y.dim() == 2 &&
                  y.size(0) == T && y.size(1) == N && y.stride(1) == 1,
              "gemm_fp8: y [T, N] bf16 or fp32 with contiguous rows");
  TORCH_CHECK(alpha.is_cuda() && alpha.scalar_type() == at::kFloat && alpha.is_contiguous() &&
                  (alpha.numel() == 1 || alpha.numel() == N),
              "gemm_fp8: fp32 alpha [1] or [N]");
  if (bias.has_value())
    TORCH_CHECK(bias->scalar_type() == at::kBFloat16 && bias->numel() == N && bias->is_contiguous(), "gemm_fp8: bias");
  TORCH_CHECK(ws.scalar_type() == at::kFloat && counters.scalar_type() == at::kInt, "gemm_fp8: workspace dtypes");
  c10::cuda::CUDAGuard g(x.device());
  const int rc = b200_gemm_fp8(y.data_ptr(), y.stride(0), y.scalar_type() == at::kFloat, x.data_ptr(), x.stride(0),
                               w.data_ptr(), bias.has_value() ? bias->data_ptr() : nullptr, alpha.data_ptr<float>(),
                               (int)alpha.numel(), T, N, K, ws.data_ptr<float>(), ws.numel(), counters.data_ptr<int>(),
                               counters.numel(), max_splits, status.has_value() ? status->data_ptr<int>() : nullptr,
                               at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(rc == 0, "b200::gemm_fp8 failed with code ", rc);
}

void fp8_quant(Tensor q, Tensor x, c10::optional<Tensor> scale, c10::optional<Tensor> amax_ws,
               c10::optional<Tensor> w_scale, c10::optional<Tensor> alpha) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1, "fp8_quant: bf16 x");
  TORCH_CHECK(q.scalar_type() == at::kFloat8_e4m3fn && q.dim() == 2 && q.size(0) == x.size(0) &&
                  q.size(1) == x.size(1) && q.stride(1) == 1,
              "fp8_quant: e4m3 q like x");
  auto fptr = [](const c10::optional<Tensor>& t) -> float* {
    if (!t.has_value()) return nullptr;
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat, "fp8_quant: fp32 device scalars");
    return t->data_ptr<float>();
  };
  unsigned* aw = nullptr;
  if (amax_ws.has_value()) {
    TORCH_CHECK(amax_ws->is_cuda() && amax_ws->scalar_type() == at::kInt, "fp8_quant: int32 amax scratch");
    aw = reinterpret_cast<unsigned*>(amax_ws->data_ptr<int>());
  }
  int alpha_n = 0;
  if (alpha.has_value()) {
    alpha_n = (int)alpha->numel();
    TORCH_CHECK(!w_scale.has_value() || w_scale->numel() == alpha_n, "fp8_quant: w_scale like alpha");
  }
  c10::cuda::CUDAGuard g(x.device());
  const int rc = b200_fp8_quant(q.data_ptr(), q.stride(0), x.data_ptr(), x.stride(0), x.size(0), x.size(1),
                                fptr(scale), aw, fptr(w_scale), fptr(alpha), alpha_n,
                                at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(rc == 0, "b200::fp8_quant failed with code ", rc);
}

void rms_norm_fp8(Tensor q, Tensor x, c10::optional<Tensor> residual, Tensor w, double eps, Tensor scale) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 2,
              "rms_norm_fp8: bf16 x [T, H]");
  TORCH_CHECK(q.scalar_type() == at::kFloat8_e4m3fn && q.is_contiguous() && q.numel() == x.numel(), "rms_norm_fp8: q");
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.numel() == x.size(1), "rms_norm_fp8: fp32 w [H]");
  TORCH_CHECK(scale.is_cuda() && scale.scalar_type() == at::kFloat, "rms_norm_fp8: fp32 scale");
  if (residual.has_value())
    TORCH_CHECK(residual->scalar_type() == at::kBFloat16 && residual->is_contiguous() &&
                    residual->numel() == x.numel(),
                "rms_norm_fp8: bf16 residual like x");
  c10::cuda::CUDAGuard g(x.device());
  const int rc = b200_rms_norm_fp8(q.data_ptr(), x.data_ptr(), residual.has_value() ? residual->data_ptr() : nullptr,
                                   w.data_ptr<float>(), x.size(0), x.size(1), (float)eps, scale.data_ptr<float>(),
                                   at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(rc == 0, "b200::rms_norm_fp8 failed with code ", rc);
}

int64_t red_region_bytes(int64_t T_cap, int64_t H_cap) { return (int64_t)b200_red_region_bytes(T_cap, H_cap); }

void gemm_set_trace(int64_t buf) { b200_gemm_set_trace(reinterpret_cast<void*>(buf)); }

int64_t gemm_bf16_allreduce(Tensor x, Tensor w, int64_t red_uc, int64_t red_mc, int64_t T_cap, int64_t H_cap,
                            int64_t max_splits, c10::optional<Tensor> status) {
  check_x_w(x, w);
  const int T = x.size(0), K = x.size(1), N = w.size(0);
  int items = 0;
  c10::cuda::CUDAGuard g(x.device());
  const int rc = b200_gemm_bf16_allreduce(x.data_ptr(), x.stride(0), w.data_ptr(), T, N, K,
                                          reinterpret_cast<void*>(red_uc), reinterpret_cast<void*>(red_mc), T_cap,
                                          H_cap, max_splits, &items,
                                          status.has_value() ? status->data_ptr<int>() : nullptr,
                                          at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(rc == 0, "b200::gemm_bf16_allreduce failed with code ", rc);
  return items;
}

void allreduce_finish(int64_t red_uc, int64_t T_cap, int64_t H_cap, int64_t expected, Tensor out,
                      c10::optional<Tensor> residual, c10::optional<Tensor> bias, c10::optional<Tensor> w, double eps,
                      int64_t num_blocks, c10::optional<Tensor> status, int64_t wait_ns) {
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.dim() == 2,
              "finish: bf16 out [T, H]");
  const int T = out.size(0), H = out.size(1);
  if (w.has_value()) {
    TORCH_CHECK(residual.has_value() && residual->scalar_type() == at::kBFloat16 && residual->is_contiguous() &&
                    residual->numel() == out.numel(),
                "finish: bf16 residual like out");
    TORCH_CHECK(w->scalar_type() == at::kFloat && w->numel() == H, "finish: fp32 norm weight [H]");
  }
  if (bias.has_value()) TORCH_CHECK(bias->scalar_type() == at::kBFloat16 && bias->numel() == H, "finish: bias");
  c10::cuda::CUDAGuard g(out.device());
  const int rc = b200_allreduce_finish(
      reinterpret_cast<void*>(red_uc), T_cap, H_cap, expected, out.data_ptr(),
      residual.has_value() ? residual->data_ptr() : nullptr, bias.has_value() ? bias->data_ptr() : nullptr,
      w.has_value() ? w->data_ptr<float>() : nullptr, (float)eps, T, H, num_blocks,
      wait_ns > 0 ? (unsigned long long)wait_ns : 0ull, status.has_value() ? status->data_ptr<int>() : nullptr,
      at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(rc == 0, "b200::allreduce_finish failed with code ", rc);
}
}  // namespace

void register_gemm_ops(torch::Library& m) {
  m.def("gemm_workspace(int T, int N, int K, int max_splits) -> int[]");
  m.def(
      "gemm_bf16(Tensor(a!) y, Tensor x, Tensor w, Tensor? bias, Tensor(b!) ws, Tensor(c!) counters, "
      "int max_splits, Tensor? status) -> ()");
  m.def(
      "gemm_scatter(int[] dst, int ldd, Tensor x, Tensor w, Tensor(a!) ws, Tensor(b!) counters, int max_splits, "
      "Tensor? status) -> ()");
  m.def(
      "gemm_fp8(Tensor(a!) y, Tensor x, Tensor w, Tensor? bias, Tensor alpha, Tensor(b!) ws, Tensor(c!) counters, "
      "int max_splits, Tensor? status) -> ()");
  m.def(
      "fp8_quant(Tensor(a!) q, Tensor x, Tensor? scale, Tensor(b!)? amax_ws, Tensor? w_scale, Tensor(c!)? alpha) -> ()");
  m.def("rms_norm_fp8(Tensor(a!) q, Tensor x, Tensor(b!)? residual, Tensor w, float eps, Tensor scale) -> ()");
  m.def("red_region_bytes(int T_cap, int H_cap) -> int");
  m.def("gemm_set_trace(int buf) -> ()");
  m.def("gemm_force_nt(int nt) -> ()");
  m.def("gemm_plan(int T, int N, int K, int max_splits, int sms) -> int[]");
  m.def(
      "gemm_bf16_allreduce(Tensor x, Tensor w, int red_uc, int red_mc, int T_cap, int H_cap, int max_splits, "
      "Tensor? status) -> int");
  m.def(
      "allreduce_finish(int red_uc, int T_cap, int H_cap, int expected, Tensor(a!) out, Tensor(b!)? residual, "
      "Tensor? bias, Tensor? w, float eps, int num_blocks, Tensor? status, int wait_ns=0) -> ()");
}

void register_gemm_impls(torch::Library& m) {
  m.impl("gemm_bf16", &gemm_bf16);
  m.impl("gemm_fp8", &gemm_fp8);
  m.impl("gemm_scatter", &gemm_scatter);
  m.impl("fp8_quant", &fp8_quant);
  m.impl("rms_norm_fp8", &rms_norm_fp8);
  m.impl("gemm_bf16_allreduce", &gemm_bf16_allreduce);
  m.impl("allreduce_finish", &allreduce_finish);
}

void register_gemm_cpu_impls(torch::Library& m) {
  m.impl("gemm_workspace", &gemm_workspace);
  m.impl("red_region_bytes", &red_region_bytes);
  m.impl("gemm_set_trace", &gemm_set_trace);
  m.impl("gemm_force_nt", &gemm_force_nt);
  m.impl("gemm_plan", &gemm_plan);
}
