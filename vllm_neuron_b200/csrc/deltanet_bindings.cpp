// torch.ops.b200 bindings of the gated-DeltaNet and gating kernels (deltanet.cu).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <cuda_runtime.h>

extern "C" {
size_t b200_gdn_workspace_bytes(int T, int B, int nv);
int b200_causal_conv1d(void* out, const void* x, int ldx, const void* w, void* conv_state, const int* qsl,
                       const int* slots, const int* init, int B, int C, int K, int max_q, int num_slots, int* status,
                       cudaStream_t s);
int b200_gdn_decode(void* out, const void* mixed, int ldm, const void* z, int ldz, const void* b, const void* a,
                    int ldab, const float* A_log, const float* dt_bias, const float* norm_w, float eps, float* state,
                    const int* qsl, const int* slots, const int* init, int B, int nk, int nv, int dk, int dv,
                    int num_slots, int* status, cudaStream_t s);
int b200_gdn_prefill(void* out, void* o_tmp, const void* mixed, int ldm, const void* z, int ldz, const void* b,
                     const void* a, int ldab, const float* A_log, const float* dt_bias, const float* norm_w,
                     float eps, float* state, const int* qsl, const int* slots, const int* init, int T, int B, int nk,
                     int nv, int dk, int dv, int num_slots, void* workspace, int* status, cudaStream_t s);
int b200_sigmoid_gate_mul(void* out, const void* x, const void* g, int ldg, int T, int N, cudaStream_t s);
int b200_gated_add(void* out, const void* x, const void* y, const void* g, int ldg, int T, int N, cudaStream_t s);
}

namespace {

using at::Tensor;

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check_i32(const Tensor& t, const char* n) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kInt && t.is_contiguous(), n, " must be contiguous int32 CUDA");
}

void check_rows(const Tensor& t, const char* n) {
  TORCH_CHECK(t.is_cuda() && t.dim() == 2 && t.stride(1) == 1 && t.scalar_type() == at::kBFloat16, n,
              " must be a bf16 [T, C] CUDA tensor with unit inner stride");
}

void causal_conv1d(Tensor out, Tensor x, Tensor w, Tensor conv_state, Tensor qsl, Tensor slots, Tensor init,
                   int64_t max_q) {
  check_rows(x, "x");
  check_i32(qsl, "qsl");
  check_i32(slots, "slots");
  check_i32(init, "init");
  TORCH_CHECK(out.is_contiguous() && w.is_contiguous() && conv_state.is_contiguous(), "contiguous tensors required");
  TORCH_CHECK(w.scalar_type() == at::kBFloat16 && conv_state.scalar_type() == at::kBFloat16, "bf16 weight / state");
  const int C = x.size(1), K = w.size(1);
  TORCH_CHECK(w.size(0) == C && conv_state.size(1) == C && conv_state.size(2) == K - 1, "conv shapes");
  c10::cuda::CUDAGuard g(x.device());
  const int rc = b200_causal_conv1d(out.data_ptr(), x.data_ptr(), x.stride(0), w.data_ptr(), conv_state.data_ptr(),
                                    qsl.data_ptr<int>(), slots.data_ptr<int>(), init.data_ptr<int>(), slots.size(0),
                                    C, K, (int)max_q, conv_state.size(0), nullptr, stream());
  TORCH_CHECK(rc == 0, "b200::causal_conv1d failed with code ", rc);
}

void gated_delta_net(Tensor out, Tensor mixed, Tensor z, Tensor b, Tensor a, Tensor A_log, Tensor dt_bias,
                     Tensor norm_w, double eps, Tensor state, Tensor qsl, Tensor slots, Tensor init, int64_t nk,
                     int64_t nv, int64_t dk, int64_t dv, bool is_decode, int64_t max_q, c10::optional<Tensor> ws) {
  check_rows(mixed, "mixed");
  check_rows(z, "z");
  check_rows(b, "b");
  check_rows(a, "a");
  check_i32(qsl, "qsl");
  check_i32(slots, "slots");
  check_i32(init, "init");
  TORCH_CHECK(b.stride(0) == a.stride(0), "b and a must share a row stride");
  TORCH_CHECK(state.scalar_type() == at::kFloat && state.is_contiguous() && state.dim() == 4 && state.size(1) == nv &&
                  state.size(2) == dk && state.size(3) == dv,
              "state must be fp32 [slots, nv, dk, dv]");
  TORCH_CHECK(A_log.scalar_type() == at::kFloat && dt_bias.scalar_type() == at::kFloat &&
                  norm_w.scalar_type() == at::kFloat,
              "fp32 A_log / dt_bias / norm weight");
  TORCH_CHECK(out.is_contiguous() && out.size(1) == nv * dv, "out must be [T, nv*dv]");
  TORCH_CHECK(mixed.size(1) >= 2 * nk * dk + nv * dv, "mixed too narrow");
  c10::cuda::CUDAGuard g(mixed.device());
  const int T = mixed.size(0), B = slots.size(0);
  int rc;
  if (is_decode) {
    rc = b200_gdn_decode(out.data_ptr(), mixed.data_ptr(), mixed.stride(0), z.data_ptr(), z.stride(0), b.data_ptr(),
                         a.data_ptr(), a.stride(0), A_log.data_ptr<float>(), dt_bias.data_ptr<float>(),
                         norm_w.data_ptr<float>(), (float)eps, state.data_ptr<float>(), qsl.data_ptr<int>(),
                         slots.data_ptr<int>(), init.data_ptr<int>(), B, nk, nv, dk, dv, state.size(0), nullptr,
                         stream());
  } else {
    const size_t need = b200_gdn_workspace_bytes(T, B, nv);
    Tensor w = ws.has_value() && (size_t)ws->numel() >= need
                   ? *ws
                   : at::empty({(int64_t)need}, mixed.options().dtype(at::kByte));
    Tensor o_tmp = at::empty({T, nv * dv}, mixed.options());
    rc = b200_gdn_prefill(out.data_ptr(), o_tmp.data_ptr(), mixed.data_ptr(), mixed.stride(0), z.data_ptr(),
                          z.stride(0), b.data_ptr(), a.data_ptr(), a.stride(0), A_log.data_ptr<float>(),
                          dt_bias.data_ptr<float>(), norm_w.data_ptr<float>(), (float)eps, state.data_ptr<float>(),
                          qsl.data_ptr<int>(), slots.data_ptr<int>(), init.data_ptr<int>(), T, B, nk, nv, dk, dv,
                          state.size(0), w.data_ptr(), nullptr, stream());
  }
  TORCH_CHECK(rc == 0, "b200::gated_delta_net failed with code ", rc);
}

void sigmoid_gate_mul(Tensor out, Tensor x, Tensor gate) {
  check_rows(gate, "gate");
  TORCH_CHECK(x.is_contiguous() && out.is_contiguous() && x.scalar_type() == at::kBFloat16, "bf16 contiguous x");
  const int T = x.size(0), N = x.numel() / std::max<int64_t>(1, x.size(0));
  TORCH_CHECK(gate.size(0) == T && gate.size(1) >= N, "gate shape");
  c10::cuda::CUDAGuard g(x.device());
  const int rc = b200_sigmoid_gate_mul(out.data_ptr(), x.data_ptr(), gate.data_ptr(), gate.stride(0), T, N, stream());
  TORCH_CHECK(rc == 0, "b200::sigmoid_gate_mul failed with code ", rc);
}

void gated_add(Tensor out, Tensor x, Tensor y, Tensor gate) {
  check_rows(gate, "gate");
  TORCH_CHECK(x.is_contiguous() && y.is_contiguous() && out.is_contiguous() && x.scalar_type() == at::kBFloat16,
              "bf16 contiguous x / y");
  const int T = x.size(0), N = x.size(1);
  c10::cuda::CUDAGuard g(x.device());
  const int rc = b200_gated_add(out.data_ptr(), x.data_ptr(), y.data_ptr(), gate.data_ptr(), gate.stride(0), T, N,
                                stream());
  TORCH_CHECK(rc == 0, "b200::gated_add failed with code ", rc);
}

}  // namespace

void register_deltanet_ops(torch::Library& m) {
  m.def(
      "causal_conv1d(Tensor(a!) out, Tensor x, Tensor w, Tensor(b!) conv_state, Tensor qsl, Tensor slots, "
      "Tensor init, int max_q) -> ()");
  m.def(
      "gated_delta_net(Tensor(a!) out, Tensor mixed, Tensor z, Tensor b, Tensor a, Tensor A_log, Tensor dt_bias, "
      "Tensor norm_w, float eps, Tensor(b!) state, Tensor qsl, Tensor slots, Tensor init, int nk, int nv, int dk, "
      "int dv, bool is_decode, int max_q, Tensor? workspace) -> ()");
  m.def("sigmoid_gate_mul(Tensor(a!) out, Tensor x, Tensor gate) -> ()");
  m.def("gated_add(Tensor(a!) out, Tensor x, Tensor y, Tensor gate) -> ()");
}

void register_deltanet_impls(torch::Library& m) {
  m.impl("causal_conv1d", &causal_conv1d);
  m.impl("gated_delta_net", &gated_delta_net);
  m.impl("sigmoid_gate_mul", &sigmoid_gate_mul);
  m.impl("gated_add", &gated_add);
}
