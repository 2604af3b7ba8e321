// torch.ops.b200.* registration.  Each op validates its tensors (device, dtype,
// contiguity, shapes) on the host and calls the raw-pointer launcher on the current
// CUDA stream.  Validation failures raise; kernel launch failures raise with the code.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <ATen/ATen.h>
#include <torch/library.h>

#include "launch.h"
#include "moe.h"

namespace {

using at::Tensor;

int dt(const Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat: return b200::kF32;
    case at::kHalf: return b200::kF16;
    case at::kBFloat16: return b200::kBF16;
    case at::kFloat8_e4m3fn: return b200::kFP8E4M3;
    case at::kByte: return b200::kU8;
    case at::kInt: return b200::kI32;
    case at::kLong: return b200::kI64;
    default: TORCH_CHECK(false, "unsupported dtype ", t.scalar_type());
  }
  return -1;
}

void check_cuda(const Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}

void check_rc(int rc, const char* op) { TORCH_CHECK(rc == 0, "b200::", op, " failed with code ", rc); }

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void rms_norm(Tensor out, Tensor x, Tensor w, double eps) {
  check_cuda(x, "x");
  TORCH_CHECK(x.is_contiguous() && out.is_contiguous(), "rms_norm: contiguous tensors required");
  TORCH_CHECK(w.scalar_type() == at::kFloat, "rms_norm: weight must be fp32");
  const int H = x.size(-1);
  const int rows = x.numel() / H;
  c10::cuda::CUDAGuard g(x.device());
  check_rc(b200_rms_norm(out.data_ptr(), x.data_ptr(), nullptr, w.data_ptr<float>(), rows, H, (float)eps, dt(x),
                         stream()),
           "rms_norm");
}

void fused_add_rms_norm(Tensor out, Tensor x, Tensor residual, Tensor w, double eps) {
  check_cuda(x, "x");
  TORCH_CHECK(x.is_contiguous() && residual.is_contiguous() && out.is_contiguous(), "contiguous tensors required");
  TORCH_CHECK(residual.scalar_type() == x.scalar_type(), "residual dtype mismatch");
  TORCH_CHECK(w.scalar_type() == at::kFloat, "weight must be fp32");
  const int H = x.size(-1);
  const int rows = x.numel() / H;
  c10::cuda::CUDAGuard g(x.device());
  check_rc(b200_rms_norm(out.data_ptr(), x.data_ptr(), residual.data_ptr(), w.data_ptr<float>(), rows, H,
                         (float)eps, dt(x), stream()),
           "fused_add_rms_norm");
}

void silu_and_mul(Tensor out, Tensor gu) {
  check_cuda(gu, "gu");
  TORCH_CHECK(gu.is_contiguous() && out.is_contiguous() && gu.scalar_type() == at::kBFloat16, "bf16 contiguous");
  const int I = gu.size(-1) / 2;
  c10::cuda::CUDAGuard g(gu.device());
  check_rc(b200_silu_and_mul(out.data_ptr(), gu.data_ptr(), gu.numel() / gu.size(-1), I, stream()), "silu_and_mul");
}

void embedding(Tensor out, Tensor ids, Tensor w, int64_t start) {
  check_cuda(w, "w");
  TORCH_CHECK(ids.scalar_type() == at::kLong && ids.is_contiguous(), "ids must be contiguous int64");
  TORCH_CHECK(w.is_contiguous() && out.is_contiguous(), "contiguous tensors required");
  c10::cuda::CUDAGuard g(w.device());
  check_rc(b200_embedding(out.data_ptr(), ids.data_ptr<int64_t>(), w.data_ptr(), ids.numel(), w.size(0), w.size(1),
                          start, dt(w), stream()),
           "embedding");
}

void rope_kv_write(Tensor qkv, Tensor positions, Tensor cos_sin, Tensor k_cache, Tensor v_cache, Tensor slots,
                   int64_t nq, int64_t nkv, int64_t d, int64_t rotary_dim, double k_scale, double v_scale,
                   c10::optional<Tensor> q_norm, c10::optional<Tensor> k_norm, double eps) {
  check_cuda(qkv, "qkv");
  TORCH_CHECK(qkv.dim() == 2 && qkv.stride(1) == 1, "qkv must be [T, C] with unit inner stride");
  TORCH_CHECK(qkv.size(1) >= (nq + 2 * nkv) * d, "qkv too narrow");
  TORCH_CHECK(positions.scalar_type() == at::kLong && slots.scalar_type() == at::kLong, "int64 positions/slots");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.size(1) == rotary_dim, "cos_sin [max_pos, rotary_dim]");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(1) == nkv && k_cache.size(3) == d, "cache [nb, nkv, bs, d]");
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous(), "contiguous caches required");
  const float* qn = q_norm.has_value() ? q_norm->data_ptr<float>() : nullptr;
  const float* kn = k_norm.has_value() ? k_norm->data_ptr<float>() : nullptr;
  c10::cuda::CUDAGuard g(qkv.device());
  check_rc(b200_rope_kv_write(qkv.data_ptr(), positions.data_ptr<int64_t>(), cos_sin.data_ptr<float>(),
                              k_cache.data_ptr(), v_cache.data_ptr(), slots.data_ptr<int64_t>(), qkv.size(0), nq, nkv,
                              d, rotary_dim, qkv.stride(0), k_cache.size(2), k_cache.size(0), (float)k_scale,
                              (float)v_scale, qn, kn, (float)eps, dt(qkv), dt(k_cache), nullptr, stream()),
           "rope_kv_write");
}

void check_q(const Tensor& q, int64_t d) {
  TORCH_CHECK(q.dim() == 3 && q.stride(2) == 1 && q.stride(1) == d, "q must be [T, heads, d] with packed heads");
}

void paged_attention_decode(Tensor out, Tensor q, Tensor k_cache, Tensor v_cache, Tensor block_tables,
                            Tensor seq_lens, c10::optional<Tensor> sinks, int64_t window, double scale,
                            double k_scale, double v_scale, c10::optional<Tensor> workspace, int64_t num_splits) {
  check_cuda(q, "q");
  const int64_t d = q.size(2);
  check_q(q, d);
  TORCH_CHECK(out.is_contiguous(), "out must be contiguous");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt, "int32 tables");
  TORCH_CHECK(block_tables.stride(1) == 1, "block_tables rows must be contiguous");
  const int B = seq_lens.size(0);
  TORCH_CHECK(q.size(0) == B, "decode expects one query token per sequence");
  const int nq = q.size(1), nkv = k_cache.size(1);
  float* ws = nullptr;
  if (num_splits > 1) {
    TORCH_CHECK(workspace.has_value(), "split-KV decode needs a workspace");
    TORCH_CHECK(workspace->numel() >= (int64_t)B * nq * num_splits * (d + 1), "workspace too small");
    ws = workspace->data_ptr<float>();
  }
  c10::cuda::CUDAGuard g(q.device());
  check_rc(b200_paged_attention_decode(out.data_ptr(), q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                                       block_tables.data_ptr<int>(), seq_lens.data_ptr<int>(),
                                       sinks.has_value() ? sinks->data_ptr<float>() : nullptr, B, nq, nkv, d,
                                       q.stride(0), k_cache.size(2), block_tables.stride(0), window, (float)scale,
                                       (float)k_scale, (float)v_scale, ws, num_splits, dt(q), dt(k_cache), stream()),
           "paged_attention_decode");
}

// VLLM_B200_TC_PREFILL=0 keeps prefill attention on the warp-MMA kernel (comparison runs).
bool tc_prefill_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("VLLM_B200_TC_PREFILL");
    v = (e != nullptr && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

void paged_attention_prefill(Tensor out, Tensor q, Tensor k_cache, Tensor v_cache, Tensor block_tables,
                             Tensor seq_lens, Tensor qsl, c10::optional<Tensor> sinks, int64_t window, double scale,
                             double k_scale, double v_scale, int64_t max_query_len) {
  check_cuda(q, "q");
  const int64_t d = q.size(2);
  check_q(q, d);
  TORCH_CHECK(out.is_contiguous(), "out must be contiguous");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt &&
                  qsl.scalar_type() == at::kInt,
              "int32 metadata");
  const int B = seq_lens.size(0);
  c10::cuda::CUDAGuard g(q.device());
  if (tc_prefill_enabled() && k_cache.is_contiguous() && v_cache.is_contiguous() &&
      b200_prefill_tc_supported(d, dt(q), dt(k_cache), k_cache.size(2))) {
    // tcgen05 / TMEM flash attention (csrc/fa_prefill.cu)
    check_rc(b200_paged_attention_prefill_tc(
                 out.data_ptr(), q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), k_cache.size(0),
                 block_tables.data_ptr<int>(), seq_lens.data_ptr<int>(), qsl.data_ptr<int>(),
                 sinks.has_value() ? sinks->data_ptr<float>() : nullptr, B, q.size(1), k_cache.size(1), d,
                 q.stride(0), k_cache.size(2), block_tables.stride(0), window, (float)scale, (float)k_scale,
                 (float)v_scale, max_query_len, (int)q.size(0), dt(q), dt(k_cache), nullptr, stream()),
             "paged_attention_prefill_tc");
    return;
  }
  check_rc(b200_paged_attention_prefill(out.data_ptr(), q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                                        block_tables.data_ptr<int>(), seq_lens.data_ptr<int>(), qsl.data_ptr<int>(),
                                        sinks.has_value() ? sinks->data_ptr<float>() : nullptr, B, q.size(0),
                                        q.size(1), k_cache.size(1), d, q.stride(0), k_cache.size(2),
                                        block_tables.stride(0), window, (float)scale, (float)k_scale, (float)v_scale,
                                        max_query_len, dt(q), dt(k_cache), stream()),
           "paged_attention_prefill");
}

void paged_attention_decode_cp(Tensor out, Tensor lse, Tensor q, Tensor k_cache, Tensor v_cache,
                               Tensor block_tables, Tensor seq_lens, int64_t window, double scale, double k_scale,
                               double v_scale, c10::optional<Tensor> workspace, int64_t num_splits, int64_t cp_rank,
                               int64_t cp_size) {
  check_cuda(q, "q");
  const int64_t d = q.size(2);
  check_q(q, d);
  TORCH_CHECK(out.is_contiguous() && lse.is_contiguous() && lse.scalar_type() == at::kFloat, "out / lse");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt, "int32 tables");
  TORCH_CHECK(block_tables.stride(1) == 1, "block_tables rows must be contiguous");
  const int B = seq_lens.size(0);
  TORCH_CHECK(q.size(0) == B, "decode expects one query token per sequence");
  const int nq = q.size(1), nkv = k_cache.size(1);
  TORCH_CHECK(lse.numel() >= (int64_t)B * nq, "lse too small");
  float* ws = nullptr;
  if (num_splits > 1 && workspace.has_value()) {
    TORCH_CHECK(workspace->numel() >= (int64_t)B * nq * num_splits * (d + 1), "workspace too small");
    ws = workspace->data_ptr<float>();
  }
  c10::cuda::CUDAGuard g(q.device());
  check_rc(b200_paged_attention_decode_cp(out.data_ptr(), lse.data_ptr<float>(), q.data_ptr(), k_cache.data_ptr(),
                                          v_cache.data_ptr(), block_tables.data_ptr<int>(), seq_lens.data_ptr<int>(),
                                          B, nq, nkv, d, q.stride(0), k_cache.size(2), block_tables.stride(0), window,
                                          (float)scale, (float)k_scale, (float)v_scale, ws, num_splits, cp_rank,
                                          cp_size, dt(q), dt(k_cache), stream()),
           "paged_attention_decode_cp");
}

void paged_attention_prefill_cp(Tensor out, Tensor lse, Tensor q, Tensor k_cache, Tensor v_cache,
                                Tensor block_tables, Tensor seq_lens, Tensor qsl, int64_t window, double scale,
                                double k_scale, double v_scale, int64_t max_query_len, int64_t cp_rank,
                                int64_t cp_size) {
  check_cuda(q, "q");
  const int64_t d = q.size(2);
  check_q(q, d);
  TORCH_CHECK(out.is_contiguous() && lse.is_contiguous() && lse.scalar_type() == at::kFloat, "out / lse");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt &&
                  qsl.scalar_type() == at::kInt,
              "int32 metadata");
  TORCH_CHECK(lse.numel() >= q.size(0) * q.size(1), "lse too small");
  const int B = seq_lens.size(0);
  c10::cuda::CUDAGuard g(q.device());
  check_rc(b200_paged_attention_prefill_cp(out.data_ptr(), lse.data_ptr<float>(), q.data_ptr(), k_cache.data_ptr(),
                                           v_cache.data_ptr(), block_tables.data_ptr<int>(),
                                           seq_lens.data_ptr<int>(), qsl.data_ptr<int>(), B, q.size(1),
                                           k_cache.size(1), d, q.stride(0), k_cache.size(2), block_tables.stride(0),
                                           window, (float)scale, (float)k_scale, (float)v_scale, max_query_len,
                                           cp_rank, cp_size, dt(q), dt(k_cache), stream()),
           "paged_attention_prefill_cp");
}

void varlen_attention(Tensor out, Tensor q, Tensor k, Tensor v, Tensor cu, double scale, bool causal,
                      int64_t max_seqlen) {
  check_cuda(q, "q");
  TORCH_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous() && out.is_contiguous(), "contiguous");
  TORCH_CHECK(cu.scalar_type() == at::kInt, "cu_seqlens int32");
  c10::cuda::CUDAGuard g(q.device());
  check_rc(b200_varlen_attention(out.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), cu.data_ptr<int>(),
                                 cu.size(0) - 1, q.size(0), q.size(1), k.size(1), q.size(2), (float)scale, causal,
                                 max_seqlen, dt(q), stream()),
           "varlen_attention");
}

void topk_softmax(Tensor ids, Tensor weights, Tensor logits, int64_t full) {
  check_cuda(logits, "logits");
  TORCH_CHECK((logits.scalar_type() == at::kFloat || logits.scalar_type() == at::kBFloat16) &&
                  logits.is_contiguous(),
              "fp32 / bf16 contiguous logits");
  c10::cuda::CUDAGuard g(logits.device());
  check_rc(b200_topk_softmax(ids.data_ptr<int>(), weights.data_ptr<float>(), logits.data_ptr(), logits.size(0),
                             logits.size(1), ids.size(1), dt(logits), (int)full, stream()),
           "topk_softmax");
}

void argmax(Tensor vals, Tensor idx, Tensor logits) {
  check_cuda(logits, "logits");
  TORCH_CHECK(logits.is_contiguous(), "contiguous logits");
  c10::cuda::CUDAGuard g(logits.device());
  check_rc(b200_argmax(vals.data_ptr<float>(), idx.data_ptr<int64_t>(), logits.data_ptr(), logits.size(0),
                       logits.size(1), dt(logits), stream()),
           "argmax");
}

void sample(Tensor out, Tensor logits, Tensor temperature, Tensor top_k, Tensor top_p, Tensor uniform,
            int64_t max_top_k) {
  check_cuda(logits, "logits");
  TORCH_CHECK(logits.is_contiguous(), "contiguous logits");
  TORCH_CHECK(top_k.scalar_type() == at::kInt, "top_k int32");
  c10::cuda::CUDAGuard g(logits.device());
  check_rc(b200_sample(out.data_ptr<int64_t>(), logits.data_ptr(), temperature.data_ptr<float>(),
                       top_k.data_ptr<int>(), top_p.data_ptr<float>(), uniform.data_ptr<float>(), logits.size(0),
                       logits.size(1), max_top_k, dt(logits), nullptr, stream()),
           "sample");
}

}  // namespace

void register_moe_ops(torch::Library& m);
void register_moe_impls(torch::Library& m);
void register_comm_ops(torch::Library& m);
void register_comm_impls(torch::Library& m);
void register_comm_cpu_impls(torch::Library& m);
void register_deltanet_ops(torch::Library& m);
void register_deltanet_impls(torch::Library& m);
void register_gemm_ops(torch::Library& m);
void register_mla_ops(torch::Library& m);
void register_mla_impls(torch::Library& m);
void register_gemm_impls(torch::Library& m);
void register_gemm_cpu_impls(torch::Library& m);

TORCH_LIBRARY(b200, m) {
  m.def("rms_norm(Tensor(a!) out, Tensor x, Tensor w, float eps) -> ()");
  m.def("fused_add_rms_norm(Tensor(a!) out, Tensor x, Tensor(b!) residual, Tensor w, float eps) -> ()");
  m.def("embedding(Tensor(a!) out, Tensor ids, Tensor w, int start) -> ()");
  m.def("silu_and_mul(Tensor(a!) out, Tensor gu) -> ()");
  m.def(
      "rope_kv_write(Tensor(a!) qkv, Tensor positions, Tensor cos_sin, Tensor(b!) k_cache, Tensor(c!) v_cache, "
      "Tensor slots, int nq, int nkv, int d, int rotary_dim, float k_scale, float v_scale, Tensor? q_norm, "
      "Tensor? k_norm, float eps) -> ()");
  m.def(
      "paged_attention_decode(Tensor(a!) out, Tensor q, Tensor k_cache, Tensor v_cache, Tensor block_tables, "
      "Tensor seq_lens, Tensor? sinks, int window, float scale, float k_scale, float v_scale, Tensor? workspace, "
      "int num_splits) -> ()");
  m.def(
      "paged_attention_prefill(Tensor(a!) out, Tensor q, Tensor k_cache, Tensor v_cache, Tensor block_tables, "
      "Tensor seq_lens, Tensor query_start_loc, Tensor? sinks, int window, float scale, float k_scale, "
      "float v_scale, int max_query_len) -> ()");
  m.def(
      "paged_attention_decode_cp(Tensor(a!) out, Tensor(b!) lse, Tensor q, Tensor k_cache, Tensor v_cache, "
      "Tensor block_tables, Tensor seq_lens, int window, float scale, float k_scale, float v_scale, "
      "Tensor? workspace, int num_splits, int cp_rank, int cp_size) -> ()");
  m.def(
      "paged_attention_prefill_cp(Tensor(a!) out, Tensor(b!) lse, Tensor q, Tensor k_cache, Tensor v_cache, "
      "Tensor block_tables, Tensor seq_lens, Tensor query_start_loc, int window, float scale, float k_scale, "
      "float v_scale, int max_query_len, int cp_rank, int cp_size) -> ()");
  m.def(
      "varlen_attention(Tensor(a!) out, Tensor q, Tensor k, Tensor v, Tensor cu_seqlens, float scale, bool causal, "
      "int max_seqlen) -> ()");
  m.def("topk_softmax(Tensor(a!) ids, Tensor(b!) weights, Tensor logits, int full=0) -> ()");
  m.def("argmax(Tensor(a!) vals, Tensor(b!) idx, Tensor logits) -> ()");
  m.def(
      "sample(Tensor(a!) out, Tensor logits, Tensor temperature, Tensor top_k, Tensor top_p, Tensor uniform, "
      "int max_top_k) -> ()");
  register_moe_ops(m);
  register_comm_ops(m);
  register_deltanet_ops(m);
  register_gemm_ops(m);
  register_mla_ops(m);
}

// ops without tensor arguments (pointer plumbing) dispatch through CompositeExplicitAutograd
TORCH_LIBRARY_IMPL(b200, CompositeExplicitAutograd, m) {
  register_comm_cpu_impls(m);
  register_gemm_cpu_impls(m);
}

TORCH_LIBRARY_IMPL(b200, CUDA, m) {
  m.impl("rms_norm", &rms_norm);
  m.impl("fused_add_rms_norm", &fused_add_rms_norm);
  m.impl("embedding", &embedding);
  m.impl("silu_and_mul", &silu_and_mul);
  m.impl("rope_kv_write", &rope_kv_write);
  m.impl("paged_attention_decode", &paged_attention_decode);
  m.impl("paged_attention_prefill", &paged_attention_prefill);
  m.impl("paged_attention_decode_cp", &paged_attention_decode_cp);
  m.impl("paged_attention_prefill_cp", &paged_attention_prefill_cp);
  m.impl("varlen_attention", &varlen_attention);
  m.impl("topk_softmax", &topk_softmax);
  m.impl("argmax", &argmax);
  m.impl("sample", &sample);
  register_moe_impls(m);
  register_comm_impls(m);
  register_deltanet_impls(m);
  register_gemm_impls(m);
  register_mla_impls(m);
}

// Python module entry so `import vllm_neuron_b200._C` loads the library.
#include <Python.h>
static struct PyModuleDef b200_module = {PyModuleDef_HEAD_INIT, "_C", nullptr, -1, nullptr};
PyMODINIT_FUNC PyInit__C(void) { return PyModule_Create(&b200_module); }
