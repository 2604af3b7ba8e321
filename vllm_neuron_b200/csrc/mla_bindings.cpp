// torch.ops.b200 registration of the MLA decode kernel (csrc/mla_decode.cu).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

extern "C" int b200_mla_decode(void* out, const void* q, const void* cache, const int* block_tables,
                               const int* seq_lens, int B, int Hq, int num_blocks, int block_size, int max_blocks,
                               float scale, float* ws, int num_splits, int* status, cudaStream_t s);

namespace {
using at::Tensor;

void mla_decode(Tensor out, Tensor q, Tensor cache, Tensor block_tables, Tensor seq_lens, double scale,
                c10::optional<Tensor> ws, int64_t num_splits, c10::optional<Tensor> status) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == at::kBFloat16 && q.is_contiguous() && q.dim() == 3 &&
                  q.size(2) == 576,
              "mla_decode: q must be contiguous bf16 [B, Hq, 576]");
  const int B = q.size(0), Hq = q.size(1);
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.numel() == (int64_t)B * Hq * 512,
              "mla_decode: out must be contiguous bf16 [B, Hq, 512]");
  TORCH_CHECK(cache.scalar_type() == at::kBFloat16 && cache.is_contiguous() && cache.dim() == 3 &&
                  cache.size(2) == 576,
              "mla_decode: cache must be contiguous bf16 [num_blocks, block_size, 576]");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && block_tables.is_contiguous() && block_tables.dim() == 2 &&
                  block_tables.size(0) == B,
              "mla_decode: block_tables int32 [B, max_blocks]");
  TORCH_CHECK(seq_lens.scalar_type() == at::kInt && seq_lens.numel() == B, "mla_decode: seq_lens int32 [B]");
  if (num_splits > 1)
    TORCH_CHECK(ws.has_value() && ws->scalar_type() == at::kFloat && ws->numel() >= (int64_t)B * Hq * num_splits * 513,
                "mla_decode: num_splits > 1 needs an fp32 workspace of B * Hq * num_splits * 513");
  c10::cuda::CUDAGuard g(q.device());
  const int rc = b200_mla_decode(out.data_ptr(), q.data_ptr(), cache.data_ptr(), block_tables.data_ptr<int>(),
                                 seq_lens.data_ptr<int>(), B, Hq, cache.size(0), cache.size(1), block_tables.size(1),
                                 (float)scale, ws.has_value() ? ws->data_ptr<float>() : nullptr, num_splits,
                                 status.has_value() ? status->data_ptr<int>() : nullptr,
                                 at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(rc == 0, "b200::mla_decode failed with code ", rc);
}
}  // namespace

void register_mla_ops(torch::Library& m) {
  m.def(
      "mla_decode(Tensor(a!) out, Tensor q, Tensor cache, Tensor block_tables, Tensor seq_lens, float scale, "
      "Tensor(b!)? ws, int num_splits, Tensor? status) -> ()");
}

void register_mla_impls(torch::Library& m) { m.impl("mla_decode", &mla_decode); }
