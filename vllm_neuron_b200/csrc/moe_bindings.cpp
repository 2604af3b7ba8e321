// torch.ops.b200.moe_mx: validation, workspace carving and launch of the MX MoE forward.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <ATen/ATen.h>
#include <torch/library.h>

#include "launch.h"
#include "moe.h"

namespace {
using at::Tensor;

void moe_mx(Tensor out, Tensor x, Tensor topk_ids, Tensor topk_w, Tensor w13, Tensor sf13, Tensor b13, Tensor w2,
            Tensor sf2, Tensor b2, int64_t expert_offset, int64_t H, int64_t I, bool a_fp4, double alpha,
            double limit, c10::optional<Tensor> status, c10::optional<Tensor> y_routes) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous(), "x: contiguous bf16 CUDA");
  TORCH_CHECK(out.is_contiguous() && out.scalar_type() == at::kBFloat16, "out: contiguous bf16");
  TORCH_CHECK(topk_ids.scalar_type() == at::kInt && topk_ids.is_contiguous(), "topk_ids: contiguous int32");
  TORCH_CHECK(topk_w.scalar_type() == at::kFloat && topk_w.is_contiguous(), "topk_w: contiguous fp32");
  TORCH_CHECK(b13.scalar_type() == at::kFloat && b2.scalar_type() == at::kFloat, "biases fp32");
  TORCH_CHECK(w13.scalar_type() == at::kByte && w2.scalar_type() == at::kByte, "weights uint8 (packed MX)");
  TORCH_CHECK(x.size(1) == H, "x hidden mismatch");
  b200::MoeShape sh{};
  sh.T = x.size(0);
  sh.k = topk_ids.size(1);
  sh.E_local = w13.size(0);
  sh.expert_offset = expert_offset;
  sh.H = H;
  sh.I = I;
  sh.K1p = (H + 127) / 128 * 128;
  sh.K2p = (I + 127) / 128 * 128;
  sh.a_fp4 = a_fp4 ? 1 : 0;
  const int routes = sh.T * sh.k;
  sh.nt = routes <= 512 ? 16 : (routes <= 2048 ? 32 : 128);
  const int64_t tw = a_fp4 ? 64 : 128;
  TORCH_CHECK(w13.dim() == 5 && w13.size(1) == (2 * I + 127) / 128 && w13.size(2) == sh.K1p / 128 &&
                  w13.size(3) == 128 && w13.size(4) == tw && w13.is_contiguous(),
              "w13 must be contiguous tiles [E, 2I/128, K1p/128, 128, 64 (fp4) | 128 (fp8)]");
  TORCH_CHECK(w2.dim() == 5 && w2.size(1) == (H + 127) / 128 && w2.size(2) == sh.K2p / 128 && w2.size(3) == 128 &&
                  w2.size(4) == tw && w2.is_contiguous(),
              "w2 must be contiguous tiles [E, H/128, K2p/128, 128, 64 | 128]");
  TORCH_CHECK(sf13.numel() == (int64_t)sh.E_local * ((2 * I + 127) / 128) * (sh.K1p / 128) * 512, "sf13 atoms size");
  TORCH_CHECK(sf2.numel() == (int64_t)sh.E_local * ((H + 127) / 128) * (sh.K2p / 128) * 512, "sf2 atoms size");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(w13.data_ptr()) % 32 == 0 && reinterpret_cast<uintptr_t>(w2.data_ptr()) % 32 == 0,
              "weights must be 32-byte aligned");
  int64_t sizes[12];
  b200_moe_workspace_sizes(&sh, sizes);
  int64_t offs[12], total = 0;
  for (int i = 0; i < 12; ++i) {
    offs[i] = total;
    total += (sizes[i] + 255) / 256 * 256;
  }
  c10::cuda::CUDAGuard g(x.device());
  Tensor buf = at::empty({total}, x.options().dtype(at::kByte));
  uint8_t* base = buf.data_ptr<uint8_t>();
  b200::MoeWorkspace ws{};
  ws.offsets = reinterpret_cast<int*>(base + offs[0]);
  ws.atom_base = reinterpret_cast<int*>(base + offs[1]);
  ws.cursor = reinterpret_cast<int*>(base + offs[2]);
  ws.row_route = reinterpret_cast<int*>(base + offs[3]);
  ws.tiles = reinterpret_cast<int*>(base + offs[4]);
  ws.num_tiles = reinterpret_cast<int*>(base + offs[5]);
  ws.xq = base + offs[6];
  ws.sf1 = base + offs[7];
  ws.act = reinterpret_cast<uint16_t*>(base + offs[8]);
  ws.aq = base + offs[9];
  ws.sf2 = base + offs[10];
  ws.y = reinterpret_cast<uint16_t*>(base + offs[11]);
  if (y_routes.has_value()) {  // per-route rows for the caller (no per-token sum here)
    TORCH_CHECK(y_routes->is_contiguous() && y_routes->scalar_type() == at::kBFloat16 &&
                    y_routes->numel() == (int64_t)sh.T * sh.k * H,
                "y_routes: contiguous bf16 [T * k, H]");
    ws.y = reinterpret_cast<uint16_t*>(y_routes->data_ptr());
  }
  int* st = status.has_value() ? status->data_ptr<int>() : nullptr;
  const int rc = b200_moe_mx_forward(y_routes.has_value() ? nullptr : out.data_ptr(), x.data_ptr(), topk_ids.data_ptr<int>(), topk_w.data_ptr<float>(),
                                     w13.data_ptr(), sf13.data_ptr<uint8_t>(), b13.data_ptr<float>(), w2.data_ptr(),
                                     sf2.data_ptr<uint8_t>(), b2.data_ptr<float>(), &sh, (float)alpha, (float)limit,
                                     &ws, st, at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(rc == 0, "b200::moe_mx failed with code ", rc);
}
void moe_bf16(Tensor out, Tensor x, Tensor topk_ids, Tensor topk_w, Tensor w13, Tensor b13, Tensor w2, Tensor b2,
              int64_t expert_offset, int64_t H, int64_t I, double alpha, double limit, c10::optional<Tensor> status) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous(), "x: contiguous bf16 CUDA");
  TORCH_CHECK(out.is_contiguous() && out.scalar_type() == at::kBFloat16, "out: contiguous bf16");
  TORCH_CHECK(topk_ids.scalar_type() == at::kInt && topk_ids.is_contiguous(), "topk_ids: contiguous int32");
  TORCH_CHECK(topk_w.scalar_type() == at::kFloat && topk_w.is_contiguous(), "topk_w: contiguous fp32");
  TORCH_CHECK(b13.scalar_type() == at::kFloat && b2.scalar_type() == at::kFloat, "biases fp32");
  TORCH_CHECK(w13.scalar_type() == at::kBFloat16 && w2.scalar_type() == at::kBFloat16, "bf16 expert weights");
  TORCH_CHECK(x.size(1) == H && H % 8 == 0 && I % 8 == 0, "H and I must be multiples of 8");
  b200::MoeShape sh{};
  sh.T = x.size(0);
  sh.k = topk_ids.size(1);
  sh.E_local = w13.size(0);
  sh.expert_offset = expert_offset;
  sh.H = H;
  sh.I = I;
  sh.K1p = (H + 63) / 64 * 64;
  sh.K2p = (I + 63) / 64 * 64;
  sh.a_fp4 = 2;
  const int routes = sh.T * sh.k;
  sh.nt = routes <= 512 ? 16 : (routes <= 2048 ? 32 : 128);
  TORCH_CHECK(w13.dim() == 5 && w13.size(1) == (2 * I + 127) / 128 && w13.size(2) == sh.K1p / 64 &&
                  w13.size(3) == 128 && w13.size(4) == 64 && w13.is_contiguous(),
              "w13 must be contiguous bf16 tiles [E, 2I/128, K1p/64, 128, 64]");
  TORCH_CHECK(w2.dim() == 5 && w2.size(1) == (H + 127) / 128 && w2.size(2) == sh.K2p / 64 && w2.size(3) == 128 &&
                  w2.size(4) == 64 && w2.is_contiguous(),
              "w2 must be contiguous bf16 tiles [E, H/128, K2p/64, 128, 64]");
  int64_t sizes[12];
  b200_moe_workspace_sizes(&sh, sizes);
  int64_t offs[12], total = 0;
  for (int i = 0; i < 12; ++i) {
    offs[i] = total;
    total += (sizes[i] + 255) / 256 * 256;
  }
  c10::cuda::CUDAGuard g(x.device());
  Tensor buf = at::empty({total}, x.options().dtype(at::kByte));
  uint8_t* base = buf.data_ptr<uint8_t>();
  b200::MoeWorkspace ws{};
  ws.offsets = reinterpret_cast<int*>(base + offs[0]);
  ws.atom_base = reinterpret_cast<int*>(base + offs[1]);
  ws.cursor = reinterpret_cast<int*>(base + offs[2]);
  ws.row_route = reinterpret_cast<int*>(base + offs[3]);
  ws.tiles = reinterpret_cast<int*>(base + offs[4]);
  ws.num_tiles = reinterpret_cast<int*>(base + offs[5]);
  ws.xq = base + offs[6];
  ws.sf1 = base + offs[7];
  ws.act = reinterpret_cast<uint16_t*>(base + offs[8]);
  ws.aq = base + offs[9];
  ws.sf2 = base + offs[10];
  ws.y = reinterpret_cast<uint16_t*>(base + offs[11]);
  int* st = status.has_value() ? status->data_ptr<int>() : nullptr;
  const int rc = b200_moe_bf16_forward(out.data_ptr(), x.data_ptr(), topk_ids.data_ptr<int>(),
                                       topk_w.data_ptr<float>(), w13.data_ptr(), b13.data_ptr<float>(), w2.data_ptr(),
                                       b2.data_ptr<float>(), &sh, (float)alpha, (float)limit, &ws, st,
                                       at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(rc == 0, "b200::moe_bf16 failed with code ", rc);
}
void moe_route_sum(Tensor out, Tensor y, Tensor topk_ids, int64_t e_local, int64_t e_off) {
  TORCH_CHECK(out.is_contiguous() && y.is_contiguous() && out.scalar_type() == at::kBFloat16 &&
                  y.scalar_type() == at::kBFloat16 && topk_ids.scalar_type() == at::kInt && topk_ids.is_contiguous(),
              "moe_route_sum: bf16 out [T, H], y [T * k, H], int32 topk_ids [T, k]");
  const int T = out.size(0), H = out.size(1), k = topk_ids.size(1);
  TORCH_CHECK(y.numel() == (int64_t)T * k * H, "moe_route_sum: y rows");
  c10::cuda::CUDAGuard g(out.device());
  const int rc = b200_moe_route_sum(out.data_ptr(), y.data_ptr(), topk_ids.data_ptr<int>(), T, k, (int)e_local,
                                    (int)e_off, H, at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(rc == 0, "b200::moe_route_sum failed with code ", rc);
}
}  // namespace

void register_moe_ops(torch::Library& m) {
  m.def(
      "moe_bf16(Tensor(a!) out, Tensor x, Tensor topk_ids, Tensor topk_w, Tensor w13, Tensor b13, Tensor w2, "
      "Tensor b2, int expert_offset, int H, int I, float alpha, float limit, Tensor? status) -> ()");
  m.def(
      "moe_mx(Tensor(a!) out, Tensor x, Tensor topk_ids, Tensor topk_w, Tensor w13, Tensor sf13, Tensor b13, "
      "Tensor w2, Tensor sf2, Tensor b2, int expert_offset, int H, int I, bool a_fp4, float alpha, float limit, "
      "Tensor? status, Tensor(b!)? y_routes=None) -> ()");
  m.def("moe_route_sum(Tensor(a!) out, Tensor y, Tensor topk_ids, int e_local, int e_off) -> ()");
}

void register_moe_impls(torch::Library& m) {
  m.impl("moe_mx", &moe_mx);
  m.impl("moe_route_sum", &moe_route_sum);
  m.impl("moe_bf16", &moe_bf16);
}
