// torch.ops.b200 registration of the fused NVLink collectives and the IPC plumbing.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

extern "C" {
int b200_comm_alloc(size_t slot_bytes, void** out);
int b200_comm_free(void* p);
int b200_ipc_get_handle(void* p, void* handle64);
int b200_ipc_open_handle(const void* handle64, void** out);
int b200_ipc_close(void* p);
int b200_allreduce_fused(void* const* bases, int rank, int world, size_t slot_bytes, const void* in, void* out,
                         void* residual, const void* bias, const float* w, float eps, int T, int H, int num_blocks,
                         unsigned long long wait_ns, int* status, cudaStream_t s, const int* topk_ids, int k,
                         int E_local, int eoff, int ll);
int b200_sp_boundary(void* const* bases, int rank, int world, size_t slot_bytes, size_t area_bytes, size_t guard_bytes,
                     int slot, const void* in, void* residual, const void* bias, const float* w, float eps, int T, int H,
                     int num_blocks, unsigned long long wait_ns, int* status, cudaStream_t s, const int* topk_ids,
                     int k, int E_local, int eoff);
int b200_kv_export(void* dst, const int64_t* kptr, const int64_t* vptr, int n_layers, const int* blocks, int T, int nh,
                   int row_bytes, int bs, cudaStream_t s);
int b200_kv_import(const void* const* part_base, const int* part_h0, const int* part_nh, int n_parts,
                   const int64_t* kptr, const int64_t* vptr, int n_layers, const int* blocks, int T, int src_T, int h0,
                   int nh, int row_bytes, int bs, int* status, cudaStream_t s);
int b200_ep_dispatch(void* const* bases, int rank, int world, size_t slot_bytes, int cpd, int T, int Tc, int H, int k,
                     int E_local, int t_begin, int t_end, const void* x, const int* ids, const float* w, void* x_recv,
                     int* ids_recv, float* w_recv, int* send_idx, int* status, cudaStream_t s);
int b200_ep_combine(void* const* bases, int rank, int world, size_t slot_bytes, int cpd, int T, int Tc, int H, int k,
                    const void* y_recv, const int* ids_recv, const int* send_idx, void* out, int* status,
                    cudaStream_t s);
}

namespace {
using at::Tensor;

int64_t comm_alloc(int64_t slot_bytes) {
  void* p = nullptr;
  const int rc = b200_comm_alloc((size_t)slot_bytes, &p);
  TORCH_CHECK(rc == 0, "comm_alloc failed: ", rc);
  return reinterpret_cast<int64_t>(p);
}

void comm_free(int64_t p) { b200_comm_free(reinterpret_cast<void*>(p)); }

// Guard ("canary") bytes of device regions: fill a byte range with a pattern, read it back.
void device_fill(int64_t p, int64_t nbytes, int64_t value) {
  const cudaError_t e = cudaMemset(reinterpret_cast<void*>(p), (int)value, (size_t)nbytes);
  TORCH_CHECK(e == cudaSuccess, "device_fill: ", cudaGetErrorString(e));
}

Tensor device_read(int64_t p, int64_t nbytes) {
  Tensor out = at::empty({nbytes}, at::TensorOptions().dtype(at::kByte));
  const cudaError_t e = cudaMemcpy(out.data_ptr(), reinterpret_cast<const void*>(p), (size_t)nbytes,
                                   cudaMemcpyDeviceToHost);
  TORCH_CHECK(e == cudaSuccess, "device_read: ", cudaGetErrorString(e));
  return out;
}

Tensor ipc_get_handle(int64_t p) {
  Tensor h = at::empty({64}, at::TensorOptions().dtype(at::kByte));
  const int rc = b200_ipc_get_handle(reinterpret_cast<void*>(p), h.data_ptr());
  TORCH_CHECK(rc == 0, "cudaIpcGetMemHandle failed: ", rc);
  return h;
}

int64_t ipc_open_handle(Tensor h) {
  TORCH_CHECK(h.numel() == 64 && h.scalar_type() == at::kByte && !h.is_cuda(), "64-byte CPU handle expected");
  void* p = nullptr;
  const int rc = b200_ipc_open_handle(h.contiguous().data_ptr(), &p);
  TORCH_CHECK(rc == 0, "cudaIpcOpenMemHandle failed: ", rc);
  return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t p) { b200_ipc_close(reinterpret_cast<void*>(p)); }

void allreduce_fused(at::IntArrayRef bases, int64_t rank, int64_t slot_bytes, Tensor input, Tensor out,
                     c10::optional<Tensor> residual, c10::optional<Tensor> bias, c10::optional<Tensor> w, double eps,
                     int64_t num_blocks, c10::optional<Tensor> status, int64_t wait_ns,
                     c10::optional<Tensor> topk_ids, int64_t e_local, int64_t e_off, int64_t ll) {
  TORCH_CHECK(input.is_cuda() && input.scalar_type() == at::kBFloat16 && input.is_contiguous(), "bf16 input");
  TORCH_CHECK(out.is_contiguous() && out.scalar_type() == at::kBFloat16, "bf16 out");
  TORCH_CHECK(bases.size() >= 1 && bases.size() <= 8, "1..8 ranks");
  const int H = input.size(-1);
  int T = input.numel() / H, k = 0;
  if (topk_ids.has_value()) {  // route mode: input holds [T * k, H] per-route rows
    TORCH_CHECK(topk_ids->is_cuda() && topk_ids->scalar_type() == at::kInt && topk_ids->is_contiguous() &&
                    topk_ids->dim() == 2,
                "topk_ids: contiguous int32 [T, k]");
    k = topk_ids->size(1);
    TORCH_CHECK((int64_t)topk_ids->size(0) * k == T, "input rows must be T * k");
    T = topk_ids->size(0);
  }
  TORCH_CHECK(out.numel() == (int64_t)T * H, "out must be [T, H]");
  void* ptrs[8];
  for (size_t i = 0; i < bases.size(); ++i) ptrs[i] = reinterpret_cast<void*>(bases[i]);
  if (w.has_value()) {
    TORCH_CHECK(residual.has_value() && residual->is_contiguous() && residual->scalar_type() == at::kBFloat16,
                "fused norm needs a bf16 residual");
    TORCH_CHECK(w->scalar_type() == at::kFloat, "norm weight fp32");
  }
  c10::cuda::CUDAGuard g(input.device());
  const int rc = b200_allreduce_fused(
      ptrs, rank, bases.size(), (size_t)slot_bytes, input.data_ptr(), out.data_ptr(),
      residual.has_value() ? residual->data_ptr() : nullptr, bias.has_value() ? bias->data_ptr() : nullptr,
      w.has_value() ? w->data_ptr<float>() : nullptr, (float)eps, T, H, num_blocks,
      wait_ns > 0 ? (unsigned long long)wait_ns : 0ull, status.has_value() ? status->data_ptr<int>() : nullptr,
      at::cuda::getCurrentCUDAStream().stream(), topk_ids.has_value() ? topk_ids->data_ptr<int>() : nullptr, k,
      (int)e_local, (int)e_off, (int)ll);
  TORCH_CHECK(rc == 0, "b200::allreduce_fused failed with code ", rc);
}
// Sequence-parallel layer boundary (csrc/comm.cu, sp_boundary_kernel); the output is the AG
// area of `slot` (read through comm_view).  input: [T, H] partial, [T * k, H] route rows with
// topk_ids, or None when gemm_scatter has stored the partial rows already.
void sp_boundary(at::IntArrayRef bases, int64_t rank, int64_t slot_bytes, int64_t area_bytes, int64_t guard_bytes,
                 int64_t slot, c10::optional<Tensor> input, Tensor residual, c10::optional<Tensor> bias, Tensor w,
                 double eps, int64_t T, int64_t num_blocks, c10::optional<Tensor> status, int64_t wait_ns,
                 c10::optional<Tensor> topk_ids, int64_t e_local, int64_t e_off) {
  const int world = bases.size();
  TORCH_CHECK(world >= 1 && world <= 8, "1..8 ranks");
  TORCH_CHECK(residual.is_cuda() && residual.scalar_type() == at::kBFloat16 && residual.is_contiguous() &&
                  residual.dim() == 2 && residual.size(0) * world == T,
              "residual: this rank's contiguous bf16 [T / world, H] rows");
  const int H = residual.size(1);
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.numel() == H, "norm weight fp32 [H]");
  if (bias.has_value())
    TORCH_CHECK(bias->scalar_type() == at::kBFloat16 && bias->numel() == H && bias->is_contiguous(), "bias [H] bf16");
  int k = 0;
  if (input.has_value()) {
    TORCH_CHECK(input->scalar_type() == at::kBFloat16 && input->is_contiguous() && input->size(-1) == H, "bf16 input");
    if (topk_ids.has_value()) {
      TORCH_CHECK(topk_ids->scalar_type() == at::kInt && topk_ids->is_contiguous() && topk_ids->dim() == 2 &&
                      topk_ids->size(0) == T,
                  "topk_ids: contiguous int32 [T, k]");
      k = topk_ids->size(1);
      TORCH_CHECK(input->numel() == (int64_t)T * k * H, "route rows must be [T * k, H]");
    } else {
      TORCH_CHECK(input->numel() == T * H, "input must be [T, H]");
    }
  } else {
    TORCH_CHECK(!topk_ids.has_value(), "route mode needs the route rows");
  }
  void* ptrs[8];
  for (int i = 0; i < world; ++i) ptrs[i] = reinterpret_cast<void*>(bases[i]);
  c10::cuda::CUDAGuard g(residual.device());
  const int rc = b200_sp_boundary(
      ptrs, rank, world, (size_t)slot_bytes, (size_t)area_bytes, (size_t)guard_bytes, slot,
      input.has_value() ? input->data_ptr() : nullptr, residual.data_ptr(), bias.has_value() ? bias->data_ptr() : nullptr,
      w.data_ptr<float>(), (float)eps, T, H, num_blocks, wait_ns > 0 ? (unsigned long long)wait_ns : 0ull,
      status.has_value() ? status->data_ptr<int>() : nullptr, at::cuda::getCurrentCUDAStream().stream(),
      topk_ids.has_value() ? topk_ids->data_ptr<int>() : nullptr, k, (int)e_local, (int)e_off);
  TORCH_CHECK(rc == 0, "b200::sp_boundary failed with code ", rc);
}

// A bf16 [rows, cols] tensor over device memory this library owns (a communicator region), on
// the device of `like`; the region outlives every view the communicator hands out.
Tensor comm_view(int64_t ptr, int64_t rows, int64_t cols, Tensor like) {
  TORCH_CHECK(like.is_cuda(), "comm_view: a CUDA tensor gives the device");
  return at::from_blob(reinterpret_cast<void*>(ptr), {rows, cols},
                       at::TensorOptions().dtype(at::kBFloat16).device(like.device()));
}

void kv_export(int64_t dst, Tensor kptr, Tensor vptr, Tensor blocks, int64_t num_tokens, int64_t nh,
               int64_t row_bytes, int64_t bs) {
  TORCH_CHECK(kptr.is_cuda() && kptr.scalar_type() == at::kLong && vptr.scalar_type() == at::kLong &&
                  kptr.numel() == vptr.numel(),
              "device int64 layer pointer tables");
  TORCH_CHECK(blocks.is_cuda() && blocks.scalar_type() == at::kInt && blocks.is_contiguous(), "int32 blocks");
  TORCH_CHECK(blocks.numel() * bs >= num_tokens, "too few blocks for the tokens");
  c10::cuda::CUDAGuard g(kptr.device());
  const int rc = b200_kv_export(reinterpret_cast<void*>(dst), kptr.data_ptr<int64_t>(), vptr.data_ptr<int64_t>(),
                                kptr.numel(), blocks.data_ptr<int>(), num_tokens, nh, row_bytes, bs,
                                at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(rc == 0, "b200::kv_export failed with code ", rc);
}

void kv_import(at::IntArrayRef part_base, at::IntArrayRef part_h0, at::IntArrayRef part_nh, Tensor kptr,
               Tensor vptr, Tensor blocks, int64_t num_tokens, int64_t src_tokens, int64_t h0, int64_t nh,
               int64_t row_bytes, int64_t bs, c10::optional<Tensor> status) {
  TORCH_CHECK(kptr.is_cuda() && kptr.scalar_type() == at::kLong && vptr.scalar_type() == at::kLong &&
                  kptr.numel() == vptr.numel(),
              "device int64 layer pointer tables");
  TORCH_CHECK(blocks.is_cuda() && blocks.scalar_type() == at::kInt && blocks.is_contiguous(), "int32 blocks");
  TORCH_CHECK(blocks.numel() * bs >= num_tokens, "too few blocks for the tokens");
  const int n = part_base.size();
  TORCH_CHECK(n >= 1 && n <= 8 && (int)part_h0.size() == n && (int)part_nh.size() == n, "1..8 producer parts");
  const void* bases[8];
  int ph0[8], pnh[8];
  for (int i = 0; i < n; ++i) {
    bases[i] = reinterpret_cast<const void*>(part_base[i]);
    ph0[i] = part_h0[i];
    pnh[i] = part_nh[i];
  }
  c10::cuda::CUDAGuard g(kptr.device());
  const int rc = b200_kv_import(bases, ph0, pnh, n, kptr.data_ptr<int64_t>(), vptr.data_ptr<int64_t>(), kptr.numel(),
                                blocks.data_ptr<int>(), num_tokens, src_tokens, h0, nh, row_bytes, bs,
                                status.has_value() ? status->data_ptr<int>() : nullptr,
                                at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(rc == 0, "b200::kv_import failed with code ", rc);
}

void ep_dispatch(at::IntArrayRef bases, int64_t rank, int64_t slot_bytes, int64_t cpd, int64_t Tc, int64_t E_local,
                 int64_t t_begin, int64_t t_end, Tensor x, Tensor ids, Tensor w, Tensor x_recv, Tensor ids_recv,
                 Tensor w_recv, Tensor send_idx, c10::optional<Tensor> status) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.dim() == 2, "bf16 x [T, H]");
  TORCH_CHECK(ids.scalar_type() == at::kInt && ids.is_contiguous() && w.scalar_type() == at::kFloat &&
                  w.is_contiguous(),
              "int32 ids / fp32 weights [T, k]");
  const int T = x.size(0), H = x.size(1), k = ids.size(1), world = bases.size();
  TORCH_CHECK(ids.size(0) == T && w.size(0) == T && w.size(1) == k, "ids / weights shape");
  TORCH_CHECK(x_recv.is_contiguous() && x_recv.numel() >= (int64_t)world * T * H && ids_recv.is_contiguous() &&
                  ids_recv.numel() >= (int64_t)world * T * k && w_recv.is_contiguous() &&
                  w_recv.numel() >= (int64_t)world * T * k && send_idx.is_contiguous() &&
                  send_idx.numel() >= (int64_t)T * world,
              "receive buffers too small");
  TORCH_CHECK(world >= 1 && world <= 8, "1..8 ranks");
  void* ptrs[8];
  for (int i = 0; i < world; ++i) ptrs[i] = reinterpret_cast<void*>(bases[i]);
  c10::cuda::CUDAGuard g(x.device());
  const int rc = b200_ep_dispatch(ptrs, rank, world, (size_t)slot_bytes, cpd, T, Tc, H, k, E_local, t_begin, t_end,
                                  x.data_ptr(), ids.data_ptr<int>(), w.data_ptr<float>(), x_recv.data_ptr(),
                                  ids_recv.data_ptr<int>(), w_recv.data_ptr<float>(), send_idx.data_ptr<int>(),
                                  status.has_value() ? status->data_ptr<int>() : nullptr,
                                  at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(rc == 0, "b200::ep_dispatch failed with code ", rc);
}

void ep_combine(at::IntArrayRef bases, int64_t rank, int64_t slot_bytes, int64_t cpd, int64_t Tc, Tensor y_recv,
                Tensor ids_recv, Tensor send_idx, Tensor out, c10::optional<Tensor> status) {
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.dim() == 2,
              "bf16 out [T, H]");
  TORCH_CHECK(y_recv.scalar_type() == at::kBFloat16 && y_recv.is_contiguous(), "bf16 expert outputs");
  const int T = out.size(0), H = out.size(1), world = bases.size();
  const int k = ids_recv.size(-1);
  TORCH_CHECK(y_recv.numel() >= (int64_t)world * T * H && ids_recv.numel() >= (int64_t)world * T * k &&
                  send_idx.numel() >= (int64_t)T * world,
              "buffers too small");
  void* ptrs[8];
  for (int i = 0; i < world; ++i) ptrs[i] = reinterpret_cast<void*>(bases[i]);
  c10::cuda::CUDAGuard g(out.device());
  const int rc = b200_ep_combine(ptrs, rank, world, (size_t)slot_bytes, cpd, T, Tc, H, k, y_recv.data_ptr(),
                                 ids_recv.data_ptr<int>(), send_idx.data_ptr<int>(), out.data_ptr(),
                                 status.has_value() ? status->data_ptr<int>() : nullptr,
                                 at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(rc == 0, "b200::ep_combine failed with code ", rc);
}
}  // namespace

void register_comm_ops(torch::Library& m) {
  m.def("comm_alloc(int slot_bytes) -> int");
  m.def(
      "sp_boundary(int[] bases, int rank, int slot_bytes, int area_bytes, int guard_bytes, int slot, Tensor? input, "
      "Tensor(a!) residual, Tensor? bias, Tensor w, float eps, int T, int num_blocks, Tensor? status, int wait_ns=0, "
      "Tensor? topk_ids=None, int e_local=0, int e_off=0) -> ()");
  m.def("comm_view(int ptr, int rows, int cols, Tensor like) -> Tensor");
  m.def("comm_free(int ptr) -> ()");
  m.def("device_fill(int ptr, int nbytes, int value) -> ()");
  m.def("device_read(int ptr, int nbytes) -> Tensor");
  m.def("ipc_get_handle(int ptr) -> Tensor");
  m.def("ipc_open_handle(Tensor handle) -> int");
  m.def("ipc_close(int ptr) -> ()");
  m.def(
      "allreduce_fused(int[] bases, int rank, int slot_bytes, Tensor input, Tensor(a!) out, Tensor(b!)? residual, "
      "Tensor? bias, Tensor? w, float eps, int num_blocks, Tensor? status, int wait_ns=0, Tensor? topk_ids=None, "
      "int e_local=0, int e_off=0, int ll=0) -> ()");
  m.def(
      "ep_dispatch(int[] bases, int rank, int slot_bytes, int cpd, int Tc, int E_local, int t_begin, int t_end, "
      "Tensor x, Tensor ids, Tensor w, Tensor(a!) x_recv, Tensor(b!) ids_recv, Tensor(c!) w_recv, "
      "Tensor(d!) send_idx, Tensor? status) -> ()");
  m.def(
      "kv_export(int dst, Tensor kptr, Tensor vptr, Tensor blocks, int num_tokens, int nh, int row_bytes, "
      "int bs) -> ()");
  m.def(
      "kv_import(int[] part_base, int[] part_h0, int[] part_nh, Tensor kptr, Tensor vptr, Tensor blocks, "
      "int num_tokens, int src_tokens, int h0, int nh, int row_bytes, int bs, Tensor? status) -> ()");
  m.def(
      "ep_combine(int[] bases, int rank, int slot_bytes, int cpd, int Tc, Tensor y_recv, Tensor ids_recv, "
      "Tensor send_idx, Tensor(a!) out, Tensor? status) -> ()");
}

void register_comm_impls(torch::Library& m) {
  m.impl("allreduce_fused", &allreduce_fused);
  m.impl("sp_boundary", &sp_boundary);
  m.impl("comm_view", &comm_view);
  m.impl("ep_dispatch", &ep_dispatch);
  m.impl("ep_combine", &ep_combine);
  m.impl("kv_export", &kv_export);
  m.impl("kv_import", &kv_import);
}

void register_comm_cpu_impls(torch::Library& m) {
  m.impl("comm_alloc", &comm_alloc);
  m.impl("comm_free", &comm_free);
  m.impl("device_fill", &device_fill);
  m.impl("device_read", &device_read);
  m.impl("ipc_get_handle", &ipc_get_handle);
  m.impl("ipc_open_handle", &ipc_open_handle);
  m.impl("ipc_close", &ipc_close);
}
