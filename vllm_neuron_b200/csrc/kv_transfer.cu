// Device-side KV transfer between two engines on one host (disaggregated prefill / decode).
//
// The reference moves a request's KV between engines with NIXL reads of the remote blocks
// (vllm/kv_connector/neuron_nixl_connector.py:318-470, head_ratio / seq_ratio mapping).  Here
// the producer (prefill) engine gathers the request's KV from its paged cache into a region of
// a device pool that it shares by CUDA IPC, and the consumer (decode) engine copies that region
// straight into its own cache blocks with plain loads from the producer's memory (NVLink when
// the engines sit on different GPUs).  No host copy, no file payload.
//
// Pool region of one producer rank for one request: [layer][k | v][token][head][d] in the
// cache's element type (bf16 or fp8), heads = the producer rank's kv heads.
//   export: cache[layer][blk(t)][h][off(t)][:] -> region          (one CTA per (8 tokens, layer, k|v))
//   import: for every kv head h the consumer rank owns, the producer part holding h supplies
//           region[layer][kv][t][h - part.h0][:] -> cache[layer][blk'(t)][h - h0][off'(t)][:]
//           for t < T (the region holds src_T >= T tokens)
// Rows move as 16-byte vectors (head_dim * element size is a multiple of 16).
#include "common.cuh"
#include "launch.h"

namespace b200 {
namespace {

constexpr int kMaxParts = 8;
constexpr int kTokPerCta = 8;  // a CTA moves 8 tokens x all heads of one (layer, k|v)

struct KvParts {
  const uint8_t* base[kMaxParts];  // producer regions (peer or local device memory)
  int h0[kMaxParts], nh[kMaxParts];
  int n;
};

__global__ void __launch_bounds__(256) kv_export_kernel(uint8_t* __restrict__ dst, const int64_t* __restrict__ kptr,
                                                        const int64_t* __restrict__ vptr,
                                                        const int* __restrict__ blocks, int T, int nh, int row_bytes,
                                                        int bs) {
  const int lk = blockIdx.y, layer = lk >> 1, kv = lk & 1;
  const uint8_t* cache = reinterpret_cast<const uint8_t*>(kv ? vptr[layer] : kptr[layer]);
  const int vec = row_bytes / 16, per_tok = nh * vec;
  const int t0 = blockIdx.x * kTokPerCta, t1 = min(T, t0 + kTokPerCta);
  for (int i = threadIdx.x; i < (t1 - t0) * per_tok; i += blockDim.x) {
    const int t = t0 + i / per_tok, h = (i % per_tok) / vec, c = i % vec;
    const int blk = blocks[t / bs], off = t % bs;
    const uint4* src = reinterpret_cast<const uint4*>(cache + (((size_t)blk * nh + h) * bs + off) * row_bytes);
    uint8_t* out = dst + (((size_t)lk * T + t) * nh + h) * row_bytes;
    reinterpret_cast<uint4*>(out)[c] = src[c];
  }
}

__global__ void __launch_bounds__(256) kv_import_kernel(KvParts parts, const int64_t* __restrict__ kptr,
                                                        const int64_t* __restrict__ vptr,
                                                        const int* __restrict__ blocks, int T, int src_T, int h0,
                                                        int nh, int row_bytes, int bs, int* status) {
  const int lk = blockIdx.y, layer = lk >> 1, kv = lk & 1;
  uint8_t* cache = reinterpret_cast<uint8_t*>(kv ? vptr[layer] : kptr[layer]);
  const int vec = row_bytes / 16, per_tok = nh * vec;
  const int t0 = blockIdx.x * kTokPerCta, t1 = min(T, t0 + kTokPerCta);
  for (int i = threadIdx.x; i < (t1 - t0) * per_tok; i += blockDim.x) {
    const int t = t0 + i / per_tok, h = (i % per_tok) / vec, c = i % vec, gh = h0 + h;
    int p = 0;
    while (p < parts.n && !(gh >= parts.h0[p] && gh < parts.h0[p] + parts.nh[p])) ++p;
    if (p == parts.n) {  // no producer part holds this head: record it, leave the row
      if (status) atomicCAS(status, 0, kBadIndex);
      continue;
    }
    const int blk = blocks[t / bs], off = t % bs;
    const uint4* src = reinterpret_cast<const uint4*>(
        parts.base[p] + (((size_t)lk * src_T + t) * parts.nh[p] + (gh - parts.h0[p])) * row_bytes);
    reinterpret_cast<uint4*>(cache + (((size_t)blk * nh + h) * bs + off) * row_bytes)[c] = src[c];
  }
}

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" int b200_kv_export(void* dst, const int64_t* kptr, const int64_t* vptr, int n_layers, const int* blocks,
                              int T, int nh, int row_bytes, int bs, cudaStream_t s) {
  if (T < 0 || n_layers < 1 || nh < 1 || row_bytes % 16 || bs < 1 || n_layers > 32768) return kBadShape;
  if (T == 0) return 0;
  kv_export_kernel<<<dim3(cdiv(T, kTokPerCta), 2 * n_layers), 256, 0, s>>>(static_cast<uint8_t*>(dst), kptr, vptr,
                                                                           blocks, T, nh, row_bytes, bs);
  return (int)cudaGetLastError();
}

extern "C" int b200_kv_import(const void* const* part_base, const int* part_h0, const int* part_nh, int n_parts,
                              const int64_t* kptr, const int64_t* vptr, int n_layers, const int* blocks, int T,
                              int src_T, int h0, int nh, int row_bytes, int bs, int* status, cudaStream_t s) {
  if (T < 0 || src_T < T || n_layers < 1 || nh < 1 || row_bytes % 16 || bs < 1 || n_parts < 1 || n_parts > kMaxParts ||
      n_layers > 32768)
    return kBadShape;
  if (T == 0) return 0;
  KvParts parts{};
  for (int i = 0; i < n_parts; ++i) {
    parts.base[i] = static_cast<const uint8_t*>(part_base[i]);
    parts.h0[i] = part_h0[i];
    parts.nh[i] = part_nh[i];
  }
  parts.n = n_parts;
  kv_import_kernel<<<dim3(cdiv(T, kTokPerCta), 2 * n_layers), 256, 0, s>>>(parts, kptr, vptr, blocks, T, src_T, h0,
                                                                           nh, row_bytes, bs, status);
  return (int)cudaGetLastError();
}
