// Fused MoE router for decode-sized batches: logits = x W^T + b, the k largest (ties -> lower
// expert id) and a softmax over those k (the GPT-OSS order; with renormalisation it equals
// softmax -> top-k -> renormalise, the Qwen order), in one kernel.
//
// One CTA of 256 threads per token: the token's row is staged in shared memory, each warp
// computes the dot products of a strided subset of experts with 16-byte loads of the router
// weight (which stays in L2 across the token CTAs), then one warp selects the top k.
// Replaces a GEMM launch, a cast and the top-k launch per layer in the decode graph; large
// (prefill) batches use the GEMM path instead, where re-reading the router weight per token
// would cost more than it saves.
#include "common.cuh"

namespace b200 {

constexpr int kRouterMaxE = 1024;
constexpr int kRouterMaxH = 8192;

__global__ void __launch_bounds__(256) router_topk_kernel(int* __restrict__ ids, float* __restrict__ wout,
                                                          const __nv_bfloat16* __restrict__ x,
                                                          const __nv_bfloat16* __restrict__ W,
                                                          const __nv_bfloat16* __restrict__ bias, int E, int H,
                                                          int k) {
  __shared__ __align__(16) __nv_bfloat16 xs[kRouterMaxH];
  __shared__ float logit[kRouterMaxE];
  const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nch = H / 8;  // 16-byte chunks per row
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)t * H);
  uint4* xs4 = reinterpret_cast<uint4*>(xs);
  for (int c = threadIdx.x; c < nch; c += blockDim.x) xs4[c] = xr[c];
  __syncthreads();
  for (int e = warp; e < E; e += 8) {
    const uint4* wr = reinterpret_cast<const uint4*>(W + (size_t)e * H);
    float acc = 0.f;
    for (int c = lane; c < nch; c += 32) {
      const uint4 a = xs4[c], b = wr[c];
      const __nv_bfloat162* pa = reinterpret_cast<const __nv_bfloat162*>(&a);
      const __nv_bfloat162* pb = reinterpret_cast<const __nv_bfloat162*>(&b);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 fa = __bfloat1622float2(pa[i]), fb = __bfloat1622float2(pb[i]);
        acc += fa.x * fb.x + fa.y * fb.y;
      }
    }
    acc = warp_sum(acc);
    if (lane == 0) logit[e] = acc + (bias ? __bfloat162float(bias[e]) : 0.f);
  }
  __syncthreads();
  if (warp != 0) return;
  float sel_v[16];
  int sel_i[16];
  for (int j = 0; j < k; ++j) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int e = lane; e < E; e += 32) {
      const float v = logit[e];
      if (v > bv || (v == bv && e < bi)) {
        bv = v;
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    sel_v[j] = bv;
    sel_i[j] = bi;
    __syncwarp();
    if (lane == 0 && bi >= 0 && bi < E) logit[bi] = -INFINITY;
    __syncwarp();
  }
  if (lane == 0) {
    const float m = sel_v[0];
    float s = 0.f;
    for (int j = 0; j < k; ++j) s += __expf(sel_v[j] - m);
    for (int j = 0; j < k; ++j) {
      ids[(size_t)t * k + j] = sel_i[j];
      wout[(size_t)t * k + j] = __expf(sel_v[j] - m) / s;
    }
  }
}

}  // namespace b200

using namespace b200;

extern "C" int b200_router_topk(int* ids, float* weights, const void* x, const void* w, const void* bias, int T,
                                int E, int H, int k, cudaStream_t s) {
  if (E > kRouterMaxE || H > kRouterMaxH || H % 8 || k > 16 || k > E) return kBadShape;
  if (T == 0) return 0;
  router_topk_kernel<<<T, 256, 0, s>>>(ids, weights, (const __nv_bfloat16*)x, (const __nv_bfloat16*)w,
                                       (const __nv_bfloat16*)bias, E, H, k);
  return (int)cudaGetLastError();
}
