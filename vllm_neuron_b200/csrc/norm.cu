// RMSNorm and fused residual-add + RMSNorm.
//
// One CTA per row; 16-byte vector loads; fp32 accumulation; the norm weight is fp32.
// out = x * rsqrt(mean(x^2) + eps) * w          (rms_norm)
// r  += x ; out = rms_norm(r)                     (fused_add_rms_norm, r updated in place)
// Semantics: GptOssRMSNorm (vllm_neuron/model/gpt_oss/model_mxfp4.py:101).
#include "common.cuh"
#include "launch_pdl.h"
#include "launch.h"

namespace b200 {

template <typename T, bool kAdd>
__global__ void __launch_bounds__(256) rms_norm_kernel(T* __restrict__ out, const T* __restrict__ x,
                                                       T* __restrict__ residual, const float* __restrict__ w,
                                                       int H, float eps) {
  pdl_wait();  // predecessor output visible (programmatic dependent launch)
  pdl_trigger();
  extern __shared__ float srow[];  // H floats (the pre-norm row)
  __shared__ float red[32];
  const int row = blockIdx.x;
  const T* xr = x + (size_t)row * H;
  T* rr = kAdd ? residual + (size_t)row * H : nullptr;
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    float v = to_float(xr[i]);
    if (kAdd) {
      v += to_float(rr[i]);
      T vt = from_float<T>(v);
      rr[i] = vt;
      v = to_float(vt);  // the stored residual is what the next layer sees
    }
    srow[i] = v;
    ss += v * v;
  }
  float tot = block_sum(ss, red);
  const float inv = rsqrtf(tot / (float)H + eps);
  T* orow = out + (size_t)row * H;
  for (int i = threadIdx.x; i < H; i += blockDim.x) orow[i] = from_float<T>(srow[i] * inv * w[i]);
}

// Vector path: bf16 rows with H % 8 == 0, each thread holds up to kMaxVec 16-byte chunks
// of the row in registers (one read, one write per element).
constexpr int kMaxVec = 4;

template <bool kAdd>
__global__ void __launch_bounds__(256) rms_norm_vec_kernel(__nv_bfloat16* __restrict__ out,
                                                           const __nv_bfloat16* __restrict__ x,
                                                           __nv_bfloat16* __restrict__ residual,
                                                           const float* __restrict__ w, int H, float eps) {
  pdl_wait();  // predecessor output visible (programmatic dependent launch)
  pdl_trigger();
  __shared__ float red[32];
  const int row = blockIdx.x;
  const int nchunk = H / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * H);
  uint4* rr = kAdd ? reinterpret_cast<uint4*>(residual + (size_t)row * H) : nullptr;
  float v[kMaxVec][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < nchunk) {
      uint4 u = xr[c];
      const __nv_bfloat16* hb = reinterpret_cast<const __nv_bfloat16*>(&u);
      if (kAdd) {
        uint4 ru = rr[c];
        const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(&ru);
        uint4 o;
        __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          ob[q] = __float2bfloat16(__bfloat162float(hb[q]) + __bfloat162float(rb[q]));
          v[i][q] = __bfloat162float(ob[q]);
        }
        rr[c] = o;
      } else {
#pragma unroll
        for (int q = 0; q < 8; ++q) v[i][q] = __bfloat162float(hb[q]);
      }
#pragma unroll
      for (int q = 0; q < 8; ++q) ss += v[i][q] * v[i][q];
    }
  }
  const float tot = block_sum(ss, red);
  const float inv = rsqrtf(tot / (float)H + eps);
  uint4* orow = reinterpret_cast<uint4*>(out + (size_t)row * H);
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < nchunk) {
      const float4 w0 = reinterpret_cast<const float4*>(w)[2 * c];
      const float4 w1 = reinterpret_cast<const float4*>(w)[2 * c + 1];
      const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      uint4 o;
      __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
      for (int q = 0; q < 8; ++q) ob[q] = __float2bfloat16(v[i][q] * inv * ww[q]);
      orow[c] = o;
    }
  }
}

template <typename T>
static void launch_norm(void* out, const void* x, void* res, const float* w, int rows, int H, float eps,
                        cudaStream_t s) {
  if (rows == 0) return;
  int threads = H >= 2048 ? 256 : (H >= 512 ? 128 : 64);
  size_t smem = (size_t)H * sizeof(float);
  if (res)
    launch_k(rms_norm_kernel<T, true>, dim3(rows), dim3(threads), smem, s, (T*)out, (const T*)x, (T*)res, w, H, eps);
  else
    launch_k(rms_norm_kernel<T, false>, dim3(rows), dim3(threads), smem, s, (T*)out, (const T*)x, nullptr, w, H, eps);
}

}  // namespace b200

extern "C" int b200_rms_norm(void* out, const void* x, void* residual, const float* w, int rows, int H,
                             float eps, int dtype, cudaStream_t s) {
  using namespace b200;
  if (H > 12288) return kBadShape;  // row staged in <= 48 KB of shared memory
  const bool aligned = ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(x) |
                         reinterpret_cast<uintptr_t>(residual) | reinterpret_cast<uintptr_t>(w)) & 15) == 0;
  if (dtype == kBF16 && H % 8 == 0 && aligned && rows > 0) {
    const int nchunk = H / 8;
    int threads = 32;
    while (threads * kMaxVec < nchunk) threads *= 2;
    if (threads <= 256) {
      if (residual)
        launch_k(rms_norm_vec_kernel<true>, dim3(rows), dim3(threads), 0, s, (__nv_bfloat16*)out, (const __nv_bfloat16*)x,
                                                           (__nv_bfloat16*)residual, w, H, eps);
      else
        launch_k(rms_norm_vec_kernel<false>, dim3(rows), dim3(threads), 0, s, (__nv_bfloat16*)out, (const __nv_bfloat16*)x, nullptr,
                                                            w, H, eps);
      return (int)cudaGetLastError();
    }
  }
  switch (dtype) {
    case kBF16: launch_norm<__nv_bfloat16>(out, x, residual, w, rows, H, eps, s); break;
    case kF16: launch_norm<__half>(out, x, residual, w, rows, H, eps, s); break;
    case kF32: launch_norm<float>(out, x, residual, w, rows, H, eps, s); break;
    default: return kBadShape;
  }
  return (int)cudaGetLastError();
}

// silu(gate) * up for [T, 2I] (gate | up halves), bf16, 16-byte vectors when I % 8 == 0.
namespace b200 {
__global__ void silu_and_mul_kernel(__nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ gu, int I) {
  const int t = blockIdx.x;
  const __nv_bfloat16* g = gu + (size_t)t * 2 * I;
  const __nv_bfloat16* u = g + I;
  __nv_bfloat16* o = out + (size_t)t * I;
  if (I % 8 == 0) {
    for (int c = threadIdx.x; c < I / 8; c += blockDim.x) {
      const uint4 gv = reinterpret_cast<const uint4*>(g)[c];
      const uint4 uv = reinterpret_cast<const uint4*>(u)[c];
      const __nv_bfloat16* gb = reinterpret_cast<const __nv_bfloat16*>(&gv);
      const __nv_bfloat16* ub = reinterpret_cast<const __nv_bfloat16*>(&uv);
      uint4 ov;
      __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&ov);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float x = __bfloat162float(gb[q]);
        ob[q] = __float2bfloat16(x / (1.f + __expf(-x)) * __bfloat162float(ub[q]));
      }
      reinterpret_cast<uint4*>(o)[c] = ov;
    }
  } else {
    for (int i = threadIdx.x; i < I; i += blockDim.x) {
      const float x = __bfloat162float(g[i]);
      o[i] = __float2bfloat16(x / (1.f + __expf(-x)) * __bfloat162float(u[i]));
    }
  }
}
}  // namespace b200

extern "C" int b200_silu_and_mul(void* out, const void* gu, int T, int I, cudaStream_t s) {
  if (T == 0) return 0;
  b200::silu_and_mul_kernel<<<T, 256, 0, s>>>((__nv_bfloat16*)out, (const __nv_bfloat16*)gu, I);
  return (int)cudaGetLastError();
}
