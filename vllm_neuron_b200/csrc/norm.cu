// RMSNorm and fused residual-add + RMSNorm.
//
// One CTA per row; 16-byte vector loads; fp32 accumulation; the norm weight is fp32.
// out = x * rsqrt(mean(x^2) + eps) * w          (rms_norm)
// r  += x ; out = rms_norm(r)                     (fused_add_rms_norm, r updated in place)
// Semantics: GptOssRMSNorm (vllm_neuron/model/gpt_oss/model_mxfp4.py:101).
#include "common.cuh"
#include "launch.h"

namespace b200 {

template <typename T, bool kAdd>
__global__ void __launch_bounds__(256) rms_norm_kernel(T* __restrict__ out, const T* __restrict__ x,
                                                       T* __restrict__ residual, const float* __restrict__ w,
                                                       int H, float eps) {
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

template <typename T>
static void launch_norm(void* out, const void* x, void* res, const float* w, int rows, int H, float eps,
                        cudaStream_t s) {
  if (rows == 0) return;
  int threads = H >= 2048 ? 256 : (H >= 512 ? 128 : 64);
  size_t smem = (size_t)H * sizeof(float);
  if (res)
    rms_norm_kernel<T, true><<<rows, threads, smem, s>>>((T*)out, (const T*)x, (T*)res, w, H, eps);
  else
    rms_norm_kernel<T, false><<<rows, threads, smem, s>>>((T*)out, (const T*)x, nullptr, w, H, eps);
}

}  // namespace b200

extern "C" int b200_rms_norm(void* out, const void* x, void* residual, const float* w, int rows, int H,
                             float eps, int dtype, cudaStream_t s) {
  using namespace b200;
  if (H > 12288) return kBadShape;  // row staged in <= 48 KB of shared memory
  switch (dtype) {
    case kBF16: launch_norm<__nv_bfloat16>(out, x, residual, w, rows, H, eps, s); break;
    case kF16: launch_norm<__half>(out, x, residual, w, rows, H, eps, s); break;
    case kF32: launch_norm<float>(out, x, residual, w, rows, H, eps, s); break;
    default: return kBadShape;
  }
  return (int)cudaGetLastError();
}
