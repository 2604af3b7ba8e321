// FP8 (e4m3) activation quantisation for the FP8 linear layers.
//
// Semantics (the reference's static FP8 paths: model/llama3/quantization.py:176 and
// functional rmsnorm_quant): q = e4m3_satfinite(y / s) with a per-tensor scale s, where y is
// either the activation itself (fp8_quant) or its RMSNorm, optionally after the residual add
// (rms_norm_fp8, the fused "rmsnorm_quant").  The GEMM then multiplies its fp32 accumulator
// by alpha = s * s_w (s_w: the weight's per-tensor scale).
//   * static scale: s read from a device scalar (the checkpoint's input_scale);
//   * dynamic scale: s = max(amax(|x|), 1e-12) / 448, computed on the device by an amax pass
//     (atomicMax on the float bit pattern, exact for non-negative floats), so a call needs no
//     host synchronisation and can be captured in a CUDA graph.
// The quantising kernel also writes alpha = s * s_w for the GEMM (block 0; s_w per tensor or
// per output feature).
#include <cuda_fp8.h>

#include <algorithm>

#include "common.cuh"
#include "launch.h"
#include "launch_pdl.h"

namespace b200 {
namespace fp8 {

constexpr float kE4M3Max = 448.f;
constexpr int kMaxVec = 4;  // 16-byte chunks per thread in the norm kernel (H <= 256 * 4 * 8)

B200_D uint16_t cvt2(float a, float b) {
  return __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
}

// 8 floats / s -> 8 e4m3 bytes (a correctly rounded division, so the bytes equal a host
// quantisation x / s -> e4m3 of the same values)
B200_D uint2 pack8(const float* v, float s) {
  uint2 o;
  o.x = (uint32_t)cvt2(v[0] / s, v[1] / s) | ((uint32_t)cvt2(v[2] / s, v[3] / s) << 16);
  o.y = (uint32_t)cvt2(v[4] / s, v[5] / s) | ((uint32_t)cvt2(v[6] / s, v[7] / s) << 16);
  return o;
}

// amax of |x| over rows x H (row stride ld) into *amax_bits (zeroed by the caller).
__global__ void __launch_bounds__(256) amax_kernel(unsigned* __restrict__ amax_bits, const __nv_bfloat16* __restrict__ x,
                                                   int rows, int H, int ld) {
  pdl_wait();
  pdl_trigger();
  const int nchunk = H / 8;
  float m = 0.f;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < (long long)rows * nchunk;
       i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i / nchunk), c = (int)(i % nchunk);
    const uint4 u = *reinterpret_cast<const uint4*>(x + (size_t)r * ld + c * 8);
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int q = 0; q < 8; ++q) m = fmaxf(m, fabsf(__bfloat162float(h[q])));
  }
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) atomicMax(amax_bits, __float_as_uint(m));
}

B200_D float scale_of(const float* scale, const unsigned* amax_bits) {
  return scale != nullptr ? scale[0] : fmaxf(__uint_as_float(*amax_bits), 1e-12f) / kE4M3Max;
}

// q[r, :] = e4m3(x[r, :] / s); grid-stride over 8-element chunks.
__global__ void __launch_bounds__(256) quant_kernel(uint8_t* __restrict__ q, int ldq, const __nv_bfloat16* __restrict__ x,
                                                    int ldx, int rows, int H, const float* __restrict__ scale,
                                                    const unsigned* __restrict__ amax_bits,
                                                    const float* __restrict__ w_scale, float* __restrict__ alpha,
                                                    int alpha_n) {
  pdl_wait();
  pdl_trigger();
  const float s = scale_of(scale, amax_bits);
  if (blockIdx.x == 0 && alpha != nullptr)
    for (int n = threadIdx.x; n < alpha_n; n += blockDim.x) alpha[n] = s * (w_scale != nullptr ? w_scale[n] : 1.f);
  const int nchunk = H / 8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < (long long)rows * nchunk;
       i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i / nchunk), c = (int)(i % nchunk);
    const uint4 u = *reinterpret_cast<const uint4*>(x + (size_t)r * ldx + c * 8);
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&u);
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = __bfloat162float(h[k]);
    *reinterpret_cast<uint2*>(q + (size_t)r * ldq + c * 8) = pack8(v, s);
  }
}

// One CTA per row: (residual += x), RMSNorm(row) * w, then e4m3 with the static scale.
template <bool kAdd>
__global__ void __launch_bounds__(256) rms_norm_fp8_kernel(uint8_t* __restrict__ q, const __nv_bfloat16* __restrict__ x,
                                                           __nv_bfloat16* __restrict__ residual,
                                                           const float* __restrict__ w, int H, float eps,
                                                           const float* __restrict__ scale) {
  pdl_wait();
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
      const uint4 u = xr[c];
      const __nv_bfloat16* hb = reinterpret_cast<const __nv_bfloat16*>(&u);
      if (kAdd) {
        const uint4 ru = rr[c];
        const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(&ru);
        uint4 o;
        __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          ob[k] = __float2bfloat16(__bfloat162float(hb[k]) + __bfloat162float(rb[k]));
          v[i][k] = __bfloat162float(ob[k]);
        }
        rr[c] = o;
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) v[i][k] = __bfloat162float(hb[k]);
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) ss += v[i][k] * v[i][k];
    }
  }
  const float tot = block_sum(ss, red);
  const float inv = rsqrtf(tot / (float)H + eps);
  const float qs = scale[0];
  uint2* orow = reinterpret_cast<uint2*>(q + (size_t)row * H);
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < nchunk) {
      const float4 w0 = reinterpret_cast<const float4*>(w)[2 * c];
      const float4 w1 = reinterpret_cast<const float4*>(w)[2 * c + 1];
      const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      float y[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) y[k] = __bfloat162float(__float2bfloat16(v[i][k] * inv * ww[k]));
      orow[c] = pack8(y, qs);
    }
  }
}

}  // namespace fp8
}  // namespace b200

using namespace b200;

// q [rows, ldq] e4m3 = x [rows, ldx] bf16 / s; s = *scale (static) or from the amax pass
// (scale null: amax_ws is one u32 of scratch); alpha (optional) [alpha_n] <- s * w_scale[0 .. alpha_n).
extern "C" int b200_fp8_quant(void* q, int ldq, const void* x, int ldx, int rows, int H, const float* scale,
                              unsigned* amax_ws, const float* w_scale, float* alpha, int alpha_n, cudaStream_t s) {
  if (rows < 0 || H <= 0 || H % 8 || ldx % 8 || ldq % 8 || ldx < H || ldq < H) return kBadShape;
  if (((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(x)) & 15)) return kBadAlignment;
  if (scale == nullptr && amax_ws == nullptr) return kBadShape;
  if (rows == 0) return 0;
  const long long chunks = (long long)rows * (H / 8);
  const int grid = (int)std::min<long long>((chunks + 255) / 256, 148 * 8);
  if (scale == nullptr) {
    cudaError_t e = cudaMemsetAsync(amax_ws, 0, sizeof(unsigned), s);
    if (e != cudaSuccess) return (int)e;
    launch_k(fp8::amax_kernel, dim3(grid), dim3(256), 0, s, amax_ws, (const __nv_bfloat16*)x, rows, H, ldx);
  }
  launch_k(fp8::quant_kernel, dim3(grid), dim3(256), 0, s, (uint8_t*)q, ldq, (const __nv_bfloat16*)x, ldx, rows, H,
           scale, (const unsigned*)amax_ws, w_scale, alpha, alpha_n);
  return (int)cudaGetLastError();
}

// Fused (residual add +) RMSNorm + static e4m3 quantisation: q [rows, H] e4m3.
extern "C" int b200_rms_norm_fp8(void* q, const void* x, void* residual, const float* w, int rows, int H, float eps,
                                 const float* scale, cudaStream_t s) {
  if (H % 8 || H > 256 * fp8::kMaxVec * 8 || rows < 0 || scale == nullptr) return kBadShape;
  if (((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(residual) |
        reinterpret_cast<uintptr_t>(w)) & 15))
    return kBadAlignment;
  if (rows == 0) return 0;
  const int nchunk = H / 8;
  int threads = 32;
  while (threads * fp8::kMaxVec < nchunk) threads *= 2;
  if (residual)
    launch_k(fp8::rms_norm_fp8_kernel<true>, dim3(rows), dim3(threads), 0, s, (uint8_t*)q, (const __nv_bfloat16*)x,
             (__nv_bfloat16*)residual, w, H, eps, scale);
  else
    launch_k(fp8::rms_norm_fp8_kernel<false>, dim3(rows), dim3(threads), 0, s, (uint8_t*)q, (const __nv_bfloat16*)x,
             (__nv_bfloat16*)nullptr, w, H, eps, scale);
  return (int)cudaGetLastError();
}
