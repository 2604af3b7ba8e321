// Fused rotary embedding + paged KV-cache write (+ optional per-head QK RMSNorm).
//
// qkv [T, stride] holds q (nq heads), k (nkv heads), v (nkv heads) of head_dim d.
// In place: optional q/k RMSNorm (Qwen3 QK-norm), rotation of the leading
// `rotary_dim` dims of q and k in split-half form (x1*c - x2*s, x2*c + x1*s).
// Then k and v of token t are stored at slot_mapping[t] of the HND cache
// [num_blocks, nkv, block_size, d]; a negative slot is padding and is skipped;
// an out-of-range block writes kBadIndex to *status and is skipped.
// Semantics: functional/attention/qkv.py:296 (in-kernel cache write) and
// GptOssRotaryEmbedding (model/gpt_oss/model_mxfp4.py:141-197).
#include "common.cuh"
#include "launch_pdl.h"
#include "launch.h"

namespace b200 {

template <typename T, typename CT>
__global__ void __launch_bounds__(256) rope_kv_kernel(T* __restrict__ qkv, const int64_t* __restrict__ pos,
                                                      const float* __restrict__ cos_sin, CT* __restrict__ kc,
                                                      CT* __restrict__ vc, const int64_t* __restrict__ slots,
                                                      int nq, int nkv, int d, int rd, int stride, int bs,
                                                      int num_blocks, float inv_ks, float inv_vs,
                                                      const float* __restrict__ qn, const float* __restrict__ kn,
                                                      float eps, int* status) {
  pdl_wait();  // predecessor output visible (programmatic dependent launch)
  pdl_trigger();
  const int t = blockIdx.x;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int64_t p = pos[t];
  const float* cs = cos_sin + p * rd;
  const int half = rd / 2;
  T* row = qkv + (size_t)t * stride;
  const int64_t slot = slots[t];
  int64_t blk = slot >= 0 ? slot / bs : -1;
  const int off = slot >= 0 ? (int)(slot % bs) : 0;
  if (blk >= num_blocks) {
    if (status) atomicCAS(status, 0, kBadIndex);
    blk = -1;
  }
  // heads: [0, nq) q, [nq, nq+nkv) k, [nq+nkv, nq+2nkv) v
  for (int h = wid; h < nq + 2 * nkv; h += nw) {
    T* x = row + (size_t)h * d;
    const bool is_v = h >= nq + nkv;
    const bool is_k = !is_v && h >= nq;
    if (!is_v) {
      float scale = 1.f;
      const float* nw_ = is_k ? kn : qn;
      if (nw_ != nullptr) {
        float ss = 0.f;
        for (int i = lane; i < d; i += 32) {
          float v = to_float(x[i]);
          ss += v * v;
        }
        ss = warp_sum(ss);
        scale = rsqrtf(ss / d + eps);
      }
      // rotate pairs (i, i+half) for i < half; copy (normed) dims >= rd
      for (int i = lane; i < half; i += 32) {
        float a = to_float(x[i]) * scale, b = to_float(x[i + half]) * scale;
        if (nw_) {
          a *= nw_[i];
          b *= nw_[i + half];
        }
        const float c = cs[i], s = cs[half + i];
        x[i] = from_float<T>(a * c - b * s);
        x[i + half] = from_float<T>(b * c + a * s);
      }
      if (nw_ != nullptr) {
        for (int i = rd + lane; i < d; i += 32) x[i] = from_float<T>(to_float(x[i]) * scale * nw_[i]);
      }
      __syncwarp();
    }
    if ((is_k || is_v) && blk >= 0) {
      const int kh = is_k ? h - nq : h - nq - nkv;
      CT* dst = (is_k ? kc : vc) + (((size_t)blk * nkv + kh) * bs + off) * d;
      const float inv = is_k ? inv_ks : inv_vs;
      for (int i = lane; i < d; i += 32) dst[i] = from_float<CT>(to_float(x[i]) * inv);
    }
  }
}

// Fast path (bf16 q/k/v, full rotary, no QK-norm): one thread per (head, group of 4 rotary
// pairs); 8-byte vector loads of both halves, 16-byte cos/sin loads, 8-byte cache stores.
template <typename CT>
__global__ void __launch_bounds__(256) rope_kv_vec_kernel(__nv_bfloat16* __restrict__ qkv,
                                                          const int64_t* __restrict__ pos,
                                                          const float* __restrict__ cos_sin, CT* __restrict__ kc,
                                                          CT* __restrict__ vc, const int64_t* __restrict__ slots,
                                                          int nq, int nkv, int d, int stride, int bs, int num_blocks,
                                                          float inv_ks, float inv_vs, int* status) {
  pdl_wait();  // predecessor output visible (programmatic dependent launch)
  pdl_trigger();
  const int t = blockIdx.x;
  const int half = d / 2, g4 = half / 4;  // groups of 4 pairs per head
  const int64_t p = pos[t];
  const float* cs = cos_sin + p * d;
  __nv_bfloat16* row = qkv + (size_t)t * stride;
  const int64_t slot = slots[t];
  int64_t blk = slot >= 0 ? slot / bs : -1;
  const int off = slot >= 0 ? (int)(slot % bs) : 0;
  if (blk >= num_blocks) {
    if (status && threadIdx.x == 0) atomicCAS(status, 0, kBadIndex);
    blk = -1;
  }
  const int nrot = (nq + nkv) * g4;
  const int nv = nkv * (d / 4);
  for (int i = threadIdx.x; i < nrot + nv; i += blockDim.x) {
    if (i < nrot) {
      const int h = i / g4, g = i % g4;
      __nv_bfloat16* x = row + (size_t)h * d;
      const uint2 a2 = *reinterpret_cast<const uint2*>(x + 4 * g);
      const uint2 b2 = *reinterpret_cast<const uint2*>(x + half + 4 * g);
      const float4 c = *reinterpret_cast<const float4*>(cs + 4 * g);
      const float4 sn = *reinterpret_cast<const float4*>(cs + half + 4 * g);
      const __nv_bfloat16* a = reinterpret_cast<const __nv_bfloat16*>(&a2);
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&b2);
      const float cc[4] = {c.x, c.y, c.z, c.w}, ss[4] = {sn.x, sn.y, sn.z, sn.w};
      float ra[4], rb[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float av = __bfloat162float(a[q]), bv = __bfloat162float(b[q]);
        ra[q] = av * cc[q] - bv * ss[q];
        rb[q] = bv * cc[q] + av * ss[q];
      }
      uint2 oa, ob;
      __nv_bfloat16* pa = reinterpret_cast<__nv_bfloat16*>(&oa);
      __nv_bfloat16* pb = reinterpret_cast<__nv_bfloat16*>(&ob);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        pa[q] = __float2bfloat16(ra[q]);
        pb[q] = __float2bfloat16(rb[q]);
      }
      *reinterpret_cast<uint2*>(x + 4 * g) = oa;
      *reinterpret_cast<uint2*>(x + half + 4 * g) = ob;
      if (h >= nq && blk >= 0) {
        CT* dst = kc + (((size_t)blk * nkv + (h - nq)) * bs + off) * d;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          dst[4 * g + q] = from_float<CT>(__bfloat162float(pa[q]) * inv_ks);
          dst[half + 4 * g + q] = from_float<CT>(__bfloat162float(pb[q]) * inv_ks);
        }
      }
    } else if (blk >= 0) {
      const int j = i - nrot, h = j / (d / 4), c4 = j % (d / 4);
      const __nv_bfloat16* x = row + (size_t)(nq + nkv + h) * d + 4 * c4;
      CT* dst = vc + (((size_t)blk * nkv + h) * bs + off) * d + 4 * c4;
      if constexpr (sizeof(CT) == 2) {
        *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(x);
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) dst[q] = from_float<CT>(__bfloat162float(x[q]) * inv_vs);
      }
    }
  }
}

template <typename T>
static int launch_rope(void* qkv, const int64_t* pos, const float* cs, void* kc, void* vc, const int64_t* slots,
                       int T_, int nq, int nkv, int d, int rd, int stride, int bs, int nb, float ks, float vs,
                       const float* qn, const float* kn, float eps, int cache_dtype, int* status, cudaStream_t s) {
  if (T_ == 0) return 0;
  const int threads = 128;
  if (cache_dtype == kFP8E4M3) {
    launch_k(rope_kv_kernel<T, __nv_fp8_e4m3>, dim3(T_), dim3(threads), 0, s, (T*)qkv, pos, cs, (__nv_fp8_e4m3*)kc,
                                                            (__nv_fp8_e4m3*)vc, slots, nq, nkv, d, rd, stride, bs, nb,
                                                            1.f / ks, 1.f / vs, qn, kn, eps, status);
  } else {
    launch_k(rope_kv_kernel<T, T>, dim3(T_), dim3(threads), 0, s, (T*)qkv, pos, cs, (T*)kc, (T*)vc, slots, nq, nkv, d, rd, stride,
                                                bs, nb, 1.f, 1.f, qn, kn, eps, status);
  }
  return (int)cudaGetLastError();
}

template <typename T>
__global__ void embedding_kernel(T* __restrict__ out, const int64_t* __restrict__ ids, const T* __restrict__ table,
                                 int rows, int H, int64_t start) {
  const int t = blockIdx.x;
  const int64_t r = ids[t] - start;
  T* o = out + (size_t)t * H;
  if (r < 0 || r >= rows) {
    for (int i = threadIdx.x; i < H; i += blockDim.x) o[i] = from_float<T>(0.f);
    return;
  }
  const T* src = table + (size_t)r * H;
  if ((H * sizeof(T)) % 16 == 0) {
    const int4* s4 = reinterpret_cast<const int4*>(src);
    int4* o4 = reinterpret_cast<int4*>(o);
    for (int i = threadIdx.x; i < (int)(H * sizeof(T) / 16); i += blockDim.x) o4[i] = s4[i];
  } else {
    for (int i = threadIdx.x; i < H; i += blockDim.x) o[i] = src[i];
  }
}

}  // namespace b200

extern "C" int b200_rope_kv_write(void* qkv, const int64_t* positions, const float* cos_sin, void* k_cache,
                                  void* v_cache, const int64_t* slot_mapping, int T, int nq, int nkv, int d,
                                  int rotary_dim, int qkv_stride, int block_size, int num_blocks, float k_scale,
                                  float v_scale, const float* q_norm_w, const float* k_norm_w, float norm_eps,
                                  int dtype, int cache_dtype, int* status, cudaStream_t s) {
  using namespace b200;
  if (rotary_dim > d || rotary_dim % 2) return kBadShape;
  const bool aligned = ((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(cos_sin)) & 15) == 0 &&
                       (qkv_stride % 8) == 0;
  if (dtype == kBF16 && rotary_dim == d && d % 8 == 0 && q_norm_w == nullptr && k_norm_w == nullptr && aligned &&
      T > 0) {
    const int work = (nq + nkv) * (d / 8) + nkv * (d / 4);
    const int threads = work >= 256 ? 256 : ((work + 31) / 32) * 32;
    if (cache_dtype == kFP8E4M3)
      launch_k(rope_kv_vec_kernel<__nv_fp8_e4m3>, dim3(T), dim3(threads), 0, s, 
          (__nv_bfloat16*)qkv, positions, cos_sin, (__nv_fp8_e4m3*)k_cache, (__nv_fp8_e4m3*)v_cache, slot_mapping, nq,
          nkv, d, qkv_stride, block_size, num_blocks, 1.f / k_scale, 1.f / v_scale, status);
    else
      launch_k(rope_kv_vec_kernel<__nv_bfloat16>, dim3(T), dim3(threads), 0, s, 
          (__nv_bfloat16*)qkv, positions, cos_sin, (__nv_bfloat16*)k_cache, (__nv_bfloat16*)v_cache, slot_mapping,
          nq, nkv, d, qkv_stride, block_size, num_blocks, 1.f, 1.f, status);
    return (int)cudaGetLastError();
  }
  switch (dtype) {
    case kBF16:
      return launch_rope<__nv_bfloat16>(qkv, positions, cos_sin, k_cache, v_cache, slot_mapping, T, nq, nkv, d,
                                        rotary_dim, qkv_stride, block_size, num_blocks, k_scale, v_scale, q_norm_w,
                                        k_norm_w, norm_eps, cache_dtype, status, s);
    case kF16:
      return launch_rope<__half>(qkv, positions, cos_sin, k_cache, v_cache, slot_mapping, T, nq, nkv, d, rotary_dim,
                                 qkv_stride, block_size, num_blocks, k_scale, v_scale, q_norm_w, k_norm_w, norm_eps,
                                 cache_dtype, status, s);
    case kF32:
      return launch_rope<float>(qkv, positions, cos_sin, k_cache, v_cache, slot_mapping, T, nq, nkv, d, rotary_dim,
                                qkv_stride, block_size, num_blocks, k_scale, v_scale, q_norm_w, k_norm_w, norm_eps,
                                cache_dtype, status, s);
  }
  return kBadShape;
}

extern "C" int b200_embedding(void* out, const int64_t* ids, const void* table, int T, int rows, int H,
                              int64_t vocab_start, int dtype, cudaStream_t s) {
  using namespace b200;
  if (T == 0) return 0;
  switch (dtype) {
    case kBF16:
      embedding_kernel<__nv_bfloat16><<<T, 128, 0, s>>>((__nv_bfloat16*)out, ids, (const __nv_bfloat16*)table, rows,
                                                        H, vocab_start);
      break;
    case kF16:
      embedding_kernel<__half><<<T, 128, 0, s>>>((__half*)out, ids, (const __half*)table, rows, H, vocab_start);
      break;
    case kF32:
      embedding_kernel<float><<<T, 128, 0, s>>>((float*)out, ids, (const float*)table, rows, H, vocab_start);
      break;
    default:
      return kBadShape;
  }
  return (int)cudaGetLastError();
}
