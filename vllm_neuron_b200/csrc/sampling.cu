// Router top-k softmax, argmax and on-device sampling.
//
// topk_softmax: per token, the k largest router logits (ties -> lower expert id) and a
//   softmax over those k values (GPT-OSS order, functional/moe/router.py:300-566); with
//   `full`, the softmax over all E logits taken at the k selected experts, not renormalised
//   (softmax -> top-k routers without norm_topk_prob).
// argmax: per row (max value, lowest index of the max).
// sample: per row, temperature -> top-k (<= max_top_k <= 1024) -> softmax -> top-p ->
//   inverse-CDF draw with a host-supplied uniform; temperature <= 0 is greedy
//   (functional/sampling.py:21).  The top-K candidates come from a 4-pass radix select
//   over order-preserving float bits, then a bitonic sort in shared memory.
#include "launch.h"
#include "common.cuh"
#include "launch_pdl.h"

namespace b200 {

template <typename LT>
__global__ void topk_softmax_kernel(int* __restrict__ ids, float* __restrict__ w, const LT* __restrict__ logits,
                                    int T, int E, int k, int full) {
  pdl_wait();  // predecessor output visible (programmatic dependent launch)
  pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  const LT* row = logits + (size_t)warp * E;
  constexpr int kMaxPer = 32;  // E <= 1024
  float v[kMaxPer];
  const int per = (E + 31) / 32;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int e = i * 32 + lane;
    v[i] = (i < per && e < E) ? to_float(row[e]) : -INFINITY;
  }
  float denom_all = 0.f;  // full: sum over all experts of exp(l - max)
  if (full) {
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) mx = fmaxf(mx, v[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sm = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) sm += v[i] == -INFINITY ? 0.f : __expf(v[i] - mx);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o);
    denom_all = sm;
  }
  float sel_v[16];
  int sel_i[16];
  for (int j = 0; j < k; ++j) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
      const int e = i * 32 + lane;
      if (i < per && e < E && (v[i] > bv || (v[i] == bv && e < bi))) {
        bv = v[i];
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
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i)
      if (i * 32 + lane == bi) v[i] = -INFINITY;
  }
  if (lane == 0) {
    const float m = sel_v[0];
    float s = 0.f;
    for (int j = 0; j < k; ++j) s += __expf(sel_v[j] - m);
    if (full) s = denom_all;  // m is the row maximum (the first selected logit)
    for (int j = 0; j < k; ++j) {
      ids[(size_t)warp * k + j] = sel_i[j];
      w[(size_t)warp * k + j] = __expf(sel_v[j] - m) / s;
    }
  }
}

// argmax: each CTA scans a slice of one row with 16-byte loads and folds its (value,
// index) into a 64-bit key [order-preserving value bits | ~index] with atomicMax, so the
// largest value wins and among equal values the lowest index; a second kernel unpacks.
B200_D uint32_t order_bits(float f) {
  const uint32_t u = __float_as_uint(f);
  if (f != f) return 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
B200_D float from_order_bits(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

template <typename T>
__global__ void __launch_bounds__(256) argmax_partial_kernel(unsigned long long* __restrict__ best,
                                                             const T* __restrict__ logits, int V, int slice) {
  const int b = blockIdx.y;
  const int lo = blockIdx.x * slice, hi = min(V, lo + slice);
  const T* row = logits + (size_t)b * V;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  constexpr int kVec = 16 / sizeof(T);
  const bool vec_ok = (reinterpret_cast<uintptr_t>(row) % 16 == 0) && (lo % kVec == 0);
  if (vec_ok) {
    const int n_vec = (hi - lo) / kVec;
    for (int c = threadIdx.x; c < n_vec; c += blockDim.x) {
      const uint4 u = reinterpret_cast<const uint4*>(row + lo)[c];
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int q = 0; q < kVec; ++q) {
        const float x = to_float(e[q]);
        if (x > bv) {
          bv = x;
          bi = lo + c * kVec + q;
        }
      }
    }
    for (int i = lo + n_vec * kVec + threadIdx.x; i < hi; i += blockDim.x) {
      const float x = to_float(row[i]);
      if (x > bv || (x == bv && i < bi)) {
        bv = x;
        bi = i;
      }
    }
  } else {
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
      const float x = to_float(row[i]);
      if (x > bv) {
        bv = x;
        bi = i;
      }
    }
  }
  unsigned long long key = bi == 0x7fffffff ? 0ull
                                            : ((unsigned long long)order_bits(bv) << 32) | (0xffffffffu - (uint32_t)bi);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
    key = other > key ? other : key;
  }
  if ((threadIdx.x & 31) == 0 && key != 0ull) atomicMax(best + b, key);
}

__global__ void argmax_finish_kernel(float* __restrict__ vals, int64_t* __restrict__ idx,
                                     const unsigned long long* __restrict__ best, int B) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const unsigned long long k = best[b];
  if (k == 0ull) {
    vals[b] = -INFINITY;
    idx[b] = 0;
    return;
  }
  vals[b] = from_order_bits((uint32_t)(k >> 32));
  idx[b] = (int64_t)(0xffffffffu - (uint32_t)(k & 0xffffffffu));
}

B200_D uint32_t order_key(float f) {
  // monotone map float -> uint32 (larger float -> larger key); NaN sorts lowest
  uint32_t u = __float_as_uint(f);
  if (f != f) return 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

constexpr int kSortN = 1024;

template <typename T>
__global__ void __launch_bounds__(1024) sample_kernel(int64_t* __restrict__ out, const T* __restrict__ logits,
                                                      const float* __restrict__ temperature,
                                                      const int* __restrict__ top_k, const float* __restrict__ top_p,
                                                      const float* __restrict__ uniform, int V, int K) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s_prefix, s_remaining, s_cnt_gt, s_cnt_eq;
  __shared__ float cv[kSortN];
  __shared__ int ci[kSortN];
  const int r = blockIdx.x;
  const T* row = logits + (size_t)r * V;
  const int tid = threadIdx.x;
  // ---- radix select the K-th largest key ----
  if (tid == 0) {
    s_prefix = 0;
    s_remaining = K;
  }
  __syncthreads();
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix;
    const uint32_t pmask = pass == 0 ? 0u : (0xffffffffu << (32 - 8 * pass));
    for (int i = tid; i < V; i += blockDim.x) {
      const uint32_t key = order_key(to_float(row[i]));
      if ((key & pmask) == prefix) atomicAdd(&hist[(key >> shift) & 0xff], 1u);
    }
    __syncthreads();
    if (tid == 0) {
      uint32_t rem = s_remaining;
      int bin = 255;
      for (; bin > 0; --bin) {
        if (hist[bin] >= rem) break;
        rem -= hist[bin];
      }
      s_prefix = prefix | ((uint32_t)bin << shift);
      s_remaining = rem;
    }
    __syncthreads();
  }
  const uint32_t thr = s_prefix;  // key of the K-th largest element
  const uint32_t need_eq = s_remaining;  // how many elements equal to thr to keep
  if (tid == 0) {
    s_cnt_gt = 0;
    s_cnt_eq = 0;
  }
  for (int i = tid; i < kSortN; i += blockDim.x) {
    cv[i] = -INFINITY;
    ci[i] = 0x7fffffff;
  }
  __syncthreads();
  // number strictly greater than thr is K - need_eq; equal ones fill after them
  const uint32_t n_gt = (uint32_t)K - need_eq;
  for (int i = tid; i < V; i += blockDim.x) {
    const float x = to_float(row[i]);
    const uint32_t key = order_key(x);
    if (key > thr) {
      const uint32_t s = atomicAdd(&s_cnt_gt, 1u);
      if (s < (uint32_t)kSortN) {
        cv[s] = x;
        ci[s] = i;
      }
    } else if (key == thr) {
      const uint32_t s = atomicAdd(&s_cnt_eq, 1u);
      // keep the lowest indices among ties: collect all, sorted below by index
      if (n_gt + s < (uint32_t)kSortN) {
        cv[n_gt + s] = x;
        ci[n_gt + s] = i;
      }
    }
  }
  __syncthreads();
  // ---- bitonic sort: value desc, index asc ----
  for (int size = 2; size <= kSortN; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < kSortN; i += blockDim.x) {
        const int j = i ^ stride;
        if (j > i) {
          const bool desc = (i & size) == 0;
          const float vi = cv[i], vj = cv[j];
          const int ii = ci[i], ij = ci[j];
          const bool i_first = (vi > vj) || (vi == vj && ii < ij);
          if (desc != i_first) {
            cv[i] = vj;
            cv[j] = vi;
            ci[i] = ij;
            ci[j] = ii;
          }
        }
      }
      __syncthreads();
    }
  }
  // ---- temperature / top-k / top-p / draw (one warp) ----
  if (tid < 32) {
    const int lane = tid;
    const float t = temperature[r];
    if (t <= 0.f) {
      if (lane == 0) out[r] = ci[0] == 0x7fffffff ? 0 : ci[0];
      return;
    }
    int kk = top_k[r];
    kk = (kk <= 0 || kk > K) ? K : kk;
    const float inv_t = 1.f / fmaxf(t, 1e-6f);
    const float m = cv[0] * inv_t;
    // softmax mass of the kept candidates
    float tot = 0.f;
    for (int i = lane; i < kk; i += 32) tot += __expf(cv[i] * inv_t - m);
    tot = warp_sum(tot);
    // top-p: keep candidate i while (cdf_before_i) < p * tot; cdf is computed serially by lane 0
    if (lane == 0) {
      const float p = top_p[r];
      float cdf = 0.f;
      int keep = 0;
      for (int i = 0; i < kk; ++i) {
        const float pi = __expf(cv[i] * inv_t - m);
        if (i > 0 && cdf >= p * tot) break;
        cdf += pi;
        keep = i + 1;
      }
      // inverse CDF over the kept mass `cdf`
      const float u = uniform[r] * cdf;
      float acc = 0.f;
      int choice = keep - 1;
      for (int i = 0; i < keep; ++i) {
        acc += __expf(cv[i] * inv_t - m);
        if (acc > u) {
          choice = i;
          break;
        }
      }
      out[r] = ci[choice] == 0x7fffffff ? 0 : ci[choice];
    }
  }
}

}  // namespace b200

using namespace b200;

extern "C" int b200_topk_softmax(int* ids, float* weights, const void* logits, int T, int E, int k, int dtype,
                                 int full, cudaStream_t s) {
  if (E > 1024 || k > 16 || k > E) return kBadShape;
  if (T == 0) return 0;
  const int warps_per_block = 4;
  if (dtype == kBF16)
    launch_k(topk_softmax_kernel<__nv_bfloat16>, dim3(cdiv(T, warps_per_block)), dim3(32 * warps_per_block), 0, s,
             ids, weights, (const __nv_bfloat16*)logits, T, E, k, full);
  else if (dtype == kF32)
    launch_k(topk_softmax_kernel<float>, dim3(cdiv(T, warps_per_block)), dim3(32 * warps_per_block), 0, s, ids,
             weights, (const float*)logits, T, E, k, full);
  else
    return kBadShape;
  return (int)cudaGetLastError();
}

extern "C" int b200_argmax(float* vals, int64_t* idx, const void* logits, int B, int V, int dtype, cudaStream_t s) {
  if (B == 0) return 0;
  // the int64 output doubles as the buffer of packed 64-bit keys, unpacked in place
  unsigned long long* best = reinterpret_cast<unsigned long long*>(idx);
  cudaError_t e = cudaMemsetAsync(best, 0, sizeof(unsigned long long) * B, s);
  if (e != cudaSuccess) return (int)e;
  const int slice = 8192;
  dim3 grid(cdiv(V, slice), B);
  switch (dtype) {
    case kBF16: argmax_partial_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(best, (const __nv_bfloat16*)logits, V, slice); break;
    case kF16: argmax_partial_kernel<__half><<<grid, 256, 0, s>>>(best, (const __half*)logits, V, slice); break;
    case kF32: argmax_partial_kernel<float><<<grid, 256, 0, s>>>(best, (const float*)logits, V, slice); break;
    default: return kBadShape;
  }
  argmax_finish_kernel<<<cdiv(B, 128), 128, 0, s>>>(vals, idx, best, B);
  return (int)cudaGetLastError();
}

extern "C" int b200_sample(int64_t* out, const void* logits, const float* temperature, const int* top_k,
                           const float* top_p, const float* uniform, int B, int V, int max_top_k, int dtype,
                           float* scratch, cudaStream_t s) {
  (void)scratch;
  if (B == 0) return 0;
  const int K = max_top_k < V ? max_top_k : V;
  if (K > kSortN || K < 1) return kBadShape;
  switch (dtype) {
    case kBF16:
      sample_kernel<__nv_bfloat16><<<B, 1024, 0, s>>>(out, (const __nv_bfloat16*)logits, temperature, top_k, top_p,
                                                      uniform, V, K);
      break;
    case kF16:
      sample_kernel<__half><<<B, 1024, 0, s>>>(out, (const __half*)logits, temperature, top_k, top_p, uniform, V, K);
      break;
    case kF32:
      sample_kernel<float><<<B, 1024, 0, s>>>(out, (const float*)logits, temperature, top_k, top_p, uniform, V, K);
      break;
    default:
      return kBadShape;
  }
  return (int)cudaGetLastError();
}
