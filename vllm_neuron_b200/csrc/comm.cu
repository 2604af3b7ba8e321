// Fused NVLink collectives for tensor-parallel decode.
//
// All-reduce (one-shot, push) fused with the ops that always follow it in the decoder:
//   out = RMSNorm(sum_ranks(partial) + bias + residual) * w,  residual <- the pre-norm sum
// (or plain out = sum when no norm is requested).  This replaces, per layer, NCCL
// all-reduce + a residual-add/RMSNorm kernel after the attention output projection and
// after the MoE (the reference's attn_tp / moe all_reduce call sites,
// model/gpt_oss/model_mxfp4.py:828,1330, each followed by RMSNorm).
//
// Memory: every rank owns one cudaMalloc'd region, mapped into its peers with CUDA IPC:
//   [flags: kMaxBlocks x kMaxRanks u32][counters: kMaxBlocks u32][pad][slot 0][slot 1]
// and each slot holds one receive area per source rank ([world][rows][H] bf16).
// Protocol per call, independently in every CTA b (so it is CUDA-graph safe and needs no
// host-side state):
//   1. epoch = counters[b] + 1; slot = epoch & 1
//   2. push this CTA's rows of the local partial into every rank's receive area for this
//      rank (NVLink stores, posted: no round trip); CTA barrier
//   3. for each peer p: st.release.sys peer_p.flags[b][me] = epoch (the release covers the
//      CTA's pushes)
//   4. spin (bounded) on the local flags until every peer's CTA b has pushed (local loads)
//   5. reduce the rows from the local receive areas (uncached loads), add bias/residual,
//      RMSNorm, store; counters[b] = epoch
// Pushing instead of pulling turns the NVLink traffic into posted writes and the waits and
// reductions into local memory accesses.  Double buffering makes the slot written at epoch e
// disjoint from the one a peer may still read at epoch e-1; reuse two calls later is safe
// because passing barrier e-1 proves every peer has finished epoch e-2 (stream order).
// Waits give up after `wait_ns` (2 s by default) and set status to kWaitTimeout.
#include "common.cuh"
#include "launch_pdl.h"
#include "launch.h"

namespace b200 {

constexpr int kMaxRanks = 8;
constexpr int kMaxBlocks = 128;
constexpr size_t kHeaderBytes = 64 * 1024;  // flags + counters, keeps slots 64 KB aligned

struct CommPeers {
  uint8_t* base[kMaxRanks];  // every rank's region (base[rank] is the local one)
  int rank, world;
  size_t slot_bytes;
};

B200_D uint32_t* flags_of(uint8_t* base) { return reinterpret_cast<uint32_t*>(base); }
B200_D uint32_t* counters_of(uint8_t* base) {
  return reinterpret_cast<uint32_t*>(base + kMaxBlocks * kMaxRanks * sizeof(uint32_t));
}
B200_D uint8_t* slot_of(uint8_t* base, int slot, size_t slot_bytes) {
  return base + kHeaderBytes + (size_t)slot * slot_bytes;
}

B200_D void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
B200_D uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
B200_D uint4 ld_volatile_v4(const void* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
B200_D uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// One CTA per group of rows; rows r = blockIdx.x, blockIdx.x + gridDim.x, ...
// H % 8 == 0; bf16 data.  kNorm: add bias + residual and RMSNorm; else plain sum.
// Route mode (topk_ids != null): `in` holds per-route rows [T * k, H] of an MoE layer and the
// partial pushed for token r is their sum over the routes to this rank's experts
// [eoff, eoff + E_local) (fp32 sum rounded to bf16, as a separate reduction kernel would store).
template <bool kNorm>
__global__ void __launch_bounds__(256) allreduce_fused_kernel(CommPeers peers, const __nv_bfloat16* __restrict__ in,
                                                              const int* __restrict__ topk_ids, int k, int E_local,
                                                              int eoff,
                                                              __nv_bfloat16* __restrict__ out,
                                                              __nv_bfloat16* __restrict__ residual,
                                                              const __nv_bfloat16* __restrict__ bias,
                                                              const float* __restrict__ w, float eps, int T, int H,
                                                              unsigned long long wait_ns, int* status) {
  pdl_wait();  // predecessor output visible (programmatic dependent launch)
  pdl_trigger();
  __shared__ float red[32];
  __shared__ uint32_t s_epoch;
  const int b = blockIdx.x;
  // a CTA without rows takes no part (every rank sees the same T, so CTA b's epoch count
  // stays equal across ranks)
  if (b >= T) return;
  uint8_t* me = peers.base[peers.rank];
  if (threadIdx.x == 0) s_epoch = counters_of(me)[b] + 1;
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const int slot = epoch & 1;
  const int nchunk = H / 8;
  const size_t part = peers.slot_bytes / peers.world;  // one source rank's receive area
  // 2. push my rows into every rank's receive area for me
  for (int r = b; r < T; r += gridDim.x) {
    const uint4* src = reinterpret_cast<const uint4*>(in + (size_t)r * H);
    int loc[16];
    int nl = 0;
    if (topk_ids != nullptr)
      for (int j = 0; j < k && j < 16; ++j) {
        const int e = topk_ids[r * k + j] - eoff;
        if (e >= 0 && e < E_local) loc[nl++] = j;
      }
    for (int c = threadIdx.x; c < nchunk; c += blockDim.x) {
      uint4 v;
      if (topk_ids != nullptr) {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int i = 0; i < nl; ++i) {
          const uint4 u = reinterpret_cast<const uint4*>(in + (size_t)(r * k + loc[i]) * H)[c];
          const __nv_bfloat16* hb = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
          for (int q = 0; q < 8; ++q) acc[q] += __bfloat162float(hb[q]);
        }
        __nv_bfloat16* vb = reinterpret_cast<__nv_bfloat16*>(&v);
#pragma unroll
        for (int q = 0; q < 8; ++q) vb[q] = __float2bfloat16(acc[q]);
      } else {
        v = src[c];
      }
      const size_t off = (size_t)peers.rank * part + ((size_t)r * nchunk + c) * 16;
      for (int p = 0; p < peers.world; ++p)
        *reinterpret_cast<uint4*>(slot_of(peers.base[p], slot, peers.slot_bytes) + off) = v;
    }
  }
  // the release store below is cumulative over the CTA's pushes (ordered by the barrier)
  __syncthreads();
  // 3. signal every peer, 4. wait for every peer (local flags)
  if (threadIdx.x < peers.world) {
    const int p = threadIdx.x;
    st_release_sys(flags_of(peers.base[p]) + b * kMaxRanks + peers.rank, epoch);
    const uint32_t* f = flags_of(me) + b * kMaxRanks + p;
    if (ld_acquire_sys(f) < epoch) {
      const uint64_t t0 = now_ns();
      for (uint32_t i = 1;; ++i) {
        if (ld_acquire_sys(f) >= epoch) break;
        if ((i & 255) == 0) {
          if (now_ns() - t0 > wait_ns) {
            if (status) atomicCAS(status, 0, kWaitTimeout);
            break;
          }
        }
      }
    }
  }
  __syncthreads();
  // 5. reduce over ranks (+ bias + residual, RMSNorm)
  for (int r = b; r < T; r += gridDim.x) {
    constexpr int kMaxVec = 4;  // H <= 256 threads * 4 chunks * 8 = 8192
    float v[kMaxVec][8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i) {
      const int c = threadIdx.x + i * blockDim.x;
      if (c < nchunk) {
#pragma unroll
        for (int q = 0; q < 8; ++q) v[i][q] = 0.f;
        const uint8_t* mine = slot_of(me, slot, peers.slot_bytes);
        for (int p = 0; p < peers.world; ++p) {
          const uint4 u = ld_volatile_v4(mine + (size_t)p * part + ((size_t)r * nchunk + c) * 16);
          const __nv_bfloat16* hb = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
          for (int q = 0; q < 8; ++q) v[i][q] += __bfloat162float(hb[q]);
        }
        if constexpr (kNorm) {
          if (bias) {
            const uint4 bu = reinterpret_cast<const uint4*>(bias)[c];
            const __nv_bfloat16* bb = reinterpret_cast<const __nv_bfloat16*>(&bu);
#pragma unroll
            for (int q = 0; q < 8; ++q) v[i][q] += __bfloat162float(bb[q]);
          }
          // the residual stream is kept in bf16, as in the unfused path
          uint4 ru = reinterpret_cast<const uint4*>(residual + (size_t)r * H)[c];
          const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(&ru);
          uint4 ro;
          __nv_bfloat16* rob = reinterpret_cast<__nv_bfloat16*>(&ro);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            // round the reduced sum to bf16 first (the unfused path stores it in bf16)
            const float sum_bf = __bfloat162float(__float2bfloat16(v[i][q]));
            rob[q] = __float2bfloat16(sum_bf + __bfloat162float(rb[q]));
            v[i][q] = __bfloat162float(rob[q]);
            ss += v[i][q] * v[i][q];
          }
          reinterpret_cast<uint4*>(residual + (size_t)r * H)[c] = ro;
        } else {
          uint4 o;
          __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
          for (int q = 0; q < 8; ++q) ob[q] = __float2bfloat16(v[i][q]);
          reinterpret_cast<uint4*>(out + (size_t)r * H)[c] = o;
        }
      }
    }
    if constexpr (kNorm) {
      const float tot = block_sum(ss, red);
      const float inv = rsqrtf(tot / (float)H + eps);
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
          reinterpret_cast<uint4*>(out + (size_t)r * H)[c] = o;
        }
      }
      __syncthreads();  // red[] reuse by the next row
    }
  }
  if (threadIdx.x == 0) counters_of(me)[b] = epoch;
}

}  // namespace b200

using namespace b200;

extern "C" int b200_comm_alloc(size_t slot_bytes, void** out) {
  const size_t total = kHeaderBytes + 2 * slot_bytes;
  cudaError_t e = cudaMalloc(out, total);
  if (e != cudaSuccess) return (int)e;
  e = cudaMemset(*out, 0, total);
  return (int)e;
}

extern "C" int b200_comm_free(void* p) { return (int)cudaFree(p); }

extern "C" int b200_ipc_get_handle(void* p, void* handle64) {
  return (int)cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(handle64), p);
}

extern "C" int b200_ipc_open_handle(const void* handle64, void** out) {
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  return (int)cudaIpcOpenMemHandle(out, h, cudaIpcMemLazyEnablePeerAccess);
}

extern "C" int b200_ipc_close(void* p) { return (int)cudaIpcCloseMemHandle(p); }

// wait_ns: limit of each CTA's wait for its peers (0 = kDefaultWaitNs).
extern "C" int b200_allreduce_fused(void* const* bases, int rank, int world, size_t slot_bytes, const void* in,
                                    void* out, void* residual, const void* bias, const float* w, float eps, int T,
                                    int H, int num_blocks, unsigned long long wait_ns, int* status, cudaStream_t s,
                                    const int* topk_ids, int k, int E_local, int eoff) {
  if (topk_ids != nullptr && (k < 1 || k > 16)) return kBadShape;
  if (wait_ns == 0) wait_ns = kDefaultWaitNs;
  if (world > kMaxRanks || world < 1 || H % 8 || H > 8192 || T < 0) return kBadShape;
  if ((size_t)T * H * 2 * world > slot_bytes || (slot_bytes / world) % 16) return kBadShape;
  if (num_blocks < 1 || num_blocks > kMaxBlocks) return kBadShape;
  if (T == 0) return 0;
  CommPeers peers{};
  for (int i = 0; i < world; ++i) peers.base[i] = static_cast<uint8_t*>(bases[i]);
  peers.rank = rank;
  peers.world = world;
  peers.slot_bytes = slot_bytes;
  if (w != nullptr)
    launch_k(allreduce_fused_kernel<true>, dim3(num_blocks), dim3(256), 0, s, peers, (const __nv_bfloat16*)in, topk_ids, k,
             E_local, eoff, (__nv_bfloat16*)out,
                                                           (__nv_bfloat16*)residual, (const __nv_bfloat16*)bias, w,
                                                           eps, T, H, wait_ns, status);
  else
    launch_k(allreduce_fused_kernel<false>, dim3(num_blocks), dim3(256), 0, s, peers, (const __nv_bfloat16*)in, topk_ids,
             k, E_local, eoff, (__nv_bfloat16*)out,
                                                            nullptr, nullptr, nullptr, eps, T, H, wait_ns, status);
  return (int)cudaGetLastError();
}
