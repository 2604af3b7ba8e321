// Fused NVLink collectives for tensor parallelism: the decode layer-boundary all-reduce (below)
// and the prefill sequence-parallel boundary (sp_boundary_kernel, further down).
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
// LL variant (the default for decode sizes): step 2 pushes LL units (data and epoch in every
// 16-byte store, st_ll) and steps 3-4 disappear: each reducing thread polls the units it reads
// until they carry the epoch.  The same reuse argument holds per CTA: CTA b of a rank pushes
// epoch e only after it has read every peer's epoch e-1 rows, which each peer's CTA b pushed
// after finishing its own epoch e-2 reads.
// Waits give up after `wait_ns` (2 s by default) and set status to kWaitTimeout.
#include <algorithm>

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

// Threads 0 .. world-1 of CTA b: publish `value` in every rank's flag word (b, me) (the
// release covers the CTA's earlier stores, ordered by the caller's barrier), then wait until
// every rank's word (b, p) of the local region holds at least `value`.  The wait gives up after
// wait_ns and records kWaitTimeout.
B200_D void signal_and_wait(const CommPeers& peers, int b, uint32_t value, unsigned long long wait_ns, int* status) {
  if (threadIdx.x < peers.world) {
    const int p = threadIdx.x;
    st_release_sys(flags_of(peers.base[p]) + b * kMaxRanks + peers.rank, value);
    const uint32_t* f = flags_of(peers.base[peers.rank]) + b * kMaxRanks + p;
    if (ld_acquire_sys(f) < value) {
      const uint64_t t0 = now_ns();
      for (uint32_t i = 1;; ++i) {
        if (ld_acquire_sys(f) >= value) break;
        if ((i & 255) == 0 && now_ns() - t0 > wait_ns) {
          if (status) atomicCAS(status, 0, kWaitTimeout);
          break;
        }
      }
    }
  }
}

// Partial row of token t in route mode: the fp32 sum of its routes to this rank's experts
// (loc: the route slots j with a local expert), rounded to bf16, for 16-byte chunk c.
B200_D uint4 route_sum_chunk(const __nv_bfloat16* in, int t, int k, const int* loc, int nl, int H, int c) {
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int i = 0; i < nl; ++i) {
    const uint4 u = reinterpret_cast<const uint4*>(in + (size_t)(t * k + loc[i]) * H)[c];
    const __nv_bfloat16* hb = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[q] += __bfloat162float(hb[q]);
  }
  uint4 v;
  __nv_bfloat16* vb = reinterpret_cast<__nv_bfloat16*>(&v);
#pragma unroll
  for (int q = 0; q < 8; ++q) vb[q] = __float2bfloat16(acc[q]);
  return v;
}

B200_D int local_routes(const int* topk_ids, int t, int k, int E_local, int eoff, int* loc) {
  int nl = 0;
  for (int j = 0; j < k && j < 16; ++j) {
    const int e = topk_ids[t * k + j] - eoff;
    if (e >= 0 && e < E_local) loc[nl++] = j;
  }
  return nl;
}

// Low-latency (LL) transfer unit: 8 bytes of data travel with two copies of the call's epoch,
// {d0, e, d1, e} in one 16-byte store, so a receiver that sees the epoch in both flag words has
// the data word beside each (each aligned 8-byte {data, flag} half lands whole) and needs no
// separate flag, release fence or round trip.  32 bytes carry one 16-byte chunk of 8 bf16.
B200_D void st_ll(uint8_t* p, const uint4& v, uint32_t e) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(e), "r"(v.y), "r"(e)
               : "memory");
  asm volatile("st.volatile.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p + 16), "r"(v.z), "r"(e), "r"(v.w), "r"(e)
               : "memory");
}

// Poll one LL chunk until both units carry epoch e; gives up at `deadline` (%globaltimer ns) or
// once another thread of the CTA has (abort), recording kWaitTimeout.
B200_D uint4 ld_ll(const uint8_t* p, uint32_t e, uint64_t deadline, int* status, volatile int* abort) {
  uint4 a, b;
  for (uint32_t i = 0;; ++i) {
    a = ld_volatile_v4(p);
    b = ld_volatile_v4(p + 16);
    if (a.y == e && a.w == e && b.y == e && b.w == e) break;
    if ((i & 63) == 63) {
      if (*abort) break;
      if (now_ns() > deadline) {
        *abort = 1;
        if (status) atomicCAS(status, 0, kWaitTimeout);
        break;
      }
    }
  }
  return make_uint4(a.x, a.z, b.x, b.z);
}

// One CTA per group of rows; rows r = blockIdx.x, blockIdx.x + gridDim.x, ...
// H % 8 == 0; bf16 data.  kNorm: add bias + residual and RMSNorm; else plain sum.
// kLL: the pushes are LL units (twice the bytes, no flag exchange: each reducing thread polls
// the units it reads); else the pushes are plain 16-byte stores followed by one release flag
// per peer (signal_and_wait).  One communicator uses one protocol for its whole life, so a
// receive area never holds the other protocol's bytes.
// Route mode (topk_ids != null): `in` holds per-route rows [T * k, H] of an MoE layer and the
// partial pushed for token r is their sum over the routes to this rank's experts
// [eoff, eoff + E_local) (fp32 sum rounded to bf16, as a separate reduction kernel would store).
template <bool kNorm, bool kLL>
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
  __shared__ int s_abort;
  const int b = blockIdx.x;
  // a CTA without rows takes no part (every rank sees the same T, so CTA b's epoch count
  // stays equal across ranks)
  if (b >= T) return;
  uint8_t* me = peers.base[peers.rank];
  if (threadIdx.x == 0) {
    s_epoch = counters_of(me)[b] + 1;
    s_abort = 0;
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const int slot = epoch & 1;
  const int nchunk = H / 8;
  const size_t part = peers.slot_bytes / peers.world;  // one source rank's receive area
  // 2. push my rows into every rank's receive area for me
  for (int r = b; r < T; r += gridDim.x) {
    const uint4* src = reinterpret_cast<const uint4*>(in + (size_t)r * H);
    int loc[16];
    const int nl = topk_ids != nullptr ? local_routes(topk_ids, r, k, E_local, eoff, loc) : 0;
    for (int c = threadIdx.x; c < nchunk; c += blockDim.x) {
      const uint4 v = topk_ids != nullptr ? route_sum_chunk(in, r, k, loc, nl, H, c) : src[c];
      if constexpr (kLL) {
        const size_t off = (size_t)peers.rank * part + ((size_t)r * nchunk + c) * 32;
        for (int pp = 0; pp < peers.world; ++pp) {
          const int p = (peers.rank + pp) % peers.world;
          st_ll(slot_of(peers.base[p], slot, peers.slot_bytes) + off, v, epoch);
        }
      } else {
        const size_t off = (size_t)peers.rank * part + ((size_t)r * nchunk + c) * 16;
        for (int p = 0; p < peers.world; ++p)
          *reinterpret_cast<uint4*>(slot_of(peers.base[p], slot, peers.slot_bytes) + off) = v;
      }
    }
  }
  if constexpr (!kLL) {
    // the release store below is cumulative over the CTA's pushes (ordered by the barrier)
    __syncthreads();
    // 3. signal every peer, 4. wait for every peer (local flags)
    signal_and_wait(peers, b, epoch, wait_ns, status);
    __syncthreads();
  }
  const uint64_t deadline = now_ns() + wait_ns;
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
          const uint4 u = kLL ? ld_ll(mine + (size_t)p * part + ((size_t)r * nchunk + c) * 32, epoch, deadline,
                                      status, &s_abort)
                              : ld_volatile_v4(mine + (size_t)p * part + ((size_t)r * nchunk + c) * 16);
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

// ------------------------------------------------------------ sequence-parallel boundary
// Prefill layer boundary under sequence parallelism.  T = world * Ts token rows; rank q owns
// rows [q Ts, (q + 1) Ts) of the residual stream.  One call replaces reduce-scatter + bias +
// residual add + RMSNorm + all-gather (the reference's SP boundary: reduce-scatter after each
// block and all-gather before the next, model/gpt_oss/model_mxfp4.py:464,685):
//   s_me = sum_ranks(partial[my rows]) + bias + residual_me        (residual_me <- s_me)
//   out  = [RMSNorm(s_0) * w; ...; RMSNorm(s_{world-1}) * w]      ([T, H] on every rank)
// Region of a rank: [header][slot 0][slot 1], slot = [RS area][guard][AG area][guard] with the
// RS area [world sources][Ts][H] and the AG area [T][H] (bf16, area_bytes each).  The host picks
// the slot (it counts its calls, the same on every rank); `out` is that slot's AG area.
// Every CTA b takes rows i = b, b + G, ... of each shard in two push phases; one monotonic flag
// word per (CTA, source) holds 2e - 1 after phase 1 of the CTA's epoch e and 2e after phase 2:
//   1. push partial row q Ts + i into rank q's RS area at [me][i], every q (skipped when the
//      producing GEMM stored its rows there itself); release 2e - 1 to every rank, wait for it
//   2. reduce RS rows [*][i], add bias and residual, normalise; push the row into every rank's
//      AG area at row me Ts + i; release 2e to every rank, wait for it
// Rank q's CTA b reads the RS rows that CTA b of every source pushed before it releases 2e, so
// a call that has returned on one rank proves that every peer has consumed its pushes: the next
// call may overwrite them.  In route mode the partial row of a token is the sum of its routes
// to this rank's experts, as in allreduce_fused_kernel.
template <bool kPushed>
__global__ void __launch_bounds__(256) sp_boundary_kernel(CommPeers peers, size_t rs_off, size_t ag_off,
                                                          const __nv_bfloat16* __restrict__ in,
                                                          const int* __restrict__ topk_ids, int k, int E_local,
                                                          int eoff, __nv_bfloat16* __restrict__ residual,
                                                          const __nv_bfloat16* __restrict__ bias,
                                                          const float* __restrict__ w, float eps, int T, int H,
                                                          unsigned long long wait_ns, int* status) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[32];
  __shared__ uint32_t s_epoch;
  const int b = blockIdx.x, world = peers.world, me = peers.rank;
  const int Ts = T / world;
  if (b >= Ts) return;  // same on every rank: CTA b's epochs stay in step
  uint8_t* mine = peers.base[me];
  if (threadIdx.x == 0) s_epoch = counters_of(mine)[b] + 1;
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const int nchunk = H / 8;
  const size_t row_bytes = (size_t)H * 2;
  if constexpr (!kPushed) {
    for (int qq = 0; qq < world; ++qq) {
      const int q = (me + 1 + qq) % world;  // ranks start at different destinations
      uint8_t* dst = peers.base[q] + rs_off + (size_t)me * Ts * row_bytes;
      for (int i = b; i < Ts; i += gridDim.x) {
        const int t = q * Ts + i;
        int loc[16];
        const int nl = topk_ids != nullptr ? local_routes(topk_ids, t, k, E_local, eoff, loc) : 0;
        for (int c = threadIdx.x; c < nchunk; c += blockDim.x) {
          const uint4 v = topk_ids != nullptr ? route_sum_chunk(in, t, k, loc, nl, H, c)
                                              : reinterpret_cast<const uint4*>(in + (size_t)t * H)[c];
          *reinterpret_cast<uint4*>(dst + (size_t)i * row_bytes + (size_t)c * 16) = v;
        }
      }
    }
  }
  __syncthreads();
  signal_and_wait(peers, b, 2 * epoch - 1, wait_ns, status);
  __syncthreads();
  for (int i = b; i < Ts; i += gridDim.x) {
    constexpr int kMaxVec = 4;  // H <= 256 threads * 4 chunks * 8
    float v[kMaxVec][8];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxVec; ++j) {
      const int c = threadIdx.x + j * blockDim.x;
      if (c < nchunk) {
#pragma unroll
        for (int q = 0; q < 8; ++q) v[j][q] = 0.f;
        for (int p = 0; p < world; ++p) {
          const uint4 u = ld_volatile_v4(mine + rs_off + ((size_t)p * Ts + i) * row_bytes + (size_t)c * 16);
          const __nv_bfloat16* hb = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
          for (int q = 0; q < 8; ++q) v[j][q] += __bfloat162float(hb[q]);
        }
        if (bias) {
          const uint4 bu = reinterpret_cast<const uint4*>(bias)[c];
          const __nv_bfloat16* bb = reinterpret_cast<const __nv_bfloat16*>(&bu);
#pragma unroll
          for (int q = 0; q < 8; ++q) v[j][q] += __bfloat162float(bb[q]);
        }
        uint4 ru = reinterpret_cast<const uint4*>(residual + (size_t)i * H)[c];
        const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(&ru);
        uint4 ro;
        __nv_bfloat16* rob = reinterpret_cast<__nv_bfloat16*>(&ro);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float sum_bf = __bfloat162float(__float2bfloat16(v[j][q]));
          rob[q] = __float2bfloat16(sum_bf + __bfloat162float(rb[q]));
          v[j][q] = __bfloat162float(rob[q]);
          ss += v[j][q] * v[j][q];
        }
        reinterpret_cast<uint4*>(residual + (size_t)i * H)[c] = ro;
      }
    }
    const float tot = block_sum(ss, red);
    const float inv = rsqrtf(tot / (float)H + eps);
    const size_t out_off = ag_off + ((size_t)me * Ts + i) * row_bytes;
#pragma unroll
    for (int j = 0; j < kMaxVec; ++j) {
      const int c = threadIdx.x + j * blockDim.x;
      if (c < nchunk) {
        const float4 w0 = reinterpret_cast<const float4*>(w)[2 * c];
        const float4 w1 = reinterpret_cast<const float4*>(w)[2 * c + 1];
        const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        uint4 o;
        __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
        for (int q = 0; q < 8; ++q) ob[q] = __float2bfloat16(v[j][q] * inv * ww[q]);
        for (int qq = 0; qq < world; ++qq) {
          const int q = (me + qq) % world;
          *reinterpret_cast<uint4*>(peers.base[q] + out_off + (size_t)c * 16) = o;
        }
      }
    }
    __syncthreads();  // red[] reuse by the next row
  }
  __syncthreads();
  signal_and_wait(peers, b, 2 * epoch, wait_ns, status);
  if (threadIdx.x == 0) counters_of(mine)[b] = epoch;
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
// ll: LL protocol (T * H * 4 bytes per source area instead of T * H * 2); a communicator must
// pass the same value on every call.
extern "C" int b200_allreduce_fused(void* const* bases, int rank, int world, size_t slot_bytes, const void* in,
                                    void* out, void* residual, const void* bias, const float* w, float eps, int T,
                                    int H, int num_blocks, unsigned long long wait_ns, int* status, cudaStream_t s,
                                    const int* topk_ids, int k, int E_local, int eoff, int ll) {
  if (topk_ids != nullptr && (k < 1 || k > 16)) return kBadShape;
  if (wait_ns == 0) wait_ns = kDefaultWaitNs;
  if (world > kMaxRanks || world < 1 || H % 8 || H > 8192 || T < 0) return kBadShape;
  if ((size_t)T * H * (ll ? 4 : 2) * world > slot_bytes || (slot_bytes / world) % 16) return kBadShape;
  if (num_blocks < 1 || num_blocks > kMaxBlocks) return kBadShape;
  if (T == 0) return 0;
  CommPeers peers{};
  for (int i = 0; i < world; ++i) peers.base[i] = static_cast<uint8_t*>(bases[i]);
  peers.rank = rank;
  peers.world = world;
  peers.slot_bytes = slot_bytes;
  const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(in);
  __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out);
  __nv_bfloat16* r = static_cast<__nv_bfloat16*>(residual);
  const __nv_bfloat16* bb = static_cast<const __nv_bfloat16*>(bias);
  const dim3 grid(num_blocks), block(256);
  if (w != nullptr && ll)
    launch_k(allreduce_fused_kernel<true, true>, grid, block, 0, s, peers, x, topk_ids, k, E_local, eoff, o, r, bb, w,
             eps, T, H, wait_ns, status);
  else if (w != nullptr)
    launch_k(allreduce_fused_kernel<true, false>, grid, block, 0, s, peers, x, topk_ids, k, E_local, eoff, o, r, bb,
             w, eps, T, H, wait_ns, status);
  else if (ll)
    launch_k(allreduce_fused_kernel<false, true>, grid, block, 0, s, peers, x, topk_ids, k, E_local, eoff, o,
             (__nv_bfloat16*)nullptr, (const __nv_bfloat16*)nullptr, (const float*)nullptr, eps, T, H, wait_ns,
             status);
  else
    launch_k(allreduce_fused_kernel<false, false>, grid, block, 0, s, peers, x, topk_ids, k, E_local, eoff, o,
             (__nv_bfloat16*)nullptr, (const __nv_bfloat16*)nullptr, (const float*)nullptr, eps, T, H, wait_ns,
             status);
  return (int)cudaGetLastError();
}

// Sequence-parallel boundary (sp_boundary_kernel).  The region's slots are slot_bytes each and
// hold [RS area: area_bytes][guard: guard_bytes][AG area: area_bytes][guard]; the output is the
// AG area of `slot` ([T, H] bf16).  in: the partial [T, H] (or, with topk_ids, the per-route rows
// [T * k, H]); null when a GEMM has already stored the partial rows into the RS areas
// (b200_gemm_bf16_scatter).  residual: this rank's [T / world, H] rows, updated in place.
extern "C" int b200_sp_boundary(void* const* bases, int rank, int world, size_t slot_bytes, size_t area_bytes,
                                size_t guard_bytes, int slot, const void* in, void* residual, const void* bias,
                                const float* w, float eps, int T, int H, int num_blocks, unsigned long long wait_ns,
                                int* status, cudaStream_t s, const int* topk_ids, int k, int E_local, int eoff) {
  if (world > kMaxRanks || world < 1 || H % 8 || H > 8192 || T < 0 || T % world) return kBadShape;
  if (slot < 0 || slot > 1 || 2 * (area_bytes + guard_bytes) > slot_bytes || area_bytes % 16 || guard_bytes % 16)
    return kBadShape;
  if ((size_t)T * H * 2 > area_bytes || residual == nullptr || w == nullptr) return kBadShape;
  if (topk_ids != nullptr && (in == nullptr || k < 1 || k > 16)) return kBadShape;
  if (num_blocks < 1 || num_blocks > kMaxBlocks) return kBadShape;
  if (T == 0) return 0;
  if (wait_ns == 0) wait_ns = kDefaultWaitNs;
  CommPeers peers{};
  for (int i = 0; i < world; ++i) peers.base[i] = static_cast<uint8_t*>(bases[i]);
  peers.rank = rank;
  peers.world = world;
  peers.slot_bytes = slot_bytes;
  const size_t rs_off = kHeaderBytes + (size_t)slot * slot_bytes;
  const size_t ag_off = rs_off + area_bytes + guard_bytes;
  const int grid = std::min(num_blocks, T / world);
  if (in != nullptr)
    launch_k(sp_boundary_kernel<false>, dim3(grid), dim3(256), 0, s, peers, rs_off, ag_off, (const __nv_bfloat16*)in,
             topk_ids, k, E_local, eoff, (__nv_bfloat16*)residual, (const __nv_bfloat16*)bias, w, eps, T, H, wait_ns,
             status);
  else
    launch_k(sp_boundary_kernel<true>, dim3(grid), dim3(256), 0, s, peers, rs_off, ag_off,
             (const __nv_bfloat16*)nullptr, (const int*)nullptr, 0, 0, 0, (__nv_bfloat16*)residual,
             (const __nv_bfloat16*)bias, w, eps, T, H, wait_ns, status);
  return (int)cudaGetLastError();
}

