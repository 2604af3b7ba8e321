// Expert-parallel token all-to-all over NVLink peer memory: dispatch and combine.
//
// Restates the reference's EP all-to-all (vllm_neuron/parallel/all2all.py:56 dispatch:
// metadata, permute, all_to_all_v; :186 combine: all_to_all_v then topk_reduce) as two
// push kernels with no host round trip, so a decode step stays one CUDA graph.
//
// Every rank owns E_local consecutive experts (expert e on rank e / E_local) and a slice
// [t_begin, t_end) of its T tokens (the whole batch with attention DP; a TP rank's share when
// the tokens are replicated over TP).  Per call:
//   dispatch: CTA (d, c) compacts the tokens that route to any expert of rank d (block
//     scan; a token goes to d once however many of its experts d owns), pushes rows
//     i = c, c + cpd, ... of that list with their k expert ids and weights into rank d's
//     receive area for this rank (NVLink stores), fills the unused rows' ids with -1,
//     releases flag [c][me] on rank d, then waits for rank d's CTA (me, c) flag on this rank
//     and copies the rows it covers into x_recv / ids_recv / w_recv ([world * T] rows, rank
//     s's rows at s * T).  The expert GEMM then runs on the received rows; -1 ids and the
//     other ranks' experts are skipped by its router.
//   combine: CTA (s, c) pushes the expert outputs of rank s's rows i = c, c + cpd, ... back
//     into rank s's return area for this rank, releases flag [c][me] on rank s, waits for
//     every peer's flags, then sums each of its tokens over the ranks it was sent to
//     (send_idx from the dispatch) into out [T, H] (zero for tokens outside the slice, so
//     out is a partial sum over the TP group, completed by the layer-boundary reduction).
// Buffers: one cudaMalloc'd region per rank, IPC-mapped by its peers:
//   [header: dispatch flags [16][8], combine flags [16][8], per-CTA dispatch / combine epochs]
//   [slot 0][slot 1], slot = [x: world][Tc][H] bf16 | ids: [world][Tc][k] i32 | w: f32 | [y: world][Tc][H] bf16
// Slots alternate by epoch.  A rank writes slot e & 1 of a peer in call e only after it has
// passed the combine barrier of call e - 1, which the peer reaches only after finishing its
// expert GEMM and combine reads of call e - 1, and so of e - 2.  Waits are bounded (~2 s)
// and set the status word.  Every rank must make the same calls with the same T.
#include "common.cuh"
#include "launch.h"
#include "launch_pdl.h"

namespace b200 {
namespace {

constexpr int kEpMaxRanks = 8;
constexpr int kEpMaxCpd = 16;
constexpr int kEpHeaderBytes = 64 * 1024;

struct EpArgs {
  uint8_t* base[kEpMaxRanks];
  int rank, world, cpd;  // grid = world * cpd CTAs
  int T, Tc, H, k, E_local, t_begin, t_end;
  size_t slot_bytes;
};

B200_D uint32_t* disp_flags(uint8_t* base) { return reinterpret_cast<uint32_t*>(base); }
B200_D uint32_t* comb_flags(uint8_t* base) { return reinterpret_cast<uint32_t*>(base) + kEpMaxCpd * kEpMaxRanks; }
B200_D uint32_t* disp_epoch(uint8_t* base) { return reinterpret_cast<uint32_t*>(base) + 2 * kEpMaxCpd * kEpMaxRanks; }
B200_D uint32_t* comb_epoch(uint8_t* base) {
  return reinterpret_cast<uint32_t*>(base) + 2 * kEpMaxCpd * kEpMaxRanks + kEpMaxCpd * kEpMaxRanks;
}

struct SlotView {
  __nv_bfloat16* x;  // [world][Tc][H]
  int* ids;          // [world][Tc][k]
  float* w;          // [world][Tc][k]
  __nv_bfloat16* y;  // [world][Tc][H]
};

B200_D SlotView slot_view(uint8_t* base, int slot, const EpArgs& a) {
  uint8_t* p = base + kEpHeaderBytes + (size_t)slot * a.slot_bytes;
  const size_t nx = (size_t)a.world * a.Tc * a.H * sizeof(__nv_bfloat16);
  const size_t nm = (size_t)a.world * a.Tc * a.k * 4;
  SlotView v;
  v.x = reinterpret_cast<__nv_bfloat16*>(p);
  v.ids = reinterpret_cast<int*>(p + nx);
  v.w = reinterpret_cast<float*>(p + nx + nm);
  v.y = reinterpret_cast<__nv_bfloat16*>(p + nx + 2 * nm);
  return v;
}

B200_D void ep_st_release(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
B200_D uint32_t ep_ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
B200_D uint64_t ep_now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// bounded wait (kDefaultWaitNs) for *f >= epoch; on timeout sets the status word and gives up
B200_D void ep_wait(const uint32_t* f, uint32_t epoch, int* status) {
  if (ep_ld_acquire(f) >= epoch) return;
  const uint64_t t0 = ep_now_ns();
  for (uint32_t i = 1;; ++i) {
    if (ep_ld_acquire(f) >= epoch) return;
    if ((i & 255) == 0 && ep_now_ns() - t0 > kDefaultWaitNs) {
      if (status) atomicCAS(status, 0, kWaitTimeout);
      return;
    }
  }
}

// exclusive prefix sum of one int per thread over a 256-thread block; returns the total
B200_D int block_exclusive_scan(int v, int* excl, int* warp_tot) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  int inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  if (lane == 31) warp_tot[wid] = inc;
  __syncthreads();
  int base = 0, total = 0;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) {
    if (i < wid) base += warp_tot[i];
    total += warp_tot[i];
  }
  *excl = base + inc - v;
  return total;
}

__global__ void __launch_bounds__(256) ep_dispatch_kernel(EpArgs a, const __nv_bfloat16* __restrict__ x,
                                                          const int* __restrict__ ids, const float* __restrict__ w,
                                                          __nv_bfloat16* __restrict__ x_recv, int* __restrict__ ids_recv,
                                                          float* __restrict__ w_recv, int* __restrict__ send_idx,
                                                          int* status) {
  pdl_wait();
  pdl_trigger();
  __shared__ uint32_t s_epoch;
  __shared__ int warp_tot[8];
  __shared__ int list[256];
  const int b = blockIdx.x, d = b % a.world, c = b / a.world;
  uint8_t* me = a.base[a.rank];
  if (threadIdx.x == 0) s_epoch = disp_epoch(me)[b] + 1;
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const int slot = epoch & 1;

  // 1. tokens of this rank's slice that route to rank d, in token order
  const int t = threadIdx.x;
  int f = 0;
  if (t < a.T && t >= a.t_begin && t < a.t_end) {
    for (int j = 0; j < a.k; ++j) {
      const int e = ids[t * a.k + j];
      if (e >= 0 && e / a.E_local == d) f = 1;
    }
  }
  int pos = 0;
  const int n_d = block_exclusive_scan(f, &pos, warp_tot);
  if (c == 0 && t < a.T) send_idx[t * a.world + d] = f ? pos : -1;
  if (f && pos % a.cpd == c) list[pos / a.cpd] = t;
  __syncthreads();

  // 2. push rows pos = c, c + cpd, ... (< n_d) and the metadata of every row i = c (mod cpd), i < T
  const SlotView dst = slot_view(a.base[d], slot, a);
  const size_t src_row0 = (size_t)a.rank * a.Tc;
  const int nchunk = a.H / 8;
  const int m = n_d > c ? (n_d - c + a.cpd - 1) / a.cpd : 0;
  for (int li = 0; li < m; ++li) {
    const int tt = list[li], i = li * a.cpd + c;
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)tt * a.H);
    uint4* out = reinterpret_cast<uint4*>(dst.x + (src_row0 + i) * a.H);
    for (int ch = threadIdx.x; ch < nchunk; ch += blockDim.x) out[ch] = src[ch];
  }
  for (int q = threadIdx.x; c + q * a.cpd < a.T; q += blockDim.x) {
    const int i = c + q * a.cpd;
    int* di = dst.ids + (src_row0 + i) * a.k;
    float* dw = dst.w + (src_row0 + i) * a.k;
    if (i < n_d) {
      const int tt = list[q];
      for (int j = 0; j < a.k; ++j) {
        di[j] = ids[tt * a.k + j];
        dw[j] = w[tt * a.k + j];
      }
    } else {
      for (int j = 0; j < a.k; ++j) {
        di[j] = -1;
        dw[j] = 0.f;
      }
    }
  }
  __syncthreads();  // the release below covers the CTA's pushes

  // 3. signal rank d; wait for rank d's CTA (me, c) to have pushed into this rank
  if (threadIdx.x == 0) {
    ep_st_release(disp_flags(a.base[d]) + c * kEpMaxRanks + a.rank, epoch);
    ep_wait(disp_flags(me) + c * kEpMaxRanks + d, epoch, status);
  }
  __syncthreads();

  // 4. copy the rows rank d sent (i = c, c + cpd, ...) into the dense receive tensors
  const SlotView mine = slot_view(me, slot, a);
  const size_t from0 = (size_t)d * a.Tc;
  for (int i = c; i < a.T; i += a.cpd) {
    const int* si = mine.ids + (from0 + i) * a.k;
    const float* sw = mine.w + (from0 + i) * a.k;
    const int r = d * a.T + i;
    const int valid = __ldcg(si) >= 0;
    if (threadIdx.x < a.k) {
      ids_recv[r * a.k + threadIdx.x] = __ldcg(si + threadIdx.x);
      w_recv[r * a.k + threadIdx.x] = __ldcg(sw + threadIdx.x);
    }
    if (valid) {
      const uint4* src = reinterpret_cast<const uint4*>(mine.x + (from0 + i) * a.H);
      uint4* out = reinterpret_cast<uint4*>(x_recv + (size_t)r * a.H);
      for (int ch = threadIdx.x; ch < nchunk; ch += blockDim.x) out[ch] = __ldcg(src + ch);
    }
  }
  if (threadIdx.x == 0) disp_epoch(me)[b] = epoch;
}

__global__ void __launch_bounds__(256) ep_combine_kernel(EpArgs a, const __nv_bfloat16* __restrict__ y_recv,
                                                         const int* __restrict__ ids_recv,
                                                         const int* __restrict__ send_idx,
                                                         __nv_bfloat16* __restrict__ out, int* status) {
  pdl_wait();
  pdl_trigger();
  __shared__ uint32_t s_epoch;
  const int b = blockIdx.x, s = b % a.world, c = b / a.world;
  uint8_t* me = a.base[a.rank];
  if (threadIdx.x == 0) s_epoch = comb_epoch(me)[b] + 1;
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const int slot = epoch & 1;
  const int nchunk = a.H / 8;

  // 1. return the expert outputs of rank s's rows i = c, c + cpd, ... to rank s
  const SlotView dst = slot_view(a.base[s], slot, a);
  const size_t to0 = (size_t)a.rank * a.Tc;
  for (int i = c; i < a.T; i += a.cpd) {
    const int r = s * a.T + i;
    if (ids_recv[r * a.k] < 0) continue;  // unused row
    const uint4* src = reinterpret_cast<const uint4*>(y_recv + (size_t)r * a.H);
    uint4* o = reinterpret_cast<uint4*>(dst.y + (to0 + i) * a.H);
    for (int ch = threadIdx.x; ch < nchunk; ch += blockDim.x) o[ch] = src[ch];
  }
  __syncthreads();

  // 2. signal rank s; wait until every rank has returned every row to this rank
  if (threadIdx.x == 0) ep_st_release(comb_flags(a.base[s]) + c * kEpMaxRanks + a.rank, epoch);
  if (threadIdx.x < a.world * a.cpd) {
    const int pd = threadIdx.x % a.world, pc = threadIdx.x / a.world;
    ep_wait(comb_flags(me) + pc * kEpMaxRanks + pd, epoch, status);
  }
  __syncthreads();

  // 3. out[t] = sum over the ranks t was sent to of their returned rows
  const SlotView mine = slot_view(me, slot, a);
  for (int t = b; t < a.T; t += gridDim.x) {
    for (int ch = threadIdx.x; ch < nchunk; ch += blockDim.x) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int d = 0; d < a.world; ++d) {
        const int si = send_idx[t * a.world + d];
        if (si < 0) continue;
        const uint4 u = __ldcg(reinterpret_cast<const uint4*>(mine.y + ((size_t)d * a.Tc + si) * a.H) + ch);
        const __nv_bfloat16* hb = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] += __bfloat162float(hb[q]);
      }
      uint4 o;
      __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
      for (int q = 0; q < 8; ++q) ob[q] = __float2bfloat16(acc[q]);
      reinterpret_cast<uint4*>(out + (size_t)t * a.H)[ch] = o;
    }
  }
  if (threadIdx.x == 0) comb_epoch(me)[b] = epoch;
}

int ep_args(EpArgs* a, void* const* bases, int rank, int world, size_t slot_bytes, int cpd, int T, int Tc, int H,
            int k, int E_local, int t_begin, int t_end) {
  if (world < 1 || world > kEpMaxRanks || rank < 0 || rank >= world) return kBadShape;
  if (cpd < 1 || cpd > kEpMaxCpd || T < 0 || T > Tc || Tc > 256 || Tc % 4) return kBadShape;
  if (H % 8 || H <= 0 || k < 1 || k > 16 || E_local < 1) return kBadShape;
  if (t_begin < 0 || t_end < t_begin || t_end > T) return kBadShape;
  if (slot_bytes < (size_t)world * Tc * (2 * (size_t)H * 2 + (size_t)k * 8)) return kBadShape;
  for (int i = 0; i < world; ++i) a->base[i] = static_cast<uint8_t*>(bases[i]);
  a->rank = rank;
  a->world = world;
  a->cpd = cpd;
  a->T = T;
  a->Tc = Tc;
  a->H = H;
  a->k = k;
  a->E_local = E_local;
  a->t_begin = t_begin;
  a->t_end = t_end;
  a->slot_bytes = slot_bytes;
  return 0;
}

}  // namespace
}  // namespace b200

using namespace b200;

extern "C" int b200_ep_dispatch(void* const* bases, int rank, int world, size_t slot_bytes, int cpd, int T, int Tc,
                                int H, int k, int E_local, int t_begin, int t_end, const void* x, const int* ids,
                                const float* w, void* x_recv, int* ids_recv, float* w_recv, int* send_idx,
                                int* status, cudaStream_t s) {
  EpArgs a;
  const int rc = ep_args(&a, bases, rank, world, slot_bytes, cpd, T, Tc, H, k, E_local, t_begin, t_end);
  if (rc) return rc;
  if (T == 0) return 0;
  launch_k(ep_dispatch_kernel, dim3(world * cpd), dim3(256), 0, s, a, (const __nv_bfloat16*)x, ids, w,
           (__nv_bfloat16*)x_recv, ids_recv, w_recv, send_idx, status);
  return (int)cudaGetLastError();
}

extern "C" int b200_ep_combine(void* const* bases, int rank, int world, size_t slot_bytes, int cpd, int T, int Tc,
                               int H, int k, const void* y_recv, const int* ids_recv, const int* send_idx, void* out,
                               int* status, cudaStream_t s) {
  EpArgs a;
  const int rc = ep_args(&a, bases, rank, world, slot_bytes, cpd, T, Tc, H, k, 1, 0, T);
  if (rc) return rc;
  if (T == 0) return 0;
  launch_k(ep_combine_kernel, dim3(world * cpd), dim3(256), 0, s, a, (const __nv_bfloat16*)y_recv, ids_recv,
           send_idx, (__nv_bfloat16*)out, status);
  return (int)cudaGetLastError();
}
