// Dense bf16 GEMM on the Blackwell tensor cores, for every linear layer of the models
// (QKV, o_proj, router, LM head, dense MLP, vision linears), with an optional fused
// all-reduce through NVSwitch.
//
//   Y[T, N] = X[T, K] . W[N, K]^T (+ bias[N])        X, W, Y bf16; fp32 accumulation
//
// Semantics of the reference's linear layers (nn/cpl.py:135, nn/rpl.py:136,
// functional/attention/qkv.py:646, functional/attention/o_proj.py:117, functional/mlp.py:29,
// functional/moe/router.py:71): a plain GEMM with bias; row-parallel layers all-reduce the
// partial products over the TP group and add the bias once.
//
// Design (B200):
//   * orientation: the weight is the MMA's M operand (128 output features per tile) and the
//     tokens its N operand (NT = 16 ... 256 per tile), D[128 x NT] = W_tile . X_tile^T in
//     TMEM.  Decode (T <= 64) is weight-streaming bound, so a narrow N keeps the activation
//     tile cheap; prefill uses NT = 256 and tiles the tokens too;
//   * both operands come straight from the row-major tensors by 2-D TMA (128-byte swizzle,
//     box 64 x 128 for W and 64 x NT for X, no multicast) into a STAGES-deep ring guarded by
//     mbarriers; one elected thread issues tcgen05.mma.kind::f16 (4 x K=16 per stage) into
//     one of two TMEM accumulators, so the epilogue of one tile overlaps the next tile's MMAs;
//   * the kernel is persistent (one CTA per SM) over work items (n tile, m tile, k split).
//     When there are fewer output tiles than SMs, K is split so that every SM streams
//     weights: each split adds its fp32 tile into a scratch with vector atomics and the
//     last split to arrive (a counter per tile and epilogue warp, no waiting) reads the
//     sums once, clears them and runs the epilogue;
//   * epilogue kStore: + bias, bf16 (or fp32, e.g. router logits), transposed through
//     shared memory into 16 / 32-byte row stores of Y;
//   * epilogue kReduce (fused all-reduce): every split of every rank adds its fp32 tile
//     into one accumulator with multimem.red.add (NVSwitch multicast: the switch performs
//     the additions in every GPU's copy), then the CTA bumps a multicast counter with a
//     release (one count per CTA and tile); `allreduce_finish` waits for the counter to reach all ranks' tile count and
//     applies bias + residual + RMSNorm (or a plain bf16 cast), zeroing the accumulator for
//     the call after next.  Without a multicast object (one GPU) the same epilogue uses
//     plain global atomics on the local accumulator.  No TMA and no library kernel ever
//     touches another GPU's memory; the only cross-GPU traffic is multimem reductions.
#include <algorithm>
#include <cstdlib>

#include "launch.h"
#include "launch_pdl.h"
#include "tcgen05.cuh"

namespace b200 {
namespace dense {

constexpr int kBM = 128;  // weight rows per tile (MMA M)
constexpr int kBK = 64;   // K elements per pipeline stage: one 128-byte swizzle row of bf16

// Shared memory: STAGES x (A + B) ring, the epilogue transpose staging, (cluster split K)
// two receive buffers of 128 x NT fp32 partials, then the mbarriers.
template <int NT, bool CL>
struct Cfg {
  static constexpr int kA = kBM * kBK * 2;  // 16 KB
  static constexpr int kB = NT * kBK * 2;
  static constexpr int kStages = CL ? (NT >= 64 ? 6 : 8) : (NT <= 64 ? 8 : NT == 128 ? 6 : NT <= 192 ? 5 : 4);
  static constexpr int kStage = kA + kB;
  static constexpr int kOffEpi = kStages * kStage;
  static constexpr int kEpiBytes = 4 * 16 * 36 * 4;  // per epilogue warp: 16 tokens x 36 floats
  static constexpr int kOffRecv = kOffEpi + kEpiBytes;
  static constexpr int kRecvBuf = CL ? kBM * NT * 4 : 0;  // one buffer: [splits][NT][128/splits] fp32
  static constexpr int kOffBar = kOffRecv + 2 * kRecvBuf;
  static constexpr int kNumBars = 2 * kStages + 4 + (CL ? 4 : 0);
  static constexpr int kBytes = kOffBar + kNumBars * 8 + 16;
  static constexpr int kAlloc = kBytes + 1024;  // slack to align the base to 1024
  static constexpr uint32_t kTmemCols = 2 * NT <= 32 ? 32 : 2 * NT <= 64 ? 64 : 2 * NT <= 128 ? 128
                                        : 2 * NT <= 256 ? 256 : 512;
  static_assert(kAlloc <= 232448, "shared memory budget");
};

enum Epi : int { kStore = 0, kReduce = 1 };

// Layout of the fused all-reduce region (one per group, symmetric across the ranks; the
// multicast mapping covers the counters and the accumulators):
//   [0]   u32 tile counter, parity 0      (multicast target)
//   [4]   u32 tile counter, parity 1      (multicast target)
//   [64]  u32 epoch (calls completed, local)
//   [68]  u32 finished-CTA counter of the current finish call (local)
//   [256] fp32 accumulator, parity 0, [T_cap, H_cap]; then parity 1
constexpr size_t kRedHeader = 256;
B200_HD size_t red_region_bytes(int T_cap, int H_cap) { return kRedHeader + 2ull * T_cap * H_cap * 4; }

struct Args {
  int T, N, K;
  int ldy;
  int m_tiles, n_tiles, splits, k_stages, sps;
  const __nv_bfloat16* bias;  // [N] or null (kStore)
  const float* alpha;         // fp8 operands: dequantisation factor, per tensor ([1]) or per feature ([N])
  int alpha_n;                // 0 (none), 1 or N
  void* y;                    // kStore: [T, ldy], bf16 (or fp32 when out_f32)
  int out_f32;
  float* ws;                  // kStore, splits > 1: fp32 sums [T, N], zero between calls
  int* counters;              // kStore, splits > 1: [tiles][4 epilogue warps], zero between calls
  uint8_t* red_uc;            // kReduce: this rank's region (unicast)
  uint8_t* red_mc;            // kReduce: multicast mapping of the region (null: local atomics)
  int H_cap, T_cap;           // kReduce accumulator geometry (row stride H_cap)
  // kStore scatter (dst_rows > 0): token row t goes to ydst[t / dst_rows] at row t % dst_rows
  // (row stride ldy, bf16), e.g. the reduce-scatter receive areas of a sequence-parallel
  // boundary on the peer GPUs (plain 16-byte stores over NVLink)
  uint8_t* ydst[8];
  int dst_rows;
  int* status;
  // optional per-CTA timeline (%globaltimer ns, 8 slots per CTA) for latency analysis:
  // entry, setup done, first TMA issued, first MMA issued, first accumulator ready, first
  // epilogue done, last epilogue done, exit.  Null in normal use.
  unsigned long long* trace;
};

B200_D void stamp(const Args& a, int slot) {
  if (a.trace != nullptr) a.trace[(size_t)blockIdx.x * 8 + slot] = tc::globaltimer_ns();
}

B200_D void mc_red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("multimem.red.relaxed.sys.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b),
               "f"(c), "f"(d)
               : "memory");
}
B200_D void mc_red_release_add_u32(uint32_t* p, uint32_t v) {
  asm volatile("multimem.red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
B200_D uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
B200_D float4 ld_cg_f4(const float* p) {
  float4 v;
  asm volatile("ld.global.cg.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
  return v;
}

// Y[t, f .. f+7] = v + bias (bf16 or fp32 row of 8 features, 16 / 32-byte stores).
B200_D void store8(const Args& a, int t, int f, const float* v) {
  float o[8];
#pragma unroll
  for (int h = 0; h < 8; ++h) {
    const float sc = a.alpha_n == 0 ? 1.f : a.alpha[a.alpha_n == 1 ? 0 : f + h];
    o[h] = v[h] * sc + (a.bias != nullptr ? __bfloat162float(a.bias[f + h]) : 0.f);
  }
  if (a.out_f32) {
    float* y = static_cast<float*>(a.y) + (size_t)t * a.ldy + f;
    *reinterpret_cast<float4*>(y) = make_float4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<float4*>(y + 4) = make_float4(o[4], o[5], o[6], o[7]);
  } else {
    uint4 u;
    __nv_bfloat162* ob = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int h = 0; h < 4; ++h) ob[h] = __floats2bfloat162_rn(o[2 * h], o[2 * h + 1]);
    __nv_bfloat16* yrow;
    if (a.dst_rows > 0) {
      const int q = t / a.dst_rows;
      yrow = reinterpret_cast<__nv_bfloat16*>(a.ydst[q]) + (size_t)(t - q * a.dst_rows) * a.ldy;
    } else {
      yrow = static_cast<__nv_bfloat16*>(a.y) + (size_t)t * a.ldy;
    }
    *reinterpret_cast<uint4*>(yrow + f) = u;
  }
}

// kReduce: count one finished tile of this CTA toward the call.  Each epilogue warp adds its
// part of the tile to the accumulator and then bumps a per-accumulator counter in shared
// memory (acq_rel at CTA scope, so the last warp has observed the others' reductions); the
// last of the 4 warps releases one count at system scope, through the multicast mapping when
// there is one (one increment per CTA and tile, not per warp).  No warp ever waits here.
B200_D void count_tile(const Args& a, int* tile_done, int s_parity) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) {
    int prev;
    asm volatile("atom.shared.acq_rel.cta.add.u32 %0, [%1], 1;" : "=r"(prev) : "r"(tc::smem_addr(tile_done)) : "memory");
    if (prev == 3) {
      *tile_done = 0;  // the next tile using this accumulator starts after all 4 warps released it
      uint32_t* cnt = reinterpret_cast<uint32_t*>(a.red_mc ? a.red_mc : a.red_uc) + s_parity;
      if (a.red_mc != nullptr) {
        mc_red_release_add_u32(cnt, 1u);
      } else {
        __threadfence();
        atomicAdd(cnt, 1u);
      }
    }
  }
}

struct Item {
  int m0, n0, split, tile, ks0, ks1;
};
// Work item w: without clusters, w enumerates (n tile, m tile, k split) with the split
// fastest; with cluster split K (split = the CTA's rank in its cluster) w enumerates tiles.
B200_D Item item_of(const Args& a, int w, int cl_split = -1) {
  Item it;
  it.split = cl_split >= 0 ? cl_split : w % a.splits;
  const int rest = cl_split >= 0 ? w : w / a.splits;
  const int mt = rest % a.m_tiles, nt = rest / a.m_tiles;
  it.tile = nt * a.m_tiles + mt;
  it.m0 = mt * kBM;
  it.n0 = nt;  // scaled by NT by the caller
  it.ks0 = it.split * a.sps;
  it.ks1 = it.split == a.splits - 1 ? a.k_stages : min(a.k_stages, it.ks0 + a.sps);
  return it;
}

// F8: both operands e4m3 (tcgen05 kind::f8f6f4, 128 K elements per 128-byte stage row),
// else bf16 (kind::f16, 64 K elements per stage row); the shared-memory layout is the same.
template <int NT, int EPI, bool CL, bool F8 = false>
__global__ void __launch_bounds__(256, 1) gemm_kernel(const __grid_constant__ CUtensorMap tmW,
                                                      const __grid_constant__ CUtensorMap tmX, Args a) {
  if (threadIdx.x == 0) stamp(a, 0);
  pdl_wait();  // predecessor output visible (programmatic dependent launch)
  pdl_trigger();
  using C = Cfg<NT, CL>;
  extern __shared__ uint8_t smem_raw[];
  // work distribution: persistent CTAs (or clusters) stride over the work items
  const int crank = CL ? (int)tc::cluster_ctarank() : -1;
  const int W = CL ? a.m_tiles * a.n_tiles : a.m_tiles * a.n_tiles * a.splits;
  const int first = CL ? (int)tc::cluster_id_x() : (int)blockIdx.x;
  const int step = CL ? (int)tc::ncluster_x() : (int)gridDim.x;
  if (!CL && first >= W) return;  // (a cluster never returns early: its CTAs synchronise)
  const uint32_t raw_off = tc::smem_addr(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_off & 1023u)) & 1023u);
  float* epi_stage = reinterpret_cast<float*>(smem + C::kOffEpi);
  float* recv = reinterpret_cast<float*>(smem + C::kOffRecv);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* empty = full + C::kStages;
  uint64_t* acc_full = empty + C::kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* recv_full = acc_empty + 2;   // CL: [2] partials of my rows arrived from every split
  uint64_t* recv_empty = recv_full + 2;  // CL: [2] every owner has consumed my partials
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffBar + C::kNumBars * 8);
  __shared__ int s_parity;
  __shared__ int s_tile_done[2];  // kReduce: epilogue warps done with the tile of each accumulator

  const int S = a.splits;               // CL: cluster size
  const int R = CL ? kBM / S : kBM;     // CL: output rows (features) reduced by each CTA
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&acc_full[i], 1);
      tc::mbar_init(&acc_empty[i], 4);  // one arrive per epilogue warp
      if constexpr (CL) {
        tc::mbar_init(&recv_full[i], S * (R >= 32 ? R / 32 : 1));  // sender warps per owner
        tc::mbar_init(&recv_empty[i], S * 4);                       // every owner's 4 warps
      }
    }
    tc::fence_barrier_init();
    tc::prefetch_tmap(&tmW);
    tc::prefetch_tmap(&tmX);
    if constexpr (EPI == kReduce) {
      const uint32_t ep = *reinterpret_cast<volatile uint32_t*>(a.red_uc + 64);
      s_parity = (int)((ep + 1u) & 1u);
    }
    s_tile_done[0] = s_tile_done[1] = 0;
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, C::kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if constexpr (CL) tc::cluster_sync();  // every CTA's mbarriers exist before any remote arrive
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0) stamp(a, 1);

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int it = 0;
      bool ok = true;
      for (int w = first; w < W && ok; w += step) {
        const Item wi = item_of(a, w, crank);
        for (int kt = wi.ks0; kt < wi.ks1; ++kt, ++it) {
          const int s = it % C::kStages, use = it / C::kStages;
          if (it >= C::kStages && !tc::mbar_wait(&empty[s], (use - 1) & 1, a.status)) {
            ok = false;
            break;
          }
          tc::mbar_arrive_expect_tx(&full[s], C::kStage);
          uint8_t* st = smem + s * C::kStage;
          constexpr int kEB = F8 ? 2 * kBK : kBK;  // K elements per 128-byte stage row
          tc::tma_load_2d(st, &tmW, kt * kEB, wi.m0, &full[s]);
          tc::tma_load_2d(st + C::kA, &tmX, kt * kEB, wi.n0 * NT, &full[s]);
          if (it == 0) stamp(a, 2);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      const uint32_t idesc = F8 ? tc::idesc_f8f6f4_e4m3(kBM, NT) : tc::idesc_f16_bf16(kBM, NT);
      int it = 0, local = 0;
      bool ok = true;
      for (int w = first; w < W && ok; w += step) {
        const Item wi = item_of(a, w, crank);
        const int acc = local & 1, ause = local >> 1;
        if (local >= 2 && !tc::mbar_wait(&acc_empty[acc], (ause - 1) & 1, a.status)) break;
        tc::fence_after_sync();
        const uint32_t t_d = tmem + acc * NT;
        for (int kt = wi.ks0; kt < wi.ks1; ++kt, ++it) {
          const int s = it % C::kStages, use = it / C::kStages;
          if (!tc::mbar_wait(&full[s], use & 1, a.status)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          uint8_t* st = smem + s * C::kStage;
          const uint64_t ad = tc::desc_sw128(st);
          const uint64_t bd = tc::desc_sw128(st + C::kA);
#pragma unroll
          for (int kb = 0; kb < 4; ++kb) {  // 4 x (K=16 bf16 or K=32 e4m3) per 128-byte stage (+32 bytes each)
            if constexpr (F8)
              tc::mma_f8f6f4(t_d, ad + 2 * kb, bd + 2 * kb, idesc, (kt > wi.ks0 || kb > 0) ? 1u : 0u);
            else
              tc::mma_f16(t_d, ad + 2 * kb, bd + 2 * kb, idesc, (kt > wi.ks0 || kb > 0) ? 1u : 0u);
          }
          tc::mma_commit(&empty[s]);
          if (it == 0) stamp(a, 3);
        }
        tc::mma_commit(&acc_full[acc]);
        ++local;
      }
    }
  } else if (warp >= 4) {
    // ---------------- epilogue (TMEM lanes 32*(warp%4) ..) ----------------
    const int ew = warp & 3;
    float* stg = epi_stage + ew * 16 * 36;  // [16 tokens][36] fp32 (32 features + pad)
    int local = 0;
    for (int w = first; w < W; w += step) {
      const Item wi = item_of(a, w, crank);
      const int acc = local & 1, ause = local >> 1;
      if (!tc::mbar_wait(&acc_full[acc], ause & 1, a.status)) break;
      tc::fence_after_sync();
      if (local == 0 && ew == 0 && lane == 0) stamp(a, 4);
      const int n0 = wi.n0 * NT;
      const int nvalid = min(NT, a.T - n0);
      const int fbase = wi.m0 + ew * 32;  // first feature of this warp
      const uint32_t lane_addr = tmem + acc * NT + ((uint32_t)(ew * 32) << 16);
      bool released = false;
      if constexpr (CL) {
        // cluster split K: the CTA of rank j owns rows [j R, (j + 1) R) of the tile.  Every
        // CTA sends its partial rows to their owners' receive buffer (DSMEM), each owner sums
        // the splits of its rows and stores them.  Buffers alternate between tiles; a
        // sender waits until every owner has consumed the buffer it used two tiles ago.
        const int b = local & 1, buse = local >> 1;
        if (local >= 2 && !tc::mbar_wait_cluster(&recv_empty[b], (buse - 1) & 1, a.status)) break;
        const uint32_t buf_local = tc::smem_addr(recv + (size_t)b * (kBM * NT));
        for (int c = 0; c < NT; c += 16) {
          if (c >= nvalid) break;
          uint32_t r[16];
          tc::tmem_ld_32x32b_x16(lane_addr + c, r);
          tc::tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) stg[i * 36 + lane] = __uint_as_float(r[i]);
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int q = lane + 32 * j, row = q >> 3, part = q & 7;
            const int feat = ew * 32 + part * 4, owner = feat / R, ml = feat % R, tok = c + row;
            if (tok < nvalid) {
              const float4 u = *reinterpret_cast<const float4*>(stg + row * 36 + part * 4);
              const uint32_t off = (uint32_t)((((crank * NT) + tok) * R + ml) * 4);  // [src][token][row]
              tc::st_cluster_v4(tc::mapa(buf_local + off, (uint32_t)owner), u.x, u.y, u.z, u.w);
            }
          }
          __syncwarp();
        }
        // the warp's DSMEM stores precede its arrivals on the owners of its rows
        __syncwarp();
        if (lane == 0) {
          const int o0 = (ew * 32) / R, o1 = (ew * 32 + 31) / R;
          for (int o = o0; o <= o1; ++o) tc::mbar_arrive_remote(tc::mapa(tc::smem_addr(&recv_full[b]), (uint32_t)o));
        }
        // the partial has left TMEM: the MMA warp may reuse the accumulator
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&acc_empty[acc]);
        released = true;
        // reduce my rows once every split has sent them
        if (!tc::mbar_wait_cluster(&recv_full[b], buse & 1, a.status)) break;
        const float* mine = recv + (size_t)b * (kBM * NT);
        const int runs = R / 8;
        for (int k = ew * 32 + lane; k < nvalid * runs; k += 128) {
          const int tok = k / runs, ml = (k % runs) * 8;
          float v8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          for (int sp = 0; sp < S; ++sp) {
            const float* p = mine + ((size_t)(sp * NT + tok) * R + ml);
            const float4 u0 = *reinterpret_cast<const float4*>(p), u1 = *reinterpret_cast<const float4*>(p + 4);
            v8[0] += u0.x, v8[1] += u0.y, v8[2] += u0.z, v8[3] += u0.w;
            v8[4] += u1.x, v8[5] += u1.y, v8[6] += u1.z, v8[7] += u1.w;
          }
          const int f = wi.m0 + crank * R + ml;
          if (f < a.N) {
            if constexpr (EPI == kReduce) {
              // the cluster's sum of these rows joins the other ranks' through NVSwitch
              float* dst = reinterpret_cast<float*>((a.red_mc ? a.red_mc : a.red_uc) + kRedHeader) +
                           (size_t)s_parity * a.T_cap * a.H_cap + (size_t)(n0 + tok) * a.H_cap + f;
              if (a.red_mc != nullptr) {
                mc_red_add_v4(dst, v8[0], v8[1], v8[2], v8[3]);
                mc_red_add_v4(dst + 4, v8[4], v8[5], v8[6], v8[7]);
              } else {
                atomicAdd(reinterpret_cast<float4*>(dst), make_float4(v8[0], v8[1], v8[2], v8[3]));
                atomicAdd(reinterpret_cast<float4*>(dst + 4), make_float4(v8[4], v8[5], v8[6], v8[7]));
              }
            } else {
              store8(a, n0 + tok, f, v8);
            }
          }
        }
        if constexpr (EPI == kReduce) count_tile(a, &s_tile_done[b], s_parity);
        // my buffer b is free again for every sender
        __syncwarp();
        if (lane == 0)
          for (int o = 0; o < S; ++o) tc::mbar_arrive_remote(tc::mapa(tc::smem_addr(&recv_empty[b]), (uint32_t)o));
      } else if constexpr (EPI == kStore) {
        if (a.splits > 1) {
          // split K without clusters (wide tiles): every split adds its tile into the fp32
          // scratch [T, N] (vector atomics in L2); the last split to arrive (a counter per
          // tile and epilogue warp: no barrier spans warps) reads the sums of its warp's 32
          // features once, clears them for the next call and stores Y.
          for (int c = 0; c < NT; c += 16) {
            if (c >= nvalid) break;
            uint32_t r[16];
            tc::tmem_ld_32x32b_x16(lane_addr + c, r);
            tc::tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i) stg[i * 36 + lane] = __uint_as_float(r[i]);
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int q = lane + 32 * j, row = q >> 3, part = q & 7;
              const int t = n0 + c + row, f = fbase + part * 4;
              if (row < nvalid - c && f < a.N)
                atomicAdd(reinterpret_cast<float4*>(a.ws + (size_t)t * a.N + f),
                          *reinterpret_cast<const float4*>(stg + row * 36 + part * 4));
            }
            __syncwarp();
          }
          __threadfence();
          __syncwarp();
          int last = 0;
          if (lane == 0) last = atomicAdd(&a.counters[wi.tile * 4 + ew], 1) == a.splits - 1;
          if (__shfl_sync(0xffffffffu, last, 0) != 0) {
            __threadfence();
            for (int c = 0; c < nvalid; c += 16) {
#pragma unroll
              for (int j = 0; j < 2; ++j) {
                const int q = lane + 32 * j, row = q >> 2, part = q & 3;
                const int t = n0 + c + row, f = fbase + part * 8;
                if (row < nvalid - c && f < a.N) {
                  float* p = a.ws + (size_t)t * a.N + f;
                  const float4 u0 = ld_cg_f4(p), u1 = ld_cg_f4(p + 4);
                  *reinterpret_cast<float4*>(p) = make_float4(0.f, 0.f, 0.f, 0.f);
                  *reinterpret_cast<float4*>(p + 4) = make_float4(0.f, 0.f, 0.f, 0.f);
                  const float v8[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
                  store8(a, t, f, v8);
                }
              }
            }
            if (lane == 0) a.counters[wi.tile * 4 + ew] = 0;  // every split has arrived
          }
        } else {
          for (int c = 0; c < NT; c += 16) {
            if (c >= nvalid) break;
            uint32_t r[16];
            tc::tmem_ld_32x32b_x16(lane_addr + c, r);
            tc::tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i) stg[i * 36 + lane] = __uint_as_float(r[i]);
            __syncwarp();
            // 16 tokens x 32 features: each lane stores 2 runs of 8 features
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const int q = lane + 32 * j, row = q >> 2, part = q & 3;
              const int t = n0 + c + row, f = fbase + part * 8;
              if (row < nvalid - c && f < a.N) store8(a, t, f, stg + row * 36 + part * 8);
            }
            __syncwarp();
          }
        }
      } else {
        float* accp = reinterpret_cast<float*>((a.red_mc ? a.red_mc : a.red_uc) + kRedHeader) +
                      (size_t)s_parity * a.T_cap * a.H_cap;
        for (int c = 0; c < NT; c += 16) {
          if (c >= nvalid) break;
          uint32_t r[16];
          tc::tmem_ld_32x32b_x16(lane_addr + c, r);
          tc::tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) stg[i * 36 + lane] = __uint_as_float(r[i]);
          __syncwarp();
          // 16 tokens x 32 features: each lane adds 4 runs of 4 features
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int q = lane + 32 * j, row = q >> 3, part = q & 7;
            const int t = n0 + c + row, f = fbase + part * 4;
            if (row < nvalid - c && f < a.N) {
              const float4 u = *reinterpret_cast<const float4*>(stg + row * 36 + part * 4);
              float* dst = accp + (size_t)t * a.H_cap + f;
              if (a.red_mc != nullptr)
                mc_red_add_v4(dst, u.x, u.y, u.z, u.w);
              else
                atomicAdd(reinterpret_cast<float4*>(dst), u);
            }
          }
          __syncwarp();
        }
        count_tile(a, &s_tile_done[acc], s_parity);
      }
      if (!released) {
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&acc_empty[acc]);
      }
      if (ew == 0 && lane == 0) stamp(a, local == 0 ? 5 : 6);
      ++local;
    }
    // scattered rows may sit in other GPUs' memory: complete them at system scope before the
    // kernel ends (the collective that follows releases its flags after this kernel)
    if (a.dst_rows > 0) __threadfence_system();
  }
  tc::fence_before_sync();
  __syncthreads();
  // no CTA of a cluster leaves while another may still write its shared memory or arrive on
  // its barriers
  if constexpr (CL) tc::cluster_sync();
  if (warp == 1) tc::tmem_dealloc(tmem, C::kTmemCols);
  if (threadIdx.x == 0) stamp(a, 7);
}

// ---------------------------------------------------------------- finish of the fused all-reduce
// One CTA per group of rows.  Waits until every rank's tiles of this call have been added
// (the parity's counter reaches `expected`), then per row:
//   kNorm: s = bf16(acc + bias); residual = bf16(s + residual); out = RMSNorm(residual) * w
//   else : out = bf16(acc + bias)
// and zeroes the accumulator rows it read.  The last CTA to finish resets the counter and
// advances the epoch (both reused two calls later; see the header comment of this file).
template <bool kNorm>
__global__ void __launch_bounds__(256) finish_kernel(uint8_t* red_uc, int H_cap, int T_cap, uint32_t expected,
                                                     __nv_bfloat16* __restrict__ out,
                                                     __nv_bfloat16* __restrict__ residual,
                                                     const __nv_bfloat16* __restrict__ bias,
                                                     const float* __restrict__ w, float eps, int T, int H,
                                                     unsigned long long wait_ns, int* status) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[32];
  __shared__ uint32_t s_epoch;
  volatile uint32_t* epoch_w = reinterpret_cast<volatile uint32_t*>(red_uc + 64);
  uint32_t* done = reinterpret_cast<uint32_t*>(red_uc + 68);
  if (threadIdx.x == 0) {
    const uint32_t e = *epoch_w + 1u;
    s_epoch = e;
    const uint32_t* cnt = reinterpret_cast<const uint32_t*>(red_uc) + (e & 1u);
    if (ld_acquire_sys_u32(cnt) < expected) {
      const uint64_t t0 = tc::globaltimer_ns();
      for (uint32_t i = 1;; ++i) {
        if (ld_acquire_sys_u32(cnt) >= expected) break;
        if ((i & 255) == 0 && tc::globaltimer_ns() - t0 > wait_ns) {
          if (status) atomicCAS(status, 0, kWaitTimeout);
          break;
        }
      }
    }
  }
  __syncthreads();
  const uint32_t e = s_epoch;
  float* acc = reinterpret_cast<float*>(red_uc + kRedHeader) + (size_t)(e & 1u) * T_cap * H_cap;
  const int nq = H / 4;
  for (int r = blockIdx.x; r < T; r += gridDim.x) {
    constexpr int kMaxVec = 8;  // H <= 256 threads * 8 * 4 = 8192
    float v[kMaxVec][4];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i) {
      const int c = threadIdx.x + i * blockDim.x;
      if (c < nq) {
        float* p = acc + (size_t)r * H_cap + 4 * c;
        const float4 s4 = ld_cg_f4(p);
        *reinterpret_cast<float4*>(p) = make_float4(0.f, 0.f, 0.f, 0.f);
        v[i][0] = s4.x;
        v[i][1] = s4.y;
        v[i][2] = s4.z;
        v[i][3] = s4.w;
        if (bias) {
#pragma unroll
          for (int q = 0; q < 4; ++q) v[i][q] += __bfloat162float(bias[4 * c + q]);
        }
        if constexpr (kNorm) {
          const __nv_bfloat162* rp = reinterpret_cast<const __nv_bfloat162*>(residual + (size_t)r * H + 4 * c);
          const float2 r0 = __bfloat1622float2(rp[0]), r1 = __bfloat1622float2(rp[1]);
          const float rr[4] = {r0.x, r0.y, r1.x, r1.y};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float sum_bf = __bfloat162float(__float2bfloat16(v[i][q]));
            v[i][q] = __bfloat162float(__float2bfloat16(sum_bf + rr[q]));
            ss += v[i][q] * v[i][q];
          }
          __nv_bfloat162* wp = reinterpret_cast<__nv_bfloat162*>(residual + (size_t)r * H + 4 * c);
          wp[0] = __floats2bfloat162_rn(v[i][0], v[i][1]);
          wp[1] = __floats2bfloat162_rn(v[i][2], v[i][3]);
        } else {
          __nv_bfloat162* op = reinterpret_cast<__nv_bfloat162*>(out + (size_t)r * H + 4 * c);
          op[0] = __floats2bfloat162_rn(v[i][0], v[i][1]);
          op[1] = __floats2bfloat162_rn(v[i][2], v[i][3]);
        }
      }
    }
    if constexpr (kNorm) {
      const float tot = block_sum(ss, red);
      const float inv = rsqrtf(tot / (float)H + eps);
#pragma unroll
      for (int i = 0; i < kMaxVec; ++i) {
        const int c = threadIdx.x + i * blockDim.x;
        if (c < nq) {
          const float4 w4 = *reinterpret_cast<const float4*>(w + 4 * c);
          __nv_bfloat162* op = reinterpret_cast<__nv_bfloat162*>(out + (size_t)r * H + 4 * c);
          op[0] = __floats2bfloat162_rn(v[i][0] * inv * w4.x, v[i][1] * inv * w4.y);
          op[1] = __floats2bfloat162_rn(v[i][2] * inv * w4.z, v[i][3] * inv * w4.w);
        }
      }
      __syncthreads();  // red[] reuse by the next row
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(done, 1u) == gridDim.x - 1) {
      // every CTA has passed its wait and read its rows
      reinterpret_cast<uint32_t*>(red_uc)[e & 1u] = 0u;
      *done = 0u;
      *epoch_w = e;
      __threadfence_system();
    }
  }
}

// ---------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// Row-major [rows, K] (bf16, or e4m3 when f8) with row stride ld elements; box of one
// 128-byte row (64 bf16 / 128 e4m3) x box_rows, 128-byte swizzle.
static int make_map(CUtensorMap* m, const void* p, int rows, int K, int ld, int box_rows, bool f8 = false) {
  auto enc = encoder();
  if (!enc) return kBadShape;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * (f8 ? 1 : 2)};
  cuuint32_t box[2] = {(cuuint32_t)(f8 ? 2 * kBK : kBK), (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, f8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(p), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : kTensorMapErrorBase + (int)r;
}

static int sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  static int cached[64] = {0};
  if (dev >= 0 && dev < 64 && cached[dev]) return cached[dev];
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (n <= 0) n = 148;
  if (dev >= 0 && dev < 64) cached[dev] = n;
  return n;
}

struct Plan {
  int nt, m_tiles, n_tiles, splits, k_stages, sps;
  bool cluster;  // the K splits of a tile are one thread-block cluster (DSMEM reduction)
};

// A forced token tile width for non-cluster plans (tile-size measurements): VLLM_B200_GEMM_NT
// at the first call, or b200_gemm_force_nt; 0 = the planner's choice.
static int g_forced_nt = -1;
static int valid_nt(int v) {
  return (v == 16 || v == 32 || v == 64 || v == 128 || v == 160 || v == 192 || v == 224 || v == 256) ? v : 0;
}
static int forced_nt() {
  if (g_forced_nt < 0) {
    const char* e = std::getenv("VLLM_B200_GEMM_NT");
    g_forced_nt = valid_nt(e != nullptr ? std::atoi(e) : 0);
  }
  return g_forced_nt;
}

// Relative cost of one token of a tile of width nt against a 256-wide tile (the per-tile
// epilogue and the shared-memory traffic per MMA grow as the tile narrows).
static double tile_cost(int nt) { return 1.0 + 0.5 * (256 - nt) / 128.0; }

// Tile width from the token count.  When the output tiles cannot occupy every SM, K is
// split: for decode widths (NT <= 64) across a cluster of 2 / 4 / 8 CTAs that reduce over
// DSMEM, chosen by a small cost model (rounds of tiles x stages per split, plus a reduction
// cost); for wider tiles with vector atomics (at least 8 stages per split, at most 4 splits).
static Plan make_plan(int T, int N, int K, int max_splits, bool allow_cluster = true, bool f8 = false,
                      int sms_override = 0) {
  Plan p;
  p.nt = T <= 16 ? 16 : T <= 32 ? 32 : T <= 64 ? 64 : T <= 128 ? 128 : 256;
  p.m_tiles = cdiv(N, kBM);
  const int sms = sms_override > 0 ? sms_override : sm_count();
  if (p.nt == 256) {
    // wide tiles: the width whose busiest SM does the least work (waves x width x the width's
    // relative cost), so the last wave is not left mostly idle (184 tiles of 256 tokens on 148
    // SMs run two waves, the second a quarter full)
    double best = 1e30;
    for (int nt : {256, 224, 192, 160, 128}) {
      const double cost = (double)cdiv(p.m_tiles * cdiv(T, nt), sms) * nt * tile_cost(nt);
      if (cost < best - 1e-9) {
        best = cost;
        p.nt = nt;
      }
    }
  }
  if (forced_nt() > 0) p.nt = forced_nt();
  // Wide token tiles that leave SMs idle (fewer tiles than SMs): halve the tile while that
  // lowers the busiest SM's share (waves x tile width); K is split only after that, since a
  // split of a wide tile reduces through global atomics.  A projection of a 512-token prefill
  // chunk at N = 2880 thus runs 92 tiles of 128 tokens instead of 46 tiles split three ways.
  while ((p.nt == 256 || p.nt == 128) && forced_nt() == 0 && p.m_tiles * cdiv(T, p.nt) < sms) {
    const int half = p.nt / 2;
    if ((long long)cdiv(p.m_tiles * cdiv(T, half), sms) * half >= (long long)cdiv(p.m_tiles * cdiv(T, p.nt), sms) * p.nt)
      break;
    p.nt = half;
  }
  p.n_tiles = cdiv(T, p.nt);
  p.k_stages = cdiv(K, f8 ? 2 * kBK : kBK);
  p.cluster = false;
  const int tiles = p.m_tiles * p.n_tiles;
  int splits = 1;
  if (p.nt <= 64 && allow_cluster && max_splits > 1) {
    double best = (double)cdiv(tiles, sms) * (p.k_stages + 1.0);
    for (int sp = 2; sp <= 8 && sp <= max_splits; sp *= 2) {
      if (p.k_stages / sp < 2) break;
      const int clusters = std::max(1, sms / sp);
      const double cost = (double)cdiv(tiles, clusters) * (cdiv(p.k_stages, sp) + 3.0);
      if (cost < best) {
        best = cost;
        splits = sp;
      }
    }
    p.cluster = splits > 1;
  } else if (tiles < sms && max_splits > 1) {
    splits = std::max(1, std::min({sms / tiles, p.k_stages / 8, max_splits, 4}));
  }
  if (p.cluster) {  // exactly `splits` non-empty ranges; the last one takes the remainder
    p.sps = p.k_stages / splits;
    p.splits = splits;
  } else {
    p.sps = cdiv(p.k_stages, splits);
    p.splits = cdiv(p.k_stages, p.sps);
  }
  return p;
}

static Plan make_plan_on(int T, int N, int K, int max_splits, int sms) {
  return make_plan(T, N, K, max_splits, true, false, sms);
}

static unsigned long long* g_trace = nullptr;  // set by b200_gemm_set_trace (analysis only)

template <int NT, int EPI, bool CL, bool F8 = false>
static int launch(const Plan& p, const void* x, int ldx, const void* w, Args a, cudaStream_t s) {
  using C = Cfg<NT, CL>;
  a.trace = g_trace;
  CUtensorMap tw, tx;
  int rc;
  if ((rc = make_map(&tw, w, a.N, a.K, a.K, kBM, F8))) return rc;
  if ((rc = make_map(&tx, x, a.T, a.K, ldx, NT, F8))) return rc;
  auto kern = gemm_kernel<NT, EPI, CL, F8>;
  static bool attr = false;
  static int max_clusters[9] = {0};
  if (!attr) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kAlloc);
    attr = true;
  }
  const int tiles = p.m_tiles * p.n_tiles;
  if constexpr (CL) {
    const int S = p.splits;
    if (max_clusters[S] == 0) {  // co-resident clusters of this size (one persistent wave)
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(S * std::max(1, sm_count() / S));
      cfg.blockDim = dim3(256);
      cfg.dynamicSmemBytes = C::kAlloc;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = S;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) n = sm_count() / S;
      cudaGetLastError();
      max_clusters[S] = n;
    }
    const int clusters = std::min(tiles, max_clusters[S]);
    launch_kc(kern, dim3(clusters * S), dim3(256), C::kAlloc, s, (unsigned)S, tw, tx, a);
  } else {
    const int grid = std::min(sm_count(), tiles * p.splits);
    launch_k(kern, dim3(grid), dim3(256), C::kAlloc, s, tw, tx, a);
  }
  return (int)cudaGetLastError();
}

template <int EPI, bool F8 = false>
static int dispatch(const Plan& p, const void* x, int ldx, const void* w, const Args& a, cudaStream_t s) {
  if (p.cluster) {
    switch (p.nt) {
      case 16: return launch<16, EPI, true, F8>(p, x, ldx, w, a, s);
      case 32: return launch<32, EPI, true, F8>(p, x, ldx, w, a, s);
      default: return launch<64, EPI, true, F8>(p, x, ldx, w, a, s);
    }
  }
  switch (p.nt) {
    case 16: return launch<16, EPI, false, F8>(p, x, ldx, w, a, s);
    case 32: return launch<32, EPI, false, F8>(p, x, ldx, w, a, s);
    case 64: return launch<64, EPI, false, F8>(p, x, ldx, w, a, s);
    case 128: return launch<128, EPI, false, F8>(p, x, ldx, w, a, s);
    case 160: return launch<160, EPI, false, F8>(p, x, ldx, w, a, s);
    case 192: return launch<192, EPI, false, F8>(p, x, ldx, w, a, s);
    case 224: return launch<224, EPI, false, F8>(p, x, ldx, w, a, s);
    default: return launch<256, EPI, false, F8>(p, x, ldx, w, a, s);
  }
}

static bool misaligned_host(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) != 0; }

static int check_common(const void* x, int ldx, const void* w, int T, int N, int K) {
  if (T < 0 || N <= 0 || K <= 0 || K % 8 || ldx % 8 || ldx < K) return kBadShape;
  if (misaligned_host(x) || misaligned_host(w)) return kBadAlignment;
  return 0;
}

}  // namespace dense
}  // namespace b200

using namespace b200;
using namespace b200::dense;

// Workspace a call of b200_gemm_bf16 needs (fp32 elements of `ws`, ints of `counters`).
extern "C" void b200_gemm_workspace(int T, int N, int K, int max_splits, int64_t* ws_floats, int64_t* n_counters) {
  const Plan p = make_plan(T, N, K, max_splits);
  const int64_t tiles = (int64_t)p.m_tiles * p.n_tiles;
  *ws_floats = p.splits > 1 ? (int64_t)T * N : 0;
  *n_counters = p.splits > 1 ? 4 * tiles : 0;
}

// Y[T, N] (row stride ldy) = X[T, K] (row stride ldx) . W[N, K]^T + bias.  ws / counters: see
// b200_gemm_workspace (counters must be zero on entry and are zero again on exit).
// Y is bf16, or fp32 when out_f32 (ldy in elements of Y).  ws must be zero on entry when K
// is split and is zero again on exit.
extern "C" int b200_gemm_bf16(void* y, int ldy, int out_f32, const void* x, int ldx, const void* w, const void* bias,
                              int T, int N, int K, float* ws, int64_t ws_floats, int* counters, int64_t n_counters,
                              int max_splits, int* status, cudaStream_t s) {
  int rc = check_common(x, ldx, w, T, N, K);
  if (rc) return rc;
  if (ldy % 8 || ldy < N || N % 8) return kBadShape;
  if (T == 0) return 0;
  const Plan p = make_plan(T, N, K, max_splits);
  Args a{};
  a.T = T, a.N = N, a.K = K, a.ldy = ldy;
  a.m_tiles = p.m_tiles, a.n_tiles = p.n_tiles, a.splits = p.splits, a.k_stages = p.k_stages, a.sps = p.sps;
  a.bias = static_cast<const __nv_bfloat16*>(bias);
  a.y = y;
  a.out_f32 = out_f32;
  a.status = status;
  if (misaligned_host(y) || (out_f32 && ldy % 4)) return kBadAlignment;
  if (p.splits > 1) {
    const int64_t tiles = (int64_t)p.m_tiles * p.n_tiles;
    if (ws == nullptr || counters == nullptr || ws_floats < (int64_t)T * N || n_counters < 4 * tiles)
      return kScratchTooSmall;
    a.ws = ws;
    a.counters = counters;
  }
  return dispatch<kStore>(p, x, ldx, w, a, s);
}

// FP8 GEMM: Y[T, N] = (X[T, K] . W[N, K]^T) * alpha + bias with X and W e4m3 (row strides ldx
// and K bytes), alpha an fp32 dequantisation factor per tensor (alpha_n = 1) or per output
// feature (alpha_n = N), bias bf16 or null; Y bf16 (or fp32).  Workspace as b200_gemm_bf16.
extern "C" int b200_gemm_fp8(void* y, int ldy, int out_f32, const void* x, int ldx, const void* w, const void* bias,
                             const float* alpha, int alpha_n, int T, int N, int K, float* ws, int64_t ws_floats,
                             int* counters, int64_t n_counters, int max_splits, int* status, cudaStream_t s) {
  if (T < 0 || N <= 0 || K <= 0 || K % 16 || ldx % 16 || ldx < K) return kBadShape;
  if (misaligned_host(x) || misaligned_host(w)) return kBadAlignment;
  if (ldy % 8 || ldy < N || N % 8 || alpha == nullptr || (alpha_n != 1 && alpha_n != N)) return kBadShape;
  if (T == 0) return 0;
  const Plan p = make_plan(T, N, K, max_splits, true, true);
  Args a{};
  a.T = T, a.N = N, a.K = K, a.ldy = ldy;
  a.m_tiles = p.m_tiles, a.n_tiles = p.n_tiles, a.splits = p.splits, a.k_stages = p.k_stages, a.sps = p.sps;
  a.bias = static_cast<const __nv_bfloat16*>(bias);
  a.alpha = alpha;
  a.alpha_n = alpha_n;
  a.y = y;
  a.out_f32 = out_f32;
  a.status = status;
  if (misaligned_host(y) || (out_f32 && ldy % 4)) return kBadAlignment;
  if (p.splits > 1 && !p.cluster) {
    const int64_t tiles = (int64_t)p.m_tiles * p.n_tiles;
    if (ws == nullptr || counters == nullptr || ws_floats < (int64_t)T * N || n_counters < 4 * tiles)
      return kScratchTooSmall;
    a.ws = ws;
    a.counters = counters;
  }
  return dispatch<kStore, true>(p, x, ldx, w, a, s);
}

// Y = X . W^T (bf16, no bias) with token row t stored at dst[t / (T / n_dst)] + (t % (T / n_dst))
// rows of ldd elements: the producer of a reduce-scatter writes every row block straight into
// its owner's receive area (n_dst ranks, T % n_dst == 0; dst pointers may be peer memory,
// which only the epilogue's plain stores touch).  Workspace as b200_gemm_bf16.
extern "C" int b200_gemm_bf16_scatter(void* const* dst, int n_dst, int ldd, const void* x, int ldx, const void* w,
                                      int T, int N, int K, float* ws, int64_t ws_floats, int* counters,
                                      int64_t n_counters, int max_splits, int* status, cudaStream_t s) {
  int rc = check_common(x, ldx, w, T, N, K);
  if (rc) return rc;
  if (n_dst < 1 || n_dst > 8 || T % n_dst || ldd % 8 || ldd < N || N % 8) return kBadShape;
  for (int q = 0; q < n_dst; ++q)
    if (dst[q] == nullptr || misaligned_host(dst[q])) return kBadAlignment;
  if (T == 0) return 0;
  const Plan p = make_plan(T, N, K, max_splits);
  Args a{};
  a.T = T, a.N = N, a.K = K, a.ldy = ldd;
  a.m_tiles = p.m_tiles, a.n_tiles = p.n_tiles, a.splits = p.splits, a.k_stages = p.k_stages, a.sps = p.sps;
  a.y = dst[0];
  for (int q = 0; q < n_dst; ++q) a.ydst[q] = static_cast<uint8_t*>(dst[q]);
  a.dst_rows = T / n_dst;
  a.status = status;
  if (p.splits > 1 && !p.cluster) {
    const int64_t tiles = (int64_t)p.m_tiles * p.n_tiles;
    if (ws == nullptr || counters == nullptr || ws_floats < (int64_t)T * N || n_counters < 4 * tiles)
      return kScratchTooSmall;
    a.ws = ws;
    a.counters = counters;
  }
  return dispatch<kStore>(p, x, ldx, w, a, s);
}

extern "C" size_t b200_red_region_bytes(int T_cap, int H_cap) { return red_region_bytes(T_cap, H_cap); }

// The planner's decision for a bf16 GEMM of this shape on `sms` SMs (0: the current device's count):
// out[0..4] = token tile width, output tiles, K splits, cluster split (0/1), k stages per split.
extern "C" void b200_gemm_plan(int T, int N, int K, int max_splits, int sms, int* out) {
  const Plan p = make_plan_on(T, N, K, max_splits, sms);
  out[0] = p.nt;
  out[1] = p.m_tiles * p.n_tiles;
  out[2] = p.splits;
  out[3] = p.cluster ? 1 : 0;
  out[4] = p.sps;
}

// Force the token tile width of later non-cluster plans (0 restores the planner's choice).
extern "C" void b200_gemm_force_nt(int nt) { g_forced_nt = valid_nt(nt); }

// Latency analysis: every later GEMM launch writes 8 %globaltimer stamps per CTA to `buf`
// (device memory of grid x 8 u64; null turns it off).
extern "C" void b200_gemm_set_trace(void* buf) { g_trace = static_cast<unsigned long long*>(buf); }

// Fused all-reduce producer: adds X . W^T of this rank into the group's accumulator
// (multimem when red_mc is set, local atomics otherwise) and counts its tiles.  Returns the
// number of counts this rank adds per call through *items (one per CTA and tile; the finish
// call expects the sum over the ranks), or an error code.  K is only split across clusters
// (the splits of a tile are summed over DSMEM and pushed once).
extern "C" int b200_gemm_bf16_allreduce(const void* x, int ldx, const void* w, int T, int N, int K, void* red_uc,
                                        void* red_mc, int T_cap, int H_cap, int max_splits, int* items, int* status,
                                        cudaStream_t s) {
  int rc = check_common(x, ldx, w, T, N, K);
  if (rc) return rc;
  if (T > T_cap || N > H_cap || N % 4 || H_cap % 4 || red_uc == nullptr) return kBadShape;
  Plan p = make_plan(T, N, K, max_splits);
  if (!p.cluster && p.splits > 1) p = make_plan(T, N, K, 1);  // no partial pushed more than once
  *items = T == 0 ? 0 : p.m_tiles * p.n_tiles * p.splits;  // one count per CTA and tile
  if (T == 0) return 0;
  Args a{};
  a.T = T, a.N = N, a.K = K, a.ldy = N;
  a.m_tiles = p.m_tiles, a.n_tiles = p.n_tiles, a.splits = p.splits, a.k_stages = p.k_stages, a.sps = p.sps;
  a.red_uc = static_cast<uint8_t*>(red_uc);
  a.red_mc = static_cast<uint8_t*>(red_mc);
  a.T_cap = T_cap, a.H_cap = H_cap;
  a.status = status;
  return dispatch<kReduce>(p, x, ldx, w, a, s);
}

// Completes a fused all-reduce call: waits for `expected` tiles (all ranks), then writes
// out = RMSNorm(sum + bias + residual) * w with residual updated (w != null) or
// out = sum + bias (w == null).  wait_ns 0 = kDefaultWaitNs.
extern "C" int b200_allreduce_finish(void* red_uc, int T_cap, int H_cap, int expected, void* out, void* residual,
                                     const void* bias, const float* w, float eps, int T, int H, int num_blocks,
                                     unsigned long long wait_ns, int* status, cudaStream_t s) {
  if (T < 0 || T > T_cap || H > H_cap || H % 4 || H > 8192 || num_blocks < 1 || expected < 0) return kBadShape;
  if (w != nullptr && residual == nullptr) return kBadShape;
  if (T == 0) return 0;
  if (wait_ns == 0) wait_ns = kDefaultWaitNs;
  const int grid = std::min(num_blocks, T);
  if (w != nullptr)
    launch_k(finish_kernel<true>, dim3(grid), dim3(256), 0, s, (uint8_t*)red_uc, H_cap, T_cap, (uint32_t)expected,
             (__nv_bfloat16*)out, (__nv_bfloat16*)residual, (const __nv_bfloat16*)bias, w, eps, T, H, wait_ns,
             status);
  else
    launch_k(finish_kernel<false>, dim3(grid), dim3(256), 0, s, (uint8_t*)red_uc, H_cap, T_cap, (uint32_t)expected,
             (__nv_bfloat16*)out, (__nv_bfloat16*)nullptr, (const __nv_bfloat16*)bias, (const float*)nullptr, eps,
             T, H, wait_ns, status);
  return (int)cudaGetLastError();
}
