// Mixture-of-experts forward on the Blackwell block-scaled tensor cores.
//
// Semantics (restated from functional/moe/moe_cte.py:448 and moe_block_tkg.py:56 of the
// Trainium plugin): for every route (token t, slot j) whose expert is local,
//   h   = W13[e] x_t + b13[e]               (gate/up rows interleaved: 2i gate, 2i+1 up)
//   a_i = min(g_i, L) * sigmoid(alpha * min(g_i, L)) * (clamp(u_i, -L, L) + 1)
//   y   = (W2[e] a + b2[e]) * w_tj
//   out_t = sum_j y_tj                        (partial over this rank's experts)
//
// Design (B200):
//   * weights stay in the checkpoint's MX format: e2m1 (or e4m3) values, ue8m0 scale per
//     32 along K; rows are re-laid out once at load time only to pad K to a multiple of
//     128 and to put the scales into 128-row x 4-block "atoms" (512 B) that tcgen05.cp
//     copies straight into tensor memory;
//   * activations are quantised per route to MXFP8 (e4m3 + ue8m0 per 32) into the same
//     atom layout, grouped by expert (device-side histogram / scan / scatter: no host sync);
//   * GEMMs are D[128 weight rows x NT routes] = W . X^T with
//     tcgen05.mma.kind::mxf8f6f4.block_scale (A = weights, B = routes), fp32 accumulators
//     in TMEM, operands staged by TMA (128-byte swizzle, no multicast) through an
//     mbarrier ring, one elected thread issuing MMAs; small N keeps decode weight-streaming
//     bound, larger N serves prefill;
//   * epilogues read TMEM with tcgen05.ld: GEMM1 adds the bias and applies the clamped
//     SwiGLU across the interleaved row pairs; GEMM2 adds the bias, scales by the route
//     affinity and writes the per-route row; a reduce kernel sums each token's routes.
#include "launch.h"
#include "launch_pdl.h"
#include "moe.h"
#include "tcgen05.cuh"

namespace b200 {

constexpr int kSfAtom = 512;  // 128 rows x 4 scale bytes

// Weight / activation formats of the grouped GEMM: block-scaled MX (weights e2m1 or e4m3,
// activations e4m3, ue8m0 scales per 32 along K; tcgen05 kind::mxf8f6f4) or plain bf16
// (tcgen05 kind::f16).  Every format stages 128-byte K rows per pipeline stage: 128
// elements of fp8 / unpacked fp4, 64 of bf16.
enum WFmt : int { kFmtFp4 = 0, kFmtFp8 = 1, kFmtBf16 = 2 };
template <int FMT>
struct FmtTraits {
  static constexpr int kKStage = FMT == kFmtBf16 ? 64 : 128;  // K elements per stage
  static constexpr bool kScaled = FMT != kFmtBf16;
};


B200_HD size_t sf_byte(int atom, int kgroups, int row_in_atom, int kb) {
  // kb = 32-element block index along K; atoms are [atom][kb/4][512]
  return ((size_t)atom * kgroups + (kb >> 2)) * kSfAtom + (row_in_atom & 31) * 16 + (row_in_atom >> 5) * 4 +
         (kb & 3);
}

// ------------------------------------------------------------------------- routing
// One CTA: histogram of local routes per expert (shared-memory atomics), a block-wide
// exclusive scan of the counts and of the tile counts (one thread per expert), the tile
// list written in parallel, then the scatter of route ids into expert order.
__global__ void __launch_bounds__(1024) moe_route_kernel(const int* __restrict__ topk_ids, int TK, int E, int off,
                                                         int nt, int max_tiles, MoeWorkspace ws) {
  pdl_wait();  // predecessor output visible (programmatic dependent launch)
  pdl_trigger();
  extern __shared__ int sm[];
  int* cnt = sm;           // [E]
  int* cur = sm + E;       // [E]   scatter cursors
  __shared__ int warp_tot[2][32];
  for (int i = threadIdx.x; i < E; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  for (int r = threadIdx.x; r < TK; r += blockDim.x) {
    const int e = topk_ids[r] - off;
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  // exclusive scan over experts of (rows, tiles); E <= blockDim.x
  const int e = threadIdx.x;
  const int lane = e & 31, wid = e >> 5;
  int v_rows = e < E ? cnt[e] : 0;
  int v_tiles = e < E ? cdiv(cnt[e], nt) : 0;
  int a = v_rows, b = v_tiles;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int ya = __shfl_up_sync(0xffffffffu, a, o), yb = __shfl_up_sync(0xffffffffu, b, o);
    if (lane >= o) {
      a += ya;
      b += yb;
    }
  }
  if (lane == 31) {
    warp_tot[0][wid] = a;
    warp_tot[1][wid] = b;
  }
  __syncthreads();
  if (wid == 0) {
    int ta = lane < (int)(blockDim.x >> 5) ? warp_tot[0][lane] : 0;
    int tb = lane < (int)(blockDim.x >> 5) ? warp_tot[1][lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int ya = __shfl_up_sync(0xffffffffu, ta, o), yb = __shfl_up_sync(0xffffffffu, tb, o);
      if (lane >= o) {
        ta += ya;
        tb += yb;
      }
    }
    warp_tot[0][lane] = ta;  // inclusive prefix of warp totals
    warp_tot[1][lane] = tb;
  }
  __syncthreads();
  const int base_rows = (wid > 0 ? warp_tot[0][wid - 1] : 0) + a - v_rows;
  const int base_tiles = (wid > 0 ? warp_tot[1][wid - 1] : 0) + b - v_tiles;
  if (e < E) {
    ws.offsets[e] = base_rows;
    ws.atom_base[e] = base_tiles;  // one 512-byte scale atom per N tile
    cur[e] = base_rows;
    for (int t = 0; t < v_tiles; ++t) {
      const int ti = base_tiles + t;
      if (ti < max_tiles) {
        ws.tiles[2 * ti] = e;
        ws.tiles[2 * ti + 1] = t * nt;
      }
    }
    if (e == E - 1) {
      ws.offsets[E] = base_rows + v_rows;
      ws.atom_base[E] = base_tiles + v_tiles;
      *ws.num_tiles = min(base_tiles + v_tiles, max_tiles);
    }
  }
  __syncthreads();
  for (int r = threadIdx.x; r < TK; r += blockDim.x) {
    const int ee = topk_ids[r] - off;
    if (ee >= 0 && ee < E) ws.row_route[atomicAdd(&cur[ee], 1)] = r;
  }
}

// ------------------------------------------------------------------ MXFP8 quantise
// One warp per permuted row.  Source row = x[row_route[r] / k] (gather) or src[r].
__global__ void __launch_bounds__(128) moe_quant_kernel(uint8_t* __restrict__ q, uint8_t* __restrict__ sf,
                                                        const __nv_bfloat16* __restrict__ src, int src_ld,
                                                        const int* __restrict__ row_route, int k_gather,
                                                        const int* __restrict__ offsets,
                                                        const int* __restrict__ atom_base, int E, int K, int Kp,
                                                        int R_max, int src_rows, int atoms_max, int nt,
                                                        int* status) {
  pdl_wait();  // predecessor output visible (programmatic dependent launch)
  pdl_trigger();
  const int groups = (Kp / 32 + 31) / 32;  // 32-block groups per row
  const int gw = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int r = gw / groups, grp = gw % groups;
  const int lane = threadIdx.x & 31;
  if (r >= R_max || r >= offsets[E]) return;
  if (offsets[E] > R_max) {
    if (lane == 0) record(status, kBadIndex, 10, offsets[E]);
    return;
  }
  // expert of row r: last e with offsets[e] <= r (binary search)
  int lo = 0, hi = E;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (offsets[mid] <= r) lo = mid;
    else hi = mid;
  }
  const int e = lo;
  const int j = r - offsets[e];
  // every N tile owns a scale atom whose first `nt` rows it uses, so the MMA always reads
  // the scale factors from the atom's first TMEM columns
  const int atom = atom_base[e] + j / nt, ra = j % nt;
  const int kgroups = Kp / 128;
  const int srow = k_gather > 0 ? row_route[r] / k_gather : r;
  if (srow < 0 || srow >= src_rows || atom >= atoms_max) {
    if (lane == 0) record(status, kBadIndex, 11, srow >= src_rows || srow < 0 ? srow : 100000 + atom);
    return;
  }
  const __nv_bfloat16* s = src + (size_t)srow * src_ld;
  uint8_t* qr = q + (size_t)r * Kp;
  if (misaligned(s, 16) || misaligned(qr, 16)) {
    if (lane == 0) record(status, kBadAlignment, 12, (int)(reinterpret_cast<uintptr_t>(s) & 0xffff));
    return;
  }
  {
    const int kb = grp * 32 + lane;
    if (kb >= Kp / 32) return;
    uint4 o[2];
    uint8_t scale = 127;
    if (kb * 32 < K) {
      float v[32];
      const uint4* p = reinterpret_cast<const uint4*>(s + kb * 32);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 u = p[c];
        const __nv_bfloat16* hb = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[c * 8 + i] = __bfloat162float(hb[i]);
      }
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
      int ex = 0;  // floor(log2(amax)) - 8 (e4m3 emax), from the exponent bits
      if (amax > 0.f) {
        const int be = (int)((__float_as_uint(amax) >> 23) & 0xff);
        ex = (be == 0 ? -127 : be - 127) - 8;
        ex = max(-127, min(127, ex));
      }
      scale = (uint8_t)(ex + 127);
      const float inv = exp2f((float)-ex);
      uint8_t* ob = reinterpret_cast<uint8_t*>(o);
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        const __nv_fp8x2_storage_t pr =
            __nv_cvt_float2_to_fp8x2(make_float2(v[i] * inv, v[i + 1] * inv), __NV_SATFINITE, __NV_E4M3);
        ob[i] = (uint8_t)(pr & 0xff);
        ob[i + 1] = (uint8_t)(pr >> 8);
      }
    } else {
      o[0] = make_uint4(0, 0, 0, 0);
      o[1] = make_uint4(0, 0, 0, 0);
    }
    uint4* qo = reinterpret_cast<uint4*>(qr + kb * 32);
    qo[0] = o[0];
    qo[1] = o[1];
    sf[sf_byte(atom, kgroups, ra, kb)] = scale;
  }
}

// ------------------------------------------------------------------ bf16 gather
// One warp per permuted row: copy x[row_route[r] / k] (bf16, K elements) to dst row r.
__global__ void __launch_bounds__(128) moe_gather_kernel(__nv_bfloat16* __restrict__ dst, int ld_dst,
                                                         const __nv_bfloat16* __restrict__ src, int src_ld,
                                                         const int* __restrict__ row_route, int k_gather,
                                                         const int* __restrict__ offsets, int E, int K, int R_max,
                                                         int src_rows, int* status) {
  pdl_wait();  // predecessor output visible (programmatic dependent launch)
  pdl_trigger();
  const int r = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (r >= R_max || r >= offsets[E]) return;
  const int srow = row_route[r] / k_gather;
  if (srow < 0 || srow >= src_rows) {
    if (lane == 0) record(status, kBadIndex, 13, srow);
    return;
  }
  const uint4* s4 = reinterpret_cast<const uint4*>(src + (size_t)srow * src_ld);
  uint4* d4 = reinterpret_cast<uint4*>(dst + (size_t)r * ld_dst);
  for (int c = lane; c < K / 8; c += 32) d4[c] = s4[c];
}

// ------------------------------------------------------------------------- GEMM
// Persistent grouped GEMM: one CTA per SM loops over work items (N tile of one expert x
// 128-row M tile, M fastest so consecutive items share the activation tile in L2).
//   warp 0 lane 0 : TMA producer through a STAGES-deep shared-memory ring (runs ahead
//                   across work items);
//   warp 1        : allocates TMEM; lane 0 issues tcgen05.cp (scale factors) and
//                   tcgen05.mma into one of two TMEM accumulators;
//   warps 4..7    : epilogue for TMEM lanes 32*(w%4).., overlapping the next item's MMAs.
enum Epi : int { kEpiSwiglu = 0, kEpiDown = 1 };

template <int NT, int STAGES>
struct GemmSmem {
  static constexpr int kA = 128 * 128;  // bytes per A stage (padded fp4 or fp8)
  static constexpr int kB = NT * 128;
  static constexpr int kOffB = STAGES * kA;
  static constexpr int kOffSfa = kOffB + STAGES * kB;
  static constexpr int kOffSfb = kOffSfa + STAGES * kSfAtom;
  static constexpr int kOffBar = kOffSfb + STAGES * kSfAtom;
  // epilogue staging: per epilogue warp one 16-token x (its 32 rows) bf16 block, so the
  // output leaves in 16-byte row segments instead of 2-byte scattered stores
  static constexpr int kOffStage = ((kOffBar + (2 * STAGES + 4) * 8 + 16 + 127) / 128) * 128;
  static constexpr int kStageBytes = 4 * 1024;
  static constexpr int kBytes = kOffStage + kStageBytes;
  static constexpr int kAlloc = kBytes + 1024;  // slack to align the base to 1024
  static constexpr int kTmemNeed = 2 * NT + 8;  // two accumulators + SFA + SFB columns
  static constexpr uint32_t kTmemCols = kTmemNeed <= 32 ? 32 : kTmemNeed <= 64 ? 64 : kTmemNeed <= 128 ? 128
                                        : kTmemNeed <= 256 ? 256 : 512;
};

struct WorkItem {
  int e, n0, row0, mt, tile;
  bool valid;
};

B200_D WorkItem decode_item(const MoeWorkspace& ws, int w, int mtiles, int E_local, int R_max, int atoms_max) {
  WorkItem it;
  it.tile = w / mtiles;
  it.mt = w % mtiles;
  it.e = ws.tiles[2 * it.tile];
  it.n0 = ws.tiles[2 * it.tile + 1];
  it.valid = it.e >= 0 && it.e < E_local && it.n0 >= 0 && it.tile < atoms_max;
  it.row0 = it.valid ? ws.offsets[it.e] + it.n0 : 0;
  it.valid = it.valid && it.row0 < R_max;
  return it;
}

template <int NT, int STAGES, int FMT, int EPI>
__global__ void __launch_bounds__(256, (NT <= 32 ? 2 : 1)) moe_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                                                          const __grid_constant__ CUtensorMap tmB,
                                                          const uint8_t* __restrict__ sfa,
                                                          const uint8_t* __restrict__ sfb, MoeWorkspace ws,
                                                          const float* __restrict__ bias,
                                                          const float* __restrict__ topk_w,
                                                          __nv_bfloat16* __restrict__ out, int M, int Kp, int ld_out,
                                                          float alpha, float limit, int E_local, int R_max,
                                                          int atoms_max, int* status) {
  pdl_wait();  // predecessor output visible (programmatic dependent launch)
  pdl_trigger();
  using L = GemmSmem<NT, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  const int mtiles = cdiv(M, 128);
  const int W = min(*ws.num_tiles, atoms_max) * mtiles;
  if ((int)blockIdx.x >= W) return;
  // align the shared-space offset (not the generic address) to 1024 for the 128-byte swizzle
  const uint32_t raw_off = tc::smem_addr(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_off & 1023u)) & 1023u);
  uint8_t* sA = smem;
  uint8_t* sB = smem + L::kOffB;
  uint8_t* sSfa = smem + L::kOffSfa;
  uint8_t* sSfb = smem + L::kOffSfb;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  using F = FmtTraits<FMT>;
  const int nk = Kp / F::kKStage;
  const int mblk = mtiles;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      tc::mbar_init(&acc_full[a], 1);
      tc::mbar_init(&acc_empty[a], 4);  // one arrive per epilogue warp
    }
    tc::fence_barrier_init();
    tc::prefetch_tmap(&tmA);
    tc::prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, L::kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int it = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < W && ok; w += gridDim.x) {
        const WorkItem wi = decode_item(ws, w, mtiles, E_local, R_max, atoms_max);
        if (!wi.valid) {
          record(status, kBadIndex, 20, wi.e);
          continue;
        }
        for (int kt = 0; kt < nk; ++kt, ++it) {
          const int s = it % STAGES, use = it / STAGES;
          if (it >= STAGES && !tc::mbar_wait(&empty[s], (use - 1) & 1, status)) {
            ok = false;
            break;
          }
          // transaction bytes count the global (packed) size: fp4 tiles are 4 bits/element
          tc::mbar_arrive_expect_tx(&full[s], (FMT == kFmtFp4 ? L::kA / 2 : L::kA) + L::kB +
                                                  (F::kScaled ? 2 * kSfAtom : 0));
          // weights are stored as contiguous 128-row x 128-byte tiles: tile index (e, m tile, k tile)
          tc::tma_load_3d(sA + s * L::kA, &tmA, 0, 0, ((wi.e * mblk) + wi.mt) * nk + kt, &full[s]);
          tc::tma_load_2d(sB + s * L::kB, &tmB, kt * F::kKStage, wi.row0, &full[s]);
          if constexpr (F::kScaled) {
            tc::bulk_load(sSfa + s * kSfAtom, sfa + (((size_t)wi.e * mblk + wi.mt) * nk + kt) * kSfAtom, kSfAtom,
                          &full[s]);
            tc::bulk_load(sSfb + s * kSfAtom, sfb + ((size_t)wi.tile * nk + kt) * kSfAtom, kSfAtom, &full[s]);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      const uint32_t idesc0 =
          F::kScaled ? tc::idesc_mxf8f6f4(FMT == kFmtFp4 ? 5 : 0, 0, 128, NT) : tc::idesc_f16_bf16(128, NT);
      const uint32_t t_sfa = tmem + 2 * NT, t_sfb = tmem + 2 * NT + 4;
      int it = 0, local = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < W && ok; w += gridDim.x) {
        const WorkItem wi = decode_item(ws, w, mtiles, E_local, R_max, atoms_max);
        if (!wi.valid) continue;
        const int acc = local & 1, ause = local >> 1;
        if (local >= 2 && !tc::mbar_wait(&acc_empty[acc], (ause - 1) & 1, status)) break;
        tc::fence_after_sync();
        const uint32_t t_d = tmem + acc * NT;
        for (int kt = 0; kt < nk; ++kt, ++it) {
          const int s = it % STAGES, use = it / STAGES;
          if (!tc::mbar_wait(&full[s], use & 1, status)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint64_t ad = tc::desc_sw128(sA + s * L::kA);
          const uint64_t bd = tc::desc_sw128(sB + s * L::kB);
          if constexpr (F::kScaled) {
            tc::utccp_32x128b_warpx4(t_sfa, tc::desc_noswizzle_16b_rows(sSfa + s * kSfAtom));
            tc::utccp_32x128b_warpx4(t_sfb, tc::desc_noswizzle_16b_rows(sSfb + s * kSfAtom));
#pragma unroll
            for (int kb = 0; kb < 4; ++kb) {  // 4 x K=32 per 128-byte stage
              tc::mma_mxf8f6f4(t_d, ad + 2 * kb, bd + 2 * kb, tc::idesc_with_sf_ids(idesc0, kb, kb),
                               t_sfa | ((uint32_t)kb << 30), t_sfb | ((uint32_t)kb << 30),
                               (kt | kb) != 0 ? 1u : 0u);
            }
          } else {
#pragma unroll
            for (int kb = 0; kb < 4; ++kb)  // 4 x K=16 bf16 per 128-byte stage
              tc::mma_f16(t_d, ad + 2 * kb, bd + 2 * kb, idesc0, (kt | kb) != 0 ? 1u : 0u);
          }
          tc::mma_commit(&empty[s]);
        }
        tc::mma_commit(&acc_full[acc]);
        ++local;
      }
    }
  } else if (warp >= 4) {
    // ---------------- epilogue ----------------
    const int ew = warp & 3;
    const int m = ew * 32 + lane;
    int local = 0;
    for (int w = blockIdx.x; w < W; w += gridDim.x) {
      const WorkItem wi = decode_item(ws, w, mtiles, E_local, R_max, atoms_max);
      if (!wi.valid) continue;
      const int acc = local & 1, ause = local >> 1;
      if (!tc::mbar_wait(&acc_full[acc], ause & 1, status)) break;
      tc::fence_after_sync();
      const int nvalid = min(NT, ws.offsets[wi.e + 1] - ws.offsets[wi.e] - wi.n0);
      const int gm = wi.mt * 128 + m;
      const float b = gm < M ? bias[(size_t)wi.e * M + gm] : 0.f;
      const uint32_t lane_addr = tmem + acc * NT + ((uint32_t)(ew * 32) << 16);
      uint8_t* stg = smem + L::kOffStage + ew * 1024;  // this warp's staging block
      for (int c = 0; c < NT; c += 16) {
        if (c >= nvalid) break;
        uint32_t r[16];
        tc::tmem_ld_32x32b_x16(lane_addr + c, r);
        tc::tmem_ld_wait();
        __syncwarp();  // the previous chunk's staged rows were copied out
        if constexpr (EPI == kEpiSwiglu) {
          // rows 2i (gate) and 2i+1 (up) sit in lanes m and m^1: the pair splits the 16 tokens,
          // the even lane taking the even ones and the odd lane the odd ones, and swaps the
          // other half of its values with its partner (every lane computes)
          const int odd = m & 1;
#pragma unroll
          for (int i2 = 0; i2 < 8; ++i2) {
            const float keep = __uint_as_float(r[2 * i2 + odd]) + b;
            const float send = __uint_as_float(r[2 * i2 + (odd ^ 1)]) + b;
            const float recv = __shfl_xor_sync(0xffffffffu, send, 1);
            float g = odd ? recv : keep, u = odd ? keep : recv, a;
            if (limit > 0.f) {
              g = fminf(g, limit);
              u = fminf(fmaxf(u, -limit), limit);
              a = __fdividef(g, 1.f + __expf(-alpha * g)) * (u + 1.f);
            } else {
              a = __fdividef(g, 1.f + __expf(-g)) * u;
            }
            // staged [16 tokens][16 features of this warp] bf16, 32 bytes per token
            *reinterpret_cast<__nv_bfloat16*>(stg + (2 * i2 + odd) * 32 + (lane >> 1) * 2) = __float2bfloat16(a);
          }
          __syncwarp();
          const int row = lane >> 1, j = c + row;
          const int f = wi.mt * 64 + ew * 16 + (lane & 1) * 8;  // output feature of this 16-byte segment
          if (j < nvalid && f < (M >> 1))
            *reinterpret_cast<uint4*>(out + (size_t)(wi.row0 + j) * ld_out + f) =
                *reinterpret_cast<const uint4*>(stg + row * 32 + (lane & 1) * 16);
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int j = c + i;
            const float v = __uint_as_float(r[i]) + b;
            const float wt = j < nvalid ? topk_w[ws.row_route[wi.row0 + j]] : 0.f;
            // staged [16 routes][32 features of this warp] bf16, 64 bytes per route
            *reinterpret_cast<__nv_bfloat16*>(stg + i * 64 + lane * 2) = __float2bfloat16(v * wt);
          }
          __syncwarp();
#pragma unroll
          for (int k2 = 0; k2 < 2; ++k2) {
            const int q = lane + 32 * k2, row = q >> 2, ch = q & 3, j = c + row;
            const int f = wi.mt * 128 + ew * 32 + ch * 8;
            if (j < nvalid && f < M) {
              const int route = ws.row_route[wi.row0 + j];
              *reinterpret_cast<uint4*>(out + (size_t)route * ld_out + f) =
                  *reinterpret_cast<const uint4*>(stg + row * 64 + ch * 16);
            }
          }
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&acc_empty[acc]);
      ++local;
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) tc::tmem_dealloc(tmem, L::kTmemCols);
}

// ------------------------------------------------------------------------- reduce
__global__ void moe_reduce_kernel(__nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ y,
                                  const int* __restrict__ topk_ids, int k, int E, int off, int H) {
  pdl_wait();  // predecessor output visible (programmatic dependent launch)
  pdl_trigger();
  const int t = blockIdx.x;
  int local[16];
  int nl = 0;
  for (int j = 0; j < k && j < 16; ++j) {
    const int e = topk_ids[t * k + j] - off;
    if (e >= 0 && e < E) local[nl++] = j;
  }
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int i = 0; i < nl; ++i) {
      const uint4 u = reinterpret_cast<const uint4*>(y + (size_t)(t * k + local[i]) * H)[c];
      const __nv_bfloat16* hb = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] += __bfloat162float(hb[q]);
    }
    uint4 o;
    __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
    for (int q = 0; q < 8; ++q) ob[q] = __float2bfloat16(acc[q]);
    reinterpret_cast<uint4*>(out + (size_t)t * H)[c] = o;
  }
}

// ------------------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
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

// Weight map over contiguous 128-row x 128-element tiles [n_tiles, 128, 128*bits/8]:
// one box = one tile = one contiguous 8 KB (fp4) / 16 KB (fp8) run.
static int make_weight_map(CUtensorMap* m, const void* w, int n_tiles, int fmt) {
  auto enc = get_encode();
  if (!enc) return kBadShape;
  const bool fp4 = fmt == kFmtFp4, b16 = fmt == kFmtBf16;
  const uint64_t row_bytes = fp4 ? 64 : 128;
  const cuuint64_t row_elems = b16 ? 64 : 128;
  cuuint64_t dims[3] = {row_elems, 128, (cuuint64_t)n_tiles};
  cuuint64_t strides[2] = {row_bytes, row_bytes * 128};
  cuuint32_t box[3] = {(cuuint32_t)row_elems, 128, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = enc(m, fp4 ? CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B
                          : (b16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8), 3,
                   const_cast<void*>(w), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : kTensorMapErrorBase + (int)r;
}

// 2-D bf16 activation map: K valid columns (TMA zero-fills beyond), row stride ld elements,
// box 64 x NT.
static int make_act_map_bf16(CUtensorMap* m, const void* a, int R, int K, int ld, int nt) {
  auto enc = get_encode();
  if (!enc) return kBadShape;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)R};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)nt};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(a), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : kTensorMapErrorBase + (int)r;
}

// 2-D activation map [R, Kp] e4m3, box 128 x NT.
static int make_act_map(CUtensorMap* m, const void* q, int R, int Kp, int nt) {
  auto enc = get_encode();
  if (!enc) return kBadShape;
  cuuint64_t dims[2] = {(cuuint64_t)Kp, (cuuint64_t)R};
  cuuint64_t strides[1] = {(cuuint64_t)Kp};
  cuuint32_t box[2] = {128, (cuuint32_t)nt};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(q), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : kTensorMapErrorBase + (int)r;
}

static int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <int NT, int STAGES, int FMT, int EPI>
static int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const uint8_t* sfa, const uint8_t* sfb,
                       const MoeWorkspace& ws, const float* bias, const float* topk_w, void* out, int M, int Kp,
                       int ld_out, float alpha, float limit, int max_tiles, int E_local, int R_max, int atoms_max,
                       int* status, cudaStream_t s) {
  using L = GemmSmem<NT, STAGES>;
  // the epilogue writes 16-byte segments of 8 features
  if (M % 16 || ld_out % 8 || (reinterpret_cast<uintptr_t>(out) & 15)) return kBadShape;
  auto kern = moe_gemm_kernel<NT, STAGES, FMT, EPI>;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
    attr = true;
  }
  // persistent: one (large tiles) or two (small tiles) CTAs per SM, never more than the
  // work items
  const int work = max_tiles * cdiv(M, 128);
  const int grid = min(num_sms() * (NT <= 32 ? 2 : 1), work);
  launch_k(kern, dim3(grid), dim3(256), L::kAlloc, s, ta, tb, sfa, sfb, ws, bias, topk_w, (__nv_bfloat16*)out, M, Kp, ld_out, alpha,
                                    limit, E_local, R_max, atoms_max, status);
  return (int)cudaGetLastError();
}

template <int NT, int STAGES, bool A_FP4>
static int run_gemms(const MoeShape& sh, const void* w13, const uint8_t* sf13, const float* b13, const void* w2,
                     const uint8_t* sf2w, const float* b2, const float* topk_w, const MoeWorkspace& ws, float alpha,
                     float limit, int R_max, int max_tiles, int atoms_max, int* status, cudaStream_t s) {
  CUtensorMap ta1, tb1, ta2, tb2;
  int rc;
  constexpr int FMT = A_FP4 ? kFmtFp4 : kFmtFp8;
  if ((rc = make_weight_map(&ta1, w13, sh.E_local * cdiv(2 * sh.I, 128) * (sh.K1p / 128), FMT))) return rc;
  if ((rc = make_act_map(&tb1, ws.xq, R_max, sh.K1p, NT))) return rc;
  if ((rc = make_weight_map(&ta2, w2, sh.E_local * cdiv(sh.H, 128) * (sh.K2p / 128), FMT))) return rc;
  if ((rc = make_act_map(&tb2, ws.aq, R_max, sh.K2p, NT))) return rc;
  rc = launch_gemm<NT, STAGES, FMT, kEpiSwiglu>(ta1, tb1, sf13, ws.sf1, ws, b13, topk_w, ws.act, 2 * sh.I,
                                                  sh.K1p, sh.I, alpha, limit, max_tiles, sh.E_local, R_max, atoms_max,
                                                  status, s);
  if (rc) return rc;
  launch_k(moe_quant_kernel, dim3(cdiv(R_max * cdiv(sh.K2p / 32, 32), 4)), dim3(128), 0, s, ws.aq, ws.sf2, (const __nv_bfloat16*)ws.act, sh.I, ws.row_route,
                                                  0, ws.offsets, ws.atom_base, sh.E_local, sh.I, sh.K2p, R_max, R_max,
                                                  atoms_max, NT, status);
  rc = launch_gemm<NT, STAGES, FMT, kEpiDown>(ta2, tb2, sf2w, ws.sf2, ws, b2, topk_w, ws.y, sh.H, sh.K2p, sh.H,
                                              alpha, limit, max_tiles, sh.E_local, R_max, atoms_max, status, s);
  return rc;
}

// bf16 experts: gathered bf16 rows -> GEMM1 (kind::f16) -> SwiGLU (bf16, row stride K2p) ->
// GEMM2 reading the activations directly.  K1p / K2p are H / I rounded up to 64.
template <int NT, int STAGES>
static int run_gemms_bf16(const MoeShape& sh, const void* w13, const float* b13, const void* w2, const float* b2,
                          const float* topk_w, const MoeWorkspace& ws, float alpha, float limit, int R_max,
                          int max_tiles, int atoms_max, int* status, cudaStream_t s) {
  CUtensorMap ta1, tb1, ta2, tb2;
  int rc;
  if ((rc = make_weight_map(&ta1, w13, sh.E_local * cdiv(2 * sh.I, 128) * (sh.K1p / 64), kFmtBf16))) return rc;
  if ((rc = make_act_map_bf16(&tb1, ws.xq, R_max, sh.H, sh.K1p, NT))) return rc;
  if ((rc = make_weight_map(&ta2, w2, sh.E_local * cdiv(sh.H, 128) * (sh.K2p / 64), kFmtBf16))) return rc;
  if ((rc = make_act_map_bf16(&tb2, ws.act, R_max, sh.I, sh.K2p, NT))) return rc;
  rc = launch_gemm<NT, STAGES, kFmtBf16, kEpiSwiglu>(ta1, tb1, nullptr, nullptr, ws, b13, topk_w, ws.act, 2 * sh.I,
                                                     sh.K1p, sh.K2p, alpha, limit, max_tiles, sh.E_local, R_max,
                                                     atoms_max, status, s);
  if (rc) return rc;
  return launch_gemm<NT, STAGES, kFmtBf16, kEpiDown>(ta2, tb2, nullptr, nullptr, ws, b2, topk_w, ws.y, sh.H, sh.K2p,
                                                     sh.H, alpha, limit, max_tiles, sh.E_local, R_max, atoms_max,
                                                     status, s);
}

}  // namespace b200

using namespace b200;

static void ws_sizes(const MoeShape& sh, int64_t* z) {
  const int64_t R = (int64_t)sh.T * sh.k;
  const int64_t max_tiles = cdiv((int)R, sh.nt) + sh.E_local;
  const int64_t atoms = max_tiles;  // one scale atom per N tile
  z[0] = (sh.E_local + 1) * 4;
  z[1] = (sh.E_local + 1) * 4;
  z[2] = sh.E_local * 4;
  z[3] = R * 4;
  z[4] = max_tiles * 2 * 4;
  z[5] = 4;
  const int64_t eb = sh.a_fp4 == 2 ? 2 : 1;  // bf16 experts keep bf16 activations
  z[6] = R * sh.K1p * eb;
  z[7] = atoms * (sh.K1p / 128) * kSfAtom;
  z[8] = R * (sh.a_fp4 == 2 ? sh.K2p : sh.I) * 2;
  z[9] = R * sh.K2p;
  z[10] = atoms * (sh.K2p / 128) * kSfAtom;
  z[11] = R * sh.H * 2;
}

extern "C" void b200_moe_workspace_sizes(const MoeShape* shape, int64_t* sizes) { ws_sizes(*shape, sizes); }

extern "C" int b200_moe_mx_forward(void* out, const void* x, const int* topk_ids, const float* topk_w,
                                   const void* w13, const uint8_t* sf13, const float* b13, const void* w2,
                                   const uint8_t* sf2w, const float* b2, const MoeShape* shape, float alpha,
                                   float limit, const MoeWorkspace* wsp, int* status, cudaStream_t s) {
  const MoeShape& sh = *shape;
  const MoeWorkspace& ws = *wsp;
  if (sh.T == 0) return 0;
  if (sh.K1p % 128 || sh.K2p % 128 || sh.H % 32 || sh.I % 32 || sh.E_local > 1024 || sh.k > 16) return kBadShape;
  if (sh.nt != 16 && sh.nt != 32 && sh.nt != 128) return kBadShape;
  const int R_max = sh.T * sh.k;
  const int max_tiles = cdiv(R_max, sh.nt) + sh.E_local;
  launch_k(moe_route_kernel, dim3(1), dim3(1024), 2 * sh.E_local * sizeof(int), s, topk_ids, R_max, sh.E_local,
                                                                          sh.expert_offset, sh.nt, max_tiles, ws);
  const int atoms_max = max_tiles;
  launch_k(moe_quant_kernel, dim3(cdiv(R_max * cdiv(sh.K1p / 32, 32), 4)), dim3(128), 0, s, ws.xq, ws.sf1, (const __nv_bfloat16*)x, sh.H, ws.row_route,
                                                  sh.k, ws.offsets, ws.atom_base, sh.E_local, sh.H, sh.K1p, R_max,
                                                  sh.T, atoms_max, sh.nt, status);
  int rc;
  if (sh.nt == 16) {
    rc = sh.a_fp4 ? run_gemms<16, 5, true>(sh, w13, sf13, b13, w2, sf2w, b2, topk_w, ws, alpha, limit, R_max,
                                           max_tiles, atoms_max, status, s)
                  : run_gemms<16, 5, false>(sh, w13, sf13, b13, w2, sf2w, b2, topk_w, ws, alpha, limit, R_max,
                                            max_tiles, atoms_max, status, s);
  } else if (sh.nt == 32) {
    rc = sh.a_fp4 ? run_gemms<32, 5, true>(sh, w13, sf13, b13, w2, sf2w, b2, topk_w, ws, alpha, limit, R_max,
                                           max_tiles, atoms_max, status, s)
                  : run_gemms<32, 5, false>(sh, w13, sf13, b13, w2, sf2w, b2, topk_w, ws, alpha, limit, R_max,
                                            max_tiles, atoms_max, status, s);
  } else {
    rc = sh.a_fp4 ? run_gemms<128, 6, true>(sh, w13, sf13, b13, w2, sf2w, b2, topk_w, ws, alpha, limit, R_max,
                                            max_tiles, atoms_max, status, s)
                  : run_gemms<128, 6, false>(sh, w13, sf13, b13, w2, sf2w, b2, topk_w, ws, alpha, limit, R_max,
                                             max_tiles, atoms_max, status, s);
  }
  if (rc) return rc;
  if (out == nullptr) return (int)cudaGetLastError();  // the caller reduces the per-route rows of ws.y
  launch_k(moe_reduce_kernel, dim3(sh.T), dim3(128), 0, s, (__nv_bfloat16*)out, (const __nv_bfloat16*)ws.y, topk_ids, sh.k,
                                         sh.E_local, sh.expert_offset, sh.H);
  return (int)cudaGetLastError();
}

extern "C" int b200_moe_bf16_forward(void* out, const void* x, const int* topk_ids, const float* topk_w,
                                     const void* w13, const float* b13, const void* w2, const float* b2,
                                     const MoeShape* shape, float alpha, float limit, const MoeWorkspace* wsp,
                                     int* status, cudaStream_t s) {
  const MoeShape& sh = *shape;
  const MoeWorkspace& ws = *wsp;
  if (sh.T == 0) return 0;
  if (sh.K1p % 64 || sh.K2p % 64 || sh.H % 8 || sh.I % 8 || sh.E_local > 1024 || sh.k > 16) return kBadShape;
  if (sh.nt != 16 && sh.nt != 32 && sh.nt != 128) return kBadShape;
  const int R_max = sh.T * sh.k;
  const int max_tiles = cdiv(R_max, sh.nt) + sh.E_local;
  launch_k(moe_route_kernel, dim3(1), dim3(1024), 2 * sh.E_local * sizeof(int), s, topk_ids, R_max, sh.E_local, sh.expert_offset,
                                                                  sh.nt, max_tiles, ws);
  launch_k(moe_gather_kernel, dim3(cdiv(R_max, 4)), dim3(128), 0, s, (__nv_bfloat16*)ws.xq, sh.K1p, (const __nv_bfloat16*)x, sh.H,
                                                   ws.row_route, sh.k, ws.offsets, sh.E_local, sh.H, R_max, sh.T,
                                                   status);
  int rc;
  if (sh.nt == 16)
    rc = run_gemms_bf16<16, 5>(sh, w13, b13, w2, b2, topk_w, ws, alpha, limit, R_max, max_tiles, max_tiles, status,
                               s);
  else if (sh.nt == 32)
    rc = run_gemms_bf16<32, 5>(sh, w13, b13, w2, b2, topk_w, ws, alpha, limit, R_max, max_tiles, max_tiles, status,
                               s);
  else
    rc = run_gemms_bf16<128, 6>(sh, w13, b13, w2, b2, topk_w, ws, alpha, limit, R_max, max_tiles, max_tiles, status,
                                s);
  if (rc) return rc;
  launch_k(moe_reduce_kernel, dim3(sh.T), dim3(128), 0, s, (__nv_bfloat16*)out, (const __nv_bfloat16*)ws.y, topk_ids, sh.k,
                                         sh.E_local, sh.expert_offset, sh.H);
  return (int)cudaGetLastError();
}

// out[t] = sum of y[t * k + j] over the slots j routed to experts [off, off + E) (the reduction
// a caller defers when it fuses it into the layer-boundary all-reduce and cannot here).
extern "C" int b200_moe_route_sum(void* out, const void* y, const int* topk_ids, int T, int k, int E, int off, int H,
                                  cudaStream_t s) {
  if (k > 16 || H % 8) return kBadShape;
  if (T == 0) return 0;
  launch_k(moe_reduce_kernel, dim3(T), dim3(128), 0, s, (__nv_bfloat16*)out, (const __nv_bfloat16*)y, topk_ids, k, E,
           off, H);
  return (int)cudaGetLastError();
}
