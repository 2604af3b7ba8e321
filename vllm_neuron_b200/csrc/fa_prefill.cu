// Prefill / chunked-prefill attention over the paged KV cache on the Blackwell tensor cores
// (tcgen05 + TMEM + TMA), head dim 64, bf16 Q / K / V.
//
// Semantics (the reference's flash_attention / segmented_attention, functional/attention/
// attention_cte.py:188 and attention_segmented_cte.py:472, fallbacks :46 and :103): the
// queries of each sequence are its last qlen positions; query p sees cached keys j with
// j <= p (causal) and, with a sliding window W, j > p - W; per-head sink logits join the
// softmax denominator only (attention_cte.py:163-173).
//
// Design: a persistent kernel, one CTA per SM, 12 warps.  A work item is 256 queries (two
// query tiles A and B of 128) x one query head x one sequence; items are visited in
// decreasing query-tile order so the longest causal rows start first.
//   warp 0     TMA producer: the item's two Q tiles (one box each from the [tokens, q_stride]
//              query rows) and the K and V tiles of 128 keys straight from the paged cache
//              (one box of block_size rows per cache block, 128-byte swizzle, no multicast)
//              into a three-stage ring that runs across items;
//   warp 1     allocates TMEM once and issues the MMAs from one thread:
//                S_X(j) = Q_X K(j)^T  (M=128 queries, N=128 keys, K=64, fp32 in TMEM),
//                O_X += P_X(j) V(j)   (M=128, N=64, K=128 keys; P from shared memory, V read
//                                      in its cache layout as an MN-major operand),
//              for X = A, B in the order PV_A(j-1), S_A(j), PV_B(j-1), S_B(j): while one
//              softmax warpgroup works on its tile the tensor core serves the other;
//   warps 4-7  softmax of tile A, warps 8-11 softmax of tile B, one thread per query row
//              (its TMEM lane): the whole S row in one TMEM round trip, masks only on tiles
//              that cross the row's visible range, P = exp2(s - m) as bf16 into 128-byte-
//              swizzled shared memory.  O stays in TMEM; it is rescaled (TMEM load, multiply,
//              store) only when a row's maximum grows by more than 8 in log2 units, so P
//              stays <= 2^8 in between (the lazy rescaling of FlashAttention-4).  At the end
//              of an item the O rows are normalised with the row sum and the sink and stored.
// Ordering facts used: tcgen05 MMAs from one thread complete in issue order and a commit
// covers all earlier MMAs, so when S_X(j) is complete PV_X(j-1) is too: the softmax may then
// rewrite P_X and rescale O_X.  Every wait is bounded and records kWaitTimeout in the
// status word; on a timeout each role stops and the CTA still frees its TMEM.
#include <cuda.h>
#include <cuda_bf16.h>

#include "common.cuh"
#include "launch.h"
#include "launch_pdl.h"
#include "tcgen05.cuh"

namespace b200 {
namespace fa {

constexpr int kBQ = 128;     // queries per tile
constexpr int kQT = 2;       // query tiles per work item
constexpr int kBK = 128;     // keys per tile
constexpr int kD = 64;       // head dim (one 128-byte swizzle row of bf16)
constexpr int kStages = 3;   // K/V ring
constexpr int kThreads = 384;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.f;  // rescale O when a row maximum grows by more than this

// shared memory (bytes from a 1024-aligned base)
constexpr int kTileBytes = kBK * kD * 2;           // one 128 x 64 bf16 tile (16 KB)
constexpr int kOffQ = 0;                           // kQT x [128 q][64], K-major SW128
constexpr int kOffK = kOffQ + kQT * kTileBytes;    // kStages x [128 keys][64]
constexpr int kOffV = kOffK + kStages * kTileBytes;
constexpr int kOffP = kOffV + kStages * kTileBytes;  // kQT x [128 q][128 keys]: two 64-key atoms each
constexpr int kPBuf = kBQ * kBK * 2;
constexpr int kOffBar = kOffP + kQT * kPBuf;
constexpr int kNumBars = 2 * kStages + 2 + 6 * kQT;
constexpr int kSmem = kOffBar + kNumBars * 8 + 16 + 1024;
static_assert(kSmem <= 232448, "shared memory");
constexpr uint32_t kTmemCols = 512;  // S_A, S_B: 128 columns each; O_A, O_B: 64 each
constexpr int kColO = kQT * kBK;

struct Args {
  __nv_bfloat16* out;        // [T, nq, 64]
  const int* block_tables;   // [B, max_blocks]
  const int* seq_lens;       // [B] keys in the cache after this step
  const int* qsl;            // [B + 1] query start locations
  const float* sinks;        // [nq] or null
  int B, nq, nkv, bs, max_blocks, window, causal;
  int n_qt;                  // 256-query tiles of the longest query run
  int num_items;             // n_qt * B * nq
  float scale_log2;          // softmax scale * log2(e)
  float v_scale;
  int* status;
};

// Byte offset of 16-byte chunk c of row r inside a [rows][128 B] tile in the 128-byte
// swizzle layout the tensor cores read (8-row groups of 1024 bytes, chunk index XOR row).
B200_D uint32_t sw128(int r, int c) { return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4)); }

// 2^x on the multi-function unit (the hardware approximation; x = -inf gives +0)
B200_D float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// three-input maximum (one instruction)
B200_D float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// (r0, r1) = (x0, x1) * s + (o, o) on the packed f32x2 pipe (one instruction for two lanes' worth)
B200_D void ffma2(float& r0, float& r1, float x0, float x1, float s, float o) {
  asm("{\n .reg .b64 a, b, c;\n mov.b64 a, {%2, %3};\n mov.b64 b, {%4, %4};\n mov.b64 c, {%5, %5};\n"
      " fma.rn.f32x2 a, a, b, c;\n mov.b64 {%0, %1}, a;\n}"
      : "=f"(r0), "=f"(r1)
      : "f"(x0), "f"(x1), "f"(s), "f"(o));
}

// (a0, a1) += (b0, b1) on the packed f32x2 pipe
B200_D void fadd2(float& a0, float& a1, float b0, float b1) {
  asm("{\n .reg .b64 a, b;\n mov.b64 a, {%0, %1};\n mov.b64 b, {%2, %3};\n add.rn.f32x2 a, a, b;\n"
      " mov.b64 {%0, %1}, a;\n}"
      : "+f"(a0), "+f"(a1)
      : "f"(b0), "f"(b1));
}

B200_D void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// kind::f16 bf16 x bf16 -> fp32, B MN-major (V in its row-per-key layout)
B200_HD uint32_t idesc_bf16_bmn(int M, int N) { return tc::idesc_f16_bf16(M, N) | (1u << 16); }

// One work item's geometry, computed identically by every role.
struct Item {
  int b, qt, head, h;  // sequence, 256-query tile, query head, kv head
  int q0, qlen, L;     // first query row of the sequence, its query count, keys after this step
  int key_lo, n;       // first key of the first KV tile (128-aligned), KV tiles
};

B200_D bool item_at(const Args& a, int k, Item& it) {
  const int per = a.B * a.nq;
  const int qt = a.n_qt - 1 - k / per;  // longest rows first
  const int rem = k % per;
  it.b = rem / a.nq;
  it.head = rem % a.nq;
  it.qt = qt;
  it.q0 = a.qsl[it.b];
  it.qlen = a.qsl[it.b + 1] - it.q0;
  if (qt * kQT * kBQ >= it.qlen) return false;
  it.L = a.seq_lens[it.b];
  it.h = it.head / (a.nq / a.nkv);
  const int pos_base = it.L - it.qlen;
  const int p_first = pos_base + qt * kQT * kBQ;
  const int p_last = pos_base + min(it.qlen, (qt + 1) * kQT * kBQ) - 1;
  int lo = a.window > 0 ? max(0, p_first - a.window + 1) : 0;
  it.key_lo = (lo / kBK) * kBK;
  const int hi = a.causal ? min(it.L, p_last + 1) : it.L;
  it.n = hi > it.key_lo ? (hi - it.key_lo + kBK - 1) / kBK : 0;
  return true;
}

__global__ void __launch_bounds__(kThreads, 1) fa_prefill_kernel(const __grid_constant__ CUtensorMap tmQ,
                                                                 const __grid_constant__ CUtensorMap tmK,
                                                                 const __grid_constant__ CUtensorMap tmV, Args a) {
  pdl_wait();  // predecessor output visible (programmatic dependent launch)
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_off = tc::smem_addr(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_off & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* kv_full = bars;                // [kStages] K and V of a tile landed (TMA transaction count)
  uint64_t* kv_empty = bars + kStages;     // [kStages] every MMA reading the stage is done
  uint64_t* q_full = bars + 2 * kStages;   // the item's Q tiles landed
  uint64_t* q_empty = q_full + 1;          // every S MMA of the item is done (Q may be replaced)
  uint64_t* s_full = q_empty + 1;          // [kQT] S_X(j) is in TMEM
  uint64_t* s_free = s_full + kQT;         // [kQT] the softmax has read S_X(j) into registers
  uint64_t* p_full = s_free + kQT;         // [kQT] P_X(j) is in shared memory, O_X rescaled
  uint64_t* pv_done = p_full + kQT;        // [kQT] PV_X(j) is complete (P_X free, O_X current)
  uint64_t* o_done = pv_done + kQT;        // [kQT] the item's last PV_X is complete
  uint64_t* o_free = o_done + kQT;         // [kQT] the item's O_X was read out
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      tc::mbar_init(&kv_full[i], 1);
      tc::mbar_init(&kv_empty[i], 1);
    }
    tc::mbar_init(q_full, 1);
    tc::mbar_init(q_empty, 1);
    for (int x = 0; x < kQT; ++x) {
      tc::mbar_init(&s_full[x], 1);
      tc::mbar_init(&s_free[x], 4);  // one arrive per softmax warp
      tc::mbar_init(&p_full[x], 4);
      tc::mbar_init(&pv_done[x], 1);
      tc::mbar_init(&o_done[x], 1);
      tc::mbar_init(&o_free[x], 4);
    }
    tc::fence_barrier_init();
    tc::prefetch_tmap(&tmQ);
    tc::prefetch_tmap(&tmK);
    tc::prefetch_tmap(&tmV);
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int g = 0;        // K/V tiles issued (ring position, across items)
      int items = 0;    // items started
      bool ok = true;
      for (int k = blockIdx.x; k < a.num_items && ok; k += gridDim.x) {
        Item it;
        if (!item_at(a, k, it) || it.n == 0) continue;
        // Q of this item once every S MMA of the previous item is done
        if (items > 0 && !tc::mbar_wait(q_empty, (items - 1) & 1, a.status)) break;
        tc::mbar_arrive_expect_tx(q_full, kQT * kTileBytes);
        for (int x = 0; x < kQT; ++x)
          tc::tma_load_2d(smem + kOffQ + x * kTileBytes, &tmQ, it.head * kD, it.q0 + (it.qt * kQT + x) * kBQ, q_full);
        ++items;
        const int* bt = a.block_tables + (size_t)it.b * a.max_blocks;
        const int nblk_seq = (it.L + a.bs - 1) / a.bs;
        const int per_tile = kBK / a.bs;
        for (int j = 0; j < it.n; ++j, ++g) {
          const int s = g % kStages;
          if (g >= kStages && !tc::mbar_wait(&kv_empty[s], ((g / kStages) - 1) & 1, a.status)) {
            ok = false;
            break;
          }
          tc::mbar_arrive_expect_tx(&kv_full[s], 2 * kTileBytes);
          const int blk0 = (it.key_lo + j * kBK) / a.bs;
          for (int i = 0; i < per_tile; ++i) {
            const int blk = blk0 + i;
            const int bid = blk < nblk_seq ? bt[blk] : 0;  // past the sequence: the null block (masked)
            const int row = (bid * a.nkv + it.h) * a.bs;
            tc::tma_load_2d(smem + kOffK + s * kTileBytes + i * a.bs * 128, &tmK, 0, row, &kv_full[s]);
            tc::tma_load_2d(smem + kOffV + s * kTileBytes + i * a.bs * 128, &tmV, 0, row, &kv_full[s]);
          }
        }
      }
      // no copy may still be landing when the CTA ends: wait (bounded) for the last stages
      for (int t = max(0, g - kStages); t < g; ++t) tc::mbar_wait(&kv_full[t % kStages], (t / kStages) & 1, a.status);
      if (items > 0) tc::mbar_wait(q_full, (items - 1) & 1, a.status);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      const uint32_t id_s = tc::idesc_f16_bf16(kBQ, kBK);
      const uint32_t id_o = idesc_bf16_bmn(kBQ, kD);
      int g = 0;      // K/V tiles consumed
      int c = 0;      // per-query-tile S/P steps (the same count for A and B)
      int items = 0;
      bool ok = true;
      auto pv = [&](int x, int stage, bool acc) {
        const uint8_t* pt = smem + kOffP + x * kPBuf;
        const uint8_t* vt = smem + kOffV + stage * kTileBytes;
#pragma unroll
        for (int ks = 0; ks < kBK / 16; ++ks)  // 16 keys per step: P along K, V rows
          tc::mma_f16(tmem + kColO + x * kD, tc::desc_sw128(pt + (ks >> 2) * (kBQ * 128) + (ks & 3) * 32),
                      tc::desc_sw128(vt + ks * 2048), id_o, (acc || ks > 0) ? 1u : 0u);
      };
      auto s_mma = [&](int x, int stage) {  // S_X = Q_X K^T
        const uint8_t* kt = smem + kOffK + stage * kTileBytes;
        const uint8_t* qx = smem + kOffQ + x * kTileBytes;
#pragma unroll
        for (int ks = 0; ks < kD / 16; ++ks)
          tc::mma_f16(tmem + x * kBK, tc::desc_sw128(qx + ks * 32), tc::desc_sw128(kt + ks * 32), id_s,
                      ks > 0 ? 1u : 0u);
        tc::mma_commit(&s_full[x]);
      };
      // Order per key tile j: S_X(j+1) as soon as the softmax has read S_X(j) (it then overlaps
      // that softmax's exponentials), PV_X(j) once P_X(j) is written.
      for (int k = blockIdx.x; k < a.num_items && ok; k += gridDim.x) {
        Item it;
        if (!item_at(a, k, it) || it.n == 0) continue;
        if (!tc::mbar_wait(q_full, items & 1, a.status)) break;
        if (!tc::mbar_wait(&kv_full[g % kStages], (g / kStages) & 1, a.status)) break;
        tc::fence_after_sync();
        for (int x = 0; x < kQT; ++x) s_mma(x, g % kStages);
        if (it.n == 1) tc::mma_commit(q_empty);
        for (int j = 0; j < it.n && ok; ++j) {
          const int s = (g + j) % kStages, sn = (g + j + 1) % kStages;
          const bool more = j + 1 < it.n;
          if (more && !tc::mbar_wait(&kv_full[sn], ((g + j + 1) / kStages) & 1, a.status)) {
            ok = false;
            break;
          }
          for (int x = 0; x < kQT && ok && more; ++x) {
            if (!tc::mbar_wait(&s_free[x], (c + j) & 1, a.status)) {
              ok = false;
              break;
            }
            tc::fence_after_sync();
            s_mma(x, sn);
          }
          if (!ok) break;
          if (j + 1 == it.n - 1) tc::mma_commit(q_empty);  // every S MMA of the item issued
          for (int x = 0; x < kQT; ++x) {
            if (!tc::mbar_wait(&p_full[x], (c + j) & 1, a.status)) {
              ok = false;
              break;
            }
            // the first PV of an item overwrites O_X: the previous item's O_X must be read out
            if (j == 0 && items > 0 && !tc::mbar_wait(&o_free[x], (items - 1) & 1, a.status)) {
              ok = false;
              break;
            }
            tc::fence_after_sync();
            pv(x, s, j > 0);
            tc::mma_commit(&pv_done[x]);
            if (j == it.n - 1) tc::mma_commit(&o_done[x]);
          }
          if (!ok) break;
          tc::mma_commit(&kv_empty[s]);  // S(j) and PV(j) of both tiles issued
        }
        g += it.n;
        c += it.n;
        ++items;
      }
      // the CTA may end (and free TMEM) only after the last MMAs: wait for a final commit
      if (items > 0) {
        tc::mma_commit(q_empty);
        tc::mbar_wait(q_empty, items & 1, a.status);
      }
    }
  } else if (warp >= 4) {
    // ---------------- softmax: warpgroup x = query tile, thread = query row (TMEM lane) ----------------
    const int x = (warp - 4) >> 2;
    const int ew = warp & 3;
    const int r = ew * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(ew * 32) << 16);
    const uint32_t s_addr = lane_base + x * kBK;
    const uint32_t o_addr = lane_base + kColO + x * kD;
    uint8_t* pbuf = smem + kOffP + x * kPBuf;
    int c = 0, items = 0;
    bool ok = true;
    for (int k = blockIdx.x; k < a.num_items && ok; k += gridDim.x) {
      Item it;
      if (!item_at(a, k, it) || it.n == 0) continue;
      const int qrow = (it.qt * kQT + x) * kBQ + r;  // this row's query index in the sequence
      const int p = it.L - it.qlen + qrow;            // its position
      const int lo_vis = a.window > 0 ? p - a.window + 1 : 0;
      const int hi_vis = a.causal ? min(p, it.L - 1) : it.L - 1;
      float m = -INFINITY, l = 0.f;
      // PV_X of the previous key tile (phase c - 1) must be complete before P_X is rewritten
      // or O_X rescaled; it was issued after this warpgroup's previous p_full arrive
      auto wait_pv = [&](int cc_) -> bool {
        if (!tc::mbar_wait(&pv_done[x], (cc_ - 1) & 1, a.status)) return false;
        tc::fence_after_sync();
        return true;
      };
      for (int j = 0; j < it.n; ++j, ++c) {
        if (!tc::mbar_wait(&s_full[x], c & 1, a.status)) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        const int key0 = it.key_lo + j * kBK;
        // a tile no row of this warp can see (the other query tile's diagonal or window edge):
        // P = 0 without reading S; the row statistics are unchanged
        if (__all_sync(0xffffffffu, key0 > hi_vis || key0 + kBK - 1 < lo_vis)) {
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&s_free[x]);
          if (j > 0 && !wait_pv(c)) {
            ok = false;
            break;
          }
#pragma unroll
          for (int ch = 0; ch < 16; ++ch)
            *reinterpret_cast<uint4*>(pbuf + (ch >> 3) * (kBQ * 128) + sw128(r, ch & 7)) = make_uint4(0, 0, 0, 0);
          fence_async_smem();
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&p_full[x]);
          continue;
        }
        float sv[kBK];
#pragma unroll
        for (int cc = 0; cc < kBK; cc += 32)
          tc::tmem_ld_32x32b_x32(s_addr + cc, *reinterpret_cast<uint32_t(*)[32]>(sv + cc));
        tc::tmem_ld_wait();
        // S_X is in registers: the tensor core may compute the next tile's S_X meanwhile
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&s_free[x]);
        if (key0 < lo_vis || key0 + kBK - 1 > hi_vis) {  // the tile crosses this row's visible range
#pragma unroll
          for (int t = 0; t < kBK; ++t) {
            const int kk = key0 + t;
            if (kk < lo_vis || kk > hi_vis) sv[t] = -INFINITY;
          }
        }
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int t = 0; t < kBK; t += 8) {  // four independent chains of three-input maxima
          mx[0] = max3(mx[0], sv[t], sv[t + 1]);
          mx[1] = max3(mx[1], sv[t + 2], sv[t + 3]);
          mx[2] = max3(mx[2], sv[t + 4], sv[t + 5]);
          mx[3] = max3(mx[3], sv[t + 6], sv[t + 7]);
        }
        const float tmax = max3(mx[0], mx[1], fmaxf(mx[2], mx[3])) * a.scale_log2;
        // lazy rescaling: move the reference maximum only when the row maximum grew by > 2^8
        const bool grow = tmax > m + kRescaleLog2 || (m == -INFINITY && tmax > -INFINITY);
        const float m_new = grow ? tmax : m;
        const float corr = grow ? ex2(m - m_new) : 1.f;  // m = -inf gives 0
        const float mref = m_new == -INFINITY ? 0.f : m_new;  // a fully masked row so far: P = 0
        // P of the whole row into registers (bf16 pairs), overlapping PV_X(j-1) on the tensor core
        float rs[4] = {0.f, 0.f, 0.f, 0.f};  // two packed (f32x2) row-sum chains
        uint32_t pk[kBK / 2];
#pragma unroll
        for (int t = 0; t < kBK; t += 2) {
          float x0, x1;
          ffma2(x0, x1, sv[t], sv[t + 1], a.scale_log2, -mref);
          const float e0 = ex2(x0);
          const float e1 = ex2(x1);
          if ((t >> 1) & 1)
            fadd2(rs[2], rs[3], e0, e1);
          else
            fadd2(rs[0], rs[1], e0, e1);
          const __nv_bfloat162 pr = __floats2bfloat162_rn(e0, e1);
          pk[t >> 1] = *reinterpret_cast<const uint32_t*>(&pr);
        }
        if (j > 0) {
          if (!wait_pv(c)) {
            ok = false;
            break;
          }
          if (__any_sync(0xffffffffu, grow)) {
            // O_X holds PV through j-1 (complete): rescale it before PV_X(j) accumulates
#pragma unroll
            for (int cc = 0; cc < kD; cc += 16) {
              uint32_t ov[16];
              tc::tmem_ld_32x32b_x16(o_addr + cc, ov);
              tc::tmem_ld_wait();
#pragma unroll
              for (int t = 0; t < 16; ++t) ov[t] = __float_as_uint(__uint_as_float(ov[t]) * corr);
              tc::tmem_st_32x32b_x16(o_addr + cc, ov);
            }
            tc::tmem_st_wait();
          }
        }
#pragma unroll
        for (int ch = 0; ch < 16; ++ch)  // 16-byte chunk ch = keys 8ch .. 8ch+7; 64 keys per swizzle atom
          *reinterpret_cast<uint4*>(pbuf + (ch >> 3) * (kBQ * 128) + sw128(r, ch & 7)) =
              make_uint4(pk[4 * ch], pk[4 * ch + 1], pk[4 * ch + 2], pk[4 * ch + 3]);
        l = l * corr + ((rs[0] + rs[1]) + (rs[2] + rs[3]));
        m = m_new;
        fence_async_smem();  // P stores visible to the tensor cores
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&p_full[x]);
      }
      if (!ok) break;
      // ---- epilogue: O_X / l (with the sink) -> bf16 rows ----
      if (!tc::mbar_wait(&o_done[x], items & 1, a.status)) break;
      tc::fence_after_sync();
      float f = 1.f;
      if (a.sinks != nullptr) {
        const float sk = a.sinks[it.head] * kLog2e;
        const float mn = fmaxf(m, sk);
        f = (m == -INFINITY) ? 0.f : ex2(m - mn);
        l = l * f + ex2(sk - mn);
      }
      const float inv = l > 0.f ? f / l * a.v_scale : 0.f;
      const bool row_ok = qrow < it.qlen;
      uint4* op = reinterpret_cast<uint4*>(a.out + (size_t)(it.q0 + qrow) * a.nq * kD + (size_t)it.head * kD);
#pragma unroll
      for (int cc = 0; cc < kD; cc += 16) {
        uint32_t ov[16];
        tc::tmem_ld_32x32b_x16(o_addr + cc, ov);
        tc::tmem_ld_wait();
        if (row_ok) {
#pragma unroll
          for (int h8 = 0; h8 < 2; ++h8) {
            uint4 u;
            __nv_bfloat162* ub = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
            for (int t = 0; t < 4; ++t)
              ub[t] = __floats2bfloat162_rn(__uint_as_float(ov[h8 * 8 + 2 * t]) * inv,
                                            __uint_as_float(ov[h8 * 8 + 2 * t + 1]) * inv);
            op[(cc >> 3) + h8] = u;
          }
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&o_free[x]);
      ++items;
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) tc::tmem_dealloc(tmem, kTmemCols);
}

// ---------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// The paged cache [num_blocks, nkv, bs, 64] as rows of 64 bf16; one box = one cache block of
// one kv head (bs rows x 128 bytes), 128-byte swizzle.
static int cache_map(CUtensorMap* m, const void* cache, int num_blocks, int nkv, int bs) {
  auto enc = encoder();
  if (!enc) return kBadShape;
  cuuint64_t dims[2] = {(cuuint64_t)kD, (cuuint64_t)num_blocks * nkv * bs};
  cuuint64_t strides[1] = {(cuuint64_t)kD * 2};
  cuuint32_t box[2] = {(cuuint32_t)kD, (cuuint32_t)bs};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(cache), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : kTensorMapErrorBase + (int)r;
}

// The query rows [T, q_stride] (head h at columns h * 64) as a 2-D map; one box = 128 rows x
// one head (128 bytes), 128-byte swizzle; rows past T read as zeros.
static int q_map(CUtensorMap* m, const void* q, int T, int nq, int q_stride) {
  auto enc = encoder();
  if (!enc) return kBadShape;
  cuuint64_t dims[2] = {(cuuint64_t)nq * kD, (cuuint64_t)T};
  cuuint64_t strides[1] = {(cuuint64_t)q_stride * 2};
  cuuint32_t box[2] = {(cuuint32_t)kD, (cuuint32_t)kBQ};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(q), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : kTensorMapErrorBase + (int)r;
}

}  // namespace fa
}  // namespace b200

using namespace b200;

// Which prefill calls the tensor-core kernel takes: head dim 64, bf16 queries and cache,
// cache blocks that tile 128 keys (8 <= block_size <= 128, a power of two).
extern "C" int b200_prefill_tc_supported(int d, int dtype, int cache_dtype, int block_size) {
  return d == fa::kD && dtype == kBF16 && cache_dtype == kBF16 && block_size >= 8 && block_size <= 128 &&
         (block_size & (block_size - 1)) == 0;
}

extern "C" int b200_paged_attention_prefill_tc(void* out, const void* q, const void* k_cache, const void* v_cache,
                                               int num_blocks, const int* block_tables, const int* seq_lens,
                                               const int* query_start_loc, const float* sinks, int B, int nq,
                                               int nkv, int d, int q_stride, int block_size, int max_blocks,
                                               int window, float scale, float k_scale, float v_scale,
                                               int max_query_len, int num_tokens, int dtype, int cache_dtype,
                                               int* status, cudaStream_t s) {
  if (!b200_prefill_tc_supported(d, dtype, cache_dtype, block_size)) return kBadShape;
  if (nkv <= 0 || nq % nkv || q_stride % 8 || q_stride < nq * d || num_blocks <= 0 || num_tokens < 0)
    return kBadShape;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_cache) |
       reinterpret_cast<uintptr_t>(v_cache) | reinterpret_cast<uintptr_t>(out)) & 15)
    return kBadAlignment;
  if (B == 0 || max_query_len == 0 || num_tokens == 0) return 0;
  CUtensorMap tq, tk, tv;
  int rc;
  if ((rc = fa::q_map(&tq, q, num_tokens, nq, q_stride))) return rc;
  if ((rc = fa::cache_map(&tk, k_cache, num_blocks, nkv, block_size))) return rc;
  if ((rc = fa::cache_map(&tv, v_cache, num_blocks, nkv, block_size))) return rc;
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaFuncSetAttribute(fa::fa_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, fa::kSmem);
    if (sms <= 0) sms = 148;
  }
  fa::Args a{};
  a.out = static_cast<__nv_bfloat16*>(out);
  a.block_tables = block_tables;
  a.seq_lens = seq_lens;
  a.qsl = query_start_loc;
  a.sinks = sinks;
  a.B = B, a.nq = nq, a.nkv = nkv, a.bs = block_size, a.max_blocks = max_blocks;
  a.window = window, a.causal = 1;
  a.n_qt = (max_query_len + fa::kQT * fa::kBQ - 1) / (fa::kQT * fa::kBQ);
  a.num_items = a.n_qt * B * nq;
  a.scale_log2 = scale * k_scale * fa::kLog2e;
  a.v_scale = v_scale;
  a.status = status;
  const int grid = a.num_items < sms ? a.num_items : sms;  // persistent: one CTA per SM
  launch_k(fa::fa_prefill_kernel, dim3(grid), dim3(fa::kThreads), fa::kSmem, s, tq, tk, tv, a);
  return (int)cudaGetLastError();
}
