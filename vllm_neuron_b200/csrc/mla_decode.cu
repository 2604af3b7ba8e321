// Multi-head latent attention (MLA) decode on tcgen05 tensor cores.
//
// Semantics (DeepSeek-style absorbed MLA; the reference plugin has no MLA model, so this
// follows the published MLA formulation): the paged cache holds one latent row per token,
//   c[t] = [kv_latent (512) | k_rope (64)]  (bf16, 576 values),
// shared by every query head.  A query head h of sequence b arrives absorbed into the same
// space, q[b, h] (576 values), and
//   s[h, t] = scale * <q[b, h], c[t]>,   p = softmax_t(s[h, :]),   o[b, h] = sum_t p[h, t] c[t][:512]
// for the tokens t < seq_lens[b] of the sequence's block table.  Output o is [B, Hq, 512]
// bf16 (the caller applies the value up-projection).
//
// Design (B200):
//   * keys are the MMA's M dimension: S^T [128 keys x NH heads] = C_tile (128 x 576) . Q^T, so
//     the 128-row tensor-core tile is full for any head count (16 .. 64 heads per CTA), and the
//     cache rows are the A operand exactly as they sit in memory (K-major, 128-byte swizzle);
//   * O^T [512 dims x NH heads] = V^T . P^T accumulates in TMEM as four 128-dim tiles; V^T is
//     the same cache tile read as an MN-major A operand (dims contiguous, keys strided);
//   * TMA (no multicast) brings one cache block per box into a ring of 32 KB stages: per
//     128-key tile, five stages of 128 latent dims for S, then four stages of the 512 value
//     dims again for P.V (the second read of a tile comes from L2);
//   * one thread issues TMA, one issues MMAs (S of the next tile while the softmax of this one
//     runs, from a second S buffer), two softmax warpgroups own the 128 TMEM lanes (lane = key
//     for S, lane = value dim for O), each for half of the tile's heads: per-head maxima are
//     reduced across lanes with a transposing warp butterfly and shared memory, O is rescaled
//     lazily (only when a head's running maximum grows by more than 2^8, FlashAttention-4's
//     rule), P goes to shared memory as the B operand of the P.V MMA (MN-major for 64 heads);
//   * split-KV over 128-key tiles, merged by a log-sum-exp combine kernel.
// Every mbarrier wait is bounded and records kWaitTimeout in `status`.
#include <algorithm>

#include "launch.h"
#include "launch_pdl.h"
#include "tcgen05.cuh"

namespace b200 {
namespace mla {

constexpr int kDqk = 576;        // latent (512) + rope (64)
constexpr int kDv = 512;         // value dims (the latent part)
constexpr int kChunks = 9;       // 64-dim (128-byte) chunks of a cache row
constexpr int kKeys = 128;       // keys per tile (MMA M)
constexpr int kChunkBytes = kKeys * 128;  // one 64-dim chunk of a tile: 16 KB
constexpr int kStageBytes = 2 * kChunkBytes;
constexpr int kQkStages = 5;     // chunks (0,1) (2,3) (4,5) (6,7) (8)
constexpr int kPvStages = 4;     // value chunks (0,1) .. (6,7): one 128-dim O tile each
constexpr int kStagesPerTile = kQkStages + kPvStages;
constexpr int kThreads = 384;  // warp 0 TMA, warp 1 MMA, warps 4-11 softmax (two groups)
constexpr int kColS = 0;         // TMEM: S^T of tile j at columns 64 (j & 1) + [0, NH), O^T tile i at 128 + i * NH
constexpr int kColO = 128;

// P^T as the MN-major B operand (a key's row of 64 heads is one 128-byte line, written with
// 16-byte stores) when the head tile is 64 wide; K-major (2-byte stores) for 16 / 32 heads.
template <int NH>
constexpr bool kPMnMajor() {
  return NH == 64;
}

template <int NH>
struct Smem {
  static constexpr int kRing = NH == 64 ? 4 : NH == 32 ? 5 : 6;
  static constexpr int kOffRing = 0;  // the ring first: any descriptor stride stays inside the CTA's shared memory
  static constexpr int kOffQ = kRing * kStageBytes;
  static constexpr int kQChunk = NH * 128;
  static constexpr int kOffP = kOffQ + kChunks * kQChunk;
  static constexpr int kOffRed = kOffP + 2 * kQChunk;          // float [4][NH]
  static constexpr int kOffM = kOffRed + 4 * NH * 4;           // float [NH] running maxima (log2 units)
  static constexpr int kOffFac = kOffM + NH * 4;               // float [NH] rescale factors of the tile
  static constexpr int kOffL = kOffFac + NH * 4;               // float [NH] final row sums
  static constexpr int kOffFlag = kOffL + NH * 4;              // int [2] rescale flag per tile parity
  static constexpr int kOffBar = (kOffFlag + 8 + 7) / 8 * 8;
  static constexpr int kNumBars = 2 * kRing + 7;  // full, empty, q_full, s_full[2], p_full, pv_done, pv_landed, pv_zeroed
  static constexpr int kBytes = kOffBar + kNumBars * 8 + 16;
  static constexpr int kAlloc = kBytes + 1024;
  static constexpr uint32_t kTmemCols = kColO + 4 * NH <= 128 ? 128 : kColO + 4 * NH <= 256 ? 256 : 512;
  static_assert(kAlloc <= 232448, "shared memory budget");
};

// MN-major operand in the 128-byte swizzle layout: rows of 128 bytes (64 MN elements), 8-row
// groups along K 1024 bytes apart (SBO), the next 64 MN elements `lbo` bytes on (LBO).
B200_D uint64_t desc_sw128_mn(const void* smem, uint32_t lbo) {
  const uint64_t a = tc::smem_addr(smem);
  uint64_t d = 0;
  d |= (a >> 4) & 0x3FFFull;
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

B200_D void named_bar_softmax() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

B200_D uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&p);
}

// Reduce N per-lane values (lane = key) across the warp's 32 lanes with a transposing
// butterfly: at each step a lane keeps half of its values and trades the other half with its
// partner, so N = 64 costs 62 shuffles instead of 320.  Afterwards lane l holds the results
// for heads 2l, 2l + 1 (N = 64) in a[0..1], head l (N = 32) or head l / 2 (N = 16) in a[0].
template <int N, bool kMax>
B200_D void lane_reduce(float (&a)[N], int lane) {
#pragma unroll
  for (int s = 0; s < 5; ++s) {
    const int off = 16 >> s;
    const int n = N >> s;  // values still held per lane
    if (n > 1) {
      const bool upper = (lane & off) != 0;
#pragma unroll
      for (int i = 0; i < n / 2; ++i) {
        const float send = upper ? a[i] : a[i + n / 2];
        const float keep = upper ? a[i + n / 2] : a[i];
        const float recv = __shfl_xor_sync(0xffffffffu, send, off);
        a[i] = kMax ? fmaxf(keep, recv) : keep + recv;
      }
    } else {
      const float recv = __shfl_xor_sync(0xffffffffu, a[0], off);
      a[0] = kMax ? fmaxf(a[0], recv) : a[0] + recv;
    }
  }
}

// Store lane_reduce's per-head results of this warp to dst[0 .. N): lane l holds heads 2l and
// 2l + 1 for N = 64, head l / (32 / N) for N <= 32 (its first lane writes it).
template <int N>
B200_D void store_lane_result(float* dst, const float (&a)[N], int lane) {
  if constexpr (N == 64) {
    dst[2 * lane] = a[0];
    dst[2 * lane + 1] = a[1];
  } else {
    constexpr int per = 32 / N;
    if (lane % per == 0) dst[lane / per] = a[0];
  }
}

// N consecutive fp32 TMEM columns of this warp's 32 lanes (N = 8, 16 or 32), waited.
template <int N>
B200_D void tmem_ld_cols(uint32_t taddr, float (&v)[N]) {
  if constexpr (N == 8) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
    tc::tmem_ld_wait();
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = __uint_as_float(r[e]);
  } else {
#pragma unroll
    for (int c = 0; c < N / 16; ++c) {
      uint32_t r[16];
      tc::tmem_ld_32x32b_x16(taddr + c * 16, r);
      tc::tmem_ld_wait();
#pragma unroll
      for (int e = 0; e < 16; ++e) v[c * 16 + e] = __uint_as_float(r[e]);
    }
  }
}

// Store N fp32 columns back (the caller waits with tmem_st_wait).
template <int N>
B200_D void tmem_st_cols(uint32_t taddr, const float (&v)[N]) {
  if constexpr (N == 8) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
                 "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
                 "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
                 "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])));
  } else {
#pragma unroll
    for (int c = 0; c < N / 16; ++c) {
      uint32_t r[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) r[e] = __float_as_uint(v[c * 16 + e]);
      tc::tmem_st_32x32b_x16(taddr + c * 16, r);
    }
  }
}

// Grid (num_splits, head groups, B).  Warp 0: TMA; warp 1: TMEM owner and MMA issuer;
// warps 4..7: softmax and epilogue.
template <int NH>
__global__ void __launch_bounds__(kThreads, 1) mla_decode_kernel(
    const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmC,
    __nv_bfloat16* __restrict__ out, float* __restrict__ ws, const int* __restrict__ block_tables,
    const int* __restrict__ seq_lens, int Hq, int num_blocks, int bs_log, int max_blocks, float scale_log2,
    int num_splits, int* status) {
  pdl_wait();
  pdl_trigger();
  using L = Smem<NH>;
  constexpr int R = L::kRing;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_off = tc::smem_addr(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_off & 1023u)) & 1023u);
  uint8_t* ring = smem + L::kOffRing;
  uint8_t* sQ = smem + L::kOffQ;
  uint8_t* sP = smem + L::kOffP;
  float* red = reinterpret_cast<float*>(smem + L::kOffRed);
  float* m_used = reinterpret_cast<float*>(smem + L::kOffM);
  float* fac = reinterpret_cast<float*>(smem + L::kOffFac);
  float* lsum = reinterpret_cast<float*>(smem + L::kOffL);
  int* flag = reinterpret_cast<int*>(smem + L::kOffFlag);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* empty = full + R;
  uint64_t* q_full = empty + R;
  uint64_t* s_full = q_full + 1;  // [2]: one per S buffer
  uint64_t* p_full = s_full + 2;
  uint64_t* pv_done = p_full + 1;
  uint64_t* pv_landed = pv_done + 1;  // the split's partial last tile: its P.V stages are in
  uint64_t* pv_zeroed = pv_landed + 1;  // ... and the softmax warps have zeroed the rows past the end
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pv_zeroed + 1);

  const int split = blockIdx.x, grp = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // this split's 128-key tiles
  const int Lseq = max(0, seq_lens[b]);
  const int tiles_all = cdiv(Lseq, kKeys);
  const int tps = cdiv(max(tiles_all, 1), num_splits);
  const int t_begin = min(split * tps, tiles_all), t_end = min(t_begin + tps, tiles_all);
  const int ntiles = t_end - t_begin;
  const int key_end = min(t_end * kKeys, Lseq);
  const int* bt = block_tables + (size_t)b * max_blocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < R; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    tc::mbar_init(q_full, 1);
    tc::mbar_init(&s_full[0], 1);
    tc::mbar_init(&s_full[1], 1);
    tc::mbar_init(p_full, 256);
    tc::mbar_init(pv_done, 1);
    tc::mbar_init(pv_landed, 1);
    tc::mbar_init(pv_zeroed, 256);
    tc::fence_barrier_init();
    tc::prefetch_tmap(&tmQ);
    tc::prefetch_tmap(&tmC);
    flag[0] = flag[1] = 0;
  }
  if (threadIdx.x >= 128 && threadIdx.x < 128 + NH) m_used[threadIdx.x - 128] = -INFINITY;  // softmax threads
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, L::kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0 && ntiles > 0) {
      // ---------------- TMA producer ----------------
      // ring order: S stages of tile 0, then per tile j: S stages of tile j + 1, P.V stages of
      // tile j (the MMA issuer consumes in the same order, so S(j + 1) overlaps softmax(j))
      tc::mbar_arrive_expect_tx(q_full, kChunks * L::kQChunk);
      for (int c = 0; c < kChunks; ++c) tc::tma_load_3d(sQ + c * L::kQChunk, &tmQ, c * 64, grp * NH, b, q_full);
      const int nb = kKeys >> bs_log;  // cache blocks per tile (bs >= 16: at most 8)
      int it = 0;
      bool ok = true;
      auto load_stages = [&](int j, bool qk) {
        const int key0 = (t_begin + j) * kKeys;
        int blk[8];
        for (int r = 0; r < nb; ++r) {
          // blocks past the sequence repeat the tile's first block: finite data, masked later
          const int key = key0 + (r << bs_log) < key_end ? key0 + (r << bs_log) : key0;
          int id = (key >> bs_log) < max_blocks ? bt[key >> bs_log] : -1;
          if (id < 0 || id >= num_blocks) {
            record(status, kBadIndex, 40, id);
            id = 0;
          }
          blk[r] = id;
        }
        const int nst = qk ? kQkStages : kPvStages;
        for (int st = 0; st < nst && ok; ++st, ++it) {
          const int slot = it % R, use = it / R;
          if (it >= R && !tc::mbar_wait(&empty[slot], (use - 1) & 1, status)) {
            ok = false;
            break;
          }
          const int nch = (qk && st == kQkStages - 1) ? 1 : 2;
          tc::mbar_arrive_expect_tx(&full[slot], nch * kChunkBytes);
          for (int cc = 0; cc < nch; ++cc)
            for (int r = 0; r < nb; ++r)
              tc::tma_load_2d(ring + slot * kStageBytes + cc * kChunkBytes + (r << bs_log) * 128, &tmC,
                              (2 * st + cc) * 64, blk[r] << bs_log, &full[slot]);
        }
      };
      load_stages(0, true);
      for (int j = 0; j < ntiles && ok; ++j) {
        if (j + 1 < ntiles) load_stages(j + 1, true);
        load_stages(j, false);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && ntiles > 0) {
      // ---------------- MMA issuer ----------------
      const uint32_t id_s = tc::idesc_f16_bf16(kKeys, NH);
      // A = V^T MN-major; B = P^T MN-major (heads contiguous) when a P row is one 128-byte line
      const uint32_t id_o = tc::idesc_f16_bf16(kKeys, NH) | (1u << 15) | (kPMnMajor<NH>() ? (1u << 16) : 0u);
      bool ok = tc::mbar_wait(q_full, 0, status);
      tc::fence_after_sync();
      int it = 0;
      auto qk = [&](int j) {
        const uint32_t t_s = tmem + kColS + (j & 1) * 64;
        for (int st = 0; st < kQkStages && ok; ++st, ++it) {
          const int slot = it % R, use = it / R;
          if (!tc::mbar_wait(&full[slot], use & 1, status)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const int nch = st == kQkStages - 1 ? 1 : 2;
          for (int cc = 0; cc < nch; ++cc) {
            const int c = 2 * st + cc;
            uint8_t* a = ring + slot * kStageBytes + cc * kChunkBytes;
            uint8_t* bq = sQ + c * L::kQChunk;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              tc::mma_f16(t_s, tc::desc_sw128(a + kk * 32), tc::desc_sw128(bq + kk * 32), id_s,
                          (c | kk) != 0 ? 1u : 0u);
          }
          tc::mma_commit(&empty[slot]);
        }
        if (ok) tc::mma_commit(&s_full[j & 1]);
      };
      if (ok) qk(0);
      for (int j = 0; j < ntiles && ok; ++j) {
        if (j + 1 < ntiles) qk(j + 1);  // S(j + 1) into the other buffer while softmax(j) runs
        if (!ok || !tc::mbar_wait(p_full, j & 1, status)) break;
        tc::fence_after_sync();
        if ((t_begin + j + 1) * kKeys > key_end) {  // partial last tile: rows past the end get zeroed first
          for (int i = 0; i < kPvStages && ok; ++i)
            ok = tc::mbar_wait(&full[(it + i) % R], ((it + i) / R) & 1, status);
          if (!ok) break;
          tc::mbar_arrive(pv_landed);
          if (!tc::mbar_wait(pv_zeroed, 0, status)) break;
          tc::fence_after_sync();
        }
        for (int i = 0; i < kPvStages && ok; ++i, ++it) {
          const int slot = it % R, use = it / R;
          if (!tc::mbar_wait(&full[slot], use & 1, status)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          uint8_t* v = ring + slot * kStageBytes;
#pragma unroll
          for (int ks = 0; ks < kKeys / 16; ++ks) {
            const uint64_t bp = kPMnMajor<NH>() ? tc::desc_sw128(sP + ks * 2048)
                                                : tc::desc_sw128(sP + (ks >> 2) * L::kQChunk + (ks & 3) * 32);
            tc::mma_f16(tmem + kColO + i * NH, desc_sw128_mn(v + ks * 2048, kChunkBytes), bp, id_o,
                        (j > 0 || ks > 0) ? 1u : 0u);
          }
          tc::mma_commit(&empty[slot]);
        }
        if (!ok) break;
        tc::mma_commit(pv_done);
      }
    }
  } else if (warp >= 4) {
    // ---------------- softmax / epilogue ----------------
    // Two warpgroups, each owning half of the tile's heads (HH = NH / 2); thread t of a group =
    // TMEM lane t (key t for S, value dim t of a 128-dim tile for O).
    constexpr int HH = NH / 2;
    const int ts = threadIdx.x - 128;     // 0 .. 255
    const int g = ts >> 7;                // head half
    const int q4 = warp & 3, t = q4 * 32 + lane;
    const int h0 = g * HH;
    const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
    float lp[HH];
#pragma unroll
    for (int h = 0; h < HH; ++h) lp[h] = 0.f;
    named_bar_softmax();  // m_used initialised
    // A failed (timed-out) wait sets ok = false but never leaves the loop: every softmax
    // thread runs the same sequence of named barriers and warp-collective TMEM accesses; the
    // waits after a recorded error return at once.
    bool ok = true;
    float v[HH];
    for (int j = 0; j < ntiles; ++j) {
      const int key0 = (t_begin + j) * kKeys;
      const int nvalid = min(kKeys, key_end - key0);
      ok = tc::mbar_wait(&s_full[j & 1], (j >> 1) & 1, status) && ok;
      tc::fence_after_sync();
      const uint32_t s_addr = tmem + lane_base + kColS + (j & 1) * 64 + h0;
      // per-head maximum of the tile over the 128 keys (lanes): transposing butterfly in the
      // warp, then the four warps through shared memory (the butterfly consumes its copy; the
      // scores are read from TMEM again below, which costs less than keeping both live)
      tmem_ld_cols<HH>(s_addr, v);
#pragma unroll
      for (int h = 0; h < HH; ++h) v[h] = t < nvalid ? v[h] * scale_log2 : -INFINITY;
      lane_reduce<HH, true>(v, lane);
      store_lane_result<HH>(red + q4 * NH + h0, v, lane);
      named_bar_softmax();
      if (ts < NH) {
        const float tm = fmaxf(fmaxf(red[ts], red[NH + ts]), fmaxf(red[2 * NH + ts], red[3 * NH + ts]));
        const float mo = m_used[ts];
        float mn = mo, f = 1.f;
        if (tm > mo + 8.f) {  // lazy rescale: exponentials stay below 2^8 otherwise
          mn = tm;
          f = mo == -INFINITY ? 0.f : exp2f(mo - mn);
          flag[j & 1] = 1;
        }
        m_used[ts] = mn;
        fac[ts] = f;
      }
      named_bar_softmax();
      const bool resc = flag[j & 1] != 0;
      if (ts == 0) flag[(j + 1) & 1] = 0;  // read by nobody until the next tile's barrier
      // exponentials (in place) while the previous tile's P.V may still run
      tmem_ld_cols<HH>(s_addr, v);
#pragma unroll
      for (int h = 0; h < HH; ++h) v[h] = t < nvalid ? v[h] * scale_log2 : -INFINITY;
#pragma unroll
      for (int h = 0; h < HH; ++h) {
        const float p = v[h] == -INFINITY ? 0.f : exp2f(v[h] - m_used[h0 + h]);
        lp[h] = lp[h] * fac[h0 + h] + p;
        v[h] = p;
      }
      // P.V of the previous tile must be done before P or O change
      if (j > 0) {
        ok = tc::mbar_wait(pv_done, (j - 1) & 1, status) && ok;
        tc::fence_after_sync();
        if (resc) {
          constexpr int CW = HH < 16 ? HH : 16;  // columns per TMEM round trip
#pragma unroll 1
          for (int i = 0; i < 4; ++i) {
#pragma unroll 1
            for (int c = 0; c < HH; c += CW) {
              float o[CW];
              const uint32_t addr = tmem + lane_base + kColO + i * NH + h0 + c;
              tmem_ld_cols<CW>(addr, o);
#pragma unroll
              for (int h = 0; h < CW; ++h) o[h] *= fac[h0 + c + h];
              tmem_st_cols<CW>(addr, o);
            }
          }
          tc::tmem_st_wait();
        }
      }
      if constexpr (kPMnMajor<NH>()) {
        // P^T MN-major: key t's row holds its 64 heads (one 128-byte line, 16-byte units
        // swizzled by t % 8); this group writes units 4g .. 4g + 3
        uint8_t* row = sP + t * 128;
#pragma unroll
        for (int u = 0; u < HH / 8; ++u) {
          uint4 w;
          w.x = pack_bf16x2(v[8 * u + 0], v[8 * u + 1]);
          w.y = pack_bf16x2(v[8 * u + 2], v[8 * u + 3]);
          w.z = pack_bf16x2(v[8 * u + 4], v[8 * u + 5]);
          w.w = pack_bf16x2(v[8 * u + 6], v[8 * u + 7]);
          const int uu = g * (HH / 8) + u;
          *reinterpret_cast<uint4*>(row + ((uu ^ (t & 7)) << 4)) = w;
        }
      } else {
        // P^T K-major: row h, key t of chunk t / 64
        uint8_t* pc = sP + (t >> 6) * L::kQChunk;
        const int kc = t & 63;
#pragma unroll
        for (int hh = 0; hh < HH; ++hh) {
          const int h = h0 + hh;
          *reinterpret_cast<__nv_bfloat16*>(pc + h * 128 + ((((kc >> 3) ^ (h & 7))) << 4) + (kc & 7) * 2) =
              __float2bfloat16(v[hh]);
        }
      }
      tc::fence_proxy_async();  // generic shared-memory writes -> the tensor core's async proxy
      tc::fence_before_sync();
      tc::mbar_arrive(p_full);
      if (nvalid < kKeys) {
        // the split's last tile ends inside it: once the MMA issuer reports its P.V stages
        // landed, zero the value rows of the keys past the end (0 x stale cache bytes could be
        // NaN in P.V); happens once per CTA, so the barriers see a single phase
        ok = tc::mbar_wait(pv_landed, 0, status) && ok;
        if (t >= nvalid) {
          const int itv = kQkStages + j * kStagesPerTile + (j + 1 < ntiles ? kQkStages : 0);
#pragma unroll 1
          for (int i = 0; i < kPvStages; ++i) {
            uint4* row = reinterpret_cast<uint4*>(ring + ((itv + i) % R) * kStageBytes + g * kChunkBytes + t * 128);
#pragma unroll
            for (int u = 0; u < 8; ++u) row[u] = make_uint4(0u, 0u, 0u, 0u);
          }
        }
        tc::fence_proxy_async();
        tc::mbar_arrive(pv_zeroed);
      }
    }
    // ---- epilogue ----
    if (ok && ntiles > 0) ok = tc::mbar_wait(pv_done, (ntiles - 1) & 1, status);
    tc::fence_after_sync();
    lane_reduce<HH, false>(lp, lane);
    store_lane_result<HH>(red + q4 * NH + h0, lp, lane);
    named_bar_softmax();
    if (ts < NH) lsum[ts] = red[ts] + red[NH + ts] + red[2 * NH + ts] + red[3 * NH + ts];
    named_bar_softmax();
    const bool have = __all_sync(0xffffffffu, ok && ntiles > 0);  // uniform per warp (tcgen05.ld is collective)
    constexpr int CW = HH < 16 ? HH : 16;  // columns per TMEM load
#pragma unroll 1
    for (int ic = 0; ic < 4 * (HH / CW); ++ic) {
      const int i = ic / (HH / CW), c = (ic % (HH / CW)) * CW;
      float o[CW];
      if (have) tmem_ld_cols<CW>(tmem + lane_base + kColO + i * NH + h0 + c, o);
#pragma unroll
      for (int hc = 0; hc < CW; ++hc) {
        const int hh = c + hc, h = h0 + hh, head = grp * NH + h;
        if (head >= Hq) continue;
        const float l = lsum[h];
        const float val = (have && l > 0.f) ? o[hc] / l : 0.f;
        const int dim = i * 128 + t;
        if (num_splits == 1) {
          out[((size_t)b * Hq + head) * kDv + dim] = __float2bfloat16(val);
        } else {
          float* w = ws + (((size_t)b * Hq + head) * num_splits + split) * (kDv + 1);
          w[dim] = val;
          if (dim == 0) w[kDv] = (have && l > 0.f) ? m_used[h] + log2f(l) : -INFINITY;
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) tc::tmem_dealloc(tmem, L::kTmemCols);
}

// Log-sum-exp merge of the splits: grid (Hq, B), 128 threads, 4 value dims each.
__global__ void __launch_bounds__(128) mla_combine_kernel(__nv_bfloat16* __restrict__ out,
                                                          const float* __restrict__ ws, int Hq, int num_splits) {
  pdl_wait();
  pdl_trigger();
  const int head = blockIdx.x, b = blockIdx.y;
  const float* w = ws + ((size_t)b * Hq + head) * num_splits * (kDv + 1);
  float M = -INFINITY;
  for (int s = 0; s < num_splits; ++s) M = fmaxf(M, w[s * (kDv + 1) + kDv]);
  float den = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int s = 0; s < num_splits; ++s) {
    const float ls = w[s * (kDv + 1) + kDv];
    if (ls == -INFINITY) continue;
    const float e = exp2f(ls - M);
    den += e;
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[q] += e * w[s * (kDv + 1) + threadIdx.x + q * 128];
  }
#pragma unroll
  for (int q = 0; q < 4; ++q)
    out[((size_t)b * Hq + head) * kDv + threadIdx.x + q * 128] = __float2bfloat16(den > 0.f ? acc[q] / den : 0.f);
}

}  // namespace mla
}  // namespace b200

using namespace b200;
using namespace b200::mla;

namespace {

PFN_cuTensorMapEncodeTiled_v12000 mla_encoder() {
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

// q [B, Hq, 576] as a 3-D map; one box = 64 dims of NH heads of one sequence (heads past Hq
// read as zeros).
int q_map(CUtensorMap* m, const void* q, int B, int Hq, int NH) {
  auto enc = mla_encoder();
  if (!enc) return kBadShape;
  cuuint64_t dims[3] = {(cuuint64_t)kDqk, (cuuint64_t)Hq, (cuuint64_t)B};
  cuuint64_t strides[2] = {(cuuint64_t)kDqk * 2, (cuuint64_t)Hq * kDqk * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)NH, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(q), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : kTensorMapErrorBase + (int)r;
}

// The paged latent cache [num_blocks, bs, 576] as rows of 576 bf16; one box = 64 dims of one
// cache block (bs rows x 128 bytes).
int cache_map(CUtensorMap* m, const void* c, int num_blocks, int bs) {
  auto enc = mla_encoder();
  if (!enc) return kBadShape;
  cuuint64_t dims[2] = {(cuuint64_t)kDqk, (cuuint64_t)num_blocks * bs};
  cuuint64_t strides[1] = {(cuuint64_t)kDqk * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)bs};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(c), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : kTensorMapErrorBase + (int)r;
}

template <int NH>
int launch_mla(void* out, const void* q, const void* cache, const int* bt, const int* sl, int B, int Hq,
               int num_blocks, int bs_log, int max_blocks, float scale, float* ws, int num_splits, int* status,
               cudaStream_t s) {
  CUtensorMap tq, tcm;
  int rc;
  if ((rc = q_map(&tq, q, B, Hq, NH))) return rc;
  if ((rc = cache_map(&tcm, cache, num_blocks, 1 << bs_log))) return rc;
  auto kern = mla_decode_kernel<NH>;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Smem<NH>::kAlloc);
    attr = true;
  }
  const dim3 grid(num_splits, cdiv(Hq, NH), B);
  launch_k(kern, grid, dim3(kThreads), Smem<NH>::kAlloc, s, tq, tcm, static_cast<__nv_bfloat16*>(out), ws, bt, sl,
           Hq, num_blocks, bs_log, max_blocks, scale * 1.4426950408889634f, num_splits, status);
  if (num_splits > 1)
    launch_k(mla_combine_kernel, dim3(Hq, B), dim3(128), 0, s, static_cast<__nv_bfloat16*>(out), (const float*)ws, Hq,
             num_splits);
  return (int)cudaGetLastError();
}

}  // namespace

// MLA decode attention (see the top of this file).  out [B, Hq, 512] bf16; q [B, Hq, 576] bf16
// contiguous; cache [num_blocks, block_size, 576] bf16; block_tables [B, max_blocks] int32;
// seq_lens [B] int32; scale: the softmax scale.  num_splits > 1 splits each sequence's 128-key
// tiles across CTAs and needs ws of B * Hq * num_splits * 513 floats (no zeroing needed).
// block_size: a power of two from 16 to 128.
extern "C" int b200_mla_decode(void* out, const void* q, const void* cache, const int* block_tables,
                               const int* seq_lens, int B, int Hq, int num_blocks, int block_size, int max_blocks,
                               float scale, float* ws, int num_splits, int* status, cudaStream_t s) {
  if (B < 0 || Hq < 1 || num_blocks < 1 || max_blocks < 1 || num_splits < 1 || num_splits > 64) return kBadShape;
  if (block_size < 16 || block_size > 128 || (block_size & (block_size - 1))) return kBadShape;
  if (num_splits > 1 && ws == nullptr) return kBadShape;
  if (((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(cache)) & 15))
    return kBadAlignment;
  if (B == 0) return 0;
  const int bs_log = 31 - __builtin_clz((unsigned)block_size);
  if (Hq <= 16)
    return launch_mla<16>(out, q, cache, block_tables, seq_lens, B, Hq, num_blocks, bs_log, max_blocks, scale, ws,
                          num_splits, status, s);
  if (Hq <= 32)
    return launch_mla<32>(out, q, cache, block_tables, seq_lens, B, Hq, num_blocks, bs_log, max_blocks, scale, ws,
                          num_splits, status, s);
  return launch_mla<64>(out, q, cache, block_tables, seq_lens, B, Hq, num_blocks, bs_log, max_blocks, scale, ws,
                        num_splits, status, s);
}
