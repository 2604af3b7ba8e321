// Paged attention with sink logits, sliding windows and fp8 KV (decode and prefill),
// plus contiguous varlen attention (vision encoder).
//
// Semantics (restated from the Trainium plugin's PyTorch fallbacks):
//   * sink logits join the softmax denominator only
//     (functional/attention/attention_cte.py:163-173, attention_decode.py:707-724);
//   * query at position p sees keys j with j <= p and, with window W > 0, j > p - W;
//   * fp8 caches hold k/k_scale, v/v_scale: k_scale is folded into the softmax scale,
//     v_scale into the output;
//   * cache layout HND [num_blocks, kv_heads, block_size, d], block_tables [B, max_blocks].
//
// Design: FlashAttention-2 style warp tiles on the tensor cores (mma.sync m16n8k16,
// bf16 in, fp32 accumulate) with cp.async double-buffered K/V tiles of 64 keys in
// XOR-swizzled shared memory.
//   decode : one CTA per (split, kv head, sequence); the GQA group of query heads is the
//            16-row M dimension (group <= 16, zero-padded), each of the 4 warps owns 16
//            of the 64 keys of a tile and keeps its own online-softmax state; the warps
//            merge in shared memory, and splits merge in a combine kernel (LSE merge).
//            M = 8..16 rows is below tcgen05's 64-row minimum, and the kernel is bound by
//            HBM reads of the cache, so the warp-level MMA is the right unit here.
//   prefill: one CTA per (64-query tile, query head, sequence), K/V read through the block
//            table, so chunked prefill and prefix-cache hits need no gather.
#include <cooperative_groups.h>

#include "launch.h"
#include "launch_pdl.h"
#include "mma_utils.cuh"
#include "noalloc.h"

namespace b200 {

constexpr int kKT = 64;  // keys per tile
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// Decode context parallelism: the tokens of a sequence are dealt to the ``size`` ranks of a
// DCP group one cache block at a time (token t lives on rank (t / bs) % size), and every rank
// stores its share densely in the same virtual blocks: local token u of block-table entry
// u / bs.  A shard computes attention over its own tokens and writes (normalised output,
// natural-log LSE) without sinks; the group merges the shards.
struct CpArgs {
  int rank, size;  // size 1: no context parallelism
  float* lse;      // [tokens, nq] partial log-sum-exp; nullptr: plain attention (sinks applied)
};

// number of this rank's tokens among global positions [0, x)
B200_D int cp_count_local(int x, int bs_log, CpArgs cp) {
  if (cp.size == 1) return x;
  const int span = cp.size << bs_log;
  const int full = x / span, rem = x - full * span;
  return (full << bs_log) + min(max(rem - (cp.rank << bs_log), 0), 1 << bs_log);
}

// global position of this rank's local token u
B200_D int cp_global_pos(int u, int bs_log, CpArgs cp) {
  if (cp.size == 1) return u;
  return ((((u >> bs_log) * cp.size) + cp.rank) << bs_log) + (u & ((1 << bs_log) - 1));
}

// ---------------------------------------------------------------------------------------
// K/V tile loader: 64 keys x D dims into swizzled bf16 shared memory.  For fp8 caches the
// raw bytes go through a staging buffer and are converted (with the cache scale left to
// the caller).
// ---------------------------------------------------------------------------------------
template <int D>
struct TileGeom {
  static constexpr int kChunks = D / 8;  // 16-byte chunks per bf16 row
  static constexpr int kTileElems = kKT * D;
};

template <int D, typename CT>
B200_D void load_kv_tile(__nv_bfloat16* Ks, __nv_bfloat16* Vs, uint8_t* stage, const CT* kc, const CT* vc,
                         const int* bt_row, int tile_key0, int key_end, int bs_log, int nkv, int h) {
  // block size is a power of two (the engine enforces it): shifts, not integer division,
  // which would run on the transcendental (XU) pipe that the softmax already saturates
  constexpr int C = TileGeom<D>::kChunks;
  const int bs_mask = (1 << bs_log) - 1;
  if constexpr (sizeof(CT) == 2) {
    for (int i = threadIdx.x; i < kKT * C; i += blockDim.x) {
      const int k = i / C, c = i % C;
      const int gk = tile_key0 + k;
      const bool ok = gk < key_end;
      size_t off = 0;
      if (ok) {
        const int blk = bt_row[gk >> bs_log];
        off = ((((size_t)blk * nkv + h) << bs_log) + (gk & bs_mask)) * D + c * 8;
      }
      cp_async16(Ks + swz(k, c, C) * 8, kc + off, ok ? 16 : 0);
      cp_async16(Vs + swz(k, c, C) * 8, vc + off, ok ? 16 : 0);
    }
  } else {
    // fp8: D bytes per row -> D/16 chunks; staged then converted by the caller
    constexpr int C8 = D / 16;
    for (int i = threadIdx.x; i < kKT * C8; i += blockDim.x) {
      const int k = i / C8, c = i % C8;
      const int gk = tile_key0 + k;
      const bool ok = gk < key_end;
      size_t off = 0;
      if (ok) {
        const int blk = bt_row[gk >> bs_log];
        off = ((((size_t)blk * nkv + h) << bs_log) + (gk & bs_mask)) * D + c * 16;
      }
      cp_async16(stage + (k * D + c * 16), reinterpret_cast<const uint8_t*>(kc) + off, ok ? 16 : 0);
      cp_async16(stage + kKT * D + (k * D + c * 16), reinterpret_cast<const uint8_t*>(vc) + off, ok ? 16 : 0);
    }
  }
}

template <int D>
B200_D void convert_fp8_tile(__nv_bfloat16* Ks, __nv_bfloat16* Vs, const uint8_t* stage) {
  constexpr int C = D / 8;
  for (int i = threadIdx.x; i < kKT * C; i += blockDim.x) {
    const int k = i / C, c = i % C;
#pragma unroll
    for (int w = 0; w < 2; ++w) {
      const uint8_t* src = stage + w * kKT * D + k * D + c * 8;
      __nv_bfloat16* dst = (w == 0 ? Ks : Vs) + swz(k, c, C) * 8;
      uint2 raw = *reinterpret_cast<const uint2*>(src);
      const uint8_t* b = reinterpret_cast<const uint8_t*>(&raw);
      uint32_t packed[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        __nv_fp8_e4m3 lo, hi;
        lo.__x = b[2 * j];
        hi.__x = b[2 * j + 1];
        packed[j] = pack_bf16(float(lo), float(hi));
      }
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<uint4*>(packed);
    }
  }
}

// ---------------------------------------------------------------------------------------
// Decode
// ---------------------------------------------------------------------------------------
template <int D, int S, typename T, typename CT>
__global__ void __launch_bounds__(128) decode_kernel(T* __restrict__ out, const T* __restrict__ q,
                                                     const CT* __restrict__ kc, const CT* __restrict__ vc,
                                                     const int* __restrict__ block_tables,
                                                     const int* __restrict__ seq_lens, const float* __restrict__ sinks,
                                                     int nq, int nkv, int q_stride, int bs, int max_blocks, int window,
                                                     float scale_log2, float v_scale, float* __restrict__ ws,
                                                     int num_splits, int cluster_merge, CpArgs cp) {
  pdl_wait();  // predecessor output visible (programmatic dependent launch)
  pdl_trigger();
  constexpr int C = D / 8;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __nv_bfloat16* Ks = reinterpret_cast<__nv_bfloat16*>(smem_raw);            // [S][64*D]
  __nv_bfloat16* Vs = Ks + S * kKT * D;                                      // [S][64*D]
  uint8_t* stage = reinterpret_cast<uint8_t*>(Vs + S * kKT * D);             // fp8 staging [S][2][64*D]

  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int G = nq / nkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qd = lane & 3, r0 = lane >> 2;
  const int bs_log = 31 - __clz(bs);
  // this rank's key range [lo, L) in local token indices (the window is in global positions)
  const int Lg = seq_lens[b];
  const int L = cp_count_local(Lg, bs_log, cp);
  const int lo = (window > 0) ? cp_count_local(max(0, Lg - window), bs_log, cp) : 0;
  // split the key range [lo, L) by whole cache blocks
  int key_begin = 0, key_end = 0;
  if (L > 0) {
    const int fb = lo / bs, lb = (L - 1) / bs, nb = lb - fb + 1;
    const int bps = cdiv(nb, num_splits);
    const int b0 = fb + split * bps, b1 = min(fb + (split + 1) * bps, lb + 1);
    if (b0 < b1) {
      key_begin = max(b0 * bs, lo);
      key_end = min(b1 * bs, L);
    }
  }
  const int* bt_row = block_tables + (size_t)b * max_blocks;
  const bool hi_rows = G > 8;  // rows r0 + 8 of the 16-row MMA hold real heads

  // S-stage cp.async ring: tiles t+1 .. t+S-1 are in flight while tile t is consumed, so a
  // CTA with few tiles (a split of a short range) pays one memory latency, not one per tile.
  // One commit group per tile slot (empty past the end) keeps the group arithmetic uniform.
  // Issued before the Q fragments are read, so the two memory round trips overlap.
  const int ntiles = key_end > key_begin ? cdiv(key_end - key_begin, kKT) : 0;
#pragma unroll
  for (int p = 0; p < S - 1; ++p) {
    if (p < ntiles)
      load_kv_tile<D, CT>(Ks + p * kKT * D, Vs + p * kKT * D, stage + p * 2 * kKT * D, kc, vc, bt_row,
                          key_begin + p * kKT, key_end, bs_log, nkv, h);
    cp_async_commit();
  }
  // Q fragments (A operand, rows = heads of the group)
  uint32_t qf[D / 16][4];
  {
    const T* qb = q + (size_t)b * q_stride + (size_t)(h * G) * D;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int hv = 0; hv < 2; ++hv) {      // rows r0 / r0+8
#pragma unroll
        for (int kh = 0; kh < 2; ++kh) {    // dims lo / hi 8
          const int row = r0 + hv * 8;
          const int dim = kk * 16 + kh * 8 + 2 * qd;
          float a = 0.f, c = 0.f;
          if (row < G) {
            a = to_float(qb[(size_t)row * D + dim]);
            c = to_float(qb[(size_t)row * D + dim + 1]);
          }
          qf[kk][kh * 2 + hv] = pack_bf16(a, c);
        }
      }
    }
  }

  float o[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};

  for (int t = 0; t < ntiles; ++t) {
    const int buf = t % S;
    cp_async_wait<S - 2>();  // groups 0..t complete: tile t landed
    __syncthreads();         // ...for every thread; and every warp is done with tile t-1
    {
      const int nt = t + S - 1, nb = nt % S;  // refill the slot tile t-1 used
      if (nt < ntiles)
        load_kv_tile<D, CT>(Ks + nb * kKT * D, Vs + nb * kKT * D, stage + nb * 2 * kKT * D, kc, vc, bt_row,
                            key_begin + nt * kKT, key_end, bs_log, nkv, h);
      cp_async_commit();
    }
    __nv_bfloat16* K = Ks + buf * kKT * D;
    __nv_bfloat16* V = Vs + buf * kKT * D;
    if constexpr (sizeof(CT) == 1) {
      convert_fp8_tile<D>(K, V, stage + buf * 2 * kKT * D);
      __syncthreads();
    }
    const int key0 = key_begin + t * kKT + warp * 16;
    // S = Q K^T for this warp's 16 keys: two n8 tiles
    float s[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const int mi = lane >> 3;
      const int krow = warp * 16 + (mi >> 1) * 8 + (lane & 7);
      const int kch = kk * 2 + (mi & 1);
      uint32_t b0, b1, b2, b3;
      ldmatrix_x4(b0, b1, b2, b3, K + swz(krow, kch, C) * 8);
      uint32_t bA[2] = {b0, b1}, bB[2] = {b2, b3};
      mma_bf16_16816(s[0], qf[kk], bA);
      mma_bf16_16816(s[1], qf[kk], bB);
    }
    // mask + online softmax, row r0 (r = 0) and row r0 + 8 (r = 1); with a group of at most
    // 8 heads the second half is zero padding and skips its exponentials (the XU pipe is the
    // decode kernel's limiter, ahead of HBM)
    float corr[2] = {1.f, 1.f};
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      if (r == 1 && !hi_rows) {
        s[0][2] = s[0][3] = s[1][2] = s[1][3] = 0.f;
        continue;
      }
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
#pragma unroll
        for (int e2 = 0; e2 < 2; ++e2) {
          const int key = key0 + j * 8 + 2 * qd + e2;
          float v = s[j][2 * r + e2] * scale_log2;
          if (key >= key_end) v = -INFINITY;
          s[j][2 * r + e2] = v;
          mx = fmaxf(mx, v);
        }
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mnew = fmaxf(m_run[r], mx);
      corr[r] = (mnew == -INFINITY) ? 1.f : exp2f(m_run[r] - mnew);
      m_run[r] = mnew;
      float rs = 0.f;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
#pragma unroll
        for (int e2 = 0; e2 < 2; ++e2) {
          const float p = (mnew == -INFINITY) ? 0.f : exp2f(s[j][2 * r + e2] - mnew);
          s[j][2 * r + e2] = p;
          rs += p;
        }
      }
      rs += __shfl_xor_sync(0xffffffffu, rs, 1);
      rs += __shfl_xor_sync(0xffffffffu, rs, 2);
      l_run[r] = l_run[r] * corr[r] + rs;
    }
#pragma unroll
    for (int n = 0; n < D / 8; ++n) {
      o[n][0] *= corr[0];
      o[n][1] *= corr[0];
      o[n][2] *= corr[1];
      o[n][3] *= corr[1];
    }
    // O += P V  (P: 16 rows x 16 keys as the A operand)
    uint32_t pa[4] = {pack_bf16(s[0][0], s[0][1]), pack_bf16(s[0][2], s[0][3]), pack_bf16(s[1][0], s[1][1]),
                      pack_bf16(s[1][2], s[1][3])};
#pragma unroll
    for (int n = 0; n < D / 8; n += 2) {
      const int mi = lane >> 3;
      const int vrow = warp * 16 + (mi & 1) * 8 + (lane & 7);
      const int vch = n + (mi >> 1);
      uint32_t b0, b1, b2, b3;
      ldmatrix_x4_trans(b0, b1, b2, b3, V + swz(vrow, vch, C) * 8);
      uint32_t bA[2] = {b0, b1}, bB[2] = {b2, b3};
      mma_bf16_16816(o[n], pa, bA);
      mma_bf16_16816(o[n + 1], pa, bB);
    }
  }
  cp_async_wait<0>();  // only empty groups can remain; keeps the reuse below obviously safe

  // ---- merge the 4 warps (shared memory reuses the K/V area) ----
  float* sm_m = reinterpret_cast<float*>(smem_raw);     // [4][16]
  float* sm_l = sm_m + 4 * 16;                          // [4][16]
  float* sm_o = sm_l + 4 * 16;                          // [4][16][D]
  float* part_o = sm_o + 4 * 16 * D;                    // [16][D]  this split's normalised output
  float* part_lse = part_o + 16 * D;                    // [16]     and its log2-sum-exp
  __syncthreads();
  if (qd == 0) {
    sm_m[warp * 16 + r0] = m_run[0];
    sm_m[warp * 16 + r0 + 8] = m_run[1];
    sm_l[warp * 16 + r0] = l_run[0];
    sm_l[warp * 16 + r0 + 8] = l_run[1];
  }
#pragma unroll
  for (int n = 0; n < D / 8; ++n) {
    const int dim = n * 8 + 2 * qd;
    sm_o[(warp * 16 + r0) * D + dim] = o[n][0];
    sm_o[(warp * 16 + r0) * D + dim + 1] = o[n][1];
    sm_o[(warp * 16 + r0 + 8) * D + dim] = o[n][2];
    sm_o[(warp * 16 + r0 + 8) * D + dim + 1] = o[n][3];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, dim = i % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, sm_m[w * 16 + g]);
    float l = 0.f, acc = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float f = exp2f(sm_m[w * 16 + g] - M);
        l += sm_l[w * 16 + g] * f;
        acc += sm_o[(w * 16 + g) * D + dim] * f;
      }
    }
    const int head = h * G + g;
    if (cluster_merge) {
      part_o[i] = l > 0.f ? acc / l : 0.f;
      if (dim == 0) part_lse[g] = (l > 0.f) ? (M + log2f(l)) : -INFINITY;
    } else if (num_splits == 1) {
      float Mt = M, lt = l, at = acc;
      if (sinks != nullptr) {
        const float sk = sinks[head] * kLog2e;
        const float Mn = fmaxf(Mt, sk);
        const float f = (Mt == -INFINITY) ? 0.f : exp2f(Mt - Mn);
        lt = lt * f + exp2f(sk - Mn);
        at *= f;
      }
      const float r = lt > 0.f ? at / lt * v_scale : 0.f;
      out[(size_t)b * nq * D + (size_t)head * D + dim] = from_float<T>(r);
      if (cp.lse != nullptr && dim == 0) cp.lse[(size_t)b * nq + head] = lt > 0.f ? (Mt + log2f(lt)) * kLn2 : -INFINITY;
    } else {
      float* w = ws + (((size_t)b * nq + head) * num_splits + split) * (D + 1);
      w[dim] = l > 0.f ? acc / l : 0.f;
      if (dim == 0) w[D] = (l > 0.f) ? (M + log2f(l)) : -INFINITY;
    }
  }
  if (cluster_merge) {
    // Split merge inside the cluster (the splits of one (sequence, kv head) are the CTAs
    // of one cluster): every CTA publishes its partial in its own shared memory, then CTA
    // r merges outputs r, r + S, ... reading the peers' partials over distributed shared
    // memory.  No workspace round trip through L2 and no second kernel.
    namespace cg = cooperative_groups;
    cg::cluster_group cl = cg::this_cluster();
    cl.sync();  // every split's partial is visible cluster-wide
    const float* peer_o[8];
    const float* peer_lse[8];
#pragma unroll
    for (int sp = 0; sp < 8; ++sp) {
      if (sp < num_splits) {
        peer_o[sp] = cl.map_shared_rank(part_o, sp);
        peer_lse[sp] = cl.map_shared_rank(part_lse, sp);
      }
    }
    for (int i = split * blockDim.x + threadIdx.x; i < G * D; i += num_splits * blockDim.x) {
      const int g = i / D, dim = i % D, head = h * G + g;
      float lse[8];
      float M = sinks ? sinks[head] * kLog2e : -INFINITY;
#pragma unroll
      for (int sp = 0; sp < 8; ++sp) {
        lse[sp] = sp < num_splits ? peer_lse[sp][g] : -INFINITY;
        M = fmaxf(M, lse[sp]);
      }
      float den = (sinks && M != -INFINITY) ? exp2f(sinks[head] * kLog2e - M) : 0.f, acc = 0.f;
#pragma unroll
      for (int sp = 0; sp < 8; ++sp) {
        if (sp < num_splits && lse[sp] != -INFINITY) {
          const float e = exp2f(lse[sp] - M);
          den += e;
          acc += e * peer_o[sp][i];
        }
      }
      out[(size_t)b * nq * D + (size_t)head * D + dim] = from_float<T>(den > 0.f ? acc / den * v_scale : 0.f);
      if (cp.lse != nullptr && dim == 0) cp.lse[(size_t)b * nq + head] = den > 0.f ? (M + log2f(den)) * kLn2 : -INFINITY;
    }
    cl.sync();  // keep this CTA's shared memory alive until every peer has read it
  }
}

template <int D, typename T>
__global__ void decode_combine_kernel(T* __restrict__ out, const float* __restrict__ ws,
                                      const float* __restrict__ sinks, int nq, int num_splits, float v_scale,
                                      float* __restrict__ lse_out) {
  pdl_wait();  // predecessor output visible (programmatic dependent launch)
  pdl_trigger();
  // LSE merge of the splits (num_splits <= 32): one warp reads every split's log-sum-exp
  // at once and turns them into weights, then each thread sums its dims over the splits.
  // Two dependent memory round trips per CTA instead of one per split and pass.
  __shared__ float wt[32];
  __shared__ float scale_s;
  const int head = blockIdx.x, b = blockIdx.y;
  const float* w = ws + ((size_t)b * nq + head) * num_splits * (D + 1);
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    const float ls = lane < num_splits ? w[lane * (D + 1) + D] : -INFINITY;
    float M = ls;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    const float sk = sinks ? sinks[head] * kLog2e : -INFINITY;
    M = fmaxf(M, sk);
    const float e = (ls == -INFINITY) ? 0.f : exp2f(ls - M);
    float den = e;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
    if (sinks) den += exp2f(sk - M);
    wt[lane] = e;
    if (lane == 0) scale_s = den > 0.f ? v_scale / den : 0.f;
    if (lane == 0 && lse_out != nullptr) lse_out[(size_t)b * nq + head] = den > 0.f ? (M + log2f(den)) * kLn2 : -INFINITY;
  }
  __syncthreads();
  const float sc = scale_s;
  for (int dim = threadIdx.x; dim < D; dim += blockDim.x) {
    float acc = 0.f;
#pragma unroll 4
    for (int s = 0; s < num_splits; ++s) acc += w[s * (D + 1) + dim] * wt[s];
    out[(size_t)b * nq * D + (size_t)head * D + dim] = from_float<T>(acc * sc);
  }
}

// VLLM_B200_DECODE_CLUSTER=0 sends every split count through the workspace + combine path.
inline bool decode_cluster_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("VLLM_B200_DECODE_CLUSTER");
    v = (e != nullptr && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

template <int D, typename T, typename CT>
static int launch_decode(void* out, const void* q, const void* kc, const void* vc, const int* bt, const int* sl,
                         const float* sinks, int B, int nq, int nkv, int q_stride, int bs, int max_blocks, int window,
                         float scale, float k_scale, float v_scale, float* ws, int num_splits, CpArgs cp,
                         cudaStream_t s) {
  if (B == 0) return 0;
  if (num_splits < 1 || num_splits > 32) return kBadShape;  // the combine merges <= 32 splits in one warp
  // 2, 4 or 8 splits merge inside a thread-block cluster; other counts go through the
  // workspace and the combine kernel
  const bool cluster = (num_splits == 2 || num_splits == 4 || num_splits == 8) && decode_cluster_enabled();
  if (num_splits > 1 && !cluster && ws == nullptr) return kBadShape;
  // pipeline depth: 3 tile slots for d <= 64 (48 KB of bf16 K/V: four CTAs per SM, so 64
  // sequences x 8 (kv head, split) CTAs run in one wave), 2 above (the fp8 staging ring
  // rides on top).  A 4-slot ring measured slower on B200: three CTAs per SM put 512
  // CTAs into two waves.
  constexpr int S = D <= 64 ? 3 : 2;
  const size_t smem_tiles = S * 2 * kKT * D * sizeof(__nv_bfloat16) + (sizeof(CT) == 1 ? S * 2 * kKT * D : 0);
  const size_t smem_merge = (4 * 16 * 2 + 4 * 16 * D + 16 * D + 16) * sizeof(float);
  const size_t smem = smem_tiles > smem_merge ? smem_tiles : smem_merge;
  auto kern = decode_kernel<D, S, T, CT>;
  static bool attr_set = false;  // host-side, once per instantiation
  if (!attr_set) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attr_set = true;
  }
  dim3 grid(num_splits, nkv, B);
  if (cluster) {
    launch_kc(kern, grid, dim3(128), smem, s, (unsigned)num_splits, (T*)out, (const T*)q, (const CT*)kc,
              (const CT*)vc, bt, sl, sinks, nq, nkv, q_stride, bs, max_blocks, window, scale * k_scale * kLog2e,
              v_scale, ws, num_splits, 1, cp);
    return (int)cudaGetLastError();
  }
  launch_k(kern, dim3(grid), dim3(128), smem, s, (T*)out, (const T*)q, (const CT*)kc, (const CT*)vc, bt, sl, sinks,
           nq, nkv, q_stride, bs, max_blocks, window, scale * k_scale * kLog2e, v_scale, ws, num_splits, 0, cp);
  if (num_splits > 1) {
    launch_k(decode_combine_kernel<D, T>, dim3(nq, B), dim3(D < 128 ? D : 128), 0, s, (T*)out, ws, sinks, nq,
             num_splits, v_scale, cp.lse);
  }
  return (int)cudaGetLastError();
}

// ---------------------------------------------------------------------------------------
// Prefill / chunked prefill over the paged cache, and contiguous varlen attention.
// ---------------------------------------------------------------------------------------
struct PagedKV {
  const int* block_tables;
  int max_blocks, bs, nkv;
};

template <int D, int DP, typename T, typename CT, bool kPaged>
__global__ void __launch_bounds__(128) prefill_kernel(T* __restrict__ out, const T* __restrict__ q,
                                                      const CT* __restrict__ kc, const CT* __restrict__ vc,
                                                      PagedKV pk, const int* __restrict__ seq_lens,
                                                      const int* __restrict__ qsl, const float* __restrict__ sinks,
                                                      int nq, int nkv, int q_stride, int kv_stride, int window,
                                                      int causal, float scale_log2, float v_scale, CpArgs cp) {
  pdl_wait();  // predecessor output visible (programmatic dependent launch)
  pdl_trigger();
  // DP: head dim padded to a multiple of 16 for the QK^T k-steps (72 -> 80)
  constexpr int C = DP / 8;
  constexpr int kTile = kKT * ((C % 8 == 0) ? C : (C | 1)) * 8;  // elements per K or V tile
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __nv_bfloat16* Ks = reinterpret_cast<__nv_bfloat16*>(smem_raw);  // [2][kTile]
  __nv_bfloat16* Vs = Ks + 2 * kTile;
  uint8_t* stage = reinterpret_cast<uint8_t*>(Vs + 2 * kTile);

  const int qt = blockIdx.x, head = blockIdx.y, b = blockIdx.z;
  const int G = nq / nkv, h = head / G;
  const int q0 = qsl[b], qlen = qsl[b + 1] - q0;
  if (qt * 64 >= qlen) return;
  const int L = kPaged ? seq_lens[b] : qlen;  // global sequence length
  const int bs_log = kPaged ? 31 - __clz(pk.bs) : 0;
  const int L_loc = kPaged ? cp_count_local(L, bs_log, cp) : L;  // this rank's cached tokens
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qd = lane & 3, r0 = lane >> 2;
  const int pos_base = L - qlen;  // absolute position of query row 0
  const int row_w = qt * 64 + warp * 16;  // first query row of this warp
  // key range needed by the CTA, in local token indices
  const int p_first = pos_base + qt * 64, p_last = pos_base + min(qlen, (qt + 1) * 64) - 1;
  int key_lo = 0, key_hi = causal ? cp_count_local(p_last + 1, bs_log, cp) : L_loc;
  if (window > 0) key_lo = cp_count_local(max(0, p_first - window + 1), bs_log, cp);
  key_lo = (key_lo / kKT) * kKT;

  uint32_t qf[DP / 16][4];
  {
#pragma unroll
    for (int kk = 0; kk < DP / 16; ++kk)
#pragma unroll
      for (int hv = 0; hv < 2; ++hv)
#pragma unroll
        for (int kh = 0; kh < 2; ++kh) {
          const int row = row_w + r0 + hv * 8;
          const int dim = kk * 16 + kh * 8 + 2 * qd;
          float a = 0.f, c = 0.f;
          if (row < qlen && dim < D) {
            const T* qp = q + (size_t)(q0 + row) * q_stride + (size_t)head * D + dim;
            a = to_float(qp[0]);
            c = to_float(qp[1]);
          }
          qf[kk][kh * 2 + hv] = pack_bf16(a, c);
        }
  }
  float o[DP / 8][4];
#pragma unroll
  for (int n = 0; n < DP / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  const int my_p[2] = {pos_base + row_w + r0, pos_base + row_w + r0 + 8};

  auto load_tile = [&](int buf, int key0) {
    __nv_bfloat16* K = Ks + buf * kTile;
    __nv_bfloat16* V = Vs + buf * kTile;
    if constexpr (kPaged) {
      const int* bt_row = pk.block_tables + (size_t)b * pk.max_blocks;
      if constexpr (D == DP) {
        load_kv_tile<D, CT>(K, V, stage + buf * 2 * kKT * D, kc, vc, bt_row, key0, min(key_hi, L_loc), bs_log, nkv,
                            h);
      }
    } else {
      // contiguous [T, nkv, D] K/V of this sequence; D may be padded to DP with zeros
      for (int i = threadIdx.x; i < kKT * C; i += blockDim.x) {
        const int k = i / C, c = i % C;
        const int gk = key0 + k;
        const bool ok = gk < L && c * 8 < D;
        const size_t off = ok ? ((size_t)(q0 + gk) * kv_stride + (size_t)h * D + c * 8) : 0;
        cp_async16(K + swz(k, c, C) * 8, kc + off, ok ? 16 : 0);
        cp_async16(V + swz(k, c, C) * 8, vc + off, ok ? 16 : 0);
      }
    }
  };

  const int ntiles = key_hi > key_lo ? cdiv(key_hi - key_lo, kKT) : 0;
  if (ntiles > 0) {
    load_tile(0, key_lo);
    cp_async_commit();
  }
  for (int t = 0; t < ntiles; ++t) {
    const int buf = t & 1;
    if (t + 1 < ntiles) {
      load_tile(buf ^ 1, key_lo + (t + 1) * kKT);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    __nv_bfloat16* K = Ks + buf * kTile;
    __nv_bfloat16* V = Vs + buf * kTile;
    if constexpr (kPaged && sizeof(CT) == 1) {
      convert_fp8_tile<D>(K, V, stage + buf * 2 * kKT * D);
      __syncthreads();
    }
    const int key0 = key_lo + t * kKT;
    // skip tiles entirely outside this warp's visible range
    // warp-uniform bounds: rows row_w .. row_w+15 sit at positions wp_lo .. wp_hi
    const int wp_lo = pos_base + row_w, wp_hi = pos_base + row_w + 15;
    const int kp_first = cp_global_pos(key0, bs_log, cp), kp_last = cp_global_pos(key0 + kKT - 1, bs_log, cp);
    const bool warp_dead = (row_w >= qlen) || (causal && kp_first > wp_hi) ||
                           (window > 0 && kp_last <= wp_lo - window);
    if (!warp_dead) {
      float s[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < DP / 16; ++kk) {
#pragma unroll
        for (int jj = 0; jj < 8; jj += 2) {
          const int mi = lane >> 3;
          const int krow = jj * 8 + (mi >> 1) * 8 + (lane & 7);
          const int kch = kk * 2 + (mi & 1);
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(b0, b1, b2, b3, K + swz(krow, kch, C) * 8);
          uint32_t bA[2] = {b0, b1}, bB[2] = {b2, b3};
          mma_bf16_16816(s[jj], qf[kk], bA);
          mma_bf16_16816(s[jj + 1], qf[kk], bB);
        }
      }
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = key0 + j * 8 + 2 * qd + (e & 1);
          const int kp = cp_global_pos(key, bs_log, cp);
          const int p = my_p[e >> 1];
          bool ok = key < L_loc;
          if (causal) ok = ok && kp <= p;
          if (window > 0) ok = ok && kp > p - window;
          const float v = ok ? s[j][e] * scale_log2 : -INFINITY;
          s[j][e] = v;
          mx[e >> 1] = fmaxf(mx[e >> 1], v);
        }
      float corr[2];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
        const float mnew = fmaxf(m_run[r], mx[r]);
        corr[r] = (mnew == -INFINITY) ? 1.f : exp2f(m_run[r] - mnew);
        m_run[r] = mnew;
      }
      float rs[2] = {0.f, 0.f};
#pragma unroll
      for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float mref = m_run[e >> 1];
          const float p = (mref == -INFINITY) ? 0.f : exp2f(s[j][e] - mref);
          s[j][e] = p;
          rs[e >> 1] += p;
        }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
        rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
        l_run[r] = l_run[r] * corr[r] + rs[r];
      }
#pragma unroll
      for (int n = 0; n < DP / 8; ++n) {
        o[n][0] *= corr[0];
        o[n][1] *= corr[0];
        o[n][2] *= corr[1];
        o[n][3] *= corr[1];
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {  // 64 keys = 4 k16 steps
        uint32_t pa[4] = {pack_bf16(s[2 * kk][0], s[2 * kk][1]), pack_bf16(s[2 * kk][2], s[2 * kk][3]),
                          pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]),
                          pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3])};
#pragma unroll
        for (int n = 0; n < DP / 8; n += 2) {
          const int mi = lane >> 3;
          const int vrow = kk * 16 + (mi & 1) * 8 + (lane & 7);
          const int vch = n + (mi >> 1);
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4_trans(b0, b1, b2, b3, V + swz(vrow, vch, C) * 8);
          uint32_t bA[2] = {b0, b1}, bB[2] = {b2, b3};
          mma_bf16_16816(o[n], pa, bA);
          if (n + 1 < DP / 8) mma_bf16_16816(o[n + 1], pa, bB);
        }
      }
    }
    __syncthreads();
  }
  // finalize with the sink
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    float l = l_run[r], M = m_run[r];
    float f = 1.f;
    if (sinks != nullptr) {
      const float sk = sinks[head] * kLog2e;
      const float Mn = fmaxf(M, sk);
      f = (M == -INFINITY) ? 0.f : exp2f(M - Mn);
      l = l * f + exp2f(sk - Mn);
    }
    const float inv = l > 0.f ? f / l * v_scale : 0.f;
    const int row = row_w + r0 + r * 8;
    if (cp.lse != nullptr && row < qlen && qd == 0)
      cp.lse[(size_t)(q0 + row) * nq + head] = l > 0.f ? (M + log2f(l)) * kLn2 : -INFINITY;
    if (row < qlen) {
      T* op = out + (size_t)(q0 + row) * nq * D + (size_t)head * D;
#pragma unroll
      for (int n = 0; n < DP / 8; ++n) {
        const int dim = n * 8 + 2 * qd;
        if (dim < D) {
          op[dim] = from_float<T>(o[n][r * 2] * inv);
          op[dim + 1] = from_float<T>(o[n][r * 2 + 1] * inv);
        }
      }
    }
  }
}

template <int D, int DP, typename T, typename CT, bool kPaged>
static int launch_prefill(void* out, const void* q, const void* kc, const void* vc, PagedKV pk, const int* sl,
                          const int* qsl, const float* sinks, int B, int nq, int nkv, int q_stride, int kv_stride,
                          int window, int causal, float scale, float k_scale, float v_scale, int max_q,
                          CpArgs cp, cudaStream_t s) {
  if (B == 0 || max_q == 0) return 0;
  const size_t tile = (size_t)kKT * row_stride_chunks(DP / 8) * 8;
  const size_t smem = 2 * 2 * tile * sizeof(__nv_bfloat16) + (sizeof(CT) == 1 ? 2 * 2 * kKT * D : 0);
  auto kern = prefill_kernel<D, DP, T, CT, kPaged>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attr_set = true;
  }
  dim3 grid(cdiv(max_q, 64), nq, B);
  launch_k(kern, dim3(grid), dim3(128), smem, s, (T*)out, (const T*)q, (const CT*)kc, (const CT*)vc, pk, sl, qsl, sinks, nq, nkv,
           q_stride, kv_stride, window, causal, scale * k_scale * kLog2e, v_scale, cp);
  return (int)cudaGetLastError();
}

}  // namespace b200

using namespace b200;

static int paged_decode(void* out, const void* q, const void* k_cache, const void* v_cache, const int* block_tables,
                        const int* seq_lens, const float* sinks, int B, int nq, int nkv, int d, int q_stride,
                        int block_size, int max_blocks, int window, float scale, float k_scale, float v_scale,
                        float* workspace, int num_splits, CpArgs cp, int dtype, int cache_dtype, cudaStream_t s) {
  if (nq % nkv || nq / nkv > 16 || dtype != kBF16) return kBadShape;
  if (cp.size < 1 || cp.rank < 0 || cp.rank >= cp.size || (cp.size > 1 && (cp.lse == nullptr || sinks != nullptr)))
    return kBadShape;  // a shard writes its LSE and leaves the sinks to the merge
  if (block_size <= 0 || (block_size & (block_size - 1))) return kBadShape;  // addressed by shifts
  const bool fp8 = cache_dtype == kFP8E4M3;
#define DEC(DD)                                                                                                    \
  return fp8 ? launch_decode<DD, __nv_bfloat16, __nv_fp8_e4m3>(out, q, k_cache, v_cache, block_tables, seq_lens,   \
                                                                sinks, B, nq, nkv, q_stride, block_size, max_blocks, \
                                                                window, scale, k_scale, v_scale, workspace,          \
                                                                num_splits, cp, s)                                   \
             : launch_decode<DD, __nv_bfloat16, __nv_bfloat16>(out, q, k_cache, v_cache, block_tables, seq_lens,   \
                                                                sinks, B, nq, nkv, q_stride, block_size, max_blocks, \
                                                                window, scale, k_scale, v_scale, workspace,          \
                                                                num_splits, cp, s);
  if (d == 64) { DEC(64) }
  if (d == 128) { DEC(128) }
  if (d == 256) { DEC(256) }
#undef DEC
  return kBadShape;
}

extern "C" int b200_paged_attention_decode(void* out, const void* q, const void* k_cache, const void* v_cache,
                                           const int* block_tables, const int* seq_lens, const float* sinks, int B,
                                           int nq, int nkv, int d, int q_stride, int block_size, int max_blocks,
                                           int window, float scale, float k_scale, float v_scale, float* workspace,
                                           int num_splits, int dtype, int cache_dtype, cudaStream_t s) {
  return paged_decode(out, q, k_cache, v_cache, block_tables, seq_lens, sinks, B, nq, nkv, d, q_stride, block_size,
                      max_blocks, window, scale, k_scale, v_scale, workspace, num_splits, CpArgs{0, 1, nullptr},
                      dtype, cache_dtype, s);
}

extern "C" int b200_paged_attention_decode_cp(void* out, float* lse, const void* q, const void* k_cache,
                                              const void* v_cache, const int* block_tables, const int* seq_lens,
                                              int B, int nq, int nkv, int d, int q_stride, int block_size,
                                              int max_blocks, int window, float scale, float k_scale, float v_scale,
                                              float* workspace, int num_splits, int cp_rank, int cp_size, int dtype,
                                              int cache_dtype, cudaStream_t s) {
  return paged_decode(out, q, k_cache, v_cache, block_tables, seq_lens, nullptr, B, nq, nkv, d, q_stride,
                      block_size, max_blocks, window, scale, k_scale, v_scale, workspace, num_splits,
                      CpArgs{cp_rank, cp_size, lse}, dtype, cache_dtype, s);
}

static int paged_prefill(void* out, const void* q, const void* k_cache, const void* v_cache, const int* block_tables,
                         const int* seq_lens, const int* query_start_loc, const float* sinks, int B, int nq, int nkv,
                         int d, int q_stride, int block_size, int max_blocks, int window, float scale, float k_scale,
                         float v_scale, int max_query_len, CpArgs cp, int dtype, int cache_dtype, cudaStream_t s) {
  if (nq % nkv || dtype != kBF16) return kBadShape;
  if (cp.size < 1 || cp.rank < 0 || cp.rank >= cp.size || (cp.size > 1 && (cp.lse == nullptr || sinks != nullptr)))
    return kBadShape;
  if (block_size <= 0 || (block_size & (block_size - 1))) return kBadShape;  // addressed by shifts
  PagedKV pk{block_tables, max_blocks, block_size, nkv};
  const bool fp8 = cache_dtype == kFP8E4M3;
#define PRE(DD)                                                                                                     \
  return fp8 ? launch_prefill<DD, DD, __nv_bfloat16, __nv_fp8_e4m3, true>(                                          \
                   out, q, k_cache, v_cache, pk, seq_lens, query_start_loc, sinks, B, nq, nkv, q_stride, 0, window,  \
                   1, scale, k_scale, v_scale, max_query_len, cp, s)                                                 \
             : launch_prefill<DD, DD, __nv_bfloat16, __nv_bfloat16, true>(                                          \
                   out, q, k_cache, v_cache, pk, seq_lens, query_start_loc, sinks, B, nq, nkv, q_stride, 0, window,  \
                   1, scale, k_scale, v_scale, max_query_len, cp, s);
  if (d == 64) { PRE(64) }
  if (d == 128) { PRE(128) }
  if (d == 256) { PRE(256) }
#undef PRE
  return kBadShape;
}

extern "C" int b200_paged_attention_prefill(void* out, const void* q, const void* k_cache, const void* v_cache,
                                            const int* block_tables, const int* seq_lens, const int* query_start_loc,
                                            const float* sinks, int B, int T, int nq, int nkv, int d, int q_stride,
                                            int block_size, int max_blocks, int window, float scale, float k_scale,
                                            float v_scale, int max_query_len, int dtype, int cache_dtype,
                                            cudaStream_t s) {
  (void)T;
  return paged_prefill(out, q, k_cache, v_cache, block_tables, seq_lens, query_start_loc, sinks, B, nq, nkv, d,
                       q_stride, block_size, max_blocks, window, scale, k_scale, v_scale, max_query_len,
                       CpArgs{0, 1, nullptr}, dtype, cache_dtype, s);
}

extern "C" int b200_paged_attention_prefill_cp(void* out, float* lse, const void* q, const void* k_cache,
                                               const void* v_cache, const int* block_tables, const int* seq_lens,
                                               const int* query_start_loc, int B, int nq, int nkv, int d,
                                               int q_stride, int block_size, int max_blocks, int window, float scale,
                                               float k_scale, float v_scale, int max_query_len, int cp_rank,
                                               int cp_size, int dtype, int cache_dtype, cudaStream_t s) {
  return paged_prefill(out, q, k_cache, v_cache, block_tables, seq_lens, query_start_loc, nullptr, B, nq, nkv, d,
                       q_stride, block_size, max_blocks, window, scale, k_scale, v_scale, max_query_len,
                       CpArgs{cp_rank, cp_size, lse}, dtype, cache_dtype, s);
}

extern "C" int b200_varlen_attention(void* out, const void* q, const void* k, const void* v, const int* cu_seqlens,
                                     int B, int T, int nq, int nkv, int d, float scale, int causal, int max_seqlen,
                                     int dtype, cudaStream_t s) {
  if (nq % nkv || dtype != kBF16) return kBadShape;
  PagedKV pk{nullptr, 0, 0, nkv};
#define VAR(DD, DDP)                                                                                           \
  return launch_prefill<DD, DDP, __nv_bfloat16, __nv_bfloat16, false>(out, q, k, v, pk, nullptr, cu_seqlens,    \
                                                                      nullptr, B, nq, nkv, nq * DD, nkv * DD, 0, \
                                                                      causal, scale, 1.f, 1.f, max_seqlen,      \
                                                                      CpArgs{0, 1, nullptr}, s);
  if (d == 64) { VAR(64, 64) }
  if (d == 72) { VAR(72, 80) }
  if (d == 80) { VAR(80, 80) }
  if (d == 128) { VAR(128, 128) }
#undef VAR
  return kBadShape;
}

// =======================================================================================
// No-allocation entry point for split-KV paged decode attention.
//
// This entry point has no counterpart in the reference plugin; it exists for callers of
// this library that cannot allocate device memory themselves, for example a host runtime
// written in C that links this library directly but has no allocator handle, or a serving
// process whose device memory is entirely reserved up front by another component's
// caching allocator, so that a cudaMalloc here would either fail or force a device-wide
// synchronisation at a moment the caller cannot afford.  Such callers pass only inputs and
// outputs; the split-KV partial results live in a fixed array in this library instead of a
// caller-provided workspace.
//
// Limits and contract:
//   * scratch is a file-scope __device__ array of kNoAllocScratchFloats floats (4 MiB).  Every
//     GPU that loads this library reserves it until the process exits.  A call needs
//     B * nq * num_splits * (d + 1) floats when its splits merge through the scratch (any
//     count above 1 except 2, 4 and 8, which merge inside a thread-block cluster, unless
//     VLLM_B200_DECODE_CLUSTER=0); a call that needs more is rejected with kScratchTooSmall
//     (1005) and launches nothing.  Bad shapes (including nkv <= 0 or nq % nkv != 0) return
//     kBadShape (1003).
//   * the device address of the array is looked up once per device with
//     cudaGetSymbolAddress, on the first call made while that device is current; issue that
//     first call before any stream capture on the device.
//   * all calls share the one array and it keeps whatever the previous call wrote.  Nothing
//     in it has to start at zero: every partial result the combine step reads is written by
//     the same call first.  Calls whose kernels overlap on the GPU (different streams, no
//     ordering between them) race on the array and give wrong results; order them.
//   * no cudaMalloc, cudaFree or allocating library routine is called.
// =======================================================================================
namespace {

constexpr size_t kNoAllocScratchFloats = size_t(1) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_decode_scratch[kNoAllocScratchFloats];

float* g_scratch_addr[kMaxDevices] = {nullptr};

// Device address of g_decode_scratch for the current device (looked up once per device).
int scratch_for_current_device(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= kMaxDevices) return kBadShape;
  float* p = __atomic_load_n(&g_scratch_addr[dev], __ATOMIC_ACQUIRE);
  if (p == nullptr) {
    void* addr = nullptr;
    e = cudaGetSymbolAddress(&addr, g_decode_scratch);
    if (e != cudaSuccess) return (int)e;
    p = static_cast<float*>(addr);
    __atomic_store_n(&g_scratch_addr[dev], p, __ATOMIC_RELEASE);
  }
  *out = p;
  return 0;
}

}  // namespace

extern "C" int b200_paged_attention_decode_noalloc(void* out, const void* q, const void* k_cache,
                                                   const void* v_cache, const int* block_tables, const int* seq_lens,
                                                   const float* sinks, int B, int nq, int nkv, int d, int q_stride,
                                                   int block_size, int max_blocks, int window, float scale,
                                                   float k_scale, float v_scale, int num_splits, int dtype,
                                                   int cache_dtype, cudaStream_t s) {
  if (num_splits < 1 || B < 0 || nq <= 0 || d <= 0 || nkv <= 0 || nq % nkv) return kBadShape;
  // 2, 4 or 8 splits merge inside a thread-block cluster and touch no scratch
  const bool cluster = (num_splits == 2 || num_splits == 4 || num_splits == 8) && decode_cluster_enabled();
  const bool uses_scratch = num_splits > 1 && !cluster;
  const size_t need = uses_scratch ? (size_t)B * nq * num_splits * (d + 1) : 0;
  if (need > kNoAllocScratchFloats) return kScratchTooSmall;
  float* ws = nullptr;
  if (uses_scratch) {
    const int rc = scratch_for_current_device(&ws);
    if (rc) return rc;
  }
  return b200_paged_attention_decode(out, q, k_cache, v_cache, block_tables, seq_lens, sinks, B, nq, nkv, d,
                                     q_stride, block_size, max_blocks, window, scale, k_scale, v_scale, ws,
                                     num_splits, dtype, cache_dtype, s);
}
