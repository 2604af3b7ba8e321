// Gated DeltaNet (Qwen3-Next linear attention) kernels for sm_100a, plus the small gating
// kernels of the Qwen3-Next blocks.
//
// The reference plugin has no linear-attention model; the math is the public gated delta
// rule (Qwen3-Next, HF transformers modeling_qwen3_next.py) in its chunked form:
//
//   per chunk of C = 64 tokens, G = in-chunk cumulative log decay,
//     L_ij = beta_i (k_i . k_j) e^(G_i - G_j)  (j < i),   T = (I + L)^-1,
//     W = T (beta e^G k),  U = T (beta v),  P_ij = (q_i . k_j) e^(G_i - G_j)  (j <= i);
//   sequentially over chunks with state S [dk, dv]:
//     V' = U - W S,   O = (e^G q) S + P V',   S <- e^(G_last) S + (e^(G_last - G) k)^T V'.
//
// Kernels:
//   conv1d_kernel / conv_state_update_kernel  depthwise causal conv (K = 4) + SiLU over a varlen
//       token batch, continuing from and updating the per-slot conv state;
//   gdn_chunk_index_kernel   chunk table of the varlen batch (device-side, no host sync);
//   gdn_chunk_prep_kernel    chunk-parallel part (grid = chunks x value heads): L2 norms, decay
//       cumsum, K K^T / Q K^T on tensor cores (mma.sync m16n8k16 bf16, fp32 accumulate), the
//       UT-transform inverse by blocked forward substitution (fp32), W and U on tensor cores;
//       writes W, U, e^G q, (e^(G_last-G) k)^T, P to a workspace;
//   gdn_chunk_scan_kernel    the sequential part (grid = sequences x value heads x 32-column
//       blocks of dv, since state columns are independent): the state block stays in registers
//       as mma accumulators, chunk operands stream through a double-buffered cp.async ring;
//   gdn_gated_norm_kernel    per-head RMSNorm gated by silu(z);
//   gdn_decode_kernel        recurrent update for decode (one CTA per (sequence, value head),
//       a thread pair owns one state column in registers), L2 norms, decay/strength and the
//       gated norm fused;
//   sigmoid_gate_mul_kernel, gated_add_kernel   attention output gate and shared-expert gate.
//
// State layouts: conv state [slots, C, K-1] (model dtype), recurrent state [slots, Hv, dk, dv]
// fp32.  Slots and the "continue from state" flags come from the runner; a slot index out of
// range is recorded in the status word and the sequence is skipped.
#include "common.cuh"
#include "mma_utils.cuh"

namespace b200 {
namespace dn {

using bf16 = __nv_bfloat16;

constexpr int kC = 64;        // chunk length
constexpr int kD = 128;       // key / value head dim
constexpr int kLd = kD + 8;   // padded smem row of a 128-wide tile (272 B = 17 x 16 B)
constexpr int kLdC = kC + 8;  // padded smem row of a 64-wide tile (144 B = 9 x 16 B)
constexpr int kLdU = 32 + 8;  // padded row of the 32-column U block
constexpr int kCB = 32;       // state columns per scan CTA

// workspace per (chunk, value head)
constexpr size_t kWsW = 0;                          // W   [64][128] bf16
constexpr size_t kWsU = kWsW + kC * kD * 2;         // U   [64][128] bf16
constexpr size_t kWsQ = kWsU + kC * kD * 2;         // e^G q [64][128] bf16
constexpr size_t kWsK = kWsQ + kC * kD * 2;         // (e^(G_last-G) k)^T [128][64] bf16
constexpr size_t kWsP = kWsK + (size_t)kD * kC * 2;  // P [64][64] bf16
constexpr size_t kWsG = kWsP + kC * kC * 2;         // G_last fp32
constexpr size_t kWsBytes = kWsG + 256;

B200_D float bf(bf16 v) { return __bfloat162float(v); }
B200_D float silu(float x) { return x / (1.f + expf(-x)); }
B200_D float softplus(float x) { return x > 20.f ? x : log1pf(expf(x)); }

// A fragment (16x16 at rows m0.., cols k0..) of a row-major bf16 smem matrix, row stride ld.
B200_D void frag_a(uint32_t a[4], const bf16* base, int ld, int m0, int k0) {
  const int l = threadIdx.x & 31;
  ldmatrix_x4(a[0], a[1], a[2], a[3], base + (size_t)(m0 + (l & 7) + ((l >> 3) & 1) * 8) * ld + k0 + (l >> 4) * 8);
}
// B fragments of the two 8-column n-tiles n0, n0+8 (16 k) from [n][k] storage.
B200_D void frag_b2(uint32_t b0[2], uint32_t b1[2], const bf16* base, int ld, int n0, int k0) {
  const int l = threadIdx.x & 31, mi = l >> 3;
  ldmatrix_x4(b0[0], b0[1], b1[0], b1[1], base + (size_t)(n0 + (mi >> 1) * 8 + (l & 7)) * ld + k0 + (mi & 1) * 8);
}
// Same from [k][n] storage (n contiguous), through transposing loads.
B200_D void frag_b2_kn(uint32_t b0[2], uint32_t b1[2], const bf16* base, int ld, int n0, int k0) {
  const int l = threadIdx.x & 31, mi = l >> 3;
  ldmatrix_x4_trans(b0[0], b0[1], b1[0], b1[1],
                    base + (size_t)(k0 + (mi & 1) * 8 + (l & 7)) * ld + n0 + (mi >> 1) * 8);
}
// accumulator element e of a 16x8 tile: row (lane/4) + 8*(e/2), col 2*(lane%4) + e%2
B200_D int acc_row(int e) { return ((threadIdx.x & 31) >> 2) + (e >> 1) * 8; }
B200_D int acc_col(int e) { return 2 * (threadIdx.x & 3) + (e & 1); }

B200_D void store_pair(bf16* p, float a, float b) { *reinterpret_cast<uint32_t*>(p) = pack_bf16(a, b); }

// ------------------------------------------------------------------------ causal conv
template <int K>
__global__ void __launch_bounds__(128) conv1d_kernel(bf16* __restrict__ out, const bf16* __restrict__ x, int ldx,
                                                     const bf16* __restrict__ w, bf16* __restrict__ cstate,
                                                     const int* __restrict__ qsl, const int* __restrict__ slots,
                                                     const int* __restrict__ init, int C, int seg, int num_slots,
                                                     int fuse_update, int* status) {
  const int c = blockIdx.x * 128 + threadIdx.x, b = blockIdx.y;
  if (c >= C) return;
  const int lo = qsl[b], len = qsl[b + 1] - lo;
  const int s0 = blockIdx.z * seg;
  if (s0 >= len) return;
  const int s1 = min(len, s0 + seg);
  const int slot = slots[b];
  if (slot < 0 || slot >= num_slots) {
    if (threadIdx.x == 0 && blockIdx.x == 0) record(status, kBadIndex, 30, slot);
    return;
  }
  bf16* st = cstate + ((size_t)slot * C + c) * (K - 1);
  const bool has = init[b] != 0;
  float wk[K], win[K - 1];
#pragma unroll
  for (int i = 0; i < K; ++i) wk[i] = bf(w[(size_t)c * K + i]);
#pragma unroll
  for (int i = 0; i < K - 1; ++i) {
    const int p = s0 - (K - 1) + i;
    win[i] = p >= 0 ? bf(x[(size_t)(lo + p) * ldx + c]) : (has ? bf(st[K - 1 + p]) : 0.f);
  }
  for (int t = s0; t < s1; ++t) {
    const float xv = bf(x[(size_t)(lo + t) * ldx + c]);
    float acc = wk[K - 1] * xv;
#pragma unroll
    for (int i = 0; i < K - 1; ++i) acc += wk[i] * win[i];
    out[(size_t)(lo + t) * C + c] = __float2bfloat16(silu(acc));
#pragma unroll
    for (int i = 0; i < K - 2; ++i) win[i] = win[i + 1];
    win[K - 2] = xv;
  }
  if (fuse_update) {  // this CTA saw the whole sequence: its window is the new state
#pragma unroll
    for (int i = 0; i < K - 1; ++i) st[i] = __float2bfloat16(win[i]);
  }
}

template <int K>
__global__ void __launch_bounds__(128) conv_state_update_kernel(const bf16* __restrict__ x, int ldx,
                                                                bf16* __restrict__ cstate,
                                                                const int* __restrict__ qsl,
                                                                const int* __restrict__ slots,
                                                                const int* __restrict__ init, int C, int num_slots) {
  const int c = blockIdx.x * 128 + threadIdx.x, b = blockIdx.y;
  if (c >= C) return;
  const int lo = qsl[b], len = qsl[b + 1] - lo;
  const int slot = slots[b];
  if (len <= 0 || slot < 0 || slot >= num_slots) return;
  bf16* st = cstate + ((size_t)slot * C + c) * (K - 1);
  const bool has = init[b] != 0;
  float nw[K - 1];
#pragma unroll
  for (int i = 0; i < K - 1; ++i) {
    const int p = len - (K - 1) + i;
    nw[i] = p >= 0 ? bf(x[(size_t)(lo + p) * ldx + c]) : (has ? bf(st[K - 1 + p]) : 0.f);
  }
#pragma unroll
  for (int i = 0; i < K - 1; ++i) st[i] = __float2bfloat16(nw[i]);
}

// ------------------------------------------------------------------------ chunk table
__global__ void gdn_chunk_index_kernel(int* __restrict__ seq_chunk_off, int* __restrict__ chunk_tab,
                                       int* __restrict__ n_chunks, const int* __restrict__ qsl, int B) {
  __shared__ int off[1025];
  for (int b = threadIdx.x; b < B; b += blockDim.x) off[b] = cdiv(max(0, qsl[b + 1] - qsl[b]), kC);
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int b = 0; b < B; ++b) {
      const int n = off[b];
      off[b] = acc;
      acc += n;
    }
    off[B] = acc;
    *n_chunks = acc;
  }
  __syncthreads();
  for (int b = threadIdx.x; b <= B; b += blockDim.x) seq_chunk_off[b] = off[b];
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    const int len = qsl[b + 1] - qsl[b];
    for (int j = 0; j * kC < len; ++j) {
      const int c = off[b] + j;
      chunk_tab[3 * c] = b;
      chunk_tab[3 * c + 1] = qsl[b] + j * kC;
      chunk_tab[3 * c + 2] = min(kC, len - j * kC);
    }
  }
}

// ------------------------------------------------------------------------ chunk prep
struct PrepSmem {
  static constexpr int kTile = kC * kLd;  // bf16 elements of one 64 x 128 tile
  static constexpr int kOffQ = kTile * 2;
  static constexpr int kOffV = kTile * 4;
  static constexpr int kOffKb = kTile * 6;
  static constexpr int kOffL = kTile * 8;                  // bytes
  static constexpr int kOffT = kOffL + kC * 65 * 4;
  static constexpr int kOffX = kOffT + kC * 65 * 4;
  static constexpr int kOffTb = kOffX + 3 * 16 * 17 * 4;
  static constexpr int kOffG = kOffTb + kC * kLdC * 2;
  static constexpr int kBytes = kOffG + 2 * kC * 4;
};

__global__ void __launch_bounds__(256) gdn_chunk_prep_kernel(uint8_t* __restrict__ ws,
                                                             const int* __restrict__ chunk_tab,
                                                             const int* __restrict__ n_chunks,
                                                             const bf16* __restrict__ mixed, int ldm,
                                                             const bf16* __restrict__ bb, const bf16* __restrict__ aa,
                                                             int ldab, const float* __restrict__ A_log,
                                                             const float* __restrict__ dt_bias, int nk, int nv,
                                                             float scale) {
  using L = PrepSmem;
  const int c = blockIdx.x, h = blockIdx.y;
  if (c >= *n_chunks) return;
  const int t0 = chunk_tab[3 * c + 1], C = chunk_tab[3 * c + 2];
  const int kh = h / (nv / nk);
  extern __shared__ __align__(16) uint8_t sm[];
  bf16* Kn = reinterpret_cast<bf16*>(sm);
  bf16* Qn = reinterpret_cast<bf16*>(sm + L::kOffQ);
  bf16* Vs = reinterpret_cast<bf16*>(sm + L::kOffV);
  bf16* Kb = reinterpret_cast<bf16*>(sm + L::kOffKb);
  float* Lf = reinterpret_cast<float*>(sm + L::kOffL);
  float* Tf = reinterpret_cast<float*>(sm + L::kOffT);
  float* Xs = reinterpret_cast<float*>(sm + L::kOffX);
  bf16* Tb = reinterpret_cast<bf16*>(sm + L::kOffTb);
  float* G = reinterpret_cast<float*>(sm + L::kOffG);
  float* Bt = G + kC;
  uint8_t* wc = ws + ((size_t)c * nv + h) * kWsBytes;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // 1. rows: L2-normalised q (times scale) and k, raw v; decay and strength
  for (int r = warp; r < kC; r += 8) {
    float q4[4] = {0.f, 0.f, 0.f, 0.f}, k4[4] = {0.f, 0.f, 0.f, 0.f}, v4[4] = {0.f, 0.f, 0.f, 0.f};
    if (r < C) {
      const bf16* row = mixed + (size_t)(t0 + r) * ldm;
      const uint2 uq = *reinterpret_cast<const uint2*>(row + kh * kD + lane * 4);
      const uint2 uk = *reinterpret_cast<const uint2*>(row + (nk + kh) * kD + lane * 4);
      const uint2 uv = *reinterpret_cast<const uint2*>(row + (2 * nk + h) * kD + lane * 4);
      const bf16* pq = reinterpret_cast<const bf16*>(&uq);
      const bf16* pk = reinterpret_cast<const bf16*>(&uk);
      const bf16* pv = reinterpret_cast<const bf16*>(&uv);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        q4[i] = bf(pq[i]);
        k4[i] = bf(pk[i]);
        v4[i] = bf(pv[i]);
      }
    }
    float sq = 0.f, sk = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      sq += q4[i] * q4[i];
      sk += k4[i] * k4[i];
    }
    sq = warp_sum(sq);
    sk = warp_sum(sk);
    const float iq = rsqrtf(sq + 1e-6f) * scale, ik = rsqrtf(sk + 1e-6f);
    bf16* dq = Qn + r * kLd + lane * 4;
    bf16* dk = Kn + r * kLd + lane * 4;
    bf16* dv = Vs + r * kLd + lane * 4;
    store_pair(dq, q4[0] * iq, q4[1] * iq);
    store_pair(dq + 2, q4[2] * iq, q4[3] * iq);
    store_pair(dk, k4[0] * ik, k4[1] * ik);
    store_pair(dk + 2, k4[2] * ik, k4[3] * ik);
    store_pair(dv, v4[0], v4[1]);
    store_pair(dv + 2, v4[2], v4[3]);
  }
  if (threadIdx.x < kC) {
    const int r = threadIdx.x;
    float g = 0.f, be = 0.f;
    if (r < C) {
      const size_t o = (size_t)(t0 + r) * ldab + h;
      g = -expf(A_log[h]) * softplus(bf(aa[o]) + dt_bias[h]);
      be = 1.f / (1.f + expf(-bf(bb[o])));
    }
    float s = g;  // inclusive scan within the warp
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    G[r] = s;
    Bt[r] = be;
  }
  __syncthreads();
  if (threadIdx.x >= 32 && threadIdx.x < kC) G[threadIdx.x] += G[31];
  __syncthreads();

  // 2. K K^T -> L (fp32, strictly lower, decayed, times beta);  Q K^T -> P (bf16, causal)
  {
    const int mt = warp & 3, nh = warp >> 2;
    float kk[4][4], qk[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) kk[j][e] = qk[j][e] = 0.f;
#pragma unroll
    for (int k0 = 0; k0 < kD; k0 += 16) {
      uint32_t ak[4], aq[4];
      frag_a(ak, Kn, kLd, mt * 16, k0);
      frag_a(aq, Qn, kLd, mt * 16, k0);
#pragma unroll
      for (int j = 0; j < 4; j += 2) {
        uint32_t b0[2], b1[2];
        frag_b2(b0, b1, Kn, kLd, nh * 32 + j * 8, k0);
        mma_bf16_16816(kk[j], ak, b0);
        mma_bf16_16816(kk[j + 1], ak, b1);
        mma_bf16_16816(qk[j], aq, b0);
        mma_bf16_16816(qk[j + 1], aq, b1);
      }
    }
    bf16* P = reinterpret_cast<bf16*>(wc + kWsP);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float pv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = mt * 16 + acc_row(e), jc = nh * 32 + j * 8 + acc_col(e);
        const float dec = jc <= i ? expf(G[i] - G[jc]) : 0.f;
        Lf[i * 65 + jc] = jc < i ? Bt[i] * kk[j][e] * dec : 0.f;
        pv[e] = (jc <= i && i < C) ? qk[j][e] * dec : 0.f;
      }
      const int i0 = mt * 16 + acc_row(0), jc0 = nh * 32 + j * 8 + acc_col(0);
      store_pair(P + i0 * kC + jc0, pv[0], pv[1]);
      store_pair(P + (i0 + 8) * kC + jc0, pv[2], pv[3]);
    }
  }
  __syncthreads();

  // 3. T = (I + L)^-1: 16x16 diagonal blocks by forward substitution (lane = column), then
  //    T_ij = -T_ii sum_{m=j}^{i-1} L_im T_mj by block distance
  if (warp < 4 && lane < 16) {
    const int o = warp * 16;
    float col[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      float acc = 0.f;
#pragma unroll
      for (int m = 0; m < r; ++m) acc += Lf[(o + r) * 65 + o + m] * col[m];
      col[r] = r < lane ? 0.f : (r == lane ? 1.f : -acc);
    }
#pragma unroll
    for (int r = 0; r < 16; ++r) Tf[(o + r) * 65 + o + lane] = col[r];
  }
  for (int e = threadIdx.x; e < kC * kC; e += blockDim.x) {  // upper blocks are zero
    const int r = e / kC, cc = e % kC;
    if ((cc >> 4) > (r >> 4)) Tf[r * 65 + cc] = 0.f;
  }
  __syncthreads();
  for (int d = 1; d < 4; ++d) {
    const int nb = 4 - d;
    for (int e = threadIdx.x; e < nb * 256; e += blockDim.x) {
      const int bi = e >> 8, r = (e >> 4) & 15, cc = e & 15;
      const int i = d + bi, j = i - d;
      float acc = 0.f;
      for (int m = j; m < i; ++m)
#pragma unroll
        for (int q = 0; q < 16; ++q) acc += Lf[(16 * i + r) * 65 + 16 * m + q] * Tf[(16 * m + q) * 65 + 16 * j + cc];
      Xs[(bi * 16 + r) * 17 + cc] = acc;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < nb * 256; e += blockDim.x) {
      const int bi = e >> 8, r = (e >> 4) & 15, cc = e & 15;
      const int i = d + bi, j = i - d;
      float acc = 0.f;
#pragma unroll
      for (int q = 0; q < 16; ++q) acc += Tf[(16 * i + r) * 65 + 16 * i + q] * Xs[(bi * 16 + q) * 17 + cc];
      Tf[(16 * i + r) * 65 + 16 * j + cc] = -acc;
    }
    __syncthreads();
  }

  // 4. operands: T (bf16), beta e^G k, beta v; write e^G q and (e^(G_last-G) k)^T
  const float gl = G[kC - 1];  // padded rows carry g = 0
  for (int e = threadIdx.x; e < kC * kC; e += blockDim.x) {
    const int r = e / kC, cc = e % kC;
    Tb[r * kLdC + cc] = __float2bfloat16(Tf[r * 65 + cc]);
  }
  bf16* Qg = reinterpret_cast<bf16*>(wc + kWsQ);
  bf16* KdT = reinterpret_cast<bf16*>(wc + kWsK);
  for (int e = threadIdx.x; e < kC * (kD / 2); e += blockDim.x) {
    const int r = e / (kD / 2), cc = (e % (kD / 2)) * 2;
    const float eg = expf(G[r]), bt = Bt[r];
    const float k0 = bf(Kn[r * kLd + cc]), k1 = bf(Kn[r * kLd + cc + 1]);
    store_pair(Kb + r * kLd + cc, bt * eg * k0, bt * eg * k1);
    store_pair(Vs + r * kLd + cc, bt * bf(Vs[r * kLd + cc]), bt * bf(Vs[r * kLd + cc + 1]));
    store_pair(Qg + r * kD + cc, bf(Qn[r * kLd + cc]) * eg, bf(Qn[r * kLd + cc + 1]) * eg);
  }
  for (int e = threadIdx.x; e < kD * (kC / 2); e += blockDim.x) {
    const int k = e / (kC / 2), t = (e % (kC / 2)) * 2;
    store_pair(KdT + k * kC + t, bf(Kn[t * kLd + k]) * expf(gl - G[t]), bf(Kn[(t + 1) * kLd + k]) * expf(gl - G[t + 1]));
  }
  if (threadIdx.x == 0) *reinterpret_cast<float*>(wc + kWsG) = gl;
  __syncthreads();

  // 5. W = T (beta e^G k),  U = T (beta v)   [64 x 128] each
  {
    const int mt = warp & 3, nh = warp >> 2;
    float w[8][4], u[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) w[j][e] = u[j][e] = 0.f;
#pragma unroll
    for (int k0 = 0; k0 < kC; k0 += 16) {
      uint32_t a[4];
      frag_a(a, Tb, kLdC, mt * 16, k0);
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        uint32_t b0[2], b1[2];
        frag_b2_kn(b0, b1, Kb, kLd, nh * 64 + j * 8, k0);
        mma_bf16_16816(w[j], a, b0);
        mma_bf16_16816(w[j + 1], a, b1);
        frag_b2_kn(b0, b1, Vs, kLd, nh * 64 + j * 8, k0);
        mma_bf16_16816(u[j], a, b0);
        mma_bf16_16816(u[j + 1], a, b1);
      }
    }
    bf16* Wg = reinterpret_cast<bf16*>(wc + kWsW);
    bf16* Ug = reinterpret_cast<bf16*>(wc + kWsU);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int r = mt * 16 + acc_row(0), cc = nh * 64 + j * 8 + acc_col(0);
      store_pair(Wg + r * kD + cc, w[j][0], w[j][1]);
      store_pair(Wg + (r + 8) * kD + cc, w[j][2], w[j][3]);
      store_pair(Ug + r * kD + cc, u[j][0], u[j][1]);
      store_pair(Ug + (r + 8) * kD + cc, u[j][2], u[j][3]);
    }
  }
}

// ------------------------------------------------------------------------ chunk scan
struct ScanSmem {
  static constexpr int kW = 0;                             // [64][kLd]
  static constexpr int kQ = kW + kC * kLd * 2;             // [64][kLd]
  static constexpr int kP = kQ + kC * kLd * 2;             // [64][kLdC]
  static constexpr int kK = kP + kC * kLdC * 2;            // [128][kLdC]
  static constexpr int kU = kK + kD * kLdC * 2;            // [64][kLdU]
  static constexpr int kStage = kU + kC * kLdU * 2;
  static constexpr int kS = 2 * kStage;                    // S^T bf16 [32][kLd]
  static constexpr int kV = kS + kCB * kLd * 2;            // V'^T bf16 [32][kLdC]
  static constexpr int kBytes = kV + kCB * kLdC * 2;
};

__global__ void __launch_bounds__(128) gdn_chunk_scan_kernel(bf16* __restrict__ o, const uint8_t* __restrict__ ws,
                                                             const int* __restrict__ seq_chunk_off,
                                                             const int* __restrict__ chunk_tab,
                                                             float* __restrict__ state, const int* __restrict__ slots,
                                                             const int* __restrict__ init, int nv, int num_slots,
                                                             int* status) {
  using L = ScanSmem;
  const int b = blockIdx.x, h = blockIdx.y, cb = blockIdx.z;
  const int c_begin = seq_chunk_off[b], c_end = seq_chunk_off[b + 1];
  if (c_end <= c_begin) return;
  const int slot = slots[b];
  if (slot < 0 || slot >= num_slots) {
    if (threadIdx.x == 0) record(status, kBadIndex, 40, slot);
    return;
  }
  extern __shared__ __align__(16) uint8_t sm[];
  bf16* Ss = reinterpret_cast<bf16*>(sm + L::kS);
  bf16* Vt = reinterpret_cast<bf16*>(sm + L::kV);
  const int warp = threadIdx.x >> 5;
  float* Sg = state + ((size_t)slot * nv + h) * kD * kD;

  float s[2][4][4];  // state rows warp*32 + mt*16 .., columns cb*32 + nt*8 ..
  const bool has = init[b] != 0;
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = warp * 32 + mt * 16 + acc_row(e), cc = cb * kCB + nt * 8 + acc_col(e);
        s[mt][nt][e] = has ? Sg[(size_t)r * kD + cc] : 0.f;
      }

  auto load_stage = [&](int buf, int ci) {
    const uint8_t* wc = ws + ((size_t)ci * nv + h) * kWsBytes;
    uint8_t* st = sm + buf * L::kStage;
    for (int i = threadIdx.x; i < kC * 16; i += blockDim.x) {  // W, e^G q: 64 rows x 16 chunks
      const int r = i >> 4, ch = i & 15;
      cp_async16(st + L::kW + (r * kLd + ch * 8) * 2, wc + kWsW + (r * kD + ch * 8) * 2, 16);
      cp_async16(st + L::kQ + (r * kLd + ch * 8) * 2, wc + kWsQ + (r * kD + ch * 8) * 2, 16);
    }
    for (int i = threadIdx.x; i < kC * 8; i += blockDim.x) {  // P: 64 rows x 8 chunks
      const int r = i >> 3, ch = i & 7;
      cp_async16(st + L::kP + (r * kLdC + ch * 8) * 2, wc + kWsP + (r * kC + ch * 8) * 2, 16);
    }
    for (int i = threadIdx.x; i < kD * 8; i += blockDim.x) {  // KdT: 128 rows x 8 chunks
      const int r = i >> 3, ch = i & 7;
      cp_async16(st + L::kK + (r * kLdC + ch * 8) * 2, wc + kWsK + (r * kC + ch * 8) * 2, 16);
    }
    for (int i = threadIdx.x; i < kC * 4; i += blockDim.x) {  // U columns of this block
      const int r = i >> 2, ch = i & 3;
      cp_async16(st + L::kU + (r * kLdU + ch * 8) * 2, wc + kWsU + (r * kD + cb * kCB + ch * 8) * 2, 16);
    }
  };

  load_stage(0, c_begin);
  cp_async_commit();
  for (int ci = c_begin; ci < c_end; ++ci) {
    const int buf = (ci - c_begin) & 1;
    if (ci + 1 < c_end) {
      load_stage(buf ^ 1, ci + 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    const uint8_t* st = sm + buf * L::kStage;
    const bf16* Ws = reinterpret_cast<const bf16*>(st + L::kW);
    const bf16* Qs = reinterpret_cast<const bf16*>(st + L::kQ);
    const bf16* Ps = reinterpret_cast<const bf16*>(st + L::kP);
    const bf16* Ks = reinterpret_cast<const bf16*>(st + L::kK);
    const bf16* Us = reinterpret_cast<const bf16*>(st + L::kU);
    // (1) S^T (bf16) to shared memory: [column][row]
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = warp * 32 + mt * 16 + acc_row(e), cc = nt * 8 + acc_col(e);
          Ss[cc * kLd + r] = __float2bfloat16(s[mt][nt][e]);
        }
    __syncthreads();
    // (2) V' = U - W S   (rows warp*16.., 32 columns)
    float vn[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) vn[j][0] = vn[j][1] = vn[j][2] = vn[j][3] = 0.f;
#pragma unroll
    for (int k0 = 0; k0 < kD; k0 += 16) {
      uint32_t a[4];
      frag_a(a, Ws, kLd, warp * 16, k0);
#pragma unroll
      for (int j = 0; j < 4; j += 2) {
        uint32_t b0[2], b1[2];
        frag_b2(b0, b1, Ss, kLd, j * 8, k0);
        mma_bf16_16816(vn[j], a, b0);
        mma_bf16_16816(vn[j + 1], a, b1);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int t = warp * 16 + acc_row(e), cc = j * 8 + acc_col(e);
        const float v = bf(Us[t * kLdU + cc]) - vn[j][e];
        Vt[cc * kLdC + t] = __float2bfloat16(v);
      }
    __syncthreads();
    // (3) O = (e^G q) S + P V'
    float ov[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) ov[j][0] = ov[j][1] = ov[j][2] = ov[j][3] = 0.f;
#pragma unroll
    for (int k0 = 0; k0 < kD; k0 += 16) {
      uint32_t a[4];
      frag_a(a, Qs, kLd, warp * 16, k0);
#pragma unroll
      for (int j = 0; j < 4; j += 2) {
        uint32_t b0[2], b1[2];
        frag_b2(b0, b1, Ss, kLd, j * 8, k0);
        mma_bf16_16816(ov[j], a, b0);
        mma_bf16_16816(ov[j + 1], a, b1);
      }
    }
#pragma unroll
    for (int k0 = 0; k0 < kC; k0 += 16) {
      uint32_t a[4];
      frag_a(a, Ps, kLdC, warp * 16, k0);
#pragma unroll
      for (int j = 0; j < 4; j += 2) {
        uint32_t b0[2], b1[2];
        frag_b2(b0, b1, Vt, kLdC, j * 8, k0);
        mma_bf16_16816(ov[j], a, b0);
        mma_bf16_16816(ov[j + 1], a, b1);
      }
    }
    {
      const int t0 = chunk_tab[3 * ci + 1], C = chunk_tab[3 * ci + 2];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int t = warp * 16 + acc_row(0), cc = cb * kCB + j * 8 + acc_col(0);
        if (t < C) store_pair(o + (size_t)(t0 + t) * nv * kD + h * kD + cc, ov[j][0], ov[j][1]);
        if (t + 8 < C) store_pair(o + (size_t)(t0 + t + 8) * nv * kD + h * kD + cc, ov[j][2], ov[j][3]);
      }
    }
    // (4) S = e^(G_last) S + (e^(G_last-G) k)^T V'
    const float eg = expf(*reinterpret_cast<const float*>(ws + ((size_t)ci * nv + h) * kWsBytes + kWsG));
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) s[mt][nt][e] *= eg;
#pragma unroll
    for (int k0 = 0; k0 < kC; k0 += 16) {
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        uint32_t a[4];
        frag_a(a, Ks, kLdC, warp * 32 + mt * 16, k0);
#pragma unroll
        for (int j = 0; j < 4; j += 2) {
          uint32_t b0[2], b1[2];
          frag_b2(b0, b1, Vt, kLdC, j * 8, k0);
          mma_bf16_16816(s[mt][j], a, b0);
          mma_bf16_16816(s[mt][j + 1], a, b1);
        }
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = warp * 32 + mt * 16 + acc_row(e), cc = cb * kCB + nt * 8 + acc_col(e);
        Sg[(size_t)r * kD + cc] = s[mt][nt][e];
      }
}

// ------------------------------------------------------------------------ gated norm
// out = (w * rmsnorm(o)) * silu(z), per (token, value head); one warp per row of 128.
__global__ void __launch_bounds__(256) gdn_gated_norm_kernel(bf16* __restrict__ out, const bf16* __restrict__ o,
                                                             const bf16* __restrict__ z, int ldz,
                                                             const float* __restrict__ w, float eps, int rows,
                                                             int nv) {
  const int gw = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (gw >= rows) return;
  const int t = gw / nv, h = gw % nv;
  const bf16* src = o + (size_t)gw * kD + lane * 4;
  const bf16* zr = z + (size_t)t * ldz + h * kD + lane * 4;
  float x[4], ss = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    x[i] = bf(src[i]);
    ss += x[i] * x[i];
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / kD + eps);
  float y[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float n = __bfloat162float(__float2bfloat16(x[i] * r));
    y[i] = n * w[lane * 4 + i] * silu(bf(zr[i]));
  }
  bf16* dst = out + (size_t)gw * kD + lane * 4;
  store_pair(dst, y[0], y[1]);
  store_pair(dst + 2, y[2], y[3]);
}

// ------------------------------------------------------------------------ decode
// One CTA of 256 threads per (value head, sequence): thread pair (2j, 2j+1) owns state column
// j, each thread 64 of its rows in registers; the row sums combine with one shuffle.
__global__ void __launch_bounds__(256) gdn_decode_kernel(bf16* __restrict__ out, const bf16* __restrict__ mixed,
                                                         int ldm, const bf16* __restrict__ z, int ldz,
                                                         const bf16* __restrict__ bb, const bf16* __restrict__ aa,
                                                         int ldab, const float* __restrict__ A_log,
                                                         const float* __restrict__ dt_bias,
                                                         const float* __restrict__ norm_w, float eps,
                                                         float* __restrict__ state, const int* __restrict__ qsl,
                                                         const int* __restrict__ slots, const int* __restrict__ init,
                                                         int nk, int nv, int num_slots, float scale, int* status) {
  constexpr int kR = kD / 2;
  const int h = blockIdx.x, b = blockIdx.y;
  const int j = threadIdx.x >> 1, half = threadIdx.x & 1, r0 = half * kR;
  const int lo = qsl[b], hi = qsl[b + 1];
  if (hi <= lo) return;
  const int slot = slots[b];
  if (slot < 0 || slot >= num_slots) {
    if (threadIdx.x == 0) record(status, kBadIndex, 50, slot);
    return;
  }
  __shared__ float qs[kD], ks[kD], red[32];
  float* Sg = state + ((size_t)slot * nv + h) * kD * kD;
  float s[kR];
  const bool has = init[b] != 0;
#pragma unroll
  for (int i = 0; i < kR; ++i) s[i] = has ? Sg[(size_t)(r0 + i) * kD + j] : 0.f;
  const int kh = h / (nv / nk);
  const float a_neg = -expf(A_log[h]), dtb = dt_bias[h], wj = norm_w[j];
  for (int t = lo; t < hi; ++t) {
    const bf16* row = mixed + (size_t)t * ldm;
    float qv = 0.f, kv = 0.f;
    if (threadIdx.x < kD) {
      qv = bf(row[kh * kD + threadIdx.x]);
      kv = bf(row[(nk + kh) * kD + threadIdx.x]);
    }
    const float sq = block_sum(qv * qv, red);
    const float sk = block_sum(kv * kv, red);
    if (threadIdx.x < kD) {
      qs[threadIdx.x] = qv * rsqrtf(sq + 1e-6f) * scale;
      ks[threadIdx.x] = kv * rsqrtf(sk + 1e-6f);
    }
    __syncthreads();
    const float vv = bf(row[(2 * nk + h) * kD + j]);
    const size_t ab = (size_t)t * ldab + h;
    const float decay = expf(a_neg * softplus(bf(aa[ab]) + dtb));
    const float beta = 1.f / (1.f + expf(-bf(bb[ab])));
    float kvm = 0.f;
#pragma unroll
    for (int i = 0; i < kR; ++i) {
      s[i] *= decay;
      kvm += s[i] * ks[r0 + i];
    }
    kvm += __shfl_xor_sync(0xffffffffu, kvm, 1);
    const float delta = (vv - kvm) * beta;
    float ov = 0.f;
#pragma unroll
    for (int i = 0; i < kR; ++i) {
      s[i] += ks[r0 + i] * delta;
      ov += s[i] * qs[r0 + i];
    }
    ov += __shfl_xor_sync(0xffffffffu, ov, 1);
    const float ob = __bfloat162float(__float2bfloat16(ov));
    const float so = block_sum(half ? 0.f : ob * ob, red);
    if (!half) {
      const float nrm = __bfloat162float(__float2bfloat16(ob * rsqrtf(so / kD + eps)));
      const float zv = bf(z[(size_t)t * ldz + h * kD + j]);
      out[(size_t)t * nv * kD + h * kD + j] = __float2bfloat16(nrm * wj * silu(zv));
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < kR; ++i) Sg[(size_t)(r0 + i) * kD + j] = s[i];
}

// ------------------------------------------------------------------------ gates
__global__ void sigmoid_gate_mul_kernel(bf16* __restrict__ out, const bf16* __restrict__ x,
                                        const bf16* __restrict__ g, int ldg, int T, int N) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)T * N) return;
  const int t = i / N, c = i % N;
  const float gv = bf(g[(size_t)t * ldg + c]);
  out[i] = __float2bfloat16(bf(x[i]) / (1.f + expf(-gv)));
}

__global__ void gated_add_kernel(bf16* __restrict__ out, const bf16* __restrict__ x, const bf16* __restrict__ y,
                                 const bf16* __restrict__ g, int ldg, int T, int N) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)T * N) return;
  const int t = i / N;
  const float gv = bf(g[(size_t)t * ldg]);
  out[i] = __float2bfloat16(bf(x[i]) + bf(y[i]) / (1.f + expf(-gv)));
}

}  // namespace dn
}  // namespace b200

using namespace b200;
using namespace b200::dn;

extern "C" {

size_t b200_gdn_workspace_bytes(int T, int B, int nv) {
  return (size_t)(T / kC + B + 1) * nv * kWsBytes + (size_t)(4 * (B + 1) + 3 * (T / kC + B + 1) + 16) * 4;
}

int b200_causal_conv1d(void* out, const void* x, int ldx, const void* w, void* conv_state, const int* qsl,
                       const int* slots, const int* init, int B, int C, int K, int max_q, int num_slots, int* status,
                       cudaStream_t s) {
  if (K != 4) return kBadShape;
  if (B == 0) return 0;
  const int seg = 64;
  const int nseg = max(1, cdiv(max_q, seg));
  dim3 grid(cdiv(C, 128), B, nseg);
  conv1d_kernel<4><<<grid, 128, 0, s>>>((bf16*)out, (const bf16*)x, ldx, (const bf16*)w, (bf16*)conv_state, qsl,
                                        slots, init, C, seg, num_slots, nseg == 1, status);
  if (nseg > 1)
    conv_state_update_kernel<4><<<dim3(cdiv(C, 128), B), 128, 0, s>>>((const bf16*)x, ldx, (bf16*)conv_state, qsl,
                                                                       slots, init, C, num_slots);
  return (int)cudaGetLastError();
}

int b200_gdn_decode(void* out, const void* mixed, int ldm, const void* z, int ldz, const void* b, const void* a,
                    int ldab, const float* A_log, const float* dt_bias, const float* norm_w, float eps, float* state,
                    const int* qsl, const int* slots, const int* init, int B, int nk, int nv, int dk, int dv,
                    int num_slots, int* status, cudaStream_t s) {
  if (dk != kD || dv != kD || nv % nk) return kBadShape;
  if (B == 0) return 0;
  gdn_decode_kernel<<<dim3(nv, B), 2 * kD, 0, s>>>((bf16*)out, (const bf16*)mixed, ldm, (const bf16*)z, ldz,
                                               (const bf16*)b, (const bf16*)a, ldab, A_log, dt_bias, norm_w, eps,
                                               state, qsl, slots, init, nk, nv, num_slots, 1.f / sqrtf((float)dk),
                                               status);
  return (int)cudaGetLastError();
}

// Chunked prefill.  `workspace` holds b200_gdn_workspace_bytes(T, B, nv) bytes (256-aligned);
// `o_tmp` is a [T, nv*dv] bf16 buffer for the pre-norm output.
int b200_gdn_prefill(void* out, void* o_tmp, const void* mixed, int ldm, const void* z, int ldz, const void* b,
                     const void* a, int ldab, const float* A_log, const float* dt_bias, const float* norm_w,
                     float eps, float* state, const int* qsl, const int* slots, const int* init, int T, int B, int nk,
                     int nv, int dk, int dv, int num_slots, void* workspace, int* status, cudaStream_t s) {
  if (dk != kD || dv != kD || nv % nk || B > 1024) return kBadShape;
  if (B == 0 || T == 0) return 0;
  const int maxC = T / kC + B + 1;
  uint8_t* ws = (uint8_t*)workspace;
  int* tab = reinterpret_cast<int*>(ws + (size_t)maxC * nv * kWsBytes);
  int* seq_off = tab + 3 * maxC;
  int* n_chunks = seq_off + B + 1;
  gdn_chunk_index_kernel<<<1, 256, 0, s>>>(seq_off, tab, n_chunks, qsl, B);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(gdn_chunk_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PrepSmem::kBytes);
    cudaFuncSetAttribute(gdn_chunk_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, ScanSmem::kBytes);
    attr = true;
  }
  gdn_chunk_prep_kernel<<<dim3(maxC, nv), 256, PrepSmem::kBytes, s>>>(
      ws, tab, n_chunks, (const bf16*)mixed, ldm, (const bf16*)b, (const bf16*)a, ldab, A_log, dt_bias, nk, nv,
      1.f / sqrtf((float)dk));
  gdn_chunk_scan_kernel<<<dim3(B, nv, kD / kCB), 128, ScanSmem::kBytes, s>>>((bf16*)o_tmp, ws, seq_off, tab, state,
                                                                             slots, init, nv, num_slots, status);
  const int rows = T * nv;
  gdn_gated_norm_kernel<<<cdiv(rows, 8), 256, 0, s>>>((bf16*)out, (const bf16*)o_tmp, (const bf16*)z, ldz, norm_w,
                                                      eps, rows, nv);
  return (int)cudaGetLastError();
}

int b200_sigmoid_gate_mul(void* out, const void* x, const void* g, int ldg, int T, int N, cudaStream_t s) {
  const size_t n = (size_t)T * N;
  if (n == 0) return 0;
  sigmoid_gate_mul_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>((bf16*)out, (const bf16*)x, (const bf16*)g,
                                                                       ldg, T, N);
  return (int)cudaGetLastError();
}

int b200_gated_add(void* out, const void* x, const void* y, const void* g, int ldg, int T, int N, cudaStream_t s) {
  const size_t n = (size_t)T * N;
  if (n == 0) return 0;
  gated_add_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>((bf16*)out, (const bf16*)x, (const bf16*)y,
                                                                (const bf16*)g, ldg, T, N);
  return (int)cudaGetLastError();
}

}  // extern "C"
