// Prefill / chunked-prefill attention over the paged KV cache on the Blackwell tensor cores
// (tcgen05 + TMEM + TMA), head dim 64, bf16 Q / K / V.
//
// Semantics (the reference's flash_attention / segmented_attention, functional/attention/
// attention_cte.py:188 and attention_segmented_cte.py:472, fallbacks :46 and :103): the
// queries of each sequence are its last qlen positions; query p sees cached keys j with
// j <= p (causal) and, with a sliding window W, j > p - W; per-head sink logits join the
// softmax denominator only (attention_cte.py:163-173).
//
// Design: one CTA per (128 queries, query head, sequence), 8 warps:
//   warp 0     TMA producer: K and V tiles of 128 keys straight from the paged cache (one
//              box of block_size rows per cache block, 128-byte swizzle, no multicast) into
//              a two-stage ring;
//   warp 1     allocates TMEM and issues the MMAs from one thread:
//                S(j) = Q K(j)^T   (M=128 queries, N=128 keys, K=64, fp32 in TMEM),
//                O(j) = P(j) V(j)  (M=128, N=64, K=128 keys; P from shared memory, V read
//                                   in its cache layout as an MN-major operand);
//   warps 4-7  softmax, one thread per query row: read S(j) from TMEM, mask, online max /
//              sum (exp2), write P(j) as bf16 into shared memory, then fold O(j-2) into
//              registers with its correction factor (the O tiles are produced two tiles
//              behind), and finally normalise with the sink and store.
// S and O live in two TMEM buffers each, P and K/V in two shared-memory buffers, so the
// tensor cores work on tile j+1 while the softmax threads work on tile j.  Every wait is
// bounded and records kWaitTimeout in the status word.
#include "launch.h"
#include "launch_pdl.h"
#include "tcgen05.cuh"

namespace b200 {
namespace fa {

constexpr int kBQ = 128;  // queries per CTA
constexpr int kBK = 128;  // keys per tile
constexpr int kD = 64;    // head dim (one 128-byte swizzle row of bf16)
constexpr float kLog2e = 1.4426950408889634f;

// shared memory (bytes from a 1024-aligned base)
constexpr int kOffQ = 0;                       // [128 q][64] bf16, K-major SW128
constexpr int kOffK = kOffQ + kBQ * kD * 2;    // 2 x [128 keys][64]
constexpr int kOffV = kOffK + 2 * kBK * kD * 2;
constexpr int kOffP = kOffV + 2 * kBK * kD * 2;  // 2 x [128 q][128 keys]: two 64-key atoms each
constexpr int kPBuf = kBQ * kBK * 2;
constexpr int kOffBar = kOffP + 2 * kPBuf;
constexpr int kNumBars = 12;
constexpr int kSmem = kOffBar + kNumBars * 8 + 16 + 1024;
constexpr uint32_t kTmemCols = 512;  // S: 2 x 128 columns, O: 2 x 64 columns
constexpr int kColO = 256;

struct Args {
  __nv_bfloat16* out;        // [T, nq, 64]
  const __nv_bfloat16* q;    // [T, *] rows of q_stride elements, head h at h * 64
  const int* block_tables;   // [B, max_blocks]
  const int* seq_lens;       // [B] keys in the cache after this step
  const int* qsl;            // [B + 1] query start locations
  const float* sinks;        // [nq] or null
  int nq, nkv, q_stride, bs, max_blocks, window, causal;
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

B200_D void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// kind::f16 bf16 x bf16 -> fp32, B MN-major (V in its row-per-key layout)
B200_HD uint32_t idesc_bf16_bmn(int M, int N) { return tc::idesc_f16_bf16(M, N) | (1u << 16); }

__global__ void __launch_bounds__(256, 1) fa_prefill_kernel(const __grid_constant__ CUtensorMap tmK,
                                                            const __grid_constant__ CUtensorMap tmV, Args a) {
  pdl_wait();  // predecessor output visible (programmatic dependent launch)
  pdl_trigger();
  const int qt = blockIdx.x, head = blockIdx.y, b = blockIdx.z;
  const int q0 = a.qsl[b], qlen = a.qsl[b + 1] - q0;
  if (qt * kBQ >= qlen) return;
  const int L = a.seq_lens[b];
  const int h = head / (a.nq / a.nkv);
  const int pos_base = L - qlen;  // position of query row 0 of the sequence
  const int p_first = pos_base + qt * kBQ, p_last = pos_base + min(qlen, (qt + 1) * kBQ) - 1;
  int key_lo = a.window > 0 ? max(0, p_first - a.window + 1) : 0;
  key_lo = (key_lo / kBK) * kBK;
  const int key_hi = a.causal ? min(L, p_last + 1) : L;
  const int ntiles = key_hi > key_lo ? (key_hi - key_lo + kBK - 1) / kBK : 0;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_off = tc::smem_addr(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_off & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* kv_full = bars;       // [2] K and V of a tile landed (TMA transaction count)
  uint64_t* kv_empty = bars + 2;  // [2] the MMAs reading a K/V stage are done
  uint64_t* s_full = bars + 4;    // [2] S(j) is in TMEM
  uint64_t* p_full = bars + 6;    // [2] P(j) is in shared memory (and S(j) was read)
  uint64_t* o_full = bars + 8;    // [2] O(j) is in TMEM (and P(j) was read)
  uint64_t* o_empty = bars + 10;  // [2] O(j) was read by the softmax warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&kv_full[i], 1);
      tc::mbar_init(&kv_empty[i], 1);
      tc::mbar_init(&s_full[i], 1);
      tc::mbar_init(&p_full[i], 4);  // one arrive per softmax warp
      tc::mbar_init(&o_full[i], 1);
      tc::mbar_init(&o_empty[i], 4);
    }
    tc::fence_barrier_init();
    tc::prefetch_tmap(&tmK);
    tc::prefetch_tmap(&tmV);
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, kTmemCols);
    tc::tmem_relinquish();
  }
  // Q tile: every thread moves 4 of the 128 x 8 16-byte chunks into the swizzled layout
  for (int ci = threadIdx.x; ci < kBQ * 8; ci += 256) {
    const int r = ci >> 3, c = ci & 7;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (qt * kBQ + r < qlen)
      v = *reinterpret_cast<const uint4*>(a.q + (size_t)(q0 + qt * kBQ + r) * a.q_stride + (size_t)head * kD + c * 8);
    *reinterpret_cast<uint4*>(smem + kOffQ + sw128(r, c)) = v;
  }
  fence_async_smem();  // the generic-proxy Q stores become visible to the tensor cores
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0 && ntiles > 0) {
      // ---------------- TMA producer: K / V tiles through the block table ----------------
      const int* bt = a.block_tables + (size_t)b * a.max_blocks;
      const int nblk_seq = (L + a.bs - 1) / a.bs;
      const int per_tile = kBK / a.bs;
      for (int j = 0; j < ntiles; ++j) {
        const int s = j & 1;
        if (j >= 2 && !tc::mbar_wait(&kv_empty[s], ((j - 2) >> 1) & 1, a.status)) break;
        tc::mbar_arrive_expect_tx(&kv_full[s], 2 * kBK * kD * 2);
        const int blk0 = (key_lo + j * kBK) / a.bs;
        for (int i = 0; i < per_tile; ++i) {
          const int blk = blk0 + i;
          const int bid = blk < nblk_seq ? bt[blk] : 0;  // past the sequence: the null block (masked)
          const int row = (bid * a.nkv + h) * a.bs;
          tc::tma_load_2d(smem + kOffK + s * (kBK * kD * 2) + i * a.bs * 128, &tmK, 0, row, &kv_full[s]);
          tc::tma_load_2d(smem + kOffV + s * (kBK * kD * 2) + i * a.bs * 128, &tmV, 0, row, &kv_full[s]);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && ntiles > 0) {
      // ---------------- MMA issuer ----------------
      const uint32_t id_s = tc::idesc_f16_bf16(kBQ, kBK);
      const uint32_t id_o = idesc_bf16_bmn(kBQ, kD);
      bool ok = true;
      for (int j = 0; j <= ntiles && ok; ++j) {
        if (j < ntiles) {  // S(j) = Q K(j)^T into S buffer j & 1
          const int s = j & 1;
          if (!tc::mbar_wait(&kv_full[s], (j >> 1) & 1, a.status)) break;
          if (j >= 2 && !tc::mbar_wait(&p_full[s], ((j - 2) >> 1) & 1, a.status)) break;  // S buffer read
          tc::fence_after_sync();
          const uint8_t* kt = smem + kOffK + s * (kBK * kD * 2);
#pragma unroll
          for (int ks = 0; ks < kD / 16; ++ks)
            tc::mma_f16(tmem + s * kBK, tc::desc_sw128(smem + kOffQ + ks * 32), tc::desc_sw128(kt + ks * 32), id_s,
                        ks > 0 ? 1u : 0u);
          tc::mma_commit(&s_full[s]);
        }
        if (j >= 1) {  // O(j-1) = P(j-1) V(j-1) into O buffer (j-1) & 1
          const int jj = j - 1, c = jj & 1;
          if (!tc::mbar_wait(&p_full[c], (jj >> 1) & 1, a.status)) {
            ok = false;
            break;
          }
          if (jj >= 2 && !tc::mbar_wait(&o_empty[c], ((jj - 2) >> 1) & 1, a.status)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint8_t* pt = smem + kOffP + c * kPBuf;
          const uint8_t* vt = smem + kOffV + c * (kBK * kD * 2);
#pragma unroll
          for (int ks = 0; ks < kBK / 16; ++ks)  // 16 keys per step: P along K, V rows
            tc::mma_f16(tmem + kColO + c * kD, tc::desc_sw128(pt + (ks >> 2) * (kBQ * 128) + (ks & 3) * 32),
                        tc::desc_sw128(vt + ks * 2048), id_o, ks > 0 ? 1u : 0u);
          tc::mma_commit(&o_full[c]);
          tc::mma_commit(&kv_empty[c]);  // K(j-1) and V(j-1) are no longer read
        }
      }
    }
  } else if (warp >= 4) {
    // ---------------- softmax: thread = query row (TMEM lane) ----------------
    const int ew = warp & 3;
    const int r = ew * 32 + lane;
    const int p = p_first + r;  // this row's position
    const bool row_ok = qt * kBQ + r < qlen;
    // visible keys lo_vis .. hi_vis (inclusive)
    const int lo_vis = a.window > 0 ? p - a.window + 1 : 0;
    const int hi_vis = a.causal ? min(p, L - 1) : L - 1;
    const uint32_t lane_base = tmem + ((uint32_t)(ew * 32) << 16);
    float o[kD];
#pragma unroll
    for (int i = 0; i < kD; ++i) o[i] = 0.f;
    float m = -INFINITY, l = 0.f;
    float pend[2] = {1.f, 1.f};  // correction factor of the O tile waiting in each buffer
    bool ok = true;

    auto fold_o = [&](int i) -> bool {  // o = o * corr(i) + O(i)
      const int c = i & 1;
      if (!tc::mbar_wait(&o_full[c], (i >> 1) & 1, a.status)) return false;
      tc::fence_after_sync();
      const float corr = pend[c];
      uint32_t v[kD];
      tc::tmem_ld_32x32b_x32(lane_base + kColO + c * kD, *reinterpret_cast<uint32_t(*)[32]>(v));
      tc::tmem_ld_32x32b_x32(lane_base + kColO + c * kD + 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
      tc::tmem_ld_wait();
#pragma unroll
      for (int t = 0; t < kD; ++t) o[t] = fmaf(o[t], corr, __uint_as_float(v[t]));
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&o_empty[c]);
      return true;
    };

    for (int j = 0; j < ntiles && ok; ++j) {
      const int s = j & 1;
      if (!tc::mbar_wait(&s_full[s], (j >> 1) & 1, a.status)) break;
      tc::fence_after_sync();
      const int key0 = key_lo + j * kBK;
      const uint32_t s_addr = lane_base + s * kBK;
      // the whole S row in registers (one TMEM round trip)
      float x[kBK];
#pragma unroll
      for (int cc = 0; cc < kBK; cc += 32)
        tc::tmem_ld_32x32b_x32(s_addr + cc, *reinterpret_cast<uint32_t(*)[32]>(x + cc));
      tc::tmem_ld_wait();
      // masks only where the tile crosses this row's visible range
      if (key0 < lo_vis || key0 + kBK - 1 > hi_vis) {
#pragma unroll
        for (int t = 0; t < kBK; ++t) {
          const int k = key0 + t;
          if (k < lo_vis || k > hi_vis) x[t] = -INFINITY;
        }
      }
      // masked row maximum (4 independent chains), in log2 units
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int t = 0; t < kBK; ++t) mx[t & 3] = fmaxf(mx[t & 3], x[t]);
      const float tmax = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * a.scale_log2;
      const float m_new = fmaxf(m, tmax);
      const float mref = m_new == -INFINITY ? 0.f : m_new;  // a fully masked row so far: P = 0
      const float corr = ex2(m - mref);
      // the O tile two behind is done (its P buffer is free again): fold it in
      if (j >= 2 && !fold_o(j - 2)) {
        ok = false;
        break;
      }
      // P = exp2(s * scale - m) as bf16 into the swizzled P buffer, row sum
      uint8_t* pbuf = smem + kOffP + s * kPBuf;
      float rs[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int cc = 0; cc < kBK; cc += 32) {
        uint32_t pk[16];
#pragma unroll
        for (int t = 0; t < 32; t += 2) {
          const float e0 = ex2(fmaf(x[cc + t], a.scale_log2, -mref));
          const float e1 = ex2(fmaf(x[cc + t + 1], a.scale_log2, -mref));
          rs[(t >> 1) & 3] += e0 + e1;
          const __nv_bfloat162 pr = __floats2bfloat162_rn(e0, e1);
          pk[t >> 1] = *reinterpret_cast<const uint32_t*>(&pr);
        }
        const int atom = cc >> 6;  // 64 keys (128 bytes) per swizzle atom
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const int chunk = ((cc & 63) >> 3) + q4;  // 16-byte chunk (8 keys) within the atom row
          *reinterpret_cast<uint4*>(pbuf + atom * (kBQ * 128) + sw128(r, chunk)) =
              make_uint4(pk[q4 * 4], pk[q4 * 4 + 1], pk[q4 * 4 + 2], pk[q4 * 4 + 3]);
        }
      }
      l = l * corr + ((rs[0] + rs[1]) + (rs[2] + rs[3]));
      m = m_new;
      pend[s] = corr;
      fence_async_smem();  // P stores visible to the tensor cores
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&p_full[s]);  // also: S(j) was read
    }
    // the last two O tiles
    for (int i = max(0, ntiles - 2); i < ntiles && ok; ++i)
      if (!fold_o(i)) ok = false;
    // normalise with the sink (it joins the denominator only) and store
    float f = 1.f;
    if (a.sinks != nullptr) {
      const float sk = a.sinks[head] * kLog2e;
      const float mn = fmaxf(m, sk);
      f = (m == -INFINITY) ? 0.f : ex2(m - mn);
      l = l * f + ex2(sk - mn);
    }
    const float inv = l > 0.f ? f / l * a.v_scale : 0.f;
    if (row_ok) {
      uint4* op = reinterpret_cast<uint4*>(a.out + (size_t)(q0 + qt * kBQ + r) * a.nq * kD + (size_t)head * kD);
#pragma unroll
      for (int c8 = 0; c8 < kD / 8; ++c8) {
        uint4 u;
        __nv_bfloat162* ub = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
        for (int t = 0; t < 4; ++t) ub[t] = __floats2bfloat162_rn(o[c8 * 8 + 2 * t] * inv, o[c8 * 8 + 2 * t + 1] * inv);
        op[c8] = u;
      }
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
                                               int max_query_len, int dtype, int cache_dtype, int* status,
                                               cudaStream_t s) {
  if (!b200_prefill_tc_supported(d, dtype, cache_dtype, block_size)) return kBadShape;
  if (nkv <= 0 || nq % nkv || q_stride % 8 || num_blocks <= 0) return kBadShape;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_cache) |
       reinterpret_cast<uintptr_t>(v_cache) | reinterpret_cast<uintptr_t>(out)) & 15)
    return kBadAlignment;
  if (B == 0 || max_query_len == 0) return 0;
  CUtensorMap tk, tv;
  int rc;
  if ((rc = fa::cache_map(&tk, k_cache, num_blocks, nkv, block_size))) return rc;
  if ((rc = fa::cache_map(&tv, v_cache, num_blocks, nkv, block_size))) return rc;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(fa::fa_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, fa::kSmem);
    attr = true;
  }
  fa::Args a{};
  a.out = static_cast<__nv_bfloat16*>(out);
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.block_tables = block_tables;
  a.seq_lens = seq_lens;
  a.qsl = query_start_loc;
  a.sinks = sinks;
  a.nq = nq, a.nkv = nkv, a.q_stride = q_stride, a.bs = block_size, a.max_blocks = max_blocks;
  a.window = window, a.causal = 1;
  a.scale_log2 = scale * k_scale * fa::kLog2e;
  a.v_scale = v_scale;
  a.status = status;
  dim3 grid((max_query_len + fa::kBQ - 1) / fa::kBQ, nq, B);
  launch_k(fa::fa_prefill_kernel, grid, dim3(256), fa::kSmem, s, tk, tv, a);
  return (int)cudaGetLastError();
}
