// Warp-level tensor-core and async-copy helpers (inline PTX).
#pragma once
#include "common.cuh"

namespace b200 {

B200_D uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

// 16-byte async copy global->shared; src_bytes < 16 zero-fills the rest.
B200_D void cp_async16(void* smem, const void* gmem, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem), "r"(src_bytes));
}
B200_D void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
B200_D void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

B200_D void ldmatrix_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
B200_D void ldmatrix_x4_trans(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}

// D[16x8] += A[16x16] (row) * B[16x8] (col), bf16 inputs, fp32 accumulators.
B200_D void mma_bf16_16816(float* d, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

B200_D uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Offset (in 16-byte chunks) of chunk `c` of row `r` in a tile whose rows hold
// `chunks_per_row` chunks.  Rows of a multiple of 8 chunks use the XOR swizzle (chunk ^
// row mod 8), which keeps the row length and removes ldmatrix bank conflicts.  Other
// widths (e.g. head dim 72 padded to 80 = 10 chunks) use an odd row stride instead,
// `row_stride_chunks(C)`, which is conflict-free for 8-row ldmatrix reads as well; the
// XOR would push chunks past the end of such rows.
B200_HD int row_stride_chunks(int chunks_per_row) {
  return (chunks_per_row % 8 == 0) ? chunks_per_row : (chunks_per_row | 1);
}
B200_D int swz(int r, int c, int chunks_per_row) {
  if (chunks_per_row % 8 == 0) return r * chunks_per_row + (c ^ (r & 7));
  return r * row_stride_chunks(chunks_per_row) + c;
}

}  // namespace b200
