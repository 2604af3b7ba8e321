// Host API of the MX-format mixture-of-experts kernels (moe.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace b200 {

// Scratch layout shared by the routing, quantisation, GEMM and reduce kernels.
// All buffers are caller-owned device memory; sizes from moe_workspace_sizes().
struct MoeWorkspace {
  int* offsets;      // [E_local + 1]   first permuted row of each local expert
  int* atom_base;    // [E_local + 1]   first N tile (= scale atom) of each expert
  int* cursor;       // [E_local]       scatter cursors
  int* row_route;    // [R_max]         route id (t*k + j) of each permuted row
  int* tiles;        // [2 * max_tiles] (expert, first row) of each N tile
  int* num_tiles;    // [1]
  uint8_t* xq;       // [R_max, K1p]    MXFP8 activations for GEMM1
  uint8_t* sf1;      // [atoms, K1p/128, 512]
  uint16_t* act;     // [R_max, I]      bf16 SwiGLU output
  uint8_t* aq;       // [R_max, K2p]    MXFP8 activations for GEMM2
  uint8_t* sf2;      // [atoms, K2p/128, 512]
  uint16_t* y;       // [T*k, H]        bf16 per-route expert outputs
};

struct MoeShape {
  int T, k, E_local, expert_offset;
  int H, I;     // hidden, intermediate
  int K1p, K2p; // H and I rounded up to 128
  int a_fp4;    // 1: weights e2m1 (MXFP4), 0: e4m3 (MXFP8), 2: bf16 weights and activations
  int nt;       // N tile (routes per CTA tile): 32 or 128
};

}  // namespace b200

extern "C" {
// Byte sizes of each workspace buffer, in MoeWorkspace field order (12 entries).
void b200_moe_workspace_sizes(const b200::MoeShape* shape, int64_t* sizes);

// Full MoE forward: route -> quantise -> GEMM1 (+bias, clamped SwiGLU) -> quantise ->
// GEMM2 (+bias, x affinity) -> per-token sum over this rank's experts.
int b200_moe_mx_forward(void* out, const void* x, const int* topk_ids, const float* topk_w, const void* w13,
                        const uint8_t* sf13, const float* b13, const void* w2, const uint8_t* sf2w, const float* b2,
                        const b200::MoeShape* shape, float alpha, float limit, const b200::MoeWorkspace* ws,
                        int* status, cudaStream_t s);

// out null: stop after GEMM2, leaving the per-route rows [T*k, H] in ws->y.
// Per-token sum of per-route rows over the local experts (the final step of the forward).
int b200_moe_route_sum(void* out, const void* y, const int* topk_ids, int T, int k, int E, int off, int H,
                       cudaStream_t s);

// bf16 experts: route -> gather -> GEMM1 (+bias, SwiGLU) -> GEMM2 (+bias, x affinity) -> sum.
// Weights are 128-row x 64-element tiles [E, ceil(rows/128), Kp/64, 128, 64]; shape.K1p /
// K2p are H / I rounded up to 64; shape.a_fp4 = 2.
int b200_moe_bf16_forward(void* out, const void* x, const int* topk_ids, const float* topk_w, const void* w13,
                          const float* b13, const void* w2, const float* b2, const b200::MoeShape* shape,
                          float alpha, float limit, const b200::MoeWorkspace* ws, int* status, cudaStream_t s);
}
