// Host-callable launchers of the sm_100a kernels.
//
// Every launcher takes raw device pointers, sizes and a stream, allocates nothing,
// and returns 0 or an error code (a cudaError_t value or a b200::StatusCode).  The
// torch bindings (bindings.cpp) validate tensors and call these.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace b200 {
enum DType : int { kF32 = 0, kF16 = 1, kBF16 = 2, kFP8E4M3 = 3, kU8 = 4, kI32 = 5, kI64 = 6 };
}

extern "C" {

int b200_rms_norm(void* out, const void* x, void* residual, const float* w, int rows, int H, float eps, int dtype,
                  cudaStream_t s);

int b200_silu_and_mul(void* out, const void* gu, int T, int I, cudaStream_t s);

int b200_embedding(void* out, const int64_t* ids, const void* table, int T, int rows, int H, int64_t vocab_start,
                   int dtype, cudaStream_t s);

int b200_rope_kv_write(void* qkv, const int64_t* positions, const float* cos_sin, void* k_cache, void* v_cache,
                       const int64_t* slot_mapping, int T, int nq, int nkv, int d, int rotary_dim, int qkv_stride,
                       int block_size, int num_blocks, float k_scale, float v_scale, const float* q_norm_w,
                       const float* k_norm_w, float norm_eps, int dtype, int cache_dtype, int* status,
                       cudaStream_t s);

int b200_paged_attention_decode(void* out, const void* q, const void* k_cache, const void* v_cache,
                                const int* block_tables, const int* seq_lens, const float* sinks, int B, int nq,
                                int nkv, int d, int q_stride, int block_size, int max_blocks, int window, float scale,
                                float k_scale, float v_scale, float* workspace, int num_splits, int dtype,
                                int cache_dtype, cudaStream_t s);

int b200_paged_attention_prefill(void* out, const void* q, const void* k_cache, const void* v_cache,
                                 const int* block_tables, const int* seq_lens, const int* query_start_loc,
                                 const float* sinks, int B, int T, int nq, int nkv, int d, int q_stride,
                                 int block_size, int max_blocks, int window, float scale, float k_scale,
                                 float v_scale, int max_query_len, int dtype, int cache_dtype, cudaStream_t s);

// Decode context parallelism: attention of one DCP shard (rank ``cp_rank`` of ``cp_size``)
// over the tokens it holds (token t on rank (t / block_size) % cp_size, stored densely in the
// same virtual blocks).  seq_lens are global lengths; windows are in global positions.  Writes
// the shard's normalised output and its natural-log LSE [tokens, nq] (-inf: no visible key);
// sinks join in the merge.
int b200_paged_attention_decode_cp(void* out, float* lse, const void* q, const void* k_cache, const void* v_cache,
                                   const int* block_tables, const int* seq_lens, int B, int nq, int nkv, int d,
                                   int q_stride, int block_size, int max_blocks, int window, float scale,
                                   float k_scale, float v_scale, float* workspace, int num_splits, int cp_rank,
                                   int cp_size, int dtype, int cache_dtype, cudaStream_t s);

int b200_paged_attention_prefill_cp(void* out, float* lse, const void* q, const void* k_cache, const void* v_cache,
                                    const int* block_tables, const int* seq_lens, const int* query_start_loc, int B,
                                    int nq, int nkv, int d, int q_stride, int block_size, int max_blocks, int window,
                                    float scale, float k_scale, float v_scale, int max_query_len, int cp_rank,
                                    int cp_size, int dtype, int cache_dtype, cudaStream_t s);

int b200_prefill_tc_supported(int d, int dtype, int cache_dtype, int block_size);

// Prefill attention on the tensor cores (tcgen05 / TMEM / TMA): head dim 64, bf16 queries and
// cache; num_blocks is the cache's block count (the TMA maps' extent).
int b200_paged_attention_prefill_tc(void* out, const void* q, const void* k_cache, const void* v_cache, int num_blocks,
                                    const int* block_tables, const int* seq_lens, const int* query_start_loc,
                                    const float* sinks, int B, int nq, int nkv, int d, int q_stride, int block_size,
                                    int max_blocks, int window, float scale, float k_scale, float v_scale,
                                    int max_query_len, int num_tokens, int dtype, int cache_dtype, int* status, cudaStream_t s);

int b200_varlen_attention(void* out, const void* q, const void* k, const void* v, const int* cu_seqlens, int B,
                          int T, int nq, int nkv, int d, float scale, int causal, int max_seqlen, int dtype,
                          cudaStream_t s);

int b200_topk_softmax(int* ids, float* weights, const void* logits, int T, int E, int k, int dtype, int full,
                      cudaStream_t s);

int b200_argmax(float* vals, int64_t* idx, const void* logits, int B, int V, int dtype, cudaStream_t s);

int b200_sample(int64_t* out, const void* logits, const float* temperature, const int* top_k, const float* top_p,
                const float* uniform, int B, int V, int max_top_k, int dtype, float* scratch, cudaStream_t s);
}
