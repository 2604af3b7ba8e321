// Entry point for callers that cannot allocate device memory.
//
// This declaration has no counterpart in the reference plugin.  It serves callers of
// this library that cannot call cudaMalloc: for instance a C host runtime that links the
// library without any allocator handle, or a process whose device memory another
// component's caching allocator has already reserved in full, where an extra cudaMalloc
// would fail or stall the whole device.  The caller passes inputs and outputs only; the
// split-KV scratch is a fixed 4 MiB array inside the library (see attention.cu for the
// size limit, the once-per-device address lookup on the first call, and the rule that
// calls sharing the array must not overlap on the GPU).
#pragma once
#include <cuda_runtime.h>

extern "C" int b200_paged_attention_decode_noalloc(void* out, const void* q, const void* k_cache,
                                                   const void* v_cache, const int* block_tables, const int* seq_lens,
                                                   const float* sinks, int B, int nq, int nkv, int d, int q_stride,
                                                   int block_size, int max_blocks, int window, float scale,
                                                   float k_scale, float v_scale, int num_splits, int dtype,
                                                   int cache_dtype, cudaStream_t s);
