// Shared device helpers for the sm_100a kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define B200_HD __host__ __device__ __forceinline__
#define B200_D __device__ __forceinline__

namespace b200 {

// Error codes written to device status words by kernels that validate inputs or
// bound their waits, and returned by the extern "C" entry points.  A kernel never
// traps: it records the first error and skips the offending access.
//
// Return-code ranges of every entry point (disjoint, so a caller can tell them apart):
//   0              success
//   1 .. 999       a cudaError_t from the launch or a runtime call
//   1001 .. 1099   a StatusCode below (validation or bounded-wait failure)
//   2000 + r       cuTensorMapEncodeTiled failed with CUresult r
enum StatusCode : int {
  kOk = 0,
  kBadIndex = 1001,         // block id / slot / token id out of range
  kWaitTimeout = 1002,      // bounded spin on a flag gave up
  kBadShape = 1003,
  kBadAlignment = 1004,
  kScratchTooSmall = 1005,  // a fixed-size scratch array cannot hold the request
};
constexpr int kTensorMapErrorBase = 2000;
// Default limit of a bounded device-side wait (ns): long enough for any peer that is
// alive, short enough that a dead peer surfaces as kWaitTimeout instead of a hang.
constexpr unsigned long long kDefaultWaitNs = 2000000000ull;

template <typename T> B200_D float to_float(T v);
template <> B200_D float to_float<float>(float v) { return v; }
template <> B200_D float to_float<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> B200_D float to_float<__half>(__half v) { return __half2float(v); }
template <> B200_D float to_float<__nv_fp8_e4m3>(__nv_fp8_e4m3 v) { return float(v); }

template <typename T> B200_D T from_float(float v);
template <> B200_D float from_float<float>(float v) { return v; }
template <> B200_D __nv_bfloat16 from_float<__nv_bfloat16>(float v) { return __float2bfloat16(v); }
template <> B200_D __half from_float<__half>(float v) { return __float2half(v); }
template <> B200_D __nv_fp8_e4m3 from_float<__nv_fp8_e4m3>(float v) { return __nv_fp8_e4m3(v); }

B200_D float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

B200_D float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum; `red` must hold >= 32 floats of shared memory.
B200_D float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.f;
  t = warp_sum(t);
  return t;
}

B200_HD int cdiv(int a, int b) { return (a + b - 1) / b; }

// Self-checks: record (code, where, value) in status[0..2] (first error wins) and let the
// caller skip the access.  status may be null.
B200_D void record(int* status, int code, int where, int value) {
  if (status && atomicCAS(status, 0, code) == 0) {
    status[1] = where;
    status[2] = value;
  }
}
B200_D bool misaligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) != 0; }

// Programmatic dependent launch: kernels of the decode chain are launched with
// programmatic stream serialisation (launch_k below), so a kernel's CTAs may start while its
// predecessor is still finishing.  pdl_wait() blocks until the predecessor grid has completed
// and its memory is visible (a no-op when launched normally); it must precede every read of the
// predecessor's output.  pdl_trigger() lets the successor grid launch once every CTA of this
// grid has started and triggered.
B200_D void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
B200_D void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace b200
