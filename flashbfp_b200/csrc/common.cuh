// common.cuh — shared helpers of libflashbfp.so (status reporting, dtype helpers).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>

#include "../../include/flashbfp.h"

namespace fbfp {

// Per-thread message for the last failed call (read through fbfp_last_error()).
int set_error(int status, const char* fmt, ...);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

#define FBFP_CHECK_ARG(cond, ...)                                   \
  do {                                                              \
    if (!(cond)) return ::fbfp::set_error(FBFP_ERR_ARG, __VA_ARGS__); \
  } while (0)

#define FBFP_CUDA_TRY(expr)                                                        \
  do {                                                                             \
    cudaError_t _e = (expr);                                                       \
    if (_e != cudaSuccess)                                                         \
      return ::fbfp::set_error(FBFP_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(_e)); \
  } while (0)

// Launch check: reports configuration errors of the launch just enqueued.
#define FBFP_LAUNCH_CHECK(name)                                                    \
  do {                                                                             \
    cudaError_t _e = cudaGetLastError();                                           \
    if (_e != cudaSuccess)                                                         \
      return ::fbfp::set_error(FBFP_ERR_CUDA, "launch of %s failed: %s", name,     \
                               cudaGetErrorString(_e));                            \
  } while (0)

// ---------------------------------------------------------------------------------
// dtype helpers
// ---------------------------------------------------------------------------------
__device__ __forceinline__ float bf16_bits_to_float(uint32_t b16) {
  return __uint_as_float(b16 << 16);
}
// fp32 -> bf16 bits, round to nearest even (finite inputs; NaN stays NaN).
__device__ __forceinline__ uint32_t float_to_bf16_bits(float f) {
  return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(f));
}
__device__ __forceinline__ float round_bf16(float f) {
  return bf16_bits_to_float(float_to_bf16_bits(f));
}
// Two values rounded to bf16 (nearest even) by one paired conversion; same results as
// round_bf16 on each.
__device__ __forceinline__ void round_bf16x2(float& a, float& b) {
  const __nv_bfloat162 h = __float22bfloat162_rn(make_float2(a, b));
  const uint32_t u = *reinterpret_cast<const uint32_t*>(&h);
  a = __uint_as_float(u << 16);
  b = __uint_as_float(u & 0xFFFF0000u);
}
__device__ __forceinline__ float load_as_float(const void* p, int dtype, int64_t i) {
  if (dtype == FBFP_F32) return reinterpret_cast<const float*>(p)[i];
  if (dtype == FBFP_BF16)
    return bf16_bits_to_float(reinterpret_cast<const uint16_t*>(p)[i]);
  return __half2float(reinterpret_cast<const __half*>(p)[i]);
}
__device__ __forceinline__ void store_from_float(void* p, int dtype, int64_t i, float v) {
  if (dtype == FBFP_F32) {
    reinterpret_cast<float*>(p)[i] = v;
  } else if (dtype == FBFP_BF16) {
    reinterpret_cast<uint16_t*>(p)[i] = (uint16_t)float_to_bf16_bits(v);
  } else {
    reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  }
}

inline bool dtype_ok(int d) { return d == FBFP_F32 || d == FBFP_BF16 || d == FBFP_F16; }
inline int dtype_size(int d) { return d == FBFP_F32 ? 4 : 2; }

// fl(m / 15) in fp32 for m = 0..15 (IEEE division, evaluated by the compiler).
#define FBFP_M15(m) ((float)(m) / 15.0f)

constexpr int kBlock = 16;         // elements per OABF block
constexpr int kChunkKb = 64;       // k-blocks per work chunk of the generic GEMV (1024 columns)
constexpr int kGroupRows = 128;    // rows per outlier group / tcgen05 row group
constexpr int kStageKb = 16;       // k-blocks per outlier stage / pipeline stage (256 columns)

}  // namespace fbfp
