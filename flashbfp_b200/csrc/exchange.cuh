// exchange.cuh — layout of a rank's exchange buffer for the tensor-parallel sum over NVLink peer
// memory, shared by the standalone all-reduce (allreduce.cu) and the GEMV's fused exchange
// (gemv_tc.cu). One buffer per rank (cudaMalloc, opened by the other ranks through CUDA IPC):
//   [0, 4)     epoch: the rank's call counter (device side, so graph replays advance it)
//   [4, 8)     error word
//   [256, ...) slots[2 parities][kXMaxWorld sources][max_elems] of {uint32 value bits, uint32 tag}
// A call with epoch e uses parity e & 1 and tag e + 1: every element travels as one aligned
// 8-byte word carrying its value and the tag, so the value and its arrival flag land together.
#pragma once
#include <stdint.h>

namespace fbfp {

constexpr int kXMaxWorld = 8;
constexpr size_t kXHeader = 256;

__device__ __forceinline__ uint32_t* xchg_epoch(uint8_t* b) { return reinterpret_cast<uint32_t*>(b); }
__device__ __forceinline__ int32_t* xchg_err(uint8_t* b) { return reinterpret_cast<int32_t*>(b + 4); }
__device__ __forceinline__ uint2* xchg_slot(uint8_t* b, int64_t max_elems, uint32_t par, int src) {
  return reinterpret_cast<uint2*>(b + kXHeader) + ((int64_t)par * kXMaxWorld + src) * max_elems;
}
__device__ __forceinline__ void xchg_store(uint2* p, uint32_t v, uint32_t tag) {
  asm volatile("st.relaxed.sys.global.v2.u32 [%0], {%1, %2};\n" ::"l"(p), "r"(v), "r"(tag) : "memory");
}
__device__ __forceinline__ uint2 xchg_load(const uint2* p) {
  uint2 w;
  asm volatile("ld.relaxed.sys.global.v2.u32 {%0, %1}, [%2];\n" : "=r"(w.x), "=r"(w.y) : "l"(p) : "memory");
  return w;
}

}  // namespace fbfp
