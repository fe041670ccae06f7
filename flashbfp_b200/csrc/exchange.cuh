// exchange.cuh — layout of a rank's exchange buffer for the tensor-parallel sum over NVLink peer
// memory, shared by the standalone all-reduce (allreduce.cu) and the GEMV's fused exchange
// (gemv_tc.cu). One buffer per rank (cudaMalloc, opened by the other ranks through CUDA IPC):
//   [0, 4)     epoch: the rank's call counter (device side, so graph replays advance it)
//   [4, 8)     error word
//   [256, ...) slots[2 parities][kXMaxWorld sources][max_elems] of {uint32 value bits, uint32 tag}
// A call with epoch e uses parity e & 1 and tag e + 1: every element travels as one aligned
// 8-byte word carrying its value (low 32 bits) and the tag (high 32 bits). The word is written
// and read with single 64-bit relaxed accesses, which the memory model makes single-copy
// atomic for an aligned 8-byte location, so a reader that sees the new tag also sees the new
// value (a two-element vector access would not carry that guarantee).
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
  const uint64_t w = ((uint64_t)tag << 32) | (uint64_t)v;
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;\n" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ uint2 xchg_load(const uint2* p) {
  uint64_t w;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];\n" : "=l"(w) : "l"(p) : "memory");
  return make_uint2((uint32_t)w, (uint32_t)(w >> 32));
}

}  // namespace fbfp
