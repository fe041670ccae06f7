// tc_args.h — argument block of the tcgen05 GEMV kernel (shared by the launcher and gemv.cu).
#pragma once
#include <stdint.h>

namespace fbfp {
struct TcArgs {
  const void* x;
  int x_dtype, m;
  int64_t ldx;
  const int8_t* ex;
  const uint16_t* sg;
  const uint2* pay;
  int64_t n_out, k_in, kb_row, npad;
  const uint32_t* entries;
  const int32_t* seg_ptr;
  const void* bias;
  int bias_dtype;
  void* y;
  int y_dtype;
  int64_t ldy;
  float* ws;
  int32_t* counters;
  int32_t* err;
  int n_stages;          // kb_row / 16
  int64_t total_units;   // ceil(npad/128) * n_stages
  int early_weights;     // 1: fetch the first weight stages before the grid-dependency wait
  // Row-parallel exchange fused into the epilogue (world > 1): y = bias + the sum over ranks of
  // their partial outputs, through the ranks' exchange buffers (exchange.cuh).
  int world, rank;
  uint8_t* xbuf[8];
  int64_t xmax;          // elements per (parity, source) slot
  int32_t* exit_count;   // CTAs of this call that have finished (in the workspace, zero between calls)
  uint64_t xchg_timeout_ns;  // bound of every wait on a peer's words (the all-reduce handle's)
};
}  // namespace fbfp
