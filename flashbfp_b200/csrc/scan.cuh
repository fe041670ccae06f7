// scan.cuh — single-block exclusive scan used by the compressor and the outlier-tile build.
#pragma once
#include <stdint.h>

namespace fbfp {

// Exclusive scan of counts[0..n) in place, counts[n] = total. One block of 1024 threads walks
// the array in tiles of 4096 counts: each thread loads 4 consecutive counts (a warp reads 512
// contiguous bytes), a warp-shuffle scan and a scan of the 32 warp totals give every thread
// its prefix within the tile, and a running carry links the tiles.
static __global__ void __launch_bounds__(1024) scan_rows_kernel(int32_t* counts, int64_t n) {
  __shared__ long long warp_tot[32];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  long long carry = 0;
  for (int64_t base = 0; base < n; base += 4096) {
    const int64_t i0 = base + 4 * (int64_t)tid;
    int32_t v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = i0 + j < n ? counts[i0 + j] : 0;
    const long long t = (long long)v[0] + v[1] + v[2] + v[3];
    long long inc = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long y = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += y;
    }
    if (lane == 31) warp_tot[wid] = inc;
    __syncthreads();
    if (wid == 0) {
      long long w = warp_tot[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const long long y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      warp_tot[lane] = w;
    }
    __syncthreads();
    long long run = carry + (wid ? warp_tot[wid - 1] : 0) + inc - t;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (i0 + j < n) counts[i0 + j] = (int32_t)run;
      run += v[j];
    }
    carry += warp_tot[31];
    __syncthreads();                            // warp_tot is rewritten by the next tile
  }
  if (tid == 0) counts[n] = (int32_t)carry;
}

}  // namespace fbfp
