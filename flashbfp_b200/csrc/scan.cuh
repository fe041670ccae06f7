// scan.cuh — single-block exclusive scan used by the compressor and the outlier-tile build.
#pragma once
#include <stdint.h>

namespace fbfp {

// Exclusive scan of counts[0..n) in place, counts[n] = total. One block of 1024 threads.
static __global__ void __launch_bounds__(1024) scan_rows_kernel(int32_t* counts, int64_t n) {
  __shared__ int64_t part[1024];
  const int tid = threadIdx.x;
  const int64_t per = (n + 1023) / 1024;
  const int64_t lo = tid * per, hi = lo + per < n ? lo + per : n;
  int64_t s = 0;
  for (int64_t i = lo; i < hi; ++i) s += counts[i];
  part[tid] = s;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {        // Hillis-Steele inclusive scan of the partials
    int64_t add = tid >= o ? part[tid - o] : 0;
    __syncthreads();
    part[tid] += add;
    __syncthreads();
  }
  int64_t run = part[tid] - s;                 // exclusive prefix of this segment
  for (int64_t i = lo; i < hi; ++i) {
    const int32_t c = counts[i];
    counts[i] = (int32_t)run;
    run += c;
  }
  if (tid == 1023) counts[n] = (int32_t)part[1023];
}

}  // namespace fbfp
