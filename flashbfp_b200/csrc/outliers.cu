// outliers.cu — outlier list layout for the fused GEMV/GEMM kernels.
//
// The compressor's COO list (ascending flat index g = n*kpad + k; compressor.py:65-80)
// becomes the (r = k, c = n, v) triples of OABFLinear.load_from_weight
// (flash_bfp/triton_kernel.py:254-291), regrouped here by (128-row group, 256-column stage)
// so that the kernel working on a group/stage reads one contiguous segment:
//   entry = fp16 bits | (column within the stage) << 16 | (row within the group) << 24,
//   seg_ptr[rg * n_stages + st] .. seg_ptr[.. + 1] delimits segment (rg, st).
// Inside a segment entries are ordered by (row, column), as in the COO list.
#include "common.cuh"
#include "scan.cuh"

namespace fbfp {

struct CooView {
  const int32_t* bidx;
  const int32_t* off;
  const uint16_t* val;
  int64_t count, kpad, n_out, k_in;
};

__device__ __forceinline__ bool coo_decode(const CooView& c, int64_t i, int64_t& n, int64_t& k) {
  const int64_t gi = (int64_t)c.bidx[i] * kBlock + c.off[i];
  k = gi % c.kpad;
  n = gi / c.kpad;
  return k < c.k_in && n < c.n_out;
}

constexpr int64_t kStageCols = kStageKb * kBlock;   // 256

__global__ void outlier_hist_kernel(CooView c, int64_t n_stages, int32_t* cnt) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < c.count;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t n, k;
    if (!coo_decode(c, i, n, k)) continue;
    const int64_t rg = n / kGroupRows, r7 = n % kGroupRows, st = k / kStageCols;
    atomicAdd(cnt + (rg * n_stages + st) * kGroupRows + r7, 1);
  }
}

// Index layout (int32 words): segment pointers [0, nseg], padded to a multiple of 4 words, then
// per segment 68 words = 136 uint16: the start of each of the 128 rows within the segment
// (relative to the segment start), entry 128 = the segment size, 7 words of padding.
__host__ __device__ constexpr int64_t roff_base_words(int64_t nseg) { return (nseg + 1 + 3) & ~(int64_t)3; }
constexpr int kRoffWords = 68;

__global__ void outlier_segptr_kernel(const int32_t* dest, int64_t nseg, int32_t* seg_ptr) {
  for (int64_t s = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; s <= nseg;
       s += (int64_t)gridDim.x * blockDim.x)
    seg_ptr[s] = dest[s * kGroupRows];     // dest[nseg * 128] holds the total
  uint16_t* roff = reinterpret_cast<uint16_t*>(seg_ptr + roff_base_words(nseg));
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < nseg * 2 * kRoffWords;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t sgm = t / (2 * kRoffWords), r = t % (2 * kRoffWords);
    roff[t] = r <= kGroupRows ? (uint16_t)(dest[sgm * kGroupRows + r] - dest[sgm * kGroupRows]) : (uint16_t)0;
  }
}

__global__ void outlier_scatter_kernel(CooView c, int64_t n_stages, const int32_t* dest,
                                       uint32_t* entries) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < c.count;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t n, k;
    if (!coo_decode(c, i, n, k)) continue;
    const int64_t st = k / kStageCols;
    // first COO index of the (row n, stage st) run: binary search on the sorted flat index
    const int64_t target = n * c.kpad + st * kStageCols;
    int64_t lo = 0, hi = i;
    while (lo < hi) {
      const int64_t mid = (lo + hi) >> 1;
      const int64_t gm = (int64_t)c.bidx[mid] * kBlock + c.off[mid];
      if (gm < target) lo = mid + 1; else hi = mid;
    }
    const int64_t rg = n / kGroupRows, r7 = n % kGroupRows;
    const int64_t pos = dest[(rg * n_stages + st) * kGroupRows + r7] + (i - lo);
    const uint32_t col = (uint32_t)(k - st * kStageCols);
    entries[pos] = (uint32_t)c.val[i] | (col << 16) | ((uint32_t)r7 << 24);
  }
}

static int grid_for(int64_t work, int threads) {
  int64_t b = (work + threads - 1) / threads;
  if (b > 148 * 32) b = 148 * 32;
  return (int)(b < 1 ? 1 : b);
}

}  // namespace fbfp

using namespace fbfp;

extern "C" int64_t fbfp_outlier_tiles_scratch_bytes(int64_t npad, int64_t kpad) {
  const int64_t n_groups = (npad + kGroupRows - 1) / kGroupRows;
  const int64_t n_stages = (kpad / kBlock + kStageKb - 1) / kStageKb;
  return (int64_t)(((size_t)(n_groups * n_stages * kGroupRows + 1) * sizeof(int32_t) + 255) & ~(size_t)255);
}

extern "C" int64_t fbfp_outlier_tiles_index_words(int64_t npad, int64_t kpad) {
  const int64_t n_groups = (npad + kGroupRows - 1) / kGroupRows;
  const int64_t n_stages = (kpad / kBlock + kStageKb - 1) / kStageKb;
  const int64_t nseg = n_groups * n_stages;
  return roff_base_words(nseg) + nseg * kRoffWords;
}

extern "C" int fbfp_outlier_tiles_build(const int32_t* block_idx, const int32_t* offset,
                                        const uint16_t* value_f16, int64_t count, int64_t kpad,
                                        int64_t npad, int64_t n_out, int64_t k_in,
                                        uint32_t* entries, int32_t* seg_ptr, void* scratch,
                                        void* stream) {
  FBFP_CHECK_ARG(seg_ptr && scratch, "null pointer");
  FBFP_CHECK_ARG(count >= 0 && kpad > 0 && kpad % kBlock == 0 && npad >= n_out && n_out > 0 &&
                 k_in > 0 && k_in <= kpad, "bad shape");
  FBFP_CHECK_ARG(count == 0 || (block_idx && offset && value_f16 && entries), "null COO pointer");
  cudaStream_t st = as_stream(stream);
  const int64_t n_groups = (npad + kGroupRows - 1) / kGroupRows;
  const int64_t n_stages = (kpad / kBlock + kStageKb - 1) / kStageKb;
  const int64_t nseg = n_groups * n_stages;
  int32_t* dest = reinterpret_cast<int32_t*>(scratch);
  FBFP_CUDA_TRY(cudaMemsetAsync(dest, 0, sizeof(int32_t) * (nseg * kGroupRows + 1), st));
  CooView c{block_idx, offset, value_f16, count, kpad, n_out, k_in};
  if (count > 0) {
    outlier_hist_kernel<<<grid_for(count, 256), 256, 0, st>>>(c, n_stages, dest);
    FBFP_LAUNCH_CHECK("outlier_hist_kernel");
  }
  scan_rows_kernel<<<1, 1024, 0, st>>>(dest, nseg * kGroupRows);
  FBFP_LAUNCH_CHECK("scan_rows_kernel");
  outlier_segptr_kernel<<<grid_for(nseg + 1, 256), 256, 0, st>>>(dest, nseg, seg_ptr);
  FBFP_LAUNCH_CHECK("outlier_segptr_kernel");
  if (count > 0) {
    outlier_scatter_kernel<<<grid_for(count, 256), 256, 0, st>>>(c, n_stages, dest, entries);
    FBFP_LAUNCH_CHECK("outlier_scatter_kernel");
  }
  return FBFP_OK;
}
