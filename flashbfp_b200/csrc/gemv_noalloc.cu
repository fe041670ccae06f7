// gemv_noalloc.cu — fbfp_gemv for callers that cannot allocate device memory.
//
// fbfp_gemv needs a zero-initialised scratch workspace (fp32 partial sums of the K split,
// arrival counters and an error word). Some callers cannot provide one: a plugin living inside
// a host application that owns every byte of GPU memory through its own pool and forbids stray
// cudaMalloc calls, or a thin foreign-language binding that has no device allocator at hand.
// fbfp_gemv_noalloc serves them from a fixed array compiled into this library instead.
//
// The array below is a file-scope __device__ symbol: every GPU that loads the library holds
// kNoAllocScratchBytes of it until the process exits. In host code its name is only a
// host-side stand-in, so its device address is looked up once per device with
// cudaGetSymbolAddress (on the first call made on that device) and handed to the kernels.
#include <mutex>

#include "common.cuh"

namespace fbfp {

constexpr size_t kNoAllocScratchBytes = (size_t)8 << 20;        // 8 MiB per device
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

static void* g_noalloc_ptr[kNoAllocMaxDevices] = {nullptr};
static std::mutex g_noalloc_mutex;

// Device address of the scratch array on the current device (looked up once per device).
static int noalloc_scratch(void** out) {
  int dev = 0;
  FBFP_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return set_error(FBFP_ERR_UNSUPPORTED, "device index %d beyond %d", dev, kNoAllocMaxDevices);
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return set_error(FBFP_ERR_CUDA, "cudaGetSymbolAddress of the built-in scratch failed: %s",
                       cudaGetErrorString(e));
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return FBFP_OK;
}

}  // namespace fbfp

using namespace fbfp;

extern "C" int fbfp_gemv_noalloc(const void* x, int x_dtype, int64_t m, int64_t ldx,
                                 const int8_t* exponents, const int16_t* signs, const int32_t* payload,
                                 int64_t n_out, int64_t k_in, int64_t kpad, int64_t npad,
                                 const uint32_t* entries, const int32_t* seg_ptr, const void* bias,
                                 int bias_dtype, void* y, int y_dtype, int64_t ldy, void* stream) {
  FBFP_CHECK_ARG(m >= 1 && m <= 16, "fbfp_gemv_noalloc needs 1 <= m <= 16 (got %lld)", (long long)m);
  FBFP_CHECK_ARG(npad > 0 && npad <= ((int64_t)1 << 40), "bad npad %lld", (long long)npad);
  const int64_t need = fbfp_gemv_workspace_bytes(m, npad);
  FBFP_CHECK_ARG((size_t)need <= kNoAllocScratchBytes,
                 "fbfp_gemv_noalloc: this matrix needs %lld bytes of scratch (m=%lld, npad=%lld) but the "
                 "built-in scratch holds %zu; use fbfp_gemv with a caller workspace",
                 (long long)need, (long long)m, (long long)npad, kNoAllocScratchBytes);
  void* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc != FBFP_OK) return rc;
  // the array keeps whatever the previous call left: clear the part this call relies on
  FBFP_CUDA_TRY(cudaMemsetAsync(scratch, 0, (size_t)need, as_stream(stream)));
  return fbfp_gemv(x, x_dtype, m, ldx, exponents, signs, payload, n_out, k_in, kpad, npad, entries,
                   seg_ptr, bias, bias_dtype, y, y_dtype, ldy, scratch, stream);
}
