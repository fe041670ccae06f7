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
// host-side stand-in, so its device address is looked up with cudaGetSymbolAddress, with the
// device current, and handed to the kernels. The lookup is cached per device together with
// the CUDA context it was made in: after cudaDeviceReset, or when the application makes
// another context current on the same device, the module is loaded anew and the address is
// looked up again.
//
// The first 4 bytes of the array are the error word of a bounded device-side wait that gave up.
// Calls do not clear it: fbfp_gemv_check(NULL, stream) reports and clears it.
#include <cuda.h>

#include <mutex>

#include "common.cuh"

namespace fbfp {

constexpr size_t kNoAllocScratchBytes = (size_t)8 << 20;        // 8 MiB per device
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

struct NoAllocEntry {
  void* ctx;       // CUDA context current when the address was looked up
  void* ptr;       // device address of g_noalloc_scratch in that context
};
static NoAllocEntry g_noalloc[kNoAllocMaxDevices] = {};
static std::mutex g_noalloc_mutex;

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

static int current_context(void** ctx) {
  static CtxGetCurrentFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !p)
      return set_error(FBFP_ERR_CUDA, "cuCtxGetCurrent is not available");
    fn = reinterpret_cast<CtxGetCurrentFn>(p);
  }
  CUcontext c = nullptr;
  if (fn(&c) != CUDA_SUCCESS) return set_error(FBFP_ERR_CUDA, "cuCtxGetCurrent failed");
  *ctx = reinterpret_cast<void*>(c);
  return FBFP_OK;
}

// Device address of the scratch array on the current device (looked up once per device and
// context). Also used by fbfp_gemv_check(NULL, ...).
int noalloc_scratch(void** out) {
  int dev = 0;
  FBFP_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return set_error(FBFP_ERR_UNSUPPORTED, "device index %d beyond %d", dev, kNoAllocMaxDevices);
  // make sure the runtime has a context on this device before asking the driver for it
  FBFP_CUDA_TRY(cudaFree(nullptr));
  void* ctx = nullptr;
  int rc = current_context(&ctx);
  if (rc != FBFP_OK) return rc;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  NoAllocEntry& e = g_noalloc[dev];
  if (!e.ptr || e.ctx != ctx) {
    void* p = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (err != cudaSuccess || p == nullptr)
      return set_error(FBFP_ERR_CUDA, "cudaGetSymbolAddress of the built-in scratch failed: %s",
                       cudaGetErrorString(err));
    e.ctx = ctx;
    e.ptr = p;
  }
  *out = e.ptr;
  return FBFP_OK;
}

int gemv_validate(const void* x, int x_dtype, int64_t m, int64_t ldx, const int8_t* exponents,
                  const int16_t* signs, const int32_t* payload, int64_t n_out, int64_t k_in,
                  int64_t kpad, int64_t npad, const uint32_t* entries, const int32_t* seg_ptr,
                  const void* bias, int bias_dtype, const void* y, int y_dtype, int64_t ldy);

}  // namespace fbfp

using namespace fbfp;

extern "C" int fbfp_gemv_noalloc(const void* x, int x_dtype, int64_t m, int64_t ldx,
                                 const int8_t* exponents, const int16_t* signs, const int32_t* payload,
                                 int64_t n_out, int64_t k_in, int64_t kpad, int64_t npad,
                                 const uint32_t* entries, const int32_t* seg_ptr, const void* bias,
                                 int bias_dtype, void* y, int y_dtype, int64_t ldy, void* stream) {
  // every argument is checked before anything is enqueued on the caller's stream
  int rc = gemv_validate(x, x_dtype, m, ldx, exponents, signs, payload, n_out, k_in, kpad, npad,
                         entries, seg_ptr, bias, bias_dtype, y, y_dtype, ldy);
  if (rc != FBFP_OK) return rc;
  FBFP_CHECK_ARG(npad <= ((int64_t)1 << 40), "bad npad %lld", (long long)npad);
  const int64_t need = fbfp_gemv_workspace_bytes(m, npad);
  FBFP_CHECK_ARG((size_t)need <= kNoAllocScratchBytes,
                 "fbfp_gemv_noalloc: this matrix needs %lld bytes of scratch (m=%lld, npad=%lld) but the "
                 "built-in scratch holds %zu; use fbfp_gemv with a caller workspace",
                 (long long)need, (long long)m, (long long)npad, kNoAllocScratchBytes);
  void* scratch = nullptr;
  rc = noalloc_scratch(&scratch);
  if (rc != FBFP_OK) return rc;
  // The array keeps whatever the previous call left: clear the part this call relies on, except
  // the error word (bytes 0-3), which stays until fbfp_gemv_check(NULL, stream) reports it.
  FBFP_CUDA_TRY(cudaMemsetAsync(static_cast<unsigned char*>(scratch) + 4, 0, (size_t)need - 4,
                                as_stream(stream)));
  return fbfp_gemv(x, x_dtype, m, ldx, exponents, signs, payload, n_out, k_in, kpad, npad, entries,
                   seg_ptr, bias, bias_dtype, y, y_dtype, ldy, scratch, stream);
}
