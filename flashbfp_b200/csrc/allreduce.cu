// allreduce.cu — one-shot fp32 sum all-reduce over NVLink peer memory for the row-parallel
// exchange of tensor parallelism (o and down projections: M x 3840 fp32 partial outputs per
// rank, 15 KB at M = 1), a latency-bound size where a collective library's per-call overhead
// dominates.
//
// Low-latency protocol: every element travels as one aligned 8-byte word {value bits, tag}, so
// the value and its arrival flag land together (an aligned 8-byte store is seen whole) and no
// fence or separate flag is needed. Each rank owns one device buffer (cudaMalloc, shared with
// its peers through CUDA IPC):
//   epoch, err           uint32  this rank's call counter (device side, so graph replays advance
//                                it) and error word
//   slots[2][kMaxWorld][max_elems] {uint32 value bits, uint32 tag}: slot [parity][src] holds
//                                src's partial of the call with that parity
// A call with epoch e (parity e & 1, tag e + 1), one CTA per 8192 elements, each on its own
// contiguous chunk (the same chunks on every rank, as n is the same):
//   1. write {y[i], tag} into slot [parity][rank] of every rank (peers through NVLink);
//   2. for every element and every rank q in rank order, wait (bounded) until the local slot
//      [parity][q] carries tag, and add its value (fixed order: every rank gets the same bits);
//   3. the last CTA to finish (a counter in the header) sets epoch = tag, unless a wait gave up.
// A CTA waits only for the peers' CTAs of its own chunk, never for another CTA of its rank, so
// the chunks progress independently whatever the CTAs' residency.
// Reusing a parity two calls later is safe: a rank starts call e + 2 only after it has received
// every peer's words of call e + 1, which peers sent after finishing call e (stream order). Every
// wait is bounded (two seconds by default, fbfp_allreduce_set_timeout): then the kernel records an
// error (fbfp_allreduce_check) and the CTA returns. The buffer layout lives in exchange.cuh: the decode GEMV's fused exchange
// (fbfp_gemv_allreduce, gemv_tc.cu) uses the same buffers and the same call counter, so both
// kinds of call may be mixed on one stream, in the same order on every rank.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "common.cuh"
#include "exchange.cuh"

namespace fbfp {

constexpr int kMaxWorld = kXMaxWorld;
constexpr int kArThreads = 1024;
constexpr size_t kArHeader = kXHeader;

struct ArHandle {
  int world = 0, rank = 0, device = 0;
  int64_t max_elems = 0;
  uint64_t timeout_ns = 2000000000ull;      // bound of every wait on a peer's words
  uint8_t* base = nullptr;                  // this rank's buffer
  uint8_t* peer[kMaxWorld] = {nullptr};     // every rank's buffer (self included)
  bool opened[kMaxWorld] = {false};
};

struct ArArgs {
  float* y;
  int64_t n;
  uint64_t timeout_ns;
  int world, rank;
  int64_t max_elems;
  uint8_t* peer[kMaxWorld];
  uint8_t* self;
};

__device__ __forceinline__ uint32_t* ar_epoch(uint8_t* b) { return xchg_epoch(b); }
__device__ __forceinline__ int32_t* ar_err(uint8_t* b) { return xchg_err(b); }
// CTAs of the current call that have finished (header word 2; the last one resets it)
__device__ __forceinline__ int32_t* ar_exit(uint8_t* b) { return reinterpret_cast<int32_t*>(b + 8); }
constexpr int64_t kArChunk = 8192;
__device__ __forceinline__ uint2* ar_slot(uint8_t* b, int64_t max_elems, uint32_t par, int src) {
  return xchg_slot(b, max_elems, par, src);
}
__device__ __forceinline__ void st_word(uint2* p, uint32_t v, uint32_t tag) { xchg_store(p, v, tag); }
__device__ __forceinline__ uint2 ld_word(const uint2* p) { return xchg_load(p); }

__global__ void __launch_bounds__(kArThreads, 1) allreduce_sum_kernel(const ArArgs a) {
  __shared__ uint32_t s_epoch;
  __shared__ volatile int s_fail;
  const int tid = threadIdx.x;
  // launched with programmatic stream serialisation: y is written by the previous kernel
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  if (tid == 0) { s_epoch = *ar_epoch(a.self); s_fail = 0; }
  __syncthreads();
  const uint32_t e = s_epoch, par = e & 1u, tag = e + 1u;
  const int64_t c0 = (int64_t)blockIdx.x * kArChunk;
  const int64_t c1 = c0 + kArChunk < a.n ? c0 + kArChunk : a.n;
  // 1. push {value, tag} words into slot [par][rank] of every rank
  for (int p = 0; p < a.world; ++p) {
    uint2* dst = ar_slot(a.peer[p], a.max_elems, par, a.rank);
    for (int64_t i = c0 + tid; i < c1; i += kArThreads) st_word(dst + i, __float_as_uint(a.y[i]), tag);
  }
  // 2. receive and sum in rank order (each thread its own elements); a wait that gives up (after
  // a.timeout_ns of the global timer) sets s_fail, and every thread then skips to the barrier
  bool stop = false;
  for (int64_t i = c0 + tid; i < c1 && !stop; i += kArThreads) {
    float acc = 0.f;
    for (int q = 0; q < a.world && !stop; ++q) {
      const uint2* src = ar_slot(a.self, a.max_elems, par, q) + i;
      uint2 w = ld_word(src);
      uint64_t t0 = 0;
      for (uint32_t it = 1; w.y != tag; ++it) {
        if ((it & 63) == 0) {
          uint64_t now;
          asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
          if (t0 == 0) t0 = now;
          if (s_fail || now - t0 > a.timeout_ns) {
            if (!s_fail) { s_fail = 1; atomicExch(ar_err(a.self), 1 + q); }
            stop = true;
            break;
          }
        }
        if (it > 256) __nanosleep(64);
        w = ld_word(src);
      }
      if (stop) break;
      acc += __uint_as_float(w.x);
    }
    if (!stop) a.y[i] = acc;
  }
  __syncthreads();
  if (tid == 0) {                                        // 3.
    __threadfence();
    if (atomicAdd(ar_exit(a.self), 1) == (int)gridDim.x - 1) {
      *ar_exit(a.self) = 0;
      if (*reinterpret_cast<volatile int32_t*>(ar_err(a.self)) == 0) *ar_epoch(a.self) = tag;
    }
  }
}

static size_t ar_bytes(int64_t max_elems) {
  return kArHeader + sizeof(uint2) * 2 * kMaxWorld * (size_t)max_elems;
}

}  // namespace fbfp

using namespace fbfp;

extern "C" int fbfp_allreduce_create(int world, int rank, int64_t max_elems, void** handle,
                                     void* ipc_handle_out) {
  FBFP_CHECK_ARG(handle && ipc_handle_out, "null pointer");
  FBFP_CHECK_ARG(world >= 1 && world <= kMaxWorld && rank >= 0 && rank < world,
                 "bad world/rank (%d, %d): 1 <= world <= %d", world, rank, kMaxWorld);
  FBFP_CHECK_ARG(max_elems > 0 && max_elems <= ((int64_t)1 << 28), "bad max_elems %lld",
                 (long long)max_elems);
  ArHandle* h = new ArHandle();
  h->world = world;
  h->rank = rank;
  h->max_elems = (max_elems + 3) / 4 * 4;
  cudaError_t e = cudaGetDevice(&h->device);
  if (e == cudaSuccess) e = cudaMalloc(&h->base, ar_bytes(h->max_elems));
  if (e == cudaSuccess) e = cudaMemset(h->base, 0, ar_bytes(h->max_elems));
  cudaIpcMemHandle_t ipc;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&ipc, h->base);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (h->base) cudaFree(h->base);
    delete h;
    return set_error(FBFP_ERR_CUDA, "fbfp_allreduce_create: %s", cudaGetErrorString(e));
  }
  h->peer[rank] = h->base;
  h->opened[rank] = true;
  memcpy(ipc_handle_out, &ipc, sizeof(ipc));
  *handle = h;
  return FBFP_OK;
}

extern "C" int64_t fbfp_allreduce_ipc_handle_bytes() { return (int64_t)sizeof(cudaIpcMemHandle_t); }

namespace fbfp {
uint64_t allreduce_timeout_ns(void* handle) {
  return reinterpret_cast<ArHandle*>(handle)->timeout_ns;
}
// For the GEMV's fused exchange: the ranks' buffers of a handle whose peers are all open.
int allreduce_buffers(void* handle, uint8_t** bufs, int* world, int* rank, int64_t* max_elems) {
  ArHandle* h = reinterpret_cast<ArHandle*>(handle);
  FBFP_CHECK_ARG(h, "null all-reduce handle");
  for (int p = 0; p < h->world; ++p) {
    FBFP_CHECK_ARG(h->opened[p], "peer %d of the all-reduce handle has not been opened", p);
    bufs[p] = h->peer[p];
  }
  *world = h->world;
  *rank = h->rank;
  *max_elems = h->max_elems;
  return FBFP_OK;
}
}  // namespace fbfp

extern "C" int fbfp_allreduce_open_peer(void* handle, int peer, const void* ipc_handle) {
  ArHandle* h = reinterpret_cast<ArHandle*>(handle);
  FBFP_CHECK_ARG(h && ipc_handle, "null pointer");
  FBFP_CHECK_ARG(peer >= 0 && peer < h->world && peer != h->rank, "bad peer %d", peer);
  cudaIpcMemHandle_t ipc;
  memcpy(&ipc, ipc_handle, sizeof(ipc));
  void* p = nullptr;
  FBFP_CUDA_TRY(cudaIpcOpenMemHandle(&p, ipc, cudaIpcMemLazyEnablePeerAccess));
  h->peer[peer] = reinterpret_cast<uint8_t*>(p);
  h->opened[peer] = true;
  return FBFP_OK;
}

extern "C" int fbfp_allreduce_sum_f32(void* handle, float* y, int64_t n, void* stream) {
  ArHandle* h = reinterpret_cast<ArHandle*>(handle);
  FBFP_CHECK_ARG(h && y, "null pointer");
  FBFP_CHECK_ARG(n >= 0 && n <= h->max_elems, "n = %lld exceeds the handle's %lld elements",
                 (long long)n, (long long)h->max_elems);
  for (int p = 0; p < h->world; ++p)
    FBFP_CHECK_ARG(h->opened[p], "peer %d has not been opened", p);
  if (n == 0) return FBFP_OK;
  ArArgs a;
  a.y = y; a.n = n; a.timeout_ns = h->timeout_ns;
  a.world = h->world; a.rank = h->rank; a.max_elems = h->max_elems;
  for (int p = 0; p < kMaxWorld; ++p) a.peer[p] = p < h->world ? h->peer[p] : nullptr;
  a.self = h->base;
  // programmatic stream serialisation: the launch overlaps the previous kernel's drain; the
  // kernel waits for it (griddepcontrol.wait) before reading anything
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((n + kArChunk - 1) / kArChunk));
  cfg.blockDim = dim3(kArThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FBFP_CUDA_TRY(cudaLaunchKernelEx(&cfg, allreduce_sum_kernel, a));
  FBFP_LAUNCH_CHECK("allreduce_sum_kernel");
  return FBFP_OK;
}

extern "C" int fbfp_allreduce_set_timeout(void* handle, int64_t timeout_us) {
  ArHandle* h = reinterpret_cast<ArHandle*>(handle);
  FBFP_CHECK_ARG(h, "null pointer");
  FBFP_CHECK_ARG(timeout_us >= 1 && timeout_us <= 60000000, "timeout %lld us outside [1 us, 60 s]",
                 (long long)timeout_us);
  h->timeout_ns = (uint64_t)timeout_us * 1000ull;
  return FBFP_OK;
}

extern "C" int fbfp_allreduce_check(void* handle, void* stream) {
  ArHandle* h = reinterpret_cast<ArHandle*>(handle);
  FBFP_CHECK_ARG(h, "null pointer");
  FBFP_CUDA_TRY(cudaStreamSynchronize(as_stream(stream)));
  int32_t err = 0;
  FBFP_CUDA_TRY(cudaMemcpy(&err, h->base + 4, sizeof(err), cudaMemcpyDeviceToHost));
  if (err) {
    const int32_t zero = 0;
    FBFP_CUDA_TRY(cudaMemcpy(h->base + 4, &zero, sizeof(zero), cudaMemcpyHostToDevice));
    return set_error(FBFP_ERR_TIMEOUT, "all-reduce: rank %d gave up waiting for rank %d", h->rank,
                     (int)err - 1);
  }
  return FBFP_OK;
}

extern "C" int fbfp_allreduce_destroy(void* handle) {
  ArHandle* h = reinterpret_cast<ArHandle*>(handle);
  if (!h) return FBFP_OK;
  cudaDeviceSynchronize();
  for (int p = 0; p < h->world; ++p)
    if (p != h->rank && h->peer[p]) cudaIpcCloseMemHandle(h->peer[p]);
  if (h->base) cudaFree(h->base);
  delete h;
  return FBFP_OK;
}
