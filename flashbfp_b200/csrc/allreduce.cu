// allreduce.cu — one-shot fp32 sum all-reduce over NVLink peer memory for the row-parallel
// exchange of tensor parallelism (o and down projections: M x 3840 fp32 partial outputs per
// rank, 15 KB at M = 1), a latency-bound size where a collective library's per-call overhead
// dominates.
//
// Each rank owns one device buffer (cudaMalloc, shared with its peers through CUDA IPC):
//   flags[2][kMaxWorld]  uint32   written by peers: flags[parity][src] = tag of src's last push
//   epoch, err           uint32   this rank's call counter (device side, so graph replays advance
//                                 it) and error word
//   data[2][kMaxWorld][max_elems] fp32: slot [parity][src] holds src's partial of that call
// A call with epoch e (parity e & 1, tag e + 1), one CTA:
//   1. push the local partial into slot [parity][rank] of every rank (peers through NVLink);
//   2. system-scope fence, then store tag into flags[parity][rank] of every rank (release);
//   3. wait (bounded) until flags[parity][q] == tag for every rank q (acquire);
//   4. y = sum over q = 0 .. world-1 of the local slots [parity][q] (fixed order: every rank gets
//      the same bits);
//   5. epoch = tag.
// Reusing a parity two calls later is safe: a rank starts call e + 2 only after it has seen every
// peer's tag for e + 1, which peers set after finishing call e (stream order). Every wait is
// bounded: after about two seconds the kernel records an error (fbfp_allreduce_check) and returns.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "common.cuh"

namespace fbfp {

constexpr int kMaxWorld = 8;
constexpr int kArThreads = 1024;
constexpr size_t kArHeader = 512;          // flags (2 x 8 x 4 B), epoch, err; 16-byte aligned data

struct ArHandle {
  int world = 0, rank = 0, device = 0;
  int64_t max_elems = 0;
  uint8_t* base = nullptr;                  // this rank's buffer
  uint8_t* peer[kMaxWorld] = {nullptr};     // every rank's buffer (self included)
  bool opened[kMaxWorld] = {false};
};

struct ArArgs {
  float* y;
  int64_t n;
  int world, rank;
  int64_t max_elems;
  uint8_t* peer[kMaxWorld];
  uint8_t* self;
};

__device__ __forceinline__ uint32_t* ar_flags(uint8_t* b) { return reinterpret_cast<uint32_t*>(b); }
__device__ __forceinline__ uint32_t* ar_epoch(uint8_t* b) { return reinterpret_cast<uint32_t*>(b + 256); }
__device__ __forceinline__ int32_t* ar_err(uint8_t* b) { return reinterpret_cast<int32_t*>(b + 260); }
__device__ __forceinline__ float* ar_slot(uint8_t* b, int64_t max_elems, uint32_t par, int src) {
  return reinterpret_cast<float*>(b + kArHeader) + ((int64_t)par * kMaxWorld + src) * max_elems;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kArThreads, 1) allreduce_sum_kernel(const ArArgs a) {
  __shared__ uint32_t s_epoch;
  __shared__ int s_fail;
  const int tid = threadIdx.x;
  if (tid == 0) { s_epoch = *ar_epoch(a.self); s_fail = 0; }
  __syncthreads();
  const uint32_t e = s_epoch, par = e & 1u, tag = e + 1u;
  const bool vec = (a.n % 4 == 0) && (a.max_elems % 4 == 0) && ((uintptr_t)a.y % 16 == 0);
  // 1. push this rank's partial into slot [par][rank] of every rank
  for (int p = 0; p < a.world; ++p) {
    float* dst = ar_slot(a.peer[p], a.max_elems, par, a.rank);
    if (vec) {
      const float4* src4 = reinterpret_cast<const float4*>(a.y);
      float4* dst4 = reinterpret_cast<float4*>(dst);
      for (int64_t i = tid; i < a.n / 4; i += kArThreads) dst4[i] = src4[i];
    } else {
      for (int64_t i = tid; i < a.n; i += kArThreads) dst[i] = a.y[i];
    }
  }
  // 2. make the pushes visible system-wide, then publish the tag to every rank
  __threadfence_system();
  __syncthreads();
  if (tid < a.world) st_release_sys(ar_flags(a.peer[tid]) + par * kMaxWorld + a.rank, tag);
  // 3. wait for every rank's tag (bounded: about two seconds)
  if (tid < a.world) {
    const uint32_t* f = ar_flags(a.self) + par * kMaxWorld + tid;
    bool ok = false;
    for (uint32_t it = 0; it < (1u << 25); ++it) {
      if (ld_acquire_sys(f) == tag) { ok = true; break; }
      if (it > 1024) __nanosleep(64);
    }
    if (!ok) {
      s_fail = 1;
      atomicExch(ar_err(a.self), 1 + tid);
    }
  }
  __syncthreads();
  if (s_fail) return;                       // the epoch stays: the handle reports the error
  // 4. sum the slots in rank order
  if (vec) {
    float4* y4 = reinterpret_cast<float4*>(a.y);
    for (int64_t i = tid; i < a.n / 4; i += kArThreads) {
      float4 acc = reinterpret_cast<const float4*>(ar_slot(a.self, a.max_elems, par, 0))[i];
      for (int q = 1; q < a.world; ++q) {
        const float4 v = reinterpret_cast<const float4*>(ar_slot(a.self, a.max_elems, par, q))[i];
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
      }
      y4[i] = acc;
    }
  } else {
    for (int64_t i = tid; i < a.n; i += kArThreads) {
      float acc = ar_slot(a.self, a.max_elems, par, 0)[i];
      for (int q = 1; q < a.world; ++q) acc += ar_slot(a.self, a.max_elems, par, q)[i];
      a.y[i] = acc;
    }
  }
  __syncthreads();
  if (tid == 0) *ar_epoch(a.self) = tag;    // 5.
}

static size_t ar_bytes(int64_t max_elems) {
  return kArHeader + sizeof(float) * 2 * kMaxWorld * (size_t)max_elems;
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
  a.y = y; a.n = n; a.world = h->world; a.rank = h->rank; a.max_elems = h->max_elems;
  for (int p = 0; p < kMaxWorld; ++p) a.peer[p] = p < h->world ? h->peer[p] : nullptr;
  a.self = h->base;
  allreduce_sum_kernel<<<1, kArThreads, 0, as_stream(stream)>>>(a);
  FBFP_LAUNCH_CHECK("allreduce_sum_kernel");
  return FBFP_OK;
}

extern "C" int fbfp_allreduce_check(void* handle, void* stream) {
  ArHandle* h = reinterpret_cast<ArHandle*>(handle);
  FBFP_CHECK_ARG(h, "null pointer");
  FBFP_CUDA_TRY(cudaStreamSynchronize(as_stream(stream)));
  int32_t err = 0;
  FBFP_CUDA_TRY(cudaMemcpy(&err, h->base + 260, sizeof(err), cudaMemcpyDeviceToHost));
  if (err) {
    const int32_t zero = 0;
    FBFP_CUDA_TRY(cudaMemcpy(h->base + 260, &zero, sizeof(zero), cudaMemcpyHostToDevice));
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
