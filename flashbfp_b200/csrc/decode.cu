// decode.cu — the non-linear work of one Gemma-3 decode token around the OABF linears: embedding,
// RMSNorms (fused with the residual add between a layer's halves), q/k RMSNorm + rotary embedding
// + KV-cache append, decode attention (GQA, optional sliding window) and the GeGLU activation.
// Every kernel reads the token and its position from device memory, so a whole token step
// (these kernels, the OABF GEMVs, lm_head and the greedy pick) replays from one CUDA graph.
// They are launched with programmatic stream serialisation: each waits for the previous kernel
// (griddepcontrol.wait) before reading anything and lets the next one launch at once, so a GEMV
// that follows starts its CTAs and fetches its weights while the small kernel runs.
//
// Arithmetic follows the Hugging Face Gemma-3 modules the reference runs around its linears
// (transformers models/gemma3/modeling_gemma3.py): RMSNorm is x * rsqrt(mean(x^2) + eps) *
// (1 + w) in fp32, rounded to bf16; the rotary embedding is q*cos + rotate_half(q)*sin with bf16
// operands and bf16 rounding after each product and the sum; the residual add is a bf16 add; the
// activation is gelu_tanh(gate) rounded to bf16, times up. Attention runs in fp32 (scores,
// softmax and the weighted sum) and rounds its output to bf16.
#include <cuda_bf16.h>

#include "common.cuh"
#include "sm100.cuh"

namespace fbfp {

typedef __nv_bfloat16 bf16;

__device__ __forceinline__ float bfr(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
__device__ __forceinline__ float ldb(const bf16* p) { return __bfloat162float(*p); }

// Sum over the block (blockDim a multiple of 32, at most 1024); `red` holds 33 floats.
__device__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float t = lane < nw ? red[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (lane == 0) red[32] = t;
  }
  __syncthreads();
  return red[32];
}

__device__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float t = lane < nw ? red[lane] : -INFINITY;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
    if (lane == 0) red[32] = t;
  }
  __syncthreads();
  return red[32];
}

constexpr int kNormThreads = 512;

__device__ __forceinline__ void pdl_prologue() {
  sm100::grid_dependency_wait();
  sm100::grid_launch_dependents();
}

// Launch with programmatic stream serialisation (see the top of this file).
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Row r of every kernel below is the token at position *pos + r (M rows: a prompt chunk, or
// one token when decoding).

// x[r] = bf16(table[tok[r]] * scale) (Gemma's scaled embedding: both operands bf16).
__global__ void embed_kernel(const int64_t* tok, const bf16* table, int64_t vocab, int hidden,
                             float scale, bf16* out, int32_t* err) {
  pdl_prologue();
  const int r = blockIdx.y;
  int64_t t = tok[r];
  if (t < 0 || t >= vocab) {
    if (threadIdx.x == 0 && blockIdx.x == 0) atomicExch(err, 1);
    t = 0;
  }
  const float s = bfr(scale);
  bf16* o = out + (int64_t)r * hidden;
  for (int d = blockIdx.x * blockDim.x + threadIdx.x; d < hidden; d += gridDim.x * blockDim.x)
    o[d] = __float2bfloat16_rn(ldb(table + t * hidden + d) * s);
}

// y[r] = bf16(x[r] * rsqrt(mean(x[r]^2) + eps) * (1 + w)); one CTA per row.
__global__ void rmsnorm_kernel(const bf16* x, const bf16* w, float eps, int hidden, bf16* y) {
  pdl_prologue();
  extern __shared__ float sh[];                  // hidden values, then 33 for the reduction
  float* red = sh + hidden;
  const int64_t off = (int64_t)blockIdx.x * hidden;
  float ss = 0.f;
  for (int d = threadIdx.x; d < hidden; d += blockDim.x) {
    const float v = ldb(x + off + d);
    sh[d] = v;
    ss += v * v;
  }
  const float r = rsqrtf(block_sum(ss, red) / (float)hidden + eps);
  for (int d = threadIdx.x; d < hidden; d += blockDim.x)
    y[off + d] = __float2bfloat16_rn(sh[d] * r * (1.f + ldb(w + d)));
}

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

// Vectorised forms of the two norm kernels for hidden a multiple of 8 and at most
// 8 * kNormThreads * NV: every thread keeps its NV groups of 8 values in registers (one 16-byte
// load each), so a row is read once and reduced once per RMSNorm (one shuffle tree, one barrier).
__device__ __forceinline__ float row_sum_fast(float v, float* red) {
  constexpr int nw = kNormThreads / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < nw; ++w) t += red[w];
  return t;
}

__device__ __forceinline__ void load8(const bf16* p, float (&f)[8]) {
  unpack8(*reinterpret_cast<const uint4*>(p), f);
}

__device__ __forceinline__ void store8(bf16* p, const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(f[2 * i]));
    const uint32_t hi = __bfloat16_as_ushort(__float2bfloat16_rn(f[2 * i + 1]));
    w[i] = lo | (hi << 16);
  }
  *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}

template <int NV>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_vec_kernel(const bf16* x, const bf16* w, float eps,
                                                                    int hidden, bf16* y) {
  pdl_prologue();
  __shared__ float red[kNormThreads / 32];
  const int64_t off = (int64_t)blockIdx.x * hidden;
  float v[NV][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int d = (threadIdx.x + i * kNormThreads) * 8;
    if (d < hidden) {
      load8(x + off + d, v[i]);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += v[i][e] * v[i][e];
    }
  }
  const float r = rsqrtf(row_sum_fast(ss, red) / (float)hidden + eps);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int d = (threadIdx.x + i * kNormThreads) * 8;
    if (d < hidden) {
      float wv[8], o[8];
      load8(w + d, wv);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = v[i][e] * r * (1.f + wv[e]);
      store8(y + off + d, o);
    }
  }
}

template <int NV>
__global__ void __launch_bounds__(kNormThreads) post_residual_pre_vec_kernel(
    const bf16* y, const bf16* w_post, bf16* resid, const bf16* w_pre, float eps, int hidden, bf16* x_next) {
  pdl_prologue();
  __shared__ float red[2][kNormThreads / 32];
  const int64_t off = (int64_t)blockIdx.x * hidden;
  float v[NV][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int d = (threadIdx.x + i * kNormThreads) * 8;
    if (d < hidden) {
      load8(y + off + d, v[i]);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += v[i][e] * v[i][e];
    }
  }
  const float r1 = rsqrtf(row_sum_fast(ss, red[0]) / (float)hidden + eps);
  float hs = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int d = (threadIdx.x + i * kNormThreads) * 8;
    if (d < hidden) {
      float wv[8], rv[8];
      load8(w_post + d, wv);
      load8(resid + off + d, rv);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float h = bfr(rv[e] + bfr(v[i][e] * r1 * (1.f + wv[e])));
        v[i][e] = h;
        hs += h * h;
      }
      store8(resid + off + d, v[i]);
    }
  }
  const float r2 = rsqrtf(row_sum_fast(hs, red[1]) / (float)hidden + eps);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int d = (threadIdx.x + i * kNormThreads) * 8;
    if (d < hidden) {
      float wv[8], o[8];
      load8(w_pre + d, wv);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = v[i][e] * r2 * (1.f + wv[e]);
      store8(x_next + off + d, o);
    }
  }
}

// Between a layer's halves, per row: h = bf16(resid + post_norm(y)); resid = h;
// x_next = pre_norm(h). One CTA per row.
__global__ void post_residual_pre_kernel(const bf16* y, const bf16* w_post, bf16* resid,
                                         const bf16* w_pre, float eps, int hidden, bf16* x_next) {
  pdl_prologue();
  extern __shared__ float sh[];
  float* red = sh + hidden;
  const int64_t off = (int64_t)blockIdx.x * hidden;
  float ss = 0.f;
  for (int d = threadIdx.x; d < hidden; d += blockDim.x) {
    const float v = ldb(y + off + d);
    sh[d] = v;
    ss += v * v;
  }
  const float r1 = rsqrtf(block_sum(ss, red) / (float)hidden + eps);
  float hs = 0.f;
  for (int d = threadIdx.x; d < hidden; d += blockDim.x) {
    const float n1 = bfr(sh[d] * r1 * (1.f + ldb(w_post + d)));
    const float h = bfr(ldb(resid + off + d) + n1);
    resid[off + d] = __float2bfloat16_rn(h);
    sh[d] = h;
    hs += h * h;
  }
  const float r2 = rsqrtf(block_sum(hs, red) / (float)hidden + eps);
  for (int d = threadIdx.x; d < hidden; d += blockDim.x)
    x_next[off + d] = __float2bfloat16_rn(sh[d] * r2 * (1.f + ldb(w_pre + d)));
}

// One CTA per (head, row) of the fused q|k|v rows: q heads 0..nh-1, then k heads. RMSNorm over
// the head, rotary embedding at the row's position (cos/sin rows of bf16 tables), then q to
// q_out [row][nh][hd] and k (with the matching v head, not normalised) appended to the cache.
__global__ void qk_rope_cache_kernel(const bf16* qkv, int nh, int nkv, int hd, const bf16* qnw,
                                     const bf16* knw, float eps, const bf16* cos_t, const bf16* sin_t,
                                     const int32_t* pos_p, int max_ctx, bf16* q_out, bf16* kc, bf16* vc,
                                     int32_t* err) {
  pdl_prologue();
  extern __shared__ float sh[];                  // hd normalised values, then 33
  float* red = sh + hd;
  const int head = blockIdx.x, row = blockIdx.y;
  const bool is_q = head < nh;
  const int p = *pos_p + row;
  if (p < 0 || p >= max_ctx) {
    if (threadIdx.x == 0) atomicExch(err, 2);
    return;
  }
  const int64_t qkv_row = (int64_t)row * (nh + 2 * nkv) * hd;
  const bf16* x = qkv + qkv_row + (int64_t)head * hd;
  const bf16* w = is_q ? qnw : knw;
  float ss = 0.f;
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    const float v = ldb(x + d);
    sh[d] = v;
    ss += v * v;
  }
  const float r = rsqrtf(block_sum(ss, red) / (float)hd + eps);
  for (int d = threadIdx.x; d < hd; d += blockDim.x) sh[d] = bfr(sh[d] * r * (1.f + ldb(w + d)));
  __syncthreads();
  const int half = hd / 2;
  const bf16* cr = cos_t + (int64_t)p * hd;
  const bf16* sr = sin_t + (int64_t)p * hd;
  const int kvh = head - nh;
  bf16* dst = is_q ? q_out + ((int64_t)row * nh + head) * hd : kc + ((int64_t)kvh * max_ctx + p) * hd;
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    const float rot = d < half ? -sh[d + half] : sh[d - half];
    const float v = bfr(bfr(sh[d] * ldb(cr + d)) + bfr(rot * ldb(sr + d)));
    dst[d] = __float2bfloat16_rn(v);
  }
  if (!is_q) {
    const bf16* vsrc = qkv + qkv_row + (int64_t)(nh + nkv + kvh) * hd;
    bf16* vdst = vc + ((int64_t)kvh * max_ctx + p) * hd;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) vdst[d] = vsrc[d];
  }
}

// One CTA per (query head, row): scores over the cached positions [lo, p] of the row's position
// p (lo = p - window + 1 for a sliding layer; causal, so a prompt row sees only its prefix),
// softmax and the weighted sum of values, all in fp32. A lane owns 8 consecutive dims (one
// 16-byte load of a cache row; head_dim <= 256, a multiple of 8); warp w takes the positions
// j = w (mod warps) for both the scores and the weighted sum, whose per-warp partial rows are
// added in shared memory at the end.
constexpr int kAttnThreads = 256;

__global__ void __launch_bounds__(kAttnThreads)
decode_attention_kernel(const bf16* q, const bf16* kc, const bf16* vc, int nh, int nkv, int hd,
                        int max_ctx, const int32_t* pos_p, int window, float scaling, bf16* out) {
  pdl_prologue();
  constexpr int nw = kAttnThreads / 32;
  extern __shared__ float sh[];                  // scores (max_ctx), partial rows (nw x hd), 33
  float* sc = sh;
  float* po = sc + max_ctx;
  float* red = po + nw * hd;
  const int head = blockIdx.x, row = blockIdx.y, kvh = head / (nh / nkv);
  const int p = *pos_p + row;
  if (p < 0 || p >= max_ctx) return;             // reported by the cache-append kernel
  const int lo = (window > 0 && p - window + 1 > 0) ? p - window + 1 : 0;
  const int n = p - lo + 1;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bool act = lane * 8 < hd;
  const int64_t qo = ((int64_t)row * nh + head) * hd;
  float qv[8];
  if (act) unpack8(*reinterpret_cast<const uint4*>(q + qo + lane * 8), qv);
  const bf16* kb = kc + ((int64_t)kvh * max_ctx + lo) * hd + lane * 8;
  const bf16* vb = vc + ((int64_t)kvh * max_ctx + lo) * hd + lane * 8;
#pragma unroll 4
  for (int j = warp; j < n; j += nw) {
    float acc = 0.f;
    if (act) {
      float kv[8];
      unpack8(*reinterpret_cast<const uint4*>(kb + (int64_t)j * hd), kv);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc += qv[i] * kv[i];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) sc[j] = acc * scaling;
  }
  __syncthreads();
  float m = -INFINITY;
  for (int j = threadIdx.x; j < n; j += blockDim.x) m = fmaxf(m, sc[j]);
  m = block_max(m, red);
  float s = 0.f;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const float e = __expf(sc[j] - m);
    sc[j] = e;
    s += e;
  }
  const float inv = 1.f / block_sum(s, red);     // ends with a barrier: every sc[j] is final
  float o8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (act) {
#pragma unroll 4
    for (int j = warp; j < n; j += nw) {
      float vv[8];
      unpack8(*reinterpret_cast<const uint4*>(vb + (int64_t)j * hd), vv);
      const float pj = sc[j];
#pragma unroll
      for (int i = 0; i < 8; ++i) o8[i] += pj * vv[i];
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) po[warp * hd + lane * 8 + i] = o8[i];
  }
  __syncthreads();
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < nw; ++w) acc += po[w * hd + d];
    out[qo + d] = __float2bfloat16_rn(acc * inv);
  }
}

// Decode attention for one new token per sequence (row r = sequence r of a batch, at its own
// position pos[r], with its own caches at seq_stride elements from the previous sequence's), with
// the q/k RMSNorm, the rotary embedding and the KV-cache append of fbfp_qk_rope_cache folded in,
// and split over positions: CTA (head, row, split) covers the cached positions
// [split * kFaChunk, (split + 1) * kFaChunk) of the row's window [lo, p]. It loads its cached
// keys and values first (the loads overlap the norms); every warp normalises and rotates the
// query head in registers; in the CTAs whose range holds p every warp also computes the new key
// and value (one warp of the first query head of each KV group writes them to the cache) and
// uses them from registers. Each CTA writes its
// softmax partial (max, sum, weighted values) to scratch; the last of a (head, row)'s CTAs to
// finish (an atomic count) merges them and returns the counter to zero for the next launch.
// Same arithmetic as the two separate kernels (bf16 roundings of the norm and the rotation, fp32
// scores and softmax), up to the order of the fp32 sums.
constexpr int kFaThreads = 256;
constexpr int kFaChunk = 64;

// One warp: RMSNorm (weights 1 + w) and rotation of one head of hd (a multiple of 16, at most
// 256) values of a fused q|k|v row, lane l owning dims 8l .. 8l + 7 (lanes past hd / 8 hold
// zeros): the sum of squares is a warp reduction, and the rotation's partner of dim d (d +- hd/2)
// sits hd / 16 lanes away. Rounded to bf16 where the separate kernel rounds: the normalised
// value, each product, their sum.
__device__ __forceinline__ void fa_warp_norm_rope(const bf16* x, const bf16* w, float eps, int hd,
                                                  const bf16* cr, const bf16* sr, float (&v)[8]) {
  const int lane = threadIdx.x & 31;
  const bool act = lane * 8 < hd;
  float xv[8], wv[8], t[8];
  if (act) {
    unpack8(*reinterpret_cast<const uint4*>(x + lane * 8), xv);
    unpack8(*reinterpret_cast<const uint4*>(w + lane * 8), wv);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) xv[i] = wv[i] = 0.f;
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss += xv[i] * xv[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = rsqrtf(ss / (float)hd + eps);
#pragma unroll
  for (int i = 0; i < 8; ++i) t[i] = bfr(xv[i] * r * (1.f + wv[i]));
  const int hl = hd >> 4;                         // lanes per half of the head
  const bool lo_half = lane < hl;
  const int partner = lo_half ? lane + hl : lane - hl;
  float cv[8], sv[8];
  if (act) {
    unpack8(*reinterpret_cast<const uint4*>(cr + lane * 8), cv);
    unpack8(*reinterpret_cast<const uint4*>(sr + lane * 8), sv);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) cv[i] = sv[i] = 0.f;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float pv = __shfl_sync(0xffffffffu, t[i], partner & 31);
    const float rot = lo_half ? -pv : pv;
    v[i] = act ? bfr(bfr(t[i] * cv[i]) + bfr(rot * sv[i])) : 0.f;
  }
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void __launch_bounds__(kFaThreads)
decode_attention_step_kernel(const bf16* qkv, int nh, int nkv, int hd, const bf16* qnw, const bf16* knw,
                             float eps, const bf16* cos_t, const bf16* sin_t, const int32_t* pos, int max_ctx,
                             bf16* kc, bf16* vc, int64_t seq_stride, int window, float scaling, int n_splits,
                             float* part, int* counters, bf16* out, int32_t* err) {
  pdl_prologue();
  constexpr int nw = kFaThreads / 32;
  constexpr int per_warp = kFaChunk / nw;
  extern __shared__ float sh[];      // scores (kFaChunk), per-warp partial rows (nw x hd)
  float* sc = sh;
  float* po = sc + kFaChunk;
  __shared__ int s_last;
  const int head = blockIdx.x, row = blockIdx.y, split = blockIdx.z, rows = gridDim.y;
  const int group = nh / nkv, kvh = head / group;
  const int p = pos[row];
  if (p < 0 || p >= max_ctx) {                   // the whole row is skipped (no CTA counts)
    if (threadIdx.x == 0 && head == 0 && split == 0) atomicExch(err, 2);
    return;
  }
  const int lo = (window > 0 && p - window + 1 > 0) ? p - window + 1 : 0;
  // the ranges that hold positions of the row's window: the others have nothing to do and are
  // not counted; a row with one such range writes its output without a merge
  const int s_lo = lo / kFaChunk, s_hi = p / kFaChunk;
  if (split < s_lo || split > s_hi) return;
  const bool single = s_lo == s_hi;
  const int c0 = max(lo, split * kFaChunk), c1 = min(p + 1, (split + 1) * kFaChunk);
  float* mine = part + (((int64_t)head * rows + row) * n_splits + split) * (hd + 2);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  {
    const bf16* xrow = qkv + (int64_t)row * (nh + 2 * nkv) * hd;
    const bf16* cr = cos_t + (int64_t)p * hd;
    const bf16* sr = sin_t + (int64_t)p * hd;
    bf16* kbase = kc + row * seq_stride + (int64_t)kvh * max_ctx * hd;
    bf16* vbase = vc + row * seq_stride + (int64_t)kvh * max_ctx * hd;
    const bool act = lane * 8 < hd;
    // the cached keys and values of this range first: their loads overlap the norms below
    // (warp w takes positions c0 + w + nw * i)
    uint4 kr[per_warp], vr[per_warp];
#pragma unroll
    for (int i = 0; i < per_warp; ++i) {
      const int j = c0 + warp + nw * i;
      const bool ld = act && j < c1 && j != p;
      kr[i] = ld ? *reinterpret_cast<const uint4*>(kbase + (int64_t)j * hd + lane * 8) : make_uint4(0, 0, 0, 0);
      vr[i] = ld ? *reinterpret_cast<const uint4*>(vbase + (int64_t)j * hd + lane * 8) : make_uint4(0, 0, 0, 0);
    }
    // every warp normalises and rotates the query head itself (registers, no block barrier)
    float q8[8];
    fa_warp_norm_rope(xrow + (int64_t)head * hd, qnw, eps, hd, cr, sr, q8);
    float kn8[8], vn8[8];
    const bool has_new = c1 == p + 1;
    if (has_new) {
      fa_warp_norm_rope(xrow + (int64_t)(nh + kvh) * hd, knw, eps, hd, cr, sr, kn8);
      const bf16* vsrc = xrow + (int64_t)(nh + nkv + kvh) * hd;
      uint4 vraw = make_uint4(0, 0, 0, 0);
      if (act) vraw = *reinterpret_cast<const uint4*>(vsrc + lane * 8);
      unpack8(vraw, vn8);
      if (head % group == 0 && warp == 0 && act) {   // the cache append, once per KV head
        store8(kbase + (int64_t)p * hd + lane * 8, kn8);
        *reinterpret_cast<uint4*>(vbase + (int64_t)p * hd + lane * 8) = vraw;
      }
    }
#pragma unroll
    for (int i = 0; i < per_warp; ++i) {
      const int j = c0 + warp + nw * i;
      float kv[8];
      if (j == p) {
#pragma unroll
        for (int e = 0; e < 8; ++e) kv[e] = kn8[e];
      } else {
        unpack8(kr[i], kv);
      }
      float acc = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc += q8[e] * kv[e];
      acc = warp_sum(acc);
      if (lane == 0 && j < c1) sc[j - c0] = acc * scaling;
    }
    __syncthreads();
    // every warp: max and sum of the range's (at most 64) scores, two per lane
    const int n = c1 - c0;
    const float s0 = lane < n ? sc[lane] : -INFINITY;
    const float s1 = lane + 32 < n ? sc[lane + 32] : -INFINITY;
    const float m = warp_max(fmaxf(s0, s1));
    const float l = warp_sum((lane < n ? __expf(s0 - m) : 0.f) + (lane + 32 < n ? __expf(s1 - m) : 0.f));
    float o8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < per_warp; ++i) {
      const int j = c0 + warp + nw * i;
      if (j >= c1) continue;
      float vv[8];
      if (j == p) {
#pragma unroll
        for (int e = 0; e < 8; ++e) vv[e] = vn8[e];
      } else {
        unpack8(vr[i], vv);
      }
      const float pj = __expf(sc[j - c0] - m);
#pragma unroll
      for (int e = 0; e < 8; ++e) o8[e] += pj * vv[e];
    }
    if (act) {
#pragma unroll
      for (int e = 0; e < 8; ++e) po[warp * hd + lane * 8 + e] = o8[e];
    }
    __syncthreads();
    bf16* orow = out + ((int64_t)row * nh + head) * hd;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
      float acc = 0.f;
#pragma unroll
      for (int w = 0; w < nw; ++w) acc += po[w * hd + d];
      if (single) orow[d] = __float2bfloat16_rn(acc * (1.f / l));
      else mine[2 + d] = acc;
    }
    if (single) return;
    if (threadIdx.x == 0) { mine[0] = m; mine[1] = l; }
  }
  // the last CTA of (head, row) merges the partials of ranges s_lo .. s_hi
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(counters + head * rows + row, 1) == s_hi - s_lo;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const float* base = part + ((int64_t)head * rows + row) * n_splits * (hd + 2);
  float M = -INFINITY;
  for (int s2 = s_lo; s2 <= s_hi; ++s2) M = fmaxf(M, __ldcg(base + (int64_t)s2 * (hd + 2)));
  float L = 0.f;
  for (int s2 = s_lo; s2 <= s_hi; ++s2) {
    const float* ps = base + (int64_t)s2 * (hd + 2);
    L += __ldcg(ps + 1) * __expf(__ldcg(ps) - M);
  }
  const float inv = 1.f / L;
  bf16* orow = out + ((int64_t)row * nh + head) * hd;
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float acc = 0.f;
    for (int s2 = s_lo; s2 <= s_hi; ++s2) {
      const float* ps = base + (int64_t)s2 * (hd + 2);
      acc += __ldcg(ps + 2 + d) * __expf(__ldcg(ps) - M);
    }
    orow[d] = __float2bfloat16_rn(acc * inv);
  }
  if (threadIdx.x == 0) counters[head * rows + row] = 0;
}

__global__ void advance_rows_kernel(int32_t* pos, int b) {
  pdl_prologue();
  if ((int)threadIdx.x < b) pos[threadIdx.x] += 1;
}

// out[r][i] = bf16(bf16(gelu_tanh(gate[r][i])) * up[r][i]) for the fused rows [gate (I) | up (I)].
__global__ void geglu_kernel(const bf16* gu, int64_t inter, int64_t total, bf16* out) {
  pdl_prologue();
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;    // sqrt(2/pi), tanh-GELU cubic
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / inter, c = i - r * inter;
    const float x = ldb(gu + 2 * inter * r + c);
    const float g = bfr(0.5f * x * (1.f + tanhf(k0 * (x + k1 * x * x * x))));
    out[i] = __float2bfloat16_rn(g * ldb(gu + 2 * inter * r + inter + c));
  }
}

__global__ void advance_kernel(int32_t* pos, int m) {
  pdl_prologue();
  *pos += m;
}

}  // namespace fbfp

using namespace fbfp;

extern "C" int fbfp_embed(const int64_t* tok, int64_t m, const void* table, int64_t vocab, int64_t hidden,
                          float scale, void* out, int32_t* err, void* stream) {
  FBFP_CHECK_ARG(tok && table && out && err && vocab > 0 && hidden > 0, "bad arguments");
  FBFP_CHECK_ARG(m >= 1 && m <= 65535, "m must be in [1, 65535]");
  const int blocks = (int)((hidden + 255) / 256);
  FBFP_CUDA_TRY(launch_pdl(embed_kernel, dim3(blocks, (unsigned)m), dim3(256), 0, as_stream(stream), tok,
                           reinterpret_cast<const bf16*>(table), vocab, (int)hidden, scale,
                           reinterpret_cast<bf16*>(out), err));
  FBFP_LAUNCH_CHECK("embed_kernel");
  return FBFP_OK;
}

extern "C" int fbfp_rmsnorm(const void* x, int64_t m, const void* w, float eps, int64_t hidden, void* y,
                            void* stream) {
  FBFP_CHECK_ARG(x && w && y && hidden > 0 && hidden <= 12000, "bad arguments (hidden <= 12000)");
  FBFP_CHECK_ARG(m >= 1 && m <= 65535, "m must be in [1, 65535]");
  const int nv = (int)((hidden + 8 * kNormThreads - 1) / (8 * kNormThreads));
  if (hidden % 8 == 0 && nv <= 3 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)w & 15) == 0 && ((uintptr_t)y & 15) == 0) {
    auto k = nv == 1 ? rmsnorm_vec_kernel<1> : nv == 2 ? rmsnorm_vec_kernel<2> : rmsnorm_vec_kernel<3>;
    FBFP_CUDA_TRY(launch_pdl(k, dim3((unsigned)m), dim3(kNormThreads), 0, as_stream(stream),
                             reinterpret_cast<const bf16*>(x), reinterpret_cast<const bf16*>(w), eps, (int)hidden,
                             reinterpret_cast<bf16*>(y)));
    FBFP_LAUNCH_CHECK("rmsnorm_vec_kernel");
    return FBFP_OK;
  }
  const size_t smem = sizeof(float) * ((size_t)hidden + 33);
  FBFP_CUDA_TRY(launch_pdl(rmsnorm_kernel, dim3((unsigned)m), dim3(kNormThreads), smem, as_stream(stream),
                           reinterpret_cast<const bf16*>(x), reinterpret_cast<const bf16*>(w), eps, (int)hidden,
                           reinterpret_cast<bf16*>(y)));
  FBFP_LAUNCH_CHECK("rmsnorm_kernel");
  return FBFP_OK;
}

extern "C" int fbfp_post_residual_norm(const void* y, int64_t m, const void* w_post, void* resid,
                                       const void* w_pre, float eps, int64_t hidden, void* x_next,
                                       void* stream) {
  FBFP_CHECK_ARG(y && w_post && resid && w_pre && x_next && hidden > 0 && hidden <= 12000,
                 "bad arguments (hidden <= 12000)");
  FBFP_CHECK_ARG(m >= 1 && m <= 65535, "m must be in [1, 65535]");
  const int nv = (int)((hidden + 8 * kNormThreads - 1) / (8 * kNormThreads));
  if (hidden % 8 == 0 && nv <= 3 && ((uintptr_t)y & 15) == 0 && ((uintptr_t)w_post & 15) == 0 &&
      ((uintptr_t)resid & 15) == 0 && ((uintptr_t)w_pre & 15) == 0 && ((uintptr_t)x_next & 15) == 0) {
    auto k = nv == 1 ? post_residual_pre_vec_kernel<1>
                     : nv == 2 ? post_residual_pre_vec_kernel<2> : post_residual_pre_vec_kernel<3>;
    FBFP_CUDA_TRY(launch_pdl(k, dim3((unsigned)m), dim3(kNormThreads), 0, as_stream(stream),
                             reinterpret_cast<const bf16*>(y), reinterpret_cast<const bf16*>(w_post),
                             reinterpret_cast<bf16*>(resid), reinterpret_cast<const bf16*>(w_pre), eps, (int)hidden,
                             reinterpret_cast<bf16*>(x_next)));
    FBFP_LAUNCH_CHECK("post_residual_pre_vec_kernel");
    return FBFP_OK;
  }
  const size_t smem = sizeof(float) * ((size_t)hidden + 33);
  FBFP_CUDA_TRY(launch_pdl(post_residual_pre_kernel, dim3((unsigned)m), dim3(kNormThreads), smem,
                           as_stream(stream), reinterpret_cast<const bf16*>(y),
                           reinterpret_cast<const bf16*>(w_post), reinterpret_cast<bf16*>(resid),
                           reinterpret_cast<const bf16*>(w_pre), eps, (int)hidden,
                           reinterpret_cast<bf16*>(x_next)));
  FBFP_LAUNCH_CHECK("post_residual_pre_kernel");
  return FBFP_OK;
}

extern "C" int fbfp_qk_rope_cache(const void* qkv, int64_t m, int64_t nh, int64_t nkv, int64_t hd,
                                  const void* q_norm_w, const void* k_norm_w, float eps, const void* cos_table,
                                  const void* sin_table, const int32_t* pos, int64_t max_ctx, void* q_out,
                                  void* k_cache, void* v_cache, int32_t* err, void* stream) {
  FBFP_CHECK_ARG(qkv && q_norm_w && k_norm_w && cos_table && sin_table && pos && q_out && k_cache && v_cache &&
                     err,
                 "null pointer");
  FBFP_CHECK_ARG(nh > 0 && nkv > 0 && nh % nkv == 0 && hd > 0 && hd % 2 == 0 && hd <= 1024 && max_ctx > 0,
                 "bad head shape (nh %lld, nkv %lld, hd %lld)", (long long)nh, (long long)nkv, (long long)hd);
  FBFP_CHECK_ARG(m >= 1 && m <= 65535, "m must be in [1, 65535]");
  const size_t smem = sizeof(float) * ((size_t)hd + 33);
  FBFP_CUDA_TRY(launch_pdl(qk_rope_cache_kernel, dim3((unsigned)(nh + nkv), (unsigned)m), dim3(128), smem,
                           as_stream(stream), reinterpret_cast<const bf16*>(qkv), (int)nh, (int)nkv, (int)hd,
                           reinterpret_cast<const bf16*>(q_norm_w), reinterpret_cast<const bf16*>(k_norm_w), eps,
                           reinterpret_cast<const bf16*>(cos_table), reinterpret_cast<const bf16*>(sin_table), pos,
                           (int)max_ctx, reinterpret_cast<bf16*>(q_out), reinterpret_cast<bf16*>(k_cache),
                           reinterpret_cast<bf16*>(v_cache), err));
  FBFP_LAUNCH_CHECK("qk_rope_cache_kernel");
  return FBFP_OK;
}

extern "C" int fbfp_decode_attention(const void* q, int64_t m, const void* k_cache, const void* v_cache,
                                     int64_t nh, int64_t nkv, int64_t hd, int64_t max_ctx, const int32_t* pos,
                                     int64_t window, float scaling, void* out, void* stream) {
  FBFP_CHECK_ARG(q && k_cache && v_cache && pos && out, "null pointer");
  FBFP_CHECK_ARG(nh > 0 && nkv > 0 && nh % nkv == 0 && hd > 0 && hd <= 256 && hd % 8 == 0,
                 "bad head shape (head_dim a multiple of 8, at most 256)");
  FBFP_CHECK_ARG(((uintptr_t)q & 15) == 0 && ((uintptr_t)k_cache & 15) == 0 && ((uintptr_t)v_cache & 15) == 0,
                 "q and the caches must be 16-byte aligned");
  FBFP_CHECK_ARG(max_ctx > 0 && max_ctx + 8 * hd <= 10000, "max_ctx + 8 * head_dim must be <= 10000");
  FBFP_CHECK_ARG(m >= 1 && m <= 65535, "m must be in [1, 65535]");
  const size_t smem = sizeof(float) * ((size_t)max_ctx + 8 * (size_t)hd + 33);
  FBFP_CUDA_TRY(launch_pdl(decode_attention_kernel, dim3((unsigned)nh, (unsigned)m), dim3(kAttnThreads), smem,
                           as_stream(stream), reinterpret_cast<const bf16*>(q), reinterpret_cast<const bf16*>(k_cache),
                           reinterpret_cast<const bf16*>(v_cache), (int)nh, (int)nkv, (int)hd, (int)max_ctx, pos,
                           (int)window, scaling, reinterpret_cast<bf16*>(out)));
  FBFP_LAUNCH_CHECK("decode_attention_kernel");
  return FBFP_OK;
}

extern "C" int fbfp_geglu(const void* gate_up, int64_t m, int64_t inter, void* out, void* stream) {
  FBFP_CHECK_ARG(gate_up && out && inter > 0 && m >= 1, "bad arguments");
  const int64_t total = m * inter;
  const int64_t want = (total + 255) / 256;
  const int blocks = (int)(want < 1184 ? want : 1184);
  FBFP_CUDA_TRY(launch_pdl(geglu_kernel, dim3(blocks), dim3(256), 0, as_stream(stream),
                           reinterpret_cast<const bf16*>(gate_up), inter, total, reinterpret_cast<bf16*>(out)));
  FBFP_LAUNCH_CHECK("geglu_kernel");
  return FBFP_OK;
}

extern "C" int fbfp_advance_position(int32_t* pos, int64_t m, void* stream) {
  FBFP_CHECK_ARG(pos && m >= 1 && m <= 65535, "bad arguments");
  FBFP_CUDA_TRY(launch_pdl(advance_kernel, dim3(1), dim3(1), 0, as_stream(stream), pos, (int)m));
  FBFP_LAUNCH_CHECK("advance_kernel");
  return FBFP_OK;
}

extern "C" int64_t fbfp_decode_attention_step_scratch_bytes(int64_t b, int64_t nh, int64_t hd, int64_t max_ctx) {
  if (b < 1 || nh < 1 || hd < 1 || max_ctx < 1) return -1;
  const int64_t splits = (max_ctx + kFaChunk - 1) / kFaChunk;
  const int64_t counters = (nh * b * 4 + 255) / 256 * 256;
  return counters + nh * b * splits * (hd + 2) * 4;
}

extern "C" int fbfp_decode_attention_step(const void* qkv, int64_t b, int64_t nh, int64_t nkv, int64_t hd,
                                          const void* q_norm_w, const void* k_norm_w, float eps,
                                          const void* cos_table, const void* sin_table, const int32_t* pos,
                                          int64_t max_ctx, void* k_cache, void* v_cache, int64_t seq_stride,
                                          int64_t window, float scaling, void* scratch, void* out, int32_t* err,
                                          void* stream) {
  FBFP_CHECK_ARG(qkv && q_norm_w && k_norm_w && cos_table && sin_table && pos && k_cache && v_cache && scratch &&
                     out && err,
                 "null pointer");
  FBFP_CHECK_ARG(nh > 0 && nkv > 0 && nh % nkv == 0 && hd > 0 && hd <= 256 && hd % 16 == 0,
                 "bad head shape (nh %lld, nkv %lld, hd %lld: hd a multiple of 16 up to 256)", (long long)nh,
                 (long long)nkv, (long long)hd);
  FBFP_CHECK_ARG(b >= 1 && b <= 65535 && max_ctx > 0 && max_ctx < (1 << 30), "bad batch %lld or max_ctx %lld",
                 (long long)b, (long long)max_ctx);
  FBFP_CHECK_ARG(b == 1 || seq_stride >= nkv * max_ctx * hd, "seq_stride %lld below one sequence's cache",
                 (long long)seq_stride);
  FBFP_CHECK_ARG(((uintptr_t)k_cache & 15) == 0 && ((uintptr_t)v_cache & 15) == 0 && (seq_stride % 8) == 0,
                 "caches must be 16-byte aligned (seq_stride a multiple of 8)");
  FBFP_CHECK_ARG(((uintptr_t)scratch & 15) == 0, "scratch must be 16-byte aligned");
  const int64_t splits = (max_ctx + kFaChunk - 1) / kFaChunk;
  FBFP_CHECK_ARG(splits <= 65535, "max_ctx too large");
  int* counters = reinterpret_cast<int*>(scratch);
  float* part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(scratch) + (nh * b * 4 + 255) / 256 * 256);
  const size_t smem = sizeof(float) * (kFaChunk + (kFaThreads / 32) * (size_t)hd);
  FBFP_CUDA_TRY(launch_pdl(decode_attention_step_kernel, dim3((unsigned)nh, (unsigned)b, (unsigned)splits),
                           dim3(kFaThreads), smem, as_stream(stream), reinterpret_cast<const bf16*>(qkv), (int)nh,
                           (int)nkv, (int)hd, reinterpret_cast<const bf16*>(q_norm_w),
                           reinterpret_cast<const bf16*>(k_norm_w), eps, reinterpret_cast<const bf16*>(cos_table),
                           reinterpret_cast<const bf16*>(sin_table), pos, (int)max_ctx,
                           reinterpret_cast<bf16*>(k_cache), reinterpret_cast<bf16*>(v_cache), seq_stride,
                           (int)window, scaling, (int)splits, part, counters, reinterpret_cast<bf16*>(out), err));
  FBFP_LAUNCH_CHECK("decode_attention_step_kernel");
  return FBFP_OK;
}

extern "C" int fbfp_advance_positions(int32_t* pos, int64_t b, void* stream) {
  FBFP_CHECK_ARG(pos && b >= 1 && b <= 1024, "bad arguments (1 <= b <= 1024)");
  FBFP_CUDA_TRY(launch_pdl(advance_rows_kernel, dim3(1), dim3((unsigned)((b + 31) / 32 * 32)), 0,
                           as_stream(stream), pos, (int)b));
  FBFP_LAUNCH_CHECK("advance_rows_kernel");
  return FBFP_OK;
}
