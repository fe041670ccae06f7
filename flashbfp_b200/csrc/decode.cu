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
__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

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
