// compress.cu — GPU OABF compressor with the reference's output bytes.
//
// Follows OABFCompressor (flash_bfp/compressor.py:11-117). The reference computes in torch
// on the CPU in the dtype of W; every rounding it performs is reproduced here:
//   * threshold (compressor.py:11-32): fp64 moments over W (one pass for the mean, one for
//     the centred moments), then the scalar chain var -> std -> kurtosis -> log -> scale ->
//     clamp, each step rounded to W's dtype exactly as the torch ops round it;
//   * block exponent floor(log2(max(bmax, 1e-8))) (compressor.py:87) from the exponent
//     bits plus the torch-log2 exception tables of log2_tables.h;
//   * mantissa clamp(round_half_even(|x| / 2^e * 15), 0, 15) with the product rounded to
//     W's dtype (compressor.py:90-94); signs and nibbles packed bit-for-bit
//     (compressor.py:97-107);
//   * outliers |x| > thr in ascending flat index order (compressor.py:65-80).
// All passes are HBM-bound streaming kernels: warps walk rows with 16-byte loads.
#include "common.cuh"
#include "log2_tables.h"
#include "scan.cuh"

namespace fbfp {

constexpr int kStatParts = 1024;      // partial-sum slots (one per block of the stats grid)
constexpr int kStatThreads = 256;

struct StatsHeader {                  // lives at the start of the scratch buffer
  double mean64;                      // exact-ish mean (fp64)
  float mean_dt;                      // mean rounded to W's dtype (torch.mean)
  float pad;
  double s2, s4;                      // reduced centred sums (debug/inspection)
};

__device__ __forceinline__ float rnd_dt(float v, int dt) {
  return dt == FBFP_BF16 ? round_bf16(v) : v;
}

// Visit every element of the [n_out, k_in] matrix once: warps take rows grid-stride;
// lanes take 8 consecutive elements per step (one 16-byte load for bf16, two for fp32
// when the row is 16-byte aligned).
template <typename F>
__device__ __forceinline__ void for_each_element(const void* w, int dt, int64_t n_out,
                                                 int64_t k_in, int64_t ldw, F&& f) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int es = dt == FBFP_F32 ? 4 : 2;
  for (int64_t n = warp; n < n_out; n += nwarps) {
    const char* row = reinterpret_cast<const char*>(w) + n * ldw * es;
    const bool vec = ((uintptr_t)row & 15) == 0;
    for (int64_t k0 = (int64_t)lane * 8; k0 < k_in; k0 += 256) {
      float v[8];
      if (vec && k0 + 8 <= k_in) {
        if (dt == FBFP_BF16) {
          const uint4 q = *reinterpret_cast<const uint4*>(row + k0 * 2);
          const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            v[2 * j] = __uint_as_float(u[j] << 16);
            v[2 * j + 1] = __uint_as_float(u[j] & 0xFFFF0000u);
          }
        } else {
          const float4 a = *reinterpret_cast<const float4*>(row + k0 * 4);
          const float4 b = *reinterpret_cast<const float4*>(row + k0 * 4 + 16);
          v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
          v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) f(v[j]);
      } else {
        for (int j = 0; j < 8 && k0 + j < k_in; ++j) f(load_as_float(row, dt, k0 + j));
      }
    }
  }
}

template <int NV>
__device__ __forceinline__ void block_reduce_store(double (&acc)[NV], double* out_parts) {
  __shared__ double red[NV][kStatThreads / 32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    double v = acc[j];
    for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
    if (lane == 0) red[j][wid] = v;
  }
  __syncthreads();
  if (threadIdx.x < NV) {
    double s = 0;
    for (int i = 0; i < kStatThreads / 32; ++i) s += red[threadIdx.x][i];
    out_parts[threadIdx.x * kStatParts + blockIdx.x] = s;
  }
}

__global__ void __launch_bounds__(kStatThreads)
stats_sum_kernel(const void* w, int dt, int64_t n_out, int64_t k_in, int64_t ldw, double* parts) {
  double acc[1] = {0.0};
  for_each_element(w, dt, n_out, k_in, ldw, [&](float x) { acc[0] += (double)x; });
  block_reduce_store<1>(acc, parts);
}

// Fixed-order reduction of the per-block partials (deterministic).
__device__ double reduce_parts(const double* parts, int nparts) {
  __shared__ double red[1024];
  double s = 0.0;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) s += parts[i];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
    __syncthreads();
  }
  const double r = red[0];
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(1024)
stats_mean_kernel(const double* parts, int nparts, int64_t numel, int dt, StatsHeader* hdr) {
  const double s1 = reduce_parts(parts, nparts);
  if (threadIdx.x == 0) {
    const double m = s1 / (double)numel;
    hdr->mean64 = m;
    hdr->mean_dt = rnd_dt(__double2float_rn(m), dt);   // torch.mean in W's dtype
  }
}

// bf16 weights: the same two sums with the per-element work in fp32 and fp64 only once per 8
// elements. The fourth-power term is computed exactly as the fp64 route computes it: d is a
// bf16 value, so d*d is exact in fp32 and d^4 = (d*d)^2 is one fp32 rounding of the exact
// product, which is what rounding the exact fp64 product to fp32 gives. The centred square
// sum uses the fp32 shift mh = fl32(mean): sum((x - m)^2) = S2 - 2 dm S1 + N dm^2 with
// S1 = sum(x - mh), S2 = sum((x - mh)^2) and dm = m - mh, taken in fp64 at the end
// (stats_threshold_kernel); each 8-element fp32 partial is added to an fp64 accumulator, so
// the rounding errors of the partials are independent, unbiased and about 2^-24 of a partial:
// their sum is far below one rounding step of the bf16 (or fp32) variance.
__global__ void __launch_bounds__(kStatThreads)
stats_central_bf16_kernel(const void* w, int64_t n_out, int64_t k_in, int64_t ldw,
                          const StatsHeader* hdr, double* parts) {
  const float mh = __double2float_rn(hdr->mean64);
  const float mdt = hdr->mean_dt;
  double acc[3] = {0.0, 0.0, 0.0};                // S2, fourth-power sum, S1
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t n = warp; n < n_out; n += nwarps) {
    const uint16_t* row = reinterpret_cast<const uint16_t*>(w) + n * ldw;
    const bool vec = ((uintptr_t)row & 15) == 0;
    for (int64_t k0 = (int64_t)lane * 8; k0 < k_in; k0 += 256) {
      float v[8];
      int cnt = 8;
      if (vec && k0 + 8 <= k_in) {
        const uint4 q = *reinterpret_cast<const uint4*>(row + k0);
        const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          v[2 * j] = __uint_as_float(u[j] << 16);
          v[2 * j + 1] = __uint_as_float(u[j] & 0xFFFF0000u);
        }
      } else {
        cnt = (int)(k_in - k0 < 8 ? k_in - k0 : 8);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = j < cnt ? bf16_bits_to_float(row[k0 + j]) : mh;
      }
      float s1 = 0.f, s2 = 0.f, s4 = 0.f;
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        const float t0 = __fsub_rn(v[j], mh), t1 = __fsub_rn(v[j + 1], mh);
        s1 = __fadd_rn(__fadd_rn(s1, t0), t1);
        s2 = __fmaf_rn(t1, t1, __fmaf_rn(t0, t0, s2));
        float d0 = __fsub_rn(v[j], mdt), d1 = __fsub_rn(v[j + 1], mdt);
        round_bf16x2(d0, d1);                                   // (W - mean) in bf16
        const float e0 = __fmul_rn(d0, d0), e1 = __fmul_rn(d1, d1);    // exact
        float p0 = __fmul_rn(e0, e0), p1 = __fmul_rn(e1, e1);
        round_bf16x2(p0, p1);                                   // ** 4 in bf16
        s4 = j < cnt ? __fadd_rn(s4, p0) : s4;
        s4 = j + 1 < cnt ? __fadd_rn(s4, p1) : s4;
      }
      acc[0] += (double)s2;
      acc[1] += (double)s4;
      acc[2] += (double)s1;
    }
  }
  block_reduce_store<3>(acc, parts);
}

__global__ void __launch_bounds__(kStatThreads)
stats_central_kernel(const void* w, int dt, int64_t n_out, int64_t k_in, int64_t ldw,
                     const StatsHeader* hdr, double* parts) {
  const double m64 = hdr->mean64;
  const float mdt = hdr->mean_dt;
  double acc[2] = {0.0, 0.0};
  for_each_element(w, dt, n_out, k_in, ldw, [&](float x) {
    const double dv = (double)x - m64;
    acc[0] += dv * dv;                                         // torch.var (fp64 accumulate)
    const float d = rnd_dt(__fsub_rn(x, mdt), dt);             // (W - mean) in W's dtype
    const double d2 = (double)d * (double)d;
    const float p = rnd_dt(__double2float_rn(d2 * d2), dt);   // ** 4 in W's dtype
    acc[1] += (double)p;
  });
  block_reduce_store<2>(acc, parts);
}

// Scalar chain of compute_dynamic_threshold (compressor.py:19-32), rounded like torch.
__global__ void __launch_bounds__(1024)
stats_threshold_kernel(const double* parts, int nparts, int64_t numel, int dt, StatsHeader* hdr,
                       float* thr_out, int shifted) {
  double s2 = reduce_parts(parts, nparts);
  const double s4 = reduce_parts(parts + kStatParts, nparts);
  if (shifted) {                                  // sums about mh = fl32(mean): recentre on the mean
    const double s1 = reduce_parts(parts + 2 * kStatParts, nparts);
    const double dm = hdr->mean64 - (double)__double2float_rn(hdr->mean64);
    s2 = s2 - 2.0 * dm * s1 + (double)numel * dm * dm;
  }
  if (threadIdx.x != 0) return;
  hdr->s2 = s2;
  hdr->s4 = s4;
  const double n = (double)numel;
  const double var64 = s2 / (n - 1.0);                               // NaN for numel == 1
  const float var = rnd_dt(__double2float_rn(var64), dt);
  const float sd = rnd_dt(__fsqrt_rn(var), dt);
  const float fourth = rnd_dt(__double2float_rn(s4 / n), dt);
  const float var2 = rnd_dt(__fmul_rn(var, var), dt);
  const float den = rnd_dt(__fadd_rn(var2, 1e-8f), dt);
  const float kurt = rnd_dt(__fdiv_rn(fourth, den), dt);
  float k3 = rnd_dt(__fdiv_rn(kurt, 3.0f), dt);
  if (!(k3 != k3) && k3 < 0.5f) k3 = 0.5f;                           // clamp(min=0.5), NaN stays
  const float lg = rnd_dt(__double2float_rn(log((double)k3)), dt);
  const float t1 = rnd_dt(__fmul_rn(0.1f, lg), dt);
  const float t2 = rnd_dt(__fadd_rn(1.0f, t1), dt);
  const float sc = rnd_dt(__fmul_rn(2.43f, t2), dt);
  float thr = rnd_dt(__fmul_rn(sd, sc), dt);
  if (!(thr != thr)) {
    const float lo = rnd_dt(0.01f, dt), hi = rnd_dt(0.2f, dt);
    thr = thr < lo ? lo : (thr > hi ? hi : thr);
  }
  *thr_out = thr;
}

// ----------------------------------------------------------------------------------
// packing
// ----------------------------------------------------------------------------------
__device__ __forceinline__ int floor_log2_torch(float x, int dt) {
  const uint32_t bits = __float_as_uint(x);
  const int be = (int)((bits >> 23) & 0xFF);
  const int e0 = be - 127;
  if (be == 0 || be == 255) return e0;            // unreachable for x >= 1e-8 finite
  if (dt == FBFP_BF16) {
    const uint32_t m7 = (bits >> 16) & 0x7F;
    return (m7 >= 128u - kLog2BumpBF16[e0 + 126]) ? e0 + 1 : e0;
  }
  const uint32_t m23 = bits & 0x7FFFFF;
  return (m23 >= (1u << 23) - kLog2BumpF32[e0 + 126]) ? e0 + 1 : e0;
}

__device__ __forceinline__ void load_block16(const void* w, int dt, int64_t n, int64_t n_out,
                                             int64_t k0, int64_t k_in, int64_t ldw, float (&v)[16]) {
  if (n >= n_out) {
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = 0.f;
    return;
  }
  const int es = dt == FBFP_F32 ? 4 : 2;
  const char* p = reinterpret_cast<const char*>(w) + (n * ldw + k0) * es;
  if (k0 + 16 <= k_in && ((uintptr_t)p & 15) == 0) {
    if (dt == FBFP_BF16) {
      const uint4 a = reinterpret_cast<const uint4*>(p)[0];
      const uint4 b = reinterpret_cast<const uint4*>(p)[1];
      const uint32_t u[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[2 * j] = __uint_as_float(u[j] << 16);
        v[2 * j + 1] = __uint_as_float(u[j] & 0xFFFF0000u);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 a = reinterpret_cast<const float4*>(p)[j];
        v[4 * j] = a.x; v[4 * j + 1] = a.y; v[4 * j + 2] = a.z; v[4 * j + 3] = a.w;
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = (k0 + j < k_in) ? load_as_float(p, dt, j) : 0.f;
  }
}

// One thread per block of the padded [npad, kpad] matrix.
__global__ void __launch_bounds__(256)
pack_kernel(const void* w, int dt, int64_t n_out, int64_t k_in, int64_t ldw, int64_t kb_row,
            int64_t nblocks, const float* thr_p, int8_t* ex, int16_t* sg, uint2* pay,
            uint16_t* masks, int32_t* row_counts) {
  const float thr = *thr_p;
  const float c1e8 = rnd_dt(1e-8f, dt);
  const float c1e7 = rnd_dt(1e-7f, dt);
  for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < nblocks;
       b += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = b / kb_row, kb = b - n * kb_row;
    float v[16];
    load_block16(w, dt, n, n_out, kb * kBlock, k_in, ldw, v);
    uint32_t omask = 0;
    float bmax = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float a = fabsf(v[j]);
      if (a > thr) { omask |= 1u << j; v[j] = 0.f; }          // outliers leave the dense part
      else bmax = fmaxf(bmax, a);
    }
    const float xm = fmaxf(bmax, c1e8);
    const int e = floor_log2_torch(xm, dt);
    const bool unit = bmax < c1e7;                            // scale = 1 for tiny blocks
    // 15 * 2^-e, exact (e >= -27 unless the block is tiny, where the scale is 1): one rounding
    // of |x| * 15 / 2^e equals the reference's rounding of (|x| / 2^e, exact) * 15
    const float inv15 = unit ? 15.0f : __uint_as_float((uint32_t)(127 - e) << 23) * 15.0f;
    uint32_t s = 0, w0 = 0, w1 = 0;
    float q[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) q[j] = __fmul_rn(fabsf(v[j]), inv15);
    if (dt == FBFP_BF16) {
#pragma unroll
      for (int j = 0; j < 16; j += 2) round_bf16x2(q[j], q[j + 1]);
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      // 0 <= q < 30: adding 1.5 * 2^23 rounds q half-to-even to an integer held in the low
      // mantissa bits; clamp to 15
      const uint32_t r = __float_as_uint(__fadd_rn(q[j], 12582912.0f)) - 0x4B400000u;
      const uint32_t m = r < 15u ? r : 15u;
      if (j < 8) w0 |= m << (4 * j); else w1 |= m << (4 * (j - 8));
      if (v[j] < 0.f) s |= 1u << j;
    }
    ex[b] = (int8_t)e;
    sg[b] = (int16_t)(uint16_t)s;
    pay[b] = make_uint2(w0, w1);
    masks[b] = (uint16_t)omask;
    // one atomic per row a warp touches (a warp's 32 consecutive blocks span one or two rows)
    const unsigned act = __activemask();
    const unsigned same = __match_any_sync(act, (unsigned long long)n);
    const int tot = __reduce_add_sync(same, __popc(omask));
    if (tot && (threadIdx.x & 31) == __ffs(same) - 1) atomicAdd(&row_counts[n], tot);
  }
}

// One warp per padded row: ordered compaction of the outlier bits of the row's blocks (the
// row's block masks are read 8 chunks of 32 at a time, so their loads overlap).
__global__ void __launch_bounds__(256)
emit_outliers_kernel(const void* w, int dt, int64_t n_out, int64_t ldw, int64_t kb_row,
                     const uint16_t* masks, const int32_t* row_offsets, int32_t* bidx,
                     int32_t* off, uint16_t* val) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int es = dt == FBFP_F32 ? 4 : 2;
  for (int64_t n = warp; n < n_out; n += nwarps) {
    int64_t base = row_offsets[n];
    if (row_offsets[n + 1] == base) continue;
    const char* row = reinterpret_cast<const char*>(w) + n * ldw * es;
    uint32_t mk[8];                              // the next 8 chunks' masks, loaded together
    for (int64_t kb0 = 0; kb0 < kb_row; kb0 += 32) {
      const int64_t kb = kb0 + lane;
      const int ci = (int)((kb0 >> 5) & 7);
      if (ci == 0) {
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          const int64_t kk = kb + 32 * c8;
          mk[c8] = kk < kb_row ? masks[n * kb_row + kk] : 0u;
        }
      }
      uint32_t m = mk[0];
#pragma unroll
      for (int c8 = 1; c8 < 8; ++c8) m = ci == c8 ? mk[c8] : m;
      const int c = __popc(m);
      int incl = c;
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      int64_t pos = base + incl - c;
      uint32_t mm = m;
      while (mm) {
        const int j = __ffs(mm) - 1;
        mm &= mm - 1;
        const float x = load_as_float(row, dt, kb * kBlock + j);
        bidx[pos] = (int32_t)(n * kb_row + kb);
        off[pos] = j;
        val[pos] = __half_as_ushort(__float2half_rn(x));
        ++pos;
      }
      base += __shfl_sync(0xffffffffu, incl, 31);
    }
  }
}

static int stats_grid(int64_t n_out) {
  int64_t warps_needed = n_out;                       // one warp per row at most
  int64_t blocks = (warps_needed * 32 + kStatThreads - 1) / kStatThreads;
  if (blocks > kStatParts) blocks = kStatParts;
  return (int)(blocks < 1 ? 1 : blocks);
}

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

struct ScratchLayout {
  size_t hdr, parts, masks, total;
};
static ScratchLayout scratch_layout(int64_t kpad, int64_t npad) {
  ScratchLayout L;
  L.hdr = 0;
  L.parts = align256(sizeof(StatsHeader));
  L.masks = L.parts + align256(sizeof(double) * 3 * kStatParts);
  L.total = L.masks + align256(sizeof(uint16_t) * (size_t)(npad * (kpad / kBlock)));
  return L;
}

}  // namespace fbfp

using namespace fbfp;

extern "C" int64_t fbfp_compress_scratch_bytes(int64_t n_out, int64_t k_in, int64_t kpad, int64_t npad) {
  (void)n_out; (void)k_in;
  return (int64_t)scratch_layout(kpad, npad).total;
}

extern "C" int fbfp_compress_threshold(const void* w, int w_dtype, int64_t n_out, int64_t k_in,
                                       int64_t ldw, float* thr_out, void* scratch, void* stream) {
  FBFP_CHECK_ARG(w && thr_out && scratch, "null pointer");
  FBFP_CHECK_ARG(w_dtype == FBFP_F32 || w_dtype == FBFP_BF16, "w_dtype must be f32 or bf16");
  FBFP_CHECK_ARG(n_out > 0 && k_in > 0 && ldw >= k_in, "bad shape");
  FBFP_CHECK_ARG(((uintptr_t)scratch & 255) == 0, "scratch must be 256-byte aligned");
  cudaStream_t st = as_stream(stream);
  const ScratchLayout L = scratch_layout(16, 0);
  char* sp = reinterpret_cast<char*>(scratch);
  StatsHeader* hdr = reinterpret_cast<StatsHeader*>(sp + L.hdr);
  double* parts = reinterpret_cast<double*>(sp + L.parts);
  const int grid = stats_grid(n_out);
  const int64_t numel = n_out * k_in;
  stats_sum_kernel<<<grid, kStatThreads, 0, st>>>(w, w_dtype, n_out, k_in, ldw, parts);
  FBFP_LAUNCH_CHECK("stats_sum_kernel");
  stats_mean_kernel<<<1, 1024, 0, st>>>(parts, grid, numel, w_dtype, hdr);
  FBFP_LAUNCH_CHECK("stats_mean_kernel");
  const int shifted = w_dtype == FBFP_BF16;
  if (shifted) {
    stats_central_bf16_kernel<<<grid, kStatThreads, 0, st>>>(w, n_out, k_in, ldw, hdr, parts);
    FBFP_LAUNCH_CHECK("stats_central_bf16_kernel");
  } else {
    stats_central_kernel<<<grid, kStatThreads, 0, st>>>(w, w_dtype, n_out, k_in, ldw, hdr, parts);
    FBFP_LAUNCH_CHECK("stats_central_kernel");
  }
  stats_threshold_kernel<<<1, 1024, 0, st>>>(parts, grid, numel, w_dtype, hdr, thr_out, shifted);
  FBFP_LAUNCH_CHECK("stats_threshold_kernel");
  return FBFP_OK;
}

extern "C" int fbfp_compress_pack(const void* w, int w_dtype, int64_t n_out, int64_t k_in,
                                  int64_t ldw, int64_t kpad, int64_t npad, const float* thr,
                                  int8_t* exponents, int16_t* signs, int32_t* payload,
                                  int32_t* row_offsets, void* scratch, void* stream) {
  FBFP_CHECK_ARG(w && thr && exponents && signs && payload && row_offsets && scratch, "null pointer");
  FBFP_CHECK_ARG(w_dtype == FBFP_F32 || w_dtype == FBFP_BF16, "w_dtype must be f32 or bf16");
  FBFP_CHECK_ARG(n_out > 0 && k_in > 0 && ldw >= k_in, "bad shape");
  FBFP_CHECK_ARG(kpad >= k_in && kpad % kBlock == 0 && kpad - k_in < kBlock, "bad kpad");
  FBFP_CHECK_ARG(npad >= n_out, "bad npad");
  FBFP_CHECK_ARG(((uintptr_t)payload & 7) == 0, "payload must be 8-byte aligned");
  FBFP_CHECK_ARG(((uintptr_t)scratch & 255) == 0, "scratch must be 256-byte aligned");
  cudaStream_t st = as_stream(stream);
  const ScratchLayout L = scratch_layout(kpad, npad);
  uint16_t* masks = reinterpret_cast<uint16_t*>(reinterpret_cast<char*>(scratch) + L.masks);
  const int64_t kb_row = kpad / kBlock;
  const int64_t nblocks = npad * kb_row;
  FBFP_CUDA_TRY(cudaMemsetAsync(row_offsets, 0, sizeof(int32_t) * (npad + 1), st));
  int64_t grid = (nblocks + 255) / 256;
  if (grid > 148 * 64) grid = 148 * 64;
  pack_kernel<<<(int)grid, 256, 0, st>>>(w, w_dtype, n_out, k_in, ldw, kb_row, nblocks, thr,
                                         exponents, signs, reinterpret_cast<uint2*>(payload),
                                         masks, row_offsets);
  FBFP_LAUNCH_CHECK("pack_kernel");
  scan_rows_kernel<<<1, 1024, 0, st>>>(row_offsets, npad);
  FBFP_LAUNCH_CHECK("scan_rows_kernel");
  return FBFP_OK;
}

extern "C" int fbfp_compress_outliers(const void* w, int w_dtype, int64_t n_out, int64_t k_in,
                                      int64_t ldw, int64_t kpad, int64_t npad,
                                      const int32_t* row_offsets, int32_t* block_idx,
                                      int32_t* offset, uint16_t* value_f16, void* scratch,
                                      void* stream) {
  FBFP_CHECK_ARG(w && row_offsets && scratch, "null pointer");
  FBFP_CHECK_ARG(w_dtype == FBFP_F32 || w_dtype == FBFP_BF16, "w_dtype must be f32 or bf16");
  FBFP_CHECK_ARG(n_out > 0 && k_in > 0 && ldw >= k_in && kpad % kBlock == 0 && npad >= n_out,
                 "bad shape");
  FBFP_CHECK_ARG(((uintptr_t)scratch & 255) == 0, "scratch must be 256-byte aligned");
  FBFP_CHECK_ARG(block_idx && offset && value_f16, "null output pointer");
  cudaStream_t st = as_stream(stream);
  const ScratchLayout L = scratch_layout(kpad, npad);
  const uint16_t* masks = reinterpret_cast<const uint16_t*>(reinterpret_cast<const char*>(scratch) + L.masks);
  int64_t grid = (n_out * 32 + 255) / 256;
  if (grid > 148 * 16) grid = 148 * 16;
  emit_outliers_kernel<<<(int)grid, 256, 0, st>>>(w, w_dtype, n_out, ldw, kpad / kBlock, masks,
                                                  row_offsets, block_idx, offset, value_f16);
  FBFP_LAUNCH_CHECK("emit_outliers_kernel");
  return FBFP_OK;
}
