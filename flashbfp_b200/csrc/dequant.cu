// dequant.cu — bit-exact OABF dequantisation and outlier scatter.
//
// Element i of block b: w = (sign_i ? -1 : +1) * fl(m_i / 15) * 2^e_b in fp32, where m_i is
// nibble i%8 of payload word i/8 and sign_i is bit i of the block's sign word — the
// formula of oabf_gemm_kernel (flash_bfp/triton_kernel.py:73-80) and of the CPU path
// (:112-122). Multiplying by 2^e (e in [-126, 127]) is exact, so the result is bit-exact;
// sign = 1 with m = 0 yields -0.0 like the reference.
#include "common.cuh"

namespace fbfp {

__constant__ float kM15[16] = {
    FBFP_M15(0),  FBFP_M15(1),  FBFP_M15(2),  FBFP_M15(3),  FBFP_M15(4),  FBFP_M15(5),
    FBFP_M15(6),  FBFP_M15(7),  FBFP_M15(8),  FBFP_M15(9),  FBFP_M15(10), FBFP_M15(11),
    FBFP_M15(12), FBFP_M15(13), FBFP_M15(14), FBFP_M15(15)};

__device__ __forceinline__ float pow2i(int e) {
  // 2^e for e in [-126, 127] from the exponent field.
  return __uint_as_float((uint32_t)(e + 127) << 23);
}

// One thread per block; grid-stride over n_out * (k_in rounded up to blocks).
__global__ void dequant_kernel(const int8_t* __restrict__ ex, const int16_t* __restrict__ sg,
                               const uint2* __restrict__ pay, int64_t n_out, int64_t k_in,
                               int64_t kb_row, int64_t kb_used, int out_dtype, void* out,
                               int64_t ldo) {
  const int64_t total = n_out * kb_used;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / kb_used, kb = i - n * kb_used;
    const int64_t b = n * kb_row + kb;
    const uint2 w = pay[b];
    const uint32_t s = (uint16_t)sg[b];
    const float scale = pow2i((int)ex[b]);
    const int64_t k0 = kb * kBlock;
    const int64_t base = n * ldo + k0;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (k0 + j < k_in) {
        const uint32_t word = j < 8 ? w.x : w.y;
        const uint32_t m = (word >> (4 * (j & 7))) & 0xF;
        float v = kM15[m] * scale;
        if ((s >> j) & 1) v = -v;
        store_from_float(out, out_dtype, base + j, v);
      }
    }
  }
}

// COO -> dense write-back of outlier values (fp16 -> fp32 exact, then to out dtype).
__global__ void scatter_outliers_kernel(const int32_t* __restrict__ bidx,
                                        const int32_t* __restrict__ off,
                                        const uint16_t* __restrict__ val, int64_t count,
                                        int64_t kpad, int64_t n_out, int64_t k_in,
                                        int out_dtype, void* out, int64_t ldo) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t g = (int64_t)bidx[i] * kBlock + off[i];
    const int64_t r = g % kpad, c = g / kpad;
    if (r < k_in && c < n_out) {
      const float v = __half2float(__ushort_as_half(val[i]));
      store_from_float(out, out_dtype, c * ldo + r, v);
    }
  }
}

static int grid_for(int64_t work, int threads) {
  int64_t b = (work + threads - 1) / threads;
  if (b > 148 * 32) b = 148 * 32;
  return (int)(b < 1 ? 1 : b);
}

}  // namespace fbfp

using namespace fbfp;

extern "C" int fbfp_dequant(const int8_t* exponents, const int16_t* signs, const int32_t* payload,
                            int64_t n_out, int64_t k_in, int64_t kpad, int out_dtype, void* out,
                            int64_t ldo, void* stream) {
  FBFP_CHECK_ARG(exponents && signs && payload && out, "null pointer");
  FBFP_CHECK_ARG(n_out > 0 && k_in > 0 && kpad >= k_in && kpad % kBlock == 0,
                 "bad shape n_out=%lld k_in=%lld kpad=%lld", (long long)n_out,
                 (long long)k_in, (long long)kpad);
  FBFP_CHECK_ARG(ldo >= k_in, "ldo < k_in");
  FBFP_CHECK_ARG(out_dtype == FBFP_F32 || out_dtype == FBFP_BF16, "out_dtype must be f32 or bf16");
  FBFP_CHECK_ARG(((uintptr_t)payload & 7) == 0, "payload must be 8-byte aligned");
  const int64_t kb_row = kpad / kBlock;
  const int64_t kb_used = (k_in + kBlock - 1) / kBlock;
  const int threads = 256;
  dequant_kernel<<<grid_for(n_out * kb_used, threads), threads, 0, as_stream(stream)>>>(
      exponents, signs, reinterpret_cast<const uint2*>(payload), n_out, k_in, kb_row, kb_used,
      out_dtype, out, ldo);
  FBFP_LAUNCH_CHECK("dequant_kernel");
  return FBFP_OK;
}

extern "C" int fbfp_scatter_outliers(const int32_t* block_idx, const int32_t* offset,
                                     const uint16_t* value_f16, int64_t count, int64_t kpad,
                                     int64_t n_out, int64_t k_in, int out_dtype, void* out,
                                     int64_t ldo, void* stream) {
  FBFP_CHECK_ARG(count >= 0, "negative count");
  if (count == 0) return FBFP_OK;
  FBFP_CHECK_ARG(block_idx && offset && value_f16 && out, "null pointer");
  FBFP_CHECK_ARG(kpad > 0 && kpad % kBlock == 0 && n_out > 0 && k_in > 0 && ldo >= k_in,
                 "bad shape");
  FBFP_CHECK_ARG(out_dtype == FBFP_F32 || out_dtype == FBFP_BF16, "out_dtype must be f32 or bf16");
  const int threads = 256;
  scatter_outliers_kernel<<<grid_for(count, threads), threads, 0, as_stream(stream)>>>(
      block_idx, offset, value_f16, count, kpad, n_out, k_in, out_dtype, out, ldo);
  FBFP_LAUNCH_CHECK("scatter_outliers_kernel");
  return FBFP_OK;
}
