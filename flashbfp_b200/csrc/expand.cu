// expand.cu — two-pass prefill for many tokens: the packed matrix is expanded once into a bf16
// scratch holding 15 x the dequantised weights, and a cuBLASLt bf16 GEMM (fp32 accumulation)
// multiplies it with the activations, scaled back by 1/15, with the bias added in its epilogue.
//
// The scratch holds exactly the A operand the fused prefill kernel (gemm_tc.cu) builds in tensor
// memory: dense elements s * m * 2^e (exact in bf16: m has at most four significant bits and
// 2^e with e in [-126, 127] is a normal power of two) and outliers bf16(15 v) in their (+0)
// slots, so the product matches the fused kernel's up to the order of the fp32 additions, and
// the reference's (flash_bfp/triton_kernel.py:22-86 dequantises w = s * fl(m / 15) * 2^e to the
// activation dtype, then multiplies) up to that one rounding.
#include <cublasLt.h>

#include "common.cuh"

namespace fbfp {

// The 16 bf16 values s * m * 2^e of one block as 8 pair words (element 2j in the low half).
// For e in [-120, 120]: a pair of nibbles placed under the biased exponent E = e + 134 reads as
// 2^e (128 + m) per element, and a paired bf16 subtraction of 2^e * 128 leaves m * 2^e exactly
// (a normal number, or zero); the signs are then xor-ed into bits 15 and 31. Other exponents take
// the fp32 product m * 2^e (exact, zero low half) element by element.
__device__ __forceinline__ void expand_pairs(uint2 w, uint32_t s, int e, uint32_t (&o)[8]) {
  // sign bit 2j at bit 2j and sign bit 2j + 1 at bit 2j + 16, so (sp << (15 - 2j)) puts pair j's
  // two signs at bits 15 and 31
  const uint32_t sp = (s & 0x5555u) | ((s & 0xAAAAu) << 15);
  if (e >= -120 && e <= 120) {
    const uint32_t K = (uint32_t)(e + 134) * 0x00800080u;
    const __nv_bfloat162 kb = *reinterpret_cast<const __nv_bfloat162*>(&K);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t word = h ? w.y : w.x;
      const uint32_t lo = word & 0x0F0F0F0Fu, hi = (word >> 4) & 0x0F0F0F0Fu;   // elements 2j', 2j'+1
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int j = 4 * h + q;
        const uint32_t pr = (__byte_perm(lo, hi, (uint32_t)(q | (q << 4) | ((4 + q) << 8) | ((4 + q) << 12))) &
                             0x000F000Fu) | K;
        __nv_bfloat162 d = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&pr), kb);
        o[j] = *reinterpret_cast<uint32_t*>(&d) ^ ((sp << (15 - 2 * j)) & 0x80008000u);
      }
    }
  } else {
    const float scale = __uint_as_float((uint32_t)(e + 127 < 0 ? 0 : e + 127) << 23);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t word = j < 4 ? w.x : w.y;
      const uint32_t m0 = (word >> (8 * (j & 3))) & 0xFu, m1 = (word >> (8 * (j & 3) + 4)) & 0xFu;
      const uint32_t f0 = __float_as_uint((float)m0 * scale) >> 16, f1 = __float_as_uint((float)m1 * scale) >> 16;
      o[j] = (f0 | (f1 << 16)) ^ ((sp << (15 - 2 * j)) & 0x80008000u);
    }
  }
}

// Tile-grouped outlier index (outliers.cu): entries by (128-row group, 256-column stage) segment,
// seg_ptr[0 .. nseg] the segment starts, then per segment 136 uint16 row starts.
struct TileIndex {
  const uint32_t* entries;   // null: no index (outliers come from the COO list)
  const int32_t* seg_ptr;
  int64_t n_stages, roff_base;
};

// Outliers of row n inside block kb: bf16(15 v) into their (+0) slots of the block's pairs.
__device__ __forceinline__ void patch_block(const TileIndex& t, int64_t n, int64_t kb, uint32_t (&o)[8]) {
  const int64_t sgm = (n >> 7) * t.n_stages + (kb >> 4);
  const int lr = (int)(n & 127);
  const uint16_t* ro = reinterpret_cast<const uint16_t*>(t.seg_ptr + t.roff_base) + sgm * 136;
  const int k0 = __ldg(ro + lr), k1 = __ldg(ro + lr + 1);
  if (k0 == k1) return;
  const uint32_t* es = t.entries + __ldg(t.seg_ptr + sgm);
  const int want = (int)(kb & 15);
  for (int k = k0; k < k1; ++k) {            // the row's entries of this stage, by column
    const uint32_t e = __ldg(es + k);
    const int c = (int)((e >> 16) & 0xFFu);
    if ((c >> 4) != want) continue;
    const float v15 = 15.0f * __half2float(__ushort_as_half((unsigned short)(e & 0xFFFFu)));
    const uint32_t bits = __bfloat16_as_ushort(__float2bfloat16_rn(v15));
    const int el = c & 15;
    const uint32_t keep = (el & 1) ? 0x0000FFFFu : 0xFFFF0000u, put = (el & 1) ? (bits << 16) : bits;
#pragma unroll
    for (int q = 0; q < 8; ++q)
      if (q == (el >> 1)) o[q] = (o[q] & keep) | put;
  }
}

// One thread per 16-weight block: 11 packed bytes in, 32 bytes out (two 16-byte stores when the
// block lies inside k_in, else element by element), with the block's outliers written in when the
// tile index is given. Rows stride over grid y, a row's blocks over grid x (no index division).
__global__ void expand_x15_kernel(const int8_t* __restrict__ ex, const int16_t* __restrict__ sg,
                                  const uint2* __restrict__ pay, int64_t n_out, int64_t k_in,
                                  int64_t kb_row, int64_t kb_used, TileIndex tix,
                                  uint16_t* __restrict__ out, int64_t ldo) {
  for (int64_t n = blockIdx.y; n < n_out; n += gridDim.y) {
    for (int64_t kb = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; kb < kb_used;
         kb += (int64_t)gridDim.x * blockDim.x) {
      const int64_t b = n * kb_row + kb;
      uint32_t o[8];
      expand_pairs(pay[b], (uint16_t)sg[b], (int)ex[b], o);
      if (tix.entries) patch_block(tix, n, kb, o);
      const int64_t k0 = kb * kBlock;
      uint16_t* dst = out + n * ldo + k0;
      if (k0 + kBlock <= k_in) {
        reinterpret_cast<uint4*>(dst)[0] = make_uint4(o[0], o[1], o[2], o[3]);
        reinterpret_cast<uint4*>(dst)[1] = make_uint4(o[4], o[5], o[6], o[7]);
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (k0 + j < k_in) dst[j] = (uint16_t)(o[j >> 1] >> (16 * (j & 1)));
      }
    }
  }
}

// Outliers into their slots as bf16(15 v) (15 v is exact in fp32; one rounding to bf16).
__global__ void scatter_x15_kernel(const int32_t* __restrict__ bidx, const int32_t* __restrict__ off,
                                   const uint16_t* __restrict__ val, int64_t count, int64_t kpad,
                                   int64_t n_out, int64_t k_in, uint16_t* __restrict__ out, int64_t ldo) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t g = (int64_t)bidx[i] * kBlock + off[i];
    const int64_t r = g % kpad, c = g / kpad;
    if (r < k_in && c < n_out) {
      const float v15 = 15.0f * __half2float(__ushort_as_half(val[i]));
      out[c * ldo + r] = __bfloat16_as_ushort(__float2bfloat16_rn(v15));
    }
  }
}

constexpr size_t kLtWorkspace = 32u << 20;

static size_t expand_matrix_bytes(int64_t n_out, int64_t kpad) {
  return ((size_t)n_out * (size_t)kpad * 2 + 255) & ~(size_t)255;
}

static int lt_check(cublasStatus_t s, const char* what) {
  if (s == CUBLAS_STATUS_SUCCESS) return FBFP_OK;
  return set_error(FBFP_ERR_CUDA, "%s failed (cublas status %d)", what, (int)s);
}

static cublasLtHandle_t lt_handle(int dev) {
  static cublasLtHandle_t h[64] = {};
  if (dev < 0 || dev >= 64) return nullptr;
  if (!h[dev] && cublasLtCreate(&h[dev]) != CUBLAS_STATUS_SUCCESS) h[dev] = nullptr;
  return h[dev];
}

// Y[m, n_out] (bf16 or fp32, row stride ldy) = (X[m, k_in] (bf16, ldx) W15[n_out, k_in]^T
// (ldw)) / 15 (+ bias, of Y's type). Column-major view for cuBLASLt: D (n_out x m, ld ldy) =
// alpha op(A) B with A = W15 (k_in x n_out, ld ldw, transposed) and B = X (k_in x m, ld ldx).
static int lt_gemm_x15(const void* x, int64_t m, int64_t ldx, const void* w15, int64_t ldw,
                       int64_t n_out, int64_t k_in, const void* bias, void* y, int y_dtype, int64_t ldy,
                       void* workspace, cudaStream_t st, int dev) {
  cublasLtHandle_t h = lt_handle(dev);
  if (!h) return set_error(FBFP_ERR_CUDA, "cublasLtCreate failed");
  cublasLtMatmulDesc_t op = nullptr;
  cublasLtMatrixLayout_t la = nullptr, lb = nullptr, lc = nullptr;
  cublasLtMatmulPreference_t pref = nullptr;
  int rc = FBFP_OK;
  const cublasOperation_t ta = CUBLAS_OP_T, tb = CUBLAS_OP_N;
  const float alpha = 1.0f / 15.0f, beta = 0.0f;
  const cudaDataType_t yt = y_dtype == FBFP_F32 ? CUDA_R_32F : CUDA_R_16BF;
  size_t wsb = kLtWorkspace;
  cublasLtMatmulHeuristicResult_t res = {};
  int found = 0;
  do {
    if ((rc = lt_check(cublasLtMatmulDescCreate(&op, CUBLAS_COMPUTE_32F, CUDA_R_32F), "MatmulDescCreate"))) break;
    if ((rc = lt_check(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_TRANSA, &ta, sizeof(ta)), "TRANSA"))) break;
    if ((rc = lt_check(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_TRANSB, &tb, sizeof(tb)), "TRANSB"))) break;
    if (bias) {
      const cublasLtEpilogue_t epi = CUBLASLT_EPILOGUE_BIAS;
      const cudaDataType_t bt = yt;
      if ((rc = lt_check(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_EPILOGUE, &epi, sizeof(epi)), "EPILOGUE"))) break;
      if ((rc = lt_check(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_BIAS_POINTER, &bias, sizeof(bias)), "BIAS_POINTER"))) break;
      if ((rc = lt_check(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_BIAS_DATA_TYPE, &bt, sizeof(bt)), "BIAS_DATA_TYPE"))) break;
    }
    if ((rc = lt_check(cublasLtMatrixLayoutCreate(&la, CUDA_R_16BF, (uint64_t)k_in, (uint64_t)n_out, ldw), "layout A"))) break;
    if ((rc = lt_check(cublasLtMatrixLayoutCreate(&lb, CUDA_R_16BF, (uint64_t)k_in, (uint64_t)m, ldx), "layout B"))) break;
    if ((rc = lt_check(cublasLtMatrixLayoutCreate(&lc, yt, (uint64_t)n_out, (uint64_t)m, ldy), "layout D"))) break;
    if ((rc = lt_check(cublasLtMatmulPreferenceCreate(&pref), "PreferenceCreate"))) break;
    if ((rc = lt_check(cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &wsb, sizeof(wsb)), "PREF_MAX_WORKSPACE"))) break;
    if ((rc = lt_check(cublasLtMatmulAlgoGetHeuristic(h, op, la, lb, lc, lc, pref, 1, &res, &found), "AlgoGetHeuristic"))) break;
    if (found < 1) { rc = set_error(FBFP_ERR_CUDA, "cuBLASLt found no algorithm for %lld x %lld x %lld",
                                    (long long)m, (long long)n_out, (long long)k_in); break; }
    rc = lt_check(cublasLtMatmul(h, op, &alpha, w15, la, x, lb, &beta, y, lc, y, lc, &res.algo, workspace,
                                 wsb, st), "cublasLtMatmul");
  } while (0);
  if (pref) cublasLtMatmulPreferenceDestroy(pref);
  if (lc) cublasLtMatrixLayoutDestroy(lc);
  if (lb) cublasLtMatrixLayoutDestroy(lb);
  if (la) cublasLtMatrixLayoutDestroy(la);
  if (op) cublasLtMatmulDescDestroy(op);
  return rc;
}

static int grid_blocks(int64_t work, int threads) {
  int64_t b = (work + threads - 1) / threads;
  if (b > 148 * 32) b = 148 * 32;
  return (int)(b < 1 ? 1 : b);
}

}  // namespace fbfp

using namespace fbfp;

extern "C" int64_t fbfp_gemm_expanded_scratch_bytes(int64_t n_out, int64_t kpad) {
  if (n_out <= 0 || kpad <= 0) return -1;
  return (int64_t)(expand_matrix_bytes(n_out, kpad) + kLtWorkspace);
}

extern "C" int fbfp_expand_x15(const int8_t* exponents, const int16_t* signs, const int32_t* payload,
                               int64_t n_out, int64_t k_in, int64_t kpad, const int32_t* block_idx,
                               const int32_t* offset, const uint16_t* value_f16, int64_t count,
                               const uint32_t* entries, const int32_t* seg_ptr, int64_t npad,
                               void* out, int64_t ldo, void* stream) {
  FBFP_CHECK_ARG(exponents && signs && payload && out, "null pointer");
  FBFP_CHECK_ARG(n_out > 0 && k_in > 0 && kpad >= k_in && kpad % kBlock == 0 && ldo >= k_in && ldo % 8 == 0,
                 "bad shape n_out=%lld k_in=%lld kpad=%lld ldo=%lld", (long long)n_out, (long long)k_in,
                 (long long)kpad, (long long)ldo);
  FBFP_CHECK_ARG(((uintptr_t)payload & 7) == 0 && ((uintptr_t)out & 15) == 0,
                 "payload must be 8-byte and out 16-byte aligned");
  const bool tiles = entries && seg_ptr;
  FBFP_CHECK_ARG(tiles || count == 0 || (count > 0 && block_idx && offset && value_f16), "bad outlier list");
  FBFP_CHECK_ARG(!tiles || npad >= n_out, "npad < n_out");
  cudaStream_t st = as_stream(stream);
  const int64_t kb_row = kpad / kBlock, kb_used = (k_in + kBlock - 1) / kBlock;
  uint16_t* o = static_cast<uint16_t*>(out);
  TileIndex tix = {nullptr, nullptr, 0, 0};
  if (tiles) {
    const int64_t n_stages = (kb_row + 15) / 16, nseg = ((npad + 127) / 128) * n_stages;
    tix = {entries, seg_ptr, n_stages, (nseg + 1 + 3) & ~(int64_t)3};
  }
  const int threads = 128;
  const int64_t gx = (kb_used + threads - 1) / threads;
  const int64_t gy = n_out < 32768 ? n_out : 32768;
  expand_x15_kernel<<<dim3((unsigned)gx, (unsigned)gy), threads, 0, st>>>(
      exponents, signs, reinterpret_cast<const uint2*>(payload), n_out, k_in, kb_row, kb_used, tix, o, ldo);
  FBFP_LAUNCH_CHECK("expand_x15_kernel");
  if (!tiles && count > 0) {
    scatter_x15_kernel<<<grid_blocks(count, 256), 256, 0, st>>>(block_idx, offset, value_f16, count, kpad,
                                                                n_out, k_in, o, ldo);
    FBFP_LAUNCH_CHECK("scatter_x15_kernel");
  }
  return FBFP_OK;
}

extern "C" int fbfp_gemm_expanded(const void* x, int64_t m, int64_t ldx, const int8_t* exponents,
                                  const int16_t* signs, const int32_t* payload, int64_t n_out, int64_t k_in,
                                  int64_t kpad, const int32_t* block_idx, const int32_t* offset,
                                  const uint16_t* value_f16, int64_t count, const uint32_t* entries,
                                  const int32_t* seg_ptr, int64_t npad, const void* bias, void* y,
                                  int y_dtype, int64_t ldy, void* scratch, int64_t scratch_bytes,
                                  void* stream) {
  FBFP_CHECK_ARG(x && y && scratch, "null pointer");
  FBFP_CHECK_ARG(y_dtype == FBFP_BF16 || y_dtype == FBFP_F32, "y_dtype must be bf16 or f32");
  const int64_t ysz = y_dtype == FBFP_F32 ? 4 : 2;
  FBFP_CHECK_ARG(m > 0 && ldx >= k_in && ldy >= n_out && ldx % 8 == 0 && (ldy * ysz) % 16 == 0,
                 "bad shape m=%lld ldx=%lld ldy=%lld", (long long)m, (long long)ldx, (long long)ldy);
  FBFP_CHECK_ARG(((uintptr_t)x & 15) == 0 && ((uintptr_t)y & 15) == 0 && ((uintptr_t)scratch & 255) == 0 &&
                 (!bias || ((uintptr_t)bias & 15) == 0),
                 "x, y and bias must be 16-byte and scratch 256-byte aligned");
  FBFP_CHECK_ARG(kpad > 0 && scratch_bytes >= fbfp_gemm_expanded_scratch_bytes(n_out, kpad),
                 "scratch of %lld bytes is smaller than fbfp_gemm_expanded_scratch_bytes (%lld)",
                 (long long)scratch_bytes, (long long)fbfp_gemm_expanded_scratch_bytes(n_out, kpad));
  int rc = fbfp_expand_x15(exponents, signs, payload, n_out, k_in, kpad, block_idx, offset, value_f16, count,
                           entries, seg_ptr, npad, scratch, kpad, stream);
  if (rc != FBFP_OK) return rc;
  int dev = 0;
  FBFP_CUDA_TRY(cudaGetDevice(&dev));
  uint8_t* lt_ws = static_cast<uint8_t*>(scratch) + expand_matrix_bytes(n_out, kpad);
  return lt_gemm_x15(x, m, ldx, scratch, kpad, n_out, k_in, bias, y, y_dtype, ldy, lt_ws, as_stream(stream),
                     dev);
}
