// gemv.cu — fused OABF dequant-GEMV for decode (1 <= M <= 16 tokens) on sm_100a.
//
// Replaces oabf_gemm_kernel (flash_bfp/triton_kernel.py:22-86) for small M together with
// the outlier SpMV and bias of OABFLinear.forward (triton_kernel.py:339-362):
//     y[m, n] = sum_k x[m, k] * W_full[n, k] + bias[n]       (fp32 accumulation)
//
// Weights stream straight from the packed reference layout (11 bytes per 16 weights) and
// are dequantised in registers into bf16 tensor-core operands:
//   * a lane owns a whole 16-element block of its two rows (g, g+8) for four consecutive
//     mma.m16n8k16 steps (the k-slots of a step belong to four different blocks — the dot
//     product does not care, and the activation fragment is permuted to match), so the
//     per-block work (sign spread, exponent) is paid once per 16 weights;
//   * a weight pair (elements q, q+4 of nibble word w) becomes the bf16 pair
//     +-(128 + m) * 2^e by bit operations only: mantissa nibble into bits 0-3, exponent
//     field (e + 134) into bits 7-14, sign into bit 15. A second MMA with the pair
//     -+128 * 2^e (same signs/exponent, no nibble) against the same activations cancels
//     the 128 offset inside the tensor core, leaving sum(s * m * 2^e * x); the 1/15 of the
//     format is applied once in the epilogue;
//   * the activation chunk is staged in shared memory permuted into fragment order, with a
//     negated copy for the cancelling MMA, 16-byte pieces XOR-swizzled by k-block.
// Work split: a CTA of 8 warps covers 64 rows x one 64-block (1024-column) chunk of K; each
// warp takes a 16-row tile and half of the chunk. Partial sums of the chunks meet in an fp32
// workspace via red.global.add; the last warp to arrive at a row tile (arrival counter)
// adds bias, converts, stores y and returns the workspace and counter to zero.
// Outliers are pre-grouped by (row tile, chunk) (fbfp_outlier_tiles_build) and handled by
// the two warps of that tile/chunk with shared-memory float atomics.
#include "common.cuh"
#include "scan.cuh"
#include "tc_args.h"

namespace fbfp {

int launch_gemv_tc(const TcArgs& a, cudaStream_t st);
bool gemv_tc_eligible(int64_t m, int64_t kb_row, int64_t k_in, int x_dtype, int64_t ldx, const void* x,
                      const void* pay, const void* sg, const void* ex);

constexpr int kGemvWarps = 8;
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kRowsPerCta = 64;        // 4 row tiles of 16
constexpr int kHalfKb = 32;            // k-blocks per warp (half a chunk)

struct GemvArgs {
  const void* x;
  int x_dtype, m;
  int64_t ldx;
  const int8_t* ex;
  const uint16_t* sg;
  const uint2* pay;
  int64_t n_out, k_in, kb_row, npad;
  const uint32_t* entries;
  const int32_t* seg_ptr;
  const void* bias;
  int bias_dtype;
  void* y;
  int y_dtype;
  int64_t ldy;
  float* ws;           // [m][npad] fp32 partial sums
  int32_t* counters;   // [ceil(npad/16)] arrivals per row tile
  int n_chunks;
  bool vec;           // 16-byte vector loads of 8-block spans are legal
};

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0,
                                               uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void red_add_f32(float* p, float v) {
  asm volatile("red.global.add.f32 [%0], %1;\n" ::"l"(p), "f"(v) : "memory");
}

// Activation element position inside the staged chunk: element el (0..15) of k-block kbl,
// token tok. Piece 0 holds pairs (0,4)(1,5)(2,6)(3,7), piece 1 pairs (8,12)..(11,15),
// pieces 2/3 the negated copies. Lane t reads k-block 8t + j, so piece p of (kbl, tok) sits
// at slot p ^ ((kbl >> 3) & 3): the four lanes of a quad hit four different bank groups.
__device__ __forceinline__ int x_piece_slot(int kbl, int tok, int m, int piece) {
  return ((kbl * m + tok) << 2) + (piece ^ ((kbl >> 3) & 3));
}

// Packed data of one row for the 8 consecutive blocks a lane owns.
struct RowBlocks {
  uint4 p[4];        // payload: p[c] = {w0, w1} of block 2c, {w0, w1} of block 2c+1
  uint4 s;           // sign words, block j in halfword j
  uint2 e;           // exponents, block j in byte j
};

__device__ __forceinline__ void load_row_blocks(const GemvArgs& a, int64_t row, int kbt, int nblk,
                                                bool vec, RowBlocks& r) {
  if (nblk == 8 && vec) {
    const int64_t b = row * a.kb_row + kbt;
    const uint4* pp = reinterpret_cast<const uint4*>(a.pay + b);
#pragma unroll
    for (int c = 0; c < 4; ++c) r.p[c] = __ldg(pp + c);
    r.s = __ldg(reinterpret_cast<const uint4*>(a.sg + b));
    r.e = __ldg(reinterpret_cast<const uint2*>(a.ex + b));
    return;
  }
  uint32_t w[16], sw[4] = {0u, 0u, 0u, 0u}, ew[2] = {0u, 0u};
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    uint2 pj = make_uint2(0u, 0u);
    uint32_t sj = 0u, ej = 0u;
    if (j < nblk) {
      const int64_t b = row * a.kb_row + kbt + j;
      pj = __ldg(a.pay + b);
      sj = __ldg(a.sg + b);
      ej = (uint32_t)(uint8_t)__ldg(a.ex + b);
    }
    w[2 * j] = pj.x;
    w[2 * j + 1] = pj.y;
    sw[j >> 1] |= sj << (16 * (j & 1));
    ew[j >> 2] |= ej << (8 * (j & 3));
  }
#pragma unroll
  for (int c = 0; c < 4; ++c) r.p[c] = make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
  r.s = make_uint4(sw[0], sw[1], sw[2], sw[3]);
  r.e = make_uint2(ew[0], ew[1]);
}

template <int NT>
__global__ void __launch_bounds__(kGemvThreads, 2)
gemv_kernel(const GemvArgs a) {
  extern __shared__ uint4 xs[];                            // [64 kb][m][4] pieces
  __shared__ float s_out[kGemvWarps][16][16];              // outlier partials [token][row]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int m = a.m;
  const int chunk = blockIdx.y;
  const int kb_c0 = chunk * kChunkKb;
  const int kb_c1 = (int)min((int64_t)kb_c0 + kChunkKb, a.kb_row);
  const int nkb = kb_c1 - kb_c0;

  // ---- issue this lane's weight loads first: 8 blocks x 2 rows, independent of X ----
  const int64_t rt = (int64_t)blockIdx.x * 4 + (warp & 3);
  const bool tile_ok = rt * 16 < a.npad;
  const int half = warp >> 2;
  const int64_t row0 = rt * 16 + g, row1 = row0 + 8;
  const bool rv0 = tile_ok && row0 < a.npad, rv1 = tile_ok && row1 < a.npad;
  const int kb_lo = kb_c0 + half * kHalfKb;
  const int kb_hi = min(kb_lo + kHalfKb, kb_c1);
  const int kbt = kb_lo + 8 * t;                           // this lane's first block
  const int nblk = max(0, min(8, kb_hi - kbt));
  const bool vec = a.vec;
  RowBlocks R0, R1;
  load_row_blocks(a, row0, kbt, rv0 ? nblk : 0, vec, R0);
  load_row_blocks(a, row1, kbt, rv1 ? nblk : 0, vec, R1);

  // ---- stage the activation chunk (bf16, permuted, with negated copy) ----
  for (int idx = threadIdx.x; idx < nkb * m; idx += kGemvThreads) {
    const int kbl = idx / m, tok = idx - kbl * m;
    const int64_t k0 = (int64_t)(kb_c0 + kbl) * kBlock;
    uint32_t h[16];
    if (a.x_dtype == FBFP_BF16) {
      const uint16_t* xr = reinterpret_cast<const uint16_t*>(a.x) + tok * a.ldx + k0;
      if (k0 + 16 <= a.k_in && ((uintptr_t)xr & 15) == 0) {
        const uint4 q0 = reinterpret_cast<const uint4*>(xr)[0];
        const uint4 q1 = reinterpret_cast<const uint4*>(xr)[1];
        const uint32_t u[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) { h[2 * j] = u[j] & 0xFFFF; h[2 * j + 1] = u[j] >> 16; }
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) h[j] = (k0 + j < a.k_in) ? xr[j] : 0u;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j)
        h[j] = (k0 + j < a.k_in) ? float_to_bf16_bits(load_as_float(a.x, a.x_dtype, tok * a.ldx + k0 + j)) : 0u;
    }
    uint4 p0, p1;
    p0.x = h[0] | (h[4] << 16);  p0.y = h[1] | (h[5] << 16);
    p0.z = h[2] | (h[6] << 16);  p0.w = h[3] | (h[7] << 16);
    p1.x = h[8] | (h[12] << 16); p1.y = h[9] | (h[13] << 16);
    p1.z = h[10] | (h[14] << 16); p1.w = h[11] | (h[15] << 16);
    const uint32_t NEG = 0x80008000u;
    const uint4 n0 = make_uint4(p0.x ^ NEG, p0.y ^ NEG, p0.z ^ NEG, p0.w ^ NEG);
    const uint4 n1 = make_uint4(p1.x ^ NEG, p1.y ^ NEG, p1.z ^ NEG, p1.w ^ NEG);
    xs[x_piece_slot(kbl, tok, m, 0)] = p0;
    xs[x_piece_slot(kbl, tok, m, 1)] = p1;
    xs[x_piece_slot(kbl, tok, m, 2)] = n0;
    xs[x_piece_slot(kbl, tok, m, 3)] = n1;
  }
  for (int i = lane; i < 256; i += 32) (&s_out[warp][0][0])[i] = 0.f;
  __syncthreads();
  if (!tile_ok) return;                                     // row tile past the matrix

  float acc[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;

  // exponent bytes -> e + 134 per byte without carries (e in [-128, 121])
  const uint32_t E0lo = (R0.e.x ^ 0x80808080u) + 0x06060606u, E0hi = (R0.e.y ^ 0x80808080u) + 0x06060606u;
  const uint32_t E1lo = (R1.e.x ^ 0x80808080u) + 0x06060606u, E1hi = (R1.e.y ^ 0x80808080u) + 0x06060606u;
  const uint32_t sw0[4] = {R0.s.x, R0.s.y, R0.s.z, R0.s.w};
  const uint32_t sw1[4] = {R1.s.x, R1.s.y, R1.s.z, R1.s.w};
  const int kbl0 = kbt - kb_c0;

#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint4 P0 = R0.p[j >> 1], P1 = R1.p[j >> 1];
    const uint32_t w00 = (j & 1) ? P0.z : P0.x, w01 = (j & 1) ? P0.w : P0.y;   // row g
    const uint32_t w10 = (j & 1) ? P1.z : P1.x, w11 = (j & 1) ? P1.w : P1.y;   // row g+8
    const uint32_t s0 = (j & 1) ? (sw0[j >> 1] >> 16) : (sw0[j >> 1] & 0xFFFFu);
    const uint32_t s1 = (j & 1) ? (sw1[j >> 1] >> 16) : (sw1[j >> 1] & 0xFFFFu);
    const uint32_t y0 = s0 | (s0 << 12), y1 = s1 | (s1 << 12);
    const uint32_t eb0 = (((j < 4) ? E0lo : E0hi) >> (8 * (j & 3))) & 0xFFu;
    const uint32_t eb1 = (((j < 4) ? E1lo : E1hi) >> (8 * (j & 3))) & 0xFFu;
    const uint32_t K0 = eb0 * 0x00800080u, K1 = eb1 * 0x00800080u;
    const bool valid = j < nblk;

    uint32_t xv[NT][8], xn[NT][8];
    const int kbl = kbl0 + j;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const int tok = n * 8 + g;
      if (valid && tok < m) {
        const uint4 q0 = xs[x_piece_slot(kbl, tok, m, 0)];
        const uint4 q1 = xs[x_piece_slot(kbl, tok, m, 1)];
        const uint4 q2 = xs[x_piece_slot(kbl, tok, m, 2)];
        const uint4 q3 = xs[x_piece_slot(kbl, tok, m, 3)];
        xv[n][0] = q0.x; xv[n][1] = q0.y; xv[n][2] = q0.z; xv[n][3] = q0.w;
        xv[n][4] = q1.x; xv[n][5] = q1.y; xv[n][6] = q1.z; xv[n][7] = q1.w;
        xn[n][0] = q2.x; xn[n][1] = q2.y; xn[n][2] = q2.z; xn[n][3] = q2.w;
        xn[n][4] = q3.x; xn[n][5] = q3.y; xn[n][6] = q3.z; xn[n][7] = q3.w;
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) { xv[n][i] = 0u; xn[n][i] = 0u; }
      }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t SM = 0x80008000u, NM = 0x000F000Fu;
      const uint32_t cA0 = ((y0 << (15 - q)) & SM) | K0;   // row g,   elements q, q+4
      const uint32_t cB0 = ((y0 << (7 - q)) & SM) | K0;    // row g,   elements q+8, q+12
      const uint32_t cA1 = ((y1 << (15 - q)) & SM) | K1;   // row g+8
      const uint32_t cB1 = ((y1 << (7 - q)) & SM) | K1;
      const uint32_t vA0 = ((w00 >> (4 * q)) & NM) | cA0;
      const uint32_t vB0 = ((w01 >> (4 * q)) & NM) | cB0;
      const uint32_t vA1 = ((w10 >> (4 * q)) & NM) | cA1;
      const uint32_t vB1 = ((w11 >> (4 * q)) & NM) | cB1;
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        mma_bf16_16816(acc[n], vA0, vA1, vB0, vB1, xv[n][q], xv[n][4 + q]);
        mma_bf16_16816(acc[n], cA0, cA1, cB0, cB1, xn[n][q], xn[n][4 + q]);
      }
    }
  }

  // ---- outliers of this row tile in this warp's 32 k-blocks: the (128-row group,
  //      16-block stage) segments covering them, filtered to the tile's 16 rows ----
  if (a.entries) {
    const int64_t rg = rt / 8;
    const int r_lo = (int)(rt % 8) * 16;
    const int n_stages = (int)((a.kb_row + kStageKb - 1) / kStageKb);
    const uint16_t* xh = reinterpret_cast<const uint16_t*>(xs);
    for (int st = kb_lo / kStageKb; st * kStageKb < kb_hi; ++st) {
      const int64_t seg = rg * n_stages + st;
      const int lo = a.seg_ptr[seg], hi = a.seg_ptr[seg + 1];
      for (int i = lo + lane; i < hi; i += 32) {
        const uint32_t e = __ldg(a.entries + i);
        const int r = (int)(e >> 24) - r_lo;
        if (r < 0 || r >= 16) continue;
        const float v = __half2float(__ushort_as_half((unsigned short)(e & 0xFFFF)));
        const int col = st * kStageKb * kBlock + (int)((e >> 16) & 0xFF) - kb_c0 * kBlock;
        const int kbl = col >> 4, el = col & 15;
        const int piece = el >> 3, e7 = el & 7;
        const int pos = ((e7 & 3) << 1) + (e7 >> 2);
        for (int tok = 0; tok < m; ++tok) {
          const float xv = bf16_bits_to_float(xh[x_piece_slot(kbl, tok, m, piece) * 8 + pos]);
          atomicAdd(&s_out[warp][tok][r], v * xv);
        }
      }
    }
    __syncwarp();
  }

  // ---- fold into the fp32 workspace ----
  const float inv15 = 1.0f / 15.0f;
#pragma unroll
  for (int n = 0; n < NT; ++n) {
    const int tk0 = n * 8 + 2 * t, tk1 = tk0 + 1;
    if (rv0) {
      if (tk0 < m) red_add_f32(a.ws + (int64_t)tk0 * a.npad + row0, acc[n][0] * inv15 + s_out[warp][tk0][g]);
      if (tk1 < m) red_add_f32(a.ws + (int64_t)tk1 * a.npad + row0, acc[n][1] * inv15 + s_out[warp][tk1][g]);
    }
    if (rv1) {
      if (tk0 < m) red_add_f32(a.ws + (int64_t)tk0 * a.npad + row1, acc[n][2] * inv15 + s_out[warp][tk0][g + 8]);
      if (tk1 < m) red_add_f32(a.ws + (int64_t)tk1 * a.npad + row1, acc[n][3] * inv15 + s_out[warp][tk1][g + 8]);
    }
  }
  __threadfence();
  __syncwarp();
  int last = 0;
  if (lane == 0) last = atomicAdd(a.counters + rt, 1) == 2 * a.n_chunks - 1;
  last = __shfl_sync(0xffffffffu, last, 0);
  if (!last) return;

  // ---- epilogue of the row tile: bias, convert, store, clear the workspace ----
  __threadfence();
  for (int idx = lane; idx < 16 * m; idx += 32) {
    const int tok = idx >> 4, r = idx & 15;
    const int64_t row = rt * 16 + r;
    if (row >= a.npad) continue;
    float* wp = a.ws + (int64_t)tok * a.npad + row;
    float v = __ldcg(wp);
    __stcg(wp, 0.f);
    if (row < a.n_out) {
      if (a.bias) v += load_as_float(a.bias, a.bias_dtype, row);
      store_from_float(a.y, a.y_dtype, (int64_t)tok * a.ldy + row, v);
    }
  }
  if (lane == 0) a.counters[rt] = 0;
}

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace fbfp

using namespace fbfp;

// Workspace layout: [error word + pad: 256 B][arrival counters: ceil(npad/16) int32]
// [fp32 partial sums: m x npad]; every region is zero between calls, so one workspace
// sized for the largest npad serves matrices of any smaller size.
static size_t ws_counters_bytes(int64_t npad) {
  return align256(sizeof(int32_t) * (size_t)((npad + 15) / 16));
}

extern "C" int64_t fbfp_gemv_workspace_bytes(int64_t m, int64_t npad) {
  return (int64_t)(256 + ws_counters_bytes(npad) + align256(sizeof(float) * (size_t)(m * npad)));
}

namespace fbfp {
// The regions of a GEMV workspace for a matrix of npad rows (shared with gemv_rec.cu).
int gemv_workspace_parts(void* workspace, int64_t npad, int32_t** err, int32_t** counters, float** ws) {
  FBFP_CHECK_ARG(workspace, "null workspace");
  char* base = reinterpret_cast<char*>(workspace);
  *err = reinterpret_cast<int32_t*>(base);
  *counters = reinterpret_cast<int32_t*>(base + 256);
  *ws = reinterpret_cast<float*>(base + 256 + ws_counters_bytes(npad));
  return FBFP_OK;
}
}  // namespace fbfp

namespace fbfp {
int noalloc_scratch(void** out);
}

extern "C" int fbfp_gemv_check(void* workspace, void* stream) {
  if (!workspace) {                       // the built-in scratch of fbfp_gemv_noalloc
    const int rc = noalloc_scratch(&workspace);
    if (rc != FBFP_OK) return rc;
  }
  cudaStream_t st = as_stream(stream);
  int32_t* errp = reinterpret_cast<int32_t*>(workspace);
  int32_t h = 0;
  FBFP_CUDA_TRY(cudaMemcpyAsync(&h, errp, sizeof(h), cudaMemcpyDeviceToHost, st));
  FBFP_CUDA_TRY(cudaStreamSynchronize(st));
  if (h != 0) {
    FBFP_CUDA_TRY(cudaMemsetAsync(errp, 0, sizeof(int32_t), st));
    if (h >= 32)
      return set_error(FBFP_ERR_TIMEOUT, "fused exchange: gave up waiting for rank %d", (int)h - 32);
    return set_error(FBFP_ERR_TIMEOUT, "a bounded device-side wait gave up (site %d)", (int)h);
  }
  return FBFP_OK;
}

namespace fbfp {
int allreduce_buffers(void* handle, uint8_t** bufs, int* world, int* rank, int64_t* max_elems);
uint64_t allreduce_timeout_ns(void* handle);
}

// resident != 0: the packed weights and outlier index were not written by the previous kernel in
// the stream, so the tcgen05 kernel may fetch its first weight stages before that kernel ends.
// allreduce != null: the row-parallel exchange through that all-reduce handle is fused into the
// tcgen05 kernel's epilogue (y = bias + the sum over ranks of their partial products).
namespace fbfp {
// Argument checks shared by every GEMV entry point (the workspace is checked by the caller).
int gemv_validate(const void* x, int x_dtype, int64_t m, int64_t ldx, const int8_t* exponents,
                  const int16_t* signs, const int32_t* payload, int64_t n_out, int64_t k_in,
                  int64_t kpad, int64_t npad, const uint32_t* entries, const int32_t* seg_ptr,
                  const void* bias, int bias_dtype, const void* y, int y_dtype, int64_t ldy) {
  FBFP_CHECK_ARG(x && exponents && signs && payload && y, "null pointer");
  FBFP_CHECK_ARG(m >= 1 && m <= 16, "fbfp_gemv needs 1 <= m <= 16 (got %lld)", (long long)m);
  FBFP_CHECK_ARG(dtype_ok(x_dtype), "x_dtype must be f32, bf16 or f16");
  FBFP_CHECK_ARG(dtype_ok(y_dtype), "y_dtype must be f32, bf16 or f16");
  FBFP_CHECK_ARG(!bias || dtype_ok(bias_dtype), "bad bias dtype");
  FBFP_CHECK_ARG(n_out > 0 && k_in > 0 && kpad >= k_in && kpad % kBlock == 0 && npad >= n_out,
                 "bad shape");
  FBFP_CHECK_ARG(ldx >= k_in && ldy >= n_out, "bad leading dimension");
  FBFP_CHECK_ARG(!entries || seg_ptr, "entries without seg_ptr");
  FBFP_CHECK_ARG(((uintptr_t)payload & 7) == 0, "payload must be 8-byte aligned");
  return FBFP_OK;
}
}  // namespace fbfp

static int gemv_impl(const void* x, int x_dtype, int64_t m, int64_t ldx,
                     const int8_t* exponents, const int16_t* signs, const int32_t* payload,
                     int64_t n_out, int64_t k_in, int64_t kpad, int64_t npad,
                     const uint32_t* entries, const int32_t* seg_ptr, const void* bias,
                     int bias_dtype, void* y, int y_dtype, int64_t ldy, void* workspace,
                     void* stream, int resident, void* allreduce) {
  const int vrc = gemv_validate(x, x_dtype, m, ldx, exponents, signs, payload, n_out, k_in, kpad, npad,
                                entries, seg_ptr, bias, bias_dtype, y, y_dtype, ldy);
  if (vrc != FBFP_OK) return vrc;
  FBFP_CHECK_ARG(workspace, "null pointer (workspace)");
  FBFP_CHECK_ARG(((uintptr_t)workspace & 255) == 0, "workspace must be 256-byte aligned");
  const int64_t kb_row = kpad / kBlock;
  const int n_chunks = (int)((kb_row + kChunkKb - 1) / kChunkKb);
  GemvArgs a;
  a.x = x; a.x_dtype = x_dtype; a.m = (int)m; a.ldx = ldx;
  a.ex = exponents; a.sg = reinterpret_cast<const uint16_t*>(signs);
  a.pay = reinterpret_cast<const uint2*>(payload);
  a.n_out = n_out; a.k_in = k_in; a.kb_row = kb_row; a.npad = npad;
  a.entries = entries; a.seg_ptr = seg_ptr;
  a.bias = bias; a.bias_dtype = bias_dtype;
  a.y = y; a.y_dtype = y_dtype; a.ldy = ldy;
  int32_t* errp = reinterpret_cast<int32_t*>(workspace);
  a.counters = reinterpret_cast<int32_t*>(reinterpret_cast<char*>(workspace) + 256);
  a.ws = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + 256 + ws_counters_bytes(npad));
  a.n_chunks = n_chunks;
  a.vec = (kb_row % 8 == 0) && ((uintptr_t)payload % 16 == 0) && ((uintptr_t)signs % 16 == 0) &&
          ((uintptr_t)exponents % 8 == 0);
  cudaStream_t st = as_stream(stream);
  const bool tc = gemv_tc_eligible(m, kb_row, k_in, x_dtype, ldx, x, payload, signs, exponents);
  FBFP_CHECK_ARG(tc || !allreduce,
                 "the fused exchange needs the tensor-core GEMV: bf16 x, 16-byte aligned operands, "
                 "kpad a multiple of 256, k_in and ldx multiples of 8");
  if (tc) {
    TcArgs t;
    t.x = x; t.x_dtype = x_dtype; t.m = (int)m; t.ldx = ldx;
    t.ex = exponents; t.sg = reinterpret_cast<const uint16_t*>(signs);
    t.pay = reinterpret_cast<const uint2*>(payload);
    t.n_out = n_out; t.k_in = k_in; t.kb_row = kb_row; t.npad = npad;
    t.entries = entries; t.seg_ptr = seg_ptr; t.bias = bias; t.bias_dtype = bias_dtype;
    t.y = y; t.y_dtype = y_dtype; t.ldy = ldy;
    t.ws = a.ws; t.counters = a.counters; t.err = errp;
    t.n_stages = (int)(kb_row / kStageKb);
    t.total_units = ((npad + kGroupRows - 1) / kGroupRows) * t.n_stages;
    t.early_weights = resident ? 1 : 0;
    t.world = 1; t.rank = 0; t.xmax = 0; t.exit_count = errp + 1; t.xchg_timeout_ns = 0;
    for (int p = 0; p < 8; ++p) t.xbuf[p] = nullptr;
    if (allreduce) {
      int rc = allreduce_buffers(allreduce, t.xbuf, &t.world, &t.rank, &t.xmax);
      if (rc != FBFP_OK) return rc;
      FBFP_CHECK_ARG(m * n_out <= t.xmax, "m * n_out = %lld exceeds the all-reduce handle's %lld elements",
                     (long long)(m * n_out), (long long)t.xmax);
      t.xchg_timeout_ns = allreduce_timeout_ns(allreduce);
    }
    return launch_gemv_tc(t, st);
  }
  const dim3 grid((unsigned)((npad + kRowsPerCta - 1) / kRowsPerCta), (unsigned)n_chunks);
  const size_t smem = sizeof(uint4) * 4 * (size_t)kChunkKb * (size_t)m;
  if (m <= 8) {
    if (smem > 48 * 1024)
      FBFP_CUDA_TRY(cudaFuncSetAttribute(gemv_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    gemv_kernel<1><<<grid, kGemvThreads, smem, st>>>(a);
  } else {
    if (smem > 48 * 1024)
      FBFP_CUDA_TRY(cudaFuncSetAttribute(gemv_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    gemv_kernel<2><<<grid, kGemvThreads, smem, st>>>(a);
  }
  FBFP_LAUNCH_CHECK("gemv_kernel");
  return FBFP_OK;
}

extern "C" int fbfp_gemv(const void* x, int x_dtype, int64_t m, int64_t ldx,
                         const int8_t* exponents, const int16_t* signs, const int32_t* payload,
                         int64_t n_out, int64_t k_in, int64_t kpad, int64_t npad,
                         const uint32_t* entries, const int32_t* seg_ptr, const void* bias,
                         int bias_dtype, void* y, int y_dtype, int64_t ldy, void* workspace,
                         void* stream) {
  return gemv_impl(x, x_dtype, m, ldx, exponents, signs, payload, n_out, k_in, kpad, npad, entries,
                   seg_ptr, bias, bias_dtype, y, y_dtype, ldy, workspace, stream, 0, nullptr);
}

extern "C" int fbfp_gemv_resident(const void* x, int x_dtype, int64_t m, int64_t ldx,
                                  const int8_t* exponents, const int16_t* signs, const int32_t* payload,
                                  int64_t n_out, int64_t k_in, int64_t kpad, int64_t npad,
                                  const uint32_t* entries, const int32_t* seg_ptr, const void* bias,
                                  int bias_dtype, void* y, int y_dtype, int64_t ldy, void* workspace,
                                  void* stream) {
  return gemv_impl(x, x_dtype, m, ldx, exponents, signs, payload, n_out, k_in, kpad, npad, entries,
                   seg_ptr, bias, bias_dtype, y, y_dtype, ldy, workspace, stream, 1, nullptr);
}

extern "C" int fbfp_gemv_allreduce(const void* x, int x_dtype, int64_t m, int64_t ldx,
                                   const int8_t* exponents, const int16_t* signs,
                                   const int32_t* payload, int64_t n_out, int64_t k_in, int64_t kpad,
                                   int64_t npad, const uint32_t* entries, const int32_t* seg_ptr,
                                   const void* bias, int bias_dtype, void* y, int y_dtype, int64_t ldy,
                                   void* workspace, void* allreduce, int resident, void* stream) {
  FBFP_CHECK_ARG(allreduce, "null all-reduce handle");
  return gemv_impl(x, x_dtype, m, ldx, exponents, signs, payload, n_out, k_in, kpad, npad, entries,
                   seg_ptr, bias, bias_dtype, y, y_dtype, ldy, workspace, stream, resident ? 1 : 0,
                   allreduce);
}

namespace fbfp {
__global__ void stream_fence_kernel() {}
}  // namespace fbfp

extern "C" int fbfp_stream_fence(void* stream) {
  stream_fence_kernel<<<1, 32, 0, as_stream(stream)>>>();
  FBFP_LAUNCH_CHECK("stream_fence_kernel");
  return FBFP_OK;
}
