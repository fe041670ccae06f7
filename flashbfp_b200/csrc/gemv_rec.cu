// gemv_rec.cu — OABF decode GEMV on the stage-record layout (tcgen05, sm_100a).
//
// Same product as fbfp_gemv (y = x W_full^T + bias for 1 <= M <= 16 bf16 tokens; replaces
// oabf_gemm_kernel, flash_bfp/triton_kernel.py:22-86, and the outlier SpMV and bias of
// OABFLinear.forward, :339-362), reading the weights and outliers from one device buffer built
// once at load time (fbfp_records_build) instead of the reference's arrays.
//
// Records buffer: a table of total_units + 1 int64 byte offsets (the last = end), padded to 256
// bytes, then one record per unit u = g * n_stages + st (128-row group g, 256-column stage st),
// starting at offset[u] (a multiple of 16), fetched with a single bulk copy:
//   [0, 20480)      fields: every weight as the 5-bit value f = 16 + s*m (s = +-1 the sign,
//                   m the 4-bit mantissa; 80 bits per 16-weight block, as signs + nibbles). Per
//                   substage c (blocks 4c .. 4c+3, 5120 bytes) three chunks, row-interleaved so
//                   that a lane reading its row's words conflicts with no other lane:
//                     [c*5120 + row*16]          words 0-3 of the row
//                     [c*5120 + 2048 + row*16]   words 4-7
//                     [c*5120 + 4096 + row*8]    words 8-9
//                   Words 0-4 hold blocks 4c and 4c+1, words 5-9 blocks 4c+2 and 4c+3. In a
//                   block pair (words w0..w4) pair P = 8b + j is elements (2j, 2j+1) of block b;
//                   for P < 15 its two fields sit at bits 5*(P%3) and 16 + 5*(P%3) of word P/3;
//                   pair 15's fields are spread over bits 15 and 31 of w0..w4 (bit i of each
//                   field in word i).
//   [20480, 22528)  biased exponents eb = e + 134 (uint8), at 20480 + c*512 + row*4 + block%4.
//   [22528, 22800)  the unit's outliers per row: 136 uint16 row starts (entry 128 = count).
//   [22816, ...)    the unit's outlier entries, uint32 fp16 bits | column << 16 | row << 24,
//                   ordered by (row, column), padded to 16 bytes.
// Dequantisation of a pair is exact bit arithmetic: with K = eb * 0x00800080 and
// C = K + 0x00100010, the bf16 pair (K | f) - C equals (f - 16) * 2^e = s*m*2^e for both
// elements: one shift, one LOP3 and one HSUB2 per pair (the format's 1/15 is applied once to
// the accumulator). -0.0 becomes +0.0, which changes no product.
//
// Kernel roles, one persistent CTA per SM (warp-specialised):
//   warp 0      weight producer: one bulk copy per record (fields, exponents and outliers, up to
//               the stage size; the rest of a long outlier list is read from global memory) into
//               an NW-deep ring, before the grid-dependency wait when the weights are resident;
//   warp 1      MMA issuer: per block one tcgen05.mma M=128 N=16 K=16, A from tensor memory,
//               B the unit's activations (K-major, 128-byte swizzle) in shared memory,
//               double-buffered fp32 accumulator in tensor memory;
//   warp 2      activation producer: per unit four 64-k tensor boxes into an NX-deep ring;
//   warps 4-7   epilogue (one per tensor-memory lane quarter, one row per lane): the row's
//               outliers times the activations in fp32 each unit, then per (row group, CTA)
//               segment the accumulator, the bias and the output (directly, or through an fp32
//               workspace with per-(row group, quarter) arrival counters when several CTAs
//               share the row group); with the row-parallel exchange fused in, the finished
//               rows are pushed to every peer and summed in rank order (exchange.cuh);
//   warps 8..   dequantisers, DQ per lane quarter: warp (quarter q, index p) turns substages
//               c = p (mod DQ) of every unit into A operands (tcgen05.st into an NS-slot ring).
// The activations have a ring of their own, as deep as the latency of a copy under full HBM
// load needs (about 2.5 us): tying them to a shallow ring serialises the units on that latency.
// Work is split stream-K over the units (each CTA a contiguous range). Every wait is bounded:
// on timeout the CTA records an error code in the workspace (fbfp_gemv_check) and winds down.
#include <cuda.h>

#include "common.cuh"
#include "sm100.cuh"
#include "tc_host.h"
#include "exchange.cuh"
#include "scan.cuh"

namespace fbfp {
using namespace sm100;

namespace rec {
constexpr int kFieldBytes = 20480;
constexpr int kExpOff = kFieldBytes;
constexpr int kRoffOff = kFieldBytes + 2048;            // 22528
constexpr int kEntOff = 22816;                          // outlier entries
constexpr int kStageBytes = 27648;                      // 27 KB: up to 1208 staged entries
constexpr int kOutCap = (kStageBytes - kEntOff) / 4;
constexpr int kTableAlign = 256;
constexpr int kAcc = 1;                                 // accumulator chains per segment
constexpr uint32_t kTmemA = 2 * kAcc * 16;              // A ring after 2 x kAcc 16-column accumulators
constexpr int kOffCache = 512;                          // record offsets cached per CTA
constexpr int kEpiWarp0 = 4;
constexpr int kDqWarp0 = 8;
}  // namespace rec

__host__ __device__ constexpr int64_t rec_table_bytes(int64_t units) {
  return ((units + 1) * 8 + rec::kTableAlign - 1) / rec::kTableAlign * rec::kTableAlign;
}

// MT token rows per activation box (8 or 16), NW weight stages, NX activation stages, NS
// tensor-memory A slots of SB substages (4 blocks each; one MMA commit per slot), DQ dequantiser
// warps per lane quarter.
// Tensor memory: two segments' accumulators (double-buffered), each kAcc chains of 16 fp32
// columns, then the A ring.
template <int MT, int NW, int NX, int NS, int DQ, int SB>
struct RecCfg {
  static constexpr int kThreads = 32 * (rec::kDqWarp0 + 4 * DQ);
  static constexpr uint32_t kSlotCols = SB * 32;
  static constexpr uint32_t kTmemCols = rec::kTmemA + NS * kSlotCols <= 256 ? 256u : 512u;
  static_assert(rec::kTmemA + NS * kSlotCols <= 512, "tensor memory budget");
  static_assert(SB == 1 || SB == 2 || SB == 4, "1, 2 or 4 substages per A slot");
  static_assert(DQ == 1 || DQ == 2 || DQ == 4, "1, 2 or 4 dequantiser warps per lane quarter");
  static constexpr int kXBox = MT * 128;                // one box: 64 k x MT token rows
  static constexpr int kXBytes = 4 * kXBox;
  static constexpr size_t kXOff = (size_t)NW * rec::kStageBytes;
  static constexpr size_t kOffOff = kXOff + (size_t)NX * kXBytes + 1024;   // (+ the MMA's
  // reads of token rows 8-15 past the last box when MT = 8)
  static constexpr size_t kBarOff = kOffOff + (rec::kOffCache + 1) * sizeof(int64_t);
  static constexpr int kNumBars = 2 * NW + 2 * NX + 2 * NS + 4 + 1;
  static constexpr size_t kSmemBytes = kBarOff + kNumBars * 8 + 16 + 1024;   // + alignment slack
};

struct RecArgs {
  const void* x;
  int m;
  int64_t ldx;
  const uint8_t* rec;        // the records buffer (offset table first)
  int64_t n_out, k_in, npad;
  int n_stages;
  int64_t total_units;
  int outliers;              // 0: dense part only
  const void* bias;
  int bias_dtype;
  void* y;
  int y_dtype;
  int64_t ldy;
  float* ws;
  int32_t* counters;
  int32_t* err;
  int early_weights;
  int world, rank;
  uint8_t* xbuf[8];
  int64_t xmax;
  int32_t* exit_count;
  uint64_t xchg_timeout_ns;
};

struct RecMaps {
  CUtensorMap x;
};

struct RecShared {
  uint8_t* wring;
  uint8_t* xring;
  int64_t* off;              // offset[u0 .. u0 + kOffCache]
  uint64_t *full_w, *empty_w, *full_x, *empty_x, *afull, *aempty, *dfull, *dempty, *mtail;
  uint32_t* tmem_slot;
  volatile int* abort_flag;
};

template <class C, int NW, int NX, int NS>
__device__ __forceinline__ RecShared rec_shared(uint8_t* smem_raw) {
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  RecShared S;
  S.wring = smem;
  S.xring = smem + C::kXOff;
  S.off = reinterpret_cast<int64_t*>(smem + C::kOffOff);
  uint64_t* b = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  S.full_w = b;
  S.empty_w = S.full_w + NW;
  S.full_x = S.empty_w + NW;
  S.empty_x = S.full_x + NX;
  S.afull = S.empty_x + NX;
  S.aempty = S.afull + NS;
  S.dfull = S.aempty + NS;
  S.dempty = S.dfull + 2;
  S.mtail = S.dempty + 2;
  S.tmem_slot = reinterpret_cast<uint32_t*>(S.mtail + 1);
  S.abort_flag = reinterpret_cast<volatile int*>(S.tmem_slot + 1);
  return S;
}

// Bounded wait that also gives up as soon as another role of the CTA has aborted (about a
// second: 2^16 polls that may each suspend the thread for up to 20 us).
__device__ __forceinline__ bool rec_wait(const RecShared& S, const RecArgs& a, uint64_t* bar,
                                         uint32_t parity, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  for (uint32_t it = 0; it < (1u << 16); ++it) {
    if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
    if ((it & 15) == 15 && *S.abort_flag) return false;
  }
  *S.abort_flag = 1;
  atomicExch(a.err, code);
  return false;
}

// Byte offset of record u0 + i within the buffer (from the CTA's cache when it holds it).
__device__ __forceinline__ int64_t rec_offset(const RecShared& S, const RecArgs& a, int64_t u0, int64_t i) {
  if (i <= rec::kOffCache) return S.off[i];
  return __ldg(reinterpret_cast<const long long*>(a.rec) + u0 + i);
}

// ---------------------------------------------------------------------------------------
// producers
template <int NW>
__device__ void rec_wproducer(const RecShared& S, const RecArgs& a, int64_t u0, int64_t u1) {
  int s = 0;
  uint32_t ph = 0;
  int64_t i = 0;
  for (int64_t u = u0; u < u1; ++u, ++i) {
    if (!rec_wait(S, a, &S.empty_w[s], ph ^ 1, 1)) break;
    const int64_t o0 = rec_offset(S, a, u0, i), o1 = rec_offset(S, a, u0, i + 1);
    const int64_t len = o1 - o0;
    const uint32_t bytes = (uint32_t)(len < rec::kStageBytes ? len : rec::kStageBytes);
    mbar_arrive_expect_tx(&S.full_w[s], bytes);
    bulk_g2s(S.wring + (size_t)s * rec::kStageBytes, a.rec + o0, bytes, &S.full_w[s]);
    if (++s == NW) { s = 0; ph ^= 1; }
  }
  // wind down: every copy issued has landed and, unless the CTA aborted, has been released
  const int64_t j0 = i > NW ? i - NW : 0;
  for (int64_t j = j0; j < i; ++j)
    mbar_wait(&S.full_w[j % NW], (uint32_t)(j / NW) & 1, 1u << 20);
  for (int64_t j = j0; j < i; ++j)
    if (*S.abort_flag || !mbar_wait(&S.empty_w[j % NW], (uint32_t)(j / NW) & 1, 1u << 22)) break;
}

template <class C, int NX>
__device__ void rec_xproducer(const RecShared& S, const RecArgs& a, const RecMaps& M, int64_t u0, int64_t u1) {
  prefetch_tmap(&M.x);
  const uint32_t xbytes = 4u * 128u * (uint32_t)a.m;
  grid_dependency_wait();                 // the activations may be written by the previous kernel
  int s = 0;
  uint32_t ph = 0;
  int64_t i = 0;
  for (int64_t u = u0; u < u1; ++u, ++i) {
    if (!rec_wait(S, a, &S.empty_x[s], ph ^ 1, 11)) break;
    uint8_t* xb = S.xring + (size_t)s * C::kXBytes;
    const int st = (int)(u % a.n_stages);
    mbar_arrive_expect_tx(&S.full_x[s], xbytes);
#pragma unroll
    for (int b = 0; b < 4; ++b) tma_2d_g2s(xb + b * C::kXBox, &M.x, st * 256 + b * 64, 0, &S.full_x[s]);
    if (++s == NX) { s = 0; ph ^= 1; }
  }
  const int64_t j0 = i > NX ? i - NX : 0;
  for (int64_t j = j0; j < i; ++j)
    mbar_wait(&S.full_x[j % NX], (uint32_t)(j / NX) & 1, 1u << 20);
  for (int64_t j = j0; j < i; ++j)
    if (*S.abort_flag || !mbar_wait(&S.empty_x[j % NX], (uint32_t)(j / NX) & 1, 1u << 22)) break;
}

// ---------------------------------------------------------------------------------------
// MMA issuer (one thread). False if a wait gave up.
template <class C, int NX, int NS, int SB>
__device__ bool rec_mma_loop(const RecShared& S, const RecArgs& a, int64_t u0, int64_t u1, uint32_t tmem,
                             int64_t& uses) {
  constexpr uint32_t IDESC = idesc_bf16_f32(128, 16, false);
  const uint64_t desc0 = smem_desc_sw128(smem_u32(S.xring), 1024);
  constexpr uint64_t kXSlotDesc = (uint64_t)(C::kXBytes >> 4);
  constexpr uint64_t kBoxDesc = (uint64_t)(C::kXBox >> 4);
  int64_t seg = 0;
  int64_t i = 0;
  for (int64_t u = u0; u < u1; ++seg) {
    const int64_t rg = u / a.n_stages;
    const int64_t seg_end = min(u1, (rg + 1) * a.n_stages);
    const int d = (int)(seg & 1);
    if (!rec_wait(S, a, &S.dempty[d], (uint32_t)((seg >> 1) & 1) ^ 1, 2)) return false;
    tc_fence_after();
    // block j of a unit accumulates into chain j % kAcc: consecutive MMAs do not wait for each
    // other's accumulator (a chain of dependent small MMAs runs at their latency, not their rate)
    const uint32_t tD = tmem + d * (rec::kAcc * 16);
    uint32_t started = 0;                       // chains that hold a partial sum this segment
    for (; u < seg_end; ++u, ++i) {
      const int sx = (int)(i % NX);
      if (!rec_wait(S, a, &S.full_x[sx], (uint32_t)(i / NX) & 1, 3)) return false;
      const uint64_t dx = desc0 + (uint64_t)sx * kXSlotDesc;
      for (int c = 0; c < 4; ++c) {
        const int64_t g = 4 * i + c;             // substage g sits in slot (g / SB) % NS
        const int64_t gs = g / SB;
        const int slot = (int)(gs % NS);
        if (g % SB == 0) {
          if (!rec_wait(S, a, &S.afull[slot], (uint32_t)(gs / NS) & 1, 4)) return false;
          tc_fence_after();
        }
        const uint32_t tA = tmem + rec::kTmemA + slot * C::kSlotCols + (uint32_t)(g % SB) * 32;
        const uint64_t db = dx + (uint64_t)c * kBoxDesc;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const int ch = (4 * c + b) % rec::kAcc;
          mma_ts(tD + ch * 16, tA + 8 * b, db + 2 * b, IDESC, (started >> ch) & 1u);
          started |= 1u << ch;
        }
        if (g % SB == SB - 1) {
          mma_commit(&S.aempty[slot]);
          ++uses;
        }
      }
      mma_commit(&S.empty_x[sx]);
    }
    mma_commit(&S.dfull[d]);
  }
  return true;
}

template <class C, int NX, int NS, int SB>
__device__ void rec_mma(const RecShared& S, const RecArgs& a, int64_t u0, int64_t u1, uint32_t tmem) {
  int64_t uses = 0;
  const bool ok = rec_mma_loop<C, NX, NS, SB>(S, a, u0, u1, tmem, uses);
  if (uses > 0) {
    // every MMA issued completes before the tensor memory is released (also on abort)
    mma_commit(S.mtail);
    mbar_wait(S.mtail, 0, 1u << 22);
  }
  if (ok) {
    // the commit arrivals on the A-slot barriers land before the shared memory is released:
    // use t of slot t % NS completes that barrier's phase t / NS
    for (int j = 0; j < NS && j < uses; ++j) {
      const int64_t last = j + (uses - 1 - j) / NS * NS;
      if (!mbar_wait(&S.aempty[j], (uint32_t)(last / NS) & 1, 1u << 22)) break;
    }
  }
}

// ---------------------------------------------------------------------------------------
// dequantisers
__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
  __nv_bfloat162 r = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&a),
                             *reinterpret_cast<const __nv_bfloat162*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t rec_field(uint32_t w, int k) { return (w >> (5 * k)) & 0x001F001Fu; }

// Blocks 2h and 2h+1 of a substage from their five words and biased exponents: o0 / o1 are
// the 8 bf16 pairs of each block (pair j = elements 2j, 2j+1).
__device__ __forceinline__ void rec_dq_pair(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3, uint32_t w4,
                                            uint32_t eb0, uint32_t eb1, uint32_t (&o0)[8], uint32_t (&o1)[8]) {
  const uint32_t K0 = eb0 * 0x00800080u, C0 = K0 + 0x00100010u;
  const uint32_t K1 = eb1 * 0x00800080u, C1 = K1 + 0x00100010u;
  o0[0] = bf16x2_sub(rec_field(w0, 0) | K0, C0);
  o0[1] = bf16x2_sub(rec_field(w0, 1) | K0, C0);
  o0[2] = bf16x2_sub(rec_field(w0, 2) | K0, C0);
  o0[3] = bf16x2_sub(rec_field(w1, 0) | K0, C0);
  o0[4] = bf16x2_sub(rec_field(w1, 1) | K0, C0);
  o0[5] = bf16x2_sub(rec_field(w1, 2) | K0, C0);
  o0[6] = bf16x2_sub(rec_field(w2, 0) | K0, C0);
  o0[7] = bf16x2_sub(rec_field(w2, 1) | K0, C0);
  o1[0] = bf16x2_sub(rec_field(w2, 2) | K1, C1);
  o1[1] = bf16x2_sub(rec_field(w3, 0) | K1, C1);
  o1[2] = bf16x2_sub(rec_field(w3, 1) | K1, C1);
  o1[3] = bf16x2_sub(rec_field(w3, 2) | K1, C1);
  o1[4] = bf16x2_sub(rec_field(w4, 0) | K1, C1);
  o1[5] = bf16x2_sub(rec_field(w4, 1) | K1, C1);
  o1[6] = bf16x2_sub(rec_field(w4, 2) | K1, C1);
  const uint32_t t = ((w0 >> 15) & 0x00010001u) | ((w1 >> 14) & 0x00020002u) | ((w2 >> 13) & 0x00040004u) |
                     ((w3 >> 12) & 0x00080008u) | ((w4 >> 11) & 0x00100010u);
  o1[7] = bf16x2_sub(t | K1, C1);
}

// Each warp's substages are pipelined: the tensor-memory stores of a substage are waited for
// (tcgen05.wait::st) and handed to the MMA only after the next substage has been dequantised, so
// the stores' latency overlaps that work instead of stalling the warp once per substage.
template <class C, int NW, int NS, int DQ, int SB>
__device__ void rec_dequant(const RecShared& S, const RecArgs& a, int64_t u0, int64_t u1, uint32_t tmem) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q4 = warp & 3;                       // tensor-memory lane quarter
  const int p = (warp - rec::kDqWarp0) >> 2;     // substages c = p (mod DQ) of every unit
  const int lr = q4 * 32 + lane;                 // row within the group
  const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
  int pending = -1;                              // A slot whose stores are in flight
  // a wait that gave up in any lane ends the warp's work, after its stores in flight have landed
  auto give_up = [&]() {
    if (pending >= 0) tmem_wait_st();
  };
  int64_t i = 0;
  for (int64_t u = u0; u < u1; ++u, ++i) {
    const int s = (int)(i % NW);
    if (!__all_sync(0xffffffffu, rec_wait(S, a, &S.full_w[s], (uint32_t)(i / NW) & 1, 5))) return give_up();
    const uint8_t* rb = S.wring + (size_t)s * rec::kStageBytes;
#pragma unroll 1
    for (int cc = 0; cc < 4 / DQ; ++cc) {
      const int c = p + DQ * cc;
      const int64_t g = 4 * i + c;
      const int64_t gs = g / SB;
      const int slot = (int)(gs % NS);
      const uint8_t* sb = rb + c * 5120;
      const uint4 A = *reinterpret_cast<const uint4*>(sb + lr * 16);
      const uint4 B = *reinterpret_cast<const uint4*>(sb + 2048 + lr * 16);
      const uint2 Cw = *reinterpret_cast<const uint2*>(sb + 4096 + lr * 8);
      const uint32_t EB = *reinterpret_cast<const uint32_t*>(rb + rec::kExpOff + c * 512 + lr * 4);
      uint32_t o0[8], o1[8], o2[8], o3[8];
      rec_dq_pair(A.x, A.y, A.z, A.w, B.x, EB & 0xFFu, (EB >> 8) & 0xFFu, o0, o1);
      rec_dq_pair(B.y, B.z, B.w, Cw.x, Cw.y, (EB >> 16) & 0xFFu, EB >> 24, o2, o3);
      if (!__all_sync(0xffffffffu, rec_wait(S, a, &S.aempty[slot], ((uint32_t)(gs / NS) & 1) ^ 1, 6)))
        return give_up();
      if (pending >= 0) {                        // the previous substage's stores are done
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.afull[pending]);
      }
      __syncwarp();
      tc_fence_after();
      const uint32_t ta = tmem + rec::kTmemA + slot * C::kSlotCols + (uint32_t)(g % SB) * 32 + lane_base;
      tmem_st_32x32b_x8(ta + 0, o0);
      tmem_st_32x32b_x8(ta + 8, o1);
      tmem_st_32x32b_x8(ta + 16, o2);
      tmem_st_32x32b_x8(ta + 24, o3);
      pending = slot;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&S.empty_w[s]);   // this unit's fields are in registers or stored
  }
  if (pending >= 0) {
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&S.afull[pending]);
  }
}

// ---------------------------------------------------------------------------------------
// epilogue: outliers per unit, then per segment the accumulator, bias, output and exchange

// Outliers of row lr in one unit (their dense slots are 0): oacc[t] += v * x[t][col] for the
// row's entries, four per step with independent loads (a step costs one chain of dependent
// shared-memory loads for four entries; entries past the row's end read as value 0, column 0).
// The entries are in the staged record (those past the stage size in the record in global
// memory, `grec`); x sits in an activation slot as four boxes of 64 k x MT token rows with
// 128-byte swizzle: column c of token t is in box c / 64, 1024-byte atom t / 8, 128-byte row
// t % 8, 16-byte chunk ((c % 64) / 8) ^ (t % 8), element c % 8.
template <class C, int MT, int NT>
__device__ __forceinline__ void rec_row_outliers(const uint8_t* rb, const uint8_t* xb, const uint8_t* grec,
                                                 int lr, float (&oacc)[MT]) {
  const uint16_t* ro = reinterpret_cast<const uint16_t*>(rb + rec::kRoffOff);
  const uint32_t* es = reinterpret_cast<const uint32_t*>(rb + rec::kEntOff);
  const uint32_t* gs = reinterpret_cast<const uint32_t*>(grec + rec::kEntOff);
  const int k1 = ro[lr + 1];
  for (int k = ro[lr]; k < k1; k += 4) {
    uint32_t e[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int kk = k + j;
      e[j] = kk < k1 ? (kk < rec::kOutCap ? es[kk] : __ldg(gs + kk)) : 0u;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float v = __half2float(__ushort_as_half((unsigned short)(e[j] & 0xFFFFu)));
      const uint32_t col = (e[j] >> 16) & 0xFFu;
      const uint8_t* xp = xb + (col >> 6) * C::kXBox + (col & 7u) * 2;
      const uint32_t chunk = (col >> 3) & 7u;
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const uint32_t rr = (uint32_t)(t & 7);
        const uint32_t off = (uint32_t)(t >> 3) * 1024u + (rr << 7) + ((chunk ^ rr) << 4);
        oacc[t] = fmaf(v, __uint_as_float((uint32_t)*reinterpret_cast<const uint16_t*>(xp + off) << 16), oacc[t]);
      }
    }
  }
}

__device__ __forceinline__ uint64_t rec_global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Waits (bounded by a.xchg_timeout_ns, or until another role of the CTA aborts) for the word of
// this call's tag at `src`; returns its value in *v.
__device__ __forceinline__ bool rec_xchg_wait(const RecShared& S, const RecArgs& a, const uint2* src,
                                              uint32_t tag, int code, float* v) {
  uint2 w = xchg_load(src);
  uint64_t t0 = 0;
  for (uint32_t it = 1; w.y != tag; ++it) {
    if ((it & 63) == 0) {
      if (*S.abort_flag) return false;
      const uint64_t now = rec_global_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > a.xchg_timeout_ns) {
        *S.abort_flag = 1;
        atomicExch(a.err, code);
        return false;
      }
    }
    if (it > 128) __nanosleep(128);
    w = xchg_load(src);
  }
  *v = __uint_as_float(w.x);
  return true;
}

// Final values of output row `row` for the m tokens from v[t]. One rank: y = v + bias. With the
// row-parallel exchange: push v to every peer's slot [par][rank], then y = bias + the sum in rank
// order of every rank's v (the same bits on every rank). False if a wait gave up.
template <int MT>
__device__ __forceinline__ bool rec_finish_row(const RecShared& S, const RecArgs& a, int64_t row,
                                               const float (&v)[MT], uint32_t tag, uint32_t par) {
  const int m = a.m;
  const float bv = a.bias ? load_as_float(a.bias, a.bias_dtype, row) : 0.f;
  if (a.world > 1) {
    for (int p = 0; p < a.world; ++p) {
      if (p == a.rank) continue;
      uint2* dst = xchg_slot(a.xbuf[p], a.xmax, par, a.rank) + row;
#pragma unroll
      for (int t = 0; t < MT; ++t)
        if (t < m) xchg_store(dst + (int64_t)t * a.n_out, __float_as_uint(v[t]), tag);
    }
  }
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    if (t >= m) continue;
    float acc = v[t];
    if (a.world > 1) {
      acc = 0.f;
      for (int q = 0; q < a.world; ++q) {
        float w = v[t];
        if (q != a.rank &&
            !rec_xchg_wait(S, a, xchg_slot(a.xbuf[a.rank], a.xmax, par, q) + (int64_t)t * a.n_out + row,
                           tag, 32 + q, &w))
          return false;
        acc += w;
      }
    }
    store_from_float(a.y, a.y_dtype, (int64_t)t * a.ldy + row, acc + bv);
  }
  return true;
}

// Epilogue warpgroup. The fused exchange cannot deadlock: all CTAs of the grid are resident,
// every rank finishes every row group, and a CTA finishes its row groups in increasing order,
// so on every rank each contribution to the lowest row group any CTA waits on is either made or
// comes from a CTA that is not waiting.
template <class C, int MT, int NW, int NX>
__device__ void rec_epilogue(const RecShared& S, const RecArgs& a, int64_t u0, int64_t u1, uint32_t tmem) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q4 = warp & 3;
  const int lr = q4 * 32 + lane;
  const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
  const int m = a.m;
  const float inv15 = 1.0f / 15.0f;
  grid_dependency_wait();                 // the workspace and y may still be in use before this
  uint32_t tag = 0, par = 0;
  if (a.world > 1) {                      // this call's exchange epoch (advanced at kernel exit)
    const uint32_t e = *reinterpret_cast<volatile uint32_t*>(xchg_epoch(a.xbuf[a.rank]));
    par = e & 1u;
    tag = e + 1u;
  }
  int64_t seg = 0, i = 0;
  for (int64_t u = u0; u < u1; ++seg) {
    const int64_t rg = u / a.n_stages;
    const int64_t seg_begin = u, seg_end = min(u1, (rg + 1) * a.n_stages);
    const int64_t row = rg * 128 + lr;
    const bool rvalid = row < a.npad;
    float val[MT];
#pragma unroll
    for (int t = 0; t < MT; ++t) val[t] = 0.f;
    for (; u < seg_end; ++u, ++i) {
      const int s = (int)(i % NW), sx = (int)(i % NX);
      // both stages are waited for even without outliers: a release may only follow the landing
      // of the copy it releases, or the stages' phases would run ahead of their copies
      if (!__all_sync(0xffffffffu, rec_wait(S, a, &S.full_w[s], (uint32_t)(i / NW) & 1, 7))) return;
      if (!__all_sync(0xffffffffu, rec_wait(S, a, &S.full_x[sx], (uint32_t)(i / NX) & 1, 9))) return;
      if (a.outliers) {
        const uint8_t* rb = S.wring + (size_t)s * rec::kStageBytes;
        const uint8_t* xb = S.xring + (size_t)sx * C::kXBytes;
        const uint8_t* grec = a.rec + rec_offset(S, a, u0, i);
        if (m == 1) rec_row_outliers<C, MT, 1>(rb, xb, grec, lr, val);
        else if (m <= 4) rec_row_outliers<C, MT, 4>(rb, xb, grec, lr, val);
        else rec_row_outliers<C, MT, MT>(rb, xb, grec, lr, val);
      }
      __syncwarp();
      if (lane == 0) { mbar_arrive(&S.empty_w[s]); mbar_arrive(&S.empty_x[sx]); }
    }
    const int d = (int)(seg & 1);
    if (!__all_sync(0xffffffffu, rec_wait(S, a, &S.dfull[d], (uint32_t)(seg >> 1) & 1, 8))) return;
    __syncwarp();
    tc_fence_after();
    float acc[16];
    tmem_ld_32x32b_x16(tmem + d * (rec::kAcc * 16) + lane_base, acc);
#pragma unroll
    for (int ch = 1; ch < rec::kAcc; ++ch) {
      float part[16];
      tmem_ld_32x32b_x16(tmem + d * (rec::kAcc * 16) + ch * 16 + lane_base, part);
      tmem_wait_ld();
#pragma unroll
      for (int t = 0; t < MT; ++t) acc[t] += part[t];
    }
    tmem_wait_ld();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&S.dempty[d]);
#pragma unroll
    for (int t = 0; t < MT; ++t) val[t] = __fmaf_rn(acc[t], inv15, val[t]);
    const bool whole = seg_begin == rg * a.n_stages && seg_end == (rg + 1) * a.n_stages;
    if (whole) {
      bool ok = true;
      if (rvalid && row < a.n_out) ok = rec_finish_row<MT>(S, a, row, val, tag, par);
      if (!__all_sync(0xffffffffu, ok)) return;
      continue;
    }
    if (rvalid) {
#pragma unroll
      for (int t = 0; t < MT; ++t)
        if (t < m)
          asm volatile("red.global.add.f32 [%0], %1;\n" ::"l"(a.ws + (int64_t)t * a.npad + row),
                       "f"(val[t]) : "memory");
    }
    __threadfence();
    __syncwarp();
    const int units = (int)(seg_end - seg_begin);
    int old = 0;
    if (lane == 0) old = atomicAdd(a.counters + rg * 4 + q4, units);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old + units == a.n_stages) {
      __threadfence();
      bool ok = true;
      if (rvalid) {
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          if (t < m) {
            float* wp = a.ws + (int64_t)t * a.npad + row;
            val[t] = __ldcg(wp);
            __stcg(wp, 0.f);
          }
        }
        if (row < a.n_out) ok = rec_finish_row<MT>(S, a, row, val, tag, par);
      }
      __syncwarp();
      if (lane == 0) a.counters[rg * 4 + q4] = 0;
      if (!__all_sync(0xffffffffu, ok)) return;
    }
  }
}

// ---------------------------------------------------------------------------------------
template <int MT, int NW, int NX, int NS, int DQ, int SB, int MINB>
__global__ void __launch_bounds__(RecCfg<MT, NW, NX, NS, DQ, SB>::kThreads, MINB)
gemv_rec_kernel(const RecArgs a, const __grid_constant__ RecMaps M) {
  using C = RecCfg<MT, NW, NX, NS, DQ, SB>;
  extern __shared__ uint8_t smem_raw[];
  const RecShared S = rec_shared<C, NW, NX, NS>(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int64_t U = a.total_units;
  const int64_t u0 = (int64_t)blockIdx.x * U / gridDim.x;
  const int64_t u1 = (int64_t)(blockIdx.x + 1) * U / gridDim.x;
  // Programmatic launch: the previous kernel in the stream may still be running. Unless the
  // caller vouched that it did not write the weights, read no global memory before it completed.
  if (!a.early_weights) grid_dependency_wait();
  if (threadIdx.x == 0) {
    // a weight stage is released by the dequantisers and the 4 epilogue warps (outliers), an
    // activation stage by the MMA's commit and the 4 epilogue warps
    for (int s = 0; s < NW; ++s) { mbar_init(&S.full_w[s], 1); mbar_init(&S.empty_w[s], 4 * DQ + 4); }
    for (int s = 0; s < NX; ++s) { mbar_init(&S.full_x[s], 1); mbar_init(&S.empty_x[s], 5); }
    for (int j = 0; j < NS; ++j) { mbar_init(&S.afull[j], 4 * SB); mbar_init(&S.aempty[j], 1); }
    for (int d = 0; d < 2; ++d) { mbar_init(&S.dfull[d], 1); mbar_init(&S.dempty[d], 4); }
    mbar_init(S.mtail, 1);
    *S.abort_flag = 0;
    fence_mbar_init();
  }
  {
    const int64_t ncache = min((int64_t)rec::kOffCache, u1 - u0);
    const long long* tab = reinterpret_cast<const long long*>(a.rec);
    for (int64_t i = threadIdx.x; i <= ncache; i += blockDim.x) S.off[i] = __ldg(tab + u0 + i);
  }
  if (warp == 1) {
    tmem_alloc(S.tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *S.tmem_slot;
  // the next kernel in the stream may launch now
  if (threadIdx.x == 0) grid_launch_dependents();

  if (warp == 0) {
    if (elect_one_sync()) rec_wproducer<NW>(S, a, u0, u1);
    __syncwarp();
  } else if (warp == 1) {
    if (elect_one_sync()) rec_mma<C, NX, NS, SB>(S, a, u0, u1, tmem);
    __syncwarp();
  } else if (warp == 2) {
    if (elect_one_sync()) rec_xproducer<C, NX>(S, a, M, u0, u1);
    __syncwarp();
  } else if (warp >= rec::kEpiWarp0 && warp < rec::kDqWarp0) {
    rec_epilogue<C, MT, NW, NX>(S, a, u0, u1, tmem);
  } else if (warp >= rec::kDqWarp0) {
    rec_dequant<C, NW, NS, DQ, SB>(S, a, u0, u1, tmem);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
  // fused exchange: the last CTA to finish advances this rank's epoch (every CTA read it at the
  // start of its epilogue, before the barrier above)
  if (a.world > 1 && threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(a.exit_count, 1) == (int)gridDim.x - 1) {
      *a.exit_count = 0;
      volatile uint32_t* ep = xchg_epoch(a.xbuf[a.rank]);
      *ep = *ep + 1u;
    }
  }
}

// ---------------------------------------------------------------------------------------
// One token (m = 1) on the CUDA cores.
//
// A tcgen05.mma of M = 128 rows and K = 16 takes as long as one with N = 256, so with N = 16
// tokens the tensor cores bound the decode GEMV at 16 MMAs per 22.5 KB record (about 2.4 TB/s
// on B200). For one token the CUDA cores do better: each weight's field becomes an fp32 with one
// shift and one LOP3, v = (1 + f/32) * 2^e (field in mantissa bits 18-22, exponent e + 127), and
// enters a packed fp32x2 FMA with its activation; since s*m*2^e = 32 v - 48 * 2^e, a block
// contributes 32 * sum(v x) - 48 * 2^e * sum(x), the activations' block sum being shared by all
// rows. fp32 accumulation throughout.
//   warp 0      weight producer (as above);
//   warp 1      activation producer: per record, the stage's 256 bf16 activations as fp32 plus
//               their 16 block sums into an NX-deep ring (four records' loads in flight);
//   warps 2-17  consumers: warp w takes rows 32 (w % 4) .. + 31 (one per lane) and substage
//               w / 4 of every record, plus every fourth of the row's outliers; at the end of a
//               (row group, CTA) segment the four substage warps of a lane quarter add their
//               row sums through shared memory in a fixed order and the first one finishes the
//               rows as the tensor-core kernel's epilogue does (direct, workspace, exchange).
namespace cc {
constexpr int kConsumers = 16;
constexpr int kThreads = 32 * (2 + kConsumers);       // 576
constexpr int kNW = 6;
constexpr int kNX = 8;
constexpr int kXSlot = 1152;                          // 256 bf16 activations, 16 fp32 block sums at byte 512
constexpr size_t kXOff = (size_t)kNW * rec::kStageBytes;
constexpr size_t kRedOff = kXOff + (size_t)kNX * kXSlot;          // [2][4][128] fp32 row sums
constexpr size_t kOffOff = kRedOff + 2 * 4 * 128 * sizeof(float);
constexpr size_t kBarOff = kOffOff + (rec::kOffCache + 1) * sizeof(int64_t);
constexpr int kNumBars = 2 * kNW + 2 * kNX;
constexpr size_t kSmemBytes = kBarOff + kNumBars * 8 + 16 + 1024;
static_assert(kSmemBytes <= 232448, "shared memory budget");
}  // namespace cc

// Field pair K of word w (bits 5K and 16 + 5K) as a bf16 pair (Kb | f): each element is
// 2^e (128 + f), exactly (Kb = eb * 0x00800080 puts the biased exponent e + 134 in both halves).
template <int K>
__device__ __forceinline__ uint32_t cc_bpair(uint32_t w, uint32_t Kb) {
  return ((K == 0 ? w : (w >> (5 * K))) & 0x001F001Fu) | Kb;
}

// acc += b.lo * x.lo + b.hi * x.hi: bf16 operands, fp32 accumulation (mixed-precision FMA, one
// rounding each, the products exact).
__device__ __forceinline__ void fma_bf16x2(float& acc, uint32_t b, uint32_t x) {
  asm("{ .reg .b16 bl, bh, xl, xh;\n"
      "  mov.b32 {bl, bh}, %1;\n"
      "  mov.b32 {xl, xh}, %2;\n"
      "  fma.rn.f32.bf16 %0, bl, xl, %0;\n"
      "  fma.rn.f32.bf16 %0, bh, xh, %0;\n"
      "}" : "+f"(acc) : "r"(b), "r"(x));
}

// Blocks 2h, 2h+1 of a substage (five words, biased exponents eb0, eb1), x their 32 bf16
// activations (16 pair words in 4 uint4), sx0 / sx1 the blocks' activation sums. Adds
// sum(b x) = 2^e (144 sum(x) + sum(s m x)) over both blocks into acc0 / acc1 (even / odd pairs)
// and 144 2^e sum(x) into corr, so that acc0 + acc1 - corr = sum of 2^e s m x.
__device__ __forceinline__ void cc_block_pair(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3, uint32_t w4,
                                              uint32_t eb0, uint32_t eb1, const uint4* x4, float sx0, float sx1,
                                              float& acc0, float& acc1, float& corr) {
  const uint32_t K0 = eb0 * 0x00800080u, K1 = eb1 * 0x00800080u;
  const uint4 xa = x4[0], xb = x4[1], xc = x4[2], xd = x4[3];
  fma_bf16x2(acc0, cc_bpair<0>(w0, K0), xa.x);
  fma_bf16x2(acc1, cc_bpair<1>(w0, K0), xa.y);
  fma_bf16x2(acc0, cc_bpair<2>(w0, K0), xa.z);
  fma_bf16x2(acc1, cc_bpair<0>(w1, K0), xa.w);
  fma_bf16x2(acc0, cc_bpair<1>(w1, K0), xb.x);
  fma_bf16x2(acc1, cc_bpair<2>(w1, K0), xb.y);
  fma_bf16x2(acc0, cc_bpair<0>(w2, K0), xb.z);
  fma_bf16x2(acc1, cc_bpair<1>(w2, K0), xb.w);
  const uint32_t t = ((w0 >> 15) & 0x00010001u) | ((w1 >> 14) & 0x00020002u) | ((w2 >> 13) & 0x00040004u) |
                     ((w3 >> 12) & 0x00080008u) | ((w4 >> 11) & 0x00100010u);
  fma_bf16x2(acc0, cc_bpair<2>(w2, K1), xc.x);
  fma_bf16x2(acc1, cc_bpair<0>(w3, K1), xc.y);
  fma_bf16x2(acc0, cc_bpair<1>(w3, K1), xc.z);
  fma_bf16x2(acc1, cc_bpair<2>(w3, K1), xc.w);
  fma_bf16x2(acc0, cc_bpair<0>(w4, K1), xd.x);
  fma_bf16x2(acc1, cc_bpair<1>(w4, K1), xd.y);
  fma_bf16x2(acc0, cc_bpair<2>(w4, K1), xd.z);
  fma_bf16x2(acc1, cc_bpair<0>(t, K1), xd.w);
  // 144 * 2^e = 1.125 * 2^(e + 7): exponent field e + 134 = eb, mantissa 1/8
  corr = fmaf(__uint_as_float((eb0 << 23) | 0x00100000u), sx0, corr);
  corr = fmaf(__uint_as_float((eb1 << 23) | 0x00100000u), sx1, corr);
}

__device__ void cc_xproducer(const RecShared& S, const RecArgs& a, int64_t u0, int64_t u1) {
  const int lane = threadIdx.x & 31;
  grid_dependency_wait();                 // the activations may be written by the previous kernel
  const __nv_bfloat16* xg = static_cast<const __nv_bfloat16*>(a.x);
  const int64_t units = u1 - u0;
  for (int64_t i0 = 0; i0 < units; i0 += 4) {
    const int nb = (int)min((int64_t)4, units - i0);
    uint4 raw[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (j >= nb) break;
      const int64_t i = i0 + j;
      if (!__all_sync(0xffffffffu, rec_wait(S, a, &S.empty_x[i % cc::kNX], ((uint32_t)(i / cc::kNX) & 1) ^ 1, 11)))
        return;
      const int64_t col = (int64_t)((u0 + i) % a.n_stages) * 256 + lane * 8;
      raw[j] = col < a.k_in ? __ldg(reinterpret_cast<const uint4*>(xg + col)) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (j >= nb) break;
      const int64_t i = i0 + j;
      const int s = (int)(i % cc::kNX);
      uint8_t* xsl = S.xring + (size_t)s * cc::kXSlot;
      const uint32_t r[4] = {raw[j].x, raw[j].y, raw[j].z, raw[j].w};
      float f[8];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        f[2 * q] = __uint_as_float(r[q] << 16);
        f[2 * q + 1] = __uint_as_float(r[q] & 0xFFFF0000u);
      }
      *reinterpret_cast<uint4*>(xsl + lane * 16) = raw[j];           // 256 bf16 activations
      float s8 = ((f[0] + f[1]) + (f[2] + f[3])) + ((f[4] + f[5]) + (f[6] + f[7]));
      s8 += __shfl_xor_sync(0xffffffffu, s8, 1);
      if ((lane & 1) == 0) reinterpret_cast<float*>(xsl + 512)[lane / 2] = s8;   // 16 block sums
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.full_x[s]);
    }
  }
  // wind down: every ring slot filled so far has been released (no copies are asynchronous here)
}

__device__ __forceinline__ void cc_named_sync() {
  asm volatile("bar.sync 1, %0;\n" ::"n"(cc::kConsumers * 32) : "memory");
}

__device__ void cc_consumer(const RecShared& S, const RecArgs& a, int64_t u0, int64_t u1, float* red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int w = warp - 2;
  const int q4 = w & 3, c = w >> 2;           // lane quarter (rows) and substage
  const int lr = q4 * 32 + lane;
  const float inv15 = 1.0f / 15.0f;
  grid_dependency_wait();                     // the workspace and y may still be in use before this
  uint32_t tag = 0, par = 0;
  if (a.world > 1) {
    const uint32_t e = *reinterpret_cast<volatile uint32_t*>(xchg_epoch(a.xbuf[a.rank]));
    par = e & 1u;
    tag = e + 1u;
  }
  int64_t seg = 0, i = 0;
  int s = 0, sx = 0;                          // ring slots of unit i and their phases
  uint32_t ph = 0, phx = 0;
  bool alive = true;
  for (int64_t u = u0; u < u1; ++seg) {
    const int64_t rg = u / a.n_stages;
    const int64_t seg_begin = u, seg_end = min(u1, (rg + 1) * a.n_stages);
    const int64_t row = rg * 128 + lr;
    float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f, corr = 0.f, oacc = 0.f;
    for (; u < seg_end; ++u, ++i) {
      if (alive) {
        alive = __all_sync(0xffffffffu, rec_wait(S, a, &S.full_w[s], ph, 5)) &&
                __all_sync(0xffffffffu, rec_wait(S, a, &S.full_x[sx], phx, 9));
      }
      if (alive) {
        const uint8_t* rb = S.wring + (size_t)s * rec::kStageBytes;
        const uint8_t* xsl = S.xring + (size_t)sx * cc::kXSlot;
        const uint4* xs = reinterpret_cast<const uint4*>(xsl + 128 * c);     // 64 bf16 of the substage
        const uint16_t* xh = reinterpret_cast<const uint16_t*>(xsl);
        const float4 sx4 = *reinterpret_cast<const float4*>(xsl + 512 + 16 * c);
        const uint8_t* sb = rb + c * 5120;
        const uint4 A = *reinterpret_cast<const uint4*>(sb + lr * 16);
        const uint4 B = *reinterpret_cast<const uint4*>(sb + 2048 + lr * 16);
        const uint2 Cw = *reinterpret_cast<const uint2*>(sb + 4096 + lr * 8);
        const uint32_t EB = *reinterpret_cast<const uint32_t*>(rb + rec::kExpOff + c * 512 + lr * 4);
        cc_block_pair(A.x, A.y, A.z, A.w, B.x, EB & 0xFFu, (EB >> 8) & 0xFFu, xs, sx4.x, sx4.y, acc0, acc1, corr);
        cc_block_pair(B.y, B.z, B.w, Cw.x, Cw.y, (EB >> 16) & 0xFFu, EB >> 24, xs + 4, sx4.z, sx4.w, acc2, acc3,
                      corr);
        if (a.outliers) {                     // every fourth of the row's entries
          const uint16_t* ro = reinterpret_cast<const uint16_t*>(rb + rec::kRoffOff);
          const uint32_t* es = reinterpret_cast<const uint32_t*>(rb + rec::kEntOff);
          const int k1 = ro[lr + 1];
          for (int k = ro[lr] + c; k < k1; k += 8) {      // two of this warp's entries per step
            uint32_t e[2];
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const int kk = k + 4 * j;
              e[j] = 0u;
              if (kk < k1) {
                if (kk < rec::kOutCap) {
                  e[j] = es[kk];
                } else {                      // beyond the staged entries: from the record
                  const uint32_t* gs =
                      reinterpret_cast<const uint32_t*>(a.rec + rec_offset(S, a, u0, i) + rec::kEntOff);
                  e[j] = __ldg(gs + kk);
                }
              }
            }
#pragma unroll
            for (int j = 0; j < 2; ++j)
              oacc = fmaf(__half2float(__ushort_as_half((unsigned short)(e[j] & 0xFFFFu))),
                          __uint_as_float((uint32_t)xh[(e[j] >> 16) & 0xFFu] << 16), oacc);
          }
        }
      }
      __syncwarp();
      if (lane == 0 && alive) { mbar_arrive(&S.empty_w[s]); mbar_arrive(&S.empty_x[sx]); }
      if (++s == cc::kNW) { s = 0; ph ^= 1u; }
      if (++sx == cc::kNX) { sx = 0; phx ^= 1u; }
    }
    // the four substage warps of this lane quarter add their row sums in a fixed order (every
    // consumer warp reaches this barrier once per segment, also after a wait gave up)
    float* rbuf = red + (seg & 1) * (4 * 128);
    rbuf[c * 128 + lr] = fmaf(((acc0 + acc1) + (acc2 + acc3)) - corr, inv15, oacc);
    cc_named_sync();
    if (c != 0) continue;
    float val[1] = {((rbuf[lr] + rbuf[128 + lr]) + rbuf[256 + lr]) + rbuf[384 + lr]};
    if (!alive) continue;
    const bool rvalid = row < a.npad;
    const bool whole = seg_begin == rg * a.n_stages && seg_end == (rg + 1) * a.n_stages;
    if (whole) {
      bool ok = true;
      if (rvalid && row < a.n_out) ok = rec_finish_row<1>(S, a, row, val, tag, par);
      alive = __all_sync(0xffffffffu, ok);
      continue;
    }
    if (rvalid) asm volatile("red.global.add.f32 [%0], %1;\n" ::"l"(a.ws + row), "f"(val[0]) : "memory");
    __threadfence();
    __syncwarp();
    const int units = (int)(seg_end - seg_begin);
    int old = 0;
    if (lane == 0) old = atomicAdd(a.counters + rg * 4 + q4, units);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old + units == a.n_stages) {
      __threadfence();
      bool ok = true;
      if (rvalid) {
        float* wp = a.ws + row;
        val[0] = __ldcg(wp);
        __stcg(wp, 0.f);
        if (row < a.n_out) ok = rec_finish_row<1>(S, a, row, val, tag, par);
      }
      __syncwarp();
      if (lane == 0) a.counters[rg * 4 + q4] = 0;
      alive = __all_sync(0xffffffffu, ok);
    }
  }
}

__global__ void __launch_bounds__(cc::kThreads, 1) gemv_cc_kernel(const RecArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  RecShared S = {};
  S.wring = smem;
  S.xring = smem + cc::kXOff;
  S.off = reinterpret_cast<int64_t*>(smem + cc::kOffOff);
  uint64_t* b = reinterpret_cast<uint64_t*>(smem + cc::kBarOff);
  S.full_w = b;
  S.empty_w = b + cc::kNW;
  S.full_x = b + 2 * cc::kNW;
  S.empty_x = b + 2 * cc::kNW + cc::kNX;
  S.abort_flag = reinterpret_cast<volatile int*>(b + cc::kNumBars);
  float* red = reinterpret_cast<float*>(smem + cc::kRedOff);
  const int warp = threadIdx.x >> 5;
  const int64_t U = a.total_units;
  const int64_t u0 = (int64_t)blockIdx.x * U / gridDim.x;
  const int64_t u1 = (int64_t)(blockIdx.x + 1) * U / gridDim.x;
  if (!a.early_weights) grid_dependency_wait();
  if (threadIdx.x == 0) {
    // a weight or activation stage is released by the 16 consumer warps
    for (int s = 0; s < cc::kNW; ++s) { mbar_init(&S.full_w[s], 1); mbar_init(&S.empty_w[s], cc::kConsumers); }
    for (int s = 0; s < cc::kNX; ++s) { mbar_init(&S.full_x[s], 1); mbar_init(&S.empty_x[s], cc::kConsumers); }
    *S.abort_flag = 0;
    fence_mbar_init();
  }
  {
    const int64_t ncache = min((int64_t)rec::kOffCache, u1 - u0);
    const long long* tab = reinterpret_cast<const long long*>(a.rec);
    for (int64_t i = threadIdx.x; i <= ncache; i += blockDim.x) S.off[i] = __ldg(tab + u0 + i);
  }
  __syncthreads();
  if (threadIdx.x == 0) grid_launch_dependents();
  if (warp == 0) {
    if (elect_one_sync()) rec_wproducer<cc::kNW>(S, a, u0, u1);
    __syncwarp();
  } else if (warp == 1) {
    cc_xproducer(S, a, u0, u1);
  } else {
    cc_consumer(S, a, u0, u1, red);
  }
  __syncthreads();
  if (a.world > 1 && threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(a.exit_count, 1) == (int)gridDim.x - 1) {
      *a.exit_count = 0;
      volatile uint32_t* ep = xchg_epoch(a.xbuf[a.rank]);
      *ep = *ep + 1u;
    }
  }
}

// ---------------------------------------------------------------------------------------
// record build
// 1. per unit the number of 16-byte groups its outlier entries take
__global__ void records_count_kernel(const int32_t* __restrict__ seg_ptr, int64_t units, int32_t* groups) {
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < units; u += (int64_t)gridDim.x * blockDim.x)
    groups[u] = seg_ptr ? (seg_ptr[u + 1] - seg_ptr[u] + 3) / 4 : 0;
}
// 2. (after the exclusive scan of the groups) the offset table
__global__ void records_table_kernel(const int32_t* __restrict__ groups, int64_t units, int64_t* table) {
  const int64_t base = rec_table_bytes(units);
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u <= units; u += (int64_t)gridDim.x * blockDim.x)
    table[u] = base + u * (int64_t)rec::kEntOff + 16 * (int64_t)groups[u];
}
// 3. fields and exponents: one thread per (row, block pair)
__global__ void records_fields_kernel(const int8_t* __restrict__ ex, const uint16_t* __restrict__ sg,
                                      const uint32_t* __restrict__ pay, int64_t npad, int64_t kb_row,
                                      int n_stages, uint8_t* __restrict__ rec, int32_t* bad) {
  const int64_t npairs = kb_row / 2;
  const int64_t total = npad * npairs;
  const int64_t* table = reinterpret_cast<const int64_t*>(rec);
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = t / npairs, bp = t % npairs;
    uint32_t w[5] = {0u, 0u, 0u, 0u, 0u};
    uint32_t eb[2];
    for (int b = 0; b < 2; ++b) {
      const int64_t blk = n * kb_row + 2 * bp + b;
      const int e = ex[blk];
      if (e > 120 && bad) atomicAdd(bad, 1);
      eb[b] = (uint32_t)(e + 134) & 0xFFu;
      const uint32_t s16 = sg[blk];
      const uint32_t p0 = pay[2 * blk], p1 = pay[2 * blk + 1];
      for (int el = 0; el < 16; ++el) {
        const uint32_t mnt = ((el < 8 ? p0 : p1) >> (4 * (el & 7))) & 0xFu;
        const uint32_t f = ((s16 >> el) & 1u) ? 16u - mnt : 16u + mnt;
        const int P = 8 * b + (el >> 1);
        const int hi = (el & 1) * 16;
        if (P < 15) {
          w[P / 3] |= f << (5 * (P % 3) + hi);
        } else {
#pragma unroll
          for (int k = 0; k < 5; ++k) w[k] |= ((f >> k) & 1u) << (15 + hi);
        }
      }
    }
    const int64_t g = n >> 7;
    const int row = (int)(n & 127);
    const int64_t st = bp >> 3;
    const int pp = (int)(bp & 7), c = pp >> 1, h = pp & 1;
    uint8_t* rb = rec + table[g * n_stages + st];
    uint8_t* sb = rb + c * 5120;
    for (int j = 0; j < 5; ++j) {
      const int wi = 5 * h + j;
      const int chunk = wi >> 2, within = wi & 3;
      uint8_t* dst = sb + chunk * 2048 + row * (chunk < 2 ? 16 : 8) + within * 4;
      *reinterpret_cast<uint32_t*>(dst) = w[j];
    }
    rb[rec::kExpOff + c * 512 + row * 4 + 2 * h] = (uint8_t)eb[0];
    rb[rec::kExpOff + c * 512 + row * 4 + 2 * h + 1] = (uint8_t)eb[1];
  }
}
// 4. outliers: per unit its 136 row starts and its entries (from the tile layout of outliers.cu)
__global__ void records_outliers_kernel(const uint32_t* __restrict__ entries, const int32_t* __restrict__ seg_ptr,
                                        int64_t units, uint8_t* __restrict__ rec) {
  const int64_t* table = reinterpret_cast<const int64_t*>(rec);
  const int64_t roff_base = (units + 1 + 3) & ~(int64_t)3;   // words of segment pointers
  for (int64_t u = blockIdx.x; u < units; u += gridDim.x) {
    uint8_t* rb = rec + table[u];
    const uint16_t* ro = reinterpret_cast<const uint16_t*>(seg_ptr + roff_base + u * 68);
    uint16_t* dro = reinterpret_cast<uint16_t*>(rb + rec::kRoffOff);
    for (int r = threadIdx.x; r < 136; r += blockDim.x) dro[r] = ro[r];
    const int32_t lo = seg_ptr[u], hi = seg_ptr[u + 1];
    uint32_t* de = reinterpret_cast<uint32_t*>(rb + rec::kEntOff);
    for (int32_t k = lo + threadIdx.x; k < hi; k += blockDim.x) de[k - lo] = entries[k];
  }
}

// ---------------------------------------------------------------------------------------
// host
static int encode_x_boxes(CUtensorMap* m, const void* x, int64_t tokens, int64_t k_in, int64_t ldx) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(FBFP_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  const cuuint64_t dims[2] = {(cuuint64_t)k_in, (cuuint64_t)tokens};
  const cuuint64_t strides[1] = {(cuuint64_t)ldx * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)tokens};
  const cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(FBFP_ERR_CUDA, "cuTensorMapEncodeTiled(x) failed (%d)", (int)r);
  return FBFP_OK;
}

template <int MT, int NW, int NX, int NS, int DQ, int SB, int MINB>
static int launch_rec(const RecArgs& a, const RecMaps& M, cudaStream_t st, int dev) {
  using C = RecCfg<MT, NW, NX, NS, DQ, SB>;
  static_assert(C::kSmemBytes <= (MINB == 2 ? 113u * 1024u : 232448u), "shared memory budget");
  static_assert(MINB == 1 || C::kTmemCols <= 256, "two CTAs per SM share the 512 tensor-memory columns");
  static bool attr_set[64] = {false};
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    FBFP_CUDA_TRY(cudaFuncSetAttribute(gemv_rec_kernel<MT, NW, NX, NS, DQ, SB, MINB>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::kSmemBytes));
    attr_set[dev] = true;
  }
  const int64_t nsm = sm_count(dev);
  const int64_t grid = nsm < a.total_units ? nsm : a.total_units;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FBFP_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemv_rec_kernel<MT, NW, NX, NS, DQ, SB, MINB>, a, M));
  FBFP_LAUNCH_CHECK("gemv_rec_kernel");
  return FBFP_OK;
}

static int launch_cc(const RecArgs& a, cudaStream_t st, int dev) {
  static bool attr_set[64] = {false};
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    FBFP_CUDA_TRY(cudaFuncSetAttribute(gemv_cc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)cc::kSmemBytes));
    attr_set[dev] = true;
  }
  const int64_t nsm = sm_count(dev);
  int64_t grid = nsm < a.total_units ? nsm : a.total_units;
  // at least four records per CTA while that keeps three quarters of the SMs: on small matrices
  // fewer, longer runs split fewer row groups across CTAs (3840x4096, 480 records: 120 CTAs at
  // 8.35 us against 148 at 9.24; six records per CTA, 80 CTAs: 11.2 us; 240 records on 60 CTAs
  // with the fused exchange: slower than on 148)
  const int64_t cap = (a.total_units + 3) / 4;
  if (grid > cap && cap * 4 >= nsm * 3) grid = cap;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(cc::kThreads);
  cfg.dynamicSmemBytes = cc::kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FBFP_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemv_cc_kernel, a));
  FBFP_LAUNCH_CHECK("gemv_cc_kernel");
  return FBFP_OK;
}

int allreduce_buffers(void* handle, uint8_t** bufs, int* world, int* rank, int64_t* max_elems);
uint64_t allreduce_timeout_ns(void* handle);
int gemv_workspace_parts(void* workspace, int64_t npad, int32_t** err, int32_t** counters, float** ws);

static int64_t rec_units(int64_t npad, int64_t kpad) {
  return ((npad + kGroupRows - 1) / kGroupRows) * (kpad / (kStageKb * kBlock));
}

}  // namespace fbfp

using namespace fbfp;

extern "C" int64_t fbfp_records_bytes(int64_t npad, int64_t kpad, int64_t outliers) {
  if (npad <= 0 || kpad <= 0 || kpad % (kStageKb * kBlock) != 0 || outliers < 0) return -1;
  const int64_t units = rec_units(npad, kpad);
  return rec_table_bytes(units) + units * (int64_t)(rec::kEntOff + 16) + 4 * outliers;
}

extern "C" int64_t fbfp_records_scratch_bytes(int64_t npad, int64_t kpad) {
  if (npad <= 0 || kpad <= 0 || kpad % (kStageKb * kBlock) != 0) return -1;
  return (rec_units(npad, kpad) + 1) * (int64_t)sizeof(int32_t);
}

extern "C" int fbfp_records_build(const int8_t* exponents, const int16_t* signs, const int32_t* payload,
                                  int64_t npad, int64_t kpad, const uint32_t* entries, const int32_t* seg_ptr,
                                  int64_t outliers, void* records, int32_t* bad_exponents, void* scratch,
                                  void* stream) {
  FBFP_CHECK_ARG(exponents && signs && payload && records && scratch, "null pointer");
  FBFP_CHECK_ARG(npad > 0 && kpad > 0 && kpad % (kStageKb * kBlock) == 0,
                 "stage records need kpad a multiple of 256 (got %lld)", (long long)kpad);
  FBFP_CHECK_ARG(outliers >= 0 && (outliers == 0 || (entries && seg_ptr)), "outliers without their layout");
  FBFP_CHECK_ARG(((uintptr_t)records & 255) == 0, "records must be 256-byte aligned");
  FBFP_CHECK_ARG(((uintptr_t)payload & 7) == 0, "payload must be 8-byte aligned");
  cudaStream_t st = as_stream(stream);
  const int64_t units = rec_units(npad, kpad);
  const int64_t bytes = fbfp_records_bytes(npad, kpad, outliers);
  int32_t* groups = static_cast<int32_t*>(scratch);
  uint8_t* rec = static_cast<uint8_t*>(records);
  FBFP_CUDA_TRY(cudaMemsetAsync(records, 0, (size_t)bytes, st));
  auto grid = [](int64_t work) {
    int64_t b = (work + 255) / 256;
    return (unsigned)(b < 1 ? 1 : (b > 148 * 64 ? 148 * 64 : b));
  };
  records_count_kernel<<<grid(units), 256, 0, st>>>(outliers ? seg_ptr : nullptr, units, groups);
  FBFP_LAUNCH_CHECK("records_count_kernel");
  scan_rows_kernel<<<1, 1024, 0, st>>>(groups, units);
  FBFP_LAUNCH_CHECK("scan_rows_kernel");
  records_table_kernel<<<grid(units + 1), 256, 0, st>>>(groups, units, reinterpret_cast<int64_t*>(rec));
  FBFP_LAUNCH_CHECK("records_table_kernel");
  const int64_t kb_row = kpad / kBlock;
  records_fields_kernel<<<grid(npad * (kb_row / 2)), 256, 0, st>>>(
      exponents, reinterpret_cast<const uint16_t*>(signs), reinterpret_cast<const uint32_t*>(payload),
      npad, kb_row, (int)(kpad / (kStageKb * kBlock)), rec, bad_exponents);
  FBFP_LAUNCH_CHECK("records_fields_kernel");
  if (outliers) {
    const unsigned nb = (unsigned)(units < 148 * 64 ? units : 148 * 64);
    records_outliers_kernel<<<nb, 128, 0, st>>>(entries, seg_ptr, units, rec);
    FBFP_LAUNCH_CHECK("records_outliers_kernel");
  }
  return FBFP_OK;
}

extern "C" int fbfp_gemv_records(const void* x, int64_t m, int64_t ldx, const void* records,
                                 int64_t n_out, int64_t k_in, int64_t kpad, int64_t npad,
                                 const void* bias, int bias_dtype, void* y, int y_dtype, int64_t ldy,
                                 void* workspace, void* allreduce, int flags, void* stream) {
  FBFP_CHECK_ARG(x && records && y && workspace, "null pointer");
  FBFP_CHECK_ARG(m >= 1 && m <= 16, "fbfp_gemv_records needs 1 <= m <= 16 (got %lld)", (long long)m);
  FBFP_CHECK_ARG(dtype_ok(y_dtype), "y_dtype must be f32, bf16 or f16");
  FBFP_CHECK_ARG(!bias || dtype_ok(bias_dtype), "bad bias dtype");
  FBFP_CHECK_ARG(n_out > 0 && k_in > 0 && kpad >= k_in && kpad % (kStageKb * kBlock) == 0 && npad >= n_out,
                 "bad shape (kpad must be a multiple of 256)");
  FBFP_CHECK_ARG(ldx >= k_in && ldy >= n_out && ldx % 8 == 0 && k_in % 8 == 0,
                 "bad leading dimension (ldx and k_in must be multiples of 8)");
  FBFP_CHECK_ARG(((uintptr_t)x & 15) == 0 && ((uintptr_t)records & 255) == 0,
                 "x must be 16-byte and records 256-byte aligned");
  FBFP_CHECK_ARG(((uintptr_t)workspace & 255) == 0, "workspace must be 256-byte aligned");
  RecArgs a;
  a.x = x; a.m = (int)m; a.ldx = ldx; a.rec = static_cast<const uint8_t*>(records);
  a.n_out = n_out; a.k_in = k_in; a.npad = npad;
  a.n_stages = (int)(kpad / (kStageKb * kBlock));
  a.total_units = rec_units(npad, kpad);
  a.outliers = (flags & FBFP_GEMV_DENSE_ONLY) ? 0 : 1;
  a.bias = bias; a.bias_dtype = bias_dtype;
  a.y = y; a.y_dtype = y_dtype; a.ldy = ldy;
  int rc = gemv_workspace_parts(workspace, npad, &a.err, &a.counters, &a.ws);
  if (rc != FBFP_OK) return rc;
  a.exit_count = a.err + 1;
  a.early_weights = (flags & FBFP_GEMV_RESIDENT) ? 1 : 0;
  a.world = 1; a.rank = 0; a.xmax = 0; a.xchg_timeout_ns = 0;
  for (int p = 0; p < 8; ++p) a.xbuf[p] = nullptr;
  if (allreduce) {
    rc = allreduce_buffers(allreduce, a.xbuf, &a.world, &a.rank, &a.xmax);
    if (rc != FBFP_OK) return rc;
    FBFP_CHECK_ARG(m * n_out <= a.xmax, "m * n_out = %lld exceeds the all-reduce handle's %lld elements",
                   (long long)(m * n_out), (long long)a.xmax);
    a.xchg_timeout_ns = allreduce_timeout_ns(allreduce);
  }
  int dev = 0;
  FBFP_CUDA_TRY(cudaGetDevice(&dev));
  cudaStream_t st = as_stream(stream);
  if (m == 1 && !(flags & FBFP_GEMV_TENSOR_CORES)) return launch_cc(a, st, dev);
  RecMaps M;
  if ((rc = encode_x_boxes(&M.x, x, m, k_in, ldx)) != FBFP_OK) return rc;
  if (m <= 8) return launch_rec<8, 6, 12, 7, 2, 2, 1>(a, M, st, dev);
  return launch_rec<16, 5, 9, 7, 2, 2, 1>(a, M, st, dev);
}
