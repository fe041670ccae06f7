// gemm_tc.cu — OABF prefill GEMM on tcgen05 (sm_100a): Y[M, N] = X[M, K] W_full[N, K]^T + bias
// for many tokens (replaces oabf_gemm_kernel, flash_bfp/triton_kernel.py:22-86, and the outlier
// SpMV/bias of OABFLinear.forward, :339-362, at prefill sizes). Tensor-core bound: each tile is
// 128 output rows x 256 tokens with an fp32 accumulator of 256 tensor-memory columns.
//
// Roles inside one persistent CTA per SM (tiles assigned round-robin, the tokens tiles of a row
// group on neighbouring CTAs so that its weights are read from HBM about once):
//   warp 0      producer: per 16-block stage a tensor copy of payload (128-byte swizzle), signs,
//               exponents, the stage's outlier entries and per-row starts into a 3-deep ring, and
//               per 64-k chunk a 64 x 256-token box of activations (128-byte swizzle, K-major B
//               operand; tokens past M read as zero, and with M < 256 the rows past M are stale
//               and only reach accumulator columns that are never stored) into a 4-deep ring;
//   warp 1      MMA issuer: per chunk 4 x tcgen05.mma (M=128, N=256, K=16), A from tensor memory;
//   warps 4-7   epilogue: drain the accumulator, scale by 1/15, add bias, convert and store;
//   warps 8-23  dequantisers (4 per tensor-memory lane quarter, one 4-block substage each, one
//               row per lane): bf16 pairs s*m*2^e exactly (dq_pair.cuh); the stage's outliers of
//               the row are written into their (otherwise +0) slots as bf16(15 v), so the tensor
//               core adds v * x (v to bf16 precision, as the reference's bf16 index_add); then
//               tcgen05.st into an 8-slot A ring.
// Every mbarrier wait is bounded; on timeout the CTA records an error code in the workspace word
// (read by fbfp_gemv_check) and winds down.
#include <cuda.h>
#include <cuda_bf16.h>

#include "common.cuh"
#include "dq_pair.cuh"
#include "sm100.cuh"
#include "tc_host.h"

namespace fbfp {
using namespace sm100;

namespace pf {
constexpr int kWStages = 3;
constexpr int kPayOff = 0;                      // 128 rows x 128 B (128-byte swizzle)
constexpr int kSgnOff = 128 * 128;              // 128 rows x 32 B
constexpr int kExpOff = kSgnOff + 128 * 32;     // 128 rows x 16 B
constexpr int kOutOff = kExpOff + 128 * 16;     // stage's outlier entries (window)
constexpr int kOutCap = 1024;
constexpr int kRoffOff = kOutOff + kOutCap * 4; // 136 uint16 row starts
constexpr int kRoffBytes = 272;
constexpr int kRangeOff = kRoffOff + 512;       // the stage's PfRange, written by the producer
constexpr int kWStageBytes = kRoffOff + 1024;   // 27 KB
constexpr uint32_t kWeightTx = kOutOff;
constexpr int kBN = 256;                        // tokens per tile
constexpr int kXSlots = 4;
constexpr int kXSlotBytes = kBN * 128;          // 64 k x 256 tokens, 128-byte rows
constexpr int kASlots = 8;
constexpr int kDq = 16, kEpiWarp0 = 4, kDqWarp0 = 8;
constexpr int kThreads = 32 * (kDqWarp0 + kDq);
constexpr uint32_t kTmemCols = 512, kTmemD = 0, kTmemA = 256;
constexpr size_t kXOff = (size_t)kWStages * kWStageBytes;
constexpr size_t kBarOff = kXOff + (size_t)kXSlots * kXSlotBytes;
constexpr int kNumBars = 2 * kWStages + 2 * kXSlots + 2 * kASlots + 3;
constexpr size_t kSmemBytes = kBarOff + kNumBars * 8 + 16 + 1024;
static_assert(kWStageBytes % 1024 == 0 && kXOff % 1024 == 0, "swizzled buffers need 1 KB alignment");
static_assert(kTmemA + kASlots * 32 <= kTmemCols, "tensor memory budget");
}  // namespace pf

struct PfArgs {
  int m;
  int64_t ldx;
  int64_t n_out, k_in, npad;
  const uint32_t* entries;
  const int32_t* seg_ptr;
  const void* bias;
  int bias_dtype;
  void* y;
  int y_dtype;
  int64_t ldy;
  int32_t* err;
  int x_rows;            // activation box height: min(256, m)
  int n_stages;          // Kpad / 256
  int n_tt;              // token tiles
  int64_t n_tiles;       // row groups x token tiles
  int64_t n_seg;         // row groups x stages (outlier index segments)
};

struct PfMaps {
  CUtensorMap pay, sgn, exp, x;
};

struct PfShared {
  uint8_t* wst;          // weight stages
  uint8_t* xst;          // activation chunks
  uint64_t *wfull, *wempty, *xfull, *xempty, *afull, *aempty, *dfull, *dempty;
  uint64_t* mtail;       // the MMA thread's last commit (its MMAs have completed)
  uint32_t* tmem_slot;
  volatile int* abort_flag;
};

__device__ __forceinline__ PfShared pf_shared(uint8_t* smem_raw) {
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  PfShared S;
  S.wst = smem;
  S.xst = smem + pf::kXOff;
  uint64_t* b = reinterpret_cast<uint64_t*>(smem + pf::kBarOff);
  S.wfull = b;
  S.wempty = S.wfull + pf::kWStages;
  S.xfull = S.wempty + pf::kWStages;
  S.xempty = S.xfull + pf::kXSlots;
  S.afull = S.xempty + pf::kXSlots;
  S.aempty = S.afull + pf::kASlots;
  S.dfull = S.aempty + pf::kASlots;
  S.dempty = S.dfull + 1;
  S.mtail = S.dempty + 1;
  S.tmem_slot = reinterpret_cast<uint32_t*>(S.mtail + 1);
  S.abort_flag = reinterpret_cast<volatile int*>(S.tmem_slot + 1);
  return S;
}

// Bounded wait (about a second), giving up early once another role has aborted.
__device__ __forceinline__ bool pf_wait(const PfShared& S, const PfArgs& a, uint64_t* bar,
                                        uint32_t parity, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  for (uint32_t it = 0; it < (1u << 16); ++it) {
    if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
    if ((it & 15) == 15 && *S.abort_flag) return false;
  }
  *S.abort_flag = 1;
  atomicExch(a.err, 100 + code);
  return false;
}

// Outlier entries of segment seg (row group x stage): [lo, hi) and the 16-byte aligned window
// [lo4, lo4 + n) staged in shared memory (capped; the rest is read from global memory).
struct PfRange { int lo, lo4, n; };
__device__ __forceinline__ PfRange pf_range(const PfArgs& a, int64_t seg) {
  PfRange r{0, 0, 0};
  if (!a.entries) return r;
  r.lo = __ldg(a.seg_ptr + seg);
  const int hi = __ldg(a.seg_ptr + seg + 1);
  if (hi > r.lo) {
    r.lo4 = r.lo & ~3;
    r.n = ((hi + 3) & ~3) - r.lo4;
    if (r.n > pf::kOutCap) r.n = pf::kOutCap;
  }
  return r;
}
__device__ __forceinline__ const uint8_t* pf_roff(const PfArgs& a, int64_t seg) {
  const int64_t base = (a.n_seg + 1 + 3) & ~(int64_t)3;
  return reinterpret_cast<const uint8_t*>(a.seg_ptr + base + seg * 68);
}

// ---------------------------------------------------------------------------------------
__device__ void pf_producer_thread(const PfShared& S, const PfArgs& a, const PfMaps& M) {
  prefetch_tmap(&M.pay); prefetch_tmap(&M.sgn); prefetch_tmap(&M.exp); prefetch_tmap(&M.x);
  int ws = 0, xs = 0;
  uint32_t wph = 0, xph = 0;
  int64_t issued_w = 0, issued_x = 0;
  bool ok = true;
  for (int64_t t = blockIdx.x; t < a.n_tiles && ok; t += gridDim.x) {
    const int rg = (int)(t / a.n_tt), tt = (int)(t % a.n_tt);
    for (int st = 0; st < a.n_stages && ok; ++st) {
      const int64_t seg = (int64_t)rg * a.n_stages + st;
      const PfRange orr = pf_range(a, seg);          // its loads overlap the wait below
      if (!(ok = pf_wait(S, a, &S.wempty[ws], wph ^ 1, 1))) break;
      uint8_t* sb = S.wst + (size_t)ws * pf::kWStageBytes;
      // the dequantisers read the range here, after the stage's full barrier
      *reinterpret_cast<int4*>(sb + pf::kRangeOff) = make_int4(orr.lo, orr.lo4, orr.n, 0);
      mbar_arrive_expect_tx(&S.wfull[ws], pf::kWeightTx + (uint32_t)orr.n * 4 +
                                              (a.entries ? pf::kRoffBytes : 0));
      tma_2d_g2s(sb + pf::kPayOff, &M.pay, st * 128, rg * 128, &S.wfull[ws]);
      tma_2d_g2s(sb + pf::kSgnOff, &M.sgn, st * kStageKb, rg * 128, &S.wfull[ws]);
      tma_2d_g2s(sb + pf::kExpOff, &M.exp, st * kStageKb, rg * 128, &S.wfull[ws]);
      if (orr.n) bulk_g2s(sb + pf::kOutOff, a.entries + orr.lo4, (uint32_t)orr.n * 4, &S.wfull[ws]);
      if (a.entries) bulk_g2s(sb + pf::kRoffOff, pf_roff(a, seg), pf::kRoffBytes, &S.wfull[ws]);
      ++issued_w;
      if (++ws == pf::kWStages) { ws = 0; wph ^= 1; }
      for (int c = 0; c < 4; ++c) {
        if (!(ok = pf_wait(S, a, &S.xempty[xs], xph ^ 1, 2))) break;
        mbar_arrive_expect_tx(&S.xfull[xs], 128u * (uint32_t)a.x_rows);
        tma_2d_g2s(S.xst + (size_t)xs * pf::kXSlotBytes, &M.x, st * 256 + c * 64, tt * pf::kBN,
                   &S.xfull[xs]);
        ++issued_x;
        if (++xs == pf::kXSlots) { xs = 0; xph ^= 1; }
      }
    }
  }
  // wind down: copies in flight must land before the CTA exits, and, unless the CTA aborted,
  // the MMA's commit arrivals that release the activation chunks must have landed before the
  // shared memory is freed
  for (int64_t j = issued_w > pf::kWStages ? issued_w - pf::kWStages : 0; j < issued_w; ++j)
    mbar_wait(&S.wfull[j % pf::kWStages], (uint32_t)(j / pf::kWStages) & 1, 1u << 20);
  const int64_t x0 = issued_x > pf::kXSlots ? issued_x - pf::kXSlots : 0;
  for (int64_t j = x0; j < issued_x; ++j)
    mbar_wait(&S.xfull[j % pf::kXSlots], (uint32_t)(j / pf::kXSlots) & 1, 1u << 20);
  for (int64_t j = x0; j < issued_x && ok; ++j)
    ok = pf_wait(S, a, &S.xempty[j % pf::kXSlots], (uint32_t)(j / pf::kXSlots) & 1, 9);
}

// ---------------------------------------------------------------------------------------
// Issues the CTA's MMAs; `uses` counts the A-slot uses committed. False if a wait gave up.
__device__ bool pf_mma_loop(const PfShared& S, const PfArgs& a, uint32_t tmem, int64_t& uses) {
  constexpr uint32_t IDESC = idesc_bf16_f32(128, pf::kBN, false);
  // B: a chunk is 256 token rows of 64 k (128-byte swizzled K-major), token groups of 8 are
  // 1024 B apart; block j of the chunk starts 32 * j bytes in
  const uint64_t desc0 = smem_desc_sw128(smem_u32(S.xst), 1024);
  constexpr uint64_t kSlotDesc = (uint64_t)(pf::kXSlotBytes >> 4);
  int xs = 0, slot = 0;
  uint32_t xph = 0, aph = 0, dph = 0;
  const uint32_t tD = tmem + pf::kTmemD;
  for (int64_t t = blockIdx.x; t < a.n_tiles; t += gridDim.x) {
    if (!pf_wait(S, a, S.dempty, dph ^ 1, 3)) return false;
    tc_fence_after();
    uint32_t acc = 0;
    for (int st = 0; st < a.n_stages; ++st) {
      for (int c = 0; c < 4; ++c) {
        if (!pf_wait(S, a, &S.xfull[xs], xph, 4)) return false;
        if (!pf_wait(S, a, &S.afull[slot], aph, 5)) return false;
        tc_fence_after();
        const uint32_t tA = tmem + pf::kTmemA + slot * 32;
        const uint64_t db = desc0 + (uint64_t)xs * kSlotDesc;
        mma_ts(tD, tA + 0, db + 0, IDESC, acc);
        mma_ts(tD, tA + 8, db + 2, IDESC, 1);
        mma_ts(tD, tA + 16, db + 4, IDESC, 1);
        mma_ts(tD, tA + 24, db + 6, IDESC, 1);
        acc = 1;
        mma_commit(&S.aempty[slot]);
        mma_commit(&S.xempty[xs]);
        ++uses;
        if (++slot == pf::kASlots) { slot = 0; aph ^= 1; }
        if (++xs == pf::kXSlots) { xs = 0; xph ^= 1; }
      }
    }
    mma_commit(S.dfull);
    dph ^= 1;
  }
  return true;
}

__device__ void pf_mma(const PfShared& S, const PfArgs& a, uint32_t tmem) {
  int64_t uses = 0;
  const bool ok = pf_mma_loop(S, a, tmem, uses);
  if (uses > 0) {
    // every MMA this thread issued completes before the tensor memory is released (also when
    // the CTA aborts with MMAs in flight)
    mma_commit(S.mtail);
    mbar_wait(S.mtail, 0, 1u << 22);
  }
  if (ok) {
    // the commit arrivals on the A-slot barriers land before the shared memory is released:
    // use t of slot t % kASlots completes that barrier's phase t / kASlots
    for (int j = 0; j < pf::kASlots && j < uses; ++j) {
      const int64_t last = j + (uses - 1 - j) / pf::kASlots * pf::kASlots;
      if (!pf_wait(S, a, &S.aempty[j], (uint32_t)(last / pf::kASlots) & 1, 10)) break;
    }
  }
}

// ---------------------------------------------------------------------------------------
__device__ void pf_dequant(const PfShared& S, const PfArgs& a, uint32_t tmem) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wi = warp - pf::kDqWarp0;
  const int q4 = warp & 3;                 // tensor-memory lane quarter
  const int par = wi >> 2;                 // substage (blocks 4 par .. 4 par + 3) of each stage
  const int lr = q4 * 32 + lane;
  const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
  const int sw = lr & 7;
  int ws = 0, ai = 0;                      // this warp's A slot is 4 * ai + par
  uint32_t wph = 0, aph = 0;
  for (int64_t t = blockIdx.x; t < a.n_tiles; t += gridDim.x) {
    const int rg = (int)(t / a.n_tt);
    const int64_t row = (int64_t)rg * 128 + lr;
    const bool rvalid = row < a.npad;
    for (int st = 0; st < a.n_stages; ++st) {
      if (!pf_wait(S, a, &S.wfull[ws], wph, 6)) return;
      const uint8_t* sb = S.wst + (size_t)ws * pf::kWStageBytes;
      const int slot = 4 * ai + par;
      const uint8_t* prow = sb + pf::kPayOff + lr * 128;
      const uint4 P0 = *reinterpret_cast<const uint4*>(prow + (((2 * par) ^ sw) << 4));
      const uint4 P1 = *reinterpret_cast<const uint4*>(prow + (((2 * par + 1) ^ sw) << 4));
      const uint2 SG = *reinterpret_cast<const uint2*>(sb + pf::kSgnOff + lr * 32 + par * 8);
      const uint32_t EX = *reinterpret_cast<const uint32_t*>(sb + pf::kExpOff + lr * 16 + par * 4);
      const uint32_t E = (EX ^ 0x80808080u) + 0x06060606u;       // e + 134 per byte
      // rows past npad arrive as zero bytes (TMA fill) and dequantise to +0
      uint32_t w[32];
      dq_block(P0.x, P0.y, SG.x & 0xFFFFu, E & 0xFFu, w + 0);
      dq_block(P0.z, P0.w, SG.x >> 16, (E >> 8) & 0xFFu, w + 8);
      dq_block(P1.x, P1.y, SG.y & 0xFFFFu, (E >> 16) & 0xFFu, w + 16);
      dq_block(P1.z, P1.w, SG.y >> 16, E >> 24, w + 24);
      if (a.entries && rvalid) {
        // outliers of this row in this substage's 64 columns go into their +0 slots as
        // bf16(15 v): the epilogue's 1/15 scale then yields v * x
        const int4 rr = *reinterpret_cast<const int4*>(sb + pf::kRangeOff);
        const PfRange orr{rr.x, rr.y, rr.z};
        const uint16_t* ro = reinterpret_cast<const uint16_t*>(sb + pf::kRoffOff);
        const uint32_t* es = reinterpret_cast<const uint32_t*>(sb + pf::kOutOff);
        const int e_end = ro[lr + 1];
        for (int k = ro[lr]; k < e_end; ++k) {
          const int o = orr.lo - orr.lo4 + k;
          const uint32_t e = o < orr.n ? es[o] : __ldg(a.entries + orr.lo + k);
          const int el = (int)((e >> 16) & 0xFFu) - 64 * par;
          if (el < 0 || el >= 64) continue;
          const float v15 = 15.0f * __half2float(__ushort_as_half((unsigned short)(e & 0xFFFFu)));
          patch_pair(w, el, float_to_bf16_bits(v15));
        }
      }
      __syncwarp();
      if (!pf_wait(S, a, &S.aempty[slot], aph ^ 1, 7)) return;
      __syncwarp();
      tc_fence_after();
      tmem_st_32x32b_x32(tmem + pf::kTmemA + slot * 32 + lane_base, w);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&S.afull[slot]);
        mbar_arrive(&S.wempty[ws]);
      }
      if (++ws == pf::kWStages) { ws = 0; wph ^= 1; }
      if (++ai == pf::kASlots / 4) { ai = 0; aph ^= 1; }
    }
  }
}

// ---------------------------------------------------------------------------------------
__device__ void pf_epilogue(const PfShared& S, const PfArgs& a, uint32_t tmem) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q4 = warp & 3;
  const int lr = q4 * 32 + lane;
  const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
  const float inv15 = 1.0f / 15.0f;
  uint32_t dph = 0;
  for (int64_t t = blockIdx.x; t < a.n_tiles; t += gridDim.x) {
    const int rg = (int)(t / a.n_tt), tt = (int)(t % a.n_tt);
    const int64_t row = (int64_t)rg * 128 + lr;
    const bool store = row < a.n_out;
    const float bv = (store && a.bias) ? load_as_float(a.bias, a.bias_dtype, row) : 0.f;
    const int tok0 = tt * pf::kBN;
    const int ntok = min(pf::kBN, a.m - tok0);
    if (!pf_wait(S, a, S.dfull, dph, 8)) return;
    __syncwarp();
    tc_fence_after();
    for (int cb = 0; cb < pf::kBN / 16; ++cb) {
      if (cb * 16 >= ntok) break;                       // warp-uniform
      float v[16];
      tmem_ld_32x32b_x16(tmem + pf::kTmemD + cb * 16 + lane_base, v);
      tmem_wait_ld();
      if (store) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int tok = cb * 16 + j;
          if (tok < ntok)
            store_from_float(a.y, a.y_dtype, (int64_t)(tok0 + tok) * a.ldy + row, fmaf(v[j], inv15, bv));
        }
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(S.dempty);
    dph ^= 1;
  }
}

__global__ void __launch_bounds__(pf::kThreads, 1)
prefill_tc_kernel(const PfArgs a, const __grid_constant__ PfMaps M) {
  extern __shared__ uint8_t smem_raw[];
  const PfShared S = pf_shared(smem_raw);
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    for (int s = 0; s < pf::kWStages; ++s) { mbar_init(&S.wfull[s], 1); mbar_init(&S.wempty[s], pf::kDq); }
    for (int s = 0; s < pf::kXSlots; ++s) { mbar_init(&S.xfull[s], 1); mbar_init(&S.xempty[s], 1); }
    for (int j = 0; j < pf::kASlots; ++j) { mbar_init(&S.afull[j], 4); mbar_init(&S.aempty[j], 1); }
    mbar_init(S.dfull, 1);
    mbar_init(S.dempty, 4);
    mbar_init(S.mtail, 1);
    *S.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(S.tmem_slot, pf::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *S.tmem_slot;

  if (warp == 0) {
    if (elect_one_sync()) pf_producer_thread(S, a, M);
    __syncwarp();
  } else if (warp == 1) {
    if (elect_one_sync()) pf_mma(S, a, tmem);
    __syncwarp();
  } else if (warp >= pf::kEpiWarp0 && warp < pf::kDqWarp0) {
    pf_epilogue(S, a, tmem);
  } else if (warp >= pf::kDqWarp0) {
    pf_dequant(S, a, tmem);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, pf::kTmemCols);
  }
}

}  // namespace fbfp

using namespace fbfp;

extern "C" int fbfp_gemm_prefill(const void* x, int x_dtype, int64_t m, int64_t ldx,
                                 const int8_t* exponents, const int16_t* signs, const int32_t* payload,
                                 int64_t n_out, int64_t k_in, int64_t kpad, int64_t npad,
                                 const uint32_t* entries, const int32_t* seg_ptr, const void* bias,
                                 int bias_dtype, void* y, int y_dtype, int64_t ldy, void* workspace,
                                 void* stream) {
  FBFP_CHECK_ARG(x && exponents && signs && payload && y && workspace, "null pointer");
  FBFP_CHECK_ARG(x_dtype == FBFP_BF16, "fbfp_gemm_prefill needs bf16 activations");
  FBFP_CHECK_ARG(m >= 1 && m <= ((int64_t)1 << 30), "bad m %lld", (long long)m);
  FBFP_CHECK_ARG(kpad > 0 && kpad % (kBlock * kStageKb) == 0,
                 "fbfp_gemm_prefill needs Kpad to be a multiple of %d (got %lld)", kBlock * kStageKb,
                 (long long)kpad);
  FBFP_CHECK_ARG(k_in > 0 && k_in <= kpad && k_in % 8 == 0 && ldx >= k_in && ldx % 8 == 0,
                 "bad k_in/ldx (%lld, %lld): need k_in <= Kpad, k_in and ldx multiples of 8",
                 (long long)k_in, (long long)ldx);
  FBFP_CHECK_ARG(npad > 0 && npad % 64 == 0 && n_out > 0 && n_out <= npad && ldy >= n_out,
                 "bad n_out/npad/ldy");
  FBFP_CHECK_ARG(((uintptr_t)x & 15) == 0 && ((uintptr_t)payload & 15) == 0 &&
                 ((uintptr_t)signs & 15) == 0 && ((uintptr_t)exponents & 15) == 0,
                 "x and the packed arrays must be 16-byte aligned");
  FBFP_CHECK_ARG((entries == nullptr) == (seg_ptr == nullptr), "entries and seg_ptr go together");
  FBFP_CHECK_ARG(y_dtype == FBFP_BF16 || y_dtype == FBFP_F16 || y_dtype == FBFP_F32, "bad y dtype");
  const int64_t kb_row = kpad / kBlock;
  PfArgs a;
  a.m = (int)m; a.ldx = ldx; a.n_out = n_out; a.k_in = k_in; a.npad = npad;
  a.entries = entries; a.seg_ptr = seg_ptr; a.bias = bias; a.bias_dtype = bias_dtype;
  a.y = y; a.y_dtype = y_dtype; a.ldy = ldy;
  a.err = reinterpret_cast<int32_t*>(workspace);
  a.n_stages = (int)(kb_row / kStageKb);
  a.x_rows = (int)(m < pf::kBN ? m : pf::kBN);
  a.n_tt = (int)((m + pf::kBN - 1) / pf::kBN);
  const int64_t n_rg = (npad + kGroupRows - 1) / kGroupRows;
  a.n_tiles = n_rg * a.n_tt;
  a.n_seg = n_rg * a.n_stages;
  PfMaps M;
  int rc;
  if ((rc = encode_2d(&M.pay, CU_TENSOR_MAP_DATA_TYPE_UINT8, payload, (uint64_t)kb_row * 8, (uint64_t)npad,
                      (uint64_t)kb_row * 8, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B)) != FBFP_OK) return rc;
  if ((rc = encode_2d(&M.sgn, CU_TENSOR_MAP_DATA_TYPE_UINT16, signs, (uint64_t)kb_row, (uint64_t)npad,
                      (uint64_t)kb_row * 2, kStageKb, 128, CU_TENSOR_MAP_SWIZZLE_NONE)) != FBFP_OK) return rc;
  if ((rc = encode_2d(&M.exp, CU_TENSOR_MAP_DATA_TYPE_UINT8, exponents, (uint64_t)kb_row, (uint64_t)npad,
                      (uint64_t)kb_row, kStageKb, 128, CU_TENSOR_MAP_SWIZZLE_NONE)) != FBFP_OK) return rc;
  if ((rc = encode_2d(&M.x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, (uint64_t)k_in, (uint64_t)m,
                      (uint64_t)ldx * 2, 64, (uint32_t)a.x_rows, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_128B)) != FBFP_OK) return rc;
  int dev = 0;
  FBFP_CUDA_TRY(cudaGetDevice(&dev));
  static bool attr_set[64] = {false};
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    FBFP_CUDA_TRY(cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)pf::kSmemBytes));
    attr_set[dev] = true;
  }
  const int64_t nsm = sm_count(dev);
  const int64_t grid = nsm < a.n_tiles ? nsm : a.n_tiles;
  prefill_tc_kernel<<<(unsigned)grid, pf::kThreads, pf::kSmemBytes, as_stream(stream)>>>(a, M);
  FBFP_LAUNCH_CHECK("prefill_tc_kernel");
  return FBFP_OK;
}
