// gemv_tc.cu — persistent warp-specialised OABF decode GEMV on tcgen05 (sm_100a).
//
// Same contract as the generic kernel in gemv.cu (y = x W_full^T + bias for 1 <= M <= 16
// tokens; replaces oabf_gemm_kernel, flash_bfp/triton_kernel.py:22-86, and the outlier
// SpMV/bias of OABFLinear.forward, :339-362), for matrices whose row length is a multiple
// of 16 blocks. Roles inside one CTA per SM:
//   warp 0      producer: tensor copies (TMA) of 128-row x 16-block stages of the packed
//               reference layout (payload with 128-byte swizzle so lane-per-row reads are
//               conflict free, signs, exponents) and of the stage's activations straight into
//               the MMA B layout (K-major core matrices, tokens >= M zero-filled) into a
//               5-deep shared-memory ring;
//   warp 1      MMA issuer: one thread issues tcgen05.mma (M=128 rows, N=16 tokens, K=16)
//               with A read from tensor memory, one MMA per block (a small-N tcgen05.mma
//               occupies the tensor pipe ~45 cycles whatever N <= 64, so one per block is
//               the budget that keeps up with HBM);
//   warps 2-3   idle;
//   warps 4-7   epilogue (one per tensor-memory lane quarter): drain the double-buffered fp32
//               accumulator of each (row group, CTA) segment while the next segment streams,
//               scale by 1/15, add outlier sums, then write y or reduce across CTAs;
//   warps 8-23  dequantisers (4 per tensor-memory lane quarter, one 4-block substage each):
//               one row per lane; each block becomes 8 bf16 pairs s*m*2^e built
//               exactly with bit operations (PRMT/LOP3 magic pair minus its offset, HSUB2) and
//               stored into a tensor-memory ring with tcgen05.st;
//               outliers ride along: the producer stages each stage's outlier entries and
//               per-row starts, and the dequantisers accumulate v * x in fp32 for the row's
//               outliers (x read from the stage's activation tile; for M <= 4 the 4 warps of
//               a row split its entries) and hand the sums to the epilogue through shared memory.
// Work: stream-K over units (128-row group, 16-block stage); each CTA takes a contiguous
// range. Every mbarrier wait is bounded: on timeout the CTA records an error code in the
// workspace and winds down (waiting, bounded, for its own copies) before freeing TMEM.
#include <cuda.h>

#include "common.cuh"
#include "sm100.cuh"
#include "tc_args.h"
#include "tc_host.h"
#include "dq_pair.cuh"
#include "exchange.cuh"

namespace fbfp {
using namespace sm100;

namespace tc {
constexpr int kStages = 5;
constexpr int kASlots = 12;                     // tensor-memory A ring (4 blocks each)
constexpr int kPayOff = 0;                      // 128 rows x 128 B, 128-byte swizzle
constexpr int kSgnOff = 128 * 128;              // 128 rows x 32 B
constexpr int kExpOff = kSgnOff + 128 * 32;     // 128 rows x 16 B
constexpr int kXOff = kExpOff + 128 * 16;       // activations: 4 boxes of 64 k x <= 16 tokens
constexpr int kXBox = 2048;                     // (128-byte swizzled rows, two 1024-byte atoms)
constexpr int kOutOff = kXOff + 4 * kXBox;                    // stage's outlier entries
constexpr int kOutCap = 2048;                                 // entries staged per stage
constexpr int kRoffOff = kOutOff + kOutCap * 4;              // 136 uint16 row starts of the stage
constexpr int kRoffBytes = 272;
constexpr int kStageBytes = kRoffOff + 1024;                  // 39936 (multiple of 1024)
constexpr uint32_t kWeightTx = kXOff;                        // payload + signs + exponents bytes
constexpr int kSegCache = 1024;                               // segment pointers cached per CTA
constexpr int kDqPerQuarter = 3;                 // dequantiser warps per tensor-memory lane quarter
constexpr int kDq = 4 * kDqPerQuarter;
static_assert(kASlots == 4 * kDqPerQuarter, "dequantiser warp p of a quarter owns A slots 4p..4p+3");                         // dequantiser warps (2..17), 4 per lane quarter
constexpr int kEpiWarp0 = 4;                    // epilogue warpgroup: warps 4-7
constexpr int kDqWarp0 = 8;                     // dequantisers: warps 8 .. 8 + kDq - 1
constexpr int kOutWarp0 = kDqWarp0 + kDq;       // outlier warpgroup: warps 20-23
constexpr int kThreads = 32 * (kOutWarp0 + 4);  // 768: 6 warps per SM sub-partition
static_assert(kDq % 4 == 0, "dequantisers come in whole warpgroups");
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemD = 0;                  // 2 accumulators x 16 columns
constexpr uint32_t kTmemA = 32;                 // 12 slots x 32 columns (4 blocks x 8)
constexpr size_t kSoutOff = (size_t)kStages * kStageBytes;
constexpr size_t kSegOff = kSoutOff;
// outlier sums handed from the outlier warps to the epilogue: [2 accumulators][16 tokens][128 rows]
// fp32 (one lane owns each row, so plain stores)
constexpr size_t kOaccOff = kSegOff + (kSegCache + 8) * sizeof(int32_t);
constexpr size_t kOaccBytes = 2 * 16 * 128 * sizeof(float);
// finished values of the rows an epilogue warp owns, [4 warps][16 tokens][32 lanes] fp32
constexpr size_t kXvOff = kOaccOff + kOaccBytes;
constexpr size_t kXvBytes = 4 * 16 * 32 * sizeof(float);
constexpr size_t kBarOff = kXvOff + kXvBytes;
constexpr int kNumBars = 2 * kStages + 2 * kASlots + 9;
constexpr size_t kSmemBytes = kBarOff + kNumBars * 8 + 16 + 1024;   // + alignment slack
static_assert(kSmemBytes <= 232448, "exceeds the 227 KB of shared memory a CTA may opt in to");
}  // namespace tc

struct TcMaps {
  CUtensorMap pay, sgn, exp, x;
};

struct TcShared {
  uint8_t* stage;
  float* s_out;
  int32_t* seg;          // seg_ptr[u0 .. u0 + kSegCache]
  uint64_t *full, *empty, *afull, *aempty, *dfull, *dempty, *ofull, *oempty;
  uint64_t* mtail;       // the MMA thread's last commit (its MMAs have completed)
  float* oacc;           // [2][16][128]
  float* xv;             // [4][16][32]
  uint32_t* tmem_slot;
  volatile int* abort_flag;
};

__device__ __forceinline__ TcShared tc_shared(uint8_t* smem_raw) {
  // stage buffers need 1024-byte alignment (128-byte swizzled TMA destination)
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  TcShared S;
  S.stage = smem;
  S.s_out = reinterpret_cast<float*>(smem + tc::kSoutOff);
  S.seg = reinterpret_cast<int32_t*>(smem + tc::kSegOff);
  uint64_t* b = reinterpret_cast<uint64_t*>(smem + tc::kBarOff);
  S.full = b;
  S.empty = S.full + tc::kStages;
  S.afull = S.empty + tc::kStages;
  S.aempty = S.afull + tc::kASlots;
  S.dfull = S.aempty + tc::kASlots;
  S.dempty = S.dfull + 2;
  S.ofull = S.dempty + 2;
  S.oempty = S.ofull + 2;
  S.oacc = reinterpret_cast<float*>(smem + tc::kOaccOff);
  S.xv = reinterpret_cast<float*>(smem + tc::kXvOff);
  S.mtail = S.oempty + 2;
  S.tmem_slot = reinterpret_cast<uint32_t*>(S.mtail + 1);
  S.abort_flag = reinterpret_cast<volatile int*>(S.tmem_slot + 1);
  return S;
}

// Bounded wait that also gives up as soon as another role of the CTA has aborted. Each poll
// may suspend the thread for up to 20 us (it wakes when the phase completes); 2^16 polls bound
// the wait to about a second.
__device__ __forceinline__ bool tc_wait(const TcShared& S, const TcArgs& a, uint64_t* bar,
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

// Outlier-entry range of local unit i (global unit u0 + i): [lo, hi) plus the 16-byte aligned
// window [lo4, lo4 + n) that the producer stages in shared memory.
struct OutRange { int lo, hi, lo4, n; };
__device__ __forceinline__ const uint8_t* roff_block(const TcArgs& a, int64_t u) {
  const int64_t base = (a.total_units + 1 + 3) & ~(int64_t)3;        // words of segment pointers
  return reinterpret_cast<const uint8_t*>(a.seg_ptr + base + u * 68);
}
__device__ __forceinline__ OutRange out_range(const TcShared& S, const TcArgs& a, int64_t u0, int64_t i) {
  OutRange r{0, 0, 0, 0};
  if (!a.entries) return r;
  if (i < tc::kSegCache) { r.lo = S.seg[i]; r.hi = S.seg[i + 1]; }
  else { r.lo = __ldg(a.seg_ptr + u0 + i); r.hi = __ldg(a.seg_ptr + u0 + i + 1); }
  if (r.hi > r.lo) {
    r.lo4 = r.lo & ~3;
    r.n = ((r.hi + 3) & ~3) - r.lo4;
    if (r.n > tc::kOutCap) r.n = tc::kOutCap;
  }
  return r;
}

// ---------------------------------------------------------------------------------------
// producer: tensor copies per stage (payload, signs, exponents, activations) plus the stage's
// outlier entries and row starts
__device__ __forceinline__ void tc_issue_weights(const TcShared& S, const TcArgs& a, const TcMaps& M,
                                                 int64_t u0, int64_t i, int64_t u, int s, uint32_t xbytes) {
  uint8_t* sb = S.stage + (size_t)s * tc::kStageBytes;
  const OutRange orr = out_range(S, a, u0, i);
  const int rg = (int)(u / a.n_stages), st = (int)(u % a.n_stages);
  mbar_arrive_expect_tx(&S.full[s], tc::kWeightTx + xbytes + (uint32_t)orr.n * 4 +
                                        (a.entries ? tc::kRoffBytes : 0));
  tma_2d_g2s(sb + tc::kPayOff, &M.pay, st * 128, rg * 128, &S.full[s]);
  tma_2d_g2s(sb + tc::kSgnOff, &M.sgn, st * kStageKb, rg * 128, &S.full[s]);
  tma_2d_g2s(sb + tc::kExpOff, &M.exp, st * kStageKb, rg * 128, &S.full[s]);
  if (orr.n) bulk_g2s(sb + tc::kOutOff, a.entries + orr.lo4, (uint32_t)orr.n * 4, &S.full[s]);
  if (a.entries) bulk_g2s(sb + tc::kRoffOff, roff_block(a, u), tc::kRoffBytes, &S.full[s]);
}
__device__ __forceinline__ void tc_issue_x(const TcShared& S, const TcArgs& a, const TcMaps& M,
                                           int64_t u, int s) {
  uint8_t* sb = S.stage + (size_t)s * tc::kStageBytes;
  const int st = (int)(u % a.n_stages);
#pragma unroll
  for (int b = 0; b < 4; ++b)
    tma_2d_g2s(sb + tc::kXOff + b * tc::kXBox, &M.x, st * 256 + b * 64, 0, &S.full[s]);
}

__device__ void tc_producer(const TcShared& S, const TcArgs& a, const TcMaps& M, int64_t u0, int64_t u1) {
  int64_t i = 0;
  if (elect_one_sync()) {
    prefetch_tmap(&M.pay); prefetch_tmap(&M.sgn); prefetch_tmap(&M.exp); prefetch_tmap(&M.x);
    const uint32_t xbytes = 4u * 128u * (uint32_t)a.m;          // 4 boxes of 64 k x m tokens
    // With resident weights (early_weights) the first stages' weights, outlier entries and row
    // starts are fetched before waiting for the previous kernel in the stream, then the
    // activations (otherwise the kernel has already waited and both waits are one).
    const int64_t npre = (u1 - u0) < tc::kStages ? (u1 - u0) : tc::kStages;
    for (int64_t j = 0; j < npre; ++j) tc_issue_weights(S, a, M, u0, j, u0 + j, (int)j, xbytes);
    grid_dependency_wait();
    for (int64_t j = 0; j < npre; ++j) tc_issue_x(S, a, M, u0 + j, (int)j);
    i = npre;
    int s = (int)(npre % tc::kStages);
    uint32_t ph = npre == tc::kStages ? 1u : 0u;
    for (int64_t u = u0 + npre; u < u1; ++u, ++i) {
      if (!tc_wait(S, a, &S.empty[s], ph ^ 1, 1)) break;
      tc_issue_weights(S, a, M, u0, i, u, s, xbytes);
      tc_issue_x(S, a, M, u, s);
      if (++s == tc::kStages) { s = 0; ph ^= 1; }
    }
    // wind down: every stage issued so far must have landed before the CTA may exit, and,
    // unless the CTA aborted, every consumer must have released it, so that no asynchronous
    // arrival (an MMA commit) is still due on a stage barrier when the shared memory is freed
    const int64_t j0 = i > tc::kStages ? i - tc::kStages : 0;
    for (int64_t j = j0; j < i; ++j)
      mbar_wait(&S.full[j % tc::kStages], (uint32_t)(j / tc::kStages) & 1, 1u << 20);
    for (int64_t j = j0; j < i; ++j)
      if (*S.abort_flag || !mbar_wait(&S.empty[j % tc::kStages], (uint32_t)(j / tc::kStages) & 1, 1u << 22))
        break;
  }
  __syncwarp();
}

// ---------------------------------------------------------------------------------------
// Issues the MMAs of units [u0, u1); `uses` counts the A-slot uses committed. False if a wait
// gave up (the CTA aborts).
__device__ bool tc_mma_loop(const TcShared& S, const TcArgs& a, int64_t u0, int64_t u1, uint32_t tmem,
                            int64_t& uses) {
  constexpr uint32_t IDESC = idesc_bf16_f32(128, 16, false);
  // B: a substage's 4 blocks are one 64-k box of tokens (rows) in 128-byte swizzled K-major
  // layout; token groups of 8 are 1024 B apart; block j of the box starts 32 * j bytes in
  const uint64_t desc0 = smem_desc_sw128(smem_u32(S.stage + tc::kXOff), 1024);
  constexpr uint64_t kStageDesc = (uint64_t)(tc::kStageBytes >> 4);
  constexpr uint64_t kBoxDesc = (uint64_t)(tc::kXBox >> 4);
  constexpr uint64_t kKbDesc = 2;                                 // 32 bytes
  int64_t seg = 0;
  int s = 0, slot = 0;
  uint32_t aph = 0;
  for (int64_t u = u0; u < u1; ++seg) {
    const int64_t rg = u / a.n_stages;
    const int64_t seg_end = min(u1, (rg + 1) * a.n_stages);
    const int d = (int)(seg & 1);
    if (!tc_wait(S, a, &S.dempty[d], (uint32_t)((seg >> 1) & 1) ^ 1, 2)) return false;
    tc_fence_after();
    const uint32_t tD = tmem + tc::kTmemD + d * 16;
    uint32_t acc = 0;
    for (; u < seg_end; ++u) {
      const uint64_t dstage = desc0 + (uint64_t)s * kStageDesc;
      for (int sub = 0; sub < 4; ++sub) {
        if (!tc_wait(S, a, &S.afull[slot], aph, 3)) return false;
        tc_fence_after();
        const uint32_t tA = tmem + tc::kTmemA + slot * 32;
        const uint64_t dsub = dstage + (uint64_t)sub * kBoxDesc;
        mma_ts(tD, tA + 0, dsub + 0 * kKbDesc, IDESC, acc);
        mma_ts(tD, tA + 8, dsub + 1 * kKbDesc, IDESC, 1);
        mma_ts(tD, tA + 16, dsub + 2 * kKbDesc, IDESC, 1);
        mma_ts(tD, tA + 24, dsub + 3 * kKbDesc, IDESC, 1);
        acc = 1;
        mma_commit(&S.aempty[slot]);
        ++uses;
        if (++slot == tc::kASlots) { slot = 0; aph ^= 1; }
      }
      mma_commit(&S.empty[s]);
      if (++s == tc::kStages) s = 0;
    }
    mma_commit(&S.dfull[d]);
  }
  return true;
}

__device__ void tc_mma(const TcShared& S, const TcArgs& a, int64_t u0, int64_t u1, uint32_t tmem) {
  int64_t uses = 0;
  const bool ok = tc_mma_loop(S, a, u0, u1, tmem, uses);
  if (uses > 0) {
    // every MMA this thread issued completes before the tensor memory is released (also when
    // the CTA aborts with MMAs in flight)
    mma_commit(S.mtail);
    mbar_wait(S.mtail, 0, 1u << 22);
  }
  if (ok) {
    // the commit arrivals on the A-slot barriers land before the shared memory is released:
    // use t of slot t % kASlots completes that barrier's phase t / kASlots
    for (int j = 0; j < tc::kASlots && j < uses; ++j) {
      const int64_t last = j + (uses - 1 - j) / tc::kASlots * tc::kASlots;
      if (!mbar_wait(&S.aempty[j], (uint32_t)(last / tc::kASlots) & 1, 1u << 22)) break;
    }
  }
}

// Outliers of row lr in one stage (their dense slots are +0): oacc[t] += v * x[t] for the first
// NT tokens over all the row's entries; x comes from the stage's activation tile: column c of
// token t is in box c / 64, 1024-byte atom t / 8, 128-byte row t % 8, 16-byte chunk
// ((c % 64) / 8) ^ (t % 8) (128-byte swizzle), element c % 8.
template <int NT>
__device__ __forceinline__ void tc_row_outliers(const uint8_t* sb, const OutRange& orr,
                                                const uint32_t* entries, int lr, float* oacc) {
  const uint16_t* ro = reinterpret_cast<const uint16_t*>(sb + tc::kRoffOff);
  const uint32_t* es = reinterpret_cast<const uint32_t*>(sb + tc::kOutOff);
  const uint8_t* xs = sb + tc::kXOff;
  const int e_end = ro[lr + 1];
  const int obase = orr.lo - orr.lo4;
  for (int k = ro[lr]; k < e_end; ++k) {
    const int o = obase + k;
    const uint32_t e = o < orr.n ? es[o] : __ldg(entries + orr.lo + k);
    const float v = __half2float(__ushort_as_half((unsigned short)(e & 0xFFFFu)));
    // box * 2048 + (c % 8) * 2 from bits 22-23 and 16-18 of the entry; chunk from bits 19-21
    const uint8_t* xp = xs + (((e >> 11) & 0x1800u) | ((e >> 15) & 0xEu));
    const uint32_t chunk = (e >> 19) & 7u;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const uint32_t r = (uint32_t)(t & 7);
      const uint32_t off = (uint32_t)(t >> 3) * 1024u + (r << 7) + ((chunk ^ r) << 4);
      oacc[t] = fmaf(v, __uint_as_float((uint32_t)*reinterpret_cast<const uint16_t*>(xp + off) << 16),
                     oacc[t]);
    }
  }
}

// Dequantisers: warp p of a lane quarter takes the stages i = p (mod 3) of the CTA's units, all
// 16 blocks of each for its 32 rows, so the three warps of a sub-partition work on different
// stages. Substage c of stage i goes to A slot 4p + c (the 12-slot ring holds 3 stages).
__device__ void tc_dequant(const TcShared& S, const TcArgs& a, int64_t u0, int64_t u1, uint32_t tmem) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wi = warp - tc::kDqWarp0;     // 0..kDq-1
  const int q4 = warp & 3;                 // tensor-memory lane quarter
  const int par = wi >> 2;                 // this warp's stages: i = par (mod 3)
  const int lr = q4 * 32 + lane;           // row within the group
  const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
  const int sw = lr & 7;                   // 128-byte swizzle phase of this row
  int i = 0;                               // local unit index
  for (int64_t u = u0; u < u1; ++u, ++i) {
    if (i % tc::kDqPerQuarter != par) continue;
    const int s = i % tc::kStages;
    if (!tc_wait(S, a, &S.full[s], (uint32_t)(i / tc::kStages) & 1, 4)) return;
    const uint8_t* sb = S.stage + (size_t)s * tc::kStageBytes;
    const uint32_t aph = (uint32_t)(i / tc::kDqPerQuarter) & 1;
    const uint8_t* prow = sb + tc::kPayOff + lr * 128;
    // not unrolled: one copy of the block dequantiser keeps the kernel's code within the
    // instruction cache next to the other roles
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {            // substages (4 blocks each)
      const int slot = 4 * par + c;
      const uint4 P0 = *reinterpret_cast<const uint4*>(prow + (((2 * c) ^ sw) << 4));
      const uint4 P1 = *reinterpret_cast<const uint4*>(prow + (((2 * c + 1) ^ sw) << 4));
      const uint2 SG = *reinterpret_cast<const uint2*>(sb + tc::kSgnOff + lr * 32 + c * 8);
      const uint32_t EX = *reinterpret_cast<const uint32_t*>(sb + tc::kExpOff + lr * 16 + c * 4);
      const uint32_t E = (EX ^ 0x80808080u) + 0x06060606u;       // e + 134 per byte
      const uint32_t sg0 = SG.x, sg1 = SG.y;
      if (!tc_wait(S, a, &S.aempty[slot], aph ^ 1, 5)) return;
      __syncwarp();
      tc_fence_after();
      // rows past npad arrive as zero bytes (TMA fill) and dequantise to +0
      const uint32_t ta = tmem + tc::kTmemA + slot * 32 + lane_base;
      uint32_t w[8];
      dq_block(P0.x, P0.y, sg0 & 0xFFFFu, E & 0xFFu, w);
      tmem_st_32x32b_x8(ta + 0, w);
      dq_block(P0.z, P0.w, sg0 >> 16, (E >> 8) & 0xFFu, w);
      tmem_st_32x32b_x8(ta + 8, w);
      dq_block(P1.x, P1.y, sg1 & 0xFFFFu, (E >> 16) & 0xFFu, w);
      tmem_st_32x32b_x8(ta + 16, w);
      dq_block(P1.z, P1.w, sg1 >> 16, E >> 24, w);
      tmem_st_32x32b_x8(ta + 24, w);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.afull[slot]);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&S.empty[s]);
  }
}

// Outlier warps (one per lane quarter, one row per lane): every stage, the row's outlier entries
// times the activations in fp32 (their dense slots are +0); at each segment end the sums go to
// the epilogue through shared memory.
__device__ void tc_outliers(const TcShared& S, const TcArgs& a, int64_t u0, int64_t u1) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q4 = warp & 3;
  const int lr = q4 * 32 + lane;
  const int m = a.m;
  int64_t seg = 0;
  int i = 0;
  for (int64_t u = u0; u < u1; ++seg) {
    const int64_t rg = u / a.n_stages;
    const int64_t seg_end = min(u1, (rg + 1) * a.n_stages);
    const bool rvalid = rg * 128 + lr < a.npad;
    float oacc[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) oacc[t] = 0.f;
    for (; u < seg_end; ++u, ++i) {
      const int s = i % tc::kStages;
      if (!tc_wait(S, a, &S.full[s], (uint32_t)(i / tc::kStages) & 1, 10)) return;
      const uint8_t* sb = S.stage + (size_t)s * tc::kStageBytes;
      if (rvalid) {
        const OutRange orr = out_range(S, a, u0, i);
        if (m == 1) tc_row_outliers<1>(sb, orr, a.entries, lr, oacc);
        else if (m <= 4) tc_row_outliers<4>(sb, orr, a.entries, lr, oacc);
        else tc_row_outliers<16>(sb, orr, a.entries, lr, oacc);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.empty[s]);
    }
    const int d = (int)(seg & 1);
    if (!tc_wait(S, a, &S.oempty[d], ((uint32_t)(seg >> 1) & 1) ^ 1, 7)) return;
    float* so = S.oacc + (size_t)(d * 16) * 128 + lr;
#pragma unroll
    for (int t = 0; t < 16; ++t)
      if (t < m) so[t * 128] = oacc[t];
    __syncwarp();
    if (lane == 0) mbar_arrive(&S.ofull[d]);
  }
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Waits (bounded by the all-reduce handle's timeout, or until another role of the CTA aborts) for the word of
// this call's tag at `src` and returns its value in *v.
__device__ __forceinline__ bool tc_xchg_wait(const TcShared& S, const TcArgs& a, const uint2* src,
                                             uint32_t tag, int code, float* v) {
  uint2 w = xchg_load(src);
  uint64_t t0 = 0;
  for (uint32_t it = 1; w.y != tag; ++it) {
    if ((it & 63) == 0) {
      if (*S.abort_flag) return false;
      const uint64_t now = global_ns();
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

// Final values of output row `row` for the m tokens; the lane's values v[t] sit at xv[32 t].
// One rank: y = v + bias. Row-parallel exchange (world > 1): push v to every peer's slot
// [par][rank], then y = bias + the sum in rank order of every rank's v (identical bits on all
// ranks). Returns false if a wait gave up.
__device__ __forceinline__ bool tc_finish_row(const TcShared& S, const TcArgs& a, int64_t row,
                                              const float* xv, uint32_t tag, uint32_t par) {
  const volatile float* v = xv;
  const int m = a.m;
  const float bv = a.bias ? load_as_float(a.bias, a.bias_dtype, row) : 0.f;
  if (a.world > 1) {
    for (int p = 0; p < a.world; ++p) {
      if (p == a.rank) continue;
      uint2* dst = xchg_slot(a.xbuf[p], a.xmax, par, a.rank) + row;
      for (int t = 0; t < m; ++t) xchg_store(dst + (int64_t)t * a.n_out, __float_as_uint(v[32 * t]), tag);
    }
  }
  for (int t = 0; t < m; ++t) {
    float acc = v[32 * t];
    if (a.world > 1) {
      acc = 0.f;
      for (int q = 0; q < a.world; ++q) {
        float w = v[32 * t];
        if (q != a.rank &&
            !tc_xchg_wait(S, a, xchg_slot(a.xbuf[a.rank], a.xmax, par, q) + (int64_t)t * a.n_out + row,
                          tag, 32 + q, &w))
          return false;
        acc += w;
      }
    }
    store_from_float(a.y, a.y_dtype, (int64_t)t * a.ldy + row, acc + bv);
  }
  return true;
}

// Epilogue warpgroup (warp w reads tensor-memory lane quarter w % 4, i.e. rows 32q .. 32q+31 of
// the group): per segment it drains the accumulator (all m tokens), adds the dequantisers'
// outlier partial sums, then either finishes the rows directly (the CTA covered the whole row
// group) or adds into the fp32 workspace; a counter per (row group, quarter) collects the units
// of all CTAs and the warp that completes it finishes the rows and returns the workspace rows to
// zero. Finishing a row writes y, after the exchange with the other ranks when it is fused in.
//
// The exchange cannot deadlock: all CTAs of the grid are resident (one per SM), every rank
// finishes every row group, and a CTA finishes its row groups in increasing order, so on every
// rank each contribution to the lowest row group any CTA waits on is either made or comes from a
// CTA that is not waiting (ranks may split K, and so their units, differently).
__device__ void tc_epilogue(const TcShared& S, const TcArgs& a, int64_t u0, int64_t u1, uint32_t tmem) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q4 = warp & 3;
  const int lr = q4 * 32 + lane;
  const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
  const int m = a.m;
  const float inv15 = 1.0f / 15.0f;
  grid_dependency_wait();                 // the workspace and y may still be in use before this
  float* xv = S.xv + q4 * 16 * 32 + lane;  // this lane's finished values, one per token
  uint32_t tag = 0, par = 0;
  if (a.world > 1) {                      // this call's exchange epoch (advanced at kernel exit)
    const uint32_t e = *reinterpret_cast<volatile uint32_t*>(xchg_epoch(a.xbuf[a.rank]));
    par = e & 1u;
    tag = e + 1u;
  }
  int64_t seg = 0;
  for (int64_t u = u0; u < u1; ++seg) {
    const int64_t rg = u / a.n_stages;
    const int64_t seg_begin = u, seg_end = min(u1, (rg + 1) * a.n_stages);
    u = seg_end;
    const int64_t row = rg * 128 + lr;
    const bool rvalid = row < a.npad;
    const int d = (int)(seg & 1);
    const uint32_t ph = (uint32_t)(seg >> 1) & 1;
    if (!tc_wait(S, a, &S.dfull[d], ph, 6)) return;
    __syncwarp();
    tc_fence_after();
    float val[16];
    tmem_ld_32x32b_x16(tmem + tc::kTmemD + d * 16 + lane_base, val);
    tmem_wait_ld();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&S.dempty[d]);
#pragma unroll
    for (int t = 0; t < 16; ++t) val[t] *= inv15;
    if (a.entries) {
      if (!tc_wait(S, a, &S.ofull[d], ph, 8)) return;
      const float* so = S.oacc + (size_t)(d * 16) * 128 + lr;     // [t][row]
#pragma unroll
      for (int t = 0; t < 16; ++t)
        if (t < m) val[t] += so[t * 128];
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.oempty[d]);
    }
    const bool whole = seg_begin == rg * a.n_stages && seg_end == (rg + 1) * a.n_stages;
    if (whole) {
      bool ok = true;
      if (rvalid && row < a.n_out) {
#pragma unroll
        for (int t = 0; t < 16; ++t)
          if (t < m) xv[32 * t] = val[t];
        ok = tc_finish_row(S, a, row, xv, tag, par);
      }
      if (!__all_sync(0xffffffffu, ok)) return;
      continue;
    }
    if (rvalid) {
#pragma unroll
      for (int t = 0; t < 16; ++t)
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
        for (int t = 0; t < m; ++t) {
          float* wp = a.ws + (int64_t)t * a.npad + row;
          xv[32 * t] = __ldcg(wp);
          __stcg(wp, 0.f);
        }
        if (row < a.n_out) ok = tc_finish_row(S, a, row, xv, tag, par);
      }
      __syncwarp();
      if (lane == 0) a.counters[rg * 4 + q4] = 0;
      if (!__all_sync(0xffffffffu, ok)) return;
    }
  }
}

__global__ void __launch_bounds__(tc::kThreads, 1)
gemv_tc_kernel(const TcArgs a, const __grid_constant__ TcMaps M) {
  extern __shared__ uint8_t smem_raw[];
  const TcShared S = tc_shared(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int64_t U = a.total_units;
  const int64_t u0 = (int64_t)blockIdx.x * U / gridDim.x;
  const int64_t u1 = (int64_t)(blockIdx.x + 1) * U / gridDim.x;
  // Programmatic launch: the previous kernel in the stream may still be running. Unless the
  // caller vouched that it did not write the weights (fbfp_gemv_resident), read no global memory
  // before it has completed; the barrier setup below still overlaps its tail.
  if (!a.early_weights) grid_dependency_wait();

  if (threadIdx.x == 0) {
    // a stage is released by the dequantiser of each lane quarter that took it, the MMA and,
    // with outliers, the 4 outlier warps
    const uint32_t rel = 4 + 1 + (a.entries ? 4 : 0);
    for (int s = 0; s < tc::kStages; ++s) { mbar_init(&S.full[s], 1); mbar_init(&S.empty[s], rel); }
    for (int j = 0; j < tc::kASlots; ++j) { mbar_init(&S.afull[j], 4); mbar_init(&S.aempty[j], 1); }
    for (int d = 0; d < 2; ++d) {
      mbar_init(&S.dfull[d], 1);
      mbar_init(&S.dempty[d], 4);                 // the 4 epilogue warps
      mbar_init(&S.ofull[d], 4);                  // the 4 outlier warps
      mbar_init(&S.oempty[d], 4);
    }
    mbar_init(S.mtail, 1);
    *S.abort_flag = 0;
    fence_mbar_init();
  }
  if (a.entries) {
    const int64_t ncache = min((int64_t)tc::kSegCache, u1 - u0);
    for (int64_t i = threadIdx.x; i <= ncache; i += blockDim.x) S.seg[i] = __ldg(a.seg_ptr + u0 + i);
  }
  if (warp == 1) {
    tmem_alloc(S.tmem_slot, tc::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *S.tmem_slot;
  // every CTA of the grid is resident (one per SM): the next kernel in the stream may launch;
  // its CTAs start as these exit (the shared-memory footprint keeps them from sharing an SM)
  if (threadIdx.x == 0) grid_launch_dependents();

  if (warp == 0) {
    tc_producer(S, a, M, u0, u1);
  } else if (warp == 1) {
    if (elect_one_sync()) tc_mma(S, a, u0, u1, tmem);
    __syncwarp();
  } else if (warp >= tc::kEpiWarp0 && warp < tc::kDqWarp0) {
    tc_epilogue(S, a, u0, u1, tmem);
  } else if (warp >= tc::kDqWarp0 && warp < tc::kOutWarp0) {
    tc_dequant(S, a, u0, u1, tmem);
  } else if (warp >= tc::kOutWarp0 && a.entries) {
    tc_outliers(S, a, u0, u1);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, tc::kTmemCols);
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
// host: tensor maps
// Activations X[m][k] (bf16, leading dim ldx) as a 2-D tensor (k, token) copied in boxes of
// 64 k x m tokens with 128-byte swizzle: each box lands as the MMA's K-major B operand for
// 4 blocks (token rows 8 and up in the second 1024-byte atom); columns >= k_in are zero-filled.
static int encode_x(CUtensorMap* m, const void* x, int64_t tokens, int64_t k_in, int64_t ldx) {
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

// Host launcher (called by fbfp_gemv when the shape qualifies). Returns FBFP_OK or an error.
int launch_gemv_tc(const TcArgs& a, cudaStream_t st) {
  int dev = 0;
  FBFP_CUDA_TRY(cudaGetDevice(&dev));
  static bool attr_set[64] = {false};
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    FBFP_CUDA_TRY(cudaFuncSetAttribute(gemv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)tc::kSmemBytes));
    attr_set[dev] = true;
  }
  TcMaps M;
  int rc;
  const uint64_t kb = (uint64_t)a.kb_row, np = (uint64_t)a.npad;
  if ((rc = encode_2d(&M.pay, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.pay, kb * 8, np, kb * 8, 128, 128,
                      CU_TENSOR_MAP_SWIZZLE_128B)) != FBFP_OK) return rc;
  if ((rc = encode_2d(&M.sgn, CU_TENSOR_MAP_DATA_TYPE_UINT16, a.sg, kb, np, kb * 2, kStageKb, 128,
                      CU_TENSOR_MAP_SWIZZLE_NONE)) != FBFP_OK) return rc;
  if ((rc = encode_2d(&M.exp, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.ex, kb, np, kb, kStageKb, 128,
                      CU_TENSOR_MAP_SWIZZLE_NONE)) != FBFP_OK) return rc;
  if ((rc = encode_x(&M.x, a.x, a.m, a.k_in, a.ldx)) != FBFP_OK) return rc;
  const int64_t nsm = sm_count(dev);
  const int64_t grid = nsm < a.total_units ? nsm : a.total_units;
  // programmatic stream serialisation: the launch may overlap the tail of the previous kernel
  // in the stream; the kernel waits for it (griddepcontrol.wait) before reading activations or
  // touching the workspace and y
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(tc::kThreads);
  cfg.dynamicSmemBytes = tc::kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FBFP_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemv_tc_kernel, a, M));
  FBFP_LAUNCH_CHECK("gemv_tc_kernel");
  return FBFP_OK;
}

bool gemv_tc_eligible(int64_t m, int64_t kb_row, int64_t k_in, int x_dtype, int64_t ldx,
                      const void* x, const void* pay, const void* sg, const void* ex) {
  return m >= 1 && m <= 16 && kb_row % kStageKb == 0 && x_dtype == FBFP_BF16 && k_in % 8 == 0 &&
         ldx % 8 == 0 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)pay & 15) == 0 &&
         ((uintptr_t)sg & 15) == 0 && ((uintptr_t)ex & 15) == 0 && encode_fn() != nullptr;
}

}  // namespace fbfp
