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
//   warps 2-3   idle (they complete the control warpgroup, which hands its registers to the
//               dequantisers with setmaxnreg);
//   warps 4-19  dequantisers (4 per tensor-memory lane quarter, one 4-block substage each):
//               one row per lane; each block becomes 8 bf16 pairs s*m*2^e built
//               exactly with bit operations (PRMT/LOP3 magic pair minus its offset, HSUB2) and
//               stored into a tensor-memory ring with tcgen05.st; they run the epilogue
//               (tcgen05.ld of the fp32 accumulator, 1/15 scale, red.add into the workspace;
//               the last CTA of a row group adds bias and writes y);
//               outliers ride along: the producer stages each stage's outlier entries and
//               per-row starts, and each dequantiser accumulates v * x in fp32 for the row's
//               outliers and its own 4 tokens (x read from the stage's activation tile), added
//               to the accumulator in the epilogue.
// Work: stream-K over units (128-row group, 16-block stage); each CTA takes a contiguous
// range. Every mbarrier wait is bounded: on timeout the CTA records an error code in the
// workspace and winds down (waiting, bounded, for its own copies) before freeing TMEM.
#include <cuda.h>

#include "common.cuh"
#include "sm100.cuh"
#include "tc_args.h"

namespace fbfp {
using namespace sm100;

namespace tc {
constexpr int kStages = 5;
constexpr int kASlots = 12;                     // tensor-memory A ring (4 blocks each)
constexpr int kPayOff = 0;                      // 128 rows x 128 B, 128-byte swizzle
constexpr int kSgnOff = 128 * 128;              // 128 rows x 32 B
constexpr int kExpOff = kSgnOff + 128 * 32;     // 128 rows x 16 B
constexpr int kXOff = kExpOff + 128 * 16;       // 16 blocks x (2 k-groups x 16 tokens x 16 B)
constexpr int kXPerKb = 512;
constexpr int kOutOff = kXOff + kStageKb * kXPerKb;           // stage's outlier entries
constexpr int kOutCap = 2048;                                 // entries staged per stage
constexpr int kRoffOff = kOutOff + kOutCap * 4;              // 136 uint16 row starts of the stage
constexpr int kRoffBytes = 272;
constexpr int kStageBytes = kRoffOff + 1024;                  // 39936 (multiple of 1024)
constexpr uint32_t kDenseTx = kOutOff;                        // bytes of the four tensor copies
constexpr int kSegCache = 1024;                               // segment pointers cached per CTA
constexpr int kDq = 16;                         // dequantiser warps (2..17), 4 per lane quarter
constexpr int kThreads = 32 * (4 + kDq);         // control warpgroup + dequantisers
// Register split: the block launches with kRegsLaunch per thread (5 warps per SM sub-partition
// fit its 16K registers only below ~102); the control warpgroup then drops to kRegsCtl and the
// dequantiser warpgroups rise to kRegsDq, drawing exactly on what the control warps released.
constexpr int kRegsLaunch = 96, kRegsCtl = 48, kRegsDq = 104;
static_assert(4 * 32 * kRegsCtl + kDq * 32 * kRegsDq <= kThreads * kRegsLaunch, "register split");
static_assert(kDq % 4 == 0, "dequantisers come in whole warpgroups");
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemD = 0;                  // 2 accumulators x 16 columns
constexpr uint32_t kTmemA = 32;                 // 12 slots x 32 columns (4 blocks x 8)
constexpr size_t kSoutOff = (size_t)kStages * kStageBytes;
constexpr size_t kSegOff = kSoutOff;
constexpr size_t kBarOff = kSegOff + (kSegCache + 8) * sizeof(int32_t);
constexpr int kNumBars = 2 * kStages + 2 * kASlots + 4 + 1;
constexpr size_t kSmemBytes = kBarOff + kNumBars * 8 + 16 + 1024;   // + alignment slack
}  // namespace tc

struct TcMaps {
  CUtensorMap pay, sgn, exp, x;
};

struct TcShared {
  uint8_t* stage;
  float* s_out;
  int32_t* seg;          // seg_ptr[u0 .. u0 + kSegCache]
  uint64_t *full, *empty, *afull, *aempty, *dfull, *dempty, *dqsync;
  uint32_t* tmem_slot;
  volatile int* abort_flag;
  int* last_flag;
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
  S.dqsync = S.dempty + 2;
  S.tmem_slot = reinterpret_cast<uint32_t*>(S.dqsync + 1);
  S.abort_flag = reinterpret_cast<volatile int*>(S.tmem_slot + 1);
  S.last_flag = reinterpret_cast<int*>(S.tmem_slot + 2);
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

// Barrier among the dequantiser warps (lane 0 of each arrives), bounded.
__device__ __forceinline__ bool dq_sync(const TcShared& S, const TcArgs& a, uint32_t& uses) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(S.dqsync);
  const bool ok = tc_wait(S, a, S.dqsync, uses & 1, 9);
  ++uses;
  __syncwarp();
  return ok;
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
// producer: four tensor copies per stage (payload, signs, exponents, activations)
__device__ void tc_producer(const TcShared& S, const TcArgs& a, const TcMaps& M, int64_t u0, int64_t u1) {
  int64_t i = 0;
  if (elect_one_sync()) {
    prefetch_tmap(&M.pay); prefetch_tmap(&M.sgn); prefetch_tmap(&M.exp); prefetch_tmap(&M.x);
    for (int64_t u = u0; u < u1; ++u, ++i) {
      const int s = (int)(i % tc::kStages);
      const uint32_t use = (uint32_t)(i / tc::kStages);
      if (!tc_wait(S, a, &S.empty[s], (use & 1) ^ 1, 1)) break;
      const int rg = (int)(u / a.n_stages), st = (int)(u % a.n_stages);
      uint8_t* sb = S.stage + (size_t)s * tc::kStageBytes;
      const OutRange orr = out_range(S, a, u0, i);
      mbar_arrive_expect_tx(&S.full[s], tc::kDenseTx + (uint32_t)orr.n * 4 + (a.entries ? tc::kRoffBytes : 0));
      tma_2d_g2s(sb + tc::kPayOff, &M.pay, st * 128, rg * 128, &S.full[s]);
      tma_2d_g2s(sb + tc::kSgnOff, &M.sgn, st * kStageKb, rg * 128, &S.full[s]);
      tma_2d_g2s(sb + tc::kExpOff, &M.exp, st * kStageKb, rg * 128, &S.full[s]);
      tma_3d_g2s(sb + tc::kXOff, &M.x, 0, 0, st * 2 * kStageKb, &S.full[s]);
      if (orr.n) bulk_g2s(sb + tc::kOutOff, a.entries + orr.lo4, (uint32_t)orr.n * 4, &S.full[s]);
      if (a.entries) bulk_g2s(sb + tc::kRoffOff, roff_block(a, u), tc::kRoffBytes, &S.full[s]);
    }
    // wind down: every stage issued so far must have landed before the CTA may exit
    for (int64_t j = i > tc::kStages ? i - tc::kStages : 0; j < i; ++j)
      mbar_wait(&S.full[j % tc::kStages], (uint32_t)(j / tc::kStages) & 1, 1u << 20);
  }
  __syncwarp();
}

// ---------------------------------------------------------------------------------------
__device__ void tc_mma(const TcShared& S, const TcArgs& a, int64_t u0, int64_t u1, uint32_t tmem) {
  constexpr uint32_t IDESC = idesc_bf16_f32(128, 16, false);
  // B tile of one block: [k-group 2][16 tokens][8 bf16]: LBO 256 B (K), SBO 128 B (N); the tiles of
  // consecutive blocks are 512 B apart, i.e. +32 in the descriptor's address field
  const uint64_t desc0 = smem_desc_noswizzle(smem_u32(S.stage + tc::kXOff), 256, 128);
  constexpr uint64_t kStageDesc = (uint64_t)(tc::kStageBytes >> 4);
  constexpr uint64_t kKbDesc = (uint64_t)(tc::kXPerKb >> 4);
  int64_t i = 0, jsub = 0, seg = 0;
  for (int64_t u = u0; u < u1; ++seg) {
    const int64_t rg = u / a.n_stages;
    const int64_t seg_end = min(u1, (rg + 1) * a.n_stages);
    const int d = (int)(seg & 1);
    if (!tc_wait(S, a, &S.dempty[d], (uint32_t)((seg >> 1) & 1) ^ 1, 2)) return;
    tc_fence_after();
    const uint32_t tD = tmem + tc::kTmemD + d * 16;
    uint32_t acc = 0;
    for (; u < seg_end; ++u, ++i) {
      const int s = (int)(i % tc::kStages);
      const uint64_t dstage = desc0 + (uint64_t)s * kStageDesc;
      for (int sub = 0; sub < 4; ++sub, ++jsub) {
        const int slot = (int)(jsub % tc::kASlots);
        if (!tc_wait(S, a, &S.afull[slot], (uint32_t)(jsub / tc::kASlots) & 1, 3)) return;
        tc_fence_after();
        const uint32_t tA = tmem + tc::kTmemA + slot * 32;
        const uint64_t dsub = dstage + (uint64_t)(sub * 4) * kKbDesc;
        mma_ts(tD, tA + 0, dsub + 0 * kKbDesc, IDESC, acc);
        mma_ts(tD, tA + 8, dsub + 1 * kKbDesc, IDESC, 1);
        mma_ts(tD, tA + 16, dsub + 2 * kKbDesc, IDESC, 1);
        mma_ts(tD, tA + 24, dsub + 3 * kKbDesc, IDESC, 1);
        acc = 1;
        mma_commit(&S.aempty[slot]);
      }
      mma_commit(&S.empty[s]);
    }
    mma_commit(&S.dfull[d]);
  }
}

// ---------------------------------------------------------------------------------------
// One block -> 8 bf16 pairs of natural elements (2j, 2j+1), each element exactly s*m*2^e:
// v = +-(128 + m) * 2^e (sign bit 15/31, exponent field e + 134, nibble in bits 0-3/16-19) and
// c = +-128 * 2^e are built with bit operations; v - c is exact in bf16.
__device__ __forceinline__ void dq_block(uint32_t w0, uint32_t w1, uint32_t s16, uint32_t eb,
                                         uint32_t* out) {
  const uint32_t SM = 0x80008000u, NM = 0x000F000Fu;
  const uint32_t y = s16 | (s16 << 15);          // sign bit b lands on 15 and 31 after << (15 - b)
  const uint32_t K = eb * 0x00800080u;
  const uint32_t t0 = w0 >> 4, t1 = w1 >> 4;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t sel = (uint32_t)j | ((uint32_t)(4 + j) << 8);   // byte j of w, byte j of w>>4
    const uint32_t c0 = ((y << (15 - 2 * j)) & SM) | K;
    const uint32_t c1 = ((y << (7 - 2 * j)) & SM) | K;
    const uint32_t v0 = (__byte_perm(w0, t0, sel) & NM) | c0;
    const uint32_t v1 = (__byte_perm(w1, t1, sel) & NM) | c1;
    __nv_bfloat162 r0 = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&v0),
                                *reinterpret_cast<const __nv_bfloat162*>(&c0));
    __nv_bfloat162 r1 = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&v1),
                                *reinterpret_cast<const __nv_bfloat162*>(&c1));
    out[j] = *reinterpret_cast<uint32_t*>(&r0);
    out[4 + j] = *reinterpret_cast<uint32_t*>(&r1);
  }
}

// Segment-end synchronisation and epilogue shared by dequantisers (and, for the barrier
// points, the outlier warps).
__device__ void tc_dequant(const TcShared& S, const TcArgs& a, int64_t u0, int64_t u1, uint32_t tmem) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wi = warp - 4;                 // 0..kDq-1
  const int q4 = warp & 3;                 // tensor-memory lane quarter
  const int par = wi >> 2;                 // which of the 4 substages of a stage (and token quarter)
  const int lr = q4 * 32 + lane;           // row within the group
  const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
  const int sw = lr & 7;                   // 128-byte swizzle phase of this row
  const int m = a.m;
  uint32_t sync_uses = 0;
  int64_t i = 0, seg = 0;
  for (int64_t u = u0; u < u1; ++seg) {
    const int64_t rg = u / a.n_stages;
    const int64_t seg_begin = u, seg_end = min(u1, (rg + 1) * a.n_stages);
    const int64_t row = rg * 128 + lr;
    const bool rvalid = row < a.npad;
    const bool do_out = a.entries && rvalid && par * 4 < m;
    float oacc[4] = {0.f, 0.f, 0.f, 0.f};
    for (; u < seg_end; ++u, ++i) {
      const int s = (int)(i % tc::kStages);
      if (!tc_wait(S, a, &S.full[s], (uint32_t)(i / tc::kStages) & 1, 4)) return;
      const uint8_t* sb = S.stage + (size_t)s * tc::kStageBytes;
      {
        const int sub = par;
        const int64_t j = 4 * i + sub;
        const int slot = (int)(j % tc::kASlots);
        const uint8_t* prow = sb + tc::kPayOff + lr * 128;
        const uint4 P0 = *reinterpret_cast<const uint4*>(prow + (((2 * sub) ^ sw) << 4));
        const uint4 P1 = *reinterpret_cast<const uint4*>(prow + (((2 * sub + 1) ^ sw) << 4));
        const uint2 SG = *reinterpret_cast<const uint2*>(sb + tc::kSgnOff + lr * 32 + sub * 8);
        const uint32_t EX = *reinterpret_cast<const uint32_t*>(sb + tc::kExpOff + lr * 16 + sub * 4);
        const uint32_t E = (EX ^ 0x80808080u) + 0x06060606u;     // e + 134 per byte
        uint32_t w[32];
        dq_block(P0.x, P0.y, SG.x & 0xFFFFu, E & 0xFFu, w + 0);
        dq_block(P0.z, P0.w, SG.x >> 16, (E >> 8) & 0xFFu, w + 8);
        dq_block(P1.x, P1.y, SG.y & 0xFFFFu, (E >> 16) & 0xFFu, w + 16);
        dq_block(P1.z, P1.w, SG.y >> 16, E >> 24, w + 24);
        if (!rvalid) {                                          // rows past npad (TMA zero fill)
#pragma unroll
          for (int r = 0; r < 32; ++r) w[r] = 0u;
        }
        if (!tc_wait(S, a, &S.aempty[slot], ((uint32_t)(j / tc::kASlots) & 1) ^ 1, 5)) return;
        tc_fence_after();
        tmem_st_32x32b_x32(tmem + tc::kTmemA + slot * 32 + lane_base, w);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.afull[slot]);
      }
      if (do_out) {
        // outliers of this row in this stage (their dense slots are +0): acc += v * x for the
        // warp's 4 tokens, x read from the stage's activation tile [k-group][16 tokens][8]
        const OutRange orr = out_range(S, a, u0, i);
        const uint16_t* ro = reinterpret_cast<const uint16_t*>(sb + tc::kRoffOff);
        const uint32_t* es = reinterpret_cast<const uint32_t*>(sb + tc::kOutOff);
        const uint8_t* xs = sb + tc::kXOff + par * 4 * 16;
        const int e_end = ro[lr + 1];
        for (int t = ro[lr]; t < e_end; ++t) {
          const int o = orr.lo + t - orr.lo4;
          const uint32_t e = o < orr.n ? es[o] : __ldg(a.entries + orr.lo + t);
          const uint32_t c = (e >> 16) & 0xFFu;
          const float v = __half2float(__ushort_as_half((unsigned short)(e & 0xFFFFu)));
          const uint8_t* xp = xs + (c >> 4) * tc::kXPerKb + ((c >> 3) & 1) * 256 + (c & 7) * 2;
#pragma unroll
          for (int tt = 0; tt < 4; ++tt)
            oacc[tt] = fmaf(v, __uint_as_float((uint32_t)*reinterpret_cast<const uint16_t*>(xp + tt * 16) << 16),
                            oacc[tt]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.empty[s]);
    }

    // ---- segment epilogue ----
    const int d = (int)(seg & 1);
    if (!tc_wait(S, a, &S.dfull[d], (uint32_t)(seg >> 1) & 1, 6)) return;
    tc_fence_after();
    float dv[4];
    tmem_ld_32x32b_x4(tmem + tc::kTmemD + d * 16 + par * 4 + lane_base, dv);
    tmem_wait_ld();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&S.dempty[d]);
    const float inv15 = 1.0f / 15.0f;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int tok = par * 4 + t;
      if (tok < m && rvalid) {
        asm volatile("red.global.add.f32 [%0], %1;\n" ::"l"(a.ws + (int64_t)tok * a.npad + row),
                     "f"(fmaf(dv[t], inv15, oacc[t])) : "memory");
      }
    }
    __threadfence();
    if (!dq_sync(S, a, sync_uses)) return;
    if (wi == 0 && lane == 0) {
      __threadfence();
      const int units = (int)(seg_end - seg_begin);
      const int old = atomicAdd(a.counters + rg, units);
      *S.last_flag = (old + units == a.n_stages);
    }
    if (!dq_sync(S, a, sync_uses)) return;
    if (*S.last_flag) {
      __threadfence();
      for (int p = wi * 32 + lane; p < 128 * m; p += 32 * tc::kDq) {
        const int tok = p >> 7, r = p & 127;
        const int64_t rw = rg * 128 + r;
        if (rw >= a.npad) continue;
        float* wp = a.ws + (int64_t)tok * a.npad + rw;
        float val = __ldcg(wp);
        __stcg(wp, 0.f);
        if (rw < a.n_out) {
          if (a.bias) val += load_as_float(a.bias, a.bias_dtype, rw);
          store_from_float(a.y, a.y_dtype, (int64_t)tok * a.ldy + rw, val);
        }
      }
      if (wi == 0 && lane == 0) a.counters[rg] = 0;
    }
    if (!dq_sync(S, a, sync_uses)) return;
  }
}

__global__ void __maxnreg__(tc::kRegsLaunch)
gemv_tc_kernel(const TcArgs a, const __grid_constant__ TcMaps M) {
  extern __shared__ uint8_t smem_raw[];
  const TcShared S = tc_shared(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int64_t U = a.total_units;
  const int64_t u0 = (int64_t)blockIdx.x * U / gridDim.x;
  const int64_t u1 = (int64_t)(blockIdx.x + 1) * U / gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < tc::kStages; ++s) { mbar_init(&S.full[s], 1); mbar_init(&S.empty[s], tc::kDq + 1); }
    for (int j = 0; j < tc::kASlots; ++j) { mbar_init(&S.afull[j], 4); mbar_init(&S.aempty[j], 1); }
    for (int d = 0; d < 2; ++d) { mbar_init(&S.dfull[d], 1); mbar_init(&S.dempty[d], tc::kDq); }
    mbar_init(S.dqsync, tc::kDq);
    *S.abort_flag = 0;
    *S.last_flag = 0;
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

  if (warp < 4) {
    regs_release<tc::kRegsCtl>();
    if (warp == 0) {
      tc_producer(S, a, M, u0, u1);
    } else if (warp == 1) {
      if (elect_one_sync()) tc_mma(S, a, u0, u1, tmem);
      __syncwarp();
    }
  } else {
    regs_acquire<tc::kRegsDq>();
    tc_dequant(S, a, u0, u1, tmem);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, tc::kTmemCols);
  }
}

static int sm_count(int dev) {
  static int cached[64] = {0};
  if (dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

// ---------------------------------------------------------------------------------------
// host: tensor maps
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

static int encode_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner,
                     uint64_t rows, uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows,
                     CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(FBFP_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(FBFP_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return FBFP_OK;
}

// Activations X[m][k] (bf16, leading dim ldx) as a 3-D tensor (8 elements, token, k-group)
// so that one copy lands a stage directly in the MMA's K-major core-matrix layout
// [k-group][16 tokens][8 elements]; tokens >= m and columns >= k_in are zero-filled.
static int encode_x(CUtensorMap* m, const void* x, int64_t tokens, int64_t k_in, int64_t ldx) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(FBFP_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  const cuuint64_t dims[3] = {8, (cuuint64_t)tokens, (cuuint64_t)(k_in / 8)};
  const cuuint64_t strides[2] = {(cuuint64_t)ldx * 2, 16};
  const cuuint32_t box[3] = {8, 16, 2 * kStageKb};
  const cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(x), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
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
  gemv_tc_kernel<<<(unsigned)grid, tc::kThreads, tc::kSmemBytes, st>>>(a, M);
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
