// rtd_gemm_ts.cu -- tensor-core GEMM for skinny token counts (batched decode, speculative
// verify): the decoded weights are written to TENSOR memory and tcgen05.mma reads its A
// operand from there, so decoded weights never pass through shared memory.
//
//   y[M, N] = x[M, K] . W^T (+ bias)      W in Q4_K / Q6_K / Q8_0 / FP8-E4M3 groups
//
// One CTA computes 128 weight rows (eight 16-row tiles: the UMMA M) x TN tokens (16, 32 or
// 64: the UMMA N) with the f32 accumulator in tensor memory, one weight GROUP (GK = 256 k
// for the K-quants, 128 for Q8_0 / FP8) per pipeline step:
//   - warp 2 (one lane) bulk-copies the group of each of the eight tiles into a
//     shared-memory slot (up to eight slots ahead); warp 0 (one lane) bulk-copies the
//     group's activation tile (staged once per call by gemm_prep_ts_kernel);
//   - sixteen decode warps in two sets take alternate groups.  In a set, the warp of
//     tensor-memory lane quarter q and tile 2q + p decodes its tile's group: thread
//     4g + t holds exactly the bytes the group layout gives lane 4g + t (whole
//     sub-blocks of rows g and g + 8, conflict-free 16-byte shared loads), turns them
//     into f16 pairs (codes exact in f16 through an exponent-bias constant, the
//     reference's per-sub-block factors rounded once to f16, one f16 FMA per pair) and
//     stores them with tcgen05.st.16x256b, whose thread pattern is that same lane
//     ownership: registers of thread 4g + t land in lanes g and g + 8, columns 2t and
//     2t + 1 of every 8-column repetition.  The k order inside a group is therefore the
//     decoder's, and the activations are staged in that order (perm_* below);
//   - one lane of warp 1 issues the group's tcgen05.mma (A from tensor memory, B from the
//     128-byte swizzled activation tile) into the accumulator and commits them to the
//     group's release barriers (tensor-memory slot and activation slot);
//   - after the last group warps 4..7 read the accumulator (tcgen05.ld, one lane quarter
//     each) and write y with the per-token activation scale, the FP8 row scale and the
//     bias, or f32 partials when K is split over CTAs.
// FP8 weights with E4M3 activations (W8A8) skip the decode: the E4M3 codes go to tensor
// memory as they are and tcgen05.mma.kind::f8f6f4 multiplies them with the E4M3 codes
// of the activations.
// Every wait is bounded by %globaltimer; a timeout records kDevWaitTimeout and the CTA
// stops issuing work, drains what it issued and returns.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "rtd_common.cuh"
#include "rtd_kernels.h"
#include "rtd_tcgen05.cuh"

namespace rtd {
namespace {

constexpr int kTsThreads = 640;     // 20 warps: 0 activations, 1 MMA, 2 weights, 3 TMEM owner, 4..19 decode
constexpr int kTsSmem = 227 * 1024;
constexpr int kTsCols = 512;        // the whole tensor memory of the SM (one CTA per SM)
constexpr int kTsMaxSlots = 8;
constexpr int kPrepThreads = 256;

// Per-format constants: GK k per group, GB bytes per 16-row group, ACOLS tensor-memory
// columns of one group's A (128 rows), NMMA instructions per group (K = 16 f16 or K = 32
// E4M3 each, 8 columns apiece), BTOK bytes of staged activations per token and group.
template <int FMT>
struct TsFmt;
template <>
struct TsFmt<FMT_Q4K> {
  static constexpr int GK = 256, GB = 2304, ACOLS = 128, NMMA = 16, BTOK = 512;
};
template <>
struct TsFmt<FMT_Q6K> {
  static constexpr int GK = 256, GB = 3360, ACOLS = 128, NMMA = 16, BTOK = 512;
};
template <>
struct TsFmt<FMT_Q80> {
  static constexpr int GK = 128, GB = 2176, ACOLS = 64, NMMA = 8, BTOK = 256;
};
template <>
struct TsFmt<FMT_FP8> {
  static constexpr int GK = 128, GB = 2048, ACOLS = 64, NMMA = 8, BTOK = 256;
};
template <>
struct TsFmt<FMT_TS_F8X> {
  static constexpr int GK = 128, GB = 2048, ACOLS = 32, NMMA = 4, BTOK = 128;
};

// Shared-memory and tensor-memory plan: SB activation slots (TN * BTOK bytes), SR
// weight slots (8 * GB bytes), SA tensor-memory A slots after the accumulator.
template <int FMT, int TN>
struct TsPlan {
  using F = TsFmt<FMT>;
  static constexpr int kB = TN * F::BTOK;
  static constexpr int kRaw = 8 * F::GB;
  // The activation ring refills a slot only after the group that used it has been
  // multiplied, so its depth (not its bytes) bounds the groups a CTA finishes per L2
  // round trip: up to 96 KB of slots, at least three, at most eight.
  static constexpr int kSbFit = (96 * 1024) / kB;
  static constexpr int SB = kSbFit < 3 ? 3 : (kSbFit > kTsMaxSlots ? kTsMaxSlots : kSbFit);
  static constexpr int kFixed = 1024 + 512 + TN * 4;  // alignment slack, barriers + misc, token scales
  static constexpr int kFitR = (kTsSmem - kFixed - SB * kB) / kRaw;
  static constexpr int SR = kFitR < kTsMaxSlots ? kFitR : kTsMaxSlots;
  static constexpr int A0 = TN < 32 ? 32 : TN;        // first A column (the accumulator holds 0 .. TN)
  static constexpr int kFitA = (kTsCols - A0) / F::ACOLS;
  static constexpr int SA = kFitA < 6 ? kFitA : 6;
  static constexpr int offB = 0;
  static constexpr int offRaw = SB * kB;
  static constexpr int offBar = offRaw + SR * kRaw;
  static constexpr int nBars = 2 * SR + 2 * SB + 2 * SA + 1;
  static constexpr int offMisc = offBar + nBars * 8;
  static constexpr int offScale = offMisc + 16;
  static constexpr int bytes = offScale + TN * 4 + 1024;
  static_assert(SR >= 2 && SA >= 2, "too few pipeline slots");
  static_assert(bytes <= kTsSmem, "shared-memory plan exceeds the CTA's share");
  // one CTA per SM (it allocates every tensor-memory column): launch with more than half
  // of the shared memory even where the plan needs less
  static constexpr int launch_bytes = bytes > kTsSmem / 2 + 1024 ? bytes : kTsSmem / 2 + 1024;
  static_assert(offRaw % 1024 == 0, "activation slots keep the 1024-byte swizzle alignment");
};

// ---------------------------------------------------------------- k order of a group
// Position p of a group's staged activations (the order in which the decode threads store
// their pairs into tensor memory) -> element k of the group.  For the f16 formats p = 16 i +
// kk is element kk of MMA slice i, i.e. column 8 i + kk / 2, half kk % 2, written by thread
// t = kk / 4 of the 16x256b pattern as its pair j = 2 i + (kk / 2) % 2.
__host__ __device__ __forceinline__ int perm_q4k(int p) {
  const int i = p >> 4, kk = p & 15, t = kk >> 2, e = (kk >> 1) & 1, h = kk & 1;
  const int j = 2 * i + e, pp = j >> 4, w = (j >> 2) & 3, ty = j & 3;
  // pair (pp, w, ty): bytes (0, 2) [ty even] or (1, 3) [ty odd] of word w of the
  // 16-byte run pp; low nibbles [ty < 2] are sub-block 2t, high nibbles sub-block 2t + 1
  const int sb = 2 * t + (ty >> 1), el = 16 * pp + 4 * w + (ty & 1) + 2 * h;
  return 32 * sb + el;
}
__host__ __device__ __forceinline__ int perm_q6k(int p) {
  const int i = p >> 4, kk = p & 15, t = kk >> 2, e = (kk >> 1) & 1, h = kk & 1;
  const int j = 2 * i + e, hh = j >> 4, par = (j >> 3) & 1, jj = j & 7;
  // pair jj (elements 2 jj, 2 jj + 1) of sub-block 8 hh + 2 t + par
  return 16 * (8 * hh + 2 * t + par) + 2 * jj + h;
}
__host__ __device__ __forceinline__ int perm_q80(int p) {  // Q8_0 and FP8 (W8A16)
  const int i = p >> 4, kk = p & 15, t = kk >> 2, e = (kk >> 1) & 1, h = kk & 1;
  return 32 * t + 2 * (2 * i + e) + h;  // element 2 j + h of the lane's 32-element block t
}
__host__ __device__ __forceinline__ int perm_f8x(int p) {  // E4M3 A: four codes a column, K = 32 a slice
  const int i = p >> 5, kk = p & 31;
  return 32 * (kk >> 3) + 8 * i + (kk & 7);
}

// ---------------------------------------------------------------- decoders
// grp: shared address of this tile's group; taddr: tensor-memory address of the tile's
// 16 lanes at the group's first A column.  Thread 4g + t (= lane) owns rows g and g + 8.
__device__ __forceinline__ void q4k_factors(uint4 h, int t, uint32_t& dl, uint32_t& nl, uint32_t& dh,
                                            uint32_t& nh) {
  const float d = hbits(h.x & 0xFFFFu), dmin = hbits(h.x >> 16);
  uint32_t sc0, m0, sc1, m1;
  scale_min_words(2 * t, h.y, h.z, h.w, sc0, m0);
  scale_min_words(2 * t + 1, h.y, h.z, h.w, sc1, m1);
  dl = h2_bits(h2_const(d * (float)sc0));
  nl = h2_bits(h2_const(-(dmin * (float)m0)));
  dh = h2_bits(h2_const(d * (float)sc1));
  nh = h2_bits(h2_const(-(dmin * (float)m1)));
}

// Low nibbles at bits 0-3 / 16-19: 0x6400 | q is 1024 + q; high nibbles at bits 4-7 /
// 20-23: 0x5400 | q << 4 is 64 + q.  The subtraction is exact, then one FMA per pair.
__device__ __forceinline__ uint32_t q4_lo(uint32_t x, uint32_t d, uint32_t n) {
  const __half2 v = __hsub2(bits_h2(lop_and_or(x, 0x000F000Fu, 0x64006400u)), __float2half2_rn(1024.0f));
  return h2_bits(__hfma2(bits_h2(d), v, bits_h2(n)));
}
__device__ __forceinline__ uint32_t q4_hi(uint32_t x, uint32_t d, uint32_t n) {
  const __half2 v = __hsub2(bits_h2(lop_and_or(x, 0x00F000F0u, 0x54005400u)), __float2half2_rn(64.0f));
  return h2_bits(__hfma2(bits_h2(d), v, bits_h2(n)));
}

__device__ __forceinline__ void ts_decode_q4k(uint32_t grp, uint32_t taddr, int lane) {
  const int g = lane >> 2, t = lane & 3;
  uint32_t dl[2], nl[2], dh[2], nh[2];
  q4k_factors(lds128(grp + 16 * g), t, dl[0], nl[0], dh[0], nh[0]);
  q4k_factors(lds128(grp + 16 * (g + 8)), t, dl[1], nl[1], dh[1], nh[1]);
#pragma unroll
  for (int pp = 0; pp < 2; ++pp) {
    // 16-byte runs of the lane's chunk t: run pp of row g (pass pp), of row g + 8 (pass 2 + pp)
    const uint4 u[2] = {lds128(grp + 256 + pp * 512 + lane * 16), lds128(grp + 256 + (2 + pp) * 512 + lane * 16)};
    uint32_t v[32];
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const uint32_t x = (&u[hr].x)[w], x8 = x >> 8;
        v[4 * (2 * w) + 0 + 2 * hr] = q4_lo(x, dl[hr], nl[hr]);       // bytes 0, 2: sub-block 2t
        v[4 * (2 * w) + 1 + 2 * hr] = q4_lo(x8, dl[hr], nl[hr]);      // bytes 1, 3
        v[4 * (2 * w + 1) + 0 + 2 * hr] = q4_hi(x, dh[hr], nh[hr]);   // sub-block 2t + 1
        v[4 * (2 * w + 1) + 1 + 2 * hr] = q4_hi(x8, dh[hr], nh[hr]);
      }
    }
    tmem_st16x256_x8(taddr + 64u * pp, v);
  }
}

__device__ __forceinline__ void ts_decode_q6k(uint32_t grp, uint32_t taddr, int lane) {
  const int g = lane >> 2;
  const float d[2] = {hbits(lds16(grp + 4 * g)), hbits(lds16(grp + 4 * g + 2))};
  const uint32_t scw[2] = {lds32(grp + 32 + lane * 8), lds32(grp + 32 + lane * 8 + 4)};
  const __half2 k1056 = __float2half2_rn(1056.0f);  // 1024 + 32
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    uint32_t wd[12];
#pragma unroll
    for (int pz = 0; pz < 3; ++pz) {
      const uint4 q = lds128(grp + 288 + (3 * hh + pz) * 512 + lane * 16);
      wd[4 * pz] = q.x;
      wd[4 * pz + 1] = q.y;
      wd[4 * pz + 2] = q.z;
      wd[4 * pz + 3] = q.w;
    }
    uint32_t v[32];
#pragma unroll
    for (int tr = 0; tr < 4; ++tr) {  // (row g, 8hh+2t), (row g+8, ..), (row g, 8hh+2t+1), (row g+8, ..)
      const int hr = tr & 1, par = tr >> 1;
      const uint32_t X = wd[3 * tr], Y = wd[3 * tr + 1], Z = wd[3 * tr + 2];
      const __half2 ds = h2_const(d[hr] * (float)(int)(int8_t)(uint8_t)(scw[hr] >> (8 * (2 * hh + par))));
      const uint32_t c[8] = {X & 0x003F003Fu,
                             (X >> 6) & 0x003F003Fu,
                             Y & 0x003F003Fu,
                             (Y >> 6) & 0x003F003Fu,
                             Z & 0x003F003Fu,
                             (Z >> 6) & 0x003F003Fu,
                             ((X >> 12) & 0x000F000Fu) | ((Z >> 8) & 0x00300030u),
                             ((Y >> 12) & 0x000F000Fu) | ((Z >> 10) & 0x00300030u)};
#pragma unroll
      for (int jj = 0; jj < 8; ++jj)
        v[4 * (4 * par + (jj >> 1)) + (jj & 1) + 2 * hr] =
            h2_bits(__hmul2(ds, __hsub2(bits_h2(c[jj] | 0x64006400u), k1056)));
    }
    tmem_st16x256_x8(taddr + 64u * hh, v);
  }
}

template <bool Q8>
__device__ __forceinline__ void ts_decode_8bit(uint32_t grp, uint32_t taddr, int lane) {
  uint32_t dq[2] = {0u, 0u};
  if constexpr (Q8) {
    dq[0] = lds16(grp + 4 * lane) * 0x10001u;
    dq[1] = lds16(grp + 4 * lane + 2) * 0x10001u;
  }
  const __half2 k1152 = __float2half2_rn(1152.0f);  // 1024 + 128
  uint32_t v[32];
#pragma unroll
  for (int p = 0; p < 4; ++p) {  // pass p: row g + 8 (p >> 1), elements 16 (p & 1) ..
    const int hr = p >> 1, pp = p & 1;
    const uint4 q = lds128(grp + (Q8 ? 128 : 0) + p * 512 + lane * 16);
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const uint32_t x = (&q.x)[w];
#pragma unroll
      for (int s = 0; s < 2; ++s) {  // bytes (0, 1) / (2, 3): elements 4w + 2s, 4w + 2s + 1
        uint32_t o;
        if constexpr (Q8) {
          const uint32_t p2 = prmt(x ^ 0x80808080u, 0x64u, s ? 0x4342u : 0x4140u);
          o = h2_bits(__hmul2(bits_h2(dq[hr]), __hsub2(bits_h2(p2), k1152)));
        } else {
          o = e4m3x2_to_f16x2((uint16_t)(s ? (x >> 16) : (x & 0xFFFFu)));
        }
        v[4 * (4 * pp + w) + s + 2 * hr] = o;
      }
    }
  }
  tmem_st16x256_x8(taddr, v);
}

// W8A8: the E4M3 codes themselves, four to a column.
__device__ __forceinline__ void ts_copy_f8x(uint32_t grp, uint32_t taddr, int lane) {
  uint4 q[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) q[p] = lds128(grp + p * 512 + lane * 16);
  uint32_t v[16];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int e = 0; e < 2; ++e)
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) v[4 * r + e + 2 * hr] = (&q[2 * hr + (r >> 1)].x)[2 * (r & 1) + e];
  tmem_st16x256_x4(taddr, v);
}

template <int FMT>
__device__ __forceinline__ void ts_decode(uint32_t grp, uint32_t taddr, int lane) {
  if constexpr (FMT == FMT_Q4K)
    ts_decode_q4k(grp, taddr, lane);
  else if constexpr (FMT == FMT_Q6K)
    ts_decode_q6k(grp, taddr, lane);
  else if constexpr (FMT == FMT_Q80)
    ts_decode_8bit<true>(grp, taddr, lane);
  else if constexpr (FMT == FMT_FP8)
    ts_decode_8bit<false>(grp, taddr, lane);
  else
    ts_copy_f8x(grp, taddr, lane);
}

// ---------------------------------------------------------------- GEMM kernel
template <int FMT, int TN>
__global__ void __launch_bounds__(kTsThreads, 1) qgemm_ts_kernel(const TsGemm a) {
  using F = TsFmt<FMT>;
  using P = TsPlan<FMT, TN>;
  constexpr bool F8 = FMT == FMT_TS_F8X;
  constexpr int SR = P::SR, SB = P::SB, SA = P::SA;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + P::offBar);
  uint64_t* raw_full = bar;
  uint64_t* raw_empty = raw_full + SR;
  uint64_t* b_full = raw_empty + SR;
  uint64_t* b_empty = b_full + SB;
  uint64_t* a_full = b_empty + SB;
  uint64_t* a_empty = a_full + SA;
  uint64_t* acc_full = a_empty + SA;
  uint32_t* misc = reinterpret_cast<uint32_t*>(sm + P::offMisc);  // [0] tensor-memory base, [1] abort flag
  float* sscale = reinterpret_cast<float*>(sm + P::offScale);

  const int64_t tile0 = (int64_t)blockIdx.y * 8;  // first 16-row tile of this CTA
  const int64_t t0 = (int64_t)blockIdx.x * TN;    // first token
  const int g_lo = (int)(a.G * blockIdx.z / a.splits);
  const int g_hi = (int)(a.G * (blockIdx.z + 1) / a.splits);
  const int ng = g_hi - g_lo;

  if (warp == 3) {
    tmem_alloc(smem_u32(&misc[0]), kTsCols);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < SR; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], 8);  // the eight tile warps of the set that decoded it
    }
    for (int s = 0; s < SB; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty[s], 1);
    }
    for (int s = 0; s < SA; ++s) {
      mbar_init(&a_full[s], 8);
      mbar_init(&a_empty[s], 1);
    }
    mbar_init(acc_full, 1);
    misc[1] = 0;
    fence_mbar_init();
  }
  pdl_trigger();  // the reduce kernel (or the next call) may launch; it waits for this grid
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc[0];
  volatile uint32_t* abort_flag = &misc[1];

  auto wait = [&](uint64_t* b, uint32_t parity) -> bool {
    if (mbar_try_wait(b, parity)) return true;
    if (*abort_flag) return false;
    if (mbar_wait_ns(b, parity, kWaitBudgetNs, a.status)) return true;
    *abort_flag = 1;
    return false;
  };

  if (warp == 0) {
    // ---- activation tiles: one bulk copy per 128-byte row (64 f16 or 128 E4M3 k) of the group
    if (lane == 0) {
      pdl_wait();  // the staged activations are the prep kernel's output
      constexpr int kRows = F8 ? 1 : F::GK / 64;
      const uint8_t* xw = static_cast<const uint8_t*>(a.xw);
      int issued = 0;
      for (int gi = 0; gi < ng; ++gi) {
        const int sb = gi % SB;
        if (gi >= SB && !wait(&b_empty[sb], (uint32_t)((gi / SB - 1) & 1))) break;
        mbar_arrive_expect_tx(&b_full[sb], (uint32_t)P::kB);
        for (int r = 0; r < kRows; ++r) {
          const int64_t kb = (int64_t)(g_lo + gi) * kRows + r;
          bulk_g2s(sm + P::offB + sb * P::kB + r * TN * 128, xw + ((size_t)kb * (a.Mp / 8) + (size_t)(t0 / 8)) * 1024,
                   TN * 128, &b_full[sb]);
        }
        ++issued;
      }
      if (*abort_flag)  // no copy may still be landing when the CTA exits
        for (int gi = (issued > SB ? issued - SB : 0); gi < issued; ++gi)
          mbar_wait_ns(&b_full[gi % SB], (uint32_t)((gi / SB) & 1), kWaitBudgetNs, a.status);
    }
  } else if (warp == 2) {
    // ---- packed groups of the eight tiles
    if (lane == 0) {
      const int64_t ntile = (a.T - tile0 < 8) ? a.T - tile0 : 8;
      int issued = 0;
      for (int gi = 0; gi < ng; ++gi) {
        const int sr = gi % SR;
        if (gi >= SR && !wait(&raw_empty[sr], (uint32_t)((gi / SR - 1) & 1))) break;
        mbar_arrive_expect_tx(&raw_full[sr], (uint32_t)(ntile * F::GB));
        for (int64_t i = 0; i < ntile; ++i)
          bulk_g2s(sm + P::offRaw + sr * P::kRaw + i * F::GB, a.w + ((tile0 + i) * a.G + g_lo + gi) * F::GB, F::GB,
                   &raw_full[sr]);
        ++issued;
      }
      if (*abort_flag)
        for (int gi = (issued > SR ? issued - SR : 0); gi < issued; ++gi)
          mbar_wait_ns(&raw_full[gi % SR], (uint32_t)((gi / SR) & 1), kWaitBudgetNs, a.status);
    }
  } else if (warp == 1) {
    // ---- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(TN);  // kind::f8f6f4 reads the same fields as E4M3 x E4M3
      const uint64_t db0 = kmajor_desc(smem_u32(sm + P::offB));
      for (int gi = 0; gi < ng; ++gi) {
        const int sa = gi % SA, sb = gi % SB;
        if (!wait(&a_full[sa], (uint32_t)((gi / SA) & 1)) || !wait(&b_full[sb], (uint32_t)((gi / SB) & 1))) break;
        tc_fence_after();
        const uint32_t a_col = tmem + (uint32_t)(P::A0 + sa * F::ACOLS);
#pragma unroll
        for (int i = 0; i < F::NMMA; ++i) {
          // slice i: 8 tensor-memory columns; in the activation slot, 128-byte row i / 4 at byte 32 (i % 4)
          const uint64_t bd = db0 + (uint64_t)((sb * P::kB + (i >> 2) * TN * 128) >> 4) + 2 * (i & 3);
          const uint32_t acc = (gi > 0 || i > 0) ? 1u : 0u;
          if constexpr (F8)
            umma_f8_ts(tmem, a_col + 8u * i, bd, idesc, acc);
          else
            umma_f16_ts(tmem, a_col + 8u * i, bd, idesc, acc);
        }
        umma_commit(&a_empty[sa]);
        umma_commit(&b_empty[sb]);
      }
      umma_commit(acc_full);  // fires once every MMA issued has completed
    }
  } else if (warp >= 4) {
    // ---- decode warps: lane quarter q = warp % 4 (tensor-memory lanes 32q ..), tile 2q + p
    const int dw = warp - 4, q = warp & 3, p = (dw >> 2) & 1, set = dw >> 3;
    const int tile = 2 * q + p;
    const bool live = tile0 + tile < a.T;
    const uint32_t tlane = (uint32_t)(32 * q + 16 * p) << 16;
    for (int gi = set; gi < ng; gi += 2) {
      const int sr = gi % SR, sa = gi % SA;
      bool ok = wait(&raw_full[sr], (uint32_t)((gi / SR) & 1));
      if (ok && gi >= SA) ok = wait(&a_empty[sa], (uint32_t)((gi / SA - 1) & 1));
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      if (live)
        ts_decode<FMT>(smem_u32(sm + P::offRaw + sr * P::kRaw + tile * F::GB),
                       tmem + tlane + (uint32_t)(P::A0 + sa * F::ACOLS), lane);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&a_full[sa]);
        mbar_arrive(&raw_empty[sr]);
      }
    }
    if (warp < 8) {
      // ---- epilogue: warps 4..7, tensor-memory lanes 32q .. 32q + 31 = weight rows
      pdl_wait();  // the token scales are the prep kernel's output
      for (int i = tid - 128; i < TN; i += 128) sscale[i] = (t0 + i < a.M) ? a.tscale[t0 + i] : 0.0f;
      named_sync(1, 128);
      const bool ok = wait(acc_full, 0u);
      tc_fence_after();
      const int r = q * 32 + lane;
      const int64_t n = tile0 * 16 + r;
      float es = 1.0f, eb = 0.0f;
      if (n < a.N) {
        if (a.row_scale) es = a.row_scale[a.scale_len == 1 ? 0 : n];
        if (a.bias) eb = a.bias[n];
      }
#pragma unroll 1
      for (int c0 = 0; c0 < TN; c0 += 16) {
        float v[16];
        tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
        if (!ok || n >= a.N) continue;
        if (a.splits > 1) {  // partial sums of this k split; the reduce kernel finishes them
          float* pp = a.partial + ((size_t)blockIdx.z * a.Mp + (size_t)(t0 + c0)) * a.N + n;
#pragma unroll
          for (int j = 0; j < 16; ++j) pp[(size_t)j * a.N] = v[j];
          continue;
        }
        const int jn = (a.M - (t0 + c0)) < 16 ? (int)(a.M - (t0 + c0)) : 16;
        const int ysz = a.y_dtype == 0 ? 4 : 2;
        uint8_t* yp = static_cast<uint8_t*>(a.y) + ((t0 + c0) * a.ldy + n) * ysz;
        const int64_t ystep = a.ldy * ysz;
#pragma unroll
        for (int j = 0; j < 16; ++j, yp += ystep) {
          if (j >= jn) break;
          const float val = v[j] * sscale[c0 + j] * es + eb;
          if (a.y_dtype == 0)
            *reinterpret_cast<float*>(yp) = val;
          else if (a.y_dtype == 1)
            *reinterpret_cast<__half*>(yp) = __float2half_rn(val);
          else
            *reinterpret_cast<__nv_bfloat16*>(yp) = __float2bfloat16_rn(val);
        }
      }
    }
  }
  // teardown: outstanding MMAs must finish before the tensor memory is released
  tc_fence_before();
  __syncthreads();
  if (warp == 1 && lane == 0 && *abort_flag) mbar_wait_ns(acc_full, 0u, kWaitBudgetNs, a.status);
  __syncthreads();
  tc_fence_after();
  if (warp == 3) tmem_dealloc(tmem, kTsCols);
}

// ---------------------------------------------------------------- activation staging
// One block per token row t < Mp.  16-bit formats: the row's max |x| gives a power-of-two
// scale; x / scale is rounded to f16 and stored in the decoder's k order (perm_*) in the
// 128-byte swizzled layout [row of 64 k][Mp / 8][8 tokens x 128 bytes].  W8A8: the
// reference encoder's E4M3 code of each x (unscaled, fp8_gemm.rs:96-101), 128 k per row.
// Tokens past M and k past K are zero.
template <int XDT>
__device__ __forceinline__ float ts_load(const void* x, int64_t off) {
  if constexpr (XDT == 0) return __ldg(static_cast<const float*>(x) + off);
  const unsigned short b = __ldg(static_cast<const unsigned short*>(x) + off);
  if constexpr (XDT == 1) return __half2float(__ushort_as_half(b));
  return __uint_as_float((uint32_t)b << 16);
}

template <int FMT>
__device__ __forceinline__ int ts_perm(int p) {
  if constexpr (FMT == FMT_Q4K) return perm_q4k(p);
  else if constexpr (FMT == FMT_Q6K) return perm_q6k(p);
  else if constexpr (FMT == FMT_TS_F8X) return perm_f8x(p);
  else return perm_q80(p);
}

template <int XDT, int FMT>
__global__ void __launch_bounds__(kPrepThreads) gemm_prep_ts_kernel(const void* x, int64_t ldx, int64_t M,
                                                                   int64_t Mp, int64_t K, int64_t kp, uint8_t* xw,
                                                                   float* tscale) {
  constexpr bool F8 = FMT == FMT_TS_F8X;
  constexpr int GK = TsFmt<FMT>::GK;
  pdl_trigger();
  pdl_wait();  // x may be the previous kernel's output
  const int64_t t = blockIdx.x;
  const bool live = t < M;
  const int64_t row = t * ldx;
  float inv = 1.0f;
  if constexpr (!F8) {
    __shared__ float red[kPrepThreads / 32];
    float m = 0.0f;
    if (live)
      for (int64_t k = threadIdx.x; k < K; k += kPrepThreads) m = fmaxf(m, fabsf(ts_load<XDT>(x, row + k)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    float mm = 0.0f;
#pragma unroll
    for (int w = 0; w < kPrepThreads / 32; ++w) mm = fmaxf(mm, red[w]);
    int e = 0;
    if (mm > 0.0f && mm <= 3.4e38f) e = min(max(ilogbf(mm) - 14, -110), 110);
    inv = ldexpf(1.0f, -e);
    if (threadIdx.x == 0) tscale[t] = ldexpf(1.0f, e);
  } else {
    if (threadIdx.x == 0) tscale[t] = 1.0f;
  }
  constexpr int UE = F8 ? 16 : 8;      // positions per 16-byte unit
  constexpr int RK = F8 ? 128 : 64;    // positions per 128-byte row
  const int64_t tg = t >> 3, r = t & 7;
  for (int64_t u = threadIdx.x; u < kp / UE; u += kPrepThreads) {
    const int64_t pos = u * UE, g = pos / GK;
    const int p0 = (int)(pos % GK);
    uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int e = 0; e < UE; ++e) {
      const int64_t k = g * GK + ts_perm<FMT>(p0 + e);
      const float f = (live && k < K) ? ts_load<XDT>(x, row + k) : 0.0f;
      if constexpr (F8) {
        w[e >> 2] |= (uint32_t)e4m3_code_of_value(e4m3_round_ref(f)) << (8 * (e & 3));
      } else {
        const __half h = __float2half_rn(f * inv);
        w[e >> 1] |= (uint32_t)__half_as_ushort(h) << (16 * (e & 1));
      }
    }
    const int64_t kb = pos / RK, c = (pos % RK) / UE;
    uint8_t* dst = xw + ((size_t)kb * (Mp / 8) + (size_t)tg) * 1024 + (size_t)r * 128 + (size_t)((c ^ r) & 7) * 16;
    *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

template <int FMT, int TN>
cudaError_t launch_ts_tn(const TsGemm& g, cudaStream_t st) {
  using P = TsPlan<FMT, TN>;
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(qgemm_ts_kernel<FMT, TN>, cudaFuncAttributeMaxDynamicSharedMemorySize, P::launch_bytes);
    if (e != cudaSuccess) return e;
    configured[dev & 63] = 1;
  }
  const dim3 grid((unsigned)(g.Mp / TN), (unsigned)((g.T + 7) / 8), (unsigned)g.splits);
  return launch_pdl(qgemm_ts_kernel<FMT, TN>, grid, dim3(kTsThreads), (size_t)P::launch_bytes, st, g);
}

template <int FMT>
cudaError_t launch_ts_fmt(const TsGemm& g, cudaStream_t st) {
  switch (g.TN) {
    case 16: return launch_ts_tn<FMT, 16>(g, st);
    case 32: return launch_ts_tn<FMT, 32>(g, st);
    default: return launch_ts_tn<FMT, 64>(g, st);
  }
}

template <int XDT>
cudaError_t launch_prep_xdt(int gfmt, const QGemvCall& c, int64_t Mp, int64_t kp, uint8_t* xw, float* tscale) {
  const dim3 grid((unsigned)Mp), block(kPrepThreads);
  switch (gfmt) {
    case FMT_Q4K: return launch_pdl(gemm_prep_ts_kernel<XDT, FMT_Q4K>, grid, block, 0, c.stream, c.x, c.ldx, c.M, Mp, c.K, kp, xw, tscale);
    case FMT_Q6K: return launch_pdl(gemm_prep_ts_kernel<XDT, FMT_Q6K>, grid, block, 0, c.stream, c.x, c.ldx, c.M, Mp, c.K, kp, xw, tscale);
    case FMT_TS_F8X: return launch_pdl(gemm_prep_ts_kernel<XDT, FMT_TS_F8X>, grid, block, 0, c.stream, c.x, c.ldx, c.M, Mp, c.K, kp, xw, tscale);
    default: return launch_pdl(gemm_prep_ts_kernel<XDT, FMT_Q80>, grid, block, 0, c.stream, c.x, c.ldx, c.M, Mp, c.K, kp, xw, tscale);
  }
}

}  // namespace

int ts_group_k(int gfmt) { return (gfmt == FMT_Q4K || gfmt == FMT_Q6K) ? 256 : 128; }

cudaError_t launch_ts_prep(const QGemvCall& c, int gfmt, int64_t Mp, int64_t kp, void* xw, float* tscale) {
  uint8_t* x8 = static_cast<uint8_t*>(xw);
  if (c.x_dtype == 0) return launch_prep_xdt<0>(gfmt, c, Mp, kp, x8, tscale);
  if (c.x_dtype == 1) return launch_prep_xdt<1>(gfmt, c, Mp, kp, x8, tscale);
  return launch_prep_xdt<2>(gfmt, c, Mp, kp, x8, tscale);
}

cudaError_t launch_ts_gemm(const TsGemm& g, cudaStream_t st) {
  switch (g.fmt) {
    case FMT_Q4K: return launch_ts_fmt<FMT_Q4K>(g, st);
    case FMT_Q6K: return launch_ts_fmt<FMT_Q6K>(g, st);
    case FMT_Q80: return launch_ts_fmt<FMT_Q80>(g, st);
    case FMT_FP8: return launch_ts_fmt<FMT_FP8>(g, st);
    default: return launch_ts_fmt<FMT_TS_F8X>(g, st);
  }
}

}  // namespace rtd
