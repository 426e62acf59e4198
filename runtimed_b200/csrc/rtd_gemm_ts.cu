// rtd_gemm_ts.cu -- tensor-core GEMM for skinny token counts (batched decode, speculative
// verify): the decoded weights are written to TENSOR memory and tcgen05.mma reads its A
// operand from there, so decoded weights never pass through shared memory.
//
//   y[M, N] = x[M, K] . W^T (+ bias)      W in Q4_K / Q6_K / Q8_0 / FP8-E4M3 groups
//
// One CTA computes 128 weight rows (eight 16-row tiles: the UMMA M) x TN tokens (16, 32 or
// 64: the UMMA N) with the f32 accumulator in tensor memory, one weight GROUP (GK = 256 k
// for the K-quants, 128 for Q8_0 / FP8) per pipeline step:
//   - each decode warp bulk-copies its own tile's groups into its part of a shared-memory
//     slot (up to eight slots ahead, refilled as soon as it has read one); warp 0 (one
//     lane) bulk-copies the group's activation tile, staged once per call by
//     gemm_prep_ts_kernel (a cp.async.bulk costs its issuing thread about the same time
//     whatever its size, so copies are few and large, and spread over threads);
//   - sixteen decode warps in two sets take alternate groups.  In a set, the warp of
//     tensor-memory lane quarter q and tile 2q + p decodes its tile's group: thread
//     4g + t holds exactly the bytes the group layout gives lane 4g + t (whole
//     sub-blocks of rows g and g + 8, conflict-free 16-byte shared loads), turns them
//     into f16 pairs -- the codes masked in place are exact f16 subnormals (code * 2^-24),
//     multiplied by the reference's per-sub-block factor times the weight's power of two
//     F (ts_decode_scale at upload, so the products are normal f16) and rounded once, one
//     f16 FMA per pair; the epilogue divides F out -- and
//     stores them with tcgen05.st.16x256b, whose thread pattern is that same lane
//     ownership: registers of thread 4g + t land in lanes g and g + 8, columns 2t and
//     2t + 1 of every 8-column repetition.  The k order inside a group is therefore the
//     decoder's, and the activations are staged in that order (perm_* below);
//   - lane 0 of warps 1 and 3 issue the tcgen05.mma of alternate groups (A from tensor
//     memory, B from the 128-byte swizzled activation tile), each into its own
//     accumulator, and commit them to the group's release barriers (tensor-memory slot and
//     activation slot);
//   - warps 4..7 (one per lane quarter) read each finished accumulator pair (tcgen05.ld),
//     add the two, and write y with the per-token activation scale, 1 / F, the row scale
//     (FP8, INT4 Marlin) and the bias, or f32 partials for a row tile shared with another
//     CTA (see the schedule below).
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

constexpr int kTsThreads = 640;     // 20 warps: 0 activations, 1 and 3 MMA (3 owns the TMEM), 2 idle, 4..19 decode
constexpr int kTsSmem = 227 * 1024;
constexpr int kTsCols = 512;        // the whole tensor memory of the SM (one CTA per SM)
constexpr int kTsMaxSlots = 8;
constexpr int kPrepThreads = 1024;  // one block per token

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
// weight slots (8 * GB bytes), SA tensor-memory A slots after the accumulators.
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
  static constexpr int kFixed = 1024 + 1024;  // alignment slack, barriers + misc
  static constexpr int kFitR = (kTsSmem - kFixed - SB * kB) / kRaw;
  // even: a decode warp refills the slot it has just read with the group SR later, which
  // belongs to its own set again
  static constexpr int SR = (kFitR < kTsMaxSlots ? kFitR : kTsMaxSlots) & ~1;
  // Two MMA-issuing threads take alternate groups into their own accumulators (summed by
  // the epilogue); NB accumulator pairs rotate over segments (two while they fit beside
  // three A slots, else one).
  static constexpr int ACC = TN < 32 ? 32 : TN;       // columns per accumulator
  static constexpr int NB = TN <= 32 ? 2 : 1;
  static constexpr int A0 = 2 * NB * ACC;              // first A column
  static constexpr int kFitA = (kTsCols - A0) / F::ACOLS;
  static constexpr int SA = kFitA < 6 ? kFitA : 6;
  static constexpr int offB = 0;
  static constexpr int offRaw = SB * kB;
  static constexpr int offBar = offRaw + SR * kRaw;
  static constexpr int nBars = 8 * SR + 3 * SB + 4 * SA + 2 * NB + 1;
  // phase index of a slot's barrier of one group parity: the slot's groups of that parity
  // recur every lcm(slots, 2) groups
  static constexpr int LA = SA % 2 ? 2 * SA : SA, LB = SB % 2 ? 2 * SB : SB;
  static constexpr int offMisc = offBar + nBars * 8;
  static constexpr int bytes = offMisc + 16 + 1024;
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
// The tensor cores get A = 2^s * w in f16, w the reference's weight: every code enters
// as an exact f16 SUBNORMAL (its bits are the code: value code * 2^-24), so a pair needs
// one mask and one f16 FMA with the factor scaled by F = 2^(24 + s) (a power of two fixed
// per weight at upload, the largest that keeps every scaled factor in the f16 range);
// the epilogue multiplies by 2^-s.  Factors are computed in f32 and rounded once to f16,
// as the products of the reference's factors with a power of two.
// grp: shared address of this tile's group; taddr: tensor-memory address of the tile's
// 16 lanes at the group's first A column.  Thread 4g + t (= lane) owns rows g and g + 8.

// Q4_K factor registers of one row: dl / nl for sub-block 2t (low nibbles), dh / nh for
// sub-block 2t + 1 (high nibbles, whose codes arrive as 16 q: dh carries F / 16), each
// duplicated into both halves.  The 6-bit scales and mins of all eight sub-blocks come
// out of the 12 packed bytes four at a time (scale_min_k4, dequant_k.rs:8-16): bytes
// 0-3 of the lo / hi words are sub-blocks 0-3 / 4-7; `hi` and `sel` are per-thread
// constants, so no thread branches.
struct Q4Fac {
  uint32_t dl, nl, dh, nh;
};
__device__ __forceinline__ Q4Fac q4k_factors(uint4 h, uint32_t hmask, uint32_t sel, float F, float A) {
  const uint32_t sc_lo = h.y & 0x3F3F3F3Fu, m_lo = h.z & 0x3F3F3F3Fu;
  const uint32_t sc_hi = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
  const uint32_t m_hi = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
  const uint32_t scw = sc_lo ^ ((sc_lo ^ sc_hi) & hmask), mw = m_lo ^ ((m_lo ^ m_hi) & hmask);
  const __half2 k1024 = __float2half2_rn(1024.0f);
  // (1024 + a, 1024 + b) -> (a, b): the two sub-blocks' integers, exact in f16
  const __half2 sc2 = __hsub2(bits_h2(prmt(scw, 0x64646464u, sel)), k1024);
  const __half2 m2 = __hsub2(bits_h2(prmt(mw, 0x64646464u, sel)), k1024);
  const float d = hbits(h.x & 0xFFFFu) * F, dmin = hbits(h.x >> 16) * A;
  // d * F is an f16 value times a power of two (exact); dmin * 2^s may fall below the f16
  // normal range, so the mins' products are formed in f32 and rounded once
  const uint32_t df = h2_bits(__hmul2(sc2, __floats2half2_rn(d, d * 0.0625f)));
  const float2 mf = __half22float2(m2);
  const uint32_t nf = h2_bits(__floats2half2_rn(-(dmin * mf.x), -(dmin * mf.y)));
  return Q4Fac{prmt(df, df, 0x1010u), prmt(nf, nf, 0x1010u), prmt(df, df, 0x3232u), prmt(nf, nf, 0x3232u)};
}

__device__ __forceinline__ uint32_t fma_h2(uint32_t a, uint32_t b, uint32_t c) {
  return h2_bits(__hfma2(bits_h2(a), bits_h2(b), bits_h2(c)));
}

__device__ __forceinline__ void ts_decode_q4k(uint32_t grp, uint32_t taddr, int lane, float F, float A) {
  const int g = lane >> 2, t = lane & 3;
  const uint32_t hmask = t >= 2 ? 0xFFFFFFFFu : 0u;
  const uint32_t sel = (t & 1) ? 0x4342u : 0x4140u;  // bytes (2t) & 3 and the next, each under a 0x64
  const Q4Fac f[2] = {q4k_factors(lds128(grp + 16 * g), hmask, sel, F, A),
                      q4k_factors(lds128(grp + 16 * (g + 8)), hmask, sel, F, A)};
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
        v[4 * (2 * w) + 0 + 2 * hr] = fma_h2(f[hr].dl, x & 0x000F000Fu, f[hr].nl);       // bytes 0, 2: sub-block 2t
        v[4 * (2 * w) + 1 + 2 * hr] = fma_h2(f[hr].dl, x8 & 0x000F000Fu, f[hr].nl);      // bytes 1, 3
        v[4 * (2 * w + 1) + 0 + 2 * hr] = fma_h2(f[hr].dh, x & 0x00F000F0u, f[hr].nh);   // sub-block 2t + 1
        v[4 * (2 * w + 1) + 1 + 2 * hr] = fma_h2(f[hr].dh, x8 & 0x00F000F0u, f[hr].nh);
      }
    }
    tmem_st16x256_x8(taddr + 64u * pp, v);
    // tcgen05.st reads its source registers asynchronously: they are not rewritten (the
    // next half reuses them) before the store has completed
    tmem_wait_st();
  }
}

// Q6_K: w = d * sc * (q - 32); with the code as a subnormal, the FMA adds -32 * F * d * sc
// * 2^-24, which is the rounded factor times -2^-19 (exact whenever it is a normal f16).
__device__ __forceinline__ void ts_decode_q6k(uint32_t grp, uint32_t taddr, int lane, float F) {
  const int g = lane >> 2;
  const float d[2] = {hbits(lds16(grp + 4 * g)) * F, hbits(lds16(grp + 4 * g + 2)) * F};
  const uint32_t scw[2] = {lds32(grp + 32 + lane * 8), lds32(grp + 32 + lane * 8 + 4)};
  const __half2 k_off = __float2half2_rn(-0.0000019073486328125f);  // -2^-19
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
      const float ds = d[hr] * (float)(int)(int8_t)(uint8_t)(scw[hr] >> (8 * (2 * hh + par)));
      const __half2 f2 = __floats2half2_rn(ds, ds);
      const uint32_t fa = h2_bits(f2), fc = h2_bits(__hmul2(f2, k_off));
      const uint32_t c[8] = {X & 0x003F003Fu,
                             (X >> 6) & 0x003F003Fu,
                             Y & 0x003F003Fu,
                             (Y >> 6) & 0x003F003Fu,
                             Z & 0x003F003Fu,
                             (Z >> 6) & 0x003F003Fu,
                             ((X >> 12) & 0x000F000Fu) | ((Z >> 8) & 0x00300030u),
                             ((Y >> 12) & 0x000F000Fu) | ((Z >> 10) & 0x00300030u)};
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) v[4 * (4 * par + (jj >> 1)) + (jj & 1) + 2 * hr] = fma_h2(fa, c[jj], fc);
    }
    tmem_st16x256_x8(taddr + 64u * hh, v);
    tmem_wait_st();  // as above: the next half reuses the source registers
  }
}

// Q8_0: w = d * b; the byte b + 128 enters as a subnormal and the FMA adds -128 * F * d *
// 2^-24 = the scaled d times -2^-17.  FP8 (W8A16): E4M3 -> f16 is exact; its row scale is
// applied in the epilogue.
template <bool Q8>
__device__ __forceinline__ void ts_decode_8bit(uint32_t grp, uint32_t taddr, int lane, float F) {
  uint32_t fa[2] = {0u, 0u}, fc[2] = {0u, 0u};
  if constexpr (Q8) {
    const __half2 k_off = __float2half2_rn(-0.00000762939453125f);  // -2^-17
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const float dv = hbits(lds16(grp + 4 * lane + 2 * hr)) * F;
      const __half2 f2 = __floats2half2_rn(dv, dv);
      fa[hr] = h2_bits(f2);
      fc[hr] = h2_bits(__hmul2(f2, k_off));
    }
  }
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
        if constexpr (Q8)
          o = fma_h2(fa[hr], prmt(x ^ 0x80808080u, 0u, s ? 0x4342u : 0x4140u), fc[hr]);
        else
          o = e4m3x2_to_f16x2((uint16_t)(s ? (x >> 16) : (x & 0xFFFFu)));
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
__device__ __forceinline__ void ts_decode(uint32_t grp, uint32_t taddr, int lane, float F, float A) {
  if constexpr (FMT == FMT_Q4K)
    ts_decode_q4k(grp, taddr, lane, F, A);
  else if constexpr (FMT == FMT_Q6K)
    ts_decode_q6k(grp, taddr, lane, F);
  else if constexpr (FMT == FMT_Q80)
    ts_decode_8bit<true>(grp, taddr, lane, F);
  else if constexpr (FMT == FMT_FP8)
    ts_decode_8bit<false>(grp, taddr, lane, F);
  else
    ts_copy_f8x(grp, taddr, lane);
}

// ---------------------------------------------------------------- GEMM kernel
// Persistent stream-K schedule.  The call's work is the sequence of units (row tile rt of
// 128 rows, group g), rt-major, U = R * G of them; CTA c of C (one per SM) takes units
// [c U / C, (c + 1) U / C) through one pipeline, so every SM gets the same number of
// groups whatever the shape.  A CTA's run crosses row tiles: each row tile's share (a
// "segment") accumulates in one of two tensor-memory accumulators in turn, so the MMAs of
// the next segment overlap the epilogue of the last.  A segment covering its whole row
// tile writes y; the first and last segments of a CTA may cover part of one and write
// f32 partials, which ts_fixup_kernel adds up in CTA order (deterministic).
__host__ __device__ __forceinline__ int ts_unit0(int c, int U, int C) { return (int)((int64_t)c * U / C); }

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
  // Barriers of the activation and A slots are split by the parity of the group (the two
  // decode sets and the two MMA issuers take alternate groups): a slot ring of odd length
  // alternates parities, and a thread waiting on a barrier whose previous phase is still
  // open would read that phase's parity as done.  Split, every barrier's phases are
  // produced and consumed in order by the same threads.
  uint64_t* raw_full = bar;  // [SR][8]: slot x 16-row tile (one warp each)
  uint64_t* b_full = raw_full + 8 * SR;  // [2][SB]: group parity x slot
  uint64_t* b_empty = b_full + 2 * SB;   // [SB] (the producer waits every phase in order)
  uint64_t* a_full = b_empty + SB;       // [2][SA]
  uint64_t* a_empty = a_full + 2 * SA;   // [2][SA]
  constexpr int NB = P::NB, LA = P::LA, LB = P::LB;
  uint64_t* acc_full = a_empty + 2 * SA; // [NB]
  uint64_t* acc_empty = acc_full + NB; // [NB]
  uint64_t* mma_done = acc_empty + NB;
  uint32_t* misc = reinterpret_cast<uint32_t*>(sm + P::offMisc);  // [0] tensor-memory base, [1] abort flag

  // unit counts fit 32 bits (the host checks); the loops below advance (row tile, group)
  // incrementally instead of dividing
  const int G = (int)a.G, U = (int)(a.R * a.G);
  const int u0 = ts_unit0(blockIdx.x, U, gridDim.x), u1 = ts_unit0(blockIdx.x + 1, U, gridDim.x);
  const int n = u1 - u0;
  const int rt0 = u0 / G, g0 = u0 - rt0 * G;  // first row tile of this CTA, its first group
  const int nseg = n > 0 ? (u1 - 1) / G - rt0 + 1 : 0;

  if (warp == 3) {
    tmem_alloc(smem_u32(&misc[0]), kTsCols);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < 8 * SR; ++s) mbar_init(&raw_full[s], 1);
    for (int s = 0; s < SB; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&b_full[SB + s], 1);
      mbar_init(&b_empty[s], 1);
    }
    for (int s = 0; s < 2 * SA; ++s) {
      mbar_init(&a_full[s], 8);   // the eight tile warps of the set
      mbar_init(&a_empty[s], 1);  // the commit of the thread that multiplied the group
    }
    for (int s = 0; s < NB; ++s) {
      mbar_init(&acc_full[s], 2);
      mbar_init(&acc_empty[s], 4);  // the four epilogue warps
    }
    mbar_init(mma_done, 2);
    misc[1] = 0;
    fence_mbar_init();
  }
  pdl_trigger();  // the fixup kernel (or the next call) may launch; it waits for this grid
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
      int issued = 0, g = g0;
      for (int gi = 0; gi < n; ++gi, g = (g + 1 == G) ? 0 : g + 1) {
        const int sb = gi % SB;
        if (gi >= SB && !wait(&b_empty[sb], (uint32_t)((gi / SB - 1) & 1))) break;
        uint64_t* bf = &b_full[(gi & 1) * SB + sb];
        mbar_arrive_expect_tx(bf, (uint32_t)P::kB);
        // the group's kRows 128-byte rows are contiguous in the staging buffer: one copy
        bulk_g2s(sm + P::offB + sb * P::kB, xw + (size_t)g * P::kB, P::kB, bf);
        ++issued;
      }
      if (*abort_flag)  // no copy may still be landing when the CTA exits
        for (int gi = (issued > SB ? issued - SB : 0); gi < issued; ++gi)
          mbar_wait_ns(&b_full[(gi & 1) * SB + gi % SB], (uint32_t)((gi / LB) & 1), kWaitBudgetNs, a.status);
    }
  } else if (warp == 1 || warp == 3) {
    // ---- MMA issuers: lane 0 of warp 1 takes the even units of the CTA's run into
    // accumulator 0 of the segment's pair, lane 0 of warp 3 the odd ones into accumulator 1.
    // An M = 128 tcgen05.mma occupies the tensor pipe ~45 cycles however small N is, and a
    // group needs eight or sixteen of them; while one thread waits for its next group's
    // barriers the other keeps the pipe busy.
    if (lane == 0) {
      const int j = warp == 1 ? 0 : 1;
      constexpr uint32_t idesc = idesc_f16(TN);  // kind::f8f6f4 reads the same fields as E4M3 x E4M3
      const uint64_t db0 = kmajor_desc(smem_u32(sm + P::offB));
      int seg = 0, g = g0;
      bool fresh = true;  // no MMA of this thread in the current segment yet
      for (int gi = 0; gi < n; ++gi, g = (g + 1 == G) ? 0 : g + 1) {
        const int bf = seg % NB;
        const bool first = gi == 0 || g == 0, last = gi == n - 1 || g == G - 1;
        if (first) {
          fresh = true;
          if (seg >= NB && !wait(&acc_empty[bf], (uint32_t)((seg / NB - 1) & 1))) break;
        }
        if ((gi & 1) == j) {
          const int sa = gi % SA, sb = gi % SB;
          if (!wait(&a_full[j * SA + sa], (uint32_t)((gi / LA) & 1)) ||
              !wait(&b_full[j * SB + sb], (uint32_t)((gi / LB) & 1)))
            break;
          tc_fence_after();
          const uint32_t acc = tmem + (uint32_t)((2 * bf + j) * P::ACC);
          const uint32_t a_col = tmem + (uint32_t)(P::A0 + sa * F::ACOLS);
          const uint64_t db = db0 + (uint64_t)((sb * P::kB) >> 4);
#pragma unroll
          for (int i = 0; i < F::NMMA; ++i) {
            // slice i: 8 tensor-memory columns; in the activation slot, 128-byte row i / 4 at byte 32 (i % 4)
            const uint64_t bd = db + (uint64_t)(((i >> 2) * TN * 128) >> 4) + 2 * (i & 3);
            const uint32_t accum = (fresh && i == 0) ? 0u : 1u;
            if constexpr (F8)
              umma_f8_ts(acc, a_col + 8u * i, bd, idesc, accum);
            else
              umma_f16_ts(acc, a_col + 8u * i, bd, idesc, accum);
          }
          fresh = false;
          umma_commit(&a_empty[j * SA + sa]);
          umma_commit(&b_empty[sb]);
        }
        if (last) {
          umma_commit(&acc_full[bf]);  // both threads: the segment's sums are complete
          ++seg;
        }
      }
      umma_commit(mma_done);  // fires once every MMA this thread issued has completed
    }
  } else if (warp >= 4) {
    // ---- decode warps: lane quarter q = warp % 4 (tensor-memory lanes 32q ..), tile 2q + p
    const int dw = warp - 4, q = warp & 3, p = (dw >> 2) & 1, set = dw >> 3;
    const int tile = 2 * q + p;
    const uint32_t tlane = (uint32_t)(32 * q + 16 * p) << 16;
    const float wa = a.wpow2 * 5.9604644775390625e-08f;  // 2^s = F * 2^-24
    // warps 4..7 (set 0, one per lane quarter) also run the epilogues, between their groups
    const bool epi = warp < 8;
    int ep = 0;           // next segment to finish
    bool scales = false;  // the prep kernel's token scales are visible
    auto epilogue = [&](int sg) {
      if (!scales) {
        pdl_wait();
        scales = true;
      }
      tc_fence_after();
      const int rt = rt0 + sg;
      const bool complete = u0 <= rt * G && u1 >= rt * G + G;
      // a one-unit segment filled only the accumulator of its unit's parity
      const int s_lo = u0 > rt * G ? u0 : rt * G, s_hi = u1 < rt * G + G ? u1 : rt * G + G;
      const bool has0 = s_hi - s_lo >= 2 || ((s_lo - u0) & 1) == 0;
      const bool has1 = s_hi - s_lo >= 2 || ((s_lo - u0) & 1) == 1;
      const int r = q * 32 + lane;
      const int64_t nrow = (int64_t)rt * 128 + r;
      // 2^-s undoes the decoders' power of two (K-quants, Q8_0); FP8 takes its row scale
      float es = (FMT == FMT_FP8 || F8) ? 1.0f : 16777216.0f / a.wpow2, eb = 0.0f;
      if (nrow < a.N) {
        if (a.row_scale) es *= a.row_scale[a.scale_len == 1 ? 0 : nrow];
        if (a.bias) eb = a.bias[nrow];
      }
      float* part = a.partial + (size_t)(2 * blockIdx.x + (sg == 0 ? 0 : 1)) * TN * 128 + r;
#pragma unroll 1
      for (int c0 = 0; c0 < TN; c0 += 16) {
        float v[16], v1[16];
        const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(2 * (sg % NB) * P::ACC + c0);
        tmem_ld16(ta, v);
        tmem_ld16(ta + (uint32_t)P::ACC, v1);
#pragma unroll
        for (int jj = 0; jj < 16; ++jj)  // the two issuers' sums, in a fixed order
          v[jj] = (has0 ? v[jj] : 0.0f) + (has1 ? v1[jj] : 0.0f);
        if (nrow >= a.N || c0 >= a.M) continue;
        if (!complete) {
#pragma unroll
          for (int j = 0; j < 16; ++j) part[(size_t)(c0 + j) * 128] = v[j];
          continue;
        }
        const int jn = (a.M - c0) < 16 ? (int)(a.M - c0) : 16;
        const int ysz = a.y_dtype == 0 ? 4 : 2;
        uint8_t* yp = static_cast<uint8_t*>(a.y) + ((int64_t)c0 * a.ldy + nrow) * ysz;
        const int64_t ystep = a.ldy * ysz;
#pragma unroll
        for (int j = 0; j < 16; ++j, yp += ystep) {
          if (j >= jn) break;
          const float val = v[j] * a.tscale[c0 + j] * es + eb;
          if (a.y_dtype == 0)
            *reinterpret_cast<float*>(yp) = val;
          else if (a.y_dtype == 1)
            *reinterpret_cast<__half*>(yp) = __float2half_rn(val);
          else
            *reinterpret_cast<__nv_bfloat16*>(yp) = __float2bfloat16_rn(val);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[sg % NB]);
    };
    // Lane 0 alone polls a barrier (512 polling threads slow every barrier operation of the
    // SM, the MMA issuers' included); once it has seen the phase complete, every lane
    // observes it once more (an already completed phase: one try_wait) for its own acquire
    // of the data.  On the epilogue warps the wait also runs every segment that completes
    // meanwhile (the MMA warps may be waiting for that accumulator).  Warp-uniform.
    auto wait_d = [&](uint64_t* b, uint32_t parity) -> bool {
     for (;;) {
      int r = 1;  // lane 0: 1 done, 0 failed, 2 an epilogue is due
      if (lane == 0) {
        if (!mbar_try_wait(b, parity)) {
          const uint64_t t_start = global_ns();
          for (;;) {
            if (epi && ep < nseg && mbar_try_wait(&acc_full[ep % NB], (uint32_t)((ep / NB) & 1))) {
              r = 2;
              break;
            }
            if (mbar_try_wait_sleep(b, parity, 2000u)) break;
            if (*abort_flag) {
              r = 0;
              break;
            }
            if (global_ns() - t_start > kWaitBudgetNs) {
              raise_status(a.status, kDevWaitTimeout);
              *abort_flag = 1;
              r = 0;
              break;
            }
          }
        }
      }
      r = __shfl_sync(0xffffffffu, r, 0);
      if (r == 2) {
        mbar_try_wait(&acc_full[ep % NB], (uint32_t)((ep / NB) & 1));
        epilogue(ep++);
        continue;
      }
      if (r == 1) mbar_try_wait(b, parity);
      return r == 1;
     }
    };
    // Each decode warp streams its own 16-row tile's groups: the slot region it has just
    // decoded is refilled at once with its tile's group SR later (bulk copies are issued
    // by sixteen threads in parallel; one thread issuing them all is too slow), so its
    // barrier [slot][tile] needs no release by any other warp.
    auto issue = [&](int gi) {  // lane 0: the tile's copy of unit u0 + gi into slot gi % SR
      const int u = u0 + gi, rt = u / G, g = u - rt * G;
      uint64_t* b = &raw_full[(gi % SR) * 8 + tile];
      const int64_t t16 = (int64_t)rt * 8 + tile;
      if (t16 < a.T) {
        mbar_arrive_expect_tx(b, (uint32_t)F::GB);
        bulk_g2s(sm + P::offRaw + (gi % SR) * P::kRaw + tile * F::GB, a.w + (t16 * G + g) * F::GB, F::GB, b);
      } else {
        mbar_arrive(b);  // rows past N: no copy, but the phase advances
      }
    };
    int issued = set;  // this warp issues units set, set + 2, ... in order
    if (lane == 0)
      for (; issued < n && issued < SR; issued += 2) issue(issued);
    for (int gi = set; gi < n; gi += 2) {
      const int sr = gi % SR, sa = gi % SA;
      const bool live = (int64_t)((u0 + gi) / G) * 8 + tile < a.T;
      bool ok = wait_d(&raw_full[sr * 8 + tile], (uint32_t)((gi / SR) & 1));
      // the slot's previous group, gi - SA, was multiplied by the issuer of its parity
      if (ok && gi >= SA) ok = wait_d(&a_empty[((gi - SA) & 1) * SA + sa], (uint32_t)(((gi - SA) / LA) & 1));
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      if (live)
        ts_decode<FMT>(smem_u32(sm + P::offRaw + sr * P::kRaw + tile * F::GB),
                       tmem + tlane + (uint32_t)(P::A0 + sa * F::ACOLS), lane, a.wpow2, wa);
      tmem_wait_st();  // before any register the stores read can be reused
      // the slot's bytes are in registers: order those reads before the async refill
      fence_async_shared();
      __syncwarp();
      if (lane == 0 && issued < n) {
        issue(issued);
        issued += 2;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[set * SA + sa]);
    }
    // no copy may still be landing when the CTA exits (only an aborted run leaves any)
    if (lane == 0 && *abort_flag)
      for (int gi = (issued - SR > set ? issued - SR : set); gi < issued; gi += 2)
        mbar_wait_ns(&raw_full[(gi % SR) * 8 + tile], (uint32_t)((gi / SR) & 1), kWaitBudgetNs, a.status);
    if (epi)
      while (ep < nseg) {
        const int ok = __shfl_sync(0xffffffffu, lane == 0 ? (int)wait(&acc_full[ep % NB], (uint32_t)((ep / NB) & 1)) : 0, 0);
        if (!ok) break;
        mbar_try_wait(&acc_full[ep % NB], (uint32_t)((ep / NB) & 1));
        epilogue(ep++);
      }
  }
  // teardown: outstanding MMAs must finish before the tensor memory is released
  tc_fence_before();
  __syncthreads();
  if (warp == 1 && lane == 0) mbar_wait_ns(mma_done, 0u, kWaitBudgetNs, a.status);  // both issuers' MMAs
  __syncthreads();
  tc_fence_after();
  if (warp == 3) tmem_dealloc(tmem, kTsCols);
}

// Row tiles whose units span several CTAs: their f32 partials (slot 2c for the first
// segment of CTA c, 2c + 1 for its last) added in CTA order, then scaled and biased as the
// GEMM's epilogue does.  Block (row tile, chunk of 8 tokens), one thread per row.
__global__ void __launch_bounds__(128) ts_fixup_kernel(const float* partial, int R, int G, int C, int TN, int M,
                                                       int64_t N, const float* tscale, const float* row_scale,
                                                       int scale_len, float escale, const float* bias, void* y,
                                                       int y_dtype, int64_t ldy) {
  pdl_trigger();
  pdl_wait();  // the partials are the GEMM's output
  const int rt = blockIdx.x, U = R * G, t0 = 8 * blockIdx.y;
  // the CTA whose units include u: the last c with floor(c U / C) <= u, i.e. c U < (u + 1) C
  auto cta_of = [&](int u) {
    const int64_t c = ((int64_t)(u + 1) * C - 1) / U;
    return (int)(c < C - 1 ? c : C - 1);
  };
  const int ca = cta_of(rt * G), cb = cta_of(rt * G + G - 1);
  const int64_t tile_u0 = (int64_t)rt * G * C;  // c's first unit is in this row tile iff c U >= rt G C
  const int64_t nrow = (int64_t)rt * 128 + threadIdx.x;
  if (ca == cb || nrow >= N) return;  // one CTA covered the row tile and wrote y itself
  const float es = row_scale ? escale * row_scale[scale_len == 1 ? 0 : nrow] : escale;
  const float eb = bias ? bias[nrow] : 0.0f;
  float s[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) s[j] = 0.0f;
  for (int c = ca; c <= cb; ++c) {
    const int which = (int64_t)c * U >= tile_u0 ? 0 : 1;
    const float* p = partial + ((size_t)(2 * c + which) * TN + t0) * 128 + threadIdx.x;
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j] += (t0 + j < TN) ? p[(size_t)j * 128] : 0.0f;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int t = t0 + j;
    if (t >= M) break;
    const float val = s[j] * tscale[t] * es + eb;
    const int64_t off = (int64_t)t * ldy + nrow;
    if (y_dtype == 0)
      static_cast<float*>(y)[off] = val;
    else if (y_dtype == 1)
      static_cast<__half*>(y)[off] = __float2half_rn(val);
    else
      static_cast<__nv_bfloat16*>(y)[off] = __float2bfloat16_rn(val);
  }
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
  return launch_pdl(qgemm_ts_kernel<FMT, TN>, dim3((unsigned)g.ctas), dim3(kTsThreads), (size_t)P::launch_bytes, st,
                    g);
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

bool ts_needs_fixup(int R, int G, int C) {
  for (int c = 1; c < C; ++c)
    if (ts_unit0(c, R * G, C) % G != 0) return true;
  return false;
}

cudaError_t launch_ts_gemm(const TsGemm& g, cudaStream_t st) {
  cudaError_t e;
  switch (g.fmt) {
    case FMT_Q4K: e = launch_ts_fmt<FMT_Q4K>(g, st); break;
    case FMT_Q6K: e = launch_ts_fmt<FMT_Q6K>(g, st); break;
    case FMT_Q80: e = launch_ts_fmt<FMT_Q80>(g, st); break;
    case FMT_FP8: e = launch_ts_fmt<FMT_FP8>(g, st); break;
    default: e = launch_ts_fmt<FMT_TS_F8X>(g, st); break;
  }
  if (e != cudaSuccess || !ts_needs_fixup((int)g.R, (int)g.G, g.ctas)) return e;
  const bool q = g.fmt != FMT_FP8 && g.fmt != FMT_TS_F8X;
  return launch_pdl(ts_fixup_kernel, dim3((unsigned)g.R, (unsigned)((g.M + 7) / 8)), dim3(128), 0, st,
                    (const float*)g.partial, (int)g.R, (int)g.G, g.ctas, g.TN, (int)g.M, g.N, g.tscale, g.row_scale,
                    g.scale_len, q ? 16777216.0f / g.wpow2 : 1.0f, g.bias, g.y, g.y_dtype, g.ldy);
}

}  // namespace rtd
