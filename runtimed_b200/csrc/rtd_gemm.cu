// rtd_gemm.cu -- tcgen05 / TMEM tensor-core GEMM for token counts past the decode
// GEMV's sweet spot, and the planner of every call of four or more tokens: up to 64
// tokens (batched decode, speculative verify) run the skinny kernel of rtd_gemm_ts.cu
// (decoded weights in tensor memory) unless RTD_GEMM_TS=0; prefill sizes run the
// kernel below (decoded weights in shared memory).
//
//   y[M, N] = x[M, K] . W^T (+ bias)      W in Q4_K / Q6_K / Q8_0 / FP8-E4M3 groups
//
// One CTA computes 128 weight rows (eight 16-row tiles: the UMMA M) x TN tokens (the
// UMMA N, 16..256) with the fp32 accumulator in tensor memory.  Per 64-element k
// stage:
//   - warp 18 (one lane) streams the packed groups of the eight tiles into shared
//     memory with cp.async.bulk (mbarrier transaction counts), up to 3-4 groups
//     ahead; warp 0 (one lane) streams the stage's activation tile the same way;
//   - warps 2..17 decode the stage's weights into f16 pairs (codes exact in f16, the
//     reference's per-sub-block factors computed in f32 and rounded once to f16, one
//     f16 FMA per pair) straight into the 128-byte swizzled K-major layout;
//   - one lane of warp 1 (even stages) or of warp 19 (odd stages) issues the four
//     K=16 tcgen05.mma of the stage into its own accumulator and commits them to the
//     stage's "empty" barrier, which releases both buffers;
//   - after the last stage warps 4..7 read both accumulators (tcgen05.ld, one TMEM
//     lane quarter each), add them, and write y with the per-token activation scale,
//     the row scale (FP8, INT4 Marlin) and the bias.
// The activations are staged once per call by gemm_prep_kernel: power-of-two-scaled
// f16 per token, already in the swizzled layout, so one bulk copy moves a tile.  The
// prep, GEMM and (split-K) reduce kernels are chained with programmatic dependent
// launch: the GEMM allocates tensor memory, loads and decodes weights while the prep
// kernel runs, and only the activation producer and the epilogue wait for it.
// Every wait is bounded by %globaltimer; a timeout records kDevWaitTimeout and the
// CTA stops issuing work, drains what it issued and returns.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdlib>
#include <type_traits>
#include <utility>

#include "rtd_common.cuh"
#include "rtd_kernels.h"
#include "rtd_tcgen05.cuh"

namespace rtd {
namespace {

// Warp roles of one CTA for DW decode warps (warps 2 .. 2 + DW - 1).  DW = 16: one CTA per
// SM with the whole 227 KB; DW = 8: two CTAs per SM, each with at most 113 KB, so that two
// independent pipelines hide each other's latencies and the grid of a skinny call fits
// the SMs in one wave.
template <int DW>
struct Roles {
  static constexpr int kDecodeWarps = DW;
  static constexpr int kGemmWarps = DW + 4;
  static constexpr int kWarpRaw = DW + 2;      // packed-group producer
  static constexpr int kWarpMmaOdd = DW + 3;   // MMA issuer of the odd k stages (warp 1: the even ones)
  static constexpr int kThreads = kGemmWarps * 32;
  static constexpr int kDecodeThreads = DW * 32;
  static constexpr int kHalvesPerThread = 512 / kDecodeThreads;  // 16-weight halves a thread takes per stage
  static constexpr int kCtasPerSm = DW == 8 ? 2 : 1;
  static constexpr int kSmem = DW == 8 ? 113 * 1024 : 227 * 1024;
};
constexpr int kBM = 128;             // weight rows per CTA (UMMA M)
constexpr int kBK = 64;              // k per stage
constexpr int kMaxStages = 8;
constexpr int kPrepThreadsG = 256;

// FP8 weights with E4M3-encoded activations (W8A8): the E4M3 tiles enter
// tcgen05.mma.kind::f8f6f4 as they are, so the "decode" warps only move 16-byte units
// into the swizzled layout.  An internal id beside the layout formats of rtd_layout.h.
constexpr int FMT_F8X = FMT_TS_F8X;

template <int FMT>
struct GemmFmt;
template <>
struct GemmFmt<FMT_F8X> {
  static constexpr int GK = 128, GB = 2048;
};
template <>
struct GemmFmt<FMT_Q4K> {
  static constexpr int GK = 256, GB = 2304;
};
template <>
struct GemmFmt<FMT_Q6K> {
  static constexpr int GK = 256, GB = 3360;
};
template <>
struct GemmFmt<FMT_Q80> {
  static constexpr int GK = 128, GB = 2176;
};
template <>
struct GemmFmt<FMT_FP8> {
  static constexpr int GK = 128, GB = 2048;
};

struct GemmArgs {
  const uint8_t* w;
  const float* row_scale;  // per output row (FP8, INT4 Marlin weights), or null
  int scale_len;
  int64_t N, T, G;         // rows, 16-row tiles, groups per row
  int nkb;                 // k stages (64 elements; 128 on the kind::f8f6f4 path)
  const __half* xw;        // staged activations [nkb][Mp / 8][1024-byte swizzled atom]
  const float* tscale;     // [Mp] per-token scale
  int64_t M, Mp;
  const float* bias;
  void* y;
  int y_dtype;
  int64_t ldy;
  int* status;
  int splits;              // K splits (grid z); > 1: write f32 partials instead of y
  float* partial;          // [splits][Mp][N] when splits > 1
};

// ---------------------------------------------------------------- stage decode
// Codes become f16 pairs without the conversion pipe: 0x6400 | v is the f16 1024 + v
// (v < 1024), and subtracting 1024 (+ a bias) is exact.  The weight is then one f16
// FMA / multiply per pair with the factor (and offset) rounded once from f32.

// 16 weights of row r of the CTA tile (tile i = r / 16, row rr = r % 16 = g + 8 * hrow):
// part and h pick its 16 of the stage's 64 k.  Eight consecutive threads share
// (part, h) and hold eight consecutive rows, so each quarter-warp stores eight 16-byte
// chunks that fall on distinct banks.
// raw_s: shared address of the eight groups of this stage's k range (group layouts of
// rtd_layout.h); sub: which 64-wide block of the group; a_s: the stage's A tile.
template <int FMT>
__device__ __forceinline__ void decode_half(uint32_t raw_s, int sub, uint32_t a_s, int r, int part, int h) {
  constexpr int GB = GemmFmt<FMT>::GB;
  const int i = r >> 4, rr = r & 15, g = rr & 7, hrow = rr >> 3;
  const uint32_t grp = raw_s + (uint32_t)(i * GB);
  uint32_t o[8];
  int k0;
  if constexpr (FMT == FMT_Q4K) {
    // chunk c = sub: low nibbles (h = 0) are sub-block 2c (local k 0..31), high
    // nibbles (h = 1) sub-block 2c + 1 (local k 32..63)
    const uint4 hdr = lds128(grp + 16 * rr);
    const float d = hbits(hdr.x & 0xFFFFu), dmin = hbits(hdr.x >> 16);
    uint32_t sc, mn;
    scale_min_words(2 * sub + h, hdr.y, hdr.z, hdr.w, sc, mn);
    const __half2 d1 = h2_const(d * (float)sc), n1 = h2_const(-(dmin * (float)mn));
    const __half2 k1024 = h2_const(1024.0f);
    const uint4 q = lds128(grp + 256 + (2 * hrow + part) * 512 + (4 * g + sub) * 16);
    const uint32_t wd[4] = {q.x, q.y, q.z, q.w};
    const int sh = 4 * h;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      // bytes (0, 2) / (1, 3) of word j / 2 -> halves 0, 1 (the unit order of the staged
      // Q4_K activations); their nibble (low or high) -> 1024 + q
      const uint32_t p2 = prmt(wd[j >> 1], 0u, (j & 1) ? 0x4341u : 0x4240u) >> sh;
      const __half2 v = __hsub2(bits_h2((p2 & 0x000F000Fu) | 0x64006400u), k1024);
      o[j] = h2_bits(__hfma2(d1, v, n1));
    }
    k0 = 32 * h + 16 * part;
  } else if constexpr (FMT == FMT_Q6K) {
    const float d = hbits(lds16(grp + 4 * g + 2 * hrow));
    const int sb = 4 * sub + 2 * part + h;  // 16-element sub-block of the superblock
    const int hh = sb >> 3, sbi = sb & 7, tq = sbi >> 1, side = sbi & 1;
    const int lane = 4 * g + tq;
    const uint32_t scw = lds32(grp + 32 + lane * 8 + 4 * hrow);  // this row's 4 scale bytes of the lane
    const __half2 ds = h2_const(d * (float)(int)(int8_t)(uint8_t)(scw >> (8 * (2 * hh + side))));
    const __half2 k1056 = h2_const(1056.0f);  // 1024 + 32
    const int w0 = 12 * hh + 3 * (2 * side + hrow);
    auto word = [&](int w) -> uint32_t { return lds32(grp + 288 + (w >> 2) * 512 + lane * 16 + (w & 3) * 4); };
    const uint32_t X = word(w0), Y = word(w0 + 1), Z = word(w0 + 2);
    // element pairs: each word holds codes at bits {0, 16} and {6, 22}; the spare bits
    // 12..15 / 28..31 of X and Y with two bits of Z each make the last four codes
    const uint32_t c[8] = {X & 0x003F003Fu,
                           (X >> 6) & 0x003F003Fu,
                           Y & 0x003F003Fu,
                           (Y >> 6) & 0x003F003Fu,
                           Z & 0x003F003Fu,
                           (Z >> 6) & 0x003F003Fu,
                           ((X >> 12) & 0x000F000Fu) | ((Z >> 8) & 0x00300030u),
                           ((Y >> 12) & 0x000F000Fu) | ((Z >> 10) & 0x00300030u)};
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = h2_bits(__hmul2(ds, __hsub2(bits_h2(c[j] | 0x64006400u), k1056)));
    k0 = 16 * (2 * part + h);
  } else {  // Q8_0 / FP8: block b = 2 * sub + part of the group, local k 32 * part + 16 * h ..
    const int lane = 4 * g + 2 * sub + part;
    const uint4 q = lds128(grp + ((FMT == FMT_Q80) ? 128 : 0) + (2 * hrow + h) * 512 + lane * 16);
    const uint32_t wd[4] = {q.x, q.y, q.z, q.w};
    if constexpr (FMT == FMT_Q80) {
      // signed byte b -> (b ^ 0x80) in the low byte of 0x64xx -> 1024 + 128 + b
      const __half2 dq = bits_h2(lds16(grp + 4 * lane + 2 * hrow) * 0x10001u);
      const __half2 k1152 = h2_const(1152.0f);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t p2 = prmt(wd[j >> 1] ^ 0x80808080u, 0x64u, (j & 1) ? 0x4342u : 0x4140u);
        o[j] = h2_bits(__hmul2(dq, __hsub2(bits_h2(p2), k1152)));
      }
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        o[2 * j] = e4m3x2_to_f16x2((uint16_t)(wd[j] & 0xFFFFu));
        o[2 * j + 1] = e4m3x2_to_f16x2((uint16_t)(wd[j] >> 16));
      }
    }
    k0 = 32 * part + 16 * h;
  }
  sts128(a_s + sw_off(r, k0), o[0], o[1], o[2], o[3]);
  sts128(a_s + sw_off(r, k0 + 8), o[4], o[5], o[6], o[7]);
}

// Q4_K, two consecutive stages of one group per iteration (four or more pipeline
// stages): thread dt decodes stage dt / 256 of the pair, row r, part p -- the 16 packed
// bytes whose low nibbles are elements 16p .. 16p + 15 of sub-block 2c and whose high
// nibbles are the same elements of sub-block 2c + 1 (dequant_k.rs:19-44), c = the stage
// within the group: 32 weights from one header read.  Pairs are bytes (0, 2) and (1, 3)
// of each word, so one LOP3 (plus a shift) makes a pair 1024 + q; the staged activations
// of Q4_K follow the matching unit order (0, 2, 1, 3, 4, 6, 5, 7).
struct Q4Thread {
  uint32_t hdr;     // the row's 16 header bytes, relative to the stage's raw slot
  uint32_t q;       // part p's 16 code bytes of chunk 0, relative to the raw slot
  uint32_t st[4];   // swizzled store offsets of the lo / hi chunks, relative to the A tile
};

__device__ __forceinline__ Q4Thread q4_thread(int dt) {
  const int w = dt & 255, r = 8 * (w >> 4) + (w & 7), p = (w >> 3) & 1;
  const int i = r >> 4, rr = r & 15, g = rr & 7, hrow = rr >> 3;
  Q4Thread t;
  t.hdr = (uint32_t)(i * GemmFmt<FMT_Q4K>::GB + 16 * rr);
  t.q = (uint32_t)(i * GemmFmt<FMT_Q4K>::GB + 256 + (2 * hrow + p) * 512 + (4 * g) * 16);
  t.st[0] = sw_off(r, 16 * p);
  t.st[1] = sw_off(r, 16 * p + 8);
  t.st[2] = sw_off(r, 32 + 16 * p);
  t.st[3] = sw_off(r, 32 + 16 * p + 8);
  return t;
}

__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t m, uint32_t c, int) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(m), "r"(c));
  return d;
}

__device__ __forceinline__ void decode_q4k_pair(uint32_t raw_s, int sub, uint32_t a_s, const Q4Thread& t) {
  const uint4 hdr = lds128(raw_s + t.hdr);
  const float d = hbits(hdr.x & 0xFFFFu), dmin = hbits(hdr.x >> 16);
  uint32_t sc0, m0, sc1, m1;
  scale_min_words(2 * sub, hdr.y, hdr.z, hdr.w, sc0, m0);
  scale_min_words(2 * sub + 1, hdr.y, hdr.z, hdr.w, sc1, m1);
  const __half2 dl = h2_const(d * (float)sc0), nl = h2_const(-(dmin * (float)m0));
  const __half2 dh = h2_const(d * (float)sc1), nh = h2_const(-(dmin * (float)m1));
  const __half2 k1024 = h2_const(1024.0f);
  const uint4 q = lds128(raw_s + t.q + 16u * (uint32_t)sub);
  const uint32_t wd[4] = {q.x, q.y, q.z, q.w};
  constexpr uint32_t M = 0x000F000Fu, C = 0x64006400u;
  uint32_t lo[8], hi[8];
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const uint32_t x = wd[w], x4 = x >> 4, x8 = x >> 8, x12 = x >> 12;
    lo[2 * w] = h2_bits(__hfma2(dl, __hsub2(bits_h2(lop_and_or(x, M, C, 0)), k1024), nl));
    lo[2 * w + 1] = h2_bits(__hfma2(dl, __hsub2(bits_h2(lop_and_or(x8, M, C, 0)), k1024), nl));
    hi[2 * w] = h2_bits(__hfma2(dh, __hsub2(bits_h2(lop_and_or(x4, M, C, 0)), k1024), nh));
    hi[2 * w + 1] = h2_bits(__hfma2(dh, __hsub2(bits_h2(lop_and_or(x12, M, C, 0)), k1024), nh));
  }
  sts128(a_s + t.st[0], lo[0], lo[1], lo[2], lo[3]);
  sts128(a_s + t.st[1], lo[4], lo[5], lo[6], lo[7]);
  sts128(a_s + t.st[2], hi[0], hi[1], hi[2], hi[3]);
  sts128(a_s + t.st[3], hi[4], hi[5], hi[6], hi[7]);
}

// FP8 (W8A8): the stage's eight groups move unit by unit (16 E4M3 codes = 16 bytes) from
// the lane-owned group layout (rtd_layout.h: pass p, lane 4g + t -> row g + 8 (p >= 2),
// codes 32t + 16 (p & 1) ..) into the 128-byte swizzled K-major tile, unchanged.
template <int NTH>
__device__ __forceinline__ void copy_stage_f8(uint32_t raw_s, uint32_t a_s, int dt) {
#pragma unroll
  for (int u = dt; u < 1024; u += NTH) {
    const int i = u >> 7, w = u & 127, p = w >> 5, L = w & 31, g = L >> 2, t = L & 3;
    const int r = 16 * i + g + 8 * (p >> 1), c = 2 * t + (p & 1);
    const uint4 v = lds128(raw_s + (uint32_t)(i * 2048 + p * 512 + L * 16));
    sts128(a_s + (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + (((c ^ r) & 7) << 4)), v.x, v.y, v.z, v.w);
  }
}

// Thread dt of the decode warps: with 16 warps it decodes one 16-weight half of a row
// (row r = 8 * (dt / 32) + dt % 8, part = (dt / 8) % 2, half h = (dt / 16) % 2); with 8
// warps both halves of row r = 8 * (dt / 16) + dt % 8.  Eight consecutive threads
// always hold eight consecutive rows with the same k chunk.
template <int FMT, int DW>
__device__ __forceinline__ void decode_stage(uint32_t raw_s, int sub, uint32_t a_s, int dt) {
  if constexpr (Roles<DW>::kHalvesPerThread == 1) {
    decode_half<FMT>(raw_s, sub, a_s, 8 * (dt >> 5) + (dt & 7), (dt >> 3) & 1, (dt >> 4) & 1);
  } else {
#pragma unroll
    for (int h = 0; h < 2; ++h) decode_half<FMT>(raw_s, sub, a_s, 8 * (dt >> 4) + (dt & 7), (dt >> 3) & 1, h);
  }
}

// ---------------------------------------------------------------- GEMM kernel
// Shared-memory plan of one CTA: kRawSlots packed-group buffers (each the eight tiles'
// groups of one k range: three for the 256-element formats, four for the 128-element
// ones, so two groups stay in flight while one is decoded), then as many k stages
// (decoded A tile + activation tile) as the rest of the 227 KB holds, at most 8.
template <int FMT, int TN, int DW>
struct GemmSmem {
  static constexpr int kSmemLimit = Roles<DW>::kSmem;
  static constexpr int kA = kBM * kBK * 2;                  // 16 KB
  static constexpr int kB = TN * kBK * 2;                   // TN * 128
  static constexpr int kRaw = 8 * GemmFmt<FMT>::GB;
  static constexpr int kRawSlots = DW == 8 ? 2 : (GemmFmt<FMT>::GK == 256 ? 3 : 4);
  static constexpr int kFixed = kRawSlots * kRaw + 1024 + 512 + TN * 4;  // + alignment slack, barriers, scales
  static constexpr int kFit = (kSmemLimit - kFixed) / (kA + kB);
  static constexpr int kStages = kFit < kMaxStages ? kFit : kMaxStages;
  static constexpr int offA = 0;
  static constexpr int offB = offA + kStages * kA;
  static constexpr int offRaw = offB + kStages * kB;
  static constexpr int offBar = (offRaw + kRawSlots * kRaw + 127) / 128 * 128;
  static constexpr int nBars = 2 * kRawSlots + 3 * kStages + 1;
  static constexpr int offMisc = offBar + nBars * 8;
  static constexpr int offScale = offMisc + 16;              // the CTA's TN token scales
  static constexpr int bytes = offScale + TN * 4 + 1024;     // + alignment slack
  static_assert(kStages >= (DW == 8 ? 2 : 3), "too few k stages");
  static_assert(bytes <= kSmemLimit, "shared-memory plan exceeds the CTA's share");
};

// The two-CTA plan exists for tile widths whose stages fit 113 KB beside two group slots.
template <int FMT, int TN>
constexpr bool two_cta_ok() {
  constexpr int raw = 2 * 8 * GemmFmt<FMT>::GB + 1024 + 512 + TN * 4;
  return TN <= 64 && (113 * 1024 - raw) / (kBM * kBK * 2 + TN * kBK * 2) >= 2;
}

template <int FMT, int TN, int DW>
__global__ void __launch_bounds__(Roles<DW>::kThreads, Roles<DW>::kCtasPerSm) qgemm_kernel(const GemmArgs a) {
  using L = GemmSmem<FMT, TN, DW>;
  using R = Roles<DW>;
  constexpr int kDecodeWarps = R::kDecodeWarps, kWarpRaw = R::kWarpRaw, kWarpMmaOdd = R::kWarpMmaOdd;
  constexpr int kDecodeThreads = R::kDecodeThreads;
  constexpr bool F8 = FMT == FMT_F8X;
  constexpr int KST = F8 ? 128 : kBK;          // k per stage (a stage is 128 bytes of every row)
  constexpr int SPG = GemmFmt<FMT>::GK / KST;  // stages per group
  constexpr int GB = GemmFmt<FMT>::GB;
  // two accumulators (even / odd k stages, one MMA-issuing thread each), added in the
  // epilogue in a fixed order
  constexpr uint32_t kAccStride = TN < 32 ? 32 : TN;
  constexpr uint32_t kCols = 2 * kAccStride;
  constexpr int kStages = L::kStages, kRawSlots = L::kRawSlots;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the operand tiles
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + L::offBar);
  uint64_t* raw_full = bar;
  uint64_t* raw_empty = bar + kRawSlots;
  uint64_t* b_full = bar + 2 * kRawSlots;
  uint64_t* a_full = b_full + kStages;
  uint64_t* st_empty = a_full + kStages;
  uint64_t* acc_full = st_empty + kStages;
  uint32_t* misc = reinterpret_cast<uint32_t*>(sm + L::offMisc);  // [0] tmem base, [1] abort flag

  const int64_t tile0 = (int64_t)blockIdx.y * 8;           // first 16-row tile of this CTA
  const int64_t t0 = (int64_t)blockIdx.x * TN;             // first token
  // this CTA's k range: whole groups [g_lo, g_hi) of the split blockIdx.z
  const int ngroups = a.nkb / SPG;
  const int g_lo = (int)((int64_t)ngroups * blockIdx.z / a.splits);
  const int g_hi = (int)((int64_t)ngroups * (blockIdx.z + 1) / a.splits);
  const int kb0 = g_lo * SPG;
  const int nkb = (g_hi - g_lo) * SPG;

  if (warp == 0) {
    tmem_alloc(smem_u32(&misc[0]), kCols);
    tmem_relinquish();
  }
  if (tid == 32) {
    for (int s = 0; s < kRawSlots; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], kDecodeWarps);
    }
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&a_full[s], kDecodeWarps);
      mbar_init(&st_empty[s], 1);
    }
    mbar_init(acc_full, 2);  // one commit per MMA-issuing thread
    misc[1] = 0;
    fence_mbar_init();
  }
  float* sscale = reinterpret_cast<float*>(sm + L::offScale);
  pdl_trigger();  // the reduce kernel (or the next call) may launch; it waits for this grid
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc[0];
  volatile uint32_t* abort_flag = &misc[1];

  // The common case -- the phase has already completed -- costs one try_wait; the
  // abort flag and the bounded wait are only consulted when it has not.
  auto wait = [&](uint64_t* b, uint32_t parity) -> bool {
    if (mbar_try_wait(b, parity)) return true;
    if (*abort_flag) return false;
    if (mbar_wait_ns(b, parity, kWaitBudgetNs, a.status)) return true;
    *abort_flag = 1;
    return false;
  };

  if (warp == 0) {
    // ---- activation tiles, one bulk copy per k stage
    if (lane == 0) {
      pdl_wait();  // the staged activations are the prep kernel's output
      const uint8_t* xw = reinterpret_cast<const uint8_t*>(a.xw);
      int stages = 0;  // copies issued so far
      for (int kb = 0; kb < nkb; ++kb) {
        const int st = kb % kStages;
        if (kb >= kStages && !wait(&st_empty[st], (uint32_t)((kb / kStages - 1) & 1))) break;
        mbar_arrive_expect_tx(&b_full[st], (uint32_t)L::kB);
        bulk_g2s(sm + L::offB + st * L::kB, xw + ((size_t)(kb0 + kb) * (a.Mp / 8) + (size_t)(t0 / 8)) * 1024,
                 L::kB, &b_full[st]);
        ++stages;
      }
      if (*abort_flag)  // no copy may still be landing when the CTA exits
        for (int kb = (stages > kStages ? stages - kStages : 0); kb < stages; ++kb)
          mbar_wait_ns(&b_full[kb % kStages], (uint32_t)((kb / kStages) & 1), kWaitBudgetNs, a.status);
    }
  } else if (warp == kWarpRaw) {
    // ---- packed groups of the eight tiles, one slot per k range of one group; runs
    // ahead of the decode by up to kRawSlots groups, independently of the k stages
    if (lane == 0) {
      const int64_t ntile = (a.T - tile0 < 8) ? a.T - tile0 : 8;
      const int ngr = g_hi - g_lo;
      int groups = 0;  // copies issued so far
      for (int s = 0; s < ngr; ++s) {
        const int rs = s % kRawSlots;
        if (s >= kRawSlots && !wait(&raw_empty[rs], (uint32_t)((s / kRawSlots - 1) & 1))) break;
        mbar_arrive_expect_tx(&raw_full[rs], (uint32_t)(ntile * GB));
        for (int64_t i = 0; i < ntile; ++i)
          bulk_g2s(sm + L::offRaw + rs * L::kRaw + i * GB, a.w + ((tile0 + i) * a.G + g_lo + s) * GB, GB,
                   &raw_full[rs]);
        ++groups;
      }
      if (*abort_flag)
        for (int s = (groups > kRawSlots ? groups - kRawSlots : 0); s < groups; ++s)
          mbar_wait_ns(&raw_full[s % kRawSlots], (uint32_t)((s / kRawSlots) & 1), kWaitBudgetNs, a.status);
    }
  } else if (warp == 1 || warp == kWarpMmaOdd) {
    // ---- MMA issuers: warp 1 the even k stages into accumulator 0, warp 19 the odd
    // ones into accumulator 1 (the issue loop of one thread is longer than a stage's
    // MMAs; two threads halve it)
    if (lane == 0) {
      const int par = warp == 1 ? 0 : 1;
      const uint32_t acc = tmem + (uint32_t)par * kAccStride;
      constexpr uint32_t idesc = idesc_f16(TN);
      // descriptors of stage 0; stage st and K slice kk add (st * tile + 32 * kk) / 16
      // to the start-address field (shared addresses stay below 2^18: no carry out)
      const uint64_t da0 = kmajor_desc(smem_u32(sm + L::offA)), db0 = kmajor_desc(smem_u32(sm + L::offB));
      for (int kb = par; kb < nkb; kb += 2) {
        const int st = kb % kStages;
        const uint32_t ph = (uint32_t)((kb / kStages) & 1);
        if (!wait(&b_full[st], ph) || !wait(&a_full[st], ph)) break;
        tc_fence_after();
        const uint64_t da = da0 + (uint64_t)((st * L::kA) >> 4), db = db0 + (uint64_t)((st * L::kB) >> 4);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {  // four K slices of 32 bytes
          if constexpr (F8)
            umma_f8(acc, da + 2 * kk, db + 2 * kk, idesc, (kb > 1 || kk) ? 1u : 0u);
          else
            umma_f16(acc, da + 2 * kk, db + 2 * kk, idesc, (kb > 1 || kk) ? 1u : 0u);
        }
        umma_commit(&st_empty[st]);
      }
      umma_commit(acc_full);  // fires once every MMA this thread issued has completed
    }
  } else {
    // ---- decode warps 2 .. 2 + DW - 1 (and, afterwards, warps 4..7 run the epilogue)
    const int dt = tid - 64;
    const Q4Thread q4t = q4_thread(dt);  // used by the Q4_K part decoder only
    // With sixteen decode warps and four or more stages the warps decode two consecutive
    // stages per iteration (always within one group: SPG is 2 or 4 and kb is even), so the
    // waits, the proxy fence and the arrivals are paid once per pair and the two decodes
    // overlap; eight decode warps take one stage per iteration.
    constexpr int KPI = (DW == 16 && kStages >= 4) ? 2 : 1;
    // Q4_K: one thread per (row, part) and stage -- 256 threads a stage
    constexpr bool kQ4Parts = FMT == FMT_Q4K && kDecodeThreads == 256 * KPI;
    for (int kb = 0; kb < nkb; kb += KPI) {
      bool ok = true;
#pragma unroll
      for (int u = 0; u < KPI; ++u) {
        const int k2 = kb + u, s = k2 / SPG, sub = k2 % SPG, st = k2 % kStages;
        if (ok && sub == 0) ok = wait(&raw_full[s % kRawSlots], (uint32_t)((s / kRawSlots) & 1));
        if (ok && k2 >= kStages) ok = wait(&st_empty[st], (uint32_t)((k2 / kStages - 1) & 1));
      }
      if (!__all_sync(0xffffffffu, ok)) break;  // warp-uniform: the arrivals below are per warp
      if constexpr (F8) {
#pragma unroll
        for (int u = 0; u < KPI; ++u) {
          const int k2 = kb + u;
          copy_stage_f8<kDecodeThreads>(smem_u32(sm + L::offRaw + ((k2 / SPG) % kRawSlots) * L::kRaw),
                                        smem_u32(sm + L::offA + (k2 % kStages) * L::kA), dt);
        }
      } else if constexpr (kQ4Parts) {
        const int k2 = kb + (dt >> 8), s = k2 / SPG;
        decode_q4k_pair(smem_u32(sm + L::offRaw + (s % kRawSlots) * L::kRaw), k2 % SPG,
                        smem_u32(sm + L::offA + (k2 % kStages) * L::kA), q4t);
      } else {
#pragma unroll
        for (int u = 0; u < KPI; ++u) {
          const int k2 = kb + u, s = k2 / SPG;
          decode_stage<FMT, DW>(smem_u32(sm + L::offRaw + (s % kRawSlots) * L::kRaw), k2 % SPG,
                            smem_u32(sm + L::offA + (k2 % kStages) * L::kA), dt);
        }
      }
      fence_async_shared();  // every writer: the tensor cores read A through the async proxy
      __syncwarp();
      if (lane == 0) {  // one arrival per warp: 512 single-thread arrivals would serialise
#pragma unroll
        for (int u = 0; u < KPI; ++u) {
          const int k2 = kb + u, s = k2 / SPG;
          mbar_arrive(&a_full[k2 % kStages]);
          if (k2 % SPG == SPG - 1) mbar_arrive(&raw_empty[s % kRawSlots]);
        }
      }
    }
    if (warp >= 4 && warp < 8) {
      const int q = warp - 4;  // TMEM lanes 32q .. 32q+31 = weight rows of this warp
      pdl_wait();                // the token scales are the prep kernel's output
      for (int i = tid - 128; i < TN; i += 128) sscale[i] = (t0 + i < a.M) ? a.tscale[t0 + i] : 0.0f;
      named_sync(1, 128);        // warps 4..7
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
        float v[16], v1[16];
        tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
        tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + kAccStride + (uint32_t)c0, v1);
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] += v1[j];
        if (!ok || n >= a.N) continue;
        if (a.splits > 1) {  // partial sums of this k split; the reduce kernel finishes them
          float* pp = a.partial + ((size_t)blockIdx.z * a.Mp + (size_t)(t0 + c0)) * a.N + n;
#pragma unroll
          for (int j = 0; j < 16; ++j) pp[(size_t)j * a.N] = v[j];
          continue;
        }
        const int jn = (a.M - (t0 + c0)) < 16 ? (int)(a.M - (t0 + c0)) : 16;  // tokens < M
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
  if (warp == 0) tmem_dealloc(tmem, kCols);
}

// ---------------------------------------------------------------- activation staging
// One block per token row t < Mp: max |x| -> power-of-two scale; the scaled f16 row
// goes to the swizzled layout [kb][Mp/8][8 rows x 128 bytes]; tokens past M
// and k past K are zero.  W8A8 rounds x with the reference E4M3 encoder first.
// The row is read once in 8-element units (one 16-byte load each for 16-bit input,
// two for f32) that stay in registers between the max and the conversion (up to
// kUnits per thread: K <= 32768 for 16-bit input, 16384 for f32); units past that
// are read a second time.
template <int XDT>
struct PrepUnit {
  static constexpr int NR = XDT == 0 ? 2 : 1;            // 16-byte words per 8 elements
  static constexpr int kUnits = XDT == 0 ? 8 : 16;       // units a thread holds
  uint4 r[NR];
};

template <int XDT>
__device__ __forceinline__ void prep_load(const void* x, int64_t row, int64_t k, int64_t K, bool vec,
                                          PrepUnit<XDT>& u) {
  constexpr int ES = XDT == 0 ? 4 : 2;
  if (vec && k + 8 <= K) {
    const uint4* p = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(x) + (row + k) * ES);
#pragma unroll
    for (int i = 0; i < PrepUnit<XDT>::NR; ++i) u.r[i] = __ldg(p + i);
    return;
  }
  uint32_t w[4 * PrepUnit<XDT>::NR];
#pragma unroll
  for (int i = 0; i < 4 * PrepUnit<XDT>::NR; ++i) w[i] = 0;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    if (k + e < K) {
      if (XDT == 0) {
        w[e] = __ldg(static_cast<const uint32_t*>(x) + row + k + e);
      } else {
        const uint32_t b = __ldg(static_cast<const unsigned short*>(x) + row + k + e);
        w[e >> 1] |= b << (16 * (e & 1));
      }
    }
  }
#pragma unroll
  for (int i = 0; i < PrepUnit<XDT>::NR; ++i) u.r[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
}

template <int XDT, bool W8A8>
__device__ __forceinline__ void prep_values(const PrepUnit<XDT>& u, float (&v)[8]) {
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const uint4 q = u.r[XDT == 0 ? (e >> 2) : 0];
    const uint32_t wd = XDT == 0 ? (&q.x)[e & 3] : (&q.x)[e >> 1];
    float f;
    if (XDT == 0)
      f = __uint_as_float(wd);
    else {
      const uint32_t b = (wd >> (16 * (e & 1))) & 0xFFFFu;
      f = XDT == 1 ? __half2float(__ushort_as_half((unsigned short)b)) : __uint_as_float(b << 16);
    }
    if constexpr (W8A8) f = e4m3_round_ref(f);
    v[e] = f;
  }
}

template <int XDT, bool W8A8, bool Q4PERM>
__global__ void __launch_bounds__(kPrepThreadsG) gemm_prep_kernel(const void* x, int64_t ldx, int64_t M, int64_t Mp,
                                                                  int64_t K, int64_t kp, bool vec, __half* xw,
                                                                  float* tscale) {
  using U = PrepUnit<XDT>;
  pdl_trigger();
  pdl_wait();  // x may be the previous kernel's output
  const int64_t t = blockIdx.x;
  const int64_t units = kp / 8, row = t * ldx;
  const bool live = t < M;
  // units held by this thread: threadIdx.x + j * kPrepThreadsG for j < nh
  const int64_t mine = units > threadIdx.x ? (units - 1 - threadIdx.x) / kPrepThreadsG + 1 : 0;
  const int nh = (int)(mine < U::kUnits ? mine : U::kUnits);
  __shared__ float red[kPrepThreadsG / 32];
  U held[U::kUnits];
#pragma unroll
  for (int j = 0; j < U::kUnits; ++j) {
#pragma unroll
    for (int i = 0; i < U::NR; ++i) held[j].r[i] = make_uint4(0u, 0u, 0u, 0u);
    if (live && j < nh) prep_load<XDT>(x, row, 8 * (threadIdx.x + (int64_t)j * kPrepThreadsG), K, vec, held[j]);
  }
  float m = 0.0f;
#pragma unroll
  for (int j = 0; j < U::kUnits; ++j) {
    if (live && j < nh) {
      float v[8];
      prep_values<XDT, W8A8>(held[j], v);
#pragma unroll
      for (int e = 0; e < 8; ++e) m = fmaxf(m, fabsf(v[e]));
    }
  }
  for (int64_t u = threadIdx.x + (int64_t)U::kUnits * kPrepThreadsG; live && u < units; u += kPrepThreadsG) {
    U p;
    prep_load<XDT>(x, row, 8 * u, K, vec, p);
    float v[8];
    prep_values<XDT, W8A8>(p, v);
#pragma unroll
    for (int e = 0; e < 8; ++e) m = fmaxf(m, fabsf(v[e]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  float mm = 0.0f;
#pragma unroll
  for (int w = 0; w < kPrepThreadsG / 32; ++w) mm = fmaxf(mm, red[w]);
  int e = 0;
  if (mm > 0.0f && mm <= 3.4e38f) e = min(max(ilogbf(mm) - 14, -110), 110);
  const float inv = ldexpf(1.0f, -e);
  if (threadIdx.x == 0) tscale[t] = ldexpf(1.0f, e);
  const int64_t tg = t >> 3, r = t & 7;
  auto store = [&](int64_t u, const U& p) {
    float v[8];
    prep_values<XDT, W8A8>(p, v);
    const int64_t kb = u / 8, kc = u % 8;
    uint8_t* dst = reinterpret_cast<uint8_t*>(xw) + ((size_t)kb * (Mp / 8) + (size_t)tg) * 1024 + (size_t)r * 128 +
                   (size_t)((kc ^ r) & 7) * 16;
    if constexpr (Q4PERM)  // Q4_K's decoder pairs elements (0, 2), (1, 3), (4, 6), (5, 7)
      *reinterpret_cast<uint4*>(dst) = make_uint4(pack_f16x2(v[0] * inv, v[2] * inv), pack_f16x2(v[1] * inv, v[3] * inv),
                                                  pack_f16x2(v[4] * inv, v[6] * inv), pack_f16x2(v[5] * inv, v[7] * inv));
    else
      *reinterpret_cast<uint4*>(dst) = make_uint4(pack_f16x2(v[0] * inv, v[1] * inv), pack_f16x2(v[2] * inv, v[3] * inv),
                                                  pack_f16x2(v[4] * inv, v[5] * inv), pack_f16x2(v[6] * inv, v[7] * inv));
  };
#pragma unroll
  for (int j = 0; j < U::kUnits; ++j)
    if (j < nh) store(threadIdx.x + (int64_t)j * kPrepThreadsG, held[j]);
  for (int64_t u = threadIdx.x + (int64_t)U::kUnits * kPrepThreadsG; u < units; u += kPrepThreadsG) {
    U p;
#pragma unroll
    for (int i = 0; i < U::NR; ++i) p.r[i] = make_uint4(0u, 0u, 0u, 0u);
    if (live) prep_load<XDT>(x, row, 8 * u, K, vec, p);
    store(u, p);
  }
}

// W8A8 staging for the kind::f8f6f4 GEMM: every activation becomes the E4M3 code of the
// reference encoder's value (unscaled, ties toward the lower magnitude, saturating at 448:
// fp8_gemm.rs:96-101), 16 codes a unit, in the same swizzled layout as the f16 staging
// (128 bytes of a row per stage); the per-token scale is 1.
template <int XDT>
__global__ void __launch_bounds__(kPrepThreadsG) gemm_prep_f8_kernel(const void* x, int64_t ldx, int64_t M,
                                                                     int64_t Mp, int64_t K, int64_t kp, uint8_t* xw,
                                                                     float* tscale) {
  pdl_trigger();
  pdl_wait();  // x may be the previous kernel's output
  const int64_t t = blockIdx.x;
  if (threadIdx.x == 0) tscale[t] = 1.0f;
  const int64_t units = kp / 16, tg = t >> 3, r = t & 7;
  for (int64_t u = threadIdx.x; u < units; u += kPrepThreadsG) {
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    if (t < M) {
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int64_t k = 16 * u + e;
        float f = 0.0f;
        if (k < K) {
          if (XDT == 0)
            f = __ldg(static_cast<const float*>(x) + t * ldx + k);
          else {
            const unsigned short b = __ldg(static_cast<const unsigned short*>(x) + t * ldx + k);
            f = XDT == 1 ? __half2float(__ushort_as_half(b)) : __uint_as_float((uint32_t)b << 16);
          }
        }
        w[e >> 2] |= (uint32_t)e4m3_code_of_value(e4m3_round_ref(f)) << (8 * (e & 3));
      }
    }
    const int64_t kb = u / 8, c = u % 8;
    uint8_t* dst = xw + ((size_t)kb * (Mp / 8) + (size_t)tg) * 1024 + (size_t)r * 128 + (size_t)((c ^ r) & 7) * 16;
    *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// y[t, n] = sum over splits of the partials, scaled and biased as the GEMM epilogue
// does; four consecutive n per thread (one 16-byte load per split) when N % 4 == 0.
__device__ __forceinline__ void reduce_store(void* y, int y_dtype, int64_t off, float v) {
  if (y_dtype == 0)
    static_cast<float*>(y)[off] = v;
  else if (y_dtype == 1)
    static_cast<__half*>(y)[off] = __float2half_rn(v);
  else
    static_cast<__nv_bfloat16*>(y)[off] = __float2bfloat16_rn(v);
}

__global__ void gemm_reduce_kernel(const float* partial, int splits, int64_t Mp, int64_t M, int64_t N,
                                   const float* tscale, const float* row_scale, int scale_len, const float* bias,
                                   void* y, int y_dtype, int64_t ldy) {
  pdl_trigger();
  pdl_wait();  // the partials are the GEMM's output
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if ((N & 3) == 0) {
    const int64_t n4 = N / 4, total = M * n4;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
      const int64_t t = i / n4, n = 4 * (i - t * n4);
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int z = 0; z < splits; ++z) {
        const float4 p = __ldg(reinterpret_cast<const float4*>(partial + ((size_t)z * Mp + (size_t)t) * N + n));
        acc.x += p.x;
        acc.y += p.y;
        acc.z += p.z;
        acc.w += p.w;
      }
      const float ts = tscale[t];
      float v[4] = {acc.x * ts, acc.y * ts, acc.z * ts, acc.w * ts};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (row_scale) v[j] *= row_scale[scale_len == 1 ? 0 : n + j];
        if (bias) v[j] += bias[n + j];
        reduce_store(y, y_dtype, t * ldy + n + j, v[j]);
      }
    }
    return;
  }
  const int64_t total = M * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t t = i / N, n = i - t * N;
    float v = 0.0f;
    for (int z = 0; z < splits; ++z) v += partial[((size_t)z * Mp + (size_t)t) * N + n];
    v *= tscale[t];
    if (row_scale) v *= row_scale[scale_len == 1 ? 0 : n];
    if (bias) v += bias[n];
    reduce_store(y, y_dtype, t * ldy + n, v);
  }
}

template <int FMT, int TN, int DW>
cudaError_t launch_gemm_tn(const GemmArgs& a, cudaStream_t st) {
  using L = GemmSmem<FMT, TN, DW>;
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev & 63]) {
    cudaError_t e =
        cudaFuncSetAttribute(qgemm_kernel<FMT, TN, DW>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::bytes);
    if (e != cudaSuccess) return e;
    configured[dev & 63] = 1;
  }
  const dim3 grid((unsigned)(a.Mp / TN), (unsigned)((a.T + 7) / 8), (unsigned)a.splits);
  return launch_pdl(qgemm_kernel<FMT, TN, DW>, grid, dim3(Roles<DW>::kThreads), (size_t)L::bytes, st, a);
}

template <int FMT, int TN>
cudaError_t launch_gemm_dw(const GemmArgs& a, int dw, cudaStream_t st) {
  if constexpr (two_cta_ok<FMT, TN>()) {
    if (dw == 8) return launch_gemm_tn<FMT, TN, 8>(a, st);
  }
  return launch_gemm_tn<FMT, TN, 16>(a, st);
}

template <int FMT>
cudaError_t launch_gemm_fmt(const GemmArgs& a, int TN, int dw, cudaStream_t st) {
  switch (TN) {
    case 16: return launch_gemm_dw<FMT, 16>(a, dw, st);
    case 32: return launch_gemm_dw<FMT, 32>(a, dw, st);
    case 64: return launch_gemm_dw<FMT, 64>(a, dw, st);
    case 128: return launch_gemm_dw<FMT, 128>(a, dw, st);
    default: return launch_gemm_dw<FMT, 256>(a, dw, st);
  }
}

template <int FMT>
bool two_cta_fmt(int TN) {
  switch (TN) {
    case 16: return two_cta_ok<FMT, 16>();
    case 32: return two_cta_ok<FMT, 32>();
    case 64: return two_cta_ok<FMT, 64>();
    default: return false;
  }
}

bool two_cta_possible(int fmt, int TN) {
  switch (fmt) {
    case FMT_Q4K: return two_cta_fmt<FMT_Q4K>(TN);
    case FMT_Q6K: return two_cta_fmt<FMT_Q6K>(TN);
    case FMT_Q80: return two_cta_fmt<FMT_Q80>(TN);
    case FMT_F8X: return two_cta_fmt<FMT_F8X>(TN);
    default: return two_cta_fmt<FMT_FP8>(TN);
  }
}

// The GEMM's format of a call: FP8 weights with W8A8 activations take the kind::f8f6f4 path.
int gemm_fmt(const QGemvCall& c) { return (c.fmt == FMT_FP8 && c.w8a8) ? FMT_F8X : c.fmt; }
// k elements of a 128-byte stage row
int gemm_kst(int gfmt) { return gfmt == FMT_F8X ? 128 : kBK; }

// Tile width and K splits from a cost model of one launch (one CTA per SM fits in
// shared memory, so CTAs run in waves of sm_count): a k stage costs the longer of its
// four MMAs (128 x TN x 16 each, about TN / 2 cycles) and the decode of its 8192
// weights by 256 threads; every CTA pays a pipeline fill and epilogue; a split launch
// adds the reduce kernel's traffic.  The candidate with the fewest estimated cycles
// wins (ties: fewer splits, then the wider tile).
struct GemmPlan {
  int TN, splits, dw;
  bool ts;   // the skinny kernel of rtd_gemm_ts.cu (decoded weights in tensor memory)
  int ctas;  // its persistent grid
  int64_t Mp, kp;
  size_t xw_bytes, partial_bytes;
};

constexpr double kDecodeStageCycles = 450.0;
constexpr double kCtaFixedCycles = 4000.0;
constexpr double kReduceFixedCycles = 3000.0;
constexpr double kCyclesPerReduceByte = 1.9e9 / 3.0e12;  // ~3 TB/s at ~1.9 GHz
// a stage of an eight-decode-warp CTA that shares its SM with a second one takes this much
// longer than a stage of the sixteen-warp CTA alone on its SM
constexpr double kTwoCtaStageFactor = 1.6;
constexpr double kCopyStageCycles = 150.0;

// The skinny kernel (up to 64 tokens): a persistent grid of one CTA per SM shares the
// (row tile x group) units evenly, so there is no tile, split or wave to choose.
GemmPlan gemm_plan_ts(const QGemvCall& c, int gfmt) {
  // persistent stream-K: one CTA per SM, each with at least kTsMinUnits groups
  constexpr int64_t kTsMinUnits = 4;
  const FmtInfo f = fmt_info(c.fmt);
  const int TN = c.M <= 16 ? 16 : c.M <= 32 ? 32 : 64;
  const int64_t R = (tiles_for(c.N) + 7) / 8, U = R * c.G;
  const int64_t sms = c.sm_count > 0 ? c.sm_count : 148;
  GemmPlan best{};
  best.TN = TN;
  best.splits = 1;
  best.dw = 16;
  best.ts = true;
  best.ctas = (int)std::max<int64_t>(1, std::min<int64_t>(sms, U / kTsMinUnits));
  best.Mp = TN;
  best.kp = c.G * f.gk;
  best.xw_bytes = (size_t)best.Mp * (size_t)best.kp * (gfmt == FMT_F8X ? 1 : 2);
  best.partial_bytes = ts_partial_floats(best.ctas, TN) * 4;
  return best;
}

GemmPlan gemm_plan(const QGemvCall& c) {
  static const int env_ts = [] {  // RTD_GEMM_TS=0 keeps skinny calls on the shared-memory GEMM
    const char* s = std::getenv("RTD_GEMM_TS");
    return s ? std::atoi(s) : 1;
  }();
  // (W8A8 rounding of f16-staged activations is the shared-memory kernel's; FP8 W8A8 runs
  // kind::f8f6f4 on either kernel)
  // (its unit indices are 32-bit)
  if (env_ts != 0 && c.M <= 64 && (!c.w8a8 || gemm_fmt(c) == FMT_F8X) &&
      (tiles_for(c.N) + 7) / 8 * c.G < (int64_t(1) << 30))
    return gemm_plan_ts(c, gemm_fmt(c));
  static const int env_dw = [] {  // tuning override: RTD_GEMM_DW=8|16
    const char* s = std::getenv("RTD_GEMM_DW");
    const int v = s ? std::atoi(s) : 0;
    return (v == 8 || v == 16) ? v : 0;
  }();
  const FmtInfo f = fmt_info(c.fmt);
  const int gfmt = gemm_fmt(c);
  const int spg = f.gk / gemm_kst(gfmt);
  const int64_t rowctas = (tiles_for(c.N) + 7) / 8;
  const int64_t sms = c.sm_count > 0 ? c.sm_count : 148;
  GemmPlan best{};
  double best_cyc = -1.0;
  for (int TN = 16; TN <= 256; TN *= 2) {
    if (TN > 16 && TN / 2 >= c.M) break;  // a narrower tile already covers every token
    const int64_t colctas = (c.M + TN - 1) / TN;
    if (colctas > 65535) continue;
    const int64_t Mp = colctas * TN;
    const int64_t most = std::max<int64_t>(1, std::min<int64_t>(16, c.G / 2));
    for (int dw : {16, 8}) {
      if (dw == 8 && !two_cta_possible(gfmt, TN)) continue;
      if (env_dw && dw != env_dw && !(env_dw == 8 && !two_cta_possible(gfmt, TN))) continue;
      const int64_t slots = sms * (dw == 8 ? 2 : 1);
      // a kind::f8f6f4 stage moves units instead of decoding them
      const double work = gfmt == FMT_F8X ? kCopyStageCycles : kDecodeStageCycles;
      const double stage = std::max(2.0 * TN, work) * (dw == 8 ? kTwoCtaStageFactor : 1.0);
      for (int64_t s = 1; s <= most; ++s) {
        const int64_t ctas = colctas * rowctas * s;
        const int64_t waves = (ctas + slots - 1) / slots;
        const int64_t stages = ((c.G + s - 1) / s) * spg;
        double cyc = (double)waves * ((double)stages * stage + kCtaFixedCycles);
        if (s > 1) cyc += kReduceFixedCycles + kCyclesPerReduceByte * (double)(s * Mp * c.N * 4 + c.M * c.N * 4);
        if (best_cyc < 0.0 || cyc < best_cyc * 0.98) {
          best_cyc = cyc;
          best.TN = TN;
          best.splits = (int)s;
          best.dw = dw;
          best.Mp = Mp;
        }
      }
    }
  }
  best.kp = c.G * f.gk;
  best.xw_bytes = (size_t)best.Mp * (size_t)best.kp * (gfmt == FMT_F8X ? 1 : 2);
  best.partial_bytes = best.splits > 1 ? (size_t)best.splits * (size_t)best.Mp * (size_t)c.N * 4 : 0;
  return best;
}

}  // namespace

size_t qgemm_workspace_bytes(const QGemvCall& c) {
  const GemmPlan p = gemm_plan(c);
  return p.xw_bytes + (((size_t)p.Mp * 4 + 255) / 256) * 256 + p.partial_bytes + 512;
}

cudaError_t launch_qgemm(const QGemvCall& c, int* plan_error) {
  *plan_error = 0;
  if (c.M <= 0 || c.N <= 0) return cudaSuccess;
  const GemmPlan p = gemm_plan(c);
  const int TN = p.TN;
  const int64_t Mp = p.Mp, kp = p.kp;
  if (TN == 0 || qgemm_workspace_bytes(c) > c.ws_bytes) {
    *plan_error = 1;
    return cudaSuccess;
  }
  uint8_t* ws = reinterpret_cast<uint8_t*>(c.ws);
  __half* xw = reinterpret_cast<__half*>(ws);
  float* tscale = reinterpret_cast<float*>(ws + p.xw_bytes);
  float* partial = reinterpret_cast<float*>(ws + p.xw_bytes + (((size_t)Mp * 4 + 255) / 256) * 256);
  const int es = c.x_dtype == 0 ? 4 : 2;
  const bool vec = (reinterpret_cast<uintptr_t>(c.x) % 16 == 0) && ((c.ldx * es) % 16 == 0);
  const dim3 pg((unsigned)Mp), pb(kPrepThreadsG);
  cudaError_t e;
  auto prep = [&](auto xdt, auto w8a8, auto perm) {
    return launch_pdl(gemm_prep_kernel<decltype(xdt)::value, decltype(w8a8)::value, decltype(perm)::value>, pg, pb, 0,
                      c.stream, c.x, c.ldx, c.M, Mp, c.K, kp, vec, xw, tscale);
  };
  using T0 = std::integral_constant<int, 0>;
  using T1 = std::integral_constant<int, 1>;
  using T2 = std::integral_constant<int, 2>;
  using Yes = std::true_type;
  using No = std::false_type;
  const int gfmt = gemm_fmt(c);
  if (p.ts) {  // the decoder's k order (rtd_gemm_ts.cu)
    e = launch_ts_prep(c, gfmt, Mp, kp, xw, tscale);
  } else if (gfmt == FMT_F8X) {  // E4M3 codes for the kind::f8f6f4 path
    uint8_t* x8 = reinterpret_cast<uint8_t*>(xw);
    e = c.x_dtype == 0   ? launch_pdl(gemm_prep_f8_kernel<0>, pg, pb, 0, c.stream, c.x, c.ldx, c.M, Mp, c.K, kp, x8, tscale)
        : c.x_dtype == 1 ? launch_pdl(gemm_prep_f8_kernel<1>, pg, pb, 0, c.stream, c.x, c.ldx, c.M, Mp, c.K, kp, x8, tscale)
                         : launch_pdl(gemm_prep_f8_kernel<2>, pg, pb, 0, c.stream, c.x, c.ldx, c.M, Mp, c.K, kp, x8, tscale);
  } else if (c.fmt == FMT_Q4K) {  // Q4_K takes no W8A8 (an FP8-only mode)
    e = c.x_dtype == 0 ? prep(T0{}, No{}, Yes{}) : c.x_dtype == 1 ? prep(T1{}, No{}, Yes{}) : prep(T2{}, No{}, Yes{});
  } else if (c.w8a8) {
    e = c.x_dtype == 0 ? prep(T0{}, Yes{}, No{}) : c.x_dtype == 1 ? prep(T1{}, Yes{}, No{}) : prep(T2{}, Yes{}, No{});
  } else {
    e = c.x_dtype == 0 ? prep(T0{}, No{}, No{}) : c.x_dtype == 1 ? prep(T1{}, No{}, No{}) : prep(T2{}, No{}, No{});
  }
  if (e != cudaSuccess) return e;
  if (p.ts) {
    TsGemm g{};
    g.fmt = gfmt;
    g.w = c.w;
    g.row_scale = c.row_scale;
    g.scale_len = c.scale_len;
    g.wpow2 = c.wpow2 > 0.0f ? c.wpow2 : 16777216.0f;
    g.N = c.N;
    g.T = tiles_for(c.N);
    g.G = c.G;
    g.R = (g.T + 7) / 8;
    g.M = c.M;
    g.Mp = Mp;
    g.TN = TN;
    g.ctas = p.ctas;
    g.xw = xw;
    g.tscale = tscale;
    g.bias = c.bias;
    g.y = c.y;
    g.y_dtype = c.y_dtype;
    g.ldy = c.ldy;
    g.status = c.status;
    g.partial = partial;
    e = launch_ts_gemm(g, c.stream);
  } else {
  GemmArgs a{};
  a.w = c.w;
  a.row_scale = c.row_scale;
  a.scale_len = c.scale_len;
  a.N = c.N;
  a.T = tiles_for(c.N);
  a.G = c.G;
  a.nkb = (int)(kp / gemm_kst(gfmt));
  a.xw = xw;
  a.tscale = tscale;
  a.M = c.M;
  a.Mp = Mp;
  a.bias = c.bias;
  a.y = c.y;
  a.y_dtype = c.y_dtype;
  a.ldy = c.ldy;
  a.status = c.status;
  a.splits = p.splits;
  a.partial = partial;
  switch (c.fmt) {
    case FMT_Q4K: e = launch_gemm_fmt<FMT_Q4K>(a, TN, p.dw, c.stream); break;
    case FMT_Q6K: e = launch_gemm_fmt<FMT_Q6K>(a, TN, p.dw, c.stream); break;
    case FMT_Q80: e = launch_gemm_fmt<FMT_Q80>(a, TN, p.dw, c.stream); break;
    default:
      e = gfmt == FMT_F8X ? launch_gemm_fmt<FMT_F8X>(a, TN, p.dw, c.stream)
                          : launch_gemm_fmt<FMT_FP8>(a, TN, p.dw, c.stream);
      break;
  }
  }
  if (e != cudaSuccess || p.splits == 1) return e;
  const int64_t total = (c.N % 4 == 0) ? c.M * c.N / 4 : c.M * c.N;
  const unsigned blocks = (unsigned)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, 8 * (int64_t)c.sm_count));
  return launch_pdl(gemm_reduce_kernel, dim3(blocks), dim3(256), 0, c.stream, (const float*)partial, p.splits, Mp,
                    c.M, c.N, (const float*)tscale, (const float*)c.row_scale,
                    c.scale_len, c.bias, c.y, c.y_dtype, c.ldy);
}

}  // namespace rtd
