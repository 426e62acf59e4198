// rtd_gemv.cu -- decode GEMV on quantized weights, sm_100a.
//
//   y[M, N] = x[M, K] . W^T (+ bias)     W in Q4_K / Q6_K / Q8_0 / FP8-E4M3 blocks
//
// Replaces QMatMul::forward behind Weights::linear
// (crates/runtimed-model/src/weights/linear_layer.rs:45-52) for decode-sized M (up to
// three tokens a call; more run the tensor-core GEMMs), and the per-call cuBLASLt FP8
// GEMM of crates/runtimed-model/src/ops/fp8_gemm.rs:88-191 at those sizes.
//
// Every weight byte is read from HBM exactly once per call; the kernels are built
// to keep HBM busy with as little synchronisation as possible:
//  * Activation staging.  Each group of GK activations gets a power-of-two scale from
//    its own max |x| (warp shuffles, no cross-CTA reduction), is rounded to f16 (f32
//    rows: an f16 hi and an f16 lo column), and is stored transposed into 16-byte
//    units so that the lanes feeding different MMA columns in one load hit distinct
//    banks; a small table per (group, column) holds the per-sub-block column sums the
//    scale algebra needs and the group's scale.  Whole-mode launches with bf16 / f16
//    rows stage x inside every CTA (stage_local_diag, no second launch); the others
//    run prep_diag_kernel first, chained by programmatic dependent launch, and the
//    GEMV bulk-copies the staged units together with the weights.
//  * GEMV kernel: every warp is an independent streaming pipeline.  The flattened
//    (16-row tile, item of IG groups) space is split over all warps of the persistent
//    grid; each warp keeps NS items in flight in its own shared-memory ring with
//    cp.async.bulk on its own mbarriers, so no CTA-wide barrier stalls the stream.  In
//    the device layout (rtd_layout.h) an item is one contiguous 16-byte aligned range.
//    Weight copies are issued before griddepcontrol.wait, so they overlap the previous
//    kernel's tail.
//  * No dequantized weight is materialised.  The 8 columns of each m16n8k16 MMA are
//    the group's SUB-BLOCKS (not tokens): every lane owns whole sub-blocks of two rows
//    (rtd_layout.h), feeds its packed codes to the MMA as exact f16 SUBNORMALS (code
//    bits in the mantissa, value code * 2^-24; one LOP3 or PRMT per pair), and only the
//    lane whose column a sub-block is supplies that sub-block's activations as B.  After
//    a group, C[row][n] is sub-block n's code-weighted dot product alone, so each lane
//    applies the reference's scale algebra for exactly its own (row, sub-block) pairs
//    in f32 (Q4_K: d*sc on the codes and -dmin*m on the column sums; Q6_K / Q8_0: the
//    code bias 32 / 128 enters as a C-init from the column sums; FP8: E4M3 -> f16 is
//    exact and the channel scale is applied on write).  Products are exact; only f32
//    rounding remains.
//  * Whole mode (enough 16-row tiles for every warp of the grid): a warp owns whole
//    tiles and writes them from its accumulators.  Split mode: the 8 warps of a CTA
//    split each tile's items, leave their partials in shared memory (double buffered,
//    named barriers) and the tile's writer warp sums them in warp order.
//  * Row-parallel tensor parallelism (split mode): the writer warp stores the tile's
//    partial into every rank's exchange buffer over NVLink as LL words (value and
//    epoch in one 8-byte store); after the CTA's last tile it waits (bounded) for
//    every rank's words of its tiles and writes their rank-ordered sum.
//  * Greedy pick (qgemv_kernel<..., true>, the LM head of greedy decode): every output
//    is folded into a packed (value, row) key per token; one atomicMax per CTA and
//    token, and the launch's last CTA writes the ids (the logits need not be written).

#include <algorithm>
#include <cstdlib>

#include "rtd_common.cuh"
#include "rtd_kernels.h"


namespace rtd {

namespace {

constexpr int kWarps = 8;  // warps per GEMV CTA, each an independent pipeline
constexpr int kThreads = kWarps * 32;
constexpr int kPrepThreads = 256;
constexpr int kMaxStages = 4;
constexpr int kTblBytes = 128;   // per-warp epilogue scratch (bias and row scale of a tile)
constexpr int kZeroPage = 512;   // zero B-fragment source for lanes that own no MMA column

template <int FMT>
struct FmtC;
// DIAG formats (the K-quants and Q8_0) use the lane-owned group layouts of
// rtd_layout.h and the sub-block-per-MMA-column decoder (do_group_diag); FP8 keeps
// the token-per-column decoder.  DIAG codes enter the MMA as f16 subnormals (code
// bits in the mantissa, exponent 0: value = code * 2^-24, exact).  XOFF: the
// column-sum table holds XOFF * sum(x) per sub-block -- plain sums for Q4_K's min
// term, and for Q6_K / Q8_0 the C-init that removes the code bias (32, 128) at the
// same 2^-24 scale.
template <>
struct FmtC<FMT_Q4K> {
  static constexpr int GK = 256, GB = 2304, SBE = 32;
  static constexpr float XOFF = 1.0f;
};
template <>
struct FmtC<FMT_Q6K> {
  static constexpr int GK = 256, GB = 3360, SBE = 16;
  static constexpr float XOFF = -0x1p-19f;  // -32 * 2^-24
};
template <>
struct FmtC<FMT_Q80> {
  static constexpr int GK = 128, GB = 2176, SBE = 32;
  static constexpr float XOFF = -0x1p-17f;  // -128 * 2^-24
};
template <>
struct FmtC<FMT_FP8> {
  static constexpr int GK = 128, GB = 2048, SBE = 32;
  static constexpr float XOFF = 0.0f;  // signed E4M3 codes carry no bias; the sums go unused
};

// Bytes one activation column occupies per group in the workspace (and in shared
// memory).  FP8 keeps its natural order; DIAG formats store a group's x as 16-byte
// units (8 elements) transposed to [unit-in-sub-block j][sub-block], so that the
// lanes supplying different sub-blocks in one load hit different banks.
__host__ __device__ constexpr int col_stride_bytes(int gk) { return gk * 2; }

// Destination of natural unit n (elements 8n..8n+7) of a group in the DIAG x order.
template <int FMT>
__host__ __device__ constexpr int diag_unit_offset(int n) {
  constexpr int UPS = FmtC<FMT>::SBE / 8, NSB = FmtC<FMT>::GK / FmtC<FMT>::SBE;
  return (n % UPS) * (NSB * 16) + 16 * (n / UPS);
}

// Q4_K's MMA pairs take elements (4u, 4u+2) and (4u+1, 4u+3) of a sub-block (the two
// 16-bit halves of one 4-byte code word); x is staged in that order.
__device__ __forceinline__ uint4 q4k_quad_order(uint4 u) {
  return make_uint4(__byte_perm(u.x, u.y, 0x5410), __byte_perm(u.x, u.y, 0x7632), __byte_perm(u.z, u.w, 0x5410),
                    __byte_perm(u.z, u.w, 0x7632));
}

// Column-sum table of DIAG formats: per (group, column) TW = GK/SBE + 4 floats --
// XOFF * sum(x) for every sub-block, then the group's activation scale (2^e) at
// index GK/SBE; rows stay 16-byte aligned.
template <int FMT>
__host__ __device__ constexpr int tab_row_floats() {
  return FmtC<FMT>::GK / FmtC<FMT>::SBE + 4;
}

// Power-of-two exponent that maps a group's max |x| into [2^14, 2^15): the staged f16
// values then keep 11 significant bits without overflow; 0 for all-zero or
// non-finite groups (non-finite values then propagate as in the reference).
__device__ __forceinline__ int group_exponent(float amax) {
  if (!(amax > 0.0f) || !(amax <= 3.4e38f)) return 0;
  return min(max(ilogbf(amax) - 14, -110), 110);
}

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

// ------------------------------------------------------------------ prep kernel
struct PrepArgs {
  const void* x;
  int x_dtype;
  int x_vec;
  int64_t ldx;
  int64_t K, kp;
  int M, P, ncol, ncol8;
  int w8a8;
  uint8_t* cols;  // [group][ncol][col_stride_bytes(GK)]
  float* tab;     // [group][ncol][GK / SBE]
  float* tscale;  // [M]
};

__device__ __forceinline__ void load8(const void* x, int dt, bool vec, int64_t ldx, int64_t K, int t, int64_t k,
                                      float (&v)[8]) {
  if (vec && k + 8 <= K) {
    if (dt == 0) {
      const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(x) + (int64_t)t * ldx + k);
      const float4 u = __ldg(p), w = __ldg(p + 1);
      v[0] = u.x; v[1] = u.y; v[2] = u.z; v[3] = u.w; v[4] = w.x; v[5] = w.y; v[6] = w.z; v[7] = w.w;
    } else {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) + (int64_t)t * ldx + k));
      const uint32_t wd[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const unsigned short lo = (unsigned short)(wd[i] & 0xFFFFu), hi = (unsigned short)(wd[i] >> 16);
        if (dt == 1) {
          v[2 * i] = __half2float(__ushort_as_half(lo));
          v[2 * i + 1] = __half2float(__ushort_as_half(hi));
        } else {
          v[2 * i] = __uint_as_float((uint32_t)lo << 16);
          v[2 * i + 1] = __uint_as_float((uint32_t)hi << 16);
        }
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t kk = k + i;
      float f = 0.0f;
      if (kk < K) {
        if (dt == 0) {
          f = static_cast<const float*>(x)[(int64_t)t * ldx + kk];
        } else {
          const unsigned short b = static_cast<const unsigned short*>(x)[(int64_t)t * ldx + kk];
          f = (dt == 1) ? __half2float(__ushort_as_half(b)) : __uint_as_float((uint32_t)b << 16);
        }
      }
      v[i] = f;
    }
  }
}

__device__ __forceinline__ uint32_t pack_h2(__half lo, __half hi) {
  return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}

// Prep for DIAG formats: one warp per (token, group) -- the group's own max |x| sets
// its scale, so no cross-CTA reduction is needed.  Writes the transposed f16 units
// (hi, and for f32 inputs the lo remainder as a second column) and the table rows.
template <int FMT>
__global__ void __launch_bounds__(kPrepThreads) prep_diag_kernel(const PrepArgs a) {
  using F = FmtC<FMT>;
  constexpr int UPG = F::GK / 8, NSB = F::GK / F::SBE, SBC = F::SBE / 8, TW = tab_row_floats<FMT>();
  constexpr int CSB = col_stride_bytes(F::GK);
  griddep_launch_dependents();
  griddep_wait();
  const int t = blockIdx.y;
  const int64_t c = (int64_t)blockIdx.x * kPrepThreads + threadIdx.x;  // chunk of 8 elements
  const int64_t nch = a.kp / 8;
  const bool valid = c < nch;  // kp / 8 is a multiple of UPG: groups never straddle warps
  float v[8];
  if (valid) {
    load8(a.x, a.x_dtype, a.x_vec != 0, a.ldx, a.K, t, 8 * c, v);
    if (a.w8a8) {  // W8A8: activations take the reference E4M3 rounding first
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = e4m3_round_ref(v[i]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.0f;
  }
  float m = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(v[i]));
#pragma unroll
  for (int o = 1; o < UPG; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const int e = group_exponent(m);
  const float inv = ldexpf(1.0f, -e);
  __half hi[8], lo[8];
  float shi = 0.0f, slo = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float sv = v[i] * inv;
    hi[i] = __float2half_rn(sv);
    const float hf = __half2float(hi[i]);
    lo[i] = __float2half_rn(sv - hf);
    shi += hf;
    slo += __half2float(lo[i]);
  }
#pragma unroll
  for (int o = 1; o < SBC; o <<= 1) {
    shi += __shfl_xor_sync(0xffffffffu, shi, o);
    slo += __shfl_xor_sync(0xffffffffu, slo, o);
  }
  if (!valid) return;
  const int64_t grp = c / UPG;
  const int n = (int)(c - grp * UPG);
  uint8_t* base = a.cols + ((size_t)grp * a.ncol + (size_t)t * a.P) * CSB + diag_unit_offset<FMT>(n);
  uint4 u;
  u.x = pack_h2(hi[0], hi[1]); u.y = pack_h2(hi[2], hi[3]);
  u.z = pack_h2(hi[4], hi[5]); u.w = pack_h2(hi[6], hi[7]);
  if constexpr (FMT == FMT_Q4K) u = q4k_quad_order(u);
  *reinterpret_cast<uint4*>(base) = u;
  if (a.P == 2) {
    u.x = pack_h2(lo[0], lo[1]); u.y = pack_h2(lo[2], lo[3]);
    u.z = pack_h2(lo[4], lo[5]); u.w = pack_h2(lo[6], lo[7]);
    if constexpr (FMT == FMT_Q4K) u = q4k_quad_order(u);
    *reinterpret_cast<uint4*>(base + CSB) = u;
  }
  float* tp = a.tab + ((size_t)grp * a.ncol + (size_t)t * a.P) * TW;
  if (n % SBC == 0) {
    tp[n / SBC] = shi * F::XOFF;
    if (a.P == 2) tp[TW + n / SBC] = slo * F::XOFF;
  }
  if (n == 0) {
    const float sc = ldexpf(1.0f, e);
    tp[NSB] = sc;
    if (a.P == 2) tp[TW + NSB] = sc;
  }
}

// ------------------------------------------------------------------ GEMV kernel
// 32-bit shared-memory accessors.  They are volatile so no load can be hoisted
// above the mbarrier wait that publishes the data; ALU work still interleaves.
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ float2 ldsf2(uint32_t a) {
  float2 v;
  asm volatile("ld.shared.v2.f32 {%0,%1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ float ldsf(uint32_t a) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ float h2f(uint32_t bits16) { return __half2float(__ushort_as_half((unsigned short)bits16)); }

// Loads at base + a compile-time offset (folded into the instruction's address).
template <int OFF>
__device__ __forceinline__ uint4 lds128o(uint32_t base) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4+%5];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(base), "n"(OFF));
  return v;
}
template <int OFF>
__device__ __forceinline__ float4 ldsf4o(uint32_t base) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4+%5];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(base), "n"(OFF));
  return v;
}
template <int OFF>
__device__ __forceinline__ float2 ldsf2o(uint32_t base) {
  float2 v;
  asm volatile("ld.shared.v2.f32 {%0,%1}, [%2+%3];" : "=f"(v.x), "=f"(v.y) : "r"(base), "n"(OFF));
  return v;
}
template <int OFF>
__device__ __forceinline__ uint2 lds64o(uint32_t base) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2+%3];" : "=r"(v.x), "=r"(v.y) : "r"(base), "n"(OFF));
  return v;
}
template <int OFF>
__device__ __forceinline__ float ldsfo(uint32_t base) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1+%2];" : "=f"(v) : "r"(base), "n"(OFF));
  return v;
}

// (a & b) | c in one LOP3.
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

template <int V>
struct IC {
  static constexpr int value = V;
};
// f(IC<0>{}), ..., f(IC<N-1>{}): a loop whose index is a constant expression.
template <int I, int N, typename Fn>
__device__ __forceinline__ void static_for(Fn&& f) {
  if constexpr (I < N) {
    f(IC<I>{});
    static_for<I + 1, N>(f);
  }
}

__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}

// The float with bits 0x4B0000XX is 2^23 + XX.  Used through an FMA the 2^23 drops
// out exactly: fmaf(s, 2^23 + XX, -2^23 * s) == s * XX, rounded once.
__device__ __forceinline__ float magic_f(uint32_t bits) { return __uint_as_float(bits); }
constexpr float kMagic = 8388608.0f;  // 2^23

// Sub-block factors of one Q4_K row for the two sub-blocks a lane owns (2t, 2t+1):
// Ea = d*sc_a*2^24 (low nibbles enter the MMA as q * 2^-24), Eb = d*sc_b*2^20 (high
// nibbles as 16q * 2^-24), Fa/b = -dmin*m (times the plain column sums).
// Header h = (d | dmin << 16, scales[0..3], scales[4..7], scales[8..11]), dequant_k.rs:8-16.
__device__ __forceinline__ void q4k_row_factors(uint4 h, bool hiq, uint32_t selA, uint32_t selB, float& Ea,
                                                float& Eb, float& Fa, float& Fb) {
  const uint32_t sc4 = hiq ? and_or(h.w, 0x0F0F0F0Fu, (h.y >> 2) & 0x30303030u) : (h.y & 0x3F3F3F3Fu);
  const uint32_t m4 = hiq ? and_or(h.w >> 4, 0x0F0F0F0Fu, (h.z >> 2) & 0x30303030u) : (h.z & 0x3F3F3F3Fu);
  const float D = h2f(h.x & 0xFFFFu), Dm = h2f(h.x >> 16);
  const float Da = D * 0x1p24f, Db = D * 0x1p20f;
  constexpr uint32_t MG = 0x4B000000u;
  Ea = fmaf(Da, magic_f(prmt(sc4, MG, selA)), -kMagic * Da);
  Eb = fmaf(Db, magic_f(prmt(sc4, MG, selB)), -kMagic * Db);
  Fa = fmaf(-Dm, magic_f(prmt(m4, MG, selA)), kMagic * Dm);
  Fb = fmaf(-Dm, magic_f(prmt(m4, MG, selB)), kMagic * Dm);
}

// One group of a DIAG format for NC activation columns.
//
// The 8 columns of each m16n8k16 MMA are SUB-BLOCKS, not tokens: lane (g, t) holds
// the A fragments of the sub-blocks it owns (k-slots 2t,2t+1 = its first sub-block,
// 2t+8,2t+9 = its second), and the B fragment of column n is the activation slice of
// sub-block n, supplied only by the lane whose MMA column is n (g == 2t or 2t+1);
// every other lane feeds zeros from a zero page.  After all MMAs of the group,
// C[row][n] is the code-weighted dot product of sub-block n alone (times 2^-24),
// so each lane applies the scales of exactly its own (row, sub-block) pairs -- no
// per-sub-block MMA chains and no shared scale table.
//   gs: group bytes; xs: column 0's x units of this group (column c at xs + c*xcs);
//   ts: table of this group, [column][sub-block] f32; z0 / z1: zero-page pointers for
//   idle b0 / b1 lanes; acc[c][0 / 1]: this lane's partial sums of rows g / g+8.
template <int FMT, int NC>
__device__ __forceinline__ void do_group_diag(uint32_t gs, uint32_t xs, uint32_t xcs, uint32_t ts, uint32_t z0,
                                              uint32_t z1, bool act0, bool act1, float (&acc)[NC][4], int lane) {
  const int g = lane >> 2, tq = lane & 3;
  constexpr int TW = tab_row_floats<FMT>();
  if constexpr (FMT == FMT_Q4K) {
    constexpr int NSB = 8;
    const uint4 hg = lds128(gs + 16 * g), hh = lds128(gs + 16 * (g + 8));
    const uint32_t qb = gs + 256 + lane * 16;
    const uint4 q0 = lds128o<0>(qb), q1 = lds128o<512>(qb), q2 = lds128o<1024>(qb), q3 = lds128o<1536>(qb);
    const bool hiq = tq >= 2;
    const uint32_t selA = 0x7440u | (uint32_t)(2 * (tq & 1)), selB = selA + 1;
    float Ea0, Eb0, Fa0, Fb0, Ea1, Eb1, Fa1, Fb1;
    q4k_row_factors(hg, hiq, selA, selB, Ea0, Eb0, Fa0, Fb0);
    q4k_row_factors(hh, hiq, selA, selB, Ea1, Eb1, Fa1, Fb1);
    const uint32_t wg[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    const uint32_t wh[8] = {q2.x, q2.y, q2.z, q2.w, q3.x, q3.y, q3.z, q3.w};
    uint32_t p0[NC], p1[NC];
    float2 T[NC];
    float S[NC];
    float C[NC][4];
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const uint32_t xc = xs + c * xcs + 32 * tq;
      p0[c] = act0 ? xc : z0;
      p1[c] = act1 ? xc + 16 : z1;
      T[c] = ldsf2(ts + (uint32_t)(c * TW + 2 * tq) * 4);
      S[c] = ldsf(ts + (uint32_t)(c * TW + NSB) * 4);
      C[c][0] = C[c][1] = C[c][2] = C[c][3] = 0.0f;
    }
    // MMA pairs per 4-byte code word u: the low nibbles (sub-block 2t, elements
    // (4u, 4u+2) | (4u+1, 4u+3)) feed MMA column 2t from the b0-lane (g == 2t); the high
    // nibbles (sub-block 2t+1) feed column 2t+1 from the b1-lane.  Each MMA takes both
    // B registers from one 16-byte load.
    static_for<0, 4>([&](auto jI) {
      constexpr int j = decltype(jI)::value;
      uint4 B0[NC], B1[NC];
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        B0[c] = lds128o<128 * j>(p0[c]);
        B1[c] = lds128o<128 * j>(p1[c]);
      }
      static_for<0, 2>([&](auto hI) {
        constexpr int hh = decltype(hI)::value;
        constexpr int u = 2 * j + hh;
        const uint32_t sg = wg[u] >> 8, sh = wh[u] >> 8;
        const uint32_t l0 = wg[u] & 0x000F000Fu, l1 = wh[u] & 0x000F000Fu;
        const uint32_t l2 = sg & 0x000F000Fu, l3 = sh & 0x000F000Fu;
        const uint32_t h0 = wg[u] & 0x00F000F0u, h1 = wh[u] & 0x00F000F0u;
        const uint32_t h2 = sg & 0x00F000F0u, h3 = sh & 0x00F000F0u;
#pragma unroll
        for (int c = 0; c < NC; ++c) {
          const uint32_t x0 = hh ? B0[c].z : B0[c].x, x1 = hh ? B0[c].w : B0[c].y;
          const uint32_t y0 = hh ? B1[c].z : B1[c].x, y1 = hh ? B1[c].w : B1[c].y;
          mma_f16_acc(C[c], l0, l1, l2, l3, x0, x1);
          mma_f16_acc(C[c], h0, h1, h2, h3, y0, y1);
        }
      });
    });
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const float v0 = fmaf(Ea0, C[c][0], fmaf(Eb0, C[c][1], fmaf(Fa0, T[c].x, Fb0 * T[c].y)));
      const float v1 = fmaf(Ea1, C[c][2], fmaf(Eb1, C[c][3], fmaf(Fa1, T[c].x, Fb1 * T[c].y)));
      acc[c][0] = fmaf(S[c], v0, acc[c][0]);
      acc[c][1] = fmaf(S[c], v1, acc[c][1]);
    }
  } else if constexpr (FMT == FMT_Q6K) {
    constexpr int NSB = 16;
    const uint32_t dd = lds32(gs + 4 * g);
    const uint2 scw = lds64(gs + 32 + lane * 8);
    const float dg = h2f(dd & 0xFFFFu) * 0x1p24f, dh = h2f(dd >> 16) * 0x1p24f;
    const uint32_t cb = gs + 288 + lane * 16;
    float V[NC][2], S[NC];
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      V[c][0] = V[c][1] = 0.0f;
      S[c] = ldsf(ts + (uint32_t)(c * TW + NSB) * 4);
    }
    constexpr uint32_t M6 = 0x003F003Fu, M4 = 0x000F000Fu, M2 = 0x00300030u;
    // code pair i (elements 2i, 2i+1 of the sub-block) of one (X, Y, Z) triple
    auto pair = [&](uint32_t X, uint32_t Y, uint32_t Z, int i) -> uint32_t {
      switch (i) {
        case 0: return X & M6;
        case 1: return (X >> 6) & M6;
        case 2: return Y & M6;
        case 3: return (Y >> 6) & M6;
        case 4: return Z & M6;
        case 5: return (Z >> 6) & M6;
        case 6: return lop_and_or(X >> 12, M4, (Z >> 8) & M2);
        default: return lop_and_or(Y >> 12, M4, (Z >> 10) & M2);
      }
    };
    static_for<0, 2>([&](auto hI) {
      constexpr int h = decltype(hI)::value;
      const uint4 v0 = lds128o<(3 * h) * 512>(cb), v1 = lds128o<(3 * h + 1) * 512>(cb),
                  v2 = lds128o<(3 * h + 2) * 512>(cb);
      // triples: (g, a) = v0.xyz, (g+8, a) = v0.w v1.xy, (g, b) = v1.zw v2.x, (g+8, b) = v2.yzw
      const float Ega = dg * (float)(int8_t)((scw.x >> (16 * h)) & 0xFFu);
      const float Egb = dg * (float)(int8_t)((scw.x >> (16 * h + 8)) & 0xFFu);
      const float Eha = dh * (float)(int8_t)((scw.y >> (16 * h)) & 0xFFu);
      const float Ehb = dh * (float)(int8_t)((scw.y >> (16 * h + 8)) & 0xFFu);
      uint32_t p0[NC], p1[NC];
      float Cc[NC][4];
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        const uint32_t xc = xs + c * xcs + 128 * h + 32 * tq;
        p0[c] = act0 ? xc : z0 + 128 * h;
        p1[c] = act1 ? xc + 16 : z1 + 128 * h;
        const float2 T = ldsf2(ts + (uint32_t)(c * TW + 8 * h + 2 * tq) * 4);
        Cc[c][0] = T.x; Cc[c][1] = T.y; Cc[c][2] = T.x; Cc[c][3] = T.y;
      }
      // sub-block a (pairs 2m, 2m+1 of triples (g,a), (g+8,a)) feeds column 2t from the
      // b0-lane, sub-block b feeds column 2t+1 from the b1-lane; one load per MMA's B
      static_for<0, 2>([&](auto jI) {
        constexpr int j = decltype(jI)::value;
        uint4 B0[NC], B1[NC];
#pragma unroll
        for (int c = 0; c < NC; ++c) {
          B0[c] = lds128o<256 * j>(p0[c]);
          B1[c] = lds128o<256 * j>(p1[c]);
        }
        static_for<0, 2>([&](auto mI) {
          constexpr int m = 2 * j + decltype(mI)::value;  // pairs 2m, 2m+1
          const uint32_t a0 = pair(v0.x, v0.y, v0.z, 2 * m), a1 = pair(v0.w, v1.x, v1.y, 2 * m);
          const uint32_t a2 = pair(v0.x, v0.y, v0.z, 2 * m + 1), a3 = pair(v0.w, v1.x, v1.y, 2 * m + 1);
          const uint32_t e0 = pair(v1.z, v1.w, v2.x, 2 * m), e1 = pair(v2.y, v2.z, v2.w, 2 * m);
          const uint32_t e2 = pair(v1.z, v1.w, v2.x, 2 * m + 1), e3 = pair(v2.y, v2.z, v2.w, 2 * m + 1);
#pragma unroll
          for (int c = 0; c < NC; ++c) {
            const bool odd = (m & 1) != 0;
            const uint32_t x0 = odd ? B0[c].z : B0[c].x, x1 = odd ? B0[c].w : B0[c].y;
            const uint32_t y0 = odd ? B1[c].z : B1[c].x, y1 = odd ? B1[c].w : B1[c].y;
            mma_f16_acc(Cc[c], a0, a1, a2, a3, x0, x1);
            mma_f16_acc(Cc[c], e0, e1, e2, e3, y0, y1);
          }
        });
      });
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        V[c][0] = fmaf(Ega, Cc[c][0], fmaf(Egb, Cc[c][1], V[c][0]));
        V[c][1] = fmaf(Eha, Cc[c][2], fmaf(Ehb, Cc[c][3], V[c][1]));
      }
    });
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      acc[c][0] = fmaf(S[c], V[c][0], acc[c][0]);
      acc[c][1] = fmaf(S[c], V[c][1], acc[c][1]);
    }
  } else if constexpr (FMT == FMT_FP8) {
    // lane t owns codes 32t..32t+31 of the group; E4M3 -> f16 is exact, and the
    // per-row scale is applied when the tile is written.  Column 2t as for Q8_0.
    constexpr int NSB = 4;
    const uint32_t qb = gs + lane * 16;
    const uint4 q0 = lds128o<0>(qb), q1 = lds128o<512>(qb), q2 = lds128o<1024>(qb), q3 = lds128o<1536>(qb);
    const uint32_t wg[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    const uint32_t wh[8] = {q2.x, q2.y, q2.z, q2.w, q3.x, q3.y, q3.z, q3.w};
    uint32_t p[NC];
    float S[NC];
    float C[NC][4];
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      p[c] = act0 ? xs + c * xcs + 16 * tq : z0;
      S[c] = ldsf(ts + (uint32_t)(c * TW + NSB) * 4);
      C[c][0] = C[c][1] = C[c][2] = C[c][3] = 0.0f;
    }
    static_for<0, 4>([&](auto jI) {
      constexpr int j = decltype(jI)::value;
      uint4 B[NC];
#pragma unroll
      for (int c = 0; c < NC; ++c) B[c] = lds128o<64 * j>(p[c]);
      static_for<0, 2>([&](auto eI) {
        constexpr int e = decltype(eI)::value;
        constexpr int t = 2 * j + e;
        const uint32_t a0 = e4m3x2_to_f16x2((uint16_t)(wg[t] & 0xFFFFu)), a1 = e4m3x2_to_f16x2((uint16_t)(wh[t] & 0xFFFFu));
        const uint32_t a2 = e4m3x2_to_f16x2((uint16_t)(wg[t] >> 16)), a3 = e4m3x2_to_f16x2((uint16_t)(wh[t] >> 16));
#pragma unroll
        for (int c = 0; c < NC; ++c) {
          const uint32_t b0 = e ? B[c].z : B[c].x, b1 = e ? B[c].w : B[c].y;
          mma_f16_acc(C[c], a0, a1, a2, a3, b0, b1);
        }
      });
    });
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      acc[c][0] = fmaf(S[c], C[c][0], acc[c][0]);
      acc[c][1] = fmaf(S[c], C[c][2], acc[c][1]);
    }
  } else {  // FMT_Q80: lane t owns block t; both k-slot pairs feed MMA column 2t
    constexpr int NSB = 4;
    const uint32_t dd = lds32(gs + 4 * lane);
    const float dg = h2f(dd & 0xFFFFu) * 0x1p24f, dh = h2f(dd >> 16) * 0x1p24f;
    const uint32_t qb = gs + 128 + lane * 16;
    const uint4 q0 = lds128o<0>(qb), q1 = lds128o<512>(qb), q2 = lds128o<1024>(qb), q3 = lds128o<1536>(qb);
    const uint32_t wg[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    const uint32_t wh[8] = {q2.x, q2.y, q2.z, q2.w, q3.x, q3.y, q3.z, q3.w};
    uint32_t p[NC];
    float T[NC], S[NC];
    float C[NC][4];
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      p[c] = act0 ? xs + c * xcs + 16 * tq : z0;
      T[c] = ldsf(ts + (uint32_t)(c * TW + tq) * 4);
      S[c] = ldsf(ts + (uint32_t)(c * TW + NSB) * 4);
      C[c][0] = T[c]; C[c][1] = 0.0f; C[c][2] = T[c]; C[c][3] = 0.0f;
    }
    static_for<0, 4>([&](auto jI) {
      constexpr int j = decltype(jI)::value;
      uint4 B[NC];
#pragma unroll
      for (int c = 0; c < NC; ++c) B[c] = lds128o<64 * j>(p[c]);
      static_for<0, 2>([&](auto eI) {
        constexpr int e = decltype(eI)::value;
        constexpr int t = 2 * j + e;
        const uint32_t ug = wg[t] ^ 0x80808080u, uh = wh[t] ^ 0x80808080u;
        const uint32_t a0 = prmt(ug, 0u, 0x4140), a1 = prmt(uh, 0u, 0x4140);
        const uint32_t a2 = prmt(ug, 0u, 0x4342), a3 = prmt(uh, 0u, 0x4342);
#pragma unroll
        for (int c = 0; c < NC; ++c) {
          const uint32_t b0 = e ? B[c].z : B[c].x, b1 = e ? B[c].w : B[c].y;
          mma_f16_acc(C[c], a0, a1, a2, a3, b0, b1);
        }
      });
    });
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      acc[c][0] = fmaf(dg * S[c], C[c][0], acc[c][0]);
      acc[c][1] = fmaf(dh * S[c], C[c][2], acc[c][1]);
    }
  }
}

struct Args {
  const uint8_t* w;
  const float* row_scale;  // per output row (FP8, INT4 Marlin), or null
  int scale_len;
  const uint8_t* cols;
  const float* tab;
  const float* tscale;
  int M, P, ncol, ncol8;
  const float* bias;
  void* y;
  int64_t ldy;
  int y_dtype;
  int64_t N;
  int G, IG, CI, T;   // groups per row, groups per item, items per tile, tiles
  int nctas, NS;
  int whole;          // 1: every warp owns whole tiles (no cross-warp reduction)
  int warp_bytes, slot_bytes, off_x, off_tab, off_tbl, off_bar, off_red;
  // local-x mode: every CTA stages the raw bf16/f16 activations itself (no prep kernel)
  int local_x;
  const void* xraw;
  int64_t ldx, K, kp;
  int x_dtype, w8a8;
  int off_xloc, xcs, off_tabloc;
  int tabw;      // table floats per group: ncol * (GK / SBE + 4)
  int off_zero;  // kZeroPage bytes of zeros
  // row-parallel reduction (tp_world > 1): every rank's exchange region
  // [2 parities][world][4 * max_n] LL words
  int tp_world, tp_rank;
  uint64_t* tp_ll[kMaxTpWorld];
  int64_t tp_max_n;
  uint32_t* tp_ctrl;  // [0] epoch, [1] finished-CTA count (device)
  // greedy argmax of the outputs (qgemv_kernel<..., true>): the launch's tokens' ids,
  // the [4] packed keys and the finished-CTA count (both zero between launches)
  int* ids;
  unsigned long long* amax_key;
  unsigned int* amax_ctl;
  int64_t amax_row0;               // added to the row in every key (a vocabulary shard's first row)
  unsigned long long* amax_out;    // non-null: the launch's tokens' keys are written here, not ids
  int* status;
};

// Packed argmax key of output v of row n: the high word maps the float order onto
// unsigned order (+0 and -0 equal, every value above the empty key 0), the low word
// prefers the lower row among equal values.  NaN is never packed.
__device__ __forceinline__ unsigned long long amax_pack(float v, int64_t n) {
  uint32_t u = __float_as_uint(v == 0.0f ? 0.0f : v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)n);
}

// The larger of key k and the key of output v at row n (NaN never wins).
__device__ __forceinline__ unsigned long long amax_take(unsigned long long k, float v, int64_t n) {
  if (v != v) return k;
  const unsigned long long c = amax_pack(v, n);
  return c > k ? c : k;
}

// The largest of k over the lanes xor distances first_xor .. 16 apart: first_xor = 4 joins
// the lanes of one token in whole mode (lane t of every group of four holds token t), 1
// joins the whole warp (split mode, one token at a time).
__device__ __forceinline__ unsigned long long amax_warp_max(unsigned long long k, int first_xor) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1)
    if (o >= first_xor) {
      const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, k, o);
      k = k2 > k ? k2 : k;
    }
  return k;
}

__device__ __forceinline__ void store_y(const Args& a, int t, int64_t n, float v) {
  const int64_t off = (int64_t)t * a.ldy + n;
  if (a.y_dtype == 0)
    static_cast<float*>(a.y)[off] = v;
  else if (a.y_dtype == 1)
    static_cast<__half*>(a.y)[off] = __float2half_rn(v);
  else
    static_cast<__nv_bfloat16*>(a.y)[off] = __float2bfloat16_rn(v);
}

__device__ __forceinline__ void named_bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

__device__ __forceinline__ void named_bar_arrive(int id, int n) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// Row-parallel tile exchange in two halves.  tp_publish_tile runs in the tile's writer
// warp as soon as the tile's 8 warp partials are in shared memory: the rank's partial of
// every (row, token) of the tile (row scale applied) goes to its slot on every rank as an
// LL word (value + epoch in one 8-byte store over NVLink), with no fence and no flag.
// tp_finish_tile runs after the CTA's last tile, so no warp waits for a peer while it
// still has groups to stream: it waits (bounded) until every rank's word of each element
// carries this launch's epoch, sums the partials in rank order -- every rank writes the
// same bits -- and adds the bias once.  A peer that never arrives ends the wait after
// 2 s with RTD_ERR_PEER_TIMEOUT in the status word.
__device__ __forceinline__ void tp_publish_tile(const Args& a, int tile, const float* rb, const float* ep,
                                                int lane, uint32_t epoch) {
  const int W = a.tp_world, R = a.tp_rank;
  const int64_t slot = 4 * a.tp_max_n;
  const int64_t base = (int64_t)(epoch & 1u) * W * slot + (int64_t)R * slot;
  for (int o = lane; o < 16 * a.M; o += 32) {
    const int r = o / a.M, t = o - r * a.M;
    const int64_t n = (int64_t)tile * 16 + r;
    float sum = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w)
      for (int p = 0; p < a.P; ++p) sum += rb[((size_t)w * 16 + r) * a.ncol8 + t * a.P + p];
    if (n < a.N) {
      const int64_t off = base + (int64_t)t * a.N + n;
      const float v = sum * ep[16 + r];
      for (int q = 1; q <= W; ++q) {  // peers first, own slot last
        const int p = (R + q) % W;
        st_ll(a.tp_ll[p] + off, v, epoch);
      }
    }
  }
  __syncwarp();
}

__device__ __forceinline__ void tp_finish_tile(const Args& a, int tile, int lane, uint32_t epoch, bool& dead) {
  const int W = a.tp_world, R = a.tp_rank;
  const int64_t slot = 4 * a.tp_max_n;
  const uint64_t* mine = a.tp_ll[R] + (int64_t)(epoch & 1u) * W * slot;
  for (int o = lane; o < 16 * a.M; o += 32) {
    const int r = o / a.M, t = o - r * a.M;
    const int64_t n = (int64_t)tile * 16 + r;
    if (n < a.N) {
      const uint64_t* src = mine + (int64_t)t * a.N + n;
      float v = 0.0f;
      for (int q = 0; q < W; ++q) v += wait_ll(src + (int64_t)q * slot, epoch, dead, a.status);
      store_y(a, t, n, v + (a.bias ? __ldg(a.bias + n) : 0.0f));
    }
  }
  __syncwarp();
}

// Local-x staging for DIAG formats.  The CTA copies the raw bf16 / f16 rows into
// shared memory (one bulk copy per token); then every warp converts groups on its
// own: a group's max |x| (warp shuffles) sets its power-of-two scale, the scaled f16
// units are rewritten in place in the transposed DIAG order, and the table row gets
// the sub-block sums and the scale.  In split mode a warp converts exactly the groups
// it will consume, so no block-wide barrier follows; in whole mode the warps share
// the work and meet once.
template <int FMT>
__device__ __forceinline__ void stage_local_diag(const Args& a, uint8_t* sm, bool whole, int* status) {
  using F = FmtC<FMT>;
  constexpr int UPG = F::GK / 8, GPI = 32 / UPG, SBC = F::SBE / 8, NSB = F::GK / F::SBE;
  constexpr int TW = tab_row_floats<FMT>();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint8_t* xloc = sm + a.off_xloc;
  uint64_t* xbar = reinterpret_cast<uint64_t*>(sm + a.off_tabloc - 16);
  float* tab = reinterpret_cast<float*>(sm + a.off_tabloc);
  const uint32_t row_bytes = (uint32_t)(a.K * 2);
  if (tid == 0) {
    mbar_init(xbar, 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(xbar, row_bytes * (uint32_t)a.M);
    for (int t = 0; t < a.M; ++t)
      bulk_g2s(xloc + (size_t)t * a.xcs, static_cast<const uint8_t*>(a.xraw) + (size_t)t * a.ldx * 2, row_bytes, xbar);
  }
  // zero the padding past K (trailing partial Q8_0 groups)
  for (int64_t i = a.K + tid; i < a.kp; i += kThreads)
    for (int t = 0; t < a.M; ++t) reinterpret_cast<uint16_t*>(xloc + (size_t)t * a.xcs)[i] = 0;
  __syncthreads();  // barrier init, zero page and padding visible to every warp
  mbar_wait_bounded(xbar, 0, status);
  // this warp's groups: split mode -> those of items warp, warp+8, ...; whole -> warp, warp+8, ...
  const int sub = lane / UPG, n = lane % UPG;  // GPI groups side by side in the warp
  const int per = whole ? (a.G - warp + kWarps - 1) / kWarps
                        : ((a.CI > warp) ? (a.CI - warp + kWarps - 1) / kWarps : 0) * a.IG;
  for (int q0 = 0; q0 < per; q0 += GPI) {
    const int q = q0 + sub;
    int gi = -1;
    if (q < per) {
      if (whole) {
        gi = warp + kWarps * q;
      } else {
        const int it = warp + kWarps * (q / a.IG);
        gi = it * a.IG + q % a.IG;
        if (gi >= a.G) gi = -1;
      }
    }
    for (int t = 0; t < a.M; ++t) {
      uint8_t* gbase = xloc + (size_t)t * a.xcs + (size_t)(gi < 0 ? 0 : gi) * F::GK * 2;
      float v[8];
      if (gi >= 0) {
        const uint4 u = reinterpret_cast<const uint4*>(gbase)[n];
        const uint32_t wd[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t b16 = (wd[i >> 1] >> (16 * (i & 1))) & 0xFFFFu;
          v[i] = (a.x_dtype == 1) ? h2f(b16) : __uint_as_float(b16 << 16);
          if (a.w8a8) v[i] = e4m3_round_ref(v[i]);  // W8A8: the reference E4M3 rounding first
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.0f;
      }
      float m = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(v[i]));
#pragma unroll
      for (int o = 1; o < UPG; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      const int e = group_exponent(m);
      const float inv = ldexpf(1.0f, -e);
      __half h[8];
      float sum = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        h[i] = __float2half_rn(v[i] * inv);
        sum += __half2float(h[i]);
      }
#pragma unroll
      for (int o = 1; o < SBC; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      uint4 cv = make_uint4(pack_h2(h[0], h[1]), pack_h2(h[2], h[3]), pack_h2(h[4], h[5]), pack_h2(h[6], h[7]));
      if constexpr (FMT == FMT_Q4K) cv = q4k_quad_order(cv);
      __syncwarp();  // every lane has read its unit before the group is rewritten in place
      if (gi >= 0) {
        *reinterpret_cast<uint4*>(gbase + diag_unit_offset<FMT>(n)) = cv;
        float* tp = tab + ((size_t)gi * a.ncol + t) * TW;
        if (n % SBC == 0) tp[n / SBC] = sum * F::XOFF;
        if (n == 0) tp[NSB] = ldexpf(1.0f, e);
      }
      __syncwarp();
    }
  }
  if (whole) __syncthreads();
  else __syncwarp();
}

// Each CTA owns a contiguous run of whole 16-row tiles; inside a tile, warp w
// takes items w, w+8, ... (an item = IG groups).  Every warp streams its own
// item sequence through a private ring of NS shared-memory stages, so warps only
// meet once per tile: to add their partial sums in shared memory (double
// buffered), after which one warp (tile index mod 8) writes the tile's outputs.
// AMAX: the greedy argmax of every token's outputs is folded into the epilogue (the
// outputs themselves are written only when a.y is set).
template <int FMT, int NT, bool AMAX>
__global__ void __launch_bounds__(kThreads, (NT <= 2 ? 2 : 1)) qgemv_kernel(const Args a) {
  using F = FmtC<FMT>;
  constexpr int CSB = col_stride_bytes(F::GK);
  constexpr int NSB = F::GK / F::SBE;
  extern __shared__ __align__(128) uint8_t sm[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, tq = lane & 3;
  const int CI = a.CI;
  const bool whole = a.whole != 0;
  int t0, t1, per_tile;
  if (whole) {  // this warp's own run of tiles, all items of each
    const int64_t gw = (int64_t)blockIdx.x * kWarps + warp, WT = (int64_t)a.nctas * kWarps;
    t0 = (int)(gw * a.T / WT);
    t1 = (int)((gw + 1) * a.T / WT);
    per_tile = CI;
  } else {  // the CTA's run of tiles, items warp, warp+8, ... of each
    t0 = (int)((int64_t)blockIdx.x * a.T / a.nctas);
    t1 = (int)((int64_t)(blockIdx.x + 1) * a.T / a.nctas);
    per_tile = (CI > warp) ? (CI - warp + kWarps - 1) / kWarps : 0;
  }
  const int n_items = per_tile * (t1 - t0);
  uint8_t* wb = sm + (size_t)warp * a.warp_bytes;
  uint64_t* bar = reinterpret_cast<uint64_t*>(wb + a.off_bar);
  uint8_t* tblw = wb + a.off_tbl;
  const uint32_t wb_s = smem_u32(wb), tb_s = smem_u32(tblw);
  float* red = reinterpret_cast<float*>(sm + a.off_red);  // [2][8 warps][16][ncol8]
  const int NS = a.NS;

  // the issue side walks its own cursor over (tile, group) a few items ahead
  const bool local_x = a.local_x != 0;
  auto bytes_of = [&](int ng) -> uint32_t {
    uint32_t b = (uint32_t)ng * F::GB;
    if (!local_x) {
      b += (uint32_t)ng * a.ncol * CSB;
      b += (uint32_t)ng * a.tabw * 4;
    }
    return b;
  };
  auto issue_w = [&](int s, int tile, int g0, int ng) {
    mbar_arrive_expect_tx(&bar[s], bytes_of(ng));
    bulk_g2s(wb + (size_t)s * a.slot_bytes, a.w + ((size_t)tile * a.G + g0) * F::GB, (uint32_t)ng * F::GB, &bar[s]);
  };
  auto issue_x = [&](int s, int g0, int ng) {
    uint8_t* slot = wb + (size_t)s * a.slot_bytes;
    bulk_g2s(slot + a.off_x, a.cols + (size_t)g0 * a.ncol * CSB, (uint32_t)ng * a.ncol * CSB, &bar[s]);
    bulk_g2s(slot + a.off_tab, a.tab + (size_t)g0 * a.tabw, (uint32_t)ng * a.tabw * 4, &bar[s]);
  };
  const int gstep = (whole ? 1 : kWarps) * a.IG;  // group stride between a warp's items in a tile
  const int gfirst = (whole ? 0 : warp) * a.IG;

  if (lane == 0) {
    for (int s = 0; s < NS; ++s) mbar_init(&bar[s], 1);
    fence_mbar_init();
  }
  __syncwarp();
  const int npro = n_items < NS ? n_items : NS;
  // issue cursor: (tile, group) of the next item to issue
  int it_tile = t0, it_g0 = gfirst, it_k = 0;
  auto advance = [&]() {
    if (++it_k == per_tile) {
      it_k = 0;
      ++it_tile;
      it_g0 = gfirst;
    } else {
      it_g0 += gstep;
    }
  };
  if (lane == 0) {
    int tt = t0, gg = gfirst, kk = 0;
    for (int s = 0; s < npro; ++s) {  // weights go out before x is known to be ready
      issue_w(s, tt, gg, min(a.IG, a.G - gg));
      if (++kk == per_tile) { kk = 0; ++tt; gg = gfirst; } else { gg += gstep; }
    }
  }
  griddep_wait();  // earlier work in the stream (x, the prep kernel's output) is visible from here on
  griddep_launch_dependents();  // the next call may launch; it waits for this grid before touching x
  // row-parallel launches: this launch's epoch (the previous TP launch, complete by now,
  // left its own in ctrl[0])
  const uint32_t tp_epoch = a.tp_world > 1 ? *reinterpret_cast<volatile uint32_t*>(a.tp_ctrl) + 1u : 0u;
  for (int s = 0; s < npro; ++s) {
    if (lane == 0 && !local_x) issue_x(s, it_g0, min(a.IG, a.G - it_g0));
    advance();
  }
  // the zero page idle B-fragment lanes read (published by the barrier below)
  for (int i = tid; i < kZeroPage / 4; i += kThreads) reinterpret_cast<uint32_t*>(sm + a.off_zero)[i] = 0u;
  // AMAX: the CTA's best key per token, in the 128 spare bytes after the split-mode
  // reduction buffer (published by the barrier below)
  unsigned long long* cta_keys =
      reinterpret_cast<unsigned long long*>(sm + a.off_red + (size_t)2 * kWarps * 16 * a.ncol8 * 4);
  if (AMAX && tid < 4) cta_keys[tid] = 0ull;
  if (local_x) {
    stage_local_diag<FMT>(a, sm, whole, &a.status[0]);
  } else {
    __syncthreads();
  }
  const uint32_t xloc_s = smem_u32(sm + a.off_xloc), tabloc_s = smem_u32(sm + a.off_tabloc);
  // idle lanes point at the zero page, on banks no active lane of the same load uses
  const uint32_t zero_s = smem_u32(sm + a.off_zero);
  const uint32_t z0 = zero_s + ((FMT == FMT_Q80 || FMT == FMT_FP8) ? 112u : 16u), z1 = zero_s;
  const bool act0 = g == 2 * tq, act1 = g == 2 * tq + 1;

  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.0f;
  int i = 0;
  int slot_i = 0;         // ring slot of item i
  uint32_t phase = 0;     // its mbarrier phase parity
  int next_issue = npro;  // items [0, next_issue) have had their copies issued
  bool aborted = false;   // a bounded wait gave up: stop issuing and computing, keep the barriers
  for (int tile = t0; tile < t1; ++tile) {
    // the warp that will write this tile prefetches its epilogue operands
    // (split mode: lane r < 16 holds row r; whole mode: each lane its rows g and g+8)
    const bool writer = whole || (warp == (tile & (kWarps - 1)));
    float eb = 0.0f, es = 1.0f, eb2 = 0.0f, es2 = 1.0f;
    if (writer && (whole || lane < 16)) {
      const int64_t n = (int64_t)tile * 16 + (whole ? g : lane), n2 = n + 8;
      if (n < a.N) {
        if (a.bias) eb = __ldg(a.bias + n);
        if (a.row_scale) es = __ldg(a.row_scale + (a.scale_len == 1 ? 0 : n));
      }
      if (whole && n2 < a.N) {
        if (a.bias) eb2 = __ldg(a.bias + n2);
        if (a.row_scale) es2 = __ldg(a.row_scale + (a.scale_len == 1 ? 0 : n2));
      }
    }
    for (int k = 0; k < per_tile; ++k, ++i) {
      if (aborted) continue;
      const int g0 = gfirst + k * gstep;
      const int ng = min(a.IG, a.G - g0);
      // every lane observes the phase itself; the verdict is made warp-uniform
      if (!__all_sync(0xffffffffu, mbar_wait_ns(&bar[slot_i], phase, kWaitBudgetNs, a.status))) {
        aborted = true;
        continue;
      }
      const uint32_t slot = wb_s + (uint32_t)(slot_i * a.slot_bytes);
      if (local_x) {
#pragma unroll 1
        for (int gi = 0; gi < ng; ++gi)
          do_group_diag<FMT, NT>(slot + gi * F::GB, xloc_s + (uint32_t)(g0 + gi) * F::GK * 2, (uint32_t)a.xcs,
                                 tabloc_s + (uint32_t)((g0 + gi) * a.tabw) * 4, z0, z1, act0, act1, acc, lane);
      } else {
#pragma unroll 1
        for (int gi = 0; gi < ng; ++gi)
          do_group_diag<FMT, NT>(slot + gi * F::GB, slot + a.off_x + gi * a.ncol * CSB, (uint32_t)CSB,
                                 slot + a.off_tab + gi * a.tabw * 4, z0, z1, act0, act1, acc, lane);
      }
      __syncwarp();
      if (i + NS < n_items) {
        if (lane == 0) {
          const int ng2 = min(a.IG, a.G - it_g0);
          issue_w(slot_i, it_tile, it_g0, ng2);
          if (!local_x) issue_x(slot_i, it_g0, ng2);
        }
        advance();
        next_issue = i + NS + 1;
      }
      if (++slot_i == NS) {
        slot_i = 0;
        phase ^= 1u;
      }
    }
    {
      // each lane holds partial sums over its own sub-blocks: add the 4 lanes of a row
#pragma unroll
      for (int c = 0; c < NT; ++c)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          float v = acc[c][r];
          v += __shfl_xor_sync(0xffffffffu, v, 1);
          v += __shfl_xor_sync(0xffffffffu, v, 2);
          acc[c][r] = v;
        }
      if (whole) {  // lane t writes token t of rows g and g+8
        unsigned long long tkey = 0ull;  // AMAX: this lane's best key of the tile (token tq)
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          const int64_t n = (int64_t)tile * 16 + g + 8 * rr;
          const float bias = rr ? eb2 : eb, cs = rr ? es2 : es;
#pragma unroll
          for (int c = 0; c < NT; ++c) {
            if (a.P == 2) {
              const int t = c >> 1;
              if ((c & 1) == 0 && c + 1 < NT && tq == t && t < a.M && n < a.N) {
                const float v = (acc[c][rr] + acc[c + 1][rr]) * cs + bias;
                if (!AMAX || a.y) store_y(a, t, n, v);
                if (AMAX) tkey = amax_take(tkey, v, n + a.amax_row0);
              }
            } else if (tq == c && c < a.M && n < a.N) {
              const float v = acc[c][rr] * cs + bias;
              if (!AMAX || a.y) store_y(a, c, n, v);
              if (AMAX) tkey = amax_take(tkey, v, n + a.amax_row0);
            }
          }
        }
        if constexpr (AMAX) {  // lanes of one tq hold one token: reduce over g, lanes 0..3 publish
          tkey = amax_warp_max(tkey, 4);
          if (g == 0 && tq < a.M && tkey != 0ull) atomicMax(cta_keys + tq, tkey);
        }
#pragma unroll
        for (int c = 0; c < NT; ++c) acc[c][0] = acc[c][1] = 0.0f;
        continue;
      }
    }
    // ---- tile end: the 8 partial sums meet in shared memory (double buffered).
    // Only the writer of the tile waits for them (bar.sync on FULL[b]); the others
    // arrive and move on.  A buffer is reused two tiles later, after its previous
    // writer has released it on EMPTY[b] (every warp but that writer syncs there).
    const int b = tile & 1;
    const int lt = tile - t0;
    if (lt >= 2) {
      const int prev_writer = (tile - 2) & (kWarps - 1);
      if (warp != prev_writer) named_bar_sync(3 + b, kThreads);
    }
    float* rb = red + (size_t)b * kWarps * 16 * a.ncol8;
    float* rw = rb + (size_t)warp * 16 * a.ncol8;
    if (tq == 0) {
#pragma unroll
      for (int c = 0; c < NT; ++c) {
        rw[g * a.ncol8 + c] = acc[c][0];
        rw[(g + 8) * a.ncol8 + c] = acc[c][1];
      }
    }
#pragma unroll
    for (int c = 0; c < NT; ++c) acc[c][0] = acc[c][1] = 0.0f;
    if (!writer) {
      named_bar_arrive(1 + b, kThreads);
    } else {
      named_bar_sync(1 + b, kThreads);
      float* ep = reinterpret_cast<float*>(tblw);  // the scale table is idle between groups
      if (lane < 16) {
        ep[lane] = eb;
        ep[16 + lane] = es;
      }
      __syncwarp();
      if (a.tp_world > 1) {
        tp_publish_tile(a, tile, rb, ep, lane, tp_epoch);  // finished after the last tile
      } else {
        unsigned long long tk[4] = {0ull, 0ull, 0ull, 0ull};  // AMAX: this lane's best key per token
        for (int o = lane; o < 16 * a.M; o += 32) {
          const int r = o / a.M, t = o - r * a.M;
          const int64_t n = (int64_t)tile * 16 + r;
          float sum = 0.0f;
#pragma unroll
          for (int w = 0; w < kWarps; ++w)
            for (int p = 0; p < a.P; ++p) sum += rb[((size_t)w * 16 + r) * a.ncol8 + t * a.P + p];
          if (n < a.N) {
            const float v = sum * ep[16 + r] + ep[r];
            if (!AMAX || a.y) store_y(a, t, n, v);
            if constexpr (AMAX) {
#pragma unroll
              for (int u = 0; u < 4; ++u)
                if (u == t) tk[u] = amax_take(tk[u], v, n + a.amax_row0);
            }
          }
        }
        if constexpr (AMAX) {  // the writer warp's keys of this tile, per token
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const unsigned long long k = amax_warp_max(tk[u], 1);
            if (lane == 0 && u < a.M && k != 0ull) atomicMax(cta_keys + u, k);
          }
        }
      }
      __syncwarp();
      if (tile + 2 < t1) named_bar_arrive(3 + b, kThreads);  // hand the buffer back
    }
  }
  // after a failed wait, drain the copies already issued before leaving
  if (aborted) {
    for (int s = 0; s < NS && s < next_issue; ++s) {
      const int last = s + ((next_issue - 1 - s) / NS) * NS;  // the last item issued into slot s
      mbar_wait_ns(&bar[s], (uint32_t)(last / NS) & 1u, kWaitBudgetNs, a.status);
    }
  }
  if (a.tp_world > 1) {  // each writer warp finishes the tiles it published (split mode)
    bool dead = false;
    for (int tile = t0; tile < t1; ++tile)
      if (warp == (tile & (kWarps - 1))) tp_finish_tile(a, tile, lane, tp_epoch, dead);
  }
  if (a.tp_world > 1) {  // the last CTA of the launch publishes its epoch for the next one
    __syncthreads();
    if (tid == 0) {
      __threadfence();
      if (atomicAdd(a.tp_ctrl + 1, 1u) == gridDim.x - 1) {
        a.tp_ctrl[1] = 0u;
        a.tp_ctrl[0] = tp_epoch;
        __threadfence();
      }
    }
  }
  if constexpr (AMAX) {  // the CTA's best key per token, one atomic each; the launch's last
                         // CTA reads the ids
    __syncthreads();
    if (tid == 0) {
      for (int u = 0; u < a.M; ++u)
        if (cta_keys[u] != 0ull) atomicMax(a.amax_key + u, cta_keys[u]);
      __threadfence();
      if (atomicAdd(a.amax_ctl, 1u) == gridDim.x - 1) {
        __threadfence();
        for (int t = 0; t < a.M; ++t) {
          const unsigned long long k = atomicExch(a.amax_key + t, 0ull);
          if (a.amax_out)
            a.amax_out[t] = k;
          else
            a.ids[t] = k != 0ull ? (int)(0xFFFFFFFFu - (uint32_t)k) : 0;
        }
        atomicExch(a.amax_ctl, 0u);
      }
    }
  }
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

struct Plan {
  int NS, warp_bytes, slot_bytes, off_x, off_tab, off_tbl, off_bar, off_red;
  int off_xloc = 0, xcs = 0, off_tabloc = 0, off_zero = 0;
  size_t smem;
};

// Column-sum table floats for `kp` elements and `ncol` columns.
inline size_t tab_floats(int fmt, int64_t kp, int ncol) {
  const FmtInfo f = fmt_info(fmt);
  return (size_t)(kp / f.gk) * (size_t)ncol * (size_t)(f.gk / f.sbe + 4);
}

// Shared-memory plan of one GEMV launch.  local_kp > 0 asks for the local-x region
// (activations staged by every CTA).
//   per warp : NS ring slots (weights [+ x units + table rows when not local]),
//              a 128-byte epilogue scratch, NS mbarriers
//   per CTA  : the double-buffered split-mode reduction, the token scales, the zero
//              page, and (local) the staged rows, amax scratch, x barrier, table
Plan make_plan(int fmt, int IG, int ncol, int ncol8, int ns_pref, int64_t local_kp = 0) {
  const FmtInfo f = fmt_info(fmt);
  const int csb = col_stride_bytes(f.gk);
  const bool local = local_kp > 0;
  Plan p{};
  const size_t off_x = align_up((size_t)IG * f.gb, 128);
  const size_t off_tab = align_up(off_x + (local ? 0 : (size_t)IG * ncol * csb), 16);
  const size_t slot = align_up(off_tab + (local ? 0 : tab_floats(fmt, (int64_t)IG * f.gk, ncol) * 4), 128);
  const size_t red = (size_t)2 * kWarps * 16 * ncol8 * 4 + 32 * 4;
  size_t loc = 0;
  if (local) {
    p.xcs = (int)align_up((size_t)local_kp * 2, 128);
    loc = 128 + (size_t)ncol * p.xcs + (size_t)32 * kWarps * 4 + 16 + tab_floats(fmt, local_kp, ncol) * 4;
  }
  // prefer two CTAs per SM (<= 113 KB each); keep at least two stages in flight
  int NS = ns_pref;
  auto warp_bytes = [&](int ns) { return align_up(ns * slot + kTblBytes + kMaxStages * 8, 128); };
  while (NS > 2 && warp_bytes(NS) * kWarps + red + kZeroPage + 128 + loc > 113 * 1024) --NS;
  p.NS = NS;
  p.slot_bytes = (int)slot;
  p.off_x = (int)off_x;
  p.off_tab = (int)off_tab;
  p.off_tbl = (int)(NS * slot);
  p.off_bar = (int)(NS * slot + kTblBytes);
  p.warp_bytes = (int)warp_bytes(NS);
  p.off_red = (int)((size_t)p.warp_bytes * kWarps);
  size_t end = (size_t)p.off_red + red;
  p.off_zero = (int)align_up(end, 128);
  end = (size_t)p.off_zero + kZeroPage;
  if (local) {
    p.off_xloc = (int)align_up(end, 128);
    p.off_tabloc = (int)align_up((size_t)p.off_xloc + (size_t)ncol * p.xcs, 16) + 32 * kWarps * 4 + 16;
    end = (size_t)p.off_tabloc + tab_floats(fmt, local_kp, ncol) * 4;
  }
  p.smem = align_up(end, 16);
  return p;
}

// Groups per item (one bulk copy): two 256-wide Q4_K groups when a row has enough of
// them, one Q6_K group (two would halve the CTAs per SM); for the 128-wide Q8_0 and
// FP8 groups the largest candidate up to ~6 KB that still spreads a tile evenly over
// the warps.
int items_group(int fmt, int64_t G) {
  static const int env_ig = [] {  // tuning override: RTD_GEMV_IG=1|2|4|8
    const char* s = std::getenv("RTD_GEMV_IG");
    const int v = s ? std::atoi(s) : 0;
    return (v == 1 || v == 2 || v == 4 || v == 8) ? v : 0;
  }();
  if (env_ig) return (int)std::min<int64_t>(env_ig, std::max<int64_t>(1, G / kWarps));
  if (fmt == FMT_Q4K) return G >= 2 * kWarps ? 2 : 1;
  if (fmt == FMT_Q6K) return 1;
  // items of at most ~6 KB keep a two-stage ring of 8 warps within shared memory
  const int cap = std::max(1, 6144 / fmt_info(fmt).gb);
  int best = 1;
  double best_eff = 0.0;
  const int cands[4] = {8, 4, 2, 1};
  for (int ig : cands) {
    if (ig > cap) continue;
    const int64_t ci = (G + ig - 1) / ig;
    const double eff = (double)G / ((double)ig * kWarps * ((ci + kWarps - 1) / kWarps));
    if (eff >= 0.85) return ig;
    if (eff > best_eff) {
      best_eff = eff;
      best = ig;
    }
  }
  return best;
}

// Resident CTAs per SM for this instantiation at this shared-memory size, cached per
// device for the few sizes a process plans with.  The kernel's dynamic shared-memory
// limit is raised to the architectural maximum once, so any planned size launches.
constexpr int kMaxGemvSmem = 227 * 1024;

template <int FMT, int NT>
int gemv_occupancy(size_t smem) {
  constexpr int kCache = 8;
  static bool configured[64] = {};
  static size_t cached_smem[64][kCache] = {};
  static int cached_occ[64][kCache] = {};
  static int next_slot[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  dev &= 63;
  if (!configured[dev]) {
    cudaFuncSetAttribute(qgemv_kernel<FMT, NT, false>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    cudaFuncSetAttribute(qgemv_kernel<FMT, NT, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxGemvSmem);
    cudaFuncSetAttribute(qgemv_kernel<FMT, NT, true>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    cudaFuncSetAttribute(qgemv_kernel<FMT, NT, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxGemvSmem);
    configured[dev] = true;
  }
  for (int i = 0; i < kCache; ++i)
    if (cached_occ[dev][i] > 0 && cached_smem[dev][i] == smem) return cached_occ[dev][i];
  int occ = 1;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, qgemv_kernel<FMT, NT, false>, kThreads, smem) != cudaSuccess ||
      occ < 1)
    occ = 1;
  const int slot = next_slot[dev]++ % kCache;
  cached_smem[dev][slot] = smem;
  cached_occ[dev][slot] = occ;
  return occ;
}

template <int FMT>
int occupancy_nt(int NT, size_t smem) {
  switch (NT) {
    case 1: return gemv_occupancy<FMT, 1>(smem);
    case 2: return gemv_occupancy<FMT, 2>(smem);
    case 3: return gemv_occupancy<FMT, 3>(smem);
    default: return gemv_occupancy<FMT, 4>(smem);
  }
}

int occupancy_of(int fmt, int NT, size_t smem) {
  switch (fmt) {
    case FMT_Q4K: return occupancy_nt<FMT_Q4K>(NT, smem);
    case FMT_Q6K: return occupancy_nt<FMT_Q6K>(NT, smem);
    case FMT_Q80: return occupancy_nt<FMT_Q80>(NT, smem);
    default: return occupancy_nt<FMT_FP8>(NT, smem);
  }
}

template <int FMT, int NT>
cudaError_t launch_gemv(const Args& a, unsigned nctas, size_t smem, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nctas);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  count_launch();
  if (a.amax_key) return cudaLaunchKernelEx(&cfg, qgemv_kernel<FMT, NT, true>, a);
  return cudaLaunchKernelEx(&cfg, qgemv_kernel<FMT, NT, false>, a);
}

template <int FMT>
cudaError_t launch_gemv_nt(const Args& a, int NT, unsigned nctas, size_t smem, cudaStream_t st) {
  switch (NT) {
    case 1: return launch_gemv<FMT, 1>(a, nctas, smem, st);
    case 2: return launch_gemv<FMT, 2>(a, nctas, smem, st);
    case 3: return launch_gemv<FMT, 3>(a, nctas, smem, st);
    default: return launch_gemv<FMT, 4>(a, nctas, smem, st);
  }
}

template <int FMT>
cudaError_t launch_prep_diag(const PrepArgs& p, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((p.kp / 8 + kPrepThreads - 1) / kPrepThreads), (unsigned)p.M);
  cfg.blockDim = dim3(kPrepThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  count_launch();
  return cudaLaunchKernelEx(&cfg, prep_diag_kernel<FMT>, p);
}

}  // namespace

__global__ void fill_rows_kernel(const float* bias, void* y, int y_dtype, int64_t ldy, int64_t M, int64_t N) {
  const int64_t total = M * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / N, n = i - m * N;
    const float v = bias ? bias[n] : 0.0f;
    const int64_t off = m * ldy + n;
    if (y_dtype == 0)
      static_cast<float*>(y)[off] = v;
    else if (y_dtype == 1)
      static_cast<__half*>(y)[off] = __float2half_rn(v);
    else
      static_cast<__nv_bfloat16*>(y)[off] = __float2bfloat16_rn(v);
  }
}

cudaError_t launch_fill_rows(const float* bias, void* y, int y_dtype, int64_t ldy, int64_t M, int64_t N,
                             cudaStream_t st) {
  if (M <= 0 || N <= 0) return cudaSuccess;
  int64_t blocks = (M * N + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  count_launch();
  fill_rows_kernel<<<(unsigned)blocks, 256, 0, st>>>(bias, y, y_dtype, ldy, M, N);
  return cudaGetLastError();
}

cudaError_t launch_qgemv(const QGemvCall& c, int* plan_error) {
  *plan_error = 0;
  if (c.M <= 0 || c.N <= 0) return cudaSuccess;
  const FmtInfo f = fmt_info(c.fmt);
  const int64_t T = tiles_for(c.N);
  const int64_t G = c.G;
  const int64_t kp = G * f.gk;
  const int IG = items_group(c.fmt, G);
  const int64_t CI = (G + IG - 1) / IG;
  const int P = (c.x_dtype == 0 && !c.w8a8) ? 2 : 1;
  // the decoders run one MMA chain per activation column: at most 4 columns a launch
  const int max_tokens = 4 / P;
  static const int env_ns = [] {
    const char* s = std::getenv("RTD_GEMV_STAGES");
    const int v = s ? std::atoi(s) : 0;
    return (v >= 2 && v <= kMaxStages) ? v : kMaxStages;
  }();
  const size_t esz = (c.x_dtype == 0) ? 4 : 2;
  const bool x_vec = ((uintptr_t)c.x % 16 == 0) && ((c.ldx * (int64_t)esz) % 16 == 0);
  static const bool env_no_local = std::getenv("RTD_GEMV_NO_LOCAL_X") != nullptr;
  if (T >= (1LL << 31) || G >= (1LL << 31)) {
    *plan_error = 1;
    return cudaSuccess;
  }

  for (int64_t m0 = 0; m0 < c.M;) {
    int Mt = (int)std::min<int64_t>(max_tokens, c.M - m0);
    // fewer tokens per launch when the activation slices would not fit shared memory
    while (Mt > 1 && make_plan(c.fmt, IG, Mt * P, 8 * ((Mt * P + 7) / 8), env_ns).smem > 220 * 1024)
      Mt = (Mt + 1) / 2;
    const int ncol = Mt * P;
    const int NT = ncol;  // template width: activation columns of this launch
    const int ncol8 = 8;  // row stride of the split-mode reduction buffer
    // Enough tiles for every warp to own at least two whole ones: no cross-warp
    // reduction at all (whole mode).  Otherwise the warps of a CTA split each tile's
    // groups; the row-parallel exchange always runs in split mode.
    Plan pl = make_plan(c.fmt, IG, ncol, ncol8, env_ns, 0);
    int occ = occupancy_of(c.fmt, NT, pl.smem);
    int64_t slots = (int64_t)c.sm_count * occ;
    bool whole = !c.tp && T >= 2 * slots * kWarps;
    // bf16 / f16 activations whose rows are bulk-copyable, in a whole-mode launch:
    // every CTA stages x itself (no prep kernel) when the staged rows and sums stay
    // small.  In split mode the prep kernel is faster: measured on B200 at M = 1, the
    // 14336-wide rows run 25-40 % faster and 4096 x 4096 about 15 % faster with it,
    // while the 151936 x 896 LM head (whole mode) runs 25 % slower with it.
    bool local_ok = false;
    const size_t local_tab = tab_floats(c.fmt, kp, ncol);
    if (whole && c.x_dtype != 0 && x_vec && (c.K % 8 == 0) && !env_no_local &&
        (size_t)ncol * kp * 2 + local_tab * 4 <= 40 * 1024) {
      const Plan pl_loc = make_plan(c.fmt, IG, ncol, ncol8, env_ns, kp);
      const int occ_loc = occupancy_of(c.fmt, NT, pl_loc.smem);
      if (T >= 2 * (int64_t)c.sm_count * occ_loc * kWarps) {  // still whole with the staged row
        pl = pl_loc;
        occ = occ_loc;
        slots = (int64_t)c.sm_count * occ;
        local_ok = true;
      }
    }
    const int nctas = (int)(whole ? slots : std::min<int64_t>(T, slots));
    // workspace carve: cols | tab | tscale
    const size_t cols_b = align_up((size_t)G * ncol * col_stride_bytes(f.gk), 256);
    const size_t tab_b = align_up(tab_floats(c.fmt, kp, ncol) * 4 + 4, 256);
    if (cols_b + tab_b + 256 > c.ws_bytes) {
      *plan_error = 1;
      return cudaSuccess;
    }
    uint8_t* ws = reinterpret_cast<uint8_t*>(c.ws);
    uint8_t* cols = ws;
    float* tab = reinterpret_cast<float*>(ws + cols_b);
    float* tscale = reinterpret_cast<float*>(ws + cols_b + tab_b);

    PrepArgs pa{};
    pa.x = static_cast<const uint8_t*>(c.x) + (size_t)(m0 * c.ldx) * esz;
    pa.x_dtype = c.x_dtype;
    pa.x_vec = x_vec ? 1 : 0;
    pa.ldx = c.ldx;
    pa.K = c.K;
    pa.kp = kp;
    pa.M = Mt;
    pa.P = P;
    pa.ncol = ncol;
    pa.ncol8 = ncol8;
    pa.w8a8 = c.w8a8;
    pa.cols = cols;
    pa.tab = tab;
    pa.tscale = tscale;
    cudaError_t e = cudaSuccess;
    if (!local_ok) {
      switch (c.fmt) {
        case FMT_Q4K: e = launch_prep_diag<FMT_Q4K>(pa, c.stream); break;
        case FMT_Q6K: e = launch_prep_diag<FMT_Q6K>(pa, c.stream); break;
        case FMT_Q80: e = launch_prep_diag<FMT_Q80>(pa, c.stream); break;
        default:      e = launch_prep_diag<FMT_FP8>(pa, c.stream); break;
      }
      if (e != cudaSuccess) return e;
    }

    Args a{};
    a.w = c.w;
    a.row_scale = c.row_scale;
    a.scale_len = c.scale_len;
    a.cols = cols;
    a.tab = tab;
    a.tscale = tscale;
    a.M = Mt;
    a.P = P;
    a.ncol = ncol;
    a.ncol8 = ncol8;
    a.bias = c.bias;
    const size_t ysz = (c.y_dtype == 0) ? 4 : 2;
    a.y = c.y ? static_cast<uint8_t*>(c.y) + (size_t)(m0 * c.ldy) * ysz : nullptr;
    a.ldy = c.ldy;
    a.y_dtype = c.y_dtype;
    a.N = c.N;
    a.G = (int)G;
    a.IG = IG;
    a.CI = (int)CI;
    a.T = (int)T;
    a.nctas = nctas;
    a.whole = whole ? 1 : 0;
    a.NS = pl.NS;
    a.warp_bytes = pl.warp_bytes;
    a.slot_bytes = pl.slot_bytes;
    a.off_x = pl.off_x;
    a.off_tab = pl.off_tab;
    a.off_tbl = pl.off_tbl;
    a.off_bar = pl.off_bar;
    a.off_red = pl.off_red;
    a.local_x = local_ok ? 1 : 0;
    a.xraw = pa.x;
    a.ldx = c.ldx;
    a.K = c.K;
    a.kp = kp;
    a.x_dtype = c.x_dtype;
    a.w8a8 = c.w8a8;
    a.off_xloc = pl.off_xloc;
    a.xcs = pl.xcs;
    a.off_tabloc = pl.off_tabloc;
    a.tabw = ncol * (f.gk / f.sbe + 4);
    a.off_zero = pl.off_zero;
    const bool amax = c.ids || c.amax_out;
    a.ids = c.ids ? c.ids + m0 : nullptr;
    a.amax_out = c.amax_out ? c.amax_out + m0 : nullptr;
    a.amax_row0 = c.amax_row0;
    a.amax_key = amax ? c.amax : nullptr;  // every launch of the call starts from clear keys
    a.amax_ctl = amax ? reinterpret_cast<unsigned int*>(c.amax + 4) : nullptr;
    a.tp_world = 1;
    if (c.tp && c.tp->world > 1) {
      const TpReduce& tp = *c.tp;
      if (c.N > tp.max_n || Mt > 4 || c.ids || c.amax_out) {  // (no argmax over a rank's partial sums)
        *plan_error = 1;
        return cudaSuccess;
      }
      a.tp_world = tp.world;
      a.tp_rank = tp.rank;
      a.tp_max_n = tp.max_n;
      a.tp_ctrl = tp.ctrl;
      for (int p = 0; p < tp.world; ++p) a.tp_ll[p] = tp.ll[p];  // the kernel picks its half by epoch
    }
    a.status = c.status;
    switch (c.fmt) {
      case FMT_Q4K: e = launch_gemv_nt<FMT_Q4K>(a, NT, (unsigned)nctas, pl.smem, c.stream); break;
      case FMT_Q6K: e = launch_gemv_nt<FMT_Q6K>(a, NT, (unsigned)nctas, pl.smem, c.stream); break;
      case FMT_Q80: e = launch_gemv_nt<FMT_Q80>(a, NT, (unsigned)nctas, pl.smem, c.stream); break;
      default:      e = launch_gemv_nt<FMT_FP8>(a, NT, (unsigned)nctas, pl.smem, c.stream); break;
    }
    if (e != cudaSuccess) return e;
    m0 += Mt;
  }
  return cudaSuccess;
}

// Workspace bytes launch_qgemv carves for this call: the largest of its token chunks,
// computed with the same chunking and plan (a call whose ws_bytes is at least this
// never fails with a plan error for lack of workspace).
size_t qgemv_workspace_bytes(const QGemvCall& c) {
  if (c.M <= 0 || c.N <= 0 || c.K <= 0) return 0;
  const FmtInfo f = fmt_info(c.fmt);
  const int64_t G = c.G;
  const int64_t kp = G * f.gk;
  const int IG = items_group(c.fmt, G);
  const int P = (c.x_dtype == 0 && !c.w8a8) ? 2 : 1;
  const int max_tokens = 4 / P;
  const int ns = [] {
    const char* s = std::getenv("RTD_GEMV_STAGES");
    const int v = s ? std::atoi(s) : 0;
    return (v >= 2 && v <= kMaxStages) ? v : kMaxStages;
  }();
  size_t need = 0;
  for (int64_t m0 = 0; m0 < c.M;) {
    int Mt = (int)std::min<int64_t>(max_tokens, c.M - m0);
    while (Mt > 1 && make_plan(c.fmt, IG, Mt * P, 8 * ((Mt * P + 7) / 8), ns).smem > 220 * 1024) Mt = (Mt + 1) / 2;
    const int ncol = Mt * P;
    const size_t cols_b = align_up((size_t)G * ncol * col_stride_bytes(f.gk), 256);
    const size_t tab_b = align_up(tab_floats(c.fmt, kp, ncol) * 4 + 4, 256);
    need = std::max(need, cols_b + tab_b + 256);
    m0 += Mt;
  }
  return need;
}

}  // namespace rtd
