// rtd_gemm.cu -- tcgen05 / TMEM tensor-core GEMM for token counts past the decode
// GEMV's sweet spot (prefill, batched decode, speculative verify).
//
//   y[M, N] = x[M, K] . W^T (+ bias)      W in Q4_K / Q6_K / Q8_0 / FP8-E4M3 groups
//
// One CTA computes 128 weight rows (eight 16-row tiles: the UMMA M) x TN tokens (the
// UMMA N, 16..256) with the fp32 accumulator in tensor memory.  Per 64-element k
// stage:
//   - warp 0 (one lane) streams the packed groups of the eight tiles and the stage's
//     activation tile into shared memory with cp.async.bulk (mbarrier transaction
//     counts);
//   - warps 2..9 decode the stage's weights into f16 (the reference formulas in f32,
//     rounded once) straight into the UMMA K-major core-matrix layout;
//   - warp 1 (one lane) issues the four K=16 tcgen05.mma of the stage and commits them
//     to the stage's "empty" barrier, which releases both buffers;
//   - after the last stage warps 4..7 read the accumulator (tcgen05.ld, one TMEM lane
//     quarter each) and write y with the per-token activation scale, the FP8 row
//     scale and the bias.
// The activations are staged once per call by gemm_prep_kernel: power-of-two-scaled
// f16 per token, already in the core-matrix layout, so one bulk copy moves a tile.
// Every wait is bounded by %globaltimer; a timeout records kDevWaitTimeout and the
// CTA stops issuing work, drains what it issued and returns.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "rtd_common.cuh"
#include "rtd_kernels.h"

namespace rtd {
namespace {

constexpr int kGemmWarps = 10;
constexpr int kGemmThreads = kGemmWarps * 32;
constexpr int kDecodeThreads = 256;  // warps 2..9
constexpr int kBM = 128;             // weight rows per CTA (UMMA M)
constexpr int kBK = 64;              // k per stage
constexpr int kStages = 3;
constexpr int kRawSlots = 2;
constexpr int kPrepThreadsG = 256;

template <int FMT>
struct GemmFmt;
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
  const float* row_scale;  // FP8
  int scale_len;
  int64_t N, T, G;         // rows, 16-row tiles, groups per row
  int nkb;                 // 64-element k blocks
  const __half* xw;        // staged activations [nkb][Mp / 8][8 k-cores][8 x 8 f16]
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

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] . B[smem desc]^T, both K-major f16, f32 accumulate.
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Shared-memory matrix descriptor of a K-major, unswizzled f16 operand: 8x8 core
// matrices of 128 contiguous bytes, the two core matrices of one K=16 step 128 bytes
// apart (leading byte offset), successive 8-row groups 1024 bytes apart (stride byte
// offset); descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)(128u >> 4) << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1 << 46;
  return d;  // base offset 0, legacy LBO mode, layout type 0 (no swizzle)
}

// Instruction descriptor: f16 x f16 -> f32, both operands K-major, UMMA M = 128.
__host__ __device__ constexpr uint32_t idesc_f16(int n) {
  return (1u << 4)                          // D format f32
         | (0u << 7) | (0u << 10)           // A, B f16
         | ((uint32_t)(n >> 3) << 17)       // N / 8
         | ((uint32_t)(kBM >> 4) << 24);    // M / 16
}

// Byte offset of element (row r, k) inside a K-major core-matrix tile of 64 k.
__device__ __forceinline__ uint32_t core_off(int r, int k) {
  return (uint32_t)((r >> 3) * 1024 + (k >> 3) * 128 + (r & 7) * 16 + (k & 7) * 2);
}

__device__ __forceinline__ uint32_t pack_f16x2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

__device__ __forceinline__ float hbits(uint32_t b16) { return __half2float(__ushort_as_half((unsigned short)b16)); }

// ---------------------------------------------------------------- stage decode
// Thread dt (0..255) of the decode warps: weight row r = dt / 2 of the CTA tile
// (tile i = r / 16, row rr = r % 16 = g + 8 * hrow), half `part` of its 64 k.
// raw: the eight groups of this stage's k range (group layouts of rtd_layout.h);
// sub: which 64-wide block of the group; a_s: the stage's A tile.
template <int FMT>
__device__ __forceinline__ void decode_stage(const uint8_t* raw, int sub, uint32_t a_s, int dt) {
  constexpr int GB = GemmFmt<FMT>::GB;
  const int r = dt >> 1, part = dt & 1;
  const int i = r >> 4, rr = r & 15, g = rr & 7, hrow = rr >> 3;
  const uint8_t* grp = raw + (size_t)i * GB;
  if constexpr (FMT == FMT_Q4K) {
    // chunk c = sub: low nibbles are sub-block 2c (local k 0..31), high nibbles 2c+1 (32..63)
    const uint8_t* hdr = grp + 16 * rr;
    const uint32_t h0 = *reinterpret_cast<const uint32_t*>(hdr);
    const float d = hbits(h0 & 0xFFFFu), dmin = hbits(h0 >> 16);
    uint32_t sc0, m0, sc1, m1;
    scale_min_k4(2 * sub, hdr + 4, sc0, m0);
    scale_min_k4(2 * sub + 1, hdr + 4, sc1, m1);
    const float d0 = d * (float)sc0, n0 = -(dmin * (float)m0);
    const float d1 = d * (float)sc1, n1 = -(dmin * (float)m1);
    const uint4 q = *reinterpret_cast<const uint4*>(grp + 256 + (2 * hrow + part) * 512 + (4 * g + sub) * 16);
    const uint32_t wd[4] = {q.x, q.y, q.z, q.w};
    uint32_t lo[8], hi[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t w = wd[j >> 1] >> (16 * (j & 1));  // bytes 2j, 2j+1
      const float a0 = (float)(w & 0xF), a1 = (float)((w >> 8) & 0xF);
      const float b0 = (float)((w >> 4) & 0xF), b1 = (float)((w >> 12) & 0xF);
      lo[j] = pack_f16x2(fmaf(d0, a0, n0), fmaf(d0, a1, n0));
      hi[j] = pack_f16x2(fmaf(d1, b0, n1), fmaf(d1, b1, n1));
    }
    const int k0 = 16 * part;
    sts128(a_s + core_off(r, k0), lo[0], lo[1], lo[2], lo[3]);
    sts128(a_s + core_off(r, k0 + 8), lo[4], lo[5], lo[6], lo[7]);
    sts128(a_s + core_off(r, 32 + k0), hi[0], hi[1], hi[2], hi[3]);
    sts128(a_s + core_off(r, 32 + k0 + 8), hi[4], hi[5], hi[6], hi[7]);
  } else if constexpr (FMT == FMT_Q6K) {
    const float d = hbits(*reinterpret_cast<const uint16_t*>(grp + 4 * g + 2 * hrow));
#pragma unroll
    for (int ii = 0; ii < 2; ++ii) {
      const int sb = 4 * sub + 2 * part + ii;  // 16-element sub-block of the superblock
      const int h = sb >> 3, sbi = sb & 7, tq = sbi >> 1, side = sbi & 1;
      const int lane = 4 * g + tq;
      const float ds = d * (float)(int8_t)grp[32 + lane * 8 + 4 * hrow + 2 * h + side];
      const int w0 = 12 * h + 3 * (2 * side + hrow);
      auto word = [&](int w) -> uint32_t {
        return *reinterpret_cast<const uint32_t*>(grp + 288 + (w >> 2) * 512 + lane * 16 + (w & 3) * 4);
      };
      const uint32_t X = word(w0), Y = word(w0 + 1), Z = word(w0 + 2);
      const int sh[4] = {0, 16, 6, 22};
      float v[16];
#pragma unroll
      for (int e = 0; e < 12; ++e) {
        const uint32_t src = e < 4 ? X : (e < 8 ? Y : Z);
        v[e] = ds * (float)((int)((src >> sh[e & 3]) & 63u) - 32);
      }
      v[12] = ds * (float)((int)(((X >> 12) & 15u) | (((Z >> 12) & 3u) << 4)) - 32);
      v[13] = ds * (float)((int)(((X >> 28) & 15u) | (((Z >> 28) & 3u) << 4)) - 32);
      v[14] = ds * (float)((int)(((Y >> 12) & 15u) | (((Z >> 14) & 3u) << 4)) - 32);
      v[15] = ds * (float)((int)(((Y >> 28) & 15u) | (((Z >> 30) & 3u) << 4)) - 32);
      const int k0 = 16 * (2 * part + ii);
      sts128(a_s + core_off(r, k0), pack_f16x2(v[0], v[1]), pack_f16x2(v[2], v[3]), pack_f16x2(v[4], v[5]),
             pack_f16x2(v[6], v[7]));
      sts128(a_s + core_off(r, k0 + 8), pack_f16x2(v[8], v[9]), pack_f16x2(v[10], v[11]),
             pack_f16x2(v[12], v[13]), pack_f16x2(v[14], v[15]));
    }
  } else {  // Q8_0 / FP8: block b = 2 * sub + part of the group, local k 32 * part ..
    const int lane = 4 * g + 2 * sub + part;
    float dq = 1.0f;
    if constexpr (FMT == FMT_Q80) dq = hbits(*reinterpret_cast<const uint16_t*>(grp + 4 * lane + 2 * hrow));
    constexpr int base = (FMT == FMT_Q80) ? 128 : 0;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const uint4 q = *reinterpret_cast<const uint4*>(grp + base + (2 * hrow + half) * 512 + lane * 16);
      const uint32_t wd[4] = {q.x, q.y, q.z, q.w};
      uint32_t o[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if constexpr (FMT == FMT_Q80) {
          const int8_t* b = reinterpret_cast<const int8_t*>(&wd[j]);
          o[2 * j] = pack_f16x2(dq * (float)b[0], dq * (float)b[1]);
          o[2 * j + 1] = pack_f16x2(dq * (float)b[2], dq * (float)b[3]);
        } else {
          o[2 * j] = e4m3x2_to_f16x2((uint16_t)(wd[j] & 0xFFFFu));
          o[2 * j + 1] = e4m3x2_to_f16x2((uint16_t)(wd[j] >> 16));
        }
      }
      const int k0 = 32 * part + 16 * half;
      sts128(a_s + core_off(r, k0), o[0], o[1], o[2], o[3]);
      sts128(a_s + core_off(r, k0 + 8), o[4], o[5], o[6], o[7]);
    }
  }
}

// ---------------------------------------------------------------- GEMM kernel
template <int FMT, int TN>
struct GemmSmem {
  static constexpr int kA = kBM * kBK * 2;                  // 16 KB
  static constexpr int kB = TN * kBK * 2;                   // TN * 128
  static constexpr int kRaw = 8 * GemmFmt<FMT>::GB;
  static constexpr int offA = 0;
  static constexpr int offB = offA + kStages * kA;
  static constexpr int offRaw = offB + kStages * kB;
  static constexpr int offBar = (offRaw + kRawSlots * kRaw + 127) / 128 * 128;
  static constexpr int nBars = 2 * kRawSlots + 3 * kStages + 1;
  static constexpr int offMisc = offBar + nBars * 8;
  static constexpr int bytes = offMisc + 16 + 1024;          // + alignment slack
};

template <int FMT, int TN>
__global__ void __launch_bounds__(kGemmThreads, 1) qgemm_kernel(const GemmArgs a) {
  using L = GemmSmem<FMT, TN>;
  constexpr int SPG = GemmFmt<FMT>::GK / kBK;  // stages per group
  constexpr int GB = GemmFmt<FMT>::GB;
  constexpr uint32_t kCols = TN < 32 ? 32 : TN;
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
      mbar_init(&raw_empty[s], kDecodeThreads);
    }
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&a_full[s], kDecodeThreads);
      mbar_init(&st_empty[s], 1);
    }
    mbar_init(acc_full, 1);
    misc[1] = 0;
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc[0];
  volatile uint32_t* abort_flag = &misc[1];

  auto wait = [&](uint64_t* b, uint32_t parity) -> bool {
    if (*abort_flag) return false;
    if (mbar_wait_ns(b, parity, kWaitBudgetNs, a.status)) return true;
    *abort_flag = 1;
    return false;
  };

  if (warp == 0) {
    // ---- producer: packed groups (per group) and activation tiles (per stage)
    if (lane == 0) {
      const uint8_t* xw = reinterpret_cast<const uint8_t*>(a.xw);
      const int64_t ntile = (a.T - tile0 < 8) ? a.T - tile0 : 8;
      int groups = 0, stages = 0;  // copies issued so far
      for (int kb = 0; kb < nkb; ++kb) {
        if (kb % SPG == 0) {
          const int s = kb / SPG, rs = s % kRawSlots;
          if (s >= kRawSlots && !wait(&raw_empty[rs], (uint32_t)((s / kRawSlots - 1) & 1))) break;
          mbar_arrive_expect_tx(&raw_full[rs], (uint32_t)(ntile * GB));
          for (int64_t i = 0; i < ntile; ++i)
            bulk_g2s(sm + L::offRaw + rs * L::kRaw + i * GB, a.w + ((tile0 + i) * a.G + g_lo + s) * GB, GB,
                     &raw_full[rs]);
          ++groups;
        }
        const int st = kb % kStages;
        if (kb >= kStages && !wait(&st_empty[st], (uint32_t)((kb / kStages - 1) & 1))) break;
        mbar_arrive_expect_tx(&b_full[st], (uint32_t)L::kB);
        bulk_g2s(sm + L::offB + st * L::kB, xw + ((size_t)(kb0 + kb) * (a.Mp / 8) + (size_t)(t0 / 8)) * 1024,
                 L::kB, &b_full[st]);
        ++stages;
      }
      if (*abort_flag) {  // no copy may still be landing when the CTA exits
        for (int s = (groups > kRawSlots ? groups - kRawSlots : 0); s < groups; ++s)
          mbar_wait_ns(&raw_full[s % kRawSlots], (uint32_t)((s / kRawSlots) & 1), kWaitBudgetNs, a.status);
        for (int kb = (stages > kStages ? stages - kStages : 0); kb < stages; ++kb)
          mbar_wait_ns(&b_full[kb % kStages], (uint32_t)((kb / kStages) & 1), kWaitBudgetNs, a.status);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(TN);
      for (int kb = 0; kb < nkb; ++kb) {
        const int st = kb % kStages;
        const uint32_t ph = (uint32_t)((kb / kStages) & 1);
        if (!wait(&a_full[st], ph) || !wait(&b_full[st], ph)) break;
        tc_fence_after();
        const uint32_t as = smem_u32(sm + L::offA + st * L::kA), bs = smem_u32(sm + L::offB + st * L::kB);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          umma_f16(tmem, kmajor_desc(as + kk * 256), kmajor_desc(bs + kk * 256), idesc, (kb | kk) ? 1u : 0u);
        umma_commit(&st_empty[st]);
      }
      umma_commit(acc_full);  // fires once every MMA issued above has completed
    }
  } else {
    // ---- decode warps (and, afterwards, warps 4..7 run the epilogue)
    const int dt = tid - 64;
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb / SPG, sub = kb % SPG, rs = s % kRawSlots;
      if (sub == 0 && !wait(&raw_full[rs], (uint32_t)((s / kRawSlots) & 1))) break;
      const int st = kb % kStages;
      if (kb >= kStages && !wait(&st_empty[st], (uint32_t)((kb / kStages - 1) & 1))) break;
      decode_stage<FMT>(sm + L::offRaw + rs * L::kRaw, sub, smem_u32(sm + L::offA + st * L::kA), dt);
      fence_async_shared();  // the tensor cores read A through the async proxy
      mbar_arrive(&a_full[st]);
      if (sub == SPG - 1) mbar_arrive(&raw_empty[rs]);
    }
    if (warp >= 4 && warp < 8) {
      const int q = warp - 4;  // TMEM lanes 32q .. 32q+31 = weight rows of this warp
      const bool ok = wait(acc_full, 0u);
      tc_fence_after();
      const int r = q * 32 + lane;
      const int64_t n = tile0 * 16 + r;
      float es = 1.0f, eb = 0.0f;
      if (n < a.N) {
        if (FMT == FMT_FP8) es = a.row_scale[a.scale_len == 1 ? 0 : n];
        if (a.bias) eb = a.bias[n];
      }
#pragma unroll 1
      for (int c0 = 0; c0 < TN; c0 += 8) {
        float v[8];
        tmem_ld8(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
        if (!ok) continue;
        if (a.splits > 1) {  // partial sums of this k split; the reduce kernel finishes them
          if (n < a.N) {
            float* pp = a.partial + ((size_t)blockIdx.z * a.Mp + (size_t)(t0 + c0)) * a.N + n;
#pragma unroll
            for (int j = 0; j < 8; ++j) pp[(size_t)j * a.N] = v[j];
          }
          continue;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int64_t t = t0 + c0 + j;
          if (n < a.N && t < a.M) {
            const float val = v[j] * a.tscale[t] * es + eb;
            const int64_t off = t * a.ldy + n;
            if (a.y_dtype == 0)
              static_cast<float*>(a.y)[off] = val;
            else if (a.y_dtype == 1)
              static_cast<__half*>(a.y)[off] = __float2half_rn(val);
            else
              static_cast<__nv_bfloat16*>(a.y)[off] = __float2bfloat16_rn(val);
          }
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
// goes to the core-matrix layout [kb][Mp/8][8 k-cores][8 rows x 8 k]; tokens past M
// and k past K are zero.  W8A8 rounds x with the reference E4M3 encoder first.
__global__ void __launch_bounds__(kPrepThreadsG) gemm_prep_kernel(const void* x, int x_dtype, int64_t ldx,
                                                                  int64_t M, int64_t Mp, int64_t K, int64_t kp,
                                                                  int w8a8, __half* xw, float* tscale) {
  const int64_t t = blockIdx.x;
  __shared__ float red[kPrepThreadsG / 32];
  auto load = [&](int64_t k) -> float {
    if (t >= M || k >= K) return 0.0f;
    float v;
    if (x_dtype == 0)
      v = static_cast<const float*>(x)[t * ldx + k];
    else {
      const unsigned short b = static_cast<const unsigned short*>(x)[t * ldx + k];
      v = (x_dtype == 1) ? __half2float(__ushort_as_half(b)) : __uint_as_float((uint32_t)b << 16);
    }
    return w8a8 ? e4m3_round_ref(v) : v;
  };
  float m = 0.0f;
  for (int64_t k = threadIdx.x; k < K; k += kPrepThreadsG) m = fmaxf(m, fabsf(load(k)));
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
  for (int64_t c = threadIdx.x; c < kp / 8; c += kPrepThreadsG) {  // 8 consecutive k per thread
    const int64_t k = 8 * c, kb = k / 64, kc = (k % 64) / 8;
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = pack_f16x2(load(k + 2 * j) * inv, load(k + 2 * j + 1) * inv);
    uint8_t* dst = reinterpret_cast<uint8_t*>(xw) + (((size_t)kb * (Mp / 8) + (size_t)tg) * 8 + (size_t)kc) * 128 +
                   (size_t)r * 16;
    *reinterpret_cast<uint4*>(dst) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// y[t, n] = sum over splits of the partials, scaled and biased as the GEMM epilogue does.
__global__ void gemm_reduce_kernel(const float* partial, int splits, int64_t Mp, int64_t M, int64_t N,
                                   const float* tscale, const float* row_scale, int scale_len, const float* bias,
                                   void* y, int y_dtype, int64_t ldy) {
  const int64_t total = M * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / N, n = i - t * N;
    float v = 0.0f;
    for (int z = 0; z < splits; ++z) v += partial[((size_t)z * Mp + (size_t)t) * N + n];
    v *= tscale[t];
    if (row_scale) v *= row_scale[scale_len == 1 ? 0 : n];
    if (bias) v += bias[n];
    const int64_t off = t * ldy + n;
    if (y_dtype == 0)
      static_cast<float*>(y)[off] = v;
    else if (y_dtype == 1)
      static_cast<__half*>(y)[off] = __float2half_rn(v);
    else
      static_cast<__nv_bfloat16*>(y)[off] = __float2bfloat16_rn(v);
  }
}

template <int FMT, int TN>
cudaError_t launch_gemm_tn(const GemmArgs& a, cudaStream_t st) {
  using L = GemmSmem<FMT, TN>;
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(qgemm_kernel<FMT, TN>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::bytes);
    if (e != cudaSuccess) return e;
    configured[dev & 63] = 1;
  }
  const dim3 grid((unsigned)(a.Mp / TN), (unsigned)((a.T + 7) / 8), (unsigned)a.splits);
  qgemm_kernel<FMT, TN><<<grid, kGemmThreads, L::bytes, st>>>(a);
  return cudaGetLastError();
}

template <int FMT>
cudaError_t launch_gemm_fmt(const GemmArgs& a, int TN, cudaStream_t st) {
  switch (TN) {
    case 16: return launch_gemm_tn<FMT, 16>(a, st);
    case 32: return launch_gemm_tn<FMT, 32>(a, st);
    case 64: return launch_gemm_tn<FMT, 64>(a, st);
    case 128: return launch_gemm_tn<FMT, 128>(a, st);
    default: return launch_gemm_tn<FMT, 256>(a, st);
  }
}

int gemm_tn_for(int64_t M) {
  if (M <= 16) return 16;
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  if (M <= 128) return 128;
  return 256;
}

// K splits: enough CTAs for one wave over the SMs (one CTA per SM fits in shared
// memory), whole groups per split, at least two groups each.
int gemm_splits(const QGemvCall& c, int TN) {
  const int64_t ctas = ((c.M + TN - 1) / TN) * ((tiles_for(c.N) + 7) / 8);
  const int64_t want = (c.sm_count + ctas - 1) / ctas;
  const int64_t most = std::max<int64_t>(1, c.G / 2);
  return (int)std::max<int64_t>(1, std::min<int64_t>(want, most));
}

struct GemmPlan {
  int TN, splits;
  int64_t Mp, kp;
  size_t xw_bytes, partial_bytes;
};

GemmPlan gemm_plan(const QGemvCall& c) {
  GemmPlan p{};
  const FmtInfo f = fmt_info(c.fmt);
  p.TN = gemm_tn_for(c.M);
  p.Mp = (c.M + p.TN - 1) / p.TN * p.TN;
  p.kp = c.G * f.gk;
  p.splits = gemm_splits(c, p.TN);
  p.xw_bytes = (size_t)p.Mp * (size_t)p.kp * 2;
  p.partial_bytes = p.splits > 1 ? (size_t)p.splits * (size_t)p.Mp * (size_t)c.N * 4 : 0;
  return p;
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
  if (qgemm_workspace_bytes(c) > c.ws_bytes || Mp / TN > 65535) {
    *plan_error = 1;
    return cudaSuccess;
  }
  uint8_t* ws = reinterpret_cast<uint8_t*>(c.ws);
  __half* xw = reinterpret_cast<__half*>(ws);
  float* tscale = reinterpret_cast<float*>(ws + p.xw_bytes);
  float* partial = reinterpret_cast<float*>(ws + p.xw_bytes + (((size_t)Mp * 4 + 255) / 256) * 256);
  gemm_prep_kernel<<<(unsigned)Mp, kPrepThreadsG, 0, c.stream>>>(c.x, c.x_dtype, c.ldx, c.M, Mp, c.K, kp, c.w8a8,
                                                                  xw, tscale);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  GemmArgs a{};
  a.w = c.w;
  a.row_scale = c.row_scale;
  a.scale_len = c.scale_len;
  a.N = c.N;
  a.T = tiles_for(c.N);
  a.G = c.G;
  a.nkb = (int)(kp / kBK);
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
    case FMT_Q4K: e = launch_gemm_fmt<FMT_Q4K>(a, TN, c.stream); break;
    case FMT_Q6K: e = launch_gemm_fmt<FMT_Q6K>(a, TN, c.stream); break;
    case FMT_Q80: e = launch_gemm_fmt<FMT_Q80>(a, TN, c.stream); break;
    default: e = launch_gemm_fmt<FMT_FP8>(a, TN, c.stream); break;
  }
  if (e != cudaSuccess || p.splits == 1) return e;
  const int64_t total = c.M * c.N;
  const unsigned blocks = (unsigned)std::min<int64_t>((total + 255) / 256, 4096);
  gemm_reduce_kernel<<<blocks, 256, 0, c.stream>>>(partial, p.splits, Mp, c.M, c.N, tscale,
                                                   c.fmt == FMT_FP8 ? c.row_scale : nullptr, c.scale_len, c.bias,
                                                   c.y, c.y_dtype, c.ldy);
  return cudaGetLastError();
}

}  // namespace rtd
