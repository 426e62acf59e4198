// rtd_common.cuh -- device helpers shared by the sm_100a kernels of libruntimed_b200.
//
// Inline PTX for the Blackwell data-movement primitives the kernels use
// (mbarrier + cp.async.bulk global->shared), the LL words of the cross-GPU
// exchanges, the m16n8k16 tensor-core MMA used by the decode GEMV, and bit-exact
// scalar conversions.
#pragma once

#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "rtd_layout.h"

namespace rtd {

// Device status word codes (mirrors RTD_ERR_* of include/rtd.h).
enum : int { kDevOk = 0, kDevPeerTimeout = 7, kDevIndex = 8, kDevWaitTimeout = 9 };

__device__ __forceinline__ void raise_status(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the warp sleeps in hardware until the phase
// completes (or about `hint_ns` passes) instead of spinning on issue slots.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait on an mbarrier phase: gives up after `budget_ns` of wall time
// (read from %globaltimer), records kDevWaitTimeout in the device status word and
// returns false.  Callers stop issuing copies after a failure and drain what is
// already in flight with a second bounded wait, so no CTA exits with a copy still
// heading for its shared memory and no wait can hold the GPU indefinitely.
__device__ __forceinline__ bool mbar_wait_ns(uint64_t* bar, uint32_t parity, uint64_t budget_ns, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    if (mbar_try_wait_sleep(bar, parity, 100000u)) return true;
    if (global_ns() - t0 > budget_ns) {
      raise_status(status, kDevWaitTimeout);
      return false;
    }
  }
}

constexpr uint64_t kWaitBudgetNs = 2000000000ull;  // 2 s: far beyond any legitimate copy latency

__device__ __forceinline__ void mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* status) {
  if (!mbar_wait_ns(bar, parity, kWaitBudgetNs, status)) mbar_wait_ns(bar, parity, kWaitBudgetNs, status);
}

// 1-D bulk copy global -> shared (TMA engine), completion counted in bytes on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------- cross-GPU LL words
// A value travels between GPUs as one 8-byte word: the f32 bits in the low half and
// the exchange epoch in the high half.  An aligned 8-byte relaxed store is single-copy
// atomic, so a reader that sees the epoch it waits for also sees the value stored with
// it: no fence and no separate flag are needed.  Buffers start zeroed and epochs start
// at 1, and every exchange alternates between two buffer halves by epoch parity, so a
// word left from an earlier exchange never carries the epoch a reader waits for.
__device__ __forceinline__ uint64_t ll_word(float v, uint32_t epoch) {
  return ((uint64_t)epoch << 32) | (uint64_t)__float_as_uint(v);
}

__device__ __forceinline__ void st_ll(uint64_t* p, float v, uint32_t epoch) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(ll_word(v, epoch)) : "memory");
}

// Two consecutive words (16-byte aligned); each 8-byte half is single-copy atomic.
__device__ __forceinline__ void st_ll2(uint64_t* p, float v0, float v1, uint32_t epoch) {
  asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(ll_word(v0, epoch)),
               "l"(ll_word(v1, epoch))
               : "memory");
}

__device__ __forceinline__ uint64_t ld_ll(const uint64_t* p) {
  uint64_t w;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}

__device__ __forceinline__ void ld_ll2(const uint64_t* p, uint64_t& w0, uint64_t& w1) {
  asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(w0), "=l"(w1) : "l"(p) : "memory");
}

// Waits (bounded) for the word at p to carry `epoch` and returns its value.  After one
// timeout in this thread (`dead`), later waits return 0 at once, so a peer that never
// arrives costs one wait budget per thread, not one per word.
__device__ __forceinline__ float wait_ll(const uint64_t* p, uint32_t epoch, bool& dead, int* status) {
  uint64_t w = ld_ll(p);
  if ((uint32_t)(w >> 32) == epoch) return __uint_as_float((uint32_t)w);
  if (dead) return 0.0f;
  const uint64_t t0 = global_ns();
  for (;;) {
    __nanosleep(20);
    w = ld_ll(p);
    if ((uint32_t)(w >> 32) == epoch) return __uint_as_float((uint32_t)w);
    if (global_ns() - t0 > 2000000000ull) {
      raise_status(status, kDevPeerTimeout);
      dead = true;
      return 0.0f;
    }
  }
}

__device__ __forceinline__ void wait_ll2(const uint64_t* p, uint32_t epoch, bool& dead, int* status, float& v0,
                                         float& v1) {
  uint64_t w0, w1;
  ld_ll2(p, w0, w1);
  if ((uint32_t)(w0 >> 32) != epoch || (uint32_t)(w1 >> 32) != epoch) {
    if (dead) {
      v0 = v1 = 0.0f;
      return;
    }
    const uint64_t t0 = global_ns();
    for (;;) {
      __nanosleep(20);
      ld_ll2(p, w0, w1);
      if ((uint32_t)(w0 >> 32) == epoch && (uint32_t)(w1 >> 32) == epoch) break;
      if (global_ns() - t0 > 2000000000ull) {
        raise_status(status, kDevPeerTimeout);
        dead = true;
        v0 = v1 = 0.0f;
        return;
      }
    }
  }
  v0 = __uint_as_float((uint32_t)w0);
  v1 = __uint_as_float((uint32_t)w1);
}

// ---------------------------------------------------------------- MMA
// D = A(16x16, f16, row) * B(16x8, f16, col) + C, f32 accumulate.
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1, float c0, float c1, float c2, float c3) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c0), "f"(c1), "f"(c2), "f"(c3));
}

// D += A(16x16, f16, row) * B(16x8, f16, col), accumulating in place (f32).
__device__ __forceinline__ void mma_f16_acc(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                            uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t mask, uint32_t orv) {
  return (a & mask) | orv;  // compiles to one LOP3
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  return __byte_perm(a, b, sel);
}

// Two E4M3 bytes (low byte -> low half) -> f16x2, exact.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t v) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(v));
  return r;
}

// ---------------------------------------------------------------- scalar
// IEEE half bits -> float, bit-exact with the reference decoder for every input
// (subnormals normalised, NaN payload kept): dequant.rs:11-33.
__device__ __forceinline__ float f16_bits_to_f32(uint32_t bits) {
  uint32_t sign = (bits >> 15) & 1u, exp = (bits >> 10) & 0x1Fu, mant = bits & 0x3FFu, out;
  if (exp == 0) {
    if (mant == 0) {
      out = sign << 31;
    } else {
      int sh = __clz(mant) - 21;  // shifts until bit 10 is set
      uint32_t m = mant << sh;
      uint32_t e = 113u - (uint32_t)sh;
      out = (sign << 31) | (e << 23) | ((m & 0x3FFu) << 13);
    }
  } else if (exp == 31) {
    out = (sign << 31) | (0xFFu << 23) | (mant << 13);
  } else {
    out = (sign << 31) | ((exp + 112u) << 23) | (mant << 13);
  }
  return __uint_as_float(out);
}

__device__ __forceinline__ float ld_f16(const uint8_t* p) {
  return f16_bits_to_f32((uint32_t)p[0] | ((uint32_t)p[1] << 8));
}

// Q4_K scale/min pair j of the 12 packed scale bytes: dequant_k.rs:8-16.
__device__ __forceinline__ void scale_min_k4(int j, const uint8_t* s, uint32_t& sc, uint32_t& m) {
  if (j < 4) {
    sc = s[j] & 63u;
    m = s[j + 4] & 63u;
  } else {
    sc = (s[j + 4] & 0xFu) | ((uint32_t)(s[j - 4] >> 6) << 4);
    m = (uint32_t)(s[j + 4] >> 4) | ((uint32_t)(s[j] >> 6) << 4);
  }
}

// E4M3 value of the reference encoder (load_safetensors.rs:53-69): nearest grid
// point, a tie goes to the lower magnitude, |x| >= 448 saturates, NaN stays NaN.
__device__ __forceinline__ float e4m3_round_ref(float x) {
  if (isnan(x)) return x;
  float a = fabsf(x);
  float v;
  if (a >= 448.0f) {
    v = 448.0f;
  } else if (a == 0.0f) {
    v = 0.0f;
  } else {
    int e = ilogbf(a);
    if (e < -6) e = -6;
    float spacing = ldexpf(1.0f, e - 3);
    float q = a / spacing;  // exact: power-of-two divisor
    float n = floorf(q);
    if (q - n > 0.5f) n += 1.0f;
    v = n * spacing;
  }
  return copysignf(v, x);
}

__device__ __forceinline__ uint8_t e4m3_code_of_value(float v) {
  if (isnan(v)) return 0x7f;
  uint8_t sign = signbit(v) ? 0x80 : 0x00;
  float a = fabsf(v);
  if (a == 0.0f) return sign;
  int e = ilogbf(a);
  if (e < -6) return sign | (uint8_t)(a * 512.0f);  // subnormal: multiples of 2^-9
  uint32_t mant = (uint32_t)((ldexpf(a, -e) - 1.0f) * 8.0f);
  return sign | (uint8_t)(((e + 7) << 3) | mant);
}

}  // namespace rtd
