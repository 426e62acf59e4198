// rtd_repack.cpp -- host re-tiling of GGUF / E4M3 weight bytes into the device
// group layout described in rtd_layout.h.  A pure permutation of bytes (Q4_K,
// Q8_0, FP8) or of 6-bit codes (Q6_K): no value changes, so the device decoders
// reproduce the reference dequantization bit for bit.  Padding (rows past N, k
// past K) is zero bytes.
#include <cmath>
#include <cstring>
#include <vector>

#include "rtd_layout.h"

namespace rtd {
namespace {

// 6-bit code of element e (0..255) of a Q6_K superblock (dequant_k.rs:87-111):
// half h = e/128, quarter k = (e%128)/32, l = e%32;
// low nibble from ql[64h + l + 32*(k&1)] (high nibble when k >= 2), high 2 bits
// from qh[32h + l] >> 2k.
inline uint32_t q6k_code(const uint8_t* blk, int e) {
  int h = e / 128, rem = e % 128, k = rem / 32, l = rem % 32;
  uint8_t qlb = blk[64 * h + l + 32 * (k & 1)];
  uint32_t lo = (k >= 2) ? (qlb >> 4) : (qlb & 0xF);
  uint32_t hi2 = (blk[128 + 32 * h + l] >> (2 * k)) & 3u;
  return lo | (hi2 << 4);
}

// Codes j = 0..3 of one lane at bit offsets {0, 16, 6, 22}: (w & 0x003F003F) is
// the pair (c0, c1) and ((w >> 6) & 0x003F003F) the pair (c2, c3).
inline uint32_t pack4(const uint32_t c[4]) {
  return c[0] | (c[1] << 16) | (c[2] << 6) | (c[3] << 22);
}

}  // namespace

void repack_host(int fmt, const uint8_t* raw, int64_t N, int64_t K, uint8_t* out) {
  const FmtInfo f = fmt_info(fmt);
  const int64_t T = tiles_for(N);
  const int64_t G = groups_for(fmt, K);
  const size_t total = (size_t)(T * G) * (size_t)f.gb;
  std::memset(out, 0, total);
  const int64_t blocks_per_row = (fmt == FMT_FP8) ? 0 : K / f.block_elems;
  const size_t row_bytes = (fmt == FMT_FP8) ? (size_t)K : (size_t)blocks_per_row * f.block_bytes;
  static const uint8_t zero_block[256] = {0};

  for (int64_t t = 0; t < T; ++t) {
    for (int64_t s = 0; s < G; ++s) {
      uint8_t* grp = out + (size_t)(t * G + s) * f.gb;
      // source pointer of (row r, column s); rows past N read zeros
      auto src = [&](int r) -> const uint8_t* {
        int64_t n = t * 16 + r;
        if (n >= N) return zero_block;
        if (fmt == FMT_FP8) return raw + (size_t)n * row_bytes;  // row start (k offset added below)
        return raw + (size_t)n * row_bytes + (size_t)s * f.block_bytes;
      };
      if (fmt == FMT_Q4K) {
        for (int r = 0; r < 16; ++r) std::memcpy(grp + 16 * r, src(r), 16);
        for (int lane = 0; lane < 32; ++lane) {
          const int g = lane >> 2, tg = lane & 3;
          for (int p = 0; p < 4; ++p)  // row g / g+8, chunk tg bytes 0-15 / 16-31
            std::memcpy(grp + 256 + p * 512 + lane * 16, src(g + 8 * (p >> 1)) + 16 + 32 * tg + 16 * (p & 1), 16);
        }
      } else if (fmt == FMT_Q80) {
        // blocks 4s .. 4s+3 of each row; blocks past K/32 stay zero (d = 0, q = 0)
        const int64_t nblk = K / 32;
        auto blk = [&](int r, int b) -> const uint8_t* {
          const int64_t n = t * 16 + r, bi = 4 * s + b;
          if (n >= N || bi >= nblk) return zero_block;
          return raw + (size_t)n * row_bytes + (size_t)bi * 34;
        };
        for (int lane = 0; lane < 32; ++lane) {
          const int g = lane >> 2, tg = lane & 3;
          std::memcpy(grp + 4 * lane, blk(g, tg), 2);
          std::memcpy(grp + 4 * lane + 2, blk(g + 8, tg), 2);
          for (int p = 0; p < 4; ++p)
            std::memcpy(grp + 128 + p * 512 + lane * 16, blk(g + 8 * (p >> 1), tg) + 2 + 16 * (p & 1), 16);
        }
      } else if (fmt == FMT_FP8) {
        for (int lane = 0; lane < 32; ++lane) {
          const int g = lane >> 2, tg = lane & 3;
          for (int p = 0; p < 4; ++p) {
            const int64_t n = t * 16 + g + 8 * (p >> 1);
            uint8_t* v = grp + p * 512 + lane * 16;
            for (int i = 0; i < 16; ++i) {
              const int64_t k = s * 128 + 32 * tg + 16 * (p & 1) + i;
              v[i] = (n < N && k < K) ? raw[(size_t)n * row_bytes + (size_t)k] : 0;
            }
          }
        }
      } else {  // FMT_Q6K
        for (int g = 0; g < 8; ++g) {
          std::memcpy(grp + 4 * g, src(g) + 208, 2);
          std::memcpy(grp + 4 * g + 2, src(g + 8) + 208, 2);
        }
        for (int lane = 0; lane < 32; ++lane) {
          const int g = lane >> 2, tg = lane & 3;
          for (int rr = 0; rr < 2; ++rr) {
            const uint8_t* sc = src(g + 8 * rr) + 192;
            uint8_t* d = grp + 32 + lane * 8 + 4 * rr;
            d[0] = sc[2 * tg];
            d[1] = sc[2 * tg + 1];
            d[2] = sc[8 + 2 * tg];
            d[3] = sc[9 + 2 * tg];
          }
          uint32_t words[24];
          for (int h = 0; h < 2; ++h)
            for (int tr = 0; tr < 4; ++tr) {  // (g, a), (g+8, a), (g, b), (g+8, b)
              const int row = g + 8 * (tr & 1), sb = 8 * h + 2 * tg + (tr >> 1);
              uint32_t c[16];
              for (int i = 0; i < 16; ++i) c[i] = q6k_code(src(row), 16 * sb + i);
              uint32_t X = pack4(c), Y = pack4(c + 4), Z = pack4(c + 8);
              X |= ((c[12] & 0xFu) << 12) | ((c[13] & 0xFu) << 28);
              Y |= ((c[14] & 0xFu) << 12) | ((c[15] & 0xFu) << 28);
              Z |= ((c[12] >> 4) << 12) | ((c[13] >> 4) << 28) | ((c[14] >> 4) << 14) | ((c[15] >> 4) << 30);
              words[12 * h + 3 * tr + 0] = X;
              words[12 * h + 3 * tr + 1] = Y;
              words[12 * h + 3 * tr + 2] = Z;
            }
          for (int w = 0; w < 24; ++w)
            std::memcpy(grp + 288 + (w / 4) * 512 + lane * 16 + (w % 4) * 4, &words[w], 4);
        }
      }
    }
  }
}

namespace {
float half_bits_to_float(uint16_t h) {
  const uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
  const float v = e == 0 ? std::ldexp((float)m, -24) : e == 31 ? INFINITY : std::ldexp((float)(m | 0x400u), (int)e - 25);
  return (h & 0x8000u) ? -v : v;
}
uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
}  // namespace

float ts_decode_scale(int fmt, const uint8_t* raw, int64_t N, int64_t K) {
  if (fmt == FMT_FP8) return 1.0f;
  const FmtInfo f = fmt_info(fmt);
  const int64_t blocks = N * (K / f.block_elems);
  float mx = 0.0f;  // the largest |factor| a decoder can form
  for (int64_t b = 0; b < blocks; ++b) {
    const uint8_t* p = raw + (size_t)b * (size_t)f.block_bytes;
    float v;
    if (fmt == FMT_Q4K)
      v = 63.0f * std::fmax(std::fabs(half_bits_to_float(rd16(p))), std::fabs(half_bits_to_float(rd16(p + 2))));
    else if (fmt == FMT_Q6K)
      v = 128.0f * std::fabs(half_bits_to_float(rd16(p + 208)));
    else
      v = std::fabs(half_bits_to_float(rd16(p)));
    if (v > mx) mx = v;  // NaN never raises it
  }
  int e = 24;
  if (mx > 0.0f && std::isfinite(mx)) e = (int)std::floor(std::log2(65504.0f / mx));
  if (e > 100) e = 100;
  if (e < -100) e = -100;
  return std::ldexp(1.0f, e);
}

}  // namespace rtd
