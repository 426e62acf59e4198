// rtd_repack.cpp -- host re-tiling of GGUF / E4M3 weight bytes into the device
// group layout described in rtd_layout.h.  A pure permutation of bytes (Q4_K,
// Q8_0, FP8) or of 6-bit codes (Q6_K): no value changes, so the device decoders
// reproduce the reference dequantization bit for bit.
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

// Copy 8 bytes swapping bytes 1 and 2 of each 4-byte word, so that the halves
// of (word & 0x000F000F) are two consecutive elements.
inline void copy8_swapped(uint8_t* dst, const uint8_t* src) {
  for (int w = 0; w < 2; ++w) {
    dst[4 * w + 0] = src[4 * w + 0];
    dst[4 * w + 1] = src[4 * w + 2];
    dst[4 * w + 2] = src[4 * w + 1];
    dst[4 * w + 3] = src[4 * w + 3];
  }
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
        for (int c = 0; c < 4; ++c)
          for (int lane = 0; lane < 32; ++lane) {
            int g = lane >> 2, tg = lane & 3;
            uint8_t* v = grp + 256 + c * 512 + lane * 16;
            copy8_swapped(v, src(g) + 16 + 32 * c + 8 * tg);
            copy8_swapped(v + 8, src(g + 8) + 16 + 32 * c + 8 * tg);
          }
      } else if (fmt == FMT_Q80) {
        for (int r = 0; r < 16; ++r) std::memcpy(grp + 2 * r, src(r), 2);
        for (int lane = 0; lane < 32; ++lane) {
          int g = lane >> 2, tg = lane & 3;
          uint8_t* v = grp + 32 + lane * 16;
          copy8_swapped(v, src(g) + 2 + 8 * tg);
          copy8_swapped(v + 8, src(g + 8) + 2 + 8 * tg);
        }
      } else if (fmt == FMT_FP8) {
        for (int lane = 0; lane < 32; ++lane) {
          int g = lane >> 2, tg = lane & 3;
          uint8_t* v = grp + lane * 16;
          for (int half = 0; half < 2; ++half) {
            int64_t n = t * 16 + g + 8 * half;
            uint8_t nat[8];
            for (int i = 0; i < 8; ++i) {
              int64_t k = s * 32 + 8 * tg + i;
              nat[i] = (n < N && k < K) ? raw[(size_t)n * row_bytes + (size_t)k] : 0;
            }
            copy8_swapped(v + 8 * half, nat);
          }
        }
      } else {  // FMT_Q6K
        for (int r = 0; r < 16; ++r) {
          std::memcpy(grp + 2 * r, src(r) + 208, 2);
          std::memcpy(grp + 32 + 16 * r, src(r) + 192, 16);
        }
        for (int lane = 0; lane < 32; ++lane) {
          int g = lane >> 2, tg = lane & 3;
          uint32_t words[24];
          for (int p = 0; p < 8; ++p) {
            uint32_t ca_g[4], ca_h[4], cb_g[4], cb_h[4];
            for (int j = 0; j < 4; ++j) {
              int ea = 16 * (2 * p) + 4 * tg + j, eb = 16 * (2 * p + 1) + 4 * tg + j;
              ca_g[j] = q6k_code(src(g), ea);
              ca_h[j] = q6k_code(src(g + 8), ea);
              cb_g[j] = q6k_code(src(g), eb);
              cb_h[j] = q6k_code(src(g + 8), eb);
            }
            uint32_t X = pack4(ca_g), Y = pack4(ca_h), Z = pack4(cb_g);
            X |= ((cb_h[0] & 0xFu) << 12) | ((cb_h[1] & 0xFu) << 28);
            Y |= ((cb_h[2] & 0xFu) << 12) | ((cb_h[3] & 0xFu) << 28);
            Z |= ((cb_h[0] >> 4) << 12) | ((cb_h[1] >> 4) << 28) | ((cb_h[2] >> 4) << 14) |
                 ((cb_h[3] >> 4) << 30);
            words[3 * p + 0] = X;
            words[3 * p + 1] = Y;
            words[3 * p + 2] = Z;
          }
          for (int w = 0; w < 24; ++w)
            std::memcpy(grp + 288 + (w / 4) * 512 + lane * 16 + (w % 4) * 4, &words[w], 4);
        }
      }
    }
  }
}

}  // namespace rtd
