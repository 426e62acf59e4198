// rtd_layout.h -- device layout of uploaded weights (shared by host and device code).
//
// GGUF stores an [N, K] quantized matrix as N rows of K/elems raw blocks
// (crates/runtimed-gguf/src/header.rs:191-205; [N, K] = [dims[1], dims[0]] per
// crates/runtimed-model/src/weights/load_gguf.rs:35).  On upload the library
// re-tiles the bytes, without changing any value, into GROUPS:
//
//   group (tile t, column s) = rows 16t .. 16t+15  x  GK consecutive k
//   device buffer            = [tile][column][group bytes], rows past N zero-filled
//
// so that one unit of GEMV work (a tile x a run of columns) is ONE contiguous,
// 16-byte aligned byte range -- a single cp.async.bulk -- and, inside a group,
// every warp lane finds the bytes of its m16n8k16 A fragment in one 16-byte
// vector (lane = 4*g + t holds rows g and g+8).
//
//   Q4_K  GK=256 GB=2304: [16 rows x (d, dmin, scales[12]) = 256 B]
//                         [qs: chunk c(4) x lane(32) x 16 B]
//                         lane 16 B = row g qs[32c+8t .. +8] ++ row g+8 qs[32c+8t .. +8]
//   Q6_K  GK=256 GB=3360: [d: 16 x 2 B][scales: 16 x 16 B]
//                         [codes: vec v(6) x lane(32) x 16 B]  (24 words per lane, see below)
//   Q8_0  GK=32  GB=544:  [d: 16 x 2 B][qs: lane(32) x 16 B, row g bytes 8t..8t+7 ++ row g+8]
//   FP8   GK=32  GB=512:  [lane(32) x 16 B, row g bytes 8t..8t+7 ++ row g+8]
//
// Q6_K code words.  The 6-bit code of element e of a superblock row is
// (ql nibble | 2 qh bits << 4), dequant_k.rs:87-111.  Sub-block sb (16 elements,
// scale index sb) is split 4 codes per lane: lane t holds elements 16*sb+4t+{0..3}.
// Window p (sub-blocks a=2p, b=2p+1) uses lane words 3p..3p+2 (X, Y, Z):
//   X = codes (a, row g):   c0@0 c1@6 c2@16 c3@22 ; spare 12-15, 28-31 = low nibbles of (b, g+8) c0, c2
//   Y = codes (a, row g+8): same ; spare = low nibbles of (b, g+8) c1, c3
//   Z = codes (b, row g):   same ; spare 12-13/14-15/28-29/30-31 = high 2 bits of (b, g+8) c0/c1/c2/c3
#pragma once

#include <stddef.h>
#include <stdint.h>

namespace rtd {

enum Fmt : int { FMT_Q4K = 0, FMT_Q6K = 1, FMT_Q80 = 2, FMT_FP8 = 3 };

struct FmtInfo {
  int gk;          // k elements per group
  int gb;          // bytes per group (16 rows)
  int sbe;         // sub-block size (elements per scale)
  int block_elems; // GGUF block: elements
  int block_bytes; // GGUF block: bytes
};

#if defined(__CUDACC__)
#define RTD_HD __host__ __device__
#else
#define RTD_HD
#endif

RTD_HD inline FmtInfo fmt_info(int fmt) {
  switch (fmt) {
    case FMT_Q4K: return FmtInfo{256, 2304, 32, 256, 144};
    case FMT_Q6K: return FmtInfo{256, 3360, 16, 256, 210};
    case FMT_Q80: return FmtInfo{32, 544, 32, 32, 34};
    default:      return FmtInfo{32, 512, 32, 1, 1};
  }
}

// Offset of the A-fragment region inside a group.
RTD_HD inline int group_payload_offset(int fmt) {
  switch (fmt) {
    case FMT_Q4K: return 256;
    case FMT_Q6K: return 288;
    case FMT_Q80: return 32;
    default:      return 0;
  }
}

// Host-side re-tiling (rtd_repack.cpp).  `raw` holds N rows of GGUF blocks
// (or E4M3 bytes, K per row, for FP8); `out` has tiles*groups*GB bytes.
void repack_host(int fmt, const uint8_t* raw, int64_t N, int64_t K, uint8_t* out);

// Number of tiles / groups for a matrix.
inline int64_t tiles_for(int64_t N) { return (N + 15) / 16; }
inline int64_t groups_for(int fmt, int64_t K) {
  FmtInfo f = fmt_info(fmt);
  return (K + f.gk - 1) / f.gk;
}

}  // namespace rtd
