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
// 16-byte aligned byte range -- a single cp.async.bulk.
//
// Inside a K-quant group every warp lane (lane = 4*g + t) owns WHOLE sub-blocks
// of rows g and g+8: the m16n8k16 decode GEMV then sums each sub-block in its own
// MMA output column (see rtd_gemv.cu), and a lane only ever needs the scales of
// the sub-blocks it owns.  A lane's bytes sit in 16-byte vectors, one per "pass":
// pass p occupies bytes [p*512, p*512+512) of the code region, lane L at L*16.
//
//   Q4_K  GK=256 GB=2304: [16 rows x (d, dmin, scales[12]) = 256 B, GGUF order]
//                         [qs: pass(4) x lane(32) x 16 B]
//         lane t owns qs chunk t (bytes 32t..32t+31: sub-blocks 2t (low nibbles)
//         and 2t+1 (high nibbles)); passes 0,1 = row g bytes 0-15, 16-31;
//         passes 2,3 = row g+8.
//   Q6_K  GK=256 GB=3360: [d: 8 x (row g, row g+8) f16 = 32 B]
//                         [scales: lane(32) x (row g 4 B, row g+8 4 B)]
//                         [codes: pass(6) x lane(32) x 16 B]
//         lane t owns sub-blocks 2t, 2t+1, 8+2t, 9+2t; its scale bytes are
//         sc[2t], sc[2t+1], sc[8+2t], sc[9+2t] of each row.  Codes: one 3-word
//         triple per (row, sub-block) -- see below -- ordered half h (passes
//         3h..3h+2): (row g, 8h+2t), (row g+8, 8h+2t), (row g, 8h+2t+1),
//         (row g+8, 8h+2t+1).
//   Q8_0  GK=128 GB=2176: [d: lane(32) x (row g, row g+8) f16 = 128 B]
//                         [qs: pass(4) x lane(32) x 16 B]
//         lane t owns block t of the group (32 int8); passes as for Q4_K.
//         K is a multiple of 32; a trailing partial group is zero-filled.
//   FP8   GK=128 GB=2048: [codes: pass(4) x lane(32) x 16 B]
//         lane t owns the 32 E4M3 codes k = 32t..32t+31 of the group; passes as
//         for Q4_K.  The per-row scales live in a separate f32 array.
//
// Q6_K code triples.  The 6-bit code of element e of a superblock row is
// (ql nibble | 2 qh bits << 4), dequant_k.rs:87-111.  The 16 codes c0..c15 of one
// (row, sub-block) fill three words:
//   X = c0@0 c1@16 c2@6 c3@22,  Y = c4..c7 likewise,  Z = c8..c11 likewise,
//   spare bits: X 12-15 / 28-31 = low nibbles of c12 / c13, Y 12-15 / 28-31 = low
//   nibbles of c14 / c15, Z 12-13 / 28-29 / 14-15 / 30-31 = high 2 bits of c12 /
//   c13 / c14 / c15.
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
    case FMT_Q80: return FmtInfo{128, 2176, 32, 32, 34};
    default:      return FmtInfo{128, 2048, 32, 1, 1};
  }
}

// Offset of the A-fragment region inside a group.
RTD_HD inline int group_payload_offset(int fmt) {
  switch (fmt) {
    case FMT_Q4K: return 256;
    case FMT_Q6K: return 288;
    case FMT_Q80: return 128;
    default:      return 0;
  }
}

// Host-side re-tiling (rtd_repack.cpp).  `raw` holds N rows of GGUF blocks
// (or E4M3 bytes, K per row, for FP8); `out` has tiles*groups*GB bytes.
void repack_host(int fmt, const uint8_t* raw, int64_t N, int64_t K, uint8_t* out);

// Power of two F = 2^e for the skinny GEMM's decoders: the largest with every scaled factor
// (Q4_K d * sc and dmin * m, Q6_K d * sc, Q8_0 d, times F) inside the f16 range, from
// the raw GGUF blocks.  1 for FP8 (its decoder needs no factor).
float ts_decode_scale(int fmt, const uint8_t* raw, int64_t N, int64_t K);

// Number of tiles / groups for a matrix.
inline int64_t tiles_for(int64_t N) { return (N + 15) / 16; }
inline int64_t groups_for(int fmt, int64_t K) {
  FmtInfo f = fmt_info(fmt);
  return (K + f.gk - 1) / f.gk;
}

}  // namespace rtd
