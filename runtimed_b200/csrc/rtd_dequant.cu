// rtd_dequant.cu -- bit-exact decode of uploaded weights (whole matrix and row
// gather) and the device E4M3 encoder.
//
// The arithmetic follows the reference decoders operation for operation, with
// explicitly rounded multiplies/subtracts so nvcc cannot contract into FMA:
//   Q4_K  value = (d*sc)*q - dmin*m        crates/runtimed-gguf/src/quant/dequant_k.rs:19-44
//   Q6_K  value = (d*sc)*(code - 32)       dequant_k.rs:87-111
//   Q8_0  value = d*q                      crates/runtimed-gguf/src/quant/dequant.rs:40-47
//   FP8   value = E4M3 table entry         crates/runtimed-model/src/weights/load_safetensors.rs:14-29
#include "rtd_common.cuh"
#include "rtd_kernels.h"

namespace rtd {

__device__ __forceinline__ uint32_t ld_u32(const uint8_t* a) {
  return (uint32_t)a[0] | ((uint32_t)a[1] << 8) | ((uint32_t)a[2] << 16) | ((uint32_t)a[3] << 24);
}

// Decode element (row r in 0..15, element e in 0..gk-1) of one group (layouts in
// rtd_layout.h: lane 4g+t owns whole sub-blocks of rows g and g+8).
template <int FMT>
__device__ __forceinline__ float decode_elem(const uint8_t* grp, int r, int e) {
  const int g = r & 7, rr = r >> 3;
  if constexpr (FMT == FMT_Q4K) {
    const uint8_t* hdr = grp + 16 * r;
    const float d = ld_f16(hdr), dmin = ld_f16(hdr + 2);
    const int c = e >> 6, rem = e & 63, j = rem & 31;
    const bool low = rem < 32;
    uint32_t sc, m;
    scale_min_k4(2 * c + (low ? 0 : 1), hdr + 4, sc, m);
    const float d1 = __fmul_rn(d, (float)sc);
    const float m1 = __fmul_rn(dmin, (float)m);
    const uint8_t byte = grp[256 + (2 * rr + (j >> 4)) * 512 + (4 * g + c) * 16 + (j & 15)];
    const float q = (float)(low ? (byte & 0xF) : (byte >> 4));
    return __fsub_rn(__fmul_rn(d1, q), m1);
  } else if constexpr (FMT == FMT_Q6K) {
    const float d = ld_f16(grp + 4 * g + 2 * rr);
    const int sb = e >> 4, i = e & 15;
    const int h = sb >> 3, t = (sb & 7) >> 1, side = sb & 1;
    const int lane = 4 * g + t;
    const int8_t sc = (int8_t)grp[32 + lane * 8 + 4 * rr + 2 * h + side];
    const int w0 = 12 * h + 3 * (2 * side + rr);  // first word of this (row, sub-block) triple
    auto word = [&](int w) -> uint32_t { return ld_u32(grp + 288 + (w >> 2) * 512 + lane * 16 + (w & 3) * 4); };
    const int shift[4] = {0, 16, 6, 22};
    uint32_t code;
    if (i < 12) {
      code = (word(w0 + (i >> 2)) >> shift[i & 3]) & 63u;
    } else {
      const uint32_t X = word(w0), Y = word(w0 + 1), Z = word(w0 + 2);
      const uint32_t lo = (i == 12) ? (X >> 12) : (i == 13) ? (X >> 28) : (i == 14) ? (Y >> 12) : (Y >> 28);
      const uint32_t hi = (i == 12) ? (Z >> 12) : (i == 13) ? (Z >> 28) : (i == 14) ? (Z >> 14) : (Z >> 30);
      code = (lo & 0xFu) | ((hi & 3u) << 4);
    }
    const float v = (float)(int)code - 32.0f;
    return __fmul_rn(__fmul_rn(d, (float)sc), v);
  } else if constexpr (FMT == FMT_Q80) {
    const int blk = e >> 5, i = e & 31, lane = 4 * g + blk;
    const float d = ld_f16(grp + 4 * lane + 2 * rr);
    const int8_t q = (int8_t)grp[128 + (2 * rr + (i >> 4)) * 512 + lane * 16 + (i & 15)];
    return __fmul_rn(d, (float)q);
  } else {
    const int blk = e >> 5, i = e & 31, lane = 4 * g + blk;
    const uint8_t b = grp[(2 * rr + (i >> 4)) * 512 + lane * 16 + (i & 15)];
    const uint32_t h = e4m3x2_to_f16x2((uint16_t)b) & 0xFFFFu;
    return __half2float(__ushort_as_half((unsigned short)h));
  }
}

// One thread per output element of row `n` (global row), k in [0, K).
template <int FMT>
__device__ __forceinline__ float decode_row_elem(const uint8_t* w, int64_t G, int64_t n, int64_t k) {
  constexpr int GK = (FMT == FMT_Q4K || FMT == FMT_Q6K) ? 256 : 128;
  constexpr int GB = (FMT == FMT_Q4K) ? 2304 : (FMT == FMT_Q6K) ? 3360 : (FMT == FMT_Q80) ? 2176 : 2048;
  const int64_t t = n >> 4, s = k / GK;
  const uint8_t* grp = w + (size_t)(t * G + s) * GB;
  return decode_elem<FMT>(grp, (int)(n & 15), (int)(k - s * GK));
}

// row_scale (INT4 Marlin weights, held as Q4_K groups that decode to q - 8): the value
// times the row's f32 scale, as marlin_gemv.rs:47-59 forms it.
template <int FMT>
__global__ void dequant_kernel(const uint8_t* __restrict__ w, int64_t row0, int64_t K, int64_t G,
                               const float* __restrict__ row_scale, float* __restrict__ y) {
  const int64_t n = row0 + blockIdx.y;
  const float s = row_scale ? row_scale[n] : 1.0f;
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < K; k += (int64_t)gridDim.x * blockDim.x) {
    const float v = decode_row_elem<FMT>(w, G, n, k);
    y[n * K + k] = row_scale ? __fmul_rn(v, s) : v;
  }
}

template <int FMT>
__global__ void embed_kernel(const uint8_t* __restrict__ w, int64_t N, int64_t K, int64_t G,
                             const uint32_t* __restrict__ ids, int64_t row0, float* __restrict__ y,
                             int* status) {
  const int64_t i = row0 + blockIdx.y;
  const uint32_t id = ids[i];
  const bool ok = (int64_t)id < N;
  if (!ok && blockIdx.x == 0 && threadIdx.x == 0) raise_status(status, kDevIndex);
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < K; k += (int64_t)gridDim.x * blockDim.x)
    y[i * K + k] = ok ? decode_row_elem<FMT>(w, G, (int64_t)id, k) : 0.0f;
}

__global__ void fp8_encode_kernel(const float* __restrict__ x, int64_t n, uint8_t* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = e4m3_code_of_value(e4m3_round_ref(x[i]));
}

static dim3 row_grid(int64_t K, int64_t rows) {
  int64_t bx = (K + 255) / 256;
  if (bx > 64) bx = 64;
  return dim3((unsigned)bx, (unsigned)rows, 1);
}

// gridDim.y is limited to 65535, so rows are walked in slabs.
cudaError_t launch_dequant(int fmt, const uint8_t* w, int64_t N, int64_t K, int64_t G, const float* row_scale,
                           float* y, cudaStream_t st) {
  for (int64_t r0 = 0; r0 < N && K > 0; r0 += 65535) {
    const int64_t rows = (N - r0 < 65535) ? N - r0 : 65535;
    const dim3 grid = row_grid(K, rows);
    count_launch();
    switch (fmt) {
      case FMT_Q4K: dequant_kernel<FMT_Q4K><<<grid, 256, 0, st>>>(w, r0, K, G, row_scale, y); break;
      case FMT_Q6K: dequant_kernel<FMT_Q6K><<<grid, 256, 0, st>>>(w, r0, K, G, row_scale, y); break;
      case FMT_Q80: dequant_kernel<FMT_Q80><<<grid, 256, 0, st>>>(w, r0, K, G, row_scale, y); break;
      default:      dequant_kernel<FMT_FP8><<<grid, 256, 0, st>>>(w, r0, K, G, row_scale, y); break;
    }
  }
  return cudaGetLastError();
}

cudaError_t launch_embed(int fmt, const uint8_t* w, int64_t N, int64_t K, int64_t G, const uint32_t* ids,
                         int64_t n, float* y, int* status, cudaStream_t st) {
  for (int64_t r0 = 0; r0 < n && K > 0; r0 += 65535) {
    const int64_t rows = (n - r0 < 65535) ? n - r0 : 65535;
    const dim3 grid = row_grid(K, rows);
    count_launch();
    switch (fmt) {
      case FMT_Q4K: embed_kernel<FMT_Q4K><<<grid, 256, 0, st>>>(w, N, K, G, ids, r0, y, status); break;
      case FMT_Q6K: embed_kernel<FMT_Q6K><<<grid, 256, 0, st>>>(w, N, K, G, ids, r0, y, status); break;
      case FMT_Q80: embed_kernel<FMT_Q80><<<grid, 256, 0, st>>>(w, N, K, G, ids, r0, y, status); break;
      default:      embed_kernel<FMT_FP8><<<grid, 256, 0, st>>>(w, N, K, G, ids, r0, y, status); break;
    }
  }
  return cudaGetLastError();
}

cudaError_t launch_fp8_encode(const float* x, int64_t n, uint8_t* out, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  count_launch();
  fp8_encode_kernel<<<(unsigned)blocks, 256, 0, st>>>(x, n, out);
  return cudaGetLastError();
}

}  // namespace rtd
