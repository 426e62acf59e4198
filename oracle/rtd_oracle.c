/*
 * rtd_oracle.c -- CPU restatement of the reference's quantized-linear arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load this library; the
 * product path (runtimed_b200, libruntimed_b200.so) never links or calls it.
 *
 * What it restates (paths relative to the syntropd/runtimed project root):
 *   - f16 -> f32 with subnormals ........ crates/runtimed-gguf/src/quant/dequant.rs:11-33
 *   - Q8_0 block decode .................. crates/runtimed-gguf/src/quant/dequant.rs:40-47
 *   - whole-tensor dispatcher + errors ... crates/runtimed-gguf/src/quant/dequant.rs:83-146
 *   - block geometry ..................... crates/runtimed-gguf/src/quant/dtype.rs:49-64
 *   - scale_min_k4 / Q4_K block .......... crates/runtimed-gguf/src/quant/dequant_k.rs:8-44
 *   - Q6_K block ......................... crates/runtimed-gguf/src/quant/dequant_k.rs:87-111
 *   - FP8 E4M3 LUT / encoder ............. crates/runtimed-model/src/weights/load_safetensors.rs:14-29,53-69
 *   - CPU FP8 GEMM fallback .............. crates/runtimed-model/src/ops/fp8_gemm.rs:55-74
 *   - CUDA FP8 GEMM semantics (x -> E4M3 unscaled, per-tensor A scale or
 *     per-channel post-scale) ............ crates/runtimed-model/src/ops/fp8_gemm.rs:96-101,128-139,180-186
 *
 * The block decoders keep the reference's float operation order (d*sc first,
 * then *q, then -m; no fused multiply-add).  Build with -ffp-contract=off so the
 * compiler cannot contract `d1 * q - m1` into an FMA.
 *
 * The quantized matmul itself is candle-core 0.11.0 `QMatMul::forward`, a
 * third-party crate that is not vendored in the reference tree.  The GEMV/GEMM
 * oracle here is therefore `y = x . dequant(W)^T` accumulated in double, the
 * definition the parity tests gate on (relative L2 <= 1e-3).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum {
    RTDO_F32 = 0, RTDO_F16 = 1, RTDO_Q4_0 = 2, RTDO_Q5_0 = 6, RTDO_Q8_0 = 8,
    RTDO_Q2_K = 10, RTDO_Q3_K = 11, RTDO_Q4_K = 12, RTDO_Q5_K = 13, RTDO_Q6_K = 14,
    RTDO_BF16 = 30
};

/* dequant_tensor error codes (GgufError variants of dequant.rs:83-146) */
enum { RTDO_OK = 0, RTDO_UNSUPPORTED = 1, RTDO_NOT_MULTIPLE = 2, RTDO_TRUNCATED = 3 };

static inline float bits_to_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f32_to_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* dequant.rs:11-33 -- IEEE half to float, subnormals normalised by shifting. */
float rtdo_f16_to_f32(uint16_t bits) {
    uint32_t sign = (bits >> 15) & 1u;
    uint32_t exp = (bits >> 10) & 0x1Fu;
    uint32_t mant = bits & 0x3FFu;
    uint32_t out;
    if (exp == 0) {
        if (mant == 0) {
            out = sign << 31;
        } else {
            uint32_t m = mant;
            int32_t e = 127 - 14;
            while ((m & 0x400u) == 0) { m <<= 1; e -= 1; }
            out = (sign << 31) | ((uint32_t)e << 23) | ((m & 0x3FFu) << 13);
        }
    } else if (exp == 31) {
        out = (sign << 31) | (0xFFu << 23) | (mant << 13);
    } else {
        out = (sign << 31) | ((exp + 112u) << 23) | (mant << 13);
    }
    return bits_to_f32(out);
}

static inline float read_f16(const uint8_t* p) {
    return rtdo_f16_to_f32((uint16_t)(p[0] | ((uint16_t)p[1] << 8)));
}

/* dtype.rs:49-64 -- (elements per block, bytes per block); -1 if undecodable. */
int rtdo_block_geometry(uint32_t type, uint64_t* elems, uint64_t* bytes) {
    uint64_t e, b;
    switch (type) {
        case RTDO_F32: e = 1; b = 4; break;
        case RTDO_F16: case RTDO_BF16: e = 1; b = 2; break;
        case RTDO_Q4_0: e = 32; b = 18; break;
        case RTDO_Q5_0: e = 32; b = 22; break;
        case RTDO_Q8_0: e = 32; b = 34; break;
        case RTDO_Q2_K: e = 256; b = 84; break;
        case RTDO_Q3_K: e = 256; b = 110; break;
        case RTDO_Q4_K: e = 256; b = 144; break;
        case RTDO_Q5_K: e = 256; b = 176; break;
        case RTDO_Q6_K: e = 256; b = 210; break;
        default: return -1;
    }
    if (elems) *elems = e;
    if (bytes) *bytes = b;
    return 0;
}

/* dequant.rs:40-47 -- y[i] = d * (i8)q[i] */
void rtdo_dequant_q8_0_block(const uint8_t* block, float* out) {
    float d = read_f16(block);
    for (int i = 0; i < 32; i++) out[i] = d * (float)(int8_t)block[2 + i];
}

/* dequant_k.rs:8-16 -- the 6-bit (scale, min) pair j of a Q4_K superblock. */
static void scale_min_k4(int j, const uint8_t* s, uint8_t* sc, uint8_t* m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (uint8_t)((s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4));
        *m = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

/* dequant_k.rs:19-44 -- four 64-value chunks; low nibbles use (d1, m1), high
 * nibbles (d2, m2); value = d_i * q - m_i with an unfused multiply and subtract. */
void rtdo_dequant_q4_k_block(const uint8_t* block, float* out) {
    float d = read_f16(block);
    float mn = read_f16(block + 2);
    const uint8_t* scales = block + 4;
    const uint8_t* qs = block + 16;
    int o = 0, is = 0;
    for (int chunk = 0; chunk < 4; chunk++) {
        const uint8_t* q = qs + chunk * 32;
        uint8_t sc, m;
        scale_min_k4(is, scales, &sc, &m);
        float d1 = d * (float)sc, m1 = mn * (float)m;
        scale_min_k4(is + 1, scales, &sc, &m);
        float d2 = d * (float)sc, m2 = mn * (float)m;
        for (int l = 0; l < 32; l++) {
            float p = d1 * (float)(q[l] & 0xF);
            out[o++] = p - m1;
        }
        for (int l = 0; l < 32; l++) {
            float p = d2 * (float)(q[l] >> 4);
            out[o++] = p - m2;
        }
        is += 2;
    }
}

/* dequant_k.rs:87-111 -- two 128-value halves; 6-bit code = low nibble | 2 high
 * bits << 4, centred by -32; value = (d * sc) * q, left to right. */
void rtdo_dequant_q6_k_block(const uint8_t* block, float* out) {
    const uint8_t* ql_all = block;
    const uint8_t* qh_all = block + 128;
    const uint8_t* sc_all = block + 192;
    float d = read_f16(block + 208);
    for (int half = 0; half < 2; half++) {
        const uint8_t* ql = ql_all + half * 64;
        const uint8_t* qh = qh_all + half * 32;
        const uint8_t* sc = sc_all + half * 8;
        float* y = out + half * 128;
        for (int l = 0; l < 32; l++) {
            int is = l / 16;
            float q[4];
            q[0] = (float)(int8_t)((ql[l] & 0xF) | ((qh[l] & 3) << 4)) - 32.0f;
            q[1] = (float)(int8_t)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32.0f;
            q[2] = (float)(int8_t)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32.0f;
            q[3] = (float)(int8_t)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32.0f;
            for (int k = 0; k < 4; k++) {
                float ds = d * (float)(int8_t)sc[is + k * 2];
                y[l + k * 32] = ds * q[k];
            }
        }
    }
}

/* dequant.rs:83-146 -- whole-tensor dispatcher.  Formats off the hot path
 * (Q4_0, Q5_0, Q5_K, Q2_K, Q3_K) report RTDO_UNSUPPORTED here. */
int rtdo_dequant_tensor(uint32_t type, const uint8_t* bytes, uint64_t nbytes,
                        uint64_t n_elements, float* out) {
    uint64_t elems, bb;
    if (rtdo_block_geometry(type, &elems, &bb) != 0) return RTDO_UNSUPPORTED;
    if (n_elements % elems != 0) return RTDO_NOT_MULTIPLE;
    uint64_t need = n_elements / elems * bb;
    if (nbytes < need) return RTDO_TRUNCATED;
    uint64_t nb = n_elements / elems;
    switch (type) {
        case RTDO_F32:
            for (uint64_t i = 0; i < nb; i++) {
                uint32_t u = (uint32_t)bytes[4 * i] | ((uint32_t)bytes[4 * i + 1] << 8) |
                             ((uint32_t)bytes[4 * i + 2] << 16) | ((uint32_t)bytes[4 * i + 3] << 24);
                out[i] = bits_to_f32(u);
            }
            return RTDO_OK;
        case RTDO_F16:
            for (uint64_t i = 0; i < nb; i++) out[i] = read_f16(bytes + 2 * i);
            return RTDO_OK;
        case RTDO_BF16:
            for (uint64_t i = 0; i < nb; i++)
                out[i] = bits_to_f32(((uint32_t)bytes[2 * i] | ((uint32_t)bytes[2 * i + 1] << 8)) << 16);
            return RTDO_OK;
        case RTDO_Q8_0:
            for (uint64_t i = 0; i < nb; i++) rtdo_dequant_q8_0_block(bytes + i * 34, out + i * 32);
            return RTDO_OK;
        case RTDO_Q4_K:
            for (uint64_t i = 0; i < nb; i++) rtdo_dequant_q4_k_block(bytes + i * 144, out + i * 256);
            return RTDO_OK;
        case RTDO_Q6_K:
            for (uint64_t i = 0; i < nb; i++) rtdo_dequant_q6_k_block(bytes + i * 210, out + i * 256);
            return RTDO_OK;
        default:
            return RTDO_UNSUPPORTED;
    }
}

/* Dequantize one row n of a [N, K] quantized matrix (rows are K/elems blocks). */
static int dequant_row(uint32_t type, const uint8_t* blocks, int64_t K, int64_t n, float* row) {
    uint64_t elems, bb;
    if (rtdo_block_geometry(type, &elems, &bb) != 0) return RTDO_UNSUPPORTED;
    if ((uint64_t)K % elems != 0) return RTDO_NOT_MULTIPLE;
    uint64_t row_bytes = (uint64_t)K / elems * bb;
    return rtdo_dequant_tensor(type, blocks + (uint64_t)n * row_bytes, row_bytes, (uint64_t)K, row);
}

/* y[m, n] = sum_k x[m, k] * dequant(W)[n, k] (+ bias[n]), accumulated in double.
 * W is GGUF-ordered: N rows of K/elems raw blocks (load_gguf.rs:35: [N, K] =
 * [dims[1], dims[0]]). */
int rtdo_qgemv_f64(uint32_t type, const uint8_t* blocks, uint64_t nbytes, int64_t N, int64_t K,
                   const float* x, int64_t M, const float* bias, double* y) {
    uint64_t elems, bb;
    if (rtdo_block_geometry(type, &elems, &bb) != 0) return RTDO_UNSUPPORTED;
    if ((uint64_t)K % elems != 0) return RTDO_NOT_MULTIPLE;
    if (nbytes < (uint64_t)N * ((uint64_t)K / elems * bb)) return RTDO_TRUNCATED;
    int rc = RTDO_OK;
#pragma omp parallel
    {
        float* row = (float*)malloc(sizeof(float) * (size_t)K);
#pragma omp for schedule(static)
        for (int64_t n = 0; n < N; n++) {
            if (dequant_row(type, blocks, K, n, row) != RTDO_OK) { rc = RTDO_UNSUPPORTED; continue; }
            for (int64_t m = 0; m < M; m++) {
                const float* xr = x + m * K;
                double acc = 0.0;
                for (int64_t k = 0; k < K; k++) acc += (double)xr[k] * (double)row[k];
                if (bias) acc += (double)bias[n];
                y[m * N + n] = acc;
            }
        }
        free(row);
    }
    return rc;
}

/* Timed CPU baseline: the restated reference CPU path.  Each row is decoded
 * with the reference block decoders, then dotted with x in f32 (the dequantize-
 * then-f32-matmul path of Weights::get + matmul).  OpenMP over `threads`. */
int rtdo_ref_cpu_linear(uint32_t type, const uint8_t* blocks, int64_t N, int64_t K,
                        const float* x, int64_t M, float* y, int threads) {
    uint64_t elems, bb;
    if (rtdo_block_geometry(type, &elems, &bb) != 0) return RTDO_UNSUPPORTED;
    if ((uint64_t)K % elems != 0) return RTDO_NOT_MULTIPLE;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#endif
#pragma omp parallel
    {
        float* row = (float*)malloc(sizeof(float) * (size_t)K);
#pragma omp for schedule(static)
        for (int64_t n = 0; n < N; n++) {
            dequant_row(type, blocks, K, n, row);
            for (int64_t m = 0; m < M; m++) {
                const float* xr = x + m * K;
                float acc = 0.0f;
#pragma omp simd reduction(+ : acc)
                for (int64_t k = 0; k < K; k++) acc += xr[k] * row[k];
                y[m * N + n] = acc;
            }
        }
        free(row);
    }
    return RTDO_OK;
}

/* ---------------------------------------------------------------- FP8 E4M3 */

/* load_safetensors.rs:14-29 -- E4M3 decode table (no infinities; 0x7f/0xff NaN). */
static float fp8_lut[256];
static int fp8_lut_ready = 0;

static void fp8_lut_init(void) {
    if (fp8_lut_ready) return;
    for (int b = 0; b < 256; b++) {
        float sign = (b & 0x80) ? -1.0f : 1.0f;
        int exp = (b >> 3) & 0x0f;
        float mant = (float)(b & 0x07);
        float v;
        if (exp == 0) v = sign * ldexpf(1.0f, -6) * (mant / 8.0f);
        else if (exp == 15 && (b & 0x07) == 0x07) v = NAN;
        else v = sign * ldexpf(1.0f, exp - 7) * (1.0f + mant / 8.0f);
        fp8_lut[b] = v;
    }
    fp8_lut_ready = 1;
}

float rtdo_fp8_e4m3_to_f32(uint8_t b) { fp8_lut_init(); return fp8_lut[b]; }

/* load_safetensors.rs:53-69 -- binary search over the 127 non-negative codes;
 * a tie between two neighbours goes to the LOWER magnitude; >= 448 saturates to
 * 0x7e; NaN encodes as 0x7f; the sign is taken from the sign bit (so -0 -> 0x80). */
uint8_t rtdo_f32_to_fp8_e4m3(float f) {
    fp8_lut_init();
    if (isnan(f)) return 0x7f;
    uint8_t sign = (f32_to_bits(f) >> 31) ? 0x80 : 0x00;
    float a = fabsf(f);
    if (a <= 0.0f) return sign;
    if (a >= 448.0f) return sign | 0x7e;
    /* lower_bound over pos[0..127) */
    int lo = 0, hi = 127;
    while (lo < hi) {
        int mid = (lo + hi) / 2;
        if (fp8_lut[mid] < a) lo = mid + 1; else hi = mid;
    }
    int idx = lo;
    if (idx < 127 && fp8_lut[idx] == a) return sign | (uint8_t)idx;
    if (idx == 0) return sign;
    if (idx >= 127) return sign | 0x7e;
    int pick = (a - fp8_lut[idx - 1] <= fp8_lut[idx] - a) ? idx - 1 : idx;
    return sign | (uint8_t)pick;
}

void rtdo_f32_to_fp8_e4m3_array(const float* x, int64_t n, uint8_t* out) {
    for (int64_t i = 0; i < n; i++) out[i] = rtdo_f32_to_fp8_e4m3(x[i]);
}

/* fp8_gemm.rs:55-74 -- CPU fallback: y = x_f32 . (LUT(w) * s)^T.  The scaled
 * weight is formed in f32 (candle broadcast_mul) and the product is accumulated
 * in double here.  scale_len is 1 (per-tensor) or N (per-channel). */
void rtdo_fp8_gemm_cpu_f64(const float* x, const uint8_t* w, const float* scale, int64_t scale_len,
                           int64_t M, int64_t N, int64_t K, double* y) {
    fp8_lut_init();
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; n++) {
        float s = scale ? scale[scale_len == 1 ? 0 : n] : 1.0f;
        for (int64_t m = 0; m < M; m++) {
            double acc = 0.0;
            for (int64_t k = 0; k < K; k++) {
                float ws = fp8_lut[w[n * K + k]] * s;
                acc += (double)x[m * K + k] * (double)ws;
            }
            y[m * N + n] = acc;
        }
    }
}

/* fp8_gemm.rs:96-101,128-139,180-186 -- the CUDA path's semantics: x is encoded
 * to E4M3 without scaling, the E4M3 x E4M3 product is accumulated (f32 in
 * cuBLASLt, double here), a single-element scale is applied as the A scale and
 * a per-channel scale multiplies the output afterwards. */
void rtdo_fp8_gemm_w8a8_f64(const float* x, const uint8_t* w, const float* scale, int64_t scale_len,
                            int64_t M, int64_t N, int64_t K, double* y) {
    fp8_lut_init();
    uint8_t* xq = (uint8_t*)malloc((size_t)(M * K));
    for (int64_t i = 0; i < M * K; i++) xq[i] = rtdo_f32_to_fp8_e4m3(x[i]);
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; n++) {
        double s = scale ? (double)scale[scale_len == 1 ? 0 : n] : 1.0;
        for (int64_t m = 0; m < M; m++) {
            double acc = 0.0;
            for (int64_t k = 0; k < K; k++)
                acc += (double)fp8_lut[w[n * K + k]] * (double)fp8_lut[xq[m * K + k]];
            y[m * N + n] = acc * s;
        }
    }
    free(xq);
}

/* Timed CPU baseline for FP8 weights: the reference CPU fallback in f32
 * (dequantize-and-scale the row, then an f32 dot), OpenMP over `threads`. */
void rtdo_ref_cpu_fp8_linear(const float* x, const uint8_t* w, const float* scale, int64_t scale_len,
                             int64_t M, int64_t N, int64_t K, float* y, int threads) {
    fp8_lut_init();
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#endif
#pragma omp parallel
    {
        float* row = (float*)malloc(sizeof(float) * (size_t)K);
#pragma omp for schedule(static)
        for (int64_t n = 0; n < N; n++) {
            float s = scale ? scale[scale_len == 1 ? 0 : n] : 1.0f;
            for (int64_t k = 0; k < K; k++) row[k] = fp8_lut[w[n * K + k]] * s;
            for (int64_t m = 0; m < M; m++) {
                float acc = 0.0f;
#pragma omp simd reduction(+ : acc)
                for (int64_t k = 0; k < K; k++) acc += x[m * K + k] * row[k];
                y[m * N + n] = acc;
            }
        }
        free(row);
    }
}

int rtdo_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
