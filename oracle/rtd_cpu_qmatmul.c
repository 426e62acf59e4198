/*
 * rtd_cpu_qmatmul.c -- the reference's CPU quantized matmul, restated for timing.
 *
 * TEST INFRASTRUCTURE ONLY (the CPU baseline of bench.py and its tests); the product
 * path never links or calls it.
 *
 * Weights::linear -> QMatMul::forward (crates/runtimed-model/src/weights/linear_layer.rs:45-52)
 * runs candle-core 0.11.0 (Cargo.lock:189-192), which is not vendored in the reference
 * tree.  Its published CPU algorithm for a quantized weight (the GGML k-quant scheme) is:
 *   1. quantize every activation row to the weight type's "vec-dot" block type:
 *      Q8_K for Q4_K / Q6_K weights (256 values: f32 scale d = max / -128 taken from the
 *      value of largest magnitude, codes round(x / d) clamped to 127, and the sums of
 *      each 16 consecutive codes), Q8_0 for Q8_0 weights (32 values: f16 scale
 *      amax / 127, codes round(x / d) half away from zero);
 *   2. per (token, weight row) an integer dot product per block, scaled in f32:
 *        Q4_K x Q8_K: d_x d_w sum_j sc_j <q4_j, q8_j> - d_x dmin_w sum_j m_j bsum_j
 *        Q6_K x Q8_K: d_x d_w sum_g sc_g (<q6u_g, q8_g> - 32 bsum_g)
 *        Q8_0 x Q8_0: d_x d_w <qw, qx>
 *      accumulated block by block into one f32 per output.
 * The integer dots run on AVX2 (unsigned x signed byte products, vpmaddubsw / vpmaddwd) when
 * the build has it, as candle's x86 kernels do; `simd = 0` selects the plain-C form of the
 * same integer arithmetic (identical results).  OpenMP splits the weight rows in tiles of
 * four; each row's codes are unpacked once per block and reused by every token, and each
 * token's block by the four rows.  (candle walks tokens outermost and re-reads the
 * weights per token; this order does the same arithmetic with far less memory traffic,
 * so the baseline it times is, if anything, faster than the reference.)
 * Accuracy against the exact product: the activations' 8-bit rounding, about 6e-3 relative
 * for Gaussian activations; against the exact product of the quantized activations, f32
 * rounding (1e-7).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif
#ifdef __AVX2__
#include <immintrin.h>
#endif

float rtdo_f16_to_f32(uint16_t bits);

static inline float rd_f16(const uint8_t* p) { return rtdo_f16_to_f32((uint16_t)(p[0] | ((uint16_t)p[1] << 8))); }

/* f32 -> f16 bits, round to nearest even (the Q8_0 activation scale is stored as f16) */
static uint16_t f32_to_f16_bits(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);  /* rounds to infinity */
    if (ax < 0x38800000u) {                                      /* f16 subnormal or zero */
        const float a = fabsf(f) * 16777216.0f;                  /* units of 2^-24, exact */
        return (uint16_t)(sign | (uint32_t)lrintf(a));
    }
    const uint32_t e = (ax >> 23) - 112u, m = ax & 0x7FFFFFu;
    uint32_t h = (e << 10) | (m >> 13);
    const uint32_t rest = m & 0x1FFFu;
    if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) h += 1u;
    return (uint16_t)(sign | h);
}

/* ------------------------------------------------------------ activation blocks */
typedef struct {
    float d;
    int8_t qs[256];
    int16_t bsums[16];
} q8k_block;

typedef struct {
    float d;  /* the f16-rounded scale, as f32 */
    int8_t qs[32];
} q8_0_block;

static void quantize_q8k(const float* x, q8k_block* b) {
    float amax = 0.0f, max = 0.0f;
    for (int j = 0; j < 256; j++) {
        const float ax = fabsf(x[j]);
        if (ax > amax) {
            amax = ax;
            max = x[j];
        }
    }
    if (amax == 0.0f) {
        memset(b, 0, sizeof(*b));
        return;
    }
    const float iscale = -128.0f / max;
    for (int j = 0; j < 256; j++) {
        const long v = lrintf(iscale * x[j]);
        b->qs[j] = (int8_t)(v > 127 ? 127 : v);
    }
    for (int g = 0; g < 16; g++) {
        int s = 0;
        for (int j = 0; j < 16; j++) s += b->qs[16 * g + j];
        b->bsums[g] = (int16_t)s;
    }
    b->d = 1.0f / iscale;
}

static void quantize_q8_0(const float* x, q8_0_block* b) {
    float amax = 0.0f;
    for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(x[j]));
    const float d = amax / 127.0f, id = d != 0.0f ? 1.0f / d : 0.0f;
    for (int j = 0; j < 32; j++) b->qs[j] = (int8_t)roundf(x[j] * id);
    b->d = rtdo_f16_to_f32(f32_to_f16_bits(d));
}

/* ------------------------------------------------------------ integer dots */
/* sum over n of u[n] * s[n]: u unsigned codes (< 64), s signed activation codes */
static inline int32_t dot_us_c(const uint8_t* u, const int8_t* s, int n) {
    int32_t acc = 0;
    for (int i = 0; i < n; i++) acc += (int32_t)u[i] * (int32_t)s[i];
    return acc;
}

static inline int32_t dot_ss_c(const int8_t* a, const int8_t* b, int n) {
    int32_t acc = 0;
    for (int i = 0; i < n; i++) acc += (int32_t)a[i] * (int32_t)b[i];
    return acc;
}

#ifdef __AVX2__
static inline int32_t hsum_i32(__m256i v) {
    __m128i s = _mm_add_epi32(_mm256_castsi256_si128(v), _mm256_extracti128_si256(v, 1));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0x4E));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0xB1));
    return _mm_cvtsi128_si32(s);
}

#endif

/* Q4_K row block against one Q8_K block: (sumi over scaled sub-blocks, summ of mins).
 * scv (AVX2): sub-block j's scale in every i16 lane of vector j. */
static inline void q4k_block_dot(const uint8_t* codes, const uint8_t* sc, const uint8_t* mn, const void* scv,
                                 const q8k_block* y, int simd, int32_t* sumi, int32_t* summ) {
#ifdef __AVX2__
    if (simd) {  /* scv: 8 vectors of sub-block scales, then one of the mins, each twice */
        const __m256i* v = (const __m256i*)scv;
        __m256i acc = _mm256_setzero_si256();
        for (int j = 0; j < 8; j++) {
            const __m256i p = _mm256_maddubs_epi16(_mm256_load_si256((const __m256i*)(codes + 32 * j)),
                                                   _mm256_loadu_si256((const __m256i*)(y->qs + 32 * j)));
            acc = _mm256_add_epi32(acc, _mm256_madd_epi16(p, v[j]));  /* pair sums (<= 3840) x scale (< 64) */
        }
        *sumi = hsum_i32(acc);
        *summ = hsum_i32(_mm256_madd_epi16(_mm256_loadu_si256((const __m256i*)y->bsums), v[8]));
        return;
    }
#endif
    (void)simd;
    (void)scv;
    int32_t si = 0, sm = 0;
    for (int j = 0; j < 8; j++) sm += (int32_t)mn[j] * ((int32_t)y->bsums[2 * j] + (int32_t)y->bsums[2 * j + 1]);
    for (int j = 0; j < 8; j++) si += (int32_t)sc[j] * dot_us_c(codes + 32 * j, y->qs + 32 * j, 32);
    *sumi = si;
    *summ = sm;
}

/* Q6_K row block (unsigned codes 0..63) against one Q8_K block.  scv (AVX2): vector h
 * holds the scale of group 2h in its low eight i16 lanes and of group 2h + 1 in the high
 * eight; off = 32 * sum_g sc_g bsum_g is the code bias, taken out once. */
static inline int32_t q6k_block_dot(const uint8_t* codes, const int8_t* sc, const void* scv, const q8k_block* y,
                                    int simd) {
#ifdef __AVX2__
    if (simd) {  /* scv: 8 vectors of group-scale pairs, then the 16 group scales */
        const __m256i* v = (const __m256i*)scv;
        __m256i acc = _mm256_setzero_si256();
        for (int h = 0; h < 8; h++) {
            const __m256i p = _mm256_maddubs_epi16(_mm256_load_si256((const __m256i*)(codes + 32 * h)),
                                                   _mm256_loadu_si256((const __m256i*)(y->qs + 32 * h)));
            acc = _mm256_add_epi32(acc, _mm256_madd_epi16(p, v[h]));  /* pair sums (<= 16128) x scale (<= 128) */
        }
        const __m256i off = _mm256_madd_epi16(_mm256_loadu_si256((const __m256i*)y->bsums), v[8]);
        return hsum_i32(_mm256_sub_epi32(acc, _mm256_slli_epi32(off, 5)));
    }
#endif
    (void)simd;
    (void)scv;
    int32_t off = 0;
    for (int g = 0; g < 16; g++) off += (int32_t)sc[g] * (int32_t)y->bsums[g];
    int32_t si = 0;
    for (int g = 0; g < 16; g++) si += (int32_t)sc[g] * dot_us_c(codes + 16 * g, y->qs + 16 * g, 16);
    return si - 32 * off;
}

static inline int32_t q8_0_block_dot(const int8_t* w, const int8_t* x, int simd) {
#ifdef __AVX2__
    if (simd) {
        const __m256i a = _mm256_loadu_si256((const __m256i*)w), b = _mm256_loadu_si256((const __m256i*)x);
        /* |a| x (b with a's sign): unsigned x signed products, pairs fit i16 (127 * 128 * 2) */
        const __m256i p = _mm256_maddubs_epi16(_mm256_sign_epi8(a, a), _mm256_sign_epi8(b, a));
        return hsum_i32(_mm256_madd_epi16(p, _mm256_set1_epi16(1)));
    }
#endif
    (void)simd;
    return dot_ss_c(w, x, 32);
}

/* ------------------------------------------------------------ unpacking one weight block */
/* Q4_K: 256 codes in element order (dequant_k.rs:19-44 order: per 64-chunk, 32 low
 * nibbles then 32 high), the 8 sub-block scales and mins (scale_min_k4, dequant_k.rs:8-16) */
static void unpack_q4k(const uint8_t* blk, uint8_t* codes, uint8_t* sc, uint8_t* mn) {
    const uint8_t* s = blk + 4;
    for (int j = 0; j < 8; j++) {
        if (j < 4) {
            sc[j] = s[j] & 63;
            mn[j] = s[j + 4] & 63;
        } else {
            sc[j] = (uint8_t)((s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4));
            mn[j] = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
        }
    }
    const uint8_t* qs = blk + 16;
    for (int c = 0; c < 4; c++)
        for (int l = 0; l < 32; l++) {
            codes[64 * c + l] = qs[32 * c + l] & 0xF;
            codes[64 * c + 32 + l] = qs[32 * c + l] >> 4;
        }
}

/* Q6_K: 256 unsigned codes (q + 32) in element order (dequant_k.rs:87-111) */
static void unpack_q6k(const uint8_t* blk, uint8_t* codes) {
    for (int half = 0; half < 2; half++) {
        const uint8_t* ql = blk + 64 * half;
        const uint8_t* qh = blk + 128 + 32 * half;
        uint8_t* o = codes + 128 * half;
        for (int l = 0; l < 32; l++) {
            o[l] = (uint8_t)((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4));
            o[l + 32] = (uint8_t)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4));
            o[l + 64] = (uint8_t)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4));
            o[l + 96] = (uint8_t)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4));
        }
    }
}

/* ------------------------------------------------------------ the matmul */
/* y[M, N] = x[M, K] . W^T for Q4_K (12), Q6_K (14) or Q8_0 (8) weights; returns 0, or
 * 1 for another type, 2 for K not a multiple of the block.  threads <= 0: OpenMP default. */
int rtdo_cpu_qmatmul(uint32_t type, const uint8_t* w, int64_t N, int64_t K, const float* x, int64_t M, float* y,
                     int threads, int simd) {
    if (type != 12 && type != 14 && type != 8) return 1;
    const int64_t QK = type == 8 ? 32 : 256;
    if (K % QK != 0) return 2;
    const int64_t nb = K / QK;
    const size_t bb = type == 12 ? 144 : type == 14 ? 210 : 34;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
    /* 1. the activations, quantized once per call, block-major (the M tokens' blocks b
     *    contiguous, so the token loop below streams them) */
    void* xq = type == 8 ? malloc(sizeof(q8_0_block) * (size_t)(M * nb)) : malloc(sizeof(q8k_block) * (size_t)(M * nb));
    if (!xq) return 3;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < M * nb; i++) {
        const int64_t m = i / nb, b = i % nb;
        const float* src = x + m * K + b * QK;
        if (type == 8)
            quantize_q8_0(src, (q8_0_block*)xq + b * M + m);
        else
            quantize_q8k(src, (q8k_block*)xq + b * M + m);
    }
    /* 2. tiles of RT weight rows over the threads: each row's block is unpacked once and
     *    used by every token, each token's block by the RT rows of the tile */
    enum { RT = 4 };
    const int64_t tiles = (N + RT - 1) / RT;
#pragma omp parallel
    {
        float* acc = (float*)malloc(sizeof(float) * (size_t)M * RT);
        uint8_t codes[RT][256] __attribute__((aligned(32)));
        int16_t scv[RT][9][16] __attribute__((aligned(32)));
        uint8_t sc4[RT][8], mn4[RT][8];
        float dw[RT], dmw[RT];
#pragma omp for schedule(static)
        for (int64_t tile = 0; tile < tiles; tile++) {
            const int64_t n0 = tile * RT;
            const int nr = (int)(N - n0 < RT ? N - n0 : RT);
            for (int64_t i = 0; i < (int64_t)M * RT; i++) acc[i] = 0.0f;
            for (int64_t b = 0; b < nb; b++) {
                for (int r = 0; r < nr; r++) {
                    const uint8_t* blk = w + ((size_t)(n0 + r) * (size_t)nb + (size_t)b) * bb;
                    if (type == 12) {
                        unpack_q4k(blk, codes[r], sc4[r], mn4[r]);
                        for (int j = 0; j < 8; j++)
                            for (int e = 0; e < 16; e++) scv[r][j][e] = sc4[r][j];
                        for (int e = 0; e < 16; e++) scv[r][8][e] = mn4[r][e / 2];
                        dw[r] = rd_f16(blk);
                        dmw[r] = rd_f16(blk + 2);
                    } else if (type == 14) {
                        unpack_q6k(blk, codes[r]);
                        const int8_t* sc = (const int8_t*)(blk + 192);
                        memcpy(sc4[r], sc, 8);
                        memcpy(mn4[r], sc + 8, 8);  /* (Q6_K: the 16 signed group scales, in sc4 | mn4) */
                        for (int h = 0; h < 8; h++)
                            for (int e = 0; e < 16; e++) scv[r][h][e] = sc[2 * h + (e >= 8)];
                        for (int e = 0; e < 16; e++) scv[r][8][e] = sc[e];
                        dw[r] = rd_f16(blk + 208);
                    } else {
                        memcpy(codes[r], blk + 2, 32);
                        dw[r] = rd_f16(blk);
                    }
                }
                for (int64_t m = 0; m < M; m++) {
                    if (type == 12) {
                        const q8k_block* yb = (const q8k_block*)xq + b * M + m;
                        for (int r = 0; r < nr; r++) {
                            int32_t si, sm;
                            q4k_block_dot(codes[r], sc4[r], mn4[r], scv[r], yb, simd, &si, &sm);
                            acc[r * M + m] += yb->d * dw[r] * (float)si - yb->d * dmw[r] * (float)sm;
                        }
                    } else if (type == 14) {
                        const q8k_block* yb = (const q8k_block*)xq + b * M + m;
                        for (int r = 0; r < nr; r++) {
                            int8_t sc[16];
                            memcpy(sc, sc4[r], 8);
                            memcpy(sc + 8, mn4[r], 8);
                            acc[r * M + m] += yb->d * dw[r] * (float)q6k_block_dot(codes[r], sc, scv[r], yb, simd);
                        }
                    } else {
                        const q8_0_block* yb = (const q8_0_block*)xq + b * M + m;
                        for (int r = 0; r < nr; r++)
                            acc[r * M + m] += yb->d * dw[r] * (float)q8_0_block_dot((const int8_t*)codes[r], yb->qs, simd);
                    }
                }
            }
            for (int r = 0; r < nr; r++)
                for (int64_t m = 0; m < M; m++) y[m * N + n0 + r] = acc[r * M + m];
        }
        free(acc);
    }
    free(xq);
    return 0;
}

/* The activation quantizers alone (for their known-answer tests): Q8_K (type 12 / 14) or
 * Q8_0 (type 8) blocks of x[K] -> codes[K], scales[K / QK] (and bsums[K / 16] for Q8_K). */
int rtdo_cpu_quantize_x(uint32_t type, const float* x, int64_t K, int8_t* codes, float* scales, int16_t* bsums) {
    const int64_t QK = type == 8 ? 32 : 256;
    if ((type != 12 && type != 14 && type != 8) || K % QK != 0) return 1;
    for (int64_t b = 0; b < K / QK; b++) {
        if (type == 8) {
            q8_0_block q;
            quantize_q8_0(x + b * QK, &q);
            memcpy(codes + b * QK, q.qs, 32);
            scales[b] = q.d;
        } else {
            q8k_block q;
            quantize_q8k(x + b * QK, &q);
            memcpy(codes + b * QK, q.qs, 256);
            scales[b] = q.d;
            if (bsums) memcpy(bsums + b * 16, q.bsums, 32);
        }
    }
    return 0;
}
