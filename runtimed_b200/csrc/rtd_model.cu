// rtd_model.cu -- the per-layer operations around the quantized linears, sm_100a.
//
// The decoder layer of crates/runtimed-model/src/arch/qwen2.rs:68-127 runs, between its
// linears, the SubstratePort operations of crates/runtimed-model/src/substrate/port.rs:
// rmsnorm (ops/norm.rs:7-11), NeoX rope (ops/rope.rs:24-60), scaled dot-product
// attention with GQA over the KV cache (ops/attention.rs:107-128, causal_mask :38-58),
// silu (ops/activation.rs:6-10) and the greedy argmax (decode/sample.rs:11-18).  Here
// they are device kernels over a PAGED f16 KV cache (fixed 16-token blocks, a block
// table per sequence; crates/runtimed-model/src/cache/paged/table.rs:57-145) with
// per-token (sequence, position) pairs, so one launch serves a prefill chunk of one
// sequence, a batched decode step of many sequences (one token each) or a speculative
// verify of k + 1 positions alike.
//
// Every kernel is memory- or latency-bound and small next to the linears; each keeps
// the reference's f32 operation order where it is cheap to do so (x / rms then * w;
// x1*cos - x2*sin; x * 1/(exp(-x) + 1)) and accumulates in f32.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cfloat>
#include <cstdint>

#include "rtd_common.cuh"
#include "rtd_kernels.h"

namespace rtd {
namespace {

__device__ __forceinline__ float load_as_f32(const void* p, int dt, int64_t i) {
  if (dt == 0) return static_cast<const float*>(p)[i];
  if (dt == 1) return __half2float(static_cast<const __half*>(p)[i]);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}

__device__ __forceinline__ void store_from_f32(void* p, int dt, int64_t i, float v) {
  if (dt == 0)
    static_cast<float*>(p)[i] = v;
  else if (dt == 1)
    static_cast<__half*>(p)[i] = __float2half_rn(v);
  else
    static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.0f;
#pragma unroll
  for (int w = 0; w < NT / 32; ++w) s += red[w];
  __syncthreads();
  return s;
}

// ------------------------------------------------------------------ RMSNorm
// One CTA per row: h += delta (the residual add that precedes every norm of the
// layer, qwen2.rs:112,126), then y = (h / sqrt(mean(h^2) + eps)) * w.
constexpr int kNormThreads = 256;

__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(float* h, int64_t ldh, const void* delta, int ddt,
                                                                   int64_t ldd, const float* w, float eps, int64_t H,
                                                                   void* y, int ydt, int64_t ldy) {
  __shared__ float red[kNormThreads / 32];
  const int64_t row = blockIdx.x;
  float* hr = h + row * ldh;
  float ss = 0.0f;
  for (int64_t i = threadIdx.x; i < H; i += kNormThreads) {
    float v = hr[i];
    if (delta) {
      v = v + load_as_f32(delta, ddt, row * ldd + i);
      hr[i] = v;
    }
    ss = fmaf(v, v, ss);
  }
  const float m2 = block_sum<kNormThreads>(ss, red) / (float)H;
  const float denom = sqrtf(m2 + eps);
  for (int64_t i = threadIdx.x; i < H; i += kNormThreads) {
    const float v = hr[i] / denom;
    store_from_f32(y, ydt, row * ldy + i, v * __ldg(w + i));
  }
}

// ------------------------------------------------------------------ RoPE + KV append
// Block (token t, head j < n_head + n_kv): query heads are rotated into q_out; key
// heads are rotated and value heads copied into the paged f16 cache at the token's
// (sequence, position).  Thread i rotates the pair (i, i + rot_dim / 2):
//   inv = theta^(-2i / rot_dim), angle = pos * inv,
//   o1 = x1 cos - x2 sin, o2 = x2 cos + x1 sin (rope.rs:37-58, products rounded first);
// dims past rot_dim pass through.
struct RopeArgs {
  const float* q;
  const float* k;
  const float* v;
  int64_t ldq, ldk, ldv;  // row strides (elements) of the linear outputs
  int n_head, n_kv, head_dim, rot_dim;
  float theta;
  const int* tok_seq;
  const int* tok_pos;
  const int* block_table;
  int max_blocks;
  void* k_cache;    // [blocks][n_kv][16][head_dim], f16 or f32
  void* v_cache;
  float* q_out;     // [T][n_head][head_dim]
};

template <typename KV>
__device__ __forceinline__ KV to_kv(float v);
template <>
__device__ __forceinline__ __half to_kv<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ float to_kv<float>(float v) { return v; }

constexpr int kKvBlock = 16;

__device__ __forceinline__ int64_t cache_row(const RopeArgs& a, int seq, int pos, int kvh) {
  const int blk = __ldg(a.block_table + (int64_t)seq * a.max_blocks + pos / kKvBlock);
  return (((int64_t)blk * a.n_kv + kvh) * kKvBlock + pos % kKvBlock) * a.head_dim;
}

template <typename KV>
__global__ void rope_kv_kernel(const RopeArgs a) {
  const int t = blockIdx.x, j = blockIdx.y;
  const int seq = __ldg(a.tok_seq + t), pos = __ldg(a.tok_pos + t);
  const int half = a.rot_dim / 2;
  KV* kc = static_cast<KV*>(a.k_cache);
  KV* vc = static_cast<KV*>(a.v_cache);
  if (j >= a.n_head + a.n_kv) {  // value head: plain copy to the cache
    const int kvh = j - a.n_head - a.n_kv;
    const float* src = a.v + (int64_t)t * a.ldv + (int64_t)kvh * a.head_dim;
    KV* dst = vc + cache_row(a, seq, pos, kvh);
    for (int d = threadIdx.x; d < a.head_dim; d += blockDim.x) dst[d] = to_kv<KV>(src[d]);
    return;
  }
  const bool is_q = j < a.n_head;
  const int hh = is_q ? j : j - a.n_head;
  const float* src = is_q ? a.q + (int64_t)t * a.ldq + (int64_t)hh * a.head_dim
                          : a.k + (int64_t)t * a.ldk + (int64_t)hh * a.head_dim;
  float* qo = is_q ? a.q_out + ((int64_t)t * a.n_head + hh) * a.head_dim : nullptr;
  KV* ko = is_q ? nullptr : kc + cache_row(a, seq, pos, hh);
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float e = (-2.0f * (float)i) / (float)a.rot_dim;
    const float inv = powf(a.theta, e);
    const float ang = (float)pos * inv;
    const float c = cosf(ang), s = sinf(ang);
    const float x1 = src[i], x2 = src[i + half];
    const float o1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
    const float o2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
    if (is_q) {
      qo[i] = o1;
      qo[i + half] = o2;
    } else {
      ko[i] = to_kv<KV>(o1);
      ko[i + half] = to_kv<KV>(o2);
    }
  }
  for (int d = a.rot_dim + threadIdx.x; d < a.head_dim; d += blockDim.x) {
    if (is_q)
      qo[d] = src[d];
    else
      ko[d] = to_kv<KV>(src[d]);
  }
}

// ------------------------------------------------------------------ attention
// Block (token t, kv head g, split s): the G = n_head / n_kv query heads of the group
// attend keys [0, pos_t] of the token's sequence (causal; a split takes one range of
// them), in chunks of kChunk keys staged in shared memory:
//   scores s[h][j] = (q_h . k_j) * scale,  online softmax per head,  acc[h] += p V.
// With one split the block writes o = acc / l; otherwise it writes its (m, l, acc) and
// attn_combine_kernel merges the splits in order.
constexpr int kAttnThreads = 128;
constexpr int kChunk = 64;
constexpr int kMaxGroup = 8;
constexpr int kMaxOutPerThread = kMaxGroup * 128 / kAttnThreads;  // G * head_dim / threads

struct AttnArgs {
  const float* q;  // [T][n_head][head_dim]
  int n_head, n_kv, head_dim;
  float scale;
  const int* tok_seq;
  const int* tok_pos;
  const int* block_table;
  int max_blocks;
  const void* k_cache;  // f16 or f32
  const void* v_cache;
  void* o;         // [T][n_head * head_dim]
  int o_dtype;
  int64_t ldo;
  int splits;
  float* part;     // [T][n_kv][splits][G * (head_dim + 2)] when splits > 1
};

template <typename KV>
__global__ void __launch_bounds__(kAttnThreads) attn_kernel(const AttnArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int t = blockIdx.x, g = blockIdx.y, sp = blockIdx.z;
  const int G = a.n_head / a.n_kv, D = a.head_dim;
  const int KP = D + 4 / (int)sizeof(KV);  // K rows padded by 4 bytes: an odd word stride, no bank conflicts
  float* sq = reinterpret_cast<float*>(smem);                    // [G][D]
  float* sp_ = sq + G * D;                                       // [G][kChunk] scores / probabilities
  float* salpha = sp_ + G * kChunk;                              // [G] rescale of this chunk
  KV* sk = reinterpret_cast<KV*>(salpha + kMaxGroup);            // [kChunk][KP]
  KV* sv = reinterpret_cast<KV*>(reinterpret_cast<uintptr_t>(sk + kChunk * KP + 15) & ~uintptr_t(15));  // [kChunk][D]
  const KV* kcache = static_cast<const KV*>(a.k_cache);
  const KV* vcache = static_cast<const KV*>(a.v_cache);
  const int seq = __ldg(a.tok_seq + t), pos = __ldg(a.tok_pos + t);
  const int L = pos + 1;
  const int per = (L + a.splits - 1) / a.splits;
  const int k_lo = min(L, sp * per), k_hi = min(L, k_lo + per);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < G * D; i += kAttnThreads) sq[i] = a.q[((int64_t)t * a.n_head + g * G) * D + i];
  float m_run[kMaxGroup], l_run[kMaxGroup];
#pragma unroll
  for (int h = 0; h < kMaxGroup; ++h) {
    m_run[h] = -INFINITY;
    l_run[h] = 0.0f;
  }
  float acc[kMaxOutPerThread];
#pragma unroll
  for (int i = 0; i < kMaxOutPerThread; ++i) acc[i] = 0.0f;
  const int n_out = G * D;
  for (int c0 = k_lo; c0 < k_hi; c0 += kChunk) {
    const int nk = min(kChunk, k_hi - c0);
    __syncthreads();  // the previous chunk's K / V / p are no longer read
    // stage K and V rows of the chunk (16-byte units; rows of one 16-token block are
    // contiguous in the cache)
    constexpr int EPU = 16 / sizeof(KV);  // elements per 16-byte unit
    const int upr = D / EPU;              // 16-byte units per row
    for (int u = tid; u < nk * upr; u += kAttnThreads) {
      const int j = u / upr, c = u - j * upr;
      const int p = c0 + j;
      const int blk = __ldg(a.block_table + (int64_t)seq * a.max_blocks + p / kKvBlock);
      const int64_t row = (((int64_t)blk * a.n_kv + g) * kKvBlock + p % kKvBlock) * D;
      const uint4 kq = __ldg(reinterpret_cast<const uint4*>(kcache + row) + c);
      uint32_t* kd = reinterpret_cast<uint32_t*>(sk + j * KP + EPU * c);
      kd[0] = kq.x;
      kd[1] = kq.y;
      kd[2] = kq.z;
      kd[3] = kq.w;
      *reinterpret_cast<uint4*>(sv + j * D + EPU * c) = __ldg(reinterpret_cast<const uint4*>(vcache + row) + c);
    }
    __syncthreads();
    // scores: thread -> key j = tid % kChunk, heads h = tid / kChunk, + 2, ...
    {
      const int j = tid % kChunk;
      for (int h = tid / kChunk; h < G; h += kAttnThreads / kChunk) {
        float s = -INFINITY;
        if (j < nk) {
          const float* qh = sq + h * D;
          const KV* kr = sk + j * KP;
          float d0 = 0.0f, d1 = 0.0f;
          for (int d = 0; d < D / 2; ++d) {
            float2 kv;
            if constexpr (sizeof(KV) == 2)
              kv = __half22float2(reinterpret_cast<const __half2*>(kr)[d]);
            else
              kv = make_float2((float)kr[2 * d], (float)kr[2 * d + 1]);
            d0 = fmaf(qh[2 * d], kv.x, d0);
            d1 = fmaf(qh[2 * d + 1], kv.y, d1);
          }
          s = (d0 + d1) * a.scale;
        }
        sp_[h * kChunk + j] = s;
      }
    }
    __syncthreads();
    // online softmax statistics: warp w takes heads w, w + 4, ...
    for (int h = warp; h < G; h += kAttnThreads / 32) {
      const float s0 = sp_[h * kChunk + lane], s1 = sp_[h * kChunk + lane + 32];
      float mx = fmaxf(s0, s1);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float m_old = m_run[h];
      const float m_new = fmaxf(m_old, mx);
      const float p0 = (s0 == -INFINITY) ? 0.0f : expf(s0 - m_new);
      const float p1 = (s1 == -INFINITY) ? 0.0f : expf(s1 - m_new);
      sp_[h * kChunk + lane] = p0;
      sp_[h * kChunk + lane + 32] = p1;
      if (lane == 0) salpha[h] = (m_old == -INFINITY) ? 0.0f : expf(m_old - m_new);
      m_run[h] = m_new;  // only the warp that owns head h keeps its running max
    }
    __syncthreads();
    // accumulate p V: thread owns outputs o = tid, tid + 128, ... of the G x D block
#pragma unroll
    for (int i = 0; i < kMaxOutPerThread; ++i) {
      const int oi = tid + i * kAttnThreads;
      if (oi < n_out) {
        const int h = oi / D, d = oi - h * D;
        float s = acc[i] * salpha[h];
        const float* ph = sp_ + h * kChunk;
        for (int j = 0; j < nk; ++j) s = fmaf(ph[j], (float)sv[j * D + d], s);
        acc[i] = s;
      }
    }
    // running denominators: l = l * alpha + sum(p), identical in every thread
    for (int h = 0; h < G; ++h) {
      float ps = 0.0f;
      for (int j = 0; j < nk; ++j) ps += sp_[h * kChunk + j];
      l_run[h] = l_run[h] * salpha[h] + ps;
    }
  }
  // the per-warp m_run copies only matter for the warps that computed them; broadcast
  // each head's final max from its owning warp through shared memory
  __syncthreads();
  if (lane == 0)
    for (int h = warp; h < G; h += kAttnThreads / 32) salpha[h] = m_run[h];
  __syncthreads();
  if (a.splits == 1) {
#pragma unroll
    for (int i = 0; i < kMaxOutPerThread; ++i) {
      const int oi = tid + i * kAttnThreads;
      if (oi < n_out) {
        const int h = oi / D, d = oi - h * D;
        const float v = l_run[h] > 0.0f ? acc[i] / l_run[h] : 0.0f;
        store_from_f32(a.o, a.o_dtype, (int64_t)t * a.ldo + (int64_t)(g * G + h) * D + d, v);
      }
    }
    return;
  }
  float* pp = a.part + (((int64_t)t * a.n_kv + g) * a.splits + sp) * (int64_t)(G * (D + 2));
#pragma unroll
  for (int i = 0; i < kMaxOutPerThread; ++i) {
    const int oi = tid + i * kAttnThreads;
    if (oi < n_out) {
      const int h = oi / D, d = oi - h * D;
      pp[h * (D + 2) + d] = acc[i];
    }
  }
  if (tid < G) {
    pp[tid * (D + 2) + D] = salpha[tid];
    pp[tid * (D + 2) + D + 1] = l_run[tid];
  }
}

// Merges the splits of attn_kernel in split order: m = max m_s, l = sum l_s e^(m_s - m),
// o = sum acc_s e^(m_s - m) / l.
__global__ void attn_combine_kernel(const AttnArgs a) {
  const int t = blockIdx.x, g = blockIdx.y;
  const int G = a.n_head / a.n_kv, D = a.head_dim;
  const float* base = a.part + ((int64_t)t * a.n_kv + g) * a.splits * (int64_t)(G * (D + 2));
  for (int oi = threadIdx.x; oi < G * D; oi += blockDim.x) {
    const int h = oi / D, d = oi - h * D;
    float m = -INFINITY;
    for (int s = 0; s < a.splits; ++s) m = fmaxf(m, base[(int64_t)s * G * (D + 2) + h * (D + 2) + D]);
    float l = 0.0f, o = 0.0f;
    for (int s = 0; s < a.splits; ++s) {
      const float* p = base + (int64_t)s * G * (D + 2) + h * (D + 2);
      if (p[D] == -INFINITY) continue;  // an empty split
      const float f = expf(p[D] - m);
      l = fmaf(p[D + 1], f, l);
      o = fmaf(p[d], f, o);
    }
    store_from_f32(a.o, a.o_dtype, (int64_t)t * a.ldo + (int64_t)(g * G + h) * D + d, l > 0.0f ? o / l : 0.0f);
  }
}

// ------------------------------------------------------------------ SiLU * up
__global__ void silu_mul_kernel(const void* gate, int gdt, int64_t ldg, const void* up, int udt, int64_t ldu,
                                int64_t T, int64_t F, void* y, int ydt, int64_t ldy) {
  const int64_t n = T * F;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / F, f = i - t * F;
    const float x = load_as_f32(gate, gdt, t * ldg + f);
    const float sig = 1.0f / (expf(-x) + 1.0f);  // activation.rs:6-10
    store_from_f32(y, ydt, t * ldy + f, (x * sig) * load_as_f32(up, udt, t * ldu + f));
  }
}

// ------------------------------------------------------------------ argmax
// One CTA per row: the index of the largest logit (the lowest index among equal
// maxima; NaN never wins).
constexpr int kArgThreads = 1024;

__global__ void __launch_bounds__(kArgThreads) argmax_kernel(const float* x, int64_t ldx, int64_t V, int* out) {
  __shared__ float sv[kArgThreads / 32];
  __shared__ int si[kArgThreads / 32];
  const float* r = x + (int64_t)blockIdx.x * ldx;
  float best = -INFINITY;
  int bi = INT32_MAX;
  for (int64_t i = threadIdx.x; i < V; i += kArgThreads) {
    const float v = r[i];
    if (v > best || (bi == INT32_MAX && v == best)) {
      best = v;
      bi = (int)i;
    }
  }
  auto better = [](float v1, int i1, float v2, int i2) { return v2 > v1 || (v2 == v1 && i2 < i1); };
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v2 = __shfl_xor_sync(0xffffffffu, best, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(best, bi, v2, i2)) {
      best = v2;
      bi = i2;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = best;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = sv[0];
    int i0 = si[0];
    for (int w = 1; w < kArgThreads / 32; ++w)
      if (better(b, i0, sv[w], si[w])) {
        b = sv[w];
        i0 = si[w];
      }
    out[blockIdx.x] = i0 == INT32_MAX ? 0 : i0;
  }
}

}  // namespace

cudaError_t launch_add_rmsnorm(float* h, int64_t ldh, const void* delta, int ddt, int64_t ldd, const float* w,
                               float eps, int64_t T, int64_t H, void* y, int ydt, int64_t ldy, cudaStream_t st) {
  if (T <= 0 || H <= 0) return cudaSuccess;
  count_launch();
  add_rmsnorm_kernel<<<(unsigned)T, kNormThreads, 0, st>>>(h, ldh, delta, ddt, ldd, w, eps, H, y, ydt, ldy);
  return cudaGetLastError();
}

cudaError_t launch_rope_kv(const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v, int64_t ldv,
                           int64_t T, int n_head, int n_kv, int head_dim, int rot_dim, float theta, const int* tok_seq,
                           const int* tok_pos, const int* block_table, int max_blocks, void* k_cache, void* v_cache,
                           int kv_f32, float* q_out, cudaStream_t st) {
  if (T <= 0) return cudaSuccess;
  RopeArgs a{q, k, v, ldq, ldk, ldv, n_head, n_kv, head_dim, rot_dim, theta, tok_seq, tok_pos, block_table,
             max_blocks, k_cache, v_cache, q_out};
  const int threads = std::max(32, std::min(256, (head_dim / 2 + 31) / 32 * 32));
  const dim3 grid((unsigned)T, (unsigned)(n_head + 2 * n_kv));
  count_launch();
  if (kv_f32)
    rope_kv_kernel<float><<<grid, threads, 0, st>>>(a);
  else
    rope_kv_kernel<__half><<<grid, threads, 0, st>>>(a);
  return cudaGetLastError();
}

size_t attn_workspace_bytes(int64_t T, int n_head, int n_kv, int head_dim, int splits) {
  if (splits <= 1) return 0;
  return (size_t)T * n_kv * splits * (size_t)(n_head / n_kv) * (head_dim + 2) * sizeof(float);
}

cudaError_t launch_attention(const float* q, int64_t T, int n_head, int n_kv, int head_dim, float scale,
                             const int* tok_seq, const int* tok_pos, const int* block_table, int max_blocks,
                             const void* k_cache, const void* v_cache, int kv_f32, void* o, int o_dtype, int64_t ldo,
                             int splits, float* part, cudaStream_t st) {
  if (T <= 0) return cudaSuccess;
  AttnArgs a{q, n_head, n_kv, head_dim, scale, tok_seq, tok_pos, block_table, max_blocks, k_cache, v_cache, o,
             o_dtype, ldo, std::max(1, splits), part};
  const int G = n_head / n_kv;
  const size_t es = kv_f32 ? 4 : 2;
  const size_t smem = (size_t)G * head_dim * 4 + (size_t)G * kChunk * 4 + kMaxGroup * 4 +
                      (size_t)kChunk * head_dim * es + 4 * kChunk + 16 + (size_t)kChunk * head_dim * es;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(attn_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
    cudaFuncSetAttribute(attn_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
    configured = true;
  }
  const dim3 grid((unsigned)T, (unsigned)n_kv, (unsigned)a.splits);
  count_launch();
  if (kv_f32)
    attn_kernel<float><<<grid, kAttnThreads, smem, st>>>(a);
  else
    attn_kernel<__half><<<grid, kAttnThreads, smem, st>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || a.splits == 1) return e;
  count_launch();
  attn_combine_kernel<<<dim3((unsigned)T, (unsigned)n_kv), 256, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_silu_mul(const void* gate, int gdt, int64_t ldg, const void* up, int udt, int64_t ldu, int64_t T,
                            int64_t F, void* y, int ydt, int64_t ldy, cudaStream_t st) {
  const int64_t n = T * F;
  if (n <= 0) return cudaSuccess;
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, 4096);
  count_launch();
  silu_mul_kernel<<<(unsigned)blocks, 256, 0, st>>>(gate, gdt, ldg, up, udt, ldu, T, F, y, ydt, ldy);
  return cudaGetLastError();
}

cudaError_t launch_argmax(const float* x, int64_t ldx, int64_t T, int64_t V, int* out, cudaStream_t st) {
  if (T <= 0) return cudaSuccess;
  count_launch();
  argmax_kernel<<<(unsigned)T, kArgThreads, 0, st>>>(x, ldx, V, out);
  return cudaGetLastError();
}

}  // namespace rtd
