// rtd_kernels.h -- host-side launchers of the CUDA kernels (internal to the library).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "rtd_layout.h"

namespace rtd {

// Kernels this library has launched (or recorded into a capturing stream) since it
// was loaded; every launch site adds one.  Read through rtd_kernel_launches.
inline std::atomic<uint64_t>& launch_counter() {
  static std::atomic<uint64_t> n{0};
  return n;
}
inline void count_launch() { launch_counter().fetch_add(1, std::memory_order_relaxed); }

// Decode all N rows of an uploaded weight to f32 [N, K] (bit-exact); row_scale (or null)
// multiplies row n's values by row_scale[n].
cudaError_t launch_dequant(int fmt, const uint8_t* w, int64_t N, int64_t K, int64_t G, const float* row_scale,
                           float* y, cudaStream_t st);
// Gather + decode rows ids[0..n) to f32 [n, K]; out-of-range ids raise the status word.
cudaError_t launch_embed(int fmt, const uint8_t* w, int64_t N, int64_t K, int64_t G, const uint32_t* ids,
                         int64_t n, float* y, int* status, cudaStream_t st);
// E4M3 encoding with the reference rounding (ties toward the lower magnitude).
cudaError_t launch_fp8_encode(const float* x, int64_t n, uint8_t* out, cudaStream_t st);

// Decode GEMV / skinny GEMM: y[M, N] = x[M, K] . W^T (+ bias), W in the group layout.
constexpr int kMaxTpWorld = 8;

// Tensor-parallel row reduction (one process per GPU).  Every exchanged value is an
// LL word (f32 value + epoch, rtd_common.cuh) stored straight into the receiving
// rank's buffer over NVLink; each exchange uses the buffer half of its epoch's parity.
//   ll : the GEMV's one-shot exchange: rank q's tile partials for rank p land in
//        ll[p][parity][q][t * N + n] (up to 4 tokens a launch), and every rank sums
//        the world's partials in rank order.
//   rs / ag : the two-shot all-reduce after the tensor-core GEMM (and rtd_tp_allreduce):
//        element i of a block goes to its owner rank's rs[owner][parity][source][...],
//        the owner sums them in rank order and stores the result into every rank's
//        ag[p][parity][i].
// Every rank therefore writes identical bits.
struct TpReduce {
  int world, rank;
  uint64_t* ll[kMaxTpWorld];
  uint64_t* rs[kMaxTpWorld];
  uint64_t* ag[kMaxTpWorld];
  int64_t max_n;        // GEMV exchange: at most 4 * max_n words per source
  int64_t rs_per_src;   // words per source in one parity half of rs
  int64_t ag_elems;     // words in one parity half of ag
  int64_t ar_max_elems; // elements one all-reduce launch may exchange
  uint32_t* ctrl;       // this rank's device words: [0] epoch of the last exchange launch,
                        // [1] CTAs finished in the current launch; a launch reads the
                        // epoch after griddepcontrol.wait and its last CTA advances it, so
                        // a CUDA graph replays with fresh epochs (all ranks make the same
                        // calls, so their epochs stay in step)
};

struct QGemvCall {
  int fmt;
  const uint8_t* w;
  int64_t N, K, G;
  const float* row_scale;  // per output row: FP8 and INT4 Marlin weights (null otherwise)
  int scale_len;           // FP8 only: 1 or N
  const void* x;
  int x_dtype;             // RTD_DT_*
  int64_t ldx;
  int64_t M;
  int w8a8;                // FP8 only: encode activations to E4M3 first
  const float* bias;       // may be null
  void* y;
  int y_dtype;
  int64_t ldy;
  float* ws;               // activation staging workspace (prep-mode calls)
  size_t ws_bytes;
  int* status;             // device status word
  int sm_count;
  cudaStream_t stream;
  const TpReduce* tp;      // null, or the row-parallel reduction of this call
  float wpow2;             // K-quant / Q8_0 weights: the power of two F of ts_decode_scale (0: none)
  // greedy argmax in the GEMV's epilogue (launch_qgemv only; null: none).  ids[t] = the
  // row of token t's largest f32 output (lowest row among equal maxima, NaN never wins,
  // 0 when every output is NaN); y may then be null.  amax: the context's [4] packed
  // keys and a finished-CTA count (word 4), zero between launches -- the last CTA of
  // each launch reads them and clears them again.
  int* ids;
  unsigned long long* amax;
  // the same epilogue, writing each token's packed key ((order-mapped f32) << 32 |
  // 0xFFFFFFFF - row) instead of its id, the rows counted from amax_row0: keys of
  // vocabulary shards combine by an unsigned max (null: ids)
  unsigned long long* amax_out;
  int64_t amax_row0;
};

// Returns cudaSuccess or the launch error; *plan_error is set (non-zero) when the
// call cannot be planned within the workspace (no launch happens then).
cudaError_t launch_qgemv(const QGemvCall& c, int* plan_error);
// Workspace bytes launch_qgemv needs for `c` (its largest token chunk).
size_t qgemv_workspace_bytes(const QGemvCall& c);

// Tensor-core (tcgen05) GEMM for larger token counts; same call description.  The
// workspace holds the staged activations (qgemm_workspace_bytes).
cudaError_t launch_qgemm(const QGemvCall& c, int* plan_error);
size_t qgemm_workspace_bytes(const QGemvCall& c);

// The skinny tensor-core GEMM (rtd_gemm_ts.cu): decoded weights written to tensor memory,
// 16..64 tokens a CTA.  launch_qgemm plans the call and runs the prep, this GEMM and (K
// split over CTAs) the reduce.  fmt: FMT_* or FMT_TS_F8X (FP8 weights x E4M3 activations).
constexpr int FMT_TS_F8X = 4;
struct TsGemm {
  int fmt;
  const uint8_t* w;
  const float* row_scale;  // per output row, or null
  int scale_len;
  float wpow2;             // the decoders' factor scale F (K-quants, Q8_0)
  int64_t N, T, G;         // rows, 16-row tiles, groups per row
  int64_t R;               // row tiles of 128 rows
  int64_t M, Mp;           // tokens (at most TN), Mp = TN
  int TN, ctas;            // tokens a CTA, persistent CTAs (stream-K over row tile x group units)
  const void* xw;          // staged activations (launch_ts_prep)
  const float* tscale;     // [Mp] per-token scale
  const float* bias;
  void* y;
  int y_dtype;
  int64_t ldy;
  int* status;
  float* partial;          // [2 * ctas][TN][128] f32: the split row tiles' partial sums
};
// f32 words of the skinny GEMM's partial-sum slots.
inline size_t ts_partial_floats(int ctas, int TN) { return (size_t)2 * ctas * TN * 128; }
// k per group of the GEMM's format, activation staging in the decoder's k order, the GEMM.
// The skinny GEMM's decoders feed the tensor cores f16 values 2^s * w (codes as exact f16
// subnormals, one FMA per pair with factors scaled by F = 2^(24 + s)); F is fixed per weight
// at upload (ts_decode_scale) so that no scaled factor exceeds the f16 range.
int ts_group_k(int gfmt);
cudaError_t launch_ts_prep(const QGemvCall& c, int gfmt, int64_t Mp, int64_t kp, void* xw, float* tscale);
cudaError_t launch_ts_gemm(const TsGemm& g, cudaStream_t st);

// y[M, N] (y_dtype, rows ldy apart) = sum over ranks of partial[M, N] (f32, rows ldp
// apart) + bias (added once), on every rank: the two-shot all-reduce over NVLink.
// M * N must not exceed tp.ar_max_elems.
cudaError_t launch_tp_allreduce(const TpReduce& tp, const float* partial, int64_t ldp, int64_t M, int64_t N,
                                const float* bias, void* y, int y_dtype, int64_t ldy, int* status, int sm_count,
                                cudaStream_t st);

// Decoder-layer operations (rtd_model.cu).
cudaError_t launch_add_rmsnorm(float* h, int64_t ldh, const void* delta, int ddt, int64_t ldd, const float* w,
                               float eps, int64_t T, int64_t H, void* y, int ydt, int64_t ldy, cudaStream_t st);
cudaError_t launch_rope_kv(const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v, int64_t ldv,
                           int64_t T, int n_head, int n_kv, int head_dim, int rot_dim, float theta, const int* tok_seq,
                           const int* tok_pos, const int* block_table, int max_blocks, void* k_cache, void* v_cache,
                           int kv_f32, float* q_out, cudaStream_t st);
size_t attn_workspace_bytes(int64_t T, int n_head, int n_kv, int head_dim, int splits);
cudaError_t launch_attention(const float* q, int64_t T, int n_head, int n_kv, int head_dim, float scale,
                             const int* tok_seq, const int* tok_pos, const int* block_table, int max_blocks,
                             const void* k_cache, const void* v_cache, int kv_f32, void* o, int o_dtype, int64_t ldo,
                             int splits, float* part, cudaStream_t st);
cudaError_t launch_silu_mul(const void* gate, int gdt, int64_t ldg, const void* up, int udt, int64_t ldu, int64_t T,
                            int64_t F, void* y, int ydt, int64_t ldy, cudaStream_t st);
cudaError_t launch_argmax(const float* x, int64_t ldx, int64_t T, int64_t V, int* out, cudaStream_t st);

// y[m, n] = bias[n] (or 0) for every row m < M: the K = 0 case of a linear.
cudaError_t launch_fill_rows(const float* bias, void* y, int y_dtype, int64_t ldy, int64_t M, int64_t N,
                             cudaStream_t st);

}  // namespace rtd
