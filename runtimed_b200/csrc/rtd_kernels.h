// rtd_kernels.h -- host-side launchers of the CUDA kernels (internal to the library).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "rtd_layout.h"

namespace rtd {

// Decode all N rows of an uploaded weight to f32 [N, K] (bit-exact).
cudaError_t launch_dequant(int fmt, const uint8_t* w, int64_t N, int64_t K, int64_t G, float* y,
                           cudaStream_t st);
// Gather + decode rows ids[0..n) to f32 [n, K]; out-of-range ids raise the status word.
cudaError_t launch_embed(int fmt, const uint8_t* w, int64_t N, int64_t K, int64_t G, const uint32_t* ids,
                         int64_t n, float* y, int* status, cudaStream_t st);
// E4M3 encoding with the reference rounding (ties toward the lower magnitude).
cudaError_t launch_fp8_encode(const float* x, int64_t n, uint8_t* out, cudaStream_t st);

// Decode GEMV / skinny GEMM: y[M, N] = x[M, K] . W^T (+ bias), W in the group layout.
constexpr int kMaxTpWorld = 8;

// Tensor-parallel row reduction attached to one GEMV: every rank computes the
// partial y of its K shard; each tile's partial goes to every rank's receive slot
// over NVLink, and each rank writes the tile once all partials have arrived.
struct TpReduce {
  int world, rank;
  float* recv[kMaxTpWorld];      // rank p's receive region [2 parities][world][4 * max_n] f32
  uint32_t* flags[kMaxTpWorld];  // rank p's arrival flags [2 parities][world][max_tiles]
  int64_t max_n, max_tiles;
  uint32_t* ctrl;                // this rank's device words: [0] epoch of the last launch,
                                 // [1] CTAs finished in the current launch; the launch reads
                                 // the epoch after griddepcontrol.wait and its last CTA
                                 // advances it, so a CUDA graph replays with fresh epochs
                                 // (all ranks make the same calls, so epochs stay in step)
};

struct QGemvCall {
  int fmt;
  const uint8_t* w;
  int64_t N, K, G;
  const float* row_scale;  // FP8 only
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
  uint32_t* counters;      // unused by the current kernels
  int64_t n_counters;
  int* status;             // device status word
  int sm_count;
  cudaStream_t stream;
  const TpReduce* tp;      // null, or the row-parallel reduction of this call
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

// y[m, n] = bias[n] (or 0) for every row m < M: the K = 0 case of a linear.
cudaError_t launch_fill_rows(const float* bias, void* y, int y_dtype, int64_t ldy, int64_t M, int64_t N,
                             cudaStream_t st);

}  // namespace rtd
