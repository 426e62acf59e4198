// rtd_tp.cu -- two-shot all-reduce of f32 row partials over NVLink, sm_100a.
//
// Replaces ring_all_reduce / RingReducer (crates/runtimed-model/src/tp/ring_reduce.rs:7-65)
// behind RowParallelLinear::forward (crates/runtimed-model/src/tp/row_linear.rs:50-66)
// for calls the tensor-core GEMM serves (four or more tokens), and as the stand-alone
// rtd_tp_allreduce.
//
// Every rank holds a partial y[M, N] (its K shard's contribution).  The flattened M*N
// elements are cut into one block per CTA, and each block into `world` equal
// sub-chunks; sub-chunk p belongs to rank p.  CTA b of every rank:
//   1. stores sub-chunk p of its block into rank p's reduce-scatter buffer (its own
//      source slot), for every p -- peer stores over NVLink, as LL words (value and
//      epoch in one 8-byte store, so no fence or flag is needed);
//   2. waits for its own sub-chunk from every rank, sums the partials in rank order,
//      adds the bias once, and stores the sums into every rank's all-gather buffer;
//   3. waits for the whole block in its all-gather buffer and writes y.
// CTA b only ever waits for CTA b of the other ranks, which never waits for anything
// before its stores, so the protocol needs no co-residency of a rank's own CTAs.  The
// result is bit-identical on every rank (one owner computes each sum, in rank order).
// Every wait is bounded (2 s); a peer that never arrives leaves RTD_ERR_PEER_TIMEOUT in
// the status word and zeros in y.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "rtd_common.cuh"
#include "rtd_kernels.h"

namespace rtd {
namespace {

constexpr int kArThreads = 256;
constexpr int64_t kArBlocks = 128;

struct ArArgs {
  const float* partial;
  int64_t ldp;
  int64_t M, N, E;   // E = M * N
  int64_t be;        // elements per block (a multiple of 2 * world)
  const float* bias;
  void* y;
  int y_dtype;
  int64_t ldy;
  int world, rank;
  uint64_t* rs[kMaxTpWorld];
  uint64_t* ag[kMaxTpWorld];
  int64_t rs_per_src, ag_elems;
  uint32_t* ctrl;
  int* status;
};

__device__ __forceinline__ float partial_at(const ArArgs& a, int64_t i) {
  if (i >= a.E) return 0.0f;
  const int64_t t = i / a.N, n = i - t * a.N;
  return __ldg(a.partial + t * a.ldp + n);
}

__device__ __forceinline__ void store_out(const ArArgs& a, int64_t i, float v) {
  if (i >= a.E) return;
  const int64_t t = i / a.N, n = i - t * a.N;
  const int64_t off = t * a.ldy + n;
  if (a.y_dtype == 0)
    static_cast<float*>(a.y)[off] = v;
  else if (a.y_dtype == 1)
    static_cast<__half*>(a.y)[off] = __float2half_rn(v);
  else
    static_cast<__nv_bfloat16*>(a.y)[off] = __float2bfloat16_rn(v);
}

__global__ void __launch_bounds__(kArThreads) tp_allreduce_kernel(const ArArgs a) {
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the partials are the previous kernel's output
  asm volatile("griddepcontrol.launch_dependents;");
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(a.ctrl) + 1u;
  const int W = a.world, R = a.rank;
  const int64_t par = (int64_t)(epoch & 1u);
  const int64_t b = blockIdx.x, sub = a.be / W;
  const int64_t blk = b * a.be;
  // 1. reduce-scatter: sub-chunk p of this block to rank p (peers first, own slot last)
  for (int q = 1; q <= W; ++q) {
    const int p = (R + q) % W;
    uint64_t* dst = a.rs[p] + (par * W + R) * a.rs_per_src + b * sub;
    for (int64_t j = 2 * (int64_t)threadIdx.x; j < sub; j += 2 * kArThreads) {
      const int64_t i = blk + (int64_t)p * sub + j;
      st_ll2(dst + j, partial_at(a, i), partial_at(a, i + 1), epoch);
    }
  }
  // 2. the owner's sums of its sub-chunk, to every rank's all-gather buffer
  bool dead = false;
  const uint64_t* src = a.rs[R] + par * W * a.rs_per_src + b * sub;
  for (int64_t j = 2 * (int64_t)threadIdx.x; j < sub; j += 2 * kArThreads) {
    const int64_t i = blk + (int64_t)R * sub + j;
    float s0 = 0.0f, s1 = 0.0f;
    for (int q = 0; q < W; ++q) {
      float v0, v1;
      wait_ll2(src + (int64_t)q * a.rs_per_src + j, epoch, dead, a.status, v0, v1);
      s0 += v0;
      s1 += v1;
    }
    if (a.bias) {
      if (i < a.E) s0 += __ldg(a.bias + (i % a.N));
      if (i + 1 < a.E) s1 += __ldg(a.bias + ((i + 1) % a.N));
    }
    for (int q = 1; q <= W; ++q) {
      const int p = (R + q) % W;
      st_ll2(a.ag[p] + par * a.ag_elems + i, s0, s1, epoch);
    }
  }
  // 3. the whole block from the all-gather buffer
  const uint64_t* got = a.ag[R] + par * a.ag_elems;
  for (int64_t j = 2 * (int64_t)threadIdx.x; j < a.be; j += 2 * kArThreads) {
    const int64_t i = blk + j;
    if (i >= a.E) break;
    float v0, v1;
    wait_ll2(got + i, epoch, dead, a.status, v0, v1);
    store_out(a, i, v0);
    store_out(a, i + 1, v1);
  }
  // the last CTA of the launch publishes its epoch for the next exchange launch
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(a.ctrl + 1, 1u) == gridDim.x - 1) {
      a.ctrl[1] = 0u;
      a.ctrl[0] = epoch;
      __threadfence();
    }
  }
}

}  // namespace

cudaError_t launch_tp_allreduce(const TpReduce& tp, const float* partial, int64_t ldp, int64_t M, int64_t N,
                                const float* bias, void* y, int y_dtype, int64_t ldy, int* status, int sm_count,
                                cudaStream_t st) {
  if (M <= 0 || N <= 0) return cudaSuccess;
  ArArgs a{};
  a.partial = partial;
  a.ldp = ldp;
  a.M = M;
  a.N = N;
  a.E = M * N;
  const int W = tp.world;
  const int64_t quantum = 2 * (int64_t)W;
  // one block per CTA, at least 2 * kArThreads elements a block, at most kArBlocks
  // blocks: a constant, so every rank cuts the elements the same way whatever its GPU
  (void)sm_count;
  int64_t nblk = std::min<int64_t>(kArBlocks, (a.E + 2 * kArThreads - 1) / (2 * kArThreads));
  nblk = std::max<int64_t>(nblk, 1);
  a.be = ((a.E + nblk - 1) / nblk + quantum - 1) / quantum * quantum;
  nblk = (a.E + a.be - 1) / a.be;
  if (nblk * a.be > tp.ag_elems || nblk * (a.be / W) > tp.rs_per_src) return cudaErrorInvalidValue;
  a.bias = bias;
  a.y = y;
  a.y_dtype = y_dtype;
  a.ldy = ldy;
  a.world = W;
  a.rank = tp.rank;
  for (int p = 0; p < W; ++p) {
    a.rs[p] = tp.rs[p];
    a.ag[p] = tp.ag[p];
  }
  a.rs_per_src = tp.rs_per_src;
  a.ag_elems = tp.ag_elems;
  a.ctrl = tp.ctrl;
  a.status = status;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)nblk);
  cfg.blockDim = dim3(kArThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  count_launch();
  return cudaLaunchKernelEx(&cfg, tp_allreduce_kernel, a);
}

}  // namespace rtd
