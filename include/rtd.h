/*
 * rtd.h -- C ABI of libruntimed_b200, the sm_100a quantized-linear hot path.
 *
 * Drop-in boundary for syntropd/runtimed's quantized forward pass.  Every entry
 * point names the reference interface it replaces (paths relative to the
 * runtimed project root).  Conventions:
 *   - plain pointers and sizes only; `stream` is a cudaStream_t passed as void*
 *     (NULL = the legacy default stream);
 *   - every call returns an rtd_status; nothing throws across the ABI;
 *   - weights are uploaded once and owned by the library (opaque handles);
 *     activations and outputs are caller-owned DEVICE buffers;
 *   - the compute entry points allocate nothing: scratch comes from the
 *     context's workspace, reserved by rtd_init.  Calls that share one context
 *     must not overlap on the GPU (the reference serialises forwards per model
 *     with Mutex<Session>: crates/runtimed-core/src/model/meta.rs:31-45).
 */
#ifndef RTD_H
#define RTD_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* The library is built with hidden visibility; only this ABI is exported. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

typedef int32_t rtd_status;

/* Status codes.  Mapping onto crates/runtimed-model/src/error.rs:6-27 ModelError:
 *   RTD_ERR_SHAPE -> ModelError::Shape; RTD_ERR_UNSUPPORTED / RTD_ERR_TRUNCATED ->
 *   ModelError::Gguf(GgufError::{Unsupported, Truncated}); everything else ->
 *   ModelError::Config(rtd_last_error(ctx)). */
enum {
    RTD_OK = 0,
    RTD_ERR_INVALID = 1,       /* null handle/pointer, bad enum value */
    RTD_ERR_SHAPE = 2,         /* dimensions inconsistent or not a block multiple */
    RTD_ERR_UNSUPPORTED = 3,   /* ggml type not on this path */
    RTD_ERR_TRUNCATED = 4,     /* byte buffer shorter than the tensor needs */
    RTD_ERR_CUDA = 5,          /* a CUDA runtime call failed */
    RTD_ERR_OOM = 6,           /* device allocation failed (upload / init only) */
    RTD_ERR_PEER_TIMEOUT = 7,  /* a bounded cross-GPU wait gave up */
    RTD_ERR_INDEX = 8,         /* an embedding id was out of range */
    RTD_ERR_DEVICE = 9,        /* a kernel raised the context's device status word */
    RTD_ERR_WORKSPACE = 10     /* the call needs more scratch than the context reserved */
};

/* GGML type ids (crates/runtimed-gguf/src/quant/dtype.rs:27-46), and the id this library
 * reports for INT4 Marlin weights (rtd_marlin_upload; not a GGUF type). */
enum { RTD_TYPE_Q8_0 = 8, RTD_TYPE_Q4_K = 12, RTD_TYPE_Q6_K = 14, RTD_TYPE_INT4_MARLIN = 1001 };

/* Activation / output element types. */
enum { RTD_DT_F32 = 0, RTD_DT_F16 = 1, RTD_DT_BF16 = 2 };

/* FP8 linear modes.  W8A16: activations stay 16/32-bit (E4M3 -> f16 is exact);
 * W8A8: activations are first encoded to E4M3 with the reference encoder
 * (crates/runtimed-model/src/ops/fp8_gemm.rs:96-101), as its cuBLASLt path does. */
enum { RTD_FP8_W8A16 = 0, RTD_FP8_W8A8 = 1 };

typedef struct rtd_ctx rtd_ctx;
typedef struct rtd_qweight rtd_qweight;
typedef struct rtd_fp8weight rtd_fp8weight;

/* ---- context ---------------------------------------------------------------
 * Replaces the device binding of Weights::ensure_current
 * (crates/runtimed-model/src/weights/store.rs:128-145): a context binds one CUDA
 * device and owns the scratch workspace and the device status word. */
rtd_status rtd_init(int device, rtd_ctx** out);
rtd_status rtd_destroy(rtd_ctx* ctx);
/* Last error message recorded on `ctx` (or on the calling thread when ctx is NULL). */
const char* rtd_last_error(const rtd_ctx* ctx);
/* No counterpart in the reference (diagnostics): kernels the library has launched,
 * or recorded into a capturing stream, since it was loaded. */
uint64_t rtd_kernel_launches(void);
/* Synchronises `stream` and reads then clears the device status word. */
rtd_status rtd_check_device_status(rtd_ctx* ctx, void* stream);
/* Block geometry (crates/runtimed-gguf/src/quant/dtype.rs:49-64). */
rtd_status rtd_block_geometry(uint32_t ggml_type, int64_t* elems, int64_t* bytes);

/* ---- quantized weights -----------------------------------------------------
 * Replaces load_quantized_tensor (crates/runtimed-model/src/weights/load_gguf.rs:28-38):
 * raw GGUF superblocks of an [N, K] matrix (N rows of K/elems blocks, the layout
 * GgufFile::tensor_bytes returns, crates/runtimed-gguf/src/header.rs:191-205) are
 * copied from host memory to the device once and re-tiled there for the kernels. */
rtd_status rtd_qweight_upload(rtd_ctx* ctx, uint32_t ggml_type, const void* host_blocks,
                              size_t nbytes, int64_t N, int64_t K, rtd_qweight** out);
rtd_status rtd_qweight_free(rtd_qweight* w);
/* INT4 Marlin weights.  Replaces MarlinWeight::new / to the device and the sm_80 PTX GEMV
 * behind marlin_gemv (crates/runtimed-model/src/ops/marlin_gemv.rs:20-31,122-202,
 * ops/ptx_marlin.rs): packed = host u32 [ceil(K / 32)][N][4] (nibble i of word w of chunk c
 * is k = 32c + 8w + i), scales = host f32 [N]; value = (q - 8) * scales[n].  The handle
 * works with rtd_qlinear (any token count) and rtd_qdequant (bit-exact with
 * MarlinWeight::dequantize); rtd_qembed and the row-parallel entry refuse it
 * (RTD_ERR_UNSUPPORTED).  rtd_qweight_info reports RTD_TYPE_INT4_MARLIN and, as raw_bytes,
 * MarlinWeight::resident_bytes. */
rtd_status rtd_marlin_upload(rtd_ctx* ctx, const uint32_t* packed, const float* scales, int64_t N, int64_t K,
                             rtd_qweight** out);
/* A copy of `src` owned by `ctx` (same or another device), made on the devices without
 * a host round trip.  Replaces Weights::to_device (crates/runtimed-model/src/weights/store.rs:170-205)
 * for quantized entries, which stay quantized (the reference leaves q_map entries in place). */
rtd_status rtd_qweight_to_device(const rtd_qweight* src, rtd_ctx* ctx, rtd_qweight** out);
/* Rows [row0, row0 + rows) of an uploaded weight as a handle that shares its device memory
 * (row0 a multiple of 16; the parent must outlive the view; freeing the view frees no
 * memory): the quantized counterpart of narrowing a weight's rows
 * (crates/runtimed-model/src/arch/qwen2.rs:182-184).  A caller can upload sibling weights
 * that read the same input as one row-concatenated matrix -- one launch serves them all --
 * and still address each by name. */
rtd_status rtd_qweight_rows(const rtd_qweight* w, int64_t row0, int64_t rows, rtd_qweight** out);

/* raw_bytes = the GGUF byte count (QTensor::storage_size_in_bytes, store.rs:57-76);
 * device_bytes = what the device copy occupies (rows padded to a tile of 16). */
rtd_status rtd_qweight_info(const rtd_qweight* w, uint32_t* ggml_type, int64_t* N, int64_t* K,
                            size_t* raw_bytes, size_t* device_bytes);

/* y[M, N] = x[M, K] . W^T (+ bias[N]).  Replaces Weights::linear -> QMatMul::forward
 * (crates/runtimed-model/src/weights/linear_layer.rs:45-52) and, with a bias,
 * Weights::linear_bias (linear_layer.rs:107-118).  x rows are `ldx` elements apart
 * and y rows `ldy` elements apart (pass K and N for dense rows).  bias is f32 on the
 * device or NULL. */
rtd_status rtd_qlinear(rtd_ctx* ctx, const rtd_qweight* w, const void* x, uint32_t x_dtype,
                       int64_t ldx, int64_t M, const float* bias, void* y, uint32_t y_dtype,
                       int64_t ldy, void* stream);

/* y[n, K] (f32) = dequantized rows ids[0..n) of W.  Replaces Weights::embed ->
 * QMatMul::embedding (crates/runtimed-model/src/weights/embed_layer.rs:16-57).
 * ids is a device array; an id >= N writes a zero row and raises RTD_ERR_INDEX in
 * the device status word (read it with rtd_check_device_status). */
rtd_status rtd_qembed(rtd_ctx* ctx, const rtd_qweight* w, const uint32_t* ids, int64_t n,
                      float* y, void* stream);

/* y[N, K] (f32) = the whole dequantized matrix, bit-exact with the reference
 * decoders (crates/runtimed-gguf/src/quant/dequant.rs:83-146).  Replaces
 * Weights::get on a q_map entry (crates/runtimed-model/src/weights/store.rs:88-97). */
rtd_status rtd_qdequant(rtd_ctx* ctx, const rtd_qweight* w, float* y, void* stream);

/* ---- FP8 E4M3 --------------------------------------------------------------
 * Replaces Fp8Weight::new (crates/runtimed-model/src/weights/fp8_weight.rs:17-41):
 * E4M3 bytes [N, K] row-major and scale[scale_len] (1 = per tensor, N = per output
 * channel), both host memory. */
rtd_status rtd_fp8weight_upload(rtd_ctx* ctx, const uint8_t* host_w, const float* host_scale,
                                int64_t scale_len, int64_t N, int64_t K, rtd_fp8weight** out);
rtd_status rtd_fp8weight_free(rtd_fp8weight* w);

/* y[M, N] = x . (E4M3(W) * scale)^T.  Replaces SubstratePort::fp8_gemm / ops::fp8_gemm
 * (crates/runtimed-model/src/substrate/port.rs:73, crates/runtimed-model/src/ops/fp8_gemm.rs:77-191). */
rtd_status rtd_fp8_linear(rtd_ctx* ctx, const rtd_fp8weight* w, const void* x, uint32_t x_dtype,
                          int64_t ldx, int64_t M, void* y, uint32_t y_dtype, int64_t ldy,
                          uint32_t mode, void* stream);

/* out[i] = E4M3 encoding of x[i] (f32, device), ties toward the lower magnitude,
 * saturating at 448.  Replaces the host loop of f32_to_fp8_e4m3
 * (crates/runtimed-model/src/weights/load_safetensors.rs:53-69) used at fp8_gemm.rs:98-99. */
rtd_status rtd_fp8_encode(rtd_ctx* ctx, const float* x, int64_t n, uint8_t* out, void* stream);

/* ---- decoder-layer operations ------------------------------------------------
 * The SubstratePort operations between the linears of a decoder layer
 * (crates/runtimed-model/src/substrate/port.rs:14-90), on device buffers.  The KV cache
 * is PAGED: k_cache / v_cache are [blocks][n_kv][16][head_dim] of kv_dtype
 * (RTD_DT_F16, or RTD_DT_F32 for the reference's f32 cache precision); block_table is
 * int32 [sequences][max_blocks] (block ids per 16-token span of a sequence); every
 * token of a call carries its own sequence (tok_seq) and position (tok_pos), int32 on
 * the device, so one call serves a prefill chunk, a batched decode step or a verify of
 * several positions. */

/* h[T, H] (f32, in place) += delta (optional, delta_dtype), then
 * y = (h / sqrt(mean(h^2) + eps)) * w: rmsnorm (crates/runtimed-model/src/ops/norm.rs:7-11)
 * fused with the residual add before it (crates/runtimed-model/src/arch/qwen2.rs:112,126). */
rtd_status rtd_rmsnorm(rtd_ctx* ctx, float* h, int64_t ldh, const void* delta, uint32_t delta_dtype, int64_t ldd,
                       const float* w, float eps, int64_t T, int64_t H, void* y, uint32_t y_dtype, int64_t ldy,
                       void* stream);
/* NeoX rope (crates/runtimed-model/src/ops/rope.rs:24-60) on the query and key heads of
 * the q / k / v linear outputs (f32), queries into q_out [T][n_head][head_dim] (f32), keys
 * and values appended to the paged cache at each token's (sequence, position):
 * SubstratePort::rope + Cache::append (crates/runtimed-model/src/arch/qwen2.rs:100-103). */
rtd_status rtd_rope_kv_append(rtd_ctx* ctx, const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v,
                              int64_t ldv, int64_t T, int32_t n_head, int32_t n_kv, int32_t head_dim, int32_t rot_dim,
                              float theta, const int32_t* tok_seq, const int32_t* tok_pos, const int32_t* block_table,
                              int32_t max_blocks, void* k_cache, void* v_cache, uint32_t kv_dtype, float* q_out,
                              void* stream);
/* o[T, n_head * head_dim] = softmax(q k^T * scale + causal mask) v with GQA, over keys
 * [0, tok_pos[t]] of each token's sequence: SubstratePort::attention + causal_mask
 * (crates/runtimed-model/src/ops/attention.rs:38-58,107-128).  max_ctx bounds
 * tok_pos + 1 (it sizes the split of long contexts across CTAs). */
rtd_status rtd_attention_paged(rtd_ctx* ctx, const float* q, int64_t T, int32_t n_head, int32_t n_kv, int32_t head_dim,
                               float scale, const int32_t* tok_seq, const int32_t* tok_pos, const int32_t* block_table,
                               int32_t max_blocks, int32_t max_ctx, const void* k_cache, const void* v_cache,
                               uint32_t kv_dtype, void* o, uint32_t o_dtype, int64_t ldo, void* stream);
/* y[t, f] = silu(gate[t, f]) * up[t, f] for t < T, f < F (rows ldg / ldu / ldy elements
 * apart; y may alias gate): SubstratePort::silu + broadcast_mul
 * (crates/runtimed-model/src/ops/activation.rs:6-10, arch/qwen2.rs:120-123). */
rtd_status rtd_silu_mul(rtd_ctx* ctx, const void* gate, uint32_t gate_dtype, int64_t ldg, const void* up,
                        uint32_t up_dtype, int64_t ldu, int64_t T, int64_t F, void* y, uint32_t y_dtype, int64_t ldy,
                        void* stream);
/* out[t] = argmax of row t of x[T, V] (f32; lowest index among equal maxima):
 * SubstratePort::argmax behind greedy sampling (crates/runtimed-model/src/decode/sample.rs:11-18). */
rtd_status rtd_argmax(rtd_ctx* ctx, const float* x, int64_t ldx, int64_t T, int64_t V, int32_t* out, void* stream);

/* The LM head and the greedy pick in one call: ids[t] = argmax over n of the f32 value of
 * y[t, n] = x[t] . W[n] (+ bias[n]), ties to the lowest row, NaN never chosen (0 when every
 * value is NaN) -- qwen2::forward's `linear(h, "output.weight")` followed by
 * SubstratePort::argmax (crates/runtimed-model/src/arch/qwen2.rs:224-228,
 * crates/runtimed-model/src/decode/sample.rs:11-18).  Fewer than four tokens (decode): the
 * argmax runs in the GEMV's epilogue, so no logits need to exist -- y may be NULL; when
 * given, the logits are written too, in y_dtype.  Four or more tokens: y (f32) is required
 * and rtd_argmax follows the linear.  ids is a device array of M int32.  The context holds
 * the epilogue's key state: calls of one context must not overlap on different streams. */
rtd_status rtd_qlinear_argmax(rtd_ctx* ctx, const rtd_qweight* w, const void* x, uint32_t x_dtype,
                              int64_t ldx, int64_t M, const float* bias, void* y, uint32_t y_dtype,
                              int64_t ldy, int32_t* ids, void* stream);

/* The same pick for one shard of a vocabulary-parallel LM head (the column-parallel head
 * with a distributed argmax: each rank holds rows [row0, row0 + N) of output.weight).
 * keys[t] (device u64) = (f32 order mapped onto unsigned, -0 as +0) << 32 | (0xFFFFFFFF -
 * (row0 + n)) of token t's largest output, 0 when every output is NaN: the unsigned maximum
 * of the ranks' keys is the key of the whole head's greedy pick, whose row is 0xFFFFFFFF
 * minus its low word (0 for the key 0).  Any M, in GEMV launches of up to four tokens; rows
 * below 2^32. */
rtd_status rtd_qlinear_argmax_keys(rtd_ctx* ctx, const rtd_qweight* w, const void* x, uint32_t x_dtype,
                                   int64_t ldx, int64_t M, const float* bias, int64_t row0, uint64_t* keys,
                                   void* stream);

/* ---- tensor-parallel row reduction -----------------------------------------
 * Replaces RowParallelLinear::forward + ring_all_reduce
 * (crates/runtimed-model/src/tp/row_linear.rs:20-66, crates/runtimed-model/src/tp/ring_reduce.rs:7-65)
 * for one process per GPU: each rank holds the [N, K/world] column shard of a
 * quantized matrix (rtd_qweight_upload of the shard's blocks) and its slice of x, and
 * every rank receives the full, reduced y[M, N] (+ bias once), bit-identical on every
 * rank.  Up to three tokens run the decode GEMV with the exchange fused into its
 * epilogue (tile partials stored into the peers' buffers over NVLink as they are
 * produced); four or more run the tensor-core GEMM into an f32 partial followed by the
 * two-shot all-reduce of rtd_tp_allreduce.  Set-up:
 *   1. rtd_tp_comm_create on every rank -> RTD_IPC_HANDLE_BYTES of handle bytes;
 *   2. the caller exchanges the handles (rank order) by its own means;
 *   3. rtd_tp_comm_open with all handles.
 * Every rank must issue the same sequence of rtd_tp_qlinear_row / rtd_tp_allreduce
 * calls with the same M and N; a rank that does not arrive within 2 s makes the others
 * finish with RTD_ERR_PEER_TIMEOUT in the device status word (rtd_check_device_status),
 * after which the communicator must be re-created.  The calls keep their exchange epoch
 * on the device, so they may be captured in a CUDA graph and replayed (all ranks
 * replaying their graphs in step). */
#define RTD_IPC_HANDLE_BYTES 64
typedef struct rtd_comm rtd_comm;
rtd_status rtd_tp_comm_create(rtd_ctx* ctx, int rank, int world, int64_t max_n, rtd_comm** out, void* handle_out);
rtd_status rtd_tp_comm_open(rtd_comm* comm, const void* handles);
rtd_status rtd_tp_comm_destroy(rtd_comm* comm);
rtd_status rtd_tp_qlinear_row(rtd_comm* comm, const rtd_qweight* shard, const void* x, uint32_t x_dtype,
                              int64_t ldx, int64_t M, const float* bias, void* y, uint32_t y_dtype, int64_t ldy,
                              void* stream);
/* y[M, N] = sum over ranks of partial[M, N] (+ bias once) on every rank: the all-reduce
 * of ring_all_reduce / RingReducer (crates/runtimed-model/src/tp/ring_reduce.rs:7-65).
 * partial is f32 on the device (rows ldp apart); y is y_dtype (rows ldy apart); N must
 * not exceed the communicator's max_n.  Two-shot over NVLink: each rank reduces one
 * sub-chunk of every block and stores the sums into every rank's buffer. */
rtd_status rtd_tp_allreduce(rtd_comm* comm, const float* partial, int64_t ldp, int64_t M, int64_t N,
                            const float* bias, void* y, uint32_t y_dtype, int64_t ldy, void* stream);

/* ---- allocation-free linear -------------------------------------------------
 * No counterpart in the reference: an addition for callers that must not allocate
 * device memory while they run (e.g. code working under another allocator's fixed
 * device-memory budget, where a cudaMalloc can fail or stall the device).
 * Same contract and dispatch as rtd_qlinear (the tensor-core GEMM from four tokens on
 * when its staging fits, the decode GEMV otherwise), but no context argument: the
 * scratch is a fixed 1 MiB array per device inside the library (256 B status word +
 * workspace); the call allocates nothing and calls no allocating routine.
 *   - The first call on a device looks the array up (cudaGetSymbolAddress) with that
 *     device current; make that first call before any stream capture.
 *   - A call whose staging would exceed the scratch returns RTD_ERR_WORKSPACE and
 *     launches nothing (bf16 / f16 rows up to K = 16384 stage on chip and need
 *     no scratch beyond their small carve; f32 rows need about 4*K*M bytes).  Calls
 *     of four or more tokens whose GEMM staging (about 2*K*M bytes plus split-K
 *     partials) does not fit run the decode GEMV in passes of up to four tokens.
 *   - Every call shares the one array: calls that overlap on the GPU race, so issue
 *     them on one stream (or serialise them).
 *   - Host-side errors are recorded on the calling thread: read them with
 *     rtd_last_error(NULL).  Device-side errors (a bounded wait that gave up) raise
 *     the array's status word, which stays raised until rtd_noalloc_check_status
 *     reads and clears it. */
rtd_status rtd_qlinear_noalloc(const rtd_qweight* w, const void* x, uint32_t x_dtype, int64_t ldx, int64_t M,
                               const float* bias, void* y, uint32_t y_dtype, int64_t ldy, void* stream);
/* No counterpart in the reference: synchronises `stream`, then reads and clears the
 * status word of `device`'s allocation-free scratch (RTD_OK, or the raised code). */
rtd_status rtd_noalloc_check_status(int device, void* stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* RTD_H */
