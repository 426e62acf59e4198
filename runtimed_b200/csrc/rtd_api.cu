// rtd_api.cu -- the C ABI of libruntimed_b200 (declared in include/rtd.h).
//
// Host-side operator surface: contexts, weight handles, argument validation and
// dispatch to the sm_100a kernels.  Weight uploads allocate (once, at load time);
// the compute entry points never allocate -- their scratch is the context
// workspace reserved by rtd_init.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <algorithm>
#include <climits>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "rtd.h"
#include "rtd_kernels.h"
#include "rtd_layout.h"

struct rtd_ctx {
  int device = 0;
  int sm_count = 148;
  float* ws = nullptr;
  size_t ws_bytes = 0;
  int* status = nullptr;
  // rtd_qlinear_argmax's epilogue state: [4] packed keys and a CTA count, zero between calls
  unsigned long long* amax = nullptr;
  std::string err;
};

struct rtd_qweight {
  rtd_ctx* ctx = nullptr;
  int fmt = 0;
  uint32_t ggml_type = 0;
  int64_t N = 0, K = 0, G = 0, T = 0;
  uint8_t* dev = nullptr;
  size_t dev_bytes = 0, raw_bytes = 0;
  bool owns = true;  // false for a row view (rtd_qweight_rows): the parent owns the memory
  float wpow2 = 0.0f;  // rtd::ts_decode_scale of the raw blocks
  // INT4 Marlin weights (rtd_marlin_upload): held as Q4_K groups whose codes decode to
  // q - 8, with the per-row f32 scale applied by every kernel's epilogue
  float* row_scale = nullptr;
  bool owns_scale = false;
};

struct rtd_fp8weight {
  rtd_ctx* ctx = nullptr;
  int64_t N = 0, K = 0, G = 0, T = 0;
  uint8_t* dev = nullptr;
  float* scale = nullptr;
  int64_t scale_len = 0;
  size_t dev_bytes = 0;
};

namespace {

constexpr size_t kWorkspaceBytes = 64ull << 20;  // activation staging (GEMV prep, GEMM tiles)
// calls with at least this many tokens go to the tensor-core GEMM: measured on B200,
// the four-column GEMV pass is slower than one TN = 16 GEMM tile from M = 4 on, and
// faster up to M = 3
constexpr int64_t kGemmMinTokens = 4;
constexpr size_t kAmaxBytes = 64;  // rtd_ctx::amax: 4 keys of 8 bytes, the count, padding

thread_local std::string g_thread_err;

rtd_status fail(rtd_ctx* ctx, rtd_status code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (ctx)
    ctx->err = buf;
  else
    g_thread_err = buf;
  return code;
}

rtd_status cuda_fail(rtd_ctx* ctx, cudaError_t e, const char* what) {
  return fail(ctx, RTD_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// Binds the context's device for the duration of a call and restores the
// caller's device afterwards (the reference re-binds per call in ensure_current).
struct DeviceGuard {
  int prev = -1;
  cudaError_t err = cudaSuccess;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) err = cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

int fmt_of_type(uint32_t t) {
  switch (t) {
    case RTD_TYPE_Q4_K: return rtd::FMT_Q4K;
    case RTD_TYPE_Q6_K: return rtd::FMT_Q6K;
    case RTD_TYPE_Q8_0: return rtd::FMT_Q80;
    default: return -1;
  }
}

bool valid_dtype(uint32_t d) { return d == RTD_DT_F32 || d == RTD_DT_F16 || d == RTD_DT_BF16; }

}  // namespace

extern "C" {

const char* rtd_last_error(const rtd_ctx* ctx) { return ctx ? ctx->err.c_str() : g_thread_err.c_str(); }

uint64_t rtd_kernel_launches(void) { return rtd::launch_counter().load(std::memory_order_relaxed); }

rtd_status rtd_block_geometry(uint32_t ggml_type, int64_t* elems, int64_t* bytes) {
  int64_t e, b;
  switch (ggml_type) {
    case 0: e = 1; b = 4; break;
    case 1: case 30: e = 1; b = 2; break;
    case 2: e = 32; b = 18; break;
    case 6: e = 32; b = 22; break;
    case 8: e = 32; b = 34; break;
    case 10: e = 256; b = 84; break;
    case 11: e = 256; b = 110; break;
    case 12: e = 256; b = 144; break;
    case 13: e = 256; b = 176; break;
    case 14: e = 256; b = 210; break;
    default: return fail(nullptr, RTD_ERR_UNSUPPORTED, "ggml type %u has no block geometry", ggml_type);
  }
  if (elems) *elems = e;
  if (bytes) *bytes = b;
  return RTD_OK;
}

rtd_status rtd_init(int device, rtd_ctx** out) {
  if (!out) return fail(nullptr, RTD_ERR_INVALID, "rtd_init: out is NULL");
  *out = nullptr;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || device < 0 || device >= n)
    return fail(nullptr, RTD_ERR_CUDA, "rtd_init: device %d not available (%d devices, %s)", device, n,
                cudaGetErrorString(e));
  rtd_ctx* c = new (std::nothrow) rtd_ctx();
  if (!c) return fail(nullptr, RTD_ERR_OOM, "rtd_init: host allocation failed");
  c->device = device;
  DeviceGuard g(device);
  if (g.err != cudaSuccess) {
    delete c;
    return fail(nullptr, RTD_ERR_CUDA, "rtd_init: cudaSetDevice: %s", cudaGetErrorString(g.err));
  }
  cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, device);
  if ((e = cudaMalloc(&c->ws, kWorkspaceBytes)) != cudaSuccess ||
      (e = cudaMalloc(&c->status, sizeof(int))) != cudaSuccess ||
      (e = cudaMemset(c->status, 0, sizeof(int))) != cudaSuccess ||
      (e = cudaMalloc(&c->amax, kAmaxBytes)) != cudaSuccess || (e = cudaMemset(c->amax, 0, kAmaxBytes)) != cudaSuccess) {
    cudaFree(c->ws);
    cudaFree(c->status);
    cudaFree(c->amax);
    delete c;
    return fail(nullptr, RTD_ERR_OOM, "rtd_init: workspace allocation failed: %s", cudaGetErrorString(e));
  }
  c->ws_bytes = kWorkspaceBytes;
  *out = c;
  return RTD_OK;
}

rtd_status rtd_destroy(rtd_ctx* ctx) {
  if (!ctx) return RTD_OK;
  DeviceGuard g(ctx->device);
  cudaFree(ctx->ws);
  cudaFree(ctx->status);
  cudaFree(ctx->amax);
  delete ctx;
  return RTD_OK;
}

rtd_status rtd_check_device_status(rtd_ctx* ctx, void* stream) {
  if (!ctx) return fail(nullptr, RTD_ERR_INVALID, "rtd_check_device_status: ctx is NULL");
  DeviceGuard g(ctx->device);
  cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "rtd_check_device_status: stream");
  int v = 0;
  if ((e = cudaMemcpy(&v, ctx->status, sizeof(int), cudaMemcpyDeviceToHost)) != cudaSuccess)
    return cuda_fail(ctx, e, "rtd_check_device_status: read");
  if (v != 0) {
    cudaMemset(ctx->status, 0, sizeof(int));
    if (v == RTD_ERR_INDEX) return fail(ctx, RTD_ERR_INDEX, "embedding id out of range");
    if (v == RTD_ERR_PEER_TIMEOUT)
      return fail(ctx, RTD_ERR_PEER_TIMEOUT, "a tensor-parallel peer did not arrive within the wait budget");
    return fail(ctx, RTD_ERR_DEVICE, "device status word raised code %d", v);
  }
  return RTD_OK;
}

rtd_status rtd_qweight_upload(rtd_ctx* ctx, uint32_t ggml_type, const void* host_blocks, size_t nbytes,
                              int64_t N, int64_t K, rtd_qweight** out) {
  if (!ctx || !out) return fail(ctx, RTD_ERR_INVALID, "rtd_qweight_upload: NULL argument");
  if (ggml_type == RTD_TYPE_INT4_MARLIN)
    return fail(ctx, RTD_ERR_UNSUPPORTED, "rtd_qweight_upload: INT4 Marlin weights go through rtd_marlin_upload");
  *out = nullptr;
  const int fmt = fmt_of_type(ggml_type);
  if (fmt < 0) return fail(ctx, RTD_ERR_UNSUPPORTED, "rtd_qweight_upload: ggml type %u is not Q4_K/Q6_K/Q8_0", ggml_type);
  if (N < 0 || K < 0) return fail(ctx, RTD_ERR_SHAPE, "rtd_qweight_upload: negative shape [%lld, %lld]", (long long)N, (long long)K);
  const rtd::FmtInfo f = rtd::fmt_info(fmt);
  if (K % f.block_elems != 0)
    return fail(ctx, RTD_ERR_SHAPE, "rtd_qweight_upload: K=%lld is not a multiple of the block size %d",
                (long long)K, f.block_elems);
  const size_t need = (size_t)N * (size_t)(K / f.block_elems) * (size_t)f.block_bytes;
  if (nbytes < need)
    return fail(ctx, RTD_ERR_TRUNCATED, "rtd_qweight_upload: %zu bytes given, %zu needed", nbytes, need);
  if (need > 0 && !host_blocks) return fail(ctx, RTD_ERR_INVALID, "rtd_qweight_upload: host_blocks is NULL");
  rtd_qweight* w = new (std::nothrow) rtd_qweight();
  if (!w) return fail(ctx, RTD_ERR_OOM, "rtd_qweight_upload: host allocation failed");
  w->ctx = ctx;
  w->fmt = fmt;
  w->ggml_type = ggml_type;
  w->N = N;
  w->K = K;
  w->T = rtd::tiles_for(N);
  w->G = rtd::groups_for(fmt, K);
  w->raw_bytes = need;
  w->dev_bytes = (size_t)(w->T * w->G) * (size_t)f.gb;
  if (w->dev_bytes > 0) {
    std::vector<uint8_t> host;
    try {
      host.resize(w->dev_bytes);
    } catch (...) {
      delete w;
      return fail(ctx, RTD_ERR_OOM, "rtd_qweight_upload: host staging allocation failed");
    }
    rtd::repack_host(fmt, static_cast<const uint8_t*>(host_blocks), N, K, host.data());
    w->wpow2 = rtd::ts_decode_scale(fmt, static_cast<const uint8_t*>(host_blocks), N, K);
    DeviceGuard g(ctx->device);
    cudaError_t e = cudaMalloc(&w->dev, w->dev_bytes);
    if (e != cudaSuccess) {
      delete w;
      return fail(ctx, RTD_ERR_OOM, "rtd_qweight_upload: cudaMalloc(%zu): %s", w->dev_bytes, cudaGetErrorString(e));
    }
    if ((e = cudaMemcpy(w->dev, host.data(), w->dev_bytes, cudaMemcpyHostToDevice)) != cudaSuccess) {
      cudaFree(w->dev);
      delete w;
      return cuda_fail(ctx, e, "rtd_qweight_upload: copy");
    }
  }
  *out = w;
  return RTD_OK;
}

// INT4 Marlin weights (marlin_gemv.rs:11-97): packed[ceil(K/32)][N][4] u32 words, nibble
// `nib` of word `w` of chunk c holding k = 32c + 8w + nib, value (q - 8) * scales[n].  They
// are held as Q4_K groups whose headers make every code decode to q - 8 exactly (d = 1,
// dmin = 8, all sub-block scales and mins 1: d*sc*q - dmin*m = q - 8), so the GEMV and
// both tensor-core GEMMs run them unchanged; the f32 row scale is applied where the FP8
// row scale is, in every epilogue.  K is padded to 256 with code 8 (value 0).
rtd_status rtd_marlin_upload(rtd_ctx* ctx, const uint32_t* packed, const float* scales, int64_t N, int64_t K,
                             rtd_qweight** out) {
  const char* who = "rtd_marlin_upload";
  if (!ctx || !out) return fail(ctx, RTD_ERR_INVALID, "%s: NULL argument", who);
  *out = nullptr;
  if (N < 0 || K < 0) return fail(ctx, RTD_ERR_SHAPE, "%s: negative shape [%lld, %lld]", who, (long long)N, (long long)K);
  if (N > 0 && K > 0 && (!packed || !scales)) return fail(ctx, RTD_ERR_INVALID, "%s: packed or scales is NULL", who);
  const int64_t kc = (K + 31) / 32, G = (K + 255) / 256;
  std::vector<uint8_t> raw;
  try {
    raw.assign((size_t)N * (size_t)G * 144, 0);
  } catch (...) {
    return fail(ctx, RTD_ERR_OOM, "%s: host staging allocation failed", who);
  }
  static const uint8_t kHeader[16] = {0x00, 0x3C, 0x00, 0x48, 1, 1, 1, 1, 1, 1, 1, 1, 0x11, 0x11, 0x11, 0x11};
  for (int64_t n = 0; n < N; ++n)
    for (int64_t g = 0; g < G; ++g) {
      uint8_t* blk = raw.data() + (size_t)(n * G + g) * 144;
      std::memcpy(blk, kHeader, 16);
      for (int e = 0; e < 256; ++e) {
        const int64_t k = g * 256 + e;
        uint32_t q = 8;
        if (k < K) q = (packed[((k / 32) * N + n) * 4 + (k % 32) / 8] >> (4 * (k % 8))) & 0xFu;
        // Q4_K element e: chunk e / 64, byte (e % 32), low nibble for e % 64 < 32
        uint8_t& b = blk[16 + 32 * (e / 64) + (e % 32)];
        b |= (uint8_t)((e % 64) < 32 ? q : (q << 4));
      }
    }
  rtd_status st = rtd_qweight_upload(ctx, RTD_TYPE_Q4_K, raw.data(), raw.size(), N, G * 256, out);
  if (st != RTD_OK) return st;
  rtd_qweight* w = *out;
  w->ggml_type = RTD_TYPE_INT4_MARLIN;
  w->K = K;                                                       // x has K columns; groups past K decode to 0
  w->raw_bytes = (size_t)kc * (size_t)N * 16 + (size_t)N * 4;     // MarlinWeight::resident_bytes
  if (N > 0) {
    DeviceGuard g(ctx->device);
    cudaError_t e = cudaMalloc(&w->row_scale, (size_t)N * sizeof(float));
    if (e == cudaSuccess) e = cudaMemcpy(w->row_scale, scales, (size_t)N * sizeof(float), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
      cudaFree(w->row_scale);
      w->row_scale = nullptr;
      rtd_qweight_free(w);
      *out = nullptr;
      return fail(ctx, RTD_ERR_OOM, "%s: scales: %s", who, cudaGetErrorString(e));
    }
    w->owns_scale = true;
  }
  return RTD_OK;
}

rtd_status rtd_qweight_to_device(const rtd_qweight* src, rtd_ctx* ctx, rtd_qweight** out) {
  const char* who = "rtd_qweight_to_device";
  if (!src || !ctx || !out) return fail(ctx, RTD_ERR_INVALID, "%s: NULL argument", who);
  *out = nullptr;
  rtd_qweight* w = new (std::nothrow) rtd_qweight(*src);
  if (!w) return fail(ctx, RTD_ERR_OOM, "%s: host allocation failed", who);
  w->ctx = ctx;
  w->dev = nullptr;
  w->owns = true;
  w->row_scale = nullptr;
  w->owns_scale = false;
  if (src->row_scale) {
    DeviceGuard g(ctx->device);
    const size_t sb = (size_t)src->N * sizeof(float);
    cudaError_t e = cudaMalloc(&w->row_scale, sb);
    if (e == cudaSuccess)
      e = (src->ctx->device == ctx->device)
              ? cudaMemcpy(w->row_scale, src->row_scale, sb, cudaMemcpyDeviceToDevice)
              : cudaMemcpyPeer(w->row_scale, ctx->device, src->row_scale, src->ctx->device, sb);
    if (e != cudaSuccess) {
      cudaFree(w->row_scale);
      delete w;
      return cuda_fail(ctx, e, who);
    }
    w->owns_scale = true;
  }
  if (w->dev_bytes > 0) {
    DeviceGuard g(ctx->device);
    cudaError_t e = cudaMalloc(&w->dev, w->dev_bytes);
    if (e != cudaSuccess) {
      delete w;
      return fail(ctx, RTD_ERR_OOM, "%s: cudaMalloc(%zu): %s", who, src->dev_bytes, cudaGetErrorString(e));
    }
    e = (src->ctx->device == ctx->device)
            ? cudaMemcpy(w->dev, src->dev, w->dev_bytes, cudaMemcpyDeviceToDevice)
            : cudaMemcpyPeer(w->dev, ctx->device, src->dev, src->ctx->device, w->dev_bytes);
    if (e != cudaSuccess) {
      cudaFree(w->dev);
      delete w;
      return cuda_fail(ctx, e, who);
    }
  }
  *out = w;
  return RTD_OK;
}

rtd_status rtd_qweight_rows(const rtd_qweight* w, int64_t row0, int64_t rows, rtd_qweight** out) {
  const char* who = "rtd_qweight_rows";
  if (!w || !out) return fail(w ? w->ctx : nullptr, RTD_ERR_INVALID, "%s: NULL argument", who);
  *out = nullptr;
  if (row0 < 0 || rows <= 0 || row0 + rows > w->N || row0 % 16 != 0)
    return fail(w->ctx, RTD_ERR_SHAPE, "%s: rows [%lld, %lld) of %lld (the first row a multiple of 16)", who,
                (long long)row0, (long long)(row0 + rows), (long long)w->N);
  rtd_qweight* v = new (std::nothrow) rtd_qweight(*w);
  if (!v) return fail(w->ctx, RTD_ERR_OOM, "%s: host allocation failed", who);
  const rtd::FmtInfo f = rtd::fmt_info(w->fmt);
  v->N = rows;
  v->T = rtd::tiles_for(rows);
  v->dev = w->dev + (size_t)(row0 / 16) * (size_t)w->G * (size_t)f.gb;
  v->dev_bytes = (size_t)v->T * (size_t)w->G * (size_t)f.gb;
  v->raw_bytes = w->raw_bytes / (size_t)(w->N > 0 ? w->N : 1) * (size_t)rows;
  v->owns = false;
  if (w->row_scale) v->row_scale = w->row_scale + row0;
  v->owns_scale = false;
  *out = v;
  return RTD_OK;
}

rtd_status rtd_qweight_free(rtd_qweight* w) {
  if (!w) return RTD_OK;
  if ((w->dev && w->owns) || (w->row_scale && w->owns_scale)) {
    DeviceGuard g(w->ctx->device);
    if (w->dev && w->owns) cudaFree(w->dev);
    if (w->row_scale && w->owns_scale) cudaFree(w->row_scale);
  }
  delete w;
  return RTD_OK;
}

rtd_status rtd_qweight_info(const rtd_qweight* w, uint32_t* ggml_type, int64_t* N, int64_t* K, size_t* raw_bytes,
                            size_t* device_bytes) {
  if (!w) return fail(nullptr, RTD_ERR_INVALID, "rtd_qweight_info: NULL handle");
  if (ggml_type) *ggml_type = w->ggml_type;
  if (N) *N = w->N;
  if (K) *K = w->K;
  if (raw_bytes) *raw_bytes = w->raw_bytes;
  if (device_bytes) *device_bytes = w->dev_bytes;
  return RTD_OK;
}

static rtd_status run_gemv(rtd_ctx* ctx, int fmt, const uint8_t* wdev, int64_t N, int64_t K, int64_t G,
                           const float* row_scale, int scale_len, const void* x, uint32_t x_dtype, int64_t ldx,
                           int64_t M, int w8a8, const float* bias, void* y, uint32_t y_dtype, int64_t ldy,
                           void* stream, const char* who, float wpow2, int32_t* ids = nullptr,
                           uint64_t* keys = nullptr, int64_t row0 = 0) {
  if (M < 0) return fail(ctx, RTD_ERR_SHAPE, "%s: M=%lld is negative", who, (long long)M);
  if (!valid_dtype(x_dtype) || !valid_dtype(y_dtype)) return fail(ctx, RTD_ERR_INVALID, "%s: bad dtype", who);
  if (M == 0 || N == 0) return RTD_OK;
  if ((K > 0 && !x) || (!y && !ids && !keys)) return fail(ctx, RTD_ERR_INVALID, "%s: x or y is NULL", who);
  if (ldx < K || (y && ldy < N))
    return fail(ctx, RTD_ERR_SHAPE, "%s: row strides ldx=%lld ldy=%lld below K=%lld N=%lld", who, (long long)ldx,
                (long long)ldy, (long long)K, (long long)N);
  DeviceGuard g(ctx->device);
  if (g.err != cudaSuccess) return cuda_fail(ctx, g.err, who);
  cudaError_t e;
  if (K == 0) {
    e = rtd::launch_fill_rows(bias, y, y_dtype, ldy, M, N, (cudaStream_t)stream);
    return e == cudaSuccess ? RTD_OK : cuda_fail(ctx, e, who);
  }
  rtd::QGemvCall c{};
  c.fmt = fmt;
  c.w = wdev;
  c.N = N;
  c.K = K;
  c.G = G;
  c.row_scale = row_scale;
  c.scale_len = scale_len;
  c.x = x;
  c.x_dtype = (int)x_dtype;
  c.ldx = ldx;
  c.M = M;
  c.w8a8 = w8a8;
  c.wpow2 = wpow2;
  c.bias = bias;
  c.y = y;
  c.y_dtype = (int)y_dtype;
  c.ldy = ldy;
  c.ws = ctx->ws;
  c.ws_bytes = ctx->ws_bytes;
  c.status = ctx->status;
  c.sm_count = ctx->sm_count;
  c.stream = (cudaStream_t)stream;
  c.ids = ids;
  c.amax_out = reinterpret_cast<unsigned long long*>(keys);
  c.amax_row0 = row0;
  c.amax = (ids || keys) ? ctx->amax : nullptr;
  int plan_err = 0;
  // four or more tokens go to the tensor-core GEMM when its staged activations fit
  // the workspace (the argmax epilogue is the GEMV's, in launches of up to four tokens)
  if (!ids && !keys && M >= kGemmMinTokens && rtd::qgemm_workspace_bytes(c) <= c.ws_bytes)
    e = rtd::launch_qgemm(c, &plan_err);
  else
    e = rtd::launch_qgemv(c, &plan_err);
  if (plan_err) return fail(ctx, RTD_ERR_WORKSPACE, "%s: [%lld x %lld] does not fit the context workspace", who, (long long)N, (long long)K);
  if (e != cudaSuccess) return cuda_fail(ctx, e, who);
  return RTD_OK;
}

rtd_status rtd_qlinear(rtd_ctx* ctx, const rtd_qweight* w, const void* x, uint32_t x_dtype, int64_t ldx, int64_t M,
                       const float* bias, void* y, uint32_t y_dtype, int64_t ldy, void* stream) {
  if (!ctx || !w) return fail(ctx, RTD_ERR_INVALID, "rtd_qlinear: NULL ctx or weight");
  return run_gemv(ctx, w->fmt, w->dev, w->N, w->K, w->G, w->row_scale, w->row_scale ? (int)w->N : 0, x, x_dtype, ldx,
                  M, 0, bias, y, y_dtype, ldy, stream, "rtd_qlinear", w->wpow2);
}

rtd_status rtd_qlinear_argmax(rtd_ctx* ctx, const rtd_qweight* w, const void* x, uint32_t x_dtype, int64_t ldx,
                              int64_t M, const float* bias, void* y, uint32_t y_dtype, int64_t ldy, int32_t* ids,
                              void* stream) {
  const char* who = "rtd_qlinear_argmax";
  if (!ctx || !w) return fail(ctx, RTD_ERR_INVALID, "%s: NULL ctx or weight", who);
  if (M < 0) return fail(ctx, RTD_ERR_SHAPE, "%s: M=%lld is negative", who, (long long)M);
  if (M == 0) return RTD_OK;
  if (!ids) return fail(ctx, RTD_ERR_INVALID, "%s: ids is NULL", who);
  if (w->N <= 0 || w->N > INT32_MAX || w->K <= 0)
    return fail(ctx, RTD_ERR_SHAPE, "%s: [%lld x %lld] (1 .. 2^31 - 1 rows, K > 0)", who, (long long)w->N,
                (long long)w->K);
  const int scale_len = w->row_scale ? (int)w->N : 0;
  if (M < kGemmMinTokens)  // decode: the argmax runs in the GEMV's epilogue, y is optional
    return run_gemv(ctx, w->fmt, w->dev, w->N, w->K, w->G, w->row_scale, scale_len, x, x_dtype, ldx, M, 0, bias, y,
                    y_dtype, ldy, stream, who, w->wpow2, ids);
  // prompt-sized calls: the logits, then the argmax kernel over them
  if (!y || y_dtype != RTD_DT_F32)
    return fail(ctx, RTD_ERR_INVALID, "%s: %lld tokens need f32 logits in y", who, (long long)M);
  rtd_status s = run_gemv(ctx, w->fmt, w->dev, w->N, w->K, w->G, w->row_scale, scale_len, x, x_dtype, ldx, M, 0, bias,
                          y, y_dtype, ldy, stream, who, w->wpow2);
  if (s != RTD_OK) return s;
  DeviceGuard g(ctx->device);
  cudaError_t e = rtd::launch_argmax(static_cast<const float*>(y), ldy, M, w->N, ids, (cudaStream_t)stream);
  return e == cudaSuccess ? RTD_OK : cuda_fail(ctx, e, who);
}

rtd_status rtd_qlinear_argmax_keys(rtd_ctx* ctx, const rtd_qweight* w, const void* x, uint32_t x_dtype,
                                   int64_t ldx, int64_t M, const float* bias, int64_t row0, uint64_t* keys,
                                   void* stream) {
  const char* who = "rtd_qlinear_argmax_keys";
  if (!ctx || !w) return fail(ctx, RTD_ERR_INVALID, "%s: NULL ctx or weight", who);
  if (M < 0) return fail(ctx, RTD_ERR_SHAPE, "%s: M=%lld is negative", who, (long long)M);
  if (M == 0) return RTD_OK;
  if (!keys) return fail(ctx, RTD_ERR_INVALID, "%s: keys is NULL", who);
  if (w->N <= 0 || w->K <= 0 || row0 < 0 || row0 + w->N > (int64_t)UINT32_MAX)
    return fail(ctx, RTD_ERR_SHAPE, "%s: rows [%lld, %lld) (below 2^32, K > 0)", who, (long long)row0,
                (long long)(row0 + w->N));
  return run_gemv(ctx, w->fmt, w->dev, w->N, w->K, w->G, w->row_scale, w->row_scale ? (int)w->N : 0, x, x_dtype, ldx,
                  M, 0, bias, nullptr, RTD_DT_F32, w->N, stream, who, w->wpow2, nullptr, keys, row0);
}

rtd_status rtd_qembed(rtd_ctx* ctx, const rtd_qweight* w, const uint32_t* ids, int64_t n, float* y, void* stream) {
  if (!ctx || !w) return fail(ctx, RTD_ERR_INVALID, "rtd_qembed: NULL ctx or weight");
  if (n < 0) return fail(ctx, RTD_ERR_SHAPE, "rtd_qembed: n=%lld is negative", (long long)n);
  if (w->row_scale) return fail(ctx, RTD_ERR_UNSUPPORTED, "rtd_qembed: INT4 Marlin weights are not an embedding format");
  if (n == 0 || w->K == 0) return RTD_OK;
  if (!ids || !y) return fail(ctx, RTD_ERR_INVALID, "rtd_qembed: ids or y is NULL");
  DeviceGuard g(ctx->device);
  cudaError_t e = rtd::launch_embed(w->fmt, w->dev, w->N, w->K, w->G, ids, n, y, ctx->status, (cudaStream_t)stream);
  return e == cudaSuccess ? RTD_OK : cuda_fail(ctx, e, "rtd_qembed");
}

rtd_status rtd_qdequant(rtd_ctx* ctx, const rtd_qweight* w, float* y, void* stream) {
  if (!ctx || !w) return fail(ctx, RTD_ERR_INVALID, "rtd_qdequant: NULL ctx or weight");
  if (w->N == 0 || w->K == 0) return RTD_OK;
  if (!y) return fail(ctx, RTD_ERR_INVALID, "rtd_qdequant: y is NULL");
  DeviceGuard g(ctx->device);
  cudaError_t e = rtd::launch_dequant(w->fmt, w->dev, w->N, w->K, w->G, w->row_scale, y, (cudaStream_t)stream);
  return e == cudaSuccess ? RTD_OK : cuda_fail(ctx, e, "rtd_qdequant");
}

rtd_status rtd_fp8weight_upload(rtd_ctx* ctx, const uint8_t* host_w, const float* host_scale, int64_t scale_len,
                                int64_t N, int64_t K, rtd_fp8weight** out) {
  if (!ctx || !out) return fail(ctx, RTD_ERR_INVALID, "rtd_fp8weight_upload: NULL argument");
  *out = nullptr;
  if (N < 0 || K < 0) return fail(ctx, RTD_ERR_SHAPE, "rtd_fp8weight_upload: negative shape");
  if (!(scale_len == 1 || scale_len == N))
    return fail(ctx, RTD_ERR_SHAPE, "rtd_fp8weight_upload: scale has %lld elements, expected 1 or N=%lld",
                (long long)scale_len, (long long)N);
  if ((N * K > 0 && !host_w) || !host_scale) return fail(ctx, RTD_ERR_INVALID, "rtd_fp8weight_upload: NULL data");
  rtd_fp8weight* w = new (std::nothrow) rtd_fp8weight();
  if (!w) return fail(ctx, RTD_ERR_OOM, "rtd_fp8weight_upload: host allocation failed");
  w->ctx = ctx;
  w->N = N;
  w->K = K;
  w->T = rtd::tiles_for(N);
  w->G = rtd::groups_for(rtd::FMT_FP8, K);
  w->scale_len = scale_len;
  w->dev_bytes = (size_t)(w->T * w->G) * (size_t)rtd::fmt_info(rtd::FMT_FP8).gb;
  DeviceGuard g(ctx->device);
  cudaError_t e = cudaMalloc(&w->scale, (size_t)scale_len * sizeof(float));
  if (e == cudaSuccess) e = cudaMemcpy(w->scale, host_scale, (size_t)scale_len * sizeof(float), cudaMemcpyHostToDevice);
  if (e == cudaSuccess && w->dev_bytes > 0) {
    std::vector<uint8_t> host(w->dev_bytes);
    rtd::repack_host(rtd::FMT_FP8, host_w, N, K, host.data());
    e = cudaMalloc(&w->dev, w->dev_bytes);
    if (e == cudaSuccess) e = cudaMemcpy(w->dev, host.data(), w->dev_bytes, cudaMemcpyHostToDevice);
  }
  if (e != cudaSuccess) {
    cudaFree(w->dev);
    cudaFree(w->scale);
    delete w;
    return fail(ctx, RTD_ERR_OOM, "rtd_fp8weight_upload: %s", cudaGetErrorString(e));
  }
  *out = w;
  return RTD_OK;
}

rtd_status rtd_fp8weight_free(rtd_fp8weight* w) {
  if (!w) return RTD_OK;
  DeviceGuard g(w->ctx->device);
  cudaFree(w->dev);
  cudaFree(w->scale);
  delete w;
  return RTD_OK;
}

rtd_status rtd_fp8_linear(rtd_ctx* ctx, const rtd_fp8weight* w, const void* x, uint32_t x_dtype, int64_t ldx,
                          int64_t M, void* y, uint32_t y_dtype, int64_t ldy, uint32_t mode, void* stream) {
  if (!ctx || !w) return fail(ctx, RTD_ERR_INVALID, "rtd_fp8_linear: NULL ctx or weight");
  if (mode != RTD_FP8_W8A16 && mode != RTD_FP8_W8A8) return fail(ctx, RTD_ERR_INVALID, "rtd_fp8_linear: bad mode %u", mode);
  return run_gemv(ctx, rtd::FMT_FP8, w->dev, w->N, w->K, w->G, w->scale, (int)w->scale_len, x, x_dtype, ldx, M,
                  mode == RTD_FP8_W8A8 ? 1 : 0, nullptr, y, y_dtype, ldy, stream, "rtd_fp8_linear", 1.0f);
}

rtd_status rtd_fp8_encode(rtd_ctx* ctx, const float* x, int64_t n, uint8_t* out, void* stream) {
  if (!ctx) return fail(nullptr, RTD_ERR_INVALID, "rtd_fp8_encode: ctx is NULL");
  if (n < 0) return fail(ctx, RTD_ERR_SHAPE, "rtd_fp8_encode: n is negative");
  if (n == 0) return RTD_OK;
  if (!x || !out) return fail(ctx, RTD_ERR_INVALID, "rtd_fp8_encode: NULL pointer");
  DeviceGuard g(ctx->device);
  cudaError_t e = rtd::launch_fp8_encode(x, n, out, (cudaStream_t)stream);
  return e == cudaSuccess ? RTD_OK : cuda_fail(ctx, e, "rtd_fp8_encode");
}

}  // extern "C"


// ---- decoder-layer operations ------------------------------------------------
// The SubstratePort operations between the linears of a decoder layer
// (crates/runtimed-model/src/substrate/port.rs:14-90), over a paged f16 KV cache.
rtd_status rtd_rmsnorm(rtd_ctx* ctx, float* h, int64_t ldh, const void* delta, uint32_t delta_dtype, int64_t ldd,
                       const float* w, float eps, int64_t T, int64_t H, void* y, uint32_t y_dtype, int64_t ldy,
                       void* stream) {
  const char* who = "rtd_rmsnorm";
  if (!ctx) return fail(nullptr, RTD_ERR_INVALID, "%s: ctx is NULL", who);
  if (T < 0 || H < 0) return fail(ctx, RTD_ERR_SHAPE, "%s: negative shape", who);
  if (T == 0 || H == 0) return RTD_OK;
  if (!h || !w || !y) return fail(ctx, RTD_ERR_INVALID, "%s: NULL pointer", who);
  if (!valid_dtype(y_dtype) || (delta && !valid_dtype(delta_dtype))) return fail(ctx, RTD_ERR_INVALID, "%s: bad dtype", who);
  if (ldh < H || ldy < H || (delta && ldd < H)) return fail(ctx, RTD_ERR_SHAPE, "%s: row strides below H", who);
  DeviceGuard g(ctx->device);
  cudaError_t e = rtd::launch_add_rmsnorm(h, ldh, delta, (int)delta_dtype, ldd, w, eps, T, H, y, (int)y_dtype, ldy,
                                          (cudaStream_t)stream);
  return e == cudaSuccess ? RTD_OK : cuda_fail(ctx, e, who);
}

namespace {
rtd_status check_heads(rtd_ctx* ctx, int32_t n_head, int32_t n_kv, int32_t head_dim, const char* who) {
  if (n_head <= 0 || n_kv <= 0 || n_head % n_kv != 0)
    return fail(ctx, RTD_ERR_SHAPE, "%s: %d query heads are not a multiple of %d kv heads", who, n_head, n_kv);
  if (n_head / n_kv > 8) return fail(ctx, RTD_ERR_SHAPE, "%s: more than 8 query heads per kv head", who);
  if (head_dim <= 0 || head_dim % 8 != 0 || head_dim > 128)
    return fail(ctx, RTD_ERR_SHAPE, "%s: head_dim %d (a multiple of 8, at most 128)", who, head_dim);
  return RTD_OK;
}
}  // namespace

rtd_status rtd_rope_kv_append(rtd_ctx* ctx, const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v,
                              int64_t ldv, int64_t T, int32_t n_head, int32_t n_kv, int32_t head_dim, int32_t rot_dim,
                              float theta, const int32_t* tok_seq, const int32_t* tok_pos, const int32_t* block_table,
                              int32_t max_blocks, void* k_cache, void* v_cache, uint32_t kv_dtype, float* q_out,
                              void* stream) {
  const char* who = "rtd_rope_kv_append";
  if (!ctx) return fail(nullptr, RTD_ERR_INVALID, "%s: ctx is NULL", who);
  rtd_status st = check_heads(ctx, n_head, n_kv, head_dim, who);
  if (st != RTD_OK) return st;
  if (rot_dim < 0 || rot_dim > head_dim || rot_dim % 2 != 0)
    return fail(ctx, RTD_ERR_SHAPE, "%s: rot_dim %d for head_dim %d", who, rot_dim, head_dim);
  if (T < 0) return fail(ctx, RTD_ERR_SHAPE, "%s: T is negative", who);
  if (T == 0) return RTD_OK;
  if (!q || !k || !v || !tok_seq || !tok_pos || !block_table || !k_cache || !v_cache || !q_out || max_blocks <= 0)
    return fail(ctx, RTD_ERR_INVALID, "%s: NULL pointer or no block table", who);
  if (ldq < (int64_t)n_head * head_dim || ldk < (int64_t)n_kv * head_dim || ldv < (int64_t)n_kv * head_dim)
    return fail(ctx, RTD_ERR_SHAPE, "%s: row strides below the head widths", who);
  if (kv_dtype != RTD_DT_F16 && kv_dtype != RTD_DT_F32) return fail(ctx, RTD_ERR_INVALID, "%s: cache dtype", who);
  DeviceGuard g(ctx->device);
  cudaError_t e = rtd::launch_rope_kv(q, ldq, k, ldk, v, ldv, T, n_head, n_kv, head_dim, rot_dim, theta, tok_seq,
                                      tok_pos, block_table, max_blocks, k_cache, v_cache, kv_dtype == RTD_DT_F32 ? 1 : 0,
                                      q_out, (cudaStream_t)stream);
  return e == cudaSuccess ? RTD_OK : cuda_fail(ctx, e, who);
}

rtd_status rtd_attention_paged(rtd_ctx* ctx, const float* q, int64_t T, int32_t n_head, int32_t n_kv, int32_t head_dim,
                               float scale, const int32_t* tok_seq, const int32_t* tok_pos, const int32_t* block_table,
                               int32_t max_blocks, int32_t max_ctx, const void* k_cache, const void* v_cache,
                               uint32_t kv_dtype, void* o, uint32_t o_dtype, int64_t ldo, void* stream) {
  const char* who = "rtd_attention_paged";
  if (!ctx) return fail(nullptr, RTD_ERR_INVALID, "%s: ctx is NULL", who);
  rtd_status st = check_heads(ctx, n_head, n_kv, head_dim, who);
  if (st != RTD_OK) return st;
  if (T < 0) return fail(ctx, RTD_ERR_SHAPE, "%s: T is negative", who);
  if (T == 0) return RTD_OK;
  if (!q || !tok_seq || !tok_pos || !block_table || !k_cache || !v_cache || !o || max_blocks <= 0)
    return fail(ctx, RTD_ERR_INVALID, "%s: NULL pointer or no block table", who);
  if (!valid_dtype(o_dtype)) return fail(ctx, RTD_ERR_INVALID, "%s: bad dtype", who);
  if (kv_dtype != RTD_DT_F16 && kv_dtype != RTD_DT_F32) return fail(ctx, RTD_ERR_INVALID, "%s: cache dtype", who);
  if (ldo < (int64_t)n_head * head_dim) return fail(ctx, RTD_ERR_SHAPE, "%s: ldo below n_head * head_dim", who);
  if (max_ctx <= 0 || max_ctx > max_blocks * 16)
    return fail(ctx, RTD_ERR_SHAPE, "%s: max_ctx %d outside the block table (%d blocks)", who, max_ctx, max_blocks);
  // split long contexts across CTAs when the (token, kv head) blocks leave SMs idle
  int splits = 1;
  const int64_t blocks = T * n_kv;
  if (blocks < ctx->sm_count && max_ctx > 256) {
    splits = (int)std::min<int64_t>({(int64_t)(max_ctx + 255) / 256, (ctx->sm_count + blocks - 1) / blocks, 32});
    while (splits > 1 && rtd::attn_workspace_bytes(T, n_head, n_kv, head_dim, splits) > ctx->ws_bytes) --splits;
  }
  DeviceGuard g(ctx->device);
  cudaError_t e = rtd::launch_attention(q, T, n_head, n_kv, head_dim, scale, tok_seq, tok_pos, block_table, max_blocks,
                                        k_cache, v_cache, kv_dtype == RTD_DT_F32 ? 1 : 0, o, (int)o_dtype, ldo, splits,
                                        ctx->ws, (cudaStream_t)stream);
  return e == cudaSuccess ? RTD_OK : cuda_fail(ctx, e, who);
}

rtd_status rtd_silu_mul(rtd_ctx* ctx, const void* gate, uint32_t gate_dtype, int64_t ldg, const void* up,
                        uint32_t up_dtype, int64_t ldu, int64_t T, int64_t F, void* y, uint32_t y_dtype, int64_t ldy,
                        void* stream) {
  const char* who = "rtd_silu_mul";
  if (!ctx) return fail(nullptr, RTD_ERR_INVALID, "%s: ctx is NULL", who);
  if (T < 0 || F < 0) return fail(ctx, RTD_ERR_SHAPE, "%s: negative shape", who);
  if (T == 0 || F == 0) return RTD_OK;
  if (!gate || !up || !y) return fail(ctx, RTD_ERR_INVALID, "%s: NULL pointer", who);
  if (!valid_dtype(gate_dtype) || !valid_dtype(up_dtype) || !valid_dtype(y_dtype))
    return fail(ctx, RTD_ERR_INVALID, "%s: bad dtype", who);
  if (ldg < F || ldu < F || ldy < F) return fail(ctx, RTD_ERR_SHAPE, "%s: row strides below F", who);
  DeviceGuard g(ctx->device);
  cudaError_t e = rtd::launch_silu_mul(gate, (int)gate_dtype, ldg, up, (int)up_dtype, ldu, T, F, y, (int)y_dtype, ldy,
                                       (cudaStream_t)stream);
  return e == cudaSuccess ? RTD_OK : cuda_fail(ctx, e, who);
}

rtd_status rtd_argmax(rtd_ctx* ctx, const float* x, int64_t ldx, int64_t T, int64_t V, int32_t* out, void* stream) {
  const char* who = "rtd_argmax";
  if (!ctx) return fail(nullptr, RTD_ERR_INVALID, "%s: ctx is NULL", who);
  if (T < 0 || V <= 0 || V > INT32_MAX) return fail(ctx, RTD_ERR_SHAPE, "%s: T=%lld V=%lld", who, (long long)T, (long long)V);
  if (T == 0) return RTD_OK;
  if (!x || !out) return fail(ctx, RTD_ERR_INVALID, "%s: NULL pointer", who);
  if (ldx < V) return fail(ctx, RTD_ERR_SHAPE, "%s: ldx below V", who);
  DeviceGuard g(ctx->device);
  cudaError_t e = rtd::launch_argmax(x, ldx, T, V, out, (cudaStream_t)stream);
  return e == cudaSuccess ? RTD_OK : cuda_fail(ctx, e, who);
}

// ---- tensor-parallel row reduction ------------------------------------------
// One communicator per rank (one process per GPU).  Its device buffer holds the three
// LL exchange regions of rtd_kernels.h (TpReduce) -- each in two parity halves -- and
// two control words; peers map it through CUDA IPC and store into it over NVLink.
//   ll : [2][world][4 * max_n]              the GEMV's one-shot tile exchange
//   rs : [2][world][rs_per_src]             the all-reduce's reduce-scatter slots
//   ag : [2][ag_elems]                      the all-reduce's all-gather slots
// The control words (epoch, finished CTAs) carry the exchange epoch from one launch to
// the next on the device, so calls can be captured in a CUDA graph.
namespace {
constexpr int64_t kArTokens = 128;       // tokens one all-reduce launch exchanges
constexpr int64_t kArBlockSlack = 4096;  // room for the per-CTA block rounding
}  // namespace

struct rtd_comm {
  rtd_ctx* ctx = nullptr;
  int world = 1, rank = 0;
  int64_t max_n = 0;
  unsigned char* base = nullptr;  // this rank's buffer (cudaMalloc, exported by IPC)
  size_t ll_off = 0, rs_off = 0, ag_off = 0, ctrl_off = 0, bytes = 0;
  unsigned char* peer[rtd::kMaxTpWorld] = {};  // mapped peer buffers (peer[rank] = base)
  bool opened = false;
  rtd::TpReduce tp{};
};

rtd_status rtd_tp_comm_create(rtd_ctx* ctx, int rank, int world, int64_t max_n, rtd_comm** out, void* handle_out) {
  const char* who = "rtd_tp_comm_create";
  if (!ctx || !out || !handle_out) return fail(ctx, RTD_ERR_INVALID, "%s: NULL argument", who);
  if (world < 1 || world > rtd::kMaxTpWorld || rank < 0 || rank >= world)
    return fail(ctx, RTD_ERR_INVALID, "%s: rank %d of world %d (1..%d ranks)", who, rank, world, rtd::kMaxTpWorld);
  if (max_n <= 0) return fail(ctx, RTD_ERR_SHAPE, "%s: max_n=%lld", who, (long long)max_n);
  DeviceGuard g(ctx->device);
  if (g.err != cudaSuccess) return cuda_fail(ctx, g.err, who);
  rtd_comm* c = new (std::nothrow) rtd_comm();
  if (!c) return fail(ctx, RTD_ERR_OOM, "%s: host allocation failed", who);
  c->ctx = ctx;
  c->world = world;
  c->rank = rank;
  c->max_n = max_n;
  const int64_t ar_max = kArTokens * max_n;
  int64_t ag_elems = ar_max + kArBlockSlack * 2 * world;
  ag_elems = (ag_elems + 1) / 2 * 2;
  int64_t rs_per_src = (ag_elems + world - 1) / world;
  rs_per_src = (rs_per_src + 1) / 2 * 2;
  auto up = [](size_t v) { return (v + 255) / 256 * 256; };
  c->ll_off = 0;
  c->rs_off = up((size_t)2 * world * 4 * (size_t)max_n * sizeof(uint64_t));
  c->ag_off = c->rs_off + up((size_t)2 * world * (size_t)rs_per_src * sizeof(uint64_t));
  c->ctrl_off = c->ag_off + up((size_t)2 * (size_t)ag_elems * sizeof(uint64_t));
  c->bytes = c->ctrl_off + 256;
  cudaError_t e = cudaMalloc(&c->base, c->bytes);
  if (e != cudaSuccess) {
    delete c;
    return fail(ctx, RTD_ERR_OOM, "%s: cudaMalloc(%zu): %s", who, c->bytes, cudaGetErrorString(e));
  }
  if ((e = cudaMemset(c->base, 0, c->bytes)) != cudaSuccess ||
      (e = cudaDeviceSynchronize()) != cudaSuccess ||
      (e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle_out), c->base)) != cudaSuccess) {
    cudaFree(c->base);
    delete c;
    return cuda_fail(ctx, e, who);
  }
  c->peer[rank] = c->base;
  c->tp.world = world;
  c->tp.rank = rank;
  c->tp.max_n = max_n;
  c->tp.rs_per_src = rs_per_src;
  c->tp.ag_elems = ag_elems;
  c->tp.ar_max_elems = ar_max;
  c->tp.ctrl = reinterpret_cast<uint32_t*>(c->base + c->ctrl_off);
  c->tp.ll[rank] = reinterpret_cast<uint64_t*>(c->base + c->ll_off);
  c->tp.rs[rank] = reinterpret_cast<uint64_t*>(c->base + c->rs_off);
  c->tp.ag[rank] = reinterpret_cast<uint64_t*>(c->base + c->ag_off);
  *out = c;
  return RTD_OK;
}

rtd_status rtd_tp_comm_open(rtd_comm* c, const void* handles) {
  const char* who = "rtd_tp_comm_open";
  if (!c || !handles) return fail(nullptr, RTD_ERR_INVALID, "%s: NULL argument", who);
  if (c->opened) return RTD_OK;
  DeviceGuard g(c->ctx->device);
  if (g.err != cudaSuccess) return cuda_fail(c->ctx, g.err, who);
  const cudaIpcMemHandle_t* h = static_cast<const cudaIpcMemHandle_t*>(handles);
  for (int p = 0; p < c->world; ++p) {
    if (p == c->rank) continue;
    void* ptr = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&ptr, h[p], cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < p; ++q)
        if (q != c->rank && c->peer[q]) cudaIpcCloseMemHandle(c->peer[q]);
      return fail(c->ctx, RTD_ERR_CUDA, "%s: mapping rank %d: %s", who, p, cudaGetErrorString(e));
    }
    c->peer[p] = static_cast<unsigned char*>(ptr);
  }
  for (int p = 0; p < c->world; ++p) {
    c->tp.ll[p] = reinterpret_cast<uint64_t*>(c->peer[p] + c->ll_off);
    c->tp.rs[p] = reinterpret_cast<uint64_t*>(c->peer[p] + c->rs_off);
    c->tp.ag[p] = reinterpret_cast<uint64_t*>(c->peer[p] + c->ag_off);
  }
  c->opened = true;
  return RTD_OK;
}

rtd_status rtd_tp_comm_destroy(rtd_comm* c) {
  if (!c) return RTD_OK;
  DeviceGuard g(c->ctx->device);
  for (int p = 0; p < c->world; ++p)
    if (p != c->rank && c->peer[p]) cudaIpcCloseMemHandle(c->peer[p]);
  cudaFree(c->base);
  delete c;
  return RTD_OK;
}

namespace {
rtd_status tp_check_common(rtd_comm* comm, int64_t M, uint32_t y_dtype, const void* y, const char* who) {
  rtd_ctx* ctx = comm->ctx;
  if (comm->world > 1 && !comm->opened) return fail(ctx, RTD_ERR_INVALID, "%s: communicator not opened", who);
  if (M < 0) return fail(ctx, RTD_ERR_SHAPE, "%s: M=%lld is negative", who, (long long)M);
  if (!valid_dtype(y_dtype)) return fail(ctx, RTD_ERR_INVALID, "%s: bad dtype", who);
  if (M > 0 && !y) return fail(ctx, RTD_ERR_INVALID, "%s: y is NULL", who);
  return RTD_OK;
}
}  // namespace

rtd_status rtd_tp_qlinear_row(rtd_comm* comm, const rtd_qweight* shard, const void* x, uint32_t x_dtype, int64_t ldx,
                              int64_t M, const float* bias, void* y, uint32_t y_dtype, int64_t ldy, void* stream) {
  const char* who = "rtd_tp_qlinear_row";
  if (!comm || !shard) return fail(nullptr, RTD_ERR_INVALID, "%s: NULL comm or weight", who);
  rtd_ctx* ctx = comm->ctx;
  rtd_status st = tp_check_common(comm, M, y_dtype, y, who);
  if (st != RTD_OK) return st;
  if (shard->ctx != ctx) return fail(ctx, RTD_ERR_INVALID, "%s: weight and communicator on different contexts", who);
  if (shard->row_scale) return fail(ctx, RTD_ERR_UNSUPPORTED, "%s: INT4 Marlin weights are not sharded", who);
  if (shard->N > comm->max_n)
    return fail(ctx, RTD_ERR_SHAPE, "%s: N=%lld above the communicator's max_n=%lld", who, (long long)shard->N,
                (long long)comm->max_n);
  if (!valid_dtype(x_dtype)) return fail(ctx, RTD_ERR_INVALID, "%s: bad dtype", who);
  if (M == 0 || shard->N == 0) return RTD_OK;
  if (shard->K > 0 && !x) return fail(ctx, RTD_ERR_INVALID, "%s: x is NULL", who);
  if (shard->K == 0) return fail(ctx, RTD_ERR_SHAPE, "%s: empty K shard", who);
  if (ldx < shard->K || ldy < shard->N)
    return fail(ctx, RTD_ERR_SHAPE, "%s: row strides ldx=%lld ldy=%lld below K=%lld N=%lld", who, (long long)ldx,
                (long long)ldy, (long long)shard->K, (long long)shard->N);
  DeviceGuard g(ctx->device);
  if (g.err != cudaSuccess) return cuda_fail(ctx, g.err, who);
  rtd::QGemvCall c{};
  c.fmt = shard->fmt;
  c.w = shard->dev;
  c.wpow2 = shard->wpow2;
  c.N = shard->N;
  c.K = shard->K;
  c.G = shard->G;
  c.x = x;
  c.x_dtype = (int)x_dtype;
  c.ldx = ldx;
  c.M = M;
  c.bias = bias;
  c.y = y;
  c.y_dtype = (int)y_dtype;
  c.ldy = ldy;
  c.ws = ctx->ws;
  c.ws_bytes = ctx->ws_bytes;
  c.status = ctx->status;
  c.sm_count = ctx->sm_count;
  c.stream = (cudaStream_t)stream;
  const bool tp = comm->world > 1;
  c.tp = tp ? &comm->tp : nullptr;
  int plan_err = 0;
  cudaError_t e = cudaSuccess;
  if (M < kGemmMinTokens || !tp) {
    // decode: the GEMV with the exchange fused into its epilogue (world 1: a plain GEMV;
    // four or more tokens on one rank go through the single-GPU dispatch)
    if (!tp && M >= kGemmMinTokens && rtd::qgemm_workspace_bytes(c) <= c.ws_bytes)
      e = rtd::launch_qgemm(c, &plan_err);
    else
      e = rtd::launch_qgemv(c, &plan_err);
  } else {
    // four or more tokens: the tensor-core GEMM writes this rank's f32 partial into the
    // top of the workspace, then the two-shot all-reduce, in chunks of kArTokens tokens
    const size_t esz = x_dtype == RTD_DT_F32 ? 4 : 2, ysz = y_dtype == RTD_DT_F32 ? 4 : 2;
    for (int64_t m0 = 0; m0 < M && e == cudaSuccess && !plan_err; m0 += kArTokens) {
      const int64_t mc = std::min<int64_t>(kArTokens, M - m0);
      const size_t part_b = ((size_t)mc * (size_t)shard->N * 4 + 255) / 256 * 256;
      if (part_b >= ctx->ws_bytes) {
        plan_err = 1;
        break;
      }
      float* part = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(ctx->ws) + (ctx->ws_bytes - part_b));
      rtd::QGemvCall gc = c;
      gc.x = static_cast<const unsigned char*>(x) + (size_t)m0 * (size_t)ldx * esz;
      gc.M = mc;
      gc.bias = nullptr;
      gc.y = part;
      gc.y_dtype = RTD_DT_F32;
      gc.ldy = shard->N;
      gc.ws_bytes = ctx->ws_bytes - part_b;
      gc.tp = nullptr;
      if (rtd::qgemm_workspace_bytes(gc) <= gc.ws_bytes)
        e = rtd::launch_qgemm(gc, &plan_err);
      else
        e = rtd::launch_qgemv(gc, &plan_err);
      if (e != cudaSuccess || plan_err) break;
      e = rtd::launch_tp_allreduce(comm->tp, part, shard->N, mc, shard->N, bias,
                                   static_cast<unsigned char*>(y) + (size_t)m0 * (size_t)ldy * ysz, (int)y_dtype, ldy,
                                   ctx->status, ctx->sm_count, (cudaStream_t)stream);
    }
  }
  if (plan_err) return fail(ctx, RTD_ERR_WORKSPACE, "%s: [%lld x %lld] does not fit the workspace", who,
                            (long long)shard->N, (long long)shard->K);
  if (e != cudaSuccess) return cuda_fail(ctx, e, who);
  return RTD_OK;
}

rtd_status rtd_tp_allreduce(rtd_comm* comm, const float* partial, int64_t ldp, int64_t M, int64_t N,
                            const float* bias, void* y, uint32_t y_dtype, int64_t ldy, void* stream) {
  const char* who = "rtd_tp_allreduce";
  if (!comm) return fail(nullptr, RTD_ERR_INVALID, "%s: NULL comm", who);
  rtd_ctx* ctx = comm->ctx;
  rtd_status st = tp_check_common(comm, M, y_dtype, y, who);
  if (st != RTD_OK) return st;
  if (N < 0) return fail(ctx, RTD_ERR_SHAPE, "%s: N=%lld is negative", who, (long long)N);
  if (N > comm->max_n)
    return fail(ctx, RTD_ERR_SHAPE, "%s: N=%lld above the communicator's max_n=%lld", who, (long long)N,
                (long long)comm->max_n);
  if (M == 0 || N == 0) return RTD_OK;
  if (!partial) return fail(ctx, RTD_ERR_INVALID, "%s: partial is NULL", who);
  if (ldp < N || ldy < N)
    return fail(ctx, RTD_ERR_SHAPE, "%s: row strides ldp=%lld ldy=%lld below N=%lld", who, (long long)ldp,
                (long long)ldy, (long long)N);
  DeviceGuard g(ctx->device);
  if (g.err != cudaSuccess) return cuda_fail(ctx, g.err, who);
  const size_t ysz = y_dtype == RTD_DT_F32 ? 4 : 2;
  cudaError_t e = cudaSuccess;
  // one rank runs the same kernel over its own buffers: y = partial + bias
  for (int64_t m0 = 0; m0 < M && e == cudaSuccess; m0 += kArTokens) {
    const int64_t mc = std::min<int64_t>(kArTokens, M - m0);
    e = rtd::launch_tp_allreduce(comm->tp, partial + m0 * ldp, ldp, mc, N, bias,
                                 static_cast<unsigned char*>(y) + (size_t)m0 * (size_t)ldy * ysz, (int)y_dtype, ldy,
                                 ctx->status, ctx->sm_count, (cudaStream_t)stream);
  }
  return e == cudaSuccess ? RTD_OK : cuda_fail(ctx, e, who);
}

// ---- allocation-free quantized linear ---------------------------------------
//
// For callers that must not allocate device memory while they run -- for example
// code that executes inside a host framework whose caching allocator owns the
// device's memory budget, where an extra cudaMalloc can fail or stall every stream
// on the device.  rtd_qlinear_noalloc dispatches like rtd_qlinear (the tensor-core
// GEMM from four tokens on when its staging fits, the decode GEMV otherwise) but
// takes its scratch -- the staged activations and the device status word -- from
// the fixed array below instead of a context workspace.
namespace {

constexpr size_t kNoAllocScratchBytes = 1u << 20;  // 1 MiB per device, fixed at build time
constexpr size_t kNoAllocStatusBytes = 256;        // the status word, then the workspace
constexpr int kNoAllocMaxDevices = 64;

__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

struct NoAllocDevice {
  bool ready = false;
  unsigned char* scratch = nullptr;  // device address of g_noalloc_scratch on this device
  int sm_count = 0;
};
std::mutex g_noalloc_mu;
NoAllocDevice g_noalloc_dev[kNoAllocMaxDevices];

// Once per device, with that device current: look up the array's device address.
rtd_status noalloc_setup(int dev, NoAllocDevice** out, const char* who) {
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoAllocDevice& d = g_noalloc_dev[dev];
  if (!d.ready) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return fail(nullptr, RTD_ERR_CUDA, "%s: cudaGetSymbolAddress: %s", who, cudaGetErrorString(e));
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return fail(nullptr, RTD_ERR_CUDA, "%s: cudaDeviceGetAttribute: %s", who, cudaGetErrorString(e));
    d.scratch = static_cast<unsigned char*>(p);
    d.sm_count = sms;
    d.ready = true;
  }
  *out = &d;
  return RTD_OK;
}

}  // namespace

rtd_status rtd_qlinear_noalloc(const rtd_qweight* w, const void* x, uint32_t x_dtype, int64_t ldx, int64_t M,
                               const float* bias, void* y, uint32_t y_dtype, int64_t ldy, void* stream) {
  const char* who = "rtd_qlinear_noalloc";
  if (!w || !w->ctx) return fail(nullptr, RTD_ERR_INVALID, "%s: NULL weight", who);
  if (M < 0) return fail(nullptr, RTD_ERR_SHAPE, "%s: M=%lld is negative", who, (long long)M);
  if (!valid_dtype(x_dtype) || !valid_dtype(y_dtype)) return fail(nullptr, RTD_ERR_INVALID, "%s: bad dtype", who);
  if (M == 0 || w->N == 0) return RTD_OK;
  if ((w->K > 0 && !x) || !y) return fail(nullptr, RTD_ERR_INVALID, "%s: x or y is NULL", who);
  if (ldx < w->K || ldy < w->N)
    return fail(nullptr, RTD_ERR_SHAPE, "%s: row strides ldx=%lld ldy=%lld below K=%lld N=%lld", who,
                (long long)ldx, (long long)ldy, (long long)w->K, (long long)w->N);
  const int dev = w->ctx->device;
  if (dev < 0 || dev >= kNoAllocMaxDevices) return fail(nullptr, RTD_ERR_INVALID, "%s: device %d out of range", who, dev);
  DeviceGuard g(dev);
  if (g.err != cudaSuccess) return cuda_fail(nullptr, g.err, who);
  NoAllocDevice* d = nullptr;
  rtd_status st = noalloc_setup(dev, &d, who);
  if (st != RTD_OK) return st;
  cudaError_t e;
  if (w->K == 0) {
    e = rtd::launch_fill_rows(bias, y, y_dtype, ldy, M, w->N, (cudaStream_t)stream);
    return e == cudaSuccess ? RTD_OK : cuda_fail(nullptr, e, who);
  }
  rtd::QGemvCall c{};
  c.fmt = w->fmt;
  c.w = w->dev;
  c.wpow2 = w->wpow2;
  c.row_scale = w->row_scale;
  c.scale_len = (int)w->N;
  c.N = w->N;
  c.K = w->K;
  c.G = w->G;
  c.x = x;
  c.x_dtype = (int)x_dtype;
  c.ldx = ldx;
  c.M = M;
  c.bias = bias;
  c.y = y;
  c.y_dtype = (int)y_dtype;
  c.ldy = ldy;
  c.ws = reinterpret_cast<float*>(d->scratch + kNoAllocStatusBytes);
  c.ws_bytes = kNoAllocScratchBytes - kNoAllocStatusBytes;
  // the status word is zero when the library loads and is cleared by
  // rtd_noalloc_check_status after it reports a raised code
  c.status = reinterpret_cast<int*>(d->scratch);
  c.sm_count = d->sm_count;
  c.stream = (cudaStream_t)stream;
  const bool gemm = M >= kGemmMinTokens && rtd::qgemm_workspace_bytes(c) <= c.ws_bytes;
  if (!gemm) {
    const size_t need = rtd::qgemv_workspace_bytes(c);
    if (need > c.ws_bytes)
      return fail(nullptr, RTD_ERR_WORKSPACE,
                  "%s: [%lld x %lld] at M=%lld needs %zu bytes of scratch; the static scratch holds %zu "
                  "(use rtd_qlinear, or fewer tokens per call)",
                  who, (long long)w->N, (long long)w->K, (long long)M, need, c.ws_bytes);
  }
  int plan_err = 0;
  e = gemm ? rtd::launch_qgemm(c, &plan_err) : rtd::launch_qgemv(c, &plan_err);
  if (plan_err) return fail(nullptr, RTD_ERR_WORKSPACE, "%s: [%lld x %lld] does not fit the static scratch", who,
                            (long long)w->N, (long long)w->K);
  if (e != cudaSuccess) return cuda_fail(nullptr, e, who);
  return RTD_OK;
}

rtd_status rtd_noalloc_check_status(int device, void* stream) {
  const char* who = "rtd_noalloc_check_status";
  if (device < 0 || device >= kNoAllocMaxDevices) return fail(nullptr, RTD_ERR_INVALID, "%s: device %d out of range", who, device);
  DeviceGuard g(device);
  if (g.err != cudaSuccess) return cuda_fail(nullptr, g.err, who);
  NoAllocDevice* d = nullptr;
  rtd_status st = noalloc_setup(device, &d, who);
  if (st != RTD_OK) return st;
  cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(nullptr, e, who);
  int v = 0;
  if ((e = cudaMemcpy(&v, d->scratch, sizeof(int), cudaMemcpyDeviceToHost)) != cudaSuccess)
    return cuda_fail(nullptr, e, who);
  if (v == 0) return RTD_OK;
  const int zero = 0;
  if ((e = cudaMemcpy(d->scratch, &zero, sizeof(int), cudaMemcpyHostToDevice)) != cudaSuccess)
    return cuda_fail(nullptr, e, who);
  if (v == RTD_ERR_PEER_TIMEOUT)
    return fail(nullptr, RTD_ERR_PEER_TIMEOUT, "a tensor-parallel peer did not arrive within the wait budget");
  return fail(nullptr, RTD_ERR_DEVICE, "%s: an allocation-free call raised device status code %d", who, v);
}
