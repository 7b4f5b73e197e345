// C ABI of the library (declared in include/slimdit_b200.h): argument validation, error
// reporting and dispatch to the kernel launchers.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/slimdit_b200.h"
#include "slim_kernels.h"
#include "slim_ptx.cuh"

namespace slim {

static std::atomic<uint64_t> g_launches{0};
uint64_t launch_count() { return g_launches.load(); }
void note_launch(uint64_t n) { g_launches.fetch_add(n); }

static thread_local char g_err[512] = {0};

static int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

static int cuda_fail(cudaError_t e, const char* what) {
  return fail(SLIM_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// Device must be sm_100 (B200). Cached per device.
static int check_arch() {
  static std::mutex mu;
  static int state[64] = {0};  // 0 unknown, 1 ok, 2 bad
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(SLIM_ERR_ARCH, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (state[dev] == 0) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    state[dev] = (major == 10 && minor == 0) ? 1 : 2;
    if (state[dev] == 2) return fail(SLIM_ERR_ARCH, "device %d is sm_%d%d; this library is built for sm_100a", dev, major, minor);
  }
  return state[dev] == 1 ? SLIM_OK : fail(SLIM_ERR_ARCH, "device %d is not sm_100", dev);
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static int check_group(int64_t K, int group) {
  if (group != 256) return fail(SLIM_ERR_GROUP, "group_size must be 256 (the convrot group), got %d", group);
  if (K <= 0 || K % 256 != 0) return fail(SLIM_ERR_GROUP, "in_features %lld not divisible by group_size 256", static_cast<long long>(K));
  if (K > (int64_t{1} << 30)) return fail(SLIM_ERR_SHAPE, "in_features %lld too large", static_cast<long long>(K));
  return SLIM_OK;
}

static int check_dtype(int dtype) {
  if (dtype != kF32 && dtype != kBF16 && dtype != kF16) return fail(SLIM_ERR_DTYPE, "unsupported dtype code %d", dtype);
  return SLIM_OK;
}

// The activation side of the linears: per-token rotation + INT8 in the reference's order
// (slimdit/hadamard.py:56-58 with slimdit/int8.py:49-51 per row), so the activation codes and
// scales are the reference's bit for bit: the certified kernel for rows of 5..64 groups, the
// reference-order kernels otherwise.
cudaError_t launch_act_quant(const void* x, int dtype, int64_t rows, int K, int8_t* q, float* scale, cudaStream_t st) {
  if (cert_supported(rows, K)) return launch_cert_rotate_quant(x, dtype, rows, K, q, scale, st);
  return launch_ref_rotate_quant(x, dtype, rows, K, q, scale, st);
}

}  // namespace slim

using namespace slim;

extern "C" {

int slim_version(void) { return SLIM_ABI_VERSION; }

int slim_last_error(char* buf, size_t len) {
  const size_t n = strlen(g_err);
  if (buf != nullptr && len > 0) {
    const size_t c = n < len - 1 ? n : len - 1;
    memcpy(buf, g_err, c);
    buf[c] = '\0';
  }
  return static_cast<int>(n);
}

uint64_t slim_launch_count(void) { return launch_count(); }

int slim_device_error(unsigned int* code) {
  if (code == nullptr) return fail(SLIM_ERR_NULL, "code is NULL");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  unsigned int v = 0;
  e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v));
  if (e != cudaSuccess) return cuda_fail(e, "read device error word");
  const unsigned int zero = 0;
  e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero));
  if (e != cudaSuccess) return cuda_fail(e, "clear device error word");
  *code = v;
  return SLIM_OK;
}

int slim_rotate_f32(const void* x, int dtype, int64_t rows, int64_t K, int group, int order,
                    float* out, void* stream) {
  SLIM_NVTX("slim_rotate_f32");
  int rc;
  if ((rc = check_group(K, group)) != SLIM_OK) return rc;
  if ((rc = check_dtype(dtype)) != SLIM_OK) return rc;
  if (rows < 0) return fail(SLIM_ERR_SHAPE, "negative row count");
  if (rows == 0) return SLIM_OK;
  if (x == nullptr || out == nullptr) return fail(SLIM_ERR_NULL, "x/out is NULL");
  if (!aligned16(x) || !aligned16(out)) return fail(SLIM_ERR_ALIGN, "x/out must be 16-byte aligned");
  if ((rc = check_arch()) != SLIM_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (order == SLIM_ORDER_REFERENCE) {
    e = launch_ref_rotate(x, dtype, rows, static_cast<int>(K), out, st);
  } else if (order == SLIM_ORDER_BUTTERFLY) {
    return fail(SLIM_ERR_DTYPE, "slim_rotate_f32 supports the reference order only; use slim_rotate_quant_i8 with rot_out");
  } else {
    return fail(SLIM_ERR_DTYPE, "unknown order %d", order);
  }
  if (e != cudaSuccess) return cuda_fail(e, "rotate launch");
  note_launch();
  return SLIM_OK;
}

int slim_rotate_quant_i8(const void* x, int dtype, int64_t rows, int64_t K, int group, int order,
                         int8_t* q, float* scale, float* rot_out, void* stream) {
  SLIM_NVTX("slim_rotate_quant_i8");
  int rc;
  if ((rc = check_group(K, group)) != SLIM_OK) return rc;
  if ((rc = check_dtype(dtype)) != SLIM_OK) return rc;
  if (rows < 0) return fail(SLIM_ERR_SHAPE, "negative row count");
  if (rows == 0) return SLIM_OK;
  if (x == nullptr || q == nullptr || scale == nullptr) return fail(SLIM_ERR_NULL, "x/q/scale is NULL");
  if (!aligned16(x) || !aligned16(q) || (rot_out != nullptr && !aligned16(rot_out)))
    return fail(SLIM_ERR_ALIGN, "x/q/rot_out must be 16-byte aligned");
  if (order == SLIM_ORDER_BUTTERFLY && K > 16384)
    return fail(SLIM_ERR_SHAPE, "butterfly order supports in_features <= 16384, got %lld", static_cast<long long>(K));
  if ((rc = check_arch()) != SLIM_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (order == SLIM_ORDER_REFERENCE) {
    if (rot_out != nullptr) {
      e = launch_ref_rotate(x, dtype, rows, static_cast<int>(K), rot_out, st);
      if (e != cudaSuccess) return cuda_fail(e, "rotate launch");
      note_launch();
      e = launch_quantize_rows(rot_out, rows, static_cast<int>(K), q, scale, st);
    } else if (cert_supported(rows, K)) {
      e = launch_cert_rotate_quant(x, dtype, rows, static_cast<int>(K), q, scale, st);
    } else {
      e = launch_ref_rotate_quant(x, dtype, rows, static_cast<int>(K), q, scale, st);
    }
  } else if (order == SLIM_ORDER_BUTTERFLY) {
    e = launch_bfly_rotate_quant(x, dtype, rows, static_cast<int>(K), q, scale, rot_out, st);
  } else {
    return fail(SLIM_ERR_DTYPE, "unknown order %d", order);
  }
  if (e != cudaSuccess) return cuda_fail(e, "rotate_quant launch");
  note_launch();
  return SLIM_OK;
}

int slim_quantize_rows_i8(const float* rotated, int64_t rows, int64_t K, int8_t* q, float* scale,
                          void* stream) {
  SLIM_NVTX("slim_quantize_rows_i8");
  int rc;
  if (rows < 0 || K <= 0 || K > (int64_t{1} << 30)) return fail(SLIM_ERR_SHAPE, "bad shape [%lld, %lld]", static_cast<long long>(rows), static_cast<long long>(K));
  if (rows == 0) return SLIM_OK;
  if (rotated == nullptr || q == nullptr || scale == nullptr) return fail(SLIM_ERR_NULL, "rotated/q/scale is NULL");
  if ((rc = check_arch()) != SLIM_OK) return rc;
  cudaError_t e = launch_quantize_rows(rotated, rows, static_cast<int>(K), q, scale, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "quantize launch");
  note_launch();
  return SLIM_OK;
}

int slim_dequant_i8(const int8_t* q, const float* scale, int64_t rows, int64_t K, int group,
                    float* out, void* stream) {
  SLIM_NVTX("slim_dequant_i8");
  int rc;
  if ((rc = check_group(K, group)) != SLIM_OK) return rc;
  if (rows < 0) return fail(SLIM_ERR_SHAPE, "negative row count");
  if (rows == 0) return SLIM_OK;
  if (q == nullptr || scale == nullptr || out == nullptr) return fail(SLIM_ERR_NULL, "q/scale/out is NULL");
  if ((rc = check_arch()) != SLIM_OK) return rc;
  cudaError_t e = launch_ref_dequant(q, scale, rows, static_cast<int>(K), out, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dequant launch");
  note_launch();
  return SLIM_OK;
}

// Output row pitch: N columns, or N/2 for the SwiGLU epilogue (one output per up/gate pair).
static int64_t out_pitch(int64_t N, int epilogue) { return epilogue == kEpiSwiGLU ? N / 2 : N; }

static int gemm_checks(const int8_t* a, const int8_t* b, const float* sa, const float* sb, const void* bias,
                       const void* out, const int32_t* acc_dbg, int64_t M, int64_t N, int64_t K, int epilogue) {
  if (M < 0 || N <= 0 || K <= 0) return fail(SLIM_ERR_SHAPE, "bad GEMM shape M=%lld N=%lld K=%lld", static_cast<long long>(M), static_cast<long long>(N), static_cast<long long>(K));
  if (K % 16 != 0) return fail(SLIM_ERR_SHAPE, "K=%lld must be a multiple of 16", static_cast<long long>(K));
  if (N % 8 != 0) return fail(SLIM_ERR_SHAPE, "N=%lld must be a multiple of 8", static_cast<long long>(N));
  if (M > (int64_t{1} << 31) || N > (int64_t{1} << 31)) return fail(SLIM_ERR_SHAPE, "GEMM dimension too large");
  if (epilogue != kEpiScaleBias && epilogue != kEpiGeluTanh && epilogue != kEpiSwiGLU)
    return fail(SLIM_ERR_DTYPE, "unknown epilogue %d", epilogue);
  if (epilogue == kEpiSwiGLU && (N % 256 != 0 || acc_dbg != nullptr))
    return fail(SLIM_ERR_SHAPE, "the SwiGLU epilogue needs N %% 256 == 0 (interleaved up/gate rows) and no accumulator copy");
  if (M == 0) return SLIM_OK;  // empty problem: nothing is read or written
  if (a == nullptr || b == nullptr || sa == nullptr || sb == nullptr || out == nullptr) return fail(SLIM_ERR_NULL, "a/b/sa/sb/out is NULL");
  if (!aligned16(a) || !aligned16(b) || !aligned16(sb) || !aligned16(out) || (bias != nullptr && !aligned16(bias)) ||
      (acc_dbg != nullptr && !aligned16(acc_dbg)))
    return fail(SLIM_ERR_ALIGN, "GEMM operands must be 16-byte aligned");
  return SLIM_OK;
}

int slim_gemm_i8(const int8_t* a, const int8_t* b, const float* sa, const float* sb, const void* bias, void* out,
                 int32_t* acc_dbg, int64_t M, int64_t N, int64_t K, int epilogue, void* stream) {
  SLIM_NVTX("slim_gemm_i8");
  int rc;
  if ((rc = gemm_checks(a, b, sa, sb, bias, out, acc_dbg, M, N, K, epilogue)) != SLIM_OK) return rc;
  if (M == 0) return SLIM_OK;
  if ((rc = check_arch()) != SLIM_OK) return rc;
  GemmI8Params p{a, b, sa, sb, bias, out, acc_dbg, M, N, K, out_pitch(N, epilogue), epilogue};
  cudaError_t e = launch_gemm_i8(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gemm launch");
  note_launch();
  return SLIM_OK;
}

int slim_int8_linear(const void* x, int x_dtype, const int8_t* qw, const float* sw, const void* bias, void* out,
                     int8_t* xq_ws, float* sx_ws, int64_t M, int64_t N, int64_t K, int group, int epilogue,
                     void* stream) {
  SLIM_NVTX("slim_int8_linear");
  int rc;
  if ((rc = check_group(K, group)) != SLIM_OK) return rc;
  if ((rc = check_dtype(x_dtype)) != SLIM_OK) return rc;
  if (K > 16384) return fail(SLIM_ERR_SHAPE, "in_features above 16384 not supported by the activation quantiser");
  if ((rc = gemm_checks(xq_ws, qw, sx_ws, sw, bias, out, nullptr, M, N, K, epilogue)) != SLIM_OK) return rc;
  if (M == 0) return SLIM_OK;
  if (x == nullptr) return fail(SLIM_ERR_NULL, "x is NULL");
  if (!aligned16(x)) return fail(SLIM_ERR_ALIGN, "x must be 16-byte aligned");
  if ((rc = check_arch()) != SLIM_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = launch_act_quant(x, x_dtype, M, static_cast<int>(K), xq_ws, sx_ws, st);
  if (e != cudaSuccess) return cuda_fail(e, "activation quant launch");
  note_launch();
  GemmI8Params p{xq_ws, qw, sx_ws, sw, bias, out, nullptr, M, N, K, out_pitch(N, epilogue), epilogue};
  e = launch_gemm_i8(p, st);
  if (e != cudaSuccess) return cuda_fail(e, "gemm launch");
  note_launch();
  return SLIM_OK;
}

int slim_ffn_i8(const void* x, int x_dtype, const int8_t* w_up, const float* s_up, const void* b_up,
                const int8_t* w_down, const float* s_down, const void* b_down, void* out, int8_t* xq_ws,
                float* sx_ws, void* h_ws, int8_t* hq_ws, float* sh_ws, int64_t M, int64_t K, int64_t F, int act,
                void* stream) {
  SLIM_NVTX("slim_ffn_i8");
  if (act != kEpiGeluTanh && act != kEpiSwiGLU)
    return fail(SLIM_ERR_DTYPE, "FFN activation must be GELU-tanh (%d) or SwiGLU (%d), got %d", kEpiGeluTanh,
                kEpiSwiGLU, act);
  if (F <= 0 || K <= 0 || M < 0) return fail(SLIM_ERR_SHAPE, "bad FFN shape M=%lld K=%lld F=%lld",
                                             static_cast<long long>(M), static_cast<long long>(K),
                                             static_cast<long long>(F));
  // up-projection: [M, K] x [F or 2F, K]^T with the activation in the epilogue -> h bf16 [M, F]
  const int64_t n_up = act == kEpiSwiGLU ? 2 * F : F;
  int rc = slim_int8_linear(x, x_dtype, w_up, s_up, b_up, h_ws, xq_ws, sx_ws, M, n_up, K, 256, act, stream);
  if (rc != SLIM_OK) return rc;
  // down-projection: h rotated and requantised per token, [M, F] x [K, F]^T -> out bf16 [M, K]
  return slim_int8_linear(h_ws, SLIM_BF16, w_down, s_down, b_down, out, hq_ws, sh_ws, M, K, F, 256, kEpiScaleBias,
                          stream);
}

int slim_peer_buffer_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  if (ptr == nullptr || ipc_handle == nullptr) return fail(SLIM_ERR_NULL, "ptr/ipc_handle is NULL");
  if (bytes == 0) return fail(SLIM_ERR_SHAPE, "empty peer buffer");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc of the peer buffer");
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "cudaIpcGetMemHandle");
  }
  memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return SLIM_OK;
}

int slim_peer_buffer_free(void* ptr) {
  if (ptr == nullptr) return SLIM_OK;
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFree of the peer buffer");
  return SLIM_OK;
}

int slim_peer_open(const void* ipc_handle, int64_t offset, void** ptr) {
  if (ipc_handle == nullptr || ptr == nullptr) return fail(SLIM_ERR_NULL, "ipc_handle/ptr is NULL");
  if (offset < 0 || offset % 16 != 0) return fail(SLIM_ERR_ALIGN, "offset %lld must be a non-negative multiple of 16", static_cast<long long>(offset));
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  *ptr = static_cast<char*>(base) + offset;
  return SLIM_OK;
}

int slim_peer_close(void* ptr, int64_t offset) {
  if (ptr == nullptr) return fail(SLIM_ERR_NULL, "ptr is NULL");
  cudaError_t e = cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcCloseMemHandle");
  return SLIM_OK;
}

int slim_copy_2d(void* dst, int64_t dpitch, const void* src, int64_t spitch, int64_t width, int64_t height,
                 void* stream) {
  SLIM_NVTX("slim_copy_2d");
  if (height == 0 || width == 0) return SLIM_OK;
  if (dst == nullptr || src == nullptr) return fail(SLIM_ERR_NULL, "dst/src is NULL");
  if (width < 0 || height < 0 || dpitch < width || spitch < width) return fail(SLIM_ERR_SHAPE, "bad 2-D copy geometry");
  cudaError_t e = cudaMemcpy2DAsync(dst, static_cast<size_t>(dpitch), src, static_cast<size_t>(spitch),
                                    static_cast<size_t>(width), static_cast<size_t>(height), cudaMemcpyDefault,
                                    static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy2DAsync");
  return SLIM_OK;
}

int slim_int8_linear_colsplit(const void* x, int x_dtype, const int8_t* qw, const float* sw, const void* bias,
                              void* const* outs, int n_outs, int64_t ldo, int8_t* xq_ws, float* sx_ws, int64_t M,
                              int64_t N, int64_t K, int group, int epilogue, void* stream) {
  SLIM_NVTX("slim_int8_linear_colsplit");
  int rc;
  if (outs == nullptr || n_outs < 1 || n_outs > kMaxPeers + 1)
    return fail(SLIM_ERR_SHAPE, "n_outs must be 1..%d, got %d", kMaxPeers + 1, n_outs);
  for (int i = 0; i < n_outs; ++i)
    if (outs[i] == nullptr || !aligned16(outs[i])) return fail(SLIM_ERR_ALIGN, "output %d is NULL or not 16-byte aligned", i);
  if (ldo < N || ldo % 8 != 0) return fail(SLIM_ERR_SHAPE, "ldo=%lld must be >= N and a multiple of 8", static_cast<long long>(ldo));
  if ((rc = check_group(K, group)) != SLIM_OK) return rc;
  if ((rc = check_dtype(x_dtype)) != SLIM_OK) return rc;
  if (K > 16384) return fail(SLIM_ERR_SHAPE, "in_features above 16384 not supported by the activation quantiser");
  if ((rc = gemm_checks(xq_ws, qw, sx_ws, sw, bias, outs[0], nullptr, M, N, K, epilogue)) != SLIM_OK) return rc;
  if (epilogue == kEpiSwiGLU) return fail(SLIM_ERR_DTYPE, "the column-split linear does not take the SwiGLU epilogue");
  if (M == 0) return SLIM_OK;
  if (x == nullptr) return fail(SLIM_ERR_NULL, "x is NULL");
  if (!aligned16(x)) return fail(SLIM_ERR_ALIGN, "x must be 16-byte aligned");
  if ((rc = check_arch()) != SLIM_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = launch_act_quant(x, x_dtype, M, static_cast<int>(K), xq_ws, sx_ws, st);
  if (e != cudaSuccess) return cuda_fail(e, "activation quant launch");
  note_launch();
  GemmI8Params p{xq_ws, qw, sx_ws, sw, bias, outs[0], nullptr, M, N, K, ldo, epilogue};
  p.n_peer = n_outs - 1;
  for (int i = 1; i < n_outs; ++i) p.peer_out[i - 1] = outs[i];
  e = launch_gemm_i8(p, st);
  if (e != cudaSuccess) return cuda_fail(e, "gemm launch");
  note_launch();
  return SLIM_OK;
}

}  // extern "C"
