// C ABI of the NVFP4 path (declared in include/slimdit_b200.h): argument validation and
// dispatch to the quantiser and block-scaled FP4 GEMM launchers. Shares the error/arch
// helpers of capi.cu (same translation unit).
#include <cuda_runtime.h>

#include "../../include/slimdit_b200.h"
#include "slim_kernels.h"

namespace slim {

static int nvfp4_k_checks(int64_t K, bool rotate) {
  if (K <= 0 || K % 64 != 0)
    return fail(SLIM_ERR_SHAPE, "NVFP4 needs in_features %% 64 == 0 (16-element blocks, 4 per scale tile), got %lld",
                static_cast<long long>(K));
  if (K > 16384) return fail(SLIM_ERR_SHAPE, "NVFP4 quantiser supports in_features <= 16384, got %lld", static_cast<long long>(K));
  if (rotate && K % 256 != 0) return fail(SLIM_ERR_GROUP, "rotation needs in_features %% 256 == 0, got %lld", static_cast<long long>(K));
  return SLIM_OK;
}

static int nvfp4_gemm_checks(const uint8_t* a, const uint8_t* a_sf, const float* a_scale, const uint8_t* b,
                             const uint8_t* b_sf, const float* b_scale, const void* bias, const void* out,
                             const float* acc_dbg, int64_t M, int64_t N, int64_t K, int epilogue) {
  if (M < 0 || N <= 0 || K <= 0) return fail(SLIM_ERR_SHAPE, "bad GEMM shape M=%lld N=%lld K=%lld", static_cast<long long>(M), static_cast<long long>(N), static_cast<long long>(K));
  if (K % 64 != 0) return fail(SLIM_ERR_SHAPE, "K=%lld must be a multiple of 64", static_cast<long long>(K));
  if (N % 128 != 0) return fail(SLIM_ERR_SHAPE, "N=%lld must be a multiple of 128 (NVFP4 weight tiling)", static_cast<long long>(N));
  if (M > (int64_t{1} << 31) || N > (int64_t{1} << 31)) return fail(SLIM_ERR_SHAPE, "GEMM dimension too large");
  if (epilogue != kEpiScaleBias && epilogue != kEpiGeluTanh)
    return fail(SLIM_ERR_DTYPE, "unknown epilogue %d (the NVFP4 GEMM takes scale+bias or GELU-tanh)", epilogue);
  if (M == 0) return SLIM_OK;
  if (a == nullptr || a_sf == nullptr || a_scale == nullptr || b == nullptr || b_sf == nullptr || b_scale == nullptr ||
      out == nullptr)
    return fail(SLIM_ERR_NULL, "a/a_sf/a_scale/b/b_sf/b_scale/out is NULL");
  if (!aligned16(a) || !aligned16(a_sf) || !aligned16(b) || !aligned16(b_sf) || !aligned16(out) ||
      (bias != nullptr && !aligned16(bias)) || (acc_dbg != nullptr && !aligned16(acc_dbg)))
    return fail(SLIM_ERR_ALIGN, "NVFP4 GEMM operands must be 16-byte aligned");
  return SLIM_OK;
}

}  // namespace slim

using namespace slim;

extern "C" {

int slim_nvfp4_pack(const void* w, int dtype, int64_t rows, int64_t K, uint8_t* q, uint8_t* block_scale,
                    float* tensor_scale, void* stream) {
  SLIM_NVTX("slim_nvfp4_pack");
  int rc;
  if ((rc = check_dtype(dtype)) != SLIM_OK) return rc;
  if ((rc = nvfp4_k_checks(K, false)) != SLIM_OK) return rc;
  if (rows <= 0 || rows % 128 != 0)
    return fail(SLIM_ERR_SHAPE, "NVFP4 tiling expects rows %% 128 == 0, got %lld", static_cast<long long>(rows));
  if (w == nullptr || q == nullptr || block_scale == nullptr || tensor_scale == nullptr)
    return fail(SLIM_ERR_NULL, "w/q/block_scale/tensor_scale is NULL");
  if (!aligned16(w) || !aligned16(q) || !aligned16(block_scale) || (reinterpret_cast<uintptr_t>(tensor_scale) & 3u))
    return fail(SLIM_ERR_ALIGN, "w/q/block_scale must be 16-byte aligned");
  if ((rc = check_arch()) != SLIM_OK) return rc;
  int launches = 0;
  cudaError_t e = launch_nvfp4_pack(w, dtype, rows, static_cast<int>(K), q, block_scale, tensor_scale, &launches,
                                    static_cast<cudaStream_t>(stream));
  note_launch(static_cast<uint64_t>(launches));
  if (e != cudaSuccess) return cuda_fail(e, "nvfp4 pack launch");
  return SLIM_OK;
}

int slim_quant_nvfp4_act(const void* x, int dtype, int64_t rows, int64_t K, int rotate, uint8_t* q,
                         uint8_t* block_scale, float* row_scale, void* stream) {
  SLIM_NVTX("slim_quant_nvfp4_act");
  int rc;
  if ((rc = check_dtype(dtype)) != SLIM_OK) return rc;
  if ((rc = nvfp4_k_checks(K, rotate != 0)) != SLIM_OK) return rc;
  if (rows < 0) return fail(SLIM_ERR_SHAPE, "negative row count");
  if (rows == 0) return SLIM_OK;
  if (x == nullptr || q == nullptr || block_scale == nullptr || row_scale == nullptr)
    return fail(SLIM_ERR_NULL, "x/q/block_scale/row_scale is NULL");
  if (!aligned16(x) || !aligned16(q)) return fail(SLIM_ERR_ALIGN, "x/q must be 16-byte aligned");
  if ((rc = check_arch()) != SLIM_OK) return rc;
  cudaError_t e = launch_nvfp4_quant_rows(x, dtype, rows, static_cast<int>(K), rotate, q, block_scale, row_scale,
                                          static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "nvfp4 activation quant launch");
  note_launch();
  return SLIM_OK;
}

int slim_nvfp4_dequant(const uint8_t* q, const uint8_t* block_scale, const float* scale, int per_row, int64_t rows,
                       int64_t K, float* out, const void* x, int x_dtype, double* err, void* stream) {
  SLIM_NVTX("slim_nvfp4_dequant");
  int rc;
  if ((rc = nvfp4_k_checks(K, false)) != SLIM_OK) return rc;
  if (rows < 0) return fail(SLIM_ERR_SHAPE, "negative row count");
  if (rows == 0) return SLIM_OK;
  if (q == nullptr || block_scale == nullptr || scale == nullptr) return fail(SLIM_ERR_NULL, "q/block_scale/scale is NULL");
  if (out == nullptr && err == nullptr) return fail(SLIM_ERR_NULL, "out and err are both NULL");
  if (err != nullptr && x == nullptr) return fail(SLIM_ERR_NULL, "err needs the original x");
  if (x != nullptr && (rc = check_dtype(x_dtype)) != SLIM_OK) return rc;
  if (!aligned16(q) || (out != nullptr && !aligned16(out)) || (x != nullptr && !aligned16(x)) ||
      (err != nullptr && (reinterpret_cast<uintptr_t>(err) & 7u)))
    return fail(SLIM_ERR_ALIGN, "q/out/x must be 16-byte aligned, err 8-byte aligned");
  if ((rc = check_arch()) != SLIM_OK) return rc;
  cudaError_t e = launch_nvfp4_dequant(q, block_scale, scale, per_row, rows, static_cast<int>(K), out, x, x_dtype,
                                       err, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "nvfp4 dequant launch");
  note_launch();
  return SLIM_OK;
}

int slim_gemm_nvfp4(const uint8_t* a, const uint8_t* a_sf, const float* a_scale, const uint8_t* b,
                    const uint8_t* b_sf, const float* b_scale, const void* bias, void* out, float* acc_dbg, int64_t M,
                    int64_t N, int64_t K, int epilogue, void* stream) {
  SLIM_NVTX("slim_gemm_nvfp4");
  int rc;
  if ((rc = nvfp4_gemm_checks(a, a_sf, a_scale, b, b_sf, b_scale, bias, out, acc_dbg, M, N, K, epilogue)) != SLIM_OK)
    return rc;
  if (M == 0) return SLIM_OK;
  if ((rc = check_arch()) != SLIM_OK) return rc;
  GemmNvf4Params p{a, b, a_sf, b_sf, a_scale, b_scale, bias, out, acc_dbg, M, N, K, N, epilogue};
  cudaError_t e = launch_gemm_nvf4(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "nvfp4 gemm launch");
  note_launch();
  return SLIM_OK;
}

int slim_nvfp4_linear(const void* x, int x_dtype, const uint8_t* qw, const uint8_t* w_sf, const float* w_scale,
                      const void* bias, void* out, uint8_t* xq_ws, uint8_t* xsf_ws, float* xs_ws, int64_t M, int64_t N,
                      int64_t K, int rotate, int epilogue, void* stream) {
  SLIM_NVTX("slim_nvfp4_linear");
  int rc;
  if ((rc = check_dtype(x_dtype)) != SLIM_OK) return rc;
  if ((rc = nvfp4_k_checks(K, rotate != 0)) != SLIM_OK) return rc;
  if ((rc = nvfp4_gemm_checks(xq_ws, xsf_ws, xs_ws, qw, w_sf, w_scale, bias, out, nullptr, M, N, K, epilogue)) != SLIM_OK)
    return rc;
  if (M == 0) return SLIM_OK;
  if (x == nullptr) return fail(SLIM_ERR_NULL, "x is NULL");
  if (!aligned16(x)) return fail(SLIM_ERR_ALIGN, "x must be 16-byte aligned");
  if ((rc = check_arch()) != SLIM_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = launch_nvfp4_quant_rows(x, x_dtype, M, static_cast<int>(K), rotate, xq_ws, xsf_ws, xs_ws, st);
  if (e != cudaSuccess) return cuda_fail(e, "nvfp4 activation quant launch");
  note_launch();
  GemmNvf4Params p{xq_ws, qw, xsf_ws, w_sf, xs_ws, w_scale, bias, out, nullptr, M, N, K, N, epilogue};
  e = launch_gemm_nvf4(p, st);
  if (e != cudaSuccess) return cuda_fail(e, "nvfp4 gemm launch");
  note_launch();
  return SLIM_OK;
}

}  // extern "C"
