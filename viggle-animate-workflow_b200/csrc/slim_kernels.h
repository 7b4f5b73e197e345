// Internal launcher declarations shared by the kernel files and the C-ABI layer.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace slim {

enum DType : int { kF32 = 0, kBF16 = 1, kF16 = 2 };

enum Epilogue : int {
  kEpiScaleBias = 0,   // y = bf16(acc * sa[m] * sb[n] + bias[n])
  kEpiGeluTanh = 1,    // y = bf16(gelu_tanh(float(bf16(acc * sa[m] * sb[n] + bias[n]))))
};

// rotate_quant.cu
cudaError_t launch_ref_rotate(const void* x, int dtype, int64_t rows, int K, float* out,
                              cudaStream_t st);
cudaError_t launch_ref_rotate_quant(const void* x, int dtype, int64_t rows, int K, int8_t* q,
                                    float* scale, cudaStream_t st);
cudaError_t launch_ref_dequant(const int8_t* q, const float* scale, int64_t rows, int K,
                               float* out, cudaStream_t st);
cudaError_t launch_bfly_rotate_quant(const void* x, int dtype, int64_t rows, int K, int8_t* q,
                                     float* scale, float* rot_out, cudaStream_t st);
cudaError_t launch_quantize_rows(const float* rot, int64_t rows, int K, int8_t* q, float* scale,
                                 cudaStream_t st);

// gemm_i8.cu
struct GemmI8Params {
  const int8_t* a;        // [M, K] row-major (token rows, rotated + quantised)
  const int8_t* b;        // [N, K] row-major (output channels)
  const float* sa;        // [M]
  const float* sb;        // [N]
  const void* bias;       // bf16 [N] or null
  void* out;              // bf16 [M, N] row-major, row pitch ldo elements
  int32_t* acc_dbg;       // int32 [M, N] or null
  int64_t M, N, K;
  int64_t ldo;
  int epilogue;
};
cudaError_t launch_gemm_i8(const GemmI8Params& p, cudaStream_t st);

// Count of kernels launched by this library since load (instrumentation for benches).
uint64_t launch_count();
void note_launch(uint64_t n = 1);

}  // namespace slim
