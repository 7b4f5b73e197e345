// Internal launcher declarations shared by the kernel files and the C-ABI layer.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

#include <cstddef>
#include <cstdint>
#include <mutex>

namespace slim {

// NVTX range around a C-ABI entry point, so that a profiler's timeline groups each call's
// kernel launches under the entry's name (header-only NVTX v3: without a profiler attached
// the push/pop calls return at once).
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};
#define SLIM_NVTX(name) ::slim::NvtxRange slim_nvtx_range_(name)

// Lazy per-device initialisation for the launchers' caches (kernel attributes, occupancy):
// run() calls init once per device under a lock, later calls only check the flag; an init that
// fails leaves the device unset so the next call retries. Devices beyond 64 run init each time.
class PerDeviceOnce {
 public:
  template <typename F>
  cudaError_t run(int dev, F&& init) {
    if (dev < 0 || dev >= 64) return init();
    std::lock_guard<std::mutex> lock(mu_);
    if (done_[dev]) return cudaSuccess;
    const cudaError_t e = init();
    if (e == cudaSuccess) done_[dev] = true;
    return e;
  }

 private:
  std::mutex mu_;
  bool done_[64] = {};
};

enum DType : int { kF32 = 0, kBF16 = 1, kF16 = 2 };

enum Epilogue : int {
  kEpiScaleBias = 0,   // y = bf16(acc * sa[m] * sb[n] + bias[n])
  kEpiGeluTanh = 1,    // y = bf16(gelu_tanh(float(bf16(acc * sa[m] * sb[n] + bias[n]))))
  kEpiSwiGLU = 2,      // rows interleaved per 256 (128 up, 128 gate): y[m, n/2 + i] = bf16(up * bf16(silu(gate)))
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

// cert_quant.cu: reference-order rotate + quantise (codes and scales bit-identical to
// launch_ref_rotate_quant) at the fast transform's cost. Rows of 5 <= K/256 <= 64 groups,
// rows < 2^32, 16-byte aligned input.
cudaError_t launch_cert_rotate_quant(const void* x, int dtype, int64_t rows, int K, int8_t* q, float* scale,
                                     cudaStream_t st);
// capi.cu: the linears' activation quantiser (reference order; certified kernel where it applies).
cudaError_t launch_act_quant(const void* x, int dtype, int64_t rows, int K, int8_t* q, float* scale, cudaStream_t st);
// Whether launch_cert_rotate_quant takes this shape.
inline bool cert_supported(int64_t rows, int64_t K) {
  const int64_t g = K / 256;
  return K % 256 == 0 && g >= 5 && g <= 64 && rows < (int64_t{1} << 32);
}

// gemm_i8.cu
constexpr int kMaxPeers = 7;  // peer destinations of the column-split linear (8 GPUs per node)

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
  // Further destinations of the output, same layout as `out` (other GPUs' buffers mapped into
  // this process): the epilogue stores every tile to `out` and to each of them.
  void* peer_out[kMaxPeers];
  int n_peer;
};
cudaError_t launch_gemm_i8(const GemmI8Params& p, cudaStream_t st);

// nvfp4_quant.cu
cudaError_t launch_nvfp4_pack(const void* w, int dtype, int64_t rows, int K, uint8_t* q, uint8_t* sf,
                              float* tensor_scale, int* launches, cudaStream_t st);
cudaError_t launch_nvfp4_quant_rows(const void* x, int dtype, int64_t rows, int K, int rotate, uint8_t* q,
                                    uint8_t* sf, float* row_scale, cudaStream_t st);
cudaError_t launch_nvfp4_dequant(const uint8_t* q, const uint8_t* sf, const float* scale, int per_row, int64_t rows,
                                 int K, float* out, const void* x, int x_dtype, double* err, cudaStream_t st);

// gemm_nvf4.cu
struct GemmNvf4Params {
  const uint8_t* a;       // [M, K/2] packed E2M1 (token rows)
  const uint8_t* b;       // [N, K/2] packed E2M1 (output channels)
  const uint8_t* sfa;     // UE4M3 block scales of a, tiled layout, [round_up(M,128), K/16]
  const uint8_t* sfb;     // UE4M3 block scales of b, tiled layout, [N, K/16]
  const float* sa;        // [M] per-token global scales
  const float* sb;        // [1] per-tensor global scale of b
  const void* bias;       // bf16 [N] or null
  void* out;              // bf16 [M, N] row-major, row pitch ldo elements
  float* acc_dbg;         // fp32 [M, N] raw accumulators or null
  int64_t M, N, K;
  int64_t ldo;
  int epilogue;
};
cudaError_t launch_gemm_nvf4(const GemmNvf4Params& p, cudaStream_t st);

// Count of kernels launched by this library since load (instrumentation for benches).
uint64_t launch_count();
void note_launch(uint64_t n = 1);

}  // namespace slim
