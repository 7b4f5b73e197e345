// Checkpoint verification on the GPU: the distances tools/verify_checkpoint.py computes with
// numpy (relative L2 error between two versions of a tensor, verify_checkpoint.py:81-118),
// reduced in fp64 on the device.
//
//   rel_l2_int8   rows of INT8 codes times per-row scales on both sides, compared in the rotated
//                 basis as load_value(rotated=True) does (verify_checkpoint.py:71-75):
//                 a = fl32(float(qa) * sa[row]), b likewise;
//   rel_l2        two tensors of any of f32/bf16/f16 (compared as fp32 values).
// Both accumulate sum (a - b)^2 and sum b^2 into out2[0], out2[1] (fp64, not cleared).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "slim_kernels.h"

namespace slim {
namespace verify {

__device__ __forceinline__ void block_accumulate(double e2, double b2, double* out2) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    e2 += __shfl_xor_sync(0xffffffffu, e2, o);
    b2 += __shfl_xor_sync(0xffffffffu, b2, o);
  }
  if ((threadIdx.x & 31) == 0) {
    atomicAdd(out2, e2);
    atomicAdd(out2 + 1, b2);
  }
}

__global__ void __launch_bounds__(256) rel_l2_int8_kernel(const int8_t* __restrict__ qa, const float* __restrict__ sa,
                                                          const int8_t* __restrict__ qb, const float* __restrict__ sb,
                                                          int64_t rows, int64_t K, double* __restrict__ out2) {
  double e2 = 0.0, b2 = 0.0;
  const int64_t vecs = K / 16;  // K % 16 == 0: 16 codes per load
  const int64_t total = rows * vecs;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / vecs;
    const float fa = __ldg(sa + r), fb = __ldg(sb + r);
    const int4 va = __ldg(reinterpret_cast<const int4*>(qa) + i);
    const int4 vb = __ldg(reinterpret_cast<const int4*>(qb) + i);
    const int wa[4] = {va.x, va.y, va.z, va.w}, wb[4] = {vb.x, vb.y, vb.z, vb.w};
#pragma unroll
    for (int w = 0; w < 4; ++w) {
#pragma unroll
      for (int byte = 0; byte < 4; ++byte) {
        const float a = __fmul_rn(static_cast<float>(static_cast<int8_t>(wa[w] >> (8 * byte))), fa);
        const float b = __fmul_rn(static_cast<float>(static_cast<int8_t>(wb[w] >> (8 * byte))), fb);
        const double d = static_cast<double>(a) - static_cast<double>(b);
        e2 += d * d;
        b2 += static_cast<double>(b) * static_cast<double>(b);
      }
    }
  }
  block_accumulate(e2, b2, out2);
}

template <int DT>
__device__ __forceinline__ float load_f(const void* p, int64_t i) {
  if (DT == kF32) return __ldg(static_cast<const float*>(p) + i);
  if (DT == kBF16) return __uint_as_float(static_cast<uint32_t>(__ldg(static_cast<const unsigned short*>(p) + i)) << 16);
  return __half2float(__ldg(static_cast<const __half*>(p) + i));
}

template <int DA, int DB>
__global__ void __launch_bounds__(256) rel_l2_kernel(const void* __restrict__ a, const void* __restrict__ b, int64_t n,
                                                     double* __restrict__ out2) {
  double e2 = 0.0, b2 = 0.0;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const double x = load_f<DA>(a, i), y = load_f<DB>(b, i);
    e2 += (x - y) * (x - y);
    b2 += y * y;
  }
  block_accumulate(e2, b2, out2);
}

template <int DA>
static cudaError_t launch_rel_l2_b(int db, const void* a, const void* b, int64_t n, double* out2, int grid,
                                   cudaStream_t st) {
  switch (db) {
    case kF32: rel_l2_kernel<DA, kF32><<<grid, 256, 0, st>>>(a, b, n, out2); break;
    case kBF16: rel_l2_kernel<DA, kBF16><<<grid, 256, 0, st>>>(a, b, n, out2); break;
    case kF16: rel_l2_kernel<DA, kF16><<<grid, 256, 0, st>>>(a, b, n, out2); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

static int grid_size() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms * 8;
}

}  // namespace verify

cudaError_t launch_rel_l2_int8(const int8_t* qa, const float* sa, const int8_t* qb, const float* sb, int64_t rows,
                               int64_t K, double* out2, cudaStream_t st) {
  verify::rel_l2_int8_kernel<<<verify::grid_size(), 256, 0, st>>>(qa, sa, qb, sb, rows, K, out2);
  return cudaGetLastError();
}

cudaError_t launch_rel_l2(const void* a, int da, const void* b, int db, int64_t n, double* out2, cudaStream_t st) {
  const int grid = verify::grid_size();
  switch (da) {
    case kF32: return verify::launch_rel_l2_b<kF32>(db, a, b, n, out2, grid, st);
    case kBF16: return verify::launch_rel_l2_b<kBF16>(db, a, b, n, out2, grid, st);
    case kF16: return verify::launch_rel_l2_b<kF16>(db, a, b, n, out2, grid, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace slim

using namespace slim;

extern "C" {

int slim_rel_l2_int8(const int8_t* qa, const float* sa, const int8_t* qb, const float* sb, int64_t rows, int64_t K,
                     double* out2, void* stream) {
  SLIM_NVTX("slim_rel_l2_int8");
  int rc;
  if (rows < 0 || K <= 0 || K % 16 != 0) return fail(SLIM_ERR_SHAPE, "rel_l2_int8 needs K %% 16 == 0, got %lld", static_cast<long long>(K));
  if (rows == 0) return SLIM_OK;
  if (qa == nullptr || sa == nullptr || qb == nullptr || sb == nullptr || out2 == nullptr)
    return fail(SLIM_ERR_NULL, "qa/sa/qb/sb/out2 is NULL");
  if (!aligned16(qa) || !aligned16(qb) || (reinterpret_cast<uintptr_t>(out2) & 7u))
    return fail(SLIM_ERR_ALIGN, "codes must be 16-byte aligned, out2 8-byte aligned");
  if ((rc = check_arch()) != SLIM_OK) return rc;
  cudaError_t e = launch_rel_l2_int8(qa, sa, qb, sb, rows, K, out2, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "rel_l2_int8 launch");
  note_launch();
  return SLIM_OK;
}

int slim_rel_l2(const void* a, int a_dtype, const void* b, int b_dtype, int64_t n, double* out2, void* stream) {
  SLIM_NVTX("slim_rel_l2");
  int rc;
  if ((rc = check_dtype(a_dtype)) != SLIM_OK) return rc;
  if ((rc = check_dtype(b_dtype)) != SLIM_OK) return rc;
  if (n < 0) return fail(SLIM_ERR_SHAPE, "negative element count");
  if (n == 0) return SLIM_OK;
  if (a == nullptr || b == nullptr || out2 == nullptr) return fail(SLIM_ERR_NULL, "a/b/out2 is NULL");
  if (reinterpret_cast<uintptr_t>(out2) & 7u) return fail(SLIM_ERR_ALIGN, "out2 must be 8-byte aligned");
  if ((rc = check_arch()) != SLIM_OK) return rc;
  cudaError_t e = launch_rel_l2(a, a_dtype, b, b_dtype, n, out2, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "rel_l2 launch");
  note_launch();
  return SLIM_OK;
}

}  // extern "C"
