// Group-256 regular-Hadamard rotation fused with per-row symmetric INT8 quantisation.
//
// H = H4 (x) H4 (x) H4 (x) H4 / 16 with H4 = [[1,1,1,-1],[1,1,-1,1],[1,-1,1,1],[-1,1,1,1]]
// (slimdit/hadamard.py:18-42). Entry (j,k) is (1/16) * prod_d H4[j_d][k_d] over the base-4
// digits of j and k, and H4[a][b] = -1 exactly when a + b == 3.
//
// Two summation orders are provided, both computed in fp32:
//
//  * REFERENCE order reproduces the reference's `np.matmul(grouped, H.T)`
//    (slimdit/hadamard.py:56-58) as executed by numpy 2.3 / OpenBLAS 0.3.30 on x86-64
//    (SkylakeX kernels). numpy issues one sgemm of shape [G,256]x[256,256] per row
//    (G = K/256), and OpenBLAS picks the kernel from G:
//      G >= 5      : plain sgemm micro-kernel, one sequential fused chain over k = 0..255
//      2 <= G <= 4 : small-matrix kernel, 16 partial sums over k mod 16 (each a
//                    sequential chain), then a pairwise tree (0+1, 2+3, ...)
//      G == 1      : sgemv kernel, 8 partial sums over k mod 8, then lanes l and l+4 are
//                    combined, then (0+1)+(2+3)
//    Every product x*h is exact (h = +-2^-4), so each chain is a sequence of exactly
//    rounded fp32 additions of +-x; the kernels accumulate +-x and scale by 1/16 at the
//    end, which is exact. Zero results are returned as +0, as the reference's
//    accumulators (which start at +0) produce.
//  * BUTTERFLY order is the fast radix-4 transform used for activations: four stages,
//    one per base-4 digit (least significant first); on each 4-tuple (a0..a3) of a stage
//    b_i = ((a0 + a1) + (a2 + a3)) - 2*a_{3-i}, each step rounded to fp32; then * 1/16.
//
// Quantisation follows slimdit/int8.py:49-51 bit for bit:
//   scale = max(fl32(absmax / 127), 1e-30f);  q = clamp(rint(fl32(v / scale)), -128, 127)
// with an IEEE (correctly rounded) division and round-half-to-even.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "slim_kernels.h"

namespace slim {

// ------------------------------------------------------------------ element loaders
template <int DT>
struct Loader;

template <>
struct Loader<kF32> {
  __device__ __forceinline__ static float at(const void* p, int64_t i) {
    return __ldg(static_cast<const float*>(p) + i);
  }
};
template <>
struct Loader<kBF16> {
  __device__ __forceinline__ static float at(const void* p, int64_t i) {
    const unsigned short u = __ldg(static_cast<const unsigned short*>(p) + i);
    return __uint_as_float(static_cast<uint32_t>(u) << 16);
  }
};
template <>
struct Loader<kF16> {
  __device__ __forceinline__ static float at(const void* p, int64_t i) {
    return __half2float(__ldg(static_cast<const __half*>(p) + i));
  }
};

__device__ __forceinline__ float h4sign(int a, int b) { return (a + b == 3) ? -1.0f : 1.0f; }

// Sign of H[j][k] (before the 1/16) as +-1.
__device__ __forceinline__ float hsign(int j, int k) {
  float s = 1.0f;
#pragma unroll
  for (int d = 0; d < 4; ++d) s *= h4sign((j >> (2 * d)) & 3, (k >> (2 * d)) & 3);
  return s;
}

__device__ __forceinline__ float canon_zero(float v) { return v == 0.0f ? 0.0f : v; }

// One output of the reference-order rotation. xs = the group's 256 inputs in shared memory
// (fp32), j = output index. Returns the fp32 rotated value.
template <int ORDER_KIND>
__device__ __forceinline__ float ref_rotate_one(const float* __restrict__ xs, int j);

// G >= 5: one sequential chain. k = 16*b + l; the sign factorises as sigma(j, b) * lam(j, l).
// The accumulator is carried as sigma_b * acc so the inner 16 steps are fma(x, lam_l, acc)
// (exact product, one rounding); at a block change it is multiplied by sigma_b*sigma_{b-1}
// (an exact sign flip). fl(s*a + s*t) = s*fl(a + t) keeps this identical to the plain chain.
template <>
__device__ __forceinline__ float ref_rotate_one<0>(const float* __restrict__ xs, int j) {
  const int j0 = j & 3, j1 = (j >> 2) & 3, j2 = (j >> 4) & 3, j3 = (j >> 6) & 3;
  float lam[16];
#pragma unroll
  for (int l = 0; l < 16; ++l) lam[l] = h4sign(j1, l >> 2) * h4sign(j0, l & 3);
  float sig[16];
#pragma unroll
  for (int b = 0; b < 16; ++b) sig[b] = h4sign(j3, b >> 2) * h4sign(j2, b & 3);
  const float4* x4 = reinterpret_cast<const float4*>(xs);
  float acc = 0.0f;
#pragma unroll
  for (int b = 0; b < 16; ++b) {
    if (b > 0) acc *= sig[b] * sig[b - 1];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 v = x4[b * 4 + q];
      acc = __fmaf_rn(v.x, lam[4 * q + 0], acc);
      acc = __fmaf_rn(v.y, lam[4 * q + 1], acc);
      acc = __fmaf_rn(v.z, lam[4 * q + 2], acc);
      acc = __fmaf_rn(v.w, lam[4 * q + 3], acc);
    }
  }
  acc *= sig[15];
  return canon_zero(acc * 0.0625f);
}

// 2 <= G <= 4: 16 chains over k mod 16 (k = 16*t + l), then the pairwise tree.
// Chain l accumulates sigma(j, t) * x in order t = 0..15; lam(j, l) is applied after
// (exact sign flip, see above).
template <>
__device__ __forceinline__ float ref_rotate_one<1>(const float* __restrict__ xs, int j) {
  const int j0 = j & 3, j1 = (j >> 2) & 3, j2 = (j >> 4) & 3, j3 = (j >> 6) & 3;
  float sig[16];
#pragma unroll
  for (int t = 0; t < 16; ++t) sig[t] = h4sign(j3, t >> 2) * h4sign(j2, t & 3);
  float u[16];
#pragma unroll
  for (int l = 0; l < 16; ++l) u[l] = 0.0f;
  const float4* x4 = reinterpret_cast<const float4*>(xs);
#pragma unroll
  for (int t = 0; t < 16; ++t) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 v = x4[t * 4 + q];
      u[4 * q + 0] = __fmaf_rn(v.x, sig[t], u[4 * q + 0]);
      u[4 * q + 1] = __fmaf_rn(v.y, sig[t], u[4 * q + 1]);
      u[4 * q + 2] = __fmaf_rn(v.z, sig[t], u[4 * q + 2]);
      u[4 * q + 3] = __fmaf_rn(v.w, sig[t], u[4 * q + 3]);
    }
  }
#pragma unroll
  for (int l = 0; l < 16; ++l) u[l] *= h4sign(j1, l >> 2) * h4sign(j0, l & 3);
#pragma unroll
  for (int w = 8; w >= 1; w >>= 1) {
#pragma unroll
    for (int i = 0; i < w; ++i) u[i] = __fadd_rn(u[2 * i], u[2 * i + 1]);
  }
  return canon_zero(u[0] * 0.0625f);
}

// G == 1: 8 chains over k mod 8 (k = 8*t + l), then u_i = c_i + c_{i+4}, then (0+1)+(2+3).
template <>
__device__ __forceinline__ float ref_rotate_one<2>(const float* __restrict__ xs, int j) {
  float c[8];
#pragma unroll
  for (int l = 0; l < 8; ++l) c[l] = 0.0f;
#pragma unroll 4
  for (int t = 0; t < 32; ++t) {
#pragma unroll
    for (int l = 0; l < 8; ++l) {
      const int k = 8 * t + l;
      c[l] = __fmaf_rn(xs[k], hsign(j, k), c[l]);
    }
  }
  float u[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) u[i] = __fadd_rn(c[i], c[i + 4]);
  const float r = __fadd_rn(__fadd_rn(u[0], u[1]), __fadd_rn(u[2], u[3]));
  return canon_zero(r * 0.0625f);
}

__device__ __forceinline__ int ref_order_kind(int groups) {
  return groups >= 5 ? 0 : (groups >= 2 ? 1 : 2);
}

template <int ORDER_KIND>
__device__ __forceinline__ float ref_rotate_dispatch(const float* xs, int j) {
  return ref_rotate_one<ORDER_KIND>(xs, j);
}

__device__ __forceinline__ int8_t quant_code(float v, float scale) {
  const float t = __fdiv_rn(v, scale);   // IEEE division, as numpy's rotated / scale
  int q = __float2int_rn(t);             // rint: round half to even
  q = max(-128, min(127, q));
  return static_cast<int8_t>(q);
}

__device__ __forceinline__ float row_scale_from_absmax(float absmax) {
  return fmaxf(__fdiv_rn(absmax, 127.0f), 1e-30f);
}

// Block-wide max of non-negative floats; every thread gets the result.
__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red may still be read by a previous call
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float m = 0.0f;
  const int nw = (blockDim.x + 31) >> 5;
  for (int w = 0; w < nw; ++w) m = fmaxf(m, red[w]);
  return m;
}

// ------------------------------------------------------------------ reference order
// One CTA of 256 threads per row; thread j produces output j of every group.
// MODE 0: write rotated fp32. MODE 1: quantise (row kept in shared memory).
// LOAD: element loader; with DEQ the input is int8 codes times the row scale
// (slimdit/int8.py:58, q.astype(f32) * scale), rounded to fp32 before rotation.
template <int DT, bool DEQ, int MODE, int ORDER_KIND>
__global__ void __launch_bounds__(256) ref_rotate_kernel(const void* __restrict__ x,
                                                         const float* __restrict__ deq_scale,
                                                         int64_t rows, int K,
                                                         float* __restrict__ rot_out,
                                                         int8_t* __restrict__ q_out,
                                                         float* __restrict__ scale_out) {
  extern __shared__ __align__(16) float smem_f[];
  float* xs = smem_f;          // 256 inputs of the current group
  float* red = smem_f + 256;   // 32 warp partials
  float* rowbuf = smem_f + 288;  // K rotated values (MODE 1)
  const int j = threadIdx.x;
  const int groups = K >> 8;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const int64_t base = row * static_cast<int64_t>(K);
    float rs = 1.0f;
    if (DEQ) rs = __ldg(deq_scale + row);
    float amax = 0.0f;
    for (int g = 0; g < groups; ++g) {
      float v;
      if (DEQ) {
        v = static_cast<float>(__ldg(static_cast<const int8_t*>(x) + base + g * 256 + j)) * rs;
      } else {
        v = Loader<DT>::at(x, base + g * 256 + j);
      }
      __syncthreads();  // previous group's xs fully consumed
      xs[j] = v;
      __syncthreads();
      const float y = ref_rotate_dispatch<ORDER_KIND>(xs, j);
      if (MODE == 0) {
        rot_out[base + g * 256 + j] = y;
      } else {
        rowbuf[g * 256 + j] = y;
        amax = fmaxf(amax, fabsf(y));
      }
    }
    if (MODE == 1) {
      const float m = block_max(amax, red);  // includes the barrier making rowbuf visible
      const float scale = row_scale_from_absmax(m);
      if (j == 0) scale_out[row] = scale;
      // 4 codes per thread per step: coalesced 4-byte stores.
      for (int c = 4 * j; c < K; c += 4 * 256) {
        const float4 v = *reinterpret_cast<const float4*>(rowbuf + c);
        char4 o;
        o.x = quant_code(v.x, scale);
        o.y = quant_code(v.y, scale);
        o.z = quant_code(v.z, scale);
        o.w = quant_code(v.w, scale);
        *reinterpret_cast<char4*>(q_out + base + c) = o;
      }
    }
  }
}

// ------------------------------------------------------------------ butterfly order
// radix-4 butterfly on (a0,a1,a2,a3) in place.
__device__ __forceinline__ void bfly4(float& a0, float& a1, float& a2, float& a3) {
  const float s = __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
  const float b0 = __fmaf_rn(-2.0f, a3, s);
  const float b1 = __fmaf_rn(-2.0f, a2, s);
  const float b2 = __fmaf_rn(-2.0f, a1, s);
  const float b3 = __fmaf_rn(-2.0f, a0, s);
  a0 = b0; a1 = b1; a2 = b2; a3 = b3;
}

// Digits 0 and 1 of a 16-element chunk held in registers (index i = 4*d1 + d0).
__device__ __forceinline__ void bfly16(float (&v)[16]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) bfly4(v[4 * q + 0], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
#pragma unroll
  for (int m = 0; m < 4; ++m) bfly4(v[m], v[4 + m], v[8 + m], v[12 + m]);
}

constexpr int kGroupPad = 272;  // floats per group in the exchange buffer (256 + 16)

// Swizzled position of element (r, i) of a group in the exchange buffer: row r holds the
// 16 values of chunk r; float4 slots are XOR-permuted by (r>>1)&3 so both the row-wise
// float4 writes and the column-wise reads are bank-conflict free.
__device__ __forceinline__ int xpos(int r, int i) {
  return 16 * r + 4 * (((i >> 2) ^ (r >> 1)) & 3) + (i & 3);
}

// Butterfly rotate + quantise. One CTA per row, blockDim = 32 * ceil(K/512): thread t
// loads chunk t (16 consecutive elements), 16 threads per 256-group, 2 groups per warp.
// The digit-2/3 stages run on the transposed chunk after a warp-local shared exchange.
template <int DT>
__global__ void __launch_bounds__(1024) bfly_rotate_quant_kernel(const void* __restrict__ x,
                                                                 int64_t rows, int K,
                                                                 int8_t* __restrict__ q_out,
                                                                 float* __restrict__ scale_out,
                                                                 float* __restrict__ rot_out) {
  extern __shared__ __align__(16) float smem_f[];
  float* red = smem_f;                  // 32 floats
  float* xbuf = smem_f + 32;            // per warp: 2 groups * kGroupPad floats
  const int t = threadIdx.x;
  const int warp = t >> 5, lane = t & 31;
  const int gl = lane >> 4;             // group within the warp
  const int r = lane & 15;              // chunk within the group
  const int nchunks = K >> 4;
  const bool active = t < nchunks;
  float* gbuf = xbuf + (warp * 2 + gl) * kGroupPad;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const int64_t base = row * static_cast<int64_t>(K) + 16 * t;
    float v[16];
    if (active) {
      if (DT == kBF16) {
        const uint4* p = reinterpret_cast<const uint4*>(static_cast<const unsigned short*>(x) + base);
        const uint4 u0 = __ldg(p), u1 = __ldg(p + 1);
        const uint32_t w[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          v[2 * e] = __uint_as_float(w[e] << 16);
          v[2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
        }
      } else if (DT == kF32) {
        const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(x) + base);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float4 f = __ldg(p + e);
          v[4 * e] = f.x; v[4 * e + 1] = f.y; v[4 * e + 2] = f.z; v[4 * e + 3] = f.w;
        }
      } else {
        const uint4* p = reinterpret_cast<const uint4*>(static_cast<const __half*>(x) + base);
        const uint4 u0 = __ldg(p), u1 = __ldg(p + 1);
        const uint32_t w[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const __half2 h = *reinterpret_cast<const __half2*>(&w[e]);
          const float2 f = __half22float2(h);
          v[2 * e] = f.x; v[2 * e + 1] = f.y;
        }
      }
      bfly16(v);  // digits 0, 1
#pragma unroll
      for (int i = 0; i < 16; i += 4)
        *reinterpret_cast<float4*>(gbuf + xpos(r, i)) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    }
    __syncwarp();
    // transposed: this thread now owns column i' = r of its group, rows r' = 0..15
    if (active) {
#pragma unroll
      for (int rr = 0; rr < 16; ++rr) v[rr] = gbuf[xpos(rr, r)];
      bfly16(v);  // digits 2, 3 (rr = 4*d3 + d2)
    }
    float amax = 0.0f;
#pragma unroll
    for (int rr = 0; rr < 16; ++rr) {
      v[rr] *= 0.0625f;
      amax = fmaxf(amax, fabsf(v[rr]));
    }
    if (!active) amax = 0.0f;
    const float m = block_max(amax, red);
    const float scale = row_scale_from_absmax(m);
    if (t == 0) scale_out[row] = scale;
    if (rot_out != nullptr) {
      __syncwarp();
      if (active) {
#pragma unroll
        for (int rr = 0; rr < 16; ++rr) gbuf[xpos(rr, r)] = v[rr];
      }
      __syncwarp();
      if (active) {
        float* o = rot_out + base;
#pragma unroll
        for (int i = 0; i < 16; i += 4)
          *reinterpret_cast<float4*>(o + i) = *reinterpret_cast<const float4*>(gbuf + xpos(r, i));
      }
    }
    // codes: transpose back through shared memory as bytes, then one 16-byte store.
    __syncwarp();
    int8_t* cbuf = reinterpret_cast<int8_t*>(gbuf);
    if (active) {
#pragma unroll
      for (int rr = 0; rr < 16; ++rr) cbuf[16 * rr + r] = quant_code(v[rr], scale);
    }
    __syncwarp();
    if (active) {
      const uint4 c = *reinterpret_cast<const uint4*>(cbuf + 16 * r);
      *reinterpret_cast<uint4*>(q_out + base) = c;
    }
    __syncwarp();
  }
}

// ------------------------------------------------------------------ quantise-only
// Rows of already-rotated fp32 values -> codes + scales (slimdit/int8.py:49-51).
__global__ void __launch_bounds__(256) quantize_rows_kernel(const float* __restrict__ rot,
                                                            int64_t rows, int K,
                                                            int8_t* __restrict__ q_out,
                                                            float* __restrict__ scale_out) {
  __shared__ float red[32];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* p = rot + row * static_cast<int64_t>(K);
    float amax = 0.0f;
    for (int c = threadIdx.x; c < K; c += blockDim.x) amax = fmaxf(amax, fabsf(p[c]));
    const float m = block_max(amax, red);
    const float scale = row_scale_from_absmax(m);
    if (threadIdx.x == 0) scale_out[row] = scale;
    for (int c = threadIdx.x; c < K; c += blockDim.x)
      q_out[row * static_cast<int64_t>(K) + c] = quant_code(p[c], scale);
  }
}

// ------------------------------------------------------------------ launchers
static int grid_for_rows(int64_t rows, int per_sm) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t cap = static_cast<int64_t>(sms) * per_sm;
  return static_cast<int>(rows < cap ? rows : cap);
}

template <int DT, bool DEQ, int MODE>
static cudaError_t launch_ref(const void* x, const float* deq_scale, int64_t rows, int K,
                              float* rot_out, int8_t* q, float* scale, cudaStream_t st) {
  const int groups = K >> 8;
  const size_t smem = (288 + (MODE == 1 ? static_cast<size_t>(K) : 0)) * sizeof(float);
  const int kind = groups >= 5 ? 0 : (groups >= 2 ? 1 : 2);
  const int grid = grid_for_rows(rows, 8);
  void (*fn)(const void*, const float*, int64_t, int, float*, int8_t*, float*) =
      kind == 0 ? ref_rotate_kernel<DT, DEQ, MODE, 0>
                : (kind == 1 ? ref_rotate_kernel<DT, DEQ, MODE, 1> : ref_rotate_kernel<DT, DEQ, MODE, 2>);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  fn<<<grid, 256, smem, st>>>(x, deq_scale, rows, K, rot_out, q, scale);
  return cudaGetLastError();
}

cudaError_t launch_ref_rotate(const void* x, int dtype, int64_t rows, int K, float* out,
                              cudaStream_t st) {
  switch (dtype) {
    case kF32: return launch_ref<kF32, false, 0>(x, nullptr, rows, K, out, nullptr, nullptr, st);
    case kBF16: return launch_ref<kBF16, false, 0>(x, nullptr, rows, K, out, nullptr, nullptr, st);
    case kF16: return launch_ref<kF16, false, 0>(x, nullptr, rows, K, out, nullptr, nullptr, st);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_ref_rotate_quant(const void* x, int dtype, int64_t rows, int K, int8_t* q,
                                    float* scale, cudaStream_t st) {
  switch (dtype) {
    case kF32: return launch_ref<kF32, false, 1>(x, nullptr, rows, K, nullptr, q, scale, st);
    case kBF16: return launch_ref<kBF16, false, 1>(x, nullptr, rows, K, nullptr, q, scale, st);
    case kF16: return launch_ref<kF16, false, 1>(x, nullptr, rows, K, nullptr, q, scale, st);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_ref_dequant(const int8_t* q, const float* scale, int64_t rows, int K,
                               float* out, cudaStream_t st) {
  return launch_ref<kF32, true, 0>(q, scale, rows, K, out, nullptr, nullptr, st);
}

size_t bfly_smem_bytes(int K) {
  const int threads = ((K >> 4) + 31) / 32 * 32;
  return (32 + static_cast<size_t>(threads / 32) * 2 * kGroupPad) * sizeof(float);
}

cudaError_t launch_bfly_rotate_quant(const void* x, int dtype, int64_t rows, int K, int8_t* q,
                                     float* scale, float* rot_out, cudaStream_t st) {
  const int threads = ((K >> 4) + 31) / 32 * 32;
  const size_t smem = bfly_smem_bytes(K);
  const int per_sm = 2048 / threads > 0 ? 2048 / threads : 1;
  const int grid = grid_for_rows(rows, per_sm * 4);
  void (*fn)(const void*, int64_t, int, int8_t*, float*, float*) =
      dtype == kBF16 ? bfly_rotate_quant_kernel<kBF16>
                     : (dtype == kF32 ? bfly_rotate_quant_kernel<kF32> : bfly_rotate_quant_kernel<kF16>);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  fn<<<grid, threads, smem, st>>>(x, rows, K, q, scale, rot_out);
  return cudaGetLastError();
}

cudaError_t launch_quantize_rows(const float* rot, int64_t rows, int K, int8_t* q, float* scale,
                                 cudaStream_t st) {
  const int grid = grid_for_rows(rows, 8);
  quantize_rows_kernel<<<grid, 256, 0, st>>>(rot, rows, K, q, scale);
  return cudaGetLastError();
}

}  // namespace slim
