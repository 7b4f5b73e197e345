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
#include "slim_ptx.cuh"

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

// G >= 5: one sequential chain per output over k = 0..255, k = 16*b + l. The sign factorises
// as sigma(j, b) * lam(j, l); the accumulator is carried as sigma_b * acc so each step is one
// fma(x, lam_l, acc) (exact product, one rounding), and at a block change it is multiplied by
// sigma_b*sigma_{b-1} (an exact sign flip): fl(s*a + s*t) = s*fl(a + t) keeps this identical
// to the plain chain.
// Four outputs at once: j, j+64, j+128, j+192 (j < 64) share the base-4 digits j0..j2,
// so they share lam(l) and the digit-2 factor h4(j2, b&3) of the block sign; they differ only
// in the digit-3 factor H4[i][b>>2], i = 0..3, which is constant over each quad of blocks.
// Each accumulator is carried as (its block sign) * acc, so every step is one
// fma(x, lam_l, acc); at a block change all four are multiplied by
// h4(j2,b&3)*h4(j2,(b-1)&3), and at a quad change output i additionally by
// H4[i][B]*H4[i][B-1] (compile-time +-1). Same roundings as the plain chain; the x loads and
// lam are shared by four independent chains.
__device__ __forceinline__ void ref_rotate_four0(const float* __restrict__ xs, int j, float (&y)[4]) {
  const int j0 = j & 3, j1 = (j >> 2) & 3, j2 = (j >> 4) & 3;
  float lam[16];
#pragma unroll
  for (int l = 0; l < 16; ++l) lam[l] = h4sign(j1, l >> 2) * h4sign(j0, l & 3);
  float s2[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) s2[c] = h4sign(j2, c);
  const float4* x4 = reinterpret_cast<const float4*>(xs);
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int b = 0; b < 16; ++b) {
    if (b > 0) {
      const float f = s2[b & 3] * s2[(b - 1) & 3];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float g = f;
        if ((b & 3) == 0 && h4sign(i, b >> 2) != h4sign(i, (b >> 2) - 1)) g = -g;
        acc[i] *= g;
      }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 v = x4[b * 4 + q];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc[i] = __fmaf_rn(v.x, lam[4 * q + 0], acc[i]);
        acc[i] = __fmaf_rn(v.y, lam[4 * q + 1], acc[i]);
        acc[i] = __fmaf_rn(v.z, lam[4 * q + 2], acc[i]);
        acc[i] = __fmaf_rn(v.w, lam[4 * q + 3], acc[i]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float last = s2[3] * h4sign(i, 3);  // the block sign of block 15 for output i
    y[i] = canon_zero(acc[i] * last * 0.0625f);
  }
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

// Reference order for G >= 5 with four outputs per thread: one CTA of 256 threads per row
// handles four groups at a time (thread t: group slot t/64, outputs t%64 + 64*i).
template <int DT, bool DEQ, int MODE>
__global__ void __launch_bounds__(256) ref_rotate4_kernel(const void* __restrict__ x,
                                                          const float* __restrict__ deq_scale,
                                                          int64_t rows, int K,
                                                          float* __restrict__ rot_out,
                                                          int8_t* __restrict__ q_out,
                                                          float* __restrict__ scale_out) {
  extern __shared__ __align__(16) float smem_f[];
  float* xs = smem_f;            // 4 groups x 256 inputs
  float* red = smem_f + 1024;    // 32 warp partials
  float* rowbuf = smem_f + 1056; // K rotated values (MODE 1)
  const int t = threadIdx.x;
  const int slot = t >> 6, j = t & 63;
  const int groups = K >> 8;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const int64_t base = row * static_cast<int64_t>(K);
    float rs = 1.0f;
    if (DEQ) rs = __ldg(deq_scale + row);
    float amax = 0.0f;
    for (int g0 = 0; g0 < groups; g0 += 4) {
      const int ng = min(4, groups - g0);
      __syncthreads();  // previous groups' inputs fully consumed
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int idx = e * 256 + t;  // input idx of the 4-group window
        if (idx < ng * 256) {
          float v;
          if (DEQ) {
            v = static_cast<float>(__ldg(static_cast<const int8_t*>(x) + base + g0 * 256 + idx)) * rs;
          } else {
            v = Loader<DT>::at(x, base + g0 * 256 + idx);
          }
          xs[idx] = v;
        }
      }
      __syncthreads();
      if (slot < ng) {
        float y[4];
        ref_rotate_four0(xs + slot * 256, j, y);
        const int64_t o = base + (g0 + slot) * 256 + j;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (MODE == 0) {
            rot_out[o + 64 * i] = y[i];
          } else {
            rowbuf[(g0 + slot) * 256 + j + 64 * i] = y[i];
            amax = fmaxf(amax, fabsf(y[i]));
          }
        }
      }
    }
    if (MODE == 1) {
      const float m = block_max(amax, red);  // includes the barrier making rowbuf visible
      const float scale = row_scale_from_absmax(m);
      if (t == 0) scale_out[row] = scale;
      for (int c = 4 * t; c < K; c += 4 * 256) {
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

// Reference order for 5 <= G <= 64 with sixteen outputs per thread: thread t of a CTA (one row
// at a time) takes group t/16 and outputs jl + 16*i, i = 0..15, jl = t%16. With the base-4
// digits of j (j0, j1 from jl; a = j2 = i%4, c = j3 = i/4) the sign of term k = 16*b + l is
// lam(l) * sig16(i, b): lam(l) = H4[j1][l/4] * H4[j0][l%4] is the same for the thread's
// sixteen outputs, so each input loaded from shared memory feeds sixteen fused adds (the
// four-output kernel loads four times as often per add). Carrying each accumulator as
// sig16(i, b) * acc, as in ref_rotate_four0, every step is fma(x, lam, acc), and at block b the
// carried value is multiplied by sig16(i, b) * sig16(i, b-1). Outputs whose multipliers have
// been equal at every block change so far hold equal carried accumulators, so one chain serves
// them: rep16(i, b) names the output whose chain output i shares during block b (H4 has -1
// exactly where the digits sum to 3, which gives one chain in block 0, two in block 1, four in
// blocks 2-3, eight in 4-7 and sixteen from 8 on: 2,736 fused adds per sixteen outputs instead
// of 4,096). Each output still sees exactly the operations of its own sequential chain.
__host__ __device__ constexpr int rep16(int i, int b) {
  return b == 0 ? 0
         : b == 1 ? ((i & 3) < 2 ? 0 : 2)
         : b < 4 ? (i & 3)
         : b < 8 ? (i & 3) + 4 * ((i >> 2) < 2 ? 0 : 2)
         : i;
}

__device__ __forceinline__ float sig16(int i, int b) { return h4sign(i & 3, b & 3) * h4sign(i >> 2, b >> 2); }

// Compile-time twins of h4sign / sig16 for the per-block template below.
__host__ __device__ constexpr float h4c(int a, int b) { return (a + b == 3) ? -1.0f : 1.0f; }
__host__ __device__ constexpr float sig16c(int i, int b) { return h4c(i & 3, b & 3) * h4c(i >> 2, b >> 2); }

// Block B of the sixteen carried chains: the class split / sign change at entry, then sixteen
// steps, pairs (2p, 2p+1) that are both chains advancing with one packed fp32x2 fma.
template <int B>
__device__ __forceinline__ void chain16_block(const float4* __restrict__ x4, const float (&lam)[16],
                                              float (&acc)[16]) {
  if constexpr (B > 0) {
    float old[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) old[i] = acc[i];
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (rep16(i, B) == i) acc[i] = old[rep16(i, B - 1)] * (sig16c(i, B) * sig16c(i, B - 1));
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 v = x4[B * 4 + q];
    const float xv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float lv = lam[4 * q + e];
#pragma unroll
      for (int pr = 0; pr < 8; ++pr) {
        const int i0 = 2 * pr, i1 = 2 * pr + 1;
        const bool r0 = rep16(i0, B) == i0, r1 = rep16(i1, B) == i1;
        if (r0 && r1) {
          const float2 r = fma2(make_float2(xv[e], xv[e]), make_float2(lv, lv), make_float2(acc[i0], acc[i1]));
          acc[i0] = r.x;
          acc[i1] = r.y;
        } else if (r0) {
          acc[i0] = __fmaf_rn(xv[e], lv, acc[i0]);
        } else if (r1) {
          acc[i1] = __fmaf_rn(xv[e], lv, acc[i1]);
        }
      }
    }
  }
}

template <int B>
struct Chain16 {
  __device__ __forceinline__ static void run(const float4* __restrict__ x4, const float (&lam)[16], float (&acc)[16]) {
    chain16_block<B>(x4, lam, acc);
    Chain16<B + 1>::run(x4, lam, acc);
  }
};
template <>
struct Chain16<16> {
  __device__ __forceinline__ static void run(const float4*, const float (&)[16], float (&)[16]) {}
};

// A thread's 16 consecutive inputs of a row (raw words: bf16/f16 2 x 16 B, fp32 4 x 16 B,
// int8 codes 16 B), loaded one row ahead and written to shared memory as fp32 after the row
// in flight is done.
template <int DT, bool DEQ>
struct Row16 {
  static constexpr int kWords = DEQ ? 1 : (DT == kF32 ? 4 : 2);
  uint4 w[kWords];
  float rs;
  __device__ __forceinline__ void load(const void* x, const float* deq_scale, int64_t row, int K, int t) {
    const int64_t e0 = row * static_cast<int64_t>(K) + 16 * t;
    const uint4* p = reinterpret_cast<const uint4*>(static_cast<const unsigned char*>(x) +
                                                     e0 * (DEQ ? 1 : (DT == kF32 ? 4 : 2)));
#pragma unroll
    for (int i = 0; i < kWords; ++i) w[i] = __ldg(p + i);
    rs = DEQ ? __ldg(deq_scale + row) : 1.0f;
  }
  __device__ __forceinline__ void store(float* dst) const {
    float f[16];
    if (DEQ) {
      const uint32_t u[4] = {w[0].x, w[0].y, w[0].z, w[0].w};
#pragma unroll
      for (int i = 0; i < 16; ++i)
        f[i] = static_cast<float>(static_cast<int8_t>((u[i >> 2] >> (8 * (i & 3))) & 0xffu)) * rs;
    } else if (DT == kF32) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        f[4 * i] = __uint_as_float(w[i].x); f[4 * i + 1] = __uint_as_float(w[i].y);
        f[4 * i + 2] = __uint_as_float(w[i].z); f[4 * i + 3] = __uint_as_float(w[i].w);
      }
    } else {
      const uint32_t u[8] = {w[0].x, w[0].y, w[0].z, w[0].w, w[1].x, w[1].y, w[1].z, w[1].w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (DT == kBF16) {
          f[2 * i] = __uint_as_float(u[i] << 16);
          f[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
        } else {
          const float2 h = __half22float2(*reinterpret_cast<const __half2*>(&u[i]));
          f[2 * i] = h.x; f[2 * i + 1] = h.y;
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 16; i += 4) *reinterpret_cast<float4*>(dst + i) = make_float4(f[i], f[i + 1], f[i + 2], f[i + 3]);
  }
};

template <int DT, bool DEQ, int MODE>
__global__ void __launch_bounds__(1024) ref_rotate16_kernel(const void* __restrict__ x,
                                                           const float* __restrict__ deq_scale,
                                                           int64_t rows, int K,
                                                           float* __restrict__ rot_out,
                                                           int8_t* __restrict__ q_out,
                                                           float* __restrict__ scale_out) {
  extern __shared__ __align__(16) float smem_f[];  // two rows of K fp32 inputs
  __shared__ float red[2][32];                     // warp maxima, by row parity
  const int t = threadIdx.x;
  const int g = t >> 4, jl = t & 15;
  const int groups = K >> 8;
  const bool active = g < groups;  // whole warps only: the threads past the last group idle
  float lam[16];
#pragma unroll
  for (int l = 0; l < 16; ++l) lam[l] = h4sign(jl >> 2, l >> 2) * h4sign(jl & 3, l & 3);
  int64_t row = blockIdx.x;
  if (row >= rows) return;  // uniform over the CTA
  Row16<DT, DEQ> nxt;
  if (active) {
    nxt.load(x, deq_scale, row, K, t);
    nxt.store(smem_f + 16 * t);
  }
  __syncthreads();
  int buf = 0;
  for (; row < rows; row += gridDim.x) {
    const int64_t base = row * static_cast<int64_t>(K);
    const int64_t next = row + gridDim.x;
    const bool have_next = next < rows;
    if (active && have_next) nxt.load(x, deq_scale, next, K, t);  // lands while this row computes
    const float* xs = smem_f + buf * K;
    float y[16];
    float amax = 0.0f;
    if (active) {
      const float4* x4 = reinterpret_cast<const float4*>(xs + g * 256);
      float acc[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[i] = 0.0f;
      Chain16<0>::run(x4, lam, acc);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        y[i] = canon_zero(acc[i] * sig16(i, 15) * 0.0625f);  // the block sign of block 15
        amax = fmaxf(amax, fabsf(y[i]));
      }
    }
    const int64_t o = base + g * 256 + jl;
    if (MODE == 1) {
      const unsigned wm = __reduce_max_sync(0xffffffffu, __float_as_uint(amax));  // amax >= 0
      if ((t & 31) == 0) red[buf][t >> 5] = __uint_as_float(wm);
    }
    if (active && have_next) nxt.store(smem_f + (buf ^ 1) * K + 16 * t);
    // one barrier per row: the warp maxima are visible, the next row is staged, and this row's
    // inputs are no longer read (red[buf] is written again two rows later, after the next one)
    __syncthreads();
    if (MODE == 0) {
      if (active) {
#pragma unroll
        for (int i = 0; i < 16; ++i) rot_out[o + 16 * i] = y[i];
      }
    } else {
      const int nw = (blockDim.x + 31) >> 5;
      const int lane = t & 31;
      const float m = __uint_as_float(__reduce_max_sync(0xffffffffu, lane < nw ? __float_as_uint(red[buf][lane]) : 0u));
      const float scale = row_scale_from_absmax(m);
      if (t == 0) scale_out[row] = scale;
      if (active) {
#pragma unroll
        for (int i = 0; i < 16; ++i) q_out[o + 16 * i] = quant_code(y[i], scale);
      }
    }
    buf ^= 1;
  }
}

// ------------------------------------------------------------------ butterfly, packed pairs
// Packed fp32x2 arithmetic: add2 / mul2 / fma2 (slim_ptx.cuh).

// bfly4 on pairs: b_i = ((a0 + a1) + (a2 + a3)) - 2*a_{3-i} in each lane.
__device__ __forceinline__ void bfly4x2(float2& a0, float2& a1, float2& a2, float2& a3) {
  const float2 m2 = make_float2(-2.0f, -2.0f);
  const float2 s = add2(add2(a0, a1), add2(a2, a3));
  const float2 b0 = fma2(m2, a3, s), b1 = fma2(m2, a2, s), b2 = fma2(m2, a1, s), b3 = fma2(m2, a0, s);
  a0 = b0; a1 = b1; a2 = b2; a3 = b3;
}

__device__ __forceinline__ void bfly16x2(float2 (&v)[16]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) bfly4x2(v[4 * q + 0], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
#pragma unroll
  for (int m = 0; m < 4; ++m) bfly4x2(v[m], v[4 + m], v[8 + m], v[12 + m]);
}

// Exchange buffer of one group pair: 16 rows (chunks) x 16 float2; 16-byte slots of a row
// are XOR-permuted by the row index so both the row-wise 16-byte writes and the
// column-wise 8-byte reads are free of bank conflicts.
__device__ __forceinline__ int xpos2(int row, int col) {  // in float2 units
  return 16 * row + 2 * ((col >> 1) ^ (row & 7)) + (col & 1);
}

// Quantise a pair of unscaled butterfly sums S (rotated value v = S/16, exact) with
// scale = max(fl(fl(max|v|)/127), 1e-30): code = clamp(rint(fl(v / scale)), -128, 127),
// the same result as slimdit/int8.py:51.
// Fast path: t = S * r16 with r16 = fl(1/(16*scale)); |t - fl(v/scale)| <= 1.5*2^-23*|t| <
// 2.3e-5 for |t| <= 128, so rint(t) is rint(fl(v/scale)) unless t lies within 2^-13 of a
// half-integer; those set `slow` and the caller redoes the pair with the IEEE division
// (about 2.4e-4 of random elements). rint(t) is taken with the 1.5*2^23 magic constant,
// whose float bit pattern then holds the code in its low byte. Rows whose maximum is tiny
// (S/16 could be subnormal) always take the exact path.
// Returns the two codes packed into the low 16 bits (lane x in bits 0-7).
__device__ __forceinline__ uint32_t quant_pair(float2 S, float2 r16x2, float scale, bool& slow) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  const float2 t = mul2(S, r16x2);
  const float2 x = add2(t, make_float2(kMagic, kMagic));
  const float2 r = add2(x, make_float2(-kMagic, -kMagic));
  const float2 d = add2(t, make_float2(-r.x, -r.y));
  slow |= fabsf(d.x) > 0.5f - 1.220703125e-4f;
  slow |= fabsf(d.y) > 0.5f - 1.220703125e-4f;
  (void)scale;
  return __byte_perm(__float_as_uint(x.x), __float_as_uint(x.y), 0x0040);
}

// Butterfly rotate + quantise with packed pairs, persistent over rows. A row of G groups is
// split into G2 = ceil(G/2) group pairs (g, g + G2); 16 threads per pair, thread (p, r)
// owns chunk r (16 consecutive elements) of both groups and carries them as the two lanes
// of float2 registers through all four radix-4 stages. Rows are staged into shared memory by
// double-buffered bulk copies. One block barrier per row (partial maxima double-buffered).
// MAXR: 88 registers in general; 72 for rows of 48+ groups (K >= 12288), whose 384+ threads
// per block would otherwise leave room for only one block (one row in flight) per SM.
template <int DT, int MAXR>
__global__ void __maxnreg__(MAXR) bfly2_rotate_quant_kernel(const void* __restrict__ x,
                                                                 int64_t rows, int K,
                                                                 int8_t* __restrict__ q_out,
                                                                 float* __restrict__ scale_out,
                                                                 float* __restrict__ rot_out) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  constexpr int kEsz = DT == kF32 ? 4 : 2;
  const uint32_t row_bytes = static_cast<uint32_t>(K) * kEsz;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem_raw);                 // 2 mbarriers
  float* red = reinterpret_cast<float*>(smem_raw + 16);                  // 2 x 32 partial maxima
  unsigned char* rowbuf = smem_raw + 272;                                // 2 staged rows
  float2* xbuf = reinterpret_cast<float2*>(rowbuf + 2 * static_cast<size_t>(row_bytes));
  const int t = threadIdx.x;
  const int warp = t >> 5, lane = t & 31;
  const int G = K >> 8;
  const int G2 = (G + 1) >> 1;
  const int p = t >> 4;                 // group pair
  const int r = t & 15;                 // chunk within the group
  const bool act_a = p < G2;
  const bool act_b = p + G2 < G;
  float2* gbuf = xbuf + (warp * 2 + ((lane >> 4) & 1)) * 256;
  const int nw = (blockDim.x + 31) >> 5;
  const unsigned char* src = static_cast<const unsigned char*>(x);

  if (t == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  int64_t row = blockIdx.x;
  uint32_t pending = 0, pending_parity = 0;
  if (t == 0) {
    for (int b = 0; b < 2; ++b) {
      const int64_t rb = row + b * static_cast<int64_t>(gridDim.x);
      if (rb < rows) {
        mbar_arrive_expect_tx(&bar[b], row_bytes);
        bulk_load(rowbuf + b * row_bytes, src + rb * row_bytes, row_bytes, &bar[b]);
        pending |= 1u << b;
      }
    }
  }
  for (int it = 0; row < rows; row += gridDim.x, ++it) {
    const int b = it & 1;
    const bool ok = mbar_wait(&bar[b], (it >> 1) & 1, kErrWaitTimeoutProducer);
    if (ok && t == 0) pending &= ~(1u << b);
    if (__syncthreads_or(!ok)) break;  // a staged row never arrived: stop (error recorded)
    const unsigned char* stage = rowbuf + b * row_bytes;
    const int ea = (p * 256 + 16 * r);            // element offset of chunk a in the row
    const int eb = ea + G2 * 256;                 // chunk b
    float2 v[16];
    if (act_a) {
      float fa[16], fb[16];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int e0 = h == 0 ? ea : eb;
        float* f = h == 0 ? fa : fb;
        if (h == 1 && !act_b) {
#pragma unroll
          for (int i = 0; i < 16; ++i) f[i] = 0.0f;
          continue;
        }
        if (DT == kF32) {
          const float4* q4 = reinterpret_cast<const float4*>(stage + 4 * e0);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float4 g = q4[e];
            f[4 * e] = g.x; f[4 * e + 1] = g.y; f[4 * e + 2] = g.z; f[4 * e + 3] = g.w;
          }
        } else {
          const uint4* q4 = reinterpret_cast<const uint4*>(stage + 2 * e0);
          const uint4 u0 = q4[0], u1 = q4[1];
          const uint32_t w[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            if (DT == kBF16) {
              f[2 * e] = __uint_as_float(w[e] << 16);
              f[2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
            } else {
              const float2 hf = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
              f[2 * e] = hf.x; f[2 * e + 1] = hf.y;
            }
          }
        }
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = make_float2(fa[i], fb[i]);
      bfly16x2(v);  // digits 0, 1
#pragma unroll
      for (int i = 0; i < 16; i += 2)
        *reinterpret_cast<float4*>(gbuf + xpos2(r, i)) = make_float4(v[i].x, v[i].y, v[i + 1].x, v[i + 1].y);
    }
    __syncwarp();
    float amax = 0.0f;
    if (act_a) {
#pragma unroll
      for (int rr = 0; rr < 16; ++rr) v[rr] = gbuf[xpos2(rr, r)];
      bfly16x2(v);  // digits 2, 3; lanes hold the unscaled sums S = 16 * rotated
#pragma unroll
      for (int rr = 0; rr < 16; ++rr) amax = fmaxf(amax, fmaxf(fabsf(v[rr].x), fabsf(v[rr].y)));
    }
    // row maximum: one redux per warp, one block barrier, every warp finishes the reduction
    float* redp = red + 32 * b;
    const unsigned wmax = __reduce_max_sync(0xffffffffu, __float_as_uint(amax));
    if (lane == 0) redp[warp] = __uint_as_float(wmax);
    __syncthreads();
    const float amax_s =
        __uint_as_float(__reduce_max_sync(0xffffffffu, lane < nw ? __float_as_uint(redp[lane]) : 0u));
    // every thread has read this row's stage: refill the buffer with the row after next
    if (t == 0) {
      const int64_t rn = row + 2 * static_cast<int64_t>(gridDim.x);
      if (rn < rows) {
        mbar_arrive_expect_tx(&bar[b], row_bytes);
        bulk_load(rowbuf + b * row_bytes, src + rn * row_bytes, row_bytes, &bar[b]);
        pending |= 1u << b;
        pending_parity = (pending_parity & ~(1u << b)) | ((((it + 2) >> 1) & 1u) << b);
      }
    }
    const float scale = row_scale_from_absmax(__fmul_rn(amax_s, 0.0625f));
    const float r16 = __frcp_rn(__fmul_rn(16.0f, scale));
    const bool tiny_row = amax_s < 8.271806125530277e-25f;  // 2^-80
    if (t == 0) scale_out[row] = scale;
    const int64_t rbase = row * static_cast<int64_t>(K);
    if (rot_out != nullptr) {
      __syncwarp();
      if (act_a) {
        const float2 s16 = make_float2(0.0625f, 0.0625f);
#pragma unroll
        for (int rr = 0; rr < 16; ++rr) gbuf[xpos2(rr, r)] = mul2(v[rr], s16);
      }
      __syncwarp();
      if (act_a) {
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          const float4 w4 = *reinterpret_cast<const float4*>(gbuf + xpos2(r, i));
          *reinterpret_cast<float2*>(rot_out + rbase + ea + i) = make_float2(w4.x, w4.z);
          if (act_b) *reinterpret_cast<float2*>(rot_out + rbase + eb + i) = make_float2(w4.y, w4.w);
        }
      }
    }
    // codes: pairs packed to 16 bits, transposed back through shared memory, de-interleaved
    __syncwarp();
    uint16_t* cbuf = reinterpret_cast<uint16_t*>(gbuf);
    if (act_a) {
      bool slow = tiny_row;
      uint32_t c2[16];
      const float2 r2 = make_float2(r16, r16);
#pragma unroll
      for (int rr = 0; rr < 16; ++rr) c2[rr] = quant_pair(v[rr], r2, scale, slow);
      if (slow) {
#pragma unroll
        for (int rr = 0; rr < 16; ++rr) {
          const int8_t ca = quant_code(__fmul_rn(v[rr].x, 0.0625f), scale);
          const int8_t cb = quant_code(__fmul_rn(v[rr].y, 0.0625f), scale);
          c2[rr] = (static_cast<uint32_t>(static_cast<uint8_t>(cb)) << 8) | static_cast<uint8_t>(ca);
        }
      }
#pragma unroll
      for (int rr = 0; rr < 16; ++rr) cbuf[16 * rr + r] = static_cast<uint16_t>(c2[rr]);
    }
    __syncwarp();
    if (act_a) {
      const uint4* c4 = reinterpret_cast<const uint4*>(cbuf + 16 * r);
      const uint4 u0 = c4[0], u1 = c4[1];  // 16 (a, b) byte pairs of chunk r
      uint4 oa, ob;
      oa.x = __byte_perm(u0.x, u0.y, 0x6420); ob.x = __byte_perm(u0.x, u0.y, 0x7531);
      oa.y = __byte_perm(u0.z, u0.w, 0x6420); ob.y = __byte_perm(u0.z, u0.w, 0x7531);
      oa.z = __byte_perm(u1.x, u1.y, 0x6420); ob.z = __byte_perm(u1.x, u1.y, 0x7531);
      oa.w = __byte_perm(u1.z, u1.w, 0x6420); ob.w = __byte_perm(u1.z, u1.w, 0x7531);
      *reinterpret_cast<uint4*>(q_out + rbase + ea) = oa;
      if (act_b) *reinterpret_cast<uint4*>(q_out + rbase + eb) = ob;
    }
    __syncwarp();
  }
  if (t == 0) {
    for (int b = 0; b < 2; ++b)
      if (pending & (1u << b)) mbar_wait(&bar[b], (pending_parity >> b) & 1u, kErrWaitTimeoutDrain);
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
  const int kind = groups >= 5 ? 0 : (groups >= 2 ? 1 : 2);
  // sixteen outputs per thread for rows of up to 64 groups read with 16-byte vector loads (the
  // four-output kernel takes longer rows and inputs that are not 16-byte aligned)
  if (kind == 0 && groups <= 64 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0) {
    const int threads = (16 * groups + 31) / 32 * 32;
    const size_t smem16 = 2 * static_cast<size_t>(K) * sizeof(float);
    auto fn16 = ref_rotate16_kernel<DT, DEQ, MODE>;
    static PerDeviceOnce smem_once;
    int dev = 0;
    cudaGetDevice(&dev);
    cudaError_t e = smem_once.run(dev, [&] {
      return cudaFuncSetAttribute(fn16, cudaFuncAttributeMaxDynamicSharedMemorySize, 128 * 1024);
    });
    if (e != cudaSuccess) return e;
    int per_sm = 1;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn16, threads, smem16);
    if (e != cudaSuccess) return e;
    const int grid16 = grid_for_rows(rows, per_sm < 1 ? 1 : per_sm);
    fn16<<<grid16, threads, smem16, st>>>(x, deq_scale, rows, K, rot_out, q, scale);
    return cudaGetLastError();
  }
  if (kind == 0) {
    const size_t smem4 = (1056 + (MODE == 1 ? static_cast<size_t>(K) : 0)) * sizeof(float);
    auto fn4 = ref_rotate4_kernel<DT, DEQ, MODE>;
    if (smem4 > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(fn4, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem4));
      if (e != cudaSuccess) return e;
    }
    int per_sm = 1;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn4, 256, smem4);
    if (e != cudaSuccess) return e;
    const int grid4 = grid_for_rows(rows, per_sm < 1 ? 1 : per_sm);
    fn4<<<grid4, 256, smem4, st>>>(x, deq_scale, rows, K, rot_out, q, scale);
    return cudaGetLastError();
  }
  const size_t smem = (288 + (MODE == 1 ? static_cast<size_t>(K) : 0)) * sizeof(float);
  const int grid = grid_for_rows(rows, 8);
  void (*fn)(const void*, const float*, int64_t, int, float*, int8_t*, float*) =
      kind == 1 ? ref_rotate_kernel<DT, DEQ, MODE, 1> : ref_rotate_kernel<DT, DEQ, MODE, 2>;
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

size_t bfly_smem_bytes(int K, int dtype) {
  const int g2 = ((K >> 8) + 1) >> 1;
  const int threads = (g2 + 1) / 2 * 32;
  const size_t esz = dtype == kF32 ? 4 : 2;
  return 272 + 2 * esz * static_cast<size_t>(K) + static_cast<size_t>(threads / 32) * 2 * 256 * sizeof(float2);
}

cudaError_t launch_bfly_rotate_quant(const void* x, int dtype, int64_t rows, int K, int8_t* q,
                                     float* scale, float* rot_out, cudaStream_t st) {
  const int g2 = ((K >> 8) + 1) >> 1;
  const int threads = (g2 + 1) / 2 * 32;
  const size_t smem = bfly_smem_bytes(K, dtype);
  void (*fn)(const void*, int64_t, int, int8_t*, float*, float*);
  if (threads >= 384)
    fn = dtype == kBF16 ? bfly2_rotate_quant_kernel<kBF16, 72>
                        : (dtype == kF32 ? bfly2_rotate_quant_kernel<kF32, 72> : bfly2_rotate_quant_kernel<kF16, 72>);
  else
    fn = dtype == kBF16 ? bfly2_rotate_quant_kernel<kBF16, 88>
                        : (dtype == kF32 ? bfly2_rotate_quant_kernel<kF32, 88> : bfly2_rotate_quant_kernel<kF16, 88>);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  int per_sm = 1;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  const int grid = grid_for_rows(rows, per_sm);
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
