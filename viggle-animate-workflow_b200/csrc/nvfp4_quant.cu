// NVFP4 quantisation: E2M1 codes in 16-element blocks along K with UE4M3 block scales and an
// fp32 global scale, the format of slimdit/nvfp4.py (weight, weight_scale, weight_scale_2;
// slimdit/nvfp4.py:3-8, docs/DEV_NOTES.md:59-71).
//
// The recipe (the reference delegates it to comfy_kitchen, slimdit/nvfp4.py:44-51,72-87):
//   global  gs = fl32(amax / 2688)                       (2688 = 448 * 6)
//   block   sf = e4m3_rne(min(fl32(fl32(block_amax / 6) / gs), 448))
//   element v  = fl32(x / fl32(gs * float(sf)))  (0 when that product is 0)
//           code = E2M1 round-half-even of v, saturating at 6, sign bit kept (0b1000 for
//                  negative values that round to zero)
// Every division is IEEE (div.rn); the E4M3 rounding is the hardware cvt.rn.satfinite.
// Packing: element 2i in the HIGH nibble of byte i, element 2i+1 in the low nibble: "two E2M1
// values per byte, high nibble first", the on-disk layout of slimdit/nvfp4.py:5 and
// docs/DEV_NOTES.md:64. The codes are formed low nibble first (the order of the hardware
// conversion) and swapped within each byte on the way out. The FP4 GEMM reads both of its
// operands in this order: swapping the two elements of every byte in both A and B permutes K
// identically on both sides, inside each 16-element scale block, so the sums are unchanged.
// Block scales are written in the cuBLAS 128x4 tiled layout: scale (r, c) of a matrix with
// C = K/16 scale columns lives at ((r/128)*(C/4) + c/4)*512 + (r%32)*16 + ((r%128)/32)*4 + c%4.
//
// Weights use one global scale per tensor (amax pass first); activations use one per token
// row (per-row amax inside the quantiser), optionally after the group-256 Hadamard rotation
// in the butterfly order of the INT8 path (bit-identical rotated values).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <algorithm>
#include <cstdint>

#include "slim_kernels.h"
#include "slim_ptx.cuh"

namespace slim {
namespace nvf4q {

__device__ __forceinline__ int64_t blocked_offset(int64_t row, int c, int ctiles) {
  return ((row >> 7) * ctiles + (c >> 2)) * 512 + (row & 31) * 16 + ((row >> 5) & 3) * 4 + (c & 3);
}

// Exact value of a UE4M3 byte (0..0x7E).
__device__ __forceinline__ float e4m3_value(uint32_t b) {
  const uint32_t e = (b >> 3) & 15u, m = b & 7u;
  return e == 0 ? static_cast<float>(m) * 0.001953125f : __uint_as_float(((e + 120u) << 23) | (m << 20));
}

__device__ __forceinline__ uint32_t e4m3_rne(float s) {
  return static_cast<uint32_t>(__nv_cvt_float_to_fp8(s, __NV_SATFINITE, __NV_E4M3));
}

// E2M1 code of v (round half to even on |v|, saturating at 6; sign in bit 3).
__device__ __forceinline__ uint32_t e2m1_code(float v) {
  const float a = fabsf(v);
  const uint32_t c = static_cast<uint32_t>(a > 0.25f) + static_cast<uint32_t>(a >= 0.75f) +
                     static_cast<uint32_t>(a > 1.25f) + static_cast<uint32_t>(a >= 1.75f) +
                     static_cast<uint32_t>(a > 2.5f) + static_cast<uint32_t>(a >= 3.5f) +
                     static_cast<uint32_t>(a > 5.0f);
  return c | ((__float_as_uint(v) >> 28) & 8u);
}

// Exchanges the two nibbles of every byte (low-first <-> high-first packing; an involution).
__device__ __forceinline__ uint32_t nibble_swap(uint32_t w) {
  return ((w & 0x0f0f0f0fu) << 4) | ((w >> 4) & 0x0f0f0f0fu);
}

// Eight values -> eight E2M1 codes in one word, value i in nibble i (value 2i in the low nibble
// of byte i): the hardware conversion rounds to the nearest grid point and saturates at 6 (ties
// never reach it, see below); the sign is the value's.
__device__ __forceinline__ uint32_t e2m1x8(float a0, float a1, float a2, float a3, float a4, float a5, float a6,
                                           float a7) {
  uint32_t r;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(r)
      : "f"(a0), "f"(a1), "f"(a2), "f"(a3), "f"(a4), "f"(a5), "f"(a6), "f"(a7));
  return r;
}

// One 16-element block -> 8 packed bytes (high nibble first) and its scale byte: quant_block16
// for one block; block_scale + block_codes2 for two blocks in the lanes of packed registers.
// The element quotient v = fl(x / total) is not formed. With r = fl(1/total), the products
// hi = fl(x * fl(r (1 + 2^-19))) and lo = fl(x * fl(r (1 - 2^-19))) bracket v in magnitude
// (three roundings move each by at most 3 * 2^-24 relative, well inside the 2^-19 offset), and
// the E2M1 code is monotone in |v| with the sign apart, so where the codes of hi and lo agree
// they are v's code. Where they differ (v within ~2^-19 of a rounding boundary, including every
// exact tie: about 1e-5 of the elements) the IEEE division decides; so does every element of a
// block whose reciprocal is not finite. The sign is x's (a zero quotient keeps x's sign, as
// the division's).

// Scale byte, element divisor and bracketing reciprocals of one block from its absmax bm; bad =
// every code of the block must come from the IEEE division.
struct BlockScale {
  uint32_t sfb;
  float total, rh, rl;
  bool bad;
};

__device__ __forceinline__ BlockScale block_scale(float bm, float gs) {
  BlockScale s;
  s.sfb = 0;
  if (gs > 0.0f) s.sfb = e4m3_rne(fminf(__fdiv_rn(__fdiv_rn(bm, 6.0f), gs), 448.0f));
  s.total = __fmul_rn(gs, e4m3_value(s.sfb));
  const float rcp = s.total != 0.0f ? __frcp_rn(s.total) : 0.0f;
  s.bad = !(rcp <= 3.402823466e38f);
  s.rh = __fmul_rn(rcp, 1.0f + 1.9073486328125e-6f);
  s.rl = __fmul_rn(rcp, 1.0f - 1.9073486328125e-6f);
  return s;
}

// Replaces the codes of the flagged elements (bits of d) of one block with the IEEE division's.
__device__ __forceinline__ void block_fixup(const float2 (&v)[16], bool lane_y, float total, uint32_t (&w)[2],
                                            const uint32_t (&d)[2]) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint32_t sh = 4 * (i & 7);
    if ((d[i >> 3] >> sh) & 15u) {
      const uint32_t code = e2m1_code(__fdiv_rn(lane_y ? v[i].y : v[i].x, total));
      w[i >> 3] = (w[i >> 3] & ~(15u << sh)) | (code << sh);
    }
  }
}

// Codes of a thread's two blocks (lane x: block a, lane y: block b) from the bracketing
// products, eight element pairs at a time; the IEEE division where they disagree; 0 where the
// divisor is 0. Packed high nibble first.
__device__ __forceinline__ void block_codes2(const float2 (&v)[16], const BlockScale& sa, const BlockScale& sb,
                                             uint2& pa, uint2& pb) {
  const float2 rh = make_float2(sa.rh, sb.rh), rl = make_float2(sa.rl, sb.rl);
  uint32_t wa[2], wb[2], da[2], db[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float2 th[8], tl[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      th[j] = mul2(v[8 * h + j], rh);
      tl[j] = mul2(v[8 * h + j], rl);
    }
    wa[h] = e2m1x8(th[0].x, th[1].x, th[2].x, th[3].x, th[4].x, th[5].x, th[6].x, th[7].x);
    da[h] = wa[h] ^ e2m1x8(tl[0].x, tl[1].x, tl[2].x, tl[3].x, tl[4].x, tl[5].x, tl[6].x, tl[7].x);
    wb[h] = e2m1x8(th[0].y, th[1].y, th[2].y, th[3].y, th[4].y, th[5].y, th[6].y, th[7].y);
    db[h] = wb[h] ^ e2m1x8(tl[0].y, tl[1].y, tl[2].y, tl[3].y, tl[4].y, tl[5].y, tl[6].y, tl[7].y);
  }
  if (sa.bad) da[0] = da[1] = 0xffffffffu;
  if (sb.bad) db[0] = db[1] = 0xffffffffu;
  if (sa.total == 0.0f) {
    wa[0] = wa[1] = 0u;
  } else if ((da[0] | da[1]) != 0u) {
    block_fixup(v, false, sa.total, wa, da);
  }
  if (sb.total == 0.0f) {
    wb[0] = wb[1] = 0u;
  } else if ((db[0] | db[1]) != 0u) {
    block_fixup(v, true, sb.total, wb, db);
  }
  pa = make_uint2(nibble_swap(wa[0]), nibble_swap(wa[1]));
  pb = make_uint2(nibble_swap(wb[0]), nibble_swap(wb[1]));
}

__device__ __forceinline__ void quant_block16(const float (&v)[16], float gs, uint2& packed, uint32_t& sfb) {
  float bm = 0.0f;
#pragma unroll
  for (int i = 0; i < 16; ++i) bm = fmaxf(bm, fabsf(v[i]));
  sfb = 0;
  if (gs > 0.0f) {
    const float s2 = fminf(__fdiv_rn(__fdiv_rn(bm, 6.0f), gs), 448.0f);
    sfb = e4m3_rne(s2);
  }
  const float total = __fmul_rn(gs, e4m3_value(sfb));
  uint32_t w[2] = {0u, 0u};
  if (total != 0.0f) {
    const float rcp = __frcp_rn(total);
    uint32_t d[2] = {0xffffffffu, 0xffffffffu};
    if (rcp <= 3.402823466e38f) {
      const float rh = __fmul_rn(rcp, 1.0f + 1.9073486328125e-6f);
      const float rl = __fmul_rn(rcp, 1.0f - 1.9073486328125e-6f);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float2 th[4], tl[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 x2 = make_float2(v[8 * h + 2 * j], v[8 * h + 2 * j + 1]);
          th[j] = mul2(x2, make_float2(rh, rh));
          tl[j] = mul2(x2, make_float2(rl, rl));
        }
        w[h] = e2m1x8(th[0].x, th[0].y, th[1].x, th[1].y, th[2].x, th[2].y, th[3].x, th[3].y);
        d[h] = w[h] ^ e2m1x8(tl[0].x, tl[0].y, tl[1].x, tl[1].y, tl[2].x, tl[2].y, tl[3].x, tl[3].y);
      }
    }
    if ((d[0] | d[1]) != 0u) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint32_t sh = 4 * (i & 7);
        if ((d[i >> 3] >> sh) & 15u) {
          const uint32_t code = e2m1_code(__fdiv_rn(v[i], total));
          w[i >> 3] = (w[i >> 3] & ~(15u << sh)) | (code << sh);
        }
      }
    }
  }
  packed = make_uint2(nibble_swap(w[0]), nibble_swap(w[1]));
}

// A thread's 16 input elements as raw 16-byte words (4 for fp32, 2 for 16-bit types): loaded
// one row ahead so the next row's HBM reads overlap this row's arithmetic.
template <int DT>
struct Raw16 {
  uint4 w[DT == kF32 ? 4 : 2];
};

template <int DT>
__device__ __forceinline__ Raw16<DT> load_raw16(const void* x, int64_t e0) {
  Raw16<DT> r;
  const uint4* p = reinterpret_cast<const uint4*>(static_cast<const unsigned char*>(x) + e0 * (DT == kF32 ? 4 : 2));
#pragma unroll
  for (int e = 0; e < (DT == kF32 ? 4 : 2); ++e) r.w[e] = __ldg(p + e);
  return r;
}

template <int DT>
__device__ __forceinline__ void unpack16(const Raw16<DT>& r, float (&f)[16]) {
  if (DT == kF32) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      f[4 * e] = __uint_as_float(r.w[e].x); f[4 * e + 1] = __uint_as_float(r.w[e].y);
      f[4 * e + 2] = __uint_as_float(r.w[e].z); f[4 * e + 3] = __uint_as_float(r.w[e].w);
    }
  } else {
    const uint32_t w[8] = {r.w[0].x, r.w[0].y, r.w[0].z, r.w[0].w, r.w[1].x, r.w[1].y, r.w[1].z, r.w[1].w};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      if (DT == kBF16) {
        f[2 * e] = __uint_as_float(w[e] << 16);
        f[2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
      } else {
        const float2 h = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
        f[2 * e] = h.x; f[2 * e + 1] = h.y;
      }
    }
  }
}

template <int DT>
__device__ __forceinline__ void load16(const void* x, int64_t e0, float (&f)[16]) {
  unpack16<DT>(load_raw16<DT>(x, e0), f);
}

constexpr int kQuantMaxStages = 3;

template <int DT>
__device__ __forceinline__ Raw16<DT> smem_raw16(const unsigned char* stage, int t) {
  Raw16<DT> r;
  const uint4* p = reinterpret_cast<const uint4*>(stage) + t * (DT == kF32 ? 4 : 2);
#pragma unroll
  for (int e = 0; e < (DT == kF32 ? 4 : 2); ++e) r.w[e] = p[e];
  return r;
}

// Radix-4 butterfly step b_i = ((a0 + a1) + (a2 + a3)) - 2*a_{3-i}, each operation rounded
// to fp32 (the product 2*a is exact, so the fma rounds once, like the subtraction).
__device__ __forceinline__ void bfly4(float& a0, float& a1, float& a2, float& a3) {
  const float s = __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
  const float b0 = __fmaf_rn(-2.0f, a3, s), b1 = __fmaf_rn(-2.0f, a2, s);
  const float b2 = __fmaf_rn(-2.0f, a1, s), b3 = __fmaf_rn(-2.0f, a0, s);
  a0 = b0; a1 = b1; a2 = b2; a3 = b3;
}

// Base-4 digits 0 and 1 of a 16-element chunk.
__device__ __forceinline__ void bfly16(float (&v)[16]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) bfly4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
#pragma unroll
  for (int m = 0; m < 4; ++m) bfly4(v[m], v[4 + m], v[8 + m], v[12 + m]);
}

// Exchange buffer of one 256-element group (16 chunks x 16 floats); 16-byte slots of a row
// are XOR-permuted by (row >> 1) & 3, so row-wise float4 writes and column-wise scalar reads
// are free of bank conflicts (groups are 272 floats apart to separate half-warps' banks).
__device__ __forceinline__ int xpos(int row, int col) {
  return 16 * row + 4 * ((col >> 2) ^ ((row >> 1) & 3)) + (col & 3);
}

// One CTA per row (persistent over rows), thread c owns 16-element block c of the row.
// Rows are staged in shared memory by bulk copies, nst (1..3, as many as shared memory holds)
// rows ahead: the HBM reads of the next rows overlap this row's arithmetic without holding
// registers. Rows in [rows, rows_pad)
// only get zero scale bytes (padding of the last 128-row tile).
// ROW_SCALE: global scale per row (written to row_scale); else per tensor from *amax_in.
template <int DT, bool ROT, bool ROW_SCALE>
__global__ void __launch_bounds__(1024) nvfp4_quant_kernel(const void* __restrict__ x, int64_t rows,
                                                           int64_t rows_pad, int K,
                                                           const float* __restrict__ amax_in,
                                                           uint8_t* __restrict__ q, uint8_t* __restrict__ sf,
                                                           float* __restrict__ row_scale, int nst) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ float red[2][32];
  const int NST = nst;
  constexpr int kEsz = DT == kF32 ? 4 : 2;
  const uint32_t row_bytes = static_cast<uint32_t>(K) * kEsz;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem_raw);                   // up to 3 mbarriers
  unsigned char* stages = smem_raw + 32;                                   // NST staged rows
  float* xch = reinterpret_cast<float*>(stages + NST * static_cast<size_t>(row_bytes));
  const unsigned char* src = static_cast<const unsigned char*>(x);
  const int t = threadIdx.x;
  const int nb = K >> 4;
  const int ctiles = K >> 6;
  const bool act = t < nb;
  const int lane = t & 31, warp = t >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  float gs_tensor = 0.0f;
  if (!ROW_SCALE) gs_tensor = __fdiv_rn(__ldg(amax_in), 2688.0f);
  float* g = xch + (t >> 4) * 272;
  const int r = t & 15;

  if (t == 0) {
    for (int b = 0; b < NST; ++b) mbar_init(&bar[b], 1);
    fence_mbar_init();
  }
  __syncthreads();
  uint32_t pending = 0, pending_parity = 0;
  if (t == 0) {
    for (int b = 0; b < NST; ++b) {
      const int64_t rb = blockIdx.x + static_cast<int64_t>(b) * gridDim.x;
      if (rb < rows) {
        mbar_arrive_expect_tx(&bar[b], row_bytes);
        bulk_load(stages + b * static_cast<size_t>(row_bytes), src + rb * row_bytes, row_bytes, &bar[b]);
        pending |= 1u << b;
      }
    }
  }
  int it = 0;
  for (int64_t row = blockIdx.x; row < rows_pad; row += gridDim.x, ++it) {
    if (row >= rows) {
      if (act) sf[blocked_offset(row, t, ctiles)] = 0;
      continue;
    }
    const int b = it % NST;
    const bool ok = mbar_wait(&bar[b], static_cast<uint32_t>(it / NST) & 1u, kErrWaitTimeoutProducer);
    if (ok && t == 0) pending &= ~(1u << b);
    if (__syncthreads_or(!ok)) break;  // a staged row never arrived: stop (error recorded)
    const unsigned char* stage = stages + b * static_cast<size_t>(row_bytes);
    float v[16];
    if (act) {
      unpack16<DT>(smem_raw16<DT>(stage, t), v);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = 0.0f;
    }
    if (ROT) {
      bfly16(v);  // digits 0, 1 (within the chunk)
      if (act) {
#pragma unroll
        for (int i = 0; i < 16; i += 4) *reinterpret_cast<float4*>(g + xpos(r, i)) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
      }
      __syncwarp();
      if (act) {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = g[xpos(i, r)];
      }
      bfly16(v);  // digits 2, 3 (across the group's chunks)
      __syncwarp();
      if (act) {
#pragma unroll
        for (int i = 0; i < 16; ++i) g[xpos(i, r)] = v[i];
      }
      __syncwarp();
      if (act) {
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
          const float4 w = *reinterpret_cast<const float4*>(g + xpos(r, i));
          v[i] = __fmul_rn(w.x, 0.0625f); v[i + 1] = __fmul_rn(w.y, 0.0625f);
          v[i + 2] = __fmul_rn(w.z, 0.0625f); v[i + 3] = __fmul_rn(w.w, 0.0625f);
        }
      }
      __syncwarp();
    }
    float gs = gs_tensor;
    if (ROW_SCALE) {
      float am = 0.0f;
#pragma unroll
      for (int i = 0; i < 16; ++i) am = fmaxf(am, fabsf(v[i]));
      const unsigned wm = __reduce_max_sync(0xffffffffu, __float_as_uint(am));
      if (lane == 0) red[it & 1][warp] = __uint_as_float(wm);
      __syncthreads();
      const float rm = __uint_as_float(__reduce_max_sync(0xffffffffu, lane < nw ? __float_as_uint(red[it & 1][lane]) : 0u));
      gs = __fdiv_rn(rm, 2688.0f);
      if (t == 0) row_scale[row] = gs;
    } else {
      __syncthreads();
    }
    // every thread has read this row's stage: refill it with the row NST iterations ahead
    if (t == 0) {
      const int64_t rn = row + static_cast<int64_t>(NST) * gridDim.x;
      if (rn < rows) {
        mbar_arrive_expect_tx(&bar[b], row_bytes);
        bulk_load(stages + b * static_cast<size_t>(row_bytes), src + rn * row_bytes, row_bytes, &bar[b]);
        pending |= 1u << b;
        pending_parity = (pending_parity & ~(1u << b)) | (((static_cast<uint32_t>(it / NST) + 1u) & 1u) << b);
      }
    }
    if (act) {
      uint2 packed;
      uint32_t sfb;
      quant_block16(v, gs, packed, sfb);
      *reinterpret_cast<uint2*>(q + row * (K >> 1) + 8 * t) = packed;
      sf[blocked_offset(row, t, ctiles)] = static_cast<uint8_t>(sfb);
    }
  }
  if (t == 0) {
    for (int b = 0; b < NST; ++b)
      if (pending & (1u << b)) mbar_wait(&bar[b], (pending_parity >> b) & 1u, kErrWaitTimeoutDrain);
  }
}

// One CTA per row (persistent over rows). Blocks (16 elements, one scale byte) are taken in
// pairs: with G = ceil(K/256) groups of 16 blocks and G2 = ceil(G/2), thread t (t < 16 G2)
// owns block t in lane x and block t + 16 G2 in lane y of packed fp32x2 registers, i.e. thread
// (p, r) holds chunk r of groups p and p + G2, the layout of the INT8 path's group-pair
// butterfly, whose packed arithmetic gives bit-identical rotated values. Rows are staged in
// shared memory by bulk copies, nst (1..3, as many as shared memory holds) rows ahead: the HBM
// reads of the next rows overlap this row's arithmetic without holding registers. Rows in
// [rows, rows_pad) only get zero scale bytes (padding of the last 128-row tile).
// ROW_SCALE as in nvfp4_quant_kernel. Rotated 16-bit rows of up to 10240 elements take this kernel,
// which keeps two CTAs per SM there at 95 registers. Measured against nvfp4_quant_kernel
// (bit-identical outputs): rotated bf16 115200 x 5120 0.696 -> 0.577 ms, 32768 x 10240
// 0.468 -> 0.364 ms, equal at 6144-8192. From 11264 on it holds one CTA per SM and is slower
// (0.523 vs 0.512 ms at 11264, 0.610 vs 0.585 at 13824). It is also slower without the rotation
// (0.170 vs 0.151 ms) and on fp32 rows (0.157 vs 0.151 ms at 10240).
template <int DT, bool ROT, bool ROW_SCALE>
__global__ void __launch_bounds__(512) nvfp4_quant_pair_kernel(const void* __restrict__ x, int64_t rows,
                                                           int64_t rows_pad, int K,
                                                           const float* __restrict__ amax_in,
                                                           uint8_t* __restrict__ q, uint8_t* __restrict__ sf,
                                                           float* __restrict__ row_scale, int nst) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ float red[2][32];
  const int NST = nst;
  constexpr int kEsz = DT == kF32 ? 4 : 2;
  const uint32_t row_bytes = static_cast<uint32_t>(K) * kEsz;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem_raw);                   // up to 3 mbarriers
  unsigned char* stages = smem_raw + 32;                                   // NST staged rows
  float2* xch = reinterpret_cast<float2*>(stages + NST * static_cast<size_t>(row_bytes));
  const unsigned char* src = static_cast<const unsigned char*>(x);
  const int t = threadIdx.x;
  const int nb = K >> 4;
  const int pairs = 16 * ((((nb + 15) >> 4) + 1) >> 1);  // 16 G2: offset of lane y's block
  const int ba = t, bb = t + pairs;
  const bool act_a = t < pairs && ba < nb, act_b = bb < nb;  // warp rounding leaves threads >= pairs idle
  const int ctiles = K >> 6;
  const int lane = t & 31, warp = t >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  float gs_tensor = 0.0f;
  if (!ROW_SCALE) gs_tensor = __fdiv_rn(__ldg(amax_in), 2688.0f);
  float2* g = xch + (t >> 4) * 256;  // this half-warp's group pair
  const int r = t & 15;

  if (t == 0) {
    for (int b = 0; b < NST; ++b) mbar_init(&bar[b], 1);
    fence_mbar_init();
  }
  __syncthreads();
  uint32_t pending = 0, pending_parity = 0;
  if (t == 0) {
    for (int b = 0; b < NST; ++b) {
      const int64_t rb = blockIdx.x + static_cast<int64_t>(b) * gridDim.x;
      if (rb < rows) {
        mbar_arrive_expect_tx(&bar[b], row_bytes);
        bulk_load(stages + b * static_cast<size_t>(row_bytes), src + rb * row_bytes, row_bytes, &bar[b]);
        pending |= 1u << b;
      }
    }
  }
  int it = 0;
  for (int64_t row = blockIdx.x; row < rows_pad; row += gridDim.x, ++it) {
    if (row >= rows) {
      if (act_a) sf[blocked_offset(row, ba, ctiles)] = 0;
      if (act_b) sf[blocked_offset(row, bb, ctiles)] = 0;
      continue;
    }
    const int b = it % NST;
    const bool ok = mbar_wait(&bar[b], static_cast<uint32_t>(it / NST) & 1u, kErrWaitTimeoutProducer);
    if (ok && t == 0) pending &= ~(1u << b);
    if (__syncthreads_or(!ok)) break;  // a staged row never arrived: stop (error recorded)
    const unsigned char* stage = stages + b * static_cast<size_t>(row_bytes);
    float2 v[16];
    {
      float fa[16], fb[16];
      if (act_a) {
        unpack16<DT>(smem_raw16<DT>(stage, ba), fa);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) fa[i] = 0.0f;
      }
      if (act_b) {
        unpack16<DT>(smem_raw16<DT>(stage, bb), fb);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) fb[i] = 0.0f;
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = make_float2(fa[i], fb[i]);
    }
    if (ROT) {  // K % 256 == 0: act_a and act_b are uniform over each half-warp
      bfly16x2(v);  // digits 0, 1 (within the chunk)
      if (act_a) {
#pragma unroll
        for (int i = 0; i < 16; i += 2)
          *reinterpret_cast<float4*>(g + xpos2(r, i)) = make_float4(v[i].x, v[i].y, v[i + 1].x, v[i + 1].y);
      }
      __syncwarp();
      if (act_a) {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = g[xpos2(i, r)];
      }
      bfly16x2(v);  // digits 2, 3 (across the groups' chunks): output 16 i + r in v[i]
      __syncwarp();
      if (act_a) {
#pragma unroll
        for (int i = 0; i < 16; ++i) g[xpos2(i, r)] = v[i];
      }
      __syncwarp();
      if (act_a) {  // back to 16 consecutive outputs per thread: the NVFP4 block
        const float2 s16 = make_float2(0.0625f, 0.0625f);
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          const float4 w = *reinterpret_cast<const float4*>(g + xpos2(r, i));
          v[i] = mul2(make_float2(w.x, w.y), s16);
          v[i + 1] = mul2(make_float2(w.z, w.w), s16);
        }
      }
      __syncwarp();
    }
    float bma = 0.0f, bmb = 0.0f;  // block maxima (inactive lanes hold zeros)
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      bma = fmaxf(bma, fabsf(v[i].x));
      bmb = fmaxf(bmb, fabsf(v[i].y));
    }
    float gs = gs_tensor;
    if (ROW_SCALE) {
      const unsigned wm = __reduce_max_sync(0xffffffffu, __float_as_uint(fmaxf(bma, bmb)));
      if (lane == 0) red[it & 1][warp] = __uint_as_float(wm);
      __syncthreads();
      const float rm = __uint_as_float(__reduce_max_sync(0xffffffffu, lane < nw ? __float_as_uint(red[it & 1][lane]) : 0u));
      gs = __fdiv_rn(rm, 2688.0f);
      if (t == 0) row_scale[row] = gs;
    } else {
      __syncthreads();
    }
    // every thread has read this row's stage: refill it with the row NST iterations ahead
    if (t == 0) {
      const int64_t rn = row + static_cast<int64_t>(NST) * gridDim.x;
      if (rn < rows) {
        mbar_arrive_expect_tx(&bar[b], row_bytes);
        bulk_load(stages + b * static_cast<size_t>(row_bytes), src + rn * row_bytes, row_bytes, &bar[b]);
        pending |= 1u << b;
        pending_parity = (pending_parity & ~(1u << b)) | (((static_cast<uint32_t>(it / NST) + 1u) & 1u) << b);
      }
    }
    if (act_a) {
      const BlockScale sa = block_scale(bma, gs), sb = block_scale(bmb, gs);
      uint2 pa, pb;
      block_codes2(v, sa, sb, pa, pb);
      *reinterpret_cast<uint2*>(q + row * (K >> 1) + 8 * ba) = pa;
      sf[blocked_offset(row, ba, ctiles)] = static_cast<uint8_t>(sa.sfb);
      if (act_b) {
        *reinterpret_cast<uint2*>(q + row * (K >> 1) + 8 * bb) = pb;
        sf[blocked_offset(row, bb, ctiles)] = static_cast<uint8_t>(sb.sfb);
      }
    }
  }
  if (t == 0) {
    for (int b = 0; b < NST; ++b)
      if (pending & (1u << b)) mbar_wait(&bar[b], (pending_parity >> b) & 1u, kErrWaitTimeoutDrain);
  }
}

// Per-tensor absmax of n elements (n % 8 == 0 for 16-bit types, % 4 for fp32) into *out
// (as the bits of a non-negative float, combined with atomicMax; *out must start at 0).
template <int DT>
__global__ void __launch_bounds__(256) nvfp4_amax_kernel(const void* __restrict__ x, int64_t n,
                                                         unsigned int* __restrict__ out) {
  float m = 0.0f;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  if (DT == kF32) {
    const float4* p = static_cast<const float4*>(x);
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n / 4; i += stride) {
      const float4 g = __ldg(p + i);
      m = fmaxf(m, fmaxf(fmaxf(fabsf(g.x), fabsf(g.y)), fmaxf(fabsf(g.z), fabsf(g.w))));
    }
  } else {
    const uint4* p = static_cast<const uint4*>(x);
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n / 8; i += stride) {
      const uint4 u = __ldg(p + i);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float lo, hi;
        if (DT == kBF16) {
          lo = __uint_as_float(w[e] << 16);
          hi = __uint_as_float(w[e] & 0xffff0000u);
        } else {
          const float2 h = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
          lo = h.x; hi = h.y;
        }
        m = fmaxf(m, fmaxf(fabsf(lo), fabsf(hi)));
      }
    }
  }
  const unsigned wm = __reduce_max_sync(0xffffffffu, __float_as_uint(m));
  if ((threadIdx.x & 31) == 0 && wm != 0u) atomicMax(out, wm);
}

// *s = fl32(*s / 2688): the per-tensor amax becomes the global scale.
__global__ void nvfp4_finalize_scale_kernel(float* s) {
  if (threadIdx.x == 0 && blockIdx.x == 0) *s = __fdiv_rn(*s, 2688.0f);
}

// out[r, k] = code * fl32(scale_r * sf) (scale per tensor, or per row when per_row), fp32.
// Optionally accumulates sum (out - x)^2 and sum x^2 over the matrix in fp64 (err[0], err[1])
// for the converter's error report (x of dtype DT, may be null).
template <int DT>
__global__ void __launch_bounds__(256) nvfp4_dequant_kernel(const uint8_t* __restrict__ q,
                                                            const uint8_t* __restrict__ sf,
                                                            const float* __restrict__ scale, int per_row,
                                                            int64_t rows, int K, float* __restrict__ out,
                                                            const void* __restrict__ x, double* __restrict__ err) {
  const int nb = K >> 4;
  const int ctiles = K >> 6;
  const int64_t total = rows * nb;
  double e2 = 0.0, x2 = 0.0;
  for (int64_t b = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; b < total;
       b += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = b / nb;
    const int c = static_cast<int>(b - row * nb);
    const float s = __ldg(scale + (per_row ? row : 0));
    const float bs = __fmul_rn(s, e4m3_value(sf[blocked_offset(row, c, ctiles)]));
    const uint2 pk_stored = *reinterpret_cast<const uint2*>(q + row * (K >> 1) + 8 * c);
    const uint2 pk = make_uint2(nibble_swap(pk_stored.x), nibble_swap(pk_stored.y));  // element 2i low
    float v[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint32_t code = ((i < 8 ? pk.x : pk.y) >> (4 * (i & 7))) & 15u;
      const uint32_t mag = code & 7u;
      const float a = mag < 4 ? 0.5f * static_cast<float>(mag) : (mag == 4 ? 2.0f : (mag == 5 ? 3.0f : (mag == 6 ? 4.0f : 6.0f)));
      v[i] = __fmul_rn((code & 8u) ? -a : a, bs);
    }
    if (out != nullptr) {
      float4* o = reinterpret_cast<float4*>(out + row * K + 16 * c);
#pragma unroll
      for (int e = 0; e < 4; ++e) o[e] = make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
    }
    if (err != nullptr) {
      float xf[16];
      load16<DT>(x, row * K + 16 * c, xf);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const double d = static_cast<double>(v[i]) - static_cast<double>(xf[i]);
        e2 += d * d;
        x2 += static_cast<double>(xf[i]) * static_cast<double>(xf[i]);
      }
    }
  }
  if (err != nullptr) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      e2 += __shfl_xor_sync(0xffffffffu, e2, o);
      x2 += __shfl_xor_sync(0xffffffffu, x2, o);
    }
    if ((threadIdx.x & 31) == 0) {
      atomicAdd(err, e2);
      atomicAdd(err + 1, x2);
    }
  }
}

static int sm_count() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

template <int DT, bool ROT, bool ROW_SCALE>
static cudaError_t launch_quant_t(const void* x, int64_t rows, int64_t rows_pad, int K, const float* amax_in,
                                  uint8_t* q, uint8_t* sf, float* row_scale, cudaStream_t st) {
  // rotated 16-bit rows of up to 10240 elements: two blocks per thread (nvfp4_quant_pair_kernel)
  bool pair = false;
  void (*fn)(const void*, int64_t, int64_t, int, const float*, uint8_t*, uint8_t*, float*, int) =
      nvfp4_quant_kernel<DT, ROT, ROW_SCALE>;
  if constexpr (ROT && DT != kF32) {
    if (K <= 10240) {
      pair = true;
      fn = nvfp4_quant_pair_kernel<DT, ROT, ROW_SCALE>;
    }
  }
  const int pairs = 16 * ((((K >> 4) + 15) / 16 + 1) / 2);  // threads owning a block pair
  const int threads = pair ? (pairs + 31) / 32 * 32 : ((K >> 4) + 31) / 32 * 32;
  const size_t xch = pair ? static_cast<size_t>(threads / 16) * 256 * sizeof(float2)
                          : static_cast<size_t>(threads / 16) * 272 * sizeof(float);
  const size_t row_bytes = static_cast<size_t>(K) * (DT == kF32 ? 4 : 2);
  const size_t fixed = 32 + (ROT ? xch : 0);
  constexpr size_t kMaxSmem = 232448 - 256;  // opt-in maximum minus the static reduction buffer
  const int nst = static_cast<int>(std::min<size_t>(kQuantMaxStages, (kMaxSmem - fixed) / row_bytes));
  if (nst < 1) return cudaErrorInvalidValue;
  const size_t smem = fixed + static_cast<size_t>(nst) * row_bytes;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  int per_sm = 1;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  const int64_t cap = static_cast<int64_t>(sm_count()) * per_sm;
  const int grid = static_cast<int>(rows_pad < cap ? rows_pad : cap);
  fn<<<grid, threads, smem, st>>>(x, rows, rows_pad, K, amax_in, q, sf, row_scale, nst);
  return cudaGetLastError();
}

template <bool ROT, bool ROW_SCALE>
static cudaError_t launch_quant_dt(int dtype, const void* x, int64_t rows, int64_t rows_pad, int K,
                                   const float* amax_in, uint8_t* q, uint8_t* sf, float* row_scale, cudaStream_t st) {
  switch (dtype) {
    case kF32: return launch_quant_t<kF32, ROT, ROW_SCALE>(x, rows, rows_pad, K, amax_in, q, sf, row_scale, st);
    case kBF16: return launch_quant_t<kBF16, ROT, ROW_SCALE>(x, rows, rows_pad, K, amax_in, q, sf, row_scale, st);
    case kF16: return launch_quant_t<kF16, ROT, ROW_SCALE>(x, rows, rows_pad, K, amax_in, q, sf, row_scale, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace nvf4q

// Number of kernel launches made by the call (for the launch counter).
cudaError_t launch_nvfp4_pack(const void* w, int dtype, int64_t rows, int K, uint8_t* q, uint8_t* sf,
                              float* tensor_scale, int* launches, cudaStream_t st) {
  *launches = 0;
  cudaError_t e = cudaMemsetAsync(tensor_scale, 0, sizeof(float), st);
  if (e != cudaSuccess) return e;
  const int64_t n = rows * static_cast<int64_t>(K);
  const int grid = nvf4q::sm_count() * 8;
  unsigned int* amax = reinterpret_cast<unsigned int*>(tensor_scale);
  switch (dtype) {
    case kF32: nvf4q::nvfp4_amax_kernel<kF32><<<grid, 256, 0, st>>>(w, n, amax); break;
    case kBF16: nvf4q::nvfp4_amax_kernel<kBF16><<<grid, 256, 0, st>>>(w, n, amax); break;
    case kF16: nvf4q::nvfp4_amax_kernel<kF16><<<grid, 256, 0, st>>>(w, n, amax); break;
    default: return cudaErrorInvalidValue;
  }
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  ++*launches;
  e = nvf4q::launch_quant_dt<false, false>(dtype, w, rows, rows, K, tensor_scale, q, sf, nullptr, st);
  if (e != cudaSuccess) return e;
  ++*launches;
  nvf4q::nvfp4_finalize_scale_kernel<<<1, 32, 0, st>>>(tensor_scale);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  ++*launches;
  return cudaSuccess;
}

cudaError_t launch_nvfp4_quant_rows(const void* x, int dtype, int64_t rows, int K, int rotate, uint8_t* q,
                                    uint8_t* sf, float* row_scale, cudaStream_t st) {
  const int64_t rows_pad = (rows + 127) / 128 * 128;
  if (rotate) return nvf4q::launch_quant_dt<true, true>(dtype, x, rows, rows_pad, K, nullptr, q, sf, row_scale, st);
  return nvf4q::launch_quant_dt<false, true>(dtype, x, rows, rows_pad, K, nullptr, q, sf, row_scale, st);
}

cudaError_t launch_nvfp4_dequant(const uint8_t* q, const uint8_t* sf, const float* scale, int per_row, int64_t rows,
                                 int K, float* out, const void* x, int x_dtype, double* err, cudaStream_t st) {
  const int grid = nvf4q::sm_count() * 8;
  switch (x == nullptr ? kF32 : x_dtype) {
    case kF32: nvf4q::nvfp4_dequant_kernel<kF32><<<grid, 256, 0, st>>>(q, sf, scale, per_row, rows, K, out, x, err); break;
    case kBF16: nvf4q::nvfp4_dequant_kernel<kBF16><<<grid, 256, 0, st>>>(q, sf, scale, per_row, rows, K, out, x, err); break;
    case kF16: nvf4q::nvfp4_dequant_kernel<kF16><<<grid, 256, 0, st>>>(q, sf, scale, per_row, rows, K, out, x, err); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace slim
