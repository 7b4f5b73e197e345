// Reference-order group-256 rotation + per-row INT8 quantisation at the cost of the fast
// transform: the certified quantiser.
//
// The reference rotates every row with np.matmul(grouped, H.T) (slimdit/hadamard.py:56-58),
// which numpy/OpenBLAS evaluate, for rows of five or more groups, as one sequential fp32 chain
// of 256 additions per output (k = 0..255; rotate_quant.cu restates the orders), and quantises
// per row (slimdit/int8.py:49-51): scale = max(fl(absmax / 127), 1e-30), code =
// clip(rint(fl(rot / scale)), -128, 127). This kernel produces the same codes and scales bit
// for bit while running the 256-step chains only for the few outputs where they can matter.
//
// Notation: S = 16 * rotated value (the sum of +-x over the group's 256 inputs; the 1/16 is
// an exact scaling), S_ref the reference chain's result, S' the radix-4 butterfly's result.
// Chunk c of a group is its inputs 16c .. 16c+15.
//
// 1. Certificate per group. Every input is a multiple of its own granularity 2^(e - p) (e = its
//    exponent, p = mantissa bits of the input format); G_c = the smallest granularity among
//    chunks 0..c and M_c = sum |x| over chunks 0..c. Every partial sum of the chain up to the
//    end of chunk c is a multiple of G_c of magnitude <= M_c, hence exact in fp32 while
//    M_c <= 2^24 G_c. Let c0 be the first chunk where that fails (16 if none). Then
//      |S_ref - S'| <= D = sum over chunks c >= c0 of 8 ulp(M_c)   (16 chain roundings of at
//                                                                   most ulp(M_c)/2 each)
//                        + 2^-20 L1                                 (the butterfly: 4 stages, 4
//                                                                   roundings per node output of
//                                                                   <= 2^-24 x the node's input
//                                                                   L1; node L1s of a stage sum
//                                                                   to L1 = M_15)
//    (times 1 + 2^-10; the M_c are taken 2^-14 high for their own rounding and for the chain's
//    accumulated error). c0 = 16 means every partial sum of either order is exact: S' = S_ref,
//    D = 0.
// 2. Row maximum. A = max(|S'| - D) <= max |S_ref| (rounded down), A0 = max |S'| over exact
//    groups, B = max(|S'| + D) over the other groups (rounded up). B < A means the maximum is
//    exact (A0). Otherwise only outputs with |S'| + D >= A can hold it: their chains are run
//    (about one per row) and a second block barrier combines them with A0.
// 3. Codes. With r16 = fl(1 / (16 scale)), rint(S' r16) equals the reference's code unless
//    S' r16 lies within 2^-13 + D r16 of a half-integer (2^-13 covers the reciprocal and the
//    reference's division rounding). Such outputs of exact groups take the IEEE division; those
//    of the other groups get a provisional code and go to a per-warp queue, which is drained one
//    output per lane, reading the inputs from global memory and overwriting the provisional code.
// A chain evaluates chunks 0..c0-1 in four independent partial sums (exact in any order) and
// only chunks c0..15 as the reference's sequential chain.
//
// Rows of fewer than five groups use another OpenBLAS order and are not handled here.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "slim_kernels.h"
#include "slim_ptx.cuh"

namespace slim {

// Queue entry key: (iteration of the CTA's row loop) << 18 | c0 << 14 | column (K <= 16384); the
// row is blockIdx.x + it * gridDim.x, so rows per CTA are limited to 2^14.
constexpr int kCertColBits = 14;
constexpr int64_t kCertMaxIters = int64_t{1} << 14;

template <int DT>
struct CertFmt {
  static constexpr int kEsz = DT == kF32 ? 4 : 2;
  static constexpr int kMant = DT == kF32 ? 23 : (DT == kF16 ? 10 : 7);
};

// 16 consecutive inputs from a 16-byte aligned generic address (shared or global), as fp32.
template <int DT>
__device__ __forceinline__ void cert_load16(const unsigned char* p, float (&f)[16]) {
  if (DT == kF32) {
    const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float4 g = q[e];
      f[4 * e] = g.x; f[4 * e + 1] = g.y; f[4 * e + 2] = g.z; f[4 * e + 3] = g.w;
    }
  } else {
    const uint4* q = reinterpret_cast<const uint4*>(p);
    const uint4 u0 = q[0], u1 = q[1];
    const uint32_t w[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
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

// The reference chain for output j of one group (grp = its 256 inputs, c0 as in step 1):
// S_ref = fl-chain of sum_k sign(j, k) x_k over k = 0..255, sign(j, k) = sig(b) lam(l) for
// k = 16 b + l. Chunks below c0 are summed exactly as four interleaved partial sums (every
// partial sum there is exact, so the grouping cannot change it); from chunk c0 on the
// accumulator is carried as sig(b) * acc, so every step is fma(x, lam_l, acc) with an exact
// product and a chunk change multiplies it by sig(b) sig(b-1) = +-1 (rounding to nearest is
// symmetric, so the carried chain rounds exactly like the plain one).
template <int DT>
__device__ __noinline__ float cert_chain(const unsigned char* grp, int j, int c0) {
  const int j0 = j & 3, j1 = (j >> 2) & 3, j2 = (j >> 4) & 3, j3 = (j >> 6) & 3;
  float lam[16];
#pragma unroll
  for (int l = 0; l < 16; ++l) lam[l] = h4sign(j1, l >> 2) * h4sign(j0, l & 3);
  constexpr int kEsz = CertFmt<DT>::kEsz;
  float part[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  for (int b0 = 0; b0 < c0; b0 += 4) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int b = b0 + u;
      if (b < c0) {
        float f[16];
        cert_load16<DT>(grp + 16 * b * kEsz, f);
        float t = 0.0f;
#pragma unroll
        for (int l = 0; l < 16; ++l) t = __fmaf_rn(f[l], lam[l], t);
        part[u] = __fmaf_rn(t, h4sign(j3, b >> 2) * h4sign(j2, b & 3), part[u]);
      }
    }
  }
  const float pre = (part[0] + part[1]) + (part[2] + part[3]);
  if (c0 >= 16) return pre;
  float sig_prev = h4sign(j3, c0 >> 2) * h4sign(j2, c0 & 3);
  float acc = pre * sig_prev;
  for (int b = c0; b < 16; ++b) {
    float f[16];
    cert_load16<DT>(grp + 16 * b * kEsz, f);
    const float sig = h4sign(j3, b >> 2) * h4sign(j2, b & 3);
    acc *= sig * sig_prev;
#pragma unroll
    for (int l = 0; l < 16; ++l) acc = __fmaf_rn(f[l], lam[l], acc);
    sig_prev = sig;
  }
  return acc * sig_prev;
}

// 2^(24 + e - p) for the granularity of the smallest |x| of a chunk prefix: the largest M with
// every partial sum exact. min_abs = 0 gives the format's smallest quantum (zeros are multiples
// of anything).
template <int DT>
__device__ __forceinline__ float cert_exact_limit(float min_abs) {
  const int te = static_cast<int>((__float_as_uint(min_abs) >> 23) & 0xffu) - CertFmt<DT>::kMant + 24;
  return te <= 0 ? 0.0f : (te >= 255 ? __uint_as_float(0x7f800000u) : __uint_as_float(static_cast<uint32_t>(te) << 23));
}

// ulp(v) = 2^(E - 150) for v > 0 with biased exponent E: a normal number for E > 23, else the
// subnormal with bit E - 1 set (2^-149 for E <= 1).
__device__ __forceinline__ float cert_ulp(float v) {
  const int E = static_cast<int>((__float_as_uint(v) >> 23) & 0xffu);
  return E > 23 ? __uint_as_float(static_cast<uint32_t>(E - 23) << 23) : __uint_as_float(1u << (E > 1 ? E - 1 : 0));
}

// Per-lane quantised pair with the residual: codes packed in the low 16 bits (lane x in bits
// 0-7), |S r16 - code| per lane in d.
__device__ __forceinline__ uint32_t cert_quant_pair(float2 S, float2 r2, float2& dabs) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23: fl(S r16 + kMagic) = kMagic + rint(S r16)
  const float2 xq = fma2(S, r2, make_float2(kMagic, kMagic));
  const float2 c = add2(xq, make_float2(-kMagic, -kMagic));
  const float2 d = fma2(S, r2, make_float2(-c.x, -c.y));
  dabs = make_float2(fabsf(d.x), fabsf(d.y));
  return __byte_perm(__float_as_uint(xq.x), __float_as_uint(xq.y), 0x0040);
}

// One lane per queued output: run its chain from global memory and overwrite the provisional
// code. The warp's entries [0, n) are read; every lane of the warp must call this.
template <int DT>
__device__ __forceinline__ void cert_drain(const unsigned char* src, int K, int8_t* q_out, const uint32_t* qkey,
                                           const float* qscale, int n, int lane) {
  __syncwarp();
  if (lane < n) {
    constexpr int kEsz = CertFmt<DT>::kEsz;
    const uint32_t key = qkey[lane];
    const int64_t row = blockIdx.x + static_cast<int64_t>(key >> 18) * gridDim.x;
    const uint32_t col = key & ((1u << kCertColBits) - 1u);
    const int c0 = static_cast<int>((key >> kCertColBits) & 15u);
    const float scale = qscale[lane];
    const int64_t e0 = row * K + (col & ~255u);
    const float S = cert_chain<DT>(src + e0 * kEsz, static_cast<int>(col & 255u), c0);
    q_out[row * K + col] = quant_code(__fmul_rn(S, 0.0625f), scale);
  }
  __syncwarp();
}

// Group bound of step 1 from a half-warp's chunk sums (l1 = sum |x| of this thread's chunk) and
// chunk minima: D (0 for an exact group) and c0 (16 when exact). r = chunk index; every lane of
// the warp calls this (the two half-warps hold different groups).
template <int DT>
__device__ __forceinline__ float cert_group_bound(float l1, float mn, int r, int lane, int& c0) {
  float m = l1, g = mn;
#pragma unroll
  for (int d = 1; d < 16; d <<= 1) {  // inclusive prefix over chunks 0..r
    const float mu = __shfl_up_sync(0xffffffffu, m, d, 16);
    const float gu = __shfl_up_sync(0xffffffffu, g, d, 16);
    if (r >= d) {
      m += mu;
      g = fminf(g, gu);
    }
  }
  const float mp = __fmul_ru(m, 1.00006103515625f);  // 1 + 2^-14
  const bool rounds = mp > cert_exact_limit<DT>(g);
  float term = rounds ? 8.0f * cert_ulp(mp) : 0.0f;
  const unsigned ball = __ballot_sync(0xffffffffu, rounds);
  const unsigned half = (ball >> (lane & 16)) & 0xffffu;
  c0 = half ? __ffs(half) - 1 : 16;
  const float l1p = __shfl_sync(0xffffffffu, mp, 15, 16);
#pragma unroll
  for (int o = 8; o >= 1; o >>= 1) term = __fadd_ru(term, __shfl_xor_sync(0xffffffffu, term, o));
  if (half == 0) return 0.0f;
  const float d = __fmaf_ru(l1p, 9.5367431640625e-07f, term);  // + 2^-20 L1
  return __fmaf_ru(d, 1.0009765625f, 7.52316385e-37f);          // (1 + 2^-10), + 2^-120
}

// Block barrier over the CTA's warps (mbarrier `cbar`, one arrival per warp) that does useful work
// while it waits: a warp whose arrival does not complete the phase drains its own queue of
// outputs awaiting their chain (if it holds at least `qmin`) before waiting. Every wait is
// bounded; returns false on a timeout (error recorded).
template <int DT>
__device__ __forceinline__ bool cert_cta_sync(uint64_t* cbar, uint32_t& parity, int lane, const unsigned char* src,
                                              int K, int8_t* q_out, const uint32_t* qkey, const float* qscale,
                                              int& qn, int qmin) {
  __syncwarp();
  if (lane == 0) mbar_arrive(cbar);
  const bool done = __any_sync(0xffffffffu, mbar_try_wait(cbar, parity));
  if (!done && qn >= qmin) {
    cert_drain<DT>(src, K, q_out, qkey, qscale, qn, lane);
    qn = 0;
  }
  const bool ok = mbar_wait(cbar, parity, kErrWaitTimeoutEpilogue);
  parity ^= 1u;
  return __all_sync(0xffffffffu, ok);
}

// Persistent over rows, as bfly2_rotate_quant_kernel: a row of G groups is split into G2 =
// ceil(G/2) group pairs (g, g + G2), 16 threads per pair; thread (p, r) holds chunk r (16
// consecutive inputs) of both groups as the two lanes of packed fp32x2 registers. Rows arrive
// in shared memory by double-buffered bulk copies.
template <int DT, int MAXR, int QN>
__global__ void __maxnreg__(MAXR) cert_rotate_quant_kernel(const void* __restrict__ x, int64_t rows, int K,
                                                           int8_t* __restrict__ q_out,
                                                           float* __restrict__ scale_out) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  constexpr int kEsz = CertFmt<DT>::kEsz;
  const uint32_t row_bytes = static_cast<uint32_t>(K) * kEsz;
  const int t = threadIdx.x;
  const int warp = t >> 5, lane = t & 31;
  const int nw = blockDim.x >> 5;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem_raw);           // 2 row-staging mbarriers, cbar
  uint64_t* cbar = bar + 2;                                        // block barrier (one arrival per warp)
  volatile uint32_t* fail_flag = reinterpret_cast<volatile uint32_t*>(smem_raw + 24);  // a staged row never arrived
  float* red = reinterpret_cast<float*>(smem_raw + 32);              // [2 parities][4 kinds][16 warps]
  uint32_t* qkey_all = reinterpret_cast<uint32_t*>(smem_raw + 544);  // [warps][QN] queued outputs
  float* qscale_all = reinterpret_cast<float*>(qkey_all + nw * QN);  // [warps][QN] their row scales
  unsigned char* rowbuf = reinterpret_cast<unsigned char*>(qscale_all + nw * QN);  // 2 staged rows
  float2* xbuf = reinterpret_cast<float2*>(rowbuf + 2 * static_cast<size_t>(row_bytes));
  uint32_t* qkey = qkey_all + warp * QN;
  float* qscale = qscale_all + warp * QN;

  const int G = K >> 8;
  const int G2 = (G + 1) >> 1;
  const int p = t >> 4;  // group pair
  const int r = t & 15;  // chunk within the group
  const bool act_a = p < G2;
  const bool act_b = p + G2 < G;
  float2* gbuf = xbuf + (warp * 2 + ((lane >> 4) & 1)) * 256;
  const unsigned char* src = static_cast<const unsigned char*>(x);
  int qn = 0;  // queued outputs of this warp (warp-uniform)

  if (t == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    mbar_init(cbar, static_cast<uint32_t>(nw));
    *fail_flag = 0u;
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
  bool failed = false;
  uint32_t cparity = 0;                // phase parity of cbar
  const int qmin = QN / 4;             // smallest queue worth draining while waiting
  for (int it = 0; row < rows; row += gridDim.x, ++it) {
    const int b = it & 1;
    const bool ok = mbar_wait(&bar[b], (it >> 1) & 1, kErrWaitTimeoutProducer);
    if (ok && t == 0) pending &= ~(1u << b);
    if (!ok) *fail_flag = 1u;  // seen by every thread after the next block barrier
    const unsigned char* stage = rowbuf + b * row_bytes;
    const int ea = p * 256 + 16 * r;  // element offset of chunk a in the row
    const int eb = ea + G2 * 256;     // chunk b
    float2 v[16];
    float l1a = 0.0f, l1b = 0.0f, mna = __uint_as_float(0x7f800000u), mnb = __uint_as_float(0x7f800000u);
    if (act_a) {
      float fa[16], fb[16];
      cert_load16<DT>(stage + ea * kEsz, fa);
      if (act_b) {
        cert_load16<DT>(stage + eb * kEsz, fb);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) fb[i] = 0.0f;
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        l1a += fabsf(fa[i]);
        l1b += fabsf(fb[i]);
        mna = fminf(mna, fabsf(fa[i]));
        mnb = fminf(mnb, fabsf(fb[i]));
        v[i] = make_float2(fa[i], fb[i]);
      }
      bfly16x2(v);  // digits 0, 1
#pragma unroll
      for (int i = 0; i < 16; i += 2)
        *reinterpret_cast<float4*>(gbuf + xpos2(r, i)) = make_float4(v[i].x, v[i].y, v[i + 1].x, v[i + 1].y);
    }
    // per group: D and c0 from the chunk prefix sums of the 16 chunk owners (half-warp)
    int c0a, c0b;
    float Da = cert_group_bound<DT>(l1a, mna, r, lane, c0a);
    float Db = cert_group_bound<DT>(l1b, mnb, r, lane, c0b);
    if (!act_a) Da = 0.0f;
    if (!act_b) Db = 0.0f;
    __syncwarp();
    float ama = 0.0f, amb = 0.0f;
    if (act_a) {
#pragma unroll
      for (int rr = 0; rr < 16; ++rr) v[rr] = gbuf[xpos2(rr, r)];
      bfly16x2(v);  // digits 2, 3: lanes hold S' for outputs 16 rr + r of groups p and p + G2
#pragma unroll
      for (int rr = 0; rr < 16; ++rr) {
        ama = fmaxf(ama, fabsf(v[rr].x));
        amb = fmaxf(amb, fabsf(v[rr].y));
      }
    }
    // row maximum bounds: one redux per kind and warp, one block barrier
    {
      const float tA0 = fmaxf(Da == 0.0f ? ama : 0.0f, Db == 0.0f ? amb : 0.0f);
      const float tA = fmaxf(fmaxf(__fsub_rd(ama, Da), __fsub_rd(amb, Db)), 0.0f);
      const float tB = fmaxf(Da > 0.0f ? __fadd_ru(ama, Da) : 0.0f, Db > 0.0f ? __fadd_ru(amb, Db) : 0.0f);
      const unsigned w0 = __reduce_max_sync(0xffffffffu, __float_as_uint(tA0));
      const unsigned w1 = __reduce_max_sync(0xffffffffu, __float_as_uint(tA));
      const unsigned w2 = __reduce_max_sync(0xffffffffu, __float_as_uint(tB));
      if (lane == 0) {
        red[(b * 4 + 0) * 16 + warp] = __uint_as_float(w0);
        red[(b * 4 + 1) * 16 + warp] = __uint_as_float(w1);
        red[(b * 4 + 2) * 16 + warp] = __uint_as_float(w2);
      }
    }
    if (!cert_cta_sync<DT>(cbar, cparity, lane, src, K, q_out, qkey, qscale, qn, qmin) || *fail_flag != 0u) {
      failed = true;  // a staged row never arrived or a barrier timed out (error recorded)
      break;
    }
    const float A0 = __uint_as_float(__reduce_max_sync(0xffffffffu, lane < nw ? __float_as_uint(red[(b * 4 + 0) * 16 + lane]) : 0u));
    const float A = __uint_as_float(__reduce_max_sync(0xffffffffu, lane < nw ? __float_as_uint(red[(b * 4 + 1) * 16 + lane]) : 0u));
    const float B = __uint_as_float(__reduce_max_sync(0xffffffffu, lane < nw ? __float_as_uint(red[(b * 4 + 2) * 16 + lane]) : 0u));
    float absmax_s = A0;
    if (B >= A && B > 0.0f) {  // uniform: the maximum may sit in an inexact group
      // candidates as a mask (bit rr: group p, bit 16 + rr: group p + G2), then one chain each
      uint32_t cmask = 0;
      if (act_a && Da > 0.0f && __fadd_ru(ama, Da) >= A) {
#pragma unroll
        for (int rr = 0; rr < 16; ++rr)
          if (__fadd_ru(fabsf(v[rr].x), Da) >= A) cmask |= 1u << rr;
      }
      if (act_b && Db > 0.0f && __fadd_ru(amb, Db) >= A) {
#pragma unroll
        for (int rr = 0; rr < 16; ++rr)
          if (__fadd_ru(fabsf(v[rr].y), Db) >= A) cmask |= 1u << (16 + rr);
      }
      float cm = 0.0f;
      while (cmask != 0u) {
        const int bit = __ffs(cmask) - 1;
        cmask &= cmask - 1u;
        const int grp = bit < 16 ? p : p + G2;
        cm = fmaxf(cm, fabsf(cert_chain<DT>(stage + grp * 256 * kEsz, 16 * (bit & 15) + r, bit < 16 ? c0a : c0b)));
      }
      const unsigned wc = __reduce_max_sync(0xffffffffu, __float_as_uint(cm));
      if (lane == 0) red[(b * 4 + 3) * 16 + warp] = __uint_as_float(wc);
      if (!cert_cta_sync<DT>(cbar, cparity, lane, src, K, q_out, qkey, qscale, qn, qmin)) {
        failed = true;
        break;
      }
      const float cmax = __uint_as_float(__reduce_max_sync(0xffffffffu, lane < nw ? __float_as_uint(red[(b * 4 + 3) * 16 + lane]) : 0u));
      absmax_s = fmaxf(A0, cmax);
    }
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
    const float scale = row_scale_from_absmax(__fmul_rn(absmax_s, 0.0625f));
    const float r16 = __frcp_rn(__fmul_rn(16.0f, scale));
    const bool tiny_row = absmax_s < 8.271806125530277e-25f;  // 2^-80: S / 16 could be subnormal
    if (t == 0) scale_out[row] = scale;
    const int64_t rbase = row * static_cast<int64_t>(K);
    // codes: provisional from S' r16, written to the transpose buffer; outputs near a rounding
    // boundary are marked (bit rr: group p, bit 16 + rr: group p + G2) and settled below
    uint32_t flags = 0;  // queued outputs (inexact groups)
    __syncwarp();
    uint16_t* cbuf = reinterpret_cast<uint16_t*>(gbuf);
    if (act_a) {
      const float2 r2 = make_float2(r16, r16);
      const float lim_a = __fsub_rd(0.5f, __fmaf_ru(Da, __fmul_ru(r16, 1.0009765625f), 1.220703125e-4f));
      const float lim_b = __fsub_rd(0.5f, __fmaf_ru(Db, __fmul_ru(r16, 1.0009765625f), 1.220703125e-4f));
      uint32_t near = 0;
#pragma unroll
      for (int rr = 0; rr < 16; ++rr) {
        float2 d;
        cbuf[16 * rr + r] = static_cast<uint16_t>(cert_quant_pair(v[rr], r2, d));
        if (d.x > lim_a) near |= 1u << rr;
        if (d.y > lim_b) near |= 1u << (16 + rr);
      }
      if (tiny_row) near = ~0u;
      if (!act_b) near &= 0xffffu;
      // inexact groups: queued for their chain; exact groups: the IEEE division on S' = S_ref
      flags = near & ((Da > 0.0f ? 0x0000ffffu : 0u) | (Db > 0.0f ? 0xffff0000u : 0u));
      near &= ~flags;
      while (near != 0u) {
        const int bit = __ffs(near) - 1;
        near &= near - 1u;
        const int rr = bit & 15;
        float sv = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (i == rr) sv = bit < 16 ? v[i].x : v[i].y;
        const uint8_t c = static_cast<uint8_t>(quant_code(__fmul_rn(sv, 0.0625f), scale));
        const uint16_t cw = cbuf[16 * rr + r];
        cbuf[16 * rr + r] = bit < 16 ? static_cast<uint16_t>((cw & 0xff00u) | c)
                                     : static_cast<uint16_t>((cw & 0x00ffu) | (static_cast<uint32_t>(c) << 8));
      }
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
    __syncwarp();  // provisional codes stored before any queued output overwrites its code
    // each round, every lane offers its lowest queued output; at most the queue's free room is
    // taken (the rest wait for the next round), and a full queue is drained at once
    while (__any_sync(0xffffffffu, flags != 0u)) {
      const int bit = flags != 0u ? __ffs(flags) - 1 : -1;
      const unsigned ball = __ballot_sync(0xffffffffu, bit >= 0);
      const int room = QN - qn;
      const int rank = __popc(ball & ((1u << lane) - 1u));
      if (bit >= 0 && rank < room) {
        const int grp = bit < 16 ? p : p + G2;
        const uint32_t c0 = static_cast<uint32_t>(bit < 16 ? c0a : c0b);
        qkey[qn + rank] = (static_cast<uint32_t>(it) << 18) | (c0 << kCertColBits) |
                          static_cast<uint32_t>(grp * 256 + 16 * (bit & 15) + r);
        qscale[qn + rank] = scale;
        flags &= flags - 1u;
      }
      qn += min(__popc(ball), room);
      if (qn == QN) {
        cert_drain<DT>(src, K, q_out, qkey, qscale, qn, lane);
        qn = 0;
      }
      __syncwarp();
    }
  }
  if (!failed && qn > 0) cert_drain<DT>(src, K, q_out, qkey, qscale, qn, lane);
  if (t == 0) {
    for (int b = 0; b < 2; ++b)
      if (pending & (1u << b)) mbar_wait(&bar[b], (pending_parity >> b) & 1u, kErrWaitTimeoutDrain);
  }
}

// Queue length per warp: 32 (one drain pass of 32 lanes); 16 for rows of 48+ groups, whose
// 14+ warps must leave room for two CTAs per SM.
static int cert_queue_len(int threads) { return threads >= 384 ? 16 : 32; }

size_t cert_smem_bytes(int K, int dtype, int threads) {
  const size_t esz = dtype == kF32 ? 4 : 2;
  const size_t nw = static_cast<size_t>(threads / 32);
  return 544 + nw * cert_queue_len(threads) * 8 + 2 * esz * static_cast<size_t>(K) + nw * 2 * 256 * sizeof(float2);
}

// Rows of 5 <= K/256 <= 64 groups. Inputs with more than 2^18 rows per CTA take the
// sixteen-output reference kernel instead.
cudaError_t launch_cert_rotate_quant(const void* x, int dtype, int64_t rows, int K, int8_t* q, float* scale,
                                     cudaStream_t st) {
  const int g2 = ((K >> 8) + 1) >> 1;
  const int threads = (g2 + 1) / 2 * 32;
  const size_t smem = cert_smem_bytes(K, dtype, threads);
  void (*fn)(const void*, int64_t, int, int8_t*, float*);
  if (threads >= 384)
    fn = dtype == kBF16 ? cert_rotate_quant_kernel<kBF16, 72, 16>
                        : (dtype == kF32 ? cert_rotate_quant_kernel<kF32, 72, 16> : cert_rotate_quant_kernel<kF16, 72, 16>);
  else
    fn = dtype == kBF16 ? cert_rotate_quant_kernel<kBF16, 96, 32>
                        : (dtype == kF32 ? cert_rotate_quant_kernel<kF32, 96, 32> : cert_rotate_quant_kernel<kF16, 96, 32>);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  int per_sm = 1;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  const int grid = grid_for_rows(rows, per_sm);
  if ((rows + grid - 1) / grid > kCertMaxIters) return launch_ref_rotate_quant(x, dtype, rows, K, q, scale, st);
  fn<<<grid, threads, smem, st>>>(x, rows, K, q, scale);
  return cudaGetLastError();
}

}  // namespace slim
