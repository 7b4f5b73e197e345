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
//    (about one per row) by the row's fixer warp, which combines them with A0.
// 3. Codes. With r16 = fl(1 / (16 scale)), rint(S' r16) equals the reference's code unless
//    S' r16 lies within 2^-13 + D r16 of a half-integer (2^-13 covers the reciprocal and the
//    reference's division rounding). Such outputs of exact groups take the IEEE division.
// Chains run on warps of their own (the fixers), behind the others (the streamers), so
// no streamer waits for one: a streamer that finds the maximum uncertain writes provisional
// codes against an interval [s_lo, s_hi] that contains the scale (an output's code is certain
// when it is the same for every scale in it) and lists the candidates for the maximum; outputs
// whose code is not certain are listed too. The fixer runs the listed chains from the staged
// row in shared memory, one output per lane, settles the scale and overwrites the provisional
// codes, then restages the row's buffer (three buffers where shared memory allows, so the
// streamers run up to two rows ahead of the fixers).
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

// Two chain steps on one packed word of two bf16 (f16) inputs: acc = fl(fl(acc + l0 x0) + l1 x1)
// with l0, l1 = +-1 packed the same way. The mixed-precision fma takes the 16-bit inputs as they
// are stored (their product with +-1 is exact in fp32) and rounds once, like the fp32 chain.
template <int DT>
__device__ __forceinline__ float cert_fma_pair(float acc, uint32_t w, uint32_t lp) {
  if (DT == kBF16) {
    asm("{\n\t.reg .b16 xl, xh, ll, lh;\n\t"
        "mov.b32 {xl, xh}, %1;\n\t"
        "mov.b32 {ll, lh}, %2;\n\t"
        "fma.rn.f32.bf16 %0, xl, ll, %0;\n\t"
        "fma.rn.f32.bf16 %0, xh, lh, %0;\n\t}"
        : "+f"(acc) : "r"(w), "r"(lp));
  } else {
    asm("{\n\t.reg .b16 xl, xh, ll, lh;\n\t"
        "mov.b32 {xl, xh}, %1;\n\t"
        "mov.b32 {ll, lh}, %2;\n\t"
        "fma.rn.f32.f16 %0, xl, ll, %0;\n\t"
        "fma.rn.f32.f16 %0, xh, lh, %0;\n\t}"
        : "+f"(acc) : "r"(w), "r"(lp));
  }
  return acc;
}

// The sixteen chain steps of one chunk: 16-bit inputs through cert_fma_pair (lp = the signs
// packed per input pair), fp32 inputs through fp32 fmas (lam).
template <int DT>
__device__ __forceinline__ float cert_chunk_steps(float acc, const uint4* q, const uint32_t (&lp)[8],
                                                  const float (&lam)[16]) {
  if (DT == kF32) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 u = q[i];
      acc = __fmaf_rn(__uint_as_float(u.x), lam[4 * i], acc);
      acc = __fmaf_rn(__uint_as_float(u.y), lam[4 * i + 1], acc);
      acc = __fmaf_rn(__uint_as_float(u.z), lam[4 * i + 2], acc);
      acc = __fmaf_rn(__uint_as_float(u.w), lam[4 * i + 3], acc);
    }
  } else {
    const uint4 u0 = q[0], u1 = q[1];
    acc = cert_fma_pair<DT>(acc, u0.x, lp[0]);
    acc = cert_fma_pair<DT>(acc, u0.y, lp[1]);
    acc = cert_fma_pair<DT>(acc, u0.z, lp[2]);
    acc = cert_fma_pair<DT>(acc, u0.w, lp[3]);
    acc = cert_fma_pair<DT>(acc, u1.x, lp[4]);
    acc = cert_fma_pair<DT>(acc, u1.y, lp[5]);
    acc = cert_fma_pair<DT>(acc, u1.z, lp[6]);
    acc = cert_fma_pair<DT>(acc, u1.w, lp[7]);
  }
  return acc;
}

// The reference chain for output j of one group (grp = its 256 inputs in shared memory, c0 as in
// step 1): S_ref = fl-chain of sum_k sign(j, k) x_k over k = 0..255, sign(j, k) = sig(b) lam(l)
// for k = 16 b + l. Chunks below c0 are summed exactly, four at a time (any grouping is exact
// there). From chunk c0 on the accumulator is carried as sig(b) * acc, so every step is
// fma(x, lam_l, acc) with an exact product and a chunk change multiplies it by sig(b) sig(b-1)
// = +-1 (rounding to nearest is symmetric, so the carried chain rounds exactly like the plain
// one).
template <int DT>
__device__ __forceinline__ float cert_chain(const unsigned char* grp, int j, int c0) {
  const int j0 = j & 3, j1 = (j >> 2) & 3, j2 = (j >> 4) & 3, j3 = (j >> 6) & 3;
  float lam[16];
  uint32_t lp[8];
  const uint32_t one = DT == kF16 ? 0x3c00u : 0x3f80u;  // 1.0 in the 16-bit format; | 0x8000 = -1.0
#pragma unroll
  for (int l = 0; l < 16; ++l) lam[l] = h4sign(j1, l >> 2) * h4sign(j0, l & 3);
#pragma unroll
  for (int e = 0; e < 8; ++e)
    lp[e] = (one | (lam[2 * e] < 0.0f ? 0x8000u : 0u)) | ((one | (lam[2 * e + 1] < 0.0f ? 0x8000u : 0u)) << 16);
  constexpr int kChunk = 16 * CertFmt<DT>::kEsz;
  float pa = 0.0f, pb = 0.0f;
  int b = 0;
  for (; b + 4 <= c0; b += 4) {  // chunks b..b+3 share digit 3 of b; their digit 2 is 0..3
    const uint4* q = reinterpret_cast<const uint4*>(grp + b * kChunk);
    const float t0 = cert_chunk_steps<DT>(0.0f, q, lp, lam);
    const float t1 = cert_chunk_steps<DT>(0.0f, q + kChunk / 16, lp, lam);
    const float t2 = cert_chunk_steps<DT>(0.0f, q + 2 * (kChunk / 16), lp, lam);
    const float t3 = cert_chunk_steps<DT>(0.0f, q + 3 * (kChunk / 16), lp, lam);
    const float s3 = h4sign(j3, b >> 2);
    pa = __fmaf_rn(__fmaf_rn(t0, h4sign(j2, 0), t2 * h4sign(j2, 2)), s3, pa);
    pb = __fmaf_rn(__fmaf_rn(t1, h4sign(j2, 1), t3 * h4sign(j2, 3)), s3, pb);
  }
  for (; b < c0; ++b) {
    const float ta = cert_chunk_steps<DT>(0.0f, reinterpret_cast<const uint4*>(grp + b * kChunk), lp, lam);
    pa = __fmaf_rn(ta, h4sign(j3, b >> 2) * h4sign(j2, b & 3), pa);
  }
  const float pre = pa + pb;
  if (c0 >= 16) return pre;
  float sig_prev = h4sign(j3, c0 >> 2) * h4sign(j2, c0 & 3);
  float acc = pre * sig_prev;
  for (b = c0; b < 16; ++b) {
    const float sig = h4sign(j3, b >> 2) * h4sign(j2, b & 3);
    acc *= sig * sig_prev;
    acc = cert_chunk_steps<DT>(acc, reinterpret_cast<const uint4*>(grp + b * kChunk), lp, lam);
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

// Provisional codes of a thread's 16 output pairs into the transpose buffer (code of output
// 16 rr + r at cbuf[16 rr + r], group p in the low byte), and the mask of outputs whose code is
// not certain: |S' rm - code| (+ |S'| w when the scale is an interval) above lim.
template <bool kInterval>
__device__ __forceinline__ uint32_t cert_codes(const float2 (&v)[16], float rm, float w, float lim_a, float lim_b,
                                               uint16_t* cbuf, int r) {
  const float2 r2 = make_float2(rm, rm);
  uint32_t near = 0;
#pragma unroll
  for (int rr = 0; rr < 16; ++rr) {
    float2 d;
    cbuf[16 * rr + r] = static_cast<uint16_t>(cert_quant_pair(v[rr], r2, d));
    if (kInterval) {
      d.x = __fmaf_ru(fabsf(v[rr].x), w, d.x);
      d.y = __fmaf_ru(fabsf(v[rr].y), w, d.y);
    }
    if (d.x > lim_a) near |= 1u << rr;
    if (d.y > lim_b) near |= 1u << (16 + rr);
  }
  return near;
}

// Float exchange buffer of one half-warp (16 rows x 16 floats): the 16-byte slot of a row is
// XOR-permuted by the row, and the second half-warp of a warp (h = 1) takes row rho ^ 1 for row
// rho, so the row-wise 16-byte writes and the column-wise 4-byte reads of the whole warp are
// free of bank conflicts (the two half-warps read complementary 16-bank halves).
__device__ __forceinline__ int xposf(int row, int col, int h) {
  const int pr = row ^ h;
  return 16 * pr + 4 * ((col >> 2) ^ ((pr >> 1) & 3)) + (col & 3);
}

// ------------------------------------------------------------------ the kernel
// Per staged row: a record and two lists (columns of the outputs whose chain is needed), filled by
// the streamer warps and settled by the fixer warp that owns the row's buffer.
struct CertRec {
  uint32_t counts;    // list lengths: candidates for the row maximum (bits 16-31), near ties (0-15)
  uint32_t pad0;
  uint32_t flags;     // kCertUnsure: the scale is settled by the fixer; kCertOverflow: a list overflowed
  float a0;           // exact part of the row maximum (S units)
  float scale;        // the row scale (certain rows)
  uint32_t pad[3];
};
constexpr uint32_t kCertUnsure = 1u, kCertOverflow = 2u;
constexpr int kCertCand = 64;   // candidate list length per row
constexpr int kCertTies = 448;  // near-tie list length per row

// Shared-memory layout (bytes) for NB staging buffers: mbarriers full[NB] (row staged), done[NB]
// (streamers finished a row), cbar (streamer block barrier); failure flag; warp partials (two
// row parities); per buffer a record, the per-group c0 and the two lists; then the NB staged rows
// and the streamers' transpose buffers.
template <int NB>
struct CertLayout {
  static constexpr int kFull = 0;
  static constexpr int kDone = 8 * NB;
  static constexpr int kCbar = 16 * NB;
  static constexpr int kFail = kCbar + 8;
  static constexpr int kRed = kFail + 8;                                   // [2][3 kinds][16 warps] floats
  static constexpr int kRec = kRed + 2 * 3 * 16 * 4;                       // [NB] CertRec
  static constexpr int kC0 = kRec + NB * static_cast<int>(sizeof(CertRec));  // [NB][64]
  static constexpr int kCand = kC0 + NB * 64;                              // [NB][kCertCand] uint16
  static constexpr int kTies = kCand + NB * kCertCand * 2;                 // [NB][kCertTies] uint16
  static constexpr int kRows = (kTies + NB * kCertTies * 2 + 127) & ~127;
};

// Appends this lane's candidates and near ties (mask bits: bit i < 16 -> group p, else group
// p + G2; output 16 (i & 15) + r) to the row's two lists: one warp reduction and one atomic on
// the packed counter reserve the warp's entries in both lists (neither half can carry: a row
// has at most 16384 outputs), then one ballot round per set bit places each lane's entries.
// On overflow the record is flagged instead.
__device__ __forceinline__ void cert_append(uint32_t cand, uint32_t near, int p, int G2, int r, int lane,
                                            uint16_t* clist, uint16_t* tlist, uint32_t* counts, uint32_t* flags) {
  const uint32_t mine = (static_cast<uint32_t>(__popc(cand)) << 16) | static_cast<uint32_t>(__popc(near));
  const uint32_t total = __reduce_add_sync(0xffffffffu, mine);
  if (total == 0u) return;
  uint32_t base = 0;
  if (lane == 0) base = atomicAdd(counts, total);
  base = __shfl_sync(0xffffffffu, base, 0);
  uint32_t kc = base >> 16, kt = base & 0xffffu;
  if (kc + (total >> 16) > static_cast<uint32_t>(kCertCand) || kt + (total & 0xffffu) > static_cast<uint32_t>(kCertTies)) {
    if (lane == 0) atomicOr(flags, kCertOverflow);
    return;
  }
  const uint32_t lt = (1u << lane) - 1u;
  while (__any_sync(0xffffffffu, (cand | near) != 0u)) {
    const bool hc = cand != 0u, ht = near != 0u;
    const uint32_t bc = __ballot_sync(0xffffffffu, hc), bt = __ballot_sync(0xffffffffu, ht);
    if (hc) {
      const int bit = __ffs(cand) - 1;
      cand &= cand - 1u;
      clist[kc + __popc(bc & lt)] = static_cast<uint16_t>((bit < 16 ? p : p + G2) * 256 + 16 * (bit & 15) + r);
    }
    if (ht) {
      const int bit = __ffs(near) - 1;
      near &= near - 1u;
      tlist[kt + __popc(bt & lt)] = static_cast<uint16_t>((bit < 16 ? p : p + G2) * 256 + 16 * (bit & 15) + r);
    }
    kc += __popc(bc);
    kt += __popc(bt);
  }
}

// Block barrier of the streamer warps (mbarrier, one arrival per warp, bounded wait).
__device__ __forceinline__ bool cert_streamer_sync(uint64_t* cbar, uint32_t& parity, int lane) {
  __syncwarp();
  if (lane == 0) mbar_arrive(cbar);
  const bool ok = mbar_wait(cbar, parity, kErrWaitTimeoutEpilogue);
  parity ^= 1u;
  return __all_sync(0xffffffffu, ok);
}

// Row scale from the maximum in S units (slimdit/int8.py:49: max(fl(absmax / 127), 1e-30)).
__device__ __forceinline__ float cert_scale(float absmax_s) { return row_scale_from_absmax(__fmul_rn(absmax_s, 0.0625f)); }

// Persistent over rows. Streamer warps (all but the last NF): a row of G groups is split into
// G2 = ceil(G/2) group pairs (g, g + G2), 16 threads per pair; thread (p, r) holds chunk r (16
// consecutive inputs) of both groups as the two lanes of packed fp32x2 registers. They compute
// S', the certificates, the row maximum bounds, the scale (or, when the maximum is uncertain, an
// interval that contains it), provisional codes, and list the outputs whose chain is needed.
// NF fixer warps (the last ones) follow the streamers: a fixer runs the listed chains of a row
// from its staging buffer in shared memory (one output per lane), settles the row's scale and
// codes, and then restages the buffer with the row NB iterations on. Rows arrive by bulk copies
// into NB buffers (iteration i uses buffer i % NB), so the streamers run up to NB - 1 rows ahead
// of the fixers: a fixer's chains plus the restaging copy hide behind NB - 1 streamer rows.
template <int DT, int MAXR, int NF, int NB, bool XH>
__global__ void __maxnreg__(MAXR) cert_rotate_quant_kernel(const void* __restrict__ x, int64_t rows, int K,
                                                           int8_t* __restrict__ q_out,
                                                           float* __restrict__ scale_out) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  constexpr int kEsz = CertFmt<DT>::kEsz;
  const uint32_t row_bytes = static_cast<uint32_t>(K) * kEsz;
  const int t = threadIdx.x;
  const int warp = t >> 5, lane = t & 31;
  const int ns = (blockDim.x >> 5) - NF;  // streamer warps; the last NF warps are the fixers
  using L = CertLayout<NB>;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw + L::kFull);
  uint64_t* done = reinterpret_cast<uint64_t*>(smem_raw + L::kDone);
  uint64_t* cbar = reinterpret_cast<uint64_t*>(smem_raw + L::kCbar);
  volatile uint32_t* fail_flag = reinterpret_cast<volatile uint32_t*>(smem_raw + L::kFail);
  float* red = reinterpret_cast<float*>(smem_raw + L::kRed);  // [2 parities][3 kinds][16 warps]
  CertRec* recs = reinterpret_cast<CertRec*>(smem_raw + L::kRec);
  uint8_t* c0tabs = smem_raw + L::kC0;                           // [NB][64]
  uint16_t* cands = reinterpret_cast<uint16_t*>(smem_raw + L::kCand);  // [NB][kCertCand]
  uint16_t* ties = reinterpret_cast<uint16_t*>(smem_raw + L::kTies);   // [NB][kCertTies]
  unsigned char* rowbuf = smem_raw + L::kRows;                   // NB staged rows
  float2* xbuf = reinterpret_cast<float2*>(rowbuf + NB * static_cast<size_t>(row_bytes));
  const unsigned char* src = static_cast<const unsigned char*>(x);
  const int G = K >> 8;
  const int G2 = (G + 1) >> 1;

  if (t == 0) {
    for (int b = 0; b < NB; ++b) {
      mbar_init(&full[b], 1);
      mbar_init(&done[b], static_cast<uint32_t>(ns));
    }
    mbar_init(cbar, static_cast<uint32_t>(ns));
    *fail_flag = 0u;
    for (int b = 0; b < NB; ++b) {
      recs[b].counts = 0u;
      recs[b].flags = 0u;
    }
    fence_mbar_init();
  }
  __syncthreads();
  if (t == 0) {
    for (int b = 0; b < NB; ++b) {
      const int64_t rb = blockIdx.x + b * static_cast<int64_t>(gridDim.x);
      if (rb < rows) {
        mbar_arrive_expect_tx(&full[b], row_bytes);
        bulk_load(rowbuf + b * row_bytes, src + rb * row_bytes, row_bytes, &full[b]);
      }
    }
  }

  if (warp < ns) {
    // ------------------------------------------------------------ streamers
    const int p = t >> 4;  // group pair
    const int r = t & 15;  // chunk within the group
    const bool act_a = p < G2;
    const bool act_b = p + G2 < G;
    const int h = (lane >> 4) & 1;
    // transpose buffer: XH = the x and y lanes in turn through 256 floats per half-warp, else
    // both at once through 256 float2
    float2* gbuf = XH ? reinterpret_cast<float2*>(reinterpret_cast<float*>(xbuf) + (warp * 2 + h) * 256)
                      : xbuf + (warp * 2 + h) * 256;
    float* hb = reinterpret_cast<float*>(gbuf);
    uint32_t cparity = 0;
    int64_t row = blockIdx.x;
    for (int it = 0; row < rows; row += gridDim.x, ++it) {
      const int b = it % NB;
      const int par = it & 1;  // slot of the warp partials
      if (!mbar_wait(&full[b], (it / NB) & 1, kErrWaitTimeoutProducer)) *fail_flag = 1u;
      CertRec* rc = recs + b;
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
        if (XH) {
#pragma unroll
          for (int i = 0; i < 16; i += 4)
            *reinterpret_cast<float4*>(hb + xposf(r, i, h)) = make_float4(v[i].x, v[i + 1].x, v[i + 2].x, v[i + 3].x);
        } else {
#pragma unroll
          for (int i = 0; i < 16; i += 2)
            *reinterpret_cast<float4*>(gbuf + xpos2(r, i)) = make_float4(v[i].x, v[i].y, v[i + 1].x, v[i + 1].y);
        }
      }
      int c0a, c0b;
      float Da = cert_group_bound<DT>(l1a, mna, r, lane, c0a);
      float Db = cert_group_bound<DT>(l1b, mnb, r, lane, c0b);
      if (!act_a) Da = 0.0f;
      if (!act_b) Db = 0.0f;
      if (r == 0) {
        if (act_a) c0tabs[b * 64 + p] = static_cast<uint8_t>(c0a);
        if (act_b) c0tabs[b * 64 + p + G2] = static_cast<uint8_t>(c0b);
      }
      __syncwarp();
      float ama = 0.0f, amb = 0.0f;
      if (XH) {  // the y lanes after the x lanes (warp-wide syncs outside the per-pair branch)
        if (act_a) {
#pragma unroll
          for (int rr = 0; rr < 16; ++rr) v[rr].x = hb[xposf(rr, r, h)];
        }
        __syncwarp();
        if (act_a) {
#pragma unroll
          for (int i = 0; i < 16; i += 4)
            *reinterpret_cast<float4*>(hb + xposf(r, i, h)) = make_float4(v[i].y, v[i + 1].y, v[i + 2].y, v[i + 3].y);
        }
        __syncwarp();
        if (act_a) {
#pragma unroll
          for (int rr = 0; rr < 16; ++rr) v[rr].y = hb[xposf(rr, r, h)];
        }
      }
      if (act_a) {
        if (!XH) {
#pragma unroll
          for (int rr = 0; rr < 16; ++rr) v[rr] = gbuf[xpos2(rr, r)];
        }
        bfly16x2(v);  // digits 2, 3: lanes hold S' for outputs 16 rr + r of groups p and p + G2
#pragma unroll
        for (int rr = 0; rr < 16; ++rr) {
          ama = fmaxf(ama, fabsf(v[rr].x));
          amb = fmaxf(amb, fabsf(v[rr].y));
        }
      }
      {  // row maximum bounds: one redux per kind and warp, one barrier of the streamers
        const float tA0 = fmaxf(Da == 0.0f ? ama : 0.0f, Db == 0.0f ? amb : 0.0f);
        const float tA = fmaxf(fmaxf(__fsub_rd(ama, Da), __fsub_rd(amb, Db)), 0.0f);
        const float tB = fmaxf(Da > 0.0f ? __fadd_ru(ama, Da) : 0.0f, Db > 0.0f ? __fadd_ru(amb, Db) : 0.0f);
        const unsigned w0 = __reduce_max_sync(0xffffffffu, __float_as_uint(tA0));
        const unsigned w1 = __reduce_max_sync(0xffffffffu, __float_as_uint(tA));
        const unsigned w2 = __reduce_max_sync(0xffffffffu, __float_as_uint(tB));
        if (lane == 0) {
          red[(par * 3 + 0) * 16 + warp] = __uint_as_float(w0);
          red[(par * 3 + 1) * 16 + warp] = __uint_as_float(w1);
          red[(par * 3 + 2) * 16 + warp] = __uint_as_float(w2);
        }
      }
      if (!cert_streamer_sync(cbar, cparity, lane) || *fail_flag != 0u) break;  // error recorded
      const float A0 = __uint_as_float(__reduce_max_sync(0xffffffffu, lane < ns ? __float_as_uint(red[(par * 3 + 0) * 16 + lane]) : 0u));
      const float A = __uint_as_float(__reduce_max_sync(0xffffffffu, lane < ns ? __float_as_uint(red[(par * 3 + 1) * 16 + lane]) : 0u));
      const float B = __uint_as_float(__reduce_max_sync(0xffffffffu, lane < ns ? __float_as_uint(red[(par * 3 + 2) * 16 + lane]) : 0u));
      // the scale, or (maximum uncertain) an interval [s_lo, s_hi] that contains it; codes are
      // taken from S' rm, and an output's code is certain unless S' rm lies within
      // 2^-13 + D r_hi + |S'| w of a half-integer (w covers the interval; 0 for a certain scale)
      const bool unsure = B >= A && B > 0.0f;
      const float top = unsure ? fmaxf(A0, B) : A0;
      const float scale = cert_scale(unsure ? A : A0);  // s_lo when unsure (provisional codes)
      const float rm = __frcp_rn(__fmul_rn(16.0f, scale));
      float w = 0.0f;
      if (unsure)
        w = __fmaf_ru(rm, 2.384185791015625e-07f,
                      __fsub_ru(__frcp_ru(__fmul_rn(16.0f, scale)), __frcp_rd(__fmul_rn(16.0f, cert_scale(top)))));
      const bool tiny_row = top < 8.271806125530277e-25f;  // 2^-80: S / 16 could be subnormal
      if (t == 0) {
        rc->a0 = A0;
        rc->scale = scale;
        if (unsure) atomicOr(&rc->flags, kCertUnsure);
        else scale_out[row] = scale;
      }
      const int64_t rbase = row * static_cast<int64_t>(K);
      uint32_t near = 0, cand = 0;  // bit rr: group p, bit 16 + rr: group p + G2
      __syncwarp();
      uint16_t* cbuf = reinterpret_cast<uint16_t*>(gbuf);
      if (act_a) {
        const float lim_a = __fsub_rd(0.5f, __fmaf_ru(Da, __fmul_ru(rm, 1.0009765625f), 1.220703125e-4f));
        const float lim_b = __fsub_rd(0.5f, __fmaf_ru(Db, __fmul_ru(rm, 1.0009765625f), 1.220703125e-4f));
        near = unsure ? cert_codes<true>(v, rm, w, lim_a, lim_b, cbuf, r) : cert_codes<false>(v, rm, w, lim_a, lim_b, cbuf, r);
        if (tiny_row) near = ~0u;
        if (!act_b) near &= 0xffffu;
        // a thread's outputs of a group can hold the maximum only if its largest |S'| + D reaches
        // A (upward rounding is monotone), so most threads skip the per-output test
        const bool ca = Da > 0.0f && __fadd_ru(ama, Da) >= A;
        const bool cb = Db > 0.0f && __fadd_ru(amb, Db) >= A;
        if (unsure) {
          if (ca || cb) {
#pragma unroll
            for (int rr = 0; rr < 16; ++rr) {
              if (ca && __fadd_ru(fabsf(v[rr].x), Da) >= A) cand |= 1u << rr;
              if (cb && __fadd_ru(fabsf(v[rr].y), Db) >= A) cand |= 1u << (16 + rr);
            }
          }
        } else {
          // exact groups with a certain scale: S' = S_ref, the IEEE division settles the code here
          uint32_t ex = near & ~((Da > 0.0f ? 0x0000ffffu : 0u) | (Db > 0.0f ? 0xffff0000u : 0u));
          near &= ~ex;
          while (ex != 0u) {
            const int bit = __ffs(ex) - 1;
            ex &= ex - 1u;
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
      cert_append(cand, near, p, G2, r, lane, cands + b * kCertCand, ties + b * kCertTies, &rc->counts, &rc->flags);
      // provisional codes and lists complete before the fixer takes the row
      __threadfence_block();
      __syncwarp();
      if (lane == 0) mbar_arrive(&done[b]);
    }
  } else {
    // ------------------------------------------------------------ fixers
    // Fixer f takes the rows of iterations f, f + NF, ...; one output per lane.
    for (int it = warp - ns; blockIdx.x + static_cast<int64_t>(it) * gridDim.x < rows; it += NF) {
      const int b = it % NB;
      const int64_t row = blockIdx.x + static_cast<int64_t>(it) * gridDim.x;
      if (!mbar_wait(&done[b], (it / NB) & 1, kErrWaitTimeoutDrain)) break;  // streamers stopped
      CertRec* rc = recs + b;
      unsigned char* buf = rowbuf + b * row_bytes;
      const uint8_t* c0tab = c0tabs + b * 64;
      const uint32_t flags = rc->flags;
      const int64_t rbase = row * static_cast<int64_t>(K);
      float scale = rc->scale;
      float m = rc->a0;
      if (flags & kCertOverflow) {
        // every output by its chain: the maximum first (phase 0), then the codes (phase 1)
        for (int phase = 0; phase < 2; ++phase) {
          for (int col = lane; col < K; col += 32) {
            const float S = cert_chain<DT>(buf + (col & ~255) * kEsz, col & 255, c0tab[col >> 8]);
            if (phase == 0) m = fmaxf(m, fabsf(S));
            else q_out[rbase + col] = quant_code(__fmul_rn(S, 0.0625f), scale);
          }
          if (phase == 0) {
            m = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(m)));
            scale = cert_scale(m);
            if (lane == 0) scale_out[row] = scale;
          }
        }
      } else {
        // one pass per 32 listed outputs, the candidates first: a chain's value does not depend
        // on the scale, so a near-tie output in the pass that completes the candidates takes its
        // code as soon as their maximum settles the scale
        const bool unsure = (flags & kCertUnsure) != 0u;
        const uint32_t cnt = rc->counts;
        const int nc = unsure ? static_cast<int>(cnt >> 16) : 0;
        const int n = nc + static_cast<int>(cnt & 0xffffu);
        bool settled = !unsure;
        for (int base = 0; base < n; base += 32) {
          const int e = base + lane;
          int col = 0;
          float S = 0.0f;
          if (e < n) {
            col = e < nc ? cands[b * kCertCand + e] : ties[b * kCertTies + (e - nc)];
            S = cert_chain<DT>(buf + (col & ~255) * kEsz, col & 255, c0tab[col >> 8]);
          }
          if (!settled) {
            if (e < nc) m = fmaxf(m, fabsf(S));
            if (base + 32 >= nc) {  // every candidate is done (the same for all lanes)
              m = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(m)));
              scale = cert_scale(m);
              if (lane == 0) scale_out[row] = scale;
              settled = true;
            }
          }
          if (e >= nc && e < n) q_out[rbase + col] = quant_code(__fmul_rn(S, 0.0625f), scale);
        }
        if (!settled) {  // an uncertain row with nothing listed: the exact part is the maximum
          scale = cert_scale(m);
          if (lane == 0) scale_out[row] = scale;
        }
      }
      __syncwarp();
      if (lane == 0) {  // the buffer is free: reset the record, stage the row NB iterations on
        rc->counts = 0u;
        rc->flags = 0u;
        const int64_t rn = row + NB * static_cast<int64_t>(gridDim.x);
        if (rn < rows) {
          fence_proxy_async_smem();
          mbar_arrive_expect_tx(&full[b], row_bytes);
          bulk_load(buf, src + rn * row_bytes, row_bytes, &full[b]);
        }
      }
      __syncwarp();
    }
  }
}

// Configuration by row width. Rows of up to 40 groups: one fixer warp, 80 registers, full
// float2 transposes (four CTAs per SM at K = 5120, two up to 44 groups). Wider rows: two fixer
// warps, 64 registers and the half-size transpose buffer, which is what lets three staged rows of
// K = 13824 keep two CTAs per SM. Measured on B200 (bit-identical outputs), the narrow
// configuration against the wide one: 0.646 vs 0.803 ms at 65536 x 6400, 0.655 vs 0.811 at
// x 7168, 0.827 vs 0.878 at x 8192, 0.438 vs 0.510 at 32768 x 9216, 0.505 vs 0.547 at x 10240;
// at 44 groups it depends on the input (0.544 vs 0.576 ms on activations, 0.647 vs 0.623 on a
// GELU hidden); from 48 groups on it holds one CTA per SM and loses (0.768 vs 0.610 at x 12288,
// 1.09 vs 0.74 on the FFN hidden at x 13824). Three staged rows where they fit in a CTA's shared memory without fewer CTAs per SM
// than two would give, else two: measured on B200 (bit-identical outputs), 32768 x 5120 bf16
// activations 0.269 -> 0.266 ms and the FFN hidden 115200 x 13824 2.91 -> 2.73 ms with three;
// four rows, or the half transpose on narrow rows (+11 % time), were slower.
static bool cert_wide(int K) { return (K >> 8) > 40; }
static int cert_fixers(int K) { return cert_wide(K) ? 2 : 1; }
constexpr size_t kCertSmemPerSM = 233472, kCertSmemPerBlock = 232448, kCertSmemReserved = 1024;  // sm_100

static size_t cert_smem_bytes_nb(int K, int dtype, int threads, int nb) {
  const size_t esz = dtype == kF32 ? 4 : 2;
  const size_t ns = static_cast<size_t>(threads / 32 - cert_fixers(K));
  const size_t head = nb == 3 ? CertLayout<3>::kRows : CertLayout<2>::kRows;
  return head + nb * esz * static_cast<size_t>(K) + ns * (cert_wide(K) ? 2048 : 4096);
}

static int cert_buffers(int K, int dtype, int threads) {
  const size_t s3 = cert_smem_bytes_nb(K, dtype, threads, 3), s2 = cert_smem_bytes_nb(K, dtype, threads, 2);
  if (s3 > kCertSmemPerBlock) return 2;
  const size_t cap = std::min(static_cast<size_t>(65536 / (threads * (cert_wide(K) ? 64 : 80))),
                              static_cast<size_t>(2048 / threads));
  const size_t per3 = std::min(cap, kCertSmemPerSM / (s3 + kCertSmemReserved));
  const size_t per2 = std::min(cap, kCertSmemPerSM / (s2 + kCertSmemReserved));
  return per3 >= per2 ? 3 : 2;
}

size_t cert_smem_bytes(int K, int dtype, int threads) {
  return cert_smem_bytes_nb(K, dtype, threads, cert_buffers(K, dtype, threads));
}

template <bool kWide, int NB>
static void (*cert_kernel_for(int dtype))(const void*, int64_t, int, int8_t*, float*) {
  constexpr int kMaxR = kWide ? 64 : 80, kNF = kWide ? 2 : 1;
  return dtype == kBF16 ? cert_rotate_quant_kernel<kBF16, kMaxR, kNF, NB, kWide>
                        : (dtype == kF32 ? cert_rotate_quant_kernel<kF32, kMaxR, kNF, NB, kWide>
                                         : cert_rotate_quant_kernel<kF16, kMaxR, kNF, NB, kWide>);
}

// Rows of 5 <= K/256 <= 64 groups: the streamer warps (16 threads per group pair) plus the fixers.
cudaError_t launch_cert_rotate_quant(const void* x, int dtype, int64_t rows, int K, int8_t* q, float* scale,
                                     cudaStream_t st) {
  const int g2 = ((K >> 8) + 1) >> 1;
  const int nf = cert_fixers(K);
  const int threads = (g2 + 1) / 2 * 32 + 32 * nf;
  const int nb = cert_buffers(K, dtype, threads);
  const size_t smem = cert_smem_bytes_nb(K, dtype, threads, nb);
  void (*fn)(const void*, int64_t, int, int8_t*, float*) =
      cert_wide(K) ? (nb == 3 ? cert_kernel_for<true, 3>(dtype) : cert_kernel_for<true, 2>(dtype))
                   : (nb == 3 ? cert_kernel_for<false, 3>(dtype) : cert_kernel_for<false, 2>(dtype));
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  int per_sm = 1;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  const int grid = grid_for_rows(rows, per_sm);
  fn<<<grid, threads, smem, st>>>(x, rows, K, q, scale);
  return cudaGetLastError();
}

}  // namespace slim
