// INT8 x INT8 -> INT32 GEMM on the sm_100a 5th-generation tensor cores (tcgen05 kind::i8)
// with a dequantising epilogue:
//
//   out[m, n] = bf16( float(sum_k A[m,k] * B[n,k]) * (sa[m] * sb[n]) + bias[n] )
//
// which is the runtime side of the convrot linear: `x_rot @ (q * scale)^T` with the
// activation quantised per token (slimdit/int8.py:9-11; the runtime op that the reference
// calls is comfy_kitchen.int8_linear, tools/bench_int8.py:65-68). A is the token matrix, B
// the weight codes; both are K-major (row-major with K contiguous), i.e. a "TN" GEMM.
//
// Structure (one CTA per SM, persistent over output tiles of 128 x 256):
//   warp 0      TMA producer: 128x128-byte A and 256x128-byte B tiles, 128-byte swizzle,
//               4-stage shared-memory ring guarded by full/empty mbarriers.
//   warp 1      allocates 512 TMEM columns (two 256-column int32 accumulators) and one
//               lane issues tcgen05.mma (M=128, N=256, K=32 per instruction, 4 per stage),
//               committing to the ring's empty barriers and to the accumulator barriers.
//   warps 2..5  epilogue: tcgen05.ld of the accumulator rows (warp w owns TMEM lanes
//               32*(w%4)..+31), scale/bias/GELU in fp32, bf16 rows staged in shared memory
//               (two 4 KB slices per warp) and written by TMA tensor stores, or, when the
//               output also goes to other GPUs or an int32 copy is asked for, by the warp with
//               each store instruction covering four 128-byte row segments; double-buffered
//               accumulators let the next tile's MMAs run under this epilogue. (Stored
//               straight from the registers, one row per thread, the 16-byte writes of 32 rows
//               per instruction slowed the MMAs sharing the SM's load/store path: 2.14 vs 2.01
//               ms at 32768 x 15360 x 5120.)
// Every mbarrier wait is bounded (slim_ptx.cuh); on a timeout the kernel records an error,
// drains its own TMA loads and MMAs, frees TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <cstring>

#include "slim_kernels.h"
#include "slim_ptx.cuh"

namespace slim {
namespace gi8 {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 128;  // bytes == int8 elements: one 128-byte swizzle row
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK;
constexpr int B_BYTES = BN * BK;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int THREADS = 192;
constexpr int TMEM_COLS = 512;
constexpr int GROUP_M = 16;
constexpr int MMA_K = 32;
constexpr uint32_t IDESC = idesc_i8(BM, BN);

constexpr int EPI_WARPS = 4;
constexpr int SLICE_BYTES = 32 * 128;       // one write-back slice: 32 rows x 64 bf16
constexpr int STAGING_BYTES = 2 * SLICE_BYTES;  // per epilogue warp: two slices in flight

struct Shared {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t drain;
  uint32_t tmem_base;
  volatile int abort;
};

constexpr size_t SMEM_BYTES =
    1024 + static_cast<size_t>(STAGES) * STAGE_BYTES + EPI_WARPS * STAGING_BYTES + sizeof(Shared) + 64;
static_assert(SMEM_BYTES <= 232448, "shared memory budget");

__device__ __forceinline__ void tile_coords(int64_t t, int tiles_m, int tiles_n, int& tm, int& tn) {
  const int64_t per_group = static_cast<int64_t>(GROUP_M) * tiles_n;
  const int64_t g = t / per_group;
  const int first_m = static_cast<int>(g * GROUP_M);
  const int gm = min(tiles_m - first_m, GROUP_M);
  const int local = static_cast<int>(t - g * per_group);
  tm = first_m + local % gm;
  tn = local / gm;
}

// GELU with the tanh approximation, 0.5 x (1 + tanh(u)) with u = sqrt(2/pi) (x + 0.044715 x^3),
// evaluated as the identical x / (1 + e^(-2u)) = x / (1 + 2^(x (c1 + c3 x^2))): one hardware ex2
// and one hardware reciprocal (relative errors below 2^-21), seven instructions, so the
// epilogue keeps pace with the tensor cores. Very negative x: the power overflows to +inf and
// the result is -0; very positive x: the power underflows to 0 and the result is x.
__device__ __forceinline__ float gelu_tanh(float x) {
  constexpr float kC1 = -2.0f * 0.7978845608028654f * 1.4426950408889634f;  // -2 sqrt(2/pi) log2(e)
  constexpr float kC3 = kC1 * 0.044715f;
  const float p = __fmul_rn(x, __fmaf_rn(kC3, __fmul_rn(x, x), kC1));
  return __fmul_rn(x, rcp_approx(__fadd_rn(1.0f, ex2_approx(p))));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ float bf16_round(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

// Eight scale/bias-applied outputs y = bf16(acc * sa * sb[n] + bias[n]) as fp32, columns n0..n0+7.
__device__ __forceinline__ void linear8(const GemmI8Params& p, const uint32_t* r, float sam, int64_t n0, float (&y)[8]) {
  const __nv_bfloat16* bias = static_cast<const __nv_bfloat16*>(p.bias);
  const float4 s0 = __ldg(reinterpret_cast<const float4*>(p.sb + n0));
  const float4 s1 = __ldg(reinterpret_cast<const float4*>(p.sb + n0 + 4));
  const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
  float bv[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (bias != nullptr) {
    const uint4 bu = __ldg(reinterpret_cast<const uint4*>(bias + n0));
    const uint32_t bw[4] = {bu.x, bu.y, bu.z, bu.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      bv[2 * e] = __uint_as_float(bw[e] << 16);
      bv[2 * e + 1] = __uint_as_float(bw[e] & 0xffff0000u);
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e)
    y[e] = bf16_round(__fmaf_rn(static_cast<float>(static_cast<int>(r[e])), sam * sv[e], bv[e]));
}

// Write-back of one slice of a warp's 32 bf16 output rows [m0, m0+32) x [n0, n0 + ROW_BYTES/2):
// lane i holds row m0 + i's ROW_BYTES bytes (w). The rows go to the warp's staging buffer in
// shared memory (16-byte chunk j of row r at chunk position j ^ ((r / (8/CH)) % CH), so that
// neither the row-wise writes nor the column-wise reads conflict), then each store instruction
// writes 32 x 16 bytes as whole row segments: 4 rows x 128 bytes, 8 x 64 or 16 x 32. Rows >= M
// and columns >= N are skipped; the same bytes go to each of the n_peer further destinations.
// All 32 lanes must call it.
template <int ROW_BYTES>
__device__ __forceinline__ void store_rows_staged(__nv_bfloat16* out, void* const* peers, int n_peer, int64_t ldo,
                                                  int64_t M, int64_t N, uint8_t* stg, const uint32_t* w, int64_t m0,
                                                  int64_t n0, int lane) {
  constexpr int CH = ROW_BYTES / 16;  // 16-byte chunks per row
  constexpr int RPI = 32 / CH;        // rows per store instruction
  static_assert(CH == 2 || CH == 4 || CH == 8, "row slice of 32, 64 or 128 bytes");
  auto swz = [](int r) { return (r / (8 / CH)) % CH; };
  uint4* srow = reinterpret_cast<uint4*>(stg + lane * ROW_BYTES);
#pragma unroll
  for (int j = 0; j < CH; ++j) srow[j ^ swz(lane)] = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
  __syncwarp();
  const int j = lane % CH;
  const bool col_ok = n0 + 8 * j < N;
#pragma unroll
  for (int i = 0; i < CH; ++i) {
    const int r = RPI * i + lane / CH;
    const uint4 v = reinterpret_cast<const uint4*>(stg + r * ROW_BYTES)[j ^ swz(r)];
    const int64_t m = m0 + r;
    if (col_ok && m < M) {
      const int64_t off = m * ldo + n0 + 8 * j;
      *reinterpret_cast<uint4*>(out + off) = v;
#pragma unroll
      for (int d = 0; d < kMaxPeers; ++d)
        if (d < n_peer) *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(peers[d]) + off) = v;
    }
  }
  __syncwarp();  // the staging rows are read before the next slice overwrites them
}

// The same slice written by a TMA tensor store (box ROW_BYTES/2 columns x 32 rows, swizzle
// matching the staging layout: 32/64/128-byte swizzle for 32/64/128-byte rows). The warp's NBUF
// staging slices of 32 x ROW_BYTES bytes take turns; lane 0 issues the store and, before a slice
// is refilled, waits until the store issued from it NBUF slices earlier has read it. Rows >= M
// and columns >= N fall outside the tensor map and are not written; m0 must be < M.
template <int ROW_BYTES, int NBUF = 2>
__device__ __forceinline__ void tma_store_slice(const CUtensorMap* tmo, uint8_t* stg, const uint32_t* w, int64_t m0,
                                                int64_t n0, int lane, uint32_t& slice) {
  constexpr int CH = ROW_BYTES / 16;
  auto swz = [](int r) { return (r / (8 / CH)) % CH; };
  uint8_t* buf = stg + (slice % NBUF) * (32 * ROW_BYTES);
  if (lane == 0) bulk_wait_group_read<NBUF - 1>();
  __syncwarp();
  uint4* srow = reinterpret_cast<uint4*>(buf + lane * ROW_BYTES);
#pragma unroll
  for (int j = 0; j < CH; ++j) srow[j ^ swz(lane)] = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
  fence_proxy_async_smem();  // the rows, written through the generic proxy, are read by TMA
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(tmo, buf, static_cast<int32_t>(n0), static_cast<int32_t>(m0));
    bulk_commit_group();
  }
  ++slice;
}

// One slice through TMA when a tensor map is given, else through the warp's own stores.
template <int ROW_BYTES>
__device__ __forceinline__ void store_slice(const GemmI8Params& p, const CUtensorMap* tmo, uint8_t* stg,
                                            const uint32_t* w, int64_t m0, int64_t n0, int lane, uint32_t& slice) {
  if (tmo != nullptr) {
    if (m0 < p.M) tma_store_slice<ROW_BYTES>(tmo, stg, w, m0, n0, lane, slice);  // no box starts past the end
  } else {
    store_rows_staged<ROW_BYTES>(static_cast<__nv_bfloat16*>(p.out), p.peer_out, p.n_peer, p.ldo, p.M, p.N, stg, w,
                                 m0, n0, lane);
  }
}

// SwiGLU epilogue: the weight rows are interleaved per 256-row tile (128 "up" rows, then the 128
// matching "gate" rows), so the tile's columns [0,128) and [128,256) pair up; the output
// column n_base/2 + i gets bf16(up * bf16(silu(gate))), with up and gate the bf16 linear
// outputs: the roundings of running the linear in bf16 and then ComfyUI's swiglu on its output.
__device__ __forceinline__ void epilogue_rows_swiglu(const GemmI8Params& p, uint32_t tbase, int64_t m0, int lane,
                                                     float sam, int64_t n_base, uint8_t* stg, const CUtensorMap* tmo,
                                                     uint32_t& slice) {
  const int64_t o_base = n_base / 2;
#pragma unroll 1
  for (int c = 0; c < BN / 64; ++c) {
    uint32_t ru[32], rg[32];
    tmem_ld_32x32b_x32(tbase + c * 32, ru);
    tmem_ld_32x32b_x32(tbase + BN / 2 + c * 32, rg);
    tmem_ld_wait();
    const int64_t nu = n_base + c * 32, ng = n_base + BN / 2 + c * 32;
    if (nu >= p.N) continue;  // warp-uniform
    uint32_t w[16];
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
      float up[8], g[8];
      linear8(p, ru + j, sam, nu + j, up);
      linear8(p, rg + j, sam, ng + j, g);
      float y[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float sl = bf16_round(__fdiv_rn(g[e], __fadd_rn(1.0f, expf(-g[e]))));
        y[e] = __fmul_rn(up[e], sl);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) w[j / 2 + e] = pack_bf16x2(y[2 * e], y[2 * e + 1]);
    }
    store_slice<64>(p, tmo, stg, w, m0, o_base + c * 32, lane, slice);
  }
}

// One accumulator tile row-slice: this thread's row m0 + lane (TMEM lane), 256 columns from
// n_base, read 64 columns at a time; scale/bias(/GELU) in fp32, bf16 rows written back through
// the warp's staging buffer `stg` (by TMA when `tmo` is given), optional int32 copy. All 32
// lanes of the warp must call it (tcgen05.ld is warp-collective).
__device__ __forceinline__ void epilogue_rows(const GemmI8Params& p, uint32_t tbase, int64_t m0, int lane,
                                              bool row_ok, float sam, int64_t n_base, uint8_t* stg,
                                              const CUtensorMap* tmo, uint32_t& slice) {
  if (p.epilogue == kEpiSwiGLU) {
    epilogue_rows_swiglu(p, tbase, m0, lane, sam, n_base, stg, tmo, slice);
    return;
  }
  const int64_t m = m0 + lane;
  const __nv_bfloat16* bias = static_cast<const __nv_bfloat16*>(p.bias);
#pragma unroll 1
  for (int c = 0; c < BN / 64; ++c) {
    uint32_t r[64];
    tmem_ld_32x32b_x32(tbase + c * 64, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
    tmem_ld_32x32b_x32(tbase + c * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
    tmem_ld_wait();
    const int64_t n0 = n_base + c * 64;
    if (n0 >= p.N) continue;  // warp-uniform
    if (row_ok && p.acc_dbg != nullptr) {
      int32_t* dst = p.acc_dbg + m * p.N + n0;
#pragma unroll
      for (int j = 0; j < 64; j += 4) {
        if (n0 + j < p.N)
          *reinterpret_cast<int4*>(dst + j) = make_int4(static_cast<int>(r[j]), static_cast<int>(r[j + 1]),
                                                        static_cast<int>(r[j + 2]), static_cast<int>(r[j + 3]));
      }
    }
    uint32_t w[32];
#pragma unroll
    for (int j = 0; j < 64; j += 8) {
      if (n0 + j >= p.N) {  // past the last column (N % 8 == 0): nothing of these 8 is stored
#pragma unroll
        for (int e = 0; e < 4; ++e) w[j / 2 + e] = 0u;
        continue;
      }
      const float4 s0 = __ldg(reinterpret_cast<const float4*>(p.sb + n0 + j));
      const float4 s1 = __ldg(reinterpret_cast<const float4*>(p.sb + n0 + j + 4));
      const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
      float bv[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (bias != nullptr) {
        const uint4 bu = __ldg(reinterpret_cast<const uint4*>(bias + n0 + j));
        const uint32_t bw[4] = {bu.x, bu.y, bu.z, bu.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          bv[2 * e] = __uint_as_float(bw[e] << 16);
          bv[2 * e + 1] = __uint_as_float(bw[e] & 0xffff0000u);
        }
      }
      float y[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float acc = static_cast<float>(static_cast<int>(r[j + e]));
        y[e] = __fmaf_rn(acc, sam * sv[e], bv[e]);
        if (p.epilogue == kEpiGeluTanh) y[e] = gelu_tanh(bf16_round(y[e]));
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) w[j / 2 + e] = pack_bf16x2(y[2 * e], y[2 * e + 1]);
    }
    store_slice<128>(p, tmo, stg, w, m0, n0, lane, slice);
  }
}

__global__ void __launch_bounds__(THREADS, 1)
gemm_i8_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
               const __grid_constant__ CUtensorMap tma_o, const GemmI8Params p, int tiles_m, int tiles_n,
               int tma_store) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023) & ~1023u) - raw_addr);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* staging = smem + STAGES * STAGE_BYTES;
  Shared& sh = *reinterpret_cast<Shared*>(staging + EPI_WARPS * STAGING_BYTES);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t total_tiles = static_cast<int64_t>(tiles_m) * tiles_n;
  const int num_kb = static_cast<int>((p.K + BK - 1) / BK);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&sh.tfull[a], 1);
      mbar_init(&sh.tempty[a], 128);
    }
    mbar_init(&sh.drain, 1);
    sh.abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&sh.tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = sh.tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tma_a);
      tma_prefetch_desc(&tma_b);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0, last_parity = 0;
      for (int64_t t = blockIdx.x; t < total_tiles && !sh.abort; t += gridDim.x) {
        int tm, tn;
        tile_coords(t, tiles_m, tiles_n, tm, tn);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&sh.empty[stage], phase ^ 1, kErrWaitTimeoutProducer)) {
            sh.abort = 1;
            break;
          }
          if (sh.abort) break;
          mbar_arrive_expect_tx(&sh.full[stage], STAGE_BYTES);
          tma_load_2d(sA + stage * A_BYTES, &tma_a, &sh.full[stage], kb * BK, tm * BM);
          tma_load_2d(sB + stage * B_BYTES, &tma_b, &sh.full[stage], kb * BK, tn * BN);
          issued |= 1u << stage;
          last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Every load this thread issued must land before the CTA may exit.
      for (int s = 0; s < STAGES; ++s)
        if (issued & (1u << s)) mbar_wait(&sh.full[s], (last_parity >> s) & 1, kErrWaitTimeoutDrain);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int as = 0;
      uint32_t aphase = 0;
      bool issued_any = false;
      for (int64_t t = blockIdx.x; t < total_tiles && !sh.abort; t += gridDim.x) {
        if (!mbar_wait(&sh.tempty[as], aphase ^ 1, kErrWaitTimeoutMma)) {
          sh.abort = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(as * BN);
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&sh.full[stage], phase, kErrWaitTimeoutMma) || sh.abort) {
            sh.abort = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / MMA_K; ++kk) {
            mma_i8(d, smem_desc_sw128(a0 + kk * MMA_K), smem_desc_sw128(b0 + kk * MMA_K), IDESC,
                   (kb | kk) != 0 ? 1u : 0u);
          }
          issued_any = true;
          mma_commit(&sh.empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit(&sh.tfull[as]);
        as ^= 1;
        if (as == 0) aphase ^= 1;
      }
      // All issued MMAs must complete before TMEM is released.
      if (issued_any) {
        mma_commit(&sh.drain);
        mbar_wait(&sh.drain, 0, kErrWaitTimeoutDrain);
      }
    }
    __syncwarp();
  } else {
    // epilogue warps 2..5
    const int quarter = warp & 3;
    const CUtensorMap* tmo = tma_store ? &tma_o : nullptr;
    uint32_t slice = 0;
    int as = 0;
    uint32_t aphase = 0;
    for (int64_t t = blockIdx.x; t < total_tiles; t += gridDim.x) {
      bool ok = mbar_wait(&sh.tfull[as], aphase, kErrWaitTimeoutEpilogue);
      ok = __all_sync(0xffffffffu, ok) && !sh.abort;
      if (!ok) {
        sh.abort = 1;
        break;
      }
      tc_fence_after();
      int tm, tn;
      tile_coords(t, tiles_m, tiles_n, tm, tn);
      const int64_t m0 = static_cast<int64_t>(tm) * BM + quarter * 32;
      const bool row_ok = m0 + lane < p.M;
      const float sam = row_ok ? __ldg(p.sa + m0 + lane) : 0.0f;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>(as * BN);
      epilogue_rows(p, tbase, m0, lane, row_ok, sam, static_cast<int64_t>(tn) * BN,
                    staging + (warp - 2) * STAGING_BYTES, tmo, slice);
      tc_fence_before();
      mbar_arrive(&sh.tempty[as]);
      as ^= 1;
      if (as == 0) aphase ^= 1;
    }
    if (lane == 0) bulk_wait_group<0>();  // the tensor stores are complete before the CTA exits
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------- CTA-pair (2-SM) variant
// A cluster of two CTAs on two SMs computes 256 x 256 output tiles with
// tcgen05.mma.cta_group::2 (M = 256: 128 rows in each CTA; B split along N: each CTA loads
// 128 of the tile's 256 weight rows, the pair's MMA reads both halves). Per SM and K-block
// that is 16 KB of A + 16 KB of B instead of 16 + 32 KB, so the L2->SM feed per MMA drops by a
// third, and the 32 KB stages allow a 6-deep ring. Protocol:
//   * each CTA's producer waits on its own empty barrier and loads its halves; both CTAs'
//     loads complete on CTA 0's full barrier (cp.async.bulk.tensor .cta_group::2), which CTA
//     0's producer arms for 2 x 32 KB;
//   * one lane of CTA 0 issues the MMAs and commits to the empty / accumulator-full barriers
//     of both CTAs (one commit per CTA, no multicast);
//   * every epilogue thread of both CTAs arrives on CTA 0's accumulator-empty barrier (256).
namespace pair {
constexpr int BNH = 128;  // weight rows per CTA
constexpr int STAGES = 6;
constexpr int A_BYTES = BM * BK;
constexpr int B_BYTES = BNH * BK;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int GROUP_M2 = 16;  // 256-row tiles per raster group
constexpr uint32_t IDESC2 = idesc_i8(2 * BM, BN);

struct SharedP {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t drain;
  uint32_t tmem_base;
  volatile int abort;
};
constexpr size_t SMEM_BYTES =
    1024 + static_cast<size_t>(STAGES) * STAGE_BYTES + EPI_WARPS * STAGING_BYTES + sizeof(SharedP) + 64;
static_assert(SMEM_BYTES <= 232448, "shared memory budget");

__device__ __forceinline__ void tile_coords2(int64_t t, int tiles_m, int tiles_n, int& tm, int& tn) {
  const int64_t per_group = static_cast<int64_t>(GROUP_M2) * tiles_n;
  const int64_t g = t / per_group;
  const int first_m = static_cast<int>(g * GROUP_M2);
  const int gm = min(tiles_m - first_m, GROUP_M2);
  const int local = static_cast<int>(t - g * per_group);
  tm = first_m + local % gm;
  tn = local / gm;
}

// tiles_m counts 256-row tiles, tiles_n 256-column tiles.
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
gemm_i8_pair_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                    const __grid_constant__ CUtensorMap tma_o, const GemmI8Params p, int tiles_m, int tiles_n,
                    int tma_store) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023) & ~1023u) - raw_addr);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* staging = smem + STAGES * STAGE_BYTES;
  SharedP& sh = *reinterpret_cast<SharedP*>(staging + EPI_WARPS * STAGING_BYTES);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int64_t pair_id = blockIdx.x >> 1;
  const int64_t npairs = gridDim.x >> 1;
  const int64_t total_tiles = static_cast<int64_t>(tiles_m) * tiles_n;
  const int num_kb = static_cast<int>((p.K + BK - 1) / BK);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&sh.tfull[a], 1);
      mbar_init(&sh.tempty[a], 2 * 128);
    }
    mbar_init(&sh.drain, 1);
    sh.abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(&sh.tmem_base, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers are initialised before any remote arrive or load
  tc_fence_after();
  const uint32_t tmem_base = sh.tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tma_a);
      tma_prefetch_desc(&tma_b);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0, last_parity = 0;
      for (int64_t t = pair_id; t < total_tiles && !sh.abort; t += npairs) {
        int tm, tn;
        tile_coords2(t, tiles_m, tiles_n, tm, tn);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&sh.empty[stage], phase ^ 1, kErrWaitTimeoutProducer)) {
            sh.abort = 1;
            break;
          }
          if (sh.abort) break;
          const uint32_t full0 = mapa_shared(smem_u32(&sh.full[stage]), 0);
          if (rank == 0) mbar_arrive_expect_tx(&sh.full[stage], 2 * STAGE_BYTES);
          tma_load_2d_pair(sA + stage * A_BYTES, &tma_a, full0, kb * BK, tm * (2 * BM) + static_cast<int>(rank) * BM);
          tma_load_2d_pair(sB + stage * B_BYTES, &tma_b, full0, kb * BK, tn * BN + static_cast<int>(rank) * BNH);
          issued |= 1u << stage;
          last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Loads must land before the CTA may exit. CTA 0 watches its full barriers; CTA 1's
      // loads are consumed (and their stages released to its empty barriers) by the MMAs.
      for (int s = 0; s < STAGES; ++s) {
        if (!(issued & (1u << s))) continue;
        if (rank == 0) mbar_wait(&sh.full[s], (last_parity >> s) & 1, kErrWaitTimeoutDrain);
        else mbar_wait(&sh.empty[s], (last_parity >> s) & 1, kErrWaitTimeoutDrain);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int as = 0;
      uint32_t aphase = 0;
      bool issued_any = false;
      for (int64_t t = pair_id; t < total_tiles && !sh.abort; t += npairs) {
        if (!mbar_wait(&sh.tempty[as], aphase ^ 1, kErrWaitTimeoutMma)) {
          sh.abort = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(as * BN);
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&sh.full[stage], phase, kErrWaitTimeoutMma) || sh.abort) {
            sh.abort = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / MMA_K; ++kk) {
            mma_i8_pair(d, smem_desc_sw128(a0 + kk * MMA_K), smem_desc_sw128(b0 + kk * MMA_K), IDESC2,
                        (kb | kk) != 0 ? 1u : 0u);
          }
          issued_any = true;
          const uint32_t e = smem_u32(&sh.empty[stage]);
          mma_commit_pair(mapa_shared(e, 0));
          mma_commit_pair(mapa_shared(e, 1));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        const uint32_t f = smem_u32(&sh.tfull[as]);
        mma_commit_pair(mapa_shared(f, 0));
        mma_commit_pair(mapa_shared(f, 1));
        as ^= 1;
        if (as == 0) aphase ^= 1;
      }
      if (issued_any) {
        mma_commit_pair(mapa_shared(smem_u32(&sh.drain), 0));
        mbar_wait(&sh.drain, 0, kErrWaitTimeoutDrain);
      }
    }
    __syncwarp();
  } else {
    const int quarter = warp & 3;
    const CUtensorMap* tmo = tma_store ? &tma_o : nullptr;
    uint32_t slice = 0;
    int as = 0;
    uint32_t aphase = 0;
    for (int64_t t = pair_id; t < total_tiles; t += npairs) {
      bool ok = mbar_wait(&sh.tfull[as], aphase, kErrWaitTimeoutEpilogue);
      ok = __all_sync(0xffffffffu, ok) && !sh.abort;
      if (!ok) {
        sh.abort = 1;
        break;
      }
      tc_fence_after();
      int tm, tn;
      tile_coords2(t, tiles_m, tiles_n, tm, tn);
      const int64_t m0 = static_cast<int64_t>(tm) * (2 * BM) + static_cast<int64_t>(rank) * BM + quarter * 32;
      const bool row_ok = m0 + lane < p.M;
      const float sam = row_ok ? __ldg(p.sa + m0 + lane) : 0.0f;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>(as * BN);
      epilogue_rows(p, tbase, m0, lane, row_ok, sam, static_cast<int64_t>(tn) * BN,
                    staging + (warp - 2) * STAGING_BYTES, tmo, slice);
      tc_fence_before();
      mbar_arrive_cluster(mapa_shared(smem_u32(&sh.tempty[as]), 0));
      as ^= 1;
      if (as == 0) aphase ^= 1;
    }
    if (lane == 0) bulk_wait_group<0>();  // the tensor stores are complete before the CTA exits
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the peer's MMAs, loads and remote arrives are finished
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}
}  // namespace pair

}  // namespace gi8

// ------------------------------------------------------------------ host side
typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                    const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                    const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled get_encode_fn() {
  static const PFN_encodeTiled fn = []() -> PFN_encodeTiled {  // looked up once, thread-safe
    void* sym = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &sym, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<PFN_encodeTiled>(sym);
    return nullptr;
  }();
  return fn;
}

// 2-D K-major int8 operand [rows, K], box = 128 bytes of K x box_rows rows, 128-byte swizzle.
static bool make_kmajor_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t K, int box_rows) {
  PFN_encodeTiled enc = get_encode_fn();
  if (enc == nullptr) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(gi8::BK), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box,
                         estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Output map for the epilogue's tensor stores: bf16 [M, cols] with row pitch ldo, boxes of
// 32 rows x (64 columns, 128-byte swizzle) or, for the half-width SwiGLU output, (32 columns,
// 64-byte swizzle): the staging layouts of tma_store_slice.
static bool make_out_map(CUtensorMap* map, void* out, int64_t M, int64_t cols, int64_t ldo, bool half_width) {
  PFN_encodeTiled enc = get_encode_fn();
  if (enc == nullptr) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(M)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ldo) * 2};
  const cuuint32_t box[2] = {half_width ? 32u : 64u, 32u};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, out, dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE,
                         half_width ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

cudaError_t launch_gemm_i8(const GemmI8Params& p, cudaStream_t st) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const bool use_pair = p.M > gi8::BM;
  CUtensorMap ma, mb, mo;
  if (!make_kmajor_map(&ma, p.a, p.M, p.K, gi8::BM)) return cudaErrorInvalidValue;
  if (!make_kmajor_map(&mb, p.b, p.N, p.K, use_pair ? gi8::pair::BNH : gi8::BN)) return cudaErrorInvalidValue;
  // tensor stores unless the tile also goes to other GPUs or to the int32 copy
  const bool half = p.epilogue == kEpiSwiGLU;
  const int tma_store = p.n_peer == 0 && p.acc_dbg == nullptr && (reinterpret_cast<uintptr_t>(p.out) & 15) == 0 &&
                        p.ldo % 8 == 0 && make_out_map(&mo, p.out, p.M, half ? p.N / 2 : p.N, p.ldo, half);
  if (!tma_store) memset(&mo, 0, sizeof(mo));
  const int tiles_n = static_cast<int>((p.N + gi8::BN - 1) / gi8::BN);
  if (use_pair) {
    const int tiles_m = static_cast<int>((p.M + 2 * gi8::BM - 1) / (2 * gi8::BM));
    static PerDeviceOnce smem_once, pairs_once;
    cudaError_t e = smem_once.run(dev, [] {
      return cudaFuncSetAttribute(gi8::pair::gemm_i8_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(gi8::pair::SMEM_BYTES));
    });
    if (e != cudaSuccess) return e;
    static int max_pairs[64] = {0};  // clusters of 2 that fit at once, per device
    int cap = sms / 2;
    pairs_once.run(dev, [&] {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2 * (sms / 2));
      cfg.blockDim = dim3(gi8::THREADS);
      cfg.dynamicSmemBytes = gi8::pair::SMEM_BYTES;
      cudaLaunchAttribute attr;
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = 2;
      attr.val.clusterDim.y = 1;
      attr.val.clusterDim.z = 1;
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      int clusters = 0;
      if (cudaOccupancyMaxActiveClusters(&clusters, gi8::pair::gemm_i8_pair_kernel, &cfg) != cudaSuccess || clusters < 1)
        clusters = sms / 2;
      if (dev >= 0 && dev < 64) max_pairs[dev] = clusters;
      cap = clusters;
      return cudaSuccess;
    });
    if (dev >= 0 && dev < 64) cap = max_pairs[dev];
    const int64_t total = static_cast<int64_t>(tiles_m) * tiles_n;
    const int pairs = static_cast<int>(total < cap ? total : cap);
    gi8::pair::gemm_i8_pair_kernel<<<2 * pairs, gi8::THREADS, gi8::pair::SMEM_BYTES, st>>>(ma, mb, mo, p, tiles_m,
                                                                                           tiles_n, tma_store);
    return cudaGetLastError();
  }
  const int tiles_m = static_cast<int>((p.M + gi8::BM - 1) / gi8::BM);
  const int64_t total = static_cast<int64_t>(tiles_m) * tiles_n;
  const int grid = static_cast<int>(total < sms ? total : sms);
  static PerDeviceOnce smem_once1;
  const cudaError_t e = smem_once1.run(dev, [] {
    return cudaFuncSetAttribute(gi8::gemm_i8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(gi8::SMEM_BYTES));
  });
  if (e != cudaSuccess) return e;
  gi8::gemm_i8_kernel<<<grid, gi8::THREADS, gi8::SMEM_BYTES, st>>>(ma, mb, mo, p, tiles_m, tiles_n, tma_store);
  return cudaGetLastError();
}

}  // namespace slim
