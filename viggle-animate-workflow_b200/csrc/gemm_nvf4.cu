// Block-scaled FP4 (NVFP4) GEMM on the sm_100a tensor cores (tcgen05.mma kind::mxf4nvf4,
// scale_vec::4X) with a dequantising epilogue:
//
//   out[m, n] = bf16( acc[m, n] * (sa[m] * sb) + bias[n] ),
//   acc[m, n] = sum_k (ea[m,k] * fa[m, k/16]) * (eb[n,k] * fb[n, k/16])   (fp32, tensor core)
//
// ea/eb are E2M1 values (packed two per byte, element 2i in the low nibble), fa/fb their
// UE4M3 block scales in the cuBLAS 128x4 tiled layout, sa the activation's per-token global
// scale and sb the weight's per-tensor global scale (slimdit/nvfp4.py:3-8: weight,
// weight_scale, weight_scale_2). This is the runtime side of an NVFP4 linear.
//
// Structure (one CTA per SM, persistent over 128 x 256 output tiles, K-blocks of 256 FP4):
//   warp 0       producer: TMA tiles of A (128 x 128 B) and B (256 x 128 B), 128-byte swizzle,
//                plus bulk copies of the k-block's scale atoms (2 KB of A, 2 x 2 KB of B), into
//                a 4-stage ring guarded by full/empty mbarriers.
//   warp 1       allocates 512 TMEM columns: a 256-column fp32 accumulator and, per stage, 48
//                scale columns; one lane issues 4 MMAs (M=128, N=256, K=64) per stage.
//   warps 2..5   scale loaders, one per TMEM lane quarter: each lane reads its 16-byte line of
//                every 512-byte scale atom of the stage from shared memory and writes it to
//                the stage's scale columns with tcgen05.st (A: 4 atoms x 4 columns, B: 8 x 4).
//                A 128-row atom sits in 32 lanes x 4 columns, line i (rows i, i+32, i+64, i+96)
//                in lane i of every quarter: the layout the MMA reads (the one tcgen05.cp
//                .32x128b.warpx4 produces). Issued by these warps, the scale writes stay out of
//                the MMA issue stream (a tcgen05.cp issued there after MMAs held back the MMAs
//                behind it: 2.7 vs 4.1 POPS measured). A stage's scale columns are written once
//                its full barrier completes: by then the MMAs that last read them are done,
//                since the producer refilled the stage only after they committed. sf_full hands
//                the columns to the MMA warp.
//   warps 6..13  epilogue: each warp reads 128 accumulator columns of its lane quarter,
//                scales + biases them (GELU if asked) and packs bf16 in registers, releases the
//                accumulator to the next tile's MMAs, then writes its 32 rows back through a
//                1 KB shared-memory buffer, 16 columns at a time, by TMA tensor stores (or, for
//                an output the tensor map cannot describe, with each store instruction of the
//                warp covering 16 rows x 32 bytes). (One row per thread, the 16-byte stores into
//                32 rows per instruction slowed the MMAs by ~12 %; the ring leaves no room for
//                a wider buffer, and moving the scale atoms out of the ring to make room put
//                their global-memory latency in front of the MMAs.)
// Every mbarrier wait is bounded; on a timeout the kernel records an error, drains its
// copies and MMAs, frees TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "slim_kernels.h"
#include "slim_ptx.cuh"

namespace slim {
namespace gf4 {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BKB = 128;                  // bytes of packed FP4 per row per k-block (256 elements)
constexpr int STAGES = 4;
constexpr int EPI_ROW_BYTES = 32;         // bf16 bytes per row of one write-back slice (16 columns)
constexpr int STAGING_BYTES = 32 * EPI_ROW_BYTES;  // per epilogue warp: what the ring leaves free
constexpr int A_BYTES = BM * BKB;         // 16 KB
constexpr int B_BYTES = BN * BKB;         // 32 KB
constexpr int ATOM = 512;                 // one 128-row x 4-scale tile of the block-scale layout
constexpr int SFA_BYTES = 4 * ATOM;       // A scales of a k-block: 4 atoms
constexpr int SFB_BYTES = 8 * ATOM;       // B scales: 2 row tiles x 4 atoms
constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;
constexpr int MMA_KB = 32;                // bytes of one MMA's K (64 FP4 elements)
constexpr int SF_WARP0 = 2;
constexpr int EPI_WARP0 = 6;
constexpr int THREADS = 14 * 32;
constexpr int TMEM_COLS = 512;
constexpr int SF_COL0 = 256;
constexpr int SF_COLS = 48;               // per stage: A 4 atoms x 4 columns, B 8 atoms x 4 columns
constexpr int GROUP_M = 16;
constexpr uint32_t IDESC = idesc_nvf4(BM, BN);

struct Shared {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t sf_full[STAGES];
  uint64_t tfull;
  uint64_t tempty;
  uint64_t drain;
  uint32_t tmem_base;
  volatile int abort;
};

constexpr size_t SMEM_BYTES =
    1024 + static_cast<size_t>(STAGES) * STAGE_BYTES + 8 * STAGING_BYTES + sizeof(Shared) + 64;
static_assert(SMEM_BYTES <= 232448, "shared memory budget");
static_assert(SF_COL0 + STAGES * SF_COLS <= TMEM_COLS, "TMEM budget");

__device__ __forceinline__ void tile_coords(int64_t t, int tiles_m, int tiles_n, int& tm, int& tn) {
  const int64_t per_group = static_cast<int64_t>(GROUP_M) * tiles_n;
  const int64_t g = t / per_group;
  const int first_m = static_cast<int>(g * GROUP_M);
  const int gm = min(tiles_m - first_m, GROUP_M);
  const int local = static_cast<int>(t - g * per_group);
  tm = first_m + local % gm;
  tn = local / gm;
}

__global__ void __launch_bounds__(THREADS, 1)
gemm_nvf4_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                 const __grid_constant__ CUtensorMap tma_o, const GemmNvf4Params p, int tiles_m, int tiles_n,
                 int tma_store) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023) & ~1023u) - raw_addr);
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * A_BYTES;
  uint8_t* sFA = sB + STAGES * B_BYTES;
  uint8_t* sFB = sFA + STAGES * SFA_BYTES;
  uint8_t* staging = smem + STAGES * STAGE_BYTES;
  Shared& sh = *reinterpret_cast<Shared*>(staging + 8 * STAGING_BYTES);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t total_tiles = static_cast<int64_t>(tiles_m) * tiles_n;
  const int64_t ctiles = p.K / 64;                       // scale atoms per 128-row tile
  const int num_kb = static_cast<int>((p.K + 255) / 256);
  const int64_t n_rowtiles = p.N / 128;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], 1);
      mbar_init(&sh.sf_full[s], 4);
    }
    mbar_init(&sh.tfull, 1);
    mbar_init(&sh.tempty, 256);
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
        const bool rb1 = 2 * static_cast<int64_t>(tn) + 1 < n_rowtiles;
        for (int kb = 0; kb < num_kb; ++kb) {
          const int64_t atom0 = 4 * static_cast<int64_t>(kb);
          const uint32_t sfbytes = static_cast<uint32_t>(ctiles - atom0 < 4 ? ctiles - atom0 : 4) * ATOM;
          if (!mbar_wait(&sh.empty[stage], phase ^ 1, kErrWaitTimeoutProducer)) {
            sh.abort = 1;
            break;
          }
          if (sh.abort) break;
          mbar_arrive_expect_tx(&sh.full[stage], A_BYTES + B_BYTES + sfbytes * (rb1 ? 3u : 2u));
          tma_load_2d(sA + stage * A_BYTES, &tma_a, &sh.full[stage], kb * BKB, tm * BM);
          tma_load_2d(sB + stage * B_BYTES, &tma_b, &sh.full[stage], kb * BKB, tn * BN);
          bulk_load(sFA + stage * SFA_BYTES, p.sfa + (static_cast<int64_t>(tm) * ctiles + atom0) * ATOM, sfbytes,
                    &sh.full[stage]);
          bulk_load(sFB + stage * SFB_BYTES, p.sfb + (2 * static_cast<int64_t>(tn) * ctiles + atom0) * ATOM, sfbytes,
                    &sh.full[stage]);
          if (rb1)
            bulk_load(sFB + stage * SFB_BYTES + 4 * ATOM,
                      p.sfb + ((2 * static_cast<int64_t>(tn) + 1) * ctiles + atom0) * ATOM, sfbytes, &sh.full[stage]);
          issued |= 1u << stage;
          last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      for (int s = 0; s < STAGES; ++s)
        if (issued & (1u << s)) mbar_wait(&sh.full[s], (last_parity >> s) & 1, kErrWaitTimeoutDrain);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t aphase = 0;
      bool issued_any = false;
      for (int64_t t = blockIdx.x; t < total_tiles && !sh.abort; t += gridDim.x) {
        if (!mbar_wait(&sh.tempty, aphase ^ 1, kErrWaitTimeoutMma)) {
          sh.abort = 1;
          break;
        }
        tc_fence_after();
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          const int64_t atom0 = 4 * static_cast<int64_t>(kb);
          const int nat = static_cast<int>(ctiles - atom0 < 4 ? ctiles - atom0 : 4);
          if (!mbar_wait(&sh.full[stage], phase, kErrWaitTimeoutMma) ||
              !mbar_wait(&sh.sf_full[stage], phase, kErrWaitTimeoutMma) || sh.abort) {
            sh.abort = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sf_t = tmem_base + static_cast<uint32_t>(SF_COL0 + stage * SF_COLS);
          const uint32_t a0 = smem_u32(sA + stage * A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * B_BYTES);
          for (int kk = 0; kk < nat; ++kk) {
            mma_nvf4(tmem_base, smem_desc_sw128(a0 + kk * MMA_KB), smem_desc_sw128(b0 + kk * MMA_KB), IDESC,
                     sf_t + kk * 4, sf_t + 16 + kk * 8, (kb | kk) != 0 ? 1u : 0u);
          }
          issued_any = true;
          mma_commit(&sh.empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit(&sh.tfull);
        aphase ^= 1;
      }
      if (issued_any) {
        mma_commit(&sh.drain);
        mbar_wait(&sh.drain, 0, kErrWaitTimeoutDrain);
      }
    }
    __syncwarp();
  } else if (warp < EPI_WARP0) {
    // scale loaders: lane quarter q = warp % 4. The stage's scale atoms arrive in shared
    // memory with its TMA tiles (full barrier); the stage's scale columns are free then too,
    // since the producer refilled the stage only after its previous MMAs completed.
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    int stage = 0;
    uint32_t phase = 0;
    for (int64_t t = blockIdx.x; t < total_tiles; t += gridDim.x) {
      bool ok = true;
      for (int kb = 0; kb < num_kb; ++kb) {
        ok = mbar_wait(&sh.full[stage], phase, kErrWaitTimeoutMma);
        ok = __all_sync(0xffffffffu, ok) && !sh.abort;
        if (!ok) {
          sh.abort = 1;
          break;
        }
        const uint4* fa = reinterpret_cast<const uint4*>(sFA + stage * SFA_BYTES) + lane;
        const uint4* fb = reinterpret_cast<const uint4*>(sFB + stage * SFB_BYTES) + lane;
        uint32_t va[16], vb[32];
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint4 a = fa[kk * (ATOM / 16)];
          const uint4 b0 = fb[kk * (ATOM / 16)];
          const uint4 b1 = fb[(4 + kk) * (ATOM / 16)];
          va[4 * kk] = a.x; va[4 * kk + 1] = a.y; va[4 * kk + 2] = a.z; va[4 * kk + 3] = a.w;
          vb[8 * kk] = b0.x; vb[8 * kk + 1] = b0.y; vb[8 * kk + 2] = b0.z; vb[8 * kk + 3] = b0.w;
          vb[8 * kk + 4] = b1.x; vb[8 * kk + 5] = b1.y; vb[8 * kk + 6] = b1.z; vb[8 * kk + 7] = b1.w;
        }
        tc_fence_after();
        const uint32_t col = tmem_base + lane_base + static_cast<uint32_t>(SF_COL0 + stage * SF_COLS);
        tmem_st_32x32b_x16(col, va);
        tmem_st_32x32b_x32(col + 16, vb);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh.sf_full[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
    }
  } else {
    // epilogue warps 6..13: lane quarter warp % 4, column half (warp - 6) / 4
    const int quarter = warp & 3;
    const int half = (warp - EPI_WARP0) >> 2;
    const int row = quarter * 32 + lane;
    const __nv_bfloat16* bias = static_cast<const __nv_bfloat16*>(p.bias);
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out);
    const float sb = __ldg(p.sb);
    uint32_t aphase = 0, slice = 0;
    for (int64_t t = blockIdx.x; t < total_tiles; t += gridDim.x) {
      bool ok = mbar_wait(&sh.tfull, aphase, kErrWaitTimeoutEpilogue);
      ok = __all_sync(0xffffffffu, ok) && !sh.abort;
      if (!ok) {
        sh.abort = 1;
        break;
      }
      tc_fence_after();
      int tm, tn;
      tile_coords(t, tiles_m, tiles_n, tm, tn);
      const int64_t m = static_cast<int64_t>(tm) * BM + row;
      const bool row_ok = m < p.M;
      const int64_t nbase = static_cast<int64_t>(tn) * BN + half * 128;
      const bool cols_ok = nbase < p.N;  // N % 128 == 0: a 128-column half is all in or all out
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(half * 128);
      const float alpha = row_ok ? __fmul_rn(__ldg(p.sa + m), sb) : 0.0f;
      const bool gelu = p.epilogue == kEpiGeluTanh;
      uint32_t pk[64];
      // 8 chunks of 16 columns; the next chunk's TMEM load and bias load are issued before this
      // chunk's arithmetic, so their latency is hidden behind it (the MMAs of the next tile wait
      // for this loop to finish)
      uint32_t r[2][16];
      uint4 bq[2][2];
      auto bias_load = [&](int c, uint4 (&b)[2]) {
        if (bias != nullptr && cols_ok) {
          const uint4* bp = reinterpret_cast<const uint4*>(bias + nbase + c * 16);
          b[0] = __ldg(bp);
          b[1] = __ldg(bp + 1);
        } else {
          b[0] = b[1] = make_uint4(0u, 0u, 0u, 0u);
        }
      };
      bias_load(0, bq[0]);
      tmem_ld_32x32b_x16(tbase, r[0]);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        tmem_ld_wait();
        reg_dep16(r[c & 1]);
        if (c + 1 < 8) {
          tmem_ld_32x32b_x16(tbase + (c + 1) * 16, r[(c + 1) & 1]);
          bias_load(c + 1, bq[(c + 1) & 1]);
        }
        const uint32_t* rc = r[c & 1];
        const int64_t n0 = nbase + c * 16;
        if (row_ok && cols_ok && p.acc_dbg != nullptr) {
          float* dst = p.acc_dbg + m * p.N + n0;
#pragma unroll
          for (int j = 0; j < 16; j += 4)
            *reinterpret_cast<float4*>(dst + j) = make_float4(__uint_as_float(rc[j]), __uint_as_float(rc[j + 1]),
                                                              __uint_as_float(rc[j + 2]), __uint_as_float(rc[j + 3]));
        }
#pragma unroll
        for (int j = 0; j < 16; j += 8) {
          const uint4 bu = bq[c & 1][j / 8];
          const uint32_t bw[4] = {bu.x, bu.y, bu.z, bu.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float y0 = __fmaf_rn(__uint_as_float(rc[j + 2 * e]), alpha, __uint_as_float(bw[e] << 16));
            float y1 = __fmaf_rn(__uint_as_float(rc[j + 2 * e + 1]), alpha, __uint_as_float(bw[e] & 0xffff0000u));
            if (gelu) {
              y0 = gi8::gelu_tanh(gi8::bf16_round(y0));
              y1 = gi8::gelu_tanh(gi8::bf16_round(y1));
            }
            pk[8 * c + j / 2 + e] = gi8::pack_bf16x2(y0, y1);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&sh.tempty);  // the accumulator is in registers: the next tile may start
      aphase ^= 1;
      const int64_t m0 = static_cast<int64_t>(tm) * BM + quarter * 32;
      if (cols_ok && m0 < p.M) {  // warp-uniform
        uint8_t* stg = staging + (warp - EPI_WARP0) * STAGING_BYTES;
#pragma unroll
        for (int c = 0; c < 256 / EPI_ROW_BYTES; ++c) {
          if (tma_store)
            gi8::tma_store_slice<EPI_ROW_BYTES, 1>(&tma_o, stg, pk + c * (EPI_ROW_BYTES / 4), m0,
                                                   nbase + c * (EPI_ROW_BYTES / 2), lane, slice);
          else
            gi8::store_rows_staged<EPI_ROW_BYTES>(out, nullptr, 0, p.ldo, p.M, p.N, stg, pk + c * (EPI_ROW_BYTES / 4),
                                                  m0, nbase + c * (EPI_ROW_BYTES / 2), lane);
        }
      }
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

}  // namespace gf4

cudaError_t launch_gemm_nvf4(const GemmNvf4Params& p, cudaStream_t st) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  CUtensorMap ma, mb;
  if (!make_kmajor_map(&ma, p.a, p.M, p.K / 2, gf4::BM)) return cudaErrorInvalidValue;
  if (!make_kmajor_map(&mb, p.b, p.N, p.K / 2, gf4::BN)) return cudaErrorInvalidValue;
  // output map for the epilogue's tensor stores: boxes of 32 rows x 16 columns, 32-byte swizzle
  CUtensorMap mo;
  int tma_store = 0;
  if ((reinterpret_cast<uintptr_t>(p.out) & 15) == 0 && p.ldo % 8 == 0) {
    PFN_encodeTiled enc = get_encode_fn();
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(p.N), static_cast<cuuint64_t>(p.M)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(p.ldo) * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(gf4::EPI_ROW_BYTES / 2), 32u};
    const cuuint32_t estr[2] = {1, 1};
    tma_store = enc != nullptr &&
                enc(&mo, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.out, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  }
  if (!tma_store) memset(&mo, 0, sizeof(mo));
  const int tiles_m = static_cast<int>((p.M + gf4::BM - 1) / gf4::BM);
  const int tiles_n = static_cast<int>((p.N + gf4::BN - 1) / gf4::BN);
  const int64_t total = static_cast<int64_t>(tiles_m) * tiles_n;
  const int grid = static_cast<int>(total < sms ? total : sms);
  static PerDeviceOnce smem_once;
  const cudaError_t e = smem_once.run(dev, [] {
    return cudaFuncSetAttribute(gf4::gemm_nvf4_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(gf4::SMEM_BYTES));
  });
  if (e != cudaSuccess) return e;
  gf4::gemm_nvf4_kernel<<<grid, gf4::THREADS, gf4::SMEM_BYTES, st>>>(ma, mb, mo, p, tiles_m, tiles_n, tma_store);
  return cudaGetLastError();
}

}  // namespace slim
