// Dense projections of the block on the 5th-generation tensor cores:
//   C[z][M, N] = A[z][M, K] . W[z][N, K]^T       (bf16 operands, fp32 accumulate)
// for the R/K/V, low-rank, output, ROSA, FFN and LM-head projections of
// yufmusicgen/model.py:107-112, 195-197, 297-311, 376-377, 421.
//
// One persistent CTA per SM walks the output tiles (128 rows x BN columns) of
// every batch z in a grouped order (8 row tiles x all column tiles per group,
// so the rows and weights a wave of CTAs shares stay in L2).  Six warps with
// fixed roles:
//   warp 0   one thread issues the TMA loads: per 64-wide K block the A box
//            (128 x 64) and the W box (BN x 64), 128-byte swizzled, into a ring
//            of shared-memory stages guarded by full/empty mbarriers;
//   warp 1   allocates two accumulators of BN columns in TMEM, and one thread
//            issues the kind::f16 UMMAs (M = 128, N = BN, K = 16; four per
//            stage), committing each stage back to its empty barrier and each
//            finished tile to the accumulator's full barrier;
//   warps 2-5  the epilogue: warp w reads TMEM lanes 32*(w % 4).., one output
//            row per thread, 32 columns per tcgen05.ld, and writes the result
//            (fp32 with an optional residual add, bf16 with an optional tanh, or
//            SiLU(in) * gate for the FFN) straight to global memory, while the
//            MMAs of the next tile run into the other accumulator.
// Every mbarrier wait is bounded (WAIT_NS); a wait that expires raises the
// CTA's abort flag, every role leaves its loop, the loads and MMAs still in
// flight are waited for (bounded) before the TMEM is freed, and the expiry is
// counted for yuf_wait_timeouts / yuf_sync_check.  No cluster multicast: each
// CTA loads its own boxes.

#include <cuda_bf16.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <mutex>

#include "common.cuh"
#include "gemm.cuh"
#include "mbarrier.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace yuf {

__device__ unsigned int g_gemm_wait_timeouts;

// Per-warp staging of the epilogue: 32 rows x 32 columns of fp32 with a row
// stride of 36 floats (16-byte rows apart by 4 banks: conflict-free float4
// writes by row and float4 reads by column group).
constexpr int GEMM_STG_LD = 36;
constexpr int GEMM_STG_FLOATS = 32 * GEMM_STG_LD;

template <int BN>
struct GemmCfg {
  static constexpr int BM = 128, BK = 64;           // BK bf16 = one 128-byte swizzle row
  static constexpr int A_BYTES = BM * BK * 2;       // 16 KB
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;   // multiple of 1024
  static constexpr int STAGES = std::min(8, (192 * 1024) / STAGE);
  // two fp32 accumulators of BN columns, ACC columns apart (a power of two, so
  // that each starts on an aligned column); TMEM_COLS a power of two as well
  static constexpr uint32_t ACC = BN <= 64 ? 64 : (BN <= 128 ? 128 : 256);
  static constexpr uint32_t TMEM_COLS = 2 * ACC;
  static constexpr int STG_BYTES = 4 * GEMM_STG_FLOATS * 4;  // the epilogue warps' staging
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM = STAGES * STAGE + STG_BYTES + BAR_BYTES + 1024;  // + alignment slack
  static constexpr uint32_t IDESC = umma_idesc_bf16(BM, BN);
  static constexpr int THREADS = 192;
  static_assert(BN == 64 || BN == 128 || BN == 160 || BN == 256, "tile width");
  static_assert(STAGE % 1024 == 0, "stages stay 1024-byte aligned for the 128-byte swizzle");
  static_assert(2 * STAGES * 8 + 4 * 8 + 8 + 8 <= BAR_BYTES, "barrier block");
};

// Tile t of the grouped walk -> (batch, row tile, column tile).
YUF_DEVICE void gemm_tile(int t, int m_tiles, int n_tiles, int& z, int& mt, int& nt) {
  constexpr int GM = 8;
  const int per = m_tiles * n_tiles;
  z = t / per;
  const int r = t - z * per;
  const int group = r / (GM * n_tiles);
  const int first = group * GM;
  const int gsz = min(GM, m_tiles - first);
  const int rr = r - group * GM * n_tiles;
  mt = first + rr % gsz;
  nt = rr / gsz;
}

// SiLU with the fast exponential and divide (about 2 ulp; the outputs are bf16
// or fp32 compared at 1e-4 relative).  For x < -88 the exponential is +inf and
// the quotient 0, the limit.
YUF_DEVICE float silu(float x) { return __fdividef(x, 1.f + __expf(-x)); }

// A bounded wait that gives up at once when another role already aborted.
YUF_DEVICE bool gemm_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (*abort_flag) return false;
  if (mbar_wait(bar, parity)) return true;
  *abort_flag = 1;
  return false;
}

// One 32 x 32 block of the calling warp's fp32 outputs (added to C when
// p.beta != 0): lane l holds row l's 32 values in v; they go through the warp's
// staging area so that each store instruction writes four whole 128-byte row
// segments instead of 16 bytes in each of 32 rows (for an fp32 tile that cut
// the [65536 x 3072] R/K/V projection from 449 to 362 us).  `rows` rows of the
// block are live; columns from `col` on, up to `ncols` of them.
YUF_DEVICE void gemm_store_block_f32(const GemmParams& p, float* stg, const float (&v)[32], int z, int row0,
                                     int rows, int col, int ncols) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < 8; ++k)
    *reinterpret_cast<float4*>(stg + lane * GEMM_STG_LD + 4 * k) =
        make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
  __syncwarp();
  const int c4 = 4 * (lane & 7);
  const bool full = p.vec && c4 + 4 <= ncols;
  float* base = static_cast<float*>(p.C) + (size_t)z * p.c_bstride + (size_t)row0 * p.ldc + col + c4;
  float4 x[8], old[8];
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    x[it] = *reinterpret_cast<const float4*>(stg + (it * 4 + (lane >> 3)) * GEMM_STG_LD + c4);
    old[it] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __syncwarp();  // the staging area is free for the next block
  if (p.beta != 0.f && full) {  // the residual's old values, all loads before the first store
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int r = it * 4 + (lane >> 3);
      if (r < rows) old[it] = *reinterpret_cast<const float4*>(base + (size_t)r * p.ldc);
    }
  }
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int r = it * 4 + (lane >> 3);
    if (r >= rows) continue;
    float* out = base + (size_t)r * p.ldc;
    if (full) {
      *reinterpret_cast<float4*>(out) =
          make_float4(x[it].x + old[it].x, x[it].y + old[it].y, x[it].z + old[it].z, x[it].w + old[it].w);
    } else {
      const float e[4] = {x[it].x, x[it].y, x[it].z, x[it].w};
      for (int c = 0; c < 4; ++c)
        if (c4 + c < ncols) out[c] = p.beta != 0.f ? e[c] + out[c] : e[c];
    }
  }
}

// bf16 outputs from one thread's row: 32 values as four 16-byte stores.
YUF_DEVICE void gemm_store_row_bf16(const GemmParams& p, const float (&v)[32], int z, int row, int col,
                                    int ncols) {
  __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.C) + (size_t)z * p.c_bstride + (size_t)row * p.ldc + col;
  if (p.vec && ncols >= 32) {
#pragma unroll
    for (int c = 0; c < 32; c += 8) {
      uint4 pk;
      __nv_bfloat162* b2 = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
      for (int e = 0; e < 4; ++e) b2[e] = __floats2bfloat162_rn(v[c + 2 * e], v[c + 2 * e + 1]);
      *reinterpret_cast<uint4*>(out + c) = pk;
    }
  } else {
    for (int c = 0; c < 32; ++c)
      if (c < ncols) out[c] = __float2bfloat16_rn(v[c]);
  }
}

// Epilogue of one output tile held in TMEM (lanes = rows, columns = outputs):
// the calling warp's 32 rows starting at `row0` (`rows` of them live), `tbase`
// the TMEM address of the warp's lane quarter at the tile's first column; tile
// column block `nt` of BN columns (SiLU-gate: BN / 2 output columns).  Every
// lane runs the TMEM loads (warp-collective); `stg` is the warp's staging area.
template <int BN, int EPI>
YUF_DEVICE void gemm_epilogue_tile(const GemmParams& p, uint32_t tbase, int z, int row0, int rows, int nt,
                                   float* stg) {
  if constexpr (EPI == GEMM_EPI_SWIGLU_F32 || EPI == GEMM_EPI_SWIGLU) {
    // tile columns per 128: [64 "in" rows | 64 "gate" rows] of the packed weight
#pragma unroll 1
    for (int sb = 0; sb < BN / 128; ++sb)
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        float vi[32], vg[32];
        tmem_ld_x32(tbase + sb * 128 + h * 32, vi);
        tmem_ld_x32(tbase + sb * 128 + 64 + h * 32, vg);
        const int col = nt * (BN / 2) + sb * 64 + h * 32;
        if (rows <= 0 || col >= p.n_out) continue;
#pragma unroll
        for (int c = 0; c < 32; ++c) vi[c] = silu(vi[c]) * vg[c];
        if constexpr (EPI == GEMM_EPI_SWIGLU) {
          if ((threadIdx.x & 31) < rows) gemm_store_row_bf16(p, vi, z, row0 + (threadIdx.x & 31), col, p.n_out - col);
        } else {
          gemm_store_block_f32(p, stg, vi, z, row0, rows, col, min(32, p.n_out - col));
        }
      }
  } else {
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
      float v[32];
      tmem_ld_x32(tbase + c0, v);
      const int col = nt * BN + c0;
      if (rows <= 0 || col >= p.N) continue;
      if (p.tanh_batch0 && z == 0) {
#pragma unroll
        for (int c = 0; c < 32; ++c) v[c] = tanhf(v[c]);
      }
      if constexpr (EPI == GEMM_EPI_BF16) {
        if ((threadIdx.x & 31) < rows) gemm_store_row_bf16(p, v, z, row0 + (threadIdx.x & 31), col, p.N - col);
      } else {
        gemm_store_block_f32(p, stg, v, z, row0, rows, col, min(32, p.N - col));
      }
    }
  }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(GemmCfg<BN>::THREADS, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tw,
                     const GemmParams p) {
  using G = GemmCfg<BN>;
  extern __shared__ __align__(1024) unsigned char gemm_smem_raw[];
  unsigned char* sm = gemm_smem_raw + ((1024u - (smem_u32(gemm_smem_raw) & 1023u)) & 1023u);
  float* stg_all = reinterpret_cast<float*>(sm + G::STAGES * G::STAGE);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + G::STAGES * G::STAGE + G::STG_BYTES);
  uint64_t* empty = full + G::STAGES;
  uint64_t* tfull = empty + G::STAGES;   // [2] accumulator ready for the epilogue
  uint64_t* tempty = tfull + 2;          // [2] accumulator drained by the epilogue
  uint64_t* drain = tempty + 2;          // final commit of the MMA thread
  uint32_t* tslot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < G::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);  // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tslot, G::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  pdl_wait();  // the set-up above overlaps the previous kernel of a PDL chain
  pdl_trigger();
  const uint32_t tmem = *tslot;
  const int total = p.m_tiles * p.n_tiles * p.batch;
  const int kblocks = (p.K + G::BK - 1) / G::BK;

  if (warp == 0) {
    if (lane == 0) {  // ---------------------------------------------- TMA producer
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      for (int t = blockIdx.x; t < total; t += gridDim.x) {
        int z, mt, nt;
        gemm_tile(t, p.m_tiles, p.n_tiles, z, mt, nt);
        const int ay = (int)(z * p.a_brows) + mt * G::BM;
        const int wy = (int)(z * p.w_brows) + nt * BN;
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!gemm_wait(&empty[stage], phase ^ 1u, abort_flag)) { ok = false; break; }
          unsigned char* st = sm + stage * G::STAGE;
          mbar_expect_tx(&full[stage], G::STAGE);
          tma_load_2d(st, &ta, &full[stage], kb * G::BK, ay);
          tma_load_2d(st + G::A_BYTES, &tw, &full[stage], kb * G::BK, wy);
          ++issued;
          if (++stage == G::STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
      }
      if (*abort_flag) {  // let the loads still in flight into this CTA's stages land
        for (int s = 0; s < G::STAGES; ++s) {
          if (issued <= s) break;
          mbar_wait(&full[s], s < stage ? phase : phase ^ 1u);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ------------------------------------------------- MMA issuer
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool any = false;
      for (int t = blockIdx.x; t < total; t += gridDim.x) {
        if (!gemm_wait(&tempty[acc], acc_phase ^ 1u, abort_flag)) break;
        tc_fence_after_sync();
        const uint32_t d = tmem + (uint32_t)acc * G::ACC;
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!gemm_wait(&full[stage], phase, abort_flag)) { ok = false; break; }
          tc_fence_after_sync();
          const uint32_t a0 = smem_u32(sm + stage * G::STAGE), b0 = a0 + G::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < G::BK / 16; ++kk)
            umma_bf16(d, umma_desc_sw128(a0 + kk * 32), umma_desc_sw128(b0 + kk * 32), G::IDESC,
                      (kb | kk) != 0 ? 1u : 0u);
          any = true;
          umma_commit(&empty[stage]);  // the stage is free once these MMAs have read it
          if (++stage == G::STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);  // the tile's accumulator is complete
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      if (any) {  // every MMA issued has finished before the columns are freed
        umma_commit(drain);
        mbar_wait(drain, 0);
      }
    }
  } else {  // ---------------------------------------------------- epilogue (warps 2-5)
    const int q = warp & 3;  // TMEM lane quarter this warp may read
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      int z, mt, nt;
      gemm_tile(t, p.m_tiles, p.n_tiles, z, mt, nt);
      bool ok = gemm_wait(&tfull[acc], acc_phase, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after_sync();
      const int row0 = mt * G::BM + q * 32;
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)acc * G::ACC;
      gemm_epilogue_tile<BN, EPI>(p, tbase, z, row0, min(32, p.M - row0), nt, stg_all + q * GEMM_STG_FLOATS);
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }
  if (threadIdx.x == 0 && *abort_flag) atomicAdd(&g_gemm_wait_timeouts, 1u);
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, G::TMEM_COLS);
  }
}

// ---------------------------------------------------------------- CTA pairs
// Large problems run on CTA pairs (a 2-CTA cluster, cta_group::2): a 256 x 256
// output tile per pair, each CTA loading 128 rows of A and 128 rows of W per K
// block (half the W traffic of a 128 x 256 tile per SM for the same MMA work),
// peer 0 issuing M = 256, N = 256 UMMAs over both SMs' operands, each CTA
// draining its own 128 accumulator rows.  Both CTAs' loads complete on peer 0's
// full barrier (peer 0 expects the bytes of both); MMA completion is committed
// to both CTAs' empty and accumulator-full barriers (multicast commit); the
// epilogue warps of both CTAs release an accumulator on peer 0's empty barrier
// (8 arrivals).  No TMA multicast: each CTA loads its own boxes.
struct GemmPairCfg {
  static constexpr int BM = 128, BN = 256, BK = 64;  // per CTA: 128 rows of A, 128 rows of W
  static constexpr int A_BYTES = BM * BK * 2;        // 16 KB
  static constexpr int B_BYTES = (BN / 2) * BK * 2;  // 16 KB
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int STAGES = 6;
  static constexpr uint32_t TMEM_COLS = 512;         // two accumulators of 256 columns
  static constexpr int STG_BYTES = 4 * GEMM_STG_FLOATS * 4;  // the epilogue warps' staging
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM = STAGES * STAGE + STG_BYTES + BAR_BYTES + 1024;
  static constexpr uint32_t IDESC = umma_idesc_bf16(256, BN);
  static constexpr int THREADS = 192;
  static_assert(STAGE % 1024 == 0, "stages stay 1024-byte aligned for the 128-byte swizzle");
};

template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(GemmPairCfg::THREADS, 1)
    gemm_bf16_pair_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tw,
                          const GemmParams p) {
  using G = GemmPairCfg;
  extern __shared__ __align__(1024) unsigned char gemm_smem_raw[];
  unsigned char* sm = gemm_smem_raw + ((1024u - (smem_u32(gemm_smem_raw) & 1023u)) & 1023u);
  float* stg_all = reinterpret_cast<float*>(sm + G::STAGES * G::STAGE);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + G::STAGES * G::STAGE + G::STG_BYTES);
  uint64_t* empty = full + G::STAGES;
  uint64_t* tfull = empty + G::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < G::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);  // four epilogue warps in each CTA
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tslot, G::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before_sync();
  cluster_sync();  // both CTAs' barriers and the pair's TMEM are ready
  tc_fence_after_sync();
  pdl_wait();
  pdl_trigger();
  const uint32_t tmem = *tslot;
  const int npairs = gridDim.x >> 1;
  const int total = p.m_tiles * p.n_tiles * p.batch;
  const int kblocks = (p.K + G::BK - 1) / G::BK;

  if (warp == 0) {
    if (lane == 0) {  // ------------------------------------------ TMA producer (both CTAs)
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      for (int t = blockIdx.x >> 1; t < total; t += npairs) {
        int z, mt, nt;
        gemm_tile(t, p.m_tiles, p.n_tiles, z, mt, nt);
        const int ay = (int)(z * p.a_brows) + mt * 256 + (int)rank * 128;
        const int wy = (int)(z * p.w_brows) + nt * G::BN + (int)rank * (G::BN / 2);
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!gemm_wait(&empty[stage], phase ^ 1u, abort_flag)) { ok = false; break; }
          if (leader) mbar_expect_tx(&full[stage], 2 * G::STAGE);
          const uint32_t bar0 = mapa_shared(smem_u32(&full[stage]), 0);
          unsigned char* st = sm + stage * G::STAGE;
          tma_load_2d_pair(st, &ta, bar0, kb * G::BK, ay);
          tma_load_2d_pair(st + G::A_BYTES, &tw, bar0, kb * G::BK, wy);
          ++issued;
          if (++stage == G::STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
      }
      if (*abort_flag) {
        if (leader) {  // the phases peer 0 expected cover both CTAs' loads
          for (int s = 0; s < G::STAGES; ++s) {
            if (issued <= s) break;
            mbar_wait(&full[s], s < stage ? phase : phase ^ 1u);
          }
        } else {  // peer 1 cannot see its loads complete: give them time to land
          const unsigned long long t0 = global_ns();
          while (global_ns() - t0 < 200000ull) __nanosleep(1000);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {  // ---------------------------------- MMA issuer (peer 0)
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool any = false;
      for (int t = blockIdx.x >> 1; t < total; t += npairs) {
        if (!gemm_wait(&tempty[acc], acc_phase ^ 1u, abort_flag)) break;
        tc_fence_after_sync();
        const uint32_t d = tmem + (uint32_t)(acc * G::BN);
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!gemm_wait(&full[stage], phase, abort_flag)) { ok = false; break; }
          tc_fence_after_sync();
          const uint32_t a0 = smem_u32(sm + stage * G::STAGE), b0 = a0 + G::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < G::BK / 16; ++kk)
            umma_bf16_pair(d, umma_desc_sw128(a0 + kk * 32), umma_desc_sw128(b0 + kk * 32), G::IDESC,
                           (kb | kk) != 0 ? 1u : 0u);
          any = true;
          umma_commit_pair_multicast(&empty[stage], 0x3);  // both CTAs' stage is free
          if (++stage == G::STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit_pair_multicast(&tfull[acc], 0x3);  // both halves of the tile are complete
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      if (any) {
        umma_commit_pair(drain);
        mbar_wait(drain, 0);
      }
    }
  } else {  // ------------------------------------------------- epilogue (both CTAs)
    const int q = warp & 3;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x >> 1; t < total; t += npairs) {
      int z, mt, nt;
      gemm_tile(t, p.m_tiles, p.n_tiles, z, mt, nt);
      bool ok = gemm_wait(&tfull[acc], acc_phase, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after_sync();
      const int row0 = mt * 256 + (int)rank * 128 + q * 32;
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * G::BN);
      gemm_epilogue_tile<G::BN, EPI>(p, tbase, z, row0, min(32, p.M - row0), nt,
                                     stg_all + q * GEMM_STG_FLOATS);
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) {
        if (leader) mbar_arrive(&tempty[acc]);
        else mbar_arrive_remote(mapa_shared(smem_u32(&tempty[acc]), 0));
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }
  if (threadIdx.x == 0 && *abort_flag) atomicAdd(&g_gemm_wait_timeouts, 1u);
  tc_fence_before_sync();
  cluster_sync();  // no CTA leaves while its peer may still read its operands or barriers
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc_pair(tmem, G::TMEM_COLS);
  }
}

// ------------------------------------------------------- split K in a cluster
// Few rows (a decode batch): too few output tiles to occupy the GPU, and every
// column tile re-reads the same activation rows.  The K blocks of one output
// tile are split over the `ks` CTAs of a cluster (ks <= 8): each CTA multiplies
// its slice into TMEM, parks the fp32 partial tile in its own shared memory,
// and after a cluster barrier reduces 128 / ks rows of the tile by reading all
// ks partials through distributed shared memory, in rank order (deterministic),
// then applies the epilogue.  One tile per cluster, no atomics.
template <int BN>
struct GemmSplitCfg {
  static constexpr int BM = 128, BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int STAGES = std::min(8, (192 * 1024) / STAGE);
  static constexpr int PSTRIDE = BN + 4;  // floats per partial row (bank spread)
  static constexpr int P_BYTES = BM * PSTRIDE * 4;
  static constexpr int BODY = STAGES * STAGE > P_BYTES ? STAGES * STAGE : P_BYTES;
  static constexpr uint32_t TMEM_COLS = BN < 32 ? 32 : BN;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM = BODY + BAR_BYTES + 1024;
  static constexpr uint32_t IDESC = umma_idesc_bf16(BM, BN);
  static constexpr int THREADS = 192;
};

// Epilogue of four consecutive output columns (col .. col+3) of one row.
// `old`: the four outputs' previous values when the caller loaded them ahead
// (p.beta != 0, whole float4 groups), else null.
template <int EPI>
YUF_DEVICE void store4(const GemmParams& p, int z, int row, int col, float4 v, const float4* old = nullptr) {
  const bool full = p.vec && col + 4 <= p.N;
  if constexpr (EPI == GEMM_EPI_F32) {
    if (p.tanh_batch0 && z == 0) {
      v.x = tanhf(v.x); v.y = tanhf(v.y); v.z = tanhf(v.z); v.w = tanhf(v.w);
    }
    float* out = static_cast<float*>(p.C) + (size_t)z * p.c_bstride + (size_t)row * p.ldc + col;
    if (full) {
      if (p.beta != 0.f) {
        const float4 o = old ? *old : *reinterpret_cast<const float4*>(out);
        v.x += o.x; v.y += o.y; v.z += o.z; v.w += o.w;
      }
      *reinterpret_cast<float4*>(out) = v;
    } else {
      const float e[4] = {v.x, v.y, v.z, v.w};
      for (int c = 0; c < 4; ++c)
        if (col + c < p.N) out[c] = p.beta != 0.f ? out[c] + e[c] : e[c];
    }
  } else {
    if (p.tanh_batch0 && z == 0) {
      v.x = tanhf(v.x); v.y = tanhf(v.y); v.z = tanhf(v.z); v.w = tanhf(v.w);
    }
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.C) + (size_t)z * p.c_bstride + (size_t)row * p.ldc + col;
    if (full) {
      uint2 pk;
      reinterpret_cast<__nv_bfloat162*>(&pk)[0] = __floats2bfloat162_rn(v.x, v.y);
      reinterpret_cast<__nv_bfloat162*>(&pk)[1] = __floats2bfloat162_rn(v.z, v.w);
      *reinterpret_cast<uint2*>(out) = pk;
    } else {
      const float e[4] = {v.x, v.y, v.z, v.w};
      for (int c = 0; c < 4; ++c)
        if (col + c < p.N) out[c] = __float2bfloat16_rn(e[c]);
    }
  }
}

// The reduction step of a K split over a cluster: the calling CTA (rank r of
// KS) sums rows [r * 128 / KS, (r + 1) * 128 / KS) of the KS partial tiles
// (fp32, row stride pstride floats, at shared address `pbase` in every CTA) in
// rank order and applies the epilogue; all `nthreads` threads of the CTA take
// part.  KS is a template argument so that a thread's KS distributed-shared-
// memory loads of one element group are all in flight at once (a remote load
// costs hundreds of cycles; issued one after another they made the reduction
// the longest phase of a decode-batch GEMM).
template <int BN, int EPI, int KS, int LOADS>
YUF_DEVICE void cluster_reduce_store_ks(const GemmParams& p, uint32_t pbase, int pstride, int r, int z, int mt,
                                        int nt, int nthreads) {
  constexpr int ks = KS;
  const int rows = 128 / ks, r0 = r * rows;
  if constexpr (EPI == GEMM_EPI_SWIGLU || EPI == GEMM_EPI_SWIGLU_F32) {
    constexpr int QC = BN / 8;  // float4 chunks of "in" columns per row (BN / 2 columns)
    constexpr int U = 2 * KS >= LOADS ? 1 : LOADS / (2 * KS);  // groups per thread and step (2 U KS loads)
    const int total = rows * QC;
    for (int i0 = threadIdx.x; i0 < total; i0 += nthreads * U) {
      float4 xs[U][KS], ys[U][KS];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = min(i0 + u * nthreads, total - 1);
        const int rr = r0 + i / QC, j = (i % QC) * 4;
        const int cin = (j / 64) * 128 + j % 64, cgate = cin + 64;
#pragma unroll
        for (int qq = 0; qq < KS; ++qq) {
          xs[u][qq] = ld_shared_cluster_f4(mapa_shared(pbase + (uint32_t)((rr * pstride + cin) * 4), qq));
          ys[u][qq] = ld_shared_cluster_f4(mapa_shared(pbase + (uint32_t)((rr * pstride + cgate) * 4), qq));
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = i0 + u * nthreads;
        if (i >= total) break;
        const int rr = r0 + i / QC, j = (i % QC) * 4;  // j: 0 .. BN/2 - 4
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f), g = a;
#pragma unroll
        for (int qq = 0; qq < KS; ++qq) {
          a.x += xs[u][qq].x; a.y += xs[u][qq].y; a.z += xs[u][qq].z; a.w += xs[u][qq].w;
          g.x += ys[u][qq].x; g.y += ys[u][qq].y; g.z += ys[u][qq].z; g.w += ys[u][qq].w;
        }
        const int row = mt * 128 + rr, col = nt * (BN / 2) + j;
        if (row >= p.M) continue;
        const float h[4] = {silu(a.x) * g.x, silu(a.y) * g.y, silu(a.z) * g.z, silu(a.w) * g.w};
        const bool full = p.vec && col + 4 <= p.n_out;
        if constexpr (EPI == GEMM_EPI_SWIGLU_F32) {
          float* out = static_cast<float*>(p.C) + (size_t)z * p.c_bstride + (size_t)row * p.ldc;
          if (full) *reinterpret_cast<float4*>(out + col) = make_float4(h[0], h[1], h[2], h[3]);
          else
            for (int c = 0; c < 4; ++c)
              if (col + c < p.n_out) out[col + c] = h[c];
        } else {
          __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.C) + (size_t)z * p.c_bstride + (size_t)row * p.ldc;
          if (full) {
            uint2 pk;
            reinterpret_cast<__nv_bfloat162*>(&pk)[0] = __floats2bfloat162_rn(h[0], h[1]);
            reinterpret_cast<__nv_bfloat162*>(&pk)[1] = __floats2bfloat162_rn(h[2], h[3]);
            *reinterpret_cast<uint2*>(out + col) = pk;
          } else {
            for (int c = 0; c < 4; ++c)
              if (col + c < p.n_out) out[col + c] = __float2bfloat16_rn(h[c]);
          }
        }
      }
    }
  } else {
    constexpr int QC = BN / 4;
    constexpr int U = KS >= LOADS ? 1 : LOADS / KS;  // groups per thread and step (U KS loads in flight)
    const int total = rows * QC;
    // the residual (p.beta != 0) is loaded with the partials, not behind them
    const bool pre = EPI == GEMM_EPI_F32 && p.beta != 0.f && p.vec;
    for (int i0 = threadIdx.x; i0 < total; i0 += nthreads * U) {
      float4 xs[U][KS], old[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = min(i0 + u * nthreads, total - 1);
        const int rr = r0 + i / QC, c = (i % QC) * 4;
#pragma unroll
        for (int qq = 0; qq < KS; ++qq)
          xs[u][qq] = ld_shared_cluster_f4(mapa_shared(pbase + (uint32_t)((rr * pstride + c) * 4), qq));
        const int row = mt * 128 + rr, col = nt * BN + c;
        old[u] = pre && row < p.M && col + 4 <= p.N
                     ? *reinterpret_cast<const float4*>(static_cast<const float*>(p.C) + (size_t)z * p.c_bstride +
                                                        (size_t)row * p.ldc + col)
                     : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = i0 + u * nthreads;
        if (i >= total) break;
        const int rr = r0 + i / QC, c = (i % QC) * 4;
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int qq = 0; qq < KS; ++qq) {
          a.x += xs[u][qq].x; a.y += xs[u][qq].y; a.z += xs[u][qq].z; a.w += xs[u][qq].w;
        }
        const int row = mt * 128 + rr, col = nt * BN + c;
        if (row < p.M && col < p.N) store4<EPI>(p, z, row, col, a, pre ? &old[u] : nullptr);
      }
    }
  }
}

// LOADS: distributed-shared-memory loads a thread keeps in flight (fewer for
// register-heavy callers).
#ifndef GEMM_SPLIT_LOADS
#define GEMM_SPLIT_LOADS 8
#endif
template <int BN, int EPI, int LOADS = GEMM_SPLIT_LOADS>
YUF_DEVICE void cluster_reduce_store(const GemmParams& p, uint32_t pbase, int pstride, int ks, int r, int z,
                                     int mt, int nt, int nthreads) {
  switch (ks) {
    case 1: cluster_reduce_store_ks<BN, EPI, 1, LOADS>(p, pbase, pstride, r, z, mt, nt, nthreads); break;
    case 2: cluster_reduce_store_ks<BN, EPI, 2, LOADS>(p, pbase, pstride, r, z, mt, nt, nthreads); break;
    case 4: cluster_reduce_store_ks<BN, EPI, 4, LOADS>(p, pbase, pstride, r, z, mt, nt, nthreads); break;
    default: cluster_reduce_store_ks<BN, EPI, 8, LOADS>(p, pbase, pstride, r, z, mt, nt, nthreads); break;
  }
}

// The epilogue from this CTA's own shared memory: `recv` holds ks slices of
// 128 / ks rows (slice q at q * (128 / ks) rows, rows of pstride floats), summed
// in slice order -- the order of cluster_reduce_store -- for rows
// [r * 128 / ks, ...) of the tile.  With ks = 1 (no K split) it is the whole
// tile straight from the partial, without distributed-shared-memory loads or
// cluster barriers.
template <int BN, int EPI>
YUF_DEVICE void local_reduce_store(const GemmParams& p, const float* recv, int pstride, int ks, int r, int z,
                                   int mt, int nt, int nthreads) {
  const int rows = 128 / ks, r0 = r * rows;
  const int slice = rows * pstride;
  if constexpr (EPI == GEMM_EPI_SWIGLU) {
    constexpr int QC = BN / 8;
    for (int i = threadIdx.x; i < rows * QC; i += nthreads) {
      const int lr = i / QC, j = (i % QC) * 4;
      const int cin = (j / 64) * 128 + j % 64, cgate = cin + 64;
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f), g = a;
      for (int qq = 0; qq < ks; ++qq) {
        const float4 x = *reinterpret_cast<const float4*>(recv + qq * slice + lr * pstride + cin);
        const float4 y = *reinterpret_cast<const float4*>(recv + qq * slice + lr * pstride + cgate);
        a.x += x.x; a.y += x.y; a.z += x.z; a.w += x.w;
        g.x += y.x; g.y += y.y; g.z += y.z; g.w += y.w;
      }
      const int row = mt * 128 + r0 + lr, col = nt * (BN / 2) + j;
      if (row >= p.M) continue;
      const float h[4] = {silu(a.x) * g.x, silu(a.y) * g.y, silu(a.z) * g.z, silu(a.w) * g.w};
      __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.C) + (size_t)z * p.c_bstride + (size_t)row * p.ldc;
      if (p.vec && col + 4 <= p.n_out) {
        uint2 pk;
        reinterpret_cast<__nv_bfloat162*>(&pk)[0] = __floats2bfloat162_rn(h[0], h[1]);
        reinterpret_cast<__nv_bfloat162*>(&pk)[1] = __floats2bfloat162_rn(h[2], h[3]);
        *reinterpret_cast<uint2*>(out + col) = pk;
      } else {
        for (int c = 0; c < 4; ++c)
          if (col + c < p.n_out) out[col + c] = __float2bfloat16_rn(h[c]);
      }
    }
  } else {
    constexpr int QC = BN / 4, U = 8;
    // the residual (p.beta != 0) of U groups is loaded before their sums
    const bool pre = EPI == GEMM_EPI_F32 && p.beta != 0.f && p.vec;
    const int total = rows * QC;
    for (int i0 = threadIdx.x; i0 < total; i0 += U * nthreads) {
      float4 old[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = i0 + u * nthreads;
        const int row = mt * 128 + r0 + i / QC, col = nt * BN + (i % QC) * 4;
        old[u] = pre && i < total && row < p.M && col + 4 <= p.N
                     ? *reinterpret_cast<const float4*>(static_cast<const float*>(p.C) + (size_t)z * p.c_bstride +
                                                        (size_t)row * p.ldc + col)
                     : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = i0 + u * nthreads;
        if (i >= total) break;
        const int lr = i / QC, c = (i % QC) * 4;
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int qq = 0; qq < ks; ++qq) {
          const float4 x = *reinterpret_cast<const float4*>(recv + qq * slice + lr * pstride + c);
          a.x += x.x; a.y += x.y; a.z += x.z; a.w += x.w;
        }
        const int row = mt * 128 + r0 + lr, col = nt * BN + c;
        if (row < p.M && col < p.N) store4<EPI>(p, z, row, col, a, pre ? &old[u] : nullptr);
      }
    }
  }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(GemmSplitCfg<BN>::THREADS, 1)
    gemm_bf16_splitk_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tw,
                            const GemmParams p, int ks, int kb_per) {
  using G = GemmSplitCfg<BN>;
  extern __shared__ __align__(1024) unsigned char gemm_smem_raw[];
  unsigned char* sm = gemm_smem_raw + ((1024u - (smem_u32(gemm_smem_raw) & 1023u)) & 1023u);
  float* part = reinterpret_cast<float*>(sm);  // the partial tile, once the MMAs are done
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + G::BODY);
  uint64_t* empty = full + G::STAGES;
  uint64_t* tfull = empty + G::STAGES;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(tfull + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = (int)cluster_rank();
  const int tile = blockIdx.x / ks;
  const int per = p.m_tiles * p.n_tiles;
  const int z = tile / per, mt = (tile % per) / p.n_tiles, nt = tile % p.n_tiles;
  const int kblocks = (p.K + G::BK - 1) / G::BK;
  const int kb0 = r * kb_per, kb1 = min(kblocks, kb0 + kb_per), nkb = max(0, kb1 - kb0);
  if (threadIdx.x == 0) {
    for (int s = 0; s < G::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tslot, G::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  // The TMA producer thread waits for the previous kernel later, after it has
  // requested its first weight tiles: the weights are not written by any
  // kernel of the chain, so their HBM latency overlaps the previous kernel's tail.
  if (warp != 0 || lane != 0) pdl_wait();
  pdl_trigger();
  const uint32_t tmem = *tslot;

  if (warp == 0) {
    if (lane == 0) {  // TMA producer over this CTA's K slice
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      const int ay = (int)(z * p.a_brows) + mt * G::BM, wy = (int)(z * p.w_brows) + nt * BN;
      const int pre = min(nkb, G::STAGES);  // stages whose weight tile goes out before the wait
      for (int i = 0; i < pre; ++i) {
        mbar_expect_tx(&full[i], G::STAGE);
        tma_load_2d(sm + i * G::STAGE + G::A_BYTES, &tw, &full[i], (kb0 + i) * G::BK, wy);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i) tma_load_2d(sm + i * G::STAGE, &ta, &full[i], (kb0 + i) * G::BK, ay);
      issued = pre;
      stage = pre % G::STAGES;
      phase = pre == G::STAGES ? 1u : 0u;
      for (int kb = kb0 + pre; kb < kb1; ++kb) {
        if (!gemm_wait(&empty[stage], phase ^ 1u, abort_flag)) break;
        unsigned char* st = sm + stage * G::STAGE;
        mbar_expect_tx(&full[stage], G::STAGE);
        tma_load_2d(st, &ta, &full[stage], kb * G::BK, ay);
        tma_load_2d(st + G::A_BYTES, &tw, &full[stage], kb * G::BK, wy);
        ++issued;
        if (++stage == G::STAGES) { stage = 0; phase ^= 1u; }
      }
      if (*abort_flag)
        for (int s = 0; s < G::STAGES; ++s) {
          if (issued <= s) break;
          mbar_wait(&full[s], s < stage ? phase : phase ^ 1u);
        }
    }
  } else if (warp == 1) {
    if (lane == 0 && nkb > 0) {  // MMA issuer
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int i = 0; i < nkb; ++i) {
        if (!gemm_wait(&full[stage], phase, abort_flag)) { ok = false; break; }
        tc_fence_after_sync();
        const uint32_t a0 = smem_u32(sm + stage * G::STAGE), b0 = a0 + G::A_BYTES;
#pragma unroll
        for (int kk = 0; kk < G::BK / 16; ++kk)
          umma_bf16(tmem, umma_desc_sw128(a0 + kk * 32), umma_desc_sw128(b0 + kk * 32), G::IDESC,
                    (i | kk) != 0 ? 1u : 0u);
        umma_commit(&empty[stage]);
        if (++stage == G::STAGES) { stage = 0; phase ^= 1u; }
      }
      umma_commit(tfull);  // also when a wait expired: every MMA issued ends before the tile is read
      (void)ok;
    }
  } else {  // epilogue warps: the partial tile into shared memory
    const int q = warp & 3;
    const int prow = q * 32 + lane;
    float* dst = part + (size_t)prow * G::PSTRIDE;
    bool ok = nkb == 0 || mbar_wait(tfull, 0);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) *abort_flag = 1;
    if (nkb > 0 && ok) {
      tc_fence_after_sync();
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        float v[32];
        tmem_ld_x32(tbase + c0, v);
#pragma unroll
        for (int c = 0; c < 32; c += 4)
          *reinterpret_cast<float4*>(dst + c0 + c) = make_float4(v[c], v[c + 1], v[c + 2], v[c + 3]);
      }
    } else {
      for (int c = 0; c < BN; c += 4) *reinterpret_cast<float4*>(dst + c) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  tc_fence_before_sync();
  if (ks > 1) {
    cluster_sync();  // every CTA's partial is in its shared memory
    // reduce rows [r * 128 / ks, (r + 1) * 128 / ks) over the ks partials, in rank order
    cluster_reduce_store<BN, EPI>(p, smem_u32(part), G::PSTRIDE, ks, r, z, mt, nt, G::THREADS);
    cluster_sync();  // no CTA leaves while a peer may still read its partial
  } else {
    __syncthreads();  // no split: the whole tile from this CTA's own shared memory
    local_reduce_store<BN, EPI>(p, part, G::PSTRIDE, 1, 0, z, mt, nt, G::THREADS);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicAdd(&g_gemm_wait_timeouts, 1u);
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, G::TMEM_COLS);
  }
}

// ------------------------------------------------------------- fp32 (3xTF32)
// fp32 weights at fp32 accuracy: every product as three kind::tf32 UMMAs,
// A_lo W_hi + A_hi W_lo + A_hi W_hi (the low parts' product, ~2^-20 relative,
// is dropped).  The weight arrives already split (host, at load time); the
// activation tile arrives as fp32 and four converter warps split it in shared
// memory -- the high part (low 13 mantissa bits cleared) in place, the
// remainder into a second tile of the same swizzled layout (the split is
// elementwise, so no index changes) -- before the MMA warp may read the stage.
// The tensor core's own accumulation drops low bits once the running sum grows
// (measured: ~1e-5 relative over K = 640 even with exact products), so each
// 32-wide K block goes into a fresh TMEM accumulator (two, alternating) and the
// epilogue warps add it to an fp32 register accumulator: the tensor core only
// ever sums 96 products.  One output tile per cluster of `ks` CTAs splitting K
// (ks = 1 for many rows), partials reduced through distributed shared memory as
// in the bf16 split-K kernel.
template <int BN>
struct GemmTf32Cfg {
  static constexpr int BM = 128, BK = 32;         // BK fp32 = one 128-byte swizzle row
  static constexpr int A_BYTES = BM * BK * 4;     // 16 KB, the high part after the split
  static constexpr int AL_BYTES = A_BYTES;        // the low part
  static constexpr int B_BYTES = BN * BK * 4;
  static constexpr int STAGE = A_BYTES + AL_BYTES + 2 * B_BYTES;
  static constexpr int STAGES = std::min(8, (192 * 1024) / STAGE);
  static constexpr int PSTRIDE = BN + 4;
  static constexpr int P_BYTES = BM * PSTRIDE * 4;
  static constexpr int BODY = STAGES * STAGE > P_BYTES ? STAGES * STAGE : P_BYTES;
  static constexpr uint32_t TMEM_COLS = 2 * BN;   // two K-block accumulators
  static constexpr int BAR_BYTES = 512;
  static constexpr int SMEM = BODY + BAR_BYTES + 1024;
  static constexpr uint32_t IDESC = umma_idesc_tf32(BM, BN);
  static constexpr int THREADS = 320;  // producer, MMA, 4 epilogue warps, 4 converter warps
  static_assert(STAGE % 1024 == 0, "stages stay 1024-byte aligned for the 128-byte swizzle");
  static_assert(BN == 64 || BN == 128, "tile width");
};

template <int BN, int EPI>
__global__ void __launch_bounds__(GemmTf32Cfg<BN>::THREADS, 1)
    gemm_tf32x3_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap twh,
                       const __grid_constant__ CUtensorMap twl, const GemmParams p, int ks, int kb_per) {
  using G = GemmTf32Cfg<BN>;
  extern __shared__ __align__(1024) unsigned char gemm_smem_raw[];
  unsigned char* sm = gemm_smem_raw + ((1024u - (smem_u32(gemm_smem_raw) & 1023u)) & 1023u);
  float* part = reinterpret_cast<float*>(sm);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + G::BODY);
  uint64_t* conv = full + G::STAGES;
  uint64_t* empty = conv + G::STAGES;
  uint64_t* tfull = empty + G::STAGES;  // [2]
  uint64_t* tempty = tfull + 2;         // [2]
  uint64_t* drain = tempty + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = (int)cluster_rank();
  const int tile = blockIdx.x / ks;
  const int per = p.m_tiles * p.n_tiles;
  const int z = tile / per, mt = (tile % per) / p.n_tiles, nt = tile % p.n_tiles;
  const int kblocks = (p.K + G::BK - 1) / G::BK;
  const int kb0 = r * kb_per, kb1 = min(kblocks, kb0 + kb_per), nkb = max(0, kb1 - kb0);
  if (threadIdx.x == 0) {
    for (int s = 0; s < G::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 4);  // one arrival per converter warp
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);  // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tslot, G::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  pdl_wait();
  pdl_trigger();
  const uint32_t tmem = *tslot;

  if (warp == 0) {
    if (lane == 0) {  // TMA: the fp32 activation tile and both weight parts
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      const int ay = (int)(z * p.a_brows) + mt * G::BM, wy = (int)(z * p.w_brows) + nt * BN;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!gemm_wait(&empty[stage], phase ^ 1u, abort_flag)) break;
        unsigned char* st = sm + stage * G::STAGE;
        mbar_expect_tx(&full[stage], G::A_BYTES + 2 * G::B_BYTES);
        tma_load_2d(st, &ta, &full[stage], kb * G::BK, ay);
        tma_load_2d(st + G::A_BYTES + G::AL_BYTES, &twh, &full[stage], kb * G::BK, wy);
        tma_load_2d(st + G::A_BYTES + G::AL_BYTES + G::B_BYTES, &twl, &full[stage], kb * G::BK, wy);
        ++issued;
        if (++stage == G::STAGES) { stage = 0; phase ^= 1u; }
      }
      if (*abort_flag)
        for (int s = 0; s < G::STAGES; ++s) {
          if (issued <= s) break;
          mbar_wait(&full[s], s < stage ? phase : phase ^ 1u);
        }
    }
  } else if (warp == 1) {
    if (lane == 0 && nkb > 0) {  // MMA issuer: a fresh accumulator per K block
      int stage = 0;
      uint32_t phase = 0;
      bool any = false;
      for (int i = 0; i < nkb; ++i) {
        const int acc = i & 1;
        if (!gemm_wait(&tempty[acc], ((uint32_t)(i >> 1) & 1u) ^ 1u, abort_flag)) break;
        if (!gemm_wait(&conv[stage], phase, abort_flag)) break;
        tc_fence_after_sync();
        const uint32_t d = tmem + (uint32_t)(acc * BN);
        const uint32_t ah = smem_u32(sm + stage * G::STAGE), al = ah + G::A_BYTES;
        const uint32_t bh = al + G::AL_BYTES, bl = bh + G::B_BYTES;
#pragma unroll
        for (int kk = 0; kk < G::BK / 8; ++kk) {
          const uint32_t o = kk * 32;
          umma_tf32(d, umma_desc_sw128(al + o), umma_desc_sw128(bh + o), G::IDESC, kk != 0 ? 1u : 0u);
          umma_tf32(d, umma_desc_sw128(ah + o), umma_desc_sw128(bl + o), G::IDESC, 1u);
          umma_tf32(d, umma_desc_sw128(ah + o), umma_desc_sw128(bh + o), G::IDESC, 1u);
        }
        any = true;
        umma_commit(&empty[stage]);
        umma_commit(&tfull[acc]);
        if (++stage == G::STAGES) { stage = 0; phase ^= 1u; }
      }
      if (any) {  // every MMA issued has finished before the columns are freed
        umma_commit(drain);
        mbar_wait(drain, 0);
      }
    }
  } else if (warp >= 6) {  // converters: split each landed activation tile
    const int ct = threadIdx.x - 192;  // 0 .. 127
    int stage = 0;
    uint32_t phase = 0;
    for (int i = 0; i < nkb; ++i) {
      bool ok = gemm_wait(&full[stage], phase, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      unsigned char* st = sm + stage * G::STAGE;
#pragma unroll
      for (int c = 0; c < G::A_BYTES / 16 / 128; ++c) {
        const int off = (c * 128 + ct) * 16;
        uint4 x = *reinterpret_cast<const uint4*>(st + off), hi, lo;
        split4(*reinterpret_cast<const float4*>(&x), hi, lo);
        *reinterpret_cast<uint4*>(st + off) = hi;
        *reinterpret_cast<uint4*>(st + G::A_BYTES + off) = lo;
      }
      fence_proxy_async();  // the split tiles become visible to the tensor core
      __syncwarp();
      if (lane == 0) mbar_arrive(&conv[stage]);
      if (++stage == G::STAGES) { stage = 0; phase ^= 1u; }
    }
  } else {  // epilogue warps 2-5: sum the K-block accumulators in fp32 registers
    const int q = warp & 3;
    const int prow = q * 32 + lane;
    const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16);
    float racc[BN];
#pragma unroll
    for (int c = 0; c < BN; ++c) racc[c] = 0.f;
    bool ok = true;
    for (int i = 0; i < nkb && ok; ++i) {
      const int acc = i & 1;
      ok = gemm_wait(&tfull[acc], (uint32_t)(i >> 1) & 1u, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after_sync();
#pragma unroll
      for (int c0 = 0; c0 < BN; c0 += 32) {
        float v[32];
        tmem_ld_x32(tbase + (uint32_t)(acc * BN + c0), v);
#pragma unroll
        for (int c = 0; c < 32; ++c) racc[c0 + c] += v[c];
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
    if (!ok) *abort_flag = 1;
    const int row = mt * G::BM + prow;
    if (ks == 1) {
      if (ok && row < p.M) {
        if constexpr (EPI == GEMM_EPI_SWIGLU_F32) {
          float* out = static_cast<float*>(p.C) + (size_t)z * p.c_bstride + (size_t)row * p.ldc;
#pragma unroll
          for (int sb = 0; sb < BN / 128; ++sb)
#pragma unroll
            for (int j = 0; j < 64; j += 4) {
              const int col = nt * (BN / 2) + sb * 64 + j;
              float h[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) h[e] = silu(racc[sb * 128 + j + e]) * racc[sb * 128 + 64 + j + e];
              if (p.vec && col + 4 <= p.n_out) *reinterpret_cast<float4*>(out + col) = make_float4(h[0], h[1], h[2], h[3]);
              else
                for (int e = 0; e < 4; ++e)
                  if (col + e < p.n_out) out[col + e] = h[e];
            }
        } else {
#pragma unroll
          for (int c = 0; c < BN; c += 4) {
            const int col = nt * BN + c;
            if (col < p.N) store4<GEMM_EPI_F32>(p, z, row, col, make_float4(racc[c], racc[c + 1], racc[c + 2], racc[c + 3]));
          }
        }
      }
    } else {
      float* dst = part + (size_t)prow * G::PSTRIDE;
#pragma unroll
      for (int c = 0; c < BN; c += 4)
        *reinterpret_cast<float4*>(dst + c) =
            ok ? make_float4(racc[c], racc[c + 1], racc[c + 2], racc[c + 3]) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  tc_fence_before_sync();
  if (ks > 1) {
    cluster_sync();  // every CTA's partial is in its shared memory
    cluster_reduce_store<BN, EPI, 2>(p, smem_u32(part), G::PSTRIDE, ks, r, z, mt, nt, G::THREADS);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicAdd(&g_gemm_wait_timeouts, 1u);
  cluster_sync();  // no CTA leaves while a peer may still read its partial
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, G::TMEM_COLS);
  }
}

// ------------------------------------------------------------------- host side
static int sm_count() {
  static int cache[128] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = 148;
    }
    cache[dev] = n;
  }
  return cache[dev];
}

// The dynamic shared-memory limit of a kernel, set once per (kernel, device);
// must precede occupancy queries as well as launches.
static cudaError_t set_smem_once(const void* fn, int smem) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, cudaError_t> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  auto key = std::make_pair(fn, dev);
  auto it = done.find(key);
  if (it != done.end()) return it->second;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) cudaGetLastError();
  done[key] = e;
  return e;
}

static bool make_bf16_map(CUtensorMap* m, const void* base, long long inner, long long rows,
                          long long ld, int box_rows) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  const cuuint64_t gdim[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  const cuuint64_t gstride[1] = {(cuuint64_t)ld * 2};
  const cuuint32_t box[2] = {64u, (cuuint32_t)box_rows};
  const cuuint32_t estride[2] = {1u, 1u};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), gdim, gstride, box,
             estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int EPI>
static yuf_status_t launch_gemm(const GemmArgs& g, GemmParams p, cudaStream_t s) {
  using G = GemmCfg<BN>;
  const cudaError_t attr_err = set_smem_once((const void*)gemm_bf16_kernel<BN, EPI>, G::SMEM);
  if (attr_err != cudaSuccess) {
    set_error("gemm: cannot set %d bytes of shared memory: %s", G::SMEM, cudaGetErrorString(attr_err));
    return YUF_ERR_CUDA;
  }
  CUtensorMap ta, tw;
  if (!make_bf16_map(&ta, g.A, g.K, g.a_rows, g.lda, G::BM) ||
      !make_bf16_map(&tw, g.W, g.K, g.w_rows, g.K, BN)) {
    set_error("gemm: cuTensorMapEncodeTiled failed (A rows %lld, lda %lld, W rows %lld, K %d)", g.a_rows,
              g.lda, g.w_rows, g.K);
    return YUF_ERR_CUDA;
  }
  p.n_tiles = (p.N + BN - 1) / BN;
  const long long total = (long long)p.m_tiles * p.n_tiles * p.batch;
  const int grid = (int)std::min<long long>(total, sm_count());
  launch_k(gemm_bf16_kernel<BN, EPI>, dim3(grid), dim3(G::THREADS), G::SMEM, s, ta, tw, p);
  return check_launch("gemm_bf16_kernel");
}

// CTA pairs of the pair kernel that can be resident at once on this device.
static int pair_slots(const void* fn, int smem) {
  static int cache[128][3] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  dev &= 127;
  const int slot = fn == (const void*)gemm_bf16_pair_kernel<GEMM_EPI_F32> ? 0
                   : fn == (const void*)gemm_bf16_pair_kernel<GEMM_EPI_BF16> ? 1 : 2;
  if (cache[dev][slot] == 0) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2 * 74, 1, 1);
    cfg.blockDim = dim3(GemmPairCfg::THREADS, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    set_smem_once(fn, smem);
    if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = sm_count() / 2;
    }
    cache[dev][slot] = n;
  }
  return cache[dev][slot];
}

template <int EPI>
static yuf_status_t launch_gemm_pair(const GemmArgs& g, GemmParams p, cudaStream_t s) {
  using G = GemmPairCfg;
  const cudaError_t attr_err = set_smem_once((const void*)gemm_bf16_pair_kernel<EPI>, G::SMEM);
  if (attr_err != cudaSuccess) {
    set_error("gemm: cannot set %d bytes of shared memory: %s", G::SMEM, cudaGetErrorString(attr_err));
    return YUF_ERR_CUDA;
  }
  CUtensorMap ta, tw;
  if (!make_bf16_map(&ta, g.A, g.K, g.a_rows, g.lda, G::BM) ||
      !make_bf16_map(&tw, g.W, g.K, g.w_rows, g.K, G::BN / 2)) {
    set_error("gemm: cuTensorMapEncodeTiled failed (A rows %lld, lda %lld, W rows %lld, K %d)", g.a_rows,
              g.lda, g.w_rows, g.K);
    return YUF_ERR_CUDA;
  }
  p.m_tiles = (p.M + 255) / 256;
  p.n_tiles = (p.N + G::BN - 1) / G::BN;
  const long long total = (long long)p.m_tiles * p.n_tiles * p.batch;
  const int pairs = (int)std::min<long long>(total, pair_slots((const void*)gemm_bf16_pair_kernel<EPI>, G::SMEM));
  launch_k(gemm_bf16_pair_kernel<EPI>, dim3(2 * pairs), dim3(G::THREADS), G::SMEM, s, ta, tw, p);
  return check_launch("gemm_bf16_pair_kernel");
}

// Clusters of `ks` CTAs of the split-K kernel that can be resident at once.
template <int BN, int EPI>
static int splitk_slots(int ks) {
  static int cache[128][9] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  dev &= 127;
  if (cache[dev][ks] == 0) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(ks * 16, 1, 1);
    cfg.blockDim = dim3(GemmSplitCfg<BN>::THREADS, 1, 1);
    cfg.dynamicSmemBytes = GemmSplitCfg<BN>::SMEM;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = ks;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    set_smem_once((const void*)gemm_bf16_splitk_kernel<BN, EPI>, GemmSplitCfg<BN>::SMEM);
    if (cudaOccupancyMaxActiveClusters(&n, gemm_bf16_splitk_kernel<BN, EPI>, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = sm_count() / (2 * ks);
    }
    cache[dev][ks] = std::max(1, n);
  }
  return cache[dev][ks];
}

template <int BN, int EPI>
static yuf_status_t launch_gemm_splitk(const GemmArgs& g, GemmParams p, int ks, cudaStream_t s) {
  using G = GemmSplitCfg<BN>;
  const cudaError_t attr_err = set_smem_once((const void*)gemm_bf16_splitk_kernel<BN, EPI>, G::SMEM);
  if (attr_err != cudaSuccess) {
    set_error("gemm: cannot set %d bytes of shared memory: %s", G::SMEM, cudaGetErrorString(attr_err));
    return YUF_ERR_CUDA;
  }
  CUtensorMap ta, tw;
  if (!make_bf16_map(&ta, g.A, g.K, g.a_rows, g.lda, G::BM) || !make_bf16_map(&tw, g.W, g.K, g.w_rows, g.K, BN)) {
    set_error("gemm: cuTensorMapEncodeTiled failed (A rows %lld, lda %lld, W rows %lld, K %d)", g.a_rows,
              g.lda, g.w_rows, g.K);
    return YUF_ERR_CUDA;
  }
  p.n_tiles = (p.N + BN - 1) / BN;
  const int kblocks = (p.K + G::BK - 1) / G::BK;
  const int kb_per = (kblocks + ks - 1) / ks;
  const long long tiles = (long long)p.m_tiles * p.n_tiles * p.batch;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(tiles * ks), 1, 1);
  cfg.blockDim = dim3(G::THREADS, 1, 1);
  cfg.dynamicSmemBytes = G::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = ks;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (pdl_enabled()) {
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 2;
  }
  cudaLaunchKernelEx(&cfg, gemm_bf16_splitk_kernel<BN, EPI>, ta, tw, p, ks, kb_per);
  return check_launch("gemm_bf16_splitk_kernel");
}

// Launch plans of the persistent kernel are compared in one cost unit: rows
// of A and W tiles that a CTA streams per 64-wide K block, times the K blocks
// it covers, times the rounds its tiles take.
struct GemmPlan {
  double cost = -1;
  int bn = 128, ks = 1;
  bool split = false;
};

// Persistent one-CTA kernel: the column tile whose rounds of tiles cost least.
static GemmPlan plan_persistent(const GemmArgs& g, const GemmParams& p, int sms) {
  const long long kblocks = (g.K + 63) / 64;
  GemmPlan best;
  for (int bn : {256, 160, 128, 64}) {
    if (g.epi == GEMM_EPI_SWIGLU && (bn == 160 || bn < 128 || g.N % bn != 0)) continue;
    const long long tiles = (long long)p.m_tiles * ((g.N + bn - 1) / bn) * g.batch;
    const long long rounds = (tiles + sms - 1) / sms;
    const double cost = (double)rounds * kblocks * (128 + bn);
    if (best.cost < 0 || cost < best.cost) best = {cost, bn, 1, false};
  }
  return best;
}

// Few rows (a decode batch, at most two 128-row tiles): every plan of the
// persistent kernel and of the split-K kernel (K split over a cluster, partial
// tiles reduced through distributed shared memory) was timed on B200 as a
// chain of dependent launches (graph replay with programmatic dependent
// launch) over 13 projection shapes of 64-256 rows, and the times fitted, in
// microseconds, with kb the 64-wide K blocks a CTA covers:
//   persistent:           3.64 + 1.515e-3 kb (128 + BN) rounds
//   split-K, ks = 1:      5.99 + 1.515e-3 kb (128 + BN) waves  (+ 2.2 with a residual)
//   split-K, ks > 1:      4.65 + 1.515e-3 kb (128 + BN) + 1.64e-2 BN (ks - 1) / ks
// The last term is the reduction's distributed-shared-memory traffic.  A K
// split is taken only when its clusters fill at most 3/4 of the resident
// cluster slots: fuller launches of 8-CTA clusters ran as two waves.
template <int EPI>
static GemmPlan plan_few_rows(const GemmArgs& g, const GemmParams& p, int sms) {
  const int kblocks = (g.K + 63) / 64;
  GemmPlan best;
  for (int bn : {64, 128, 256}) {
    if (EPI == GEMM_EPI_SWIGLU && (bn < 128 || g.N % bn != 0)) continue;
    const long long tiles = (long long)p.m_tiles * ((g.N + bn - 1) / bn) * g.batch;
    const long long rounds = (tiles + sms - 1) / sms;
    const double per_kb = 1.515e-3 * (128 + bn);
    GemmPlan cand{3.64 + per_kb * kblocks * rounds, bn, 1, false};
    if (best.cost < 0 || cand.cost < best.cost) best = cand;
    for (int ks : {1, 2, 4, 8}) {
      if (ks > kblocks && ks > 1) continue;
      const int slots = bn == 64 ? splitk_slots<64, EPI>(ks)
                                 : (bn == 128 ? splitk_slots<128, EPI>(ks) : splitk_slots<256, EPI>(ks));
      if (ks > 1 && 4 * tiles > 3LL * slots) continue;
      const long long kb_per = (kblocks + ks - 1) / ks;
      const long long waves = (tiles + slots - 1) / slots;
      const double cost = ks == 1 ? 5.99 + per_kb * kb_per * waves + (g.beta != 0.f ? 2.2 : 0.0)
                                  : 4.65 + per_kb * kb_per + 1.64e-2 * bn * (ks - 1) / ks;
      if (cost < best.cost) best = {cost, bn, ks, true};
    }
  }
  return best;
}

template <int EPI>
static yuf_status_t launch_splitk_plan(const GemmArgs& g, const GemmParams& p, const GemmPlan& plan,
                                       cudaStream_t s) {
  if (plan.bn == 64) return launch_gemm_splitk<64, EPI>(g, p, plan.ks, s);
  if (plan.bn == 128) return launch_gemm_splitk<128, EPI>(g, p, plan.ks, s);
  return launch_gemm_splitk<256, EPI>(g, p, plan.ks, s);
}

yuf_status_t gemm_bf16(const GemmArgs& g, cudaStream_t s) {
  if (g.M <= 0 || g.N <= 0 || g.batch <= 0) return YUF_OK;
  const bool a_ok = (reinterpret_cast<uintptr_t>(g.A) & 15) == 0 && g.lda % 8 == 0;
  const bool w_ok = (reinterpret_cast<uintptr_t>(g.W) & 15) == 0;
  if (!a_ok || !w_ok || g.K % 8 != 0 || g.K <= 0) {
    set_error("gemm: operands need 16-byte aligned rows (A %p lda %lld, W %p, K %d)", g.A, g.lda, g.W, g.K);
    return YUF_ERR_INVALID_ARGUMENT;
  }
  GemmParams p{};
  p.C = g.C;
  p.ldc = g.ldc;
  p.c_bstride = g.c_bstride;
  p.M = g.M;
  p.N = g.N;
  p.K = g.K;
  p.batch = g.batch;
  p.a_brows = g.a_brows;
  p.w_brows = g.w_brows;
  p.beta = g.beta;
  p.tanh_batch0 = g.tanh_batch0;
  p.n_out = g.epi == GEMM_EPI_SWIGLU ? g.n_out : g.N;
  p.m_tiles = (g.M + 127) / 128;
  const int esz = g.epi == GEMM_EPI_F32 ? 4 : 2;
  const int vec_elems = 16 / esz;
  p.vec = (reinterpret_cast<uintptr_t>(g.C) & 15) == 0 && g.ldc % vec_elems == 0 &&
          g.c_bstride % vec_elems == 0;
  const int sms = sm_count();
  GemmPlan persistent = plan_persistent(g, p, sms);
  // a decode batch: the K split over a cluster or the persistent kernel,
  // whichever the timed model prefers
  if (p.m_tiles <= 2 && (g.epi != GEMM_EPI_SWIGLU || g.N % 128 == 0)) {
    GemmPlan few;
    if (g.epi == GEMM_EPI_F32) few = plan_few_rows<GEMM_EPI_F32>(g, p, sms);
    else if (g.epi == GEMM_EPI_BF16) few = plan_few_rows<GEMM_EPI_BF16>(g, p, sms);
    else few = plan_few_rows<GEMM_EPI_SWIGLU>(g, p, sms);
    if (few.split) {
      if (g.epi == GEMM_EPI_F32) return launch_splitk_plan<GEMM_EPI_F32>(g, p, few, s);
      if (g.epi == GEMM_EPI_BF16) return launch_splitk_plan<GEMM_EPI_BF16>(g, p, few, s);
      return launch_splitk_plan<GEMM_EPI_SWIGLU>(g, p, few, s);
    }
    persistent = few;
  }
  // enough 256 x 256 tiles to fill the pairs: the CTA-pair kernel
  const long long pair_tiles = (long long)((g.M + 255) / 256) * ((g.N + 255) / 256) * g.batch;
  if (g.M >= 512 && g.N >= 512 && pair_tiles >= sms / 2 && (g.epi != GEMM_EPI_SWIGLU || g.N % 256 == 0)) {
    if (g.epi == GEMM_EPI_F32) return launch_gemm_pair<GEMM_EPI_F32>(g, p, s);
    if (g.epi == GEMM_EPI_BF16) return launch_gemm_pair<GEMM_EPI_BF16>(g, p, s);
    return launch_gemm_pair<GEMM_EPI_SWIGLU>(g, p, s);
  }
  if (g.epi == GEMM_EPI_SWIGLU) {
    if (g.N % 128 != 0) {
      set_error("gemm: the SiLU-gate weight must hold whole 128-row groups (N = %d)", g.N);
      return YUF_ERR_INVALID_ARGUMENT;
    }
    return persistent.bn == 256 ? launch_gemm<256, GEMM_EPI_SWIGLU>(g, p, s)
                                : launch_gemm<128, GEMM_EPI_SWIGLU>(g, p, s);
  }
  const int bn = persistent.bn;
  if (g.epi == GEMM_EPI_F32) {
    if (bn == 64) return launch_gemm<64, GEMM_EPI_F32>(g, p, s);
    if (bn == 128) return launch_gemm<128, GEMM_EPI_F32>(g, p, s);
    if (bn == 160) return launch_gemm<160, GEMM_EPI_F32>(g, p, s);
    return launch_gemm<256, GEMM_EPI_F32>(g, p, s);
  }
  if (bn == 64) return launch_gemm<64, GEMM_EPI_BF16>(g, p, s);
  if (bn == 128) return launch_gemm<128, GEMM_EPI_BF16>(g, p, s);
  if (bn == 160) return launch_gemm<160, GEMM_EPI_BF16>(g, p, s);
  return launch_gemm<256, GEMM_EPI_BF16>(g, p, s);
}

// ---------------------------------------------------------------- 3xTF32 host
void split_tf32_host(const float* w, size_t n, float* hi, float* lo) {
  for (size_t i = 0; i < n; ++i) {
    uint32_t u;
    std::memcpy(&u, &w[i], 4);
    u &= 0xffffe000u;
    float h;
    std::memcpy(&h, &u, 4);
    hi[i] = h;
    lo[i] = w[i] - h;
  }
}

static bool make_f32_map(CUtensorMap* m, const void* base, long long inner, long long rows, long long ld,
                         int box_rows) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  const cuuint64_t gdim[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  const cuuint64_t gstride[1] = {(cuuint64_t)ld * 4};
  const cuuint32_t box[2] = {32u, (cuuint32_t)box_rows};
  const cuuint32_t estride[2] = {1u, 1u};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), gdim, gstride, box, estride,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int EPI>
static int tf32_slots(int ks) {
  static int cache[128][9] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  dev &= 127;
  if (cache[dev][ks] == 0) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(ks * 16, 1, 1);
    cfg.blockDim = dim3(GemmTf32Cfg<BN>::THREADS, 1, 1);
    cfg.dynamicSmemBytes = GemmTf32Cfg<BN>::SMEM;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = ks;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    set_smem_once((const void*)gemm_tf32x3_kernel<BN, EPI>, GemmTf32Cfg<BN>::SMEM);
    if (cudaOccupancyMaxActiveClusters(&n, gemm_tf32x3_kernel<BN, EPI>, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = sm_count() / (2 * ks);
    }
    cache[dev][ks] = std::max(1, n);
  }
  return cache[dev][ks];
}

template <int BN, int EPI>
static yuf_status_t launch_tf32(const GemmArgs& g, const void* W_lo, GemmParams p, int ks, cudaStream_t s) {
  using G = GemmTf32Cfg<BN>;
  const cudaError_t attr_err = set_smem_once((const void*)gemm_tf32x3_kernel<BN, EPI>, G::SMEM);
  if (attr_err != cudaSuccess) {
    set_error("gemm: cannot set %d bytes of shared memory: %s", G::SMEM, cudaGetErrorString(attr_err));
    return YUF_ERR_CUDA;
  }
  CUtensorMap ta, twh, twl;
  if (!make_f32_map(&ta, g.A, g.K, g.a_rows, g.lda, G::BM) || !make_f32_map(&twh, g.W, g.K, g.w_rows, g.K, BN) ||
      !make_f32_map(&twl, W_lo, g.K, g.w_rows, g.K, BN)) {
    set_error("gemm: cuTensorMapEncodeTiled failed (fp32; A rows %lld, lda %lld, W rows %lld, K %d)", g.a_rows,
              g.lda, g.w_rows, g.K);
    return YUF_ERR_CUDA;
  }
  p.n_tiles = (p.N + BN - 1) / BN;
  const int kblocks = (p.K + G::BK - 1) / G::BK;
  const int kb_per = (kblocks + ks - 1) / ks;
  const long long tiles = (long long)p.m_tiles * p.n_tiles * p.batch;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)(tiles * ks), 1, 1);
  cfg.blockDim = dim3(G::THREADS, 1, 1);
  cfg.dynamicSmemBytes = G::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = ks;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (pdl_enabled()) {
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 2;
  }
  cudaLaunchKernelEx(&cfg, gemm_tf32x3_kernel<BN, EPI>, ta, twh, twl, p, ks, kb_per);
  return check_launch("gemm_tf32x3_kernel");
}

template <int EPI>
static yuf_status_t dispatch_tf32(const GemmArgs& g, const void* W_lo, const GemmParams& p, cudaStream_t s) {
  const int kblocks = (g.K + 31) / 32;
  const int sms = sm_count();
  int best_bn = 0, best_ks = 1;
  long long best_cost = -1;
  for (int bn : {64, 128}) {
    if ((EPI == GEMM_EPI_SWIGLU_F32) && (bn < 128 || g.N % bn != 0)) continue;
    const long long tiles = (long long)p.m_tiles * ((g.N + bn - 1) / bn) * g.batch;
    for (int ks : {8, 4, 2, 1}) {
      if (ks > 1 && (ks > kblocks || p.m_tiles > 2)) continue;  // the K split serves few rows
      const int slots = bn == 64 ? tf32_slots<64, EPI>(ks) : tf32_slots<128, EPI>(ks);
      if (ks > 1 && tiles > slots) continue;
      const long long kb_per = (kblocks + ks - 1) / ks;
      const long long waves = (tiles + (ks == 1 ? sms : slots) - 1) / (ks == 1 ? sms : slots);
      const long long cost = (128 + 2 * bn) * kb_per * waves;
      if (best_cost < 0 || cost < best_cost) {
        best_cost = cost;
        best_bn = bn;
        best_ks = ks;
      }
    }
  }
  if (best_bn == 64) return launch_tf32<64, EPI>(g, W_lo, p, best_ks, s);
  return launch_tf32<128, EPI>(g, W_lo, p, best_ks, s);
}

yuf_status_t gemm_tf32x3(const GemmArgs& g, const void* W_lo, cudaStream_t s) {
  if (g.M <= 0 || g.N <= 0 || g.batch <= 0) return YUF_OK;
  const bool ok = (reinterpret_cast<uintptr_t>(g.A) & 15) == 0 && g.lda % 4 == 0 &&
                  (reinterpret_cast<uintptr_t>(g.W) & 15) == 0 && (reinterpret_cast<uintptr_t>(W_lo) & 15) == 0 &&
                  g.K % 4 == 0 && g.K > 0;
  if (!ok) {
    set_error("gemm (fp32): operands need 16-byte aligned rows (lda %lld, K %d)", g.lda, g.K);
    return YUF_ERR_INVALID_ARGUMENT;
  }
  if (g.epi != GEMM_EPI_F32 && g.epi != GEMM_EPI_SWIGLU_F32) {
    set_error("gemm (fp32): epilogue %d writes bf16", g.epi);
    return YUF_ERR_INVALID_ARGUMENT;
  }
  GemmParams p{};
  p.C = g.C;
  p.ldc = g.ldc;
  p.c_bstride = g.c_bstride;
  p.M = g.M;
  p.N = g.N;
  p.K = g.K;
  p.batch = g.batch;
  p.a_brows = g.a_brows;
  p.w_brows = g.w_brows;
  p.beta = g.beta;
  p.tanh_batch0 = g.tanh_batch0;
  p.n_out = g.epi == GEMM_EPI_SWIGLU_F32 ? g.n_out : g.N;
  p.m_tiles = (g.M + 127) / 128;
  p.vec = (reinterpret_cast<uintptr_t>(g.C) & 15) == 0 && g.ldc % 4 == 0 && g.c_bstride % 4 == 0;
  if (g.epi == GEMM_EPI_SWIGLU_F32) {
    if (g.N % 128 != 0) {
      set_error("gemm: the SiLU-gate weight must hold whole 128-row groups (N = %d)", g.N);
      return YUF_ERR_INVALID_ARGUMENT;
    }
    return dispatch_tf32<GEMM_EPI_SWIGLU_F32>(g, W_lo, p, s);
  }
  return dispatch_tf32<GEMM_EPI_F32>(g, W_lo, p, s);
}

unsigned int gemm_wait_timeouts() {
  unsigned int n = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&n, g_gemm_wait_timeouts, sizeof(n)) != cudaSuccess ||
      cudaMemcpyToSymbol(g_gemm_wait_timeouts, &zero, sizeof(zero)) != cudaSuccess) {
    cudaGetLastError();
    return ~0u;
  }
  return n;
}

}  // namespace yuf

using namespace yuf;

extern "C" yuf_status_t yuf_gemm_bf16(const void* A, long long lda, long long a_batch_rows, const void* W,
                                      long long w_batch_rows, void* C, long long ldc,
                                      long long c_batch_stride, int M, int N, int K, int batch,
                                      int epilogue, int accumulate, int n_out, void* stream) {
  if (!A || !W || !C || M < 0 || N < 0 || K <= 0 || batch < 0 || lda < K || ldc < 1) {
    set_error("gemm: null operand or bad sizes (M=%d N=%d K=%d batch=%d lda=%lld ldc=%lld)", M, N, K, batch,
              lda, ldc);
    return YUF_ERR_INVALID_ARGUMENT;
  }
  if (epilogue < YUF_GEMM_F32 || epilogue > YUF_GEMM_SILU_GATE) {
    set_error("gemm: unknown epilogue %d", epilogue);
    return YUF_ERR_INVALID_ARGUMENT;
  }
  if (accumulate && epilogue != YUF_GEMM_F32) {
    set_error("gemm: accumulate needs the fp32 epilogue");
    return YUF_ERR_INVALID_ARGUMENT;
  }
  if (epilogue == YUF_GEMM_SILU_GATE && (n_out <= 0 || 2 * (long long)n_out > N)) {
    set_error("gemm: the SiLU-gate epilogue needs 0 < n_out <= N / 2 (n_out=%d N=%d)", n_out, N);
    return YUF_ERR_INVALID_ARGUMENT;
  }
  if (batch > 1 && (a_batch_rows < M || w_batch_rows < N)) {
    set_error("gemm: batches overlap (a_batch_rows %lld < M or w_batch_rows %lld < N)", a_batch_rows,
              w_batch_rows);
    return YUF_ERR_INVALID_ARGUMENT;
  }
  GemmArgs g{};
  g.A = A;
  g.lda = lda;
  g.a_brows = batch > 1 ? a_batch_rows : 0;
  g.a_rows = (long long)(batch > 1 ? batch - 1 : 0) * g.a_brows + M;
  g.W = W;
  g.w_brows = batch > 1 ? w_batch_rows : 0;
  g.w_rows = (long long)(batch > 1 ? batch - 1 : 0) * g.w_brows + N;
  g.C = C;
  g.ldc = ldc;
  g.c_bstride = c_batch_stride;
  g.M = M;
  g.N = N;
  g.K = K;
  g.batch = batch;
  g.epi = epilogue == YUF_GEMM_F32 ? GEMM_EPI_F32
                                   : (epilogue == YUF_GEMM_SILU_GATE ? GEMM_EPI_SWIGLU : GEMM_EPI_BF16);
  g.beta = accumulate ? 1.f : 0.f;
  g.tanh_batch0 = epilogue == YUF_GEMM_BF16_TANH0;
  g.n_out = n_out;
  return gemm_bf16(g, static_cast<cudaStream_t>(stream));
}

extern "C" yuf_status_t yuf_gemm_tf32x3(const float* A, long long lda, long long a_batch_rows, const float* W_hi,
                                        const float* W_lo, long long w_batch_rows, float* C, long long ldc,
                                        long long c_batch_stride, int M, int N, int K, int batch, int epilogue,
                                        int accumulate, int n_out, void* stream) {
  if (!A || !W_hi || !W_lo || !C || M < 0 || N < 0 || K <= 0 || batch < 0 || lda < K || ldc < 1) {
    set_error("gemm (fp32): null operand or bad sizes (M=%d N=%d K=%d batch=%d lda=%lld ldc=%lld)", M, N, K,
              batch, lda, ldc);
    return YUF_ERR_INVALID_ARGUMENT;
  }
  if (epilogue != YUF_GEMM_F32 && epilogue != YUF_GEMM_F32_TANH0 && epilogue != YUF_GEMM_SILU_GATE_F32) {
    set_error("gemm (fp32): epilogue %d has no fp32 form", epilogue);
    return YUF_ERR_INVALID_ARGUMENT;
  }
  if (accumulate && epilogue != YUF_GEMM_F32) {
    set_error("gemm (fp32): accumulate needs the plain fp32 epilogue");
    return YUF_ERR_INVALID_ARGUMENT;
  }
  if (epilogue == YUF_GEMM_SILU_GATE_F32 && (n_out <= 0 || 2 * (long long)n_out > N)) {
    set_error("gemm (fp32): the SiLU-gate epilogue needs 0 < n_out <= N / 2 (n_out=%d N=%d)", n_out, N);
    return YUF_ERR_INVALID_ARGUMENT;
  }
  if (batch > 1 && (a_batch_rows < M || w_batch_rows < N)) {
    set_error("gemm (fp32): batches overlap");
    return YUF_ERR_INVALID_ARGUMENT;
  }
  GemmArgs g{};
  g.A = A;
  g.lda = lda;
  g.a_brows = batch > 1 ? a_batch_rows : 0;
  g.a_rows = (long long)(batch > 1 ? batch - 1 : 0) * g.a_brows + M;
  g.W = W_hi;
  g.w_brows = batch > 1 ? w_batch_rows : 0;
  g.w_rows = (long long)(batch > 1 ? batch - 1 : 0) * g.w_brows + N;
  g.C = C;
  g.ldc = ldc;
  g.c_bstride = c_batch_stride;
  g.M = M;
  g.N = N;
  g.K = K;
  g.batch = batch;
  g.epi = epilogue == YUF_GEMM_SILU_GATE_F32 ? GEMM_EPI_SWIGLU_F32 : GEMM_EPI_F32;
  g.beta = accumulate ? 1.f : 0.f;
  g.tanh_batch0 = epilogue == YUF_GEMM_F32_TANH0;
  g.n_out = n_out;
  return gemm_tf32x3(g, W_lo, static_cast<cudaStream_t>(stream));
}

extern "C" yuf_status_t yuf_tf32_split(const float* w, size_t n, float* hi, float* lo) {
  if ((n > 0) && (!w || !hi || !lo)) {
    set_error("tf32_split: null buffer");
    return YUF_ERR_INVALID_ARGUMENT;
  }
  split_tf32_host(w, n, hi, lo);
  return YUF_OK;
}
