// Head-mixing GEMM of the layered recurrence on the 5th-generation tensor
// cores (tcgen05 + TMEM + TMA), with fp32-level accuracy by operand splitting.
//
// Per layer (gfn/layers/base.py:305-317, the out_proj_x / out_proj_v Linear
// without its bias) the two products
//     z_x = cat_x . W_x^T,   z_v = cat_v . W_v^T      ([B, d] x [d, d] each)
// are computed from fp16 pieces: every activation c = c0 + c1 (written by the
// head-step kernel as rows [c0 | c0 | c1] of width 3d) and every weight,
// scaled by a power of two s per layer, w s = w0 + w1 (packed as rows
// [w0 | w1 | w0]).  The three products of order >= 2^-11,
//     c0 w0 + c0 w1 + c1 w0,
// accumulate in one fp32 TMEM accumulator and the epilogue multiplies by
// 1/s.  The dropped term c1 w1 is below 2^-22 of |c w|.
//
// Structure (one CTA per SM, persistent over output tiles of 128 or 256 rows):
//   warp 0      TMA producer: per K-block of BK (64 or 32) the four operand
//               tiles c0, c1 [128 x BK] and w0, w1 [BN x BK] (2*BK-byte swizzle)
//               into a STAGES-deep shared-memory ring;
//   warp 1      allocates TMEM (two BN-column accumulators) and issues the
//               tcgen05.mma instructions (M=128, N=BN, K=16) from one thread,
//               releasing each ring slot with tcgen05.commit;
//   warps 2..    epilogue (4 per 128 rows): tcgen05.ld of the accumulator (each warp its
//               32-lane quarter of TMEM, one row per thread), scale, fp32
//               stores of z and the row's partial sum of (z + bias)^2 over
//               the tile (the next RMSNorm's statistics, so no separate
//               reduction pass reads z); the second accumulator lets the
//               next tile's MMAs run meanwhile.
// Tiles: (matrix, 128-row block, BN-column block), column blocks fastest so
// that CTAs running together share their activation rows in L2.
#pragma once
#include <cuda.h>

#include "umma.cuh"

namespace gfn {

struct MixUmmaArgs {
  float* z;            // [nmat][B][N] fp32
  float* spart;        // [nmat][ntiles][B] partial sums of (z + bias)^2 over each column tile, or null
  const float* bias;   // [nmat][N] (the layer's bx, bv, contiguous in the pack), or null
  const float* alpha;  // device scalar: 1 / (product of the operands' split scales)
  int B, d, layer;     // rows; d = K = N for the mixing GEMM (see K, N)
  int mtiles, ntiles;  // BM-row blocks of B, BN-column blocks of N
  int K, N;            // reduction and output widths (the mixing GEMM: both d)
  int nmat;            // products in one launch (the mixing GEMM: x and v, 2)
  int out_bias;        // 1: z = alpha (A B^T) + bias; 0: z = alpha (A B^T)
};

// Tile shape: BM = 128 * MH rows (MH halves of 128, one M=128 MMA each, the
// B tile shared), BN columns, K blocks of BK.  TMEM holds two BN-column
// accumulators: double-buffered across tiles when MH == 1, the two row
// halves of one tile when MH == 2 (half the operand bytes per FLOP of B).
template <int BN, int BK_ = 64, int MH_ = 1>
struct MixCfg {
  static constexpr int MH = MH_, BM = 128 * MH, BK = BK_;
  static constexpr int SWZ = BK * 2;  // bytes per tile row = swizzle span
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE = 2 * A_BYTES + 2 * B_BYTES;
  static constexpr int STAGES_FIT = (200 * 1024) / STAGE;
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  static constexpr int TMEM_COLS = 2 * BN;  // power of two for BN in {64, 128, 256}
  static constexpr int NBUF = 2 / MH;       // accumulator buffers (tiles in flight)
  static constexpr int EPI_WARPS = 4 * MH;  // one per (TMEM lane quarter, row half)
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr size_t SMEM = (size_t)STAGES * STAGE + 1024 /* alignment slack */ + 256 /* barriers */;
  static_assert(BN == 64 || BN == 128 || BN == 256, "N tile");
  static_assert(STAGES >= 2, "ring depth");
  static_assert(BK == 32 || BK == 64, "K tile");
  static_assert(MH == 1 || MH == 2, "M tile");
};

template <int BN, int BK, int MH>
__global__ void __launch_bounds__(MixCfg<BN, BK, MH>::THREADS, 1)
    mix_umma_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const MixUmmaArgs a) {
  using C = MixCfg<BN, BK, MH>;
  extern __shared__ __align__(1024) uint8_t mix_smem_raw[];
  // operand tiles need 1024-byte alignment (swizzle atoms)
  const uint32_t raw = smem_u32(mix_smem_raw);
  uint8_t* sm = mix_smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + (size_t)C::STAGES * C::STAGE);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* done = tempty + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], C::EPI_WARPS);  // one arrive per epilogue warp
    }
    mbar_init(done, 1);
    fence_mbar_init();
    umma::prefetch_tmap(&tmA);
    umma::prefetch_tmap(&tmB);
  }
  if (warp == 1) umma::tmem_alloc(tslot, C::TMEM_COLS);
  umma::tc_fence_before();
  __syncthreads();
  umma::tc_fence_after();
  const uint32_t tbase = *tslot;
  // the previous kernel (the head step) wrote the A operand and still reads
  // this GEMM's output buffers until it completes
  umma::gdc_launch_dependents();
  umma::gdc_wait();

  const int ntiles_total = a.nmat * a.mtiles * a.ntiles;
  const int kblocks = a.K / C::BK;
  auto decode = [&](int t, int& which, int& mt, int& nt) {
    nt = t % a.ntiles;
    const int rest = t / a.ntiles;
    mt = rest % a.mtiles;
    which = rest / a.mtiles;
  };

  if (warp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles_total && ok; t += gridDim.x) {
        int which, mt, nt;
        decode(t, which, mt, nt);
        const int arow = which * a.B + mt * C::BM;
        const int brow = which * a.N + nt * BN;
        for (int kb = 0; kb < kblocks && ok; ++kb) {
          ok = umma::mbar_wait_spin(&empty[s], ph ^ 1u);
          if (!ok) break;
          mbar_arrive_expect_tx(&full[s], C::STAGE);
          uint8_t* st = sm + (size_t)s * C::STAGE;
          const int k = kb * C::BK;
          umma::tma_load_2d(st, &tmA, &full[s], k, arow);                           // c0
          umma::tma_load_2d(st + C::A_BYTES, &tmA, &full[s], 2 * a.K + k, arow);     // c1
          umma::tma_load_3d(st + 2 * C::A_BYTES, &tmB, &full[s], k, brow, a.layer);  // w0
          umma::tma_load_3d(st + 2 * C::A_BYTES + C::B_BYTES, &tmB, &full[s], a.K + k, brow,
                            a.layer);                                                // w1
          if (++s == C::STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma::idesc_f16_f32(128, BN);
      constexpr uint32_t AH = 128 * C::SWZ;  // bytes of one 128-row half of an A tile
      int s = 0;
      uint32_t ph = 0;
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles_total && ok; t += gridDim.x, ++it) {
        const int buf = it % C::NBUF;
        const uint32_t use = (uint32_t)(it / C::NBUF);
        ok = umma::mbar_wait_spin(&tempty[buf], (use & 1u) ^ 1u);
        umma::tc_fence_after();
        const uint32_t dt = tbase + (uint32_t)(buf * MH * BN);
        for (int kb = 0; kb < kblocks && ok; ++kb) {
          ok = umma::mbar_wait_spin(&full[s], ph);
          if (!ok) break;
          umma::tc_fence_after();
          const uint32_t st = smem_u32(sm + (size_t)s * C::STAGE);
          const uint32_t a0 = st, a1 = st + C::A_BYTES;
          const uint32_t b0 = st + 2 * C::A_BYTES, b1 = b0 + C::B_BYTES;
#pragma unroll
          for (int kk = 0; kk < C::BK / 16; ++kk) {
            const uint32_t off = (uint32_t)kk * 32u;  // 16 fp16 along K
            const uint64_t db0 = umma::desc_kmajor<C::SWZ>(b0 + off);
            const uint64_t db1 = umma::desc_kmajor<C::SWZ>(b1 + off);
#pragma unroll
            for (int h = 0; h < MH; ++h) {
              const uint32_t dh = dt + (uint32_t)(h * BN);
              const uint64_t da0 = umma::desc_kmajor<C::SWZ>(a0 + h * AH + off);
              const uint64_t da1 = umma::desc_kmajor<C::SWZ>(a1 + h * AH + off);
              umma::mma_f16(dh, da0, db0, idesc, (kb | kk) != 0);
              umma::mma_f16(dh, da0, db1, idesc, 1u);
              umma::mma_f16(dh, da1, db0, idesc, 1u);
            }
          }
          umma::mma_commit(&empty[s]);
          if (++s == C::STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        umma::mma_commit(&tfull[buf]);
      }
      // every MMA issued has completed before the accumulator columns are
      // freed: one more commit, waited for (bounded)
      umma::mma_commit(done);
      umma::mbar_wait_spin(done, 0);
    }
  } else {
    const int q = warp & 3;         // TMEM lane quarter this warp may access
    const int h = (warp - 2) >> 2;  // row half of the tile (MH == 2)
    const int r = h * 128 + 32 * q + lane;
    const float alpha = *a.alpha;
    int it = 0;
    for (int t = blockIdx.x; t < ntiles_total; t += gridDim.x, ++it) {
      int which, mt, nt;
      decode(t, which, mt, nt);
      const int buf = it % C::NBUF;
      const uint32_t use = (uint32_t)(it / C::NBUF);
      // all lanes wait, so the warp leaves together if the wait gives up
      if (!umma::mbar_wait_sleep(&tfull[buf], use & 1u)) break;
      umma::tc_fence_after();
      const int b = mt * C::BM + r;
      float* zr = a.z + ((long long)which * a.B + b) * a.N + nt * BN;
      const float4* bias = a.bias ? reinterpret_cast<const float4*>(a.bias + which * a.N + nt * BN) : nullptr;
      const uint32_t tcol = tbase + ((uint32_t)(32 * q) << 16) + (uint32_t)((buf * MH + h) * BN);
      float ss = 0.f;  // this row's sum of (z + bias)^2 over the tile's columns (RMSNorm)
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        float v[32];
        umma::tmem_ld32(tcol + (uint32_t)(c * 32), v);
        if (b < a.B) {
          float4* dst = reinterpret_cast<float4*>(zr + c * 32);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 o = make_float4(v[4 * j] * alpha, v[4 * j + 1] * alpha, v[4 * j + 2] * alpha,
                                         v[4 * j + 3] * alpha);
            const float4 bb = bias ? __ldg(bias + c * 8 + j) : make_float4(0.f, 0.f, 0.f, 0.f);
            const float e0 = o.x + bb.x, e1 = o.y + bb.y, e2 = o.z + bb.z, e3 = o.w + bb.w;
            ss = fmaf(e0, e0, ss);
            ss = fmaf(e1, e1, ss);
            ss = fmaf(e2, e2, ss);
            ss = fmaf(e3, e3, ss);
            dst[j] = a.out_bias ? make_float4(e0, e1, e2, e3) : o;
          }
        }
      }
      if (b < a.B && a.spart) a.spart[((long long)which * a.ntiles + nt) * a.B + b] = ss;
      umma::tc_fence_before();
      __syncwarp();
      if (lane == 0) umma::mbar_arrive(&tempty[buf]);
    }
  }
  umma::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    umma::tc_fence_after();
    umma::tmem_dealloc(tbase, C::TMEM_COLS);
  }
}

}  // namespace gfn
