// Leapfrog head step of the layered recurrence with the friction gate's
// contraction on the tensor cores (tcgen05, TMEM accumulator).
//
// One CTA computes one layer's head step (gfn/integrators/symplectic/
// leapfrog.py:50-114 with the Christoffel term of gfn/geometry/lowrank.py:
// 93-98,125-127) for 128 batch rows of one head:
//   - thread pair (r, half) owns row r and HD/2 of the head's columns
//     (warp w: TMEM lane quarter w & 3, column half w >> 2); x, v and the
//     force of its columns stay in registers;
//   - the gate x . W_f^T (a 128 x HD x HD product per kick) is computed as
//     c0 w0 + c0 w1 + c1 w0 from fp16 pieces, x = c0 + c1 (written to shared
//     memory as a K-major swizzled UMMA operand by the threads) and
//     W_f s = w0 + w1 (packed per head with a power-of-two scale s, copied
//     in with one bulk copy): three tcgen05.mma (M=128, N=HD, K=16 steps)
//     into a TMEM accumulator, issued by one thread;
//   - while the MMAs run, every thread forms its part of p = v . U; the two
//     halves of a row combine p through shared memory in a fixed order;
//     then Gamma = 20 tanh(((p^2) s) . W^T / 20) and the implicit kick
//     v' = (v + h (F - Gamma)) / (1 + h * 5 sigmoid(gate + b_f)) per column,
//     the gate read from TMEM (tcgen05.ld, one row per thread).
// Input: the carried state (first layer of a token) or the previous layer's
// mixing output with its RMSNorm (row statistics from the mixing GEMM's
// epilogue or the row-statistics kernel) and saturation applied on load.
// Output: the concat (x', v') as split fp16 rows [c0 | c0 | c1] for the
// mixing GEMM.
#pragma once
#include <cuda.h>

#include "layered.cuh"
#include "umma.cuh"

namespace gfn {

template <int HD, int P, int NDUP = 1>
struct HeadUmmaCfg {
  // PARTS threads per row (one warp per TMEM lane quarter and column part).
  // NDUP 1, PARTS 8: 128-row tiles, 1024 threads, the force staged in shared
  //   memory, one CTA per SM; PARTS 4: 512 threads, the force in registers,
  //   two CTAs per SM.
  // NDUP 2 / 4: 64- / 32-row tiles, 8 columns per thread (512 / 256 threads).
  //   The gate's A operand holds the tile's rows NDUP times (MMA rows r,
  //   r + RROWS, ...; M = 128 keeps the one-row-per-TMEM-lane accumulator
  //   layout), and the warps of each group of 4 / NDUP lane quarters read the
  //   next HD / NDUP columns of the same rows: more, shorter tiles at the same
  //   work per thread, no register spills.
  static constexpr int ROWS = 128;                          // MMA rows
  static constexpr int RROWS = 128 / NDUP;                  // batch rows per tile
  static constexpr int WPQ = NDUP == 1 ? P : HD / (8 * NDUP);  // warps per lane quarter
  static constexpr int PARTS = NDUP == 1 ? P : NDUP * WPQ;  // threads (column parts) per row
  static constexpr int THREADS = 128 * WPQ;
  static constexpr int CPT = HD / PARTS;
  static constexpr bool F_SMEM = NDUP == 1 && P == 8;
  static constexpr int MIN_BLOCKS = NDUP == 4 ? 3 : (NDUP == 2 || P != 8) ? 2 : 1;
  static constexpr int ROWB = HD * 2;             // bytes per fp16 operand row
  static constexpr int A_BYTES = ROWS * ROWB;     // one fp16 piece of x (or v)
  static constexpr int VO_BYTES = RROWS * ROWB;   // one fp16 piece of the v' output
  static constexpr int W_BYTES = HD * ROWB;       // one fp16 piece of W_f
  static constexpr int ZBOX = RROWS * 128;        // one [RROWS][32] fp32 box
  // shared memory (bytes):
  //   staging: z boxes [x lo | x hi | v lo | v hi]; then x pieces c0 | c1
  //            (the gate's A operand; x' is also the output) and v' pieces
  //   the token's force, [128][HD] fp32 as two swizzled boxes (F_SMEM only)
  //   W_f pieces w0 | w1; bias / gain of the previous layer [4][HD];
  //   U [HD][RK]; W^T [RK][HD]; b_f [HD]; p parts [PARTS][RROWS][RK]; barriers
  static constexpr int STAGE = (4 * ZBOX > 2 * A_BYTES + 2 * VO_BYTES) ? 4 * ZBOX : 2 * A_BYTES + 2 * VO_BYTES;
  static constexpr int OFF_F = STAGE;
  static constexpr int OFF_W = OFF_F + (F_SMEM ? 2 * ZBOX : 0);
  static constexpr int OFF_F32 = OFF_W + 2 * W_BYTES;
  static_assert(HD == 64, "head dim (one 128-byte swizzle row per operand row)");
  static_assert(CPT % 8 == 0, "whole 16-byte units of fp16 pieces per thread");
  static_assert(NDUP == 1 || NDUP == 2 || NDUP == 4, "row duplication");
};

template <int RK, int HD, int P, int NDUP = 1>
constexpr size_t head_umma_smem() {
  using C = HeadUmmaCfg<HD, P, NDUP>;
  return 1024 /* alignment */ + C::OFF_F32 +
         (size_t)(4 * HD + HD * RK + RK * HD + HD + C::PARTS * C::RROWS * RK) * 4 + 64;
}

// fp16 pieces of 8 consecutive values as two 16-byte units (c0, c1); flags
// |c| >= 2^15 (the split's range).
GFN_DEV void split8(const float* c, uint4& u0, uint4& u1) {
  bool bad = false;
  unsigned h0[4], h1[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float a = c[2 * i], b = c[2 * i + 1];
    bad |= !(fabsf(a) < 32768.f) || !(fabsf(b) < 32768.f);
    // packed pair conversions (one f32x2 -> f16x2 round, one f16x2 -> f32x2
    // widen): the same round-to-nearest pieces as per-value conversions, off
    // the special-function pipe the transcendentals use
    const __half2 p0 = __floats2half2_rn(a, b);
    const float2 r0 = __half22float2(p0);
    const __half2 p1 = __floats2half2_rn(a - r0.x, b - r0.y);
    h0[i] = *reinterpret_cast<const unsigned*>(&p0);
    h1[i] = *reinterpret_cast<const unsigned*>(&p1);
  }
  if (bad) gfn_flag_error(kDevErrF16Range);
  u0 = make_uint4(h0[0], h0[1], h0[2], h0[3]);
  u1 = make_uint4(h1[0], h1[1], h1[2], h1[3]);
}

// 16-byte shared-memory load the compiler may not hoist out of a loop or keep
// across iterations (head weights are re-read where used instead of pinning
// registers for them).
GFN_DEV float4 lds4_fresh(const float* p) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(smem_u32(p)));
  return v;
}

// 16-byte global -> shared copy through L2 (cp.async); src_bytes 0 fills zeros.
GFN_DEV void cp_async16(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(src_bytes)
               : "memory");
}

// TMA tile store shared -> global (3-D map), tracked by the bulk async-group.
GFN_DEV void tma_store_3d(const void* tmap, const void* src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];"
               ::"l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}

// Measurement hook: thread 0 of each CTA stamps the global timer at phase
// boundaries into prof[cta * 8 + slot].
#define GFN_HEAD_STAMP(slot)                                                                    \
  do {                                                                                          \
    if (a.prof && threadIdx.x == 0)                                                             \
      a.prof[(blockIdx.y * gridDim.x + blockIdx.x) * 8 + (slot)] = (long long)umma::global_ns(); \
  } while (0)

// tmz: the previous layer's mixing output z [2B][d] fp32 in [128 x 32] boxes
// (128-byte swizzle; unused for a layer that starts from the carried state).
// tmo: the split output rows catkh viewed as [2][B][3d] fp16 in [1][128][64]
// boxes (128-byte swizzle); rows past B are clipped by the map.
template <int RK, int HD, int P, int NDUP = 1>
__global__ void __launch_bounds__(HeadUmmaCfg<HD, P, NDUP>::THREADS, HeadUmmaCfg<HD, P, NDUP>::MIN_BLOCKS)
    layered_head_umma_kernel(const __grid_constant__ CUtensorMap tmz, const __grid_constant__ CUtensorMap tmo,
                             const LayPreArgs a) {
  using C = HeadUmmaCfg<HD, P, NDUP>;
  static_assert(RK % 4 == 0, "rank");
  constexpr int CPT = C::CPT;
  extern __shared__ __align__(1024) uint8_t hu_smem_raw[];
  const uint32_t raw = smem_u32(hu_smem_raw);
  uint8_t* sm = hu_smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  uint8_t* sZ = sm;                        // z boxes, later the x / v pieces
  uint8_t* sA = sm;                        // x pieces c0 | c1 (K-major, swizzled)
  uint8_t* sVo = sm + 2 * C::A_BYTES;      // v' pieces c0 | c1 (output only)
  uint8_t* sF = sm + C::OFF_F;             // force boxes [lo | hi] (fp32) or [128][64] bf16
  uint8_t* sW = sm + C::OFF_W;             // W_f pieces w0 | w1 (K-major, swizzled)
  float* sBG = reinterpret_cast<float*>(sm + C::OFF_F32);  // previous layer's bx, bv, gx, gv
  float* sU = sBG + 4 * HD;                                // [HD][RK]
  float* sWg = sU + HD * RK;                               // [RK][HD]
  float* sbf = sWg + RK * HD;                              // [HD]
  float* sP = sbf + HD;                                    // [PARTS][RROWS][RK]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + C::PARTS * C::RROWS * RK);  // w, z, mma
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 3);

  const int d = a.d, B = a.B, h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = warp & 3;                      // TMEM lane quarter this warp reads
  // row within the tile (TMEM lane 32 q + lane holds it, or a duplicate) and
  // the column part: each group of 4 / NDUP quarters (one copy of the rows)
  // takes the next HD / NDUP columns
  constexpr int QPD = 4 / NDUP;  // lane quarters per copy of the rows
  const int r = 32 * (q % QPD) + lane;
  const int part = NDUP == 1 ? (warp >> 2) : (q / QPD) * C::WPQ + (warp >> 2);
  const int b0 = blockIdx.x * C::RROWS;
  const int b = b0 + r;                        // batch row
  const bool live = b < B;
  const int c0 = part * CPT;                   // first head column of this thread
  const int gc = h * HD + c0;                  // first model column
  const LayOffsets o = lay_offsets(a.H, HD, RK, d);
  const float* lay = a.lay;
  GFN_HEAD_STAMP(0);

  const bool zin = a.z != nullptr;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 3; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
    // the head's weights (constant: issued before waiting on the previous kernel)
    constexpr int UWB = (2 * HD * RK + HD) * 4;  // U | W^T | b_f bytes
    mbar_arrive_expect_tx(&bars[0], 2 * C::W_BYTES + UWB + (zin ? 4 * HD * 4 : 0));
    bulk_g2s(sW, lay + o.HU + (long long)h * (HD * HD), 2 * C::W_BYTES, &bars[0]);
    bulk_g2s(sU, lay + (long long)h * o.hblock + HD * HD, UWB, &bars[0]);
    if (zin) {
      const int offs[4] = {o.bx, o.bv, o.gx, o.gv};
#pragma unroll
      for (int i = 0; i < 4; ++i) bulk_g2s(sBG + i * HD, a.prev + offs[i] + h * HD, HD * 4, &bars[0]);
    }
  }
  // the token's force for this thread's columns, fetched now (it is used in
  // both kicks): fp32 into two swizzled [128][32] boxes, bf16 into one
  // swizzled [128][64] tile
  const bool fbf = a.fbf16 != nullptr;
  float fm = 0.f;
  float F[CPT];
  {
    const void* src = nullptr;
    if (live) {
      const long long idx = (long long)b * a.L + a.t;
      fm = a.mask ? a.mask[idx] : 1.f;
      if (a.f32) {
        src = a.f32 + idx * d + gc;
      } else if (fbf) {
        src = a.fbf16 + idx * d + gc;
      } else {
        const long long id = a.ids[idx];
        if (id < 0 || id >= a.vocab) {
          if (part == 0) gfn_flag_error(kDevErrBadToken);
        } else {
          src = a.table + id * d + gc;
        }
      }
    }
    if constexpr (C::F_SMEM) {
      const uint32_t nb = src ? 16u : 0u;
      const void* s0 = src ? src : static_cast<const void*>(lay);  // any valid address when zero-filling
      if (fbf) {
        cp_async16(sF + r * 128 + (((c0 >> 3) ^ (r & 7)) << 4), s0, nb);
      } else {
        uint8_t* fb = sF + (c0 >> 5) * C::ZBOX + r * 128;
#pragma unroll
        for (int u = 0; u < 2; ++u)
          cp_async16(fb + (((((c0 & 31) >> 2) + u) ^ (r & 7)) << 4),
                     static_cast<const float*>(s0) + (src ? 4 * u : 0), nb);
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
    } else {
#pragma unroll
      for (int j = 0; j < CPT; ++j) F[j] = 0.f;
      if (src && fbf) {
#pragma unroll
        for (int u = 0; u < CPT / 8; ++u) {
          const uint4 w4 = __ldg(reinterpret_cast<const uint4*>(src) + u);
          const unsigned w[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            F[8 * u + 2 * i] = __uint_as_float(w[i] << 16);
            F[8 * u + 2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
          }
        }
      } else if (src) {
#pragma unroll
        for (int j = 0; j < CPT; j += 4) {
          const float4 f = ldg4(static_cast<const float*>(src) + j);
          F[j] = f.x; F[j + 1] = f.y; F[j + 2] = f.z; F[j + 3] = f.w;
        }
      }
    }
  }
  if (warp == 0) umma::tmem_alloc(tslot, 2 * HD);
  __syncthreads();  // barriers initialised before any thread waits on them
  // the previous kernel (the mixing GEMM or the finalize) wrote z / the state
  // and still reads this kernel's output buffer until it completes
  umma::gdc_launch_dependents();
  umma::gdc_wait();
  if (threadIdx.x == 0 && zin) {
    mbar_arrive_expect_tx(&bars[1], 4 * C::ZBOX);
#pragma unroll
    for (int i = 0; i < 4; ++i)  // (x, v) x (column half)
      umma::tma_load_2d(sZ + i * C::ZBOX, &tmz, &bars[1], h * HD + (i & 1) * 32, (i >> 1) * B + b0);
  }
  // RMSNorm factors of this row from the mixing GEMM's partial sums (issued
  // first: their latency overlaps the copies below)
  float rx = 0.f, rv = 0.f;
  if (a.z && live) {
    if (a.spart) {
      float sx = 0.f, sv = 0.f;
      for (int p = 0; p < a.nparts; ++p) {
        sx += a.spart[(long long)p * B + b];
        sv += a.spart[((long long)a.nparts + p) * B + b];
      }
      rx = 1.f / sqrtf(sx * (1.f / (float)d) + 1.1920928955078125e-07f);
      rv = 1.f / sqrtf(sv * (1.f / (float)d) + 1.1920928955078125e-07f);
    } else {
      rx = a.stat[b];
      rv = a.stat[B + b];
    }
  }

  const float eff = a.base_dt * lay[o.sc + h];
  const float hh = 0.5f * eff;
  const float inv_s = lay[o.HUs + 2 * h + 1];

  // ---- x, v: the previous layer's RMSNorm + saturation applied to the staged
  // z rows, or the carried state
  float X[CPT], V[CPT];
#pragma unroll
  for (int j = 0; j < CPT; ++j) X[j] = V[j] = 0.f;
  bool ok = true;
  if (a.z) {
    GFN_HEAD_STAMP(1);
    ok = umma::mbar_wait_sleep(&bars[1], 0);
    GFN_HEAD_STAMP(2);
    const uint8_t* zxb = sZ + (c0 >> 5) * C::ZBOX + r * 128;
    const uint8_t* zvb = sZ + (2 + (c0 >> 5)) * C::ZBOX + r * 128;
#pragma unroll
    for (int u = 0; u < CPT / 4; ++u) {
      const int so = ((((c0 & 31) >> 2) + u) ^ (r & 7)) << 4;
      const float4 ux = *reinterpret_cast<const float4*>(zxb + so);
      const float4 uv = *reinterpret_cast<const float4*>(zvb + so);
      const int j = 4 * u;
      const float4 bx = *reinterpret_cast<const float4*>(sBG + c0 + j);
      const float4 bv = *reinterpret_cast<const float4*>(sBG + HD + c0 + j);
      const float4 gx = *reinterpret_cast<const float4*>(sBG + 2 * HD + c0 + j);
      const float4 gv = *reinterpret_cast<const float4*>(sBG + 3 * HD + c0 + j);
      X[j + 0] = ((ux.x + bx.x) * rx) * gx.x;
      X[j + 1] = ((ux.y + bx.y) * rx) * gx.y;
      X[j + 2] = ((ux.z + bx.z) * rx) * gx.z;
      X[j + 3] = ((ux.w + bx.w) * rx) * gx.w;
      V[j + 0] = saturate100(((uv.x + bv.x) * rv) * gv.x);
      V[j + 1] = saturate100(((uv.y + bv.y) * rv) * gv.y);
      V[j + 2] = saturate100(((uv.z + bv.z) * rv) * gv.z);
      V[j + 3] = saturate100(((uv.w + bv.w) * rv) * gv.w);
    }
  } else if (live) {
    const float* xr = a.x_in + (long long)b * a.in_stride + gc;
    const float* vr = a.v_in + (long long)b * a.in_stride + gc;
#pragma unroll
    for (int j = 0; j < CPT; j += 4) {
      const float4 x4 = ldg4(xr + j), v4 = ldg4(vr + j);
      X[j] = x4.x; X[j + 1] = x4.y; X[j + 2] = x4.z; X[j + 3] = x4.w;
      V[j] = v4.x; V[j + 1] = v4.y; V[j + 2] = v4.z; V[j + 3] = v4.w;
    }
  }
  if (!live) {
#pragma unroll
    for (int j = 0; j < CPT; ++j) X[j] = V[j] = 0.f;
  }
  if constexpr (C::F_SMEM) {
    asm volatile("cp.async.wait_all;" ::: "memory");  // this thread's force copies landed
    if (fbf) {
      const uint4 u = *reinterpret_cast<const uint4*>(sF + r * 128 + (((c0 >> 3) ^ (r & 7)) << 4));
      const unsigned w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        F[2 * i] = __uint_as_float(w[i] << 16);
        F[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
      }
    } else {
      const uint8_t* fb = sF + (c0 >> 5) * C::ZBOX + r * 128;
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const float4 f = *reinterpret_cast<const float4*>(fb + (((((c0 & 31) >> 2) + u) ^ (r & 7)) << 4));
        F[4 * u] = f.x; F[4 * u + 1] = f.y; F[4 * u + 2] = f.z; F[4 * u + 3] = f.w;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < CPT; ++j) F[j] *= fm;
  if (ok) ok = umma::mbar_wait_sleep(&bars[0], 0);  // W_f pieces, U, W^T, b_f landed
  __syncthreads();  // z boxes consumed (the pieces overwrite them)
  umma::tc_fence_after();
  const uint32_t tbase = *tslot;
  const uint32_t idesc = umma::idesc_f16_f32(128, HD);


  // ---- kick 1 at x (then the drift), kick 2 at x' (one copy of the code)
#pragma unroll 1
  for (int kick = 0; kick < 2; ++kick) {
    const uint32_t tacc = tbase + (uint32_t)(kick * HD);
#pragma unroll
    for (int u8 = 0; u8 < CPT / 8; ++u8) {  // A operand: fp16 pieces of x for the gate product
      uint4 p0, p1;
      split8(X + 8 * u8, p0, p1);
      const int aoff = umma_kmajor_off(r, c0 + 8 * u8, C::ROWB);
      *reinterpret_cast<uint4*>(sA + aoff) = p0;
      *reinterpret_cast<uint4*>(sA + C::A_BYTES + aoff) = p1;
#pragma unroll
      for (int k = 1; k < NDUP; ++k) {  // the duplicate MMA rows r + k RROWS
        const int doff = umma_kmajor_off(r + k * C::RROWS, c0 + 8 * u8, C::ROWB);
        *reinterpret_cast<uint4*>(sA + doff) = p0;
        *reinterpret_cast<uint4*>(sA + C::A_BYTES + doff) = p1;
      }
    }
    // generic-proxy writes -> visible to the tensor core's async proxy
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    {  // partial p = v . U over this thread's columns, published for the row
      float pp[RK];
#pragma unroll
      for (int k = 0; k < RK; ++k) pp[k] = 0.f;
#pragma unroll
      for (int j = 0; j < CPT; ++j)
#pragma unroll
        for (int k = 0; k < RK; k += 4) {
          const float4 u = lds4_fresh(sU + (c0 + j) * RK + k);
          pp[k] = fmaf(V[j], u.x, pp[k]);
          pp[k + 1] = fmaf(V[j], u.y, pp[k + 1]);
          pp[k + 2] = fmaf(V[j], u.z, pp[k + 2]);
          pp[k + 3] = fmaf(V[j], u.w, pp[k + 3]);
        }
      float* dst = sP + (part * C::RROWS + r) * RK;
#pragma unroll
      for (int k = 0; k < RK; k += 4)
        *reinterpret_cast<float4*>(dst + k) = make_float4(pp[k], pp[k + 1], pp[k + 2], pp[k + 3]);
    }
    umma::tc_fence_before();
    __syncthreads();
    umma::tc_fence_after();
    GFN_HEAD_STAMP(3 + 2 * kick);
    if (threadIdx.x == 0) {
      const uint32_t a0 = smem_u32(sA), a1 = a0 + C::A_BYTES;
      const uint32_t w0 = smem_u32(sW), w1 = w0 + C::W_BYTES;
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) {
        const uint32_t off = (uint32_t)kk * 32u;
        const uint64_t da0 = umma::desc_kmajor<C::ROWB>(a0 + off), da1 = umma::desc_kmajor<C::ROWB>(a1 + off);
        const uint64_t db0 = umma::desc_kmajor<C::ROWB>(w0 + off), db1 = umma::desc_kmajor<C::ROWB>(w1 + off);
        umma::mma_f16(tacc, da0, db0, idesc, kk != 0);
        umma::mma_f16(tacc, da0, db1, idesc, 1u);
        umma::mma_f16(tacc, da1, db0, idesc, 1u);
      }
      umma::mma_commit(&bars[2]);
    }
    // Gamma's row factor from the parts of p (fixed order)
    float p[RK];
#pragma unroll
    for (int k = 0; k < RK; ++k) p[k] = 0.f;
#pragma unroll
    for (int pt = 0; pt < C::PARTS; ++pt)
#pragma unroll
      for (int k = 0; k < RK; k += 4) {
        const float4 pk = *reinterpret_cast<const float4*>(sP + (pt * C::RROWS + r) * RK + k);
        p[k] += pk.x; p[k + 1] += pk.y; p[k + 2] += pk.z; p[k + 3] += pk.w;
      }
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < RK; ++k) ss = fmaf(p[k], p[k], ss);
    const float sc = 1.f / ((1.f + sqrtf(ss)) + 1e-6f);
#pragma unroll
    for (int k = 0; k < RK; ++k) p[k] = (p[k] * p[k]) * sc;
    if (ok) ok = umma::mbar_wait_sleep(&bars[2], (uint32_t)kick);
    umma::tc_fence_after();
    GFN_HEAD_STAMP(4 + 2 * kick);
    float g[CPT];
    umma::tmem_ld<CPT>(tacc + ((uint32_t)(32 * q) << 16) + (uint32_t)c0, g);  // CPT = 8 or 16
#pragma unroll
    for (int j4 = 0; j4 < CPT; j4 += 4) {
      float gm[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int k = 0; k < RK; ++k) {
        const float4 w = lds4_fresh(sWg + k * HD + c0 + j4);
        gm[0] = fmaf(p[k], w.x, gm[0]);
        gm[1] = fmaf(p[k], w.y, gm[1]);
        gm[2] = fmaf(p[k], w.z, gm[2]);
        gm[3] = fmaf(p[k], w.w, gm[3]);
      }
      const float4 bf4 = lds4_fresh(sbf + c0 + j4);
      const float bj[4] = {bf4.x, bf4.y, bf4.z, bf4.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int j = j4 + i;
        // Gamma = 20 tanh(y) = 20 (et - 1) / (et + 1), et = exp(2y), y = gm / 20
        // clamped to +-9 (tanh(9) rounds to 1 in float32);
        // v' = (v + h (F - Gamma)) / (1 + h * 5 sigmoid(gate))
        //    = num * ope / (ope + 5h), ope = 1 + exp(-gate), the exponent
        // clamped to 60 (sigmoid < 1e-26: no friction in float32).  Both
        // quotients share one reciprocal of dt * df (both >= 1, product < 1e35).
        const float et = __expf(fminf(fmaxf(gm[i] * 0.1f, -18.f), 18.f));
        const float ope = 1.f + __expf(fminf(-(g[j] * inv_s + bj[i]), 60.f));
        const float dt = et + 1.f, df = ope + 5.f * hh;
        const float rr = __fdividef(1.f, dt * df);
        const float gam = 20.f * (et - 1.f) * (df * rr);
        const float num = V[j] + hh * (F[j] - gam);
        V[j] = num * ope * (dt * rr);
      }
    }
    if (kick == 0) {
#pragma unroll
      for (int j = 0; j < CPT; ++j) X[j] = X[j] + eff * V[j];  // drift
    }
    umma::tc_fence_before();
    __syncthreads();  // p and the A pieces are rewritten next
  }

  // ---- output: x' pieces are the last gate operand (still in sA); v' pieces
  // next to them; TMA stores write [c0 | c0 | c1] of x' and v'
#pragma unroll
  for (int u8 = 0; u8 < CPT / 8; ++u8) {
    uint4 p0, p1;
    split8(V + 8 * u8, p0, p1);
    const int aoff = umma_kmajor_off(r, c0 + 8 * u8, C::ROWB);
    *reinterpret_cast<uint4*>(sVo + aoff) = p0;
    *reinterpret_cast<uint4*>(sVo + C::VO_BYTES + aoff) = p1;
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncthreads();
  if (threadIdx.x == 0) {
    const int col = h * HD;
#pragma unroll
    for (int w = 0; w < 2; ++w) {
      const uint8_t* pc = w == 0 ? sA : sVo;
      const int c1off = w == 0 ? C::A_BYTES : C::VO_BYTES;
      tma_store_3d(&tmo, pc, col, b0, w);                        // c0
      tma_store_3d(&tmo, pc, d + col, b0, w);                    // c0
      tma_store_3d(&tmo, pc + c1off, 2 * d + col, b0, w);        // c1
    }
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // smem read before exit
  }
  if (warp == 0) {
    umma::tc_fence_after();
    umma::tmem_dealloc(tbase, 2 * HD);
  }
  GFN_HEAD_STAMP(7);
}

}  // namespace gfn
