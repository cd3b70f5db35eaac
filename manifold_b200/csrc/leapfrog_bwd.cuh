// BPTT backward of the fused leapfrog recurrence (reverse replay).
//
// The reference trains this path with torch autograd through its per-token
// Python loop (gfn/model.py:377-402; its CUDA backwards are incomplete, see
// gfn/cuda/src/integrators/leapfrog_backward.cu:61-85).  Here one persistent
// launch walks the tokens and layers in reverse.  The forward stored every
// layer step's input state (x, v); each reverse step recomputes that step
// (head step, mixing, RMSNorm) from it and back-propagates:
//   saturation / RMSNorm  -> dz (mixing pre-activations, this CTA's columns)
//   mixing                -> dx_cat = Wx^T dz (streamed transposed weights)
//   head step (leapfrog)  -> dx_in, dv_in, dF and the per-step gradient
//                            signals of U, W, Wf, bf, dt_params
// The cluster decomposition is the forward's (K CTAs x R rows, (row, head)
// units in registers).  Four exchanges per step, each completing on the
// receiver's mbarrier: the concat (x', v'), the RMSNorm sums of squares, the
// RMSNorm backward dot products and the concat of dz.
//
// Parameter gradients are sums over (token, row) of outer products; the
// kernel writes the per-step factors ("signals") and the host reduces them
// with GEMMs / column sums, so the result is deterministic.
//
// Head-step gradient (per element j of a head; h = dt_eff / 2):
//   v' = N2/D2, N2 = vh + h (F - G2), D2 = 1 + h mu2:  dN2 = dv'/D2, dD2 = -dv' v'/D2
//   mu = 5 sigmoid(z): dz = dmu mu (1 - mu/5);  z = x Wf^T + bf: dx += Wf^T dz
//   G = 20 tanh(g/20): dg = dG (1 - (G/20)^2);  g = q W^T, q = p^2 s, p = vU,
//   s = 1/(1 + |p| + 1e-6): dp = 2 p s (W^T dg) - s^2 (sum_r p_r^2 dq_r) p/|p|
//   x' = x + dt_eff vh, vh = N1/D1 likewise; d dt_eff collects x' and h terms.
#pragma once
#include "leapfrog_seq.cuh"

namespace gfn {

constexpr int BWD_NW = 8;
constexpr int BWD_CT = BWD_NW * 32;
constexpr int BWD_THREADS = BWD_CT + 32;
constexpr int BWD_MAXU = 3;
constexpr int BWD_NSIG = 11;  // [NL][L][B][d] signal tensors
constexpr int BWD_NSMALL = 4; // [NL][L][B][H][r] signal tensors
// signal order in the workspace
enum { SIG_X2, SIG_V2, SIG_DZX, SIG_DZV, SIG_SGX, SIG_SGV, SIG_DZ1, SIG_DZ2, SIG_VH, SIG_DG1, SIG_DG2 };
enum { SML_Q1, SML_Q2, SML_DP1, SML_DP2 };

struct BwdArgs {
  const float* f32;
  const __nv_bfloat16* fbf16;
  const long long* ids;
  const float* table;
  long long vocab;
  const float* mask;
  const float* pack;    // training layout
  const float* traj;    // [2][NL][L][B][d]: layer-step inputs x then v
  const float* gx_seq;  // [B][L][d] or null
  const float* gv_seq;
  const float* gx_fin;  // [B][d] or null
  const float* gv_fin;
  float* dx0;           // [B][d]
  float* dv0;
  float* dforces;       // [B][L][d] or null
  float* ws;            // signals: NSIG x [NL][L][B][d], NSMALL x [NL][L][B][H][r], [NL][L][B][H]
  int B, L, d, H, hd, NL;
  int K, R, C, hpc, KC, nchunk, NST;
  int HS, HST, CF;
  long long LF;
  int mix;
  int TR, NG, tiles, S, logC;
  float base_dt;
  int o_head, o_chunk, o_ox, o_ov, o_catx, o_catv, o_dcx, o_dcv, o_part, o_part2, o_px, o_pv;
};

// Force element (the forward's source, any of the three kinds).
GFN_DEV float bwd_force(const BwdArgs& a, int t, int b, int col) {
  const long long idx = (long long)b * a.L + t;
  float f;
  if (a.f32) f = __ldg(a.f32 + idx * a.d + col);
  else if (a.fbf16) f = __bfloat162float(a.fbf16[idx * a.d + col]);
  else {
    const long long id = __ldg(a.ids + idx);
    f = (id < 0 || id >= a.vocab) ? 0.f : __ldg(a.table + id * a.d + col);
  }
  if (a.mask) f = f * __ldg(a.mask + idx);
  return f;
}

// Projection p = vU (warp all-reduced), s and q of one unit's Gamma.
template <int RK, int EPL>
GFN_DEV void bwd_proj(const float (&vv)[EPL], const float* __restrict__ U, const bool (&ok)[EPL],
                      const int (&jj)[EPL], float (&p)[RK], float& n, float& s) {
#pragma unroll
  for (int q = 0; q < RK; ++q) p[q] = 0.f;
#pragma unroll
  for (int e = 0; e < EPL; ++e)
    if (ok[e])
#pragma unroll
      for (int q = 0; q < RK; ++q) p[q] = fmaf(vv[e], U[jj[e] * RK + q], p[q]);
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1)
#pragma unroll
    for (int q = 0; q < RK; ++q) p[q] += __shfl_xor_sync(0xffffffffu, p[q], m);
  float ss = 0.f;
#pragma unroll
  for (int q = 0; q < RK; ++q) ss = fmaf(p[q], p[q], ss);
  n = sqrtf(ss);
  s = 1.f / ((1.f + n) + 1e-6f);
}

template <int RK, int EPL>
GFN_DEV void bwd_gamma(const float (&p)[RK], float s, const float* __restrict__ W,
                       const bool (&ok)[EPL], const int (&jj)[EPL], float (&G)[EPL]) {
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    float g = 0.f;
    if (ok[e])
#pragma unroll
      for (int q = 0; q < RK; ++q) g = fmaf((p[q] * p[q]) * s, W[jj[e] * RK + q], g);
    G[e] = soft_clamp20(g);
  }
}

// z = x Wf^T + bf with x broadcast by shuffles; WfT is [k][j].
template <int EPL, int HDC>
GFN_DEV void bwd_friction_pre_impl(const float (&xx)[EPL], const float* __restrict__ WfT,
                              const float* __restrict__ bf, int hd_rt, const int (&jj)[EPL],
                              float (&z)[EPL]) {
  const int hd = HDC ? HDC : hd_rt;
  float z0[EPL], z1[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) z0[e] = z1[e] = 0.f;
#pragma unroll
  for (int e2 = 0; e2 < EPL; ++e2)
#pragma unroll
    for (int kk = 0; kk < 32; kk += 2) {
      const int k = e2 * 32 + kk;
      if (k < hd) {
        const float xa = __shfl_sync(0xffffffffu, xx[e2], kk);
        const float xb = __shfl_sync(0xffffffffu, xx[e2], kk + 1);
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
          z0[e] = fmaf(xa, WfT[k * hd + jj[e]], z0[e]);
          z1[e] = fmaf(xb, WfT[(k + 1) * hd + jj[e]], z1[e]);
        }
      }
    }
#pragma unroll
  for (int e = 0; e < EPL; ++e) z[e] = (z0[e] + z1[e]) + bf[jj[e]];
}

template <int EPL>
GFN_DEV void bwd_friction_pre(const float (&xx)[EPL], const float* __restrict__ WfT,
                              const float* __restrict__ bf, int hd, const int (&jj)[EPL],
                              float (&z)[EPL]) {
  // compile-time head_dim when it fills the lanes (no per-k bounds checks)
  if (hd == 32 * EPL)
    bwd_friction_pre_impl<EPL, 32 * EPL>(xx, WfT, bf, hd, jj, z);
  else
    bwd_friction_pre_impl<EPL, 0>(xx, WfT, bf, hd, jj, z);
}

// out_k = sum_j dz_j Wf[j][k] (Wf untransposed [j][k]) for the lane's k.
template <int EPL, int HDC>
GFN_DEV void bwd_friction_t_impl(const float (&dz)[EPL], const float* __restrict__ Wf, int hd_rt,
                            const int (&jj)[EPL], float (&out)[EPL]) {
  const int hd = HDC ? HDC : hd_rt;
  float o0[EPL], o1[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) o0[e] = o1[e] = 0.f;
#pragma unroll
  for (int e2 = 0; e2 < EPL; ++e2)
#pragma unroll
    for (int jl = 0; jl < 32; jl += 2) {
      const int j = e2 * 32 + jl;
      if (j < hd) {
        const float da = __shfl_sync(0xffffffffu, dz[e2], jl);
        const float db = __shfl_sync(0xffffffffu, dz[e2], jl + 1);
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
          o0[e] = fmaf(da, Wf[j * hd + jj[e]], o0[e]);
          o1[e] = fmaf(db, Wf[(j + 1) * hd + jj[e]], o1[e]);
        }
      }
    }
#pragma unroll
  for (int e = 0; e < EPL; ++e) out[e] = o0[e] + o1[e];
}

template <int EPL>
GFN_DEV void bwd_friction_t(const float (&dz)[EPL], const float* __restrict__ Wf, int hd,
                            const int (&jj)[EPL], float (&out)[EPL]) {
  // compile-time head_dim when it fills the lanes (no per-k bounds checks)
  if (hd == 32 * EPL)
    bwd_friction_t_impl<EPL, 32 * EPL>(dz, Wf, hd, jj, out);
  else
    bwd_friction_t_impl<EPL, 0>(dz, Wf, hd, jj, out);
}

// Backward of G = Gamma(v) given dG: returns dv (added to dv), writes the
// dg signal (per element) and q, dp (per unit, r values).
template <int RK, int EPL>
GFN_DEV void bwd_gamma_back(const float (&dG)[EPL], const float (&G)[EPL], const float (&p)[RK],
                            float n, float s, const float* __restrict__ U,
                            const float* __restrict__ W, const bool (&ok)[EPL],
                            const int (&jj)[EPL], float (&dv)[EPL], float (&dg)[EPL],
                            float (&q_out)[RK], float (&dp)[RK]) {
  float dq[RK];
#pragma unroll
  for (int q = 0; q < RK; ++q) dq[q] = 0.f;
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    const float t = G[e] / 20.f;
    dg[e] = ok[e] ? dG[e] * (1.f - t * t) : 0.f;
    if (ok[e])
#pragma unroll
      for (int q = 0; q < RK; ++q) dq[q] = fmaf(dg[e], W[jj[e] * RK + q], dq[q]);
  }
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1)
#pragma unroll
    for (int q = 0; q < RK; ++q) dq[q] += __shfl_xor_sync(0xffffffffu, dq[q], m);
  float ds = 0.f;
#pragma unroll
  for (int q = 0; q < RK; ++q) {
    q_out[q] = (p[q] * p[q]) * s;
    ds = fmaf(dq[q], p[q] * p[q], ds);
  }
  const float dn = -ds * s * s;
  const float inv_n = n > 0.f ? 1.f / n : 0.f;
#pragma unroll
  for (int q = 0; q < RK; ++q) dp[q] = dq[q] * 2.f * p[q] * s + dn * p[q] * inv_n;
#pragma unroll
  for (int e = 0; e < EPL; ++e)
    if (ok[e])
#pragma unroll
      for (int q = 0; q < RK; ++q) dv[e] = fmaf(dp[q], U[jj[e] * RK + q], dv[e]);
}

// Mixing GEMV over the chunk ring: out[row][n] = sum_k cat[row][k] chunk[k][n]
// for this CTA's 2C columns (x block then v block), plus bias if given.
template <int CT>
GFN_DEV void bwd_mix(const BwdArgs& a, const float* catx, const float* catv, float* ox, float* ov,
                     const float* bx, const float* bv, float* chunk_ring, uint64_t* chunk_full,
                     uint64_t* chunk_empty, int& cslot, uint32_t& cphase, int tid, int lane) {
  const int C = a.C, R = a.R, S = a.S, CS = chunk_row_stride(C), swz = chunk_swizzle_mask(C);
  const bool active = tid < a.tiles * S;
  const int ms = tid % S, mtile = tid / S;
  const int mng = mtile % a.NG, mrg = mtile / a.NG;
  const int mn0 = mng * 4, mr0 = mrg * a.TR;
  const float* mcat = (mn0 < C) ? catx : catv;
  float acc[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i] = 0.f;
  for (int i = 0; i < a.nchunk; ++i) {
    const int slot = cslot;
    mbar_wait(&chunk_full[slot], cphase);
    if (++cslot == a.NST) {
      cslot = 0;
      cphase ^= 1u;
    }
    const float* wc = chunk_ring + (long long)slot * a.CF;
    if (active) {
      const int k0 = i * a.KC;
      for (int kk = 4 * ms; kk < a.KC; kk += 4 * S) {
        const int kg = k0 + kk;
        const float* cblk = a.logC >= 0 ? mcat + ((kg >> a.logC) * R) * C + (kg & (C - 1))
                                        : mcat + ((kg / C) * R) * C + (kg % C);
        const float* wq = wc + kk * CS + ((((mn0 >> 2) ^ ((kk >> 2) & swz))) << 2);
        const float4 w0 = *reinterpret_cast<const float4*>(wq);
        const float4 w1 = *reinterpret_cast<const float4*>(wq + CS);
        const float4 w2 = *reinterpret_cast<const float4*>(wq + 2 * CS);
        const float4 w3 = *reinterpret_cast<const float4*>(wq + 3 * CS);
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) {
          if (rr < a.TR && mr0 + rr < R) {
            const float4 c4 = *reinterpret_cast<const float4*>(cblk + (mr0 + rr) * C);
            float* ac = acc + rr * 4;
            ac[0] = fmaf(c4.x, w0.x, ac[0]); ac[1] = fmaf(c4.x, w0.y, ac[1]);
            ac[2] = fmaf(c4.x, w0.z, ac[2]); ac[3] = fmaf(c4.x, w0.w, ac[3]);
            ac[0] = fmaf(c4.y, w1.x, ac[0]); ac[1] = fmaf(c4.y, w1.y, ac[1]);
            ac[2] = fmaf(c4.y, w1.z, ac[2]); ac[3] = fmaf(c4.y, w1.w, ac[3]);
            ac[0] = fmaf(c4.z, w2.x, ac[0]); ac[1] = fmaf(c4.z, w2.y, ac[1]);
            ac[2] = fmaf(c4.z, w2.z, ac[2]); ac[3] = fmaf(c4.z, w2.w, ac[3]);
            ac[0] = fmaf(c4.w, w3.x, ac[0]); ac[1] = fmaf(c4.w, w3.y, ac[1]);
            ac[2] = fmaf(c4.w, w3.z, ac[2]); ac[3] = fmaf(c4.w, w3.w, ac[3]);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&chunk_empty[slot]);
  }
  if (active) {
    int base, cnt;
    reduce_scatter16(acc, S, lane, base, cnt);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      if (i < cnt) {
        const int e = base + i;
        const int rr = e >> 2, c = e & 3;
        const int n = mn0 + c, row = mr0 + rr;
        if (rr < a.TR && row < R) {
          if (n < C) ox[row * C + n] = acc[i] + (bx ? bx[n] : 0.f);
          else ov[row * C + n - C] = acc[i] + (bv ? bv[n - C] : 0.f);
        }
      }
    }
  }
}

template <int RK, int EPL>
__global__ void __launch_bounds__(BWD_THREADS, 1) leapfrog_bwd_kernel(const BwdArgs a) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw);
  uint64_t* head_full = bars;        // [2]
  uint64_t* head_empty = bars + 2;   // [2]
  uint64_t* xch_bar = bars + 4;      // E1: concat of (x', v')
  uint64_t* part_bar = bars + 5;     // E2: sums of squares
  uint64_t* part2_bar = bars + 6;    // E3: RMSNorm backward dot products
  uint64_t* dxch_bar = bars + 7;     // E4: concat of dz
  uint64_t* chunk_full = bars + 8;
  uint64_t* chunk_empty = bars + 8 + a.NST;
  float* sm = reinterpret_cast<float*>(smem_raw + SEQ_BAR_BYTES);
  float* head_ring = sm + a.o_head;
  float* chunk_ring = sm + a.o_chunk;
  float* ox = sm + a.o_ox;
  float* ov = sm + a.o_ov;
  float* catx = sm + a.o_catx;
  float* catv = sm + a.o_catv;
  float* dcx = sm + a.o_dcx;
  float* dcv = sm + a.o_dcv;
  float* part = sm + a.o_part;
  float* part2 = sm + a.o_part2;
  float* px = sm + a.o_px;
  float* pv = sm + a.o_pv;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t crank = cluster_ctarank();
  const int row0 = (blockIdx.x / a.K) * a.R;
  const int C = a.C, R = a.R, d = a.d, hd = a.hd, hpc = a.hpc, K = a.K, B = a.B, L = a.L;
  const int H = a.H, NL = a.NL;
  const int col0 = (int)crank * C;
  const HeadOffsets ho = head_offsets(hpc, hd, RK, C);
  const long long total_steps = (long long)L * NL;
  const float* my_pack = a.pack + (long long)crank * a.LF;
  const long long layer_stride = (long long)K * a.LF;
  const uint32_t blk_bytes = (uint32_t)(R * C * 4);
  const uint32_t xch_bytes = 2u * (uint32_t)(K - 1) * blk_bytes;
  const uint32_t part_bytes = (uint32_t)(K * R * 2 * 4);
  const long long BD = (long long)B * d;
  const long long sig_stride = (long long)NL * L * BD;
  const long long sml_stride = (long long)NL * L * B * H * RK;

  if (tid == 0) {
    for (int i = 0; i < 8 + 2 * a.NST; ++i) {
      const bool is_empty = (i >= 2 && i < 4) || (i >= 8 + a.NST);
      mbar_init(&bars[i], is_empty ? BWD_NW : 1);
    }
    fence_mbar_init();
    if (a.mix) {
      if (K > 1) {
        mbar_arrive_expect_tx(xch_bar, xch_bytes);
        mbar_arrive_expect_tx(dxch_bar, xch_bytes);
      }
      mbar_arrive_expect_tx(part_bar, part_bytes);
      mbar_arrive_expect_tx(part2_bar, part_bytes);
    }
  }
  __syncthreads();
  cluster_sync();

  if (warp == BWD_NW) {
    // ---------------------------------------------- producer: reverse order
    if (lane == 0) {
      int slot = 0, l = NL - 1;
      uint32_t empty_phase = 0;
      bool first_lap = true;
      // only the transposed mixing chunks: the forward's mixing outputs are
      // stored, not recomputed
      const int nck = a.mix ? a.nchunk : 0;
      for (long long g = 0; g < total_steps; ++g) {
        const int hslot = (int)(g & 1);
        if (g >= 2) mbar_wait(&head_empty[hslot], (uint32_t)(((g >> 1) - 1) & 1), kProducerSleepNs);
        mbar_arrive_expect_tx(&head_full[hslot], (uint32_t)a.HST * 4u);
        bulk_g2s(head_ring + hslot * a.HST, my_pack + l * layer_stride, (uint32_t)a.HST * 4u,
                 &head_full[hslot]);
        for (int i = 0; i < nck; ++i) {
          if (!first_lap) mbar_wait(&chunk_empty[slot], empty_phase, kProducerSleepNs);
          mbar_arrive_expect_tx(&chunk_full[slot], (uint32_t)a.CF * 4u);
          bulk_g2s(chunk_ring + (long long)slot * a.CF,
                   my_pack + l * layer_stride + a.HST + (long long)(a.nchunk + i) * a.CF, (uint32_t)a.CF * 4u,
                   &chunk_full[slot]);
          if (++slot == a.NST) {
            slot = 0;
            if (first_lap) first_lap = false; else empty_phase ^= 1u;
          }
        }
        if (--l < 0) l = NL - 1;
      }
    }
    __syncwarp();
    cluster_sync();
    return;
  }

  // ---------------------------------------------- compute warps
  const int nunits = R * hpc;
  int urow[BWD_MAXU], uhl[BWD_MAXU];
  bool uok[BWD_MAXU];
#pragma unroll
  for (int i = 0; i < BWD_MAXU; ++i) {
    const int u = warp + BWD_NW * i;
    uok[i] = u < nunits;
    urow[i] = uok[i] ? u / hpc : 0;
    uhl[i] = uok[i] ? u - urow[i] * hpc : 0;
  }
  int jj[EPL];
  bool eok[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    jj[e] = lane + 32 * e;
    eok[e] = jj[e] < hd;
    if (!eok[e]) jj[e] = hd - 1;
  }
  auto valid = [&](int i, int e) { return uok[i] && eok[e] && row0 + urow[i] < B; };
  auto colof = [&](int i, int e) { return col0 + uhl[i] * hd + jj[e]; };

  // upstream gradients of this unit's elements (dL/dx_out, dL/dv_out)
  float dxu[BWD_MAXU][EPL], dvu[BWD_MAXU][EPL], fsum[BWD_MAXU][EPL];
#pragma unroll
  for (int i = 0; i < BWD_MAXU; ++i)
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      dxu[i][e] = dvu[i][e] = fsum[i][e] = 0.f;
      if (valid(i, e)) {
        const long long off = (long long)(row0 + urow[i]) * d + colof(i, e);
        if (a.gx_fin) dxu[i][e] = a.gx_fin[off];
        if (a.gv_fin) dvu[i][e] = a.gv_fin[off];
      }
    }

  int cslot = 0;
  uint32_t cphase = 0;
  const float inv_d = 1.f / (float)d;
  const float rms_eps = 1.1920928955078125e-07f;
  long long g = 0;
  for (int t = L - 1; t >= 0; --t) {
    // upstream from this token's outputs
#pragma unroll
    for (int i = 0; i < BWD_MAXU; ++i)
#pragma unroll
      for (int e = 0; e < EPL; ++e)
        if (valid(i, e)) {
          const long long off = ((long long)(row0 + urow[i]) * L + t) * d + colof(i, e);
          if (a.gx_seq) dxu[i][e] += a.gx_seq[off];
          if (a.gv_seq) dvu[i][e] += a.gv_seq[off];
        }
    float fc[BWD_MAXU][EPL];
#pragma unroll
    for (int i = 0; i < BWD_MAXU; ++i)
#pragma unroll
      for (int e = 0; e < EPL; ++e)
        fc[i][e] = valid(i, e) ? bwd_force(a, t, row0 + urow[i], colof(i, e)) : 0.f;

    for (int l = NL - 1; l >= 0; --l, ++g) {
      const int hslot = (int)(g & 1);
      const float* hs = head_ring + hslot * a.HST;
      mbar_wait(&head_full[hslot], (uint32_t)((g >> 1) & 1));
      const long long step_off = ((long long)l * L + t) * BD;  // [l][t] slice of [NL][L][B][d]
      // layer-step input state
      float xin[BWD_MAXU][EPL], vin[BWD_MAXU][EPL];
#pragma unroll
      for (int i = 0; i < BWD_MAXU; ++i)
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
          xin[i][e] = vin[i][e] = 0.f;
          if (valid(i, e)) {
            const long long off = step_off + (long long)(row0 + urow[i]) * d + colof(i, e);
            xin[i][e] = a.traj[off];
            vin[i][e] = a.traj[sig_stride + off];
          }
        }
      float dxo[BWD_MAXU][EPL], dvo[BWD_MAXU][EPL];  // grads at the head-step outputs
      // ---- 1. recompute the head step forward -> (x', v')
      float x2s[BWD_MAXU][EPL], v2s[BWD_MAXU][EPL];
#pragma unroll
      for (int i = 0; i < BWD_MAXU; ++i) {
        if (!uok[i]) continue;
        const int hl = uhl[i];
        const float* U = hs + ho.U + hl * hd * RK;
        const float* Wg = hs + ho.W + hl * hd * RK;
        const float* WfT = hs + ho.WfT + hl * hd * hd;
        const float* bfh = hs + ho.bf + hl * hd;
        const float eff = a.base_dt * hs[ho.sc + hl];
        const float hh = 0.5f * eff;
        float p[RK], n, s, G[EPL], z[EPL];
        bwd_proj<RK, EPL>(vin[i], U, eok, jj, p, n, s);
        bwd_gamma<RK, EPL>(p, s, Wg, eok, jj, G);
        bwd_friction_pre<EPL>(xin[i], WfT, bfh, hd, jj, z);
        float vh[EPL];
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
          const float mu = sigmoid_f(z[e]) * 5.f;
          vh[e] = (vin[i][e] + hh * (fc[i][e] - G[e])) / (1.f + hh * mu);
          x2s[i][e] = xin[i][e] + eff * vh[e];
        }
        bwd_proj<RK, EPL>(vh, U, eok, jj, p, n, s);
        bwd_gamma<RK, EPL>(p, s, Wg, eok, jj, G);
        bwd_friction_pre<EPL>(x2s[i], WfT, bfh, hd, jj, z);
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
          const float mu = sigmoid_f(z[e]) * 5.f;
          v2s[i][e] = (vh[e] + hh * (fc[i][e] - G[e])) / (1.f + hh * mu);
        }
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
          if (!eok[e]) continue;
          if (valid(i, e)) {
            const long long off = step_off + (long long)(row0 + urow[i]) * d + colof(i, e);
            a.ws[SIG_X2 * sig_stride + off] = x2s[i][e];
            a.ws[SIG_V2 * sig_stride + off] = v2s[i][e];
          }
          if (a.mix) {
            const int cidx = ((int)crank * R + urow[i]) * C + hl * hd + jj[e];
            catx[cidx] = x2s[i][e];
            catv[cidx] = v2s[i][e];
          }
        }
      }

      if (a.mix) {
        // ---- the forward's mixing outputs of this CTA's columns (stored by
        // the training forward; no concat exchange, mixing recompute or
        // sums-of-squares exchange)
        const long long nlbd = (long long)NL * L * BD;
#pragma unroll
        for (int i = 0; i < BWD_MAXU; ++i) {
          if (!uok[i]) continue;
#pragma unroll
          for (int e = 0; e < EPL; ++e) {
            if (!eok[e]) continue;
            const int col = uhl[i] * hd + jj[e];
            float zx = 0.f, zv = 0.f;
            if (valid(i, e)) {
              const long long off = step_off + (long long)(row0 + urow[i]) * d + col0 + col;
              zx = a.traj[2 * nlbd + off];
              zv = a.traj[3 * nlbd + off];
            }
            ox[urow[i] * C + col] = zx;
            ov[urow[i] * C + col] = zv;
          }
        }
        // ---- RMSNorm / saturation backward, first half
        float rxs[BWD_MAXU], rvs[BWD_MAXU], dyx[BWD_MAXU][EPL], dyv[BWD_MAXU][EPL];
#pragma unroll
        for (int i = 0; i < BWD_MAXU; ++i) {
          rxs[i] = rvs[i] = 0.f;
          if (!uok[i]) continue;
          const int row = urow[i];
          float rx = 1.f, rv = 1.f;
          if (row0 + row < B) {  // [2][NL][L][B] after the inputs and mixing outputs
            const long long ro = 4 * nlbd + ((long long)l * L + t) * B + row0 + row;
            rx = a.traj[ro];
            rv = a.traj[ro + (long long)NL * L * B];
          }
          rxs[i] = rx;
          rvs[i] = rv;
#pragma unroll
          for (int e = 0; e < EPL; ++e) {
            const int col = uhl[i] * hd + jj[e];
            const float zx = ox[row * C + col], zv = ov[row * C + col];
            const float gxw = hs[ho.gx + col], gvw = hs[ho.gv + col];
            const float yx = zx * rx, yv = zv * rv;
            const float w = yv * gvw;
            const float vn = 100.f * tanhf(w / 100.f);
            const float dw = dvu[i][e] * (1.f - (vn / 100.f) * (vn / 100.f));
            dyx[i][e] = dxu[i][e] * gxw;
            dyv[i][e] = dw * gvw;
            if (eok[e]) {
              px[row * C + col] = dyx[i][e] * zx;
              pv[row * C + col] = dyv[i][e] * zv;
            }
            if (valid(i, e)) {
              const long long off = step_off + (long long)(row0 + row) * d + col0 + col;
              a.ws[SIG_SGX * sig_stride + off] = dxu[i][e] * yx;
              a.ws[SIG_SGV * sig_stride + off] = dw * yv;
            }
          }
        }
        named_sync<BWD_CT>();
        // ---- E3: row dot products sum_k dy_k z_k
        for (int row = warp; row < R; row += BWD_NW) {
          float sx = 0.f, sv = 0.f;
          for (int j = lane; j < C; j += 32) {
            sx += px[row * C + j];
            sv += pv[row * C + j];
          }
          sx = warp_sum(sx);
          sv = warp_sum(sv);
          if (lane < K)
            st_async2(dsmem_addr(part2 + ((int)crank * R + row) * 2, lane), sx, sv,
                      dsmem_addr(part2_bar, lane));
        }
        mbar_wait(part2_bar, (uint32_t)(g & 1));
        if (tid == 0) mbar_arrive_expect_tx(part2_bar, part_bytes);
#pragma unroll
        for (int i = 0; i < BWD_MAXU; ++i) {
          if (!uok[i]) continue;
          const int row = urow[i];
          float s3x = 0.f, s3v = 0.f;
          for (int c2 = 0; c2 < K; ++c2) {
            s3x += part2[(c2 * R + row) * 2];
            s3v += part2[(c2 * R + row) * 2 + 1];
          }
          const float rx = rxs[i], rv = rvs[i];
#pragma unroll
          for (int e = 0; e < EPL; ++e) {
            if (!eok[e]) continue;
            const int col = uhl[i] * hd + jj[e];
            const float zx = ox[row * C + col], zv = ov[row * C + col];
            const float dzx = rx * dyx[i][e] - (rx * rx * rx * inv_d) * zx * s3x;
            const float dzv = rv * dyv[i][e] - (rv * rv * rv * inv_d) * zv * s3v;
            const int cidx = ((int)crank * R + row) * C + col;
            dcx[cidx] = dzx;
            dcv[cidx] = dzv;
            if (valid(i, e)) {
              const long long off = step_off + (long long)(row0 + row) * d + col0 + col;
              a.ws[SIG_DZX * sig_stride + off] = dzx;
              a.ws[SIG_DZV * sig_stride + off] = dzv;
            }
          }
        }
        // ---- E4: all-gather dz, then dx_cat = Wx^T dz for this CTA's columns
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        named_sync<BWD_CT>();
        if (tid < K && tid != (int)crank) {
          const uint32_t off = (uint32_t)((int)crank * R * C);
          const uint32_t rb = dsmem_addr(dxch_bar, tid);
          bulk_s2peer(dsmem_addr(dcx + off, tid), dcx + off, blk_bytes, rb);
          bulk_s2peer(dsmem_addr(dcv + off, tid), dcv + off, blk_bytes, rb);
        }
        if (K > 1) mbar_wait(dxch_bar, (uint32_t)(g & 1));
        if (tid == 0 && K > 1) mbar_arrive_expect_tx(dxch_bar, xch_bytes);
        bwd_mix<BWD_CT>(a, dcx, dcv, ox, ov, nullptr, nullptr, chunk_ring, chunk_full, chunk_empty,
                        cslot, cphase, tid, lane);
        named_sync<BWD_CT>();
#pragma unroll
        for (int i = 0; i < BWD_MAXU; ++i)
#pragma unroll
          for (int e = 0; e < EPL; ++e) {
            const int col = uhl[i] * hd + jj[e];
            dxo[i][e] = uok[i] ? ox[urow[i] * C + col] : 0.f;
            dvo[i][e] = uok[i] ? ov[urow[i] * C + col] : 0.f;
          }
      } else {
#pragma unroll
        for (int i = 0; i < BWD_MAXU; ++i)
#pragma unroll
          for (int e = 0; e < EPL; ++e) {
            const float vn = 100.f * tanhf(v2s[i][e] / 100.f);
            dxo[i][e] = dxu[i][e];
            dvo[i][e] = dvu[i][e] * (1.f - (vn / 100.f) * (vn / 100.f));
          }
      }

      // ---- 2. head step backward (recomputing its intermediates)
#pragma unroll
      for (int i = 0; i < BWD_MAXU; ++i) {
        if (!uok[i]) continue;
        const int hl = uhl[i];
        const int h = (int)crank * hpc + hl;
        const float* U = hs + ho.U + hl * hd * RK;
        const float* Wg = hs + ho.W + hl * hd * RK;
        const float* WfT = hs + ho.WfT + hl * hd * hd;
        const float* Wfn = hs + a.HS + hl * hd * hd;  // untransposed [j][k]
        const float* bfh = hs + ho.bf + hl * hd;
        const float eff = a.base_dt * hs[ho.sc + hl];
        const float hh = 0.5f * eff;
        float p1[RK], n1, s1, G1[EPL], z1[EPL], mu1[EPL], D1[EPL], vh[EPL];
        float p2[RK], n2, s2, G2[EPL], z2[EPL], mu2[EPL], D2[EPL];
        bwd_proj<RK, EPL>(vin[i], U, eok, jj, p1, n1, s1);
        bwd_gamma<RK, EPL>(p1, s1, Wg, eok, jj, G1);
        bwd_friction_pre<EPL>(xin[i], WfT, bfh, hd, jj, z1);
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
          mu1[e] = sigmoid_f(z1[e]) * 5.f;
          D1[e] = 1.f + hh * mu1[e];
          vh[e] = (vin[i][e] + hh * (fc[i][e] - G1[e])) / D1[e];
        }
        bwd_proj<RK, EPL>(vh, U, eok, jj, p2, n2, s2);
        bwd_gamma<RK, EPL>(p2, s2, Wg, eok, jj, G2);
        bwd_friction_pre<EPL>(x2s[i], WfT, bfh, hd, jj, z2);
        float dvh[EPL], dG[EPL], dz[EPL], dx[EPL], dv[EPL], dFe[EPL];
        float dh = 0.f, deff = 0.f;
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
          mu2[e] = sigmoid_f(z2[e]) * 5.f;
          D2[e] = 1.f + hh * mu2[e];
          const float dN2 = dvo[i][e] / D2[e];
          const float dD2 = -dvo[i][e] * v2s[i][e] / D2[e];
          const float dmu2 = dD2 * hh;
          dvh[e] = dN2;
          dFe[e] = dN2 * hh;
          dG[e] = -dN2 * hh;
          if (eok[e]) dh += dD2 * mu2[e] + dN2 * (fc[i][e] - G2[e]);
          dz[e] = eok[e] ? dmu2 * mu2[e] * (1.f - mu2[e] / 5.f) : 0.f;
        }
        float wt[EPL];
        bwd_friction_t<EPL>(dz, Wfn, hd, jj, wt);
        float dg[EPL], qv[RK], dp[RK];
#pragma unroll
        for (int e = 0; e < EPL; ++e) dx[e] = dxo[i][e] + wt[e];
        bwd_gamma_back<RK, EPL>(dG, G2, p2, n2, s2, U, Wg, eok, jj, dvh, dg, qv, dp);
        const long long rowbase = step_off + (long long)(row0 + urow[i]) * d;
        const bool rowok = row0 + urow[i] < B;
        const long long smlbase = ((((long long)l * L + t) * B + row0 + urow[i]) * H + h) * RK;
#pragma unroll
        for (int e = 0; e < EPL; ++e)
          if (valid(i, e)) {
            const long long off = rowbase + colof(i, e);
            a.ws[SIG_DZ2 * sig_stride + off] = dz[e];
            a.ws[SIG_DG2 * sig_stride + off] = dg[e];
            a.ws[SIG_VH * sig_stride + off] = vh[e];
          }
        if (rowok && lane < RK) {
          float qs = qv[0], ps = dp[0];
#pragma unroll
          for (int q = 1; q < RK; ++q)
            if (lane == q) { qs = qv[q]; ps = dp[q]; }
          a.ws[BWD_NSIG * sig_stride + SML_Q2 * sml_stride + smlbase + lane] = qs;
          a.ws[BWD_NSIG * sig_stride + SML_DP2 * sml_stride + smlbase + lane] = ps;
        }
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
          if (eok[e]) {
            dvh[e] += eff * dx[e];
            deff += dx[e] * vh[e];
          }
          const float dN1 = dvh[e] / D1[e];
          const float dD1 = -dvh[e] * vh[e] / D1[e];
          const float dmu1 = dD1 * hh;
          if (eok[e]) dh += dD1 * mu1[e] + dN1 * (fc[i][e] - G1[e]);
          dv[e] = dN1;
          dFe[e] += dN1 * hh;
          dG[e] = -dN1 * hh;
          dz[e] = eok[e] ? dmu1 * mu1[e] * (1.f - mu1[e] / 5.f) : 0.f;
        }
        bwd_friction_t<EPL>(dz, Wfn, hd, jj, wt);
#pragma unroll
        for (int e = 0; e < EPL; ++e) dx[e] += wt[e];
        bwd_gamma_back<RK, EPL>(dG, G1, p1, n1, s1, U, Wg, eok, jj, dv, dg, qv, dp);
#pragma unroll
        for (int e = 0; e < EPL; ++e)
          if (valid(i, e)) {
            const long long off = rowbase + colof(i, e);
            a.ws[SIG_DZ1 * sig_stride + off] = dz[e];
            a.ws[SIG_DG1 * sig_stride + off] = dg[e];
          }
        if (rowok && lane < RK) {
          float qs = qv[0], ps = dp[0];
#pragma unroll
          for (int q = 1; q < RK; ++q)
            if (lane == q) { qs = qv[q]; ps = dp[q]; }
          a.ws[BWD_NSIG * sig_stride + SML_Q1 * sml_stride + smlbase + lane] = qs;
          a.ws[BWD_NSIG * sig_stride + SML_DP1 * sml_stride + smlbase + lane] = ps;
        }
        const float deff_tot = warp_sum(deff + 0.5f * dh);
        if (rowok && lane == 0)
          a.ws[BWD_NSIG * sig_stride + BWD_NSMALL * sml_stride +
               (((long long)l * L + t) * B + row0 + urow[i]) * H + h] = deff_tot;
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
          dxu[i][e] = eok[e] ? dx[e] : 0.f;
          dvu[i][e] = eok[e] ? dv[e] : 0.f;
          fsum[i][e] += eok[e] ? dFe[e] : 0.f;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&head_empty[hslot]);
    }
    // ---- token done: force gradient (times the mask, as the force was)
#pragma unroll
    for (int i = 0; i < BWD_MAXU; ++i)
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        if (valid(i, e) && a.dforces) {
          const long long idx = (long long)(row0 + urow[i]) * L + t;
          const float m = a.mask ? a.mask[idx] : 1.f;
          a.dforces[idx * d + colof(i, e)] = fsum[i][e] * m;
        }
        fsum[i][e] = 0.f;
      }
  }
#pragma unroll
  for (int i = 0; i < BWD_MAXU; ++i)
#pragma unroll
    for (int e = 0; e < EPL; ++e)
      if (valid(i, e)) {
        const long long off = (long long)(row0 + urow[i]) * d + colof(i, e);
        a.dx0[off] = dxu[i][e];
        a.dv0[off] = dvu[i][e];
      }
  cluster_sync();
}

}  // namespace gfn
