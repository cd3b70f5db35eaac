// Persistent fused leapfrog recurrence: all tokens x all layers x all heads in
// one launch, (x, v) resident in shared memory for the whole sequence.
//
// Semantics (one layer step, Euclidean, leapfrog, per head of width hd):
//   Gamma(v) = 20 tanh(((vU)^2 / (1 + |vU| + 1e-6)) W^T / 20)   gfn/geometry/lowrank.py:93-98,125-127
//   mu(x)    = 5 sigmoid(x Wf^T + bf)                             gfn/integrators/symplectic/leapfrog.py:72-81
//   v_half   = (v + h (F - Gamma(v))) / (1 + h mu(x))            leapfrog.py:85
//   x'       = x + dt_eff v_half                                  leapfrog.py:88
//   v'       = (v_half + h (F - Gamma(v_half))) / (1 + h mu(x'))  leapfrog.py:114
//   dt_eff   = base_dt softplus(dt_params[h]), h = dt_eff / 2     gfn/layers/base.py:220, leapfrog.py:55-56
// then, when heads > 1, head mixing + RMSNorm + velocity saturation
//   x_next = RMSNorm_gx(x' Wx^T + bx), v_next = 100 tanh(RMSNorm_gv(v' Wv^T + bv)/100)
//                                                                 gfn/layers/base.py:305-335
// and the token loop with F_t = F[:, t] * mask[:, t]              gfn/model.py:377-402.
//
// Decomposition.  A thread-block cluster of K CTAs owns a block of R batch
// rows for the whole sequence.  CTA c of the cluster owns C = d/K columns,
// i.e. hpc = H/K whole heads, of every layer.  Per layer step:
//   1. head step for its heads on its R rows (all operands in SMEM);
//   2. DSMEM all-gather of (x', v') so every CTA holds the R x d concat;
//   3. mixing GEMM for its C output columns of both x and v, split-K over
//      the 256 threads, weights streamed as k-chunks by the bulk-copy engine
//      through a ring of NST shared-memory slots, issued NST chunks ahead
//      (they do not depend on the data, so the copy of layer l+1's weights
//      overlaps layer l's math);
//   4. DSMEM exchange of per-row partial sums of squares -> RMSNorm,
//      saturation; the CTA now holds its columns of the next layer's input.
// Two cluster barriers per layer step; no grid-wide synchronisation (rows
// are independent), no atomics (bitwise-deterministic for a fixed plan).
#pragma once
#include "common.cuh"

namespace gfn {

constexpr int SEQ_THREADS = 256;
constexpr int SEQ_OPT = 4;          // head-step outputs per thread: R*C <= 1024
constexpr int SEQ_RED_FLOATS = 4096;  // split-K partials: S*R*2C <= 256*16

struct HeadOffsets {
  int WfT, U, W, bf, bx, bv, gx, gv, dt, total;
};

// Per-(layer, CTA) "head section" of the packed weights, in floats.
// WfT is the forget-gate weight transposed to [hpc][k][j] so that the
// threads of a warp (consecutive j) read consecutive words.
__host__ __device__ inline HeadOffsets head_offsets(int hpc, int hd, int r, int C) {
  HeadOffsets o;
  o.WfT = 0;
  o.U = hpc * hd * hd;
  o.W = o.U + hpc * hd * r;
  o.bf = o.W + hpc * hd * r;
  o.bx = o.bf + C;
  o.bv = o.bx + C;
  o.gx = o.bv + C;
  o.gv = o.gx + C;
  o.dt = o.gv + C;
  o.total = ((o.dt + hpc + 31) / 32) * 32;
  return o;
}

struct SeqArgs {
  const float* x0;
  const float* v0;
  long long state_stride;  // floats between rows of x0/v0 (0: one row broadcast)
  const float* f32;        // forces [B, L, d] float32, or
  const __nv_bfloat16* fbf16;  // forces [B, L, d] bfloat16, or
  const long long* ids;    // token ids [B, L] + table [vocab, d]
  const float* table;
  long long vocab;
  const float* mask;  // [B, L] or null
  const float* pack;
  float* x_seq;
  float* v_seq;
  float* x_out;
  float* v_out;
  int B, L, d, H, hd, NL;
  int K, R, C, hpc, KC, nchunk, NST;
  int HS, CF;
  long long LF;
  int mix;
  int TR, NG, tiles, S;
  float base_dt;
  int o_head, o_chunk, o_xs, o_vs, o_ox, o_ov, o_catx, o_catv, o_part, o_p, o_red;
};

GFN_DEV void seq_load_force(const SeqArgs& a, int t, int row0, int col0, const int* orow,
                            const int* ocol, float* f) {
#pragma unroll
  for (int i = 0; i < SEQ_OPT; ++i) {
    f[i] = 0.f;
    if (orow[i] < 0) continue;
    const int b = row0 + orow[i];
    if (b >= a.B) continue;
    const long long idx = (long long)b * a.L + t;
    const long long col = col0 + ocol[i];
    float v;
    if (a.f32) {
      v = a.f32[idx * a.d + col];
    } else if (a.fbf16) {
      v = __bfloat162float(a.fbf16[idx * a.d + col]);
    } else {
      const long long id = a.ids[idx];
      if (id < 0 || id >= a.vocab) {
        gfn_flag_error(kDevErrBadToken);
        v = 0.f;
      } else {
        v = a.table[id * a.d + col];
      }
    }
    if (a.mask) v = v * a.mask[idx];
    f[i] = v;
  }
}

// p[row][hl][q] = sum_k v[row][hl*hd + k] U[hl][k][q]: one warp per (row, head).
template <int RK>
GFN_DEV void seq_head_proj(const float* __restrict__ vsrc, const float* __restrict__ U,
                           float* __restrict__ pbuf, int R, int hpc, int hd, int C, int warp,
                           int lane, int nwarps) {
  for (int pair = warp; pair < R * hpc; pair += nwarps) {
    const int row = pair / hpc, hl = pair - row * hpc;
    const float* vr = vsrc + row * C + hl * hd;
    const float* Uh = U + hl * hd * RK;
    float acc[RK];
#pragma unroll
    for (int q = 0; q < RK; ++q) acc[q] = 0.f;
    for (int k = lane; k < hd; k += 32) {
      const float vv = vr[k];
      if constexpr (RK % 4 == 0) {
#pragma unroll
        for (int q4 = 0; q4 < RK; q4 += 4) {
          const float4 u = *reinterpret_cast<const float4*>(Uh + k * RK + q4);
          acc[q4 + 0] = fmaf(vv, u.x, acc[q4 + 0]);
          acc[q4 + 1] = fmaf(vv, u.y, acc[q4 + 1]);
          acc[q4 + 2] = fmaf(vv, u.z, acc[q4 + 2]);
          acc[q4 + 3] = fmaf(vv, u.w, acc[q4 + 3]);
        }
      } else {
#pragma unroll
        for (int q = 0; q < RK; ++q) acc[q] = fmaf(vv, Uh[k * RK + q], acc[q]);
      }
    }
#pragma unroll
    for (int q = 0; q < RK; ++q) acc[q] = warp_sum(acc[q]);
    if (lane < RK) {
      float mine = acc[0];
#pragma unroll
      for (int q = 1; q < RK; ++q)
        if (lane == q) mine = acc[q];
      pbuf[(row * hpc + hl) * RK + lane] = mine;
    }
  }
}

// Gamma for one output column jj of head hl from that head's projection p.
template <int RK>
GFN_DEV float seq_gamma(const float* __restrict__ p, const float* __restrict__ Wrow) {
  float pr[RK];
  float ss = 0.f;
#pragma unroll
  for (int q = 0; q < RK; ++q) {
    pr[q] = p[q];
    ss = fmaf(pr[q], pr[q], ss);
  }
  const float nrm = sqrtf(ss);
  const float sc = 1.f / ((1.f + nrm) + 1e-6f);
  float g = 0.f;
#pragma unroll
  for (int q = 0; q < RK; ++q) g = fmaf((pr[q] * pr[q]) * sc, Wrow[q], g);
  return soft_clamp20(g);
}

// Friction pre-activation z = x_head . Wf[j, :] + bf[j] for one output.
GFN_DEV float seq_friction_pre(const float* __restrict__ xr, const float* __restrict__ wt, int hd,
                               float bias) {
  float s0 = 0.f, s1 = 0.f;
  int k = 0;
  for (; k + 1 < hd; k += 2) {
    s0 = fmaf(xr[k], wt[k * hd], s0);
    s1 = fmaf(xr[k + 1], wt[(k + 1) * hd], s1);
  }
  if (k < hd) s0 = fmaf(xr[k], wt[k * hd], s0);
  return (s0 + s1) + bias;
}

template <int RK>
__global__ void __launch_bounds__(SEQ_THREADS, 1) leapfrog_seq_kernel(const SeqArgs a) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw);
  uint64_t* head_full = bars;       // [2]
  uint64_t* chunk_full = bars + 2;  // [NST]
  float* sm = reinterpret_cast<float*>(smem_raw + 128);
  float* head_ring = sm + a.o_head;
  float* chunk_ring = sm + a.o_chunk;
  float* xs = sm + a.o_xs;
  float* vs = sm + a.o_vs;
  float* ox = sm + a.o_ox;
  float* ov = sm + a.o_ov;
  float* catx = sm + a.o_catx;
  float* catv = sm + a.o_catv;
  float* part = sm + a.o_part;
  float* pbuf = sm + a.o_p;
  float* red = sm + a.o_red;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int NW = SEQ_THREADS / 32;
  const uint32_t crank = cluster_ctarank();
  const int cl = blockIdx.x / a.K;
  const int row0 = cl * a.R;
  const int C = a.C, R = a.R, d = a.d, hd = a.hd, hpc = a.hpc, K = a.K;
  const int col0 = (int)crank * C;
  const HeadOffsets ho = head_offsets(hpc, hd, RK, C);
  const long long total_steps = (long long)a.L * a.NL;
  const long long total_chunks = a.mix ? total_steps * a.nchunk : 0;
  const float* my_pack = a.pack + (long long)crank * a.LF;
  const long long layer_stride = (long long)K * a.LF;

  auto issue_head = [&](long long g) {
    const int l = (int)(g % a.NL);
    uint64_t* bar = &head_full[g & 1];
    mbar_arrive_expect_tx(bar, (uint32_t)a.HS * 4u);
    bulk_g2s(head_ring + (g & 1) * a.HS, my_pack + l * layer_stride, (uint32_t)a.HS * 4u, bar);
  };
  auto issue_chunk = [&](long long q) {
    const long long g = q / a.nchunk;
    const int i = (int)(q - g * a.nchunk);
    const int l = (int)(g % a.NL);
    const int slot = (int)(q % a.NST);
    uint64_t* bar = &chunk_full[slot];
    mbar_arrive_expect_tx(bar, (uint32_t)a.CF * 4u);
    bulk_g2s(chunk_ring + (long long)slot * a.CF,
             my_pack + l * layer_stride + a.HS + (long long)i * a.CF, (uint32_t)a.CF * 4u, bar);
  };

  if (tid == 0) {
    for (int i = 0; i < 2 + a.NST; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) {
    if (total_steps > 0) issue_head(0);
    for (long long q = 0; q < total_chunks && q < a.NST; ++q) issue_chunk(q);
  }

  // This thread's head-step outputs (row, column), fixed for the launch.
  const int RC = R * C;
  int orow[SEQ_OPT], ocol[SEQ_OPT], ohl[SEQ_OPT], ojj[SEQ_OPT];
#pragma unroll
  for (int i = 0; i < SEQ_OPT; ++i) {
    const int o = tid + i * SEQ_THREADS;
    if (o < RC) {
      orow[i] = o / C;
      ocol[i] = o - orow[i] * C;
      ohl[i] = ocol[i] / hd;
      ojj[i] = ocol[i] - ohl[i] * hd;
    } else {
      orow[i] = -1;
      ocol[i] = ohl[i] = ojj[i] = 0;
    }
  }
#pragma unroll
  for (int i = 0; i < SEQ_OPT; ++i) {
    if (orow[i] < 0) continue;
    const int b = row0 + orow[i];
    float xv = 0.f, vv = 0.f;
    if (b < a.B) {
      const long long off = (long long)b * a.state_stride + col0 + ocol[i];
      xv = a.x0[off];
      vv = a.v0[off];
    }
    xs[orow[i] * C + ocol[i]] = xv;
    vs[orow[i] * C + ocol[i]] = vv;
  }

  // Mixing tile of this thread: rows r0..r0+TR-1, columns n0..n0+3 of the
  // [x | v] output block, k-split s of S.
  const bool mix_active = tid < a.tiles * a.S;
  const int mtile = tid % a.tiles, ms = tid / a.tiles;
  const int mng = mtile % a.NG, mrg = mtile / a.NG;
  const int mn0 = mng * 4, mr0 = mrg * a.TR;
  const float* mcat = (mn0 < C) ? catx : catv;
  const int C2 = 2 * C;
  const float inv_d = 1.f / (float)d;
  const float rms_eps = 1.1920928955078125e-07f;  // float32 machine epsilon

  float fnext[SEQ_OPT];
  if (a.L > 0) seq_load_force(a, 0, row0, col0, orow, ocol, fnext);
  cluster_sync();  // every CTA of the cluster is resident before any DSMEM store

  long long g = 0, q = 0;
  for (int t = 0; t < a.L; ++t) {
    float fcur[SEQ_OPT];
#pragma unroll
    for (int i = 0; i < SEQ_OPT; ++i) fcur[i] = fnext[i];
    if (t + 1 < a.L) seq_load_force(a, t + 1, row0, col0, orow, ocol, fnext);

    for (int l = 0; l < a.NL; ++l, ++g) {
      if (tid == 0 && g + 1 < total_steps) issue_head(g + 1);
      const float* hs = head_ring + (g & 1) * a.HS;
      mbar_wait(&head_full[g & 1], (uint32_t)((g >> 1) & 1));

      float z[SEQ_OPT], hh[SEQ_OPT], eff[SEQ_OPT];
      // ---- kick 1: projections of v and friction of x
      seq_head_proj<RK>(vs, hs + ho.U, pbuf, R, hpc, hd, C, warp, lane, NW);
#pragma unroll
      for (int i = 0; i < SEQ_OPT; ++i) {
        if (orow[i] < 0) continue;
        z[i] = seq_friction_pre(xs + orow[i] * C + ohl[i] * hd,
                                hs + ho.WfT + ohl[i] * hd * hd + ojj[i], hd, hs[ho.bf + ocol[i]]);
        const float sc = softplus_f(hs[ho.dt + ohl[i]]);
        eff[i] = a.base_dt * sc;
        hh[i] = 0.5f * eff[i];
      }
      __syncthreads();
      // ---- kick 1 update + drift
#pragma unroll
      for (int i = 0; i < SEQ_OPT; ++i) {
        if (orow[i] < 0) continue;
        const int o = orow[i] * C + ocol[i];
        const float gm = seq_gamma<RK>(pbuf + (orow[i] * hpc + ohl[i]) * RK,
                                       hs + ho.W + (ohl[i] * hd + ojj[i]) * RK);
        const float mu = sigmoid_f(z[i]) * 5.f;
        const float vh = (vs[o] + hh[i] * (fcur[i] - gm)) / (1.f + hh[i] * mu);
        xs[o] = xs[o] + eff[i] * vh;
        vs[o] = vh;
      }
      __syncthreads();
      // ---- kick 2: projections of v_half, friction at x'
      seq_head_proj<RK>(vs, hs + ho.U, pbuf, R, hpc, hd, C, warp, lane, NW);
#pragma unroll
      for (int i = 0; i < SEQ_OPT; ++i) {
        if (orow[i] < 0) continue;
        z[i] = seq_friction_pre(xs + orow[i] * C + ohl[i] * hd,
                                hs + ho.WfT + ohl[i] * hd * hd + ojj[i], hd, hs[ho.bf + ocol[i]]);
      }
      __syncthreads();
#pragma unroll
      for (int i = 0; i < SEQ_OPT; ++i) {
        if (orow[i] < 0) continue;
        const int o = orow[i] * C + ocol[i];
        const float gm = seq_gamma<RK>(pbuf + (orow[i] * hpc + ohl[i]) * RK,
                                       hs + ho.W + (ohl[i] * hd + ojj[i]) * RK);
        const float mu = sigmoid_f(z[i]) * 5.f;
        const float vn = (vs[o] + hh[i] * (fcur[i] - gm)) / (1.f + hh[i] * mu);
        if (a.mix) {
          const float xn = xs[o];
          const int cidx = orow[i] * d + col0 + ocol[i];
          for (int k = 0; k < K; ++k) {
            dsmem_st(dsmem_addr(catx + cidx, k), xn);
            dsmem_st(dsmem_addr(catv + cidx, k), vn);
          }
        } else {
          vs[o] = saturate100(vn);
        }
      }

      if (a.mix) {
        cluster_sync();  // concat of all heads complete in every CTA
        // ---- head mixing: [R x d] . [d x 2C] for this CTA's columns
        float acc[4][4];
#pragma unroll
        for (int rr = 0; rr < 4; ++rr)
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) acc[rr][cc] = 0.f;
        for (int i = 0; i < a.nchunk; ++i, ++q) {
          const int slot = (int)(q % a.NST);
          mbar_wait(&chunk_full[slot], (uint32_t)((q / a.NST) & 1));
          const float* wc = chunk_ring + (long long)slot * a.CF;
          if (mix_active) {
            const float* catk = mcat + i * a.KC;
            for (int kk = ms; kk < a.KC; kk += a.S) {
              const float4 w = *reinterpret_cast<const float4*>(wc + kk * C2 + mn0);
#pragma unroll
              for (int rr = 0; rr < 4; ++rr) {
                if (rr < a.TR) {
                  const float xv = catk[(mr0 + rr) * d + kk];
                  acc[rr][0] = fmaf(xv, w.x, acc[rr][0]);
                  acc[rr][1] = fmaf(xv, w.y, acc[rr][1]);
                  acc[rr][2] = fmaf(xv, w.z, acc[rr][2]);
                  acc[rr][3] = fmaf(xv, w.w, acc[rr][3]);
                }
              }
            }
          }
          __syncthreads();  // slot consumed by every thread
          if (tid == 0 && q + a.NST < total_chunks) issue_chunk(q + a.NST);
        }
        if (mix_active) {
#pragma unroll
          for (int rr = 0; rr < 4; ++rr)
            if (rr < a.TR)
              *reinterpret_cast<float4*>(red + (ms * R + mr0 + rr) * C2 + mn0) =
                  make_float4(acc[rr][0], acc[rr][1], acc[rr][2], acc[rr][3]);
        }
        __syncthreads();
        for (int o = tid; o < R * C2; o += SEQ_THREADS) {
          const int row = o / C2, n = o - row * C2;
          float s = 0.f;
          for (int sp = 0; sp < a.S; ++sp) s += red[(sp * R + row) * C2 + n];
          if (n < C)
            ox[row * C + n] = s + hs[ho.bx + n];
          else
            ov[row * C + n - C] = s + hs[ho.bv + n - C];
        }
        __syncthreads();
        // ---- per-row partial sums of squares -> every CTA of the cluster
        for (int row = warp; row < R; row += NW) {
          float sx = 0.f, sv = 0.f;
          for (int j = lane; j < C; j += 32) {
            const float u = ox[row * C + j];
            const float w = ov[row * C + j];
            sx = fmaf(u, u, sx);
            sv = fmaf(w, w, sv);
          }
          sx = warp_sum(sx);
          sv = warp_sum(sv);
          if (lane < K) dsmem_st2(dsmem_addr(part + ((int)crank * R + row) * 2, lane), sx, sv);
        }
        cluster_sync();
        // ---- RMSNorm + saturation -> next layer's input
#pragma unroll
        for (int i = 0; i < SEQ_OPT; ++i) {
          if (orow[i] < 0) continue;
          const int row = orow[i];
          float ssx = 0.f, ssv = 0.f;
          for (int c2 = 0; c2 < K; ++c2) {
            ssx += part[(c2 * R + row) * 2];
            ssv += part[(c2 * R + row) * 2 + 1];
          }
          const float rx = 1.f / sqrtf(ssx * inv_d + rms_eps);
          const float rv = 1.f / sqrtf(ssv * inv_d + rms_eps);
          const int o = row * C + ocol[i];
          xs[o] = (ox[o] * rx) * hs[ho.gx + ocol[i]];
          vs[o] = saturate100((ov[o] * rv) * hs[ho.gv + ocol[i]]);
        }
      }
      __syncthreads();  // layer step done: head slot and xs/vs settled
    }
    // ---- token output (state after the last layer)
#pragma unroll
    for (int i = 0; i < SEQ_OPT; ++i) {
      if (orow[i] < 0) continue;
      const int b = row0 + orow[i];
      if (b >= a.B) continue;
      const long long off = ((long long)b * a.L + t) * d + col0 + ocol[i];
      const int o = orow[i] * C + ocol[i];
      if (a.x_seq) a.x_seq[off] = xs[o];
      if (a.v_seq) a.v_seq[off] = vs[o];
    }
  }
#pragma unroll
  for (int i = 0; i < SEQ_OPT; ++i) {
    if (orow[i] < 0) continue;
    const int b = row0 + orow[i];
    if (b >= a.B) continue;
    const long long off = (long long)b * d + col0 + ocol[i];
    const int o = orow[i] * C + ocol[i];
    if (a.x_out) a.x_out[off] = xs[o];
    if (a.v_out) a.v_out[off] = vs[o];
  }
  cluster_sync();  // no CTA leaves while a peer may still address its SMEM
}

}  // namespace gfn
