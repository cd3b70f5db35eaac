// Persistent fused leapfrog recurrence: all tokens x all layers x all heads in
// one launch, (x, v) resident on chip for the whole sequence.
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
// rows for the whole sequence.  CTA c owns C = d/K columns (hpc = H/K whole
// heads) of every layer.  Inside the CTA a "unit" is one (row, head): warp w
// owns units w, w+8, ..., and lane l holds elements l, l+32, ... of each
// unit's x, v and force in registers across all layers and tokens.
// Per layer step:
//   1. head step of each unit entirely in registers: the v.U projection is
//      a warp butterfly, the friction GEMV broadcasts x by shuffles and reads
//      the forget-gate weight from shared memory -- no block barrier;
//   2. all-gather of (x', v'): every unit st.async-stores its columns into
//      every peer's concat buffer; the stores complete on the receiver's
//      mbarrier (transaction bytes), so no cluster barrier and no fence;
//   3. mixing for the CTA's 2C output columns (x and v), split-K over the
//      256 compute threads, k-vectorised, partials combined by a warp
//      reduce-scatter; weights stream through a ring of shared-memory slots
//      filled by a producer warp with 1-D bulk copies (independent of the
//      data, so layer l+1's copies overlap layer l's math);
//   4. one block barrier, per-row sums of squares exchanged like step 2,
//      RMSNorm and saturation applied by each unit in registers.
// No grid-wide synchronisation (rows are independent) and no atomics: for a
// fixed launch plan the result is bitwise deterministic.
#pragma once
#include "common.cuh"

namespace gfn {

// The kernel runs NW compute warps (8 or 16) plus one producer warp.  With
// 9 warps a thread may hold 168 registers (3 warps share an SM
// sub-partition), with 17 warps ~96; units per warp follow from that.
template <int NW>
struct SeqShape {
  static constexpr int CWARPS = NW;
  static constexpr int CTHREADS = NW * 32;
  static constexpr int THREADS = CTHREADS + 32;
  static constexpr int MAXU = NW == 8 ? 3 : 2;  // units per warp: R*hpc <= NW*MAXU
  // The 8-warp form runs two CTAs per SM (two independent row blocks whose
  // dependent chains interleave); the 16-warp form one.
  static constexpr int MINB = NW == 8 ? 2 : 1;
};
constexpr int SEQ_NBAR = 48;                        // mbarrier slots reserved
// Back-off of the weight-producer warp between barrier polls (the poll itself
// suspends in hardware; a long sleep only delays the refill).
constexpr uint32_t kProducerSleepNs = 128;
constexpr int SEQ_BAR_BYTES = SEQ_NBAR * 8;
constexpr int SEQ_MAX_NST = (SEQ_NBAR - 6) / 2;     // ring depth limit
constexpr int SEQ_PROF_N = 12;

struct HeadOffsets {
  int WfT, U, W, bf, bx, bv, gx, gv, sc, total;
};

// Per-(layer, CTA) "head section" of the packed weights, in floats.
// WfT is the forget-gate weight transposed to [hpc][k][j] so that lanes
// with consecutive j read consecutive words; sc = softplus(dt_params).
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
  o.sc = o.gv + C;
  o.total = ((o.sc + hpc + 31) / 32) * 32;
  return o;
}

// Row stride (floats) of a mixing chunk [KC][2C + 4]: the 4-float pad
// rotates consecutive k rows across bank groups for the k-split lanes.
__host__ __device__ inline int chunk_row_stride(int C) { return 2 * C + 4; }
// 16-byte units of weight-chunk row k are XOR-permuted by (k / 4) & 7 (when
// a row's 2C/4 data units are a multiple of 8): the mixing loop's lanes read
// rows 4 apart, which the 4-float pad alone would map onto two bank groups.
__host__ __device__ inline int chunk_swizzle_mask(int C) { return ((2 * C / 4) % 8 == 0) ? 7 : 0; }

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
  long long* prof;  // optional per-phase cycle counters (CTA 0), SEQ_PROF_N entries
  int B, L, d, H, hd, NL;
  int K, R, C, hpc, KC, nchunk, NST;
  int HS, CF;
  long long LF;
  int mix;
  int TR, NG, tiles, S;   // mixing tiles: TR rows x 4 columns, S-way k split
  int logC;               // log2(C) when C is a power of two, else -1
  float base_dt;
  int o_head, o_chunk, o_ox, o_ov, o_catx, o_catv, o_part;
  int chunk_base;   // offset of the first weight chunk in a (layer, CTA) pack run
  float* traj;      // optional, for BPTT: [2][NL][L][B][d] every layer step's input (x, v),
                    // then [2][NL][L][B][d] its mixing outputs (z_x, z_v, bias included),
                    // then [2][NL][L][B] its RMSNorm factors (r_x, r_v)
};

// ---------------------------------------------------------------- PTX bits
template <int CT>
GFN_DEV void named_sync() { asm volatile("bar.sync 1, %0;" ::"n"(CT) : "memory"); }

GFN_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// st.async of floats into a peer CTA's shared memory, completing on that
// CTA's mbarrier (4 / 8 transaction bytes).
GFN_DEV void st_async1(uint32_t raddr, float v, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.f32 [%0], %1, [%2];" ::"r"(raddr),
               "f"(v), "r"(rbar)
               : "memory");
}

GFN_DEV void st_async2(uint32_t raddr, float a, float b, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(
                   raddr),
               "f"(a), "f"(b), "r"(rbar)
               : "memory");
}

// Bulk copy of this CTA's shared memory into a peer CTA's shared memory,
// completing on the peer's mbarrier (bytes a multiple of 16, 16-B aligned).
GFN_DEV void bulk_s2peer(uint32_t rdst, const void* src, uint32_t bytes, uint32_t rbar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          rdst),
      "r"(smem_u32(src)), "r"(bytes), "r"(rbar)
      : "memory");
}

// ---------------------------------------------------------------- shared helpers
// (also used by the single-head kernels in ops_small.cuh)

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
#pragma unroll
      for (int q4 = 0; q4 < RK; q4 += 4) {
        const float4 u = *reinterpret_cast<const float4*>(Uh + k * RK + q4);
        acc[q4 + 0] = fmaf(vv, u.x, acc[q4 + 0]);
        acc[q4 + 1] = fmaf(vv, u.y, acc[q4 + 1]);
        acc[q4 + 2] = fmaf(vv, u.z, acc[q4 + 2]);
        acc[q4 + 3] = fmaf(vv, u.w, acc[q4 + 3]);
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

// Gamma for one output column from its head's projection and W row.
template <int RK>
GFN_DEV float seq_gamma(const float* __restrict__ pr, float sc, const float* __restrict__ Wrow) {
  float g = 0.f;
#pragma unroll
  for (int q = 0; q < RK; ++q) g = fmaf((pr[q] * pr[q]) * sc, Wrow[q], g);
  return soft_clamp20(g);
}

// s = 1 / (1 + |p| + 1e-6) (gfn/geometry/lowrank.py:95-96).
template <int RK>
GFN_DEV float seq_proj_scale(const float* __restrict__ p, float* pr) {
  float ss = 0.f;
#pragma unroll
  for (int q = 0; q < RK; ++q) {
    pr[q] = p[q];
    ss = fmaf(pr[q], pr[q], ss);
  }
  return 1.f / ((1.f + sqrtf(ss)) + 1e-6f);
}

// Reduce-scatter of 16 values over the S (<= 16) lanes that differ in the
// low log2(S) lane bits (butterfly, fixed order).  Level L halves the live
// set (8 >> L values exchanged over lane bit S >> (L+1)); on return the lane
// holds cnt = 16 / S fully reduced values v[0..cnt) for entries
// base..base+cnt-1.  Halves are compile-time so v stays in registers.
GFN_DEV void reduce_scatter16(float (&v)[16], int S, int lane, int& base, int& cnt) {
  base = 0;
  cnt = 16;
#pragma unroll
  for (int L = 0; L < 4; ++L) {
    const int half = 8 >> L;
    const int m = S >> (L + 1);
    if (m >= 1) {
      const bool upper = (lane & m) != 0;
#pragma unroll
      for (int i = 0; i < half; ++i) {
        const float send = upper ? v[i] : v[i + half];
        const float keep = upper ? v[i + half] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, m);
      }
      if (upper) base += half;
      cnt = half;
    }
  }
}

// ---------------------------------------------------------------- unit helpers
// Force element of row b, column col at token t.
GFN_DEV float seq_load_force(const SeqArgs& a, int t, int b, int col) {
  const long long idx = (long long)b * a.L + t;
  float f;
  if (a.f32) {
    f = __ldg(a.f32 + idx * a.d + col);
  } else if (a.fbf16) {
    f = __bfloat162float(a.fbf16[idx * a.d + col]);
  } else {
    const long long id = __ldg(a.ids + idx);
    if (id < 0 || id >= a.vocab) {
      gfn_flag_error(kDevErrBadToken);
      f = 0.f;
    } else {
      f = __ldg(a.table + id * a.d + col);
    }
  }
  if (a.mask) f = f * __ldg(a.mask + idx);
  return f;
}

// Gamma(v) for the lane's EPL elements of one unit (lane-resident v).
template <int RK, int EPL>
GFN_DEV void unit_gamma(const float (&vv)[EPL], const float* __restrict__ U,
                        const float* __restrict__ W, const bool (&ok)[EPL], const int (&jj)[EPL],
                        float (&g)[EPL]) {
  float p[RK];
#pragma unroll
  for (int q = 0; q < RK; ++q) p[q] = 0.f;
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    if (ok[e]) {
#pragma unroll
      for (int q4 = 0; q4 < RK; q4 += 4) {
        const float4 u = *reinterpret_cast<const float4*>(U + jj[e] * RK + q4);
        p[q4 + 0] = fmaf(vv[e], u.x, p[q4 + 0]);
        p[q4 + 1] = fmaf(vv[e], u.y, p[q4 + 1]);
        p[q4 + 2] = fmaf(vv[e], u.z, p[q4 + 2]);
        p[q4 + 3] = fmaf(vv[e], u.w, p[q4 + 3]);
      }
    }
  }
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1)
#pragma unroll
    for (int q = 0; q < RK; ++q) p[q] += __shfl_xor_sync(0xffffffffu, p[q], m);
  float ss = 0.f;
#pragma unroll
  for (int q = 0; q < RK; ++q) ss = fmaf(p[q], p[q], ss);
  const float sc = 1.f / ((1.f + sqrtf(ss)) + 1e-6f);
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    float acc = 0.f;
    if (ok[e]) {
#pragma unroll
      for (int q4 = 0; q4 < RK; q4 += 4) {
        const float4 w = *reinterpret_cast<const float4*>(W + jj[e] * RK + q4);
        acc = fmaf((p[q4 + 0] * p[q4 + 0]) * sc, w.x, acc);
        acc = fmaf((p[q4 + 1] * p[q4 + 1]) * sc, w.y, acc);
        acc = fmaf((p[q4 + 2] * p[q4 + 2]) * sc, w.z, acc);
        acc = fmaf((p[q4 + 3] * p[q4 + 3]) * sc, w.w, acc);
      }
    }
    g[e] = soft_clamp20(acc);
  }
}

// mu(x) = 5 sigmoid(x Wf^T + bf) for the lane's elements; x is broadcast
// across the warp by shuffles, WfT is [k][j] in shared memory.
template <int EPL, int HDC>
GFN_DEV void unit_friction_impl(const float (&xx)[EPL], const float* __restrict__ WfT,
                           const float* __restrict__ bf, int hd_rt, const int (&jj)[EPL],
                           float (&mu)[EPL]) {
  const int hd = HDC ? HDC : hd_rt;
  float z0[EPL], z1[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) z0[e] = z1[e] = 0.f;
#pragma unroll
  for (int e2 = 0; e2 < EPL; ++e2) {
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
  }
#pragma unroll
  for (int e = 0; e < EPL; ++e) mu[e] = sigmoid_f((z0[e] + z1[e]) + bf[jj[e]]) * 5.f;
}

template <int EPL>
GFN_DEV void unit_friction(const float (&xx)[EPL], const float* __restrict__ WfT,
                           const float* __restrict__ bf, int hd, const int (&jj)[EPL],
                           float (&mu)[EPL]) {
  // compile-time head_dim when it fills the lanes (no per-k bounds checks)
  if (hd == 32 * EPL)
    unit_friction_impl<EPL, 32 * EPL>(xx, WfT, bf, hd, jj, mu);
  else
    unit_friction_impl<EPL, 0>(xx, WfT, bf, hd, jj, mu);
}

template <int RK, int EPL, int NW>
__global__ void __launch_bounds__(SeqShape<NW>::THREADS, SeqShape<NW>::MINB) leapfrog_seq_kernel(const SeqArgs a) {
  constexpr int SEQ_CWARPS = SeqShape<NW>::CWARPS;
  constexpr int SEQ_CTHREADS = SeqShape<NW>::CTHREADS;
  constexpr int SEQ_MAXU = SeqShape<NW>::MAXU;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw);
  uint64_t* head_full = bars;            // [2]
  uint64_t* head_empty = bars + 2;       // [2]
  uint64_t* xch_bar = bars + 4;          // concat exchange
  uint64_t* part_bar = bars + 5;         // partial sums exchange
  uint64_t* chunk_full = bars + 6;       // [NST]
  uint64_t* chunk_empty = bars + 6 + a.NST;  // [NST]
  float* sm = reinterpret_cast<float*>(smem_raw + SEQ_BAR_BYTES);
  float* head_ring = sm + a.o_head;
  float* chunk_ring = sm + a.o_chunk;
  float* ox = sm + a.o_ox;
  float* ov = sm + a.o_ov;
  float* catx = sm + a.o_catx;
  float* catv = sm + a.o_catv;
  float* part = sm + a.o_part;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t crank = cluster_ctarank();
  const int cl = blockIdx.x / a.K;
  const int row0 = cl * a.R;
  const int C = a.C, R = a.R, d = a.d, hd = a.hd, hpc = a.hpc, K = a.K;
  const int col0 = (int)crank * C;
  const HeadOffsets ho = head_offsets(hpc, hd, RK, C);
  const long long total_steps = (long long)a.L * a.NL;
  const float* my_pack = a.pack + (long long)crank * a.LF;
  const long long layer_stride = (long long)K * a.LF;
  // Concat buffers are [K][R][C]: CTA c's columns for all rows are one
  // contiguous block, copied to every peer with one bulk copy each.
  const uint32_t blk_bytes = (uint32_t)(R * C * 4);
  const uint32_t xch_bytes = 2u * (uint32_t)(K - 1) * blk_bytes;
  const uint32_t part_bytes = (uint32_t)(K * R * 2 * 4);

  if (tid == 0) {
    for (int i = 0; i < 6 + 2 * a.NST; ++i) {
      const bool is_empty = (i >= 2 && i < 4) || (i >= 6 + a.NST);
      mbar_init(&bars[i], is_empty ? SEQ_CWARPS : 1);
    }
    fence_mbar_init();
    if (a.mix) {
      if (K > 1) mbar_arrive_expect_tx(xch_bar, xch_bytes);
      mbar_arrive_expect_tx(part_bar, part_bytes);
    }
  }
  __syncthreads();
  cluster_sync();  // peers' barriers initialised before any st.async reaches them

  if (warp == SEQ_CWARPS) {
    // ------------------------------------------------------- producer warp
    if (lane == 0) {
      // Ring position tracked incrementally (no integer division per chunk).
      int slot = 0, l = 0;
      uint32_t empty_phase = 0;  // parity of the release this slot's next fill waits for
      bool first_lap = true;
      for (long long g = 0; g < total_steps; ++g) {
        const int hslot = (int)(g & 1);
        if (g >= 2) mbar_wait(&head_empty[hslot], (uint32_t)(((g >> 1) - 1) & 1), kProducerSleepNs);
        mbar_arrive_expect_tx(&head_full[hslot], (uint32_t)a.HS * 4u);
        bulk_g2s(head_ring + hslot * a.HS, my_pack + l * layer_stride, (uint32_t)a.HS * 4u,
                 &head_full[hslot]);
        for (int i = 0; a.mix && i < a.nchunk; ++i) {
          if (!first_lap) mbar_wait(&chunk_empty[slot], empty_phase, kProducerSleepNs);
          mbar_arrive_expect_tx(&chunk_full[slot], (uint32_t)a.CF * 4u);
          bulk_g2s(chunk_ring + (long long)slot * a.CF,
                   my_pack + l * layer_stride + a.chunk_base + (long long)i * a.CF, (uint32_t)a.CF * 4u,
                   &chunk_full[slot]);
          if (++slot == a.NST) {
            slot = 0;
            if (first_lap) first_lap = false; else empty_phase ^= 1u;
          }
        }
        if (++l == a.NL) l = 0;
      }
    }
    __syncwarp();
    cluster_sync();
    return;
  }

  // ------------------------------------------------------- compute warps
  // Optional phase counters: thread 0 of CTA 0 keeps them in shared memory
  // (not registers) so the counters cost the hot path nothing when off.
  const bool prof = a.prof != nullptr && blockIdx.x == 0 && tid == 0;
  __shared__ long long pacc[SEQ_PROF_N];
  __shared__ long long pt_s;
  if (prof) {
    for (int i = 0; i < SEQ_PROF_N; ++i) pacc[i] = 0;
    pt_s = clock64();
  }
  auto mark = [&](int i) {
    if (prof) {
      const long long now = clock64();
      pacc[i] += now - pt_s;
      pt_s = now;
    }
  };

  // Units of this warp: u = warp + 8 i -> (row u / hpc, head u % hpc).
  const int nunits = R * hpc;
  int urow[SEQ_MAXU], uhl[SEQ_MAXU];
  bool uok[SEQ_MAXU];
#pragma unroll
  for (int i = 0; i < SEQ_MAXU; ++i) {
    const int u = warp + SEQ_CWARPS * i;
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
    if (!eok[e]) jj[e] = hd - 1;  // harmless in-range index for idle lanes
  }

  float xr[SEQ_MAXU][EPL], vr[SEQ_MAXU][EPL], fc[SEQ_MAXU][EPL], fn[SEQ_MAXU][EPL];
#pragma unroll
  for (int i = 0; i < SEQ_MAXU; ++i)
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      xr[i][e] = vr[i][e] = fc[i][e] = fn[i][e] = 0.f;
      const int b = row0 + urow[i];
      if (uok[i] && eok[e] && b < a.B) {
        const long long off = (long long)b * a.state_stride + col0 + uhl[i] * hd + jj[e];
        xr[i][e] = a.x0[off];
        vr[i][e] = a.v0[off];
        if (a.L > 0) fn[i][e] = seq_load_force(a, 0, b, col0 + uhl[i] * hd + jj[e]);
      }
    }

  // Mixing tile of this thread: rows r0..r0+TR-1, columns n0..n0+3 of the
  // [x | v] block, k-split ms (low lane bits) of S.
  const int S = a.S;
  const bool mix_active = tid < a.tiles * S;
  const int ms = tid % S, mtile = tid / S;
  const int mng = mtile % a.NG, mrg = mtile / a.NG;
  const int mn0 = mng * 4, mr0 = mrg * a.TR;
  const float* mcat = (mn0 < C) ? catx : catv;
  const int CS = chunk_row_stride(C);
  const int swz = chunk_swizzle_mask(C);
  const float inv_d = 1.f / (float)d;
  const float rms_eps = 1.1920928955078125e-07f;  // float32 machine epsilon

  long long g = 0;
  int cslot = 0;            // chunk ring position of the consumers
  uint32_t cphase = 0;
  for (int t = 0; t < a.L; ++t) {
#pragma unroll
    for (int i = 0; i < SEQ_MAXU; ++i)
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        fc[i][e] = fn[i][e];
        const int b = row0 + urow[i];
        if (t + 1 < a.L && uok[i] && eok[e] && b < a.B)
          fn[i][e] = seq_load_force(a, t + 1, b, col0 + uhl[i] * hd + jj[e]);
      }

    for (int l = 0; l < a.NL; ++l, ++g) {
      const int hslot = (int)(g & 1);
      const float* hs = head_ring + hslot * a.HS;
      mbar_wait(&head_full[hslot], (uint32_t)((g >> 1) & 1));
      mark(0);
      if (a.traj) {  // checkpoint of this layer step's input for the backward
        const long long BD = (long long)a.B * d;
        const long long so = ((long long)l * a.L + t) * BD;
#pragma unroll
        for (int i = 0; i < SEQ_MAXU; ++i)
#pragma unroll
          for (int e = 0; e < EPL; ++e) {
            const int b = row0 + urow[i];
            if (!uok[i] || !eok[e] || b >= a.B) continue;
            const long long off = so + (long long)b * d + col0 + uhl[i] * hd + jj[e];
            a.traj[off] = xr[i][e];
            a.traj[(long long)a.NL * a.L * BD + off] = vr[i][e];
          }
      }

      // ---- head step of every unit, in registers
#pragma unroll
      for (int i = 0; i < SEQ_MAXU; ++i) {
        if (!uok[i]) continue;
        const int hl = uhl[i];
        const float* U = hs + ho.U + hl * hd * RK;
        const float* Wg = hs + ho.W + hl * hd * RK;
        const float* WfT = hs + ho.WfT + hl * hd * hd;
        const float* bfh = hs + ho.bf + hl * hd;
        const float eff = a.base_dt * hs[ho.sc + hl];
        const float hh = 0.5f * eff;
        float gm[EPL], mu[EPL];
        // kick 1 (implicit friction at x), drift
        unit_gamma<RK, EPL>(vr[i], U, Wg, eok, jj, gm);
        unit_friction<EPL>(xr[i], WfT, bfh, hd, jj, mu);
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
          const float vh = (vr[i][e] + hh * (fc[i][e] - gm[e])) / (1.f + hh * mu[e]);
          xr[i][e] = xr[i][e] + eff * vh;
          vr[i][e] = vh;
        }
        // kick 2 at x'
        unit_gamma<RK, EPL>(vr[i], U, Wg, eok, jj, gm);
        unit_friction<EPL>(xr[i], WfT, bfh, hd, jj, mu);
#pragma unroll
        for (int e = 0; e < EPL; ++e)
          vr[i][e] = (vr[i][e] + hh * (fc[i][e] - gm[e])) / (1.f + hh * mu[e]);
        if (a.mix) {
#pragma unroll
          for (int e = 0; e < EPL; ++e) {
            if (!eok[e]) continue;
            const int cidx = ((int)crank * R + urow[i]) * C + hl * hd + jj[e];
            catx[cidx] = xr[i][e];
            catv[cidx] = vr[i][e];
          }
        } else {
#pragma unroll
          for (int e = 0; e < EPL; ++e) vr[i][e] = saturate100(vr[i][e]);
        }
      }
      mark(1);

      if (a.mix) {
        // Own block complete -> bulk-copy it into every peer's concat buffer
        // (completing on the peer's mbarrier).  The generic-proxy writes
        // must be visible to the async proxy that reads the source.
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        named_sync<SEQ_CTHREADS>();
        if (tid < K && tid != (int)crank) {
          const uint32_t off = (uint32_t)((int)crank * R * C);
          const uint32_t rb = dsmem_addr(xch_bar, tid);
          bulk_s2peer(dsmem_addr(catx + off, tid), catx + off, blk_bytes, rb);
          bulk_s2peer(dsmem_addr(catv + off, tid), catv + off, blk_bytes, rb);
        }
        if (K > 1) mbar_wait(xch_bar, (uint32_t)(g & 1));  // every CTA's columns have landed
        mark(2);
        // Arm the next phase.  Threads still polling this phase's parity keep
        // seeing it complete: the next phase needs this CTA's own next sends,
        // which come after the block barrier below.
        if (tid == 0 && K > 1) mbar_arrive_expect_tx(xch_bar, xch_bytes);
        // ---- head mixing: [R x d] . [d x 2C] for this CTA's columns
        float acc[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[i] = 0.f;
        for (int i = 0; i < a.nchunk; ++i) {
          const int slot = cslot;
          mbar_wait(&chunk_full[slot], cphase);
          if (++cslot == a.NST) {  // ring position, tracked without division
            cslot = 0;
            cphase ^= 1u;
          }
          mark(8);
          const float* wc = chunk_ring + (long long)slot * a.CF;
          if (mix_active) {
            const int k0 = i * a.KC;
            for (int kk = 4 * ms; kk < a.KC; kk += 4 * S) {
              // concat element k lives in column block k / C (C = 2^logC when a
              // chunk spans blocks; otherwise the chunk lies inside one block)
              const int kg = k0 + kk;
              const float* cblk = a.logC >= 0
                  ? mcat + ((kg >> a.logC) * R) * C + (kg & (C - 1))
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
          mark(3);
        }
        mark(3);
        if (mix_active) {
          int base, cnt;
          reduce_scatter16(acc, S, lane, base, cnt);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            if (i < cnt) {
              const int e = base + i;
              const int rr = e >> 2, c = e & 3;
              const int n = mn0 + c, row = mr0 + rr;
              if (rr < a.TR && row < R) {
                if (n < C)
                  ox[row * C + n] = acc[i] + hs[ho.bx + n];
                else
                  ov[row * C + n - C] = acc[i] + hs[ho.bv + n - C];
              }
            }
          }
        }
        named_sync<SEQ_CTHREADS>();
        mark(4);
        // ---- per-row partial sums of squares -> every CTA of the cluster
        for (int row = warp; row < R; row += SEQ_CWARPS) {
          float sx = 0.f, sv = 0.f;
          for (int j = lane; j < C; j += 32) {
            const float u = ox[row * C + j];
            const float w = ov[row * C + j];
            sx = fmaf(u, u, sx);
            sv = fmaf(w, w, sv);
          }
          sx = warp_sum(sx);
          sv = warp_sum(sv);
          if (lane < K)
            st_async2(dsmem_addr(part + ((int)crank * R + row) * 2, lane), sx, sv,
                      dsmem_addr(part_bar, lane));
        }
        mbar_wait(part_bar, (uint32_t)(g & 1));
        if (tid == 0) mbar_arrive_expect_tx(part_bar, part_bytes);  // arm the next phase
        mark(5);
        // ---- RMSNorm + saturation of each unit, in registers
#pragma unroll
        for (int i = 0; i < SEQ_MAXU; ++i) {
          if (!uok[i]) continue;
          const int row = urow[i];
          float ssx = 0.f, ssv = 0.f;
          for (int c2 = 0; c2 < K; ++c2) {
            const float2 pp = *reinterpret_cast<const float2*>(part + (c2 * R + row) * 2);
            ssx += pp.x;
            ssv += pp.y;
          }
          const float rx = 1.f / sqrtf(ssx * inv_d + rms_eps);
          const float rv = 1.f / sqrtf(ssv * inv_d + rms_eps);
          if (a.traj) {  // the mixing outputs and RMSNorm factors, for the backward
            const long long BD = (long long)a.B * d;
            const long long nlb = (long long)a.NL * a.L;
            const long long so = ((long long)l * a.L + t) * BD;
            const int b = row0 + row;
            if (b < a.B) {
#pragma unroll
              for (int e = 0; e < EPL; ++e) {
                if (!eok[e]) continue;
                const int col = uhl[i] * hd + jj[e];
                const long long off = so + (long long)b * d + col0 + col;
                a.traj[2 * nlb * BD + off] = ox[row * C + col];
                a.traj[3 * nlb * BD + off] = ov[row * C + col];
              }
              if (crank == 0 && uhl[i] == 0 && lane == 0) {
                const long long ro = 4 * nlb * BD + ((long long)l * a.L + t) * a.B + b;
                a.traj[ro] = rx;
                a.traj[ro + nlb * a.B] = rv;
              }
            }
          }
#pragma unroll
          for (int e = 0; e < EPL; ++e) {
            const int col = uhl[i] * hd + jj[e];
            xr[i][e] = (ox[row * C + col] * rx) * hs[ho.gx + col];
            vr[i][e] = saturate100((ov[row * C + col] * rv) * hs[ho.gv + col]);
          }
        }
        mark(6);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&head_empty[hslot]);  // head slot free
    }
    // ---- token output (state after the last layer)
#pragma unroll
    for (int i = 0; i < SEQ_MAXU; ++i)
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        const int b = row0 + urow[i];
        if (!uok[i] || !eok[e] || b >= a.B) continue;
        const long long off = ((long long)b * a.L + t) * d + col0 + uhl[i] * hd + jj[e];
        if (a.x_seq) __stcs(a.x_seq + off, xr[i][e]);
        if (a.v_seq) __stcs(a.v_seq + off, vr[i][e]);
      }
    mark(7);
  }
#pragma unroll
  for (int i = 0; i < SEQ_MAXU; ++i)
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const int b = row0 + urow[i];
      if (!uok[i] || !eok[e] || b >= a.B) continue;
      const long long off = (long long)b * d + col0 + uhl[i] * hd + jj[e];
      if (a.x_out) a.x_out[off] = xr[i][e];
      if (a.v_out) a.v_out[off] = vr[i][e];
    }
  if (prof) {
    pacc[SEQ_PROF_N - 1] = (long long)a.L * a.NL;
    for (int i = 0; i < SEQ_PROF_N; ++i) a.prof[i] = pacc[i];
  }
  cluster_sync();  // no CTA leaves while a peer may still address its SMEM
}

}  // namespace gfn
