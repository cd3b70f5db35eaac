// Single-layer operators of the reference's gfn.cuda boundary:
//   christoffel_fused : Gamma(v) for one head            (gfn/cuda/ops.py:88-118)
//   leapfrog_fused    : one head's leapfrog integrator   (gfn/cuda/ops.py:131-182,
//                       semantics gfn/integrators/symplectic/leapfrog.py:50-114)
// Both reuse the head-step device code of the fused recurrence.
#pragma once
#include "leapfrog_seq.cuh"

namespace gfn {

constexpr int SMALL_THREADS = 256;

// Gamma of output column j from the row's projection p (recomputes the scale).
template <int RK>
GFN_DEV float small_gamma(const float* __restrict__ p, const float* __restrict__ Wrow) {
  float pr[RK];
  const float sc = seq_proj_scale<RK>(p, pr);
  return seq_gamma<RK>(pr, sc, Wrow);
}

// z = x_head . Wf[j, :] + bf[j] with WfT stored [k][j].
GFN_DEV float small_friction_pre(const float* __restrict__ xr, const float* __restrict__ wt, int hd,
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
constexpr int SMALL_ROWS = 8;  // rows per block

struct HeadArgs {
  const float* x;
  const float* v;
  const float* f;     // [B, hd] or null (zero force)
  const float* U;     // [hd, r]
  const float* W;     // [hd, r]
  const float* Wf;    // [hd, hd] or null (no friction)
  const float* bf;    // [hd] or null
  const float* dt_scale;  // 1 or B values, or null (1.0)
  int dt_scale_n;
  float dt;
  int steps;
  float* x_out;
  float* v_out;
  float* gamma_out;   // christoffel only
  int B, hd;
};

// Shared-memory layout for SMALL_ROWS rows of one head.
struct SmallSmem {
  int WfT, U, W, bf, xs, vs, fs, zb, pb, total;
};

__host__ __device__ inline SmallSmem small_smem(int hd, int r) {
  SmallSmem s;
  s.WfT = 0;
  s.U = hd * hd;
  s.W = s.U + hd * r;
  s.bf = s.W + hd * r;
  s.xs = ((s.bf + hd + 3) / 4) * 4;
  s.vs = s.xs + SMALL_ROWS * hd;
  s.fs = s.vs + SMALL_ROWS * hd;
  s.zb = s.fs + SMALL_ROWS * hd;
  s.pb = s.zb + SMALL_ROWS * hd;
  s.total = s.pb + SMALL_ROWS * r;
  return s;
}

template <int RK>
GFN_DEV void small_load_weights(const HeadArgs& a, float* sm, const SmallSmem& L, bool friction) {
  const int hd = a.hd;
  for (int i = threadIdx.x; i < hd * RK; i += blockDim.x) {
    sm[L.U + i] = a.U[i];
    sm[L.W + i] = a.W[i];
  }
  if (friction) {
    for (int i = threadIdx.x; i < hd * hd; i += blockDim.x) {
      const int k = i / hd, j = i - k * hd;
      sm[L.WfT + i] = a.Wf[j * hd + k];
    }
    for (int i = threadIdx.x; i < hd; i += blockDim.x) sm[L.bf + i] = a.bf ? a.bf[i] : 0.f;
  }
}

template <int RK>
__global__ void __launch_bounds__(SMALL_THREADS) christoffel_kernel(const HeadArgs a) {
  extern __shared__ __align__(16) float sm[];
  const SmallSmem L = small_smem(a.hd, RK);
  const int hd = a.hd, row0 = blockIdx.x * SMALL_ROWS;
  const int rows = min(SMALL_ROWS, a.B - row0);
  small_load_weights<RK>(a, sm, L, false);
  for (int i = threadIdx.x; i < SMALL_ROWS * hd; i += blockDim.x) {
    const int r = i / hd;
    sm[L.vs + i] = r < rows ? a.v[(long long)(row0 + r) * hd + (i - r * hd)] : 0.f;
  }
  __syncthreads();
  seq_head_proj<RK>(sm + L.vs, sm + L.U, sm + L.pb, SMALL_ROWS, 1, hd, hd, threadIdx.x >> 5,
                    threadIdx.x & 31, SMALL_THREADS / 32);
  __syncthreads();
  for (int i = threadIdx.x; i < rows * hd; i += blockDim.x) {
    const int r = i / hd, j = i - r * hd;
    a.gamma_out[(long long)(row0 + r) * hd + j] = small_gamma<RK>(sm + L.pb + r * RK, sm + L.W + j * RK);
  }
}

template <int RK>
__global__ void __launch_bounds__(SMALL_THREADS) leapfrog_head_kernel(const HeadArgs a) {
  extern __shared__ __align__(16) float sm[];
  const SmallSmem L = small_smem(a.hd, RK);
  const int hd = a.hd, row0 = blockIdx.x * SMALL_ROWS;
  const int rows = min(SMALL_ROWS, a.B - row0);
  const bool friction = a.Wf != nullptr;
  small_load_weights<RK>(a, sm, L, friction);
  for (int i = threadIdx.x; i < SMALL_ROWS * hd; i += blockDim.x) {
    const int r = i / hd;
    const bool ok = r < rows;
    const long long g = (long long)(row0 + r) * hd + (i - r * hd);
    sm[L.xs + i] = ok ? a.x[g] : 0.f;
    sm[L.vs + i] = ok ? a.v[g] : 0.f;
    sm[L.fs + i] = (ok && a.f) ? a.f[g] : 0.f;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int s = 0; s < a.steps; ++s) {
    for (int half = 0; half < 2; ++half) {
      seq_head_proj<RK>(sm + L.vs, sm + L.U, sm + L.pb, SMALL_ROWS, 1, hd, hd, warp, lane,
                        SMALL_THREADS / 32);
      for (int i = threadIdx.x; i < SMALL_ROWS * hd; i += blockDim.x) {
        const int r = i / hd, j = i - r * hd;
        sm[L.zb + i] = friction ? small_friction_pre(sm + L.xs + r * hd, sm + L.WfT + j, hd, sm[L.bf + j])
                                : 0.f;
      }
      __syncthreads();
      for (int i = threadIdx.x; i < SMALL_ROWS * hd; i += blockDim.x) {
        const int r = i / hd, j = i - r * hd;
        float sc = 1.f;
        if (a.dt_scale) sc = a.dt_scale[a.dt_scale_n == 1 ? 0 : min(row0 + r, a.B - 1)];
        const float eff = a.dt * sc;
        const float h = 0.5f * eff;
        const float gm = small_gamma<RK>(sm + L.pb + r * RK, sm + L.W + j * RK);
        const float mu = friction ? sigmoid_f(sm[L.zb + i]) * 5.f : 0.f;
        const float vn = (sm[L.vs + i] + h * (sm[L.fs + i] - gm)) / (1.f + h * mu);
        sm[L.vs + i] = vn;
        if (half == 0) sm[L.xs + i] = sm[L.xs + i] + eff * vn;
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < rows * hd; i += blockDim.x) {
    const int r = i / hd;
    const long long g = (long long)(row0 + r) * hd + (i - r * hd);
    a.x_out[g] = sm[L.xs + i];
    a.v_out[g] = sm[L.vs + i];
  }
}

}  // namespace gfn
