// Latency floor of one layer step of the fused recurrence.
//
// The recurrence is a dependent chain: a layer step cannot start before the
// previous one's RMSNorm, and inside a step every phase needs the previous
// one.  This kernel runs only that chain's unavoidable parts, with real data
// dependencies and the same primitives as leapfrog_seq_kernel, on the same
// cluster shape (K CTAs, one warp each):
//   2 x kick: Gamma's rank reduction (5-level butterfly of RK values), sqrt
//             and reciprocal, W contraction, 20 tanh(./20) clamp; the friction
//             dot product as a 5-level butterfly (its minimum depth), sigmoid;
//             the implicit-friction division; the drift FMA
//   concat exchange: st.async of the CTA's value to every peer, completing
//             on the receiver's mbarrier
//   mixing: the d-long dot product as K partial values + a 5-level butterfly
//   RMSNorm exchange: partial sums of squares to every peer (st.async)
//   RMSNorm + saturation: rsqrt, scale, 100 tanh(./100)
// No weights stream, nothing is loaded from memory, every warp does one
// unit: cycles per step is the floor the fused kernel's layer step is
// compared against (its "latency roofline").
#pragma once
#include "leapfrog_seq.cuh"

namespace gfn {

template <int RK>
GFN_DEV float probe_butterfly(float v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  return v;
}

template <int RK, int K>
__global__ void __launch_bounds__(32) latency_probe_kernel(int steps, long long* cycles) {
  __shared__ __align__(16) float recv[2][K];
  __shared__ __align__(8) uint64_t bars[2];
  const int lane = threadIdx.x;
  const uint32_t crank = cluster_ctarank();
  if (lane == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(&bars[0], K * 4);
    mbar_arrive_expect_tx(&bars[1], K * 4);
  }
  __syncwarp();
  cluster_sync();
  float x = 0.01f * (float)(lane + 1) + 0.001f * (float)crank;
  float v = 0.02f * (float)(lane + 1);
  const float hh = 0.05f, eff = 0.1f, F = 0.3f;
  long long t0 = clock64();
#pragma unroll 1
  for (int s = 0; s < steps; ++s) {
#pragma unroll
    for (int kick = 0; kick < 2; ++kick) {
      float p[RK];
#pragma unroll
      for (int q = 0; q < RK; ++q) p[q] = v * (0.1f + 0.01f * q);
#pragma unroll
      for (int m = 16; m >= 1; m >>= 1)
#pragma unroll
        for (int q = 0; q < RK; ++q) p[q] += __shfl_xor_sync(0xffffffffu, p[q], m);
      float ss = 0.f;
#pragma unroll
      for (int q = 0; q < RK; ++q) ss = fmaf(p[q], p[q], ss);
      const float sc = 1.f / ((1.f + sqrtf(ss)) + 1e-6f);
      float gs = 0.f;
#pragma unroll
      for (int q = 0; q < RK; ++q) gs = fmaf((p[q] * p[q]) * sc, 0.05f, gs);
      const float g = soft_clamp20(gs);
      const float z = probe_butterfly<RK>(x * 0.03f);
      const float mu = sigmoid_f(z) * 5.f;
      const float vh = (v + hh * (F - g)) / (1.f + hh * mu);
      if (kick == 0) x = x + eff * vh;
      v = vh;
    }
    // concat exchange
    const uint32_t ph = (uint32_t)(s & 1);
    if (lane < K) st_async1(dsmem_addr(&recv[0][crank], lane), x + v, dsmem_addr(&bars[0], lane));
    mbar_wait(&bars[0], ph, 0);
    if (lane == 0) mbar_arrive_expect_tx(&bars[0], K * 4);
    // mixing: K partials in, one dot-product reduction
    float acc = 0.f;
#pragma unroll
    for (int c = 0; c < K; ++c) acc = fmaf(recv[0][c], 0.01f * (c + 1), acc);
    acc = probe_butterfly<RK>(acc * (lane + 1));
    // RMSNorm partial sums exchange
    if (lane < K) st_async1(dsmem_addr(&recv[1][crank], lane), acc * acc, dsmem_addr(&bars[1], lane));
    mbar_wait(&bars[1], ph, 0);
    if (lane == 0) mbar_arrive_expect_tx(&bars[1], K * 4);
    float sq = 0.f;
#pragma unroll
    for (int c = 0; c < K; ++c) sq += recv[1][c];
    const float r = 1.f / sqrtf(sq * (1.f / 256.f) + 1.1920928955078125e-07f);
    x = (acc * r) * 0.9f + 0.01f * x;
    v = saturate100((acc * r) * 1.1f) * 0.5f + 0.5f * v;
  }
  long long t1 = clock64();
  if (lane == 0 && crank == 0 && blockIdx.x == 0) *cycles = t1 - t0;
  if (lane == 0 && crank == 0) recv[0][0] = x + v;  // keep the chain live
  cluster_sync();
}

}  // namespace gfn
