// Linear-recurrence scans of the parallel path (gfn/scan.py, gfn/layers/parallel.py).
//
//   y_t = a_t y_{t-1} + x_t   (y_{-1} = 0)   over t for every (b, column).
//
// The reference evaluates this with Hillis-Steele doubling (O(L log L) work,
// ~2 log2(L) passes over HBM).  Here the B*D columns are independent, so the
// work-efficient form is one sequential pass per column with the columns
// spread over threads: each thread owns 4 adjacent columns (128-bit loads,
// coalesced across the warp) and keeps 8 time steps of loads in flight.
// That reads a and x once and writes y once -- 12 bytes per element, the
// HBM minimum.  When B*D is too small to fill the GPU, the time axis is
// split into P chunks: pass 1 reduces each chunk to (prod a, local y),
// pass 2 chains the chunk carries, pass 3 rescans each chunk from its carry.
#pragma once
#include "common.cuh"

namespace gfn {

constexpr int SCAN_THREADS = 256;
constexpr int SCAN_UNROLL = 8;

// One column group (4 columns) over t in [t0, t1) starting from carry y.
// a == null means a == 1 (running sum).
GFN_DEV float4 scan_run(const float* __restrict__ a, const float* __restrict__ x, float* __restrict__ y,
                        long long base, long long stride, int t0, int t1, float4 c, float4* aprod) {
  float4 ap = make_float4(1.f, 1.f, 1.f, 1.f);
  int t = t0;
  for (; t + SCAN_UNROLL <= t1; t += SCAN_UNROLL) {
    float4 av[SCAN_UNROLL], xv[SCAN_UNROLL];
#pragma unroll
    for (int u = 0; u < SCAN_UNROLL; ++u) {
      const long long off = base + (long long)(t + u) * stride;
      xv[u] = __ldcs(reinterpret_cast<const float4*>(x + off));
      av[u] = a ? __ldcs(reinterpret_cast<const float4*>(a + off)) : make_float4(1.f, 1.f, 1.f, 1.f);
    }
#pragma unroll
    for (int u = 0; u < SCAN_UNROLL; ++u) {
      c.x = av[u].x * c.x + xv[u].x;
      c.y = av[u].y * c.y + xv[u].y;
      c.z = av[u].z * c.z + xv[u].z;
      c.w = av[u].w * c.w + xv[u].w;
      if (aprod) {
        ap.x *= av[u].x; ap.y *= av[u].y; ap.z *= av[u].z; ap.w *= av[u].w;
      }
      if (y) __stcs(reinterpret_cast<float4*>(y + base + (long long)(t + u) * stride), c);
    }
  }
  for (; t < t1; ++t) {
    const long long off = base + (long long)t * stride;
    const float4 xv = *reinterpret_cast<const float4*>(x + off);
    const float4 av = a ? *reinterpret_cast<const float4*>(a + off) : make_float4(1.f, 1.f, 1.f, 1.f);
    c.x = av.x * c.x + xv.x;
    c.y = av.y * c.y + xv.y;
    c.z = av.z * c.z + xv.z;
    c.w = av.w * c.w + xv.w;
    if (aprod) {
      ap.x *= av.x; ap.y *= av.y; ap.z *= av.z; ap.w *= av.w;
    }
    if (y) *reinterpret_cast<float4*>(y + off) = c;
  }
  if (aprod) *aprod = ap;
  return c;
}

struct ScanArgs {
  const float* a;  // [B, L, D] or null (a == 1)
  const float* x;  // [B, L, D]
  float* y;        // [B, L, D]
  float* ws;       // chunk aggregates: [2][P][B*D] floats (P > 1 only)
  int B, L, D, P;
};

// P == 1: one pass.  grid covers B*D/4 column groups.
__global__ void __launch_bounds__(SCAN_THREADS) scan_single_kernel(const ScanArgs s) {
  const long long g = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  const long long groups = (long long)s.B * (s.D / 4);
  if (g >= groups) return;
  const long long b = g / (s.D / 4), cg = g - b * (s.D / 4);
  const long long base = b * (long long)s.L * s.D + cg * 4;
  scan_run(s.a, s.x, s.y, base, s.D, 0, s.L, make_float4(0.f, 0.f, 0.f, 0.f), nullptr);
}

// Pass 1: chunk aggregates.  grid: (groups, P)
__global__ void __launch_bounds__(SCAN_THREADS) scan_chunk_reduce_kernel(const ScanArgs s) {
  const long long g = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  const int p = blockIdx.y;
  const long long groups = (long long)s.B * (s.D / 4);
  if (g >= groups) return;
  const long long b = g / (s.D / 4), cg = g - b * (s.D / 4);
  const long long base = b * (long long)s.L * s.D + cg * 4;
  const int cl = (s.L + s.P - 1) / s.P;
  const int t0 = p * cl, t1 = min(s.L, t0 + cl);
  float4 ap;
  const float4 yl = scan_run(s.a, s.x, nullptr, base, s.D, t0, max(t0, t1), make_float4(0.f, 0.f, 0.f, 0.f), &ap);
  const long long BD = (long long)s.B * s.D;
  *reinterpret_cast<float4*>(s.ws + (long long)p * BD + g * 4) = ap;
  *reinterpret_cast<float4*>(s.ws + ((long long)s.P + p) * BD + g * 4) = yl;
}

// Pass 2: carry into chunk p = fold of chunks 0..p-1; stored over the local y slot.
__global__ void __launch_bounds__(SCAN_THREADS) scan_chunk_carry_kernel(const ScanArgs s) {
  const long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  const long long BD = (long long)s.B * s.D;
  if (e >= BD) return;
  float c = 0.f;
  for (int p = 0; p < s.P; ++p) {
    const float ap = s.ws[(long long)p * BD + e];
    const float yl = s.ws[((long long)s.P + p) * BD + e];
    s.ws[((long long)s.P + p) * BD + e] = c;  // carry-in of chunk p
    c = ap * c + yl;
  }
}

// Pass 3: rescan each chunk from its carry.
__global__ void __launch_bounds__(SCAN_THREADS) scan_chunk_apply_kernel(const ScanArgs s) {
  const long long g = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  const int p = blockIdx.y;
  const long long groups = (long long)s.B * (s.D / 4);
  if (g >= groups) return;
  const long long b = g / (s.D / 4), cg = g - b * (s.D / 4);
  const long long base = b * (long long)s.L * s.D + cg * 4;
  const int cl = (s.L + s.P - 1) / s.P;
  const int t0 = p * cl, t1 = min(s.L, t0 + cl);
  const long long BD = (long long)s.B * s.D;
  const float4 c = *reinterpret_cast<const float4*>(s.ws + ((long long)s.P + p) * BD + g * 4);
  scan_run(s.a, s.x, s.y, base, s.D, t0, max(t0, t1), c, nullptr);
}

// ParallelMLayer recurrence fused into one pass (gfn/layers/parallel.py:101-121):
//   A = sigmoid(zA), dt = softplus(zdt) * base_dt * 1.5^head, Bv = zB * dt,
//   v_t = A_t v_{t-1} + Bv_t,  x_t = x_{t-1} + v_t dt_t.
// zA | zdt | zB are the three D-wide slices of one [B*L, 3D] GEMM output
// (row stride 3D).  Reads 12 B and writes 8 B per element.
struct PScanArgs {
  const float* z;  // [B, L, 3D]
  float* x_seq;    // [B, L, D]
  float* v_seq;    // [B, L, D]
  int B, L, D, H;
  float base_dt;
};

__global__ void __launch_bounds__(SCAN_THREADS) parallel_layer_scan_kernel(const PScanArgs s) {
  const long long g = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  const long long groups = (long long)s.B * (s.D / 4);
  if (g >= groups) return;
  const long long b = g / (s.D / 4), cg = g - b * (s.D / 4);
  const int col = (int)cg * 4;
  const int hd = s.D / s.H;
  float hs[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    hs[u] = 1.f;  // 1.5^head, exact in float for every head count used
    for (int i = 0; i < (col + u) / hd; ++i) hs[u] *= 1.5f;
  }
  const long long zb = b * (long long)s.L * 3 * s.D + col;
  const long long ob = b * (long long)s.L * s.D + col;
  float v[4] = {0.f, 0.f, 0.f, 0.f}, x[4] = {0.f, 0.f, 0.f, 0.f};
  for (int t = 0; t < s.L; t += SCAN_UNROLL) {
    float4 za[SCAN_UNROLL], zd[SCAN_UNROLL], zbv[SCAN_UNROLL];
#pragma unroll
    for (int u = 0; u < SCAN_UNROLL; ++u) {
      if (t + u < s.L) {
        const float* zr = s.z + zb + (long long)(t + u) * 3 * s.D;
        za[u] = __ldcs(reinterpret_cast<const float4*>(zr));
        zd[u] = __ldcs(reinterpret_cast<const float4*>(zr + s.D));
        zbv[u] = __ldcs(reinterpret_cast<const float4*>(zr + 2 * s.D));
      }
    }
#pragma unroll
    for (int u = 0; u < SCAN_UNROLL; ++u) {
      if (t + u >= s.L) break;
      const float zaa[4] = {za[u].x, za[u].y, za[u].z, za[u].w};
      const float zdd[4] = {zd[u].x, zd[u].y, zd[u].z, zd[u].w};
      const float zbb[4] = {zbv[u].x, zbv[u].y, zbv[u].z, zbv[u].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float A = sigmoid_f(zaa[e]);
        const float dt = (softplus_f(zdd[e]) * s.base_dt) * hs[e];
        const float Bv = zbb[e] * dt;
        v[e] = A * v[e] + Bv;
        x[e] = x[e] + v[e] * dt;
      }
      const long long off = ob + (long long)(t + u) * s.D;
      __stcs(reinterpret_cast<float4*>(s.v_seq + off), make_float4(v[0], v[1], v[2], v[3]));
      __stcs(reinterpret_cast<float4*>(s.x_seq + off), make_float4(x[0], x[1], x[2], x[3]));
    }
  }
}

}  // namespace gfn
