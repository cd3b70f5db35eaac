// Layer-by-layer leapfrog recurrence for large batches.
//
// Same arithmetic as leapfrog_seq_kernel (gfn/layers/base.py:198-338 per
// layer, gfn/model.py:377-402 per token), organised for throughput when the
// batch makes the head mixing a real GEMM ([B x d] . [d x d], e.g. 4096 decode
// streams at d = 1024): per layer
//   rowstat : per-row RMSNorm factors of the previous layer's mixing output
//   pre     : previous layer's RMSNorm + saturation, then the leapfrog head
//             step for one head on a block of rows (the head's weights staged
//             once in shared memory), writing the concat (x', v')
//   mixing  : one batched fp32 GEMM for x and v (cuBLAS, no TF32)
// and after the last layer `finalize` applies the last RMSNorm/saturation and
// writes x_seq / v_seq and the carried state.
#pragma once
#include "leapfrog_seq.cuh"

namespace gfn {

constexpr int LAY_THREADS = 256;
constexpr int LAY_ROWS = 32;  // rows per pre-kernel block

// Per-layer layered pack offsets (floats).  Per head: WfT [hd][hd], U, W
// [hd][r], bf [hd] (each head block padded to 4); then softplus(dt) [H] (pad
// 4), bx, bv, gx, gv [d], then Wx, Wv [d][d] ([out][in], contiguous pair).
// Then the split-bf16 copy of the mixing weights WK [2][d][6d] (bf16): each
// fp32 weight w = w0 + w1 + w2 (three bf16 pieces, round to nearest), laid
// along K as [w0 w1 w0 w2 w1 w0] against the activations' [c0 c0 c1 c0 c1 c2],
// so one bf16 GEMM with K = 6d and fp32 accumulation sums the six products
// c_i w_j with i + j <= 2.  The dropped terms are below 2^-26 of |c w|.
struct LayOffsets {
  int head, hblock, sc, bx, bv, gx, gv;
  long long Wx, Wv, WK;
  long long total;
};
constexpr int LAY_SPLIT = 6;

__host__ __device__ inline LayOffsets lay_offsets(int H, int hd, int r, int d) {
  LayOffsets o;
  o.head = 0;
  o.hblock = ((hd * hd + 2 * hd * r + hd + 3) / 4) * 4;
  o.sc = H * o.hblock;
  o.bx = o.sc + ((H + 3) / 4) * 4;
  o.bv = o.bx + d;
  o.gx = o.bv + d;
  o.gv = o.gx + d;
  o.Wx = o.gv + d;
  o.Wv = o.Wx + (long long)d * d;
  o.WK = o.Wv + (long long)d * d;
  o.total = o.WK + (long long)LAY_SPLIT * d * d;  // 2 * d * 6d bf16
  return o;
}

struct LayPackArgs {
  const float *U, *W, *Wf, *bf, *dtp, *Wx, *bx, *gx, *Wv, *bv, *gv;
  float* out;
  int NL, d, H, hd, r;
  long long LF;
};

__global__ void layered_pack_kernel(const LayPackArgs a) {
  const LayOffsets o = lay_offsets(a.H, a.hd, a.r, a.d);
  const long long total = (long long)a.NL * a.LF;
  const int hd = a.hd, r = a.r, d = a.d;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const int l = (int)(e / a.LF);
    const long long off = e - (long long)l * a.LF;
    float v = 0.f;
    if (off < o.sc) {
      const int h = (int)(off / o.hblock), q = (int)(off - (long long)h * o.hblock);
      const long long lh = (long long)l * a.H + h;
      if (q < hd * hd) {
        const int k = q / hd, j = q - k * hd;
        v = a.Wf[(lh * hd + j) * hd + k];  // transposed: [k][j]
      } else if (q < hd * hd + hd * r) {
        v = a.U[lh * hd * r + (q - hd * hd)];
      } else if (q < hd * hd + 2 * hd * r) {
        v = a.W[lh * hd * r + (q - hd * hd - hd * r)];
      } else if (q < hd * hd + 2 * hd * r + hd) {
        v = a.bf[lh * hd + (q - hd * hd - 2 * hd * r)];
      }
    } else if (off < o.bx) {
      const int h = (int)(off - o.sc);
      if (h < a.H) v = softplus_f(a.dtp[(long long)l * a.H + h]);
    } else if (off < o.Wx) {
      const int which = (int)((off - o.bx) / d), j = (int)((off - o.bx) % d);
      const float* src = which == 0 ? a.bx : which == 1 ? a.bv : which == 2 ? a.gx : a.gv;
      v = src[(long long)l * d + j];
    } else if (off < o.Wv) {
      v = a.Wx[(long long)l * d * d + (off - o.Wx)];
    } else if (off < o.WK) {
      v = a.Wv[(long long)l * d * d + (off - o.Wv)];
    } else {
      // two bf16 of WK per float slot
      const long long q = 2 * (off - o.WK);
      __nv_bfloat16 pr[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const long long qq = q + u;
        const long long rowk = (long long)LAY_SPLIT * d;
        const int which = (int)(qq / ((long long)d * rowk));
        const long long rem = qq - (long long)which * d * rowk;
        const int orow = (int)(rem / rowk), kk = (int)(rem - (long long)orow * rowk);
        const int seg = kk / d, col = kk - seg * d;
        const float w = (which == 0 ? a.Wx : a.Wv)[((long long)l * d + orow) * d + col];
        const __nv_bfloat16 w0 = __float2bfloat16_rn(w);
        const float r1 = w - __bfloat162float(w0);
        const __nv_bfloat16 w1 = __float2bfloat16_rn(r1);
        const __nv_bfloat16 w2 = __float2bfloat16_rn(r1 - __bfloat162float(w1));
        // [w0 w1 w0 w2 w1 w0]
        pr[u] = seg == 1 || seg == 4 ? w1 : seg == 3 ? w2 : w0;
      }
      v = __uint_as_float((unsigned)__bfloat16_as_ushort(pr[0]) |
                          ((unsigned)__bfloat16_as_ushort(pr[1]) << 16));
    }
    a.out[e] = v;
  }
}

// Per-row RMSNorm factor 1/sqrt(mean((z + b)^2) + eps) of zx and zv.
__global__ void layered_rowstat_kernel(const float* __restrict__ z, const float* __restrict__ bx,
                                       const float* __restrict__ bv, float* __restrict__ stat,
                                       int B, int d) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= 2 * B) return;
  const int which = warp / B, b = warp - which * B;
  const float* row = z + ((long long)which * B + b) * d;
  const float* bias = which == 0 ? bx : bv;
  float s = 0.f;
  for (int j = lane; j < d; j += 32) {
    const float u = row[j] + bias[j];
    s = fmaf(u, u, s);
  }
  s = warp_sum(s);
  if (lane == 0) stat[which * B + b] = 1.f / sqrtf(s * (1.f / (float)d) + 1.1920928955078125e-07f);
}

struct LayPreArgs {
  // layer input: either the carried state (first layer of a token) ...
  const float* x_in;
  const float* v_in;
  long long in_stride;  // 0: one row broadcast
  // ... or the previous layer's mixing output z [2][B][d] with its params
  const float* z;
  const float* stat;    // [2][B]
  const float* prev;    // previous layer's pack run (bias / norm gains)
  // force of token t
  const float* f32;
  const __nv_bfloat16* fbf16;
  const long long* ids;
  const float* table;
  long long vocab;
  const float* mask;
  int t, L;
  const float* lay;     // this layer's pack run
  float* cat;           // [2][B][d] head-step outputs (x', v'), or NULL
  __nv_bfloat16* catk;  // [2][B][6d] split-bf16 head-step outputs, or NULL
  int B, d, H, hd;
  float base_dt;
};

template <int RK, int EPL>
__global__ void __launch_bounds__(LAY_THREADS, EPL >= 4 ? 2 : 4) layered_pre_kernel(const LayPreArgs a) {
  extern __shared__ __align__(16) float hsm[];  // this head's WfT | U | W | bf
  const int hd = a.hd, d = a.d, B = a.B;
  const int h = blockIdx.y;
  const LayOffsets o = lay_offsets(a.H, hd, RK, d);
  const float* src = a.lay + h * o.hblock;
  for (int i = threadIdx.x; i < o.hblock; i += blockDim.x) hsm[i] = src[i];
  __syncthreads();
  const float* WfT = hsm;
  const float* U = hsm + hd * hd;
  const float* Wg = U + hd * RK;
  const float* bfh = Wg + hd * RK;
  const float eff = a.base_dt * a.lay[o.sc + h];
  const float hh = 0.5f * eff;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int jj[EPL];
  bool eok[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    jj[e] = lane + 32 * e;
    eok[e] = jj[e] < hd;
    if (!eok[e]) jj[e] = hd - 1;
  }
  const LayOffsets po = lay_offsets(a.H, hd, RK, d);
  const int rend = min(B, (int)(blockIdx.x + 1) * LAY_ROWS);
  for (int b = blockIdx.x * LAY_ROWS + warp; b < rend; b += LAY_THREADS / 32) {
    float x[EPL], v[EPL], F[EPL];
    const long long idx = (long long)b * a.L + a.t;
    long long id = 0;
    if (a.ids) {
      id = a.ids[idx];
      if (id < 0 || id >= a.vocab) {
        if (lane == 0) gfn_flag_error(kDevErrBadToken);
        id = -1;
      }
    }
    const float m = a.mask ? a.mask[idx] : 1.f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const int col = h * hd + jj[e];
      if (a.z) {
        const float rx = a.stat[b], rv = a.stat[B + b];
        const float zx = a.z[(long long)b * d + col] + a.prev[po.bx + col];
        const float zv = a.z[((long long)B + b) * d + col] + a.prev[po.bv + col];
        x[e] = (zx * rx) * a.prev[po.gx + col];
        v[e] = saturate100((zv * rv) * a.prev[po.gv + col]);
      } else {
        x[e] = a.x_in[(long long)b * a.in_stride + col];
        v[e] = a.v_in[(long long)b * a.in_stride + col];
      }
      float f;
      if (a.f32) f = a.f32[idx * d + col];
      else if (a.fbf16) f = __bfloat162float(a.fbf16[idx * d + col]);
      else f = id < 0 ? 0.f : a.table[id * d + col];
      F[e] = a.mask ? f * m : f;
    }
    float gm[EPL], mu[EPL];
    unit_gamma<RK, EPL>(v, U, Wg, eok, jj, gm);
    unit_friction<EPL>(x, WfT, bfh, hd, jj, mu);
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const float vh = (v[e] + hh * (F[e] - gm[e])) / (1.f + hh * mu[e]);
      x[e] = x[e] + eff * vh;
      v[e] = vh;
    }
    unit_gamma<RK, EPL>(v, U, Wg, eok, jj, gm);
    unit_friction<EPL>(x, WfT, bfh, hd, jj, mu);
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      v[e] = (v[e] + hh * (F[e] - gm[e])) / (1.f + hh * mu[e]);
      if (eok[e]) {
        const int col = h * hd + jj[e];
        if (a.cat) {
          a.cat[(long long)b * d + col] = x[e];
          a.cat[((long long)B + b) * d + col] = v[e];
        }
        if (a.catk) {
#pragma unroll
          for (int w = 0; w < 2; ++w) {
            const float c = w == 0 ? x[e] : v[e];
            const __nv_bfloat16 c0 = __float2bfloat16_rn(c);
            const float r1 = c - __bfloat162float(c0);
            const __nv_bfloat16 c1 = __float2bfloat16_rn(r1);
            const __nv_bfloat16 c2 = __float2bfloat16_rn(r1 - __bfloat162float(c1));
            __nv_bfloat16* row = a.catk + ((long long)w * B + b) * (LAY_SPLIT * d) + col;
            // [c0 c0 c1 c0 c1 c2]
            row[0] = c0; row[d] = c0; row[2 * d] = c1;
            row[3 * d] = c0; row[4 * d] = c1; row[5 * d] = c2;
          }
        }
      }
    }
  }
}

// Last layer's RMSNorm + saturation -> x_seq[:, t], v_seq[:, t] and the state.
__global__ void layered_finalize_kernel(const float* __restrict__ z, const float* __restrict__ stat,
                                        const float* __restrict__ lay, int H, int hd, int r, int B,
                                        int d, int L, int t, float* x_seq, float* v_seq,
                                        float* xs, float* vs) {
  const LayOffsets o = lay_offsets(H, hd, r, d);
  const long long n = (long long)B * d;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n;
       e += (long long)gridDim.x * blockDim.x) {
    const int b = (int)(e / d), col = (int)(e - (long long)b * d);
    const float zx = z[e] + lay[o.bx + col];
    const float zv = z[n + e] + lay[o.bv + col];
    const float x = (zx * stat[b]) * lay[o.gx + col];
    const float v = saturate100((zv * stat[B + b]) * lay[o.gv + col]);
    xs[e] = x;
    vs[e] = v;
    const long long so = ((long long)b * L + t) * d + col;
    if (x_seq) x_seq[so] = x;
    if (v_seq) v_seq[so] = v;
  }
}

}  // namespace gfn
