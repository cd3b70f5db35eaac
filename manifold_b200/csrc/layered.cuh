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
#include <cuda_fp16.h>

#include "leapfrog_seq.cuh"

namespace gfn {

constexpr int LAY_THREADS = 256;

// Per-layer layered pack offsets (floats).  Per head: WfT [hd][hd], U
// [hd][r], W^T [r][hd], bf [hd] (each head block padded to 4); then softplus(dt) [H] (pad
// 4), bx, bv, gx, gv [d], then Wx, Wv [d][d] ([out][in], contiguous pair).
// Then the split-bf16 copy of the mixing weights WK [2][d][6d] (bf16): each
// fp32 weight w = w0 + w1 + w2 (three bf16 pieces, round to nearest), laid
// along K as [w0 w1 w0 w2 w1 w0] against the activations' [c0 c0 c1 c0 c1 c2],
// so one bf16 GEMM with K = 6d and fp32 accumulation sums the six products
// c_i w_j with i + j <= 2.  The dropped terms are below 2^-26 of |c w|.
// Then the split-fp16 copy WH [2][d][3d] (fp16): weights scaled by s (a power
// of two per layer), w s = w0 + w1 laid along K as [w0 w1 w0] against the
// activations' [c0 c0 c1]; then 4 floats: max|W|, s, 1/s, 0.
// Then, for the tensor-core head step, per head the friction weight W_f
// scaled by a power of two s_h and split into two fp16 pieces, each stored
// as the shared-memory image of a K-major [hd][hd] UMMA operand tile
// (hd * 2-byte rows, 16-byte units XOR-swizzled by row & 7): HU [H][2][hd][hd]
// fp16; then per head 2 floats (max|W_f|, 1/s_h), padded to 4.
struct LayOffsets {
  int head, hblock, sc, bx, bv, gx, gv;
  long long Wx, Wv, WK, WH, wsc, HU, HUs;
  long long total;
};
constexpr int LAY_SPLIT = 6;
constexpr int LAY_SPLIT_H = 3;

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
  o.WH = o.WK + (long long)LAY_SPLIT * d * d;     // after 2 * d * 6d bf16
  o.wsc = o.WH + (long long)LAY_SPLIT_H * d * d;  // after 2 * d * 3d fp16
  o.HU = o.wsc + 4;
  o.HUs = o.HU + (long long)H * hd * hd;          // after H * 2 * hd * hd fp16
  o.total = o.HUs + ((2 * H + 3) / 4) * 4;
  return o;
}

// Power-of-two weight scale putting max|W| s in [2^13, 2^14): the small fp16
// pieces of the scaled weights stay normal; 1 for an all-zero layer.
GFN_DEV float lay_weight_scale(float m) {
  if (!(m > 0.f)) return 1.f;
  int e;
  frexpf(m, &e);  // m = f 2^e, f in [0.5, 1)
  return ldexpf(1.f, 14 - e);
}

// max |Wx|, |Wv| of each layer into the pack's scale slot (non-negative
// floats order like their bit patterns, so an integer atomic max works).
// The slot is zeroed first.
__global__ void layered_absmax_kernel(const float* __restrict__ Wx, const float* __restrict__ Wv,
                                      float* out, int NL, int d, long long LF, long long wsc) {
  const long long n = (long long)d * d;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < 2 * NL * n;
       e += (long long)gridDim.x * blockDim.x) {
    const int which = (int)(e / (NL * n));
    const long long r = e - (long long)which * NL * n;
    const int l = (int)(r / n);
    const float w = fabsf((which == 0 ? Wx : Wv)[r]);
    if (w > 0.f)
      atomicMax(reinterpret_cast<unsigned*>(out + (long long)l * LF + wsc), __float_as_uint(w));
  }
}

// Byte offset of element (n, k) in the shared-memory image of a K-major
// fp16 operand tile whose rows are `rowbytes` (64 or 128) long, with the
// matching swizzle (the pattern the TMA engine writes and the UMMA
// descriptor reads): address bits [4, 7) are XORed with bits [7, 10), i.e.
// the 16-byte unit u of row n is stored at unit u ^ ((n * rowbytes / 128) mod units).
__host__ __device__ inline int umma_kmajor_xor(int n, int rowbytes) {
  return ((n * rowbytes) >> 7) & ((rowbytes >> 4) - 1);
}
__host__ __device__ inline int umma_kmajor_off(int n, int k, int rowbytes) {
  const int u = (k * 2) >> 4;  // 16-byte unit within the row
  return n * rowbytes + ((u ^ umma_kmajor_xor(n, rowbytes)) << 4) + ((k * 2) & 15);
}

// max |W_f| of every (layer, head) into the pack's HUs slots (zeroed first).
__global__ void layered_head_absmax_kernel(const float* __restrict__ Wf, float* out, int NL, int H,
                                           int hd, long long LF, long long HUs) {
  const int lh = blockIdx.x;  // layer * H + head
  if (lh >= NL * H) return;
  const int l = lh / H, h = lh - l * H;
  float m = 0.f;
  for (int i = threadIdx.x; i < hd * hd; i += blockDim.x) m = fmaxf(m, fabsf(Wf[(long long)lh * hd * hd + i]));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
  if ((threadIdx.x & 31) == 0 && m > 0.f)
    atomicMax(reinterpret_cast<unsigned*>(out + (long long)l * LF + HUs + 2 * h), __float_as_uint(m));
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
        const int t = q - hd * hd - hd * r, qq = t / hd, j = t - qq * hd;
        v = a.W[lh * hd * r + j * r + qq];  // transposed: [q][j]
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
    } else if (off >= o.HUs) {
      const int q = (int)(off - o.HUs);
      if (q >= 2 * a.H || (q & 1) == 0) {
        if (q >= 2 * a.H) a.out[e] = 0.f;
        continue;  // max|W_f| slots are written by layered_head_absmax_kernel
      }
      v = 1.f / lay_weight_scale(a.out[(long long)l * a.LF + o.HUs + (q - 1)]);
    } else if (off >= o.HU) {
      // two fp16 of HU per float slot; slot pair -> (head, piece, byte offset)
      const long long q = 2 * (off - o.HU);  // fp16 index within the section
      const int per_piece = hd * hd, per_head = 2 * per_piece;
      const int h = (int)(q / per_head);
      const int rem = (int)(q - (long long)h * per_head);
      const int piece = rem / per_piece;
      const int boff = (rem - piece * per_piece) * 2;  // byte offset inside the tile image
      const int rowbytes = hd * 2;
      const float s = lay_weight_scale(a.out[(long long)l * a.LF + o.HUs + 2 * h]);
      __half pr[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        // invert umma_kmajor_off: row n, swizzled unit, element within unit
        const int bo = boff + 2 * u;
        const int n = bo / rowbytes;
        const int wi = bo - n * rowbytes;
        const int k = (((wi >> 4) ^ umma_kmajor_xor(n, rowbytes)) << 3) + ((wi & 15) >> 1);
        const float w = a.Wf[(((long long)l * a.H + h) * hd + n) * hd + k] * s;  // W_f[n][k]
        const __half w0 = __float2half_rn(w);
        pr[u] = piece == 0 ? w0 : __float2half_rn(w - __half2float(w0));
      }
      v = __uint_as_float((unsigned)__half_as_ushort(pr[0]) | ((unsigned)__half_as_ushort(pr[1]) << 16));
    } else if (off >= o.wsc) {
      const int q = (int)(off - o.wsc);
      if (q == 0) continue;  // max|W|, written by layered_absmax_kernel
      const float s = lay_weight_scale(a.out[(long long)l * a.LF + o.wsc]);
      v = q == 1 ? s : q == 2 ? 1.f / s : 0.f;
    } else if (off >= o.WH) {
      // two fp16 of WH per float slot: [w0 w1 w0] of the scaled weight
      const float s = lay_weight_scale(a.out[(long long)l * a.LF + o.wsc]);
      const long long q = 2 * (off - o.WH);
      __half pr[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const long long qq = q + u;
        const long long rowk = (long long)LAY_SPLIT_H * d;
        const int which = (int)(qq / ((long long)d * rowk));
        const long long rem = qq - (long long)which * d * rowk;
        const int orow = (int)(rem / rowk), kk = (int)(rem - (long long)orow * rowk);
        const int seg = kk / d, col = kk - seg * d;
        const float w = (which == 0 ? a.Wx : a.Wv)[((long long)l * d + orow) * d + col] * s;
        const __half w0 = __float2half_rn(w);
        const __half w1 = __float2half_rn(w - __half2float(w0));
        pr[u] = seg == 1 ? w1 : w0;
      }
      v = __uint_as_float((unsigned)__half_as_ushort(pr[0]) | ((unsigned)__half_as_ushort(pr[1]) << 16));
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

// 1/sqrt(mean((z + b)^2) + eps) of one d-long row, by one warp (128-bit
// loads, d % 4 == 0); the same order of operations wherever it runs.
GFN_DEV float row_rms_factor(const float* __restrict__ zrow, const float* __restrict__ bias, int d,
                             int lane) {
  const float4* row = reinterpret_cast<const float4*>(zrow);
  const float4* bb = reinterpret_cast<const float4*>(bias);
  float s = 0.f;
  for (int j = lane; j < d / 4; j += 32) {
    const float4 u = row[j], c = __ldg(bb + j);
    const float a0 = u.x + c.x, a1 = u.y + c.y, a2 = u.z + c.z, a3 = u.w + c.w;
    s = fmaf(a0, a0, s);
    s = fmaf(a1, a1, s);
    s = fmaf(a2, a2, s);
    s = fmaf(a3, a3, s);
  }
  s = warp_sum(s);
  return 1.f / sqrtf(s * (1.f / (float)d) + 1.1920928955078125e-07f);
}

// Per-row RMSNorm factors of zx and zv (one warp per row).
__global__ void layered_rowstat_kernel(const float* __restrict__ z, const float* __restrict__ bx,
                                       const float* __restrict__ bv, float* __restrict__ stat,
                                       int B, int d) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= 2 * B) return;
  const int which = warp / B, b = warp - which * B;
  const float r = row_rms_factor(z + ((long long)which * B + b) * d, which == 0 ? bx : bv, d, lane);
  if (lane == 0) stat[which * B + b] = r;
}

struct LayPreArgs {
  // layer input: either the carried state (first layer of a token) ...
  const float* x_in;
  const float* v_in;
  long long in_stride;  // 0: one row broadcast
  // ... or the previous layer's mixing output z [2][B][d] with its params
  const float* z;
  const float* stat;    // [2][B], or NULL: the block computes its rows' factors
  const float* spart;   // or [2][nparts][B] partial sums of squares from the mixing GEMM
  int nparts;
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
  __half* catkh;        // [2][B][3d] split-fp16 head-step outputs, or NULL
  int B, d, H, hd;
  float base_dt;
  long long* prof;  // measurement only: per-CTA phase timestamps, or NULL
};

// Tile of the head-step kernel: TR rows of one head; thread (ty, tx) owns
// rows ty*RPT .. +RPT-1 and columns 4tx .. 4tx+3 of the head.
template <int HD, int TR_>
struct LayTile {
  static constexpr int TR = TR_;
  static constexpr int CG = HD / 4;             // column groups of 4
  static constexpr int RG = LAY_THREADS / CG;   // row groups
  static constexpr int RPT = TR / RG;           // rows per thread
  static_assert(RPT >= 1 && RG * RPT == TR && TR >= 16 && TR * 4 >= LAY_THREADS / 4,
                "tile shape");
};

// Transposed tile [HD][TR] with the 16-byte units of each column XOR-swizzled
// by the column's group of four: a thread's 4 consecutive columns land in
// distinct units, so its float4 row-group stores/loads take the minimum
// number of wavefronts, while the friction loop's reads (one column, a
// broadcast row group per half warp) stay conflict-free.
template <int TR>
GFN_DEV int tsw(int k, int r) {
  constexpr int UM = (TR / 4 < 8 ? TR / 4 : 8) - 1;
  return k * TR + ((((r >> 2) ^ ((k >> 2) & UM)) << 2) | (r & 3));
}

template <int N>
GFN_DEV void lds_rows(const float* p, float (&r)[N]) {
  if constexpr (N == 4) {
    const float4 t = *reinterpret_cast<const float4*>(p);
    r[0] = t.x; r[1] = t.y; r[2] = t.z; r[3] = t.w;
  } else if constexpr (N == 2) {
    const float2 t = *reinterpret_cast<const float2*>(p);
    r[0] = t.x; r[1] = t.y;
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) r[i] = p[i];
  }
}

template <int N>
GFN_DEV void sts_rows(float* p, const float (&r)[N]) {
  if constexpr (N == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(r[0], r[1], r[2], r[3]);
  } else if constexpr (N == 2) {
    *reinterpret_cast<float2*>(p) = make_float2(r[0], r[1]);
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) p[i] = r[i];
  }
}

GFN_DEV float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

// Gamma(v) for the thread's micro-tile, all in registers
// (gfn/geometry/lowrank.py:93-98,125-127): partial p = v . U over the
// thread's 4 columns, completed by a butterfly over the CG lanes that share
// the rows, then g = 20 tanh((p^2 / (1 + |p| + 1e-6)) . W^T / 20).
template <int RK, int HD, int TR>
GFN_DEV void tile_gamma(const float (&v)[LayTile<HD, TR>::RPT][4], const float* U,
                        const float* WgT, int c0, float (&g)[LayTile<HD, TR>::RPT][4]) {
  using T = LayTile<HD, TR>;
  constexpr int RPT = T::RPT;
  float p[RPT][RK];
#pragma unroll
  for (int i = 0; i < RPT; ++i)
#pragma unroll
    for (int q = 0; q < RK; ++q) p[i][q] = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int q4 = 0; q4 < RK; q4 += 4) {
      const float4 u = *reinterpret_cast<const float4*>(U + (c0 + j) * RK + q4);
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        p[i][q4 + 0] = fmaf(v[i][j], u.x, p[i][q4 + 0]);
        p[i][q4 + 1] = fmaf(v[i][j], u.y, p[i][q4 + 1]);
        p[i][q4 + 2] = fmaf(v[i][j], u.z, p[i][q4 + 2]);
        p[i][q4 + 3] = fmaf(v[i][j], u.w, p[i][q4 + 3]);
      }
    }
  }
#pragma unroll
  for (int m = 1; m < T::CG; m <<= 1)
#pragma unroll
    for (int i = 0; i < RPT; ++i)
#pragma unroll
      for (int q = 0; q < RK; ++q) p[i][q] += __shfl_xor_sync(0xffffffffu, p[i][q], m);
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    float ss = 0.f;
#pragma unroll
    for (int q = 0; q < RK; ++q) ss = fmaf(p[i][q], p[i][q], ss);
    const float sc = 1.f / ((1.f + sqrtf(ss)) + 1e-6f);
#pragma unroll
    for (int q = 0; q < RK; ++q) p[i][q] = (p[i][q] * p[i][q]) * sc;
  }
#pragma unroll
  for (int i = 0; i < RPT; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) g[i][j] = 0.f;
#pragma unroll
  for (int q = 0; q < RK; ++q) {
    const float4 w = *reinterpret_cast<const float4*>(WgT + q * HD + c0);
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      g[i][0] = fmaf(p[i][q], w.x, g[i][0]);
      g[i][1] = fmaf(p[i][q], w.y, g[i][1]);
      g[i][2] = fmaf(p[i][q], w.z, g[i][2]);
      g[i][3] = fmaf(p[i][q], w.w, g[i][3]);
    }
  }
#pragma unroll
  for (int i = 0; i < RPT; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) g[i][j] = soft_clamp20(g[i][j]);
}

// One implicit kick for the thread's micro-tile: friction mu = 5 sigma(x Wf^T
// + b_f) from the transposed x tile (a TR x HD x HD product in registers),
// then v_new = (v + h (F - Gamma(v))) / (1 + h mu)
// (gfn/integrators/symplectic/leapfrog.py:72-114).
template <int RK, int HD, int TR>
GFN_DEV void tile_kick(const float* xT, const float* WfT, const float* U, const float* WgT,
                       const float* bfh, int r0, int c0, float hh,
                       const float (&F)[LayTile<HD, TR>::RPT][4],
                       const float (&v)[LayTile<HD, TR>::RPT][4],
                       float (&vn)[LayTile<HD, TR>::RPT][4]) {
  using T = LayTile<HD, TR>;
  constexpr int RPT = T::RPT;
  constexpr int UM = (TR / 4 < 8 ? TR / 4 : 8) - 1;
  float g[RPT][4];
  tile_gamma<RK, HD, TR>(v, U, WgT, c0, g);
  int offs[UM + 1];  // swizzled offset of the thread's row group, per column group
#pragma unroll
  for (int u = 0; u <= UM; ++u) offs[u] = (((r0 >> 2) ^ u) << 2) | (r0 & 3);
  float acc[RPT][4];
#pragma unroll
  for (int i = 0; i < RPT; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  constexpr int KG = 4 * (UM + 1) < HD ? 4 * (UM + 1) : HD;  // one swizzle period
#pragma unroll 1
  for (int kb = 0; kb < HD; kb += KG) {
#pragma unroll
    for (int u = 0; u < KG; ++u) {
      const int k = kb + u;
      const float4 w = *reinterpret_cast<const float4*>(WfT + k * HD + c0);
      float xr[RPT];
      lds_rows<RPT>(xT + k * TR + offs[(u >> 2) & UM], xr);
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        acc[i][0] = fmaf(xr[i], w.x, acc[i][0]);
        acc[i][1] = fmaf(xr[i], w.y, acc[i][1]);
        acc[i][2] = fmaf(xr[i], w.z, acc[i][2]);
        acc[i][3] = fmaf(xr[i], w.w, acc[i][3]);
      }
    }
  }
  const float4 b4 = *reinterpret_cast<const float4*>(bfh + c0);
  const float bj[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
  for (int i = 0; i < RPT; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float mu = sigmoid_f(acc[i][j] + bj[j]) * 5.f;
      vn[i][j] = (v[i][j] + hh * (F[i][j] - g[i][j])) / (1.f + hh * mu);
    }
}

GFN_DEV void store_split6(__nv_bfloat16* row, int d, const float (&c)[4]) {
  // [c0 c0 c1 c0 c1 c2] per column, 4 columns per 8-byte store
  __nv_bfloat16 p0[4], p1[4], p2[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    p0[j] = __float2bfloat16_rn(c[j]);
    const float r1 = c[j] - __bfloat162float(p0[j]);
    p1[j] = __float2bfloat16_rn(r1);
    p2[j] = __float2bfloat16_rn(r1 - __bfloat162float(p1[j]));
  }
  auto pack4 = [](const __nv_bfloat16 (&q)[4]) {
    uint2 u;
    u.x = (unsigned)__bfloat16_as_ushort(q[0]) | ((unsigned)__bfloat16_as_ushort(q[1]) << 16);
    u.y = (unsigned)__bfloat16_as_ushort(q[2]) | ((unsigned)__bfloat16_as_ushort(q[3]) << 16);
    return u;
  };
  const uint2 u0 = pack4(p0), u1 = pack4(p1), u2 = pack4(p2);
  *reinterpret_cast<uint2*>(row) = u0;
  *reinterpret_cast<uint2*>(row + d) = u0;
  *reinterpret_cast<uint2*>(row + 2 * d) = u1;
  *reinterpret_cast<uint2*>(row + 3 * d) = u0;
  *reinterpret_cast<uint2*>(row + 4 * d) = u1;
  *reinterpret_cast<uint2*>(row + 5 * d) = u2;
}

GFN_DEV void store_split3h(__half* row, int d, const float (&c)[4]) {
  // [c0 c0 c1] per column, 4 columns per 8-byte store; |c| >= 2^15 is flagged
  __half p0[4], p1[4];
  bool bad = false;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    bad |= !(fabsf(c[j]) < 32768.f);
    p0[j] = __float2half_rn(c[j]);
    p1[j] = __float2half_rn(c[j] - __half2float(p0[j]));
  }
  if (bad) gfn_flag_error(kDevErrF16Range);
  uint2 u0, u1;
  u0.x = (unsigned)__half_as_ushort(p0[0]) | ((unsigned)__half_as_ushort(p0[1]) << 16);
  u0.y = (unsigned)__half_as_ushort(p0[2]) | ((unsigned)__half_as_ushort(p0[3]) << 16);
  u1.x = (unsigned)__half_as_ushort(p1[0]) | ((unsigned)__half_as_ushort(p1[1]) << 16);
  u1.y = (unsigned)__half_as_ushort(p1[2]) | ((unsigned)__half_as_ushort(p1[3]) << 16);
  *reinterpret_cast<uint2*>(row) = u0;
  *reinterpret_cast<uint2*>(row + d) = u0;
  *reinterpret_cast<uint2*>(row + 2 * d) = u1;
}

// Head step of one layer for TR rows of one head (grid: row tiles x heads).
// Input: the carried state (first layer of a token) or the previous layer's
// mixing output with its RMSNorm / saturation applied on load.  Output: the
// concat (x', v') as fp32 (cat) or split bf16 (catk).
template <int RK, int HD, int TR>
__global__ void __launch_bounds__(LAY_THREADS, (TR * HD <= 2048 && RK <= 8) ? 3 : 2) layered_pre_kernel(const LayPreArgs a) {
  using T = LayTile<HD, TR>;
  constexpr int RPT = T::RPT;
  extern __shared__ __align__(16) float hsm[];
  const int d = a.d, B = a.B, h = blockIdx.y;
  const LayOffsets o = lay_offsets(a.H, HD, RK, d);
  {
    const float* src = a.lay + (long long)h * o.hblock;
    for (int i = threadIdx.x * 4; i < o.hblock; i += LAY_THREADS * 4)
      *reinterpret_cast<float4*>(hsm + i) = ldg4(src + i);
  }
  const float* WfT = hsm;
  const float* U = hsm + HD * HD;
  const float* WgT = U + HD * RK;
  const float* bfh = WgT + HD * RK;
  float* xT = hsm + o.hblock;
  float* sstat = xT + HD * TR;  // [2][TR] RMSNorm factors when computed here
  if (a.z && !a.stat && a.spart) {
    for (int q = threadIdx.x; q < 2 * TR; q += LAY_THREADS) {
      const int which = q / TR, r = q - which * TR, b = blockIdx.x * TR + r;
      float f = 0.f;
      if (b < B) {
        float s = 0.f;
        for (int p = 0; p < a.nparts; ++p) s += a.spart[((long long)which * a.nparts + p) * B + b];
        f = 1.f / sqrtf(s * (1.f / (float)d) + 1.1920928955078125e-07f);
      }
      sstat[q] = f;
    }
    __syncthreads();
  } else if (a.z && !a.stat) {
    const int w = threadIdx.x >> 5, ln = threadIdx.x & 31;
    for (int q = w; q < 2 * TR; q += LAY_THREADS / 32) {
      const int which = q / TR, r = q - which * TR, b = blockIdx.x * TR + r;
      float f = 0.f;
      if (b < B)
        f = row_rms_factor(a.z + ((long long)which * B + b) * d, a.prev + (which ? o.bv : o.bx), d, ln);
      if (ln == 0) sstat[q] = f;
    }
    __syncthreads();
  }
  const int tx = threadIdx.x % T::CG, ty = threadIdx.x / T::CG;
  const int c0 = 4 * tx, r0 = ty * RPT;
  const int gc = h * HD + c0;
  const int row0 = blockIdx.x * T::TR;
  const float eff = a.base_dt * a.lay[o.sc + h];
  const float hh = 0.5f * eff;

  float F[RPT][4], X[RPT][4], V[RPT][4];
  float xc[4][RPT];  // the thread's x tile, column-major for the stores
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int b = row0 + r0 + i;
    float xv[4] = {0.f, 0.f, 0.f, 0.f}, vv[4] = {0.f, 0.f, 0.f, 0.f};
    F[i][0] = F[i][1] = F[i][2] = F[i][3] = 0.f;
    if (b < B) {
      if (a.z) {
        const float rx = a.stat ? a.stat[b] : sstat[r0 + i];
        const float rv = a.stat ? a.stat[B + b] : sstat[TR + r0 + i];
        const float4 zx = ldg4(a.z + (long long)b * d + gc);
        const float4 zv = ldg4(a.z + ((long long)B + b) * d + gc);
        const float4 bx = ldg4(a.prev + o.bx + gc), bv = ldg4(a.prev + o.bv + gc);
        const float4 gx = ldg4(a.prev + o.gx + gc), gv = ldg4(a.prev + o.gv + gc);
        xv[0] = ((zx.x + bx.x) * rx) * gx.x; xv[1] = ((zx.y + bx.y) * rx) * gx.y;
        xv[2] = ((zx.z + bx.z) * rx) * gx.z; xv[3] = ((zx.w + bx.w) * rx) * gx.w;
        vv[0] = saturate100(((zv.x + bv.x) * rv) * gv.x);
        vv[1] = saturate100(((zv.y + bv.y) * rv) * gv.y);
        vv[2] = saturate100(((zv.z + bv.z) * rv) * gv.z);
        vv[3] = saturate100(((zv.w + bv.w) * rv) * gv.w);
      } else {
        const float4 x4 = ldg4(a.x_in + (long long)b * a.in_stride + gc);
        const float4 v4 = ldg4(a.v_in + (long long)b * a.in_stride + gc);
        xv[0] = x4.x; xv[1] = x4.y; xv[2] = x4.z; xv[3] = x4.w;
        vv[0] = v4.x; vv[1] = v4.y; vv[2] = v4.z; vv[3] = v4.w;
      }
      const long long idx = (long long)b * a.L + a.t;
      float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
      if (a.f32) {
        f = ldg4(a.f32 + idx * d + gc);
      } else if (a.fbf16) {
        const uint2 u = __ldg(reinterpret_cast<const uint2*>(a.fbf16 + idx * d + gc));
        f.x = __uint_as_float(u.x << 16); f.y = __uint_as_float(u.x & 0xffff0000u);
        f.z = __uint_as_float(u.y << 16); f.w = __uint_as_float(u.y & 0xffff0000u);
      } else {
        const long long id = a.ids[idx];
        if (id < 0 || id >= a.vocab) {
          if (tx == 0) gfn_flag_error(kDevErrBadToken);
        } else {
          f = ldg4(a.table + id * d + gc);
        }
      }
      if (a.mask) {
        const float m = a.mask[idx];
        f.x *= m; f.y *= m; f.z *= m; f.w *= m;
      }
      F[i][0] = f.x; F[i][1] = f.y; F[i][2] = f.z; F[i][3] = f.w;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      xc[j][i] = X[i][j] = xv[j];
      V[i][j] = vv[j];
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) sts_rows<RPT>(xT + tsw<T::TR>(c0 + j, r0), xc[j]);
  __syncthreads();
  // kick 1 at x, drift, kick 2 at x' (one loop body: one copy of the kick code)
#pragma unroll 1
  for (int kick = 0; kick < 2; ++kick) {
    float vn[RPT][4];
    tile_kick<RK, HD, TR>(xT, WfT, U, WgT, bfh, r0, c0, hh, F, V, vn);
#pragma unroll
    for (int i = 0; i < RPT; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) V[i][j] = vn[i][j];
    if (kick == 0) {
#pragma unroll
      for (int i = 0; i < RPT; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) X[i][j] = X[i][j] + eff * V[i][j];
      __syncthreads();
#pragma unroll
      for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int i = 0; i < RPT; ++i) xc[j][i] = X[i][j];
        sts_rows<RPT>(xT + tsw<T::TR>(c0 + j, r0), xc[j]);
      }
      __syncthreads();
    }
  }
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int b = row0 + r0 + i;
    if (b >= B) continue;
    if (a.cat) {
      *reinterpret_cast<float4*>(a.cat + (long long)b * d + gc) =
          make_float4(X[i][0], X[i][1], X[i][2], X[i][3]);
      *reinterpret_cast<float4*>(a.cat + ((long long)B + b) * d + gc) =
          make_float4(V[i][0], V[i][1], V[i][2], V[i][3]);
    }
    if (a.catk) {
      store_split6(a.catk + (long long)b * (LAY_SPLIT * d) + gc, d, X[i]);
      store_split6(a.catk + ((long long)B + b) * (LAY_SPLIT * d) + gc, d, V[i]);
    }
    if (a.catkh) {
      store_split3h(a.catkh + (long long)b * (LAY_SPLIT_H * d) + gc, d, X[i]);
      store_split3h(a.catkh + ((long long)B + b) * (LAY_SPLIT_H * d) + gc, d, V[i]);
    }
  }
}

template <int RK, int HD, int TR>
constexpr size_t layered_pre_smem(int hblock) {
  return ((size_t)hblock + HD * TR + 2 * TR) * 4;
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
