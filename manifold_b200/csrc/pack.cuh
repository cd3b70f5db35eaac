// Packs the reference's stacked layer parameters into the per-(layer, CTA)
// streaming layout read by leapfrog_seq_kernel:
//   [head section: WfT | U | W | bf | bx | bv | gx | gv | softplus(dt_params) | pad]
//   [mixing chunk 0 .. nchunk-1: each [KC][2C + 4], k-major, x columns then v, 4 pad]
// so that every piece a CTA needs for one layer step is a contiguous run
// that one bulk copy moves into shared memory.
#pragma once
#include "leapfrog_seq.cuh"

namespace gfn {

struct PackArgs {
  const float* U;    // [NL*H, hd, r]
  const float* W;    // [NL*H, hd, r]
  const float* Wf;   // [NL*H, hd, hd]  ([out, in])
  const float* bf;   // [NL*H, hd]
  const float* dtp;  // [NL*H] raw dt_params (softplus applied here)
  const float* Wx;   // [NL, d, d] or null (heads == 1)
  const float* bx;   // [NL, d]
  const float* gx;   // [NL, d]
  const float* Wv;
  const float* bv;
  const float* gv;
  float* out;
  int NL, d, H, hd, r, K, C, hpc, KC, nchunk, HS, CF;
  long long LF;
  // Training layout (train != 0): after the head section, the forget-gate
  // weight untransposed [hpc][j][k] (padded to HST floats in total), then the
  // nchunk forward chunks, then nchunk transposed chunks: element [kk][n] of
  // transposed chunk i is Wx[i*KC + kk][c*C + n] (v columns after x), the
  // operand of dx_cat = Wx^T dz for this CTA's input columns.
  int train, HST;
};

__global__ void pack_kernel(const PackArgs a) {
  const long long total = (long long)a.NL * a.K * a.LF;
  const HeadOffsets ho = head_offsets(a.hpc, a.hd, a.r, a.C);
  const int hd = a.hd, r = a.r, C = a.C, d = a.d;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const long long per_layer = (long long)a.K * a.LF;
    const int l = (int)(e / per_layer);
    const long long rem = e - l * per_layer;
    const int c = (int)(rem / a.LF);
    const long long off = rem - (long long)c * a.LF;
    float val = 0.f;
    const int chunk_base = a.train ? a.HST : a.HS;
    if (a.train && off >= a.HS && off < a.HST) {
      const int o2 = (int)(off - a.HS);
      if (o2 < a.hpc * hd * hd) {
        const int hl = o2 / (hd * hd), r2 = o2 - hl * hd * hd;
        val = a.Wf[((long long)l * a.H + c * a.hpc + hl) * hd * hd + r2];
      }
    } else if (off < a.HS) {
      const int o = (int)off;
      if (o < ho.U) {
        const int hl = o / (hd * hd), r2 = o - hl * hd * hd, k = r2 / hd, jj = r2 - k * hd;
        const int h = c * a.hpc + hl;
        val = a.Wf[(((long long)l * a.H + h) * hd + jj) * hd + k];
      } else if (o < ho.W) {
        const int o2 = o - ho.U, hl = o2 / (hd * r), r2 = o2 - hl * hd * r;
        val = a.U[((long long)l * a.H + c * a.hpc + hl) * hd * r + r2];
      } else if (o < ho.bf) {
        const int o2 = o - ho.W, hl = o2 / (hd * r), r2 = o2 - hl * hd * r;
        val = a.W[((long long)l * a.H + c * a.hpc + hl) * hd * r + r2];
      } else if (o < ho.bx) {
        const int j = o - ho.bf;
        val = a.bf[((long long)l * a.H) * hd + (long long)c * C + j];
      } else if (o < ho.sc) {
        const int which = (o - ho.bx) / C, j = (o - ho.bx) - which * C;
        const float* src = which == 0 ? a.bx : which == 1 ? a.bv : which == 2 ? a.gx : a.gv;
        val = src ? src[(long long)l * d + (long long)c * C + j] : (which >= 2 ? 1.f : 0.f);
      } else if (o < ho.sc + a.hpc) {
        val = softplus_f(a.dtp[(long long)l * a.H + c * a.hpc + (o - ho.sc)]);
      }
    } else {
      const long long o2 = off - chunk_base;
      int i = (int)(o2 / a.CF);
      const bool transposed = i >= a.nchunk;
      if (transposed) i -= a.nchunk;
      const int e2 = (int)(o2 - (long long)(transposed ? i + a.nchunk : i) * a.CF);
      const int CS = chunk_row_stride(C);
      const int kk = e2 / CS, np = e2 - kk * CS;
      // stored unit np/4 holds logical unit (np/4) ^ ((kk/4) & mask) (the pad unit is not permuted)
      const int n = np < 2 * C ? ((((np >> 2) ^ ((kk >> 2) & chunk_swizzle_mask(C)))) << 2) + (np & 3) : np;
      const int k = i * a.KC + kk;
      if (k < d && n < 2 * C && transposed) {
        if (n < C)
          val = a.Wx[((long long)l * d + k) * d + (long long)c * C + n];
        else
          val = a.Wv[((long long)l * d + k) * d + (long long)c * C + n - C];
      } else if (k < d && n < 2 * C) {
        if (n < C)
          val = a.Wx[((long long)l * d + (long long)c * C + n) * d + k];
        else
          val = a.Wv[((long long)l * d + (long long)c * C + n - C) * d + k];
      }
    }
    a.out[e] = val;
  }
}

}  // namespace gfn
