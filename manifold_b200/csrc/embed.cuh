// FunctionalEmbedding (mode 'binary') forward: token id -> force vector.
// gfn/embeddings.py:171-206 (bits -> {-1,1} coords -> 3 SIREN layers
// sin(omega_0 (h W^T + b)) -> out_proj -> * impulse_scale -> 0 for id 0),
// SineLayer gfn/embeddings.py:24-49.
//
// All [B, L] tokens are independent, so this runs ahead of the recurrence
// as one launch.  A block embeds 32 tokens: the three 64-wide SIREN layers
// run out of shared memory, then each thread keeps one out_proj row (64
// floats) in registers and emits that column for all 32 tokens, writing
// float32 or bfloat16 forces.
#pragma once
#include "common.cuh"

namespace gfn {

constexpr int EMB_THREADS = 256;
constexpr int EMB_TOK = 32;
constexpr int EMB_HID = 64;
constexpr int EMB_COORD = 16;

struct EmbArgs {
  const long long* ids;
  long long n;  // number of tokens
  const float *W0, *b0, *W1, *b1, *W2, *b2;  // [64,16],[64],[64,64],[64],[64,64],[64]
  const float *Wo, *bo;                      // [d, 64], [d]
  const float* impulse;                      // scalar (device)
  float omega0;
  int d;
  float* out_f32;
  __nv_bfloat16* out_bf16;
};

__global__ void __launch_bounds__(EMB_THREADS) siren_embed_kernel(const EmbArgs a) {
  __shared__ float sW0[EMB_HID * EMB_COORD], sb0[EMB_HID];
  __shared__ float sW1[EMB_HID * EMB_HID], sb1[EMB_HID];
  __shared__ float sb2[EMB_HID];
  __shared__ float hA[EMB_TOK][EMB_HID + 1], hB[EMB_TOK][EMB_HID + 1];
  __shared__ float coords[EMB_TOK][EMB_COORD + 1];
  __shared__ float active[EMB_TOK];
  const int tid = threadIdx.x;
  for (int i = tid; i < EMB_HID * EMB_COORD; i += EMB_THREADS) sW0[i] = a.W0[i];
  for (int i = tid; i < EMB_HID * EMB_HID; i += EMB_THREADS) {
    sW1[i] = a.W1[i];
  }
  for (int i = tid; i < EMB_HID; i += EMB_THREADS) {
    sb0[i] = a.b0[i];
    sb1[i] = a.b1[i];
    sb2[i] = a.b2[i];
  }
  const long long tok0 = (long long)blockIdx.x * EMB_TOK;
  for (int i = tid; i < EMB_TOK * EMB_COORD; i += EMB_THREADS) {
    const int t = i / EMB_COORD, bit = i - t * EMB_COORD;
    const long long id = (tok0 + t < a.n) ? a.ids[tok0 + t] : 0;
    coords[t][bit] = ((id >> bit) & 1) ? 1.f : -1.f;
  }
  if (tid < EMB_TOK) {
    const long long id = (tok0 + tid < a.n) ? a.ids[tok0 + tid] : 0;
    active[tid] = (id & ((1ll << EMB_COORD) - 1)) != 0 ? 1.f : 0.f;
  }
  __syncthreads();
  // layer 0: 16 -> 64
  for (int i = tid; i < EMB_TOK * EMB_HID; i += EMB_THREADS) {
    const int t = i / EMB_HID, n = i - t * EMB_HID;
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < EMB_COORD; ++k) s = fmaf(coords[t][k], sW0[n * EMB_COORD + k], s);
    hA[t][n] = sinf(a.omega0 * (s + sb0[n]));
  }
  __syncthreads();
  for (int i = tid; i < EMB_TOK * EMB_HID; i += EMB_THREADS) {
    const int t = i / EMB_HID, n = i - t * EMB_HID;
    float s = 0.f;
#pragma unroll 16
    for (int k = 0; k < EMB_HID; ++k) s = fmaf(hA[t][k], sW1[n * EMB_HID + k], s);
    hB[t][n] = sinf(a.omega0 * (s + sb1[n]));
  }
  __syncthreads();
  for (int i = tid; i < EMB_HID * EMB_HID; i += EMB_THREADS) sW1[i] = a.W2[i];  // reuse for layer 2
  __syncthreads();
  for (int i = tid; i < EMB_TOK * EMB_HID; i += EMB_THREADS) {
    const int t = i / EMB_HID, n = i - t * EMB_HID;
    float s = 0.f;
#pragma unroll 16
    for (int k = 0; k < EMB_HID; ++k) s = fmaf(hB[t][k], sW1[n * EMB_HID + k], s);
    hA[t][n] = sinf(a.omega0 * (s + sb2[n]));
  }
  __syncthreads();
  const float imp = *a.impulse;
  const long long left = a.n - tok0;
  const int ntok = left < EMB_TOK ? (int)left : EMB_TOK;
  for (int col = tid; col < a.d; col += EMB_THREADS) {
    float w[EMB_HID];
#pragma unroll
    for (int k = 0; k < EMB_HID; k += 4) {
      const float4 q = *reinterpret_cast<const float4*>(a.Wo + (long long)col * EMB_HID + k);
      w[k] = q.x; w[k + 1] = q.y; w[k + 2] = q.z; w[k + 3] = q.w;
    }
    const float bias = a.bo[col];
    for (int t = 0; t < ntok; ++t) {
      float s = 0.f;
#pragma unroll
      for (int k = 0; k < EMB_HID; ++k) s = fmaf(hA[t][k], w[k], s);
      const float v = ((s + bias) * imp) * active[t];
      const long long off = (tok0 + t) * a.d + col;
      if (a.out_f32) a.out_f32[off] = v;
      else a.out_bf16[off] = __float2bfloat16_rn(v);
    }
  }
}

}  // namespace gfn
