// Readout GEMMs (logits = y W^T + b and its two backward products) on the
// tensor cores at fp32-level accuracy: each fp32 operand, scaled by a power
// of two, is split into two fp16 pieces x s = x0 + x1 (11 significant bits
// each); along K the A operand is laid out [x0 x0 x1] and the B operand
// [x0 x1 x0], so one fp16 GEMM with K' = 3K and fp32 accumulation sums
// x0 y0 + x0 y1 + x1 y0.  The dropped terms are below 2^-22 of |x y|: the
// result carries a few float32 ulps (~1e-6 relative), a few times a plain
// fp32 GEMM's error.  The per-matrix scale puts
// max|x| s in [2^13, 2^14), so any operand magnitude fits fp16 (the readout's
// logit gradients are ~1/N).
#include <cuda_fp16.h>

#include <mutex>

#include <cublas_v2.h>

#include "abi.h"
#include "common.cuh"

using namespace gfn_abi;

constexpr long long GFN_SPLIT_KB = 512;

namespace {

__global__ void split_absmax_kernel(const float* __restrict__ x, long long n, float* slot) {
  float m = 0.f;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    m = fmaxf(m, fabsf(x[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0 && m > 0.f) atomicMax(reinterpret_cast<unsigned*>(slot), __float_as_uint(m));
}

// Power-of-two scale putting max|x| s in [2^13, 2^14), capped at 2^60 so
// that a tiny (or zero) operand never gives s = inf; the product of two
// scales then stays below 2^120, so 1/(s_a s_b) is a normal float.
GFN_DEV float split_scale(float m) {
  if (!(m > 0.f) || !(m < 3.0e38f)) return 1.f;
  int e;
  frexpf(m, &e);  // m = f 2^e, f in [0.5, 1)
  return ldexpf(1.f, min(14 - e, 60));
}

// x [rows][cols] fp32 -> out fp16 with K' = 3K along the K dimension
// (k_rows: K = rows, out [3 rows][cols]; else K = cols, out [rows][3 cols]).
// K is cut into blocks of GFN_SPLIT_KB; block j (width w) occupies K' range
// [3 j KB, 3 j KB + 3 w) as [x0 | seg1 | seg2], seg1/seg2 = x0/x1 for the A
// role, x1/x0 for the B role.  A GEMM over any whole-block range is then one
// strided matrix, so long K can be summed block by block in fp32.
__global__ void split_f16_kernel(const float* __restrict__ x, long long rows, long long cols, int k_rows,
                                 int role_b, __half* __restrict__ out, float* slot) {
  const float s = split_scale(slot[0]);
  if (blockIdx.x == 0 && threadIdx.x == 0) slot[1] = s;
  const long long n = rows * cols;
  const long long K = k_rows ? rows : cols;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float v = x[i] * s;
    const __half p0 = __float2half_rn(v);
    const __half p1 = __float2half_rn(v - __half2float(p0));
    const __half seg1 = role_b ? p1 : p0, seg2 = role_b ? p0 : p1;
    const long long r = i / cols, c = i - r * cols;
    const long long k = k_rows ? r : c;
    const long long j = k / GFN_SPLIT_KB, kk = k - j * GFN_SPLIT_KB;
    const long long w = (K - j * GFN_SPLIT_KB) < GFN_SPLIT_KB ? (K - j * GFN_SPLIT_KB) : GFN_SPLIT_KB;
    const long long k0 = 3 * j * GFN_SPLIT_KB + kk;  // K' index of segment 0
    if (k_rows) {
      out[k0 * cols + c] = p0;
      out[(k0 + w) * cols + c] = seg1;
      out[(k0 + 2 * w) * cols + c] = seg2;
    } else {
      __half* o = out + r * 3 * cols;
      o[k0] = p0;
      o[k0 + w] = seg1;
      o[k0 + 2 * w] = seg2;
    }
  }
}

__global__ void split_alpha_kernel(const float* sa, const float* sb, float beta, float* ab) {
  // scales are powers of two: 1/(s_a s_b) = 2^-(e_a + e_b) exactly
  int ea, eb;
  frexpf(sa[1], &ea);
  frexpf(sb[1], &eb);
  ab[0] = ldexpf(1.f, 2 - ea - eb);
  ab[1] = beta;
  ab[2] = 1.f;
}

std::mutex g_mu;
cublasHandle_t g_h[64] = {};
// One lock per device handle, held from cublasSetStream to the last GEMM of a
// call, so two host threads never interleave stream or pointer-mode changes.
std::mutex g_use_mu[64];

int handle(cublasHandle_t* out, int* dev_out = nullptr) {
  int dev;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(GFN_ERR_UNSUPPORTED, "device %d", dev);
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_h[dev]) {
    if (cublasCreate(&g_h[dev]) != CUBLAS_STATUS_SUCCESS) return fail(GFN_ERR_CUDA, "cublasCreate failed");
    cublasSetMathMode(g_h[dev], CUBLAS_DEFAULT_MATH);
  }
  *out = g_h[dev];
  if (dev_out) *dev_out = dev;
  return GFN_OK;
}

}  // namespace

namespace gfn_abi {
cudaError_t error_word_readout(int* v, int reset, cudaStream_t s) { return gfn_unit_error_word(v, reset, s); }
}  // namespace gfn_abi

extern "C" {

int gfn_split_f16(const float* x, long long rows, long long cols, int k_along_rows, int role_b, void* out,
                  float* scale, gfn_stream_t stream) {
  if (!x || !out || !scale || rows <= 0 || cols <= 0)
    return fail(GFN_ERR_INVALID, "split_f16: bad arguments");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(scale, 0, 2 * sizeof(float), s);
  if (e != cudaSuccess) return cuda_status(e, "split_f16: scale slot");
  const long long n = rows * cols;
  const unsigned blocks = (unsigned)(n / 256 + 1 < 148 * 16 ? n / 256 + 1 : 148 * 16);
  split_absmax_kernel<<<blocks, 256, 0, s>>>(x, n, scale);
  split_f16_kernel<<<blocks, 256, 0, s>>>(x, rows, cols, k_along_rows, role_b,
                                          reinterpret_cast<__half*>(out), scale);
  return launch_status("split_f16");
}

int gfn_gemm_split_f16(int M, int N, int K, const void* a2, int a_k_rows, const void* b2, int b_k_rows,
                       const float* scale_a, const float* scale_b, float beta, float* c,
                       float* alpha_beta, gfn_stream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0 || !a2 || !b2 || !scale_a || !scale_b || !c || !alpha_beta)
    return fail(GFN_ERR_INVALID, "gemm_split_f16: bad arguments");
  cublasHandle_t h;
  int hdev = 0;
  int st = handle(&h, &hdev);
  if (st) return st;
  std::lock_guard<std::mutex> use(g_use_mu[hdev]);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  split_alpha_kernel<<<1, 1, 0, s>>>(scale_a, scale_b, beta, alpha_beta);
  st = launch_status("gemm_split_f16 alpha");
  if (st) return st;
  if (cublasSetStream(h, s) != CUBLAS_STATUS_SUCCESS) return fail(GFN_ERR_CUDA, "cublasSetStream");
  const int K3 = 3 * K;
  // row-major C[M][N] = A'[M][K'] B'[K'][N]  <=>  column-major C^T = B'^T A'^T
  // B'^T (N x K'): B2 stored [K'][N] (K along rows) -> op N, ld N; stored [N][K'] -> op T, ld K'
  // A'^T (K' x M): A2 stored [M][K'] (K along cols) -> op N, ld K'; stored [K'][M] -> op T, ld M
  // One GEMM per K block, summed in fp32 through beta: the tensor cores' own
  // accumulation error grows with K (measured on B200: 10x an fp32 GEMM's at
  // K = 32000 in one call, below it in 512-wide blocks).
  const cublasOperation_t opb = b_k_rows ? CUBLAS_OP_N : CUBLAS_OP_T;
  const cublasOperation_t opa = a_k_rows ? CUBLAS_OP_T : CUBLAS_OP_N;
  const int ldb = b_k_rows ? N : K3, lda = a_k_rows ? M : K3;
  const __half* A = reinterpret_cast<const __half*>(a2);
  const __half* Bm = reinterpret_cast<const __half*>(b2);
  cublasSetPointerMode(h, CUBLAS_POINTER_MODE_DEVICE);
  cublasStatus_t cs = CUBLAS_STATUS_SUCCESS;
  for (long long k0 = 0; k0 < K && cs == CUBLAS_STATUS_SUCCESS; k0 += GFN_SPLIT_KB) {
    const long long w = (K - k0) < GFN_SPLIT_KB ? (K - k0) : GFN_SPLIT_KB;
    const long long kp = 3 * k0;  // first K' index of the block
    const __half* Ab = a_k_rows ? A + kp * M : A + kp;
    const __half* Bb = b_k_rows ? Bm + kp * N : Bm + kp;
    // the first block uses the caller's beta, later ones accumulate (beta slot 2 = 1)
    cs = cublasGemmEx(h, opb, opa, N, M, (int)(3 * w), alpha_beta, Bb, CUDA_R_16F, ldb, Ab, CUDA_R_16F,
                      lda, k0 == 0 ? alpha_beta + 1 : alpha_beta + 2, c, CUDA_R_32F, N,
                      CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
  }
  cublasSetPointerMode(h, CUBLAS_POINTER_MODE_HOST);
  if (cs != CUBLAS_STATUS_SUCCESS) return fail(GFN_ERR_CUDA, "gemm_split_f16: cublasGemmEx %d", (int)cs);
  return GFN_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Next-token cross-entropy over the readout's logits, the loss of the
// reference's training loops (nn.CrossEntropyLoss() on logits.view(-1, V),
// demos/wikitext/train_wikitext.py:162,185; ignore_index as in
// demos/copy_task/train_copy_task.py:175).  One CTA per row, both passes
// HBM-bound streams of float4:
//   forward   one read of the row: online (max m, sum exp(x - m)) per thread,
//             merged across the CTA; the row keeps (m, ls = log(sum)) apart
//             (their sum rounds at the ulp of m, too coarse for large logits);
//             loss = (m - x[t]) + ls;
//   backward  one read, one write: g = (exp((x - m) - ls) - [j == t]) * scale,
//             scale = dL/dloss / (number of rows not ignored), read from
//             device memory so the upstream gradient needs no host sync.
namespace {

constexpr int XENT_THREADS = 256;

// (max, sum of exp(x - max)) pairs merged; an empty side has max = -inf.
GFN_DEV void lse_merge(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  if (mn == -INFINITY) return;
  s = s * expf(m - mn) + s2 * expf(m2 - mn);
  m = mn;
}

GFN_DEV void lse_add4(float& m, float& s, float4 v) {
  const float c = fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w));
  if (c > m) {
    s = (m == -INFINITY) ? 0.f : s * expf(m - c);
    m = c;
  }
  if (m == -INFINITY) return;  // all -inf so far: nothing to add
  s += expf(v.x - m) + expf(v.y - m) + expf(v.z - m) + expf(v.w - m);
}

template <bool VEC>
__global__ void __launch_bounds__(XENT_THREADS) xent_forward_kernel(const float* __restrict__ logits,
                                                                   const long long* __restrict__ tgt,
                                                                   int V, long long ignore,
                                                                   float* __restrict__ row_loss,
                                                                   float2* __restrict__ row_stats) {
  const long long row = blockIdx.x;
  const float* x = logits + row * (long long)V;
  float m = -INFINITY, s = 0.f;
  if (VEC) {
    const float4* x4 = reinterpret_cast<const float4*>(x);
    for (int i = threadIdx.x; i < V / 4; i += XENT_THREADS) lse_add4(m, s, __ldcs(x4 + i));
  } else {
    for (int i = threadIdx.x; i < V; i += XENT_THREADS) {
      const float v = x[i];
      if (v > m) {
        s = (m == -INFINITY) ? 0.f : s * expf(m - v);
        m = v;
      }
      if (m != -INFINITY) s += expf(v - m);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    lse_merge(m, s, m2, s2);
  }
  __shared__ float sm[XENT_THREADS / 32], ss[XENT_THREADS / 32];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sm[w] = m; ss[w] = s; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int k = 1; k < XENT_THREADS / 32; ++k) lse_merge(m, s, sm[k], ss[k]);
    const float ls = logf(s);
    const long long t = tgt[row];
    float loss = 0.f;
    if (t != ignore) {
      if (t < 0 || t >= V) {
        gfn_flag_error(kDevErrBadToken);
        loss = __int_as_float(0x7fc00000);  // NaN: the row has no valid target
      } else {
        loss = (m - x[t]) + ls;
      }
    }
    row_loss[row] = loss;
    row_stats[row] = make_float2(m, ls);
  }
}

template <bool VEC>
__global__ void __launch_bounds__(XENT_THREADS) xent_backward_kernel(const float* logits,
                                                                    const long long* __restrict__ tgt,
                                                                    const float2* __restrict__ row_stats,
                                                                    int V, long long ignore,
                                                                    const float* __restrict__ scale_p,
                                                                    float* grad) {
  // logits and grad may be the same buffer: every element is read, then
  // written, by one thread
  const long long row = blockIdx.x;
  const float* x = logits + row * (long long)V;
  float* g = grad + row * (long long)V;
  const long long t = tgt[row];
  const bool skip = (t == ignore) || t < 0 || t >= V;
  const float scale = skip ? 0.f : *scale_p;
  const float2 st = row_stats[row];
  const float m = st.x, ls = st.y;
  if (VEC) {
    const float4* x4 = reinterpret_cast<const float4*>(x);
    float4* g4 = reinterpret_cast<float4*>(g);
    for (int i = threadIdx.x; i < V / 4; i += XENT_THREADS) {
      const float4 v = __ldcs(x4 + i);
      float4 o;
      o.x = skip ? 0.f : expf((v.x - m) - ls) * scale;
      o.y = skip ? 0.f : expf((v.y - m) - ls) * scale;
      o.z = skip ? 0.f : expf((v.z - m) - ls) * scale;
      o.w = skip ? 0.f : expf((v.w - m) - ls) * scale;
      if (!skip && t >= 4LL * i && t < 4LL * i + 4) {
        const int k = (int)(t - 4LL * i);
        if (k == 0) o.x -= scale; else if (k == 1) o.y -= scale; else if (k == 2) o.z -= scale; else o.w -= scale;
      }
      __stcs(g4 + i, o);
    }
  } else {
    for (int i = threadIdx.x; i < V; i += XENT_THREADS) {
      float o = skip ? 0.f : expf((x[i] - m) - ls) * scale;
      if (!skip && i == t) o -= scale;
      g[i] = o;
    }
  }
}

bool xent_vec(const void* a, const void* b, int V) {
  return V % 4 == 0 && ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 15u) == 0;
}

}  // namespace

extern "C" {

int gfn_cross_entropy_forward(const float* logits, const long long* targets, long long rows, int V,
                              long long ignore_index, float* row_loss, float* row_stats, gfn_stream_t stream) {
  if (rows < 0 || V <= 0 || (rows > 0 && (!logits || !targets || !row_loss || !row_stats)))
    return fail(GFN_ERR_INVALID, "cross_entropy_forward: bad arguments");
  if (rows > 0x7fffffffLL) return fail(GFN_ERR_INVALID, "cross_entropy_forward: rows > 2^31 - 1");
  if (rows == 0) return GFN_OK;
  if (reinterpret_cast<uintptr_t>(row_stats) & 7u)
    return fail(GFN_ERR_ALIGN, "cross_entropy_forward: row_stats must be 8-byte aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  float2* st = reinterpret_cast<float2*>(row_stats);
  if (xent_vec(logits, logits, V))
    xent_forward_kernel<true><<<(unsigned)rows, XENT_THREADS, 0, s>>>(logits, targets, V, ignore_index, row_loss, st);
  else
    xent_forward_kernel<false><<<(unsigned)rows, XENT_THREADS, 0, s>>>(logits, targets, V, ignore_index, row_loss, st);
  return launch_status("cross_entropy_forward");
}

int gfn_cross_entropy_backward(const float* logits, const long long* targets, const float* row_stats,
                               long long rows, int V, long long ignore_index, const float* grad_scale,
                               float* grad_logits, gfn_stream_t stream) {
  if (rows < 0 || V <= 0 ||
      (rows > 0 && (!logits || !targets || !row_stats || !grad_scale || !grad_logits)))
    return fail(GFN_ERR_INVALID, "cross_entropy_backward: bad arguments");
  if (rows > 0x7fffffffLL) return fail(GFN_ERR_INVALID, "cross_entropy_backward: rows > 2^31 - 1");
  if (rows == 0) return GFN_OK;
  if (reinterpret_cast<uintptr_t>(row_stats) & 7u)
    return fail(GFN_ERR_ALIGN, "cross_entropy_backward: row_stats must be 8-byte aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const float2* st = reinterpret_cast<const float2*>(row_stats);
  if (xent_vec(logits, grad_logits, V))
    xent_backward_kernel<true><<<(unsigned)rows, XENT_THREADS, 0, s>>>(logits, targets, st, V, ignore_index,
                                                                       grad_scale, grad_logits);
  else
    xent_backward_kernel<false><<<(unsigned)rows, XENT_THREADS, 0, s>>>(logits, targets, st, V, ignore_index,
                                                                        grad_scale, grad_logits);
  return launch_status("cross_entropy_backward");
}

}  // extern "C"
