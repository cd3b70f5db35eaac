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
