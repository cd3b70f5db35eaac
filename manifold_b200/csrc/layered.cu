// Layered recurrence (large batches): the C ABI of the head-step kernels
// (layered.cuh) around a batched cuBLAS mixing GEMM per layer.
#include <atomic>
#include <vector>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <utility>

#include <cublas_v2.h>
#include <cudaTypedefs.h>

#include "abi.h"
#include "layered.cuh"
#include "head_umma.cuh"
#include "mix_umma.cuh"

using namespace gfn;
using namespace gfn_abi;

namespace gfn_abi {
cudaError_t error_word_layered(int* v, int reset, cudaStream_t s) { return gfn_unit_error_word(v, reset, s); }
}  // namespace gfn_abi


namespace {

std::atomic<int> g_lay_mode{GFN_MIX_UMMA_F16};
// cuBLAS workspace carved from the caller's workspace (4 MiB, 256-byte
// aligned): the GEMMs allocate nothing.
constexpr long long kLayCublasWsFloats = 1LL << 20;
std::mutex g_cublas_mu;
cublasHandle_t g_cublas[64] = {};
// One lock per device handle, held for a whole forward call that uses cuBLAS
// (stream, workspace and pointer-mode changes plus the GEMMs), so two host
// threads never interleave them on the shared handle.
std::mutex g_cublas_use_mu[64];

int cublas_for_device(cublasHandle_t* out) {
  int dev;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(GFN_ERR_UNSUPPORTED, "device %d", dev);
  std::lock_guard<std::mutex> lock(g_cublas_mu);
  if (!g_cublas[dev]) {
    if (cublasCreate(&g_cublas[dev]) != CUBLAS_STATUS_SUCCESS)
      return fail(GFN_ERR_CUDA, "cublasCreate failed");
    // full fp32 products: no TF32
    cublasSetMathMode(g_cublas[dev], CUBLAS_DEFAULT_MATH);
  }
  *out = g_cublas[dev];
  return GFN_OK;
}

// ---------------------------------------------------------------- UMMA mixing
// cuTensorMapEncodeTiled from the driver (no link-time libcuda dependency).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// fp16 tensor map whose inner box (box[0] elements, 64 or 128 bytes) is the
// swizzle span.
int encode_map(CUtensorMap* m, CUtensorMapDataType dt, int esize, const void* base, int rank,
               const cuuint64_t* dims, const cuuint64_t* strides_bytes, const cuuint32_t* box) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return fail(GFN_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, dt, (cuuint32_t)rank, const_cast<void*>(base), dims,
                   strides_bytes, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   box[0] * esize == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(GFN_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return GFN_OK;
}

int encode_f16_map(CUtensorMap* m, const void* base, int rank, const cuuint64_t* dims,
                   const cuuint64_t* strides_bytes, const cuuint32_t* box) {
  return encode_map(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, rank, dims, strides_bytes, box);
}

// Tile of the UMMA mixing GEMM.  256 x 256 tiles (K blocks of 32, three ring
// stages) read the fewest operand bytes per FLOP: used when they still give
// most SMs a tile.  Smaller problems use 128-row tiles and the widest column
// tile that gives every SM work (K blocks of 64).
struct MixShape { int bn, bk, mh; };

MixShape pick_mix_shape(int batch, int dim, int sms, int nmat = 2, int K = 0) {
  MixShape m{64, 64, 1};
  const long long mt1 = (batch + 127) / 128, mt2 = (batch + 255) / 256;
  if (dim % 256 == 0 && nmat * mt2 * (dim / 256) >= (sms * 3) / 4) m = {256, 32, 2};
  else if (dim % 256 == 0 && nmat * mt1 * (dim / 256) >= sms) m = {256, 64, 1};
  else if (dim % 128 == 0 && nmat * mt1 * (dim / 128) >= (sms * 3) / 4) m = {128, 64, 1};
  if (K && K % m.bk) m.bk = 32;  // K blocks must divide the reduction
  if (const char* env = getenv("GFN_MIX_TILE")) {  // tuning override "BN,BK,MH"
    int bn, bk, mh;
    if (sscanf(env, "%d,%d,%d", &bn, &bk, &mh) == 3 && (bn == 64 || bn == 128 || bn == 256) &&
        (bk == 32 || bk == 64) && (mh == 1 || mh == 2) && dim % bn == 0)
      m = {bn, bk, mh};
  }
  return m;
}

struct MixUmmaPlan {
  CUtensorMap ta, tb;
  size_t smem;
  int bn, bk, mh, grid, threads;
};

template <int BN, int BK, int MH>
int mix_plan_for(MixUmmaPlan* p, int sms, int batch, int d, int nmat = 2) {
  using C = MixCfg<BN, BK, MH>;
  p->smem = C::SMEM;
  p->threads = C::THREADS;
  const int tiles = nmat * ((batch + C::BM - 1) / C::BM) * (d / BN);
  p->grid = tiles < sms ? tiles : sms;
  cudaError_t e = cudaFuncSetAttribute(mix_umma_kernel<BN, BK, MH>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p->smem);
  return e == cudaSuccess ? GFN_OK : cuda_status(e, "mixing GEMM: shared memory attribute");
}

#define GFN_MIX_SHAPES(X) X(256, 32, 2) X(256, 32, 1) X(256, 64, 1) X(128, 32, 1) X(128, 64, 1) \
  X(128, 32, 2) X(64, 32, 1) X(64, 64, 1) X(64, 32, 2) X(64, 64, 2)

// Tensor maps of one forward call: activations catkh [2B][3d] and the packed
// split weights WH of every layer, [NL][2d][3d] with the pack's layer stride.
int make_mix_plan(MixUmmaPlan* p, const __half* catkh, const float* packed, const LayOffsets& lo,
                  int batch, int dim, int num_layers, int sms) {
  const MixShape sh = pick_mix_shape(batch, dim, sms);
  p->bn = sh.bn;
  p->bk = sh.bk;
  p->mh = sh.mh;
  int st = GFN_ERR_UNSUPPORTED;
#define GFN_MIX_PLAN(BN, BK, MH) \
  if (sh.bn == BN && sh.bk == BK && sh.mh == MH) st = mix_plan_for<BN, BK, MH>(p, sms, batch, dim);
  GFN_MIX_SHAPES(GFN_MIX_PLAN)
#undef GFN_MIX_PLAN
  if (st) return st == GFN_ERR_UNSUPPORTED ? fail(st, "mixing GEMM: no kernel for the tile") : st;
  const cuuint64_t adims[2] = {(cuuint64_t)3 * dim, (cuuint64_t)2 * batch};
  const cuuint64_t astr[1] = {(cuuint64_t)6 * dim};
  const cuuint32_t abox[2] = {(cuuint32_t)sh.bk, (cuuint32_t)(128 * sh.mh)};
  st = encode_f16_map(&p->ta, catkh, 2, adims, astr, abox);
  if (st) return st;
  const cuuint64_t bdims[3] = {(cuuint64_t)3 * dim, (cuuint64_t)2 * dim, (cuuint64_t)num_layers};
  const cuuint64_t bstr[2] = {(cuuint64_t)6 * dim, (cuuint64_t)lo.total * 4};
  const cuuint32_t bbox[3] = {(cuuint32_t)sh.bk, (cuuint32_t)sh.bn, 1};
  return encode_f16_map(&p->tb, packed + lo.WH, 3, bdims, bstr, bbox);
}

// Programmatic dependent launch of the layered path's tensor-core kernels:
// each may start its prologue (barriers, TMEM, weight copies, the token's
// force) while the previous kernel of the stream finishes; the kernels wait
// for it (griddepcontrol.wait) before touching its outputs.  GFN_LAY_PDL=0
// launches them plainly.
bool use_pdl() {
  static const bool on = [] {
    const char* env = getenv("GFN_LAY_PDL");
    return !(env && atoi(env) == 0);
  }();
  return on;
}

template <typename... KArgs, typename... Args>
void launch_maybe_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                      Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = use_pdl() ? 1 : 0;
  cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

void launch_mix(const MixUmmaPlan& p, const MixUmmaArgs& ma, cudaStream_t s) {
#define GFN_MIX_LAUNCH(BN, BK, MH)                                                       \
  if (p.bn == BN && p.bk == BK && p.mh == MH) {                                          \
    launch_maybe_pdl(mix_umma_kernel<BN, BK, MH>, dim3(p.grid), dim3(p.threads), p.smem, s, p.ta, p.tb, ma); \
    return;                                                                              \
  }
  GFN_MIX_SHAPES(GFN_MIX_LAUNCH)
#undef GFN_MIX_LAUNCH
}

// Tensor-core head step (head_dim 64, UMMA mixing); measured faster than the
// SIMT head step at every C4 batch (512 to 4096 rows).  GFN_LAY_HEAD=0/1
// forces it off/on.
bool use_head_umma(int batch, int heads, int hd, int rank, int mode, int sms) {
  (void)batch; (void)heads; (void)sms;
  if (hd != 64 || mode != GFN_MIX_UMMA_F16 || (rank != 4 && rank != 8 && rank != 16)) return false;
  if (const char* env = getenv("GFN_LAY_HEAD")) return atoi(env) != 0;
  return true;
}

// Threads per row of the tensor-core head step: 4 (two 512-thread CTAs per
// SM) when there are at least as many tiles as SMs (C4 at 2048 and 4096
// rows), else 8 (half the work per thread, a shorter chain per tile: 512 rows
// 27.3 -> 24.9 us, 1024 rows 29.3 -> 25.1 us).  GFN_LAY_HEAD_PARTS=4/8 overrides.
int head_parts(int batch, int heads, int sms) {
  if (const char* env = getenv("GFN_LAY_HEAD_PARTS")) return atoi(env) == 8 ? 8 : 4;
  return (long long)((batch + 127) / 128) * heads >= sms ? 4 : 8;
}

// Rows per head-step tile: 64 (HeadUmmaCfg NDUP 2: twice the tiles of 128-row
// tiles, 8 columns per thread, no spills; C4 at 4096 rows 76.3 -> 60.0 us per
// launch), or 32 (NDUP 4) when 64-row tiles would leave SMs idle (512 rows:
// step 0.76 -> 0.69 ms).  GFN_LAY_HEAD_ROWS=32/64/128 overrides.
int head_rows(int batch, int heads, int sms) {
  if (const char* env = getenv("GFN_LAY_HEAD_ROWS")) {
    const int v = atoi(env);
    return v == 128 ? 128 : v == 32 ? 32 : 64;
  }
  return (long long)((batch + 63) / 64) * heads < sms ? 32 : 64;
}

template <int P, int NDUP>
void launch_head_umma_p(int rank, const CUtensorMap& tmz, const CUtensorMap& tmo, const LayPreArgs& a,
                        dim3 grid, cudaStream_t s) {
  constexpr int T = HeadUmmaCfg<64, P, NDUP>::THREADS;
  if (rank == 4)
    launch_maybe_pdl(layered_head_umma_kernel<4, 64, P, NDUP>, grid, dim3(T), head_umma_smem<4, 64, P, NDUP>(), s,
                     tmz, tmo, a);
  else if (rank == 8)
    launch_maybe_pdl(layered_head_umma_kernel<8, 64, P, NDUP>, grid, dim3(T), head_umma_smem<8, 64, P, NDUP>(), s,
                     tmz, tmo, a);
  else
    launch_maybe_pdl(layered_head_umma_kernel<16, 64, P, NDUP>, grid, dim3(T), head_umma_smem<16, 64, P, NDUP>(),
                     s, tmz, tmo, a);
}

void launch_head_umma(int rank, const CUtensorMap& tmz, const CUtensorMap& tmo, const LayPreArgs& a,
                      dim3 grid, cudaStream_t s, int sms, int rows) {
  if (rows == 32)
    launch_head_umma_p<8, 4>(rank, tmz, tmo, a, grid, s);
  else if (rows == 64)
    launch_head_umma_p<8, 2>(rank, tmz, tmo, a, grid, s);
  else if (head_parts(a.B, a.H, sms) == 4)
    launch_head_umma_p<4, 1>(rank, tmz, tmo, a, grid, s);
  else
    launch_head_umma_p<8, 1>(rank, tmz, tmo, a, grid, s);
}

// The split head-step output catkh as [2][B][3d] fp16 in [1][rows][64] boxes.
int make_out_map(CUtensorMap* m, const __half* catkh, int batch, int dim, int rows) {
  const cuuint64_t dims[3] = {(cuuint64_t)3 * dim, (cuuint64_t)batch, 2};
  const cuuint64_t str[2] = {(cuuint64_t)6 * dim, (cuuint64_t)6 * dim * batch};
  const cuuint32_t box[3] = {64, (cuuint32_t)rows, 1};
  return encode_f16_map(m, catkh, 3, dims, str, box);
}

// z [2B][d] fp32 in [rows x 32] boxes with the 128-byte swizzle.
int make_z_map(CUtensorMap* m, const float* z, int batch, int dim, int rows) {
  const cuuint64_t dims[2] = {(cuuint64_t)dim, (cuuint64_t)2 * batch};
  const cuuint64_t str[1] = {(cuuint64_t)dim * 4};
  const cuuint32_t box[2] = {32, (cuuint32_t)rows};
  return encode_map(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, z, 2, dims, str, box);
}

template <int P, int NDUP>
cudaError_t set_head_umma_smem_p() {
  cudaError_t e = cudaFuncSetAttribute(layered_head_umma_kernel<4, 64, P, NDUP>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)head_umma_smem<4, 64, P, NDUP>());
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(layered_head_umma_kernel<8, 64, P, NDUP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)head_umma_smem<8, 64, P, NDUP>());
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(layered_head_umma_kernel<16, 64, P, NDUP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)head_umma_smem<16, 64, P, NDUP>());
  return e;
}

int set_head_umma_smem() {
  cudaError_t e = set_head_umma_smem_p<8, 1>();
  if (e == cudaSuccess) e = set_head_umma_smem_p<4, 1>();
  if (e == cudaSuccess) e = set_head_umma_smem_p<8, 2>();
  if (e == cudaSuccess) e = set_head_umma_smem_p<8, 4>();
  return e == cudaSuccess ? GFN_OK : cuda_status(e, "head step: shared memory attribute");
}

// ---------------------------------------------------------------- timing
// Optional per-kernel CUDA-event timing of the layered path (measurement
// only): while enabled, each layer's head-step and mixing launches are
// bracketed by events recorded on the launch stream.
std::mutex g_time_mu;
bool g_time_on = false;
long long* g_head_prof = nullptr;  // gfn_debug_head_profile
std::vector<cudaEvent_t> g_time_ev;  // triplets: head start, mix start, mix end
size_t g_time_used = 0;

cudaEvent_t time_event() {
  if (g_time_used == g_time_ev.size()) {
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
    g_time_ev.push_back(e);
  }
  return g_time_ev[g_time_used++];
}

void time_mark(cudaStream_t s) {
  if (!g_time_on) return;
  std::lock_guard<std::mutex> lock(g_time_mu);
  if (cudaEvent_t e = time_event()) cudaEventRecord(e, s);
}

using LayPreKernel = void (*)(LayPreArgs);
struct LayPreInst {
  LayPreKernel fn;
  int tr;
  size_t smem;
};

// Row tile: the largest of 32 / 16 rows (64 for head_dim 16) that still gives two blocks
// per SM (small batches need short tiles to fill the GPU), never below the
// tile's minimum row count (one row per thread row-group).
int pick_tile_rows(int batch, int heads, int hd, int sms) {
  const int min_tr = hd >= 64 ? 16 : hd == 32 ? 32 : 64;
  // 32-row tiles (at most 2 rows per thread for head_dim <= 64) run three
  // blocks per SM; measured faster than 64-row tiles at C4 (1.15M vs 1.08M
  // tokens/s).  head_dim 16 needs 64 rows (one per thread row group).
  const int max_tr = hd == 16 ? 64 : 32;
  if (const char* env = getenv("GFN_LAY_TILE_ROWS")) {  // tuning override
    const int t = atoi(env);
    if (t >= min_tr && t <= max_tr && (t & (t - 1)) == 0) return t;
  }
  for (int tr = max_tr; tr > min_tr; tr >>= 1)
    if ((long long)((batch + tr - 1) / tr) * heads >= 2LL * sms) return tr;
  return min_tr;
}

bool lay_pre_for(int r, int hd, int tr, int hblock, LayPreInst* out) {
#define GFN_L(RK, HD, TR)                                                         \
  if (r == RK && hd == HD && tr == TR) {                                          \
    *out = {layered_pre_kernel<RK, HD, TR>, TR, layered_pre_smem<RK, HD, TR>(hblock)}; \
    return true;                                                                  \
  }
#define GFN_LR(RK) \
  GFN_L(RK, 16, 64) GFN_L(RK, 32, 64) GFN_L(RK, 32, 32) GFN_L(RK, 64, 64) GFN_L(RK, 64, 32) \
  GFN_L(RK, 64, 16) GFN_L(RK, 128, 32) GFN_L(RK, 128, 16)
  GFN_LR(4) GFN_LR(8) GFN_LR(16)
#undef GFN_LR
#undef GFN_L
  return false;
}

}  // namespace

namespace {
__global__ void split_alpha_tc_kernel(const float* sa, const float* sb, float* alpha) {
  // the split scales are powers of two: 1 / (s_a s_b) = 2^-(e_a + e_b) exactly
  int ea, eb;
  frexpf(sa[1], &ea);
  frexpf(sb[1], &eb);
  alpha[0] = ldexpf(1.f, 2 - ea - eb);
}
}  // namespace

extern "C" {

int gfn_debug_head_profile(long long* device_stamps) {
  g_head_prof = device_stamps;
  return GFN_OK;
}

int gfn_debug_layered_timing(int enable) {
  std::lock_guard<std::mutex> lock(g_time_mu);
  g_time_on = enable != 0;
  if (g_time_on) g_time_used = 0;
  return GFN_OK;
}

int gfn_debug_layered_timing_read(double* head_ms, double* mix_ms, int* layer_steps) {
  if (!head_ms || !mix_ms || !layer_steps) return fail(GFN_ERR_INVALID, "timing read: NULL output");
  std::lock_guard<std::mutex> lock(g_time_mu);
  double hs = 0.0, ms = 0.0;
  const size_t n = g_time_used / 3;
  for (size_t i = 0; i < n; ++i) {
    float a = 0.f, b = 0.f;
    cudaError_t e = cudaEventSynchronize(g_time_ev[3 * i + 2]);
    if (e == cudaSuccess) e = cudaEventElapsedTime(&a, g_time_ev[3 * i], g_time_ev[3 * i + 1]);
    if (e == cudaSuccess) e = cudaEventElapsedTime(&b, g_time_ev[3 * i + 1], g_time_ev[3 * i + 2]);
    if (e != cudaSuccess) return cuda_status(e, "timing read");
    hs += a;
    ms += b;
  }
  *head_ms = hs;
  *mix_ms = ms;
  *layer_steps = (int)n;
  return GFN_OK;
}

long long gfn_leapfrog_layered_pack_floats(int dim, int heads, int rank, int num_layers) {
  Layout L;
  if (make_layout(dim, heads, rank, num_layers, &L) != GFN_OK || heads < 2) return -1;
  return (long long)num_layers * lay_offsets(heads, L.hd, rank, dim).total;
}

int gfn_leapfrog_layered_pack(const float* U_stack, const float* W_stack,
                              const float* W_forget_stack, const float* b_forget_stack,
                              const float* dt_params, const float* mix_x_w, const float* mix_x_b,
                              const float* norm_x_w, const float* mix_v_w, const float* mix_v_b,
                              const float* norm_v_w, int dim, int heads, int rank, int num_layers,
                              float* packed, long long packed_floats, gfn_stream_t stream) {
  Layout L;
  int st = make_layout(dim, heads, rank, num_layers, &L);
  if (st) return st;
  if (heads < 2) return fail(GFN_ERR_UNSUPPORTED, "layered path needs heads > 1 (head mixing)");
  if (!U_stack || !W_stack || !W_forget_stack || !b_forget_stack || !dt_params || !mix_x_w ||
      !mix_x_b || !norm_x_w || !mix_v_w || !mix_v_b || !norm_v_w || !packed)
    return fail(GFN_ERR_INVALID, "layered pack: NULL operand");
  LayPackArgs a;
  a.U = U_stack; a.W = W_stack; a.Wf = W_forget_stack; a.bf = b_forget_stack; a.dtp = dt_params;
  a.Wx = mix_x_w; a.bx = mix_x_b; a.gx = norm_x_w; a.Wv = mix_v_w; a.bv = mix_v_b; a.gv = norm_v_w;
  a.out = packed; a.NL = num_layers; a.d = dim; a.H = heads; a.hd = L.hd; a.r = rank;
  a.LF = lay_offsets(heads, L.hd, rank, dim).total;
  if (packed_floats < a.LF * num_layers) return fail(GFN_ERR_INVALID, "layered pack: buffer too small");
  if (!aligned16(packed)) return fail(GFN_ERR_ALIGN, "layered pack: output not 16-byte aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const LayOffsets lo = lay_offsets(heads, L.hd, rank, dim);
  // per-layer max|W| slot: zeroed, then atomic max over both mixing matrices
  cudaError_t e = cudaMemset2DAsync(packed + lo.wsc, (size_t)a.LF * 4, 0, 4, (size_t)num_layers, s);
  if (e != cudaSuccess) return cuda_status(e, "layered pack: scale slots");
  layered_absmax_kernel<<<148 * 4, 256, 0, s>>>(mix_x_w, mix_v_w, packed, num_layers, dim, a.LF, lo.wsc);
  e = cudaMemset2DAsync(packed + lo.HUs, (size_t)a.LF * 4, 0, (size_t)(2 * heads) * 4, (size_t)num_layers, s);
  if (e != cudaSuccess) return cuda_status(e, "layered pack: head scale slots");
  layered_head_absmax_kernel<<<num_layers * heads, 256, 0, s>>>(W_forget_stack, packed, num_layers, heads,
                                                                L.hd, a.LF, lo.HUs);
  layered_pack_kernel<<<148 * 8, 256, 0, s>>>(a);
  return launch_status("layered_pack_kernel");
}

int gfn_gemm_split_f16_tc(int M, int N, int K, const void* a2, const void* b2, const float* scale_a,
                          const float* scale_b, const float* bias, float* c, float* alpha_slot,
                          gfn_stream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0 || !a2 || !b2 || !scale_a || !scale_b || !c || !alpha_slot)
    return fail(GFN_ERR_INVALID, "gemm_split_f16_tc: bad arguments");
  if (K > 512 || K % 32 || N % 64)
    return fail(GFN_ERR_UNSUPPORTED, "gemm_split_f16_tc: needs K <= 512, K %% 32 == 0, N %% 64 == 0 "
                "(K=%d, N=%d)", K, N);
  if ((reinterpret_cast<uintptr_t>(a2) | reinterpret_cast<uintptr_t>(b2)) & 15u || (bias && !aligned16(bias)) ||
      !aligned16(c))
    return fail(GFN_ERR_ALIGN, "gemm_split_f16_tc: operands must be 16-byte aligned");
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const MixShape sh = pick_mix_shape(M, N, sms, 1, K);
  MixUmmaPlan p;
  p.bn = sh.bn; p.bk = sh.bk; p.mh = sh.mh;
  int st = GFN_ERR_UNSUPPORTED;
#define GFN_GEMM_PLAN(BN, BK, MH) \
  if (sh.bn == BN && sh.bk == BK && sh.mh == MH) st = mix_plan_for<BN, BK, MH>(&p, sms, M, N, 1);
  GFN_MIX_SHAPES(GFN_GEMM_PLAN)
#undef GFN_GEMM_PLAN
  if (st) return st == GFN_ERR_UNSUPPORTED ? fail(st, "gemm_split_f16_tc: no kernel for the tile") : st;
  const cuuint64_t adims[2] = {(cuuint64_t)3 * K, (cuuint64_t)M};
  const cuuint64_t astr[1] = {(cuuint64_t)6 * K};
  const cuuint32_t abox[2] = {(cuuint32_t)sh.bk, (cuuint32_t)(128 * sh.mh)};
  st = encode_f16_map(&p.ta, a2, 2, adims, astr, abox);
  if (st) return st;
  const cuuint64_t bdims[3] = {(cuuint64_t)3 * K, (cuuint64_t)N, 1};
  const cuuint64_t bstr[2] = {(cuuint64_t)6 * K, (cuuint64_t)6 * K * N};
  const cuuint32_t bbox[3] = {(cuuint32_t)sh.bk, (cuuint32_t)sh.bn, 1};
  st = encode_f16_map(&p.tb, b2, 3, bdims, bstr, bbox);
  if (st) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  split_alpha_tc_kernel<<<1, 1, 0, s>>>(scale_a, scale_b, alpha_slot);
  MixUmmaArgs ma = {};
  ma.z = c; ma.spart = nullptr; ma.bias = bias; ma.alpha = alpha_slot; ma.B = M; ma.d = K; ma.layer = 0;
  ma.mtiles = (M + 128 * sh.mh - 1) / (128 * sh.mh); ma.ntiles = N / sh.bn; ma.K = K; ma.N = N; ma.nmat = 1;
  ma.out_bias = bias != nullptr;
  launch_mix(p, ma, s);
  return launch_status("gemm_split_f16_tc");
}

int gfn_leapfrog_layered_set_mixing(int mode) {
  if (mode == -1) return g_lay_mode.load();
  if (mode != GFN_MIX_SPLIT_BF16 && mode != GFN_MIX_FP32_SIMT && mode != GFN_MIX_SPLIT_F16 &&
      mode != GFN_MIX_UMMA_F16)
    return -fail(GFN_ERR_INVALID, "mixing mode %d", mode);
  return g_lay_mode.exchange(mode);
}

// Workspace: cat / split activations / z / state (12 B d), row statistics
// (2 B + 4), the mixing GEMM's partial row sums (2 B ceil(d / 64)), then the
// cuBLAS workspace (rounded up to a 256-byte boundary inside the slack).
static long long lay_ws_base(int batch, int dim) {
  return 12LL * batch * dim + 2LL * batch + 4 + 2LL * batch * ((dim + 63) / 64);
}

long long gfn_leapfrog_layered_workspace_floats(int batch, int dim) {
  return lay_ws_base(batch, dim) + 64 + kLayCublasWsFloats;
}

int gfn_leapfrog_layered_forward(const float* x_init, const float* v_init,
                                 long long state_row_stride, const float* forces_f32,
                                 const void* forces_bf16, const long long* token_ids,
                                 const float* embed_table, long long vocab, const float* mask,
                                 const float* packed, long long packed_floats, int batch,
                                 int seq_len, int dim, int heads, int rank, int num_layers,
                                 float base_dt, float* x_seq, float* v_seq, float* x_final,
                                 float* v_final, float* workspace, long long workspace_floats,
                                 gfn_stream_t stream) {
  Layout L;
  int st = make_layout(dim, heads, rank, num_layers, &L);
  if (st) return st;
  if (heads < 2) return fail(GFN_ERR_UNSUPPORTED, "layered path needs heads > 1 (head mixing)");
  if (batch < 0 || seq_len < 0) return fail(GFN_ERR_INVALID, "layered: bad sizes");
  if (!x_init || !v_init || !packed || !workspace) return fail(GFN_ERR_INVALID, "layered: NULL operand");
  if (!aligned16(x_init) || !aligned16(v_init) || !aligned16(packed) || !aligned16(workspace) ||
      (forces_f32 && !aligned16(forces_f32)) || (embed_table && !aligned16(embed_table)) ||
      (forces_bf16 && (reinterpret_cast<uintptr_t>(forces_bf16) & 7u)) || state_row_stride % 4)
    return fail(GFN_ERR_ALIGN, "layered: operands must be 16-byte aligned (bf16 forces 8-byte), "
                "state row stride a multiple of 4");
  const int nsrc = (forces_f32 != nullptr) + (forces_bf16 != nullptr) + (token_ids != nullptr);
  if (seq_len > 0 && nsrc != 1) return fail(GFN_ERR_INVALID, "layered: give exactly one force source");
  if (token_ids && (!embed_table || vocab <= 0)) return fail(GFN_ERR_INVALID, "layered: ids need a table");
  const LayOffsets lo = lay_offsets(heads, L.hd, rank, dim);
  if (packed_floats < lo.total * num_layers) return fail(GFN_ERR_INVALID, "layered: packed too small");
  if (workspace_floats < gfn_leapfrog_layered_workspace_floats(batch, dim))
    return fail(GFN_ERR_INVALID, "layered: workspace too small");
  if (batch == 0 || seq_len == 0) return GFN_OK;
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (dev < 0 || dev >= 64) return fail(GFN_ERR_UNSUPPORTED, "device %d", dev);
  LayPreInst inst;
  if (!lay_pre_for(rank, L.hd, pick_tile_rows(batch, heads, L.hd, sms), lo.hblock, &inst))
    return fail(GFN_ERR_UNSUPPORTED, "layered: head_dim %d must be 16, 32, 64 or 128", L.hd);
  LayPreKernel pre = inst.fn;
  const long long BD = (long long)batch * dim;
  int mode = g_lay_mode.load();
  // the tcgen05 kernel tiles K by 64 and N by at least 64 columns
  if (mode == GFN_MIX_UMMA_F16 && (dim % 64 != 0 || 3LL * dim > (1LL << 31) / 4))
    mode = GFN_MIX_SPLIT_F16;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // cuBLAS only for the library-GEMM mixing modes (the default uses none)
  cublasHandle_t hb = nullptr;
  std::unique_lock<std::mutex> cublas_use(g_cublas_use_mu[dev], std::defer_lock);
  if (mode != GFN_MIX_UMMA_F16) {
    st = cublas_for_device(&hb);
    if (st) return st;
    cublas_use.lock();
    if (cublasSetStream(hb, s) != CUBLAS_STATUS_SUCCESS) return fail(GFN_ERR_CUDA, "cublasSetStream");
    // cuBLAS wants a 256-byte aligned workspace: round the absolute address up
    const uintptr_t p0 = reinterpret_cast<uintptr_t>(workspace + lay_ws_base(batch, dim));
    const uintptr_t p1 = (p0 + 255) & ~(uintptr_t)255;
    float* cws = reinterpret_cast<float*>(p1);
    const size_t bytes = (size_t)(workspace_floats * 4) - (size_t)(p1 - reinterpret_cast<uintptr_t>(workspace));
    if (cublasSetWorkspace(hb, cws, bytes) != CUBLAS_STATUS_SUCCESS)
      return fail(GFN_ERR_CUDA, "cublasSetWorkspace");
  }
  float* cat = workspace;
  __nv_bfloat16* catk = reinterpret_cast<__nv_bfloat16*>(workspace + 2 * BD);
  float* z = workspace + 8 * BD;
  float* xs = workspace + 10 * BD;
  float* vs = workspace + 11 * BD;
  float* stat = workspace + 12 * BD;
  float* spart = stat + 2LL * batch + 4;
  MixUmmaPlan mix;
  if (mode == GFN_MIX_UMMA_F16) {
    st = make_mix_plan(&mix, reinterpret_cast<const __half*>(catk), packed, lo, batch, dim, num_layers, sms);
    if (st) return st;
  }
  const bool head_tc = use_head_umma(batch, heads, L.hd, rank, mode, sms);
  const int hrows = head_rows(batch, heads, sms);
  CUtensorMap zmap, omap;
  if (head_tc) {
    st = set_head_umma_smem();
    if (!st) st = make_z_map(&zmap, z, batch, dim, hrows);
    if (!st) st = make_out_map(&omap, reinterpret_cast<const __half*>(catk), batch, dim, hrows);
    if (st) return st;
  }
  const dim3 head_grid((batch + hrows - 1) / hrows, heads);
  const size_t pre_smem = inst.smem;
  cudaError_t ae = cudaFuncSetAttribute(pre, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pre_smem);
  if (ae != cudaSuccess) return cuda_status(ae, "layered: shared memory attribute");
  const dim3 pre_grid((batch + inst.tr - 1) / inst.tr, heads);
  // Small problems: each head-step block computes its rows' RMSNorm factors
  // itself (every head re-reads the rows: batch * heads * dim * 8 bytes per
  // layer from L2) instead of a separate launch.
  const bool fuse_stat = (long long)batch * heads * dim * 8 <= (32LL << 20);
  const unsigned stat_blocks = (unsigned)((2LL * batch * 32 + 255) / 256);
  const float one = 1.f, zero = 0.f;
  for (int t = 0; t < seq_len; ++t) {
    for (int l = 0; l < num_layers; ++l) {
      const float* lay = packed + (long long)l * lo.total;
      LayPreArgs a = {};
      if (l == 0) {
        a.x_in = t == 0 ? x_init : xs;
        a.v_in = t == 0 ? v_init : vs;
        a.in_stride = t == 0 ? state_row_stride : dim;
      } else {
        const float* prev = packed + (long long)(l - 1) * lo.total;
        a.z = z;
        a.prev = prev;
        if (mode == GFN_MIX_UMMA_F16) {  // the GEMM epilogue left partial row sums
          a.spart = spart;
          a.nparts = dim / mix.bn;
        } else {
          if (!fuse_stat)
            layered_rowstat_kernel<<<stat_blocks, 256, 0, s>>>(z, prev + lo.bx, prev + lo.bv, stat,
                                                               batch, dim);
          a.stat = fuse_stat ? nullptr : stat;
        }
      }
      a.f32 = forces_f32; a.fbf16 = reinterpret_cast<const __nv_bfloat16*>(forces_bf16);
      a.ids = token_ids; a.table = embed_table; a.vocab = vocab; a.mask = mask;
      a.t = t; a.L = seq_len; a.lay = lay; a.B = batch;
      if (mode == GFN_MIX_SPLIT_BF16) a.catk = catk;
      else if (mode == GFN_MIX_SPLIT_F16 || mode == GFN_MIX_UMMA_F16) a.catkh = reinterpret_cast<__half*>(catk);
      else a.cat = cat; a.d = dim; a.H = heads;
      a.hd = L.hd; a.base_dt = base_dt;
      a.prof = g_head_prof;
      time_mark(s);
      if (head_tc)
        launch_head_umma(rank, zmap, omap, a, head_grid, s, sms, hrows);
      else
        pre<<<pre_grid, LAY_THREADS, pre_smem, s>>>(a);
      time_mark(s);
      if (mode == GFN_MIX_UMMA_F16) {
        MixUmmaArgs ma;
        ma.z = z; ma.alpha = lay + lo.wsc + 2; ma.spart = spart; ma.bias = lay + lo.bx; ma.B = batch; ma.d = dim; ma.layer = l;
        ma.K = dim; ma.N = dim; ma.nmat = 2; ma.out_bias = 0;
        ma.mtiles = (batch + 128 * mix.mh - 1) / (128 * mix.mh); ma.ntiles = dim / mix.bn;
        launch_mix(mix, ma, s);
        time_mark(s);
        continue;
      }
      // z[i] = cat[i] . W_i^T for i in {x, v}: column-major view z^T = W cat^T
      cublasStatus_t cs;
      if (mode == GFN_MIX_SPLIT_BF16) {
        const int K = LAY_SPLIT * dim;
        cs = cublasGemmStridedBatchedEx(
            hb, CUBLAS_OP_T, CUBLAS_OP_N, dim, batch, K, &one, lay + lo.WK, CUDA_R_16BF, K,
            (long long)dim * K, catk, CUDA_R_16BF, K, (long long)batch * K, &zero, z, CUDA_R_32F,
            dim, BD, 2, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
      } else if (mode == GFN_MIX_SPLIT_F16) {
        // alpha = 1/s and beta = 0 live in the pack (device pointer mode)
        const int K = LAY_SPLIT_H * dim;
        cublasSetPointerMode(hb, CUBLAS_POINTER_MODE_DEVICE);
        cs = cublasGemmStridedBatchedEx(
            hb, CUBLAS_OP_T, CUBLAS_OP_N, dim, batch, K, lay + lo.wsc + 2, lay + lo.WH, CUDA_R_16F, K,
            (long long)dim * K, catk, CUDA_R_16F, K, (long long)batch * K, lay + lo.wsc + 3, z,
            CUDA_R_32F, dim, BD, 2, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
        cublasSetPointerMode(hb, CUBLAS_POINTER_MODE_HOST);
      } else {
        cs = cublasSgemmStridedBatched(hb, CUBLAS_OP_T, CUBLAS_OP_N, dim, batch, dim, &one,
                                       lay + lo.Wx, dim, (long long)dim * dim, cat, dim, BD, &zero,
                                       z, dim, BD, 2);
      }
      time_mark(s);
      if (cs != CUBLAS_STATUS_SUCCESS) return fail(GFN_ERR_CUDA, "mixing GEMM failed (%d)", (int)cs);
    }
    const float* last = packed + (long long)(num_layers - 1) * lo.total;
    layered_rowstat_kernel<<<stat_blocks, 256, 0, s>>>(z, last + lo.bx, last + lo.bv, stat, batch, dim);
    layered_finalize_kernel<<<148 * 8, 256, 0, s>>>(z, stat, last, heads, L.hd, rank, batch, dim,
                                                    seq_len, t, x_seq, v_seq, xs, vs);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_status(e, "layered kernels");
  if (x_final) e = cudaMemcpyAsync(x_final, xs, BD * 4, cudaMemcpyDeviceToDevice, s);
  if (e == cudaSuccess && v_final) e = cudaMemcpyAsync(v_final, vs, BD * 4, cudaMemcpyDeviceToDevice, s);
  return cuda_status(e, "layered final state copy");
}

}  // extern "C"
