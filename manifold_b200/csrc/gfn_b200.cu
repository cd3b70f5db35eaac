// gfn_b200: the C ABI (include/gfn_b200.h) over the sm_100a kernels.
// One translation unit: every kernel header is included here.
#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>

#include <cuda.h>

#include "../../include/gfn_b200.h"
#include "embed.cuh"
#include "leapfrog_seq.cuh"
#include "leapfrog_bwd.cuh"
#include "ops_small.cuh"
#include "pack.cuh"
#include "scan.cuh"
#include "abi.h"

using namespace gfn;
using namespace gfn_abi;

namespace gfn_abi {
thread_local char g_msg[512] = "";
long long* g_phase_prof = nullptr;  // gfn_debug_set_phase_profile

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return status;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return GFN_OK;
  return fail(GFN_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int launch_status(const char* what) { return cuda_status(cudaGetLastError(), what); }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
}  // namespace gfn_abi

namespace {

struct DevInfo {
  int sms = 0;
  int max_smem = 0;
};

int dev_info(DevInfo* out) {
  int dev;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  static thread_local int cached_dev = -1;
  static thread_local DevInfo cached;
  if (dev != cached_dev) {
    e = cudaDeviceGetAttribute(&cached.sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_status(e, "cudaDeviceGetAttribute");
    e = cudaDeviceGetAttribute(&cached.max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return cuda_status(e, "cudaDeviceGetAttribute");
    cached_dev = dev;
  }
  *out = cached;
  return GFN_OK;
}

}  // namespace

// ------------------------------------------------------------------ plans
namespace gfn_abi {
int make_layout(int d, int H, int r, int NL, Layout* L) {
  if (d <= 0 || H <= 0 || r <= 0 || NL <= 0 || d % H != 0)
    return fail(GFN_ERR_INVALID, "bad shape dim=%d heads=%d rank=%d layers=%d", d, H, r, NL);
  const int hd = d / H;
  if (hd % 4 != 0 || hd > 128)
    return fail(GFN_ERR_UNSUPPORTED, "head_dim %d must be a multiple of 4 and <= 128", hd);
  if (r != 4 && r != 8 && r != 16)
    return fail(GFN_ERR_UNSUPPORTED, "per-head rank %d not in {4, 8, 16}", r);
  int K = 1;
  while (K * 2 <= 8 && H % (K * 2) == 0) K *= 2;
  L->d = d; L->H = H; L->hd = hd; L->r = r; L->NL = NL;
  L->K = K; L->C = d / K; L->hpc = H / K;
  L->mix = H > 1;
  // k-chunk (~8 KB of each of x and v weights).  With C a power of two the
  // kernel finds a concat element's column block by shifts, so a chunk may
  // span blocks; otherwise the chunk is a multiple of 4 dividing C.
  const bool c_pow2 = (L->C & (L->C - 1)) == 0;
  int kc_target = 4096;  // weight floats per chunk row block (measured best on B200 for C1-C5)
  if (const char* env = getenv("GFN_SEQ_CHUNK_FLOATS")) {  // tuning override
    const int v = atoi(env);
    if (v >= 256) kc_target = v;
  }
  int KC = kc_target / L->C;
  if (c_pow2) {
    int p = 4;
    while (p * 2 <= KC && d % (p * 2) == 0) p *= 2;
    KC = p;
  } else {
    if (KC > L->C) KC = L->C;
    KC -= KC % 4;
    if (KC < 4) KC = 4;
    while (L->C % KC) KC -= 4;
  }
  L->KC = KC;
  L->nchunk = L->mix ? d / KC : 0;
  L->CF = KC * chunk_row_stride(L->C);
  L->HS = head_offsets(L->hpc, hd, r, L->C).total;
  L->LF = (long long)L->HS + (long long)L->nchunk * L->CF;
  L->HST = L->HS + ((L->hpc * hd * hd + 31) / 32) * 32;
  L->LFT = (long long)L->HST + 2LL * L->nchunk * L->CF;
  return GFN_OK;
}

}  // namespace gfn_abi

namespace {

struct SeqPlan {
  Layout L;
  int NW;  // compute warps
  int R, TR, NG, tiles, S, NST, nclusters, max_active;
  size_t smem;
  int o_head, o_chunk, o_ox, o_ov, o_catx, o_catv, o_part;
};

size_t plan_smem(const Layout& L, int R, int NST, SeqPlan* p) {
  int off = 0;
  auto take = [&](int n) { int o = off; off += ((n + 31) / 32) * 32; return o; };
  p->o_head = take(2 * L.HS);
  p->o_chunk = take(L.mix ? NST * L.CF : 0);
  p->o_ox = take(L.mix ? R * L.C : 0);
  p->o_ov = take(L.mix ? R * L.C : 0);
  p->o_catx = take(L.mix ? R * L.d : 0);
  p->o_catv = take(L.mix ? R * L.d : 0);
  p->o_part = take(L.mix ? L.K * R * 2 : 0);
  return SEQ_BAR_BYTES + (size_t)off * 4;
}

// The kernel instance for (rank, elements per lane).
using SeqKernel = void (*)(SeqArgs);

SeqKernel seq_kernel_for(int r, int epl, int nw) {
#define GFN_K(RK, E, W) \
  if (r == RK && epl == E && nw == W) return leapfrog_seq_kernel<RK, E, W>;
  GFN_K(4, 1, 8) GFN_K(4, 2, 16) GFN_K(4, 4, 16) GFN_K(8, 1, 8) GFN_K(8, 2, 16) GFN_K(8, 4, 16)
  GFN_K(16, 1, 8) GFN_K(16, 2, 16) GFN_K(16, 4, 16)
#undef GFN_K
  return nullptr;
}

// Heads of width <= 32 (one element per lane, short per-CTA work): 8 compute
// warps with 168 registers each; wider heads need the latency hiding of 16.
int seq_warps(const Layout& L) { return L.hd <= 32 ? 8 : 16; }
int seq_maxu(int nw) { return nw == 8 ? SeqShape<8>::MAXU : SeqShape<16>::MAXU; }

int seq_epl(const Layout& L) { return L.hd <= 32 ? 1 : L.hd <= 64 ? 2 : 4; }

// Row-block geometry for R rows: mixing tiles and the split-K factor.
bool plan_rows(const Layout& L, int R, SeqPlan* p) {
  const int CT = p->NW * 32;
  if (R < 1 || R * L.hpc > p->NW * seq_maxu(p->NW)) return false;
  const int TR = R < 4 ? R : 4;
  const int NG = 2 * L.C / 4;
  const int tiles = NG * ((R + TR - 1) / TR);
  if (L.mix && tiles > CT) return false;
  p->R = R; p->TR = TR; p->NG = NG; p->tiles = L.mix ? tiles : 1;
  int S = 1;
  while (L.mix && S < 16 && S * 2 * tiles <= CT) S *= 2;
  p->S = S;
  return true;
}

int set_cluster_cfg(cudaLaunchConfig_t* cfg, cudaLaunchAttribute* attr, const SeqPlan& p) {
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.L.K;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg->blockDim = dim3(p.NW * 32 + 32);
  cfg->dynamicSmemBytes = p.smem;
  cfg->attrs = attr;
  cfg->numAttrs = 1;
  return GFN_OK;
}

int query_active_clusters(SeqKernel kern, const SeqPlan& p, int* out) {
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem);
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(smem)");
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  set_cluster_cfg(&cfg, attr, p);
  cfg.gridDim = dim3((unsigned)p.L.K);
  e = cudaOccupancyMaxActiveClusters(out, kern, &cfg);
  if (e != cudaSuccess) return cuda_status(e, "cudaOccupancyMaxActiveClusters");
  return GFN_OK;
}

// Chooses rows per cluster R so that all ceil(B / R) clusters are resident
// at once: a persistent cluster left for a second wave doubles the time.
int make_plan(int B, const Layout& L, const DevInfo& di, SeqPlan* p) {
  p->L = L;
  p->NW = seq_warps(L);
  SeqKernel kern = seq_kernel_for(L.r, seq_epl(L), p->NW);
  if (!kern) return fail(GFN_ERR_UNSUPPORTED, "no kernel for rank %d head_dim %d", L.r, L.hd);
  auto fit = [&](int R) -> bool {
    if (!plan_rows(L, R, p)) return false;
    // Ring depth: up to two layers of chunks (+2), so the copies of the next
    // layer's weights are in flight a whole layer ahead, as shared memory allows.
    const int want = L.mix ? 2 * L.nchunk + 2 : 2;
    // two CTAs per SM for the 8-warp form: each gets a bit under half the SM
    size_t budget = p->NW == 8 ? (size_t)114 * 1024 : (size_t)di.max_smem;
    if (const char* env = getenv("GFN_SEQ_SMEM_KB")) {  // tuning override
      const int kb = atoi(env);
      if (kb > 0 && (size_t)kb * 1024 <= (size_t)di.max_smem) budget = (size_t)kb * 1024;
    }
    for (int NST = want < SEQ_MAX_NST ? want : SEQ_MAX_NST; NST >= 2; --NST) {
      const size_t smem = plan_smem(L, R, NST, p);
      if (smem + 256 <= budget) {  // 256 B: the kernels' static shared memory
        p->NST = NST;
        p->smem = smem;
        return true;
      }
    }
    return false;
  };
  int Rmax = 0;
  for (int R = 1; R <= B && R <= p->NW * seq_maxu(p->NW); ++R)
    if (fit(R)) Rmax = R;
  if (Rmax == 0)
    return fail(GFN_ERR_RESOURCES, "no sequence plan fits %d bytes of shared memory", di.max_smem);
  // Fewest rows per cluster (most clusters, shortest per-CTA chain) such
  // that every cluster is resident in one wave.
  int R = 1;
  // Tuning override: GFN_SEQ_ROWS=<rows per cluster> (clamped to what fits)
  if (const char* env = getenv("GFN_SEQ_ROWS")) {
    const int want = atoi(env);
    if (want >= 1) {
      R = want < Rmax ? want : Rmax;
      if (!fit(R)) return fail(GFN_ERR_RESOURCES, "sequence plan for %d rows does not fit", R);
      int active = 0;
      const int st = query_active_clusters(kern, *p, &active);
      if (st) return st;
      p->max_active = active;
      p->nclusters = (B + p->R - 1) / p->R;
      return GFN_OK;
    }
  }
  for (int it = 0; it < 8; ++it) {
    if (!fit(R)) return fail(GFN_ERR_RESOURCES, "sequence plan for %d rows does not fit", R);
    int active = 0;
    const int st = query_active_clusters(kern, *p, &active);
    if (st) return st;
    p->max_active = active;
    if (active <= 0) return fail(GFN_ERR_RESOURCES, "a %d-CTA cluster cannot be scheduled", L.K);
    const int need = (B + active - 1) / active;
    if (need <= R || R == Rmax) break;
    R = need < Rmax ? need : Rmax;
  }
  p->nclusters = (B + p->R - 1) / p->R;
  return GFN_OK;
}

int launch_seq(SeqKernel kern, const SeqArgs& a, const SeqPlan& p, cudaStream_t stream) {
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem);
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(smem)");
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  set_cluster_cfg(&cfg, attr, p);
  cfg.gridDim = dim3((unsigned)(p.nclusters * p.L.K));
  cfg.stream = stream;
  e = cudaLaunchKernelEx(&cfg, kern, a);
  return cuda_status(e, "leapfrog_seq_kernel launch");
}

}  // namespace

static int pack_impl(bool train, const float* U_stack, const float* W_stack, const float* W_forget_stack,
                      const float* b_forget_stack, const float* dt_params, const float* mix_x_w,
                      const float* mix_x_b, const float* norm_x_w, const float* mix_v_w,
                      const float* mix_v_b, const float* norm_v_w, int dim, int heads, int rank,
                      int num_layers, float* packed, long long packed_floats, gfn_stream_t stream) {
  Layout L;
  int st = make_layout(dim, heads, rank, num_layers, &L);
  if (st) return st;
  if (!U_stack || !W_stack || !W_forget_stack || !b_forget_stack || !dt_params || !packed)
    return fail(GFN_ERR_INVALID, "pack: NULL head parameter");
  if (L.mix && (!mix_x_w || !mix_v_w))
    return fail(GFN_ERR_INVALID, "pack: heads > 1 needs the mixing weights");
  const long long LFx = train ? L.LFT : L.LF;
  const long long need = (long long)num_layers * L.K * LFx;
  if (packed_floats < need) return fail(GFN_ERR_INVALID, "pack: buffer %lld < %lld floats", packed_floats, need);
  if (!aligned16(packed)) return fail(GFN_ERR_ALIGN, "pack: output not 16-byte aligned");
  PackArgs a;
  a.U = U_stack; a.W = W_stack; a.Wf = W_forget_stack; a.bf = b_forget_stack; a.dtp = dt_params;
  a.Wx = mix_x_w; a.bx = mix_x_b; a.gx = norm_x_w; a.Wv = mix_v_w; a.bv = mix_v_b; a.gv = norm_v_w;
  a.out = packed; a.NL = num_layers; a.d = dim; a.H = heads; a.hd = L.hd; a.r = rank; a.K = L.K;
  a.C = L.C; a.hpc = L.hpc; a.KC = L.KC; a.nchunk = L.nchunk; a.HS = L.HS; a.CF = L.CF; a.LF = LFx;
  a.train = train ? 1 : 0; a.HST = L.HST;
  long long blocks = (need + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  pack_kernel<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return launch_status("pack_kernel");
}


static int seq_forward_impl(bool train, float* traj, const float* x_init, const float* v_init,
                                  long long state_row_stride, const float* forces_f32,
                                  const void* forces_bf16, const long long* token_ids,
                                  const float* embed_table, long long vocab, const float* mask,
                                  const float* packed, long long packed_floats, int batch,
                                  int seq_len, int dim, int heads, int rank, int num_layers,
                                  float base_dt, float* x_seq, float* v_seq, float* x_final,
                                  float* v_final, gfn_stream_t stream) {
  Layout L;
  int st = make_layout(dim, heads, rank, num_layers, &L);
  if (st) return st;
  if (batch < 0 || seq_len < 0) return fail(GFN_ERR_INVALID, "sequence: batch=%d seq_len=%d", batch, seq_len);
  if (!x_init || !v_init || !packed) return fail(GFN_ERR_INVALID, "sequence: NULL state or weights");
  if (state_row_stride < 0) return fail(GFN_ERR_INVALID, "sequence: negative state stride");
  const int nsrc = (forces_f32 != nullptr) + (forces_bf16 != nullptr) + (token_ids != nullptr);
  if (seq_len > 0 && nsrc != 1)
    return fail(GFN_ERR_INVALID, "sequence: give exactly one of forces_f32, forces_bf16, token_ids");
  if (token_ids && (!embed_table || vocab <= 0))
    return fail(GFN_ERR_INVALID, "sequence: token_ids need embed_table and vocab > 0");
  const long long LFx = train ? L.LFT : L.LF;
  const long long need = (long long)num_layers * L.K * LFx;
  if (packed_floats < need) return fail(GFN_ERR_INVALID, "sequence: packed %lld < %lld floats", packed_floats, need);
  if (!aligned16(packed)) return fail(GFN_ERR_ALIGN, "sequence: packed weights not 16-byte aligned");
  if (batch == 0) return GFN_OK;
  DevInfo di;
  st = dev_info(&di);
  if (st) return st;
  SeqPlan p;
  st = make_plan(batch, L, di, &p);
  if (st) return st;
  SeqArgs a = {};
  a.x0 = x_init; a.v0 = v_init; a.state_stride = state_row_stride;
  a.f32 = forces_f32; a.fbf16 = reinterpret_cast<const __nv_bfloat16*>(forces_bf16);
  a.ids = token_ids; a.table = embed_table; a.vocab = vocab; a.mask = mask; a.pack = packed;
  a.x_seq = x_seq; a.v_seq = v_seq; a.x_out = x_final; a.v_out = v_final;
  a.B = batch; a.L = seq_len; a.d = dim; a.H = heads; a.hd = L.hd; a.NL = num_layers;
  a.K = L.K; a.R = p.R; a.C = L.C; a.hpc = L.hpc; a.KC = L.KC; a.nchunk = L.nchunk; a.NST = p.NST;
  a.HS = L.HS; a.CF = L.CF; a.LF = LFx; a.mix = L.mix;
  a.chunk_base = train ? L.HST : L.HS; a.traj = traj;
  a.TR = p.TR; a.NG = p.NG; a.tiles = p.tiles; a.S = p.S;
  a.base_dt = base_dt; a.prof = g_phase_prof;
  a.o_head = p.o_head; a.o_chunk = p.o_chunk; a.o_ox = p.o_ox; a.o_ov = p.o_ov;
  a.o_catx = p.o_catx; a.o_catv = p.o_catv; a.o_part = p.o_part;
  a.logC = (L.C & (L.C - 1)) == 0 ? __builtin_ctz(L.C) : -1;
  return launch_seq(seq_kernel_for(rank, seq_epl(L), p.NW), a, p,
                    reinterpret_cast<cudaStream_t>(stream));
}


extern "C" {

const char* gfn_status_string(int s) {
  switch (s) {
    case GFN_OK: return "ok";
    case GFN_ERR_INVALID: return "invalid argument";
    case GFN_ERR_UNSUPPORTED: return "unsupported configuration";
    case GFN_ERR_ALIGN: return "misaligned pointer";
    case GFN_ERR_CUDA: return "CUDA error";
    case GFN_ERR_RESOURCES: return "insufficient device resources";
    default: return "unknown status";
  }
}

const char* gfn_last_error_message(void) { return g_msg; }

const char* gfn_build_info(void) {
  return "gfn_b200 sm_100a; kernels: leapfrog_seq (cluster/DSMEM/bulk-copy), leapfrog_head, "
         "christoffel, scan, parallel_layer_scan, siren_embed, pack";
}

int gfn_get_device_error(int* bits, int reset, gfn_stream_t stream) {
  if (!bits) return fail(GFN_ERR_INVALID, "bits is NULL");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int v0 = 0, v1 = 0, v2 = 0, v3 = 0;
  cudaError_t e = gfn_unit_error_word(&v0, reset, s);
  if (e == cudaSuccess) e = error_word_layered(&v1, reset, s);
  if (e == cudaSuccess) e = error_word_probe(&v2, reset, s);
  if (e == cudaSuccess) e = error_word_readout(&v3, reset, s);
  if (e != cudaSuccess) return cuda_status(e, "device error word");
  *bits = v0 | v1 | v2 | v3;
  return GFN_OK;
}

int gfn_christoffel_fused(const float* v, const float* U, const float* W, float* gamma,
                          const float* x, const float* V_w, int batch, int dim, int rank,
                          float plasticity, float sing_thresh, float sing_strength, int topology,
                          float R_val, float r_val, gfn_stream_t stream) {
  (void)x; (void)sing_thresh; (void)sing_strength; (void)R_val; (void)r_val;
  if (!v || !U || !W || !gamma) return fail(GFN_ERR_INVALID, "christoffel: NULL operand");
  if (batch < 0 || dim <= 0) return fail(GFN_ERR_INVALID, "christoffel: batch=%d dim=%d", batch, dim);
  if (topology != 0 || plasticity != 0.f || V_w)
    return fail(GFN_ERR_UNSUPPORTED, "christoffel: only the Euclidean, plasticity-free form");
  if (rank != 4 && rank != 8 && rank != 16)
    return fail(GFN_ERR_UNSUPPORTED, "christoffel: rank %d not in {4, 8, 16}", rank);
  if (rank % 4 == 0 && !aligned16(U)) return fail(GFN_ERR_ALIGN, "christoffel: U not 16-byte aligned");
  if (batch == 0) return GFN_OK;
  HeadArgs a = {};
  a.v = v; a.U = U; a.W = W; a.gamma_out = gamma; a.B = batch; a.hd = dim;
  const size_t smem = (size_t)small_smem(dim, rank).total * 4;
  if (smem > 200 * 1024) return fail(GFN_ERR_RESOURCES, "christoffel: dim %d too large", dim);
  dim3 grid((batch + SMALL_ROWS - 1) / SMALL_ROWS);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
#define GFN_CH(RK)                                                                                   \
  case RK:                                                                                           \
    cudaFuncSetAttribute(christoffel_kernel<RK>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    christoffel_kernel<RK><<<grid, SMALL_THREADS, smem, s>>>(a);                                     \
    break;
  switch (rank) { GFN_CH(4) GFN_CH(8) GFN_CH(16) }
#undef GFN_CH
  return launch_status("christoffel_kernel");
}

int gfn_leapfrog_fused(const float* x, const float* v, const float* f, const float* U,
                       const float* W, const float* W_forget, const float* b_forget, float* x_new,
                       float* v_new, float dt, const float* dt_scales, int dt_scales_count,
                       int batch, int dim, int rank, int steps, int topology, float plasticity,
                       float R_val, float r_val, gfn_stream_t stream) {
  (void)R_val; (void)r_val;
  if (!x || !v || !U || !W || !x_new || !v_new) return fail(GFN_ERR_INVALID, "leapfrog: NULL operand");
  if (batch < 0 || dim <= 0 || steps < 0) return fail(GFN_ERR_INVALID, "leapfrog: bad sizes");
  if (topology != 0 || plasticity != 0.f)
    return fail(GFN_ERR_UNSUPPORTED, "leapfrog: only topology 0 without plasticity");
  if (rank != 4 && rank != 8 && rank != 16)
    return fail(GFN_ERR_UNSUPPORTED, "leapfrog: rank %d not in {4, 8, 16}", rank);
  if (!aligned16(U)) return fail(GFN_ERR_ALIGN, "leapfrog: U not 16-byte aligned");
  if (dt_scales && dt_scales_count != 1 && dt_scales_count != batch)
    return fail(GFN_ERR_INVALID, "leapfrog: dt_scales_count %d (need 1 or batch)", dt_scales_count);
  if ((W_forget == nullptr) != (b_forget == nullptr) && W_forget == nullptr)
    return fail(GFN_ERR_INVALID, "leapfrog: b_forget without W_forget");
  if (batch == 0) return GFN_OK;
  HeadArgs a = {};
  a.x = x; a.v = v; a.f = f; a.U = U; a.W = W; a.Wf = W_forget; a.bf = b_forget;
  a.dt_scale = dt_scales; a.dt_scale_n = dt_scales_count; a.dt = dt; a.steps = steps;
  a.x_out = x_new; a.v_out = v_new; a.B = batch; a.hd = dim;
  const size_t smem = (size_t)small_smem(dim, rank).total * 4;
  if (smem > 200 * 1024) return fail(GFN_ERR_RESOURCES, "leapfrog: dim %d too large", dim);
  dim3 grid((batch + SMALL_ROWS - 1) / SMALL_ROWS);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
#define GFN_LF(RK)                                                                                     \
  case RK:                                                                                             \
    cudaFuncSetAttribute(leapfrog_head_kernel<RK>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    leapfrog_head_kernel<RK><<<grid, SMALL_THREADS, smem, s>>>(a);                                     \
    break;
  switch (rank) { GFN_LF(4) GFN_LF(8) GFN_LF(16) }
#undef GFN_LF
  return launch_status("leapfrog_head_kernel");
}

int gfn_debug_set_phase_profile(long long* device_counters) {
  g_phase_prof = device_counters;
  return GFN_OK;
}

long long gfn_leapfrog_pack_floats(int dim, int heads, int rank, int num_layers) {
  Layout L;
  if (make_layout(dim, heads, rank, num_layers, &L) != GFN_OK) return -1;
  return (long long)num_layers * L.K * L.LF;
}

int gfn_leapfrog_plan(int batch, int dim, int heads, int rank, int num_layers, int* out8) {
  int* out6 = out8;
  if (!out6) return fail(GFN_ERR_INVALID, "plan: out6 NULL");
  Layout L;
  int st = make_layout(dim, heads, rank, num_layers, &L);
  if (st) return st;
  DevInfo di;
  st = dev_info(&di);
  if (st) return st;
  SeqPlan p;
  st = make_plan(batch > 0 ? batch : 1, L, di, &p);
  if (st) return st;
  out6[0] = L.K; out6[1] = p.R; out6[2] = p.nclusters; out6[3] = (int)p.smem;
  out6[4] = L.KC; out6[5] = p.NST; out6[6] = p.max_active; out6[7] = p.S;
  return GFN_OK;
}

int gfn_leapfrog_pack(const float* U_stack, const float* W_stack, const float* W_forget_stack,
                      const float* b_forget_stack, const float* dt_params, const float* mix_x_w,
                      const float* mix_x_b, const float* norm_x_w, const float* mix_v_w,
                      const float* mix_v_b, const float* norm_v_w, int dim, int heads, int rank,
                      int num_layers, float* packed, long long packed_floats, gfn_stream_t stream) {
  return pack_impl(false, U_stack, W_stack, W_forget_stack, b_forget_stack, dt_params, mix_x_w,
                   mix_x_b, norm_x_w, mix_v_w, mix_v_b, norm_v_w, dim, heads, rank, num_layers,
                   packed, packed_floats, stream);
}

long long gfn_leapfrog_pack_train_floats(int dim, int heads, int rank, int num_layers) {
  Layout L;
  if (make_layout(dim, heads, rank, num_layers, &L) != GFN_OK) return -1;
  return (long long)num_layers * L.K * L.LFT;
}

int gfn_leapfrog_pack_train(const float* U_stack, const float* W_stack,
                            const float* W_forget_stack, const float* b_forget_stack,
                            const float* dt_params, const float* mix_x_w, const float* mix_x_b,
                            const float* norm_x_w, const float* mix_v_w, const float* mix_v_b,
                            const float* norm_v_w, int dim, int heads, int rank, int num_layers,
                            float* packed, long long packed_floats, gfn_stream_t stream) {
  return pack_impl(true, U_stack, W_stack, W_forget_stack, b_forget_stack, dt_params, mix_x_w,
                   mix_x_b, norm_x_w, mix_v_w, mix_v_b, norm_v_w, dim, heads, rank, num_layers,
                   packed, packed_floats, stream);
}

int gfn_leapfrog_sequence_forward(const float* x_init, const float* v_init,
                                  long long state_row_stride, const float* forces_f32,
                                  const void* forces_bf16, const long long* token_ids,
                                  const float* embed_table, long long vocab, const float* mask,
                                  const float* packed, long long packed_floats, int batch,
                                  int seq_len, int dim, int heads, int rank, int num_layers,
                                  float base_dt, float* x_seq, float* v_seq, float* x_final,
                                  float* v_final, gfn_stream_t stream) {
  return seq_forward_impl(false, nullptr, x_init, v_init, state_row_stride, forces_f32, forces_bf16,
                          token_ids, embed_table, vocab, mask, packed, packed_floats, batch, seq_len,
                          dim, heads, rank, num_layers, base_dt, x_seq, v_seq, x_final, v_final,
                          stream);
}

int gfn_leapfrog_sequence_forward_train(const float* x_init, const float* v_init,
                                        long long state_row_stride, const float* forces_f32,
                                        const void* forces_bf16, const long long* token_ids,
                                        const float* embed_table, long long vocab,
                                        const float* mask, const float* packed_train,
                                        long long packed_floats, int batch, int seq_len, int dim,
                                        int heads, int rank, int num_layers, float base_dt,
                                        float* x_seq, float* v_seq, float* x_final, float* v_final,
                                        float* traj, gfn_stream_t stream) {
  if (!traj) return fail(GFN_ERR_INVALID, "forward_train: traj is NULL");
  return seq_forward_impl(true, traj, x_init, v_init, state_row_stride, forces_f32, forces_bf16,
                          token_ids, embed_table, vocab, mask, packed_train, packed_floats, batch,
                          seq_len, dim, heads, rank, num_layers, base_dt, x_seq, v_seq, x_final,
                          v_final, stream);
}

long long gfn_parallel_scan_workspace_floats(int batch, int seq_len, int dim) {
  (void)seq_len;
  return 2LL * 64 * batch * dim;
}

int gfn_parallel_scan(const float* a, const float* x, float* y, float* workspace,
                      long long workspace_floats, int batch, int seq_len, int dim,
                      gfn_stream_t stream) {
  if (!x || !y) return fail(GFN_ERR_INVALID, "scan: NULL x or y");
  if (batch < 0 || seq_len < 0 || dim <= 0) return fail(GFN_ERR_INVALID, "scan: bad sizes");
  if (dim % 4) return fail(GFN_ERR_UNSUPPORTED, "scan: dim %d must be a multiple of 4", dim);
  if (!aligned16(x) || !aligned16(y) || (a && !aligned16(a)))
    return fail(GFN_ERR_ALIGN, "scan: operands must be 16-byte aligned");
  if (batch == 0 || seq_len == 0) return GFN_OK;
  DevInfo di;
  int st = dev_info(&di);
  if (st) return st;
  ScanArgs s;
  s.a = a; s.x = x; s.y = y; s.ws = workspace; s.B = batch; s.L = seq_len; s.D = dim; s.P = 1;
  const long long groups = (long long)batch * (dim / 4);
  const long long want_threads = (long long)di.sms * 1024;
  int P = 1;
  if (workspace && groups < want_threads / 4) {
    while (P < 64 && groups * P * 2 <= want_threads && seq_len / (P * 2) >= 64) P *= 2;
  }
  if (P > 1 && workspace_floats < 2LL * P * batch * dim) P = 1;
  s.P = P;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  const unsigned gx = (unsigned)((groups + SCAN_THREADS - 1) / SCAN_THREADS);
  if (P == 1) {
    scan_single_kernel<<<gx, SCAN_THREADS, 0, cs>>>(s);
    return launch_status("scan_single_kernel");
  }
  scan_chunk_reduce_kernel<<<dim3(gx, P), SCAN_THREADS, 0, cs>>>(s);
  const long long BD = (long long)batch * dim;
  scan_chunk_carry_kernel<<<(unsigned)((BD + SCAN_THREADS - 1) / SCAN_THREADS), SCAN_THREADS, 0, cs>>>(s);
  scan_chunk_apply_kernel<<<dim3(gx, P), SCAN_THREADS, 0, cs>>>(s);
  return launch_status("scan_chunk kernels");
}

int gfn_parallel_layer_scan(const float* z, float* x_seq, float* v_seq, int batch, int seq_len,
                            int dim, int heads, float base_dt, gfn_stream_t stream) {
  if (!z || !x_seq || !v_seq) return fail(GFN_ERR_INVALID, "layer scan: NULL operand");
  if (batch < 0 || seq_len < 0 || dim <= 0 || heads <= 0 || dim % heads)
    return fail(GFN_ERR_INVALID, "layer scan: bad sizes");
  if (dim % 4) return fail(GFN_ERR_UNSUPPORTED, "layer scan: dim %d must be a multiple of 4", dim);
  if (!aligned16(z) || !aligned16(x_seq) || !aligned16(v_seq))
    return fail(GFN_ERR_ALIGN, "layer scan: operands must be 16-byte aligned");
  if (batch == 0 || seq_len == 0) return GFN_OK;
  PScanArgs s;
  s.z = z; s.x_seq = x_seq; s.v_seq = v_seq; s.B = batch; s.L = seq_len; s.D = dim; s.H = heads;
  s.base_dt = base_dt;
  const long long groups = (long long)batch * (dim / 4);
  parallel_layer_scan_kernel<<<(unsigned)((groups + SCAN_THREADS - 1) / SCAN_THREADS), SCAN_THREADS, 0,
                               reinterpret_cast<cudaStream_t>(stream)>>>(s);
  return launch_status("parallel_layer_scan_kernel");
}

int gfn_functional_embedding(const long long* ids, long long n, const float* W0, const float* b0,
                             const float* W1, const float* b1, const float* W2, const float* b2,
                             const float* Wo, const float* bo, const float* impulse, float omega0,
                             int dim, float* out_f32, void* out_bf16, gfn_stream_t stream) {
  if (!ids || !W0 || !b0 || !W1 || !b1 || !W2 || !b2 || !Wo || !bo || !impulse)
    return fail(GFN_ERR_INVALID, "embedding: NULL operand");
  if ((out_f32 == nullptr) == (out_bf16 == nullptr))
    return fail(GFN_ERR_INVALID, "embedding: give exactly one of out_f32, out_bf16");
  if (n < 0 || dim <= 0) return fail(GFN_ERR_INVALID, "embedding: bad sizes");
  if (!aligned16(Wo)) return fail(GFN_ERR_ALIGN, "embedding: Wo not 16-byte aligned");
  if (n == 0) return GFN_OK;
  EmbArgs a;
  a.ids = ids; a.n = n; a.W0 = W0; a.b0 = b0; a.W1 = W1; a.b1 = b1; a.W2 = W2; a.b2 = b2;
  a.Wo = Wo; a.bo = bo; a.impulse = impulse; a.omega0 = omega0; a.d = dim;
  a.out_f32 = out_f32; a.out_bf16 = reinterpret_cast<__nv_bfloat16*>(out_bf16);
  const long long blocks = (n + EMB_TOK - 1) / EMB_TOK;
  siren_embed_kernel<<<(unsigned)blocks, EMB_THREADS, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return launch_status("siren_embed_kernel");
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Scan without caller-provided scratch.
//
// Some callers cannot allocate device memory at the point where they run a
// scan: code inside a custom allocator or memory-pool callback, plugins whose
// host framework owns every allocation, or callers with a fixed memory
// budget.  gfn_parallel_scan_noalloc keeps the chunk aggregates of the
// time-split scan in the fixed array below instead of a workspace argument.
// The array is part of the library image: every GPU that loads the library
// holds GFN_SCAN_STATIC_FLOATS floats (8 MiB) of it until the process exits.
namespace {

constexpr long long GFN_SCAN_STATIC_FLOATS = 2LL * 1024 * 1024;
constexpr long long GFN_SCAN_STATIC_MAX_COLUMNS = GFN_SCAN_STATIC_FLOATS / 4;  // batch * dim

static __device__ __align__(256) float g_scan_static_scratch[GFN_SCAN_STATIC_FLOATS];

// Device address of g_scan_static_scratch, looked up once per (device,
// context).  In host code the symbol name is only a host-side stand-in, so
// the address has to come from cudaGetSymbolAddress with that device
// current.  The cache is keyed by the context's unique id as well: after a
// cudaDeviceReset the primary context (and the module holding the array) is
// created anew, and the lookup is repeated.
constexpr int GFN_MAX_DEVICES = 64;
float* g_scan_static_ptr[GFN_MAX_DEVICES] = {};
unsigned long long g_scan_static_ctx[GFN_MAX_DEVICES] = {};
std::mutex g_scan_static_mu;

// Unique id of the calling thread's current context (0 if unavailable).
unsigned long long current_context_id() {
  using GetCurrent = CUresult (*)(CUcontext*);
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrent>(p);
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetId>(p);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current && get_id && get_current(&ctx) == CUDA_SUCCESS && ctx) get_id(ctx, &id);
  return id;
}

int scan_static_scratch(int dev, float** out) {
  if (dev < 0 || dev >= GFN_MAX_DEVICES) return fail(GFN_ERR_UNSUPPORTED, "device %d", dev);
  // cudaFree(0) makes the device's primary context current if it is not yet
  cudaError_t e = cudaFree(nullptr);
  if (e != cudaSuccess) return cuda_status(e, "context init");
  const unsigned long long ctx = current_context_id();
  std::lock_guard<std::mutex> lock(g_scan_static_mu);
  if (!g_scan_static_ptr[dev] || g_scan_static_ctx[dev] != ctx || ctx == 0) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_scan_static_scratch);
    if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(scan scratch)");
    g_scan_static_ptr[dev] = static_cast<float*>(p);
    g_scan_static_ctx[dev] = ctx;
  }
  *out = g_scan_static_ptr[dev];
  return GFN_OK;
}

}  // namespace

extern "C" int gfn_parallel_scan_noalloc(const float* a, const float* x, float* y, int batch,
                                         int seq_len, int dim, gfn_stream_t stream) {
  if (!x || !y) return fail(GFN_ERR_INVALID, "scan (no-alloc): NULL x or y");
  if (batch < 0 || seq_len < 0 || dim <= 0) return fail(GFN_ERR_INVALID, "scan (no-alloc): bad sizes");
  if (dim % 4) return fail(GFN_ERR_UNSUPPORTED, "scan (no-alloc): dim %d must be a multiple of 4", dim);
  if (!aligned16(x) || !aligned16(y) || (a && !aligned16(a)))
    return fail(GFN_ERR_ALIGN, "scan (no-alloc): operands must be 16-byte aligned");
  const long long BD = (long long)batch * dim;
  if (BD > GFN_SCAN_STATIC_MAX_COLUMNS)
    return fail(GFN_ERR_INVALID,
                "scan (no-alloc): batch*dim = %lld exceeds the static scratch limit of %lld columns; "
                "use gfn_parallel_scan with a workspace",
                BD, GFN_SCAN_STATIC_MAX_COLUMNS);
  if (batch == 0 || seq_len == 0) return GFN_OK;
  int dev;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  float* scratch = nullptr;
  int st = scan_static_scratch(dev, &scratch);
  if (st) return st;
  DevInfo di;
  st = dev_info(&di);
  if (st) return st;
  // Same time-split rule as gfn_parallel_scan, capped by the array size.
  const long long groups = (long long)batch * (dim / 4);
  const long long want_threads = (long long)di.sms * 1024;
  int P = 1;
  if (groups < want_threads / 4)
    while (P < 64 && groups * P * 2 <= want_threads && seq_len / (P * 2) >= 64) P *= 2;
  while (P > 1 && 2LL * P * BD > GFN_SCAN_STATIC_FLOATS) P /= 2;
  ScanArgs s;
  s.a = a; s.x = x; s.y = y; s.ws = scratch; s.B = batch; s.L = seq_len; s.D = dim; s.P = P;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  const unsigned gx = (unsigned)((groups + SCAN_THREADS - 1) / SCAN_THREADS);
  if (P == 1) {
    scan_single_kernel<<<gx, SCAN_THREADS, 0, cs>>>(s);
    return launch_status("scan_single_kernel (no-alloc)");
  }
  // Pass 1 overwrites every aggregate slot it uses before pass 2 reads it,
  // so nothing left in the array by an earlier call is ever read.
  scan_chunk_reduce_kernel<<<dim3(gx, P), SCAN_THREADS, 0, cs>>>(s);
  scan_chunk_carry_kernel<<<(unsigned)((BD + SCAN_THREADS - 1) / SCAN_THREADS), SCAN_THREADS, 0, cs>>>(s);
  scan_chunk_apply_kernel<<<dim3(gx, P), SCAN_THREADS, 0, cs>>>(s);
  return launch_status("scan_chunk kernels (no-alloc)");
}

// ---------------------------------------------------------------------------
// BPTT backward
namespace {

struct BwdPlan {
  SeqPlan s;  // rows, mixing tiles (NW = BWD_NW)
  int NST, max_active;
  size_t smem;
  int o_head, o_chunk, o_ox, o_ov, o_catx, o_catv, o_dcx, o_dcv, o_part, o_part2, o_px, o_pv;
};

size_t bwd_smem(const Layout& L, int R, int NST, BwdPlan* p) {
  int off = 0;
  auto take = [&](int n) { int o = off; off += ((n + 31) / 32) * 32; return o; };
  p->o_head = take(2 * L.HST);
  p->o_chunk = take(L.mix ? NST * L.CF : 0);
  p->o_ox = take(R * L.C);
  p->o_ov = take(R * L.C);
  p->o_catx = take(L.mix ? R * L.d : 0);
  p->o_catv = take(L.mix ? R * L.d : 0);
  p->o_dcx = take(L.mix ? R * L.d : 0);
  p->o_dcv = take(L.mix ? R * L.d : 0);
  p->o_part = take(L.mix ? L.K * R * 2 : 0);
  p->o_part2 = take(L.mix ? L.K * R * 2 : 0);
  p->o_px = take(R * L.C);
  p->o_pv = take(R * L.C);
  return SEQ_BAR_BYTES + (size_t)off * 4;
}

using BwdKernel = void (*)(BwdArgs);
BwdKernel bwd_kernel_for(int r, int epl) {
#define GFN_B(RK, E) if (r == RK && epl == E) return leapfrog_bwd_kernel<RK, E>;
  GFN_B(4, 1) GFN_B(4, 2) GFN_B(8, 1) GFN_B(8, 2) GFN_B(16, 1) GFN_B(16, 2)
#undef GFN_B
  return nullptr;
}

int bwd_cfg(BwdKernel kern, const BwdPlan& p, int K, unsigned grid, cudaStream_t stream,
            cudaLaunchConfig_t* cfg, cudaLaunchAttribute* attr) {
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem);
  if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(bwd smem)");
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = K;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  *cfg = cudaLaunchConfig_t{};
  cfg->gridDim = dim3(grid);
  cfg->blockDim = dim3(BWD_THREADS);
  cfg->dynamicSmemBytes = p.smem;
  cfg->stream = stream;
  cfg->attrs = attr;
  cfg->numAttrs = 1;
  return GFN_OK;
}

int make_bwd_plan(int B, const Layout& L, const DevInfo& di, BwdPlan* p) {
  BwdKernel kern = bwd_kernel_for(L.r, seq_epl(L));
  if (!kern) return fail(GFN_ERR_UNSUPPORTED, "backward: no kernel for rank %d head_dim %d (<= 64)", L.r, L.hd);
  p->s.L = L;
  p->s.NW = BWD_NW;
  auto fit = [&](int R) -> bool {
    if (R * L.hpc > BWD_NW * BWD_MAXU || !plan_rows(L, R, &p->s)) return false;
    const int want = L.mix ? 2 * 2 * L.nchunk + 2 : 2;
    for (int NST = want < SEQ_MAX_NST - 1 ? want : SEQ_MAX_NST - 1; NST >= 2; --NST) {
      const size_t smem = bwd_smem(L, R, NST, p);
      if (smem + 256 <= (size_t)di.max_smem) {  // 256 B: the kernels' static shared memory
        p->NST = NST;
        p->smem = smem;
        return true;
      }
    }
    return false;
  };
  int Rmax = 0;
  for (int R = 1; R <= B && R <= BWD_NW * BWD_MAXU; ++R)
    if (fit(R)) Rmax = R;
  if (Rmax == 0) return fail(GFN_ERR_RESOURCES, "no backward plan fits shared memory");
  const int per_wave = di.sms / L.K > 0 ? di.sms / L.K : 1;
  int R = (B + per_wave - 1) / per_wave;
  if (R < 1) R = 1;
  if (R > Rmax) R = Rmax;
  for (int it = 0; it < 8; ++it) {
    if (!fit(R)) return fail(GFN_ERR_RESOURCES, "backward plan for %d rows does not fit", R);
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr[1];
    int st = bwd_cfg(kern, *p, L.K, (unsigned)L.K, nullptr, &cfg, attr);
    if (st) return st;
    int active = 0;
    cudaError_t e = cudaOccupancyMaxActiveClusters(&active, kern, &cfg);
    if (e != cudaSuccess) return cuda_status(e, "cudaOccupancyMaxActiveClusters(bwd)");
    if (active <= 0) return fail(GFN_ERR_RESOURCES, "backward: a %d-CTA cluster cannot be scheduled", L.K);
    p->max_active = active;
    const int need = (B + active - 1) / active;
    if (need <= R || R == Rmax) break;
    R = need < Rmax ? need : Rmax;
  }
  p->s.nclusters = (B + p->s.R - 1) / p->s.R;
  return GFN_OK;
}

}  // namespace

extern "C" {

long long gfn_leapfrog_backward_workspace_floats(int batch, int seq_len, int dim, int heads,
                                                 int rank, int num_layers) {
  if (batch < 0 || seq_len < 0 || dim <= 0 || heads <= 0 || rank <= 0 || num_layers <= 0) return -1;
  const long long steps = (long long)num_layers * seq_len * batch;
  return BWD_NSIG * steps * dim + BWD_NSMALL * steps * heads * rank + steps * heads;
}

int gfn_leapfrog_sequence_backward(const float* traj, const float* forces_f32,
                                   const void* forces_bf16, const long long* token_ids,
                                   const float* embed_table, long long vocab, const float* mask,
                                   const float* packed_train, long long packed_floats,
                                   const float* gx_seq, const float* gv_seq,
                                   const float* gx_final, const float* gv_final, int batch,
                                   int seq_len, int dim, int heads, int rank, int num_layers,
                                   float base_dt, float* dx_init, float* dv_init, float* d_forces,
                                   float* workspace, long long workspace_floats,
                                   gfn_stream_t stream) {
  Layout L;
  int st = make_layout(dim, heads, rank, num_layers, &L);
  if (st) return st;
  if (batch < 0 || seq_len < 0) return fail(GFN_ERR_INVALID, "backward: bad sizes");
  if (!traj || !packed_train || !dx_init || !dv_init || !workspace)
    return fail(GFN_ERR_INVALID, "backward: NULL traj, weights, output or workspace");
  const int nsrc = (forces_f32 != nullptr) + (forces_bf16 != nullptr) + (token_ids != nullptr);
  if (seq_len > 0 && nsrc != 1)
    return fail(GFN_ERR_INVALID, "backward: give exactly one force source (as in the forward)");
  const long long need = (long long)num_layers * L.K * L.LFT;
  if (packed_floats < need) return fail(GFN_ERR_INVALID, "backward: packed %lld < %lld floats", packed_floats, need);
  const long long wneed = gfn_leapfrog_backward_workspace_floats(batch, seq_len, dim, heads, rank, num_layers);
  if (workspace_floats < wneed)
    return fail(GFN_ERR_INVALID, "backward: workspace %lld < %lld floats", workspace_floats, wneed);
  if (!aligned16(packed_train)) return fail(GFN_ERR_ALIGN, "backward: packed weights not 16-byte aligned");
  if (batch == 0 || seq_len == 0) return GFN_OK;
  DevInfo di;
  st = dev_info(&di);
  if (st) return st;
  BwdPlan p;
  st = make_bwd_plan(batch, L, di, &p);
  if (st) return st;
  BwdArgs a = {};
  a.f32 = forces_f32; a.fbf16 = reinterpret_cast<const __nv_bfloat16*>(forces_bf16);
  a.ids = token_ids; a.table = embed_table; a.vocab = vocab; a.mask = mask;
  a.pack = packed_train; a.traj = traj; a.gx_seq = gx_seq; a.gv_seq = gv_seq;
  a.gx_fin = gx_final; a.gv_fin = gv_final; a.dx0 = dx_init; a.dv0 = dv_init; a.dforces = d_forces;
  a.ws = workspace;
  a.B = batch; a.L = seq_len; a.d = dim; a.H = heads; a.hd = L.hd; a.NL = num_layers;
  a.K = L.K; a.R = p.s.R; a.C = L.C; a.hpc = L.hpc; a.KC = L.KC; a.nchunk = L.nchunk; a.NST = p.NST;
  a.HS = L.HS; a.HST = L.HST; a.CF = L.CF; a.LF = L.LFT; a.mix = L.mix;
  a.TR = p.s.TR; a.NG = p.s.NG; a.tiles = p.s.tiles; a.S = p.s.S;
  a.logC = (L.C & (L.C - 1)) == 0 ? __builtin_ctz(L.C) : -1;
  a.base_dt = base_dt;
  a.o_head = p.o_head; a.o_chunk = p.o_chunk; a.o_ox = p.o_ox; a.o_ov = p.o_ov;
  a.o_catx = p.o_catx; a.o_catv = p.o_catv; a.o_dcx = p.o_dcx; a.o_dcv = p.o_dcv;
  a.o_part = p.o_part; a.o_part2 = p.o_part2; a.o_px = p.o_px; a.o_pv = p.o_pv;
  BwdKernel kern = bwd_kernel_for(rank, seq_epl(L));
  cudaLaunchConfig_t cfg;
  cudaLaunchAttribute attr[1];
  st = bwd_cfg(kern, p, L.K, (unsigned)(p.s.nclusters * L.K), reinterpret_cast<cudaStream_t>(stream),
               &cfg, attr);
  if (st) return st;
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, a), "leapfrog_bwd_kernel launch");
}

}  // extern "C"

