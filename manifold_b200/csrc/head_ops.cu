// C ABI of the single-head operators in head_ops.cuh: the leapfrog step with
// the input-gate friction term and the toroidal topology, the Christoffel
// contraction on the torus, and the backward passes of both.
#include "../../include/gfn_b200.h"
#include "head_ops_host.h"

using namespace gfn;
using namespace gfn_abi;

namespace {

using namespace gfn_head_ops;

template <int RK, int EPL>
struct FwdLaunch {
  static int run(const hops::Params& p, size_t smem, cudaStream_t s) {
    cudaError_t e = cudaFuncSetAttribute(hops::head_fwd_kernel<RK, EPL>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_status(e, "head op: shared memory attribute");
    const unsigned grid = (unsigned)((p.B + hops::WARPS - 1) / hops::WARPS);
    hops::head_fwd_kernel<RK, EPL><<<grid, hops::WARPS * 32, smem, s>>>(p);
    return launch_status("head_fwd_kernel");
  }
};

template <int RK, int EPL>
struct BwdLaunch {
  static int run(const hops::Params& p, size_t smem, cudaStream_t s) {
    cudaError_t e = cudaFuncSetAttribute(hops::head_bwd_kernel<RK, EPL>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_status(e, "head op: shared memory attribute");
    const unsigned grid = (unsigned)((p.B + hops::WARPS - 1) / hops::WARPS);
    hops::head_bwd_kernel<RK, EPL><<<grid, hops::WARPS * 32, smem, s>>>(p);
    return launch_status("head_bwd_kernel");
  }
};

template <int RK, int EPL>
struct GammaBwdLaunch {
  static int run(const hops::Params& p, size_t smem, cudaStream_t s) {
    cudaError_t e = cudaFuncSetAttribute(hops::gamma_bwd_kernel<RK, EPL>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_status(e, "head op: shared memory attribute");
    const unsigned grid = (unsigned)((p.B + hops::WARPS - 1) / hops::WARPS);
    hops::gamma_bwd_kernel<RK, EPL><<<grid, hops::WARPS * 32, smem, s>>>(p);
    return launch_status("gamma_bwd_kernel");
  }
};

void outer_sum(const float* A, long long sA, const float* Bm, long long sB, long long modB, int I, int J,
               long long N, float* out, cudaStream_t s) {
  const int n = I * J;
  hops::outer_sum_kernel<<<(n + 127) / 128, 128, 0, s>>>(A, sA, Bm, sB, modB, I, J, N, out);
}

}  // namespace

extern "C" {

int gfn_leapfrog_fused_gated(const float* x, const float* v, const float* f, const float* U, const float* W,
                             const float* W_forget, const float* b_forget, const float* W_input, float* x_new,
                             float* v_new, float dt, const float* dt_scales, int dt_scales_count, int batch,
                             int dim, int rank, int steps, int topology, float plasticity, float R_val,
                             float r_val, gfn_stream_t stream) {
  int st = check_common("leapfrog", batch, dim, rank, topology, plasticity, R_val, r_val);
  if (st) return st;
  if (!x || !v || !x_new || !v_new || (topology == 0 && (!U || !W)))
    return fail(GFN_ERR_INVALID, "leapfrog: NULL operand");
  if (steps < 0) return fail(GFN_ERR_INVALID, "leapfrog: steps %d", steps);
  if (dt_scales && dt_scales_count != 1 && dt_scales_count != batch)
    return fail(GFN_ERR_INVALID, "leapfrog: dt_scales_count %d (need 1 or batch)", dt_scales_count);
  if (b_forget && !W_forget) return fail(GFN_ERR_INVALID, "leapfrog: b_forget without W_forget");
  if (W_input && !f) return fail(GFN_ERR_INVALID, "leapfrog: W_input without a force");
  if (batch == 0) return GFN_OK;
  hops::Params p = {};
  p.x = x; p.v = v; p.f = f; p.U = topology ? nullptr : U; p.W = topology ? nullptr : W;
  p.Wf = W_forget; p.bf = b_forget; p.Wi = W_input;
  p.dt_scale = dt_scales; p.dt_scale_n = dt_scales_count; p.dt = dt; p.steps = steps;
  p.topo = topology; p.R = R_val; p.r = r_val; p.B = batch; p.hd = dim; p.fin = topology ? 2 * dim : dim;
  p.x_out = x_new; p.v_out = v_new;
  if (topology) rank = 4;
  const size_t smem = smem_bytes(dim, rank, p.fin, W_forget != nullptr, W_input != nullptr);
  if (smem > kMaxSmem) return fail(GFN_ERR_RESOURCES, "leapfrog: head dim %d too large for the gates", dim);
  return dispatch<FwdLaunch>(rank, dim, p, smem, reinterpret_cast<cudaStream_t>(stream));
}

int gfn_christoffel_torus(const float* v, const float* x, float* gamma, int batch, int dim, float R_val,
                          float r_val, gfn_stream_t stream) {
  int st = check_common("christoffel (torus)", batch, dim, 4, 1, 0.f, R_val, r_val);
  if (st) return st;
  if (!v || !x || !gamma) return fail(GFN_ERR_INVALID, "christoffel (torus): NULL operand");
  if (batch == 0) return GFN_OK;
  hops::Params p = {};
  p.v = v; p.x = x; p.gamma_out = gamma; p.topo = 1; p.R = R_val; p.r = r_val; p.B = batch; p.hd = dim;
  p.fin = dim;
  return dispatch<FwdLaunch>(4, dim, p, smem_bytes(dim, 4, dim, false, false),
                             reinterpret_cast<cudaStream_t>(stream));
}

long long gfn_christoffel_backward_workspace_floats(int batch, int dim, int rank) {
  if (batch < 0 || dim <= 0 || rank <= 0) return -1;
  return (long long)batch * (dim + 2 * rank);
}

int gfn_christoffel_backward(const float* grad_gamma, const float* v, const float* U, const float* W,
                             const float* x, const float* V_w, float* grad_v, float* grad_U, float* grad_W,
                             float* grad_x, float* grad_V_w, int batch, int dim, int rank, float plasticity,
                             float sing_thresh, float sing_strength, int topology, float R_val, float r_val,
                             float* workspace, long long workspace_floats, gfn_stream_t stream) {
  (void)sing_thresh; (void)sing_strength;
  int st = check_common("christoffel backward", batch, dim, rank, topology, plasticity, R_val, r_val);
  if (st) return st;
  if (V_w || grad_V_w) return fail(GFN_ERR_UNSUPPORTED, "christoffel backward: singularity potential");
  if (!grad_gamma || !v || !grad_v) return fail(GFN_ERR_INVALID, "christoffel backward: NULL operand");
  if (topology == 1 && !x) return fail(GFN_ERR_INVALID, "christoffel backward: the torus needs x");
  if (topology == 0 && (!U || !W || !grad_U || !grad_W || !workspace))
    return fail(GFN_ERR_INVALID, "christoffel backward: NULL U/W/grad/workspace");
  if (topology == 0 && workspace_floats < gfn_christoffel_backward_workspace_floats(batch, dim, rank))
    return fail(GFN_ERR_INVALID, "christoffel backward: workspace too small");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (topology) rank = 4;
  if (batch == 0) {
    cudaError_t e = cudaSuccess;
    if (topology == 0) e = cudaMemsetAsync(grad_U, 0, (size_t)dim * rank * 4, s);
    if (e == cudaSuccess && topology == 0) e = cudaMemsetAsync(grad_W, 0, (size_t)dim * rank * 4, s);
    return cuda_status(e, "christoffel backward: zero gradients");
  }
  hops::Params p = {};
  p.v = v; p.x = x; p.U = topology ? nullptr : U; p.W = topology ? nullptr : W; p.gg_in = grad_gamma;
  p.gv = grad_v; p.gx = grad_x; p.ws = workspace; p.topo = topology; p.R = R_val; p.r = r_val; p.B = batch;
  p.hd = dim; p.fin = dim;
  st = dispatch<GammaBwdLaunch>(rank, dim, p, smem_bytes(dim, rank, dim, false, false), s);
  if (st || topology) return st;
  const long long SR = dim + 2 * rank;
  // grad_U[k][q] = sum_b v[b][k] gp_b[q];  grad_W[k][q] = sum_b gpre_b[k] e_b[q]
  outer_sum(v, dim, workspace + dim + rank, SR, 1LL << 62, dim, rank, batch, grad_U, s);
  outer_sum(workspace, SR, workspace + dim, SR, 1LL << 62, dim, rank, batch, grad_W, s);
  return launch_status("christoffel backward sums");
}

long long gfn_leapfrog_step_backward_workspace_floats(int batch, int dim, int rank, int steps, int topology) {
  if (batch < 0 || dim <= 0 || rank <= 0 || steps < 0) return -1;
  const int fin = topology ? 2 * dim : dim;
  return (long long)steps * batch * (2LL * dim + 2LL * hops::signal_floats(dim, fin, rank));
}

int gfn_leapfrog_backward(const float* grad_x_new, const float* grad_v_new, const float* x, const float* v,
                          const float* f, const float* U, const float* W, const float* W_forget,
                          const float* b_forget, const float* W_input, float* grad_x, float* grad_v,
                          float* grad_f, float* grad_U, float* grad_W, float* grad_W_forget,
                          float* grad_b_forget, float* grad_W_input, float* grad_dt_scale, int batch, int dim,
                          int rank, float dt,
                          const float* dt_scales, int dt_scales_count, int steps, int topology, float R_val,
                          float r_val, float* workspace, long long workspace_floats, gfn_stream_t stream) {
  int st = check_common("leapfrog backward", batch, dim, rank, topology, 0.f, R_val, r_val);
  if (st) return st;
  if (!x || !v || !grad_x || !grad_v || (topology == 0 && (!U || !W || !grad_U || !grad_W)))
    return fail(GFN_ERR_INVALID, "leapfrog backward: NULL operand");
  if (steps < 0) return fail(GFN_ERR_INVALID, "leapfrog backward: steps %d", steps);
  if (dt_scales && dt_scales_count != 1 && dt_scales_count != batch)
    return fail(GFN_ERR_INVALID, "leapfrog backward: dt_scales_count %d", dt_scales_count);
  if (b_forget && !W_forget) return fail(GFN_ERR_INVALID, "leapfrog backward: b_forget without W_forget");
  if (W_forget && (!grad_W_forget || !grad_b_forget))
    return fail(GFN_ERR_INVALID, "leapfrog backward: W_forget needs grad_W_forget and grad_b_forget");
  if (W_input && (!f || !grad_W_input))
    return fail(GFN_ERR_INVALID, "leapfrog backward: W_input needs the force and grad_W_input");
  if (workspace_floats < gfn_leapfrog_step_backward_workspace_floats(batch, dim, rank, steps, topology) ||
      (!workspace && steps > 0 && batch > 0))
    return fail(GFN_ERR_INVALID, "leapfrog backward: workspace too small");
  const int fin = topology ? 2 * dim : dim;
  if (topology) rank = 4;
  const size_t smem = smem_bytes(dim, rank, fin, W_forget != nullptr, W_input != nullptr);
  if (smem > kMaxSmem) return fail(GFN_ERR_RESOURCES, "leapfrog backward: head dim %d too large", dim);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const long long N = 2LL * steps * batch;  // signal records
  if (batch == 0 || steps == 0) {
    // identity map: gradients pass through, parameters get zero
    cudaError_t e = cudaSuccess;
    const size_t bd = (size_t)batch * dim * 4;
    if (bd && grad_x_new) e = cudaMemcpyAsync(grad_x, grad_x_new, bd, cudaMemcpyDeviceToDevice, s);
    else if (bd) e = cudaMemsetAsync(grad_x, 0, bd, s);
    if (e == cudaSuccess && bd && grad_v_new) e = cudaMemcpyAsync(grad_v, grad_v_new, bd, cudaMemcpyDeviceToDevice, s);
    else if (e == cudaSuccess && bd) e = cudaMemsetAsync(grad_v, 0, bd, s);
    if (e == cudaSuccess && grad_f && bd) e = cudaMemsetAsync(grad_f, 0, bd, s);
    if (e == cudaSuccess && topology == 0) e = cudaMemsetAsync(grad_U, 0, (size_t)dim * rank * 4, s);
    if (e == cudaSuccess && topology == 0) e = cudaMemsetAsync(grad_W, 0, (size_t)dim * rank * 4, s);
    if (e == cudaSuccess && W_forget) e = cudaMemsetAsync(grad_W_forget, 0, (size_t)dim * fin * 4, s);
    if (e == cudaSuccess && W_forget) e = cudaMemsetAsync(grad_b_forget, 0, (size_t)dim * 4, s);
    if (e == cudaSuccess && W_input) e = cudaMemsetAsync(grad_W_input, 0, (size_t)dim * dim * 4, s);
    if (e == cudaSuccess && grad_dt_scale && batch) e = cudaMemsetAsync(grad_dt_scale, 0, (size_t)batch * 4, s);
    return cuda_status(e, "leapfrog backward: empty problem");
  }
  hops::Params p = {};
  p.x = x; p.v = v; p.f = f; p.U = topology ? nullptr : U; p.W = topology ? nullptr : W;
  p.Wf = W_forget; p.bf = b_forget; p.Wi = W_input;
  p.dt_scale = dt_scales; p.dt_scale_n = dt_scales_count; p.dt = dt; p.steps = steps;
  p.topo = topology; p.R = R_val; p.r = r_val; p.B = batch; p.hd = dim; p.fin = fin;
  p.gx_in = grad_x_new; p.gv_in = grad_v_new; p.gx = grad_x; p.gv = grad_v; p.gf = grad_f; p.ws = workspace;
  p.gdt = grad_dt_scale;
  st = dispatch<BwdLaunch>(rank, dim, p, smem, s);
  if (st) return st;
  const float* sig = workspace + (long long)steps * batch * 2 * dim;
  const long long SR = hops::signal_floats(dim, fin, rank);
  const long long big = 1LL << 62;
  // record: [v point | gpre | gz | feat | e | gp]
  if (topology == 0) {
    outer_sum(sig, SR, sig + 3 * dim + fin + rank, SR, big, dim, rank, N, grad_U, s);
    outer_sum(sig + dim, SR, sig + 3 * dim + fin, SR, big, dim, rank, N, grad_W, s);
  }
  if (W_forget) {
    outer_sum(sig + 2 * dim, SR, sig + 3 * dim, SR, big, dim, fin, N, grad_W_forget, s);
    outer_sum(sig + 2 * dim, SR, nullptr, 0, big, dim, 1, N, grad_b_forget, s);
  }
  // the force of record n is row n % batch (records are [steps][2][batch])
  if (W_input) outer_sum(sig + 2 * dim, SR, f, dim, batch, dim, dim, N, grad_W_input, s);
  return launch_status("leapfrog backward sums");
}

}  // extern "C"
