// C ABI of the multi-scheme integrator kernel (head_ops.cuh:
// integrate_kernel): the reference's non-leapfrog integrators and the
// leapfrog over every head of a layer in one launch.
#include "../../include/gfn_b200.h"
#include "head_ops_host.h"

using namespace gfn;
using namespace gfn_abi;
using namespace gfn_head_ops;

namespace {

template <int EPL>
int integ_launch(const hops::IntegArgs& ia, size_t smem, cudaStream_t s) {
  cudaError_t e = cudaFuncSetAttribute(hops::integrate_kernel<EPL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return cuda_status(e, "integrator: shared memory attribute");
  const dim3 grid((unsigned)((ia.p.B + hops::WARPS - 1) / hops::WARPS), (unsigned)ia.heads);
  hops::integrate_kernel<EPL><<<grid, hops::WARPS * 32, smem, s>>>(ia);
  return launch_status("integrate_kernel");
}

// Scheme coefficients as float32 (the reference multiplies its Python-float
// coefficients into float32 tensors).
void scheme_coeffs(int scheme, float* c) {
  for (int i = 0; i < 20; ++i) c[i] = 0.f;
  const double cbrt2 = 1.2599210498948732;  // 2^(1/3)
  if (scheme == hops::kYoshida) {  // gfn/integrators/symplectic/yoshida.py:24-35
    const double w1 = 1.0 / (2.0 - cbrt2), w0 = -cbrt2 / (2.0 - cbrt2);
    const double cc[4] = {w1 / 2.0, (w0 + w1) / 2.0, (w0 + w1) / 2.0, w1 / 2.0};
    const double dd[3] = {w1, w0, w1};
    for (int i = 0; i < 4; ++i) c[i] = (float)cc[i];
    for (int i = 0; i < 3; ++i) c[5 + i] = (float)dd[i];
  } else if (scheme == hops::kForestRuth) {  // forest_ruth.py:28-38
    const double th = 1.0 / (2.0 - cbrt2);
    const double cc[4] = {th / 2.0, (1.0 - th) / 2.0, (1.0 - th) / 2.0, th / 2.0};
    const double dd[3] = {th, 1.0 - 2.0 * th, th};
    for (int i = 0; i < 4; ++i) c[i] = (float)cc[i];
    for (int i = 0; i < 3; ++i) c[5 + i] = (float)dd[i];
  } else if (scheme == hops::kOmelyan) {  // omelyan.py:26-41
    const double xi = 0.1786178958448091, lam = -0.2123418310626054, chi = -0.06626458266981849;
    const double cc[5] = {xi, chi, 1.0 - 2.0 * (chi + xi), chi, xi};
    const double dd[4] = {(1.0 - 2.0 * lam) / 2.0, lam, lam, (1.0 - 2.0 * lam) / 2.0};
    for (int i = 0; i < 5; ++i) c[i] = (float)cc[i];
    for (int i = 0; i < 4; ++i) c[5 + i] = (float)dd[i];
  } else if (scheme == hops::kDormandPrince) {  // dormand_prince.py:30-41
    const double a[15] = {1.0 / 5,
                          3.0 / 40, 9.0 / 40,
                          44.0 / 45, -56.0 / 15, 32.0 / 9,
                          19372.0 / 6561, -25360.0 / 2187, 64448.0 / 6561, -212.0 / 729,
                          9017.0 / 3168, -355.0 / 33, 46732.0 / 5247, 49.0 / 176, -5103.0 / 18656};
    const double b[5] = {35.0 / 384, 500.0 / 1113, 125.0 / 192, -2187.0 / 6784, 11.0 / 84};
    for (int i = 0; i < 15; ++i) c[i] = (float)a[i];
    for (int i = 0; i < 5; ++i) c[15 + i] = (float)b[i];
  }
}

}  // namespace

extern "C" {

int gfn_integrator_heads(int scheme, const float* x, const float* v, const float* f, const float* U_stack,
                         const float* W_stack, const float* W_forget_stack, const float* b_forget_stack,
                         const float* W_input_stack, float* x_new, float* v_new, float dt, const float* dt_scales,
                         int dt_scales_count, int batch, int heads, int head_dim, int rank, int steps, int topology,
                         float R_val, float r_val, float plasticity, const float* V_stack, const float* V_bias,
                         int singularity_mode, float sing_thresh, float sing_strength, gfn_stream_t stream) {
  if (topology == 0 && (rank < 1 || rank > 16))
    return fail(GFN_ERR_UNSUPPORTED, "integrator: rank %d not in [1, 16]", rank);
  int st = check_common("integrator", batch, head_dim, topology ? 4 : 4, topology, 0.f, R_val, r_val);
  if (st) return st;
  if (scheme < hops::kEuler || scheme > hops::kLeapfrog)
    return fail(GFN_ERR_UNSUPPORTED, "integrator: scheme %d", scheme);
  if (heads < 1) return fail(GFN_ERR_INVALID, "integrator: heads %d", heads);
  if (!x || !v || !x_new || !v_new || (topology == 0 && (!U_stack || !W_stack)))
    return fail(GFN_ERR_INVALID, "integrator: NULL operand");
  if (steps < 0) return fail(GFN_ERR_INVALID, "integrator: steps %d", steps);
  const long long per_rh = (long long)batch * heads;
  if (dt_scales && dt_scales_count != 1 && dt_scales_count != (heads > 1 ? heads : batch) &&
      dt_scales_count != per_rh)
    return fail(GFN_ERR_INVALID, "integrator: dt_scales_count %d (need 1, one per %s, or batch * heads)",
                dt_scales_count, heads > 1 ? "head" : "row");
  if (singularity_mode < 0 || singularity_mode > 2 || (singularity_mode && !V_stack))
    return fail(GFN_ERR_INVALID, "integrator: singularity mode %d needs V_stack", singularity_mode);
  if (b_forget_stack && !W_forget_stack) return fail(GFN_ERR_INVALID, "integrator: b_forget without W_forget");
  if (W_input_stack && !f) return fail(GFN_ERR_INVALID, "integrator: W_input without a force");
  if (batch == 0) return GFN_OK;
  if (topology) rank = 4;
  const int fin = topology ? 2 * head_dim : head_dim;
  hops::IntegArgs ia = {};
  hops::Params& p = ia.p;
  p.x = x; p.v = v; p.f = f; p.U = topology ? nullptr : U_stack; p.W = topology ? nullptr : W_stack;
  p.Wf = W_forget_stack; p.bf = b_forget_stack; p.Wi = W_input_stack;
  p.dt_scale = dt_scales; p.dt_scale_n = dt_scales_count; p.dt = dt; p.steps = steps;
  p.topo = topology; p.R = R_val; p.r = r_val; p.B = batch; p.hd = head_dim; p.fin = fin;
  p.x_out = x_new; p.v_out = v_new;
  ia.scheme = scheme; ia.heads = heads; ia.ld = (long long)heads * head_dim;
  ia.hU = (long long)head_dim * rank; ia.hWf = (long long)head_dim * fin; ia.hWi = (long long)head_dim * head_dim;
  ia.hb = head_dim;
  ia.dts_row_head = dt_scales && heads > 1 && dt_scales_count == per_rh && per_rh != heads;
  ia.dts_per_head = dt_scales && heads > 1 && dt_scales_count == heads;
  ia.plasticity = plasticity;
  ia.Vw = singularity_mode ? V_stack : nullptr;
  ia.Vb = singularity_mode ? V_bias : nullptr;
  ia.sing_hard = singularity_mode == 2;
  ia.sing_thr = sing_thresh;
  ia.sing_strength = sing_strength;
  scheme_coeffs(scheme, ia.c);
  const size_t smem = smem_bytes(head_dim, rank, fin, W_forget_stack != nullptr, W_input_stack != nullptr);
  if (smem > kMaxSmem) return fail(GFN_ERR_RESOURCES, "integrator: head dim %d too large for the gates", head_dim);
  ia.rank = rank;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
  switch (epl_for(head_dim)) {
    case 1: return integ_launch<1>(ia, smem, cs);
    case 2: return integ_launch<2>(ia, smem, cs);
    case 4: return integ_launch<4>(ia, smem, cs);
    default: return integ_launch<8>(ia, smem, cs);
  }
}

}  // extern "C"
