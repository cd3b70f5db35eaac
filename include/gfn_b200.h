/*
 * gfn_b200 -- C ABI of the B200 (sm_100a) kernels for the recurrent
 * geodesic-flow hot path of Manifold-Laboratory/manifold (package `gfn`).
 *
 * Conventions
 *  - Plain device pointers, contiguous row-major float32 unless stated.
 *    The caller owns and allocates every buffer; no entry point allocates
 *    device memory.  Optional inputs are NULL.
 *  - Every entry point is asynchronous on `stream` and returns a status
 *    (GFN_OK == 0).  Arguments are validated before anything is launched;
 *    gfn_last_error_message() describes the last failure of this thread.
 *  - Device-side faults are never raised with a trap: kernels record them in
 *    a device error word (gfn_get_device_error) and finish their launch.
 *  - `rank` is the per-head Christoffel rank (U.size(-1)), as in the
 *    reference's launchers; `heads * head_dim == dim`.
 *  - Thread safety: entry points may be called from several host threads.
 *    The library's per-device cuBLAS handles (used only by the library-GEMM
 *    mixing modes and the readout GEMMs) are locked for the whole call that
 *    uses them; the default tensor-core paths use no library handle.
 *
 * Each function names the reference entry point it replaces
 * (gfn/cuda/cuda_kernels.cpp is the reference's pybind/C boundary).
 */
#ifndef GFN_B200_H
#define GFN_B200_H

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* gfn_stream_t; /* == cudaStream_t */

enum {
  GFN_OK = 0,
  GFN_ERR_INVALID = 1,     /* bad size / null pointer */
  GFN_ERR_UNSUPPORTED = 2, /* a configuration this build does not implement */
  GFN_ERR_ALIGN = 3,       /* pointer not 16-byte aligned where required */
  GFN_ERR_CUDA = 4,        /* a CUDA runtime call or launch failed */
  GFN_ERR_RESOURCES = 5,   /* no launch plan fits the device (shared memory) */
};

/* Device error bits recorded by kernels. */
enum {
  GFN_DEVERR_MBAR_TIMEOUT = 1, /* a bounded wait for a bulk copy gave up */
  GFN_DEVERR_BAD_TOKEN = 2,    /* a token id outside [0, vocab) (force 0 used) */
  GFN_DEVERR_F16_RANGE = 4,    /* layered GFN_MIX_SPLIT_F16: an activation |x| >= 2^15 */
};

const char* gfn_status_string(int status);
const char* gfn_last_error_message(void);
const char* gfn_build_info(void);

/* Synchronises `stream`, stores the device error bits in *bits and, when
 * reset != 0, clears them. */
int gfn_get_device_error(int* bits, int reset, gfn_stream_t stream);

/* ------------------------------------------------------------------------
 * Christoffel contraction Gamma(v) = 20 tanh(((vU)^2 s) W^T / 20),
 * s = 1/(1 + |vU| + 1e-6), for one head.
 * Replaces launch_christoffel_fused (gfn/cuda/cuda_kernels.cpp:14-19) for the
 * configuration the leapfrog path uses: x/V_w NULL, plasticity 0,
 * topology 0 (anything else returns GFN_ERR_UNSUPPORTED).
 * Semantics: gfn/geometry/lowrank.py:93-98,125-127.
 * v [batch, dim], U, W [dim, rank], gamma [batch, dim].
 */
int gfn_christoffel_fused(const float* v, const float* U, const float* W, float* gamma,
                          const float* x, const float* V_w, int batch, int dim, int rank,
                          float plasticity, float sing_thresh, float sing_strength, int topology,
                          float R_val, float r_val, gfn_stream_t stream);

/* ------------------------------------------------------------------------
 * One head's leapfrog (kick-drift-kick with implicit friction), `steps`
 * times.  Replaces launch_leapfrog_fused (gfn/cuda/cuda_kernels.cpp:74-83).
 * Semantics: gfn/integrators/symplectic/leapfrog.py:50-114.
 * x, v, f [batch, dim] (f may be NULL: zero force); U, W [dim, rank];
 * W_forget [dim, dim] + b_forget [dim] (NULL: no friction);
 * dt_scales: NULL (1.0), 1 value, or `batch` values (dt_scales_count).
 */
int gfn_leapfrog_fused(const float* x, const float* v, const float* f, const float* U,
                       const float* W, const float* W_forget, const float* b_forget, float* x_new,
                       float* v_new, float dt, const float* dt_scales, int dt_scales_count,
                       int batch, int dim, int rank, int steps, int topology, float plasticity,
                       float R_val, float r_val, gfn_stream_t stream);

/* ------------------------------------------------------------------------
 * One head's leapfrog with the full friction gate and both topologies.
 * Same operation as launch_leapfrog_fused (gfn/cuda/cuda_kernels.cpp:74-83)
 * plus the two terms that entry cannot express:
 *   - the input gate: mu = 5 sigmoid((feat(x) W_forget^T + b_forget) + f W_input^T),
 *     the friction the reference's Christoffel computes when no forget stack
 *     is given (gfn/geometry/lowrank.py:114-123); W_input [dim, dim] or NULL;
 *   - topology 1 (torus): Gamma of gfn/geometry/toroidal.py:70-108 (U, W
 *     unused, R_val / r_val the radii), friction features [sin x, cos x]
 *     (W_forget [dim, 2 dim]) and x wrapped into [0, 2 pi) after the drift
 *     (gfn/integrators/symplectic/leapfrog.py:74-91, gfn/geometry/boundaries.py:4-17).
 * dim <= 256; rank 4, 8 or 16 (topology 0).
 */
int gfn_leapfrog_fused_gated(const float* x, const float* v, const float* f, const float* U,
                             const float* W, const float* W_forget, const float* b_forget,
                             const float* W_input, float* x_new, float* v_new, float dt,
                             const float* dt_scales, int dt_scales_count, int batch, int dim,
                             int rank, int steps, int topology, float plasticity, float R_val,
                             float r_val, gfn_stream_t stream);

/* Toroidal Christoffel term for one head: the topology-1 form of
 * launch_christoffel_fused (gfn/cuda/cuda_kernels.cpp:14-19), with the
 * semantics of gfn/geometry/toroidal.py:70-108.  v, x, gamma [batch, dim]. */
int gfn_christoffel_torus(const float* v, const float* x, float* gamma, int batch, int dim,
                          float R_val, float r_val, gfn_stream_t stream);

/* ------------------------------------------------------------------------
 * The reference's other integrators, and the leapfrog, over every head of a
 * layer in one launch.  Replaces launch_euler_fused, launch_heun_fused,
 * launch_rk4_fused, launch_verlet_fused, launch_yoshida_fused,
 * launch_dormand_prince_fused (gfn/cuda/cuda_kernels.cpp:85-126; the
 * reference's generic_integrator_cuda takes the scheme the same way) and the
 * Python-only Forest-Ruth and Omelyan integrators.  scheme:
 *   0 Euler (gfn/integrators/runge_kutta/euler.py:46-62)
 *   1 Heun (runge_kutta/heun.py:46-77)      2 RK4 (runge_kutta/rk4.py:46-82)
 *   3 Verlet (symplectic/verlet.py:41-72)   4 Yoshida (symplectic/yoshida.py:24-86)
 *   5 Forest-Ruth (symplectic/forest_ruth.py:28-89)
 *   6 Omelyan PEFRL (symplectic/omelyan.py:26-96)
 *   7 Dormand-Prince 5th order (runge_kutta/dormand_prince.py:26-122)
 *   8 leapfrog (symplectic/leapfrog.py:50-114, implicit friction)
 * Schemes 0-7 step with a(x, v) = f - C(v, x), C the Christoffel term in its
 * combined form: low-rank 20 tanh((((vU)^2 s) W^T + mu v) / 20)
 * (gfn/geometry/lowrank.py:128-131), torus Gamma_torus + mu v
 * (gfn/geometry/toroidal.py:146-148); mu = 5 sigmoid((feat(x) W_forget^T +
 * b_forget) + f W_input^T), 0 without W_forget.
 * x, v, f, x_new, v_new [batch, heads * head_dim] (head h at columns
 * h * head_dim); stacks per head: U, W [heads, head_dim, rank],
 * W_forget [heads, head_dim, fin] (fin = head_dim, 2 head_dim on the torus),
 * b_forget [heads, head_dim], W_input [heads, head_dim, head_dim].
 * dt_scales: NULL, 1 value, one per head (heads > 1), one per row (heads == 1),
 * or [batch][heads] (the dynamic-time gate, gfn/layers/base.py:222-229).
 * Active inference (the Christoffel term times M, gfn/geometry/reactive.py:53-81,
 * gfn/geometry/toroidal.py:126-141): plasticity != 0 multiplies by
 * 1 + plasticity tanh(mean_k v_k^2); singularity_mode 1 (low-rank: soft,
 * sigmoid(10 (p - thresh))) or 2 (torus: p > thresh) multiplies by
 * 1 + s (strength - 1), p = sigmoid(feat(x) . V + b), V_stack [heads, fin],
 * V_bias [heads] or NULL; singularity_mode 0 leaves V unused.
 * head_dim <= 256 (the gates' weights must fit in shared memory).
 */
int gfn_integrator_heads(int scheme, const float* x, const float* v, const float* f,
                         const float* U_stack, const float* W_stack, const float* W_forget_stack,
                         const float* b_forget_stack, const float* W_input_stack, float* x_new,
                         float* v_new, float dt, const float* dt_scales, int dt_scales_count,
                         int batch, int heads, int head_dim, int rank, int steps, int topology,
                         float R_val, float r_val, float plasticity, const float* V_stack,
                         const float* V_bias, int singularity_mode, float sing_thresh,
                         float sing_strength, gfn_stream_t stream);

/* ------------------------------------------------------------------------
 * Backward of the Christoffel term.  Replaces launch_christoffel_backward
 * (gfn/cuda/cuda_kernels.cpp:21-29) for plasticity 0 and no singularity
 * potential (V_w / grad_V_w must be NULL).
 * topology 0: grad_v = dGamma/dv^T grad_gamma, grad_U / grad_W [dim, rank]
 *   summed over the batch (overwritten, fixed summation order), grad_x
 *   (optional) zero; needs gfn_christoffel_backward_workspace_floats floats.
 * topology 1: grad_v and grad_x (x required); U, W, grad_U, grad_W unused.
 */
long long gfn_christoffel_backward_workspace_floats(int batch, int dim, int rank);
int gfn_christoffel_backward(const float* grad_gamma, const float* v, const float* U,
                             const float* W, const float* x, const float* V_w, float* grad_v,
                             float* grad_U, float* grad_W, float* grad_x, float* grad_V_w,
                             int batch, int dim, int rank, float plasticity, float sing_thresh,
                             float sing_strength, int topology, float R_val, float r_val,
                             float* workspace, long long workspace_floats, gfn_stream_t stream);

/* ------------------------------------------------------------------------
 * Backward of gfn_leapfrog_fused / gfn_leapfrog_fused_gated (`steps` steps,
 * reverse replay: each step's forward is recomputed from its stored input).
 * Replaces launch_leapfrog_backward (gfn/cuda/cuda_kernels.cpp:123), which
 * takes no friction operands and leaves dU / dW out; this entry returns the
 * gradients of every operand:
 *   grad_x, grad_v [batch, dim] (from grad_x_new / grad_v_new; NULL = 0),
 *   grad_f [batch, dim] (optional), grad_U / grad_W [dim, rank] (topology 0),
 *   grad_W_forget [dim, fin] + grad_b_forget [dim] when W_forget is given,
 *   grad_W_input [dim, dim] when W_input is given.
 * Parameter gradients are batch sums in a fixed order (overwritten).
 * grad_dt_scale (optional, [batch]): dL/d dt_scale of each row (sum the rows
 * for a shared scale).  Workspace:
 * gfn_leapfrog_step_backward_workspace_floats(batch, dim, rank, steps, topology).
 */
long long gfn_leapfrog_step_backward_workspace_floats(int batch, int dim, int rank, int steps,
                                                      int topology);
int gfn_leapfrog_backward(const float* grad_x_new, const float* grad_v_new, const float* x,
                          const float* v, const float* f, const float* U, const float* W,
                          const float* W_forget, const float* b_forget, const float* W_input,
                          float* grad_x, float* grad_v, float* grad_f, float* grad_U,
                          float* grad_W, float* grad_W_forget, float* grad_b_forget,
                          float* grad_W_input, float* grad_dt_scale, int batch, int dim, int rank,
                          float dt,
                          const float* dt_scales, int dt_scales_count, int steps, int topology,
                          float R_val, float r_val, float* workspace, long long workspace_floats,
                          gfn_stream_t stream);

/* ------------------------------------------------------------------------
 * Whole-sequence fused leapfrog recurrence (all tokens x layers x heads in
 * one persistent launch).  The reference has no leapfrog entry here: its
 * launch_recurrent_manifold_fused (gfn/cuda/cuda_kernels.cpp:41-52) is
 * excluded for leapfrog at gfn/model.py:207 and the per-token Python loop
 * (gfn/model.py:377-402 over gfn/layers/base.py:198-338) runs instead; this
 * entry computes exactly that loop.
 *
 * Weights go through gfn_leapfrog_pack first (once per weight update).
 *
 * x_init, v_init: initial state, row r at x_init + r*state_row_stride
 *   (stride 0 broadcasts one [dim] row, as the model's x0/v0 parameters).
 * Forces, exactly one of:
 *   forces_f32 [batch, seq_len, dim] float32,
 *   forces_bf16 [batch, seq_len, dim] bfloat16 (raw uint16 storage),
 *   token_ids [batch, seq_len] int64 + embed_table [vocab, dim] (fused
 *   nn.Embedding gather, gfn/model.py:55,163).
 * mask [batch, seq_len] or NULL (force_t *= mask_t, gfn/model.py:381).
 * Outputs (any may be NULL): x_seq, v_seq [batch, seq_len, dim] = state
 * after the last layer at every token; x_final, v_final [batch, dim].
 * base_dt: the layers' base_dt; heads == 1 means no head mixing.
 */
int gfn_leapfrog_sequence_forward(const float* x_init, const float* v_init,
                                  long long state_row_stride, const float* forces_f32,
                                  const void* forces_bf16, const long long* token_ids,
                                  const float* embed_table, long long vocab, const float* mask,
                                  const float* packed, long long packed_floats, int batch,
                                  int seq_len, int dim, int heads, int rank, int num_layers,
                                  float base_dt, float* x_seq, float* v_seq, float* x_final,
                                  float* v_final, gfn_stream_t stream);

/* Number of floats of the packed weight buffer for these shapes. */
long long gfn_leapfrog_pack_floats(int dim, int heads, int rank, int num_layers);

/* Pack the stacked layer parameters (the stacks the reference builds for
 * launch_recurrent_manifold_fused, gfn/model.py:222-293, plus the mixing
 * parameters of every layer) into `packed`:
 *   U_stack, W_stack [num_layers*heads, head_dim, rank]
 *   W_forget_stack [num_layers*heads, head_dim, head_dim], b_forget_stack [num_layers*heads, head_dim]
 *   dt_params [num_layers*heads]           (raw; softplus is applied in-kernel)
 *   mix_x_w/mix_v_w [num_layers, dim, dim] out_proj weights ([out, in]),
 *   mix_x_b/mix_v_b [num_layers, dim] biases, norm_x_w/norm_v_w [num_layers, dim]
 *   RMSNorm weights (all six NULL when heads == 1). */
int gfn_leapfrog_pack(const float* U_stack, const float* W_stack, const float* W_forget_stack,
                      const float* b_forget_stack, const float* dt_params, const float* mix_x_w,
                      const float* mix_x_b, const float* norm_x_w, const float* mix_v_w,
                      const float* mix_v_b, const float* norm_v_w, int dim, int heads, int rank,
                      int num_layers, float* packed, long long packed_floats, gfn_stream_t stream);

/* Testing/profiling aid: when device_counters (12 int64 on the device) is
 * non-NULL, later sequence launches record per-phase clock64 cycle totals
 * of CTA 0 there (head wait, head step + sends, exchange wait, mixing,
 * reduction, norm exchange, norm, token I/O, unused x3, layer steps).
 * NULL turns it off.  Not thread-safe; no reference counterpart. */
int gfn_debug_set_phase_profile(long long* device_counters);

/* Launch plan the sequence kernel would use for `batch` rows:
 * out[0..7] = cluster size K, rows per cluster, clusters, shared bytes,
 * k-chunk, ring slots, max co-resident clusters, k-split lanes. */
int gfn_leapfrog_plan(int batch, int dim, int heads, int rank, int num_layers, int* out8);

/* ------------------------------------------------------------------------
 * Training (BPTT).  The reference trains this path with torch autograd
 * through its per-token loop (gfn/model.py:377-402, train mode) -- its CUDA
 * backwards launch_leapfrog_backward (gfn/cuda/cuda_kernels.cpp:123) and
 * launch_recurrent_manifold_backward (:54-72) are incomplete or unused for
 * leapfrog.  These entries give the same gradients.
 *
 * Training pack: the inference pack plus the untransposed forget-gate weight
 * and transposed mixing chunks (same arguments as gfn_leapfrog_pack). */
long long gfn_leapfrog_pack_train_floats(int dim, int heads, int rank, int num_layers);
int gfn_leapfrog_pack_train(const float* U_stack, const float* W_stack,
                            const float* W_forget_stack, const float* b_forget_stack,
                            const float* dt_params, const float* mix_x_w, const float* mix_x_b,
                            const float* norm_x_w, const float* mix_v_w, const float* mix_v_b,
                            const float* norm_v_w, int dim, int heads, int rank, int num_layers,
                            float* packed, long long packed_floats, gfn_stream_t stream);

/* gfn_leapfrog_sequence_forward on the training pack that also stores, for
 * every layer step, what the backward replays from: traj holds
 * [2][num_layers][seq_len][batch][dim] the step's input state (x then v),
 * then [2][num_layers][seq_len][batch][dim] its head-mixing outputs z_x, z_v
 * (bias included, before the RMSNorm), then [2][num_layers][seq_len][batch]
 * its RMSNorm factors r_x, r_v: 4 L B d NL + 2 L B NL floats. */
int gfn_leapfrog_sequence_forward_train(const float* x_init, const float* v_init,
                                        long long state_row_stride, const float* forces_f32,
                                        const void* forces_bf16, const long long* token_ids,
                                        const float* embed_table, long long vocab,
                                        const float* mask, const float* packed_train,
                                        long long packed_floats, int batch, int seq_len, int dim,
                                        int heads, int rank, int num_layers, float base_dt,
                                        float* x_seq, float* v_seq, float* x_final, float* v_final,
                                        float* traj, gfn_stream_t stream);

/* Reverse replay.  Upstream gradients: gx_seq, gv_seq [batch, seq_len, dim]
 * (dL/dx_seq, dL/dv_seq), gx_final, gv_final [batch, dim]; any may be NULL.
 * Outputs: dx_init, dv_init [batch, dim] (per row), d_forces [batch,
 * seq_len, dim] (may be NULL; already multiplied by the mask), and the
 * per-step gradient signals in `workspace`, from which the host forms the
 * parameter gradients (all tensors row-major, N = num_layers*seq_len*batch
 * rows in [layer][token][row] order, S = N*dim):
 *   [0S,1S) x'  [1S,2S) v'   (head-step outputs = mixing inputs)
 *   [2S,3S) dzx [3S,4S) dzv  (grads of the mixing pre-activations)
 *   [4S,5S) dL/dxn * RMSNorm_x(z) [5S,6S) the v analogue   (norm-weight grads)
 *   [6S,7S) dz1 [7S,8S) dz2  (friction pre-activation grads, kick 1 / kick 2)
 *   [8S,9S) v_half [9S,10S) dg1 [10S,11S) dg2  (Gamma pre-clamp grads)
 *   then 4 blocks of N*heads*rank: q1, q2, dp1, dp2, then N*heads d dt_eff.
 * dWx = sum_n dzx^T x', dbx = sum dzx, dgx = sum block 4, dWf = sum dz1^T x
 * + dz2^T x', dbf = sum (dz1 + dz2), dU = sum v^T dp1 + v_half^T dp2, dW =
 * sum dg1^T q1 + dg2^T q2 (per head), d dt_params = sum d dt_eff * base_dt *
 * sigmoid(dt_params).  head_dim <= 64. */
long long gfn_leapfrog_backward_workspace_floats(int batch, int seq_len, int dim, int heads,
                                                 int rank, int num_layers);
int gfn_leapfrog_sequence_backward(const float* traj, const float* forces_f32,
                                   const void* forces_bf16, const long long* token_ids,
                                   const float* embed_table, long long vocab, const float* mask,
                                   const float* packed_train, long long packed_floats,
                                   const float* gx_seq, const float* gv_seq,
                                   const float* gx_final, const float* gv_final, int batch,
                                   int seq_len, int dim, int heads, int rank, int num_layers,
                                   float base_dt, float* dx_init, float* dv_init, float* d_forces,
                                   float* workspace, long long workspace_floats,
                                   gfn_stream_t stream);

/* ------------------------------------------------------------------------
 * Layer-by-layer form of gfn_leapfrog_sequence_forward for large batches
 * (heads > 1).  Same semantics, operands and results (gfn/model.py:377-402
 * per token, gfn/layers/base.py:198-338 per layer); per token and layer it
 * runs a head-step kernel (previous layer's RMSNorm/saturation fused in) and
 * one batched fp32 GEMM (cuBLAS, no TF32) for both mixing projections, so
 * the d x d mixing runs at GEMM rate when batch * dim is large.
 * `packed` comes from gfn_leapfrog_layered_pack (same operands as
 * gfn_leapfrog_pack); `workspace` holds at least
 * gfn_leapfrog_layered_workspace_floats(batch, dim) floats (16-byte aligned,
 * 256-byte preferred) and includes the GEMM library's workspace, so calls
 * allocate nothing; the first call on a device creates that device's cuBLAS
 * handle (the one allocation, kept for the process lifetime).
 */
long long gfn_leapfrog_layered_pack_floats(int dim, int heads, int rank, int num_layers);
int gfn_leapfrog_layered_pack(const float* U_stack, const float* W_stack,
                              const float* W_forget_stack, const float* b_forget_stack,
                              const float* dt_params, const float* mix_x_w, const float* mix_x_b,
                              const float* norm_x_w, const float* mix_v_w, const float* mix_v_b,
                              const float* norm_v_w, int dim, int heads, int rank, int num_layers,
                              float* packed, long long packed_floats, gfn_stream_t stream);
long long gfn_leapfrog_layered_workspace_floats(int batch, int dim);
/* Arithmetic of the layered path's mixing GEMM (process-wide; returns the
 * previous mode, or a negative status for an unknown mode; mode -1 only
 * returns the current one):
 *   GFN_MIX_UMMA_F16 (default) the split-fp16 products below computed by this
 *     library's own tcgen05 kernel (TMA-fed, TMEM accumulator, three MMAs per
 *     K step: c0 w0 + c0 w1 + c1 w0); needs dim % 64 == 0, otherwise the
 *     call uses GFN_MIX_SPLIT_F16.
 *   GFN_MIX_SPLIT_F16 each operand split into two fp16 pieces
 *     (weights scaled by a power of two per layer so their small pieces stay
 *     normal); the three products of order >= 2^-11 summed by one fp16
 *     tensor-core GEMM with fp32 accumulation (K = 3 * dim): error ~2^-22 per
 *     product, the order of an fp32 SGEMM's own accumulation error.
 *     Activations must stay below 2^15 in magnitude; larger ones set
 *     GFN_DEVERR_F16_RANGE.
 *   GFN_MIX_SPLIT_BF16 each fp32 operand split into three bf16 pieces, the
 *     six cross products of order <= 2^-16 summed by one bf16 tensor-core
 *     GEMM (K = 6 * dim): full fp32 range, twice the GEMM cost.
 *   GFN_MIX_FP32_SIMT  plain fp32 SGEMM on the CUDA cores. */
enum { GFN_MIX_SPLIT_BF16 = 0, GFN_MIX_FP32_SIMT = 1, GFN_MIX_SPLIT_F16 = 2, GFN_MIX_UMMA_F16 = 3 };
int gfn_leapfrog_layered_set_mixing(int mode);
int gfn_leapfrog_layered_forward(const float* x_init, const float* v_init,
                                 long long state_row_stride, const float* forces_f32,
                                 const void* forces_bf16, const long long* token_ids,
                                 const float* embed_table, long long vocab, const float* mask,
                                 const float* packed, long long packed_floats, int batch,
                                 int seq_len, int dim, int heads, int rank, int num_layers,
                                 float base_dt, float* x_seq, float* v_seq, float* x_final,
                                 float* v_final, float* workspace, long long workspace_floats,
                                 gfn_stream_t stream);

/* ------------------------------------------------------------------------
 * Measurement: per-kernel timing of the layered path.  While enabled (enable
 * = 1 also clears earlier records), every layer step of
 * gfn_leapfrog_layered_forward brackets its head-step and mixing-GEMM
 * launches with CUDA events on the launch stream; _read synchronises them
 * and returns the summed milliseconds of each kernel and the number of
 * layer steps recorded.  Not for production calls (events cost launches). */
int gfn_debug_layered_timing(int enable);
/* Measurement: while `device_stamps` is non-NULL, every launch of the
 * tensor-core head-step kernel writes global-timer stamps of its phases to
 * device_stamps[cta * 8 + phase] (cta = head * row_tiles + row_tile), each
 * launch overwriting the last. */
int gfn_debug_head_profile(long long* device_stamps);
int gfn_debug_layered_timing_read(double* head_ms, double* mix_ms, int* layer_steps);

/* ------------------------------------------------------------------------
 * Measurement: cycles of `steps` iterations of the layer-step latency floor
 * (the fused recurrence's dependent chain with no weight traffic: Gamma and
 * friction reductions, the kick arithmetic, the concat and RMSNorm cluster
 * exchanges, the mixing reduction; 8-CTA clusters, one warp per CTA) on
 * `clusters` clusters; CTA 0's clock64 difference is written to the device
 * pointer `cycles`.  Per-head rank 4, 8 or 16. */
int gfn_debug_latency_probe(int rank, int clusters, int steps, long long* cycles,
                            gfn_stream_t stream);

/* The same split-fp16 product, C = A' B'^T (+ bias) for operands split with
 * K along their columns (k_along_rows = 0: a2 [M][3K] role A, b2 [N][3K] role
 * B), on the library's own tcgen05 GEMM kernel (the layered path's mixing
 * kernel, one product per launch) instead of the library GEMM.  Serves the
 * readout's logits (gfn/model.py:393-397) and the scan path's projections
 * (gfn/layers/parallel.py:91-108).  K <= 512 and a multiple of 32, N a
 * multiple of 64, 16-byte aligned operands; bias [N] or NULL; alpha_slot: one
 * float of device scratch for 1/(s_a s_b).  C [M][N] fp32 is overwritten. */
int gfn_gemm_split_f16_tc(int M, int N, int K, const void* a2, const void* b2, const float* scale_a,
                          const float* scale_b, const float* bias, float* c, float* alpha_slot,
                          gfn_stream_t stream);

/* ------------------------------------------------------------------------
 * Readout GEMMs at fp32-level accuracy on the tensor cores (the readout
 * nn.Linear(d -> vocab) of gfn/model.py:393-397 and its backward, which the
 * reference runs as fp32 torch matmuls).  gfn_split_f16 scales an fp32
 * matrix x [rows][cols] by a power of two s (max|x| s in [2^13, 2^14); s is
 * written to scale[1], scale[0] is scratch) and splits it into two fp16
 * pieces along its K dimension: K = cols gives out [rows][3 cols], K = rows
 * (k_along_rows) gives out [3 rows][cols]; segments [x0 x0 x1] for the A
 * operand, [x0 x1 x0] for the B operand (role_b).  gfn_gemm_split_f16 then
 * forms row-major C[M][N] = op(A) op(B) / (s_A s_B) + beta C with one fp16
 * GEMM (K' = 3K, fp32 accumulation); op(A) is [M][K] (A split with K along
 * its columns, or along its rows for a transposed A), op(B) is [K][N].
 * K is laid out and multiplied in 512-wide blocks whose products are summed
 * in fp32 (the tensor cores' accumulation error grows with K).
 * alpha_beta: 3 device floats of scratch. */
int gfn_split_f16(const float* x, long long rows, long long cols, int k_along_rows, int role_b, void* out,
                  float* scale, gfn_stream_t stream);
int gfn_gemm_split_f16(int M, int N, int K, const void* a2, int a_k_rows, const void* b2, int b_k_rows,
                       const float* scale_a, const float* scale_b, float beta, float* c,
                       float* alpha_beta, gfn_stream_t stream);

/* ------------------------------------------------------------------------
 * y_t = a_t y_{t-1} + x_t along t of [batch, seq_len, dim] (a NULL: a == 1).
 * Replaces parallel_scan_fused (gfn/cuda/src/layers/parallel_scan_fused.cu:81,
 * called from gfn/scan.py:20); semantics gfn/scan.py:11-104.
 * dim % 4 == 0, 16-byte aligned pointers.  `workspace` (may be NULL) of
 * gfn_parallel_scan_workspace_floats() floats lets short-batch, long
 * sequences split the time axis; without it one pass is used.
 */
long long gfn_parallel_scan_workspace_floats(int batch, int seq_len, int dim);
int gfn_parallel_scan(const float* a, const float* x, float* y, float* workspace,
                      long long workspace_floats, int batch, int seq_len, int dim,
                      gfn_stream_t stream);

/* The same scan for callers that cannot allocate device memory where they
 * call it -- for example code running inside an allocator or memory-pool
 * callback, plugins whose host framework owns every allocation, or
 * services with a fixed device-memory budget.  It takes no workspace and
 * allocates nothing: the chunk aggregates of the time-split path live in
 * an 8 MiB array compiled into this library, which every GPU that loads
 * the library keeps until the process exits.
 *  - Limit: batch * dim <= 524288; larger sizes return GFN_ERR_INVALID
 *    (use gfn_parallel_scan with a workspace instead).
 *  - The first call on a device looks up that array's device address
 *    (cudaGetSymbolAddress) with the device current; make that first call
 *    before any stream capture on the device.  The lookup is repeated when
 *    the device's context has been re-created (after cudaDeviceReset).
 *  - All calls share the one array and it keeps the last call's contents
 *    (nothing in it is read before the same call writes it).  Calls whose
 *    executions overlap on the GPU, e.g. on two streams at once, race on
 *    it: serialise them.
 * Results match gfn_parallel_scan to float32 rounding (the time axis may
 * be split into fewer chunks).  No counterpart in the reference. */
int gfn_parallel_scan_noalloc(const float* a, const float* x, float* y, int batch, int seq_len,
                              int dim, gfn_stream_t stream);

/* ParallelMLayer recurrence (gfn/layers/parallel.py:101-121) from the
 * pre-activations z = [to_A(f) | to_dt(f) | to_B(f)] of shape
 * [batch, seq_len, 3*dim]: v_seq, x_seq [batch, seq_len, dim]. */
int gfn_parallel_layer_scan(const float* z, float* x_seq, float* v_seq, int batch, int seq_len,
                            int dim, int heads, float base_dt, gfn_stream_t stream);

/* ------------------------------------------------------------------------
 * FunctionalEmbedding, mode 'binary', coord_dim 16, hidden 64, 2 hidden
 * SIREN layers (gfn/embeddings.py:121-206): ids [n] -> forces [n, dim],
 * float32 (out_f32) or bfloat16 (out_bf16, raw uint16 storage).
 * impulse: device pointer to the scalar impulse_scale. */
int gfn_functional_embedding(const long long* ids, long long n, const float* W0, const float* b0,
                             const float* W1, const float* b1, const float* W2, const float* b2,
                             const float* Wo, const float* bo, const float* impulse, float omega0,
                             int dim, float* out_f32, void* out_bf16, gfn_stream_t stream);

/* ------------------------------------------------------------------------
 * Next-token cross-entropy over the readout's logits: the loss of the
 * reference's training loops, nn.CrossEntropyLoss() on logits.view(-1, V)
 * (demos/wikitext/train_wikitext.py:162,185; ignore_index as in
 * demos/copy_task/train_copy_task.py:175), computed on fp32 logits [rows][V]
 * with int64 targets [rows].
 *
 * Forward: row_loss[r] = logsumexp(logits[r]) - logits[r][t_r] (0 where
 * t_r == ignore_index) and row_stats[r] = (m_r, log sum_j exp(logits[r][j] -
 * m_r)), m_r the row maximum: two floats per row, 8-byte aligned, kept apart
 * so large logits lose no precision to their sum.  The mean loss
 * is sum(row_loss) / (number of rows not ignored), summed by the caller.  A
 * target outside [0, V) that is not ignore_index sets GFN_DEVERR_BAD_TOKEN
 * and a NaN row loss.
 * Backward: grad_logits[r][j] = (softmax(logits[r])[j] - [j == t_r])
 * * grad_scale[0] (zero rows where t_r is ignored or out of range);
 * grad_scale is ONE float in device memory (dL/dloss / rows not ignored), so
 * no host sync is needed.  grad_logits may alias logits.  rows < 2^31. */
int gfn_cross_entropy_forward(const float* logits, const long long* targets, long long rows, int V,
                              long long ignore_index, float* row_loss, float* row_stats, gfn_stream_t stream);
int gfn_cross_entropy_backward(const float* logits, const long long* targets, const float* row_stats,
                               long long rows, int V, long long ignore_index, const float* grad_scale,
                               float* grad_logits, gfn_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* GFN_B200_H */
