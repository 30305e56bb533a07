/*
 * tt-splat B200 — C ABI of the matrix-native 3DGS render/train hot path (sm_100a).
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream (as void*, NULL = the
 * legacy default stream), launches asynchronously on that stream, performs no host<->device
 * synchronisation and no allocation (the setup calls tts_peer_alloc / tts_ipc_* excepted), and
 * returns a status code (TTS_OK = 0).  On failure,
 * tts_last_error() describes the problem (thread-local).  Scratch memory is passed in by the
 * caller; each *_workspace_bytes() function gives the size an entry point needs.
 *
 * Data layout (all fp32 unless stated, row-major, views outermost):
 *   params   [59*G + 1]   means3d[G,3] | log_scales[G,3] | quats[G,4] (w,x,y,z) | opacity_raw[G]
 *                         | color_dc[G,3] | color_rest[G,15,3] | w_b_raw
 *            (the GaussianModel parameters of spike/model.py:28-47, flattened)
 *   cams     [V][TTS_CAM_FLOATS]   R_v[9], t_v[3], fx, fy, cx, cy, centre[3], pad
 *   proj     [V][G][TTS_PROJ_FLOATS] mu2d.x, mu2d.y, conic a, b, c, color_o r, g, b, keo, depth, 0, 0
 *   mu2d     [V][G][2], keep [V][G] (uint8)
 *   tiles    T = (H/16)*(W/16), tile t = ty*(W/16) + tx, H and W multiples of 16
 *   idx      [V][T][K] int32 gaussian id per slot in canonical order, -1 when unused
 *   count    [V][T] int32 = min(cand, K);  cand [V][T] int32 = candidates (overflow = cand-K)
 *   inv      [V][G][(2R+1)^2] int32 flat slot t*K+k of gaussian g at stencil offset j, or -1
 *   slots    [V][T][K][TTS_SLOT_FLOATS]  theta_u[6] (tile-local), color_o[3], o_col, dead, 0
 *            (dead = 1 when the binning found the slot's weight zero at every pixel of its tile:
 *            the tile kernels skip it, bit-identically; rows with 0 there are always evaluated) 
 *            or, compact bf16: [V][T][K][TTS_SLOT_BF16] bf16 theta_hi[6], theta_lo[6] (theta_u =
 *            hi + lo), color_o[3], o_col
 *   img      [V][H][W][3], den [V][H][W], gimg like img
 *   slot_grads [V][T][K][TTS_SLOT_GRAD_FLOATS]  gtheta_u[6], gcolor_o[3], go_col
 */
#ifndef TTSPLAT_B200_H
#define TTSPLAT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TTS_OK 0
#define TTS_ERR_INVALID 1   /* bad argument (size, alignment, range) */
#define TTS_ERR_CUDA 2      /* a CUDA launch or runtime call failed */
#define TTS_ERR_CAPACITY 3  /* workspace too small */

#define TTS_CAM_FLOATS 20
#define TTS_PROJ_FLOATS 12
#define TTS_SLOT_FLOATS 12
#define TTS_SLOT_BF16 16
#define TTS_SLOT_GRAD_FLOATS 10
#define TTS_PARAM_FLOATS 59

int tts_version(void);
const char* tts_last_error(void);

/* Device status word written by kernels instead of trapping (bounded waits that gave up):
 * 1 = a bulk-copy wait of the forward, 2 = a relocation grid barrier, 4 = a peer barrier;
 * 8 = a cached binning table that spreads a gaussian over more than its stencil.
 * Synchronous read + clear.  A non-zero word means a step skipped work: the Python train step
 * reads it at check_status / check_replicas and at the end of fit / train_mcmc, and raises. */
int tts_read_status(int* status_host);

/* ---- geometry + SH colour + activations --------------------------------------------------
 * Replaces spike/geometry.py:10-57 (quat_to_rotmat, cov3d, project_ewa), spike/sh.py:49-72
 * (eval_sh_color on means - camera centre, spike/render.py:22-25) and the activations of
 * _operands, tools/m4_train_binned.py:194-202 (o = sigmoid, keo = keep*o, color_o = keo*colour).
 * Also counts kept gaussians per home cell into cell_count[V][T] (zeroed here first) and writes
 * each gaussian's (cell, rank-in-cell) into cell_rank[V][G][2] for the binning scatter.
 * depth_bt (device float[2] = depth_beta, depth_tau, or NULL) selects arm B (spike/arms.py:34-37):
 * the opacity is scaled by sigmoid(depth_beta * (depth_tau - z)) of the camera-space z. */
int tts_project(const float* params, int G, int sh_degree, const float* cams, int V, int H, int W,
                float blur, float near_plane, float* proj, float* mu2d, uint8_t* keep,
                int32_t* cell_count, int32_t* cell_rank, const float* depth_bt, void* stream);

/* ---- spatial-hash binning ----------------------------------------------------------------
 * Replaces assign_bins, tools/m4_train_binned.py:75-127 (canonical = stable order of its key
 * tile*2048 + clamp(long(dist2),0,2047), ties by stencil offset j then gaussian id), plus the
 * inverse table of tools/m9_scatter_oracle.py:20-35 (indexed by stencil offset) and, when
 * proj/slots are given, the operand gather of _operands :207-211 with theta_u_gathered
 * :130-143.  G < 2^31, K <= 256, R <= 3.  inv may be NULL (forward-only rendering).
 * tts_bin_pack writes fp32 slot rows (slot_format 0) or compact bf16 rows (slot_format 1, the
 * forward-only bf16 path of tts_render_fwd) for the count[t] valid slots of each tile only; the
 * tile kernels read no further, and a caller that hands the rows on as [T,K] operands zeroes the
 * rest itself (the reference's operands are zero in invalid slots).  With fp32 slot rows, a slot
 * marked dead in its row (zero weight at every pixel of the tile) has no inverse entry (-1): its
 * gradient is zero, and tts_backward_params skips it. */
size_t tts_bin_workspace_bytes(int G, int V, int H, int W);
int tts_bin_from_mu2d(const float* mu2d, const uint8_t* keep, int G, int V, int H, int W, int R,
                      int K, int32_t* idx, int32_t* count, int32_t* cand, int32_t* inv,
                      void* workspace, size_t workspace_bytes, void* stream);
/* Allocation-free variant of tts_bin_from_mu2d (no counterpart in the reference): for callers
 * that cannot allocate device memory when they bin (inside CUDA-graph stream capture, or embedded
 * in a host runtime that owns the allocator).  Scratch comes from a 16 MiB static device array per
 * GPU, held until exit; problems whose tts_bin_workspace_bytes exceeds 16 MiB are rejected with
 * TTS_ERR_CAPACITY.  The first call on a device looks up that array's address (set-up), so make
 * it before any stream capture.  All calls share the array: calls that overlap on the GPU race.
 * The looked-up address is kept for the life of the process and belongs to the device's
 * context at the time of that first call: after cudaDeviceReset (a new primary context) it is
 * stale, so do not call this entry point on a device that has been reset. */
int tts_bin_from_mu2d_noalloc(const float* mu2d, const uint8_t* keep, int G, int V, int H, int W,
                              int R, int K, int32_t* idx, int32_t* count, int32_t* cand,
                              int32_t* inv, void* stream);
int tts_bin_pack(const float* mu2d, const uint8_t* keep, const float* proj,
                 const int32_t* cell_count, const int32_t* cell_rank, int G, int V, int H, int W,
                 int R, int K, float k_poly, int32_t* idx, int32_t* count, int32_t* cand,
                 int32_t* inv, void* slots, int slot_format, void* workspace,
                 size_t workspace_bytes, void* stream);

/* Operands from cached tables (replaces the cached_bins branch of _operands,
 * tools/m4_train_binned.py:203-207): idx_in[V][T][K] holds gaussian ids from an earlier binning,
 * -1 for invalid slots, the valid slots first in each tile.  Writes idx (may alias idx_in),
 * count[V][T], the fp32 slot rows of the current projection and, when inv is not NULL, an inverse
 * table: each gaussian's slot in the tile at (dx, dy) of the (2R+1)^2 box that starts at the
 * smallest tile column and row it occupies.  Tables that spread a gaussian wider than that box
 * OR 8 into the status word.  Workspace: tts_pack_cached_workspace_bytes. */
size_t tts_pack_cached_workspace_bytes(int G, int V);
int tts_pack_cached(const float* proj, int G, int V, int H, int W, int R, int K, float k_poly,
                    const int32_t* idx_in, int32_t* idx, int32_t* count, int32_t* inv, float* slots,
                    void* workspace, size_t workspace_bytes, void* stream);

/* ---- operands in the reference layout -> slot rows ---------------------------------------
 * Packs theta_u[V*T,6,K], color_o[V*T,K,3], o_col[V*T,K,1] (the operands of
 * _DevRenderBinned.apply, tools/m4_train_binned.py:154-166) into slot rows, and the
 * per-slot grads back into the reference layout. */
int tts_pack_operands(const float* theta_u, const float* color_o, const float* o_col, int VT, int K,
                      float* slots, void* stream);
int tts_unpack_slot_grads(const float* slot_grads, int VT, int K, float* gtheta_u, float* gcolor_o,
                          float* go_col, void* stream);

/* ---- fused per-tile forward ----------------------------------------------------------------
 * Replaces _DevRenderBinned.forward, tools/m4_train_binned.py:156-166 (= render_binned_cpu
 * :226-230, WSRPolySplatHot.forward spike/backward.py:28-41): Q = Phi.theta_u per tile,
 * w = relu(Q)^2, C = (sum w color_o + w_b c_b) / (sum w o_col + w_b); img[gidx] = C.
 * slots_bf16 != 0 reads compact bf16 slot rows (tts_bin_pack slot_format 1; bf16 in, fp32
 * accumulate).
 * The background weight is read on the device: w_b = softplus(*w_b) when w_b_is_raw != 0
 * (the model's w_b_raw), else *w_b as given (the activated operand of _DevRenderBinned). */
int tts_render_fwd(const void* slots, int slots_bf16, const int32_t* count, int V, int H, int W,
                   int K, const float* w_b, int w_b_is_raw, const float* c_b, float* img,
                   float* den, void* stream);

/* ---- fused per-tile backward -------------------------------------------------------------
 * Replaces _DevRenderBinned.backward, tools/m4_train_binned.py:169-186 (= WSRPolySplatHot
 * .backward, spike/backward.py:43-58): per slot gtheta_u = Phi^T (2 relu(Q) gw),
 * gcolor_o = w^T gnum, go_col = w^T gden; per tile partial gw_b = sum(gnum c_b + gden). */
int tts_render_bwd(const float* slots, const int32_t* count, int V, int H, int W, int K,
                   const float* c_b, const float* img, const float* den, const float* gimg,
                   float* slot_grads, float* gwb_partial, void* stream);

/* Arm RV (revealage compositing; replaces blend_RV, spike/arms.py:70-83, on the binned path):
 * W = w_geo * o_col per (pixel, slot), den = sum W + 1e-6, Cavg = sum w_geo color_o / den,
 * R = exp(sum log1p(-clamp(W, 0, 1 - 1e-4))), C = Cavg (1 - R) + c_b R.  fp32 slot rows only;
 * writes img, den and aux[V,H,W,4] = (Cavg, R), 16-byte aligned.  The backward takes the same
 * den/aux and writes slot grads in the arm-A layout and zero w_b partials (w_b is unused). */
int tts_render_fwd_rv(const float* slots, const int32_t* count, int V, int H, int W, int K,
                      const float* c_b, float* img, float* den, float* aux, void* stream);
int tts_render_bwd_rv(const float* slots, const int32_t* count, int V, int H, int W, int K,
                      const float* c_b, const float* den, const float* aux, const float* gimg,
                      float* slot_grads, float* gwb_partial, void* stream);

/* ---- photometric loss ------------------------------------------------------------------
 * Replaces metrics.loss_fn, spike/metrics.py:26-28 ((1-l) L1 + l (1-SSIM), SSIM on inputs
 * clamped to [0,1], 11-tap sigma-1.5 window shrunk for small images :15-19) with the manual
 * gradient of tools/loss_manual.py:78-105.  gimg = grad_scale * dloss/dimg; loss[v] written,
 * and, when loss_sum is not NULL, loss_sum[0] = loss[0] + ... + loss[V-1] (view order).
 * lambda = 0 is the L1 loss alone: one pass over the pixels, no SSIM work. */
size_t tts_loss_workspace_bytes(int V, int H, int W);
int tts_loss_l1_ssim(const float* img, const float* target, int V, int H, int W, float lambda,
                     float grad_scale, float* gimg, float* loss, float* loss_sum, void* workspace,
                     size_t workspace_bytes, void* stream);

/* ---- slot -> gaussian reduction + geometry/SH/activation backward ------------------------
 * Replaces the index_add of tools/operands_manual.py:94-98 (= build_inv/gather_reduce,
 * tools/m9_scatter_oracle.py), _theta_bwd :65-80, geom_bwd.bwd tools/geom_bwd.py:67-152, the
 * activation grads of operands_manual.bwd_manual :103-110 and the SH colour backward; sums
 * over the V views in view order; adds the reg_loss gradient (spike/mcmc.py:18-22) and the
 * w_b_raw gradient from the per-tile partials.  grads has the params layout (overwritten).
 * proj is the tts_project output for the same params and cameras (its 2-D means and conics
 * feed the theta-build backward).  Arm B: depth_bt as given to tts_project, and g_depth_bt
 * (device float[2]) receives d/d depth_beta and d/d depth_tau; both NULL for arm A.  The per-(view, gaussian) gathered records go through the
 * workspace (tts_backward_workspace_bytes). */
size_t tts_backward_workspace_bytes(int G, int V);
int tts_backward_params(const float* params, int G, int sh_degree, const float* cams, int V,
                        int H, int W, int R, int K, float k_poly, float blur, float near_plane,
                        const float* proj, const int32_t* inv, const float* slot_grads,
                        const float* gwb_partial,
                        float lambda_o, float lambda_s, float* grads, const float* depth_bt,
                        float* g_depth_bt, void* workspace, size_t workspace_bytes, void* stream);

/* ---- Adam + SGLD ----------------------------------------------------------------------
 * torch.optim.Adam step (spike/train.py:19,29; groups spike/model.py:82-95) over the flat
 * params, then add_sgld_noise (spike/mcmc.py:25-34) when noise_lr > 0.  lr[7] = means,
 * log_scales, quats, opacity_raw, color_dc, color_rest, w_b_raw.  The step number is read from
 * *step (device int, already incremented for this step).  eps_noise [G,3] injects the
 * Gaussian draw; when NULL a Philox4x32-10 stream keyed by (seed, step) is used. */
int tts_adam_sgld(float* params, const float* grads, float* m, float* v, int G, int sh_degree,
                  const int32_t* step, const double* lr7, double beta1, double beta2, double eps,
                  float noise_lr, const float* eps_noise, uint64_t seed, void* stream);
int tts_step_begin(int32_t* step, void* stream);
/* torch.optim.Adam on a vector of n <= 1024 floats with one learning rate: the depth group
 * (depth_beta, depth_tau) of GaussianModel.param_groups, spike/model.py:93, trained under arm B. */
int tts_adam_vec(float* p, const float* g, float* m, float* v, int n, const int32_t* step, double lr,
                 double beta1, double beta2, double eps, void* stream);
/* add_sgld_noise alone (spike/mcmc.py:25-34) with lr = lr_means; same noise stream/injection. */
int tts_sgld(float* params, int G, double lr_means, float noise_lr, const float* eps_noise,
             const int32_t* step, uint64_t seed, void* stream);

/* ---- MCMC relocation ---------------------------------------------------------------------
 * relocate + reset_adam_state (spike/mcmc.py:41-87): dead = o < thr, targets drawn with
 * replacement proportional to o over the alive set, target opacity split o/(n+1), dead slots
 * take the target's parameters (+ offset * N(0,1) on means), moments of every touched
 * gaussian zeroed.  thr = dead_thr when dead_frac <= 0, else the torch.quantile of o at
 * dead_frac.  targets_in [n_dead] / offset_noise_in [n_dead,3] inject the draws (NULL: Philox
 * keyed by (seed, step)).  n_dead_out receives the number moved (device int). */
size_t tts_relocate_workspace_bytes(int G);
int tts_relocate(float* params, float* m, float* v, int G, float dead_thr, float dead_frac,
                 float offset, const int32_t* targets_in, const float* offset_noise_in,
                 const int32_t* step, uint64_t seed, int32_t* n_dead_out, int32_t* targets_out,
                 void* workspace, size_t workspace_bytes, void* stream);
/* The SGLD step of tts_sgld (spike/mcmc.py:25-34, the lr of the means at lr7[0]; eps_noise
 * [G,3] injects its noise, NULL: Philox) followed by tts_relocate, in one launch: the MCMC
 * order of an iteration that relocates (spike/mcmc.py:97-111), the same results as the two
 * calls in turn. */
int tts_sgld_relocate(float* params, float* m, float* v, int G, const double* lr7, float noise_lr,
                      const float* eps_noise, float dead_thr, float dead_frac, float offset,
                      const int32_t* targets_in, const float* offset_noise_in, const int32_t* step,
                      uint64_t seed, int32_t* n_dead_out, int32_t* targets_out, void* workspace,
                      size_t workspace_bytes, void* stream);
/* The same for one rank of the multi-GPU step: tts_peer_sgld (waits, with an iteration limit,
 * for every rank's phase-1 flag) followed by tts_relocate, in one launch; flags/rank/N as in
 * tts_peer_sgld. */
int tts_peer_sgld_relocate(float* params, float* m, float* v, int G, const double* lr7,
                           float noise_lr, const float* eps_noise, float dead_thr, float dead_frac,
                           float offset, const int32_t* step, uint64_t seed, int32_t* n_dead_out,
                           int32_t* targets_out, int32_t* const* flags, int rank, int N,
                           void* workspace, size_t workspace_bytes, void* stream);

/* ---- multi-GPU optimizer step over NVLink peer memory -------------------------------------
 * Replaces the gradient all-reduce + replicated torch.optim.Adam of a view-split batch
 * (spike/train.py:27-29 with the views spread over N ranks).  Buffers shared between the
 * ranks of one node are allocated here (tts_peer_alloc: cudaMalloc, zero-filled) and
 * exchanged with CUDA IPC handles (tts_ipc_handle_bytes bytes each; the host moves them).
 * Per step: tts_peer_signal(phase 0) once this rank's gradient and loss are written;
 * tts_adam_peer: waits until every rank signalled phase 0, sums the N gradients of this rank's
 * 1/N shard in rank order, updates the shard (and, on rank N-1, w_b_raw) with its moments m, v,
 * stores the new values into all N parameter buffers, and its last block to finish signals
 * phase 1; loss_total = sum of the N losses; then tts_peer_sgld (SGLD after waiting for phase
 * 1 of every rank) or tts_peer_wait(phase 1) before the parameters are read again.
 * tts_peer_barrier = signal + wait in one kernel.  params/grads/loss/flags are host arrays of N
 * device pointers (index = rank; this rank's own buffers included); flags point at 32 int32 per
 * rank, zero at start; epoch is a device int that grows every step (the step counter).  A wait
 * that runs too long ORs 4 into the status word (tts_read_status) and gives up; the Adam and
 * SGLD blocks whose wait gave up skip their part of the update (no partial gradient sums).
 * N <= 8. */
size_t tts_ipc_handle_bytes(void);
int tts_peer_alloc(size_t bytes, void** ptr);
int tts_peer_free(void* ptr);
int tts_ipc_export(void* ptr, void* handle_out);
int tts_ipc_open(const void* handle, void** ptr_out);
int tts_ipc_close(void* ptr);
int tts_peer_barrier(int32_t* const* flags, int rank, int N, int phase, const int32_t* epoch,
                     void* stream);
int tts_peer_signal(int32_t* const* flags, int rank, int N, int phase, const int32_t* epoch,
                    void* stream);
int tts_peer_wait(int32_t* const* flags, int rank, int N, int phase, const int32_t* epoch,
                  void* stream);
int tts_adam_peer(float* const* params, const float* const* grads, float* m, float* v, int G,
                  int sh_degree, int rank, int N, const int32_t* step, const double* lr7,
                  double beta1, double beta2, double eps, const float* const* loss,
                  float* loss_total, int32_t* const* flags, void* stream);
int tts_peer_sgld(float* params, int G, double lr_means, float noise_lr, const float* eps_noise,
                  const int32_t* step, uint64_t seed, int32_t* const* flags, int rank, int N,
                  void* stream);

/* ---- the composable spike API: building blocks, forward and backward -------------------------
 * The reference's differentiable functions of spike/geometry.py, spike/sh.py and
 * spike/forward.py as standalone kernels, for callers that compose them by hand (the hot path
 * fuses them into tts_project / tts_backward_params).  dtype 0 = float32, 1 = float64 for every
 * floating pointer of a call; n counts the leading (batch) elements.  Each *_bwd returns the
 * gradients of the differentiable inputs for the given output gradients (NULL = zero where
 * allowed).  Camera poses, intrinsics and pixel grids are constants (never differentiated).
 * Reductions over pixels write per-chunk partials into a caller workspace of
 * tts_spike_workspace_bytes(P, G, dtype) bytes and sum them in a fixed order. */
size_t tts_spike_workspace_bytes(long long P, long long G, int dtype);
/* quat_to_rotmat, spike/geometry.py:10-19: q[n,4] (w,x,y,z; normalised with the norm clamped at
 * 1e-12) -> R[n,3,3]. */
int tts_quat_to_rotmat(const void* q, long long n, void* R, int dtype, void* stream);
int tts_quat_to_rotmat_bwd(const void* q, const void* gR, long long n, void* gq, int dtype, void* stream);
/* cov3d, spike/geometry.py:22-25: scales[n,3] (already exponentiated), R[n,3,3] ->
 * R diag(s^2) R^T [n,3,3]. */
int tts_cov3d(const void* scales, const void* R, long long n, void* cov, int dtype, void* stream);
int tts_cov3d_bwd(const void* scales, const void* R, const void* gcov, long long n, void* gscales,
                  void* gR, int dtype, void* stream);
/* project_ewa, spike/geometry.py:28-57: means[G,3], cov[G,3,3] (any 3x3), cam16 = host
 * double[16] {R_v row-major, t_v, fx, fy, cx, cy} -> mu2d[G,2], conic[G,3] (a, b, c of the
 * inverse of J R_v cov R_v^T J^T + blur I, det clamped at 1e-12 as the reference does),
 * depth[G] (camera z), keep[G] (uint8, z > near).  Backward: grads of means and cov. */
int tts_project_ewa(const void* means, const void* cov, long long G, const double* cam16, double blur,
                    double near_plane, void* mu2d, void* conic, void* depth, uint8_t* keep, int dtype,
                    void* stream);
int tts_project_ewa_bwd(const void* means, const void* cov, long long G, const double* cam16,
                        double blur, double near_plane, const void* gmu2d, const void* gconic,
                        const void* gdepth, void* gmeans, void* gcov, int dtype, void* stream);
/* eval_sh_color, spike/sh.py:49-72: coeffs[G,nc,nch] (nc >= (deg+1)^2), dirs[G,3] (normalised
 * with the norm clamped at 1e-12) -> out[G,nch] = clamp(0.5 + sum_k basis_k coeffs_k, min 0), or
 * the bare sum when raw != 0.  Backward: grads of coeffs (zero beyond (deg+1)^2) and dirs. */
int tts_eval_sh(int deg, const void* coeffs, int nc, int nch, const void* dirs, long long G, int raw,
                void* out, int dtype, void* stream);
int tts_eval_sh_bwd(int deg, const void* coeffs, int nc, int nch, const void* dirs, long long G,
                    int raw, const void* gout, void* gcoeffs, void* gdirs, int dtype, void* stream);
/* color_from_dc, spike/forward.py:69-71: clamp(0.5 + C0 dc, min 0); with gout != NULL writes
 * the gradient d/d dc instead. */
int tts_color_from_dc(const void* dc, long long n, const void* gout, void* out, int dtype, void* stream);
/* phi, spike/forward.py:42-44: px[P], py[P] -> Phi[P,6] = [px^2, py^2, px py, px, py, 1]. */
int tts_phi(const void* px, const void* py, long long P, void* Phi, int dtype, void* stream);
int tts_phi_bwd(const void* px, const void* py, const void* gPhi, long long P, void* gpx, void* gpy,
                int dtype, void* stream);
/* theta_from_conic, spike/forward.py:23-39: conic[n,3], mu[n,2] (minus origins[i/per][2] when
 * origins != NULL) -> theta_Q[n,6] and/or theta_u[n,6] = -theta_Q/k + e5 (layout 0), or theta_u
 * as [n/per,6,per] in the op order of theta_u_gathered, tools/m4_train_binned.py:130-143
 * (layout 1).  Backward (layout-0 gradients): grads of conic and mu. */
int tts_theta_from_conic(const void* conic, const void* mu, const void* origins, long long per,
                         long long n, double k, int layout, void* theta_Q, void* theta_u, int dtype,
                         void* stream);
int tts_theta_from_conic_bwd(const void* conic, const void* mu, const void* origins, long long per,
                             long long n, double k, const void* gtheta_Q, const void* gtheta_u,
                             void* gconic, void* gmu, int dtype, void* stream);
/* quad_form, spike/forward.py:13-20: Q[P,G] = a dx^2 + 2 b dx dy + c dy^2, (dx, dy) = pixel -
 * mean.  Backward: grads of mu2d and conic (pixel sums through the workspace). */
int tts_quad_form(const void* px, const void* py, const void* mu2d, const void* conic, long long P,
                  long long G, void* Q, int dtype, void* stream);
int tts_quad_form_bwd(const void* px, const void* py, const void* mu2d, const void* conic,
                      const void* gQ, long long P, long long G, void* gmu2d, void* gconic,
                      void* workspace, size_t workspace_bytes, int dtype, void* stream);
/* Q = Phi theta^T ([P,6] x [G,6]^T), the GEMM of quad_form_tilelocal, spike/forward.py:47-58.
 * Backward: gPhi and/or gtheta (either may be NULL; gtheta uses the workspace). */
int tts_phi_theta(const void* Phi, const void* theta, long long P, long long G, void* Q, int dtype,
                  void* stream);
int tts_phi_theta_bwd(const void* Phi, const void* theta, const void* gQ, long long P, long long G,
                      void* gPhi, void* gtheta, void* workspace, size_t workspace_bytes, int dtype,
                      void* stream);
/* poly_splat_wgeo, spike/forward.py:61-66: w[P,G] = max(0, 1 - Q/k)^2 * keep[g] (keep uint8 or
 * NULL); with gout != NULL writes dL/dQ instead. */
int tts_poly_splat_wgeo(const void* Q, long long P, long long G, double k, const uint8_t* keep,
                        const void* gout, void* out, int dtype, void* stream);

/* ---- dense WSR (spike/backward.py:61-63, wsr_polysplat) -----------------------------------
 * C[P,3] from theta_u[G,6], o[G], color[G,3], w_b (device scalar), Phi[P,6], c_b[3], keep[G]
 * (fp32 0/1, may be NULL), and its backward. */
int tts_wsr_dense_fwd(const float* theta_u, const float* o, const float* color, const float* w_b,
                      const float* Phi, const float* c_b, const float* keep, int P, int G,
                      float* C, float* den, void* stream);
int tts_wsr_dense_bwd(const float* theta_u, const float* o, const float* color, const float* w_b,
                      const float* Phi, const float* c_b, const float* keep, int P, int G,
                      const float* C, const float* den, const float* gC, float* gtheta, float* go,
                      float* gcolor, float* gw_b_partial, void* stream);

/* ---- 8-bit target images ------------------------------------------------------------------
 * dst[i] = src[i] / 255 (correctly rounded, = numpy's float32(x) / float32(255)): the [0, 1]
 * floats of 8-bit images as spike/data.py produces them, expanded on the device so that a train
 * step uploads and holds its targets as uint8.  src and dst 16-byte aligned. */
int tts_unit_from_u8(const uint8_t* src, long long n, float* dst, void* stream);

/* ---- measurement ----------------------------------------------------------------------------
 * FP32 FMA-pipe throughput probe (no counterpart in the reference): `blocks` blocks of 256
 * threads run 8 independent packed fma.rn.f32x2 chains for `iters` rounds and write one float
 * per thread to out[blocks*256]; tts_fma_probe_flops gives the flops of such a launch.  Timed
 * by the caller, it is the measured FP32 peak the FP32-bound tile kernels are reported against. */
long long tts_fma_probe_flops(int blocks, int iters);
int tts_fma_probe(int blocks, int iters, float* out, void* stream);

#ifdef __cplusplus
}
#endif
#endif
