/*
 * dsmezo.h - C ABI of the B200-native DS-MeZO optimizer hot path (libdsmezo.so).
 *
 * Plain pointers, sizes and a cudaStream_t (passed as void*); no torch types. Every
 * entry point returns DSMZ_OK (0) or an error code, and dsmz_last_error() returns the
 * message of the last failure on the calling thread. Device memory is never allocated
 * inside: callers pass device workspaces sized by the *_workspace_bytes queries.
 * Launches go to the given stream; nothing synchronises the host.
 *
 * Two layers:
 *  1. Per-op drop-ins for the four functions of the reference module ds_mezo/kernels.py
 *     (same arguments and results as the Python functions cited on each entry point).
 *  2. The grouped optimizer step: one plan per adapter set (all modules of all layers),
 *     then one launch sequence per phase for every matrix at once, replacing the
 *     per-module Python loops of ds_mezo/controller.py:165-176, 236-292.
 */
#ifndef DSMEZO_H_
#define DSMEZO_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DSMZ_ABI_VERSION 3

typedef void* dsmz_stream_t; /* cudaStream_t */

enum dsmz_dtype { DSMZ_F32 = 0, DSMZ_BF16 = 1 };

enum dsmz_status {
  DSMZ_OK = 0,
  DSMZ_ERR_INVALID = 1,     /* bad argument (shape, stride, alignment, null pointer) */
  DSMZ_ERR_WORKSPACE = 2,   /* workspace too small */
  DSMZ_ERR_CUDA = 3,        /* a CUDA launch or copy failed */
  DSMZ_ERR_UNSUPPORTED = 4  /* size beyond what the kernels support */
};

#define DSMZ_MAX_RANK 128      /* adapter rank r and basis width R supported by the kernels */
#define DSMZ_MAX_NS_ITERS 16

/* Last error message of the calling thread ("" when none). */
const char* dsmz_last_error(void);
int dsmz_abi_version(void);

/* ---------------------------------------------------------------------------------
 * Newton-Schulz schedules: iteration k uses S_k = c[k][0] I + c[k][1] G + c[k][2] G^2.
 * ------------------------------------------------------------------------------- */
typedef struct dsmz_ns_schedule {
  int32_t iters;
  double c[DSMZ_MAX_NS_ITERS][3];
} dsmz_ns_schedule;

/* The 12-step degree-3 minimax schedule computed at import in ds_mezo/kernels.py:5-24. */
int dsmz_ns_schedule_cubic(dsmz_ns_schedule* out);
/* Five quintic steps (3.4445, -4.7750, 2.0315); no counterpart in ds_mezo/kernels.py. */
int dsmz_ns_schedule_quintic(dsmz_ns_schedule* out);

/* ---------------------------------------------------------------------------------
 * Per-op drop-ins (ds_mezo/kernels.py).
 * Strides are in elements. The factor tensor (param/base/pos/neg) is F32 or BF16,
 * everything else is F32.
 * ------------------------------------------------------------------------------- */

/* Replaces zo_muon_update (ds_mezo/kernels.py:167-186): scratch <- NS(buf) (the final
 * orthogonalised matrix X), param <- param - eta * X. M >= N takes the tall form
 * (G = X^T X), otherwise the wide form (G = X X^T). min(M, N) <= DSMZ_MAX_RANK.
 * scratch may be NULL (then X is not stored). schedule NULL = cubic. */
size_t dsmz_zo_muon_update_workspace_bytes(int64_t M, int64_t N);
int dsmz_zo_muon_update(int32_t param_dtype, void* param, int64_t param_s0, int64_t param_s1,
                        const float* buf, int64_t buf_s0, int64_t buf_s1,
                        float* scratch, int64_t scratch_s0, int64_t scratch_s1,
                        int64_t M, int64_t N, float eta, float norm_floor,
                        const dsmz_ns_schedule* schedule,
                        void* workspace, size_t workspace_bytes, dsmz_stream_t stream);

/* No counterpart in the reference. The same update as dsmz_zo_muon_update for callers that
 * cannot allocate device memory when they update an adapter: a process whose rollout engine
 * has reserved nearly all of HBM up front (the vLLM engine DS-MeZO drives is created with
 * gpu_memory_utilization=0.95), or a plain C host without a device allocator of its own.
 * Its scratch is a fixed DSMZ_NOALLOC_SCRATCH_BYTES array inside the library (every GPU
 * that loads the library keeps it until exit); no cudaMalloc/cudaFree or allocating
 * library call happens. Sizes whose workspace (dsmz_zo_muon_update_workspace_bytes) exceeds
 * the array return DSMZ_ERR_UNSUPPORTED. The first call on a device looks up the array's
 * device address, so make that first call before any stream capture. All calls share the
 * array: calls that overlap on the GPU (other streams, other host threads) race. */
#define DSMZ_NOALLOC_SCRATCH_BYTES (2u * 1024u * 1024u)
int dsmz_zo_muon_update_noalloc(int32_t param_dtype, void* param, int64_t param_s0, int64_t param_s1,
                                const float* buf, int64_t buf_s0, int64_t buf_s1,
                                float* scratch, int64_t scratch_s0, int64_t scratch_s1,
                                int64_t M, int64_t N, float eta, float norm_floor,
                                const dsmz_ns_schedule* schedule, dsmz_stream_t stream);

/* Replaces fused_power_iter (ds_mezo/kernels.py:249-265): out <- num_iters x
 * {W = H^T (H V); QR(W)}, the Q factor with positive diagonal R (what the reference's
 * modified Gram-Schmidt at ds_mezo/kernels.py:227-240 yields). H is T x D (F32 or BF16,
 * any strides), V is D x R (F32, any strides), out is D x R contiguous F32. */
size_t dsmz_power_iter_workspace_bytes(int64_t T, int64_t D, int64_t R);

/* Contrastive scoring loss (ds_mezo/controller.py:14-15, 194-201): out[0] (device fp64) =
 * sum_i advantages[i] * mean over the scored tokens t of sequence i of nll_t, where
 * nll_t = -log softmax(logits row t)[targets[t]] (the logprob vLLM reports for the token,
 * ds_mezo/backend.py:98-103; kind DSMZ_SCORE_LOGITS_F32 / _BF16, rows of V logits, row
 * pitch ld) or nll_t = -src[t] (kind DSMZ_SCORE_LOGPROBS_F32: one logprob per token).
 * Sequence i owns token rows [seq_start[i], seq_start[i+1]); seq_start (nseq + 1 entries,
 * 0 .. ntok) and advantages (nseq) are host arrays, nseq <= 128, every sequence non-empty.
 * Deterministic (fixed summation order). A target outside [0, V) makes out[0] NaN.
 * dd = (loss(pos) - loss(neg)) / (2 eps) as ds_mezo/controller.py:307. */
#define DSMZ_SCORE_LOGITS_F32 0
#define DSMZ_SCORE_LOGITS_BF16 1
#define DSMZ_SCORE_LOGPROBS_F32 2
size_t dsmz_contrastive_loss_workspace_bytes(int64_t ntok);
int dsmz_contrastive_loss(int32_t kind, const void* src, int64_t V, int64_t ld, const int32_t* targets, int64_t ntok,
                          const int64_t* seq_start, const double* advantages, int32_t nseq, double* out,
                          void* workspace, size_t workspace_bytes, dsmz_stream_t stream);

/* Device-resident activation handoff. Replaces the round trip of each captured module
 * input through pinned host memory (ds_mezo/backend.py:68-93: hook, .float(), pinned copy)
 * and back (ds_mezo/controller.py:171: .cuda()). Converts rows 0..n-1 of a strided source
 * (F32 or BF16, element (t, c) at src[t*src_s0 + c*src_s1]) into the T x D activation
 * buffer dst (row pitch ld_dst elements, F32 or BF16), rows n..T-1 zero; fp32 -> bf16
 * rounds to nearest even, bit for bit as torch's .to(torch.bfloat16) on the GPU. Asynchronous
 * on `stream`. */
int dsmz_activation_load(int32_t dst_dtype, void* dst, int64_t T, int64_t D, int64_t ld_dst, int32_t src_dtype,
                         const void* src, int64_t n, int64_t src_s0, int64_t src_s1, dsmz_stream_t stream);
int dsmz_power_iter(int32_t h_dtype, const void* H, int64_t T, int64_t D, int64_t h_s0, int64_t h_s1,
                    const float* V, int64_t R, int64_t v_s0, int64_t v_s1,
                    float* out, int32_t num_iters, float norm_floor,
                    void* workspace, size_t workspace_bytes, dsmz_stream_t stream);

/* Replaces fused_agzo_perturbation (ds_mezo/kernels.py:371-397):
 * z_B = eps * Zc_B V^T (R x d_in), Q = QR(B V)[:, :min(R,RC)],
 * z_A = eps * Zc_A Q^T (d_out x R). B: R x d_in (any strides), V: d_in x RC (any strides),
 * z_coeff_B: R x RC contiguous, z_coeff_A: d_out x min(R,RC) contiguous,
 * z_A, z_B contiguous outputs. */
size_t dsmz_agzo_perturbation_workspace_bytes(int64_t R, int64_t d_in, int64_t RC, int64_t d_out);
int dsmz_agzo_perturbation(const float* B, int64_t R, int64_t d_in, int64_t b_s0, int64_t b_s1,
                           const float* V, int64_t RC, int64_t v_s0, int64_t v_s1,
                           const float* z_coeff_B, const float* z_coeff_A, int64_t d_out,
                           float* z_A, float* z_B, float eps, float norm_floor,
                           void* workspace, size_t workspace_bytes, dsmz_stream_t stream);

/* Replaces fused_perturb_dual (ds_mezo/kernels.py:415-422): pos = base + z,
 * neg = base - z over n contiguous elements (base/pos/neg in `dtype`, z F32). */
int dsmz_perturb_dual(int32_t dtype, const void* base, const float* z, void* pos, void* neg,
                      int64_t n, dsmz_stream_t stream);

/* ---------------------------------------------------------------------------------
 * torch CUDA generator layout (ATen DistributionTemplates.h calc_execution_policy):
 * a draw of n normals uses threads = 256 * min(ceil(n/256), sm_count*max_threads_per_sm/256)
 * and advances the generator offset by ((n-1)/(4*threads)+1)*4.
 * ------------------------------------------------------------------------------- */
int64_t dsmz_randn_threads(int64_t n, int32_t sm_count, int32_t max_threads_per_sm);
uint64_t dsmz_randn_offset_increment(int64_t n, int32_t sm_count, int32_t max_threads_per_sm);

/* Writes n normals exactly as torch.randn(n, generator=g) on a CUDA device with the given
 * layout would, for a generator at (seed, offset). Used to check the stream bit for bit. */
int dsmz_randn(float* out, int64_t n, uint64_t seed, uint64_t offset, int32_t sm_count,
               int32_t max_threads_per_sm, dsmz_stream_t stream);

/* ---------------------------------------------------------------------------------
 * Grouped optimizer step over an adapter set.
 * A module owns A (d_out x r) and B (r x d_in) as F32 masters, as the reference keeps
 * them (upcast at load, ds_mezo/controller.py:66-67), each with Kalman mean/variance
 * (F32, ds_mezo/controller.py:90-100), the F32 perturbation z (the reference's z_A, z_B)
 * and an optional NS output buffer. What the rollout engine loads is in the plan's copy
 * dtype: the +/- copies (pos = copy(A + z), neg = copy(A - z), the sum taken in F32 and
 * then rounded, as the reference's fp32 pos/neg are cast at export, ds_mezo/backend.py:
 * 21-36) and an optional shadow of the updated masters (shadow = copy(A) after each
 * update; NULL when not wanted). All tensors of one side share its row stride and have
 * unit column stride. Modules must be given in the controller's order (sorted by
 * (layer, module name), ds_mezo/model_config.py:37): it fixes the random draws.
 * ------------------------------------------------------------------------------- */
typedef struct dsmz_module_spec {
  float* A;  float* B;                  /* F32 masters, updated in place */
  void* pos_A; void* pos_B; void* neg_A; void* neg_B;   /* copy dtype */
  void* shadow_A; void* shadow_B;       /* copy dtype, may be NULL */
  float* mu_A; float* mu_B; float* var_A; float* var_B;
  float* z_A; float* z_B;
  float* scratch_A; float* scratch_B;   /* may be NULL */
  int64_t d_out, d_in, r;
  int64_t ld_A, ld_B;
  int32_t basis;                        /* index of the module's activation basis */
  int32_t layer;
} dsmz_module_spec;

typedef struct dsmz_basis_spec {
  const void* H; int32_t h_dtype;       /* activation T x D (row stride ld_H, unit column stride) */
  int64_t T, D, ld_H;
  float* V; int64_t R;                  /* basis D x R contiguous F32, updated in place */
} dsmz_basis_spec;

typedef struct dsmz_plan_desc {
  int32_t copy_dtype;                   /* DSMZ_F32 or DSMZ_BF16: the +/- copies and shadows */
  int32_t num_modules;
  const dsmz_module_spec* modules;
  int32_t num_bases;
  const dsmz_basis_spec* bases;
  int32_t sm_count;                     /* device layout of the torch generator */
  int32_t max_threads_per_sm;
  uint64_t rng_offset_before;           /* generator advance of the draws that precede
                                           these modules (other ranks' modules); 0 on 1 GPU */
  uint32_t flags;                       /* DSMZ_PLAN_* bits */
  /* Many-direction SPSA (no reference counterpart: the reference perturbs one direction
   * per step). directions K in [1, DSMZ_MAX_DIRECTIONS] (0 = 1). Direction k writes its
   * +/- copies at the module's pos/neg pointers + k * dir_stride_factor elements and its z
   * at z + k * dir_stride_z (fp32 elements), and draws from the generator at
   * offset + k * rng_direction_stride (0 = this plan's own one-direction advance, i.e. the
   * whole model is in this plan), so direction k takes exactly the draws that K successive
   * one-direction steps would take. */
  int32_t directions;
  int32_t pad0;
  int64_t dir_stride_factor;
  int64_t dir_stride_z;
  uint64_t rng_direction_stride;
  /* Host array of num_modules generator offsets (relative to the step's base offset) at
   * which each module's two draws start, for a plan whose modules are not one contiguous
   * run of the whole model's controller order (a rank holding parts of layers); the offset
   * of module i is the sum of the draw advances of every module before it in that order.
   * NULL: the draws follow rng_offset_before, module after module. */
  const uint64_t* module_rng_offsets;
} dsmz_plan_desc;

#define DSMZ_MAX_DIRECTIONS 32

/* Power iteration on CUDA cores (fp32 FFMA) even where the tcgen05 path applies. The
 * tcgen05 path needs bf16 activations, D a multiple of 8 and R a multiple of 16. */
#define DSMZ_PLAN_SIMT_POWER_ITER 1u
/* Tensor-core power iteration in a single pass over the activations per iteration (R <= 64):
 * one persistent launch whose Y pipeline streams each activation from HBM and whose W
 * pipeline re-reads each 256-token tile from L2 once its Y rows are complete. Without the
 * flag each iteration runs two products (Y = H V, then W = H^T Y), each reading every
 * activation from HBM; at the 7B shapes that is the faster of the two (the single pass is
 * bound by its split-K reductions and loses about half of its L2 re-reads). */
#define DSMZ_PLAN_SINGLE_PASS_POWER_ITER 2u
/* Perturbation's row products on the CUDA cores (fp32 FFMA inside the streaming kernel)
 * even where the tensor-core kernel applies. The tensor-core kernel (the default) computes
 * z^T / eps = X C^T per 128-vector tile on tcgen05 (kind::tf32 with both operands split
 * into tf32 pairs, fp32 accumulation in TMEM) and streams the tile's arrays in 16-byte
 * units; it needs r <= 64 (padded to 16, 32 or 64), a basis width <= 64 and unit-stride,
 * 16-byte-aligned arrays. */
#define DSMZ_PLAN_CUDA_CORE_PERTURB 4u

typedef struct dsmz_plan dsmz_plan;

/* Host-only: validates the specs and builds the launch schedule. All modules share one
 * adapter rank r and all bases one width R (both <= DSMZ_MAX_RANK). */
int dsmz_plan_create(const dsmz_plan_desc* desc, dsmz_plan** out);
void dsmz_plan_destroy(dsmz_plan* plan);
size_t dsmz_plan_table_bytes(const dsmz_plan* plan);      /* device bytes for the tables */
size_t dsmz_plan_workspace_bytes(const dsmz_plan* plan);  /* device scratch of the step */
uint64_t dsmz_plan_rng_increment(const dsmz_plan* plan);  /* generator advance of this plan's draws */
int32_t dsmz_plan_launch_count(const dsmz_plan* plan, int32_t num_iters);  /* kernels per full step */
/* Binds device memory for the tables and the workspace and copies the tables there
 * (one async copy from host memory the plan keeps). Call once before the first step. */
int dsmz_plan_bind(dsmz_plan* plan, void* device_tables, size_t table_bytes,
                   void* workspace, size_t workspace_bytes, dsmz_stream_t stream);

/* How the plan runs the power iteration: 0 on CUDA cores, 1 on tcgen05 tensor cores as two
 * products per iteration, 2 on tcgen05 tensor cores in a single pass over the activations. */
int32_t dsmz_plan_uses_tensor_cores(const dsmz_plan* plan);
/* 1 when the plan runs the perturbation on the tensor cores. */
int32_t dsmz_plan_perturb_on_tensor_cores(const dsmz_plan* plan);
/* Reads and clears the plan's device error word (synchronises the stream): nonzero when a
 * tensor-core kernel gave up on a barrier wait after its time limit. */
int32_t dsmz_plan_device_error(const dsmz_plan* plan, dsmz_stream_t stream);

/* Phase 1 (ds_mezo/controller.py:165-176): power iteration of every basis. */
int dsmz_step_power_iteration(const dsmz_plan* plan, int32_t num_iters, float norm_floor, dsmz_stream_t stream);
/* Same with flags. DSMZ_PI_BASIS_UNCHANGED: the caller guarantees that no basis was written
 * since this plan's last power iteration; the tensor-core path then takes the first
 * iteration's bf16 split of the bases from that iteration's QR apply instead of recomputing
 * it (one launch less). Without a previous iteration on this binding the flag is ignored.
 * No reference counterpart (the reference recomputes from the basis every call). */
#define DSMZ_PI_BASIS_UNCHANGED 1u
int dsmz_step_power_iteration_ex(const dsmz_plan* plan, int32_t num_iters, float norm_floor, uint32_t flags,
                                 dsmz_stream_t stream);

/* Phase 2 (ds_mezo/controller.py:178-193, 236-251, 260-270): Gaussian draws regenerated
 * from the torch Philox stream at (seed, offset), AGZO perturbation z, pos/neg copies,
 * and the rank-local Kalman sums (sum z*beta*mu, sum z^2*(beta^2 var + q)) as two
 * doubles at dsmz_step_kalman_sums(). Sum those across ranks before phase 3. */
int dsmz_step_perturb(const dsmz_plan* plan, uint64_t seed, uint64_t offset, float eps,
                      float beta, float q, float norm_floor, dsmz_stream_t stream);
double* dsmz_step_kalman_sums(const dsmz_plan* plan);   /* 2 doubles per direction */

/* Fused +/- all-gather (one process per GPU of one node, no reference counterpart: the
 * reference has one process). npeers (<= 7) byte distances, multiples of 16, from this
 * plan's +/- copy buffers to each peer's buffers mapped into this process (dsmz_ipc_*):
 * every +/- element the perturbation stores (tensor-core or CUDA-core kernel) is also
 * stored at those distances, so the peers receive this rank's shard over NVLink while the
 * perturbation runs. The buffers are this rank's slices of gather buffers laid out the same
 * on every rank. The stores are complete and visible system-wide when the perturbation
 * kernel has finished: a stream-ordered collective after it (the Kalman-sum all-reduce)
 * orders every rank's reads after every rank's stores. shadow_delta (or NULL): the same for
 * the bf16 factor shadow the update writes (the factor all-gather; a stream-ordered
 * collective after the update orders it). npeers 0 turns both off. */
int dsmz_plan_set_gather_peers(dsmz_plan* plan, int32_t npeers, const int64_t* pos_delta, const int64_t* neg_delta,
                               const int64_t* shadow_delta);
/* CUDA IPC of a device buffer: export writes the 64-byte handle of the allocation holding
 * ptr and ptr's offset in it; import (in another process on the same node) maps it and
 * returns the buffer's address there; close unmaps what import returned. */
#define DSMZ_IPC_HANDLE_BYTES 64
int dsmz_ipc_export(const void* ptr, void* handle, int64_t* offset);
int dsmz_ipc_import(const void* handle, int64_t offset, void** ptr);
int dsmz_ipc_close(void* ptr, int64_t offset);
/* One device-to-device copy of `bytes` on `stream`, for pushing this rank's shard into a
 * peer's buffer mapped by dsmz_ipc_import: a copy engine moves it over NVLink, so it runs
 * beside kernels that hold every SM (the factor all-gather beside the next power iteration).
 * One call per copy. */
int dsmz_peer_copy(void* dst, const void* src, int64_t bytes, dsmz_stream_t stream);

/* The Zc_A draws of direction 0 of the perturbation at (seed, offset)
 * (ds_mezo/controller.py:187-188), issued ahead: they depend on nothing the step computes,
 * so a host can run them on a second stream while dsmz_step_power_iteration runs, and make
 * the perturbation's stream wait for them. The next dsmz_step_perturb with the same seed and
 * offset then skips its own draw. No reference counterpart (an ordering of the same work). */
int dsmz_step_draw(const dsmz_plan* plan, uint64_t seed, uint64_t offset, dsmz_stream_t stream);
int32_t dsmz_plan_directions(const dsmz_plan* plan);

/* Frobenius norms of the plan's fp32 master factors, A then B of each module in module
 * order (2 * num_modules floats into the device array `norms`), with fp64 sums in a fixed
 * order. The reference's perturbation scale is their median times FLT_EPSILON^(1/3)
 * (ds_mezo/controller.py:78-82: torch.median, i.e. the lower middle value of an even count);
 * on several ranks gather the norms, not the factors. */
int dsmz_plan_factor_norms(const dsmz_plan* plan, float* norms, dsmz_stream_t stream);

/* First-step calibration of the bases (replaces the torch.svd_lowrank loop of
 * ds_mezo/controller.py:156-163; the rank choice of :137-154 stays on the host): every
 * basis V becomes V of torch.svd_lowrank(H, q = R, niter), i.e. the top-R Ritz vectors of
 * H^T H on the randomized range finder's subspace, columns by descending singular value,
 * each signed so that its largest entry in the rotation is positive (torch's signs are those
 * of its SVD backend). The sketches are torch.randn(D, R) (T >= D) or torch.randn(T, R)
 * (T < D, where svd_lowrank works on H^T), drawn in basis order from the generator at
 * (seed, offset); the generator advance is dsmz_plan_calibration_rng_increment. R must not
 * exceed min(T, D). singular_values (device, num_bases x R floats, or NULL) receives the
 * values svd_lowrank returns. workspace: device memory of
 * dsmz_plan_calibration_workspace_bytes, 256-byte aligned, free after the call's stream
 * work. */
size_t dsmz_plan_calibration_workspace_bytes(const dsmz_plan* plan);
uint64_t dsmz_plan_calibration_rng_increment(const dsmz_plan* plan);
int32_t dsmz_plan_calibration_launch_count(const dsmz_plan* plan, int32_t niter);
int dsmz_plan_calibrate(const dsmz_plan* plan, uint64_t seed, uint64_t offset, int32_t niter, float norm_floor,
                        void* workspace, size_t workspace_bytes, float* singular_values, dsmz_stream_t stream);

/* Phase 3 (ds_mezo/controller.py:272-286): Kalman observation update of mu/var with the
 * summed scalars, ZO-Muon Newton-Schulz of every updated mu, param -= eta * X.
 * schedule NULL = cubic. */
int dsmz_step_update(const dsmz_plan* plan, float dd, float beta, float q, float eta,
                     float norm_floor, const dsmz_ns_schedule* schedule, dsmz_stream_t stream);

/* Phase 3 for K directions (no reference counterpart; K = 1 is dsmz_step_update): one
 * Kalman observation update with the K projected-gradient scalars dd[0..K-1] (host array)
 * and the summed (y_hat_k, s_k), treating the K x K innovation covariance
 * sum(var1 * z_k * z_l) as diagonal (its off-diagonal terms are O(1/sqrt(n)) for
 * independent directions over n adapter elements):
 *   mu2  = mu1 + var1 * sum_k z_k (dd_k - y_hat_k) / (s_k + norm_floor)
 *   var2 = var1 * (1 - var1 * sum_k z_k^2 / (s_k + norm_floor))
 * then the same Newton-Schulz update of param as dsmz_step_update. */
int dsmz_step_update_directions(const dsmz_plan* plan, const float* dd, int32_t n, float beta, float q,
                                float eta, float norm_floor, const dsmz_ns_schedule* schedule,
                                dsmz_stream_t stream);

/* ---------------------------------------------------------------------------------
 * Timing probes: while set, every launch of kernel `kernel` by the grouped step records
 * start[i] / stop[i] (caller-created cudaEvent_t, passed as void*) on the launch stream,
 * for i = 0 .. capacity-1 in launch order. capacity 0 removes the probe.
 * ------------------------------------------------------------------------------- */
enum dsmz_kernel_id {
  DSMZ_KID_PI_Y = 0,       /* power iteration Y = H V */
  DSMZ_KID_PI_W = 1,       /* power iteration W = H^T Y */
  DSMZ_KID_PI_GRAM = 2,    /* Gram of W (CholeskyQR) */
  DSMZ_KID_PI_CHOL = 3,    /* Cholesky + triangular inverse */
  DSMZ_KID_PI_APPLY = 4,   /* W R^-1 */
  DSMZ_KID_BSIDE = 5,      /* B V and var_B V^2 partial sums */
  DSMZ_KID_COEF = 6,       /* Zc_B draw and QR(B V) per module */
  DSMZ_KID_PERTURB = 7,    /* z, pos/neg, Kalman partial sums */
  DSMZ_KID_KALMAN_SUM = 8, /* sum of the Kalman partials */
  DSMZ_KID_GRAM = 9,       /* Gram of the Kalman-updated momentum */
  DSMZ_KID_NS_SOLVE = 10,  /* Newton-Schulz in Gram space */
  DSMZ_KID_APPLY = 11,     /* Kalman update + param -= eta X */
  DSMZ_KID_PI_SPLIT = 12,  /* [V_hi | V_lo]^T for the tensor-core products */
  DSMZ_KID_DRAW = 13,      /* Zc_A draws in torch's launch layout */
  DSMZ_KID_KALMAN_DIRS = 14, /* K-direction Kalman observation update */
  DSMZ_KID_PI_FUSED = 15,  /* power iteration W = H^T (H V) in one pass (single-pass path) */
  DSMZ_NUM_KIDS = 16
};
int dsmz_plan_set_probe(dsmz_plan* plan, int32_t kernel, void** start_events, void** stop_events,
                        int32_t capacity);
int32_t dsmz_plan_probe_count(const dsmz_plan* plan, int32_t kernel);

#ifdef __cplusplus
}
#endif
#endif /* DSMEZO_H_ */
