/*
 * ipc_b200.h -- C ABI of the B200 (sm_100a) incremental-predictive-coding step.
 *
 * These entry points replace the three fused TileLang operators of
 * laghzen/Lich (package ipc_tilelang) and the trainer's per-step launch loop.
 * Every function takes plain device pointers, sizes and a CUDA stream
 * (cudaStream_t passed as void*; NULL = legacy default stream), allocates
 * nothing, and returns IPC_OK (0) or a negative IPC_ERR_* code; the message
 * of the last failure on the calling thread is ipc_last_error().
 *
 * Layout (reference README.md:43-50): activations are feature-major,
 * row-major [features, batch]; W[l] is row-major [d_l, d_{l+1}]; grouped
 * operands are `groups` such matrices stacked contiguously.  Storage dtype
 * is one of IPC_DT_*; accumulation is always fp32.  Kernels mutate their
 * in/out operands in place, like the reference kernels.
 */
#ifndef IPC_B200_H
#define IPC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define IPC_ABI_VERSION 4

/* return codes */
#define IPC_OK 0
#define IPC_ERR_ARG (-1)         /* bad shape / flag / pointer (reference raises ValueError) */
#define IPC_ERR_UNSUPPORTED (-2) /* valid request this build cannot serve */
#define IPC_ERR_CUDA (-3)        /* a CUDA runtime call failed; see ipc_last_error() */
#define IPC_ERR_TIMEOUT (-4)     /* a bounded device-side wait gave up */
#define IPC_ERR_DEVICE (-5)      /* no sm_100 device current */

/* activations (reference src/ipc_tilelang/activations.py:6-29; identity from
 * weight_update_specialization.py:86) */
#define IPC_ACT_RELU 0
#define IPC_ACT_TANH 1
#define IPC_ACT_SIGMOID 2
#define IPC_ACT_SILU 3
#define IPC_ACT_GELU 4 /* tanh approximation */
#define IPC_ACT_IDENTITY 5

/* storage dtypes */
#define IPC_DT_F32 0
#define IPC_DT_F16 1
#define IPC_DT_BF16 2

/* algorithm selector (`algo` argument); IPC_ALGO_AUTO picks by shape */
#define IPC_ALGO_AUTO 0
#define IPC_ALGO_SIMT 1    /* tiled CUDA-core / mma.sync kernel, any shape */
#define IPC_ALGO_TCGEN05 2 /* tcgen05 + TMEM + TMA tensor-core kernel (16-bit storage) */
#define IPC_ALGO_OUTER 3   /* weight update only: outer-product kernel for small B */

/* Library identity: IPC_ABI_VERSION. */
int ipc_abi_version(void);

/* Message of the last failed call on this thread ("" if none). */
const char* ipc_last_error(void);

/* Number of kernels this library has launched since load (all entry points). */
unsigned long long ipc_launch_count(void);

/*
 * Prediction + error:  E[g] = cast(X_lo[g]) - cast(W[g] @ f(X_up[g]))
 *   x_up [groups, K, B], w [groups, M, K], x_lo [groups, M, B], e [groups, M, B].
 * Replaces build_prediction_error (src/ipc_tilelang/tilelang_kernels.py:114-177)
 * and build_prediction_error_batched (src/ipc_tilelang/layer_batching.py:89-150).
 */
int ipc_pred_err(const void* x_up, const void* w, const void* x_lo, void* e,
                 int M, int K, int B, int groups, int act, int dtype, int algo, void* stream);

/*
 * Prediction + error from a saved activation: same as ipc_pred_err but the
 * first operand is A = f(X_up) already, so no activation is applied.
 * Used by the save-A schedule; no reference counterpart (the reference always
 * recomputes f in this operator, tilelang_kernels.py:159-167).
 */
int ipc_pred_err_saved(const void* a_up, const void* w, const void* x_lo, void* e,
                       int M, int K, int B, int groups, int dtype, int algo, void* stream);

/*
 * Inference update:  X[g] += gamma * (-E[g] + f'(X[g]) * (W_low[g]^T @ E_low[g]))
 *   x [groups, M, B] (in/out), e [groups, M, B], w_low [groups, K, M],
 *   e_low [groups, K, B], a_out [groups, M, B] or NULL.
 * When a_out is non-NULL it receives f(x_new) (save-activation variant).
 * Replaces build_inference_update (tilelang_kernels.py:180-265) and
 * build_inference_update_batched (layer_batching.py:153-248).
 */
int ipc_infer_update(void* x, const void* e, const void* w_low, const void* e_low, void* a_out,
                     int M, int K, int B, int groups, float gamma, int act, int dtype, int algo,
                     void* stream);

/*
 * Weight update:  W[g] = cast(W[g] + alpha * E[g] @ A[g]^T)
 *   w [groups, M, K] (in/out), e [groups, M, B], x_up [groups, K, B].
 * recompute != 0: A = f(x_up);  recompute == 0: x_up already holds A.
 * algo IPC_ALGO_OUTER selects the small-batch outer-product kernel (any B,
 * intended for B <= 16).  The sign is +alpha for every algorithm (the
 * reference's eager small-B path subtracts, weight_update_specialization.py:102;
 * its GEMM kernel and its oracle add, tilelang_kernels.py:320, reference.py:57).
 * Replaces build_weight_update (tilelang_kernels.py:268-349),
 * build_weight_update_batched (layer_batching.py:251-346) and
 * SmallBWeightUpdater (weight_update_specialization.py:63-128).
 */
int ipc_weight_update(void* w, const void* e, const void* x_up, int M, int K, int B, int groups,
                      float alpha, int recompute, int act, int dtype, int algo, void* stream);

/*
 * Weight delta in fp32 without touching W (data-parallel path):
 *   dw[g] (+)= alpha * E[g] @ A[g]^T ; accumulate != 0 adds into dw.
 * Followed by a sum-allreduce of dw across ranks and ipc_weight_apply.
 * No reference counterpart (the reference is single-GPU).
 */
int ipc_weight_delta(float* dw, const void* e, const void* x_up, int M, int K, int B, int groups,
                     float alpha, int recompute, int accumulate, int act, int dtype, int algo,
                     void* stream);

/* Accuracy of a batch on the device: *count += the number of columns b whose
 * largest logit (first on ties) sits in row labels[b].  logits [C, B] in
 * `dtype` (the output of the forward sweep, TileLangIPC.predict), labels int64
 * [B], count one device int (not cleared).  The reference takes the argmax on
 * the host after predict (scripts/train_mnist.py:80-81). */
int ipc_count_correct(const void* logits, int C, int B, const long long* labels, int* count, int dtype,
                      void* stream);
/* W = cast(float(W) + dw) over n elements (the epilogue of ipc_weight_update, split off). */
int ipc_weight_apply(void* w, const float* dw, long long n, int dtype, void* stream);

/*
 * Forward prediction:  OUT[g] = cast(W[g] @ f(X_up[g]))
 *   x_up [groups, K, B], w [groups, M, K], out [groups, M, B].
 * The forward-init sweep of TileLangIPC.initialize_batch (trainer.py:512-515)
 * and the layers of TileLangIPC.predict (trainer.py:828-833), which the
 * reference runs as eager torch matmuls.
 */
int ipc_forward(const void* x_up, const void* w, void* out, int M, int K, int B, int groups, int act, int dtype,
                int algo, void* stream);

/*
 * General fused GEMM: one entry for every operator above, with the operand
 * roles fixed by `mode` (all row-major, `groups` stacked contiguously):
 *   IPC_MODE_PRED    a = W [M,K]     b = X_up/A_up [K,B]  aux = X_lo [M,B]  out = E [M,B]
 *   IPC_MODE_FORWARD a = W [M,K]     b = X_up/A_up [K,B]  out [M,B]; aux2 = f(cast(out)) or NULL
 *   IPC_MODE_INFER   a = W_low [K,M] b = E_low [K,B]      aux = E [M,B]  out = X [M,B] (in/out)
 *                    aux2 = A_out or NULL, scale = gamma
 *   IPC_MODE_WEIGHT  a = E [M,B]     b = X_up/A_up [K,B]  out = W [M,K] (in/out), scale = alpha
 *   IPC_MODE_WDELTA  as WEIGHT with out = dw (fp32 [M,K])
 * flags: IPC_FLAG_ACTIVATE_B applies f to b (otherwise b is a saved activation);
 * IPC_FLAG_AOUT_STORED makes A_out = f(cast(x_new)), the value the recompute
 * mode reads back (default f(x_new), tilelang_kernels.py:231);
 * IPC_FLAG_ACCUMULATE adds into dw.  Without a workspace the tcgen05 kernel
 * serves calls without IPC_FLAG_ACTIVATE_B only (with it, ipc_fused_gemm_ws
 * below).  No single reference counterpart: it subsumes the entries above.
 *
 * IPC_FLAG_MULTIMEM_RED (WDELTA only; tensor-core shapes, 16-bit operands, a
 * stored activation, no IPC_FLAG_ACCUMULATE): `out` is the multicast (NVLS)
 * address of an fp32 buffer bound on every GPU of a group (for example the
 * multicast_ptr of a torch symmetric-memory rendezvous).  The epilogue adds
 * scale * acc into every GPU's copy through the NVSwitch
 * (multimem.red.add.v4.f32), so the weight delta and its all-reduce are one
 * kernel: the reduction traffic leaves each SM tile by tile while later tiles
 * accumulate.  The caller zeroes every copy before the first rank's call and
 * orders all ranks' calls before anyone reads the sum (e.g. a stream-ordered
 * collective on a small tensor); each thread fences at system scope before the
 * kernel ends.  The sum is identical on every GPU but not bitwise repeatable
 * from run to run (the switch adds contributions in arrival order).  Other
 * shapes return IPC_ERR_UNSUPPORTED.  Replaces the data-parallel ΔW
 * reduce-scatter / all-gather; the reference is single-GPU.
 */
#define IPC_MODE_PRED 0
#define IPC_MODE_INFER 1
#define IPC_MODE_WEIGHT 2
#define IPC_MODE_WDELTA 3
#define IPC_MODE_FORWARD 4
#define IPC_FLAG_ACTIVATE_B 1
#define IPC_FLAG_AOUT_STORED 2
#define IPC_FLAG_ACCUMULATE 4
#define IPC_FLAG_MULTIMEM_RED 8
int ipc_fused_gemm(int mode, const void* a, const void* b, void* out, const void* aux, void* aux2, int M, int K,
                   int B, int groups, float scale, int flags, int act, int dtype, int algo, void* stream);

/*
 * ipc_fused_gemm with a caller-owned fp32 workspace (16-byte aligned device
 * memory, contents need not be initialised).  A weight update (WEIGHT /
 * WDELTA) whose output has fewer 128-row tiles than half the SMs and whose
 * batch reduction is long is split over the batch ("split-K"): each split
 * writes an fp32 partial tile into the workspace and a second pass sums the
 * partials in split order (deterministic) and applies the epilogue.  The
 * number of splits is bounded by workspace_bytes / (groups*M*K*4), so any
 * size works; 0 bytes is exactly ipc_fused_gemm.  Calls sharing a workspace
 * must be ordered on one stream.
 * With IPC_FLAG_ACTIVATE_B (P, FORWARD, WEIGHT, WDELTA) and a tensor-core
 * shape, the head of the workspace (groups*K*B 16-bit elements, rounded up to
 * 256 bytes) first receives A = cast(f(b)) in one elementwise pass, and the
 * tcgen05 GEMM runs on that stored activation; the rest of the workspace
 * serves the split-K partials.  This is the path of the reference's
 * recompute-mode operators (build_prediction_error, tilelang_kernels.py:
 * 143-167; build_weight_update(recompute_activation=True), :288-321), which
 * apply f to the B tile inside the GEMM: on tensor cores that would evaluate f
 * once per 128-row output tile (M/128 times per element).  A workspace too
 * small for the activation leaves such a call on the generic kernel, which
 * applies f while staging its tiles.  ipc_fused_gemm_ws_bytes gives the size.
 * No reference counterpart for the split: the reference's weight kernel
 * reduces the batch inside one CTA per output tile (tilelang_kernels.py:
 * 269-320).
 */
int ipc_fused_gemm_ws(int mode, const void* a, const void* b, void* out, const void* aux, void* aux2, int M, int K,
                      int B, int groups, float scale, int flags, int act, int dtype, int algo, void* workspace,
                      size_t workspace_bytes, void* stream);
/* Per-call overrides of the tensor-core kernel's launch heuristics; 0 in a field
 * keeps the library's choice.  They change which tiles, splits and CTA count
 * compute a result, never what is computed: the output of a weight update can
 * differ in its last bits between split counts (another summation order).
 * Filled from a per-shape tuning table (KernelConfig rows of the reference's
 * tuning.py:10-108 format; a sweep on the target GPU measures them). */
typedef struct ipc_gemm_tune {
  int bn;       /* output tile width, 128 or 256 */
  int splits;   /* weight modes: 1 = no split-K; >= 2 = that many batch ranges
                   (bounded by the workspace and the batch's 64-column blocks) */
  int raster;   /* M-tiles per raster band of the persistent tile walk */
  int max_ctas; /* persistent CTAs (also bounded by ipc_set_max_ctas and the SMs) */
  int pair;     /* CTA pairs -- 256 x 256 tiles computed by two CTAs of a cluster with
                   cta_group::2 MMAs (each CTA holds 128 rows of A and 128 columns of B);
                   for tiles of width 256 that do not split the batch.  0: the launcher's
                   choice (pairs unless row padding makes single CTAs cheaper), 1: single
                   CTAs, 2: pairs */
} ipc_gemm_tune_t;
/* ipc_fused_gemm_ws with optional overrides (tune == NULL: exactly
 * ipc_fused_gemm_ws).  IPC_ERR_ARG for bn outside {0, 128, 256} or negative
 * fields.  Calls the tensor-core kernel does not serve ignore tune.  No
 * reference counterpart (the reference passes a KernelConfig to its JIT
 * compiler, tilelang_kernels.py:114-349). */
int ipc_fused_gemm_tuned(int mode, const void* a, const void* b, void* out, const void* aux, void* aux2, int M,
                         int K, int B, int groups, float scale, int flags, int act, int dtype, int algo,
                         void* workspace, size_t workspace_bytes, const ipc_gemm_tune_t* tune, void* stream);
/* Split-K partials: this many bytes cover every weight update the kernel splits. */
#define IPC_SPLITK_WS_BYTES (16u << 20)
/* Workspace bytes ipc_fused_gemm_ws uses for this call (*bytes = 0: it needs
 * none): the stored activation when IPC_FLAG_ACTIVATE_B meets a tensor-core
 * shape, plus IPC_SPLITK_WS_BYTES for a tensor-core weight update.  Launches
 * nothing; the answer depends only on the arguments and the current device.
 * No reference counterpart (cf. a library's workspace-size query). */
int ipc_fused_gemm_ws_bytes(int mode, int M, int K, int B, int groups, int flags, int dtype, int algo,
                            size_t* bytes);

/*
 * Split-K weight update that allocates nothing: ipc_fused_gemm_ws for
 * IPC_MODE_WEIGHT / IPC_MODE_WDELTA (same operands, flags, act, algo) with
 * the fp32 partial tiles in a scratch array compiled into this library,
 * IPC_NOALLOC_SCRATCH_BYTES per device, instead of caller memory.  For
 * callers that hold no device allocator of their own: a host runtime bound
 * over the C ABI (cgo, JNI, ctypes) that was handed only the operand buffers
 * and must not cudaMalloc behind the back of the framework that owns the
 * device memory (a caching allocator that does not see such memory can run
 * the device out of it), or a step that runs under a fixed memory budget.
 *   - Limit: groups*M*K <= IPC_NOALLOC_MAX_OUT_ELEMS; larger requests return
 *     IPC_ERR_ARG (use ipc_fused_gemm_ws with a caller workspace instead).
 *     Within the limit the split count equals ipc_fused_gemm_ws with a
 *     16 MiB workspace.  Other modes return IPC_ERR_ARG.
 *   - Nothing in the scratch has to start at zero: every partial tile is
 *     written before the reduce pass reads it.
 *   - The scratch is one array per device, shared by every caller in the
 *     process: calls on one device whose kernels can overlap (different
 *     streams, or host threads without ordering) race on it.  Order them on
 *     one stream.
 *   - The first call on each device does set-up (looks up the scratch
 *     address with cudaGetSymbolAddress, with that device current); make it
 *     before any stream capture.  The address is kept for the life of the
 *     process: after a cudaDeviceReset of that device it is stale, so do not
 *     call this entry point on a device that was reset.
 *   - sm_100 devices only (IPC_ERR_DEVICE elsewhere), like every entry point
 *     of this library; a split-K weight update is all it ever runs.
 * No counterpart in the reference.
 */
#define IPC_NOALLOC_SCRATCH_BYTES (16u << 20)
#define IPC_NOALLOC_MAX_OUT_ELEMS (1u << 20)
int ipc_weight_update_noalloc(int mode, const void* e, const void* a_up, void* out, int M, int K, int B, int groups,
                              float alpha, int flags, int act, int dtype, int algo, void* stream);

/*
 * Weight update with an optimizer applied where the product meets W, so no
 * gradient tensor is written to memory (the reference lists a fused AdamW /
 * SGD epilogue as future work, README.md:168, PERFORMANCE_CHECKLIST.md:
 * 103-104; no counterpart exists).  The gradient of the energy
 * sum_l |e_l|^2 / 2 with respect to W is g = -E @ A^T (summed over the batch),
 * A = f(x_up) when recompute != 0.  Per element of W (fp32 arithmetic, W
 * stored in `dtype`, state in fp32 with W's layout, 16-byte aligned):
 *   IPC_OPT_SGD   (torch.optim.SGD, dampening 0, no Nesterov; buffer starts at 0):
 *       g += weight_decay * w;  m = momentum * m + g (if m != NULL);  w -= lr * m (or g)
 *   IPC_OPT_ADAMW (torch.optim.AdamW; step t >= 1 counts from 1):
 *       w *= 1 - lr * weight_decay;  m = b1 m + (1 - b1) g;  v = b2 v + (1 - b2) g^2;
 *       w -= lr / (1 - b1^t) * m / (sqrt(v) / sqrt(1 - b2^t) + eps)
 * IPC_OPT_SGD with momentum 0, weight_decay 0 is ipc_weight_update with
 * alpha = lr.  Paths: tcgen05 (epilogue, or the split-K reduce pass with the
 * workspace), the small-batch outer-product kernel; shapes neither serves
 * need workspace_bytes >= groups*M*K*4 (an fp32 product, then the step).
 */
#define IPC_OPT_SGD 1
#define IPC_OPT_ADAMW 2
typedef struct ipc_optim {
  int kind;
  float lr, momentum, weight_decay, beta1, beta2, eps;
  int step;  /* AdamW: this update's step number, >= 1 */
  float* m;  /* SGD momentum buffer (NULL without momentum) / AdamW first moment */
  float* v;  /* AdamW second moment */
} ipc_optim_t;
int ipc_weight_update_opt(void* w, const void* e, const void* x_up, int M, int K, int B, int groups,
                          const ipc_optim_t* opt, int recompute, int act, int dtype, int algo, void* workspace,
                          size_t workspace_bytes, void* stream);
/* First error a device-side bounded wait recorded since the last clear
 * (IPC_OK if none; IPC_ERR_TIMEOUT when a pipeline wait gave up).  Synchronises
 * with the device; clear != 0 resets the word.  No reference counterpart. */
int ipc_device_status(int* status, int clear);

/* Failure-detection self-test of the bounded device waits: launches a 2-CTA
 * kernel in which one CTA never reaches the grid barrier used by the wide
 * small-batch kernel; the other gives up after limit_us microseconds (1 ..
 * 1e6), records IPC_ERR_TIMEOUT in the device status (ipc_device_status) and
 * returns.  Nothing faults and the context stays usable.  sync:
 * IPC_NET_SYNC_BYTES of device memory.  No reference counterpart. */
int ipc_selftest_barrier_timeout(void* sync, int limit_us, void* stream);

/* Cap on the CTAs of the persistent tensor-core GEMM (max_ctas = 0: one per
 * SM, the default).  Its CTAs otherwise fill every SM, so a collective
 * launched beside it (the data-parallel path's NCCL all-reduce of the weight
 * deltas, issued while later layers' deltas are still being formed) waits for
 * them; with SMs left over the two run concurrently.  Process-wide, read when
 * a GEMM is launched; IPC_ERR_ARG for max_ctas < 0.  No reference
 * counterpart. */
int ipc_set_max_ctas(int max_ctas);

/* A = cast(f(X)) over n elements (materialise a saved activation). */
int ipc_activate(void* a, const void* x, long long n, int act, int dtype, void* stream);

/* ---------------------------------------------------------------------------
 * Persistent multi-layer network kernel (small widths).
 *
 * One launch runs `steps` training steps of `nets` independent networks.
 * Network n's buffers are the n-th slab of each stacked array below.
 * A training step is: (optionally) load a batch from the pool into x[L] and
 * x[0]; (optionally) the forward-init sweep x[l] = W[l] f(x[l+1]),
 * l = L-1..1 (trainer.py:509-516); T inference iterations, each all
 * prediction errors then all state updates (trainer.py:609-638); then, if
 * update_weights, W[l] += alpha e[l] f(x[l+1])^T for every l with the errors
 * of the last iteration and the updated states (reference.py:52-57).
 * With pool == NULL, forward_init == 0, T == 1 and update_weights == 1 a call
 * is exactly TileLangIPC.step_initialized (trainer.py:601-679).
 * Two kernels serve it (ipc_net_plan answers which, and whether either can):
 *  - small widths: d_0 .. d_{L-1} <= 64, d_L a multiple of 8, B a multiple of
 *    8 and <= 256, the per-CTA layout fits in shared memory; one cluster of
 *    CTAs per network, any number of networks (nets);
 *  - wide networks at small batch (everything else with 1 <= B <= 16, every
 *    d_l <= 4096, nets == 1): one cooperative grid, one CTA per SM, phases
 *    separated by bounded grid barriers; needs run->sync.
 * Both: 1 <= L <= IPC_NET_MAX_LAYERS, 16-bit storage, recompute mode.
 * --------------------------------------------------------------------------- */
#define IPC_NET_MAX_LAYERS 8

typedef struct ipc_net {
  int L;                            /* number of weight matrices */
  int dims[IPC_NET_MAX_LAYERS + 1]; /* d_0 (classes) .. d_L (input) */
  int B;                            /* batch columns per network */
  int nets;                         /* independent networks */
  void* w[IPC_NET_MAX_LAYERS];      /* W[l]: [nets, d_l, d_{l+1}] */
  void* x[IPC_NET_MAX_LAYERS + 1];  /* x[l]: [nets, d_l, B] */
  void* e[IPC_NET_MAX_LAYERS + 1];  /* e[l]: [nets, d_l, B] (e[L] unused, may be NULL) */
  void* a[IPC_NET_MAX_LAYERS + 1];  /* optional activation cache a[l] = cast(f(x[l])), [nets, d_l, B],
                                       l >= 1, used by the wide small-batch kernel (contents on
                                       entry ignored; NULL entries: f is recomputed where read) */
} ipc_net_t;

typedef struct ipc_net_run {
  const void* pool_x; /* [pool_batches, nets, d_L, B] or NULL (use x[L] as is) */
  const void* pool_y; /* [pool_batches, nets, d_0, B] or NULL (use x[0] as is) */
  int pool_batches;
  int first_batch;    /* step s uses batch (first_batch + s) % pool_batches */
  int steps;          /* training steps in this launch */
  int T;              /* inference iterations per training step */
  int forward_init;   /* run the forward-init sweep at the start of each step */
  int update_weights; /* weight update after the T-th iteration */
  int recompute;      /* 1: f recomputed from stored x (reference recompute mode) */
  float alpha, gamma;
  int act, dtype;
  int cluster;        /* CTAs per network (0 = auto) */
  float* energy;      /* [steps, nets] or NULL: sum_l<L mean(e[l]^2) of the last iteration of
                         each step (reference.py:58); zeroed by the call */
  long long* phase_ns; /* [min(steps, IPC_NET_TRACE_STEPS), IPC_NET_TRACE_PHASES] or NULL:
                          %globaltimer stamps (ns) taken by CTA 0 of network 0 at the end of
                          each phase of a step (tracing; no work is skipped).  The wide
                          small-batch kernel fills slots 0-6: step start, batch ready,
                          forward sweep done, first P, first I, last iteration, weights */
  void* sync;         /* IPC_NET_SYNC_BYTES of device memory for the grid barrier of the
                         wide small-batch kernel (zeroed by the call; one per launch in
                         flight); NULL for the small-width kernel */
} ipc_net_run_t;

#define IPC_NET_SYNC_BYTES 64

#define IPC_NET_TRACE_STEPS 64
#define IPC_NET_TRACE_PHASES 12 /* start, mu-partial, barrier A, mu-sum, forward, iterations,
                                   energy, barrier B, input-layer update, hidden updates,
                                   batch ready, end */

/* Whether ipc_net_train can run this network: IPC_OK and the cluster size
 * (CTAs per network; 0 for the wide small-batch kernel, whose grid is one
 * CTA per SM) and dynamic shared memory per CTA it would use, or an IPC_ERR_*
 * code.  cluster = 0 lets the library choose.  Launches nothing.
 * No reference counterpart (a planning query of the persistent kernel). */
int ipc_net_plan(const ipc_net_t* net, int cluster, int* cluster_out, int* smem_bytes_out);

/* Replaces the TileLangIPC.step_initialized launch loop (trainer.py:601-679)
 * and the steady-state graph of IPCGraphRunner (cuda_graph.py:22-31). */
int ipc_net_train(const ipc_net_t* net, const ipc_net_run_t* run, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* IPC_B200_H */
