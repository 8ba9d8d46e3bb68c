#include <cmath>
// C ABI entry points (include/ipc_b200.h): argument checks, algorithm choice,
// error reporting.  No allocation happens here; all buffers are caller-owned.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "ipc_common.cuh"
#include "ipc_elementwise.cuh"
#include "ipc_generic.cuh"
#include "ipc_tc.cuh"

namespace ipc {

namespace {
thread_local char g_last_error[512] = "";
std::atomic<unsigned long long> g_launches{0};
int g_arch_ok[64] = {0};  // 0 unknown, 1 sm_100, -1 other
}  // namespace

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return set_error(IPC_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(err));
  return IPC_OK;
}

void count_launch(unsigned long long n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

int require_sm100() {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return set_error(IPC_ERR_DEVICE, "no CUDA device: %s", cudaGetErrorString(err));
  if (dev >= 0 && dev < 64 && g_arch_ok[dev] == 1) return IPC_OK;
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0) {
    if (dev >= 0 && dev < 64) g_arch_ok[dev] = -1;
    return set_error(IPC_ERR_DEVICE, "this library is built for sm_100a (B200); device %d is sm_%d%d", dev, major,
                     minor);
  }
  if (dev >= 0 && dev < 64) g_arch_ok[dev] = 1;
  return IPC_OK;
}

}  // namespace ipc

using namespace ipc;

#define IPC_REQUIRE(cond, ...) \
  do {                         \
    if (!(cond)) return set_error(IPC_ERR_ARG, __VA_ARGS__); \
  } while (0)

// Bytes of workspace the stored activation A = cast(f(B)) of a [groups][K][B] 16-bit operand takes (a
// multiple of 256, so the split-K partials behind it stay aligned).
static size_t activation_ws_bytes(int groups, int K, int B) {
  return ((size_t)groups * K * B * 2 + 255) / 256 * 256;
}

static int common_checks(int M, int K, int B, int groups, int act, int dtype, int algo) {
  IPC_REQUIRE(M >= 0 && K >= 0 && B >= 0, "negative size (M=%d K=%d B=%d)", M, K, B);
  IPC_REQUIRE(groups >= 1, "groups must be >= 1 (got %d)", groups);
  IPC_REQUIRE(act >= IPC_ACT_RELU && act <= IPC_ACT_IDENTITY, "unknown activation code %d", act);
  IPC_REQUIRE(dtype >= IPC_DT_F32 && dtype <= IPC_DT_BF16, "unknown dtype code %d", dtype);
  IPC_REQUIRE(algo >= IPC_ALGO_AUTO && algo <= IPC_ALGO_OUTER, "unknown algo code %d", algo);
  return require_sm100();
}

extern "C" {

int ipc_abi_version(void) { return IPC_ABI_VERSION; }

const char* ipc_last_error(void) { return g_last_error; }

unsigned long long ipc_launch_count(void) { return g_launches.load(); }

static int pred_err_impl(const void* x_up, const void* w, const void* x_lo, void* e, int M, int K, int B,
                         int groups, int act, int dtype, int algo, void* stream, bool bact) {
  int rc = common_checks(M, K, B, groups, act, dtype, algo);
  if (rc) return rc;
  IPC_REQUIRE(algo != IPC_ALGO_OUTER, "IPC_ALGO_OUTER applies to the weight update only");
  if (M == 0 || B == 0) return IPC_OK;
  IPC_REQUIRE(x_lo && e && (K == 0 || (x_up && w)), "null operand pointer");
  GemmArgs p{};
  p.A = w; p.lda = K; p.gsA = (long long)M * K;
  p.Bm = x_up; p.ldb = B; p.gsB = (long long)K * B;
  p.Mg = M; p.Ng = B; p.Kg = K; p.groups = groups;
  p.out = e; p.gsOut = (long long)M * B;
  p.aux = x_lo; p.gsAux = (long long)M * B;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (tc_eligible(MODE_P, M, K, B, dtype, algo, bact)) return launch_tc(p, MODE_P, act, dtype, s);
  if (algo == IPC_ALGO_TCGEN05) return set_error(IPC_ERR_UNSUPPORTED, "tcgen05 path: shape/dtype not eligible (M=%d K=%d B=%d dtype=%d)", M, K, B, dtype);
  if (skinny_eligible(MODE_P, M, K, B, dtype, algo)) return launch_skinny(p, MODE_P, bact, act, dtype, s);
  return launch_generic(p, MODE_P, bact, act, dtype, s);
}

int ipc_pred_err(const void* x_up, const void* w, const void* x_lo, void* e, int M, int K, int B, int groups,
                 int act, int dtype, int algo, void* stream) {
  return pred_err_impl(x_up, w, x_lo, e, M, K, B, groups, act, dtype, algo, stream, true);
}

int ipc_pred_err_saved(const void* a_up, const void* w, const void* x_lo, void* e, int M, int K, int B, int groups,
                       int dtype, int algo, void* stream) {
  return pred_err_impl(a_up, w, x_lo, e, M, K, B, groups, IPC_ACT_IDENTITY, dtype, algo, stream, false);
}

int ipc_forward(const void* x_up, const void* w, void* out, int M, int K, int B, int groups, int act, int dtype,
                int algo, void* stream) {
  int rc = common_checks(M, K, B, groups, act, dtype, algo);
  if (rc) return rc;
  IPC_REQUIRE(algo != IPC_ALGO_OUTER, "IPC_ALGO_OUTER applies to the weight update only");
  if (M == 0 || B == 0) return IPC_OK;
  IPC_REQUIRE(out && (K == 0 || (x_up && w)), "null operand pointer");
  GemmArgs p{};
  p.A = w; p.lda = K; p.gsA = (long long)M * K;
  p.Bm = x_up; p.ldb = B; p.gsB = (long long)K * B;
  p.Mg = M; p.Ng = B; p.Kg = K; p.groups = groups;
  p.out = out; p.gsOut = (long long)M * B;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (tc_eligible(MODE_F, M, K, B, dtype, algo, true)) return launch_tc(p, MODE_F, act, dtype, s);
  if (algo == IPC_ALGO_TCGEN05) return set_error(IPC_ERR_UNSUPPORTED, "tcgen05 path: shape/dtype not eligible (M=%d K=%d B=%d dtype=%d)", M, K, B, dtype);
  if (skinny_eligible(MODE_F, M, K, B, dtype, algo)) return launch_skinny(p, MODE_F, true, act, dtype, s);
  return launch_generic(p, MODE_F, true, act, dtype, s);
}

int ipc_infer_update(void* x, const void* e, const void* w_low, const void* e_low, void* a_out, int M, int K, int B,
                     int groups, float gamma, int act, int dtype, int algo, void* stream) {
  int rc = common_checks(M, K, B, groups, act, dtype, algo);
  if (rc) return rc;
  IPC_REQUIRE(algo != IPC_ALGO_OUTER, "IPC_ALGO_OUTER applies to the weight update only");
  if (M == 0 || B == 0) return IPC_OK;
  IPC_REQUIRE(x && e && (K == 0 || (w_low && e_low)), "null operand pointer");
  GemmArgs p{};
  p.A = w_low; p.lda = M; p.gsA = (long long)K * M;
  p.Bm = e_low; p.ldb = B; p.gsB = (long long)K * B;
  p.Mg = M; p.Ng = B; p.Kg = K; p.groups = groups;
  p.out = x; p.gsOut = (long long)M * B;
  p.aux = e; p.gsAux = (long long)M * B;
  p.aux2 = a_out; p.gsAux2 = (long long)M * B;
  p.scale = gamma;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (tc_eligible(MODE_I, M, K, B, dtype, algo, false)) return launch_tc(p, MODE_I, act, dtype, s);
  if (algo == IPC_ALGO_TCGEN05) return set_error(IPC_ERR_UNSUPPORTED, "tcgen05 path: shape/dtype not eligible (M=%d K=%d B=%d dtype=%d)", M, K, B, dtype);
  if (skinny_eligible(MODE_I, M, K, B, dtype, algo)) return launch_skinny(p, MODE_I, false, act, dtype, s);
  return launch_generic(p, MODE_I, false, act, dtype, s);
}

static int weight_impl(void* out, const void* e, const void* x_up, int M, int K, int B, int groups, float alpha,
                       int recompute, int accumulate, int act, int dtype, int algo, void* stream, bool delta) {
  int rc = common_checks(M, K, B, groups, act, dtype, algo);
  if (rc) return rc;
  if (M == 0 || K == 0) return IPC_OK;
  IPC_REQUIRE(out && (B == 0 || (e && x_up)), "null operand pointer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool bact = recompute != 0;
  if (algo == IPC_ALGO_OUTER || (algo == IPC_ALGO_AUTO && B <= 16))
    return launch_outer(out, e, x_up, M, K, B, groups, alpha, bact, delta, accumulate, act, dtype, s);
  GemmArgs p{};
  p.A = e; p.lda = B; p.gsA = (long long)M * B;
  p.Bm = x_up; p.ldb = B; p.gsB = (long long)K * B;
  p.Mg = M; p.Ng = K; p.Kg = B; p.groups = groups;
  p.out = out; p.gsOut = (long long)M * K;
  p.scale = alpha;
  p.accumulate = accumulate;
  const int mode = delta ? MODE_WD : MODE_W;
  if (tc_eligible(mode, M, K, B, dtype, algo, bact)) return launch_tc(p, mode, act, dtype, s);
  if (algo == IPC_ALGO_TCGEN05) return set_error(IPC_ERR_UNSUPPORTED, "tcgen05 path: shape/dtype not eligible (M=%d K=%d B=%d dtype=%d)", M, K, B, dtype);
  return launch_generic(p, mode, bact, act, dtype, s);
}

int ipc_weight_update(void* w, const void* e, const void* x_up, int M, int K, int B, int groups, float alpha,
                      int recompute, int act, int dtype, int algo, void* stream) {
  return weight_impl(w, e, x_up, M, K, B, groups, alpha, recompute, 0, act, dtype, algo, stream, false);
}

int ipc_weight_delta(float* dw, const void* e, const void* x_up, int M, int K, int B, int groups, float alpha,
                     int recompute, int accumulate, int act, int dtype, int algo, void* stream) {
  return weight_impl(dw, e, x_up, M, K, B, groups, alpha, recompute, accumulate, act, dtype, algo, stream, true);
}

int ipc_weight_update_opt(void* w, const void* e, const void* x_up, int M, int K, int B, int groups,
                          const ipc_optim_t* opt, int recompute, int act, int dtype, int algo, void* workspace,
                          size_t workspace_bytes, void* stream) {
  int rc = common_checks(M, K, B, groups, act, dtype, algo);
  if (rc) return rc;
  IPC_REQUIRE(opt != nullptr, "null optimizer descriptor");
  IPC_REQUIRE(opt->kind == IPC_OPT_SGD || opt->kind == IPC_OPT_ADAMW, "unknown optimizer kind %d", opt->kind);
  IPC_REQUIRE(workspace != nullptr || workspace_bytes == 0, "workspace_bytes > 0 with a null workspace");
  IPC_REQUIRE(reinterpret_cast<uintptr_t>(workspace) % 16 == 0, "workspace must be 16-byte aligned");
  const bool adam = opt->kind == IPC_OPT_ADAMW;
  IPC_REQUIRE(!adam || (opt->m && opt->v), "AdamW needs both moment buffers");
  IPC_REQUIRE(!adam || opt->step >= 1, "AdamW step must be >= 1 (got %d)", opt->step);
  IPC_REQUIRE(adam || opt->momentum == 0.f || opt->m, "SGD with momentum needs its buffer");
  IPC_REQUIRE(((reinterpret_cast<uintptr_t>(opt->m) | reinterpret_cast<uintptr_t>(opt->v)) & 15) == 0,
              "optimizer state must be 16-byte aligned");
  if (M == 0 || K == 0 || B == 0) return IPC_OK;  // an empty batch leaves W and the state as they are
  IPC_REQUIRE(w && e && x_up, "null operand pointer");
  OptParams o{};
  o.kind = opt->kind;
  o.lr = opt->lr;
  o.momentum = opt->momentum;
  o.wd = opt->weight_decay;
  o.b1 = opt->beta1;
  o.b2 = opt->beta2;
  o.eps = opt->eps;
  o.m = opt->m;
  o.v = adam ? opt->v : nullptr;
  if (!adam && opt->momentum == 0.f) o.m = nullptr;
  if (adam) {
    o.step_size = (float)(opt->lr / (1.0 - std::pow((double)opt->beta1, (double)opt->step)));
    o.rsqrt_bc2 = (float)(1.0 / std::sqrt(1.0 - std::pow((double)opt->beta2, (double)opt->step)));
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool bact = recompute != 0;
  if (algo == IPC_ALGO_OUTER || (algo == IPC_ALGO_AUTO && B <= 16))
    return launch_outer(w, e, x_up, M, K, B, groups, 1.f, bact, false, 0, act, dtype, s, &o);
  GemmArgs p{};
  p.A = e; p.lda = B; p.gsA = (long long)M * B;
  p.Bm = x_up; p.ldb = B; p.gsB = (long long)K * B;
  p.Mg = M; p.Ng = K; p.Kg = B; p.groups = groups;
  p.out = w; p.gsOut = (long long)M * K;
  p.scale = 1.f;
  p.opt = o;
  float* ws = static_cast<float*>(workspace);
  size_t ws_bytes = workspace_bytes;
  if (bact) {  // f(x_up) stored once in the head of the workspace (the tensor-core kernel reads it as is)
    const size_t act_bytes = activation_ws_bytes(groups, K, B);
    if (tc_eligible(MODE_WO, M, K, B, dtype, algo, false, false) && ws != nullptr && ws_bytes >= act_bytes &&
        (reinterpret_cast<uintptr_t>(x_up) & 15) == 0) {
      rc = launch_activate(ws, x_up, (long long)groups * K * B, act, dtype, s);
      if (rc) return rc;
      p.Bm = ws;
      ws = ws_bytes > act_bytes ? reinterpret_cast<float*>(reinterpret_cast<char*>(ws) + act_bytes) : nullptr;
      ws_bytes = ws ? ws_bytes - act_bytes : 0;
      return launch_tc(p, MODE_WO, act, dtype, s, ws, ws_bytes);
    }
  } else if (tc_eligible(MODE_WO, M, K, B, dtype, algo, false, ws != nullptr)) {
    return launch_tc(p, MODE_WO, act, dtype, s, ws, ws_bytes);
  }
  // other shapes: the fp32 product E A^T in the workspace, then the step
  IPC_REQUIRE(ws != nullptr && workspace_bytes >= (size_t)groups * M * K * 4,
              "optimizer update of this shape needs workspace_bytes >= groups*M*K*4 (%lld)",
              (long long)groups * M * K * 4);
  p.out = workspace;
  p.scale = 1.f;
  p.accumulate = 0;
  rc = launch_generic(p, MODE_WD, bact, act, dtype, s);
  if (rc) return rc;
  return launch_opt_apply(w, static_cast<const float*>(workspace), (long long)groups * M * K, dtype, o, s);
}

int ipc_count_correct(const void* logits, int C, int B, const long long* labels, int* count, int dtype,
                      void* stream) {
  int rc = common_checks(1, 1, 1, 1, IPC_ACT_IDENTITY, dtype, IPC_ALGO_AUTO);
  if (rc) return rc;
  IPC_REQUIRE(C >= 1 && B >= 0, "C must be >= 1 and B >= 0 (C=%d B=%d)", C, B);
  if (B == 0) return IPC_OK;
  IPC_REQUIRE(logits && labels && count, "null operand pointer");
  return launch_count_correct(logits, C, B, labels, count, dtype, reinterpret_cast<cudaStream_t>(stream));
}

int ipc_weight_apply(void* w, const float* dw, long long n, int dtype, void* stream) {
  int rc = common_checks(1, 1, 1, 1, IPC_ACT_IDENTITY, dtype, IPC_ALGO_AUTO);
  if (rc) return rc;
  IPC_REQUIRE(n >= 0, "negative element count");
  if (n == 0) return IPC_OK;
  IPC_REQUIRE(w && dw, "null operand pointer");
  return launch_apply(w, dw, n, dtype, reinterpret_cast<cudaStream_t>(stream));
}

int ipc_activate(void* a, const void* x, long long n, int act, int dtype, void* stream) {
  int rc = common_checks(1, 1, 1, 1, act, dtype, IPC_ALGO_AUTO);
  if (rc) return rc;
  IPC_REQUIRE(n >= 0, "negative element count");
  if (n == 0) return IPC_OK;
  IPC_REQUIRE(a && x, "null operand pointer");
  return launch_activate(a, x, n, act, dtype, reinterpret_cast<cudaStream_t>(stream));
}

static int fused_gemm_impl(int mode, const void* a, const void* b, void* out, const void* aux, void* aux2, int M, int K,
                           int B, int groups, float scale, int flags, int act, int dtype, int algo, float* ws,
                           size_t ws_bytes, void* stream, const TcTune* tune = nullptr) {
  int rc = common_checks(M, K, B, groups, act, dtype, algo);
  if (rc) return rc;
  IPC_REQUIRE(mode >= MODE_P && mode <= MODE_F, "unknown mode %d", mode);
  IPC_REQUIRE(algo != IPC_ALGO_OUTER || mode == MODE_W || mode == MODE_WD,
              "IPC_ALGO_OUTER applies to the weight update only");
  const bool bact = (flags & IPC_FLAG_ACTIVATE_B) != 0;
  IPC_REQUIRE(!(mode == MODE_I && bact), "the inference update takes E_low as is");
  GemmArgs p{};
  p.scale = scale;
  p.accumulate = (flags & IPC_FLAG_ACCUMULATE) != 0;
  p.a_out_from_stored = (flags & IPC_FLAG_AOUT_STORED) != 0;
  p.groups = groups;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (flags & IPC_FLAG_MULTIMEM_RED) {
    // the weight delta added into a multicast buffer on every GPU of a group: tcgen05 staged epilogue only
    IPC_REQUIRE(mode == MODE_WD, "IPC_FLAG_MULTIMEM_RED applies to IPC_MODE_WDELTA only");
    IPC_REQUIRE(!p.accumulate && !bact, "IPC_FLAG_MULTIMEM_RED excludes IPC_FLAG_ACCUMULATE and IPC_FLAG_ACTIVATE_B");
    if (M == 0 || K == 0) return IPC_OK;
    IPC_REQUIRE(out && (B == 0 || (a && b)), "null operand pointer");
    if (B == 0 || algo == IPC_ALGO_SIMT || algo == IPC_ALGO_OUTER ||
        !tc_eligible(mode, M, K, B, dtype, algo, false, false))
      return set_error(IPC_ERR_UNSUPPORTED, "IPC_FLAG_MULTIMEM_RED: M=%d K=%d B=%d dtype=%d is not a tcgen05 weight delta",
                       M, K, B, dtype);
    p.A = a; p.lda = B; p.gsA = (long long)M * B;
    p.Bm = b; p.ldb = B; p.gsB = (long long)K * B;
    p.Mg = M; p.Ng = K; p.Kg = B;
    p.out = out; p.gsOut = (long long)M * K;
    p.mcast = 1;
    return launch_tc(p, mode, act, dtype, s, nullptr, 0, tune);
  }
  if (mode == MODE_W || mode == MODE_WD) {
    if (M == 0 || K == 0) return IPC_OK;
    IPC_REQUIRE(out && (B == 0 || (a && b)), "null operand pointer");
    if (algo == IPC_ALGO_OUTER || (algo == IPC_ALGO_AUTO && B <= 16))
      return launch_outer(out, a, b, M, K, B, groups, scale, bact, mode == MODE_WD, p.accumulate, act, dtype, s);
    p.A = a; p.lda = B; p.gsA = (long long)M * B;
    p.Bm = b; p.ldb = B; p.gsB = (long long)K * B;
    p.Mg = M; p.Ng = K; p.Kg = B;
    p.out = out; p.gsOut = (long long)M * K;
  } else {
    if (M == 0 || B == 0) return IPC_OK;
    IPC_REQUIRE(out && (K == 0 || (a && b)), "null operand pointer");
    IPC_REQUIRE(mode != MODE_P || aux, "prediction error needs X_lo (aux)");
    IPC_REQUIRE(mode != MODE_I || aux, "inference update needs E (aux)");
    p.A = a; p.lda = (mode == MODE_I) ? M : K; p.gsA = (long long)M * K;
    p.Bm = b; p.ldb = B; p.gsB = (long long)K * B;
    p.Mg = M; p.Ng = B; p.Kg = K;
    p.out = out; p.gsOut = (long long)M * B;
    p.aux = aux; p.gsAux = (long long)M * B;
    p.aux2 = aux2; p.gsAux2 = (long long)M * B;
  }
  const bool weight = (mode == MODE_W || mode == MODE_WD);
  if (bact && ws != nullptr) {
    // f on the B operand: materialise A = cast(f(B)) once into the head of the workspace, then run the
    // tensor-core GEMM on the stored activation (the rest of the workspace holds split-K partials).
    // Inside the GEMM f would be evaluated once per 128-row output tile, M/128 times per element.
    const size_t act_bytes = activation_ws_bytes(groups, K, B);
    const bool stored_ok = tc_eligible(mode, M, K, B, dtype, algo, false, weight && ws_bytes > act_bytes);
    if (stored_ok && ws_bytes >= act_bytes && (reinterpret_cast<uintptr_t>(b) & 15) == 0) {
      rc = launch_activate(ws, b, (long long)groups * K * B, act, dtype, s);
      if (rc) return rc;
      p.Bm = ws;
      float* part = ws_bytes > act_bytes ? reinterpret_cast<float*>(reinterpret_cast<char*>(ws) + act_bytes) : nullptr;
      return launch_tc(p, mode, act, dtype, s, part, part ? ws_bytes - act_bytes : 0, tune);
    }
  }
  const bool splitk = ws != nullptr && weight;
  if (tc_eligible(mode, M, K, B, dtype, algo, bact, splitk))
    return launch_tc(p, mode, act, dtype, s, ws, ws_bytes, tune);
  if (algo == IPC_ALGO_TCGEN05)
    return set_error(IPC_ERR_UNSUPPORTED, "tcgen05 path: not eligible (mode=%d M=%d K=%d B=%d dtype=%d activate_b=%d)",
                     mode, M, K, B, dtype, (int)bact);
  if (skinny_eligible(mode, M, K, B, dtype, algo)) return launch_skinny(p, mode, bact, act, dtype, s);
  return launch_generic(p, mode, bact, act, dtype, s);
}

int ipc_fused_gemm(int mode, const void* a, const void* b, void* out, const void* aux, void* aux2, int M, int K, int B,
                   int groups, float scale, int flags, int act, int dtype, int algo, void* stream) {
  return fused_gemm_impl(mode, a, b, out, aux, aux2, M, K, B, groups, scale, flags, act, dtype, algo, nullptr, 0,
                         stream);
}

int ipc_fused_gemm_tuned(int mode, const void* a, const void* b, void* out, const void* aux, void* aux2, int M,
                         int K, int B, int groups, float scale, int flags, int act, int dtype, int algo,
                         void* workspace, size_t workspace_bytes, const ipc_gemm_tune_t* tune, void* stream) {
  IPC_REQUIRE(workspace != nullptr || workspace_bytes == 0, "workspace_bytes > 0 with a null workspace");
  IPC_REQUIRE(reinterpret_cast<uintptr_t>(workspace) % 16 == 0, "workspace must be 16-byte aligned");
  TcTune t{};
  if (tune != nullptr) {
    IPC_REQUIRE(tune->bn == 0 || tune->bn == 128 || tune->bn == 256, "tune.bn must be 0, 128 or 256 (got %d)",
                tune->bn);
    IPC_REQUIRE(tune->splits >= 0 && tune->raster >= 0 && tune->max_ctas >= 0,
                "tune.splits / raster / max_ctas must be >= 0");
    IPC_REQUIRE(tune->pair >= 0 && tune->pair <= 2, "tune.pair must be 0, 1 or 2 (got %d)", tune->pair);
    t.pair = tune->pair;
    t.bn = tune->bn;
    t.splits = tune->splits;
    t.raster = tune->raster;
    t.max_ctas = tune->max_ctas;
  }
  return fused_gemm_impl(mode, a, b, out, aux, aux2, M, K, B, groups, scale, flags, act, dtype, algo,
                         static_cast<float*>(workspace), workspace_bytes, stream, tune ? &t : nullptr);
}

int ipc_fused_gemm_ws_bytes(int mode, int M, int K, int B, int groups, int flags, int dtype, int algo,
                            size_t* bytes) {
  int rc = common_checks(M, K, B, groups, IPC_ACT_IDENTITY, dtype, algo);
  if (rc) return rc;
  IPC_REQUIRE(mode >= MODE_P && mode <= MODE_F, "unknown mode %d", mode);
  IPC_REQUIRE(bytes != nullptr, "null result pointer");
  const bool weight = (mode == MODE_W || mode == MODE_WD);
  const bool bact = (flags & IPC_FLAG_ACTIVATE_B) != 0 && mode != MODE_I;
  size_t need = 0;
  if (!weight || algo == IPC_ALGO_OUTER || (algo == IPC_ALGO_AUTO && B <= 16)) {
    if (bact && !weight && tc_eligible(mode, M, K, B, dtype, algo, false, false))
      need = activation_ws_bytes(groups, K, B);
  } else if (tc_eligible(mode, M, K, B, dtype, algo, false, true)) {
    need = (bact ? activation_ws_bytes(groups, K, B) : 0) + IPC_SPLITK_WS_BYTES;
  }
  *bytes = need;
  return IPC_OK;
}

int ipc_fused_gemm_ws(int mode, const void* a, const void* b, void* out, const void* aux, void* aux2, int M, int K,
                      int B, int groups, float scale, int flags, int act, int dtype, int algo, void* workspace,
                      size_t workspace_bytes, void* stream) {
  IPC_REQUIRE(workspace != nullptr || workspace_bytes == 0, "workspace_bytes > 0 with a null workspace");
  IPC_REQUIRE(reinterpret_cast<uintptr_t>(workspace) % 16 == 0, "workspace must be 16-byte aligned");
  return fused_gemm_impl(mode, a, b, out, aux, aux2, M, K, B, groups, scale, flags, act, dtype, algo,
                         static_cast<float*>(workspace), workspace_bytes, stream);
}

int ipc_set_max_ctas(int max_ctas) { return set_max_ctas(max_ctas); }

int ipc_selftest_barrier_timeout(void* sync, int limit_us, void* stream) {
  int rc = require_sm100();
  if (rc) return rc;
  return wide_selftest_timeout(sync, limit_us, reinterpret_cast<cudaStream_t>(stream));
}

int ipc_device_status(int* status, int clear) {
  int rc = require_sm100();
  if (rc) return rc;
  int tc = 0, wide = 0, net = 0;
  rc = read_device_status(&tc, clear);
  if (rc) return rc;
  rc = read_wide_status(&wide, clear);
  if (rc) return rc;
  rc = read_net_status(&net, clear);
  if (rc) return rc;
  if (status) *status = tc != 0 ? tc : (wide != 0 ? wide : net);
  return IPC_OK;
}

}  // extern "C"
