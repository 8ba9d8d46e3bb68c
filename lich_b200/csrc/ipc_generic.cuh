// Argument block of the fused GEMM kernels (generic and tensor-core).
#pragma once
#include <cuda_runtime.h>

#include "../../include/ipc_b200.h"

namespace ipc {

enum GemmMode { MODE_P = 0, MODE_I = 1, MODE_W = 2, MODE_WD = 3, MODE_F = 4, MODE_WO = 5 };

// Optimizer step applied where a weight update meets W (MODE_WO and the small-batch / split-K paths), so no
// gradient tensor is written to memory.  The gradient of the energy sum_l |e_l|^2 / 2 with respect to W[l]
// is g = -E A^T (summed over the batch); kind IPC_OPT_SGD with momentum 0 and weight decay 0 is therefore
// the plain iPC update W += lr E A^T.  SGD follows torch.optim.SGD (dampening 0, no Nesterov; the
// momentum buffer starts at zero), AdamW torch.optim.AdamW (decoupled decay, bias-corrected moments).
struct OptParams {
  int kind;                  // 0: none, IPC_OPT_SGD, IPC_OPT_ADAMW
  float lr, momentum, wd;    // SGD: momentum; both: weight decay
  float b1, b2, eps;         // AdamW
  float step_size, rsqrt_bc2;  // AdamW: lr / (1 - b1^t), 1 / sqrt(1 - b2^t)
  float* m;                  // SGD momentum buffer / AdamW first moment (fp32, the layout of W); may be null for
  float* v;                  //   SGD without momentum; AdamW second moment
};

// One element: w (fp32 value of the stored weight), g its gradient, i its index into m / v.
__device__ __forceinline__ float opt_step(const OptParams& o, float w, float g, long long i) {
  if (o.kind == IPC_OPT_ADAMW) {
    w *= 1.f - o.lr * o.wd;
    const float m = o.b1 * o.m[i] + (1.f - o.b1) * g;
    const float v = o.b2 * o.v[i] + (1.f - o.b2) * g * g;
    o.m[i] = m;
    o.v[i] = v;
    return w - o.step_size * m / (sqrtf(v) * o.rsqrt_bc2 + o.eps);
  }
  g += o.wd * w;  // SGD
  if (o.m != nullptr) {
    const float b = o.momentum * o.m[i] + g;
    o.m[i] = b;
    g = b;
  }
  return w - o.lr * g;
}

// C[m,n] = sum_k A(m,k) B(k,n) per group, then a MODE epilogue on the
// row-major [Mg, Ng] output.  Orientation (fixed by MODE):
//   P, F : A(m,k) = A[m*lda + k]   B(k,n) = B[k*ldb + n]   (Mg,Ng,Kg) = (M,B,K)
//   I : A(m,k) = A[k*lda + m]   B(k,n) = B[k*ldb + n]   (Mg,Ng,Kg) = (M,B,K)
//   W : A(m,k) = A[m*lda + k]   B(k,n) = B[n*ldb + k]   (Mg,Ng,Kg) = (M,K,B)
struct GemmArgs {
  const void* A;
  long long lda, gsA;
  const void* Bm;
  long long ldb, gsB;
  int Mg, Ng, Kg, groups;
  void* out;        // P: E   I: X   W: W   WD: dw (fp32)   F: out
  long long gsOut;
  const void* aux;  // P: X_lo   I: E
  long long gsAux;
  void* aux2;       // I: A_out (may be null)
  long long gsAux2;
  float scale;      // I: gamma   W/WD: alpha
  int accumulate;   // WD
  int a_out_from_stored;  // I: A_out = f(cast(x_new)) (what recompute mode reads back) instead of f(x_new)
  OptParams opt;    // WO: the optimizer step applied to W
  int mcast;        // WD: out is a multicast (NVLS) address, the epilogue adds with multimem.red
};

int launch_generic(const GemmArgs& p, int mode, bool bact, int act, int dtype, cudaStream_t s);

// Small-batch path of P / I / F (N = B <= 16, 16-bit storage, IPC_ALGO_AUTO): a cluster of CTAs per
// 16 output rows splits K and reduces over distributed shared memory (ipc_skinny.cu).
bool skinny_eligible(int mode, int M, int K, int B, int dtype, int algo);
int launch_skinny(const GemmArgs& p, int mode, bool bact, int act, int dtype, cudaStream_t s);

}  // namespace ipc
