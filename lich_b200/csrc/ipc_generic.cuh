// Argument block of the fused GEMM kernels (generic and tensor-core).
#pragma once
#include <cuda_runtime.h>

namespace ipc {

enum GemmMode { MODE_P = 0, MODE_I = 1, MODE_W = 2, MODE_WD = 3, MODE_F = 4 };

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
};

int launch_generic(const GemmArgs& p, int mode, bool bact, int act, int dtype, cudaStream_t s);

// Small-batch path of P / I / F (N = B <= 16, 16-bit storage, IPC_ALGO_AUTO): a cluster of CTAs per
// 16 output rows splits K and reduces over distributed shared memory (ipc_skinny.cu).
bool skinny_eligible(int mode, int M, int K, int B, int dtype, int algo);
int launch_skinny(const GemmArgs& p, int mode, bool bact, int act, int dtype, cudaStream_t s);

}  // namespace ipc
