// Generic fused P / I / W kernels for any shape (tails, tiny M = 10, B = 1).
//
//   fp32 storage : CUDA-core FMA tiles (the exact-mode path, 1e-5 parity).
//   16-bit       : mma.sync m16n8k16 tiles with fp32 accumulators.
//
// Each kernel is one tiled GEMM  C[m,n] = sum_k A(m,k) B(k,n)  with the
// operand orientation and the epilogue chosen by MODE:
//   P  (tilelang_kernels.py:114-177)  A = W[M,K]        B = f(X_up)[K,B]      E = cast(X_lo) - cast(C)
//   I  (tilelang_kernels.py:180-265)  A = W_low^T       B = E_low[K,B]        X += g(-E + f'(X) C) [, A_out]
//   W  (tilelang_kernels.py:268-349)  A = E[M,B]        B = f(X_up)^T          W = cast(W + a C)
//   WD (no reference counterpart)     as W, but dw (+)= a C in fp32
//   F  (trainer.py:512-515, 828-833)  as P                                   OUT = cast(C) [, A_out = f(OUT)]
// Padding of the activated operand stays zero (tilelang_kernels.py:165-167).
#include <cstdio>

#include "ipc_common.cuh"
#include "ipc_generic.cuh"
#include "ipc_epilogue.cuh"

namespace ipc {

namespace {

constexpr int BM = 64, BN = 64, BK = 32, NTHREADS = 128;

// Operand orientation per mode.
template <int MODE>
struct Orient {
  static constexpr bool a_kcontig = (MODE != MODE_I);  // I reads W_low [K,M]: m contiguous
  static constexpr bool b_ncontig = (MODE == MODE_P || MODE == MODE_I || MODE == MODE_F);
};

// Load element A(m,k) / B(k,n) of the current group (zero outside the matrix).
template <typename T, int MODE>
__device__ __forceinline__ float load_a(const GemmArgs& p, const T* A, int m, int k) {
  if (m >= p.Mg || k >= p.Kg) return 0.f;
  const long long off = Orient<MODE>::a_kcontig ? (long long)m * p.lda + k : (long long)k * p.lda + m;
  return St<T>::ld(A[off]);
}
template <typename T, int ACT, int MODE, bool BACT>
__device__ __forceinline__ float load_b(const GemmArgs& p, const T* Bm, int k, int n) {
  if (k >= p.Kg || n >= p.Ng) return 0.f;
  const long long off = Orient<MODE>::b_ncontig ? (long long)k * p.ldb + n : (long long)n * p.ldb + k;
  const float v = St<T>::ld(Bm[off]);
  return BACT ? rnd<T>(act_f<ACT>(v)) : v;
}

// ------------------------------- fp32 SIMT ---------------------------------
template <int ACT, int MODE, bool BACT>
__global__ void __launch_bounds__(NTHREADS) gemm_simt_kernel(GemmArgs p) {
  __shared__ float sA[BK][BM + 4];
  __shared__ float sB[BK][BN + 4];
  const int g = blockIdx.z;
  const float* A = reinterpret_cast<const float*>(p.A) + g * p.gsA;
  const float* Bm = reinterpret_cast<const float*>(p.Bm) + g * p.gsB;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int tid = threadIdx.x;
  const int tn = tid % 8, tm = tid / 8;  // 8 x 16 threads, 8 n x 4 m each
  float acc[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  for (int k0 = 0; k0 < p.Kg; k0 += BK) {
    // A tile: BM x BK elements, coalesced along the contiguous global dim.
#pragma unroll 4
    for (int it = tid; it < BM * BK; it += NTHREADS) {
      int m, k;
      if (Orient<MODE>::a_kcontig) { k = it % BK; m = it / BK; } else { m = it % BM; k = it / BM; }
      sA[k][m] = load_a<float, MODE>(p, A, m0 + m, k0 + k);
    }
#pragma unroll 4
    for (int it = tid; it < BN * BK; it += NTHREADS) {
      int n, k;
      if (Orient<MODE>::b_ncontig) { n = it % BN; k = it / BN; } else { k = it % BK; n = it / BK; }
      sB[k][n] = load_b<float, ACT, MODE, BACT>(p, Bm, k0 + k, n0 + n);
    }
    __syncthreads();
#pragma unroll 8
    for (int k = 0; k < BK; ++k) {
      float a[4], b[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = sA[k][tm * 4 + i];
#pragma unroll
      for (int j = 0; j < 8; ++j) b[j] = sB[k][tn * 8 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + tm * 4 + i;
    if (m >= p.Mg) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int n = n0 + tn * 8 + j;
      if (n < p.Ng) epilogue<float, ACT, MODE>(p, g, m, n, acc[i][j]);
    }
  }
}

// ----------------------------- 16-bit mma.sync ------------------------------
template <typename T>
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  if constexpr (std::is_same<T, __half>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  }
}

template <typename T, int ACT, int MODE, bool BACT>
__global__ void __launch_bounds__(NTHREADS) gemm_mma_kernel(GemmArgs p) {
  constexpr int LDS = BK + 8;  // 40 halves: conflict-free 32-bit fragment reads
  __shared__ __align__(16) T sA[BM][LDS];
  __shared__ __align__(16) T sB[BN][LDS];
  const int g = blockIdx.z;
  const T* A = reinterpret_cast<const T*>(p.A) + g * p.gsA;
  const T* Bm = reinterpret_cast<const T*>(p.Bm) + g * p.gsB;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int wm = warp >> 1, wn = warp & 1;
  const int gq = lane >> 2, tq = lane & 3;
  float acc[2][4][4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[i][j][r] = 0.f;

  for (int k0 = 0; k0 < p.Kg; k0 += BK) {
#pragma unroll 4
    for (int it = tid; it < BM * BK; it += NTHREADS) {
      int m, k;
      if (Orient<MODE>::a_kcontig) { k = it % BK; m = it / BK; } else { m = it % BM; k = it / BM; }
      sA[m][k] = St<T>::st(load_a<T, MODE>(p, A, m0 + m, k0 + k));
    }
#pragma unroll 4
    for (int it = tid; it < BN * BK; it += NTHREADS) {
      int n, k;
      if (Orient<MODE>::b_ncontig) { n = it % BN; k = it / BN; } else { k = it % BK; n = it / BK; }
      sB[n][k] = St<T>::st(load_b<T, ACT, MODE, BACT>(p, Bm, k0 + k, n0 + n));
    }
    __syncthreads();
#pragma unroll
    for (int ks = 0; ks < BK; ks += 16) {
      uint32_t a[2][4], b[4][2];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const int r = wm * 32 + mt * 16 + gq;
        a[mt][0] = *reinterpret_cast<const uint32_t*>(&sA[r][ks + 2 * tq]);
        a[mt][1] = *reinterpret_cast<const uint32_t*>(&sA[r + 8][ks + 2 * tq]);
        a[mt][2] = *reinterpret_cast<const uint32_t*>(&sA[r][ks + 2 * tq + 8]);
        a[mt][3] = *reinterpret_cast<const uint32_t*>(&sA[r + 8][ks + 2 * tq + 8]);
      }
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int c = wn * 32 + nt * 8 + gq;
        b[nt][0] = *reinterpret_cast<const uint32_t*>(&sB[c][ks + 2 * tq]);
        b[nt][1] = *reinterpret_cast<const uint32_t*>(&sB[c][ks + 2 * tq + 8]);
      }
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) mma16816<T>(acc[mt][nt], a[mt], b[nt]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int m = m0 + wm * 32 + mt * 16 + gq + (r >= 2 ? 8 : 0);
        const int n = n0 + wn * 32 + nt * 8 + 2 * tq + (r & 1);
        if (m < p.Mg && n < p.Ng) epilogue<T, ACT, MODE>(p, g, m, n, acc[mt][nt][r]);
      }
}

template <typename T, int ACT, int MODE, bool BACT>
int launch_one(const GemmArgs& p, cudaStream_t s) {
  dim3 grid((p.Ng + BN - 1) / BN, (p.Mg + BM - 1) / BM, p.groups);
  if (grid.y > 65535u || grid.z > 65535u)
    return set_error(IPC_ERR_ARG, "generic GEMM grid too large (M=%d groups=%d)", p.Mg, p.groups);
  if constexpr (std::is_same<T, float>::value) {
    gemm_simt_kernel<ACT, MODE, BACT><<<grid, NTHREADS, 0, s>>>(p);
  } else {
    gemm_mma_kernel<T, ACT, MODE, BACT><<<grid, NTHREADS, 0, s>>>(p);
  }
  count_launch();
  return check_launch("generic GEMM");
}

}  // namespace

int launch_generic(const GemmArgs& p, int mode, bool bact, int act, int dtype, cudaStream_t s) {
  if (p.Mg <= 0 || p.Ng <= 0 || p.groups <= 0) return IPC_OK;  // empty output: nothing to do
  IPC_DISPATCH_DT(dtype, TT, {
    if (!bact && mode != MODE_I && !(mode == MODE_F && p.aux2 != nullptr)) {
      // the activation only enters through the B operand -> one instantiation
      switch (mode) {
        case MODE_P: return launch_one<TT, IPC_ACT_IDENTITY, MODE_P, false>(p, s);
        case MODE_W: return launch_one<TT, IPC_ACT_IDENTITY, MODE_W, false>(p, s);
        case MODE_WD: return launch_one<TT, IPC_ACT_IDENTITY, MODE_WD, false>(p, s);
        case MODE_F: return launch_one<TT, IPC_ACT_IDENTITY, MODE_F, false>(p, s);
        default: break;
      }
    }
    IPC_DISPATCH_ACT(act, AC, {
      switch (mode) {
        case MODE_P: return launch_one<TT, AC, MODE_P, true>(p, s);
        case MODE_I: return launch_one<TT, AC, MODE_I, false>(p, s);
        case MODE_W: return launch_one<TT, AC, MODE_W, true>(p, s);
        case MODE_WD: return launch_one<TT, AC, MODE_WD, true>(p, s);
        case MODE_F:
          return bact ? launch_one<TT, AC, MODE_F, true>(p, s) : launch_one<TT, AC, MODE_F, false>(p, s);
        default: return set_error(IPC_ERR_ARG, "bad GEMM mode %d", mode);
      }
    });
  });
  return IPC_OK;
}

}  // namespace ipc
