// Per-element fused epilogues of the generic and small-batch GEMM kernels.
#pragma once
#include "ipc_common.cuh"
#include "ipc_generic.cuh"

namespace ipc {

// Epilogue of output element (m, n) of group g with fp32 accumulator `acc`
// (rounding points of tilelang_kernels.py:173, 229-231, 320).
template <typename T, int ACT, int MODE>
__device__ __forceinline__ void epilogue(const GemmArgs& p, int g, int m, int n, float acc) {
  const long long idx = (long long)m * p.Ng + n;
  if constexpr (MODE == MODE_P) {
    const T* xlo = reinterpret_cast<const T*>(p.aux) + g * p.gsAux;
    T* e = reinterpret_cast<T*>(p.out) + g * p.gsOut;
    e[idx] = St<T>::st(St<T>::ld(xlo[idx]) - rnd<T>(acc));
  } else if constexpr (MODE == MODE_I) {
    T* x = reinterpret_cast<T*>(p.out) + g * p.gsOut;
    const T* e = reinterpret_cast<const T*>(p.aux) + g * p.gsAux;
    const float xv = St<T>::ld(x[idx]);
    const float ev = St<T>::ld(e[idx]);
    const float xn = xv + p.scale * (-ev + act_df<ACT>(xv) * acc);
    x[idx] = St<T>::st(xn);
    if (p.aux2 != nullptr)
      reinterpret_cast<T*>(p.aux2)[g * p.gsAux2 + idx] = St<T>::st(act_f<ACT>(p.a_out_from_stored ? rnd<T>(xn) : xn));
  } else if constexpr (MODE == MODE_W) {
    T* w = reinterpret_cast<T*>(p.out) + g * p.gsOut;
    w[idx] = St<T>::st(St<T>::ld(w[idx]) + p.scale * acc);
  } else if constexpr (MODE == MODE_F) {
    T* o = reinterpret_cast<T*>(p.out) + g * p.gsOut;
    o[idx] = St<T>::st(acc);
    if (p.aux2 != nullptr) reinterpret_cast<T*>(p.aux2)[g * p.gsAux2 + idx] = St<T>::st(act_f<ACT>(rnd<T>(acc)));
  } else {
    float* dw = reinterpret_cast<float*>(p.out) + g * p.gsOut;
    const float v = p.scale * acc;
    dw[idx] = p.accumulate ? dw[idx] + v : v;
  }
}

}  // namespace ipc
