// Shared device helpers: activations, storage types, error plumbing.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/ipc_b200.h"

namespace ipc {

// ---------------------------------------------------------------------------
// Activations.  f and f' follow src/ipc_tilelang/activations.py:9-29 and the
// in-kernel forms of src/ipc_tilelang/tilelang_kernels.py:61-96; they are
// always evaluated in fp32 (the reference kernels evaluate f' on the fp32 up-
// cast of the stored x, tilelang_kernels.py:227-229).  tanh/exp are CUDA's
// own tanhf/expf.
// ---------------------------------------------------------------------------
constexpr float kGeluC = 0.044715f;
constexpr float kGeluK = 0.7978845608028654f;

template <int ACT>
__device__ __forceinline__ float act_f(float x) {
  if constexpr (ACT == IPC_ACT_RELU) {
    return x > 0.f ? x : 0.f;
  } else if constexpr (ACT == IPC_ACT_TANH) {
    return tanhf(x);
  } else if constexpr (ACT == IPC_ACT_SIGMOID) {
    return 1.f / (1.f + expf(-x));
  } else if constexpr (ACT == IPC_ACT_SILU) {
    return x / (1.f + expf(-x));
  } else if constexpr (ACT == IPC_ACT_GELU) {
    float u = kGeluK * (x + kGeluC * x * x * x);
    return 0.5f * x * (1.f + tanhf(u));
  } else {
    return x;
  }
}

template <int ACT>
__device__ __forceinline__ float act_df(float x) {
  if constexpr (ACT == IPC_ACT_RELU) {
    return x > 0.f ? 1.f : 0.f;
  } else if constexpr (ACT == IPC_ACT_TANH) {
    float y = tanhf(x);
    return 1.f - y * y;
  } else if constexpr (ACT == IPC_ACT_SIGMOID) {
    float y = 1.f / (1.f + expf(-x));
    return y * (1.f - y);
  } else if constexpr (ACT == IPC_ACT_SILU) {
    float s = 1.f / (1.f + expf(-x));
    return s * (1.f + x * (1.f - s));
  } else if constexpr (ACT == IPC_ACT_GELU) {
    float u = kGeluK * (x + kGeluC * x * x * x);
    float t = tanhf(u);
    float du = kGeluK * (1.f + 3.f * kGeluC * x * x);
    return 0.5f * (1.f + t) + 0.5f * x * (1.f - t * t) * du;
  } else {
    return 1.f;
  }
}

// ---------------------------------------------------------------------------
// Hardware-approximate activations for 16-bit storage.  tanh.approx.f32 and
// ex2.approx.f32 are single MUFU instructions with a relative error near
// 2^-11, the size of one fp16 rounding step, so on the 16-bit path they move
// results by about one storage ulp.  The fp32 path always uses the accurate
// forms above.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float tanh_hw(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float sigmoid_hw(float x) {
  // 1 / (1 + 2^(-x log2 e)), exponent and reciprocal on the MUFU unit
  float t, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(t) : "f"(-1.4426950408889634f * x));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.f + t));
  return r;
}

template <int ACT>
__device__ __forceinline__ float act_f_hw(float x) {
  if constexpr (ACT == IPC_ACT_TANH) {
    return tanh_hw(x);
  } else if constexpr (ACT == IPC_ACT_SIGMOID) {
    return sigmoid_hw(x);
  } else if constexpr (ACT == IPC_ACT_SILU) {
    return x * sigmoid_hw(x);
  } else if constexpr (ACT == IPC_ACT_GELU) {
    return 0.5f * x * (1.f + tanh_hw(kGeluK * (x + kGeluC * x * x * x)));
  } else {
    return act_f<ACT>(x);
  }
}

template <int ACT>
__device__ __forceinline__ float act_df_hw(float x) {
  if constexpr (ACT == IPC_ACT_TANH) {
    const float y = tanh_hw(x);
    return 1.f - y * y;
  } else if constexpr (ACT == IPC_ACT_SIGMOID) {
    const float y = sigmoid_hw(x);
    return y * (1.f - y);
  } else if constexpr (ACT == IPC_ACT_SILU) {
    const float s = sigmoid_hw(x);
    return s * (1.f + x * (1.f - s));
  } else if constexpr (ACT == IPC_ACT_GELU) {
    const float t = tanh_hw(kGeluK * (x + kGeluC * x * x * x));
    return 0.5f * (1.f + t) + 0.5f * x * (1.f - t * t) * kGeluK * (1.f + 3.f * kGeluC * x * x);
  } else {
    return act_df<ACT>(x);
  }
}

// ---------------------------------------------------------------------------
// Storage types.
// ---------------------------------------------------------------------------
template <typename T>
struct St;
template <>
struct St<float> {
  static __device__ __forceinline__ float ld(float v) { return v; }
  static __device__ __forceinline__ float st(float v) { return v; }
  static constexpr int code = IPC_DT_F32;
};
template <>
struct St<__half> {
  static __device__ __forceinline__ float ld(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half st(float v) { return __float2half_rn(v); }
  static constexpr int code = IPC_DT_F16;
};
template <>
struct St<__nv_bfloat16> {
  static __device__ __forceinline__ float ld(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 st(float v) { return __float2bfloat16_rn(v); }
  static constexpr int code = IPC_DT_BF16;
};

// Round an fp32 value through the storage type (the reference's T.cast).
template <typename T>
__device__ __forceinline__ float rnd(float v) {
  return St<T>::ld(St<T>::st(v));
}

// ---------------------------------------------------------------------------
// Host-side error plumbing (defined in ipc_abi.cu).
// ---------------------------------------------------------------------------
int set_error(int code, const char* fmt, ...);
int check_launch(const char* what);
void count_launch(unsigned long long n = 1);
int require_sm100();

// Dispatch helpers: turn runtime act / dtype codes into template arguments.
#define IPC_DISPATCH_ACT(act, ACTC, ...)                                   \
  switch (act) {                                                            \
    case IPC_ACT_RELU: { constexpr int ACTC = IPC_ACT_RELU; __VA_ARGS__; break; }       \
    case IPC_ACT_TANH: { constexpr int ACTC = IPC_ACT_TANH; __VA_ARGS__; break; }       \
    case IPC_ACT_SIGMOID: { constexpr int ACTC = IPC_ACT_SIGMOID; __VA_ARGS__; break; } \
    case IPC_ACT_SILU: { constexpr int ACTC = IPC_ACT_SILU; __VA_ARGS__; break; }       \
    case IPC_ACT_GELU: { constexpr int ACTC = IPC_ACT_GELU; __VA_ARGS__; break; }       \
    case IPC_ACT_IDENTITY: { constexpr int ACTC = IPC_ACT_IDENTITY; __VA_ARGS__; break; } \
    default: return set_error(IPC_ERR_ARG, "unknown activation code %d", act);        \
  }

#define IPC_DISPATCH_DT(dtype, TT, ...)                                    \
  switch (dtype) {                                                          \
    case IPC_DT_F32: { using TT = float; __VA_ARGS__; break; }              \
    case IPC_DT_F16: { using TT = __half; __VA_ARGS__; break; }             \
    case IPC_DT_BF16: { using TT = __nv_bfloat16; __VA_ARGS__; break; }     \
    default: return set_error(IPC_ERR_ARG, "unknown dtype code %d", dtype); \
  }

#define IPC_DISPATCH_DT16(dtype, TT, ...)                                   \
  switch (dtype) {                                                           \
    case IPC_DT_F16: { using TT = __half; __VA_ARGS__; break; }              \
    case IPC_DT_BF16: { using TT = __nv_bfloat16; __VA_ARGS__; break; }      \
    default: return set_error(IPC_ERR_UNSUPPORTED, "dtype code %d: this kernel needs 16-bit storage", dtype); \
  }

inline size_t dt_size(int dtype) { return dtype == IPC_DT_F32 ? 4 : 2; }

// cudaFuncSetAttribute for a kernel's dynamic shared memory (and, with non_portable, the opt-in to
// clusters of more than 8 CTAs) once per kernel, device and size instead of on every launch: the
// attributes last as long as the device's context, and setting them costs microseconds of host time
// in front of launches that are themselves tens of microseconds long.  The record is per process; a
// context destroyed by cudaDeviceReset loses the attributes, and the next launch that needs them
// fails with a launch error.
template <auto KERN>
cudaError_t ensure_kernel_smem(int bytes, bool non_portable = false) {
  static int done[64][2] = {};  // per device: dynamic bytes set, non-portable set (benign races)
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = -1;
  if (dev >= 0 && done[dev][0] >= bytes && (!non_portable || done[dev][1])) return cudaSuccess;
  cudaError_t err = cudaFuncSetAttribute(KERN, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (err == cudaSuccess && non_portable)
    err = cudaFuncSetAttribute(KERN, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (err == cudaSuccess && dev >= 0) {
    if (done[dev][0] < bytes) done[dev][0] = bytes;
    if (non_portable) done[dev][1] = 1;
  }
  return err;
}

}  // namespace ipc
