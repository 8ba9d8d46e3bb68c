// Small-batch outer-product weight update and element-wise helpers.
//
// ipc_weight_update(algo = IPC_ALGO_OUTER):  W[m, k] += alpha * sum_b E[m,b] A[k,b]
// For B <= 16 the update is bound by the read-modify-write of W in HBM
// (arithmetic intensity ~B/2 FLOP/B), so each thread owns 8 consecutive
// elements of one W row (one 16-byte vector), the CTA stages its E rows and
// the activated A rows in shared memory, and W is touched exactly once.
// Replaces SmallBWeightUpdater (src/ipc_tilelang/weight_update_specialization.py:90-104),
// which forms a [B, M, K] temporary with torch.bmm; the sign here is +alpha.
#include "ipc_common.cuh"
#include "ipc_elementwise.cuh"
#include "ipc_generic.cuh"

namespace ipc {
namespace {

constexpr int OT_ROWS = 8;          // W rows per CTA
constexpr int OT_COLS = 256;        // W cols per CTA (32 threads x 8)
constexpr int OT_BB = 16;           // batch chunk staged per pass
constexpr int OT_THREADS = OT_ROWS * (OT_COLS / 8);

template <typename T>
struct Vec8 {
  static __device__ __forceinline__ void load(const T* p, float (&v)[8]) {
    const uint4 raw = *reinterpret_cast<const uint4*>(p);
    const T* h = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = St<T>::ld(h[j]);
  }
  static __device__ __forceinline__ void store(T* p, const float (&v)[8]) {
    uint4 raw;
    T* h = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int j = 0; j < 8; ++j) h[j] = St<T>::st(v[j]);
    *reinterpret_cast<uint4*>(p) = raw;
  }
};

template <typename T, int ACT, bool BACT, bool DELTA>
__global__ void __launch_bounds__(OT_THREADS) outer_update_kernel(void* __restrict__ out, const T* __restrict__ E,
                                                                   const T* __restrict__ X, int M, int K, int B,
                                                                   float alpha, int accumulate, int vec_ok,
                                                                   const OptParams opt) {
  __shared__ float sE[OT_ROWS][OT_BB];
  __shared__ __align__(16) float sA[OT_BB][OT_COLS];
  const int g = blockIdx.z;
  E += (long long)g * M * B;
  X += (long long)g * K * B;
  const int tid = threadIdx.x;
  const int r = tid / (OT_COLS / 8);        // row within the tile
  const int c8 = (tid % (OT_COLS / 8)) * 8; // first col within the tile
  const int m = blockIdx.y * OT_ROWS + r;
  const int k0 = blockIdx.x * OT_COLS + c8;
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;

  for (int b0 = 0; b0 < B; b0 += OT_BB) {
    const int nb = min(OT_BB, B - b0);
    for (int it = tid; it < OT_ROWS * OT_BB; it += OT_THREADS) {
      const int rr = it / OT_BB, bb = it % OT_BB;
      const int mm = blockIdx.y * OT_ROWS + rr;
      sE[rr][bb] = (mm < M && bb < nb) ? St<T>::ld(E[(long long)mm * B + b0 + bb]) : 0.f;
    }
    for (int it = tid; it < OT_COLS * OT_BB; it += OT_THREADS) {
      const int kk = it / OT_BB, bb = it % OT_BB;  // consecutive threads: consecutive b
      const int k = blockIdx.x * OT_COLS + kk;
      float v = 0.f;
      if (k < K && bb < nb) {
        v = St<T>::ld(X[(long long)k * B + b0 + bb]);
        if (BACT) v = rnd<T>(act_f<ACT>(v));
      }
      sA[bb][kk] = v;
    }
    __syncthreads();
    for (int bb = 0; bb < nb; ++bb) {
      const float ev = sE[r][bb];
      const float4 a0 = *reinterpret_cast<const float4*>(&sA[bb][c8]);
      const float4 a1 = *reinterpret_cast<const float4*>(&sA[bb][c8 + 4]);
      acc[0] = fmaf(ev, a0.x, acc[0]);
      acc[1] = fmaf(ev, a0.y, acc[1]);
      acc[2] = fmaf(ev, a0.z, acc[2]);
      acc[3] = fmaf(ev, a0.w, acc[3]);
      acc[4] = fmaf(ev, a1.x, acc[4]);
      acc[5] = fmaf(ev, a1.y, acc[5]);
      acc[6] = fmaf(ev, a1.z, acc[6]);
      acc[7] = fmaf(ev, a1.w, acc[7]);
    }
    __syncthreads();
  }
  if (m >= M) return;
  if constexpr (DELTA) {
    float* dw = reinterpret_cast<float*>(out) + (long long)g * M * K + (long long)m * K;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int k = k0 + j;
      if (k < K) dw[k] = (accumulate ? dw[k] : 0.f) + alpha * acc[j];
    }
  } else if (opt.kind != 0) {  // optimizer step: g = -acc, state at W's index
    T* w = reinterpret_cast<T*>(out) + (long long)g * M * K + (long long)m * K;
    const long long base = (long long)g * M * K + (long long)m * K;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int k = k0 + j;
      if (k < K) w[k] = St<T>::st(opt_step(opt, St<T>::ld(w[k]), -acc[j], base + k));
    }
  } else {
    T* w = reinterpret_cast<T*>(out) + (long long)g * M * K + (long long)m * K;
    if (vec_ok && k0 + 8 <= K && sizeof(T) == 2) {
      float v[8];
      Vec8<T>::load(w + k0, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] += alpha * acc[j];
      Vec8<T>::store(w + k0, v);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int k = k0 + j;
        if (k < K) w[k] = St<T>::st(St<T>::ld(w[k]) + alpha * acc[j]);
      }
    }
  }
}

template <typename T, int ACT>
__global__ void activate_kernel(T* __restrict__ a, const T* __restrict__ x, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    a[i] = St<T>::st(act_f<ACT>(St<T>::ld(x[i])));
}

// 16-bit storage, both pointers 16-byte aligned: 8 elements per 16-byte access, two accesses in flight per
// thread, f in its MUFU form (the form the tensor-core epilogues use; the result is rounded to 16 bits).
// HBM-bound: 4 bytes of traffic per element.
template <typename T, int ACT>
__global__ void __launch_bounds__(256) activate16_kernel(T* __restrict__ a, const T* __restrict__ x, long long n) {
  const long long n8 = n / 8;
  const uint4* src = reinterpret_cast<const uint4*>(x);
  uint4* dst = reinterpret_cast<uint4*>(a);
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8; i += 2 * stride) {
    const bool two = i + stride < n8;
    uint4 v0 = src[i], v1 = two ? src[i + stride] : make_uint4(0, 0, 0, 0);
    T* h0 = reinterpret_cast<T*>(&v0);
    T* h1 = reinterpret_cast<T*>(&v1);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      h0[j] = St<T>::st(act_f_hw<ACT>(St<T>::ld(h0[j])));
      h1[j] = St<T>::st(act_f_hw<ACT>(St<T>::ld(h1[j])));
    }
    dst[i] = v0;
    if (two) dst[i + stride] = v1;
  }
  for (long long i = n8 * 8 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride)
    a[i] = St<T>::st(act_f_hw<ACT>(St<T>::ld(x[i])));
}

// Optimizer step from an fp32 product already in memory: g = -dw (the workspace path of shapes the fused
// kernels do not serve).
template <typename T>
__global__ void opt_apply_kernel(T* __restrict__ w, const float* __restrict__ dw, long long n, const OptParams opt) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    w[i] = St<T>::st(opt_step(opt, St<T>::ld(w[i]), -dw[i], i));
}

template <typename T>
__global__ void apply_kernel(T* __restrict__ w, const float* __restrict__ dw, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    w[i] = St<T>::st(St<T>::ld(w[i]) + dw[i]);
}

int grid_1d(long long n) {
  long long b = (n + 255) / 256;
  if (b > 148LL * 32) b = 148LL * 32;
  return (int)(b < 1 ? 1 : b);
}

}  // namespace

int launch_outer(void* out, const void* e, const void* x, int M, int K, int B, int groups, float alpha,
                 bool bact, bool delta, int accumulate, int act, int dtype, cudaStream_t s, const OptParams* opt) {
  const OptParams o = opt != nullptr ? *opt : OptParams{};
  if (M <= 0 || K <= 0 || groups <= 0) return IPC_OK;
  if (B <= 0 && !delta) return IPC_OK;  // W + alpha * (empty sum) = W; a delta still writes its zeros
  dim3 grid((K + OT_COLS - 1) / OT_COLS, (M + OT_ROWS - 1) / OT_ROWS, groups);
  if (grid.y > 65535u || grid.z > 65535u) return set_error(IPC_ERR_ARG, "outer update grid too large");
  const int vec_ok = (K % 8 == 0) && ((reinterpret_cast<uintptr_t>(out) & 15) == 0);
  IPC_DISPATCH_DT(dtype, TT, {
    const TT* E = reinterpret_cast<const TT*>(e);
    const TT* X = reinterpret_cast<const TT*>(x);
    if (!bact) {
      if (delta)
        outer_update_kernel<TT, IPC_ACT_IDENTITY, false, true><<<grid, OT_THREADS, 0, s>>>(out, E, X, M, K, B, alpha, accumulate, vec_ok, o);
      else
        outer_update_kernel<TT, IPC_ACT_IDENTITY, false, false><<<grid, OT_THREADS, 0, s>>>(out, E, X, M, K, B, alpha, accumulate, vec_ok, o);
    } else {
      IPC_DISPATCH_ACT(act, AC, {
        if (delta)
          outer_update_kernel<TT, AC, true, true><<<grid, OT_THREADS, 0, s>>>(out, E, X, M, K, B, alpha, accumulate, vec_ok, o);
        else
          outer_update_kernel<TT, AC, true, false><<<grid, OT_THREADS, 0, s>>>(out, E, X, M, K, B, alpha, accumulate, vec_ok, o);
      });
    }
  });
  count_launch();
  return check_launch("outer-product weight update");
}

int launch_activate(void* a, const void* x, long long n, int act, int dtype, cudaStream_t s) {
  if (n <= 0) return IPC_OK;
  const bool vec = dtype != IPC_DT_F32 &&
                   ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(x)) & 15) == 0;
  IPC_DISPATCH_DT(dtype, TT, {
    IPC_DISPATCH_ACT(act, AC, {
      if constexpr (sizeof(TT) == 2) {
        if (vec) {
          activate16_kernel<TT, AC><<<148 * 8, 256, 0, s>>>(reinterpret_cast<TT*>(a), reinterpret_cast<const TT*>(x),
                                                            n);
          break;
        }
      }
      activate_kernel<TT, AC><<<grid_1d(n), 256, 0, s>>>(reinterpret_cast<TT*>(a), reinterpret_cast<const TT*>(x), n);
    });
  });
  count_launch();
  return check_launch("activate");
}

int launch_opt_apply(void* w, const float* dw, long long n, int dtype, const OptParams& opt, cudaStream_t s) {
  if (n <= 0) return IPC_OK;
  IPC_DISPATCH_DT(dtype, TT, {
    opt_apply_kernel<TT><<<grid_1d(n), 256, 0, s>>>(reinterpret_cast<TT*>(w), dw, n, opt);
  });
  count_launch();
  return check_launch("optimizer step");
}

int launch_apply(void* w, const float* dw, long long n, int dtype, cudaStream_t s) {
  if (n <= 0) return IPC_OK;
  IPC_DISPATCH_DT(dtype, TT, {
    apply_kernel<TT><<<grid_1d(n), 256, 0, s>>>(reinterpret_cast<TT*>(w), dw, n);
  });
  count_launch();
  return check_launch("weight apply");
}

}  // namespace ipc

namespace ipc {
namespace {

// Correct predictions of one batch: per column b, the row of the largest logit (the first on ties, as
// torch.argmax) against labels[b]; one thread per column (rows are B apart, so a warp's loads of one
// row are contiguous), a block-wide count, one atomic per block.
template <typename T>
__global__ void __launch_bounds__(256) count_correct_kernel(const T* __restrict__ logits, int C, int B,
                                                            const long long* __restrict__ labels, int* count) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  int hit = 0;
  if (b < B) {
    int best = 0;
    float bv = St<T>::ld(logits[b]);
    for (int c = 1; c < C; ++c) {
      const float v = St<T>::ld(logits[(long long)c * B + b]);
      if (v > bv) { bv = v; best = c; }
    }
    hit = (long long)best == labels[b];
  }
  const int n = __syncthreads_count(hit);
  if (threadIdx.x == 0 && n) atomicAdd(count, n);
}

}  // namespace

int launch_count_correct(const void* logits, int C, int B, const long long* labels, int* count, int dtype,
                         cudaStream_t s) {
  if (B <= 0) return IPC_OK;
  IPC_DISPATCH_DT(dtype, TT, {
    count_correct_kernel<TT><<<(B + 255) / 256, 256, 0, s>>>(reinterpret_cast<const TT*>(logits), C, B, labels,
                                                             count);
  });
  count_launch();
  return check_launch("count correct");
}

}  // namespace ipc
