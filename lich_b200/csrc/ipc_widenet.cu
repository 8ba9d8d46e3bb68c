// Persistent training-step kernel for wide networks at small batch (B <= 16,
// widths up to 4096): the small-batch regime of the reference's weight-update
// specialisation (weight_update_specialization.py:63-128) run as whole steps.
//
// At B <= 16 every GEMM of a step is a read of one W (a few MB, resident in
// the 126 MB L2 for the whole launch) against a thin operand of a few KB, so
// the 3L-1 separate launches of the operator path (trainer.py:601-679) spend
// almost all their time in launch and memory latency.  Here one cooperative
// launch (one CTA per SM, 512 threads) runs `steps` training steps; the
// phases of a step are separated by grid barriers:
//   batch   x[L], x[0] <- pool (when a pool is given)
//   forward x[l] = cast(W[l] f(x[l+1])), l = L-1 .. 1   (one phase per layer)
//   T x     P: e[l] = cast(x[l]) - cast(W[l] f(x[l+1])) for all l   (one phase)
//           I: x[l] += g(-e[l] + f'(x[l]) W[l-1]^T e[l-1]) for l >= 1 (one phase)
//   W       W[l] = cast(W[l] + a e[l] f(x[l+1])^T) for all l          (one phase)
// A GEMM phase is a list of units (layer, 32 output rows).  A CTA stages the
// unit's thin operand (K x B, f applied or read from the activation cache) in
// shared memory as rows of 16 batch columns; its 16 warps cover 2 row tiles x 8
// K slices, load their W fragments straight from L2 (ld.global.cg: W and the
// states change between phases, and L1 is not coherent across SMs), take the
// B fragments with ldmatrix.trans and run mma.sync m16n8k16; the 8 K-slice
// partials are summed in shared memory in fixed order and the fused epilogue
// of the phase stores the result.  The weight phase runs dW tiles as mma.sync
// with the batch (B <= 16, zero-padded) as the reduction.
// Rounding points are those of the operator kernels: tilelang_kernels.py:163,
// 173, 229-230, 320 and the forward sweep trainer.py:513-515.
//
// Grid barrier: a launch-wide arrival counter in caller memory (ipc_net_run_t.sync,
// zeroed by the call), release reductions to arrive, acquire polls to wait.  Every wait is bounded (2 s of
// %globaltimer): on expiry the waiting CTA records IPC_ERR_TIMEOUT in this
// file's device status word, raises an abort flag that every other waiter
// also polls, and all CTAs return.
#include "ipc_common.cuh"

namespace ipc {

__device__ int g_wide_status = 0;

namespace {

constexpr int WN_THREADS = 512;
constexpr int WN_WARPS = WN_THREADS / 32;
constexpr int WN_ROWS = 32;     // output rows per unit: two m16 tiles
constexpr int WN_KSLICES = WN_WARPS / 2;
constexpr int WN_NC = 16;       // batch columns padded to two n8 tiles
constexpr int WN_MAX_DIM = 4096;
constexpr int WN_MAX_B = 16;
constexpr long long WN_WAIT_NS = 2000000000LL;

template <typename T>
struct WideParams {
  int L, B, kmax;
  int dims[IPC_NET_MAX_LAYERS + 1];
  T* w[IPC_NET_MAX_LAYERS];
  T* x[IPC_NET_MAX_LAYERS + 1];
  T* e[IPC_NET_MAX_LAYERS + 1];
  T* a[IPC_NET_MAX_LAYERS + 1];  // activation cache (all of a[1..L] set) or all null
  int acache;
  const T* pool_x;
  const T* pool_y;
  int pool_batches, first_batch, steps, T_it, forward_init, update_weights;
  float alpha, gamma;
  float* energy;
  unsigned* sync;  // [0] arrivals over the launch, [2] abort
  long long* phase_ns;  // [IPC_NET_TRACE_STEPS][IPC_NET_TRACE_PHASES] or null
  // resident weights (RES): this CTA's P unit's rows of W[l] ([32][res_kp + 8]) and its I unit's
  // columns of W[l-1] ([res_ki][WN_WI_LD]) stay in shared memory for the whole launch
  int res_kp, res_ki;
};

constexpr int WN_WI_LD = 40;  // row stride (elements) of the resident W[l-1] columns: 80 B, ldmatrix conflict-free

// Trace slots of the wide kernel (CTA 0 after the barrier closing each phase).
enum { WT_START = 0, WT_BATCH = 1, WT_FORWARD = 2, WT_P0 = 3, WT_I0 = 4, WT_ITER = 5, WT_W = 6 };

__device__ __forceinline__ long long wn_now() {
  long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

template <typename T>
__device__ __forceinline__ float ldcg(const T* p) {
  const unsigned short u = __ldcg(reinterpret_cast<const unsigned short*>(p));
  T v;
  *reinterpret_cast<unsigned short*>(&v) = u;
  return St<T>::ld(v);
}

__device__ __forceinline__ void wn_red_release_add(unsigned* addr, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned wn_ld_acquire(const unsigned* addr) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

// Grid-wide barrier: sync[0] counts arrivals over the whole launch (zeroed by the host before it);
// barrier number `epoch` (1, 2, ...) is complete when it reaches epoch * gridDim.x.  Thread 0 of
// each CTA arrives with a release reduction (its CTA's writes, ordered before it by __syncthreads,
// become visible with it) and polls with acquire loads; the wait is bounded by limit_ns, after
// which the CTA records IPC_ERR_TIMEOUT and raises the abort word sync[2] that every poller also
// watches.  Returns false when the launch is being abandoned.
__device__ __forceinline__ bool wn_grid_sync(unsigned* sync, unsigned& epoch, long long limit_ns = WN_WAIT_NS) {
  __shared__ int ok_s;
  __syncthreads();
  ++epoch;
  if (threadIdx.x == 0) {
    int ok = 1;
    const unsigned target = epoch * gridDim.x;
    wn_red_release_add(sync, 1u);
    if (wn_ld_acquire(sync) < target) {
      const long long t0 = wn_now();
      while (wn_ld_acquire(sync) < target) {
        if (wn_ld_acquire(sync + 2) != 0u) { ok = 0; break; }
        if (wn_now() - t0 > limit_ns) {
          atomicCAS(&g_wide_status, 0, IPC_ERR_TIMEOUT);
          atomicExch(sync + 2, 1u);
          ok = 0;
          break;
        }
      }
    }
    ok_s = ok;
  }
  __syncthreads();
  return ok_s != 0;
}

template <typename T>
__device__ __forceinline__ void wn_mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __half>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

enum { WN_F = 0, WN_P = 1, WN_I = 2 };

// A pair (A(m,k), A(m,k+1)) of the phase's weight operand, packed; zero outside.
//   F / P: A(m,k) = W[l][m][k]  (M = d_l, K = d_{l+1})
//   I    : A(m,k) = W[l-1][k][m] (M = d_l, K = d_{l-1})
template <int MODE>
__device__ __forceinline__ uint32_t wn_load_a(const unsigned short* A, int M, int K, int m, int k) {
  if (m >= M || k >= K) return 0u;
  if constexpr (MODE == WN_I) {
    const uint32_t lo = __ldcg(A + k * M + m);
    const uint32_t hi = (k + 1 < K) ? __ldcg(A + (k + 1) * M + m) : 0u;
    return lo | (hi << 16);
  } else {
    const int off = m * K + k;  // W has at most 4096 x 4096 elements
    if ((K & 1) == 0 && k + 1 < K) return __ldcg(reinterpret_cast<const unsigned int*>(A + off));
    const uint32_t lo = __ldcg(A + off);
    const uint32_t hi = (k + 1 < K) ? __ldcg(A + off + 1) : 0u;
    return lo | (hi << 16);
  }
}

// Thin operands live in shared memory as sT[k][16] (the batch columns of row k, zero past B),
// 32 bytes per row, the two 16-byte halves of a row swapped on every other group of four rows so
// that ldmatrix reads of 8 consecutive rows hit 8 distinct bank groups.
__device__ __forceinline__ int wn_swz(int k, int n) { return k * WN_NC + ((((n >> 3) ^ (k >> 2)) & 1) << 3) + (n & 7); }

// Stage src [K][B] (row-major) into sT rows [0, K) with f applied (APPLY_F) and rounded to the
// storage type, and zero rows [K, Kz).  Columns n >= B are zeroed once per launch and never
// written.  B = 16 rows are 16-byte vector copies; other widths go element by element.
template <typename T, int ACT, bool APPLY_F>
__device__ __forceinline__ void wn_stage(const T* __restrict__ src, int K, int B, int Kz, T* sT) {
  constexpr int NV = 2;  // 16-byte vectors per thread per round, all loaded before any is stored
  const int tid = threadIdx.x;
  if (B == WN_NC && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
    const int nvec = 2 * K;  // two halves per row
    const uint4* sv = reinterpret_cast<const uint4*>(src);
    for (int base = tid; base < nvec; base += WN_THREADS * NV) {
      uint4 v[NV];
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int c = base + j * WN_THREADS;
        if (c < nvec) v[j] = __ldcg(sv + c);
      }
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int c = base + j * WN_THREADS;
        if (c >= nvec) break;
        if constexpr (APPLY_F) {
          T* h = reinterpret_cast<T*>(&v[j]);
#pragma unroll
          for (int q = 0; q < 8; ++q) h[q] = St<T>::st(act_f<ACT>(St<T>::ld(h[q])));
        }
        const int k = c >> 1;
        *reinterpret_cast<uint4*>(sT + wn_swz(k, (c & 1) * 8)) = v[j];
      }
    }
  } else {
    for (int idx = tid; idx < K * B; idx += WN_THREADS) {
      const int k = idx / B, n = idx - k * B;
      float f = ldcg(src + idx);
      if constexpr (APPLY_F) f = act_f<ACT>(f);
      sT[wn_swz(k, n)] = St<T>::st(f);
    }
  }
  for (int i = tid; i < (Kz - K) * WN_NC; i += WN_THREADS) sT[K * WN_NC + i] = St<T>::st(0.f);
}

__device__ __forceinline__ void wn_ldmatrix_x4_trans(uint32_t (&r)[4], const void* p) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}

__device__ __forceinline__ void wn_ldmatrix_x4(uint32_t (&r)[4], const void* p) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}

// Unit u of a phase over layers [l0, l1] (units of 32 rows, layer by layer): its layer and first row.
template <typename T>
__device__ __forceinline__ bool wn_unit(const WideParams<T>& p, int l0, int l1, int u, int& l, int& row0) {
  if (u < 0) return false;
  for (l = l0; l <= l1; ++l) {
    const int n = (p.dims[l] + WN_ROWS - 1) / WN_ROWS;
    if (u < n) {
      row0 = u * WN_ROWS;
      return true;
    }
    u -= n;
  }
  return false;
}

// One 16-bit element through L2 (weights change between phases; L1 is not coherent across SMs).
template <typename T>
__device__ __forceinline__ T wn_ldcg_t(const T* ptr) {
  const unsigned short u = __ldcg(reinterpret_cast<const unsigned short*>(ptr));
  T v;
  *reinterpret_cast<unsigned short*>(&v) = u;
  return v;
}

// Resident rows: Wp[r][k] = W[l][row0 + r][k] of this CTA's P unit (zero outside), row stride res_kp + 8.
template <typename T>
__device__ void wn_load_rows(const WideParams<T>& p, T* Wp) {
  const int ld = p.res_kp + 8, nv = p.res_kp / 8;
  int l = 0, row0 = 0;
  const bool has = wn_unit(p, 0, p.L - 1, (int)blockIdx.x, l, row0);
  const int M = has ? p.dims[l] : 0, K = has ? p.dims[l + 1] : 0;
  const T* W = has ? p.w[l] : nullptr;
  for (int i = threadIdx.x; i < WN_ROWS * nv; i += WN_THREADS) {
    const int r = i / nv, k = (i - r * nv) * 8, m = row0 + r;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (m < M && k < K) {
      if ((K & 7) == 0) {
        v = __ldcg(reinterpret_cast<const uint4*>(W + (long long)m * K + k));
      } else {
        T* h = reinterpret_cast<T*>(&v);
        for (int j = 0; j < 8 && k + j < K; ++j) h[j] = wn_ldcg_t(W + (long long)m * K + k + j);
      }
    }
    *reinterpret_cast<uint4*>(Wp + r * ld + k) = v;
  }
}

// Resident columns: Wi[k][j] = W[l-1][k][row0 + j] of this CTA's I unit (zero outside), row stride
// WN_WI_LD; rows [0, res_ki).
template <typename T>
__device__ void wn_load_cols(const WideParams<T>& p, T* Wi) {
  int l = 0, row0 = 0;
  const bool has = p.L > 1 && wn_unit(p, 1, p.L - 1, (int)blockIdx.x, l, row0);
  const int M = has ? p.dims[l] : 0, K = has ? p.dims[l - 1] : 0;
  const T* W = has ? p.w[l - 1] : nullptr;
  for (int i = threadIdx.x; i < p.res_ki * 4; i += WN_THREADS) {
    const int k = i >> 2, j = (i & 3) * 8, m = row0 + j;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (k < K && m < M) {
      if ((M & 7) == 0) {
        v = __ldcg(reinterpret_cast<const uint4*>(W + (long long)k * M + m));
      } else {
        T* h = reinterpret_cast<T*>(&v);
        for (int q = 0; q < 8 && m + q < M; ++q) h[q] = wn_ldcg_t(W + (long long)k * M + m + q);
      }
    }
    *reinterpret_cast<uint4*>(Wi + k * WN_WI_LD + j) = v;
  }
}

// One GEMM phase over layers [l0, l1].  energy != nullptr: add sum_l mean(e[l]^2) (P only).
// PAIRS (I only, every hidden width even): W_low fragments from 32-bit loads of row pairs.
// RES: this CTA's unit is fixed (P and forward: its P-order unit, I: its I-order unit) and the A
// fragments come from the resident copies (Wp rows for P / forward, Wi columns for I) by ldmatrix.
template <typename T, int ACT, int MODE, bool PAIRS, bool ACC, bool RES = false>
__device__ void wn_gemm_phase(const WideParams<T>& p, int l0, int l1, float* energy, float* red, T* sT,
                              const T* Wp = nullptr, const T* Wi = nullptr) {
  constexpr int KSTEPS = 8;  // k16 steps whose W fragments a warp loads before using any
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gq = lane >> 2, tq = lane & 3;
  const int tile = warp & 1, ksl = warp >> 1;
  const int B = p.B;
  // ldmatrix.x4.trans row address of this lane: matrix (lane >> 3) = (k half, n half), row lane & 7
  const int lm_k = (lane & 7) + ((lane >> 3) & 1) * 8, lm_n = (lane >> 4) * 8;
  int total = 0;
  for (int l = l0; l <= l1; ++l) total += (p.dims[l] + WN_ROWS - 1) / WN_ROWS;
  // forward phases (one layer) on resident rows: the unit is this CTA's P-order unit, if in layer l0
  int ubase = 0;
  if (RES && MODE == WN_F)
    for (int l = 0; l < l0; ++l) ubase += (p.dims[l] + WN_ROWS - 1) / WN_ROWS;
  for (int u = (int)blockIdx.x - ubase; u < total; u += gridDim.x) {
    if (u < 0) continue;
    int l = l0, r = u;
    while (r >= (p.dims[l] + WN_ROWS - 1) / WN_ROWS) {
      r -= (p.dims[l] + WN_ROWS - 1) / WN_ROWS;
      ++l;
    }
    const int row0 = r * WN_ROWS;
    const int M = p.dims[l];
    const int K = (MODE == WN_I) ? p.dims[l - 1] : p.dims[l + 1];
    const int Kp = (K + 15) & ~15;
    constexpr bool from_cache = (MODE != WN_I) && ACC;
    const T* src = (MODE == WN_I) ? p.e[l - 1] : (from_cache ? p.a[l + 1] : p.x[l + 1]);
    const unsigned short* A =
        reinterpret_cast<const unsigned short*>((MODE == WN_I) ? p.w[l - 1] : p.w[l]);
    // the epilogue's own operands are fixed during the phase: fetch them now, under the GEMM
    const int erow = tid / WN_NC, ecol = tid % WN_NC;
    const int em = row0 + erow;
    const bool eval = em < M && ecol < B;
    const int eidx = em * B + ecol;
    float xv = 0.f, ev = 0.f;
    if (MODE != WN_F && eval) xv = ldcg(p.x[l] + eidx);
    if (MODE == WN_I && eval) ev = ldcg(p.e[l] + eidx);
    // I reads W_low [K][M] (M contiguous): with M even, fragment rows gq / gq + 8 of a tile are the
    // physical row pair 2gq / 2gq + 1, so each register pair comes from two 32-bit loads + a byte permute
    constexpr bool pairs = (MODE == WN_I) && PAIRS;
    float acc[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[j][q] = 0.f;
    const int ks = ((Kp + WN_KSLICES - 1) / WN_KSLICES + 15) & ~15;
    const int kb0 = ksl * ks, kb1 = min(kb0 + ks, Kp);
    const int r0 = row0 + 16 * tile + gq, r1 = r0 + 8;
    bool staged = false;
    // the first block of W fragments is in flight while the thin operand is staged
    for (int kb = kb0; kb < kb1 || !staged; kb += 16 * KSTEPS) {
      uint32_t a[KSTEPS][4];
      if constexpr (RES) {
        // A fragments come from shared memory right before their MMA (below)
      } else if constexpr (pairs) {
        const int mp = row0 + 16 * tile + 2 * gq;
#pragma unroll
        for (int st = 0; st < KSTEPS; ++st) {
          const int k = kb + 16 * st + 2 * tq;
          const bool in = kb + 16 * st < kb1 && mp < M;
          const uint32_t* w32 = reinterpret_cast<const uint32_t*>(A);
          const int o = (k * M + mp) >> 1;  // in 32-bit words; M even
          const int hm = M >> 1;
          const uint32_t u0 = (in && k < K) ? __ldcg(w32 + o) : 0u;
          const uint32_t v0 = (in && k + 1 < K) ? __ldcg(w32 + o + hm) : 0u;
          const uint32_t u1 = (in && k + 8 < K) ? __ldcg(w32 + o + 8 * hm) : 0u;
          const uint32_t v1 = (in && k + 9 < K) ? __ldcg(w32 + o + 9 * hm) : 0u;
          a[st][0] = __byte_perm(u0, v0, 0x5410);
          a[st][1] = __byte_perm(u0, v0, 0x7632);
          a[st][2] = __byte_perm(u1, v1, 0x5410);
          a[st][3] = __byte_perm(u1, v1, 0x7632);
        }
      } else {
#pragma unroll
        for (int st = 0; st < KSTEPS; ++st) {
          const int k = kb + 16 * st + 2 * tq;
          const bool in = kb + 16 * st < kb1;
          a[st][0] = in ? wn_load_a<MODE>(A, M, K, r0, k) : 0u;
          a[st][1] = in ? wn_load_a<MODE>(A, M, K, r1, k) : 0u;
          a[st][2] = in ? wn_load_a<MODE>(A, M, K, r0, k + 8) : 0u;
          a[st][3] = in ? wn_load_a<MODE>(A, M, K, r1, k + 8) : 0u;
        }
      }
      if (!staged) {
        wn_stage<T, ACT, (MODE != WN_I) && !from_cache>(src, K, B, Kp, sT);
        __syncthreads();
        staged = true;
      }
#pragma unroll
      for (int st = 0; st < KSTEPS; ++st) {
        if (kb + 16 * st >= kb1) break;
        if constexpr (RES) {
          const int k16 = kb + 16 * st, mat = lane >> 3, rr = lane & 7;
          if constexpr (MODE == WN_I)  // A(m, k) = Wi[k][m]: transposed 8x8 blocks
            wn_ldmatrix_x4_trans(a[st], Wi + (k16 + rr + (mat >> 1) * 8) * WN_WI_LD + 16 * tile + (mat & 1) * 8);
          else  // A(m, k) = Wp[m][k]
            wn_ldmatrix_x4(a[st], Wp + (16 * tile + rr + (mat & 1) * 8) * (p.res_kp + 8) + k16 + (mat >> 1) * 8);
        }
        uint32_t b[4];  // b0, b1 of n-tile 0, then of n-tile 1
        const int k = kb + 16 * st + lm_k;
        wn_ldmatrix_x4_trans(b, sT + wn_swz(k, lm_n));
        wn_mma<T>(acc[0], a[st], b[0], b[1]);
        wn_mma<T>(acc[1], a[st], b[2], b[3]);
      }
    }
    // partials by physical row of the tile
    const int pr0 = pairs ? 2 * gq : gq, pr1 = pairs ? 2 * gq + 1 : gq + 8;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int c = 8 * j + 2 * tq;
      red[(warp * 16 + pr0) * WN_NC + c] = acc[j][0];
      red[(warp * 16 + pr0) * WN_NC + c + 1] = acc[j][1];
      red[(warp * 16 + pr1) * WN_NC + c] = acc[j][2];
      red[(warp * 16 + pr1) * WN_NC + c + 1] = acc[j][3];
    }
    __syncthreads();
    float esum = 0.f;
    if (eval) {  // 32 rows x 16 columns = 512 threads
      const int t = erow >> 4, ri = erow & 15;
      float sum = 0.f;
#pragma unroll
      for (int s = 0; s < WN_KSLICES; ++s) sum += red[((2 * s + t) * 16 + ri) * WN_NC + ecol];
      if constexpr (MODE == WN_F) {
        const T xs = St<T>::st(sum);
        p.x[l][eidx] = xs;
        if constexpr (ACC) p.a[l][eidx] = St<T>::st(act_f<ACT>(St<T>::ld(xs)));
      } else if constexpr (MODE == WN_P) {
        const float e16 = rnd<T>(xv - rnd<T>(sum));
        p.e[l][eidx] = St<T>::st(e16);
        esum = e16 * e16 / ((float)M * (float)B);
      } else {
        const T xs = St<T>::st(xv + p.gamma * (-ev + act_df<ACT>(xv) * sum));
        p.x[l][eidx] = xs;
        if constexpr (ACC) p.a[l][eidx] = St<T>::st(act_f<ACT>(St<T>::ld(xs)));
      }
    }
    if (MODE == WN_P && energy != nullptr) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) esum += __shfl_xor_sync(0xffffffffu, esum, o);
      if (lane == 0 && esum != 0.f) atomicAdd(energy, esum);
    }
    __syncthreads();  // sT / red are rewritten by the next unit
  }
}

// W[l] = cast(W[l] + alpha e[l] f(x[l+1])^T) for every layer.  dW of a 16 x 8 tile is one
// mma.sync m16n8k16 with the batch (B <= 16, zero-padded) as the reduction: A = the unit's rows of
// e[l] (sE[32][16]), B(n, c) = f(x[l+1])[c][n] straight from the staged rows of sT.
// RES: the unit is this CTA's P-order unit and W is read from (and written back to) its resident
// rows as well as global memory.
template <typename T, int ACT, bool ACC, bool RES = false>
__device__ void wn_weight_phase(const WideParams<T>& p, T* sE, T* sT, T* Wp = nullptr) {
  constexpr int NT = 8;  // n-tiles whose W values a warp loads before updating any
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gq = lane >> 2, tq = lane & 3;
  const int mt = warp & 1, wq = warp >> 1;  // m-tile, and this warp's share of the n-tiles
  const int B = p.B;
  int total = 0;
  for (int l = 0; l < p.L; ++l) total += (p.dims[l] + WN_ROWS - 1) / WN_ROWS;
  for (int u = blockIdx.x; u < total; u += gridDim.x) {
    int l = 0, r = u;
    while (r >= (p.dims[l] + WN_ROWS - 1) / WN_ROWS) {
      r -= (p.dims[l] + WN_ROWS - 1) / WN_ROWS;
      ++l;
    }
    const int row0 = r * WN_ROWS;
    const int M = p.dims[l], K = p.dims[l + 1];
    const int K8 = (K + 7) & ~7;
    for (int i = tid; i < WN_ROWS * WN_NC; i += WN_THREADS) {
      const int rr = i / WN_NC, n = i % WN_NC;
      const int m = row0 + rr;
      sE[i] = St<T>::st((m < M && n < B) ? ldcg(p.e[l] + m * B + n) : 0.f);
    }
    wn_stage<T, ACT, !ACC>(ACC ? p.a[l + 1] : p.x[l + 1], K, B, K8, sT);
    __syncthreads();
    uint32_t a[4];
    {
      const T* e0 = sE + (mt * 16 + gq) * WN_NC + 2 * tq;
      a[0] = *reinterpret_cast<const uint32_t*>(e0);
      a[1] = *reinterpret_cast<const uint32_t*>(e0 + 8 * WN_NC);
      a[2] = *reinterpret_cast<const uint32_t*>(e0 + 8);
      a[3] = *reinterpret_cast<const uint32_t*>(e0 + 8 * WN_NC + 8);
    }
    const int m0 = row0 + mt * 16 + gq, m1 = m0 + 8;
    const bool even = (K % 2) == 0;
    T* W = p.w[l];
    const int ntiles = K8 / 8;
    for (int j0 = wq; j0 < ntiles; j0 += WN_KSLICES * NT) {
      uint32_t w0[NT], w1[NT];
#pragma unroll
      for (int q = 0; q < NT; ++q) {
        const int c = (j0 + q * WN_KSLICES) * 8 + 2 * tq;
        w0[q] = w1[q] = 0u;
        if (even && c < K) {
          if constexpr (RES) {
            const int ld = p.res_kp + 8;
            if (m0 < M) w0[q] = *reinterpret_cast<const uint32_t*>(Wp + (mt * 16 + gq) * ld + c);
            if (m1 < M) w1[q] = *reinterpret_cast<const uint32_t*>(Wp + (mt * 16 + gq + 8) * ld + c);
          } else {
            if (m0 < M) w0[q] = __ldcg(reinterpret_cast<const uint32_t*>(W + m0 * K + c));
            if (m1 < M) w1[q] = __ldcg(reinterpret_cast<const uint32_t*>(W + m1 * K + c));
          }
        }
      }
#pragma unroll
      for (int q = 0; q < NT; ++q) {
        const int j = j0 + q * WN_KSLICES;
        if (j >= ntiles) break;
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(sT + wn_swz(j * 8 + gq, 2 * tq));
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(sT + wn_swz(j * 8 + gq, 2 * tq + 8));
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        wn_mma<T>(d, a, b0, b1);
        const int c = j * 8 + 2 * tq;
        if (even) {
          if (c < K && m0 < M) {
            T* h = reinterpret_cast<T*>(&w0[q]);
            h[0] = St<T>::st(St<T>::ld(h[0]) + p.alpha * d[0]);
            h[1] = St<T>::st(St<T>::ld(h[1]) + p.alpha * d[1]);
            *reinterpret_cast<uint32_t*>(W + m0 * K + c) = w0[q];
            if constexpr (RES) *reinterpret_cast<uint32_t*>(Wp + (mt * 16 + gq) * (p.res_kp + 8) + c) = w0[q];
          }
          if (c < K && m1 < M) {
            T* h = reinterpret_cast<T*>(&w1[q]);
            h[0] = St<T>::st(St<T>::ld(h[0]) + p.alpha * d[2]);
            h[1] = St<T>::st(St<T>::ld(h[1]) + p.alpha * d[3]);
            *reinterpret_cast<uint32_t*>(W + m1 * K + c) = w1[q];
            if constexpr (RES) *reinterpret_cast<uint32_t*>(Wp + (mt * 16 + gq + 8) * (p.res_kp + 8) + c) = w1[q];
          }
        } else {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (c + h >= K) continue;
            if (m0 < M) W[m0 * K + c + h] = St<T>::st(ldcg(W + m0 * K + c + h) + p.alpha * d[h]);
            if (m1 < M) W[m1 * K + c + h] = St<T>::st(ldcg(W + m1 * K + c + h) + p.alpha * d[2 + h]);
            if constexpr (RES) {
              const int ld = p.res_kp + 8;
              if (m0 < M) Wp[(mt * 16 + gq) * ld + c + h] = W[m0 * K + c + h];
              if (m1 < M) Wp[(mt * 16 + gq + 8) * ld + c + h] = W[m1 * K + c + h];
            }
          }
        }
      }
    }
    __syncthreads();
  }
}

template <typename T, int ACT, bool PAIRS, bool ACC, bool RES>
__global__ void __launch_bounds__(WN_THREADS, 1) wide_net_kernel(const __grid_constant__ WideParams<T> p) {
  extern __shared__ __align__(16) uint8_t wn_smem[];
  float* red = reinterpret_cast<float*>(wn_smem);                 // [16 warps][16][16] fp32
  T* sE = reinterpret_cast<T*>(red + WN_WARPS * 16 * WN_NC);      // [32][16]
  T* sT = sE + WN_ROWS * WN_NC;                                   // [kmax][16], swizzled halves
  T* Wp = sT + p.kmax * WN_NC;                                    // RES: [32][res_kp + 8]
  T* Wi = Wp + WN_ROWS * (p.res_kp + 8);                          // RES: [res_ki][WN_WI_LD]
  const int L = p.L, B = p.B;
  unsigned epoch = 0;  // grid barriers passed in this launch
  if (B < WN_NC)  // batch columns past B stay zero for the whole launch (staging never writes them)
    for (int i = threadIdx.x; i < p.kmax * WN_NC; i += WN_THREADS) sT[i] = St<T>::st(0.f);
  if constexpr (RES) {  // this CTA's rows of its P unit and columns of its I unit, for the whole launch
    wn_load_rows(p, Wp);
    wn_load_cols(p, Wi);
  }
  __syncthreads();
  for (int step = 0; step < p.steps; ++step) {
    long long* tr = (p.phase_ns != nullptr && step < IPC_NET_TRACE_STEPS && blockIdx.x == 0 && threadIdx.x == 0)
                        ? p.phase_ns + (long long)step * IPC_NET_TRACE_PHASES
                        : nullptr;
    if (tr) tr[WT_START] = wn_now();
    if (p.pool_x != nullptr || ACC) {
      // elementwise: the step's batch (pool), the input activation a[L], and without a forward
      // sweep the cache of every hidden state
      const long long nx = (long long)p.dims[L] * B, ny = (long long)p.dims[0] * B;
      const int b = p.pool_x != nullptr ? (p.first_batch + step) % p.pool_batches : 0;
      const long long gstride = (long long)gridDim.x * WN_THREADS;
      const long long g0 = blockIdx.x * (long long)WN_THREADS + threadIdx.x;
      if (p.pool_x != nullptr) {
        const T* py = p.pool_y + (long long)b * ny;
        for (long long i = g0; i < ny; i += gstride) p.x[0][i] = py[i];
      }
      const T* px = p.pool_x != nullptr ? p.pool_x + (long long)b * nx : nullptr;
      for (long long i = g0; i < nx; i += gstride) {
        const T v = px != nullptr ? px[i] : p.x[L][i];
        if (px != nullptr) p.x[L][i] = v;
        if constexpr (ACC) p.a[L][i] = St<T>::st(act_f<ACT>(St<T>::ld(v)));
      }
      if (ACC && !p.forward_init) {
        for (int l = 1; l < L; ++l) {
          const long long n = (long long)p.dims[l] * B;
          for (long long i = g0; i < n; i += gstride) p.a[l][i] = St<T>::st(act_f<ACT>(ldcg(p.x[l] + i)));
        }
      }
      if (!wn_grid_sync(p.sync, epoch)) return;
    }
    if (tr) tr[WT_BATCH] = wn_now();
    if (p.forward_init) {
      for (int l = L - 1; l >= 1; --l) {
        wn_gemm_phase<T, ACT, WN_F, false, ACC, RES>(p, l, l, nullptr, red, sT, Wp, Wi);
        if (!wn_grid_sync(p.sync, epoch)) return;
      }
    }
    if (tr) tr[WT_FORWARD] = wn_now();
    for (int t = 0; t < p.T_it; ++t) {
      float* en = (t == p.T_it - 1 && p.energy != nullptr) ? p.energy + step : nullptr;
      wn_gemm_phase<T, ACT, WN_P, false, ACC, RES>(p, 0, L - 1, en, red, sT, Wp, Wi);
      if (!wn_grid_sync(p.sync, epoch)) return;
      if (tr && t == 0) tr[WT_P0] = wn_now();
      if (L > 1) {
        wn_gemm_phase<T, ACT, WN_I, PAIRS, ACC, RES>(p, 1, L - 1, nullptr, red, sT, Wp, Wi);
        if (!wn_grid_sync(p.sync, epoch)) return;
      }
      if (tr && t == 0) tr[WT_I0] = wn_now();
    }
    if (tr) tr[WT_ITER] = wn_now();
    if (p.update_weights) {
      wn_weight_phase<T, ACT, ACC, RES>(p, sE, sT, Wp);
      if (!wn_grid_sync(p.sync, epoch)) return;
      if constexpr (RES) {  // the resident columns were updated by their rows' CTAs: reload them
        wn_load_cols(p, Wi);
        __syncthreads();
      }
    }
    if (tr) tr[WT_W] = wn_now();
  }
}

// Failure-detection self-test: CTA 1 returns without arriving, so CTA 0's barrier wait must expire.
__global__ void wn_selftest_kernel(unsigned* sync, long long limit_ns) {
  if (blockIdx.x != 0) return;
  unsigned epoch = 0;
  wn_grid_sync(sync, epoch, limit_ns);
}

template <typename T>
int wn_prepare(WideParams<T>& p, const ipc_net_t* net, const ipc_net_run_t* run, size_t* smem) {
  p = WideParams<T>{};
  p.L = net->L;
  p.B = net->B;
  int kmax = 16;
  for (int l = 0; l <= net->L; ++l) {
    p.dims[l] = net->dims[l];
    kmax = max(kmax, net->dims[l]);
    p.x[l] = reinterpret_cast<T*>(net->x[l]);
    p.e[l] = l < net->L ? reinterpret_cast<T*>(net->e[l]) : nullptr;
  }
  for (int l = 0; l < net->L; ++l) p.w[l] = reinterpret_cast<T*>(net->w[l]);
  p.acache = 1;
  for (int l = 1; l <= net->L; ++l) {
    p.a[l] = reinterpret_cast<T*>(net->a[l]);
    if (p.a[l] == nullptr) p.acache = 0;
  }
  if (!p.acache)
    for (int l = 0; l <= net->L; ++l) p.a[l] = nullptr;
  p.kmax = (kmax + 63) & ~63;
  if (run != nullptr) {
    p.pool_x = reinterpret_cast<const T*>(run->pool_x);
    p.pool_y = reinterpret_cast<const T*>(run->pool_y);
    p.pool_batches = run->pool_batches;
    p.first_batch = run->first_batch;
    p.steps = run->steps;
    p.T_it = run->T;
    p.forward_init = run->forward_init;
    p.update_weights = run->update_weights;
    p.alpha = run->alpha;
    p.gamma = run->gamma;
    p.energy = run->energy;
    p.sync = reinterpret_cast<unsigned*>(run->sync);
    p.phase_ns = run->phase_ns;
  }
  *smem = (size_t)WN_WARPS * 16 * WN_NC * sizeof(float) + (size_t)WN_ROWS * WN_NC * sizeof(T) +
          (size_t)p.kmax * WN_NC * sizeof(T);
  return IPC_OK;
}

template <typename T, int ACT, bool PAIRS, bool ACC, bool RES = false>
int wn_launch(const WideParams<T>& p, size_t smem, cudaStream_t s) {
  auto kern = wide_net_kernel<T, ACT, PAIRS, ACC, RES>;
  cudaError_t err = ensure_kernel_smem<wide_net_kernel<T, ACT, PAIRS, ACC, RES>>((int)smem);
  if (err != cudaSuccess) return set_error(IPC_ERR_CUDA, "wide net kernel smem attribute: %s", cudaGetErrorString(err));
  int dev = 0, sms = 0, per_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // residency check once per device and size (the answer does not change within a process)
  static long long checked[64] = {};  // smem bytes + 1 of the last successful check
  if (dev >= 0 && dev < 64 && checked[dev] == (long long)smem + 1) {
    per_sm = 1;
  } else {
    err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, WN_THREADS, smem);
    if (err == cudaSuccess && per_sm >= 1 && dev >= 0 && dev < 64) checked[dev] = (long long)smem + 1;
  }
  if (err != cudaSuccess || per_sm < 1)
    return set_error(IPC_ERR_UNSUPPORTED, "wide net kernel: no resident CTA per SM (%s)", cudaGetErrorString(err));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sms, 1, 1);  // one CTA per SM: all co-resident (cooperative launch)
  cfg.blockDim = dim3(WN_THREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  err = cudaLaunchKernelEx(&cfg, kern, p);
  if (err != cudaSuccess) return set_error(IPC_ERR_CUDA, "wide net kernel launch: %s", cudaGetErrorString(err));
  count_launch();
  return check_launch("wide net kernel");
}

}  // namespace

// Whether the wide small-batch kernel can run this network (16-bit storage is checked at launch).
bool wide_net_fits(const ipc_net_t* net) {
  if (net == nullptr || net->nets != 1 || net->B < 1 || net->B > WN_MAX_B) return false;
  if (net->L < 1 || net->L > IPC_NET_MAX_LAYERS) return false;
  for (int l = 0; l <= net->L; ++l)
    if (net->dims[l] < 1 || net->dims[l] > WN_MAX_DIM) return false;
  return true;
}

int wide_net_smem(const ipc_net_t* net) {
  WideParams<__half> p;
  size_t smem = 0;
  wn_prepare(p, net, nullptr, &smem);
  return (int)smem;
}

int wide_net_train(const ipc_net_t* net, const ipc_net_run_t* run, cudaStream_t s) {
  if (run->sync == nullptr) return set_error(IPC_ERR_ARG, "wide net kernel: run->sync (IPC_NET_SYNC_BYTES) is required");
  // the launch-wide arrival counter must not wrap: barriers x CTAs < 2^32
  const long long barriers = (long long)run->steps * (net->L + 2LL * run->T + 2);
  if (barriers * 1024 >= (1LL << 32))
    return set_error(IPC_ERR_ARG, "wide net kernel: steps=%d too many for one launch (split it)", run->steps);
  cudaError_t err = cudaMemsetAsync(run->sync, 0, IPC_NET_SYNC_BYTES, s);
  if (err != cudaSuccess) return set_error(IPC_ERR_CUDA, "sync memset: %s", cudaGetErrorString(err));
  IPC_DISPATCH_DT16(run->dtype, TT, {
    WideParams<TT> p;
    size_t smem = 0;
    wn_prepare(p, net, run, &smem);
    bool pairs = true;  // every state-update width even: row-pair loads of W_low
    for (int l = 1; l < net->L; ++l) pairs = pairs && (net->dims[l] % 2 == 0);
    // resident weights: with at most one P unit and one I unit per CTA (one CTA per SM), each CTA keeps
    // its P unit's rows of W[l] and its I unit's columns of W[l-1] in shared memory for the launch, so
    // no phase reads W from L2 (the weight phase updates the rows in place and the columns are
    // reloaded once per step)
    int sms = 0;
    {
      int dev = 0;
      cudaGetDevice(&dev);
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    }
    int total_p = 0, total_i = 0, kp = 16, ki = 16;
    for (int l = 0; l < net->L; ++l) {
      total_p += (net->dims[l] + WN_ROWS - 1) / WN_ROWS;
      kp = max(kp, net->dims[l + 1]);
      if (l >= 1) {
        total_i += (net->dims[l] + WN_ROWS - 1) / WN_ROWS;
        ki = max(ki, net->dims[l - 1]);
      }
    }
    kp = (kp + 15) & ~15;
    ki = (ki + 15) & ~15;
    const size_t smem_res = smem + (size_t)WN_ROWS * (kp + 8) * sizeof(TT) + (size_t)ki * WN_WI_LD * sizeof(TT);
    const bool res = p.acache && total_p <= sms && total_i <= sms && smem_res + 256 <= 227u * 1024u;
    IPC_DISPATCH_ACT(run->act, AC, {
      if (res) {
        p.res_kp = kp;
        p.res_ki = ki;
        return wn_launch<TT, AC, false, true, true>(p, smem_res, s);
      }
      if (p.acache)
        return pairs ? wn_launch<TT, AC, true, true>(p, smem, s) : wn_launch<TT, AC, false, true>(p, smem, s);
      return pairs ? wn_launch<TT, AC, true, false>(p, smem, s) : wn_launch<TT, AC, false, false>(p, smem, s);
    });
  });
  return IPC_OK;
}

int wide_selftest_timeout(void* sync, int limit_us, cudaStream_t s) {
  if (sync == nullptr || limit_us < 1 || limit_us > 1000000)
    return set_error(IPC_ERR_ARG, "selftest: sync must be non-null and limit_us in [1, 1e6]");
  cudaError_t err = cudaMemsetAsync(sync, 0, IPC_NET_SYNC_BYTES, s);
  if (err != cudaSuccess) return set_error(IPC_ERR_CUDA, "sync memset: %s", cudaGetErrorString(err));
  wn_selftest_kernel<<<2, 32, 0, s>>>(reinterpret_cast<unsigned*>(sync), 1000LL * limit_us);
  count_launch();
  return check_launch("barrier self-test");
}

int read_wide_status(int* status, int clear) {
  int v = 0;
  cudaError_t err = cudaMemcpyFromSymbol(&v, g_wide_status, sizeof(int));
  if (err != cudaSuccess) return set_error(IPC_ERR_CUDA, "device status read: %s", cudaGetErrorString(err));
  if (clear && v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_wide_status, &zero, sizeof(int));
  }
  if (status) *status = v;
  return IPC_OK;
}

}  // namespace ipc
