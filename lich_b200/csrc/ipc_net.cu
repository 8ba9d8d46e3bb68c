// Persistent multi-layer iPC kernel for small widths (hidden <= 64).
//
// One launch runs `steps` whole training steps of `nets` independent
// networks; the work the reference spreads over 3L-1 launches per iPC step
// (src/ipc_tilelang/trainer.py:601-679) plus its eager forward-init sweep
// (trainer.py:509-516) happens inside one kernel, so launch latency -- the
// cost that dominates at hidden 64 -- is paid once per launch.
//
// Decomposition.  Network n runs on a cluster of C CTAs; CTA c owns batch
// columns [c*NCOL, (c+1)*NCOL).  Prediction errors and state updates are
// column-local, so the T inference iterations need only __syncthreads.  All
// W[l] with l < L-1 live in shared memory; W[L-1] (the wide input layer,
// e.g. 64 x 784) is streamed from L2 once per training step to form
// mu_top = W[L-1] f(x_L) for the CTA's columns, which is then reused by the
// forward-init sweep and by all T prediction passes (W and x_L are fixed
// within a training step, so this is the same number the reference computes
// T+1 times).  The weight update reduces over all B columns: every CTA writes
// its x / e columns to their global homes (they are outputs anyway), the
// cluster synchronises, and each CTA updates a disjoint set of 32-column
// blocks of the W matrices, reading E and f(x) rows for all columns from L2.
//
// Tensor cores: mma.sync m16n8k16 with fp32 accumulators, fragments from
// shared memory via ldmatrix.  At hidden 64 every GEMM here is a handful of
// 16x8x16 tiles; register-resident fragments avoid the TMEM round trip that
// tcgen05 would add to each of the ~40 dependent phases of a step.
//
// Rounding points follow the reference kernels: a = cast(f(x_stored))
// (tilelang_kernels.py:163), e = cast(x) - cast(acc) (:173),
// x = cast(x + g(-e + f'(x) acc)) (:229-230), W = cast(W + a acc) (:320), and
// the forward sweep x[l] = cast(W[l] @ f(x[l+1])) (trainer.py:513-515).
#include <cstdio>

#include "ipc_common.cuh"

namespace ipc {
namespace {

constexpr int NET_THREADS = 256;
constexpr int NET_WARPS = NET_THREADS / 32;
constexpr int WLD = 72;        // smem row stride (halves) of resident W tiles (<= 64 cols + 8)
constexpr int KC = 64;         // K chunk of the streamed input layer
constexpr int WU_COLS = 32;    // W columns per weight-update work item
constexpr int MAXL = IPC_NET_MAX_LAYERS;

template <typename T>
struct NetParams {
  int L, B, nets, C;
  int dims[MAXL + 1];
  int rows16[MAXL + 1];  // dims rounded up to 16
  T* w[MAXL];
  T* x[MAXL + 1];
  T* e[MAXL + 1];
  T* a[MAXL + 1];
  const T* pool_x;
  const T* pool_y;
  int pool_batches, first_batch, steps, T_it, forward_init, update_weights, recompute;
  float alpha, gamma;
  float* energy;  // [steps, nets] or null
  // shared-memory layout (offsets in elements of T)
  int off_w[MAXL];
  int off_x[MAXL], off_a[MAXL], off_e[MAXL];
  int off_mu, off_stage, sld, eld;
};

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t (&r)[2], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];\n"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t (&r)[2], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];\n" : "=r"(r[0]), "=r"(r[1]) : "r"(addr));
}

template <typename T>
__device__ __forceinline__ void mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __half>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// A fragment (16x16) from row-major [m][k] shared memory.
__device__ __forceinline__ void frag_a_rowmajor(uint32_t (&r)[4], const void* base, int ld, int m0, int k0, int lane) {
  const int q = lane >> 3, j = lane & 7;
  const char* p = reinterpret_cast<const char*>(base) + 2 * ((m0 + j + (q & 1) * 8) * ld + k0 + (q >> 1) * 8);
  ldsm_x4(r, smem_addr(p));
}
// A fragment (16x16) of S^T where S is row-major [k][m] in shared memory.
__device__ __forceinline__ void frag_a_trans(uint32_t (&r)[4], const void* base, int ld, int m0, int k0, int lane) {
  const int q = lane >> 3, j = lane & 7;
  const char* p = reinterpret_cast<const char*>(base) + 2 * ((k0 + j + (q >> 1) * 8) * ld + m0 + (q & 1) * 8);
  ldsm_x4_t(r, smem_addr(p));
}
// B fragment (16x8, k x n) from row-major [k][n] shared memory.
__device__ __forceinline__ void frag_b_kn(uint32_t (&r)[2], const void* base, int ld, int k0, int n0, int lane) {
  const int q = (lane >> 3) & 1, j = lane & 7;
  const char* p = reinterpret_cast<const char*>(base) + 2 * ((k0 + j + q * 8) * ld + n0);
  ldsm_x2_t(r, smem_addr(p));
}
// B fragment (16x8, k x n) from row-major [n][k] shared memory.
__device__ __forceinline__ void frag_b_nk(uint32_t (&r)[2], const void* base, int ld, int k0, int n0, int lane) {
  const int q = (lane >> 3) & 1, j = lane & 7;
  const char* p = reinterpret_cast<const char*>(base) + 2 * ((n0 + j) * ld + k0 + q * 8);
  ldsm_x2(r, smem_addr(p));
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}

template <typename T>
__device__ __forceinline__ void st2(T* p, float v0, float v1) {
  T h[2] = {St<T>::st(v0), St<T>::st(v1)};
  *reinterpret_cast<uint32_t*>(p) = *reinterpret_cast<uint32_t*>(h);
}

// Copy a [rows x cols] block (global row stride gld, starting at column gc0)
// into shared memory (row stride sld), optionally through f.  Vectorised
// (16 B) when the global rows are 16-byte aligned; columns past `cols_valid`
// and rows past `rows` are written as zero up to rows_pad x cols_pad.
template <typename T, int ACT, bool APPLY, bool CG>
__device__ void load_block(T* s, int sld, const T* g, long long gld, int rows, int rows_pad, int gc0, int cols_valid,
                           int cols_pad, bool vec) {
  const int tid = threadIdx.x;
  if (vec) {
    const int vpr = cols_pad / 8;  // vectors per row
    for (int it = tid; it < rows_pad * vpr; it += NET_THREADS) {
      const int r = it / vpr, c = (it % vpr) * 8;
      uint4 raw = make_uint4(0, 0, 0, 0);
      if (r < rows && c + 8 <= cols_valid) {
        const uint4* src = reinterpret_cast<const uint4*>(g + (long long)r * gld + gc0 + c);
        raw = CG ? __ldcg(src) : *src;
        if (APPLY) {
          T* h = reinterpret_cast<T*>(&raw);
#pragma unroll
          for (int j = 0; j < 8; ++j) h[j] = St<T>::st(act_f<ACT>(St<T>::ld(h[j])));
        }
      } else if (r < rows) {
        T* h = reinterpret_cast<T*>(&raw);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float v = 0.f;
          if (c + j < cols_valid) {
            v = St<T>::ld(g[(long long)r * gld + gc0 + c + j]);
            if (APPLY) v = rnd<T>(act_f<ACT>(v));
          }
          h[j] = St<T>::st(v);
        }
      }
      *reinterpret_cast<uint4*>(s + r * sld + c) = raw;
    }
  } else {
    for (int it = tid; it < rows_pad * cols_pad; it += NET_THREADS) {
      const int r = it / cols_pad, c = it % cols_pad;
      float v = 0.f;
      if (r < rows && c < cols_valid) {
        v = St<T>::ld(g[(long long)r * gld + gc0 + c]);
        if (APPLY) v = rnd<T>(act_f<ACT>(v));
      }
      s[r * sld + c] = St<T>::st(v);
    }
  }
}

// Store the CTA's [rows x NCOL] slice of a state array to its global home.
template <typename T, int NCOL>
__device__ void store_cols(T* g, int B, int c0, const T* s, int sld, int rows) {
  constexpr int VPR = NCOL / 8;
  for (int it = threadIdx.x; it < rows * VPR; it += NET_THREADS) {
    const int r = it / VPR, c = (it % VPR) * 8;
    *reinterpret_cast<uint4*>(g + (long long)r * B + c0 + c) = *reinterpret_cast<const uint4*>(s + r * sld + c);
  }
}

template <typename T, int ACT, int NCOL>
__global__ void __launch_bounds__(NET_THREADS, 1) net_kernel(const __grid_constant__ NetParams<T> p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  T* sm = reinterpret_cast<T*>(smem_raw);
  const int cta = blockIdx.x;          // rank within the cluster (cluster spans x)
  const int net = blockIdx.y;
  const int c0 = cta * NCOL;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gq = lane >> 2, tq = lane & 3;
  const int L = p.L;
  const int B = p.B;
  const int dL = p.dims[L];
  const int dTop = p.dims[L - 1];
  const int SLD = p.sld;

  // zero all of shared memory once: padding rows / columns must stay zero
  {
    uint4* z = reinterpret_cast<uint4*>(smem_raw);
    const int n16 = p.off_stage * (int)sizeof(T) / 16;
    for (int i = threadIdx.x; i < n16; i += NET_THREADS) z[i] = make_uint4(0, 0, 0, 0);
  }
  __syncthreads();

  // per-network global slabs
  T* gw[MAXL];
  T* gx[MAXL + 1];
  T* ge[MAXL + 1];
  T* ga[MAXL + 1];
#pragma unroll
  for (int l = 0; l < MAXL; ++l)
    gw[l] = l < L ? p.w[l] + (long long)net * p.dims[l] * p.dims[l + 1] : nullptr;
#pragma unroll
  for (int l = 0; l <= MAXL; ++l) {
    gx[l] = l <= L ? p.x[l] + (long long)net * p.dims[l] * B : nullptr;
    ge[l] = (l < L) ? p.e[l] + (long long)net * p.dims[l] * B : nullptr;
    ga[l] = (l <= L && p.a[l] != nullptr) ? p.a[l] + (long long)net * p.dims[l] * B : nullptr;
  }

  // resident W tiles (l < L-1)
  auto load_resident_w = [&]() {
    for (int l = 0; l < L - 1; ++l) {
      const int cols = p.dims[l + 1];
      load_block<T, ACT, false, true>(sm + p.off_w[l], WLD, gw[l], cols, p.dims[l], p.rows16[l], 0, cols,
                                      ((cols + 15) / 16) * 16, (cols % 8) == 0);
    }
  };
  load_resident_w();
  __syncthreads();

  T* sMu = sm + p.off_mu;      // cast(mu_top) [rows16(L-1)][SLD]
  T* sStage = sm + p.off_stage;

  for (int step = 0; step < p.steps; ++step) {
    const T* xL;
    const T* y;
    if (p.pool_x != nullptr) {
      const int b = (p.first_batch + step) % p.pool_batches;
      xL = p.pool_x + ((long long)b * p.nets + net) * (long long)dL * B;
      y = p.pool_y + ((long long)b * p.nets + net) * (long long)p.dims[0] * B;
    } else {
      xL = gx[L];
      y = gx[0];
    }
    // ---- x[0] (target) columns ----
    load_block<T, ACT, false, true>(sm + p.off_x[0], SLD, y, B, p.dims[0], p.rows16[0], c0, NCOL, NCOL, true);

    // ---- mu_top = W[L-1] f(x_L) for this CTA's columns (streamed over K) ----
    {
      constexpr int NT = NCOL / 8;
      const int mtiles = p.rows16[L - 1] / 16;
      const int units = mtiles * NT;
      float acc[4][4];  // up to 4 units per warp (mtiles*NT <= 4*8=32 -> 4 per warp)
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
      T* sWt = sStage;                 // [64][WLD]
      T* sXt = sStage + 64 * WLD;      // [KC][SLD]
      const bool wvec = (dL % 8) == 0;
      for (int k0 = 0; k0 < dL; k0 += KC) {
        const int kv = min(KC, dL - k0);
        load_block<T, ACT, false, true>(sWt, WLD, gw[L - 1], dL, dTop, p.rows16[L - 1], k0, kv, KC, wvec);
        // x_L rows k0.., this CTA's columns, through f
        load_block<T, ACT, true, true>(sXt, SLD, xL + (long long)k0 * B, B, kv, KC, c0, NCOL, NCOL, true);
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int u = warp + i * NET_WARPS;
          if (u < units) {
            const int mt = u / NT, nt = u % NT;
#pragma unroll
            for (int kk = 0; kk < KC; kk += 16) {
              uint32_t af[4], bf[2];
              frag_a_rowmajor(af, sWt, WLD, mt * 16, kk, lane);
              frag_b_kn(bf, sXt, SLD, kk, nt * 8, lane);
              mma<T>(acc[i], af, bf[0], bf[1]);
            }
          }
        }
        __syncthreads();
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int u = warp + i * NET_WARPS;
        if (u < units) {
          const int mt = u / NT, nt = u % NT;
          const int r = mt * 16 + gq, c = nt * 8 + 2 * tq;
          st2<T>(sMu + r * SLD + c, acc[i][0], acc[i][1]);
          st2<T>(sMu + (r + 8) * SLD + c, acc[i][2], acc[i][3]);
        }
      }
    }
    __syncthreads();

    // ---- states for the step: forward-init sweep, or the stored x ----
    auto act_rows = [&](int l) {  // a[l] = cast(f(x[l])) over the valid rows
      T* sx = sm + p.off_x[l];
      T* sa = sm + p.off_a[l];
      for (int it = threadIdx.x; it < p.dims[l] * NCOL; it += NET_THREADS) {
        const int r = it / NCOL, c = it % NCOL;
        sa[r * SLD + c] = St<T>::st(act_f<ACT>(St<T>::ld(sx[r * SLD + c])));
      }
    };
    if (p.forward_init) {
      if (L - 1 >= 1) {
        T* sx = sm + p.off_x[L - 1];
        for (int it = threadIdx.x; it < p.rows16[L - 1] * NCOL; it += NET_THREADS) {
          const int r = it / NCOL, c = it % NCOL;
          sx[r * SLD + c] = r < dTop ? sMu[r * SLD + c] : St<T>::st(0.f);
        }
        __syncthreads();
        act_rows(L - 1);
        __syncthreads();
      }
      for (int l = L - 2; l >= 1; --l) {
        constexpr int NT = NCOL / 8;
        const int mtiles = p.rows16[l] / 16;
        const int ksteps = p.rows16[l + 1] / 16;
        for (int u = warp; u < mtiles * NT; u += NET_WARPS) {
          const int mt = u / NT, nt = u % NT;
          float acc[4] = {0.f, 0.f, 0.f, 0.f};
          for (int ks = 0; ks < ksteps; ++ks) {
            uint32_t af[4], bf[2];
            frag_a_rowmajor(af, sm + p.off_w[l], WLD, mt * 16, ks * 16, lane);
            frag_b_kn(bf, sm + p.off_a[l + 1], SLD, ks * 16, nt * 8, lane);
            mma<T>(acc, af, bf[0], bf[1]);
          }
          const int r = mt * 16 + gq, c = nt * 8 + 2 * tq;
          T* sx = sm + p.off_x[l];
          const bool v0 = r < p.dims[l], v1 = r + 8 < p.dims[l];
          st2<T>(sx + r * SLD + c, v0 ? acc[0] : 0.f, v0 ? acc[1] : 0.f);
          st2<T>(sx + (r + 8) * SLD + c, v1 ? acc[2] : 0.f, v1 ? acc[3] : 0.f);
        }
        __syncthreads();
        act_rows(l);
        __syncthreads();
      }
    } else {
      for (int l = 1; l < L; ++l)
        load_block<T, ACT, false, true>(sm + p.off_x[l], SLD, gx[l], B, p.dims[l], p.rows16[l], c0, NCOL, NCOL, true);
      __syncthreads();
      for (int l = 1; l < L; ++l) act_rows(l);
      __syncthreads();
    }

    // ---- T inference iterations ----
    for (int t = 0; t < p.T_it; ++t) {
      const bool last = (t == p.T_it - 1);
      // P: e[l] = cast(x[l]) - cast(W[l] a[l+1]), l < L-1 on tensor cores
      {
        constexpr int NT = NCOL / 8;
        int base = 0;
        for (int l = 0; l < L - 1; ++l) {
          const int mtiles = p.rows16[l] / 16;
          const int ksteps = p.rows16[l + 1] / 16;
          const int units = mtiles * NT;
          // global unit index space is shared across layers for balance
          for (int u = (warp - base % NET_WARPS + NET_WARPS) % NET_WARPS; u < units; u += NET_WARPS) {
            const int mt = u / NT, nt = u % NT;
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            for (int ks = 0; ks < ksteps; ++ks) {
              uint32_t af[4], bf[2];
              frag_a_rowmajor(af, sm + p.off_w[l], WLD, mt * 16, ks * 16, lane);
              frag_b_kn(bf, sm + p.off_a[l + 1], SLD, ks * 16, nt * 8, lane);
              mma<T>(acc, af, bf[0], bf[1]);
            }
            const int r = mt * 16 + gq, c = nt * 8 + 2 * tq;
            const T* sx = sm + p.off_x[l];
            T* se = sm + p.off_e[l];
            if (r < p.dims[l])
              st2<T>(se + r * SLD + c, St<T>::ld(sx[r * SLD + c]) - rnd<T>(acc[0]),
                     St<T>::ld(sx[r * SLD + c + 1]) - rnd<T>(acc[1]));
            if (r + 8 < p.dims[l])
              st2<T>(se + (r + 8) * SLD + c, St<T>::ld(sx[(r + 8) * SLD + c]) - rnd<T>(acc[2]),
                     St<T>::ld(sx[(r + 8) * SLD + c + 1]) - rnd<T>(acc[3]));
          }
          base += units;
        }
        // top layer: the hoisted product
        {
          const T* sx = sm + p.off_x[L - 1];
          T* se = sm + p.off_e[L - 1];
          for (int it = threadIdx.x; it < dTop * NCOL; it += NET_THREADS) {
            const int r = it / NCOL, c = it % NCOL;
            se[r * SLD + c] = St<T>::st(St<T>::ld(sx[r * SLD + c]) - St<T>::ld(sMu[r * SLD + c]));
          }
        }
      }
      __syncthreads();
      // I: x[l] += g(-e[l] + f'(x[l]) (W[l-1]^T e[l-1])), l = 1..L-1
      {
        constexpr int NT = NCOL / 8;
        int base = 0;
        for (int l = 1; l < L; ++l) {
          const int mtiles = p.rows16[l] / 16;
          const int ksteps = p.rows16[l - 1] / 16;
          const int units = mtiles * NT;
          for (int u = (warp - base % NET_WARPS + NET_WARPS) % NET_WARPS; u < units; u += NET_WARPS) {
            const int mt = u / NT, nt = u % NT;
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            for (int ks = 0; ks < ksteps; ++ks) {
              uint32_t af[4], bf[2];
              frag_a_trans(af, sm + p.off_w[l - 1], WLD, mt * 16, ks * 16, lane);
              frag_b_kn(bf, sm + p.off_e[l - 1], SLD, ks * 16, nt * 8, lane);
              mma<T>(acc, af, bf[0], bf[1]);
            }
            const int rbase = mt * 16 + gq, c = nt * 8 + 2 * tq;
            T* sx = sm + p.off_x[l];
            T* sa = sm + p.off_a[l];
            const T* se = sm + p.off_e[l];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int r = rbase + 8 * h;
              if (r >= p.dims[l]) continue;
              float xn[2], an[2];
#pragma unroll
              for (int j = 0; j < 2; ++j) {
                const float xv = St<T>::ld(sx[r * SLD + c + j]);
                const float ev = St<T>::ld(se[r * SLD + c + j]);
                xn[j] = xv + p.gamma * (-ev + act_df<ACT>(xv) * acc[2 * h + j]);
                an[j] = act_f<ACT>(rnd<T>(xn[j]));  // recompute semantics: f of the stored x
              }
              st2<T>(sx + r * SLD + c, xn[0], xn[1]);
              st2<T>(sa + r * SLD + c, an[0], an[1]);
              if (last && !p.recompute && ga[l] != nullptr) {
                // save-activation variant: A_out = cast(f(x_new)) of the wide x_new (tilelang_kernels.py:231)
                T* gdst = ga[l] + (long long)r * B + c0 + c;
                st2<T>(gdst, act_f<ACT>(xn[0]), act_f<ACT>(xn[1]));
              }
            }
          }
          base += units;
        }
      }
      __syncthreads();
    }

    // ---- energy of the last iteration: sum_l mean(e[l]^2) (reference.py:58) ----
    if (p.energy != nullptr) {
      float part = 0.f;
      for (int l = 0; l < L; ++l) {
        const T* se = sm + p.off_e[l];
        float sl = 0.f;
        for (int it = threadIdx.x; it < p.dims[l] * NCOL; it += NET_THREADS) {
          const float v = St<T>::ld(se[(it / NCOL) * SLD + it % NCOL]);
          sl = fmaf(v, v, sl);
        }
        part += sl / ((float)p.dims[l] * (float)B);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
      if (lane == 0) atomicAdd(p.energy + (long long)step * p.nets + net, part);
    }

    // ---- publish states / errors (outputs; also the weight-update exchange) ----
    for (int l = 1; l < L; ++l) store_cols<T, NCOL>(gx[l], B, c0, sm + p.off_x[l], SLD, p.dims[l]);
    for (int l = 0; l < L; ++l) store_cols<T, NCOL>(ge[l], B, c0, sm + p.off_e[l], SLD, p.dims[l]);
    if (p.pool_x != nullptr && step == p.steps - 1) {
      // the trainer's x[0] / x[L] hold the batch it trained on (trainer.py:509,516)
      store_cols<T, NCOL>(gx[0], B, c0, sm + p.off_x[0], SLD, p.dims[0]);
      for (int it = threadIdx.x; it < dL * (NCOL / 8); it += NET_THREADS) {
        const int r = it / (NCOL / 8), c = (it % (NCOL / 8)) * 8;
        *reinterpret_cast<uint4*>(gx[L] + (long long)r * B + c0 + c) =
            __ldcg(reinterpret_cast<const uint4*>(xL + (long long)r * B + c0 + c));
      }
    }

    if (p.update_weights) {
      cluster_sync_all();
      // ---- weight update: W[l] += alpha * E[l] A[l+1]^T over all B columns ----
      const int ELD = p.eld;  // B + 8
      const int B16 = ((B + 15) / 16) * 16;  // columns zero-filled up to the mma K granule (<= ELD)
      T* sEx = sStage;                       // [64][ELD]  E[l] rows, all columns
      T* sAx = sStage + 64 * ELD;            // [32][ELD]  A[l+1] rows n0..n0+31, all columns
      int item = 0;
      int loaded_layer = -1;
      for (int l = 0; l < L; ++l) {
        const int Ncols = p.dims[l + 1];
        const int nblk = (Ncols + WU_COLS - 1) / WU_COLS;
        for (int blk = 0; blk < nblk; ++blk, ++item) {
          if (item % p.C != cta) continue;
          const int n0 = blk * WU_COLS;
          const int nv = min(WU_COLS, Ncols - n0);
          if (loaded_layer != l) {
            __syncthreads();
            load_block<T, ACT, false, true>(sEx, ELD, ge[l], B, p.dims[l], p.rows16[l], 0, B, B16, true);
            loaded_layer = l;
          } else {
            __syncthreads();
          }
          // A rows: f(x[l+1]) (recompute / the input layer) or the saved activation
          const bool use_saved = (!p.recompute) && (l + 1 < L) && ga[l + 1] != nullptr;
          const T* src = (l + 1 == L) ? xL : (use_saved ? ga[l + 1] : gx[l + 1]);
          if (use_saved)
            load_block<T, ACT, false, true>(sAx, ELD, src + (long long)n0 * B, B, nv, WU_COLS, 0, B, B16, true);
          else
            load_block<T, ACT, true, true>(sAx, ELD, src + (long long)n0 * B, B, nv, WU_COLS, 0, B, B16, true);
          __syncthreads();
          const int mtiles = p.rows16[l] / 16;
          const int units = mtiles * (WU_COLS / 8);
          for (int u = warp; u < units; u += NET_WARPS) {
            const int mt = u / (WU_COLS / 8), nt = u % (WU_COLS / 8);
            if (nt * 8 >= nv) continue;
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            for (int k0 = 0; k0 < B; k0 += 16) {
              uint32_t af[4], bf[2];
              frag_a_rowmajor(af, sEx, ELD, mt * 16, k0, lane);
              frag_b_nk(bf, sAx, ELD, k0, nt * 8, lane);
              mma<T>(acc, af, bf[0], bf[1]);
            }
            const int r = mt * 16 + gq, cl = nt * 8 + 2 * tq;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int m = r + 8 * h;
              if (m >= p.dims[l]) continue;
#pragma unroll
              for (int j = 0; j < 2; ++j) {
                const int n = n0 + cl + j;
                if (n - n0 >= nv) continue;
                T* wp = gw[l] + (long long)m * Ncols + n;
                *wp = St<T>::st(St<T>::ld(*wp) + p.alpha * acc[2 * h + j]);
              }
            }
          }
        }
      }
      cluster_sync_all();
      if (step + 1 < p.steps) {
        load_resident_w();
        __syncthreads();
      }
    } else {
      __syncthreads();
    }
  }
}

template <typename T, int ACT, int NCOL>
int launch_net_t(NetParams<T>& p, size_t smem, cudaStream_t s) {
  auto kern = net_kernel<T, ACT, NCOL>;
  cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err != cudaSuccess) return set_error(IPC_ERR_CUDA, "net kernel smem attribute: %s", cudaGetErrorString(err));
  if (p.C > 8) {
    err = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (err != cudaSuccess) return set_error(IPC_ERR_CUDA, "net kernel cluster attribute: %s", cudaGetErrorString(err));
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.C, p.nets, 1);
  cfg.blockDim = dim3(NET_THREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  err = cudaLaunchKernelEx(&cfg, kern, p);
  if (err != cudaSuccess) return set_error(IPC_ERR_CUDA, "net kernel launch: %s", cudaGetErrorString(err));
  count_launch();
  return check_launch("net kernel");
}

template <typename T>
int run_net(const ipc_net_t* net, const ipc_net_run_t* run, cudaStream_t s) {
  NetParams<T> p{};
  const int L = net->L;
  p.L = L;
  p.B = net->B;
  p.nets = net->nets;
  for (int l = 0; l <= L; ++l) {
    p.dims[l] = net->dims[l];
    p.rows16[l] = ((net->dims[l] + 15) / 16) * 16;
    p.x[l] = reinterpret_cast<T*>(net->x[l]);
    p.e[l] = l < L ? reinterpret_cast<T*>(net->e[l]) : nullptr;
    p.a[l] = nullptr;
  }
  for (int l = 0; l < L; ++l) p.w[l] = reinterpret_cast<T*>(net->w[l]);
  p.pool_x = reinterpret_cast<const T*>(run->pool_x);
  p.pool_y = reinterpret_cast<const T*>(run->pool_y);
  p.pool_batches = run->pool_batches;
  p.first_batch = run->first_batch;
  p.steps = run->steps;
  p.T_it = run->T;
  p.forward_init = run->forward_init;
  p.update_weights = run->update_weights;
  p.recompute = 1;
  p.alpha = run->alpha;
  p.gamma = run->gamma;
  p.energy = run->energy;

  // columns per CTA: the widest NCOL (<= 32) whose cluster fits in 8 CTAs,
  // unless the caller asked for a cluster size
  int C = run->cluster;
  if (C <= 0) {
    // prefer 16 columns per CTA, then 8, then 32, within a portable cluster (<= 8 CTAs)
    const int pref[3] = {16, 8, 32};
    C = 0;
    for (int i = 0; i < 3 && C == 0; ++i)
      if (p.B % pref[i] == 0 && p.B / pref[i] <= 8) C = p.B / pref[i];
    if (C == 0) return set_error(IPC_ERR_UNSUPPORTED, "net kernel: no cluster of <= 8 CTAs splits B=%d into 8/16/32 columns", p.B);
  }
  if (C < 1 || C > 16 || p.B % C != 0)
    return set_error(IPC_ERR_ARG, "net kernel: cluster %d does not divide B=%d", C, p.B);
  const int NCOL = p.B / C;
  if (NCOL != 8 && NCOL != 16 && NCOL != 32)
    return set_error(IPC_ERR_UNSUPPORTED, "net kernel: B/cluster = %d columns per CTA (need 8, 16 or 32)", NCOL);
  p.C = C;
  p.sld = (NCOL < 16 ? 16 : NCOL) + 8;
  p.eld = p.B + 8;

  // shared-memory layout (elements of T); every region 16-byte aligned
  int off = 0;
  auto take = [&](int elems) {
    int o = off;
    off += ((elems + 7) / 8) * 8;
    return o;
  };
  for (int l = 0; l < L - 1; ++l) p.off_w[l] = take(p.rows16[l] * WLD);
  for (int l = 0; l < L; ++l) {
    p.off_x[l] = take(p.rows16[l] * p.sld);
    p.off_a[l] = take(p.rows16[l] * p.sld);
    p.off_e[l] = take(p.rows16[l] * p.sld);
  }
  p.off_mu = take(p.rows16[L - 1] * p.sld);
  p.off_stage = off;
  const int stage_top = 64 * WLD + KC * p.sld;
  const int stage_wu = 64 * p.eld + WU_COLS * p.eld;
  off += stage_top > stage_wu ? stage_top : stage_wu;
  const size_t smem = (size_t)off * sizeof(T);
  if (smem > 227 * 1024)
    return set_error(IPC_ERR_UNSUPPORTED, "net kernel: %zu bytes of shared memory needed (> 227 KB)", smem);

  int rc = IPC_OK;
  IPC_DISPATCH_ACT(run->act, AC, {
    switch (NCOL) {
      case 8: rc = launch_net_t<T, AC, 8>(p, smem, s); break;
      case 16: rc = launch_net_t<T, AC, 16>(p, smem, s); break;
      default: rc = launch_net_t<T, AC, 32>(p, smem, s); break;
    }
  });
  return rc;
}

}  // namespace
}  // namespace ipc

using namespace ipc;

extern "C" int ipc_net_train(const ipc_net_t* net, const ipc_net_run_t* run, void* stream) {
  if (net == nullptr || run == nullptr) return set_error(IPC_ERR_ARG, "null net / run descriptor");
  const int L = net->L;
  if (L < 1 || L > IPC_NET_MAX_LAYERS) return set_error(IPC_ERR_ARG, "L=%d outside [1, %d]", L, IPC_NET_MAX_LAYERS);
  if (net->nets < 1 || net->nets > 65535) return set_error(IPC_ERR_ARG, "nets=%d outside [1, 65535]", net->nets);
  if (net->B < 8 || net->B > 256 || net->B % 8 != 0)
    return set_error(IPC_ERR_UNSUPPORTED, "net kernel: B=%d must be a multiple of 8 in [8, 256]", net->B);
  for (int l = 0; l <= L; ++l)
    if (net->dims[l] < 1) return set_error(IPC_ERR_ARG, "dims[%d]=%d", l, net->dims[l]);
  for (int l = 0; l < L; ++l)
    if (net->dims[l] > 64) return set_error(IPC_ERR_UNSUPPORTED, "net kernel: d_%d=%d > 64", l, net->dims[l]);
  for (int l = 0; l < L; ++l)
    if (!net->w[l] || !net->e[l]) return set_error(IPC_ERR_ARG, "null W / e pointer at layer %d", l);
  for (int l = 0; l <= L; ++l)
    if (!net->x[l]) return set_error(IPC_ERR_ARG, "null x pointer at layer %d", l);
  if (run->steps < 0 || run->T < 1) return set_error(IPC_ERR_ARG, "steps=%d T=%d (need steps >= 0, T >= 1)", run->steps, run->T);
  if ((run->pool_x == nullptr) != (run->pool_y == nullptr)) return set_error(IPC_ERR_ARG, "pool_x and pool_y go together");
  if (run->pool_x != nullptr && run->pool_batches < 1) return set_error(IPC_ERR_ARG, "pool_batches=%d", run->pool_batches);
  if (run->act < IPC_ACT_RELU || run->act > IPC_ACT_IDENTITY) return set_error(IPC_ERR_ARG, "unknown activation %d", run->act);
  if (run->recompute == 0) return set_error(IPC_ERR_UNSUPPORTED, "net kernel: save-activation mode not available; use recompute");
  int rc = require_sm100();
  if (rc) return rc;
  if (run->steps == 0) return IPC_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (run->energy != nullptr) {
    cudaError_t err = cudaMemsetAsync(run->energy, 0, sizeof(float) * (size_t)run->steps * net->nets, s);
    if (err != cudaSuccess) return set_error(IPC_ERR_CUDA, "energy memset: %s", cudaGetErrorString(err));
  }
  IPC_DISPATCH_DT16(run->dtype, TT, { return run_net<TT>(net, run, s); });
  return IPC_OK;
}
