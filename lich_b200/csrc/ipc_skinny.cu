// Small-batch fused GEMMs (N = B <= 16) for the prediction error P, the state
// update I and the forward sweep F -- the small-batch regime of the weight
// update specialisation (reference weight_update_specialization.py:63-128 and
// the P / I kernels it runs beside, tilelang_kernels.py:114-265).
//
// At B <= 16 these products are matrix x thin-matrix: the work is one read of
// W (M x K, 16-bit) from HBM, while the B operand (K x B: a few KB) fits in
// every CTA's shared memory.  The tiled kernel of ipc_generic.cu gives such a
// shape one CTA per 64 rows walking all of K, i.e. 16 CTAs for M = 1024.
// Here the decomposition is chosen for parallelism and a single DRAM latency:
//  * a cluster of C CTAs owns 16 output rows; CTA c reads the K slice
//    [c*ks, (c+1)*ks) and its 4 warps split that slice again, so M/16 x C
//    CTAs (about two per SM) pull W in parallel;
//  * every warp issues the A-fragment loads of four k16 steps straight from
//    global memory into registers before its first mma.sync: each 32-byte
//    sector of W is consumed whole by the fragment lanes (P / F read W rows;
//    I reads W_low columns, one 16-bit load per element);
//  * B fragments come from the CTA's shared copy of its K slice of the thin
//    operand, stored transposed ([n][k]) for the col-major mma operand, with
//    f applied while staging when the caller asks for it (recompute mode);
//  * the fp32 partials of the 4C warps go to CTA 0 over distributed shared
//    memory (stores only), one cluster barrier, and CTA 0 sums them in a fixed
//    order (deterministic) and applies the fused epilogue of the mode.
#include "ipc_common.cuh"
#include "ipc_epilogue.cuh"
#include "ipc_generic.cuh"

namespace ipc {

namespace {

constexpr int SK_WARPS = 4;
constexpr int SK_THREADS = 32 * SK_WARPS;
constexpr int SK_MAX_CLUSTER = 8;
constexpr int SK_MAX_SLICE = 4096;  // k per CTA: 16 x (4096 + 8) halves of shared memory at most
constexpr int SK_MAX_B = 16;

__device__ __forceinline__ uint32_t sk_smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint32_t sk_mapa(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void sk_st_cluster_v2(uint32_t addr, float a, float b) {
  asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(addr), "f"(a), "f"(b) : "memory");
}
__device__ __forceinline__ void sk_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t sk_cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

template <typename T>
__device__ __forceinline__ void sk_mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
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

__device__ __forceinline__ uint32_t sk_pack(uint16_t lo, uint16_t hi) { return (uint32_t)lo | ((uint32_t)hi << 16); }

// The A pair (A(m,k), A(m,k+1)) packed for an mma fragment register; zero outside the matrix.
template <typename T, int MODE>
__device__ __forceinline__ uint32_t sk_load_a(const GemmArgs& p, const T* A, int m, int k, bool vec) {
  if (m >= p.Mg || k >= p.Kg) return 0u;
  const uint16_t* a16 = reinterpret_cast<const uint16_t*>(A);
  if constexpr (MODE == MODE_I) {  // A(m,k) = W_low[k][m]
    const uint16_t lo = __ldg(a16 + (long long)k * p.lda + m);
    const uint16_t hi = (k + 1 < p.Kg) ? __ldg(a16 + (long long)(k + 1) * p.lda + m) : (uint16_t)0;
    return sk_pack(lo, hi);
  } else {  // A(m,k) = W[m][k]
    const long long off = (long long)m * p.lda + k;
    if (vec && k + 1 < p.Kg) return __ldg(reinterpret_cast<const uint32_t*>(a16 + off));
    const uint16_t lo = __ldg(a16 + off);
    const uint16_t hi = (k + 1 < p.Kg) ? __ldg(a16 + off + 1) : (uint16_t)0;
    return sk_pack(lo, hi);
  }
}

// grid (C, ceil(M/16), groups), cluster (C, 1, 1), 128 threads.
// Dynamic shared memory: red [4C][16][8*NB] fp32 (read in CTA 0), then sX [8*NB][ks + 8] of T.
template <typename T, int ACT, int MODE, bool BACT, int NB>
__global__ void __launch_bounds__(SK_THREADS) skinny_kernel(const __grid_constant__ GemmArgs p, int ks, int kw) {
  extern __shared__ __align__(16) uint8_t sk_smem[];
  constexpr int NC = 8 * NB;  // padded columns
  const int C = gridDim.x;
  const int crank = (int)sk_cluster_rank();
  const int g = blockIdx.z;
  const int m0 = blockIdx.y * 16;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gq = lane >> 2, tq = lane & 3;
  float* red = reinterpret_cast<float*>(sk_smem);
  T* sX = reinterpret_cast<T*>(sk_smem + (size_t)SK_WARPS * C * 16 * NC * sizeof(float));
  const int sld = ks + 8;
  const T* A = reinterpret_cast<const T*>(p.A) + g * p.gsA;
  const T* Bm = reinterpret_cast<const T*>(p.Bm) + g * p.gsB;
  const int k_base = crank * ks;

  // stage the K slice of the thin operand, transposed: sX[n][kl] = B(k_base + kl, n)
  for (int i = tid; i < ks * NC; i += SK_THREADS) {
    const int n = i % NC, kl = i / NC;
    const int k = k_base + kl;
    float v = 0.f;
    if (n < p.Ng && k < p.Kg) {
      v = St<T>::ld(Bm[(long long)k * p.ldb + n]);
      if constexpr (BACT) v = rnd<T>(act_f<ACT>(v));
    }
    sX[n * sld + kl] = St<T>::st(v);
  }
  __syncthreads();

  float acc[NB][4];
#pragma unroll
  for (int j = 0; j < NB; ++j)
#pragma unroll
    for (int r = 0; r < 4; ++r) acc[j][r] = 0.f;
  const bool vec = (MODE != MODE_I) && (p.lda % 2 == 0) && ((reinterpret_cast<uintptr_t>(A) & 3) == 0);
  const int kw0 = k_base + warp * kw;
  const int kw1 = min(min(kw0 + kw, k_base + ks), p.Kg);
  const int r0 = m0 + gq, r1 = m0 + gq + 8;
  for (int kb = kw0; kb < kw1; kb += 64) {
    uint32_t a[4][4];
#pragma unroll
    for (int s = 0; s < 4; ++s) {  // all loads of four k16 steps first: one DRAM latency for the group
      const int k = kb + 16 * s + 2 * tq;
      const bool in = kb + 16 * s < kw1;
      a[s][0] = in ? sk_load_a<T, MODE>(p, A, r0, k, vec) : 0u;
      a[s][1] = in ? sk_load_a<T, MODE>(p, A, r1, k, vec) : 0u;
      a[s][2] = in ? sk_load_a<T, MODE>(p, A, r0, k + 8, vec) : 0u;
      a[s][3] = in ? sk_load_a<T, MODE>(p, A, r1, k + 8, vec) : 0u;
    }
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      if (kb + 16 * s >= kw1) break;
      const int kl = kb + 16 * s - k_base + 2 * tq;  // within the staged slice (zero past K)
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        const T* col = sX + (8 * j + gq) * sld + kl;
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(col);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(col + 8);
        sk_mma<T>(acc[j], a[s], b0, b1);
      }
    }
  }

  // partials of this warp -> slot (crank * 4 + warp) of CTA 0
  const int slot = crank * SK_WARPS + warp;
  const uint32_t red0 = sk_mapa(sk_smem_addr(red), 0);
#pragma unroll
  for (int j = 0; j < NB; ++j) {
    const int c = 8 * j + 2 * tq;
    sk_st_cluster_v2(red0 + 4u * (uint32_t)((slot * 16 + gq) * NC + c), acc[j][0], acc[j][1]);
    sk_st_cluster_v2(red0 + 4u * (uint32_t)((slot * 16 + gq + 8) * NC + c), acc[j][2], acc[j][3]);
  }
  sk_cluster_sync();
  if (crank != 0) return;
  const int nslots = SK_WARPS * C;
  for (int i = tid; i < 16 * NC; i += SK_THREADS) {
    const int r = i / NC, n = i % NC;
    const int m = m0 + r;
    if (m >= p.Mg || n >= p.Ng) continue;
    float sum = 0.f;
    for (int s = 0; s < nslots; ++s) sum += red[(s * 16 + r) * NC + n];
    epilogue<T, ACT, MODE>(p, g, m, n, sum);
  }
}

template <typename T, int ACT, int MODE, bool BACT, int NB>
int launch_skinny_t(const GemmArgs& p, cudaStream_t s) {
  const int mtiles = (p.Mg + 15) / 16;
  const long long tiles = (long long)mtiles * p.groups;
  int sms = 148;
  {
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  // about two CTAs per SM, every CTA at least 64 deep in K, at most 8 per cluster
  int C = (int)((2LL * sms + tiles - 1) / tiles);
  C = max(1, min(C, SK_MAX_CLUSTER));
  C = min(C, max(1, (p.Kg + 63) / 64));
  int ks = (p.Kg + C - 1) / C;
  ks = (ks + 63) / 64 * 64;  // row stride ks + 8 halves = 4 words mod 32: conflict-free fragment reads
  while (ks > SK_MAX_SLICE && C < SK_MAX_CLUSTER) {
    ++C;
    ks = ((p.Kg + C - 1) / C + 63) / 64 * 64;
  }
  if (ks > SK_MAX_SLICE) return set_error(IPC_ERR_UNSUPPORTED, "small-batch GEMM: K=%d too deep", p.Kg);
  C = (p.Kg + ks - 1) / ks;  // no empty CTA
  const int kw = ((ks + SK_WARPS - 1) / SK_WARPS + 15) / 16 * 16;
  const size_t smem = (size_t)SK_WARPS * C * 16 * (8 * NB) * sizeof(float) + (size_t)(8 * NB) * (ks + 8) * sizeof(T);
  if (mtiles > 65535 || p.groups > 65535)
    return set_error(IPC_ERR_ARG, "small-batch GEMM grid too large (M=%d groups=%d)", p.Mg, p.groups);
  auto kern = skinny_kernel<T, ACT, MODE, BACT, NB>;
  cudaError_t err = ensure_kernel_smem<skinny_kernel<T, ACT, MODE, BACT, NB>>((int)smem);
  if (err != cudaSuccess) return set_error(IPC_ERR_CUDA, "small-batch GEMM smem attribute: %s", cudaGetErrorString(err));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(C, mtiles, p.groups);
  cfg.blockDim = dim3(SK_THREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  err = cudaLaunchKernelEx(&cfg, kern, p, ks, kw);
  if (err != cudaSuccess) return set_error(IPC_ERR_CUDA, "small-batch GEMM launch: %s", cudaGetErrorString(err));
  count_launch();
  return check_launch("small-batch GEMM");
}

template <typename T, int ACT, int MODE, bool BACT>
int launch_skinny_nb(const GemmArgs& p, cudaStream_t s) {
  return p.Ng <= 8 ? launch_skinny_t<T, ACT, MODE, BACT, 1>(p, s) : launch_skinny_t<T, ACT, MODE, BACT, 2>(p, s);
}

}  // namespace

bool skinny_eligible(int mode, int M, int K, int B, int dtype, int algo) {
  if (algo != IPC_ALGO_AUTO) return false;
  if (dtype != IPC_DT_F16 && dtype != IPC_DT_BF16) return false;
  if (mode != MODE_P && mode != MODE_I && mode != MODE_F) return false;
  return M >= 1 && B >= 1 && B <= SK_MAX_B && K >= 1 && K <= SK_MAX_CLUSTER * SK_MAX_SLICE;
}

int launch_skinny(const GemmArgs& p, int mode, bool bact, int act, int dtype, cudaStream_t s) {
  if (p.Mg <= 0 || p.Ng <= 0 || p.groups <= 0) return IPC_OK;
  IPC_DISPATCH_DT16(dtype, TT, {
    if (!bact && mode != MODE_I && !(mode == MODE_F && p.aux2 != nullptr)) {
      if (mode == MODE_P) return launch_skinny_nb<TT, IPC_ACT_IDENTITY, MODE_P, false>(p, s);
      return launch_skinny_nb<TT, IPC_ACT_IDENTITY, MODE_F, false>(p, s);
    }
    IPC_DISPATCH_ACT(act, AC, {
      switch (mode) {
        case MODE_P: return launch_skinny_nb<TT, AC, MODE_P, true>(p, s);
        case MODE_I: return launch_skinny_nb<TT, AC, MODE_I, false>(p, s);
        case MODE_F:
          return bact ? launch_skinny_nb<TT, AC, MODE_F, true>(p, s) : launch_skinny_nb<TT, AC, MODE_F, false>(p, s);
        default: return set_error(IPC_ERR_ARG, "small-batch GEMM: bad mode %d", mode);
      }
    });
  });
  return IPC_OK;
}

}  // namespace ipc
