// Persistent multi-layer iPC kernel for small widths (every width but the
// input <= 64).
//
// One launch runs `steps` whole training steps of `nets` independent networks.
// The reference spreads one iPC step over 3L-1 launches
// (src/ipc_tilelang/trainer.py:601-679) plus an eager forward-init sweep
// (trainer.py:509-516); here the forward sweep, T inference iterations and the
// weight update of every step happen inside one kernel, so launch latency --
// the cost that dominates at hidden 64 -- is paid once per launch, and the
// network state never leaves the chip between steps.
//
// Decomposition.  Network n runs on a cluster of C CTAs (C <= 8, or 16 on request).
//  * Batch columns: CTA c owns columns [c*NCOL, (c+1)*NCOL) of every state.
//    Prediction errors and state updates are column-local, so the T inference
//    iterations need only __syncthreads.
//  * Hidden weights W[l], l < L-1 (<= 64 x 64): replicated in every CTA's
//    shared memory.
//  * Input-layer weight W[L-1] (e.g. 64 x 784): split by its K columns; CTA c
//    keeps W[L-1][:, c*KS .. (c+1)*KS) stationary in shared memory for the
//    whole launch, together with f(x_L) of the same K rows for ALL batch
//    columns.  mu = W[L-1] f(x_L) is formed as C partial products that are
//    reduce-scattered over distributed shared memory (DSMEM); mu is fixed
//    for a training step (W and x_L do not change inside it), so it is
//    computed once and reused by the forward sweep and all T prediction
//    passes -- the same number the reference recomputes T+1 times.
//  * Weight update (a reduction over all B columns): every CTA *pushes* its
//    columns of e[L-1] to all CTAs and its columns of e[l], f(x[l+1]) to the
//    CTA that owns hidden layer l (l mod C); after one cluster barrier each
//    CTA updates its input-layer slice and its hidden layer(s) from local
//    shared memory and stores the new hidden weights into every replica.
//    The exchange is DSMEM stores only (no remote loads, so no round-trip
//    latency on the critical path); the next batch is prefetched with
//    cp.async while the update runs.
//  * Two cluster barriers per training step; global memory is touched only
//    for the batch (read once) and the outputs at the end of the launch.
//
// Shared-memory state tiles are [rows][NCOL] with the 16-byte chunks of each
// row XOR-swizzled by row, so ldmatrix reads of 8 consecutive rows hit 8
// distinct bank groups without padding.
//
// Tensor cores: mma.sync m16n8k16 with fp32 accumulators, fragments from
// shared memory via ldmatrix.  Every GEMM here is a handful of 16x8x16 tiles
// on a dependent chain of ~20 phases per step; register-resident fragments
// avoid the TMEM round trip tcgen05 would add to each phase.
//
// Rounding points follow the reference kernels: a = cast(f(x_stored))
// (tilelang_kernels.py:163), e = cast(x) - cast(acc) (:173),
// x = cast(x + g(-e + f'(x) acc)) (:229-230), W = cast(W + a acc) (:320), and
// the forward sweep x[l] = cast(W[l] @ f(x[l+1])) (trainer.py:513-515).
// f and f' use the MUFU approximations of ipc_common.cuh (16-bit storage).
#include <cstdio>

#include "ipc_common.cuh"

namespace ipc {
namespace {

constexpr int NET_THREADS = 512;
constexpr int NET_WARPS = NET_THREADS / 32;
constexpr int WLD = 72;  // smem row stride (elements) of replicated hidden W tiles (<= 64 cols + 8)
constexpr int MAXL = IPC_NET_MAX_LAYERS;
constexpr int MAX_CLUSTER = 16;           // above 8 CTAs the cluster is non-portable (opt-in attribute)
constexpr int MAX_PORTABLE_CLUSTER = 8;
constexpr int MAX_OWN = MAXL;  // hidden layers owned per CTA
constexpr int SMEM_LIMIT = 227 * 1024;

template <typename T>
struct NetParams {
  int L, B, nets, C, KS, KSP, nown;  // KS: input-layer K slice per CTA (multiple of 8), KSP = KS rounded to 16
  int dims[MAXL + 1];
  int rows16[MAXL + 1];
  T* w[MAXL];
  T* x[MAXL + 1];
  T* e[MAXL + 1];
  const T* pool_x;
  const T* pool_y;
  int pool_batches, first_batch, steps, T_it, forward_init, update_weights;
  float alpha, gamma;
  float* energy;
  float inv_cnt[MAXL + 1];  // 1 / (dims[l] * B): layer l's weight in the energy sum_l mean(e[l]^2)
  long long* phase_ns;
  // shared-memory layout, byte offsets
  int o_w[MAXL], o_x[MAXL], o_a[MAXL], o_e[MAXL];
  int o_ge[MAX_OWN], o_ga[MAX_OWN];
  int o_mu, o_wt, o_al, o_recv, o_gt, o_bar, o_obar, nblk;
  int wtld, ald, gld;
  int smem_bytes;
};

// ------------------------------------------------------------ PTX helpers
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t (&r)[2], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];\n" : "=r"(r[0]), "=r"(r[1]) : "r"(addr));
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

// First error a bounded wait of this kernel recorded (read by ipc_device_status).
__device__ int g_net_status = 0;
constexpr long long NET_WAIT_NS = 2000000000LL;

__device__ __forceinline__ void nbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void nbar_expect(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// The launch's abort flag: one word at the same shared-memory offset in every CTA of the cluster.  A
// bounded wait that expires raises it in all of them (remote stores); from then on no CTA issues
// another bulk copy, and before leaving each CTA lets the copies already in flight towards it land
// (bounded), so no copy reaches the shared memory of a CTA that has exited.  The outputs of such a
// launch are undefined; the status word (ipc_device_status) says IPC_ERR_TIMEOUT.
__device__ __forceinline__ void raise_abort(uint32_t flag, int C) {
  for (int r = 0; r < C; ++r) {
    uint32_t a;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(flag), "r"(r));
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(a), "r"(1u) : "memory");
  }
}
__device__ __forceinline__ bool aborted(uint32_t flag) {
  uint32_t v;
  asm volatile("ld.volatile.shared.u32 %0, [%1];" : "=r"(v) : "r"(flag) : "memory");
  return v != 0;
}
// Bounded wait on a phase of a local mbarrier; on expiry the status word is set, the abort flag is
// raised in every CTA and the caller goes on (every CTA keeps reaching every cluster barrier, so the
// launch still ends).
__device__ __forceinline__ void nbar_wait(uint32_t bar, uint32_t parity, uint32_t flag, int C) {
  long long tstart = -1;
  while (true) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return;
    long long now;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
    if (tstart < 0) tstart = now;
    if (now - tstart > NET_WAIT_NS) {
      atomicCAS(&g_net_status, 0, IPC_ERR_TIMEOUT);
      raise_abort(flag, C);
      return;
    }
  }
}
// After an abort: let copies still in flight towards this CTA complete their phase (at most 1 ms).
__device__ __forceinline__ void nbar_drain(uint32_t bar, uint32_t parity) {
  long long t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  while (true) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    long long now;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
    if (ok || now - t0 > 1000000LL) return;
  }
}
// Bulk copy of `bytes` from this CTA's shared memory to the same offset in CTA `rank`, completing
// `bytes` of the transaction count of that CTA's mbarrier `bar` (a shared::cta offset here).
__device__ __forceinline__ void bulk_to_peer(uint32_t local, uint32_t bytes, uint32_t bar, uint32_t rank) {
  uint32_t dst, rbar;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(dst) : "r"(local), "r"(rank));
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rbar) : "r"(bar), "r"(rank));
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "r"(local), "r"(bytes), "r"(rbar)
      : "memory");
}

// Bulk copy of `bytes` from this CTA's shared memory (`src`) to offset `dst` of CTA `rank`'s shared
// memory, completing `bytes` of that CTA's mbarrier `bar` (dst and bar given as local offsets).
__device__ __forceinline__ void bulk_to(uint32_t dst, uint32_t src, uint32_t bytes, uint32_t bar, uint32_t rank) {
  uint32_t rdst, rbar;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rdst) : "r"(dst), "r"(rank));
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rbar) : "r"(bar), "r"(rank));
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(rdst),
      "r"(src), "r"(bytes), "r"(rbar)
      : "memory");
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
__device__ __forceinline__ uint32_t mapa(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_dsmem_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared::cluster.v4.u32 [%0], {%1,%2,%3,%4};\n" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }
__device__ __forceinline__ long long globaltimer_ns() {
  long long t;
  asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
  return t;
}

template <typename T>
__device__ __forceinline__ uint16_t bits(float v) {
  T h = St<T>::st(v);
  return *reinterpret_cast<uint16_t*>(&h);
}
template <typename T>
__device__ __forceinline__ uint32_t bits2(float a, float b) {
  return (uint32_t)bits<T>(a) | ((uint32_t)bits<T>(b) << 16);
}
template <typename T>
__device__ __forceinline__ void unpack2(uint32_t v, float& a, float& b) {
  const uint16_t lo = v & 0xffffu, hi = v >> 16;
  a = St<T>::ld(*reinterpret_cast<const T*>(&lo));
  b = St<T>::ld(*reinterpret_cast<const T*>(&hi));
}

// ---- two storage values packed in one 32-bit register ----------------------
// Elementwise work on stored 16-bit states runs on pairs: one cvt packs two
// fp32 results, the error x - cast(acc) is one hsub2 (a single rounding of the
// exact difference; the fp32 form rounds the fp32 difference, which is the
// same value unless the operands are more than 2^13 apart), and f of a stored
// value is one MUFU op for two elements (tanh.approx.{f16x2,bf16x2}; sigmoid
// as 0.5 + 0.5 tanh(x / 2); relu as a packed max).
template <typename T>
struct Pk;
template <>
struct Pk<__half> {
  using V2 = __half2;
  static __device__ __forceinline__ V2 as(uint32_t v) { return *reinterpret_cast<const V2*>(&v); }
  static __device__ __forceinline__ uint32_t bits(V2 v) { return *reinterpret_cast<const uint32_t*>(&v); }
  static __device__ __forceinline__ uint32_t pack(float a, float b) { return bits(__floats2half2_rn(a, b)); }
  static __device__ __forceinline__ float2 unpack(uint32_t v) { return __half22float2(as(v)); }
  static __device__ __forceinline__ uint32_t sub(uint32_t x, uint32_t y) { return bits(__hsub2(as(x), as(y))); }
  static __device__ __forceinline__ uint32_t fma(uint32_t a, uint32_t b, uint32_t c) {
    return bits(__hfma2(as(a), as(b), as(c)));
  }
  static __device__ __forceinline__ uint32_t mul(uint32_t a, uint32_t b) { return bits(__hmul2(as(a), as(b))); }
  static __device__ __forceinline__ uint32_t max(uint32_t a, uint32_t b) { return bits(__hmax2(as(a), as(b))); }
  static __device__ __forceinline__ uint32_t splat(float v) { return bits(__float2half2_rn(v)); }
  static __device__ __forceinline__ uint32_t tanh(uint32_t x) {
    uint32_t r;
    asm("tanh.approx.f16x2 %0, %1;" : "=r"(r) : "r"(x));
    return r;
  }
};
template <>
struct Pk<__nv_bfloat16> {
  using V2 = __nv_bfloat162;
  static __device__ __forceinline__ V2 as(uint32_t v) { return *reinterpret_cast<const V2*>(&v); }
  static __device__ __forceinline__ uint32_t bits(V2 v) { return *reinterpret_cast<const uint32_t*>(&v); }
  static __device__ __forceinline__ uint32_t pack(float a, float b) { return bits(__floats2bfloat162_rn(a, b)); }
  static __device__ __forceinline__ float2 unpack(uint32_t v) { return __bfloat1622float2(as(v)); }
  static __device__ __forceinline__ uint32_t sub(uint32_t x, uint32_t y) { return bits(__hsub2(as(x), as(y))); }
  static __device__ __forceinline__ uint32_t fma(uint32_t a, uint32_t b, uint32_t c) {
    return bits(__hfma2(as(a), as(b), as(c)));
  }
  static __device__ __forceinline__ uint32_t mul(uint32_t a, uint32_t b) { return bits(__hmul2(as(a), as(b))); }
  static __device__ __forceinline__ uint32_t max(uint32_t a, uint32_t b) { return bits(__hmax2(as(a), as(b))); }
  static __device__ __forceinline__ uint32_t splat(float v) { return bits(__float2bfloat162_rn(v)); }
  static __device__ __forceinline__ uint32_t tanh(uint32_t x) {
    uint32_t r;
    asm("tanh.approx.bf16x2 %0, %1;" : "=r"(r) : "r"(x));
    return r;
  }
};

// f of a stored pair, packed where the activation has a packed form (else per element)
template <typename T, int ACT>
__device__ __forceinline__ uint32_t act_pair(uint32_t x) {
  if constexpr (ACT == IPC_ACT_RELU) {
    return Pk<T>::max(x, 0u);
  } else if constexpr (ACT == IPC_ACT_IDENTITY) {
    return x;
  } else {
    const float2 v = Pk<T>::unpack(x);
    return Pk<T>::pack(act_f_hw<ACT>(v.x), act_f_hw<ACT>(v.y));
  }
}

// Element offset of (row r, column c) in a swizzled [rows][NCOL] state tile:
// 16-byte chunk j of row r is stored at chunk j ^ s(r).
template <int NCOL>
__device__ __forceinline__ int sw(int r, int c) {
  constexpr int VPR = NCOL / 8;
  const int s = ((r * VPR) >> 3) & (VPR - 1);
  return r * NCOL + ((((c >> 3) ^ s)) << 3) + (c & 7);
}

// A fragment (16x16) from row-major [m][k] shared memory (ld in elements).
__device__ __forceinline__ void frag_a(uint32_t (&r)[4], uint32_t base, int ld, int m0, int k0, int lane) {
  const int q = lane >> 3, j = lane & 7;
  ldsm_x4(r, base + 2 * ((m0 + j + (q & 1) * 8) * ld + k0 + (q >> 1) * 8));
}
// A fragment (16x16) of S^T where S is row-major [k][m].
__device__ __forceinline__ void frag_a_t(uint32_t (&r)[4], uint32_t base, int ld, int m0, int k0, int lane) {
  const int q = lane >> 3, j = lane & 7;
  ldsm_x4_t(r, base + 2 * ((k0 + j + (q >> 1) * 8) * ld + m0 + (q & 1) * 8));
}
// B fragment (16x8) from row-major [k][n] (plain layout).
__device__ __forceinline__ void frag_b_kn(uint32_t (&r)[2], uint32_t base, int ld, int k0, int n0, int lane) {
  const int q = (lane >> 3) & 1, j = lane & 7;
  ldsm_x2_t(r, base + 2 * ((k0 + j + q * 8) * ld + n0));
}
// B fragment (16x8) from a swizzled state tile [k][NCOL].
template <int NCOL>
__device__ __forceinline__ void frag_b_sw(uint32_t (&r)[2], uint32_t base, int k0, int n0, int lane) {
  const int q = (lane >> 3) & 1, j = lane & 7;
  ldsm_x2_t(r, base + 2 * sw<NCOL>(k0 + j + q * 8, n0));
}
// B fragment (16x8) from row-major [n][k].
__device__ __forceinline__ void frag_b_nk(uint32_t (&r)[2], uint32_t base, int ld, int k0, int n0, int lane) {
  const int q = (lane >> 3) & 1, j = lane & 7;
  ldsm_x2(r, base + 2 * ((n0 + j) * ld + k0 + q * 8));
}
// Gathered operands of the weight update are "blocked": [k / NCOL][R rows][NCOL], block c being a
// byte copy of CTA c's swizzled state tile (row r, 8-column chunk j stored at chunk j ^ s(r)).
template <int NCOL>
__device__ __forceinline__ int blk_off(int R, int row, int k) {
  constexpr int VPR = NCOL / 8;
  const int s = ((row * VPR) >> 3) & (VPR - 1);
  return ((k / NCOL) * R + row) * NCOL + ((((k % NCOL) >> 3) ^ s) << 3);
}
// A fragment (16x16) of a blocked [m][k] operand.
template <int NCOL>
__device__ __forceinline__ void frag_a_blk(uint32_t (&r)[4], uint32_t base, int R, int m0, int k0, int lane) {
  const int q = lane >> 3, j = lane & 7;
  ldsm_x4(r, base + 2 * blk_off<NCOL>(R, m0 + j + (q & 1) * 8, k0 + (q >> 1) * 8));
}
// B fragment (16x8) of a blocked [n][k] operand.
template <int NCOL>
__device__ __forceinline__ void frag_b_blk(uint32_t (&r)[2], uint32_t base, int R, int k0, int n0, int lane) {
  const int q = (lane >> 3) & 1, j = lane & 7;
  ldsm_x2(r, base + 2 * blk_off<NCOL>(R, n0 + j, k0 + q * 8));
}

// --------------------------------------------------------- kernel helpers
// cp.async rows [0, rows) x columns [0, ncol) of a row-major global matrix
// (ld gld) into a plain shared array (ld sld); ncol multiple of 8.
template <typename T>
__device__ __forceinline__ void async_plain(uint8_t* smem, int off, int sld, const T* g, long long gld, int rows,
                                            int ncol) {
  const int vpr = ncol / 8;
  for (int it = threadIdx.x; it < rows * vpr; it += NET_THREADS) {
    const int r = it / vpr, c = (it % vpr) * 8;
    cp_async16(smem_addr(smem + off) + 2 * (r * sld + c), g + (long long)r * gld + c);
  }
}
// cp.async rows [0, rows) x the CTA's NCOL columns (starting at c0) into a swizzled state tile.
template <typename T, int NCOL>
__device__ __forceinline__ void async_state(uint8_t* smem, int off, const T* g, long long gld, int rows, int c0) {
  constexpr int VPR = NCOL / 8;
  for (int it = threadIdx.x; it < rows * VPR; it += NET_THREADS) {
    const int r = it / VPR, c = (it % VPR) * 8;
    cp_async16(smem_addr(smem + off) + 2 * sw<NCOL>(r, c), g + (long long)r * gld + c0 + c);
  }
}

template <typename T, int ACT, int NCOL, bool EN>
__global__ void __launch_bounds__(NET_THREADS, 1) net_kernel_act(const __grid_constant__ NetParams<T> p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  constexpr int NT = NCOL / 8;   // n8 tiles per CTA column block
  constexpr int VPR = NCOL / 8;  // 16-byte chunks per state row
  const int cta = blockIdx.x;    // == %cluster_ctarank: the cluster spans gridDim.x
  const int net = blockIdx.y;
  const int C = p.C;
  const int c0 = cta * NCOL;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gq = lane >> 2, tq = lane & 3;
  const int L = p.L, Lt = L - 1, B = p.B;
  const int dL = p.dims[L], dT = p.dims[Lt];
  const int B16 = ((B + 15) / 16) * 16;
  const int k_lo = cta * p.KS;
  const int kcnt = max(0, min(p.KS, dL - k_lo));  // input-layer K rows owned by this CTA
  const uint32_t sbase = smem_addr(smem);
  auto S = [&](int off) { return reinterpret_cast<T*>(smem + off); };
  auto U32 = [&](int off, int elem) -> uint32_t& { return *reinterpret_cast<uint32_t*>(smem + off + 2 * elem); };

  const bool tracer = p.phase_ns != nullptr && net == 0 && cta == 0 && threadIdx.x == 0;
  auto trace = [&](int step, int phase) {
    if (tracer && step < IPC_NET_TRACE_STEPS) p.phase_ns[step * IPC_NET_TRACE_PHASES + phase] = globaltimer_ns();
  };

  // zero everything once: padding rows / columns of every operand stay zero
  for (int i = threadIdx.x; i < p.smem_bytes / 16; i += NET_THREADS)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
  __syncthreads();

  // Hidden-weight replicas: the owner of layer l (CTA l % C) updates its own copy and bulk-copies
  // the tile to every peer; each CTA's mbarrier expects, per step, the bytes of the layers it does
  // not own, and is waited on before the replicas are next read.
  const uint32_t wbar = sbase + p.o_bar;
  uint32_t incoming = 0;
  for (int l = 0; l < Lt; ++l)
    if (l % C != cta) incoming += (uint32_t)(p.rows16[l] * WLD * (int)sizeof(T));
  // Weight-update operands: every CTA sends its e[L-1] tile to every CTA and its e[l], f(x[l+1])
  // tiles to the owner of layer l, one bulk copy each; obar expects this CTA's share per step.
  const uint32_t obar = sbase + p.o_obar;
  const uint32_t abort_flag = sbase + p.o_bar + 8;  // the 8 bytes behind wbar (zeroed with the rest)
  uint32_t operands = (uint32_t)(C * p.rows16[Lt] * NCOL * (int)sizeof(T));
  for (int slot = 0; slot < p.nown; ++slot) {
    const int l = cta + slot * C;
    if (l < Lt) operands += (uint32_t)(C * (p.rows16[l] + p.rows16[l + 1]) * NCOL * (int)sizeof(T));
  }
  if (p.update_weights && threadIdx.x == 0) {
    nbar_init(wbar, 1);
    nbar_expect(wbar, incoming);  // phase 0: the replicas of step 0
    nbar_init(obar, 1);
    nbar_expect(obar, operands);  // phase 0: the operands of step 0
  }
  __syncthreads();

  // this network's global slabs
  auto gw = [&](int l) { return p.w[l] + (long long)net * p.dims[l] * p.dims[l + 1]; };
  auto gx = [&](int l) { return p.x[l] + (long long)net * p.dims[l] * B; };
  auto ge = [&](int l) { return p.e[l] + (long long)net * p.dims[l] * B; };
  auto batch_x = [&](int step) -> const T* {
    if (p.pool_x == nullptr) return gx(L);
    const int b = (p.first_batch + step) % p.pool_batches;
    return p.pool_x + ((long long)b * p.nets + net) * (long long)dL * B;
  };
  auto batch_y = [&](int step) -> const T* {
    if (p.pool_y == nullptr) return gx(0);
    const int b = (p.first_batch + step) % p.pool_batches;
    return p.pool_y + ((long long)b * p.nets + net) * (long long)p.dims[0] * B;
  };
  // f over the owned K rows of the batch, all columns (plain [KSP][ald] tile)
  auto activate_batch = [&]() {
    for (int it = threadIdx.x; it < kcnt * (B / 2); it += NET_THREADS) {
      const int r = it / (B / 2), c = (it % (B / 2)) * 2;
      uint32_t& v = U32(p.o_al, r * p.ald + c);
      v = act_pair<T, ACT>(v);
    }
  };
  // a[l] = cast(f(x[l])) over the valid rows of the CTA's columns
  auto act_rows = [&](int l) {
    for (int it = threadIdx.x; it < p.dims[l] * (NCOL / 2); it += NET_THREADS) {
      const int r = it / (NCOL / 2), c = (it % (NCOL / 2)) * 2;
      U32(p.o_a[l], sw<NCOL>(r, c)) = act_pair<T, ACT>(U32(p.o_x[l], sw<NCOL>(r, c)));
    }
  };

  // ---- resident weights: hidden replicas and this CTA's input-layer slice ----
  for (int l = 0; l < Lt; ++l) {
    const int cols = p.dims[l + 1];
    const T* src = gw(l);
    for (int it = threadIdx.x; it < p.dims[l] * cols; it += NET_THREADS)
      S(p.o_w[l])[(it / cols) * WLD + it % cols] = src[it];
  }
  {
    const T* src = gw(Lt);
    for (int it = threadIdx.x; it < dT * kcnt; it += NET_THREADS) {
      const int r = it / kcnt, k = it % kcnt;
      S(p.o_wt)[r * p.wtld + k] = src[(long long)r * dL + k_lo + k];
    }
  }
  // ---- first batch: owned K rows of x_L (all columns), targets of the owned columns ----
  async_plain<T>(smem, p.o_al, p.ald, batch_x(0) + (long long)k_lo * B, B, kcnt, B);
  async_state<T, NCOL>(smem, p.o_x[0], batch_y(0), B, p.dims[0], c0);
  if (!p.forward_init)
    for (int l = 1; l <= Lt; ++l) async_state<T, NCOL>(smem, p.o_x[l], gx(l), B, p.dims[l], c0);
  cp_async_wait_all();
  __syncthreads();
  activate_batch();
  if (!p.forward_init)
    for (int l = 1; l <= Lt; ++l) act_rows(l);
  __syncthreads();

  const uint32_t recv_base = sbase + p.o_recv;

  for (int step = 0; step < p.steps; ++step) {
    trace(step, 0);
    if (!p.update_weights && step > 0) cluster_sync_all();  // peers done with their receive buffers

    // ---- mu partial: W[L-1][:, own K] f(x_L)[own K, all columns] -> owner CTAs ----
    {
      const int mtiles = p.rows16[Lt] / 16, ntiles = B / 8, ksteps = (kcnt + 15) / 16;
      for (int u = warp; u < mtiles * ntiles; u += NET_WARPS) {
        const int mt = u / ntiles, nt = u % ntiles;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int ks = 0; ks < ksteps; ++ks) {
          uint32_t af[4], bf[2];
          frag_a(af, sbase + p.o_wt, p.wtld, mt * 16, ks * 16, lane);
          frag_b_kn(bf, sbase + p.o_al, p.ald, ks * 16, nt * 8, lane);
          mma<T>(acc, af, bf[0], bf[1]);
        }
        // lanes tq, tq ^ 1 swap halves so each sends four consecutive columns of one row in a
        // single 16-byte store: even tq row gq, odd tq row gq + 8
        const bool odd = tq & 1;
        const float s0 = odd ? acc[0] : acc[2], s1 = odd ? acc[1] : acc[3];
        const float o0 = __shfl_xor_sync(0xffffffffu, s0, 1), o1 = __shfl_xor_sync(0xffffffffu, s1, 1);
        const int r = mt * 16 + gq + (odd ? 8 : 0), n = nt * 8 + 2 * (tq & ~1);
        const int owner = n / NCOL, lc = n % NCOL;
        const uint32_t dst = mapa(recv_base + 4 * ((cta * p.rows16[Lt] + r) * NCOL + lc), owner);
        const uint4 v = odd ? make_uint4(__float_as_uint(o0), __float_as_uint(o1), __float_as_uint(acc[2]),
                                         __float_as_uint(acc[3]))
                            : make_uint4(__float_as_uint(acc[0]), __float_as_uint(acc[1]), __float_as_uint(o0),
                                         __float_as_uint(o1));
        st_dsmem_v4(dst, v);
      }
    }
    trace(step, 1);
    cluster_sync_all();  // (A) partials delivered; every peer finished with last step's pushes / broadcasts
    trace(step, 2);

    // ---- mu for the owned columns: sum of the C partials in a fixed order ----
    for (int it = threadIdx.x; it < p.rows16[Lt] * (NCOL / 2); it += NET_THREADS) {
      const int r = it / (NCOL / 2), j = (it % (NCOL / 2)) * 2;
      float s0 = 0.f, s1 = 0.f;
      for (int cc = 0; cc < C; ++cc) {
        const float2 v = reinterpret_cast<const float2*>(smem + p.o_recv)[((cc * p.rows16[Lt] + r) * NCOL + j) / 2];
        s0 += v.x;
        s1 += v.y;
      }
      U32(p.o_mu, sw<NCOL>(r, j)) = r < dT ? bits2<T>(s0, s1) : 0u;
    }
    if (p.update_weights && step > 0 && threadIdx.x == 0) {
      nbar_wait(wbar, (uint32_t)((step - 1) & 1), abort_flag, C);  // last step's replicas have landed
      nbar_expect(wbar, incoming);                  // this step's
    }
    __syncthreads();
    trace(step, 3);

    // ---- forward-init sweep: x[L-1] = cast(mu), x[l] = cast(W[l] f(x[l+1])) ----
    if (p.forward_init) {
      if (Lt >= 1) {
        for (int it = threadIdx.x; it < dT * (NCOL / 2); it += NET_THREADS) {
          const int r = it / (NCOL / 2), c = (it % (NCOL / 2)) * 2;
          const uint32_t v = U32(p.o_mu, sw<NCOL>(r, c));
          U32(p.o_x[Lt], sw<NCOL>(r, c)) = v;
          U32(p.o_a[Lt], sw<NCOL>(r, c)) = act_pair<T, ACT>(v);
        }
        __syncthreads();
      }
      for (int l = Lt - 1; l >= 1; --l) {
        const int mtiles = p.rows16[l] / 16, ksteps = p.rows16[l + 1] / 16;
        for (int u = warp; u < mtiles * NT; u += NET_WARPS) {
          const int mt = u / NT, nt = u % NT;
          float acc[4] = {0.f, 0.f, 0.f, 0.f};
          for (int ks = 0; ks < ksteps; ++ks) {
            uint32_t af[4], bf[2];
            frag_a(af, sbase + p.o_w[l], WLD, mt * 16, ks * 16, lane);
            frag_b_sw<NCOL>(bf, sbase + p.o_a[l + 1], ks * 16, nt * 8, lane);
            mma<T>(acc, af, bf[0], bf[1]);
          }
          const int c = nt * 8 + 2 * tq;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int rr = mt * 16 + gq + 8 * h;
            if (rr >= p.dims[l]) continue;
            const uint32_t xs = Pk<T>::pack(acc[2 * h], acc[2 * h + 1]);
            U32(p.o_x[l], sw<NCOL>(rr, c)) = xs;
            U32(p.o_a[l], sw<NCOL>(rr, c)) = act_pair<T, ACT>(xs);
          }
        }
        __syncthreads();
      }
    }
    trace(step, 4);

    // ---- T inference iterations ----
    // the energy of the last iteration accumulates in the P phase where each e is produced (a second pass
    // over the e tiles after the iterations cost ~2.8 us of a 25 us step at configs[1])
    float esq = 0.f;
    for (int t = 0; t < p.T_it; ++t) {
      const bool want_e = EN && t == p.T_it - 1;  // EN: a launch that reports energy
      // P: e[l] = cast(x[l]) - cast(W[l] f(x[l+1])), l < L-1 on tensor cores; the input layer uses mu
      {
        int base = 0;
#pragma unroll
        for (int l = 0; l < MAXL; ++l) {  // unrolled: the per-layer offsets become constant-bank operands
          if (l >= Lt) break;
          const int mtiles = p.rows16[l] / 16, ksteps = p.rows16[l + 1] / 16, units = mtiles * NT;
          for (int u = (warp - base % NET_WARPS + NET_WARPS) % NET_WARPS; u < units; u += NET_WARPS) {
            const int mt = u / NT, nt = u % NT;
            // all fragments first, then two accumulator chains (even / odd k steps): the legacy
            // mma.sync latency, not its throughput, bounds these reductions of at most 4 steps
            // (every width the kernel accepts is <= 64, checked at launch)
            float acc[4] = {0.f, 0.f, 0.f, 0.f}, acc2[4] = {0.f, 0.f, 0.f, 0.f};
            uint32_t af[4][4], bf[4][2];
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              if (ks < ksteps) {
                frag_a(af[ks], sbase + p.o_w[l], WLD, mt * 16, ks * 16, lane);
                frag_b_sw<NCOL>(bf[ks], sbase + p.o_a[l + 1], ks * 16, nt * 8, lane);
              }
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              if (ks < ksteps) mma<T>((ks & 1) ? acc2 : acc, af[ks], bf[ks][0], bf[ks][1]);
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[j] += acc2[j];
            const int c = nt * 8 + 2 * tq;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int rr = mt * 16 + gq + 8 * h;
              if (rr >= p.dims[l]) continue;
              const int i = sw<NCOL>(rr, c);
              const uint32_t ev = Pk<T>::sub(U32(p.o_x[l], i), Pk<T>::pack(acc[2 * h], acc[2 * h + 1]));
              U32(p.o_e[l], i) = ev;
              if (want_e) {
                const float2 f = Pk<T>::unpack(ev);
                esq = fmaf(fmaf(f.x, f.x, f.y * f.y), p.inv_cnt[l], esq);
              }
            }
          }
          base += units;
        }
        for (int it = threadIdx.x; it < dT * (NCOL / 2); it += NET_THREADS) {
          const int r = it / (NCOL / 2), c = (it % (NCOL / 2)) * 2;
          const int i = sw<NCOL>(r, c);
          const uint32_t ev = Pk<T>::sub(U32(p.o_x[Lt], i), U32(p.o_mu, i));
          U32(p.o_e[Lt], i) = ev;
          if (want_e) {
            const float2 f = Pk<T>::unpack(ev);
            esq = fmaf(fmaf(f.x, f.x, f.y * f.y), p.inv_cnt[Lt], esq);
          }
        }
      }
      __syncthreads();
      // I: x[l] += g(-e[l] + f'(x[l]) (W[l-1]^T e[l-1])), l = 1..L-1
      {
        int base = 0;
#pragma unroll
        for (int l = 1; l <= MAXL; ++l) {
          if (l > Lt) break;
          const int mtiles = p.rows16[l] / 16, ksteps = p.rows16[l - 1] / 16, units = mtiles * NT;
          for (int u = (warp - base % NET_WARPS + NET_WARPS) % NET_WARPS; u < units; u += NET_WARPS) {
            const int mt = u / NT, nt = u % NT;
            float acc[4] = {0.f, 0.f, 0.f, 0.f}, acc2[4] = {0.f, 0.f, 0.f, 0.f};
            uint32_t af[4][4], bf[4][2];
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              if (ks < ksteps) {
                frag_a_t(af[ks], sbase + p.o_w[l - 1], WLD, mt * 16, ks * 16, lane);
                frag_b_sw<NCOL>(bf[ks], sbase + p.o_e[l - 1], ks * 16, nt * 8, lane);
              }
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              if (ks < ksteps) mma<T>((ks & 1) ? acc2 : acc, af[ks], bf[ks][0], bf[ks][1]);
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[j] += acc2[j];
            const int c = nt * 8 + 2 * tq;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int rr = mt * 16 + gq + 8 * h;
              if (rr >= p.dims[l]) continue;
              const int i = sw<NCOL>(rr, c);
              const float2 xv = Pk<T>::unpack(U32(p.o_x[l], i));
              const float2 ev = Pk<T>::unpack(U32(p.o_e[l], i));
              const uint32_t xs = Pk<T>::pack(xv.x + p.gamma * (-ev.x + act_df_hw<ACT>(xv.x) * acc[2 * h]),
                                              xv.y + p.gamma * (-ev.y + act_df_hw<ACT>(xv.y) * acc[2 * h + 1]));
              U32(p.o_x[l], i) = xs;
              U32(p.o_a[l], i) = act_pair<T, ACT>(xs);
            }
          }
          base += units;
        }
      }
      __syncthreads();
    }
    trace(step, 5);

    // ---- energy of the last iteration: sum_l mean(e[l]^2) (reference.py:58) ----
    if constexpr (EN) {
      float part = esq;  // this thread's e^2 of the last iteration, each weighted 1 / (dims[l] * B)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
      if (lane == 0) atomicAdd(p.energy + (long long)step * p.nets + net, part);
    }
    trace(step, 6);

    const bool more = step + 1 < p.steps;
    if (p.update_weights) {
      // ---- send the weight-update operands: one bulk copy per tile and destination ----
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the state tiles, to the copy engine
      __syncthreads();
      if (threadIdx.x == 0 && !aborted(abort_flag)) {
        const uint32_t top = (uint32_t)(p.rows16[Lt] * NCOL * (int)sizeof(T));
        for (int cc = 0; cc < C; ++cc)  // e[L-1] -> every CTA's E_top, block cta
          bulk_to(sbase + p.o_gt + (uint32_t)cta * top, sbase + p.o_e[Lt], top, obar, (uint32_t)cc);
        const uint32_t blk = (uint32_t)(64 * NCOL * (int)sizeof(T));
        for (int l = 0; l < Lt; ++l) {  // e[l], f(x[l+1]) -> the owner of layer l, block cta
          const uint32_t owner = (uint32_t)(l % C), slot = (uint32_t)(l / C);
          bulk_to(sbase + p.o_ge[slot] + (uint32_t)cta * blk, sbase + p.o_e[l],
                  (uint32_t)(p.rows16[l] * NCOL * (int)sizeof(T)), obar, owner);
          bulk_to(sbase + p.o_ga[slot] + (uint32_t)cta * blk, sbase + p.o_a[l + 1],
                  (uint32_t)(p.rows16[l + 1] * NCOL * (int)sizeof(T)), obar, owner);
        }
      }
      if (threadIdx.x == 0) {
        // (B) this CTA's update operands have arrived: every peer finished its iterations
        nbar_wait(obar, (uint32_t)(step & 1), abort_flag, C);
        nbar_expect(obar, operands);  // the next step's
      }
      __syncthreads();
      trace(step, 7);
      // ---- input layer: W[L-1][:, own K] += alpha E[L-1] f(x_L)^T (local slice) ----
      {
        const int mtiles = p.rows16[Lt] / 16, ntiles = p.KSP / 8;
        for (int u = warp; u < mtiles * ntiles; u += NET_WARPS) {
          const int mt = u / ntiles, nt = u % ntiles;
          if (nt * 8 >= kcnt) continue;
          float acc[4] = {0.f, 0.f, 0.f, 0.f};
          for (int b0 = 0; b0 < B16; b0 += 16) {
            uint32_t af[4], bf[2];
            frag_a_blk<NCOL>(af, sbase + p.o_gt, p.rows16[Lt], mt * 16, b0, lane);
            frag_b_nk(bf, sbase + p.o_al, p.ald, b0, nt * 8, lane);
            mma<T>(acc, af, bf[0], bf[1]);
          }
          const int k = nt * 8 + 2 * tq;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int rr = mt * 16 + gq + 8 * h;
            if (rr >= dT) continue;
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              if (k + j >= kcnt) continue;
              T& wv = S(p.o_wt)[rr * p.wtld + k + j];
              wv = St<T>::st(St<T>::ld(wv) + p.alpha * acc[2 * h + j]);
            }
          }
        }
      }
      __syncthreads();  // f(x_L) of this step no longer needed
      trace(step, 8);
      if (more) {
        async_plain<T>(smem, p.o_al, p.ald, batch_x(step + 1) + (long long)k_lo * B, B, kcnt, B);
        async_state<T, NCOL>(smem, p.o_x[0], batch_y(step + 1), B, p.dims[0], c0);
      }
      // ---- owned hidden layers: full reduction over B, new tiles stored into every replica ----
      for (int slot = 0; slot < p.nown; ++slot) {
        const int l = cta + slot * C;
        if (l >= Lt) break;
        const int cols = p.dims[l + 1];
        const int mtl = p.rows16[l] / 16, ntl = p.rows16[l + 1] / 8;
        for (int u = warp; u < mtl * ntl; u += NET_WARPS) {
          const int mt = u / ntl, nt = u % ntl;
          float acc[4] = {0.f, 0.f, 0.f, 0.f};
          for (int b0 = 0; b0 < B16; b0 += 16) {
            uint32_t af[4], bf[2];
            frag_a_blk<NCOL>(af, sbase + p.o_ge[slot], 64, mt * 16, b0, lane);
            frag_b_blk<NCOL>(bf, sbase + p.o_ga[slot], 64, b0, nt * 8, lane);
            mma<T>(acc, af, bf[0], bf[1]);
          }
          const int n = nt * 8 + 2 * tq;
          if (cols % 8 == 0) {
            // whole 8-column segments: the 4 lanes of a row gather their pairs so one lane per row
            // pushes the segment to every replica as a single 16-byte store
            uint32_t v[2] = {0u, 0u};
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int rr = mt * 16 + gq + 8 * h;
              if (rr < p.dims[l] && n < cols) {
                float w0, w1;
                unpack2<T>(U32(p.o_w[l], rr * WLD + n), w0, w1);
                v[h] = bits2<T>(w0 + p.alpha * acc[2 * h], w1 + p.alpha * acc[2 * h + 1]);
              }
            }
            uint32_t seg[4];
            const int h = tq & 1;  // tq 0 pushes row gq, tq 1 row gq + 8
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t a0 = __shfl_sync(0xffffffffu, v[0], gq * 4 + j);
              const uint32_t a1 = __shfl_sync(0xffffffffu, v[1], gq * 4 + j);
              seg[j] = h ? a1 : a0;
            }
            const int rr = mt * 16 + gq + 8 * h;
            if (tq < 2 && rr < p.dims[l] && nt * 8 < cols)
              *reinterpret_cast<uint4*>(smem + p.o_w[l] + 2 * (rr * WLD + nt * 8)) =
                  make_uint4(seg[0], seg[1], seg[2], seg[3]);
          } else {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int rr = mt * 16 + gq + 8 * h;
              if (rr >= p.dims[l] || n >= cols) continue;
              const int idx = rr * WLD + n;
              if (n + 1 < cols) {
                float w0, w1;
                unpack2<T>(U32(p.o_w[l], idx), w0, w1);
                U32(p.o_w[l], idx) = bits2<T>(w0 + p.alpha * acc[2 * h], w1 + p.alpha * acc[2 * h + 1]);
              } else {
                S(p.o_w[l])[idx] = St<T>::st(St<T>::ld(S(p.o_w[l])[idx]) + p.alpha * acc[2 * h]);
              }
            }
          }
        }
      }
      // the new tiles of the owned layers go to every peer as one bulk copy each (the copy engine
      // reads them after the generic stores above are made visible to the async proxy)
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncthreads();
      if (threadIdx.x == 0 && !aborted(abort_flag)) {
        for (int slot = 0; slot < p.nown; ++slot) {
          const int l = cta + slot * C;
          if (l >= Lt) break;
          const uint32_t bytes = (uint32_t)(p.rows16[l] * WLD * (int)sizeof(T));
          for (int cc = 0; cc < C; ++cc)
            if (cc != cta) bulk_to_peer(sbase + p.o_w[l], bytes, wbar, (uint32_t)cc);
        }
      }
      trace(step, 9);
      if (more) {
        cp_async_wait_all();
        __syncthreads();
        activate_batch();
      }
      __syncthreads();
      trace(step, 10);
    } else if (more) {
      async_plain<T>(smem, p.o_al, p.ald, batch_x(step + 1) + (long long)k_lo * B, B, kcnt, B);
      async_state<T, NCOL>(smem, p.o_x[0], batch_y(step + 1), B, p.dims[0], c0);
      cp_async_wait_all();
      __syncthreads();
      activate_batch();
      __syncthreads();
    }
    trace(step, 11);
  }

  // ---- outputs: states / errors of the owned columns, weights, the trained batch ----
  if (p.update_weights) {
    if (p.steps > 0 && threadIdx.x == 0) nbar_wait(wbar, (uint32_t)((p.steps - 1) & 1), abort_flag, C);
    if (threadIdx.x == 0 && aborted(abort_flag)) {
      // copies already issued towards this CTA land before it leaves (their phases may be the current or
      // the next one; both are drained, each bounded)
      nbar_drain(wbar, 0u);
      nbar_drain(wbar, 1u);
      nbar_drain(obar, 0u);
      nbar_drain(obar, 1u);
    }
    __syncthreads();
    cluster_sync_all();  // every replica holds every owner's new tiles; no copy is still in flight
    if (cta == 0) {
      for (int l = 0; l < Lt; ++l) {
        const int cols = p.dims[l + 1];
        T* dst = gw(l);
        for (int it = threadIdx.x; it < p.dims[l] * cols; it += NET_THREADS)
          dst[it] = S(p.o_w[l])[(it / cols) * WLD + it % cols];
      }
    }
    T* dst = gw(Lt);
    for (int it = threadIdx.x; it < dT * kcnt; it += NET_THREADS) {
      const int r = it / kcnt, k = it % kcnt;
      dst[(long long)r * dL + k_lo + k] = S(p.o_wt)[r * p.wtld + k];
    }
  }
  for (int l = 0; l <= Lt; ++l) {
    const bool write_x = (l >= 1) || (p.pool_y != nullptr);
    for (int it = threadIdx.x; it < p.dims[l] * VPR; it += NET_THREADS) {
      const int r = it / VPR, c = (it % VPR) * 8;
      const int i = sw<NCOL>(r, c);
      if (write_x)
        *reinterpret_cast<uint4*>(gx(l) + (long long)r * B + c0 + c) = *reinterpret_cast<const uint4*>(S(p.o_x[l]) + i);
      *reinterpret_cast<uint4*>(ge(l) + (long long)r * B + c0 + c) = *reinterpret_cast<const uint4*>(S(p.o_e[l]) + i);
    }
  }
  if (p.pool_x != nullptr) {  // the trainer's x[L] holds the batch it trained on (trainer.py:509)
    const T* src = batch_x(p.steps - 1);
    for (int it = threadIdx.x; it < dL * VPR; it += NET_THREADS) {
      const int r = it / VPR, c = (it % VPR) * 8;
      *reinterpret_cast<uint4*>(gx(L) + (long long)r * B + c0 + c) =
          *reinterpret_cast<const uint4*>(src + (long long)r * B + c0 + c);
    }
  }
}

// ------------------------------------------------------------------- host
template <typename T>
int make_layout(NetParams<T>& p, int C, int NCOL) {
  const int L = p.L, Lt = L - 1;
  p.C = C;
  p.KS = ((p.dims[L] + C - 1) / C + 7) / 8 * 8;
  p.KSP = (p.KS + 15) / 16 * 16;
  p.wtld = p.KSP + 8;
  p.ald = ((p.B + 15) / 16) * 16 + 8;
  p.gld = p.ald;
  p.nown = Lt > 0 ? (Lt + C - 1) / C : 0;
  int off = 0;
  auto take = [&](int bytes) {
    int o = off;
    off += (bytes + 127) / 128 * 128;
    return o;
  };
  const int es = (int)sizeof(T);
  for (int l = 0; l < Lt; ++l) p.o_w[l] = take(p.rows16[l] * WLD * es);
  for (int l = 0; l <= Lt; ++l) {
    p.o_x[l] = take(p.rows16[l] * NCOL * es);
    p.o_a[l] = take(p.rows16[l] * NCOL * es);
    p.o_e[l] = take(p.rows16[l] * NCOL * es);
  }
  p.o_mu = take(p.rows16[Lt] * NCOL * es);
  p.o_wt = take(p.rows16[Lt] * p.wtld * es);
  p.o_al = take(p.KSP * p.ald * es);
  p.o_recv = take(C * p.rows16[Lt] * NCOL * 4);
  // gathered weight-update operands, one block per source CTA plus zero blocks up to B rounded to 16
  p.nblk = ((p.B + 15) / 16 * 16) / NCOL;
  p.o_gt = take(p.nblk * p.rows16[Lt] * NCOL * es);
  p.o_bar = take(16);   // mbarrier counting the hidden-weight replicas arriving from their owners
  p.o_obar = take(16);  // mbarrier counting the gathered operands of this CTA's updates
  for (int s = 0; s < p.nown; ++s) {
    p.o_ge[s] = take(p.nblk * 64 * NCOL * es);
    p.o_ga[s] = take(p.nblk * 64 * NCOL * es);
  }
  p.smem_bytes = off;
  return off;
}

// Pick columns per CTA and the cluster size whose layout fits in shared memory.  One network
// per launch is latency-bound, so it is spread over as many SMs as a cluster can have (8
// columns per CTA, up to 16 CTAs: a non-portable cluster; 29.8 vs 34.1 us per configs[1]
// depth-6 step); many networks are throughput-bound and keep portable clusters of <= 8 CTAs
// with 16 columns each.  `want` > 0 forces the cluster size (up to 16).
template <typename T>
int choose_plan(NetParams<T>& p, int want, int* ncol_out) {
  const bool one = p.nets == 1 && want == 0;
  const int pref_one[3] = {8, 16, 32}, pref_many[3] = {16, 8, 32};
  const int* pref = one ? pref_one : pref_many;
  for (int i = 0; i < 3; ++i) {
    const int ncol = pref[i];
    if (p.B % ncol != 0) continue;
    const int C = p.B / ncol;
    const int cmax = (want > 0 || one) ? MAX_CLUSTER : MAX_PORTABLE_CLUSTER;
    if (C > cmax || (want > 0 && C != want)) continue;
    if (make_layout(p, C, ncol) <= SMEM_LIMIT) {
      *ncol_out = ncol;
      return IPC_OK;
    }
  }
  return set_error(IPC_ERR_UNSUPPORTED,
                   "net kernel: no cluster of <= 8 (16 on request) CTAs with 8/16/32 columns each fits B=%d%s in "
                   "shared memory", p.B,
                   want > 0 ? " with the requested cluster size" : "");
}

template <typename T, int ACT, int NCOL, bool EN>
int launch_net_t(NetParams<T>& p, cudaStream_t s) {
  auto kern = net_kernel_act<T, ACT, NCOL, EN>;
  cudaError_t err = ensure_kernel_smem<net_kernel_act<T, ACT, NCOL, EN>>(p.smem_bytes, p.C > MAX_PORTABLE_CLUSTER);
  if (err != cudaSuccess) return set_error(IPC_ERR_CUDA, "net kernel smem attribute: %s", cudaGetErrorString(err));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.C, p.nets, 1);
  cfg.blockDim = dim3(NET_THREADS, 1, 1);
  cfg.dynamicSmemBytes = p.smem_bytes;
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
void fill_params(NetParams<T>& p, const ipc_net_t* net) {
  p = NetParams<T>{};
  p.L = net->L;
  p.B = net->B;
  p.nets = net->nets;
  for (int l = 0; l <= net->L; ++l) {
    p.dims[l] = net->dims[l];
    p.rows16[l] = ((net->dims[l] + 15) / 16) * 16;
    p.x[l] = reinterpret_cast<T*>(net->x[l]);
    p.e[l] = l < net->L ? reinterpret_cast<T*>(net->e[l]) : nullptr;
  }
  for (int l = 0; l < net->L; ++l) p.w[l] = reinterpret_cast<T*>(net->w[l]);
}

template <typename T>
int run_net(const ipc_net_t* net, const ipc_net_run_t* run, cudaStream_t s) {
  NetParams<T> p;
  fill_params(p, net);
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
  for (int l = 0; l <= p.L; ++l) p.inv_cnt[l] = 1.f / ((float)p.dims[l] * (float)p.B);
  p.phase_ns = run->phase_ns;
  int ncol = 0;
  int rc = choose_plan(p, run->cluster, &ncol);
  if (rc) return rc;
  IPC_DISPATCH_ACT(run->act, AC, {
    switch (ncol) {
      case 8: rc = p.energy ? launch_net_t<T, AC, 8, true>(p, s) : launch_net_t<T, AC, 8, false>(p, s); break;
      case 16: rc = p.energy ? launch_net_t<T, AC, 16, true>(p, s) : launch_net_t<T, AC, 16, false>(p, s); break;
      default: rc = p.energy ? launch_net_t<T, AC, 32, true>(p, s) : launch_net_t<T, AC, 32, false>(p, s); break;
    }
  });
  return rc;
}

int check_net(const ipc_net_t* net) {
  if (net == nullptr) return set_error(IPC_ERR_ARG, "null net descriptor");
  const int L = net->L;
  if (L < 1 || L > IPC_NET_MAX_LAYERS) return set_error(IPC_ERR_ARG, "L=%d outside [1, %d]", L, IPC_NET_MAX_LAYERS);
  if (net->nets < 1 || net->nets > 65535) return set_error(IPC_ERR_ARG, "nets=%d outside [1, 65535]", net->nets);
  if (net->B < 8 || net->B > 256 || net->B % 8 != 0)
    return set_error(IPC_ERR_UNSUPPORTED, "net kernel: B=%d must be a multiple of 8 in [8, 256]", net->B);
  for (int l = 0; l <= L; ++l)
    if (net->dims[l] < 1) return set_error(IPC_ERR_ARG, "dims[%d]=%d", l, net->dims[l]);
  if (net->dims[L] % 8 != 0)
    return set_error(IPC_ERR_UNSUPPORTED, "net kernel: input width %d must be a multiple of 8", net->dims[L]);
  for (int l = 0; l < L; ++l)
    if (net->dims[l] > 64) return set_error(IPC_ERR_UNSUPPORTED, "net kernel: d_%d=%d > 64", l, net->dims[l]);
  return IPC_OK;
}

}  // namespace
}  // namespace ipc

using namespace ipc;

namespace ipc {
// The wide small-batch step kernel (ipc_widenet.cu): networks the cluster kernel cannot hold.
bool wide_net_fits(const ipc_net_t* net);
int wide_net_smem(const ipc_net_t* net);
int wide_net_train(const ipc_net_t* net, const ipc_net_run_t* run, cudaStream_t s);
}  // namespace ipc

namespace ipc {
int read_net_status(int* status, int clear) {
  int v = 0;
  cudaError_t err = cudaMemcpyFromSymbol(&v, g_net_status, sizeof(int));
  if (err != cudaSuccess) return set_error(IPC_ERR_CUDA, "device status read: %s", cudaGetErrorString(err));
  if (clear && v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_net_status, &zero, sizeof(int));
  }
  if (status) *status = v;
  return IPC_OK;
}
}  // namespace ipc

extern "C" int ipc_net_plan(const ipc_net_t* net, int cluster, int* cluster_out, int* smem_bytes_out) {
  int rc = check_net(net);
  if (rc == IPC_ERR_UNSUPPORTED && wide_net_fits(net)) {
    if (cluster_out) *cluster_out = 0;  // one cooperative grid per network
    if (smem_bytes_out) *smem_bytes_out = wide_net_smem(net);
    return IPC_OK;
  }
  if (rc) return rc;
  NetParams<__half> p;
  fill_params(p, net);
  int ncol = 0;
  rc = choose_plan(p, cluster, &ncol);
  if (rc) return rc;
  if (cluster_out) *cluster_out = p.C;
  if (smem_bytes_out) *smem_bytes_out = p.smem_bytes;
  return IPC_OK;
}

extern "C" int ipc_net_train(const ipc_net_t* net, const ipc_net_run_t* run, void* stream) {
  if (net == nullptr || run == nullptr) return set_error(IPC_ERR_ARG, "null net / run descriptor");
  int rc = check_net(net);
  const bool wide = (rc == IPC_ERR_UNSUPPORTED && wide_net_fits(net));
  if (wide) rc = IPC_OK;
  if (rc) return rc;
  const int L = net->L;
  for (int l = 0; l < L; ++l)
    if (!net->w[l] || !net->e[l]) return set_error(IPC_ERR_ARG, "null W / e pointer at layer %d", l);
  for (int l = 0; l <= L; ++l)
    if (!net->x[l]) return set_error(IPC_ERR_ARG, "null x pointer at layer %d", l);
  if (run->steps < 0 || run->T < 1)
    return set_error(IPC_ERR_ARG, "steps=%d T=%d (need steps >= 0, T >= 1)", run->steps, run->T);
  if ((run->pool_x == nullptr) != (run->pool_y == nullptr)) return set_error(IPC_ERR_ARG, "pool_x and pool_y go together");
  if (run->pool_x != nullptr && run->pool_batches < 1) return set_error(IPC_ERR_ARG, "pool_batches=%d", run->pool_batches);
  if (run->act < IPC_ACT_RELU || run->act > IPC_ACT_IDENTITY) return set_error(IPC_ERR_ARG, "unknown activation %d", run->act);
  if (run->recompute == 0)
    return set_error(IPC_ERR_UNSUPPORTED, "net kernel: save-activation mode not available; use recompute");
  rc = require_sm100();
  if (rc) return rc;
  if (run->steps == 0) return IPC_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (run->energy != nullptr) {
    cudaError_t err = cudaMemsetAsync(run->energy, 0, sizeof(float) * (size_t)run->steps * net->nets, s);
    if (err != cudaSuccess) return set_error(IPC_ERR_CUDA, "energy memset: %s", cudaGetErrorString(err));
  }
  if (wide) return wide_net_train(net, run, s);
  IPC_DISPATCH_DT16(run->dtype, TT, { return run_net<TT>(net, run, s); });
  return IPC_OK;
}
