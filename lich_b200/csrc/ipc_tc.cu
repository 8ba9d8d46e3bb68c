// tcgen05 / TMEM / TMA tensor-core kernel for the fused P / I / W / forward
// GEMMs of wide layers (16-bit storage, fp32 accumulation).
//
// One persistent CTA per SM walks the output tiles (128 x BN, BN = 256 or
// 128).  Warp roles:
//   warp 0      TMA producer: a 4-stage ring of 64-deep K blocks, 128-byte
//               swizzled tiles loaded with cp.async.bulk.tensor (no multicast).
//   warp 1      TMEM owner and MMA issuer: one thread issues
//               tcgen05.mma.cta_group::1.kind::f16 (M = 128, N = BN, K = 16)
//               into one of two TMEM accumulators (2 x BN fp32 columns);
//               tcgen05.commit releases smem stages / publishes accumulators.
//   warps 2..9  epilogue: tcgen05.ld of the accumulator rows (thread = row),
//               the mode's fused element-wise epilogue; the second
//               accumulator lets the next tile's MMAs run meanwhile.  Two
//               warps share each TMEM lane quarter (warp % 4), one per half
//               of the BN accumulator columns.  P and W read their in/out
//               operand (X_lo, W) with coalesced loads a tile ahead and pass
//               it through a shared-memory transpose buffer (the row threads
//               update it in place; coalesced stores write it back); I stages
//               E and X with TMA loads and writes X / A_out with TMA stores.
//               Either way a warp instruction moves whole 128-byte lines:
//               row-per-thread global accesses would split it into 32
//               requests.  F, dW (WD) and split-K partials store directly.
// All 32 lanes of warps 0 and 1 walk their loops (so the final CTA barrier is
// reached convergently); lane 0 alone issues TMA, MMA and commits.
// Operand orientation per mode (UMMA "K-major" = reduction dim contiguous):
//   P, F : A = W [M, K]          K-major    B = A_up [K, N]        MN-major
//   I    : A = W_low [K, M]      MN-major   B = E_low [K, N]       MN-major
//   W, WD: A = E [M, Bt]         K-major    B = A_up [Kw, Bt]      K-major
// The B operand is taken as stored (a saved activation): applying f inside
// the GEMM would repeat it M/128 times per element; callers materialise
// f(X) once (ipc_activate, or the A_out of the state update / forward sweep).
// Tails in M, N, K are handled by TMA zero fill, TMA store clipping and
// epilogue masks; inner dimensions must be multiples of 8 elements (16-byte
// TMA strides) and operands 16-byte aligned (else the generic kernel runs).
//
// Every mbarrier wait is bounded (about 2 s of %globaltimer); on expiry the
// kernel records IPC_ERR_TIMEOUT in a device status word, every role stops
// issuing work, and TMEM is freed before the CTA returns (ipc_device_status
// reads the word).
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "ipc_common.cuh"
#include "ipc_generic.cuh"
#include "ipc_tc.cuh"

namespace ipc {

__device__ int g_device_status = 0;  // first error code raised by a device-side bounded wait

namespace {

constexpr int TC_BM = 128;
constexpr int TC_BK = 64;
constexpr int TC_STAGES = 4;
constexpr int TC_STAGES_PAIR = 6;  // a pair CTA's stage holds 128 rows of A and BN/2 of B: 32 KB
constexpr int TC_EPI_WARPS = 8;                     // two per TMEM lane quarter
constexpr int TC_THREADS = 64 + 32 * TC_EPI_WARPS;  // TMA warp + MMA warp + epilogue
constexpr long long TC_WAIT_NS = 2000000000LL;

// Epilogue staging through shared memory (P, W, F, WD, I without split-K).  P / W / F / WD use 4 KB
// per epilogue warp as one 32-row x 128-byte transpose buffer; I uses two slots per warp, each holding
// an E tile and an X tile of 32 rows: 16 columns (2 KB slots) in the single-CTA form, 32 columns
// (4 KB slots, 64-byte rows) in the CTA-pair form, whose mainloop then has one stage less (5 x 32 KB).
// The I epilogue streams four operands (E, X in; X, A_out out) and bounds the kernel when the
// reduction is short (K = 1000: a tile's MMAs take ~7 us).
constexpr int EPI_SLOT = 2048;
// I epilogue chunk width: 16 columns (32-byte rows) in the single-CTA form, 32 (64-byte rows, whole
// DRAM bursts per row) in the pair form; a slot holds the E and the X tile of one chunk
__host__ __device__ constexpr int epi_cw(int pair) { return pair ? 32 : 16; }
__host__ __device__ constexpr int epi_slot_bytes(int mode, int pair) {
  return mode == MODE_I ? 2 * 32 * epi_cw(pair) * 2 : EPI_SLOT;
}
__host__ __device__ constexpr int epi_slots(int mode, int pair) { return 2; }
__host__ __device__ constexpr int epi_warp_bytes(int mode, int pair) {
  return epi_slots(mode, pair) * epi_slot_bytes(mode, pair);
}
__host__ __device__ constexpr int epi_bytes(int mode, int pair) { return TC_EPI_WARPS * epi_warp_bytes(mode, pair); }
__host__ __device__ constexpr int tc_stages(int mode, int pair) {
  return pair ? (mode == MODE_I ? TC_STAGES_PAIR - 1 : TC_STAGES_PAIR) : TC_STAGES;
}

constexpr int TC_RASTER = 16;  // default M-tiles per raster band: a wave covers ~16 x 9 tiles, both operands in L2

struct TcParams {
  int Mg, Ng, Kg, groups;
  int tiles_m, tiles_n, tiles;
  void* out;
  long long ld_out, gs_out;
  const void* aux;
  long long gs_aux;
  void* aux2;
  long long gs_aux2;
  float scale;
  int accumulate;
  int a_out_from_stored;  // I: A_out = f(cast(x_new)) (what recompute mode reads back) instead of f(x_new)
  // split-K (weight update with few output tiles): `splits` K ranges of `kps` 64-deep blocks each; the
  // fp32 partial tiles go to ws[split][group][m][n] and ws_reduce_kernel applies the epilogue
  int splits, kps;
  float* ws;
  int staged;  // P / W / I: epilogue staged through shared memory with TMA loads and stores
  // WD on CTA pairs: the two batch halves of a tile (splits == 2) are added into a zeroed dw with fp32
  // vector atomics; 0 + a + b == 0 + b + a exactly, so the result does not depend on their order
  int atomic;
  int mcast;  // WD: out is a multicast (NVLS) address; the epilogue adds into every GPU's copy
  int raster;  // M-tiles per raster band of the tile walk
  OptParams opt;  // WO: optimizer step applied to W in the epilogue
};

// ------------------------------------------------------------ PTX helpers
__device__ __forceinline__ uint32_t saddr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ long long now_ns() {
  long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false (and the device status set) if the phase never completes.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try(bar, parity)) return true;
  const long long t0 = now_ns();
  while (true) {
    if (mbar_try(bar, parity)) return true;
    if (*abort_flag) return false;
    if (now_ns() - t0 > TC_WAIT_NS) {
      atomicCAS(&g_device_status, 0, IPC_ERR_TIMEOUT);
      *abort_flag = 1;
      return false;
    }
  }
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];"
               ::"l"(reinterpret_cast<uint64_t>(map)), "r"(src), "r"(x), "r"(y), "r"(z)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ void sts128(uint32_t a, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
// Let a TMA load that is still in flight land (exit path after an aborted wait); bounded at 1 ms.
__device__ __forceinline__ void mbar_drain(uint32_t bar, uint32_t parity) {
  const long long t0 = now_ns();
  while (!mbar_try(bar, parity) && now_ns() - t0 < 1000000LL) {
  }
}

// Tile t -> (group, first row, first column).  Rows are walked in bands of
// p.raster M-tiles, all N-tiles of a band before the next band, so the CTAs of
// one wave share a few A row-blocks and B column-blocks in L2.
// With split-K the split index is the fastest-varying part of t.
// tm: rows of a tile (128, or 256 for a CTA pair); rank: the CTA's half of a pair tile (its m0 is the
// first row it owns: tile row + 128 rank).
__device__ __forceinline__ void tile_coords(const TcParams& p, int t, int bn, int& g, int& m0, int& n0, int& s,
                                            int tm = TC_BM, int rank = 0) {
  s = t % p.splits;
  t /= p.splits;
  const int tiles_mn = p.tiles_m * p.tiles_n;
  g = t / tiles_mn;
  const int r = t % tiles_mn;
  const int band = r / (p.raster * p.tiles_n);
  const int first_m = band * p.raster;
  const int band_m = min(p.raster, p.tiles_m - first_m);
  const int within = r - band * p.raster * p.tiles_n;
  m0 = (first_m + within % band_m) * tm + TC_BM * rank;
  n0 = (within / band_m) * bn;
}

// ---- CTA-pair (cta_group::2) helpers: a 256 x BN tile computed by two CTAs of a cluster, each holding
// 128 rows of A and BN/2 columns of B; the even CTA (the leader) issues the MMAs, the odd CTA's TMA
// loads complete on the leader's stage barriers, the commits arrive at both CTAs' barriers.
__device__ __forceinline__ uint32_t cta_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t mapa0(uint32_t addr) {  // the same shared variable in the leader CTA
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(r) : "r"(addr));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y,
                                                 int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void tc_mma_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
}
// Arrive on the barrier at this offset in both CTAs of the pair once the issued MMAs are done.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"((uint16_t)3)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2), version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

template <typename T>
struct Vec8 {
  static __device__ __forceinline__ void st(T* p, const float (&v)[8]) {
    uint4 raw;
    T* h = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int j = 0; j < 8; ++j) h[j] = St<T>::st(v[j]);
    *reinterpret_cast<uint4*>(p) = raw;
  }
};

// Direct epilogue for 8 consecutive columns [n, n+8) of output row m, used by the modes without a
// staged epilogue: WD (dw = alpha acc, or += with accumulate, fp32), WO (an optimizer step on W) and F (OUT = cast(acc) and
// f(OUT), f in its MUFU form: one fp16 rounding step, every result is stored in 16 bits).
template <typename T, int ACT, int MODE>
__device__ __forceinline__ void epi8(const TcParams& p, int g, int m, int n, const float (&acc)[8]) {
  const long long idx = (long long)m * p.ld_out + n;
  if constexpr (MODE == MODE_WD) {
    float4* dw = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + g * p.gs_out + idx);
    float4 a = make_float4(p.scale * acc[0], p.scale * acc[1], p.scale * acc[2], p.scale * acc[3]);
    float4 b = make_float4(p.scale * acc[4], p.scale * acc[5], p.scale * acc[6], p.scale * acc[7]);
    if (p.accumulate) {
      const float4 a0 = dw[0], b0 = dw[1];
      a.x += a0.x; a.y += a0.y; a.z += a0.z; a.w += a0.w;
      b.x += b0.x; b.y += b0.y; b.z += b0.z; b.w += b0.w;
    }
    dw[0] = a;
    dw[1] = b;
  } else if constexpr (MODE == MODE_WO) {
    // optimizer step on 8 weights: g = -acc (the gradient of the energy), state in fp32 at the same index
    T* w = reinterpret_cast<T*>(p.out) + g * p.gs_out + idx;
    uint4 raw = *reinterpret_cast<const uint4*>(w);
    T* h = reinterpret_cast<T*>(&raw);
    const long long base = g * p.gs_out + idx;
#pragma unroll
    for (int j = 0; j < 8; ++j) h[j] = St<T>::st(opt_step(p.opt, St<T>::ld(h[j]), -acc[j], base + j));
    *reinterpret_cast<uint4*>(w) = raw;
  } else if constexpr (MODE == MODE_F) {
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = acc[j];
    Vec8<T>::st(reinterpret_cast<T*>(p.out) + g * p.gs_out + idx, o);
    if (p.aux2 != nullptr) {
      float an[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) an[j] = act_f_hw<ACT>(rnd<T>(acc[j]));
      Vec8<T>::st(reinterpret_cast<T*>(p.aux2) + g * p.gs_aux2 + idx, an);
    }
  }
}

// The staged epilogue on one 16-byte vector (8 columns) of a thread's row: P e = cast(x - cast(acc)),
// W cast(w + alpha acc); I x_new = cast(x + gamma (-e + f'(x) acc)) and A_out = cast(f(x_new)) (of
// cast(x_new) with a_out_from_stored), f and f' in their MUFU forms.
template <typename T, int MODE>
__device__ __forceinline__ uint4 epi_vec_pw(uint4 in, const uint32_t* acc8, float scale) {
  const T* h = reinterpret_cast<const T*>(&in);
  uint4 o;
  T* oh = reinterpret_cast<T*>(&o);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float a = __uint_as_float(acc8[j]);
    if constexpr (MODE == MODE_P)
      oh[j] = St<T>::st(St<T>::ld(h[j]) - rnd<T>(a));
    else
      oh[j] = St<T>::st(St<T>::ld(h[j]) + scale * a);
  }
  return o;
}

// F through the transpose buffer: a row thread packs 8 accumulators into cast(acc) ...
template <typename T>
__device__ __forceinline__ uint4 pack_vec(const uint32_t* acc8) {
  uint4 o;
  T* oh = reinterpret_cast<T*>(&o);
#pragma unroll
  for (int j = 0; j < 8; ++j) oh[j] = St<T>::st(__uint_as_float(acc8[j]));
  return o;
}
// ... and the coalesced pass stores it and cast(f(x)) of the stored x (the A_out of the forward sweep)
template <typename T, int ACT>
__device__ __forceinline__ uint4 act_vec(uint4 x) {
  const T* h = reinterpret_cast<const T*>(&x);
  uint4 o;
  T* oh = reinterpret_cast<T*>(&o);
#pragma unroll
  for (int j = 0; j < 8; ++j) oh[j] = St<T>::st(act_f_hw<ACT>(St<T>::ld(h[j])));
  return o;
}

template <typename T, int ACT>
__device__ __forceinline__ void epi_vec_i(uint4 ev, uint4& xv, uint4& av, const uint32_t* acc8, float gamma,
                                          int from_stored) {
  const T* eh = reinterpret_cast<const T*>(&ev);
  T* xh = reinterpret_cast<T*>(&xv);
  T* ah = reinterpret_cast<T*>(&av);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float x0 = St<T>::ld(xh[j]);
    const float xn = x0 + gamma * (-St<T>::ld(eh[j]) + act_df_hw<ACT>(x0) * __uint_as_float(acc8[j]));
    xh[j] = St<T>::st(xn);
    ah[j] = St<T>::st(act_f_hw<ACT>(from_stored ? rnd<T>(xn) : xn));
  }
}

// TMA loads of one I epilogue chunk into a slot: the E tile (map0) and the X tile (map1).
__device__ __forceinline__ void epi_load_i(const CUtensorMap* map0, const CUtensorMap* map1, uint32_t slot,
                                           uint32_t bar, uint32_t tile_bytes, int n, int r0, int g) {
  mbar_expect_tx(bar, 2 * tile_bytes);
  tma_load_3d(slot, map0, bar, n, r0, g);
  tma_load_3d(slot + tile_bytes, map1, bar, n, r0, g);
}

template <typename T, int ACT, int MODE, int BN, int PAIR>
__global__ void __launch_bounds__(TC_THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmE0, const __grid_constant__ CUtensorMap tmE1,
                   const __grid_constant__ CUtensorMap tmE2, const __grid_constant__ TcParams p) {
  // tmE0..2: the I epilogue's operand maps (E, X, A_out)
  constexpr bool A_MN = (MODE == MODE_I);
  constexpr bool B_MN = (MODE == MODE_P || MODE == MODE_I || MODE == MODE_F);
  constexpr int NCTA = PAIR ? 2 : 1;
  constexpr int TM = TC_BM * NCTA;    // rows of a tile
  constexpr int BNL = BN / NCTA;      // columns of B this CTA loads
  constexpr int STAGES = tc_stages(MODE, PAIR);
  constexpr int NSL = epi_slots(MODE, PAIR);             // I epilogue slots per warp
  constexpr int EPI_WARP_BYTES = epi_warp_bytes(MODE, PAIR);
  constexpr uint32_t A_BYTES = TC_BM * TC_BK * 2;
  constexpr uint32_t B_BYTES = BNL * TC_BK * 2;
  constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr uint32_t TMEM_COLS = 2 * BN;  // two accumulators
  // instruction descriptor: fp32 accumulate, A/B fp16 or bf16, majors, N, M = 128 (256 for a pair)
  constexpr uint32_t FMT = std::is_same<T, __half>::value ? 0u : 1u;
  constexpr uint32_t IDESC = (1u << 4) | (FMT << 7) | (FMT << 10) | ((A_MN ? 1u : 0u) << 15) |
                             ((B_MN ? 1u : 0u) << 16) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(TM >> 4) << 24);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr bool EPI_STAGED =
      (MODE == MODE_P || MODE == MODE_W || MODE == MODE_I || MODE == MODE_F || MODE == MODE_WD);
  constexpr uint32_t EPI_REGION = EPI_STAGED ? epi_bytes(MODE, PAIR) : 0;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES + EPI_REGION);
  // bars: full[S], empty[S], tfull[2], tempty[2], epilogue slots[NSL per epilogue warp]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4 + NSL * TC_EPI_WARPS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const uint32_t full0 = saddr(bars), empty0 = saddr(bars + STAGES);
  const uint32_t tfull0 = saddr(bars + 2 * STAGES), tempty0 = saddr(bars + 2 * STAGES + 2);
  const uint32_t ebar0 = saddr(bars + 2 * STAGES + 4);
  // a pair: rank 0 leads (its stage barriers count both CTAs' loads, its tempty both CTAs' epilogues)
  const int rank = PAIR ? (int)cta_rank() : 0;
  const int unit0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int units = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull0 + 8 * b, 1);
      mbar_init(tempty0 + 8 * b, 32 * TC_EPI_WARPS * NCTA);
    }
    for (int b = 0; b < NSL * TC_EPI_WARPS; ++b) mbar_init(ebar0 + 8 * b, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {  // a pair allocates collectively: the same warp of both CTAs, the same columns in each
    if constexpr (PAIR) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(tmem_slot)),
                   "r"(TMEM_COLS));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(tmem_slot)),
                   "r"(TMEM_COLS));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // both CTAs' barriers exist before either signals the other's
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int nk = (p.Kg + TC_BK - 1) / TC_BK;
  // an epilogue thread has read its part of an accumulator: arrive on the leader's tempty barrier
  auto release_acc = [&](uint32_t bar) {
    if constexpr (PAIR) {
      if (rank == 0) mbar_arrive(bar); else mbar_arrive_remote(mapa0(bar));
    } else {
      mbar_arrive(bar);
    }
  };

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
    }
    int s = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int t = unit0; t < p.tiles && ok; t += units) {
      int g, m0, n0, sp;
      tile_coords(p, t, BN, g, m0, n0, sp, TM, rank);  // m0: this CTA's first row
      const int nb = n0 + BNL * rank;                  // this CTA's first B column
      const int kb_end = min(nk, (sp + 1) * p.kps);
      for (int kb = sp * p.kps; kb < kb_end; ++kb) {
        ok = mbar_wait(empty0 + 8 * s, phase ^ 1, abort_flag);
        __syncwarp();
        if (!ok) break;
        if (lane == 0) {
          const uint32_t full = full0 + 8 * s;
          const uint32_t sa = saddr(smem + s * STAGE_BYTES), sb = sa + A_BYTES;
          const int k0 = kb * TC_BK;
          if constexpr (PAIR) {
            // both CTAs' halves complete on the leader's barrier; the leader expects the pair's bytes
            const uint32_t fl = mapa0(full);
            if (rank == 0) mbar_expect_tx(full, 2 * STAGE_BYTES);
            if constexpr (A_MN) {
              tma_load_3d_pair(sa, &tmA, fl, m0, k0, g);
              tma_load_3d_pair(sa + A_BYTES / 2, &tmA, fl, m0 + 64, k0, g);
            } else {
              tma_load_3d_pair(sa, &tmA, fl, k0, m0, g);
            }
            if constexpr (B_MN) {
#pragma unroll
              for (int j = 0; j < BNL / 64; ++j)
                tma_load_3d_pair(sb + j * (64 * TC_BK * 2), &tmB, fl, nb + 64 * j, k0, g);
            } else {
              tma_load_3d_pair(sb, &tmB, fl, k0, nb, g);
            }
          } else {
            mbar_expect_tx(full, STAGE_BYTES);
            if constexpr (A_MN) {
              tma_load_3d(sa, &tmA, full, m0, k0, g);
              tma_load_3d(sa + A_BYTES / 2, &tmA, full, m0 + 64, k0, g);
            } else {
              tma_load_3d(sa, &tmA, full, k0, m0, g);
            }
            if constexpr (B_MN) {
#pragma unroll
              for (int j = 0; j < BN / 64; ++j) tma_load_3d(sb + j * (64 * TC_BK * 2), &tmB, full, n0 + 64 * j, k0, g);
            } else {
              tma_load_3d(sb, &tmB, full, k0, n0, g);
            }
          }
        }
        __syncwarp();
        if (++s == STAGES) { s = 0; phase ^= 1; }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer -------------------------------
    // (a pair's odd CTA issues nothing: the leader's cta_group::2 MMAs read both CTAs' stages)
    if (rank == 0) {
    int s = 0, acc = 0;
    uint32_t phase = 0, aphase = 0;
    bool ok = true;
    for (int t = unit0; t < p.tiles && ok; t += units) {
      ok = mbar_wait(tempty0 + 8 * acc, aphase ^ 1, abort_flag);
      __syncwarp();
      if (!ok) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BN;
      const int sp = t % p.splits;
      const int kb_begin = sp * p.kps, kb_end = min(nk, (sp + 1) * p.kps);
      for (int kb = kb_begin; kb < kb_end; ++kb) {
        ok = mbar_wait(full0 + 8 * s, phase, abort_flag);
        __syncwarp();
        if (!ok) break;
        tc_fence_after();
        if (lane == 0) {
          const uint32_t sa = saddr(smem + s * STAGE_BYTES), sb = sa + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < TC_BK / 16; ++kk) {
            // K-major: +32 B per 16-element step inside the 128-byte swizzle row.
            // MN-major: +2 groups of 8 K-rows (2 KB) per step; 64-element MN blocks 8 KB apart.
            const uint64_t ad = A_MN ? smem_desc(sa + kk * 2048, 64 * TC_BK * 2, 1024) : smem_desc(sa + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? smem_desc(sb + kk * 2048, 64 * TC_BK * 2, 1024) : smem_desc(sb + kk * 32, 16, 1024);
            if constexpr (PAIR)
              tc_mma_pair(d_tmem, ad, bd, IDESC, (kb > kb_begin || kk > 0) ? 1u : 0u);
            else
              tc_mma(d_tmem, ad, bd, IDESC, (kb > kb_begin || kk > 0) ? 1u : 0u);
          }
          // stage free (in both CTAs of a pair) once these MMAs have read it
          if constexpr (PAIR) tc_commit_pair(empty0 + 8 * s); else tc_commit(empty0 + 8 * s);
        }
        __syncwarp();
        if (++s == STAGES) { s = 0; phase ^= 1; }
      }
      if (!ok) break;
      if (lane == 0) {  // accumulator ready (a pair: each CTA's half of it)
        if constexpr (PAIR) tc_commit_pair(tfull0 + 8 * acc); else tc_commit(tfull0 + 8 * acc);
      }
      __syncwarp();
      if (++acc == 2) { acc = 0; aphase ^= 1; }
    }
    }  // rank 0
  } else {
    // ------------------------------- epilogue --------------------------------
    const int q = warp & 3;     // TMEM lane quarter this warp may access
    constexpr int HC = BN / 2;  // accumulator columns per epilogue warp
    const int c_lo = ((warp - 2) >> 2) * HC;
    int acc = 0;
    uint32_t aphase = 0;
    bool staged = false;
    if constexpr (EPI_STAGED) staged = p.staged != 0;
    const bool xpose = (MODE == MODE_P || MODE == MODE_W || MODE == MODE_F) && staged;
    if (xpose) {
      {
        // P / W: the warp's 32 x HC block of the in/out operand (X_lo or W) is read with coalesced
        // 16-byte loads into registers while the tile's MMAs run (the next tile's block as soon as
        // this one is in shared memory), then per 64-column chunk: registers -> swizzled shared
        // buffer, each row thread applies the epilogue to its row in place, and the chunk leaves
        // with coalesced 16-byte stores (a warp instruction covers 4 rows x 128 bytes).
        // F has no input block: the row threads write cast(acc) into the buffer, and the coalesced
        // pass stores it and, when A_out is given, cast(f(x)) beside it.
        constexpr bool HAS_IN = (MODE != MODE_F);
        constexpr int NCH = HC / 64;        // 64-column chunks per warp and tile
        constexpr int NPRE = 8 * NCH;       // prefetched 16-byte vectors per thread
        const uint32_t xb = saddr(smem + STAGES * STAGE_BYTES) + (warp - 2) * EPI_WARP_BYTES;
        const T* src = reinterpret_cast<const T*>(MODE == MODE_P ? p.aux : p.out);
        const long long gsrc = MODE == MODE_P ? p.gs_aux : p.gs_out;
        T* dst = reinterpret_cast<T*>(p.out);
        const int cr = lane >> 3, cj = lane & 7;  // coalesced layout: row 4i + cr, vector cj
        uint4 pre[NPRE];
        auto prefetch = [&](int t) {
          int g, m0, n0, sp;
          tile_coords(p, t, BN, g, m0, n0, sp, TM, rank);
          const int r0 = m0 + 32 * q, nw = n0 + c_lo;
#pragma unroll
          for (int cc = 0; cc < NCH; ++cc) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int r = r0 + 4 * i + cr, n = nw + 64 * cc + 8 * cj;
              if (r < p.Mg && n < p.Ng)
                pre[8 * cc + i] = *reinterpret_cast<const uint4*>(src + g * gsrc + (long long)r * p.ld_out + n);
            }
          }
        };
        if (HAS_IN && unit0 < p.tiles) prefetch(unit0);
        for (int t = unit0; t < p.tiles; t += units) {
          int g, m0, n0, sp;
          tile_coords(p, t, BN, g, m0, n0, sp, TM, rank);
          const int r0 = m0 + 32 * q, nw = n0 + c_lo;
          const bool ok = mbar_wait(tfull0 + 8 * acc, aphase, abort_flag);
          __syncwarp();
          if (!ok) break;
          tc_fence_after();
          const uint32_t trow = tmem_base + ((uint32_t)(32 * q) << 16) + acc * BN;
#pragma unroll
          for (int cc = 0; cc < NCH; ++cc) {
            if constexpr (HAS_IN) {
              // registers -> shared (row 4i + cr, vector cj; 128-byte rows, vector index ^ (row & 7))
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const int r = 4 * i + cr;
                sts128(xb + r * 128 + ((cj ^ (r & 7)) << 4), pre[8 * cc + i]);
              }
              if (cc == NCH - 1 && t + units < p.tiles) prefetch(t + units);
            }
            __syncwarp();
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
              uint32_t raw[32];
              tmem_ld32(trow + c_lo + 64 * cc + 32 * hf, raw);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const uint32_t a = xb + lane * 128 + (((4 * hf + j) ^ (lane & 7)) << 4);
                if constexpr (HAS_IN)
                  sts128(a, epi_vec_pw<T, MODE>(lds128(a), raw + 8 * j, p.scale));
                else
                  sts128(a, pack_vec<T>(raw + 8 * j));
              }
            }
            if (cc == NCH - 1) {  // every accumulator column read: release it to the MMA warp
              tc_fence_before();
              release_acc(tempty0 + 8 * acc);
            }
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int r = 4 * i + cr, n = nw + 64 * cc + 8 * cj;
              const uint4 v = lds128(xb + r * 128 + ((cj ^ (r & 7)) << 4));
              if (r0 + r < p.Mg && n < p.Ng) {
                *reinterpret_cast<uint4*>(dst + g * p.gs_out + (long long)(r0 + r) * p.ld_out + n) = v;
                if constexpr (MODE == MODE_F) {
                  if (p.aux2 != nullptr)
                    *reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.aux2) + g * p.gs_aux2 +
                                              (long long)(r0 + r) * p.ld_out + n) = act_vec<T, ACT>(v);
                }
              }
            }
            __syncwarp();
          }
          if (++acc == 2) { acc = 0; aphase ^= 1; }
        }
      }
    } else if (staged) {
      if constexpr (MODE == MODE_I) {
        // I: E and X staged through shared memory in CW-column chunks (NSL slots per warp, each an E
        // and an X tile of 32 rows).  The first NSL chunks are requested with TMA before the
        // accumulator is ready; later chunks as the TMA stores (X, and A_out when given) of the chunk
        // before free its slot.  Rows of CW x 2 bytes: 32 (32-byte swizzle) or 64 (64-byte swizzle).
        constexpr int CW = epi_cw(PAIR);
        constexpr int CPL = 32 / CW;            // chunks per 32-column TMEM load
        constexpr int VPR = CW / 8;             // 16-byte vectors per row
        constexpr int NSUB = HC / CW;
        static_assert(NSUB >= NSL && (NSL & (NSL - 1)) == 0, "I epilogue: slots a power of two, <= chunks");
        constexpr uint32_t TILE = 32 * CW * 2;  // one 32-row operand tile
        constexpr uint32_t SLOT = epi_slot_bytes(MODE, PAIR);
        auto swz = [&](int row) { return CW == 16 ? ((row >> 2) & 1) : ((row >> 1) & 3); };
        const uint32_t ebase = saddr(smem + STAGES * STAGE_BYTES) + (warp - 2) * EPI_WARP_BYTES;
        const uint32_t ebar = ebar0 + 8 * NSL * (warp - 2);
        uint32_t eph = 0, pending = 0;
        bool ok = true;
        for (int t = unit0; t < p.tiles && ok; t += units) {
          int g, m0, n0, sp;
          tile_coords(p, t, BN, g, m0, n0, sp, TM, rank);
          const int r0 = m0 + 32 * q;
          const bool live = r0 < p.Mg;
          const int nw = n0 + c_lo;
          if (live && lane == 0) {
            bulk_wait_read0();  // the previous tile's stores have read every slot
#pragma unroll
            for (int s = 0; s < NSL; ++s) {
              if (nw + CW * s < p.Ng) {
                epi_load_i(&tmE0, &tmE1, ebase + s * SLOT, ebar + 8 * s, TILE, nw + CW * s, r0, g);
                pending |= 1u << s;
              }
            }
          }
          __syncwarp();
          if (!mbar_wait(tfull0 + 8 * acc, aphase, abort_flag)) ok = false;
          __syncwarp();
          if (!ok) break;
          tc_fence_after();
          const uint32_t trow = tmem_base + ((uint32_t)(32 * q) << 16) + acc * BN;
#pragma unroll 1
          for (int c = 0; c < HC / 32 && ok; ++c) {
            uint32_t raw[32];
            tmem_ld32(trow + c_lo + 32 * c, raw);
#pragma unroll
            for (int h = 0; h < CPL; ++h) {
              const int sidx = CPL * c + h, slot = sidx & (NSL - 1);
              const int n = nw + CW * sidx;
              if (!live || n >= p.Ng || !ok) continue;
              if (!mbar_wait(ebar + 8 * slot, (eph >> slot) & 1u, abort_flag)) {
                ok = false;
                continue;
              }
              eph ^= 1u << slot;
              pending &= ~(1u << slot);
              const uint32_t sb = ebase + slot * SLOT;
#pragma unroll
              for (int j = 0; j < VPR; ++j) {  // row = lane; TMA swizzle: vector j ^ swz(row)
                const uint32_t off = lane * (CW * 2) + ((j ^ swz(lane)) << 4);
                uint4 xv = lds128(sb + TILE + off), av;
                epi_vec_i<T, ACT>(lds128(sb + off), xv, av, raw + CW * h + 8 * j, p.scale, p.a_out_from_stored);
                sts128(sb + TILE + off, xv);
                if (p.aux2 != nullptr) sts128(sb + off, av);
              }
              fence_async_smem();
              __syncwarp();
              if (lane == 0) {
                tma_store_3d(&tmE1, sb + TILE, n, r0, g);
                if (p.aux2 != nullptr) tma_store_3d(&tmE2, sb, n, r0, g);
                bulk_commit();
                // refill: with two slots, this chunk's slot once its stores have read it; with more, the
                // previous chunk's slot, whose stores were issued a chunk earlier (waiting on all but the
                // newest store group keeps this chunk's stores off the critical path)
                constexpr int D = NSL >= 3 ? 1 : 0;
                const int rs = sidx - D;
                if (rs >= 0 && rs + NSL < NSUB && nw + CW * (rs + NSL) < p.Ng) {
                  if constexpr (D == 1) bulk_wait_read1(); else bulk_wait_read0();
                  const int rslot = rs & (NSL - 1);
                  epi_load_i(&tmE0, &tmE1, ebase + rslot * SLOT, ebar + 8 * rslot, TILE, nw + CW * (rs + NSL), r0,
                             g);
                  pending |= 1u << rslot;
                }
              }
              __syncwarp();
            }
          }
          if (!ok) break;
          tc_fence_before();
          release_acc(tempty0 + 8 * acc);
          if (++acc == 2) { acc = 0; aphase ^= 1; }
        }
        if (lane == 0) {
          // loads still in flight (only after an aborted wait) land before the CTA exits
#pragma unroll
          for (int s = 0; s < NSL; ++s)
            if ((pending >> s) & 1u) mbar_drain(ebar + 8 * s, (eph >> s) & 1u);
          bulk_wait0();
        }
        __syncwarp();
      } else if constexpr (MODE == MODE_WD) {
        // WD (dw = scale * acc in fp32): per 32-column chunk the row threads write their scaled
        // accumulators into the swizzled buffer (128-byte rows, vector index ^ (row & 7)), and the warp
        // stores the chunk with coalesced 16-byte stores (an instruction covers 4 rows x 128 bytes)
        const uint32_t xb = saddr(smem + STAGES * STAGE_BYTES) + (warp - 2) * EPI_WARP_BYTES;
        float* dst = reinterpret_cast<float*>(p.out);
        const int cr = lane >> 3, cj = lane & 7;
        for (int t = unit0; t < p.tiles; t += units) {
          int g, m0, n0, sp;
          tile_coords(p, t, BN, g, m0, n0, sp, TM, rank);
          const int r0 = m0 + 32 * q, nw = n0 + c_lo;
          const bool ok = mbar_wait(tfull0 + 8 * acc, aphase, abort_flag);
          __syncwarp();
          if (!ok) break;
          tc_fence_after();
          const uint32_t trow = tmem_base + ((uint32_t)(32 * q) << 16) + acc * BN;
#pragma unroll 1
          for (int c = 0; c < HC / 32; ++c) {
            uint32_t raw[32];
            tmem_ld32(trow + c_lo + 32 * c, raw);
            if (c == HC / 32 - 1) {  // every accumulator column read: release it to the MMA warp
              tc_fence_before();
              release_acc(tempty0 + 8 * acc);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j)
              sts128(xb + lane * 128 + ((j ^ (lane & 7)) << 4),
                     make_uint4(__float_as_uint(p.scale * __uint_as_float(raw[4 * j])),
                                __float_as_uint(p.scale * __uint_as_float(raw[4 * j + 1])),
                                __float_as_uint(p.scale * __uint_as_float(raw[4 * j + 2])),
                                __float_as_uint(p.scale * __uint_as_float(raw[4 * j + 3]))));
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int r = 4 * i + cr, n = nw + 32 * c + 4 * cj;
              const uint4 v = lds128(xb + r * 128 + ((cj ^ (r & 7)) << 4));
              if (r0 + r < p.Mg && n < p.Ng) {
                float* o = dst + g * p.gs_out + (long long)(r0 + r) * p.ld_out + n;
                if (p.mcast)
                  asm volatile("multimem.red.relaxed.sys.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(o),
                               "f"(__uint_as_float(v.x)), "f"(__uint_as_float(v.y)), "f"(__uint_as_float(v.z)),
                               "f"(__uint_as_float(v.w))
                               : "memory");
                else if (p.atomic)
                  atomicAdd(reinterpret_cast<float4*>(o), make_float4(__uint_as_float(v.x), __uint_as_float(v.y),
                                                                      __uint_as_float(v.z), __uint_as_float(v.w)));
                else
                  *reinterpret_cast<uint4*>(o) = v;
              }
            }
            __syncwarp();
          }
          if (++acc == 2) { acc = 0; aphase ^= 1; }
        }
        // multicast adds performed at system scope before the kernel ends (the caller's cross-GPU
        // ordering starts from this kernel's completion)
        if (p.mcast) asm volatile("fence.acq_rel.sys;" ::: "memory");
      }
    } else {
      for (int t = unit0; t < p.tiles; t += units) {
        int g, m0, n0, sp;
        tile_coords(p, t, BN, g, m0, n0, sp, TM, rank);
        const int m = m0 + 32 * q + lane;
        const bool ok = mbar_wait(tfull0 + 8 * acc, aphase, abort_flag);
        __syncwarp();
        if (!ok) break;
        tc_fence_after();
        const uint32_t trow = tmem_base + ((uint32_t)(32 * q) << 16) + acc * BN;
#pragma unroll 1
        for (int c = 0; c < HC / 32; ++c) {
          uint32_t raw[32];
          tmem_ld32(trow + c_lo + 32 * c, raw);
          if (m < p.Mg) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              const int n = n0 + c_lo + 32 * c + 8 * v;
              if (n >= p.Ng) continue;
              if (p.splits > 1) {  // fp32 partial of this K range; the reduce pass applies the epilogue
                float4* dst = reinterpret_cast<float4*>(
                    p.ws + (((long long)sp * p.groups + g) * p.Mg + m) * (long long)p.Ng + n);
                dst[0] = make_float4(__uint_as_float(raw[8 * v]), __uint_as_float(raw[8 * v + 1]),
                                     __uint_as_float(raw[8 * v + 2]), __uint_as_float(raw[8 * v + 3]));
                dst[1] = make_float4(__uint_as_float(raw[8 * v + 4]), __uint_as_float(raw[8 * v + 5]),
                                     __uint_as_float(raw[8 * v + 6]), __uint_as_float(raw[8 * v + 7]));
              } else {
                float a8[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) a8[j] = __uint_as_float(raw[8 * v + j]);
                epi8<T, ACT, MODE>(p, g, m, n, a8);  // F, WD (P / I / W are staged)
              }
            }
          }
        }
        tc_fence_before();
        release_acc(tempty0 + 8 * acc);
        if (++acc == 2) { acc = 0; aphase ^= 1; }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // the leader's MMAs and the odd CTA's loads are done with both CTAs
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS));
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS));
  }
}

// ------------------------------------------------------------------- host
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 3-D map over a [groups][rows][inner] row-major array (element strides ld, gs).
int make_map(CUtensorMap* map, const void* base, int dtype, long long inner, long long rows, long long groups,
             long long ld, long long gs, int box_inner, int box_rows,
             CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto fn = encode_fn();
  if (fn == nullptr) return set_error(IPC_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)rows, (cuuint64_t)groups};
  const cuuint64_t strides[2] = {(cuuint64_t)(ld * 2), (cuuint64_t)(gs * 2)};
  const cuuint32_t box[3] = {(cuuint32_t)box_inner, (cuuint32_t)box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType dt = dtype == IPC_DT_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUresult r = fn(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(IPC_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return IPC_OK;
}

std::atomic<int> g_max_ctas{0};  // ipc_set_max_ctas: 0 = one persistent CTA per SM

int num_sms() {
  static int n[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (n[dev] == 0) cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev);
  return n[dev] > 0 ? n[dev] : 148;
}

// CTAs a persistent launch may use: every SM, or fewer while a caller leaves SMs to a collective.
int grid_cap() {
  const int n = num_sms(), c = g_max_ctas.load(std::memory_order_relaxed);
  return (c > 0 && c < n) ? c : n;
}

// Split-K second pass: out = epilogue(sum over splits of the fp32 partials), summed in split order
// (deterministic).  W: W = cast(W + scale * sum); WD: dw = (accumulate ? dw : 0) + scale * sum.
template <typename T, int MODE>
__global__ void ws_reduce_kernel(const float* __restrict__ ws, int splits, long long n4, void* out, float scale,
                                 int accumulate, const OptParams opt) {
  const float4* part = reinterpret_cast<const float4*>(ws);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    float4 acc = part[i];
    for (int sp = 1; sp < splits; ++sp) {
      const float4 v = part[(long long)sp * n4 + i];
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    if constexpr (MODE == MODE_WD) {
      float4* dw = reinterpret_cast<float4*>(out) + i;
      float4 o = make_float4(scale * acc.x, scale * acc.y, scale * acc.z, scale * acc.w);
      if (accumulate) {
        const float4 d = *dw;
        o.x += d.x; o.y += d.y; o.z += d.z; o.w += d.w;
      }
      *dw = o;
    } else if constexpr (MODE == MODE_WO) {
      T* w = reinterpret_cast<T*>(out) + 4 * i;
      w[0] = St<T>::st(opt_step(opt, St<T>::ld(w[0]), -acc.x, 4 * i));
      w[1] = St<T>::st(opt_step(opt, St<T>::ld(w[1]), -acc.y, 4 * i + 1));
      w[2] = St<T>::st(opt_step(opt, St<T>::ld(w[2]), -acc.z, 4 * i + 2));
      w[3] = St<T>::st(opt_step(opt, St<T>::ld(w[3]), -acc.w, 4 * i + 3));
    } else {
      T* w = reinterpret_cast<T*>(out) + 4 * i;
      w[0] = St<T>::st(St<T>::ld(w[0]) + scale * acc.x);
      w[1] = St<T>::st(St<T>::ld(w[1]) + scale * acc.y);
      w[2] = St<T>::st(St<T>::ld(w[2]) + scale * acc.z);
      w[3] = St<T>::st(St<T>::ld(w[3]) + scale * acc.w);
    }
  }
}

template <typename T, int ACT, int MODE, int BN, int PAIR>
int launch_tc_t(const GemmArgs& a, int dtype, cudaStream_t s, float* ws, size_t ws_bytes, const TcTune* tune) {
  constexpr bool A_MN = (MODE == MODE_I);
  constexpr bool B_MN = (MODE == MODE_P || MODE == MODE_I || MODE == MODE_F);
  constexpr int TM = PAIR ? 2 * TC_BM : TC_BM;  // rows of a tile
  constexpr int BNL = PAIR ? BN / 2 : BN;       // B columns one CTA loads
  CUtensorMap ta, tb;
  int rc;
  // A operand: rows are the M side (K-major) or the K side (MN-major)
  if (A_MN)
    rc = make_map(&ta, a.A, dtype, a.Mg, a.Kg, a.groups, a.lda, a.gsA, 64, TC_BK);
  else
    rc = make_map(&ta, a.A, dtype, a.Kg, a.Mg, a.groups, a.lda, a.gsA, TC_BK, TC_BM);
  if (rc) return rc;
  if (B_MN)
    rc = make_map(&tb, a.Bm, dtype, a.Ng, a.Kg, a.groups, a.ldb, a.gsB, 64, TC_BK);
  else
    rc = make_map(&tb, a.Bm, dtype, a.Kg, a.Ng, a.groups, a.ldb, a.gsB, TC_BK, BNL);
  if (rc) return rc;
  TcParams p{};
  p.Mg = a.Mg; p.Ng = a.Ng; p.Kg = a.Kg; p.groups = a.groups;
  p.tiles_m = (a.Mg + TM - 1) / TM;
  p.tiles_n = (a.Ng + BN - 1) / BN;
  p.tiles = p.tiles_m * p.tiles_n * a.groups;
  p.out = a.out; p.ld_out = a.Ng; p.gs_out = a.gsOut;
  p.aux = a.aux; p.gs_aux = a.gsAux;
  p.aux2 = a.aux2; p.gs_aux2 = a.gsAux2;
  p.scale = a.scale; p.accumulate = a.accumulate;
  p.a_out_from_stored = a.a_out_from_stored;
  // default band: 16 single-CTA row tiles = 8 pair tiles (2048 rows either way), so a wave of CTAs covers
  // a roughly square block of output tiles and re-reads each operand block about as often as the other
  p.raster = (tune != nullptr && tune->raster > 0) ? tune->raster : (PAIR ? TC_RASTER / 2 : TC_RASTER);
  p.opt = a.opt;
  // split-K: a weight update with fewer output tiles than half the SMs and a long batch reduction
  const int nk = (a.Kg + TC_BK - 1) / TC_BK;
  p.splits = 1;
  p.kps = nk;
  p.ws = nullptr;
  int cap = grid_cap();
  if (tune != nullptr && tune->max_ctas > 0 && tune->max_ctas < cap) cap = tune->max_ctas;
  const int want = tune != nullptr ? tune->splits : 0;  // 0: heuristic, 1: never, >= 2: requested
  const int units = PAIR ? max(1, cap / 2) : cap;  // tiles walked at once: CTAs, or CTA pairs
  if ((MODE == MODE_W || MODE == MODE_WD || MODE == MODE_WO) && ws != nullptr && want != 1 &&
      (want >= 2 || (p.tiles < units / 2 && nk >= 8)) &&
      a.gsOut == (long long)a.Mg * a.Ng) {  // the reduce pass walks out as one dense [groups][M][N] array
    const long long tile_bytes = (long long)a.groups * a.Mg * a.Ng * 4;
    int splits = want >= 2 ? min(want, nk) : min(units / p.tiles, nk / 4);  // heuristic: one wave of units
    const long long fit = (long long)(ws_bytes / (size_t)tile_bytes);
    if (fit < splits) splits = (int)fit;
    if (splits >= 2) {
      p.kps = (nk + splits - 1) / splits;
      p.splits = (nk + p.kps - 1) / p.kps;  // every split non-empty
      p.ws = ws;
    }
  }
  // CTA pairs, fp32 dW (not accumulating): each tile's batch reduction in two halves added into a dw
  // zeroed first, where the half tiles fill the last wave (4096^2 = 256 pair tiles on 74 pairs: 4 waves,
  // 3.5 with halves); taken for a saving of >= 5 % of the tile time (or on request, tc_splits >= 2)
  p.atomic = 0;
  p.mcast = a.mcast;
  if (MODE == MODE_WD && PAIR && p.splits == 1 && !a.accumulate && want != 1 && nk >= 16 &&
      a.gsOut == (long long)a.Mg * a.Ng) {
    const long long units = cap / 2 > 0 ? cap / 2 : 1;
    const long long w1 = (p.tiles + units - 1) / units, w2 = (2LL * p.tiles + units - 1) / units;
    if (want >= 2 || w2 * 20 <= 2 * w1 * 19) {
      p.splits = 2;
      p.kps = (nk + 1) / 2;
      p.atomic = 1;
    }
  }
  p.tiles *= p.splits;
  // staged epilogue (no split-K): P / W through the transpose buffer, I through TMA with three maps
  // (E, X, A_out) of 32-row x 16-column boxes, 32-byte swizzle
  constexpr bool EPI_STAGED =
      (MODE == MODE_P || MODE == MODE_W || MODE == MODE_I || MODE == MODE_F || MODE == MODE_WD);
  CUtensorMap te[3];
  memset(te, 0, sizeof(te));
  // WD accumulating into dw reads dw back per element: the row-per-thread path
  p.staged = EPI_STAGED && (p.splits == 1 || p.atomic) && !(MODE == MODE_WD && a.accumulate);
  if (MODE == MODE_I && p.staged) {
    const void* src[3] = {a.aux, a.out, a.aux2};
    const long long gs[3] = {a.gsAux, a.gsOut, a.gsAux2};
    for (int i = 0; i < 3; ++i) {
      if (src[i] == nullptr) continue;
      rc = make_map(&te[i], src[i], dtype, a.Ng, a.Mg, a.groups, a.Ng, gs[i], epi_cw(PAIR), 32,
                    PAIR ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
      if (rc) return rc;
    }
  }
  constexpr int STAGE_BYTES = (TC_BM + BNL) * TC_BK * 2;
  constexpr int STAGES = tc_stages(MODE, PAIR);
  // barriers (2 per stage, 4 accumulator, one per epilogue slot), the TMEM slot and the abort word
  constexpr int TAIL = ((2 * STAGES + 4 + epi_slots(MODE, PAIR) * TC_EPI_WARPS) * 8 + 8 + 255) / 256 * 256;
  const int smem = STAGES * STAGE_BYTES + (EPI_STAGED ? epi_bytes(MODE, PAIR) : 0) + 1024 + TAIL;
  auto kern = tc_gemm_kernel<T, ACT, MODE, BN, PAIR>;
  cudaError_t err = ensure_kernel_smem<tc_gemm_kernel<T, ACT, MODE, BN, PAIR>>(smem);
  if (err != cudaSuccess) return set_error(IPC_ERR_CUDA, "tcgen05 kernel smem attribute: %s", cudaGetErrorString(err));
  if (p.atomic && !p.mcast) {  // the two halves of each tile add into zeros (a multicast dw: the caller's)
    err = cudaMemsetAsync(a.out, 0, (size_t)a.groups * a.Mg * a.Ng * sizeof(float), s);
    if (err != cudaSuccess) return set_error(IPC_ERR_CUDA, "dw zero fill: %s", cudaGetErrorString(err));
  }
  if constexpr (PAIR) {
    // clusters of two CTAs, one pair per two SMs, each pair walking 256-row tiles
    const int pairs = p.tiles < cap / 2 ? p.tiles : cap / 2;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (pairs > 0 ? pairs : 1), 1, 1);
    cfg.blockDim = dim3(TC_THREADS, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    err = cudaLaunchKernelEx(&cfg, kern, ta, tb, te[0], te[1], te[2], p);
    if (err != cudaSuccess) return set_error(IPC_ERR_CUDA, "tcgen05 pair GEMM launch: %s", cudaGetErrorString(err));
  } else {
    const int grid = p.tiles < cap ? p.tiles : cap;
    kern<<<grid, TC_THREADS, smem, s>>>(ta, tb, te[0], te[1], te[2], p);
  }
  count_launch();
  int rc2 = check_launch("tcgen05 GEMM");
  if (rc2 || p.splits == 1 || p.atomic) return rc2;
  if constexpr (MODE == MODE_W || MODE == MODE_WD || MODE == MODE_WO) {
    const long long n4 = (long long)a.groups * a.Mg * a.Ng / 4;
    long long blocks = (n4 + 255) / 256;
    if (blocks > 148LL * 16) blocks = 148LL * 16;
    ws_reduce_kernel<T, MODE><<<(int)blocks, 256, 0, s>>>(ws, p.splits, n4, a.out, a.scale, a.accumulate, a.opt);
    count_launch();
    return check_launch("split-K reduce");
  }
  return IPC_OK;
}

template <typename T, int MODE, int BN, int PAIR>
int dispatch_act(const GemmArgs& a, int act, int dtype, cudaStream_t s, float* ws, size_t ws_bytes,
                 const TcTune* tune) {
  if constexpr (MODE == MODE_P || MODE == MODE_W || MODE == MODE_WD || MODE == MODE_WO) {
    return launch_tc_t<T, IPC_ACT_IDENTITY, MODE, BN, PAIR>(a, dtype, s, ws, ws_bytes, tune);  // f only in I / F
  } else {
    IPC_DISPATCH_ACT(act, AC, { return launch_tc_t<T, AC, MODE, BN, PAIR>(a, dtype, s, ws, ws_bytes, tune); });
  }
  return IPC_OK;
}

template <typename T, int BN, int PAIR>
int dispatch_mode(const GemmArgs& a, int mode, int act, int dtype, cudaStream_t s, float* ws, size_t ws_bytes,
                  const TcTune* tune) {
  switch (mode) {
    case MODE_P: return dispatch_act<T, MODE_P, BN, PAIR>(a, act, dtype, s, ws, ws_bytes, tune);
    case MODE_I: return dispatch_act<T, MODE_I, BN, PAIR>(a, act, dtype, s, ws, ws_bytes, tune);
    case MODE_W: return dispatch_act<T, MODE_W, BN, PAIR>(a, act, dtype, s, ws, ws_bytes, tune);
    case MODE_WD: return dispatch_act<T, MODE_WD, BN, PAIR>(a, act, dtype, s, ws, ws_bytes, tune);
    case MODE_F: return dispatch_act<T, MODE_F, BN, PAIR>(a, act, dtype, s, ws, ws_bytes, tune);
    case MODE_WO: return dispatch_act<T, MODE_WO, BN, PAIR>(a, act, dtype, s, ws, ws_bytes, tune);
    default: return set_error(IPC_ERR_ARG, "bad GEMM mode %d", mode);
  }
}

}  // namespace

bool tc_eligible(int mode, int M, int K, int B, int dtype, int algo, bool b_activated, bool splitk) {
  if (algo != IPC_ALGO_AUTO && algo != IPC_ALGO_TCGEN05) return false;
  if (dtype != IPC_DT_F16 && dtype != IPC_DT_BF16) return false;
  if (b_activated) return false;  // f on the B operand is materialised once by the caller
  int Mg = M, Ng = B, Kg = K;
  const bool weight = (mode == MODE_W || mode == MODE_WD || mode == MODE_WO);
  if (weight) { Ng = K; Kg = B; }
  if (Mg < 1 || Ng < 1 || Kg < 1) return false;
  if (M % 8 || K % 8 || B % 8) return false;  // 16-byte row strides for TMA and the epilogue vectors
  if (algo == IPC_ALGO_AUTO) {
    // a weight update with a long batch reduction spreads it over the SMs (split-K)
    if (weight && splitk && Kg >= 1024 && Mg >= 16 && Ng >= 16) return true;
    // below ~128 x 256 x 256 the generic kernel's lower latency wins; 64 <= M < 128 still pays on
    // tensor cores (the tile's missing rows are TMA zero fill, masked in the epilogue)
    if (Mg < 64 || Ng < 128 || Kg < 64) return false;
    if ((double)Mg * Ng * Kg < 128.0 * 256 * 256) return false;
  }
  return true;
}

int launch_tc(const GemmArgs& a, int mode, int act, int dtype, cudaStream_t s, float* ws, size_t ws_bytes,
              const TcTune* tune) {
  if (a.Mg <= 0 || a.Ng <= 0 || a.groups <= 0) return IPC_OK;
  if (a.Kg <= 0) return launch_generic(a, mode, false, act, dtype, s);  // nothing to multiply
  // TMA maps and 16-byte epilogue vectors need 16-byte aligned operands; a view that starts mid-vector
  // takes the generic kernel
  const uintptr_t mis = reinterpret_cast<uintptr_t>(a.A) | reinterpret_cast<uintptr_t>(a.Bm) |
                        reinterpret_cast<uintptr_t>(a.out) | reinterpret_cast<uintptr_t>(a.aux) |
                        reinterpret_cast<uintptr_t>(a.aux2);
  if (mis & 15) {
    if (a.mcast) return set_error(IPC_ERR_ARG, "IPC_FLAG_MULTIMEM_RED: operands must be 16-byte aligned");
    return launch_generic(a, mode, false, act, dtype, s);
  }
  // Tile width: the persistent walk takes ceil(tiles / CTAs) waves of one tile time each.  A 128 x 128
  // tile takes about 0.81 of a 128 x 256 tile's time (measured on B200 at 4096^2 x 65536: the MMAs are
  // bound by shared-memory operand reads, and the wide tile reads a third less per FLOP), so a tile
  // costs ~(BN + 416) units and the estimate is waves x (BN + 416); 128 x 256 tiles on a tie.  A weight
  // update that splits its batch reduction (split-K) fills the SMs with splits instead and keeps the
  // wide tile.
  const long long tm = (a.Mg + TC_BM - 1) / TC_BM;
  const long long t256 = tm * ((a.Ng + 255) / 256) * a.groups, t128 = tm * ((a.Ng + 127) / 128) * a.groups;
  const long long cap = grid_cap();
  const bool splitk = (mode == MODE_W || mode == MODE_WD || mode == MODE_WO) && ws != nullptr && t256 < cap / 2 &&
                      (a.Kg + TC_BK - 1) / TC_BK >= 8 && a.gsOut == (long long)a.Mg * a.Ng &&
                      ws_bytes >= (size_t)(2LL * a.groups * a.Mg * a.Ng * 4);
  const long long cost256 = ((t256 + cap - 1) / cap) * (256 + 416), cost128 = ((t128 + cap - 1) / cap) * (128 + 416);
  bool wide = a.Ng >= 256 && (cost256 <= cost128 || splitk);
  if (tune != nullptr && (tune->bn == 128 || tune->bn == 256)) wide = tune->bn == 256;
  // CTA pairs (256 x 256 tiles, cta_group::2): a pair tile takes ~0.9 of a 128 x 256 tile's time for twice
  // the rows (measured at 4096^2 x 8192: P 0.81 -> 0.89 of the cuBLAS burst, I 0.69 -> 0.81, W 0.75 ->
  // 0.84; each SM reads half the B operand from shared memory), over cap/2 pairs; so the estimate is
  // ceil(pair tiles / (cap / 2)) x 0.9 x (256 + 416).  Rows beyond M in a pair's second half are padding
  // (M = 384: single CTAs win).
  const long long tp = ((a.Mg + 255) / 256) * ((a.Ng + 255) / 256) * a.groups;
  const long long cost_pair = ((tp + cap / 2 - 1) / (cap / 2)) * (256 + 416) * 9 / 10;
  bool pair = a.Ng >= 256 && !splitk && cap >= 2 && cost_pair < (cost256 < cost128 ? cost256 : cost128);
  // a split weight update on pairs: s batch ranges per pair tile over cap/2 pairs against per 128 x 256
  // tile over cap CTAs (each range 1/s of a tile time; workspace bounds s): 1024^2 x 65536 splits 16 pair
  // tiles 4 ways on 74 pairs instead of 32 tiles 4 ways on 148 CTAs, at 0.9 of the tile time
  if (splitk && a.Ng >= 256 && cap >= 4) {
    const long long nk = (a.Kg + TC_BK - 1) / TC_BK;
    const long long fit = (long long)(ws_bytes / (size_t)(4LL * a.groups * a.Mg * a.Ng));
    const long long u2 = cap / 2;
    const long long s1 = std::min(std::min((long long)cap / t256, nk / 4), fit);
    const long long s2 = std::min(std::min(u2 / tp, nk / 4), fit);
    if (s1 >= 2 && s2 >= 2) {
      const long long c1 = ((t256 * s1 + cap - 1) / cap) * (256 + 416) * 10 / s1;
      const long long c2 = ((tp * s2 + u2 - 1) / u2) * (256 + 416) * 9 / s2;
      pair = c2 < c1;
    }
  }
  if (tune != nullptr && tune->pair == 1) pair = false;
  if (tune != nullptr && tune->pair == 2) pair = a.Ng >= 256;
  if (tune != nullptr && tune->bn == 128) pair = false;
  if (pair)
    return dtype == IPC_DT_F16 ? dispatch_mode<__half, 256, 1>(a, mode, act, dtype, s, ws, ws_bytes, tune)
                               : dispatch_mode<__nv_bfloat16, 256, 1>(a, mode, act, dtype, s, ws, ws_bytes, tune);
  if (dtype == IPC_DT_F16)
    return wide ? dispatch_mode<__half, 256, 0>(a, mode, act, dtype, s, ws, ws_bytes, tune)
                : dispatch_mode<__half, 128, 0>(a, mode, act, dtype, s, ws, ws_bytes, tune);
  return wide ? dispatch_mode<__nv_bfloat16, 256, 0>(a, mode, act, dtype, s, ws, ws_bytes, tune)
              : dispatch_mode<__nv_bfloat16, 128, 0>(a, mode, act, dtype, s, ws, ws_bytes, tune);
}

int set_max_ctas(int max_ctas) {
  if (max_ctas < 0) return set_error(IPC_ERR_ARG, "max_ctas must be >= 0 (got %d)", max_ctas);
  g_max_ctas.store(max_ctas, std::memory_order_relaxed);
  return IPC_OK;
}

int read_device_status(int* status, int clear) {
  int v = 0;
  cudaError_t err = cudaMemcpyFromSymbol(&v, g_device_status, sizeof(int));
  if (err != cudaSuccess) return set_error(IPC_ERR_CUDA, "device status read: %s", cudaGetErrorString(err));
  if (clear && v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int));
  }
  if (status) *status = v;
  return IPC_OK;
}

}  // namespace ipc
