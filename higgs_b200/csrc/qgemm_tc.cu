// qgemm_tc.cu -- W4 g64 quantized matmul for M >= 17 tokens on the tcgen05
// tensor cores (batched decode, speculative verify, prefill).
//
// Reference op replaced: ops::quantized_matmul (qwen3_next.rs:174-183) in its
// matrix form.  MLX evaluates many-token quantized matmuls by dequantizing the
// weights to the activation type first (qmm); so does this kernel:
// w = bf16(s*q + b) with one rounding (a bf16x2 fused multiply-add of the exact
// nibble value), then bf16 x bf16 -> f32 on the tensor cores.
//
// Work split (stream-K): the (tile, 64-wide k group) units of the whole matmul
// -- a tile is 128 weight rows x BN tokens -- are cut into one contiguous range
// per CTA, one CTA per SM, so every SM streams the same share of the weights
// whatever the tile count.  A tile split between CTAs is finished by the last
// of them, which adds the f32 partials in CTA order (the same bits whichever
// CTA ends last).
//
// Per CTA (448 threads):
//   * loader warp, lane 0: TMA streams the packed weight tile of each unit
//     (128 rows x 32 bytes) into a deep shared-memory ring, starting before the
//     grid dependency wait (weights never depend on the previous kernel);
//     lane 1: TMA brings the x tile (BN tokens x 64 k, 128-byte swizzle) into
//     its own ring, released by the MMA that read it;
//   * 8 dequant warps: warp w owns TMEM lanes 32(w%4).. and k half w/4; each
//     thread dequantizes 32 weights of its row (LOP3 / bf16x2 FMA / PRMT) and
//     writes them with tcgen05.st straight into a TMEM A-operand stage, so the
//     dequantized tile never passes through shared memory;
//   * MMA warp: one lane issues tcgen05.mma (A from TMEM, x from shared memory,
//     M=128, N=BN, K=16) x 4 per unit into one of two TMEM accumulators;
//     tcgen05.commit releases the A stage, the x stage and, at the end of a
//     tile, the accumulator;
//   * 4 epilogue warps read a finished accumulator (tcgen05.ld) while the MMA
//     already fills the other one: bf16 / f32 store, residual add, SwiGLU (gate
//     and up tiles share the CTA), or the f32 partial of a split tile.
// TMEM is allocated only after griddepcontrol.wait, so a kernel launched early
// never holds tensor memory that its predecessor still needs.  Every mbarrier
// wait is bounded (about 2 s, or at once after another CTA failed): on timeout
// the kernel records an error that higgs_tc_error reports and finishes.
#include <cuda.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"
#include "kernels.cuh"

namespace higgs {

namespace {

constexpr int kTcRows = 128;               // weight rows per tile (UMMA M)
constexpr int kTcDequant = 256;            // 8 dequant warps
constexpr int kMmaWarp = kTcDequant / 32;  // 8, 9: MMA issuers (even / odd units)
constexpr int kIssuers = 2;
constexpr int kLoadWarp = kMmaWarp + kIssuers;  // 10
constexpr int kEpiWarp0 = kLoadWarp + 1;        // 11..14
constexpr int kTcEpilogue = 128;
constexpr int kTcThreads = kTcDequant + 32 * (kIssuers + 1) + kTcEpilogue;
constexpr int kPkTile = kTcRows * 32;  // 128 rows x 64 packed nibbles = 4 KB
constexpr int kRing = 8;               // scale / bias units prefetched per dequant thread
constexpr int kSmemBudget = 200 * 1024;
constexpr int kTmemCols = 512;
constexpr int kTcMaxTiles = 16384;  // stream-K tile counters in the workspace
constexpr size_t kTcCounterBytes = kTcMaxTiles * sizeof(int);

// Per-instantiation pipeline shape.
template <int BN, bool SWIGLU>
struct TcCfg {
  static constexpr int NA = SWIGLU ? 2 : 1;  // weight tiles per unit (gate, up)
  static constexpr int kTileB = BN * 128;    // x tile: BN tokens x 64 bf16
  static constexpr int XS = (49152 / kTileB) > 8 ? 8 : (49152 / kTileB);
  static constexpr int kPk = NA * kPkTile;  // packed bytes per unit
  static constexpr int PS0 = (kSmemBudget - XS * kTileB) / kPk;
  static constexpr int PS = PS0 > 32 ? 32 : PS0;  // packed units in flight
  static constexpr int ACC = NA * BN;             // TMEM columns of one accumulator
  // accumulators: one per issuer, double-buffered across tiles when TMEM allows
  static constexpr int NB = 2 * kIssuers * ACC <= 256 ? 2 : 1;
  static constexpr int A0 = kIssuers * NB * ACC < 128 ? 128 : kIssuers * NB * ACC;  // first A column
  static constexpr int AS = (kTmemCols - A0) / (NA * 32);  // A-operand stages
  static constexpr size_t kSmem = (size_t)XS * kTileB + (size_t)PS * kPk + 1024;
  static_assert(A0 <= 256, "accumulators leave half of TMEM to the A stages");
  static_assert(AS >= 4 && XS >= 3 && PS >= 16, "pipeline depth");
  // more than half the SM's shared memory: one CTA per SM, so all of TMEM is ours
  static_assert(kSmem <= 227 * 1024 && kSmem > 114 * 1024, "one CTA per SM");
};

struct TcArgs {
  int M, K, N;
  int m_tiles, tiles;  // tile t = n_tile * m_tiles + m_tile
  int nseg;
  int seg_end[3];
  const uint16_t* s[3];
  const uint16_t* b[3];
  const uint16_t* s2;  // up projection (SwiGLU)
  const uint16_t* b2;
  uint16_t* y;
  float* y_f32;
  const uint16_t* residual;
  float* part;    // f32 partials of split tiles: 2 slots per CTA
  int* counters;  // one per tile, self-resetting
  int* err;
};

// ---- mbarrier / TMA / tcgen05 primitives -----------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
// Bounded wait for the completion of phase `parity`.  False (and *err set) on
// timeout; false at once when any CTA has already failed.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity, int* err) {
  const uint32_t a = smem_u32(bar);
  const long long t0 = clock64();
  for (unsigned it = 1;; ++it) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(a), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((it & 1023) == 0) {
      if (*reinterpret_cast<volatile int*>(err)) return false;
      if (clock64() - t0 > (1ll << 32)) break;  // ~2 s at 2 GHz
    }
  }
  atomicExch(err, 1);
  return false;
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_alloc(uint32_t* dst, int cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(cols)
               : "memory");
}
__device__ __forceinline__ void tc_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tc_dealloc(uint32_t taddr, int cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
// D[tmem] (+)= A[tmem] . B[smem]^T
__device__ __forceinline__ void tc_mma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::
          "r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accum)
      : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// 16 consecutive 32-bit columns of this thread's TMEM lane
__device__ __forceinline__ void tc_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tc_st16(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void epilogue_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kTcEpilogue) : "memory"); }
// true on every epilogue thread iff v is true on all of them
__device__ __forceinline__ bool epilogue_all(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, 1, %2, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(kTcEpilogue)
      : "memory");
  return r != 0;
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;            // leading byte offset (unused by swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;  // stride byte offset
  d |= (uint64_t)1 << 46;            // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;            // SWIZZLE_128B
  return d;
}

// 8 weights of one packed word -> 4 bf16 pairs in k order: w = bf16(s*q + b)
__device__ __forceinline__ void dequant8(uint32_t w, __nv_bfloat162 s2, __nv_bfloat162 b2, uint32_t* out) {
  const __nv_bfloat162 c128 = __floats2bfloat162_rn(128.f, 128.f);
  uint32_t p[4] = {lop3_and_or(w, 0x000F000Fu, 0x43004300u), lop3_and_or(w >> 4, 0x000F000Fu, 0x43004300u),
                   lop3_and_or(w >> 8, 0x000F000Fu, 0x43004300u), lop3_and_or(w >> 12, 0x000F000Fu, 0x43004300u)};
  uint32_t q[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    // (128 + q) - 128 = q exactly; then one rounding of s*q + b
    const __nv_bfloat162 qq = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&p[i]), c128);
    const __nv_bfloat162 r = __hfma2(s2, qq, b2);
    q[i] = *reinterpret_cast<const uint32_t*>(&r);
  }
  // q[i] = (w_i, w_{i+4}) -> k order (0,1) (2,3) (4,5) (6,7)
  out[0] = prmt(q[0], q[1], 0x5410);
  out[1] = prmt(q[2], q[3], 0x5410);
  out[2] = prmt(q[0], q[1], 0x7632);
  out[3] = prmt(q[2], q[3], 0x7632);
}

// Weight tiles of a unit: the packed rows [row0, row0 + 128) of one tensor, 64 k.
struct WMaps {
  CUtensorMap w[3];  // q | k | v segments (or the single tensor)
  CUtensorMap up;    // SwiGLU up projection
};

// Tile t -> row segment, its first row inside the segment, and the tile origin.
struct TilePos {
  int seg, row0, n0, m0;
};
template <int BN>
__device__ __forceinline__ TilePos tile_pos(const TcArgs& a, int t) {
  TilePos p;
  const int n_tile = t / a.m_tiles;
  p.m0 = (t - n_tile * a.m_tiles) * BN;
  p.n0 = n_tile * kTcRows;
  p.seg = 0;
  for (int i = 1; i < a.nseg; ++i)
    if (p.n0 >= a.seg_end[i - 1]) p.seg = i;
  p.row0 = p.n0 - (p.seg ? a.seg_end[p.seg - 1] : 0);
  return p;
}

// Units [begin(c), begin(c + 1)) belong to CTA c; owner(u) is the CTA holding unit u.
__device__ __forceinline__ long long unit_begin(long long U, int P, int c) { return (long long)c * U / P; }
__device__ __forceinline__ int unit_owner(long long U, int P, long long u) {
  return (int)(((u + 1) * P + U - 1) / U) - 1;
}

// 16 tokens of output row n from f32 accumulators (gate / up for SwiGLU).
template <bool SWIGLU>
__device__ __forceinline__ void tc_emit(const TcArgs& a, int n, int tok0, const float* g, const float* u) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int tok = tok0 + j;
    if (tok >= a.M) break;
    const size_t o = (size_t)tok * a.N + n;
    if constexpr (SWIGLU) {
      const float gv = round_bf(g[j]), uv = round_bf(u[j]);
      a.y[o] = f2bf(gv / (1.0f + expf(-gv)) * uv);
    } else {
      const float v = g[j];
      if (a.y_f32) a.y_f32[o] = v;
      if (a.y) {
        uint16_t rv = f2bf(v);
        if (a.residual) rv = f2bf(bf2f(rv) + bf2f(a.residual[o]));
        a.y[o] = rv;
      }
    }
  }
}

template <int BN, bool SWIGLU>
__global__ void __launch_bounds__(kTcThreads, 1)
    qgemm_tc_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ WMaps wm, TcArgs a) {
  using C = TcCfg<BN, SWIGLU>;
  constexpr int NA = C::NA, AS = C::AS, XS = C::XS, PS = C::PS, kPk = C::kPk, kTileB = C::kTileB;
  constexpr int ACC = C::ACC, A0 = C::A0, NB = C::NB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* xsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* pk = xsm + XS * kTileB;  // packed ring (1024-aligned)
  __shared__ __align__(8) uint64_t a_full[AS];
  __shared__ __align__(8) uint64_t a_empty[AS];
  __shared__ __align__(8) uint64_t x_full[XS];
  __shared__ __align__(8) uint64_t x_empty[XS];
  __shared__ __align__(8) uint64_t pk_full[PS];
  __shared__ __align__(8) uint64_t pk_empty[PS];
  __shared__ __align__(8) uint64_t acc_full[NB];
  __shared__ __align__(8) uint64_t acc_empty[NB];
  __shared__ __align__(8) uint64_t done_bar;
  __shared__ uint32_t tmem_base;
  __shared__ int is_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = a.K / 64;
  const int P = gridDim.x;
  const long long U = (long long)a.tiles * G;
  const long long ub = unit_begin(U, P, blockIdx.x), ue = unit_begin(U, P, blockIdx.x + 1);
  const int nst = (int)(ue - ub);
  const int t_first = (int)(ub / G), g_first = (int)(ub - (long long)t_first * G);

  if (threadIdx.x == 0) {
    for (int i = 0; i < AS; ++i) {
      mbar_init(&a_full[i], kTcDequant);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < XS; ++i) {
      mbar_init(&x_full[i], 1);
      mbar_init(&x_empty[i], 1);
    }
    for (int i = 0; i < PS; ++i) {
      mbar_init(&pk_full[i], 1);
      mbar_init(&pk_empty[i], kTcDequant);
    }
    for (int i = 0; i < NB; ++i) {
      mbar_init(&acc_full[i], kIssuers);
      mbar_init(&acc_empty[i], kTcEpilogue);
    }
    mbar_init(&done_bar, kIssuers);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  // ---- before the grid dependency wait: weights only ----
  // loader lane 0 cursor (unit -> tile / group) and the first PS packed units
  int lg = g_first, lt = t_first;
  TilePos lp = tile_pos<BN>(a, lt);
  auto load_pk = [&](int i) {
    const int slot = i % PS;
    mbar_arrive_expect_tx(&pk_full[slot], kPk);
    uint8_t* dst = pk + slot * kPk;
    tma_load_2d(dst, &wm.w[lp.seg], lg * 32, lp.row0, &pk_full[slot]);
    if constexpr (SWIGLU) tma_load_2d(dst + kPkTile, &wm.up, lg * 32, lp.row0, &pk_full[slot]);
    if (++lg == G) {
      lg = 0;
      lp = tile_pos<BN>(a, ++lt);
    }
  };
  if (warp == kLoadWarp && lane == 0)
    for (int i = 0; i < PS && i < nst; ++i) load_pk(i);

  // dequant threads: row r of the tile, k half hf; scale / bias register ring
  const int q4 = warp & 3, hf = (warp >> 2) & 1, r = q4 * 32 + lane;
  const bool dequant = warp < kMmaWarp;
  const bool issuer = warp >= kMmaWarp && warp < kMmaWarp + kIssuers;
  // raw bf16 loads, first used kRing units later: combining them at fetch time would
  // stall the thread on each load's latency
  __nv_bfloat16 sr[kRing][NA], br[kRing][NA];
  int ft = t_first, fg = g_first;
  const uint16_t *S = nullptr, *Bb = nullptr, *S2 = nullptr, *B2 = nullptr;
  auto sb_rows = [&]() {
    const TilePos p = tile_pos<BN>(a, ft);
    const size_t off = (size_t)(p.row0 + r) * G;
    S = a.s[p.seg] + off;
    Bb = a.b[p.seg] + off;
    if constexpr (SWIGLU) {
      S2 = a.s2 + (size_t)(p.n0 + r) * G;
      B2 = a.b2 + (size_t)(p.n0 + r) * G;
    }
  };
  auto fetch_sb = [&](int d) {  // the cursor's unit into ring slot d, then advance
    sr[d][0] = reinterpret_cast<const __nv_bfloat16*>(S)[fg];
    br[d][0] = reinterpret_cast<const __nv_bfloat16*>(Bb)[fg];
    if constexpr (SWIGLU) {
      sr[d][1] = reinterpret_cast<const __nv_bfloat16*>(S2)[fg];
      br[d][1] = reinterpret_cast<const __nv_bfloat16*>(B2)[fg];
    }
    if (++fg == G) {
      fg = 0;
      ++ft;
      if (ft < a.tiles) sb_rows();
    }
  };
  if (dequant) {
    sb_rows();
#pragma unroll
    for (int d = 0; d < kRing; ++d)
      if (d < nst) fetch_sb(d);
  }

  pdl_wait();  // x, the residual and the workspace come from earlier kernels
  if (warp == kMmaWarp) {
    tc_alloc(&tmem_base, kTmemCols);
    tc_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_base;
  pdl_launch();

  if (warp == kLoadWarp) {
    if (lane == 0) {
      // ---- packed weights: refill each slot once the dequant warps drained it ----
      for (int i = PS; i < nst; ++i) {
        if (!mbar_wait(&pk_empty[i % PS], ((i / PS) - 1) & 1, a.err)) break;
        load_pk(i);
      }
      for (int p = 0; p < PS && p < nst; ++p)  // own copies in flight (no-op unless a wait failed)
        mbar_wait(&pk_full[p], ((nst - 1 - p) / PS) & 1, a.err);
    } else if (lane == 1) {
      // ---- x tiles: refill each slot once the MMAs that read it completed ----
      int g = g_first, t = t_first;
      int m0 = tile_pos<BN>(a, t).m0;
      for (int i = 0; i < nst; ++i) {
        const int xs = i % XS;
        if (i >= XS && !mbar_wait(&x_empty[xs], ((i / XS) - 1) & 1, a.err)) break;
        mbar_arrive_expect_tx(&x_full[xs], kTileB);
        tma_load_2d(xsm + xs * kTileB, &xmap, g * 64, m0, &x_full[xs]);
        if (++g == G) {
          g = 0;
          m0 = tile_pos<BN>(a, ++t).m0;
        }
      }
      for (int p = 0; p < XS && p < nst; ++p) mbar_wait(&x_full[p], ((nst - 1 - p) / XS) & 1, a.err);
    }
    __syncwarp();
  } else if (issuer) {
    // ---- MMA: issuer w takes the units of parity w into its own accumulator, so one
    // issuer's barrier waits and commits overlap the other's MMAs; commits release the
    // A / x stages and, at the end of a tile, the issuer's share of the accumulator ----
    if (lane == 0) {
      const int w = warp - kMmaWarp;
      const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                             ((uint32_t)(kTcRows >> 4) << 24);
      int g = g_first, s = 0;
      bool ok = true, started = false;
      for (int i = 0; i < nst && ok; ++i) {
        const int b = NB == 2 ? (s & 1) : 0;
        const bool last = i == nst - 1 || g == G - 1;
        // before touching (or signalling) accumulator b again, its previous tile must be read
        const bool need_empty = !started && s >= NB && ((i & 1) == w || last);
        if (need_empty) ok = mbar_wait(&acc_empty[b], ((s / NB) - 1) & 1, a.err);
        if (ok && (i & 1) == w) {
          const int slot = i % AS, xs = i % XS;
          ok = mbar_wait(&a_full[slot], (i / AS) & 1, a.err);
          ok = ok && mbar_wait(&x_full[xs], (i / XS) & 1, a.err);
          if (!ok) break;
          tc_fence_after();
          const uint32_t sbx = smem_u32(xsm + xs * kTileB);
          const uint32_t d = tbase + (w * NB + b) * ACC;
#pragma unroll
          for (int t = 0; t < NA; ++t)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              tc_mma_ts(d + t * BN, tbase + A0 + slot * (NA * 32) + t * 32 + kk * 8, sw128_desc(sbx + kk * 32),
                        idesc, (started || kk > 0) ? 1u : 0u);
          tc_commit(&a_empty[slot]);
          tc_commit(&x_empty[xs]);
          started = true;
        }
        if (ok && last) {  // this issuer's share of the tile is complete (or empty)
          if (started)
            tc_commit(&acc_full[b]);
          else
            mbar_arrive(&acc_full[b]);
          started = false;
          ++s;
        }
        if (++g == G) g = 0;
      }
      tc_commit(&done_bar);
    }
    __syncwarp();
  } else if (dequant) {
    // ---- dequant: packed smem -> bf16 pairs -> TMEM A stage ----
    const uint32_t tl = tbase + ((uint32_t)(q4 * 32) << 16) + A0 + hf * 16;
    bool ok = true;
    for (int i0 = 0; i0 < nst && ok; i0 += kRing) {
#pragma unroll
      for (int d = 0; d < kRing; ++d) {
        const int i = i0 + d;
        if (i >= nst) break;
        const int ps = i % PS, slot = i % AS;
        // warp-uniform outcome: the tcgen05 st / wait below need the whole warp
        if (!(ok = __all_sync(0xffffffffu, mbar_wait(&pk_full[ps], (i / PS) & 1, a.err)))) break;
        uint4 wv[NA];
#pragma unroll
        for (int t = 0; t < NA; ++t)
          wv[t] = *reinterpret_cast<const uint4*>(pk + ps * kPk + t * kPkTile + r * 32 + hf * 16);
        if (i >= AS && !(ok = __all_sync(0xffffffffu, mbar_wait(&a_empty[slot], ((i / AS) - 1) & 1, a.err)))) break;
        tc_fence_after();
#pragma unroll
        for (int t = 0; t < NA; ++t) {
          const __nv_bfloat162 s2 = __bfloat162bfloat162(sr[d][t]);
          const __nv_bfloat162 b2 = __bfloat162bfloat162(br[d][t]);
          const uint32_t* w = &wv[t].x;
          uint32_t v[16];
#pragma unroll
          for (int j = 0; j < 4; ++j) dequant8(w[j], s2, b2, v + 4 * j);
          tc_st16(tl + slot * (NA * 32) + t * 32, v);
        }
        // release the packed slot only once its words have been consumed: the refill is an
        // async-proxy (TMA) write, which the barrier does not order behind a load in flight
        mbar_arrive(&pk_empty[ps]);
        tc_wait_st();
        tc_fence_before();
        mbar_arrive(&a_full[slot]);
        if (i + kRing < nst) fetch_sb(d);
      }
    }
  } else {
    // ---- epilogue: one finished tile at a time, TMEM lanes 32(warp % 4).. ----
    const int ep = threadIdx.x - kEpiWarp0 * 32;
    const uint32_t tl = tbase + ((uint32_t)(q4 * 32) << 16);
    int s = 0;
    // the tile's columns c0..c0+15 of gate (and up): the issuers' accumulators added
    float gv[16], uv[16];
    auto read_acc = [&](uint32_t tacc0, bool both, int c0) {
      float g2[16], u2[16];
      tc_ld16(tacc0 + c0, gv);
      if constexpr (SWIGLU) tc_ld16(tacc0 + BN + c0, uv);
      if (both) {
        tc_ld16(tacc0 + NB * ACC + c0, g2);
        if constexpr (SWIGLU) tc_ld16(tacc0 + NB * ACC + BN + c0, u2);
      }
      tc_wait_ld();
      if (both) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          gv[j] += g2[j];
          if constexpr (SWIGLU) uv[j] += u2[j];
        }
      }
    };
    for (int t = t_first; (long long)t * G < ue; ++t, ++s) {
      const int b = NB == 2 ? (s & 1) : 0;
      if (!epilogue_all(mbar_wait(&acc_full[b], (s / NB) & 1, a.err))) break;
      tc_fence_after();
      const TilePos p = tile_pos<BN>(a, t);
      const int n = p.n0 + r;
      const long long tu = (long long)t * G;
      const int c_lo = unit_owner(U, P, tu), c_hi = unit_owner(U, P, tu + G - 1);
      // units of this tile held here: [i0, i1]; issuer w owns the ones of parity w
      const int i0 = (int)std::max<long long>(0, tu - ub), i1 = (int)std::min<long long>(nst - 1, tu + G - 1 - ub);
      const bool w0 = i1 > i0 || (i0 & 1) == 0, w1 = i1 > i0 || (i0 & 1) == 1;
      const uint32_t tacc = tl + (w0 ? 0 : NB * ACC) + b * ACC;  // the first contributing issuer
      const bool both = w0 && w1;
      if (c_lo == c_hi) {  // the whole tile is ours
        for (int c0 = 0; c0 < BN && p.m0 + c0 < a.M; c0 += 16) {
          read_acc(tacc, both, c0);
          tc_emit<SWIGLU>(a, n, p.m0 + c0, gv, uv);
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[b]);
        continue;
      }
      // split tile: publish this CTA's partial; the last contributor finishes it
      constexpr size_t kPart = (size_t)NA * kTcRows * BN;
      float* mine = a.part + ((size_t)blockIdx.x * 2 + (t == t_first ? 0 : 1)) * kPart;
      for (int c0 = 0; c0 < BN && p.m0 + c0 < a.M; c0 += 16) {
        read_acc(tacc, both, c0);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          mine[(size_t)(c0 + j) * kTcRows + r] = gv[j];
          if constexpr (SWIGLU) mine[(size_t)(BN + c0 + j) * kTcRows + r] = uv[j];
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[b]);
      __threadfence();
      epilogue_sync();
      if (ep == 0) is_last = atomicAdd(a.counters + t, 1) == c_hi - c_lo;
      epilogue_sync();
      if (is_last) {
        __threadfence();
        for (int c0 = 0; c0 < BN && p.m0 + c0 < a.M; c0 += 16) {
          float gv[16], uv[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) gv[j] = uv[j] = 0.f;
          for (int c = c_lo; c <= c_hi; ++c) {  // CTA order
            const int slot = unit_begin(U, P, c) >= tu ? 0 : 1;  // first tile of CTA c, or its last
            const float* q = a.part + ((size_t)c * 2 + slot) * kPart;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              gv[j] += __ldcg(q + (size_t)(c0 + j) * kTcRows + r);
              if constexpr (SWIGLU) uv[j] += __ldcg(q + (size_t)(BN + c0 + j) * kTcRows + r);
            }
          }
          tc_emit<SWIGLU>(a, n, p.m0 + c0, gv, uv);
        }
        if (ep == 0) a.counters[t] = 0;
      }
      epilogue_sync();
    }
  }
  __syncthreads();
  if (warp == kMmaWarp) {
    mbar_wait(&done_bar, 0, a.err);
    __syncwarp();
    tc_fence_after();
    tc_dealloc(tbase, kTmemCols);
  }
}

// ---- host side ---------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// x [M, K] bf16 as TMA tiles of 64 k x BN tokens, 128-byte swizzle (cached per buffer)
bool x_tensor_map(const void* x, int M, int K, int BN, CUtensorMap* out) {
  static std::mutex mu;
  static std::map<std::tuple<const void*, int, int, int>, CUtensorMap> cache;
  std::lock_guard<std::mutex> lk(mu);
  auto key = std::make_tuple(x, M, K, BN);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return true;
  }
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  CUtensorMap m;
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
  const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)BN};
  const cuuint32_t estr[2] = {1, 1};
  if (fn(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), dims, strides, box, estr,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  if (cache.size() > 4096) cache.clear();
  cache[key] = m;
  *out = m;
  return true;
}

// packed weights [rows, K/2 bytes] as TMA tiles of 32 bytes (64 k) x 128 rows (cached)
bool w_tensor_map(const void* w, int rows, int K, CUtensorMap* out) {
  static std::mutex mu;
  static std::map<std::tuple<const void*, int, int>, CUtensorMap> cache;
  std::lock_guard<std::mutex> lk(mu);
  auto key = std::make_tuple(w, rows, K);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return true;
  }
  EncodeTiledFn fn = encode_fn();
  if (!fn || ((uintptr_t)w & 15)) return false;
  CUtensorMap m;
  const cuuint64_t dims[2] = {(cuuint64_t)K / 2, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)K / 2};
  const cuuint32_t box[2] = {32, (cuuint32_t)kTcRows};
  const cuuint32_t estr[2] = {1, 1};
  if (fn(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(w), dims, strides, box, estr,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  if (cache.size() > 65536) cache.clear();
  cache[key] = m;
  *out = m;
  return true;
}

int* tc_err_ptr() {
  static int* p = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    if (cudaMalloc(&p, sizeof(int)) == cudaSuccess) cudaMemset(p, 0, sizeof(int));
  });
  return p;
}

int tc_sms() {
  static int n = 0;
  static std::once_flag once;
  std::call_once(once, [] {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 1)
      n = 148;
  });
  return n;
}

// tokens per tile: 32 / 64 / 128 (SwiGLU stops at 64: two double-buffered
// accumulators of gate and up must leave TMEM room for the A stages)
int tc_bn(int M, bool swiglu) { return M <= 32 ? 32 : (M <= 64 || swiglu ? 64 : 128); }

template <int BN, bool SWIGLU>
cudaError_t launch_bn(const CUtensorMap& map, const WMaps& wm, const TcArgs& a, int P, cudaStream_t st) {
  constexpr size_t smem = TcCfg<BN, SWIGLU>::kSmem;
  auto k = qgemm_tc_kernel<BN, SWIGLU>;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  return launch_pdl(k, dim3(P), dim3(kTcThreads), smem, st, map, wm, a);
}

}  // namespace

// K % 256 == 0, N (and every row segment) % 128 == 0, x 16-byte aligned, no fused norm.
bool qgemm_tc_supported(const QLinArgs& a) {
  if (a.M < 1 || a.K % 256 || a.N % kTcRows || ((uintptr_t)a.x & 15) || a.norm_w || a.moe_items) return false;
  if (a.nseg > 1)
    for (int i = 0; i < a.nseg; ++i)
      if (a.seg_end[i] % kTcRows) return false;
  return encode_fn() != nullptr;
}

// A fixed counter region (one int per tile, up to kTcMaxTiles, zero between
// calls), then two f32 partial tiles per CTA.  The fixed region lets matmuls of
// every shape -- and the stream-K GEMV, whose counters sit in the same bytes --
// share one workspace back to back on a stream.
size_t qgemm_tc_workspace(int M, int K, int N, bool swiglu) {
  (void)K;
  (void)N;
  const int BN = tc_bn(M, swiglu);
  return kTcCounterBytes + (size_t)tc_sms() * 2 * (swiglu ? 2 : 1) * kTcRows * BN * sizeof(float);
}

cudaError_t launch_qgemm_tc(const QLinArgs& q, int epi, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (!qgemm_tc_supported(q)) return cudaErrorInvalidValue;
  const bool swiglu = epi == EPI_SWIGLU;
  const int BN = tc_bn(q.M, swiglu);
  CUtensorMap map;
  if (!x_tensor_map(q.x, q.M, q.K, BN, &map)) return cudaErrorInvalidValue;
  TcArgs a{};
  a.M = q.M;
  a.K = q.K;
  a.N = q.N;
  a.m_tiles = (q.M + BN - 1) / BN;
  a.tiles = (q.N / kTcRows) * a.m_tiles;
  a.nseg = q.nseg > 1 ? q.nseg : 1;
  const uint32_t* w[3] = {q.w, nullptr, nullptr};
  if (q.nseg > 1) {
    for (int i = 0; i < 3; ++i) {
      a.seg_end[i] = q.seg_end[i];
      w[i] = q.wseg[i];
      a.s[i] = q.sseg[i];
      a.b[i] = q.bseg[i];
    }
  } else {
    a.s[0] = q.s;
    a.b[0] = q.b;
  }
  a.s2 = q.s2;
  a.b2 = q.b2;
  a.y = q.y;
  a.y_f32 = q.y_f32;
  a.residual = q.residual;
  a.err = tc_err_ptr();
  if (!a.err) return cudaErrorMemoryAllocation;
  WMaps wm;
  memset(&wm, 0, sizeof(wm));
  for (int i = 0; i < a.nseg; ++i) {
    const int rows = a.nseg > 1 ? a.seg_end[i] - (i ? a.seg_end[i - 1] : 0) : q.N;
    if (!w_tensor_map(w[i], rows, q.K, &wm.w[i])) return cudaErrorInvalidValue;
  }
  if (swiglu && !w_tensor_map(q.w2, q.N, q.K, &wm.up)) return cudaErrorInvalidValue;
  // stream-K over every SM when the workspace allows it, else one CTA per tile
  const long long U = (long long)a.tiles * (q.K / 64);
  int P = a.tiles;
  const size_t need = qgemm_tc_workspace(q.M, q.K, q.N, swiglu);
  if (ws && ws_bytes >= need && ((uintptr_t)ws & 255) == 0 && a.tiles <= kTcMaxTiles) {
    P = (int)std::min<long long>(tc_sms(), (U + 3) / 4);
    a.counters = static_cast<int*>(ws);
    a.part = reinterpret_cast<float*>(static_cast<char*>(ws) + kTcCounterBytes);
  }
  if (P < 1) P = 1;
  if (swiglu) {
    if (BN == 32) return launch_bn<32, true>(map, wm, a, P, st);
    return launch_bn<64, true>(map, wm, a, P, st);
  }
  if (BN == 32) return launch_bn<32, false>(map, wm, a, P, st);
  if (BN == 64) return launch_bn<64, false>(map, wm, a, P, st);
  return launch_bn<128, false>(map, wm, a, P, st);
}

// one-time host state (error flag, driver entry point, SM count): call before any stream capture
void qgemm_tc_prepare() {
  tc_err_ptr();
  encode_fn();
  tc_sms();
}

int qgemm_tc_error_and_clear() {
  int* p = tc_err_ptr();
  if (!p) return 0;
  int v = 0;
  cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost);
  if (v) cudaMemset(p, 0, sizeof(int));
  return v;
}

}  // namespace higgs

extern "C" int higgs_tc_error(int* out) {
  HG_CHECK_ARG(out, "higgs_tc_error: null argument");
  *out = higgs::qgemm_tc_error_and_clear();
  return HIGGS_OK;
}
