// qgemm_tc.cu -- W4 g64 quantized matmul for M >= 17 tokens on the tcgen05
// tensor cores (batched decode, speculative verify, prefill).
//
// Reference op replaced: ops::quantized_matmul (qwen3_next.rs:174-183) in its
// matrix form.  MLX evaluates many-token quantized matmuls by dequantizing the
// weights to the activation type first (qmm); so does this kernel:
// w = bf16(s*q + b) with one rounding (a bf16x2 fused multiply-add of the exact
// nibble value), then bf16 x bf16 -> f32 on the tensor cores.
//
// One CTA computes a 128-row x BN-token tile over a slice of K (split-K when the
// tile count alone cannot fill the GPU):
//   * loader warp, lane 0: TMA streams the packed weight tile (128 rows x 32
//     bytes per 64-wide k group) into an 8-stage shared-memory ring, starting
//     before the grid dependency wait (weights never depend on the previous
//     kernel); lane 1: TMA brings the x tiles (BN tokens x 64 k, 128-byte swizzle)
//     into their own ring, each as soon as the MMAs of the stage XS earlier completed;
//   * 8 producer warps: thread (row, half) takes 16 packed bytes per operand tile from
//     the ring, dequantizes them with LOP3 / bf16x2 FMA / PRMT and stores the bf16 row
//     slice in the 128-byte-swizzled K-major layout the MMA reads;
//   * NA x NS MMA warps: one lane each issues tcgen05.mma (M=128, N=BN, K=16) x 4 per
//     group for one operand tile (gate or up) and the stages i = j (mod NS) into its own
//     TMEM accumulator; tcgen05.commit releases the operand and x slots;
//   * the producers then read TMEM (tcgen05.ld, 32 lanes per warp quarter), add the NS
//     accumulators in order and run the epilogue: bf16 / f32 store, residual add, SwiGLU
//     (gate and up tiles share the CTA), or a split-K partial reduced in split order by
//     the last CTA.
// TMEM is allocated only after griddepcontrol.wait, so a kernel launched early
// never holds tensor memory that its predecessor still needs.  Every mbarrier
// wait is bounded (about 2 s): on timeout the kernel records an error that
// higgs_tc_error reports, and finishes.
#include <cuda.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"
#include "kernels.cuh"
#include "tcgen05.cuh"

namespace higgs {

namespace {

constexpr int kTcRows = 128;       // weight rows per tile (UMMA M)
constexpr int kTcProducers = 256;      // 8 warps, thread = (row, half of 64 k)
// MMA-issuing warps: one tcgen05.mma issue costs a thread ~140 SM cycles (~190 with a
// commit per stage) whatever the shape, and several issuing warps overlap (measured on
// B200 with higgs_diag_tc_mma_rate: 1 / 2 / 4 warps 142 / 71 / 40 cycles per M=128 x N=32
// MMA), so one issuing thread capped a 64-k weight stage (4 MMAs) at ~770 cycles.  Each
// operand tile (gate, up) has its own warps, and NS warps per tile take the stages
// i = j (mod NS) into their own TMEM accumulators; NS divides the operand ring depth, so a
// ring slot is always consumed by the same warps (its parity waits stay exact).  The
// epilogue adds a tile's NS accumulators in order j = 0, 1, ... (a fixed summation order).
constexpr int tc_as(bool swiglu) { return swiglu ? 3 : 4; }  // bf16 operand stages
// x tiles have their own ring, deeper than the operand ring: a tile is requested as soon as
// the MMAs of the stage XS earlier completed, instead of when its operand slot frees (that
// put an L2 -> shared round trip into every slot cycle).  NS divides XS (fixed warps per slot).
constexpr int tc_xs(int BN, bool swiglu) { return swiglu ? (BN <= 64 ? 6 : (BN <= 128 ? 3 : 2)) : (BN <= 128 ? 8 : 4); }
// the largest stage interleave (the operand ring depth, else 2, else 1) that divides both
// rings and fits TMEM
constexpr int tc_ns(int BN, bool swiglu) {
  const int na = swiglu ? 2 : 1, as = tc_as(swiglu), xs = tc_xs(BN, swiglu);
  if (xs % as == 0 && na * as * BN <= 512) return as;
  if (as % 2 == 0 && xs % 2 == 0 && na * 2 * BN <= 512) return 2;
  return 1;
}
int tc_sms();
// token-tile width: 256 tokens per MMA (each dequantized weight tile serves twice as many
// tokens) when that still gives every SM two tiles without a K split; measured on B200: the
// 2048-token gate/up of Qwen3-8B 700 -> 475 us, but 256- and 512-token prefills of
// Qwen3-1.7B slower with too few tiles
inline int tc_bn(int M, int N) {
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  if (M <= 128 || (long long)(N / kTcRows) * ((M + 255) / 256) < 2LL * tc_sms()) return 128;
  return 256;
}
constexpr int tc_mma_warps(int BN, bool swiglu) { return (swiglu ? 2 : 1) * tc_ns(BN, swiglu); }
constexpr int tc_threads(int BN, bool swiglu) { return kTcProducers + 32 * (tc_mma_warps(BN, swiglu) + 1); }
constexpr int kTileA = kTcRows * 128;  // 128 rows x 64 bf16 = 16 KB
constexpr int kPkTile = kTcRows * 32;  // 128 rows x 64 packed nibbles = 4 KB
constexpr int kPkStages = 8;           // packed weight stages in flight (TMA)
constexpr int kRing = 8;               // scale / bias groups prefetched per producer thread
constexpr int kTcMaxTiles = 16384;     // split-K tile counters in the workspace
constexpr size_t kTcCounterBytes = kTcMaxTiles * sizeof(int);

struct TcArgs {
  int M, K, N;
  int nseg;
  int seg_end[3];
  const uint32_t* w[3];
  const uint16_t* s[3];
  const uint16_t* b[3];
  const uint32_t* w2;  // up projection (SwiGLU)
  const uint16_t* s2;
  const uint16_t* b2;
  uint16_t* y;
  float* y_f32;
  const uint16_t* residual;
  int splits, groups_per_split;
  float* part;    // split-K partials
  int* counters;  // one per (n tile, m tile), self-resetting
  int* err;
};

__device__ __forceinline__ void producers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kTcProducers) : "memory"); }

// 8 weights of one packed word -> 16 bytes of bf16 in k order: w = bf16(s*q + b)
__device__ __forceinline__ uint4 dequant8(uint32_t w, __nv_bfloat162 s2, __nv_bfloat162 b2) {
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
  return make_uint4(prmt(q[0], q[1], 0x5410), prmt(q[2], q[3], 0x5410), prmt(q[0], q[1], 0x7632),
                    prmt(q[2], q[3], 0x7632));
}

// Weight tiles of a CTA: the packed rows [row0, row0 + 128) of one tensor, 64 k per stage.
struct WMaps {
  CUtensorMap w[3];  // q | k | v segments (or the single tensor)
  CUtensorMap up;    // SwiGLU up projection
};

template <int BN, bool SWIGLU>
__global__ void __launch_bounds__(tc_threads(BN, SWIGLU), 1)
    qgemm_tc_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ WMaps wm, TcArgs a) {
  constexpr int NA = SWIGLU ? 2 : 1;
  constexpr int AS = tc_as(SWIGLU);  // bf16 operand stages
  constexpr int kTileB = BN * 128;
  constexpr int XS = tc_xs(BN, SWIGLU);
  constexpr int kStage = NA * kTileA;
  constexpr int kPk = NA * kPkTile;  // packed bytes per stage
  constexpr int NS = tc_ns(BN, SWIGLU);         // stage interleave per operand tile
  constexpr int NMW = tc_mma_warps(BN, SWIGLU);  // NA x NS issuing warps
  static_assert(AS % NS == 0 && XS % NS == 0, "a ring slot maps to fixed warps");
  // accumulator (j, t) at TMEM column (j * NA + t) * BN
  constexpr int TCOLS = (NMW * BN <= 32) ? 32 : (NMW * BN <= 64) ? 64 : (NMW * BN <= 128) ? 128
                        : (NMW * BN <= 256) ? 256 : 512;
  static_assert(NMW * BN <= 512, "TMEM columns");
  constexpr int HC = BN / 2;  // accumulator columns read per producer warp
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* xr = smem + AS * kStage;  // x ring (1024-aligned: every tile size is a multiple of 1024)
  uint8_t* pk = xr + XS * kTileB;     // packed ring
  __shared__ __align__(8) uint64_t full_bar[AS];
  __shared__ __align__(8) uint64_t empty_bar[AS];
  __shared__ __align__(8) uint64_t x_full[XS];
  __shared__ __align__(8) uint64_t x_empty[XS];
  __shared__ __align__(8) uint64_t pk_full[kPkStages];
  __shared__ __align__(8) uint64_t pk_empty[kPkStages];
  __shared__ __align__(8) uint64_t done_bar;
  __shared__ uint32_t tmem_base;
  __shared__ int is_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tile = blockIdx.x, m_tile = blockIdx.y, split = blockIdx.z;
  const int n0 = n_tile * kTcRows, m0 = m_tile * BN;
  const int G = a.K / 64;
  const int g0 = split * a.groups_per_split;
  const int g1 = min(G, g0 + a.groups_per_split);
  const int nst = g1 - g0;

  int seg = 0;
  for (int i = 1; i < a.nseg; ++i)
    if (n0 >= a.seg_end[i - 1]) seg = i;
  const int row0 = n0 - (seg ? a.seg_end[seg - 1] : 0);

  if (threadIdx.x == 0) {
    for (int i = 0; i < AS; ++i) {
      mbar_init(&full_bar[i], kTcProducers);
      mbar_init(&empty_bar[i], NA);  // one commit per operand tile's warp
    }
    for (int i = 0; i < XS; ++i) {
      mbar_init(&x_full[i], 1);
      mbar_init(&x_empty[i], NA);
    }
    for (int i = 0; i < kPkStages; ++i) {
      mbar_init(&pk_full[i], 1);
      mbar_init(&pk_empty[i], kTcProducers);
    }
    mbar_init(&done_bar, NMW);  // one final commit per MMA warp
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  const int pid = threadIdx.x;
  const int r = pid >> 1, hf = pid & 1;
  const bool producer = pid < kTcProducers;
  const int mma_warp = kTcProducers / 32, load_warp = mma_warp + NMW;

  // weights never depend on the previous kernel: the loader fills the whole packed
  // ring before the grid dependency wait (no waits needed for the first pass)
  const CUtensorMap* wmap = &wm.w[seg];
  auto load_stage = [&](int i) {
    const int slot = i % kPkStages;
    mbar_arrive_expect_tx(&pk_full[slot], kPk);
    uint8_t* dst = pk + slot * kPk;
    tma_load_2d(dst, wmap, (g0 + i) * 32, row0, &pk_full[slot]);
    if constexpr (SWIGLU) tma_load_2d(dst + kPkTile, &wm.up, (g0 + i) * 32, row0, &pk_full[slot]);
  };
  if (warp == load_warp && lane == 0)
    for (int i = 0; i < kPkStages && i < nst; ++i) load_stage(i);

  // scales / biases: a small register ring, also before the wait
  const uint16_t* S = a.s[seg] + (size_t)(row0 + r) * G;
  const uint16_t* Bb = a.b[seg] + (size_t)(row0 + r) * G;
  const uint16_t* S2 = SWIGLU ? a.s2 + (size_t)(row0 + r) * G : nullptr;
  const uint16_t* B2 = SWIGLU ? a.b2 + (size_t)(row0 + r) * G : nullptr;
  // raw bf16 loads, first used kRing groups later (combining them at fetch time would
  // stall the thread on each load)
  __nv_bfloat16 sr[kRing][NA], br[kRing][NA];
  auto fetch_sb = [&](int i, int d) {
    const int g = g0 + i;
    sr[d][0] = reinterpret_cast<const __nv_bfloat16*>(S)[g];
    br[d][0] = reinterpret_cast<const __nv_bfloat16*>(Bb)[g];
    if constexpr (SWIGLU) {
      sr[d][1] = reinterpret_cast<const __nv_bfloat16*>(S2)[g];
      br[d][1] = reinterpret_cast<const __nv_bfloat16*>(B2)[g];
    }
  };
  if (producer) {
#pragma unroll
    for (int d = 0; d < kRing; ++d)
      if (d < nst) fetch_sb(d, d);
  }

  pdl_wait();  // x and the residual come from the previous kernel
  if (warp == mma_warp) {
    tc_alloc(&tmem_base, TCOLS);
    tc_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_base;
  pdl_launch();

  if (warp == load_warp) {
    // ---------------- loaders: lane 0 refills each packed weight slot once the producers
    // drained it; lane 1 brings each x tile once the MMAs of that stage slot are done
    if (lane == 0) {
      for (int i = kPkStages; i < nst; ++i) {
        mbar_wait(&pk_empty[i % kPkStages], ((i / kPkStages) - 1) & 1, a.err);
        load_stage(i);
      }
    } else if (lane == 1) {
      for (int i = 0; i < nst; ++i) {
        const int xs = i % XS;
        if (i >= XS) mbar_wait(&x_empty[xs], ((i / XS) - 1) & 1, a.err);
        mbar_arrive_expect_tx(&x_full[xs], kTileB);
        tma_load_2d(xr + xs * kTileB, &xmap, (g0 + i) * 64, m0, &x_full[xs]);
      }
    }
    __syncwarp();
  } else if (warp >= mma_warp && warp < load_warp) {
    // ---------------- MMA warps: warp (j, t) issues operand tile t of the stages i = j (mod NS)
    // into its own accumulator; its commit is one of the NA arrivals that release the stage
    const int mw = warp - mma_warp, tj = mw / NA, tt = mw % NA;
    if (lane == 0) {
      const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                             ((uint32_t)(kTcRows >> 4) << 24);
      const uint32_t tacc = tbase + (uint32_t)(tj * NA + tt) * BN;
      for (int i = tj; i < nst; i += NS) {
        const int slot = i % AS, xs = i % XS;
        mbar_wait(&x_full[xs], (i / XS) & 1, a.err);
        mbar_wait(&full_bar[slot], (i / AS) & 1, a.err);
        tc_fence_after();
        const uint32_t sbx = smem_u32(xr + xs * kTileB);
        const uint32_t sa = smem_u32(smem + slot * kStage + tt * kTileA);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc_mma(tacc, sw128_desc(sa + kk * 32), sw128_desc(sbx + kk * 32), idesc, (i >= NS || kk > 0) ? 1u : 0u);
        tc_commit(&empty_bar[slot]);
        tc_commit(&x_empty[xs]);
      }
      tc_commit(&done_bar);
    }
    __syncwarp();
  } else if (producer) {
    // ---------------- producers: packed smem -> bf16 swizzled A tiles ----------------
    for (int i0 = 0; i0 < nst; i0 += kRing) {
#pragma unroll
      for (int d = 0; d < kRing; ++d) {
        const int i = i0 + d;
        if (i >= nst) break;
        const int ps = i % kPkStages, slot = i % AS;
        mbar_wait(&pk_full[ps], (i / kPkStages) & 1, a.err);
        uint4 wv[NA];
#pragma unroll
        for (int t = 0; t < NA; ++t)
          wv[t] = *reinterpret_cast<const uint4*>(pk + ps * kPk + t * kPkTile + r * 32 + hf * 16);
        if (i >= AS) mbar_wait(&empty_bar[slot], ((i / AS) - 1) & 1, a.err);
        uint8_t* st = smem + slot * kStage;
#pragma unroll
        for (int t = 0; t < NA; ++t) {
          const __nv_bfloat162 s2 = __bfloat162bfloat162(sr[d][t]);
          const __nv_bfloat162 b2 = __bfloat162bfloat162(br[d][t]);
          const uint32_t* w = &wv[t].x;
          uint8_t* rowp = st + t * kTileA + r * 128;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int c = hf * 4 + j;  // 16-byte chunk of the 128-byte row
            *reinterpret_cast<uint4*>(rowp + ((c ^ (r & 7)) << 4)) = dequant8(w[j], s2, b2);
          }
        }
        // release the packed slot only once its words have been consumed: the refill is an
        // async-proxy (TMA) write, which the barrier does not order behind a load in flight
        mbar_arrive(&pk_empty[ps]);
        fence_proxy_async();
        mbar_arrive(&full_bar[slot]);
        if (i + kRing < nst) fetch_sb(i + kRing, d);
      }
    }

    // ---------------- epilogue, in chunks of 16 accumulator columns ----------------
    mbar_wait(&done_bar, 0, a.err);
    tc_fence_after();
    const int sub = warp & 3, chalf = warp >> 2;
    const int row = sub * 32 + lane;
    const uint32_t lane_base = tbase + ((uint32_t)(sub * 32) << 16);
    // columns [c, c + 16) of this warp's half: tile t's accumulators summed over the stage
    // interleave j = 0, 1, ... (those that received a stage), in that order
    auto load_chunk = [&](int c, float (&acc)[NA][16]) {
#pragma unroll
      for (int t = 0; t < NA; ++t) tc_ld16(lane_base + t * BN + chalf * HC + c, acc[t]);
      tc_wait_ld();
#pragma unroll
      for (int j = 1; j < NS; ++j) {
        if (j >= nst) break;
#pragma unroll
        for (int t = 0; t < NA; ++t) {
          float v[16];
          tc_ld16(lane_base + (j * NA + t) * BN + chalf * HC + c, v);
          tc_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) acc[t][e] += v[e];
        }
      }
    };
    const int n = n0 + row;
    auto store_chunk = [&](int c, const float (&acc)[NA][16]) {
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
        const int tok = m0 + chalf * HC + c + jj;
        if (tok >= a.M) break;
        const size_t o = (size_t)tok * a.N + n;
        if constexpr (SWIGLU) {
          const float gv = round_bf(acc[0][jj]), uv = round_bf(acc[1][jj]);
          a.y[o] = f2bf(gv / (1.0f + expf(-gv)) * uv);
        } else {
          const float v = acc[0][jj];
          if (a.y_f32) a.y_f32[o] = v;
          if (a.y) {
            uint16_t rv = f2bf(v);
            if (a.residual) rv = f2bf(bf2f(rv) + bf2f(a.residual[o]));
            a.y[o] = rv;
          }
        }
      }
    };
    const int tile = m_tile * gridDim.x + n_tile;
    if (a.splits == 1) {
      for (int c = 0; c < HC; c += 16) {
        if (m0 + chalf * HC + c >= a.M) break;  // no token of this chunk exists
        float acc[NA][16];
        load_chunk(c, acc);
        store_chunk(c, acc);
      }
      tc_fence_before();
    } else {
      float* mine = a.part + ((size_t)tile * a.splits + split) * NA * kTcRows * BN;
      for (int c = 0; c < HC; c += 16) {
        float acc[NA][16];
        load_chunk(c, acc);
#pragma unroll
        for (int t = 0; t < NA; ++t)
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) mine[(t * BN + chalf * HC + c + jj) * kTcRows + row] = acc[t][jj];
      }
      tc_fence_before();
      __threadfence();
      producers_sync();
      if (pid == 0) is_last = atomicAdd(a.counters + tile, 1) == a.splits - 1;
      producers_sync();
      if (is_last) {
        __threadfence();
        // sum every split in split order (the same bits whichever CTA finishes last)
        for (int c = 0; c < HC; c += 16) {
          float acc[NA][16];
#pragma unroll
          for (int t = 0; t < NA; ++t)
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) acc[t][jj] = 0.f;
          for (int sp = 0; sp < a.splits; ++sp) {
            const float* p = a.part + ((size_t)tile * a.splits + sp) * NA * kTcRows * BN;
#pragma unroll
            for (int t = 0; t < NA; ++t)
#pragma unroll
              for (int jj = 0; jj < 16; ++jj) acc[t][jj] += __ldcg(p + (t * BN + chalf * HC + c + jj) * kTcRows + row);
          }
          store_chunk(c, acc);
        }
        if (pid == 0) a.counters[tile] = 0;
      }
    }
  }
  __syncthreads();
  if (warp == mma_warp) {
    tc_fence_after();
    tc_dealloc(tbase, TCOLS);
  }
}

// ---- MMA issue-rate probe ------------------------------------------------------
// The matmul above issues 4 MMAs (M = 128, N = BN, K = 16) per 64-k weight stage into
// one accumulator.  This probe times that instruction stream alone: one CTA per SM with
// zero operands resident in shared memory (the same 128-byte-swizzled K-major tiles and
// descriptors), `warps` issuing warps (lane 0 of each), each issuing `iters` stages of 4
// MMAs of M x N x 16, a stage's MMAs (spread 0) or each single MMA (spread 1) dealt
// round-robin to that warp's `nacc` TMEM accumulators of N columns, and a tcgen05.commit
// every `commit_every` stages (0: only the final one).  cycles[cta] = clock64 from the
// first issue to the completion of every warp's last MMA.  Waits are bounded (the
// device flag higgs_tc_error reports).
constexpr int kProbeWarps = 4;
__global__ void __launch_bounds__(32 * kProbeWarps, 1)
    tc_rate_kernel(int m, int n, int nacc, int spread, int iters, int commit_every, int warps, long long* cycles,
                   int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t bars[2 * kProbeWarps];
  __shared__ uint32_t tmem_base;
  __shared__ long long t_first, t_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int words = (kTileA + n * 128) / 16;
  for (int i = threadIdx.x; i < words; i += blockDim.x) reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
  fence_proxy_async();  // the zeros, written by the generic proxy, are read by the MMAs
  const int commits = commit_every > 0 ? iters / commit_every : 0;
  if (threadIdx.x == 0) {
    for (int w = 0; w < kProbeWarps; ++w) {
      mbar_init(&bars[2 * w], commits > 0 ? commits : 1);  // one phase: every intermediate commit
      mbar_init(&bars[2 * w + 1], 1);
    }
    t_first = 0x7fffffffffffffffll;
    t_last = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    tc_alloc(&tmem_base, 512);
    tc_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_base;
  if (warp < warps && lane == 0) {
    const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) |
                           ((uint32_t)(m >> 4) << 24);
    const uint32_t sa = smem_u32(smem), sb = smem_u32(smem + kTileA);
    const uint32_t tw = tbase + warp * nacc * n;
    const long long t0 = clock64();
    for (int i = 0; i < iters; ++i) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int acc = spread ? (i * 4 + kk) % nacc : i % nacc;
        tc_mma(tw + acc * n, sw128_desc(sa + kk * 32), sw128_desc(sb + kk * 32), idesc, 1u);
      }
      if (commit_every > 0 && (i + 1) % commit_every == 0) tc_commit(&bars[2 * warp]);
    }
    tc_commit(&bars[2 * warp + 1]);
    bool ok = mbar_wait(&bars[2 * warp + 1], 0, err);
    if (commits > 0) ok = mbar_wait(&bars[2 * warp], 0, err) && ok;
    const long long t1 = clock64();
    atomicMin(reinterpret_cast<unsigned long long*>(&t_first), (unsigned long long)t0);
    atomicMax(reinterpret_cast<unsigned long long*>(&t_last), ok ? (unsigned long long)t1 : ~0ull);
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0)
    cycles[blockIdx.x] = t_last == (long long)~0ull ? -1 : t_last - t_first;
  if (warp == 0) {
    tc_fence_after();
    tc_dealloc(tbase, 512);
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

template <int BN, bool SWIGLU>
cudaError_t launch_bn(const CUtensorMap& map, const WMaps& wm, const TcArgs& a, dim3 grid, cudaStream_t st) {
  constexpr int NA = SWIGLU ? 2 : 1;
  constexpr int AS = tc_as(SWIGLU);
  constexpr size_t smem = (size_t)AS * NA * kTileA + (size_t)tc_xs(BN, SWIGLU) * BN * 128 +
                          (size_t)kPkStages * NA * kPkTile + 1024;
  static_assert(smem <= 227 * 1024, "shared memory budget");
  auto k = qgemm_tc_kernel<BN, SWIGLU>;
  static PerDeviceOnce attr;
  cudaError_t e = attr.run(
      [&] { return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); });
  if (e != cudaSuccess) return e;
  return launch_pdl(k, grid, dim3(tc_threads(BN, SWIGLU)), smem, st, map, wm, a);
}

int tc_sms() { return sm_count(); }

// K splits of a launch: the count that minimises waves x (k groups per split + a fixed
// cost per wave, in k-group units), at most g_tc_waves waves of one CTA per SM and at
// least 4 groups of 64 per split.  A wave the tiles fill only partly costs a whole wave.
// Measured at B=32 decode (Qwen3-8B): one wave for every shape 6.84 ms per step, two
// 7.16 ms, three 7.97 ms; this choice (wave cost 8) 6.70 ms.  Both knobs are higgs_set_option values ("gemm_tc_waves",
// "gemm_tc_wave_cost"); change them only between captures (workspace sizes follow).
int g_tc_waves = 2;
int g_tc_wave_cost = 8;

int tc_splits(int M, int K, int N) {
  const int BN = tc_bn(M, N);
  const long long tiles = (long long)(N / kTcRows) * ((M + BN - 1) / BN);
  const int G = K / 64;
  if (tiles == 0 || M < 1 || tiles > kTcMaxTiles) return 1;  // no tile, or beyond the counters
  const long long sms = tc_sms();
  int best = 1;
  long long best_cost = -1;
  for (int s = 1; s <= G / 4 && s <= 64; ++s) {
    const long long waves = (tiles * s + sms - 1) / sms;
    if (s > 1 && waves > g_tc_waves) break;
    const long long cost = waves * ((G + s - 1) / s + g_tc_wave_cost);
    if (best_cost < 0 || cost < best_cost) {
      best = s;
      best_cost = cost;
    }
  }
  return best;
}

}  // namespace

// the current device's timeout flag of the tensor-core kernels, allocated by higgs_init
int* tc_err_ptr() { return device_state(current_device()).tc_err; }

// K % 256 == 0, N (and every row segment) % 128 == 0, x 16-byte aligned, no fused norm.
bool qgemm_tc_supported(const QLinArgs& a) {
  if (a.M < 1 || a.K % 256 || a.N % kTcRows || ((uintptr_t)a.x & 15) || a.norm_w || a.moe_items) return false;
  if (a.nseg > 1)
    for (int i = 0; i < a.nseg; ++i)
      if (a.seg_end[i] % kTcRows) return false;
  return encode_fn() != nullptr;
}

// A fixed counter region (one int per tile, up to kTcMaxTiles, zero between
// calls), then the split-K partial tiles.  Split launches fill at most g_tc_waves
// waves of CTAs, so the partials never exceed that many CTAs' tiles whatever N and
// K are: the size depends on M (the tile width) and the options only, and one
// workspace sized for the largest M serves every shape back to back on a stream --
// the stream-K GEMV's counters sit in the same first bytes.
size_t qgemm_tc_workspace(int M, int K, int N, bool swiglu) {
  (void)K;
  (void)N;
  const int BN = M <= 32 ? 32 : (M <= 64 ? 64 : (M <= 128 ? 128 : 256));  // the widest tile M may use
  return kTcCounterBytes +
         (size_t)g_tc_waves * tc_sms() * (swiglu ? 2 : 1) * kTcRows * BN * sizeof(float);
}

cudaError_t launch_qgemm_tc(const QLinArgs& q, int epi, void* ws, size_t ws_bytes, cudaStream_t st) {
  if (!qgemm_tc_supported(q)) return cudaErrorInvalidValue;
  const bool swiglu = epi == EPI_SWIGLU;
  const int BN = tc_bn(q.M, q.N);
  CUtensorMap map;
  if (!x_tensor_map(q.x, q.M, q.K, BN, &map)) return cudaErrorInvalidValue;
  TcArgs a{};
  a.M = q.M;
  a.K = q.K;
  a.N = q.N;
  a.nseg = q.nseg > 1 ? q.nseg : 1;
  if (q.nseg > 1) {
    for (int i = 0; i < 3; ++i) {
      a.seg_end[i] = q.seg_end[i];
      a.w[i] = q.wseg[i];
      a.s[i] = q.sseg[i];
      a.b[i] = q.bseg[i];
    }
  } else {
    a.w[0] = q.w;
    a.s[0] = q.s;
    a.b[0] = q.b;
  }
  a.w2 = q.w2;
  a.s2 = q.s2;
  a.b2 = q.b2;
  a.y = q.y;
  a.y_f32 = q.y_f32;
  a.residual = q.residual;
  a.err = tc_err_ptr();
  WMaps wm;
  memset(&wm, 0, sizeof(wm));
  for (int i = 0; i < a.nseg; ++i) {
    const int rows = a.nseg > 1 ? a.seg_end[i] - (i ? a.seg_end[i - 1] : 0) : q.N;
    if (!w_tensor_map(a.w[i], rows, q.K, &wm.w[i])) return cudaErrorInvalidValue;
  }
  if (swiglu && !w_tensor_map(a.w2, q.N, q.K, &wm.up)) return cudaErrorInvalidValue;
  const int n_tiles = q.N / kTcRows, m_tiles = (q.M + BN - 1) / BN;
  const int G = q.K / 64;
  int splits = 1;
  const size_t need = qgemm_tc_workspace(q.M, q.K, q.N, swiglu);
  if (need && ws && ws_bytes >= need && ((uintptr_t)ws & 255) == 0) {
    splits = tc_splits(q.M, q.K, q.N);
    a.counters = static_cast<int*>(ws);
    a.part = reinterpret_cast<float*>(static_cast<char*>(ws) + kTcCounterBytes);
  }
  a.groups_per_split = (G + splits - 1) / splits;
  a.splits = (G + a.groups_per_split - 1) / a.groups_per_split;  // every split holds >= 1 group
  const dim3 grid(n_tiles, m_tiles, a.splits);
  if (swiglu) {
    if (BN == 32) return launch_bn<32, true>(map, wm, a, grid, st);
    if (BN == 64) return launch_bn<64, true>(map, wm, a, grid, st);
    if (BN == 128) return launch_bn<128, true>(map, wm, a, grid, st);
    return launch_bn<256, true>(map, wm, a, grid, st);
  }
  if (BN == 32) return launch_bn<32, false>(map, wm, a, grid, st);
  if (BN == 64) return launch_bn<64, false>(map, wm, a, grid, st);
  if (BN == 128) return launch_bn<128, false>(map, wm, a, grid, st);
  return launch_bn<256, false>(map, wm, a, grid, st);
}

void set_gemm_tc_waves(int w) { g_tc_waves = w < 1 ? 1 : (w > 8 ? 8 : w); }
void set_gemm_tc_wave_cost(int c) { g_tc_wave_cost = c < 0 ? 0 : (c > 1000 ? 1000 : c); }

// one-time host state (the driver's tensor-map encoder): call before any stream capture
void qgemm_tc_prepare() { encode_fn(); }

int qgemm_tc_error_and_clear() {
  int* p = tc_err_ptr();
  if (!p) return 0;
  int v = 0;
  cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost);
  if (v) cudaMemset(p, 0, sizeof(int));
  return v;
}

}  // namespace higgs

extern "C" int higgs_diag_tc_mma_rate(higgs_ctx* ctx, int m, int n, int nacc, int spread, int iters,
                                      int commit_every, int warps, int ctas, long long* cycles, void* stream) {
  HG_CHECK_ARG(ctx && cycles, "higgs_diag_tc_mma_rate: null argument");
  HG_CHECK_ARG(m == 64 || m == 128, "higgs_diag_tc_mma_rate: M must be 64 or 128");
  HG_CHECK_ARG(n >= 16 && n <= 256 && n % 16 == 0, "higgs_diag_tc_mma_rate: N must be 16..256, a multiple of 16");
  HG_CHECK_ARG(warps >= 1 && warps <= higgs::kProbeWarps, "higgs_diag_tc_mma_rate: warps 1..4");
  HG_CHECK_ARG(nacc >= 1 && warps * nacc * n <= 512,
               "higgs_diag_tc_mma_rate: warps x nacc accumulators of N columns exceed TMEM");
  HG_CHECK_ARG(iters >= 1 && iters <= (1 << 20) && commit_every >= 0 && (spread == 0 || spread == 1),
               "higgs_diag_tc_mma_rate: iters 1..2^20, commit_every >= 0, spread 0/1");
  HG_DEVICE(ctx);
  HG_CHECK_ARG(ctas >= 1 && ctas <= higgs::sm_count(), "higgs_diag_tc_mma_rate: ctas 1..SM count");
  // 160 KB of shared memory: at most one CTA per SM, so each holds all 512 TMEM columns
  const size_t smem = 160 * 1024;
  static higgs::PerDeviceOnce attr;
  HG_CUDA(attr.run([&] {
    return cudaFuncSetAttribute(higgs::tc_rate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  }));
  higgs::tc_rate_kernel<<<ctas, 32 * higgs::kProbeWarps, smem, (cudaStream_t)stream>>>(
      m, n, nacc, spread, iters, commit_every, warps, cycles, higgs::tc_err_ptr());
  HG_CUDA(cudaGetLastError());
  return HIGGS_OK;
}

extern "C" int higgs_tc_error(higgs_ctx* ctx, int* out) {
  HG_CHECK_ARG(ctx && out, "higgs_tc_error: null argument");
  HG_DEVICE(ctx);
  *out = higgs::qgemm_tc_error_and_clear();
  return HIGGS_OK;
}
