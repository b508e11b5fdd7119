// prefill_attn.cu -- causal paged attention of prefill chunks on the tcgen05 tensor cores.
//
// Reference op replaced: fast::scaled_dot_product_attention with the causal mask
// (crates/higgs-models/src/utils.rs:45-60, masks 64-125) when a prompt chunk of many tokens
// attends to the cache (run_prefill, crates/higgs-engine/src/simple.rs:239-302 ->
// Attention::forward, crates/higgs-models/src/transformer.rs:246-294).  Behind
// higgs_paged_attention for launches of more than 64 query rows (G x Lq, G = Hq / Hkv).
//
// A tile is 128 query rows of one (sequence, kv head) -- TQ = 128 / G consecutive tokens x the
// G query heads that share the kv head, so every K / V tile serves all of them -- walking the
// keys 0 .. its last token's position in blocks of 128 (8 pages).  The kernel is persistent:
// one CTA per SM takes the next tile left (a global counter, tiles ordered longest causal
// range first) whenever it starts one, and every ring runs on across its tiles, so the next
// tile's Q load and first S = Q K^T overlap the current tile's last blocks and its epilogue.
//   * 4 loader warps: 16-byte cp.async copies of Q and of each block's pages of K and V (zero-
//     filled past the keys the tile can see) into 128-byte-swizzled shared tiles with the keys
//     as rows, which is K-major for S = Q K^T and MN-major for O += P V; a 3-stage ring (4 at
//     D = 64);
//   * 2 MMA warps, one issuing lane each: S_J = Q K_J^T (M = 128 rows, N = 128 keys, K = D)
//     into one of two TMEM S buffers, and O += P_J V_J (M = 128, N = D, K = 128 keys) with P
//     read from one of two TMEM P buffers, so S_{J+1} is computed while the softmax of block J
//     runs and the softmax waits for P V only where it rescales O;
//   * 8 softmax warps, two threads per query row (TMEM lane), one per half of the block's keys,
//     exchanging the block maximum through shared memory when it may move the row's running
//     maximum (a barrier reduction tells): the causal mask, the running maximum and sum in the
//     exp2 domain, P as bf16 into TMEM, and the rescale of O in TMEM (each thread half of the
//     row's columns) when a row's maximum grew by more than 2^8; at the end of a tile O / l as
//     bf16.
// TMEM is allocated once, after
// griddepcontrol.wait.  Every mbarrier wait is bounded (about 2 s; the first timeout makes the
// CTA's other waits give up too, and sets the flag higgs_tc_error reports).
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"
#include "tcgen05.cuh"

namespace higgs {

namespace {

constexpr int kPfRows = 128;     // query rows per CTA (UMMA M)
constexpr int kPfKeys = 128;     // keys per block (N of S, K of P V)
// Two softmax threads per query row: warps 0-7, warp w takes rows (TMEM lanes) 32 (w % 4)..
// and key half w / 4 of each block (D / 2 columns of O at the end); warp 8 issues S = Q K^T,
// warp 9 O += P V; warps 10-13 load.  (Four threads per row measured no faster on B200.)
constexpr int kPfHalves = 2;
constexpr int kPfSoftmax = 128 * kPfHalves;
constexpr int kPfQkWarp = kPfSoftmax / 32, kPfPvWarp = kPfQkWarp + 1;
constexpr int kPfLoaders = 128;
constexpr int kPfThreads = kPfSoftmax + 64 + kPfLoaders;
constexpr int kPfTmemCols = 512;
constexpr int pf_stages(int D) { return D == 128 ? 3 : 4; }
constexpr uint32_t pf_q_bytes(int D) { return (uint32_t)kPfRows * D * 2; }
constexpr uint32_t pf_kv_bytes(int D) { return (uint32_t)kPfKeys * D * 2; }  // K or V of one block
constexpr size_t pf_smem(int D) { return 1024 + pf_q_bytes(D) + (size_t)pf_stages(D) * 2 * pf_kv_bytes(D); }
static_assert(pf_smem(128) <= 227 * 1024 && pf_smem(64) <= 227 * 1024, "shared memory budget");

bool g_prefill_tc = true;

struct PfArgs {
  const uint16_t* q;
  const uint16_t* kc;
  const uint16_t* vc;
  int64_t page_stride, head_stride;
  const int32_t* bt;
  int max_blocks;
  const int32_t* seq_lens;
  int B, Lq, Hq, Hkv;
  float scale_log2;
  uint16_t* out;
  int* err;
  int* counters;  // [0] next tile, [1] CTAs finished: zero before the launch, zero after it
};

// 16 bytes global -> shared, or 16 zero bytes when !ok (nothing is read then)
__device__ __forceinline__ void cp_async16_zfill(void* dst, const void* src, bool ok) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(ok ? 16 : 0)
               : "memory");
}

// Bounded wait for phase `parity`.  On timeout the CTA's abort flag and *err are set; once the
// abort flag is set every other wait of the CTA gives up at its next check.
__device__ __forceinline__ bool pf_wait(uint64_t* bar, unsigned parity, volatile int* abort, int* err) {
  const uint32_t a = smem_u32(bar);
  const long long t0 = clock64();
  for (unsigned it = 0;; ++it) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(a), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((it & 63) == 63) {
      if (*abort) return false;
      if (clock64() - t0 > (1ll << 32)) break;  // ~2 s at 2 GHz
    }
  }
  *abort = 1;
  atomicExch(err, 1);
  return false;
}

// 2^x (PTX ex2.approx, flush-to-zero: 2^x for x <= -126 is 0, which P rounds to anyway)
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// The running maximum m of a row moves only when a block's maximum exceeds it by more than
// kPfSlack (log2 units): P = 2^(s - m) then stays below 2^kPfSlack and O is rescaled in TMEM
// for only a few blocks.  O / l is the same softmax whatever m is.
constexpr float kPfSlack = 8.0f;

// the two softmax threads of a row quarter (warps q and q + 4)
__device__ __forceinline__ void pf_pair_sync(int quarter) {
  asm volatile("bar.sync %0, 64;" ::"r"(1 + quarter) : "memory");
}
// the same barrier, returning whether `pred` held for any of the 64 threads
__device__ __forceinline__ bool pf_pair_any(int quarter, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.or.pred q, %2, 64, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(1 + quarter)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// Tile i of a launch: query tile nqt - 1 - i / (B Hkv) (the longest causal ranges first) of
// (sequence, kv head) i % (B Hkv)
struct PfTile {
  int b, hkv, t0, t_end, pos0, kv_len, nkb;
};
__device__ __forceinline__ PfTile pf_tile(const PfArgs& a, int i, int nqt) {
  PfTile T;
  const int TQ = kPfRows / (a.Hq / a.Hkv), bh = a.B * a.Hkv;
  const int qt = nqt - 1 - i / bh;
  T.b = (i % bh) / a.Hkv;
  T.hkv = i % a.Hkv;
  T.t0 = qt * TQ;
  T.t_end = min(a.Lq, T.t0 + TQ);              // the tile's tokens [t0, t_end)
  T.pos0 = a.seq_lens[T.b] - a.Lq;             // position of query token 0
  T.kv_len = max(0, T.pos0 + T.t_end);         // keys seen by the tile's last token
  T.nkb = (T.kv_len + kPfKeys - 1) / kPfKeys;  // 128-key blocks
  return T;
}

constexpr int kPfTileRing = 4;  // tile indices handed from the scheduling thread to the roles

__device__ __forceinline__ void pf_loaders_sync() {
  asm volatile("bar.sync 5, %0;" ::"n"(kPfLoaders) : "memory");
}

template <int D>
__global__ void __launch_bounds__(kPfThreads, 1) prefill_attn_tc_kernel(PfArgs a) {
  constexpr int S = pf_stages(D);
  constexpr uint32_t kQ = pf_q_bytes(D), kKV = pf_kv_bytes(D);
  constexpr int DC = D / 8;  // 16-byte chunks per row
  // TMEM columns: S double buffer, P double buffer (bf16 pairs), O
  constexpr int COL_S = 0, COL_P = 2 * kPfKeys, COL_O = COL_P + kPfKeys;
  static_assert(COL_O + D <= kPfTmemCols, "TMEM columns");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* qs = smem;        // [D / 64 panels][128 rows][128 B], 128-byte swizzle
  uint8_t* kvs = smem + kQ;  // stage s: K at kvs + 2 s kKV, V after it; [D / 64][128 keys][128 B]
  // Every ring counts blocks J over the CTA's whole tile sequence, so the phases carry across
  // tiles: q_full / q_empty (the S MMAs of a tile are done with Q) and o_free (the softmax
  // threads have read a tile's O) have one phase per tile.
  __shared__ __align__(8) uint64_t q_full, q_empty, o_free;
  __shared__ __align__(8) uint64_t kv_full[S];
  __shared__ __align__(8) uint64_t kv_empty[S];
  __shared__ __align__(8) uint64_t s_full[2];
  __shared__ __align__(8) uint64_t s_free[2];
  __shared__ __align__(8) uint64_t p_full[2];
  __shared__ __align__(8) uint64_t pv_done[2];
  // [half][row]: block maxima, then the sums (a second pair barrier after each read keeps the
  // next write behind the partner's read)
  __shared__ float xch[kPfHalves][kPfRows];
  // tiles are taken dynamically, the longest causal ranges first: the first loader thread takes
  // the CTA's next tile index from a global counter (the first round's is blockIdx.x) and hands
  // it to the MMA lanes and the softmax threads through a small ring
  __shared__ int tile_ring[kPfTileRing];
  __shared__ __align__(8) uint64_t t_full[kPfTileRing];
  __shared__ __align__(8) uint64_t t_empty[kPfTileRing];
  __shared__ int loader_tile;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = a.Hq / a.Hkv, TQ = kPfRows / G;
  const int nqt = (a.Lq + TQ - 1) / TQ;
  const int ntiles = nqt * a.B * a.Hkv;
  volatile int* abort = &abort_flag;

  if (threadIdx.x == 0) {
    mbar_init(&q_full, kPfLoaders);
    mbar_init(&q_empty, 1);
    mbar_init(&o_free, kPfSoftmax);
    for (int s = 0; s < S; ++s) {
      mbar_init(&kv_full[s], kPfLoaders);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], kPfSoftmax);
      mbar_init(&p_full[i], kPfSoftmax);
      mbar_init(&pv_done[i], 1);
    }
    for (int i = 0; i < kPfTileRing; ++i) {
      mbar_init(&t_full[i], 1);
      mbar_init(&t_empty[i], kPfSoftmax + 2);
    }
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  // the tile of round k for the MMA lanes and the softmax threads (ntiles once none is left)
  auto next_tile = [&](int k) {
    pf_wait(&t_full[k % kPfTileRing], (k / kPfTileRing) & 1, abort, a.err);
    const int i = *abort ? ntiles : tile_ring[k % kPfTileRing];
    mbar_arrive(&t_empty[k % kPfTileRing]);
    return i;
  };

  pdl_wait();  // q, the cache and the lengths come from earlier kernels
  if (warp == kPfQkWarp) {
    tc_alloc(&tmem_base, kPfTmemCols);
    tc_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tb = tmem_base;
  pdl_launch();

  if (warp > kPfPvWarp) {
    // ---------------- loaders ----------------
    const int lt = threadIdx.x - (kPfSoftmax + 64);
    // this thread's 16-byte column dc of keys k0, k0 + KSTEP, ... of every block
    constexpr int KSTEP = kPfLoaders / DC, KPT = kPfKeys / KSTEP;
    const int dc = lt % DC, k0 = lt / DC;
    const uint32_t so0 = (dc >> 3) * (kPfKeys * 128) + (((dc & 7) ^ (k0 & 7)) << 4);  // KSTEP % 8 == 0
    // block J is released once block J + 1 is in flight (wait for all but the newest copy
    // group): with S >= 3 stages the release never waits on a stage that needs it
    static_assert(S >= 3 && KSTEP % 8 == 0, "loader pipeline");
    int J = 0;
    for (int k = 0;; ++k) {
      if (lt == 0) {
        int i = k == 0 ? blockIdx.x : gridDim.x + atomicAdd(a.counters, 1);
        if (i > ntiles || *abort) i = ntiles;
        if (k >= kPfTileRing) pf_wait(&t_empty[k % kPfTileRing], ((k / kPfTileRing) - 1) & 1, abort, a.err);
        tile_ring[k % kPfTileRing] = i;
        mbar_arrive(&t_full[k % kPfTileRing]);
        loader_tile = i;
      }
      pf_loaders_sync();
      const int i = loader_tile;
      pf_loaders_sync();  // every loader has read it before the next round's write
      if (i >= ntiles) break;
      const PfTile T = pf_tile(a, i, nqt);
      // Q row r = (token t0 + r / G, query head hkv G + r % G), once the previous tile's
      // S MMAs are done with the buffer
      if (k >= 1) pf_wait(&q_empty, (k - 1) & 1, abort, a.err);
      for (int e = lt; e < kPfRows * DC; e += kPfLoaders) {
        const int r = e / DC, c = e % DC;
        const int t = T.t0 + r / G;
        const bool ok = t < T.t_end;
        const uint16_t* src = a.q + (((size_t)T.b * a.Lq + (ok ? t : 0)) * a.Hq + T.hkv * G + r % G) * D + c * 8;
        cp_async16_zfill(qs + (c >> 3) * (kPfRows * 128) + r * 128 + (((c & 7) ^ (r & 7)) << 4), src, ok);
      }
      cp_async_commit();
      cp_async_wait<0>();
      fence_proxy_async();  // generic-proxy writes -> the tensor core's (async proxy) reads
      mbar_arrive(&q_full);
      const int32_t* btr = a.bt + (size_t)T.b * a.max_blocks;
      const size_t col = (size_t)T.hkv * a.head_stride + dc * 8;
      for (int j = 0; j < T.nkb; ++j, ++J) {
        const int s = J % S;
        if (J >= S) pf_wait(&kv_empty[s], ((J / S) - 1) & 1, abort, a.err);
        uint8_t* ks = kvs + (size_t)s * 2 * kKV;
        uint8_t* vs = ks + kKV;
        int pg[KPT];
#pragma unroll
        for (int q = 0; q < KPT; ++q) {
          const int kg = j * kPfKeys + k0 + q * KSTEP;
          pg[q] = kg < T.kv_len ? btr[kg >> 4] : -1;
        }
#pragma unroll
        for (int q = 0; q < KPT; ++q) {
          const int kg = j * kPfKeys + k0 + q * KSTEP;
          const size_t off = pg[q] >= 0 ? (size_t)pg[q] * a.page_stride + col + (size_t)(kg & 15) * D : 0;
          const uint32_t so = so0 + (k0 + q * KSTEP) * 128;
          cp_async16_zfill(ks + so, a.kc + off, pg[q] >= 0);
          cp_async16_zfill(vs + so, a.vc + off, pg[q] >= 0);
        }
        cp_async_commit();
        if (j >= 1) {
          cp_async_wait<1>();
          fence_proxy_async();
          mbar_arrive(&kv_full[(J - 1) % S]);
        }
      }
      if (T.nkb > 0) {
        cp_async_wait<0>();
        fence_proxy_async();
        mbar_arrive(&kv_full[(J - 1) % S]);
      }
    }
  } else if (warp == kPfQkWarp) {
    // ---------------- S_J = Q K_J^T (one lane) ----------------
    // A thread issues one tcgen05.mma every ~140 cycles whatever its shape (measured on B200),
    // about twice the tensor pipe's time for M = 128 x N = 128 x K = 16: QK^T and PV each get
    // their own issuing warp.  They share no accumulator; P_J (softmax, after S_J completed)
    // orders S_J before P_J V_J, so the PV warp's commit also covers the K half of a stage.
    if (lane == 0) {
      constexpr uint32_t idS = tc_idesc_bf16(kPfRows, kPfKeys);
      const uint32_t sq = smem_u32(qs);
      int J = 0;
      for (int k = 0;; ++k) {
        const int i = next_tile(k);
        if (i >= ntiles) break;
        const PfTile T = pf_tile(a, i, nqt);
        pf_wait(&q_full, k & 1, abort, a.err);
        for (int j = 0; j < T.nkb; ++j, ++J) {
          const int s = J % S, sb = J & 1;
          pf_wait(&kv_full[s], (J / S) & 1, abort, a.err);
          if (J >= 2) pf_wait(&s_free[sb], ((J >> 1) - 1) & 1, abort, a.err);
          tc_fence_after();
          const uint32_t sk = smem_u32(kvs + (size_t)s * 2 * kKV);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            tc_mma(tb + COL_S + sb * kPfKeys, sw128_desc(sq + (kk >> 2) * (kPfRows * 128) + (kk & 3) * 32),
                   sw128_desc(sk + (kk >> 2) * (kPfKeys * 128) + (kk & 3) * 32), idS, kk > 0 ? 1u : 0u);
          tc_commit(&s_full[sb]);
        }
        tc_commit(&q_empty);  // once this tile's S MMAs completed (at once if it had none)
      }
    }
    __syncwarp();
  } else if (warp == kPfPvWarp) {
    // ---------------- O += P_J V_J (one lane) ----------------
    if (lane == 0) {
      constexpr uint32_t idO = tc_idesc_bf16(kPfRows, D, true);
      int J = 0;
      for (int k = 0;; ++k) {
        const int i = next_tile(k);
        if (i >= ntiles) break;
        const PfTile T = pf_tile(a, i, nqt);
        for (int j = 0; j < T.nkb; ++j, ++J) {
          const int s = J % S;
          // a tile's first P V overwrites O: the softmax threads have read the previous tile's
          if (j == 0 && k >= 1) pf_wait(&o_free, (k - 1) & 1, abort, a.err);
          pf_wait(&p_full[J & 1], (J >> 1) & 1, abort, a.err);
          tc_fence_after();
          const uint32_t sv = smem_u32(kvs + (size_t)s * 2 * kKV + kKV);
#pragma unroll
          for (int kk = 0; kk < kPfKeys / 16; ++kk)  // 16 keys = two 8-row atoms = 2 KB
            tc_mma_ta(tb + COL_O, tb + COL_P + (J & 1) * (kPfKeys / 2) + kk * 8,
                      sw128_mn_desc(sv + kk * 2048, kPfKeys * 128), idO, (j > 0 || kk > 0) ? 1u : 0u);
          tc_commit(&pv_done[J & 1]);
          tc_commit(&kv_empty[s]);
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------- softmax: thread = (query row = TMEM lane, key half hf) ----------------
    const int quarter = warp & 3, hf = warp >> 2;
    const int r = quarter * 32 + lane;
    const uint32_t lrow = tb + ((uint32_t)(quarter * 32) << 16);
    constexpr int HK = kPfKeys / 2;  // keys (S columns) per thread
    constexpr int HD = D / 2;        // O columns rescaled / stored per thread
    int J = 0;
    for (int k = 0;; ++k) {
      const int i = next_tile(k);
      if (i >= ntiles) break;
      const PfTile T = pf_tile(a, i, nqt);
      const int t = T.t0 + r / G;
      const bool valid = t < T.t_end;
      const int pos = valid ? T.pos0 + t : -1;  // keys 0 .. pos are visible
      float m = -INFINITY, l = 0.f;             // l: this half's share of the row sum
      for (int j = 0; j < T.nkb; ++j, ++J) {
        const int sb = J & 1;
        pf_wait(&s_full[sb], (J >> 1) & 1, abort, a.err);
        tc_fence_after();
        float v[HK];
#pragma unroll
        for (int c = 0; c < HK / 16; ++c) tc_ld16(lrow + COL_S + sb * kPfKeys + hf * HK + 16 * c, v + 16 * c);
        tc_wait_ld();
        tc_fence_before();
        mbar_arrive(&s_free[sb]);  // S buffer sb may take S_{J+2}
        const int lim = pos - j * kPfKeys - hf * HK;  // key i of this half is visible iff i <= lim
        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        if (lim >= HK - 1) {  // every key of this half visible: no mask
#pragma unroll
          for (int q = 0; q < HK; ++q) mx4[q & 3] = fmaxf(mx4[q & 3], v[q]);
        } else {
#pragma unroll
          for (int q = 0; q < HK; ++q) {
            v[q] = q <= lim ? v[q] : -INFINITY;
            mx4[q & 3] = fmaxf(mx4[q & 3], v[q]);
          }
        }
        // raw scores: the scale (> 0) is applied to the maximum and folded into the exponent's FMA
        float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * a.scale_log2;
        // the row maximum moves only if one half's block maximum exceeds m + slack: one barrier
        // tells the 32 rows of the quarter whether any does; only then are the halves' maxima
        // exchanged (both threads of a row then take the same decision from the same (m, mx))
        bool grow = false;
        if (pf_pair_any(quarter, mx > m + kPfSlack || (m == -INFINITY && mx != -INFINITY))) {
          xch[hf][r] = mx;
          pf_pair_sync(quarter);
          mx = fmaxf(mx, xch[hf ^ 1][r]);  // the block maximum of the whole row
          pf_pair_sync(quarter);
          grow = mx > m + kPfSlack || (m == -INFINITY && mx != -INFINITY);
        }
        const float alpha = grow ? ex2(m - mx) : 1.f;  // m = -inf: 0 (O and l are still zero)
        if (grow) m = mx;
        float sum4[4] = {0.f, 0.f, 0.f, 0.f};
        uint32_t pk[HK / 2];
        if (m == -INFINITY) {  // nothing visible yet in this row
#pragma unroll
          for (int q = 0; q < HK / 2; ++q) pk[q] = 0u;
        } else {
#pragma unroll
          for (int q = 0; q < HK / 2; ++q) {
            const float p0 = ex2(fmaf(v[2 * q], a.scale_log2, -m));
            const float p1 = ex2(fmaf(v[2 * q + 1], a.scale_log2, -m));
            sum4[q & 3] += p0 + p1;
            pk[q] = pack_bf16x2(p0, p1);
          }
        }
        l = l * alpha + ((sum4[0] + sum4[1]) + (sum4[2] + sum4[3]));
        if (J >= 2) {  // P buffer sb is free once P_{J-2} V_{J-2} is done
          pf_wait(&pv_done[sb], ((J >> 1) - 1) & 1, abort, a.err);
          tc_fence_after();
        }
        if (j >= 1 && __any_sync(0xffffffffu, alpha != 1.f)) {  // a row maximum grew: O *= alpha
          pf_wait(&pv_done[sb ^ 1], ((J - 1) >> 1) & 1, abort, a.err);  // after P_{J-1} V_{J-1}
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < HD / 16; ++c) {
            float o[16];
            tc_ld16(lrow + COL_O + hf * HD + 16 * c, o);
            tc_wait_ld();
            uint32_t w[16];
#pragma unroll
            for (int q = 0; q < 16; ++q) w[q] = __float_as_uint(o[q] * alpha);
            tc_st16(lrow + COL_O + hf * HD + 16 * c, w);
          }
        }
#pragma unroll
        for (int c = 0; c < HK / 32; ++c)
          tc_st16(lrow + COL_P + sb * (kPfKeys / 2) + hf * (HK / 2) + 16 * c, pk + 16 * c);
        tc_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full[sb]);
      }
      // ---- O / l -> bf16 (this thread: columns [hf D / 2, (hf + 1) D / 2) of its row) ----
      if (T.nkb > 0) {
        pf_wait(&pv_done[(J - 1) & 1], ((J - 1) >> 1) & 1, abort, a.err);
        tc_fence_after();
      }
      xch[hf][r] = l;
      pf_pair_sync(quarter);
      const float lt = hf == 0 ? l + xch[1][r] : xch[0][r] + l;  // l0 + l1 in both
      pf_pair_sync(quarter);
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      float o[HD];
      if (T.nkb > 0) {
#pragma unroll
        for (int c = 0; c < HD / 16; ++c) tc_ld16(lrow + COL_O + hf * HD + 16 * c, o + 16 * c);
        tc_wait_ld();
      } else {
#pragma unroll
        for (int q = 0; q < HD; ++q) o[q] = 0.f;
      }
      tc_fence_before();
      mbar_arrive(&o_free);  // the next tile's first P V may overwrite O
      if (valid) {
        uint4* dst = reinterpret_cast<uint4*>(
            a.out + (((size_t)T.b * a.Lq + t) * a.Hq + T.hkv * G + r % G) * D + hf * HD);
#pragma unroll
        for (int c = 0; c < HD / 8; ++c)
          dst[c] = make_uint4(pack_bf16x2(o[8 * c] * inv, o[8 * c + 1] * inv),
                              pack_bf16x2(o[8 * c + 2] * inv, o[8 * c + 3] * inv),
                              pack_bf16x2(o[8 * c + 4] * inv, o[8 * c + 5] * inv),
                              pack_bf16x2(o[8 * c + 6] * inv, o[8 * c + 7] * inv));
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kPfQkWarp) {
    tc_fence_after();
    tc_dealloc(tb, kPfTmemCols);
  }
  if (threadIdx.x == 0) {  // the last CTA to finish leaves the tile counters at zero
    __threadfence();
    if (atomicAdd(a.counters + 1, 1) == (int)gridDim.x - 1) {
      a.counters[0] = 0;
      a.counters[1] = 0;
      __threadfence();
    }
  }
}

template <int D>
cudaError_t launch_pf(const PfArgs& a, cudaStream_t st) {
  auto k = prefill_attn_tc_kernel<D>;
  static PerDeviceOnce attr;
  const cudaError_t e =
      attr.run([&] { return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pf_smem(D)); });
  if (e != cudaSuccess) return e;
  // persistent: one CTA per SM (shared memory and TMEM allow one), each taking the next tile
  // left (the longest causal ranges first)
  const int TQ = kPfRows / (a.Hq / a.Hkv);
  const long long ntiles = (long long)((a.Lq + TQ - 1) / TQ) * a.B * a.Hkv;
  const int grid = (int)std::min<long long>(ntiles, sm_count());
  return launch_pdl(k, dim3(grid), dim3(kPfThreads), pf_smem(D), st, a);
}

}  // namespace

void prefill_attn_tc_set(int on) { g_prefill_tc = on != 0; }

// Launches of more than 64 query rows (the decode kernel would take three or more launches of
// 32 rows, each over every page), G dividing 128, 16-byte aligned rows and pages.
bool prefill_attn_tc_fits(int Lq, int Hq, int Hkv, int D, const void* q, const void* kc, const void* vc,
                          const void* out, int64_t page_stride, int64_t head_stride) {
  if (!g_prefill_tc || Hkv <= 0 || Hq % Hkv) return false;
  const int G = Hq / Hkv;
  const uintptr_t al = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(kc) |
                       reinterpret_cast<uintptr_t>(vc) | reinterpret_cast<uintptr_t>(out);
  return (D == 64 || D == 128) && kPfRows % G == 0 && (long long)G * Lq > 64 && (al & 15) == 0 &&
         page_stride % 8 == 0 && head_stride % 8 == 0;
}

cudaError_t launch_prefill_attn_tc(const void* q, int B, int Lq, int Hq, int Hkv, int D, const void* kc,
                                   const void* vc, int64_t page_stride, int64_t head_stride, const int32_t* bt,
                                   int max_blocks, const int32_t* seq_lens, float scale, void* out, int* counters,
                                   int* err, cudaStream_t st) {
  PfArgs a;
  a.q = (const uint16_t*)q;
  a.kc = (const uint16_t*)kc;
  a.vc = (const uint16_t*)vc;
  a.page_stride = page_stride;
  a.head_stride = head_stride;
  a.bt = bt;
  a.max_blocks = max_blocks;
  a.seq_lens = seq_lens;
  a.B = B;
  a.Lq = Lq;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.out = (uint16_t*)out;
  a.err = err;
  a.counters = counters;
  return D == 64 ? launch_pf<64>(a, st) : launch_pf<128>(a, st);
}

}  // namespace higgs
