// prefill_attn.cu -- causal paged attention of prefill chunks on the tcgen05 tensor cores.
//
// Reference op replaced: fast::scaled_dot_product_attention with the causal mask
// (crates/higgs-models/src/utils.rs:45-60, masks 64-125) when a prompt chunk of many tokens
// attends to the cache (run_prefill, crates/higgs-engine/src/simple.rs:239-302 ->
// Attention::forward, crates/higgs-models/src/transformer.rs:246-294).  Behind
// higgs_paged_attention for launches of more than 64 query rows (G x Lq, G = Hq / Hkv).
//
// One CTA takes 128 query rows of one (sequence, kv head) -- TQ = 128 / G consecutive tokens
// x the G query heads that share the kv head, so every K / V tile serves all of them -- and
// walks the keys 0 .. its last token's position in blocks of 128 (8 pages):
//   * 4 loader warps: 16-byte cp.async copies of the block's pages of K and V (zero-filled past
//     the keys the tile can see) into 128-byte-swizzled shared tiles with the keys as rows,
//     which is K-major for S = Q K^T and MN-major for O += P V; a 3-stage ring (4 at D = 64);
//   * 2 MMA warps, one issuing lane each: S_j = Q K_j^T (M = 128 rows, N = 128 keys, K = D) into
//     one of two TMEM buffers, and O += P_j V_j (M = 128, N = D, K = 128 keys) with P read from
//     one of two TMEM buffers, so S_{j+1} is computed while the softmax of block j runs and the
//     softmax waits for P V only where it rescales O;
//   * 8 softmax warps, two threads per query row (TMEM lane), one per half of the block's keys,
//     exchanging the block maximum through shared memory: the causal mask, the running maximum
//     and sum in the exp2 domain, P as bf16 into TMEM, and the rescale of O in TMEM (each
//     thread half of the row's columns) when a row's maximum grew by more than 2^8; at the end
//     O / l as bf16.
// Tiles with the longest key ranges are scheduled first.  TMEM is allocated after
// griddepcontrol.wait.  Every mbarrier wait is bounded (about 2 s; the first timeout makes the
// CTA's other waits give up too, and sets the flag higgs_tc_error reports).
#include "common.cuh"
#include "kernels.cuh"
#include "tcgen05.cuh"

namespace higgs {

namespace {

constexpr int kPfRows = 128;     // query rows per CTA (UMMA M)
constexpr int kPfKeys = 128;     // keys per block (N of S, K of P V)
// NG softmax threads per query row: warps 0 .. 4 NG - 1, warp w takes rows (TMEM lanes)
// 32 (w % 4).. and key group w / 4 (kPfKeys / NG keys of each block, D / NG columns of O);
// then two MMA-issuing warps (S = Q K^T; O += P V), then the loader warps
constexpr int pf_softmax(int NG) { return 128 * NG; }
constexpr int pf_mma_warp(int NG) { return 4 * NG; }
constexpr int kPfLoaders = 128;
constexpr int pf_threads(int NG) { return pf_softmax(NG) + 64 + kPfLoaders; }  // + 2 MMA warps
constexpr int kPfTmemCols = 512;
constexpr int pf_stages(int D) { return D == 128 ? 3 : 4; }
constexpr uint32_t pf_q_bytes(int D) { return (uint32_t)kPfRows * D * 2; }
constexpr uint32_t pf_kv_bytes(int D) { return (uint32_t)kPfKeys * D * 2; }  // K or V of one block
constexpr size_t pf_smem(int D) { return 1024 + pf_q_bytes(D) + (size_t)pf_stages(D) * 2 * pf_kv_bytes(D); }
static_assert(pf_smem(128) <= 227 * 1024 && pf_smem(64) <= 227 * 1024, "shared memory budget");

bool g_prefill_tc = true;
int g_prefill_ng = 2;  // softmax threads per query row (2 or 4)

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

// the NG softmax warps of one row quarter (warps q, q + 4, ...)
__device__ __forceinline__ void pf_group_sync(int quarter, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(1 + quarter), "r"(nthreads) : "memory");
}

// x rounded up to a bf16 (toward +inf), as its bits: the threads of a row exchange block maxima
// this way, and all of them take the maximum of the same rounded values
__device__ __forceinline__ uint16_t bf16_up(float x) {
  uint32_t u = __float_as_uint(x);
  if ((u & 0xFFFFu) != 0 && (u >> 31) == 0) u += 0x10000u;  // positive and inexact: next bf16 up
  return (uint16_t)(u >> 16);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

template <int D, int NG>
__global__ void __launch_bounds__(pf_threads(NG), 1) prefill_attn_tc_kernel(PfArgs a) {
  constexpr int kPfSoftmax = pf_softmax(NG), kPfMmaWarp = pf_mma_warp(NG);
  constexpr int S = pf_stages(D);
  constexpr uint32_t kQ = pf_q_bytes(D), kKV = pf_kv_bytes(D);
  constexpr int DC = D / 8;  // 16-byte chunks per row
  // TMEM columns: S double buffer, P double buffer (bf16 pairs), O
  constexpr int COL_S = 0, COL_P = 2 * kPfKeys, COL_O = COL_P + kPfKeys;
  static_assert(COL_O + D <= kPfTmemCols, "TMEM columns");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* qs = smem;       // [D / 64 panels][128 rows][128 B], 128-byte swizzle
  uint8_t* kvs = smem + kQ;  // stage s: K at kvs + 2 s kKV, V after it; [D / 64][128 keys][128 B]
  __shared__ __align__(8) uint64_t q_full;
  __shared__ __align__(8) uint64_t kv_full[S];
  __shared__ __align__(8) uint64_t kv_empty[S];
  __shared__ __align__(8) uint64_t s_full[2];
  __shared__ __align__(8) uint64_t s_free[2];
  __shared__ __align__(8) uint64_t p_full[2];
  __shared__ __align__(8) uint64_t pv_done[2];
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = a.Hq / a.Hkv, TQ = kPfRows / G;
  const int tile = gridDim.x - 1 - blockIdx.x;  // the longest key ranges first
  const int hkv = blockIdx.y, b = blockIdx.z;
  const int t0 = tile * TQ;
  const int t_end = min(a.Lq, t0 + TQ);  // this CTA's tokens [t0, t_end)
  volatile int* abort = &abort_flag;

  if (threadIdx.x == 0) {
    mbar_init(&q_full, kPfLoaders);
    for (int s = 0; s < S; ++s) {
      mbar_init(&kv_full[s], kPfLoaders);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], kPfSoftmax);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&p_full[i], kPfSoftmax);
      mbar_init(&pv_done[i], 1);
    }
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  pdl_wait();  // q, the cache and the lengths come from earlier kernels
  const int pos0 = a.seq_lens[b] - a.Lq;  // position of query token 0
  const int kv_len = max(0, pos0 + t_end);  // keys seen by the CTA's last token
  const int nkb = (kv_len + kPfKeys - 1) / kPfKeys;
  if (warp == kPfMmaWarp) {
    tc_alloc(&tmem_base, kPfTmemCols);
    tc_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tb = tmem_base;
  pdl_launch();

  if (warp > kPfMmaWarp + 1) {
    // ---------------- loaders ----------------
    const int lt = threadIdx.x - (kPfSoftmax + 64);
    // Q row r = (token t0 + r / G, query head hkv G + r % G)
    for (int e = lt; e < kPfRows * DC; e += kPfLoaders) {
      const int r = e / DC, dc = e % DC;
      const int t = t0 + r / G;
      const bool ok = t < t_end;
      const uint16_t* src = a.q + (((size_t)b * a.Lq + (ok ? t : 0)) * a.Hq + hkv * G + r % G) * D + dc * 8;
      cp_async16_zfill(qs + (dc >> 3) * (kPfRows * 128) + r * 128 + (((dc & 7) ^ (r & 7)) << 4), src, ok);
    }
    cp_async_commit();
    cp_async_wait<0>();
    fence_proxy_async();  // generic-proxy writes -> the tensor core's (async proxy) reads
    mbar_arrive(&q_full);
    const int32_t* btr = a.bt + (size_t)b * a.max_blocks;
    // this thread's 16-byte column dc of keys k0, k0 + KSTEP, ... of every block
    constexpr int KSTEP = kPfLoaders / DC, KPT = kPfKeys / KSTEP;
    const int dc = lt % DC, k0 = lt / DC;
    const size_t col = (size_t)hkv * a.head_stride + dc * 8;
    const uint32_t so0 = (dc >> 3) * (kPfKeys * 128) + (((dc & 7) ^ (k0 & 7)) << 4);  // KSTEP % 8 == 0
    // block j is released once block j + 1 is in flight (wait for all but the newest copy
    // group): with S >= 3 stages the release never waits on a stage that needs it
    static_assert(S >= 3 && KSTEP % 8 == 0, "loader pipeline");
    for (int j = 0; j < nkb; ++j) {
      const int s = j % S;
      if (j >= S) pf_wait(&kv_empty[s], ((j / S) - 1) & 1, abort, a.err);
      uint8_t* ks = kvs + (size_t)s * 2 * kKV;
      uint8_t* vs = ks + kKV;
      int pg[KPT];
#pragma unroll
      for (int i = 0; i < KPT; ++i) {
        const int kg = j * kPfKeys + k0 + i * KSTEP;
        pg[i] = kg < kv_len ? btr[kg >> 4] : -1;
      }
#pragma unroll
      for (int i = 0; i < KPT; ++i) {
        const int kg = j * kPfKeys + k0 + i * KSTEP;
        const size_t off = pg[i] >= 0 ? (size_t)pg[i] * a.page_stride + col + (size_t)(kg & 15) * D : 0;
        const uint32_t so = so0 + (k0 + i * KSTEP) * 128;
        cp_async16_zfill(ks + so, a.kc + off, pg[i] >= 0);
        cp_async16_zfill(vs + so, a.vc + off, pg[i] >= 0);
      }
      cp_async_commit();
      if (j >= 1) {
        cp_async_wait<1>();
        fence_proxy_async();  // generic-proxy writes -> the tensor core's (async proxy) reads
        mbar_arrive(&kv_full[(j - 1) % S]);
      }
    }
    if (nkb > 0) {
      cp_async_wait<0>();
      fence_proxy_async();
      mbar_arrive(&kv_full[(nkb - 1) % S]);
    }
  } else if (warp == kPfMmaWarp) {
    // ---------------- S_j = Q K_j^T (one lane) ----------------
    // A thread issues one tcgen05.mma every ~140 cycles whatever its shape (measured on B200),
    // about twice the tensor pipe's time for M = 128 x N = 128 x K = 16: QK^T and PV each get
    // their own issuing warp.  They share no accumulator; P_j (softmax, after S_j completed)
    // orders S_j before P_j V_j, so the PV warp's commit also covers the K half of a stage.
    if (lane == 0) {
      constexpr uint32_t idS = tc_idesc_bf16(kPfRows, kPfKeys);
      const uint32_t sq = smem_u32(qs);
      pf_wait(&q_full, 0, abort, a.err);
      for (int j = 0; j < nkb; ++j) {
        const int s = j % S, sb = j & 1;
        pf_wait(&kv_full[s], (j / S) & 1, abort, a.err);
        if (j >= 2) pf_wait(&s_free[sb], ((j >> 1) - 1) & 1, abort, a.err);
        tc_fence_after();
        const uint32_t sk = smem_u32(kvs + (size_t)s * 2 * kKV);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          tc_mma(tb + COL_S + sb * kPfKeys, sw128_desc(sq + (kk >> 2) * (kPfRows * 128) + (kk & 3) * 32),
                 sw128_desc(sk + (kk >> 2) * (kPfKeys * 128) + (kk & 3) * 32), idS, kk > 0 ? 1u : 0u);
        tc_commit(&s_full[sb]);
      }
    }
    __syncwarp();
  } else if (warp == kPfMmaWarp + 1) {
    // ---------------- O += P_j V_j (one lane) ----------------
    if (lane == 0) {
      constexpr uint32_t idO = tc_idesc_bf16(kPfRows, D, true);
      for (int jp = 0; jp < nkb; ++jp) {
        const int s = jp % S;
        pf_wait(&p_full[jp & 1], (jp >> 1) & 1, abort, a.err);
        tc_fence_after();
        const uint32_t sv = smem_u32(kvs + (size_t)s * 2 * kKV + kKV);
#pragma unroll
        for (int kk = 0; kk < kPfKeys / 16; ++kk)  // 16 keys = two 8-row atoms = 2 KB
          tc_mma_ta(tb + COL_O, tb + COL_P + (jp & 1) * (kPfKeys / 2) + kk * 8,
                    sw128_mn_desc(sv + kk * 2048, kPfKeys * 128), idO, (jp > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&pv_done[jp & 1]);
        tc_commit(&kv_empty[s]);
      }
    }
    __syncwarp();
  } else {
    // ---------------- softmax: thread = (query row = TMEM lane, key group g) ----------------
    __shared__ uint16_t xch[NG][kPfRows];  // [group][row]: block maxima rounded up to bf16
    const int quarter = warp & 3, g = warp >> 2;
    const int r = quarter * 32 + lane;
    const int t = t0 + r / G;
    const bool valid = t < t_end;
    const int pos = valid ? pos0 + t : -1;  // keys 0 .. pos are visible
    const uint32_t lrow = tb + ((uint32_t)(quarter * 32) << 16);
    constexpr int HK = kPfKeys / NG;  // keys (S columns) per thread
    constexpr int HD = D / NG;        // O columns rescaled / stored per thread
    float m = -INFINITY, l = 0.f;  // l: this group's share of the row sum
    for (int j = 0; j < nkb; ++j) {
      const int sb = j & 1;
      pf_wait(&s_full[sb], (j >> 1) & 1, abort, a.err);
      tc_fence_after();
      float v[HK];
#pragma unroll
      for (int c = 0; c < HK / 16; ++c) tc_ld16(lrow + COL_S + sb * kPfKeys + g * HK + 16 * c, v + 16 * c);
      tc_wait_ld();
      tc_fence_before();
      mbar_arrive(&s_free[sb]);  // S buffer sb may take S_{j+2}
      const int lim = pos - j * kPfKeys - g * HK;  // key i of this group is visible iff i <= lim
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      if (lim >= HK - 1) {  // every key of this group visible: no mask
#pragma unroll
        for (int i = 0; i < HK; ++i) mx4[i & 3] = fmaxf(mx4[i & 3], v[i]);
      } else {
#pragma unroll
        for (int i = 0; i < HK; ++i) {
          v[i] = i <= lim ? v[i] : -INFINITY;
          mx4[i & 3] = fmaxf(mx4[i & 3], v[i]);
        }
      }
      // raw scores: the scale (> 0) is applied to the maximum and folded into the exponent's FMA;
      // the row's block maximum, rounded up to bf16 (an upper bound is all the reference needs)
      xch[g][r] = bf16_up(fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * a.scale_log2);
      pf_group_sync(quarter, 32 * NG);
      float mx = -INFINITY;
#pragma unroll
      for (int q = 0; q < NG; ++q) mx = fmaxf(mx, __uint_as_float((uint32_t)xch[q][r] << 16));
      pf_group_sync(quarter, 32 * NG);  // every read done before the next block's writes
      // all threads of a row take the same decision from the same (m, mx)
      const bool grow = mx > m + kPfSlack || (m == -INFINITY && mx != -INFINITY);
      const float alpha = grow ? ex2(m - mx) : 1.f;  // m = -inf: 0 (O and l are still zero)
      if (grow) m = mx;
      float sum4[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t pk[HK / 2];
      if (m == -INFINITY) {  // nothing visible yet in this row
#pragma unroll
        for (int i = 0; i < HK / 2; ++i) pk[i] = 0u;
      } else {
#pragma unroll
        for (int i = 0; i < HK / 2; ++i) {
          const float p0 = ex2(fmaf(v[2 * i], a.scale_log2, -m));
          const float p1 = ex2(fmaf(v[2 * i + 1], a.scale_log2, -m));
          sum4[i & 3] += p0 + p1;
          pk[i] = pack_bf16x2(p0, p1);
        }
      }
      l = l * alpha + ((sum4[0] + sum4[1]) + (sum4[2] + sum4[3]));
      if (j >= 2) {  // P buffer sb is free once P_{j-2} V_{j-2} is done
        pf_wait(&pv_done[sb], ((j >> 1) - 1) & 1, abort, a.err);
        tc_fence_after();
      }
      if (j >= 1 && __any_sync(0xffffffffu, alpha != 1.f)) {  // a row maximum grew: O *= alpha
        pf_wait(&pv_done[sb ^ 1], ((j - 1) >> 1) & 1, abort, a.err);  // after P_{j-1} V_{j-1}
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < HD / 16; ++c) {
          float o[16];
          tc_ld16(lrow + COL_O + g * HD + 16 * c, o);
          tc_wait_ld();
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) w[i] = __float_as_uint(o[i] * alpha);
          tc_st16(lrow + COL_O + g * HD + 16 * c, w);
        }
      }
#pragma unroll
      for (int c = 0; c < HK / 32; ++c)
        tc_st16(lrow + COL_P + sb * (kPfKeys / 2) + g * (HK / 2) + 16 * c, pk + 16 * c);
      tc_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[sb]);
    }
    // ---- O / l -> bf16 (this thread: columns [g D / NG, (g + 1) D / NG) of its row) ----
    if (nkb > 0) {
      pf_wait(&pv_done[(nkb - 1) & 1], ((nkb - 1) >> 1) & 1, abort, a.err);
      tc_fence_after();
    }
    // the row's sum over the groups, in group order, through the K / V ring (every copy into it
    // and every MMA reading it has completed by now)
    float* xl = reinterpret_cast<float*>(kvs);
    xl[g * kPfRows + r] = l;
    pf_group_sync(quarter, 32 * NG);
    float lt = 0.f;
#pragma unroll
    for (int q = 0; q < NG; ++q) lt += xl[q * kPfRows + r];
    const float inv = lt > 0.f ? 1.f / lt : 0.f;
    uint16_t* dst = a.out + (((size_t)b * a.Lq + (valid ? t : 0)) * a.Hq + hkv * G + r % G) * D + g * HD;
#pragma unroll
    for (int c = 0; c < HD / 16; ++c) {
      float o[16];
      if (nkb > 0) {
        tc_ld16(lrow + COL_O + g * HD + 16 * c, o);
        tc_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) o[i] = 0.f;
      }
      uint4 w0, w1;
      w0.x = pack_bf16x2(o[0] * inv, o[1] * inv), w0.y = pack_bf16x2(o[2] * inv, o[3] * inv);
      w0.z = pack_bf16x2(o[4] * inv, o[5] * inv), w0.w = pack_bf16x2(o[6] * inv, o[7] * inv);
      w1.x = pack_bf16x2(o[8] * inv, o[9] * inv), w1.y = pack_bf16x2(o[10] * inv, o[11] * inv);
      w1.z = pack_bf16x2(o[12] * inv, o[13] * inv), w1.w = pack_bf16x2(o[14] * inv, o[15] * inv);
      if (valid) {
        reinterpret_cast<uint4*>(dst + 16 * c)[0] = w0;
        reinterpret_cast<uint4*>(dst + 16 * c)[1] = w1;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kPfMmaWarp) {
    tc_fence_after();
    tc_dealloc(tb, kPfTmemCols);
  }
}

template <int D, int NG>
cudaError_t launch_pf(const PfArgs& a, cudaStream_t st) {
  auto k = prefill_attn_tc_kernel<D, NG>;
  static PerDeviceOnce attr;
  const cudaError_t e =
      attr.run([&] { return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pf_smem(D)); });
  if (e != cudaSuccess) return e;
  const int TQ = kPfRows / (a.Hq / a.Hkv);
  return launch_pdl(k, dim3((a.Lq + TQ - 1) / TQ, a.Hkv, a.B), dim3(pf_threads(NG)), pf_smem(D), st, a);
}

}  // namespace

void prefill_attn_tc_set(int on) { g_prefill_tc = on != 0; }
void prefill_attn_tc_set_groups(int ng) { g_prefill_ng = ng <= 2 ? 2 : 4; }

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
                                   int max_blocks, const int32_t* seq_lens, float scale, void* out, int* err,
                                   cudaStream_t st) {
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
  if (g_prefill_ng == 2) return D == 64 ? launch_pf<64, 2>(a, st) : launch_pf<128, 2>(a, st);
  return D == 64 ? launch_pf<64, 4>(a, st) : launch_pf<128, 4>(a, st);
}

}  // namespace higgs
