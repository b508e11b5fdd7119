// attention.cu -- paged decode attention (GQA, causal for Lq > 1) over bf16
// pages and over TurboQuant 4-bit pages.
//
// Reference op replaced: fast::scaled_dot_product_attention (utils.rs:45-60)
// with the decode masks of utils.rs:64-125; the contiguous per-sequence cache
// of cache.rs:130-312 is the special case of a block table whose pages are
// consecutive (page_stride / head_stride describe either layout).
//
// Design:
//  * grid (splits, Hkv, B), 4 warps per CTA.  The query rows of one kv head
//    (G = Hq/Hkv heads x Lq query tokens) form a 16- or 32-row MMA tile, so
//    K and V bytes are read once for all heads of the group;
//  * each warp streams its own pages (16 tokens) into shared memory with
//    cp.async (double-buffered, XOR-swizzled rows), computes S = Q K^T and
//    O += P V with mma.sync m16n8k16 and an online softmax in base 2;
//  * the 4 warps merge in shared memory; with several splits each CTA writes
//    a normalised partial (O, log-sum-exp) to the workspace and the last CTA of
//    a (sequence, kv head) to arrive -- counted with an atomic -- merges them,
//    so no second kernel is launched;
//  * TurboQuant pages: K codes feed the MMA directly as bf16 (128 + c) against
//    the rotated query (the constant offset is removed per row), V codes are
//    expanded to exact bf16 (c - 8) in shared memory with the per-token scale
//    folded into P, and the merged output is rotated back with the inverse
//    Hadamard transform.
#include <cooperative_groups.h>

#include <mutex>

#include "common.cuh"
#include "kernels.cuh"
#include "timeline.cuh"

namespace higgs {

constexpr int kAttnThreads = 128;
constexpr int kCounterBytes = 4096;
constexpr int kTargetCtas = 2 * 148;
constexpr int kTargetCtasTq4 = 3 * 148;  // the swapped-role TurboQuant kernel: three per SM
constexpr int kTq4Stages = 6;  // per-warp page ring of the TurboQuant kernel (a pair + 4 in flight)

struct AttnArgs {
  const uint16_t* q;
  int B, Lq, Hq, Hkv;
  int tq0, lq_chunk;  // query tokens [tq0, tq0 + lq_chunk) of Lq handled by this launch
  const uint16_t* kc;
  const uint16_t* vc;
  const uint8_t* kcode;
  const __half* kscale;
  const uint8_t* vcode;
  const __half* vscale;
  const int8_t* signs;
  int64_t page_stride, head_stride;
  const int32_t* bt;
  int max_blocks;
  const int32_t* seq_lens;
  float scale_log2;
  uint16_t* out;
  int splits, pages_per_split;
  float* ws_o;
  float* ws_lse;
  int* counters;
  // fused front half (higgs_fused_attention): q/k/v come from the q|k|v
  // projection output and the new K/V are appended by the kernel itself
  const uint16_t* qkv;
  const uint16_t* qn;
  const uint16_t* kn;
  float eps;
  const int32_t* pos;
  const float* inv_freq;
  const int64_t* slots;
  uint16_t* kc_w;
  uint16_t* vc_w;
  // weights of a later launch to pull into L2 (the decode step's next GEMVs): this
  // kernel is latency-bound at small batches and leaves HBM idle
  L2Prefetch pf;
};

__device__ __forceinline__ int swz(int row, int chunk) { return chunk ^ (row & 7); }

// Loads one page (16 rows x D bf16) into a swizzled smem tile; rows >= valid
// are zero-filled so masked garbage can never become NaN in P*V.
template <int D>
__device__ __forceinline__ void load_page_bf16(uint16_t* dst, const uint16_t* src, int valid,
                                               int lane) {
  constexpr int CH = D / 8;
#pragma unroll
  for (int i = 0; i < (16 * CH) / 32; ++i) {
    const int qd = lane + 32 * i;
    const int r = qd / CH, c = qd % CH;
    const uint32_t sdst = smem_u32(dst + r * D + swz(r, c) * 8);
    const void* gsrc = src + r * D + c * 8;
    const int bytes = r < valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sdst), "l"(gsrc),
                 "r"(bytes));
  }
}

template <int NT>
__device__ __forceinline__ void row_stats_update(float (&m)[2], float (&l)[2], float (&s)[NT][4],
                                                 float (&alpha)[2]) {
#pragma unroll
  for (int hlf = 0; hlf < 2; ++hlf) {
    float mx = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) mx = fmaxf(mx, fmaxf(s[nt][2 * hlf], s[nt][2 * hlf + 1]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mn = fmaxf(m[hlf], mx);
    alpha[hlf] = (mn == -INFINITY) ? 1.0f : exp2f(m[hlf] - mn);
    m[hlf] = mn;
    float rs = 0.0f;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float& v = s[nt][2 * hlf + e];
        v = (mn == -INFINITY) ? 0.0f : exp2f(v - mn);
        rs += v;
      }
    l[hlf] = l[hlf] * alpha[hlf] + rs;
  }
}

// Common tail: CTA-level merge of the 4 warps, then either the final store or a
// split partial plus the last-CTA merge.  o_sm rows are in "physical" d order;
// `finish` converts a merged f32 row to the bf16 output (TurboQuant rotates
// back there).
template <int D, int MT, typename Finish, bool CL = false>
__device__ __forceinline__ void attn_epilogue(const AttnArgs& a, float (&m)[MT][2],
                                              float (&l)[MT][2], float (&o)[MT][D / 8][4],
                                              float* smem_f, int b, int h, int split, int R,
                                              Finish finish) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  constexpr int RP = 16 * MT;
  float* sm_m = smem_f;                    // [4][RP]
  float* sm_l = sm_m + 4 * RP;             // [4][RP]
  float* sm_lse = sm_l + 4 * RP;           // [RP]
  float* sm_o = sm_lse + RP;               // [4][RP][D]
  __syncthreads();  // page buffers are dead from here on
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int hlf = 0; hlf < 2; ++hlf) {
      float lv = l[mt][hlf];
      lv += __shfl_xor_sync(0xffffffffu, lv, 1);
      lv += __shfl_xor_sync(0xffffffffu, lv, 2);
      const int row = mt * 16 + g + 8 * hlf;
      if (row >= R) continue;  // padding rows of the MMA tile are never read
      if (t == 0) {
        sm_m[warp * RP + row] = m[mt][hlf];
        sm_l[warp * RP + row] = lv;
      }
#pragma unroll
      for (int dt = 0; dt < D / 8; ++dt)
#pragma unroll
        for (int e = 0; e < 2; ++e)
          sm_o[(warp * RP + row) * D + dt * 8 + 2 * t + e] = o[mt][dt][2 * hlf + e];
    }
  __syncthreads();
  // merge the 4 warps into warp 0's slot, normalised; each (row, d) is read and
  // written by one thread only
  for (int i = threadIdx.x; i < R * D; i += kAttnThreads) {
    const int row = i / D, d = i % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, sm_m[w * RP + row]);
    float L = 0.0f, O = 0.0f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float mw = sm_m[w * RP + row];
      const float sc = (mw == -INFINITY) ? 0.0f : exp2f(mw - M);
      L += sc * sm_l[w * RP + row];
      O += sc * sm_o[(w * RP + row) * D + d];
    }
    sm_o[row * D + d] = L > 0.0f ? O / L : 0.0f;
    if (d == 0) sm_lse[row] = L > 0.0f ? M + log2f(L) : -INFINITY;
  }
  __syncthreads();
  const int bh = b * a.Hkv + h;
  if (a.splits == 1) {
    finish(sm_o, R, b, h);
    HG_TL_END(3001);
    return;
  }
  if constexpr (CL) {
    // The splits of this (sequence, kv head) are one thread-block cluster: every CTA merges
    // a slice of d for every row, reading the splits' normalised partials and log-sum-exps
    // straight from their shared memory (no workspace round trip, no arrival counter).  The
    // fold is the one below -- running maximum, weights exp2(lse - M), splits in order.
    namespace cg = cooperative_groups;
    cg::cluster_group cl = cg::this_cluster();
    cl.sync();
    const int S = (int)cl.num_blocks(), rk = (int)cl.block_rank();
    const int dper = (D + S - 1) / S, d0 = rk * dper, d1 = min(D, d0 + dper), nd = max(0, d1 - d0);
    const int G = a.Hq / a.Hkv;
    for (int i = threadIdx.x; i < R * nd; i += kAttnThreads) {
      const int row = i / nd, d = d0 + i % nd;
      float M = -INFINITY;
      for (int s = 0; s < S; ++s) M = fmaxf(M, cl.map_shared_rank(sm_lse, s)[row]);
      float W = 0.0f, acc = 0.0f;
      if (M != -INFINITY) {
        for (int s = 0; s < S; ++s) {
          const float ls = cl.map_shared_rank(sm_lse, s)[row];
          const float w = (ls == -INFINITY) ? 0.0f : exp2f(ls - M);
          W += w;
          acc = fmaf(w, cl.map_shared_rank(sm_o, s)[row * D + d], acc);
        }
      }
      const int tq = a.tq0 + row / G, hq = h * G + row % G;
      a.out[(((size_t)b * a.Lq + tq) * a.Hq + hq) * D + d] = f2bf(W > 0.0f ? acc * (1.0f / W) : 0.0f);
    }
    cl.sync();  // the partials stay in shared memory until every CTA has read them
    HG_TL_END(3004);
    return;
  }
  // write the split partial (valid rows only)
  float* po = a.ws_o + ((size_t)bh * a.splits + split) * RP * D;
  float* pl = a.ws_lse + ((size_t)bh * a.splits + split) * RP;
  for (int i = threadIdx.x; i < R * D; i += kAttnThreads) po[i] = sm_o[i];
  for (int i = threadIdx.x; i < R; i += kAttnThreads) pl[i] = sm_lse[i];
  __threadfence();
  __syncthreads();
  __shared__ int is_last;
  if (threadIdx.x == 0) is_last = (atomicAdd(a.counters + bh, 1) == a.splits - 1);
  __syncthreads();
  HG_TL_MARK(6);
  if (!is_last) {
    HG_TL_END(3002);
    return;
  }
  __threadfence();
  const float* base_o = a.ws_o + (size_t)bh * a.splits * RP * D;
  const float* base_l = a.ws_lse + (size_t)bh * a.splits * RP;
  // every thread owns 4 consecutive d of one row; the lse and the float4 partials of up
  // to 16 splits are loaded together and folded with a running maximum, so the merge
  // costs one L2 round trip per 16 splits (measured on B200: 24 at a time, one round trip
  // for B=1's 17 splits at ctx 2048, lengthened the decode step, 2.14 -> 2.20 ms)
  constexpr int CH = 16;
  for (int i4 = threadIdx.x; i4 < R * D / 4; i4 += kAttnThreads) {
    const int row = (i4 * 4) / D;
    float M = -INFINITY, W = 0.0f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = 0; s0 < a.splits; s0 += CH) {
      float ls[CH];
      float4 v[CH];
#pragma unroll
      for (int u = 0; u < CH; ++u) {
        const bool in = s0 + u < a.splits;
        ls[u] = in ? __ldcg(base_l + (size_t)(s0 + u) * RP + row) : -INFINITY;
        v[u] = in ? __ldcg(reinterpret_cast<const float4*>(base_o + (size_t)(s0 + u) * RP * D) + i4)
                  : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      float Mc = M;
#pragma unroll
      for (int u = 0; u < CH; ++u) Mc = fmaxf(Mc, ls[u]);
      if (Mc == -INFINITY) continue;  // no key of this row in these splits
      const float r = (M == -INFINITY) ? 0.0f : exp2f(M - Mc);
      W *= r;
      acc.x *= r;
      acc.y *= r;
      acc.z *= r;
      acc.w *= r;
#pragma unroll
      for (int u = 0; u < CH; ++u) {
        const float w = (ls[u] == -INFINITY) ? 0.0f : exp2f(ls[u] - Mc);
        W += w;
        acc.x = fmaf(w, v[u].x, acc.x);
        acc.y = fmaf(w, v[u].y, acc.y);
        acc.z = fmaf(w, v[u].z, acc.z);
        acc.w = fmaf(w, v[u].w, acc.w);
      }
      M = Mc;
    }
    const float inv = W > 0.0f ? 1.0f / W : 0.0f;
    sm_o[i4 * 4 + 0] = acc.x * inv;
    sm_o[i4 * 4 + 1] = acc.y * inv;
    sm_o[i4 * 4 + 2] = acc.z * inv;
    sm_o[i4 * 4 + 3] = acc.w * inv;
  }
  __syncthreads();
  if (threadIdx.x == 0) a.counters[bh] = 0;
  finish(sm_o, R, b, h);
  HG_TL_END(3003);
}

template <int D>
struct FinishBf16 {
  const AttnArgs* a;
  __device__ void operator()(const float* sm_o, int R, int b, int h) const {
    const int G = a->Hq / a->Hkv;
    for (int i = threadIdx.x; i < R * (D / 2); i += kAttnThreads) {
      const int row = i / (D / 2), d = 2 * (i % (D / 2));
      const int tq = a->tq0 + row / G, hq = h * G + row % G;
      uint16_t* op = a->out + (((size_t)b * a->Lq + tq) * a->Hq + hq) * D + d;
      *reinterpret_cast<uint32_t*>(op) = pack_bf2(sm_o[row * D + d], sm_o[row * D + d + 1]);
    }
  }
};

// ---------------------------------------------------------------------------
// bf16 pages
// ---------------------------------------------------------------------------
template <int D, int MT>
__global__ void __launch_bounds__(kAttnThreads) paged_attn_bf16_kernel(AttnArgs a) {
  constexpr int RP = 16 * MT;
  constexpr int PAGE_ELEMS = 16 * D;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint16_t* Qs = reinterpret_cast<uint16_t*>(smem_raw);              // [RP][D]
  uint16_t* KV = Qs + RP * D;                                         // [4 warps][2 stages][K|V]
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int G = a.Hq / a.Hkv;
  const int R = G * a.lq_chunk;

  pdl_wait();
  const int L = a.seq_lens[b];
  const int n_pages = min((L + 15) / 16, a.max_blocks);
  const int pg0 = split * a.pages_per_split;
  const int pg1 = min(n_pages, pg0 + a.pages_per_split);

  // Q tile (rows >= R zero)
  for (int i = threadIdx.x; i < RP * (D / 8); i += kAttnThreads) {
    const int row = i / (D / 8), c = i % (D / 8);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (row < R) {
      const int tq = a.tq0 + row / G, hq = h * G + row % G;
      v = *reinterpret_cast<const uint4*>(a.q + (((size_t)b * a.Lq + tq) * a.Hq + hq) * D + c * 8);
    }
    *reinterpret_cast<uint4*>(Qs + row * D + swz(row, c) * 8) = v;
  }
  __syncthreads();

  float m[MT][2], l[MT][2], o[MT][D / 8][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    m[mt][0] = m[mt][1] = -INFINITY;
    l[mt][0] = l[mt][1] = 0.0f;
#pragma unroll
    for (int dt = 0; dt < D / 8; ++dt)
#pragma unroll
      for (int c = 0; c < 4; ++c) o[mt][dt][c] = 0.0f;
  }

  uint16_t* my = KV + warp * 2 * 2 * PAGE_ELEMS;
  auto kbuf = [&](int st) { return my + st * 2 * PAGE_ELEMS; };
  auto vbuf = [&](int st) { return my + st * 2 * PAGE_ELEMS + PAGE_ELEMS; };
  auto issue = [&](int pg, int st) {
    const int pid = a.bt[(size_t)b * a.max_blocks + pg];
    const size_t off = (size_t)pid * a.page_stride + (size_t)h * a.head_stride;
    const int valid = min(16, L - pg * 16);
    load_page_bf16<D>(kbuf(st), a.kc + off, valid, lane);
    load_page_bf16<D>(vbuf(st), a.vc + off, valid, lane);
  };

  int stage = 0;
  int pg = pg0 + warp;
  if (pg < pg1) issue(pg, 0);
  cp_async_commit();
  for (; pg < pg1; pg += 4) {
    if (pg + 4 < pg1) issue(pg + 4, stage ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncwarp();
    const uint16_t* Ks = kbuf(stage);
    const uint16_t* Vs = vbuf(stage);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int kt = 0; kt < D / 16; ++kt) {
        uint32_t qa[4], kb[4];
        {
          const int mi = lane >> 3;
          const int row = mt * 16 + (mi & 1) * 8 + (lane & 7);
          ldmatrix_x4(qa, Qs + row * D + swz(row, 2 * kt + (mi >> 1)) * 8);
          const int tok = (mi >> 1) * 8 + (lane & 7);
          ldmatrix_x4(kb, Ks + tok * D + swz(tok, 2 * kt + (mi & 1)) * 8);
        }
        mma_bf16_16816(s[0], qa[0], qa[1], qa[2], qa[3], kb[0], kb[1]);
        mma_bf16_16816(s[1], qa[0], qa[1], qa[2], qa[3], kb[2], kb[3]);
      }
      // scale + causal mask
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int j = pg * 16 + nt * 8 + 2 * t + (c & 1);
          const int row = mt * 16 + g + 8 * (c >> 1);
          const int qpos = L - a.Lq + a.tq0 + row / G;
          const bool ok = row < R && j <= qpos;
          s[nt][c] = ok ? s[nt][c] * a.scale_log2 : -INFINITY;
        }
      float alpha[2];
      row_stats_update(m[mt], l[mt], s, alpha);
#pragma unroll
      for (int dt = 0; dt < D / 8; ++dt) {
        o[mt][dt][0] *= alpha[0];
        o[mt][dt][1] *= alpha[0];
        o[mt][dt][2] *= alpha[1];
        o[mt][dt][3] *= alpha[1];
      }
      // P as hi + lo bf16 pairs: the two MMAs carry ~16 mantissa bits of P
      uint32_t ph[4], pl[4];
      split_bf2(s[0][0], s[0][1], ph[0], pl[0]);
      split_bf2(s[0][2], s[0][3], ph[1], pl[1]);
      split_bf2(s[1][0], s[1][1], ph[2], pl[2]);
      split_bf2(s[1][2], s[1][3], ph[3], pl[3]);
#pragma unroll
      for (int d2 = 0; d2 < D / 16; ++d2) {
        uint32_t vb[4];
        const int mi = lane >> 3;
        const int tok = (mi & 1) * 8 + (lane & 7);
        ldmatrix_x4_trans(vb, Vs + tok * D + swz(tok, 2 * d2 + (mi >> 1)) * 8);
        mma_bf16_16816(o[mt][2 * d2], ph[0], ph[1], ph[2], ph[3], vb[0], vb[1]);
        mma_bf16_16816(o[mt][2 * d2 + 1], ph[0], ph[1], ph[2], ph[3], vb[2], vb[3]);
        mma_bf16_16816(o[mt][2 * d2], pl[0], pl[1], pl[2], pl[3], vb[0], vb[1]);
        mma_bf16_16816(o[mt][2 * d2 + 1], pl[0], pl[1], pl[2], pl[3], vb[2], vb[3]);
      }
    }
    __syncwarp();
    stage ^= 1;
  }
  cp_async_wait<0>();
  pdl_launch();

  float* smem_f = reinterpret_cast<float*>(KV);
  FinishBf16<D> fin{&a};
  attn_epilogue<D, MT>(a, m, l, o, smem_f, b, h, split, R, fin);
}

// ---------------------------------------------------------------------------
// Fused decode attention (bf16 pages): q/k RMSNorm + RoPE + KV append + SDPA.
//
// The context pages of a split do not depend on the kernel that produced q|k|v,
// so each warp starts streaming its first pages into shared memory BEFORE
// griddepcontrol.wait; their DRAM latency overlaps the previous kernel's tail.
// After the wait the CTA builds its normalised, rotated query rows, computes
// the new tokens' K/V that fall in its page range, stores them to the cache
// and patches them into the prefetched page tiles (a split is the only reader
// of its own pages in this launch).  Requires G * Lq <= 32 (one row tile).
// ---------------------------------------------------------------------------
template <int D>
__device__ __forceinline__ void fa_load_head(const uint16_t* src, int lane, float (&lo)[D / 64],
                                             float (&hi)[D / 64]) {
  constexpr int E = D / 64;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    lo[e] = bf2f(src[lane * E + e]);
    hi[e] = bf2f(src[D / 2 + lane * E + e]);
  }
}

template <int D>
__device__ __forceinline__ void fa_norm(float (&lo)[D / 64], float (&hi)[D / 64], const uint16_t* w,
                                        float eps, int lane) {
  constexpr int E = D / 64;
  float ss = 0.0f;
#pragma unroll
  for (int e = 0; e < E; ++e) ss += lo[e] * lo[e] + hi[e] * hi[e];
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(ss / (float)D + eps);
#pragma unroll
  for (int e = 0; e < E; ++e) {
    lo[e] = round_bf(lo[e] * inv * bf2f(w[lane * E + e]));
    hi[e] = round_bf(hi[e] * inv * bf2f(w[D / 2 + lane * E + e]));
  }
}

template <int D>
__device__ __forceinline__ void fa_rope(float (&lo)[D / 64], float (&hi)[D / 64], int pos,
                                        const float* inv_freq, int lane) {
  constexpr int E = D / 64;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const float th = (float)pos * inv_freq[lane * E + e];
    float sn, cs;
    sincosf(th, &sn, &cs);
    const float x0 = lo[e], x1 = hi[e];
    lo[e] = round_bf(x0 * cs - x1 * sn);
    hi[e] = round_bf(x1 * cs + x0 * sn);
  }
}

// fa_norm / fa_rope with the weight and frequency operands already in registers
template <int D>
__device__ __forceinline__ void fa_norm_r(float (&lo)[D / 64], float (&hi)[D / 64], const float (&wlo)[D / 64],
                                          const float (&whi)[D / 64], float eps) {
  constexpr int E = D / 64;
  float ss = 0.0f;
#pragma unroll
  for (int e = 0; e < E; ++e) ss += lo[e] * lo[e] + hi[e] * hi[e];
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(ss / (float)D + eps);
#pragma unroll
  for (int e = 0; e < E; ++e) {
    lo[e] = round_bf(lo[e] * inv * wlo[e]);
    hi[e] = round_bf(hi[e] * inv * whi[e]);
  }
}
template <int D>
__device__ __forceinline__ void fa_rope_r(float (&lo)[D / 64], float (&hi)[D / 64], int pos,
                                          const float (&ifq)[D / 64]) {
  constexpr int E = D / 64;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const float th = (float)pos * ifq[e];
    float sn, cs;
    sincosf(th, &sn, &cs);
    const float x0 = lo[e], x1 = hi[e];
    lo[e] = round_bf(x0 * cs - x1 * sn);
    hi[e] = round_bf(x1 * cs + x0 * sn);
  }
}

// write a head (lane layout of fa_load_head) to a swizzled smem row
template <int D>
__device__ __forceinline__ void fa_store_row(uint16_t* tile, int row, int lane,
                                             const float (&lo)[D / 64], const float (&hi)[D / 64]) {
  constexpr int E = D / 64;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int i0 = lane * E + e, i1 = D / 2 + lane * E + e;
    tile[row * D + swz(row, i0 / 8) * 8 + (i0 & 7)] = f2bf(lo[e]);
    tile[row * D + swz(row, i1 / 8) * 8 + (i1 & 7)] = f2bf(hi[e]);
  }
}

template <int D>
__device__ __forceinline__ void fa_store_gmem(uint16_t* dst, int lane, const float (&lo)[D / 64],
                                              const float (&hi)[D / 64]) {
  constexpr int E = D / 64;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    dst[lane * E + e] = f2bf(lo[e]);
    dst[D / 2 + lane * E + e] = f2bf(hi[e]);
  }
}

template <int D, int MT, int S, bool CL = false>
__global__ void __launch_bounds__(kAttnThreads) fused_attn_bf16_kernel(AttnArgs a) {
  constexpr int RP = 16 * MT;
  constexpr int PAGE_ELEMS = 16 * D;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint16_t* Qs = reinterpret_cast<uint16_t*>(smem_raw);    // [RP][D]
  uint16_t* NK = Qs + RP * D;                              // [Lq][2][D] new K / V (natural order)
  uint16_t* KV = NK + ((2 * a.Lq * D + 63) / 64) * 64;    // [4 warps][S stages][K | V]
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  HG_TL_MARK(0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int G = a.Hq / a.Hkv;
  const int Lq = a.Lq;
  const int R = G * Lq;
  const int nh = a.Hq + 2 * a.Hkv;

  // block table and lengths are host inputs of the step: safe before the wait
  const int L = a.seq_lens[b];
  const int n_pages = min((L + 15) / 16, a.max_blocks);
  const int pg0 = split * a.pages_per_split;
  const int pg1 = min(n_pages, pg0 + a.pages_per_split);
  uint16_t* my = KV + warp * S * 2 * PAGE_ELEMS;
  auto kbuf = [&](int st) { return my + st * 2 * PAGE_ELEMS; };
  auto vbuf = [&](int st) { return my + st * 2 * PAGE_ELEMS + PAGE_ELEMS; };
  auto issue = [&](int pg, int st) {
    const int pid = a.bt[(size_t)b * a.max_blocks + pg];
    const size_t off = (size_t)pid * a.page_stride + (size_t)h * a.head_stride;
    const int valid = min(16, L - pg * 16);
    load_page_bf16<D>(kbuf(st), a.kc + off, valid, lane);
    load_page_bf16<D>(vbuf(st), a.vc + off, valid, lane);
  };
#pragma unroll
  for (int s = 0; s < S - 1; ++s) {
    const int pg = pg0 + warp + 4 * s;
    if (pg < pg1) issue(pg, s);
    cp_async_commit();
  }
  issue_l2_prefetch(a.pf, (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x,
                    gridDim.x * gridDim.y * gridDim.z);

  // norm weights and RoPE frequencies are constants of the model: into registers before
  // the wait, so the query / key preparation after it waits on one load only
  constexpr int E = D / 64;
  float qwl[E], qwh[E], kwl[E], kwh[E], ifq[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    qwl[e] = a.qn ? bf2f(a.qn[lane * E + e]) : 1.0f;
    qwh[e] = a.qn ? bf2f(a.qn[D / 2 + lane * E + e]) : 1.0f;
    kwl[e] = a.kn ? bf2f(a.kn[lane * E + e]) : 1.0f;
    kwh[e] = a.kn ? bf2f(a.kn[D / 2 + lane * E + e]) : 1.0f;
    ifq[e] = a.inv_freq[lane * E + e];
  }

  pdl_wait();
  HG_TL_MARK(1);
  pdl_launch();

  // query rows: RMSNorm (Qwen3) + RoPE, straight into the swizzled Q tile
  for (int r = warp; r < RP; r += 4) {
    if (r < R) {
      const int tq = r / G, hq = h * G + r % G;
      const int tok = b * Lq + tq;
      float lo[D / 64], hi[D / 64];
      fa_load_head<D>(a.qkv + ((size_t)tok * nh + hq) * D, lane, lo, hi);
      const int ptok = a.pos[tok];
      if (a.qn) fa_norm_r<D>(lo, hi, qwl, qwh, a.eps);
      fa_rope_r<D>(lo, hi, ptok, ifq);
      fa_store_row<D>(Qs, r, lane, lo, hi);
    } else {
      for (int i = lane; i < D; i += 32) Qs[r * D + i] = 0;
    }
  }
  // the new tokens whose slots fall in this split: K (norm + RoPE) and V, to the
  // cache and to shared memory for patching the prefetched tiles
  for (int tq = warp; tq < Lq; tq += 4) {
    const int p = L - Lq + tq;
    const int pgi = p / 16;
    if (p < 0 || pgi < pg0 || pgi >= pg1) continue;
    const int tok = b * Lq + tq;
    float klo[D / 64], khi[D / 64], vlo[D / 64], vhi[D / 64];
    fa_load_head<D>(a.qkv + ((size_t)tok * nh + a.Hq + h) * D, lane, klo, khi);
    const int ptok = a.pos[tok];
    if (a.kn) fa_norm_r<D>(klo, khi, kwl, kwh, a.eps);
    fa_rope_r<D>(klo, khi, ptok, ifq);
    fa_load_head<D>(a.qkv + ((size_t)tok * nh + a.Hq + a.Hkv + h) * D, lane, vlo, vhi);
    fa_store_gmem<D>(NK + (tq * 2) * D, lane, klo, khi);
    fa_store_gmem<D>(NK + (tq * 2 + 1) * D, lane, vlo, vhi);
    const int64_t slot = a.slots ? a.slots[tok] : -1;
    if (slot >= 0) {
      const int64_t page = slot / HIGGS_PAGE_SIZE;
      const int sl = (int)(slot % HIGGS_PAGE_SIZE);
      const size_t off = (size_t)page * a.page_stride + (size_t)h * a.head_stride + (size_t)sl * D;
      fa_store_gmem<D>(a.kc_w + off, lane, klo, khi);
      fa_store_gmem<D>(a.vc_w + off, lane, vlo, vhi);
    }
  }
  __syncthreads();
  HG_TL_MARK(4);

  float m[MT][2], l[MT][2], o[MT][D / 8][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    m[mt][0] = m[mt][1] = -INFINITY;
    l[mt][0] = l[mt][1] = 0.0f;
#pragma unroll
    for (int dt = 0; dt < D / 8; ++dt)
#pragma unroll
      for (int c = 0; c < 4; ++c) o[mt][dt][c] = 0.0f;
  }

  int i = 0;
  for (int pg = pg0 + warp; pg < pg1; pg += 4, ++i) {
    const int nxt = pg + 4 * (S - 1);
    if (nxt < pg1) issue(nxt, (i + S - 1) % S);
    cp_async_commit();
    cp_async_wait<S - 1>();
    __syncwarp();
    uint16_t* Ks = kbuf(i % S);
    uint16_t* Vs = vbuf(i % S);
    // patch this launch's new tokens into the tile (the prefetch may predate them)
    for (int tq = 0; tq < Lq; ++tq) {
      const int p = L - Lq + tq;
      if (p < 0 || p / 16 != pg) continue;
      const int row = p % 16;
      for (int c = lane; c < 2 * (D / 8); c += 32) {
        const int kv = c / (D / 8), ch = c % (D / 8);
        const uint4 v = *reinterpret_cast<const uint4*>(NK + (tq * 2 + kv) * D + ch * 8);
        uint16_t* dst = (kv ? Vs : Ks) + row * D + swz(row, ch) * 8;
        *reinterpret_cast<uint4*>(dst) = v;
      }
    }
    __syncwarp();
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int kt = 0; kt < D / 16; ++kt) {
        uint32_t qa[4], kb[4];
        const int mi = lane >> 3;
        const int row = mt * 16 + (mi & 1) * 8 + (lane & 7);
        ldmatrix_x4(qa, Qs + row * D + swz(row, 2 * kt + (mi >> 1)) * 8);
        const int tok = (mi >> 1) * 8 + (lane & 7);
        ldmatrix_x4(kb, Ks + tok * D + swz(tok, 2 * kt + (mi & 1)) * 8);
        mma_bf16_16816(sc[0], qa[0], qa[1], qa[2], qa[3], kb[0], kb[1]);
        mma_bf16_16816(sc[1], qa[0], qa[1], qa[2], qa[3], kb[2], kb[3]);
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int j = pg * 16 + nt * 8 + 2 * t + (c & 1);
          const int row = mt * 16 + g + 8 * (c >> 1);
          const int qpos = L - Lq + row / G;
          const bool ok = row < R && j <= qpos;
          sc[nt][c] = ok ? sc[nt][c] * a.scale_log2 : -INFINITY;
        }
      float alpha[2];
      row_stats_update(m[mt], l[mt], sc, alpha);
#pragma unroll
      for (int dt = 0; dt < D / 8; ++dt) {
        o[mt][dt][0] *= alpha[0];
        o[mt][dt][1] *= alpha[0];
        o[mt][dt][2] *= alpha[1];
        o[mt][dt][3] *= alpha[1];
      }
      uint32_t ph[4], pl[4];
      split_bf2(sc[0][0], sc[0][1], ph[0], pl[0]);
      split_bf2(sc[0][2], sc[0][3], ph[1], pl[1]);
      split_bf2(sc[1][0], sc[1][1], ph[2], pl[2]);
      split_bf2(sc[1][2], sc[1][3], ph[3], pl[3]);
#pragma unroll
      for (int d2 = 0; d2 < D / 16; ++d2) {
        uint32_t vb[4];
        const int mi = lane >> 3;
        const int tok = (mi & 1) * 8 + (lane & 7);
        ldmatrix_x4_trans(vb, Vs + tok * D + swz(tok, 2 * d2 + (mi >> 1)) * 8);
        mma_bf16_16816(o[mt][2 * d2], ph[0], ph[1], ph[2], ph[3], vb[0], vb[1]);
        mma_bf16_16816(o[mt][2 * d2 + 1], ph[0], ph[1], ph[2], ph[3], vb[2], vb[3]);
        mma_bf16_16816(o[mt][2 * d2], pl[0], pl[1], pl[2], pl[3], vb[0], vb[1]);
        mma_bf16_16816(o[mt][2 * d2 + 1], pl[0], pl[1], pl[2], pl[3], vb[2], vb[3]);
      }
    }
    __syncwarp();
  }
  cp_async_wait<0>();

  float* smem_f = reinterpret_cast<float*>(KV);
  AttnArgs ao = a;
  ao.tq0 = 0;
  FinishBf16<D> fin{&ao};
  HG_TL_MARK(5);
  attn_epilogue<D, MT, FinishBf16<D>, CL>(a, m, l, o, smem_f, b, h, split, R, fin);
}

// ---------------------------------------------------------------------------
// TurboQuant pages (D = 128)
// ---------------------------------------------------------------------------
// Physical position j within an 8-wide d chunk holds natural nibble kPerm[j].
__device__ __constant__ int kPerm[8] = {0, 4, 1, 5, 2, 6, 3, 7};

// Inverse rotation R^T = diag(sign) H / sqrt(128) of one row held as lane l:
// natural elements 2l, 2l+1, 64+2l, 65+2l.
__device__ __forceinline__ void tq_unrotate_lane(float (&f)[4], const int8_t* signs, int lane) {
  {
    float a0 = f[0], b0 = f[1];
    f[0] = a0 + b0;
    f[1] = a0 - b0;
    a0 = f[2];
    b0 = f[3];
    f[2] = a0 + b0;
    f[3] = a0 - b0;
  }
#pragma unroll
  for (int hl = 1; hl <= 16; hl <<= 1) {
    const bool upper = (lane & hl) != 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float other = __shfl_xor_sync(0xffffffffu, f[e], hl);
      f[e] = upper ? other - f[e] : f[e] + other;
    }
  }
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const float a0 = f[e], b0 = f[e + 2];
    f[e] = a0 + b0;
    f[e + 2] = a0 - b0;
  }
  const int idx[4] = {2 * lane, 2 * lane + 1, 64 + 2 * lane, 65 + 2 * lane};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    f[e] *= 0.0883883476483184406f;
    if (signs[idx[e]] < 0) f[e] = -f[e];
  }
}

__device__ __forceinline__ void tq_rotate_lane(float (&f)[4], const int8_t* signs, int lane) {
  const int idx[4] = {2 * lane, 2 * lane + 1, 64 + 2 * lane, 65 + 2 * lane};
#pragma unroll
  for (int e = 0; e < 4; ++e)
    if (signs[idx[e]] < 0) f[e] = -f[e];
  {
    float a0 = f[0], b0 = f[1];
    f[0] = a0 + b0;
    f[1] = a0 - b0;
    a0 = f[2];
    b0 = f[3];
    f[2] = a0 + b0;
    f[3] = a0 - b0;
  }
#pragma unroll
  for (int hl = 1; hl <= 16; hl <<= 1) {
    const bool upper = (lane & hl) != 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float other = __shfl_xor_sync(0xffffffffu, f[e], hl);
      f[e] = upper ? other - f[e] : f[e] + other;
    }
  }
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const float a0 = f[e], b0 = f[e + 2];
    f[e] = a0 + b0;
    f[e + 2] = a0 - b0;
  }
#pragma unroll
  for (int e = 0; e < 4; ++e) f[e] *= 0.0883883476483184406f;
}

struct FinishTq4 {
  const AttnArgs* a;
  __device__ void operator()(const float* sm_o, int R, int b, int h) const {
    const int G = a->Hq / a->Hkv;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int row = warp; row < R; row += 4) {
      // gather natural order from the physical (chunk-permuted) layout
      auto phys = [](int d) {
        const int c = d >> 3, n = d & 7;
        // natural nibble n sits at physical j with kPerm[j] == n
        const int j = (n < 4) ? 2 * n : 2 * (n - 4) + 1;
        return c * 8 + j;
      };
      const float* r = sm_o + row * 128;
      float f[4] = {r[phys(2 * lane)], r[phys(2 * lane + 1)], r[phys(64 + 2 * lane)],
                    r[phys(65 + 2 * lane)]};
      tq_unrotate_lane(f, a->signs, lane);
      const int tq = a->tq0 + row / G, hq = h * G + row % G;
      uint16_t* op = a->out + (((size_t)b * a->Lq + tq) * a->Hq + hq) * 128;
      *reinterpret_cast<uint32_t*>(op + 2 * lane) = pack_bf2(f[0], f[1]);
      *reinterpret_cast<uint32_t*>(op + 64 + 2 * lane) = pack_bf2(f[2], f[3]);
    }
  }
};

template <int MT, bool PLO = true>
__global__ void __launch_bounds__(kAttnThreads) paged_attn_tq4_kernel(AttnArgs a) {
  constexpr int D = 128;
  constexpr int RP = 16 * MT;
  // smem: qfrag [MT][8 kt][32 lanes][hi 4 | lo 4] u32 | qsum [RP] f32 |
  //       per warp: kTq4Stages stages x {kcodes 1 KB, vcodes 1 KB, kscale 32 B, vscale 32 B},
  //       two V tiles bf16 4 KB each | qrot [RP][128] f32 query scratch
  // (the rings fill before the query rotation, so the scratch cannot share their bytes)
  constexpr int S = kTq4Stages;
  constexpr int STAGE_BYTES = 1024 + 1024 + 32 + 32;
  constexpr int WARP_BYTES = S * STAGE_BYTES + 2 * 16 * D * 2;  // + two V tiles
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint32_t* qfrag = reinterpret_cast<uint32_t*>(smem_raw);
  float* qsum = reinterpret_cast<float*>(qfrag + MT * 8 * 32 * 8);
  uint8_t* wbase = reinterpret_cast<uint8_t*>(qsum + RP);
  float* qrot = reinterpret_cast<float*>(wbase + 4 * WARP_BYTES);
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int G = a.Hq / a.Hkv;
  const int R = G * a.lq_chunk;

  // block table and lengths are inputs of the step (not written by the previous kernel)
  const int L = a.seq_lens[b];
  const int n_pages = min((L + 15) / 16, a.max_blocks);
  const int pg0 = split * a.pages_per_split;
  const int pg1 = min(n_pages, pg0 + a.pages_per_split);
  uint8_t* my = wbase + warp * WARP_BYTES;
  auto kcb = [&](int st) { return my + st * STAGE_BYTES; };
  auto vcb = [&](int st) { return my + st * STAGE_BYTES + 1024; };
  auto ksb = [&](int st) { return reinterpret_cast<__half*>(my + st * STAGE_BYTES + 2048); };
  auto vsb = [&](int st) { return reinterpret_cast<__half*>(my + st * STAGE_BYTES + 2080); };
  auto issue = [&](int pg, int st) {
    const int pid = a.bt[(size_t)b * a.max_blocks + pg];
    const size_t off = (size_t)pid * a.page_stride + (size_t)h * a.head_stride;
    const size_t soff = (size_t)pid * (a.page_stride / 64) + (size_t)h * (a.head_stride / 64);
    const int valid = min(16, L - pg * 16);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int qd = lane + 32 * i;  // 64 chunks of 16 B = 16 rows x 64 B
      const int r = qd >> 2;
      const int bytes = r < valid ? 16 : 0;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(kcb(st) + qd * 16)),
                   "l"(a.kcode + off + qd * 16), "r"(bytes));
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(vcb(st) + qd * 16)),
                   "l"(a.vcode + off + qd * 16), "r"(bytes));
    }
    if (lane < 2) {
      const int bytes = (lane * 8 < valid) ? 16 : 0;  // each 16 B chunk = 8 scales
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(ksb(st) + lane * 8)),
                   "l"(a.kscale + soff + lane * 8), "r"(bytes));
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(vsb(st) + lane * 8)),
                   "l"(a.vscale + soff + lane * 8), "r"(bytes));
    }
  };
  // the first PRO pages of this warp into the ring; pages holding only tokens of earlier
  // steps (the previous kernel appends this step's) are fetched before the dependency wait
  constexpr int PRO = S - 2;  // pages in flight beyond the pair being processed
  int pre = 0;
  const int old_end = L - a.Lq;  // positions below this were written by earlier steps
  for (; pre < PRO; ++pre) {
    const int pgs = pg0 + warp + 4 * pre;
    if (pgs >= pg1 || (pgs + 1) * 16 > old_end) break;
    issue(pgs, pre);
    cp_async_commit();
  }
  pdl_wait();
  for (; pre < PRO; ++pre) {
    const int pgs = pg0 + warp + 4 * pre;
    if (pgs < pg1) issue(pgs, pre);
    cp_async_commit();
  }

  // rotate the query rows: q' = R q, rounded to bf16 (the MMA operand), and
  // the per-row sum of the rounded q' (removes the +136 code offset)
  for (int row = warp; row < RP; row += 4) {
    float f[4] = {0.f, 0.f, 0.f, 0.f};
    if (row < R) {
      const int tq = a.tq0 + row / G, hq = h * G + row % G;
      const uint16_t* qp = a.q + (((size_t)b * a.Lq + tq) * a.Hq + hq) * D;
      f[0] = bf2f(qp[2 * lane]);
      f[1] = bf2f(qp[2 * lane + 1]);
      f[2] = bf2f(qp[64 + 2 * lane]);
      f[3] = bf2f(qp[65 + 2 * lane]);
      tq_rotate_lane(f, a.signs, lane);
    }
    // q' goes to the MMA as hi + lo bf16; the offset correction uses their exact sum
    float sum = 0.0f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float hi = round_bf(f[e]);
      f[e] = hi + round_bf(f[e] - hi);
      sum += f[e];
    }
    sum = warp_sum(sum);
    if (lane == 0) qsum[row] = sum;
    float* dst = qrot + row * D;
    dst[2 * lane] = f[0];
    dst[2 * lane + 1] = f[1];
    dst[64 + 2 * lane] = f[2];
    dst[65 + 2 * lane] = f[3];
  }
  __syncthreads();
  // A fragments in the code-nibble k order: tile kt, lane (g, t):
  //   lo = 32t + 8(kt>>1) + 2(kt&1): a0 = (lo, lo+4), a2 = (lo+1, lo+5); a1/a3 row g+8
  for (int i = threadIdx.x; i < MT * 8 * 32; i += kAttnThreads) {
    const int mt = i / 256, kt = (i / 32) % 8, ln = i % 32;
    const int gg = ln >> 2, tt = ln & 3;
    const int lo = 32 * tt + 8 * (kt >> 1) + 2 * (kt & 1);
    const float* r0 = qrot + (mt * 16 + gg) * D;
    const float* r1 = qrot + (mt * 16 + gg + 8) * D;
    uint32_t* dst = qfrag + (size_t)i * 8;
    split_bf2(r0[lo], r0[lo + 4], dst[0], dst[4]);
    split_bf2(r1[lo], r1[lo + 4], dst[1], dst[5]);
    split_bf2(r0[lo + 1], r0[lo + 5], dst[2], dst[6]);
    split_bf2(r1[lo + 1], r1[lo + 5], dst[3], dst[7]);
  }
  __syncthreads();

  float m[MT][2], l[MT][2], o[MT][D / 8][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    m[mt][0] = m[mt][1] = -INFINITY;
    l[mt][0] = l[mt][1] = 0.0f;
#pragma unroll
    for (int dt = 0; dt < D / 8; ++dt)
#pragma unroll
      for (int c = 0; c < 4; ++c) o[mt][dt][c] = 0.0f;
  }
  float qs[MT][2];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    qs[mt][0] = qsum[mt * 16 + g];
    qs[mt][1] = qsum[mt * 16 + g + 8];
  }
  // one 16-row tile: its query fragments stay in registers for the whole page loop
  // instead of being re-read from shared memory for every page
  uint4 qreg[MT == 1 ? 8 : 1][2];
  if constexpr (MT == 1) {
#pragma unroll
    for (int kt = 0; kt < 8; ++kt) {
      const uint4* qp = reinterpret_cast<const uint4*>(qfrag + (kt * 32 + lane) * 8);
      qreg[kt][0] = qp[0];
      qreg[kt][1] = qp[1];
    }
  }

  // two pages per iteration: their score chains interleave and one online-softmax update
  // covers both (32 keys); a page past the split is empty (its keys are masked)
  uint16_t* vtile0 = reinterpret_cast<uint16_t*>(my + S * STAGE_BYTES);
  uint16_t* vtile1 = vtile0 + 16 * D;
  auto expand_v = [&](int st, uint16_t* vtile) {
    // V codes to exact bf16 (c - 8): lane -> token lane/2, half lane&1
    const int r = lane >> 1, hlf = lane & 1;
    const uint4* src = reinterpret_cast<const uint4*>(vcb(st) + r * 64 + hlf * 32);
#pragma unroll
    for (int v4 = 0; v4 < 2; ++v4) {
      const uint4 w4 = src[v4];
      const uint32_t ws[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
      for (int wi = 0; wi < 4; ++wi) {
        const int chunk = hlf * 8 + v4 * 4 + wi;
        const uint32_t off136 = 0x43084308u;  // bf16 pair (136, 136)
        const __nv_bfloat162 o136 = *reinterpret_cast<const __nv_bfloat162*>(&off136);
        uint32_t p[4] = {nib_pair_bf16<0>(ws[wi]), nib_pair_bf16<4>(ws[wi]), nib_pair_bf16<8>(ws[wi]),
                         nib_pair_bf16<12>(ws[wi])};
        uint32_t q[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const __nv_bfloat162 d = __hsub2(*reinterpret_cast<__nv_bfloat162*>(&p[e]), o136);
          q[e] = *reinterpret_cast<const uint32_t*>(&d);
        }
        *reinterpret_cast<uint4*>(vtile + r * D + swz(r, chunk) * 8) = make_uint4(q[0], q[1], q[2], q[3]);
      }
    }
  };

  int j = 0;  // this warp's local page index (the pair j, j + 1)
  for (int pg = pg0 + warp; pg < pg1; pg += 8, j += 2) {
#pragma unroll
    for (int u = 0; u < 2; ++u) {  // refill the slots the previous pair released
      const int p2 = pg + 4 * (PRO + u);
      if (p2 < pg1) issue(p2, (j + PRO + u) % S);
      cp_async_commit();
    }
    cp_async_wait<PRO>();  // pages j and j + 1 have landed
    __syncwarp();
    const int st0 = j % S, st1 = (j + 1) % S;
    const int pgp[2] = {pg, pg + 4};
    expand_v(st0, vtile0);
    expand_v(st1, vtile1);
    __syncwarp();
    // per-token scales of the key columns this lane owns (n-tiles 0-1 page a, 2-3 page b)
    float ksc[4][2], vsc[4][2];
#pragma unroll
    for (int pp = 0; pp < 2; ++pp) {
      // a second page past this split's range (it may still be in the sequence) is empty
      const int valid = pgp[pp] < pg1 ? min(16, L - pgp[pp] * 16) : 0;
      const __half* ks = ksb(pp ? st1 : st0);
      const __half* vs = vsb(pp ? st1 : st0);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int jj = nt * 8 + 2 * t + e;
          ksc[2 * pp + nt][e] = jj < valid ? __half2float(ks[jj]) : 0.0f;
          vsc[2 * pp + nt][e] = jj < valid ? __half2float(vs[jj]) : 0.0f;
        }
    }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      // the hi and lo halves of q' accumulate separately: short, independent MMA chains
      float s[4][4], sl[4][4];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int c = 0; c < 4; ++c) s[nt][c] = sl[nt][c] = 0.0f;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const uint8_t* kc = kcb((nt >> 1) ? st1 : st0);
        const uint4 kw = *reinterpret_cast<const uint4*>(kc + ((nt & 1) * 8 + g) * 64 + 16 * t);
        const uint32_t kws[4] = {kw.x, kw.y, kw.z, kw.w};
#pragma unroll
        for (int kt = 0; kt < 8; ++kt) {
          uint4 qa, ql;
          if constexpr (MT == 1) {
            qa = qreg[kt][0];
            ql = qreg[kt][1];
          } else {
            const uint4* qp = reinterpret_cast<const uint4*>(qfrag + ((mt * 8 + kt) * 32 + lane) * 8);
            qa = qp[0];
            ql = qp[1];
          }
          const uint32_t w = kws[kt >> 1];
          const uint32_t b0 = (kt & 1) ? nib_pair_bf16<8>(w) : nib_pair_bf16<0>(w);
          const uint32_t b1 = (kt & 1) ? nib_pair_bf16<12>(w) : nib_pair_bf16<4>(w);
          mma_bf16_16816(s[nt], qa.x, qa.y, qa.z, qa.w, b0, b1);
          mma_bf16_16816(sl[nt], ql.x, ql.y, ql.z, ql.w, b0, b1);
        }
      }
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int jk = pgp[nt >> 1] * 16 + (nt & 1) * 8 + 2 * t + (c & 1);
          const int row = mt * 16 + g + 8 * (c >> 1);
          const int qpos = L - a.Lq + a.tq0 + row / G;
          const bool ok = row < R && jk <= qpos && pgp[nt >> 1] < pg1;
          const float raw = (s[nt][c] + sl[nt][c]) - 136.0f * qs[mt][c >> 1];
          s[nt][c] = ok ? raw * ksc[nt][c & 1] * a.scale_log2 : -INFINITY;
        }
      float alpha[2];
      row_stats_update(m[mt], l[mt], s, alpha);
#pragma unroll
      for (int dt = 0; dt < D / 8; ++dt) {
        o[mt][dt][0] *= alpha[0];
        o[mt][dt][1] *= alpha[0];
        o[mt][dt][2] *= alpha[1];
        o[mt][dt][3] *= alpha[1];
      }
      // P scaled by the per-token V scale; page a's keys are the first k-step, page b's the
      // second.  PLO: P enters the MMA as hi + lo bf16 halves; without it, as its bf16 rounding
      // (half the P x V MMAs; measured error within the TurboQuant attention bound)
      uint32_t ph[2][4], pl[2][4];
#pragma unroll
      for (int pp = 0; pp < 2; ++pp) {
        const int n0 = 2 * pp;
        split_bf2(s[n0][0] * vsc[n0][0], s[n0][1] * vsc[n0][1], ph[pp][0], pl[pp][0]);
        split_bf2(s[n0][2] * vsc[n0][0], s[n0][3] * vsc[n0][1], ph[pp][1], pl[pp][1]);
        split_bf2(s[n0 + 1][0] * vsc[n0 + 1][0], s[n0 + 1][1] * vsc[n0 + 1][1], ph[pp][2], pl[pp][2]);
        split_bf2(s[n0 + 1][2] * vsc[n0 + 1][0], s[n0 + 1][3] * vsc[n0 + 1][1], ph[pp][3], pl[pp][3]);
      }
#pragma unroll
      for (int d2 = 0; d2 < D / 16; ++d2) {
        const int mi = lane >> 3;
        const int tok = (mi & 1) * 8 + (lane & 7);
#pragma unroll
        for (int pp = 0; pp < 2; ++pp) {
          uint32_t vb[4];
          ldmatrix_x4_trans(vb, (pp ? vtile1 : vtile0) + tok * D + swz(tok, 2 * d2 + (mi >> 1)) * 8);
          mma_bf16_16816(o[mt][2 * d2], ph[pp][0], ph[pp][1], ph[pp][2], ph[pp][3], vb[0], vb[1]);
          mma_bf16_16816(o[mt][2 * d2 + 1], ph[pp][0], ph[pp][1], ph[pp][2], ph[pp][3], vb[2], vb[3]);
          if constexpr (PLO) {
            mma_bf16_16816(o[mt][2 * d2], pl[pp][0], pl[pp][1], pl[pp][2], pl[pp][3], vb[0], vb[1]);
            mma_bf16_16816(o[mt][2 * d2 + 1], pl[pp][0], pl[pp][1], pl[pp][2], pl[pp][3], vb[2], vb[3]);
          }
        }
      }
    }
    __syncwarp();
  }
  cp_async_wait<0>();
  pdl_launch();

  float* smem_f = reinterpret_cast<float*>(wbase);  // rings and query scratch are dead now
  FinishTq4 fin{&a};
  attn_epilogue<D, MT>(a, m, l, o, smem_f, b, h, split, R, fin);
}

// TurboQuant decode with the MMA roles swapped, for launches of at most 4 query rows (one
// token of a GQA group of 4 or fewer heads -- C5's decode).  The kernel above puts the
// query rows on the 16-row side of m16n8k16, so 12 of its 16 rows are padding, and splits
// q' into hi + lo halves on separate MMAs.  Here the keys are the 16 rows: a page's scores
// are S^T = K q'^T with the 8 columns holding the rows' hi halves (columns 0-3) and lo
// halves (columns 4-7) of q', so one MMA per 16 d does what took eight; the output is
// O^T = V^T P^T with the head dimension on the rows (8 MMAs per page instead of 16), P^T
// formed from the score fragments by lane shuffles.  Accumulators: 32 registers of O^T and
// 16 of q' instead of 64 and 64.  Same page ring, masking and epilogue as the kernel above;
// V is expanded to 128 + c and the offset removed once per row (results differ from the
// kernel above only in f32 summation order).
template <int S>
__global__ void __launch_bounds__(kAttnThreads, 3) paged_attn_tq4_swap_kernel(AttnArgs a) {
  constexpr int D = 128;
  constexpr int STAGE_BYTES = 1024 + 1024 + 32 + 32;
  constexpr int WARP_BYTES = S * STAGE_BYTES + 2 * 16 * D * 2;  // + two V tiles
  // smem: qsum [4] | pad | qrot [4][128] f32 | per warp: S stages + two V tiles
  extern __shared__ __align__(128) uint8_t smem_raw[];
  float* qsum = reinterpret_cast<float*>(smem_raw);
  float* qrot = qsum + 32;
  uint8_t* wbase = reinterpret_cast<uint8_t*>(qrot + 4 * D);
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int G = a.Hq / a.Hkv;
  const int R = G * a.lq_chunk;  // <= 4

  const int L = a.seq_lens[b];
  const int n_pages = min((L + 15) / 16, a.max_blocks);
  const int pg0 = split * a.pages_per_split;
  const int pg1 = min(n_pages, pg0 + a.pages_per_split);
  uint8_t* my = wbase + warp * WARP_BYTES;
  auto kcb = [&](int st) { return my + st * STAGE_BYTES; };
  auto vcb = [&](int st) { return my + st * STAGE_BYTES + 1024; };
  auto ksb = [&](int st) { return reinterpret_cast<__half*>(my + st * STAGE_BYTES + 2048); };
  auto vsb = [&](int st) { return reinterpret_cast<__half*>(my + st * STAGE_BYTES + 2080); };
  auto issue = [&](int pg, int st) {
    const int pid = a.bt[(size_t)b * a.max_blocks + pg];
    const size_t off = (size_t)pid * a.page_stride + (size_t)h * a.head_stride;
    const size_t soff = (size_t)pid * (a.page_stride / 64) + (size_t)h * (a.head_stride / 64);
    const int valid = min(16, L - pg * 16);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int qd = lane + 32 * i;  // 64 chunks of 16 B = 16 rows x 64 B
      const int r = qd >> 2;
      const int bytes = r < valid ? 16 : 0;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(kcb(st) + qd * 16)),
                   "l"(a.kcode + off + qd * 16), "r"(bytes));
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(vcb(st) + qd * 16)),
                   "l"(a.vcode + off + qd * 16), "r"(bytes));
    }
    if (lane < 2) {
      const int bytes = (lane * 8 < valid) ? 16 : 0;  // each 16 B chunk = 8 scales
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(ksb(st) + lane * 8)),
                   "l"(a.kscale + soff + lane * 8), "r"(bytes));
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(vsb(st) + lane * 8)),
                   "l"(a.vscale + soff + lane * 8), "r"(bytes));
    }
  };
  // the first PRO pages of this warp into the ring; pages holding only tokens of earlier
  // steps are fetched before the dependency wait
  constexpr int PRO = S - 2;
  int pre = 0;
  const int old_end = L - a.Lq;
  for (; pre < PRO; ++pre) {
    const int pgs = pg0 + warp + 4 * pre;
    if (pgs >= pg1 || (pgs + 1) * 16 > old_end) break;
    issue(pgs, pre);
    cp_async_commit();
  }
  pdl_wait();
  for (; pre < PRO; ++pre) {
    const int pgs = pg0 + warp + 4 * pre;
    if (pgs < pg1) issue(pgs, pre);
    cp_async_commit();
  }

  // rotate the query rows (warp w: row w): q' = R q; the scores use its hi + lo bf16 halves
  // and the code offset correction their exact sum
  {
    const int row = warp;
    float f[4] = {0.f, 0.f, 0.f, 0.f};
    if (row < R) {
      const int tq = a.tq0 + row / G, hq = h * G + row % G;
      const uint16_t* qp = a.q + (((size_t)b * a.Lq + tq) * a.Hq + hq) * D;
      f[0] = bf2f(qp[2 * lane]);
      f[1] = bf2f(qp[2 * lane + 1]);
      f[2] = bf2f(qp[64 + 2 * lane]);
      f[3] = bf2f(qp[65 + 2 * lane]);
      tq_rotate_lane(f, a.signs, lane);
    }
    float sum = 0.0f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float hi = round_bf(f[e]);
      sum += hi + round_bf(f[e] - hi);
    }
    sum = warp_sum(sum);
    if (lane == 0) qsum[row] = sum;
    float* dst = qrot + row * D;
    dst[2 * lane] = f[0];
    dst[2 * lane + 1] = f[1];
    dst[64 + 2 * lane] = f[2];
    dst[65 + 2 * lane] = f[3];
  }
  __syncthreads();
  // B fragments of q'^T in the code-nibble k order of the K codes (k-step kt, lane (g, t):
  // lo = 32t + 8(kt>>1) + 2(kt&1), k rows 2t, 2t+1 <-> d lo, lo+4 and 2t+8, 2t+9 <-> lo+1,
  // lo+5); column g is row g's hi half (g < 4) or row g-4's lo half, zero past R
  uint32_t qb[8][2];
  {
    const int row = g & 3;
    const bool use_lo = g >= 4;
    const float* r = qrot + row * D;
#pragma unroll
    for (int kt = 0; kt < 8; ++kt) {
      const int lo = 32 * t + 8 * (kt >> 1) + 2 * (kt & 1);
      uint32_t h0, l0, h1, l1;
      split_bf2(r[lo], r[lo + 4], h0, l0);
      split_bf2(r[lo + 1], r[lo + 5], h1, l1);
      qb[kt][0] = row < R ? (use_lo ? l0 : h0) : 0u;
      qb[kt][1] = row < R ? (use_lo ? l1 : h1) : 0u;
    }
  }
  // this lane's score columns after the hi + lo fold: rows ra = 2(t & 1) and ra + 1
  const int ra = 2 * (t & 1);
  const float qs0 = qsum[ra], qs1 = qsum[ra + 1];
  const int qpos0 = L - a.Lq + a.tq0 + ra / G, qpos1 = L - a.Lq + a.tq0 + (ra + 1) / G;
  float o[D / 16][4];  // O^T: tile d2 = rows d 16 d2 + g (+8), columns = query rows 2t, 2t + 1
#pragma unroll
  for (int d2 = 0; d2 < D / 16; ++d2)
#pragma unroll
    for (int c = 0; c < 4; ++c) o[d2][c] = 0.0f;
  float mr[2] = {-INFINITY, -INFINITY}, lr[2] = {0.0f, 0.0f};  // rows ra, ra + 1
  float pr[2] = {0.0f, 0.0f};  // sum of the bf16 P x V-scale weights this lane fed the MMA

  uint16_t* vtile0 = reinterpret_cast<uint16_t*>(my + S * STAGE_BYTES);
  uint16_t* vtile1 = vtile0 + 16 * D;
  auto expand_v = [&](int st, uint16_t* vtile) {
    // V codes to the exact bf16 128 + c (the offset 136 of the dequantized c - 8 comes off
    // once per row at the end); lane -> token lane/2, half lane&1, its 16-byte chunks visited
    // in an order staggered by token pair and half so that neither the code reads nor the
    // swizzled tile writes of a quarter-warp share a bank
    const int r = lane >> 1, hlf = lane & 1;
    const uint4* src = reinterpret_cast<const uint4*>(vcb(st) + r * 64 + hlf * 32);
#pragma unroll
    for (int v4i = 0; v4i < 2; ++v4i) {
      const int v4 = v4i ^ ((r >> 1) & 1);
      const uint4 w4 = src[v4];
      const uint32_t ws[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
      for (int wi0 = 0; wi0 < 4; ++wi0) {
        const uint32_t w = hlf ? ws[wi0 ^ 2] : ws[wi0];
        const int chunk = hlf * 8 + v4 * 4 + (wi0 ^ (2 * hlf));
        *reinterpret_cast<uint4*>(vtile + r * D + swz(r, chunk) * 8) =
            make_uint4(nib_pair_bf16<0>(w), nib_pair_bf16<4>(w), nib_pair_bf16<8>(w), nib_pair_bf16<12>(w));
      }
    }
  };

  int j = 0;  // this warp's local page index (the pair j, j + 1)
  for (int pg = pg0 + warp; pg < pg1; pg += 8, j += 2) {
#pragma unroll
    for (int u = 0; u < 2; ++u) {  // refill the slots the previous pair released
      const int p2 = pg + 4 * (PRO + u);
      if (p2 < pg1) issue(p2, (j + PRO + u) % S);
      cp_async_commit();
    }
    cp_async_wait<PRO>();  // pages j and j + 1 have landed
    __syncwarp();
    const int st0 = j % S, st1 = (j + 1) % S;
    const int pgp[2] = {pg, pg + 4};
    expand_v(st0, vtile0);
    expand_v(st1, vtile1);
    __syncwarp();
    // scores S^T of both pages: sc[pp][c], c = 0 (key g, row ra), 1 (key g, row ra + 1),
    // 2 (key g + 8, row ra), 3 (key g + 8, row ra + 1)
    float sc[2][4], vs[2][2];
#pragma unroll
    for (int pp = 0; pp < 2; ++pp) {
      const int st = pp ? st1 : st0;
      const int valid = pgp[pp] < pg1 ? min(16, L - pgp[pp] * 16) : 0;
      const uint8_t* kc = kcb(st);
      const uint4 kv0 = *reinterpret_cast<const uint4*>(kc + g * 64 + 16 * t);
      const uint4 kv1 = *reinterpret_cast<const uint4*>(kc + (g + 8) * 64 + 16 * t);
      const uint32_t k0[4] = {kv0.x, kv0.y, kv0.z, kv0.w}, k1[4] = {kv1.x, kv1.y, kv1.z, kv1.w};
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kt = 0; kt < 8; ++kt) {
        const uint32_t w0 = k0[kt >> 1], w1 = k1[kt >> 1];
        const uint32_t a0 = (kt & 1) ? nib_pair_bf16<8>(w0) : nib_pair_bf16<0>(w0);
        const uint32_t a2 = (kt & 1) ? nib_pair_bf16<12>(w0) : nib_pair_bf16<4>(w0);
        const uint32_t a1 = (kt & 1) ? nib_pair_bf16<8>(w1) : nib_pair_bf16<0>(w1);
        const uint32_t a3 = (kt & 1) ? nib_pair_bf16<12>(w1) : nib_pair_bf16<4>(w1);
        mma_bf16_16816(acc, a0, a1, a2, a3, qb[kt][0], qb[kt][1]);
      }
      // the lo-half columns (lanes t ^ 2) onto the hi-half ones: every lane gets rows ra, ra + 1
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[c] += __shfl_xor_sync(0xffffffffu, acc[c], 2);
      const __half* ks = ksb(st);
      const __half* vsp = vsb(st);
      const float kg = g < valid ? __half2float(ks[g]) : 0.0f;
      const float kg8 = g + 8 < valid ? __half2float(ks[g + 8]) : 0.0f;
      vs[pp][0] = g < valid ? __half2float(vsp[g]) : 0.0f;
      vs[pp][1] = g + 8 < valid ? __half2float(vsp[g + 8]) : 0.0f;
      const int key0 = pgp[pp] * 16 + g, key1 = key0 + 8;
      const bool inpg = pgp[pp] < pg1;
      sc[pp][0] = (ra < R && key0 <= qpos0 && inpg) ? (acc[0] - 136.0f * qs0) * kg * a.scale_log2 : -INFINITY;
      sc[pp][1] = (ra + 1 < R && key0 <= qpos1 && inpg) ? (acc[1] - 136.0f * qs1) * kg * a.scale_log2 : -INFINITY;
      sc[pp][2] = (ra < R && key1 <= qpos0 && inpg) ? (acc[2] - 136.0f * qs0) * kg8 * a.scale_log2 : -INFINITY;
      sc[pp][3] = (ra + 1 < R && key1 <= qpos1 && inpg) ? (acc[3] - 136.0f * qs1) * kg8 * a.scale_log2 : -INFINITY;
    }
    // online softmax per query row (a column of S^T): the maximum over the 32 keys of the
    // pair lives across the 8 lanes g of a column pair
    float alpha[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float mx = fmaxf(fmaxf(sc[0][r], sc[0][r + 2]), fmaxf(sc[1][r], sc[1][r + 2]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
      const float mn = fmaxf(mr[r], mx);
      alpha[r] = (mn == -INFINITY) ? 1.0f : exp2f(mr[r] - mn);
      mr[r] = mn;
      float rs = 0.0f;
#pragma unroll
      for (int pp = 0; pp < 2; ++pp)
#pragma unroll
        for (int e = r; e < 4; e += 2) {
          float& v = sc[pp][e];
          v = (mn == -INFINITY) ? 0.0f : exp2f(v - mn);
          rs += v;
        }
      lr[r] = lr[r] * alpha[r] + rs;  // this lane's keys; summed over the lanes at the end
      pr[r] *= alpha[r];
    }
#pragma unroll
    for (int d2 = 0; d2 < D / 16; ++d2) {
      o[d2][0] *= alpha[0];
      o[d2][2] *= alpha[0];
      o[d2][1] *= alpha[1];
      o[d2][3] *= alpha[1];
    }
    // O^T += V^T P^T per page: P (times the key's V scale, rounded to bf16) gathered into the
    // B fragment of lane (g, t) = column row g, keys 2t, 2t + 1 | 2t + 8, 2t + 9, from the
    // lanes (2t, g/2) and (2t + 1, g/2) that hold those keys' scores
#pragma unroll
    for (int pp = 0; pp < 2; ++pp) {
      const uint32_t pk0 = pack_bf2(sc[pp][0] * vs[pp][0], sc[pp][1] * vs[pp][0]);
      const uint32_t pk1 = pack_bf2(sc[pp][2] * vs[pp][1], sc[pp][3] * vs[pp][1]);
      pr[0] += bf_lo(pk0) + bf_lo(pk1);
      pr[1] += bf_hi(pk0) + bf_hi(pk1);
      const int rr = g & 3;
      const int l1 = (2 * t) * 4 + (rr >> 1), l2 = (2 * t + 1) * 4 + (rr >> 1);
      const uint32_t u0 = __shfl_sync(0xffffffffu, pk0, l1), u1 = __shfl_sync(0xffffffffu, pk0, l2);
      const uint32_t u2 = __shfl_sync(0xffffffffu, pk1, l1), u3 = __shfl_sync(0xffffffffu, pk1, l2);
      const uint32_t sel = (rr & 1) ? 0x7632u : 0x5410u;
      const uint32_t pb0 = g < R ? prmt(u0, u1, sel) : 0u;
      const uint32_t pb1 = g < R ? prmt(u2, u3, sel) : 0u;
      const uint16_t* vt = pp ? vtile1 : vtile0;
      const int mi = lane >> 3;
      const int tok = (mi & 1) * 8 + (lane & 7);
#pragma unroll
      for (int d2 = 0; d2 < D / 16; ++d2) {
        uint32_t vb[4];
        ldmatrix_x4_trans(vb, vt + tok * D + swz(tok, 2 * d2 + (mi >> 1)) * 8);
        mma_bf16_16816(o[d2], vb[0], vb[2], vb[1], vb[3], pb0, pb1);
      }
    }
    __syncwarp();
  }
  cp_async_wait<0>();
  pdl_launch();

#pragma unroll
  for (int r = 0; r < 2; ++r) {
    lr[r] += __shfl_xor_sync(0xffffffffu, lr[r], 4);
    lr[r] += __shfl_xor_sync(0xffffffffu, lr[r], 8);
    lr[r] += __shfl_xor_sync(0xffffffffu, lr[r], 16);
    pr[r] += __shfl_xor_sync(0xffffffffu, pr[r], 4);
    pr[r] += __shfl_xor_sync(0xffffffffu, pr[r], 8);
    pr[r] += __shfl_xor_sync(0xffffffffu, pr[r], 16);
  }
  // the MMAs saw V as 128 + c: O^T[d][row] -= 136 * (the weights of that row)
#pragma unroll
  for (int d2 = 0; d2 < D / 16; ++d2) {
    o[d2][0] -= 136.0f * pr[0];
    o[d2][2] -= 136.0f * pr[0];
    o[d2][1] -= 136.0f * pr[1];
    o[d2][3] -= 136.0f * pr[1];
  }
  // to the kernel above's fragment layout (rows = query rows) through this warp's ring
  float* ot = reinterpret_cast<float*>(my);  // [4][D] O rows | m [4] | l [4]
  __syncwarp();
  if (t < 2) {
#pragma unroll
    for (int d2 = 0; d2 < D / 16; ++d2) {
      const int d = 16 * d2 + g;
      ot[(2 * t) * D + d] = o[d2][0];
      ot[(2 * t + 1) * D + d] = o[d2][1];
      ot[(2 * t) * D + d + 8] = o[d2][2];
      ot[(2 * t + 1) * D + d + 8] = o[d2][3];
    }
    if (g == 0) {
      ot[4 * D + 2 * t] = mr[0];
      ot[4 * D + 2 * t + 1] = mr[1];
      ot[4 * D + 4 + 2 * t] = lr[0];
      ot[4 * D + 4 + 2 * t + 1] = lr[1];
    }
  }
  __syncwarp();
  float m[1][2], l[1][2], os[1][D / 8][4];
  const bool vrow = g < R;
  m[0][0] = vrow ? ot[4 * D + g] : -INFINITY;
  m[0][1] = -INFINITY;
  l[0][0] = (vrow && t == 0) ? ot[4 * D + 4 + g] : 0.0f;  // the epilogue sums l over t
  l[0][1] = 0.0f;
#pragma unroll
  for (int dt = 0; dt < D / 8; ++dt) {
    os[0][dt][0] = vrow ? ot[g * D + 8 * dt + 2 * t] : 0.0f;
    os[0][dt][1] = vrow ? ot[g * D + 8 * dt + 2 * t + 1] : 0.0f;
    os[0][dt][2] = 0.0f;
    os[0][dt][3] = 0.0f;
  }
  float* smem_f = reinterpret_cast<float*>(wbase);  // rings are dead now
  FinishTq4 fin{&a};
  attn_epilogue<D, 1>(a, m, l, os, smem_f, b, h, split, R, fin);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct SplitPlan {
  int splits, pps, rows_pad, lq_chunk, chunks;
};

static SplitPlan plan_split(int B, int Lq, int Hq, int Hkv, int max_seq_len, int min_pps = 4,
                            int target = kTargetCtas) {
  SplitPlan p;
  const int G = Hq / Hkv;
  // query tokens per launch so that G * chunk <= 32 rows
  p.lq_chunk = G >= 32 ? 1 : (32 / G < Lq ? 32 / G : Lq);
  p.chunks = (Lq + p.lq_chunk - 1) / p.lq_chunk;
  p.rows_pad = (G * p.lq_chunk <= 16) ? 16 : 32;
  const int max_pages = (max_seq_len + 15) / 16 > 0 ? (max_seq_len + 15) / 16 : 1;
  // as many splits as keep every CTA in one resident wave (two per SM): a partial
  // second wave costs more than longer splits (measured on B200, Qwen3-8B shapes at
  // ctx 2048: B=8 3.35 vs 3.72 ms per decode step, B=32 7.99 vs 8.44)
  int want = target / (B * Hkv);
  if (want < 1) want = 1;
  if (want > 128) want = 128;
  // at least min_pps pages (one per warp) per split (measured: capping the pages per
  // split to raise the CTA count for long contexts was slower on B200)
  int pps = (max_pages + want - 1) / want;
  if (pps < min_pps) pps = min_pps;
  // the final merge stages splits x rows weights in 3 * RP * D (>= 3 * 16 * 64) floats
  // of shared memory: keep splits * rows_pad <= 3072
  while ((max_pages + pps - 1) / pps * p.rows_pad > 3072) pps *= 2;
  p.pps = pps;
  p.splits = (max_pages + pps - 1) / pps;
  return p;
}

static size_t attn_ws_bytes(const SplitPlan& p, int B, int Hkv, int D) {
  if (p.splits == 1) return kCounterBytes;
  return kCounterBytes + (size_t)B * Hkv * p.splits * p.rows_pad * (D + 1) * sizeof(float);
}

static size_t smem_bf16(int D, int MT) {
  const size_t q = (size_t)16 * MT * D * 2;
  const size_t kv = (size_t)4 * 2 * 2 * 16 * D * 2;
  const size_t merge = (size_t)(9 * 16 * MT + 4 * 16 * MT * D) * 4;
  return q + (kv > merge ? kv : merge);
}

static size_t smem_tq4(int MT) {
  const size_t head = (size_t)MT * 8 * 32 * 8 * 4 + 16 * MT * 4;
  const size_t warps = (size_t)4 * (kTq4Stages * (1024 + 1024 + 32 + 32) + 2 * 16 * 128 * 2);
  const size_t qrot = (size_t)16 * MT * 128 * 4;
  const size_t merge = (size_t)(9 * 16 * MT + 4 * 16 * MT * 128) * 4;
  size_t body = warps + qrot;  // the query scratch follows the rings
  if (merge > body) body = merge;
  return head + body;
}

static size_t smem_tq4_swap(int S) {
  return (size_t)32 * 4 + (size_t)4 * 128 * 4 + (size_t)4 * (S * (1024 + 1024 + 32 + 32) + 2 * 16 * 128 * 2);
}

constexpr int kFusedStages = 3;
// pages per split of the fused kernel: two per warp by default, so the prefetch
// issued before the grid dependency wait covers a whole split (tunable through
// higgs_set_option("attn_min_pages", n), n >= 4; the workspace is sized for 4)
static int g_fused_min_pages = 8;
void attention_set_min_pages(int n) { g_fused_min_pages = n < 4 ? 4 : (n > 4096 ? 4096 : n); }
// largest thread-block cluster the fused kernel's splits may form (0 = no clusters): the splits
// of a (sequence, kv head) then merge through distributed shared memory instead of the
// workspace and an arrival counter, at up to twice the pages per split
static int g_attn_cluster = 16;
// TurboQuant attention: P x V with P's hi + lo bf16 halves (1) or its bf16 rounding only (0,
// the default: within the same tolerance of the oracle, C5 step 18.7 -> 17.2 ms on a B200)
static bool g_tq4_p_lo = false;
void attention_set_tq4_p_lo(int on) { g_tq4_p_lo = on != 0; }
// TurboQuant launches of at most 4 query rows: the swapped-role kernel with this many ring
// stages per warp (4 or 6), or 0 for the kernel with the query rows on the MMA's 16 rows
static int g_tq4_swap = 4;
void attention_set_tq4_swap(int n) { g_tq4_swap = n >= 6 ? 6 : (n >= 4 ? 4 : 0); }
void attention_set_cluster(int n) { g_attn_cluster = n >= 16 ? 16 : (n >= 8 ? 8 : (n >= 2 ? n : 0)); }

static size_t smem_fused(int D, int MT, int Lq) {
  const size_t q = (size_t)16 * MT * D * 2;
  const size_t nk = (size_t)((2 * Lq * D + 63) / 64) * 64 * 2;
  const size_t kv = (size_t)4 * kFusedStages * 2 * 16 * D * 2;
  const size_t merge = (size_t)(9 * 16 * MT + 4 * 16 * MT * D) * 4;
  return q + nk + (kv > merge ? kv : merge);
}

// Raise the dynamic shared-memory limit of every attention instantiation, once
// per device (the limit is a per-device setting), outside any stream capture.
static cudaError_t attention_prepare_device() {
  cudaError_t e = cudaSuccess;
  auto set = [&](void (*k)(AttnArgs), size_t smem) {
    cudaError_t r = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (r != cudaSuccess) e = r;
  };
  set(paged_attn_bf16_kernel<64, 1>, smem_bf16(64, 1));
  set(paged_attn_bf16_kernel<64, 2>, smem_bf16(64, 2));
  set(paged_attn_bf16_kernel<128, 1>, smem_bf16(128, 1));
  set(paged_attn_bf16_kernel<128, 2>, smem_bf16(128, 2));
  set(paged_attn_tq4_kernel<1>, smem_tq4(1));
  set(paged_attn_tq4_kernel<2>, smem_tq4(2));
  set(paged_attn_tq4_kernel<1, false>, smem_tq4(1));
  set(paged_attn_tq4_kernel<2, false>, smem_tq4(2));
  set(paged_attn_tq4_swap_kernel<4>, smem_tq4_swap(4));
  set(paged_attn_tq4_swap_kernel<6>, smem_tq4_swap(6));
  set(fused_attn_bf16_kernel<64, 1, kFusedStages>, smem_fused(64, 1, 32));
  set(fused_attn_bf16_kernel<64, 2, kFusedStages>, smem_fused(64, 2, 32));
  set(fused_attn_bf16_kernel<128, 1, kFusedStages>, smem_fused(128, 1, 32));
  set(fused_attn_bf16_kernel<128, 2, kFusedStages>, smem_fused(128, 2, 32));
  auto setc = [&](void (*k)(AttnArgs), size_t smem) {
    set(k, smem);
    const cudaError_t r = cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (r != cudaSuccess) e = r;
  };
  setc(fused_attn_bf16_kernel<64, 1, kFusedStages, true>, smem_fused(64, 1, 32));
  setc(fused_attn_bf16_kernel<64, 2, kFusedStages, true>, smem_fused(64, 2, 32));
  setc(fused_attn_bf16_kernel<128, 1, kFusedStages, true>, smem_fused(128, 1, 32));
  setc(fused_attn_bf16_kernel<128, 2, kFusedStages, true>, smem_fused(128, 2, 32));
  return e;
}

static PerDeviceOnce g_attn_prepared;

cudaError_t attention_prepare() { return g_attn_prepared.run(attention_prepare_device); }

template <typename K>
static cudaError_t launch_attn(K kernel, size_t smem, const AttnArgs& a, const SplitPlan& p,
                               cudaStream_t st) {
  cudaError_t e = attention_prepare();
  if (e != cudaSuccess) return e;
  for (int c = 0; c < p.chunks; ++c) {
    AttnArgs ac = a;
    ac.tq0 = c * p.lq_chunk;
    ac.lq_chunk = (a.Lq - ac.tq0) < p.lq_chunk ? (a.Lq - ac.tq0) : p.lq_chunk;
    e = launch_pdl(kernel, dim3(p.splits, a.Hkv, a.B), dim3(kAttnThreads), smem, st, ac);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace higgs

using namespace higgs;

extern "C" size_t higgs_paged_attention_workspace_size(int B, int Lq, int Hq, int Hkv, int D,
                                                       int max_seq_len) {
  if (B <= 0 || Lq <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv) return 0;
  // the larger of the two split plans (the TurboQuant swapped-role kernel keeps three CTAs
  // per SM resident), so one workspace serves either kernel
  const size_t a = attn_ws_bytes(plan_split(B, Lq, Hq, Hkv, max_seq_len), B, Hkv, D);
  const size_t b = attn_ws_bytes(plan_split(B, Lq, Hq, Hkv, max_seq_len, 4, kTargetCtasTq4), B, Hkv, D);
  return a > b ? a : b;
}

extern "C" size_t higgs_paged_attention_tq4_workspace_size(int B, int Lq, int Hq, int Hkv,
                                                           int max_seq_len) {
  return higgs_paged_attention_workspace_size(B, Lq, Hq, Hkv, 128, max_seq_len);
}

static int validate_attn(int B, int Lq, int Hq, int Hkv, int max_blocks, int max_seq_len,
                         size_t ws_bytes, size_t need, const void* ws) {
  HG_CHECK_ARG(((uintptr_t)ws & 15) == 0, "paged attention: workspace must be 16-byte aligned");
  HG_CHECK_ARG(B > 0 && Lq > 0 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0,
               "paged attention: bad batch / head shape");
  HG_CHECK_ARG(B * Hkv * 1 <= kCounterBytes / 4, "paged attention: B * Hkv exceeds 1024");
  HG_CHECK_ARG(max_seq_len >= Lq, "paged attention: max_seq_len < Lq");
  HG_CHECK_ARG((int64_t)max_blocks * 16 >= max_seq_len, "paged attention: block table too short");
  if (ws_bytes < need)
    return fail(HIGGS_ERR_WORKSPACE, "paged attention: workspace too small (need " +
                                         std::to_string(need) + " bytes)");
  return HIGGS_OK;
}

extern "C" int higgs_paged_attention(higgs_ctx* ctx, const void* q, int B, int Lq, int Hq, int Hkv,
                                     int D, const void* k_cache, const void* v_cache,
                                     int64_t page_stride, int64_t head_stride,
                                     const int32_t* block_table, int max_blocks,
                                     const int32_t* seq_lens, int max_seq_len, float scale,
                                     void* out, void* workspace, size_t workspace_bytes,
                                     void* stream) {
  HG_CHECK_ARG(ctx && q && k_cache && v_cache && block_table && seq_lens && out && workspace,
               "higgs_paged_attention: null argument");
  HG_CHECK_ARG(D == 64 || D == 128, "higgs_paged_attention: D must be 64 or 128");
  HG_DEVICE(ctx);
  const SplitPlan p = plan_split(B, Lq, Hq, Hkv, max_seq_len);
  int rc = validate_attn(B, Lq, Hq, Hkv, max_blocks, max_seq_len, workspace_bytes,
                         attn_ws_bytes(p, B, Hkv, D), workspace);
  if (rc) return rc;
  if (prefill_attn_tc_fits(Lq, Hq, Hkv, D, q, k_cache, v_cache, out, page_stride, head_stride)) {
    // prefill chunks: 128-row query tiles on the tensor cores, one launch, no workspace
    HG_CUDA(launch_prefill_attn_tc(q, B, Lq, Hq, Hkv, D, k_cache, v_cache, page_stride, head_stride,
                                   block_table, max_blocks, seq_lens, scale, out, (int*)workspace, tc_err_ptr(),
                                   (cudaStream_t)stream));
    return HIGGS_OK;
  }
  AttnArgs a = {};
  a.q = (const uint16_t*)q;
  a.B = B;
  a.Lq = Lq;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.kc = (const uint16_t*)k_cache;
  a.vc = (const uint16_t*)v_cache;
  a.page_stride = page_stride;
  a.head_stride = head_stride;
  a.bt = block_table;
  a.max_blocks = max_blocks;
  a.seq_lens = seq_lens;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.out = (uint16_t*)out;
  a.splits = p.splits;
  a.pages_per_split = p.pps;
  a.counters = (int*)workspace;
  a.ws_lse = (float*)((char*)workspace + kCounterBytes);
  a.ws_o = a.ws_lse + (size_t)B * Hkv * p.splits * p.rows_pad;
  cudaStream_t st = (cudaStream_t)stream;
  const int MT = p.rows_pad / 16;
  cudaError_t e;
  if (D == 64)
    e = MT == 1 ? launch_attn(paged_attn_bf16_kernel<64, 1>, smem_bf16(64, 1), a, p, st)
                : launch_attn(paged_attn_bf16_kernel<64, 2>, smem_bf16(64, 2), a, p, st);
  else
    e = MT == 1 ? launch_attn(paged_attn_bf16_kernel<128, 1>, smem_bf16(128, 1), a, p, st)
                : launch_attn(paged_attn_bf16_kernel<128, 2>, smem_bf16(128, 2), a, p, st);
  HG_CUDA(e);
  return HIGGS_OK;
}

extern "C" int higgs_paged_attention_tq4(higgs_ctx* ctx, const void* q, int B, int Lq, int Hq,
                                         int Hkv, const uint8_t* k_codes, const void* k_scales,
                                         const uint8_t* v_codes, const void* v_scales,
                                         int64_t page_stride, int64_t head_stride,
                                         const int32_t* block_table, int max_blocks,
                                         const int32_t* seq_lens, int max_seq_len,
                                         const int8_t* signs, float scale, void* out,
                                         void* workspace, size_t workspace_bytes, void* stream) {
  HG_CHECK_ARG(ctx && q && k_codes && k_scales && v_codes && v_scales && block_table && seq_lens &&
                   out && workspace && signs,
               "higgs_paged_attention_tq4: null argument");
  HG_CHECK_ARG(page_stride % 64 == 0 && head_stride % 64 == 0,
               "higgs_paged_attention_tq4: strides must be multiples of 64 bytes");
  HG_DEVICE(ctx);
  const SplitPlan p0 = plan_split(B, Lq, Hq, Hkv, max_seq_len);
  const bool swap = !g_tq4_p_lo && g_tq4_swap && (Hq / Hkv) * p0.lq_chunk <= 4;
  const SplitPlan p = swap ? plan_split(B, Lq, Hq, Hkv, max_seq_len, 4, kTargetCtasTq4) : p0;
  int rc = validate_attn(B, Lq, Hq, Hkv, max_blocks, max_seq_len, workspace_bytes,
                         attn_ws_bytes(p, B, Hkv, 128), workspace);
  if (rc) return rc;
  AttnArgs a = {};
  a.q = (const uint16_t*)q;
  a.B = B;
  a.Lq = Lq;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.kcode = k_codes;
  a.kscale = (const __half*)k_scales;
  a.vcode = v_codes;
  a.vscale = (const __half*)v_scales;
  a.signs = signs;
  a.page_stride = page_stride;
  a.head_stride = head_stride;
  a.bt = block_table;
  a.max_blocks = max_blocks;
  a.seq_lens = seq_lens;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.out = (uint16_t*)out;
  a.splits = p.splits;
  a.pages_per_split = p.pps;
  a.counters = (int*)workspace;
  a.ws_lse = (float*)((char*)workspace + kCounterBytes);
  a.ws_o = a.ws_lse + (size_t)B * Hkv * p.splits * p.rows_pad;
  cudaStream_t st = (cudaStream_t)stream;
  const int MT = p.rows_pad / 16;
  cudaError_t e;
  if (swap)
    e = g_tq4_swap == 6 ? launch_attn(paged_attn_tq4_swap_kernel<6>, smem_tq4_swap(6), a, p, st)
                        : launch_attn(paged_attn_tq4_swap_kernel<4>, smem_tq4_swap(4), a, p, st);
  else if (g_tq4_p_lo)
    e = MT == 1 ? launch_attn(paged_attn_tq4_kernel<1>, smem_tq4(1), a, p, st)
                : launch_attn(paged_attn_tq4_kernel<2>, smem_tq4(2), a, p, st);
  else
    e = MT == 1 ? launch_attn(paged_attn_tq4_kernel<1, false>, smem_tq4(1), a, p, st)
                : launch_attn(paged_attn_tq4_kernel<2, false>, smem_tq4(2), a, p, st);
  HG_CUDA(e);
  return HIGGS_OK;
}

extern "C" size_t higgs_fused_attention_workspace_size(int B, int Lq, int Hq, int Hkv, int D,
                                                       int max_seq_len) {
  if (B <= 0 || Lq <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv) return 0;
  return attn_ws_bytes(plan_split(B, Lq, Hq, Hkv, max_seq_len, g_fused_min_pages), B, Hkv, D);
}

namespace higgs {
int fused_attention_launch(higgs_ctx* ctx, const void* qkv, int B, int Lq, int Hq, int Hkv, int D,
                           const void* q_norm_w, const void* k_norm_w, float eps,
                           const int32_t* positions, const float* inv_freq,
                           const int64_t* slot_mapping, void* k_cache, void* v_cache,
                           int64_t page_stride, int64_t head_stride, const int32_t* block_table,
                           int max_blocks, const int32_t* seq_lens, int max_seq_len, float scale,
                           void* out, void* workspace, size_t workspace_bytes, void* stream,
                           const L2Prefetch* pf) {
  HG_CHECK_ARG(ctx && qkv && positions && inv_freq && k_cache && v_cache && block_table &&
                   seq_lens && out && workspace,
               "higgs_fused_attention: null argument");
  HG_CHECK_ARG(D == 64 || D == 128, "higgs_fused_attention: D must be 64 or 128");
  HG_CHECK_ARG((q_norm_w == nullptr) == (k_norm_w == nullptr),
               "higgs_fused_attention: give both q and k norm weights or neither");
  HG_CHECK_ARG(Hkv > 0 && Hq % Hkv == 0 && (Hq / Hkv) * Lq <= 32,
               "higgs_fused_attention: needs (Hq / Hkv) * Lq <= 32");
  HG_DEVICE(ctx);
  SplitPlan p = plan_split(B, Lq, Hq, Hkv, max_seq_len, g_fused_min_pages);
  int rc = validate_attn(B, Lq, Hq, Hkv, max_blocks, max_seq_len, workspace_bytes,
                         attn_ws_bytes(p, B, Hkv, D), workspace);
  if (rc) return rc;
  // cluster merge: the split count rounded up to a power of two (at most g_attn_cluster), the
  // pages spread over it, as long as a split gets at most twice the planned pages, for launches
  // of at most kClusterPairs (sequence, kv head) pairs (measured on B200: B=1 step 2.173 -> 2.147
  // ms; with 32 pairs it was slower: B=4 on one GPU 2.96 -> 3.72 ms, B=8 with 4 kv heads per
  // rank on two GPUs 2.85 -> 3.65 ms)
  constexpr int kClusterPairs = 8;
  int cluster = 0;
  if (g_attn_cluster >= 2 && p.splits > 1 && B * Hkv <= kClusterPairs) {
    int c = 2;
    while (c < p.splits && c < g_attn_cluster) c *= 2;
    const int max_pages = (max_seq_len + 15) / 16;
    const int pps = (max_pages + c - 1) / c;
    if (pps <= 2 * p.pps) {
      p.splits = c;
      p.pps = pps;
      cluster = c;
    }
  }
  AttnArgs a = {};
  a.B = B;
  a.Lq = Lq;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.lq_chunk = Lq;
  a.kc = (const uint16_t*)k_cache;
  a.vc = (const uint16_t*)v_cache;
  a.kc_w = (uint16_t*)k_cache;
  a.vc_w = (uint16_t*)v_cache;
  a.page_stride = page_stride;
  a.head_stride = head_stride;
  a.bt = block_table;
  a.max_blocks = max_blocks;
  a.seq_lens = seq_lens;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.out = (uint16_t*)out;
  a.splits = p.splits;
  a.pages_per_split = p.pps;
  a.counters = (int*)workspace;
  a.ws_lse = (float*)((char*)workspace + kCounterBytes);
  a.ws_o = a.ws_lse + (size_t)B * Hkv * p.splits * p.rows_pad;
  a.qkv = (const uint16_t*)qkv;
  a.qn = (const uint16_t*)q_norm_w;
  a.kn = (const uint16_t*)k_norm_w;
  a.eps = eps;
  a.pos = positions;
  a.inv_freq = inv_freq;
  a.slots = slot_mapping;
  if (pf) a.pf = *pf;
  HG_CUDA(attention_prepare());
  const int MT = p.rows_pad / 16;
  const size_t smem = smem_fused(D, MT, Lq);
  cudaStream_t st = (cudaStream_t)stream;
  const dim3 grid(p.splits, Hkv, B);
  const dim3 blk(kAttnThreads);
  cudaError_t e;
  if (cluster) {
    if (D == 64)
      e = MT == 1 ? launch_pdl_cluster(fused_attn_bf16_kernel<64, 1, kFusedStages, true>, grid, blk, smem, st, cluster, a)
                  : launch_pdl_cluster(fused_attn_bf16_kernel<64, 2, kFusedStages, true>, grid, blk, smem, st, cluster, a);
    else
      e = MT == 1 ? launch_pdl_cluster(fused_attn_bf16_kernel<128, 1, kFusedStages, true>, grid, blk, smem, st, cluster, a)
                  : launch_pdl_cluster(fused_attn_bf16_kernel<128, 2, kFusedStages, true>, grid, blk, smem, st, cluster, a);
  } else if (D == 64) {
    e = MT == 1 ? launch_pdl(fused_attn_bf16_kernel<64, 1, kFusedStages>, grid, blk, smem, st, a)
                : launch_pdl(fused_attn_bf16_kernel<64, 2, kFusedStages>, grid, blk, smem, st, a);
  } else {
    e = MT == 1 ? launch_pdl(fused_attn_bf16_kernel<128, 1, kFusedStages>, grid, blk, smem, st, a)
                : launch_pdl(fused_attn_bf16_kernel<128, 2, kFusedStages>, grid, blk, smem, st, a);
  }
  HG_CUDA(e);
  return HIGGS_OK;
}
}  // namespace higgs

extern "C" int higgs_fused_attention(higgs_ctx* ctx, const void* qkv, int B, int Lq, int Hq,
                                     int Hkv, int D, const void* q_norm_w, const void* k_norm_w,
                                     float eps, const int32_t* positions, const float* inv_freq,
                                     const int64_t* slot_mapping, void* k_cache, void* v_cache,
                                     int64_t page_stride, int64_t head_stride,
                                     const int32_t* block_table, int max_blocks,
                                     const int32_t* seq_lens, int max_seq_len, float scale,
                                     void* out, void* workspace, size_t workspace_bytes,
                                     void* stream) {
  return fused_attention_launch(ctx, qkv, B, Lq, Hq, Hkv, D, q_norm_w, k_norm_w, eps, positions,
                                inv_freq, slot_mapping, k_cache, v_cache, page_stride, head_stride,
                                block_table, max_blocks, seq_lens, max_seq_len, scale, out, workspace,
                                workspace_bytes, stream, nullptr);
}

// ---------------------------------------------------------------------------
// Allocation-free variant of higgs_paged_attention.
//
// Some callers cannot allocate device memory at all on their serving path:
// hosts that hand this library a fixed device-memory arena sized at start-up
// and account for every byte themselves, or real-time decode loops that must
// never block in the driver's allocator.  They cannot provide the split-K
// workspace that higgs_paged_attention takes.  This entry point keeps that
// scratch in a file-scope device array instead: kNoAllocScratchBytes on every
// GPU that loads the library, for the life of the process.
//
// The array's host-side name is only a stand-in for the device symbol, so its
// device address is looked up once per device with cudaGetSymbolAddress, with
// that device current, on the first call made on that device.
// ---------------------------------------------------------------------------
namespace higgs {

constexpr size_t kNoAllocScratchBytes = 8u << 20;  // 8 MiB
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

static void* noalloc_scratch_ptr(int device, cudaError_t* err) {
  static std::mutex mu;
  static void* ptrs[128] = {};
  std::lock_guard<std::mutex> lock(mu);
  *err = cudaSuccess;
  if (device < 0 || device >= 128) {
    *err = cudaErrorInvalidDevice;
    return nullptr;
  }
  if (!ptrs[device]) {
    void* p = nullptr;
    *err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (*err != cudaSuccess) return nullptr;
    ptrs[device] = p;
  }
  return ptrs[device];
}

}  // namespace higgs

extern "C" int higgs_paged_attention_noalloc(higgs_ctx* ctx, const void* q, int B, int Lq, int Hq,
                                             int Hkv, int D, const void* k_cache,
                                             const void* v_cache, int64_t page_stride,
                                             int64_t head_stride, const int32_t* block_table,
                                             int max_blocks, const int32_t* seq_lens,
                                             int max_seq_len, float scale, void* out,
                                             void* stream) {
  HG_CHECK_ARG(ctx && q && k_cache && v_cache && block_table && seq_lens && out,
               "higgs_paged_attention_noalloc: null argument");
  HG_CHECK_ARG(D == 64 || D == 128, "higgs_paged_attention_noalloc: D must be 64 or 128");
  HG_CHECK_ARG(B > 0 && Lq > 0 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0,
               "higgs_paged_attention_noalloc: bad batch / head shape");
  HG_DEVICE(ctx);
  const size_t need = attn_ws_bytes(plan_split(B, Lq, Hq, Hkv, max_seq_len), B, Hkv, D);
  if (need > kNoAllocScratchBytes)
    return fail(HIGGS_ERR_WORKSPACE,
                "higgs_paged_attention_noalloc: this shape needs " + std::to_string(need) +
                    " bytes of scratch, more than the built-in " +
                    std::to_string(kNoAllocScratchBytes) +
                    " bytes; use higgs_paged_attention with a caller-provided workspace");
  cudaError_t err;
  void* scratch = noalloc_scratch_ptr(ctx->device, &err);
  if (!scratch) return cuda_fail(err, "cudaGetSymbolAddress(g_noalloc_scratch)");
  // the split counters must start at zero whatever an earlier call left behind
  HG_CUDA(cudaMemsetAsync(scratch, 0, kCounterBytes, (cudaStream_t)stream));
  return higgs_paged_attention(ctx, q, B, Lq, Hq, Hkv, D, k_cache, v_cache, page_stride,
                               head_stride, block_table, max_blocks, seq_lens, max_seq_len, scale,
                               out, scratch, kNoAllocScratchBytes, stream);
}

HG_TL_FETCH_FN(higgs_timeline_fetch_attn)
