// qgemv_m1.cu -- W4 g64 GEMV for a single token (decode at batch 1): packed
// weights loaded straight into registers, the quantization groups carried in
// the MMA's output columns.
//
// Reference op replaced: ops::quantized_matmul (qwen3_next.rs:174-183) at one
// token, with the preceding nn::RmsNorm (transformer.rs:407, 415) optionally fused.
//
// One token leaves seven of the eight MMA columns of m16n8k16 idle; this kernel
// uses them to keep groups apart instead.  A warp owns 16 rows (fragment rows g
// and g+8) and a K range in units of 256 (4 groups of 64).  Per unit and row,
// the four quad lanes t load 64 contiguous bytes twice (LDG.128 at bytes
// 64h + 16t, h = 0, 1), so in the MMAs of half h lanes t = 0, 1 carry group 2h
// and lanes 2, 3 group 2h + 1.  The B operand routes group j of an even unit
// into output column j and of an odd unit into column 4 + j (the B fragment of
// column c is zero except in the two lanes (c, t) whose data is group c % 4), so
// the 32 MMAs of a unit pair build the 8 (row x group) dot products of each row
// pair in one accumulator, and the per-group fold
//     y += s * acc + (b - 128 s) * sum(x)
// runs once per unit pair over fully used accumulators.  Weights enter the MMA
// as the exact bf16 values 128 + q (one shift and one LOP3 per pair of codes);
// x enters as bf16 itself, so staging it is a permutation (plus the fused
// RMSNorm): one pass, no scaling.  Per unit a warp issues 4 LDG.128, 112 ALU
// unpack ops, 16 mma.sync and 8 LDS.128 (x fragments; lanes whose column is
// unused read a zero block); the next D units of weights stay in flight in
// registers, and the first D are requested before the kernel waits on its
// predecessor.  Before the wait each CTA also asks L2 for every weight byte it
// will stream (cp.async.bulk.prefetch), so HBM streams the CTA's whole slice from
// its start while the register ring reads L2.  CTAs walk tile groups round-robin
// (one group each by default; optionally a grid capped at the resident slots).
#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "kernels.cuh"
#include "timeline.cuh"

namespace higgs {

namespace {

constexpr int kM1Threads = 256;
constexpr int kM1CtasPerSm = 2;  // register bound: 128 registers a thread
constexpr int kM1MaxK = 32768;  // staged x: K / 256 * 512 B + sums + 1 KB
constexpr int kM1RegChunks = 4;   // fused norm: x chunks held in registers between the passes (K <= 8192)
constexpr int kM1NormChunks = 2;  // fused norm: norm-weight chunks loaded before the wait (K <= 4096)

struct M1Seg {
  const uint32_t* W;
  const uint16_t* S;
  const uint16_t* B;
  int row0;
};

// D = A(16x16 bf16, row) * B(16x8 bf16, col) + D (f32); no side effects, so the
// compiler may schedule it freely among the unpack ops
__device__ __forceinline__ void m1_mma(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                       uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// weights: L1-allocating loads, so lines pulled in by m1_prefetch_l1 are hit there
__device__ __forceinline__ uint4 m1_ldg128(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ void m1_prefetch_l1(const void* p) {
  asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}

__device__ __forceinline__ uint4 m1_lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

__host__ __device__ inline size_t m1_xf_bytes(int K) { return (size_t)(K / 256) * 512; }
// x fragments | 64 pad | 512 B of zeros (at 64 mod 128) | 64 pad | sum(x) per group | reduction [8][16]
inline size_t m1_smem_bytes(int K) { return m1_xf_bytes(K) + 640 + (size_t)(K / 64) * 4 + 8 * 16 * 4; }

// B fragments of chunk x[8c .. 8c+7]: (x0, x4) (x1, x5) (x2, x6) (x3, x7), the pairs the
// A side forms from one word of codes (nibbles i and i + 4 of each word)
__device__ __forceinline__ uint4 m1_frag(uint4 v) {
  return make_uint4(prmt(v.x, v.z, 0x5410), prmt(v.x, v.z, 0x7632), prmt(v.y, v.w, 0x5410),
                    prmt(v.y, v.w, 0x7632));
}

__device__ __forceinline__ unsigned m1_ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void m1_st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned* m1_tp_flag(const TpFuse& tp, int q, int src, int word) {
  return reinterpret_cast<unsigned*>(tp.peer[q]) + ((size_t)tp.call * tp.world + src) * tp.max_ctas + word;
}

// Chunk c (8 elements) of the GEMV input: x itself, or (tensor-parallel pull) the residual
// stream plus the ranks' pushed partials, h + bf16(sum_q partial_q) with the ranks in order --
// the all-reduce kernel's formula, so the same bits.  CTA 0 stores the new residual stream.
template <bool PULL>
__device__ __forceinline__ uint4 m1_x_chunk(const QLinArgs& a, int c) {
  if constexpr (!PULL) return *reinterpret_cast<const uint4*>(a.x + 8 * c);
  const TpFuse& tp = a.tp;
  const uint4 hv = *reinterpret_cast<const uint4*>(tp.h_in + 8 * c);
  const float* mine = reinterpret_cast<const float*>(tp.peer[tp.rank] + tp.flag_bytes) +
                      (size_t)tp.call * tp.world * tp.words + 8 * (size_t)c;
  float y[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int q = 0; q < tp.world; ++q) {
    const float4 p0 = __ldcg(reinterpret_cast<const float4*>(mine + (size_t)q * tp.words));
    const float4 p1 = __ldcg(reinterpret_cast<const float4*>(mine + (size_t)q * tp.words + 4));
    y[0] += p0.x, y[1] += p0.y, y[2] += p0.z, y[3] += p0.w;
    y[4] += p1.x, y[5] += p1.y, y[6] += p1.z, y[7] += p1.w;
  }
  const uint32_t* hp = &hv.x;
  uint4 out;
  uint32_t* op = &out.x;
#pragma unroll
  for (int j = 0; j < 4; ++j)
    op[j] = pack_bf2(bf_lo(hp[j]) + round_bf(y[2 * j]), bf_hi(hp[j]) + round_bf(y[2 * j + 1]));
  return out;
}

// WK warps split the K range of each 16-row tile; RT = 8 / WK tiles per CTA (SwiGLU: RT / 2
// gate/up pairs).  D units of weights in flight per warp (even).
template <int WK, int EPI, bool NORM, int D, bool PULL = false>
__global__ void __launch_bounds__(kM1Threads, kM1CtasPerSm) qgemv_m1_kernel(QLinArgs a) {
  static_assert(!PULL || NORM, "the tensor-parallel pull feeds a fused-norm GEMV");
  static_assert(D % 2 == 0, "units are folded in pairs");
  constexpr int RT = 8 / WK;
  constexpr int ROT = (EPI == EPI_SWIGLU) ? RT / 2 : RT;
  extern __shared__ __align__(128) uint8_t smem[];
  HG_TL_MARK(0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int rt = warp / WK, kw = warp % WK;
  const int K = a.K, N = a.N, KW = K / 8, G = K / 64;
  const int units = K / 256;

  uint8_t* xf = smem;
  uint8_t* zero = smem + m1_xf_bytes(K) + 64;
  float* xs = reinterpret_cast<float*>(zero + 576);  // sum(x) per group
  float* red = xs + G;                               // [8 warps][16 rows]

  // tile groups (ROT output tiles each) are dealt round-robin to the resident CTAs
  const int n_groups = (N / 16 + ROT - 1) / ROT;
  // this warp's 16-row tile of group grp and its K range [ub, ue) (empty past N)
  struct Tile {
    M1Seg sg;
    int ub, ue;
  };
  auto tile_of = [&](int grp) {
    Tile tl;
    int out_tile, which = 0;
    if (EPI == EPI_SWIGLU) {
      out_tile = grp * ROT + rt / 2;
      which = rt & 1;
    } else {
      out_tile = grp * ROT + rt;
    }
    const int n0 = out_tile * 16;
    const bool ok = n0 < N;
    tl.sg.W = which ? a.w2 : a.w;
    tl.sg.S = which ? a.s2 : a.s;
    tl.sg.B = which ? a.b2 : a.b;
    tl.sg.row0 = ok ? n0 : 0;
    if (EPI != EPI_SWIGLU && a.nseg > 1) {
#pragma unroll
      for (int i = 1; i < 3; ++i)
        if (i < a.nseg && ok && n0 >= a.seg_end[i - 1]) {
          tl.sg.W = a.wseg[i];
          tl.sg.S = a.sseg[i];
          tl.sg.B = a.bseg[i];
          tl.sg.row0 = n0 - a.seg_end[i - 1];
        }
    }
    tl.ub = ok ? (units * kw) / WK : 0;
    tl.ue = ok ? (units * (kw + 1)) / WK : 0;
    return tl;
  };

  issue_l2_prefetch(a.pf, blockIdx.x, gridDim.x);
  if (a.self_prefetch && kw == 0 && lane < 3) {
    // every tile this CTA will stream -> L2 now, one contiguous request per tile (its 16
    // rows are adjacent: 16 x K/2 bytes; lanes 1, 2 take the scales and biases), so the
    // register ring below (D units deep) reads L2 instead of waiting on HBM round trips
    for (int grp = blockIdx.x; grp < n_groups; grp += gridDim.x) {
      const Tile tl = tile_of(grp);
      if (tl.ub >= tl.ue) continue;
      if (lane == 0)
        l2_prefetch_range(tl.sg.W + (size_t)tl.sg.row0 * KW, (size_t)16 * KW * 4);
      else
        l2_prefetch_range((lane == 1 ? tl.sg.S : tl.sg.B) + (size_t)tl.sg.row0 * G, (size_t)16 * G * 2);
    }
  }

  // lane (g, t): rows g and g+8; per unit the 16-byte chunks t and 4 + t of the row's 128 B;
  // scales / biases of groups (4 u0 + 2t, +1) of a unit pair starting at u0, as bf16 pairs
  const uint4 *wg, *w8;
  const uint32_t *sgp, *sg8, *bgp, *bg8;
  int ub, ue;
  auto bind = [&](const Tile& tl) {
    ub = tl.ub;
    ue = tl.ue;
    wg = reinterpret_cast<const uint4*>(tl.sg.W + (size_t)(tl.sg.row0 + g) * KW) + t;
    w8 = wg + (size_t)2 * KW;  // 8 rows further (K / 32 uint4 per row)
    sgp = reinterpret_cast<const uint32_t*>(tl.sg.S + (size_t)(tl.sg.row0 + g) * G) + t;
    sg8 = sgp + (size_t)4 * G;  // (8 rows * G bf16) / 2
    bgp = reinterpret_cast<const uint32_t*>(tl.sg.B + (size_t)(tl.sg.row0 + g) * G) + t;
    bg8 = bgp + (size_t)4 * G;
  };

  uint4 buf[D][4];
  uint32_t sb[D / 2][4];
  auto load_unit = [&](uint4 (&b)[4], int u) {
    b[0] = m1_ldg128(wg + 8 * u);
    b[1] = m1_ldg128(wg + 8 * u + 4);
    b[2] = m1_ldg128(w8 + 8 * u);
    b[3] = m1_ldg128(w8 + 8 * u + 4);
  };
  auto load_scales = [&](uint32_t (&q)[4], int u0) {
    // this lane folds unit u0 + t/2; past the range it folds nothing (scales 0)
    const bool ok = u0 + (t >> 1) < ue;
    q[0] = ok ? __ldg(sgp + 2 * u0) : 0u;
    q[1] = ok ? __ldg(sg8 + 2 * u0) : 0u;
    q[2] = ok ? __ldg(bgp + 2 * u0) : 0u;
    q[3] = ok ? __ldg(bg8 + 2 * u0) : 0u;
  };
  auto prologue = [&]() {
#pragma unroll
    for (int d = 0; d < D; ++d) {
      if (ub + d < ue) load_unit(buf[d], ub + d);
      if ((d & 1) == 0) load_scales(sb[d / 2], ub + d);
    }
  };

  // the first group's first D units and scales, and the norm weights of this thread's
  // first chunks: none of them depends on the previous kernel
  bind(tile_of(blockIdx.x));
  prologue();
  uint4 nwr[NORM ? kM1NormChunks : 1];
  if constexpr (NORM) {
#pragma unroll
    for (int r = 0; r < kM1NormChunks; ++r) {
      const int c = threadIdx.x + r * kM1Threads;
      nwr[r] = c < K / 8 ? *reinterpret_cast<const uint4*>(a.norm_w + 8 * c) : make_uint4(0, 0, 0, 0);
    }
  }
  pdl_wait();
  HG_TL_MARK(1);
  pdl_launch();
  if constexpr (PULL) {
    // every rank's partial of this call must have landed here (bounded wait, ~1 s)
    if (threadIdx.x < a.tp.world) {
      const unsigned s = *a.tp.step;
      const unsigned* f = m1_tp_flag(a.tp, a.tp.rank, threadIdx.x, kTpFlagWord);
      const long long t0 = clock64();
      while (m1_ld_acquire_sys(f) != s) {
        if (clock64() - t0 > (1ll << 31)) {
          atomicExch(a.tp.err, 1);
          break;
        }
        __nanosleep(32);
      }
    }
    __syncthreads();
  }

  if (threadIdx.x < 32) reinterpret_cast<uint4*>(zero)[threadIdx.x] = make_uint4(0, 0, 0, 0);
  const uint16_t* x = a.x;
  // ---- fused RMSNorm: the token's sum of squares (its chunks kept for the staging) ----
  // (measured on B200: every warp summing the whole token itself, to drop the barrier below,
  // lengthened the B=1 decode step 2.15 -> 2.39 ms: 16 dependent L2 loads per lane)
  __shared__ float s_ss[8];
  uint4 xr[NORM ? kM1RegChunks : 1];
  float inv = 1.0f;
  if constexpr (NORM) {
    float ss = 0.f;
#pragma unroll
    for (int r = 0; r < kM1RegChunks; ++r) xr[r] = make_uint4(0, 0, 0, 0);
    for (int c = threadIdx.x, r = 0; c < K / 8; c += kM1Threads, ++r) {
      const uint4 v = m1_x_chunk<PULL>(a, c);
      if (PULL && blockIdx.x == 0) *reinterpret_cast<uint4*>(a.tp.h_out + 8 * c) = v;
#pragma unroll
      for (int j = 0; j < kM1RegChunks; ++j)
        if (j == r) xr[j] = v;
      const uint32_t* vp = &v.x;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float lo = bf_lo(vp[j]), hi = bf_hi(vp[j]);
        ss += lo * lo + hi * hi;
      }
    }
    ss = warp_sum(ss);
    if (lane == 0) s_ss[warp] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) tot += s_ss[w];
    inv = 1.0f / sqrtf(tot / (float)K + a.eps);
  }

  // ---- x fragments: chunk c = 32u + 16h + 4t + e (x[8c .. 8c+7]) at
  // xf + ((u * 8 + h * 4 + e) * 4 + t) * 16; sum(x) per group (8 consecutive chunks).
  // Whole warps iterate (K / 8 is a multiple of 32).
  for (int base = warp * 32, r = 0; base < K / 8; base += kM1Threads, ++r) {
    const int c = base + lane;
    uint4 v;
    if constexpr (NORM) {
      v = xr[0];
#pragma unroll
      for (int j = 1; j < kM1RegChunks; ++j)
        if (j == r) v = xr[j];
      if (r >= kM1RegChunks) v = m1_x_chunk<PULL>(a, c);
      uint4 wv = nwr[0];
#pragma unroll
      for (int j = 1; j < kM1NormChunks; ++j)
        if (j == r) wv = nwr[j];
      if (r >= kM1NormChunks) wv = *reinterpret_cast<const uint4*>(a.norm_w + 8 * c);
      uint32_t* vp = &v.x;
      const uint32_t* wp = &wv.x;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        vp[j] = pack_bf2(bf_lo(vp[j]) * inv * bf_lo(wp[j]), bf_hi(vp[j]) * inv * bf_hi(wp[j]));
    } else {
      v = *reinterpret_cast<const uint4*>(x + 8 * c);
    }
    const int u = c >> 5, h = (c >> 4) & 1, tt = (c >> 2) & 3, e = c & 3;
    *reinterpret_cast<uint4*>(xf + ((u * 8 + h * 4 + e) * 4 + tt) * 16) = m1_frag(v);
    const uint32_t* vp = &v.x;
    float x1 = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) x1 += bf_lo(vp[j]) + bf_hi(vp[j]);
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) x1 += __shfl_xor_sync(0xffffffffu, x1, o);
    if ((lane & 7) == 0) xs[c >> 3] = x1;
  }
  __syncthreads();

  // lane (g, t) supplies B column g: in half h of a unit of parity p it carries data iff
  // g == 4p + 2h + t/2, else it reads the zero block
  const uint32_t xreal = smem_u32(xf) + t * 16;
  const uint32_t xzero = smem_u32(zero);
  const float2* xs2 = reinterpret_cast<const float2*>(xs);
  const int l1d = a.m1_l1_ahead;

  for (int grp = blockIdx.x; grp < n_groups; grp += gridDim.x) {
    if (grp != (int)blockIdx.x) {
      bind(tile_of(grp));
      prologue();
    }
    float acc[2][4];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[h][c] = 0.f;
    float yg = 0.f, yg8 = 0.f;

    // ---- main loop over this warp's units ----
    for (int base = ub; base < ue; base += D) {
#pragma unroll
      for (int d = 0; d < D; ++d) {
        const int u = base + d;
        if (u >= ue) break;  // uniform over the warp
        const int p = d & 1;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const bool act = g == 4 * p + 2 * h + (t >> 1);
          const uint32_t xb = (act ? xreal + u * 512 : xzero) + h * 256;
          uint4 xv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) xv[e] = m1_lds128(xb + e * 64);
          const uint32_t* wa = &buf[d][h].x;
          const uint32_t* wb = &buf[d][2 + h].x;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const uint32_t A = wa[e], B = wb[e];
            m1_mma(acc[h], nib_pair_bf16<0>(A), nib_pair_bf16<0>(B), nib_pair_bf16<4>(A),
                   nib_pair_bf16<4>(B), xv[e].x, xv[e].y);
            m1_mma(acc[h], nib_pair_bf16<8>(A), nib_pair_bf16<8>(B), nib_pair_bf16<12>(A),
                   nib_pair_bf16<12>(B), xv[e].z, xv[e].w);
          }
        }
        // buffer d is consumed: request unit u + D into it, and unit u + D + l1d into L1
        // (lane t == 0 of each row pair: the rows' 128-byte lines)
        if (u + D < ue) load_unit(buf[d], u + D);
        if (l1d > 0 && t == 0 && u + D + l1d < ue) {
          m1_prefetch_l1(wg + 8 * (u + D + l1d));
          m1_prefetch_l1(w8 + 8 * (u + D + l1d));
        }
        if (p == 1 || u + 1 == ue) {
          // fold the pair (u0, u0 + 1): lane t holds columns 2t, 2t+1 = groups 4 u0 + 2t, +1;
          // the MMA saw 128 + q, so y += s * acc + (b - 128 s) * sum(x)
          const int u0 = u - p;
          const bool ok = u0 + (t >> 1) < ue;
          const float2 X = xs2[ok ? 2 * u0 + t : 0];
          const uint32_t* q = sb[d / 2];
          const float sa = bf_lo(q[0]), sb_ = bf_hi(q[0]), s8a = bf_lo(q[1]), s8b = bf_hi(q[1]);
          const float ba = fmaf(-128.0f, sa, bf_lo(q[2])), bb = fmaf(-128.0f, sb_, bf_hi(q[2]));
          const float b8a = fmaf(-128.0f, s8a, bf_lo(q[3])), b8b = fmaf(-128.0f, s8b, bf_hi(q[3]));
          yg = fmaf(sa, acc[0][0] + acc[1][0], fmaf(ba, X.x, yg));
          yg = fmaf(sb_, acc[0][1] + acc[1][1], fmaf(bb, X.y, yg));
          yg8 = fmaf(s8a, acc[0][2] + acc[1][2], fmaf(b8a, X.x, yg8));
          yg8 = fmaf(s8b, acc[0][3] + acc[1][3], fmaf(b8b, X.y, yg8));
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[h][c] = 0.f;
          if (u0 + D < ue) load_scales(sb[d / 2], u0 + D);
        }
      }
    }

    // ---- reduction over the quad, then over the K-split warps ----
    yg += __shfl_xor_sync(0xffffffffu, yg, 1);
    yg += __shfl_xor_sync(0xffffffffu, yg, 2);
    yg8 += __shfl_xor_sync(0xffffffffu, yg8, 1);
    yg8 += __shfl_xor_sync(0xffffffffu, yg8, 2);
    if (t == 0) {
      red[warp * 16 + g] = yg;
      red[warp * 16 + g + 8] = yg8;
    }
    __syncthreads();
    if ((int)threadIdx.x < ROT * 16) {
      const int r = threadIdx.x >> 4, j = threadIdx.x & 15;
      const int tile = grp * ROT + r;
      const int row = tile * 16 + j;
      if (tile * 16 < N) {
        if (EPI == EPI_SWIGLU) {
          float vg = 0.f, vu = 0.f;
#pragma unroll
          for (int w = 0; w < WK; ++w) {
            vg += red[((2 * r) * WK + w) * 16 + j];
            vu += red[((2 * r + 1) * WK + w) * 16 + j];
          }
          const float gv = round_bf(vg), uv = round_bf(vu);
          a.y[row] = f2bf(gv / (1.0f + expf(-gv)) * uv);
        } else {
          float v = 0.f;
#pragma unroll
          for (int w = 0; w < WK; ++w) v += red[(r * WK + w) * 16 + j];
          if (a.y_f32) a.y_f32[row] = v;
          if (a.y) {
            uint16_t o = f2bf(v);
            if (a.residual) o = f2bf(bf2f(o) + bf2f(a.residual[row]));
            a.y[row] = o;
          }
          if (a.tp_push) {  // this row of the partial into slot (call, rank) of every rank
            for (int q = 0; q < a.tp.world; ++q)
              reinterpret_cast<float*>(a.tp.peer[q] + a.tp.flag_bytes)
                  [((size_t)a.tp.call * a.tp.world + a.tp.rank) * a.tp.words + row] = v;
          }
        }
      }
    }
    __syncthreads();  // red is rewritten by the next group
  }
  if (a.tp_push && threadIdx.x == 0) {
    // the CTA that completes this rank's count publishes "rank pushed call" on every rank
    __threadfence_system();
    unsigned* cnt = m1_tp_flag(a.tp, a.tp.rank, a.tp.rank, kTpCountWord);
    if (atomicAdd(cnt, 1u) == gridDim.x - 1) {
      *cnt = 0u;
      __threadfence_system();
      const unsigned s = *a.tp.step;
      for (int q = 0; q < a.tp.world; ++q) m1_st_release_sys(m1_tp_flag(a.tp, q, a.tp.rank, kTpFlagWord), s);
    }
  }
  HG_TL_END(1000 + EPI * 100 + NORM * 10 + WK);
}

// ---------------------------------------------------------------------------
// Decode chain: the GEMVs between two attention launches of a one-token decode
// step -- o_proj (+ residual), RMSNorm + gate/up + SwiGLU, down (+ residual),
// RMSNorm + the next layer's q|k|v (or the final norm + LM head) -- as the
// phases of one persistent launch of kChainCtasPerSm CTAs per SM.  Each phase
// is the single-token GEMV above with its K split, tiles and summation order
// (so its outputs equal the separate launches' bit for bit); phases are
// separated by grid barriers (an arrival counter per phase, bounded waits).
// What the separate launches cannot do: a CTA issues the next phase's weight
// loads into its registers, and (l2_ahead) asks L2 for its next slice, before
// it waits at the barrier, so HBM keeps streaming weights through the
// dependency points instead of idling between launches.
// ---------------------------------------------------------------------------
struct ChainArgs {
  ChainPhase ph[kChainMaxPhases];
  int nph;
  float eps;
  unsigned* bar;  // kChainBarWords per phase, zero at launch and zeroed again by the launch
  int* err;       // set when a barrier wait gives up
  int l2_ahead;   // 1: a phase's L2 requests are issued while the previous phase runs
};

// Barrier of one phase, 64 words: arrival counters of CTA groups (kChainGroup CTAs each), the
// count of finished groups, and the release flag the waiting CTAs poll (its own 128 bytes,
// apart from the counters the arrivals update).  The last CTA of a group adds its group to
// the top count; the last group raises the release flag.  Counters are reset by the CTAs that
// finish them; release flags by the last CTA of the launch.
constexpr int kChainGroup = 16;
constexpr int kChainTop = 32;      // word of the finished-group count
constexpr int kChainRelease = 48;  // word of the release flag

__device__ __forceinline__ unsigned chain_ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void chain_st_release(unsigned* p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// This CTA's arrival at barrier b (after every thread's writes of the phase); true in thread
// 0 of the CTA that completed the barrier.
__device__ __forceinline__ bool chain_arrive(unsigned* b) {
  __syncthreads();
  bool last = false;
  if (threadIdx.x == 0) {
    const unsigned nct = gridDim.x;
    const unsigned gi = blockIdx.x / kChainGroup;
    const unsigned ng = (nct + kChainGroup - 1) / kChainGroup;
    const unsigned gsize = min((unsigned)kChainGroup, nct - gi * kChainGroup);
    __threadfence();
    if (atomicAdd(b + gi, 1u) == gsize - 1) {
      b[gi] = 0u;  // every CTA of the group has arrived
      __threadfence();
      if (atomicAdd(b + kChainTop, 1u) == ng - 1) {
        b[kChainTop] = 0u;
        chain_st_release(b + kChainRelease, 1u);
        last = true;
      }
    }
  }
  return last;
}

// Wait for barrier b's release; gives up (and sets *err) after ~2^24 polls.
__device__ __forceinline__ void chain_wait(const unsigned* b, int* err) {
  if (threadIdx.x == 0) {
    unsigned it = 0;
    while (chain_ld_acquire(b + kChainRelease) == 0u) {
      if (++it > (1u << 24)) {
        if (err) atomicExch(err, 1);
        break;
      }
      __nanosleep(20);
    }
  }
  __syncthreads();
}

template <int D>
__global__ void __launch_bounds__(kM1Threads, kM1CtasPerSm) chain_kernel(const __grid_constant__ ChainArgs a) {
  static_assert(D % 2 == 0, "units are folded in pairs");
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float s_ss[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;

  struct Tile {
    const uint32_t* W;
    const uint16_t* S;
    const uint16_t* B;
    int row0, ub, ue;
  };
  // warp's tile of group grp in phase P (same mapping as qgemv_m1_kernel)
  auto tile_of = [&](const ChainPhase& P, int grp) {
    const int WK = P.wk, RT = 8 / WK, ROT = P.swiglu ? RT / 2 : RT;
    const int rt = warp / WK, kw = warp % WK;
    const int units = P.K / 256;
    Tile tl;
    int out_tile, which = 0;
    if (P.swiglu) {
      out_tile = grp * ROT + rt / 2;
      which = rt & 1;
    } else {
      out_tile = grp * ROT + rt;
    }
    const int n0 = out_tile * 16;
    const bool ok = n0 < P.N;
    tl.W = which ? P.w2 : P.w[0];
    tl.S = which ? P.s2 : P.s[0];
    tl.B = which ? P.b2 : P.b[0];
    tl.row0 = ok ? n0 : 0;
    if (!P.swiglu && P.nseg > 1) {
#pragma unroll
      for (int i = 1; i < 3; ++i)
        if (i < P.nseg && ok && n0 >= P.seg_end[i - 1]) {
          tl.W = P.w[i];
          tl.S = P.s[i];
          tl.B = P.b[i];
          tl.row0 = n0 - P.seg_end[i - 1];
        }
    }
    tl.ub = ok ? (units * kw) / WK : 0;
    tl.ue = ok ? (units * (kw + 1)) / WK : 0;
    return tl;
  };
  auto n_groups_of = [&](const ChainPhase& P) {
    const int RT = 8 / P.wk, ROT = P.swiglu ? RT / 2 : RT;
    return (P.N / 16 + ROT - 1) / ROT;
  };
  // every tile this CTA streams in phase P -> L2, one request per tile (lanes 1, 2: scales,
  // biases), issued by the warps that own a tile's first K range
  auto l2_slice = [&](const ChainPhase& P) {
    if (warp % P.wk != 0 || lane >= 3) return;
    const int KW = P.K / 8, G = P.K / 64;
    for (int grp = blockIdx.x; grp < n_groups_of(P); grp += gridDim.x) {
      const Tile tl = tile_of(P, grp);
      if (tl.ub >= tl.ue) continue;
      if (lane == 0)
        l2_prefetch_range(tl.W + (size_t)tl.row0 * KW, (size_t)16 * KW * 4);
      else
        l2_prefetch_range((lane == 1 ? tl.S : tl.B) + (size_t)tl.row0 * G, (size_t)16 * G * 2);
    }
  };

  const uint4 *wg = nullptr, *w8 = nullptr;
  const uint32_t *sgp = nullptr, *sg8 = nullptr, *bgp = nullptr, *bg8 = nullptr;
  int ub = 0, ue = 0;
  auto bind = [&](const ChainPhase& P, const Tile& tl) {
    const int KW = P.K / 8, G = P.K / 64;
    ub = tl.ub;
    ue = tl.ue;
    wg = reinterpret_cast<const uint4*>(tl.W + (size_t)(tl.row0 + g) * KW) + t;
    w8 = wg + (size_t)2 * KW;
    sgp = reinterpret_cast<const uint32_t*>(tl.S + (size_t)(tl.row0 + g) * G) + t;
    sg8 = sgp + (size_t)4 * G;
    bgp = reinterpret_cast<const uint32_t*>(tl.B + (size_t)(tl.row0 + g) * G) + t;
    bg8 = bgp + (size_t)4 * G;
  };
  uint4 buf[D][4];
  uint32_t sb[D / 2][4];
  auto load_unit = [&](uint4 (&bb)[4], int u) {
    bb[0] = m1_ldg128(wg + 8 * u);
    bb[1] = m1_ldg128(wg + 8 * u + 4);
    bb[2] = m1_ldg128(w8 + 8 * u);
    bb[3] = m1_ldg128(w8 + 8 * u + 4);
  };
  auto load_scales = [&](uint32_t (&q)[4], int u0) {
    const bool ok = u0 + (t >> 1) < ue;
    q[0] = ok ? __ldg(sgp + 2 * u0) : 0u;
    q[1] = ok ? __ldg(sg8 + 2 * u0) : 0u;
    q[2] = ok ? __ldg(bgp + 2 * u0) : 0u;
    q[3] = ok ? __ldg(bg8 + 2 * u0) : 0u;
  };
  auto prologue = [&]() {
#pragma unroll
    for (int d = 0; d < D; ++d) {
      if (ub + d < ue) load_unit(buf[d], ub + d);
      if ((d & 1) == 0) load_scales(sb[d / 2], ub + d);
    }
  };

  // phase 0's slice and first weights: none depends on the previous kernel
  l2_slice(a.ph[0]);
  if (a.l2_ahead && a.nph > 1) l2_slice(a.ph[1]);
  bind(a.ph[0], tile_of(a.ph[0], blockIdx.x));
  prologue();
#pragma unroll 1
  for (int p = 0; p < a.nph; ++p) {
    const ChainPhase& P = a.ph[p];
    const int K = P.K, N = P.N, WK = P.wk, G = K / 64;
    const int RT = 8 / WK, ROT = P.swiglu ? RT / 2 : RT;
    const bool norm = P.norm_w != nullptr;
    uint4 nwr[kM1NormChunks];
    if (norm) {
#pragma unroll
      for (int r = 0; r < kM1NormChunks; ++r) {
        const int c = threadIdx.x + r * kM1Threads;
        nwr[r] = c < K / 8 ? *reinterpret_cast<const uint4*>(P.norm_w + 8 * c) : make_uint4(0, 0, 0, 0);
      }
    }
    if (p == 0) {
      pdl_wait();
      pdl_launch();
    } else {
      chain_wait(a.bar + (p - 1) * kChainBarWords, a.err);
    }
    uint8_t* xf = smem;
    uint8_t* zero = smem + m1_xf_bytes(K) + 64;
    float* xs = reinterpret_cast<float*>(zero + 576);
    float* red = xs + G;
    if (threadIdx.x < 32) reinterpret_cast<uint4*>(zero)[threadIdx.x] = make_uint4(0, 0, 0, 0);
    // activations were written by other CTAs of this launch: read them from L2 (ld.cg)
    const uint16_t* x = P.x;
    uint4 xr[kM1RegChunks];
    float inv = 1.0f;
    if (norm) {
      float ss = 0.f;
#pragma unroll
      for (int r = 0; r < kM1RegChunks; ++r) xr[r] = make_uint4(0, 0, 0, 0);
      for (int c = threadIdx.x, r = 0; c < K / 8; c += kM1Threads, ++r) {
        const uint4 v = __ldcg(reinterpret_cast<const uint4*>(x + 8 * c));
#pragma unroll
        for (int j = 0; j < kM1RegChunks; ++j)
          if (j == r) xr[j] = v;
        const uint32_t* vp = &v.x;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float lo = bf_lo(vp[j]), hi = bf_hi(vp[j]);
          ss += lo * lo + hi * hi;
        }
      }
      ss = warp_sum(ss);
      if (lane == 0) s_ss[warp] = ss;
      __syncthreads();
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) tot += s_ss[w];
      inv = 1.0f / sqrtf(tot / (float)K + a.eps);
    }
    for (int base = warp * 32, r = 0; base < K / 8; base += kM1Threads, ++r) {
      const int c = base + lane;
      uint4 v;
      if (norm) {
        v = xr[0];
#pragma unroll
        for (int j = 1; j < kM1RegChunks; ++j)
          if (j == r) v = xr[j];
        if (r >= kM1RegChunks) v = __ldcg(reinterpret_cast<const uint4*>(x + 8 * c));
        uint4 wv = nwr[0];
#pragma unroll
        for (int j = 1; j < kM1NormChunks; ++j)
          if (j == r) wv = nwr[j];
        if (r >= kM1NormChunks) wv = *reinterpret_cast<const uint4*>(P.norm_w + 8 * c);
        uint32_t* vp = &v.x;
        const uint32_t* wp = &wv.x;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          vp[j] = pack_bf2(bf_lo(vp[j]) * inv * bf_lo(wp[j]), bf_hi(vp[j]) * inv * bf_hi(wp[j]));
      } else {
        v = __ldcg(reinterpret_cast<const uint4*>(x + 8 * c));
      }
      const int u = c >> 5, h = (c >> 4) & 1, tt = (c >> 2) & 3, e = c & 3;
      *reinterpret_cast<uint4*>(xf + ((u * 8 + h * 4 + e) * 4 + tt) * 16) = m1_frag(v);
      const uint32_t* vp = &v.x;
      float x1 = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) x1 += bf_lo(vp[j]) + bf_hi(vp[j]);
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) x1 += __shfl_xor_sync(0xffffffffu, x1, o);
      if ((lane & 7) == 0) xs[c >> 3] = x1;
    }
    __syncthreads();
    if (a.l2_ahead && p + 2 < a.nph) l2_slice(a.ph[p + 2]);

    const uint32_t xreal = smem_u32(xf) + t * 16;
    const uint32_t xzero = smem_u32(zero);
    const float2* xs2 = reinterpret_cast<const float2*>(xs);
    const int n_groups = n_groups_of(P);
    for (int grp = blockIdx.x; grp < n_groups; grp += gridDim.x) {
      if (grp != (int)blockIdx.x) {
        bind(P, tile_of(P, grp));
        prologue();
      }
      float acc[2][4];
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[h][c] = 0.f;
      float yg = 0.f, yg8 = 0.f;
      for (int base = ub; base < ue; base += D) {
#pragma unroll
        for (int d = 0; d < D; ++d) {
          const int u = base + d;
          if (u >= ue) break;
          const int pp = d & 1;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const bool act = g == 4 * pp + 2 * h + (t >> 1);
            const uint32_t xb = (act ? xreal + u * 512 : xzero) + h * 256;
            uint4 xv[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) xv[e] = m1_lds128(xb + e * 64);
            const uint32_t* wa = &buf[d][h].x;
            const uint32_t* wb = &buf[d][2 + h].x;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const uint32_t A = wa[e], B = wb[e];
              m1_mma(acc[h], nib_pair_bf16<0>(A), nib_pair_bf16<0>(B), nib_pair_bf16<4>(A),
                     nib_pair_bf16<4>(B), xv[e].x, xv[e].y);
              m1_mma(acc[h], nib_pair_bf16<8>(A), nib_pair_bf16<8>(B), nib_pair_bf16<12>(A),
                     nib_pair_bf16<12>(B), xv[e].z, xv[e].w);
            }
          }
          if (u + D < ue) load_unit(buf[d], u + D);
          if (pp == 1 || u + 1 == ue) {
            const int u0 = u - pp;
            const bool ok = u0 + (t >> 1) < ue;
            const float2 X = xs2[ok ? 2 * u0 + t : 0];
            const uint32_t* q = sb[d / 2];
            const float sa = bf_lo(q[0]), sb_ = bf_hi(q[0]), s8a = bf_lo(q[1]), s8b = bf_hi(q[1]);
            const float ba = fmaf(-128.0f, sa, bf_lo(q[2])), bb = fmaf(-128.0f, sb_, bf_hi(q[2]));
            const float b8a = fmaf(-128.0f, s8a, bf_lo(q[3])), b8b = fmaf(-128.0f, s8b, bf_hi(q[3]));
            yg = fmaf(sa, acc[0][0] + acc[1][0], fmaf(ba, X.x, yg));
            yg = fmaf(sb_, acc[0][1] + acc[1][1], fmaf(bb, X.y, yg));
            yg8 = fmaf(s8a, acc[0][2] + acc[1][2], fmaf(b8a, X.x, yg8));
            yg8 = fmaf(s8b, acc[0][3] + acc[1][3], fmaf(b8b, X.y, yg8));
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
              for (int c = 0; c < 4; ++c) acc[h][c] = 0.f;
            if (u0 + D < ue) load_scales(sb[d / 2], u0 + D);
          }
        }
      }
      yg += __shfl_xor_sync(0xffffffffu, yg, 1);
      yg += __shfl_xor_sync(0xffffffffu, yg, 2);
      yg8 += __shfl_xor_sync(0xffffffffu, yg8, 1);
      yg8 += __shfl_xor_sync(0xffffffffu, yg8, 2);
      if (t == 0) {
        red[warp * 16 + g] = yg;
        red[warp * 16 + g + 8] = yg8;
      }
      __syncthreads();
      if ((int)threadIdx.x < ROT * 16) {
        const int r = threadIdx.x >> 4, j = threadIdx.x & 15;
        const int tile = grp * ROT + r;
        const int row = tile * 16 + j;
        if (tile * 16 < N) {
          if (P.swiglu) {
            float vg = 0.f, vu = 0.f;
            for (int w = 0; w < WK; ++w) {
              vg += red[((2 * r) * WK + w) * 16 + j];
              vu += red[((2 * r + 1) * WK + w) * 16 + j];
            }
            const float gv = round_bf(vg), uv = round_bf(vu);
            P.y[row] = f2bf(gv / (1.0f + expf(-gv)) * uv);
          } else {
            float v = 0.f;
            for (int w = 0; w < WK; ++w) v += red[(r * WK + w) * 16 + j];
            if (P.y_f32) P.y_f32[row] = v;
            if (P.y) {
              uint16_t o = f2bf(v);
              if (P.residual) o = f2bf(bf2f(o) + bf2f(__ldcg(P.residual + row)));
              P.y[row] = o;
            }
          }
        }
      }
      __syncthreads();
    }
    // the next phase's first weights go in flight before the barrier
    if (p + 1 < a.nph) {
      const ChainPhase& Q = a.ph[p + 1];
      if (!a.l2_ahead) l2_slice(Q);
      bind(Q, tile_of(Q, blockIdx.x));
      prologue();
    }
    const bool last = chain_arrive(a.bar + p * kChainBarWords);
    if (p + 1 == a.nph && last) {
      // the last CTA out: every other CTA has passed every wait of this launch
      for (int i = 0; i < a.nph; ++i) a.bar[i * kChainBarWords + kChainRelease] = 0u;
      __threadfence();
    }
  }
}

bool g_m1_on = true;
bool g_m1_l2 = true;  // each CTA prefetches its whole weight slice to L2 before the wait
int g_m1_wk = 0;      // forced K split (1, 2, 4, 8), 0 = cost model
int g_m1_depth = 2;   // units in flight per warp (2 or 4)
// grid capped at the resident slots, CTAs looping over tile groups; off = one CTA per group.
// Measured on B200 (B=1 Qwen3-8B step, same box): one CTA per group with the L2 prefetch
// 2.278 ms, capped grid 2.326 (no prefetch) / 2.369 (prefetch), one CTA per group without
// the prefetch 2.426, the multi-token ring kernel 2.415; capping gate/up alone (its
// late second wave folded into resident CTAs) 2.232 vs 2.146 on another box
int g_m1_persist = 0;  // 1: every launch; 2: gate/up only, at its one-CTA-per-group split
int g_m1_l1 = 0;  // units ahead of the register ring that are prefetched into L1 (0 = off)

template <int WK, int EPI, bool NORM, int D>
cudaError_t m1_launch_cfg(const QLinArgs& a, int ctas, size_t smem, cudaStream_t st) {
  if constexpr (NORM && D == 2) {
    if (a.tp_pull) {
      auto kp = qgemv_m1_kernel<WK, EPI, NORM, D, true>;
      static PerDeviceOnce attr_p;
      const cudaError_t e = attr_p.run(
          [&] { return cudaFuncSetAttribute(kp, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024); });
      if (e != cudaSuccess) return e;
      return launch_pdl(kp, dim3(ctas), dim3(kM1Threads), smem, st, a);
    }
  }
  if (a.tp_pull) return cudaErrorInvalidValue;  // pulls run only the fused-norm, depth-2 kernel
  auto k = qgemv_m1_kernel<WK, EPI, NORM, D>;
  static PerDeviceOnce attr;
  const cudaError_t e =
      attr.run([&] { return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024); });
  if (e != cudaSuccess) return e;
  return launch_pdl(k, dim3(ctas), dim3(kM1Threads), smem, st, a);
}

}  // namespace

// K split of a one-CTA-per-group launch (the default): single matrices take the most K splits
// whose CTAs fit one wave, so every CTA is resident (and has asked L2 for its whole slice) from
// the start; wider outputs take wk = 1.  Gate/up (twice the bytes per row tile) takes the
// fewest splits that fill every slot -- at wk = 1 its 57 MB is not in L2 by the time its input
// is.  Per-launch times inside the B=1 Qwen3-8B step on B200 (us, by wk 1/2/4/8): qkv
// 12.6/9.5/6.0/8.7, o_proj 14.8/9.6/6.0/4.7, down 32.1/24.4/18.8/12.0, LM head 89/96/120/178;
// gate/up wk 2 20.7, wk 1 25.7 (18.9 only behind a slow o_proj).  The decode-chain kernel
// takes the same split, so its results equal these launches' bit for bit.
int m1_default_wk(int N, int K, bool swiglu, int slots) {
  const int nrt = N / 16, units = K / 256;
  const int max_wk = swiglu ? 4 : 8;
  int wk;
  if (swiglu) {
    wk = max_wk;
    for (int c = 1; c <= max_wk; c *= 2) {
      const int rot = (8 / c) / 2;
      if ((nrt + rot - 1) / rot >= slots) {
        wk = c;
        break;
      }
    }
  } else {
    wk = 1;
    for (int c = max_wk; c >= 1; c /= 2)
      if ((nrt + 8 / c - 1) / (8 / c) <= slots) {
        wk = c;
        break;
      }
  }
  if (g_m1_wk > 0) wk = g_m1_wk > max_wk ? max_wk : g_m1_wk;
  while (wk > 1 && units < wk) wk >>= 1;
  return wk;
}

namespace {

template <int EPI, bool NORM, int D>
cudaError_t m1_launch_d(const QLinArgs& a_in, cudaStream_t st) {
  QLinArgs a = a_in;
  if (g_m1_l2) a.self_prefetch = 1;
  a.m1_l1_ahead = g_m1_l1;
  const int nrt = a.N / 16;
  const int units = a.K / 256;
  const size_t smem = m1_smem_bytes(a.K);
  const int slots = kM1CtasPerSm * sm_count();
  // Capped grid (persist mode 1): cost of a K split = the resident CTAs' iterations over
  // tile groups x (units per warp + 1, the per-group reduction); ties go to more splits
  // (more warps streaming).  It picks the split that is fastest for each Qwen3-8B shape
  // when timed alone on B200 (qkv 4, o_proj / down 8, gate/up 4, LM head 2).
  const int max_wk = EPI == EPI_SWIGLU ? 4 : 8;
  int wk = 1;
  long long best = -1;
  for (int c = 1; c <= max_wk && c <= units; c *= 2) {
    const int rot = EPI == EPI_SWIGLU ? (8 / c) / 2 : 8 / c;
    const long long groups = (nrt + rot - 1) / rot;
    const long long cost = (groups + slots - 1) / slots * ((units + c - 1) / c + 1);
    if (best < 0 || cost <= best) {
      best = cost;
      wk = c;
    }
  }
  const bool persist = g_m1_persist == 1 || (g_m1_persist == 2 && EPI == EPI_SWIGLU);
  if (g_m1_persist != 1) {
    wk = m1_default_wk(a.N, a.K, EPI == EPI_SWIGLU, slots);  // one CTA per group
  } else {
    if (g_m1_wk > 0) wk = g_m1_wk > max_wk ? max_wk : g_m1_wk;
    while (wk > 1 && units < wk) wk >>= 1;
  }
  const int rot = EPI == EPI_SWIGLU ? (8 / wk) / 2 : 8 / wk;
  const int groups = (nrt + rot - 1) / rot;
  const int ctas = (persist && groups > slots) ? slots : groups;
  switch (wk) {
    case 8:
      if constexpr (EPI != EPI_SWIGLU) return m1_launch_cfg<8, EPI, NORM, D>(a, ctas, smem, st);
      return cudaErrorInvalidValue;
    case 4: return m1_launch_cfg<4, EPI, NORM, D>(a, ctas, smem, st);
    case 2: return m1_launch_cfg<2, EPI, NORM, D>(a, ctas, smem, st);
    default: return m1_launch_cfg<1, EPI, NORM, D>(a, ctas, smem, st);
  }
}

template <int EPI, bool NORM>
cudaError_t m1_launch_norm(const QLinArgs& a, cudaStream_t st) {
  return g_m1_depth == 4 ? m1_launch_d<EPI, NORM, 4>(a, st) : m1_launch_d<EPI, NORM, 2>(a, st);
}

}  // namespace

// One token, not a grouped-expert launch, K within the staged-x limit.
bool qgemv_m1_supported(const QLinArgs& a) {
  return g_m1_on && a.M == 1 && a.moe_items == nullptr && a.K % 256 == 0 && a.K <= kM1MaxK &&
         a.N % 16 == 0;
}

cudaError_t launch_qgemv_m1(const QLinArgs& a, int epi, cudaStream_t st) {
  if (!qgemv_m1_supported(a)) return cudaErrorInvalidValue;
  if (epi == EPI_SWIGLU)
    return a.norm_w ? m1_launch_norm<EPI_SWIGLU, true>(a, st) : m1_launch_norm<EPI_SWIGLU, false>(a, st);
  return a.norm_w ? m1_launch_norm<EPI_STORE, true>(a, st) : m1_launch_norm<EPI_STORE, false>(a, st);
}

void qgemv_m1_set(int on, int wk, int depth, int l2, int persist, int l1) {
  if (l1 >= 0) g_m1_l1 = l1 > 16 ? 16 : l1;
  if (persist >= 0) g_m1_persist = persist > 2 ? 2 : persist;
  if (l2 >= 0) g_m1_l2 = l2 != 0;
  if (on >= 0) g_m1_on = on != 0;
  if (wk >= 0) g_m1_wk = (wk == 1 || wk == 2 || wk == 4 || wk == 8) ? wk : 0;
  if (depth >= 0) g_m1_depth = depth == 4 ? 4 : 2;
}

// ---- decode chain host side ----
// Off by default: measured on B200 inside the B=1 Qwen3-8B step it is slower than the
// separate launches (2.64 ms with one arrival counter per phase, 2.84 ms with grouped
// counters and a release flag, vs 2.14 ms): a grid barrier costs more than a kernel
// boundary with programmatic dependent launch.
static bool g_chain_on = false;
static int g_chain_l2_ahead = 1;

void decode_chain_set(int on, int l2_ahead) {
  if (on >= 0) g_chain_on = on != 0;
  if (l2_ahead >= 0) g_chain_l2_ahead = l2_ahead != 0;
}

bool decode_chain_on() { return g_chain_on && g_m1_on; }

bool decode_chain_fits(const ChainPhase& p) {
  return p.K % 256 == 0 && p.K <= kM1MaxK && p.N % 16 == 0 && p.N > 0 &&
         (!p.norm_w || p.K <= 8 * kM1Threads * kM1RegChunks) && (!p.swiglu || p.N % 32 == 0);
}

cudaError_t launch_decode_chain(ChainPhase* ph, int nph, float eps, unsigned* bar, cudaStream_t st) {
  if (nph < 1 || nph > kChainMaxPhases || !bar) return cudaErrorInvalidValue;
  ChainArgs a;
  memset(&a, 0, sizeof(a));
  const int slots = kM1CtasPerSm * sm_count();
  size_t smem = 0;
  for (int i = 0; i < nph; ++i) {
    if (!decode_chain_fits(ph[i])) return cudaErrorInvalidValue;
    ph[i].wk = m1_default_wk(ph[i].N, ph[i].K, ph[i].swiglu != 0, slots);
    a.ph[i] = ph[i];
    smem = std::max(smem, m1_smem_bytes(ph[i].K));
  }
  a.nph = nph;
  a.eps = eps;
  a.bar = bar;
  a.err = device_state(current_device()).tc_err;
  a.l2_ahead = g_chain_l2_ahead;
  auto k = chain_kernel<2>;
  static PerDeviceOnce attr;
  const cudaError_t e =
      attr.run([&] { return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024); });
  if (e != cudaSuccess) return e;
  // one CTA per resident slot: every CTA of the grid is resident at once, which the
  // barriers between phases rely on
  return launch_pdl(k, dim3(slots), dim3(kM1Threads), smem, st, a);
}

}  // namespace higgs

HG_TL_FETCH_FN(higgs_timeline_fetch_gemv)

extern "C" int higgs_decode_chain(higgs_ctx* ctx, const higgs_chain_gemv* phases, int n_phases,
                                  float eps, uint32_t* barriers, void* stream) {
  using namespace higgs;
  HG_CHECK_ARG(ctx && phases && barriers, "higgs_decode_chain: null argument");
  HG_CHECK_ARG(n_phases >= 1 && n_phases <= kChainMaxPhases, "higgs_decode_chain: 1..4 phases");
  ChainPhase ph[kChainMaxPhases];
  for (int i = 0; i < n_phases; ++i) {
    const higgs_chain_gemv& q = phases[i];
    HG_CHECK_ARG(q.x && q.w[0] && q.s[0] && q.b[0] && (q.y || q.y_f32),
                 "higgs_decode_chain: phase without input, weights or output");
    HG_CHECK_ARG(q.nseg >= 1 && q.nseg <= 3, "higgs_decode_chain: nseg must be 1..3");
    HG_CHECK_ARG(!q.swiglu || (q.w2 && q.s2 && q.b2 && q.y && q.nseg == 1),
                 "higgs_decode_chain: SwiGLU needs up weights, a bf16 y and one segment");
    HG_CHECK_ARG(!q.residual || q.y, "higgs_decode_chain: residual needs a bf16 y");
    ChainPhase& p = ph[i];
    p = ChainPhase{};
    p.x = (const uint16_t*)q.x;
    p.norm_w = (const uint16_t*)q.norm_w;
    p.K = q.K;
    p.N = q.N;
    p.swiglu = q.swiglu != 0;
    p.nseg = q.nseg;
    for (int j = 0; j < 3; ++j) {
      p.seg_end[j] = q.seg_end[j];
      p.w[j] = q.w[j];
      p.s[j] = (const uint16_t*)q.s[j];
      p.b[j] = (const uint16_t*)q.b[j];
    }
    if (q.nseg > 1)
      for (int j = 0; j < q.nseg; ++j)
        HG_CHECK_ARG(p.w[j] && p.s[j] && p.b[j] && p.seg_end[j] % 16 == 0 &&
                         (j == 0 ? p.seg_end[0] > 0 : p.seg_end[j] > p.seg_end[j - 1]) &&
                         (j + 1 < q.nseg || p.seg_end[j] == q.N),
                     "higgs_decode_chain: bad row segments");
    p.w2 = q.w2;
    p.s2 = (const uint16_t*)q.s2;
    p.b2 = (const uint16_t*)q.b2;
    p.y = (uint16_t*)q.y;
    p.y_f32 = q.y_f32;
    p.residual = (const uint16_t*)q.residual;
    HG_CHECK_ARG(decode_chain_fits(p), "higgs_decode_chain: shape outside the chain's limits");
  }
  HG_DEVICE(ctx);
  HG_CUDA(launch_decode_chain(ph, n_phases, eps, barriers, (cudaStream_t)stream));
  return HIGGS_OK;
}
