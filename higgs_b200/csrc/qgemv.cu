// qgemv.cu -- W4 g64 GEMV for decode batches, weights streamed through
// per-warp cp.async rings in shared memory.
//
// Reference op replaced: ops::quantized_matmul (qwen3_next.rs:174-183), with
// the preceding nn::RmsNorm (transformer.rs:407, 415) optionally fused.
//
// Layout of the work: a CTA owns RT 16-row tiles; its 8 warps split the K
// range of those tiles (WK = 8 / RT ways) and reduce through shared memory at
// the end.  Per warp, K advances in "units" of 256 (4 groups of 64): a unit is
// 16 rows x 128 B of packed weights + 16 x 4 scales + 16 x 4 biases, copied by
// cp.async into a ring of S stages already in MMA-fragment order, so up to S-1
// units are in flight per warp without occupying registers.
//
// When x (M tokens x K) fits, it is staged once per CTA as fp16 MMA fragments,
// scaled per token by a power of two that puts its largest value in
// [2^13, 2^14) -- exact for bf16 inputs -- and unscaled at the end.  fp16's
// 10-bit mantissa lets one LOP3 turn the nibbles at bits 0-3 of both halves of
// a word into the exact values 1024 + q, and those at bits 4-7 into 1024 + 16 q,
// so 8 weights cost one shift and four LOP3s.  Even- and odd-position nibbles
// accumulate in separate MMA tiles, and the per-group f32 fold is
//   y += s * (acc_even + acc_odd / 16) - s * X2 + b * X1,
//   X1 = sum(x), X2 = 1024 * (sum_even(x) + sum_odd(x) / 16)
// (MLX's s * sum(x q) + b * sum(x) with the offsets removed).  The inner loop
// is 2 LDS.64 of weights, 2 LDS.128 of x, 20 ALU unpack ops and 4 mma.sync
// m16n8k16 per 16 x 64 block.  Without the staged x (M > 8 or very long K)
// the bf16 path reads x from global memory: nibbles -> bf16 128 + q, sum(x)
// from an MMA against an all-ones tile.
#include "common.cuh"
#include "kernels.cuh"

namespace higgs {

namespace {

constexpr int kUnitW = 16 * 128;      // packed weight bytes of a unit
constexpr int kUnitS = 16 * 4 * 2;    // scale bytes of a unit
constexpr int kStage = kUnitW + 2 * kUnitS;  // + biases
// x staged in shared memory (and an input RMSNorm fused into the staging) up to this size;
// higgs_set_option("gemv_xsmem_max", bytes), at most the grouped kernel's 72 KB
size_t g_xsmem_max = 32 * 1024;
constexpr size_t kXsmemGroupedMax = 72 * 1024; // grouped experts always stage 8 pairs

// bytes of the fragment-ordered x tile: per token G groups x 4 lane slots x 32 B, padded
inline size_t xfrag_bytes(int M, int K) { return (size_t)M * ((K / 64) * 128 + 16); }

__device__ __forceinline__ void cp_async8(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(smem)), "l"(gmem));
}

struct Seg {
  const uint32_t* W;
  const uint16_t* S;
  const uint16_t* B;
  int row0;  // first row of the tile within its weight tensor
};

// Issue the cp.asyncs of one unit into a stage.  Weights land as
// [group j][row r][t][8 B] so lane (g, t) later reads rows g and g+8 with two
// conflict-free LDS.64; scales / biases as [row][4 groups] bf16.
__device__ __forceinline__ void issue_unit(uint8_t* stage, const Seg& sg, int KW, int G, int unit,
                                           int lane) {
  // chunk (row r, group j, half p) of the 16 x 128 B slab; within each 8-lane
  // phase the 8 destinations fall in distinct 16-byte bank groups
  const int p = lane & 1, j = lane >> 3;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = ((lane >> 1) & 3) + 4 * i;
    const uint32_t* src = sg.W + (size_t)(sg.row0 + r) * KW + unit * 32 + (2 * j + p) * 4;
    cp_async16(stage + ((j * 16 + r) * 4 + 2 * p) * 8, src);
  }
  const int r = lane & 15;
  const uint16_t* src = (lane < 16 ? sg.S : sg.B) + (size_t)(sg.row0 + r) * G + unit * 4;
  cp_async8(stage + kUnitW + (lane >> 4) * kUnitS + r * 8, src);
}

// fp16 A-operand pairs: nibbles at bits 0-3 of each half -> 1024 + q (exact),
// nibbles at bits 4-7 -> 1024 + 16 q (exact): no shift for either.
__device__ __forceinline__ uint32_t nib_even_f16(uint32_t w) {
  return lop3_and_or(w, 0x000F000Fu, 0x64006400u);
}
__device__ __forceinline__ uint32_t nib_odd_f16(uint32_t w) {
  return lop3_and_or(w, 0x00F000F0u, 0x64006400u);
}

__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                              uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// ONE: a single token (M == 1); only its outputs are folded.
template <int NT8, int WK, int EPI, int S, bool XSMEM, bool NORM, bool F16, bool GATHER, bool ONE = false>
__global__ void __launch_bounds__(256) qgemv_ring_kernel(QLinArgs a) {
  static_assert(!GATHER || (XSMEM && NT8 == 1), "grouped experts use the staged-x path");
  static_assert(!ONE || (XSMEM && NT8 == 1 && !GATHER && !F16), "single-token fold: staged bf16 x");
  constexpr int RT = 8 / WK;
  constexpr int ROT = (EPI == EPI_SWIGLU) ? RT / 2 : RT;
  constexpr int MT = 8 * NT8;  // token slots
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int rt = warp / WK, kw = warp % WK;
  const int K = a.K, N = a.N;
  int M = a.M;
  // token m reads x row xrow(m) and writes output row orow(m) (identity unless GATHER)
  __shared__ int s_xrow[GATHER ? MT : 1], s_orow[GATHER ? MT : 1];
  auto xrow = [&](int m) { return GATHER ? s_xrow[m] : m; };
  auto orow = [&](int m) { return GATHER ? s_orow[m] : m; };
  const int KW = K / 8, G = K / 64;
  const int units = G / 4;

  // smem carve: rings | x fragments | sum(x) | norm partials
  uint8_t* ring = smem + warp * S * kStage;
  const int xtok_bytes = G * 128 + 16;  // per token, padded against bank conflicts
  uint8_t* xf = smem + 8 * S * kStage;
  float* xsum = reinterpret_cast<float*>(xf + (XSMEM ? M * xtok_bytes : 0));  // [G][MT]

  int out_tile, which = 0;
  if (EPI == EPI_SWIGLU) {
    out_tile = blockIdx.x * ROT + rt / 2;
    which = rt & 1;
  } else {
    out_tile = blockIdx.x * ROT + rt;
  }
  const int n0 = out_tile * 16;
  const bool tile_ok = n0 < N;
  Seg sg;
  sg.W = which ? a.w2 : a.w;
  sg.S = which ? a.s2 : a.s;
  sg.B = which ? a.b2 : a.b;
  sg.row0 = n0;
  if (EPI != EPI_SWIGLU && a.nseg > 1) {
#pragma unroll
    for (int i = 1; i < 3; ++i)
      if (i < a.nseg && n0 >= a.seg_end[i - 1]) {
        sg.W = a.wseg[i];
        sg.S = a.sseg[i];
        sg.B = a.bseg[i];
        sg.row0 = n0 - a.seg_end[i - 1];
      }
  }
  const int ub = tile_ok ? (units * kw) / WK : 0;
  const int ue = tile_ok ? (units * (kw + 1)) / WK : 0;

  // weights of the step's next GEMV -> L2, while this kernel's chain runs
  issue_l2_prefetch(a.pf, blockIdx.y * gridDim.x + blockIdx.x, gridDim.x * gridDim.y);
  if constexpr (!GATHER) {
    if (a.self_prefetch && tile_ok && kw == 0 && lane == 0) {
      // this tile's whole weight rows -> L2 (the ring below keeps only S-1 units in flight)
      l2_prefetch_range(sg.W + (size_t)sg.row0 * KW, (size_t)16 * KW * 4);
      l2_prefetch_range(sg.S + (size_t)sg.row0 * G, (size_t)16 * G * 2);
      l2_prefetch_range(sg.B + (size_t)sg.row0 * G, (size_t)16 * G * 2);
    }
    // prefetch the first S-1 units (weights never depend on the previous kernel)
#pragma unroll
    for (int s = 0; s < S - 1; ++s) {
      if (ub + s < ue) issue_unit(ring + s * kStage, sg, KW, G, ub + s, lane);
      cp_async_commit();
    }
    pdl_wait();
    pdl_launch();
  } else {
    // the expert and its pairs come from the router's plan: read it first
    pdl_wait();
    pdl_launch();
    if ((int)blockIdx.y >= *a.moe_n_items) return;  // uniform over the CTA
    const int4 it = a.moe_items[blockIdx.y];
    if (a.moe_e_n && (it.x < a.moe_e_lo || it.x >= a.moe_e_lo + a.moe_e_n)) return;  // another rank's
    M = it.z;
    const long long el = it.x - a.moe_e_lo;  // index among the experts held here
    sg.W += el * a.moe_ew;
    sg.S += el * a.moe_es;
    sg.B += el * a.moe_es;
    if (a.self_prefetch && tile_ok && kw == 0 && lane == 0) {
      l2_prefetch_range(sg.W + (size_t)sg.row0 * KW, (size_t)16 * KW * 4);
      l2_prefetch_range(sg.S + (size_t)sg.row0 * G, (size_t)16 * G * 2);
      l2_prefetch_range(sg.B + (size_t)sg.row0 * G, (size_t)16 * G * 2);
    }
    if (threadIdx.x < MT) {
      const int pr = threadIdx.x < M ? a.moe_sorted[it.y + threadIdx.x] : 0;
      s_xrow[threadIdx.x] = pr / a.moe_xdiv;
      s_orow[threadIdx.x] = pr;
    }
#pragma unroll
    for (int s = 0; s < S - 1; ++s) {
      if (ub + s < ue) issue_unit(ring + s * kStage, sg, KW, G, ub + s, lane);
      cp_async_commit();
    }
    __syncthreads();
  }

  // XSMEM path: x in fp16 fragments, scaled per token by 2^e (exact for bf16
  // inputs) into fp16 range; X1 = sum(x), X2 = 1024 * (sum_even(x) + sum_odd(x) / 16)
  // per (group, token), where even / odd are the k positions fed to the MMA as
  // 1024 + q and 1024 + 16 q.
  float* x1s = xsum;                // [G][MT]
  float* x2s = xsum + G * MT;       // [G][MT]
  __shared__ float unscale[MT];     // 2^-e per token
  if constexpr (XSMEM) {
    __shared__ float inv_rms[MT];
    __shared__ float red[8][MT];
    __shared__ float redm[8][MT];
    // one pass over x when every staging task below fits one thread (fused norm, bf16
    // operands): the values loaded for the RMS statistics stay in registers for the staging
    const bool one_pass = NORM && !F16 && M * G * 4 <= 256;
    uint4 pv0 = make_uint4(0, 0, 0, 0), pv1 = make_uint4(0, 0, 0, 0), pw0 = pv0, pw1 = pv0;
    if (one_pass && (int)threadIdx.x < M * G * 4) {
      const int task = threadIdx.x;
      const int k0 = ((task / 4) % G) * 64 + 16 * (task % 4);
      const uint16_t* src = a.x + (size_t)xrow(task / (G * 4)) * K + k0;
      pv0 = *reinterpret_cast<const uint4*>(src);
      pv1 = *reinterpret_cast<const uint4*>(src + 8);
      pw0 = *reinterpret_cast<const uint4*>(a.norm_w + k0);  // with the same round trip
      pw1 = *reinterpret_cast<const uint4*>(a.norm_w + k0 + 8);
    }
    if constexpr (!NORM && !F16) {
      // plain bf16 staging: no statistics needed
      if (threadIdx.x < MT) {
        inv_rms[threadIdx.x] = 1.0f;
        unscale[threadIdx.x] = threadIdx.x < M ? 1.0f : 0.0f;
        red[0][threadIdx.x] = 1.0f;
      }
      __syncthreads();
    } else {
      float ss[MT], mx[MT];
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        ss[m] = 0.f;
        mx[m] = 0.f;
      }
      if (one_pass && (int)threadIdx.x < M * G * 4) {
        const int m = threadIdx.x / (G * 4);
        const uint32_t* p0 = &pv0.x;
        const uint32_t* p1 = &pv1.x;
        float acc = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float a0 = bf_lo(p0[e]), a1 = bf_hi(p0[e]), b0 = bf_lo(p1[e]), b1 = bf_hi(p1[e]);
          acc += a0 * a0 + a1 * a1 + b0 * b0 + b1 * b1;
        }
#pragma unroll
        for (int mm = 0; mm < MT; ++mm)
          if (mm == m) ss[mm] += acc;
      }
      for (int vi = one_pass ? M * (K / 8) : (int)threadIdx.x; vi < M * (K / 8); vi += 256) {
        const int m = vi / (K / 8), k8 = vi % (K / 8);
        const uint4 v = *reinterpret_cast<const uint4*>(a.x + (size_t)xrow(m) * K + k8 * 8);
        const uint32_t* vp = &v.x;
        uint4 wv = make_uint4(0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u);
        if constexpr (NORM && F16) wv = *reinterpret_cast<const uint4*>(a.norm_w + k8 * 8);
        const uint32_t* wp = &wv.x;
        float acc = 0.f, am = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float lo = bf_lo(vp[j]), hi = bf_hi(vp[j]);
          acc += lo * lo + hi * hi;
          if constexpr (F16)  // the fp16 operand scale needs the largest |x * w|
            am = fmaxf(am, fmaxf(fabsf(lo * bf_lo(wp[j])), fabsf(hi * bf_hi(wp[j]))));
        }
#pragma unroll
        for (int mm = 0; mm < MT; ++mm)
          if (mm == m) {
            ss[mm] += acc;
            mx[mm] = fmaxf(mx[mm], am);
          }
      }
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        if (m >= M) break;  // M is uniform over the CTA
        const float r = warp_sum(ss[m]);
        const float q = F16 ? warp_max(mx[m]) : 0.f;
        if (lane == 0) {
          red[warp][m] = r;
          redm[warp][m] = q;
        }
      }
      __syncthreads();
      if (threadIdx.x < MT) {
        float tot = 0.f, amax = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
          tot += red[w][threadIdx.x];
          amax = fmaxf(amax, redm[w][threadIdx.x]);
        }
        const float inv = NORM ? 1.0f / sqrtf(tot / (float)K + a.eps) : 1.0f;
        inv_rms[threadIdx.x] = inv;
        // largest |x| -> [2^13, 2^14): exact fp16 for every bf16 value of the token
        int ex = 0;
        const float xm = amax * inv;
        if (xm > 0.f && isfinite(xm)) {
          frexpf(xm, &ex);
          ex = 14 - ex;
        } else {
          ex = 0;
        }
        ex = F16 ? max(-100, min(100, ex)) : 0;
        inv_rms[threadIdx.x] = inv;
        unscale[threadIdx.x] = ldexpf(1.0f, -ex);
        red[0][threadIdx.x] = ldexpf(1.0f, ex);  // reused as the per-token scale
      }
      __syncthreads();
    }
    // one task = (token m, group j, lane-slot tt): 16 values -> 8 u32 fragment words.
    // Whole warps iterate together (the group sums below shuffle across 4 lanes).
    const int n_tasks = M * G * 4;
    for (int base = warp * 32; base < n_tasks; base += 256) {
      const int task = base + lane;
      const bool valid = task < n_tasks;
      const int m = valid ? task / (G * 4) : 0, j = valid ? (task / 4) % G : 0, tt = task % 4;
      const uint16_t* src = a.x + (size_t)xrow(m) * K + j * 64 + 16 * tt;
      uint4 v0 = make_uint4(0, 0, 0, 0), v1 = make_uint4(0, 0, 0, 0);
      if (one_pass) {  // this thread's only task, loaded above
        v0 = pv0;
        v1 = pv1;
      } else if (valid) {
        v0 = *reinterpret_cast<const uint4*>(src);
        v1 = *reinterpret_cast<const uint4*>(src + 8);
      }
      float xv[16];
      {
        const uint32_t* p0 = &v0.x;
        const uint32_t* p1 = &v1.x;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          xv[2 * e] = bf_lo(p0[e]);
          xv[2 * e + 1] = bf_hi(p0[e]);
          xv[8 + 2 * e] = bf_lo(p1[e]);
          xv[8 + 2 * e + 1] = bf_hi(p1[e]);
        }
      }
      if constexpr (NORM) {
        const float inv = inv_rms[m];
        const uint4 w0 = one_pass ? pw0 : *reinterpret_cast<const uint4*>(a.norm_w + j * 64 + 16 * tt);
        const uint4 w1 = one_pass ? pw1 : *reinterpret_cast<const uint4*>(a.norm_w + j * 64 + 16 * tt + 8);
        const uint32_t* q0 = &w0.x;
        const uint32_t* q1 = &w1.x;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          xv[2 * e] = round_bf(xv[2 * e] * inv * bf_lo(q0[e]));
          xv[2 * e + 1] = round_bf(xv[2 * e + 1] * inv * bf_hi(q0[e]));
          xv[8 + 2 * e] = round_bf(xv[8 + 2 * e] * inv * bf_lo(q1[e]));
          xv[8 + 2 * e + 1] = round_bf(xv[8 + 2 * e + 1] * inv * bf_hi(q1[e]));
        }
      }
      const float sc = red[0][m];
#pragma unroll
      for (int e = 0; e < 16; ++e) xv[e] *= sc;  // exact (power of two)
      // even k positions (nibbles 0,2,4,6 of a word) and odd ones (1,3,5,7)
      float se = 0.f, so = 0.f;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        if (e & 1)
          so += xv[e];
        else
          se += xv[e];
      }
      uint4 f0, f1;
      if constexpr (F16) {
        // E0:(0,4)(2,6) E1:(8,12)(10,14) | O0:(1,5)(3,7) O1:(9,13)(11,15)
        f0.x = pack_h2(xv[0], xv[4]);
        f0.y = pack_h2(xv[2], xv[6]);
        f0.z = pack_h2(xv[8], xv[12]);
        f0.w = pack_h2(xv[10], xv[14]);
        f1.x = pack_h2(xv[1], xv[5]);
        f1.y = pack_h2(xv[3], xv[7]);
        f1.z = pack_h2(xv[9], xv[13]);
        f1.w = pack_h2(xv[11], xv[15]);
      } else {
        // bf16 B fragments of the 4 k16 tiles, (k, k+4) pairs as the A side pairs nibbles:
        // (0,4)(1,5) | (2,6)(3,7) | (8,12)(9,13) | (10,14)(11,15)
        f0.x = pack_bf2(xv[0], xv[4]);
        f0.y = pack_bf2(xv[1], xv[5]);
        f0.z = pack_bf2(xv[2], xv[6]);
        f0.w = pack_bf2(xv[3], xv[7]);
        f1.x = pack_bf2(xv[8], xv[12]);
        f1.y = pack_bf2(xv[9], xv[13]);
        f1.z = pack_bf2(xv[10], xv[14]);
        f1.w = pack_bf2(xv[11], xv[15]);
      }
      if (valid) {
        uint4* dst = reinterpret_cast<uint4*>(xf + m * xtok_bytes + (j * 4 + tt) * 32);
        dst[0] = f0;
        dst[1] = f1;
      }
      se += __shfl_xor_sync(0xffffffffu, se, 1);
      se += __shfl_xor_sync(0xffffffffu, se, 2);
      so += __shfl_xor_sync(0xffffffffu, so, 1);
      so += __shfl_xor_sync(0xffffffffu, so, 2);
      if (valid && tt == 0) {
        x1s[j * MT + m] = se + so;
        x2s[j * MT + m] = F16 ? 1024.0f * (se + so * 0.0625f) : 128.0f * (se + so);
      }
    }
    for (int i = threadIdx.x; i < G * MT; i += 256)
      if (i % MT >= M) {
        x1s[i] = 0.f;
        x2s[i] = 0.f;
      }
    if (threadIdx.x < MT && threadIdx.x >= M) unscale[threadIdx.x] = 0.f;
    __syncthreads();
  }

  const uint32_t ONES = 0x3F803F80u;
  float y[NT8][4];
#pragma unroll
  for (int j = 0; j < NT8; ++j)
#pragma unroll
    for (int c = 0; c < 4; ++c) y[j][c] = 0.f;

  for (int u = ub, i = 0; u < ue; ++u, ++i) {
    if (u + S - 1 < ue) issue_unit(ring + ((i + S - 1) % S) * kStage, sg, KW, G, u + S - 1, lane);
    cp_async_commit();
    cp_async_wait<S - 1>();
    __syncwarp();
    const uint8_t* st = ring + (i % S) * kStage;
    const uint2 s0 = *reinterpret_cast<const uint2*>(st + kUnitW + g * 8);
    const uint2 s1 = *reinterpret_cast<const uint2*>(st + kUnitW + (g + 8) * 8);
    const uint2 b0 = *reinterpret_cast<const uint2*>(st + kUnitW + kUnitS + g * 8);
    const uint2 b1 = *reinterpret_cast<const uint2*>(st + kUnitW + kUnitS + (g + 8) * 8);
    const float sgv[4] = {bf_lo(s0.x), bf_hi(s0.x), bf_lo(s0.y), bf_hi(s0.y)};
    const float sg8[4] = {bf_lo(s1.x), bf_hi(s1.x), bf_lo(s1.y), bf_hi(s1.y)};
    const float bgv[4] = {bf_lo(b0.x), bf_hi(b0.x), bf_lo(b0.y), bf_hi(b0.y)};
    const float bg8[4] = {bf_lo(b1.x), bf_hi(b1.x), bf_lo(b1.y), bf_hi(b1.y)};
#pragma unroll
    for (int gi = 0; gi < 4; ++gi) {
      const int grp = u * 4 + gi;
      const uint2 wr0 = *reinterpret_cast<const uint2*>(st + ((gi * 16 + g) * 4 + t) * 8);
      const uint2 wr1 = *reinterpret_cast<const uint2*>(st + ((gi * 16 + g + 8) * 4 + t) * 8);
      const uint32_t wA = wr0.x, wB = wr0.y, wC = wr1.x, wD = wr1.y;
      if constexpr (XSMEM && !F16) {
        const uint32_t A[4][4] = {
            {nib_pair_bf16<0>(wA), nib_pair_bf16<0>(wC), nib_pair_bf16<4>(wA), nib_pair_bf16<4>(wC)},
            {nib_pair_bf16<8>(wA), nib_pair_bf16<8>(wC), nib_pair_bf16<12>(wA), nib_pair_bf16<12>(wC)},
            {nib_pair_bf16<0>(wB), nib_pair_bf16<0>(wD), nib_pair_bf16<4>(wB), nib_pair_bf16<4>(wD)},
            {nib_pair_bf16<8>(wB), nib_pair_bf16<8>(wD), nib_pair_bf16<12>(wB), nib_pair_bf16<12>(wD)}};
#pragma unroll
        for (int j = 0; j < NT8; ++j) {
          const int tok = 8 * j + g;
          uint4 X0 = make_uint4(0, 0, 0, 0), X1 = make_uint4(0, 0, 0, 0);
          if constexpr (ONE) {
            // every lane takes token 0's fragment: the other MMA columns are never stored
            const uint4* xp = reinterpret_cast<const uint4*>(xf + (grp * 4 + t) * 32);
            X0 = xp[0];
            X1 = xp[1];
          } else if (tok < M) {
            const uint4* xp = reinterpret_cast<const uint4*>(xf + tok * xtok_bytes + (grp * 4 + t) * 32);
            X0 = xp[0];
            X1 = xp[1];
          }
          float acc[4] = {0.f, 0.f, 0.f, 0.f};
          mma_bf16_16816(acc, A[0][0], A[0][1], A[0][2], A[0][3], X0.x, X0.y);
          mma_bf16_16816(acc, A[1][0], A[1][1], A[1][2], A[1][3], X0.z, X0.w);
          mma_bf16_16816(acc, A[2][0], A[2][1], A[2][2], A[2][3], X1.x, X1.y);
          mma_bf16_16816(acc, A[3][0], A[3][1], A[3][2], A[3][3], X1.z, X1.w);
          // y += s * acc + (b - 128 s) * sum(x): the MMA saw 128 + q
          const float bb0 = fmaf(-128.0f, sgv[gi], bgv[gi]), bb1 = fmaf(-128.0f, sg8[gi], bg8[gi]);
          if constexpr (ONE) {  // token 0 sits in lanes t == 0, outputs 0 and 2
            const float x1 = x1s[grp * MT + 2 * t];
            y[j][0] = fmaf(sgv[gi], acc[0], fmaf(bb0, x1, y[j][0]));
            y[j][2] = fmaf(sg8[gi], acc[2], fmaf(bb1, x1, y[j][2]));
          } else {
            const float2 x1 = *reinterpret_cast<const float2*>(x1s + grp * MT + 8 * j + 2 * t);
            y[j][0] = fmaf(sgv[gi], acc[0], fmaf(bb0, x1.x, y[j][0]));
            y[j][1] = fmaf(sgv[gi], acc[1], fmaf(bb0, x1.y, y[j][1]));
            y[j][2] = fmaf(sg8[gi], acc[2], fmaf(bb1, x1.x, y[j][2]));
            y[j][3] = fmaf(sg8[gi], acc[3], fmaf(bb1, x1.y, y[j][3]));
          }
        }
      } else if constexpr (XSMEM && F16) {
        const uint32_t wA8 = wA >> 8, wB8 = wB >> 8, wC8 = wC >> 8, wD8 = wD >> 8;
        // tiles E0, E1 (even nibbles: 1024 + q) and O0, O1 (odd nibbles: 1024 + 16 q)
        const uint32_t AE[2][4] = {
            {nib_even_f16(wA), nib_even_f16(wC), nib_even_f16(wA8), nib_even_f16(wC8)},
            {nib_even_f16(wB), nib_even_f16(wD), nib_even_f16(wB8), nib_even_f16(wD8)}};
        const uint32_t AO[2][4] = {
            {nib_odd_f16(wA), nib_odd_f16(wC), nib_odd_f16(wA8), nib_odd_f16(wC8)},
            {nib_odd_f16(wB), nib_odd_f16(wD), nib_odd_f16(wB8), nib_odd_f16(wD8)}};
        const float s16a = sgv[gi] * 0.0625f, s16b = sg8[gi] * 0.0625f;
#pragma unroll
        for (int j = 0; j < NT8; ++j) {
          const int tok = 8 * j + g;
          uint4 X0 = make_uint4(0, 0, 0, 0), X1 = make_uint4(0, 0, 0, 0);
          if (tok < M) {
            const uint4* xp = reinterpret_cast<const uint4*>(xf + tok * xtok_bytes + (grp * 4 + t) * 32);
            X0 = xp[0];
            X1 = xp[1];
          }
          float ae[4] = {0.f, 0.f, 0.f, 0.f}, ao[4] = {0.f, 0.f, 0.f, 0.f};
          mma_f16_16816(ae, AE[0][0], AE[0][1], AE[0][2], AE[0][3], X0.x, X0.y);
          mma_f16_16816(ae, AE[1][0], AE[1][1], AE[1][2], AE[1][3], X0.z, X0.w);
          mma_f16_16816(ao, AO[0][0], AO[0][1], AO[0][2], AO[0][3], X1.x, X1.y);
          mma_f16_16816(ao, AO[1][0], AO[1][1], AO[1][2], AO[1][3], X1.z, X1.w);
          const float2 x1 = *reinterpret_cast<const float2*>(x1s + grp * MT + 8 * j + 2 * t);
          const float2 x2 = *reinterpret_cast<const float2*>(x2s + grp * MT + 8 * j + 2 * t);
          // y += s (ae + ao/16) - s X2 + b X1
          y[j][0] = fmaf(sgv[gi], ae[0], fmaf(s16a, ao[0], fmaf(bgv[gi], x1.x, fmaf(-sgv[gi], x2.x, y[j][0]))));
          y[j][1] = fmaf(sgv[gi], ae[1], fmaf(s16a, ao[1], fmaf(bgv[gi], x1.y, fmaf(-sgv[gi], x2.y, y[j][1]))));
          y[j][2] = fmaf(sg8[gi], ae[2], fmaf(s16b, ao[2], fmaf(bg8[gi], x1.x, fmaf(-sg8[gi], x2.x, y[j][2]))));
          y[j][3] = fmaf(sg8[gi], ae[3], fmaf(s16b, ao[3], fmaf(bg8[gi], x1.y, fmaf(-sg8[gi], x2.y, y[j][3]))));
        }
      } else {
        const uint32_t A[4][4] = {
            {nib_pair_bf16<0>(wA), nib_pair_bf16<0>(wC), nib_pair_bf16<4>(wA), nib_pair_bf16<4>(wC)},
            {nib_pair_bf16<8>(wA), nib_pair_bf16<8>(wC), nib_pair_bf16<12>(wA), nib_pair_bf16<12>(wC)},
            {nib_pair_bf16<0>(wB), nib_pair_bf16<0>(wD), nib_pair_bf16<4>(wB), nib_pair_bf16<4>(wD)},
            {nib_pair_bf16<8>(wB), nib_pair_bf16<8>(wD), nib_pair_bf16<12>(wB), nib_pair_bf16<12>(wD)}};
        const float bb0 = fmaf(-128.0f, sgv[gi], bgv[gi]);
        const float bb1 = fmaf(-128.0f, sg8[gi], bg8[gi]);
#pragma unroll
        for (int j = 0; j < NT8; ++j) {
          const int tok = 8 * j + g;
          uint4 X0 = make_uint4(0, 0, 0, 0), X1 = make_uint4(0, 0, 0, 0);
          if (tok < M) {
            const uint16_t* xp = a.x + (size_t)tok * K + grp * 64 + 16 * t;
            X0 = ldg_u4(xp);
            X1 = ldg_u4(xp + 8);
          }
          const uint32_t Bf[4][2] = {{prmt(X0.x, X0.z, 0x5410), prmt(X0.x, X0.z, 0x7632)},
                                     {prmt(X0.y, X0.w, 0x5410), prmt(X0.y, X0.w, 0x7632)},
                                     {prmt(X1.x, X1.z, 0x5410), prmt(X1.x, X1.z, 0x7632)},
                                     {prmt(X1.y, X1.w, 0x5410), prmt(X1.y, X1.w, 0x7632)}};
          float acc[4] = {0.f, 0.f, 0.f, 0.f}, xs[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int kt = 0; kt < 4; ++kt) {
            mma_bf16_16816(acc, A[kt][0], A[kt][1], A[kt][2], A[kt][3], Bf[kt][0], Bf[kt][1]);
            mma_bf16_16816(xs, ONES, ONES, ONES, ONES, Bf[kt][0], Bf[kt][1]);
          }
          y[j][0] = fmaf(sgv[gi], acc[0], fmaf(bb0, xs[0], y[j][0]));
          y[j][1] = fmaf(sgv[gi], acc[1], fmaf(bb0, xs[1], y[j][1]));
          y[j][2] = fmaf(sg8[gi], acc[2], fmaf(bb1, xs[0], y[j][2]));
          y[j][3] = fmaf(sg8[gi], acc[3], fmaf(bb1, xs[1], y[j][3]));
        }
      }
    }
    __syncwarp();
  }
  cp_async_wait<0>();

  if constexpr (XSMEM) {
#pragma unroll
    for (int j = 0; j < NT8; ++j) {
      const float u0 = unscale[8 * j + 2 * t], u1 = unscale[8 * j + 2 * t + 1];
      y[j][0] *= u0;
      y[j][1] *= u1;
      y[j][2] *= u0;
      y[j][3] *= u1;
    }
  }
  // cross-warp K reduction (the rings are free now)
  __syncthreads();
  float* red = reinterpret_cast<float*>(smem);  // [8 warps][NT8*4][32]
#pragma unroll
  for (int j = 0; j < NT8; ++j)
#pragma unroll
    for (int c = 0; c < 4; ++c) red[(warp * NT8 * 4 + j * 4 + c) * 32 + lane] = y[j][c];
  __syncthreads();
  const bool leader = (kw == 0) && (EPI != EPI_SWIGLU || which == 0);
  if (!leader || !tile_ok) return;
#pragma unroll
  for (int j = 0; j < NT8; ++j)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float v = 0.f, v2 = 0.f;
#pragma unroll
      for (int w = 0; w < WK; ++w) {
        v += red[((rt * WK + w) * NT8 * 4 + j * 4 + c) * 32 + lane];
        if (EPI == EPI_SWIGLU) v2 += red[(((rt + 1) * WK + w) * NT8 * 4 + j * 4 + c) * 32 + lane];
      }
      const int row = n0 + g + 8 * (c >> 1);
      const int tok = 8 * j + 2 * t + (c & 1);
      if (tok >= M) continue;
      const size_t o = (size_t)orow(tok) * N + row;
      if (EPI == EPI_SWIGLU) {
        const float gv = round_bf(v), uv = round_bf(v2);
        a.y[o] = f2bf(gv / (1.0f + expf(-gv)) * uv);
      } else {
        if (a.y_f32) a.y_f32[o] = v;
        if (a.y) {
          uint16_t r = f2bf(v);
          if (a.residual) r = f2bf(bf2f(r) + bf2f(a.residual[o]));
          a.y[o] = r;
        }
      }
    }
}

// K-split ways per row tile forced through higgs_set_option("gemv_wk", 1|2|4|8); 0 = heuristic
int g_force_wk = 0;

template <int NT8, int WK, int EPI, int S, bool XSMEM, bool NORM, bool F16, bool GATHER, bool ONE>
cudaError_t launch_cfg(const QLinArgs& a, int ctas, size_t smem, cudaStream_t st) {
  auto k = qgemv_ring_kernel<NT8, WK, EPI, S, XSMEM, NORM, F16, GATHER, ONE>;
  static PerDeviceOnce attr;
  const cudaError_t e =
      attr.run([&] { return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024); });
  if (e != cudaSuccess) return e;
  return launch_pdl(k, dim3(ctas, GATHER ? a.moe_max_items : 1), dim3(256), smem, st, a);
}

template <int NT8, int EPI, int S, bool XSMEM, bool NORM, bool F16, bool GATHER = false, bool ONE = false>
cudaError_t launch_wk(const QLinArgs& a, cudaStream_t st) {
  const int nrt = a.N / 16;
  const int units = a.K / 256;
  const int mt = GATHER ? 8 : a.M;  // a grouped item holds up to 8 pairs
  const size_t xs_bytes = XSMEM ? xfrag_bytes(mt, a.K) + 2 * (size_t)(a.K / 64) * 8 * NT8 * 4 : 0;
  const size_t ring = (size_t)8 * S * kStage;
  const size_t red = (size_t)8 * NT8 * 4 * 32 * 4;
  const size_t smem = (ring + xs_bytes) > red ? ring + xs_bytes : red;
  int per_sm = (int)((227 * 1024) / (smem + 1024));
  if (per_sm > 3) per_sm = 3;
  if (per_sm < 1) per_sm = 1;
  const int slots = per_sm * sm_count();
  // row tiles competing for the slots (grouped experts: every work item's tiles)
  const long long work = (long long)nrt * (GATHER ? a.moe_max_items : 1);
  // largest row-tile count per CTA that still fills the slots; every warp keeps >= 1 unit
  int wk;
  if (EPI == EPI_SWIGLU) {
    wk = 4;  // 2 warp tiles (one gate/up pair) per CTA
    if ((work + 1) / 2 >= slots && units >= 2) wk = 2;
    if ((work + 3) / 4 >= slots) wk = 1;
    if (g_force_wk == 1 || g_force_wk == 2 || g_force_wk == 4) wk = g_force_wk;
    while (wk > 1 && units < wk) wk >>= 1;
    if (wk > 4) wk = 4;
    const int rot = (8 / wk) / 2;
    const int ctas = (nrt + rot - 1) / rot;
    if (wk == 4) return launch_cfg<NT8, 4, EPI, S, XSMEM, NORM, F16, GATHER, ONE>(a, ctas, smem, st);
    if (wk == 2) return launch_cfg<NT8, 2, EPI, S, XSMEM, NORM, F16, GATHER, ONE>(a, ctas, smem, st);
    return launch_cfg<NT8, 1, EPI, S, XSMEM, NORM, F16, GATHER, ONE>(a, ctas, smem, st);
  }
  // measured on B200 (M=1): K split 8 ways while the tiles alone cannot fill the
  // slots, else 4 ways -- more CTAs beat fewer fatter ones even for the LM head
  wk = (work / 2 >= slots) ? 4 : 8;
  // very wide outputs (the LM head: ~9.5k row tiles): fewer K splits, fatter warps
  // (measured, N = 151936: M=1 wk 2 103.7 vs 106.7 us; M=8 wk 1 129.6 vs 146.6 us)
  if (!GATHER && work >= 16LL * slots) wk = a.M >= 4 ? 1 : 2;
  if (g_force_wk > 0) wk = g_force_wk;
  while (wk > 1 && units < wk) wk >>= 1;
  const int rot = 8 / wk;
  const int ctas = (nrt + rot - 1) / rot;
  switch (wk) {
    case 8: return launch_cfg<NT8, 8, EPI, S, XSMEM, NORM, F16, GATHER, ONE>(a, ctas, smem, st);
    case 4: return launch_cfg<NT8, 4, EPI, S, XSMEM, NORM, F16, GATHER, ONE>(a, ctas, smem, st);
    case 2: return launch_cfg<NT8, 2, EPI, S, XSMEM, NORM, F16, GATHER, ONE>(a, ctas, smem, st);
    default: return launch_cfg<NT8, 1, EPI, S, XSMEM, NORM, F16, GATHER, ONE>(a, ctas, smem, st);
  }
}

// fragment format of the shared-memory x path (bf16 by default; fp16 selectable
// for measurement through higgs_set_option)
bool g_gemv_f16 = false;

template <int EPI>
cudaError_t launch_epi(const QLinArgs& a, cudaStream_t st) {
  const bool xsmem = a.M <= 8 && xfrag_bytes(a.M, a.K) <= g_xsmem_max;
  if (a.M <= 8) {
    if (g_gemv_f16) {
      if (a.norm_w) return launch_wk<1, EPI, 3, true, true, true>(a, st);
      if (xsmem) return launch_wk<1, EPI, 3, true, false, true>(a, st);
    } else {
      if (a.M == 1) {  // one token: fold only its outputs
        if (a.norm_w) return launch_wk<1, EPI, 3, true, true, false, false, true>(a, st);
        if (xsmem) return launch_wk<1, EPI, 3, true, false, false, false, true>(a, st);
      }
      if (a.norm_w) return launch_wk<1, EPI, 3, true, true, false>(a, st);
      if (xsmem) return launch_wk<1, EPI, 3, true, false, false>(a, st);
    }
    return launch_wk<1, EPI, 3, false, false, false>(a, st);
  }
  if (a.M <= 16) return launch_wk<2, EPI, 3, false, false, false>(a, st);
  return launch_wk<4, EPI, 3, false, false, false>(a, st);
}

}  // namespace

// M rows per pass: <= 32 (a fused norm needs M <= 8 and the x tile in shared memory).
bool qgemv_ring_can_fuse_norm(int M, int K);
static bool g_gemm_tc = true;  // route M >= g_gemm_tc_rows to the tensor-core path
static int g_gemm_tc_rows = 17;
void set_gemm_tc(bool on) { g_gemm_tc = on; }
void set_gemm_tc_rows(int m) { g_gemm_tc_rows = m < 1 ? 1 : m; }

cudaError_t launch_qgemv_ring(const QLinArgs& a, int epi, cudaStream_t st) {
  if (a.norm_w && !qgemv_ring_can_fuse_norm(a.M, a.K)) return cudaErrorInvalidValue;
  if (g_gemm_tc && a.M >= g_gemm_tc_rows && qgemm_tc_supported(a))
    return launch_qgemm_tc(a, epi, a.tc_ws, a.tc_ws_bytes, st);
  if (a.tp_push || a.tp_pull)  // the fused tensor-parallel sum lives in the register-fed kernel
    return (a.M == 1 && qgemv_m1_supported(a)) ? launch_qgemv_m1(a, epi, st) : cudaErrorInvalidValue;
  if (a.M == 1 && qgemv_tma_supported(a)) return launch_qgemv_tma(a, epi, st);  // qgemv_tma.cu
  if (a.M == 1 && qgemv_m1_supported(a)) return launch_qgemv_m1(a, epi, st);    // qgemv_m1.cu
  QLinArgs c = a;
  for (int m0 = 0; m0 < a.M; m0 += 32) {
    c.M = (a.M - m0) < 32 ? (a.M - m0) : 32;
    c.x = a.x + (size_t)m0 * a.K;
    if (a.y) c.y = a.y + (size_t)m0 * a.N;
    if (a.y_f32) c.y_f32 = a.y_f32 + (size_t)m0 * a.N;
    if (a.residual) c.residual = a.residual + (size_t)m0 * a.N;
    cudaError_t e = epi == EPI_SWIGLU ? launch_epi<EPI_SWIGLU>(c, st) : launch_epi<EPI_STORE>(c, st);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

bool qgemv_ring_can_fuse_norm(int M, int K) { return M <= 8 && xfrag_bytes(M, K) <= g_xsmem_max; }
void qgemv_set_xsmem_max(int bytes) {
  g_xsmem_max = bytes < 0 ? 0 : ((size_t)bytes > kXsmemGroupedMax ? kXsmemGroupedMax : (size_t)bytes);
}

// Grouped-expert GEMV over a routing plan (a.moe_* set, a.M ignored): one
// grid row per potential work item, items past the plan's count exit at once.
bool qgemv_grouped_supported(int K) { return xfrag_bytes(8, K) <= kXsmemGroupedMax; }
cudaError_t launch_qgemv_grouped(const QLinArgs& a, int epi, cudaStream_t st) {
  if (!qgemv_grouped_supported(a.K) || a.moe_max_items <= 0 || a.moe_max_items > 65535)
    return cudaErrorInvalidValue;
  return epi == EPI_SWIGLU ? launch_wk<1, EPI_SWIGLU, 3, true, false, false, true>(a, st)
                           : launch_wk<1, EPI_STORE, 3, true, false, false, true>(a, st);
}

void qgemv_set_f16(bool on) { g_gemv_f16 = on; }
void qgemv_set_wk(int wk) { g_force_wk = (wk == 1 || wk == 2 || wk == 4 || wk == 8) ? wk : 0; }

// L2 prefetch of GEMV weights: bit 0 = the step's next GEMV, bit 1 = each CTA's
// own tiles.  Off by default: measured on B200 it lengthened the decode step.
static int g_l2_prefetch = 0;
void set_l2_prefetch(int mode) { g_l2_prefetch = mode & 3; }
bool l2_prefetch_next() { return (g_l2_prefetch & 1) != 0; }
bool l2_prefetch_self() { return (g_l2_prefetch & 2) != 0; }

}  // namespace higgs
