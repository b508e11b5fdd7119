// qgemv_tma.cu -- W4 g64 GEMV for a single token with the weights streamed by
// TMA into a shared-memory ring.
//
// Reference op replaced: ops::quantized_matmul (qwen3_next.rs:174-183) at one
// token, with the preceding nn::RmsNorm (transformer.rs:407, 415) optionally fused.
//
// The arithmetic is the single-token GEMV's (qgemv_m1.cu): a warp owns 16 rows
// and a K range in units of 256, codes enter mma.sync m16n8k16 as the exact bf16
// values 128 + q, the idle MMA columns keep the quantization groups apart, and one
// fold y += s * acc + (b - 128 s) * sum(x) per unit pair.  What changes is how the
// weights arrive.  Loaded into registers, a warp keeps two units in flight and the
// SM streams ~30 KB at a time: at HBM latency that is a third of the bandwidth.
// Here one producer warp per CTA issues cp.async.bulk.tensor loads of every
// consumer warp's next unit pair (codes, scales, biases) into a 2-stage ring of
// 36 KB stages, two CTAs per SM: up to 144 KB per SM in flight, independent of
// the consumers' registers.  CTAs are persistent (at most two per SM) and walk
// the tile groups round-robin; the producer runs ahead across group boundaries,
// so the stream does not drain between groups.  The first stages are issued
// before the grid dependency wait (weights never depend on the previous kernel).
// Every mbarrier wait is bounded (about 2 s): on timeout the kernel records an
// error (higgs_tc_error) and finishes.
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

constexpr int kTwConsumers = 8;                       // consumer warps per CTA
constexpr int kTwThreads = (kTwConsumers + 1) * 32;   // + the producer warp
constexpr int kTwCtasPerSm = 2;
constexpr int kTwStages = 2;
constexpr int kTwUnit = 16 * 128;                     // 16 rows x 256 k of packed codes
constexpr int kTwSB = 16 * 16;                        // 16 rows x 8 groups of bf16 scales (or biases)
constexpr int kTwSlot = 2 * kTwUnit + 2 * kTwSB;      // a warp's unit pair + scales + biases
constexpr int kTwStage = kTwConsumers * kTwSlot;      // 36 KB
constexpr int kTwMaxK = 12288;

__host__ __device__ inline size_t tw_xf_bytes(int K) { return (size_t)(K / 256) * 512; }
// ring | x fragments | 64 pad | 512 B of zeros | 64 pad | sum(x) per group | reduction [8][16]
inline size_t tw_smem_bytes(int K) {
  return 1024 + (size_t)kTwStages * kTwStage + tw_xf_bytes(K) + 640 + (size_t)(K / 64) * 4 + 8 * 16 * 4;
}

struct TwMaps {
  CUtensorMap w[3], s[3], b[3];  // per row segment (SwiGLU: 0 = gate, 1 = up)
};

struct TwArgs {
  const uint16_t* x;
  const uint16_t* norm_w;
  float eps;
  int K, N, wk, swiglu, nseg;
  int seg_end[3];
  uint16_t* y;
  float* y_f32;
  const uint16_t* residual;
  int* err;
};

__device__ __forceinline__ void tw_mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void tw_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tw_arrive_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool tw_wait(uint64_t* bar, unsigned parity, int* err) {
  const uint32_t a = smem_u32(bar);
  const long long t0 = clock64();
  while (true) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(a), "r"(parity)
        : "memory");
    if (ok) return true;
    if (clock64() - t0 > (1ll << 32)) break;  // ~2 s
  }
  if (err) atomicExch(err, 1);
  return false;
}
__device__ __forceinline__ void tw_tma(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ uint4 tw_lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t tw_lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ void tw_mma(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                       uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint4 tw_frag(uint4 v) {
  return make_uint4(prmt(v.x, v.z, 0x5410), prmt(v.x, v.z, 0x7632), prmt(v.y, v.w, 0x5410),
                    prmt(v.y, v.w, 0x7632));
}
__device__ __forceinline__ void tw_consumers_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kTwConsumers * 32) : "memory");
}

__global__ void __launch_bounds__(kTwThreads, kTwCtasPerSm)
    qgemv_tma_kernel(const __grid_constant__ TwMaps maps, const TwArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t full[kTwStages];
  __shared__ __align__(8) uint64_t empty[kTwStages];
  __shared__ float s_ss[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int K = a.K, N = a.N, WK = a.wk, G = K / 64;
  const int units = K / 256;
  const int RT = 8 / WK, ROT = a.swiglu ? RT / 2 : RT;
  const int n_groups = (N / 16 + ROT - 1) / ROT;
  const int npairs = ((units + WK - 1) / WK + 1) / 2;  // unit pairs per warp and group

  uint8_t* ring = smem;
  uint8_t* xf = smem + kTwStages * kTwStage;
  uint8_t* zero = xf + tw_xf_bytes(K) + 64;
  float* xs = reinterpret_cast<float*>(zero + 576);
  float* red = xs + G;

  // consumer warp w's tile of group grp: (tensor map index, row within it, unit range)
  struct Tile {
    int m, row0, ub, ue;
  };
  auto tile_of = [&](int w, int grp) {
    const int rt = w / WK, kw = w % WK;
    Tile tl;
    int out_tile, which = 0;
    if (a.swiglu) {
      out_tile = grp * ROT + rt / 2;
      which = rt & 1;
    } else {
      out_tile = grp * ROT + rt;
    }
    const int n0 = out_tile * 16;
    const bool ok = n0 < N;
    tl.m = which;
    tl.row0 = ok ? n0 : 0;
    if (!a.swiglu && a.nseg > 1) {
      for (int i = 1; i < a.nseg; ++i)
        if (ok && n0 >= a.seg_end[i - 1]) {
          tl.m = i;
          tl.row0 = n0 - a.seg_end[i - 1];
        }
    }
    tl.ub = ok ? (units * kw) / WK : 0;
    tl.ue = ok ? (units * (kw + 1)) / WK : 0;
    return tl;
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < kTwStages; ++i) {
      tw_mbar_init(&full[i], 1);
      tw_mbar_init(&empty[i], kTwConsumers);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == kTwConsumers) {
    // ---------------- producer: one lane issues every load of the CTA ----------------
    pdl_launch();
    if (lane == 0) {
      int it = 0;
      for (int grp = blockIdx.x; grp < n_groups; grp += gridDim.x) {
        Tile tl[kTwConsumers];
#pragma unroll
        for (int w = 0; w < kTwConsumers; ++w) tl[w] = tile_of(w, grp);
        for (int p = 0; p < npairs; ++p, ++it) {
          const int st = it % kTwStages;
          if (it >= kTwStages) tw_wait(&empty[st], ((it / kTwStages) - 1) & 1, a.err);
          unsigned bytes = 0;
#pragma unroll
          for (int w = 0; w < kTwConsumers; ++w) {
            const int u0 = tl[w].ub + 2 * p;
            if (u0 < tl[w].ue) bytes += kTwUnit + 2 * kTwSB + (u0 + 1 < tl[w].ue ? kTwUnit : 0);
          }
          tw_arrive_tx(&full[st], bytes);
          uint8_t* stage = ring + st * kTwStage;
#pragma unroll
          for (int w = 0; w < kTwConsumers; ++w) {
            const int u0 = tl[w].ub + 2 * p;
            if (u0 >= tl[w].ue) continue;
            uint8_t* slot = stage + w * kTwSlot;
            const int m = tl[w].m;
            tw_tma(slot, &maps.w[m], u0 * 128, tl[w].row0, &full[st]);
            if (u0 + 1 < tl[w].ue) tw_tma(slot + kTwUnit, &maps.w[m], (u0 + 1) * 128, tl[w].row0, &full[st]);
            tw_tma(slot + 2 * kTwUnit, &maps.s[m], 4 * u0, tl[w].row0, &full[st]);
            tw_tma(slot + 2 * kTwUnit + kTwSB, &maps.b[m], 4 * u0, tl[w].row0, &full[st]);
          }
        }
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  uint4 nwr[2];
  const bool norm = a.norm_w != nullptr;
  if (norm) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int c = threadIdx.x + r * 256;
      nwr[r] = c < K / 8 ? *reinterpret_cast<const uint4*>(a.norm_w + 8 * c) : make_uint4(0, 0, 0, 0);
    }
  }
  pdl_wait();
  pdl_launch();
  if (threadIdx.x < 32) reinterpret_cast<uint4*>(zero)[threadIdx.x] = make_uint4(0, 0, 0, 0);
  const uint16_t* x = a.x;
  float inv = 1.0f;
  if (norm) {
    float ss = 0.f;
    for (int c = threadIdx.x; c < K / 8; c += 256) {
      const uint4 v = *reinterpret_cast<const uint4*>(x + 8 * c);
      const uint32_t* vp = &v.x;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float lo = bf_lo(vp[j]), hi = bf_hi(vp[j]);
        ss += lo * lo + hi * hi;
      }
    }
    ss = warp_sum(ss);
    if (lane == 0) s_ss[warp] = ss;
    tw_consumers_sync();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) tot += s_ss[w];
    inv = 1.0f / sqrtf(tot / (float)K + a.eps);
  }
  for (int base = warp * 32, r = 0; base < K / 8; base += 256, ++r) {
    const int c = base + lane;
    uint4 v = *reinterpret_cast<const uint4*>(x + 8 * c);
    if (norm) {
      uint4 wv = r == 0 ? nwr[0] : (r == 1 ? nwr[1] : *reinterpret_cast<const uint4*>(a.norm_w + 8 * c));
      uint32_t* vp = &v.x;
      const uint32_t* wp = &wv.x;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        vp[j] = pack_bf2(bf_lo(vp[j]) * inv * bf_lo(wp[j]), bf_hi(vp[j]) * inv * bf_hi(wp[j]));
    }
    const int u = c >> 5, h = (c >> 4) & 1, tt = (c >> 2) & 3, e = c & 3;
    *reinterpret_cast<uint4*>(xf + ((u * 8 + h * 4 + e) * 4 + tt) * 16) = tw_frag(v);
    const uint32_t* vp = &v.x;
    float x1 = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) x1 += bf_lo(vp[j]) + bf_hi(vp[j]);
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) x1 += __shfl_xor_sync(0xffffffffu, x1, o);
    if ((lane & 7) == 0) xs[c >> 3] = x1;
  }
  tw_consumers_sync();

  const uint32_t xreal = smem_u32(xf) + t * 16;
  const uint32_t xzero = smem_u32(zero);
  const float2* xs2 = reinterpret_cast<const float2*>(xs);
  int it = 0;
  for (int grp = blockIdx.x; grp < n_groups; grp += gridDim.x) {
    const Tile tl = tile_of(warp, grp);
    float yg = 0.f, yg8 = 0.f;
    for (int p = 0; p < npairs; ++p, ++it) {
      const int st = it % kTwStages;
      tw_wait(&full[st], (it / kTwStages) & 1, a.err);
      const int u0 = tl.ub + 2 * p;
      if (u0 < tl.ue) {
        const uint32_t slot = smem_u32(ring + st * kTwStage + warp * kTwSlot);
        float acc[2][4];
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int c = 0; c < 4; ++c) acc[h][c] = 0.f;
#pragma unroll
        for (int d = 0; d < 2; ++d) {
          const int u = u0 + d;
          if (u >= tl.ue) break;
          const uint32_t U = slot + d * kTwUnit;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const bool act = g == 4 * d + 2 * h + (t >> 1);
            const uint32_t xb = (act ? xreal + u * 512 : xzero) + h * 256;
            uint4 xv[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) xv[e] = tw_lds128(xb + e * 64);
            const uint4 wa4 = tw_lds128(U + g * 128 + (t + 4 * h) * 16);
            const uint4 wb4 = tw_lds128(U + (g + 8) * 128 + (t + 4 * h) * 16);
            const uint32_t* wa = &wa4.x;
            const uint32_t* wb = &wb4.x;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const uint32_t A = wa[e], B = wb[e];
              tw_mma(acc[h], nib_pair_bf16<0>(A), nib_pair_bf16<0>(B), nib_pair_bf16<4>(A),
                     nib_pair_bf16<4>(B), xv[e].x, xv[e].y);
              tw_mma(acc[h], nib_pair_bf16<8>(A), nib_pair_bf16<8>(B), nib_pair_bf16<12>(A),
                     nib_pair_bf16<12>(B), xv[e].z, xv[e].w);
            }
          }
        }
        // fold the pair: lane t holds columns 2t, 2t+1 = groups 4 u0 + 2t, +1 (zero past the range)
        const bool ok = u0 + (t >> 1) < tl.ue;
        const uint32_t sc = slot + 2 * kTwUnit;
        const uint32_t q0 = ok ? tw_lds32(sc + g * 16 + t * 4) : 0u;
        const uint32_t q1 = ok ? tw_lds32(sc + (g + 8) * 16 + t * 4) : 0u;
        const uint32_t q2 = ok ? tw_lds32(sc + kTwSB + g * 16 + t * 4) : 0u;
        const uint32_t q3 = ok ? tw_lds32(sc + kTwSB + (g + 8) * 16 + t * 4) : 0u;
        const float2 X = xs2[ok ? 2 * u0 + t : 0];
        const float sa = bf_lo(q0), sb_ = bf_hi(q0), s8a = bf_lo(q1), s8b = bf_hi(q1);
        const float ba = fmaf(-128.0f, sa, bf_lo(q2)), bb = fmaf(-128.0f, sb_, bf_hi(q2));
        const float b8a = fmaf(-128.0f, s8a, bf_lo(q3)), b8b = fmaf(-128.0f, s8b, bf_hi(q3));
        yg = fmaf(sa, acc[0][0] + acc[1][0], fmaf(ba, X.x, yg));
        yg = fmaf(sb_, acc[0][1] + acc[1][1], fmaf(bb, X.y, yg));
        yg8 = fmaf(s8a, acc[0][2] + acc[1][2], fmaf(b8a, X.x, yg8));
        yg8 = fmaf(s8b, acc[0][3] + acc[1][3], fmaf(b8b, X.y, yg8));
      }
      __syncwarp();
      if (lane == 0) tw_arrive(&empty[st]);
    }
    // reduction over the quad, then over the K-split warps
    yg += __shfl_xor_sync(0xffffffffu, yg, 1);
    yg += __shfl_xor_sync(0xffffffffu, yg, 2);
    yg8 += __shfl_xor_sync(0xffffffffu, yg8, 1);
    yg8 += __shfl_xor_sync(0xffffffffu, yg8, 2);
    if (t == 0) {
      red[warp * 16 + g] = yg;
      red[warp * 16 + g + 8] = yg8;
    }
    tw_consumers_sync();
    if ((int)threadIdx.x < ROT * 16) {
      const int r = threadIdx.x >> 4, j = threadIdx.x & 15;
      const int tile = grp * ROT + r;
      const int row = tile * 16 + j;
      if (tile * 16 < N) {
        if (a.swiglu) {
          float vg = 0.f, vu = 0.f;
          for (int w = 0; w < WK; ++w) {
            vg += red[((2 * r) * WK + w) * 16 + j];
            vu += red[((2 * r + 1) * WK + w) * 16 + j];
          }
          const float gv = round_bf(vg), uv = round_bf(vu);
          a.y[row] = f2bf(gv / (1.0f + expf(-gv)) * uv);
        } else {
          float v = 0.f;
          for (int w = 0; w < WK; ++w) v += red[(r * WK + w) * 16 + j];
          if (a.y_f32) a.y_f32[row] = v;
          if (a.y) {
            uint16_t o = f2bf(v);
            if (a.residual) o = f2bf(bf2f(o) + bf2f(a.residual[row]));
            a.y[row] = o;
          }
        }
      }
    }
    tw_consumers_sync();  // red is rewritten by the next group
  }
}

// ---- host side ---------------------------------------------------------------
typedef CUresult (*TwEncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                               const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                               CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

TwEncodeFn tw_encode() {
  static TwEncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<TwEncodeFn>(p);
  });
  return fn;
}

// 2-D map of a row-major [rows, cols] tensor with `elem`-byte elements, box {box_cols, 16 rows}
// (cached by address and shape: capture records the map by value)
bool tw_map(const void* base, int rows, int cols, int elem, int box_cols, CUtensorMap* out) {
  static std::mutex mu;
  static std::map<std::tuple<const void*, int, int, int, int>, CUtensorMap> cache;
  std::lock_guard<std::mutex> lk(mu);
  const auto key = std::make_tuple(base, rows, cols, elem, box_cols);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return true;
  }
  TwEncodeFn fn = tw_encode();
  if (!fn || ((uintptr_t)base & 15) || ((size_t)cols * elem) % 16) return false;
  CUtensorMap m;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * elem};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, 16};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt = elem == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  if (fn(&m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
         CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
      CUDA_SUCCESS)
    return false;
  if (cache.size() > 65536) cache.clear();
  cache[key] = m;
  *out = m;
  return true;
}

// Off by default: measured on B200 it streams no faster than the register-fed kernel -- LM head
// (350 MB) 97.6 vs 88.8 us, gate/up 19.4 vs 18.4 us inside a graph of back-to-back launches,
// B=1 Qwen3-8B step 2.31 vs 2.14 ms; ncu shows both at 42-47 % DRAM throughput with the same
// long-scoreboard-dominated stalls (~4.5 cycles per issued instruction) at ~36 % issue.
bool g_tw_on = false;

// K split for the persistent grid: the smallest per-CTA load, groups x (pairs per warp + 1
// for the group's reduction), among splits whose per-warp ranges hold whole unit pairs.
int tw_pick_wk(int N, int K, bool swiglu, int ctas) {
  const int nrt = N / 16, units = K / 256;
  int best = -1;
  long long best_cost = 0;
  for (int wk = 1; wk <= (swiglu ? 4 : 8); wk *= 2) {
    if (units % (2 * wk) != 0) continue;
    const int rot = swiglu ? (8 / wk) / 2 : 8 / wk;
    const long long groups = (nrt + rot - 1) / rot;
    const long long cost = (groups + ctas - 1) / ctas * ((long long)units / wk / 2 + 1);
    if (best < 0 || cost <= best_cost) {
      best = wk;
      best_cost = cost;
    }
  }
  return best;
}

}  // namespace

bool qgemv_tma_supported(const QLinArgs& a) {
  if (!g_tw_on || a.M != 1 || a.moe_items != nullptr || a.K % 512 != 0 || a.K > kTwMaxK || a.N % 16 != 0)
    return false;
  return tw_pick_wk(a.N, a.K, a.w2 != nullptr, 1) > 0;
}

cudaError_t launch_qgemv_tma(const QLinArgs& q, int epi, cudaStream_t st) {
  if (!qgemv_tma_supported(q)) return cudaErrorInvalidValue;
  const bool swiglu = epi == EPI_SWIGLU;
  TwArgs a;
  memset(&a, 0, sizeof(a));
  a.x = q.x;
  a.norm_w = q.norm_w;
  a.eps = q.eps;
  a.K = q.K;
  a.N = q.N;
  a.swiglu = swiglu;
  a.y = q.y;
  a.y_f32 = q.y_f32;
  a.residual = q.residual;
  a.err = device_state(current_device()).tc_err;
  TwMaps maps;
  memset(&maps, 0, sizeof(maps));
  const int G = q.K / 64;
  auto add = [&](int i, const uint32_t* w, const uint16_t* s, const uint16_t* b, int rows) {
    return tw_map(w, rows, q.K / 2, 1, 128, &maps.w[i]) && tw_map(s, rows, G, 2, 8, &maps.s[i]) &&
           tw_map(b, rows, G, 2, 8, &maps.b[i]);
  };
  if (swiglu) {
    if (!add(0, q.w, q.s, q.b, q.N) || !add(1, q.w2, q.s2, q.b2, q.N)) return cudaErrorInvalidValue;
    a.nseg = 1;
  } else if (q.nseg > 1) {
    a.nseg = q.nseg;
    for (int i = 0; i < q.nseg; ++i) {
      const int r0 = i ? q.seg_end[i - 1] : 0;
      a.seg_end[i] = q.seg_end[i];
      if ((q.seg_end[i] - r0) % 16 || !add(i, q.wseg[i], q.sseg[i], q.bseg[i], q.seg_end[i] - r0))
        return cudaErrorInvalidValue;
    }
  } else {
    a.nseg = 1;
    if (!add(0, q.w, q.s, q.b, q.N)) return cudaErrorInvalidValue;
  }
  const int slots = kTwCtasPerSm * sm_count();
  a.wk = tw_pick_wk(q.N, q.K, swiglu, slots);
  if (a.wk <= 0) return cudaErrorInvalidValue;
  const int rot = swiglu ? (8 / a.wk) / 2 : 8 / a.wk;
  const int groups = (q.N / 16 + rot - 1) / rot;
  const int ctas = std::min(groups, slots);
  const size_t smem = tw_smem_bytes(q.K);
  static PerDeviceOnce attr;
  const cudaError_t e = attr.run([] {
    return cudaFuncSetAttribute(qgemv_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)tw_smem_bytes(kTwMaxK));
  });
  if (e != cudaSuccess) return e;
  return launch_pdl(qgemv_tma_kernel, dim3(ctas), dim3(kTwThreads), smem, st, maps, a);
}

void qgemv_tma_set(int on) { g_tw_on = on != 0; }

}  // namespace higgs
