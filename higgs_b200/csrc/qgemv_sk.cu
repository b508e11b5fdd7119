// qgemv_sk.cu -- stream-K W4 g64 GEMV for decode batches (M <= 8), with the
// preceding RMSNorm optionally fused into its prologue.
//
// Reference ops replaced: ops::quantized_matmul (qwen3_next.rs:174-183) and,
// when fused, the nn::RmsNorm before it (transformer.rs:407, 415).
//
// Work decomposition: the weight matrix is cut into 16-row tiles x 256-wide K
// units.  A persistent grid (2 CTAs per SM, 8 warps each) gives every warp an
// equal, contiguous range of (tile, unit) work, so each SM streams the same
// number of weight bytes whatever N is -- no partial last wave.  A warp's range
// covers pieces of at most a few tiles; for each piece it writes its f32
// partial sums to a dedicated scratch slot and bumps the tile's counter; the
// warp that completes a tile sums the slots in slot order (deterministic) and
// applies the epilogue (bf16 / f32 store, residual add, or SwiGLU of the
// gate/up tile pair), then resets the counter.
//
// Per-unit arithmetic is the one of qlinear.cu: rows g and g+8 of a tile as
// 8-byte words, nibbles -> exact bf16 (128 + q) with one LOP3 per pair,
// mma.sync m16n8k16 with the weights as A, sum(x) from an all-ones A tile, and
// the per-group f32 fold y += s*acc + (b - 128 s)*sum(x).
//
// The first two units of a warp's range are fetched before griddepcontrol.wait,
// and dependents are released right after it, so consecutive kernels overlap
// their weight streams with the previous kernel's tail.
#include <algorithm>
#include <string>

#include "common.cuh"
#include "kernels.cuh"

namespace higgs {

namespace {

struct WUnitSk {
  uint2 w0[4];
  uint2 w1[4];
  uint2 s0, s1, b0, b1;
};

__device__ __forceinline__ void sk_load(WUnitSk& u, const uint32_t* W, const uint16_t* S,
                                        const uint16_t* Bi, int r0, int KW, int G, int unit,
                                        int t) {
  const uint32_t* wr0 = W + (size_t)r0 * KW + unit * 32 + 2 * t;
  const uint32_t* wr1 = wr0 + (size_t)8 * KW;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    u.w0[i] = ldg_stream_u2(wr0 + i * 8);
    u.w1[i] = ldg_stream_u2(wr1 + i * 8);
  }
  const uint16_t* s0 = S + (size_t)r0 * G + unit * 4;
  const uint16_t* b0 = Bi + (size_t)r0 * G + unit * 4;
  u.s0 = ldg_stream_u2(s0);
  u.s1 = ldg_stream_u2(s0 + (size_t)8 * G);
  u.b0 = ldg_stream_u2(b0);
  u.b1 = ldg_stream_u2(b0 + (size_t)8 * G);
}

struct TilePtr {
  const uint32_t* W;
  const uint16_t* S;
  const uint16_t* B;
  int r0;  // row of lane-group g within the segment
};

__device__ __forceinline__ TilePtr tile_ptr(const SkArgs& a, int tt, int g) {
  TilePtr p;
  if (a.swiglu) {
    const int which = tt & 1;
    p.W = which ? a.wseg[1] : a.wseg[0];
    p.S = which ? a.sseg[1] : a.sseg[0];
    p.B = which ? a.bseg[1] : a.bseg[0];
    p.r0 = (tt >> 1) * 16 + g;
    return p;
  }
  const int row = tt * 16;
  int seg = 0, base = 0;
#pragma unroll
  for (int i = 1; i < 3; ++i)
    if (i < a.nseg && row >= a.seg_end[i - 1]) {
      seg = i;
      base = a.seg_end[i - 1];
    }
  p.W = a.wseg[seg];
  p.S = a.sseg[seg];
  p.B = a.bseg[seg];
  p.r0 = row - base + g;
  return p;
}

// first warp whose range contains unit x (ranges are [floor(T*w/W), floor(T*(w+1)/W)))
__device__ __forceinline__ int warp_of_unit(int64_t x, int64_t W, int64_t T) {
  return (int)(((x + 1) * W + T - 1) / T) - 1;
}

template <bool NORM>
__global__ void __launch_bounds__(256, 2) qgemv_sk_kernel(SkArgs a) {
  extern __shared__ __align__(16) uint16_t xs[];  // NORM: [M][K + 8] bf16
  __shared__ float red[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int K = a.K, M = a.M;
  const int KW = K / 8, G = K / 64, UPT = K / 256;
  const int64_t T = (int64_t)a.n_tiles * UPT;
  const int64_t W = (int64_t)gridDim.x * 8;
  const int gw = blockIdx.x * 8 + warp;
  const int64_t u0 = T * gw / W, u1 = T * (gw + 1) / W;
  const int XS = K + 8;

  WUnitSk cur, nxt;
  TilePtr tp{};
  if (u0 < u1) {
    tp = tile_ptr(a, (int)(u0 / UPT), g);
    sk_load(cur, tp.W, tp.S, tp.B, tp.r0, KW, G, (int)(u0 % UPT), t);
  }

  pdl_wait();
  pdl_launch();

  if constexpr (NORM) {
    // stage bf16(h * rsqrt(mean(h^2) + eps) * w) for every token, as rmsnorm_kernel does
    const int nv = K / 8;
    for (int m = 0; m < M; ++m) {
      const uint16_t* hr = a.x + (size_t)m * K;
      float ss = 0.0f;
      for (int vi = threadIdx.x; vi < nv; vi += 256) {
        const uint4 v = *reinterpret_cast<const uint4*>(hr + vi * 8);
        const uint32_t* vp = &v.x;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float lo = bf_lo(vp[j]), hi = bf_hi(vp[j]);
          ss += lo * lo + hi * hi;
        }
      }
      ss = warp_sum(ss);
      __syncthreads();
      if (lane == 0) red[warp] = ss;
      __syncthreads();
      float tot = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) tot += red[i];
      const float inv = 1.0f / sqrtf(tot / (float)K + a.eps);
      for (int vi = threadIdx.x; vi < nv; vi += 256) {
        const uint4 v = *reinterpret_cast<const uint4*>(hr + vi * 8);
        const uint4 wv = *reinterpret_cast<const uint4*>(a.norm_w + vi * 8);
        const uint32_t* vp = &v.x;
        const uint32_t* wp = &wv.x;
        uint4 o;
        uint32_t* op = &o.x;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          op[j] = pack_bf2(bf_lo(vp[j]) * inv * bf_lo(wp[j]), bf_hi(vp[j]) * inv * bf_hi(wp[j]));
        *reinterpret_cast<uint4*>(xs + m * XS + vi * 8) = o;
      }
    }
    __syncthreads();
  }

  const uint32_t ONES = 0x3F803F80u;
  float y[4] = {0.f, 0.f, 0.f, 0.f};
  int seg_units = 0;
  for (int64_t u = u0; u < u1; ++u) {
    const int tt = (int)(u / UPT), unit = (int)(u % UPT);
    const bool more = u + 1 < u1;
    const bool tile_end = !more || ((u + 1) / UPT) != tt;
    if (more) {
      TilePtr np = tile_end ? tile_ptr(a, tt + 1, g) : tp;
      sk_load(nxt, np.W, np.S, np.B, np.r0, KW, G, (int)((u + 1) % UPT), t);
      if (tile_end) tp = np;
    }
    const float sg[4] = {bf_lo(cur.s0.x), bf_hi(cur.s0.x), bf_lo(cur.s0.y), bf_hi(cur.s0.y)};
    const float sg8[4] = {bf_lo(cur.s1.x), bf_hi(cur.s1.x), bf_lo(cur.s1.y), bf_hi(cur.s1.y)};
    const float bg[4] = {bf_lo(cur.b0.x), bf_hi(cur.b0.x), bf_lo(cur.b0.y), bf_hi(cur.b0.y)};
    const float bg8[4] = {bf_lo(cur.b1.x), bf_hi(cur.b1.x), bf_lo(cur.b1.y), bf_hi(cur.b1.y)};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int k0 = unit * 256 + i * 64 + 16 * t;
      uint4 X0 = make_uint4(0, 0, 0, 0), X1 = make_uint4(0, 0, 0, 0);
      if (g < M) {
        if constexpr (NORM) {
          X0 = *reinterpret_cast<const uint4*>(xs + g * XS + k0);
          X1 = *reinterpret_cast<const uint4*>(xs + g * XS + k0 + 8);
        } else {
          const uint16_t* xp = a.x + (size_t)g * K + k0;
          X0 = ldg_u4(xp);
          X1 = ldg_u4(xp + 8);
        }
      }
      const uint32_t wA = cur.w0[i].x, wB = cur.w0[i].y;
      const uint32_t wC = cur.w1[i].x, wD = cur.w1[i].y;
      const uint32_t A[4][4] = {
          {nib_pair_bf16<0>(wA), nib_pair_bf16<0>(wC), nib_pair_bf16<4>(wA), nib_pair_bf16<4>(wC)},
          {nib_pair_bf16<8>(wA), nib_pair_bf16<8>(wC), nib_pair_bf16<12>(wA), nib_pair_bf16<12>(wC)},
          {nib_pair_bf16<0>(wB), nib_pair_bf16<0>(wD), nib_pair_bf16<4>(wB), nib_pair_bf16<4>(wD)},
          {nib_pair_bf16<8>(wB), nib_pair_bf16<8>(wD), nib_pair_bf16<12>(wB), nib_pair_bf16<12>(wD)}};
      const uint32_t Bf[4][2] = {{prmt(X0.x, X0.z, 0x5410), prmt(X0.x, X0.z, 0x7632)},
                                 {prmt(X0.y, X0.w, 0x5410), prmt(X0.y, X0.w, 0x7632)},
                                 {prmt(X1.x, X1.z, 0x5410), prmt(X1.x, X1.z, 0x7632)},
                                 {prmt(X1.y, X1.w, 0x5410), prmt(X1.y, X1.w, 0x7632)}};
      float acc[4] = {0.f, 0.f, 0.f, 0.f}, xsum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kt = 0; kt < 4; ++kt) {
        mma_bf16_16816(acc, A[kt][0], A[kt][1], A[kt][2], A[kt][3], Bf[kt][0], Bf[kt][1]);
        mma_bf16_16816(xsum, ONES, ONES, ONES, ONES, Bf[kt][0], Bf[kt][1]);
      }
      const float bb0 = fmaf(-128.0f, sg[i], bg[i]);
      const float bb1 = fmaf(-128.0f, sg8[i], bg8[i]);
      y[0] = fmaf(sg[i], acc[0], fmaf(bb0, xsum[0], y[0]));
      y[1] = fmaf(sg[i], acc[1], fmaf(bb0, xsum[1], y[1]));
      y[2] = fmaf(sg8[i], acc[2], fmaf(bb1, xsum[2], y[2]));
      y[3] = fmaf(sg8[i], acc[3], fmaf(bb1, xsum[3], y[3]));
    }
    ++seg_units;
    if (tile_end) {
      // partial -> slot (gw - first warp of this tile)
      const int slot = gw - warp_of_unit((int64_t)tt * UPT, W, T);
      float* part = a.partials + ((size_t)tt * a.max_slots + slot) * 16 * 8;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int tok = 2 * t + (c & 1);
        if (tok < M) part[tok * 16 + g + 8 * (c >> 1)] = y[c];
      }
      __threadfence();
      __syncwarp();
      const int out_tile = a.swiglu ? (tt >> 1) : tt;
      const int target = a.swiglu ? 2 * UPT : UPT;
      int done = 0;
      if (lane == 0) done = (atomicAdd(a.counters + out_tile, seg_units) + seg_units == target);
      done = __shfl_sync(0xffffffffu, done, 0);
      if (done) {
        __threadfence();
        // sum every slot of the tile(s) in slot order
        float v[4] = {0.f, 0.f, 0.f, 0.f}, v2[4] = {0.f, 0.f, 0.f, 0.f};
        const int n_parts = a.swiglu ? 2 : 1;
        for (int pi = 0; pi < n_parts; ++pi) {
          const int ti = a.swiglu ? out_tile * 2 + pi : tt;
          // the owners of the tile's units, in unit order (each owner once)
          const int s_first = warp_of_unit((int64_t)ti * UPT, W, T);
          int prev = -1;
          for (int ux = 0; ux < UPT; ++ux) {
            const int owner = warp_of_unit((int64_t)ti * UPT + ux, W, T);
            if (owner == prev) continue;
            prev = owner;
            const int sl = owner - s_first;
            const float* pp = a.partials + ((size_t)ti * a.max_slots + sl) * 16 * 8;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const int tok = 2 * t + (c & 1);
              if (tok < M) {
                const float pv = __ldcg(pp + tok * 16 + g + 8 * (c >> 1));
                if (pi == 0)
                  v[c] += pv;
                else
                  v2[c] += pv;
              }
            }
          }
        }
        if (lane == 0) a.counters[out_tile] = 0;
        const int n0 = out_tile * 16;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int tok = 2 * t + (c & 1);
          if (tok >= M) continue;
          const int row = n0 + g + 8 * (c >> 1);
          const size_t o = (size_t)tok * a.N + row;
          if (a.swiglu) {
            const float gv = round_bf(v[c]), uv = round_bf(v2[c]);
            a.y[o] = f2bf(gv / (1.0f + expf(-gv)) * uv);
          } else {
            if (a.y_f32) a.y_f32[o] = v[c];
            if (a.y) {
              uint16_t r = f2bf(v[c]);
              if (a.residual) r = f2bf(bf2f(r) + bf2f(a.residual[o]));
              a.y[o] = r;
            }
          }
        }
      }
      y[0] = y[1] = y[2] = y[3] = 0.f;
      seg_units = 0;
    }
    if (more) cur = nxt;
  }
}

}  // namespace

static int sk_grid(int n_tiles, int K) {
  const int64_t T = (int64_t)n_tiles * (K / 256);
  int64_t grid = 2 * (int64_t)sm_count();
  const int64_t need = (T + 7) / 8;  // at least one unit per warp
  if (need < grid) grid = need;
  return (int)(grid < 1 ? 1 : grid);
}

static int sk_max_slots(int n_tiles, int K, int grid) {
  const int64_t T = (int64_t)n_tiles * (K / 256);
  const int64_t W = (int64_t)grid * 8;
  const int64_t upt = K / 256;
  return (int)((upt * W + T - 1) / T) + 2;
}

// Workspace: a fixed counter region (one int per tile, up to kSkMaxTiles, kept
// zero between calls) followed by the partial-sum slots.  The fixed size lets
// GEMVs of different shapes share one workspace back to back.
constexpr int kSkMaxTiles = 16384;
constexpr size_t kSkCounterBytes = kSkMaxTiles * sizeof(int);

size_t qgemv_sk_workspace(int M, int K, int n_tiles) {
  const int grid = sk_grid(n_tiles, K);
  const size_t parts = (size_t)n_tiles * sk_max_slots(n_tiles, K, grid) * 16 * 8 * sizeof(float);
  return kSkCounterBytes + parts;
}

cudaError_t launch_qgemv_sk(SkArgs a, void* workspace, cudaStream_t st) {
  if (a.n_tiles > kSkMaxTiles) return cudaErrorInvalidValue;
  const int grid = sk_grid(a.n_tiles, a.K);
  a.max_slots = sk_max_slots(a.n_tiles, a.K, grid);
  char* ws = (char*)workspace;
  a.counters = (int*)ws;
  a.partials = (float*)(ws + kSkCounterBytes);
  if (a.norm_w) {
    const size_t smem = (size_t)a.M * (a.K + 8) * 2;
    static PerDeviceOnce attr;
    const cudaError_t e = attr.run([] {
      return cudaFuncSetAttribute(qgemv_sk_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  8 * (8192 + 8) * 2);
    });
    if (e != cudaSuccess) return e;
    return launch_pdl(qgemv_sk_kernel<true>, dim3(grid), dim3(256), smem, st, a);
  }
  return launch_pdl(qgemv_sk_kernel<false>, dim3(grid), dim3(256), 0, st, a);
}

}  // namespace higgs

using namespace higgs;

extern "C" size_t higgs_qlinear_sk_workspace_size(int M, int K, int N_rows) {
  if (M <= 0 || K <= 0 || K % 256 || N_rows <= 0 || N_rows % 16) return 0;
  if (M > 8)  // the tensor-core path: the same counter region, then its partial tiles
    return std::max({kSkCounterBytes, qgemm_tc_workspace(M, K, N_rows, false),
                     qgemm_tc_workspace(M, K, N_rows / 2, true)});
  return qgemv_sk_workspace(M, K, N_rows / 16);
}

// M > 8 rows without a fused norm: the ring GEMV (< 17 rows) or the tensor-core
// matmul, which splits K over this workspace when its tiles alone cannot fill the GPU.
static int wide_qlinear(const char* fn, QLinArgs a, int epi, void* workspace, size_t workspace_bytes,
                        void* stream) {
  const size_t need = higgs_qlinear_sk_workspace_size(a.M, a.K, epi == EPI_SWIGLU ? 2 * a.N : a.N);
  if (workspace_bytes < need)
    return fail(HIGGS_ERR_WORKSPACE,
                std::string(fn) + ": workspace too small (need " + std::to_string(need) + " bytes)");
  a.tc_ws = workspace;
  a.tc_ws_bytes = workspace_bytes;
  HG_CUDA(launch_qgemv_ring(a, epi, (cudaStream_t)stream));
  return HIGGS_OK;
}

extern "C" int higgs_rmsnorm_qlinear_w4g64(higgs_ctx* ctx, const void* x, int M, int K,
                                           const void* norm_w, float eps, const uint32_t* w,
                                           const void* scales, const void* biases, int N, void* y,
                                           float* y_f32, const void* residual, void* workspace,
                                           size_t workspace_bytes, void* stream) {
  HG_CHECK_ARG(ctx && x && w && scales && biases && workspace, "higgs_rmsnorm_qlinear_w4g64: null argument");
  HG_CHECK_ARG(y || y_f32, "higgs_rmsnorm_qlinear_w4g64: need y or y_f32");
  HG_CHECK_ARG(M >= 1 && (M <= 8 || !norm_w), "higgs_rmsnorm_qlinear_w4g64: fused norm needs M in [1, 8]");
  HG_CHECK_ARG(K % 256 == 0 && N % 16 == 0 && N > 0, "higgs_rmsnorm_qlinear_w4g64: need K % 256 == 0, N % 16 == 0");
  HG_CHECK_ARG(!residual || y, "higgs_rmsnorm_qlinear_w4g64: residual needs a bf16 y");
  HG_DEVICE(ctx);
  if (M > 8) {
    QLinArgs q = {};
    q.x = (const uint16_t*)x;
    q.M = M;
    q.K = K;
    q.N = N;
    q.w = w;
    q.s = (const uint16_t*)scales;
    q.b = (const uint16_t*)biases;
    q.y = (uint16_t*)y;
    q.y_f32 = y_f32;
    q.residual = (const uint16_t*)residual;
    return wide_qlinear("higgs_rmsnorm_qlinear_w4g64", q, EPI_STORE, workspace, workspace_bytes, stream);
  }
  HG_CHECK_ARG(!norm_w || K <= 8192, "higgs_rmsnorm_qlinear_w4g64: fused norm needs K <= 8192");
  HG_CHECK_ARG(N / 16 <= kSkMaxTiles, "higgs_rmsnorm_qlinear_w4g64: N must be <= 262144");
  const size_t need = qgemv_sk_workspace(M, K, N / 16);
  if (workspace_bytes < need)
    return fail(HIGGS_ERR_WORKSPACE, "higgs_rmsnorm_qlinear_w4g64: workspace too small (need " +
                                         std::to_string(need) + " bytes)");
  if (M == 1) {  // one token: the register-fed GEMV (no workspace use)
    QLinArgs q = {};
    q.x = (const uint16_t*)x;
    q.M = 1;
    q.K = K;
    q.N = N;
    q.w = w;
    q.s = (const uint16_t*)scales;
    q.b = (const uint16_t*)biases;
    q.y = (uint16_t*)y;
    q.y_f32 = y_f32;
    q.residual = (const uint16_t*)residual;
    q.norm_w = (const uint16_t*)norm_w;
    q.eps = eps;
    if (qgemv_tma_supported(q)) {
      HG_CUDA(launch_qgemv_tma(q, EPI_STORE, (cudaStream_t)stream));
      return HIGGS_OK;
    }
    if (qgemv_m1_supported(q)) {
      HG_CUDA(launch_qgemv_m1(q, EPI_STORE, (cudaStream_t)stream));
      return HIGGS_OK;
    }
  }
  SkArgs a{};
  a.x = (const uint16_t*)x;
  a.norm_w = (const uint16_t*)norm_w;
  a.eps = eps;
  a.M = M;
  a.K = K;
  a.N = N;
  a.n_tiles = N / 16;
  a.nseg = 1;
  a.seg_end[0] = N;
  a.wseg[0] = w;
  a.sseg[0] = (const uint16_t*)scales;
  a.bseg[0] = (const uint16_t*)biases;
  a.y = (uint16_t*)y;
  a.y_f32 = y_f32;
  a.residual = (const uint16_t*)residual;
  HG_CUDA(launch_qgemv_sk(a, workspace, (cudaStream_t)stream));
  return HIGGS_OK;
}

extern "C" int higgs_rmsnorm_gate_up_swiglu(higgs_ctx* ctx, const void* x, int M, int K,
                                            const void* norm_w, float eps, const uint32_t* w_gate,
                                            const void* s_gate, const void* b_gate,
                                            const uint32_t* w_up, const void* s_up,
                                            const void* b_up, int N, void* y, void* workspace,
                                            size_t workspace_bytes, void* stream) {
  HG_CHECK_ARG(ctx && x && w_gate && s_gate && b_gate && w_up && s_up && b_up && y && workspace,
               "higgs_rmsnorm_gate_up_swiglu: null argument");
  HG_CHECK_ARG(M >= 1 && (M <= 8 || !norm_w), "higgs_rmsnorm_gate_up_swiglu: fused norm needs M in [1, 8]");
  HG_CHECK_ARG(K % 256 == 0 && N % 16 == 0 && N > 0, "higgs_rmsnorm_gate_up_swiglu: need K % 256 == 0, N % 16 == 0");
  HG_DEVICE(ctx);
  if (M > 8) {
    QLinArgs q = {};
    q.x = (const uint16_t*)x;
    q.M = M;
    q.K = K;
    q.N = N;
    q.w = w_gate;
    q.s = (const uint16_t*)s_gate;
    q.b = (const uint16_t*)b_gate;
    q.w2 = w_up;
    q.s2 = (const uint16_t*)s_up;
    q.b2 = (const uint16_t*)b_up;
    q.y = (uint16_t*)y;
    return wide_qlinear("higgs_rmsnorm_gate_up_swiglu", q, EPI_SWIGLU, workspace, workspace_bytes, stream);
  }
  HG_CHECK_ARG(!norm_w || K <= 8192, "higgs_rmsnorm_gate_up_swiglu: fused norm needs K <= 8192");
  HG_CHECK_ARG(2 * N / 16 <= kSkMaxTiles, "higgs_rmsnorm_gate_up_swiglu: N must be <= 131072");
  const size_t need = qgemv_sk_workspace(M, K, 2 * N / 16);
  if (workspace_bytes < need)
    return fail(HIGGS_ERR_WORKSPACE, "higgs_rmsnorm_gate_up_swiglu: workspace too small (need " +
                                         std::to_string(need) + " bytes)");
  if (M == 1) {  // one token: the register-fed GEMV (no workspace use)
    QLinArgs q = {};
    q.x = (const uint16_t*)x;
    q.M = 1;
    q.K = K;
    q.N = N;
    q.w = w_gate;
    q.s = (const uint16_t*)s_gate;
    q.b = (const uint16_t*)b_gate;
    q.w2 = w_up;
    q.s2 = (const uint16_t*)s_up;
    q.b2 = (const uint16_t*)b_up;
    q.y = (uint16_t*)y;
    q.norm_w = (const uint16_t*)norm_w;
    q.eps = eps;
    if (qgemv_tma_supported(q)) {
      HG_CUDA(launch_qgemv_tma(q, EPI_SWIGLU, (cudaStream_t)stream));
      return HIGGS_OK;
    }
    if (qgemv_m1_supported(q)) {
      HG_CUDA(launch_qgemv_m1(q, EPI_SWIGLU, (cudaStream_t)stream));
      return HIGGS_OK;
    }
  }
  SkArgs a{};
  a.x = (const uint16_t*)x;
  a.norm_w = (const uint16_t*)norm_w;
  a.eps = eps;
  a.M = M;
  a.K = K;
  a.N = N;
  a.n_tiles = 2 * N / 16;
  a.swiglu = 1;
  a.nseg = 2;
  a.wseg[0] = w_gate;
  a.sseg[0] = (const uint16_t*)s_gate;
  a.bseg[0] = (const uint16_t*)b_gate;
  a.wseg[1] = w_up;
  a.sseg[1] = (const uint16_t*)s_up;
  a.bseg[1] = (const uint16_t*)b_up;
  a.y = (uint16_t*)y;
  HG_CUDA(launch_qgemv_sk(a, workspace, (cudaStream_t)stream));
  return HIGGS_OK;
}
