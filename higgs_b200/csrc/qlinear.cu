// qlinear.cu -- MLX-affine W4 g64 quantized linear layers for decode (M <= 32
// rows per pass), embedding gather-dequant and plain dequantize.
//
// Reference ops replaced: ops::quantized_matmul (qwen3_next.rs:174-183),
// ops::dequantize + take (qwen3_next.rs:248-257), swiglu (qwen3_next.rs:275-277).
//
// GEMV design (HBM-bound at decode sizes):
//  * weights are read straight from the MLX layout (u32 [N, K/8]): each lane
//    of a warp streams two 8-byte words per 64-wide group for rows g and g+8 of
//    a 16-row tile; the four lanes of a row read one 32-byte sector, so every
//    byte fetched is used exactly once;
//  * nibbles become exact bf16 values (128 + q) with one LOP3 per pair and are
//    fed to mma.sync m16n8k16 (weights = A, activations = B) -- the tensor pipe
//    does the multiply-adds so the ALUs only unpack;
//  * the group scale and bias are folded in f32 per group exactly as MLX's
//    matrix-vector algorithm does: y += s * sum(x q) + b * sum(x), where
//    sum(x (128 + q)) comes from the weight MMA and sum(x) from an MMA against
//    a constant all-ones A tile, so y = s*acc + (b - 128 s)*sum(x);
//  * 8 warps per CTA split the K range, reduce through shared memory and apply
//    the epilogue (bf16 / f32 store, residual add, or SwiGLU of a gate/up pair);
//  * programmatic dependent launch: the first weight unit is fetched before
//    griddepcontrol.wait, overlapping the previous kernel's tail.
#include "common.cuh"
#include "kernels.cuh"

namespace higgs {

// One unit = 4 groups = 256 k.  Per lane: rows g and g+8, words 2t and 2t+1 of
// each group (uint2), plus 4 bf16 scales / biases per row (uint2 each).
struct WUnit {
  uint2 w0[4];  // row g, group i
  uint2 w1[4];  // row g + 8, group i
  uint2 s0, s1, b0, b1;
};

__device__ __forceinline__ void load_unit(WUnit& u, const uint32_t* wrow0, const uint32_t* wrow1,
                                          const uint16_t* srow0, const uint16_t* srow1,
                                          const uint16_t* brow0, const uint16_t* brow1, int unit,
                                          int t) {
  const int wofs = unit * 32 + 2 * t;  // u32 words: unit*4 groups*8 words + 2t
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    u.w0[i] = ldg_stream_u2(wrow0 + wofs + i * 8);
    u.w1[i] = ldg_stream_u2(wrow1 + wofs + i * 8);
  }
  u.s0 = ldg_stream_u2(srow0 + unit * 4);
  u.s1 = ldg_stream_u2(srow1 + unit * 4);
  u.b0 = ldg_stream_u2(brow0 + unit * 4);
  u.b1 = ldg_stream_u2(brow1 + unit * 4);
}

template <int NT8, int WK, int EPI>
__global__ void __launch_bounds__(256, (NT8 == 1) ? 2 : 1) qlinear_w4_kernel(QLinArgs a) {
  constexpr int RT = 8 / WK;                      // warp row tiles per CTA
  constexpr int ROT = (EPI == EPI_SWIGLU) ? RT / 2 : RT;  // output row tiles per CTA
  static_assert(EPI != EPI_SWIGLU || RT >= 2, "SwiGLU needs gate/up tile pairs");
  __shared__ float red[8][NT8 * 4][32];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int rt = warp / WK, kw = warp % WK;
  const int K = a.K, N = a.N, M = a.M;
  const int KW = K / 8, G = K / 64;

  int out_tile, which = 0;
  if (EPI == EPI_SWIGLU) {
    out_tile = blockIdx.x * ROT + rt / 2;
    which = rt & 1;
  } else {
    out_tile = blockIdx.x * ROT + rt;
  }
  const int n0 = out_tile * 16;
  const bool tile_ok = n0 < N;
  const uint32_t* W = which ? a.w2 : a.w;
  const uint16_t* S = which ? a.s2 : a.s;
  const uint16_t* Bi = which ? a.b2 : a.b;
  int nbase = 0;  // first row of the segment holding this tile
  if (EPI != EPI_SWIGLU && a.nseg > 1) {
#pragma unroll
    for (int i = 1; i < 3; ++i)
      if (i < a.nseg && n0 >= a.seg_end[i - 1]) {
        W = a.wseg[i];
        S = a.sseg[i];
        Bi = a.bseg[i];
        nbase = a.seg_end[i - 1];
      }
  }
  const int r0 = tile_ok ? n0 - nbase + g : 0, r1 = tile_ok ? n0 - nbase + g + 8 : 0;
  const uint32_t* wrow0 = W + (size_t)r0 * KW;
  const uint32_t* wrow1 = W + (size_t)r1 * KW;
  const uint16_t* srow0 = S + (size_t)r0 * G;
  const uint16_t* srow1 = S + (size_t)r1 * G;
  const uint16_t* brow0 = Bi + (size_t)r0 * G;
  const uint16_t* brow1 = Bi + (size_t)r1 * G;

  const int units = G / 4;
  const int u_begin = (units * kw) / WK, u_end = (units * (kw + 1)) / WK;

  float y[NT8][4];
#pragma unroll
  for (int j = 0; j < NT8; ++j)
#pragma unroll
    for (int c = 0; c < 4; ++c) y[j][c] = 0.0f;

  WUnit cur;
  const bool active = tile_ok && u_begin < u_end;
  if (active) load_unit(cur, wrow0, wrow1, srow0, srow1, brow0, brow1, u_begin, t);

  pdl_wait();  // x / residual may come from the previous kernel

  const uint32_t ONES = 0x3F803F80u;
  if (active) {
    for (int u = u_begin; u < u_end; ++u) {
      WUnit nxt;
      const bool more = (u + 1) < u_end;
      if (more) load_unit(nxt, wrow0, wrow1, srow0, srow1, brow0, brow1, u + 1, t);

      // activations: token 8j+g, k = unit*256 + i*64 + 16t .. +15.  With one
      // token tile the whole unit is fetched up front; wider tiles fetch per
      // group to bound register use.
      constexpr int XG = (NT8 == 1) ? 4 : 1;
      uint4 xa[NT8][XG][2];
      auto load_x = [&](int i, int slot) {
#pragma unroll
        for (int j = 0; j < NT8; ++j) {
          const int tok = 8 * j + g;
          if (tok < M) {
            const uint16_t* xp = a.x + (size_t)tok * K + u * 256 + i * 64 + 16 * t;
            xa[j][slot][0] = ldg_u4(xp);
            xa[j][slot][1] = ldg_u4(xp + 8);
          } else {
            xa[j][slot][0] = make_uint4(0, 0, 0, 0);
            xa[j][slot][1] = make_uint4(0, 0, 0, 0);
          }
        }
      };
      if constexpr (XG == 4) {
#pragma unroll
        for (int i = 0; i < 4; ++i) load_x(i, i);
      }

      const float sg[4] = {bf_lo(cur.s0.x), bf_hi(cur.s0.x), bf_lo(cur.s0.y), bf_hi(cur.s0.y)};
      const float sg8[4] = {bf_lo(cur.s1.x), bf_hi(cur.s1.x), bf_lo(cur.s1.y), bf_hi(cur.s1.y)};
      const float bg[4] = {bf_lo(cur.b0.x), bf_hi(cur.b0.x), bf_lo(cur.b0.y), bf_hi(cur.b0.y)};
      const float bg8[4] = {bf_lo(cur.b1.x), bf_hi(cur.b1.x), bf_lo(cur.b1.y), bf_hi(cur.b1.y)};

#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if constexpr (XG == 1) load_x(i, 0);
        const int xs_slot = (XG == 1) ? 0 : i;
        const uint32_t wA = cur.w0[i].x, wB = cur.w0[i].y;
        const uint32_t wC = cur.w1[i].x, wD = cur.w1[i].y;
        // A fragments of the 4 k16 tiles (see file header for the k mapping)
        const uint32_t A[4][4] = {
            {nib_pair_bf16<0>(wA), nib_pair_bf16<0>(wC), nib_pair_bf16<4>(wA), nib_pair_bf16<4>(wC)},
            {nib_pair_bf16<8>(wA), nib_pair_bf16<8>(wC), nib_pair_bf16<12>(wA), nib_pair_bf16<12>(wC)},
            {nib_pair_bf16<0>(wB), nib_pair_bf16<0>(wD), nib_pair_bf16<4>(wB), nib_pair_bf16<4>(wD)},
            {nib_pair_bf16<8>(wB), nib_pair_bf16<8>(wD), nib_pair_bf16<12>(wB), nib_pair_bf16<12>(wD)}};
        const float bb0 = fmaf(-128.0f, sg[i], bg[i]);
        const float bb1 = fmaf(-128.0f, sg8[i], bg8[i]);
#pragma unroll
        for (int j = 0; j < NT8; ++j) {
          const uint4 X0 = xa[j][xs_slot][0], X1 = xa[j][xs_slot][1];
          const uint32_t Bf[4][2] = {{prmt(X0.x, X0.z, 0x5410), prmt(X0.x, X0.z, 0x7632)},
                                     {prmt(X0.y, X0.w, 0x5410), prmt(X0.y, X0.w, 0x7632)},
                                     {prmt(X1.x, X1.z, 0x5410), prmt(X1.x, X1.z, 0x7632)},
                                     {prmt(X1.y, X1.w, 0x5410), prmt(X1.y, X1.w, 0x7632)}};
          float acc[4] = {0.f, 0.f, 0.f, 0.f};
          float xs[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int kt = 0; kt < 4; ++kt) {
            mma_bf16_16816(acc, A[kt][0], A[kt][1], A[kt][2], A[kt][3], Bf[kt][0], Bf[kt][1]);
            mma_bf16_16816(xs, ONES, ONES, ONES, ONES, Bf[kt][0], Bf[kt][1]);
          }
          y[j][0] = fmaf(sg[i], acc[0], fmaf(bb0, xs[0], y[j][0]));
          y[j][1] = fmaf(sg[i], acc[1], fmaf(bb0, xs[1], y[j][1]));
          y[j][2] = fmaf(sg8[i], acc[2], fmaf(bb1, xs[2], y[j][2]));
          y[j][3] = fmaf(sg8[i], acc[3], fmaf(bb1, xs[3], y[j][3]));
        }
      }
      if (more) cur = nxt;
    }
  }

  pdl_launch();

  // cross-warp K reduction
#pragma unroll
  for (int j = 0; j < NT8; ++j)
#pragma unroll
    for (int c = 0; c < 4; ++c) red[warp][j * 4 + c][lane] = y[j][c];
  __syncthreads();

  const bool leader = (kw == 0) && (EPI != EPI_SWIGLU || which == 0);
  if (!leader || !tile_ok) return;

  float v[NT8][4], v2[NT8][4];
#pragma unroll
  for (int j = 0; j < NT8; ++j)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float s = 0.f, s2 = 0.f;
#pragma unroll
      for (int w = 0; w < WK; ++w) {
        s += red[rt * WK + w][j * 4 + c][lane];
        if (EPI == EPI_SWIGLU) s2 += red[(rt + 1) * WK + w][j * 4 + c][lane];
      }
      v[j][c] = s;
      v2[j][c] = s2;
    }

#pragma unroll
  for (int j = 0; j < NT8; ++j)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int row = n0 + g + 8 * (c >> 1);
      const int tok = 8 * j + 2 * t + (c & 1);
      if (tok >= M) continue;
      const size_t o = (size_t)tok * N + row;
      if (EPI == EPI_SWIGLU) {
        const float gv = round_bf(v[j][c]), uv = round_bf(v2[j][c]);
        a.y[o] = f2bf(gv / (1.0f + expf(-gv)) * uv);
      } else {
        if (a.y_f32) a.y_f32[o] = v[j][c];
        if (a.y) {
          uint16_t r = f2bf(v[j][c]);
          if (a.residual) r = f2bf(bf2f(r) + bf2f(a.residual[o]));
          a.y[o] = r;
        }
      }
    }
}

template <int NT8, int EPI>
static cudaError_t launch_qlinear_nt(const QLinArgs& a, cudaStream_t st) {
  const int nrt = (a.N + 15) / 16;
  const int sms = sm_count();
  // Pick the K split: keep >= 2 CTAs per SM in flight, and >= 1 unit per warp.
  const int units = a.K / 256;
  int wk;
  if constexpr (EPI == EPI_SWIGLU) {
    // RT = 8/wk warp tiles = 4/wk gate/up pairs per CTA
    wk = 4;
    if (nrt / 2 >= 2 * sms && units >= 2) wk = 2;
    if (nrt / 4 >= 2 * sms && units >= 1) wk = 1;
    while (wk > 1 && units < wk) wk >>= 1;
    const int rot = (8 / wk) / 2;
    dim3 grid((nrt + rot - 1) / rot);
    if (wk == 4) return launch_pdl(qlinear_w4_kernel<NT8, 4, EPI>, grid, dim3(256), 0, st, a);
    if (wk == 2) return launch_pdl(qlinear_w4_kernel<NT8, 2, EPI>, grid, dim3(256), 0, st, a);
    return launch_pdl(qlinear_w4_kernel<NT8, 1, EPI>, grid, dim3(256), 0, st, a);
  } else {
    wk = 8;
    if (nrt / 2 >= 2 * sms) wk = 4;
    if (nrt / 4 >= 2 * sms) wk = 2;
    if (nrt / 8 >= 2 * sms) wk = 1;
    while (wk > 1 && units < wk) wk >>= 1;
    const int rot = 8 / wk;
    dim3 grid((nrt + rot - 1) / rot);
    switch (wk) {
      case 8: return launch_pdl(qlinear_w4_kernel<NT8, 8, EPI>, grid, dim3(256), 0, st, a);
      case 4: return launch_pdl(qlinear_w4_kernel<NT8, 4, EPI>, grid, dim3(256), 0, st, a);
      case 2: return launch_pdl(qlinear_w4_kernel<NT8, 2, EPI>, grid, dim3(256), 0, st, a);
      default: return launch_pdl(qlinear_w4_kernel<NT8, 1, EPI>, grid, dim3(256), 0, st, a);
    }
  }
}

template <int EPI>
static cudaError_t launch_qlinear_epi(QLinArgs a, cudaStream_t st) {
  const int M = a.M;
  for (int m0 = 0; m0 < M; m0 += 32) {
    QLinArgs c = a;
    c.M = (M - m0) < 32 ? (M - m0) : 32;
    c.x = a.x + (size_t)m0 * a.K;
    if (a.y) c.y = a.y + (size_t)m0 * a.N;
    if (a.y_f32) c.y_f32 = a.y_f32 + (size_t)m0 * a.N;
    if (a.residual) c.residual = a.residual + (size_t)m0 * a.N;
    cudaError_t e;
    if (c.M <= 8)
      e = launch_qlinear_nt<1, EPI>(c, st);
    else if (c.M <= 16)
      e = launch_qlinear_nt<2, EPI>(c, st);
    else
      e = launch_qlinear_nt<4, EPI>(c, st);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_qlinear(const QLinArgs& a, int epi, cudaStream_t st) {
  return epi == EPI_SWIGLU ? launch_qlinear_epi<EPI_SWIGLU>(a, st) : launch_qlinear_epi<EPI_STORE>(a, st);
}

// ---------------------------------------------------------------------------
// embedding gather + dequantize
// ---------------------------------------------------------------------------
__global__ void embed_gather_kernel(const int32_t* ids, const uint32_t* w, const uint16_t* s,
                                    const uint16_t* b, int V, int H, uint16_t* out) {
  pdl_wait();
  const int i = blockIdx.x;
  const int r = ids[i];
  const int KW = H / 8, G = H / 64;
  for (int wi = threadIdx.x; wi < KW; wi += blockDim.x) {
    uint4 o;
    uint32_t* op = &o.x;
    if (r >= 0 && r < V) {
      const uint32_t word = w[(size_t)r * KW + wi];
      const float sc = bf2f(s[(size_t)r * G + wi / 8]), bi = bf2f(b[(size_t)r * G + wi / 8]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float q0 = (float)((word >> (8 * j)) & 0xF), q1 = (float)((word >> (8 * j + 4)) & 0xF);
        op[j] = pack_bf2(fmaf(sc, q0, bi), fmaf(sc, q1, bi));
      }
    } else {
      o = make_uint4(0, 0, 0, 0);
    }
    *reinterpret_cast<uint4*>(out + (size_t)i * H + wi * 8) = o;
  }
  pdl_launch();
}

__global__ void dequant_kernel(const uint32_t* w, const uint16_t* s, const uint16_t* b, int N,
                               int K, uint16_t* out) {
  const int64_t total = (int64_t)N * (K / 8);
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = idx / (K / 8), wi = idx % (K / 8);
    const uint32_t word = w[idx];
    const float sc = bf2f(s[n * (K / 64) + wi / 8]), bi = bf2f(b[n * (K / 64) + wi / 8]);
    uint4 o;
    uint32_t* op = &o.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float q0 = (float)((word >> (8 * j)) & 0xF), q1 = (float)((word >> (8 * j + 4)) & 0xF);
      op[j] = pack_bf2(fmaf(sc, q0, bi), fmaf(sc, q1, bi));
    }
    *reinterpret_cast<uint4*>(out + n * K + wi * 8) = o;
  }
}

// One thread per (row, 64-group); the rounding sequence is the oracle's:
// scale = bf16((hi - lo) / 15) (1 if that is 0), bias = bf16(lo),
// q = clamp(rint((w - bias) / scale), 0, 15).
__global__ void quantize_kernel(const float* w, int64_t N, int K, uint32_t* q, uint16_t* s,
                                uint16_t* b) {
  const int G = K / 64;
  const int64_t total = N * G;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = idx / G, g = idx % G;
    const float* src = w + n * K + g * 64;
    float v[64];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float4 f = reinterpret_cast<const float4*>(src)[i];
      v[4 * i] = f.x;
      v[4 * i + 1] = f.y;
      v[4 * i + 2] = f.z;
      v[4 * i + 3] = f.w;
    }
    float lo = v[0], hi = v[0];
#pragma unroll
    for (int i = 1; i < 64; ++i) {
      lo = v[i] < lo ? v[i] : lo;
      hi = v[i] > hi ? v[i] : hi;
    }
    uint16_t sb = f2bf(__fdiv_rn(__fsub_rn(hi, lo), 15.0f));
    if (bf2f(sb) == 0.0f) sb = f2bf(1.0f);
    const uint16_t bb = f2bf(lo);
    const float sc = bf2f(sb), bi = bf2f(bb);
    s[idx] = sb;
    b[idx] = bb;
#pragma unroll
    for (int w8 = 0; w8 < 8; ++w8) {
      uint32_t word = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float c = rintf(__fdiv_rn(__fsub_rn(v[w8 * 8 + j], bi), sc));
        c = fminf(fmaxf(c, 0.0f), 15.0f);
        word |= ((uint32_t)c) << (4 * j);
      }
      q[n * (K / 8) + g * 8 + w8] = word;
    }
  }
}

}  // namespace higgs

using namespace higgs;

extern "C" int higgs_w4_quantize(higgs_ctx* ctx, const float* w, int64_t N, int K, uint32_t* q,
                                 void* scales, void* biases, void* stream) {
  HG_CHECK_ARG(ctx && w && q && scales && biases, "higgs_w4_quantize: null argument");
  HG_CHECK_ARG(N >= 0 && K > 0 && K % 64 == 0, "higgs_w4_quantize: need K % 64 == 0");
  HG_DEVICE(ctx);
  if (N == 0) return HIGGS_OK;
  const int64_t total = N * (K / 64);
  const int64_t want = (total + 127) / 128;
  const int blocks = (int)(want < 64 * sm_count() ? want : 64 * sm_count());
  quantize_kernel<<<blocks, 128, 0, (cudaStream_t)stream>>>(w, N, K, q, (uint16_t*)scales,
                                                             (uint16_t*)biases);
  HG_CUDA(cudaGetLastError());
  return HIGGS_OK;
}

extern "C" int higgs_w4_dequantize(higgs_ctx* ctx, const uint32_t* w, const void* scales,
                                   const void* biases, int N, int K, void* out, void* stream) {
  HG_CHECK_ARG(ctx && w && scales && biases && out, "higgs_w4_dequantize: null argument");
  HG_CHECK_ARG(N > 0 && K > 0 && K % 64 == 0, "higgs_w4_dequantize: need N > 0, K % 64 == 0");
  HG_DEVICE(ctx);
  const int64_t total = (int64_t)N * (K / 8);
  const int blocks = (int)((total + 255) / 256 < 8 * sm_count() ? (total + 255) / 256 : 8 * sm_count());
  dequant_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(
      w, (const uint16_t*)scales, (const uint16_t*)biases, N, K, (uint16_t*)out);
  HG_CUDA(cudaGetLastError());
  return HIGGS_OK;
}

extern "C" int higgs_embed_gather_w4(higgs_ctx* ctx, const int32_t* ids, int n_ids,
                                     const uint32_t* w, const void* scales, const void* biases,
                                     int V, int H, void* out, void* stream) {
  HG_CHECK_ARG(ctx && ids && w && scales && biases && out, "higgs_embed_gather_w4: null argument");
  HG_CHECK_ARG(n_ids >= 0 && V > 0 && H > 0 && H % 64 == 0,
               "higgs_embed_gather_w4: need H % 64 == 0");
  HG_DEVICE(ctx);
  if (n_ids == 0) return HIGGS_OK;
  HG_CUDA(launch_pdl(embed_gather_kernel, dim3(n_ids), dim3(128), 0, (cudaStream_t)stream, ids, w,
                     (const uint16_t*)scales, (const uint16_t*)biases, V, H, (uint16_t*)out));
  return HIGGS_OK;
}

extern "C" int higgs_qlinear_w4g64(higgs_ctx* ctx, const void* x, int M, int K, const uint32_t* w,
                                   const void* scales, const void* biases, int N, void* y,
                                   float* y_f32, const void* residual, void* stream) {
  HG_CHECK_ARG(ctx && x && w && scales && biases, "higgs_qlinear_w4g64: null argument");
  HG_CHECK_ARG(y || y_f32, "higgs_qlinear_w4g64: need y or y_f32");
  HG_CHECK_ARG(!residual || y, "higgs_qlinear_w4g64: residual needs a bf16 y");
  HG_CHECK_ARG(M >= 0 && K > 0 && N > 0, "higgs_qlinear_w4g64: bad shape");
  HG_CHECK_ARG(K % 256 == 0, "higgs_qlinear_w4g64: K must be a multiple of 256");
  HG_CHECK_ARG(N % 16 == 0, "higgs_qlinear_w4g64: N must be a multiple of 16");
  HG_DEVICE(ctx);
  if (M == 0) return HIGGS_OK;
  QLinArgs a = {};
  a.x = (const uint16_t*)x;
  a.M = M;
  a.K = K;
  a.N = N;
  a.w = w;
  a.s = (const uint16_t*)scales;
  a.b = (const uint16_t*)biases;
  a.y = (uint16_t*)y;
  a.y_f32 = y_f32;
  a.residual = (const uint16_t*)residual;
  a.self_prefetch = l2_prefetch_self();
  HG_CUDA(launch_qgemv_ring(a, EPI_STORE, (cudaStream_t)stream));
  return HIGGS_OK;
}

extern "C" int higgs_qlinear_gate_up_swiglu(higgs_ctx* ctx, const void* x, int M, int K,
                                            const uint32_t* w_gate, const void* s_gate,
                                            const void* b_gate, const uint32_t* w_up,
                                            const void* s_up, const void* b_up, int N, void* y,
                                            void* stream) {
  HG_CHECK_ARG(ctx && x && w_gate && s_gate && b_gate && w_up && s_up && b_up && y,
               "higgs_qlinear_gate_up_swiglu: null argument");
  HG_CHECK_ARG(M >= 0 && K > 0 && N > 0, "higgs_qlinear_gate_up_swiglu: bad shape");
  HG_CHECK_ARG(K % 256 == 0, "higgs_qlinear_gate_up_swiglu: K must be a multiple of 256");
  HG_CHECK_ARG(N % 16 == 0, "higgs_qlinear_gate_up_swiglu: N must be a multiple of 16");
  HG_DEVICE(ctx);
  if (M == 0) return HIGGS_OK;
  QLinArgs a = {};
  a.x = (const uint16_t*)x;
  a.M = M;
  a.K = K;
  a.N = N;
  a.w = w_gate;
  a.s = (const uint16_t*)s_gate;
  a.b = (const uint16_t*)b_gate;
  a.w2 = w_up;
  a.s2 = (const uint16_t*)s_up;
  a.b2 = (const uint16_t*)b_up;
  a.y = (uint16_t*)y;
  a.self_prefetch = l2_prefetch_self();
  HG_CUDA(launch_qgemv_ring(a, EPI_SWIGLU, (cudaStream_t)stream));
  return HIGGS_OK;
}
