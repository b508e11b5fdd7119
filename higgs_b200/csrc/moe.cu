// moe.cu -- mixture-of-experts router, routing plan and combine.
//
// Reference op replaced: Qwen3MoeMlpBlock::forward_moe
// (crates/higgs-models/src/qwen3_moe.rs:293-322): softmax(router logits) ->
// argpartition(-k) -> take_along_axis -> renormalise (norm_topk_prob) ->
// SwitchMlpWeights::forward_gather (qwen3_next.rs:844-904, three gather_qmm)
// -> multiply by the scores and sum over k.
//
// MLX's gather_qmm evaluates each (token, expert) pair against the stacked
// expert weights.  Here the router also emits a routing plan: the pairs
// p = t*k + j grouped by expert (ascending p inside an expert, so the order is
// a pure function of the routing) and cut into work items of at most 8 pairs
// of one expert.  The grouped W4 GEMV (qgemv.cu, GATHER mode) runs one CTA row
// per work item, so every expert's weight tile is streamed once per 8 tokens
// that chose it instead of once per token.
#include "common.cuh"
#include "kernels.cuh"

namespace higgs {

size_t moe_plan_bytes(int T, int E, int k) {
  const int P = T * k;
  return 16 + 16 * (size_t)moe_max_items(P, E) + 4 * (size_t)P + 4 * (size_t)E;
}

namespace {

constexpr int kRouteThreads = 1024;

__device__ __forceinline__ float key_value(unsigned long long key) {
  const uint32_t o = (uint32_t)(key >> 32);
  return __uint_as_float((o & 0x80000000u) ? (o & 0x7fffffffu) : ~o);
}

// One CTA: phase 1 routes every token (one warp per token), phase 2 builds the
// plan.  NV = logits held per lane (E <= 32 * NV).
template <int NV, bool BF16IN>
__global__ void __launch_bounds__(kRouteThreads) moe_route_kernel(const void* logits, int T, int E,
                                                                  int k, int norm, int32_t* idx,
                                                                  float* scores, int* plan,
                                                                  int max_items) {
  extern __shared__ int sm[];
  int* counts = sm;            // [E]
  int* cursor = sm + E;        // [E]
  int* item_off = sm + 2 * E;  // [E + 1]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = T * k;
  if (plan)
    for (int e = threadIdx.x; e < E; e += kRouteThreads) counts[e] = 0;
  pdl_wait();
  for (int t = warp; t < T; t += kRouteThreads / 32) {
    float v[NV];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int e = lane + 32 * i;
      float x = -INFINITY;
      if (e < E) {
        x = BF16IN ? bf2f(static_cast<const uint16_t*>(logits)[(size_t)t * E + e])
                   : static_cast<const float*>(logits)[(size_t)t * E + e];
        if (x > mx) mx = x;  // NaN never raises the max
      }
      v[i] = x;
    }
    mx = warp_max(mx);
    float den = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i)
      if (lane + 32 * i < E) den = __fadd_rn(den, det_exp(__fsub_rn(v[i], mx)));
    den = warp_sum(den);
    uint32_t taken = 0;
    float ssum = 0.f, my_score = 0.f;
    int my_idx = 0;
    for (int j = 0; j < k; ++j) {
      unsigned long long best = 0ull;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int e = lane + 32 * i;
        if (e < E && !((taken >> i) & 1u)) best = max(best, argmax_key(v[i], e));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
      const int e = (int)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull));
      if ((e & 31) == lane) taken |= 1u << (e >> 5);
      const float g = __fdiv_rn(det_exp(__fsub_rn(key_value(best), mx)), den);
      ssum = __fadd_rn(ssum, g);
      if (lane == j) {
        my_idx = e;
        my_score = g;
      }
    }
    if (lane < k) {
      idx[(size_t)t * k + lane] = my_idx;
      scores[(size_t)t * k + lane] = norm ? __fdiv_rn(my_score, ssum) : my_score;
    }
  }
  pdl_launch();
  if (!plan) return;
  __syncthreads();  // idx visible to the whole CTA
  for (int p = threadIdx.x; p < P; p += kRouteThreads) atomicAdd(&counts[idx[p]], 1);
  __syncthreads();
  if (warp == 0) {
    // exclusive scans of counts (pair offsets) and ceil(counts / 8) (item offsets)
    int run_p = 0, run_i = 0;
    for (int base = 0; base < E; base += 32) {
      const int e = base + lane;
      const int c = e < E ? counts[e] : 0;
      const int ci = (c + 7) >> 3;
      int sp = c, si = ci;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int a = __shfl_up_sync(0xffffffffu, sp, o);
        const int b = __shfl_up_sync(0xffffffffu, si, o);
        if (lane >= o) {
          sp += a;
          si += b;
        }
      }
      if (e < E) {
        cursor[e] = run_p + sp - c;
        item_off[e] = run_i + si - ci;
      }
      run_p += __shfl_sync(0xffffffffu, sp, 31);
      run_i += __shfl_sync(0xffffffffu, si, 31);
    }
    if (lane == 0) {
      item_off[E] = run_i;
      plan[0] = run_i;
      plan[1] = P;
      plan[2] = E;
      plan[3] = k;
    }
  }
  __syncthreads();
  int4* items = reinterpret_cast<int4*>(plan + 4);
  int* sorted = plan + 4 + 4 * max_items;
  int* pcounts = sorted + P;
  for (int e = threadIdx.x; e < E; e += kRouteThreads) {
    const int c = counts[e];
    pcounts[e] = c;
    for (int i = 0, s0 = cursor[e]; i < (c + 7) / 8; ++i)
      items[item_off[e] + i] = make_int4(e, s0 + 8 * i, min(8, c - 8 * i), 0);
  }
  __syncthreads();  // cursor is read above before warp 0 advances it below
  if (warp == 0) {
    // stable placement: pairs in ascending order, 32 at a time
    for (int base = 0; base < P; base += 32) {
      const int p = base + lane;
      const bool valid = p < P;
      const unsigned act = __ballot_sync(0xffffffffu, valid);
      if (valid) {
        const int e = idx[p];
        const unsigned peers = __match_any_sync(act, e);
        const int rank = __popc(peers & ((1u << lane) - 1u));
        sorted[cursor[e] + rank] = p;
        __syncwarp(act);
        if (rank == 0) cursor[e] += __popc(peers);
      }
      __syncwarp();
    }
  }
}

// Router logits in a fixed summation order: for each (row, group) the 64 products
// x*q and the 64 x values are summed in k order, then the group terms s*sxq + b*sx
// are added in group order -- the order of the quantized-matmul restatement, so any
// implementation that follows it gets bit-identical logits.  Top-k selection is a
// discontinuous function of the logits; this keeps expert choice reproducible.
// Block = R rows x G groups (R*G <= 256 threads); grid (E / R, T).
__global__ void __launch_bounds__(256) moe_router_kernel(const uint16_t* x, int K,
                                                         const uint32_t* w, const uint16_t* s,
                                                         const uint16_t* b, int E, int R,
                                                         uint16_t* out) {
  __shared__ float part[256];
  const int G = K / 64;
  const int t = blockIdx.y;
  const int r = threadIdx.x / G, g = threadIdx.x % G;
  const int n = blockIdx.x * R + r;
  pdl_wait();
  if (r < R && n < E) {
    const uint16_t* xr = x + (size_t)t * K + g * 64;
    const uint32_t* wr = w + (size_t)n * (K / 8) + g * 8;
    float sxq = 0.f, sx = 0.f;
    for (int w8 = 0; w8 < 8; ++w8) {
      const uint32_t word = wr[w8];
      const uint4 xv = ldg_u4(xr + w8 * 8);
      const uint32_t* xp = &xv.x;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float xf = (j & 1) ? bf_hi(xp[j >> 1]) : bf_lo(xp[j >> 1]);
        sxq = __fadd_rn(sxq, __fmul_rn(xf, (float)((word >> (4 * j)) & 0xF)));
        sx = __fadd_rn(sx, xf);
      }
    }
    part[threadIdx.x] = __fadd_rn(__fmul_rn(bf2f(s[(size_t)n * G + g]), sxq),
                                  __fmul_rn(bf2f(b[(size_t)n * G + g]), sx));
  }
  __syncthreads();
  pdl_launch();
  if (threadIdx.x < R && blockIdx.x * R + threadIdx.x < E) {
    float acc = 0.f;
    for (int gg = 0; gg < G; ++gg) acc = __fadd_rn(acc, part[threadIdx.x * G + gg]);
    out[(size_t)t * E + blockIdx.x * R + threadIdx.x] = f2bf(acc);
  }
}

// h[t] = bf16(h[t] + bf16(sum_j bf16(s_j) * y[t*k+j])): 8 columns per thread.
__global__ void __launch_bounds__(128) moe_combine_kernel(const uint16_t* y, const float* scores,
                                                          int T, int k, int H, uint16_t* h) {
  pdl_wait();
  const int t = blockIdx.y;
  const int c8 = blockIdx.x * 128 + threadIdx.x;
  if (c8 * 8 < H) {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    for (int j = 0; j < k; ++j) {
      const float sc = round_bf(scores[(size_t)t * k + j]);
      const uint4 v = ldg_u4(y + ((size_t)t * k + j) * H + c8 * 8);
      const uint32_t* vp = &v.x;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc[2 * i] = __fadd_rn(acc[2 * i], __fmul_rn(sc, bf_lo(vp[i])));
        acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], __fmul_rn(sc, bf_hi(vp[i])));
      }
    }
    uint4* hp = reinterpret_cast<uint4*>(h + (size_t)t * H + c8 * 8);
    const uint4 hv = *hp;
    const uint32_t* hq = &hv.x;
    uint4 o;
    uint32_t* op = &o.x;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      op[i] = pack_bf2(__fadd_rn(bf_lo(hq[i]), round_bf(acc[2 * i])),
                       __fadd_rn(bf_hi(hq[i]), round_bf(acc[2 * i + 1])));
    *hp = o;
  }
  pdl_launch();
}

// Expert parallelism: part[t] = sum over this rank's pairs j of bf16(s_j) * y[t*k+j], f32 in
// j order (the all-reduce then adds the ranks' shares and the residual, rounding once).
__global__ void __launch_bounds__(128) moe_combine_partial_kernel(const uint16_t* y, const float* scores,
                                                                  const int32_t* idx, int T, int k,
                                                                  int H, int e_lo, int e_n,
                                                                  float* part) {
  pdl_wait();
  const int t = blockIdx.y;
  const int c8 = blockIdx.x * 128 + threadIdx.x;
  if (c8 * 8 < H) {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    for (int j = 0; j < k; ++j) {
      const int e = idx[(size_t)t * k + j];
      if (e < e_lo || e >= e_lo + e_n) continue;
      const float sc = round_bf(scores[(size_t)t * k + j]);
      const uint4 v = ldg_u4(y + ((size_t)t * k + j) * H + c8 * 8);
      const uint32_t* vp = &v.x;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc[2 * i] = __fadd_rn(acc[2 * i], __fmul_rn(sc, bf_lo(vp[i])));
        acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], __fmul_rn(sc, bf_hi(vp[i])));
      }
    }
    float4* pp = reinterpret_cast<float4*>(part + (size_t)t * H + c8 * 8);
    pp[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    pp[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
  pdl_launch();
}

template <bool BF16IN>
cudaError_t launch_route_nv(const void* logits, int T, int E, int k, int norm, int32_t* idx,
                            float* scores, int* plan, cudaStream_t st) {
  const size_t smem = (size_t)(3 * E + 1) * sizeof(int);
  const int mi = moe_max_items(T * k, E);
  if (E <= 128)
    return launch_pdl(moe_route_kernel<4, BF16IN>, dim3(1), dim3(kRouteThreads), smem, st, logits,
                      T, E, k, norm, idx, scores, plan, mi);
  if (E <= 256)
    return launch_pdl(moe_route_kernel<8, BF16IN>, dim3(1), dim3(kRouteThreads), smem, st, logits,
                      T, E, k, norm, idx, scores, plan, mi);
  if (E <= 512)
    return launch_pdl(moe_route_kernel<16, BF16IN>, dim3(1), dim3(kRouteThreads), smem, st, logits,
                      T, E, k, norm, idx, scores, plan, mi);
  return launch_pdl(moe_route_kernel<32, BF16IN>, dim3(1), dim3(kRouteThreads), smem, st, logits, T,
                    E, k, norm, idx, scores, plan, mi);
}

}  // namespace

cudaError_t launch_moe_route(const void* logits, bool bf16_in, int T, int E, int k, int norm,
                             int32_t* idx, float* scores, void* plan, cudaStream_t st) {
  return bf16_in ? launch_route_nv<true>(logits, T, E, k, norm, idx, scores, (int*)plan, st)
                 : launch_route_nv<false>(logits, T, E, k, norm, idx, scores, (int*)plan, st);
}

cudaError_t launch_moe_grouped(const uint16_t* x, int T, int K, int k, bool x_per_pair,
                               const void* plan, int E, int N, const uint32_t* w, const uint16_t* s,
                               const uint16_t* b, const uint32_t* w2, const uint16_t* s2,
                               const uint16_t* b2, uint16_t* y, cudaStream_t st, int e_lo, int e_n) {
  QLinArgs a{};
  a.x = x;
  a.M = 8;
  a.K = K;
  a.N = N;
  a.w = w;
  a.s = s;
  a.b = b;
  a.nseg = 1;
  a.w2 = w2;
  a.s2 = s2;
  a.b2 = b2;
  a.y = y;
  const int P = T * k;
  a.moe_max_items = moe_max_items(P, E);
  a.moe_n_items = static_cast<const int*>(plan);
  a.moe_items = reinterpret_cast<const int4*>(static_cast<const int*>(plan) + 4);
  a.moe_sorted = static_cast<const int*>(plan) + 4 + 4 * a.moe_max_items;
  a.moe_xdiv = x_per_pair ? 1 : k;
  a.moe_ew = (long long)N * (K / 8);
  a.moe_es = (long long)N * (K / 64);
  a.moe_e_lo = e_lo;
  a.moe_e_n = e_n;
  a.self_prefetch = l2_prefetch_self();
  return launch_qgemv_grouped(a, w2 ? EPI_SWIGLU : EPI_STORE, st);
}

cudaError_t launch_moe_router(const uint16_t* x, int T, int K, const uint32_t* w,
                              const uint16_t* s, const uint16_t* b, int E, uint16_t* out,
                              cudaStream_t st) {
  const int G = K / 64;
  const int R = 256 / G;
  return launch_pdl(moe_router_kernel, dim3((E + R - 1) / R, T), dim3(256), 0, st, x, K, w, s, b, E,
                    R, out);
}

cudaError_t launch_moe_combine_partial(const uint16_t* y, const float* scores, const int32_t* idx,
                                       int T, int k, int H, int e_lo, int e_n, float* part,
                                       cudaStream_t st) {
  const dim3 grid((H / 8 + 127) / 128, T);
  return launch_pdl(moe_combine_partial_kernel, grid, dim3(128), 0, st, y, scores, idx, T, k, H, e_lo, e_n,
                    part);
}

cudaError_t launch_moe_combine(const uint16_t* y, const float* scores, int T, int k, int H,
                               uint16_t* h, cudaStream_t st) {
  const dim3 grid((H / 8 + 127) / 128, T);
  return launch_pdl(moe_combine_kernel, grid, dim3(128), 0, st, y, scores, T, k, H, h);
}

}  // namespace higgs

using namespace higgs;

extern "C" size_t higgs_moe_plan_size(int T, int E, int k) {
  if (T <= 0 || E <= 0 || k <= 0) return 0;
  return moe_plan_bytes(T, E, k);
}

extern "C" int higgs_moe_route_topk(higgs_ctx* ctx, const void* logits, int dtype, int T, int E,
                                    int k, int norm_topk_prob, int32_t* idx, float* scores,
                                    void* plan, size_t plan_bytes, void* stream) {
  HG_CHECK_ARG(ctx && logits && idx && scores, "higgs_moe_route_topk: null argument");
  HG_CHECK_ARG(dtype == HIGGS_DTYPE_BF16 || dtype == HIGGS_DTYPE_F32,
               "higgs_moe_route_topk: logits must be bf16 or f32");
  HG_CHECK_ARG(E > 0 && E <= 1024, "higgs_moe_route_topk: E must be in [1, 1024]");
  HG_CHECK_ARG(k > 0 && k <= 32 && k <= E, "higgs_moe_route_topk: k must be in [1, min(E, 32)]");
  HG_CHECK_ARG(T >= 0 && (int64_t)T * k <= 65536, "higgs_moe_route_topk: T * k must be <= 65536");
  HG_DEVICE(ctx);
  if (T == 0) return HIGGS_OK;
  if (plan)
    HG_CHECK_ARG(plan_bytes >= moe_plan_bytes(T, E, k) && ((uintptr_t)plan & 15) == 0,
                 "higgs_moe_route_topk: plan smaller than higgs_moe_plan_size or not 16-byte aligned");
  HG_CUDA(launch_moe_route(logits, dtype == HIGGS_DTYPE_BF16, T, E, k, norm_topk_prob, idx, scores,
                           plan, (cudaStream_t)stream));
  return HIGGS_OK;
}

extern "C" int higgs_moe_grouped_w4(higgs_ctx* ctx, const void* x, int T, int K, int k,
                                    int x_per_pair, const void* plan, const uint32_t* w,
                                    const void* scales, const void* biases, const uint32_t* w_up,
                                    const void* scales_up, const void* biases_up, int E, int N,
                                    void* y, void* stream) {
  HG_CHECK_ARG(ctx && x && plan && w && scales && biases && y, "higgs_moe_grouped_w4: null argument");
  HG_CHECK_ARG(!w_up == !scales_up && !w_up == !biases_up,
               "higgs_moe_grouped_w4: w_up, scales_up and biases_up go together");
  HG_CHECK_ARG(K > 0 && K % 256 == 0 && N > 0 && N % 16 == 0,
               "higgs_moe_grouped_w4: K % 256 == 0 and N % 16 == 0 required");
  HG_CHECK_ARG(qgemv_grouped_supported(K), "higgs_moe_grouped_w4: K too large for the staged x tile");
  HG_CHECK_ARG(E > 0 && k > 0 && T >= 0 && moe_max_items(T * k, E) <= 65535,
               "higgs_moe_grouped_w4: bad T / k / E");
  HG_CHECK_ARG(((uintptr_t)plan & 15) == 0, "higgs_moe_grouped_w4: plan must be 16-byte aligned");
  HG_DEVICE(ctx);
  if (T == 0) return HIGGS_OK;
  HG_CUDA(launch_moe_grouped((const uint16_t*)x, T, K, k, x_per_pair != 0, plan, E, N, w,
                             (const uint16_t*)scales, (const uint16_t*)biases, w_up,
                             (const uint16_t*)scales_up, (const uint16_t*)biases_up, (uint16_t*)y,
                             (cudaStream_t)stream));
  return HIGGS_OK;
}

extern "C" int higgs_moe_router(higgs_ctx* ctx, const void* x, int T, int K, const uint32_t* w,
                                const void* scales, const void* biases, int E, void* logits,
                                void* stream) {
  HG_CHECK_ARG(ctx && x && w && scales && biases && logits, "higgs_moe_router: null argument");
  HG_CHECK_ARG(T >= 0 && T <= 65535 && E > 0 && K > 0 && K % 64 == 0 && K / 64 <= 256,
               "higgs_moe_router: bad shape (K % 64 == 0, K <= 16384, T <= 65535)");
  HG_DEVICE(ctx);
  if (T == 0) return HIGGS_OK;
  HG_CUDA(launch_moe_router((const uint16_t*)x, T, K, w, (const uint16_t*)scales,
                            (const uint16_t*)biases, E, (uint16_t*)logits, (cudaStream_t)stream));
  return HIGGS_OK;
}

extern "C" int higgs_moe_combine(higgs_ctx* ctx, const void* y, const float* scores, int T, int k,
                                 int H, void* h, void* stream) {
  HG_CHECK_ARG(ctx && y && scores && h, "higgs_moe_combine: null argument");
  HG_CHECK_ARG(T >= 0 && k > 0 && H > 0 && H % 8 == 0 && T <= 65535,
               "higgs_moe_combine: bad shape (H % 8 == 0, T <= 65535)");
  HG_DEVICE(ctx);
  if (T == 0) return HIGGS_OK;
  HG_CUDA(launch_moe_combine((const uint16_t*)y, scores, T, k, H, (uint16_t*)h, (cudaStream_t)stream));
  return HIGGS_OK;
}
