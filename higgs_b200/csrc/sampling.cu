// sampling.cu -- greedy argmax, temperature sampling, speculative acceptance
// and repetition/frequency/presence penalties, on the device.
//
// Reference ops replaced: sample / argmax_axis / categorical (lib.rs:373-385)
// and apply_penalties (lib.rs:278-363).  Speculative acceptance has no
// reference counterpart.
//
// Probabilities are exact integers: e_j = det_exp((l_j - max) / T) is held as
// E_j = floor(e_j * 2^32), and every sum / prefix sum is an exact u64, so a
// draw is a deterministic function of (logits, T, u) whatever the reduction
// order.  det_exp is a Cody-Waite + degree-7 Taylor exp built from correctly
// rounded f32 operations only, so the CPU checker computes the same bits.
#include "common.cuh"

namespace higgs {

constexpr int kSampThreads = 1024;

__device__ __forceinline__ float det_exp(float x) {
  if (!(x >= -87.0f)) return 0.0f;
  if (x > 88.0f) x = 88.0f;
  const float kf = rintf(__fmul_rn(x, 1.44269504088896341f));
  float r = __fmaf_rn(-kf, 0.693145751953125f, x);
  r = __fmaf_rn(-kf, 1.42860682030941723e-6f, r);
  float p = 1.98412698412698413e-4f;
  p = __fmaf_rn(p, r, 1.38888888888888889e-3f);
  p = __fmaf_rn(p, r, 8.33333333333333333e-3f);
  p = __fmaf_rn(p, r, 4.16666666666666667e-2f);
  p = __fmaf_rn(p, r, 1.66666666666666667e-1f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const int k = (int)kf;
  return __fmul_rn(p, __uint_as_float((uint32_t)(k + 127) << 23));
}

__device__ __forceinline__ uint64_t fixed_mass(float l, float inv_t, float mxs) {
  const float e = det_exp(__fsub_rn(__fmul_rn(l, inv_t), mxs));
  return (uint64_t)__dmul_rn((double)e, 4294967296.0);
}

// ---- block reductions (1024 threads) ---------------------------------------
__device__ float block_max(float v, float* sh) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  float r = -INFINITY;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) r = fmaxf(r, sh[i]);
  return r;
}

__device__ __forceinline__ uint64_t shfl_up_u64(uint64_t v, int d) {
  const uint32_t lo = __shfl_up_sync(0xffffffffu, (uint32_t)v, d);
  const uint32_t hi = __shfl_up_sync(0xffffffffu, (uint32_t)(v >> 32), d);
  return ((uint64_t)hi << 32) | lo;
}

// exclusive prefix of v over the block; returns it and writes the total
__device__ uint64_t block_exscan_u64(uint64_t v, uint64_t* sh, uint64_t* total) {
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  uint64_t inc = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const uint64_t o = shfl_up_u64(inc, d);
    if (l >= d) inc += o;
  }
  __syncthreads();
  if (l == 31) sh[w] = inc;
  __syncthreads();
  uint64_t before = 0, tot = 0;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) {
    if (i < w) before += sh[i];
    tot += sh[i];
  }
  *total = tot;
  return before + inc - v;
}

struct RowDist {
  const float* logits;
  float inv_t, mxs;
};

__device__ RowDist make_dist(const float* logits, int V, float inv_t, float* shf) {
  float mx = -INFINITY;
  for (int j = threadIdx.x; j < V; j += blockDim.x) mx = fmaxf(mx, logits[j]);
  mx = block_max(mx, shf);
  RowDist d;
  d.logits = logits;
  d.inv_t = inv_t;
  d.mxs = __fmul_rn(mx, inv_t);
  return d;
}

// Mass functions: kind 0 = target P, kind 1 = residual max(P/tp - Q/tq, 0) * 2^40
struct Masses {
  RowDist p, q;
  uint64_t tp, tq;
  int kind;
  __device__ uint64_t operator()(int j) const {
    const uint64_t P = fixed_mass(p.logits[j], p.inv_t, p.mxs);
    if (kind == 0) return P;
    const uint64_t Q = fixed_mass(q.logits[j], q.inv_t, q.mxs);
    const double d = __dsub_rn(__ddiv_rn((double)P, (double)tp), __ddiv_rn((double)Q, (double)tq));
    return d > 0.0 ? (uint64_t)__dmul_rn(d, 1099511627776.0) : 0ull;
  }
};

// Sum of masses over [0, V) (exact).
template <typename F>
__device__ uint64_t block_mass_total(const F& f, int V, uint64_t* shu) {
  const int C = (V + blockDim.x - 1) / blockDim.x;
  const int j0 = threadIdx.x * C, j1 = min(V, j0 + C);
  uint64_t s = 0;
  for (int j = j0; j < j1; ++j) s += f(j);
  uint64_t tot;
  block_exscan_u64(s, shu, &tot);
  return tot;
}

// Smallest j whose inclusive prefix of masses exceeds floor(u * total).
template <typename F>
__device__ int block_inverse_cdf(const F& f, int V, float u, uint64_t* shu, int* shi) {
  const int C = (V + blockDim.x - 1) / blockDim.x;
  const int j0 = threadIdx.x * C, j1 = min(V, j0 + C);
  uint64_t s = 0;
  for (int j = j0; j < j1; ++j) s += f(j);
  uint64_t tot;
  const uint64_t before = block_exscan_u64(s, shu, &tot);
  uint64_t target = (uint64_t)__dmul_rn((double)u, (double)tot);
  if (target >= tot) target = tot > 0 ? tot - 1 : 0;
  __syncthreads();
  if (threadIdx.x == 0) *shi = V - 1;
  __syncthreads();
  if (s > 0 && before <= target && target < before + s) {
    uint64_t c = before;
    for (int j = j0; j < j1; ++j) {
      c += f(j);
      if (c > target) {
        *shi = j;
        break;
      }
    }
  }
  __syncthreads();
  return *shi;
}

__device__ int block_argmax(const float* x, int V, float* shf, int* shi) {
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int j = threadIdx.x; j < V; j += blockDim.x) {
    const float v = x[j];
    if (v > bv || (v == bv && j < bi)) {  // NaN never wins
      bv = v;
      bi = j;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) {
    shf[w] = bv;
    shi[w] = bi;
  }
  __syncthreads();
  float rv = -INFINITY;
  int ri = 0x7fffffff;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i)
    if (shf[i] > rv || (shf[i] == rv && shi[i] < ri)) {
      rv = shf[i];
      ri = shi[i];
    }
  __syncthreads();
  return ri == 0x7fffffff ? 0 : ri;
}

__global__ void __launch_bounds__(kSampThreads) argmax_kernel(const float* logits, int V,
                                                              int32_t* out) {
  pdl_wait();
  __shared__ float shf[32];
  __shared__ int shi[32];
  const int r = block_argmax(logits + (size_t)blockIdx.x * V, V, shf, shi);
  if (threadIdx.x == 0) out[blockIdx.x] = r;
  pdl_launch();
}

__global__ void __launch_bounds__(kSampThreads) sample_kernel(const float* logits, int V,
                                                              float inv_t, int greedy,
                                                              const float* uniforms,
                                                              int32_t* out) {
  pdl_wait();
  __shared__ float shf[32];
  __shared__ int shi[32];
  __shared__ uint64_t shu[32];
  __shared__ int sres;
  const float* row = logits + (size_t)blockIdx.x * V;
  int r;
  if (greedy) {
    r = block_argmax(row, V, shf, shi);
  } else {
    Masses m;
    m.p = make_dist(row, V, inv_t, shf);
    m.q = m.p;
    m.tp = m.tq = 1;
    m.kind = 0;
    r = block_inverse_cdf(m, V, uniforms[blockIdx.x], shu, &sres);
  }
  if (threadIdx.x == 0) out[blockIdx.x] = r;
  pdl_launch();
}

__global__ void __launch_bounds__(kSampThreads) spec_accept_kernel(
    const float* target, const float* draft, const int32_t* dtok, int k, int V, float inv_t,
    int greedy, const float* au, const float* su, int32_t* accepted, int32_t* out_tokens) {
  pdl_wait();
  __shared__ float shf[32];
  __shared__ int shi[32];
  __shared__ uint64_t shu[32];
  __shared__ int sres;
  const int b = blockIdx.x;
  int32_t* ot = out_tokens + (size_t)b * (k + 1);
  for (int i = threadIdx.x; i <= k; i += blockDim.x) ot[i] = -1;
  __syncthreads();
  int n = 0;
  int final_tok = -1;
  if (greedy) {
    for (; n < k; ++n) {
      const int am = block_argmax(target + ((size_t)b * (k + 1) + n) * V, V, shf, shi);
      if (am != dtok[b * k + n]) break;
      if (threadIdx.x == 0) ot[n] = am;
    }
    final_tok = block_argmax(target + ((size_t)b * (k + 1) + n) * V, V, shf, shi);
  } else {
    bool rejected = false;
    for (; n < k; ++n) {
      const int x = dtok[b * k + n];
      Masses m;
      m.p = make_dist(target + ((size_t)b * (k + 1) + n) * V, V, inv_t, shf);
      m.q = make_dist(draft + ((size_t)b * k + n) * V, V, inv_t, shf);
      m.kind = 0;
      m.tp = block_mass_total(m, V, shu);
      Masses mq = m;
      mq.p = m.q;
      const uint64_t tq = block_mass_total(mq, V, shu);
      m.tq = tq;
      const bool in_range = x >= 0 && x < V;
      const double Px = in_range ? (double)fixed_mass(m.p.logits[x], inv_t, m.p.mxs) : 0.0;
      const double Qx = in_range ? (double)fixed_mass(m.q.logits[x], inv_t, m.q.mxs) : 0.0;
      const double lhs = __dmul_rn((double)au[b * k + n], __dmul_rn(Qx, (double)m.tp));
      const double rhs = __dmul_rn(Px, (double)tq);
      if (!(lhs < rhs)) {
        m.kind = 1;
        const uint64_t rt = block_mass_total(m, V, shu);
        if (rt == 0) {
          m.kind = 0;
          final_tok = block_inverse_cdf(m, V, su[b], shu, &sres);
        } else {
          final_tok = block_inverse_cdf(m, V, su[b], shu, &sres);
        }
        rejected = true;
        break;
      }
      if (threadIdx.x == 0) ot[n] = x;
    }
    if (!rejected) {
      Masses m;
      m.p = make_dist(target + ((size_t)b * (k + 1) + k) * V, V, inv_t, shf);
      m.q = m.p;
      m.tp = m.tq = 1;
      m.kind = 0;
      final_tok = block_inverse_cdf(m, V, su[b], shu, &sres);
    }
  }
  if (threadIdx.x == 0) {
    ot[n] = final_tok;
    accepted[b] = n;
  }
  pdl_launch();
}

__global__ void penalties_kernel(float* logits, int V, const int32_t* hist, const int32_t* lens,
                                 int max_hist, float rep, float freq, float pres) {
  pdl_wait();
  const int b = blockIdx.x;
  const int n = min(lens[b], max_hist);
  const int32_t* h = hist + (size_t)b * max_hist;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int tok = h[i];
    if (tok < 0 || tok >= V) continue;
    bool first = true;
    int cnt = 0;
    for (int j = 0; j < n; ++j) {
      if (h[j] == tok) {
        if (j < i) first = false;
        ++cnt;
      }
    }
    if (!first) continue;
    float l = logits[(size_t)b * V + tok];
    if (rep != 1.0f) l = l > 0.0f ? __fmul_rn(l, 1.0f / rep) : __fmul_rn(l, rep);
    if (freq != 0.0f) l = __fsub_rn(l, __fmul_rn(freq, (float)cnt));
    if (pres != 0.0f) l = __fsub_rn(l, pres);
    logits[(size_t)b * V + tok] = l;
  }
  pdl_launch();
}

}  // namespace higgs

using namespace higgs;

extern "C" int higgs_argmax(higgs_ctx* ctx, const float* logits, int B, int V, int32_t* out,
                            void* stream) {
  HG_CHECK_ARG(ctx && logits && out, "higgs_argmax: null argument");
  HG_CHECK_ARG(B >= 0 && V > 0, "higgs_argmax: bad shape");
  if (B == 0) return HIGGS_OK;
  HG_CUDA(launch_pdl(argmax_kernel, dim3(B), dim3(kSampThreads), 0, (cudaStream_t)stream, logits,
                     V, out));
  return HIGGS_OK;
}

extern "C" int higgs_sample(higgs_ctx* ctx, const float* logits, int B, int V, float temperature,
                            const float* uniforms, int32_t* out, void* stream) {
  HG_CHECK_ARG(ctx && logits && out, "higgs_sample: null argument");
  HG_CHECK_ARG(B >= 0 && V > 0, "higgs_sample: bad shape");
  HG_CHECK_ARG(temperature >= 0.0f, "higgs_sample: negative temperature");
  HG_CHECK_ARG(temperature == 0.0f || uniforms, "higgs_sample: uniforms required when T > 0");
  if (B == 0) return HIGGS_OK;
  const int greedy = temperature == 0.0f;
  const float inv_t = greedy ? 1.0f : 1.0f / temperature;
  HG_CUDA(launch_pdl(sample_kernel, dim3(B), dim3(kSampThreads), 0, (cudaStream_t)stream, logits,
                     V, inv_t, greedy, uniforms, out));
  return HIGGS_OK;
}

extern "C" int higgs_spec_accept(higgs_ctx* ctx, const float* target_logits,
                                 const float* draft_logits, const int32_t* draft_tokens, int B,
                                 int k, int V, float temperature, const float* accept_uniforms,
                                 const float* sample_uniforms, int32_t* accepted,
                                 int32_t* out_tokens, void* stream) {
  HG_CHECK_ARG(ctx && target_logits && draft_tokens && accepted && out_tokens,
               "higgs_spec_accept: null argument");
  HG_CHECK_ARG(B >= 0 && k >= 1 && V > 0, "higgs_spec_accept: bad shape");
  HG_CHECK_ARG(temperature >= 0.0f, "higgs_spec_accept: negative temperature");
  HG_CHECK_ARG(temperature == 0.0f || (draft_logits && accept_uniforms && sample_uniforms),
               "higgs_spec_accept: draft logits and uniforms required when T > 0");
  if (B == 0) return HIGGS_OK;
  const int greedy = temperature == 0.0f;
  const float inv_t = greedy ? 1.0f : 1.0f / temperature;
  HG_CUDA(launch_pdl(spec_accept_kernel, dim3(B), dim3(kSampThreads), 0, (cudaStream_t)stream,
                     target_logits, draft_logits, draft_tokens, k, V, inv_t, greedy,
                     accept_uniforms, sample_uniforms, accepted, out_tokens));
  return HIGGS_OK;
}

extern "C" int higgs_apply_penalties(higgs_ctx* ctx, float* logits, int B, int V,
                                     const int32_t* history, const int32_t* hist_lens,
                                     int max_hist, float rep, float freq, float pres,
                                     void* stream) {
  HG_CHECK_ARG(ctx && logits, "higgs_apply_penalties: null argument");
  HG_CHECK_ARG(B >= 0 && V > 0 && max_hist >= 0, "higgs_apply_penalties: bad shape");
  HG_CHECK_ARG(max_hist == 0 || (history && hist_lens), "higgs_apply_penalties: null history");
  HG_CHECK_ARG(rep > 0.0f, "higgs_apply_penalties: repetition penalty must be > 0");
  if (B == 0 || max_hist == 0) return HIGGS_OK;
  HG_CUDA(launch_pdl(penalties_kernel, dim3(B), dim3(256), 0, (cudaStream_t)stream, logits, V,
                     history, hist_lens, max_hist, rep, freq, pres));
  return HIGGS_OK;
}
