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
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace higgs {

constexpr int kSampThreads = 1024;


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

// Greedy argmax of one row split across a cluster of kArgmaxCluster CTAs: each
// CTA reduces a slice to a single u64 key, then CTA 0 reads the others' keys
// through distributed shared memory.  key = (ordered value bits << 32) |
// (~index), so the u64 maximum is the largest value and, among equal values,
// the lowest index; NaN maps to the smallest key (it wins only when the whole
// row is NaN, giving index 0) and -0 is folded onto +0 so they compare equal.
constexpr int kArgmaxCluster = 8;
constexpr int kArgmaxThreads = 512;


__global__ void __cluster_dims__(kArgmaxCluster, 1, 1) __launch_bounds__(kArgmaxThreads)
    argmax_cluster_kernel(const float* logits, int V, int offset, int32_t* out,
                          unsigned long long* key_out) {
  __shared__ unsigned long long warp_best[kArgmaxThreads / 32];
  __shared__ unsigned long long cta_best;
  const int rank = blockIdx.x;  // cluster spans the whole x dimension
  const float* row = logits + (size_t)blockIdx.y * V;
  // slice bounds on 4-float boundaries so vector loads stay aligned
  const int nv4 = V / 4;
  const int per = (nv4 + kArgmaxCluster - 1) / kArgmaxCluster;
  const int v0 = rank * per, v1 = min(nv4, v0 + per);
  const bool vec = ((reinterpret_cast<uintptr_t>(row) & 15) == 0);
  pdl_wait();
  unsigned long long best = 0ull;
  if (vec) {
    const float4* r4 = reinterpret_cast<const float4*>(row);
    int i = v0 + threadIdx.x;
    for (; i + 3 * kArgmaxThreads < v1; i += 4 * kArgmaxThreads) {
      float4 q[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) q[u] = __ldg(r4 + i + u * kArgmaxThreads);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int j = 4 * (i + u * kArgmaxThreads);
        best = max(best, argmax_key(q[u].x, offset + j));
        best = max(best, argmax_key(q[u].y, offset + j + 1));
        best = max(best, argmax_key(q[u].z, offset + j + 2));
        best = max(best, argmax_key(q[u].w, offset + j + 3));
      }
    }
    for (; i < v1; i += kArgmaxThreads) {
      const float4 q = __ldg(r4 + i);
      const int j = offset + 4 * i;
      best = max(best, argmax_key(q.x, j));
      best = max(best, argmax_key(q.y, j + 1));
      best = max(best, argmax_key(q.z, j + 2));
      best = max(best, argmax_key(q.w, j + 3));
    }
    // the V % 4 tail belongs to the last CTA
    if (rank == kArgmaxCluster - 1)
      for (int j = 4 * nv4 + threadIdx.x; j < V; j += kArgmaxThreads)
        best = max(best, argmax_key(row[j], offset + j));
  } else {
    const int per1 = (V + kArgmaxCluster - 1) / kArgmaxCluster;
    const int e = min(V, (rank + 1) * per1);
    for (int j = rank * per1 + threadIdx.x; j < e; j += kArgmaxThreads)
      best = max(best, argmax_key(row[j], offset + j));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
  if ((threadIdx.x & 31) == 0) warp_best[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x < 32) {
    unsigned long long b = threadIdx.x < kArgmaxThreads / 32 ? warp_best[threadIdx.x] : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) b = max(b, __shfl_xor_sync(0xffffffffu, b, o));
    if (threadIdx.x == 0) cta_best = b;
  }
  pdl_launch();
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  if (rank == 0 && threadIdx.x < 32) {
    unsigned long long b = 0ull;
    if (threadIdx.x < kArgmaxCluster) b = *cluster.map_shared_rank(&cta_best, threadIdx.x);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) b = max(b, __shfl_xor_sync(0xffffffffu, b, o));
    if (threadIdx.x == 0) {
      if (key_out) key_out[blockIdx.y] = b;
      else out[blockIdx.y] = (int32_t)(0xFFFFFFFFu - (uint32_t)(b & 0xFFFFFFFFull));
    }
  }
  cluster.sync();  // peers keep their shared memory until CTA 0 has read it
}

// ---- one row over a cluster of CTAs ------------------------------------------
// Sampling and speculative acceptance of a row spread over the kRowCluster CTAs of a
// thread-block cluster: CTA r owns the slice [r * per, min(V, (r + 1) * per)) of the
// vocabulary, reduces it inside the CTA, and the CTAs combine their results through
// distributed shared memory (each writes its value into its own slot of an alternating
// pair, the cluster syncs, threads 0-7 read the 8 slots).  Every combined quantity is a
// maximum, an exact u64 sum or a minimum, so each CTA holds the same bits, equal to the
// single-CTA kernels' (a draw is the smallest j whose inclusive prefix of masses exceeds
// floor(u * total), whatever the partition).  One sequence used to be one CTA of the 148
// SMs walking its row several times per draft position.
constexpr int kRowCluster = 8;
constexpr int kRowThreads = 512;

struct ClRow {
  int j0, j1;  // this CTA's slice of the row
  int phase;   // exchange slot in use
  uint64_t* xch;  // [2] this CTA's published values
  uint64_t* xin;  // [kRowCluster] the values read back
};

// op 0: u64 sum, 1: u64 max, 2: u64 min
__device__ uint64_t cl_combine(uint64_t v, int op, ClRow& c) {
  cg::cluster_group cl = cg::this_cluster();
  if (threadIdx.x == 0) c.xch[c.phase] = v;
  cl.sync();
  if (threadIdx.x < kRowCluster) c.xin[threadIdx.x] = *cl.map_shared_rank(&c.xch[c.phase], threadIdx.x);
  __syncthreads();
  uint64_t r = c.xin[0];
  for (int q = 1; q < kRowCluster; ++q) {
    const uint64_t o = c.xin[q];
    r = op == 0 ? r + o : (op == 1 ? (o > r ? o : r) : (o < r ? o : r));
  }
  c.phase ^= 1;
  return r;
}

__device__ __forceinline__ uint64_t f2ord(float f) {  // order-preserving map of a float
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? (uint64_t)(~u) : (uint64_t)(u | 0x80000000u);
}
__device__ __forceinline__ float ord2f(uint64_t o) {
  const uint32_t u = (uint32_t)o;
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}

__device__ RowDist cl_make_dist(const float* logits, float inv_t, float* shf, ClRow& c) {
  float mx = -INFINITY;
  for (int j = c.j0 + threadIdx.x; j < c.j1; j += blockDim.x) mx = fmaxf(mx, logits[j]);
  mx = block_max(mx, shf);
  mx = ord2f(cl_combine(f2ord(mx), 1, c));
  RowDist d;
  d.logits = logits;
  d.inv_t = inv_t;
  d.mxs = __fmul_rn(mx, inv_t);
  return d;
}

template <typename F>
__device__ uint64_t cl_mass_total(const F& f, uint64_t* shu, ClRow& c) {
  const int n = c.j1 - c.j0;
  const int C = (n + blockDim.x - 1) / blockDim.x;
  const int a = c.j0 + threadIdx.x * C, e = min(c.j1, a + C);
  uint64_t s = 0;
  for (int j = a; j < e; ++j) s += f(j);
  uint64_t tot;
  block_exscan_u64(s, shu, &tot);
  return cl_combine(tot, 0, c);
}

// Smallest j whose inclusive prefix of masses exceeds floor(u * total); V - 1 if none.
template <typename F>
__device__ int cl_inverse_cdf(const F& f, int V, float u, uint64_t* shu, int* shi, ClRow& c) {
  const int n = c.j1 - c.j0;
  const int C = (n + blockDim.x - 1) / blockDim.x;
  const int a = c.j0 + threadIdx.x * C, e = min(c.j1, a + C);
  uint64_t s = 0;
  for (int j = a; j < e; ++j) s += f(j);
  uint64_t cta_tot;
  const uint64_t before = block_exscan_u64(s, shu, &cta_tot);
  // every CTA's total: the slices before this one and the whole row
  cg::cluster_group cl = cg::this_cluster();
  if (threadIdx.x == 0) c.xch[c.phase] = cta_tot;
  cl.sync();
  if (threadIdx.x < kRowCluster) c.xin[threadIdx.x] = *cl.map_shared_rank(&c.xch[c.phase], threadIdx.x);
  __syncthreads();
  c.phase ^= 1;
  const int rank = (int)cl.block_rank();
  uint64_t below = 0, tot = 0;
  for (int q = 0; q < kRowCluster; ++q) {
    if (q < rank) below += c.xin[q];
    tot += c.xin[q];
  }
  uint64_t target = (uint64_t)__dmul_rn((double)u, (double)tot);
  if (target >= tot) target = tot > 0 ? tot - 1 : 0;
  if (threadIdx.x == 0) *shi = 0x7fffffff;
  __syncthreads();
  const uint64_t mine = below + before;
  if (s > 0 && mine <= target && target < mine + s) {
    uint64_t acc = mine;
    for (int j = a; j < e; ++j) {
      acc += f(j);
      if (acc > target) {
        *shi = j;
        break;
      }
    }
  }
  __syncthreads();
  const int r = (int)cl_combine((uint64_t)(uint32_t)*shi, 2, c);
  return r == 0x7fffffff ? V - 1 : r;
}

__device__ int cl_argmax(const float* x, unsigned long long* shk, ClRow& c) {
  unsigned long long best = 0ull;
  for (int j = c.j0 + threadIdx.x; j < c.j1; j += blockDim.x) best = max(best, argmax_key(x[j], j));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) shk[threadIdx.x >> 5] = best;
  __syncthreads();
  unsigned long long b = 0ull;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) b = max(b, shk[w]);
  b = cl_combine(b, 1, c);
  return (int)(0xFFFFFFFFu - (uint32_t)(b & 0xFFFFFFFFull));
}

__device__ __forceinline__ ClRow cl_row(int V, uint64_t* xch, uint64_t* xin) {
  ClRow c;
  const int per = (V + kRowCluster - 1) / kRowCluster;
  const int r = (int)cg::this_cluster().block_rank();
  c.j0 = min(V, r * per);
  c.j1 = min(V, c.j0 + per);
  c.phase = 0;
  c.xch = xch;
  c.xin = xin;
  return c;
}

// sample() at T > 0 for one row per cluster (the plain draw, no filters)
__global__ void __cluster_dims__(kRowCluster, 1, 1) __launch_bounds__(kRowThreads)
    sample_cluster_kernel(const float* logits, int V, float inv_t, const float* uniforms, int32_t* out) {
  __shared__ float shf[32];
  __shared__ int shi;
  __shared__ uint64_t shu[32];
  __shared__ uint64_t xch[2], xin[kRowCluster];
  pdl_wait();
  ClRow c = cl_row(V, xch, xin);
  const float* row = logits + (size_t)blockIdx.y * V;
  Masses m;
  m.p = cl_make_dist(row, inv_t, shf, c);
  m.q = m.p;
  m.tp = m.tq = 1;
  m.kind = 0;
  const int r = cl_inverse_cdf(m, V, uniforms[blockIdx.y], shu, &shi, c);
  if (blockIdx.x == 0 && threadIdx.x == 0) out[blockIdx.y] = r;
  pdl_launch();
  cg::this_cluster().sync();  // peers keep their shared memory until every read is done
}

// Speculative acceptance of one sequence per cluster: the rule of spec_accept_kernel with
// every row reduction spread over the cluster.  draft_stride: elements between the draft
// rows of consecutive positions of one sequence (V for [B, k, V], B * V for [k, B, V]).
__global__ void __cluster_dims__(kRowCluster, 1, 1) __launch_bounds__(kRowThreads)
    spec_accept_cluster_kernel(const float* target, const float* draft, size_t draft_stride,
                               size_t draft_seq, const int32_t* dtok, int k, int V, float inv_t,
                               int greedy, const float* au, const float* su, int32_t* accepted,
                               int32_t* out_tokens) {
  __shared__ float shf[32];
  __shared__ int shi;
  __shared__ uint64_t shu[32];
  __shared__ unsigned long long shk[kRowThreads / 32];
  __shared__ uint64_t xch[2], xin[kRowCluster];
  pdl_wait();
  const int b = blockIdx.y;
  const bool writer = blockIdx.x == 0 && threadIdx.x == 0;
  ClRow c = cl_row(V, xch, xin);
  int32_t* ot = out_tokens + (size_t)b * (k + 1);
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i <= k; i += blockDim.x) ot[i] = -1;
  const float* trow = target + (size_t)b * (k + 1) * V;
  const float* drow = draft ? draft + (size_t)b * draft_seq : nullptr;
  int n = 0;
  int final_tok = -1;
  if (greedy) {
    for (; n < k; ++n) {
      const int am = cl_argmax(trow + (size_t)n * V, shk, c);
      if (am != dtok[b * k + n]) break;
      if (writer) ot[n] = am;
    }
    final_tok = cl_argmax(trow + (size_t)n * V, shk, c);
  } else {
    bool rejected = false;
    for (; n < k; ++n) {
      const int x = dtok[b * k + n];
      Masses m;
      m.p = cl_make_dist(trow + (size_t)n * V, inv_t, shf, c);
      m.q = cl_make_dist(drow + (size_t)n * draft_stride, inv_t, shf, c);
      m.kind = 0;
      m.tp = cl_mass_total(m, shu, c);
      Masses mq = m;
      mq.p = m.q;
      const uint64_t tq = cl_mass_total(mq, shu, c);
      m.tq = tq;
      const bool in_range = x >= 0 && x < V;
      const double Px = in_range ? (double)fixed_mass(m.p.logits[x], inv_t, m.p.mxs) : 0.0;
      const double Qx = in_range ? (double)fixed_mass(m.q.logits[x], inv_t, m.q.mxs) : 0.0;
      const double lhs = __dmul_rn((double)au[b * k + n], __dmul_rn(Qx, (double)m.tp));
      const double rhs = __dmul_rn(Px, (double)tq);
      if (!(lhs < rhs)) {
        m.kind = 1;
        const uint64_t rt = cl_mass_total(m, shu, c);
        if (rt == 0) m.kind = 0;  // no residual mass: draw from the target distribution
        final_tok = cl_inverse_cdf(m, V, su[b], shu, &shi, c);
        rejected = true;
        break;
      }
      if (writer) ot[n] = x;
    }
    if (!rejected) {
      Masses m;
      m.p = cl_make_dist(trow + (size_t)k * V, inv_t, shf, c);
      m.q = m.p;
      m.tp = m.tq = 1;
      m.kind = 0;
      final_tok = cl_inverse_cdf(m, V, su[b], shu, &shi, c);
    }
  }
  if (writer) {
    ot[n] = final_tok;
    accepted[b] = n;
  }
  pdl_launch();
  cg::this_cluster().sync();  // peers keep their shared memory until every read is done
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

cudaError_t launch_argmax_keys(const float* logits, int B, int V, int offset, unsigned long long* keys,
                               cudaStream_t st) {
  return launch_pdl(argmax_cluster_kernel, dim3(kArgmaxCluster, B), dim3(kArgmaxThreads), 0, st,
                    logits, V, offset, (int32_t*)nullptr, keys);
}

// ---------------------------------------------------------------------------
// Filtered sampling: top-k / top-p / min-p (sample_filtered, lib.rs:392-460).
//
// One row per cluster of kFiltCtas CTAs; CTA r owns a contiguous slice of the
// vocabulary and keeps its fixed-point masses E_j in shared memory.  Tokens are
// ranked by the 57-bit key (E_j << 24) | (2^24 - 1 - j): mass descending, ties
// to the lower index.  Every filter keeps a prefix of that order, so the kept
// set is {j : key_j >= theta}; theta comes from radix selections over the keys
// (8-bit digits, top down): by count for the top-k boundary (the key of rank
// k - 1), by mass for the top-p boundary (the first key whose inclusive mass
// prefix exceeds top_p * S); min-p is a bound on E alone.  Per digit pass each
// warp histograms its keys (shared atomics), the CTA folds its warps, and every
// CTA of the cluster reads the kFiltCtas CTA histograms through distributed
// shared memory and takes the same decision.  The draw is the inverse CDF of
// the kept masses in index order (the rule of sample_kernel).
// ---------------------------------------------------------------------------
constexpr int kFiltCtas = 8;
constexpr int kFiltThreads = 512;
constexpr int kFiltWarps = kFiltThreads / 32;
constexpr int kFiltSlice = 20480;  // vocabulary entries per CTA: V <= 163840
constexpr size_t kFiltSmem = (size_t)kFiltSlice * 8 + (size_t)kFiltWarps * 256 * 8 + 256 * 8 * 2;

__device__ __forceinline__ uint64_t filt_key(uint64_t E, int j) {
  return (E << 24) | (uint64_t)(0xFFFFFF - j);
}

// Returns the largest bucket d whose cumulative value (strictly-above total
// `above` plus the buckets > d plus bucket d) exceeds `target` (count mode:
// an integer rank; mass mode: a double bound), and the cumulative strictly
// above d; d = -1 when no bucket does.  Warp 0 only.
__device__ __forceinline__ int filt_bucket(const uint64_t* h, uint64_t above, double target,
                                           uint64_t* above_out) {
  const int lane = threadIdx.x & 31;
  uint64_t v[8], tot = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[i] = h[lane * 8 + i];
    tot += v[i];
  }
  // exclusive suffix sum over lanes above this one
  uint64_t suf = tot;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t lo = __shfl_down_sync(0xffffffffu, (uint32_t)suf, o);
    const uint32_t hi = __shfl_down_sync(0xffffffffu, (uint32_t)(suf >> 32), o);
    if (lane + o < 32) suf += ((uint64_t)hi << 32) | lo;
  }
  uint64_t c = above + (suf - tot);  // everything in higher lanes
  int found = -1;
  uint64_t found_above = 0;
#pragma unroll
  for (int i = 7; i >= 0; --i) {
    if (found < 0 && (double)(c + v[i]) > target) {
      found = lane * 8 + i;
      found_above = c;
    }
    c += v[i];
  }
  const unsigned m = __ballot_sync(0xffffffffu, found >= 0);
  if (m == 0) return -1;
  const int src = 31 - __clz(m);
  const int d = __shfl_sync(0xffffffffu, found, src);
  const uint64_t fa = ((uint64_t)__shfl_sync(0xffffffffu, (uint32_t)(found_above >> 32), src) << 32) |
                      __shfl_sync(0xffffffffu, (uint32_t)found_above, src);
  *above_out = fa;
  return d;
}

struct FiltArgs {
  const float* logits;
  int V;
  float inv_t;
  int top_k;     // 1..V-1 to filter, else off
  float top_p;   // < 1 to filter
  float min_p;   // > 0 to filter (clamped to 1)
  const float* uniforms;
  int32_t* out;
};

__global__ void __cluster_dims__(kFiltCtas, 1, 1) __launch_bounds__(kFiltThreads)
    sample_filtered_kernel(FiltArgs a) {
  extern __shared__ __align__(16) unsigned char filt_smem[];
  uint64_t* E = reinterpret_cast<uint64_t*>(filt_smem);
  uint64_t* whist = E + kFiltSlice;                // [warps][256]
  uint64_t* cta_hist = whist + kFiltWarps * 256;   // [256], read by the cluster
  uint64_t* comb = cta_hist + 256;                 // [256], this CTA's copy of the cluster sum
  __shared__ float red_f[32];
  __shared__ uint64_t red_u[32];
  __shared__ float cta_max;
  __shared__ uint64_t cta_sum, cta_top, cta_kept;
  __shared__ int sel_d;
  __shared__ uint64_t sel_above;

  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int V = a.V;
  const float* row = a.logits + (size_t)blockIdx.y * V;
  const int per = (V + kFiltCtas - 1) / kFiltCtas;
  const int v0 = rank * per;
  const int n = max(0, min(V - v0, per));
  const int C = (n + kFiltThreads - 1) / kFiltThreads;  // contiguous chunk per thread
  const int i0 = min(n, (int)threadIdx.x * C), i1 = min(n, i0 + C);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_wait();

  // 1. row maximum
  float mx = -INFINITY;
  for (int i = i0; i < i1; ++i) mx = fmaxf(mx, row[v0 + i]);
  mx = block_max(mx, red_f);
  if (threadIdx.x == 0) cta_max = mx;
  cluster.sync();
  mx = -INFINITY;
  for (int r = 0; r < kFiltCtas; ++r) mx = fmaxf(mx, *cluster.map_shared_rank(&cta_max, r));
  const float mxs = __fmul_rn(mx, a.inv_t);

  // 2. fixed-point masses, their sum and the top key
  uint64_t s = 0, top = 0;
  for (int i = i0; i < i1; ++i) {
    const uint64_t e = fixed_mass(row[v0 + i], a.inv_t, mxs);
    E[i] = e;
    s += e;
    top = max(top, filt_key(e, v0 + i));
  }
  uint64_t tot;
  block_exscan_u64(s, red_u, &tot);
  __syncthreads();
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint32_t lo = __shfl_xor_sync(0xffffffffu, (uint32_t)top, o);
    const uint32_t hi = __shfl_xor_sync(0xffffffffu, (uint32_t)(top >> 32), o);
    top = max(top, ((uint64_t)hi << 32) | lo);
  }
  if (lane == 0) red_u[warp] = top;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint64_t t = 0;
    for (int w = 0; w < kFiltWarps; ++w) t = max(t, red_u[w]);
    cta_top = t;
    cta_sum = tot;
  }
  cluster.sync();
  uint64_t S = 0;
  top = 0;
  for (int r = 0; r < kFiltCtas; ++r) {
    S += *cluster.map_shared_rank(&cta_sum, r);
    top = max(top, *cluster.map_shared_rank(&cta_top, r));
  }

  // 3. the kept-set threshold
  uint64_t theta = 0;
  if (a.min_p > 0.0f) {
    const double t = __dmul_rn((double)fminf(a.min_p, 1.0f), (double)(top >> 24));
    theta = max(theta, (uint64_t)ceil(t) << 24);
  }
  for (int mode = 0; mode < 2; ++mode) {
    // mode 0: top-k (count), mode 1: top-p (mass)
    if (mode == 0 && !(a.top_k >= 1 && a.top_k < V)) continue;
    if (mode == 1 && !(a.top_p < 1.0f)) continue;
    const double target = mode == 0 ? (double)(a.top_k - 1) : __dmul_rn((double)a.top_p, (double)S);
    uint64_t prefix = 0, above = 0;
    bool all = false;
    for (int shift = 56; shift >= 0; shift -= 8) {
      for (int i = threadIdx.x; i < kFiltWarps * 256; i += kFiltThreads) whist[i] = 0;
      __syncthreads();
      uint64_t* wh = whist + warp * 256;
      for (int i = i0; i < i1; ++i) {
        const uint64_t key = filt_key(E[i], v0 + i);
        if (shift < 56 && (key >> (shift + 8)) != (prefix >> (shift + 8))) continue;
        const int d = (int)((key >> shift) & 255);
        atomicAdd((unsigned long long*)&wh[d], mode == 0 ? 1ull : (unsigned long long)E[i]);
      }
      __syncthreads();
      if (threadIdx.x < 256) {
        uint64_t h = 0;
        for (int w = 0; w < kFiltWarps; ++w) h += whist[w * 256 + threadIdx.x];
        cta_hist[threadIdx.x] = h;
      }
      cluster.sync();
      if (threadIdx.x < 256) {
        uint64_t h = 0;
        for (int r = 0; r < kFiltCtas; ++r) h += cluster.map_shared_rank(cta_hist, r)[threadIdx.x];
        comb[threadIdx.x] = h;
      }
      cluster.sync();  // every CTA has read the histograms before they are rebuilt
      if (warp == 0) {
        uint64_t ab = 0;
        const int d = filt_bucket(comb, above, target, &ab);
        if (lane == 0) {
          sel_d = d;
          sel_above = ab;
        }
      }
      __syncthreads();
      if (sel_d < 0) {  // mass mode: every remaining key stays within top_p
        all = true;
        break;
      }
      prefix |= (uint64_t)sel_d << shift;
      above = sel_above;
      __syncthreads();
    }
    if (mode == 0) {
      theta = max(theta, prefix);  // the key of rank k - 1
    } else if (!all) {
      theta = max(theta, prefix == top ? top : prefix + 1);  // rank 0 always stays
    }
  }

  // 4. inverse CDF of the kept masses in index order
  uint64_t w = 0;
  for (int i = i0; i < i1; ++i)
    if (filt_key(E[i], v0 + i) >= theta) w += E[i];
  uint64_t kept;
  const uint64_t before = block_exscan_u64(w, red_u, &kept);
  if (threadIdx.x == 0) cta_kept = kept;
  cluster.sync();
  uint64_t off = 0, total = 0;
  for (int r = 0; r < kFiltCtas; ++r) {
    const uint64_t t = *cluster.map_shared_rank(&cta_kept, r);
    if (r < rank) off += t;
    total += t;
  }
  if (total == 0) {
    if (rank == 0 && threadIdx.x == 0) a.out[blockIdx.y] = 0xFFFFFF - (int)(top & 0xFFFFFF);
  } else {
    uint64_t target = (uint64_t)__dmul_rn((double)a.uniforms[blockIdx.y], (double)total);
    if (target >= total) target = total - 1;
    if (target >= off && target < off + kept) {
      const uint64_t t = target - off;
      if (w > 0 && before <= t && t < before + w) {
        uint64_t c = before;
        for (int i = i0; i < i1; ++i) {
          if (filt_key(E[i], v0 + i) < theta) continue;
          c += E[i];
          if (c > t) {
            a.out[blockIdx.y] = v0 + i;
            break;
          }
        }
      }
    }
  }
  pdl_launch();
  cluster.sync();  // peers keep their shared memory until every CTA has read it
}

// ---------------------------------------------------------------------------
// LogprobArrays::compute (lib.rs:495-533): log-softmax of the scaled logits,
// the chosen token's value and the top_n largest.  Z = sum of
// floor(det_exp(s_j - m) * 2^44) is an exact integer; lp_j = f32((double)
// (s_j - m) - log(Z * 2^-44)).  The top_n come from top_n block maxima over
// the ordered (value, lower index first) keys.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kSampThreads) logprobs_kernel(const float* logits, int V, float inv_t,
                                                                const int32_t* tokens, int top_n,
                                                                float* token_lp, int32_t* top_ids,
                                                                float* top_lp) {
  pdl_wait();
  __shared__ float shf[32];
  __shared__ uint64_t shu[32];
  __shared__ unsigned long long shk[32];
  const int b = blockIdx.x;
  const float* row = logits + (size_t)b * V;
  float m = -INFINITY;
  for (int j = threadIdx.x; j < V; j += blockDim.x) m = fmaxf(m, __fmul_rn(row[j], inv_t));
  m = block_max(m, shf);
  uint64_t z = 0;
  for (int j = threadIdx.x; j < V; j += blockDim.x)
    z += (uint64_t)__dmul_rn((double)det_exp(__fsub_rn(__fmul_rn(row[j], inv_t), m)), 17592186044416.0);
  uint64_t Z;
  block_exscan_u64(z, shu, &Z);
  const double L = log(__dmul_rn((double)Z, 5.684341886080801486968994140625e-14));
  if (threadIdx.x == 0) {
    const int t = tokens[b];
    token_lp[b] = (t >= 0 && t < V)
                      ? (float)__dsub_rn((double)__fsub_rn(__fmul_rn(row[t], inv_t), m), L)
                      : -INFINITY;
  }
  unsigned long long prev = ~0ull;
  for (int i = 0; i < top_n; ++i) {
    unsigned long long best = 0ull;
    bool any = false;
    for (int j = threadIdx.x; j < V; j += blockDim.x) {
      const unsigned long long k = argmax_key(__fmul_rn(row[j], inv_t), j);
      if (k < prev && (!any || k > best)) {
        best = k;
        any = true;
      }
    }
    // keys are unique per index, so 0 doubles as "none" only for an exhausted row
    best = any ? best + 1 : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) shk[threadIdx.x >> 5] = best;
    __syncthreads();
    best = 0ull;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) best = max(best, shk[w]);
    if (best == 0ull) {
      if (threadIdx.x == 0) {
        top_ids[(size_t)b * top_n + i] = -1;
        top_lp[(size_t)b * top_n + i] = -INFINITY;
      }
      continue;
    }
    best -= 1;
    prev = best;
    const int j = (int)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull));
    if (threadIdx.x == 0) {
      top_ids[(size_t)b * top_n + i] = j;
      top_lp[(size_t)b * top_n + i] =
          (float)__dsub_rn((double)__fsub_rn(__fmul_rn(row[j], inv_t), m), L);
    }
  }
  pdl_launch();
}

// Constraint::apply_mask (constrained.rs:79-110): logits += allowed ? 0 : -inf.
__global__ void token_mask_kernel(float* logits, int V, const uint32_t* allowed, int words) {
  pdl_wait();
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  const int b = blockIdx.y;
  if (j < V) {
    const uint32_t w = allowed[(size_t)b * words + (j >> 5)];
    float* l = logits + (size_t)b * V + j;
    *l = __fadd_rn(*l, ((w >> (j & 31)) & 1u) ? 0.0f : -INFINITY);
  }
  pdl_launch();
}

}  // namespace higgs

using namespace higgs;

extern "C" int higgs_argmax(higgs_ctx* ctx, const float* logits, int B, int V, int32_t* out,
                            void* stream) {
  HG_CHECK_ARG(ctx && logits && out, "higgs_argmax: null argument");
  HG_CHECK_ARG(B >= 0 && V > 0, "higgs_argmax: bad shape");
  HG_DEVICE(ctx);
  if (B == 0) return HIGGS_OK;
  HG_CHECK_ARG(B <= 65535, "higgs_argmax: B > 65535");
  HG_CUDA(launch_pdl(argmax_cluster_kernel, dim3(kArgmaxCluster, B), dim3(kArgmaxThreads), 0,
                     (cudaStream_t)stream, logits, V, 0, out, (unsigned long long*)nullptr));
  return HIGGS_OK;
}

extern "C" int higgs_sample(higgs_ctx* ctx, const float* logits, int B, int V, float temperature,
                            const float* uniforms, int32_t* out, void* stream) {
  HG_CHECK_ARG(ctx && logits && out, "higgs_sample: null argument");
  HG_CHECK_ARG(B >= 0 && V > 0, "higgs_sample: bad shape");
  HG_CHECK_ARG(temperature >= 0.0f, "higgs_sample: negative temperature");
  HG_CHECK_ARG(temperature == 0.0f || uniforms, "higgs_sample: uniforms required when T > 0");
  HG_DEVICE(ctx);
  if (B == 0) return HIGGS_OK;
  HG_CHECK_ARG(B <= 65535, "higgs_sample: B > 65535");
  cudaStream_t st = (cudaStream_t)stream;
  if (temperature == 0.0f) {
    HG_CUDA(launch_pdl(argmax_cluster_kernel, dim3(kArgmaxCluster, B), dim3(kArgmaxThreads), 0, st,
                       logits, V, 0, out, (unsigned long long*)nullptr));
    return HIGGS_OK;
  }
  HG_CUDA(launch_pdl(sample_cluster_kernel, dim3(kRowCluster, B), dim3(kRowThreads), 0, st, logits, V,
                     1.0f / temperature, uniforms, out));
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
  HG_DEVICE(ctx);
  if (B == 0) return HIGGS_OK;
  HG_CHECK_ARG(B <= 65535, "higgs_spec_accept: B > 65535");
  const int greedy = temperature == 0.0f;
  const float inv_t = greedy ? 1.0f : 1.0f / temperature;
  HG_CUDA(launch_pdl(spec_accept_cluster_kernel, dim3(kRowCluster, B), dim3(kRowThreads), 0,
                     (cudaStream_t)stream, target_logits, draft_logits, (size_t)V, (size_t)k * V,
                     draft_tokens, k, V, inv_t, greedy, accept_uniforms, sample_uniforms, accepted,
                     out_tokens));
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
  HG_DEVICE(ctx);
  if (B == 0 || max_hist == 0) return HIGGS_OK;
  HG_CUDA(launch_pdl(penalties_kernel, dim3(B), dim3(256), 0, (cudaStream_t)stream, logits, V,
                     history, hist_lens, max_hist, rep, freq, pres));
  return HIGGS_OK;
}

extern "C" int higgs_sample_filtered(higgs_ctx* ctx, const float* logits, int B, int V,
                                     float temperature, int top_k, float top_p, float min_p,
                                     const float* uniforms, int32_t* out, void* stream) {
  HG_CHECK_ARG(ctx && logits && out, "higgs_sample_filtered: null argument");
  HG_CHECK_ARG(B >= 0 && V > 0, "higgs_sample_filtered: bad shape");
  HG_CHECK_ARG(B <= 65535, "higgs_sample_filtered: B > 65535");
  HG_CHECK_ARG(temperature >= 0.0f, "higgs_sample_filtered: negative temperature");
  HG_CHECK_ARG(temperature == 0.0f || uniforms, "higgs_sample_filtered: uniforms required when T > 0");
  HG_CHECK_ARG(top_k >= 0, "higgs_sample_filtered: negative top_k");
  HG_CHECK_ARG(top_p >= 0.0f, "higgs_sample_filtered: negative top_p");
  HG_CHECK_ARG(V <= kFiltCtas * kFiltSlice,
               "higgs_sample_filtered: V above 163840 (the per-row shared-memory capacity)");
  HG_DEVICE(ctx);
  if (B == 0) return HIGGS_OK;
  cudaStream_t st = (cudaStream_t)stream;
  if (temperature == 0.0f) {
    HG_CUDA(launch_pdl(argmax_cluster_kernel, dim3(kArgmaxCluster, B), dim3(kArgmaxThreads), 0, st,
                       logits, V, 0, out, (unsigned long long*)nullptr));
    return HIGGS_OK;
  }
  const float inv_t = 1.0f / temperature;
  const bool filt = (top_k >= 1 && top_k < V) || top_p < 1.0f || min_p > 0.0f;
  if (!filt) {  // no filter keeps every token: the plain draw
    HG_CUDA(launch_pdl(sample_cluster_kernel, dim3(kRowCluster, B), dim3(kRowThreads), 0, st, logits, V,
                       inv_t, uniforms, out));
    return HIGGS_OK;
  }
  static PerDeviceOnce attr;
  HG_CUDA(attr.run([] {
    return cudaFuncSetAttribute(sample_filtered_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)kFiltSmem);
  }));
  FiltArgs a;
  a.logits = logits;
  a.V = V;
  a.inv_t = inv_t;
  a.top_k = top_k;
  a.top_p = top_p;
  a.min_p = min_p;
  a.uniforms = uniforms;
  a.out = out;
  HG_CUDA(launch_pdl(sample_filtered_kernel, dim3(kFiltCtas, B), dim3(kFiltThreads), kFiltSmem, st, a));
  return HIGGS_OK;
}

extern "C" int higgs_logprobs(higgs_ctx* ctx, const float* logits, int B, int V, float temperature,
                              const int32_t* tokens, int top_n, float* token_logprob,
                              int32_t* top_ids, float* top_logprobs, void* stream) {
  HG_CHECK_ARG(ctx && logits && tokens && token_logprob, "higgs_logprobs: null argument");
  HG_CHECK_ARG(B >= 0 && V > 0 && top_n >= 0, "higgs_logprobs: bad shape");
  HG_CHECK_ARG(top_n == 0 || (top_ids && top_logprobs), "higgs_logprobs: null top-n outputs");
  HG_CHECK_ARG(temperature >= 0.0f, "higgs_logprobs: negative temperature");
  HG_DEVICE(ctx);
  if (B == 0) return HIGGS_OK;
  // simple.rs:269-275: unscaled at T <= f32::EPSILON, else logits * (1 / T)
  const float inv_t = temperature <= 1.1920928955078125e-7f ? 1.0f : 1.0f / temperature;
  HG_CUDA(launch_pdl(logprobs_kernel, dim3(B), dim3(kSampThreads), 0, (cudaStream_t)stream, logits, V,
                     inv_t, tokens, top_n, token_logprob, top_ids, top_logprobs));
  return HIGGS_OK;
}

extern "C" int higgs_apply_token_mask(higgs_ctx* ctx, float* logits, int B, int V,
                                      const uint32_t* allowed, int words_per_row, void* stream) {
  HG_CHECK_ARG(ctx && logits && allowed, "higgs_apply_token_mask: null argument");
  HG_CHECK_ARG(B >= 0 && V > 0, "higgs_apply_token_mask: bad shape");
  HG_CHECK_ARG(B <= 65535, "higgs_apply_token_mask: B > 65535");
  HG_CHECK_ARG((int64_t)words_per_row * 32 >= V, "higgs_apply_token_mask: mask rows shorter than V bits");
  HG_DEVICE(ctx);
  if (B == 0) return HIGGS_OK;
  HG_CUDA(launch_pdl(token_mask_kernel, dim3((V + 255) / 256, B), dim3(256), 0, (cudaStream_t)stream,
                     logits, V, allowed, words_per_row));
  return HIGGS_OK;
}
