// norm_rope.cu -- RMSNorm (+ residual add), RoPE, and the fused
// q/k-norm + RoPE + paged-KV append (bf16 or TurboQuant 4-bit pages).
//
// Reference ops replaced: nn::RmsNorm / fast::rms_norm (transformer.rs:375-377,
// 407, 415, 525; qk-norm 193-207), fast::rope (utils.rs:16-26) and the cache
// append of SteppingKeyValueCache::update_and_fetch (cache.rs:236-311).
#include "common.cuh"

namespace higgs {

// ---------------------------------------------------------------------------
// RMSNorm: one CTA per row, 16-byte vectors.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) rmsnorm_kernel(const uint16_t* x, const uint16_t* res,
                                                      int H, const uint16_t* w, float eps,
                                                      uint16_t* y, uint16_t* h_out,
                                                      int64_t in_stride) {
  pdl_wait();
  const int r = blockIdx.x;
  const int nv = H / 8;
  __shared__ float red[8];
  // H <= 8192 -> at most 4 vectors per thread
  float h[4][8];
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int vi = threadIdx.x + i * 256;
    if (vi < nv) {
      const uint4 xv = *reinterpret_cast<const uint4*>(x + (size_t)r * in_stride + vi * 8);
      const uint32_t* xp = &xv.x;
      uint4 rv = make_uint4(0, 0, 0, 0);
      if (res) rv = *reinterpret_cast<const uint4*>(res + (size_t)r * H + vi * 8);
      const uint32_t* rp = &rv.x;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float a = bf_lo(xp[j]), b = bf_hi(xp[j]);
        if (res) {
          a = round_bf(a + bf_lo(rp[j]));
          b = round_bf(b + bf_hi(rp[j]));
        }
        h[i][2 * j] = a;
        h[i][2 * j + 1] = b;
        ss += a * a + b * b;
      }
      if (h_out) {
        uint4 o;
        uint32_t* op = &o.x;
#pragma unroll
        for (int j = 0; j < 4; ++j) op[j] = pack_bf2(h[i][2 * j], h[i][2 * j + 1]);
        *reinterpret_cast<uint4*>(h_out + (size_t)r * H + vi * 8) = o;
      }
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float inv = 1.0f / sqrtf(tot / (float)H + eps);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int vi = threadIdx.x + i * 256;
    if (vi < nv) {
      const uint4 wv = *reinterpret_cast<const uint4*>(w + vi * 8);
      const uint32_t* wp = &wv.x;
      uint4 o;
      uint32_t* op = &o.x;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        op[j] = pack_bf2(h[i][2 * j] * inv * bf_lo(wp[j]), h[i][2 * j + 1] * inv * bf_hi(wp[j]));
      *reinterpret_cast<uint4*>(y + (size_t)r * H + vi * 8) = o;
    }
  }
  pdl_launch();
}

// ---------------------------------------------------------------------------
// One warp per (token, head).  Lane l owns elements i = l*E + e of the first
// half and i + D/2 of the second half (E = D/64), so a RoPE pair is lane-local.
// ---------------------------------------------------------------------------
template <int D>
__device__ __forceinline__ void load_head(const uint16_t* src, int lane, float (&lo)[D / 64],
                                          float (&hi)[D / 64]) {
  constexpr int E = D / 64;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    lo[e] = bf2f(src[lane * E + e]);
    hi[e] = bf2f(src[D / 2 + lane * E + e]);
  }
}

template <int D>
__device__ __forceinline__ void head_rmsnorm(float (&lo)[D / 64], float (&hi)[D / 64],
                                             const uint16_t* w, float eps, int lane) {
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
__device__ __forceinline__ void head_rope(float (&lo)[D / 64], float (&hi)[D / 64], int pos,
                                          const float* inv_freq, int lane) {
  constexpr int E = D / 64;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const float th = (float)pos * inv_freq[lane * E + e];
    float s, c;
    sincosf(th, &s, &c);
    const float a = lo[e], b = hi[e];
    lo[e] = round_bf(a * c - b * s);
    hi[e] = round_bf(b * c + a * s);
  }
}

template <int D>
__device__ __forceinline__ void store_head(uint16_t* dst, int lane, const float (&lo)[D / 64],
                                           const float (&hi)[D / 64]) {
  constexpr int E = D / 64;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    dst[lane * E + e] = f2bf(lo[e]);
    dst[D / 2 + lane * E + e] = f2bf(hi[e]);
  }
}

template <int D>
__global__ void rope_kernel(const uint16_t* x, int rows, int heads, const int32_t* pos,
                            const float* inv_freq, uint16_t* y) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int item = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (item < rows * heads) {
    const int r = item / heads;
    float lo[D / 64], hi[D / 64];
    load_head<D>(x + (size_t)item * D, lane, lo, hi);
    head_rope<D>(lo, hi, pos[r], inv_freq, lane);
    store_head<D>(y + (size_t)item * D, lane, lo, hi);
  }
  pdl_launch();
}

struct KvWriteArgs {
  const uint16_t* qkv;
  int T, Hq, Hkv;
  const uint16_t* qn;
  const uint16_t* kn;
  float eps;
  const int32_t* pos;
  const float* inv_freq;
  const int64_t* slots;
  uint16_t* kc;
  uint16_t* vc;
  int64_t page_stride, head_stride;
  uint16_t* q_out;
  // TurboQuant cache (D = 128)
  const int8_t* signs;
  uint8_t* kcode;
  __half* kscale;
  uint8_t* vcode;
  __half* vscale;
};

// TurboQuant encode of one 128-vector held as lane l: elements 2l, 2l+1 (lo)
// and 64+2l, 65+2l (hi).  The butterfly order and every rounding match
// orc_tq4_encode in the oracle bit for bit (explicit _rn intrinsics keep the
// compiler from fusing anything).
__device__ __forceinline__ void tq4_encode_lane(const float (&lo_in)[2], const float (&hi_in)[2],
                                                const int8_t* signs, int lane, uint8_t* codes,
                                                __half* scale) {
  float f[4] = {lo_in[0], lo_in[1], hi_in[0], hi_in[1]};
  const int idx[4] = {2 * lane, 2 * lane + 1, 64 + 2 * lane, 65 + 2 * lane};
#pragma unroll
  for (int e = 0; e < 4; ++e)
    if (signs[idx[e]] < 0) f[e] = -f[e];
  // stage h = 1: pairs (2l, 2l+1) are lane-local
  {
    float a = f[0], b = f[1];
    f[0] = __fadd_rn(a, b);
    f[1] = __fsub_rn(a, b);
    a = f[2];
    b = f[3];
    f[2] = __fadd_rn(a, b);
    f[3] = __fsub_rn(a, b);
  }
  // stages h = 2..32: partner lane l ^ (h/2)
#pragma unroll
  for (int hl = 1; hl <= 16; hl <<= 1) {
    const bool upper = (lane & hl) != 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float other = __shfl_xor_sync(0xffffffffu, f[e], hl);
      f[e] = upper ? __fsub_rn(other, f[e]) : __fadd_rn(f[e], other);
    }
  }
  // stage h = 64: (i, i + 64) lane-local
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const float a = f[e], b = f[e + 2];
    f[e] = __fadd_rn(a, b);
    f[e + 2] = __fsub_rn(a, b);
  }
  float amax = 0.0f;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    f[e] = __fmul_rn(f[e], 0.0883883476483184406f);
    amax = fmaxf(amax, fabsf(f[e]));
  }
  amax = warp_max(amax);
  const __half sh = __float2half_rn(__fdiv_rn(amax, 7.0f));
  const float s = __half2float(sh);
  int c[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    if (s == 0.0f) {
      c[e] = 8;
    } else {
      float v = rintf(__fdiv_rn(f[e], s));
      v = fminf(fmaxf(v, -8.0f), 7.0f);
      c[e] = (int)v + 8;
    }
  }
  codes[lane] = (uint8_t)(c[0] | (c[1] << 4));
  codes[32 + lane] = (uint8_t)(c[2] | (c[3] << 4));
  if (lane == 0) *scale = sh;
}

template <int D, bool TQ>
__global__ void qknorm_rope_kv_kernel(KvWriteArgs a) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int nh = a.Hq + 2 * a.Hkv;
  const int item = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (item < a.T * nh) {
    const int t = item / nh, h = item % nh;
    const uint16_t* src = a.qkv + (size_t)t * nh * D + (size_t)h * D;
    float lo[D / 64], hi[D / 64];
    load_head<D>(src, lane, lo, hi);
    const int64_t slot = a.slots ? a.slots[t] : -1;
    const int64_t page = slot >= 0 ? slot / HIGGS_PAGE_SIZE : 0;
    const int s_in = slot >= 0 ? (int)(slot % HIGGS_PAGE_SIZE) : 0;
    if (h < a.Hq) {
      if (a.qn) head_rmsnorm<D>(lo, hi, a.qn, a.eps, lane);
      head_rope<D>(lo, hi, a.pos[t], a.inv_freq, lane);
      store_head<D>(a.q_out + ((size_t)t * a.Hq + h) * D, lane, lo, hi);
    } else if (h < a.Hq + a.Hkv) {
      const int hk = h - a.Hq;
      if (a.kn) head_rmsnorm<D>(lo, hi, a.kn, a.eps, lane);
      head_rope<D>(lo, hi, a.pos[t], a.inv_freq, lane);
      if (slot >= 0) {
        if constexpr (TQ) {
          const int64_t base = page * a.page_stride + hk * a.head_stride + (int64_t)s_in * 64;
          const int64_t sidx = page * (a.page_stride / 64) + hk * (a.head_stride / 64) + s_in;
          tq4_encode_lane(lo, hi, a.signs, lane, a.kcode + base, a.kscale + sidx);
        } else {
          store_head<D>(a.kc + page * a.page_stride + hk * a.head_stride + (int64_t)s_in * D, lane,
                        lo, hi);
        }
      }
    } else {
      const int hk = h - a.Hq - a.Hkv;
      if (slot >= 0) {
        if constexpr (TQ) {
          const int64_t base = page * a.page_stride + hk * a.head_stride + (int64_t)s_in * 64;
          const int64_t sidx = page * (a.page_stride / 64) + hk * (a.head_stride / 64) + s_in;
          tq4_encode_lane(lo, hi, a.signs, lane, a.vcode + base, a.vscale + sidx);
        } else {
          store_head<D>(a.vc + page * a.page_stride + hk * a.head_stride + (int64_t)s_in * D, lane,
                        lo, hi);
        }
      }
    }
  }
  pdl_launch();
}

// bare encode: one warp per vector (natural layout [n, 64] codes, [n] scales)
__global__ void tq4_encode_kernel(const uint16_t* x, int64_t n, const int8_t* signs,
                                  uint8_t* codes, __half* scales) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t item = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (item < n) {
    const uint16_t* src = x + item * 128;
    const float lo[2] = {bf2f(src[2 * lane]), bf2f(src[2 * lane + 1])};
    const float hi[2] = {bf2f(src[64 + 2 * lane]), bf2f(src[65 + 2 * lane])};
    tq4_encode_lane(lo, hi, signs, lane, codes + item * 64, scales + item);
  }
  pdl_launch();
}

}  // namespace higgs

using namespace higgs;

extern "C" int higgs_rmsnorm(higgs_ctx* ctx, const void* x, const void* residual, int rows, int H,
                             const void* weight, float eps, void* y, void* h_out, void* stream) {
  HG_CHECK_ARG(ctx && x && weight && y, "higgs_rmsnorm: null argument");
  HG_CHECK_ARG(rows >= 0 && H > 0 && H % 8 == 0 && H <= 8192,
               "higgs_rmsnorm: need H % 8 == 0 and H <= 8192");
  HG_DEVICE(ctx);
  if (rows == 0) return HIGGS_OK;
  HG_CUDA(launch_pdl(rmsnorm_kernel, dim3(rows), dim3(256), 0, (cudaStream_t)stream,
                     (const uint16_t*)x, (const uint16_t*)residual, H, (const uint16_t*)weight, eps,
                     (uint16_t*)y, (uint16_t*)h_out, (int64_t)H));
  return HIGGS_OK;
}

extern "C" int higgs_rmsnorm_strided(higgs_ctx* ctx, const void* x, int64_t in_stride, int rows,
                                     int H, const void* weight, float eps, void* y, void* stream) {
  HG_CHECK_ARG(ctx && x && weight && y, "higgs_rmsnorm_strided: null argument");
  HG_CHECK_ARG(rows >= 0 && H > 0 && H % 8 == 0 && H <= 8192 && in_stride >= H && in_stride % 8 == 0,
               "higgs_rmsnorm_strided: need H % 8 == 0, H <= 8192, in_stride >= H, in_stride % 8 == 0");
  HG_DEVICE(ctx);
  if (rows == 0) return HIGGS_OK;
  HG_CUDA(launch_pdl(rmsnorm_kernel, dim3(rows), dim3(256), 0, (cudaStream_t)stream,
                     (const uint16_t*)x, (const uint16_t*)nullptr, H, (const uint16_t*)weight, eps,
                     (uint16_t*)y, (uint16_t*)nullptr, in_stride));
  return HIGGS_OK;
}

extern "C" int higgs_rope(higgs_ctx* ctx, const void* x, int rows, int heads, int D,
                          const int32_t* positions, const float* inv_freq, void* y, void* stream) {
  HG_CHECK_ARG(ctx && x && positions && inv_freq && y, "higgs_rope: null argument");
  HG_CHECK_ARG(D == 64 || D == 128, "higgs_rope: D must be 64 or 128");
  HG_CHECK_ARG(rows >= 0 && heads > 0, "higgs_rope: bad shape");
  HG_DEVICE(ctx);
  if (rows == 0) return HIGGS_OK;
  const int items = rows * heads;
  dim3 grid((items + 3) / 4);
  cudaStream_t st = (cudaStream_t)stream;
  if (D == 64)
    HG_CUDA(launch_pdl(rope_kernel<64>, grid, dim3(128), 0, st, (const uint16_t*)x, rows, heads,
                       positions, inv_freq, (uint16_t*)y));
  else
    HG_CUDA(launch_pdl(rope_kernel<128>, grid, dim3(128), 0, st, (const uint16_t*)x, rows, heads,
                       positions, inv_freq, (uint16_t*)y));
  return HIGGS_OK;
}

extern "C" int higgs_qknorm_rope_kv_write(higgs_ctx* ctx, const void* qkv, int T, int Hq, int Hkv,
                                          int D, const void* q_norm_w, const void* k_norm_w,
                                          float eps, const int32_t* positions,
                                          const float* inv_freq, const int64_t* slot_mapping,
                                          void* k_cache, void* v_cache, int64_t page_stride,
                                          int64_t head_stride, void* q_out, void* stream) {
  HG_CHECK_ARG(ctx && qkv && positions && inv_freq && q_out, "higgs_qknorm_rope_kv_write: null argument");
  HG_CHECK_ARG(!slot_mapping || (k_cache && v_cache), "higgs_qknorm_rope_kv_write: null cache");
  HG_CHECK_ARG(D == 64 || D == 128, "higgs_qknorm_rope_kv_write: D must be 64 or 128");
  HG_CHECK_ARG(T >= 0 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0, "higgs_qknorm_rope_kv_write: bad heads");
  HG_CHECK_ARG((q_norm_w == nullptr) == (k_norm_w == nullptr),
               "higgs_qknorm_rope_kv_write: give both q and k norm weights or neither");
  HG_DEVICE(ctx);
  if (T == 0) return HIGGS_OK;
  KvWriteArgs a = {};
  a.qkv = (const uint16_t*)qkv;
  a.T = T;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.qn = (const uint16_t*)q_norm_w;
  a.kn = (const uint16_t*)k_norm_w;
  a.eps = eps;
  a.pos = positions;
  a.inv_freq = inv_freq;
  a.slots = slot_mapping;
  a.kc = (uint16_t*)k_cache;
  a.vc = (uint16_t*)v_cache;
  a.page_stride = page_stride;
  a.head_stride = head_stride;
  a.q_out = (uint16_t*)q_out;
  const int items = T * (Hq + 2 * Hkv);
  dim3 grid((items + 3) / 4);
  cudaStream_t st = (cudaStream_t)stream;
  if (D == 64)
    HG_CUDA(launch_pdl(qknorm_rope_kv_kernel<64, false>, grid, dim3(128), 0, st, a));
  else
    HG_CUDA(launch_pdl(qknorm_rope_kv_kernel<128, false>, grid, dim3(128), 0, st, a));
  return HIGGS_OK;
}

extern "C" int higgs_qknorm_rope_kv_write_tq4(
    higgs_ctx* ctx, const void* qkv, int T, int Hq, int Hkv, const void* q_norm_w,
    const void* k_norm_w, float eps, const int32_t* positions, const float* inv_freq,
    const int64_t* slot_mapping, const int8_t* signs, uint8_t* k_codes, void* k_scales,
    uint8_t* v_codes, void* v_scales, int64_t page_stride, int64_t head_stride, void* q_out,
    void* stream) {
  HG_CHECK_ARG(ctx && qkv && positions && inv_freq && q_out && signs,
               "higgs_qknorm_rope_kv_write_tq4: null argument");
  HG_CHECK_ARG(!slot_mapping || (k_codes && k_scales && v_codes && v_scales),
               "higgs_qknorm_rope_kv_write_tq4: null cache");
  HG_CHECK_ARG(T >= 0 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0,
               "higgs_qknorm_rope_kv_write_tq4: bad heads");
  HG_CHECK_ARG(page_stride % 64 == 0 && head_stride % 64 == 0,
               "higgs_qknorm_rope_kv_write_tq4: strides must be multiples of 64 bytes");
  HG_CHECK_ARG((q_norm_w == nullptr) == (k_norm_w == nullptr),
               "higgs_qknorm_rope_kv_write_tq4: give both q and k norm weights or neither");
  HG_DEVICE(ctx);
  if (T == 0) return HIGGS_OK;
  KvWriteArgs a = {};
  a.qkv = (const uint16_t*)qkv;
  a.T = T;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.qn = (const uint16_t*)q_norm_w;
  a.kn = (const uint16_t*)k_norm_w;
  a.eps = eps;
  a.pos = positions;
  a.inv_freq = inv_freq;
  a.slots = slot_mapping;
  a.page_stride = page_stride;
  a.head_stride = head_stride;
  a.q_out = (uint16_t*)q_out;
  a.signs = signs;
  a.kcode = k_codes;
  a.kscale = (__half*)k_scales;
  a.vcode = v_codes;
  a.vscale = (__half*)v_scales;
  const int items = T * (Hq + 2 * Hkv);
  HG_CUDA(launch_pdl(qknorm_rope_kv_kernel<128, true>, dim3((items + 3) / 4), dim3(128), 0,
                     (cudaStream_t)stream, a));
  return HIGGS_OK;
}

extern "C" int higgs_tq4_encode(higgs_ctx* ctx, const void* x, int64_t n, const int8_t* signs,
                                uint8_t* codes, void* scales, void* stream) {
  HG_CHECK_ARG(ctx && x && signs && codes && scales, "higgs_tq4_encode: null argument");
  HG_CHECK_ARG(n >= 0, "higgs_tq4_encode: bad count");
  HG_DEVICE(ctx);
  if (n == 0) return HIGGS_OK;
  HG_CUDA(launch_pdl(tq4_encode_kernel, dim3((unsigned)((n + 3) / 4)), dim3(128), 0,
                     (cudaStream_t)stream, (const uint16_t*)x, n, signs, codes, (__half*)scales));
  return HIGGS_OK;
}
