/*
 * higgs_oracle.c -- CPU restatement of the higgs decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * path in higgs_b200/ and the timed CPU baseline in bench.py.  The product
 * (libhiggs_cuda.so and everything that ships) never links, loads or calls
 * it; only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * --impl reference legs may.
 *
 * The reference (panbanda/higgs) does all of its arithmetic inside the
 * third-party MLX library (mlx-rs 0.25.3 / mlx-sys 0.2.0, git rev af21d79,
 * Cargo.lock:1931-1958), which is not vendored and cannot be built here (no
 * Rust toolchain, no Metal).  Each function below restates the published
 * algorithm of the MLX op that a reference call site uses, citing that call
 * site.  Parity is pinned by the reference's own known-answer tests
 * (tests/test_oracle_kat.py); the quantizer rounding, the TurboQuant KV codes,
 * paged KV and speculative acceptance have no reference code, so those are
 * defined here and the CUDA kernels must match them bit for bit.
 *
 * Numeric conventions (mirrored by the CUDA kernels):
 *   - bf16 <-> f32 conversions round to nearest even;
 *   - every op accumulates in f32 and rounds its output once to bf16;
 *   - compiled with -ffp-contract=off so a*b+c is never silently fused: the
 *     places that must be bit-exact (TurboQuant encode, the sampling CDF)
 *     use explicit fmaf() exactly where the CUDA code uses __fmaf_rn().
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* scalar helpers                                                            */
/* ------------------------------------------------------------------------ */

static inline float bf2f(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline uint16_t f2bf(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static inline float round_bf(float f) { return bf2f(f2bf(f)); }

static inline float h2f(uint16_t h) {
  _Float16 v;
  memcpy(&v, &h, 2);
  return (float)v;
}

/*
 * Summation order of the floating-point reductions below that have no order
 * fixed by the reference (MLX leaves them to its kernels): 0 = the order each
 * function documents; 1 = a second, equally valid order (matrix-form lane sums
 * folded in reverse, vector-form groups summed last to first, attention dot
 * products over d in reverse).  Comparing the two measures the rounding noise
 * that any change of summation order alone puts into a bf16 forward -- the
 * floor against which a GPU kernel's different order is judged.  The exact
 * paths (router logits, sampling, TurboQuant codes) are only defined, and
 * only used, at order 0.
 */
static int g_order = 0;
int orc_set_order(int mode) {
  const int old = g_order;
  g_order = mode ? 1 : 0;
  return old;
}

/* OpenMP team size for every parallel loop below; returns the size in force.
 * A launcher may have set OMP_NUM_THREADS=1 in the environment (torchrun does),
 * so the CPU baselines set it explicitly. */
int orc_set_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
  return omp_get_max_threads();
}

static inline uint16_t f2h(float f) {
  _Float16 v = (_Float16)f; /* IEEE round to nearest even */
  uint16_t h;
  memcpy(&h, &v, 2);
  return h;
}

static inline float u2f(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/*
 * Deterministic exp used by every sampling / acceptance computation, so the
 * CUDA kernels (which use the identical sequence of correctly rounded
 * operations) produce bit-identical probabilities.  Method: Cody-Waite range
 * reduction x = k*ln2 + r with a two-part ln2, then the degree-7 Taylor
 * polynomial of e^r in Horner form (truncation error < 6e-9 for |r| <= ln2/2),
 * then scaling by 2^k through the exponent field.
 */
float orc_exp(float x) {
  if (!(x >= -87.0f)) return 0.0f; /* also maps NaN / -inf to 0 */
  if (x > 88.0f) x = 88.0f;
  const float kf = rintf(x * 1.44269504088896341f);
  float r = fmaf(-kf, 0.693145751953125f, x);
  r = fmaf(-kf, 1.42860682030941723e-6f, r);
  float p = 1.98412698412698413e-4f; /* 1/5040 */
  p = fmaf(p, r, 1.38888888888888889e-3f); /* 1/720 */
  p = fmaf(p, r, 8.33333333333333333e-3f); /* 1/120 */
  p = fmaf(p, r, 4.16666666666666667e-2f); /* 1/24 */
  p = fmaf(p, r, 1.66666666666666667e-1f); /* 1/6 */
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  const int k = (int)kf; /* in [-126, 127] */
  return p * u2f((uint32_t)(k + 127) << 23);
}

/* ------------------------------------------------------------------------ */
/* MLX-affine 4-bit, group 64 (reference: qwen3_next.rs:174-183 quantized_matmul,
 * qwen3_next.rs:248-257 dequantize; layout transformer.rs:943-951 after
 * nn::quantize).  weight u32 [N, K/8], element k of a row sits in word k/8 at
 * bits 4*(k%8); scales / biases bf16 [N, K/64]; w = scale*q + bias.          */
/* ------------------------------------------------------------------------ */

/*
 * This build's documented quantizer (the reference never pins ops::quantize's
 * rounding, so synthetic weights are produced by this rule and the packed
 * (q, scales, biases) tensors are the ground truth):
 *   lo = min(group), hi = max(group)
 *   scale = bf16((hi - lo) / 15)   (scale := 1 when that rounds to 0)
 *   bias  = bf16(lo)
 *   q     = clamp(rint((w - bias) / scale), 0, 15)
 */
void orc_w4_quantize(const float* w, int64_t N, int64_t K, uint32_t* q, uint16_t* scales,
                     uint16_t* biases) {
  const int64_t G = K / 64;
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    for (int64_t g = 0; g < G; ++g) {
      const float* src = w + n * K + g * 64;
      float lo = src[0], hi = src[0];
      for (int i = 1; i < 64; ++i) {
        lo = src[i] < lo ? src[i] : lo;
        hi = src[i] > hi ? src[i] : hi;
      }
      uint16_t sb = f2bf((hi - lo) / 15.0f);
      if (bf2f(sb) == 0.0f) sb = f2bf(1.0f);
      const uint16_t bb = f2bf(lo);
      const float s = bf2f(sb), b = bf2f(bb);
      scales[n * G + g] = sb;
      biases[n * G + g] = bb;
      for (int w8 = 0; w8 < 8; ++w8) {
        uint32_t word = 0;
        for (int j = 0; j < 8; ++j) {
          float v = rintf((src[w8 * 8 + j] - b) / s);
          v = v < 0.0f ? 0.0f : (v > 15.0f ? 15.0f : v);
          word |= ((uint32_t)v) << (4 * j);
        }
        q[n * (K / 8) + g * 8 + w8] = word;
      }
    }
  }
}

/* Unpack the 4-bit codes of an [N, K/8] u32 tensor to bytes [N, K]. */
void orc_w4_unpack(const uint32_t* q, int64_t N, int64_t K, uint8_t* out) {
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n)
    for (int64_t k = 0; k < K; ++k) out[n * K + k] = (q[n * (K / 8) + k / 8] >> (4 * (k % 8))) & 0xF;
}

/* ops::dequantize (qwen3_next.rs:249-256): bf16(scale*q + bias), one rounding. */
void orc_w4_dequantize(const uint32_t* q, const uint16_t* scales, const uint16_t* biases,
                       int64_t N, int64_t K, uint16_t* out) {
  const int64_t G = K / 64;
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n)
    for (int64_t k = 0; k < K; ++k) {
      const float s = bf2f(scales[n * G + k / 64]), b = bf2f(biases[n * G + k / 64]);
      const float qv = (float)((q[n * (K / 8) + k / 8] >> (4 * (k % 8))) & 0xF);
      out[n * K + k] = f2bf(s * qv + b);
    }
}

/* QEmbedding::forward (qwen3_next.rs:248-257): dequantize then take rows. */
void orc_embed_gather(const int32_t* ids, int64_t n_ids, const uint32_t* q, const uint16_t* scales,
                      const uint16_t* biases, int64_t V, int64_t H, uint16_t* out) {
  const int64_t G = H / 64;
  for (int64_t i = 0; i < n_ids; ++i) {
    const int64_t r = ids[i];
    if (r < 0 || r >= V) {
      for (int64_t k = 0; k < H; ++k) out[i * H + k] = 0;
      continue;
    }
    for (int64_t k = 0; k < H; ++k) {
      const float s = bf2f(scales[r * G + k / 64]), b = bf2f(biases[r * G + k / 64]);
      const float qv = (float)((q[r * (H / 8) + k / 8] >> (4 * (k % 8))) & 0xF);
      out[i * H + k] = f2bf(s * qv + b);
    }
  }
}

/*
 * ops::quantized_matmul(x, w, scales, biases, transpose=true, 64, 4)
 * (qwen3_next.rs:174-183; QLinear::forward qwen3_next.rs:211-220).  MLX's
 * published matrix-vector algorithm accumulates, per group, sum(x*q) and
 * sum(x) in f32 and folds them as scale*sum(x*q) + bias*sum(x).  y is f32
 * [M, N] (y_f32, optional) and bf16 [M, N] (y_bf16, optional).
 */
void orc_qmatmul(const uint16_t* x, int64_t M, int64_t K, const uint32_t* q,
                 const uint16_t* scales, const uint16_t* biases, int64_t N, float* y_f32,
                 uint16_t* y_bf16) {
  const int64_t G = K / 64;
  float* xf = (float*)malloc(sizeof(float) * (size_t)(M * K));
  for (int64_t i = 0; i < M * K; ++i) xf[i] = bf2f(x[i]);
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    const uint32_t* row = q + n * (K / 8);
    for (int64_t m = 0; m < M; ++m) {
      const float* xr = xf + m * K;
      float acc = 0.0f;
      for (int64_t gi = 0; gi < G; ++gi) {
        const int64_t g = g_order == 0 ? gi : G - 1 - gi;
        float sxq = 0.0f, sx = 0.0f;
        for (int w8 = 0; w8 < 8; ++w8) {
          const uint32_t word = row[g * 8 + w8];
          for (int j = 0; j < 8; ++j) {
            const float xv = xr[g * 64 + w8 * 8 + j];
            sxq += xv * (float)((word >> (4 * j)) & 0xF);
            sx += xv;
          }
        }
        acc += bf2f(scales[n * G + g]) * sxq + bf2f(biases[n * G + g]) * sx;
      }
      if (y_f32) y_f32[m * N + n] = acc;
      if (y_bf16) y_bf16[m * N + n] = f2bf(acc);
    }
  }
  free(xf);
}

/*
 * The matrix (many-token) form of quantized_matmul: MLX's qmm dequantizes each
 * weight to the activation type before the dot products, so here
 * w = bf16(s*q + b) (one rounding of the exact value) and each output is an
 * f32 dot product in a fixed order: eight lane sums s_j = sum over k = j mod 8
 * (k ascending) of x_k*w_k, then y = ((s0+s1)+(s2+s3)) + ((s4+s5)+(s6+s7)).
 * (MLX's tiled kernels fix no order either; the GPU tests bound the
 * difference.)  The decode form above (qmv) keeps q exact.
 *
 * Blocked for speed only: rows of W are dequantized 16 at a time into an f32
 * panel, and four outputs share each load of x.  The lane structure lets the
 * compiler use 8-wide vectors (an AVX2 clone is picked at run time where the
 * host has it) without reassociating any sum.
 */
#define DQ_ROWS 16
__attribute__((target_clones("avx2", "default")))
static void dq_panel(const float* xf, int64_t M, int64_t K, const float* wp, int nrows,
                     int64_t n0, int64_t N, float* y_f32, uint16_t* y_bf16) {
  for (int64_t m = 0; m < M; ++m) {
    const float* xr = xf + m * K;
    for (int r = 0; r < nrows; r += 4) {
      float acc[4][8];
      for (int i = 0; i < 4; ++i)
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
      const int nr = nrows - r < 4 ? nrows - r : 4;
      for (int64_t k = 0; k < K; k += 8) {
        for (int i = 0; i < 4; ++i) {
          const float* wr = wp + (int64_t)(r + (i < nr ? i : 0)) * K + k;
          for (int j = 0; j < 8; ++j) acc[i][j] += xr[k + j] * wr[j];
        }
      }
      for (int i = 0; i < nr; ++i) {
        const float* a = acc[i];
        const float v = g_order == 0
                            ? ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]))
                            : ((a[7] + a[6]) + (a[5] + a[4])) + ((a[3] + a[2]) + (a[1] + a[0]));
        const int64_t n = n0 + r + i;
        if (y_f32) y_f32[m * N + n] = v;
        if (y_bf16) y_bf16[m * N + n] = f2bf(v);
      }
    }
  }
}

void orc_qmatmul_dq(const uint16_t* x, int64_t M, int64_t K, const uint32_t* q,
                    const uint16_t* scales, const uint16_t* biases, int64_t N, float* y_f32,
                    uint16_t* y_bf16) {
  const int64_t G = K / 64;
  float* xf = (float*)malloc(sizeof(float) * (size_t)(M * K));
  for (int64_t i = 0; i < M * K; ++i) xf[i] = bf2f(x[i]);
  const int64_t panels = (N + DQ_ROWS - 1) / DQ_ROWS;
#pragma omp parallel
  {
    float* wp = (float*)malloc(sizeof(float) * (size_t)(DQ_ROWS * K));
#pragma omp for schedule(dynamic)
    for (int64_t pi = 0; pi < panels; ++pi) {
      const int64_t n0 = pi * DQ_ROWS;
      const int nrows = (int)(N - n0 < DQ_ROWS ? N - n0 : DQ_ROWS);
      for (int r = 0; r < nrows; ++r) {
        const int64_t n = n0 + r;
        const uint32_t* row = q + n * (K / 8);
        for (int64_t k = 0; k < K; ++k) {
          const float sv = bf2f(scales[n * G + k / 64]), bv = bf2f(biases[n * G + k / 64]);
          const float qv = (float)((row[k / 8] >> (4 * (k % 8))) & 0xF);
          wp[r * K + k] = bf2f(f2bf(sv * qv + bv));
        }
      }
      dq_panel(xf, M, K, wp, nrows, n0, N, y_f32, y_bf16);
    }
    free(wp);
  }
  free(xf);
}

/* ------------------------------------------------------------------------ */
/* Norms, residuals, activations                                             */
/* ------------------------------------------------------------------------ */

/*
 * fast::rms_norm via nn::RmsNorm (transformer.rs:375-377,407,415; qk-norm
 * transformer.rs:193-207,264-269):  y = bf16(x * rsqrt(mean(x^2) + eps) * w).
 * With `residual` non-NULL the input is first h = bf16(x + residual)
 * (TransformerBlock::forward transformer.rs:404-418: h = x.add(residual)),
 * and h is written to h_out when that is non-NULL.
 */
void orc_rmsnorm(const uint16_t* x, const uint16_t* residual, int64_t rows, int64_t H,
                 const uint16_t* w, float eps, uint16_t* y, uint16_t* h_out) {
  for (int64_t r = 0; r < rows; ++r) {
    float* h = (float*)malloc(sizeof(float) * (size_t)H);
    double ss = 0.0;
    for (int64_t k = 0; k < H; ++k) {
      float v = bf2f(x[r * H + k]);
      if (residual) v = round_bf(v + bf2f(residual[r * H + k]));
      h[k] = v;
      ss += (double)v * (double)v;
      if (h_out) h_out[r * H + k] = f2bf(v);
    }
    const float inv = 1.0f / sqrtf((float)(ss / (double)H) + eps);
    for (int64_t k = 0; k < H; ++k) y[r * H + k] = f2bf(h[k] * inv * bf2f(w[k]));
    free(h);
  }
}

/*
 * fast::rope, traditional=false, scale=1 (utils.rs:16-26, built at
 * transformer.rs:209-214; per-request offsets transformer.rs:762-779).
 * x: [rows, heads, D] bf16, row r at absolute position pos[r].  For
 * i < D/2: a = x[i], b = x[i + D/2], theta = pos * inv_freq[i]:
 *   out[i] = a cos - b sin,  out[i + D/2] = b cos + a sin.
 * inv_freq[i] = base^(-2i/D) is supplied by the caller (computed once in
 * double and rounded to f32, the same table the CUDA kernel receives).
 */
void orc_rope(const uint16_t* x, int64_t rows, int64_t heads, int64_t D, const int32_t* pos,
              const float* inv_freq, uint16_t* out) {
  const int64_t half = D / 2;
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t h = 0; h < heads; ++h) {
      const uint16_t* xi = x + (r * heads + h) * D;
      uint16_t* o = out + (r * heads + h) * D;
      for (int64_t i = 0; i < half; ++i) {
        const float th = (float)pos[r] * inv_freq[i];
        const float c = cosf(th), s = sinf(th);
        const float a = bf2f(xi[i]), b = bf2f(xi[i + half]);
        o[i] = f2bf(a * c - b * s);
        o[i + half] = f2bf(b * c + a * s);
      }
    }
}

/* swiglu / Mlp::forward (qwen3_next.rs:275-277; transformer.rs:349-353):
 * bf16(silu(g) * u) computed in f32 with one rounding. */
void orc_silu_mul(const uint16_t* g, const uint16_t* u, int64_t n, uint16_t* out) {
  for (int64_t i = 0; i < n; ++i) {
    const float gv = bf2f(g[i]);
    out[i] = f2bf(gv / (1.0f + expf(-gv)) * bf2f(u[i]));
  }
}

/* ------------------------------------------------------------------------ */
/* Attention                                                                 */
/* ------------------------------------------------------------------------ */

/*
 * fast::scaled_dot_product_attention with GQA (utils.rs:45-60), over a paged
 * KV cache (block size `page`).  The reference's masks become positions:
 * query t of sequence b sits at absolute position seq_lens[b] - Lq + t and
 * attends to keys 0..that position (utils.rs:64-73 causal mask with offset;
 * utils.rs:114-125 batched decode mask, j < len_i).
 *   q   [B, Lq, Hq, D] bf16 (after RoPE)
 *   k/v page p, kv head h, slot s at element  p*page_stride + h*head_stride + s*D
 *   block_table [B, max_blocks] int32; out [B, Lq, Hq, D] bf16.
 * Scores and softmax in f32 (libm expf); one bf16 rounding of the output.
 */
void orc_paged_attention(const uint16_t* q, int64_t B, int64_t Lq, int64_t Hq, int64_t Hkv,
                         int64_t D, const uint16_t* kc, const uint16_t* vc, int64_t page,
                         int64_t page_stride, int64_t head_stride, const int32_t* block_table,
                         int64_t max_blocks, const int32_t* seq_lens, float scale, uint16_t* out) {
  const int64_t grp = Hq / Hkv;
#pragma omp parallel for collapse(2) schedule(dynamic)
  for (int64_t b = 0; b < B; ++b)
    for (int64_t hq = 0; hq < Hq; ++hq) {
      const int64_t hk = hq / grp;
      const int64_t L = seq_lens[b];
      float* sc = (float*)malloc(sizeof(float) * (size_t)(L > 0 ? L : 1));
      float* acc = (float*)malloc(sizeof(float) * (size_t)D);
      for (int64_t t = 0; t < Lq; ++t) {
        const int64_t qpos = L - Lq + t;
        const uint16_t* qv = q + ((b * Lq + t) * Hq + hq) * D;
        float mx = -INFINITY;
        for (int64_t j = 0; j <= qpos; ++j) {
          const int64_t pg = block_table[b * max_blocks + j / page];
          const uint16_t* kv = kc + pg * page_stride + hk * head_stride + (j % page) * D;
          float s = 0.0f;
          for (int64_t di = 0; di < D; ++di) {
            const int64_t d = g_order == 0 ? di : D - 1 - di;
            s += bf2f(qv[d]) * bf2f(kv[d]);
          }
          sc[j] = s * scale;
          mx = sc[j] > mx ? sc[j] : mx;
        }
        float den = 0.0f;
        for (int64_t d = 0; d < D; ++d) acc[d] = 0.0f;
        for (int64_t j = 0; j <= qpos; ++j) {
          const float p = expf(sc[j] - mx);
          den += p;
          const int64_t pg = block_table[b * max_blocks + j / page];
          const uint16_t* vv = vc + pg * page_stride + hk * head_stride + (j % page) * D;
          for (int64_t d = 0; d < D; ++d) acc[d] += p * bf2f(vv[d]);
        }
        uint16_t* o = out + ((b * Lq + t) * Hq + hq) * D;
        for (int64_t d = 0; d < D; ++d) o[d] = f2bf(qpos >= 0 ? acc[d] / den : 0.0f);
      }
      free(sc);
      free(acc);
    }
}

/* ------------------------------------------------------------------------ */
/* TurboQuant-style 4-bit KV (no reference code: defined by this build)      */
/* ------------------------------------------------------------------------ */

/*
 * Rotation R = H * diag(sign) / sqrt(128), H the 128-point Sylvester Hadamard
 * matrix applied as 7 in-place butterfly stages (stride 1, 2, ..., 64; each
 * output is one f32 add or subtract, so any parallel schedule of the same
 * stages is bit-identical).
 */
static void tq_rotate(float* f, const int8_t* sign) {
  for (int i = 0; i < 128; ++i)
    if (sign[i] < 0) f[i] = -f[i];
  for (int h = 1; h < 128; h <<= 1)
    for (int i = 0; i < 128; i += 2 * h)
      for (int j = i; j < i + h; ++j) {
        const float a = f[j], b = f[j + h];
        f[j] = a + b;
        f[j + h] = a - b;
      }
  for (int i = 0; i < 128; ++i) f[i] = f[i] * 0.0883883476483184406f; /* 1/sqrt(128) */
}

/* Inverse rotation R^T = diag(sign) * H / sqrt(128). */
static void tq_unrotate(float* f, const int8_t* sign) {
  for (int h = 1; h < 128; h <<= 1)
    for (int i = 0; i < 128; i += 2 * h)
      for (int j = i; j < i + h; ++j) {
        const float a = f[j], b = f[j + h];
        f[j] = a + b;
        f[j + h] = a - b;
      }
  for (int i = 0; i < 128; ++i) {
    f[i] = f[i] * 0.0883883476483184406f;
    if (sign[i] < 0) f[i] = -f[i];
  }
}

/*
 * Encode n head vectors (D = 128, bf16) to 64 bytes of codes + one fp16 scale:
 *   v' = R v (f32);  s = fp16(max|v'| / 7);
 *   c_i = clamp(rint(v'_i / s), -8, 7) + 8;  byte j = c_{2j} | c_{2j+1} << 4.
 * A zero scale stores all codes as 8 (value 0).
 */
void orc_tq4_encode(const uint16_t* x, int64_t n, const int8_t* sign, uint8_t* codes,
                    uint16_t* scales) {
  for (int64_t r = 0; r < n; ++r) {
    float f[128];
    for (int i = 0; i < 128; ++i) f[i] = bf2f(x[r * 128 + i]);
    tq_rotate(f, sign);
    float amax = 0.0f;
    for (int i = 0; i < 128; ++i) {
      const float a = fabsf(f[i]);
      amax = a > amax ? a : amax;
    }
    const uint16_t sh = f2h(amax / 7.0f);
    const float s = h2f(sh);
    scales[r] = sh;
    for (int j = 0; j < 64; ++j) {
      int c[2];
      for (int e = 0; e < 2; ++e) {
        if (s == 0.0f) {
          c[e] = 8;
        } else {
          float v = rintf(f[2 * j + e] / s);
          v = v < -8.0f ? -8.0f : (v > 7.0f ? 7.0f : v);
          c[e] = (int)v + 8;
        }
      }
      codes[r * 64 + j] = (uint8_t)(c[0] | (c[1] << 4));
    }
  }
}

/* Decode back to the original basis (f32): v = R^T ((c - 8) * s). */
void orc_tq4_decode(const uint8_t* codes, const uint16_t* scales, int64_t n, const int8_t* sign,
                    float* out) {
  for (int64_t r = 0; r < n; ++r) {
    float f[128];
    const float s = h2f(scales[r]);
    for (int j = 0; j < 64; ++j) {
      f[2 * j] = (float)((codes[r * 64 + j] & 0xF) - 8) * s;
      f[2 * j + 1] = (float)((codes[r * 64 + j] >> 4) - 8) * s;
    }
    tq_unrotate(f, sign);
    memcpy(out + r * 128, f, sizeof(f));
  }
}

/*
 * Decode attention over TurboQuant pages.  Codes page p, head h, slot s at
 * byte  p*page_stride + h*head_stride + s*64; scales (fp16) at element
 * p*(page_stride/64) + h*(head_stride/64) + s.  Scores use the rotated query
 * q' = R q (an orthogonal R preserves dot products); the output is rotated back
 * with R^T.  Same position / mask semantics as orc_paged_attention.
 */
void orc_paged_attention_tq4(const uint16_t* q, int64_t B, int64_t Lq, int64_t Hq, int64_t Hkv,
                             const uint8_t* kcodes, const uint16_t* kscales,
                             const uint8_t* vcodes, const uint16_t* vscales, int64_t page,
                             int64_t page_stride, int64_t head_stride, const int32_t* block_table,
                             int64_t max_blocks, const int32_t* seq_lens, const int8_t* sign,
                             float scale, uint16_t* out) {
  const int64_t grp = Hq / Hkv, D = 128;
  const int64_t sps = page_stride / 64, shs = head_stride / 64;
#pragma omp parallel for collapse(2) schedule(dynamic)
  for (int64_t b = 0; b < B; ++b)
    for (int64_t hq = 0; hq < Hq; ++hq) {
      const int64_t hk = hq / grp;
      const int64_t L = seq_lens[b];
      float* sc = (float*)malloc(sizeof(float) * (size_t)(L > 0 ? L : 1));
      for (int64_t t = 0; t < Lq; ++t) {
        const int64_t qpos = L - Lq + t;
        float qr[128], acc[128];
        for (int d = 0; d < 128; ++d) qr[d] = bf2f(q[((b * Lq + t) * Hq + hq) * D + d]);
        tq_rotate(qr, sign);
        float mx = -INFINITY;
        for (int64_t j = 0; j <= qpos; ++j) {
          const int64_t pg = block_table[b * max_blocks + j / page];
          const uint8_t* kc = kcodes + pg * page_stride + hk * head_stride + (j % page) * 64;
          const float ks = h2f(kscales[pg * sps + hk * shs + (j % page)]);
          float s = 0.0f;
          for (int d = 0; d < 64; ++d) {
            s += qr[2 * d] * (float)((kc[d] & 0xF) - 8);
            s += qr[2 * d + 1] * (float)((kc[d] >> 4) - 8);
          }
          sc[j] = s * ks * scale;
          mx = sc[j] > mx ? sc[j] : mx;
        }
        float den = 0.0f;
        for (int d = 0; d < 128; ++d) acc[d] = 0.0f;
        for (int64_t j = 0; j <= qpos; ++j) {
          const float p = expf(sc[j] - mx);
          den += p;
          const int64_t pg = block_table[b * max_blocks + j / page];
          const uint8_t* vcc = vcodes + pg * page_stride + hk * head_stride + (j % page) * 64;
          const float w = p * h2f(vscales[pg * sps + hk * shs + (j % page)]);
          for (int d = 0; d < 64; ++d) {
            acc[2 * d] += w * (float)((vcc[d] & 0xF) - 8);
            acc[2 * d + 1] += w * (float)((vcc[d] >> 4) - 8);
          }
        }
        for (int d = 0; d < 128; ++d) acc[d] = qpos >= 0 ? acc[d] / den : 0.0f;
        tq_unrotate(acc, sign);
        uint16_t* o = out + ((b * Lq + t) * Hq + hq) * D;
        for (int d = 0; d < 128; ++d) o[d] = f2bf(acc[d]);
      }
      free(sc);
    }
}

/* ------------------------------------------------------------------------ */
/* Token selection                                                           */
/* ------------------------------------------------------------------------ */

/* sample() with temperature 0 (lib.rs:373-377): argmax over the last axis,
 * ties -> first index (lib.rs:838-843).  NaN never wins. */
void orc_argmax(const float* logits, int64_t B, int64_t V, int32_t* out) {
  for (int64_t b = 0; b < B; ++b) {
    int64_t best = 0;
    float bv = logits[b * V];
    for (int64_t j = 1; j < V; ++j)
      if (logits[b * V + j] > bv || (bv != bv && logits[b * V + j] == logits[b * V + j])) {
        bv = logits[b * V + j];
        best = j;
      }
    out[b] = (int32_t)best;
  }
}

/*
 * Deterministic probability mass: e_j = orc_exp((l_j - max) * inv_t), held as
 * the fixed-point integer E_j = floor(e_j * 2^32) (exact for e_j <= 1), so
 * sums and prefix sums are exact integers whatever the summation order.
 * Returns the total.
 */
static uint64_t fixed_probs(const float* logits, int64_t V, float inv_t, uint64_t* E) {
  float mx = logits[0];
  for (int64_t j = 1; j < V; ++j) mx = logits[j] > mx ? logits[j] : mx;
  const float mxs = mx * inv_t;
  uint64_t tot = 0;
  for (int64_t j = 0; j < V; ++j) {
    const float e = orc_exp(logits[j] * inv_t - mxs);
    E[j] = (uint64_t)((double)e * 4294967296.0);
    tot += E[j];
  }
  return tot;
}

/* Smallest j whose inclusive prefix sum of W exceeds floor(u * total). */
static int64_t inverse_cdf(const uint64_t* W, int64_t V, uint64_t total, float u) {
  uint64_t target = (uint64_t)((double)u * (double)total);
  if (target >= total) target = total - 1;
  uint64_t c = 0;
  for (int64_t j = 0; j < V; ++j) {
    c += W[j];
    if (c > target) return j;
  }
  return V - 1;
}

/*
 * sample() with temperature > 0 (lib.rs:379-384, categorical(logits / T)):
 * one seeded uniform per row drives an inverse-CDF draw over the
 * deterministic fixed-point distribution above.  (MLX's own key stream is not
 * reproducible outside MLX; the uniforms are an explicit input instead.)
 */
void orc_sample(const float* logits, int64_t B, int64_t V, float temperature,
                const float* uniforms, int32_t* out) {
  if (temperature == 0.0f) {
    orc_argmax(logits, B, V, out);
    return;
  }
  const float inv_t = 1.0f / temperature;
  uint64_t* E = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)V);
  for (int64_t b = 0; b < B; ++b) {
    const uint64_t tot = fixed_probs(logits + b * V, V, inv_t, E);
    out[b] = (int32_t)inverse_cdf(E, V, tot, uniforms[b]);
  }
  free(E);
}

/*
 * Speculative acceptance (no reference code; standard speculative sampling).
 * For each sequence b with k draft tokens x_1..x_k:
 *   p_i = softmax(target_logits[b, i] / T) (i = 0..k), q_i = softmax(draft_logits[b, i] / T)
 *   accept x_i while  u_i * q_i(x_i) < p_i(x_i)   (u = accept_uniforms[b, i])
 *   first rejection at i: resample from norm(max(p_i - q_i, 0)) with sample_uniforms[b]
 *   (from p_i when that residual is empty); all accepted: bonus token from p_k.
 * Both comparisons and the residual use the fixed-point masses of
 * fixed_probs(), evaluated in double with the same operation order as the
 * CUDA kernel, so accepted counts are bit-exact given identical uniforms.
 * T == 0 is the greedy limit: accept while x_i == argmax(target_i), then emit
 * argmax(target at the first mismatch / at k).
 * Outputs: accepted[b] in 0..k; out_tokens[b, 0..k] = accepted drafts, then the
 * corrected / bonus token, then -1 padding.
 */
void orc_spec_accept(const float* target_logits, const float* draft_logits,
                     const int32_t* draft_tokens, int64_t B, int64_t k, int64_t V,
                     float temperature, const float* accept_uniforms,
                     const float* sample_uniforms, int32_t* accepted, int32_t* out_tokens) {
  uint64_t* P = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)V);
  uint64_t* Q = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)V);
  uint64_t* R = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)V);
  for (int64_t b = 0; b < B; ++b) {
    int32_t* ot = out_tokens + b * (k + 1);
    for (int64_t i = 0; i <= k; ++i) ot[i] = -1;
    int64_t n = 0;
    if (temperature == 0.0f) {
      int32_t am;
      for (; n < k; ++n) {
        orc_argmax(target_logits + (b * (k + 1) + n) * V, 1, V, &am);
        if (am != draft_tokens[b * k + n]) break;
        ot[n] = am;
      }
      orc_argmax(target_logits + (b * (k + 1) + n) * V, 1, V, &am);
      ot[n] = am;
      accepted[b] = (int32_t)n;
      continue;
    }
    const float inv_t = 1.0f / temperature;
    for (; n < k; ++n) {
      const int32_t x = draft_tokens[b * k + n];
      const uint64_t tp = fixed_probs(target_logits + (b * (k + 1) + n) * V, V, inv_t, P);
      const uint64_t tq = fixed_probs(draft_logits + (b * k + n) * V, V, inv_t, Q);
      const int in_range = x >= 0 && x < V;
      const double Px = in_range ? (double)P[x] : 0.0, Qx = in_range ? (double)Q[x] : 0.0;
      const double lhs = (double)accept_uniforms[b * k + n] * (Qx * (double)tp);
      const double rhs = Px * (double)tq;
      if (!(lhs < rhs)) {
        /* residual max(p - q, 0) in fixed point 2^40 */
        uint64_t rt = 0;
        for (int64_t j = 0; j < V; ++j) {
          const double d = (double)P[j] / (double)tp - (double)Q[j] / (double)tq;
          R[j] = d > 0.0 ? (uint64_t)(d * 1099511627776.0) : 0;
          rt += R[j];
        }
        if (rt == 0)
          ot[n] = (int32_t)inverse_cdf(P, V, tp, sample_uniforms[b]);
        else
          ot[n] = (int32_t)inverse_cdf(R, V, rt, sample_uniforms[b]);
        break;
      }
      ot[n] = x;
    }
    if (n == k) {
      const uint64_t tp = fixed_probs(target_logits + (b * (k + 1) + k) * V, V, inv_t, P);
      ot[k] = (int32_t)inverse_cdf(P, V, tp, sample_uniforms[b]);
    }
    accepted[b] = (int32_t)n;
  }
  free(P);
  free(Q);
  free(R);
}

/*
 * apply_penalties (lib.rs:278-363): for every token id seen in `history`,
 * repetition: positive logits divided by rep, negative multiplied by rep;
 * frequency: subtract freq * count; presence: subtract pres.  In place.
 */
void orc_apply_penalties(float* logits, int64_t V, const int32_t* history, int64_t n_hist,
                         float rep, float freq, float pres) {
  int32_t* cnt = (int32_t*)calloc((size_t)V, sizeof(int32_t));
  for (int64_t i = 0; i < n_hist; ++i)
    if (history[i] >= 0 && history[i] < V) cnt[history[i]]++;
  for (int64_t j = 0; j < V; ++j) {
    if (!cnt[j]) continue;
    float l = logits[j];
    if (rep != 1.0f) l = l > 0.0f ? l * (1.0f / rep) : l * rep;
    if (freq != 0.0f) l = l - freq * (float)cnt[j];
    if (pres != 0.0f) l = l - pres;
    logits[j] = l;
  }
  free(cnt);
}

/*
 * Constraint::apply_mask (crates/higgs-engine/src/constrained.rs:79-110):
 * logits + mask, mask 0 for allowed tokens and -inf for the others.  The
 * allowed set of row b is a bitmask: bit (j % 32) of word j / 32 of
 * allowed[b * words ...] set = token j allowed.  One f32 add per logit.
 */
void orc_apply_token_mask(float* logits, int64_t B, int64_t V, const uint32_t* allowed,
                          int64_t words) {
  for (int64_t b = 0; b < B; ++b)
    for (int64_t j = 0; j < V; ++j) {
      const int on = (allowed[b * words + j / 32] >> (j % 32)) & 1u;
      logits[b * V + j] = logits[b * V + j] + (on ? 0.0f : -INFINITY);
    }
}

/*
 * sample() with top-k / top-p / min-p filtering (lib.rs:373-385 calling
 * sample_filtered lib.rs:392-460), over the same fixed-point masses as
 * orc_sample:
 *   E_j = fixed_probs(logits / T), S = sum E_j;  rank order = E descending,
 *   ties to the lower index (a stable descending sort);
 *   keep rank r iff  r < k  (top_k; 0 = off, clamped to [1, V]),
 *                and (r == 0 or cum_r <= top_p * S)  (cum_r = inclusive sum
 *                    of E over ranks 0..r; off when top_p >= 1),
 *                and E_r >= min_p * E_max  (min_p clamped to [0, 1]; off when
 *                    min_p <= 0);
 *   then an inverse-CDF draw (uniform u, index order, the rule of orc_sample)
 *   over the kept masses.  The products top_p * S and min_p * E_max are IEEE
 *   double; every other quantity is an exact integer.  Each filter keeps a
 *   prefix of the rank order, so the kept set is {j : key_j >= theta} for the
 *   key (E_j << 24) | (2^24 - 1 - j) (V < 2^24).  T == 0 is the argmax.
 */
static int cmp_u64_desc(const void* a, const void* b) {
  const uint64_t x = *(const uint64_t*)a, y = *(const uint64_t*)b;
  return x < y ? 1 : (x > y ? -1 : 0);
}

void orc_sample_filtered(const float* logits, int64_t B, int64_t V, float temperature,
                         int64_t top_k, float top_p, float min_p, const float* uniforms,
                         int32_t* out) {
  if (temperature == 0.0f) {
    orc_argmax(logits, B, V, out);
    return;
  }
  const float inv_t = 1.0f / temperature;
  uint64_t* E = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)V);
  uint64_t* key = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)V);
  for (int64_t b = 0; b < B; ++b) {
    const uint64_t S = fixed_probs(logits + b * V, V, inv_t, E);
    for (int64_t j = 0; j < V; ++j) key[j] = (E[j] << 24) | (uint64_t)(0xFFFFFF - j);
    qsort(key, (size_t)V, sizeof(uint64_t), cmp_u64_desc);
    const int64_t k = (top_k <= 0 || top_k > V) ? V : top_k;
    const double pS = (double)top_p * (double)S;
    const float mp = min_p > 1.0f ? 1.0f : min_p;
    const double thr = (double)mp * (double)(key[0] >> 24);
    int64_t n = 0;
    uint64_t cum = 0;
    for (; n < V; ++n) {
      const uint64_t En = key[n] >> 24;
      cum += En;
      if (n >= k) break;
      if (top_p < 1.0f && n > 0 && !((double)cum <= pS)) break;
      if (min_p > 0.0f && !((double)En >= thr)) break;
    }
    const uint64_t theta = key[n - 1]; /* n >= 1: rank 0 always passes */
    uint64_t tot = 0;
    for (int64_t j = 0; j < V; ++j) {
      const uint64_t kj = (E[j] << 24) | (uint64_t)(0xFFFFFF - j);
      if (kj < theta) E[j] = 0;
      tot += E[j];
    }
    out[b] = (int32_t)inverse_cdf(E, V, tot, uniforms[b]);
  }
  free(E);
  free(key);
}

/*
 * LogprobArrays::compute (lib.rs:495-533): log_softmax of the temperature-
 * scaled logits (s_j = l_j * (1/T), unscaled when T <= FLT_EPSILON as at
 * simple.rs:269-275), the chosen token's log-probability and the top_n
 * largest (ties to the lower index) with their log-probabilities.
 *   m = max s;  Z = sum floor(orc_exp(s_j - m) * 2^44) * 2^-44  (exact sum);
 *   lp_j = f32((double)(s_j - m) - log(Z))   (s_j - m in f32).
 */
void orc_logprobs(const float* logits, int64_t B, int64_t V, float temperature,
                  const int32_t* tokens, int64_t top_n, float* token_lp, int32_t* top_ids,
                  float* top_lp) {
  const float inv_t = temperature <= 1.1920928955078125e-7f ? 1.0f : 1.0f / temperature;
  for (int64_t b = 0; b < B; ++b) {
    const float* l = logits + b * V;
    float m = l[0] * inv_t;
    for (int64_t j = 1; j < V; ++j) {
      const float s = l[j] * inv_t;
      m = s > m ? s : m;
    }
    uint64_t z = 0;
    for (int64_t j = 0; j < V; ++j)
      z += (uint64_t)((double)orc_exp(l[j] * inv_t - m) * 17592186044416.0);
    const double L = log((double)z * 5.684341886080801486968994140625e-14);
    const int32_t t = tokens[b];
    token_lp[b] = (t >= 0 && t < V) ? (float)((double)(l[t] * inv_t - m) - L) : -INFINITY;
    /* top_n by (s_j, lower index first) */
    int64_t prev = -1;
    float prev_s = INFINITY;
    for (int64_t i = 0; i < top_n; ++i) {
      int64_t best = -1;
      float bs = -INFINITY;
      for (int64_t j = 0; j < V; ++j) {
        const float s = l[j] * inv_t;
        const int after = s < prev_s || (s == prev_s && j > prev);
        if (!after) continue;
        if (best < 0 || s > bs) {
          best = j;
          bs = s;
        }
      }
      if (best < 0) {
        top_ids[b * top_n + i] = -1;
        top_lp[b * top_n + i] = -INFINITY;
        continue;
      }
      top_ids[b * top_n + i] = (int32_t)best;
      top_lp[b * top_n + i] = (float)((double)(bs - m) - L);
      prev = best;
      prev_s = bs;
    }
  }
}

/* ------------------------------------------------------------------------ */
/* Mixture of experts                                                        */
/* ------------------------------------------------------------------------ */

/*
 * Qwen3MoeMlpBlock::forward_moe router (qwen3_moe.rs:303-316):
 * gates = softmax(logits) in f32 (orc_exp, the deterministic exp), the k
 * experts with the largest logits -- softmax is monotonic, so these are the
 * top-k gates of MLX's argpartition(-k) -- with ties to the lower expert index
 * and NaN never preferred, listed in descending order; scores = their gates,
 * renormalised to sum 1 (summed in selection order) when norm_topk_prob.
 * logits [T, E] f32.
 */
static int moe_better(float a, int64_t ia, float b, int64_t ib) {
  /* a strictly preferred over b: larger, NaN lowest, -0 == +0, ties -> lower index */
  if (a != a) return (b != b) && ia < ib;
  if (b != b) return 1;
  if (a != b) return a > b;
  return ia < ib;
}

void orc_moe_route_topk(const float* logits, int64_t T, int64_t E, int64_t k, int norm,
                        int32_t* idx, float* scores) {
  char* taken = (char*)malloc((size_t)E);
  for (int64_t t = 0; t < T; ++t) {
    const float* l = logits + t * E;
    float mx = -INFINITY;
    for (int64_t e = 0; e < E; ++e)
      if (l[e] > mx) mx = l[e];
    float den = 0.0f;
    for (int64_t e = 0; e < E; ++e) den += orc_exp(l[e] - mx);
    memset(taken, 0, (size_t)E);
    float ssum = 0.0f;
    for (int64_t i = 0; i < k; ++i) {
      int64_t best = -1;
      for (int64_t e = 0; e < E; ++e)
        if (!taken[e] && (best < 0 || moe_better(l[e], e, l[best], best))) best = e;
      taken[best] = 1;
      const float g = orc_exp(l[best] - mx) / den;
      idx[t * k + i] = (int32_t)best;
      scores[t * k + i] = g;
      ssum += g;
    }
    if (norm)
      for (int64_t i = 0; i < k; ++i) scores[t * k + i] /= ssum;
  }
  free(taken);
}

/*
 * The weighted sum over the k expert outputs and the residual add
 * (qwen3_moe.rs:319-320, 384-385) with MLX's bf16 rounding points:
 * h[t] = bf16(h[t] + bf16(sum_j bf16(s_j) * y[t*k+j])), f32 in j order.
 * y bf16 [T*k, H], scores f32 [T, k], h bf16 [T, H] in place.
 */
void orc_moe_combine(const uint16_t* y, const float* scores, int64_t T, int64_t k, int64_t H,
                     uint16_t* h) {
  for (int64_t t = 0; t < T; ++t)
    for (int64_t c = 0; c < H; ++c) {
      float acc = 0.0f;
      for (int64_t j = 0; j < k; ++j) {
        const float sc = bf2f(f2bf(scores[t * k + j]));
        acc = acc + sc * bf2f(y[(t * k + j) * H + c]);
      }
      h[t * H + c] = f2bf(bf2f(h[t * H + c]) + bf2f(f2bf(acc)));
    }
}
