/*
 * higgs_cuda.h -- C ABI of libhiggs_cuda.so, the B200 (sm_100a) decode hot
 * path for higgs.
 *
 * Each entry point replaces one mlx-rs / mlx-sys op that higgs-models calls
 * today; the citation above each declaration is the reference call site it
 * replaces (paths relative to the higgs repository).
 *
 * Conventions
 *   - Every function returns 0 on success or a negative HIGGS_ERR_* code and
 *     never aborts; higgs_last_error() returns the calling thread's message
 *     for the most recent failure.
 *   - All tensor arguments are caller-owned DEVICE pointers on the context's
 *     device, row-major and densely packed unless a stride says otherwise.
 *     "bf16" / "fp16" buffers are passed as void*.  Every call that takes a
 *     context (or a model / communicator / graph built on one) runs on that
 *     context's device whatever device is current, and restores the caller's
 *     current device before it returns; one process may hold contexts on
 *     several GPUs (device ordinals 0..63).
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Calls only
 *     enqueue work; they do not synchronise.  Device memory is allocated only
 *     by higgs_init() (one int per device, the first time a device is
 *     initialised), higgs_model_finalize() (a RoPE table) and
 *     higgs_comm_create() (the peer-exchange buffers); every other call takes
 *     its scratch from caller-provided workspace whose size a
 *     *_workspace_size() query returns.
 *   - Per-device state lives until the process exits and does not survive a
 *     device reset (cudaDeviceReset, or the primary context being destroyed):
 *     after one, the library must not be used again in that process.
 *   - A context may be used by one host thread at a time; distinct contexts
 *     are independent.
 *   - Kernels start early behind the previous kernel on the stream
 *     (programmatic dependent launch) and fetch what cannot depend on it
 *     first: weights, and for the attention calls the block table, the
 *     sequence lengths and the KV pages of earlier steps.  Those inputs must
 *     therefore not be written by the kernel enqueued immediately before the
 *     call (host copies, or any earlier kernel, are fine).
 *   - Quantized weights use the MLX affine layout: weight u32 [N, K/8] with
 *     element k of a row in word k/8 at bits 4*(k%8); scales and biases bf16
 *     [N, K/64]; w = scale * q + bias (group size 64, 4 bits).
 */
#ifndef HIGGS_CUDA_H
#define HIGGS_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HIGGS_OK 0
#define HIGGS_ERR_INVALID_ARG -1
#define HIGGS_ERR_CUDA -2
#define HIGGS_ERR_UNSUPPORTED -3
#define HIGGS_ERR_WORKSPACE -4
#define HIGGS_ERR_TIMEOUT -5
#define HIGGS_ERR_STATE -6
#define HIGGS_ERR_OUT_OF_PAGES -7

#define HIGGS_PAGE_SIZE 16 /* tokens per KV page */

#define HIGGS_DTYPE_U32 0
#define HIGGS_DTYPE_BF16 1
#define HIGGS_DTYPE_F32 2
#define HIGGS_DTYPE_F16 3

#define HIGGS_KV_BF16 0 /* bf16 pages [pages, Hkv, 16, D] */
#define HIGGS_KV_TQ4 1  /* TurboQuant pages: codes [pages, Hkv, 16, 64] + fp16 scales */

typedef struct higgs_ctx higgs_ctx;
typedef struct higgs_model higgs_model;
typedef struct higgs_graph higgs_graph;
typedef struct higgs_block_pool higgs_block_pool;
typedef struct higgs_prefix_cache higgs_prefix_cache;
typedef struct higgs_comm higgs_comm;
typedef struct higgs_safetensors higgs_safetensors;

/* ---- context and errors ------------------------------------------------ */

/* Replaces the process-global MLX error handler registration
 * (crates/higgs-models/src/qwen3_next.rs:29-51) and default-stream setup
 * (crates/higgs-engine/src/simple.rs:450-452). */
int higgs_init(int device, higgs_ctx** out);
int higgs_destroy(higgs_ctx* ctx);
/* Message of the calling thread's last failure ("" if none).  Replaces the
 * error text captured at crates/higgs-models/src/qwen3_next.rs:337-360. */
const char* higgs_last_error(void);
int higgs_version(void);

/* Process-wide tuning switches (no reference counterpart).  "gemv_f16" (0/1,
 * default 0): decode GEMVs with x staged in shared memory feed the tensor cores
 * fp16 operands (x scaled per token by a power of two, exact for bf16 inputs)
 * instead of bf16 ones.  "attn_min_pages" (4..4096, default 8): KV pages per split
 * of higgs_fused_attention; change it only between captures, since workspace
 * sizes depend on it.  "l2_prefetch" (bit mask, default 0): bit 0 makes the
 * decode step ask the TMA unit to pull later GEMVs' weights into L2 ahead of them
 * (the fused attention kernel requests o_proj's and the MLP's, o_proj down_proj's,
 * gate/up the next layer's q|k|v), bit 1 makes each multi-token GEMV CTA pull its
 * own weight tiles (hints; results are unchanged; measured on B200, both lengthen
 * the Qwen3-8B decode step at B=1 and B=8).  "gemm_tc" (0/1, default 1): quantized linears over 17 or more
 * rows use the tcgen05 tensor-core kernel (weights dequantized to bf16 first,
 * MLX's qmm form) instead of the decode GEMV; "gemm_tc_waves" (1..8, default 2) and "gemm_tc_wave_cost"
 * (default 8): the tensor-core kernel picks the K-split count that minimises
 * waves x (k groups per split + wave cost) within that many waves of one CTA
 * per SM (change them only between captures: workspace sizes depend on them).  "gemm_tc_rows" (default 17) moves
 * that threshold (fused-RMSNorm decode launches always stay on the GEMV).  "gemv_wk" (0, 1, 2, 4, 8; default
 * 0 = heuristic): ways each 16-row tile of the decode GEMV splits K over warps.
 * One-token linears (M == 1, every entry above including the fused-RMSNorm ones)
 * run the register-fed single-token GEMV: "gemv_m1" (0/1, default 1) switches it
 * off (back to the multi-token GEMV); "gemv_m1_wk" (0, 1, 2, 4, 8; default 0 =
 * heuristic) forces its K split; "gemv_m1_depth" (2 or 4, default 2) sets the
 * weight units each warp keeps in flight; "gemv_m1_l2" (0/1, default 1) makes each
 * of its CTAs ask L2 for its whole weight slice before waiting on the previous
 * kernel (a hint); "gemv_m1_persist" (0, 1, 2; default 0) caps its grid at the
 * resident CTA slots with CTAs looping over row-tile groups (1: every launch, 2:
 * gate/up launches only); "gemv_m1_l1" (0..16, default 0) prefetches that many
 * weight units into L1 ahead of each warp's register ring.  "decode_chain" (0/1,
 * default 0): a one-token decode step on one GPU runs the GEMVs between two
 * attention launches (o_proj, norm + gate/up, down, norm + the next q|k|v or the
 * final norm + LM head) as one persistent launch with grid barriers, each phase
 * the register-fed single-token GEMV with its K split and summation order (the
 * same bits as that GEMV); "decode_chain_l2_ahead" (0/1, default 1): its CTAs ask
 * L2 for the next phase's weights while the current phase runs.  "gemv_tma" (0/1,
 * default 0): one-token linears (K a multiple of 512, up to 12288) stream their
 * weights by TMA into a shared-memory ring instead of loading them into
 * registers.  "attn_cluster" (0, 2..16, default 16): the largest thread-block
 * cluster the splits of one (sequence, kv head) of the fused decode attention
 * form to merge through distributed shared memory (0: workspace merge by the
 * last CTA).  "tq4_p_lo" (0/1, default 0): TurboQuant attention multiplies V by
 * P's hi + lo bf16 halves (1) instead of its bf16 rounding (0).  "tq4_swap" (0, 4
 * or 6, default 4): TurboQuant launches of at most 4 query rows run the kernel
 * with the keys on the MMA's 16 rows and that many page-ring stages per warp
 * (0: the kernel with the query rows there).  "tp_fuse" (0/1,
 * default 0): one-token tensor-parallel decode sums the row-parallel partials
 * inside the GEMVs (pushed by the producing GEMV, pulled by the next fused-norm
 * GEMV) instead of all-reduce launches.  "attn_prefill_tc" (0/1, default 1):
 * higgs_paged_attention launches of more than 64 query rows (Hq / Hkv x Lq; G =
 * Hq / Hkv dividing 128, 16-byte aligned buffers and strides) run the tcgen05
 * prefill kernel (128-row tiles of tokens x GQA heads, S and O in tensor memory)
 * instead of the decode kernel's 32-row query chunks.
 * Unknown names return HIGGS_ERR_INVALID_ARG. */
int higgs_set_option(const char* name, int value);

/* Nonzero when a bounded wait of the tensor-core quantized matmul or of the
 * decode-chain kernel's barriers gave up on the context's device since the
 * last call (the device's flag is then cleared; the results of that call are
 * undefined).  Synchronising. */
int higgs_tc_error(higgs_ctx* ctx, int* out);

/* Diagnostic (not a reference op): the tensor-core issue rate that bounds the
 * matrix-form quantized matmul at decode sizes.  One CTA on each of `ctas` SMs;
 * lane 0 of each of `warps` (1..4) warps issues `iters` stages of 4 tcgen05.mma
 * (M = m (64 or 128), N = n, K = 16, bf16 operands from shared memory, f32
 * accumulators in TMEM), the stage's MMAs (spread 0) or each MMA (spread 1)
 * dealt round-robin to that warp's `nacc` accumulators, with a tcgen05.commit
 * every `commit_every` stages (0: only at the end).
 * cycles: device int64 [ctas], SM clocks from the first issue until every MMA
 * completed (-1 if a bounded wait gave up; higgs_tc_error then reports it).
 * n 16..256 (multiple of 16), warps * nacc * n <= 512.  Asynchronous on `stream`. */
int higgs_diag_tc_mma_rate(higgs_ctx* ctx, int m, int n, int nacc, int spread, int iters,
                           int commit_every, int warps, int ctas, long long* cycles, void* stream);

/* ---- a1/a2: W4 g64 quantized linear and embedding ----------------------- */

/* ops::dequantize (crates/higgs-models/src/qwen3_next.rs:249-256):
 * out bf16 [N, K] = bf16(scale * q + bias). */
int higgs_w4_dequantize(higgs_ctx* ctx, const uint32_t* w, const void* scales, const void* biases,
                        int N, int K, void* out, void* stream);

/* ops::quantize(w, 64, 4) as used to build weights in the reference's tests
 * (crates/higgs-models/src/qwen3_next.rs:2113-2116), with this library's
 * documented rounding (MLX's own is not pinned by any reference test):
 * per 64-group scale = bf16((max - min) / 15) (1 if that rounds to 0),
 * bias = bf16(min), q = clamp(rint((w - bias) / scale), 0, 15).
 * w f32 [N, K] -> q u32 [N, K/8], scales / biases bf16 [N, K/64]. */
int higgs_w4_quantize(higgs_ctx* ctx, const float* w, int64_t N, int K, uint32_t* q, void* scales,
                      void* biases, void* stream);

/* QEmbedding::forward (crates/higgs-models/src/qwen3_next.rs:248-257):
 * out bf16 [n_ids, H] = dequantized rows ids[i] of the [V, H] table.  Ids
 * outside [0, V) produce zero rows. */
int higgs_embed_gather_w4(higgs_ctx* ctx, const int32_t* ids, int n_ids, const uint32_t* w,
                          const void* scales, const void* biases, int V, int H, void* out,
                          void* stream);

/* ops::quantized_matmul(x, w, scales, biases, transpose=true, 64, 4)
 * (crates/higgs-models/src/qwen3_next.rs:174-183, QLinear::forward 211-220;
 * MaybeQuantized<nn::Linear> crates/higgs-models/src/transformer.rs:943-951;
 * tied head QEmbedding::as_linear qwen3_next.rs:259-268).
 *   x bf16 [M, K]; y = x . W^T with W [N, K].
 *   y       bf16 [M, N] (may be NULL when y_f32 is given)
 *   y_f32   f32  [M, N] (optional, unrounded accumulator)
 *   residual bf16 [M, N] (optional): y = bf16(bf16(x W^T) + residual), the
 *            residual add of TransformerBlock::forward transformer.rs:410,417.
 * K must be a multiple of 256; any M >= 1. */
int higgs_qlinear_w4g64(higgs_ctx* ctx, const void* x, int M, int K, const uint32_t* w,
                        const void* scales, const void* biases, int N, void* y, float* y_f32,
                        const void* residual, void* stream);

/* Workspace variants of the two linear ops above.  For M <= 8 the preceding
 * nn::RmsNorm can be fused in (transformer.rs:407-416: input_layernorm before
 * q/k/v, post_attention_layernorm before the MLP): when norm_w != NULL, x is
 * the residual stream h and the op consumes bf16(h * rsqrt(mean(h^2) + eps) *
 * norm_w) (K <= 8192); with norm_w == NULL they equal higgs_qlinear_w4g64 /
 * higgs_qlinear_gate_up_swiglu, for any M >= 1.  M <= 8 balances the weight
 * stream over every SM (stream-K GEMV); from 17 rows the tensor-core matmul
 * splits K over the workspace when its tiles alone cannot fill the GPU.  They
 * need higgs_qlinear_sk_workspace_size(M, K, rows) bytes (rows = N, or 2N for
 * the SwiGLU pair, at most 262144) whose first 65536 bytes (tile counters) must
 * be zero before the first call; each call leaves them zero, so one workspace
 * of the largest size serves every shape back to back on a stream.  Results
 * are deterministic (partial sums are combined in a fixed order). */
size_t higgs_qlinear_sk_workspace_size(int M, int K, int N_rows);
int higgs_rmsnorm_qlinear_w4g64(higgs_ctx* ctx, const void* x, int M, int K, const void* norm_w,
                                float eps, const uint32_t* w, const void* scales,
                                const void* biases, int N, void* y, float* y_f32,
                                const void* residual, void* workspace, size_t workspace_bytes,
                                void* stream);
int higgs_rmsnorm_gate_up_swiglu(higgs_ctx* ctx, const void* x, int M, int K, const void* norm_w,
                                 float eps, const uint32_t* w_gate, const void* s_gate,
                                 const void* b_gate, const uint32_t* w_up, const void* s_up,
                                 const void* b_up, int N, void* y, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* Mlp::forward gate/up half (crates/higgs-models/src/transformer.rs:349-353,
 * swiglu qwen3_next.rs:275-277): y bf16 [M, N] = silu(x Wg^T) * (x Wu^T),
 * both projections rounded to bf16 first, one bf16 rounding of the product. */
int higgs_qlinear_gate_up_swiglu(higgs_ctx* ctx, const void* x, int M, int K,
                                 const uint32_t* w_gate, const void* s_gate, const void* b_gate,
                                 const uint32_t* w_up, const void* s_up, const void* b_up, int N,
                                 void* y, void* stream);

/* One GEMV of a one-token decode chain: y = W x (bf16 x [K]) with optional
 * fused RMSNorm of x (norm_w), SwiGLU over gate w / up w2 (y = silu(g) * u),
 * q|k|v-style row segments (nseg <= 3: rows [seg_end[i-1], seg_end[i]) from
 * w[i]), and outputs bf16 y (optionally + residual) and / or f32 y_f32. */
typedef struct higgs_chain_gemv {
  const void* x;
  const void* norm_w;
  int K, N, swiglu, nseg;
  int seg_end[3];
  const uint32_t* w[3];
  const void* s[3];
  const void* b[3];
  const uint32_t* w2;
  const void* s2;
  const void* b2;
  void* y;
  float* y_f32;
  const void* residual;
} higgs_chain_gemv;

/* The GEMVs of a transformer block after its attention at one token, as one
 * persistent launch: TransformerBlock::forward's residual adds and post-attention
 * RMSNorm with Mlp::forward (crates/higgs-models/src/transformer.rs:404-418,
 * 345-353) -- h += o_proj(attn); act = swiglu(gate(norm(h)), up(norm(h)));
 * h += down(act); then the next block's norm + q|k|v (or the final norm + LM
 * head) -- each phase an ops::quantized_matmul (qwen3_next.rs:174-183) with
 * the register-fed single-token GEMV's K split and summation order (the same
 * bits as separate higgs_qlinear_w4g64 / higgs_rmsnorm_* calls at M = 1 with
 * the "gemv_tma" option off), phases
 * separated by grid barriers.  n_phases <= 4; K <= 32768 (8192 with a fused
 * norm), multiples of 256; N multiple of 16 (32 with SwiGLU).  barriers:
 * 64 * n_phases u32 words, zero on entry and left zero.  A phase's input may be
 * an earlier phase's output.  The launch's CTAs (two per SM) must all be
 * resident at once, so the GPU must not be running a concurrent kernel that
 * never finishes; a barrier wait that gives up sets the flag higgs_tc_error
 * reports. */
int higgs_decode_chain(higgs_ctx* ctx, const higgs_chain_gemv* phases, int n_phases, float eps,
                       uint32_t* barriers, void* stream);

/* ---- a3/a4: norms and RoPE ---------------------------------------------- */

/* nn::RmsNorm / fast::rms_norm (crates/higgs-models/src/transformer.rs:375-377,
 * 407, 415, 525): y = bf16(h * rsqrt(mean(h^2) + eps) * weight), rows x H,
 * with h = bf16(x + residual) when residual != NULL (written to h_out when
 * h_out != NULL), else h = x. */
int higgs_rmsnorm(higgs_ctx* ctx, const void* x, const void* residual, int rows, int H,
                  const void* weight, float eps, void* y, void* h_out, void* stream);

/* higgs_rmsnorm over rows that are in_stride elements apart (e.g. the last
 * token of each sequence before the LM head, transformer.rs:525); y dense
 * [rows, H]. */
int higgs_rmsnorm_strided(higgs_ctx* ctx, const void* x, int64_t in_stride, int rows, int H,
                          const void* weight, float eps, void* y, void* stream);

/* fast::rope, traditional=false, scale=1 (crates/higgs-models/src/utils.rs:16-26):
 * x, y bf16 [rows, heads, D]; row r rotated at absolute position positions[r];
 * inv_freq f32 [D/2] = base^(-2i/D). */
int higgs_rope(higgs_ctx* ctx, const void* x, int rows, int heads, int D,
               const int32_t* positions, const float* inv_freq, void* y, void* stream);

/* Attention::forward front half (crates/higgs-models/src/transformer.rs:246-289)
 * fused with the cache append of SteppingKeyValueCache::update_and_fetch
 * (crates/higgs-models/src/cache.rs:236-311), on a paged cache:
 *   qkv bf16 [T, (Hq + 2 Hkv) * D]  (the fused q|k|v projection output)
 *   q/k head RMSNorm with q_norm_w / k_norm_w bf16 [D] when non-NULL (Qwen3,
 *   transformer.rs:193-207), then RoPE at positions[t], then
 *   q_out bf16 [T, Hq, D]; K and V of token t stored at page
 *   slot_mapping[t] / 16, slot slot_mapping[t] % 16: element
 *   page * page_stride + h * head_stride + slot * D of k_cache / v_cache.
 *   slot_mapping[t] < 0 skips the store. */
int higgs_qknorm_rope_kv_write(higgs_ctx* ctx, const void* qkv, int T, int Hq, int Hkv, int D,
                               const void* q_norm_w, const void* k_norm_w, float eps,
                               const int32_t* positions, const float* inv_freq,
                               const int64_t* slot_mapping, void* k_cache, void* v_cache,
                               int64_t page_stride, int64_t head_stride, void* q_out,
                               void* stream);

/* ---- a5/a6/a13: paged decode attention ----------------------------------- */

/* fast::scaled_dot_product_attention with GQA (crates/higgs-models/src/utils.rs:45-60)
 * and the masks of utils.rs:64-125, over a paged KV cache.
 *   q   bf16 [B, Lq, Hq, D] (D = 64 or 128; launches of more than 64 query rows,
 *       Hq / Hkv * Lq, run the tensor-core prefill kernel: option "attn_prefill_tc")
 *   query t of sequence b sits at position seq_lens[b] - Lq + t and attends
 *   to keys 0..that position (causal, includes itself).
 *   block_table int32 [B, max_blocks]; page p of the cache holds key/value
 *   slot s of kv head h at element p * page_stride + h * head_stride + s * D.
 *   out bf16 [B, Lq, Hq, D].
 * max_seq_len bounds every seq_lens[b] (it sizes the split-K grid; the
 * kernel reads the real lengths on the device, so a captured graph stays valid
 * while lengths grow up to that bound).  workspace: at least
 * higgs_paged_attention_workspace_size() bytes; its first 4096 bytes hold
 * split counters that must be zero before the first call (each call leaves
 * them zero). */
size_t higgs_paged_attention_workspace_size(int B, int Lq, int Hq, int Hkv, int D,
                                            int max_seq_len);
int higgs_paged_attention(higgs_ctx* ctx, const void* q, int B, int Lq, int Hq, int Hkv, int D,
                          const void* k_cache, const void* v_cache, int64_t page_stride,
                          int64_t head_stride, const int32_t* block_table, int max_blocks,
                          const int32_t* seq_lens, int max_seq_len, float scale, void* out,
                          void* workspace, size_t workspace_bytes, void* stream);

/* Attention::forward from the q|k|v projection to the attention output
 * (crates/higgs-models/src/transformer.rs:246-294) in one kernel: q/k head
 * RMSNorm (when the weights are given), RoPE at positions[t], the cache append
 * of the new tokens at slot_mapping[t] (cache.rs:236-311), and the paged SDPA
 * of higgs_paged_attention over the updated cache.  qkv bf16
 * [B * Lq, (Hq + 2 Hkv) * D]; out bf16 [B, Lq, Hq, D]; needs (Hq / Hkv) * Lq <= 32
 * (decode and speculative verify).  Workspace rules as higgs_paged_attention,
 * sized by higgs_fused_attention_workspace_size. */
size_t higgs_fused_attention_workspace_size(int B, int Lq, int Hq, int Hkv, int D,
                                            int max_seq_len);
int higgs_fused_attention(higgs_ctx* ctx, const void* qkv, int B, int Lq, int Hq, int Hkv, int D,
                          const void* q_norm_w, const void* k_norm_w, float eps,
                          const int32_t* positions, const float* inv_freq,
                          const int64_t* slot_mapping, void* k_cache, void* v_cache,
                          int64_t page_stride, int64_t head_stride, const int32_t* block_table,
                          int max_blocks, const int32_t* seq_lens, int max_seq_len, float scale,
                          void* out, void* workspace, size_t workspace_bytes, void* stream);

/* higgs_paged_attention without a workspace argument, for callers that cannot
 * allocate device memory on their serving path (a host that owns a fixed
 * device arena and budgets every byte itself, or a real-time decode loop that
 * must never block in the driver's allocator).  No counterpart in the
 * reference.  The split-K scratch is an 8 MiB array built into the library
 * (held on every GPU that loads it until the process exits).  The split plan
 * keeps a launch within one resident wave of CTAs, so every shape the call
 * accepts (B * Hkv <= 1024, D 64 or 128) fits; a shape needing more would be
 * rejected with HIGGS_ERR_WORKSPACE before any launch.  The first call on a device looks
 * up that array's device address, so make that first call before any stream
 * capture.  Every call shares the one array: calls that overlap on the GPU
 * (concurrent streams, several host threads) race and must be serialised by
 * the caller.  Each call clears the split counters itself before launching. */
int higgs_paged_attention_noalloc(higgs_ctx* ctx, const void* q, int B, int Lq, int Hq, int Hkv,
                                  int D, const void* k_cache, const void* v_cache,
                                  int64_t page_stride, int64_t head_stride,
                                  const int32_t* block_table, int max_blocks,
                                  const int32_t* seq_lens, int max_seq_len, float scale, void* out,
                                  void* stream);

/* ---- a14: TurboQuant-style 4-bit KV (no reference counterpart; the
 * KeyValueCache trait only reserves is_quantized/group_size/bits hooks,
 * crates/higgs-models/src/cache.rs:4-18) ------------------------------------ */

/* Encode n head vectors x bf16 [n, 128]: v' = H diag(signs) x / sqrt(128)
 * (signs int8 [128] of +-1), fp16 scale s = max|v'| / 7,
 * code = clamp(rint(v'/s), -8, 7) + 8, byte j = c[2j] | c[2j+1] << 4.
 * codes u8 [n, 64], scales fp16 [n]. */
int higgs_tq4_encode(higgs_ctx* ctx, const void* x, int64_t n, const int8_t* signs,
                     uint8_t* codes, void* scales, void* stream);

/* higgs_qknorm_rope_kv_write with a TurboQuant cache (D = 128): codes of token
 * t, kv head h go to byte page * page_stride + h * head_stride + slot * 64 of
 * k_codes / v_codes, scales (fp16) to element
 * page * (page_stride / 64) + h * (head_stride / 64) + slot. */
int higgs_qknorm_rope_kv_write_tq4(higgs_ctx* ctx, const void* qkv, int T, int Hq, int Hkv,
                                   const void* q_norm_w, const void* k_norm_w, float eps,
                                   const int32_t* positions, const float* inv_freq,
                                   const int64_t* slot_mapping, const int8_t* signs,
                                   uint8_t* k_codes, void* k_scales, uint8_t* v_codes,
                                   void* v_scales, int64_t page_stride, int64_t head_stride,
                                   void* q_out, void* stream);

/* Decode attention over TurboQuant pages (D = 128), same semantics and
 * workspace rules as higgs_paged_attention; the query is rotated into the
 * code basis in-kernel and the output rotated back. */
size_t higgs_paged_attention_tq4_workspace_size(int B, int Lq, int Hq, int Hkv, int max_seq_len);
int higgs_paged_attention_tq4(higgs_ctx* ctx, const void* q, int B, int Lq, int Hq, int Hkv,
                              const uint8_t* k_codes, const void* k_scales,
                              const uint8_t* v_codes, const void* v_scales, int64_t page_stride,
                              int64_t head_stride, const int32_t* block_table, int max_blocks,
                              const int32_t* seq_lens, int max_seq_len, const int8_t* signs,
                              float scale, void* out, void* workspace, size_t workspace_bytes,
                              void* stream);

/* ---- a10/a15: token selection -------------------------------------------- */

/* sample() at temperature 0 (crates/higgs-models/src/lib.rs:373-377):
 * out[b] = argmax_j logits[b, j], ties -> lowest index (lib.rs:838-843). */
int higgs_argmax(higgs_ctx* ctx, const float* logits, int B, int V, int32_t* out, void* stream);

/* sample() at temperature > 0 (crates/higgs-models/src/lib.rs:379-384,
 * categorical(logits / T)): inverse-CDF draw with the caller's uniforms[b]
 * in [0, 1) over a fixed-point softmax (exact integer prefix sums), so the
 * token is a deterministic function of (logits, T, u).  T == 0 -> argmax. */
int higgs_sample(higgs_ctx* ctx, const float* logits, int B, int V, float temperature,
                 const float* uniforms, int32_t* out, void* stream);

/* Speculative acceptance (no reference counterpart).  target_logits f32
 * [B, k+1, V], draft_logits f32 [B, k, V], draft_tokens int32 [B, k]:
 * accept draft i while u_i * q_i(x_i) < p_i(x_i) (p, q the temperature
 * softmaxes), resample the first rejected position from norm(max(p - q, 0)),
 * or draw a bonus token from p_k when all k are accepted.  accepted int32 [B];
 * out_tokens int32 [B, k+1] (accepted drafts, then the corrected / bonus
 * token, then -1).  temperature 0 = greedy verification. */
int higgs_spec_accept(higgs_ctx* ctx, const float* target_logits, const float* draft_logits,
                      const int32_t* draft_tokens, int B, int k, int V, float temperature,
                      const float* accept_uniforms, const float* sample_uniforms,
                      int32_t* accepted, int32_t* out_tokens, void* stream);

/* apply_penalties (crates/higgs-models/src/lib.rs:278-363), in place on
 * logits f32 [B, V]; history int32 [B, max_hist] with hist_lens[b] valid
 * entries.  rep = 1, freq = 0, pres = 0 disable the respective penalty. */
int higgs_apply_penalties(higgs_ctx* ctx, float* logits, int B, int V, const int32_t* history,
                          const int32_t* hist_lens, int max_hist, float rep, float freq,
                          float pres, void* stream);

/* sample() with filtering (crates/higgs-models/src/lib.rs:373-385 calling
 * sample_filtered lib.rs:392-460): out int32 [B] from logits f32 [B, V] at
 * `temperature`, keeping the tokens that pass top_k (0 = off), top_p (>= 1 =
 * off) and min_p (<= 0 = off, clamped to 1) before an inverse-CDF draw with
 * uniforms[b].  Masses are the fixed-point E_j of higgs_sample; ranks order
 * them by mass, ties to the lower index; rank r is kept iff r < top_k, and
 * (r == 0 or its inclusive mass prefix <= top_p * sum E), and E_r >= min_p *
 * max E (the products in IEEE double), so a draw is exact given the uniform.
 * temperature 0 is the argmax; no active filter is higgs_sample.  V <= 163840.
 * One cluster of 8 CTAs per row. */
int higgs_sample_filtered(higgs_ctx* ctx, const float* logits, int B, int V, float temperature,
                          int top_k, float top_p, float min_p, const float* uniforms,
                          int32_t* out, void* stream);

/* LogprobArrays::compute (crates/higgs-models/src/lib.rs:495-533) on the
 * logits scaled as its callers do (crates/higgs-engine/src/simple.rs:269-277:
 * unscaled when temperature <= FLT_EPSILON, else times 1/T): token_logprob f32
 * [B] of tokens[b], and the top_n (ties to the lower index) as top_ids int32
 * [B, top_n] and top_logprobs f32 [B, top_n] (-1 / -inf past the vocabulary).
 * log Z is the log of an exact fixed-point sum (2^-44 units) in double. */
int higgs_logprobs(higgs_ctx* ctx, const float* logits, int B, int V, float temperature,
                   const int32_t* tokens, int top_n, float* token_logprob, int32_t* top_ids,
                   float* top_logprobs, void* stream);

/* Constraint::apply_mask (crates/higgs-engine/src/constrained.rs:79-110), in
 * place: logits f32 [B, V] += 0 where the token is allowed, -inf elsewhere.
 * allowed u32 [B, words_per_row]: bit (j % 32) of word j / 32 = token j
 * allowed (words_per_row * 32 >= V).  The set itself comes from the host's
 * FSM each step, as in the reference. */
int higgs_apply_token_mask(higgs_ctx* ctx, float* logits, int B, int V, const uint32_t* allowed,
                           int words_per_row, void* stream);

/* ---- a9: mixture of experts (qwen3_moe.rs Qwen3MoeMlpBlock) ------------- */

/* Bytes of the routing plan higgs_moe_route_topk writes for T tokens, E
 * experts and top-k: the (token, slot) pairs p = t*k + j grouped by expert
 * and cut into work items of at most 8 pairs of one expert, which
 * higgs_moe_grouped_w4 consumes. */
size_t higgs_moe_plan_size(int T, int E, int k);

/* Router of Qwen3MoeMlpBlock::forward_moe (crates/higgs-models/src/
 * qwen3_moe.rs:303-316): gates = softmax(logits) in f32, the k experts with
 * the largest logits (ties -> lower expert index; softmax is monotonic, so
 * this is MLX's argpartition(-k) over the gates with the tie order fixed),
 * scores = their gates, renormalised to sum 1 when norm_topk_prob.
 * logits [T, E] (dtype HIGGS_DTYPE_BF16 -- the router QLinear's output -- or
 * HIGGS_DTYPE_F32); idx int32 [T, k] and scores f32 [T, k] in descending
 * order.  plan (nullable) receives the routing plan.  E <= 1024, k <= 32,
 * T*k <= 65536. */
int higgs_moe_route_topk(higgs_ctx* ctx, const void* logits, int dtype, int T, int E, int k,
                         int norm_topk_prob, int32_t* idx, float* scores, void* plan,
                         size_t plan_bytes, void* stream);

/* The router QLinear of Qwen3MoeMlpBlock (qwen3_moe.rs:301-303, `gate`):
 * logits bf16 [T, E] = x bf16 [T, K] . dequant(w [E, K/8])^T, summed in a
 * fixed order -- per (row, group of 64) the products x*q and the x values in
 * k order, then s*sum(xq) + b*sum(x) added in group order -- so the expert
 * choice downstream (a discontinuous function of these logits) is
 * reproducible bit for bit.  K % 64 == 0, K <= 16384. */
int higgs_moe_router(higgs_ctx* ctx, const void* x, int T, int K, const uint32_t* w,
                     const void* scales, const void* biases, int E, void* logits, void* stream);

/* gather_qmm (crates/higgs-models/src/qwen3_next.rs:294-363) as used by
 * SwitchMlpWeights::forward_gather (qwen3_next.rs:844-904): for every pair p
 * of the plan, y[p] = x[row(p)] . dequant(w[expert(p)])^T, row(p) = p / k when
 * x_per_pair = 0 (x has T rows: the gate / up projections) or p when 1 (x has
 * T*k rows: the down projection).  w u32 [E, N, K/8], scales / biases bf16
 * [E, N, K/64] (MLX SwitchLinear layout).  With w_up set the call is the fused
 * gate / up pair and y[p] = silu(gate) * up (swiglu, qwen3_next.rs:275-277).
 * y bf16 [T*k, N]. */
int higgs_moe_grouped_w4(higgs_ctx* ctx, const void* x, int T, int K, int k, int x_per_pair,
                         const void* plan, const uint32_t* w, const void* scales,
                         const void* biases, const uint32_t* w_up, const void* scales_up,
                         const void* biases_up, int E, int N, void* y, void* stream);

/* The weighted sum over the k expert outputs and the residual add of the
 * decoder layer (qwen3_moe.rs:319-320, 384-385): h[t] = bf16(h[t] +
 * bf16(sum_j bf16(scores[t,j]) * y[t*k+j])), f32 accumulation in j order.
 * y bf16 [T*k, H]; h bf16 [T, H] in place. */
int higgs_moe_combine(higgs_ctx* ctx, const void* y, const float* scores, int T, int k, int H,
                      void* h, void* stream);

/* ---- (e): tensor-parallel collectives over NVLink peer memory ------------ */

/* A communicator of `world` ranks (one process per GPU).  Each rank allocates
 * a buffer of n_calls call regions (one per collective call site of a decode
 * step, 2 x layers + 1 for the decode runner) of words_per_call u32 words per
 * rank, and gets its CUDA IPC handle (higgs_comm_handle_size() bytes) in
 * ipc_handle_out; the host exchanges the handles (any side channel) and passes
 * all `world` of them, in rank order, to higgs_comm_connect.  Collectives are
 * one-shot pushes into every rank's buffer with per-CTA flags; every rank must
 * issue the same calls in the same order, and higgs_comm_step once per step
 * before them.  A wait that sees no progress for about a second gives up and
 * sets the flag that higgs_comm_error returns (and clears); the results of that
 * step are then undefined.  After a nonzero higgs_comm_error the ranks may no
 * longer agree on the step number, so every rank must destroy its communicator
 * and create and connect a new one before the next collective. */
size_t higgs_comm_handle_size(void);
int higgs_comm_create(higgs_ctx* ctx, int rank, int world, size_t words_per_call, int n_calls,
                      higgs_comm** out, void* ipc_handle_out);
int higgs_comm_connect(higgs_comm* comm, const void* handles);
int higgs_comm_destroy(higgs_comm* comm);
int higgs_comm_error(higgs_comm* comm, int* out);
int higgs_comm_step(higgs_comm* comm, void* stream);
/* h bf16 [n] += bf16(sum over ranks of partial f32 [n]), summed in rank order. */
int higgs_allreduce_residual(higgs_comm* comm, int call, const float* partial, int n, void* h,
                             void* stream);
/* out int32 [n] = index of the max over ranks of keys u64 [n] (argmax keys). */
int higgs_allreduce_argmax(higgs_comm* comm, int call, const uint64_t* keys, int n, int32_t* out,
                           void* stream);

/* ---- a7/a11: native decode step (transformer.rs Model) ------------------ */

/* ModelArgs (crates/higgs-models/src/transformer.rs:69-97) reduced to what the
 * step needs.  qk_norm = 1 for model_type "qwen3" (transformer.rs:193).
 * Qwen3-MoE (Qwen3MoeModelArgs, qwen3_moe.rs:37-97): num_experts > 0 enables
 * the sparse block on every layer that registers "mlp.gate" (router) and
 * "mlp.switch_mlp.{gate,up,down}_proj"; the others stay dense. */
typedef struct {
  int hidden, layers, intermediate, heads, kv_heads, head_dim, vocab;
  float rms_eps, rope_theta;
  int tie_word_embeddings;
  int qk_norm;
  int kv_mode; /* HIGGS_KV_BF16 or HIGGS_KV_TQ4 */
  int num_experts, experts_per_tok, moe_intermediate, norm_topk_prob;
  /* Tensor parallelism (no reference counterpart): with tp_world > 1 the model
   * is this rank's shard -- heads, kv_heads and intermediate are the per-rank
   * counts (column-parallel q|k|v and gate|up, row-parallel o_proj / down_proj
   * over K), the LM head holds rows [tp_rank*head_rows, (tp_rank+1)*head_rows)
   * of the vocabulary (the embedding stays whole), and a communicator from
   * higgs_comm_create / higgs_model_set_comm sums the row-parallel partials
   * and reduces the greedy argmax over the shards.  head_rows = vocab when
   * tp_world <= 1. */
  int tp_world, tp_rank, head_rows;
} higgs_model_config;

/* One forward over B sequences x Lq new tokens (Lq = 1 decode, k+1 verify,
 * larger for a prefill chunk).  All vectors are device memory:
 *   tokens, positions int32 [B*Lq]; slot_mapping int64 [B*Lq] (page*16+slot,
 *   <0 = do not store); block_table int32 [B, max_blocks]; seq_lens int32 [B]
 *   (cache length after this step).  max_seq_len bounds seq_lens.
 *   n_layers > 0 runs only the first n_layers (layer-skip draft), 0 = all.
 *   last_only = 1 applies the LM head to the last token of each sequence only.
 *   logits f32 [rows, V] and/or argmax int32 [rows] (rows = B or B*Lq);
 *   hidden_out bf16 [rows, hidden] (optional) receives the final-norm output. */
typedef struct {
  int B, Lq;
  const int32_t* tokens;
  const int32_t* positions;
  const int64_t* slot_mapping;
  const int32_t* block_table;
  int max_blocks;
  const int32_t* seq_lens;
  int max_seq_len;
  int n_layers;
  int last_only;
  float* logits;
  int32_t* argmax;
  void* hidden_out;
  void* workspace;
  size_t workspace_bytes;
} higgs_forward_args;

/* Model::new + load_model (crates/higgs-models/src/transformer.rs:552, 922-960).
 * Tensors are registered by their MLX safetensors names (lib.rs:604-723), e.g.
 * "model.layers.3.self_attn.q_proj.weight" u32 [N, K/8], "...scales" bf16;
 * nothing is copied: pointers must stay valid for the model's lifetime. */
int higgs_model_create(higgs_ctx* ctx, const higgs_model_config* cfg, higgs_model** out);
int higgs_model_set_tensor(higgs_model* m, const char* name, const void* ptr, int dtype,
                           const int64_t* shape, int ndim);
int higgs_model_finalize(higgs_model* m);
/* Attach the communicator of a tensor-parallel shard (cfg.tp_world > 1); it
 * must hold at least 2 x layers + 1 call regions of B*Lq*hidden words. */
int higgs_model_set_comm(higgs_model* m, higgs_comm* comm);
int higgs_model_destroy(higgs_model* m);

/* Paged KV pools for all layers: bf16 [layers, pages, Hkv, 16, D] each; or
 * TurboQuant codes u8 [layers, pages, Hkv, 16, 64] + fp16 scales
 * [layers, pages, Hkv, 16] with the Hadamard signs int8 [128].  Replaces the
 * per-request SteppingKeyValueCache (crates/higgs-models/src/cache.rs:130-312). */
int higgs_model_set_kv_cache(higgs_model* m, void* k_pool, void* v_pool, int64_t num_pages);
int higgs_model_set_kv_cache_tq4(higgs_model* m, uint8_t* k_codes, void* k_scales,
                                 uint8_t* v_codes, void* v_scales, int64_t num_pages,
                                 const int8_t* signs);

/* Bytes of scratch higgs_model_forward needs for (B, Lq, max_seq_len, last_only).
 * The workspace must be zero-filled before its first use; every forward leaves
 * its counters (attention splits, decode-chain barriers) zeroed again. */
size_t higgs_model_workspace_size(const higgs_model* m, int B, int Lq, int max_seq_len,
                                  int last_only);

/* AnyModel::forward / forward_batched (crates/higgs-models/src/lib.rs:123,165;
 * transformer.rs:590-598, 663-827) on the device; enqueues only. */
int higgs_model_forward(higgs_model* m, const higgs_forward_args* args, void* stream);

/* Capture one higgs_model_forward into a CUDA graph (replaces the per-token
 * async_eval submission, crates/higgs-engine/src/simple.rs:539-562).  The
 * graph re-reads the argument vectors on every launch, so updating tokens /
 * positions / slots / lengths in place and relaunching runs the next step. */
int higgs_model_capture(higgs_model* m, const higgs_forward_args* args, void* stream,
                        higgs_graph** out);
int higgs_graph_launch(higgs_graph* g, void* stream);
/* Kernel launches one replay of the captured graph performs. */
int higgs_graph_num_kernels(const higgs_graph* g);
int higgs_graph_destroy(higgs_graph* g);

/* ---- a12/a13: KV page pool and radix prefix cache (host side) ----------- */

/* Refcounted pool of KV page ids [0, num_pages).  Replaces per-request cache
 * growth (crates/higgs-models/src/cache.rs:245-277): a sequence owns the pages
 * of its block-table row; shared prefix pages carry one reference per owner.
 * alloc is all-or-nothing (HIGGS_ERR_OUT_OF_PAGES); release frees a page when
 * its count reaches zero.  Host memory only; not thread-safe. */
int higgs_block_pool_create(int64_t num_pages, higgs_block_pool** out);
int higgs_block_pool_destroy(higgs_block_pool* pool);
int64_t higgs_block_pool_num_free(const higgs_block_pool* pool);
int higgs_block_pool_alloc(higgs_block_pool* pool, int n, int32_t* pages);
int higgs_block_pool_retain(higgs_block_pool* pool, const int32_t* pages, int n);
int higgs_block_pool_release(higgs_block_pool* pool, const int32_t* pages, int n);
int higgs_block_pool_refcount(const higgs_block_pool* pool, int32_t page);

/* PrefixCache (crates/higgs-engine/src/prompt_cache.rs:41-311) over pages:
 * a compressed radix trie of token ids whose entries hold page ids.  Only the
 * whole 16-token pages of a stored prefix are kept (never the partly filled
 * last page), matches need >= 16 tokens (prompt_cache.rs:8), the deepest
 * match wins, and entries beyond max_entries are evicted least recently used.
 * Unlike the reference, which reuses a stored prompt only when all of it
 * prefixes the query, any shared prefix is reused in whole pages (pages are
 * immutable, so a stored prompt's leading pages serve every prefix of it). 
 * lookup copies the matched pages to pages_out, sets *matched_tokens (0 = no
 * hit) and retains those pages for the caller, who releases them with the
 * sequence.  store retains the pages it keeps. */
int higgs_prefix_cache_create(higgs_block_pool* pool, int max_entries, higgs_prefix_cache** out);
int higgs_prefix_cache_destroy(higgs_prefix_cache* pc);
int higgs_prefix_cache_len(const higgs_prefix_cache* pc);
int higgs_prefix_cache_clear(higgs_prefix_cache* pc);
int higgs_prefix_cache_lookup(higgs_prefix_cache* pc, const int32_t* tokens, int n,
                              int32_t* pages_out, int max_pages, int* matched_tokens);
int higgs_prefix_cache_store(higgs_prefix_cache* pc, const int32_t* tokens, int n,
                             const int32_t* pages, int n_pages);

/* ---- (f)2: MLX-format safetensors model directories --------------------- */

/* collect_safetensors_files + Array::load_safetensors
 * (crates/higgs-models/src/lib.rs:604-723): opens model_dir's
 * model.safetensors.index.json (every file its weight_map names) or its single
 * model.safetensors, and memory-maps the files.  Tensor names are looked up
 * as stored or with ".inner" segments removed (the reverse of
 * remap_quantized_key, lib.rs:709-723), so both naming styles load.
 * dtypes: U32 / I32 (packed codes, HIGGS_DTYPE_U32), BF16, F32, F16. */
int higgs_safetensors_open(const char* model_dir, higgs_safetensors** out);
int higgs_safetensors_close(higgs_safetensors* st);
int higgs_safetensors_count(const higgs_safetensors* st);
/* Index of the tensor called `name`, or -1 (not an error). */
int higgs_safetensors_find(const higgs_safetensors* st, const char* name);
/* Tensor i: its name (the ".inner"-free form; valid until close), dtype,
 * rank and shape (up to 8 dims, written to shape[0..ndim)). */
int higgs_safetensors_info(const higgs_safetensors* st, int i, const char** name, int* dtype,
                           int* ndim, int64_t* shape);
/* Copies rows [row0, row0 + rows) x columns [col0, col0 + cols) of tensor i
 * (leading dims flattened into rows, columns = elements of the last dim) to
 * dst, densely packed (row pitch cols * element size): host memory, or (with
 * dst_on_device and a context) device memory through `stream`, complete on
 * return.  A tensor-parallel rank reads only its own shard this way. */
int higgs_safetensors_read(higgs_ctx* ctx, const higgs_safetensors* st, int i, int64_t row0,
                           int64_t rows, int64_t col0, int64_t cols, void* dst, int dst_on_device,
                           void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HIGGS_CUDA_H */
