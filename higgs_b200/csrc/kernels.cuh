// kernels.cuh -- internal (C++) launch interfaces shared by the C-ABI entry
// points and the native decode-step runner.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace higgs {

enum { EPI_STORE = 0, EPI_SWIGLU = 1 };

constexpr int kMaxRanks = 8;  // tensor-parallel ranks per communicator

// tensor-parallel collectives (comm.cu)
cudaError_t comm_step(higgs_comm* c, cudaStream_t st);
cudaError_t comm_allreduce_residual(higgs_comm* c, int call, const float* partial, int n, uint16_t* h,
                                    cudaStream_t st);
cudaError_t comm_allreduce_argmax(higgs_comm* c, int call, const unsigned long long* keys, int n,
                                  int32_t* out, cudaStream_t st);
// greedy argmax keys of rows of f32 logits whose column j is vocabulary id j + offset
cudaError_t launch_argmax_keys(const float* logits, int B, int V, int offset, unsigned long long* keys,
                               cudaStream_t st);

// Tensor-parallel sum fused into a row-parallel one-token GEMV (the producer) and the
// fused-norm GEMV that consumes its result (comm.cu's buffers and step counter).
//   producer (push): every CTA writes its f32 output rows straight into slot (call, rank) of
//     every rank's buffer; the CTA that completes this rank's arrival count publishes flag
//     (call, rank) = step on every rank.
//   consumer (pull): waits until flag (call, q) == step for every rank q, then forms
//     x = bf16(h_in + bf16(sum_q slot_q)) (ranks in order: the all-reduce kernel's bits);
//     CTA 0 also stores it to h_out, the residual stream of the rest of the step.
struct TpFuse {
  char* peer[kMaxRanks];  // each rank's buffer (flags | data)
  int rank, world, call, max_ctas;
  size_t flag_bytes, words;
  const unsigned* step;
  int* err;
  const uint16_t* h_in;
  uint16_t* h_out;
};
// flag words of a call's (call, src) flag block used by the fused protocol (the all-reduce
// kernel uses the block's first max_ctas - 2 words)
constexpr int kTpFlagWord = 31;   // "rank src has pushed call", value = step
constexpr int kTpCountWord = 30;  // this rank's arrival count for the call (own buffer only)

struct QLinArgs {
  const uint16_t* x;
  int M, K, N;
  const uint32_t* w;
  const uint16_t* s;
  const uint16_t* b;
  // optional row segments: rows [seg_end[i-1], seg_end[i]) come from weight i
  // (segment 0 is w/s/b); lets q|k|v run as one launch over separate tensors
  int nseg;
  int seg_end[3];
  const uint32_t* wseg[3];
  const uint16_t* sseg[3];
  const uint16_t* bseg[3];
  const uint32_t* w2;  // up projection (SwiGLU)
  const uint16_t* s2;
  const uint16_t* b2;
  uint16_t* y;
  float* y_f32;
  const uint16_t* residual;
  // optional fused RMSNorm of x (ring GEMV only): x is the residual stream h
  const uint16_t* norm_w;
  float eps;
  // grouped experts (MoE, ring GEMV only): blockIdx.y picks a work item
  // {expert, first slot in moe_sorted, pairs} of the routing plan; x row of pair
  // p = p / moe_xdiv, output row = p; w/s/b (and w2/s2/b2) advance by
  // expert * moe_ew u32 words / expert * moe_es bf16 elements.
  const int4* moe_items;
  const int* moe_n_items;
  const int* moe_sorted;
  int moe_max_items;
  int moe_xdiv;
  long long moe_ew, moe_es;
  // expert parallelism: only experts [moe_e_lo, moe_e_lo + moe_e_n) live here (0 = all)
  int moe_e_lo, moe_e_n;
  // scratch for the tensor-core path's split-K partials (M >= 17; may be null)
  void* tc_ws;
  size_t tc_ws_bytes;
  // weights of a later launch to pull into L2 (the next GEMV of the step)
  L2Prefetch pf;
  // also prefetch this CTA's own weight tiles to L2 at its start
  int self_prefetch;
  // single-token GEMV: weight units prefetched into L1 ahead of its register ring (0 = off)
  int m1_l1_ahead;
  // single-token GEMV only: push the f32 output to every rank / pull the ranks' sum into x
  int tp_push, tp_pull;
  TpFuse tp;
};
// the TpFuse of call `call` of communicator c
TpFuse comm_tp_fuse(const higgs_comm* c, int call);

// Routing plan of the MoE router (moe.cu), in one buffer:
//   int  header[4]  {n_items, n_pairs, E, k}
//   int4 items[max_items]   {expert, first slot, pairs (<= 8), 0}
//   int  sorted[T*k]        pairs grouped by expert, ascending within an expert
//   int  counts[E]
inline int moe_max_items(int P, int E) { return P / 8 + (E < P ? E : P) + 1; }
size_t moe_plan_bytes(int T, int E, int k);
cudaError_t launch_moe_route(const void* logits, bool bf16_in, int T, int E, int k, int norm,
                             int32_t* idx, float* scores, void* plan, cudaStream_t st);
cudaError_t launch_moe_grouped(const uint16_t* x, int T, int K, int k, bool x_per_pair,
                               const void* plan, int E, int N, const uint32_t* w, const uint16_t* s,
                               const uint16_t* b, const uint32_t* w2, const uint16_t* s2,
                               const uint16_t* b2, uint16_t* y, cudaStream_t st, int e_lo = 0,
                               int e_n = 0);
// expert parallelism: this rank's share of the weighted sum, f32 [T, H], pairs whose expert
// lies outside [e_lo, e_lo + e_n) contribute nothing
cudaError_t launch_moe_combine_partial(const uint16_t* y, const float* scores, const int32_t* idx,
                                       int T, int k, int H, int e_lo, int e_n, float* part,
                                       cudaStream_t st);
cudaError_t launch_moe_router(const uint16_t* x, int T, int K, const uint32_t* w,
                              const uint16_t* s, const uint16_t* b, int E, uint16_t* out,
                              cudaStream_t st);
cudaError_t launch_moe_combine(const uint16_t* y, const float* scores, int T, int k, int H,
                               uint16_t* h, cudaStream_t st);

// W4 GEMV with per-warp cp.async rings (any M, 32 rows per pass; norm_w needs
// qgemv_ring_can_fuse_norm(M, K)).
cudaError_t launch_qgemv_ring(const QLinArgs& a, int epi, cudaStream_t st);
// process-wide switches for the L2 prefetch fields (QLinArgs::pf, self_prefetch)
bool l2_prefetch_next();
bool l2_prefetch_self();
bool qgemv_ring_can_fuse_norm(int M, int K);
// higgs_fused_attention with an L2 prefetch list for the decode step's later GEMVs
int fused_attention_launch(higgs_ctx* ctx, const void* qkv, int B, int Lq, int Hq, int Hkv, int D,
                           const void* q_norm_w, const void* k_norm_w, float eps,
                           const int32_t* positions, const float* inv_freq,
                           const int64_t* slot_mapping, void* k_cache, void* v_cache,
                           int64_t page_stride, int64_t head_stride, const int32_t* block_table,
                           int max_blocks, const int32_t* seq_lens, int max_seq_len, float scale,
                           void* out, void* workspace, size_t workspace_bytes, void* stream,
                           const L2Prefetch* pf);
// M == 1 (decode at batch 1): the register-fed GEMV of qgemv_m1.cu; launch_qgemv_ring routes there itself.
bool qgemv_m1_supported(const QLinArgs& a);
cudaError_t launch_qgemv_m1(const QLinArgs& a, int epi, cudaStream_t st);
// one token, weights streamed by TMA into a shared-memory ring (qgemv_tma.cu)
bool qgemv_tma_supported(const QLinArgs& a);
cudaError_t launch_qgemv_tma(const QLinArgs& a, int epi, cudaStream_t st);
void qgemv_tma_set(int on);

// One GEMV phase of a decode chain (qgemv_m1.cu): y = W x for one token, with an optional
// fused RMSNorm of x, SwiGLU over gate (w) / up (w2), q|k|v row segments and a residual
// epilogue; wk (the K split) is filled in by launch_decode_chain.
constexpr int kChainMaxPhases = 4;
constexpr int kChainBarWords = 64;  // u32 barrier words per phase
struct ChainPhase {
  const uint16_t* x;       // input [K] (bf16), written before the launch or by an earlier phase
  const uint16_t* norm_w;  // fused RMSNorm of x (null: none)
  int K, N, wk, swiglu;
  int nseg;  // row segments (q|k|v); segment 0 is w[0]
  int seg_end[3];
  const uint32_t* w[3];
  const uint16_t* s[3];
  const uint16_t* b[3];
  const uint32_t* w2;  // up projection (SwiGLU)
  const uint16_t* s2;
  const uint16_t* b2;
  uint16_t* y;
  float* y_f32;
  const uint16_t* residual;
};
// Whether the persistent decode chain replaces the separate one-token GEMV launches
// (higgs_set_option("decode_chain")) and whether a phase fits it.
bool decode_chain_on();
bool decode_chain_fits(const ChainPhase& p);
// nph (<= kChainMaxPhases) phases in one launch; bar: nph * kChainBarWords zeroed u32 words
// this launch leaves zeroed again.  Bounded waits report through the per-device timeout flag.
cudaError_t launch_decode_chain(ChainPhase* ph, int nph, float eps, unsigned* bar, cudaStream_t st);
void decode_chain_set(int on, int l2_ahead);
void qgemv_m1_set(int on, int wk, int depth, int l2, int persist, int l1);  // -1 leaves a setting as it is
// M >= 17: the tcgen05 matrix path (qgemm_tc.cu); launch_qgemv_ring routes there itself.
bool qgemm_tc_supported(const QLinArgs& a);
size_t qgemm_tc_workspace(int M, int K, int N, bool swiglu);
cudaError_t launch_qgemm_tc(const QLinArgs& a, int epi, void* ws, size_t ws_bytes, cudaStream_t st);
void qgemm_tc_prepare();
// Grouped-expert variant (the a.moe_* fields set): K * 8 tokens must fit the staged-x tile.
cudaError_t launch_qgemv_grouped(const QLinArgs& a, int epi, cudaStream_t st);
bool qgemv_grouped_supported(int K);

// M may exceed 32 (processed in 32-row passes); K % 256 == 0, N % 16 == 0.
cudaError_t launch_qlinear(const QLinArgs& a, int epi, cudaStream_t st);

// Stream-K GEMV (M <= 8), optional fused RMSNorm of x with norm_w.
struct SkArgs {
  const uint16_t* x;
  const uint16_t* norm_w;
  float eps;
  int M, K, N;
  int n_tiles;  // 16-row weight tiles (SwiGLU: gate/up interleaved, 2 per output tile)
  int swiglu;
  int nseg;
  int seg_end[3];
  const uint32_t* wseg[3];
  const uint16_t* sseg[3];
  const uint16_t* bseg[3];
  uint16_t* y;
  float* y_f32;
  const uint16_t* residual;
  // filled by the launcher from the workspace
  int max_slots;
  int* counters;
  float* partials;
};
size_t qgemv_sk_workspace(int M, int K, int n_tiles);
cudaError_t launch_qgemv_sk(SkArgs a, void* workspace, cudaStream_t st);

// prefill_attn.cu: causal paged attention of prefill chunks on the tcgen05 tensor cores
bool prefill_attn_tc_fits(int Lq, int Hq, int Hkv, int D, const void* q, const void* kc, const void* vc,
                          const void* out, int64_t page_stride, int64_t head_stride);
cudaError_t launch_prefill_attn_tc(const void* q, int B, int Lq, int Hq, int Hkv, int D, const void* kc,
                                   const void* vc, int64_t page_stride, int64_t head_stride, const int32_t* bt,
                                   int max_blocks, const int32_t* seq_lens, float scale, void* out, int* counters,
                                   int* err, cudaStream_t st);
int* tc_err_ptr();

}  // namespace higgs
