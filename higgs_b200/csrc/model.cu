// model.cu -- native decode/verify/prefill step of the dense transformer
// (Llama / Mistral / Qwen2 / Qwen3) over a paged KV cache, and CUDA-graph
// capture of that step.
//
// Mirrors Model::forward / forward_batched of the reference
// (crates/higgs-models/src/transformer.rs:487-526, 663-827): embedding ->
// N x [RMSNorm -> q|k|v -> (qk-norm) -> RoPE -> KV append -> SDPA -> o_proj +
// residual -> RMSNorm -> SwiGLU MLP + residual] -> RMSNorm -> LM head (tied to
// the embedding when tie_word_embeddings, transformer.rs:830-838).  The
// per-request host loop of forward_batched (transformer.rs:747-802) is gone:
// RoPE positions, cache slots and sequence lengths are device vectors, so one
// launch sequence serves any mix of sequence lengths and the whole step can be
// captured once and replayed.
//
// Weights are caller-owned device tensors registered under their MLX
// safetensors names (lib.rs:604-723 loads the same keys); nothing is copied.
#include <algorithm>
#include <cmath>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"
#include "kernels.cuh"

namespace higgs {

struct TensorRef {
  const void* ptr = nullptr;
  int dtype = 0;  // HIGGS_DTYPE_*
  std::vector<int64_t> shape;
};

struct QW {
  const uint32_t* w = nullptr;
  const uint16_t* s = nullptr;
  const uint16_t* b = nullptr;
  int N = 0, K = 0;
};

struct LayerW {
  const uint16_t* ln_in = nullptr;
  const uint16_t* ln_post = nullptr;
  QW q, k, v, o, gate, up, down;
  const uint16_t* qn = nullptr;
  const uint16_t* kn = nullptr;
  // sparse block (Qwen3MoeMlpBlock): router [E, H] and stacked experts [E, N, K]
  bool moe = false;
  QW router, egate, eup, edown;  // e*: w/s/b point at expert 0, N/K per expert
};

cudaError_t attention_prepare();

// One-token steps of a dense tensor-parallel model: the sum over ranks after each
// row-parallel GEMV is pushed by that GEMV's CTAs and pulled by the next fused-norm GEMV
// (no all-reduce launch; higgs_set_option("tp_fuse")).  Off by default: measured on two
// B200s it lengthened the B=1 step (2.43 ms against 2.00 with the all-reduce launches).
static bool g_tp_fuse = false;
void model_set_tp_fuse(int on) { g_tp_fuse = on != 0; }

}  // namespace higgs

using namespace higgs;

struct higgs_model {
  higgs_ctx* ctx = nullptr;
  higgs_model_config cfg{};
  std::unordered_map<std::string, TensorRef> tensors;
  bool finalized = false;
  std::vector<LayerW> layers;
  QW embed, head;
  const uint16_t* final_norm = nullptr;
  float* inv_freq = nullptr;  // device [D/2]
  // KV pools
  void* k_pool = nullptr;
  void* v_pool = nullptr;
  void* k_scales = nullptr;
  void* v_scales = nullptr;
  const int8_t* signs = nullptr;
  int64_t num_pages = 0;
  higgs_comm* comm = nullptr;  // tensor-parallel shard: sums / argmax over ranks
};

struct higgs_graph {
  int device = 0;  // the capturing model's device
  cudaGraphExec_t exec = nullptr;
  int kernel_nodes = 0;
};

namespace {

constexpr size_t kAlign = 256;

size_t align_up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

struct WsLayout {
  size_t h, h2, x, qkv, q, attn, act, xl, logits, moe_rl, moe_idx, moe_sc, moe_plan, moe_act, moe_y,
      tp_part, tp_keys, tc_ws, tc_ws_bytes, chain_bar, attn_ws, total;
};

int head_rows(const higgs_model_config& c) { return c.tp_world > 1 ? c.head_rows : c.vocab; }




WsLayout layout(const higgs_model_config& c, int B, int Lq, int max_seq_len, bool last_only) {
  const size_t T = (size_t)B * Lq;
  const size_t rows_lm = last_only ? (size_t)B : T;
  const int D = c.head_dim;
  WsLayout L{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += align_up(bytes);
    return o;
  };
  L.h = take(T * c.hidden * 2);
  L.h2 = take(T * c.hidden * 2);  // the other residual buffer of the fused tensor-parallel sum
  L.x = take(T * c.hidden * 2);
  L.qkv = take(T * (size_t)(c.heads + 2 * c.kv_heads) * D * 2);
  L.q = take(T * (size_t)c.heads * D * 2);
  L.attn = take(T * (size_t)c.heads * D * 2);
  L.act = take(T * (size_t)c.intermediate * 2);
  L.xl = take(rows_lm * c.hidden * 2);
  L.logits = take(rows_lm * (size_t)head_rows(c) * 4);
  if (c.tp_world > 1) {
    L.tp_part = take(T * c.hidden * 4);
    L.tp_keys = take(rows_lm * 8);
  }
  {  // split-K partials of the tensor-core path (a few MB; used from 17 rows by default)
    const int H = c.hidden, Hd = c.heads * D, Nqkv = (c.heads + 2 * c.kv_heads) * D;
    size_t need = qgemm_tc_workspace((int)T, H, Nqkv, false);
    need = std::max(need, qgemm_tc_workspace((int)T, Hd, H, false));
    need = std::max(need, qgemm_tc_workspace((int)T, H, c.intermediate, true));
    need = std::max(need, qgemm_tc_workspace((int)T, c.intermediate, H, false));
    need = std::max(need, qgemm_tc_workspace((int)rows_lm, H, head_rows(c), false));
    L.tc_ws_bytes = need;
    L.tc_ws = take(need);
  }
  if (c.num_experts > 0) {
    const size_t P = T * c.experts_per_tok;
    L.moe_rl = take(T * (size_t)c.num_experts * 2);
    L.moe_idx = take(P * 4);
    L.moe_sc = take(P * 4);
    L.moe_plan = take(moe_plan_bytes((int)T, c.num_experts, c.experts_per_tok));
    L.moe_act = take(P * (size_t)c.moe_intermediate * 2);
    L.moe_y = take(P * (size_t)c.hidden * 2);
  }
  // decode-chain barrier counters, kChainMaxPhases per layer (zero between launches)
  L.chain_bar = take((size_t)c.layers * kChainMaxPhases * kChainBarWords * 4);
  const size_t aws = higgs_paged_attention_workspace_size(B, Lq, c.heads, c.kv_heads, D, max_seq_len);
  L.attn_ws = take(aws);
  L.total = off;
  return L;
}

int get_q(higgs_model* m, const std::string& base, int N, int K, QW& out) {
  auto it_w = m->tensors.find(base + ".weight");
  auto it_s = m->tensors.find(base + ".scales");
  auto it_b = m->tensors.find(base + ".biases");
  if (it_w == m->tensors.end() || it_s == m->tensors.end() || it_b == m->tensors.end())
    return fail(HIGGS_ERR_STATE, "model: missing quantized tensor " + base + ".{weight,scales,biases}");
  const TensorRef& w = it_w->second;
  const TensorRef& s = it_s->second;
  const TensorRef& b = it_b->second;
  auto shape_is = [](const TensorRef& t, int64_t a, int64_t bb) {
    return t.shape.size() == 2 && t.shape[0] == a && t.shape[1] == bb;
  };
  if (w.dtype != HIGGS_DTYPE_U32 || !shape_is(w, N, K / 8))
    return fail(HIGGS_ERR_INVALID_ARG, "model: " + base + ".weight must be u32 [" +
                                           std::to_string(N) + ", " + std::to_string(K / 8) + "]");
  if (s.dtype != HIGGS_DTYPE_BF16 || !shape_is(s, N, K / 64) || b.dtype != HIGGS_DTYPE_BF16 ||
      !shape_is(b, N, K / 64))
    return fail(HIGGS_ERR_INVALID_ARG, "model: " + base + ".{scales,biases} must be bf16 [" +
                                           std::to_string(N) + ", " + std::to_string(K / 64) + "]");
  out.w = (const uint32_t*)w.ptr;
  out.s = (const uint16_t*)s.ptr;
  out.b = (const uint16_t*)b.ptr;
  out.N = N;
  out.K = K;
  return HIGGS_OK;
}

// stacked expert tensor [E, N, K/8] u32 + [E, N, K/64] bf16 scales / biases
int get_q3(higgs_model* m, const std::string& base, int E, int N, int K, QW& out) {
  auto it_w = m->tensors.find(base + ".weight");
  auto it_s = m->tensors.find(base + ".scales");
  auto it_b = m->tensors.find(base + ".biases");
  if (it_w == m->tensors.end() || it_s == m->tensors.end() || it_b == m->tensors.end())
    return fail(HIGGS_ERR_STATE, "model: missing quantized tensor " + base + ".{weight,scales,biases}");
  auto shape_is = [](const TensorRef& t, int64_t a, int64_t b, int64_t c) {
    return t.shape.size() == 3 && t.shape[0] == a && t.shape[1] == b && t.shape[2] == c;
  };
  const std::string dims = "[" + std::to_string(E) + ", " + std::to_string(N) + ", ";
  if (it_w->second.dtype != HIGGS_DTYPE_U32 || !shape_is(it_w->second, E, N, K / 8))
    return fail(HIGGS_ERR_INVALID_ARG, "model: " + base + ".weight must be u32 " + dims +
                                           std::to_string(K / 8) + "]");
  for (auto* t : {&it_s->second, &it_b->second})
    if (t->dtype != HIGGS_DTYPE_BF16 || !shape_is(*t, E, N, K / 64))
      return fail(HIGGS_ERR_INVALID_ARG, "model: " + base + ".{scales,biases} must be bf16 " + dims +
                                             std::to_string(K / 64) + "]");
  out.w = (const uint32_t*)it_w->second.ptr;
  out.s = (const uint16_t*)it_s->second.ptr;
  out.b = (const uint16_t*)it_b->second.ptr;
  out.N = N;
  out.K = K;
  return HIGGS_OK;
}

int get_vec(higgs_model* m, const std::string& name, int n, const uint16_t*& out) {
  auto it = m->tensors.find(name);
  if (it == m->tensors.end()) return fail(HIGGS_ERR_STATE, "model: missing tensor " + name);
  const TensorRef& t = it->second;
  if (t.dtype != HIGGS_DTYPE_BF16 || t.shape.size() != 1 || t.shape[0] != n)
    return fail(HIGGS_ERR_INVALID_ARG, "model: " + name + " must be bf16 [" + std::to_string(n) + "]");
  out = (const uint16_t*)t.ptr;
  return HIGGS_OK;
}

int forward_impl(higgs_model* m, const higgs_forward_args* f, cudaStream_t st) {
  const higgs_model_config& c = m->cfg;
  const int B = f->B, Lq = f->Lq;
  const int T = B * Lq;
  const int D = c.head_dim, H = c.hidden;
  const bool tq = c.kv_mode == HIGGS_KV_TQ4;
  const int n_layers = f->n_layers > 0 ? f->n_layers : c.layers;
  const WsLayout L = layout(c, B, Lq, f->max_seq_len, f->last_only != 0);
  if (f->workspace_bytes < L.total)
    return fail(HIGGS_ERR_WORKSPACE, "higgs_model_forward: workspace too small (need " +
                                         std::to_string(L.total) + " bytes)");
  char* ws = (char*)f->workspace;
  uint16_t* h = (uint16_t*)(ws + L.h);
  uint16_t* x = (uint16_t*)(ws + L.x);
  uint16_t* qkv = (uint16_t*)(ws + L.qkv);
  uint16_t* q = (uint16_t*)(ws + L.q);
  uint16_t* attn = (uint16_t*)(ws + L.attn);
  uint16_t* act = (uint16_t*)(ws + L.act);
  uint16_t* xl = (uint16_t*)(ws + L.xl);
  float* logits = f->logits ? f->logits : (float*)(ws + L.logits);
  void* aws = ws + L.attn_ws;
  const size_t aws_bytes = L.total - L.attn_ws;
  const float scale = 1.0f / std::sqrt((float)D);
  const int64_t kv_layer_elems = m->num_pages * c.kv_heads * HIGGS_PAGE_SIZE * (int64_t)D;
  const int64_t tq_layer_bytes = m->num_pages * c.kv_heads * HIGGS_PAGE_SIZE * 64;
  const int64_t tq_layer_scales = m->num_pages * c.kv_heads * HIGGS_PAGE_SIZE;

  // decode batches fuse each RMSNorm into the GEMV that consumes it
  const bool fuse = qgemv_ring_can_fuse_norm(T, H);
  void* tc_ws = L.tc_ws_bytes ? (void*)(ws + L.tc_ws) : nullptr;
  // L2 prefetch lists: each GEMV asks for the weights of a later GEMV of the step
  const bool pfon = l2_prefetch_next(), pfself = l2_prefetch_self();
  auto add_q = [&](L2Prefetch& pf, const QW& w, size_t max_bytes = ~(size_t)0) {
    if (!pfon || !w.w || pf.n + 3 > L2Prefetch::kMax) return;
    const size_t wb = (size_t)w.N * w.K / 2, sb = (size_t)w.N * (w.K / 64) * 2;
    const double f = max_bytes < wb ? (double)max_bytes / wb : 1.0;  // leading rows only
    const size_t rows = (size_t)(w.N * f) / 16 * 16;
    pf.ptr[pf.n] = w.w;
    pf.bytes[pf.n++] = rows * (w.K / 2);
    pf.ptr[pf.n] = w.s;
    pf.bytes[pf.n++] = rows * (w.K / 64) * 2;
    pf.ptr[pf.n] = w.b;
    pf.bytes[pf.n++] = rows * (w.K / 64) * 2;
    (void)sb;
  };
  auto lin = [&](const QW& w, const uint16_t* xin, const uint16_t* norm, uint16_t* y, float* yf,
                 const uint16_t* res, const L2Prefetch* pf = nullptr) {
    QLinArgs a{};
    a.self_prefetch = pfself;
    a.tc_ws = tc_ws;
    a.tc_ws_bytes = L.tc_ws_bytes;
    if (pf) a.pf = *pf;
    a.x = xin;
    a.norm_w = norm;
    a.eps = c.rms_eps;
    a.M = T;
    a.K = w.K;
    a.N = w.N;
    a.w = w.w;
    a.s = w.s;
    a.b = w.b;
    a.nseg = 1;
    a.y = y;
    a.y_f32 = yf;
    a.residual = res;
    return launch_qgemv_ring(a, EPI_STORE, st);
  };
  const bool tp = c.tp_world > 1;
  float* part = tp ? (float*)(ws + L.tp_part) : nullptr;
  if (tp) HG_CUDA(comm_step(m->comm, st));
  // fused tensor-parallel sum (one token, dense layers): the residual stream alternates
  // between h and h2, each pull writing the other
  const bool tpf = tp && T == 1 && fuse && g_tp_fuse && c.num_experts == 0;
  uint16_t* hc = h;
  uint16_t* ha = (uint16_t*)(ws + L.h2);
  int pull_call = -1;  // the pushed call the next fused-norm GEMV pulls (-1: none)
  auto set_pull = [&](QLinArgs& a) {
    if (pull_call < 0) return;
    a.tp_pull = 1;
    a.tp = comm_tp_fuse(m->comm, pull_call);
    a.tp.h_in = hc;
    a.tp.h_out = ha;
    a.x = hc;
  };
  auto after_pull = [&](const QLinArgs& a) {
    if (a.tp_pull) {
      std::swap(hc, ha);
      pull_call = -1;
    }
  };
  auto push_row_parallel = [&](const QW& w, const uint16_t* xin, int call) -> int {
    QLinArgs a{};
    a.x = xin;
    a.M = T;
    a.K = w.K;
    a.N = w.N;
    a.w = w.w;
    a.s = w.s;
    a.b = w.b;
    a.nseg = 1;
    a.tp_push = 1;
    a.tp = comm_tp_fuse(m->comm, call);
    HG_CUDA(launch_qgemv_ring(a, EPI_STORE, st));
    pull_call = call;
    return HIGGS_OK;
  };
  // row-parallel GEMV (o_proj / down_proj): this rank's K slice, then the sum over
  // ranks added to the residual stream, or the residual epilogue on one GPU
  auto row_parallel = [&](const QW& w, const uint16_t* xin, int call, const L2Prefetch* pf) -> int {
    if (!tp) {
      HG_CUDA(lin(w, xin, nullptr, h, nullptr, h, pf));
      return HIGGS_OK;
    }
    HG_CUDA(lin(w, xin, nullptr, nullptr, part, nullptr, pf));
    HG_CUDA(comm_allreduce_residual(m->comm, call, part, T * H, h, st));
    return HIGGS_OK;
  };
  // greedy tokens from this rank's logits (vocabulary shard under tensor parallelism)
  auto emit_argmax = [&](const float* lg, int rows) -> int {
    if (!tp) return higgs_argmax(m->ctx, lg, rows, c.vocab, f->argmax, st);
    unsigned long long* keys = (unsigned long long*)(ws + L.tp_keys);
    HG_CUDA(launch_argmax_keys(lg, rows, c.head_rows, c.tp_rank * c.head_rows, keys, st));
    HG_CUDA(comm_allreduce_argmax(m->comm, 2 * c.layers, keys, rows, f->argmax, st));
    return HIGGS_OK;
  };
  int rc = higgs_embed_gather_w4(m->ctx, f->tokens, T, m->embed.w, m->embed.s, m->embed.b, c.vocab,
                                 H, h, st);
  if (rc) return rc;
  // One token on one GPU: the GEMVs between two attention launches run as one persistent
  // decode-chain launch (o_proj, norm + gate/up, down, norm + the next q|k|v or the head).
  const bool chain = !tp && T == 1 && fuse && !tq && decode_chain_on() &&
                     (c.heads / c.kv_heads) * Lq <= 32;
  unsigned* chain_bar = (unsigned*)(ws + L.chain_bar);
  bool qkv_ready = false;   // the previous chain launch wrote this layer's q|k|v
  bool head_done = false;   // the last chain launch wrote the logits
  auto chain_qkv = [&](const LayerW& Ln, ChainPhase& P) {
    P = ChainPhase{};
    P.x = h;
    P.norm_w = Ln.ln_in;
    P.K = H;
    P.N = Ln.q.N + Ln.k.N + Ln.v.N;
    P.nseg = 3;
    P.seg_end[0] = Ln.q.N;
    P.seg_end[1] = Ln.q.N + Ln.k.N;
    P.seg_end[2] = P.N;
    P.w[0] = Ln.q.w, P.s[0] = Ln.q.s, P.b[0] = Ln.q.b;
    P.w[1] = Ln.k.w, P.s[1] = Ln.k.s, P.b[1] = Ln.k.b;
    P.w[2] = Ln.v.w, P.s[2] = Ln.v.s, P.b[2] = Ln.v.b;
    P.y = qkv;
  };
  for (int li = 0; li < n_layers; ++li) {
    const LayerW& Lw = m->layers[li];
    L2Prefetch next_pf{};
    const bool attn_fused = !tq && (c.heads / c.kv_heads) * Lq <= 32;
    if (!qkv_ready) {
      if (!fuse) {
        rc = higgs_rmsnorm(m->ctx, h, nullptr, T, H, Lw.ln_in, c.rms_eps, x, nullptr, st);
        if (rc) return rc;
      }
      QLinArgs a{};
      a.x = fuse ? h : x;
      a.norm_w = fuse ? Lw.ln_in : nullptr;
      if (tpf) set_pull(a);
      a.eps = c.rms_eps;
      a.M = T;
      a.K = H;
      a.N = Lw.q.N + Lw.k.N + Lw.v.N;
      a.w = Lw.q.w;
      a.s = Lw.q.s;
      a.b = Lw.q.b;
      a.nseg = 3;
      a.seg_end[0] = Lw.q.N;
      a.seg_end[1] = Lw.q.N + Lw.k.N;
      a.seg_end[2] = a.N;
      a.wseg[0] = Lw.q.w;
      a.sseg[0] = Lw.q.s;
      a.bseg[0] = Lw.q.b;
      a.wseg[1] = Lw.k.w;
      a.sseg[1] = Lw.k.s;
      a.bseg[1] = Lw.k.b;
      a.wseg[2] = Lw.v.w;
      a.sseg[2] = Lw.v.s;
      a.bseg[2] = Lw.v.b;
      a.y = qkv;
      a.self_prefetch = pfself;
      a.tc_ws = tc_ws;
      a.tc_ws_bytes = L.tc_ws_bytes;
      // the next GEMVs' weights: requested by the fused attention kernel when it runs
      // (latency-bound, HBM idle), else by this launch
      add_q(next_pf, Lw.o);
      if (Lw.moe) {
        add_q(next_pf, Lw.router);
      } else {
        add_q(next_pf, Lw.gate);
        add_q(next_pf, Lw.up);
      }
      if (!attn_fused) a.pf = next_pf;
      HG_CUDA(launch_qgemv_ring(a, EPI_STORE, st));
      after_pull(a);
    }
    qkv_ready = false;
    if (tq) {
      rc = higgs_qknorm_rope_kv_write_tq4(
          m->ctx, qkv, T, c.heads, c.kv_heads, Lw.qn, Lw.kn, c.rms_eps, f->positions, m->inv_freq,
          f->slot_mapping, m->signs, (uint8_t*)m->k_pool + li * tq_layer_bytes,
          (uint16_t*)m->k_scales + li * tq_layer_scales, (uint8_t*)m->v_pool + li * tq_layer_bytes,
          (uint16_t*)m->v_scales + li * tq_layer_scales, c.kv_heads * HIGGS_PAGE_SIZE * 64,
          HIGGS_PAGE_SIZE * 64, q, st);
      if (rc) return rc;
      rc = higgs_paged_attention_tq4(
          m->ctx, q, B, Lq, c.heads, c.kv_heads, (const uint8_t*)m->k_pool + li * tq_layer_bytes,
          (const uint16_t*)m->k_scales + li * tq_layer_scales,
          (const uint8_t*)m->v_pool + li * tq_layer_bytes,
          (const uint16_t*)m->v_scales + li * tq_layer_scales, c.kv_heads * HIGGS_PAGE_SIZE * 64,
          HIGGS_PAGE_SIZE * 64, f->block_table, f->max_blocks, f->seq_lens, f->max_seq_len,
          m->signs, scale, attn, aws, aws_bytes, st);
      if (rc) return rc;
    } else if ((c.heads / c.kv_heads) * Lq <= 32) {
      // decode / verify: norm + RoPE + append + attention in one kernel
      uint16_t* kc = (uint16_t*)m->k_pool + li * kv_layer_elems;
      uint16_t* vc = (uint16_t*)m->v_pool + li * kv_layer_elems;
      rc = fused_attention_launch(m->ctx, qkv, B, Lq, c.heads, c.kv_heads, D, Lw.qn, Lw.kn,
                                  c.rms_eps, f->positions, m->inv_freq, f->slot_mapping, kc, vc,
                                  (int64_t)c.kv_heads * HIGGS_PAGE_SIZE * D,
                                  (int64_t)HIGGS_PAGE_SIZE * D, f->block_table, f->max_blocks,
                                  f->seq_lens, f->max_seq_len, scale, attn, aws, aws_bytes, st,
                                  &next_pf);
      if (rc) return rc;
    } else {
      uint16_t* kc = (uint16_t*)m->k_pool + li * kv_layer_elems;
      uint16_t* vc = (uint16_t*)m->v_pool + li * kv_layer_elems;
      rc = higgs_qknorm_rope_kv_write(m->ctx, qkv, T, c.heads, c.kv_heads, D, Lw.qn, Lw.kn,
                                      c.rms_eps, f->positions, m->inv_freq, f->slot_mapping, kc, vc,
                                      (int64_t)c.kv_heads * HIGGS_PAGE_SIZE * D,
                                      (int64_t)HIGGS_PAGE_SIZE * D, q, st);
      if (rc) return rc;
      rc = higgs_paged_attention(m->ctx, q, B, Lq, c.heads, c.kv_heads, D, kc, vc,
                                 (int64_t)c.kv_heads * HIGGS_PAGE_SIZE * D,
                                 (int64_t)HIGGS_PAGE_SIZE * D, f->block_table, f->max_blocks,
                                 f->seq_lens, f->max_seq_len, scale, attn, aws, aws_bytes, st);
      if (rc) return rc;
    }
    if (chain && !Lw.moe) {
      ChainPhase ph[kChainMaxPhases];
      int n = 0;
      ChainPhase& o = ph[n++];  // h = h + o_proj(attn)
      o = ChainPhase{};
      o.x = attn, o.K = Lw.o.K, o.N = Lw.o.N, o.nseg = 1;
      o.w[0] = Lw.o.w, o.s[0] = Lw.o.s, o.b[0] = Lw.o.b;
      o.y = h, o.residual = h;
      ChainPhase& gu = ph[n++];  // act = swiglu(gate(norm(h)), up(norm(h)))
      gu = ChainPhase{};
      gu.x = h, gu.norm_w = Lw.ln_post, gu.K = H, gu.N = c.intermediate, gu.swiglu = 1, gu.nseg = 1;
      gu.w[0] = Lw.gate.w, gu.s[0] = Lw.gate.s, gu.b[0] = Lw.gate.b;
      gu.w2 = Lw.up.w, gu.s2 = Lw.up.s, gu.b2 = Lw.up.b;
      gu.y = act;
      ChainPhase& dn = ph[n++];  // h = h + down(act)
      dn = ChainPhase{};
      dn.x = act, dn.K = Lw.down.K, dn.N = Lw.down.N, dn.nseg = 1;
      dn.w[0] = Lw.down.w, dn.s[0] = Lw.down.s, dn.b[0] = Lw.down.b;
      dn.y = h, dn.residual = h;
      if (li + 1 < n_layers && !m->layers[li + 1].moe) {
        chain_qkv(m->layers[li + 1], ph[n]);
        if (decode_chain_fits(ph[n])) {
          ++n;
          qkv_ready = true;
        }
      } else if (li + 1 == n_layers && (f->logits || f->argmax) && !f->hidden_out) {
        ChainPhase& hd = ph[n];  // logits = head(norm(h))
        hd = ChainPhase{};
        hd.x = h, hd.norm_w = m->final_norm, hd.K = H, hd.N = m->head.N, hd.nseg = 1;
        hd.w[0] = m->head.w, hd.s[0] = m->head.s, hd.b[0] = m->head.b;
        hd.y_f32 = logits;
        if (decode_chain_fits(hd)) {
          ++n;
          head_done = true;
        }
      }
      HG_CUDA(launch_decode_chain(ph, n, c.rms_eps,
                                  chain_bar + (size_t)li * kChainMaxPhases * kChainBarWords, st));
      continue;
    }
    // h = h + o_proj(attn)   (in place: each element read then written by one thread)
    if (tpf) {
      if ((rc = push_row_parallel(Lw.o, attn, 2 * li))) return rc;
    } else {
      L2Prefetch pf{};
      if (!Lw.moe) add_q(pf, Lw.down);
      if ((rc = row_parallel(Lw.o, attn, 2 * li, &pf))) return rc;
    }
    if (Lw.moe) {
      // Qwen3MoeMlpBlock::forward_moe: router -> top-k plan -> grouped gate/up SwiGLU ->
      // grouped down -> weighted sum + residual
      const int E = c.num_experts, kk = c.experts_per_tok, F = c.moe_intermediate;
      uint16_t* rl = (uint16_t*)(ws + L.moe_rl);
      int32_t* idx = (int32_t*)(ws + L.moe_idx);
      float* sc = (float*)(ws + L.moe_sc);
      void* plan = ws + L.moe_plan;
      uint16_t* pact = (uint16_t*)(ws + L.moe_act);
      uint16_t* py = (uint16_t*)(ws + L.moe_y);
      rc = higgs_rmsnorm(m->ctx, h, nullptr, T, H, Lw.ln_post, c.rms_eps, x, nullptr, st);
      if (rc) return rc;
      {
        L2Prefetch pf{};
        if (li + 1 < n_layers) {
          add_q(pf, m->layers[li + 1].q);
          add_q(pf, m->layers[li + 1].k);
          add_q(pf, m->layers[li + 1].v);
        }
        (void)pf;
        HG_CUDA(launch_moe_router(x, T, H, Lw.router.w, Lw.router.s, Lw.router.b, E, rl, st));
      }
      HG_CUDA(launch_moe_route(rl, true, T, E, kk, c.norm_topk_prob, idx, sc, plan, st));
      // expert parallelism: this rank holds experts [e_lo, e_lo + e_n)
      const int e_n = tp ? E / c.tp_world : 0, e_lo = tp ? c.tp_rank * e_n : 0;
      HG_CUDA(launch_moe_grouped(x, T, H, kk, false, plan, E, F, Lw.egate.w, Lw.egate.s, Lw.egate.b,
                                 Lw.eup.w, Lw.eup.s, Lw.eup.b, pact, st, e_lo, e_n));
      HG_CUDA(launch_moe_grouped(pact, T, F, kk, true, plan, E, H, Lw.edown.w, Lw.edown.s,
                                 Lw.edown.b, nullptr, nullptr, nullptr, py, st, e_lo, e_n));
      if (tp) {
        HG_CUDA(launch_moe_combine_partial(py, sc, idx, T, kk, H, e_lo, e_n, part, st));
        HG_CUDA(comm_allreduce_residual(m->comm, 2 * li + 1, part, T * H, h, st));
      } else {
        HG_CUDA(launch_moe_combine(py, sc, T, kk, H, h, st));
      }
      continue;
    }
    {
      if (!fuse) {
        rc = higgs_rmsnorm(m->ctx, h, nullptr, T, H, Lw.ln_post, c.rms_eps, x, nullptr, st);
        if (rc) return rc;
      }
      QLinArgs a{};
      a.x = fuse ? h : x;
      a.norm_w = fuse ? Lw.ln_post : nullptr;
      if (tpf) set_pull(a);
      a.eps = c.rms_eps;
      a.M = T;
      a.K = H;
      a.N = c.intermediate;
      a.w = Lw.gate.w;
      a.s = Lw.gate.s;
      a.b = Lw.gate.b;
      a.w2 = Lw.up.w;
      a.s2 = Lw.up.s;
      a.b2 = Lw.up.b;
      a.nseg = 1;
      a.y = act;
      a.self_prefetch = pfself;
      a.tc_ws = tc_ws;
      a.tc_ws_bytes = L.tc_ws_bytes;
      if (li + 1 < n_layers) {
        const LayerW& Ln = m->layers[li + 1];
        add_q(a.pf, Ln.q);
        add_q(a.pf, Ln.k);
        add_q(a.pf, Ln.v);
      } else {
        add_q(a.pf, m->head, (size_t)48 << 20);  // the head's leading 48 MB
      }
      HG_CUDA(launch_qgemv_ring(a, EPI_SWIGLU, st));
      after_pull(a);
    }
    if (tpf) {
      if ((rc = push_row_parallel(Lw.down, act, 2 * li + 1))) return rc;
    } else if ((rc = row_parallel(Lw.down, act, 2 * li + 1, nullptr))) {
      return rc;
    }
  }
  // final norm (+ last-token selection) and LM head
  const int rows_lm = f->last_only ? B : T;
  if (fuse && (Lq == 1 || !f->last_only) && !f->hidden_out) {
    if ((f->logits || f->argmax) && !head_done) {
      if (pull_call >= 0) {  // the final norm pulls the last layer's sum over ranks
        QLinArgs a{};
        a.norm_w = m->final_norm;
        set_pull(a);
        a.eps = c.rms_eps;
        a.M = T;
        a.K = H;
        a.N = m->head.N;
        a.w = m->head.w;
        a.s = m->head.s;
        a.b = m->head.b;
        a.nseg = 1;
        a.y_f32 = logits;
        HG_CUDA(launch_qgemv_ring(a, EPI_STORE, st));
        after_pull(a);
      } else {
        HG_CUDA(lin(m->head, h, m->final_norm, nullptr, logits, nullptr));
      }
    }
    if (f->argmax) {
      rc = emit_argmax(logits, rows_lm);
      if (rc) return rc;
    }
    return HIGGS_OK;
  }
  if (f->last_only) {
    rc = higgs_rmsnorm_strided(m->ctx, h + (size_t)(Lq - 1) * H, (int64_t)Lq * H, B, H,
                               m->final_norm, c.rms_eps, xl, st);
  } else {
    rc = higgs_rmsnorm(m->ctx, h, nullptr, T, H, m->final_norm, c.rms_eps, xl, nullptr, st);
  }
  if (rc) return rc;
  if (f->logits || f->argmax) {
    QLinArgs a{};
    a.x = xl;
    a.M = rows_lm;
    a.K = H;
    a.N = m->head.N;
    a.w = m->head.w;
    a.s = m->head.s;
    a.b = m->head.b;
    a.nseg = 1;
    a.y_f32 = logits;
    a.self_prefetch = pfself;
    a.tc_ws = tc_ws;
    a.tc_ws_bytes = L.tc_ws_bytes;
    HG_CUDA(launch_qgemv_ring(a, EPI_STORE, st));
  }
  if (f->argmax) {
    rc = emit_argmax(logits, rows_lm);
    if (rc) return rc;
  }
  if (f->hidden_out) {
    HG_CUDA(cudaMemcpyAsync(f->hidden_out, xl, (size_t)rows_lm * H * 2, cudaMemcpyDeviceToDevice, st));
  }
  return HIGGS_OK;
}

int validate_forward(higgs_model* m, const higgs_forward_args* f) {
  HG_CHECK_ARG(m && f, "higgs_model_forward: null argument");
  if (!m->finalized) return fail(HIGGS_ERR_STATE, "higgs_model_forward: call higgs_model_finalize first");
  if (!m->k_pool || !m->v_pool) return fail(HIGGS_ERR_STATE, "higgs_model_forward: no KV cache set");
  HG_CHECK_ARG(f->B > 0 && f->Lq > 0, "higgs_model_forward: B and Lq must be positive");
  HG_CHECK_ARG(f->tokens && f->positions && f->slot_mapping && f->block_table && f->seq_lens,
               "higgs_model_forward: null input vector");
  HG_CHECK_ARG(f->n_layers >= 0 && f->n_layers <= m->cfg.layers, "higgs_model_forward: bad n_layers");
  HG_CHECK_ARG(f->max_seq_len >= f->Lq && (int64_t)f->max_blocks * HIGGS_PAGE_SIZE >= f->max_seq_len,
               "higgs_model_forward: max_seq_len / max_blocks inconsistent");
  HG_CHECK_ARG(f->workspace, "higgs_model_forward: null workspace");
  if (m->cfg.tp_world > 1 && !m->comm)
    return fail(HIGGS_ERR_STATE, "higgs_model_forward: tensor-parallel shard without a communicator");
  HG_CHECK_ARG(m->cfg.num_experts == 0 || (int64_t)f->B * f->Lq * m->cfg.experts_per_tok <= 65536,
               "higgs_model_forward: MoE routes at most 65536 (token, expert) pairs per call");
  return HIGGS_OK;
}

}  // namespace

extern "C" int higgs_model_create(higgs_ctx* ctx, const higgs_model_config* cfg, higgs_model** out) {
  HG_CHECK_ARG(ctx && cfg && out, "higgs_model_create: null argument");
  HG_DEVICE(ctx);
  *out = nullptr;
  const higgs_model_config& c = *cfg;
  HG_CHECK_ARG(c.hidden > 0 && c.hidden % 256 == 0, "higgs_model_create: hidden must be a multiple of 256");
  HG_CHECK_ARG(c.layers > 0 && c.heads > 0 && c.kv_heads > 0 && c.heads % c.kv_heads == 0,
               "higgs_model_create: bad layer / head counts");
  HG_CHECK_ARG(c.head_dim == 64 || c.head_dim == 128, "higgs_model_create: head_dim must be 64 or 128");
  HG_CHECK_ARG(c.intermediate > 0 && c.intermediate % 256 == 0,
               "higgs_model_create: intermediate must be a multiple of 256");
  HG_CHECK_ARG(c.vocab > 0 && c.vocab % 16 == 0, "higgs_model_create: vocab must be a multiple of 16");
  HG_CHECK_ARG((c.heads * c.head_dim) % 256 == 0, "higgs_model_create: heads*head_dim must be a multiple of 256");
  HG_CHECK_ARG(c.kv_mode == HIGGS_KV_BF16 || (c.kv_mode == HIGGS_KV_TQ4 && c.head_dim == 128),
               "higgs_model_create: TurboQuant KV needs head_dim 128");
  if (c.tp_world > 1) {
    HG_CHECK_ARG(c.tp_world <= kMaxRanks && c.tp_rank >= 0 && c.tp_rank < c.tp_world,
                 "higgs_model_create: bad tp_rank / tp_world (tp_world <= 8)");
    HG_CHECK_ARG(c.head_rows > 0 && c.head_rows % 16 == 0 && (int64_t)c.head_rows * c.tp_world == c.vocab,
                 "higgs_model_create: head_rows * tp_world must equal vocab (head_rows % 16 == 0)");
    HG_CHECK_ARG(c.num_experts % c.tp_world == 0,
                 "higgs_model_create: expert parallelism needs num_experts % tp_world == 0");
  }
  if (c.num_experts > 0) {
    HG_CHECK_ARG(c.num_experts <= 1024 && c.num_experts % 16 == 0,
                 "higgs_model_create: num_experts must be a multiple of 16, at most 1024");
    HG_CHECK_ARG(c.experts_per_tok > 0 && c.experts_per_tok <= 32 && c.experts_per_tok <= c.num_experts,
                 "higgs_model_create: experts_per_tok must be in [1, min(32, num_experts)]");
    HG_CHECK_ARG(c.moe_intermediate > 0 && c.moe_intermediate % 256 == 0,
                 "higgs_model_create: moe_intermediate must be a multiple of 256");
    HG_CHECK_ARG(qgemv_grouped_supported(c.hidden) && qgemv_grouped_supported(c.moe_intermediate),
                 "higgs_model_create: hidden / moe_intermediate too large for the grouped experts");
  } else {
    HG_CHECK_ARG(c.num_experts == 0, "higgs_model_create: negative num_experts");
  }
  higgs_model* m = new higgs_model;
  m->ctx = ctx;
  m->cfg = c;
  *out = m;
  return HIGGS_OK;
}

extern "C" int higgs_model_destroy(higgs_model* m) {
  if (!m) return HIGGS_OK;
  DeviceGuard guard;
  guard.enter(m->ctx->device);
  if (m->inv_freq) cudaFree(m->inv_freq);
  delete m;
  return HIGGS_OK;
}

extern "C" int higgs_model_set_tensor(higgs_model* m, const char* name, const void* ptr, int dtype,
                                      const int64_t* shape, int ndim) {
  HG_CHECK_ARG(m && name && ptr && (ndim == 0 || shape) && ndim >= 0 && ndim <= 4,
               "higgs_model_set_tensor: bad argument");
  HG_CHECK_ARG(dtype == HIGGS_DTYPE_U32 || dtype == HIGGS_DTYPE_BF16 || dtype == HIGGS_DTYPE_F32,
               "higgs_model_set_tensor: unknown dtype");
  HG_DEVICE(m->ctx);
  TensorRef t;
  t.ptr = ptr;
  t.dtype = dtype;
  t.shape.assign(shape, shape + ndim);
  m->tensors[name] = t;
  m->finalized = false;
  return HIGGS_OK;
}

extern "C" int higgs_model_finalize(higgs_model* m) {
  HG_CHECK_ARG(m, "higgs_model_finalize: null model");
  HG_DEVICE(m->ctx);
  const higgs_model_config& c = m->cfg;
  const int H = c.hidden, D = c.head_dim;
  int rc = get_q(m, "model.embed_tokens", c.vocab, H, m->embed);
  if (rc) return rc;
  if (c.tie_word_embeddings) {
    m->head = m->embed;
    if (c.tp_world > 1) {  // this rank's rows of the tied table
      const size_t r0 = (size_t)c.tp_rank * c.head_rows;
      m->head.w += r0 * (H / 8);
      m->head.s += r0 * (H / 64);
      m->head.b += r0 * (H / 64);
      m->head.N = c.head_rows;
    }
  } else {
    rc = get_q(m, "lm_head", head_rows(c), H, m->head);
    if (rc) return rc;
  }
  rc = get_vec(m, "model.norm.weight", H, m->final_norm);
  if (rc) return rc;
  m->layers.assign(c.layers, LayerW{});
  for (int i = 0; i < c.layers; ++i) {
    const std::string p = "model.layers." + std::to_string(i) + ".";
    LayerW& L = m->layers[i];
    if ((rc = get_vec(m, p + "input_layernorm.weight", H, L.ln_in))) return rc;
    if ((rc = get_vec(m, p + "post_attention_layernorm.weight", H, L.ln_post))) return rc;
    if ((rc = get_q(m, p + "self_attn.q_proj", c.heads * D, H, L.q))) return rc;
    if ((rc = get_q(m, p + "self_attn.k_proj", c.kv_heads * D, H, L.k))) return rc;
    if ((rc = get_q(m, p + "self_attn.v_proj", c.kv_heads * D, H, L.v))) return rc;
    if ((rc = get_q(m, p + "self_attn.o_proj", H, c.heads * D, L.o))) return rc;
    if (c.qk_norm) {
      if ((rc = get_vec(m, p + "self_attn.q_norm.weight", D, L.qn))) return rc;
      if ((rc = get_vec(m, p + "self_attn.k_norm.weight", D, L.kn))) return rc;
    }
    L.moe = c.num_experts > 0 && m->tensors.count(p + "mlp.gate.weight");
    if (L.moe) {
      const int E = c.num_experts, F = c.moe_intermediate;
      const int El = c.tp_world > 1 ? E / c.tp_world : E;  // experts held by this rank
      const std::string sw = p + "mlp.switch_mlp.";
      if ((rc = get_q(m, p + "mlp.gate", E, H, L.router))) return rc;
      if ((rc = get_q3(m, sw + "gate_proj", El, F, H, L.egate))) return rc;
      if ((rc = get_q3(m, sw + "up_proj", El, F, H, L.eup))) return rc;
      if ((rc = get_q3(m, sw + "down_proj", El, H, F, L.edown))) return rc;
      continue;
    }
    if ((rc = get_q(m, p + "mlp.gate_proj", c.intermediate, H, L.gate))) return rc;
    if ((rc = get_q(m, p + "mlp.up_proj", c.intermediate, H, L.up))) return rc;
    if ((rc = get_q(m, p + "mlp.down_proj", H, c.intermediate, L.down))) return rc;
  }
  if (!m->inv_freq) {
    std::vector<float> f(D / 2);
    for (int i = 0; i < D / 2; ++i) f[i] = (float)std::pow((double)c.rope_theta, -(2.0 * i) / D);
    HG_CUDA(cudaMalloc(&m->inv_freq, f.size() * sizeof(float)));
    HG_CUDA(cudaMemcpy(m->inv_freq, f.data(), f.size() * sizeof(float), cudaMemcpyHostToDevice));
  }
  HG_CUDA(attention_prepare());
  m->finalized = true;
  return HIGGS_OK;
}

extern "C" int higgs_model_set_comm(higgs_model* m, higgs_comm* comm) {
  HG_CHECK_ARG(m && comm, "higgs_model_set_comm: null argument");
  HG_CHECK_ARG(m->cfg.tp_world > 1, "higgs_model_set_comm: the model is not a tensor-parallel shard");
  HG_DEVICE(m->ctx);
  m->comm = comm;
  return HIGGS_OK;
}

extern "C" int higgs_model_set_kv_cache(higgs_model* m, void* k_pool, void* v_pool,
                                        int64_t num_pages) {
  HG_CHECK_ARG(m && k_pool && v_pool && num_pages > 0, "higgs_model_set_kv_cache: bad argument");
  HG_CHECK_ARG(m->cfg.kv_mode == HIGGS_KV_BF16, "higgs_model_set_kv_cache: model uses TurboQuant KV");
  HG_DEVICE(m->ctx);
  m->k_pool = k_pool;
  m->v_pool = v_pool;
  m->num_pages = num_pages;
  return HIGGS_OK;
}

extern "C" int higgs_model_set_kv_cache_tq4(higgs_model* m, uint8_t* k_codes, void* k_scales,
                                            uint8_t* v_codes, void* v_scales, int64_t num_pages,
                                            const int8_t* signs) {
  HG_CHECK_ARG(m && k_codes && k_scales && v_codes && v_scales && signs && num_pages > 0,
               "higgs_model_set_kv_cache_tq4: bad argument");
  HG_CHECK_ARG(m->cfg.kv_mode == HIGGS_KV_TQ4, "higgs_model_set_kv_cache_tq4: model uses bf16 KV");
  HG_DEVICE(m->ctx);
  m->k_pool = k_codes;
  m->v_pool = v_codes;
  m->k_scales = k_scales;
  m->v_scales = v_scales;
  m->signs = signs;
  m->num_pages = num_pages;
  return HIGGS_OK;
}

extern "C" size_t higgs_model_workspace_size(const higgs_model* m, int B, int Lq, int max_seq_len,
                                             int last_only) {
  if (!m || B <= 0 || Lq <= 0) return 0;
  return layout(m->cfg, B, Lq, max_seq_len, last_only != 0).total;
}

extern "C" int higgs_model_forward(higgs_model* m, const higgs_forward_args* f, void* stream) {
  int rc = validate_forward(m, f);
  if (rc) return rc;
  HG_DEVICE(m->ctx);
  return forward_impl(m, f, (cudaStream_t)stream);
}

extern "C" int higgs_model_capture(higgs_model* m, const higgs_forward_args* f, void* stream,
                                   higgs_graph** out) {
  HG_CHECK_ARG(m && out && stream, "higgs_model_capture: needs a model, a non-default stream and an out pointer");
  HG_DEVICE(m->ctx);
  *out = nullptr;
  int rc = validate_forward(m, f);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  HG_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
  rc = forward_impl(m, f, st);
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamEndCapture(st, &graph);
  if (rc) {
    if (graph) cudaGraphDestroy(graph);
    return rc;
  }
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
  size_t n_nodes = 0;
  int kernels = 0;
  if (cudaGraphGetNodes(graph, nullptr, &n_nodes) == cudaSuccess && n_nodes > 0) {
    std::vector<cudaGraphNode_t> nodes(n_nodes);
    if (cudaGraphGetNodes(graph, nodes.data(), &n_nodes) == cudaSuccess)
      for (size_t i = 0; i < n_nodes; ++i) {
        cudaGraphNodeType ty;
        if (cudaGraphNodeGetType(nodes[i], &ty) == cudaSuccess && ty == cudaGraphNodeTypeKernel) ++kernels;
      }
  }
  cudaGraphExec_t exec = nullptr;
  e = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGraphInstantiate");
  higgs_graph* g = new higgs_graph;
  g->device = m->ctx->device;
  g->exec = exec;
  g->kernel_nodes = kernels;
  *out = g;
  return HIGGS_OK;
}

extern "C" int higgs_graph_launch(higgs_graph* g, void* stream) {
  HG_CHECK_ARG(g && g->exec, "higgs_graph_launch: null graph");
  HG_DEVICE(g);
  HG_CUDA(cudaGraphLaunch(g->exec, (cudaStream_t)stream));
  return HIGGS_OK;
}

extern "C" int higgs_graph_num_kernels(const higgs_graph* g) { return g ? g->kernel_nodes : -1; }

extern "C" int higgs_graph_destroy(higgs_graph* g) {
  if (!g) return HIGGS_OK;
  DeviceGuard guard;
  guard.enter(g->device);
  if (g->exec) cudaGraphExecDestroy(g->exec);
  delete g;
  return HIGGS_OK;
}
