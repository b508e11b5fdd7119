"""Torch-facing wrappers of the C ABI, named after the mlx-rs ops they replace.

Every function takes CUDA tensors, enqueues on torch's current stream and
returns new tensors (or fills ``out``).  bf16 activations, u32 packed weights
and bf16 scales/biases follow the MLX affine layout (see include/higgs_cuda.h).
Reference call sites are cited per function.
"""
from __future__ import annotations

import math

import torch

from . import ffi

PAGE = 16


def _p(t):
    return None if t is None else t.data_ptr()


def _st(dev: torch.device):
    return torch.cuda.current_stream(dev).cuda_stream


def _ctx(t: torch.Tensor) -> int:
    if not t.is_cuda:
        raise ValueError("higgs ops take CUDA tensors (there is no CPU fallback)")
    return ffi.ctx(t.device.index)


def _chk(t: torch.Tensor, dtype, name: str):
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


# ---- a1/a2 ----------------------------------------------------------------

def quantized_matmul(x, w, scales, biases, transpose: bool = True, group_size: int = 64,
                     bits: int = 4, *, residual=None, out_f32: bool = False):
    """ops::quantized_matmul (qwen3_next.rs:174-183): y = x . dequant(w)^T.

    x bf16 [..., K]; w u32 [N, K/8]; scales/biases bf16 [N, K/64].
    Returns bf16 [..., N] (f32 when out_f32).  ``residual`` (bf16 [..., N])
    is added after rounding the product to bf16 (TransformerBlock residual).
    """
    if not transpose or group_size != 64 or bits != 4:
        raise NotImplementedError("only transpose=True, group_size=64, bits=4 (MLX affine W4 g64)")
    _chk(x, torch.bfloat16, "x")
    K = x.shape[-1]
    N = w.shape[0]
    if w.shape[1] * 8 != K:
        raise ValueError(f"w has {w.shape[1] * 8} inputs, x has {K}")
    M = x.numel() // K
    y = torch.empty(*x.shape[:-1], N, dtype=torch.float32 if out_f32 else torch.bfloat16,
                    device=x.device)
    ffi.call("higgs_qlinear_w4g64", _ctx(x), _p(x), M, K, _p(w), _p(scales), _p(biases), N,
             None if out_f32 else _p(y), _p(y) if out_f32 else None, _p(residual), _st(x.device))
    return y


def gate_up_swiglu(x, wg, sg, bg, wu, su, bu):
    """swiglu(gate_proj(x), up_proj(x)) fused (transformer.rs:349-353, qwen3_next.rs:275-277)."""
    _chk(x, torch.bfloat16, "x")
    K = x.shape[-1]
    N = wg.shape[0]
    M = x.numel() // K
    y = torch.empty(*x.shape[:-1], N, dtype=torch.bfloat16, device=x.device)
    ffi.call("higgs_qlinear_gate_up_swiglu", _ctx(x), _p(x), M, K, _p(wg), _p(sg), _p(bg),
             _p(wu), _p(su), _p(bu), N, _p(y), _st(x.device))
    return y


def chain_gemv(x, w, scales, biases, *, norm_w=None, up=None, segments=None, y=None, y_f32=None,
               residual=None) -> "ffi.ChainGemv":
    """One phase of decode_chain: y = quantized_matmul(norm(x), w) at one token.  up = (w2, s2,
    b2) makes it a SwiGLU phase; segments = [(w, s, b), ...] (q|k|v) replaces w/scales/biases."""
    c = ffi.ChainGemv()
    segs = segments or [(w, scales, biases)]
    c.x, c.norm_w = _p(x), _p(norm_w)
    c.K = x.shape[-1]
    c.N = sum(t[0].shape[0] for t in segs)
    c.swiglu, c.nseg = int(up is not None), len(segs)
    end = 0
    for i, (wi, si, bi) in enumerate(segs):
        end += wi.shape[0]
        c.seg_end[i] = end
        c.w[i], c.s[i], c.b[i] = _p(wi), _p(si), _p(bi)
    if up is not None:
        c.w2, c.s2, c.b2 = _p(up[0]), _p(up[1]), _p(up[2])
    c.y, c.y_f32, c.residual = _p(y), _p(y_f32), _p(residual)
    return c


def decode_chain(phases, eps: float, barriers, device):
    """higgs_decode_chain: the phases (chain_gemv) in one persistent launch; barriers is a zeroed
    int32 tensor of at least 64 * len(phases) entries (left zeroed)."""
    arr = (ffi.ChainGemv * len(phases))(*phases)
    ffi.call("higgs_decode_chain", ffi.ctx(torch.device(device).index or 0), arr, len(phases),
             float(eps), _p(barriers), _st(torch.device(device)))


def sk_workspace(M: int, K: int, rows: int, device) -> torch.Tensor:
    n = ffi.load().higgs_qlinear_sk_workspace_size(M, K, rows)
    return torch.zeros(n, dtype=torch.uint8, device=device)


def rmsnorm_quantized_matmul(h, norm_w, eps, w, scales, biases, *, residual=None,
                             out_f32: bool = False, workspace=None):
    """nn::RmsNorm (norm_w, or none when norm_w is None) then quantized_matmul.

    M <= 8 with or without the norm (stream-K GEMV); any M without it (from 17 rows the
    tensor-core matmul, which splits K over the workspace when its tiles are few)."""
    _chk(h, torch.bfloat16, "h")
    K = h.shape[-1]
    M = h.numel() // K
    N = w.shape[0]
    if workspace is None:
        workspace = sk_workspace(M, K, N, h.device)
    y = torch.empty(*h.shape[:-1], N, dtype=torch.float32 if out_f32 else torch.bfloat16,
                    device=h.device)
    ffi.call("higgs_rmsnorm_qlinear_w4g64", _ctx(h), _p(h), M, K, _p(norm_w), float(eps), _p(w),
             _p(scales), _p(biases), N, None if out_f32 else _p(y), _p(y) if out_f32 else None,
             _p(residual), _p(workspace), workspace.numel(), _st(h.device))
    return y


def rmsnorm_gate_up_swiglu(h, norm_w, eps, wg, sg, bg, wu, su, bu, workspace=None):
    """nn::RmsNorm (or none when norm_w is None) then swiglu(gate_proj, up_proj); M <= 8
    with the norm, any M without it."""
    _chk(h, torch.bfloat16, "h")
    K = h.shape[-1]
    M = h.numel() // K
    N = wg.shape[0]
    if workspace is None:
        workspace = sk_workspace(M, K, 2 * N, h.device)
    y = torch.empty(*h.shape[:-1], N, dtype=torch.bfloat16, device=h.device)
    ffi.call("higgs_rmsnorm_gate_up_swiglu", _ctx(h), _p(h), M, K, _p(norm_w), float(eps), _p(wg),
             _p(sg), _p(bg), _p(wu), _p(su), _p(bu), N, _p(y), _p(workspace), workspace.numel(),
             _st(h.device))
    return y


def dequantize(w, scales, biases, group_size: int = 64, bits: int = 4):
    """ops::dequantize (qwen3_next.rs:249-256): bf16 [N, K]."""
    if group_size != 64 or bits != 4:
        raise NotImplementedError("only group_size=64, bits=4")
    N, K = w.shape[0], w.shape[1] * 8
    out = torch.empty(N, K, dtype=torch.bfloat16, device=w.device)
    ffi.call("higgs_w4_dequantize", _ctx(w), _p(w), _p(scales), _p(biases), N, K, _p(out),
             _st(w.device))
    return out


def quantize(w, group_size: int = 64, bits: int = 4):
    """ops::quantize with this library's rounding: f32 [N, K] -> (u32-as-int32 [N, K/8], bf16 s, b)."""
    if group_size != 64 or bits != 4:
        raise NotImplementedError("only group_size=64, bits=4")
    _chk(w, torch.float32, "w")
    N, K = w.shape
    q = torch.empty(N, K // 8, dtype=torch.int32, device=w.device)
    s = torch.empty(N, K // 64, dtype=torch.bfloat16, device=w.device)
    b = torch.empty(N, K // 64, dtype=torch.bfloat16, device=w.device)
    ffi.call("higgs_w4_quantize", _ctx(w), _p(w), N, K, _p(q), _p(s), _p(b), _st(w.device))
    return q, s, b


def embed_gather(ids, w, scales, biases):
    """QEmbedding::forward (qwen3_next.rs:248-257): bf16 [*ids.shape, H]."""
    _chk(ids, torch.int32, "ids")
    V, H = w.shape[0], w.shape[1] * 8
    out = torch.empty(*ids.shape, H, dtype=torch.bfloat16, device=ids.device)
    ffi.call("higgs_embed_gather_w4", _ctx(ids), _p(ids), ids.numel(), _p(w), _p(scales),
             _p(biases), V, H, _p(out), _st(ids.device))
    return out


# ---- a3/a4 ------------------------------------------------------------------

def rms_norm(x, weight, eps: float, residual=None, want_h: bool = False):
    """fast::rms_norm (transformer.rs:375-377): returns y, or (y, h) with h = x + residual."""
    _chk(x, torch.bfloat16, "x")
    H = x.shape[-1]
    rows = x.numel() // H
    y = torch.empty_like(x)
    h = torch.empty_like(x) if (residual is not None and want_h) else None
    ffi.call("higgs_rmsnorm", _ctx(x), _p(x), _p(residual), rows, H, _p(weight), float(eps),
             _p(y), _p(h), _st(x.device))
    return (y, h) if want_h else y


def rope_inv_freq(dims: int, base: float, device=None) -> torch.Tensor:
    """inv_freq[i] = base^(-2i/dims), computed in f64 and rounded to f32."""
    f = [base ** (-(2.0 * i) / dims) for i in range(dims // 2)]
    return torch.tensor(f, dtype=torch.float32, device=device)


def rope(x, positions, inv_freq):
    """fast::rope(traditional=false, scale=1) (utils.rs:16-26); x bf16 [rows, heads, D]."""
    _chk(x, torch.bfloat16, "x")
    rows, heads, D = x.shape
    y = torch.empty_like(x)
    ffi.call("higgs_rope", _ctx(x), _p(x), rows, heads, D, _p(positions), _p(inv_freq), _p(y),
             _st(x.device))
    return y


def qknorm_rope_kv_write(qkv, Hq: int, Hkv: int, D: int, q_norm_w, k_norm_w, eps: float,
                         positions, inv_freq, slot_mapping, k_cache, v_cache, page_stride=None,
                         head_stride=None):
    """Attention front half + cache append (transformer.rs:246-289, cache.rs:236-311).

    Caches are [num_pages, Hkv, 16, D] bf16 unless strides are given.  Returns q bf16 [T, Hq, D].
    """
    T = qkv.shape[0]
    if page_stride is None:
        page_stride = Hkv * PAGE * D
    if head_stride is None:
        head_stride = PAGE * D
    q = torch.empty(T, Hq, D, dtype=torch.bfloat16, device=qkv.device)
    ffi.call("higgs_qknorm_rope_kv_write", _ctx(qkv), _p(qkv), T, Hq, Hkv, D, _p(q_norm_w),
             _p(k_norm_w), float(eps), _p(positions), _p(inv_freq), _p(slot_mapping), _p(k_cache),
             _p(v_cache), int(page_stride), int(head_stride), _p(q), _st(qkv.device))
    return q


# ---- a6/a13/a14 -------------------------------------------------------------

def attention_workspace(B, Lq, Hq, Hkv, D, max_seq_len, device) -> torch.Tensor:
    n = ffi.load().higgs_paged_attention_workspace_size(B, Lq, Hq, Hkv, D, max_seq_len)
    return torch.zeros(max(n, 4096), dtype=torch.uint8, device=device)


def paged_attention(q, k_cache, v_cache, block_table, seq_lens, max_seq_len: int, scale=None,
                    page_stride=None, head_stride=None, workspace=None):
    """fast::scaled_dot_product_attention over a paged cache (utils.rs:45-60, masks 64-125).

    q bf16 [B, Lq, Hq, D]; caches [num_pages, Hkv, 16, D] (or explicit strides);
    block_table int32 [B, max_blocks]; seq_lens int32 [B].
    """
    B, Lq, Hq, D = q.shape
    Hkv = k_cache.shape[1] if head_stride is None else None
    if Hkv is None:
        raise ValueError("give Hkv through the cache shape")
    if page_stride is None:
        page_stride = Hkv * PAGE * D
    if head_stride is None:
        head_stride = PAGE * D
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if workspace is None:
        workspace = attention_workspace(B, Lq, Hq, Hkv, D, max_seq_len, q.device)
    out = torch.empty_like(q)
    ffi.call("higgs_paged_attention", _ctx(q), _p(q), B, Lq, Hq, Hkv, D, _p(k_cache),
             _p(v_cache), int(page_stride), int(head_stride), _p(block_table),
             block_table.shape[1], _p(seq_lens), int(max_seq_len), float(scale), _p(out),
             _p(workspace), workspace.numel(), _st(q.device))
    return out


def fused_attention(qkv, Hq: int, Hkv: int, D: int, q_norm_w, k_norm_w, eps: float, positions,
                    inv_freq, slot_mapping, k_cache, v_cache, block_table, seq_lens,
                    max_seq_len: int, Lq: int = 1, scale=None, workspace=None):
    """Attention::forward from q|k|v to the output (transformer.rs:246-294) in one kernel:
    q/k norm, RoPE, cache append at slot_mapping, paged SDPA.  qkv bf16 [B*Lq, (Hq+2Hkv)*D]."""
    T = qkv.shape[0]
    B = T // Lq
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if workspace is None:
        n = ffi.load().higgs_fused_attention_workspace_size(B, Lq, Hq, Hkv, D, max_seq_len)
        workspace = torch.zeros(max(n, 4096), dtype=torch.uint8, device=qkv.device)
    out = torch.empty(B, Lq, Hq, D, dtype=torch.bfloat16, device=qkv.device)
    ffi.call("higgs_fused_attention", _ctx(qkv), _p(qkv), B, Lq, Hq, Hkv, D, _p(q_norm_w),
             _p(k_norm_w), float(eps), _p(positions), _p(inv_freq), _p(slot_mapping), _p(k_cache),
             _p(v_cache), Hkv * PAGE * D, PAGE * D, _p(block_table), block_table.shape[1],
             _p(seq_lens), int(max_seq_len), float(scale), _p(out), _p(workspace),
             workspace.numel(), _st(qkv.device))
    return out


def tq4_encode(x, signs):
    """TurboQuant encode of bf16 [n, 128] -> (codes u8 [n, 64], scales fp16 [n])."""
    n = x.numel() // 128
    codes = torch.empty(n, 64, dtype=torch.uint8, device=x.device)
    scales = torch.empty(n, dtype=torch.float16, device=x.device)
    ffi.call("higgs_tq4_encode", _ctx(x), _p(x), n, _p(signs), _p(codes), _p(scales),
             _st(x.device))
    return codes, scales


def qknorm_rope_kv_write_tq4(qkv, Hq: int, Hkv: int, q_norm_w, k_norm_w, eps: float, positions,
                             inv_freq, slot_mapping, signs, k_codes, k_scales, v_codes, v_scales):
    """As qknorm_rope_kv_write, storing TurboQuant codes [pages, Hkv, 16, 64] + fp16 scales."""
    T = qkv.shape[0]
    q = torch.empty(T, Hq, 128, dtype=torch.bfloat16, device=qkv.device)
    ffi.call("higgs_qknorm_rope_kv_write_tq4", _ctx(qkv), _p(qkv), T, Hq, Hkv, _p(q_norm_w),
             _p(k_norm_w), float(eps), _p(positions), _p(inv_freq), _p(slot_mapping), _p(signs),
             _p(k_codes), _p(k_scales), _p(v_codes), _p(v_scales), Hkv * PAGE * 64, PAGE * 64,
             _p(q), _st(qkv.device))
    return q


def paged_attention_tq4(q, k_codes, k_scales, v_codes, v_scales, block_table, seq_lens,
                        max_seq_len: int, signs, scale=None, workspace=None):
    """Decode attention over TurboQuant pages [num_pages, Hkv, 16, 64] (+ fp16 scales)."""
    B, Lq, Hq, D = q.shape
    assert D == 128
    Hkv = k_codes.shape[1]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if workspace is None:
        workspace = attention_workspace(B, Lq, Hq, Hkv, 128, max_seq_len, q.device)
    out = torch.empty_like(q)
    ffi.call("higgs_paged_attention_tq4", _ctx(q), _p(q), B, Lq, Hq, Hkv, _p(k_codes),
             _p(k_scales), _p(v_codes), _p(v_scales), Hkv * PAGE * 64, PAGE * 64,
             _p(block_table), block_table.shape[1], _p(seq_lens), int(max_seq_len), _p(signs),
             float(scale), _p(out), _p(workspace), workspace.numel(), _st(q.device))
    return out


# ---- a10/a15 ----------------------------------------------------------------

def argmax(logits):
    """sample() at T=0 (lib.rs:373-377); logits f32 [B, V] -> int32 [B], ties -> first."""
    _chk(logits, torch.float32, "logits")
    B, V = logits.shape
    out = torch.empty(B, dtype=torch.int32, device=logits.device)
    ffi.call("higgs_argmax", _ctx(logits), _p(logits), B, V, _p(out), _st(logits.device))
    return out


def sample(logits, temperature: float, uniforms=None):
    """sample() (lib.rs:373-385) with explicit uniforms [B] for T > 0."""
    _chk(logits, torch.float32, "logits")
    B, V = logits.shape
    out = torch.empty(B, dtype=torch.int32, device=logits.device)
    ffi.call("higgs_sample", _ctx(logits), _p(logits), B, V, float(temperature), _p(uniforms),
             _p(out), _st(logits.device))
    return out


def sample_filtered(logits, temperature: float, top_k: int = 0, top_p: float = 1.0,
                    min_p: float = 0.0, uniforms=None):
    """sample() with sample_filtered's top-k / top-p / min-p (lib.rs:373-460), explicit
    uniforms [B] for T > 0; int32 [B]."""
    _chk(logits, torch.float32, "logits")
    B, V = logits.shape
    out = torch.empty(B, dtype=torch.int32, device=logits.device)
    ffi.call("higgs_sample_filtered", _ctx(logits), _p(logits), B, V, float(temperature),
             int(top_k), float(top_p), float(min_p), _p(uniforms), _p(out), _st(logits.device))
    return out


def logprobs(logits, temperature: float, tokens, top_n: int = 0):
    """LogprobArrays::compute (lib.rs:495-533): (token logprob f32 [B], top ids int32 [B, n],
    top logprobs f32 [B, n])."""
    _chk(logits, torch.float32, "logits")
    B, V = logits.shape
    dev = logits.device
    lp = torch.empty(B, dtype=torch.float32, device=dev)
    ids = torch.empty(B, top_n, dtype=torch.int32, device=dev)
    tl = torch.empty(B, top_n, dtype=torch.float32, device=dev)
    ffi.call("higgs_logprobs", _ctx(logits), _p(logits), B, V, float(temperature), _p(tokens),
             int(top_n), _p(lp), _p(ids) if top_n else None, _p(tl) if top_n else None, _st(dev))
    return lp, ids, tl


def apply_token_mask(logits, allowed_bits):
    """Constraint::apply_mask (constrained.rs:79-110) in place: f32 [B, V] += 0 / -inf from an
    int32 bitmask [B, ceil(V/32)] (bit j%32 of word j/32 = token j allowed)."""
    _chk(logits, torch.float32, "logits")
    B, V = logits.shape
    ffi.call("higgs_apply_token_mask", _ctx(logits), _p(logits), B, V, _p(allowed_bits),
             allowed_bits.shape[1], _st(logits.device))
    return logits


def spec_accept(target_logits, draft_logits, draft_tokens, temperature: float,
                accept_uniforms=None, sample_uniforms=None):
    """Speculative acceptance: (accepted int32 [B], out_tokens int32 [B, k+1])."""
    B, k1, V = target_logits.shape
    k = k1 - 1
    acc = torch.empty(B, dtype=torch.int32, device=target_logits.device)
    toks = torch.empty(B, k1, dtype=torch.int32, device=target_logits.device)
    ffi.call("higgs_spec_accept", _ctx(target_logits), _p(target_logits), _p(draft_logits),
             _p(draft_tokens), B, k, V, float(temperature), _p(accept_uniforms),
             _p(sample_uniforms), _p(acc), _p(toks), _st(target_logits.device))
    return acc, toks


def apply_penalties(logits, history, hist_lens, rep: float = 1.0, freq: float = 0.0,
                    pres: float = 0.0):
    """apply_penalties (lib.rs:278-363), in place on f32 [B, V]."""
    B, V = logits.shape
    ffi.call("higgs_apply_penalties", _ctx(logits), _p(logits), B, V, _p(history), _p(hist_lens),
             history.shape[1], float(rep), float(freq), float(pres), _st(logits.device))
    return logits


# ---- a9: mixture of experts ------------------------------------------------------------------

def moe_plan(T: int, E: int, k: int, device) -> torch.Tensor:
    """Buffer for the routing plan of T tokens, E experts, top-k (higgs_moe_plan_size)."""
    n = ffi.load().higgs_moe_plan_size(T, E, k)
    return torch.zeros(max(n, 16), dtype=torch.uint8, device=device)


def moe_router(x, w, scales, biases):
    """Router QLinear of Qwen3MoeMlpBlock (qwen3_moe.rs:301-303) in the fixed summation order
    of the quantized-matmul restatement: bf16 logits [T, E], bit-reproducible."""
    _chk(x, torch.bfloat16, "x")
    T, K = x.shape
    E = w.shape[0]
    out = torch.empty(T, E, dtype=torch.bfloat16, device=x.device)
    ffi.call("higgs_moe_router", _ctx(x), _p(x), T, K, _p(w), _p(scales), _p(biases), E, _p(out),
             _st(x.device))
    return out


def moe_route_topk(logits, k: int, norm_topk_prob: bool, plan=None):
    """Router of Qwen3MoeMlpBlock::forward_moe (qwen3_moe.rs:303-316): softmax gates, top-k
    experts (ties -> lower index), optional renormalisation.  logits bf16 or f32 [T, E].
    Returns (idx int32 [T, k], scores f32 [T, k]); fills ``plan`` (from moe_plan) if given."""
    if logits.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError("logits must be bf16 or f32")
    _chk(logits, logits.dtype, "logits")
    T, E = logits.shape
    idx = torch.empty(T, k, dtype=torch.int32, device=logits.device)
    sc = torch.empty(T, k, dtype=torch.float32, device=logits.device)
    dt = ffi.DTYPE_BF16 if logits.dtype == torch.bfloat16 else ffi.DTYPE_F32
    ffi.call("higgs_moe_route_topk", _ctx(logits), _p(logits), dt, T, E, k, int(norm_topk_prob),
             _p(idx), _p(sc), _p(plan), 0 if plan is None else plan.numel(), _st(logits.device))
    return idx, sc


def moe_grouped_w4(x, k: int, plan, w, scales, biases, w_up=None, scales_up=None, biases_up=None,
                   x_per_pair: bool = False):
    """gather_qmm (qwen3_next.rs:294-363) over the routing plan: one output row per (token,
    slot) pair.  w u32 [E, N, K/8]; scales/biases bf16 [E, N, K/64].  x bf16 [T, K] (pair p
    reads row p // k) or, with x_per_pair, [T*k, K].  With w_up: swiglu(gate, up) fused.
    Returns bf16 [T*k, N]."""
    _chk(x, torch.bfloat16, "x")
    E, N, K8 = w.shape
    K = K8 * 8
    P = x.shape[0] if x_per_pair else x.shape[0] * k
    T = P // k
    y = torch.empty(P, N, dtype=torch.bfloat16, device=x.device)
    ffi.call("higgs_moe_grouped_w4", _ctx(x), _p(x), T, K, k, int(x_per_pair), _p(plan), _p(w),
             _p(scales), _p(biases), _p(w_up), _p(scales_up), _p(biases_up), E, N, _p(y),
             _st(x.device))
    return y


def moe_combine(y, scores, h):
    """sum_j bf16(score_j) * y[t*k+j] added to the residual h in place (qwen3_moe.rs:319-320,
    384-385).  y bf16 [T*k, H]; scores f32 [T, k]; h bf16 [T, H]."""
    _chk(y, torch.bfloat16, "y")
    _chk(scores, torch.float32, "scores")
    _chk(h, torch.bfloat16, "h")
    T, k = scores.shape
    H = h.shape[-1]
    ffi.call("higgs_moe_combine", _ctx(h), _p(y), _p(scores), T, k, H, _p(h), _st(h.device))
    return h


# ---- diagnostics ---------------------------------------------------------------

def tc_mma_rate(n: int, nacc: int = 1, spread: int = 0, iters: int = 4096, commit_every: int = 1,
                m: int = 128, warps: int = 1, ctas: int | None = None, device="cuda:0") -> dict:
    """Tensor-core issue rate of the matrix-form quantized matmul's instruction stream
    (higgs_diag_tc_mma_rate): SM cycles per tcgen05.mma m x n x 16 over all issuing warps,
    median over one CTA per SM.  Synchronising."""
    import ctypes
    dev = torch.device(device)
    if ctas is None:
        ctas = torch.cuda.get_device_properties(dev).multi_processor_count
    cycles = torch.zeros(ctas, dtype=torch.int64, device=dev)
    ffi.call("higgs_diag_tc_mma_rate", ffi.ctx(dev.index or 0), int(m), int(n), int(nacc), int(spread),
             int(iters), int(commit_every), int(warps), int(ctas), _p(cycles), _st(dev))
    torch.cuda.synchronize(dev)
    err = ctypes.c_int(0)
    ffi.call("higgs_tc_error", ffi.ctx(dev.index or 0), ctypes.byref(err))
    c = cycles.cpu().numpy()
    if err.value or (c < 0).any():
        raise RuntimeError("tc_mma_rate: a bounded wait gave up")
    med = float(sorted(c)[len(c) // 2])
    mmas = 4 * iters * warps
    return {"m": m, "n": n, "warps": warps, "nacc": nacc, "spread": spread, "commit_every": commit_every,
            "iters": iters, "cycles_per_mma": med / mmas, "flops_per_cycle": 2 * m * n * 16 * mmas / med}
