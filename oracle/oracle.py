"""numpy front end of the CPU oracle (liboracle.so, built from higgs_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / --impl reference legs of bench.py, never by the product
(higgs_b200/).  bf16 tensors are numpy uint16 bit patterns, fp16 are float16.
Every function cites the reference call site its C restatement follows.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")

_lib = None


def build() -> str:
    """Compile liboracle.so with the committed Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(
                os.path.join(HERE, "higgs_oracle.c")):
            build()
        _lib = ctypes.CDLL(LIB)
        _lib.orc_exp.restype = ctypes.c_float
        _lib.orc_exp.argtypes = [ctypes.c_float]
    return _lib


def set_threads(n: int) -> int:
    """OpenMP threads for the oracle's parallel loops (n <= 0: unchanged); returns the count
    in force."""
    return int(lib().orc_set_threads(int(n)))


class summation_order:
    """Context manager: run the oracle's unordered floating-point reductions in the second
    valid order (orc_set_order(1)) -- two restatements of the same arithmetic whose difference
    is the rounding noise of summation order alone."""

    def __init__(self, mode: int = 1):
        self.mode = mode

    def __enter__(self):
        self.old = lib().orc_set_order(self.mode)
        return self

    def __exit__(self, *exc):
        lib().orc_set_order(self.old)


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


I64 = ctypes.c_int64
F = ctypes.c_float


# ---- bf16 helpers -----------------------------------------------------------

def f32_to_bf16(x) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bits (uint16)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_to_f32(h) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    return (h.astype(np.uint32) << 16).view(np.float32)


def round_bf16(x) -> np.ndarray:
    return bf16_to_f32(f32_to_bf16(x))


# ---- W4 g64 ------------------------------------------------------------------

def w4_quantize(w: np.ndarray):
    """This build's affine quantizer (see higgs_oracle.c): (q u32 [N,K/8], s, b bf16 [N,K/64])."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, K = w.shape
    assert K % 64 == 0
    q = np.empty((N, K // 8), np.uint32)
    s = np.empty((N, K // 64), np.uint16)
    b = np.empty((N, K // 64), np.uint16)
    lib().orc_w4_quantize(_ptr(w), I64(N), I64(K), _ptr(q), _ptr(s), _ptr(b))
    return q, s, b


def w4_unpack(q: np.ndarray) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.uint32)
    N, K = q.shape[0], q.shape[1] * 8
    out = np.empty((N, K), np.uint8)
    lib().orc_w4_unpack(_ptr(q), I64(N), I64(K), _ptr(out))
    return out


def w4_dequantize(q, s, b) -> np.ndarray:
    """ops::dequantize (qwen3_next.rs:249-256) -> bf16 bits [N, K]."""
    q = np.ascontiguousarray(q, dtype=np.uint32)
    N, K = q.shape[0], q.shape[1] * 8
    out = np.empty((N, K), np.uint16)
    lib().orc_w4_dequantize(_ptr(q), _ptr(np.ascontiguousarray(s)), _ptr(np.ascontiguousarray(b)),
                            I64(N), I64(K), _ptr(out))
    return out


def embed_gather(ids, q, s, b) -> np.ndarray:
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    V, H = q.shape[0], q.shape[1] * 8
    out = np.empty((ids.size, H), np.uint16)
    lib().orc_embed_gather(_ptr(ids), I64(ids.size), _ptr(q), _ptr(s), _ptr(b), I64(V), I64(H),
                           _ptr(out))
    return out.reshape(*ids.shape, H)


def qmatmul_dq(x_bf16, q, s, b, want_f32: bool = False):
    """quantized_matmul in MLX's matrix form (qmm): weights dequantized to bf16 first."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    K = x.shape[-1]
    M = x.size // K
    N = q.shape[0]
    yb = np.empty((M, N), np.uint16)
    yf = np.empty((M, N), np.float32) if want_f32 else None
    lib().orc_qmatmul_dq(_ptr(x), I64(M), I64(K), _ptr(np.ascontiguousarray(q)),
                         _ptr(np.ascontiguousarray(s)), _ptr(np.ascontiguousarray(b)), I64(N),
                         _ptr(yf), _ptr(yb))
    yb = yb.reshape(*x.shape[:-1], N)
    return (yb, yf.reshape(*x.shape[:-1], N)) if want_f32 else yb


def qmatmul(x_bf16, q, s, b, want_f32: bool = False):
    """ops::quantized_matmul (qwen3_next.rs:174-183): x bf16 [M,K] -> bf16 [M,N] (and f32)."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    K = x.shape[-1]
    M = x.size // K
    N = q.shape[0]
    yb = np.empty((M, N), np.uint16)
    yf = np.empty((M, N), np.float32) if want_f32 else None
    lib().orc_qmatmul(_ptr(x), I64(M), I64(K), _ptr(np.ascontiguousarray(q)),
                      _ptr(np.ascontiguousarray(s)), _ptr(np.ascontiguousarray(b)), I64(N),
                      _ptr(yf), _ptr(yb))
    yb = yb.reshape(*x.shape[:-1], N)
    return (yb, yf.reshape(*x.shape[:-1], N)) if want_f32 else yb


# ---- norms / rope / activations ------------------------------------------------

def rmsnorm(x, w, eps, residual=None):
    """fast::rms_norm (transformer.rs:375-377); returns (y, h) bf16."""
    x = np.ascontiguousarray(x, dtype=np.uint16)
    H = x.shape[-1]
    rows = x.size // H
    y = np.empty_like(x)
    h = np.empty_like(x)
    lib().orc_rmsnorm(_ptr(x), _ptr(None if residual is None else np.ascontiguousarray(residual)),
                      I64(rows), I64(H), _ptr(np.ascontiguousarray(w)), F(eps), _ptr(y), _ptr(h))
    return y, h


def rope_inv_freq(dims: int, base: float) -> np.ndarray:
    return np.array([base ** (-(2.0 * i) / dims) for i in range(dims // 2)], dtype=np.float32)


def rope(x, pos, inv_freq):
    """fast::rope traditional=false (utils.rs:16-26); x bf16 [rows, heads, D]."""
    x = np.ascontiguousarray(x, dtype=np.uint16)
    rows, heads, D = x.shape
    out = np.empty_like(x)
    lib().orc_rope(_ptr(x), I64(rows), I64(heads), I64(D),
                   _ptr(np.ascontiguousarray(pos, dtype=np.int32)),
                   _ptr(np.ascontiguousarray(inv_freq, dtype=np.float32)), _ptr(out))
    return out


def silu_mul(g, u):
    g = np.ascontiguousarray(g, dtype=np.uint16)
    out = np.empty_like(g)
    lib().orc_silu_mul(_ptr(g), _ptr(np.ascontiguousarray(u, dtype=np.uint16)), I64(g.size),
                       _ptr(out))
    return out


# ---- attention ---------------------------------------------------------------

def paged_attention(q, k_cache, v_cache, block_table, seq_lens, scale=None):
    """SDPA over paged caches [pages, Hkv, 16, D] (utils.rs:45-60, masks 64-125)."""
    q = np.ascontiguousarray(q, dtype=np.uint16)
    B, Lq, Hq, D = q.shape
    P, Hkv, page, D2 = k_cache.shape
    assert D2 == D
    bt = np.ascontiguousarray(block_table, dtype=np.int32)
    out = np.empty_like(q)
    if scale is None:
        scale = 1.0 / np.sqrt(D)
    lib().orc_paged_attention(_ptr(q), I64(B), I64(Lq), I64(Hq), I64(Hkv), I64(D),
                              _ptr(np.ascontiguousarray(k_cache)), _ptr(np.ascontiguousarray(v_cache)),
                              I64(page), I64(Hkv * page * D), I64(page * D), _ptr(bt),
                              I64(bt.shape[1]), _ptr(np.ascontiguousarray(seq_lens, dtype=np.int32)),
                              F(scale), _ptr(out))
    return out


def tq4_encode(x, signs):
    """TurboQuant encode (no reference counterpart): codes u8 [n, 64], scales fp16 [n]."""
    x = np.ascontiguousarray(x, dtype=np.uint16).reshape(-1, 128)
    n = x.shape[0]
    codes = np.empty((n, 64), np.uint8)
    scales = np.empty(n, np.float16)
    lib().orc_tq4_encode(_ptr(x), I64(n), _ptr(np.ascontiguousarray(signs, dtype=np.int8)),
                         _ptr(codes), _ptr(scales))
    return codes, scales


def tq4_decode(codes, scales, signs) -> np.ndarray:
    codes = np.ascontiguousarray(codes, dtype=np.uint8).reshape(-1, 64)
    n = codes.shape[0]
    out = np.empty((n, 128), np.float32)
    lib().orc_tq4_decode(_ptr(codes), _ptr(np.ascontiguousarray(scales, dtype=np.float16)), I64(n),
                         _ptr(np.ascontiguousarray(signs, dtype=np.int8)), _ptr(out))
    return out


def paged_attention_tq4(q, k_codes, k_scales, v_codes, v_scales, block_table, seq_lens, signs,
                        scale=None):
    q = np.ascontiguousarray(q, dtype=np.uint16)
    B, Lq, Hq, D = q.shape
    P, Hkv, page, _ = k_codes.shape
    bt = np.ascontiguousarray(block_table, dtype=np.int32)
    out = np.empty_like(q)
    if scale is None:
        scale = 1.0 / np.sqrt(D)
    lib().orc_paged_attention_tq4(
        _ptr(q), I64(B), I64(Lq), I64(Hq), I64(Hkv), _ptr(np.ascontiguousarray(k_codes)),
        _ptr(np.ascontiguousarray(k_scales)), _ptr(np.ascontiguousarray(v_codes)),
        _ptr(np.ascontiguousarray(v_scales)), I64(page), I64(Hkv * page * 64), I64(page * 64),
        _ptr(bt), I64(bt.shape[1]), _ptr(np.ascontiguousarray(seq_lens, dtype=np.int32)),
        _ptr(np.ascontiguousarray(signs, dtype=np.int8)), F(scale), _ptr(out))
    return out


# ---- token selection -----------------------------------------------------------

def det_exp(x: float) -> float:
    return float(lib().orc_exp(F(x)))


def argmax(logits) -> np.ndarray:
    """sample() at T=0 (lib.rs:373-377); ties -> first index (lib.rs:838-843)."""
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    B, V = lg.reshape(-1, lg.shape[-1]).shape
    out = np.empty(B, np.int32)
    lib().orc_argmax(_ptr(lg), I64(B), I64(V), _ptr(out))
    return out


def sample(logits, temperature, uniforms) -> np.ndarray:
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    B, V = lg.shape
    out = np.empty(B, np.int32)
    u = None if uniforms is None else np.ascontiguousarray(uniforms, dtype=np.float32)
    lib().orc_sample(_ptr(lg), I64(B), I64(V), F(temperature), _ptr(u), _ptr(out))
    return out


def spec_accept(target_logits, draft_logits, draft_tokens, temperature, accept_u, sample_u):
    tl = np.ascontiguousarray(target_logits, dtype=np.float32)
    B, k1, V = tl.shape
    k = k1 - 1
    dl = None if draft_logits is None else np.ascontiguousarray(draft_logits, dtype=np.float32)
    acc = np.empty(B, np.int32)
    toks = np.empty((B, k1), np.int32)
    au = None if accept_u is None else np.ascontiguousarray(accept_u, dtype=np.float32)
    su = None if sample_u is None else np.ascontiguousarray(sample_u, dtype=np.float32)
    lib().orc_spec_accept(_ptr(tl), _ptr(dl), _ptr(np.ascontiguousarray(draft_tokens, dtype=np.int32)),
                          I64(B), I64(k), I64(V), F(temperature), _ptr(au), _ptr(su), _ptr(acc),
                          _ptr(toks))
    return acc, toks


def apply_token_mask(logits, allowed_bits) -> np.ndarray:
    """Constraint::apply_mask (constrained.rs:79-110): logits + (0 | -inf) from a per-row bitmask
    u32 [B, ceil(V/32)] (bit j%32 of word j/32 = token j allowed); returns a new array."""
    lg = np.array(logits, dtype=np.float32)
    B, V = lg.shape
    bits = np.ascontiguousarray(allowed_bits, dtype=np.uint32)
    lib().orc_apply_token_mask(_ptr(lg), I64(B), I64(V), _ptr(bits), I64(bits.shape[1]))
    return lg


def allowed_bits(allowed_ids_per_row, V: int) -> np.ndarray:
    """Bitmask u32 [B, ceil(V/32)] from per-row lists of allowed token ids."""
    W = (V + 31) // 32
    out = np.zeros((len(allowed_ids_per_row), W), np.uint32)
    for b, ids in enumerate(allowed_ids_per_row):
        ids = np.asarray([i for i in ids if 0 <= i < V], np.int64)
        np.bitwise_or.at(out[b], ids // 32, (np.uint32(1) << (ids % 32).astype(np.uint32)))
    return out


def sample_filtered(logits, temperature, top_k=0, top_p=1.0, min_p=0.0, uniforms=None) -> np.ndarray:
    """sample() with top-k / top-p / min-p (lib.rs:373-460) over the fixed-point masses."""
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    B, V = lg.shape
    out = np.empty(B, np.int32)
    u = None if uniforms is None else np.ascontiguousarray(uniforms, dtype=np.float32)
    lib().orc_sample_filtered(_ptr(lg), I64(B), I64(V), F(temperature), I64(int(top_k)), F(top_p),
                              F(min_p), _ptr(u), _ptr(out))
    return out


def logprobs(logits, temperature, tokens, top_n: int):
    """LogprobArrays::compute (lib.rs:495-533): (token logprob f32 [B], top ids int32 [B, n],
    top logprobs f32 [B, n])."""
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    B, V = lg.shape
    lp = np.empty(B, np.float32)
    ids = np.empty((B, max(top_n, 0)), np.int32)
    tl = np.empty((B, max(top_n, 0)), np.float32)
    lib().orc_logprobs(_ptr(lg), I64(B), I64(V), F(temperature),
                       _ptr(np.ascontiguousarray(tokens, dtype=np.int32)), I64(top_n), _ptr(lp),
                       _ptr(ids), _ptr(tl))
    return lp, ids, tl


def apply_penalties(logits, history, rep=1.0, freq=0.0, pres=0.0) -> np.ndarray:
    """apply_penalties (lib.rs:278-363) on one row; returns a new array."""
    lg = np.array(logits, dtype=np.float32).reshape(-1)
    h = np.ascontiguousarray(history, dtype=np.int32)
    lib().orc_apply_penalties(_ptr(lg), I64(lg.size), _ptr(h), I64(h.size), F(rep), F(freq),
                              F(pres))
    return lg


def moe_route_topk(logits, k: int, norm: bool):
    """Qwen3MoeMlpBlock router (qwen3_moe.rs:303-316): (idx int32 [T,k], scores f32 [T,k]).
    Top-k by logit, ties to the lower expert index; gates softmax in f32."""
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    T, E = lg.shape
    idx = np.empty((T, k), np.int32)
    sc = np.empty((T, k), np.float32)
    lib().orc_moe_route_topk(_ptr(lg), I64(T), I64(E), I64(k), ctypes.c_int(int(norm)), _ptr(idx),
                             _ptr(sc))
    return idx, sc


def moe_combine(y, scores, h):
    """sum_j score_j * y_j + residual (qwen3_moe.rs:319-320, 384-385) with MLX's bf16
    rounding points; y bf16 [T*k, H], scores f32 [T, k], h bf16 [T, H] -> new h."""
    sc = np.ascontiguousarray(scores, dtype=np.float32)
    T, k = sc.shape
    yy = np.ascontiguousarray(y, dtype=np.uint16)
    out = np.array(h, dtype=np.uint16, copy=True)
    H = out.shape[-1]
    lib().orc_moe_combine(_ptr(yy), _ptr(sc), I64(T), I64(k), I64(H), _ptr(out))
    return out


def moe_experts(x, idx, w_gate, w_up, w_down):
    """SwitchMlpWeights::forward_gather (qwen3_next.rs:844-904) for each (token, slot) pair,
    evaluated one expert at a time with qmatmul (gather_qmm == per-expert quantized_matmul,
    qwen3_next.rs:2151-2206).  x bf16 [T, H]; idx int32 [T, k]; w_* = (q [E,N,K/8], s, b).
    Returns bf16 [T*k, H]."""
    T, k = idx.shape
    Hd = w_down[0].shape[1]
    out = np.zeros((T * k, Hd), np.uint16)
    for e in np.unique(idx):
        pairs = np.nonzero(idx.reshape(-1) == e)[0]
        xe = np.ascontiguousarray(x[pairs // k])
        g = qmatmul(xe, w_gate[0][e], w_gate[1][e], w_gate[2][e])
        u = qmatmul(xe, w_up[0][e], w_up[1][e], w_up[2][e])
        out[pairs] = qmatmul(silu_mul(g, u), w_down[0][e], w_down[1][e], w_down[2][e])
    return out
