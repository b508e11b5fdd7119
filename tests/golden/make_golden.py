"""Regenerate the golden fixtures in this directory.

    python tests/golden/make_golden.py

reference_kat.json -- known-answer values read (as text) from the higgs
    reference's own unit tests for the hot path; each entry cites its source.
oracle_vectors.npz -- small seeded inputs with the CPU oracle's outputs, so the
    oracle is pinned against regressions and GPU parity tests have fixed
    vectors that need neither the reference nor the oracle at run time.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", ".."))

from oracle import oracle as orc  # noqa: E402  (test infrastructure)

REFERENCE_KAT = {
    "argmax": [
        {"src": "crates/higgs-models/src/lib.rs:751-756 test_sample_greedy",
         "logits": [[0.1, 0.9, 0.0]], "expect": [1]},
        {"src": "crates/higgs-models/src/lib.rs:838-843 sample_uniform_logits_greedy",
         "logits": [[1.0, 1.0, 1.0, 1.0]], "expect": [0]},
        {"src": "crates/higgs-models/src/lib.rs:831-836 sample_single_element_logits",
         "logits": [[5.0]], "expect": [0]},
    ],
    # "expect": the token every uniform must give (the other tokens carry no mass after the
    # filter, or exp underflows), or null where the reference test checks only the shape and
    # the draw is left to the uniform ("allowed" then lists the tokens the filter keeps)
    "sample_filtered": [
        {"src": "crates/higgs-models/src/lib.rs:1070-1085 sample_top_k_limits_to_k_tokens",
         "logits": [[0.0, 0.0, 0.0, 100.0]], "temperature": 1.0, "top_k": 2, "top_p": 1.0,
         "min_p": 0.0, "expect": 3},
        {"src": "crates/higgs-models/src/lib.rs:1086-1098 sample_top_k_larger_than_vocab_is_no_op",
         "logits": [[0.1, 100.0, 0.0]], "temperature": 1.0, "top_k": 100, "top_p": 1.0,
         "min_p": 0.0, "expect": 1},
        {"src": "crates/higgs-models/src/lib.rs:1100-1115 sample_min_p_filters_low_probability",
         "logits": [[100.0, 0.0, 0.0, 0.0]], "temperature": 1.0, "top_k": 0, "top_p": 1.0,
         "min_p": 0.5, "expect": 0},
        {"src": "crates/higgs-models/src/lib.rs:826-829 sample_with_top_p",
         "logits": [[0.0, 100.0, 0.0]], "temperature": 1.0, "top_k": 0, "top_p": 0.5,
         "min_p": 0.0, "expect": 1},
        {"src": "crates/higgs-models/src/lib.rs:821-824 sample_with_temperature",
         "logits": [[0.1, 100.0, 0.0]], "temperature": 0.5, "top_k": 0, "top_p": 1.0,
         "min_p": 0.0, "expect": 1},
        {"src": "crates/higgs-models/src/lib.rs:850-853 sample_top_p_with_uniform_logits",
         "logits": [[1.0, 1.0, 1.0, 1.0]], "temperature": 1.0, "top_k": 0, "top_p": 0.3,
         "min_p": 0.0, "expect": None, "allowed": [0]},
        {"src": "crates/higgs-models/src/lib.rs:845-848 sample_uniform_logits_with_temperature",
         "logits": [[1.0, 1.0, 1.0, 1.0]], "temperature": 1.0, "top_k": 0, "top_p": 1.0,
         "min_p": 0.0, "expect": None, "allowed": [0, 1, 2, 3]},
    ],
    "penalties": [
        {"src": "crates/higgs-models/src/lib.rs:1137-1154 apply_repetition_penalty",
         "logits": [4.0, 2.0, 6.0], "history": [0, 2], "rep": 2.0, "freq": 0.0, "pres": 0.0,
         "expect": [2.0, 2.0, 3.0]},
        {"src": "crates/higgs-models/src/lib.rs:1155-1172 apply_repetition_penalty_negative_logits",
         "logits": [-4.0, 2.0, -6.0], "history": [0, 2], "rep": 2.0, "freq": 0.0, "pres": 0.0,
         "expect": [-8.0, 2.0, -12.0]},
        {"src": "crates/higgs-models/src/lib.rs:1173-1191 apply_frequency_penalty",
         "logits": [4.0, 2.0, 6.0], "history": [1, 1, 2], "rep": 1.0, "freq": 1.0, "pres": 0.0,
         "expect": [4.0, 0.0, 5.0]},
        {"src": "crates/higgs-models/src/lib.rs:1192-1208 apply_presence_penalty",
         "logits": [4.0, 2.0, 6.0], "history": [0, 0, 2], "rep": 1.0, "freq": 0.0, "pres": 1.5,
         "expect": [2.5, 2.0, 4.5]},
    ],
    "causal_mask": [
        {"src": "crates/higgs-models/src/utils.rs:133-158 test_create_causal_mask_n4",
         "n": 4, "offset": 0,
         "expect": [[1, 0, 0, 0], [1, 1, 0, 0], [1, 1, 1, 0], [1, 1, 1, 1]]},
        {"src": "crates/higgs-models/src/utils.rs:160-167 test_create_causal_mask_n1",
         "n": 1, "offset": 0, "expect": [[1]]},
        {"src": "crates/higgs-models/src/utils.rs:169-184 test_create_causal_mask_with_offset",
         "n": 2, "offset": 3, "expect": [[1, 1, 1, 1, 0], [1, 1, 1, 1, 1]]},
    ],
    "batched_decode_mask": [
        {"src": "crates/higgs-models/src/utils.rs:309-318 test_batched_decode_mask_values",
         "kv_lengths": [3, 5], "max_kv_len": 5,
         "expect": [[1, 1, 1, 0, 0], [1, 1, 1, 1, 1]]},
        {"src": "crates/higgs-models/src/utils.rs:300-307 test_batched_decode_mask_single_request",
         "kv_lengths": [4], "max_kv_len": 4, "expect": [[1, 1, 1, 1]]},
    ],
    "sdpa_single_key": [
        {"src": "crates/higgs-models/src/utils.rs:259-273 test_scaled_dot_product_attention_single_head_single_token",
         "q": [1.0, 1.0], "k": [1.0, 1.0], "v": [3.0, 7.0], "expect": [3.0, 7.0], "atol": 1e-4},
    ],
    "swiglu": [
        {"src": "crates/higgs-models/src/qwen3_next.rs:1927-1950 test_swiglu_numeric_correctness",
         "gate": [0.0, 1.0], "x": [5.0, 1.0], "expect": [0.0, 0.7310586], "atol": 1e-6},
    ],
    "cache_values_preserved": [
        {"src": "crates/higgs-models/src/cache.rs:469-493 test_stepping_cache_values_preserved",
         "appends": [[[1.0, 1.0, 1.0, 1.0], [1.0, 1.0, 1.0, 1.0]], [[2.0, 2.0, 2.0, 2.0]]],
         "expect_first": [1.0, 1.0, 2.0]},
    ],
    "gather_equals_dense": [
        {"src": "crates/higgs-models/src/qwen3_next.rs:2151-2206 test_gather_qmm_matches_per_expert",
         "experts": 4, "out": 64, "in": 64, "expert": 2, "max_abs": 1e-5},
    ],
}


def oracle_vectors() -> dict[str, np.ndarray]:
    rng = np.random.default_rng(1234)
    v: dict[str, np.ndarray] = {}
    # W4 quantize / qmatmul
    w = rng.normal(0, 0.02, size=(48, 512)).astype(np.float32)
    q, s, b = orc.w4_quantize(w)
    x = orc.f32_to_bf16(rng.normal(0, 1, size=(3, 512)))
    yb, yf = orc.qmatmul(x, q, s, b, want_f32=True)
    v.update(qm_w=w, qm_q=q, qm_s=s, qm_b=b, qm_x=x, qm_yb=yb, qm_yf=yf,
             qm_deq=orc.w4_dequantize(q, s, b))
    # rmsnorm with residual
    xr = orc.f32_to_bf16(rng.normal(0, 1, size=(2, 256)))
    rr = orc.f32_to_bf16(rng.normal(0, 1, size=(2, 256)))
    nw = orc.f32_to_bf16(rng.uniform(0.5, 1.5, size=256))
    y, h = orc.rmsnorm(xr, nw, 1e-6, rr)
    v.update(rn_x=xr, rn_r=rr, rn_w=nw, rn_y=y, rn_h=h)
    # rope
    xq = orc.f32_to_bf16(rng.normal(0, 1, size=(3, 2, 128)))
    pos = np.array([0, 7, 4095], np.int32)
    inv = orc.rope_inv_freq(128, 1000000.0)
    v.update(rp_x=xq, rp_pos=pos, rp_inv=inv, rp_y=orc.rope(xq, pos, inv))
    # TurboQuant encode (bit-exact contract)
    signs = np.where(rng.random(128) < 0.5, -1, 1).astype(np.int8)
    xt = orc.f32_to_bf16(rng.normal(0, 1, size=(40, 128)))
    xt[3] = 0  # zero vector -> zero scale, codes 8
    codes, scales = orc.tq4_encode(xt, signs)
    v.update(tq_signs=signs, tq_x=xt, tq_codes=codes, tq_scales=scales)
    # paged attention (2 sequences, ragged, GQA 4:2, Lq 2)
    D, Hkv, Hq = 64, 2, 4
    kc = orc.f32_to_bf16(rng.normal(0, 1, size=(6, Hkv, 16, D)))
    vc = orc.f32_to_bf16(rng.normal(0, 1, size=(6, Hkv, 16, D)))
    bt = np.array([[4, 1, 0], [2, 5, 3]], np.int32)
    sl = np.array([20, 37], np.int32)
    qa = orc.f32_to_bf16(rng.normal(0, 1, size=(2, 2, Hq, D)))
    v.update(at_q=qa, at_k=kc, at_v=vc, at_bt=bt, at_sl=sl,
             at_out=orc.paged_attention(qa, kc, vc, bt, sl))
    # sampling / acceptance (bit-exact given uniforms)
    lg = (rng.normal(0, 2, size=(3, 1000))).astype(np.float32)
    u = rng.random(3).astype(np.float32)
    v.update(sm_logits=lg, sm_u=u, sm_t07=orc.sample(lg, 0.7, u), sm_t0=orc.sample(lg, 0.0, None))
    B, k, V = 3, 4, 500
    tl = rng.normal(0, 1.5, size=(B, k + 1, V)).astype(np.float32)
    dl = (tl[:, :k] + rng.normal(0, 0.7, size=(B, k, V))).astype(np.float32)
    dt = rng.integers(0, V, size=(B, k)).astype(np.int32)
    dt[0] = np.argmax(dl[0], axis=-1)  # a likely-accepted row
    au = rng.random((B, k)).astype(np.float32)
    su = rng.random(B).astype(np.float32)
    acc, toks = orc.spec_accept(tl, dl, dt, 0.7, au, su)
    v.update(sa_tl=tl, sa_dl=dl, sa_dt=dt, sa_au=au, sa_su=su, sa_acc=acc, sa_toks=toks)
    # filtered sampling (top-k / top-p / min-p), logprobs, constraint mask
    fl = (rng.normal(0, 3, size=(4, 2000))).astype(np.float32)
    fl[1, 100:110] = fl[1, 5]  # ties across the top-k boundary
    fu = rng.random(4).astype(np.float32)
    v.update(sf_logits=fl, sf_u=fu,
             sf_k40=orc.sample_filtered(fl, 0.8, top_k=40, uniforms=fu),
             sf_p09=orc.sample_filtered(fl, 0.8, top_p=0.9, uniforms=fu),
             sf_m01=orc.sample_filtered(fl, 0.8, min_p=0.1, uniforms=fu),
             sf_all=orc.sample_filtered(fl, 1.3, top_k=100, top_p=0.8, min_p=0.02, uniforms=fu))
    toks = rng.integers(0, 2000, size=4).astype(np.int32)
    lp, ids, tlp = orc.logprobs(fl, 0.7, toks, 5)
    v.update(lp_tokens=toks, lp_lp=lp, lp_ids=ids, lp_top=tlp)
    allowed = [rng.choice(2000, size=n, replace=False) for n in (1, 7, 300, 2000)]
    bits = orc.allowed_bits(allowed, 2000)
    v.update(mk_bits=bits, mk_out=orc.apply_token_mask(fl, bits))
    return v


def main():
    with open(os.path.join(HERE, "reference_kat.json"), "w") as f:
        json.dump(REFERENCE_KAT, f, indent=1)
    np.savez_compressed(os.path.join(HERE, "oracle_vectors.npz"), **oracle_vectors())
    print("wrote", HERE)


if __name__ == "__main__":
    main()
