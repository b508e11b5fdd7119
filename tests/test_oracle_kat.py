"""CPU: pin the oracle against the reference's own known-answer tests and the
committed golden vectors, and check its internal consistency."""
import numpy as np
import pytest

from oracle import oracle as orc


def np_sdpa(q, k, v, mask, scale):
    """float64 softmax(q k^T * scale + mask) v with a bool keep-mask."""
    s = (q.astype(np.float64) @ k.astype(np.float64).T) * scale
    s = np.where(mask, s, -np.inf)
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    return p @ v.astype(np.float64)


# ---- reference known-answer tests --------------------------------------------

def test_kat_argmax(kat):
    for case in kat["argmax"]:
        got = orc.argmax(np.array(case["logits"], np.float32))
        assert got.tolist() == case["expect"], case["src"]


def test_kat_sample_filtered(kat):
    """The reference's top-k / top-p / min-p tests (lib.rs:821-853, 1070-1115): the kept tokens
    and, where the filter leaves one token with mass, the token itself, for any uniform."""
    us = np.linspace(0, 1, 64, endpoint=False, dtype=np.float32)
    for case in kat["sample_filtered"]:
        lg = np.array(case["logits"], np.float32)
        got = {int(orc.sample_filtered(lg, case["temperature"], case["top_k"], case["top_p"],
                                       case["min_p"], np.array([u], np.float32))[0]) for u in us}
        want = {case["expect"]} if case["expect"] is not None else set(case["allowed"])
        assert got == want, (case["src"], got, want)


def test_kat_penalties(kat):
    for case in kat["penalties"]:
        got = orc.apply_penalties(np.array(case["logits"], np.float32), case["history"],
                                  case["rep"], case["freq"], case["pres"])
        np.testing.assert_allclose(got, case["expect"], atol=1e-5, err_msg=case["src"])


def _paged(k_rows, v_rows, Hkv, D):
    """Lay [L, Hkv, D] rows into pages [P, Hkv, 16, D] with block table 0..P-1."""
    L = k_rows.shape[0]
    P = (L + 15) // 16
    kc = np.zeros((P, Hkv, 16, D), np.uint16)
    vc = np.zeros((P, Hkv, 16, D), np.uint16)
    for j in range(L):
        kc[j // 16, :, j % 16] = k_rows[j]
        vc[j // 16, :, j % 16] = v_rows[j]
    return kc, vc, np.arange(P, dtype=np.int32)[None]


@pytest.mark.parametrize("which", ["causal_mask", "batched_decode_mask"])
def test_kat_masks_through_positions(kat, which):
    """The reference's mask patterns (utils.rs) are exactly what the position
    rule of the paged attention reproduces: query t of a sequence of length L
    with Lq queries attends keys 0..L-Lq+t."""
    rng = np.random.default_rng(0)
    D = 64
    for case in kat[which]:
        mask = np.array(case["expect"], bool)
        if which == "causal_mask":
            n, off = case["n"], case["offset"]
            L = off + n
            seqs = [(n, L, mask)]
        else:
            seqs = [(1, l, mask[i:i + 1, :l]) for i, l in enumerate(case["kv_lengths"])]
        for Lq, L, m in seqs:
            kr = orc.f32_to_bf16(rng.normal(size=(L, 1, D)))
            vr = orc.f32_to_bf16(rng.normal(size=(L, 1, D)))
            q = orc.f32_to_bf16(rng.normal(size=(1, Lq, 1, D)))
            kc, vc, bt = _paged(kr, vr, 1, D)
            got = orc.bf16_to_f32(orc.paged_attention(q, kc, vc, bt, np.array([L], np.int32)))
            ref = np_sdpa(orc.bf16_to_f32(q[0, :, 0]), orc.bf16_to_f32(kr[:, 0]),
                          orc.bf16_to_f32(vr[:, 0]), m[:, :L], 1 / np.sqrt(D))
            np.testing.assert_allclose(got[0, :, 0], ref, atol=2e-2, rtol=1e-2, err_msg=case["src"])


def test_kat_sdpa_single_key(kat):
    for case in kat["sdpa_single_key"]:
        D = len(case["q"])
        q = orc.f32_to_bf16(np.array(case["q"], np.float32).reshape(1, 1, 1, D))
        kc = np.zeros((1, 1, 16, D), np.uint16)
        vc = np.zeros((1, 1, 16, D), np.uint16)
        kc[0, 0, 0] = orc.f32_to_bf16(np.array(case["k"], np.float32))
        vc[0, 0, 0] = orc.f32_to_bf16(np.array(case["v"], np.float32))
        out = orc.paged_attention(q, kc, vc, np.zeros((1, 1), np.int32), np.array([1], np.int32),
                                  scale=1 / np.sqrt(2.0))
        np.testing.assert_allclose(orc.bf16_to_f32(out).reshape(-1), case["expect"],
                                   atol=case["atol"], err_msg=case["src"])


def test_kat_swiglu(kat):
    for case in kat["swiglu"]:
        g = orc.f32_to_bf16(np.array(case["gate"], np.float32))
        x = orc.f32_to_bf16(np.array(case["x"], np.float32))
        got = orc.bf16_to_f32(orc.silu_mul(g, x))
        # the reference test is in f32; the op here emits bf16 (one rounding)
        np.testing.assert_allclose(got, case["expect"], rtol=2 ** -8, atol=case["atol"],
                                   err_msg=case["src"])


def test_kat_cache_values_preserved(kat):
    """Appends land at consecutive slots and earlier values survive (cache.rs:469-493)."""
    for case in kat["cache_values_preserved"]:
        rows = [r for app in case["appends"] for r in app]
        kr = orc.f32_to_bf16(np.array(rows, np.float32)[:, None, :])
        kc, _, _ = _paged(kr, kr, 1, kr.shape[-1])
        first = orc.bf16_to_f32(kc[0, 0, :len(rows), 0])
        assert first.tolist() == case["expect_first"], case["src"]


def test_kat_gather_equals_dense_relation(kat):
    """gather_qmm == per-expert quantized_matmul (qwen3_next.rs:2151-2206) holds
    trivially for the oracle's per-expert evaluation; the GPU grouped kernel is
    checked against it in test_kernels_gpu."""
    case = kat["gather_equals_dense"][0]
    rng = np.random.default_rng(3)
    w = rng.uniform(0, 1, size=(case["experts"], case["out"], case["in"])).astype(np.float32)
    x = orc.f32_to_bf16(rng.uniform(0, 1, size=(1, case["in"])))
    e = case["expert"]
    q, s, b = orc.w4_quantize(w[e])
    allq = [orc.w4_quantize(w[i]) for i in range(case["experts"])]
    y1 = orc.qmatmul(x, q, s, b, want_f32=True)[1]
    y2 = orc.qmatmul(x, *allq[e], want_f32=True)[1]
    assert np.max(np.abs(y1 - y2)) < case["max_abs"]


# ---- golden vectors ---------------------------------------------------------------

def test_golden_reproduced(golden):
    g = golden
    q, s, b = orc.w4_quantize(g["qm_w"])
    assert np.array_equal(q, g["qm_q"]) and np.array_equal(s, g["qm_s"]) and np.array_equal(b, g["qm_b"])
    yb, yf = orc.qmatmul(g["qm_x"], q, s, b, want_f32=True)
    assert np.array_equal(yb, g["qm_yb"])
    np.testing.assert_array_equal(yf, g["qm_yf"])
    assert np.array_equal(orc.w4_dequantize(q, s, b), g["qm_deq"])
    y, h = orc.rmsnorm(g["rn_x"], g["rn_w"], 1e-6, g["rn_r"])
    assert np.array_equal(y, g["rn_y"]) and np.array_equal(h, g["rn_h"])
    assert np.array_equal(orc.rope(g["rp_x"], g["rp_pos"], g["rp_inv"]), g["rp_y"])
    c, sc = orc.tq4_encode(g["tq_x"], g["tq_signs"])
    assert np.array_equal(c, g["tq_codes"]) and np.array_equal(sc.view(np.uint16), g["tq_scales"].view(np.uint16))
    out = orc.paged_attention(g["at_q"], g["at_k"], g["at_v"], g["at_bt"], g["at_sl"])
    assert np.array_equal(out, g["at_out"])
    assert np.array_equal(orc.sample(g["sm_logits"], 0.7, g["sm_u"]), g["sm_t07"])
    assert np.array_equal(orc.sample(g["sm_logits"], 0.0, None), g["sm_t0"])
    acc, toks = orc.spec_accept(g["sa_tl"], g["sa_dl"], g["sa_dt"], 0.7, g["sa_au"], g["sa_su"])
    assert np.array_equal(acc, g["sa_acc"]) and np.array_equal(toks, g["sa_toks"])
    fl, fu = g["sf_logits"], g["sf_u"]
    assert np.array_equal(orc.sample_filtered(fl, 0.8, top_k=40, uniforms=fu), g["sf_k40"])
    assert np.array_equal(orc.sample_filtered(fl, 0.8, top_p=0.9, uniforms=fu), g["sf_p09"])
    assert np.array_equal(orc.sample_filtered(fl, 0.8, min_p=0.1, uniforms=fu), g["sf_m01"])
    assert np.array_equal(orc.sample_filtered(fl, 1.3, top_k=100, top_p=0.8, min_p=0.02, uniforms=fu),
                          g["sf_all"])
    lp, ids, tlp = orc.logprobs(fl, 0.7, g["lp_tokens"], 5)
    assert np.array_equal(lp, g["lp_lp"]) and np.array_equal(ids, g["lp_ids"])
    assert np.array_equal(tlp, g["lp_top"])
    assert np.array_equal(orc.apply_token_mask(fl, g["mk_bits"]), g["mk_out"])


def _filtered_reference(lg, T, top_k, top_p, min_p):
    """A plain restatement of sample_filtered's masks (lib.rs:392-460) on the oracle's
    fixed-point masses: a stable descending argsort, the three masks, their product."""
    inv_t = np.float32(1.0) / np.float32(T)
    s = (lg.astype(np.float32) * inv_t).astype(np.float32)
    mxs = np.float32(lg.max()) * inv_t
    E = np.array([np.uint64(np.float64(orc.det_exp(float(np.float32(v - mxs)))) * 4294967296.0)
                  for v in s], np.uint64)
    order = np.argsort(-E.astype(np.float64), kind="stable")
    Es = E[order]
    V = lg.size
    k = V if top_k <= 0 or top_k > V else top_k
    rank_ok = np.arange(V) < k
    cum = np.cumsum(Es.astype(np.uint64))
    p_ok = (cum.astype(np.float64) <= np.float64(np.float32(top_p)) * np.float64(E.sum())) \
        if top_p < 1.0 else np.ones(V, bool)
    p_ok[0] = True
    m_ok = (Es.astype(np.float64) >= np.float64(np.float32(min(min_p, 1.0))) * np.float64(Es[0])) \
        if min_p > 0 else np.ones(V, bool)
    keep = np.zeros(V, bool)
    keep[order] = rank_ok & p_ok & m_ok
    return keep


@pytest.mark.parametrize("top_k,top_p,min_p", [(5, 1.0, 0.0), (0, 0.6, 0.0), (0, 1.0, 0.05),
                                               (30, 0.95, 0.01), (1, 1.0, 0.0), (0, 0.0, 0.0)])
def test_sample_filtered_keeps_exactly_the_mask_product(top_k, top_p, min_p):
    """Every draw lands in the kept set of the plain restatement, and with a dense grid of
    uniforms every kept token is drawn with its renormalised mass."""
    rng = np.random.default_rng(11)
    lg = rng.normal(0, 1.5, size=(1, 64)).astype(np.float32)
    lg[0, 10:14] = lg[0, 3]  # ties
    T = 0.9
    keep = _filtered_reference(lg[0], T, top_k, top_p, min_p)
    us = np.linspace(0, 1, 20000, endpoint=False, dtype=np.float32)
    toks = orc.sample_filtered(np.repeat(lg, len(us), 0), T, top_k, top_p, min_p, us)
    assert keep[toks].all()
    p = np.exp(lg[0].astype(np.float64) / T - lg[0].max() / T) * keep
    p /= p.sum()
    np.testing.assert_allclose(np.bincount(toks, minlength=64) / len(us), p, atol=2e-3)


def test_logprobs_match_float64_log_softmax():
    rng = np.random.default_rng(12)
    lg = rng.normal(0, 4, size=(3, 5000)).astype(np.float32)
    toks = np.array([0, 17, 4999], np.int32)
    for T in (0.0, 0.7, 1.5):
        lp, ids, tlp = orc.logprobs(lg, T, toks, 6)
        inv = np.float32(1.0) if T <= 1.1920929e-07 else np.float32(1.0) / np.float32(T)
        s = (lg * inv).astype(np.float64)
        ref = s - s.max(1, keepdims=True)
        ref = ref - np.log(np.exp(ref).sum(1, keepdims=True))
        np.testing.assert_allclose(lp, ref[np.arange(3), toks], atol=2e-6)
        order = np.argsort(-(lg * inv), axis=1, kind="stable")[:, :6]
        assert np.array_equal(ids, order)
        np.testing.assert_allclose(tlp, np.take_along_axis(ref, order, 1), atol=2e-6)


def test_token_mask_adds_minus_inf():
    lg = np.array([[1.0, -2.0, 0.5, 3.0, -0.0, 7.0]], np.float32)
    bits = orc.allowed_bits([[1, 4]], 6)
    out = orc.apply_token_mask(lg, bits)
    assert out[0, 1] == -2.0 and out[0, 4] == 0.0 and not np.signbit(out[0, 4])
    assert np.all(np.isneginf(out[0, [0, 2, 3, 5]]))


# ---- oracle self-consistency ---------------------------------------------------------

def test_w4_pack_layout_bit_exact():
    """Element k of a row sits in word k/8 at bits 4*(k%8) (MLX affine layout)."""
    rng = np.random.default_rng(5)
    codes = rng.integers(0, 16, size=(3, 128)).astype(np.uint32)
    words = np.zeros((3, 16), np.uint32)
    for k in range(128):
        words[:, k // 8] |= codes[:, k] << (4 * (k % 8))
    assert np.array_equal(orc.w4_unpack(words), codes.astype(np.uint8))


def test_quantize_roundtrip_and_matmul():
    rng = np.random.default_rng(6)
    w = rng.normal(0, 0.02, size=(64, 256)).astype(np.float32)
    q, s, b = orc.w4_quantize(w)
    deq = orc.bf16_to_f32(orc.w4_dequantize(q, s, b))
    step = orc.bf16_to_f32(s).repeat(64, axis=1)
    assert np.all(np.abs(deq - w) <= 0.51 * step + 2e-3 * np.abs(w) + 1e-6)
    x = orc.f32_to_bf16(rng.normal(size=(2, 256)))
    _, yf = orc.qmatmul(x, q, s, b, want_f32=True)
    # exact affine dequant in f64 as the contract
    codes = orc.w4_unpack(q).astype(np.float64)
    wexact = codes * np.repeat(orc.bf16_to_f32(s), 64, 1) + np.repeat(orc.bf16_to_f32(b), 64, 1)
    ref = orc.bf16_to_f32(x).astype(np.float64) @ wexact.T
    np.testing.assert_allclose(yf, ref, rtol=1e-5, atol=1e-5)


def test_det_exp_accuracy():
    xs = np.linspace(-87, 0, 20001, dtype=np.float32)
    got = np.array([orc.det_exp(float(x)) for x in xs[::97]])
    ref = np.exp(xs[::97].astype(np.float64))
    np.testing.assert_allclose(got, ref, rtol=4e-7)
    assert orc.det_exp(-200.0) == 0.0 and orc.det_exp(0.0) == 1.0


def test_sample_distribution_and_greedy_limit():
    rng = np.random.default_rng(7)
    lg = rng.normal(0, 1, size=(1, 8)).astype(np.float32)
    T = 0.7
    p = np.exp(lg[0] / T - (lg[0] / T).max())
    p /= p.sum()
    us = np.linspace(0, 1, 4001, endpoint=False, dtype=np.float32)
    toks = np.array([orc.sample(lg, T, np.array([u], np.float32))[0] for u in us])
    freq = np.bincount(toks, minlength=8) / len(us)
    np.testing.assert_allclose(freq, p, atol=2e-3)
    assert orc.sample(lg, 0.0, None)[0] == np.argmax(lg[0])


def test_spec_accept_edge_cases():
    rng = np.random.default_rng(8)
    B, k, V = 2, 3, 50
    tl = rng.normal(size=(B, k + 1, V)).astype(np.float32)
    # identical draft and target: every draft accepted (u < 1 = p/q)
    dl = tl[:, :k].copy()
    dt = rng.integers(0, V, size=(B, k)).astype(np.int32)
    au = rng.random((B, k)).astype(np.float32)
    su = rng.random(B).astype(np.float32)
    acc, toks = orc.spec_accept(tl, dl, dt, 0.7, au, su)
    assert acc.tolist() == [k, k]
    assert np.array_equal(toks[:, :k], dt) and np.all(toks[:, k] >= 0)
    # greedy: accept while draft == argmax(target)
    am = np.argmax(tl, axis=-1).astype(np.int32)
    dt2 = am[:, :k].copy()
    dt2[1, 1] = (dt2[1, 1] + 1) % V
    acc, toks = orc.spec_accept(tl, None, dt2, 0.0, None, None)
    assert acc.tolist() == [k, 1]
    assert toks[0].tolist() == am[0].tolist()
    assert toks[1].tolist() == [am[1, 0], am[1, 1], -1, -1]
    # an out-of-range draft token is rejected, never indexed
    dt3 = dt.copy()
    dt3[0, 0] = V + 5
    acc, _ = orc.spec_accept(tl, dl, dt3, 0.7, au, su)
    assert acc[0] == 0


def test_tq4_roundtrip_error_bound():
    rng = np.random.default_rng(9)
    signs = np.where(rng.random(128) < 0.5, -1, 1).astype(np.int8)
    x = orc.f32_to_bf16(rng.normal(size=(64, 128)))
    codes, scales = orc.tq4_encode(x, signs)
    dec = orc.tq4_decode(codes, scales, signs)
    xf = orc.bf16_to_f32(x)
    # per coordinate error in the rotated basis <= s/2 (+ fp16 scale rounding); orthogonal R
    # keeps the vector error norm <= sqrt(128) * s / 2
    err = np.linalg.norm(dec - xf, axis=1)
    bound = np.sqrt(128) * scales.astype(np.float32) * 0.51 + 1e-3
    assert np.all(err <= bound)
    rel = err / np.linalg.norm(xf, axis=1)
    assert rel.mean() < 0.12


def test_moe_route_topk():
    lg = np.array([[0.1, 2.0, -1.0, 2.0, 0.5]], np.float32)
    idx, sc = orc.moe_route_topk(lg, 3, True)
    assert idx.tolist() == [[1, 3, 4]]  # ties -> lower index first
    np.testing.assert_allclose(sc.sum(), 1.0, rtol=1e-6)
    idx2, sc2 = orc.moe_route_topk(lg, 2, False)
    p = np.exp(lg[0] - lg[0].max())
    p /= p.sum()
    np.testing.assert_allclose(sc2[0], p[[1, 3]], rtol=1e-6)


def test_moe_route_nan_signed_zero_and_ties():
    """NaN is never preferred, -0 == +0 (lower index first), exact ties -> lower index."""
    lg = np.array([[np.nan, 0.0, -0.0, 1.0, 1.0, -np.inf]], np.float32)
    idx, _ = orc.moe_route_topk(lg, 5, False)
    assert idx.tolist() == [[3, 4, 1, 2, 5]]
    lg2 = np.array([[-0.0, 0.0]], np.float32)
    assert orc.moe_route_topk(lg2, 1, True)[0].tolist() == [[0]]


def test_moe_combine_rounding_points():
    """h + bf16(sum_j bf16(s_j) y_j): scores rounded to bf16 before the product."""
    y = orc.f32_to_bf16(np.array([[1.0], [1.0]], np.float32))
    sc = np.array([[0.3, 0.7]], np.float32)
    h = orc.f32_to_bf16(np.array([[256.0]], np.float32))
    out = orc.bf16_to_f32(orc.moe_combine(y, sc, h))
    s_bf = orc.bf16_to_f32(orc.f32_to_bf16(sc))[0]
    acc = orc.bf16_to_f32(orc.f32_to_bf16(np.float32(s_bf[0] + s_bf[1])))
    assert out[0, 0] == orc.bf16_to_f32(orc.f32_to_bf16(np.float32(256.0) + acc))


def test_moe_experts_equal_dense_per_expert():
    """gather over experts == quantized_matmul on each expert's slice (qwen3_next.rs:2151-2206)."""
    rng = np.random.default_rng(8)
    E, F, H, T, k = 4, 256, 256, 3, 2
    mk = lambda N, K: [a.reshape(E, N, -1) for a in orc.w4_quantize(
        rng.normal(0, 0.02, size=(E * N, K)).astype(np.float32))]
    wg, wu, wd = mk(F, H), mk(F, H), mk(H, F)
    x = orc.f32_to_bf16(rng.normal(0, 1, size=(T, H)))
    idx = np.array([[2, 0], [1, 2], [3, 3]], np.int32)
    y = orc.moe_experts(x, idx, wg, wu, wd)
    for t_ in range(T):
        for j in range(k):
            e = idx[t_, j]
            g = orc.qmatmul(x[t_:t_ + 1], wg[0][e], wg[1][e], wg[2][e])
            u = orc.qmatmul(x[t_:t_ + 1], wu[0][e], wu[1][e], wu[2][e])
            d = orc.qmatmul(orc.silu_mul(g, u), wd[0][e], wd[1][e], wd[2][e])
            assert np.array_equal(y[t_ * k + j], d[0])
