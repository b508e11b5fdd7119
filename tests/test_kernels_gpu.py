"""GPU parity: every C-ABI kernel against the CPU oracle on the same seeded inputs.

Bars: bit-exact for integer/byte work (unpack/dequant, embedding rows, cache
slots, TurboQuant codes, sampled / accepted tokens given uniforms); floating
point within the stated tolerance (north star: max-abs 2e-2 / rel 1e-2 in bf16;
the per-op bounds below are tighter).
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as orc

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def ops():
    from higgs_b200 import ops as o
    return o


def t(a, dtype=None):
    x = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        x = x.view(dtype)
    return x.to(DEV)


def bf(a):
    return t(np.ascontiguousarray(a, dtype=np.uint16), torch.bfloat16)


def to_np_bf(x):
    return x.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def qweights(rng, N, K, sd=0.02):
    w = rng.normal(0, sd, size=(N, K)).astype(np.float32)
    return orc.w4_quantize(w)


def bf_ulps(a_bits, b_bits):
    """distance in bf16 ulps between two bf16 bit arrays (sign-magnitude aware)."""
    def key(x):
        x = x.astype(np.int32)
        return np.where(x & 0x8000, -(x & 0x7FFF), x)
    return np.abs(key(a_bits) - key(b_bits))


# ---- a1/a2 --------------------------------------------------------------------

@pytest.mark.parametrize("M,K,N", [(1, 256, 16), (1, 4096, 1024), (3, 2048, 512), (8, 4096, 256),
                                   (13, 1024, 128), (32, 2048, 64), (40, 512, 96), (1, 12288, 256)])
def test_qlinear_vs_oracle(M, K, N):
    rng = np.random.default_rng(M * 1000 + K + N)
    q, s, b = qweights(rng, N, K)
    x = orc.f32_to_bf16(rng.normal(0, 1, size=(M, K)))
    yb_ref, yf_ref = orc.qmatmul(x, q, s, b, want_f32=True)
    o = ops()
    yf = o.quantized_matmul(bf(x), t(q.view(np.int32)), bf(s), bf(b), out_f32=True).cpu().numpy()
    scale = np.abs(yf_ref).max()
    np.testing.assert_allclose(yf, yf_ref, rtol=1e-3, atol=1e-4 * scale + 1e-6)
    yb = to_np_bf(o.quantized_matmul(bf(x), t(q.view(np.int32)), bf(s), bf(b)))
    # bf16 output: within one bf16 rounding of the f32 reference plus the f32 summation noise
    # (~1e-5 of the output scale: an output 1000x below the scale can sit 2 ulps away), and
    # within one ulp of the oracle's bf16 wherever that noise is far below an ulp
    np.testing.assert_allclose(orc.bf16_to_f32(yb), yf_ref, rtol=2 ** -7, atol=1e-4 * scale + 1e-6)
    big = np.abs(yf_ref) >= 1e-2 * scale
    assert bf_ulps(yb, yb_ref)[big].max() <= 1


@pytest.mark.parametrize("wk,depth", [(0, 2), (1, 2), (2, 4), (4, 2), (8, 4)])
@pytest.mark.parametrize("K,N", [(2304, 64), (768, 48)])
def test_qlinear_one_token_splits(wk, depth, K, N):
    """The single-token GEMV under every K split and pipeline depth.  K = 9 and 3 units of
    256 leave warps with odd unit counts (a lone last unit folded without its pair); the
    results must match the oracle and the multi-token kernel run on the same row."""
    from higgs_b200 import ffi
    rng = np.random.default_rng(K + N + wk)
    q, s, b = qweights(rng, N, K)
    x = orc.f32_to_bf16(rng.normal(0, 1, size=(1, K)))
    r = orc.f32_to_bf16(rng.normal(size=(1, N)))
    yb_ref, yf_ref = orc.qmatmul(x, q, s, b, want_f32=True)
    o = ops()
    try:
        ffi.call("higgs_set_option", b"gemv_m1_wk", wk)
        ffi.call("higgs_set_option", b"gemv_m1_depth", depth)
        yf = o.quantized_matmul(bf(x), t(q.view(np.int32)), bf(s), bf(b), out_f32=True).cpu().numpy()
        yr = to_np_bf(o.quantized_matmul(bf(x), t(q.view(np.int32)), bf(s), bf(b), residual=bf(r)))
        ffi.call("higgs_set_option", b"gemv_m1", 0)
        yf_ring = o.quantized_matmul(bf(x), t(q.view(np.int32)), bf(s), bf(b), out_f32=True).cpu().numpy()
    finally:
        ffi.call("higgs_set_option", b"gemv_m1", 1)
        ffi.call("higgs_set_option", b"gemv_m1_wk", 0)
        ffi.call("higgs_set_option", b"gemv_m1_depth", 2)
    scale = np.abs(yf_ref).max()
    np.testing.assert_allclose(yf, yf_ref, rtol=1e-3, atol=1e-4 * scale + 1e-6)
    np.testing.assert_allclose(yf, yf_ring, rtol=1e-3, atol=1e-4 * scale + 1e-6)
    # y is rounded to bf16 before the residual add: a 1-ulp flip of y (a rounding tie broken
    # by f32 noise) is one ulp of y in the sum, however small the sum is after cancellation
    yv, rv = orc.bf16_to_f32(yb_ref), orc.bf16_to_f32(r)
    res_ref = orc.bf16_to_f32(orc.f32_to_bf16(yv + rv))
    bound = 2.0 ** -7 * (np.abs(yv) + np.abs(res_ref)) + 1e-30  # one ulp of each: <= 2^-7 relative
    assert (np.abs(orc.bf16_to_f32(yr) - res_ref) <= bound).all()


def test_qlinear_golden(golden):
    g = golden
    o = ops()
    yb = to_np_bf(o.quantized_matmul(bf(g["qm_x"]), t(g["qm_q"].view(np.int32)), bf(g["qm_s"]),
                                     bf(g["qm_b"])))
    assert bf_ulps(yb, g["qm_yb"]).max() <= 1


def test_qlinear_residual_epilogue():
    rng = np.random.default_rng(11)
    M, K, N = 2, 1024, 256
    q, s, b = qweights(rng, N, K)
    x = orc.f32_to_bf16(rng.normal(size=(M, K)))
    r = orc.f32_to_bf16(rng.normal(size=(M, N)))
    yb_ref = orc.qmatmul(x, q, s, b)
    ref = orc.f32_to_bf16(orc.bf16_to_f32(yb_ref) + orc.bf16_to_f32(r))
    got = to_np_bf(ops().quantized_matmul(bf(x), t(q.view(np.int32)), bf(s), bf(b), residual=bf(r)))
    assert bf_ulps(got, ref).max() <= 1


@pytest.mark.parametrize("M", [1, 5, 17])
def test_gate_up_swiglu(M):
    rng = np.random.default_rng(12 + M)
    K, N = 2048, 512
    qg, sg, bg = qweights(rng, N, K)
    qu, su, bu = qweights(rng, N, K)
    x = orc.f32_to_bf16(rng.normal(size=(M, K)))
    qm = orc.qmatmul_dq if M >= 17 else orc.qmatmul  # the GPU's matrix form from 17 rows
    ref = orc.silu_mul(qm(x, qg, sg, bg), qm(x, qu, su, bu))
    got = to_np_bf(ops().gate_up_swiglu(bf(x), t(qg.view(np.int32)), bf(sg), bf(bg),
                                        t(qu.view(np.int32)), bf(su), bf(bu)))
    # gate/up are rounded to bf16 before the product: a 1-ulp flip there moves the output by ~2 ulps
    assert np.percentile(bf_ulps(got, ref), 99) <= 2
    np.testing.assert_allclose(orc.bf16_to_f32(got), orc.bf16_to_f32(ref), atol=2e-3, rtol=2e-2)


def test_dequantize_and_embed_bit_exact():
    rng = np.random.default_rng(13)
    V, H = 300, 512
    q, s, b = qweights(rng, V, H)
    o = ops()
    deq = to_np_bf(o.dequantize(t(q.view(np.int32)), bf(s), bf(b)))
    assert np.array_equal(deq, orc.w4_dequantize(q, s, b))
    ids = np.array([0, 299, 17, -1, 300, 17], np.int32)
    got = to_np_bf(o.embed_gather(t(ids), t(q.view(np.int32)), bf(s), bf(b)))
    assert np.array_equal(got, orc.embed_gather(ids, q, s, b))
    assert not got[3].any() and not got[4].any()


# ---- a3/a4 --------------------------------------------------------------------------

@pytest.mark.parametrize("H", [64, 2048, 4096])
def test_rmsnorm(H, golden):
    rng = np.random.default_rng(H)
    x = orc.f32_to_bf16(rng.normal(size=(3, H)))
    r = orc.f32_to_bf16(rng.normal(size=(3, H)))
    w = orc.f32_to_bf16(rng.uniform(0.5, 1.5, size=H))
    y_ref, h_ref = orc.rmsnorm(x, w, 1e-6, r)
    y, h = ops().rms_norm(bf(x), bf(w), 1e-6, residual=bf(r), want_h=True)
    assert np.array_equal(to_np_bf(h), h_ref)
    assert bf_ulps(to_np_bf(y), y_ref).max() <= 1
    y2 = ops().rms_norm(bf(x), bf(w), 1e-5)
    assert bf_ulps(to_np_bf(y2), orc.rmsnorm(x, w, 1e-5)[0]).max() <= 1
    g = golden
    yg, hg = ops().rms_norm(bf(g["rn_x"]), bf(g["rn_w"]), 1e-6, residual=bf(g["rn_r"]), want_h=True)
    assert np.array_equal(to_np_bf(hg), g["rn_h"]) and bf_ulps(to_np_bf(yg), g["rn_y"]).max() <= 1


@pytest.mark.parametrize("D", [64, 128])
def test_rope(D):
    rng = np.random.default_rng(D)
    x = orc.f32_to_bf16(rng.normal(size=(5, 3, D)))
    pos = np.array([0, 1, 127, 2048, 32767], np.int32)
    inv = orc.rope_inv_freq(D, 500000.0)
    ref = orc.rope(x, pos, inv)
    got = to_np_bf(ops().rope(bf(x), t(pos), t(inv)))
    assert bf_ulps(got, ref).max() <= 1


def _kvwrite_case(rng, T, Hq, Hkv, D, qknorm):
    nh = Hq + 2 * Hkv
    qkv = orc.f32_to_bf16(rng.normal(size=(T, nh * D)))
    qn = orc.f32_to_bf16(rng.uniform(0.5, 1.5, size=D)) if qknorm else None
    kn = orc.f32_to_bf16(rng.uniform(0.5, 1.5, size=D)) if qknorm else None
    pos = rng.integers(0, 4000, size=T).astype(np.int32)
    inv = orc.rope_inv_freq(D, 1000000.0)
    return qkv, qn, kn, pos, inv


def _kvwrite_ref(qkv, qn, kn, pos, inv, T, Hq, Hkv, D):
    x = qkv.reshape(T, Hq + 2 * Hkv, D)
    qh, kh, vh = x[:, :Hq], x[:, Hq:Hq + Hkv], x[:, Hq + Hkv:]
    if qn is not None:
        qh = orc.rmsnorm(qh.reshape(-1, D), qn, 1e-6)[0].reshape(T, Hq, D)
        kh = orc.rmsnorm(kh.reshape(-1, D), kn, 1e-6)[0].reshape(T, Hkv, D)
    return orc.rope(qh, pos, inv), orc.rope(np.ascontiguousarray(kh), pos, inv), vh


@pytest.mark.parametrize("Hq,Hkv,D,qknorm", [(32, 8, 64, False), (16, 8, 128, True), (32, 4, 128, True)])
def test_qknorm_rope_kv_write(Hq, Hkv, D, qknorm):
    rng = np.random.default_rng(Hq + Hkv + D)
    T = 5
    qkv, qn, kn, pos, inv = _kvwrite_case(rng, T, Hq, Hkv, D, qknorm)
    P = 4
    sentinel = 0x3F80  # bf16 1.0
    kc = torch.full((P, Hkv, 16, D), 1.0, dtype=torch.bfloat16, device=DEV)
    vc = torch.full((P, Hkv, 16, D), 1.0, dtype=torch.bfloat16, device=DEV)
    slots = np.array([3 * 16 + 0, 0 * 16 + 15, -1, 2 * 16 + 7, 1 * 16 + 1], np.int64)
    q = ops().qknorm_rope_kv_write(bf(qkv), Hq, Hkv, D, None if qn is None else bf(qn),
                                   None if kn is None else bf(kn), 1e-6, t(pos), t(inv), t(slots), kc, vc)
    q_ref, k_ref, v_ref = _kvwrite_ref(qkv, qn, kn, pos, inv, T, Hq, Hkv, D)
    assert bf_ulps(to_np_bf(q), q_ref).max() <= 1
    kcn, vcn = to_np_bf(kc), to_np_bf(vc)
    written = np.zeros((P, 16), bool)
    for i, sl in enumerate(slots):
        if sl < 0:
            continue
        p, s = sl // 16, sl % 16
        written[p, s] = True
        assert bf_ulps(kcn[p, :, s], k_ref[i]).max() <= 1
        assert np.array_equal(vcn[p, :, s], v_ref[i])
    kt_, vt_ = kcn.transpose(0, 2, 1, 3), vcn.transpose(0, 2, 1, 3)  # [P, 16, Hkv, D]
    assert np.all(kt_[~written] == sentinel) and np.all(vt_[~written] == sentinel)


# ---- a6/a13: paged attention ---------------------------------------------------------------

def _paged_case(rng, B, Lq, Hq, Hkv, D, lens, shuffle=True):
    maxb = max((l + 15) // 16 for l in lens)
    P = B * maxb + 3
    kc = orc.f32_to_bf16(rng.normal(size=(P, Hkv, 16, D)))
    vc = orc.f32_to_bf16(rng.normal(size=(P, Hkv, 16, D)))
    perm = rng.permutation(P) if shuffle else np.arange(P)
    bt = perm[:B * maxb].reshape(B, maxb).astype(np.int32)
    q = orc.f32_to_bf16(rng.normal(size=(B, Lq, Hq, D)))
    return q, kc, vc, bt, np.array(lens, np.int32)


@pytest.mark.parametrize("B,Lq,Hq,Hkv,D,lens", [
    (1, 1, 32, 8, 128, [1]),
    (1, 1, 32, 8, 128, [2048]),
    (2, 1, 16, 8, 128, [37, 512]),
    (3, 1, 32, 8, 64, [130, 7, 16]),
    (4, 6, 32, 8, 128, [300, 1000, 64, 6]),
    (2, 1, 32, 4, 128, [4096, 100]),
    (1, 6, 32, 4, 128, [257]),
    (2, 2, 8, 8, 64, [3, 33]),
])
def test_paged_attention(B, Lq, Hq, Hkv, D, lens):
    rng = np.random.default_rng(B * 7 + Lq + D + sum(lens))
    q, kc, vc, bt, sl = _paged_case(rng, B, Lq, Hq, Hkv, D, lens)
    ref = orc.bf16_to_f32(orc.paged_attention(q, kc, vc, bt, sl))
    got = ops().paged_attention(bf(q), bf(kc), bf(vc), t(bt), t(sl), max(lens))
    got = orc.bf16_to_f32(to_np_bf(got))
    np.testing.assert_allclose(got, ref, atol=1e-2, rtol=1e-2)
    # a second call reuses the workspace counters (they must be left at zero)
    ws = ops().attention_workspace(B, Lq, Hq, Hkv, D, max(lens), DEV)
    o = ops()
    a1 = to_np_bf(o.paged_attention(bf(q), bf(kc), bf(vc), t(bt), t(sl), max(lens), workspace=ws))
    a2 = to_np_bf(o.paged_attention(bf(q), bf(kc), bf(vc), t(bt), t(sl), max(lens), workspace=ws))
    assert np.array_equal(a1, a2)


@pytest.mark.parametrize("B,Lq,Hq,Hkv,D,lens", [
    (1, 128, 32, 8, 128, [128]),         # a whole prompt in one chunk
    (1, 300, 32, 8, 128, [300]),         # a partial last query tile and key block
    (2, 200, 16, 8, 128, [200, 1000]),   # a chunk after 800 cached tokens
    (1, 512, 32, 8, 128, [512]),
    (2, 96, 16, 16, 64, [96, 130]),      # G = 1, D = 64
    (1, 40, 32, 4, 128, [2100]),         # G = 8, deep into the context
    (3, 17, 32, 8, 64, [17, 40, 333]),   # 68 rows: the smallest launch the kernel takes
    (2, 1000, 16, 4, 128, [1000, 1500]),  # 256 tiles: CTAs walk several tiles of mixed lengths
    (4, 256, 32, 32, 64, [256, 300, 512, 260]),  # G = 1, 256 tiles
])
def test_prefill_attention_tc(B, Lq, Hq, Hkv, D, lens):
    """Launches of more than 64 query rows run the tcgen05 prefill kernel (128-row tiles of
    tokens x GQA heads, S and O in tensor memory): against the oracle, against the mma.sync
    decode kernel on the same inputs (option attn_prefill_tc 0), and run to run."""
    from higgs_b200 import ffi
    rng = np.random.default_rng(B * 11 + Lq + D + sum(lens))
    q, kc, vc, bt, sl = _paged_case(rng, B, Lq, Hq, Hkv, D, lens)
    ref = orc.bf16_to_f32(orc.paged_attention(q, kc, vc, bt, sl))
    o = ops()
    args = (bf(q), bf(kc), bf(vc), t(bt), t(sl), max(lens))
    got = to_np_bf(o.paged_attention(*args))
    np.testing.assert_allclose(orc.bf16_to_f32(got), ref, atol=1e-2, rtol=1e-2)
    # one workspace twice: the tile counters in its first 4 KB are left at zero
    ws = o.attention_workspace(B, Lq, Hq, Hkv, D, max(lens), DEV)
    assert np.array_equal(got, to_np_bf(o.paged_attention(*args, workspace=ws)))
    assert np.array_equal(got, to_np_bf(o.paged_attention(*args, workspace=ws)))
    assert int(ws[:4096].count_nonzero()) == 0
    ffi.call("higgs_set_option", b"attn_prefill_tc", 0)
    try:
        old = to_np_bf(o.paged_attention(*args))
    finally:
        ffi.call("higgs_set_option", b"attn_prefill_tc", 1)
    np.testing.assert_allclose(orc.bf16_to_f32(got), orc.bf16_to_f32(old), atol=1e-2, rtol=1e-2)
    v = ctypes.c_int(-1)
    ffi.call("higgs_tc_error", ffi.ctx(0), ctypes.byref(v))
    assert v.value == 0


def test_paged_attention_golden(golden):
    g = golden
    got = ops().paged_attention(bf(g["at_q"]), bf(g["at_k"]), bf(g["at_v"]), t(g["at_bt"]),
                                t(g["at_sl"]), int(g["at_sl"].max()))
    np.testing.assert_allclose(orc.bf16_to_f32(to_np_bf(got)), orc.bf16_to_f32(g["at_out"]),
                               atol=1e-2, rtol=1e-2)


def test_contiguous_layout_strides():
    """A contiguous [B, Hkv, S_cap, D] cache (cache.rs:130-312) through page/head strides."""
    rng = np.random.default_rng(21)
    B, Hkv, Hq, D, S_cap = 2, 2, 8, 64, 256
    lens = [100, 256]
    k = orc.f32_to_bf16(rng.normal(size=(B, Hkv, S_cap, D)))
    v = orc.f32_to_bf16(rng.normal(size=(B, Hkv, S_cap, D)))
    q = orc.f32_to_bf16(rng.normal(size=(B, 1, Hq, D)))
    nb = S_cap // 16
    bt = np.array([[b * Hkv * nb + i for i in range(nb)] for b in range(B)], np.int32)
    # reference through explicit pages
    kp = k.reshape(B, Hkv, nb, 16, D).transpose(0, 2, 1, 3, 4).reshape(B * nb, Hkv, 16, D)
    vp = v.reshape(B, Hkv, nb, 16, D).transpose(0, 2, 1, 3, 4).reshape(B * nb, Hkv, 16, D)
    btp = np.arange(B * nb, dtype=np.int32).reshape(B, nb)
    ref = orc.bf16_to_f32(orc.paged_attention(q, kp, vp, btp, np.array(lens, np.int32)))
    o = ops()
    ws = o.attention_workspace(B, 1, Hq, Hkv, D, S_cap, DEV)
    out = torch.empty(B, 1, Hq, D, dtype=torch.bfloat16, device=DEV)
    from higgs_b200 import ffi
    qt, kt, vt = bf(q), bf(k), bf(v)
    btt, slt = t(bt), t(np.array(lens, np.int32))
    ffi.call("higgs_paged_attention", ffi.ctx(0), qt.data_ptr(), B, 1, Hq, Hkv, D, kt.data_ptr(),
             vt.data_ptr(), 16 * D, S_cap * D, btt.data_ptr(), nb, slt.data_ptr(), S_cap,
             float(1 / np.sqrt(D)), out.data_ptr(), ws.data_ptr(), ws.numel(),
             torch.cuda.current_stream().cuda_stream)
    np.testing.assert_allclose(orc.bf16_to_f32(to_np_bf(out)), ref, atol=1e-2, rtol=1e-2)


def test_cache_append_values_preserved(kat):
    """cache.rs:469-493 on the device: append 2 ones then 1 two, read back 1,1,2."""
    case = kat["cache_values_preserved"][0]
    D = 64
    kc = torch.zeros(1, 1, 16, D, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    inv = t(orc.rope_inv_freq(D, 10000.0))
    o = ops()
    pos0 = 0
    for app in case["appends"]:
        n = len(app)
        rows = np.zeros((n, 3 * D), np.float32)
        for i in range(n):
            rows[i, 2 * D:2 * D + 4] = app[i]  # the V head (no RoPE) carries the values
        o.qknorm_rope_kv_write(bf(orc.f32_to_bf16(rows)), 1, 1, D, None, None, 1e-6,
                               t(np.arange(pos0, pos0 + n, dtype=np.int32)), inv,
                               t(np.arange(pos0, pos0 + n, dtype=np.int64)), kc, vc)
        pos0 += n
    first = vc[0, 0, :pos0, 0].float().cpu().numpy()
    assert first.tolist() == case["expect_first"]


# ---- a14: TurboQuant ---------------------------------------------------------------------

def test_tq4_encode_bit_exact(golden):
    g = golden
    codes, scales = ops().tq4_encode(bf(g["tq_x"]), t(g["tq_signs"]))
    assert np.array_equal(codes.cpu().numpy(), g["tq_codes"])
    assert np.array_equal(scales.cpu().numpy().view(np.uint16), g["tq_scales"].view(np.uint16))
    rng = np.random.default_rng(31)
    signs = np.where(rng.random(128) < 0.5, -1, 1).astype(np.int8)
    x = orc.f32_to_bf16(np.concatenate([rng.normal(0, 1, size=(500, 128)),
                                        rng.normal(0, 300, size=(20, 128)),
                                        rng.normal(0, 1e-3, size=(20, 128))]))
    c_ref, s_ref = orc.tq4_encode(x, signs)
    c, s = ops().tq4_encode(bf(x), t(signs))
    assert np.array_equal(c.cpu().numpy(), c_ref)
    assert np.array_equal(s.cpu().numpy().view(np.uint16), s_ref.view(np.uint16))


def test_tq4_kv_write_bit_exact():
    rng = np.random.default_rng(32)
    T, Hq, Hkv, D = 4, 16, 8, 128
    qkv, qn, kn, pos, inv = _kvwrite_case(rng, T, Hq, Hkv, D, True)
    signs = np.where(rng.random(128) < 0.5, -1, 1).astype(np.int8)
    P = 3
    kcode = torch.zeros(P, Hkv, 16, 64, dtype=torch.uint8, device=DEV)
    vcode = torch.zeros_like(kcode)
    ksc = torch.zeros(P, Hkv, 16, dtype=torch.float16, device=DEV)
    vsc = torch.zeros_like(ksc)
    slots = np.array([5, 16 + 3, 2 * 16 + 15, 0], np.int64)
    o = ops()
    q = o.qknorm_rope_kv_write_tq4(bf(qkv), Hq, Hkv, bf(qn), bf(kn), 1e-6, t(pos), t(inv), t(slots),
                                   t(signs), kcode, ksc, vcode, vsc)
    # the K that was encoded: same device code path, bf16 cache
    kc = torch.zeros(P, Hkv, 16, D, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    q2 = o.qknorm_rope_kv_write(bf(qkv), Hq, Hkv, D, bf(qn), bf(kn), 1e-6, t(pos), t(inv), t(slots), kc, vc)
    assert torch.equal(q, q2)
    kcn, vcn = to_np_bf(kc), to_np_bf(vc)
    for i, sl in enumerate(slots):
        p, s = sl // 16, sl % 16
        ck, sk = orc.tq4_encode(kcn[p, :, s], signs)
        cv, sv = orc.tq4_encode(vcn[p, :, s], signs)
        assert np.array_equal(kcode[p, :, s].cpu().numpy(), ck)
        assert np.array_equal(vcode[p, :, s].cpu().numpy(), cv)
        assert np.array_equal(ksc[p, :, s].cpu().numpy().view(np.uint16), sk.view(np.uint16))
        assert np.array_equal(vsc[p, :, s].cpu().numpy().view(np.uint16), sv.view(np.uint16))


@pytest.mark.parametrize("variant", ["swap4", "swap6", "rows16", "p_lo"])
@pytest.mark.parametrize("B,Lq,Hq,Hkv,lens", [(1, 1, 32, 8, [1]), (2, 1, 32, 8, [2048, 77]),
                                             (3, 1, 16, 8, [16, 500, 33]), (2, 6, 32, 8, [300, 64]),
                                             (1, 1, 32, 4, [4096]), (2, 2, 16, 8, [40, 1000])])
def test_paged_attention_tq4(B, Lq, Hq, Hkv, lens, variant):
    """Against the oracle within the TurboQuant attention bound: launches of at most 4 query
    rows on the swapped-role kernel (4 or 6 ring stages, the default 4), or on the kernel with
    the query rows on the MMA's 16 rows (tq4_swap 0), with P x V on P's bf16 rounding, and
    that kernel with P's hi + lo halves (tq4_p_lo 1)."""
    from higgs_b200 import ffi
    swap, p_lo = {"swap4": (4, 0), "swap6": (6, 0), "rows16": (0, 0), "p_lo": (4, 1)}[variant]
    ffi.call("higgs_set_option", b"tq4_swap", swap)
    ffi.call("higgs_set_option", b"tq4_p_lo", p_lo)
    try:
        _tq4_attention_case(B, Lq, Hq, Hkv, lens)
    finally:
        ffi.call("higgs_set_option", b"tq4_p_lo", 0)  # the defaults
        ffi.call("higgs_set_option", b"tq4_swap", 4)


def _tq4_attention_case(B, Lq, Hq, Hkv, lens):
    rng = np.random.default_rng(B + Lq + Hq + sum(lens))
    signs = np.where(rng.random(128) < 0.5, -1, 1).astype(np.int8)
    maxb = max((l + 15) // 16 for l in lens)
    P = B * maxb + 2
    kx = orc.f32_to_bf16(rng.normal(size=(P * Hkv * 16, 128)))
    vx = orc.f32_to_bf16(rng.normal(size=(P * Hkv * 16, 128)))
    kcode, ksc = orc.tq4_encode(kx, signs)
    vcode, vsc = orc.tq4_encode(vx, signs)
    kcode, vcode = kcode.reshape(P, Hkv, 16, 64), vcode.reshape(P, Hkv, 16, 64)
    ksc, vsc = ksc.reshape(P, Hkv, 16), vsc.reshape(P, Hkv, 16)
    bt = rng.permutation(P)[:B * maxb].reshape(B, maxb).astype(np.int32)
    q = orc.f32_to_bf16(rng.normal(size=(B, Lq, Hq, 128)))
    sl = np.array(lens, np.int32)
    ref = orc.bf16_to_f32(orc.paged_attention_tq4(q, kcode, ksc, vcode, vsc, bt, sl, signs))
    got = ops().paged_attention_tq4(bf(q), t(kcode), t(ksc), t(vcode), t(vsc), t(bt), t(sl),
                                    max(lens), t(signs))
    got = orc.bf16_to_f32(to_np_bf(got))
    np.testing.assert_allclose(got, ref, atol=1.5e-2, rtol=1e-2)


# ---- a10/a15 ----------------------------------------------------------------------------------

def test_argmax(kat):
    o = ops()
    for case in kat["argmax"]:
        got = o.argmax(t(np.array(case["logits"], np.float32))).cpu().numpy()
        assert got.tolist() == case["expect"], case["src"]
    rng = np.random.default_rng(41)
    lg = rng.normal(size=(4, 151936)).astype(np.float32)
    lg[2, 100] = lg[2, 5000] = lg[2].max() + 1.0  # tie -> first
    lg[3, 150000] = lg[3, 7] = lg[3].max() + 1.0  # tie across cluster slices -> first
    assert np.array_equal(o.argmax(t(lg)).cpu().numpy(), orc.argmax(lg))


@pytest.mark.parametrize("V", [1, 3, 7, 31, 4099, 32001, 151937])
def test_argmax_edges(V):
    """Ragged rows (V % 4 != 0 leaves odd rows unaligned), NaN, -0/+0, all -inf."""
    o = ops()
    rng = np.random.default_rng(V)
    lg = rng.normal(size=(5, V)).astype(np.float32)
    lg[0, :] = np.nan                      # all NaN -> 0
    lg[1, :] = -np.inf                     # all -inf -> 0
    lg[1, V // 2] = np.nan                 # NaN never beats -inf
    lg[2, :] = -1.0
    lg[2, V - 1] = 0.0
    lg[2, V // 3] = -0.0                   # -0 == +0 -> the lower index
    lg[3, V - 1] = 1e30                    # winner in the ragged tail
    lg[4, rng.integers(0, V, size=max(1, V // 7))] = np.nan
    assert np.array_equal(o.argmax(t(lg)).cpu().numpy(), orc.argmax(lg))


def test_sample_bit_exact(golden):
    g = golden
    o = ops()
    got = o.sample(t(g["sm_logits"]), 0.7, t(g["sm_u"])).cpu().numpy()
    assert np.array_equal(got, g["sm_t07"])
    assert np.array_equal(o.sample(t(g["sm_logits"]), 0.0).cpu().numpy(), g["sm_t0"])
    rng = np.random.default_rng(42)
    lg = rng.normal(0, 1, size=(8, 151936)).astype(np.float32)
    u = rng.random(8).astype(np.float32)
    u[0] = 0.0
    u[1] = np.float32(0.99999994)
    for T in (0.7, 1.0, 0.05):
        assert np.array_equal(o.sample(t(lg), T, t(u)).cpu().numpy(), orc.sample(lg, T, u))


@pytest.mark.parametrize("V", [1, 5, 9, 1000, 32003])
def test_sample_small_and_ragged_vocab(V):
    """The row is spread over an 8-CTA cluster: slices that are empty (V < 8) or ragged."""
    o = ops()
    rng = np.random.default_rng(V)
    lg = rng.normal(0, 2, size=(3, V)).astype(np.float32)
    u = np.array([0.0, 0.5, 0.99999994], np.float32)
    for T in (0.7, 1.0):
        assert np.array_equal(o.sample(t(lg), T, t(u)).cpu().numpy(), orc.sample(lg, T, u))
    assert np.array_equal(o.sample(t(lg), 0.0).cpu().numpy(), orc.argmax(lg))


@pytest.mark.parametrize("T", [0.7, 0.0, 1.3])
def test_spec_accept_bit_exact(T, golden):
    o = ops()
    if T == 0.7:
        g = golden
        acc, toks = o.spec_accept(t(g["sa_tl"]), t(g["sa_dl"]), t(g["sa_dt"]), 0.7, t(g["sa_au"]),
                                  t(g["sa_su"]))
        assert np.array_equal(acc.cpu().numpy(), g["sa_acc"])
        assert np.array_equal(toks.cpu().numpy(), g["sa_toks"])
    rng = np.random.default_rng(int(T * 10) + 43)
    B, k, V = 4, 5, 151936
    tl = rng.normal(0, 1, size=(B, k + 1, V)).astype(np.float32)
    dl = (tl[:, :k] + rng.normal(0, 0.5, size=(B, k, V))).astype(np.float32)
    # drafts drawn from the draft distribution itself (the realistic case)
    dt = np.stack([orc.sample(dl[:, i], max(T, 0.7), rng.random(B).astype(np.float32))
                   for i in range(k)], axis=1).astype(np.int32)
    if T == 0.0:
        dt[:2] = np.argmax(tl[:2, :k], axis=-1)
    au = rng.random((B, k)).astype(np.float32)
    su = rng.random(B).astype(np.float32)
    acc_ref, toks_ref = orc.spec_accept(tl, dl, dt, T, au, su)
    acc, toks = o.spec_accept(t(tl), t(dl), t(dt), T, t(au), t(su))
    assert np.array_equal(acc.cpu().numpy(), acc_ref)
    assert np.array_equal(toks.cpu().numpy(), toks_ref)


def test_penalties(kat):
    o = ops()
    for case in kat["penalties"]:
        lg = t(np.array([case["logits"]], np.float32))
        hist = t(np.array([case["history"]], np.int32))
        lens = t(np.array([len(case["history"])], np.int32))
        o.apply_penalties(lg, hist, lens, case["rep"], case["freq"], case["pres"])
        np.testing.assert_allclose(lg.cpu().numpy()[0], case["expect"], atol=1e-5, err_msg=case["src"])
    rng = np.random.default_rng(44)
    V = 1000
    lg = rng.normal(size=(2, V)).astype(np.float32)
    hist = rng.integers(0, V, size=(2, 64)).astype(np.int32)
    lens = np.array([64, 10], np.int32)
    lt = t(lg.copy())
    o.apply_penalties(lt, t(hist), t(lens), 1.3, 0.2, 0.5)
    for bidx in range(2):
        ref = orc.apply_penalties(lg[bidx], hist[bidx, :lens[bidx]], 1.3, 0.2, 0.5)
        np.testing.assert_array_equal(lt.cpu().numpy()[bidx], ref)


def test_sample_filtered_kat_and_golden(kat, golden):
    """The reference's top-k / top-p / min-p tests (lib.rs:821-853, 1070-1115) and the golden
    oracle draws, bit for bit."""
    o = ops()
    us = np.linspace(0, 1, 32, endpoint=False, dtype=np.float32)
    for case in kat["sample_filtered"]:
        lg = np.repeat(np.array(case["logits"], np.float32), len(us), 0)
        got = set(o.sample_filtered(t(lg), case["temperature"], case["top_k"], case["top_p"],
                                    case["min_p"], t(us)).cpu().numpy().tolist())
        want = {case["expect"]} if case["expect"] is not None else set(case["allowed"])
        assert got == want, (case["src"], got, want)
    g = golden
    fl, fu = t(g["sf_logits"]), t(g["sf_u"])
    assert np.array_equal(o.sample_filtered(fl, 0.8, top_k=40, uniforms=fu).cpu().numpy(), g["sf_k40"])
    assert np.array_equal(o.sample_filtered(fl, 0.8, top_p=0.9, uniforms=fu).cpu().numpy(), g["sf_p09"])
    assert np.array_equal(o.sample_filtered(fl, 0.8, min_p=0.1, uniforms=fu).cpu().numpy(), g["sf_m01"])
    assert np.array_equal(o.sample_filtered(fl, 1.3, 100, 0.8, 0.02, uniforms=fu).cpu().numpy(),
                          g["sf_all"])


@pytest.mark.parametrize("V,T,top_k,top_p,min_p", [
    (151936, 0.7, 50, 1.0, 0.0), (151936, 0.7, 0, 0.9, 0.0), (151936, 1.0, 0, 1.0, 0.05),
    (151936, 0.8, 40, 0.95, 0.02), (128256, 1.5, 1, 1.0, 0.0), (128256, 0.6, 0, 0.0, 0.0),
    (4099, 2.0, 4098, 0.999, 0.0), (163840, 1.0, 1000, 0.5, 0.001), (7, 1.0, 3, 0.7, 0.2)])
def test_sample_filtered_bit_exact(V, T, top_k, top_p, min_p):
    """Tokens equal the oracle's for identical uniforms over many rows: vocabularies of the
    benchmark models and the largest supported, ties at the filter boundaries, extreme
    uniforms, flat rows (every token within top_p) and peaked ones."""
    o = ops()
    rng = np.random.default_rng(V + top_k)
    B = 24
    lg = rng.normal(0, 2, size=(B, V)).astype(np.float32)
    lg[1] = 0.25                                    # flat row
    lg[2, : min(V, 64)] = lg[2].max()               # a block of tied maxima
    lg[3, rng.integers(0, V, size=max(1, V // 50))] = lg[3].max() - 0.5  # ties inside the set
    lg[4, V - 1] = lg[4].max() + 30.0               # one dominant token at the end
    u = rng.random(B).astype(np.float32)
    u[0], u[5] = 0.0, np.float32(0.99999994)
    got = o.sample_filtered(t(lg), T, top_k, top_p, min_p, t(u)).cpu().numpy()
    ref = orc.sample_filtered(lg, T, top_k, top_p, min_p, u)
    assert np.array_equal(got, ref), np.nonzero(got != ref)[0].tolist()


def test_sample_filtered_rejects_oversized_vocab():
    from higgs_b200 import ffi
    o = ops()
    lg = t(np.zeros((1, 163841), np.float32))
    with pytest.raises(ffi.HiggsError, match="163840"):
        o.sample_filtered(lg, 1.0, 5, uniforms=t(np.zeros(1, np.float32)))


@pytest.mark.parametrize("V,T,top_n", [(151936, 0.7, 5), (128256, 0.0, 20), (1000, 1.3, 0),
                                       (7, 1.0, 10)])
def test_logprobs_match_oracle(V, T, top_n, golden):
    o = ops()
    g = golden
    lp, ids, tl = o.logprobs(t(g["sf_logits"]), 0.7, t(g["lp_tokens"]), 5)
    assert np.array_equal(ids.cpu().numpy(), g["lp_ids"])
    np.testing.assert_allclose(lp.cpu().numpy(), g["lp_lp"], rtol=0, atol=1e-6)
    np.testing.assert_allclose(tl.cpu().numpy(), g["lp_top"], rtol=0, atol=1e-6)
    rng = np.random.default_rng(V)
    lg = rng.normal(0, 3, size=(6, V)).astype(np.float32)
    lg[1, : min(V, 30)] = lg[1].max()  # tied top values
    toks = rng.integers(0, V, size=6).astype(np.int32)
    toks[0] = V  # out of range -> -inf
    lp, ids, tl = o.logprobs(t(lg), T, t(toks), top_n)
    rlp, rids, rtl = orc.logprobs(lg, T, toks, top_n)
    assert np.array_equal(ids.cpu().numpy(), rids)
    np.testing.assert_allclose(lp.cpu().numpy(), rlp, rtol=0, atol=1e-6)
    np.testing.assert_allclose(tl.cpu().numpy(), rtl, rtol=0, atol=1e-6)


def test_token_mask_bit_exact(golden):
    o = ops()
    g = golden
    lg = t(g["sf_logits"].copy())
    o.apply_token_mask(lg, t(g["mk_bits"].view(np.int32)))
    assert np.array_equal(lg.cpu().numpy().view(np.uint32), g["mk_out"].view(np.uint32))


# ---- stream-K GEMV with fused RMSNorm (decode batches) -----------------------------------

@pytest.mark.parametrize("M,K,N,norm", [(1, 256, 16, False), (1, 4096, 6144, True), (3, 2048, 512, True),
                                        (8, 4096, 1024, True), (5, 12288, 256, False),
                                        (2, 1024, 4096 + 16, False), (1, 4096, 151936, True),
                                        (1, 8192, 512, True)])
def test_rmsnorm_qlinear_sk(M, K, N, norm):
    rng = np.random.default_rng(M + K + N)
    q, s, b = qweights(rng, N, K)
    h = orc.f32_to_bf16(rng.normal(0, 1, size=(M, K)))
    nw = orc.f32_to_bf16(rng.uniform(0.5, 1.5, size=K))
    x = orc.rmsnorm(h, nw, 1e-6)[0] if norm else h
    yb_ref, yf_ref = orc.qmatmul(x, q, s, b, want_f32=True)
    o = ops()
    ws = o.sk_workspace(M, K, N, DEV)
    yf = o.rmsnorm_quantized_matmul(bf(h), bf(nw) if norm else None, 1e-6, t(q.view(np.int32)), bf(s),
                                    bf(b), out_f32=True, workspace=ws).cpu().numpy()
    scale = np.abs(yf_ref).max()
    # the fused norm may round an input element 1 ulp differently from the oracle's norm
    tol = 3e-3 if norm else 1e-3
    np.testing.assert_allclose(yf, yf_ref, rtol=tol, atol=tol * 0.1 * scale + 1e-6)
    # deterministic, and the workspace is left reusable
    y1 = o.rmsnorm_quantized_matmul(bf(h), bf(nw) if norm else None, 1e-6, t(q.view(np.int32)), bf(s),
                                    bf(b), workspace=ws)
    y2 = o.rmsnorm_quantized_matmul(bf(h), bf(nw) if norm else None, 1e-6, t(q.view(np.int32)), bf(s),
                                    bf(b), workspace=ws)
    assert torch.equal(y1, y2)
    # bf16 output: within one bf16 rounding of the f32 reference, plus the f32 noise near zero
    np.testing.assert_allclose(orc.bf16_to_f32(to_np_bf(y1)), yf_ref, rtol=2 ** -7,
                               atol=tol * 0.1 * scale + 1e-6)


@pytest.mark.parametrize("M,norm", [(1, True), (4, False), (8, True)])
def test_rmsnorm_gate_up_swiglu_sk(M, norm):
    rng = np.random.default_rng(70 + M)
    K, N = 2048, 768
    qg, sg, bg = qweights(rng, N, K)
    qu, su, bu = qweights(rng, N, K)
    h = orc.f32_to_bf16(rng.normal(size=(M, K)))
    nw = orc.f32_to_bf16(rng.uniform(0.5, 1.5, size=K))
    x = orc.rmsnorm(h, nw, 1e-6)[0] if norm else h
    ref = orc.silu_mul(orc.qmatmul(x, qg, sg, bg), orc.qmatmul(x, qu, su, bu))
    got = to_np_bf(ops().rmsnorm_gate_up_swiglu(bf(h), bf(nw) if norm else None, 1e-6,
                                                t(qg.view(np.int32)), bf(sg), bf(bg),
                                                t(qu.view(np.int32)), bf(su), bf(bu)))
    np.testing.assert_allclose(orc.bf16_to_f32(got), orc.bf16_to_f32(ref), atol=3e-3, rtol=3e-2)
    assert np.percentile(bf_ulps(got, ref), 99) <= 3


# ---- fused decode attention (norm + RoPE + append + SDPA) --------------------------------

@pytest.mark.parametrize("B,Lq,Hq,Hkv,D,qknorm,lens", [
    (1, 1, 32, 8, 128, True, [2048]),
    (1, 1, 32, 8, 128, True, [17]),
    (3, 1, 16, 8, 128, True, [1, 16, 300]),
    (2, 1, 32, 8, 64, False, [129, 4000]),
    (2, 6, 32, 8, 128, True, [700, 6]),
    (1, 2, 32, 4, 128, True, [33]),
])
def test_fused_attention_equals_unfused(B, Lq, Hq, Hkv, D, qknorm, lens):
    rng = np.random.default_rng(B * 100 + Lq + D + sum(lens))
    T = B * Lq
    nh = Hq + 2 * Hkv
    qkv = orc.f32_to_bf16(rng.normal(size=(T, nh * D)))
    qn = orc.f32_to_bf16(rng.uniform(0.5, 1.5, size=D)) if qknorm else None
    kn = orc.f32_to_bf16(rng.uniform(0.5, 1.5, size=D)) if qknorm else None
    inv = orc.rope_inv_freq(D, 1000000.0)
    maxb = max((n + 15) // 16 for n in lens)
    P = B * maxb + 2
    bt = rng.permutation(P)[:B * maxb].reshape(B, maxb).astype(np.int32)
    pos = np.array([[n - Lq + tq for tq in range(Lq)] for n in lens], np.int32).reshape(-1)
    slots = np.array([bt[b, p // 16] * 16 + p % 16 for b in range(B) for p in pos[b * Lq:(b + 1) * Lq]],
                     np.int64)
    kc0 = orc.f32_to_bf16(rng.normal(size=(P, Hkv, 16, D)))
    vc0 = orc.f32_to_bf16(rng.normal(size=(P, Hkv, 16, D)))
    sl = np.array(lens, np.int32)
    o = ops()
    # unfused: kv write then attention
    kc1, vc1 = bf(kc0), bf(vc0)
    q = o.qknorm_rope_kv_write(bf(qkv), Hq, Hkv, D, None if qn is None else bf(qn),
                               None if kn is None else bf(kn), 1e-6, t(pos), t(inv), t(slots), kc1, vc1)
    ref = o.paged_attention(q.view(B, Lq, Hq, D), kc1, vc1, t(bt), t(sl), max(lens))
    # fused
    kc2, vc2 = bf(kc0), bf(vc0)
    got = o.fused_attention(bf(qkv), Hq, Hkv, D, None if qn is None else bf(qn),
                            None if kn is None else bf(kn), 1e-6, t(pos), t(inv), t(slots), kc2, vc2,
                            t(bt), t(sl), max(lens), Lq=Lq)
    assert torch.equal(kc1, kc2) and torch.equal(vc1, vc2)  # identical cache append
    np.testing.assert_allclose(got.float().cpu().numpy(), ref.float().cpu().numpy(), atol=1e-2, rtol=1e-2)
    # and against the oracle on the updated cache
    ref_o = orc.paged_attention(to_np_bf(q).reshape(B, Lq, Hq, D), to_np_bf(kc2), to_np_bf(vc2), bt, sl)
    np.testing.assert_allclose(got.float().cpu().numpy(), orc.bf16_to_f32(ref_o), atol=1e-2, rtol=1e-2)


# ---- a1 matrix form: tcgen05 path for M >= 17 ---------------------------------------------------

def _tc_matmul(path, x, q, s, b, **kw):
    """quantized_matmul without a workspace (one CTA per tile, "tiles") or through the
    workspace entry, which splits K over the CTAs of small tile counts ("ws")."""
    o = ops()
    if path == "tiles":
        return o.quantized_matmul(x, q, s, b, **kw)
    return o.rmsnorm_quantized_matmul(x, None, 0.0, q, s, b, **kw)


@pytest.mark.parametrize("path", ["tiles", "ws"])
@pytest.mark.parametrize("M,K,N", [(17, 256, 128), (20, 4096, 1024), (32, 4096, 4096), (33, 2048, 256),
                                   (64, 12288, 512), (100, 1024, 384), (300, 512, 256), (40, 768, 6144)])
def test_qgemm_tc_vs_oracle(M, K, N, path):
    """M >= 17 rows run on the tensor cores with weights dequantized to bf16 (MLX's qmm form)."""
    rng = np.random.default_rng(M * 7 + K + N)
    q, s, b = qweights(rng, N, K)
    x = orc.f32_to_bf16(rng.normal(0, 1, size=(M, K)))
    yb_ref, yf_ref = orc.qmatmul_dq(x, q, s, b, want_f32=True)
    qt, st_, bt_ = t(q.view(np.int32)), bf(s), bf(b)
    yf = _tc_matmul(path, bf(x), qt, st_, bt_, out_f32=True).cpu().numpy()
    scale = np.abs(yf_ref).max()
    np.testing.assert_allclose(yf, yf_ref, rtol=1e-3, atol=1e-4 * scale + 1e-6)
    yb = to_np_bf(_tc_matmul(path, bf(x), qt, st_, bt_))
    # outputs that are small next to the row scale come out of cancellation, where the f32
    # summation order (tensor core vs sequential) moves many of their low bits
    big = np.abs(yf_ref) >= 1e-2 * scale
    assert bf_ulps(yb, yb_ref)[big].max() <= 1
    assert np.all(np.abs(orc.bf16_to_f32(yb) - orc.bf16_to_f32(yb_ref))
                  <= 2e-3 * scale + np.abs(yf_ref) * 2.0 ** -7)
    # residual epilogue: one ulp of y may survive the add, bounded by the operands' magnitude
    res = orc.f32_to_bf16(rng.normal(0, 1, size=(M, N)))
    yr = to_np_bf(_tc_matmul(path, bf(x), qt, st_, bt_, residual=bf(res)))
    ref_r = orc.f32_to_bf16(orc.bf16_to_f32(yb_ref) + orc.bf16_to_f32(res))
    mag = np.maximum(np.abs(orc.bf16_to_f32(yb_ref)), np.abs(orc.bf16_to_f32(res)))
    assert np.all(np.abs(orc.bf16_to_f32(yr) - orc.bf16_to_f32(ref_r)) <= mag * 2.0 ** -6 + 2e-3 * scale)


@pytest.mark.parametrize("path", ["tiles", "ws"])
@pytest.mark.parametrize("M,K,N", [(17, 1024, 256), (48, 4096, 1536), (130, 512, 128), (32, 4096, 3072)])
def test_qgemm_tc_swiglu_vs_oracle(M, K, N, path):
    rng = np.random.default_rng(M + K + N)
    qg, sg, bg = qweights(rng, N, K)
    qu, su, bu = qweights(rng, N, K)
    x = orc.f32_to_bf16(rng.normal(0, 1, size=(M, K)))
    ref = orc.silu_mul(orc.qmatmul_dq(x, qg, sg, bg), orc.qmatmul_dq(x, qu, su, bu))
    args = (bf(x), t(qg.view(np.int32)), bf(sg), bf(bg), t(qu.view(np.int32)), bf(su), bf(bu))
    if path == "tiles":
        got = to_np_bf(ops().gate_up_swiglu(*args))
    else:
        got = to_np_bf(ops().rmsnorm_gate_up_swiglu(args[0], None, 0.0, *args[1:]))
    sa = np.abs(orc.bf16_to_f32(ref)).max()
    np.testing.assert_allclose(orc.bf16_to_f32(got), orc.bf16_to_f32(ref), atol=2e-3 * sa, rtol=2e-2)
    assert np.mean(bf_ulps(got, ref) <= 1) > 0.99


def test_qgemm_tc_shared_workspace():
    """One zeroed workspace serves matmuls of several shapes back to back (tile counters reset
    themselves), and the split-tile sums are deterministic."""
    import torch
    o = ops()
    rng = np.random.default_rng(5)
    shapes = [(32, 4096, 6144), (17, 12288, 4096), (64, 4096, 1024), (24, 1024, 128)]
    ws = o.sk_workspace(64, 12288, 2 * 6144, "cuda")
    outs = []
    for rep in range(2):
        for M, K, N in shapes:
            r2 = np.random.default_rng(M + K + N)
            q, s, b = qweights(r2, N, K)
            x = orc.f32_to_bf16(r2.normal(0, 1, size=(M, K)))
            y = o.rmsnorm_quantized_matmul(bf(x), None, 0.0, t(q.view(np.int32)), bf(s), bf(b),
                                           out_f32=True, workspace=ws)
            if rep == 0:
                outs.append(y)
                yf_ref = orc.qmatmul_dq(x, q, s, b, want_f32=True)[1]
                np.testing.assert_allclose(y.cpu().numpy(), yf_ref, rtol=1e-3,
                                           atol=1e-4 * np.abs(yf_ref).max() + 1e-6)
            else:
                assert torch.equal(y, outs[shapes.index((M, K, N))])
    torch.cuda.synchronize()
    assert int(ws[:65536].count_nonzero()) == 0


def test_qgemm_tc_no_timeouts():
    """No bounded mbarrier wait of the tensor-core kernel gave up in the tests above."""
    from higgs_b200 import ffi
    v = ctypes.c_int(-1)
    ffi.call("higgs_tc_error", ffi.ctx(0), ctypes.byref(v))
    assert v.value == 0


# ---- decode chain (one-token GEMVs of a block in one persistent launch) ------------------------

@pytest.mark.parametrize("H,Hd,F,Nq,Nkv", [(4096, 4096, 12288, 4096, 1024), (2048, 2048, 8192, 2048, 512),
                                           (512, 512, 768, 512, 256)])
def test_decode_chain_entry_equals_separate_ops(H, Hd, F, Nq, Nkv):
    """higgs_decode_chain's four phases equal the separate one-token ops on the register-fed
    single-token GEMV (gemv_tma off) bit for bit -- same K split, same summation order: h +=
    o_proj(attn); act = swiglu(gate/up(norm(h))); h += down(act); qkv = q|k|v(norm(h)) as three
    row segments vs one concatenated matrix."""
    _decode_chain_vs_ops(H, Hd, F, Nq, Nkv)


def _decode_chain_vs_ops(H, Hd, F, Nq, Nkv):
    o = ops()
    rng = np.random.default_rng(H + F)

    def wq(N, K):
        q, s, b = orc.w4_quantize(rng.normal(0, 0.02, size=(N, K)).astype(np.float32))
        return t(q.view(np.int32)), bf(s), bf(b)
    Wo, Wg, Wu, Wd = wq(H, Hd), wq(F, H), wq(F, H), wq(H, F)
    Wq, Wk, Wv = wq(Nq, H), wq(Nkv, H), wq(Nkv, H)
    ln_post = bf(orc.f32_to_bf16(rng.uniform(0.5, 1.5, H)))
    ln_in = bf(orc.f32_to_bf16(rng.uniform(0.5, 1.5, H)))
    attn = bf(orc.f32_to_bf16(rng.normal(0, 1, Hd)))
    h0 = bf(orc.f32_to_bf16(rng.normal(0, 1, H)))
    eps = 1e-6
    # separate launches
    h1 = o.quantized_matmul(attn[None], *Wo, residual=h0[None])
    act = o.rmsnorm_gate_up_swiglu(h1, ln_post, eps, *Wg, *Wu)
    h2 = o.quantized_matmul(act, *Wd, residual=h1)
    cat = tuple(torch.cat([a, b_, c], 0) for a, b_, c in zip(Wq, Wk, Wv))
    qkv_ref = o.rmsnorm_quantized_matmul(h2, ln_in, eps, *cat)
    # one chain launch
    h = h0.clone()
    act_c = torch.zeros(F, dtype=torch.bfloat16, device=DEV)
    qkv = torch.zeros(Nq + 2 * Nkv, dtype=torch.bfloat16, device=DEV)
    bars = torch.zeros(4 * 64, dtype=torch.int32, device=DEV)
    ph = [o.chain_gemv(attn, *Wo, y=h, residual=h),
          o.chain_gemv(h, *Wg, norm_w=ln_post, up=Wu, y=act_c),
          o.chain_gemv(act_c, *Wd, y=h, residual=h),
          o.chain_gemv(h, None, None, None, norm_w=ln_in, segments=[Wq, Wk, Wv], y=qkv)]
    for rep in range(2):  # twice: the barrier counters are left zeroed for the next launch
        h.copy_(h0)
        o.decode_chain(ph, eps, bars, DEV)
        torch.cuda.synchronize()
        assert torch.equal(act_c, act[0]), rep
        assert torch.equal(h, h2[0]), rep
        assert torch.equal(qkv, qkv_ref[0]), rep
        assert int(bars.count_nonzero()) == 0
    # and the last phase against the oracle's vector-form restatement on the same input
    wcat = (cat[0].cpu().numpy().view(np.uint32), to_np_bf(cat[1]), to_np_bf(cat[2]))
    ref = orc.qmatmul(orc.rmsnorm(to_np_bf(h2), to_np_bf(ln_in), eps)[0], *wcat)
    np.testing.assert_allclose(orc.bf16_to_f32(to_np_bf(qkv)), orc.bf16_to_f32(ref[0]), atol=2e-2,
                               rtol=1e-2)


def test_decode_chain_rejects_bad_phases():
    from higgs_b200 import ffi
    o = ops()
    x = torch.zeros(300, dtype=torch.bfloat16, device=DEV)
    w = torch.zeros(16, 300 // 8, dtype=torch.int32, device=DEV)
    s = torch.zeros(16, 4, dtype=torch.bfloat16, device=DEV)
    y = torch.zeros(16, dtype=torch.bfloat16, device=DEV)
    bars = torch.zeros(4 * 64, dtype=torch.int32, device=DEV)
    with pytest.raises(ffi.HiggsError, match="limits"):
        o.decode_chain([o.chain_gemv(x, w, s, s, y=y)], 1e-6, bars, DEV)  # K not a multiple of 256


@pytest.mark.parametrize("M_shape", [(4096, 4096, False, None), (4096, 12288, False, None),
                                     (12288, 4096, True, None), (151936, 4096, False, None),
                                     (2048, 2048, False, None), (6144, 4096, False, (4096, 1024, 1024))])
def test_qgemv_tma_vs_oracle(M_shape):
    """The TMA-fed single-token GEMV (option gemv_tma, off by default) against the oracle's
    vector form: plain, SwiGLU, fused RMSNorm, q|k|v row segments, the LM head's width."""
    from higgs_b200 import ffi
    o = ops()
    N, K, swiglu, segs = M_shape
    rng = np.random.default_rng(N + K)

    def wq(n):
        q, s, b = orc.w4_quantize(rng.normal(0, 0.02, size=(n, K)).astype(np.float32))
        return q, s, b
    x = orc.f32_to_bf16(rng.normal(0, 1, size=(1, K)))
    nw = orc.f32_to_bf16(rng.uniform(0.5, 1.5, K))
    ffi.call("higgs_set_option", b"gemv_tma", 1)
    try:
        if swiglu:
            g_, u_ = wq(N), wq(N)
            got = o.gate_up_swiglu(bf(x), t(g_[0].view(np.int32)), bf(g_[1]), bf(g_[2]),
                                   t(u_[0].view(np.int32)), bf(u_[1]), bf(u_[2]))
            ref = orc.silu_mul(orc.qmatmul(x, *g_), orc.qmatmul(x, *u_))
            np.testing.assert_allclose(orc.bf16_to_f32(to_np_bf(got)), orc.bf16_to_f32(ref), atol=2e-2, rtol=1e-2)
        elif segs:
            parts = [wq(n) for n in segs]
            cat = [np.concatenate([p_[i] for p_ in parts]) for i in range(3)]
            got = o.rmsnorm_quantized_matmul(bf(x), bf(nw), 1e-6, t(cat[0].view(np.int32)), bf(cat[1]),
                                             bf(cat[2]), out_f32=True)
            xn = orc.rmsnorm(x, nw, 1e-6)[0]
            ref = orc.qmatmul(xn, *cat, want_f32=True)[1]
            np.testing.assert_allclose(got.cpu().numpy(), ref, rtol=1e-3, atol=1e-4 * np.abs(ref).max())
        else:
            q, s, b = wq(N)
            got = o.quantized_matmul(bf(x), t(q.view(np.int32)), bf(s), bf(b), out_f32=True)
            ref = orc.qmatmul(x, q, s, b, want_f32=True)[1]
            np.testing.assert_allclose(got.cpu().numpy(), ref, rtol=1e-3, atol=1e-4 * np.abs(ref).max())
        v = ctypes.c_int(-1)
        ffi.call("higgs_tc_error", ffi.ctx(0), ctypes.byref(v))
        assert v.value == 0
    finally:
        ffi.call("higgs_set_option", b"gemv_tma", 0)
