"""GPU: the mixture-of-experts path (router top-k, routing plan, grouped W4 experts,
combine, and the Qwen3-MoE decode step) against the CPU oracle.

Bars: expert indices and the routing plan bit-exact; scores within f32 summation-order
noise; the combine bit-exact given the same expert outputs; grouped expert GEMVs
within 1 bf16 ulp of the per-expert quantized_matmul (the reference's own check,
qwen3_next.rs:2151-2206) and of the oracle; the model within the north-star logits
tolerance.
"""
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


def bf_ulps(a, b):
    def key(x):
        x = x.astype(np.int32)
        return np.where(x & 0x8000, -(x & 0x7FFF), x)
    return np.abs(key(a) - key(b))


def experts(rng, E, N, K, sd=0.02):
    q, s, b = orc.w4_quantize(rng.normal(0, sd, size=(E * N, K)).astype(np.float32))
    return q.reshape(E, N, K // 8), s.reshape(E, N, K // 64), b.reshape(E, N, K // 64)


def dev3(w):
    q, s, b = (np.ascontiguousarray(a) for a in w)
    return t(q.view(np.int32)), bf(s), bf(b)


def decode_plan(plan, T, E, k):
    raw = plan.cpu().numpy().view(np.int32)
    P = T * k
    mi = P // 8 + min(E, P) + 1
    n_items = int(raw[0])
    items = raw[4:4 + 4 * mi].reshape(mi, 4)[:n_items]
    sorted_ = raw[4 + 4 * mi:4 + 4 * mi + P]
    counts = raw[4 + 4 * mi + P:4 + 4 * mi + P + E]
    return raw[:4], items, sorted_, counts


@pytest.mark.parametrize("T,E,k,norm,dtype", [(1, 128, 8, True, "bf16"), (37, 128, 8, False, "bf16"),
                                              (5, 60, 3, True, "f32"), (64, 512, 10, True, "bf16"),
                                              (3, 1024, 32, False, "f32"), (9, 16, 1, True, "bf16")])
def test_route_topk_matches_oracle(T, E, k, norm, dtype):
    rng = np.random.default_rng(T * 7 + E + k)
    lg = rng.normal(0, 1, size=(T, E)).astype(np.float32)
    lg[0, 3] = lg[0, 9] = lg[0].max() + 0.5          # tie at the top -> lower index first
    if T > 2:
        lg[2, :] = np.round(lg[2] * 4) / 4            # many exact ties
    if dtype == "bf16":
        lbits = orc.f32_to_bf16(lg)
        lg = orc.bf16_to_f32(lbits)
        gl = bf(lbits)
    else:
        gl = t(lg)
    idx_ref, sc_ref = orc.moe_route_topk(lg, k, norm)
    plan = ops().moe_plan(T, E, k, DEV)
    idx, sc = ops().moe_route_topk(gl, k, norm, plan)
    torch.cuda.synchronize()
    assert np.array_equal(idx.cpu().numpy(), idx_ref)
    np.testing.assert_allclose(sc.cpu().numpy(), sc_ref, rtol=2e-6, atol=1e-9)
    hdr, items, sorted_, counts = decode_plan(plan, T, E, k)
    P = T * k
    assert hdr.tolist()[1:] == [P, E, k]
    flat = idx_ref.reshape(-1)
    assert np.array_equal(counts, np.bincount(flat, minlength=E))
    # pairs grouped by expert, ascending inside an expert: a stable sort by expert
    assert np.array_equal(sorted_, np.argsort(flat, kind="stable"))
    covered = np.concatenate([sorted_[s0:s0 + n] for _, s0, n, _ in items])
    assert np.array_equal(np.sort(covered), np.arange(P))
    for e, s0, n, _ in items:
        assert 1 <= n <= 8 and np.all(flat[sorted_[s0:s0 + n]] == e)


def test_gather_qmm_matches_per_expert():
    """The reference's check (qwen3_next.rs:2151-2206): gather_qmm with expert 2 of 4
    equals quantized_matmul on that expert's slice."""
    rng = np.random.default_rng(3)
    E, N, K = 4, 64, 256
    w = experts(rng, E, N, K)
    x = orc.f32_to_bf16(rng.uniform(0, 1, size=(1, K)))
    lg = np.full((1, E), -1.0, np.float32)
    lg[0, 2] = 1.0
    plan = ops().moe_plan(1, E, 1, DEV)
    ops().moe_route_topk(t(lg), 1, False, plan)
    got = to_np_bf(ops().moe_grouped_w4(bf(x), 1, plan, *dev3(w)))
    q, s, b = (a[2] for a in w)
    per = to_np_bf(ops().quantized_matmul(bf(x), t(np.ascontiguousarray(q).view(np.int32)),
                                          bf(np.ascontiguousarray(s)), bf(np.ascontiguousarray(b))))
    assert bf_ulps(got, per).max() <= 1
    assert bf_ulps(got, orc.qmatmul(x, q, s, b)).max() <= 1


@pytest.mark.parametrize("T,E,k,H,F,skew", [(1, 128, 8, 2048, 768, False), (32, 128, 8, 2048, 768, False),
                                            (5, 16, 4, 512, 256, False), (40, 8, 2, 512, 256, True)])
def test_grouped_experts_match_oracle(T, E, k, H, F, skew):
    """gate/up SwiGLU then down over the plan, against the oracle's per-expert loop; skew
    routes most tokens to one expert (several 8-pair work items for it)."""
    rng = np.random.default_rng(T + E + H)
    wg, wu, wd = experts(rng, E, F, H), experts(rng, E, F, H), experts(rng, E, H, F)
    x = orc.f32_to_bf16(rng.normal(0, 1, size=(T, H)))
    lg = rng.normal(0, 1, size=(T, E)).astype(np.float32)
    if skew:
        lg[:, 5] += 10.0
    idx_ref, _ = orc.moe_route_topk(lg, k, True)
    plan = ops().moe_plan(T, E, k, DEV)
    ops().moe_route_topk(t(lg), k, True, plan)
    act = ops().moe_grouped_w4(bf(x), k, plan, *dev3(wg), *dev3(wu))
    y = to_np_bf(ops().moe_grouped_w4(act, k, plan, *dev3(wd), x_per_pair=True))
    torch.cuda.synchronize()
    # the down projection against the oracle on the GPU's own activations (isolates each GEMV)
    act_np = to_np_bf(act)
    g_ref = np.zeros_like(act_np)
    y_ref = np.zeros_like(y)
    flat = idx_ref.reshape(-1)
    for e in np.unique(flat):
        pr = np.nonzero(flat == e)[0]
        xe = np.ascontiguousarray(x[pr // k])
        g_ref[pr] = orc.silu_mul(orc.qmatmul(xe, wg[0][e], wg[1][e], wg[2][e]),
                                 orc.qmatmul(xe, wu[0][e], wu[1][e], wu[2][e]))
        y_ref[pr] = orc.qmatmul(np.ascontiguousarray(act_np[pr]), wd[0][e], wd[1][e], wd[2][e])
    # grouped == the plain per-expert GPU kernel up to the K-split summation order (the two
    # launches may split K over a different number of warps); the plain kernel is held to
    # its vector form, which the grouped kernel always uses
    from higgs_b200 import ffi
    ffi.call("higgs_set_option", b"gemm_tc", 0)
    try:
        sa = np.abs(orc.bf16_to_f32(act_np)).max()
        for e in np.unique(flat)[:16]:
            pr = np.nonzero(flat == e)[0]
            xe = bf(np.ascontiguousarray(x[pr // k]))
            dense = to_np_bf(ops().gate_up_swiglu(xe, *dev3([a[e] for a in wg]), *dev3([a[e] for a in wu])))
            np.testing.assert_allclose(orc.bf16_to_f32(act_np[pr]), orc.bf16_to_f32(dense), atol=5e-4 * sa,
                                       rtol=8e-3, err_msg=f"expert {e}")
    finally:
        ffi.call("higgs_set_option", b"gemm_tc", 1)
    # and the oracle, bounded relative to each row's scale: outputs near zero come out
    # of cancellation, where f32 summation order moves many of their low bits
    sa = np.abs(orc.bf16_to_f32(g_ref)).max()
    np.testing.assert_allclose(orc.bf16_to_f32(act_np), orc.bf16_to_f32(g_ref), atol=2e-3 * sa,
                               rtol=2e-2)
    sy = np.abs(orc.bf16_to_f32(y_ref)).max()
    np.testing.assert_allclose(orc.bf16_to_f32(y), orc.bf16_to_f32(y_ref), atol=2e-3 * sy, rtol=2e-2)
    # and the whole expert block against the oracle end to end
    full = orc.moe_experts(x, idx_ref, wg, wu, wd)
    np.testing.assert_allclose(orc.bf16_to_f32(y), orc.bf16_to_f32(full), atol=2e-3, rtol=2e-2)


@pytest.mark.parametrize("T,k,H", [(1, 8, 2048), (7, 3, 512), (32, 8, 4096)])
def test_combine_bit_exact(T, k, H):
    rng = np.random.default_rng(T * k)
    y = orc.f32_to_bf16(rng.normal(0, 0.1, size=(T * k, H)))
    sc = rng.dirichlet(np.ones(k), size=T).astype(np.float32)
    h = orc.f32_to_bf16(rng.normal(0, 1, size=(T, H)))
    ref = orc.moe_combine(y, sc, h)
    hg = bf(h)
    ops().moe_combine(bf(y), t(sc), hg)
    assert np.array_equal(to_np_bf(hg), ref)


def test_route_rejects_bad_shapes():
    from higgs_b200 import ffi
    lib = ffi.load()
    z = torch.zeros(16, dtype=torch.float32, device=DEV)
    i = torch.zeros(16, dtype=torch.int32, device=DEV)
    # k > E, E > 1024, T*k > 65536: rejected on the host before any launch
    assert lib.higgs_moe_route_topk(ffi.ctx(0), z.data_ptr(), ffi.DTYPE_F32, 1, 4, 5, 1, i.data_ptr(),
                                    z.data_ptr(), None, 0, None) == -1
    assert lib.higgs_moe_route_topk(ffi.ctx(0), z.data_ptr(), ffi.DTYPE_F32, 1, 2048, 8, 1, i.data_ptr(),
                                    z.data_ptr(), None, 0, None) == -1
    assert lib.higgs_moe_route_topk(ffi.ctx(0), z.data_ptr(), ffi.DTYPE_F32, 9000, 128, 8, 1,
                                    i.data_ptr(), z.data_ptr(), None, 0, None) == -1


@pytest.mark.parametrize("T,E,K", [(1, 128, 2048), (32, 128, 2048), (5, 32, 512), (3, 64, 4096)])
def test_router_logits_bit_exact(T, E, K):
    """The router's fixed summation order reproduces the oracle's quantized matmul bit for bit
    (N(0, 1) router weights: the logits are large, so a one-ulp difference would move gates)."""
    rng = np.random.default_rng(T + E + K)
    q, s, b = orc.w4_quantize(rng.normal(0, 1, size=(E, K)).astype(np.float32))
    x = orc.f32_to_bf16(rng.normal(0, 1, size=(T, K)))
    got = to_np_bf(ops().moe_router(bf(x), t(q.view(np.int32)), bf(s), bf(b)))
    assert np.array_equal(got, orc.qmatmul(x, q, s, b))
