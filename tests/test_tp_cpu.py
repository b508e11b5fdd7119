"""CPU: the tensor-parallel decomposition of the decode step, checked with the oracle.

Two gloo ranks each run the oracle on their shard (shard_weights): column-parallel
q|k|v and gate|up, row-parallel o_proj / down_proj whose f32 partials are summed
across ranks (all_reduce) before the single bf16 rounding and the residual add,
and a vocabulary-sharded LM head whose greedy argmax is reduced across ranks.
The result must equal the unsharded oracle forward (up to f32 summation order in
the two sums).  This is the host-side logic the GPU path (comm.cu + model.cu)
implements with one-shot peer-memory pushes.
"""
import dataclasses
import os

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as orc
from oracle.model_ref import RefModel, synth_weights_numpy


def tp_args():
    """Small qwen3 shapes that split 2 and 4 ways (8 / 4 heads, FFN 1024)."""
    from higgs_b200.model import ModelArgs
    return ModelArgs("qwen3", 512, 2, 1024, 8, 4, 128, 4096, 1e-6, 1000000.0, False)


def _tp_forward(args, w, tokens, rank, world):
    """Oracle forward of a prompt (one sequence, no cache reuse) on this rank's shard."""
    from higgs_b200.model import shard_weights
    sw = shard_weights(args, w, rank, world)
    H, D = args.hidden_size, args.head_dim
    Hq, Hkv = args.num_attention_heads // world, args.num_key_value_heads // world
    T = tokens.size
    q = lambda n: (sw[n + ".weight"], sw[n + ".scales"], sw[n + ".biases"])  # noqa: E731
    h = orc.embed_gather(tokens, *q("model.embed_tokens"))
    inv = np.array([args.rope_theta ** (-(2.0 * i) / D) for i in range(D // 2)], np.float32)
    pos = np.arange(T, dtype=np.int32)

    def allreduce_residual(part_f32, h):
        import torch
        t = torch.from_numpy(np.ascontiguousarray(part_f32))
        dist.all_reduce(t)  # rank-order-independent here up to f32 rounding
        y = orc.f32_to_bf16(t.numpy())
        return orc.f32_to_bf16(orc.bf16_to_f32(h) + orc.bf16_to_f32(y))

    for li in range(args.num_hidden_layers):
        p = f"model.layers.{li}."
        x = orc.rmsnorm(h, sw[p + "input_layernorm.weight"], args.rms_norm_eps)[0]
        qh = orc.qmatmul(x, *q(p + "self_attn.q_proj")).reshape(T, Hq, D)
        kh = orc.qmatmul(x, *q(p + "self_attn.k_proj")).reshape(T, Hkv, D)
        vh = orc.qmatmul(x, *q(p + "self_attn.v_proj")).reshape(T, Hkv, D)
        qh = orc.rmsnorm(qh.reshape(-1, D), sw[p + "self_attn.q_norm.weight"], args.rms_norm_eps)[0].reshape(T, Hq, D)
        kh = orc.rmsnorm(kh.reshape(-1, D), sw[p + "self_attn.k_norm.weight"], args.rms_norm_eps)[0].reshape(T, Hkv, D)
        qr, kr = orc.rope(qh, pos, inv), orc.rope(kh, pos, inv)
        P = (T + 15) // 16
        kp = np.zeros((P * 16, Hkv, D), np.uint16)
        vp = np.zeros((P * 16, Hkv, D), np.uint16)
        kp[:T], vp[:T] = kr, vh
        kp = kp.reshape(P, 16, Hkv, D).transpose(0, 2, 1, 3)
        vp = vp.reshape(P, 16, Hkv, D).transpose(0, 2, 1, 3)
        attn = orc.paged_attention(qr[None], kp, vp, np.arange(P, dtype=np.int32)[None],
                                   np.array([T], np.int32))[0]
        _, of = orc.qmatmul(attn.reshape(T, Hq * D), *q(p + "self_attn.o_proj"), want_f32=True)
        h = allreduce_residual(of, h)
        x = orc.rmsnorm(h, sw[p + "post_attention_layernorm.weight"], args.rms_norm_eps)[0]
        g = orc.qmatmul(x, *q(p + "mlp.gate_proj"))
        u = orc.qmatmul(x, *q(p + "mlp.up_proj"))
        _, df = orc.qmatmul(orc.silu_mul(g, u), *q(p + "mlp.down_proj"), want_f32=True)
        h = allreduce_residual(df, h)
    x = orc.rmsnorm(h[-1:], sw["model.norm.weight"], args.rms_norm_eps)[0]
    _, lg = orc.qmatmul(x, *q("lm_head"), want_f32=True)
    # vocabulary-sharded greedy argmax: (value, -global index) max over ranks
    import torch
    j = int(orc.argmax(lg)[0])
    key = torch.tensor([float(lg[0, j]), -float(rank * lg.shape[1] + j)], dtype=torch.float64)
    keys = [torch.zeros(2, dtype=torch.float64) for _ in range(world)]
    dist.all_gather(keys, key)
    best = max(keys, key=lambda k: (k[0].item(), k[1].item()))
    return int(-best[1].item()), lg


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        args = tp_args()
        w = synth_weights_numpy(args, seed=0)
        tokens = np.random.default_rng(4).integers(0, args.vocab_size, 12).astype(np.int32)
        tok, lg = _tp_forward(args, w, tokens, rank, world)
        q.put((rank, tok, lg))
    except Exception as e:  # report instead of leaving the parent waiting
        import traceback
        q.put((rank, None, traceback.format_exc()))
        raise e
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_tp_decomposition_matches_unsharded_oracle():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 1000
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p_ in ps:
        p_.start()
    res = sorted((q.get(timeout=300) for _ in range(world)), key=lambda r: r[0])
    for p_ in ps:
        p_.join(timeout=60)
    for r in res:
        assert r[1] is not None, r[2]
    args = tp_args()
    w = synth_weights_numpy(args, seed=0)
    tokens = np.random.default_rng(4).integers(0, args.vocab_size, 12).astype(np.int32)
    ref = RefModel(args, w).forward(tokens[None], [RefModel(args, w).new_cache()])[0, -1]
    full = np.concatenate([r[2][0] for r in res])  # vocabulary shards in rank order
    np.testing.assert_allclose(full, ref, atol=2e-2, rtol=1e-2)
    assert res[0][1] == res[1][1] == int(np.argmax(full))


def test_shard_weights_slices():
    from higgs_b200.model import shard_weights
    args = dataclasses.replace(tp_args(), num_hidden_layers=1)
    w = synth_weights_numpy(args, seed=0)
    for world in (2, 4):
        parts = [shard_weights(args, w, r, world) for r in range(world)]
        p = "model.layers.0."
        for n in ("self_attn.q_proj", "mlp.gate_proj", "mlp.up_proj"):
            for leaf in ("weight", "scales", "biases"):
                cat = np.concatenate([s[p + n + "." + leaf] for s in parts], 0)
                assert np.array_equal(cat, w[p + n + "." + leaf])
        for n in ("self_attn.o_proj", "mlp.down_proj"):
            for leaf in ("weight", "scales", "biases"):
                cat = np.concatenate([s[p + n + "." + leaf] for s in parts], 1)
                assert np.array_equal(cat, w[p + n + "." + leaf])
        # row-parallel partial products sum to the whole (f32, up to summation order)
        x = orc.f32_to_bf16(np.random.default_rng(1).normal(size=(3, args.num_attention_heads * args.head_dim)))
        Kp = x.shape[1] // world
        tot = sum(orc.qmatmul(np.ascontiguousarray(x[:, r * Kp:(r + 1) * Kp]),
                              *(parts[r][p + "self_attn.o_proj." + l] for l in ("weight", "scales", "biases")),
                              want_f32=True)[1] for r in range(world))
        _, full = orc.qmatmul(x, *(w[p + "self_attn.o_proj." + l] for l in ("weight", "scales", "biases")),
                              want_f32=True)
        np.testing.assert_allclose(tot, full, rtol=1e-4, atol=1e-5)
    with pytest.raises(ValueError):
        shard_weights(args, w, 0, 3)  # 8 heads do not split 3 ways


def _ep_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        import torch
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from higgs_b200.model import shard_weights, tiny_args
        args = tiny_args("qwen3_moe", layers=1)
        w = synth_weights_numpy(args, seed=0)
        sw = shard_weights(args, w, rank, world)
        p = "model.layers.0.mlp."
        rng = np.random.default_rng(6)
        T, k, H = 5, args.num_experts_per_tok, args.hidden_size
        x = orc.f32_to_bf16(rng.normal(0, 1, size=(T, H)))
        rl = orc.qmatmul(x, sw[p + "gate.weight"], sw[p + "gate.scales"], sw[p + "gate.biases"])
        idx, sc = orc.moe_route_topk(orc.bf16_to_f32(rl), k, args.norm_topk_prob)
        El = args.num_experts // world
        e_lo = rank * El
        trip = lambda n: tuple(sw[p + "switch_mlp." + n + "." + l] for l in ("weight", "scales", "biases"))  # noqa: E731
        g, u, d = trip("gate_proj"), trip("up_proj"), trip("down_proj")
        part = np.zeros((T, H), np.float32)
        for t_ in range(T):
            for j in range(k):
                e = int(idx[t_, j])
                if not e_lo <= e < e_lo + El:
                    continue
                el = e - e_lo
                xe = x[t_:t_ + 1]
                a = orc.silu_mul(orc.qmatmul(xe, g[0][el], g[1][el], g[2][el]),
                                 orc.qmatmul(xe, u[0][el], u[1][el], u[2][el]))
                y = orc.qmatmul(a, d[0][el], d[1][el], d[2][el])
                part[t_] += orc.bf16_to_f32(orc.f32_to_bf16(sc[t_, j])) * orc.bf16_to_f32(y[0])
        tt = torch.from_numpy(part)
        dist.all_reduce(tt)
        q.put((rank, tt.numpy(), x, idx, sc))
    except Exception:
        import traceback
        q.put((rank, None, traceback.format_exc(), None, None))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_ep_moe_decomposition_matches_oracle():
    """Expert parallelism: each rank runs only its experts' pairs and the f32 shares summed
    over ranks equal the whole block (oracle moe_experts + combine) before the final rounding."""
    from higgs_b200.model import tiny_args
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29650 + os.getpid() % 1000
    ps = [ctx.Process(target=_ep_worker, args=(r, world, port, q)) for r in range(world)]
    for p_ in ps:
        p_.start()
    res = sorted((q.get(timeout=300) for _ in range(world)), key=lambda r: r[0])
    for p_ in ps:
        p_.join(timeout=60)
    for r in res:
        assert r[1] is not None, r[2]
    args = tiny_args("qwen3_moe", layers=1)
    w = synth_weights_numpy(args, seed=0)
    p = "model.layers.0.mlp.switch_mlp."
    trip = lambda n: tuple(w[p + n + "." + l] for l in ("weight", "scales", "biases"))  # noqa: E731
    _, _, x, idx, sc = res[0]
    y = orc.moe_experts(x, idx, trip("gate_proj"), trip("up_proj"), trip("down_proj"))
    h0 = np.zeros(x.shape, np.uint16)
    full = orc.bf16_to_f32(orc.moe_combine(y, sc, h0))  # bf16(sum) on a zero residual
    ep = orc.bf16_to_f32(orc.f32_to_bf16(res[0][1]))
    np.testing.assert_array_equal(res[0][1], res[1][1])
    np.testing.assert_allclose(ep, full, atol=1e-3 * np.abs(full).max(), rtol=1e-2)


def test_shard_weights_replicates_kv_heads_when_fewer_than_ranks():
    from higgs_b200.model import ModelArgs, kv_heads_per_rank, shard_weights
    args = ModelArgs("qwen3", 512, 1, 1024, 8, 2, 128, 4096, 1e-6, 1000000.0, False)
    w = synth_weights_numpy(args, seed=0)
    assert kv_heads_per_rank(args, 4) == 1
    k = "model.layers.0.self_attn.k_proj.weight"
    parts = [shard_weights(args, w, r, 4)[k] for r in range(4)]
    D = args.head_dim
    for r in range(4):  # ranks 0,1 hold kv head 0 (query heads 0-3), ranks 2,3 kv head 1
        assert np.array_equal(parts[r], w[k][(r // 2) * D:(r // 2 + 1) * D])
