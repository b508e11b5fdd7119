"""GPU (2 devices): the tensor-parallel decode step.

Two processes, one per GPU, each hold a shard of the same model (shard_weights) and a
peer-memory communicator (comm.cu).  Their greedy streams must be identical to each
other and to the oracle's (up to the oracle's own near-ties), and no collective may
have timed out.  Skipped on a box with fewer than two GPUs.
"""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")]

STEPS = 32


def moe_tp_args():
    """Tiny Qwen3-MoE (layer 1 dense) whose dense FFN splits two ways."""
    import dataclasses
    from higgs_b200.model import tiny_args
    return dataclasses.replace(tiny_args("qwen3_moe", layers=3), intermediate_size=1024)


def n_seqs(kind):
    return 1 if kind == "dense_fused" else 2


def _worker(rank, world, port, q, kind="dense"):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120))
        torch.cuda.set_device(rank)
        from oracle.model_ref import synth_weights_numpy
        from higgs_b200.engine import Engine
        from higgs_b200.model import Model, TPGroup, shard_weights, weights_to_device
        from tests.test_tp_cpu import tp_args
        args = moe_tp_args() if kind == "moe" else tp_args()
        w = synth_weights_numpy(args, seed=0)
        dev = f"cuda:{rank}"
        if kind == "dense_fused":  # one sequence: the GEMV-fused sum over ranks (option tp_fuse)
            from higgs_b200 import ffi
            ffi.call("higgs_set_option", b"tp_fuse", 1)
        wd = weights_to_device(shard_weights(args, w, rank, world), dev)

        def gather(b):
            out = [None] * world
            dist.all_gather_object(out, b)
            return out
        tp = TPGroup(rank, world, words_per_call=32 * args.hidden_size,
                     n_calls=2 * args.num_hidden_layers + 1, all_gather=gather, device=dev)
        m = Model(args, wd, num_pages=128, device=dev, tp=tp)
        pr = np.random.default_rng(1).integers(0, args.vocab_size, size=(n_seqs(kind), 20)).astype(np.int32)
        toks = Engine(m, max_seq_len=256).generate_greedy(list(pr), STEPS, use_prefix=False)
        torch.cuda.synchronize()
        q.put((rank, toks, tp.error()))
        del m
        tp.close()
    except Exception:
        import traceback
        q.put((rank, None, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("kind", ["dense", "dense_fused", "moe"])
def test_tp2_greedy_matches_oracle(kind):
    """Dense: tensor parallel.  Dense fused: one sequence with the sum over ranks inside the
    GEMVs (pushed by the row-parallel GEMV, pulled by the next fused-norm GEMV).  MoE:
    attention tensor parallel, experts split over the two ranks (expert parallelism) with
    the expert outputs summed by the same all-reduce."""
    from oracle.model_ref import RefModel, synth_weights_numpy
    from tests.test_tp_cpu import tp_args
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + os.getpid() % 1000 + {"dense": 0, "dense_fused": 3, "moe": 7}[kind]
    ps = [ctx.Process(target=_worker, args=(r, world, port, q, kind)) for r in range(world)]
    for p_ in ps:
        p_.start()
    res = sorted((q.get(timeout=600) for _ in range(world)), key=lambda r: r[0])
    for p_ in ps:
        p_.join(timeout=120)
    for r in res:
        assert r[1] is not None, r[2]
        assert r[2] == 0, "a collective timed out"
    assert np.array_equal(res[0][1], res[1][1])
    args = moe_tp_args() if kind == "moe" else tp_args()
    w = synth_weights_numpy(args, seed=0)
    nb = n_seqs(kind)
    pr = np.random.default_rng(1).integers(0, args.vocab_size, size=(nb, 20)).astype(np.int32)
    ref = RefModel(args, w)
    ref_tok, ref_lg = ref.greedy(pr, STEPS)
    top2 = np.sort(ref_lg, axis=-1)[..., -2:]
    margin = top2[..., 1] - top2[..., 0]  # [steps, B]
    near = ref.step_route_near  # MoE routings within one bf16 ulp of a swap
    for b in range(nb):
        d = np.nonzero(res[0][1][b] != ref_tok[b])[0]
        if d.size:
            k = int(d[0])
            assert margin[k, b] < 4e-2 or near[:k + 1, b].any(), (
                f"seq {b} diverges at step {k} with margin {margin[k, b]:.3f}")
