"""Decode throughput of the B200 hot path (4-bit Qwen3-8B architecture).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One "step" = one greedy decode step (all 36 layers + LM head + argmax) for a
batch of B sequences at a synthetic KV context (default 2048 tokens).  The
headline `value` is decode tok/s at B=1 on one GPU with every input resident in
HBM; B=8 and B=32 are reported under `by_batch`.  `e2e` is the same metric
through the public engine API with per-step host->device inputs and a
device->host read of the sampled tokens inside the timed region.

Weights are random-init N(0, 0.02) quantized to MLX-affine W4 g64 (no
checkpoint available offline); the KV context is synthetic random bf16 (decode
cost does not depend on the values).  Weights (4.26 GB/step) exceed L2, so
every step streams them from HBM.

With N > 1 (torchrun), the same model and batch run tensor-parallel over the N
GPUs (strong scaling): each rank holds a column / row shard of every projection
and a vocabulary shard of the LM head, and the ranks sum their partials with a
peer-memory all-reduce after attention and after the MLP of every layer.
`value` is the batch's tokens over the maximum time over ranks.  `tp_parity`
checks the tensor-parallel model's greedy stream and logits against the same
weights on one GPU; `comm_errors` counts collectives whose bounded wait gave up
(the run fails if any did).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

MODEL = "qwen3-8b"
CTX = 2048
BATCHES = (1, 8, 32)
METRIC = "decode tok/s at B=1/8/32 (4-bit Qwen3-8B arch) @1/2/4/8 GPU; % HBM roofline"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ctx", type=int, default=CTX)
    ap.add_argument("--batches", default=",".join(map(str, BATCHES)))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--quick", action="store_true", help="headline B only, no kernel table (profiling)")
    ap.add_argument("--configs", default="c1,c2,c3,c4,c5",
                    help="other BASELINE configs to run at N=1 (comma list, '' for none)")
    ap.add_argument("--chain-roofline", action="store_true",
                    help="also time the persistent decode-chain kernel (off in the step by default)")
    ap.add_argument("--option", action="append", default=[],
                    help="library tuning switch name=value (higgs_set_option), repeatable")
    ap.add_argument("--kernel-case", default=None,
                    help="run one small kernel case for ncu: qkv|o_proj|gate_up_swiglu|down|lm_head[:tokens]"
                         "|attention|attention_tq4|prefill_attn|argmax|tc_rate|decode_eager:<batch>")
    return ap.parse_args()


# ---------------------------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------------------------
def dist_setup():
    import torch
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime
        os.environ.setdefault("NCCL_DEBUG", "WARN")  # stdout carries only the JSON line

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return ws, rank, local


def allmax(x: float) -> float:
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()):
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier():
    import torch
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize()


# ---------------------------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------------------------
class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self.proc = None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 8:
                self.samples.append(parts)

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[4 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.samples)}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def bf16_peak():
    """Dense bf16 TFLOP/s (burst: the kernels below are timed alone) and where it came from."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def prefill_case(a, L, dev, copies=1):
    """One prompt chunk of L tokens of the bench model's attention shape over a paged cache
    holding exactly those L tokens (query t at position t): q, caches, block table, lengths."""
    import torch
    Hq, Hkv, D = a.num_attention_heads, a.num_key_value_heads, a.head_dim
    P = (L + 15) // 16
    q = torch.randn(1, L, Hq, D, device=dev).to(torch.bfloat16)
    caches = [(torch.randn(P, Hkv, 16, D, device=dev).to(torch.bfloat16),
               torch.randn(P, Hkv, 16, D, device=dev).to(torch.bfloat16)) for _ in range(copies)]
    bt = torch.arange(P, dtype=torch.int32, device=dev).view(1, P)
    sl = torch.tensor([L], dtype=torch.int32, device=dev)
    return q, caches, bt, sl


def prefill_attn_roofline(a, dev, lengths=(2048, 8192)):
    """Causal prefill attention of one prompt chunk (the bench model's heads), one launch of
    the tcgen05 kernel against the mma.sync decode kernel's 32-row chunks (option
    attn_prefill_tc 0) on the same inputs.  FLOPs: 4 * Hq * D * (L (L + 1) / 2) (QK^T and PV
    over the causal triangle)."""
    import torch

    from higgs_b200 import ffi
    from higgs_b200 import ops
    peak, kind = bf16_peak()
    Hq, Hkv, D = a.num_attention_heads, a.num_key_value_heads, a.head_dim
    rows = []
    for L in lengths:
        q, caches, bt, sl = prefill_case(a, L, dev)
        kc, vc = caches[0]
        ws = ops.attention_workspace(1, L, Hq, Hkv, D, L, dev)
        flops = 4.0 * Hq * D * (L * (L + 1) / 2)

        def timed(reps):
            for _ in range(3):
                ops.paged_attention(q, kc, vc, bt, sl, L, workspace=ws)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                ops.paged_attention(q, kc, vc, bt, sl, L, workspace=ws)
            e1.record()
            e1.synchronize()
            return e0.elapsed_time(e1) * 1e3 / reps
        us = timed(20)
        ffi.call("higgs_set_option", b"attn_prefill_tc", 0)
        try:
            us_old = timed(3)
        finally:
            ffi.call("higgs_set_option", b"attn_prefill_tc", 1)
        rows.append({"prompt_tokens": L, "us": round(us, 1), "tflops": round(flops / us / 1e6, 1),
                     "frac": round(flops / us / 1e6 / peak, 4), "us_mma_sync_chunks": round(us_old, 1)})
        del q, caches, kc, vc, ws
        torch.cuda.empty_cache()
    return {"kernel": "prefill_attn_tc_kernel<%d> (causal, Hq %d / Hkv %d)" % (D, Hq, Hkv),
            "bound": "tensor", "peak": peak, "peak_kind": kind, "unit": "TFLOP/s", "per_length": rows}


# ---------------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------------
def make_tp_group(args_m, rank, world, max_tokens, device):
    """This rank's peer-memory communicator; IPC handles exchanged over a gloo group.  Each call
    region holds at least 64 tokens: tp_parity prefills a 32-token prompt."""
    max_tokens = max(max_tokens, 64)
    import torch.distributed as dist

    from higgs_b200.model import TPGroup
    gloo = dist.new_group(backend="gloo")

    def gather(b):
        out = [None] * world
        dist.all_gather_object(out, b, group=gloo)
        return out
    return TPGroup(rank, world, words_per_call=max_tokens * args_m.hidden_size,
                   n_calls=2 * args_m.num_hidden_layers + 1, all_gather=gather, device=device)


def setup_model(args_m, batches, ctx, total_steps, device, world=1, rank=0):
    """The model on one GPU, or (world > 1) this rank's tensor-parallel shard with its
    peer-memory communicator (the unsharded weights are kept for the parity check)."""
    import torch

    from higgs_b200.engine import Engine, Sequence
    from higgs_b200.model import Model, TPGroup, shard_weights, synth_weights_device

    weights = synth_weights_device(args_m, seed=0, device=device)
    per_seq_pages = math.ceil((ctx + total_steps + 2) / 16)
    num_pages = max(max(batches), 4) * per_seq_pages + 16  # >= the 4 sequences of C3
    tp = None
    full = None
    if world > 1:
        full = weights
        weights = shard_weights(args_m, weights, rank, world)
        tp = make_tp_group(args_m, rank, world, max(batches), device)
    model = Model(args_m, weights, num_pages=num_pages, device=device, tp=tp)
    # synthetic KV context (random bf16; decode cost does not depend on the values)
    g = torch.Generator(device=device)
    g.manual_seed(2)
    for pool in (model.k_pool, model.v_pool):
        for li in range(pool.shape[0]):
            pool[li].copy_(torch.randn(pool[li].shape, generator=g, device=device).to(torch.bfloat16))
    eng = Engine(model, max_seq_len=ctx + total_steps + 2, prefix_entries=0)
    return model, eng, Sequence, full


def make_seqs(eng, Sequence, B, ctx, vocab, seed=1):
    rng = np.random.default_rng(seed)
    seqs = []
    for _ in range(B):
        s = Sequence(prompt=np.zeros(0, np.int32))
        s.pages = eng.pool.alloc(math.ceil((ctx + 1) / 16)).tolist()
        s.length = ctx
        s.last_token = int(rng.integers(0, vocab))
        seqs.append(s)
    return seqs


def time_device_resident(eng, seqs, steps, warmup):
    """Graph replays with all per-step inputs pre-staged in HBM; CUDA events on the stream."""
    import torch
    B = len(seqs)
    g = eng._graph_for(B)
    total = warmup + steps
    for s in seqs:  # pages for every position the replays will write
        eng._ensure_pages(s, s.length + total + 1)
    # stage step 0 through the public path, then precompute every step's vectors on device
    base = [s.length for s in seqs]
    eng.stage_step(seqs, g, first=True)
    torch.cuda.current_stream().synchronize()
    host = np.zeros((total, 4 * B), np.int32)
    for k in range(total):
        for i, s in enumerate(seqs):
            L = base[i] + k
            host[k, i] = L
            host[k, B + i] = L + 1
        slots = np.array([s.pages[(b + k) // 16] * 16 + (b + k) % 16 for s, b in zip(seqs, base)],
                         np.int64)
        host[k, 2 * B:] = slots.view(np.int32)
    staged = torch.from_numpy(host).to(g.step_dev.device)
    stream = torch.cuda.current_stream()
    for k in range(warmup):
        g.step_dev.copy_(staged[k], non_blocking=True)
        g.run()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for k in range(warmup, total):
        g.step_dev.copy_(staged[k], non_blocking=True)
        g.run()
    e1.record(stream)
    e1.synchronize()
    barrier()
    ms = e0.elapsed_time(e1)
    for s, b in zip(seqs, base):  # the replays wrote KV at these positions
        s.length = b + total
    return ms, g.graph.num_kernels if g.graph is not None else None


def time_e2e(eng, seqs, steps, warmup):
    """Public API: Engine.decode_steps stages inputs from the host each step and reads the tokens back."""
    import torch
    eng.decode_steps(seqs, warmup)
    barrier()
    t0 = time.perf_counter()
    eng.decode_steps(seqs, steps)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    barrier()
    return (t1 - t0) * 1e3


def graph_time(fns, reps=10):
    """Seconds per replay of a CUDA graph holding fns() back to back (PDL edges kept)."""
    import torch
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for f in fns:
            f()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for f in fns:
            f()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cur = torch.cuda.current_stream()
    e0.record(cur)
    for _ in range(reps):
        g.replay()
    e1.record(cur)
    e1.synchronize()
    return e0.elapsed_time(e1) / reps * 1e-3


def gemv_shapes(model):
    """(name, per-layer weight triples, K, launches per step) of every W4 GEMV of a decode step."""
    import torch
    a = model.args
    w = model.weights
    L = a.num_hidden_layers
    H, D = a.hidden_size, a.head_dim

    def trip(name):
        return (w[name + ".weight"], w[name + ".scales"], w[name + ".biases"])

    lay = [f"model.layers.{i}." for i in range(L)]
    qkv = [tuple(torch.cat([trip(p + "self_attn." + n)[k] for n in ("q_proj", "k_proj", "v_proj")])
                 for k in range(3)) for p in lay]
    head = "model.embed_tokens" if a.tie_word_embeddings else "lm_head"
    o = [trip(p + "self_attn.o_proj") for p in lay]
    d = [trip(p + "mlp.down_proj") for p in lay]
    # K from the tensors: a tensor-parallel shard holds a K slice of o_proj / down_proj
    return [("qkv", qkv, H, L),
            ("o_proj", o, o[0][0].shape[1] * 8, L),
            ("gate_up_swiglu", [trip(p + "mlp.gate_proj") + trip(p + "mlp.up_proj") for p in lay], H, L),
            ("down", d, d[0][0].shape[1] * 8, L),
            ("lm_head", [trip(head)] * 4, H, 1)]


def gemv_roofline(model, M=1):
    """Each W4 GEMV shape of one decode step timed inside a CUDA graph of back-to-back
    launches over every layer's own weights (so no launch finds its weights in L2),
    exactly as the step runs them; per-launch time = graph time / launches."""
    import torch

    from higgs_b200 import ops
    rows = []
    for name, ws, K, count in gemv_shapes(model):
        x = torch.randn(M, K, device=model.device).to(torch.bfloat16)
        N = ws[0][0].shape[0]
        wbytes = sum(t.numel() * t.element_size() for t in ws[0])
        # > 8 rows: through the workspace entry (split-K tensor-core matmul), as the model step runs it
        sk = ops.sk_workspace(M, K, 2 * N, model.device) if M > 8 else None
        if name == "gate_up_swiglu":
            if sk is None:
                fns = [lambda w=w: ops.gate_up_swiglu(x, *w) for w in ws]
            else:
                fns = [lambda w=w: ops.rmsnorm_gate_up_swiglu(x, None, 0.0, *w, workspace=sk) for w in ws]
            nbytes = wbytes + M * K * 2 + M * N * 2
        else:
            f32 = name == "lm_head"
            if sk is None:
                fns = [lambda w=w, f=f32: ops.quantized_matmul(x, *w, out_f32=f) for w in ws]
            else:
                fns = [lambda w=w, f=f32: ops.rmsnorm_quantized_matmul(x, None, 0.0, *w, out_f32=f, workspace=sk)
                       for w in ws]
            nbytes = wbytes + M * K * 2 + M * N * (4 if f32 else 2)
        us = graph_time(fns) / len(fns) * 1e6
        rows.append({"shape": name, "launches_per_step": count, "bytes": int(nbytes), "us": round(us, 2),
                     "gbs": round(nbytes / us / 1e3, 1)})
        del fns
    return rows


def chain_roofline(model, reps=10):
    """The decode-chain kernel as the B=1 step runs it: one launch per layer (o_proj + residual,
    norm + gate/up SwiGLU, down + residual, norm + the next layer's q|k|v) over that layer's
    own weights, all layers back to back in one CUDA graph so no launch finds its weights in L2;
    per-launch time = graph time / layers.  Returns (bytes per launch, us per launch)."""
    import torch

    from higgs_b200 import ops
    a = model.args
    w = model.weights
    dev = model.device
    L, H = a.num_hidden_layers, a.hidden_size
    g = torch.Generator(device=dev)
    g.manual_seed(9)
    attn = torch.randn(a.num_attention_heads * a.head_dim, generator=g, device=dev).to(torch.bfloat16)
    h = torch.randn(H, generator=g, device=dev).to(torch.bfloat16)
    act = torch.zeros(a.intermediate_size, dtype=torch.bfloat16, device=dev)
    qkv = torch.zeros((a.num_attention_heads + 2 * a.num_key_value_heads) * a.head_dim,
                      dtype=torch.bfloat16, device=dev)
    bars = torch.zeros(4 * 64 * L, dtype=torch.int32, device=dev)

    def trip(n):
        return w[n + ".weight"], w[n + ".scales"], w[n + ".biases"]
    launches, nbytes = [], 0
    for li in range(L):
        p, pn = f"model.layers.{li}.", f"model.layers.{(li + 1) % L}."
        ph = [ops.chain_gemv(attn, *trip(p + "self_attn.o_proj"), y=h, residual=h),
              ops.chain_gemv(h, *trip(p + "mlp.gate_proj"), norm_w=w[p + "post_attention_layernorm.weight"],
                             up=trip(p + "mlp.up_proj"), y=act),
              ops.chain_gemv(act, *trip(p + "mlp.down_proj"), y=h, residual=h),
              ops.chain_gemv(h, None, None, None, norm_w=w[pn + "input_layernorm.weight"],
                             segments=[trip(pn + "self_attn." + n) for n in ("q_proj", "k_proj", "v_proj")],
                             y=qkv)]
        launches.append((ph, bars[256 * li:256 * li + 256]))
        if li == 0:
            for n in ("self_attn.o_proj", "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj"):
                nbytes += sum(t.numel() * t.element_size() for t in trip(p + n))
            nbytes += sum(sum(t.numel() * t.element_size() for t in trip(pn + "self_attn." + n))
                          for n in ("q_proj", "k_proj", "v_proj"))
            # activations read and written once: attn, h (3 reads, 2 writes), act (w + r), qkv
            nbytes += attn.numel() * 2 + 5 * H * 2 + 2 * act.numel() * 2 + qkv.numel() * 2
    fns = [lambda ph=ph, b=b: ops.decode_chain(ph, a.rms_norm_eps, b, dev) for ph, b in launches]
    us = graph_time(fns, reps) / L * 1e6
    return int(nbytes), us


def kernel_case(opt):
    """Small standalone launches of one hot kernel, for ncu captures (-k / -c)."""
    import torch

    from higgs_b200 import ops
    from higgs_b200.model import PRESETS
    dev = "cuda:0"
    a = PRESETS[MODEL]
    H = a.hidden_size
    torch.manual_seed(0)

    def mk(N, K):
        return (torch.randint(-2**31, 2**31 - 1, (N, K // 8), dtype=torch.int32, device=dev),
                (torch.rand(N, K // 64, device=dev) * 0.01).to(torch.bfloat16),
                (torch.randn(N, K // 64, device=dev) * 0.01).to(torch.bfloat16))
    case, _, mrows = opt.kernel_case.partition(":")  # "<shape>[:<tokens>]", default 1 token
    M = int(mrows) if mrows else 1
    if case in ("qkv", "o_proj", "down", "lm_head", "gate_up_swiglu"):
        K, N = {"qkv": (H, (a.num_attention_heads + 2 * a.num_key_value_heads) * a.head_dim),
                "o_proj": (a.num_attention_heads * a.head_dim, H), "down": (a.intermediate_size, H),
                "lm_head": (H, a.vocab_size), "gate_up_swiglu": (H, a.intermediate_size)}[case]
        reps = 2 if case == "lm_head" else 8  # > 126 MB of distinct weights in flight
        ws = [mk(N, K) + (mk(N, K) if case == "gate_up_swiglu" else ()) for _ in range(reps)]
        x = torch.randn(M, K, device=dev).to(torch.bfloat16)
        sk = ops.sk_workspace(M, K, 2 * N, dev) if M > 8 else None  # split-K tensor-core path
        for it in range(3):
            for w in ws:
                if case == "gate_up_swiglu":
                    if sk is None:
                        ops.gate_up_swiglu(x, *w)
                    else:
                        ops.rmsnorm_gate_up_swiglu(x, None, 0.0, *w, workspace=sk)
                elif sk is None:
                    ops.quantized_matmul(x, *w, out_f32=case == "lm_head")
                else:
                    ops.rmsnorm_quantized_matmul(x, None, 0.0, *w, out_f32=case == "lm_head", workspace=sk)
    elif case == "attention":
        B, Hq, Hkv, D, L = 1, a.num_attention_heads, a.num_key_value_heads, a.head_dim, opt.ctx
        P = L // 16 + 1
        nh = Hq + 2 * Hkv
        caches = [(torch.randn(P, Hkv, 16, D, device=dev).to(torch.bfloat16),
                   torch.randn(P, Hkv, 16, D, device=dev).to(torch.bfloat16)) for _ in range(8)]
        qkv = torch.randn(1, nh * D, device=dev).to(torch.bfloat16)
        qn = torch.ones(D, device=dev).to(torch.bfloat16)
        inv = ops.rope_inv_freq(D, a.rope_theta, dev)
        pos = torch.tensor([L - 1], dtype=torch.int32, device=dev)
        slots = torch.tensor([L - 1], dtype=torch.int64, device=dev)
        bt = torch.arange(P, dtype=torch.int32, device=dev).view(1, P)
        sl = torch.tensor([L], dtype=torch.int32, device=dev)
        for it in range(3):
            for kc, vc in caches:
                ops.fused_attention(qkv, Hq, Hkv, D, qn, qn, a.rms_norm_eps, pos, inv, slots, kc, vc, bt,
                                    sl, L)
    elif case == "prefill_attn":  # one prompt chunk of --ctx tokens on the tcgen05 prefill kernel
        L = opt.ctx
        q, caches, bt, sl = prefill_case(a, L, dev, copies=2)
        ws = ops.attention_workspace(1, L, a.num_attention_heads, a.num_key_value_heads, a.head_dim, L, dev)
        for it in range(3):
            for kc, vc in caches:
                ops.paged_attention(q, kc, vc, bt, sl, L, workspace=ws)
    elif case == "attention_tq4":  # C5 shapes: B=16, ctx 32768, TurboQuant pages
        B, Hq, Hkv, L = 16, a.num_attention_heads, a.num_key_value_heads, 32768
        maxb = L // 16
        P = B * maxb
        caches = []
        for _ in range(2):  # 2 x 1.1 GB of codes: no launch finds its pages in L2
            caches.append((torch.randint(0, 256, (P, Hkv, 16, 64), dtype=torch.uint8, device=dev),
                           (torch.rand(P, Hkv, 16, device=dev) * 0.1).to(torch.float16),
                           torch.randint(0, 256, (P, Hkv, 16, 64), dtype=torch.uint8, device=dev),
                           (torch.rand(P, Hkv, 16, device=dev) * 0.1).to(torch.float16)))
        q = torch.randn(B, 1, Hq, 128, device=dev).to(torch.bfloat16)
        bt = torch.arange(P, dtype=torch.int32, device=dev).view(B, maxb)
        sl = torch.full((B,), L, dtype=torch.int32, device=dev)
        signs = torch.where(torch.rand(128, device=dev) < 0.5, -1, 1).to(torch.int8)
        ws = ops.attention_workspace(B, 1, Hq, Hkv, 128, L, dev)
        for it in range(3):
            for kc, ks, vc, vs in caches:
                ops.paged_attention_tq4(q, kc, ks, vc, vs, bt, sl, L, signs, workspace=ws)
    elif case == "decode_eager":  # three decode steps of the bench model at batch M, launches not in a graph
        model, eng, Sequence, _ = setup_model(a, [M], opt.ctx, 8, dev)
        seqs = make_seqs(eng, Sequence, M, opt.ctx, a.vocab_size)
        eng.use_graph = False
        eng.decode_steps(seqs, 3)
    elif case == "tc_rate":  # tensor-core issue rate behind the matrix-form W4 matmul
        rows = []
        for m in (128, 64):
            for n in (32, 64, 128, 256):
                for warps in (1, 2, 4):
                    for ce in (0, 1):
                        if warps * n > 512:
                            continue
                        ops.tc_mma_rate(n, 1, 0, 256, ce, m=m, warps=warps)  # warm-up
                        rows.append(ops.tc_mma_rate(n, 1, 0, 4096, ce, m=m, warps=warps))
        for n in (32, 128):  # several accumulators behind one issuing warp
            for nacc in (2, 4):
                rows.append(ops.tc_mma_rate(n, nacc, 1, 4096, 1))
        for r in rows:
            print(json.dumps({k: (round(v, 2) if isinstance(v, float) else v) for k, v in r.items()}))
    elif case == "argmax":
        lg = torch.randn(1, a.vocab_size, device=dev)
        for it in range(3):
            ops.argmax(lg)
    else:
        raise SystemExit(f"unknown --kernel-case {case}")
    torch.cuda.synchronize()
    print(json.dumps({"kernel_case": case, "ok": True}))


def tp_parity(args_m, full_w, tp_model, device, steps=64, prompt_len=32, seed=7):
    """Greedy decode of `steps` tokens from one seeded prompt on this rank's tensor-parallel
    model (every rank takes part) and on an unsharded copy of the same weights on this rank's
    GPU alone.  Tokens: the free-running TP stream against the one-GPU stream.  Logits: the
    TP model teacher-forced on the one-GPU stream, this rank's vocabulary shard against the
    same slice of the one-GPU logits.  Maxima are taken over ranks."""
    import torch

    from higgs_b200.engine import Engine
    from higgs_b200.model import Model
    world, rank = tp_model.tp.world, tp_model.tp.rank
    pr = np.random.default_rng(seed).integers(0, args_m.vocab_size, size=(1, prompt_len)).astype(np.int32)
    msl = prompt_len + steps + 16
    # the tensor-parallel model: free-running stream (collectives on every rank, same order)
    tp_free = Engine(tp_model, max_seq_len=msl, prefix_entries=0).generate_greedy(list(pr), steps,
                                                                                   use_prefix=False)
    # the same weights on this GPU alone
    one = Model(args_m, full_w, num_pages=math.ceil(msl / 16) + 4, device=device)
    e1 = Engine(one, max_seq_len=msl, prefix_entries=0, keep_logits=True)
    s1 = e1.prefill(pr[0], use_prefix=False)
    first = s1.last_token
    one_rest = e1.decode_steps([s1], steps - 1)
    one_tok = np.concatenate([[first], one_rest[0]]).astype(np.int32)
    one_lg = np.stack(e1.step_logits)[:, 0]  # [steps-1, V]
    del e1, s1, one
    torch.cuda.empty_cache()
    # the TP model teacher-forced on the one-GPU stream
    et = Engine(tp_model, max_seq_len=msl, prefix_entries=0, keep_logits=True)
    st = et.prefill(pr[0], use_prefix=False)
    st.last_token = int(one_tok[0])
    # the forced steps' argmax over the whole vocabulary (the TP model's sharded argmax)
    forced = et.decode_steps([st], steps - 1, force=one_tok[None, :steps - 1])[0]
    shard = args_m.vocab_size // world
    tp_lg = np.stack(et.step_logits)[:, 0, :shard]
    ref = one_lg[:, rank * shard:(rank + 1) * shard]
    err = allmax(float(np.max(np.abs(tp_lg - ref))))
    std = allmax(float(np.std(tp_lg - ref)))  # a systematic TP error would show here, not just in the max
    rel = float(np.max(np.abs(tp_lg - ref) / (np.abs(ref) + 1e-6)))
    et.release(st)
    diff = np.nonzero(tp_free[0] != one_tok)[0]
    first_diff = int(diff[0]) if diff.size else None
    top2 = np.sort(one_lg, axis=-1)[:, -2:]
    margin = top2[:, 1] - top2[:, 0]  # the one-GPU top-2 margin at each decode step
    margin_at = (float(margin[first_diff - 1]) if first_diff is not None and first_diff >= 1 else None)
    # teacher-forced argmax disagreements, and those not explained by the measured logit noise
    # (a step whose top-2 margin exceeds twice the largest logit difference cannot flip)
    dis = np.nonzero(forced != one_tok[1:])[0]
    beyond = [int(k) for k in dis if margin[k] > 2 * err]
    return {"tokens": steps, "tokens_equal": bool(allmax(float(first_diff is not None)) == 0.0),
            "first_diff": first_diff, "margin_at_first_diff": margin_at,
            "max_logit_abs": round(err, 6), "logit_diff_std": round(std, 6),
            "max_logit_rel": round(allmax(rel), 6),
            "forced_argmax_disagreements": int(dis.size),
            "near_tie_steps": int(np.sum(margin <= 2 * err)),
            "disagreements_beyond_noise": len(beyond),
            "prompt": f"{prompt_len} uniform ids (seed {seed}), B=1, one GPU vs tp{world}"}


def comm_errors(model) -> int:
    """Collectives of this rank's communicator whose bounded wait gave up, plus tensor-core
    matmul timeouts on this GPU (both flags are cleared by the read)."""
    import ctypes

    from higgs_b200 import ffi
    n = 0
    if model.tp is not None:
        n += model.tp.error()
    v = ctypes.c_int(0)
    ffi.call("higgs_tc_error", ffi.ctx(model.device.index or 0), ctypes.byref(v))
    return n + v.value


def host_threads() -> int:
    """Host cores this process may run on; the oracle's OpenMP team is set to this many
    explicitly, since torchrun exports OMP_NUM_THREADS=1 to every rank."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def oracle_step_time(model_args, ctx, budget_s=20.0):
    """Seconds per B=1 decode step of the full model through the oracle port on the host,
    with every host core (returns seconds, sample description, threads used).

    Timed at true shapes on 2- and 6-layer slices (embedding, final norm, LM head and
    KV context included) and extrapolated linearly to all layers, since every layer
    costs the same.  Packed weights are random codes / scales: the oracle's cost does
    not depend on the values.  Returns (seconds_per_step, sample description)."""
    import dataclasses

    from oracle import oracle as orc
    from oracle.model_ref import RefModel
    from higgs_b200.model import tensor_specs
    threads = orc.set_threads(host_threads())
    rng = np.random.default_rng(5)

    def packed(shape):
        N, K = shape
        return (rng.integers(0, 2**32, size=(N, K // 8), dtype=np.uint64).astype(np.uint32),
                orc.f32_to_bf16(rng.uniform(1e-3, 3e-3, size=(N, K // 64))),
                orc.f32_to_bf16(rng.uniform(-0.02, 0, size=(N, K // 64))))

    def build(L):
        a = dataclasses.replace(model_args, num_hidden_layers=L)
        w = {}
        for name, kind, shape in tensor_specs(a):
            if kind == "norm":
                w[name] = np.full(shape, 0x3F80, np.uint16)
            else:
                w[name + ".weight"], w[name + ".scales"], w[name + ".biases"] = packed(shape)
        ref = RefModel(a, w)
        cache = ref.new_cache()
        Hkv, D = a.num_key_value_heads, a.head_dim
        for li in range(L):
            cache[li] = [orc.f32_to_bf16(rng.normal(size=(ctx, Hkv, D))),
                         orc.f32_to_bf16(rng.normal(size=(ctx, Hkv, D)))]
        return ref, cache

    times = {}
    reps = {}
    for L in (2, 6):
        ref, cache = build(L)
        tok = np.array([[7]], np.int32)
        ref.forward(tok, [cache])  # warm
        n, t0 = 0, time.perf_counter()
        while n < 3 and (n == 0 or time.perf_counter() - t0 < budget_s / 4):
            lg = ref.forward(tok, [cache])
            tok = orc.argmax(lg[:, -1]).reshape(1, 1).astype(np.int32)
            n += 1
        times[L] = (time.perf_counter() - t0) / n
        reps[L] = n
        del ref, cache
    per_layer = max(0.0, (times[6] - times[2]) / 4)
    full = times[2] + (model_args.num_hidden_layers - 2) * per_layer
    desc = (f"oracle port on {threads} OpenMP threads, B=1 decode at ctx {ctx}: {reps[2]} steps of a "
            f"2-layer and {reps[6]} of a 6-layer slice at true shapes, extrapolated to "
            f"{model_args.num_hidden_layers} layers")
    return full, desc, threads


# ---------------------------------------------------------------------------------------------
# the other BASELINE configurations (reported under "by_config"; the headline is C-headline)
# ---------------------------------------------------------------------------------------------
def _synth_model(args_m, device, num_pages, kv_mode="bf16", weights=None):
    from higgs_b200.model import Model, synth_weights_device
    w = weights if weights is not None else synth_weights_device(args_m, seed=0, device=device)
    return Model(args_m, w, num_pages=num_pages, kv_mode=kv_mode, device=device), w


def _fill_kv(model, seed=2):
    import torch
    g = torch.Generator(device=model.device)
    g.manual_seed(seed)
    if model.kv_mode == "tq4":
        for pool in (model.k_pool, model.v_pool):
            for li in range(pool.shape[0]):
                pool[li].copy_(torch.randint(0, 256, pool[li].shape, generator=g, device=model.device,
                                             dtype=torch.int32).to(torch.uint8))
        for sc in (model.k_scales, model.v_scales):
            sc.fill_(0.05)
    else:
        for pool in (model.k_pool, model.v_pool):
            for li in range(pool.shape[0]):
                pool[li].copy_(torch.randn(pool[li].shape, generator=g, device=model.device).to(torch.bfloat16))


def _entry(args_m, B, ctx, ms_step, hbm, kv_mode="bf16", experts_touched=0.0, extra=None):
    w_bytes = args_m.weight_bytes_per_step(experts_touched)
    kv = B * ctx * args_m.kv_bytes_per_token(kv_mode)
    e = {"tok_s": round(B * 1e3 / ms_step, 1), "ms_per_step": round(ms_step, 4),
         "step_bytes": int(w_bytes + kv),
         "step_hbm_frac": round((w_bytes + kv) / (ms_step / 1e3) / 1e9 / hbm, 4)}
    if extra:
        e.update(extra)
    return e


def config_c1(device, hbm, steps):
    """C1: Llama-3.2-1B arch, B=1, 128-token prompt, greedy decode (device-resident replays)."""
    from higgs_b200.engine import Engine, Sequence
    from higgs_b200.model import PRESETS
    a = PRESETS["llama-3.2-1b"]
    model, _ = _synth_model(a, device, num_pages=64)
    eng = Engine(model, max_seq_len=512, prefix_entries=0)
    rng = np.random.default_rng(1)
    seq = eng.prefill(rng.integers(0, a.vocab_size, 128).astype(np.int32), use_prefix=False)
    ms, _ = time_device_resident(eng, [seq], steps, 4)
    return _entry(a, 1, 128 + steps // 2, ms / steps, hbm,
                  extra={"workload": "llama-3.2-1b B=1 prompt 128, greedy"})


def config_c2(device, hbm, steps):
    """C2: Qwen3-1.7B arch, 8 sequences of 512-token prompts sharing a 256-token prefix (radix
    cache), then greedy decode of all 8 together through the public engine API."""
    import torch

    from higgs_b200.engine import Engine
    from higgs_b200.model import PRESETS
    a = PRESETS["qwen3-1.7b"]
    model, _ = _synth_model(a, device, num_pages=8 * 48 + 64)
    eng = Engine(model, max_seq_len=768, prefix_entries=16)
    rng = np.random.default_rng(2)
    shared = rng.integers(0, a.vocab_size, 256).astype(np.int32)
    prompts = [np.concatenate([shared, rng.integers(0, a.vocab_size, 256).astype(np.int32)])
               for _ in range(8)]
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    seqs = [eng.prefill(p_, use_prefix=True) for p_ in prompts]
    torch.cuda.synchronize()
    t_pre = time.perf_counter() - t0
    hits = [s.prefix_hit for s in seqs]
    eng.decode_steps(seqs, 4)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    eng.decode_steps(seqs, steps)
    torch.cuda.synchronize()
    ms = (time.perf_counter() - t0) * 1e3
    return _entry(a, 8, 512 + steps // 2, ms / steps, hbm,
                  extra={"workload": "qwen3-1.7b 8 seqs, 512-token prompts (256 shared), greedy; "
                                     "e2e through Engine.decode_steps",
                         "prefill_s": round(t_pre, 3), "prefix_hit_tokens": hits})


def config_c3(model, eng, Sequence, device, hbm, steps, ctx):
    """C3: self-speculative decoding on the Qwen3-8B model: draft = first 9 layers + the shared
    head, k=5, one batched verify of 6 tokens, rejection sampling at T=0.7 (uniforms seed 3)."""
    import torch

    from higgs_b200.engine import SpecDecoder
    B, k = 4, 5
    seqs = make_seqs(eng, Sequence, B, ctx, model.args.vocab_size, seed=21)
    sd = SpecDecoder(eng, B, k=k, draft_layers=9, temperature=0.7)
    rng = np.random.default_rng(3)
    sd.steps(seqs, 3, rng)
    n0 = sum(len(s.generated) for s in seqs)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    acc = sd.steps(seqs, steps, rng)
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    toks = sum(len(s.generated) for s in seqs) - n0
    parts = sd.time_parts()
    for s in seqs:
        eng.release(s)
    del sd
    # plain greedy decode of the same batch on the same model, for comparison
    plain = make_seqs(eng, Sequence, B, ctx, model.args.vocab_size, seed=22)
    ms_plain, _ = time_device_resident(eng, plain, steps, 3)
    for s in plain:
        eng.release(s)
    # acceptance per draft position alpha (E[accepted] = alpha + ... + alpha^k), and the alpha
    # at which a speculative step (its measured device parts) yields as many tokens per ms as
    # the plain step: (1 - alpha^(k+1)) / (1 - alpha) = spec ms / plain ms
    def tokens(al):
        return float(sum(al ** i for i in range(k + 1)))

    def solve(target):
        lo, hi = 0.0, 1.0
        for _ in range(60):
            mid = 0.5 * (lo + hi)
            lo, hi = (mid, hi) if tokens(mid) < target else (lo, mid)
        return lo
    spec_ms = sum(parts.values())
    plain_ms = ms_plain / steps
    return {"workload": "qwen3-8b self-spec B=4 ctx 2048, draft 9 layers, k=5, T=0.7; e2e",
            "tok_s": round(toks / dt, 1), "ms_per_spec_step": round(dt * 1e3 / steps, 3),
            "accepted_per_step_mean": round(float(acc.mean()), 3),
            "tokens_per_step_mean": round(float(acc.mean()) + 1.0, 3),
            "acceptance_per_draft": round(solve(float(acc.mean()) + 1.0), 3),
            "break_even_acceptance": (round(solve(spec_ms / plain_ms), 3)
                                      if spec_ms / plain_ms < k + 1 else None),
            "parts_device": parts,
            "plain_greedy_b4": {"tok_s": round(B * steps / (ms_plain / 1e3), 1),
                                "ms_per_step": round(plain_ms, 4)}}


def config_c4(device, hbm, steps, world=1, rank=0):
    """C4: Qwen3-30B-A3B arch (128 experts, top-8), B=32 decode at ctx 4096; on N GPUs
    attention is tensor parallel and the experts are split over the ranks (expert
    parallelism), both reduced by the peer-memory all-reduce.  Returns (entry, parity,
    errors): on N GPUs, the greedy parity of the sharded model against the unsharded
    weights on one GPU and the count of collectives that timed out; (entry, None, 0) on one."""
    import torch

    from higgs_b200.engine import Engine, Sequence
    from higgs_b200.model import PRESETS, Model, shard_weights, synth_weights_device
    a = PRESETS["qwen3-30b-a3b"]
    B, ctx = 32, 4096
    pages = B * math.ceil((ctx + steps + 16) / 16) + 16
    w = synth_weights_device(a, seed=0, device=device)
    tp = None
    full = None
    if world > 1:
        full = w
        w = shard_weights(a, w, rank, world)
        tp = make_tp_group(a, rank, world, B, device)
    model = Model(a, w, num_pages=pages, device=device, tp=tp)
    _fill_kv(model)
    eng = Engine(model, max_seq_len=ctx + steps + 16, prefix_entries=0)
    seqs = make_seqs(eng, Sequence, B, ctx, a.vocab_size, seed=31)
    ms, _ = time_device_resident(eng, seqs, steps, 4)
    ms = allmax(ms)
    touched = 128 * (1 - (1 - 8 / 128) ** B)  # expected distinct experts per layer
    out = _entry(a, B, ctx + steps // 2, ms / steps, hbm, experts_touched=touched,
                 extra={"workload": "qwen3-30b-a3b B=32 ctx 4096 greedy (router logits N(0,1))",
                        "experts_touched_per_layer": round(touched, 1),
                        "parallelism": f"tp{world} attention + ep{world} experts" if world > 1 else "single GPU"})
    if world > 1:
        out["step_hbm_frac"] = round(out["step_hbm_frac"] / world, 4)  # per-GPU bytes
    for s_ in seqs:
        eng.release(s_)
    parity, errors = None, 0
    if world > 1:
        errors = int(allmax(float(comm_errors(model))))
        del eng
        torch.cuda.empty_cache()
        parity = tp_parity(a, full, model, device)
        errors += int(allmax(float(comm_errors(model))))
    del model, w, full
    torch.cuda.empty_cache()
    return out, parity, errors


def config_c5(weights, device, hbm, steps):
    """C5: Qwen3-8B with TurboQuant 4-bit KV pages, B=16 at ctx 32768."""
    import torch

    from higgs_b200.engine import Engine, Sequence
    from higgs_b200.model import PRESETS
    a = PRESETS[MODEL]
    B, ctx = 16, 32768
    pages = B * math.ceil((ctx + steps + 16) / 16) + 16
    model, _ = _synth_model(a, device, num_pages=pages, kv_mode="tq4", weights=weights)
    _fill_kv(model)
    eng = Engine(model, max_seq_len=ctx + steps + 16, prefix_entries=0)
    seqs = make_seqs(eng, Sequence, B, ctx, a.vocab_size, seed=51)
    ms, _ = time_device_resident(eng, seqs, steps, 4)
    out = _entry(a, B, ctx + steps // 2, ms / steps, hbm, kv_mode="tq4",
                 extra={"workload": "qwen3-8b TurboQuant KV B=16 ctx 32768 greedy"})
    del eng, model
    torch.cuda.empty_cache()
    return out


def ncu_traffic(rows):
    """Per-launch DRAM bytes (read + write) of the W4 GEMV launches of one step, from the
    committed ncu summary (profiles/qgemv_m1_dram_traffic.json: dram__bytes_read.sum +
    dram__bytes_write.sum per shape, captured on the --kernel-case runs); null if absent."""
    path = os.path.join(ROOT, "profiles", "qgemv_m1_dram_traffic.json")
    try:
        with open(path) as f:
            per = json.load(f)["dram_bytes_per_launch"]
        tot = sum(per[r["shape"]] * r["launches_per_step"] for r in rows)
        return int(tot / sum(r["launches_per_step"] for r in rows))
    except (OSError, KeyError, ValueError):
        return None


def bench_config(ws: int, B: int, ctx: int) -> dict:
    """The headline workload (shared by both arms)."""
    return {"workload": f"{MODEL} decode B={B} ctx={ctx}", "model": MODEL, "global_batch": B,
            "seq_len": ctx, "parallelism": f"tp{ws} (peer-memory all-reduce)" if ws > 1 else "single GPU",
            "l2": "weights 4.26 GB/step > 126 MB L2 (no flush needed)"}


def run_ours(opt):
    import torch

    from higgs_b200.model import PRESETS
    ws, rank, local = dist_setup()
    device = f"cuda:{local}"
    torch.cuda.set_device(local)
    a = PRESETS[MODEL]
    batches = [int(b) for b in opt.batches.split(",")]
    if opt.quick:
        batches = batches[:1]
    total_steps = 2 * (opt.steps + opt.warmup) + 4
    model, eng, Sequence, full_weights = setup_model(a, batches, opt.ctx, total_steps, device, ws, rank)
    hbm, peak_kind = peaks()
    w_bytes = a.weight_bytes_per_step()
    by_batch = {}
    gpu_launches = None
    clocks = None
    for B in batches:
        seqs = make_seqs(eng, Sequence, B, opt.ctx, a.vocab_size, seed=1)  # same on every rank
        with ClockSampler(local) as cs:
            ms, nk = time_device_resident(eng, seqs, opt.steps, opt.warmup)
        ms = allmax(ms)
        # KV bytes read per step: every sequence's context (average over the timed steps)
        kv_bytes = B * (opt.ctx + opt.warmup + opt.steps // 2) * a.kv_bytes_per_token()
        step_ms = ms / opt.steps
        tok_s = B * opt.steps / (ms / 1e3)  # one model over all ranks (tensor parallel)
        gpu_bytes = (w_bytes + kv_bytes) / ws  # each rank streams its shard
        by_batch[str(B)] = {"tok_s": round(tok_s, 1), "ms_per_step": round(step_ms, 4),
                            "step_bytes": int(w_bytes + kv_bytes),
                            "step_hbm_frac": round(gpu_bytes / (step_ms / 1e3) / 1e9 / hbm, 4)}
        if B == batches[0]:
            clocks = cs.summary()
            gpu_launches = nk * opt.steps if nk else None
            head = (B, ms, step_ms, tok_s, seqs)
        for s in seqs:
            eng.release(s)
    B, ms, step_ms, tok_s, _ = head
    # e2e through the public API at the headline batch
    seqs = make_seqs(eng, Sequence, B, opt.ctx, a.vocab_size, seed=11)
    e2e_ms = allmax(time_e2e(eng, seqs, opt.steps, opt.warmup))
    for s in seqs:
        eng.release(s)
    e2e_tok_s = B * opt.steps / (e2e_ms / 1e3)
    n_comm_err = int(allmax(float(comm_errors(model))))
    out = {
        "metric": METRIC, "value": round(tok_s, 1), "unit": "tok/s", "n_gpus": ws,
        "steps": opt.steps, "warmup": opt.warmup, "ms_per_step": round(step_ms, 4),
        "higher_is_better": True, "scaling": "strong" if ws > 1 else "weak", "vs_baseline": None,
        "dtype": "w4a16 (u4 weights, bf16 act, f32 acc)",
        "data": "synthetic: random-init N(0,0.02) W4 g64 weights, random KV context, uniform token ids",
        "config": bench_config(ws, B, opt.ctx),
        "by_batch": by_batch,
        "e2e": {"value": round(e2e_tok_s, 1), "unit": "tok/s", "h2d_bytes_per_step": 16 * B,
                "d2h_bytes_per_step": 4 * B},
        "gpu_launches": gpu_launches, "clocks": clocks, "comm_errors": n_comm_err,
    }
    if ws > 1:
        parity = {"dense_b1": tp_parity(a, full_weights, model, device)}
        del full_weights
        torch.cuda.empty_cache()
        parity_err = int(allmax(float(comm_errors(model))))
    if rank == 0 and not opt.quick:
        rows = gemv_roofline(model)
        tot_bytes = sum(r["bytes"] * r["launches_per_step"] for r in rows)
        tot_us = sum(r["us"] * r["launches_per_step"] for r in rows)
        gemv_achieved = tot_bytes / tot_us / 1e3
        out["roofline"] = {"kernel": "qgemv_m1_kernel (every W4 GEMV launch of one B=1 step; per-launch "
                                     "averages, byte-weighted over shapes)",
                           "bound": "hbm", "achieved": round(gemv_achieved, 1), "peak": hbm,
                           "peak_kind": peak_kind, "unit": "GB/s", "frac": round(gemv_achieved / hbm, 4),
                           "algorithmic_bytes": int(tot_bytes / sum(r["launches_per_step"] for r in rows)),
                           # the committed capture is of one-GPU shapes: no figure for a TP shard
                           "traffic": ncu_traffic(rows) if ws == 1 else None, "per_shape": rows}
        if ws == 1 and opt.chain_roofline:
            # the persistent decode chain (off in the step by default), timed the same way
            cb, cus = chain_roofline(model)
            out["chain_roofline"] = {"kernel": "chain_kernel (o_proj + gate/up + down + next q|k|v)",
                                     "achieved": round(cb / cus / 1e3, 1), "frac": round(cb / cus / 1e3 / hbm, 4),
                                     "algorithmic_bytes": cb, "us_per_launch": round(cus, 2)}
        if ws == 1:
            out["prefill_attention"] = prefill_attn_roofline(a, device)
        sb = by_batch[str(B)]["step_bytes"]
        out["step_roofline"] = {"bytes_per_step": sb, "achieved_gbs": round(sb / (step_ms / 1e3) / 1e9, 1),
                                "peak": hbm, "frac": by_batch[str(B)]["step_hbm_frac"]}
    if rank == 0 and ws == 1 and not opt.quick and opt.configs:
        cfgs = {}
        n = 16
        want = opt.configs.split(",")
        if "c3" in want:
            cfgs["C3"] = config_c3(model, eng, Sequence, device, hbm, n, opt.ctx)
        weights = model.weights
        if "c5" in want:
            cfgs["C5"] = config_c5(weights, device, hbm, n)
        if "c1" in want:
            cfgs["C1"] = config_c1(device, hbm, 64)
        if "c2" in want:
            cfgs["C2"] = config_c2(device, hbm, 64)
        if "c4" in want:
            del eng, model, weights
            import gc
            gc.collect()
            torch.cuda.empty_cache()
            cfgs["C4"] = config_c4(device, hbm, n)[0]
        out["by_config"] = cfgs
    elif ws > 1 and not opt.quick and "c4" in opt.configs.split(","):
        del eng, model
        import gc
        gc.collect()
        torch.cuda.empty_cache()
        c4, c4_parity, c4_err = config_c4(device, hbm, 16, ws, rank)  # every rank takes part
        parity["c4_ep"] = c4_parity
        parity_err += c4_err
        if rank == 0:
            out["by_config"] = {"C4": c4}
    if ws > 1:
        out["tp_parity"] = parity
        out["comm_errors"] += parity_err
    if rank == 0 and ws == 1 and not opt.no_cpu_baseline and not opt.quick:
        sec, desc, threads = oracle_step_time(a, opt.ctx)
        out["cpu_baseline"] = {"value": round(1.0 / sec, 4), "unit": "tok/s", "cores": threads,
                               "kind": "port", "sample": desc}
    if rank == 0:
        print(json.dumps(out), flush=True)
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()


# ---------------------------------------------------------------------------------------------
# reference arm: the reference path's arithmetic restated on the host (oracle port)
# ---------------------------------------------------------------------------------------------
def run_reference(opt):
    """The reference path restated on the host (oracle port), all host threads, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from higgs_b200.model import PRESETS
    a = PRESETS[MODEL]
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    B = int(opt.batches.split(",")[0])
    sec, desc, threads = oracle_step_time(a, opt.ctx)
    v = 1.0 / sec
    out = {"impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "tok/s", "n_gpus": ws,
           "steps": opt.steps, "warmup": opt.warmup, "ms_per_step": round(sec * 1e3, 2),
           "higher_is_better": True, "scaling": "strong" if ws > 1 else "weak", "vs_baseline": None,
           "dtype": "w4a16 (u4 weights, bf16 act, f32 acc)",
           "data": "synthetic packed W4 weights and random KV context",
           "config": bench_config(ws, B, opt.ctx),
           "cpu_baseline": {"value": round(v, 4), "unit": "tok/s", "cores": threads, "kind": "port",
                            "sample": desc + "; the reference's own mlx-rs CPU backend cannot be built here "
                                             "(no Rust toolchain, MLX not vendored)"},
           "e2e": {"value": round(v, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def main():
    opt = parse()
    if opt.option and opt.impl != "reference":
        from higgs_b200 import ffi
        for o in opt.option:
            name, _, val = o.partition("=")
            ffi.call("higgs_set_option", name.encode(), int(val))
    if opt.kernel_case:
        kernel_case(opt)
    elif opt.impl == "reference":
        run_reference(opt)
    else:
        run_ours(opt)


if __name__ == "__main__":
    main()
