"""GPU: the native decode step end to end against the CPU reference model.

logits within max-abs 2e-2 / rel 1e-2 (bf16 path, f32 logits)
and greedy token streams identical for the first 64 tokens.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from oracle.model_ref import RefModel, synth_weights_numpy

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def build(model_type, layers=2, kv_mode="bf16", pages=256):
    from higgs_b200.model import Model, hadamard_signs, tiny_args, weights_to_device
    args = tiny_args(model_type, layers)
    w = synth_weights_numpy(args, seed=0)
    signs = hadamard_signs()
    m = Model(args, weights_to_device(w, DEV), num_pages=pages, kv_mode=kv_mode, device=DEV,
              signs=signs)
    return args, w, m, signs


def prompts(args, B, P, seed=1):
    rng = np.random.default_rng(seed)
    return rng.integers(0, args.vocab_size, size=(B, P)).astype(np.int32)


def first_divergence(a, b):
    d = np.nonzero(a != b)[0]
    return int(d[0]) if d.size else -1


def check_against_oracle(m, ref, pr, steps, max_seq_len=256):
    """Teacher-forced parity: the GPU decodes the oracle's own token stream, so every step
    compares logits for identical inputs (no divergence cascade).  Returns the free-running
    stream, the oracle stream and per-step logits errors."""
    from higgs_b200.engine import Engine
    B = pr.shape[0]
    ref_tok, ref_lg = ref.greedy(pr, steps)
    eng = Engine(m, max_seq_len=max_seq_len, keep_logits=True)
    seqs = [eng.prefill(p, use_prefix=False) for p in pr]
    gpu_first = np.array([s.last_token for s in seqs])
    for s, t0 in zip(seqs, ref_tok[:, 0]):
        s.last_token = int(t0)
    forced_argmax = eng.decode_steps(seqs, steps - 1, force=ref_tok[:, :steps - 1])
    gl = np.stack(eng.step_logits)  # [steps-1, B, V], logits after feeding ref_tok[:, k]
    for s in seqs:
        eng.release(s)
    free = Engine(m, max_seq_len=max_seq_len).generate_greedy(list(pr), steps, use_prefix=False)
    return ref_tok, ref_lg, gpu_first, forced_argmax, gl, free


def assert_greedy_parity(ref_tok, ref_lg, gpu_first, forced_argmax, gl, free, atol=2e-2, rtol=1e-2):
    np.testing.assert_allclose(gl, ref_lg[1:], atol=atol, rtol=rtol)
    noise = float(np.max(np.abs(gl - ref_lg[1:])))
    # greedy agreement wherever the oracle's top-2 margin exceeds twice the measured noise
    top2 = np.sort(ref_lg, axis=-1)[..., -2:]
    margin = top2[..., 1] - top2[..., 0]  # [steps, B]
    agree = np.concatenate([gpu_first[None], forced_argmax.T], 0) == ref_tok.T
    ties = margin <= 2 * noise
    assert np.all(agree | ties), (
        f"greedy disagreement at a margin above the noise ({noise:.2e}): "
        f"{np.argwhere(~agree & ~ties).tolist()}")
    # free-running streams identical up to the first near-tie (or for all steps)
    for b in range(ref_tok.shape[0]):
        d = np.nonzero(free[b] != ref_tok[b])[0]
        if d.size:
            k = int(d[0])
            assert ties[k, b], f"seq {b}: free stream diverges at {k} with margin {margin[k, b]:.2e} > 2x noise {noise:.2e}"
    return noise


@pytest.mark.parametrize("model_type", ["qwen3", "llama"])
def test_greedy_stream_and_logits_match_oracle(model_type):
    args, w, m, _ = build(model_type)
    pr = prompts(args, 2, 20)
    res = check_against_oracle(m, RefModel(args, w), pr, 64)
    assert_greedy_parity(*res)


def test_graph_replay_equals_eager():
    from higgs_b200.engine import Engine
    args, w, m, _ = build("qwen3")
    pr = prompts(args, 3, 17, seed=5)
    a = Engine(m, max_seq_len=128, use_graph=True).generate_greedy(list(pr), 24, use_prefix=False)
    b = Engine(m, max_seq_len=128, use_graph=False).generate_greedy(list(pr), 24, use_prefix=False)
    assert np.array_equal(a, b)


def test_prefix_cache_reuse_is_exact():
    """A prompt whose first 32 tokens hit the radix cache decodes exactly as a cold prompt."""
    from higgs_b200.engine import Engine
    args, w, m, _ = build("qwen3")
    rng = np.random.default_rng(9)
    shared = rng.integers(0, args.vocab_size, size=40).astype(np.int32)
    p1 = np.concatenate([shared, rng.integers(0, args.vocab_size, size=5).astype(np.int32)])
    p2 = np.concatenate([shared, rng.integers(0, args.vocab_size, size=9).astype(np.int32)])
    eng = Engine(m, max_seq_len=256)
    s1 = eng.prefill(p1)
    assert s1.prefix_hit == 0
    s2 = eng.prefill(p2)
    assert s2.prefix_hit == 32  # whole pages of the shared 40 tokens
    assert s2.pages[:2] == s1.pages[:2]
    hot = eng.decode_steps([s1, s2], 16)
    cold_eng = Engine(m, max_seq_len=256)
    c1, c2 = cold_eng.prefill(p1, use_prefix=False), cold_eng.prefill(p2, use_prefix=False)
    assert (s1.last_token, s2.last_token) != (-1, -1)
    cold = cold_eng.decode_steps([c1, c2], 16)
    assert np.array_equal(hot, cold)


def test_tq4_kv_model_matches_oracle():
    """TurboQuant KV end to end.  Codes are bit-exact given the same bf16 K/V
    (test_tq4_kv_write_bit_exact), but the GPU and the CPU reach K/V through
    different f32 summation orders, and a 1-ulp K/V difference can move a 4-bit
    code by a whole step.  Measured on the oracle alone (1-ulp noise on 1% of
    the Q/K elements): TQ4 logits move by 1.6e-2 mean / 0.10 max, bf16-KV logits
    by 2.7e-3 / 1.4e-2.  The bounds below are that TQ4 noise band; greedy
    agreement is still required wherever the top-2 margin exceeds it."""
    args, w, m, signs = build("qwen3", kv_mode="tq4")
    pr = prompts(args, 1, 24, seed=3)
    res = check_against_oracle(m, RefModel(args, w, kv_mode="tq4", signs=signs), pr, 32)
    gl, ref_lg = res[4], res[1][1:]
    assert float(np.mean(np.abs(gl - ref_lg))) < 1.6e-2
    assert_greedy_parity(*res, atol=1e-1, rtol=1e-2)


def test_layer_skip_draft_forward():
    """n_layers truncation (self-speculative draft) equals a model with fewer layers."""
    from higgs_b200.model import Model, weights_to_device
    args, w, m, _ = build("qwen3", layers=3)
    pr = prompts(args, 1, 18, seed=4)
    ref = RefModel(args, w)
    caches = [ref.new_cache()]
    ref_lg = ref.forward(pr, caches, n_layers=1)[:, -1]
    dev = torch.device(DEV)
    n = pr.shape[1]
    pos = torch.arange(n, dtype=torch.int32, device=dev).view(1, n)
    slots = torch.arange(n, dtype=torch.int64, device=dev).view(1, n)
    bt = torch.arange(4, dtype=torch.int32, device=dev).view(1, 4)
    lg, am = m.forward(torch.from_numpy(pr).to(dev), pos, slots, bt,
                       torch.tensor([n], dtype=torch.int32, device=dev), 64, n_layers=1, last_only=True)
    np.testing.assert_allclose(lg.cpu().numpy(), ref_lg, atol=2e-2, rtol=1e-2)


def test_moe_model_matches_oracle():
    """Qwen3-MoE decode step (router -> plan -> grouped experts -> combine, plus one dense
    layer from mlp_only_layers) teacher-forced against the oracle model.

    Expert choice is a discontinuous function of the router logits: where the oracle's k-th
    and (k+1)-th logits of a step lie within one bf16 ulp, a last-bit difference upstream may
    swap an expert on one side only.  Those (step, sequence) rows are excluded from the
    logits bound (and must stay a small minority).  Every other row meets the dense bar, or --
    where the oracle's own rounding noise reaches past it -- stays within 1.5x of the noise
    the oracle shows under a second valid summation order (orc_set_order(1))."""
    args, w, m, _ = build("qwen3_moe", layers=3)
    assert [args.is_moe_layer(i) for i in range(3)] == [True, False, True]
    pr = prompts(args, 2, 20, seed=3)
    ref = RefModel(args, w)
    ref_tok, ref_lg, gpu_first, forced, gl, free = check_against_oracle(m, ref, pr, 24)
    near = ref.step_route_near[1:]  # rows of gl
    assert near.mean() < 0.35, f"too many near-tie routings: {near.mean():.2f}"
    keep = ~near
    with orc.summation_order(1):
        alt = ref.teacher_forced(pr, ref_tok)
    err = np.abs(gl[keep] - ref_lg[1:][keep])
    floor = np.abs(alt[1:][keep] - ref_lg[1:][keep])
    inside = err <= 2e-2 + 1e-2 * np.abs(ref_lg[1:][keep])
    print(f"\nMoE logits: max {err.max():.3e} std {err.std():.3e} inside the bar {inside.mean():.4f}; "
          f"reordered oracle max {floor.max():.3e} std {floor.std():.3e}")
    assert inside.all() or (err.max() <= 1.5 * floor.max() + 1e-3
                            and err.std() <= 1.5 * floor.std() + 1e-4)
    agree = forced.T == ref_tok[:, 1:].T
    top2 = np.sort(ref_lg[1:], axis=-1)[..., -2:]
    margin = top2[..., 1] - top2[..., 0]
    assert np.all(agree | ~keep | (margin <= 4e-2)), np.argwhere(~agree & keep & (margin > 4e-2)).tolist()


def test_spec_decode_greedy_equals_plain_greedy():
    """At temperature 0 self-speculative decoding must emit the target's greedy stream,
    whatever the draft proposes (accepted drafts equal the target argmax and the correction
    is the target argmax).  The verify forward runs 6 tokens per sequence through kernels
    sized for that, plain decoding one, so their f32 sums may differ in the last bits: the
    streams must agree up to the first step whose top-2 logit margin is below 2e-2."""
    from higgs_b200.engine import Engine, SpecDecoder
    args, w, m, _ = build("qwen3", layers=4, pages=512)
    pr = prompts(args, 2, 20, seed=7)
    eng = Engine(m, max_seq_len=256, keep_logits=True)
    n = 40
    ref = eng.generate_greedy(list(pr), n, use_prefix=False)
    lg = np.stack(eng.step_logits)  # [n-1, B, V]: logits that chose tokens 1..n-1
    top2 = np.sort(lg, axis=-1)[..., -2:]
    margin = top2[..., 1] - top2[..., 0]
    eng = Engine(m, max_seq_len=256)
    seqs = [eng.prefill(p, use_prefix=False) for p in pr]
    sd = SpecDecoder(eng, 2, k=5, draft_layers=1, temperature=0.0)
    rng = np.random.default_rng(3)
    acc = []
    while min(len(s.generated) for s in seqs) < n - 1:
        acc.append(sd.steps(seqs, 1, rng))
    for b, s in enumerate(seqs):
        got = np.array([ref[b, 0]] + s.generated[:n - 1])
        d = np.nonzero(got != ref[b])[0]
        if d.size:
            k = int(d[0])
            assert k >= 1 and margin[k - 1, b] < 2e-2, f"seq {b}: diverges at {k}, margin {margin[k - 1, b]:.3g}"
        eng.release(s)
    assert np.concatenate(acc).max() <= 5


def test_spec_decode_sampled_step_matches_oracle_accept():
    """Temperature 0.7: each draft token is the oracle's inverse-CDF draw from the GPU's draft
    logits with the staged uniform, and the accepted counts / emitted tokens are the oracle's
    spec_accept of the GPU's target and draft logits (layouts and uniform slicing of the
    captured step), over several steps."""
    from higgs_b200.engine import Engine, SpecDecoder
    args, w, m, _ = build("qwen3", layers=3, pages=512)
    pr = prompts(args, 2, 18, seed=9)
    eng = Engine(m, max_seq_len=256)
    seqs = [eng.prefill(p, use_prefix=False) for p in pr]
    B, k, T = 2, 4, 0.7
    sd = SpecDecoder(eng, B, k=k, draft_layers=1, temperature=T)
    rng = np.random.default_rng(3)
    total_acc = 0
    for it in range(6):
        u = rng.random(2 * k * B + B, dtype=np.float32)
        sd.stage(seqs, u, first=(it == 0))
        sd.graph.replay()
        torch.cuda.synchronize()
        dl = sd.draft_logits.cpu().numpy()
        drafts = sd.tok[1:].cpu().numpy()
        for i in range(k):
            assert np.array_equal(drafts[i], orc.sample(dl[i], T, u[i * B:(i + 1) * B])), (it, i)
        acc_ref, tok_ref = orc.spec_accept(sd.target_logits.cpu().numpy(), sd.draft_bkv.cpu().numpy(),
                                           sd.dtok.cpu().numpy(), T, u[k * B:2 * k * B].reshape(B, k),
                                           u[2 * k * B:])
        acc = sd.accepted.cpu().numpy()
        toks = sd.out_tokens.cpu().numpy()
        assert np.array_equal(acc, acc_ref)
        for b in range(B):
            assert np.array_equal(toks[b, :acc[b] + 1], tok_ref[b, :acc[b] + 1])
        total_acc += int(acc.sum())
        last = np.empty(B, np.int32)
        for b, s in enumerate(seqs):
            s.length += int(acc[b]) + 1
            s.last_token = int(toks[b, acc[b]])
            last[b] = s.last_token
        sd.tok[0].copy_(torch.from_numpy(last))
    for s in seqs:
        eng.release(s)


def test_sampled_decode_processors_match_oracle():
    """Sampled decode through Engine.decode_steps_sampled: every step's logits pass through the
    penalties (over the generated tokens), the constraint mask, the top-k / top-p / min-p draw
    and logprobs on the device, in the reference's order (simple.rs:318-347).  Each step is
    checked bit for bit against the oracle's processors applied to the same raw logits with
    the same uniforms (the draws, masked tokens and penalised values are integer / exact)."""
    from higgs_b200.engine import Engine, SamplingParams
    args, w, m, _ = build("qwen3")
    pr = prompts(args, 2, 16, seed=21)
    eng = Engine(m, max_seq_len=128, keep_logits=True)
    seqs = [eng.prefill(p, use_prefix=False) for p in pr]
    for s in seqs:
        s.generated.append(s.last_token)
    params = SamplingParams(temperature=0.8, top_p=0.9, top_k=50, min_p=0.01,
                            repetition_penalty=1.3, frequency_penalty=0.2, presence_penalty=0.1)
    steps = 12
    rng = np.random.default_rng(5)
    u = rng.random((steps, 2)).astype(np.float32)
    allowed_sets = {k: [rng.choice(args.vocab_size, size=300, replace=False).tolist() for _ in range(2)]
                    for k in range(0, steps, 2)}
    hist0 = [list(s.generated) for s in seqs]
    eng.step_logits.clear()
    toks, lps, tids, tlps = eng.decode_steps_sampled(seqs, steps, params, u, top_logprobs=4,
                                                     allowed=lambda k: allowed_sets.get(k))
    hist = [list(h) for h in hist0]
    for k in range(steps):
        raw = eng.step_logits[k]
        for b in range(2):
            lg = orc.apply_penalties(raw[b], hist[b], params.repetition_penalty,
                                     params.frequency_penalty, params.presence_penalty)[None]
            if k in allowed_sets:
                lg = orc.apply_token_mask(lg, orc.allowed_bits([allowed_sets[k][b]], args.vocab_size))
                assert toks[b, k] in set(allowed_sets[k][b])
            ref = orc.sample_filtered(lg, params.temperature, params.top_k, params.top_p,
                                      params.min_p, u[k, b:b + 1])
            assert toks[b, k] == ref[0], (k, b)
            rlp, rids, rtl = orc.logprobs(lg, params.temperature, toks[b:b + 1, k], 4)
            np.testing.assert_allclose(lps[b, k], rlp[0], atol=1e-6)
            assert np.array_equal(tids[b, k], rids[0])
            np.testing.assert_allclose(tlps[b, k], rtl[0], atol=1e-6)
            hist[b].append(int(toks[b, k]))
    for s in seqs:
        eng.release(s)


def test_model_loaded_from_mlx_checkpoint(tmp_path):
    """An MLX-format directory (config.json + two safetensors files with an index) loaded by
    higgs_b200.loader onto the GPU gives the same device tensors and the same greedy stream as
    the weights it was written from."""
    from higgs_b200.engine import Engine
    from higgs_b200.loader import load_model_args, load_weights
    from higgs_b200.model import Model
    from tests.mlx_checkpoint import write_model_dir
    args, w, m, _ = build("qwen3")
    write_model_dir(str(tmp_path), args, w, shards=2, inner_names=True)
    a2 = load_model_args(str(tmp_path))
    assert a2 == args
    wd = load_weights(str(tmp_path), a2, DEV)
    for k, v in w.items():
        t = wd[k].view(torch.int16) if wd[k].dtype == torch.bfloat16 else wd[k]
        got = t.cpu().numpy().view(v.dtype)
        assert got.shape == v.shape and np.array_equal(got, v), k
    m2 = Model(a2, wd, num_pages=256, device=DEV)
    pr = prompts(args, 2, 20, seed=13)
    a = Engine(m, max_seq_len=128).generate_greedy(list(pr), 16, use_prefix=False)
    b = Engine(m2, max_seq_len=128).generate_greedy(list(pr), 16, use_prefix=False)
    assert np.array_equal(a, b)


@pytest.mark.parametrize("model_type,layers", [("qwen3", 3), ("llama", 2)])
def test_decode_chain_equals_separate_launches(model_type, layers):
    """The persistent decode chain (one-token steps on one GPU) runs each GEMV with the same K
    split and summation order as the separate launches, so logits and tokens are identical
    bit for bit, including the LM head it computes in the last layer's launch."""
    from higgs_b200 import ffi
    from higgs_b200.engine import Engine
    args, w, m, _ = build(model_type, layers=layers)
    pr = prompts(args, 1, 21, seed=17)
    outs = []
    try:
        for on in (1, 0):
            ffi.call("higgs_set_option", b"decode_chain", on)
            eng = Engine(m, max_seq_len=128, keep_logits=True)
            toks = eng.generate_greedy(list(pr), 24, use_prefix=False)
            outs.append((toks, np.stack(eng.step_logits)))
    finally:
        ffi.call("higgs_set_option", b"decode_chain", 0)
    assert np.array_equal(outs[0][0], outs[1][0])
    assert np.array_equal(outs[0][1].view(np.uint32), outs[1][1].view(np.uint32))
    v = ctypes.c_int(-1)
    ffi.call("higgs_tc_error", ffi.ctx(0), ctypes.byref(v))
    assert v.value == 0, "a decode-chain barrier wait gave up"
