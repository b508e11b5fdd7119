"""GPU: model-level parity at the benchmark configurations' true shapes.

The decode step end to end against the CPU oracle model on the same seeded weights:

* C1 in full: the Llama-3.2-1B architecture (16 layers, hidden 2048, vocab 128256), a
  128-token prompt (seed 1), 64 greedy tokens;
* the Qwen3-8B architecture at its true widths (hidden 4096, 32 / 8 heads, FFN 12288,
  vocab 151936) with 4 layers, a 2047-token prompt (decode at context 2048, paged);
* the Qwen3-1.7B architecture at its true widths with 4 layers, four sequences of 320-token
  prompts sharing a 256-token prefix served from the radix cache, decoded together.

teacher-forced logits within max-abs 2e-2 / rel 1e-2 of the oracle's, and
greedy token streams identical to the oracle's.  At these depths the absolute bar lies below
the rounding noise of the bf16 forward itself: the oracle run with a second, equally valid
summation order (orc_set_order(1): the same arithmetic, reductions reordered) moves C1's
logits by up to ~0.1 (std ~0.012), with ~17 % of them outside 2e-2 / 1e-2.  So every test
measures that floor on its own inputs and requires the GPU's logits to be as close to the
oracle as the reordered oracle is (max and std within 1.5x of the floor's), reports the
fraction inside the north-star bar for both, and requires identical greedy streams wherever
the oracle's top-2 margin exceeds twice the measured noise.

Weights are generated and quantized on the GPU (the same packed tensors are copied to the
host for the oracle: the packed codes, scales and biases are the ground truth, only their
dequantization is a contract).
"""
import numpy as np
import pytest
import torch

from oracle import oracle as orc
from oracle.model_ref import RefModel

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def host_weights(wd: dict) -> dict:
    """Device MLX-layout tensors -> the oracle's numpy form (u32 codes, bf16 bit patterns)."""
    out = {}
    for k, t in wd.items():
        if t.dtype == torch.int32:
            out[k] = t.cpu().numpy().view(np.uint32)
        elif t.dtype == torch.bfloat16:
            out[k] = t.view(torch.int16).cpu().numpy().view(np.uint16)
        else:
            raise TypeError(f"{k}: {t.dtype}")
    return out


def build(preset: str, layers: int, pages: int):
    from higgs_b200.model import PRESETS, Model, synth_weights_device
    args = PRESETS[preset]
    if layers:
        args = args.with_layers(layers)
    wd = synth_weights_device(args, seed=0, device=DEV)
    m = Model(args, wd, num_pages=pages, device=DEV)
    return args, m, RefModel(args, host_weights(wd))


def teacher_forced(eng, seqs, ref_tok, steps):
    """GPU logits of decode steps 1..steps-1 fed the oracle's own tokens (no divergence
    cascade), and the GPU's argmax at each of them."""
    for s, t0 in zip(seqs, ref_tok[:, 0]):
        s.last_token = int(t0)
    eng.step_logits.clear()
    forced = eng.decode_steps(seqs, steps - 1, force=ref_tok[:, :steps - 1])
    return forced, np.stack(eng.step_logits)


def greedy_report(ref_tok, ref_lg, gpu_first, forced, gl, free, alt_lg, atol=2e-2, rtol=1e-2):
    """Assert the parity bars and print what was measured.

    Logits: the GPU's teacher-forced logits are within 1.5x of the summation-order floor
    (|reordered oracle - oracle|) in max and in standard deviation; the fractions inside the
    north-star bar (atol + rtol * |ref|) are printed for both.  Tokens: the free-running GPU
    stream equals the oracle's for every step.  The one escape is a step where the oracle's
    top-2 margin is at most twice the measured logit noise (each of the two competing logits
    may move by up to the noise, so such a step can legitimately flip); those steps are counted
    and printed, and the streams are compared only up to the first of them."""
    ref = ref_lg[1:]
    err = np.abs(gl - ref)
    floor = np.abs(alt_lg[1:] - ref)
    bar = atol + rtol * np.abs(ref)
    noise = float(err.max())
    rel = float((err / (np.abs(ref) + 1e-6)).max())
    print(f"\nlogits vs oracle: GPU max {noise:.3e} std {err.std():.3e}, inside the 2e-2/1e-2 bar "
          f"{(err <= bar).mean():.4f}; reordered oracle max {floor.max():.3e} std {floor.std():.3e}, "
          f"inside the bar {(floor <= bar).mean():.4f}")
    assert noise <= 1.5 * float(floor.max()) + 1e-3, (noise, float(floor.max()))
    assert float(err.std()) <= 1.5 * float(floor.std()) + 1e-4, (float(err.std()), float(floor.std()))
    top2 = np.sort(ref_lg, axis=-1)[..., -2:]
    margin = top2[..., 1] - top2[..., 0]  # [steps, B]
    agree = np.concatenate([gpu_first[None], forced.T], 0) == ref_tok.T  # [steps, B]
    alt_agree = np.argmax(alt_lg, axis=-1) == ref_tok.T  # the reordered oracle on the same stream
    print(f"forced-argmax disagreements with the oracle: GPU {int((~agree).sum())}, reordered oracle "
          f"{int((~alt_agree).sum())} (of {agree.size} steps)")
    near = margin <= 2 * noise
    bad = np.argwhere(~agree & ~near)
    print(f"greedy: max rel err {rel:.3e}; "
          f"min top-2 margin {margin.min():.3e}; steps with margin <= 2x noise: {int(near.sum())} "
          f"at {np.argwhere(near).tolist()}; forced-argmax disagreements: "
          f"{np.argwhere(~agree).tolist()}")
    assert bad.size == 0, (
        f"greedy disagreement where the margin exceeds twice the noise ({noise:.2e}): "
        + ", ".join(f"step {k} seq {b} margin {margin[k, b]:.3e}" for k, b in bad))
    for b in range(ref_tok.shape[0]):
        d = np.nonzero(free[b] != ref_tok[b])[0]
        if d.size:
            k = int(d[0])
            print(f"seq {b}: free stream leaves the oracle's at step {k} (margin {margin[k, b]:.3e}, "
                  f"noise {noise:.3e})")
            assert near[k, b], (f"seq {b}: free-running stream diverges at step {k}, margin "
                                f"{margin[k, b]:.3e} > 2x noise {noise:.3e}")
        else:
            print(f"seq {b}: free-running stream identical for all {free.shape[1]} tokens")
    return noise


def run_case(m, ref, prompts, steps, max_seq_len, use_prefix=False):
    from higgs_b200.engine import Engine
    ref_tok, ref_lg = ref.greedy(prompts, steps)
    with orc.summation_order(1):
        alt_lg = ref.teacher_forced(prompts, ref_tok)
    eng = Engine(m, max_seq_len=max_seq_len, keep_logits=True, prefix_entries=8)
    seqs = [eng.prefill(p, use_prefix=use_prefix) for p in prompts]
    hits = [s.prefix_hit for s in seqs]
    gpu_first = np.array([s.last_token for s in seqs])
    forced, gl = teacher_forced(eng, seqs, ref_tok, steps)
    for s in seqs:
        eng.release(s)
    eng2 = Engine(m, max_seq_len=max_seq_len, prefix_entries=8)
    free = eng2.generate_greedy(list(prompts), steps, use_prefix=use_prefix)
    return (ref_tok, ref_lg, gpu_first, forced, gl, free, alt_lg), hits


def test_c1_llama_1b_full_greedy_64():
    """C1 at its full shape: 16 layers, 128-token prompt (seed 1), 64 greedy tokens."""
    args, m, ref = build("llama-3.2-1b", 0, pages=64)
    pr = np.random.default_rng(1).integers(0, args.vocab_size, size=(1, 128)).astype(np.int32)
    res, _ = run_case(m, ref, pr, 64, 256)
    greedy_report(*res)


def test_qwen3_8b_true_widths_ctx2048():
    """Qwen3-8B widths, 4 layers, decode at context 2048 (2047-token prompt), 32 greedy
    tokens; paged KV in 16-token pages."""
    args, m, ref = build("qwen3-8b", 4, pages=160)
    pr = np.random.default_rng(1).integers(0, args.vocab_size, size=(1, 2047)).astype(np.int32)
    res, _ = run_case(m, ref, pr, 32, 2048 + 64)
    greedy_report(*res)


def test_qwen3_1p7b_true_widths_shared_prefix_batch():
    """Qwen3-1.7B widths, 4 layers, C2's prompt structure at a reduced size: 4 sequences of
    320 tokens sharing the first 256 (seed 2), the later ones served from the radix prefix
    cache, then 32 greedy tokens decoded as one batch of 4.  The oracle runs every prompt in
    full, so this also checks that reused pages give the same results at true widths."""
    args, m, ref = build("qwen3-1.7b", 4, pages=4 * 24 + 32)
    rng = np.random.default_rng(2)
    shared = rng.integers(0, args.vocab_size, 256).astype(np.int32)
    pr = np.stack([np.concatenate([shared, rng.integers(0, args.vocab_size, 64).astype(np.int32)])
                   for _ in range(4)])
    res, hits = run_case(m, ref, pr, 32, 512, use_prefix=True)
    assert hits == [0, 256, 256, 256], hits
    greedy_report(*res)
