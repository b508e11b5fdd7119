"""Per-launch timeline of one decode step at batch 1 (a diagnostic, not a product path).

    python -m higgs_b200.build --timeline      # libhiggs_cuda_timeline.so
    python -m higgs_b200.timeline [--ctx 2048]

Loads the timeline build of the library (the same kernels with per-CTA %globaltimer stamps,
see csrc/timeline.cuh), sets up bench.py's synthetic Qwen3-8B model, replays its captured
B=1 decode step once, and prints for every kind of instrumented launch (the single-token
GEMVs and the fused decode attention) the mean time from its predecessor's completion (its
first CTA past griddepcontrol.wait) to its last CTA's exit ("post"), the mean time from the
previous instrumented launch's end to that release ("gap"), and the fused attention
kernel's phases (per-CTA medians).  ncu serialises launches; this timeline keeps the PDL
overlap of the real step.
"""
from __future__ import annotations

import argparse
import ctypes
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

REC = np.dtype([("tg", "u8"), ("bs", "u8"), ("t0", "u8"), ("t1", "u8"), ("t2", "u8"),
                ("m4", "u8"), ("m5", "u8"), ("m6", "u8")])


def fetch(lib, name: str, reset: bool) -> np.ndarray:
    fn = getattr(lib, name)
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
    n = fn(None, 1 << 30, 0)  # the count (max only caps it)
    if n < 0:
        raise RuntimeError(f"{name} failed")
    buf = np.zeros(max(n, 1), dtype=REC)
    n = fn(buf.ctypes.data, len(buf), 1 if reset else 0)
    if n < 0:
        raise RuntimeError(f"{name} failed")
    return buf[:n]


def launches(r: np.ndarray):
    """Records grouped per launch: every CTA of a launch starts before any CTA of the launch
    that depends on it, so in entry order each launch is `grid` consecutive records."""
    r = r[np.argsort(r["t0"], kind="stable")]
    out, i = [], 0
    while i < len(r):
        g = int(r["tg"][i] & 0xFFFFFFFF)
        out.append(r[i:i + g])
        i += g
    return out


def summarise(recs: np.ndarray) -> list[str]:
    lines = []
    agg: dict[str, list] = {}
    phases = []
    prev_end, prev_kind = None, None
    ls = launches(recs)
    for j, R in enumerate(ls):
        tag = int(R["tg"][0] >> 32)
        t1, t2 = int(R["t1"].min()), int(R["t2"].max())
        if tag >= 3000:
            kind = "attention"
            i64 = lambda x: x.astype(np.int64)  # noqa: E731
            last = (R["tg"] >> 32) == 3003
            phases.append([np.median(i64(R["m4"]) - i64(R["t1"])), np.median(i64(R["m5"]) - i64(R["m4"])),
                           np.median(i64(R["m6"]) - i64(R["m5"])),
                           np.median(i64(R["t2"][last]) - i64(R["m6"][last])) if last.any() else 0.0,
                           t2 - int(R["m6"].max())])
        else:
            epi, norm = (tag - 1000) // 100, ((tag - 1000) // 10) % 10
            if epi == 1:
                kind = "gate_up"
            elif norm:
                kind = "lm_head" if j == len(ls) - 1 else "qkv"
            else:
                kind = "o_proj" if prev_kind == "attention" else "down"
        agg.setdefault(kind, []).append(((t2 - t1) / 1e3, (t1 - prev_end) / 1e3 if prev_end else 0.0))
        prev_end, prev_kind = t2, kind
    span = (int(recs["t2"].max()) - int(recs["t0"].min())) / 1e3
    lines.append(f"{len(ls)} instrumented launches over {span:.1f} us")
    lines.append(f"{'launch':10s} {'count':>5s} {'post us':>8s} {'gap us':>7s}")
    for k, v in agg.items():
        v = np.array(v)
        lines.append(f"{k:10s} {len(v):5d} {v[:, 0].mean():8.2f} {v[:, 1].mean():7.2f}")
    if phases:
        p = np.array(phases, dtype=np.float64).mean(0) / 1e3
        lines.append("fused attention (per-CTA medians, us): wait -> query prep %.2f, page loop %.2f, "
                     "partials + counter %.2f, last CTA's split merge %.2f; launch tail after the last "
                     "partial %.2f" % tuple(p))
    return lines


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ctx", type=int, default=2048)
    opt = ap.parse_args()
    from higgs_b200 import build, ffi
    if not os.path.exists(build.LIB_TL):
        raise SystemExit("libhiggs_cuda_timeline.so is missing: python -m higgs_b200.build --timeline")
    lib = ffi.load(build.LIB_TL)  # every op of this process now runs the timeline build
    import torch
    sys.path.insert(0, ROOT)
    import bench
    from higgs_b200.model import PRESETS
    a = PRESETS[bench.MODEL]
    torch.cuda.set_device(0)
    model, eng, Sequence = bench.setup_model(a, [1], opt.ctx, 64, "cuda:0")
    seqs = bench.make_seqs(eng, Sequence, 1, opt.ctx, a.vocab_size, seed=1)
    bench.time_device_resident(eng, seqs, 4, 4)  # capture and warm the step
    torch.cuda.synchronize()
    for name in ("higgs_timeline_fetch_gemv", "higgs_timeline_fetch_attn"):
        fetch(lib, name, reset=True)
    ms, _ = bench.time_device_resident(eng, seqs, 1, 0)
    torch.cuda.synchronize()
    recs = np.concatenate([fetch(lib, n, reset=True) for n in ("higgs_timeline_fetch_gemv",
                                                               "higgs_timeline_fetch_attn")])
    print(f"one decode step (B=1, ctx {opt.ctx}): {ms:.3f} ms by CUDA events, timeline build")
    for line in summarise(recs):
        print(line)


if __name__ == "__main__":
    main()
