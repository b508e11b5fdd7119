"""The decode-step timeline's host side (higgs_b200.timeline): launch grouping and labels,
on synthetic records (no GPU)."""
import numpy as np

from higgs_b200.timeline import REC, launches, summarise


def _recs(spec):
    """spec: [(tag, [(t0, t1, t2, m4, m5, m6, tag_override or None) per CTA])]"""
    rows = []
    for tag, ctas in spec:
        for i, (t0, t1, t2, m4, m5, m6, tg) in enumerate(ctas):
            rows.append((((tg or tag) << 32) | len(ctas), i << 32, t0, t1, t2, m4, m5, m6))
    return np.array(rows, dtype=REC)


def test_launch_grouping_and_labels():
    us = 1000
    spec = [
        (1000 + 10 + 4, [(0, 1 * us, 6 * us, 0, 0, 0, None), (1, 2 * us, 7 * us, 0, 0, 0, None)]),  # qkv
        (3000, [(8 * us, 8 * us, 12 * us, 9 * us, 10 * us, 11 * us, 3002),                        # attention
                (8 * us + 1, 8 * us, 20 * us, 9 * us, 10 * us, 12 * us, 3003)]),
        (1000 + 8, [(21 * us, 21 * us, 25 * us, 0, 0, 0, None), (21 * us + 1, 21 * us, 25 * us, 0, 0, 0, None)]),
        (1100 + 10 + 2, [(26 * us, 26 * us, 40 * us, 0, 0, 0, None), (26 * us + 1, 27 * us, 40 * us, 0, 0, 0, None)]),
        (1000 + 8, [(41 * us, 41 * us, 50 * us, 0, 0, 0, None), (41 * us + 1, 41 * us, 50 * us, 0, 0, 0, None)]),
        (1000 + 10 + 1, [(51 * us, 51 * us, 90 * us, 0, 0, 0, None), (51 * us + 1, 51 * us, 90 * us, 0, 0, 0, None),
                         (51 * us + 2, 52 * us, 91 * us, 0, 0, 0, None)]),
    ]
    r = _recs(spec)
    rng = np.random.default_rng(0)
    ls = launches(r[rng.permutation(len(r))])  # record order on the device is arbitrary
    assert [len(x) for x in ls] == [2, 2, 2, 2, 2, 3]
    out = "\n".join(summarise(r))
    rows = {l.split()[0]: l.split() for l in out.splitlines()[2:] if l and not l.startswith("fused")}
    assert set(rows) == {"qkv", "attention", "o_proj", "gate_up", "down", "lm_head"}
    assert float(rows["qkv"][2]) == 6.0            # first release (1 us) -> last exit (7 us)
    assert float(rows["attention"][2]) == 12.0     # 8 -> 20 us
    assert float(rows["attention"][3]) == 1.0      # qkv ended at 7, attention released at 8
    assert float(rows["down"][2]) == 9.0
    assert float(rows["lm_head"][2]) == 40.0       # 51 -> 91 us
    # attention phases: query prep 1, page loop 1, partials 1.5 (median of 1 and 2), merge 8, tail 8
    assert "query prep 1.00, page loop 1.00, partials + counter 1.50, last CTA's split merge 8.00" in out
