"""GPU: the allocation-free attention entry point agrees with the workspace one and
with the CPU oracle.

higgs_paged_attention_noalloc serves callers that cannot allocate device
memory on their serving path (a host that owns a fixed device arena, or a
real-time decode loop that must never block in the driver's allocator): its
split-K scratch is a fixed array inside the library instead of a
caller-provided workspace.  This file is collected last, so a failure here
never hides another test; it also passes when run alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as orc

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _case(rng, B, Lq, Hq, Hkv, D, lens):
    maxb = max((n + 15) // 16 for n in lens)
    P = B * maxb + 2
    kc = torch.randn(P, Hkv, 16, D, device=DEV).to(torch.bfloat16)
    vc = torch.randn(P, Hkv, 16, D, device=DEV).to(torch.bfloat16)
    bt = torch.from_numpy(rng.permutation(P)[:B * maxb].reshape(B, maxb).astype(np.int32)).to(DEV)
    q = torch.randn(B, Lq, Hq, D, device=DEV).to(torch.bfloat16)
    sl = torch.tensor(lens, dtype=torch.int32, device=DEV)
    return q, kc, vc, bt, sl


def _noalloc(q, kc, vc, bt, sl, max_seq_len):
    from higgs_b200 import ffi
    B, Lq, Hq, D = q.shape
    Hkv = kc.shape[1]
    out = torch.empty_like(q)
    ffi.call("higgs_paged_attention_noalloc", ffi.ctx(0), q.data_ptr(), B, Lq, Hq, Hkv, D,
             kc.data_ptr(), vc.data_ptr(), Hkv * 16 * D, 16 * D, bt.data_ptr(), bt.shape[1],
             sl.data_ptr(), max_seq_len, float(1.0 / np.sqrt(D)), out.data_ptr(),
             torch.cuda.current_stream().cuda_stream)
    return out


def _bits(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


# (2, 12, 32, 8, 128): 48 query rows per kv head, so one call runs several query chunks that
# reuse the shared split counters, with the largest scratch of these cases (4.5 MiB);
# (37, 1, 32, 8, 128): B * Hkv = 296 split counters, long contexts.
@pytest.mark.parametrize("B,Lq,Hq,Hkv,D,lens", [(1, 1, 32, 8, 128, [2048]),
                                                 (3, 1, 16, 8, 128, [700, 33, 1500]),
                                                 (2, 6, 32, 8, 64, [300, 90]),
                                                 (2, 12, 32, 8, 128, [2000, 1500]),
                                                 (37, 1, 32, 8, 128, [4096 - 97 * i for i in range(37)])])
def test_noalloc_matches_workspace_entry_point(B, Lq, Hq, Hkv, D, lens):
    """Two calls in a row (they share the built-in scratch) against the workspace entry
    point and against orc.paged_attention on the same inputs; tolerance abs / rel 1e-2, the
    attention tests' bound."""
    from higgs_b200 import ops
    rng = np.random.default_rng(sum(lens) + Lq)
    for call in range(2):
        q, kc, vc, bt, sl = _case(rng, B, Lq, Hq, Hkv, D, lens)
        ref = ops.paged_attention(q, kc, vc, bt, sl, max(lens))
        got = _noalloc(q, kc, vc, bt, sl, max(lens))
        torch.cuda.synchronize()
        g = got.float().cpu().numpy()
        np.testing.assert_allclose(g, ref.float().cpu().numpy(), atol=1e-2, rtol=1e-2,
                                   err_msg=f"call {call}: vs workspace entry point")
        orc_out = orc.paged_attention(_bits(q), _bits(kc), _bits(vc), bt.cpu().numpy(),
                                      sl.cpu().numpy())
        np.testing.assert_allclose(g, orc.bf16_to_f32(orc_out), atol=1e-2, rtol=1e-2,
                                   err_msg=f"call {call}: vs oracle")


def test_noalloc_rejects_bad_arguments_on_the_host():
    """Argument checks run on the host before anything is launched or read (here: a head
    size the kernels do not build)."""
    from higgs_b200 import ffi
    lib = ffi.load()
    q = torch.zeros(1, dtype=torch.bfloat16, device=DEV)
    bt = torch.zeros(1, dtype=torch.int32, device=DEV)
    rc = lib.higgs_paged_attention_noalloc(ffi.ctx(0), q.data_ptr(), 1, 1, 32, 8, 96,
                                           q.data_ptr(), q.data_ptr(), 2048, 2048, bt.data_ptr(),
                                           1, bt.data_ptr(), 16, ctypes.c_float(0.1),
                                           q.data_ptr(), None)
    assert rc == -1
    assert b"D must be 64 or 128" in lib.higgs_last_error()
