"""GPU (2 devices): one process, contexts on two GPUs, the other device current.

Every entry point runs on its context's device and restores the caller's current device;
per-device state (kernel shared-memory limits, the tensor-core matmul's timeout flag) is
kept per device.  Skipped on a box with fewer than two GPUs.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as orc

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")]


def _weights(rng, N, K):
    q, s, b = orc.w4_quantize(rng.normal(0, 0.02, size=(N, K)).astype(np.float32))
    return q, s, b


def _to(dev, q, s, b):
    return (torch.from_numpy(q.view(np.int32)).to(dev),
            torch.from_numpy(s.view(np.int16)).view(torch.bfloat16).to(dev),
            torch.from_numpy(b.view(np.int16)).view(torch.bfloat16).to(dev))


@pytest.mark.parametrize("M", [1, 5, 32])
def test_ops_on_second_device_with_first_current(M):
    """The same linear on cuda:1 (with cuda:0 current) and on cuda:0 gives the same bits and
    matches the oracle; the decode GEMV (M = 1, 5) and the tensor-core matmul (M = 32, which
    sets a per-device kernel attribute and reads the per-device timeout flag)."""
    import ctypes

    from higgs_b200 import ffi, ops
    rng = np.random.default_rng(M)
    K, N = 4096, 1024
    q, s, b = _weights(rng, N, K)
    x = orc.f32_to_bf16(rng.normal(0, 1, size=(M, K)))
    outs = []
    torch.cuda.set_device(0)
    for dev in ("cuda:1", "cuda:0"):
        w = _to(dev, q, s, b)
        xt = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).to(dev)
        y = ops.quantized_matmul(xt, *w, out_f32=True)
        torch.cuda.synchronize(dev)
        assert torch.cuda.current_device() == 0, "the caller's current device was not restored"
        outs.append(y.cpu().numpy())
    assert np.array_equal(outs[0], outs[1])
    ref = (orc.qmatmul_dq if M >= 17 else orc.qmatmul)(x, q, s, b, want_f32=True)[1]
    np.testing.assert_allclose(outs[0], ref, rtol=1e-3, atol=1e-4 * np.abs(ref).max() + 1e-6)
    for d in (0, 1):
        v = ctypes.c_int(-1)
        ffi.call("higgs_tc_error", ffi.ctx(d), ctypes.byref(v))
        assert v.value == 0
        assert torch.cuda.current_device() == 0


def test_attention_on_second_device_with_first_current():
    """Paged attention on cuda:1 while cuda:0 is current (the attention kernels' shared-memory
    limits are raised per device on first use) against the oracle."""
    from higgs_b200 import ops
    torch.cuda.set_device(0)
    dev = "cuda:1"
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    B, Hq, Hkv, D, L = 2, 32, 8, 128, 700
    P = 2 * 44
    kc = torch.randn(P, Hkv, 16, D, generator=g, device=dev).to(torch.bfloat16)
    vc = torch.randn(P, Hkv, 16, D, generator=g, device=dev).to(torch.bfloat16)
    q = torch.randn(B, 1, Hq, D, generator=g, device=dev).to(torch.bfloat16)
    bt = torch.arange(P, dtype=torch.int32, device=dev).view(B, P // B)
    sl = torch.tensor([L, L - 300], dtype=torch.int32, device=dev)
    out = ops.paged_attention(q, kc, vc, bt, sl, L)
    torch.cuda.synchronize(dev)
    assert torch.cuda.current_device() == 0

    def bits(t):
        return t.view(torch.int16).cpu().numpy().view(np.uint16)
    ref = orc.paged_attention(bits(q), bits(kc), bits(vc), bt.cpu().numpy(), sl.cpu().numpy())
    np.testing.assert_allclose(out.float().cpu().numpy(), orc.bf16_to_f32(ref), atol=1e-2, rtol=1e-2)
