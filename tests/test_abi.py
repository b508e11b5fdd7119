"""CPU: the C-ABI library builds/loads and exports every symbol include/*.h declares."""
import ctypes
import glob
import os
import re

import pytest

from tests.conftest import ROOT

HEADERS = sorted(glob.glob(os.path.join(ROOT, "include", "*.h")))
LIB = os.path.join(ROOT, "higgs_b200", "libhiggs_cuda.so")


def declared_functions():
    names = set()
    for h in HEADERS:
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"\b(higgs_[a-z0-9_]+)\s*\(", src):
            names.add(m.group(1))
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(LIB):
        from higgs_b200 import build
        build.build()
    return ctypes.CDLL(LIB)


def test_headers_present():
    assert HEADERS, "no include/*.h"
    assert len(declared_functions()) >= 20


def test_every_declared_symbol_exported(lib):
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_ffi_signature_table_matches_header():
    from higgs_b200 import ffi
    assert set(ffi.SIGNATURES) == set(declared_functions())


def test_no_device_errors_cleanly(lib):
    """Without a GPU, init fails with a status code and a message; it never aborts."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    lib.higgs_init.restype = ctypes.c_int
    lib.higgs_last_error.restype = ctypes.c_char_p
    h = ctypes.c_void_p()
    rc = lib.higgs_init(0, ctypes.byref(h))
    assert rc < 0
    assert lib.higgs_last_error().decode()


def test_argument_validation_without_device(lib):
    """Shape checks run before any CUDA call and report HIGGS_ERR_INVALID_ARG (-1)."""
    lib.higgs_qlinear_w4g64.restype = ctypes.c_int
    lib.higgs_last_error.restype = ctypes.c_char_p
    fake = ctypes.c_void_p(16)
    # K not a multiple of 256
    rc = lib.higgs_qlinear_w4g64(fake, fake, 1, 100, fake, fake, fake, 16, fake, None, None, None)
    assert rc == -1
    assert b"K must be a multiple of 256" in lib.higgs_last_error()
    # null context
    rc = lib.higgs_qlinear_w4g64(None, fake, 1, 256, fake, fake, fake, 16, fake, None, None, None)
    assert rc == -1


def test_workspace_size_queries_without_device(lib):
    """Workspace size queries are host arithmetic: they answer without a GPU, cover the
    fixed 64 KB counter region, and return 0 for shapes the ops reject."""
    f = lib.higgs_qlinear_sk_workspace_size
    f.restype = ctypes.c_size_t
    f.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int]
    # decode GEMV (M <= 8) and the wide tensor-core path, including outputs below one
    # 128-row tile and the SwiGLU reading of the row count
    for M, K, rows in [(1, 4096, 4096), (8, 12288, 4096), (9, 1024, 128), (17, 256, 128),
                       (17, 256, 64), (32, 4096, 6144), (64, 12288, 24576), (300, 512, 256)]:
        assert f(M, K, rows) >= 65536, (M, K, rows)
    # larger problems need at least as much
    assert f(32, 4096, 12288) >= f(32, 4096, 6144)
    for M, K, rows in [(0, 4096, 4096), (1, 100, 4096), (1, 4096, 10), (-1, 256, 16)]:
        assert f(M, K, rows) == 0, (M, K, rows)


def test_noalloc_attention_scratch_covers_every_shape(lib):
    """The allocation-free attention entry point keeps its split partials in a fixed 8 MiB
    array.  The split plan caps the CTAs of a launch at one resident wave, so every shape
    the entry accepts (B * Hkv <= 1024, D <= 128) fits; checked here on the host with the
    workspace query the entry point uses."""
    f = lib.higgs_paged_attention_workspace_size
    f.restype = ctypes.c_size_t
    f.argtypes = [ctypes.c_int] * 6
    worst = 0
    for B in (1, 2, 3, 8, 17, 32, 37, 64, 100, 148, 256, 295, 296, 297, 512, 1024):
        for Hkv in (1, 2, 4, 8):
            if B * Hkv > 1024:
                continue
            for G in (1, 4, 8, 16, 32):
                for Lq in (1, 2, 5, 8, 33):
                    for D in (64, 128):
                        for L in (16, 2048, 32768, 131072):
                            worst = max(worst, f(B, Lq, G * Hkv, Hkv, D, max(L, Lq)))
    assert 0 < worst <= 8 << 20, worst


def test_one_workspace_serves_every_shape(lib):
    """The workspace contract: a workspace sized for the largest shape of a given row
    count serves every smaller shape (the split choice may differ per shape)."""
    f = lib.higgs_qlinear_sk_workspace_size
    f.restype = ctypes.c_size_t
    f.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int]
    shapes = [(4096, 6144), (4096, 4096), (4096, 24576), (12288, 4096), (4096, 151936),
              (768, 2048), (2048, 768 * 2), (256, 128)]
    for M in (1, 8, 17, 32, 33, 64, 100, 300):
        big = f(M, 12288, 151936 * 2)
        for K, rows in shapes:
            assert 0 < f(M, K, rows) <= big, (M, K, rows)
