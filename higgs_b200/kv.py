"""Python handles over the native KV page pool and radix prefix cache
(higgs_block_pool_* / higgs_prefix_cache_* in include/higgs_cuda.h)."""
from __future__ import annotations

import ctypes

import numpy as np

from . import ffi

PAGE = 16


def _i32p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


class BlockPool:
    """Refcounted KV page ids [0, num_pages)."""

    def __init__(self, num_pages: int):
        h = ffi.P()
        ffi.call("higgs_block_pool_create", num_pages, ctypes.byref(h))
        self.handle = h.value
        self.num_pages = num_pages

    def __del__(self):
        try:
            ffi.load().higgs_block_pool_destroy(self.handle)
        except Exception:
            pass

    @property
    def num_free(self) -> int:
        return int(ffi.load().higgs_block_pool_num_free(self.handle))

    def alloc(self, n: int) -> np.ndarray:
        out = np.empty(n, np.int32)
        ffi.call("higgs_block_pool_alloc", self.handle, n, _i32p(out))
        return out

    def retain(self, pages) -> None:
        p = np.ascontiguousarray(pages, dtype=np.int32)
        ffi.call("higgs_block_pool_retain", self.handle, _i32p(p), p.size)

    def release(self, pages) -> None:
        p = np.ascontiguousarray(pages, dtype=np.int32)
        ffi.call("higgs_block_pool_release", self.handle, _i32p(p), p.size)

    def refcount(self, page: int) -> int:
        return int(ffi.load().higgs_block_pool_refcount(self.handle, page))


class PrefixCache:
    """PrefixCache (prompt_cache.rs:41-311) over whole KV pages."""

    def __init__(self, pool: BlockPool, max_entries: int = 8):
        h = ffi.P()
        ffi.call("higgs_prefix_cache_create", pool.handle, max_entries, ctypes.byref(h))
        self.handle = h.value
        self.pool = pool  # keeps the pool alive

    def __del__(self):
        try:
            ffi.load().higgs_prefix_cache_destroy(self.handle)
        except Exception:
            pass

    def __len__(self) -> int:
        return int(ffi.load().higgs_prefix_cache_len(self.handle))

    def clear(self) -> None:
        ffi.call("higgs_prefix_cache_clear", self.handle)

    def lookup(self, tokens) -> tuple[int, np.ndarray]:
        """(matched_tokens, pages); the returned pages are retained for the caller."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.empty(max(1, t.size // PAGE), np.int32)
        m = ctypes.c_int(0)
        ffi.call("higgs_prefix_cache_lookup", self.handle, _i32p(t), t.size, _i32p(out), out.size,
                 ctypes.byref(m))
        return m.value, out[: m.value // PAGE].copy()

    def store(self, tokens, pages) -> None:
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        p = np.ascontiguousarray(pages, dtype=np.int32)
        ffi.call("higgs_prefix_cache_store", self.handle, _i32p(t), t.size, _i32p(p), p.size)
