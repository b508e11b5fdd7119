"""ctypes binding of libhiggs_cuda.so (the C ABI declared in include/higgs_cuda.h).

The library is built in-tree by ``higgs_b200.build``; importing an op without
it raises ``HiggsUnavailable`` -- there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libhiggs_cuda.so")

P = ctypes.c_void_p
I = ctypes.c_int
I64 = ctypes.c_int64
F = ctypes.c_float
SZ = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/higgs_cuda.h
SIGNATURES: dict[str, tuple] = {
    "higgs_init": (I, [I, ctypes.POINTER(P)]),
    "higgs_destroy": (I, [P]),
    "higgs_last_error": (ctypes.c_char_p, []),
    "higgs_version": (I, []),
    "higgs_set_option": (I, [ctypes.c_char_p, I]),
    "higgs_tc_error": (I, [P, ctypes.POINTER(I)]),
    "higgs_diag_tc_mma_rate": (I, [P, I, I, I, I, I, I, I, I, P, P]),
    "higgs_w4_dequantize": (I, [P, P, P, P, I, I, P, P]),
    "higgs_w4_quantize": (I, [P, P, I64, I, P, P, P, P]),
    "higgs_embed_gather_w4": (I, [P, P, I, P, P, P, I, I, P, P]),
    "higgs_qlinear_w4g64": (I, [P, P, I, I, P, P, P, I, P, P, P, P]),
    "higgs_qlinear_gate_up_swiglu": (I, [P, P, I, I, P, P, P, P, P, P, I, P, P]),
    "higgs_qlinear_sk_workspace_size": (SZ, [I, I, I]),
    "higgs_rmsnorm_qlinear_w4g64": (I, [P, P, I, I, P, F, P, P, P, I, P, P, P, P, SZ, P]),
    "higgs_rmsnorm_gate_up_swiglu": (I, [P, P, I, I, P, F, P, P, P, P, P, P, I, P, P, SZ, P]),
    "higgs_rmsnorm": (I, [P, P, P, I, I, P, F, P, P, P]),
    "higgs_decode_chain": (I, [P, P, I, F, P, P]),
    "higgs_rope": (I, [P, P, I, I, I, P, P, P, P]),
    "higgs_qknorm_rope_kv_write": (I, [P, P, I, I, I, I, P, P, F, P, P, P, P, P, I64, I64, P, P]),
    "higgs_paged_attention_workspace_size": (SZ, [I, I, I, I, I, I]),
    "higgs_paged_attention": (I, [P, P, I, I, I, I, I, P, P, I64, I64, P, I, P, I, F, P, P, SZ, P]),
    "higgs_fused_attention_workspace_size": (SZ, [I, I, I, I, I, I]),
    "higgs_fused_attention": (I, [P, P, I, I, I, I, I, P, P, F, P, P, P, P, P, I64, I64, P, I, P, I, F, P, P, SZ, P]),
    "higgs_paged_attention_noalloc": (I, [P, P, I, I, I, I, I, P, P, I64, I64, P, I, P, I, F, P, P]),
    "higgs_tq4_encode": (I, [P, P, I64, P, P, P, P]),
    "higgs_qknorm_rope_kv_write_tq4": (I, [P, P, I, I, I, P, P, F, P, P, P, P, P, P, P, P, I64, I64, P, P]),
    "higgs_paged_attention_tq4_workspace_size": (SZ, [I, I, I, I, I]),
    "higgs_paged_attention_tq4": (I, [P, P, I, I, I, I, P, P, P, P, I64, I64, P, I, P, I, P, F, P, P, SZ, P]),
    "higgs_argmax": (I, [P, P, I, I, P, P]),
    "higgs_sample": (I, [P, P, I, I, F, P, P, P]),
    "higgs_spec_accept": (I, [P, P, P, P, I, I, I, F, P, P, P, P, P]),
    "higgs_apply_penalties": (I, [P, P, I, I, P, P, I, F, F, F, P]),
    "higgs_sample_filtered": (I, [P, P, I, I, F, I, F, F, P, P, P]),
    "higgs_logprobs": (I, [P, P, I, I, F, P, I, P, P, P, P]),
    "higgs_apply_token_mask": (I, [P, P, I, I, P, I, P]),
    "higgs_rmsnorm_strided": (I, [P, P, I64, I, I, P, F, P, P]),
    "higgs_moe_plan_size": (SZ, [I, I, I]),
    "higgs_moe_route_topk": (I, [P, P, I, I, I, I, I, P, P, P, SZ, P]),
    "higgs_moe_grouped_w4": (I, [P, P, I, I, I, I, P, P, P, P, P, P, P, I, I, P, P]),
    "higgs_moe_combine": (I, [P, P, P, I, I, I, P, P]),
    "higgs_moe_router": (I, [P, P, I, I, P, P, P, I, P, P]),
    "higgs_comm_handle_size": (SZ, []),
    "higgs_comm_create": (I, [P, I, I, SZ, I, ctypes.POINTER(P), P]),
    "higgs_comm_connect": (I, [P, P]),
    "higgs_comm_destroy": (I, [P]),
    "higgs_comm_error": (I, [P, ctypes.POINTER(I)]),
    "higgs_comm_step": (I, [P, P]),
    "higgs_allreduce_residual": (I, [P, I, P, I, P, P]),
    "higgs_allreduce_argmax": (I, [P, I, P, I, P, P]),
    "higgs_model_set_comm": (I, [P, P]),
    "higgs_model_create": (I, [P, P, ctypes.POINTER(P)]),
    "higgs_model_set_tensor": (I, [P, ctypes.c_char_p, P, I, ctypes.POINTER(I64), I]),
    "higgs_model_finalize": (I, [P]),
    "higgs_model_destroy": (I, [P]),
    "higgs_model_set_kv_cache": (I, [P, P, P, I64]),
    "higgs_model_set_kv_cache_tq4": (I, [P, P, P, P, P, I64, P]),
    "higgs_model_workspace_size": (SZ, [P, I, I, I, I]),
    "higgs_model_forward": (I, [P, P, P]),
    "higgs_model_capture": (I, [P, P, P, ctypes.POINTER(P)]),
    "higgs_graph_launch": (I, [P, P]),
    "higgs_graph_destroy": (I, [P]),
    "higgs_graph_num_kernels": (I, [P]),
    "higgs_block_pool_create": (I, [I64, ctypes.POINTER(P)]),
    "higgs_block_pool_destroy": (I, [P]),
    "higgs_block_pool_num_free": (I64, [P]),
    "higgs_block_pool_alloc": (I, [P, I, P]),
    "higgs_block_pool_retain": (I, [P, P, I]),
    "higgs_block_pool_release": (I, [P, P, I]),
    "higgs_block_pool_refcount": (I, [P, ctypes.c_int32]),
    "higgs_prefix_cache_create": (I, [P, I, ctypes.POINTER(P)]),
    "higgs_prefix_cache_destroy": (I, [P]),
    "higgs_prefix_cache_len": (I, [P]),
    "higgs_prefix_cache_clear": (I, [P]),
    "higgs_prefix_cache_lookup": (I, [P, P, I, P, I, ctypes.POINTER(I)]),
    "higgs_prefix_cache_store": (I, [P, P, I, P, I]),
    "higgs_safetensors_open": (I, [ctypes.c_char_p, ctypes.POINTER(P)]),
    "higgs_safetensors_close": (I, [P]),
    "higgs_safetensors_count": (I, [P]),
    "higgs_safetensors_find": (I, [P, ctypes.c_char_p]),
    "higgs_safetensors_info": (I, [P, I, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(I),
                                   ctypes.POINTER(I), ctypes.POINTER(I64)]),
    "higgs_safetensors_read": (I, [P, P, I, I64, I64, I64, I64, P, I, P]),
}


class ChainGemv(ctypes.Structure):
    """higgs_chain_gemv (include/higgs_cuda.h)."""
    _fields_ = [("x", P), ("norm_w", P), ("K", I), ("N", I), ("swiglu", I), ("nseg", I),
                ("seg_end", I * 3), ("w", P * 3), ("s", P * 3), ("b", P * 3), ("w2", P), ("s2", P),
                ("b2", P), ("y", P), ("y_f32", P), ("residual", P)]


class ModelConfig(ctypes.Structure):
    """higgs_model_config (include/higgs_cuda.h)."""
    _fields_ = [("hidden", I), ("layers", I), ("intermediate", I), ("heads", I), ("kv_heads", I),
                ("head_dim", I), ("vocab", I), ("rms_eps", F), ("rope_theta", F),
                ("tie_word_embeddings", I), ("qk_norm", I), ("kv_mode", I), ("num_experts", I),
                ("experts_per_tok", I), ("moe_intermediate", I), ("norm_topk_prob", I),
                ("tp_world", I), ("tp_rank", I), ("head_rows", I)]


class ForwardArgs(ctypes.Structure):
    """higgs_forward_args (include/higgs_cuda.h)."""
    _fields_ = [("B", I), ("Lq", I), ("tokens", P), ("positions", P), ("slot_mapping", P),
                ("block_table", P), ("max_blocks", I), ("seq_lens", P), ("max_seq_len", I),
                ("n_layers", I), ("last_only", I), ("logits", P), ("argmax", P), ("hidden_out", P),
                ("workspace", P), ("workspace_bytes", SZ)]


DTYPE_U32, DTYPE_BF16, DTYPE_F32, DTYPE_F16 = 0, 1, 2, 3
KV_BF16, KV_TQ4 = 0, 1


class HiggsUnavailable(RuntimeError):
    """libhiggs_cuda.so is missing or cannot be loaded."""


class HiggsError(RuntimeError):
    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed ({code}): {msg}")
        self.code = code


_lib = None
_lock = threading.Lock()


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the library once and attach the declared signatures."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise HiggsUnavailable(
                f"{path} not found: build it with `python -m higgs_b200.build` (no CPU fallback)")
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def call(name: str, *args) -> int:
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != 0:
        raise HiggsError(name, rc, lib.higgs_last_error().decode())
    return rc


_ctx: dict[int, int] = {}


def ctx(device: int) -> int:
    """Per-device context handle (created on first use)."""
    if device not in _ctx:
        lib = load()
        h = P()
        rc = lib.higgs_init(device, ctypes.byref(h))
        if rc != 0:
            raise HiggsError("higgs_init", rc, lib.higgs_last_error().decode())
        _ctx[device] = h.value
    return _ctx[device]
