"""MLX-format model directories -> weights for the native runner.

Mirrors the loading half of higgs-models: load_model_args (config.json,
crates/higgs-models/src/transformer.rs:844-848; Qwen3MoeModelArgs
crates/higgs-models/src/qwen3_moe.rs:37-97), collect_safetensors_files and
load_quantized_safetensors_weights (crates/higgs-models/src/lib.rs:604-723)
with its key remap (lib.rs:709-723).  The files are read by the library's
safetensors reader (higgs_safetensors_* in include/higgs_cuda.h), which
copies each tensor -- or, for a tensor-parallel rank, only that rank's slice
of it -- from the memory-mapped file straight into the device buffer.
"""
from __future__ import annotations

import ctypes
import json
import os

import numpy as np
import torch

from . import ffi
from .model import ModelArgs, kv_heads_per_rank, shard_plan, tensor_specs

_TORCH = {ffi.DTYPE_U32: torch.int32, ffi.DTYPE_BF16: torch.bfloat16, ffi.DTYPE_F32: torch.float32,
          ffi.DTYPE_F16: torch.float16}
_NP = {ffi.DTYPE_U32: np.uint32, ffi.DTYPE_BF16: np.uint16, ffi.DTYPE_F32: np.float32,
       ffi.DTYPE_F16: np.float16}


def load_model_args(model_dir: str) -> ModelArgs:
    """ModelArgs from config.json.  Defaults follow the reference's serde defaults (rope_theta
    10000, tie_word_embeddings false); head_dim is the config's when given, else
    hidden_size / num_attention_heads (transformer.rs:117-126).  Only MLX affine 4-bit,
    group-64 quantized checkpoints are accepted (the quantization block of config.json)."""
    with open(os.path.join(model_dir, "config.json")) as f:
        c = json.load(f)
    q = c.get("quantization")
    if not q or int(q.get("group_size", 0)) != 64 or int(q.get("bits", 0)) != 4:
        raise ValueError(f"{model_dir}: only 4-bit group-64 quantized MLX checkpoints are supported "
                         f"(config.json quantization = {q})")
    mt = c["model_type"]
    if mt not in ("llama", "qwen3", "qwen3_moe", "qwen2", "mistral"):
        raise ValueError(f"{model_dir}: model_type {mt!r} is not on this path")
    H, nh = int(c["hidden_size"]), int(c["num_attention_heads"])
    return ModelArgs(
        model_type=mt, hidden_size=H, num_hidden_layers=int(c["num_hidden_layers"]),
        intermediate_size=int(c.get("intermediate_size", 0)), num_attention_heads=nh,
        num_key_value_heads=int(c.get("num_key_value_heads", nh)),
        head_dim=int(c.get("head_dim") or H // nh), vocab_size=int(c["vocab_size"]),
        rms_norm_eps=float(c["rms_norm_eps"]), rope_theta=float(c.get("rope_theta", 10000.0)),
        tie_word_embeddings=bool(c.get("tie_word_embeddings", False)),
        num_experts=int(c.get("num_experts", 0)), num_experts_per_tok=int(c.get("num_experts_per_tok", 0)),
        moe_intermediate_size=int(c.get("moe_intermediate_size", 0)),
        norm_topk_prob=bool(c.get("norm_topk_prob", False)),
        decoder_sparse_step=int(c.get("decoder_sparse_step", 1) or 1),
        mlp_only_layers=tuple(int(i) for i in c.get("mlp_only_layers", ())))


class SafetensorsDir:
    """An open model directory (higgs_safetensors_open); use as a context manager."""

    def __init__(self, model_dir: str):
        h = ffi.P()
        ffi.call("higgs_safetensors_open", os.fsencode(model_dir), ctypes.byref(h))
        self.handle = h.value

    def close(self):
        if self.handle:
            ffi.load().higgs_safetensors_close(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def names(self) -> list[str]:
        lib = ffi.load()
        return [self.info(i)[0] for i in range(lib.higgs_safetensors_count(self.handle))]

    def find(self, name: str) -> int:
        return int(ffi.load().higgs_safetensors_find(self.handle, name.encode()))

    def info(self, i: int):
        name = ctypes.c_char_p()
        dt, nd = ctypes.c_int(), ctypes.c_int()
        shape = (ctypes.c_int64 * 8)()
        ffi.call("higgs_safetensors_info", self.handle, i, ctypes.byref(name), ctypes.byref(dt),
                 ctypes.byref(nd), shape)
        return name.value.decode(), dt.value, tuple(shape[:nd.value])

    def read_host(self, i: int, row0=0, rows=None, col0=0, cols=None) -> np.ndarray:
        """A 2-D slice of tensor i (leading dims flattened into rows) as a numpy array."""
        _, dt, shape = self.info(i)
        nrows = int(np.prod(shape[:-1])) if len(shape) > 1 else 1
        ncols = shape[-1] if shape else 1
        rows = nrows - row0 if rows is None else rows
        cols = ncols - col0 if cols is None else cols
        out = np.empty((rows, cols), _NP[dt])
        ffi.call("higgs_safetensors_read", None, self.handle, i, row0, rows, col0, cols,
                 out.ctypes.data_as(ctypes.c_void_p), 0, None)
        return out

    def read_device(self, i: int, device, row0, rows, col0, cols) -> torch.Tensor:
        _, dt, _ = self.info(i)
        dev = torch.device(device)
        out = torch.empty(rows, cols, dtype=_TORCH[dt], device=dev)
        ffi.call("higgs_safetensors_read", ffi.ctx(dev.index or 0), self.handle, i, row0, rows, col0,
                 cols, out.data_ptr(), 1, torch.cuda.current_stream(dev).cuda_stream)
        return out


def _want_dtype(leaf: str, kind: str) -> int:
    if kind == "norm":
        return ffi.DTYPE_BF16
    return ffi.DTYPE_U32 if leaf == "weight" else ffi.DTYPE_BF16


def load_weights(model_dir: str, args: ModelArgs, device="cuda:0", rank: int = 0,
                 world: int = 1) -> dict[str, torch.Tensor]:
    """Every tensor the runner needs (tensor_specs(args)), read from the directory onto
    `device`: the whole tensor, or with world > 1 this rank's tensor-parallel slice (the
    slices of shard_weights).  Shapes and dtypes are checked against the architecture."""
    out = {}
    with SafetensorsDir(model_dir) as st:
        for name, kind, shape in tensor_specs(args):
            leaves = [("", shape)] if kind == "norm" else [
                (".weight", shape[:-1] + (shape[-1] // 8,)), (".scales", shape[:-1] + (shape[-1] // 64,)),
                (".biases", shape[:-1] + (shape[-1] // 64,))]
            for suffix, full in leaves:
                key = name + suffix
                i = st.find(key)
                if i < 0:
                    raise KeyError(f"{model_dir}: missing tensor {key}")
                _, dt, got = st.info(i)
                if tuple(got) != tuple(full):
                    raise ValueError(f"{key}: shape {got} in the file, {full} for this architecture")
                want = _want_dtype(suffix.lstrip(".") or "weight", kind)
                if dt != want:
                    raise ValueError(f"{key}: dtype code {dt} in the file, {want} expected "
                                     "(u32 packed codes, bf16 scales / biases / norms)")
                rows = int(np.prod(full[:-1])) if len(full) > 1 else 1
                r0, nr, c0, nc = shard_plan(args, key, rows, full[-1], rank, world)
                t = st.read_device(i, device, r0, nr, c0, nc)
                lead = full[:-1]
                if len(full) > 1 and nr != rows:  # a slice of the leading (row) dimension
                    lead = (nr // (rows // full[0]),) + tuple(full[1:-1]) if len(full) > 2 else (nr,)
                out[key] = t.view(*lead, nc) if len(full) > 1 else t.view(nc)
    return out
