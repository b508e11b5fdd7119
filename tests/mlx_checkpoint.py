"""Test helper: writes an MLX-format model directory (config.json + safetensors files, sharded
with a model.safetensors.index.json) from MLX-layout numpy weights, in the published
safetensors layout (8-byte little-endian header length, JSON header, raw data)."""
from __future__ import annotations

import json
import os

import numpy as np

_DT = {np.dtype(np.uint32): "U32", np.dtype(np.uint16): "BF16", np.dtype(np.float32): "F32",
       np.dtype(np.float16): "F16"}


def write_safetensors(path: str, tensors: dict[str, np.ndarray]) -> None:
    header, blobs, off = {"__metadata__": {"format": "mlx"}}, [], 0
    for name in sorted(tensors):
        a = np.ascontiguousarray(tensors[name])
        b = a.tobytes()
        header[name] = {"dtype": _DT[a.dtype], "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(len(h).to_bytes(8, "little"))
        f.write(h)
        for b in blobs:
            f.write(b)


def write_model_dir(model_dir: str, args, weights: dict[str, np.ndarray], shards: int = 2,
                    inner_names: bool = False) -> None:
    """config.json in the reference's schema plus `shards` safetensors files; with inner_names
    the quantized tensors are stored as `<module>.inner.<leaf>` (the mlx-rs parameter names)."""
    os.makedirs(model_dir, exist_ok=True)
    cfg = {"model_type": args.model_type, "hidden_size": args.hidden_size,
           "num_hidden_layers": args.num_hidden_layers, "intermediate_size": args.intermediate_size,
           "num_attention_heads": args.num_attention_heads,
           "num_key_value_heads": args.num_key_value_heads, "head_dim": args.head_dim,
           "vocab_size": args.vocab_size, "rms_norm_eps": args.rms_norm_eps,
           "rope_theta": args.rope_theta, "tie_word_embeddings": args.tie_word_embeddings,
           "max_position_embeddings": 40960,
           "quantization": {"group_size": 64, "bits": 4}}
    if args.num_experts:
        cfg.update(num_experts=args.num_experts, num_experts_per_tok=args.num_experts_per_tok,
                   moe_intermediate_size=args.moe_intermediate_size, norm_topk_prob=args.norm_topk_prob,
                   decoder_sparse_step=args.decoder_sparse_step, mlp_only_layers=list(args.mlp_only_layers))
    with open(os.path.join(model_dir, "config.json"), "w") as f:
        json.dump(cfg, f)
    names = sorted(weights)
    weight_map = {}
    for s in range(shards):
        part = {}
        for n in names[s::shards]:
            stored = n
            if inner_names and n.endswith((".weight", ".scales", ".biases")) and not n.endswith("norm.weight"):
                base, _, leaf = n.rpartition(".")
                stored = f"{base}.inner.{leaf}"
            part[stored] = weights[n]
            weight_map[stored] = f"model-{s + 1:05d}-of-{shards:05d}.safetensors"
        write_safetensors(os.path.join(model_dir, f"model-{s + 1:05d}-of-{shards:05d}.safetensors"), part)
    if shards > 1:
        with open(os.path.join(model_dir, "model.safetensors.index.json"), "w") as f:
            json.dump({"metadata": {"total_size": 0}, "weight_map": weight_map}, f)
    else:
        os.replace(os.path.join(model_dir, "model-00001-of-00001.safetensors"),
                   os.path.join(model_dir, "model.safetensors"))
