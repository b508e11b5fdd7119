"""Host-side mirror of higgs-models for the B200 path.

``ModelArgs`` follows ModelArgs (crates/higgs-models/src/transformer.rs:69-97);
``Model`` owns the native decode-step runner (higgs_model_* in
include/higgs_cuda.h) and its paged KV pools.  Weights are MLX-layout tensors
keyed by their safetensors names (crates/higgs-models/src/lib.rs:604-723).
"""
from __future__ import annotations

import ctypes
import dataclasses
import hashlib
import math

import numpy as np
import torch

from . import ffi

PAGE = 16


@dataclasses.dataclass(frozen=True)
class ModelArgs:
    model_type: str
    hidden_size: int
    num_hidden_layers: int
    intermediate_size: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    vocab_size: int
    rms_norm_eps: float
    rope_theta: float
    tie_word_embeddings: bool
    # Qwen3-MoE (Qwen3MoeModelArgs, crates/higgs-models/src/qwen3_moe.rs:37-97)
    num_experts: int = 0
    num_experts_per_tok: int = 0
    moe_intermediate_size: int = 0
    norm_topk_prob: bool = False
    decoder_sparse_step: int = 1
    mlp_only_layers: tuple = ()

    @property
    def qk_norm(self) -> bool:
        # Attention::new enables q/k RMSNorm for model_type "qwen3" (transformer.rs:193)
        return self.model_type in ("qwen3", "qwen3_moe")

    def is_moe_layer(self, i: int) -> bool:
        """Qwen3MoeModelArgs::is_moe_layer (qwen3_moe.rs:88-96)."""
        if self.num_experts <= 0 or self.decoder_sparse_step <= 0:
            return False
        if i in self.mlp_only_layers:
            return False
        return (i + 1) % self.decoder_sparse_step == 0

    def with_layers(self, n: int) -> "ModelArgs":
        return dataclasses.replace(self, num_hidden_layers=n)

    def weight_bytes_per_step(self, experts_touched: float = 0.0) -> int:
        """Bytes of packed weights one decode step streams (embedding: one row).  MoE layers
        count the router plus `experts_touched` distinct experts per layer."""
        H, D = self.hidden_size, self.head_dim
        attn = self.num_attention_heads * D * H * 2 + 2 * self.num_key_value_heads * D * H
        params = self.vocab_size * H
        for i in range(self.num_hidden_layers):
            if self.is_moe_layer(i):
                params += attn + self.num_experts * H + experts_touched * 3 * self.moe_intermediate_size * H
            else:
                params += attn + 3 * self.intermediate_size * H
        return int(params * 0.5625) + self.num_hidden_layers * 2 * H * 2 + H * 2

    def kv_bytes_per_token(self, kv_mode: str = "bf16") -> int:
        per_head = self.head_dim * 2 if kv_mode == "bf16" else 66
        return self.num_hidden_layers * 2 * self.num_key_value_heads * per_head


PRESETS = {
    # Llama-3.2-1B: 16 layers, hidden 2048, 32/8 heads, head_dim 64, FFN 8192, vocab 128256, tied
    "llama-3.2-1b": ModelArgs("llama", 2048, 16, 8192, 32, 8, 64, 128256, 1e-5, 500000.0, True),
    # Qwen3-1.7B: 28 layers, hidden 2048, 16/8 heads, head_dim 128, FFN 6144, vocab 151936, tied
    "qwen3-1.7b": ModelArgs("qwen3", 2048, 28, 6144, 16, 8, 128, 151936, 1e-6, 1000000.0, True),
    # Qwen3-8B: 36 layers, hidden 4096, 32/8 heads, head_dim 128, FFN 12288, vocab 151936, untied
    "qwen3-8b": ModelArgs("qwen3", 4096, 36, 12288, 32, 8, 128, 151936, 1e-6, 1000000.0, False),
    # Qwen3-30B-A3B: 48 layers, hidden 2048, 32/4 heads, head_dim 128, 128 experts top-8 of FFN 768
    "qwen3-30b-a3b": ModelArgs("qwen3_moe", 2048, 48, 6144, 32, 4, 128, 151936, 1e-6, 1000000.0, False,
                               num_experts=128, num_experts_per_tok=8, moe_intermediate_size=768,
                               norm_topk_prob=True),
}


def tiny_args(model_type: str = "qwen3", layers: int = 2, vocab: int = 4096) -> ModelArgs:
    """Small shapes for parity tests (same structure, CPU-oracle friendly)."""
    if model_type == "llama":
        return ModelArgs("llama", 512, layers, 1024, 8, 2, 64, vocab, 1e-5, 500000.0, True)
    if model_type == "qwen3_moe":
        # layer 1 dense (mlp_only_layers), the others sparse: 32 experts, top-4 of FFN 256
        return ModelArgs("qwen3_moe", 512, layers, 768, 4, 2, 128, vocab, 1e-6, 1000000.0, False,
                         num_experts=32, num_experts_per_tok=4, moe_intermediate_size=256,
                         norm_topk_prob=True, mlp_only_layers=(1,))
    return ModelArgs("qwen3", 512, layers, 768, 4, 2, 128, vocab, 1e-6, 1000000.0, False)


def tensor_specs(args: ModelArgs) -> list[tuple[str, str, tuple[int, ...]]]:
    """(name, kind, shape) of every tensor, kind in {"q4": [N, K] quantized, "q4router": [E, K]
    quantized router (N(0, 1/K) init: N(0, 1) logits), "q4e": [E, N, K] stacked experts,
    "norm": [n]}."""
    H, D = args.hidden_size, args.head_dim
    specs = [("model.embed_tokens", "q4", (args.vocab_size, H)), ("model.norm.weight", "norm", (H,))]
    if not args.tie_word_embeddings:
        specs.append(("lm_head", "q4", (args.vocab_size, H)))
    for i in range(args.num_hidden_layers):
        p = f"model.layers.{i}."
        specs += [
            (p + "input_layernorm.weight", "norm", (H,)),
            (p + "post_attention_layernorm.weight", "norm", (H,)),
            (p + "self_attn.q_proj", "q4", (args.num_attention_heads * D, H)),
            (p + "self_attn.k_proj", "q4", (args.num_key_value_heads * D, H)),
            (p + "self_attn.v_proj", "q4", (args.num_key_value_heads * D, H)),
            (p + "self_attn.o_proj", "q4", (H, args.num_attention_heads * D)),
        ]
        if args.is_moe_layer(i):
            E, F = args.num_experts, args.moe_intermediate_size
            specs += [
                (p + "mlp.gate", "q4router", (E, H)),
                (p + "mlp.switch_mlp.gate_proj", "q4e", (E, F, H)),
                (p + "mlp.switch_mlp.up_proj", "q4e", (E, F, H)),
                (p + "mlp.switch_mlp.down_proj", "q4e", (E, H, F)),
            ]
        else:
            specs += [
                (p + "mlp.gate_proj", "q4", (args.intermediate_size, H)),
                (p + "mlp.up_proj", "q4", (args.intermediate_size, H)),
                (p + "mlp.down_proj", "q4", (H, args.intermediate_size)),
            ]
        if args.qk_norm:
            specs += [(p + "self_attn.q_norm.weight", "norm", (D,)),
                      (p + "self_attn.k_norm.weight", "norm", (D,))]
    return specs


def _seed(seed: int, name: str) -> int:
    return int.from_bytes(hashlib.sha256(f"{seed}:{name}".encode()).digest()[:8], "little") >> 1


def weights_to_device(w: dict[str, np.ndarray], device) -> dict[str, torch.Tensor]:
    out = {}
    for k, v in w.items():
        t = torch.from_numpy(np.ascontiguousarray(v))
        if v.dtype == np.uint32:
            t = t.view(torch.int32)
        elif v.dtype == np.uint16:
            t = t.view(torch.bfloat16)
        out[k] = t.to(device)
    return out


@torch.no_grad()
def synth_weights_device(args: ModelArgs, seed: int = 0, device="cuda:0", std: float = 0.02,
                         chunk_rows: int = 8192) -> dict[str, torch.Tensor]:
    """Seeded N(0, std) weights generated and quantized on the GPU (for full-size models)."""
    from . import ops
    out = {}
    g = torch.Generator(device=device)
    for name, kind, shape in tensor_specs(args):
        if kind == "norm":
            out[name] = torch.ones(shape, dtype=torch.bfloat16, device=device)
            continue
        lead, K = shape[:-1], shape[-1]
        N = math.prod(lead)
        # router: N(0, 1/H) weights give N(0, 1) logits for unit-RMS inputs
        sd = 1.0 / math.sqrt(K) if kind == "q4router" else std
        g.manual_seed(_seed(seed, name))
        q = torch.empty(N, K // 8, dtype=torch.int32, device=device)
        s = torch.empty(N, K // 64, dtype=torch.bfloat16, device=device)
        b = torch.empty(N, K // 64, dtype=torch.bfloat16, device=device)
        for r0 in range(0, N, chunk_rows):
            r1 = min(N, r0 + chunk_rows)
            w = torch.randn(r1 - r0, K, generator=g, device=device, dtype=torch.float32) * sd
            q[r0:r1], s[r0:r1], b[r0:r1] = ops.quantize(w)
        out[name + ".weight"] = q.view(*lead, K // 8)
        out[name + ".scales"] = s.view(*lead, K // 64)
        out[name + ".biases"] = b.view(*lead, K // 64)
    return out


def hadamard_signs(seed: int = 4) -> np.ndarray:
    """Seeded +-1 signs of the TurboQuant rotation (seed 4 per the benchmark plan)."""
    rng = np.random.default_rng(seed)
    return np.where(rng.random(128) < 0.5, -1, 1).astype(np.int8)


# ---- tensor parallelism ----------------------------------------------------------------------

# column-parallel (output rows split) and row-parallel (input columns split) projections
_COL = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "mlp.gate_proj", "mlp.up_proj")
_ROW = ("self_attn.o_proj", "mlp.down_proj")


def kv_heads_per_rank(args: ModelArgs, world: int) -> int:
    """kv heads a rank holds: an even share, or one head replicated over world / Hkv ranks
    when there are fewer kv heads than ranks (each rank's query heads then belong to it)."""
    return max(1, args.num_key_value_heads // world)


def check_tp(args: ModelArgs, world: int):
    """The shapes a `world`-way split needs: whole query heads per rank and kv heads either
    split evenly or replicated, K slices of the row-parallel projections in whole 256-column
    units, 16-row vocabulary shards, and (MoE) whole experts per rank."""
    D, Hq, Hkv = args.head_dim, args.num_attention_heads, args.num_key_value_heads
    kv_ok = Hkv % world == 0 or (world % Hkv == 0 and Hq // world <= Hq // Hkv)
    dense = any(not args.is_moe_layer(i) for i in range(args.num_hidden_layers))
    ok = (Hq % world == 0 and kv_ok and (Hq // world * D) % 256 == 0
          and (not dense or args.intermediate_size % (256 * world) == 0)
          and args.vocab_size % (16 * world) == 0
          and (args.num_experts == 0 or args.num_experts % world == 0))
    if not ok:
        raise ValueError(f"{args.model_type} cannot be split {world} ways")


def shard_plan(args: ModelArgs, name: str, rows: int, cols: int, rank: int, world: int):
    """This rank's slice (row0, rows, col0, cols) of tensor `name` viewed as 2-D (leading dims
    flattened into rows): rows of the column-parallel projections and of the LM head, K columns
    (whole 64-wide groups) of the row-parallel ones, its kv head(s), its experts (expert
    parallelism: experts [rank*E/world, (rank+1)*E/world), contiguous rows); everything else
    (norms, the router, the embedding -- a tied head is sliced by the runner) whole."""
    if world == 1:
        return 0, rows, 0, cols
    D, Hkv = args.head_dim, args.num_key_value_heads
    kvr = kv_heads_per_rank(args, world)
    kv0 = (rank * Hkv) // world if Hkv < world else rank * kvr  # first kv head of this rank
    base, _, _ = name.rpartition(".")
    mod = base.split(".", 3)[-1] if base.startswith("model.layers.") else base
    if mod in ("self_attn.k_proj", "self_attn.v_proj"):
        return kv0 * D, kvr * D, 0, cols
    if mod in _COL or base == "lm_head" or mod.startswith("mlp.switch_mlp."):
        n = rows // world
        return rank * n, n, 0, cols
    if mod in _ROW:
        n = cols // world  # words (weight) or groups (scales / biases)
        return 0, rows, rank * n, n
    return 0, rows, 0, cols


def shard_weights(args: ModelArgs, weights: dict, rank: int, world: int) -> dict:
    """This rank's slices (shard_plan) of MLX-layout weights (numpy arrays or torch tensors)."""
    check_tp(args, world)

    def cont(a):
        return a.contiguous() if isinstance(a, torch.Tensor) else np.ascontiguousarray(a)
    out = {}
    for name, t in weights.items():
        shape = tuple(t.shape)
        rows = int(np.prod(shape[:-1])) if len(shape) > 1 else 1
        r0, nr, c0, nc = shard_plan(args, name, rows, shape[-1], rank, world)
        if (r0, nr, c0, nc) == (0, rows, 0, shape[-1]):
            out[name] = t
            continue
        per = rows // shape[0] if len(shape) > 1 else 1  # flattened rows per leading index
        if c0 == 0 and nc == shape[-1]:  # a run of leading indices
            out[name] = t[r0 // per:(r0 + nr) // per]
        else:
            out[name] = cont(t[..., c0:c0 + nc])
    return out


class TPGroup:
    """This rank's communicator (higgs_comm_*): IPC handles exchanged with `all_gather`, a
    callable taking this rank's handle bytes and returning every rank's, in rank order
    (torch.distributed.all_gather_object in the bench and tests)."""

    def __init__(self, rank: int, world: int, words_per_call: int, n_calls: int, all_gather,
                 device=None):
        self.rank, self.world = rank, world
        n = int(ffi.load().higgs_comm_handle_size())
        hdl = ctypes.create_string_buffer(n)
        h = ffi.P()
        ctx = ffi.ctx(torch.device(device).index if device is not None else torch.cuda.current_device())
        ffi.call("higgs_comm_create", ctx, rank, world, words_per_call, n_calls, ctypes.byref(h), hdl)
        self.handle = h.value
        allh = all_gather(bytes(hdl.raw))
        buf = ctypes.create_string_buffer(b"".join(allh), n * world)
        ffi.call("higgs_comm_connect", self.handle, buf)

    def error(self) -> int:
        v = ctypes.c_int(0)
        ffi.call("higgs_comm_error", self.handle, ctypes.byref(v))
        return v.value

    def close(self):
        if getattr(self, "handle", None):
            ffi.load().higgs_comm_destroy(self.handle)
            self.handle = None


class Graph:
    """A captured forward; relaunch after updating the argument vectors in place."""

    def __init__(self, handle: int, keepalive):
        self.handle = handle
        self._keep = keepalive

    @property
    def num_kernels(self) -> int:
        return int(ffi.load().higgs_graph_num_kernels(self.handle))

    def launch(self, stream=None):
        st = (stream or torch.cuda.current_stream()).cuda_stream
        ffi.call("higgs_graph_launch", self.handle, st)

    def __del__(self):
        try:
            if self.handle:
                ffi.load().higgs_graph_destroy(self.handle)
        except Exception:
            pass


class Model:
    """The native runner plus its paged KV pools (AnyModel::forward on the device)."""

    def __init__(self, args: ModelArgs, weights: dict[str, torch.Tensor], num_pages: int,
                 kv_mode: str = "bf16", device="cuda:0", signs: np.ndarray | None = None,
                 tp: TPGroup | None = None):
        """With `tp`, `weights` are this rank's shard (shard_weights) and the model is one
        rank of a tensor-parallel group: greedy tokens are identical on every rank."""
        self.args = args
        self.device = torch.device(device)
        self.weights = weights
        self.kv_mode = kv_mode
        self.num_pages = num_pages
        self.tp = tp
        w = tp.world if tp else 1
        if tp:
            check_tp(args, w)
        cfg = ffi.ModelConfig(args.hidden_size, args.num_hidden_layers, args.intermediate_size // w,
                              args.num_attention_heads // w, kv_heads_per_rank(args, w),
                              args.head_dim, args.vocab_size, args.rms_norm_eps, args.rope_theta,
                              int(args.tie_word_embeddings), int(args.qk_norm),
                              ffi.KV_TQ4 if kv_mode == "tq4" else ffi.KV_BF16, args.num_experts,
                              args.num_experts_per_tok, args.moe_intermediate_size,
                              int(args.norm_topk_prob), w, tp.rank if tp else 0,
                              args.vocab_size // w)
        h = ffi.P()
        ctx = ffi.ctx(self.device.index or 0)
        ffi.call("higgs_model_create", ctx, ctypes.byref(cfg), ctypes.byref(h))
        self.handle = h.value
        for name, t in weights.items():
            dt = {torch.int32: ffi.DTYPE_U32, torch.bfloat16: ffi.DTYPE_BF16,
                  torch.float32: ffi.DTYPE_F32}[t.dtype]
            shape = (ctypes.c_int64 * t.dim())(*t.shape)
            ffi.call("higgs_model_set_tensor", self.handle, name.encode(), t.data_ptr(), dt, shape,
                     t.dim())
        ffi.call("higgs_model_finalize", self.handle)
        if tp:
            ffi.call("higgs_model_set_comm", self.handle, tp.handle)
        L, Hkv, D = args.num_hidden_layers, kv_heads_per_rank(args, w), args.head_dim
        if kv_mode == "tq4":
            self.signs = torch.from_numpy(hadamard_signs() if signs is None else signs).to(self.device)
            self.k_pool = torch.zeros(L, num_pages, Hkv, PAGE, 64, dtype=torch.uint8, device=self.device)
            self.v_pool = torch.zeros_like(self.k_pool)
            self.k_scales = torch.zeros(L, num_pages, Hkv, PAGE, dtype=torch.float16, device=self.device)
            self.v_scales = torch.zeros_like(self.k_scales)
            ffi.call("higgs_model_set_kv_cache_tq4", self.handle, self.k_pool.data_ptr(),
                     self.k_scales.data_ptr(), self.v_pool.data_ptr(), self.v_scales.data_ptr(),
                     num_pages, self.signs.data_ptr())
        else:
            self.k_pool = torch.zeros(L, num_pages, Hkv, PAGE, D, dtype=torch.bfloat16, device=self.device)
            self.v_pool = torch.zeros_like(self.k_pool)
            ffi.call("higgs_model_set_kv_cache", self.handle, self.k_pool.data_ptr(),
                     self.v_pool.data_ptr(), num_pages)
        self._ws: dict[tuple, torch.Tensor] = {}

    def __del__(self):
        try:
            if getattr(self, "handle", None):
                ffi.load().higgs_model_destroy(self.handle)
        except Exception:
            pass

    def workspace(self, B: int, Lq: int, max_seq_len: int, last_only: bool) -> torch.Tensor:
        key = (B, Lq, max_seq_len, last_only)
        if key not in self._ws:
            n = ffi.load().higgs_model_workspace_size(self.handle, B, Lq, max_seq_len, int(last_only))
            self._ws[key] = torch.zeros(n, dtype=torch.uint8, device=self.device)
        return self._ws[key]

    def forward_args(self, tokens, positions, slot_mapping, block_table, seq_lens, max_seq_len: int,
                     n_layers: int = 0, last_only: bool = False, logits=None, argmax=None,
                     hidden_out=None) -> ffi.ForwardArgs:
        B, Lq = tokens.shape
        ws = self.workspace(B, Lq, max_seq_len, last_only)
        return ffi.ForwardArgs(B, Lq, tokens.data_ptr(), positions.data_ptr(), slot_mapping.data_ptr(),
                               block_table.data_ptr(), block_table.shape[1], seq_lens.data_ptr(),
                               int(max_seq_len), int(n_layers), int(last_only),
                               None if logits is None else logits.data_ptr(),
                               None if argmax is None else argmax.data_ptr(),
                               None if hidden_out is None else hidden_out.data_ptr(),
                               ws.data_ptr(), ws.numel())

    def forward(self, tokens, positions, slot_mapping, block_table, seq_lens, max_seq_len: int,
                n_layers: int = 0, last_only: bool = False, want_logits: bool = True):
        """tokens/positions int32 [B, Lq], slot_mapping int64 [B, Lq], block_table int32
        [B, max_blocks], seq_lens int32 [B] (all CUDA).  Returns (logits f32, argmax int32)."""
        B, Lq = tokens.shape
        rows = B if last_only else B * Lq
        vocab_out = self.args.vocab_size // (self.tp.world if self.tp else 1)  # this rank's shard
        logits = (torch.empty(rows, vocab_out, dtype=torch.float32, device=self.device)
                  if want_logits else None)
        am = torch.empty(rows, dtype=torch.int32, device=self.device)
        fa = self.forward_args(tokens, positions, slot_mapping, block_table, seq_lens, max_seq_len,
                               n_layers, last_only, logits, am)
        ffi.call("higgs_model_forward", self.handle, ctypes.byref(fa),
                 torch.cuda.current_stream(self.device).cuda_stream)
        return logits, am

    def capture(self, fa: ffi.ForwardArgs, stream: torch.cuda.Stream) -> Graph:
        g = ffi.P()
        ffi.call("higgs_model_capture", self.handle, ctypes.byref(fa), stream.cuda_stream,
                 ctypes.byref(g))
        return Graph(g.value, (fa,))


def rope_inv_freq(args: ModelArgs) -> np.ndarray:
    return np.array([args.rope_theta ** (-(2.0 * i) / args.head_dim)
                     for i in range(args.head_dim // 2)], dtype=np.float32)


def attention_scale(args: ModelArgs) -> float:
    return 1.0 / math.sqrt(args.head_dim)
