"""CPU restatement of the full dense forward (test infrastructure only).

Follows Model::forward / forward_batched (crates/higgs-models/src/transformer.rs:
404-418 block, 246-294 attention, 487-526 model, 663-827 batched decode,
830-838 head) with the oracle's per-op functions and the same bf16 rounding
points as the CUDA runner: every linear / norm / RoPE / attention output and
every residual sum is rounded to bf16; logits stay f32.  The KV cache is a
contiguous per-sequence list (cache.rs:236-311 semantics).
"""
from __future__ import annotations

import hashlib

import numpy as np

from . import oracle as orc


def _seed(seed: int, name: str) -> int:
    return int.from_bytes(hashlib.sha256(f"{seed}:{name}".encode()).digest()[:8], "little") >> 1


def synth_weights_numpy(args, seed: int = 0, std: float = 0.02) -> dict:
    """Seeded N(0, std) weights quantized with the documented W4 g64 rule (numpy);
    norm weights 1.  Same tensor names as higgs_b200.model.tensor_specs."""
    from higgs_b200.model import tensor_specs
    out = {}
    for name, kind, shape in tensor_specs(args):
        if kind == "norm":
            out[name] = np.full(shape, 0x3F80, np.uint16)
            continue
        rng = np.random.default_rng(_seed(seed, name))
        lead, K = shape[:-1], shape[-1]
        sd = 1.0 / np.sqrt(K) if kind == "q4router" else std  # router logits N(0, 1)
        w = rng.normal(0, sd, size=(int(np.prod(lead)), K)).astype(np.float32)
        q, s, b = orc.w4_quantize(w)
        out[name + ".weight"] = q.reshape(*lead, K // 8)
        out[name + ".scales"] = s.reshape(*lead, K // 64)
        out[name + ".biases"] = b.reshape(*lead, K // 64)
    return out


def _add_bf(a, b):
    return orc.f32_to_bf16(orc.bf16_to_f32(a) + orc.bf16_to_f32(b))


class RefModel:
    def __init__(self, args, w: dict, kv_mode: str = "bf16", signs=None):
        self.a = args
        self.w = w
        self.kv_mode = kv_mode
        self.signs = signs
        self.inv = np.array([args.rope_theta ** (-(2.0 * i) / args.head_dim)
                             for i in range(args.head_dim // 2)], dtype=np.float32)

    def _note_route_margin(self, lf, k, B, Lq):
        """Flag sequences whose k-th and (k+1)-th router logits lie within one bf16 ulp: there a
        last-bit difference in the router's input may legitimately swap an expert."""
        srt = -np.sort(-lf, axis=1)
        if srt.shape[1] <= k:
            return
        top, nxt = srt[:, k - 1], srt[:, k]
        ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(top), 1e-30))) - 7)
        near = (top - nxt) <= ulp
        self.route_near |= near.reshape(B, Lq).any(axis=1)

    def lin(self, x, name, want_f32=False):
        """quantized_matmul in the GPU path's form: MLX's matrix form (weights dequantized
        to bf16 first) for >= 17 rows when the output width is a multiple of 128, the exact
        vector form otherwise."""
        q, s, b = self.q(name)
        rows = x.size // x.shape[-1]
        if rows >= 17 and q.shape[0] % 128 == 0 and x.shape[-1] % 256 == 0:
            return orc.qmatmul_dq(x, q, s, b, want_f32=want_f32)
        return orc.qmatmul(x, q, s, b, want_f32=want_f32)

    def q(self, name):
        return self.w[name + ".weight"], self.w[name + ".scales"], self.w[name + ".biases"]

    def new_cache(self):
        L = self.a.num_hidden_layers
        return [[np.zeros((0, self.a.num_key_value_heads, self.a.head_dim), np.uint16),
                 np.zeros((0, self.a.num_key_value_heads, self.a.head_dim), np.uint16)]
                for _ in range(L)]

    def forward(self, tokens, caches, n_layers: int = 0, last_only: bool = False):
        """tokens int [B, Lq]; caches: one new_cache() per sequence (appended in place).
        Returns f32 logits [B, Lq, V] ([B, 1, V] for the last position with last_only)."""
        a = self.a
        B, Lq = tokens.shape
        H, D, Hq, Hkv = a.hidden_size, a.head_dim, a.num_attention_heads, a.num_key_value_heads
        nl = n_layers or a.num_hidden_layers
        self.route_near = np.zeros(B, bool)
        h = orc.embed_gather(tokens.reshape(-1), *self.q("model.embed_tokens"))  # [T, H]
        offs = [c[0][0].shape[0] for c in caches]
        for li in range(nl):
            p = f"model.layers.{li}."
            x = orc.rmsnorm(h, self.w[p + "input_layernorm.weight"], a.rms_norm_eps)[0]
            qh = self.lin(x, p + "self_attn.q_proj").reshape(B, Lq, Hq, D)
            kh = self.lin(x, p + "self_attn.k_proj").reshape(B, Lq, Hkv, D)
            vh = self.lin(x, p + "self_attn.v_proj").reshape(B, Lq, Hkv, D)
            if a.qk_norm:
                qh = orc.rmsnorm(qh.reshape(-1, D), self.w[p + "self_attn.q_norm.weight"],
                                 a.rms_norm_eps)[0].reshape(B, Lq, Hq, D)
                kh = orc.rmsnorm(kh.reshape(-1, D), self.w[p + "self_attn.k_norm.weight"],
                                 a.rms_norm_eps)[0].reshape(B, Lq, Hkv, D)
            attn = np.zeros((B, Lq, Hq, D), np.uint16)
            for b in range(B):
                pos = np.arange(offs[b], offs[b] + Lq, dtype=np.int32)
                qr = orc.rope(np.ascontiguousarray(qh[b]), pos, self.inv)
                kr = orc.rope(np.ascontiguousarray(kh[b]), pos, self.inv)
                kc, vc = caches[b][li]
                kc = np.concatenate([kc, kr])
                vc = np.concatenate([vc, vh[b]])
                caches[b][li] = [kc, vc]
                S = kc.shape[0]
                P = (S + 15) // 16
                kp = np.zeros((P * 16, Hkv, D), np.uint16)
                vp = np.zeros((P * 16, Hkv, D), np.uint16)
                kp[:S], vp[:S] = kc, vc
                kp = kp.reshape(P, 16, Hkv, D).transpose(0, 2, 1, 3)
                vp = vp.reshape(P, 16, Hkv, D).transpose(0, 2, 1, 3)
                bt = np.arange(P, dtype=np.int32)[None]
                if self.kv_mode == "tq4":
                    kcode, ksc = orc.tq4_encode(kp.reshape(-1, D), self.signs)
                    vcode, vsc = orc.tq4_encode(vp.reshape(-1, D), self.signs)
                    attn[b] = orc.paged_attention_tq4(
                        qr[None], kcode.reshape(P, Hkv, 16, 64), ksc.reshape(P, Hkv, 16),
                        vcode.reshape(P, Hkv, 16, 64), vsc.reshape(P, Hkv, 16), bt,
                        np.array([S], np.int32), self.signs)[0]
                else:
                    attn[b] = orc.paged_attention(qr[None], kp, vp, bt, np.array([S], np.int32))[0]
            o = self.lin(attn.reshape(B * Lq, Hq * D), p + "self_attn.o_proj")
            h = _add_bf(h, o)
            x = orc.rmsnorm(h, self.w[p + "post_attention_layernorm.weight"], a.rms_norm_eps)[0]
            if a.is_moe_layer(li):
                # Qwen3MoeMlpBlock::forward_moe (qwen3_moe.rs:293-322): bf16 router logits
                rl = orc.qmatmul(x, *self.q(p + "mlp.gate"))
                lf = orc.bf16_to_f32(rl)
                idx, sc = orc.moe_route_topk(lf, a.num_experts_per_tok, a.norm_topk_prob)
                self._note_route_margin(lf, a.num_experts_per_tok, B, Lq)
                sw = p + "mlp.switch_mlp."
                y = orc.moe_experts(x, idx, self.q(sw + "gate_proj"), self.q(sw + "up_proj"),
                                    self.q(sw + "down_proj"))
                h = orc.moe_combine(y, sc, h)
                continue
            g = self.lin(x, p + "mlp.gate_proj")
            u = self.lin(x, p + "mlp.up_proj")
            d = self.lin(orc.silu_mul(g, u), p + "mlp.down_proj")
            h = _add_bf(h, d)
        if last_only:
            h = np.ascontiguousarray(h.reshape(B, Lq, -1)[:, -1])
            Lq = 1
        x = orc.rmsnorm(h, self.w["model.norm.weight"], a.rms_norm_eps)[0]
        head = "model.embed_tokens" if a.tie_word_embeddings else "lm_head"
        _, logits = self.lin(x, head, want_f32=True)
        return logits.reshape(B, Lq, -1)

    def teacher_forced(self, prompts: np.ndarray, tokens: np.ndarray):
        """Logits [steps, B, V] of the prefill's last position and of decode steps fed
        tokens[:, k] (k < steps - 1): the oracle on a given token stream."""
        B, steps = tokens.shape
        caches = [self.new_cache() for _ in range(B)]
        out = [self.forward(prompts, caches, last_only=True)[:, -1]]
        for k in range(steps - 1):
            out.append(self.forward(tokens[:, k:k + 1].astype(np.int32), caches)[:, -1])
        return np.stack(out)

    def greedy(self, prompts: np.ndarray, steps: int):
        """Prefill [B, P] prompts then `steps` greedy decode tokens; returns (tokens [B, steps],
        logits of each step [steps, B, V])."""
        B = prompts.shape[0]
        caches = [self.new_cache() for _ in range(B)]
        lg = self.forward(prompts, caches, last_only=True)[:, -1]
        toks, all_lg, near = [], [], []
        for _ in range(steps):
            nxt = orc.argmax(lg)
            toks.append(nxt)
            all_lg.append(lg)
            near.append(self.route_near.copy())
            lg = self.forward(nxt.reshape(B, 1).astype(np.int32), caches)[:, -1]
        # [steps, B]: the MoE routing of that step's logits had a near-tie (always False
        # for dense models)
        self.step_route_near = np.stack(near)
        return np.stack(toks, 1), np.stack(all_lg)
