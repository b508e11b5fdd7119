"""Generation loop over the native runner: prefill with prefix-cache reuse, then
CUDA-graph-replayed decode steps for a batch of sequences.

Mirrors the engine side of higgs (crates/higgs-engine/src/simple.rs:239-353
prefill / decode_step; batch_engine.rs:479-559 batched decode round; prefix
lookup / store simple.rs:209-223, batch_engine.rs:579-595), with paged KV:
a sequence owns a row of page ids, shared prefix pages come from the radix
cache, and each decode step is one graph launch whose inputs (token, position,
cache slot, length) are device vectors refreshed by one small host->device copy.
"""
from __future__ import annotations

import dataclasses
import math

import numpy as np
import torch

from .kv import PAGE, BlockPool, PrefixCache
from .model import Model


@dataclasses.dataclass
class Sequence:
    prompt: np.ndarray
    pages: list = dataclasses.field(default_factory=list)
    length: int = 0  # tokens in the KV cache
    last_token: int = -1
    generated: list = dataclasses.field(default_factory=list)
    prefix_hit: int = 0


class _DecodeGraph:
    """Device buffers + captured forward for a fixed batch size."""

    def __init__(self, model: Model, B: int, max_blocks: int, max_seq_len: int, use_graph: bool,
                 want_logits: bool):
        dev = model.device
        self.B = B
        self.tokens = torch.zeros(B, 1, dtype=torch.int32, device=dev)
        # packed per-step vector: positions [B] i32 | seq_lens [B] i32 | slots [B] i64
        self.step_dev = torch.zeros(4 * B, dtype=torch.int32, device=dev)
        self.step_host = torch.zeros(4 * B, dtype=torch.int32, pin_memory=True)
        self.positions = self.step_dev[:B].view(B, 1)
        self.seq_lens = self.step_dev[B:2 * B]
        self.slots = self.step_dev[2 * B:].view(torch.int64).view(B, 1)
        self.block_table = torch.zeros(B, max_blocks, dtype=torch.int32, device=dev)
        self.bt_host = np.zeros((B, max_blocks), np.int32)
        self.out_host = torch.zeros(B, dtype=torch.int32, pin_memory=True)
        self.logits = (torch.empty(B, model.args.vocab_size, dtype=torch.float32, device=dev)
                       if want_logits else None)
        # argmax is written straight into the token buffer: the next step reads it in place
        self.fa = model.forward_args(self.tokens, self.positions, self.slots, self.block_table,
                                     self.seq_lens, max_seq_len, logits=self.logits,
                                     argmax=self.tokens.view(B))
        self.model = model
        self.graph = None
        if use_graph:
            self.stream = torch.cuda.Stream(dev)
            self.graph = model.capture(self.fa, self.stream)

    def run(self):
        import ctypes

        from . import ffi
        if self.graph is not None:
            self.graph.launch(torch.cuda.current_stream(self.model.device))
        else:
            ffi.call("higgs_model_forward", self.model.handle, ctypes.byref(self.fa),
                     torch.cuda.current_stream(self.model.device).cuda_stream)


class Engine:
    def __init__(self, model: Model, max_seq_len: int = 4096, prefix_entries: int = 8,
                 use_graph: bool = True, keep_logits: bool = False):
        self.model = model
        self.pool = BlockPool(model.num_pages)
        self.prefix = PrefixCache(self.pool, prefix_entries)
        self.max_seq_len = max_seq_len
        self.max_blocks = math.ceil(max_seq_len / PAGE)
        self.use_graph = use_graph
        self.keep_logits = keep_logits
        self._graphs: dict[int, _DecodeGraph] = {}
        self.step_logits: list[np.ndarray] = []

    # ---- pages -------------------------------------------------------------------------
    def _ensure_pages(self, seq: Sequence, new_len: int):
        need = math.ceil(new_len / PAGE) - len(seq.pages)
        if need > 0:
            seq.pages.extend(self.pool.alloc(need).tolist())

    def release(self, seq: Sequence):
        if seq.pages:
            self.pool.release(np.array(seq.pages, np.int32))
        seq.pages = []

    # ---- prefill -------------------------------------------------------------------------
    def prefill(self, prompt, use_prefix: bool = True) -> Sequence:
        """Run the prompt (after any cached prefix) and sample the first token greedily."""
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        if prompt.size + 1 > self.max_seq_len:
            raise ValueError("prompt longer than max_seq_len")
        seq = Sequence(prompt=prompt)
        if use_prefix and prompt.size > 1:
            matched, pages = self.prefix.lookup(prompt[:-1])  # keep >= 1 token to compute
            seq.pages = pages.tolist()
            seq.length = matched
            seq.prefix_hit = matched
        self._ensure_pages(seq, prompt.size)
        new = prompt[seq.length:]
        n = new.size
        dev = self.model.device
        pos = np.arange(seq.length, prompt.size, dtype=np.int32)
        pg = np.array(seq.pages, np.int32)
        slots = (pg[pos // PAGE].astype(np.int64) * PAGE + pos % PAGE)
        bt = np.zeros((1, self.max_blocks), np.int32)
        bt[0, :len(pg)] = pg
        logits, am = self.model.forward(
            torch.from_numpy(new.reshape(1, n)).to(dev), torch.from_numpy(pos.reshape(1, n)).to(dev),
            torch.from_numpy(slots.reshape(1, n)).to(dev), torch.from_numpy(bt).to(dev),
            torch.tensor([prompt.size], dtype=torch.int32, device=dev), self.max_seq_len,
            last_only=True, want_logits=self.keep_logits)
        seq.length = prompt.size
        seq.last_token = int(am.cpu()[0])
        if self.keep_logits:
            seq.first_logits = logits.cpu().numpy()[0]
        if use_prefix:
            self.prefix.store(prompt, np.array(seq.pages, np.int32))
        return seq

    # ---- decode ----------------------------------------------------------------------------
    def _graph_for(self, B: int) -> _DecodeGraph:
        if B not in self._graphs:
            self._graphs[B] = _DecodeGraph(self.model, B, self.max_blocks, self.max_seq_len,
                                           self.use_graph, self.keep_logits)
        return self._graphs[B]

    def stage_step(self, seqs: list[Sequence], g: _DecodeGraph, first: bool):
        """Host part of a decode step: pages, positions, slots, lengths -> one H2D copy."""
        B = len(seqs)
        sh = g.step_host.numpy()
        bt_dirty = first
        for i, s in enumerate(seqs):
            before = len(s.pages)
            self._ensure_pages(s, s.length + 1)
            if len(s.pages) != before or first:
                g.bt_host[i, :len(s.pages)] = s.pages
                bt_dirty = True
            sh[i] = s.length  # position of the token being fed
            sh[B + i] = s.length + 1
        slots = np.array([s.pages[s.length // PAGE] * PAGE + s.length % PAGE for s in seqs], np.int64)
        sh[2 * B:] = slots.view(np.int32)
        stream = torch.cuda.current_stream(self.model.device)
        g.step_dev.copy_(g.step_host, non_blocking=True)
        if bt_dirty:
            g.block_table.copy_(torch.from_numpy(g.bt_host), non_blocking=False)
        if first:
            g.tokens.copy_(torch.tensor([[s.last_token] for s in seqs], dtype=torch.int32))
        return stream

    def decode_steps(self, seqs: list[Sequence], steps: int, force=None) -> np.ndarray:
        """`steps` greedy decode steps for all sequences; returns tokens [B, steps].

        With `force` ([B, steps] tokens) step k feeds force[:, k] instead of the previous
        step's argmax (teacher forcing, for parity checks); the argmax is still returned."""
        B = len(seqs)
        g = self._graph_for(B)
        out = np.zeros((B, steps), np.int32)
        for k in range(steps):
            self.stage_step(seqs, g, first=(k == 0))
            if force is not None:
                g.tokens.copy_(torch.from_numpy(np.ascontiguousarray(force[:, k:k + 1], dtype=np.int32)))
            g.run()
            g.out_host.copy_(g.tokens.view(B), non_blocking=True)
            if self.keep_logits:
                self.step_logits.append(g.logits.cpu().numpy())
            torch.cuda.current_stream(self.model.device).synchronize()
            toks = g.out_host.numpy()
            for i, s in enumerate(seqs):
                s.length += 1
                s.last_token = int(toks[i])
                s.generated.append(s.last_token)
            out[:, k] = toks
        return out

    def generate_greedy(self, prompts, max_new_tokens: int, use_prefix: bool = True) -> np.ndarray:
        """Prefill each prompt, then decode all of them together; tokens [B, max_new_tokens]
        (the first column is the prefill's token)."""
        seqs = [self.prefill(p, use_prefix) for p in prompts]
        first = np.array([[s.last_token] for s in seqs], np.int32)
        if max_new_tokens <= 1:
            return first[:, :max_new_tokens]
        rest = self.decode_steps(seqs, max_new_tokens - 1)
        for s in seqs:
            self.release(s)
        return np.concatenate([first, rest], axis=1)
