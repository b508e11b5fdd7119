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
class SamplingParams:
    """SamplingParams (crates/higgs-models/src/lib.rs:30-68).  top_k 0, top_p 1, min_p 0 and the
    neutral penalty values (1, 0, 0) mean "off"; temperature 0 is greedy."""
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = 0
    min_p: float = 0.0
    repetition_penalty: float = 1.0
    frequency_penalty: float = 0.0
    presence_penalty: float = 0.0

    def has_penalties(self) -> bool:
        return (self.repetition_penalty != 1.0 or self.frequency_penalty != 0.0
                or self.presence_penalty != 0.0)


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
        self.positions = self.step_dev[:B].view(B, 1)
        self.seq_lens = self.step_dev[B:2 * B]
        self.slots = self.step_dev[2 * B:].view(torch.int64).view(B, 1)
        self.block_table = torch.zeros(B, max_blocks, dtype=torch.int32, device=dev)
        self.bt_host = np.zeros((B, max_blocks), np.int32)  # the host's copy of every row
        # Two pinned staging slots, so the host can stage step k+1 while step k still runs:
        # a slot is rewritten only after the event of the step that last used it.
        self.step_ring = [torch.zeros(4 * B, dtype=torch.int32, pin_memory=True) for _ in range(2)]
        self.bt_ring = [torch.zeros(B, max_blocks, dtype=torch.int32, pin_memory=True)
                        for _ in range(2)]
        self.out_ring = [torch.zeros(B, dtype=torch.int32, pin_memory=True) for _ in range(2)]
        self.done = [None, None]
        self.k = 0
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

    def acquire(self) -> int:
        """The staging slot of the next step, once the step that last used it has finished."""
        i = self.k % 2
        self.k += 1
        if self.done[i] is not None:
            self.done[i].synchronize()
            self.done[i] = None
        return i

    def finish(self, i: int, stream):
        """Queue the D2H read of this step's tokens into slot i and mark the slot busy."""
        self.out_ring[i].copy_(self.tokens.view(self.B), non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(stream)
        self.done[i] = ev

    def collect(self, i: int) -> np.ndarray:
        """Tokens of the step staged in slot i (waits for that step only)."""
        if self.done[i] is not None:
            self.done[i].synchronize()
        return self.out_ring[i].numpy().copy()

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

    def stage_step(self, seqs: list[Sequence], g: _DecodeGraph, first: bool) -> int:
        """Host part of a decode step: pages, positions, slots, lengths -> one H2D copy from a
        pinned staging slot (returned).  Each sequence's length advances here, when the step
        is staged, so the next step can be staged before this one's tokens are read back."""
        B = len(seqs)
        i = g.acquire()
        sh = g.step_ring[i].numpy()
        bt_dirty = first
        for b, s in enumerate(seqs):
            before = len(s.pages)
            self._ensure_pages(s, s.length + 1)
            if len(s.pages) != before or first:
                g.bt_host[b, :len(s.pages)] = s.pages
                bt_dirty = True
            sh[b] = s.length  # position of the token being fed
            sh[B + b] = s.length + 1
        slots = np.array([s.pages[s.length // PAGE] * PAGE + s.length % PAGE for s in seqs], np.int64)
        sh[2 * B:] = slots.view(np.int32)
        for s in seqs:
            s.length += 1
        g.step_dev.copy_(g.step_ring[i], non_blocking=True)
        if bt_dirty:
            g.bt_ring[i].numpy()[:] = g.bt_host
            g.block_table.copy_(g.bt_ring[i], non_blocking=True)
        if first:
            g.tokens.copy_(torch.tensor([[s.last_token] for s in seqs], dtype=torch.int32))
        return i

    def decode_steps(self, seqs: list[Sequence], steps: int, force=None) -> np.ndarray:
        """`steps` greedy decode steps for all sequences; returns tokens [B, steps].

        Pipelined like the reference's decode loop (crates/higgs-engine/src/simple.rs:539-562:
        build step N+1, then sync on step N): the argmax lands in the graph's own token buffer,
        so step k+1 is staged and launched before step k's tokens are read back, and the host's
        bookkeeping for step k overlaps step k+1 on the device.

        With `force` ([B, steps] tokens) step k feeds force[:, k] instead of the previous
        step's argmax (teacher forcing, for parity checks); the argmax is still returned."""
        B = len(seqs)
        g = self._graph_for(B)
        out = np.zeros((B, steps), np.int32)
        stream = torch.cuda.current_stream(self.model.device)
        pending = None  # (step, staging slot) launched but not yet read back
        for k in range(steps + 1):
            if k < steps:
                i = self.stage_step(seqs, g, first=(k == 0))
                if force is not None:
                    g.tokens.copy_(torch.from_numpy(np.ascontiguousarray(force[:, k:k + 1],
                                                                         dtype=np.int32)))
                g.run()
                if self.keep_logits:
                    self.step_logits.append(g.logits.cpu().numpy())
                g.finish(i, stream)
            if pending is not None:
                kp, ip = pending
                toks = g.collect(ip)
                for b, s in enumerate(seqs):
                    s.last_token = int(toks[b])
                    s.generated.append(s.last_token)
                out[:, kp] = toks
            pending = (k, i) if k < steps else None
        return out

    def decode_steps_sampled(self, seqs: list[Sequence], steps: int, params: SamplingParams,
                             uniforms: np.ndarray, top_logprobs: int | None = None,
                             allowed=None):
        """`steps` sampled decode steps: each step's logits go through the reference's logits
        processors on the device, in its order (crates/higgs-engine/src/simple.rs:318-347):
        penalties over the tokens generated so far, the constraint mask, sample() with the
        top-k / top-p / min-p filters, and logprobs of the scaled, masked logits.

        uniforms f32 [steps, B] drive the draws; allowed(step) -> list of B allowed-token-id
        lists (or None for no constraint at that step) stands for the host-side FSM.  Returns
        (tokens [B, steps], logprobs [B, steps] or None, top ids / top logprobs [B, steps, n]
        or None)."""
        from . import ops
        B = len(seqs)
        dev = self.model.device
        V = self.model.args.vocab_size
        g = self._graph_for_logits(B)
        out = np.zeros((B, steps), np.int32)
        lps = np.zeros((B, steps), np.float32) if top_logprobs is not None else None
        n = top_logprobs or 0
        tids = np.zeros((B, steps, n), np.int32)
        tlps = np.zeros((B, steps, n), np.float32)
        u_dev = torch.empty(B, dtype=torch.float32, device=dev)
        tok_dev = torch.empty(B, dtype=torch.int32, device=dev)
        for k in range(steps):
            self.stage_step(seqs, g, first=(k == 0))
            u_dev.copy_(torch.from_numpy(np.ascontiguousarray(uniforms[k], dtype=np.float32)))
            g.run()
            logits = g.logits[:, :V]
            if self.keep_logits:  # the model's logits, before the processors
                self.step_logits.append(logits.cpu().numpy())
            if params.has_penalties():
                hmax = max(1, max(len(s.generated) for s in seqs))
                hist = np.zeros((B, hmax), np.int32)
                lens = np.array([len(s.generated) for s in seqs], np.int32)
                for i, s in enumerate(seqs):
                    hist[i, :len(s.generated)] = s.generated
                ops.apply_penalties(logits, torch.from_numpy(hist).to(dev), torch.from_numpy(lens).to(dev),
                                    params.repetition_penalty, params.frequency_penalty,
                                    params.presence_penalty)
            sets = allowed(k) if allowed is not None else None
            if sets is not None:
                bits = np.zeros((B, (V + 31) // 32), np.uint32)
                for i, ids in enumerate(sets):
                    ids = np.asarray(ids, np.int64)
                    ids = ids[(ids >= 0) & (ids < V)]
                    np.bitwise_or.at(bits[i], ids // 32, np.uint32(1) << (ids % 32).astype(np.uint32))
                ops.apply_token_mask(logits, torch.from_numpy(bits.view(np.int32)).to(dev))
            tok = ops.sample_filtered(logits, params.temperature, params.top_k, params.top_p,
                                      params.min_p, u_dev)
            tok_dev.copy_(tok)
            if top_logprobs is not None:
                lp, ti, tl = ops.logprobs(logits, params.temperature, tok_dev, n)
            g.tokens.view(B).copy_(tok_dev)  # the next step feeds the sampled token
            toks = tok_dev.cpu().numpy()
            if top_logprobs is not None:
                lps[:, k] = lp.cpu().numpy()
                tids[:, k] = ti.cpu().numpy()
                tlps[:, k] = tl.cpu().numpy()
            for i, s in enumerate(seqs):
                s.last_token = int(toks[i])
                s.generated.append(s.last_token)
            out[:, k] = toks
        if top_logprobs is None:
            return out, None, None, None
        return out, lps, tids, tlps

    def _graph_for_logits(self, B: int) -> _DecodeGraph:
        """The decode graph of batch B with its logits kept on the device."""
        key = ("logits", B)
        if key not in self._graphs:
            self._graphs[key] = _DecodeGraph(self.model, B, self.max_blocks, self.max_seq_len,
                                             self.use_graph, True)
        return self._graphs[key]

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


class SpecDecoder:
    """Self-speculative decoding with a layer-skip draft for a fixed batch of sequences.

    Per step: k draft forwards through the first `draft_layers` layers plus the shared
    LM head (each sampled at `temperature` with explicit uniforms), one verify forward of
    the k+1 tokens [last, d1..dk] through every layer, then higgs_spec_accept keeps the
    accepted drafts and draws the corrected (or bonus) token.  Rollback is only a length:
    cache entries past the accepted prefix are overwritten by later steps.  The whole
    step is one CUDA graph; per step the host copies in one packed vector (positions,
    slots, lengths, uniforms) and copies out the accepted counts and tokens.

    The reference engine has no speculative path (one token per forward,
    crates/higgs-engine/src/simple.rs:880-971); the draft is Model::forward truncated
    to its first layers (the n_layers field of higgs_forward_args)."""

    def __init__(self, engine: "Engine", B: int, k: int = 5, draft_layers: int = 9,
                 temperature: float = 0.7, use_graph: bool = True):
        from . import ffi, ops  # noqa: F401
        m = engine.model
        dev = m.device
        V = m.args.vocab_size
        self.engine, self.B, self.k, self.T = engine, B, k, float(temperature)
        self.draft_layers = draft_layers
        k1 = k + 1
        self.tok = torch.zeros(k1, B, dtype=torch.int32, device=dev)  # row 0 last, row i+1 draft i
        self.vtok = torch.zeros(B, k1, dtype=torch.int32, device=dev)
        self.dtok = torch.zeros(B, k, dtype=torch.int32, device=dev)
        # packed step vector (int32 words; the i64 slot arrays first, on 8-byte boundaries):
        # draft slots [k,B] i64 | verify slots [B,k1] i64 | draft pos [k,B] | draft lens [k,B]
        # | verify pos [B,k1] | verify lens [B] | uniforms f32 [2kB + B]
        n_words = 4 * k * B + 3 * B * k1 + B + 2 * k * B + B
        self.step_host = torch.zeros(n_words, dtype=torch.int32, pin_memory=True)
        self.step_dev = torch.zeros(n_words, dtype=torch.int32, device=dev)
        o = 0

        def take(n):
            nonlocal o
            v = self.step_dev[o:o + n]
            o += n
            return v
        self.d_slots = take(2 * k * B).view(torch.int64).view(k, B)
        self.v_slots = take(2 * B * k1).view(torch.int64).view(B, k1)
        self.d_pos = take(k * B).view(k, B)
        self.d_lens = take(k * B).view(k, B)
        self.v_pos = take(B * k1).view(B, k1)
        self.v_lens = take(B)
        u = take(2 * k * B + B).view(torch.float32)
        self.u_draft = u[:k * B].view(k, B)
        self.u_accept = u[k * B:2 * k * B].view(B, k)
        self.u_final = u[2 * k * B:]
        self.block_table = torch.zeros(B, engine.max_blocks, dtype=torch.int32, device=dev)
        self.bt_host = np.zeros((B, engine.max_blocks), np.int32)
        self.draft_logits = torch.empty(k, B, V, dtype=torch.float32, device=dev)
        self.draft_bkv = torch.empty(B, k, V, dtype=torch.float32, device=dev)
        self.target_logits = torch.empty(B, k1, V, dtype=torch.float32, device=dev)
        self.accepted = torch.zeros(B, dtype=torch.int32, device=dev)
        self.out_tokens = torch.zeros(B, k1, dtype=torch.int32, device=dev)
        self.out_host = torch.zeros(B * (k1 + 1), dtype=torch.int32, pin_memory=True)
        msl = engine.max_seq_len
        self.fa_draft = [m.forward_args(self.tok[i].view(B, 1), self.d_pos[i].view(B, 1),
                                        self.d_slots[i].view(B, 1), self.block_table, self.d_lens[i],
                                        msl, n_layers=draft_layers, logits=self.draft_logits[i])
                         for i in range(k)]
        self.fa_verify = m.forward_args(self.vtok, self.v_pos, self.v_slots, self.block_table,
                                        self.v_lens, msl, last_only=False,
                                        logits=self.target_logits.view(B * k1, V))
        self.graph = None
        if use_graph:
            s = torch.cuda.Stream(dev)
            s.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(s):
                self._launch()  # warm-up outside capture (first-call attributes, workspaces)
            torch.cuda.synchronize(dev)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=s):
                self._launch()
        self.launches_per_step = None

    def _launch(self, parts=("draft", "verify", "accept")):
        import ctypes

        from . import ffi
        m = self.engine.model
        st = torch.cuda.current_stream(m.device).cuda_stream
        ctx = ffi.ctx(m.device.index or 0)
        B, k, V = self.B, self.k, m.args.vocab_size
        if "draft" in parts:
            for i in range(k):
                ffi.call("higgs_model_forward", m.handle, ctypes.byref(self.fa_draft[i]), st)
                ffi.call("higgs_sample", ctx, self.draft_logits[i].data_ptr(), B, V, self.T,
                         self.u_draft[i].data_ptr(), self.tok[i + 1].data_ptr(), st)
        if "verify" in parts:
            self.vtok.copy_(self.tok.t())
            self.dtok.copy_(self.tok[1:].t())
            ffi.call("higgs_model_forward", m.handle, ctypes.byref(self.fa_verify), st)
        if "accept" in parts:
            self.draft_bkv.copy_(self.draft_logits.transpose(0, 1))
            ffi.call("higgs_spec_accept", ctx, self.target_logits.data_ptr(), self.draft_bkv.data_ptr(),
                     self.dtok.data_ptr(), B, k, V, self.T, self.u_accept.data_ptr(),
                     self.u_final.data_ptr(), self.accepted.data_ptr(), self.out_tokens.data_ptr(), st)

    def time_parts(self, reps: int = 10) -> dict:
        """Device milliseconds of one speculative step's parts -- the k draft forwards with
        their draws, the batched verify forward, the acceptance -- each captured as its own
        CUDA graph over the currently staged inputs and timed with CUDA events.  (The parts
        rewrite KV slots past the sequences' lengths, which later steps overwrite anyway.)"""
        dev = self.engine.model.device
        out = {}
        for part in ("draft", "verify", "accept"):
            s = torch.cuda.Stream(dev)
            s.wait_stream(torch.cuda.current_stream(dev))
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                self._launch((part,))
            for _ in range(2):
                g.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            cur = torch.cuda.current_stream(dev)
            e0.record(cur)
            for _ in range(reps):
                g.replay()
            e1.record(cur)
            e1.synchronize()
            out[part + "_ms"] = round(e0.elapsed_time(e1) / reps, 4)
            del g
        return out

    def stage(self, seqs: list[Sequence], uniforms: np.ndarray, first: bool):
        """uniforms f32 [2kB + B]: draft draws [k, B], accept tests [B, k], final draws [B]."""
        eng, B, k = self.engine, self.B, self.k
        k1 = k + 1
        sh = self.step_host.numpy()
        bt_dirty = first
        d_pos = np.zeros((k, B), np.int32)
        d_slots = np.zeros((k, B), np.int64)
        v_pos = np.zeros((B, k1), np.int32)
        v_slots = np.zeros((B, k1), np.int64)
        for b, s in enumerate(seqs):
            before = len(s.pages)
            eng._ensure_pages(s, s.length + k1)
            if len(s.pages) != before or first:
                self.bt_host[b, :len(s.pages)] = s.pages
                bt_dirty = True
            pos = s.length + np.arange(k1)
            pg = np.array(s.pages, np.int64)
            sl = pg[pos // PAGE] * PAGE + pos % PAGE
            v_pos[b], v_slots[b] = pos, sl
            d_pos[:, b], d_slots[:, b] = pos[:k], sl[:k]
        o = 0
        sh[o:o + 2 * k * B] = d_slots.reshape(-1).view(np.int32)
        o += 2 * k * B
        sh[o:o + 2 * B * k1] = v_slots.reshape(-1).view(np.int32)
        o += 2 * B * k1
        sh[o:o + k * B] = d_pos.reshape(-1)
        o += k * B
        sh[o:o + k * B] = (d_pos + 1).reshape(-1)
        o += k * B
        sh[o:o + B * k1] = v_pos.reshape(-1)
        o += B * k1
        sh[o:o + B] = v_pos[:, -1] + 1
        o += B
        sh[o:] = np.ascontiguousarray(uniforms, dtype=np.float32).view(np.int32)
        self.step_dev.copy_(self.step_host, non_blocking=True)
        if bt_dirty:
            self.block_table.copy_(torch.from_numpy(self.bt_host), non_blocking=False)
        if first:
            self.tok[0].copy_(torch.tensor([s.last_token for s in seqs], dtype=torch.int32))

    def steps(self, seqs: list[Sequence], n_steps: int, rng: np.random.Generator):
        """Run n_steps speculative steps; returns (tokens generated per sequence, accepted counts
        [n_steps, B])."""
        B, k = self.B, self.k
        assert len(seqs) == B
        dev = self.engine.model.device
        acc_hist = np.zeros((n_steps, B), np.int32)
        for it in range(n_steps):
            u = rng.random(2 * k * B + B, dtype=np.float32)
            self.stage(seqs, u, first=(it == 0))
            if self.graph is not None:
                self.graph.replay()
            else:
                self._launch()
            oh = self.out_host
            oh[:B].copy_(self.accepted, non_blocking=True)
            oh[B:].copy_(self.out_tokens.view(-1), non_blocking=True)
            torch.cuda.current_stream(dev).synchronize()
            acc = oh[:B].numpy().copy()
            toks = oh[B:].numpy().reshape(B, k + 1)
            acc_hist[it] = acc
            last = np.empty(B, np.int32)
            for b, s in enumerate(seqs):
                n = int(acc[b])
                new = toks[b, :n + 1]
                s.generated.extend(int(x) for x in new)
                s.length += n + 1
                s.last_token = int(new[-1])
                last[b] = s.last_token
            self.tok[0].copy_(torch.from_numpy(last), non_blocking=True)
        return acc_hist
