"""Standalone engine: requests, paged KV, sampling, graphs.

Public API (what a user calls)::

    engine = LLMEngine.colocated(engine_config)          # or AFD roles via workers
    outputs = engine.generate(prompts, max_tokens=16)   # list[list[int]]

    rid = engine.add_request(prompt_ids, max_tokens, sampling=SamplingParams(...))
    while engine.has_unfinished():
        engine.step()                                   # {req_id: token}

A step is either a prefill (whole prompts, or chunks of at most
``max_num_batched_tokens``) or a decode of every running request.  Decode
steps copy their inputs host->device from pinned buffers, replay the captured
graph of the padded batch size (eager when none fits or a sparse-attention
step needs selection), and read the tokens back; sampled requests draw from
the step's logits (``runtime/sampling.py``).  Optional prefix caching shares
the KV blocks of common prompt prefixes; ``hold_kv`` / ``export_kv`` /
``add_prefilled_request`` hand a request's cache rows to another engine
(``runtime/kv_transfer.py``); ``abort`` ends a request early.

With ``EngineConfig.async_scheduling`` a steady decode (no request waiting,
on every Attention rank; greedy or sampled on the device, no penalties or
logprobs) launches step t+1 before it reads step t's tokens:
the next input ids are gathered on the device from step t's output, the host
stages positions and block tables one token ahead, and the bookkeeping of
step t (appending tokens, ending requests) runs while step t+1 is on the GPU.
A ``step()`` then returns the previous step's tokens; a request that stopped
on step t has already been decoded once more on step t+1, and that token is
dropped.  Any other step first drains the step in flight.

On AFD Attention ranks several engines (one per rank, data parallel) step in
lockstep: a per-step exchange over the Attention group agrees on eager vs
graph mode and the padded size, the same agreement vLLM's DP metadata provides
in the reference (``attention_model_runner.py:198-283``).
"""

from __future__ import annotations

import itertools
import math
import time
from dataclasses import dataclass, field

import torch
import torch.distributed as dist

from afd_plugin_b200.engine_config import EngineConfig
from afd_plugin_b200.runtime.cuda_graph import graph_settings, pad_to_capture_size
from afd_plugin_b200.runtime.ffn_executor import FFNExecutor, LocalFFNExecutor
from afd_plugin_b200.runtime.kv_cache import PAD_BLOCK, KVCache, block_hashes
from afd_plugin_b200.runtime.model_runner import ModelRunner
from afd_plugin_b200.runtime.sampling import (GREEDY, SamplingParams, apply_penalties, make_generator, mask_tokens,
                                             sample, token_logprobs)


@dataclass
class Request:
    req_id: int
    prompt: list[int]
    max_tokens: int
    output: list[int] = field(default_factory=list)
    blocks: list[int] = field(default_factory=list)
    state_slot: int = -1  # linear-attention state row (Gated DeltaNet models)
    hold_kv: bool = False  # keep the cache rows after finishing, for export to a decode engine
    aborted: bool = False  # ended by abort() before reaching max_tokens
    synthetic_prefill: bool = False  # decode-bench: prompt KV is whatever the cache holds; output[0] is the
    # last prompt token, not a generated one
    sampling: SamplingParams = GREEDY
    generator: torch.Generator | None = None  # the request's own noise stream (seeded requests)
    stop_ids: frozenset[int] = frozenset()  # EOS and stop tokens that end generation
    cached_len: int = 0  # prompt tokens whose KV came from the prefix cache
    # with sampling.logprobs: per output token its logprob (None if another engine produced it)
    # and the top alternatives
    token_logprobs: list = field(default_factory=list)
    top_logprobs: list = field(default_factory=list)

    preemptions: int = 0  # times its blocks were taken back under cache pressure

    @property
    def num_tokens(self) -> int:
        return len(self.prompt) + len(self.output)

    @property
    def kv_tokens(self) -> list[int]:
        """Tokens whose KV a prefill must produce before decoding (re)starts: the prompt, plus the
        generated tokens but the last for a request resumed after preemption."""
        return self.prompt + self.output[:-1] if self.output else self.prompt

    @property
    def stopped(self) -> bool:
        """The last generated token is a stop token (a decode-bench request's output[0] is not generated)."""
        first = 1 if self.synthetic_prefill else 0
        return (bool(self.stop_ids) and len(self.output) > max(first, self.sampling.min_tokens)
                and self.output[-1] in self.stop_ids)

    @property
    def finished(self) -> bool:
        return len(self.output) >= self.max_tokens or self.stopped

    @property
    def finish_reason(self) -> str:
        return "abort" if self.aborted else ("stop" if self.stopped else "length")


@dataclass
class _InFlight:
    """A launched decode step whose tokens the host has not read yet (async scheduling)."""

    reqs: list[Request]  # the step's rows, in order
    host: torch.Tensor  # pinned int32 tokens, filled by the step's device->host copy
    done: torch.cuda.Event  # recorded after that copy
    status: torch.Tensor | None = None  # pinned copy of the device status word behind the step


class _HostEvent:
    """Stands in for a CUDA event on a CPU engine, whose copies and steps complete in order on the host."""

    def record(self) -> None:
        pass

    def synchronize(self) -> None:
        pass


class AttentionCoordinator:
    """Per-step agreement among Attention (DP) ranks; trivial for one rank."""

    def __init__(self, group=None, size: int = 1, rank: int = 0):
        self.group, self.size, self.rank = group, size, rank
        self.any_sparse = False  # after exchange(): some rank needs a sparse-attention decode step

    def exchange(self, num_tokens: int, is_prefill: bool, *, sparse: bool = False) -> list[tuple[int, bool]]:
        if self.group is None or self.size == 1:
            self.any_sparse = sparse
            return [(num_tokens, is_prefill)]
        mine = torch.tensor([num_tokens, int(is_prefill), int(sparse)], dtype=torch.int64)
        out = [torch.empty_like(mine) for _ in range(self.size)]
        dist.all_gather(out, mine, group=self.group)
        self.any_sparse = any(bool(t[2]) for t in out)
        return [(int(t[0]), bool(t[1])) for t in out]

    def agree_pipelined(self, num_tokens: int, *, sparse: bool = False) -> list[int]:
        """Async scheduling: every rank's launch size for a pipelined decode step (-1: it cannot);
        ``any_sparse`` afterwards says whether some rank's step selects sparse positions."""
        if self.group is None or self.size == 1:
            self.any_sparse = sparse
            return [num_tokens]
        mine = torch.tensor([num_tokens, int(sparse)], dtype=torch.int64)
        out = [torch.empty_like(mine) for _ in range(self.size)]
        dist.all_gather(out, mine, group=self.group)
        self.any_sparse = any(bool(t[1]) for t in out)
        return [int(t[0]) for t in out]


class LLMEngine:
    def __init__(
        self,
        engine_config: EngineConfig,
        model,
        ffn_executor: FFNExecutor | None = None,
        *,
        coordinator: AttentionCoordinator | None = None,
        num_blocks: int | None = None,
    ):
        self.config = engine_config
        self.model = model
        self.device = model.device
        mc, cc = engine_config.model_config, engine_config.cache_config
        self.block_size = cc.block_size
        self.max_batch = engine_config.max_num_seqs
        self.max_blocks_per_seq = math.ceil(mc.max_model_len / self.block_size)
        if num_blocks is None:
            num_blocks = cc.num_blocks or self._auto_num_blocks(model, cc)
        # One linear-attention state row per running request plus a padding row.
        self.kv = KVCache(getattr(model, "cache_arch", model.arch), num_blocks, self.block_size, model.dtype,
                          self.device, max_seqs=self.max_batch + 1)
        self._free_state_slots = list(range(self.max_batch - 1, -1, -1))
        self.ffn = ffn_executor or LocalFFNExecutor(model)
        num_ub = engine_config.parallel_config.num_ubatches if engine_config.parallel_config.use_ubatching else 1
        self.runner = ModelRunner(model, self.kv, self.ffn, max_batch=self.max_batch,
                                  max_blocks_per_seq=self.max_blocks_per_seq, num_ubatches=num_ub)
        self.coordinator = coordinator or AttentionCoordinator()
        # Prefix caching shares KV blocks between prompts; recurrent (Gated
        # DeltaNet) state is per request, so hybrid models never share.
        self.prefix_caching = bool(getattr(cc, "enable_prefix_caching", False)) and not self.runner.has_linear_state
        policy = graph_settings(engine_config, role="attention")
        self.use_graphs = (policy.enabled and self.device.type == "cuda"
                           and getattr(self.ffn, "supports_graph_capture", True))
        self.capture_sizes = sorted(engine_config.compilation_config.cudagraph_capture_sizes) if self.use_graphs else []
        self._ids = itertools.count()
        self.waiting: list[Request] = []
        self.running: list[Request] = []
        self.finished: dict[int, Request] = {}
        # Prefill -> decode hand-off: finished requests whose cache rows are kept
        # for export, and imported requests waiting for a batch slot.
        self.held: dict[int, tuple[Request, float]] = {}
        # called before every step (workers install the peer-heartbeat check)
        self.health_check = None
        self.num_preemptions = 0
        # chunked prefill: admitted requests part-way through their prompt
        self.prefilling: list[Request] = []
        self.max_batched_tokens = engine_config.max_num_batched_tokens
        self._kv_waiting: list[tuple[Request, object]] = []
        pin = self.device.type == "cuda"
        mk = lambda *s, dt: torch.zeros(*s, dtype=dt, pin_memory=pin)  # noqa: E731
        self._h_ids = mk(self.max_batch, dt=torch.int32)
        self._h_pos = mk(self.max_batch, dt=torch.int64)
        self._h_slot = mk(self.max_batch, dt=torch.int64)
        self._h_table = mk(self.max_batch, self.max_blocks_per_seq, dt=torch.int32)
        self._h_lens = mk(self.max_batch, dt=torch.int32)
        self._h_next = mk(self.max_batch, dt=torch.int32)
        # async scheduling: the decode step whose tokens have not been read yet,
        # a second pinned token buffer (two steps' tokens can be on their way)
        # and the gather index for survivors of a step that ended requests
        self.async_scheduling = bool(getattr(engine_config, "async_scheduling", False))
        self._inflight: _InFlight | None = None
        self._next_bufs = [self._h_next] + ([mk(self.max_batch, dt=torch.int32)] if self.async_scheduling else [])
        self._flip = 0
        self.num_async_steps = 0  # decode steps launched ahead of their predecessor's read-back
        self._h_idx = mk(self.max_batch, dt=torch.int64)
        self._d_idx = torch.zeros(self.max_batch, dtype=torch.int64, device=self.device)
        event = torch.cuda.Event if self.device.type == "cuda" else _HostEvent
        self._events = [event() for _ in range(2)]
        self._h_status = [mk(1, dt=torch.int32) for _ in range(2)]
        self._staged = event()
        self._h_state = mk(self.max_batch, dt=torch.int32)
        # numpy views of the pinned staging tensors: a decode step fills them
        # with a few vectorised writes instead of per-element tensor indexing
        self._n_ids, self._n_pos, self._n_slot, self._n_table, self._n_lens, self._n_next, self._n_state = (
            t.numpy() for t in (self._h_ids, self._h_pos, self._h_slot, self._h_table, self._h_lens, self._h_next,
                                self._h_state))
        # (req_id, number of blocks) each staged block-table row holds; rows are rewritten only on change
        self._row_key: list[tuple[int, int] | None] = [None] * self.max_batch
        self.last_h2d_bytes = 0
        self.last_d2h_bytes = 0
        from afd_plugin_b200.utils.profiler import RoleProfiler

        self.profiler = RoleProfiler("attention")
        from afd_plugin_b200.utils.metrics import StepMetrics

        self.metrics = StepMetrics()
        from afd_plugin_b200.utils.roofline import weight_bytes_per_step

        # HBM bytes a decode step of this rank must move: its weights once, plus the KV
        # rows of the running sequences (added per step from the staged lengths).
        self._weight_bytes = weight_bytes_per_step(model)
        self.last_hbm_bytes = 0
        self._last_phase = "decode"
        # noise for sampled requests without their own seed (same seed on every
        # tensor-parallel peer, so peers draw the same tokens)
        self._sample_gen = make_generator(engine_config.model_config.seed, self.device)

    # ------------------------------------------------------------ helpers
    def _auto_num_blocks(self, model, cc) -> int:
        """Enough blocks for every sequence at full length, capped on a GPU by
        ``memory_fraction`` of its free memory (requests are preempted when the
        capped pool runs out)."""
        worst = self.max_batch * self.max_blocks_per_seq + 1
        if self.device.type != "cuda":
            return worst
        arch = getattr(model, "cache_arch", model.arch)
        per_block = max(1, KVCache.bytes_per_block(arch, self.block_size, model.dtype))
        free, _ = torch.cuda.mem_get_info(self.device)
        state = KVCache.state_bytes_per_seq(arch, model.dtype) * (self.max_batch + 1)
        fit = int((cc.memory_fraction * free - state) // per_block)
        return max(2, min(worst, fit))

    @classmethod
    def colocated(cls, engine_config: EngineConfig, *, device="cuda", seed: int | None = None) -> "LLMEngine":
        from afd_plugin_b200.models import build_model

        mc = engine_config.model_config
        model = build_model(mc.arch, role="colocated", dtype=mc.dtype, device=device,
                            seed=mc.seed if seed is None else seed, checkpoint=mc.checkpoint,
                            max_positions=mc.max_model_len)
        return cls(engine_config, model)

    def capture_graphs(self) -> None:
        for size in self.capture_sizes:
            if size <= self.max_batch:
                self.runner.capture(size)

    def add_request(self, prompt: list[int], max_tokens: int, *, hold_kv: bool = False,
                    sampling: SamplingParams | None = None) -> int:
        """Queue a request; with ``hold_kv`` its cache rows outlive it until :meth:`export_kv`.

        ``sampling`` (default greedy) sets temperature / top-k / top-p / seed.
        """
        if len(prompt) + max_tokens > self.config.model_config.max_model_len:
            raise ValueError("prompt + max_tokens exceeds max_model_len")
        if math.ceil((len(prompt) + max_tokens) / self.block_size) > self.kv.allocator.num_blocks - 1:
            raise ValueError("prompt + max_tokens needs more KV blocks than the cache holds")
        req = Request(next(self._ids), list(prompt), max_tokens, hold_kv=hold_kv)
        self._set_sampling(req, sampling)
        self.waiting.append(req)
        return req.req_id

    def _set_sampling(self, req: Request, sampling: SamplingParams | None) -> None:
        sp = sampling if sampling is not None else GREEDY
        req.sampling = sp
        if sp.seed is not None and not sp.greedy:
            req.generator = make_generator(sp.seed, self.device)
        eos = () if sp.ignore_eos else self.model.arch.eos_token_id
        req.stop_ids = frozenset(eos) | frozenset(sp.stop_token_ids)

    def _sample(self, reqs: list[Request], tokens: torch.Tensor) -> torch.Tensor:
        """Replace the argmax of sampled requests' rows in ``tokens`` (from the runner's last logits)
        and record log-probabilities for requests that asked for them."""
        plain = True
        for r in reqs:
            if (not r.sampling.greedy or r.sampling.logprobs is not None or r.sampling.penalized
                    or self._holds_stops(r)):
                plain = False
                break
        if plain:
            return tokens
        logits = self.runner.last_logits[: len(reqs)]
        params = [r.sampling for r in reqs]
        penalized = any(p.penalized for p in params)
        held = [sorted(r.stop_ids) if self._holds_stops(r) else [] for r in reqs]
        if penalized or any(held) or not all(p.greedy for p in params):
            chosen_from = logits
            if penalized:
                chosen_from = apply_penalties(logits, params, [r.prompt for r in reqs], [r.output for r in reqs])
            if any(held):
                chosen_from = mask_tokens(chosen_from.float().clone() if chosen_from is logits else chosen_from,
                                          held)
            drawn = sample(chosen_from, params, [r.generator for r in reqs], self._sample_gen)
            tokens[: len(reqs)].copy_(drawn)
        rows = [i for i, r in enumerate(reqs) if r.sampling.logprobs is not None]
        if rows:
            idx = torch.tensor(rows, device=logits.device)
            top_n = max(reqs[i].sampling.logprobs for i in rows)
            chosen, tops = token_logprobs(logits.index_select(0, idx), tokens[: len(reqs)].index_select(0, idx),
                                          top_n)
            for i, c, t in zip(rows, chosen, tops):
                r = reqs[i]
                pad = len(r.output) - len(r.token_logprobs)  # tokens this engine did not produce
                r.token_logprobs.extend([None] * pad + [c])
                r.top_logprobs.extend([[]] * pad + [t[: r.sampling.logprobs]])
        return tokens

    @staticmethod
    def _holds_stops(r: Request) -> bool:
        """The token about to be chosen is still inside the request's ``min_tokens``."""
        return bool(r.stop_ids) and len(r.output) < r.sampling.min_tokens

    def abort(self, req_id: int) -> bool:
        """End a waiting or running request now (client gone); it moves to ``finished`` with
        ``aborted`` set and the tokens it has.  Returns False if it is not live."""
        for lst in (self.waiting, self.running, self.prefilling):
            for i, r in enumerate(lst):
                if r.req_id == req_id:
                    del lst[i]
                    r.aborted, r.hold_kv = True, False
                    self._finish(r)
                    return True
        for i, (r, _) in enumerate(self._kv_waiting):
            if r.req_id == req_id:
                del self._kv_waiting[i]
                r.aborted = True
                self.finished[req_id] = r
                return True
        return False

    def request(self, req_id: int) -> Request | None:
        """The request with this id (waiting, running, imported or finished), or None."""
        if req_id in self.finished:
            return self.finished[req_id]
        for r in self.running:
            if r.req_id == req_id:
                return r
        for r in self.waiting + self.prefilling:
            if r.req_id == req_id:
                return r
        for r, _ in self._kv_waiting:
            if r.req_id == req_id:
                return r
        return None

    # -------------------------------------------- prefill -> decode hand-off
    def export_kv(self, req_id: int) -> bytes:
        """Serialise a held request's cache rows and recurrent state, then free them."""
        from afd_plugin_b200.runtime import kv_transfer as kt

        req, _ = self.held.pop(req_id)
        try:
            n = req.num_tokens - 1
            tensors = kt.export_request_state(self.kv, req.blocks, n, req.state_slot)
            tokens = (req.prompt + req.output)[:n]
            rng = req.generator.get_state() if req.generator is not None else None
            return kt.pack(kt.RequestState(tokens, req.output[-1], len(req.prompt), tensors, rng))
        finally:
            self._release(req)

    def release_kv(self, req_id: int) -> bool:
        """Drop a held request's cache rows without exporting them."""
        entry = self.held.pop(req_id, None)
        if entry is not None:
            self._release(entry[0])
        return entry is not None

    def expire_held(self, max_age_s: float) -> list[int]:
        """Release held cache rows older than ``max_age_s`` (a decode side that never fetched)."""
        now = time.monotonic()
        old = [rid for rid, (_, t) in self.held.items() if now - t > max_age_s]
        for rid in old:
            self.release_kv(rid)
        return old

    def add_prefilled_request(self, blob: bytes, max_tokens: int, *, prompt: list[int] | None = None,
                              sampling: SamplingParams | None = None) -> tuple[int, list[int]]:
        """Queue a request whose prompt was prefilled elsewhere (payload from :meth:`export_kv`).

        The request joins the running batch at the next step with a free slot;
        its first decode step feeds the exporter's next token.  ``prompt``, when
        given, must equal the payload's prompt.  Returns the request id and the
        token ids whose cache rows came with the payload.
        """
        from afd_plugin_b200.runtime import kv_transfer as kt

        state = kt.unpack(blob)
        if prompt is not None and state.tokens[: state.prompt_len] != list(prompt):
            raise ValueError("the KV payload was prefilled for a different prompt")
        n = len(state.tokens)
        if n + max_tokens > self.config.model_config.max_model_len:
            raise ValueError("prefilled tokens + max_tokens exceeds max_model_len")
        if max_tokens < 1:
            raise ValueError("max_tokens must be positive")
        geo = kt.geometry(self.kv)
        for name, t in state.tensors.items():
            if name not in geo:
                raise ValueError(f"KV payload carries tensors this engine has no cache for: {name!r}")
        req = Request(next(self._ids), state.tokens, max_tokens)
        self._set_sampling(req, sampling)
        if req.generator is not None and state.rng_state is not None:
            req.generator.set_state(state.rng_state)  # continue the prefill side's noise stream
        req.output.append(state.next_token)
        self._kv_waiting.append((req, state))
        return req.req_id, state.tokens

    def _admit_prefilled(self) -> None:
        from afd_plugin_b200.runtime import kv_transfer as kt

        while self._kv_waiting and len(self.running) < self.max_batch:
            if self._blocks_short(self._kv_waiting[0][0]) > self.kv.allocator.num_free:
                break  # waits until blocks free up
            req, state = self._kv_waiting.pop(0)
            n = len(req.prompt)
            self._ensure_blocks(req, n + 1)
            req.state_slot = self._free_state_slots.pop()
            if state is not None:
                try:
                    kt.import_request_state(self.kv, req.blocks, req.state_slot, state.tensors, n)
                except ValueError:
                    self._release(req)
                    raise
            (self._finish(req) if req.finished else self.running.append(req))

    def add_synthetic_request(self, prompt: list[int], max_tokens: int, *,
                              sampling: SamplingParams | None = None) -> int:
        """Queue a decode-bench request: every prompt token but the last counts as prefilled
        (its cache rows are whatever the cache holds, e.g. after :meth:`KVCache.fill_random_`),
        and decoding starts by feeding the last prompt token.  ``max_tokens`` tokens are
        generated; ``output[0]`` is that last prompt token.  The serving counterpart of the
        reference's ``AFDDecodeBenchConnector`` (``tools/benchmarks/decode_bench.py:41-140``)."""
        if len(prompt) < 1 or max_tokens < 1:
            raise ValueError("decode-bench requests need a prompt and max_tokens >= 1")
        if len(prompt) + max_tokens > self.config.model_config.max_model_len:
            raise ValueError("prompt + max_tokens exceeds max_model_len")
        req = Request(next(self._ids), list(prompt[:-1]), max_tokens + 1, synthetic_prefill=True)
        self._set_sampling(req, sampling)
        req.output.append(int(prompt[-1]))
        self._kv_waiting.append((req, None))
        return req.req_id

    def admit_prefilled(self, prompts: list[list[int]], first_tokens: list[int], *, reserve_tokens: int = 0) -> list[int]:
        """Admit requests whose prompt KV is already in the cache (decode-only mode; EOS is ignored).

        The decode-benchmark counterpart of the reference's
        ``AFDDecodeBenchConnector`` (``tools/benchmarks/decode_bench.py:41-140``),
        which reports every prompt token but the last as remotely prefilled:
        blocks for ``len(prompt) + reserve_tokens`` positions are allocated, the
        caller fills the cache (e.g. :meth:`KVCache.fill_random_`), and each
        request starts decoding from ``first_tokens[i]``.
        """
        ids = []
        for p, t in zip(prompts, first_tokens):
            req = Request(next(self._ids), list(p), max(1, self.config.model_config.max_model_len - len(p)))
            self._ensure_blocks(req, len(p) + max(1, reserve_tokens))
            req.state_slot = self._free_state_slots.pop()
            req.output.append(int(t))
            self.running.append(req)
            ids.append(req.req_id)
        return ids

    def load_decode_batch(self) -> int:
        """Copy the running batch's decode inputs into the runner's device buffers.

        Returns the batch size; used to prime device-resident decode loops.
        """
        b = self.runner.buf
        reqs = self.running
        self._stage_decode_inputs(reqs, len(reqs))
        n = len(reqs)
        b.state_slots[:n].copy_(self._h_state[:n])
        b.input_ids[:n].copy_(self._h_ids[:n])
        b.positions[:n].copy_(self._h_pos[:n])
        b.slot_mapping[:n].copy_(self._h_slot[:n])
        b.block_table[:n].copy_(self._h_table[:n])
        b.seq_lens[:n].copy_(self._h_lens[:n])
        return n

    def has_unfinished(self) -> bool:
        return bool(self.waiting or self.running or self._kv_waiting or self.prefilling
                    or self._inflight is not None)

    def _ensure_blocks(self, req: Request, upto_tokens: int) -> None:
        need = math.ceil(upto_tokens / self.block_size) - len(req.blocks)
        if need > 0:
            req.blocks.extend(self.kv.allocator.allocate(need))

    def _release(self, req: Request) -> None:
        self.kv.allocator.free(req.blocks)
        req.blocks = []
        if req.state_slot >= 0:
            self._free_state_slots.append(req.state_slot)
            req.state_slot = -1

    def _finish(self, req: Request) -> None:
        if req.hold_kv:
            self.held[req.req_id] = (req, time.monotonic())
        else:
            self._release(req)
        self.finished[req.req_id] = req

    # ---------------------------------------------------------------- step
    def step(self) -> dict[int, int]:
        if self.health_check is not None:
            self.health_check()  # e.g. a peer stopped heartbeating: fail before waiting on it
        t0 = time.perf_counter()
        out = self._step()
        self.metrics.record(phase=self._last_phase, batch=len(out), tokens=len(out),
                            ms=(time.perf_counter() - t0) * 1e3, h2d_bytes=self.last_h2d_bytes,
                            d2h_bytes=self.last_d2h_bytes,
                            hbm_bytes=self.last_hbm_bytes if self._last_phase == "decode" else 0)
        if self.runner.timer.enabled and self._last_phase == "decode":
            self.metrics.phases = self.runner.timer.summary()
        self.profiler.step()
        return out

    def reload_weights(self, checkpoint: str | None = None, *, seed: int = 0) -> None:
        """Reload this engine's weights in place between steps; captured decode graphs stay valid."""
        self.model.reload_weights(checkpoint, seed=seed)

    def close(self) -> None:
        """Read back a decode step still in flight (its tokens are appended), then flush an active
        profiler trace and the metrics stream."""
        if self._inflight is not None:
            self._drain()
        self.profiler.close()
        self.metrics.close()

    def _step(self) -> dict[int, int]:
        if self.async_scheduling:
            out = self._step_async()
            if out is not None:
                self._last_phase = "decode"
                return out
        if self._kv_waiting:
            self._admit_prefilled()
            if not (self.waiting or self.running or self.prefilling) and self.coordinator.size == 1:
                return {}  # every imported request finished on its transferred token
        self._reserve_decode_blocks()
        plan = self._plan_prefill()
        is_prefill = bool(plan)
        ntok = sum(take for _, take in plan) if is_prefill else len(self.running)
        sparse = self._needs_sparse(self.running)
        votes = self.coordinator.exchange(ntok, is_prefill, sparse=sparse)
        if any(p for _, p in votes):
            self._last_phase = "prefill"
            with torch.profiler.record_function("afd_prefill_step"):
                return self._prefill_step(plan, votes)
        self._last_phase = "decode"
        with torch.profiler.record_function("afd_decode_step"):
            return self._decode_step(votes)

    def _plan_prefill(self) -> list[tuple[Request, int]]:
        """(request, prompt tokens to compute this step) for the next prefill step, or [] for a decode step.

        Requests part-way through their prompt (chunked prefill) continue
        first, then waiting ones are admitted while batch slots and the
        ``max_num_batched_tokens`` budget last.  With chunking, a step that
        follows a prefill step decodes when requests are running, so long
        prompts do not stall generation.
        """
        if not (self.prefilling or self.waiting):
            return []
        if self.max_batched_tokens is not None and self._last_phase == "prefill" and self.running:
            return []
        left = self.max_batched_tokens if self.max_batched_tokens is not None else float("inf")
        work, self.prefilling = self.prefilling, []
        reserved = sum(self._blocks_short(r) for r in work)
        while self.waiting and len(self.running) + len(work) < self.max_batch and left > sum(
                len(r.kv_tokens) - r.cached_len for r in work):
            r = self.waiting[0]
            if self.prefix_caching:
                self._reuse_prefix(r)
            need = self._blocks_short(r)
            if reserved + need > self.kv.allocator.num_free:
                if r.cached_len:  # give the cached blocks back until it can be admitted
                    self._release(r)
                    r.cached_len = 0
                break  # admission waits for blocks to free up
            reserved += need
            work.append(self.waiting.pop(0))
        plan = []
        for r in work:
            take = min(len(r.kv_tokens) - r.cached_len, left)
            if take <= 0:
                self.prefilling.append(r)  # keeps its place (and any cached blocks) for the next step
                continue
            plan.append((r, int(take)))
            left -= take
        return plan

    def _prefill_step(self, plan: list[tuple[Request, int]], votes) -> dict[int, int]:
        admit = [r for r, _ in plan]
        if not admit:
            # Another Attention rank prefills: take part with one placeholder row.
            admit_tokens, tables, starts, slots = [[0]], [[PAD_BLOCK]], [0], None
        else:
            for r in admit:
                self._ensure_blocks(r, len(r.kv_tokens) + 1)
                if r.state_slot < 0:
                    r.state_slot = self._free_state_slots.pop()
            admit_tokens = [r.kv_tokens[r.cached_len : r.cached_len + take] for r, take in plan]
            tables = [r.blocks for r in admit]
            starts = [r.cached_len for r in admit]
            slots = [r.state_slot for r in admit]
        toks = self.runner.prefill(admit_tokens, tables, starts, slots,
                                   **self._across(votes, sum(len(t) for t in admit_tokens)))
        out = {}
        if not admit:
            return out
        for r, take in plan:
            r.cached_len += take
        done = [i for i, r in enumerate(admit) if r.cached_len == len(r.kv_tokens)]
        for r in admit:
            if r.cached_len < len(r.kv_tokens):
                self.prefilling.append(r)  # more chunks to come: no token yet
        resumed = [i for i in done if admit[i].output]
        for i in resumed:  # preempted earlier: its next token is known, decoding simply continues
            self.running.append(admit[i])
        done = [i for i in done if not admit[i].output]
        if not done:
            return out
        final = [admit[i] for i in done]
        if len(done) < len(admit):
            idx = torch.tensor(done, device=toks.device)
            toks = toks.index_select(0, idx)
            self.runner.last_logits = self.runner.last_logits.index_select(0, idx)
        toks = self._sample(final, toks)
        if self.prefix_caching:
            for r in final:  # the prompt's full blocks now hold its KV
                for b, h in zip(r.blocks, block_hashes(r.prompt, self.block_size)):
                    self.kv.allocator.register(b, h)
        for r, t in zip(final, toks.cpu().tolist()):
            r.output.append(int(t))
            out[r.req_id] = int(t)
            (self._finish(r) if r.finished else self.running.append(r))
        return out

    def _blocks_short(self, r: Request) -> int:
        """Blocks ``r`` still lacks to prefill its KV tokens and decode one position."""
        return max(0, math.ceil((len(r.kv_tokens) + 1) / self.block_size) - len(r.blocks))

    def _preempt(self, r: Request) -> None:
        """Take back a running request's blocks; it is recomputed from its tokens when re-admitted."""
        self._release(r)
        r.cached_len = 0
        r.preemptions += 1
        self.num_preemptions += 1
        self.waiting.insert(0, r)

    def _reserve_decode_blocks(self) -> None:
        """Give every running request a block for the position it decodes next; when the cache is
        full, preempt the most recently admitted requests (before the step's token counts are agreed)."""
        bs = self.block_size
        i = 0
        while i < len(self.running):
            r = self.running[i]
            need = (r.num_tokens - 1) // bs + 1 - len(r.blocks)
            if need <= 0:
                i += 1
                continue
            while self.kv.allocator.num_free < need and len(self.running) > i + 1:
                self._preempt(self.running.pop())
            if self.kv.allocator.num_free < need:
                self._preempt(self.running.pop(i))
                continue
            r.blocks.extend(self.kv.allocator.allocate(need))
            i += 1

    def _reuse_prefix(self, r: Request) -> None:
        """Take the cached blocks of the longest shared prompt prefix (at least one token is computed)."""
        if r.blocks or r.cached_len:
            return
        kv = r.kv_tokens
        usable = (len(kv) - 1) // self.block_size
        if usable <= 0:
            return
        hit = self.kv.allocator.lookup(block_hashes(kv[: usable * self.block_size], self.block_size))
        r.blocks = hit
        r.cached_len = len(hit) * self.block_size

    def reset_prefix_cache(self) -> int:
        """Forget the cached prompt prefixes; returns how many blocks were cached."""
        return self.kv.allocator.reset_cache()

    def _across(self, votes, mine: int) -> dict:
        if len(votes) == 1:
            return {}
        # Ranks that are not prefilling join with one placeholder row.
        return {"tokens_across_attn": {0: tuple(max(1, n) if p else 1 for n, p in votes)}}

    def _stage_decode_inputs(self, reqs: list[Request], run_b: int, lag: int = 0) -> None:
        """Fill the pinned staging rows ``[0, run_b)`` for a decode step (padding rows after the requests).

        ``lag`` = 1 stages the position after the one of the step in flight
        (async scheduling); the input ids then come from that step's output
        on the device and are not staged.
        """
        bs = self.block_size
        B = len(reqs)
        pos = [r.num_tokens - 1 + lag for r in reqs]
        for r, p in zip(reqs, pos):
            if len(r.blocks) * bs <= p:
                self._ensure_blocks(r, p + 1)
        if not lag:
            self._n_ids[:B] = [r.output[-1] if r.output else r.prompt[-1] for r in reqs]
        self._n_pos[:B] = pos
        self._n_slot[:B] = [r.blocks[p // bs] * bs + p % bs for r, p in zip(reqs, pos)]
        self._n_lens[:B] = self._n_pos[:B] + 1
        self._n_state[:B] = [r.state_slot for r in reqs]
        table, keys = self._n_table, self._row_key
        for i, r in enumerate(reqs):
            key = (r.req_id, len(r.blocks))
            if keys[i] != key:
                n = len(r.blocks)
                table[i, :n] = r.blocks
                table[i, n:] = PAD_BLOCK
                keys[i] = key
        if run_b > B:
            self._n_ids[B:run_b] = 0
            self._n_pos[B:run_b] = 0
            self._n_slot[B:run_b] = PAD_BLOCK * bs
            self._n_lens[B:run_b] = 1
            self._n_state[B:run_b] = self.runner.pad_state_slot
            for i in range(B, run_b):
                if keys[i] is not None:
                    table[i] = PAD_BLOCK
                    keys[i] = None

    def _decode_step(self, votes) -> dict[int, int]:
        from afd_plugin_b200.runtime.model_runner import ubatch_splits

        reqs = self.running
        B = len(reqs)
        top = max(max(n for n, _ in votes), 1)
        padded = pad_to_capture_size(top, self.capture_sizes) if self.use_graphs else None
        # Graphs hold the dense decode: a step that must select sparse
        # positions (DeepSeek sparse attention past index_topk) runs eagerly.
        sparse = self.coordinator.any_sparse
        use_graph = padded is not None and padded in self.runner.graphs and not sparse
        self.runner.sparse_decode = sparse
        # All Attention ranks run the same (padded) batch so FFN stages line up.
        run_b = padded if use_graph else top
        self._stage_decode_inputs(reqs, run_b)
        b = self.runner.buf
        if self.runner.has_linear_state:
            b.state_slots[:run_b].copy_(self._h_state[:run_b], non_blocking=True)
        b.input_ids[:run_b].copy_(self._h_ids[:run_b], non_blocking=True)
        b.positions[:run_b].copy_(self._h_pos[:run_b], non_blocking=True)
        b.slot_mapping[:run_b].copy_(self._h_slot[:run_b], non_blocking=True)
        b.block_table[:run_b].copy_(self._h_table[:run_b], non_blocking=True)
        b.seq_lens[:run_b].copy_(self._h_lens[:run_b], non_blocking=True)
        self.last_h2d_bytes = run_b * (4 + 8 + 8 + 4 + 4 * self.max_blocks_per_seq
                                       + (4 if self.runner.has_linear_state else 0))
        from afd_plugin_b200.utils.roofline import kv_bytes_per_step

        self.last_hbm_bytes = self._weight_bytes + kv_bytes_per_step(getattr(self.model, "cache_arch", self.model.arch), int(self._h_lens[:B].sum()),
                                                                      elem_bytes=self.model.dtype.itemsize)
        flags = {}
        if len(votes) > 1:
            sp = ubatch_splits(run_b, self.runner.num_ubatches)
            flags["tokens_across_attn"] = {
                s: tuple(sp[s + 1] - sp[s] for _ in votes) for s in range(len(sp) - 1)
            }
        nxt = self._sample(reqs, self.runner.decode_step(run_b, use_graph=use_graph, **flags))
        self._h_next[:run_b].copy_(nxt, non_blocking=True)
        if self.device.type == "cuda":
            torch.cuda.current_stream(self.device).synchronize()
            check = getattr(self.ffn, "check_device_status", None)
            if check is not None:
                check()
        self.last_d2h_bytes = run_b * 4
        out = {}
        still = []
        for r, t in zip(reqs, self._n_next[:B].tolist()):
            r.output.append(t)
            out[r.req_id] = t
            (self._finish(r) if r.finished else still.append(r))
        self.running = still
        return out

    # ------------------------------------------------------ async scheduling
    def _step_async(self) -> dict[int, int] | None:
        """A pipelined decode step, a drain of the step in flight, or None (the step runs synchronously).

        Attention ranks agree first (one exchange of launch sizes): they
        pipeline only when every rank can, at the largest rank's batch, so
        their FFN stages line up.
        """
        launch = self._pipeline_batch()
        sparse = self._needs_sparse(launch, lag=0 if self._inflight is None else 1) if launch else False
        sizes = self.coordinator.agree_pipelined(-1 if launch is None else len(launch), sparse=sparse)
        if min(sizes) > 0:
            with torch.profiler.record_function("afd_decode_step"):
                return self._decode_step_async(launch, max(sizes), len(sizes), self.coordinator.any_sparse)
        if self._inflight is not None:
            return self._drain()
        return None

    def _pipeline_batch(self) -> list[Request] | None:
        """The requests the next step decodes if it may launch before the previous step's tokens are
        read (a decode without penalties, logprobs or min_tokens, with no prompt or imported request
        waiting and enough free KV blocks)."""
        if not self.running or self.waiting or self.prefilling or self._kv_waiting:
            return None
        # penalties, logprobs and min_tokens read the generated tokens on the host (one behind here)
        for r in self.running:
            sp = r.sampling
            if sp.logprobs is not None or sp.penalized or sp.min_tokens:
                return None
        lag = 0 if self._inflight is None else 1
        # a request whose token in flight is its last one is not decoded again
        launch = [r for r in self.running if len(r.output) + 1 < r.max_tokens] if lag else self.running
        if not launch:
            return None
        bs = self.block_size
        need = 0
        for r in launch:
            need += max(0, (r.num_tokens - 1 + lag) // bs + 1 - len(r.blocks))
        return launch if need <= self.kv.allocator.num_free else None

    def _needs_sparse(self, reqs: list[Request], lag: int = 0) -> bool:
        """DeepSeek sparse attention: some request's context (with ``lag`` tokens still in flight)
        is past ``index_topk``, so the step selects positions (eagerly) instead of replaying a graph."""
        topk = getattr(self.model.arch, "index_topk", 0)
        return bool(topk) and any(r.num_tokens + lag > topk for r in reqs)

    def _decode_step_async(self, launch: list[Request], top: int, nranks: int,
                           sparse: bool = False) -> dict[int, int]:
        """Launch a decode step of ``launch`` (padded to ``top`` rows, the largest Attention rank's batch)
        from staged positions and the device-resident tokens of the step in flight, then read that step's
        tokens."""
        from afd_plugin_b200.runtime.model_runner import ubatch_splits

        prev = self._inflight
        lag = 0 if prev is None else 1
        B = len(launch)
        padded = pad_to_capture_size(top, self.capture_sizes) if self.use_graphs else None
        use_graph = padded is not None and padded in self.runner.graphs and not sparse
        run_b = padded if use_graph else top
        flags = {}
        if nranks > 1:
            sp = ubatch_splits(run_b, self.runner.num_ubatches)
            flags["tokens_across_attn"] = {s: (sp[s + 1] - sp[s],) * nranks for s in range(len(sp) - 1)}
        self.runner.sparse_decode = sparse
        # the pinned staging rows are rewritten below: the previous step's
        # host->device copies of them must have run
        self._staged.synchronize()
        self._stage_decode_inputs(launch, run_b, lag=lag)
        b = self.runner.buf
        h2d = run_b * (8 + 8 + 4 + 4 * self.max_blocks_per_seq)
        if self.runner.has_linear_state:
            b.state_slots[:run_b].copy_(self._h_state[:run_b], non_blocking=True)
            h2d += run_b * 4
        if not lag:
            b.input_ids[:run_b].copy_(self._h_ids[:run_b], non_blocking=True)
            h2d += run_b * 4
        else:
            if run_b > B:  # padding rows
                b.input_ids[B:run_b].copy_(self._h_ids[B:run_b], non_blocking=True)
                h2d += (run_b - B) * 4
            if B == len(prev.reqs):  # no request ended: the rows line up
                b.input_ids[:B].copy_(b.next_tokens[:B])
            else:
                row = {id(r): i for i, r in enumerate(prev.reqs)}
                self._h_idx.numpy()[:B] = [row[id(r)] for r in launch]
                self._d_idx[:B].copy_(self._h_idx[:B], non_blocking=True)
                b.input_ids[:B].copy_(b.next_tokens.index_select(0, self._d_idx[:B]))
                h2d += B * 8
        b.positions[:run_b].copy_(self._h_pos[:run_b], non_blocking=True)
        b.slot_mapping[:run_b].copy_(self._h_slot[:run_b], non_blocking=True)
        b.block_table[:run_b].copy_(self._h_table[:run_b], non_blocking=True)
        b.seq_lens[:run_b].copy_(self._h_lens[:run_b], non_blocking=True)
        self._staged.record()
        self.last_h2d_bytes = h2d
        from afd_plugin_b200.utils.roofline import kv_bytes_per_step

        self.last_hbm_bytes = self._weight_bytes + kv_bytes_per_step(getattr(self.model, "cache_arch", self.model.arch),
                                                                      int(self._h_lens[:B].sum()),
                                                                      elem_bytes=self.model.dtype.itemsize)
        nxt = self.runner.decode_step(run_b, use_graph=use_graph, **flags)
        if any(not r.sampling.greedy for r in launch):
            # drawn on the device from this step's logits, before the next replay overwrites them
            nxt = self._sample(launch, nxt)
        host = self._next_bufs[self._flip]
        host[:run_b].copy_(nxt, non_blocking=True)
        status = None
        word_of = getattr(self.ffn, "device_status_word", None)
        if word_of is not None:  # read after the step's event instead of a blocking read
            status = self._h_status[self._flip]
            status.copy_(word_of(), non_blocking=True)
        done = self._events[self._flip]
        done.record()
        self._flip ^= 1
        self.num_async_steps += 1
        self.last_d2h_bytes = run_b * 4 + (4 if status is not None else 0)
        self._inflight = _InFlight(launch, host, done, status)
        return self._consume(prev) if prev is not None else {}

    def _consume(self, fl: _InFlight) -> dict[int, int]:
        """Read a launched step's tokens and append them; requests that ended before it drop theirs."""
        fl.done.synchronize()
        check = getattr(self.ffn, "check_device_status", None)
        if check is not None:
            if fl.status is not None:
                check(int(fl.status[0]))
            else:
                check()
        out = {}
        ended = False
        for r, t in zip(fl.reqs, fl.host.numpy()[: len(fl.reqs)].tolist()):
            if r.aborted or r.finished:
                continue
            r.output.append(t)
            out[r.req_id] = t
            if r.finished:
                self._finish(r)
                ended = True
        if ended:
            self.running = [r for r in self.running if not (r.finished or r.aborted)]
        return out

    def _drain(self) -> dict[int, int]:
        """Read the step in flight without launching another (before any step that is not pipelined)."""
        fl, self._inflight = self._inflight, None
        return self._consume(fl)

    def generate(self, prompts: list[list[int]], max_tokens: int,
                 sampling: SamplingParams | None = None) -> list[list[int]]:
        """Run the prompts to completion; returns each one's generated tokens."""
        ids = [self.add_request(p, max_tokens, sampling=sampling) for p in prompts]
        while self.has_unfinished():
            self.step()
        return [self.finished[i].output for i in ids]


__all__ = ["AttentionCoordinator", "LLMEngine", "Request"]
