"""Attention-side (or colocated) model runner: prefill, decode, graphs, DBO.

One decode step runs ``embed -> layers -> final norm -> LM head -> argmax``
over static device buffers.  The FFN of every layer goes through an
:class:`~afd_plugin_b200.runtime.ffn_executor.FFNExecutor`.

DBO (two ubatches) is a cooperative schedule of two generators: each ubatch
runs its attention, hands its FFN input to the executor and yields; the other
ubatch's attention is then issued before the first one collects its FFN
output.  Every op lands on one CUDA stream in that interleaved order, so a
decode step -- both ubatches, all layers -- captures as ONE CUDA graph
(``FULL_DECODE_ONLY``).  This replaces the reference's two Python threads and
``dbo_yield`` custom op (``afd_plugin/v1/worker/dbo.py:12-73``,
``ubatch_wrapper.py:70-252``).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from afd_plugin_b200 import ops
from afd_plugin_b200.models.layers import AttentionMetadata
from afd_plugin_b200.runtime.ffn_executor import FFNExecutor
from afd_plugin_b200.runtime.kv_cache import PAD_BLOCK, KVCache
from afd_plugin_b200.utils.phase_timer import NULL_TIMER, PhaseTimer, phase_timing_requested


@dataclass
class DecodeBuffers:
    """Static device inputs of a decode step (graph-stable addresses)."""

    input_ids: torch.Tensor
    positions: torch.Tensor
    slot_mapping: torch.Tensor
    block_table: torch.Tensor
    seq_lens: torch.Tensor
    next_tokens: torch.Tensor
    state_slots: torch.Tensor  # linear-attention state row of each batch row
    rows: torch.Tensor         # 0..max_batch (one-token sequence bounds)

    @classmethod
    def allocate(cls, max_batch: int, max_blocks: int, device) -> "DecodeBuffers":
        z = lambda *s, dt: torch.zeros(*s, dtype=dt, device=device)  # noqa: E731
        return cls(
            input_ids=z(max_batch, dt=torch.int32),
            positions=z(max_batch, dt=torch.int64),
            slot_mapping=z(max_batch, dt=torch.int64),
            block_table=z(max_batch, max_blocks, dt=torch.int32),
            seq_lens=torch.ones(max_batch, dtype=torch.int32, device=device),
            next_tokens=z(max_batch, dt=torch.int32),
            state_slots=z(max_batch, dt=torch.int32),
            rows=torch.arange(max_batch + 1, dtype=torch.int32, device=device),
        )


@dataclass
class _Graph:
    graph: torch.cuda.CUDAGraph
    batch: int
    ubatch_splits: tuple[int, ...]
    logits: torch.Tensor | None = None  # the graph's logits output (static address)


def ubatch_splits(batch: int, num_ubatches: int) -> tuple[int, ...]:
    """Request-boundary split points: ``(0, b0, batch)`` for two ubatches."""
    if num_ubatches <= 1 or batch < 2:
        return (0, batch)
    half = (batch + 1) // 2
    return (0, half, batch)


class ModelRunner:
    def __init__(
        self,
        model,
        kv_cache: KVCache,
        ffn_executor: FFNExecutor,
        *,
        max_batch: int,
        max_blocks_per_seq: int,
        num_ubatches: int = 1,
    ):
        self.model = model
        self.kv = kv_cache
        self.ffn = ffn_executor
        self.device = model.device
        self.max_batch = max_batch
        self.max_blocks = max_blocks_per_seq
        self.num_ubatches = num_ubatches
        self.buf = DecodeBuffers.allocate(max_batch, max_blocks_per_seq, self.device)
        self.graphs: dict[int, _Graph] = {}
        self.graph_pool = None
        # Gated DeltaNet layers keep per-sequence state; the last state row pads.
        self.has_linear_state = bool(model.arch.linear_attention_layers)
        self.pad_state_slot = kv_cache.max_seqs - 1
        self.buf.state_slots.fill_(self.pad_state_slot)
        # DeepSeek sparse attention: set by the engine for eager decode steps
        # in which some sequence is longer than index_topk.
        self.sparse_decode = False
        # logits of the last prefill (one row per sequence) or decode step (one per row)
        self.last_logits: torch.Tensor | None = None
        # Device-side phase marks of each step (off unless AFD_PHASE_TIMING=1).
        self.timer = PhaseTimer(self.device) if phase_timing_requested() and self.device.type == "cuda" else NULL_TIMER
        self.ffn.timer = self.timer

    # ------------------------------------------------------------ forward
    def _layers(self, h: torch.Tensor, meta: AttentionMetadata, stage: int):
        """Generator over one ubatch; yields after each layer's FFN send."""
        model = self.model
        residual = None
        timer = self.timer
        for layer in range(model.num_layers):
            attn_out, residual = model.run_attention(layer, h, residual, meta, self.kv.layer(layer))
            timer.mark("attn")
            handle = self.ffn.send(layer, attn_out, residual, stage)
            timer.mark("ffn_send")
            yield None
            h, residual = self.ffn.recv(layer, handle, stage)
            timer.mark("ffn_recv")
        yield (h, residual)

    def _run_stages(self, embeds: list[torch.Tensor], metas: list[AttentionMetadata]):
        gens = [self._layers(h, m, s) for s, (h, m) in enumerate(zip(embeds, metas))]
        results: list = [None] * len(gens)
        live = list(range(len(gens)))
        while live:
            for s in list(live):
                out = next(gens[s])
                if out is not None:
                    results[s] = out
                    live.remove(s)
        return results

    def forward(self, input_ids: torch.Tensor, metas: list[AttentionMetadata], splits: tuple[int, ...],
                **step_flags) -> torch.Tensor:
        """Logits for the last position of each token row (decode) or all rows (prefill)."""
        counts = {s: splits[s + 1] - splits[s] for s in range(len(splits) - 1)}
        self.ffn.begin_step(counts, **step_flags)
        self.ffn.step_prologue()
        self.timer.begin_step()
        for s, m in enumerate(metas):
            m.input_ids = input_ids[splits[s] : splits[s + 1]]
        embeds = [self.model.embed(input_ids[splits[s] : splits[s + 1]]) for s in range(len(splits) - 1)]
        outs = self._run_stages(embeds, metas)
        self.ffn.end_step()
        logits = [self.model.final_logits(h, r) for h, r in outs]
        return logits[0] if len(logits) == 1 else torch.cat(logits, dim=0)

    # ------------------------------------------------------------- decode
    def _decode_metas(self, batch: int, splits: tuple[int, ...]) -> list[AttentionMetadata]:
        b = self.buf
        metas = []
        for s in range(len(splits) - 1):
            lo, hi = splits[s], splits[s + 1]
            metas.append(AttentionMetadata(
                positions=b.positions[lo:hi],
                slot_mapping=b.slot_mapping[lo:hi],
                block_table=b.block_table[lo:hi],
                seq_lens=b.seq_lens[lo:hi],
                is_decode=True,
                state_slots=b.state_slots[lo:hi] if self.has_linear_state else None,
                cu_seqlens=b.rows[: hi - lo + 1] if self.has_linear_state else None,
                sparse_decode=self.sparse_decode,
            ))
        return metas

    def _decode_body(self, batch: int, splits: tuple[int, ...], **flags) -> torch.Tensor:
        b = self.buf
        logits = self.forward(b.input_ids[:batch], self._decode_metas(batch, splits), splits, **flags)
        b.next_tokens[:batch].copy_(ops.argmax(logits))
        return logits

    def decode_step(self, batch: int, *, use_graph: bool = True, **flags) -> torch.Tensor:
        """Run one decode step on ``buf[:batch]``; returns ``next_tokens[:batch]`` (device)."""
        g = self.graphs.get(batch) if use_graph else None
        if g is not None:
            self.ffn.begin_step({s: g.ubatch_splits[s + 1] - g.ubatch_splits[s]
                                 for s in range(len(g.ubatch_splits) - 1)}, is_graph_replaying=True, **flags)
            g.graph.replay()
            self.last_logits = g.logits
        else:
            self.last_logits = self._decode_body(batch, ubatch_splits(batch, self.num_ubatches), **flags)
        return self.buf.next_tokens[:batch]

    def advance_on_device(self, batch: int, *, wrap_at: int = 0, wrap_to: int = 0) -> None:
        """Feed ``next_tokens`` back as inputs and move every row one position.

        Used by device-resident decode loops (benchmarks); rows must own KV
        blocks for the next position already.
        """
        from afd_plugin_b200.ops._ext import ops as cuda_ops

        b = self.buf
        cuda_ops().decode_advance(b.input_ids[:batch], b.positions[:batch], b.slot_mapping[:batch],
                                  b.seq_lens[:batch], b.next_tokens[:batch], b.block_table[:batch],
                                  self.kv.block_size, wrap_at, wrap_to)

    def capture(self, batch: int, *, warmup: int = 2) -> None:
        """Capture one FULL decode graph for a padded batch size."""
        splits = ubatch_splits(batch, self.num_ubatches)
        self.sparse_decode = False  # graphs hold the dense decode
        self._pad_rows(0, batch)
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self._decode_body(batch, splits, is_warmup=True)
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        graph = torch.cuda.CUDAGraph()
        if self.graph_pool is None:
            self.graph_pool = torch.cuda.graph_pool_handle()
        # Control traffic for the capture pass goes out eagerly, outside the graph.
        counts = {i: splits[i + 1] - splits[i] for i in range(len(splits) - 1)}
        self.ffn.begin_step(counts, is_graph_capturing=True)
        begin = self.ffn.begin_step
        self.ffn.begin_step = lambda *a, **k: None  # suppressed inside the graph
        try:
            # named like the reference's capture ranges (attention_model_runner.py:491-496)
            with torch.profiler.record_function(f"capture_{batch}_{'dbo' if len(splits) > 2 else 'full'}"), \
                    torch.cuda.graph(graph, pool=self.graph_pool):
                logits = self._decode_body(batch, splits)
        finally:
            self.ffn.begin_step = begin
        torch.cuda.synchronize(self.device)
        self.graphs[batch] = _Graph(graph, batch, splits, logits)

    def _pad_rows(self, lo: int, hi: int) -> None:
        """Padding rows read/write only the reserved padding block."""
        b = self.buf
        b.input_ids[lo:hi] = 0
        b.positions[lo:hi] = 0
        b.slot_mapping[lo:hi] = PAD_BLOCK * self.kv.block_size
        b.block_table[lo:hi] = PAD_BLOCK
        b.seq_lens[lo:hi] = 1
        b.state_slots[lo:hi] = self.pad_state_slot

    def release_graphs(self) -> None:
        self.graphs.clear()
        self.graph_pool = None

    # ------------------------------------------------------------ prefill
    def prefill(self, token_lists: list[list[int]], block_tables: list[list[int]], start_positions: list[int],
                state_slots: list[int] | None = None, **flags) -> torch.Tensor:
        """Run prompt tokens (eager, one stage); returns the next token of each sequence.

        ``state_slots`` gives each sequence's linear-attention state row (the
        padding row when None); a sequence starting at position 0 starts from a
        zero state.
        """
        bs = self.kv.block_size
        ids, pos, slots, seqs = [], [], [], []
        t = 0
        max_blocks = max(len(bt) for bt in block_tables)
        table = torch.full((len(token_lists), max_blocks), PAD_BLOCK, dtype=torch.int32)
        for i, (toks, bt, p0) in enumerate(zip(token_lists, block_tables, start_positions)):
            table[i, : len(bt)] = torch.tensor(bt, dtype=torch.int32)
            n = len(toks)
            ids.extend(toks)
            pp = list(range(p0, p0 + n))
            pos.extend(pp)
            slots.extend(bt[p // bs] * bs + p % bs for p in pp)
            seqs.append((t, t + n, i))
            t += n
        dev = self.device
        meta = AttentionMetadata(
            positions=torch.tensor(pos, dtype=torch.int64, device=dev),
            slot_mapping=torch.tensor(slots, dtype=torch.int64, device=dev),
            block_table=table.to(dev),
            seq_lens=torch.tensor([p0 + len(x) for x, p0 in zip(token_lists, start_positions)], dtype=torch.int32, device=dev),
            is_decode=False,
            prefill_seqs=seqs,
        )
        if self.has_linear_state:
            slots_l = state_slots if state_slots is not None else [self.pad_state_slot] * len(token_lists)
            cu = [0]
            for toks in token_lists:
                cu.append(cu[-1] + len(toks))
            meta.state_slots = torch.tensor(slots_l, dtype=torch.int32, device=dev)
            meta.cu_seqlens = torch.tensor(cu, dtype=torch.int32, device=dev)
            meta.state_reset = torch.tensor([int(p0 == 0) for p0 in start_positions], dtype=torch.int32, device=dev)
        input_ids = torch.tensor(ids, dtype=torch.int32, device=dev)
        logits = self.forward(input_ids, [meta], (0, t), **flags)
        last = torch.tensor([e - 1 for _, e, _ in seqs], device=dev)
        self.last_logits = logits[last]
        return ops.argmax(self.last_logits)


__all__ = ["DecodeBuffers", "ModelRunner", "ubatch_splits"]
