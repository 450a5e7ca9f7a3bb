"""B200 fused AFD connector: dispatch and combine inside the kernels, over NVLink.

Data path (no library call, no host hop), at most one token row over NVLink
per FFN rank:

* Attention rank, per layer and ubatch -- ``afd_dispatch``: residual add +
  post-attention RMSNorm (one CTA per token), which stores the normalised row
  into every FFN rank's token buffer for an MoE layer (only the home rank's
  for a dense layer) while the router has not decided yet -- with 2-4 FFN
  ranks a token's top-6/8 experts reach 82-99 % of them -- then the router on
  the tensor cores + top-k, which stores the routing (ids, weights) into every
  FFN rank; FFN ranks that own none of a token's experts ignore its row.  The
  last CTA publishes the token count and bumps every FFN rank's arrival
  counter.
* FFN rank -- ``afd_wait`` for all Attention ranks; ``afd_expand`` copies
  rows into per-expert segments (local HBM); tcgen05 grouped ``gate_up``
  (SwiGLU fused) and ``down`` GEMMs, whose epilogue writes routing-weighted
  rows into a local staging slot per (source, token, expert slot);
  ``afd_combine_send`` sums each token's slots and stores ONE row into the
  source Attention rank's combine slot for this FFN rank (peer memory), then
  bumps every Attention rank's combine counter.
* Attention rank -- ``afd_combine`` waits for every FFN rank and sums the
  token's FFN slots.

Routing always runs on the Attention side here (the Attention role loads the
MoE gate), so expert parallelism across FFN ranks needs no FFN-side
all-to-all; with several FFN ranks each holds ``E / F`` routed experts and a
replica of the shared experts / dense MLPs.

The control plane (per-step payload Attention -> FFN over gloo) only tells the
FFN host loop to replay its captured step; token counts stay on the device, so
one FFN graph serves every routing (key: stages and capacity).

Counters only grow and are compared with ``epoch[stage] * arrivals`` (a
per-stage device epoch bumped inside every captured step that uses the
stage; prefill steps use one stage, DBO decode steps two), so graphs replay
without resets.  Every wait is bounded (``wait_timeout_ms``) and reports through the
device status word instead of hanging.

Semantics follow the reference connector contract
(``afd_plugin/connectors/base.py:37-307``); the transfer mechanism follows the
shape of the reference's Ascend ``a2e``/``e2a`` kernels (device-initiated
peer copies with epoch-tagged flags, ``csrc/npu/a2e/op_kernel/a2e.h:26-382``)
re-designed for NVLink: push instead of pull, per-expert slots, and the FFN
GEMM epilogue as the sender.
"""

from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass
from typing import Any

import torch
import torch.distributed as dist

from afd_plugin_b200.config import AFDConfig
from afd_plugin_b200.config_utils import coerce_extra_bool, coerce_extra_positive_int
from afd_plugin_b200.connectors.base import AFDConnectorBase, ConnectorExtraInfo
from afd_plugin_b200.connectors.metadata import AFDA2FTransferPayload, AFDTransferContext
from afd_plugin_b200.connectors.p2p_nccl import P2pNcclAFDControlPlane
from afd_plugin_b200.parallel.symm_heap import HeapLayout
from afd_plugin_b200.parallel.topology import build_rank_mapping
from afd_plugin_b200.runtime.ffn_executor import FFNExecutor

_EXTRA_KEYS = {"max_tokens_per_rank", "wait_timeout_ms", "fp8_dispatch", "expert_capacity_factor"}


@dataclass(frozen=True)
class B200FusedExtraInfo(ConnectorExtraInfo):
    max_tokens_per_rank: int | None = None  # per Attention rank and ubatch; default: max_num_seqs
    wait_timeout_ms: int = 5000
    fp8_dispatch: bool = False
    # Receive rows per expert as a multiple of the mean load (None: worst case,
    # every token of every Attention rank).  Overflowing rows are dropped and
    # reported through the device status word.
    expert_capacity_factor: float | None = None

    @classmethod
    def from_mapping(cls, raw: Mapping[str, Any] | None) -> "B200FusedExtraInfo":
        raw = dict(raw or {})
        unknown = set(raw) - _EXTRA_KEYS
        if unknown:
            raise ValueError(f"B200FusedAFDConnector: unknown connector_extra_config keys {sorted(unknown)}")
        out = cls(
            max_tokens_per_rank=(coerce_extra_positive_int(raw["max_tokens_per_rank"], field_name="max_tokens_per_rank")
                                 if "max_tokens_per_rank" in raw else None),
            wait_timeout_ms=coerce_extra_positive_int(raw.get("wait_timeout_ms", 5000), field_name="wait_timeout_ms"),
            fp8_dispatch=coerce_extra_bool(raw.get("fp8_dispatch", False), field_name="fp8_dispatch"),
            expert_capacity_factor=_positive_float(raw.get("expert_capacity_factor")),
        )
        return out

    def to_mapping(self) -> dict[str, Any]:
        return {"max_tokens_per_rank": self.max_tokens_per_rank, "wait_timeout_ms": self.wait_timeout_ms,
                "fp8_dispatch": self.fp8_dispatch, "expert_capacity_factor": self.expert_capacity_factor}


def _positive_float(v) -> float | None:
    if v is None or v == "":
        return None
    if isinstance(v, bool):
        raise TypeError("expert_capacity_factor must be a number")
    f = float(v)
    if f <= 0:
        raise ValueError(f"expert_capacity_factor must be positive, got {f}")
    return f


@dataclass(frozen=True)
class FusedLayout:
    """Dimensions shared by every rank (pure arithmetic, CPU-testable)."""

    num_attn: int
    num_ffn: int
    stages: int
    layers: int
    hidden: int
    experts: int
    top_k: int
    t_cap: int  # tokens per Attention rank per stage
    capacity_factor: float | None = None
    # Rows travel as e4m3 with one fp32 scale per 128 columns (half the NVLink bytes).
    fp8: bool = False

    @property
    def ratio(self) -> int:
        return self.num_attn // self.num_ffn

    @property
    def e_local(self) -> int:
        return self.experts // self.num_ffn

    @property
    def cap(self) -> int:
        """Receive rows per routed expert (worst case: every token of every Attention rank)."""
        worst = self.num_attn * self.t_cap
        if self.capacity_factor is None:
            return worst
        mean = worst * self.top_k / max(1, self.experts)
        return min(worst, int(self.capacity_factor * mean) + 64)

    @property
    def rows(self) -> int:
        """Rows of the FFN-side per-expert segments."""
        return self.e_local * self.cap

    @property
    def slots(self) -> int:
        """Combine slots per token: top-k routed + one shared/dense."""
        return self.top_k + 1

    def heap_layout(self) -> HeapLayout:
        """Regions every rank maps (peers write into them)."""
        L = HeapLayout()
        S, A, F = self.stages, self.num_attn, self.num_ffn
        if self.fp8:
            L.add("tok", (S, A, self.t_cap, self.hidden), torch.uint8)     # FFN side: e4m3 token rows per source
            L.add("tok_scale", (S, A, self.t_cap, self.hidden // 128), torch.float32)
        else:
            L.add("tok", (S, A, self.t_cap, self.hidden), torch.bfloat16)  # FFN side: token rows per source
        L.add("rid", (S, A, self.t_cap, self.top_k), torch.int32)          # FFN side: routed expert ids
        L.add("rwt", (S, A, self.t_cap, self.top_k), torch.float32)        # FFN side: routing weights
        L.add("tcount", (S, A), torch.int32)                               # FFN side: tokens per source
        L.add("arrive", (S, self.layers), torch.int64)                     # FFN side: dispatch arrivals
        L.add("comb", (S, self.t_cap, F, self.hidden), torch.bfloat16)     # Attention side: one row per FFN rank
        L.add("comb_flag", (S, self.layers), torch.int64)                  # Attention side: combine arrivals
        L.add("epoch", (S,), torch.int64)
        L.add("done", (S, 4), torch.int32)
        return L

    def stage_bytes(self, layout: HeapLayout, name: str) -> int:
        reg = layout[name]
        return reg.nbytes // self.stages


class B200FusedAFDConnector(AFDConnectorBase):
    supports_graph_capture = True

    @classmethod
    def parse_extra_config(cls, raw: Mapping[str, Any] | None) -> ConnectorExtraInfo:
        if raw is not None and not isinstance(raw, Mapping):
            raise TypeError("B200FusedAFDConnector connector_extra_config must be a mapping")
        return B200FusedExtraInfo.from_mapping(raw)

    def __init__(self, rank: int, local_rank: int, engine_config: Any, afd_config: AFDConfig, role_rank: int) -> None:
        super().__init__(rank, local_rank, engine_config, afd_config, role_rank)
        self.mapping = build_rank_mapping(afd_config, role_rank)
        self.world_rank = self.mapping.world_rank
        self.attn_size = self.mapping.attention_size
        self.ffn_size = self.mapping.ffn_size
        self.min_size = self.mapping.min_size
        self.ratio = self.mapping.ratio
        self.dst_list = list(self.mapping.dp_metadata_destinations)
        self.p2p_rank = self.mapping.p2p_rank
        arch = engine_config.model_config.hf_config
        self.arch = arch
        par = engine_config.parallel_config
        stages = 2 if getattr(par, "use_ubatching", False) else 1
        t_cap = self.extra_info.max_tokens_per_rank or engine_config.max_num_seqs
        if stages == 2:
            t_cap = (t_cap + 1) // 2
        if arch.n_routed_experts and arch.n_routed_experts % self.ffn_size:
            raise ValueError(f"{arch.n_routed_experts} experts do not split over {self.ffn_size} FFN ranks")
        self.dims = FusedLayout(
            num_attn=self.attn_size, num_ffn=self.ffn_size, stages=stages, layers=arch.num_hidden_layers,
            hidden=arch.hidden_size, experts=max(arch.n_routed_experts, self.ffn_size),
            top_k=max(arch.num_experts_per_tok, 1), t_cap=t_cap,
            capacity_factor=self.extra_info.expert_capacity_factor, fp8=bool(self.extra_info.fp8_dispatch))
        if self.dims.fp8 and arch.hidden_size % 128:
            raise ValueError("fp8_dispatch needs the hidden size to be a multiple of 128")
        self.timeout_ns = int(self.extra_info.wait_timeout_ms) * 1_000_000
        self.heap = None
        self.control_group = None
        self._initialized = False
        # P2P control plane semantics (payload per step, first min(A,F) Attention ranks send).
        self.control_plane = P2pNcclAFDControlPlane(self)
        self.dp_metadata_list: dict = {}
        self.tensor_metadata_list: dict = {}
        self._peer_specs: dict = {}
        self._recv_buffers: dict = {}
        self._ids_buffers: dict = {}
        self.group_size = len(self.mapping.subgroup_ranks)
        self.hidden_size = arch.hidden_size
        self.dtype = engine_config.model_config.dtype
        self.device = torch.device("cuda", local_rank)

    # --------------------------------------------------------- lifecycle
    def init_afd_connector(self) -> None:
        if self._initialized:
            return
        from afd_plugin_b200.parallel.symm_heap import SymmetricHeap

        if not dist.is_initialized() or dist.get_world_size() != self.attn_size + self.ffn_size:
            raise RuntimeError("B200FusedAFDConnector needs the AFD world initialised with A + F ranks")
        if dist.get_rank() != self.world_rank:
            raise RuntimeError(f"process has world rank {dist.get_rank()}, AFD topology expects {self.world_rank}")
        group = dist.new_group(list(range(self.ffn_size + self.min_size)), backend="gloo")
        self.control_group = group if self.mapping.participates_in_dp_metadata_group else None
        self.layout = self.dims.heap_layout()
        self.heap = SymmetricHeap(self.layout, device=self.local_rank)
        self._build_views()
        self._initialized = True

    def _build_views(self) -> None:
        d, h = self.dims, self.heap
        for name in ("tok", "rid", "rwt", "tcount", "arrive", "comb", "comb_flag", "epoch", "done"):
            setattr(self, name, h.view(name))
        self.tok_scale = h.view("tok_scale") if d.fp8 else None
        self.fmask = torch.zeros(d.stages, d.t_cap, dtype=torch.int32, device=self.device)
        # dispatch completion counters: [0] send kernel, [1:] router token tiles of 16
        self.dctr = torch.zeros(d.stages, 1 + (d.t_cap + 15) // 16, dtype=torch.int32, device=self.device)
        F, A = d.num_ffn, d.num_attn
        ffn_world = list(range(F))
        attn_world = list(range(F, F + A))
        sb = lambda name: d.stage_bytes(self.layout, name)  # noqa: E731
        # Attention side, per stage: [5, F] -> tok, rid, rwt, tcount, arrive on each FFN rank.
        # FFN side, per stage: comb / comb_flag on each Attention rank.
        self.dispatch_ptrs, self.comb_ptrs, self.comb_flag_ptrs = [], [], []
        names = ("tok", "rid", "rwt", "tcount", "arrive") + (("tok_scale",) if d.fp8 else ())
        for s in range(d.stages):
            rows = [h.ptr_table(ffn_world, n, s * sb(n)) for n in names]
            self.dispatch_ptrs.append(torch.stack(rows))
            self.comb_ptrs.append(h.ptr_table(attn_world, "comb", s * sb("comb")))
            self.comb_flag_ptrs.append(h.ptr_table(attn_world, "comb_flag", s * sb("comb_flag")))

    def close(self) -> None:
        if self.heap is not None:
            self.heap.close()
        self.heap = None
        self.control_group = None
        self._initialized = False

    @property
    def is_initialized(self) -> bool:
        return self._initialized

    def flush(self) -> None:
        return None

    def read_status(self) -> int:
        return int(torch.ops.afd_b200.read_status(self.local_rank))

    # ---------------------------------------------- role-specific engines
    def make_executor(self, model) -> "FusedAttentionExecutor":
        return FusedAttentionExecutor(model, self)

    def make_ffn_runner(self, model) -> "FusedFFNRunner":
        return FusedFFNRunner(model, self, self.engine_config)

    # ------------------------------------------- reference data-path API
    def send_attn_output(self, hidden_states: torch.Tensor, context: AFDTransferContext, **kwargs: Any) -> None:
        raise NotImplementedError(
            "B200FusedAFDConnector sends from the fused dispatch kernel; use make_executor(model)")

    def recv_ffn_output(self, ref_tensor: torch.Tensor, ubatch_idx: int = 0, **kwargs: Any) -> torch.Tensor:
        raise NotImplementedError("B200FusedAFDConnector combines in afd_combine; use make_executor(model)")

    def recv_attn_output(self, ubatch_idx: int = 0, **kwargs: Any) -> AFDA2FTransferPayload:
        raise NotImplementedError("B200FusedAFDConnector FFN side is driven by make_ffn_runner(model)")

    def send_ffn_output(self, ffn_output: torch.Tensor, context: AFDTransferContext, **kwargs: Any) -> None:
        raise NotImplementedError("B200FusedAFDConnector FFN side is driven by make_ffn_runner(model)")


def _routing_cfg(arch) -> tuple[int, int, int, int, int]:
    grouped = arch.topk_method in ("group_limited_greedy", "noaux_tc")
    from afd_plugin_b200.ops import SCORING_IDS

    scoring = SCORING_IDS[arch.scoring_func]
    return (scoring, int(arch.norm_topk_prob), arch.n_group if grouped else 1, arch.topk_group if grouped else 1,
            arch.num_experts_per_tok)


class FusedAttentionExecutor(FFNExecutor):
    """Attention-side FFN boundary on the fused kernels."""

    def __init__(self, model, connector: B200FusedAFDConnector):
        if model.compute_gate_on_attention:
            raise ValueError("B200FusedAFDConnector keeps dense MLPs on the FFN side; use compute_gate_on_attention=false")
        self.model = model
        self.c = connector
        self.arch = model.arch

    def begin_step(self, stage_tokens, **flags) -> None:
        from afd_plugin_b200.connectors.metadata import AFDControlPayload, AFDDPMetadata

        across = flags.get("tokens_across_attn")
        stages = sorted(stage_tokens)
        self._stages = tuple(stages)
        dpl = {}
        for s in stages:
            counts = list(across[s]) if across is not None else [stage_tokens[s]] * self.c.attn_size
            dpl[s] = AFDDPMetadata(num_tokens_across_dp_cpu=counts)
        payload = AFDControlPayload(
            dp_metadata_list=dpl,
            is_graph_capturing=bool(flags.get("is_graph_capturing", False)),
            is_warmup=bool(flags.get("is_warmup", False)),
            is_graph_replaying=bool(flags.get("is_graph_replaying", False)),
        )
        self.c.control_plane.send_dp_metadata_list(payload)

    def step_prologue(self) -> None:
        for s in getattr(self, "_stages", (0,)):
            torch.ops.afd_b200.afd_epoch(self.c.epoch[s : s + 1])

    def check_device_status(self, status: int | None = None) -> None:
        """Raise if a bounded device wait expired; ``status`` is a value already read from
        ``device_status_word()`` (reading the word here synchronises with the current stream)."""
        st = self.c.read_status() if status is None else int(status)
        if st:
            raise RuntimeError(f"Attention step failed on the device (status {st}: a peer wait timed out)")

    def device_status_word(self) -> torch.Tensor:
        """The device's status word (int32 [1]); an async-scheduled engine copies it to the host behind
        each step instead of reading it synchronously."""
        return torch.ops.afd_b200.status_word(self.c.local_rank)

    def send(self, layer_idx, attn_out, residual, stage_idx):
        c, d, a = self.c, self.c.dims, self.arch
        is_moe = a.is_moe_layer(layer_idx)
        layer = self.model.layers[layer_idx]
        T = int(attn_out.shape[0])
        if T > d.t_cap:
            raise ValueError(f"{T} tokens exceed the connector capacity {d.t_cap} per rank and ubatch")
        gate = layer.gate_only
        if is_moe and gate is None:
            raise RuntimeError("fused dispatch needs the MoE gate on the Attention role")
        scoring, renorm, n_group, topk_group, k = _routing_cfg(a)
        has_shared = (not is_moe) or a.has_shared_experts
        cfg = [a.n_routed_experts if is_moe else 1, d.top_k, scoring, renorm, n_group, topk_group, int(is_moe),
               int(has_shared), d.num_ffn, d.e_local, d.t_cap, c.role_rank, c.role_rank // d.ratio, layer_idx]
        gate_w = gate.weight if is_moe else layer.post_attention_layernorm.weight
        bias = gate.e_score_correction_bias if is_moe else None
        hash_table = ids = None
        if is_moe and gate.tid2eid is not None:
            hash_table = gate.tid2eid
        if self.model.fused_post_norm:
            x, res, norm_w, eps = attn_out.contiguous(), residual, layer.post_attention_layernorm.weight, \
                layer.post_attention_layernorm.eps
        else:
            # The model's own residual scheme (mHC) produces the FFN input; the
            # kernel only routes and sends it.
            x, residual = self.model.post_attention_norm(layer_idx, attn_out, residual)
            x = x.contiguous()
            res, norm_w, eps = x, x, 0.0
            cfg.append(1)
        if hash_table is not None:
            ids = self.model.ffn_extra(layer_idx, residual)["input_ids"].to(torch.int32).contiguous()
        torch.ops.afd_b200.afd_dispatch(
            x, res, norm_w, eps, gate_w, bias, float(a.routed_scaling_factor), c.dispatch_ptrs[stage_idx],
            c.fmask[stage_idx], c.dctr[stage_idx], cfg, hash_table, ids)
        return (T, residual)

    def recv(self, layer_idx, handle, stage_idx):
        T, residual = handle
        c, d = self.c, self.c.dims
        if self.timer.enabled:  # split the wait for the FFN ranks from the combine itself
            torch.ops.afd_b200.afd_wait(c.comb_flag[stage_idx], layer_idx, c.epoch[stage_idx : stage_idx + 1],
                                        d.num_ffn, c.timeout_ns)
            self.timer.mark("ffn_wait")
        out = torch.ops.afd_b200.afd_combine(
            c.comb[stage_idx], c.fmask[stage_idx], T, c.comb_flag[stage_idx], layer_idx,
            c.epoch[stage_idx : stage_idx + 1], d.num_ffn, c.timeout_ns)
        return out, residual

    def shutdown_remote(self) -> None:
        from afd_plugin_b200.connectors.metadata import AFDControlPayload, AFDDPMetadata

        payload = AFDControlPayload(dp_metadata_list={0: AFDDPMetadata(num_tokens_across_dp_cpu=[1])},
                                    is_graph_capturing=False, is_warmup=False, is_shutdown=True)
        self.c.control_plane.send_dp_metadata_list(payload)


class FusedFFNRunner:
    """FFN-side step: expand (after a bounded arrival wait), tcgen05 grouped GEMMs, combine-send."""

    def __init__(self, model, connector: B200FusedAFDConnector, engine_config):
        from afd_plugin_b200.runtime.cuda_graph import graph_settings

        self.model = model
        self.c = connector
        self.config = engine_config
        self.device = model.device
        self.use_cuda_graph = graph_settings(engine_config, role="ffn").enabled
        d = connector.dims
        dev = self.device
        S, A, H = d.stages, d.num_attn, d.hidden
        self.f_rank = connector.role_rank
        self.home_a0 = self.f_rank * d.ratio
        self.e_offset = self.f_rank * d.e_local
        # Shared experts packed as virtual experts (chunks of the routed width):
        # home rows are copied into their segments and run in the routed GEMMs.
        self.n_chunks = max((l.mlp.experts.n_extra for i, l in enumerate(model.layers)
                             if model.arch.is_moe_layer(i)), default=0)
        self.J = d.top_k + max(1, self.n_chunks)  # staging slots per token
        self.shared_base = d.rows
        self.shared_stride = d.ratio * d.t_cap
        rows = d.rows + self.n_chunks * self.shared_stride
        # Local buffers (never touched by peers).
        self.x = torch.empty(S, max(1, rows), H, dtype=torch.bfloat16, device=dev)
        self.meta = torch.zeros(S, max(1, rows), dtype=torch.int32, device=dev)
        self.rw = torch.zeros(S, max(1, rows), dtype=torch.float32, device=dev)
        self.counts = torch.zeros(S, d.e_local + max(d.ratio, self.n_chunks), dtype=torch.int32, device=dev)
        self.staging = torch.empty(S, A, d.t_cap, self.J, H, dtype=torch.bfloat16, device=dev)
        # e4m3 rows: expand writes bf16 copies of the home sources' rows here
        self.home_x = (torch.zeros(S, d.ratio * d.t_cap, H, dtype=torch.bfloat16, device=dev) if d.fp8 else None)
        stage_stride = self.staging[0, 0].numel() * self.staging.element_size()
        self.staging_ptrs = [
            torch.tensor([self.staging[s].data_ptr() + a * stage_stride for a in range(A)], dtype=torch.int64,
                         device=dev) for s in range(S)]
        self.off_routed = torch.arange(d.e_local, dtype=torch.int32, device=dev) * d.cap
        self.off_all = torch.cat([self.off_routed, self.shared_base + torch.arange(
            self.n_chunks, dtype=torch.int32, device=dev) * self.shared_stride]).to(torch.int32)
        self.off_shared = torch.arange(d.ratio, dtype=torch.int32, device=dev) * d.t_cap
        # Shared / dense rows are the home sources' token rows; their (source, token, slot) map is static.
        t = torch.arange(d.t_cap, dtype=torch.int32)
        self.meta_shared = torch.cat([((self.home_a0 + i) << 24) | (t << 8) | d.top_k for i in range(d.ratio)]).to(dev)
        self.rw_shared = torch.ones(d.ratio * d.t_cap, dtype=torch.float32, device=dev)
        self.no_flags = torch.zeros(1, dtype=torch.int64, device=dev)
        from afd_plugin_b200.ops.moe import moe_rows_hint, moe_sync_buffer

        self.sync = moe_sync_buffer(dev, d.e_local + self.n_chunks)
        # routed rows per expert (all Attention ranks' tokens) and the home rows of a shared chunk
        self.rows_hint = moe_rows_hint(A * d.t_cap, d.top_k, d.experts, self.n_chunks, d.ratio * d.t_cap)
        self._graphs: dict = {}
        self._pool = None
        self._prepare_weights()
        self.steps = 0
        # Set by benchmarks: count the kernels of the next eager step.
        self.count_next_eager = False
        self.kernels_per_step = 0
        from afd_plugin_b200.utils.phase_timer import NULL_TIMER, PhaseTimer, phase_timing_requested

        self.timer = PhaseTimer(dev) if phase_timing_requested() else NULL_TIMER

    def _prepare_weights(self) -> None:
        """Per layer: routed (w13, w2) and the home-token weights (shared experts or dense MLP)."""
        a = self.model.arch
        self.layer_w = []
        self.layer_s = []  # fp8 block scales matching layer_w (None entries for bf16 weights)
        self.shared_gate_w = []  # per MoE layer: shared-expert gate weight [1, H] or None
        u = lambda t: None if t is None else t.unsqueeze(0)  # noqa: E731
        for i, layer in enumerate(self.model.layers):
            mlp = layer.mlp
            if a.is_moe_layer(i):
                ex = mlp.experts
                if self.n_chunks:
                    self.layer_w.append((ex.w13_all, ex.w2_all, None, None))
                    self.layer_s.append((None, None, None, None))
                    self.shared_gate_w.append(mlp.shared_expert_gate)
                    continue
                if mlp.shared_expert_gate is not None:
                    raise NotImplementedError("fused FFN path: a gated shared expert needs the packed (chunked) layout")
                self.shared_gate_w.append(None)
                shared = mlp.shared_experts
                sw13 = shared.w13.unsqueeze(0) if shared is not None else None
                sw2 = shared.w2.unsqueeze(0) if shared is not None else None
                self.layer_w.append((ex.w13, ex.w2, sw13, sw2))
                self.layer_s.append((ex.w13_scale, ex.w2_scale, u(shared.w13_scale) if shared is not None else None,
                                     u(shared.w2_scale) if shared is not None else None))
            else:
                self.layer_w.append((None, None, mlp.w13.unsqueeze(0), mlp.w2.unsqueeze(0)))
                self.layer_s.append((None, None, u(mlp.w13_scale), u(mlp.w2_scale)))
                self.shared_gate_w.append(None)

    def _layer(self, layer_idx: int, s: int) -> None:
        c, d = self.c, self.c.dims
        C = torch.ops.afd_b200
        A, H = d.num_attn, d.hidden
        w13, w2, sw13, sw2 = self.layer_w[layer_idx]
        s13, s2, ss13, ss2 = self.layer_s[layer_idx]

        def gemm1(x, w, scale, off, cnt, ne):
            if scale is not None:
                return C.grouped_gemm_w8(x, w, scale, off, cnt, 1, ne)
            return C.grouped_gemm_ex(x, w, off, cnt, 1, ne)
        is_moe = w13 is not None
        merged = is_moe and self.n_chunks > 0
        counts = self.counts[s]
        n_chunks = self.n_chunks if merged else 0
        timer = self.timer
        if timer.enabled:  # split the wait for the Attention ranks from the expand copy
            C.afd_wait(c.arrive[s], layer_idx, c.epoch[s : s + 1], A, c.timeout_ns)
            timer.mark("arrive_wait")
        # expand waits (bounded) for every Attention rank's arrival first
        C.afd_expand(c.tok[s], c.rid[s], c.rwt[s], c.tcount[s], self.x[s], self.meta[s], self.rw[s], counts,
                     [A, d.t_cap, d.top_k, d.e_local, self.e_offset, d.cap, d.ratio, self.home_a0, int(is_moe),
                      n_chunks, self.shared_base, self.shared_stride],
                     c.arrive[s], layer_idx, c.epoch[s : s + 1], A, c.timeout_ns,
                     c.tok_scale[s] if d.fp8 else None, self.home_x[s] if d.fp8 else None)
        if d.fp8:
            home_rows = self.home_x[s]
        else:
            home_rows = c.tok[s][self.home_a0 : self.home_a0 + d.ratio].reshape(d.ratio * d.t_cap, H)
        launches = []
        sgw = self.shared_gate_w[layer_idx]
        if merged and sgw is not None:
            # Gated shared expert: each home row's weight is sigmoid(x . w), set in
            # the rows' routing weights before the down projection applies them.
            span = self.shared_stride
            rows = self.x[s][self.shared_base : self.shared_base + span]
            C.gate_sigmoid_rows(rows, sgw[0].contiguous(), self.rw[s][self.shared_base :], n_chunks, span)
        if merged and w13.dtype == torch.bfloat16:
            # routed experts and shared-expert chunks: gate_up -> SwiGLU -> down
            # in one persistent launch whose epilogue scatters into staging
            ne = d.e_local + n_chunks
            total = int(C.moe_ffn_grid(ne, w13.shape[1], w2.shape[1]))
            C.moe_ffn(self.x[s], w13, w2, self.off_all, counts[:ne], self.sync, self.rows_hint, -1, self.meta[s],
                      self.rw[s], self.staging_ptrs[s], self.no_flags, c.done[s, 1:2], counts,
                      [self.J, H, total, 0, layer_idx])
        elif merged:
            ne = d.e_local + n_chunks
            h_r = C.grouped_gemm_ex(self.x[s], w13, self.off_all, counts[:ne], 1, ne)
            launches.append((h_r, w2, self.off_all, counts[:ne], ne, self.meta[s], self.rw[s], None))
        elif is_moe:
            h_r = gemm1(self.x[s], w13, s13, self.off_routed, counts[: d.e_local], d.e_local)
            launches.append((h_r, w2, self.off_routed, counts[: d.e_local], d.e_local, self.meta[s], self.rw[s], s2))
        if sw13 is not None:
            h_s = gemm1(home_rows, sw13, ss13, self.off_shared, counts[d.e_local : d.e_local + d.ratio], 1)
            launches.append((h_s, sw2, self.off_shared, counts[d.e_local : d.e_local + d.ratio], 1, self.meta_shared,
                             self.rw_shared, ss2))
        timer.mark("expand")
        total = sum(int(C.grouped_gemm_grid((H // 128) * int(ln[3].numel()))) for ln in launches)
        for h, w, off, cnt, wexp, meta, rw, scale in launches:
            # Expert outputs land in local staging slots; the last CTA clears the counters.
            C.grouped_gemm_scatter(h, w, off, cnt, wexp, meta, rw, self.staging_ptrs[s], self.no_flags,
                                   c.done[s, 1:2], counts, [self.J, H, total, 0, layer_idx], scale)
        timer.mark("experts")
        has_home = merged or sw13 is not None
        C.afd_combine_send(self.staging[s], c.rid[s], c.rwt[s], c.tcount[s], c.comb_ptrs[s], c.comb_flag_ptrs[s],
                           c.done[s, 2:3], H,
                           [A, d.t_cap, d.top_k, self.J, d.e_local, self.e_offset, d.ratio, self.home_a0,
                            int(is_moe), int(has_home), self.f_rank, d.num_ffn, layer_idx, 0,
                            n_chunks if merged else 1])
        timer.mark("combine_send")

    def _step(self, stages) -> None:
        for s in stages:
            torch.ops.afd_b200.afd_epoch(self.c.epoch[s : s + 1])
        self.timer.begin_step()
        for layer in range(self.model.num_layers):
            for s in stages:
                self._layer(layer, s)

    def execute_model(self, payload) -> None:
        from afd_plugin_b200.runtime.cuda_graph import RunMode, capacity_graph_key, pick_run_mode

        stages = tuple(sorted(payload.dp_metadata_list))
        key = capacity_graph_key(stages, self.c.dims.t_cap)
        entry = self._graphs.get(key)
        mode = pick_run_mode(warmup=payload.is_warmup, capturing=payload.is_graph_capturing,
                             replaying=payload.is_graph_replaying, graphs_on=self.use_cuda_graph,
                             have_graph=entry is not None)
        self.steps += 1
        if mode is RunMode.REPLAY:
            entry.replay()
            return
        if mode is RunMode.CAPTURE and self.use_cuda_graph:
            g = torch.cuda.CUDAGraph()
            if self._pool is None:
                self._pool = torch.cuda.graph_pool_handle()
            with torch.profiler.record_function(f"ffn_capture_{self.c.dims.t_cap}_{len(stages)}"), \
                    torch.cuda.graph(g, pool=self._pool):
                self._step(stages)
            self._graphs[key] = g
            return
        if self.count_next_eager and mode is RunMode.EAGER:
            from afd_plugin_b200.utils.launch_count import count_afd_kernels

            self.count_next_eager = False
            self.kernels_per_step = count_afd_kernels(lambda: self._step(stages))
            return
        self._step(stages)

    def serve(self, *, max_steps: int | None = None, stop=None, check_every: int = 16) -> int:
        """Replay one step per control payload.

        Steps are launched without waiting for the previous one: the captured
        step itself waits (bounded) for the Attention side's arrivals, so the
        host can queue the next step while the device runs.  Behind every step
        the device status word is copied into pinned memory (stream-ordered,
        no host wait); the host checks the latest landed copy before each
        launch, reads the live word every ``check_every`` steps and at the end.
        """
        from afd_plugin_b200.utils.profiler import RoleProfiler

        cp = self.c.control_plane
        prof = RoleProfiler("ffn")
        word = torch.ops.afd_b200.status_word(self.c.local_rank)
        seen = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        n = 0
        try:
            while (max_steps is None or n < max_steps) and not (stop is not None and stop.is_set()):
                check = getattr(self, "health_check", None)
                if check is not None:
                    check()  # a peer stopped heartbeating: fail before waiting on it
                if int(seen[0]):
                    self._check()
                payload = cp.recv_dp_metadata_list()
                if payload.is_shutdown:
                    break
                self.execute_model(payload)
                seen.copy_(word, non_blocking=True)
                n += 1
                prof.step()
                if n % check_every == 0:
                    self._check()
        finally:
            torch.cuda.synchronize(self.device)
            prof.close()
        self._check()
        return n

    def _check(self) -> None:
        st = self.c.read_status()
        if st:
            raise RuntimeError(f"FFN step failed on the device (status {st}: a peer wait timed out)")

    def release_graphs(self) -> None:
        self._graphs.clear()
        self._pool = None

    def reload_weights(self, checkpoint: str | None = None, *, seed: int = 0) -> None:
        """Reload the expert weights in place between steps; captured graphs stay valid."""
        self.model.reload_weights(checkpoint, seed=seed)
        self._prepare_weights()


__all__ = ["B200FusedAFDConnector", "B200FusedExtraInfo", "FusedAttentionExecutor", "FusedFFNRunner", "FusedLayout"]
