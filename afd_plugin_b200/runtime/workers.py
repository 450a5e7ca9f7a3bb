"""Role workers: one process per GPU (or per CPU rank in tests).

``AFDAttentionWorker`` owns an :class:`LLMEngine` whose FFN boundary goes
through the configured connector; ``AFDFFNWorker`` owns an
:class:`FFNModelRunner` and serves it from a daemon thread, capturing loop
errors and re-raising them on :meth:`AFDFFNWorker.raise_ffn_loop_error_if_any`
(the failure-propagation contract of ``afd_plugin/v1/worker/ffn_worker.py:146-232``).

Group construction is collective: every rank of the AFD world calls
:func:`init_afd_groups` in the same order.
"""

from __future__ import annotations

import logging
import threading
from dataclasses import dataclass

import torch
import torch.distributed as dist

from afd_plugin_b200.config import B200_FUSED_CONNECTOR, AFDConfig, parse_afd_config
from afd_plugin_b200.connectors.factory import AFDConnectorFactory
from afd_plugin_b200.engine_config import EngineConfig
from afd_plugin_b200.parallel.topology import AFDRankMapping, build_rank_mapping, role_of_world_rank
from afd_plugin_b200.validation import assert_compatible_afd_stack

log = logging.getLogger(__name__)
FFN_SHUTDOWN_TIMEOUT_SECONDS = 5.0


@dataclass
class AFDGroups:
    attention_group: object | None  # gloo group over Attention ranks (step agreement)
    ffn_group: object | None  # group over FFN ranks (expert parallel exchange)
    tp_group: object | None = None  # this Attention rank's tensor-parallel peers (tp_size > 1)
    tp_cpu_group: object | None = None  # the same peers over gloo (host-side request fan-out)
    tp_leader: int = -1  # world rank of this rank's TP leader (tp_size > 1)


def init_afd_groups(mapping: AFDRankMapping, tp_size: int = 1) -> AFDGroups:
    """Collective over the whole AFD world.

    Tensor-parallel groups are consecutive Attention role ranks
    ``[dp * tp, dp * tp + tp)`` (the reference's role-rank linearisation).
    """
    attn = dist.new_group(list(mapping.attention_world_ranks), backend="gloo")
    backend = dist.get_backend()
    ffn = dist.new_group(list(mapping.ffn_world_ranks), backend=backend)
    mine = mine_cpu = None
    leader = -1
    if tp_size > 1:
        ranks = list(mapping.attention_world_ranks)
        for start in range(0, len(ranks), tp_size):
            peers = ranks[start : start + tp_size]
            grp = dist.new_group(peers, backend=backend)
            grp_cpu = dist.new_group(peers, backend="gloo")
            if mapping.role == "attention" and mapping.world_rank in peers:
                mine, mine_cpu, leader = grp, grp_cpu, peers[0]
    return AFDGroups(
        attention_group=attn if mapping.role == "attention" else None,
        ffn_group=ffn if mapping.role == "ffn" else None,
        tp_group=mine,
        tp_cpu_group=mine_cpu,
        tp_leader=leader,
    )


def _device_for(local_rank: int) -> torch.device:
    if torch.cuda.is_available() and dist.is_initialized() and dist.get_backend() == "nccl":
        torch.cuda.set_device(local_rank)
        return torch.device("cuda", local_rank)
    return torch.device("cpu")


class _WorkerBase:
    def __init__(self, engine_config: EngineConfig, *, local_rank: int = 0):
        if not dist.is_initialized():
            raise RuntimeError("AFD workers need torch.distributed initialised over the AFD world")
        self.config = engine_config
        self.world_rank = dist.get_rank()
        self.afd: AFDConfig = parse_afd_config(engine_config)
        role, role_rank = role_of_world_rank(
            self.world_rank, attention_size=self.afd.num_attention_ranks, ffn_size=self.afd.num_ffn_ranks)
        if role != self.afd.role:
            raise RuntimeError(f"world rank {self.world_rank} is an {role} rank but config role is {self.afd.role!r}")
        assert_compatible_afd_stack(engine_config, self.afd)
        self.role_rank = role_rank
        self.mapping = build_rank_mapping(self.afd, role_rank)
        self.local_rank = local_rank
        self.device = _device_for(local_rank)
        self.connector = AFDConnectorFactory.create_connector(
            self.world_rank, local_rank, engine_config, self.afd, role_rank)
        self.connector.init_afd_connector()
        self.tp_size = int(getattr(engine_config.parallel_config, "tensor_parallel_size", 1))
        self.groups = init_afd_groups(self.mapping, self.tp_size)
        self.watchdog = self._start_watchdog()

    def _start_watchdog(self):
        """Peer heartbeats over the world's store when ``AFD_HEARTBEAT_TIMEOUT_S`` is set."""
        from afd_plugin_b200.envs import heartbeat_timeout_s

        timeout = heartbeat_timeout_s()
        if timeout is None:
            return None
        from torch.distributed.distributed_c10d import _get_default_store

        from afd_plugin_b200.runtime.watchdog import HeartbeatWatchdog

        return HeartbeatWatchdog(_get_default_store(), self.world_rank, dist.get_world_size(),
                                 period_s=min(0.5, timeout / 5), timeout_s=timeout, prefix="afd_hb").start()

    def check_peers(self) -> None:
        """Raise before launching work that would wait on a peer that stopped heartbeating."""
        if self.watchdog is not None:
            self.watchdog.raise_if_peer_dead()

    def _stop_watchdog(self) -> None:
        if self.watchdog is not None:
            self.watchdog.stop()
            self.watchdog = None


class AFDAttentionWorker(_WorkerBase):
    def __init__(self, engine_config: EngineConfig, *, local_rank: int = 0, seed: int | None = None):
        super().__init__(engine_config, local_rank=local_rank)
        from afd_plugin_b200.models import build_model
        from afd_plugin_b200.runtime.engine import AttentionCoordinator, LLMEngine
        from afd_plugin_b200.runtime.ffn_executor import ConnectorFFNExecutor

        from afd_plugin_b200.models.layers import TPInfo

        mc = engine_config.model_config
        self.peer_ar = None
        if self.tp_size > 1 and self.device.type == "cuda" and mc.dtype == torch.bfloat16:
            # the row-parallel o_proj's partial sums go over peer memory (NCCL for larger tensors)
            from afd_plugin_b200.parallel.tp_allreduce import PeerAllReduce

            self.peer_ar = PeerAllReduce(self.groups.tp_group, max_rows=max(256, engine_config.max_num_seqs),
                                         hidden=mc.arch.hidden_size, device=self.device.index)
        tp = TPInfo(self.role_rank % self.tp_size, self.tp_size, self.groups.tp_group, self.peer_ar)
        self.model = build_model(
            mc.arch, role="attention", dtype=mc.dtype, device=self.device,
            compute_gate_on_attention=self.afd.compute_gate_on_attention,
            route_on_attention=self.afd.connector == B200_FUSED_CONNECTOR,
            seed=mc.seed if seed is None else seed, checkpoint=mc.checkpoint, max_positions=mc.max_model_len, tp=tp)
        A = self.afd.num_attention_ranks
        if self.afd.connector == B200_FUSED_CONNECTOR:
            executor = self.connector.make_executor(self.model)
        else:
            executor = ConnectorFFNExecutor(self.model, self.connector, attn_dp_group=self.groups.attention_group,
                                            attn_size=A, attn_rank=self.role_rank)
        self.executor = executor
        coord = AttentionCoordinator(self.groups.attention_group, A, self.role_rank)
        self.engine = LLMEngine(engine_config, self.model, executor, coordinator=coord)
        if self.watchdog is not None:
            self.engine.health_check = self.check_peers

    def reload_weights(self, checkpoint: str | None = None, *, seed: int | None = None) -> None:
        """Reload the Attention-side weights in place from ``checkpoint`` (default: the configured source)."""
        mc = self.config.model_config
        self.model.reload_weights(checkpoint if checkpoint is not None else mc.checkpoint,
                                  seed=mc.seed if seed is None else seed)

    def shutdown(self) -> None:
        """Stop the FFN loops (control senders only) and release graphs."""
        self._stop_watchdog()
        if self.engine.device.type == "cuda":
            # an async-scheduled decode step may still run: finish it before its graph and the
            # connector's peer memory go away
            torch.cuda.synchronize(self.engine.device)
        self.engine.runner.release_graphs()
        stop = getattr(self.executor, "shutdown_remote", None)
        if callable(stop):
            stop()
        self.connector.close()
        if self.peer_ar is not None:
            torch.cuda.synchronize(self.device)
            self.peer_ar.close()
            self.peer_ar = None


class AFDFFNWorker(_WorkerBase):
    def __init__(self, engine_config: EngineConfig, *, local_rank: int = 0, seed: int | None = None):
        super().__init__(engine_config, local_rank=local_rank)
        from afd_plugin_b200.models import build_model
        from afd_plugin_b200.runtime.ffn_runner import FFNModelRunner

        mc = engine_config.model_config
        F = self.afd.num_ffn_ranks
        self.model = build_model(
            mc.arch, role="ffn", dtype=mc.dtype, device=self.device,
            compute_gate_on_attention=self.afd.compute_gate_on_attention,
            ep_rank=self.role_rank, ep_size=F,
            seed=mc.seed if seed is None else seed, checkpoint=mc.checkpoint)
        if self.afd.connector == B200_FUSED_CONNECTOR:
            self.model_runner = self.connector.make_ffn_runner(self.model)
        else:
            self.model_runner = FFNModelRunner(self.model, self.connector, engine_config,
                                               ep_group=self.groups.ffn_group, ep_size=F, ep_rank=self.role_rank)
        if self.watchdog is not None:
            self.model_runner.health_check = self.check_peers
        self._thread: threading.Thread | None = None
        self._stop: threading.Event | None = None
        self._error: BaseException | None = None

    def execute_model(self, *args, **kwargs):
        raise RuntimeError("AFD FFN workers are connector-driven; scheduler-driven execute_model() is not supported.")

    def start_ffn_server_loop(self) -> None:
        if self._thread is not None and self._thread.is_alive():
            self.raise_ffn_loop_error_if_any()
            return
        self.raise_ffn_loop_error_if_any()
        self._stop = threading.Event()
        self._error = None

        def loop() -> None:
            try:
                if self.device.type == "cuda":
                    torch.cuda.set_device(self.device)
                self.model_runner.serve(stop=self._stop)
            except BaseException as exc:  # noqa: BLE001 - surfaced via raise_ffn_loop_error_if_any
                self._error = exc
                log.exception("AFD FFN worker loop failed")

        self._thread = threading.Thread(target=loop, name="afd-ffn-worker-loop", daemon=True)
        self._thread.start()

    def run_ffn_server_loop(self, max_steps: int | None = None) -> int:
        """Serve in the calling thread (used by benchmarks and tests)."""
        return self.model_runner.serve(max_steps=max_steps)

    def raise_ffn_loop_error_if_any(self) -> None:
        err, self._error = self._error, None
        if err is not None:
            raise RuntimeError("AFD FFN worker loop failed") from err

    def is_loop_alive(self) -> bool:
        return self._thread is not None and self._thread.is_alive()

    def stop_ffn_server_loop(self) -> None:
        if self._stop is not None:
            self._stop.set()
        t = self._thread
        if t is not None:
            t.join(timeout=FFN_SHUTDOWN_TIMEOUT_SECONDS)
        self._thread = None
        self._stop = None
        self.raise_ffn_loop_error_if_any()

    def reload_weights(self, checkpoint: str | None = None, *, seed: int | None = None) -> None:
        """Reload the FFN weights in place; the serving loop must be stopped (no step in flight)."""
        if self.is_loop_alive():
            raise RuntimeError("stop the FFN server loop before reloading weights")
        mc = self.config.model_config
        self.model_runner.reload_weights(checkpoint if checkpoint is not None else mc.checkpoint,
                                         seed=mc.seed if seed is None else seed)

    def shutdown(self) -> None:
        self._stop_watchdog()
        self.stop_ffn_server_loop()
        release = getattr(self.model_runner, "release_graphs", None)
        if callable(release):
            release()
        self.connector.close()


__all__ = ["AFDAttentionWorker", "AFDFFNWorker", "AFDGroups", "FFN_SHUTDOWN_TIMEOUT_SECONDS", "init_afd_groups"]
