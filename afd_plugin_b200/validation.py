"""Fail-fast validation of an AFD deployment before any device work.

Checks follow the reference's stack validation
(``afd_plugin/validation.py:36-296``) restated for the standalone runtime:
pipeline parallelism, sequence-parallel MoE, EPLB and elastic EP are refused;
graph mode must be ``FULL_DECODE_ONLY`` with exactly two ubatches when DBO is
on; Qwen3-MoE keeps its gate on the FFN side; Attention rank count must equal
DP x TP of the Attention deployment.
"""

from __future__ import annotations

from typing import Any

from afd_plugin_b200.config import AFD_ASYNC_CONNECTOR, AFDConfig
from afd_plugin_b200.runtime.cuda_graph import graph_settings

AFD_ATTENTION_WORKER_QUALNAME = "afd_plugin_b200.runtime.workers.AFDAttentionWorker"
AFD_FFN_WORKER_QUALNAME = "afd_plugin_b200.runtime.workers.AFDFFNWorker"


def afd_worker_qualname(role: str) -> str:
    if role == "attention":
        return AFD_ATTENTION_WORKER_QUALNAME
    if role == "ffn":
        return AFD_FFN_WORKER_QUALNAME
    raise ValueError(f"unknown AFD role {role!r}")


def assert_worker_matches_role(worker_cls: str | None, afd: AFDConfig) -> None:
    if worker_cls in (None, "", "auto"):
        return
    expected = afd_worker_qualname(afd.role)
    if worker_cls != expected:
        raise ValueError(f"AFD role {afd.role!r} requires worker_cls={expected!r}, got {worker_cls!r}")


def assert_compatible_afd_stack(engine_config: Any, afd: AFDConfig, *, worker_cls: str | None = None) -> None:
    afd.validate()
    assert_worker_matches_role(worker_cls, afd)
    par = engine_config.parallel_config
    if int(getattr(par, "pipeline_parallel_size", 1)) != 1:
        raise ValueError("AFD does not support pipeline parallelism")
    if bool(getattr(par, "use_sequence_parallel_moe", False)):
        raise ValueError("AFD does not support sequence-parallel MoE")
    if bool(getattr(par, "enable_eplb", False)):
        raise ValueError("AFD does not support EPLB")
    if bool(getattr(par, "enable_elastic_ep", False)):
        raise ValueError("AFD does not support elastic expert parallelism")
    if afd.async_dp or afd.connector == AFD_ASYNC_CONNECTOR:
        raise ValueError("AFD async DP (CAMAsyncAFDConnector) is Ascend-only and unavailable on B200")
    if bool(getattr(par, "use_ubatching", False)) and int(getattr(par, "num_ubatches", 0)) != 2:
        raise ValueError("AFD DBO requires exactly two ubatches")
    graph_settings(engine_config, role=afd.role)
    arch = engine_config.model_config.hf_config
    if arch.architecture.startswith("Qwen3") and afd.compute_gate_on_attention:
        raise ValueError("Qwen3-MoE AFD supports compute_gate_on_attention=false only")
    if afd.compute_gate_on_attention and arch.n_routed_experts == 0:
        raise ValueError("compute_gate_on_attention requires a MoE model")
    if afd.role == "attention":
        dp = int(getattr(par, "data_parallel_size", 1))
        tp = int(getattr(par, "tensor_parallel_size", 1))
        pcp = int(getattr(par, "prefill_context_parallel_size", 1))
        if dp * tp * pcp not in (1, afd.num_attention_ranks):
            raise ValueError(
                f"num_attention_ranks={afd.num_attention_ranks} must equal DP*PCP*TP={dp * pcp * tp} "
                "of the Attention deployment"
            )


__all__ = [
    "AFD_ATTENTION_WORKER_QUALNAME",
    "AFD_FFN_WORKER_QUALNAME",
    "afd_worker_qualname",
    "assert_compatible_afd_stack",
    "assert_worker_matches_role",
]
