"""Peer-memory all-reduce for tensor-parallel attention (two GPUs, one process each).

Each rank sums different bf16 partials in place; the result must equal the
fp32 sum of every rank's input (rounded once to bf16), eagerly and replayed
from a CUDA graph, and no bounded wait may expire.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, results) -> None:
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                device_id=torch.device("cuda", rank))
        from afd_plugin_b200.ops._ext import ops
        from afd_plugin_b200.parallel.tp_allreduce import PeerAllReduce

        C = ops()
        C.reset_status(rank)
        ar = PeerAllReduce(dist.group.WORLD, max_rows=64, hidden=2048, device=rank, timeout_ms=5000)
        worst = 0.0
        shapes = [(1, 2048), (37, 2048), (64, 2048), (5, 7168 // 4)]
        for it, (rows, hidden) in enumerate(shapes * 3):  # several calls: both slot parities, reuse
            g = torch.Generator(device="cuda").manual_seed(1000 * it + rank)
            x = torch.randn(rows, hidden, device="cuda", generator=g).to(torch.bfloat16)
            ref = x.float().clone()
            dist.all_reduce(ref)
            ar(x)
            torch.cuda.synchronize()
            worst = max(worst, float((x.float() - ref).abs().max() / ref.abs().max()))
        # CUDA graph: the epoch advances on the device, so replays line up across ranks
        x = torch.zeros(16, 2048, device="cuda", dtype=torch.bfloat16)
        src = torch.empty_like(x)
        graph = torch.cuda.CUDAGraph()
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            x.copy_(src)
            ar(x)
        torch.cuda.current_stream().wait_stream(stream)
        with torch.cuda.graph(graph):
            x.copy_(src)
            ar(x)
        for rep in range(3):
            g = torch.Generator(device="cuda").manual_seed(77 + rep * 10 + rank)
            src.copy_(torch.randn(16, 2048, device="cuda", generator=g).to(torch.bfloat16))
            ref = src.float().clone()
            dist.all_reduce(ref)
            dist.barrier()
            graph.replay()
            torch.cuda.synchronize()
            worst = max(worst, float((x.float() - ref).abs().max() / ref.abs().max()))
        del graph
        status = int(C.read_status(rank))
        dist.barrier()
        ar.close()
        results.put((rank, worst, status))
        dist.destroy_process_group()
    except BaseException as exc:  # noqa: BLE001 - reported to the parent
        results.put((rank, f"{type(exc).__name__}: {exc}", -1))
        raise


def test_peer_allreduce_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    got = [results.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, worst, status in got:
        assert not isinstance(worst, str), (rank, worst)
        assert status == 0, (rank, status)
        assert worst <= 1e-2, (rank, worst)  # one bf16 rounding of an fp32 sum
