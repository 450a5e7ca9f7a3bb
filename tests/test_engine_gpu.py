"""End-to-end decode on the GPU: kernels vs reference model, graphs vs eager."""

import pytest
import torch

from afd_plugin_b200.engine_config import CompilationConfig, EngineConfig, ModelConfig
from afd_plugin_b200.models import build_model, get_preset
from afd_plugin_b200.runtime.engine import LLMEngine

pytestmark = pytest.mark.gpu


def _engine(preset, *, eager, sizes=(8,), device="cuda", dtype=torch.bfloat16, max_len=256, seqs=8, init_on=None,
            async_scheduling=False):
    arch = get_preset(preset)
    ec = EngineConfig(ModelConfig(arch, dtype=dtype, enforce_eager=eager, max_model_len=max_len),
                      compilation_config=CompilationConfig(cudagraph_capture_sizes=list(sizes)), max_num_seqs=seqs,
                      async_scheduling=async_scheduling)
    m = build_model(arch, role="colocated", dtype=dtype, device=device, seed=0, max_positions=max_len,
                    init_on=init_on)
    return LLMEngine(ec, m)


def _prompts(n, length, vocab, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (n, length), generator=g).tolist()


@pytest.mark.parametrize("preset", ["tiny-dsv2", "tiny-dsv2-mla512", "tiny-qwen3-moe", "tiny-qwen3.5", "tiny-dsv4",
                                    "tiny-dsv1"])
def test_graph_decode_matches_eager(preset):
    prompts = _prompts(6, 20, 1024)
    eager = _engine(preset, eager=True).generate(prompts, 8)
    eng = _engine(preset, eager=False)
    eng.capture_graphs()
    assert 8 in eng.runner.graphs
    assert eng.generate(prompts, 8) == eager


@pytest.mark.parametrize("preset", ["tiny-dsv2", "tiny-qwen3.5"])
def test_async_scheduling_graph_decode_matches_sync(preset):
    """Graph replays launched before the previous step's tokens are read (input ids gathered on the
    device, requests of different lengths ending between steps, seeded sampling on the device) give
    the sync engine's tokens."""
    from afd_plugin_b200.runtime.sampling import SamplingParams

    prompts = _prompts(6, 20, 1024)
    lens = [5, 9, 12, 7, 12, 3]
    # greedy rows plus seeded sampled rows (drawn on the device after each replay)
    sps = [SamplingParams(), SamplingParams(temperature=0.8, seed=7), SamplingParams(),
           SamplingParams(temperature=1.1, top_k=40, seed=3), SamplingParams(temperature=0.7, top_p=0.9, seed=9),
           SamplingParams()]

    def run(async_scheduling):
        eng = _engine(preset, eager=False, async_scheduling=async_scheduling)
        eng.capture_graphs()
        ids = [eng.add_request(p, n, sampling=sp) for p, n, sp in zip(prompts, lens, sps)]
        while eng.has_unfinished():
            eng.step()
        return [eng.finished[i].output for i in ids], eng.num_async_steps

    want, _ = run(False)
    got, n_async = run(True)
    assert got == want
    assert n_async >= 8


@pytest.mark.parametrize("async_scheduling", [False, True], ids=["sync", "async"])
def test_dsa_dense_steps_replay_graphs_then_sparse_steps_run_eagerly(async_scheduling):
    """DeepSeek sparse attention: within index_topk the captured dense graph replays; past it the
    engine selects positions eagerly (also with steps launched ahead of their predecessor's
    read-back).  Tokens equal an all-eager engine's."""
    prompts = _prompts(4, 5, 1024)  # index_topk 8: decode steps 1-3 dense, later ones sparse
    eager = _engine("tiny-dsv32", eager=True).generate(prompts, 8)
    eng = _engine("tiny-dsv32", eager=False, async_scheduling=async_scheduling)
    eng.capture_graphs()
    assert 8 in eng.runner.graphs
    assert eng.generate(prompts, 8) == eager
    assert (eng.num_async_steps > 0) == async_scheduling


def test_gpu_prefill_logits_track_fp32_reference():
    """bf16 kernel path vs the fp32 reference model: next-token logits stay close."""
    from afd_plugin_b200.runtime.engine import Request

    arch = get_preset("tiny-dsv2-mla512")
    prompts = _prompts(3, 16, arch.vocab_size, seed=4)
    res = {}
    first_cpu = None
    for dev, dt in (("cpu", torch.float32), ("cuda", torch.bfloat16)):
        e = _engine("tiny-dsv2-mla512", eager=True, device=dev, dtype=dt, init_on="cpu")
        reqs = [Request(i, p, 1) for i, p in enumerate(prompts)]
        for r in reqs:
            e._ensure_blocks(r, len(r.prompt) + 2)
        # prefill then one decode step through the kernels
        first = e.runner.prefill([r.prompt for r in reqs], [r.blocks for r in reqs], [0] * 3)
        if first_cpu is None:
            first_cpu = first.cpu()
        first = first_cpu  # both paths decode the same next inputs
        b = e.runner.buf
        for i, r in enumerate(reqs):
            pos = len(r.prompt)
            b.input_ids[i] = int(first[i])
            b.positions[i] = pos
            b.slot_mapping[i] = r.blocks[pos // e.block_size] * e.block_size + pos % e.block_size
            b.block_table[i, : len(r.blocks)] = torch.tensor(r.blocks, dtype=torch.int32)
            b.seq_lens[i] = pos + 1
        logits = e.runner.forward(b.input_ids[:3], e.runner._decode_metas(3, (0, 3)), (0, 3))
        res[dev] = (first.cpu(), logits.float().cpu())
    torch.testing.assert_close(res["cuda"][1], res["cpu"][1], atol=0.05, rtol=0.05)


def test_dbo_graph_matches_single_ubatch():
    from afd_plugin_b200.engine_config import ParallelConfig

    arch = get_preset("tiny-dsv2-mla512")
    prompts = _prompts(8, 12, 1024, seed=7)
    base = _engine("tiny-dsv2-mla512", eager=True).generate(prompts, 6)
    ec = EngineConfig(ModelConfig(arch, dtype=torch.bfloat16, enforce_eager=False, max_model_len=256),
                      parallel_config=ParallelConfig(use_ubatching=True, num_ubatches=2),
                      compilation_config=CompilationConfig(cudagraph_capture_sizes=[8]), max_num_seqs=8)
    m = build_model(arch, role="colocated", dtype=torch.bfloat16, device="cuda", seed=0, max_positions=256)
    eng = LLMEngine(ec, m)
    eng.capture_graphs()
    assert eng.generate(prompts, 6) == base


def test_qwen3_5_logits_track_fp32_reference():
    """Gated DeltaNet + gated attention + gated shared expert: bf16 kernels vs the fp32 CPU model."""
    from afd_plugin_b200.runtime.engine import Request

    arch = get_preset("tiny-qwen3.5")
    prompts = _prompts(3, 16, arch.vocab_size, seed=5)
    res = {}
    first_cpu = None
    for dev, dt in (("cpu", torch.float32), ("cuda", torch.bfloat16)):
        e = _engine("tiny-qwen3.5", eager=True, device=dev, dtype=dt, init_on="cpu")
        reqs = [Request(i, p, 1) for i, p in enumerate(prompts)]
        for r in reqs:
            e._ensure_blocks(r, len(r.prompt) + 2)
        first = e.runner.prefill([r.prompt for r in reqs], [r.blocks for r in reqs], [0] * 3, [0, 1, 2])
        if first_cpu is None:
            first_cpu = first.cpu()
        first = first_cpu
        b = e.runner.buf
        for i, r in enumerate(reqs):
            pos = len(r.prompt)
            b.input_ids[i] = int(first[i])
            b.positions[i] = pos
            b.slot_mapping[i] = r.blocks[pos // e.block_size] * e.block_size + pos % e.block_size
            b.block_table[i, : len(r.blocks)] = torch.tensor(r.blocks, dtype=torch.int32)
            b.seq_lens[i] = pos + 1
            b.state_slots[i] = i
        logits = e.runner.forward(b.input_ids[:3], e.runner._decode_metas(3, (0, 3)), (0, 3))
        res[dev] = logits.float().cpu()
    torch.testing.assert_close(res["cuda"], res["cpu"], atol=0.05, rtol=0.05)
