"""Per-request decode state hand-off between engines (prefill -> decode disaggregation).

A prefill engine runs a request's prompt, keeps its cache rows (``hold_kv``)
and exports them; a decode engine imports them into freshly allocated blocks
and continues from the next token.  The exported state is exactly what the
decode kernels read:

* MLA layers: the latent rows ``kv [L, n, kv_lora + rope]`` (and the
  sparse-attention indexer's keys ``index_k [L, n, index_head_dim]``);
* GQA layers: ``k`` / ``v`` ``[L, n, kv_heads, head_dim]``;
* Gated DeltaNet layers: the request's ``conv_state`` and fp32 ``ssm_state``.

``n`` is the number of positions whose cache rows have been written (the
prompt plus every generated token but the last).  The blob is a safetensors
file whose metadata carries the token ids and the next token; the importing
engine checks every tensor's shape against its own cache, so a decode engine
with a different model refuses the payload instead of decoding garbage.

The reference leaves the transfer to vLLM KV connectors (LMCache and the
like) driven by its proxy tool (``tools/proxy_server.py:850-867`` builds the
``kv_transfer_params`` of the prefill leg); this module is the framework's own
transport-neutral payload, carried over HTTP by ``serving/api_server.py``.
"""

from __future__ import annotations

import json
import struct
from dataclasses import dataclass

import torch

from afd_plugin_b200.runtime.kv_cache import KVCache

FORMAT = "afd-b200-kv/1"


@dataclass
class RequestState:
    tokens: list[int]  # positions whose cache rows are in ``tensors``
    next_token: int  # the token the decode engine feeds first
    prompt_len: int
    tensors: dict[str, torch.Tensor]
    # a seeded sampled request's generator state, so the decode side continues its noise stream
    rng_state: torch.Tensor | None = None


_RNG_KEY = "__rng_state__"


def _slots(blocks: list[int], n: int, block_size: int, device) -> torch.Tensor:
    pos = torch.arange(n, dtype=torch.int64)
    table = torch.tensor(blocks, dtype=torch.int64)
    return (table[pos // block_size] * block_size + pos % block_size).to(device)


def geometry(cache: KVCache) -> dict:
    """Shapes a payload must match, excluding the token dimension."""
    g: dict = {}
    if cache.kv is not None:
        g["kv"] = [cache.kv.shape[0], cache.kv.shape[3]]
    if cache.index_k is not None:
        g["index_k"] = [cache.index_k.shape[0], cache.index_k.shape[3]]
    if cache.k is not None:
        g["k"] = g["v"] = [cache.k.shape[0], *cache.k.shape[3:]]
    if cache.conv_state is not None:
        g["conv_state"] = [cache.conv_state.shape[0], *cache.conv_state.shape[2:]]
        g["ssm_state"] = [cache.ssm_state.shape[0], *cache.ssm_state.shape[2:]]
    return g


def export_request_state(cache: KVCache, blocks: list[int], n: int, state_slot: int) -> dict[str, torch.Tensor]:
    """Host copies of one request's cache rows for positions ``[0, n)`` and its recurrent state."""
    out: dict[str, torch.Tensor] = {}
    if cache.kv is not None or cache.k is not None:
        dev = (cache.kv if cache.kv is not None else cache.k).device
        slots = _slots(blocks, n, cache.block_size, dev)
        if cache.kv is not None:
            L, W = cache.kv.shape[0], cache.kv.shape[3]
            out["kv"] = cache.kv.view(L, -1, W).index_select(1, slots).cpu()
            if cache.index_k is not None:
                Wi = cache.index_k.shape[3]
                out["index_k"] = cache.index_k.view(L, -1, Wi).index_select(1, slots).cpu()
        else:
            L, tail = cache.k.shape[0], cache.k.shape[3:]
            out["k"] = cache.k.view(L, -1, *tail).index_select(1, slots).cpu()
            out["v"] = cache.v.view(L, -1, *tail).index_select(1, slots).cpu()
    if cache.conv_state is not None:
        out["conv_state"] = cache.conv_state[:, state_slot].cpu()
        out["ssm_state"] = cache.ssm_state[:, state_slot].cpu()
    return out


def import_request_state(cache: KVCache, blocks: list[int], state_slot: int, tensors: dict[str, torch.Tensor],
                         n: int) -> None:
    """Write an exported request into ``blocks`` / ``state_slot`` of ``cache`` (shapes checked)."""
    geo = geometry(cache)
    for name, want in geo.items():
        t = tensors.get(name)
        if t is None:
            raise ValueError(f"KV payload lacks {name!r}")
        paged = name in ("kv", "index_k", "k", "v")
        got = [t.shape[0], *t.shape[2:]] if paged else [t.shape[0], *t.shape[1:]]
        if got != list(want) or (paged and t.shape[1] != n):
            raise ValueError(f"KV payload {name} has shape {tuple(t.shape)}; this engine expects {want} "
                             f"with {n} positions")
    extra = set(tensors) - set(geo)
    if extra:
        raise ValueError(f"KV payload carries tensors this engine has no cache for: {sorted(extra)}")
    if cache.kv is not None or cache.k is not None:
        dev = (cache.kv if cache.kv is not None else cache.k).device
        slots = _slots(blocks, n, cache.block_size, dev)
        if cache.kv is not None:
            L, W = cache.kv.shape[0], cache.kv.shape[3]
            cache.kv.view(L, -1, W).index_copy_(1, slots, tensors["kv"].to(dev, cache.kv.dtype))
            if cache.index_k is not None:
                Wi = cache.index_k.shape[3]
                cache.index_k.view(L, -1, Wi).index_copy_(1, slots, tensors["index_k"].to(dev, cache.index_k.dtype))
        else:
            L, tail = cache.k.shape[0], cache.k.shape[3:]
            cache.k.view(L, -1, *tail).index_copy_(1, slots, tensors["k"].to(dev, cache.k.dtype))
            cache.v.view(L, -1, *tail).index_copy_(1, slots, tensors["v"].to(dev, cache.v.dtype))
    if cache.conv_state is not None:
        cache.conv_state[:, state_slot].copy_(tensors["conv_state"])
        cache.ssm_state[:, state_slot].copy_(tensors["ssm_state"])


def pack(state: RequestState) -> bytes:
    from safetensors.torch import save

    meta = {"format": FORMAT, "tokens": state.tokens, "next_token": int(state.next_token),
            "prompt_len": int(state.prompt_len)}
    tensors = {k: v.contiguous() for k, v in state.tensors.items()}
    if state.rng_state is not None:
        tensors[_RNG_KEY] = state.rng_state.contiguous()
    return save(tensors, metadata={"afd_kv": json.dumps(meta)})


def unpack(blob: bytes) -> RequestState:
    from safetensors.torch import load

    if len(blob) < 8:
        raise ValueError("KV payload is truncated")
    (hlen,) = struct.unpack("<Q", blob[:8])
    header = json.loads(blob[8 : 8 + hlen])
    raw = (header.get("__metadata__") or {}).get("afd_kv")
    if raw is None:
        raise ValueError("not an AFD KV payload")
    meta = json.loads(raw)
    if meta.get("format") != FORMAT:
        raise ValueError(f"unsupported KV payload format {meta.get('format')!r}")
    tensors = load(blob)
    rng = tensors.pop(_RNG_KEY, None)
    return RequestState([int(t) for t in meta["tokens"]], int(meta["next_token"]), int(meta["prompt_len"]),
                        tensors, rng)


__all__ = ["FORMAT", "RequestState", "export_request_state", "geometry", "import_request_state", "pack", "unpack"]
