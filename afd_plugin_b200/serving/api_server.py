"""OpenAI-style completions server over :class:`LLMEngine`.

``EngineLoop`` owns the engine on a background thread: requests are queued
from any thread, the loop admits them and steps the engine while work is
pending, and each request's future resolves with its tokens.  In an AFD
deployment every Attention rank runs an ``EngineLoop``; rank 0 serves HTTP
and the ranks agree each iteration (over the Attention group) whether any of
them has work, so all of them step together (the coordinator pads idle ranks
with a placeholder row, as the reference's DP dummy batches do).

Endpoints: ``GET /health``, ``GET /metrics`` (engine counters),
``POST /v1/completions`` with ``{"prompt": str | [int], "max_tokens": int,
"stream": bool}`` (streamed as server-sent events, one chunk per token),
``POST /v1/chat/completions`` (``messages``; rendered by the tokenizer's chat
template, or :func:`chat_prompt` without one),
and for prefill -> decode disaggregation ``GET`` / ``DELETE /v1/kv/{id}``.

Disaggregated prefill uses the request field ``kv_transfer_params`` with the
keys of the reference's proxy tool (``tools/proxy_server.py:850-867``):
``{"do_remote_decode": true}`` makes this server prefill, keep the request's
cache rows and answer with ``kv_transfer_params`` naming where to fetch them;
``{"do_remote_prefill": true, "remote_request_id", "remote_host",
"remote_port"}`` makes it pull those rows (``runtime/kv_transfer.py``) and
decode from the transferred token on.

Without a tokenizer in the image, text is mapped to token ids byte by byte
(``byte_tokenize``) unless a tokenizer is given (``serving/tokenizer.py``; the
CLI loads the checkpoint's), which keeps the server usable for smoke tests and
benchmark drivers that send token ids directly.
"""

from __future__ import annotations

import json
import queue
import threading
import time
from concurrent.futures import Future
from dataclasses import dataclass, field

import torch
import torch.distributed as dist
from pydantic import BaseModel

from afd_plugin_b200.runtime.sampling import SamplingParams
from afd_plugin_b200.serving.tokenizer import ByteTokenizer, StreamDetokenizer, Tokenizer, render_chat


class SamplingFields(BaseModel):
    """OpenAI-style sampling fields; an omitted or zero ``temperature`` decodes greedily."""

    temperature: float | None = None
    top_p: float | None = None
    top_k: int | None = None
    seed: int | None = None
    stop_token_ids: list[int] | None = None
    ignore_eos: bool | None = None
    # completions: an int (top alternatives per token); chat: a bool, with top_logprobs
    logprobs: int | bool | None = None
    top_logprobs: int | None = None
    n: int = 1
    stop: str | list[str] | None = None  # text stop sequences (checked on the decoded text)
    presence_penalty: float | None = None
    frequency_penalty: float | None = None
    repetition_penalty: float | None = None
    min_tokens: int | None = None
    logit_bias: dict[str, float] | None = None  # token id (as a string, per the OpenAI API) -> bias

    def stop_strings(self) -> list[str]:
        if self.stop is None:
            return []
        return [self.stop] if isinstance(self.stop, str) else [x for x in self.stop if x]

    def n_logprobs(self) -> int | None:
        if self.logprobs is None or self.logprobs is False:
            return None
        if self.logprobs is True:
            return int(self.top_logprobs or 0)
        return int(self.logprobs)

    def sampling(self, index: int = 0) -> SamplingParams | None:
        """The parameters of choice ``index`` (seeded choices use seed + index)."""
        lp = self.n_logprobs()
        if all(v is None for v in (self.temperature, self.top_p, self.top_k, self.seed, self.stop_token_ids,
                                   self.ignore_eos, lp, self.presence_penalty, self.frequency_penalty,
                                   self.repetition_penalty, self.min_tokens, self.logit_bias)):
            return None
        return SamplingParams(temperature=float(self.temperature or 0.0),
                              top_k=max(0, int(self.top_k or 0)),  # vLLM's -1 = off
                              top_p=float(self.top_p if self.top_p is not None else 1.0),
                              seed=None if self.seed is None else self.seed + index,
                              stop_token_ids=tuple(int(t) for t in self.stop_token_ids or ()),
                              ignore_eos=bool(self.ignore_eos), logprobs=lp,
                              presence_penalty=float(self.presence_penalty or 0.0),
                              frequency_penalty=float(self.frequency_penalty or 0.0),
                              repetition_penalty=1.0 if self.repetition_penalty is None else float(self.repetition_penalty),
                              min_tokens=int(self.min_tokens or 0),
                              logit_bias=tuple((int(t), float(b)) for t, b in (self.logit_bias or {}).items()))


class CompletionRequest(SamplingFields):
    # one prompt (text or token ids) or a batch of them
    prompt: str | list[int] | list[str] | list[list[int]]
    max_tokens: int = 16
    model: str | None = None
    kv_transfer_params: dict | None = None
    stream: bool = False
    echo: bool = False  # the returned text starts with the prompt


class ChatMessage(BaseModel):
    role: str
    # a string, or OpenAI content parts ([{"type": "text", "text": ...}, ...]); text parts are joined
    content: str | list[dict] | None = None

    @property
    def text(self) -> str:
        if self.content is None:
            return ""
        if isinstance(self.content, str):
            return self.content
        parts = []
        for part in self.content:
            if part.get("type", "text") != "text":
                raise ValueError(f"chat content part of type {part.get('type')!r} is not served (text only)")
            parts.append(str(part.get("text", "")))
        return "".join(parts)


class ChatCompletionRequest(SamplingFields):
    messages: list[ChatMessage]
    max_tokens: int | None = None
    max_completion_tokens: int | None = None
    model: str | None = None
    kv_transfer_params: dict | None = None
    stream: bool = False


def chat_prompt(messages: list[ChatMessage]) -> str:
    """Plain role-tagged transcript ending in the assistant tag (chat without a template)."""
    return render_chat([{"role": m.role, "content": m.text} for m in messages])


def byte_tokenize(text: str, vocab_size: int) -> list[int]:
    return [b % vocab_size for b in text.encode("utf-8")] or [0]


def byte_detokenize(ids: list[int]) -> str:
    return bytes(i % 256 for i in ids).decode("utf-8", errors="replace")


@dataclass
class _Pending:
    prompt: list[int]
    max_tokens: int
    future: Future
    submitted: float = field(default_factory=time.perf_counter)
    hold_kv: bool = False
    kv_blob: bytes | None = None  # prefilled elsewhere: the exported cache rows
    first_token_at: float | None = None
    # streaming: every new token goes here as it is produced, then None (or the error)
    stream: queue.Queue | None = None
    req: object | None = None  # the engine's Request, for streaming
    sent: int = 0
    sampling: SamplingParams | None = None
    # text stop sequences: decoded text so far and the text cut before the stop
    stop_strings: list[str] = field(default_factory=list)
    text: str = ""
    checked: int = 0
    stop_text: str | None = None


class EngineLoop:
    """Steps an engine on a background thread.

    ``group`` / ``world`` / ``rank``: the Attention ranks that must step
    together (None for a single engine).  With attention tensor parallelism
    (``tp_size > 1``) only the TP leader (world rank ``tp_src``) takes
    requests; each iteration it broadcasts the new ones over ``tp_group`` (a
    gloo group of its TP peers) and every peer admits the same requests in the
    same order, so their engines hold identical batches.
    """

    def __init__(self, engine, *, group=None, world: int = 1, rank: int = 0, idle_sleep_s: float = 0.001,
                 kv_hold_timeout_s: float = 120.0, tp_group=None, tp_size: int = 1, tp_src: int = 0,
                 decode_bench: bool = False):
        self.engine = engine
        self.tokenizer = None  # set by build_app: decodes text for stop sequences
        # decode-bench serving: prompts are taken as prefilled (no prefill step)
        self.decode_bench = decode_bench
        self.group, self.world, self.rank = group, world, rank
        self.tp_group, self.tp_size, self.tp_src = tp_group, tp_size, tp_src
        self.tp_leader = tp_size <= 1 or dist.get_rank() == tp_src
        self.idle_sleep_s = idle_sleep_s
        self.kv_hold_timeout_s = kv_hold_timeout_s
        self._queue: list[_Pending] = []
        self._calls: list[tuple[object, Future]] = []
        self._lock = threading.Lock()
        self._inflight: dict[int, _Pending] = {}
        self._stop = threading.Event()
        self._thread: threading.Thread | None = None
        self.error: BaseException | None = None
        self.stats = {"requests": 0, "completed": 0, "aborted": 0, "generated_tokens": 0, "steps": 0,
                      "ttft_s_sum": 0.0, "ttft_count": 0, "tpot_s_sum": 0.0, "tpot_count": 0}

    # ------------------------------------------------------------ clients
    def _check_entry(self, handoff: bool) -> None:
        if self.error is not None:
            raise RuntimeError("engine loop has failed") from self.error
        if not self.tp_leader:
            raise RuntimeError("requests enter through the TP leader's loop")
        if handoff and self.tp_size > 1:
            raise ValueError("prefill/decode KV hand-off is not supported with attention tensor parallelism")

    def submit(self, prompt: list[int], max_tokens: int, *, hold_kv: bool = False,
               stream: queue.Queue | None = None, sampling: SamplingParams | None = None,
               stop: list[str] | None = None) -> Future:
        """Queue a request; the future resolves with its tokens and carries ``req_id`` once admitted.

        With ``stream`` every token is also put on that queue as soon as it is
        produced, followed by None (or the exception that ended the request).
        """
        self._check_entry(hold_kv)
        if stop and self.tp_size > 1:  # ending a request early would need the TP peers to end it too
            raise ValueError("text stop sequences are not supported with attention tensor parallelism")
        limit = self.engine.config.model_config.max_model_len
        if len(prompt) + int(max_tokens) > limit:
            raise ValueError(f"prompt ({len(prompt)}) + max_tokens ({max_tokens}) exceeds max_model_len {limit}")
        fut: Future = Future()
        with self._lock:
            self._queue.append(_Pending(list(prompt), int(max_tokens), fut, hold_kv=hold_kv, stream=stream,
                                        sampling=sampling, stop_strings=list(stop or [])))
            self.stats["requests"] += 1
        return fut

    def submit_prefilled(self, prompt: list[int], kv_blob: bytes, max_tokens: int, *,
                         stream: queue.Queue | None = None, sampling: SamplingParams | None = None,
                         stop: list[str] | None = None) -> Future:
        """Queue a request whose prompt was prefilled by another engine (see ``export_kv``)."""
        self._check_entry(True)
        if stop and self.tp_size > 1:
            raise ValueError("text stop sequences are not supported with attention tensor parallelism")
        fut: Future = Future()
        with self._lock:
            self._queue.append(_Pending(list(prompt), int(max_tokens), fut, kv_blob=kv_blob, stream=stream,
                                        sampling=sampling, stop_strings=list(stop or [])))
            self.stats["requests"] += 1
        return fut

    def abort(self, req_id: int) -> Future:
        """Stop a request whose client went away (resolves with the tokens it has).

        Not available with attention tensor parallelism: the TP peers would
        keep the request, so it runs to completion there.
        """
        if self.tp_size > 1:
            fut: Future = Future()
            fut.set_result(False)
            return fut
        return self.call(lambda eng: eng.abort(req_id))

    def call(self, fn) -> Future:
        """Run ``fn(engine)`` on the loop thread between steps (engine state is not thread-safe)."""
        fut: Future = Future()
        with self._lock:
            self._calls.append((fn, fut))
        return fut

    # --------------------------------------------------------------- loop
    def start(self) -> "EngineLoop":
        self._thread = threading.Thread(target=self._run, name="afd-engine-loop", daemon=True)
        self._thread.start()
        return self

    def stop(self, timeout: float = 60.0) -> None:
        """Stop this loop; with peers, every rank's loop leaves at the same iteration."""
        self._stop.set()
        self.join(timeout)

    def join(self, timeout: float | None = None) -> None:
        """Wait until the loop ends (a peer's stop ends it on every rank)."""
        if self._thread is not None:
            self._thread.join(timeout)
            if not self._thread.is_alive():
                self._thread = None

    def _hit_stop(self, p: _Pending) -> bool:
        """Decode the request's new tokens; True (and the text cut before it) once a stop string shows."""
        tok = self.tokenizer
        if tok is None or p.req is None:
            return False
        first = 1 if getattr(p.req, "synthetic_prefill", False) else 0
        ids = p.req.output[first:]
        p.text = tok.decode(ids)
        p.checked = len(ids)
        cut = min((i for i in (p.text.find(st) for st in p.stop_strings) if i >= 0), default=-1)
        if cut < 0:
            return False
        p.stop_text = p.text[:cut]
        return True

    @staticmethod
    def _push_tokens(p: _Pending) -> None:
        out = p.req.output if p.req is not None else []
        for t in out[p.sent :]:
            p.stream.put(t)
        p.sent = len(out)

    def _fan_out(self, new: list[_Pending]) -> list[_Pending]:
        """TP leader -> peers: this iteration's new requests (one gloo broadcast)."""
        obj = [[(p.prompt, p.max_tokens, p.sampling) for p in new]] if self.tp_leader else [None]
        dist.broadcast_object_list(obj, src=self.tp_src, group=self.tp_group)
        if self.tp_leader:
            return new
        return [_Pending(list(pr), int(mt), Future(), sampling=sp) for pr, mt, sp in obj[0]]

    def _agree(self, work: bool, stop: bool) -> tuple[bool, bool]:
        """(any rank has work, any rank stops) -- one collective per iteration on every rank."""
        if self.group is None or self.world <= 1:
            return work, stop
        flag = torch.tensor([int(work), int(stop)])
        dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=self.group)
        return bool(flag[0]), bool(flag[1])

    def _run(self) -> None:
        eng = self.engine
        try:
            if eng.device.type == "cuda":
                torch.cuda.set_device(eng.device)
            while True:
                with self._lock:
                    new, self._queue = self._queue, []
                    calls, self._calls = self._calls, []
                if self.tp_size > 1:
                    new = self._fan_out(new)
                for fn, fut in calls:
                    try:
                        fut.set_result(fn(eng))
                    except Exception as exc:  # noqa: BLE001 - handed to the caller
                        fut.set_exception(exc)
                if calls:
                    self._resolve_finished(time.perf_counter())  # e.g. requests a call aborted
                if eng.held:
                    eng.expire_held(self.kv_hold_timeout_s)
                for p in new:
                    try:
                        if p.kv_blob is not None:
                            rid, _ = eng.add_prefilled_request(p.kv_blob, p.max_tokens, prompt=p.prompt,
                                                               sampling=p.sampling)
                        elif self.decode_bench and not p.hold_kv:
                            rid = eng.add_synthetic_request(p.prompt, p.max_tokens, sampling=p.sampling)
                            p.sent = 1  # output[0] is the last prompt token: never streamed
                        else:
                            rid = eng.add_request(p.prompt, p.max_tokens, hold_kv=p.hold_kv, sampling=p.sampling)
                    except ValueError as exc:
                        p.future.set_exception(exc)
                        if p.stream is not None:
                            p.stream.put(exc)
                        continue
                    p.future.req_id = rid
                    self._inflight[rid] = p
                    if p.stream is not None or p.stop_strings:
                        p.req = eng.request(rid)
                    if p.stream is not None:
                        self._push_tokens(p)  # a transferred first token streams at once
                work, stop = self._agree(eng.has_unfinished(), self._stop.is_set())
                if stop:
                    break
                if not work:
                    time.sleep(self.idle_sleep_s)
                    continue
                produced = eng.step()
                now = time.perf_counter()
                self.stats["steps"] += 1
                for rid in produced:
                    p = self._inflight.get(rid)
                    if p is None:
                        continue
                    if p.first_token_at is None:
                        p.first_token_at = now
                        self.stats["ttft_s_sum"] += now - p.submitted
                        self.stats["ttft_count"] += 1
                    if p.stop_strings and self._hit_stop(p):
                        eng.abort(rid)  # ends it now; resolved below with finish_reason "stop"
                        continue
                    if p.stream is not None:
                        self._push_tokens(p)
                self._resolve_finished(now)
        except BaseException as exc:  # noqa: BLE001 - surfaced to every waiting client
            self._fail_all(exc)

    def _resolve_finished(self, now: float) -> None:
        eng = self.engine
        for rid in [r for r in self._inflight if r in eng.finished]:
            p = self._inflight.pop(rid)
            req = eng.finished.pop(rid)
            out = req.output[1:] if req.synthetic_prefill else req.output
            stopped = p.stop_text is not None
            self.stats["aborted" if req.aborted and not stopped else "completed"] += 1
            self.stats["generated_tokens"] += len(out)
            if p.first_token_at is not None and len(out) > 1 and not req.aborted:
                self.stats["tpot_s_sum"] += (now - p.first_token_at) / (len(out) - 1)
                self.stats["tpot_count"] += 1
            p.future.finish_reason = "stop" if p.stop_text is not None else req.finish_reason
            if p.stop_text is not None:
                p.future.text = p.stop_text
            skip = 1 if req.synthetic_prefill else 0
            p.future.logprobs = (req.token_logprobs[skip:], req.top_logprobs[skip:])
            if p.stream is not None:
                self._push_tokens(p)
                p.stream.put(None)
            p.future.set_result(out)

    def _fail_all(self, exc: BaseException) -> None:
        self.error = exc
        for p in list(self._inflight.values()) + self._queue:
            if not p.future.done():
                p.future.set_exception(exc)
            if p.stream is not None:
                p.stream.put(exc)
        for _, fut in self._calls:
            if not fut.done():
                fut.set_exception(exc)


def build_app(loop: EngineLoop, *, model_name: str = "afd-b200", request_timeout_s: float = 600.0,
              advertise_host: str = "127.0.0.1", advertise_port: int = 8000, tokenizer: Tokenizer | None = None):
    """FastAPI app serving ``loop`` (rank 0 of the Attention side).

    ``advertise_host`` / ``advertise_port`` are what a prefill answer tells the
    decode server to fetch the cache rows from.
    """
    import requests
    from fastapi import FastAPI, HTTPException
    from fastapi.responses import Response, StreamingResponse

    vocab = loop.engine.model.arch.vocab_size
    tok = tokenizer or ByteTokenizer(vocab)
    if loop.tokenizer is None:
        loop.tokenizer = tok
    app = FastAPI(title="afd_plugin_b200")

    def _fetch_kv(params: dict) -> bytes:
        try:
            url = f"http://{params['remote_host']}:{int(params['remote_port'])}/v1/kv/{int(params['remote_request_id'])}"
        except (KeyError, TypeError, ValueError) as exc:
            raise HTTPException(status_code=400, detail=f"incomplete kv_transfer_params: {exc}") from exc
        try:
            r = requests.get(url, timeout=request_timeout_s)
        except requests.RequestException as exc:
            raise HTTPException(status_code=502, detail=f"KV fetch from {url} failed: {exc}") from exc
        if r.status_code != 200:
            raise HTTPException(status_code=502, detail=f"KV fetch from {url}: HTTP {r.status_code}")
        return r.content

    def _new_id(chat: bool) -> tuple[str, int]:
        import uuid

        return ("chatcmpl-" if chat else "cmpl-") + uuid.uuid4().hex, int(time.time())

    def _chunk(chat: bool, model: str, tokens: list[int], text: str, finish: str | None,
               usage: dict | None = None, ident: tuple[str, int] = ("", 0)) -> str:
        if chat:
            delta = {"role": "assistant", "content": text} if tokens or text else {}
            msg = {"id": ident[0], "object": "chat.completion.chunk", "created": ident[1], "model": model,
                   "choices": [{"index": 0, "delta": delta, "token_ids": tokens, "finish_reason": finish}]}
        else:
            msg = {"id": ident[0], "object": "text_completion", "created": ident[1], "model": model,
                   "choices": [{"index": 0, "token_ids": tokens, "text": text, "finish_reason": finish}]}
        if usage is not None:
            msg["usage"] = usage
        return "data: " + json.dumps(msg) + "\n\n"

    async def _sse(tokens: queue.Queue, fut: Future, n_prompt: int, model: str, chat: bool,
                   ident: tuple[str, int] = ("", 0)):
        """Server-sent events: one chunk per token, a final chunk with usage, then ``[DONE]``.

        Runs on the event loop; a client that disconnects cancels it at its
        next await, and the request is then aborted so it stops taking a
        batch slot.
        """
        import functools

        import anyio

        n, ended = 0, False
        detok = StreamDetokenizer(tok)
        deadline = time.monotonic() + request_timeout_s
        try:
            while True:
                try:
                    t = await anyio.to_thread.run_sync(functools.partial(tokens.get, timeout=0.25))
                except queue.Empty:
                    if time.monotonic() < deadline:
                        continue
                    t = TimeoutError("no token within the request timeout")
                if t is None:
                    break
                if isinstance(t, BaseException):
                    ended = True
                    yield "data: " + json.dumps({"error": {"message": str(t), "type": type(t).__name__}}) + "\n\n"
                    return
                n += 1
                deadline = time.monotonic() + request_timeout_s
                yield _chunk(chat, model, [t], detok.push(t), None, ident=ident)
            ended = True
            yield _chunk(chat, model, [], detok.flush(), getattr(fut, "finish_reason", "length"),
                         {"prompt_tokens": n_prompt, "completion_tokens": n, "total_tokens": n_prompt + n}, ident)
            yield "data: [DONE]\n\n"
        finally:
            rid = getattr(fut, "req_id", None)
            if not ended and rid is not None:
                loop.abort(rid)

    def _logprobs_block(chat: bool, out: list[int], lps: tuple[list, list]) -> dict:
        chosen, tops = lps
        pieces = [tok.decode([t]) for t in out]
        if chat:
            return {"content": [{"token": piece, "logprob": c,
                                 "top_logprobs": [{"token": tok.decode([i]), "logprob": v} for i, v in top]}
                                for piece, c, top in zip(pieces, chosen, tops)]}
        offsets, pos = [], 0
        for piece in pieces:
            offsets.append(pos)
            pos += len(piece)
        return {"tokens": pieces, "token_logprobs": chosen, "text_offset": offsets,
                "top_logprobs": [{tok.decode([i]): v for i, v in top} for top in tops]}

    def _generate(ids: list[int], max_tokens: int, params: dict | None, stream_req: bool, model: str, chat: bool,
                  fields: SamplingFields):
        try:
            n = int(fields.n)
            if n < 1:
                raise ValueError("n must be >= 1")
            samplings = [fields.sampling(i) for i in range(n)]
        except ValueError as exc:
            raise HTTPException(status_code=400, detail=str(exc)) from exc
        if max_tokens < 1:
            raise HTTPException(status_code=400, detail="max_tokens must be positive")
        if any((not isinstance(t, int)) or t < 0 or t >= vocab for t in ids):
            raise HTTPException(status_code=400, detail=f"prompt token ids must be in [0, {vocab})")
        params = params or {}
        prefill_only = bool(params.get("do_remote_decode"))
        if n > 1 and (stream_req or prefill_only or params.get("do_remote_prefill")):
            raise HTTPException(status_code=400, detail="n > 1 is served without streaming or KV hand-off")
        echo = bool(getattr(fields, "echo", False)) and not chat
        if echo and stream_req:
            raise HTTPException(status_code=400, detail="echo is served without streaming")
        stream = queue.Queue() if stream_req and not prefill_only else None
        try:
            stops = fields.stop_strings()
            if params.get("do_remote_prefill"):
                futs = [loop.submit_prefilled(ids, _fetch_kv(params), max_tokens, stream=stream,
                                              sampling=samplings[0], stop=stops)]
            else:
                futs = [loop.submit(ids, max_tokens, hold_kv=prefill_only, stream=stream, sampling=sp, stop=stops)
                        for sp in samplings]
            if stream is not None:
                return StreamingResponse(_sse(stream, futs[0], len(ids), model, chat, _new_id(chat)),
                                         media_type="text/event-stream")
            outs = [f.result(timeout=request_timeout_s) for f in futs]
        except ValueError as exc:
            raise HTTPException(status_code=400, detail=str(exc)) from exc
        except RuntimeError as exc:  # the engine loop failed (or this rank takes no requests)
            raise HTTPException(status_code=503, detail=str(exc)) from exc
        n_out = sum(len(o) for o in outs)
        usage = {"prompt_tokens": len(ids), "completion_tokens": n_out, "total_tokens": len(ids) + n_out}
        choices = []
        for i, (f, out) in enumerate(zip(futs, outs)):
            reason = getattr(f, "finish_reason", "length")
            text = getattr(f, "text", None)
            text = tok.decode(out) if text is None else text
            if chat:
                c = {"index": i, "message": {"role": "assistant", "content": text}, "token_ids": out,
                     "finish_reason": reason}
            else:
                c = {"index": i, "token_ids": out, "text": (tok.decode(ids) + text) if echo else text,
                     "finish_reason": reason}
            if samplings[i] is not None and samplings[i].logprobs is not None:
                c["logprobs"] = _logprobs_block(chat, out, getattr(f, "logprobs", ([], [])))
            choices.append(c)
        ident = _new_id(chat)
        body = {"id": ident[0], "object": "chat.completion" if chat else "text_completion", "created": ident[1],
                "model": model, "usage": usage, "choices": choices}
        if prefill_only:
            body["kv_transfer_params"] = {
                "do_remote_prefill": True, "do_remote_decode": False,
                "remote_request_id": futs[0].req_id, "remote_host": advertise_host, "remote_port": advertise_port,
            }
        return body

    @app.get("/v1/kv/{req_id}")
    def get_kv(req_id: int):
        try:
            blob = loop.call(lambda eng: eng.export_kv(req_id)).result(timeout=request_timeout_s)
        except KeyError as exc:
            raise HTTPException(status_code=404, detail=f"no held KV for request {req_id}") from exc
        return Response(content=blob, media_type="application/octet-stream")

    @app.delete("/v1/kv/{req_id}")
    def drop_kv(req_id: int):
        released = loop.call(lambda eng: eng.release_kv(req_id)).result(timeout=request_timeout_s)
        return {"released": bool(released)}

    @app.get("/v1/models")
    def models():
        return {"object": "list", "data": [{
            "id": model_name, "object": "model", "owned_by": "afd_plugin_b200",
            "max_model_len": loop.engine.config.model_config.max_model_len,
            "architecture": loop.engine.model.arch.architecture}]}

    @app.post("/reset_prefix_cache")
    def reset_prefix_cache():
        if not getattr(loop.engine, "prefix_caching", False):
            return {"reset": False, "reason": "prefix caching is off"}
        n = loop.call(lambda eng: eng.reset_prefix_cache()).result(timeout=request_timeout_s)
        return {"reset": True, "cached_blocks_dropped": n}

    @app.get("/health")
    def health():
        if loop.error is not None:
            raise HTTPException(status_code=503, detail=f"engine failed: {loop.error!r}")
        return {"status": "ok"}

    @app.get("/metrics")
    def metrics():
        out = dict(loop.stats)
        st = loop.stats
        out["mean_ttft_s"] = round(st["ttft_s_sum"] / st["ttft_count"], 6) if st["ttft_count"] else None
        out["mean_tpot_s"] = round(st["tpot_s_sum"] / st["tpot_count"], 6) if st["tpot_count"] else None
        m = getattr(loop.engine, "metrics", None)
        if m is not None:
            out.update(m.summary())
        alloc = loop.engine.kv.allocator
        if getattr(loop.engine, "prefix_caching", False):
            out["prefix_cache_hit_rate"] = round(alloc.hits / alloc.queries, 4) if alloc.queries else None
        out["kv_blocks_free"] = alloc.num_free
        out["preemptions"] = getattr(loop.engine, "num_preemptions", 0)
        out["async_steps"] = getattr(loop.engine, "num_async_steps", 0)
        return out

    @app.get("/metrics/prometheus")
    def metrics_prometheus():
        """The /metrics counters and gauges in the Prometheus text exposition format."""
        from fastapi.responses import PlainTextResponse

        m = metrics()
        kinds = {"requests": "counter", "completed": "counter", "aborted": "counter", "generated_tokens": "counter",
                 "steps": "counter", "preemptions": "counter", "decode_tokens": "counter", "async_steps": "counter"}
        lines = []
        for key, value in sorted(m.items()):
            if not isinstance(value, (int, float)) or isinstance(value, bool):
                continue
            name = "afd_" + key + ("_total" if kinds.get(key) == "counter" else "")
            lines.append(f"# TYPE {name} {kinds.get(key, 'gauge')}")
            lines.append(f'{name}{{model="{model_name}"}} {float(value)}')
        return PlainTextResponse("\n".join(lines) + "\n", media_type="text/plain; version=0.0.4")

    @app.post("/v1/completions")
    def completions(req: CompletionRequest):
        p = req.prompt
        batch = isinstance(p, list) and bool(p) and all(isinstance(x, (str, list)) for x in p)
        if not batch:
            ids = p if isinstance(p, list) else tok.encode(p)
            return _generate(ids, req.max_tokens, req.kv_transfer_params, req.stream, req.model or model_name,
                             False, req)
        if req.stream or req.kv_transfer_params:
            raise HTTPException(status_code=400, detail="a batch of prompts is served without streaming or KV hand-off")
        # a batch: the prompts run concurrently; choice i*n + j is prompt i's j-th completion
        from concurrent.futures import ThreadPoolExecutor

        all_ids = [x if isinstance(x, list) else tok.encode(x) for x in p]
        with ThreadPoolExecutor(min(16, len(all_ids))) as ex:
            bodies = list(ex.map(lambda ids: _generate(ids, req.max_tokens, None, False, req.model or model_name,
                                                       False, req), all_ids))
        choices, usage = [], {"prompt_tokens": 0, "completion_tokens": 0, "total_tokens": 0}
        for body in bodies:
            for c in body["choices"]:
                choices.append(dict(c, index=len(choices)))
            for k in usage:
                usage[k] += body["usage"][k]
        ident = _new_id(False)
        return {"id": ident[0], "object": "text_completion", "created": ident[1], "model": req.model or model_name,
                "usage": usage, "choices": choices}

    @app.post("/v1/chat/completions")
    def chat_completions(req: ChatCompletionRequest):
        try:
            ids = tok.encode_chat([{"role": m.role, "content": m.text} for m in req.messages])
        except ValueError as exc:
            raise HTTPException(status_code=400, detail=str(exc)) from exc
        # no limit given: the rest of the context (the chat API has no default cap)
        max_tokens = req.max_completion_tokens or req.max_tokens or max(
            1, loop.engine.config.model_config.max_model_len - len(ids))
        return _generate(ids, max_tokens, req.kv_transfer_params, req.stream, req.model or model_name, True, req)

    return app


__all__ = ["EngineLoop", "build_app", "byte_detokenize", "byte_tokenize", "chat_prompt"]
