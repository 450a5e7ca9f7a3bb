"""Text <-> token ids for the completions server.

``HFTokenizer`` loads a Hugging Face tokenizer from a local directory (the
checkpoint's ``tokenizer.json`` / ``tokenizer_config.json``, no network) and
renders chat requests with the tokenizer's chat template when it has one.
``ByteTokenizer`` is the fallback when no tokenizer is at hand (random-init
benchmark models): UTF-8 bytes modulo the vocabulary.

Streaming needs text per token; ``StreamDetokenizer`` decodes the whole
sequence so far and emits the new suffix, holding back a trailing partial
UTF-8 character until the tokens that complete it arrive.
"""

from __future__ import annotations

import os
from typing import Protocol


class Tokenizer(Protocol):
    def encode(self, text: str) -> list[int]: ...

    def decode(self, ids: list[int]) -> str: ...

    def encode_chat(self, messages: list[dict]) -> list[int]: ...


def render_chat(messages: list[dict]) -> str:
    """Role-tagged transcript ending in the assistant tag (used without a chat template)."""
    return "".join(f"<|{m['role']}|>{m['content']}\n" for m in messages) + "<|assistant|>"


class ByteTokenizer:
    def __init__(self, vocab_size: int):
        self.vocab_size = vocab_size

    def encode(self, text: str) -> list[int]:
        return [b % self.vocab_size for b in text.encode("utf-8")] or [0]

    def decode(self, ids: list[int]) -> str:
        return bytes(i % 256 for i in ids).decode("utf-8", errors="replace")

    def encode_chat(self, messages: list[dict]) -> list[int]:
        return self.encode(render_chat(messages))


class HFTokenizer:
    def __init__(self, path: str):
        from transformers import AutoTokenizer

        if not os.path.isdir(path):
            raise FileNotFoundError(f"tokenizer directory {path!r} does not exist")
        self.tok = AutoTokenizer.from_pretrained(path, local_files_only=True)

    def encode(self, text: str) -> list[int]:
        return list(self.tok.encode(text, add_special_tokens=True)) or [0]

    def decode(self, ids: list[int]) -> str:
        return self.tok.decode(ids, skip_special_tokens=True)

    def encode_chat(self, messages: list[dict]) -> list[int]:
        if getattr(self.tok, "chat_template", None):
            out = self.tok.apply_chat_template(messages, tokenize=True, add_generation_prompt=True)
            if isinstance(out, dict) or hasattr(out, "input_ids"):
                out = out["input_ids"]
            return list(out)
        return self.encode(render_chat(messages))


def load_tokenizer(path: str | None, vocab_size: int) -> Tokenizer:
    """The HF tokenizer at ``path`` if it has one, else the byte fallback."""
    if path and any(os.path.exists(os.path.join(path, f)) for f in ("tokenizer.json", "tokenizer_config.json",
                                                                     "tokenizer.model")):
        return HFTokenizer(path)
    return ByteTokenizer(vocab_size)


class StreamDetokenizer:
    """Incremental text for a token stream: ``push(token) -> new text``."""

    def __init__(self, tokenizer: Tokenizer):
        self.tok = tokenizer
        self.ids: list[int] = []
        self.sent = ""

    def push(self, token: int) -> str:
        self.ids.append(int(token))
        text = self.tok.decode(self.ids)
        if text.endswith("\ufffd"):  # a multi-byte character still incomplete (or invalid)
            return ""
        return self._emit(text)

    def flush(self) -> str:
        """Whatever text was held back (the stream has ended)."""
        return self._emit(self.tok.decode(self.ids))

    def _emit(self, text: str) -> str:
        new = text[len(self.sent):] if text.startswith(self.sent) else text
        self.sent = text
        return new


__all__ = ["ByteTokenizer", "HFTokenizer", "StreamDetokenizer", "Tokenizer", "load_tokenizer", "render_chat"]
