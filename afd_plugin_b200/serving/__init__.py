"""HTTP serving front end (OpenAI-style completions) over the AFD engine."""

from afd_plugin_b200.serving.api_server import EngineLoop, build_app, byte_detokenize, byte_tokenize
from afd_plugin_b200.serving.tokenizer import ByteTokenizer, HFTokenizer, load_tokenizer

__all__ = ["ByteTokenizer", "EngineLoop", "HFTokenizer", "build_app", "byte_detokenize", "byte_tokenize",
           "load_tokenizer"]
