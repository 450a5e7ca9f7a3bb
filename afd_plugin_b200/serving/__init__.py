"""HTTP serving front end (OpenAI-style completions) over the AFD engine."""

from afd_plugin_b200.serving.api_server import EngineLoop, build_app, byte_tokenize, byte_detokenize

__all__ = ["EngineLoop", "build_app", "byte_detokenize", "byte_tokenize"]
