"""Serving: an async front end over LLMEngine and an OpenAI-style HTTP server.

Entry point: ``python -m vllm_suffix_hybrid_b200.serve --model llama3-8b ...``
(one process per GPU under torchrun for TP > 1; rank 0 serves HTTP).
"""
from .async_engine import AsyncEngine, EngineOp
from .tokenizer import ByteTokenizer, load_tokenizer

__all__ = ["AsyncEngine", "EngineOp", "ByteTokenizer", "load_tokenizer"]
