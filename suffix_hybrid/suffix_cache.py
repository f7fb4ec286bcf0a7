"""Public compatibility import of the native corpus."""
from vllm_suffix_hybrid_b200._native import SuffixCache

__all__ = ["SuffixCache"]
