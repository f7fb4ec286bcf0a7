"""Proposer surface: native classes plus the custom-class HybridProposer."""
from vllm_suffix_hybrid_b200._native import (  # noqa: F401
    VERSION,
    Engine,
    HybridMixer,
    SuffixCache,
    V2SuffixProposer,
    rejection_greedy_accept,
)
from vllm_suffix_hybrid_b200.proposer.hybrid_proposer import HybridProposer  # noqa: F401

__all__ = [
    "VERSION",
    "Engine",
    "HybridMixer",
    "HybridProposer",
    "SuffixCache",
    "V2SuffixProposer",
    "rejection_greedy_accept",
]
