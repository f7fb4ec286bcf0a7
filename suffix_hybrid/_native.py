"""Alias of :mod:`vllm_suffix_hybrid_b200._native` under the reference's name."""
from vllm_suffix_hybrid_b200._native import *  # noqa: F401,F403
from vllm_suffix_hybrid_b200._native import (  # noqa: F401
    VERSION,
    Engine,
    HybridMixer,
    SuffixCache,
    V2SuffixProposer,
    rejection_greedy_accept,
)
