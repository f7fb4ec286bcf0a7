"""Public compatibility import of the custom-class proposer."""
from vllm_suffix_hybrid_b200.proposer.hybrid_proposer import HybridProposer

__all__ = ["HybridProposer"]
