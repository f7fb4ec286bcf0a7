"""Drop-in import alias for code written against the reference's package.

``from suffix_hybrid._native import Engine`` (and the other proposer classes)
and ``suffix_hybrid.hybrid_proposer.HybridProposer`` resolve to this
framework's native implementation; no Python algorithm lives here.
"""
__version__ = "0.3.0"
