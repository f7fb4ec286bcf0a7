"""vLLM custom-class drafter backed by the native weight-free Engine.

The class keeps the reference's constructor and call signature, so a vLLM
speculative config that names it as ``custom_class`` works unchanged
(reference: suffix_hybrid/hybrid_proposer.py:22-55):

    HybridProposer(vllm_config)
    propose(sampled_token_ids, num_tokens_no_spec, token_ids_cpu, *, slot_mappings=None)
        -> list[list[int]]       one draft (possibly empty) per batch row

Everything behind the signature is this package's own: the C++ ``Engine``
(row identity, suffix corpus, in-request n-gram index) does the work, and
``engine.telemetry.CallTelemetry`` owns the stats-line / JSONL cadence.
``token_ids_cpu`` rows already hold the sampled tokens; ``sampled_token_ids``
is only read for which rows sampled anything this step.  ``slot_mappings``
is accepted for interface compatibility and unused (the proposer is host
only).
"""
from __future__ import annotations

import logging
import time

from vllm_suffix_hybrid_b200._native import VERSION, Engine
from vllm_suffix_hybrid_b200.engine.telemetry import CallTelemetry

logger = logging.getLogger("suffix_hybrid")

_DEFAULT_K = 8
_DEFAULT_MAX_LEN = 32768


def _shape_from_config(vllm_config):
    """(draft length k, max context length) from a vLLM-style config object, with defaults."""
    spec = getattr(vllm_config, "speculative_config", None)
    model = getattr(vllm_config, "model_config", None)
    k = getattr(spec, "num_speculative_tokens", None)
    max_len = getattr(model, "max_model_len", None)
    k = _DEFAULT_K if k is None else k
    max_len = _DEFAULT_MAX_LEN if max_len is None else max_len
    return int(k), int(max_len)


class HybridProposer:
    def __init__(self, vllm_config=None):
        k, max_len = _shape_from_config(vllm_config)
        self._engine = Engine(k, max_len)
        self._telemetry = CallTelemetry.from_env(self._engine.get_stats, self._engine.record_total)
        logger.info("suffix_hybrid %s: native C++ proposer, k=%d, max_model_len=%d", VERSION,
                    self._engine.num_speculative_tokens, max_len)

    # Attributes a vLLM drafter wrapper reads.
    @property
    def suffix_cache(self):
        return self._engine.suffix_cache

    @property
    def num_speculative_tokens(self) -> int:
        return self._engine.num_speculative_tokens

    @property
    def use_ngram(self) -> bool:
        return self._engine.use_ngram

    @property
    def stats_file(self) -> str:
        return self._telemetry.stats_file

    def propose(self, sampled_token_ids, num_tokens_no_spec, token_ids_cpu, *, slot_mappings=None):
        t0 = time.perf_counter_ns()
        drafts = self._engine.propose(sampled_token_ids, num_tokens_no_spec, token_ids_cpu)
        self._telemetry.after_call(time.perf_counter_ns() - t0)
        return drafts

    def get_stats(self) -> dict:
        return self._engine.get_stats()
