"""Weight-free custom-class proposer (suffix corpus + in-request n-gram).

Same positional contract as the reference's custom-class proposer
(reference: suffix_hybrid/hybrid_proposer.py:22-55):
``propose(sampled_token_ids, num_tokens_no_spec, token_ids_cpu, *,
slot_mappings=None)``.  The CPU rows already contain the sampled tokens; the
native Engine reads them in place.  Telemetry: a JSON stats line every
``SUFFIX_HYBRID_LOG_INTERVAL`` calls and, when ``SUFFIX_HYBRID_STATS_FILE``
is set, a JSONL record every ``SUFFIX_HYBRID_STATS_INTERVAL`` calls.
"""
import json
import logging
import os
import time

from vllm_suffix_hybrid_b200._native import VERSION, Engine

logger = logging.getLogger("suffix_hybrid")


class HybridProposer:
    def __init__(self, vllm_config=None):
        spec = getattr(vllm_config, "speculative_config", None)
        model = getattr(vllm_config, "model_config", None)
        self._engine = Engine(getattr(spec, "num_speculative_tokens", 8),
                              getattr(model, "max_model_len", 32768))
        self.suffix_cache = self._engine.suffix_cache
        self.num_speculative_tokens = self._engine.num_speculative_tokens
        self.use_ngram = self._engine.use_ngram
        self.stats_file = os.environ.get("SUFFIX_HYBRID_STATS_FILE", "").strip()
        logger.info("suffix_hybrid version=%s backend=native-cpp", VERSION)

    def propose(self, sampled_token_ids, num_tokens_no_spec, token_ids_cpu, *, slot_mappings=None):
        started = time.perf_counter_ns()
        drafts = self._engine.propose(sampled_token_ids, num_tokens_no_spec, token_ids_cpu)
        elapsed = time.perf_counter_ns() - started
        log_due, stats_due = self._engine.record_total(elapsed)
        if log_due or (stats_due and self.stats_file):
            stats = self.get_stats()
            stats["ts"] = time.time()
            line = json.dumps(stats, sort_keys=True)
            if log_due:
                logger.info("suffix_hybrid %s", line)
            if stats_due and self.stats_file:
                try:
                    with open(self.stats_file, "a", encoding="utf-8") as stream:
                        stream.write(line + "\n")
                except OSError:
                    logger.exception("suffix_hybrid cannot write telemetry")
            self._engine.record_total(time.perf_counter_ns() - started - elapsed)
        return drafts

    def get_stats(self):
        return self._engine.get_stats()
