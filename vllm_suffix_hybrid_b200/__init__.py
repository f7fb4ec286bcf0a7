"""B200-native hybrid speculative-decoding inference engine.

Layers (bottom up):

* ``_native``   -- C++ proposer core: suffix corpus, in-request n-gram,
  hybrid native/suffix mixer, suffix-only proposer, greedy verify oracle.
* ``_C``        -- sm_100a CUDA kernels (tcgen05/TMEM GEMMs, paged attention,
  fused norms, verify/commit, GDN, MoE, MLA, DSA) and the NVLink comm kernels.
* ``ops``       -- thin, loud Python wrappers around ``_C``.
* ``parallel``  -- process groups, symmetric memory, fused collectives, NCCL
  baseline paths.
* ``models``    -- Llama, Qwen3-Next hybrid MoE, DeepSeek-V3.2, Kimi-K2 and
  the toy config, plus EAGLE/MTP draft heads.
* ``engine``    -- config, weight loading, paged KV cache, scheduler, model
  runner, speculative-decoding loop.
* ``proposer``  -- Python surface of the proposer (HybridProposer ABI).
* ``serve``     -- OpenAI-style HTTP server, async engine front end, warm-start,
  SFT and decider routes.
* ``tune``      -- online MTP-head tuning and in-place SFT of the served model.
* ``bench``     -- microbenchmarks of the kernels, comm paths and proposer.
"""

__version__ = "0.3.0"
