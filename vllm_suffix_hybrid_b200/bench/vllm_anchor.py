"""Same-box anchor: stock vLLM (the installed release, NOT the reference's pinned build) on config 1.

Runs the installed vLLM engine on the config-1 workload so the headline
number of this framework has a stock NCCL + cuBLAS / FlashInfer engine on
the same box next to it: Llama-3-8B shape with dummy (random) weights,
64 requests x 2048-token synthetic prompts (the same span-reuse streams as
bench.py), 512 greedy output tokens each (EOS ignored), k = 5 n-gram
speculation (vLLM's prompt-lookup drafter; EAGLE needs a trained head).
The prompt-only pass (max_tokens = 1) is timed separately, so the decode
throughput is (outputs - prompts' first tokens) / (full time - prefill time).

Run: python -m vllm_suffix_hybrid_b200.bench.vllm_anchor [--tp N] [--spec ngram|none]
This does not replace `bench.py --impl reference` (the reference arm).
"""
from __future__ import annotations

import argparse
import json
import os
import tempfile
import time


def llama3_8b_dir(max_len: int) -> str:
    d = tempfile.mkdtemp(prefix="llama3_8b_shape_")
    cfg = {
        "architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": 4096,
        "intermediate_size": 14336, "num_hidden_layers": 32, "num_attention_heads": 32,
        "num_key_value_heads": 8, "head_dim": 128, "vocab_size": 128256, "rope_theta": 500000.0,
        "max_position_embeddings": max(8192, max_len), "rms_norm_eps": 1e-5, "torch_dtype": "bfloat16",
        "hidden_act": "silu", "tie_word_embeddings": False, "bos_token_id": 128000, "eos_token_id": 128001,
    }
    with open(os.path.join(d, "config.json"), "w") as fh:
        json.dump(cfg, fh)
    return d


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--prompt-len", type=int, default=2048)
    ap.add_argument("--max-new", type=int, default=512)
    ap.add_argument("--k", type=int, default=5)
    ap.add_argument("--spec", default="ngram", choices=["ngram", "none"])
    a = ap.parse_args()

    from vllm import LLM, SamplingParams
    from vllm.inputs import TokensPrompt

    from vllm_suffix_hybrid_b200.bench.synthetic import make_streams

    max_len = a.prompt_len + a.max_new + 64
    spec = ({"method": "ngram", "num_speculative_tokens": a.k, "prompt_lookup_max": 4, "prompt_lookup_min": 2}
            if a.spec == "ngram" else None)
    llm = LLM(model=llama3_8b_dir(max_len), load_format="dummy", skip_tokenizer_init=True, dtype="bfloat16",
              tensor_parallel_size=a.tp, max_num_seqs=a.batch, max_model_len=max_len, gpu_memory_utilization=0.85,
              enable_prefix_caching=False, speculative_config=spec, seed=0)
    prompts = [TokensPrompt(prompt_token_ids=[int(t) for t in row])
               for row in make_streams(a.batch, a.prompt_len, 128256, seed=1234)]
    llm.generate(prompts[:2], SamplingParams(max_tokens=8, temperature=0.0, ignore_eos=True))  # warm-up
    t0 = time.perf_counter()
    llm.generate(prompts, SamplingParams(max_tokens=1, temperature=0.0, ignore_eos=True))
    t_prefill = time.perf_counter() - t0
    t0 = time.perf_counter()
    outs = llm.generate(prompts, SamplingParams(max_tokens=a.max_new, temperature=0.0, ignore_eos=True))
    t_full = time.perf_counter() - t0
    tokens = sum(len(o.outputs[0].token_ids) for o in outs)
    decode_tokens = tokens - len(outs)
    print(json.dumps({
        "anchor": f"stock vLLM {__import__('vllm').__version__} (installed release, not the reference build)",
        "model": "llama3-8b-shape (dummy weights)", "tp": a.tp, "batch": a.batch, "prompt_len": a.prompt_len,
        "max_new": a.max_new, "spec": a.spec, "k": a.k if spec else 0, "output_tokens": tokens,
        "e2e_s": round(t_full, 3), "prefill_s": round(t_prefill, 3),
        "e2e_tok_s": round(tokens / t_full, 1),
        "decode_tok_s": round(decode_tokens / max(t_full - t_prefill, 1e-9), 1),
    }))


if __name__ == "__main__":
    main()
