"""Serve a model over HTTP.

  python -m vllm_suffix_hybrid_b200.serve --model llama3-8b --port 8000
  torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m vllm_suffix_hybrid_b200.serve --model llama3-8b --tp 8

--model is a preset (toy, llama3-8b, qwen3-next, deepseek-v3.2, kimi-k2) or "auto" (config.json of --weights);
--weights loads a safetensors checkpoint directory into it (random init
otherwise); --tokenizer is a local Hugging Face tokenizer directory (byte
tokenizer otherwise).  Under torchrun rank 0 serves HTTP and the other ranks
follow its engine in lockstep.
"""
import argparse
import logging
import os


def main(argv=None):
    ap = argparse.ArgumentParser(prog="vllm_suffix_hybrid_b200.serve")
    ap.add_argument("--model", default="toy")
    ap.add_argument("--weights", default=None)
    ap.add_argument("--tokenizer", default=None)
    ap.add_argument("--served-model-name", default=None)
    ap.add_argument("--tp", type=int, default=int(os.environ.get("WORLD_SIZE", "1")))
    ap.add_argument("--method", default="hybrid", choices=["hybrid", "native", "suffix", "ngram", "none"])
    ap.add_argument("--k", type=int, default=5)
    ap.add_argument("--max-num-seqs", type=int, default=64)
    ap.add_argument("--max-model-len", type=int, default=8192)
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--no-graphs", action="store_true")
    ap.add_argument("--comm", default="fused", choices=["fused", "nccl"])
    ap.add_argument("--shrink", action="store_true", help="test-size model of the same architecture")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--async-scheduling", action="store_true", help="lag-1 drafting (SUFFIX_HYBRID_ASYNC=1)")
    import sys

    from . import dev_args

    argv = list(sys.argv[1:] if argv is None else argv)
    applied = dev_args.apply(argv)  # SUFFIX_HYBRID_DEV_ARGS=1: splice a reviewed flag delta
    a = ap.parse_args(argv)
    logging.basicConfig(level=logging.INFO)
    if applied:
        logging.getLogger(__name__).warning("dev args applied: %s -> argv %s", applied, argv)
    from ..utils.gpu_mon import GpuMonitor

    mon = GpuMonitor.from_env()  # SUFFIX_HYBRID_GPU_MON=<seconds>
    if mon is not None:
        mon.start()

    from ..engine.config import PRESETS, CacheConfig, EngineConfig, ParallelConfig, SpecConfig, shrink
    from ..engine.llm import LLMEngine
    from ..parallel import state
    from .api_server import build_app
    from .async_engine import AsyncEngine
    from .tokenizer import load_tokenizer

    st = state.init(tp=a.tp, backend=None if a.device == "cuda" else "gloo")
    if a.model == "auto":
        if not a.weights:
            raise SystemExit("--model auto needs --weights <checkpoint dir>")
        from ..engine.loader import config_from_hf

        mcfg = config_from_hf(a.weights)
    else:
        mcfg = PRESETS[a.model]()
    if a.shrink:
        mcfg = shrink(mcfg)
        if a.device != "cuda":
            mcfg.dtype = "float32"
    cfg = EngineConfig(model=mcfg, spec=SpecConfig(method=a.method, k=a.k, async_scheduling=a.async_scheduling),
                       parallel=ParallelConfig(tp=a.tp, comm=a.comm),
                       cache=CacheConfig(max_model_len=a.max_model_len), max_num_seqs=a.max_num_seqs, device=a.device,
                       cuda_graphs=(a.device == "cuda" and not a.no_graphs), weights=a.weights)
    engine = LLMEngine(cfg)
    aeng = AsyncEngine(engine, st.rank, st.world, st.cpu_group)
    if st.rank != 0:
        aeng.worker_loop()
        state.shutdown()
        return
    aeng.start()
    import uvicorn

    app = build_app(aeng, load_tokenizer(a.tokenizer), a.served_model_name or a.model)
    try:
        uvicorn.run(app, host=a.host, port=a.port, log_level="info")
    finally:
        aeng.shutdown()
        state.shutdown()


if __name__ == "__main__":
    main()
