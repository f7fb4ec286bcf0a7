"""Typed engine configuration with SUFFIX_HYBRID_* environment overlay.

Model presets cover the five benchmark configurations: the CPU toy decoder
(config 0), Llama-3-8B (config 1), the Qwen3-Next hybrid GDN/attention MoE
(config 2), DeepSeek-V3.2 sparse-MLA MoE (config 3) and the Kimi-K2 long
context stress (config 4).  The proposer knobs keep the reference's names
and defaults (reference: src/lib.rs:115-124, src/engine.rs:217-241,
suffix_hybrid/wrap_v2.py:442-449).
"""
from __future__ import annotations

import dataclasses
import os
from dataclasses import dataclass, field
from typing import Optional


@dataclass
class ModelConfig:
    arch: str = "llama"  # llama | qwen3_next | deepseek_v32 | kimi_k2
    hidden: int = 4096
    layers: int = 32
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 14336
    vocab: int = 128256
    rope_theta: float = 500000.0
    rope_scaling: Optional[dict] = None  # HF rope_scaling / rope_parameters (llama3, yarn)
    norm_eps: float = 1e-5
    norm_offset: float = 0.0  # checkpoint RMSNorm gains are stored as (gain - offset), e.g. 1 for Qwen3-Next
    max_position: int = 131072
    tie_embeddings: bool = False
    dtype: str = "bfloat16"
    init_std: float = 0.02
    # --- MoE ---
    num_experts: int = 0
    top_k: int = 0
    expert_ffn: int = 0
    shared_experts: int = 0
    shared_ffn: int = 0
    router: str = "softmax"  # softmax | sigmoid_grouped
    n_groups: int = 1
    topk_groups: int = 1
    routed_scale: float = 1.0
    first_dense_layers: int = 0
    # --- hybrid GDN (Qwen3-Next) ---
    layer_pattern: str = ""  # e.g. "LLLA" repeated: L = linear (GDN), A = full attention
    gdn_qk_heads: int = 0
    gdn_v_heads: int = 0
    gdn_head_dim: int = 128
    gdn_conv: int = 4
    gdn_chunk: int = 64
    attn_gated: bool = False
    partial_rotary: float = 1.0
    # --- MLA / DSA (DeepSeek-V3.2, Kimi-K2) ---
    q_lora: int = 0
    kv_lora: int = 0
    qk_nope: int = 0
    qk_rope: int = 0
    v_head: int = 0
    dsa_heads: int = 0
    dsa_head_dim: int = 128
    dsa_topk: int = 0
    # --- quantisation ---
    weight_format: str = "bf16"  # bf16 | fp8_block | nvfp4
    kv_format: str = "bf16"  # bf16 | fp8 | nvfp4
    # --- draft head ---
    draft: str = "eagle"  # eagle | mtp | none
    draft_layers: int = 1

    @property
    def q_size(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.kv_heads * self.head_dim

    def layer_kind(self, i: int) -> str:
        """'A' full attention, 'L' linear attention (GDN), 'M' MLA."""
        if self.arch in ("deepseek_v32", "kimi_k2"):
            return "M"
        if self.layer_pattern:
            return self.layer_pattern[i % len(self.layer_pattern)]
        return "A"

    def layer_is_moe(self, i: int) -> bool:
        return self.num_experts > 0 and i >= self.first_dense_layers


def toy_config() -> ModelConfig:
    """Config 0: 2-layer, 256-dim, 4-head fp32 decoder, vocab 32000, 1-layer MTP head."""
    return ModelConfig(arch="llama", hidden=256, layers=2, heads=4, kv_heads=4, head_dim=64, ffn=1024,
                       vocab=32000, rope_theta=10000.0, dtype="float32", draft="mtp", max_position=16384)


def llama3_8b_config() -> ModelConfig:
    """Config 1: Llama-3-8B shape with a 1-layer EAGLE head of the same width."""
    return ModelConfig(arch="llama", hidden=4096, layers=32, heads=32, kv_heads=8, head_dim=128, ffn=14336,
                       vocab=128256, rope_theta=500000.0, dtype="bfloat16", draft="eagle")


def qwen3_next_config() -> ModelConfig:
    """Config 2: 48 layers, 3 GDN : 1 gated attention, 512 experts top-10 + shared."""
    return ModelConfig(arch="qwen3_next", hidden=2048, layers=48, heads=16, kv_heads=2, head_dim=256,
                       ffn=512, vocab=151936, rope_theta=10000000.0, norm_eps=1e-6, num_experts=512, top_k=10,
                       expert_ffn=512, shared_experts=1, shared_ffn=512, router="softmax", layer_pattern="LLLA",
                       gdn_qk_heads=16, gdn_v_heads=32, gdn_head_dim=128, gdn_conv=4, gdn_chunk=64,
                       attn_gated=True, partial_rotary=0.25, dtype="bfloat16", draft="mtp")


def deepseek_v32_config() -> ModelConfig:
    """Config 3: 61 layers (3 dense), MLA, DSA top-2048, 256 experts top-8, NVFP4."""
    return ModelConfig(arch="deepseek_v32", hidden=7168, layers=61, heads=128, kv_heads=1, head_dim=192,
                       ffn=18432, vocab=129280, rope_theta=10000.0, norm_eps=1e-6, num_experts=256, top_k=8,
                       expert_ffn=2048, shared_experts=1, shared_ffn=2048, router="sigmoid_grouped", n_groups=8,
                       topk_groups=4, routed_scale=2.5, first_dense_layers=3, q_lora=1536, kv_lora=512,
                       qk_nope=128, qk_rope=64, v_head=128, dsa_heads=64, dsa_head_dim=128, dsa_topk=2048,
                       weight_format="nvfp4", kv_format="nvfp4", dtype="bfloat16", draft="mtp")


def kimi_k2_config() -> ModelConfig:
    """Config 4: 61 layers, 64-head MLA, 384 experts top-8 + shared, NVFP4 weights and KV."""
    return ModelConfig(arch="kimi_k2", hidden=7168, layers=61, heads=64, kv_heads=1, head_dim=192, ffn=18432,
                       vocab=163840, rope_theta=50000.0, norm_eps=1e-6, num_experts=384, top_k=8, expert_ffn=2048,
                       shared_experts=1, shared_ffn=2048, router="sigmoid_grouped", n_groups=1, topk_groups=1,
                       routed_scale=2.827, first_dense_layers=1, q_lora=1536, kv_lora=512, qk_nope=128,
                       qk_rope=64, v_head=128, dsa_heads=0, dsa_topk=0, weight_format="nvfp4", kv_format="nvfp4",
                       dtype="bfloat16", draft="mtp")


PRESETS = {
    "toy": toy_config,
    "llama3-8b": llama3_8b_config,
    "qwen3-next": qwen3_next_config,
    "deepseek-v3.2": deepseek_v32_config,
    "kimi-k2": kimi_k2_config,
}


def shrink(cfg: ModelConfig, layers: int = 2, hidden: int = 256, vocab: int = 1024) -> ModelConfig:
    """Same architecture at test size (keeps every structural feature on)."""
    c = dataclasses.replace(cfg)
    scale = hidden / cfg.hidden
    c.hidden = hidden
    c.layers = layers
    c.vocab = vocab
    c.ffn = max(64, int(cfg.ffn * scale) // 64 * 64)
    if cfg.arch == "llama":
        c.heads, c.kv_heads, c.head_dim = 4, 2, 64
    if cfg.num_experts:
        c.num_experts = min(cfg.num_experts, 16)
        c.top_k = min(cfg.top_k, 4)
        c.expert_ffn = 64
        c.shared_ffn = 64
        c.n_groups = min(cfg.n_groups, 4)
        c.topk_groups = min(cfg.topk_groups, 2)
        c.first_dense_layers = min(cfg.first_dense_layers, 1)
    if cfg.arch == "qwen3_next":
        c.heads, c.kv_heads, c.head_dim = 4, 2, 64
        c.gdn_qk_heads, c.gdn_v_heads, c.gdn_head_dim = 2, 4, 32
        c.gdn_chunk = 16
        c.layers = max(layers, 4)
    if cfg.arch in ("deepseek_v32", "kimi_k2"):
        c.heads = 4
        # kernel-supported test geometry: latent 64 + rope 64 (C = 128), indexer 16 heads x 128
        c.q_lora, c.kv_lora, c.qk_nope, c.qk_rope, c.v_head = 64, 64, 32, 64, 32
        c.head_dim = c.qk_nope + c.qk_rope
        if cfg.dsa_heads:
            c.dsa_heads, c.dsa_head_dim, c.dsa_topk = 16, 128, 32
    c.max_position = 8192
    return c


@dataclass
class SpecConfig:
    method: str = "hybrid"  # hybrid | native | suffix | ngram | none
    k: int = 5
    split: str = "legacy"  # legacy | diverge (SUFFIX_HYBRID_SPLIT)
    uniform_k: bool = True  # suffix-only: publish width k for every row (static verify shape)
    width_gate: bool = False  # SUFFIX_HYBRID_EWMA_WIDTH
    min_len: int = 1  # SUFFIX_HYBRID_SUFFIX_MIN
    async_scheduling: bool = False  # SUFFIX_HYBRID_ASYNC: lag-1 host candidates, drafts resolved on the device
    async_hyb_min: int = 0  # SUFFIX_HYBRID_ASYNC_HYB_MIN (0 = k): real suffix drafts that replace native ones
    # Verify only as wide as the longest real draft of the step (SUFFIX_HYBRID_ADAPTIVE_WIDTH=0 / 1 overrides).
    adaptive_width: bool = True


@dataclass
class ParallelConfig:
    tp: int = 1
    ep: int = 1
    dp: int = 1
    comm: str = "fused"  # fused (own NVLink kernels) | nccl (baseline)


@dataclass
class CacheConfig:
    block_size: int = 64
    num_blocks: int = 0  # 0: size from free memory
    gpu_memory_fraction: float = 0.85
    max_model_len: int = 4096
    # host KV tier (DSA sparse-attention models on CUDA): latent rows in mapped host memory, hot rows on the
    # device (engine/host_tier.py); hot_rows 0 = (k + 2) x top-k; host_kv_gb caps the host pool
    host_kv: bool = False
    host_kv_hot_rows: int = 0
    host_kv_gb: float = 64.0


@dataclass
class EngineConfig:
    model: ModelConfig = field(default_factory=llama3_8b_config)
    spec: SpecConfig = field(default_factory=SpecConfig)
    parallel: ParallelConfig = field(default_factory=ParallelConfig)
    cache: CacheConfig = field(default_factory=CacheConfig)
    max_num_seqs: int = 64
    max_prefill_tokens: int = 16384
    # a prompt longer than max_prefill_tokens is prefilled in chunks of that size, alternating with decode
    # steps of the running requests (attention-only models; recurrent-state models prefill it whole)
    chunked_prefill: bool = True
    device: str = "cuda"
    seed: int = 0
    cuda_graphs: bool = True
    weights: Optional[str] = None  # safetensors directory; None = random init


def _env(name: str) -> Optional[str]:
    v = os.environ.get("SUFFIX_HYBRID_" + name)
    return v.strip() if v is not None and v.strip() != "" else None


def apply_env(cfg: EngineConfig) -> EngineConfig:
    """Overlay the SUFFIX_HYBRID_* serving knobs onto a config."""
    if _env("SPLIT") == "diverge":
        cfg.spec.split = "diverge"
    if _env("SUFFIX_ONLY") == "1":
        cfg.spec.method = "suffix"
    if _env("UNIFORM_K") is not None:
        cfg.spec.uniform_k = _env("UNIFORM_K") == "1"
    if _env("ADAPTIVE_WIDTH") in ("0", "1"):
        cfg.spec.adaptive_width = _env("ADAPTIVE_WIDTH") == "1"
    if _env("EWMA_WIDTH") == "1":
        cfg.spec.width_gate = True
    v = _env("SUFFIX_MIN")
    if v is not None and v.isdigit():
        cfg.spec.min_len = max(1, int(v))
    if _env("ASYNC") == "1":
        cfg.spec.async_scheduling = True
    v = _env("ASYNC_HYB_MIN")
    if v is not None and v.isdigit():
        cfg.spec.async_hyb_min = int(v)
    v = _env("MAX_SPEC_TOKENS")
    if v is not None and v.isdigit() and int(v) > 0:
        cfg.spec.k = int(v)
    if _env("CHUNKED_PREFILL") in ("0", "1"):
        cfg.chunked_prefill = _env("CHUNKED_PREFILL") == "1"
    if _env("HOST_KV") == "1":
        cfg.cache.host_kv = True
    v = _env("HOST_KV_HOT_ROWS")
    if v is not None and v.isdigit():
        cfg.cache.host_kv_hot_rows = int(v)
    return cfg
