"""Typed configuration for models, engine and kernels, with environment overrides.

The reference configures everything through one environment flag per feature
(flashnext/kaggle/README.md:279; dotsnote/engine/arcstats_pkg/arcstats/__init__.py:294-380) plus mode JSON files.
Here every knob lives in a dataclass; ``FW_<FIELD>`` environment variables override fields at construction
(:func:`apply_env`), so a flag-for-flag mapping of the reference's switches is still possible.

Model shapes
------------
``fn_config()`` is the Flash-Next-shaped MoE (Qwen3.8-Flash-Next as served by the reference's `fnext` overlay).
The reference tree does not contain that model's config.json; its dims are taken from what the tree does fix:

* hidden 2560, expert FFN 640, 512 experts of which 320 kept, top-10 softmax routing, 48 layers + 1 MTP layer,
  12 sparse-attention layers (flashnext/kaggle/README.md:30,175; k2_l4cfg.json marlin shapes 1280x2560 / 2560x640);
* Gated-DeltaNet projections 2560 -> 8192 and 3072 -> 2560 per TP2 rank in k2_l4cfg.json, i.e. 16 key heads and
  48 value heads of dim 128 (qkv 10240 + z 6144 = 16384 = 2 x 8192; value width 6144 = 2 x 3072);
* hyper-connection width 10240 = 4 x 2560 (k2_l4cfg.json "10240x336"), mixing rank 336;
* attention: 16 query heads, 2 KV heads, head_dim 256, partial rotary 0.25, sigmoid output gate; block indexer
  of 20 heads x 128 with compress ratio 4 and a 2048-token budget (2560 -> 7296 per TP2 rank in k2_l4cfg.json =
  4096 q+gate + 512 kv + 2688 indexer);
* PLE n-gram embedding: 3-grams, 8 heads per n-gram order, 160-wide fp8 rows (320M x 160, README.md:314).

``d3_config()`` is the Dots3-Note-shaped MoE (dotsnote/training/README.md:192-243; student.py:177-340):
hidden 5120, 256 experts (144 kept), expert FFN 1536, top-8 sigmoid routing with correction bias, MLA with a
DSA indexer (latent 512 + rope 64, top-2048) on 13 layers and sliding-window MLA (latent 1024 + rope 64,
window 513) on the rest, vocab 152064.

``tiny_config()`` is the CPU-checkable hybrid of BASELINE config 1.
"""
from __future__ import annotations

import dataclasses
import os
from dataclasses import dataclass, field


def _coerce(v: str, like):
    if isinstance(like, bool):
        return v.lower() in ("1", "true", "yes", "on")
    if isinstance(like, int):
        return int(v)
    if isinstance(like, float):
        return float(v)
    if isinstance(like, (list, tuple)):
        return type(like)(int(x) for x in v.split(",") if x)
    return v


def apply_env(obj, prefix: str = "FW_"):
    """Override dataclass fields from ``<prefix><FIELD>`` environment variables (in place; returns obj)."""
    for f in dataclasses.fields(obj):
        key = prefix + f.name.upper()
        if key in os.environ:
            setattr(obj, f.name, _coerce(os.environ[key], getattr(obj, f.name)))
    return obj


@dataclass
class FNConfig:
    """Flash-Next-shaped hybrid (Gated DeltaNet + block-sparse attention) MoE with hyper-connections."""
    name: str = "flashnext-shaped"
    vocab_size: int = 151936
    hidden_size: int = 2560
    num_layers: int = 48
    full_attn_interval: int = 4          # every 4th layer is sparse full attention (12 of 48)
    hc_count: int = 4
    hc_rank: int = 336
    rms_eps: float = 1e-6
    # Gated DeltaNet
    lin_k_heads: int = 16
    lin_v_heads: int = 48
    lin_k_dim: int = 128
    lin_v_dim: int = 128
    conv_kernel: int = 4
    gdn_gate: str = "silu"               # output gate of the gated RMSNorm (silu, or sigmoid)
    # attention
    n_heads: int = 16
    n_kv_heads: int = 2
    head_dim: int = 256
    partial_rotary: float = 0.25
    rope_theta: float = 10_000_000.0
    indexer_heads: int = 20
    indexer_dim: int = 128
    indexer_ratio: int = 4
    indexer_budget: int = 2048
    # MoE
    n_experts_orig: int = 512
    n_experts: int = 320
    top_k: int = 10
    moe_inter: int = 640
    shared_inter: int = 640
    expert_bits: tuple = (4, 3)          # bit widths, split evenly over the kept experts
    # PLE n-gram embedding
    ple_layers: tuple = (0,)             # layers with a PLE block (all share one n-gram table)
    ple_conv: int = 4
    ngram_size: int = 3
    heads_per_ngram: int = 8
    ple_dim: int = 160
    ple_rows: int = 320_000_000
    eos_token_id: int = 151645
    # draft (MTP) layer
    mtp_layers: int = 1
    dense_fp8: bool = True               # non-expert weights FP8 block-scaled 128x128

    def layer_kind(self, l: int) -> str:
        return "attention" if (l + 1) % self.full_attn_interval == 0 else "linear"

    @property
    def rope_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary)

    @property
    def indexer_blocks(self) -> int:
        return self.indexer_budget // self.indexer_ratio

    def bits_of(self, e: int) -> int:
        nb = len(self.expert_bits)
        return self.expert_bits[min(nb - 1, e * nb // self.n_experts)]


@dataclass
class D3Config:
    """Dots3-Note-shaped MLA MoE with DSA (indexed sparse) and SWA layers."""
    name: str = "dots3-shaped"
    vocab_size: int = 152064
    hidden_size: int = 5120
    num_layers: int = 46                 # layer 0 dense, 1..45 MoE
    n_dense_layers: int = 1
    dense_inter: int = 12288
    rms_eps: float = 1e-6
    n_heads: int = 128
    q_lora_rank: int = 1536
    kv_lora_rank: int = 512              # DSA layers latent
    swa_kv_lora_rank: int = 1024         # SWA layers latent
    qk_nope_dim: int = 128
    qk_rope_dim: int = 64
    v_head_dim: int = 128
    swa_window: int = 513
    swa_n_heads: int = 64                # SWA layers have their own head count (16 per TP4 rank)
    swa_rope_theta: float = 10000.0
    kv_rescale: bool = True              # MLA q/kv LoRA rescale sqrt(hidden / rank)
    dense_fp8: bool = True               # dense weights block-FP8 128x128
    eos_token_id: int = 1
    dsa_pattern: str = "FFSFSFSFSFFSF"   # index-share pattern over the DSA layers (used when index_share is on)
    index_share: bool = False            # DSA layers marked 'S' reuse the top-k of the latest 'F' layer
    shard_index: bool = False            # under TP: rank r keeps the index keys of positions = r (mod TP size)
    dsa_every: int = 0                   # 0: DSA layers spread evenly (13 of 46)
    n_dsa_layers: int = 13
    index_heads: int = 64
    index_dim: int = 128
    index_topk: int = 2048
    rope_theta: float = 10000.0
    n_experts_orig: int = 256
    n_experts: int = 144
    top_k: int = 8
    moe_inter: int = 1536
    shared_inter: int = 1536
    expert_bits: tuple = (3, 2)
    route_scale: float = 2.5
    mtp_layers: int = 1

    def heads_of(self, l: int) -> int:
        return self.n_heads if self.layer_kind(l) == "dsa" else self.swa_n_heads

    def latent_of(self, l: int) -> int:
        return self.kv_lora_rank if self.layer_kind(l) == "dsa" else self.swa_kv_lora_rank

    def is_moe(self, l: int) -> bool:
        return l >= self.n_dense_layers

    def layer_kind(self, l: int) -> str:
        step = self.num_layers / self.n_dsa_layers
        dsa = {int(i * step) for i in range(self.n_dsa_layers)}
        return "dsa" if l in dsa else "swa"

    def dsa_layers(self) -> list:
        return [l for l in range(self.num_layers) if self.layer_kind(l) == "dsa"]

    def shared_index_layers(self) -> set:
        """DSA layers that skip their own indexer and reuse the top-k of the most recent indexing ('F') layer
        (the reference's index_share.py: one 'F'/'S' character per DSA layer in model order, the first 'F')."""
        if not self.index_share:
            return set()
        dsa = self.dsa_layers()
        p = self.dsa_pattern.strip().upper()
        if len(p) != len(dsa) or set(p) - {"F", "S"} or p[0] != "F":
            raise ValueError(f"dsa_pattern {self.dsa_pattern!r}: need {len(dsa)} characters of F/S starting with F")
        return {l for l, c in zip(dsa, p) if c == "S"}

    def bits_of(self, e: int) -> int:
        # 96 experts at 3-bit and 48 at 2-bit in the shipped build
        return self.expert_bits[0] if e < (2 * self.n_experts) // 3 else self.expert_bits[1]


def fn_config(**kw) -> FNConfig:
    return apply_env(FNConfig(**kw), "FW_FN_")


def d3_config(**kw) -> D3Config:
    return apply_env(D3Config(**kw), "FW_D3_")


def d3_small_config(**kw) -> D3Config:
    """A small D3-shaped model for tests: both attention kinds, dense + MoE layers, tiny dims."""
    base = dict(name="d3-small", vocab_size=4096, hidden_size=256, num_layers=4, n_dense_layers=1, dense_inter=256,
                n_heads=4, swa_n_heads=2, q_lora_rank=128, kv_lora_rank=128, swa_kv_lora_rank=256, qk_nope_dim=32,
                qk_rope_dim=64, v_head_dim=64, swa_window=9, n_dsa_layers=2, index_heads=2, index_dim=128,
                index_topk=16, n_experts_orig=16, n_experts=8, top_k=2, moe_inter=128, shared_inter=128,
                expert_bits=(3, 2), route_scale=2.5)
    base.update(kw)
    return D3Config(**base)


def tiny_config(**kw) -> FNConfig:
    """4 layers, hidden 512, 8x64 attention, alternating GDN / full attention, 32 experts
    top-4 with FFN 256, 4-bit symmetric g128 experts, vocab 32000."""
    base = dict(name="tiny-hybrid", vocab_size=32000, hidden_size=512, num_layers=4, full_attn_interval=2,
                hc_count=2, hc_rank=32, lin_k_heads=4, lin_v_heads=8, lin_k_dim=64, lin_v_dim=64,
                n_heads=8, n_kv_heads=2, head_dim=64, partial_rotary=0.5, rope_theta=10000.0,
                indexer_heads=4, indexer_dim=64, indexer_ratio=4, indexer_budget=1 << 30,
                n_experts_orig=32, n_experts=32, top_k=4, moe_inter=256, shared_inter=256, expert_bits=(4,),
                ple_layers=(), mtp_layers=1, dense_fp8=False, eos_token_id=2, ple_rows=4096, ple_dim=32,
                heads_per_ngram=2)
    base.update(kw)
    return FNConfig(**base)


def fn_small_config(**kw) -> FNConfig:
    """A small FN-shaped model for GPU tests: every feature on, tiny dims."""
    base = dict(name="fn-small", vocab_size=4096, hidden_size=256, num_layers=4, full_attn_interval=2,
                hc_count=2, hc_rank=64, lin_k_heads=2, lin_v_heads=4, lin_k_dim=128, lin_v_dim=128,
                n_heads=4, n_kv_heads=2, head_dim=128, partial_rotary=0.5, indexer_heads=2, indexer_dim=128,
                indexer_ratio=4, indexer_budget=64, n_experts_orig=16, n_experts=8, top_k=2, moe_inter=128,
                shared_inter=128, expert_bits=(4, 3), ple_layers=(0,), ple_rows=4096, ple_dim=64,
                heads_per_ngram=2, eos_token_id=1)
    base.update(kw)
    return FNConfig(**base)


@dataclass
class EngineConfig:
    """Serving-engine knobs (the reference's vLLM args + FN_*/ARC_* flags)."""
    max_seqs: int = 64
    max_model_len: int = 20480
    block_size: int = 64                 # tokens per paged-KV block
    kv_blocks: int = 0                   # paged-KV blocks in the pool (0: every slot can reach max_model_len)
    kv_dtype: str = "fp8"                # fp8 (e4m3) or bf16 attention KV
    state_dtype: str = "bf16"            # recurrent (GDN) state dtype
    cuda_graphs: bool = True
    graph_batch_sizes: tuple = (1, 2, 4, 8, 16, 32, 64, 128)
    spec_tokens: int = 0                 # MTP / n-gram draft length (0 = off)
    spec_method: str = "mtp"             # mtp | ngram
    tp: int = 1
    ep: int = 1
    comm: str = "fused"                  # fused (in-kernel NVLink) | nccl (baseline)
    seed: int = 0
    gpu_mem_fraction: float = 0.92
    session_ctx_guard: int = 0           # refuse session pushes that would exceed this many tokens (0 = off)

    @staticmethod
    def from_env(**kw) -> "EngineConfig":
        return apply_env(EngineConfig(**kw), "FW_")


@dataclass
class TrainConfig:
    """Repair-training knobs (flashnext/training/rl/train_rl.py:44-70)."""
    trainable: tuple = ("scales", "router")
    lr_scales: float = 3e-4
    lr_router: float = 1.5e-5
    lr_norms: float = 1e-5
    warmup: int = 3
    clip_adv: float = 2.0
    ppo_clip: float = 0.0
    kl_anchor: float = 0.0
    tok_norm: float = 16384.0
    chunk: int = 1024
    rollouts: int = 8
    grad_bucket_mb: int = 64
    save_every: int = 5
    seed: int = 0
    extra: dict = field(default_factory=dict)
