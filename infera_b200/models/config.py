"""Model architecture descriptions.

Presets follow the shapes named by the serving configurations: a
Llama-3.1-8B-shaped and a 70B-shaped dense GQA decoder, a Qwen3-32B-shaped
dense decoder (with per-head q/k RMSNorm) and a DeepSeek-V3-shaped MLA + MoE
decoder. Weights are random-initialised from a seed (no checkpoints are
loaded), so only the shapes matter for compute.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass, field


@dataclass
class DenseConfig:
    name: str = "llama-3.1-8b"
    num_layers: int = 32
    hidden: int = 4096
    num_heads: int = 32
    num_kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 14336
    vocab: int = 128256
    rope_theta: float = 500000.0
    rope_scaling: dict | None = field(default_factory=lambda: {
        "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
        "original_max_position_embeddings": 8192})
    rms_eps: float = 1e-5
    qk_norm: bool = False           # Qwen3: RMSNorm over each q / k head
    max_model_len: int = 32768 + 1024
    weight_dtype: str = "bf16"      # "bf16" or "fp8" (e4m3, 128x128 block scales)
    eos_token_id: int = 128001
    # mixture-of-experts FFN (0 experts: dense). Layers >= moe_first_layer
    # use routed experts (+ shared experts) instead of the dense MLP.
    num_experts: int = 0
    moe_top_k: int = 0
    moe_ffn: int = 0
    moe_first_layer: int = 0
    moe_n_groups: int = 1
    moe_topk_groups: int = 1
    moe_routed_scaling: float = 1.0
    moe_num_shared: int = 0
    moe_softmax: bool = False

    kv_channels: int = 2  # K and V caches

    def is_moe_layer(self, i: int) -> bool:
        return self.num_experts > 0 and i >= self.moe_first_layer

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    @property
    def qkv_size(self) -> int:
        return self.q_size + 2 * self.kv_size

    def params(self) -> int:
        per_layer = (self.hidden * self.qkv_size + self.q_size * self.hidden + 3 * self.hidden * self.ffn
                     + 2 * self.hidden)
        return self.num_layers * per_layer + 2 * self.vocab * self.hidden + self.hidden

    def kv_bytes_per_token(self, dtype_bytes: int = 2) -> int:
        return 2 * self.num_layers * self.kv_size * dtype_bytes

    def to_dict(self) -> dict:
        return asdict(self)


@dataclass
class MoEConfig:
    """DeepSeek-V3-shaped decoder: MLA attention and routed experts."""

    name: str = "deepseek-v3"
    num_layers: int = 61
    num_dense_layers: int = 3
    hidden: int = 7168
    dense_ffn: int = 18432
    num_heads: int = 128
    q_lora_rank: int = 1536
    kv_lora_rank: int = 512
    qk_rope_dim: int = 64
    qk_nope_dim: int = 128
    v_head_dim: int = 128
    num_experts: int = 256
    num_shared_experts: int = 1
    moe_ffn: int = 2048
    top_k: int = 8
    n_groups: int = 8
    topk_groups: int = 4
    routed_scaling: float = 2.5
    vocab: int = 129280
    rope_theta: float = 10000.0
    rms_eps: float = 1e-6
    max_model_len: int = 16384 + 1024
    weight_dtype: str = "fp8"
    eos_token_id: int = 1

    @property
    def latent_dim(self) -> int:
        return self.kv_lora_rank + self.qk_rope_dim  # 576 per token per layer

    # the paged cache holds one latent row per token (no separate V)
    kv_channels: int = 1

    @property
    def kv_size(self) -> int:
        return self.latent_dim

    @property
    def num_kv_heads(self) -> int:
        return 1

    @property
    def head_dim(self) -> int:
        return self.qk_nope_dim + self.qk_rope_dim

    # activation widths for memory sizing
    @property
    def q_size(self) -> int:
        return self.num_heads * self.latent_dim

    @property
    def qkv_size(self) -> int:
        return self.q_lora_rank + self.num_heads * self.head_dim + self.latent_dim

    @property
    def ffn(self) -> int:
        return max(self.dense_ffn, self.moe_ffn * max(1, self.num_shared_experts))

    def is_moe_layer(self, i: int) -> bool:
        return self.num_experts > 0 and i >= self.num_dense_layers

    def kv_bytes_per_token(self, dtype_bytes: int = 2) -> int:
        return self.num_layers * self.latent_dim * dtype_bytes

    def to_dict(self) -> dict:
        return asdict(self)


PRESETS: dict[str, DenseConfig | MoEConfig] = {
    "llama-3.1-8b": DenseConfig(),
    "llama-3.1-70b": DenseConfig(name="llama-3.1-70b", num_layers=80, hidden=8192, num_heads=64, num_kv_heads=8,
                                 ffn=28672, weight_dtype="fp8"),
    "qwen3-32b": DenseConfig(name="qwen3-32b", num_layers=64, hidden=5120, num_heads=64, num_kv_heads=8, ffn=25600,
                             vocab=151936, rope_theta=1000000.0, rope_scaling=None, rms_eps=1e-6, qk_norm=True,
                             max_model_len=65536 + 4096, eos_token_id=151645),
    "deepseek-v3": MoEConfig(),
    # GQA attention + routed experts (Qwen3-30B-A3B shape)
    "qwen3-30b-a3b": DenseConfig(name="qwen3-30b-a3b", num_layers=48, hidden=2048, num_heads=32, num_kv_heads=4,
                                 ffn=6144, vocab=151936, rope_theta=1000000.0, rope_scaling=None, rms_eps=1e-6,
                                 qk_norm=True, eos_token_id=151645, num_experts=128, moe_top_k=8, moe_ffn=768,
                                 moe_softmax=True),
    # small shapes for tests (same structure, tiny sizes)
    "tiny-dense": DenseConfig(name="tiny-dense", num_layers=2, hidden=256, num_heads=4, num_kv_heads=2, ffn=512,
                              vocab=1024, max_model_len=2048, eos_token_id=1),
    "tiny-dense-gpu": DenseConfig(name="tiny-dense-gpu", num_layers=2, hidden=1024, num_heads=8, num_kv_heads=2,
                                  ffn=2048, vocab=4096, max_model_len=4096, eos_token_id=1),
    "tiny-dense-fp8": DenseConfig(name="tiny-dense-fp8", num_layers=2, hidden=256, num_heads=4, num_kv_heads=2,
                                  ffn=512, vocab=1024, max_model_len=2048, eos_token_id=1, weight_dtype="fp8"),
    "tiny-dense-fp8-gpu": DenseConfig(name="tiny-dense-fp8-gpu", num_layers=2, hidden=1024, num_heads=8,
                                      num_kv_heads=2, ffn=2048, vocab=4096, max_model_len=4096, eos_token_id=1,
                                      weight_dtype="fp8"),
    "tiny-moe-gqa": DenseConfig(name="tiny-moe-gqa", num_layers=3, hidden=256, num_heads=4, num_kv_heads=2,
                                ffn=512, vocab=1024, max_model_len=2048, eos_token_id=1, num_experts=8, moe_top_k=2,
                                moe_ffn=128, moe_first_layer=1, moe_n_groups=2, moe_topk_groups=1,
                                moe_routed_scaling=1.5, moe_num_shared=1),
    "tiny-moe-gqa-gpu": DenseConfig(name="tiny-moe-gqa-gpu", num_layers=3, hidden=1024, num_heads=8, num_kv_heads=2,
                                    ffn=2048, vocab=4096, max_model_len=4096, eos_token_id=1, num_experts=16,
                                    moe_top_k=4, moe_ffn=512, moe_first_layer=1, moe_n_groups=4,
                                    moe_topk_groups=2, moe_routed_scaling=2.0, moe_num_shared=1),
    "tiny-mla-gpu": MoEConfig(name="tiny-mla-gpu", num_layers=3, num_dense_layers=1, hidden=1024, dense_ffn=2048,
                              num_heads=16, q_lora_rank=512, kv_lora_rank=512, qk_rope_dim=64, qk_nope_dim=128,
                              v_head_dim=128, num_experts=16, moe_ffn=512, top_k=4, n_groups=4, topk_groups=2,
                              vocab=4096, max_model_len=4096, weight_dtype="fp8"),
    "tiny-moe": MoEConfig(name="tiny-moe", num_layers=3, num_dense_layers=1, hidden=256, dense_ffn=512,
                          num_heads=4, q_lora_rank=128, kv_lora_rank=64, qk_rope_dim=32, qk_nope_dim=32,
                          v_head_dim=32, num_experts=8, moe_ffn=128, top_k=2, n_groups=2, topk_groups=1,
                          vocab=1024, max_model_len=2048, weight_dtype="bf16"),
}


def get_config(name: str) -> DenseConfig | MoEConfig:
    if name not in PRESETS:
        raise KeyError(f"unknown model preset {name!r}; known: {sorted(PRESETS)}")
    import copy

    return copy.deepcopy(PRESETS[name])
