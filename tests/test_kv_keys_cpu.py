"""KV index keys and types: model families, compatibility keys (every part
that shapes the KV bytes changes the key, nothing else does), tier order,
overlap summaries."""

import pytest

from infera_b200.kv.compat_key import compat_key
from infera_b200.kv.families import family_of
from infera_b200.kv.types import OverlapBlocks, Tier


@pytest.mark.parametrize("name,fam", [
    ("deepseek-ai/DeepSeek-V3", "deepseek-v3"), ("DeepSeek-R1-0528", "deepseek-v3"),
    ("moonshotai/Kimi-K2-Instruct", "kimi-k2"), ("meta-llama/Llama-3.1-8B-Instruct", "llama-3"),
    ("llama-3.1-8b", "llama-3"), ("Qwen/Qwen3-32B", "qwen3"), ("Qwen2.5-7B", "qwen2"),
    ("zai-org/GLM-4.6", "glm"), ("mistralai/Mixtral-8x7B", "mistral"), ("openai/gpt-oss-120b", "gpt-oss"),
    ("Some Custom_Model v2", "some-custom-model-v2"), ("///", "unknown"),
])
def test_family_of(name, fam):
    assert family_of(name) == fam


def test_compat_key_sensitivity():
    base = dict(model_name="llama-3.1-8b", tokenizer_digest="abc", block_size=16, kv_dtype="bf16", role="mixed")
    k0 = compat_key(**base)
    assert k0 == compat_key(**base) and len(k0) == 24
    for field, other in (("model_name", "llama-3.1-70b"), ("tokenizer_digest", "abd"), ("block_size", 32),
                         ("kv_dtype", "fp8"), ("role", "decode")):
        assert compat_key(**{**base, field: other}) != k0, field
    assert compat_key(**base, extra={"lora": "x"}) != k0


def test_tier_order_and_overlap():
    assert sorted(Tier, key=lambda t: t.rank) == [Tier.DEVICE, Tier.HOST, Tier.DISK, Tier.FABRIC]
    o = OverlapBlocks("w0", {Tier.DEVICE: 3, Tier.HOST: 7})
    assert o.best() == 7 and o.device() == 3
    assert OverlapBlocks("w1").best() == 0 and OverlapBlocks("w1").device() == 0
