"""A HuggingFace-style model directory for the random-init benchmark models,
so that stock engines (vLLM with ``--load-format dummy``) can serve the same
architecture without a checkpoint.

The tokenizer is word-level: token id ``i`` is the word ``t<i>`` and words
are split on whitespace, so a trace of token ids becomes a text prompt
that any HF tokenizer loader turns back into exactly those ids (no special
tokens are added), and generated text maps back to ids the same way.
"""

from __future__ import annotations

import json
import os

from infera_b200.models.config import DenseConfig, get_config


def ids_to_text(ids) -> str:
    return " ".join(f"t{i}" for i in ids)


def text_to_ids(text: str) -> list[int]:
    out = []
    for w in text.split():
        if w.startswith("t") and w[1:].isdigit():
            out.append(int(w[1:]))
    return out


def write_model_dir(path: str, model: str = "llama-3.1-8b", max_position: int = 131072) -> str:
    cfg: DenseConfig = get_config(model)
    os.makedirs(path, exist_ok=True)
    bos, eos = 128000, 128001
    hf = {
        "architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": cfg.hidden,
        "intermediate_size": cfg.ffn, "num_hidden_layers": cfg.num_layers, "num_attention_heads": cfg.num_heads,
        "num_key_value_heads": cfg.num_kv_heads, "head_dim": cfg.head_dim, "vocab_size": cfg.vocab,
        "rms_norm_eps": cfg.rms_eps, "rope_theta": cfg.rope_theta, "max_position_embeddings": max_position,
        "hidden_act": "silu", "tie_word_embeddings": False, "torch_dtype": "bfloat16", "bos_token_id": bos,
        "eos_token_id": eos, "attention_bias": False, "mlp_bias": False,
    }
    if cfg.rope_scaling:
        hf["rope_scaling"] = dict(cfg.rope_scaling, rope_type="llama3")
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(hf, f, indent=1)
    with open(os.path.join(path, "generation_config.json"), "w") as f:
        json.dump({"bos_token_id": bos, "eos_token_id": eos, "do_sample": False}, f)
    tok_path = os.path.join(path, "tokenizer.json")
    if not os.path.exists(tok_path):
        from tokenizers import Tokenizer, decoders, models, pre_tokenizers

        vocab = {f"t{i}": i for i in range(cfg.vocab)}
        tok = Tokenizer(models.WordLevel(vocab, unk_token="t0"))
        tok.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
        tok.decoder = decoders.WordPiece(prefix="##", cleanup=False)
        tok.save(tok_path)
    with open(os.path.join(path, "tokenizer_config.json"), "w") as f:
        json.dump({"tokenizer_class": "PreTrainedTokenizerFast", "bos_token": f"t{bos}", "eos_token": f"t{eos}",
                   "unk_token": "t0", "pad_token": "t0", "add_bos_token": False, "add_eos_token": False,
                   "clean_up_tokenization_spaces": False, "model_max_length": max_position,
                   "chat_template": "{% for m in messages %}{{ m['content'] }} {% endfor %}"}, f)
    return path
