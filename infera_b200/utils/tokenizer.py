"""Tokenizers shared by the router (block hashing) and the engine (inputs).

The router must tokenize a request exactly as the engine does, or every
prefix lookup misses. Both sides therefore call :func:`request_token_ids`
with the same tokenizer:

* a ``prompt`` that is a list of ints is taken as token ids verbatim;
* a string ``prompt`` is encoded;
* chat ``messages`` are rendered with the tokenizer's chat template, then
  encoded (OpenAI content blocks: text parts are concatenated).

:class:`ByteTokenizer` is the built-in tokenizer (no files needed): UTF-8
bytes at ids [BYTE_BASE, BYTE_BASE + 256) plus a few special ids.
:class:`HFTokenizer` wraps a HuggingFace ``tokenizer.json``.
"""

from __future__ import annotations

import hashlib
import json
from typing import Any

CANARY_STRING = "The quick brown fox jumps over the lazy dog. 0123456789 ~!@#$%^&*() é中文"


class ByteTokenizer:
    def __init__(self, vocab_size: int = 128256, bos_id: int | None = None, eos_id: int | None = None):
        self.vocab_size = vocab_size
        # bytes live at [BYTE_BASE, BYTE_BASE + 256); small test vocabularies start them at 0
        self.BYTE_BASE = 1000 if vocab_size >= 2048 else 0
        if bos_id is None:
            bos_id = 128000 if vocab_size > 128010 else vocab_size - 16
        if eos_id is None:
            eos_id = bos_id + 1
        self.bos_id = bos_id
        self.eos_id = eos_id
        self.start_id = bos_id + 6   # <|start_header|>
        self.end_id = bos_id + 9     # <|eot|>
        self.name = f"infera-byte-v1-{vocab_size}"

    def encode(self, text: str, add_bos: bool = False) -> list[int]:
        ids = [self.BYTE_BASE + b for b in text.encode("utf-8")]
        return [self.bos_id] + ids if add_bos else ids

    def decode(self, ids) -> str:
        bs = bytes(i - self.BYTE_BASE for i in ids if self.BYTE_BASE <= i < self.BYTE_BASE + 256)
        return bs.decode("utf-8", errors="replace")

    def decode_token(self, i: int) -> str:
        if self.BYTE_BASE <= i < self.BYTE_BASE + 256:
            return bytes([i - self.BYTE_BASE]).decode("latin-1")
        return ""

    def apply_chat_template(self, messages: list[dict], add_generation_prompt: bool = True) -> list[int]:
        out = [self.bos_id]
        for m in messages:
            out.append(self.start_id)
            out += self.encode(str(m.get("role", "user")) + "\n")
            out += self.encode(_content_text(m.get("content")))
            out.append(self.end_id)
        if add_generation_prompt:
            out.append(self.start_id)
            out += self.encode("assistant\n")
        return out

    def digest(self) -> str:
        return hashlib.sha256(self.name.encode()).hexdigest()


class HFTokenizer:
    def __init__(self, path: str):
        from tokenizers import Tokenizer

        self.path = path
        self.tok = Tokenizer.from_file(path)
        self.vocab_size = self.tok.get_vocab_size()
        self.eos_id = None
        self.bos_id = None
        self.name = path
        self._template = None
        try:
            import os

            cfg = os.path.join(os.path.dirname(path), "tokenizer_config.json")
            with open(cfg) as f:
                c = json.load(f)
            self._template = c.get("chat_template")
        except Exception:
            pass

    def encode(self, text: str, add_bos: bool = False) -> list[int]:
        return self.tok.encode(text, add_special_tokens=add_bos).ids

    def decode(self, ids) -> str:
        return self.tok.decode(list(ids))

    def decode_token(self, i: int) -> str:
        return self.tok.decode([i])

    def apply_chat_template(self, messages: list[dict], add_generation_prompt: bool = True) -> list[int]:
        text = ""
        for m in messages:
            text += f"<|{m.get('role', 'user')}|>\n{_content_text(m.get('content'))}\n"
        if add_generation_prompt:
            text += "<|assistant|>\n"
        return self.encode(text)

    def digest(self) -> str:
        with open(self.path, "rb") as f:
            return hashlib.sha256(f.read()).hexdigest()


def _content_text(content: Any) -> str:
    if isinstance(content, str):
        return content
    if isinstance(content, list):
        parts = []
        for b in content:
            if isinstance(b, dict) and b.get("type") in ("text", "input_text"):
                parts.append(str(b.get("text", "")))
            elif isinstance(b, str):
                parts.append(b)
        return "".join(parts)
    return "" if content is None else str(content)


def load_tokenizer(spec: str | None = None, vocab_size: int = 128256):
    if spec and spec.endswith(".json"):
        return HFTokenizer(spec)
    return ByteTokenizer(vocab_size=vocab_size)


def canary(tok) -> list[int]:
    return tok.encode(CANARY_STRING)


def request_token_ids(body: dict, tok) -> list[int]:
    """Token ids of a completions / chat-completions request body."""
    cached = body.get("_infera_token_ids")
    if isinstance(cached, list):
        return cached
    prompt = body.get("prompt")
    if prompt is not None:
        if isinstance(prompt, list) and (not prompt or isinstance(prompt[0], int)):
            ids = [int(x) for x in prompt]
        elif isinstance(prompt, list) and prompt and isinstance(prompt[0], list):
            ids = [int(x) for x in prompt[0]]
        elif isinstance(prompt, list):
            ids = tok.encode(str(prompt[0]))
        else:
            ids = tok.encode(str(prompt))
    else:
        ids = tok.apply_chat_template(body.get("messages") or [], add_generation_prompt=True)
    return ids
