"""Tokenizer loading with an offline byte-level fallback.

``load_tokenizer(model_dir)`` returns the HF tokenizer saved next to a
checkpoint when its files are present.  Otherwise (random-init benchmarks, no
network) it returns ``ByteTokenizer``: ids 0-255 are raw bytes, the Qwen chat /
vision special tokens keep their Qwen ids when the vocabulary is large enough
(151643 ``<|endoftext|>``, 151644 ``<|im_start|>``, 151645 ``<|im_end|>``,
151652 ``<|vision_start|>``, 151653 ``<|vision_end|>``, 151655
``<|image_pad|>``, 151656 ``<|video_pad|>``) and sit at the top of the vocabulary
for small test vocabularies.  Any other id decodes to a short placeholder word.
"""

from __future__ import annotations

import os
import re
from typing import Dict, List, Optional, Sequence

QWEN_SPECIALS = {
    "<|endoftext|>": 151643, "<|im_start|>": 151644, "<|im_end|>": 151645,
    "<|vision_start|>": 151652, "<|vision_end|>": 151653, "<|image_pad|>": 151655, "<|video_pad|>": 151656,
}


class ByteTokenizer:
    def __init__(self, vocab_size: int = 151936, specials: Optional[Dict[str, int]] = None):
        self.vocab_size = int(vocab_size)
        if specials is None:
            if self.vocab_size > max(QWEN_SPECIALS.values()):
                specials = dict(QWEN_SPECIALS)
            else:
                names = list(QWEN_SPECIALS)
                specials = {n: self.vocab_size - len(names) + i for i, n in enumerate(names)}
        self.specials = dict(specials)
        self.id_to_special = {v: k for k, v in self.specials.items()}
        self._split = re.compile("(" + "|".join(re.escape(s) for s in sorted(self.specials, key=len, reverse=True)) + ")")
        self.eos_token_id = self.specials["<|im_end|>"]
        self.pad_token_id = self.specials["<|endoftext|>"]
        self.image_token_id = self.specials["<|image_pad|>"]
        self.vision_start_token_id = self.specials["<|vision_start|>"]
        self.vision_end_token_id = self.specials["<|vision_end|>"]
        self.video_token_id = self.specials["<|video_pad|>"]

    def encode(self, text: str, add_special_tokens: bool = False) -> List[int]:
        out: List[int] = []
        for piece in self._split.split(text):
            if not piece:
                continue
            if piece in self.specials:
                out.append(self.specials[piece])
            else:
                out.extend(piece.encode("utf-8"))
        return out

    def __call__(self, text: str, **_):
        return {"input_ids": self.encode(text)}

    def decode(self, ids: Sequence[int], skip_special_tokens: bool = True, **_) -> str:
        parts: List[str] = []
        buf = bytearray()
        for t in ids:
            t = int(t)
            if t < 256:
                buf.append(t)
                continue
            if buf:
                parts.append(buf.decode("utf-8", errors="replace"))
                buf = bytearray()
            if t in self.id_to_special:
                if not skip_special_tokens:
                    parts.append(self.id_to_special[t])
            else:
                parts.append(f" w{t}")
        if buf:
            parts.append(buf.decode("utf-8", errors="replace"))
        return "".join(parts)

    def get_eos_token_id(self) -> int:
        return self.eos_token_id


def load_tokenizer(model_dir: Optional[str], vocab_size: int = 151936):
    if model_dir and any(os.path.exists(os.path.join(model_dir, f)) for f in ("tokenizer.json", "tokenizer_config.json")):
        try:
            from transformers import AutoTokenizer

            return AutoTokenizer.from_pretrained(model_dir, trust_remote_code=False)
        except Exception:
            pass
    return ByteTokenizer(vocab_size)


def special_id(tokenizer, name: str, default: int) -> int:
    """Resolve a special token id from any tokenizer flavour."""
    specials = getattr(tokenizer, "specials", None)
    if isinstance(specials, dict) and name in specials:
        return int(specials[name])
    conv = getattr(tokenizer, "convert_tokens_to_ids", None)
    if callable(conv):
        try:
            val = conv(name)
            if val is not None and int(val) >= 0:
                return int(val)
        except Exception:
            pass
    return int(default)


__all__ = ["ByteTokenizer", "load_tokenizer", "special_id", "QWEN_SPECIALS"]
