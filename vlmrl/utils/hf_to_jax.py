"""HuggingFace snapshot -> converted checkpoint directory (reference ``utils/hf_to_jax.py:1-135``).

``python -m vlmrl.utils.hf_to_jax --model_dir=checkpoints/qwen3vl_4b --hf_dir=/path/to/snapshot``

Writes ``<model_dir>/params.pkl`` (the pickled ``{"params": tree, "_timestamp"}``
layout of ``vlmrl.utils.checkpoint.Checkpoint``, with Flax-named ``[in, out]``
kernels) and copies the config, tokenizer, preprocessor, generation and chat
template JSON files beside it.  ``--model_type`` picks the model family
(``qwen3vl`` default repo ``Qwen/Qwen3-VL-4B-Instruct``; ``qwen25vl`` default
``Qwen/Qwen2.5-VL-7B-Instruct``).  Without ``--hf_dir`` the snapshot is looked
up in the local HuggingFace cache only (``local_files_only``): this framework
runs without network access.
"""

from __future__ import annotations

import argparse
import importlib
import os
import shutil
from typing import Optional

from vlmrl.utils.checkpoint import Checkpoint

DEFAULT_REPOS = {"qwen25vl": "Qwen/Qwen2.5-VL-7B-Instruct", "qwen3vl": "Qwen/Qwen3-VL-4B-Instruct"}
BASE_FILES = ["config.json", "tokenizer_config.json", "tokenizer.json", "preprocessor_config.json",
              "generation_config.json", "chat_template.json"]


def resolve_hf_dir(hf_dir: Optional[str], hf_repo: str, revision: Optional[str] = None,
                   cache_dir: Optional[str] = None) -> str:
    """Local snapshot directory: ``hf_dir`` when given, else the cached snapshot of ``hf_repo``."""
    if hf_dir:
        return os.path.join(os.path.expanduser(hf_dir), "")
    from huggingface_hub import snapshot_download

    path = snapshot_download(repo_id=hf_repo, revision=revision, local_files_only=True,
                             cache_dir=None if cache_dir is None else os.path.expanduser(cache_dir))
    return os.path.join(path, "")


def convert(hf_dir: str, model_dir: str, model_type: str = "qwen3vl") -> str:
    """Convert one snapshot; returns the path of the written ``params.pkl``."""
    mod = importlib.import_module(f"vlmrl.models.{model_type}")
    _, params = mod.create_model_from_hf(hf_dir)
    os.makedirs(model_dir, exist_ok=True)
    path = os.path.join(model_dir, "params.pkl")
    ckpt = Checkpoint(path, parallel=False)
    ckpt.params = params
    ckpt.save()
    files = BASE_FILES + (["video_preprocessor_config.json"] if model_type == "qwen3vl" else [])
    for fname in files:
        src = os.path.join(hf_dir, fname)
        if os.path.exists(src):
            shutil.copy(src, os.path.join(model_dir, fname))
            print(f"Copied: {fname}")
        else:
            print(f"Warning: {fname} not found in HF directory; skipped copy.")
    return path


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description="Convert HF Qwen VL weights to a vlmrl checkpoint.")
    ap.add_argument("--model_type", default="qwen3vl", choices=sorted(DEFAULT_REPOS))
    ap.add_argument("--model_dir", required=True, help="output directory (created if missing)")
    ap.add_argument("--hf_dir", default=None, help="local HF snapshot directory")
    ap.add_argument("--hf_repo", default=None, help="repo id looked up in the local HF cache")
    ap.add_argument("--revision", default=None)
    ap.add_argument("--cache_dir", default=None)
    args = ap.parse_args(argv)
    repo = args.hf_repo or DEFAULT_REPOS[args.model_type]
    hf_dir = resolve_hf_dir(args.hf_dir, repo, args.revision, args.cache_dir)
    print(f"Using HF snapshot at: {hf_dir}")
    print(f"Wrote {convert(hf_dir, os.path.expanduser(args.model_dir), args.model_type)}")


if __name__ == "__main__":
    main()
