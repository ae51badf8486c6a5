"""Model path resolution (HF snapshot with a diffusers-layout allow-list, or a local dir).

Reference: ``difflet/pipeline/path_resolver.py:17-80``.  Offline runs use
``random_init=True`` (no download) or a local directory.
"""

from __future__ import annotations

import os

DEFAULT_DIFFUSERS_PATTERNS = (
    "model_index.json", "*/config.json", "*/*.json", "*/*.safetensors", "*/*.txt", "*/*.model",
    "*/spiece.model", "*/tokenizer*", "scheduler/*",
)


def resolve_model_path(model_id: str, *, revision=None, local_files_only=False, allow_patterns=None,
                       random_init=False) -> str:
    if random_init:
        return ""
    if os.path.isdir(model_id):
        return os.path.abspath(model_id)
    try:
        from huggingface_hub import snapshot_download
    except ImportError as exc:  # pragma: no cover
        raise RuntimeError("huggingface_hub is required to download models") from exc
    return snapshot_download(model_id, revision=revision, local_files_only=local_files_only,
                             allow_patterns=list(allow_patterns or DEFAULT_DIFFUSERS_PATTERNS))
