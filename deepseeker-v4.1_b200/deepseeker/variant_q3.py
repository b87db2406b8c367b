"""DEEPSEEKER_VARIANT handling -- drop-in for the reference's ``deepseeker.variant_q3``
(src/deepseeker/variant_q3.py:15-34): a variant name ending in "q3" (any case)
selects the 3-bit manifest and model root; anything else the MXFP4 baseline.
"""
from __future__ import annotations

import os
from pathlib import Path


def is_q3(variant: str | None = None) -> bool:
    name = os.environ.get("DEEPSEEKER_VARIANT", "") if variant is None else variant
    return name.lower().endswith("q3")


def paths_for_variant(revision: str, repo_root: Path, snapshot_name: str,
                      variant: str | None = None) -> tuple[Path, Path]:
    """(model_root, manifest_path) for the active variant; the model root falls
    back to models/DeepSeek-V4.1-Flash-1017 when the variant's root is absent."""
    profile_dir = Path(repo_root) / "profiles" / "deepseek-v4.1-flash" / revision
    models = Path(repo_root) / "models"
    if is_q3(variant):
        manifest = profile_dir / os.environ.get("DEEPSEEKER_Q3_MANIFEST", "model-manifest-q3.json")
        root = models / f"{snapshot_name}-Q3"
    else:
        manifest = profile_dir / "model-manifest.json"
        root = models / snapshot_name
    if not root.exists():
        root = models / "DeepSeek-V4.1-Flash-1017"
    return root, manifest
