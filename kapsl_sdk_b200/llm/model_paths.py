"""Locating a model's files inside an unpacked package.

``find_model_root`` walks up from a path to the nearest directory holding a
``metadata.json``; ``find_model_asset`` looks for a file next to it or in its
``onnx-export/`` sub-directory (reference: crates/kapsl-llm/src/model_paths.rs:1-44).
"""
from __future__ import annotations

import os
from typing import Optional


def find_model_root(path: str) -> Optional[str]:
    p = os.path.abspath(path)
    if os.path.isfile(p):
        p = os.path.dirname(p)
    while True:
        if os.path.isfile(os.path.join(p, "metadata.json")):
            return p
        parent = os.path.dirname(p)
        if parent == p:
            return None
        p = parent


def find_model_asset(root: str, name: str) -> Optional[str]:
    for cand in (os.path.join(root, name), os.path.join(root, "onnx-export", name)):
        if os.path.exists(cand):
            return cand
    return None
