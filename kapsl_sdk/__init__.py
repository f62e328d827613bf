"""kapsl_sdk: Python client SDK for kapsl runtimes (C++ extension ``kapsl_sdk.kapsl_sdk``).

Public surface (same names and call signatures as the reference SDK,
crates/kapsl-pyo3/kapsl_sdk/__init__.py): ``KapslClient``, ``KapslShmClient``,
``KapslHybridClient`` and the bundled voice-embedding helpers ``list_voices`` /
``load_voice`` (float32 blobs stored next to this file as ``<name>.bin``).
"""
import pathlib

from .kapsl_sdk import KapslClient, KapslHybridClient, KapslShmClient

__all__ = ["KapslClient", "KapslHybridClient", "KapslShmClient", "load_voice", "list_voices"]

_HERE = pathlib.Path(__file__).resolve().parent


def list_voices() -> list:
    """Sorted names (file stems) of the bundled ``*.bin`` voice embeddings."""
    return sorted(p.stem for p in _HERE.glob("*.bin"))


def load_voice(name: str) -> bytes:
    """Raw float32 bytes of voice ``name``; view as ``(-1, 1, 256)`` and index
    by token count to get the style vector for an utterance."""
    path = _HERE / f"{name}.bin"
    if not path.is_file():
        raise FileNotFoundError(f"Voice '{name}' not found. Available: {list_voices()}")
    return path.read_bytes()
