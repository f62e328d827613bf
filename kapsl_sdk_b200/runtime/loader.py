"""Model packages and engine construction (crates/kapsl-core/src/loader.rs,
requirements.rs; crates/kapsl-llm/src/llm_backend.rs:392-516).

* ``.aimod`` package = tar.gz with ``metadata.json`` (the Manifest), the model
  file and sibling assets.  Packages are extracted once into a content-addressed
  cache directory (sha256 of path, size and mtime) that is trimmed LRU-by-mtime
  under ``KAPSL_MODEL_CACHE_MAX_BYTES`` / ``..._MAX_MIB`` while keeping
  ``KAPSL_MODEL_CACHE_RESERVED_FREE_BYTES`` / ``..._MIB`` free (``KAPSL_LITE_*``
  variants accepted).  Raw ``.gguf`` / ``.onnx`` / safetensors directories load
  without a package (``from_raw_file``).
* ``build_llm_engine`` reads the manifest's ``metadata.llm`` hints (max_seq_len,
  max_num_seqs, kv_cache.block_size / total_blocks / eviction, scheduler
  budget), the ``KAPSL_LLM_*`` environment overrides, loads weights (GGUF,
  safetensors, ONNX initializers, or random init for an architecture preset)
  and returns ``(LLMEngine, tokenizer, RuntimeConfig)``.
"""
from __future__ import annotations

import hashlib
import json
import os
import shutil
import tarfile
import tempfile
from dataclasses import dataclass, field
from typing import Optional


@dataclass
class HardwareRequirements:
    preferred_provider: Optional[str] = None
    fallback_providers: list = field(default_factory=list)
    min_memory_mb: Optional[int] = None
    min_vram_mb: Optional[int] = None
    gpu_memory_reservation_mb: Optional[int] = None
    gpu_memory_limit_mb: Optional[int] = None
    gpu_compute_share_milli: Optional[int] = None
    isolation_mode: Optional[str] = None
    min_cuda_version: Optional[str] = None
    required_precision: Optional[str] = None
    optimized_for: list = field(default_factory=list)
    graph_optimization_level: Optional[str] = None
    device_id: Optional[int] = None
    gpu_device_ids: list = field(default_factory=list)
    strategy: Optional[str] = None

    @classmethod
    def from_dict(cls, d: Optional[dict]) -> "HardwareRequirements":
        d = d or {}
        known = {k: d[k] for k in cls.__dataclass_fields__ if k in d}
        return cls(**known)


@dataclass
class Manifest:
    project_name: str
    framework: str
    version: str
    model_file: str
    created_at: str = ""
    metadata: dict = field(default_factory=dict)
    hardware_requirements: HardwareRequirements = field(default_factory=HardwareRequirements)
    cron_jobs: list = field(default_factory=list)

    @classmethod
    def from_dict(cls, d: dict) -> "Manifest":
        for k in ("project_name", "framework", "version", "model_file"):
            if k not in d:
                raise ValueError(f"metadata.json is missing '{k}'")
        return cls(project_name=d["project_name"], framework=d["framework"], version=str(d["version"]),
                   model_file=d["model_file"], created_at=d.get("created_at", ""), metadata=d.get("metadata") or {},
                   hardware_requirements=HardwareRequirements.from_dict(d.get("hardware_requirements")),
                   cron_jobs=d.get("cron_jobs") or [])

    def llm_hints(self) -> dict:
        return dict((self.metadata or {}).get("llm") or {})


@dataclass
class LoadedPackage:
    manifest: Manifest
    root: str
    model_path: str


def _env_int(*names) -> Optional[int]:
    for n in names:
        v = os.environ.get(n)
        if v:
            try:
                return int(v)
            except ValueError:
                pass
    return None


class PackageLoader:
    def __init__(self, cache_dir: Optional[str] = None, max_bytes: Optional[int] = None,
                 reserved_free_bytes: Optional[int] = None):
        self.cache_dir = cache_dir or os.environ.get("KAPSL_MODEL_CACHE_DIR") or os.environ.get(
            "KAPSL_LITE_MODEL_CACHE_DIR") or os.path.join(tempfile.gettempdir(), "kapsl-model-cache")
        mib = _env_int("KAPSL_MODEL_CACHE_MAX_MIB", "KAPSL_LITE_MODEL_CACHE_MAX_MIB")
        self.max_bytes = max_bytes if max_bytes is not None else (
            _env_int("KAPSL_MODEL_CACHE_MAX_BYTES", "KAPSL_LITE_MODEL_CACHE_MAX_BYTES") or
            (mib << 20 if mib else None))
        rmib = _env_int("KAPSL_MODEL_CACHE_RESERVED_FREE_MIB", "KAPSL_LITE_MODEL_CACHE_RESERVED_FREE_MIB")
        self.reserved_free = reserved_free_bytes if reserved_free_bytes is not None else (
            _env_int("KAPSL_MODEL_CACHE_RESERVED_FREE_BYTES", "KAPSL_LITE_MODEL_CACHE_RESERVED_FREE_BYTES") or
            (rmib << 20 if rmib else 0))
        os.makedirs(self.cache_dir, exist_ok=True)

    @staticmethod
    def cache_key(path: str) -> str:
        st = os.stat(path)
        h = hashlib.sha256(f"{os.path.abspath(path)}|{st.st_size}|{st.st_mtime_ns}".encode()).hexdigest()
        return h[:32]

    def load(self, package_path: str) -> LoadedPackage:
        """Extract (or reuse the cached extraction of) an ``.aimod`` package."""
        if not os.path.isfile(package_path):
            raise FileNotFoundError(package_path)
        dest = os.path.join(self.cache_dir, self.cache_key(package_path))
        if not os.path.isfile(os.path.join(dest, "metadata.json")):
            tmp = tempfile.mkdtemp(prefix=".extract-", dir=self.cache_dir)
            try:
                with tarfile.open(package_path, "r:gz") as tf:
                    for m in tf.getmembers():
                        target = os.path.realpath(os.path.join(tmp, m.name))
                        if not target.startswith(os.path.realpath(tmp) + os.sep) and target != os.path.realpath(tmp):
                            raise ValueError(f"unsafe path in package: {m.name}")
                        if m.issym() or m.islnk():
                            raise ValueError(f"links are not allowed in packages: {m.name}")
                    tf.extractall(tmp)
                root = tmp
                if not os.path.isfile(os.path.join(root, "metadata.json")):
                    subs = [os.path.join(root, d) for d in os.listdir(root)]
                    subs = [s for s in subs if os.path.isfile(os.path.join(s, "metadata.json"))]
                    if not subs:
                        raise ValueError("package has no metadata.json")
                    root = subs[0]
                if os.path.exists(dest):
                    shutil.rmtree(dest)
                shutil.move(root, dest)
            finally:
                if os.path.isdir(tmp):
                    shutil.rmtree(tmp, ignore_errors=True)
            self.evict(keep=dest)
        os.utime(dest)  # LRU by mtime
        with open(os.path.join(dest, "metadata.json")) as f:
            man = Manifest.from_dict(json.load(f))
        return LoadedPackage(man, dest, os.path.join(dest, man.model_file))

    @staticmethod
    def from_raw_file(path: str) -> LoadedPackage:
        """A bare model file or directory: framework from the extension."""
        p = os.path.abspath(path)
        if os.path.isdir(p):
            meta = os.path.join(p, "metadata.json")
            if os.path.isfile(meta):
                with open(meta) as f:
                    man = Manifest.from_dict(json.load(f))
                return LoadedPackage(man, p, os.path.join(p, man.model_file))
            man = Manifest(os.path.basename(p), "llm", "1.0", ".")
            return LoadedPackage(man, p, p)
        ext = os.path.splitext(p)[1].lower()
        fw = {".gguf": "gguf", ".onnx": "onnx", ".safetensors": "llm"}.get(ext)
        if fw is None:
            raise ValueError(f"unsupported model file {path}")
        man = Manifest(os.path.splitext(os.path.basename(p))[0], fw, "1.0", os.path.basename(p))
        return LoadedPackage(man, os.path.dirname(p), p)

    def _entries(self) -> list:
        out = []
        for d in os.listdir(self.cache_dir):
            full = os.path.join(self.cache_dir, d)
            if d.startswith(".") or not os.path.isdir(full):
                continue
            size = sum(os.path.getsize(os.path.join(r, f)) for r, _, fs in os.walk(full) for f in fs)
            out.append((os.path.getmtime(full), size, full))
        return sorted(out)

    def evict(self, keep: Optional[str] = None) -> int:
        """Remove least-recently-used extractions beyond the size / free-space limits."""
        removed = 0
        entries = self._entries()
        total = sum(s for _, s, _ in entries)
        for mtime, size, path in entries:
            over = self.max_bytes is not None and total > self.max_bytes
            free = shutil.disk_usage(self.cache_dir).free
            low_free = self.reserved_free and free < self.reserved_free
            if not (over or low_free):
                break
            if keep and os.path.samefile(path, keep):
                continue
            shutil.rmtree(path, ignore_errors=True)
            total -= size
            removed += 1
        return removed


def llm_env_overrides(hints: dict) -> dict:
    """``KAPSL_LLM_*`` environment overrides of the manifest's KV/scheduler hints
    (crates/kapsl-llm/src/engine.rs:1328-1421)."""
    h = dict(hints)
    kv = dict(h.get("kv_cache") or {})
    m = {"KAPSL_LLM_KV_CACHE_MODE": ("mode", str), "KAPSL_LLM_KV_CACHE_BLOCK_SIZE": ("block_size", int),
         "KAPSL_LLM_KV_CACHE_TOTAL_BLOCKS": ("total_blocks", int), "KAPSL_LLM_KV_CACHE_EVICTION": ("eviction", str),
         "KAPSL_LLM_KV_ADMISSION_SOFT_LIMIT_BYTES": ("admission_soft_limit_bytes", int),
         "KAPSL_LLM_KV_ADMISSION_HARD_LIMIT_BYTES": ("admission_hard_limit_bytes", int)}
    for env, (key, typ) in m.items():
        v = os.environ.get(env)
        if v:
            kv[key] = typ(v)
    h["kv_cache"] = kv
    return h


def engine_config_from_hints(hints: dict, device_type: str = "cuda"):
    from ..llm.engine import EngineConfig

    h = llm_env_overrides(hints)
    kv = h.get("kv_cache") or {}
    sched = h.get("scheduler") or {}
    ev = str(kv.get("eviction", "lru")).lower()
    e = EngineConfig(
        max_num_seqs=int(sched.get("max_num_seqs", h.get("max_num_seqs", 256 if device_type == "cuda" else 16))),
        max_num_batched_tokens=int(sched.get("max_num_batched_tokens", h.get("chunked_prefill_tokens", 2048))),
        max_model_len=int(h.get("max_sequence_length", h.get("max_seq_len", 4096))),
        block_size=int(kv.get("block_size", 16)),
        num_blocks=int(kv.get("total_blocks", 0)),
        eviction="fifo" if ev.startswith("fifo") else "lru",
        enable_prefix_cache=str(kv.get("mode", "paged")).lower() != "dense",
        max_session_tokens=int(h.get("max_session_tokens", 0)),
        kv_soft_limit_bytes=int(kv.get("admission_soft_limit_bytes", 0)),
        kv_hard_limit_bytes=int(kv.get("admission_hard_limit_bytes", 0)),
    )
    if e.block_size != 16 and device_type == "cuda":
        raise ValueError("the GPU paged-attention kernels use 16-token KV blocks")
    return e


def build_llm_engine(model_path: str, device: Optional[str] = None, tp_comm=None):
    """Package / directory / file -> (LLMEngine, tokenizer, RuntimeConfig)."""
    import torch

    from ..llm.backend import load_runtime_config
    from ..llm.engine import LLMEngine
    from ..llm.tokenizer import load_tokenizer

    pkg = PackageLoader().load(model_path) if model_path.endswith(".aimod") else PackageLoader.from_raw_file(model_path)
    hints = pkg.manifest.llm_hints()
    if device is None:
        hw = pkg.manifest.hardware_requirements
        want_cpu = (hw.preferred_provider or "").lower() == "cpu"
        device = "cpu" if want_cpu or not torch.cuda.is_available() else f"cuda:{hw.device_id or 0}"
    dev = torch.device(device)
    try:
        cfg, weights, tokenizer = load_model_weights(pkg.model_path, pkg.root, hints, dev, tp_comm)
    except OnnxNotMappable:
        # a decoder export whose weights do not map onto the native model: the graph
        # itself serves (interpreter, per-sequence KV as its present tensors)
        from ..llm.onnx_decoder import OnnxDecoderEngine

        if tp_comm is not None and tp_comm.world_size > 1:
            raise ValueError("ONNX decoder graphs without Hugging Face weight names serve on one device")
        engine = OnnxDecoderEngine(pkg.model_path, pkg.root, device=str(dev),
                                   max_model_len=engine_config_from_hints(hints, dev.type).max_model_len)
        c = engine.cfg
        return engine, load_tokenizer(pkg.root, c.vocab_size, c.bos_token_id, c.eos_token_id), \
            load_runtime_config(pkg.root)
    ecfg = engine_config_from_hints(hints, dev.type)
    ecfg.max_model_len = min(ecfg.max_model_len, cfg.max_position)
    engine = LLMEngine(cfg, weights=weights, device=dev, engine_cfg=ecfg, tp_comm=tp_comm)
    rc = load_runtime_config(pkg.root)
    if tokenizer is None:
        tokenizer = load_tokenizer(pkg.root, cfg.vocab_size, cfg.bos_token_id, cfg.eos_token_id)
    if pkg.manifest.framework == "gguf":
        rc.use_chat_template = False  # GGUF prompts are raw UTF-8, greedy (gguf_backend.rs:65-76)
        rc.sampling.temperature = 0.0
    return engine, tokenizer, rc


class OnnxNotMappable(ValueError):
    """An ONNX decoder export whose initializers do not carry Hugging Face weight names."""


def load_model_weights(model_path: str, root: str, hints: dict, device, tp_comm=None):
    """Returns (ModelConfig, weights for the device, tokenizer or None)."""
    from ..models.config import ModelConfig, get_preset

    tp = 1 if tp_comm is None else tp_comm.world_size
    rank = 0 if tp_comm is None else tp_comm.rank
    if model_path.endswith(".gguf"):
        from ..loaders.gguf import load_gguf_model

        return load_gguf_model(model_path, device, tp, rank)
    if model_path.endswith(".onnx"):
        from ..loaders.onnx import load_onnx_llm

        try:
            return load_onnx_llm(model_path, root, device, tp, rank)
        except ValueError as e:
            if "lacks initializer" in str(e):
                raise OnnxNotMappable(str(e)) from e
            raise
    cfg_path = os.path.join(root, "config.json")
    if os.path.isdir(model_path) or model_path.endswith(".safetensors"):
        from ..loaders.hf import load_hf_model

        return load_hf_model(model_path if os.path.isdir(model_path) else root, device, tp, rank)
    preset = hints.get("architecture") or hints.get("preset")
    if preset:
        cfg = get_preset(preset)
    elif os.path.isfile(cfg_path):
        cfg = ModelConfig.from_hf_config(cfg_path)
    else:
        raise ValueError(f"cannot determine the model architecture for {model_path}")
    return cfg, None, None
