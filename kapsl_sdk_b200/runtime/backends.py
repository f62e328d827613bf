"""Backends, the backend factory and the engine pool (crates/kapsl-backends).

* ``OnnxBackend``: an :class:`Engine` over :class:`~kapsl_sdk_b200.loaders.onnx.OnnxGraph`
  (GPU when available).  Shape-bucketed graph instances are kept in an LRU of
  ``KAPSL_ORT_SESSION_BUCKETS`` entries (reference onnx.rs:367-441); inputs are
  validated per dtype; additional named inputs are fed by name.
* ``BackendFactory``: ``gguf`` and ``llm`` frameworks -> :class:`LLMBackend`,
  ``onnx`` -> ``OnnxBackend``; provider order preferred -> fallbacks ->
  fastest available (cuda, cpu); ``validate_requirements`` checks RAM, VRAM and
  CUDA version against the probed devices and understands the multi-device
  strategies pool / round-robin / data-parallel / pipeline / tensor-parallel /
  auto (factory.rs:17-579).
* ``EnginePool``: LRU ``(model_id, device_id) -> engine`` with health-checked
  ``get``, an eviction callback, warm-up and a background health task
  (engine_pool.rs:13-292).
"""
from __future__ import annotations

import collections
import os
import threading
import time
from typing import Callable, Optional

import numpy as np

from ..engine_api import (BinaryTensorPacket, Engine, EngineError, EngineMetrics, EngineModelInfo,
                          InferenceRequest, TensorDtype)
from ..hal.device import DeviceInfo, probe
from .loader import HardwareRequirements, Manifest


class OnnxBackend(Engine):
    def __init__(self, device: Optional[str] = None, max_buckets: Optional[int] = None):
        import torch

        self.device = device or ("cuda:0" if torch.cuda.is_available() else "cpu")
        self.max_buckets = max_buckets or int(os.environ.get("KAPSL_ORT_SESSION_BUCKETS", "4"))
        self.model = None
        self.graph = None
        self._lock = threading.Lock()
        self._m = EngineMetrics()
        self._times: list = []

    def load(self, model_path: str) -> None:
        """Decodes the graph; the interpreter keeps one plan per input-shape set (the
        values that depend only on initializers and input shapes, computed on the
        first request of that shape), an LRU of ``KAPSL_ORT_SESSION_BUCKETS`` entries:
        the counterpart of the reference's per-shape-bucket ORT sessions
        (crates/kapsl-backends/src/onnx.rs:367-441)."""
        from ..loaders.onnx import OnnxGraph, read_model

        try:
            self.model = read_model(model_path)
            self.graph = OnnxGraph(self.model, self.device, plan_cache=self.max_buckets)
        except (OSError, ValueError) as e:
            raise EngineError.model_load(model_path, str(e))

    def infer(self, request: InferenceRequest) -> BinaryTensorPacket:
        import torch

        if self.model is None:
            raise EngineError.model_not_loaded()
        request.input.validate()
        if request.input.dtype is TensorDtype.UTF8:
            raise EngineError.invalid_input("ONNX backend expects numeric input")
        feeds = {self.model.inputs[0]: request.input.to_numpy()}
        seen = set()
        for nt in request.additional_inputs:  # reference onnx.rs:747-764
            if nt.name in seen:
                raise EngineError.invalid_input(f"Duplicate additional input name: {nt.name}")
            seen.add(nt.name)
        for nt in request.additional_inputs:
            nt.tensor.validate()
            feeds[nt.name] = nt.tensor.to_numpy()
        self._fill_decoder_inputs(feeds)
        missing = [n for n in self.model.inputs if n not in feeds]
        if missing:
            raise EngineError.invalid_input(f"missing model inputs: {missing}")
        t0 = time.perf_counter()
        try:
            with torch.no_grad(), self._lock:  # one run at a time: plans and stats are shared
                out = self.graph.run(feeds)[self.model.outputs[0]]
        except Exception as e:
            raise EngineError.inference(str(e))
        dt = time.perf_counter() - t0
        self._m.inference_time = dt
        arr = out.detach().cpu().numpy()
        if arr.dtype == np.float16 or arr.dtype == np.float64:
            arr = arr.astype(np.float32) if arr.dtype == np.float16 else arr
        if arr.dtype == np.bool_:
            arr = arr.astype(np.uint8)
        return BinaryTensorPacket.from_numpy(arr)

    def _fill_decoder_inputs(self, feeds: dict) -> None:
        """Inputs of decoder exports that the request leaves out, filled as the
        reference backend fills them (crates/kapsl-backends/src/onnx.rs:903-1000), with
        batch and sequence length from the main input [batch, seq]: ``*attention_mask*``
        all ones [batch, seq] int64, ``*position_ids*`` 0..seq-1 per row int64, and
        ``past_key_values*`` empty [batch, heads, 0, head_dim] caches, heads and head_dim
        from the declared input shape (1 and 64 where it is symbolic)."""
        main = feeds[self.model.inputs[0]]
        batch = int(main.shape[0]) if main.ndim > 0 else 1
        seq = int(main.shape[1]) if main.ndim > 1 else 1
        dtypes = {1: np.float32, 10: np.float16, 11: np.float64}
        for name in self.model.inputs[1:]:
            if name in feeds:
                continue
            if "attention_mask" in name:
                feeds[name] = np.ones((batch, seq), np.int64)
            elif "position_ids" in name:
                feeds[name] = np.tile(np.arange(seq, dtype=np.int64), (batch, 1))
            elif name.startswith("past_key_values"):
                elem, dims = self.model.input_types.get(name, (None, []))
                if len(dims) == 4:
                    h = dims[1] if dims[1] and dims[1] > 0 else 1
                    d = dims[3] if dims[3] and dims[3] > 0 else 64
                    feeds[name] = np.zeros((batch, h, 0, d), dtypes.get(elem, np.float32))

    def model_info(self) -> EngineModelInfo:
        if self.model is None:
            return EngineModelInfo()
        names = {1: "float32", 11: "float64", 10: "float16", 6: "int32", 7: "int64", 2: "uint8", 8: "string"}

        def describe(types, keys):  # declared shapes (-1 for symbolic dims) and dtype names, as ORT reports them
            shapes = [[-1 if d is None else d for d in types.get(k, (None, []))[1]] for k in keys]
            dts = [names.get(types.get(k, (None, []))[0], "unknown") for k in keys]
            return shapes, dts

        ins, in_dt = describe(self.model.input_types, self.model.inputs)
        outs, out_dt = describe(self.model.output_types, self.model.outputs)
        peak = os.environ.get("KAPSL_MODEL_PEAK_CONCURRENCY")
        return EngineModelInfo(input_names=list(self.model.inputs), output_names=list(self.model.outputs),
                               input_shapes=ins, output_shapes=outs, input_dtypes=in_dt, output_dtypes=out_dt,
                               framework="onnx", peak_concurrency=max(1, int(peak)) if peak else None)

    def metrics(self) -> EngineMetrics:
        return self._m

    def health_check(self) -> bool:
        return self.model is not None

    def unload(self) -> None:
        self.model = None
        self.graph = None


class BackendFactory:
    PROVIDER_ORDER = ["tensorrt", "cuda", "coreml", "rocm", "directml", "openvino", "cpu"]

    def __init__(self, device_info: Optional[DeviceInfo] = None):
        self.info = device_info or probe()

    def available_providers(self) -> list:
        return (["cuda"] if self.info.has_cuda() else []) + ["cpu"]

    def provider_chain(self, hw: HardwareRequirements) -> list:
        avail = self.available_providers()
        policy = os.environ.get("KAPSL_PROVIDER_POLICY", "fastest").lower()
        chain = []
        if hw.preferred_provider:
            chain.append(hw.preferred_provider.lower())
        chain += [p.lower() for p in hw.fallback_providers]
        if policy == "fastest" or not chain:
            chain += [p for p in self.PROVIDER_ORDER if p in avail]
        seen = []
        for p in chain:
            p = "cuda" if p == "tensorrt" else p
            if p in avail and p not in seen:
                seen.append(p)
        if "cpu" not in seen:
            seen.append("cpu")
        return seen

    @staticmethod
    def check_requirements(req: HardwareRequirements, info: DeviceInfo) -> Optional[str]:
        """The reference's requirement check (crates/kapsl-backends/src/factory.rs:414-586)
        with its error texts: None when the host memory suffices and one of the
        preferred / fallback providers has a device that meets the VRAM and CUDA
        version minimums (any device of the backend under a multi-device strategy,
        else ``device_id``, default 0); otherwise the reason(s).  CUDA versions are
        compared numerically (the reference compares the strings)."""
        if req.min_memory_mb is not None and info.total_memory_mb < req.min_memory_mb:
            return f"Insufficient memory: need {req.min_memory_mb}MB, have {info.total_memory_mb}MB"
        providers = ([req.preferred_provider] if req.preferred_provider else []) + list(req.fallback_providers)
        if not providers:
            return None
        strategy = (req.strategy or "").lower()
        multi = strategy in ("pool", "round-robin", "data-parallel", "pipeline", "pipeline-parallel",
                             "tensor-parallel", "auto")

        def ver(v):
            return tuple(int(x) for x in str(v).split(".") if x.isdigit())

        def too_old(backend) -> Optional[str]:
            if backend != "cuda" or not req.min_cuda_version:
                return None
            if not info.cuda_version:
                return "Unknown CUDA version on device"
            if ver(info.cuda_version) < ver(req.min_cuda_version):
                return f"CUDA version too old: {info.cuda_version} < required {req.min_cuda_version}"
            return None

        reasons = []
        for provider in providers:
            backend = {"tensorrt": "cuda", "coreml": "metal"}.get(provider.lower(), provider.lower())
            if backend == "cpu":
                return None
            if not info.has_provider(backend):
                reasons.append(f"Provider {provider} not available")
                continue
            devs = [d for d in info.devices if d.backend.value == backend]
            if multi:
                if any((req.min_vram_mb is None or d.total_memory_mb >= req.min_vram_mb) and too_old(backend) is None
                       for d in devs):
                    return None
                reasons.append(f"No devices meet requirements for provider {provider}")
                continue
            dev_id = req.device_id or 0
            d = next((d for d in devs if d.id == dev_id), None)
            if d is None:
                reasons.append(f"Device ID {dev_id} not found for provider {provider}")
                continue
            if req.min_vram_mb is not None and d.total_memory_mb < req.min_vram_mb:
                reasons.append(f"Provider {provider} (Device {dev_id}) has insufficient VRAM: "
                               f"{d.total_memory_mb}MB < required {req.min_vram_mb}MB")
                continue
            old = too_old(backend)
            if old:
                reasons.append(old)
                continue
            return None
        return "No compatible provider found. Reasons: " + repr(reasons)

    def validate_requirements(self, manifest: Manifest, provider: str = "cuda") -> list:
        """Unmet requirements as messages (empty list = OK)."""
        hw = manifest.hardware_requirements
        errs = []
        if hw.min_memory_mb and self.info.total_memory_mb and self.info.total_memory_mb < hw.min_memory_mb:
            errs.append(f"needs {hw.min_memory_mb} MB RAM, host has {self.info.total_memory_mb} MB")
        if provider == "cuda":
            gpus = self.info.gpus()
            ids = hw.gpu_device_ids or ([hw.device_id] if hw.device_id is not None else [])
            strategy = (hw.strategy or "auto").lower()
            if strategy in ("pipeline", "tensor-parallel", "data-parallel", "round-robin", "pool") and ids:
                missing = [i for i in ids if i >= len(gpus)]
                if missing:
                    errs.append(f"strategy {strategy} needs GPUs {ids}; {len(gpus)} present")
            if hw.min_vram_mb:
                cand = [g for g in gpus if not ids or g.id in ids]
                if not any(g.total_memory_mb >= hw.min_vram_mb for g in cand):
                    errs.append(f"needs {hw.min_vram_mb} MB of GPU memory")
            if hw.min_cuda_version and self.info.cuda_version:
                def v(s):
                    return tuple(int(x) for x in s.split(".")[:2])

                if v(self.info.cuda_version) < v(hw.min_cuda_version):
                    errs.append(f"needs CUDA {hw.min_cuda_version}, have {self.info.cuda_version}")
            if not gpus:
                errs.append("no CUDA device")
        return errs

    def create_backend(self, manifest: Manifest, model_path: str) -> Engine:
        from ..llm.backend import LLMBackend

        fw = manifest.framework.lower()
        last = None
        for provider in self.provider_chain(manifest.hardware_requirements):
            if self.validate_requirements(manifest, provider) and provider != "cpu":
                continue
            try:
                if fw in ("llm", "gguf"):
                    from .loader import build_llm_engine

                    dev = "cpu" if provider == "cpu" else f"cuda:{manifest.hardware_requirements.device_id or 0}"
                    eng, tok, rc = build_llm_engine(model_path, device=dev)
                    return LLMBackend(eng, tok, rc)
                b = OnnxBackend(device="cpu" if provider == "cpu" else "cuda:0")
                b.load(model_path)
                return b
            except EngineError as e:
                last = e
            except Exception as e:  # provider failure: fall back to the next one
                last = EngineError.model_load(model_path, str(e))
        raise last or EngineError.model_load(model_path, "no provider could load the model")


class EnginePool:
    def __init__(self, capacity: int = 8, on_evict: Optional[Callable] = None):
        self.capacity = capacity
        self.on_evict = on_evict
        self._m: "collections.OrderedDict" = collections.OrderedDict()
        self._lock = threading.RLock()
        self._stop = threading.Event()
        self._thread = None
        self._stats = {"hit": 0, "failure": 0, "evictions": 0}

    def put(self, model_id: int, device_id: int, engine: Engine, warmup: bool = False) -> None:
        if warmup:
            engine.warmup()
        with self._lock:
            self._m[(model_id, device_id)] = engine
            self._m.move_to_end((model_id, device_id))
            while len(self._m) > self.capacity:
                key, old = self._m.popitem(last=False)
                self._stats["evictions"] += 1
                self._evict(key, old)

    def warmup(self, configs: list, factory: Callable) -> None:
        """Pre-create engines: ``factory(model_id, device_id)`` for each pair; one
        whose creation fails is skipped and the others still load (reference
        engine_pool.rs:250-285)."""
        for model_id, device_id in configs:
            try:
                eng = factory(model_id, device_id)
            except Exception:
                continue
            self.put(model_id, device_id, eng)

    def pool_metrics(self) -> dict:
        """Hits (healthy gets), failures (gets that found an unhealthy engine, which
        is removed), LRU evictions and the hit rate (reference engine_pool.rs:14-19, 287-291)."""
        with self._lock:
            m = dict(self._stats)
        tot = m["hit"] + m["failure"]
        m["hit_rate"] = m["hit"] / tot if tot else 0.0
        return m

    def _evict(self, key, eng) -> None:
        try:
            eng.unload()
        finally:
            if self.on_evict:
                self.on_evict(key)

    def get(self, model_id: int, device_id: int) -> Optional[Engine]:
        with self._lock:
            eng = self._m.get((model_id, device_id))
            if eng is None:
                return None
            if not eng.health_check():
                del self._m[(model_id, device_id)]
                self._stats["failure"] += 1
                self._evict((model_id, device_id), eng)
                return None
            self._m.move_to_end((model_id, device_id))
            self._stats["hit"] += 1
            return eng

    def remove(self, model_id: int, device_id: int) -> bool:
        with self._lock:
            eng = self._m.pop((model_id, device_id), None)
        if eng is not None:
            self._evict((model_id, device_id), eng)
        return eng is not None

    def __len__(self) -> int:
        return len(self._m)

    def check_health(self) -> int:
        """Evict unhealthy engines; returns how many were removed."""
        bad = []
        with self._lock:
            for k, e in list(self._m.items()):
                if not e.health_check():
                    bad.append((k, self._m.pop(k)))
        for k, e in bad:
            self._evict(k, e)
        return len(bad)

    def start_health_task(self, period_s: float = 10.0) -> None:
        def run():
            while not self._stop.wait(period_s):
                self.check_health()

        self._thread = threading.Thread(target=run, daemon=True, name="kapsl-engine-pool-health")
        self._thread.start()

    def stop(self) -> None:
        self._stop.set()
