"""Device discovery (crates/kapsl-hal/src/device.rs).

Enumerates the CPU and NVIDIA GPUs (NVML through ``nvidia_ml_py`` when it
loads, otherwise ``nvidia-smi --query-gpu`` CSV with an 800 ms timeout).
Results are cached for the process.  ``GpuPreference`` parses ``cuda:1``,
PCI bus ids, name substrings and ``mig:``/``partition:`` ids; ``best_gpu`` picks
the largest memory, then the highest compute capability.

Graphics-API device kinds of the reference (Metal, DirectML, Vulkan, WebGPU,
OpenCL) are unavailable on this box and are not probed; they parse as backend
names only.
"""
from __future__ import annotations

import enum
import functools
import os
import subprocess
from dataclasses import dataclass, field
from typing import Optional


class DeviceBackend(enum.Enum):
    CPU = "cpu"
    CUDA = "cuda"
    ROCM = "rocm"
    METAL = "metal"
    DIRECTML = "directml"
    ONEAPI = "oneapi"
    VULKAN = "vulkan"
    WEBGPU = "webgpu"
    OPENCL = "opencl"


@dataclass
class Device:
    id: int
    name: str
    backend: DeviceBackend
    total_memory_mb: int = 0
    free_memory_mb: int = 0
    compute_capability: Optional[tuple] = None
    pci_bus_id: Optional[str] = None
    partition_id: Optional[str] = None
    sm_count: int = 0


@dataclass
class DeviceInfo:
    cpu_cores: int
    total_memory_mb: int
    devices: list = field(default_factory=list)
    cuda_version: Optional[str] = None
    driver_version: Optional[str] = None

    def gpus(self) -> list:
        return [d for d in self.devices if d.backend is DeviceBackend.CUDA]

    def cuda_devices(self) -> list:
        return self.gpus()

    def _has(self, backend: DeviceBackend) -> bool:
        return any(d.backend is backend for d in self.devices)

    def has_cuda(self) -> bool:
        return self._has(DeviceBackend.CUDA)

    def best_gpu(self) -> Optional[Device]:
        """The accelerator (any backend but the CPU) with the most memory, then the
        highest compute capability (reference device.rs:770-793)."""
        g = [d for d in self.devices if d.backend is not DeviceBackend.CPU]
        if not g:
            return None
        return max(g, key=lambda d: (d.total_memory_mb, d.compute_capability or (0, 0), -d.id))

    def best_gpu_with_preference(self, preference: "GpuPreference") -> Optional[Device]:
        """The first accelerator the preference matches, or None."""
        return next((d for d in self.devices if d.backend is not DeviceBackend.CPU and preference.matches(d)), None)

    def get_best_provider(self) -> str:
        """cuda > metal > rocm > oneapi > directml > cpu over the backends present
        (reference device.rs:807-826)."""
        for b in (DeviceBackend.CUDA, DeviceBackend.METAL, DeviceBackend.ROCM, DeviceBackend.ONEAPI,
                  DeviceBackend.DIRECTML):
            if self._has(b):
                return b.value
        return "cpu"

    def has_provider(self, provider: str) -> bool:
        """Whether an execution provider can run here; ``coreml`` rides on Metal
        and ``cpu`` is always there (reference device.rs:828-850)."""
        key = provider.strip().lower()
        if key == "cpu":
            return True
        if key == "coreml":
            key = "metal"
        return any(d.backend.value == key for d in self.devices)

    def select(self, preference: Optional[str]) -> Optional[Device]:
        p = GpuPreference.parse(preference or "")
        if p is None:
            return self.best_gpu()
        for d in self.devices:
            if p.matches(d):
                return d
        return None


@dataclass
class GpuPreference:
    kind: str
    value: str
    id: int = 0

    @classmethod
    def parse(cls, spec: str) -> Optional["GpuPreference"]:
        s = spec.strip()
        if not s:
            return None
        low = s.lower()
        for pre in ("mig:", "partition:"):
            if low.startswith(pre) and s[len(pre):].strip():
                return cls("partition", s[len(pre):].strip())
        if ":" in low:
            b, _, i = low.partition(":")
            if i.strip().isdigit():
                return cls("backend_id", b.strip(), int(i.strip()))
        if ":" in s and "." in s:
            return cls("pci", s)
        return cls("name", low)

    def matches(self, d: Device) -> bool:
        if self.kind == "backend_id":
            return d.backend.value == self.value and d.id == self.id
        if self.kind == "pci":
            return (d.pci_bus_id or "").lower() == self.value.lower()
        if self.kind == "name":
            return self.value in d.name.lower()
        return (d.partition_id or "").lower() == self.value.lower()


def _mem_total_mb() -> int:
    try:
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemTotal:"):
                    return int(line.split()[1]) // 1024
    except OSError:
        pass
    return 0


def _probe_nvml() -> Optional[list]:
    try:
        import pynvml as nv  # from nvidia_ml_py
    except Exception:
        return None
    try:
        nv.nvmlInit()
    except Exception:
        return None
    out = []
    try:
        for i in range(nv.nvmlDeviceGetCount()):
            h = nv.nvmlDeviceGetHandleByIndex(i)
            mem = nv.nvmlDeviceGetMemoryInfo(h)
            name = nv.nvmlDeviceGetName(h)
            name = name.decode() if isinstance(name, bytes) else name
            try:
                cc = nv.nvmlDeviceGetCudaComputeCapability(h)
            except Exception:
                cc = None
            try:
                pci = nv.nvmlDeviceGetPciInfo(h).busId
                pci = pci.decode() if isinstance(pci, bytes) else pci
            except Exception:
                pci = None
            out.append(Device(i, name, DeviceBackend.CUDA, mem.total // (1 << 20), mem.free // (1 << 20),
                              tuple(cc) if cc else None, pci))
    finally:
        try:
            nv.nvmlShutdown()
        except Exception:
            pass
    return out


def _probe_nvidia_smi() -> list:
    try:
        r = subprocess.run(["nvidia-smi", "--query-gpu=index,name,memory.total,memory.free,pci.bus_id,compute_cap",
                            "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=0.8)
    except (OSError, subprocess.TimeoutExpired):
        return []
    out = []
    for line in r.stdout.strip().splitlines():
        p = [x.strip() for x in line.split(",")]
        if len(p) < 6:
            continue
        try:
            cc = tuple(int(x) for x in p[5].split(".")) if p[5] and p[5][0].isdigit() else None
            out.append(Device(int(p[0]), p[1], DeviceBackend.CUDA, int(float(p[2])), int(float(p[3])), cc, p[4]))
        except ValueError:
            continue
    return out


@functools.lru_cache(maxsize=1)
def probe() -> DeviceInfo:
    cpu = Device(0, "cpu", DeviceBackend.CPU, _mem_total_mb(), 0)
    gpus = _probe_nvml()
    if gpus is None:
        gpus = _probe_nvidia_smi()
    cuda = None
    try:
        import torch

        cuda = torch.version.cuda
        if gpus and torch.cuda.is_available():
            for g in gpus:
                if g.id < torch.cuda.device_count():
                    g.sm_count = torch.cuda.get_device_properties(g.id).multi_processor_count
    except Exception:
        pass
    return DeviceInfo(cpu_cores=os.cpu_count() or 1, total_memory_mb=cpu.total_memory_mb, devices=[cpu] + gpus,
                      cuda_version=cuda)
