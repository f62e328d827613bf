"""ONNX graph optimizer.

``GraphOptimizer(config).optimize(input_path, output_path)`` loads a model
with the package's protobuf decoder (:mod:`kapsl_sdk_b200.loaders.onnx`),
applies the enabled passes and writes the result:

* constant folding — nodes whose inputs are all initializers are evaluated
  once with the ONNX interpreter and become initializers;
* operator fusion — Identity / Dropout nodes are bypassed and back-to-back
  Transposes whose permutations compose to the identity are removed;
* dead-code elimination — nodes and initializers that no graph output
  depends on are dropped.

A model whose attributes the writer cannot encode (strings, graphs, tensor
attributes that are not folded) is copied unchanged and the report says so.
The reference ships the same API with every pass a no-op and ``save``
copying the file (crates/kapsl-optimizer/src/{graph.rs:4-78, optimizer.rs,
config.rs}); here the passes do the work.
"""
from __future__ import annotations

import shutil
import time
from dataclasses import dataclass, field
from typing import Optional

import numpy as np

LEVELS = ("O0", "O1", "O2", "O3")


@dataclass
class OptimizationConfig:
    level: str = "O1"
    enable_fusion: bool = True
    enable_constant_folding: bool = True
    enable_dead_code_elimination: bool = True
    enable_shape_inference: bool = True
    target_backend: Optional[str] = None
    custom_passes: list = field(default_factory=list)

    def __post_init__(self):
        self.level = self.level.upper()
        if self.level not in LEVELS:
            raise ValueError(f"Invalid optimization level: {self.level}")
        if self.level == "O0":
            self.enable_fusion = self.enable_constant_folding = self.enable_dead_code_elimination = False


@dataclass
class OptimizationReport:
    original_nodes: int
    optimized_nodes: int
    applied_passes: list
    duration_ms: float
    copied_unchanged: bool = False

    @property
    def nodes_removed(self) -> int:
        return self.original_nodes - self.optimized_nodes


class _Pass:
    name = "pass"

    def apply(self, m) -> bool:
        raise NotImplementedError


class ConstantFoldingPass(_Pass):
    name = "constant_folding"

    def apply(self, m) -> bool:
        import torch

        from ..loaders.onnx import OnnxGraph

        changed = False
        keep = []
        interp = None
        for n in m.nodes:
            ins = [i for i in n.inputs if i]
            foldable = n.op in OnnxGraph.SUPPORTED and n.op not in ("Shape", "Dropout") and \
                ((ins and all(i in m.initializers for i in ins)) or (n.op == "Constant" and "value" in n.attrs))
            if not foldable:
                keep.append(n)
                continue
            if interp is None:
                interp = OnnxGraph.__new__(OnnxGraph)
                interp.device = torch.device("cpu")
            args = [torch.from_numpy(np.ascontiguousarray(m.initializers[i])) if i else None for i in n.inputs]
            try:
                out = interp._op(n, args)
            except Exception:
                keep.append(n)
                continue
            outs = out if isinstance(out, (list, tuple)) else [out]
            for name, v in zip(n.outputs, outs):
                m.initializers[name] = v.detach().cpu().numpy() if hasattr(v, "detach") else np.asarray(v)
            changed = True
        m.nodes = keep
        return changed


class OperatorFusionPass(_Pass):
    name = "operator_fusion"

    def apply(self, m) -> bool:
        changed = False
        rename = {}
        keep = []
        producers = {}
        for n in m.nodes:
            n.inputs = [rename.get(i, i) for i in n.inputs]
            if n.op in ("Identity", "Dropout") and n.inputs and n.outputs[0] not in m.outputs:
                rename[n.outputs[0]] = n.inputs[0]
                changed = True
                continue
            if n.op == "Transpose" and n.inputs[0] in producers and producers[n.inputs[0]].op == "Transpose" \
                    and n.outputs[0] not in m.outputs:
                p1 = list(producers[n.inputs[0]].attrs.get("perm", []))
                p2 = list(n.attrs.get("perm", []))
                if p1 and len(p1) == len(p2) and [p1[i] for i in p2] == list(range(len(p1))):
                    rename[n.outputs[0]] = producers[n.inputs[0]].inputs[0]
                    changed = True
                    continue
            keep.append(n)
            for o in n.outputs:
                producers[o] = n
        m.nodes = keep
        m.outputs = [rename.get(o, o) for o in m.outputs]
        return changed


class DeadCodeEliminationPass(_Pass):
    name = "dead_code_elimination"

    def apply(self, m) -> bool:
        needed = set(m.outputs)
        keep = []
        for n in reversed(m.nodes):
            if any(o in needed for o in n.outputs):
                keep.append(n)
                needed.update(i for i in n.inputs if i)
        keep.reverse()
        inits = {k: v for k, v in m.initializers.items() if k in needed}
        changed = len(keep) != len(m.nodes) or len(inits) != len(m.initializers)
        m.nodes, m.initializers = keep, inits
        return changed


def _encodable(m) -> bool:
    for n in m.nodes:
        for v in n.attrs.values():
            if isinstance(v, bool) or not isinstance(v, (int, float, list, tuple)):
                return False
            if isinstance(v, (list, tuple)) and not all(isinstance(i, int) for i in v):
                return False
    return all(np.asarray(v).dtype in (np.float32, np.int64, np.int32, np.float16) for v in m.initializers.values())


class GraphOptimizer:
    def __init__(self, config: Optional[OptimizationConfig] = None):
        self.config = config or OptimizationConfig()
        c = self.config
        self.passes = []
        if c.enable_constant_folding:
            self.passes.append(ConstantFoldingPass())
        if c.enable_fusion:
            self.passes.append(OperatorFusionPass())
        if c.enable_dead_code_elimination:
            self.passes.append(DeadCodeEliminationPass())

    def optimize_model(self, m) -> list:
        applied = []
        for p in self.passes:
            if p.apply(m):
                applied.append(p.name)
        return applied

    def optimize(self, input_path: str, output_path: str) -> OptimizationReport:
        from ..loaders.onnx import encode_model, read_model

        t0 = time.perf_counter()
        m = read_model(input_path)
        n0 = len(m.nodes)
        applied = self.optimize_model(m)
        copied = False
        if _encodable(m):
            with open(output_path, "wb") as f:
                f.write(encode_model(m.nodes, m.inputs, m.outputs, m.initializers, m.opset))
        else:
            shutil.copyfile(input_path, output_path)
            copied, applied = True, []
        return OptimizationReport(n0, n0 if copied else len(m.nodes), applied, (time.perf_counter() - t0) * 1e3,
                                  copied)
