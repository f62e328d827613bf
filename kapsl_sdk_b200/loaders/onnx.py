"""ONNX models without ONNX Runtime.

No ``onnx`` / ``onnxruntime`` package exists here, so this module decodes the
protobuf wire format of ``ModelProto`` directly (varints and length-delimited
fields; field numbers from the public onnx.proto) and provides:

* ``read_model`` -> graph nodes, inputs/outputs, initializers as numpy arrays
  (raw_data or typed repeated fields; external data files next to the model);
* ``OnnxGraph`` -> a PyTorch interpreter for an explicitly scoped op subset
  (MatMul, Gemm, Add, Sub, Mul, Div, Relu, Sigmoid, Tanh, Softmax, Reshape,
  Flatten, Transpose, Identity, Constant, Conv, MaxPool, AveragePool,
  GlobalAveragePool, Concat, Gather, Unsqueeze, Squeeze, Cast, Erf, Sqrt, Pow,
  ReduceMean, LayerNormalization, Shape, Slice).  Graphs using other ops are
  rejected at load time with the op names listed;
* ``load_onnx_llm`` -> LLM weights from initializers named like a HF
  checkpoint (``model.layers.{i}.self_attn.q_proj.weight`` ...), the way an
  ONNX export of a decoder keeps them.

Reference: the reference serves any ONNX graph through ONNX Runtime
(crates/kapsl-backends/src/onnx.rs) and LLM exports through ORT sessions.
"""
from __future__ import annotations

import os
import struct
from dataclasses import dataclass, field
from typing import Optional

import numpy as np
import torch

# TensorProto.DataType
_NP = {1: np.float32, 2: np.uint8, 3: np.int8, 4: np.uint16, 5: np.int16, 6: np.int32, 7: np.int64, 9: np.bool_,
       10: np.float16, 11: np.float64, 12: np.uint32, 13: np.uint64}
BFLOAT16 = 16


def _varint(b: bytes, i: int):
    shift = v = 0
    while True:
        x = b[i]
        i += 1
        v |= (x & 0x7F) << shift
        if x < 0x80:
            return v, i
        shift += 7


def _fields(b: bytes):
    """Yields (field_number, wire_type, value) over one message."""
    i, n = 0, len(b)
    while i < n:
        key, i = _varint(b, i)
        f, wt = key >> 3, key & 7
        if wt == 0:
            v, i = _varint(b, i)
        elif wt == 1:
            v = b[i:i + 8]
            i += 8
        elif wt == 2:
            ln, i = _varint(b, i)
            v = b[i:i + ln]
            i += ln
        elif wt == 5:
            v = b[i:i + 4]
            i += 4
        else:
            raise ValueError(f"unsupported protobuf wire type {wt}")
        yield f, wt, v


def _packed_varints(v, wt):
    if wt == 0:
        return [v]
    out, i = [], 0
    while i < len(v):
        x, i = _varint(v, i)
        out.append(x)
    return out


def _signed64(x: int) -> int:
    return x - (1 << 64) if x >= 1 << 63 else x


@dataclass
class Node:
    op: str
    inputs: list
    outputs: list
    name: str = ""
    attrs: dict = field(default_factory=dict)


@dataclass
class OnnxModel:
    nodes: list
    inputs: list
    outputs: list
    initializers: dict
    opset: int = 13


def _tensor(b: bytes, base_dir: Optional[str]) -> tuple:
    dims, dtype, name, raw = [], 1, "", None
    floats, int32s, int64s, doubles = [], [], [], []
    ext = {}
    for f, wt, v in _fields(b):
        if f == 1:
            dims += [_signed64(x) for x in _packed_varints(v, wt)]
        elif f == 2:
            dtype = v
        elif f == 4:
            floats += list(struct.unpack(f"<{len(v) // 4}f", v)) if wt == 2 else [struct.unpack("<f", v)[0]]
        elif f == 5:
            int32s += [_signed64(x) for x in _packed_varints(v, wt)]
        elif f == 7:
            int64s += [_signed64(x) for x in _packed_varints(v, wt)]
        elif f == 8:
            name = v.decode()
        elif f == 9:
            raw = bytes(v)
        elif f == 10:
            doubles += list(struct.unpack(f"<{len(v) // 8}d", v)) if wt == 2 else [struct.unpack("<d", v)[0]]
        elif f == 13:
            k = val = None
            for ff, _, vv in _fields(v):
                if ff == 1:
                    k = vv.decode()
                elif ff == 2:
                    val = vv.decode()
            ext[k] = val
    if ext.get("location"):
        with open(os.path.join(base_dir or ".", ext["location"]), "rb") as fh:
            fh.seek(int(ext.get("offset", 0)))
            ln = ext.get("length")
            raw = fh.read(int(ln)) if ln else fh.read()
    if dtype == BFLOAT16:
        u16 = np.frombuffer(raw, np.uint16) if raw is not None else np.asarray(int32s, np.uint16)
        arr = (u16.astype(np.uint32) << 16).view(np.float32)
    elif raw is not None:
        arr = np.frombuffer(raw, _NP[dtype]).copy()
    elif dtype in (1,):
        arr = np.asarray(floats, np.float32)
    elif dtype == 11:
        arr = np.asarray(doubles, np.float64)
    elif dtype == 7:
        arr = np.asarray(int64s, np.int64)
    elif dtype == 10:
        arr = np.asarray(int32s, np.uint16).view(np.float16)
    else:
        arr = np.asarray(int32s, _NP.get(dtype, np.int32))
    return name, arr.reshape(dims) if dims else arr.reshape(())


def _attr(b: bytes, base_dir):
    name, val, kind = "", None, None
    ints, floats, strs = [], [], []
    for f, wt, v in _fields(b):
        if f == 1:
            name = v.decode()
        elif f == 2:
            val = struct.unpack("<f", v)[0]
        elif f == 3:
            val = _signed64(v)
        elif f == 4:
            val = v.decode(errors="replace")
        elif f == 5:
            val = _tensor(v, base_dir)[1]
        elif f == 7:
            floats += list(struct.unpack(f"<{len(v) // 4}f", v)) if wt == 2 else [struct.unpack("<f", v)[0]]
        elif f == 8:
            ints += [_signed64(x) for x in _packed_varints(v, wt)]
        elif f == 9:
            strs.append(v.decode(errors="replace"))
        elif f == 20:
            kind = v
    if ints:
        val = ints
    elif floats:
        val = floats
    elif strs:
        val = strs
    return name, val


def _value_info_name(b: bytes) -> str:
    for f, _, v in _fields(b):
        if f == 1:
            return v.decode()
    return ""


def read_model(path: str) -> OnnxModel:
    with open(path, "rb") as fh:
        data = fh.read()
    base = os.path.dirname(os.path.abspath(path))
    graph = None
    opset = 13
    for f, _, v in _fields(data):
        if f == 7:
            graph = v
        elif f == 8:
            for ff, _, vv in _fields(v):
                if ff == 2:
                    opset = vv
    if graph is None:
        raise ValueError("ONNX file has no graph")
    nodes, inputs, outputs, inits = [], [], [], {}
    for f, _, v in _fields(graph):
        if f == 1:
            n = Node("", [], [])
            for ff, _, vv in _fields(v):
                if ff == 1:
                    n.inputs.append(vv.decode())
                elif ff == 2:
                    n.outputs.append(vv.decode())
                elif ff == 3:
                    n.name = vv.decode()
                elif ff == 4:
                    n.op = vv.decode()
                elif ff == 5:
                    k, a = _attr(vv, base)
                    n.attrs[k] = a
            nodes.append(n)
        elif f == 5:
            k, a = _tensor(v, base)
            inits[k] = a
        elif f == 11:
            inputs.append(_value_info_name(v))
        elif f == 12:
            outputs.append(_value_info_name(v))
    inputs = [i for i in inputs if i not in inits]
    return OnnxModel(nodes, inputs, outputs, inits, opset)


# ---------------------------------------------------------- interpreter
def _conv_pads(a, nd):
    p = a.get("pads") or [0] * (2 * nd)
    return p[:nd], p[nd:]


class OnnxGraph:
    SUPPORTED = {"MatMul", "Gemm", "Add", "Sub", "Mul", "Div", "Relu", "Sigmoid", "Tanh", "Softmax", "Reshape",
                 "Flatten", "Transpose", "Identity", "Constant", "Conv", "MaxPool", "AveragePool",
                 "GlobalAveragePool", "Concat", "Gather", "Unsqueeze", "Squeeze", "Cast", "Erf", "Sqrt", "Pow",
                 "ReduceMean", "LayerNormalization", "Shape", "Slice", "Dropout", "BatchNormalization",
                 # elementwise
                 "Exp", "Log", "Neg", "Abs", "Reciprocal", "Floor", "Ceil", "Round", "Sign", "Sin", "Cos", "Not",
                 "IsNaN", "Softplus", "Softsign", "Elu", "Selu", "LeakyRelu", "HardSigmoid", "HardSwish", "Gelu",
                 "Clip", "PRelu", "Max", "Min", "Sum", "Mean", "Equal", "Less", "Greater", "LessOrEqual",
                 "GreaterOrEqual", "And", "Or", "Xor", "Mod", "Where", "LogSoftmax",
                 # shapes
                 "Expand", "Tile", "Split", "Pad", "ConstantOfShape", "Range", "Size", "Resize", "Trilu", "CumSum",
                 # reductions / selection
                 "ReduceSum", "ReduceMax", "ReduceMin", "ReduceProd", "ReduceL2", "ArgMax", "ArgMin", "TopK",
                 # layers
                 "InstanceNormalization", "ConvTranspose", "Einsum", "GlobalMaxPool",
                 # indexing, quantization, normalization
                 "GatherElements", "ScatterElements", "ScatterND", "GatherND", "OneHot", "NonZero",
                 "DepthToSpace", "SpaceToDepth", "QuantizeLinear", "DequantizeLinear", "GroupNormalization",
                 "LpNormalization", "ReduceLogSumExp", "ReduceSumSquare", "ReduceL1", "Mish", "Celu",
                 "ThresholdedRelu", "Shrink", "Compress", "BitShift"}

    def __init__(self, model: OnnxModel, device="cpu"):
        bad = sorted({n.op for n in model.nodes} - self.SUPPORTED)
        if bad:
            raise ValueError(f"unsupported ONNX ops: {', '.join(bad)}")
        self.m = model
        self.device = torch.device(device)
        self.consts = {k: torch.from_numpy(np.ascontiguousarray(v)).to(self.device) for k, v in model.initializers.items()}

    def run(self, feeds: dict) -> dict:
        env = dict(self.consts)
        for k, v in feeds.items():
            env[k] = v if isinstance(v, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(v))
            env[k] = env[k].to(self.device)
        for n in self.m.nodes:
            args = [env[i] if i else None for i in n.inputs]
            outs = self._op(n, args)
            if not isinstance(outs, (list, tuple)):
                outs = [outs]
            for name, val in zip(n.outputs, outs):
                env[name] = val
        return {o: env[o] for o in self.m.outputs}

    def _op(self, n: Node, x: list):
        a, op = n.attrs, n.op
        F = torch.nn.functional
        if op == "MatMul":
            return torch.matmul(x[0], x[1])
        if op == "Gemm":
            A = x[0].T if a.get("transA") else x[0]
            B = x[1].T if a.get("transB") else x[1]
            y = a.get("alpha", 1.0) * (A @ B)
            if len(x) > 2 and x[2] is not None:
                y = y + a.get("beta", 1.0) * x[2]
            return y
        if op in ("Add", "Sub", "Mul", "Div", "Pow"):
            f = {"Add": torch.add, "Sub": torch.sub, "Mul": torch.mul, "Div": torch.div, "Pow": torch.pow}[op]
            return f(x[0], x[1])
        if op == "Relu":
            return torch.relu(x[0])
        if op == "Sigmoid":
            return torch.sigmoid(x[0])
        if op == "Tanh":
            return torch.tanh(x[0])
        if op == "Erf":
            return torch.erf(x[0])
        if op == "Sqrt":
            return torch.sqrt(x[0])
        if op == "Softmax":
            return torch.softmax(x[0], dim=a.get("axis", -1))
        if op in ("Identity", "Dropout"):
            return x[0]
        if op == "Constant":
            v = a.get("value")
            return torch.from_numpy(np.ascontiguousarray(v)).to(self.device)
        if op == "Reshape":
            shape = [int(s) for s in x[1].tolist()]
            shape = [x[0].shape[i] if s == 0 else s for i, s in enumerate(shape)]
            return x[0].reshape(shape)
        if op == "Flatten":
            ax = a.get("axis", 1)
            return x[0].reshape(int(np.prod(x[0].shape[:ax])) if ax else 1, -1)
        if op == "Transpose":
            perm = a.get("perm") or list(reversed(range(x[0].dim())))
            return x[0].permute(*perm)
        if op == "Conv":
            nd = x[1].dim() - 2
            lo, hi = _conv_pads(a, nd)
            xin = F.pad(x[0], [p for pair in zip(reversed(lo), reversed(hi)) for p in pair]) if any(lo + hi) else x[0]
            fn = {1: F.conv1d, 2: F.conv2d, 3: F.conv3d}[nd]
            return fn(xin, x[1], x[2] if len(x) > 2 else None, stride=a.get("strides") or 1,
                      dilation=a.get("dilations") or 1, groups=a.get("group", 1))
        if op in ("MaxPool", "AveragePool"):
            nd = x[0].dim() - 2
            lo, hi = _conv_pads(a, nd)
            xin = F.pad(x[0], [p for pair in zip(reversed(lo), reversed(hi)) for p in pair],
                        value=float("-inf") if op == "MaxPool" else 0.0) if any(lo + hi) else x[0]
            k = a["kernel_shape"]
            s = a.get("strides") or k
            fn = getattr(F, ("max" if op == "MaxPool" else "avg") + f"_pool{nd}d")
            return fn(xin, k, s)
        if op == "GlobalAveragePool":
            return x[0].mean(dim=tuple(range(2, x[0].dim())), keepdim=True)
        if op == "BatchNormalization":
            return F.batch_norm(x[0], x[3], x[4], x[1], x[2], False, 0.0, a.get("epsilon", 1e-5))
        if op == "Concat":
            return torch.cat(x, dim=a.get("axis", 0))
        if op == "Gather":
            return torch.index_select(x[0], a.get("axis", 0), x[1].long().flatten()).reshape(
                *x[0].shape[:a.get("axis", 0)], *x[1].shape, *x[0].shape[a.get("axis", 0) + 1:])
        if op in ("Unsqueeze", "Squeeze"):
            axes = a.get("axes") if "axes" in a else (x[1].tolist() if len(x) > 1 and x[1] is not None else None)
            y = x[0]
            if op == "Unsqueeze":
                for ax in sorted(axes):
                    y = y.unsqueeze(ax)
                return y
            return y.squeeze() if axes is None else y.squeeze(tuple(axes))
        if op == "Cast":
            to = a["to"]
            return x[0].to({1: torch.float32, 6: torch.int32, 7: torch.int64, 10: torch.float16, 11: torch.float64,
                            9: torch.bool, 16: torch.bfloat16}.get(to, torch.float32))
        if op == "ReduceMean":
            axes = a.get("axes") or (x[1].tolist() if len(x) > 1 and x[1] is not None else None)
            return x[0].mean(dim=tuple(axes) if axes else None, keepdim=bool(a.get("keepdims", 1)))
        if op == "LayerNormalization":
            ax = a.get("axis", -1)
            shape = x[0].shape[ax:]
            return F.layer_norm(x[0], shape, x[1], x[2] if len(x) > 2 else None, a.get("epsilon", 1e-5))
        if op == "Shape":
            return torch.tensor(list(x[0].shape), dtype=torch.int64, device=self.device)
        if op == "Slice":
            starts, ends = x[1].tolist(), x[2].tolist()
            axes = x[3].tolist() if len(x) > 3 and x[3] is not None else list(range(len(starts)))
            steps = x[4].tolist() if len(x) > 4 and x[4] is not None else [1] * len(starts)
            sl = [slice(None)] * x[0].dim()
            for s, e, ax, st in zip(starts, ends, axes, steps):
                sl[ax] = slice(s, e if e < (1 << 62) else None, st)
            return x[0][tuple(sl)]
        return self._op_more(n, x)

    def _op_more(self, n: Node, x: list):
        """Operators beyond the core set (opset 13+ semantics: axes / k / pads
        arrive as inputs where that opset moved them there)."""
        a, op = n.attrs, n.op
        F = torch.nn.functional
        unary = {"Exp": torch.exp, "Log": torch.log, "Neg": torch.neg, "Abs": torch.abs,
                 "Reciprocal": torch.reciprocal, "Floor": torch.floor, "Ceil": torch.ceil, "Round": torch.round,
                 "Sign": torch.sign, "Sin": torch.sin, "Cos": torch.cos, "Not": torch.logical_not,
                 "IsNaN": torch.isnan, "Softplus": F.softplus, "Softsign": F.softsign}
        if op in unary:
            return unary[op](x[0])
        if op == "Elu":
            return F.elu(x[0], alpha=a.get("alpha", 1.0))
        if op == "Selu":
            al, ga = a.get("alpha", 1.67326319217681884765625), a.get("gamma", 1.05070102214813232421875)
            return ga * torch.where(x[0] > 0, x[0], al * (torch.exp(x[0]) - 1))
        if op == "LeakyRelu":
            return F.leaky_relu(x[0], a.get("alpha", 0.01))
        if op == "HardSigmoid":
            return torch.clamp(a.get("alpha", 0.2) * x[0] + a.get("beta", 0.5), 0.0, 1.0)
        if op == "HardSwish":
            return x[0] * torch.clamp(x[0] / 6 + 0.5, 0.0, 1.0)
        if op == "Gelu":
            ap = a.get("approximate", "none")
            return F.gelu(x[0], approximate=ap.decode() if isinstance(ap, bytes) else ap)
        if op == "Clip":
            lo = x[1] if len(x) > 1 and x[1] is not None else a.get("min")
            hi = x[2] if len(x) > 2 and x[2] is not None else a.get("max")
            y = x[0]
            if lo is not None:
                y = torch.maximum(y, torch.as_tensor(lo, dtype=y.dtype, device=y.device))
            if hi is not None:
                y = torch.minimum(y, torch.as_tensor(hi, dtype=y.dtype, device=y.device))
            return y
        if op == "PRelu":
            return torch.where(x[0] >= 0, x[0], x[0] * x[1])
        if op in ("Max", "Min", "Sum", "Mean"):
            y = x[0]
            for z in x[1:]:
                y = {"Max": torch.maximum, "Min": torch.minimum}.get(op, torch.add)(y, z)
            return y / len(x) if op == "Mean" else y
        cmp = {"Equal": torch.eq, "Less": torch.lt, "Greater": torch.gt, "LessOrEqual": torch.le,
               "GreaterOrEqual": torch.ge, "And": torch.logical_and, "Or": torch.logical_or,
               "Xor": torch.logical_xor}
        if op in cmp:
            return cmp[op](x[0], x[1])
        if op == "Mod":
            return torch.fmod(x[0], x[1]) if a.get("fmod", 0) else torch.remainder(x[0], x[1])
        if op == "Where":
            return torch.where(x[0].bool(), x[1], x[2])
        if op == "LogSoftmax":
            return torch.log_softmax(x[0], dim=a.get("axis", -1))
        if op == "Expand":
            shape = [int(v) for v in x[1].tolist()]
            nd = max(len(shape), x[0].dim())
            src = [1] * (nd - x[0].dim()) + list(x[0].shape)
            shape = [1] * (nd - len(shape)) + shape
            out = [max(s, t) if s == 1 or t == 1 else t for s, t in zip(src, shape)]
            return x[0].reshape(src).expand(out)
        if op == "Tile":
            return x[0].repeat(*[int(v) for v in x[1].tolist()])
        if op == "Split":
            ax = a.get("axis", 0)
            if len(x) > 1 and x[1] is not None:
                sizes = [int(v) for v in x[1].tolist()]
            elif a.get("split"):
                sizes = list(a["split"])
            else:
                k = a.get("num_outputs", len(n.outputs))
                d = x[0].shape[ax]
                sizes = [-(-d // k)] * (k - 1) + [d - -(-d // k) * (k - 1)]
            return list(torch.split(x[0], sizes, dim=ax))
        if op == "Pad":
            pads = [int(v) for v in (x[1].tolist() if len(x) > 1 and x[1] is not None else a.get("pads", []))]
            value = float(x[2].item()) if len(x) > 2 and x[2] is not None else float(a.get("value", 0.0))
            nd = x[0].dim()
            axes = ([int(v) for v in x[3].tolist()] if len(x) > 3 and x[3] is not None else list(range(nd)))
            axes = [ax % nd for ax in axes]
            full = [0] * (2 * nd)
            for i, ax in enumerate(axes):
                full[ax], full[nd + ax] = pads[i], pads[len(axes) + i]
            tp = []
            for ax in reversed(range(nd)):
                tp += [full[ax], full[nd + ax]]
            mode = a.get("mode", "constant")
            mode = mode.decode() if isinstance(mode, bytes) else mode
            if mode == "constant":
                return F.pad(x[0], tp, value=value)
            if mode not in ("reflect", "edge"):
                raise ValueError(f"Pad mode {mode!r} is not supported")
            pairs = [(full[ax], full[nd + ax]) for ax in range(nd)]
            return torch.from_numpy(np.pad(x[0].cpu().numpy(), pairs, mode=mode)).to(self.device)
        if op == "ConstantOfShape":
            v = a.get("value")
            arr = np.asarray(v if v is not None else np.zeros(1, np.float32)).reshape(-1)
            return torch.full([int(s) for s in x[0].tolist()], arr[0].item(),
                              dtype=torch.from_numpy(arr[:1].copy()).dtype, device=self.device)
        if op == "Range":
            return torch.arange(x[0].item(), x[1].item(), x[2].item(), device=self.device).to(x[0].dtype)
        if op == "Size":
            return torch.tensor(x[0].numel(), dtype=torch.int64, device=self.device)
        if op == "Resize":
            mode = a.get("mode", "nearest")
            mode = mode.decode() if isinstance(mode, bytes) else mode
            sizes = x[3] if len(x) > 3 and x[3] is not None and x[3].numel() else None
            scales = x[2] if len(x) > 2 and x[2] is not None and x[2].numel() else None
            if sizes is not None:
                out = [int(v) for v in sizes.tolist()][2:]
                kw = {"size": out}
            else:
                kw = {"scale_factor": [float(v) for v in scales.tolist()][2:]}
            if mode == "nearest":
                return F.interpolate(x[0], mode="nearest", **kw)
            ctm = a.get("coordinate_transformation_mode", "half_pixel")
            ctm = ctm.decode() if isinstance(ctm, bytes) else ctm
            lin = {3: "linear", 4: "bilinear", 5: "trilinear"}[x[0].dim()]
            return F.interpolate(x[0], mode=lin, align_corners=ctm == "align_corners", **kw)
        if op == "Trilu":
            k = int(x[1].item()) if len(x) > 1 and x[1] is not None else 0
            return torch.triu(x[0], k) if a.get("upper", 1) else torch.tril(x[0], k)
        if op == "CumSum":
            ax = int(x[1].item())
            y = x[0].flip(ax) if a.get("reverse", 0) else x[0]
            c = torch.cumsum(y, ax)
            if a.get("exclusive", 0):
                c = c - y
            return c.flip(ax) if a.get("reverse", 0) else c
        if op in ("ReduceSum", "ReduceMax", "ReduceMin", "ReduceProd", "ReduceL2"):
            axes = a.get("axes") or (x[1].tolist() if len(x) > 1 and x[1] is not None else None)
            keep = bool(a.get("keepdims", 1))
            if not axes:
                if a.get("noop_with_empty_axes", 0) and op == "ReduceSum":
                    return x[0]
                axes = list(range(x[0].dim()))
            y = x[0]
            if op == "ReduceSum":
                return y.sum(dim=tuple(axes), keepdim=keep)
            if op == "ReduceL2":
                return y.pow(2).sum(dim=tuple(axes), keepdim=keep).sqrt()
            for ax in sorted((ax % y.dim() for ax in axes), reverse=True):
                y = {"ReduceMax": lambda t: t.amax(ax, keepdim=True), "ReduceMin": lambda t: t.amin(ax, keepdim=True),
                     "ReduceProd": lambda t: t.prod(ax, keepdim=True)}[op](y)
            if not keep:
                for ax in sorted((ax % x[0].dim() for ax in axes), reverse=True):
                    y = y.squeeze(ax)
            return y
        if op in ("ArgMax", "ArgMin"):
            ax, keep = a.get("axis", 0), bool(a.get("keepdims", 1))
            y = x[0].flip(ax) if a.get("select_last_index", 0) else x[0]
            r = (torch.argmax if op == "ArgMax" else torch.argmin)(y, dim=ax, keepdim=keep)
            return (y.shape[ax] - 1 - r) if a.get("select_last_index", 0) else r
        if op == "TopK":
            k = int(x[1].reshape(-1)[0].item())
            v, i = torch.topk(x[0], k, dim=a.get("axis", -1), largest=bool(a.get("largest", 1)),
                              sorted=bool(a.get("sorted", 1)))
            return [v, i]
        if op == "InstanceNormalization":
            return F.instance_norm(x[0], weight=x[1], bias=x[2], eps=a.get("epsilon", 1e-5))
        if op == "GlobalMaxPool":
            return x[0].amax(dim=tuple(range(2, x[0].dim())), keepdim=True)
        if op == "ConvTranspose":
            nd = x[1].dim() - 2
            lo, hi = _conv_pads(a, nd)
            if lo != hi:
                raise ValueError("ConvTranspose with asymmetric pads is not supported")
            fn = {1: F.conv_transpose1d, 2: F.conv_transpose2d, 3: F.conv_transpose3d}[nd]
            return fn(x[0], x[1], x[2] if len(x) > 2 else None, stride=a.get("strides") or 1, padding=lo,
                      output_padding=a.get("output_padding") or 0, groups=a.get("group", 1),
                      dilation=a.get("dilations") or 1)
        if op == "Einsum":
            eq = a["equation"]
            return torch.einsum(eq.decode() if isinstance(eq, bytes) else eq, *x)
        return self._op_extra(n, x)

    def _op_extra(self, n: Node, x: list):
        """Indexing, quantization and normalization operators (opset 13+ semantics)."""
        a, op = n.attrs, n.op
        F = torch.nn.functional
        if op == "GatherElements":
            ax = a.get("axis", 0)
            idx = x[1].long()
            idx = torch.where(idx < 0, idx + x[0].shape[ax], idx)
            return torch.gather(x[0], ax, idx)
        if op == "ScatterElements":
            ax, red = a.get("axis", 0), a.get("reduction", b"none")
            red = red.decode() if isinstance(red, bytes) else red
            idx = x[1].long()
            idx = torch.where(idx < 0, idx + x[0].shape[ax], idx)
            if red == "none":
                return x[0].scatter(ax, idx, x[2])
            return x[0].scatter_reduce(ax, idx, x[2], {"add": "sum", "mul": "prod", "max": "amax",
                                                        "min": "amin"}[red], include_self=True)
        if op == "ScatterND":
            y = x[0].clone()
            idx = x[1].long()
            k = idx.shape[-1]
            flat_idx = idx.reshape(-1, k)
            upd = x[2].reshape(flat_idx.shape[0], *x[0].shape[k:])
            for i in range(flat_idx.shape[0]):
                y[tuple(flat_idx[i].tolist())] = upd[i]
            return y
        if op == "GatherND":
            b = a.get("batch_dims", 0)
            if b:
                raise ValueError("GatherND with batch_dims is not supported")
            idx = x[1].long()
            k = idx.shape[-1]
            flat = idx.reshape(-1, k)
            out = torch.stack([x[0][tuple(r.tolist())] for r in flat]) if flat.shape[0] else \
                x[0].new_zeros((0, *x[0].shape[k:]))
            return out.reshape(*idx.shape[:-1], *x[0].shape[k:])
        if op == "OneHot":
            depth = int(x[1].reshape(-1)[0].item())
            vals = x[2].reshape(-1)
            idx = x[0].long()
            idx = torch.where(idx < 0, idx + depth, idx)
            valid = ((idx >= 0) & (idx < depth)).unsqueeze(-1)
            oh = (F.one_hot(idx.clamp(0, depth - 1), depth) * valid).to(vals.dtype)
            y = vals[0] + oh * (vals[1] - vals[0])
            ax = a.get("axis", -1)
            return y if ax in (-1, y.dim() - 1) else torch.movedim(y, -1, ax)
        if op == "NonZero":
            return torch.nonzero(x[0]).T.contiguous()
        if op in ("DepthToSpace", "SpaceToDepth"):
            bs = a["blocksize"]
            N, C, H, W = x[0].shape
            if op == "SpaceToDepth":
                y = x[0].reshape(N, C, H // bs, bs, W // bs, bs).permute(0, 3, 5, 1, 2, 4)
                return y.reshape(N, C * bs * bs, H // bs, W // bs)
            mode = a.get("mode", b"DCR")
            mode = mode.decode() if isinstance(mode, bytes) else mode
            if mode == "DCR":
                y = x[0].reshape(N, bs, bs, C // (bs * bs), H, W).permute(0, 3, 4, 1, 5, 2)
            else:
                y = x[0].reshape(N, C // (bs * bs), bs, bs, H, W).permute(0, 1, 4, 2, 5, 3)
            return y.reshape(N, C // (bs * bs), H * bs, W * bs)
        if op == "QuantizeLinear":
            scale = x[1]
            zp = x[2] if len(x) > 2 and x[2] is not None else torch.zeros((), dtype=torch.uint8)
            ax = a.get("axis", 1)
            if scale.dim() == 1 and x[0].dim() > 1:
                shape = [1] * x[0].dim()
                shape[ax] = -1
                scale, zp = scale.reshape(shape), zp.reshape(shape)
            lo, hi = (0, 255) if zp.dtype == torch.uint8 else (-128, 127)
            q = torch.round(x[0] / scale) + zp.to(torch.float32)  # round half to even, as ONNX specifies
            return q.clamp(lo, hi).to(zp.dtype)
        if op == "DequantizeLinear":
            scale = x[1]
            zp = x[2] if len(x) > 2 and x[2] is not None else torch.zeros((), dtype=x[0].dtype)
            ax = a.get("axis", 1)
            if scale.dim() == 1 and x[0].dim() > 1:
                shape = [1] * x[0].dim()
                shape[ax] = -1
                scale, zp = scale.reshape(shape), zp.reshape(shape)
            return (x[0].to(torch.float32) - zp.to(torch.float32)) * scale
        if op == "GroupNormalization":
            g = a["num_groups"]
            y = F.group_norm(x[0], g, eps=a.get("epsilon", 1e-5))
            C = x[0].shape[1]
            if x[1].numel() == C:  # opset 21: per-channel scale and bias
                shape = [1, C] + [1] * (x[0].dim() - 2)
                return y * x[1].reshape(shape) + x[2].reshape(shape)
            rep = C // g  # opset 18: per-group scale and bias
            shape = [1, C] + [1] * (x[0].dim() - 2)
            return y * x[1].repeat_interleave(rep).reshape(shape) + x[2].repeat_interleave(rep).reshape(shape)
        if op == "LpNormalization":
            return F.normalize(x[0], p=a.get("p", 2), dim=a.get("axis", -1))
        if op in ("ReduceLogSumExp", "ReduceSumSquare", "ReduceL1"):
            axes = a.get("axes") if "axes" in a else (x[1].tolist() if len(x) > 1 and x[1] is not None else None)
            keep = bool(a.get("keepdims", 1))
            dims = tuple(axes) if axes else tuple(range(x[0].dim()))
            if op == "ReduceLogSumExp":
                return torch.logsumexp(x[0], dim=dims, keepdim=keep)
            if op == "ReduceSumSquare":
                return (x[0] * x[0]).sum(dim=dims, keepdim=keep)
            return x[0].abs().sum(dim=dims, keepdim=keep)
        if op == "Mish":
            return x[0] * torch.tanh(F.softplus(x[0]))
        if op == "Celu":
            al = a.get("alpha", 1.0)
            return torch.clamp(x[0], min=0) + torch.clamp(al * (torch.exp(x[0] / al) - 1), max=0)
        if op == "ThresholdedRelu":
            return torch.where(x[0] > a.get("alpha", 1.0), x[0], torch.zeros_like(x[0]))
        if op == "Shrink":
            lam, bias = a.get("lambd", 0.5), a.get("bias", 0.0)
            return torch.where(x[0] < -lam, x[0] + bias, torch.where(x[0] > lam, x[0] - bias, torch.zeros_like(x[0])))
        if op == "Compress":
            cond = x[1].bool()
            if "axis" not in a:
                return x[0].flatten()[cond[: x[0].numel()].nonzero().flatten()]
            ax = a["axis"]
            keep = cond[: x[0].shape[ax]].nonzero().flatten()
            return torch.index_select(x[0], ax, keep)
        if op == "BitShift":
            d = a["direction"]
            d = d.decode() if isinstance(d, bytes) else d
            return x[0] << x[1] if d == "LEFT" else x[0] >> x[1]
        raise ValueError(f"unsupported ONNX op {op}")


# ------------------------------------------------------------------ LLMs
def load_onnx_llm(path: str, root: str, device, tp: int = 1, rank: int = 0):
    """LLM weights from an ONNX export whose initializers keep HF names."""
    from ..models.config import ModelConfig
    from ..models.cpu_model import CPUCausalLM
    from ..models.llama import weights_from_full

    model = read_model(path)
    cfg = ModelConfig.from_hf_config(os.path.join(root, "config.json"))
    W = {k: torch.from_numpy(np.ascontiguousarray(v)).float() for k, v in model.initializers.items()}

    def get(name):
        if name in W:
            return W[name]
        raise ValueError(f"ONNX export lacks initializer {name}; only exports keeping HF tensor names are supported")

    def stream():
        emb = get("model.embed_tokens.weight")
        yield "embed", emb
        yield "lm_head", W.get("lm_head.weight", emb)
        yield "final_norm", get("model.norm.weight")
        for i in range(cfg.num_layers):
            p = f"model.layers.{i}."
            a = p + "self_attn."
            full = {"q": get(a + "q_proj.weight"), "k": get(a + "k_proj.weight"), "v": get(a + "v_proj.weight"),
                    "o": get(a + "o_proj.weight"), "in_norm": get(p + "input_layernorm.weight"),
                    "post_norm": get(p + "post_attention_layernorm.weight"), "gate": get(p + "mlp.gate_proj.weight"),
                    "up": get(p + "mlp.up_proj.weight"), "down": get(p + "mlp.down_proj.weight")}
            if a + "q_proj.bias" in W:
                full["q_b"], full["k_b"], full["v_b"] = W[a + "q_proj.bias"], W[a + "k_proj.bias"], W[a + "v_proj.bias"]
            yield "layer", full

    dev = torch.device(device)
    if dev.type == "cpu":
        items = list(stream())
        d = dict((k, v) for k, v in items if k != "layer")
        return cfg, CPUCausalLM(cfg, d["embed"], d["lm_head"], d["final_norm"],
                                [v for k, v in items if k == "layer"]), None
    conv = ((k, v.to(dev, torch.bfloat16) if isinstance(v, torch.Tensor)
             else {kk: vv.to(dev, torch.bfloat16) for kk, vv in v.items()}) for k, v in stream())
    return cfg, weights_from_full(cfg, conv, dev, tp, rank), None


# ------------------------------------------------------------ writing
def _enc_varint(x: int) -> bytes:
    out = bytearray()
    x &= (1 << 64) - 1
    while True:
        b = x & 0x7F
        x >>= 7
        out.append(b | (0x80 if x else 0))
        if not x:
            return bytes(out)


def _key(f: int, wt: int) -> bytes:
    return _enc_varint((f << 3) | wt)


def _ld(f: int, b: bytes) -> bytes:
    return _key(f, 2) + _enc_varint(len(b)) + b


def encode_tensor(name: str, a: np.ndarray) -> bytes:
    dt = {np.dtype(np.float32): 1, np.dtype(np.uint8): 2, np.dtype(np.int8): 3, np.dtype(np.int32): 6,
          np.dtype(np.int64): 7, np.dtype(np.bool_): 9, np.dtype(np.float16): 10}[a.dtype]
    b = b"".join(_key(1, 0) + _enc_varint(d) for d in a.shape)
    b += _key(2, 0) + _enc_varint(dt) + _ld(8, name.encode()) + _ld(9, np.ascontiguousarray(a).tobytes())
    return b


def encode_model(nodes: list, inputs: list, outputs: list, initializers: dict, opset: int = 13) -> bytes:
    """Minimal ModelProto writer (for tests and synthetic exports)."""
    g = b""
    for n in nodes:
        nb = b"".join(_ld(1, i.encode()) for i in n.inputs) + b"".join(_ld(2, o.encode()) for o in n.outputs)
        nb += _ld(3, (n.name or n.op).encode()) + _ld(4, n.op.encode())
        for k, v in n.attrs.items():
            ab = _ld(1, k.encode())
            if isinstance(v, float):
                ab += _key(2, 5) + struct.pack("<f", v) + _key(20, 0) + _enc_varint(1)
            elif isinstance(v, int):
                ab += _key(3, 0) + _enc_varint(v) + _key(20, 0) + _enc_varint(2)
            elif isinstance(v, (list, tuple)):
                ab += b"".join(_key(8, 0) + _enc_varint(int(i)) for i in v) + _key(20, 0) + _enc_varint(7)
            elif isinstance(v, str):
                ab += _ld(4, v.encode()) + _key(20, 0) + _enc_varint(3)
            elif isinstance(v, np.ndarray):
                ab += _ld(5, encode_tensor(k, v)) + _key(20, 0) + _enc_varint(4)
            nb += _ld(5, ab)
        g += _ld(1, nb)
    g += _ld(2, b"graph")
    for k, v in initializers.items():
        g += _ld(5, encode_tensor(k, v))
    for i in inputs:
        g += _ld(11, _ld(1, i.encode()))
    for o in outputs:
        g += _ld(12, _ld(1, o.encode()))
    m = _key(1, 0) + _enc_varint(8) + _ld(2, b"kapsl") + _ld(7, g) + _ld(8, _key(2, 0) + _enc_varint(opset))
    return m
