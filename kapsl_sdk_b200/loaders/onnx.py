"""ONNX models without ONNX Runtime.

No ``onnx`` / ``onnxruntime`` package exists here, so this module decodes the
protobuf wire format of ``ModelProto`` directly (varints and length-delimited
fields; field numbers from the public onnx.proto) and provides:

* ``read_model`` -> graph nodes, inputs/outputs, initializers as numpy arrays
  (raw_data or typed repeated fields; external data files next to the model);
* ``OnnxGraph`` -> a PyTorch interpreter for the operators listed in
  ``OnnxGraph.SUPPORTED`` (tensor math, convolution and pooling, shapes and
  indexing, reductions, normalizations, quantize / dequantize and the
  integer / QLinear products, Resize per the spec's coordinate modes,
  NonMaxSuppression, control flow with subgraphs (If, Loop, Scan) and the
  recurrent layers RNN / GRU / LSTM).  Graphs using other ops (checked through
  every subgraph) are rejected at load time with the op names listed;
* ``load_onnx_llm`` -> LLM weights from initializers named like a HF
  checkpoint (``model.layers.{i}.self_attn.q_proj.weight`` ...), the way an
  ONNX export of a decoder keeps them.

Reference: the reference serves any ONNX graph through ONNX Runtime
(crates/kapsl-backends/src/onnx.rs) and LLM exports through ORT sessions.
"""
from __future__ import annotations

import collections
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
_TORCH_DT = {1: torch.float32, 2: torch.uint8, 3: torch.int8, 5: torch.int16, 6: torch.int32, 7: torch.int64,
             9: torch.bool, 10: torch.float16, 11: torch.float64, 16: torch.bfloat16}


def _contig(v: np.ndarray) -> np.ndarray:
    """C-contiguous view or copy that keeps 0-d arrays 0-d (np.ascontiguousarray makes them 1-d)."""
    v = np.asarray(v)
    return v if v.flags.c_contiguous else np.ascontiguousarray(v)


def _saturate(v: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Round-to-nearest-even values already rounded, clamped to an integer dtype's range."""
    info = torch.iinfo(dtype)
    return v.clamp(info.min, info.max).to(dtype)


def _varint(b: bytes, i: int):
    shift = v = 0
    while True:
        if i >= len(b):
            raise ValueError("malformed protobuf: truncated varint")
        x = b[i]
        i += 1
        v |= (x & 0x7F) << shift
        if x < 0x80:
            return v, i
        shift += 7
        if shift > 63:
            raise ValueError("malformed protobuf: varint longer than 10 bytes")


def _fields(b: bytes):
    """Yields (field_number, wire_type, value) over one message."""
    i, n = 0, len(b)
    while i < n:
        key, i = _varint(b, i)
        f, wt = key >> 3, key & 7
        if wt == 0:
            v, i = _varint(b, i)
            yield f, wt, v
            continue
        if wt == 1:
            ln = 8
        elif wt == 2:
            ln, i = _varint(b, i)
        elif wt == 5:
            ln = 4
        else:
            raise ValueError(f"unsupported protobuf wire type {wt}")
        if i + ln > n:
            raise ValueError(f"malformed protobuf: field {f} runs {i + ln - n} bytes past the message")
        yield f, wt, b[i:i + ln]
        i += ln


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
    domain: str = ""  # "" / "ai.onnx" for standard operators, e.g. "com.microsoft" for contrib ones


@dataclass
class OnnxModel:
    nodes: list
    inputs: list
    outputs: list
    initializers: dict
    opset: int = 13
    # declared input types: name -> (TensorProto element type or None, dims with None for symbolic ones)
    input_types: dict = field(default_factory=dict)
    output_types: dict = field(default_factory=dict)


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
        elif f == 6:  # GraphProto (If / Loop / Scan bodies)
            val = _graph(v, base_dir)
        elif f == 20:
            kind = v
    if ints:
        val = ints
    elif floats:
        val = floats
    elif strs:
        val = strs
    return name, val


def _value_info_type(b: bytes) -> tuple:
    """ValueInfoProto -> (element type or None, [dim or None]) of a tensor type."""
    elem, dims = None, []
    for f, _, v in _fields(b):
        if f != 2:  # TypeProto
            continue
        for ft, _, tv in _fields(v):
            if ft != 1:  # TypeProto.Tensor
                continue
            for fe, _, ev in _fields(tv):
                if fe == 1:
                    elem = ev
                elif fe == 2:  # TensorShapeProto
                    for fd, _, dv in _fields(ev):
                        if fd == 1:
                            d = None
                            for fv, _, vv in _fields(dv):
                                if fv == 1:
                                    d = _signed64(vv)
                            dims.append(d)
    return elem, dims


def _value_info_name(b: bytes) -> str:
    for f, _, v in _fields(b):
        if f == 1:
            return v.decode()
    return ""


def _graph(graph: bytes, base: Optional[str], opset: int = 13) -> OnnxModel:
    """GraphProto -> OnnxModel (nodes, declared inputs and outputs, initializers).
    Subgraphs keep their initializer-backed inputs out of ``inputs`` like the
    main graph; names they use without defining come from the enclosing scope."""
    nodes, inputs, outputs, inits, types, out_types = [], [], [], {}, {}, {}
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
                elif ff == 7:
                    n.domain = vv.decode()
            nodes.append(n)
        elif f == 5:
            k, a = _tensor(v, base)
            inits[k] = a
        elif f == 11:
            inputs.append(_value_info_name(v))
            types[inputs[-1]] = _value_info_type(v)
        elif f == 12:
            outputs.append(_value_info_name(v))
            out_types[outputs[-1]] = _value_info_type(v)
    inputs = [i for i in inputs if i not in inits]
    return OnnxModel(nodes, inputs, outputs, inits, opset, {k: t for k, t in types.items() if k in inputs}, out_types)


def read_model(path: str) -> OnnxModel:
    """Decodes an ONNX file; any malformed content raises ValueError."""
    with open(path, "rb") as fh:
        data = fh.read()
    try:
        return _read_model_bytes(data, path)
    except (IndexError, struct.error, UnicodeDecodeError, TypeError, OverflowError) as e:
        raise ValueError(f"malformed ONNX file {path}: {e}") from e
    except ValueError as e:
        if "malformed" in str(e) or "protobuf" in str(e):
            raise
        raise ValueError(f"malformed ONNX file {path}: {e}") from e


def _read_model_bytes(data: bytes, path: str) -> OnnxModel:
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
    return _graph(graph, base, opset)


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
                 "ThresholdedRelu", "Shrink", "Compress", "BitShift",
                 # control flow, recurrent layers
                 "If", "Loop", "Scan", "RNN", "GRU", "LSTM",
                 # trigonometric, quantized, detection, sampling, normalization, sequences
                 "Tan", "Asin", "Acos", "Atan", "Sinh", "Cosh", "Asinh", "Acosh", "Atanh", "IsInf", "CastLike",
                 "EyeLike", "Hardmax", "LRN", "MeanVarianceNormalization", "RMSNormalization", "ReverseSequence",
                 "Unique", "Det", "LpPool", "GlobalLpPool", "MatMulInteger", "QLinearMatMul", "ConvInteger",
                 "QLinearConv", "NonMaxSuppression", "GridSample", "RandomNormal", "RandomUniform",
                 "RandomNormalLike", "RandomUniformLike", "Bernoulli", "Upsample",
                 # transformer graphs (standard opset 23 and the com.microsoft fused ops)
                 "Attention", "RotaryEmbedding", "SkipLayerNormalization", "SimplifiedLayerNormalization",
                 "SkipSimplifiedLayerNormalization", "FastGelu", "BiasGelu", "QuickGelu", "BiasAdd",
                 "MultiHeadAttention", "MatMulNBits", "GroupQueryAttention"}

    CONTROL = {"If", "Loop", "Scan"}
    # a Loop whose trip count and condition are both absent runs until this many
    # iterations, then fails (the spec's unbounded loop)
    MAX_LOOP_ITERS = 1 << 24

    # ops whose inputs after the first are read on the host (shapes, axes, counts):
    # those inputs stay where they are, so shape arithmetic never syncs the device
    HOST_ARG_OPS = {"Reshape", "Expand", "Tile", "Slice", "Range", "ConstantOfShape", "Resize", "Upsample", "Pad",
                    "OneHot", "Split", "Unsqueeze", "Squeeze", "ReduceMean", "ReduceSum", "ReduceMax", "ReduceMin",
                    "ReduceProd", "ReduceL2", "ReduceL1", "ReduceLogSumExp", "ReduceSumSquare", "TopK", "Trilu",
                    "CumSum", "Shape", "Size"}
    # ops whose output shape depends on input values
    DATA_SHAPED_OPS = {"NonZero", "Unique", "NonMaxSuppression", "Compress", "If", "Loop", "Scan"}
    RANDOM_OPS = {"RandomNormal", "RandomUniform", "RandomNormalLike", "RandomUniformLike", "Bernoulli"}
    STATIC_CACHE_MAX_NUMEL = 1 << 24
    SMALL_INT_NUMEL = 64

    def __init__(self, model: OnnxModel, device="cpu", plan_cache: int = 4):
        bad = sorted(self.ops_used(model) - self.SUPPORTED)
        if bad:
            raise ValueError(f"unsupported ONNX ops: {', '.join(bad)}")
        self.m = model
        self.device = torch.device(device)
        self.consts = {k: self._place(torch.from_numpy(_contig(v))) for k, v in model.initializers.items()}
        self._sub_consts: dict[int, dict] = {}
        self._static = self._static_values(model)
        self.plan_cache = max(0, plan_cache)
        self._plans: "collections.OrderedDict" = collections.OrderedDict()
        self.stats = {"plans_built": 0, "plan_hits": 0, "nodes_skipped": 0}

    def _place(self, t: torch.Tensor) -> torch.Tensor:
        """Small integer tensors (shapes, axes, indices of shape arithmetic) live on
        the host; everything else on the interpreter's device."""
        if not t.is_floating_point() and t.dtype != torch.bool and t.numel() <= self.SMALL_INT_NUMEL:
            return t.cpu()
        return t.to(self.device)

    def _static_values(self, model: OnnxModel) -> set:
        """Names whose values depend only on the initializers and the input shapes
        (Shape / Size of a value whose shape is fixed by the input shapes, and
        deterministic ops over such values).  For one set of input shapes they are
        computed once and reused (the per-shape plan)."""
        static = set(model.initializers)
        stable = set(model.initializers) | set(model.inputs)
        for n in model.nodes:
            ins = [i for i in n.inputs if i]
            if n.op in ("Shape", "Size"):
                is_static = all(i in stable for i in ins[:1])
            else:
                is_static = n.op not in self.RANDOM_OPS and n.op not in self.CONTROL and all(i in static for i in ins)
            value_args = ins if n.op in ("ConstantOfShape", "Range") else ins[1:]
            is_stable = is_static or (all(i in stable for i in ins) and n.op not in self.DATA_SHAPED_OPS and
                                      (n.op not in self.HOST_ARG_OPS or all(i in static for i in value_args)))
            for o in n.outputs:
                if o and is_static:
                    static.add(o)
                if o and is_stable:
                    stable.add(o)
        return static - set(model.initializers)

    @staticmethod
    def ops_used(model: OnnxModel) -> set:
        """Operator types of a graph and of every subgraph it holds."""
        ops = set()
        for n in model.nodes:
            ops.add(n.op)
            for v in n.attrs.values():
                if isinstance(v, OnnxModel):
                    ops |= OnnxGraph.ops_used(v)
        return ops

    def run(self, feeds: dict) -> dict:
        env = dict(self.consts)
        for k, v in feeds.items():
            if not isinstance(v, torch.Tensor):
                v = _contig(v)
                v = torch.from_numpy(v if v.flags.writeable else v.copy())  # request buffers are read-only
            env[k] = v
            env[k] = env[k].to(self.device)
        key = tuple((k, tuple(v.shape), str(v.dtype)) for k, v in sorted(env.items()) if k in feeds)
        plan = self._plans.get(key) if self.plan_cache else None
        if plan is not None:
            self._plans.move_to_end(key)
            env.update(plan)
            self.stats["plan_hits"] += 1
            self._exec(self.m, env, skip=plan)
        else:
            self._exec(self.m, env)
            if self.plan_cache and self._static:
                self._plans[key] = {k: env[k] for k in self._static
                                    if k in env and isinstance(env[k], torch.Tensor)
                                    and env[k].numel() <= self.STATIC_CACHE_MAX_NUMEL}
                self.stats["plans_built"] += 1
                while len(self._plans) > self.plan_cache:
                    self._plans.popitem(last=False)
        return {o: env[o] for o in self.m.outputs}

    def _exec(self, m: OnnxModel, env: dict, skip: Optional[dict] = None) -> None:
        for n in m.nodes:
            if skip and n.outputs and all((not o) or o in skip for o in n.outputs):
                self.stats["nodes_skipped"] += 1
                continue
            args = [env[i] if i else None for i in n.inputs]
            if n.op in self.CONTROL:
                outs = self._control(n, args, env)
            else:
                outs = self._op(n, self._harmonize(n.op, args))
            if not isinstance(outs, (list, tuple)):
                outs = [outs]
            for name, val in zip(n.outputs, outs):
                if name:
                    env[name] = val

    def _harmonize(self, op: str, args: list) -> list:
        """Host-resident small tensors join a device operand's device, except the
        host-read arguments of shape operators."""
        devs = {t.device for t in args if isinstance(t, torch.Tensor) and t.device.type != "cpu"}
        if not devs:
            return args
        dev = next(iter(devs))
        first_only = op in self.HOST_ARG_OPS
        return [t.to(dev) if isinstance(t, torch.Tensor) and t.device.type == "cpu" and (i == 0 or not first_only)
                else t for i, t in enumerate(args)]

    def _sub(self, g: OnnxModel, env: dict, bind: dict) -> list:
        """Runs subgraph ``g`` in a child scope of ``env`` (outer names stay visible,
        the subgraph's own initializers and bound inputs shadow them)."""
        consts = self._sub_consts.get(id(g))
        if consts is None:
            consts = {k: self._place(torch.from_numpy(_contig(v))) for k, v in g.initializers.items()}
            self._sub_consts[id(g)] = consts
        scope = dict(env)
        scope.update(consts)
        scope.update(bind)
        self._exec(g, scope)
        return [scope[o] for o in g.outputs]

    def _control(self, n: Node, x: list, env: dict):
        """If / Loop / Scan (ONNX control flow, opset 11+ / 13+ / 9+ semantics)."""
        a, op = n.attrs, n.op
        if op == "If":
            branch = a["then_branch"] if bool(x[0].reshape(-1)[0]) else a["else_branch"]
            return self._sub(branch, env, {})
        body = a["body"]
        if op == "Loop":
            trip = int(x[0].reshape(-1)[0]) if len(x) > 0 and x[0] is not None else None
            keep = bool(x[1].reshape(-1)[0]) if len(x) > 1 and x[1] is not None else True
            vs = list(x[2:])
            nv = len(vs)
            scans: list = []
            i = 0
            while (trip is None or i < trip) and keep:
                if trip is None and (len(x) < 2 or x[1] is None) and i >= self.MAX_LOOP_ITERS:
                    raise ValueError("Loop without trip count or condition did not end")
                # iteration number and condition are host values, like other shape arithmetic
                bind = {body.inputs[0]: torch.tensor(i, dtype=torch.int64), body.inputs[1]: torch.tensor(keep)}
                bind.update({name: v for name, v in zip(body.inputs[2:], vs)})
                out = self._sub(body, env, bind)
                keep = bool(out[0].reshape(-1)[0])
                vs = out[1:1 + nv]
                if not scans:
                    scans = [[] for _ in out[1 + nv:]]
                for acc, v in zip(scans, out[1 + nv:]):
                    acc.append(v)
                i += 1
            n_scan = len(body.outputs) - 1 - nv
            stacked = [torch.stack(acc) for acc in scans] if scans else \
                [torch.empty(0, device=self.device) for _ in range(n_scan)]
            return vs + stacked
        # Scan
        m = a["num_scan_inputs"]
        ns = len(x) - m
        states, ins = list(x[:ns]), list(x[ns:])
        in_axes = [ax % t.dim() for ax, t in zip(a.get("scan_input_axes") or [0] * m, ins)]
        in_dirs = a.get("scan_input_directions") or [0] * m
        T = ins[0].shape[in_axes[0]]
        k = len(body.outputs) - ns
        acc = [[] for _ in range(k)]
        for t in range(T):
            slices = [v.select(ax, T - 1 - t if d else t) for v, ax, d in zip(ins, in_axes, in_dirs)]
            out = self._sub(body, env, {name: v for name, v in zip(body.inputs, states + slices)})
            states = out[:ns]
            for lst, v in zip(acc, out[ns:]):
                lst.append(v)
        out_axes = a.get("scan_output_axes") or [0] * k
        out_dirs = a.get("scan_output_directions") or [0] * k
        res = []
        for lst, ax, d in zip(acc, out_axes, out_dirs):
            if d:
                lst = lst[::-1]
            r = lst[0].dim() + 1
            res.append(torch.stack(lst, dim=ax % r))
        return states + res

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
            return self._place(torch.from_numpy(_contig(v)))
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
            ax = a.get("axis", 0) % x[0].dim()
            idx = x[1].long()
            idx = torch.where(idx < 0, idx + x[0].shape[ax], idx)  # negative indices count from the end
            return torch.index_select(x[0], ax, idx.flatten()).reshape(
                [*x[0].shape[:ax], *x[1].shape, *x[0].shape[ax + 1:]])
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
            return torch.tensor(list(x[0].shape), dtype=torch.int64)  # host-resident shape
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
            r = torch.arange(x[0].item(), x[1].item(), x[2].item()).to(x[0].dtype)
            return self._place(r)
        if op == "Size":
            return torch.tensor(x[0].numel(), dtype=torch.int64)
        if op == "Resize":
            def sa(k, d):
                v = a.get(k, d)
                return v.decode() if isinstance(v, bytes) else v

            def opt(i):
                return x[i] if len(x) > i and x[i] is not None and x[i].numel() else None

            return self._resize(x[0], opt(1), opt(2), opt(3), sa("mode", "nearest"),
                                sa("coordinate_transformation_mode", "half_pixel"),
                                sa("nearest_mode", "round_prefer_floor"), a.get("cubic_coeff_a", -0.75),
                                a.get("exclude_outside", 0), a.get("extrapolation_value", 0.0), a.get("axes"),
                                sa("keep_aspect_ratio_policy", "stretch"), a.get("antialias", 0))
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
        if op in ("RNN", "GRU", "LSTM"):
            return self._recurrent(op, x, a)
        return self._op_late(n, x)

    @staticmethod
    def _rnn_act(name: str, alpha, beta):
        """ONNX recurrent-layer activation by name (alpha / beta as the spec defines them)."""
        name = name.decode() if isinstance(name, bytes) else name
        F = torch.nn.functional
        k = name.lower()
        if k == "sigmoid":
            return torch.sigmoid
        if k == "tanh":
            return torch.tanh
        if k == "relu":
            return torch.relu
        if k == "affine":
            return lambda v: (1.0 if alpha is None else alpha) * v + (0.0 if beta is None else beta)
        if k == "leakyrelu":
            return lambda v: F.leaky_relu(v, 0.01 if alpha is None else alpha)
        if k == "thresholdedrelu":
            return lambda v: torch.where(v > (1.0 if alpha is None else alpha), v, torch.zeros_like(v))
        if k == "scaledtanh":
            return lambda v: (1.0 if alpha is None else alpha) * torch.tanh((1.0 if beta is None else beta) * v)
        if k == "hardsigmoid":
            return lambda v: torch.clamp((0.2 if alpha is None else alpha) * v + (0.5 if beta is None else beta), 0, 1)
        if k == "elu":
            return lambda v: F.elu(v, 1.0 if alpha is None else alpha)
        if k == "softsign":
            return F.softsign
        if k == "softplus":
            return F.softplus
        raise ValueError(f"unsupported recurrent activation {name}")

    def _recurrent(self, op: str, x: list, a: dict):
        """RNN / GRU / LSTM over [seq, batch, input] (layout 0) or [batch, seq, input]
        (layout 1): gate orders i, o, f, c (LSTM) and z, r, h (GRU), optional
        biases, per-batch sequence lengths (steps past a length leave Y zero and
        Y_h at the last valid state; the reverse direction walks each sequence's
        valid part backwards), initial states, LSTM peepholes and input_forget,
        GRU linear_before_reset, clip, forward / reverse / bidirectional."""
        def arg(i):
            return x[i] if len(x) > i and x[i] is not None else None

        layout = a.get("layout", 0)
        X, W, R, B, lens, h0 = x[0], x[1], x[2], arg(3), arg(4), arg(5)
        c0, P = (arg(6), arg(7)) if op == "LSTM" else (None, None)
        if layout:
            X = X.transpose(0, 1)
            h0 = h0.transpose(0, 1) if h0 is not None else None
            c0 = c0.transpose(0, 1) if c0 is not None else None
        direction = a.get("direction", "forward")
        direction = direction.decode() if isinstance(direction, bytes) else direction
        nd = 2 if direction == "bidirectional" else 1
        H = a["hidden_size"]
        G = {"RNN": 1, "GRU": 3, "LSTM": 4}[op]
        seq, batch = X.shape[0], X.shape[1]
        default_acts = {"RNN": ["Tanh"], "GRU": ["Sigmoid", "Tanh"], "LSTM": ["Sigmoid", "Tanh", "Tanh"]}[op]
        names = a.get("activations") or default_acts * nd
        if len(names) == len(default_acts) and nd == 2:
            names = list(names) * 2
        alphas, betas = a.get("activation_alpha") or [], a.get("activation_beta") or []
        acts = [self._rnn_act(nm, alphas[i] if i < len(alphas) else None, betas[i] if i < len(betas) else None)
                for i, nm in enumerate(names)]
        clip = a.get("clip")
        lens = lens.long() if lens is not None else torch.full((batch,), seq, dtype=torch.long, device=X.device)
        Y = X.new_zeros(seq, nd, batch, H)
        Yh = X.new_zeros(nd, batch, H)
        Yc = X.new_zeros(nd, batch, H)
        bidx = torch.arange(batch, device=X.device)
        for d in range(nd):
            rev = direction == "reverse" or d == 1
            f_, g_, h_ = (acts[d * len(default_acts) + j] for j in range(len(default_acts))) if op == "LSTM" else \
                ((acts[d * len(default_acts)], acts[d * len(default_acts) + 1], None) if op == "GRU" else
                 (acts[d], None, None))
            Wd, Rd = W[d], R[d]
            Bd = B[d] if B is not None else X.new_zeros(2 * G * H)
            Wb, Rb = Bd[:G * H], Bd[G * H:]
            h = h0[d] if h0 is not None else X.new_zeros(batch, H)
            c = c0[d] if c0 is not None else X.new_zeros(batch, H)

            def cl(v):
                return v.clamp(-clip, clip) if clip is not None else v

            for step in range(seq):
                valid = step < lens
                t = (lens - 1 - step).clamp(min=0) if rev else torch.full_like(lens, step)
                xt = X[t, bidx]
                if op == "RNN":
                    hn = f_(cl(xt @ Wd.T + Wb + h @ Rd.T + Rb))
                elif op == "GRU":
                    gx = xt @ Wd.T + Wb
                    Rz, Rr, Rh = Rd[:H], Rd[H:2 * H], Rd[2 * H:]
                    z = f_(cl(gx[:, :H] + h @ Rz.T + Rb[:H]))
                    r = f_(cl(gx[:, H:2 * H] + h @ Rr.T + Rb[H:2 * H]))
                    if a.get("linear_before_reset", 0):
                        hh = g_(cl(gx[:, 2 * H:] + r * (h @ Rh.T + Rb[2 * H:])))
                    else:
                        hh = g_(cl(gx[:, 2 * H:] + (r * h) @ Rh.T + Rb[2 * H:]))
                    hn = (1 - z) * hh + z * h
                else:
                    gs = xt @ Wd.T + Wb + h @ Rd.T + Rb
                    gi, go, gf, gc = gs[:, :H], gs[:, H:2 * H], gs[:, 2 * H:3 * H], gs[:, 3 * H:]
                    if P is not None:
                        gi = gi + P[d][:H] * c
                        gf = gf + P[d][2 * H:] * c
                    i_ = f_(cl(gi))
                    fg = 1 - i_ if a.get("input_forget", 0) else f_(cl(gf))
                    cn = fg * c + i_ * g_(cl(gc))
                    if P is not None:
                        go = go + P[d][H:2 * H] * cn
                    hn = f_(cl(go)) * h_(cn)
                    c = torch.where(valid[:, None], cn, c)
                h = torch.where(valid[:, None], hn, h)
                Y[t[valid], d, bidx[valid]] = hn[valid]
            Yh[d] = h
            Yc[d] = c
        if layout:
            outs = [Y.permute(2, 0, 1, 3), Yh.transpose(0, 1), Yc.transpose(0, 1)]
        else:
            outs = [Y, Yh, Yc]
        return outs if op == "LSTM" else outs[:2]

    def _op_late(self, n: Node, x: list):
        """Trigonometric / hyperbolic functions, integer and quantized-linear
        products and convolutions, detection (NonMaxSuppression), sampling
        (GridSample), normalizations and sequence utilities (opset 13-23 semantics)."""
        a, op = n.attrs, n.op
        F = torch.nn.functional

        def sattr(k, d):
            v = a.get(k, d)
            return v.decode() if isinstance(v, bytes) else v

        trig = {"Tan": torch.tan, "Asin": torch.asin, "Acos": torch.acos, "Atan": torch.atan, "Sinh": torch.sinh,
                "Cosh": torch.cosh, "Asinh": torch.asinh, "Acosh": torch.acosh, "Atanh": torch.atanh}
        if op in trig:
            return trig[op](x[0])
        if op == "IsInf":
            v = x[0]
            pos = torch.isposinf(v) if a.get("detect_positive", 1) else torch.zeros_like(v, dtype=torch.bool)
            neg = torch.isneginf(v) if a.get("detect_negative", 1) else torch.zeros_like(v, dtype=torch.bool)
            return pos | neg
        if op == "CastLike":
            return x[0].to(x[1].dtype)
        if op == "EyeLike":
            dt = _TORCH_DT.get(a["dtype"], x[0].dtype) if "dtype" in a else x[0].dtype
            r, c = x[0].shape
            rows = torch.arange(r, device=x[0].device)
            cols = rows + a.get("k", 0)
            ok = (cols >= 0) & (cols < c)
            y = torch.zeros(r, c, dtype=torch.float64, device=x[0].device)
            y[rows[ok], cols[ok]] = 1
            return y.to(dt)
        if op == "Hardmax":
            ax = a.get("axis", -1)
            idx = x[0].argmax(dim=ax, keepdim=True)
            return torch.zeros_like(x[0]).scatter(ax, idx, 1.0)
        if op == "LRN":
            size = a["size"]
            al, be, bias = a.get("alpha", 1e-4), a.get("beta", 0.75), a.get("bias", 1.0)
            lo, hi = (size - 1) // 2, size - 1 - (size - 1) // 2
            sq = F.pad(x[0] * x[0], [0, 0] * (x[0].dim() - 2) + [lo, hi])
            C = x[0].shape[1]
            acc = sum(sq[:, i:i + C] for i in range(size))
            return x[0] / (bias + al / size * acc) ** be
        if op == "MeanVarianceNormalization":
            axes = tuple(a.get("axes") or [0, 2, 3])
            mean = x[0].mean(dim=axes, keepdim=True)
            var = (x[0] * x[0]).mean(dim=axes, keepdim=True) - mean * mean
            return (x[0] - mean) / (torch.sqrt(var) + 1e-9)
        if op == "RMSNormalization":
            ax = a.get("axis", -1) % x[0].dim()
            xf = x[0].float()
            ms = (xf * xf).mean(dim=tuple(range(ax, x[0].dim())), keepdim=True)
            return (xf * torch.rsqrt(ms + a.get("epsilon", 1e-5)) * x[1].float()).to(x[0].dtype)
        if op == "ReverseSequence":
            bax, tax = a.get("batch_axis", 1), a.get("time_axis", 0)
            y = x[0].clone()
            for b, L in enumerate(x[1].tolist()):
                src = x[0].select(bax, b)
                t_ax = tax if tax < bax else tax - 1
                y.select(bax, b).narrow(t_ax, 0, L).copy_(src.narrow(t_ax, 0, L).flip(t_ax))
            return y
        if op == "Unique":
            v = x[0].cpu().numpy()
            ax = a.get("axis")
            vals, first, inv, cnt = np.unique(v if ax is not None else v.reshape(-1), return_index=True,
                                               return_inverse=True, return_counts=True, axis=ax)
            inv = inv.reshape(-1)
            if not a.get("sorted", 1):  # order of first occurrence
                order = np.argsort(first, kind="stable")
                rank = np.empty_like(order)
                rank[order] = np.arange(len(order))
                vals = np.take(vals, order, axis=ax if ax is not None else 0)
                first, cnt, inv = first[order], cnt[order], rank[inv]
            dev = x[0].device
            return [torch.from_numpy(_contig(vals)).to(dev),
                    torch.from_numpy(first.astype(np.int64)).to(dev), torch.from_numpy(inv.astype(np.int64)).to(dev),
                    torch.from_numpy(cnt.astype(np.int64)).to(dev)]
        if op == "Det":
            return torch.linalg.det(x[0])
        if op in ("LpPool", "GlobalLpPool"):
            p = a.get("p", 2)
            v = x[0].abs() ** p
            nd = x[0].dim() - 2
            if op == "GlobalLpPool":
                return v.sum(dim=tuple(range(2, x[0].dim())), keepdim=True) ** (1.0 / p)
            k = a["kernel_shape"]
            lo, hi = _conv_pads(a, nd)
            if any(lo + hi):
                v = F.pad(v, [q for pair in zip(reversed(lo), reversed(hi)) for q in pair])
            s = a.get("strides") or [1] * nd
            pooled = getattr(F, f"avg_pool{nd}d")(v, k, s) * float(np.prod(k))
            return pooled ** (1.0 / p)
        if op == "MatMulInteger":
            A = x[0].to(torch.int64)
            B = x[1].to(torch.int64)
            if len(x) > 2 and x[2] is not None:
                az = x[2].to(torch.int64)
                A = A - (az.reshape(-1, 1) if az.dim() == 1 and az.numel() > 1 else az)
            if len(x) > 3 and x[3] is not None:
                B = B - x[3].to(torch.int64)
            return torch.matmul(A.double(), B.double()).round().to(torch.int32)
        if op == "QLinearMatMul":
            A = x[0].double() - x[2].double()
            B = x[3].double() - x[5].double()
            real = torch.matmul(A * x[1].double(), B * x[4].double())
            return _saturate(torch.round(real / x[6].double()) + x[7].double(), x[7].dtype)
        if op in ("ConvInteger", "QLinearConv"):
            if op == "ConvInteger":
                xi, w = x[0].double(), x[1].double()
                xz = x[2].double() if len(x) > 2 and x[2] is not None else 0.0
                wz = x[3].double() if len(x) > 3 and x[3] is not None else None
            else:
                xi, w = x[0].double(), x[3].double()
                xz, wz = x[2].double(), x[5].double()
            nd = w.dim() - 2
            if wz is not None:
                w = w - (wz.reshape(-1, *([1] * (nd + 1))) if wz.dim() == 1 and wz.numel() > 1 else wz)
            xi = xi - xz
            lo, hi = _conv_pads(a, nd)
            if any(lo + hi):  # zero-point padding: padded input equals the zero point, i.e. 0 after the shift
                xi = F.pad(xi, [q for pair in zip(reversed(lo), reversed(hi)) for q in pair])
            fn = {1: F.conv1d, 2: F.conv2d, 3: F.conv3d}[nd]
            acc = fn(xi, w, None, stride=a.get("strides") or 1, dilation=a.get("dilations") or 1,
                     groups=a.get("group", 1))
            if op == "ConvInteger":
                return acc.round().to(torch.int32)
            if len(x) > 8 and x[8] is not None:
                acc = acc + x[8].double().reshape(1, -1, *([1] * nd))
            ws = x[4].double()
            scale = x[1].double() * (ws.reshape(1, -1, *([1] * nd)) if ws.numel() > 1 else ws)
            return _saturate(torch.round(acc * scale / x[6].double()) + x[7].double(), x[7].dtype)
        if op == "NonMaxSuppression":
            return self._nms(x, a)
        if op == "GridSample":
            mode = sattr("mode", "bilinear")
            mode = {"linear": "bilinear", "cubic": "bicubic"}.get(mode, mode)
            return F.grid_sample(x[0], x[1], mode=mode, padding_mode=sattr("padding_mode", "zeros"),
                                 align_corners=bool(a.get("align_corners", 0)))
        if op in ("RandomNormal", "RandomUniform", "RandomNormalLike", "RandomUniformLike", "Bernoulli"):
            g = torch.Generator(device="cpu")
            if "seed" in a:
                g.manual_seed(int(a["seed"]))
            else:
                g.seed()
            if op == "Bernoulli":
                y = torch.bernoulli(x[0].detach().cpu().double(), generator=g)
                return y.to(_TORCH_DT.get(a.get("dtype"), x[0].dtype)).to(x[0].device)
            shape = list(x[0].shape) if op.endswith("Like") else a["shape"]
            dt = _TORCH_DT.get(a.get("dtype"), x[0].dtype if op.endswith("Like") else torch.float32)
            if "Normal" in op:
                y = torch.randn(shape, generator=g, dtype=torch.float64) * a.get("scale", 1.0) + a.get("mean", 0.0)
            else:
                lo, hi = a.get("low", 0.0), a.get("high", 1.0)
                y = torch.rand(shape, generator=g, dtype=torch.float64) * (hi - lo) + lo
            return y.to(dt).to(self.device)
        if op == "Upsample":
            return self._resize(x[0], None, x[1], None, sattr("mode", "nearest"), "asymmetric", "floor", -0.75, 0, 0.0)
        return self._op_transformer(n, x)

    def _op_transformer(self, n: Node, x: list):
        """Operators of exported transformer graphs: the standard Attention and
        RotaryEmbedding (opset 23) and the com.microsoft fused ops that ONNX Runtime's
        transformer optimizer writes (SkipLayerNormalization, SimplifiedLayerNormalization,
        SkipSimplifiedLayerNormalization, FastGelu, BiasGelu, QuickGelu, BiasAdd,
        MultiHeadAttention, MatMulNBits block-quantized weights)."""
        a, op = n.attrs, n.op
        F = torch.nn.functional

        def opt(i):
            return x[i] if len(x) > i and x[i] is not None else None

        if op == "Attention":
            return self._attention(x, a)
        if op == "RotaryEmbedding" and n.domain == "com.microsoft":
            # contrib form: (input, position_ids, cos_cache, sin_cache); position_ids of
            # one element is the start position of every row
            X, pos, cos, sin = x[0], x[1], x[2], x[3]
            seq = X.shape[-2] if X.dim() == 4 else X.shape[1]
            if pos.numel() == 1:
                pos = (pos.reshape(1, 1).long() + torch.arange(seq, device=pos.device)[None, :]).expand(X.shape[0], -1)
            return self._rotary(X, cos, sin, pos.long(), a.get("interleaved", 0), a.get("num_heads", 0),
                                a.get("rotary_embedding_dim", 0))
        if op == "GroupQueryAttention":
            return self._gqa(x, a)
        if op == "RotaryEmbedding":
            return self._rotary(x[0], x[1], x[2], opt(3), a.get("interleaved", 0), a.get("num_heads", 0),
                                a.get("rotary_embedding_dim", 0))
        if op in ("SkipLayerNormalization", "SkipSimplifiedLayerNormalization"):
            s_ = x[0] + x[1]
            bias = opt(4) if op == "SkipLayerNormalization" else opt(3)
            if bias is not None:
                s_ = s_ + bias
            eps = a.get("epsilon", 1e-12)
            sf = s_.float()
            if op == "SkipLayerNormalization":
                mean = sf.mean(-1, keepdim=True)
                var = ((sf - mean) ** 2).mean(-1, keepdim=True)
                inv = torch.rsqrt(var + eps)
                y = (sf - mean) * inv * x[2].float()
                if opt(3) is not None:
                    y = y + x[3].float()
            else:
                mean = torch.zeros_like(sf[..., :1])
                inv = torch.rsqrt((sf * sf).mean(-1, keepdim=True) + eps)
                y = sf * inv * x[2].float()
            return [y.to(x[0].dtype), mean, inv, s_]
        if op == "SimplifiedLayerNormalization":
            ax = a.get("axis", -1) % x[0].dim()
            xf = x[0].float()
            inv = torch.rsqrt((xf * xf).mean(dim=tuple(range(ax, x[0].dim())), keepdim=True) + a.get("epsilon", 1e-5))
            return [(xf * inv * x[1].float()).to(x[0].dtype), inv]
        if op == "FastGelu":
            v = x[0] + x[1] if opt(1) is not None else x[0]
            return F.gelu(v, approximate="tanh")
        if op == "BiasGelu":
            return F.gelu(x[0] + x[1])
        if op == "QuickGelu":
            return x[0] * torch.sigmoid(a.get("alpha", 1.702) * x[0])
        if op == "BiasAdd":
            return x[0] + x[1] + x[2]
        if op == "MultiHeadAttention":
            return self._mha(x, a)
        if op == "MatMulNBits":
            w = self._nbits_weight(x, a)
            y = torch.matmul(x[0], w.to(x[0].dtype).T)
            return y + x[5] if opt(5) is not None else y
        raise ValueError(f"unsupported ONNX op {op}")

    @staticmethod
    def _rotary(X, cos, sin, pos, interleaved, num_heads, rot):
        """Rotary position embedding of [B, H, S, D] or [B, S, H * D] (num_heads) input:
        cos / sin rows [positions, rot / 2] picked by ``pos`` [B, S] (or already
        [B, S, rot / 2]); the first ``rot`` dims of each head rotate, as pairs
        (2i, 2i+1) when interleaved, else as halves; the rest pass through."""
        three = X.dim() == 3
        Xh = X
        if three:
            B_, S_, hid = X.shape
            Xh = X.reshape(B_, S_, num_heads, hid // num_heads).transpose(1, 2)
        if pos is not None:
            cos, sin = cos[pos], sin[pos]
        cos, sin = cos.unsqueeze(1).to(Xh.dtype), sin.unsqueeze(1).to(Xh.dtype)  # [B, 1, S, rot/2]
        rot = rot or Xh.shape[-1]
        xr, rest = Xh[..., :rot], Xh[..., rot:]
        if interleaved:
            x1, x2 = xr[..., 0::2], xr[..., 1::2]
            y = torch.stack([x1 * cos - x2 * sin, x2 * cos + x1 * sin], -1).reshape(xr.shape)
        else:
            x1, x2 = xr[..., :rot // 2], xr[..., rot // 2:]
            y = torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], -1)
        y = torch.cat([y, rest], -1)
        return y.transpose(1, 2).reshape(X.shape) if three else y

    def _gqa(self, x: list, a: dict):
        """com.microsoft GroupQueryAttention: query [B, S, Hq * D] (or packed q|k|v
        when key is absent), key / value [B, S, Hkv * D], past key / value
        [B, Hkv, P, D] of which the first seqlens_k[b] + 1 - S positions are valid,
        optional rotary on q and k at positions past_len.. (do_rotary, cos / sin
        caches), causal attention over past + new keys with an optional local
        window, softcap and scale (default 1/sqrt(D)); present key / value hold the
        valid past and the new keys ([B, Hkv, total, D], rows past a sequence's
        length zero)."""
        def opt(i):
            return x[i] if len(x) > i and x[i] is not None else None

        hq, hk = a["num_heads"], a["kv_num_heads"]
        q, k, v = x[0], opt(1), opt(2)
        pk, pv, seqlens, total = opt(3), opt(4), x[5].long(), int(x[6].reshape(-1)[0])
        cos, sin = opt(7), opt(8)
        B_, S_ = q.shape[0], q.shape[1]
        if k is None:  # packed q | k | v
            D = q.shape[-1] // (hq + 2 * hk)
            q, k, v = q[..., :hq * D], q[..., hq * D:(hq + hk) * D], q[..., (hq + hk) * D:]
        D = q.shape[-1] // hq
        qh = q.reshape(B_, S_, hq, D).transpose(1, 2)
        kh = k.reshape(B_, S_, hk, D).transpose(1, 2)
        vh = v.reshape(B_, S_, hk, D).transpose(1, 2)
        past_len = seqlens + 1 - S_  # [B]
        if a.get("do_rotary", 0):
            pos = past_len[:, None] + torch.arange(S_, device=q.device)[None, :]
            il = a.get("rotary_interleaved", 0)
            qh = self._rotary(qh, cos, sin, pos, il, hq, 0)
            kh = self._rotary(kh, cos, sin, pos, il, hk, 0)
        Tn = max(total, int((past_len + S_).max()))
        pres_k = q.new_zeros(B_, hk, Tn, D)
        pres_v = q.new_zeros(B_, hk, Tn, D)
        for b in range(B_):
            P = int(past_len[b])
            if P > 0:
                pres_k[b, :, :P] = pk[b, :, :P]
                pres_v[b, :, :P] = pv[b, :, :P]
            pres_k[b, :, P:P + S_] = kh[b]
            pres_v[b, :, P:P + S_] = vh[b]
        rep = hq // hk
        kk = pres_k.repeat_interleave(rep, 1).float()
        vv = pres_v.repeat_interleave(rep, 1).float()
        scale = a.get("scale", 0.0) or 1.0 / np.sqrt(D)
        scores = qh.float() @ kk.transpose(-1, -2) * scale
        sc = a.get("softcap", 0.0)
        if sc and sc > 0:
            scores = sc * torch.tanh(scores / sc)
        qpos = past_len[:, None] + torch.arange(S_, device=q.device)[None, :]  # [B, S]
        kpos = torch.arange(Tn, device=q.device)
        keep = kpos[None, None, :] <= qpos[:, :, None]
        win = a.get("local_window_size", -1)
        if win is not None and win > 0:
            keep = keep & (kpos[None, None, :] > qpos[:, :, None] - win)
        scores = scores.masked_fill(~keep[:, None], float("-inf"))
        y = torch.softmax(scores, -1) @ vv
        return [y.transpose(1, 2).reshape(B_, S_, hq * D).to(q.dtype), pres_k, pres_v]

    @staticmethod
    def _nbits_weight(x: list, a: dict) -> torch.Tensor:
        """MatMulNBits weights [N, K]: `bits`-bit codes packed low bits first in each
        byte, blocks of `block_size` along K with one scale each, zero point per
        block (packed codes or the scales' type; 2^(bits-1) when absent)."""
        K, N, bits, bs = a["K"], a["N"], a.get("bits", 4), a["block_size"]
        if bits not in (2, 4, 8):
            raise ValueError(f"MatMulNBits with {bits}-bit codes is not supported")
        nb = (K + bs - 1) // bs
        raw = x[1].reshape(N, nb, -1).to(torch.int64)
        per = 8 // bits
        shifts = torch.arange(per, device=raw.device) * bits
        q = ((raw.unsqueeze(-1) >> shifts) & ((1 << bits) - 1)).reshape(N, nb, -1)[:, :, :bs]
        scales = x[2].reshape(N, nb).float()
        zp = x[3] if len(x) > 3 and x[3] is not None else None
        if zp is None:
            z = torch.full((N, nb), float(1 << (bits - 1)), device=raw.device)
        elif zp.dtype == torch.uint8:
            zb = zp.reshape(N, -1).to(torch.int64)
            z = ((zb.unsqueeze(-1) >> shifts) & ((1 << bits) - 1)).reshape(N, -1)[:, :nb].float()
        else:
            z = zp.reshape(N, nb).float()
        w = (q.float() - z.unsqueeze(-1)) * scales.unsqueeze(-1)
        return w.reshape(N, nb * bs)[:, :K]

    def _attention(self, x: list, a: dict):
        """Attention (opset 23): 3-D [B, S, heads * D] or 4-D [B, heads, S, D] Q/K/V,
        grouped KV heads, past key / value concatenated (present outputs), boolean
        (True attends) or additive mask, is_causal (upper-left aligned lower
        triangle), scale (default 1/sqrt(D)), softcap; qk_matmul_output_mode picks
        the 4th output (0 scores, 1 + mask, 2 + softcap, 3 softmax)."""
        Q, K, V = x[0], x[1], x[2]
        mask = x[3] if len(x) > 3 and x[3] is not None else None
        pk = x[4] if len(x) > 4 and x[4] is not None else None
        pv = x[5] if len(x) > 5 and x[5] is not None else None
        three = Q.dim() == 3
        if three:
            hq, hk = a["q_num_heads"], a["kv_num_heads"]
            B_ = Q.shape[0]
            Q = Q.reshape(B_, Q.shape[1], hq, -1).transpose(1, 2)
            K = K.reshape(B_, K.shape[1], hk, -1).transpose(1, 2)
            V = V.reshape(B_, V.shape[1], hk, -1).transpose(1, 2)
        if pk is not None:
            K = torch.cat([pk, K], 2)
        if pv is not None:
            V = torch.cat([pv, V], 2)
        present_k, present_v = K, V
        hq, hk = Q.shape[1], K.shape[1]
        if hq != hk:
            K = K.repeat_interleave(hq // hk, 1)
            V = V.repeat_interleave(hq // hk, 1)
        scale = a.get("scale", 1.0 / np.sqrt(Q.shape[-1]))
        qf, kf, vf = Q.float(), K.float(), V.float()
        scores = qf @ kf.transpose(-1, -2) * scale
        L, S = scores.shape[-2], scores.shape[-1]
        bias = torch.zeros(L, S, device=scores.device)
        if a.get("is_causal", 0):
            bias = bias.masked_fill(~torch.ones(L, S, dtype=torch.bool, device=scores.device).tril(), float("-inf"))
        if mask is not None:
            bias = bias + (torch.zeros(mask.shape, device=scores.device).masked_fill(~mask, float("-inf"))
                           if mask.dtype == torch.bool else mask.float())
        masked = scores + bias
        sc = a.get("softcap", 0.0)
        capped = sc * torch.tanh(masked / sc) if sc and sc > 0 else masked
        probs = torch.softmax(capped, -1)
        y = (probs @ vf).to(x[0].dtype)
        if three:
            y = y.transpose(1, 2).reshape(y.shape[0], L, -1)
        mode = a.get("qk_matmul_output_mode", 0)
        qk = [scores, masked, capped, probs][mode]
        return [y, present_k, present_v, qk]

    def _mha(self, x: list, a: dict):
        """com.microsoft MultiHeadAttention over [B, S, heads * D] query / key / value:
        optional packed bias (q, k, v), key_padding_mask ([B] valid lengths or [B, L]
        0 / 1), additive attention_bias, past key / value ([B, heads, P, D]),
        unidirectional (causal with the past offset), scale (default 1/sqrt(D));
        masked positions get mask_filter_value."""
        def opt(i):
            return x[i] if len(x) > i and x[i] is not None else None

        H = a["num_heads"]
        q, k, v = x[0], opt(1), opt(2)
        bias, kpm, ab, pk, pv = opt(3), opt(4), opt(5), opt(6), opt(7)
        B_, S_, hq = q.shape
        if bias is not None:
            dq = hq
            dk = k.shape[-1]
            q, k, v = q + bias[:dq], k + bias[dq:dq + dk], v + bias[dq + dk:]
        D = hq // H

        def heads(t):
            return t.reshape(B_, t.shape[1], H, -1).transpose(1, 2)

        qh, kh, vh = heads(q), heads(k), heads(v)
        if pk is not None:
            kh = torch.cat([pk, kh], 2)
            vh = torch.cat([pv, vh], 2)
        Lk = kh.shape[2]
        scale = a.get("scale", 0.0) or 1.0 / np.sqrt(D)
        scores = qh.float() @ kh.float().transpose(-1, -2) * scale
        fill = a.get("mask_filter_value", -10000.0)
        keep = torch.ones(B_, 1, S_, Lk, dtype=torch.bool, device=q.device)
        if kpm is not None:
            if kpm.dim() == 1:
                keep = keep & (torch.arange(Lk, device=q.device)[None, :] < kpm.long()[:, None])[:, None, None, :]
            else:
                keep = keep & (kpm != 0)[:, None, None, :]
        if a.get("unidirectional", 0):
            past = Lk - S_
            keep = keep & (torch.arange(Lk, device=q.device)[None, :] <=
                           torch.arange(S_, device=q.device)[:, None] + past)
        scores = torch.where(keep, scores, torch.full_like(scores, fill))
        if ab is not None:
            scores = scores + ab.float()
        y = torch.softmax(scores, -1) @ vh.float()
        return [y.transpose(1, 2).reshape(B_, S_, -1).to(q.dtype), kh, vh]

    @staticmethod
    def _resize_weights(n_in: int, n_out: int, scale: float, mode: str, ctm: str, nearest_mode: str, cubic_a: float,
                        exclude_outside: int, roi: tuple) -> tuple:
        """[n_out, n_in] interpolation matrix of one axis (ONNX Resize): output index
        -> input coordinate by the coordinate transformation mode, then nearest
        (rounded by nearest_mode), linear (2 taps) or cubic (4 taps, Keys kernel with
        coefficient a) weights on clamped neighbour indices (edge values beyond the
        border; exclude_outside zeroes and renormalises the outside taps).  Returns
        the matrix and a mask of rows outside a tf_crop_and_resize window."""
        Wm = np.zeros((n_out, n_in), np.float64)
        outside = np.zeros(n_out, bool)
        for o in range(n_out):
            if ctm == "half_pixel":
                xo = (o + 0.5) / scale - 0.5
            elif ctm == "pytorch_half_pixel":
                xo = (o + 0.5) / scale - 0.5 if n_out > 1 else 0.0
            elif ctm == "align_corners":
                xo = 0.0 if n_out == 1 else o * (n_in - 1) / (n_out - 1)
            elif ctm == "asymmetric":
                xo = o / scale
            elif ctm == "half_pixel_symmetric":
                adj = n_out / (scale * n_in)
                xo = n_in / 2 * (1 - adj) + (o + 0.5) / scale - 0.5
            elif ctm == "tf_crop_and_resize":
                st, en = roi
                xo = st * (n_in - 1) + o * (en - st) * (n_in - 1) / (n_out - 1) if n_out > 1 else \
                    0.5 * (st + en) * (n_in - 1)
                if xo < 0 or xo > n_in - 1:
                    outside[o] = True
                    continue
            else:
                raise ValueError(f"unsupported coordinate_transformation_mode {ctm}")
            base = int(np.floor(xo))
            r = xo - base
            if mode == "nearest":
                if nearest_mode == "round_prefer_floor":
                    pick = base if r <= 0.5 else base + 1
                elif nearest_mode == "round_prefer_ceil":
                    pick = base if r < 0.5 else base + 1
                elif nearest_mode == "floor":
                    pick = base
                elif nearest_mode == "ceil":
                    pick = base if r == 0 else base + 1
                else:
                    raise ValueError(f"unsupported nearest_mode {nearest_mode}")
                Wm[o, min(max(pick, 0), n_in - 1)] = 1.0
                continue
            if mode == "linear":
                taps, coef = [base, base + 1], [1 - r, r]
            elif mode == "cubic":
                A = cubic_a

                def k(t):  # Keys (1981) cubic convolution kernel
                    t = abs(t)
                    if t <= 1:
                        return ((A + 2) * t - (A + 3)) * t * t + 1
                    if t < 2:
                        return ((A * t - 5 * A) * t + 8 * A) * t - 4 * A
                    return 0.0
                taps = [base - 1, base, base + 1, base + 2]
                coef = [k(r + 1), k(r), k(1 - r), k(2 - r)]
            else:
                raise ValueError(f"unsupported Resize mode {mode}")
            if exclude_outside:
                coef = [c if 0 <= t < n_in else 0.0 for t, c in zip(taps, coef)]
                tot = sum(coef)
                coef = [c / tot for c in coef] if tot else coef
            for t, c in zip(taps, coef):
                Wm[o, min(max(t, 0), n_in - 1)] += c
        return Wm, outside

    def _resize(self, X, roi, scales, sizes, mode, ctm, nearest_mode, cubic_a, exclude_outside, extrapolation,
                axes=None, keep_aspect="stretch", antialias=0):
        """ONNX Resize (and Upsample) as one interpolation matrix per resized axis."""
        nd = X.dim()
        axes = [ax % nd for ax in axes] if axes else list(range(nd))
        ins = [X.shape[ax] for ax in axes]
        if sizes is not None:
            want = [int(v) for v in sizes.tolist()]
            sc = [w / i for w, i in zip(want, ins)]
            if keep_aspect != "stretch":
                pick = min(sc) if keep_aspect == "not_larger" else max(sc)
                sc = [pick] * len(sc)
                want = [int(np.floor(pick * i + 0.5)) for i in ins]
        else:
            sc = [float(v) for v in scales.tolist()]
            want = None
        rois = [(0.0, 1.0)] * len(axes)
        if roi is not None:
            rv = [float(v) for v in roi.tolist()]
            h = len(rv) // 2
            rois = list(zip(rv[:h], rv[h:]))
            if h == nd and len(axes) != nd:
                rois = [rois[ax] for ax in axes]
        if want is None:
            want = [int(np.floor(i * s * ((en - st) if ctm == "tf_crop_and_resize" else 1.0)))
                    for i, s, (st, en) in zip(ins, sc, rois)]
        y = X
        for ax, n_in, n_out, s, r in zip(axes, ins, want, sc, rois):
            if n_in == n_out and s == 1.0 and ctm != "tf_crop_and_resize":
                continue
            if antialias and s < 1 and mode != "nearest":
                raise ValueError("Resize with antialias on a downscaled axis is not supported")
            Wm, outside = self._resize_weights(n_in, n_out, s, mode, ctm, nearest_mode, cubic_a, exclude_outside, r)
            moved = y.movedim(ax, -1)
            if mode == "nearest" and not outside.any():
                idx = torch.from_numpy(Wm.argmax(1)).to(y.device)
                out = moved.index_select(-1, idx)
            else:
                out = (moved.double() @ torch.from_numpy(Wm.T).to(y.device)).to(y.dtype)
                if outside.any():
                    out[..., torch.from_numpy(outside).to(y.device)] = extrapolation
            y = out.movedim(-1, ax)
        return y

    def _nms(self, x: list, a: dict) -> torch.Tensor:
        """NonMaxSuppression: per batch and class, boxes above score_threshold in
        descending score order, each kept unless its IoU with a kept box exceeds
        iou_threshold, at most max_output_boxes_per_class; rows (batch, class, box)."""
        boxes, scores = x[0].double().cpu(), x[1].double().cpu()
        mx = int(x[2].reshape(-1)[0]) if len(x) > 2 and x[2] is not None and x[2].numel() else 0
        iou_t = float(x[3].reshape(-1)[0]) if len(x) > 3 and x[3] is not None and x[3].numel() else 0.0
        sc_t = float(x[4].reshape(-1)[0]) if len(x) > 4 and x[4] is not None and x[4].numel() else None
        if a.get("center_point_box", 0):
            cx, cy, w, h = boxes.unbind(-1)
            y1, x1, y2, x2 = cy - h / 2, cx - w / 2, cy + h / 2, cx + w / 2
        else:
            ya, xa, yb, xb = boxes.unbind(-1)
            y1, y2 = torch.minimum(ya, yb), torch.maximum(ya, yb)
            x1, x2 = torch.minimum(xa, xb), torch.maximum(xa, xb)
        area = (y2 - y1) * (x2 - x1)
        out = []
        for b in range(scores.shape[0]):
            for c in range(scores.shape[1]):
                sc = scores[b, c]
                order = sorted(range(sc.numel()), key=lambda i: -float(sc[i]))
                kept: list = []
                for i in order:
                    if len(kept) >= mx:
                        break
                    if sc_t is not None and not float(sc[i]) > sc_t:
                        break
                    ok = True
                    for j in kept:
                        ih = min(float(y2[b, i]), float(y2[b, j])) - max(float(y1[b, i]), float(y1[b, j]))
                        iw = min(float(x2[b, i]), float(x2[b, j])) - max(float(x1[b, i]), float(x1[b, j]))
                        inter = max(ih, 0.0) * max(iw, 0.0)
                        union = float(area[b, i]) + float(area[b, j]) - inter
                        if union > 0 and inter / union > iou_t:
                            ok = False
                            break
                    if ok:
                        kept.append(i)
                out += [[b, c, i] for i in kept]
        return torch.tensor(out, dtype=torch.int64, device=x[0].device).reshape(-1, 3)


# ------------------------------------------------------------------ LLMs
def load_onnx_llm(path: str, root: str, device, tp: int = 1, rank: int = 0):
    """LLM weights from an ONNX export whose initializers keep HF names."""
    from ..models.config import ModelConfig
    from ..models.cpu_model import CPUCausalLM
    from ..models.llama import weights_from_full

    model = read_model(path)
    if "model.embed_tokens.weight" not in model.initializers:
        raise ValueError("ONNX export lacks initializer model.embed_tokens.weight; only exports keeping HF tensor "
                         "names are supported")
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


def encode_model(nodes: list, inputs: list, outputs: list, initializers: dict, opset: int = 13,
                 input_types: Optional[dict] = None) -> bytes:
    """Minimal ModelProto writer (for tests and synthetic exports).  A node
    attribute given as an :class:`OnnxModel` is written as a subgraph."""
    g = _encode_graph(nodes, inputs, outputs, initializers, input_types)
    return _key(1, 0) + _enc_varint(8) + _ld(2, b"kapsl") + _ld(7, g) + _ld(8, _key(2, 0) + _enc_varint(opset))


def _encode_graph(nodes: list, inputs: list, outputs: list, initializers: dict, input_types: Optional[dict] = None
                  ) -> bytes:
    g = b""
    for n in nodes:
        nb = b"".join(_ld(1, i.encode()) for i in n.inputs) + b"".join(_ld(2, o.encode()) for o in n.outputs)
        nb += _ld(3, (n.name or n.op).encode()) + _ld(4, n.op.encode())
        if n.domain:
            nb += _ld(7, n.domain.encode())
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
            elif isinstance(v, OnnxModel):
                ab += _ld(6, _encode_graph(v.nodes, v.inputs, v.outputs, v.initializers)) + _key(20, 0) + _enc_varint(5)
            nb += _ld(5, ab)
        g += _ld(1, nb)
    g += _ld(2, b"graph")
    for k, v in initializers.items():
        g += _ld(5, encode_tensor(k, v))
    for i in inputs:
        vi = _ld(1, i.encode())
        if input_types and i in input_types:  # TypeProto.Tensor: element type and shape
            elem, dims = input_types[i]
            shp = b"".join(_ld(1, _key(1, 0) + _enc_varint(d) if d is not None else _ld(2, b"n")) for d in dims)
            vi += _ld(2, _ld(1, _key(1, 0) + _enc_varint(elem) + _ld(2, shp)))
        g += _ld(11, vi)
    for o in outputs:
        g += _ld(12, _ld(1, o.encode()))
    return g
