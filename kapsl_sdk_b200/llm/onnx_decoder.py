"""LLM serving of ONNX decoder exports whose weights this framework cannot map
onto its own model (block-quantized MatMulNBits weights, fused contrib attention,
renamed initializers): the graph itself runs through the ONNX interpreter, one
sequence at a time, with each sequence's KV cache kept as the graph's present
tensors and fed back as its past inputs on the next step.

The input / output naming is that of decoder exports (``input_ids``,
``attention_mask``, ``position_ids``, ``past_key_values.{i}.key|value`` ->
``logits``, ``present.{i}.key|value``), which is how the reference engine drives
ONNX Runtime decoder sessions (crates/kapsl-llm/src/engine.rs:1054-2100 load and
geometry, 3170-3914 decode).  Sampling, stop ids and seeds follow the reference
sampler (engine.rs:5817-5927; penalty 3104-3123).  Exports that keep Hugging Face
initializer names load onto the native model instead
(``loaders.onnx.load_onnx_llm``).

:class:`OnnxDecoderEngine` has the engine interface :class:`~.backend.LLMBackend`
drives (``add_request`` / ``step`` / ``abort`` / ``has_unfinished`` / ``kv_stats``).
"""
from __future__ import annotations

import collections
import json
import os
import re
import types
from dataclasses import dataclass, field
from typing import Optional

import numpy as np
import torch

from ..engine_api import EngineError
from ..loaders.onnx import OnnxGraph, OnnxModel, read_model
from ..ops import reference as ref
from .sequence import SamplingParams

_PAST = re.compile(r"^past_key_values\.(\d+)\.(key|value)$")
_PRESENT = re.compile(r"^present\.(\d+)\.(key|value)$")


@dataclass
class DecoderIO:
    input_ids: str
    logits: str
    attention_mask: Optional[str] = None
    position_ids: Optional[str] = None
    past: list = field(default_factory=list)      # [(key input, value input)] per layer
    present: list = field(default_factory=list)   # [(key output, value output)] per layer


def inspect_decoder(model: OnnxModel) -> Optional[DecoderIO]:
    """The decoder inputs / outputs of a graph, or None when it is not a decoder export."""
    if "input_ids" not in model.inputs or "logits" not in model.outputs:
        return None
    io = DecoderIO("input_ids", "logits")
    io.attention_mask = "attention_mask" if "attention_mask" in model.inputs else None
    io.position_ids = "position_ids" if "position_ids" in model.inputs else None
    past, present = {}, {}
    for name in model.inputs:
        m = _PAST.match(name)
        if m:
            past.setdefault(int(m.group(1)), {})[m.group(2)] = name
    for name in model.outputs:
        m = _PRESENT.match(name)
        if m:
            present.setdefault(int(m.group(1)), {})[m.group(2)] = name
    if sorted(past) != sorted(present) or any(len(v) != 2 for v in list(past.values()) + list(present.values())):
        raise ValueError("decoder export: past_key_values.* inputs and present.* outputs do not pair up")
    io.past = [(past[i]["key"], past[i]["value"]) for i in sorted(past)]
    io.present = [(present[i]["key"], present[i]["value"]) for i in sorted(present)]
    return io


def _geometry(root: str, model: OnnxModel) -> dict:
    """KV heads, head size, vocabulary, special ids and context length from
    genai_config.json or config.json next to the model."""
    g = {}
    gp = os.path.join(root, "genai_config.json")
    if os.path.isfile(gp):
        with open(gp) as f:
            m = json.load(f).get("model", {})
        d = m.get("decoder", {})
        g.update(kv_heads=d.get("num_key_value_heads"), head_dim=d.get("head_size"), vocab=m.get("vocab_size"),
                 bos=m.get("bos_token_id"), eos=m.get("eos_token_id"), ctx=m.get("context_length"))
    cp = os.path.join(root, "config.json")
    if os.path.isfile(cp):
        with open(cp) as f:
            c = json.load(f)
        heads = c.get("num_attention_heads")
        g.setdefault("kv_heads", None)
        g["kv_heads"] = g["kv_heads"] or c.get("num_key_value_heads") or heads
        g["head_dim"] = g.get("head_dim") or c.get("head_dim") or (
            c["hidden_size"] // heads if heads and c.get("hidden_size") else None)
        g["vocab"] = g.get("vocab") or c.get("vocab_size")
        g["bos"] = g.get("bos") if g.get("bos") is not None else c.get("bos_token_id")
        g["eos"] = g.get("eos") if g.get("eos") is not None else c.get("eos_token_id")
        g["ctx"] = g.get("ctx") or c.get("max_position_embeddings")
    if not g.get("kv_heads") or not g.get("head_dim"):
        raise ValueError("decoder export: KV geometry needs genai_config.json or config.json next to the model")
    if isinstance(g.get("eos"), list):
        g["eos_list"] = [int(v) for v in g["eos"]]
        g["eos"] = g["eos_list"][0] if g["eos_list"] else None
    floats = [v for v in model.initializers.values() if v.dtype in (np.float16, np.float32)]
    g["dtype"] = torch.float16 if floats and max(floats, key=lambda v: v.size).dtype == np.float16 else torch.float32
    return g


@dataclass
class _Seq:
    request_id: str
    prompt_ids: list      # this turn's prompt, after any session history
    params: SamplingParams
    rng: int
    output_ids: list = field(default_factory=list)
    past: Optional[list] = None   # [(key, value)] per layer covering the first `cached` tokens
    cached: int = 0
    session_id: Optional[str] = None
    finish_reason: Optional[str] = None

    @property
    def length(self) -> int:
        return len(self.prompt_ids) + len(self.output_ids)


class OnnxDecoderEngine:
    def __init__(self, model_path: str, root: Optional[str] = None, device: str = "cpu",
                 max_model_len: Optional[int] = None, max_sessions: int = 64, max_session_tokens: int = 0):
        self.model = read_model(model_path)
        io = inspect_decoder(self.model)
        if io is None:
            raise ValueError("not a decoder export (needs an input_ids input and a logits output)")
        self.io = io
        self.device = torch.device(device)
        self.graph = OnnxGraph(self.model, self.device)
        g = _geometry(root or os.path.dirname(os.path.abspath(model_path)), self.model)
        self.geom = g
        self.cfg = types.SimpleNamespace(vocab_size=int(g.get("vocab") or 0), bos_token_id=g.get("bos"),
                                         eos_token_id=g.get("eos"), max_position=int(g.get("ctx") or 4096))
        self.max_model_len = min(max_model_len or self.cfg.max_position, self.cfg.max_position)
        self.stop_ids = set(x for x in (g.get("eos"), g.get("bos")) if x is not None) | set(g.get("eos_list", []))
        self.live: "dict[str, _Seq]" = {}
        self._next_seq_id = 1
        # session id -> (token ids, past KV covering all but the last, cached count); LRU
        self.sessions: "collections.OrderedDict[str, tuple]" = collections.OrderedDict()
        self.max_sessions = max_sessions
        self.max_session_tokens = max_session_tokens or self.max_model_len

    # ------------------------------------------------------------ requests
    def add_request(self, request_id: str, prompt_ids: list, params: SamplingParams, session_id=None,
                    admission_control=None, **_):
        if not prompt_ids:
            raise EngineError.invalid_input("empty prompt")
        if self.cfg.vocab_size and any(not 0 <= t < self.cfg.vocab_size for t in prompt_ids):
            raise EngineError.invalid_input("prompt token id outside the vocabulary")
        seq_id = self._next_seq_id
        self._next_seq_id += 1
        ids, past, cached = list(prompt_ids), None, 0
        prev = self.sessions.get(session_id) if session_id is not None else None
        if prev is not None:
            # continue the session: the new turn follows the previous turn's tokens, whose
            # KV (all but the last token) is reused
            hist, hpast, hcached = prev
            if len(hist) + len(ids) + params.max_new_tokens <= self.max_session_tokens:
                ids, past, cached = hist + ids, hpast, hcached
            self.sessions.move_to_end(session_id)
        if len(ids) >= self.max_model_len:
            raise EngineError.invalid_input(f"prompt of {len(ids)} tokens exceeds the context ({self.max_model_len})")
        s = _Seq(request_id, ids, params, ref.seed_state(params.seed, request_id, seq_id), past=past, cached=cached,
                 session_id=session_id)
        self.live[request_id] = s
        return s

    def has_unfinished(self) -> bool:
        return bool(self.live)

    def abort(self, request_id: str) -> None:
        s = self.live.pop(request_id, None)
        if s is not None:
            s.finish_reason = "aborted"

    # ---------------------------------------------------------------- step
    def _feeds(self, s: _Seq) -> dict:
        new = (s.prompt_ids + s.output_ids)[s.cached:]
        past_len = s.cached
        n = len(new)
        feeds = {self.io.input_ids: torch.tensor([new], dtype=torch.int64)}
        if self.io.attention_mask:
            feeds[self.io.attention_mask] = torch.ones(1, past_len + n, dtype=torch.int64)
        if self.io.position_ids:
            feeds[self.io.position_ids] = torch.arange(past_len, past_len + n, dtype=torch.int64)[None]
        H, D, dt = self.geom["kv_heads"], self.geom["head_dim"], self.geom["dtype"]
        for li, (kn, vn) in enumerate(self.io.past):
            if s.past is None:
                feeds[kn] = torch.zeros(1, H, 0, D, dtype=dt)
                feeds[vn] = torch.zeros(1, H, 0, D, dtype=dt)
            else:
                feeds[kn], feeds[vn] = s.past[li]
        return feeds

    def _stop(self, s: _Seq, tok: int) -> Optional[str]:
        p = s.params
        if not p.ignore_eos and (tok in self.stop_ids or tok in p.stop_token_ids):
            return "stop"
        if len(s.output_ids) >= p.max_new_tokens or s.length >= self.max_model_len:
            return "length"
        return None

    def step(self) -> list:
        outs = []
        for rid, s in list(self.live.items()):
            with torch.no_grad():
                res = self.graph.run(self._feeds(s))
            s.past = [(res[kn], res[vn]) for kn, vn in self.io.present]
            s.cached = s.length
            logits = res[self.io.logits][0, -1].float().cpu().numpy()
            p = s.params
            if p.repetition_penalty != 1.0:
                logits = ref.apply_repetition_penalty(logits, s.prompt_ids + s.output_ids, p.repetition_penalty)
            tok, s.rng = ref.sample_next_token(logits, p.temperature, p.top_k, p.top_p, s.rng)
            s.output_ids.append(tok)
            reason = self._stop(s, tok)
            if reason is not None:
                s.finish_reason = reason
                del self.live[rid]
                if s.session_id is not None:
                    self.sessions[s.session_id] = (s.prompt_ids + s.output_ids, s.past, s.cached)
                    self.sessions.move_to_end(s.session_id)
                    while len(self.sessions) > self.max_sessions:
                        self.sessions.popitem(last=False)
            outs.append(types.SimpleNamespace(request_id=rid, new_token=tok, finished=reason is not None, seq=s))
        return outs

    def generate(self, prompts: list, params: SamplingParams) -> list:
        """Offline helper: every prompt to completion, the output ids of each."""
        seqs = [self.add_request(f"gen-{i}", ids, params) for i, ids in enumerate(prompts)]
        while self.has_unfinished():
            self.step()
        return [s.output_ids for s in seqs]

    # ------------------------------------------------------------ reporting
    def kv_stats(self) -> dict:
        used = sum(t.numel() * t.element_size() for s in self.live.values() if s.past for kv in s.past for t in kv)
        return {"blocks_total": 0, "blocks_free": 0, "bytes_capacity": used, "bytes_used": used,
                "sequences": len(self.live)}

    def shutdown(self) -> None:
        self.live.clear()
        self.sessions.clear()
