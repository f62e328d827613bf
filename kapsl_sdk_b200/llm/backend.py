"""LLMBackend: the serving :class:`~kapsl_sdk_b200.engine_api.Engine` over
:class:`~kapsl_sdk_b200.llm.engine.LLMEngine`.

Mirrors crates/kapsl-llm/src/llm_backend.rs:
* runtime config from the model directory: ``generation_config.json``
  (temperature, max_new_tokens / max_length, top_p, top_k, repetition_penalty,
  eos/bos stop ids), ``config.json`` (eos/bos fallback), ``chat_template.jinja``
  (Llama-3 header format, or generic ``<|user|>``/``<|assistant|>`` tags, plus a
  ``<think>`` suffix when the template has one) and ``tokenizer.json``
  (llm_backend.rs:72-321);
* defaults 512 new tokens, T 0.7, top_p 0.9, top_k 40, penalty 1.15 (55-65);
* ``infer_stream`` accepts only ``string`` input, wraps the chat template,
  applies metadata overrides (max_new_tokens, temperature, top_p, top_k,
  repetition_penalty, seed, stop_token_ids appended), picks the request id from
  metadata, then session id, then a uuid, and yields incremental UTF-8 text
  deltas as ``[1, len]`` string packets (576-736); ``infer`` concatenates them.

One engine thread owns the LLMEngine: it drains a request queue, steps the
engine, and pushes per-request outputs to per-request queues (the role of the
tokio task and mpsc channels in the reference).
"""
from __future__ import annotations

import json
import os
import queue
import threading
import time
import uuid
from dataclasses import dataclass, field, replace
from typing import Iterator, Optional

import numpy as np

from ..engine_api import (BinaryTensorPacket, Engine, EngineError, EngineMetrics, EngineModelInfo,
                          InferenceRequest, TensorDtype)
from .sequence import SamplingParams


@dataclass
class RuntimeConfig:
    use_chat_template: bool = False
    prompt_prefix: str = ""
    prompt_suffix: str = ""
    sampling: SamplingParams = field(default_factory=SamplingParams)
    add_bos: bool = False


def _read_json(path: str) -> Optional[dict]:
    try:
        with open(path) as f:
            return json.load(f)
    except (OSError, ValueError):
        return None


def find_model_asset(root: str, name: str) -> Optional[str]:
    """Reference crates/kapsl-llm/src/model_paths.rs: look in the root and ``onnx-export/``."""
    for p in (os.path.join(root, name), os.path.join(root, "onnx-export", name)):
        if os.path.isfile(p):
            return p
    return None


def _stop_ids(obj: dict) -> list:
    out = []

    def push(v):
        if isinstance(v, int) and v not in out:
            out.append(v)

    for v in obj.get("eos_token_ids") or []:
        push(v)
    e = obj.get("eos_token_id")
    for v in (e if isinstance(e, list) else [e]):
        push(v)
    push(obj.get("bos_token_id"))
    return out


def load_runtime_config(model_dir: Optional[str]) -> RuntimeConfig:
    rc = RuntimeConfig()
    if not model_dir:
        return rc
    s = rc.sampling
    gen = _read_json(find_model_asset(model_dir, "generation_config.json") or "")
    if gen:
        if isinstance(gen.get("temperature"), (int, float)):
            s.temperature = float(gen["temperature"])
        if gen.get("max_new_tokens"):
            s.max_new_tokens = int(gen["max_new_tokens"])
        elif gen.get("max_length"):
            s.max_new_tokens = int(gen["max_length"])
        if isinstance(gen.get("top_p"), (int, float)):
            s.top_p = float(gen["top_p"])
        if isinstance(gen.get("top_k"), int):
            s.top_k = int(gen["top_k"])
        if isinstance(gen.get("repetition_penalty"), (int, float)):
            s.repetition_penalty = float(gen["repetition_penalty"])
        ids = _stop_ids(gen)
        if ids:
            s.stop_token_ids = ids
    cfg = _read_json(find_model_asset(model_dir, "config.json") or "")
    if not s.stop_token_ids and cfg:
        s.stop_token_ids = _stop_ids(cfg)
    tpl_path = find_model_asset(model_dir, "chat_template.jinja")
    tok = _read_json(find_model_asset(model_dir, "tokenizer.json") or "")
    if tpl_path:
        with open(tpl_path) as f:
            tpl = f.read()
        think = "<think>\n" if "<think>" in tpl else ""
        rc.use_chat_template = True
        if "<|start_header_id|>" in tpl and "<|end_header_id|>" in tpl and "<|eot_id|>" in tpl:
            bos = ""
            bos_id = (cfg or {}).get("bos_token_id")
            for t in (tok or {}).get("added_tokens", []):
                if t.get("id") == bos_id:
                    bos = t.get("content", "")
            rc.prompt_prefix = f"{bos}<|start_header_id|>user<|end_header_id|>\n\n"
            rc.prompt_suffix = f"<|eot_id|><|start_header_id|>assistant<|end_header_id|>\n\n{think}"
        else:
            user = _find_tag(tpl, "user") or "<|user|>"
            asst = _find_tag(tpl, "assistant") or "<|assistant|>"
            rc.prompt_prefix = f"{user}\n"
            rc.prompt_suffix = f"\n{asst}\n{think}"
    return rc


def _find_tag(template: str, label: str) -> Optional[str]:
    i = 0
    low = label.lower()
    while True:
        a = template.find("<", i)
        if a < 0:
            return None
        b = template.find(">", a)
        if b < 0:
            return None
        tag = template[a:b + 1]
        if low in tag.lower():
            return tag
        i = b + 1


def _native_mod():
    try:
        from .._ext import native

        return native()
    except Exception:  # pragma: no cover - the native module is part of the build
        return None


class _Pending:
    __slots__ = ("request_id", "prompt_ids", "params", "session_id", "out", "cancel", "seq", "channel")

    def __init__(self, request_id, prompt_ids, params, session_id, cancel, channel=None):
        self.request_id = request_id
        self.prompt_ids = prompt_ids
        self.params = params
        self.session_id = session_id
        self.out: "queue.Queue" = queue.Queue()
        self.cancel = cancel
        self.seq = None
        # native TokenChannel of a token-id stream served by the native server, else None
        self.channel = channel

    def fail(self, err) -> None:
        if self.channel is not None:
            self.channel.fail(str(err))
        else:
            self.out.put(err)

    def cancelled(self) -> bool:
        return (self.cancel is not None and self.cancel.is_cancelled()) or \
            (self.channel is not None and self.channel.cancelled())


class LLMBackend(Engine):
    """Engine over an LLMEngine run by a dedicated thread.

    ``load(path)`` builds the model on that thread, so all of a CPU model's
    compute happens on one thread and uses one OpenMP worker team (PyTorch's
    libgomp throttles its workers when two threads each drive a team, which
    slows every matmul).  A caller that builds the engine itself can pass
    ``own_thread=False`` and run the loop on its own thread with :meth:`run`."""

    def __init__(self, engine=None, tokenizer=None, runtime_config: Optional[RuntimeConfig] = None,
                 admission_control: bool = False, own_thread: bool = True):
        self.engine = engine
        self.tokenizer = tokenizer
        self.rc = runtime_config or RuntimeConfig()
        self.admission_control = admission_control
        self._inbox: "queue.Queue" = queue.Queue()
        self._live: dict = {}
        self._thread: Optional[threading.Thread] = None
        self._stop = threading.Event()
        self._loop_done = threading.Event()
        self._caller_loop = False
        self._lock = threading.Lock()
        self._stats = {"requests": 0, "errors": 0, "tokens": 0, "busy_s": 0.0}
        self._peak = 0
        if engine is not None:
            self._default_tokenizer()
            if own_thread:
                self._start()

    # -------------------------------------------------------------- load
    def load(self, model_path: str) -> None:
        """Load a model directory or package (see :mod:`kapsl_sdk_b200.runtime.loader`)
        on the engine thread, which then serves it."""
        from ..runtime.loader import build_llm_engine

        ready, err = threading.Event(), []

        def body():
            try:
                self.engine, self.tokenizer, self.rc = build_llm_engine(model_path)
                self._default_tokenizer()
            except BaseException as e:  # reported to the caller of load()
                err.append(e)
                return
            finally:
                ready.set()
            self._loop()

        self._stop.clear()
        self._thread = threading.Thread(target=body, name="kapsl-llm-engine", daemon=True)
        self._thread.start()
        ready.wait()
        if err:
            self._thread.join()
            self._thread = None
            raise err[0]

    def run(self) -> None:
        """Serve on the calling thread until :meth:`unload` (for ``own_thread=False``)."""
        self._stop.clear()
        self._caller_loop = True
        self._loop_done.clear()
        self._thread = threading.current_thread()
        try:
            self._loop()
        finally:
            self._loop_done.set()

    def _default_tokenizer(self) -> None:
        if self.tokenizer is None:
            from .tokenizer import ByteTokenizer

            c = self.engine.cfg
            self.tokenizer = ByteTokenizer(c.vocab_size, c.bos_token_id, c.eos_token_id)

    def _start(self) -> None:
        self._stop.clear()
        self._thread = threading.Thread(target=self._loop, name="kapsl-llm-engine", daemon=True)
        self._thread.start()

    def unload(self) -> None:
        self._stop.set()
        t = self._thread
        if t is not None and t is not threading.current_thread():
            if self._caller_loop:  # run() on a caller's thread: wait for the loop, not the thread
                self._loop_done.wait(timeout=30)
            else:
                t.join(timeout=30)
        self._thread = None
        if self.engine is not None:
            self.engine.shutdown()
        self.engine = None

    # ------------------------------------------------------------ engine loop
    def _loop(self) -> None:
        try:
            self._serve_loop()
        finally:
            # the loop ended (unload): a request still waiting for tokens gets an error
            # instead of a stream that never ends
            gone = EngineError.model_not_loaded()
            for p in list(self._live.values()):
                p.fail(gone)
            self._live.clear()
            while True:
                try:
                    self._inbox.get_nowait().fail(gone)
                except queue.Empty:
                    break

    def _serve_loop(self) -> None:
        eng = self.engine
        while not self._stop.is_set():
            drained = False
            while True:
                try:
                    p = self._inbox.get_nowait()
                except queue.Empty:
                    break
                drained = True
                try:
                    p.seq = eng.add_request(p.request_id, p.prompt_ids, p.params, session_id=p.session_id,
                                            admission_control=self.admission_control)
                    self._live[p.request_id] = p
                except EngineError as e:
                    p.fail(e)
                except Exception as e:  # pragma: no cover - defensive
                    p.fail(EngineError.backend(str(e)))
            for rid, p in list(self._live.items()):
                if p.cancelled():
                    eng.abort(rid)
                    p.fail(EngineError.cancelled("Request cancelled"))
                    del self._live[rid]
            if not eng.has_unfinished():
                if not drained:
                    time.sleep(0.002)
                continue
            t0 = time.perf_counter()
            try:
                outs = eng.step()
            except Exception as e:
                # a failed batch fails only the requests in it (reference engine.rs:2501-2534)
                err = e if isinstance(e, EngineError) else EngineError.inference(f"LLM execution error: {e}")
                for rid, p in list(self._live.items()):
                    eng.abort(rid)
                    p.fail(err)
                    del self._live[rid]
                continue
            self._stats["busy_s"] += time.perf_counter() - t0
            self._peak = max(self._peak, len(self._live))
            chans, ctoks, cfins = [], [], []
            for o in outs:
                p = self._live.get(o.request_id)
                if p is None:
                    continue
                if p.channel is not None:
                    chans.append(p.channel)
                    ctoks.append(int(o.new_token))
                    cfins.append(bool(o.finished))
                else:
                    p.out.put((o.new_token, o.finished, o.seq.finish_reason))
                self._stats["tokens"] += 1
                if o.finished:
                    del self._live[o.request_id]
            if chans:  # one native call for every channel-streamed token of the step
                _native_mod().push_tokens(chans, ctoks, cfins)

    # ------------------------------------------------------------- serving
    def _params_for(self, request: InferenceRequest) -> SamplingParams:
        s = replace(self.rc.sampling, stop_token_ids=list(self.rc.sampling.stop_token_ids))
        m = request.metadata
        if m is not None:
            if m.max_new_tokens:
                s.max_new_tokens = int(m.max_new_tokens)
            if m.temperature is not None:
                s.temperature = float(m.temperature)
            if m.top_p is not None:
                s.top_p = float(m.top_p)
            if m.top_k is not None:
                s.top_k = int(m.top_k)
            if m.repetition_penalty is not None:
                s.repetition_penalty = float(m.repetition_penalty)
            if m.seed is not None:
                s.seed = int(m.seed)
            for t in m.stop_token_ids or []:
                if t not in s.stop_token_ids:
                    s.stop_token_ids.append(int(t))
            if m.priority is not None:
                s.priority = int(m.priority)
        return s

    def infer_stream_native(self, request: InferenceRequest):
        """A token-id request (int32 / int64 input) as a native ``TokenChannel`` the
        native server streams from without the GIL (the same frames as
        :meth:`infer_stream`: one int32 [1, 1] chunk per token, then END, or ERR
        and END); ``None`` for text requests or without the native module."""
        if request.input.dtype not in (TensorDtype.INT32, TensorDtype.INT64):
            return None
        nat = _native_mod()
        if nat is None or not hasattr(nat, "TokenChannel"):
            return None
        if self.engine is None:
            raise EngineError.model_not_loaded()
        ids = np.frombuffer(request.input.data, dtype=np.int32 if request.input.dtype is TensorDtype.INT32
                            else np.int64).astype(np.int64).tolist()
        if not ids:
            raise EngineError.invalid_input("empty prompt")
        rid = (request.metadata.request_id if request.metadata and request.metadata.request_id else None) \
            or request.session_id or str(uuid.uuid4())
        ch = nat.TokenChannel()
        p = _Pending(rid, ids, self._params_for(request), request.session_id, request.cancellation, channel=ch)
        self._stats["requests"] += 1
        self._inbox.put(p)
        return ch

    def infer_stream(self, request: InferenceRequest) -> Iterator[BinaryTensorPacket]:
        """Utf8 input -> streamed text deltas (the reference's behaviour).  An int32 or
        int64 input is taken as prompt token ids (no template, no BOS) and the
        stream carries each new token id as an int32 [1, 1] packet; the
        reference accepts text only."""
        if self.engine is None:
            raise EngineError.model_not_loaded()
        as_ids = request.input.dtype in (TensorDtype.INT32, TensorDtype.INT64)
        if as_ids:
            ids = np.frombuffer(request.input.data, dtype=np.int32 if request.input.dtype is TensorDtype.INT32
                                else np.int64).astype(np.int64).tolist()
        else:
            if request.input.dtype is not TensorDtype.UTF8:
                raise EngineError.invalid_input("LLM backend expects Utf8 input")
            try:
                prompt = request.input.data.decode("utf-8")
            except UnicodeDecodeError:
                raise EngineError.invalid_input("Invalid UTF-8 input")
            if self.rc.use_chat_template:
                prompt = f"{self.rc.prompt_prefix}{prompt}{self.rc.prompt_suffix}"
            ids = self.tokenizer.encode(prompt, add_bos=self.rc.add_bos)
        if not ids:
            raise EngineError.invalid_input("empty prompt")
        rid = (request.metadata.request_id if request.metadata and request.metadata.request_id else None) \
            or request.session_id or str(uuid.uuid4())
        p = _Pending(rid, ids, self._params_for(request), request.session_id, request.cancellation)
        self._stats["requests"] += 1
        self._inbox.put(p)
        return self._stream_ids(p) if as_ids else self._stream(p)

    def _stream_ids(self, p: _Pending) -> Iterator[BinaryTensorPacket]:
        finished = False
        try:
            while True:
                item = p.out.get()
                if isinstance(item, EngineError):
                    self._stats["errors"] += 1
                    raise item
                tok, done, reason = item
                yield BinaryTensorPacket([1, 1], TensorDtype.INT32, np.int32(tok).tobytes())
                if done:
                    finished = True
                    return
        finally:
            if not finished and p.cancel is None:
                from ..engine_api import CancellationToken

                tok = CancellationToken()
                tok.cancel()
                p.cancel = tok

    def _stream(self, p: _Pending) -> Iterator[BinaryTensorPacket]:
        toks: list = []
        emitted = ""
        finished = False
        try:
            while True:
                item = p.out.get()
                if isinstance(item, EngineError):
                    self._stats["errors"] += 1
                    raise item
                tok, done, reason = item
                toks.append(tok)
                text = self.tokenizer.decode(toks)
                if text.startswith(emitted):
                    chunk, emitted = text[len(emitted):], text
                else:
                    chunk = text
                    emitted += text
                if chunk:
                    b = chunk.encode("utf-8")
                    yield BinaryTensorPacket([1, len(b)], TensorDtype.UTF8, b)
                if done:
                    finished = True
                    return
        finally:
            if not finished and p.cancel is None:
                # consumer went away: the engine thread sees the token and aborts the request
                from ..engine_api import CancellationToken

                tok = CancellationToken()
                tok.cancel()
                p.cancel = tok

    def infer(self, request: InferenceRequest) -> BinaryTensorPacket:
        text = b"".join(pkt.data for pkt in self.infer_stream(request))
        return BinaryTensorPacket([1, max(len(text), 1)], TensorDtype.UTF8, text)

    # ------------------------------------------------------------- metrics
    def metrics(self) -> EngineMetrics:
        m = EngineMetrics()
        if self.engine is not None:
            kv = self.engine.kv_stats()
            m.kv_cache_bytes_used = kv["bytes_used"]
            m.kv_cache_bytes_capacity = kv["bytes_capacity"]
            m.kv_cache_blocks_total = kv["blocks_total"]
            m.kv_cache_blocks_free = kv["blocks_free"]
            m.kv_cache_sequences = kv["sequences"]
            m.kv_cache_evicted_blocks = kv["evicted_blocks_total"]
            m.queue_depth = len(self._live) + self._inbox.qsize()
        m.error_rate = self._stats["errors"] / max(1, self._stats["requests"])
        m.throughput = self._stats["tokens"] / max(1e-9, self._stats["busy_s"])
        return m

    def model_info(self) -> EngineModelInfo:
        return EngineModelInfo(input_names=["prompt"], output_names=["text"], input_shapes=[[1, -1]],
                               output_shapes=[[1, -1]], input_dtypes=["string"], output_dtypes=["string"],
                               framework="llm", peak_concurrency=max(1, self._peak))

    def health_check(self) -> bool:
        eng = self.engine
        return (eng is not None and self._thread is not None and self._thread.is_alive()
                and getattr(eng, "failed", None) is None)
