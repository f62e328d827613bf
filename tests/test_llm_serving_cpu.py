"""End-to-end LLM serving on the CPU backend: LLMEngine (chunked prefill,
paged KV, reference sampler) behind LLMBackend, served by the C++ socket
server and consumed with the C++ client SDK."""
import os
import tempfile
import time

import numpy as np
import pytest
import torch

from kapsl_sdk_b200.engine_api import BinaryTensorPacket, InferenceRequest, RequestMetadata, TensorDtype
from kapsl_sdk_b200.llm.engine import EngineConfig, LLMEngine
from kapsl_sdk_b200.llm.sequence import SamplingParams
from kapsl_sdk_b200.models.config import ModelConfig


def tiny_cfg(**kw):
    c = ModelConfig(name="t", arch="llama", vocab_size=300, hidden_size=64, intermediate_size=128, num_layers=2,
                    num_heads=4, num_kv_heads=2, head_dim=16, rope_theta=10000.0, max_position=512,
                    bos_token_id=1, eos_token_id=2)
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def cpu_engine(cfg, **kw):
    return LLMEngine(cfg, device="cpu", engine_cfg=EngineConfig(max_num_seqs=4, max_num_batched_tokens=kw.pop(
        "chunk", 32), max_model_len=256, num_blocks=64, **kw), seed=0)


def test_chunked_prefill_matches_dense_oracle():
    from kapsl_sdk_b200.models.llama import reference_forward

    cfg = tiny_cfg()
    eng = cpu_engine(cfg, chunk=16)
    prompt = list(range(5, 45))
    out = eng.generate([prompt], SamplingParams.greedy(6, ignore_eos=True))[0]
    m = eng.model
    layers = [{k: v for k, v in L.items()} for L in m.layers]
    toks = list(prompt)
    for _ in range(6):
        lg = reference_forward(cfg, layers, m.embed, m.lm_head, m.final_norm, toks)[-1]
        toks.append(int(lg.argmax()))
    assert out == toks[len(prompt):]


def test_reference_seeded_sampling_is_reproducible():
    cfg = tiny_cfg()
    p = SamplingParams(max_new_tokens=8, seed=1234, ignore_eos=True)
    a = cpu_engine(cfg).generate([[3, 4, 5, 6]], p)[0]
    b = cpu_engine(cfg).generate([[3, 4, 5, 6]], p)[0]
    assert a == b and len(a) == 8


@pytest.mark.parametrize("mode", ["recompute", "swap"])
def test_preemption_keeps_outputs(mode):
    """A pool too small for the batch forces preemptions; recomputed or swapped
    sequences continue their sampler streams, so outputs match a roomy pool."""
    cfg = tiny_cfg()
    prompts = [list(range(3 + i, 43 + i)) for i in range(4)]
    p = SamplingParams(max_new_tokens=24, ignore_eos=True)
    want = cpu_engine(cfg).generate(prompts, p)
    eng = LLMEngine(
        cfg, device="cpu", engine_cfg=EngineConfig(max_num_seqs=4, max_num_batched_tokens=32, max_model_len=256,
                                                   num_blocks=9, preemption=mode), seed=0)
    got = eng.generate(prompts, p)
    st = eng.kv_stats()
    assert got == want
    assert st["preemptions"] > 0
    if mode == "swap":
        assert st["swap_out_total"] > 0 and st["swap_in_total"] == st["swap_out_total"] and not eng._swapped_kv


def test_rollback_truncates_and_regenerates():
    """Rolling a live request back keeps the KV below the cut; greedy decoding
    then regenerates exactly the tokens that were cut."""
    cfg = tiny_cfg()
    prompt = list(range(5, 45))
    full = cpu_engine(cfg).generate([prompt], SamplingParams.greedy(12, ignore_eos=True))[0]
    eng = cpu_engine(cfg)
    seq = eng.add_request("r", prompt, SamplingParams.greedy(12, ignore_eos=True))
    while len(seq.output_ids) < 8:
        eng.step()
    blocks_before = len(seq.block_ids)
    assert eng.rollback("r", len(prompt) + 3) == 1
    assert seq.output_ids == full[:3] and seq.num_computed == len(prompt) + 2
    assert len(seq.block_ids) <= blocks_before
    while eng.has_unfinished():
        eng.step()
    assert seq.output_ids == full
    # back into the prompt: the prompt itself is cut, then generation restarts from it
    seq2 = eng.add_request("r2", prompt, SamplingParams.greedy(5, ignore_eos=True))
    while len(seq2.output_ids) < 2:
        eng.step()
    eng.rollback("r2", 30)
    assert seq2.prompt_ids == prompt[:30] and seq2.output_ids == []
    while eng.has_unfinished():
        eng.step()
    want = cpu_engine(cfg).generate([prompt[:30]], SamplingParams.greedy(5, ignore_eos=True))[0]
    assert seq2.output_ids == want
    assert eng.allocator.num_free() == eng.allocator.num_blocks


def test_session_rollback_shortens_history():
    cfg = tiny_cfg()
    eng = cpu_engine(cfg)
    s1 = eng.add_request("a", [10, 11, 12, 13], SamplingParams.greedy(4, ignore_eos=True), session_id="s")
    while eng.has_unfinished():
        eng.step()
    first = s1.output_ids[0]
    eng.rollback_session("s", 5)
    s2 = eng.add_request("b", [20], SamplingParams.greedy(2, ignore_eos=True), session_id="s")
    assert s2.prompt_ids == [10, 11, 12, 13, first, 20]


def test_sessions_continue_previous_turn():
    cfg = tiny_cfg()
    eng = cpu_engine(cfg)
    s1 = eng.add_request("a", [10, 11, 12], SamplingParams.greedy(3, ignore_eos=True), session_id="s")
    while eng.has_unfinished():
        eng.step()
    s2 = eng.add_request("b", [13], SamplingParams.greedy(2, ignore_eos=True), session_id="s")
    assert s2.prompt_ids == [10, 11, 12] + s1.output_ids + [13]
    while eng.has_unfinished():
        eng.step()
    assert s2.num_cached_prefix > 0 or len(s2.prompt_ids) < 16


def test_backend_stream_over_unix_socket():
    from kapsl_sdk import KapslClient
    from kapsl_sdk_b200.llm.backend import LLMBackend
    from kapsl_sdk_b200.server import KapslServer

    cfg = tiny_cfg(vocab_size=259 + 3)
    backend = LLMBackend(cpu_engine(cfg))
    d = tempfile.mkdtemp(prefix="kapsl-llm-")
    path = os.path.join(d, "s.sock")
    srv = KapslServer(models={0: backend}).listen_unix(path).start()
    try:
        c = KapslClient(path)
        chunks = list(c.infer_stream(0, [1, 5], "string", b"hello"))
        text = b"".join(chunks)
        assert len(chunks) >= 1
        # unary infer returns the concatenated text; greedy requests repeat exactly
        # (seeded sampling mixes in the per-request sequence id, as the reference does)
        req = InferenceRequest(BinaryTensorPacket([1, 5], TensorDtype.UTF8, b"hello"),
                               metadata=RequestMetadata(request_id="fixed", max_new_tokens=5, temperature=0.0))
        direct = backend.infer(req).data
        again = backend.infer(req).data
        assert direct == again
        with pytest.raises(RuntimeError, match="expects Utf8"):
            c.infer(0, [1], "float32", b"\0\0\0\0")
        # token-id prompts stream one int32 token per packet
        ids = np.array([5, 9, 13, 40], dtype=np.int32)
        toks = [np.frombuffer(b, np.int32)[0] for b in c.infer_stream(0, [1, 4], "int32", ids.tobytes())]
        assert 1 <= len(toks) <= backend.rc.sampling.max_new_tokens and all(0 <= t < cfg.vocab_size for t in toks)
        assert backend.health_check()
        m = backend.metrics()
        assert m.kv_cache_blocks_total == 64
    finally:
        srv.stop()
        backend.unload()


def test_token_id_streams_use_the_native_channel():
    """Token-id prompts are streamed by the native server from a TokenChannel (no
    Python generator per token): the same greedy tokens as the Python packet path,
    errors as ERR frames, and a client that hangs up mid-stream cancels its request."""
    import socket
    import time

    from kapsl_sdk import KapslClient
    from kapsl_sdk_b200._ext import native
    from kapsl_sdk_b200.llm.backend import LLMBackend
    from kapsl_sdk_b200.server import KapslServer
    from kapsl_sdk_b200.server import wire

    cfg = tiny_cfg(vocab_size=259 + 3)
    backend = LLMBackend(cpu_engine(cfg))
    backend.rc.sampling = SamplingParams.greedy(12, ignore_eos=True)
    d = tempfile.mkdtemp(prefix="kapsl-llm-")
    path = os.path.join(d, "s.sock")
    srv = KapslServer(models={0: backend}).listen_unix(path).start()
    try:
        ids = np.array([5, 9, 13, 40, 7], dtype=np.int32)
        req = InferenceRequest(BinaryTensorPacket([1, 5], TensorDtype.INT32, ids.tobytes()))
        assert isinstance(srv.dispatcher._target(0).infer_stream_native(req), native().TokenChannel)
        time.sleep(0.5)  # let that probe request finish on the engine loop
        want = [int(np.frombuffer(p.data, np.int32)[0]) for p in backend.infer_stream(req)]  # Python packets
        c = KapslClient(path)
        got = [int(np.frombuffer(b, np.int32)[0]) for b in c.infer_stream(0, [1, 5], "int32", ids.tobytes())]
        assert got == want and len(got) == 12
        with pytest.raises(RuntimeError, match="empty prompt"):
            list(c.infer_stream(0, [1, 0], "int32", b""))
        # hang up after the first chunk: the request is aborted, not run to its end
        backend.rc.sampling = SamplingParams.greedy(200, ignore_eos=True)
        s = socket.socket(socket.AF_UNIX)
        s.connect(path)
        body = wire.encode_request(([1, 5], "int32", ids.tobytes()))
        s.sendall(wire.request_header(0, wire.OP_INFER_STREAM, len(body)) + body)
        assert len(s.recv(8)) == 8
        s.close()
        t0 = time.time()
        while (backend._live or backend._inbox.qsize()) and time.time() - t0 < 20:
            time.sleep(0.05)
        assert not backend._live
        assert backend.engine.has_unfinished() is False
    finally:
        srv.stop()
        backend.unload()


def test_unload_ends_open_streams_with_an_error():
    """Unloading while requests stream: the Python stream raises and the native
    channel reports an error, instead of either waiting forever."""
    import threading

    from kapsl_sdk_b200.engine_api import EngineError
    from kapsl_sdk_b200.llm.backend import LLMBackend

    cfg = tiny_cfg(vocab_size=259 + 3)
    backend = LLMBackend(cpu_engine(cfg))
    backend.rc.sampling = SamplingParams.greedy(240, ignore_eos=True)
    ids = np.array([5, 9, 13, 40], np.int32).tobytes()
    req = InferenceRequest(BinaryTensorPacket([1, 4], TensorDtype.INT32, ids))
    ch = backend.infer_stream_native(req)
    got, err = [], []

    def consume():
        try:
            for pkt in backend.infer_stream(req):
                got.append(pkt)
        except EngineError as e:
            err.append(e)

    t = threading.Thread(target=consume)
    t.start()
    t0 = time.time()
    while not got and time.time() - t0 < 30:
        time.sleep(0.01)
    backend.unload()
    t.join(30)
    assert not t.is_alive() and err and got
    status = None
    for _ in range(200):
        status, toks, msg = ch.pop(100)
        if status in (1, 2):
            break
    assert status == 2 and msg


def test_backend_serves_on_the_callers_thread():
    """own_thread=False: the engine loop runs in run() on the calling thread
    (the thread that built the model keeps the only OpenMP team), and unload()
    from another thread ends it."""
    import threading

    from kapsl_sdk_b200.llm.backend import LLMBackend

    cfg = tiny_cfg(vocab_size=259 + 3)
    backend = LLMBackend(cpu_engine(cfg), own_thread=False)
    assert backend._thread is None
    req = InferenceRequest(BinaryTensorPacket([1, 4], TensorDtype.INT32, np.array([5, 9, 13, 40], np.int32).tobytes()),
                           metadata=RequestMetadata(max_new_tokens=4, temperature=0.0))
    out = []
    t = threading.Thread(target=lambda: (out.extend(backend.infer_stream(req)), backend.unload()))
    t.start()
    backend.run()  # returns after unload()
    t.join(30)
    assert len(out) >= 1 and not t.is_alive()


def test_backend_load_builds_on_the_engine_thread(tmp_path):
    import threading

    from kapsl_sdk_b200.llm.backend import LLMBackend
    from kapsl_sdk_b200.loaders.gguf import write_gguf_model
    from kapsl_sdk_b200.models.llama import random_full_weights

    cfg = tiny_cfg(vocab_size=320)
    p = str(tmp_path / "m.gguf")
    write_gguf_model(p, cfg, random_full_weights(cfg, torch.device("cpu"), seed=0), quant="f32")
    seen = {}
    import kapsl_sdk_b200.runtime.loader as loader

    orig = loader.build_llm_engine

    def spy(path, *a, **kw):
        seen["thread"] = threading.current_thread().name
        return orig(path, *a, **kw)

    loader.build_llm_engine = spy
    try:
        be = LLMBackend()
        be.load(p)
        assert seen["thread"] == "kapsl-llm-engine" and be.health_check()
        be.unload()
        with pytest.raises(Exception):
            LLMBackend().load(str(tmp_path / "missing.gguf"))
    finally:
        loader.build_llm_engine = orig


@pytest.mark.parametrize("num_blocks,mode", [(400, "recompute"), (14, "recompute"), (10, "recompute"),
                                             (14, "swap"), (10, "swap")])
def test_overlapped_steps_match_serial_steps(num_blocks, mode):
    """Launching step k+1 before step k's tokens are applied (the GPU engines'
    default) changes no output: seeded sampling, stop ids hit at random
    points (a finished sequence may already sit in the next launched step),
    length limits, a queue deeper than the batch, and a small pool that makes
    the scheduler skip or preempt."""
    cfg = tiny_cfg()
    rnd = np.random.default_rng(7)
    prompts = [rnd.integers(3, 300, int(n)).tolist() for n in rnd.integers(5, 60, 10)]
    stops = list(range(3, 300, 7))  # ~1 in 7 tokens ends a request
    params = [SamplingParams(max_new_tokens=int(m), seed=100 + i, stop_token_ids=stops if i % 2 else [],
                             ignore_eos=i % 2 == 0) for i, m in enumerate(rnd.integers(1, 25, 10))]

    def run(overlap):
        eng = LLMEngine(cfg, device="cpu", engine_cfg=EngineConfig(
            max_num_seqs=4, max_num_batched_tokens=32, max_model_len=256, num_blocks=num_blocks,
            overlap_steps=overlap, preemption=mode), seed=0)
        seqs = [eng.add_request(f"r{i}", p, params[i]) for i, p in enumerate(prompts)]
        outs = []
        while eng.has_unfinished():
            outs += eng.step()
        assert all(s.pending is None and -1 not in s.output_ids for s in seqs)
        streamed = {}
        for o in outs:
            streamed.setdefault(o.request_id, []).append(o.new_token)
        return [s.output_ids for s in seqs], streamed, [s.finish_reason for s in seqs]

    serial, stream_s, why_s = run(False)
    over, stream_o, why_o = run(True)
    assert over == serial
    assert why_o == why_s
    assert stream_o == stream_s  # every token reported once, in order
    assert any(r == "stop" for r in why_s) and any(r == "length" for r in why_s)
