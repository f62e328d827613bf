"""LLMEngine: continuous-batching generation loop over one GPU (one TP rank set).

Counterpart of the reference ``LLMEngine`` (crates/kapsl-llm/src/engine.rs:816-2499):
request ingestion with session continuation, seeds
``splitmix64((seed ?? fnv1a(request_id)) ^ seq_id * golden)`` (seq ids from 1),
KV admission control (``Overloaded`` above the soft limit, ``ResourceExhausted``
above the hard one, engine.rs:2144-2263), scheduling, execution, sampling and
stop handling (EOS, stop ids incl. BOS, max_new_tokens, max length).
"""
from __future__ import annotations

import itertools
import os
import time
from dataclasses import dataclass, field
from typing import Callable, Optional

import numpy as np
import torch

from ..engine_api import EngineError
from ..models.config import ModelConfig
from ..models.llama import CausalLM, ModelWeights, random_weights
from ..ops import reference as ref
from .block_manager import make_allocator
from .kv_cache import KVLayout, KVPool
from .model_runner import ModelRunner
from .scheduler import Scheduler
from .sequence import PENDING_TOKEN, SamplingParams, Sequence, SequenceStatus


@dataclass
class StepOutput:
    request_id: str
    seq: Sequence
    new_token: int
    finished: bool


@dataclass
class EngineConfig:
    max_num_seqs: int = 256
    max_num_batched_tokens: int = 2048
    max_model_len: int = 4096
    block_size: int = 16
    num_blocks: int = 0                 # 0 = size from memory
    kv_memory_fraction: float = 0.85    # of free memory after weights
    enable_prefix_cache: bool = True
    eviction: str = "lru"
    use_cuda_graph: bool = True
    chunked_prefill: bool = True
    max_session_tokens: int = 0         # 0 = max_model_len
    kv_soft_limit_bytes: int = 0        # 0 = 90% of hard
    kv_hard_limit_bytes: int = 0        # 0 = pool size
    shareable_kv: bool = False          # pool mappable by another process (disaggregated decode side)
    preemption: str = "recompute"       # or "swap": preempted KV pages go to host memory
    swap_space_bytes: int = 4 << 30     # host memory for swapped pages
    # launch step k+1 before reading step k's tokens: None = on for GPU engines (the CPU
    # backend computes inside launch, so overlapping would only delay its tokens), True / False force
    overlap_steps: Optional[bool] = None
    capture_graphs_at_start: bool = True  # capture every decode bucket when the engine is built


class LLMEngine:
    def __init__(self, cfg: ModelConfig, weights: Optional[ModelWeights] = None, device="cuda",
                 engine_cfg: Optional[EngineConfig] = None, tp_comm=None, moe=None, seed: int = 0, pp_stage=None,
                 model_cls=None):
        """``pp_stage``: a :class:`~kapsl_sdk_b200.parallel.pp.PipelineStage`; the engine then
        holds that stage's layers (and their KV pages) and steps in micro-batches.
        ``model_cls``: the GPU model class (default :class:`CausalLM`; the library
        baseline passes :class:`~kapsl_sdk_b200.models.baseline.BaselineCausalLM`)."""
        self.cfg = cfg
        self.ecfg = engine_cfg or EngineConfig()
        self.device = torch.device(device)
        self.pp = pp_stage
        e = self.ecfg
        nlayers = len(pp_stage.layers) if pp_stage is not None else cfg.num_layers
        if self.device.type == "cpu":
            from ..models.cpu_model import CPUCausalLM
            from .cpu_runner import CPUModelRunner

            if isinstance(weights, CPUCausalLM):
                self.model = weights
                self.model.stage = pp_stage
            else:
                self.model = CPUCausalLM.random(cfg, seed, layers=pp_stage.layers if pp_stage else None,
                                                stage=pp_stage)
            layout = KVLayout(nlayers, cfg.num_kv_heads, cfg.head_dim, e.block_size, torch.float32)
            nblocks = e.num_blocks or e.max_num_seqs * ((e.max_model_len + e.block_size - 1) // e.block_size)
            self.pool = KVPool(layout, nblocks, self.device)
            self.runner = CPUModelRunner(self.model, self.pool)
            self._finish_init(cfg, e, nblocks, tp_comm)
            return
        if cfg.cpu_only:
            raise ValueError(f"{cfg.arch} layers (q/k norms, GeGLU, soft-capping or sliding windows) run on the "
                             "CPU backend only")
        if weights is None:
            tp = 1 if tp_comm is None else tp_comm.world_size
            rank = 0 if tp_comm is None else tp_comm.rank
            weights = random_weights(cfg, self.device, tp=tp, rank=rank, seed=seed,
                                     layers=pp_stage.layers if pp_stage else None)
        if moe is None and cfg.is_moe:
            from ..models.moe import MoE

            moe = MoE(cfg, self.device, tp_comm)
        self.model = (model_cls or CausalLM)(cfg, weights, self.device, tp_comm=tp_comm, moe=moe, stage=pp_stage)
        self.model.configure_tp(e.max_num_batched_tokens + e.max_num_seqs, sample_rows=e.max_num_seqs + 1)
        if pp_stage is not None:
            e.use_cuda_graph = False  # stages exchange hidden states inside the step
        layout = KVLayout(nlayers, self.model.hkv, cfg.head_dim, e.block_size)
        nblocks = e.num_blocks
        if nblocks <= 0:
            free, _ = torch.cuda.mem_get_info(self.device)
            reserve = 6 << 30  # activations, graphs, workspaces
            nblocks = KVPool.blocks_for_bytes(layout, int(max(free - reserve, 1 << 30) * e.kv_memory_fraction))
            if tp_comm is not None and tp_comm.world_size > 1:
                nblocks = tp_comm.min_int(nblocks)
        self.pool = KVPool(layout, nblocks, self.device, shareable=e.shareable_kv)
        self.runner = ModelRunner(self.model, self.pool, e.max_num_seqs, e.max_num_batched_tokens, e.max_model_len,
                                  e.use_cuda_graph)
        self._finish_init(cfg, e, nblocks, tp_comm)
        if e.use_cuda_graph and e.capture_graphs_at_start:
            self.runner.capture_all()

    def _finish_init(self, cfg: ModelConfig, e: EngineConfig, nblocks: int, tp_comm) -> None:
        self.allocator = make_allocator(nblocks, e.block_size, e.enable_prefix_cache, e.eviction)
        self.scheduler = Scheduler(self.allocator, e.max_num_seqs, e.max_num_batched_tokens, e.chunked_prefill,
                                   e.max_model_len, e.preemption,
                                   e.swap_space_bytes // self.pool.layout.bytes_per_block())
        self._swapped_kv: dict = {}  # seq_id -> host copy of its computed pages
        self._inflight = None  # launched step whose tokens the host has not applied yet
        self.failed: Optional[EngineError] = None  # set when a step failed on the device
        self._seq_ids = itertools.count(1)
        self.sessions: dict[str, Sequence] = {}
        self.finished: list[Sequence] = []
        self.stop_ids = set(x for x in (cfg.eos_token_id, cfg.bos_token_id) if x is not None)
        self.bytes_per_token = cfg.kv_bytes_per_token() // (1 if tp_comm is None else 1)
        hard = e.kv_hard_limit_bytes or self.pool.nbytes
        self.kv_hard = hard
        self.kv_soft = e.kv_soft_limit_bytes or int(hard * 0.9)
        # Disaggregated prefill: called with the sequences that finish in a step,
        # before their KV blocks go back to the allocator (the KV connector copies
        # them out on the same stream, so later reuse of the blocks is ordered after it).
        self.kv_export: Optional[Callable] = None
        # KAPSL_NVTX=1: NVTX ranges per step and phase for Nsight timelines (GPU engines)
        self._nvtx = os.environ.get("KAPSL_NVTX", "0") == "1" and self.device.type == "cuda"
        self.profile = None
        if os.environ.get("KAPSL_LLM_PROFILE", os.environ.get("KAPSL_LLM_PROFILE_DECODE", "0")) == "1":
            self.profile = {"steps": 0, "decode_steps": 0, "tokens": 0, "schedule_s": 0.0, "prepare_s": 0.0,
                            "gpu_wait_s": 0.0, "postprocess_s": 0.0}
            if hasattr(self.runner, "prof"):
                self.runner.prof = self.profile  # the GPU runner adds launch / sync / device times

    # ------------------------------------------------------------ requests
    def _reserved_bytes(self) -> int:
        tot = 0
        for s in list(self.scheduler.running) + list(self.scheduler.waiting):
            tot += (len(s.prompt_ids) + s.params.max_new_tokens) * self.pool.layout.bytes_per_block() // \
                self.pool.layout.block_size
        return tot

    def add_request(self, request_id: str, prompt_ids: list, params: Optional[SamplingParams] = None,
                    session_id: Optional[str] = None, on_token: Optional[Callable] = None,
                    admission_control: bool = False) -> Sequence:
        params = params or SamplingParams()
        prompt_ids = [int(t) for t in prompt_ids]
        if not prompt_ids:
            raise EngineError.invalid_input("empty prompt")
        bad = [t for t in prompt_ids if t < 0 or t >= self.cfg.vocab_size]
        if bad:
            raise EngineError.invalid_input(f"token id {bad[0]} outside vocab of {self.cfg.vocab_size}")
        if admission_control:
            need = (len(prompt_ids) + params.max_new_tokens) * self.pool.layout.bytes_per_block() // \
                self.pool.layout.block_size
            cur = self._reserved_bytes()
            if need > self.kv_hard:
                raise EngineError.resource_exhausted(
                    f"request needs {need} KV bytes, hard limit {self.kv_hard}")
            if cur + need > self.kv_soft:
                raise EngineError.overloaded(f"KV reservation {cur + need} bytes above soft limit {self.kv_soft}")
        seq_id = next(self._seq_ids)
        if session_id is not None and session_id in self.sessions:
            # continue the session: new turn appended to the previous sequence's tokens
            prev = self.sessions[session_id]
            max_sess = self.ecfg.max_session_tokens or self.ecfg.max_model_len
            history = prev.prompt_ids + prev.output_ids
            if len(history) + len(prompt_ids) + params.max_new_tokens <= max_sess:
                prompt_ids = history + prompt_ids
        rng = ref.seed_state(params.seed, request_id, seq_id)
        if len(prompt_ids) + 1 > self.ecfg.max_model_len:
            raise EngineError.invalid_input(
                f"prompt of {len(prompt_ids)} tokens exceeds max_model_len {self.ecfg.max_model_len}")
        return self.adopt_request(request_id, prompt_ids, params, seq_id, rng, session_id, on_token)

    def adopt_request(self, request_id: str, prompt_ids: list, params: SamplingParams, seq_id: int,
                      rng_state: int, session_id: Optional[str] = None, on_token: Optional[Callable] = None
                      ) -> Sequence:
        """Queue a request whose checks, session history and sampler seed another
        engine already resolved (the leader of a tensor-parallel serving group
        publishes exactly these fields, so every rank queues identical sequences)."""
        seq = Sequence(seq_id=seq_id, request_id=request_id, prompt_ids=list(prompt_ids), params=params,
                       rng_state=rng_state, session_id=session_id, on_token=on_token)
        self.scheduler.add(seq)
        if session_id is not None:
            self.sessions[session_id] = seq
        return seq

    def add_prefilled(self, request_id: str, prompt_ids: list, first_token: int, block_ids: list,
                      params: Optional[SamplingParams] = None, rng_state: Optional[int] = None) -> Sequence:
        """Adopt a sequence whose prompt KV another engine computed and wrote into
        ``block_ids`` of this engine's pool (disaggregated decode).  ``rng_state``
        is the sampler state after the first token was drawn."""
        params = params or SamplingParams()
        seq_id = next(self._seq_ids)
        if rng_state is None:
            rng_state = ref.seed_state(params.seed, request_id, seq_id)
        seq = Sequence(seq_id=seq_id, request_id=request_id, prompt_ids=[int(t) for t in prompt_ids],
                       params=params, rng_state=rng_state)
        seq.output_ids.append(int(first_token))
        seq.block_ids = list(block_ids)
        seq.num_computed = len(seq.prompt_ids)
        seq.first_token_time = time.perf_counter()
        seq.token_times.append(seq.first_token_time)
        if self._stop(seq, int(first_token)) is not None:
            seq.finish_time = seq.first_token_time
            seq.finish_reason = "length"
            self.scheduler.finish(seq, SequenceStatus.FINISHED_LENGTH)
            self.finished.append(seq)
            return seq
        self.scheduler.add(seq)
        return seq

    def abort(self, request_id: str) -> None:
        self._drain()
        for s in self.scheduler.abort(request_id):
            s.finish_time = time.perf_counter()
            s.finish_reason = "aborted"
            self._swapped_kv.pop(s.seq_id, None)

    def rollback(self, request_id: str, length: int) -> int:
        """Truncate the live request ``request_id`` to its first ``length`` tokens
        (prompt + output); generation then continues from there.  Returns the
        number of sequences changed."""
        self._drain()
        table = getattr(self.runner, "rng_table", None)
        hit = [s for s in list(self.scheduler.running) + list(self.scheduler.waiting) + list(self.scheduler.swapped)
               if s.request_id == request_id]
        readmit = []
        for s in hit:
            self._swapped_kv.pop(s.seq_id, None)
            running = s in self.scheduler.running
            if running and table is not None:  # keep the sampler stream (state lives in the slot)
                s.rng_state = int(table[s.slot].item()) & ((1 << 64) - 1)
            self.scheduler.rollback(s, length)
            if running and s in self.scheduler.running:
                readmit.append(s)
        if readmit:
            self.runner.reset_slots(readmit)  # penalty counts from the kept tokens, sampler state
        return len(hit)

    def rollback_session(self, session_id: str, length: int) -> None:
        """Drop the history of ``session_id`` past its first ``length`` tokens; the
        next turn continues from the shortened history (its cached prefix pages
        are reused up to there)."""
        s = self.sessions.get(session_id)
        if s is None:
            raise KeyError(session_id)
        if s.status.finished:
            ids = s.all_ids[:length]
            s.prompt_ids, s.output_ids = ids, []
        else:
            self.rollback(s.request_id, length)

    def has_unfinished(self) -> bool:
        return self.scheduler.has_work() or self._inflight is not None

    # ---------------------------------------------------------------- step
    def _stop(self, s: Sequence, tok: int) -> Optional[str]:
        p = s.params
        if not p.ignore_eos and (tok in self.stop_ids or tok in p.stop_token_ids):
            return "stop"
        if len(s.output_ids) >= p.max_new_tokens:
            return "length"
        if s.length >= self.ecfg.max_model_len:
            return "length"
        return None

    # ------------------------------------------------------------------
    # Overlapped stepping (GPU runner): step() schedules and launches the next
    # step BEFORE it waits for the one in flight, so the host's scheduling,
    # input staging and kernel launches run while the GPU executes.  Sampled
    # tokens a launched step has not returned yet are PENDING_TOKEN in
    # ``output_ids``; the next step's decode rows take them from the device.
    # While a step is in flight the scheduler does not preempt (a victim could
    # hold such a token); a step that needs preemption waits for the in-flight
    # one first.  Pipeline stages and the disaggregated prefill side
    # (``kv_export``) keep the step-at-a-time path.
    def _overlap_ok(self) -> bool:
        on = self.ecfg.overlap_steps
        if on is None:
            on = self.device.type == "cuda"
        return bool(on) and self.pp is None and self.kv_export is None

    def health_check(self) -> bool:
        """False once a step failed on the device (see :class:`DeviceError`)."""
        return self.failed is None

    def step(self) -> list[StepOutput]:
        if self.failed is not None:
            raise self.failed
        if self.pp is not None or self.kv_export is not None:
            outs = self._drain()
            return outs + self._step_serial()
        prof = self.profile is not None
        t0 = time.perf_counter() if prof else 0.0
        overlap = self._overlap_ok()
        if self._inflight is None or not overlap or self.scheduler.blocked:
            outs = self._drain()
            batch = self._schedule(True)
            if batch.empty:
                return outs
            t1 = time.perf_counter() if prof else 0.0
            inf = self._launch(batch)
            if prof:
                self._prof_step(batch, t1 - t0)
            if overlap:
                self._inflight = inf
                return outs
            return outs + self._complete(inf)
        batch = self._schedule(False)
        t1 = time.perf_counter() if prof else 0.0
        new = self._launch(batch) if not batch.empty else None
        if prof and new is not None:
            self._prof_step(batch, t1 - t0)
        old, self._inflight = self._inflight, new
        return self._complete(old)

    def _drain(self) -> list[StepOutput]:
        """Wait for the step in flight (if any) and apply its tokens."""
        if self._inflight is None:
            return []
        inf, self._inflight = self._inflight, None
        return self._complete(inf)

    def _schedule(self, allow_preempt: bool):
        nv = self._nvtx
        if nv:
            torch.cuda.nvtx.range_push("schedule")
        batch = self.scheduler.schedule(allow_preempt=allow_preempt)
        if batch.preempted or batch.swap_in or batch.swap_out:
            self._apply_preemptions(batch)
        if nv:
            torch.cuda.nvtx.range_pop()
        return batch

    def _prof_step(self, batch, schedule_s: float) -> None:
        p = self.profile
        p["steps"] += 1
        p["schedule_s"] += schedule_s
        p["prepare_s"] += self.runner.last_prepare_s
        p["tokens"] += batch.num_tokens
        if not batch.prefill:
            p["decode_steps"] += 1

    def _launch(self, batch):
        """Launch ``batch`` and advance the host state as of its completion: computed
        token counts, and a PENDING_TOKEN per sampling sequence."""
        nv = self._nvtx
        if nv:
            torch.cuda.nvtx.range_push(f"launch T={batch.num_tokens} decode={len(batch.decode)}")
        if batch.admitted:
            self.runner.admit(batch.admitted)
        inf = self.runner.launch(batch)
        if nv:
            torch.cuda.nvtx.range_pop()
        for s in batch.decode:
            s.num_computed += 1
        for s, n in batch.prefill:
            s.num_computed += n
        max_len = self.ecfg.max_model_len
        for r, s in enumerate(inf.seqs):
            s.output_ids.append(PENDING_TOKEN)
            s.pending = (inf.step_id, r)
            inf.out_idx.append(len(s.output_ids) - 1)
            if len(s.output_ids) >= s.params.max_new_tokens or s.length >= max_len:
                s.pending_finish = True  # this token is its last whatever its value
        return inf

    def _complete(self, inf) -> list[StepOutput]:
        """Wait for launched step ``inf``, put its tokens in place and retire the
        sequences that stopped.  A sequence that stopped here while a later step
        is already in flight drops that step's placeholder (its token is ignored
        when that step completes: the sequence is finished by then)."""
        prof = self.profile is not None
        try:
            seqs, toks = self.runner.collect(inf)
        except EngineError as e:
            # a kernel's bounded wait ran out (lost peer, stalled copy): the step's
            # tokens are invalid and the engine stops serving; health_check turns
            # false so a replica pool routes around it
            self.failed = e
            self._inflight = None
            raise
        now = time.perf_counter()
        outs = []
        for s, idx, tok in zip(seqs, inf.out_idx, toks.tolist()):
            if s.status.finished:
                continue
            s.output_ids[idx] = tok
            if s.pending is not None and s.pending[0] == inf.step_id:
                s.pending = None
            if s.first_token_time is None:
                s.first_token_time = now
            s.token_times.append(now)
            reason = self._stop_at(s, tok, idx + 1)
            if reason is not None:
                del s.output_ids[idx + 1:]
                s.num_computed = min(s.num_computed, s.length)
                s.pending = None
                s.pending_finish = False
                s.finish_time = now
                s.finish_reason = reason
                self.scheduler.finish(s, SequenceStatus.FINISHED_STOPPED if reason == "stop"
                                      else SequenceStatus.FINISHED_LENGTH, keep_blocks=False)
                self.finished.append(s)
            if s.on_token is not None:
                s.on_token(s, tok, reason is not None)
            outs.append(StepOutput(s.request_id, s, tok, reason is not None))
        if prof:
            self.profile["postprocess_s"] += time.perf_counter() - now
        return outs

    def _stop_at(self, s: Sequence, tok: int, n_out: int) -> Optional[str]:
        """Stop reason after output token ``n_out`` (1-based) of ``s`` is ``tok``."""
        p = s.params
        if not p.ignore_eos and (tok in self.stop_ids or tok in p.stop_token_ids):
            return "stop"
        if n_out >= p.max_new_tokens:
            return "length"
        if len(s.prompt_ids) + n_out >= self.ecfg.max_model_len:
            return "length"
        return None

    def _step_serial(self) -> list[StepOutput]:
        """One step at a time: pipeline stages, the disaggregated prefill side and
        the CPU runner."""
        prof = self.profile is not None
        t0 = time.perf_counter() if prof else 0.0
        nv = self._nvtx
        if nv:
            torch.cuda.nvtx.range_push("kapsl.step")
            torch.cuda.nvtx.range_push("schedule")
        batch = self.scheduler.schedule()
        if batch.preempted or batch.swap_in:
            self._apply_preemptions(batch)
        if nv:
            torch.cuda.nvtx.range_pop()
        if batch.empty:
            if nv:
                torch.cuda.nvtx.range_pop()
            return []
        t1 = time.perf_counter() if prof else 0.0
        if nv:
            torch.cuda.nvtx.range_push(f"execute T={batch.num_tokens} decode={len(batch.decode)}")
        if self.pp is not None:
            seqs, toks = self._pipeline_execute(batch)
        else:
            if batch.admitted:
                self.runner.admit(batch.admitted)
            seqs, toks = self.runner.execute(batch)
        if nv:
            torch.cuda.nvtx.range_pop()
            torch.cuda.nvtx.range_pop()
        now = time.perf_counter()
        if prof:
            p = self.profile
            p["steps"] += 1
            p["schedule_s"] += t1 - t0
            p["prepare_s"] += self.runner.last_prepare_s
            p["gpu_wait_s"] += now - t1 - self.runner.last_prepare_s
            p["tokens"] += batch.num_tokens
            if not batch.prefill:
                p["decode_steps"] += 1
        for s in batch.decode:
            s.num_computed += 1
        for s, n in batch.prefill:
            s.num_computed += n
        outs = []
        reasons = []
        for s, tok in zip(seqs, toks.tolist()):
            s.output_ids.append(tok)
            if s.first_token_time is None:
                s.first_token_time = now
            s.token_times.append(now)
            reasons.append(self._stop(s, tok))
        if self.kv_export is not None:
            done = [s for s, r in zip(seqs, reasons) if r is not None]
            if done:
                self.kv_export(done)
        for s, reason in zip(seqs, reasons):
            tok = s.output_ids[-1]
            if reason is not None:
                s.finish_time = now
                s.finish_reason = reason
                self.scheduler.finish(s, SequenceStatus.FINISHED_STOPPED if reason == "stop"
                                      else SequenceStatus.FINISHED_LENGTH, keep_blocks=False)
                self.finished.append(s)
            if s.on_token is not None:
                s.on_token(s, tok, reason is not None)
            outs.append(StepOutput(s.request_id, s, tok, reason is not None))
        if prof:
            self.profile["postprocess_s"] += time.perf_counter() - now
        return outs

    def _apply_preemptions(self, batch) -> None:
        """Keep the sampler stream of preempted sequences (the GPU runner holds the
        LCG state per slot on the device) and move swapped pages: restores first,
        then copies out, all queued before this step's kernels."""
        table = getattr(self.runner, "rng_table", None)
        if batch.preempted and table is not None:
            idx = torch.as_tensor(batch.preempted_slots, dtype=torch.long, device=table.device)
            for s, v in zip(batch.preempted, table.index_select(0, idx).tolist()):
                s.rng_state = v & ((1 << 64) - 1)
        for s, blocks in batch.swap_in:
            self.pool.restore(self._swapped_kv.pop(s.seq_id), blocks)
        for s, blocks in batch.swap_out:
            self._swapped_kv[s.seq_id] = self.pool.offload(blocks)

    def _pipeline_execute(self, batch):
        """One step as micro-batches through this pipeline stage; tokens come from the last stage."""
        from ..parallel.pp import split_batch

        seqs, parts = [], []
        for sb in split_batch(batch, self.pp.micro_batches):
            if sb.admitted:
                self.runner.admit(sb.admitted)
            s, t = self.runner.execute(sb)
            seqs += s
            parts.append(np.asarray(t, dtype=np.int64))
        toks = torch.from_numpy(np.concatenate(parts) if parts else np.zeros(0, np.int64))
        if self.device.type == "cuda":
            toks = toks.to(self.device)
        toks = self.pp.broadcast_tokens(toks)
        return seqs, toks.cpu().numpy()

    def profile_summary(self) -> dict:
        """Per-phase host timings when ``KAPSL_LLM_PROFILE=1`` (reference:
        KAPSL_LLM_PROFILE_DECODE, crates/kapsl-llm/src/engine.rs:102-115)."""
        return dict(self.profile or {})

    def generate(self, prompts: list, params: Optional[SamplingParams] = None) -> list[list[int]]:
        """Run ``prompts`` (lists of token ids) to completion; returns output ids in order."""
        seqs = [self.add_request(f"gen-{next(self._seq_ids)}-{i}", p, params) for i, p in enumerate(prompts)]
        while self.has_unfinished():
            self.step()
        return [s.output_ids for s in seqs]

    # ------------------------------------------------------------- metrics
    def kv_stats(self) -> dict:
        a = self.allocator
        bpb = self.pool.layout.bytes_per_block()
        return {
            "blocks_total": a.num_blocks, "blocks_free": a.num_free(),
            "bytes_capacity": a.num_blocks * bpb, "bytes_used": a.num_used() * bpb,
            "sequences": len(self.scheduler.running), "evicted_blocks_total": a.evicted_blocks,
            "preemptions": self.scheduler.num_preemptions, "swapped": len(self.scheduler.swapped),
            "swap_out_total": self.scheduler.num_swap_out, "swap_in_total": self.scheduler.num_swap_in,
        }

    def shutdown(self) -> None:
        self._drain()
        self.runner.release_graphs()
        if hasattr(self.pool, "close"):
            self.pool.close()
