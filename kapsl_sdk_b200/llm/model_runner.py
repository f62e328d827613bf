"""Builds device inputs for a scheduled batch, runs the model, samples.

Host work per step is a handful of numpy writes into a pinned int32 staging
buffer and a pinned int64 buffer, copied to the device with two async copies;
every kernel input is a fixed view of the device copies.  Decode-only steps
replay a CUDA graph captured per batch-size bucket (model forward + sampler +
penalty-count update), so a decode step costs one graph launch.

A step is split into :meth:`ModelRunner.launch` (fill, copy, launch, start
the token read-back; returns at once) and :meth:`ModelRunner.collect` (wait
for that step's tokens).  The engine launches step k+1 before it collects
step k, so host scheduling overlaps the GPU: the staging and read-back
buffers are double-buffered, and a decode row whose input token step k has
sampled but the host has not read yet names that token's sampler row
(``src`` region); the embedding kernel reads it from the device.

Reference counterpart: the per-step input preparation, KV gather/pack and
sampling of crates/kapsl-llm/src/engine.rs:3170-3914 (batched decode) and
2613-3168 (batched prefill), which run on the host around an ORT session.
"""
from __future__ import annotations

import bisect
import time
from typing import Optional

import numpy as np
import torch

from .. import ops
from .._ext import launch_count
from ..engine_api import EngineError, ErrorKind
from ..models.llama import CausalLM, ForwardBatch
from ..ops import reference as ref
from .kv_cache import KVPool
from .scheduler import ScheduledBatch
from .sequence import Sequence


class _Layout:
    """Offsets of every input region inside the staging buffers."""

    def __init__(self, max_tokens: int, max_seqs: int, max_blocks: int, max_work: int):
        self.T, self.S, self.MB, self.W = max_tokens, max_seqs, max_blocks, max_work
        o = 0
        self.ids = o; o += max_tokens
        self.pos = o; o += max_tokens
        self.ctx = o; o += max_seqs
        self.bt = o; o += max_seqs * max_blocks
        self.work = o; o += max_work * 2
        self.sinfo = o; o += max_seqs * 4
        self.topk = o; o += max_seqs
        self.sslot = o; o += max_seqs
        self.temp = o; o += max_seqs
        self.topp = o; o += max_seqs
        self.pen = o; o += max_seqs
        self.adm_slot = o; o += max_seqs
        self.src = o; o += max_seqs  # decode rows: previous step's sampler row of the input token, or -1
        self.n32 = o
        o = 0
        self.slots = o; o += max_tokens
        self.lidx = o; o += max_seqs
        self.adm_rng = o; o += max_seqs
        self.n64 = o


class Inflight:
    """A launched step: its sampling sequences (row order of ``out_tokens``), the
    pinned buffer its tokens are read back into, and the event after that copy."""
    __slots__ = ("step_id", "seqs", "R", "h_out", "done", "start", "kind", "num_tokens", "out_idx", "launch_s",
                 "h_err")

    def __init__(self, step_id, seqs, R, h_out, done, start, kind, num_tokens):
        self.step_id, self.seqs, self.R, self.h_out = step_id, seqs, R, h_out
        self.done, self.start, self.kind, self.num_tokens = done, start, kind, num_tokens
        self.out_idx: list = []
        self.launch_s = 0.0
        self.h_err = None


class DeviceError(EngineError):
    """A kernel of the step recorded a status code: a bounded wait on a peer or a
    pipeline stage ran out (a lost tensor-parallel rank, a stalled copy).  The
    step's results are not valid and the engine stops serving."""

    def __init__(self, code: int):
        super().__init__(ErrorKind.BACKEND, ops.describe_error(code))
        self.code = code


class ModelRunner:
    pf_tile = 64  # query tokens per prefill-attention work item (the model's kernel decides)

    def __init__(self, model: CausalLM, pool: KVPool, max_num_seqs: int = 256, max_num_batched_tokens: int = 2048,
                 max_model_len: int = 4096, use_cuda_graph: bool = True, graph_sizes: Optional[list] = None):
        self.model = model
        self.pf_tile = getattr(model, "prefill_tile", 64)
        self.pool = pool
        self.device = model.device
        self.bs = pool.layout.block_size
        self.max_seqs = max_num_seqs
        self.max_tokens = max_num_batched_tokens + max_num_seqs
        self.max_blocks = (max_model_len + self.bs - 1) // self.bs
        self.vocab = model.cfg.vocab_size
        S = max_num_seqs + 1  # one spare slot for graph padding rows
        self.pad_slot = max_num_seqs
        W = (max_num_batched_tokens + self.pf_tile - 1) // self.pf_tile + max_num_seqs
        self.L = _Layout(self.max_tokens, S, self.max_blocks, W)
        # two pinned staging sets, used by alternate steps: while step k's copies may still
        # be queued, step k+1 is filled into the other set
        self._h32s = [torch.zeros(self.L.n32, dtype=torch.int32, pin_memory=True) for _ in range(2)]
        self._h64s = [torch.zeros(self.L.n64, dtype=torch.int64, pin_memory=True) for _ in range(2)]
        self._houts = [torch.zeros(S, dtype=torch.int32, pin_memory=True) for _ in range(2)]
        # the kernels' status words, read back with every step's tokens (no extra sync)
        self._herrs = [torch.zeros(16, dtype=torch.int32, pin_memory=True) for _ in range(2)]
        self._buf = 1
        self._select(0)
        self.d32 = torch.zeros(self.L.n32, dtype=torch.int32, device=self.device)
        self.d64 = torch.zeros(self.L.n64, dtype=torch.int64, device=self.device)
        # per-sequence device tables
        self.rng_table = torch.zeros(S, dtype=torch.int64, device=self.device)
        self.counts = torch.zeros(S, self.vocab, dtype=torch.int32, device=self.device)
        # per slot: the ids that occurred (first-seen order), so the sampler's
        # repetition penalty touches only those logits
        self.occ = torch.zeros(S, max(self.max_blocks * self.bs, 1), dtype=torch.int32, device=self.device)
        self.occ_n = torch.zeros(S, dtype=torch.int32, device=self.device)
        self.full_scratch: Optional[torch.Tensor] = None  # whole-vocabulary sampling rows
        self.out_tokens = torch.zeros(S, dtype=torch.int32, device=self.device)
        self._admit_seqs: list = []
        self._step_id = 0
        self.use_graph = use_cuda_graph
        self.graph_sizes = sorted(graph_sizes or self._default_graph_sizes(max_num_seqs))
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.graph_launches: dict[int, int] = {}
        self.graph_pool = None
        self.launches = 0  # kernels launched by steps (eager count + graph replays x graph size)
        self.last_prepare_s = 0.0
        # per-step host/device breakdown (a dict shared with the engine's profile, or None):
        # launch_s host time issuing kernels, sync_s host wait for the step, device_s the
        # step's span on the stream (CUDA events), split by graph / eager steps
        self.prof: Optional[dict] = None
        self.stats = {"steps": 0, "graph_steps": 0, "h2d_bytes": 0, "d2h_bytes": 0}

    def _select(self, buf: int) -> None:
        """Make staging set ``buf`` the one _fill writes and _h2d copies."""
        self._buf = buf
        self.h32, self.h64, self.h_out = self._h32s[buf], self._h64s[buf], self._houts[buf]
        self.h_err = self._herrs[buf]
        self.n32 = self.h32.numpy()
        self.n64 = self.h64.numpy()
        self.f32view = self.n32.view(np.float32)

    @staticmethod
    def _default_graph_sizes(max_seqs: int) -> list[int]:
        sizes = [1, 2, 4, 8, 16, 24, 32]
        s = 48
        while s < max_seqs:
            sizes.append(s)
            s += 16 if s < 128 else 32
        sizes.append(max_seqs)
        return sorted(set(x for x in sizes if x <= max_seqs))

    # ------------------------------------------------------------ views
    def _v32(self, off: int, n: int) -> torch.Tensor:
        return self.d32[off:off + n]

    def _f32(self, off: int, n: int) -> torch.Tensor:
        return self.d32[off:off + n].view(torch.float32)

    def _bt(self, nrows: int) -> torch.Tensor:
        return self.d32[self.L.bt:self.L.bt + nrows * self.max_blocks].view(nrows, self.max_blocks)

    def _forward_batch(self, T: int, S: int, R: int, Bd: int, max_ctx: int, nwork: int, nsplit: int,
                       nsrc: int = 0) -> ForwardBatch:
        L = self.L
        return ForwardBatch(
            src_rows=self._v32(L.src, nsrc) if nsrc else None, prev_tokens=self.out_tokens if nsrc else None,
            input_ids=self._v32(L.ids, T), positions=self._v32(L.pos, T), slots=self.d64[L.slots:L.slots + T],
            block_tables=self._bt(max(S, 1)), ctx_lens=self._v32(L.ctx, max(S, 1)),
            logits_idx=self.d64[L.lidx:L.lidx + R], num_tokens=T, num_decode=Bd, max_decode_ctx=max_ctx,
            pf_work=self._v32(L.work, nwork * 2).view(nwork, 2) if nwork else None,
            pf_seq_info=self._v32(L.sinfo, (S - Bd) * 4).view(S - Bd, 4) if S > Bd else None,
            decode_splits=nsplit)

    FULL_CTAS = 32  # rows sampled over the whole vocabulary at once

    @staticmethod
    def _needs_full(seqs) -> bool:
        """A row samples over the whole vocabulary (T > 0 with top_k 0 or > 1024)."""
        return any(s.params.temperature > 0 and not 0 < s.params.top_k <= ops.SAMPLE_MAX_TOP_K for s in seqs)

    def _sample(self, logits: torch.Tensor, R: int, full: bool = False) -> None:
        L = self.L
        args = (self._f32(L.temp, R), self._v32(L.topk, R), self._f32(L.topp, R))
        if getattr(self.model, "library_sampler", False):  # the library baseline samples with torch ops
            slots = self._v32(L.sslot, R)
            self.model.sample(logits, *args, self.out_tokens, self._f32(L.pen, R), self.counts, slots)
            self._count(slots, self.out_tokens[:R])
            return
        tp = self.model.tp
        if self.model.tp_size > 1 and not full:  # logits hold this rank's vocabulary slice
            tp.vocab_sample(logits, self.model.vocab_start, self.vocab, *args, self.rng_table, self.out_tokens[:R],
                            rep_penalty=self._f32(L.pen, R), counts=self.counts, slots=self._v32(L.sslot, R),
                            occ=self.occ, occ_n=self.occ_n)
        else:
            if full and self.full_scratch is None:
                self.full_scratch = ops.sample_full_scratch(self.vocab, self.device, self.FULL_CTAS)
            ops.sample(logits, *args, self.rng_table, self.out_tokens[:R], rep_penalty=self._f32(L.pen, R),
                       counts=self.counts, slots=self._v32(L.sslot, R), occ=self.occ, occ_n=self.occ_n,
                       full_scratch=self.full_scratch if full else None, full_ctas=self.FULL_CTAS if full else 0)
        self._count(self._v32(L.sslot, R), self.out_tokens[:R])

    def _count(self, rows: torch.Tensor, ids: torch.Tensor) -> None:
        """counts[rows[i], ids[i]] += 1 (and first occurrences appended to the slot lists)."""
        if getattr(self.model, "library_sampler", False):
            self.counts.index_put_((rows.long(), ids.long()), torch.ones_like(ids), accumulate=True)
        else:
            ops.count_tokens(self.counts, rows, ids, self.occ, self.occ_n)

    # ------------------------------------------------------- host inputs
    def _fill(self, batch: ScheduledBatch, pad_to: int = 0):
        """Write the batch into the pinned staging buffers; returns shape info.
        Decode rows and sampling rows are written as whole arrays (one numpy
        assignment per field), not element by element."""
        L, n32, n64, f32 = self.L, self.n32, self.n64, self.f32view
        MB, bs = self.max_blocks, self.bs
        dec = batch.decode
        Bd = len(dec)
        # decode rows
        if Bd:
            lens = np.array([s.length for s in dec], dtype=np.int64)
            pos = lens - 1
            bts = [s.block_table() for s in dec]
            nbs = np.array([len(b) for b in bts], dtype=np.int64)
            flat = np.concatenate(bts)
            starts = np.cumsum(nbs) - nbs
            # an input token that the previous step sampled and the host has not read yet
            # (``pending``) is taken on the device from that step's sampler row
            pend = [s.pending[1] if s.pending is not None else -1 for s in dec]
            n32[L.src:L.src + Bd] = pend
            n32[L.ids:L.ids + Bd] = [0 if p >= 0 else (s.output_ids[-1] if s.output_ids else s.prompt_ids[-1])
                                     for s, p in zip(dec, pend)]
            n32[L.pos:L.pos + Bd] = pos
            n64[L.slots:L.slots + Bd] = flat[starts + pos // bs].astype(np.int64) * bs + pos % bs
            n32[L.ctx:L.ctx + Bd] = lens
            # block-table rows: element g of `flat` (row i) goes to L.bt + i * MB + (g - starts[i])
            n32[L.bt + np.arange(flat.size) + np.repeat(np.arange(Bd, dtype=np.int64) * MB - starts, nbs)] = flat
        Bpad = max(Bd, pad_to)
        if Bpad > Bd:  # CUDA-graph padding rows: no KV write, 1-token context on block 0
            n32[L.ids + Bd:L.ids + Bpad] = 0
            n32[L.src + Bd:L.src + Bpad] = -1
            n32[L.pos + Bd:L.pos + Bpad] = 0
            n64[L.slots + Bd:L.slots + Bpad] = -1
            n32[L.ctx + Bd:L.ctx + Bpad] = 1
            n32[L.bt + np.arange(Bd, Bpad, dtype=np.int64) * MB] = 0
        t = Bpad
        # prefill chunks
        nwork = 0
        sample_seqs = list(dec)
        lrows = list(range(Bd))
        for j, (s, n) in enumerate(batch.prefill):
            row = Bpad + j
            p0 = s.num_computed
            npr = len(s.prompt_ids)
            toks = s.prompt_ids[p0:p0 + n] if p0 + n <= npr else (s.prompt_ids + s.output_ids)[p0:p0 + n]
            n32[L.ids + t:L.ids + t + n] = toks
            ppos = np.arange(p0, p0 + n, dtype=np.int64)
            n32[L.pos + t:L.pos + t + n] = ppos
            blk = s.block_table()
            n64[L.slots + t:L.slots + t + n] = blk[ppos // bs].astype(np.int64) * bs + ppos % bs
            n32[L.ctx + row] = p0 + n
            n32[L.bt + row * MB:L.bt + row * MB + len(blk)] = blk
            si = L.sinfo + j * 4
            n32[si:si + 4] = (t, n, p0 + n, row)
            tile = self.pf_tile
            k = (n + tile - 1) // tile  # work items of this chunk
            n32[L.work + 2 * nwork:L.work + 2 * (nwork + k):2] = j
            n32[L.work + 2 * nwork + 1:L.work + 2 * (nwork + k):2] = np.arange(0, n, tile, dtype=np.int32)
            nwork += k
            if p0 + n >= s.length:  # chunk completes the prompt: sample from its last token
                sample_seqs.append(s)
                lrows.append(t + n - 1)
            t += n
        R = len(sample_seqs)
        Rpad = max(R, pad_to) if pad_to else R
        if R:
            n64[L.lidx:L.lidx + R] = lrows
            n32[L.sslot:L.sslot + R] = [s.slot for s in sample_seqs]
            f32[L.temp:L.temp + R] = [s.params.temperature for s in sample_seqs]
            n32[L.topk:L.topk + R] = [s.params.top_k for s in sample_seqs]
            f32[L.topp:L.topp + R] = [s.params.top_p for s in sample_seqs]
            f32[L.pen:L.pen + R] = [s.params.repetition_penalty for s in sample_seqs]
        if Rpad > R:
            n64[L.lidx + R:L.lidx + Rpad] = np.arange(R, Rpad, dtype=np.int64)
            n32[L.sslot + R:L.sslot + Rpad] = self.pad_slot
            f32[L.temp + R:L.temp + Rpad] = 0.0
            n32[L.topk + R:L.topk + Rpad] = 0
            f32[L.topp + R:L.topp + Rpad] = 1.0
            f32[L.pen + R:L.pen + Rpad] = 1.0
        S = Bpad + len(batch.prefill)
        return t, S, R, Rpad, Bd, Bpad, nwork, sample_seqs

    def _h2d(self) -> None:
        self.d32.copy_(self.h32, non_blocking=True)
        self.d64.copy_(self.h64, non_blocking=True)
        self.stats["h2d_bytes"] += self.h32.numel() * 4 + self.h64.numel() * 8

    def admit(self, seqs: list) -> None:
        """Initialise per-slot device state (LCG seed, penalty counts) for new
        sequences; applied on the stream by the next :meth:`launch`, before its kernels."""
        self._admit_seqs.extend(seqs)

    def _write_admissions(self) -> None:
        seqs, self._admit_seqs = self._admit_seqs, []
        if not seqs:
            return
        L = self.L
        for i, s in enumerate(seqs):
            self.n32[L.adm_slot + i] = s.slot
            st = s.rng_state
            self.n64[L.adm_rng + i] = st - (1 << 64) if st >= (1 << 63) else st
        # (the H2D copy of the staging set happens next; admission runs after it on the stream)
        self._pending_admit = len(seqs)
        self._admit_prompts = [(s.slot, s.prompt_ids + s.output_ids) for s in seqs]

    def reset_slots(self, seqs: list) -> None:
        """Re-initialise the per-slot state (LCG state, penalty counts) of running
        sequences now, on the current stream (between steps, e.g. after a rollback)."""
        if not seqs:
            return
        slots = torch.as_tensor([s.slot for s in seqs], dtype=torch.long).to(self.device)
        rng = torch.as_tensor([s.rng_state - (1 << 64) if s.rng_state >= (1 << 63) else s.rng_state for s in seqs],
                              dtype=torch.int64).to(self.device)
        self.rng_table.index_copy_(0, slots, rng)
        self.counts.index_fill_(0, slots, 0)
        self.occ_n.index_fill_(0, slots, 0)
        rows = np.concatenate([np.full(len(s.all_ids), s.slot, dtype=np.int32) for s in seqs])
        ids = np.concatenate([np.asarray(s.all_ids, dtype=np.int32) for s in seqs])
        self._count(torch.from_numpy(rows).to(self.device), torch.from_numpy(ids).to(self.device))

    def _apply_admissions(self) -> None:
        n = getattr(self, "_pending_admit", 0)
        if not n:
            return
        L = self.L
        slots_d = self._v32(L.adm_slot, n).long()
        self.rng_table.index_copy_(0, slots_d, self.d64[L.adm_rng:L.adm_rng + n])
        self.counts.index_fill_(0, slots_d, 0)
        self.occ_n.index_fill_(0, slots_d, 0)
        rows = np.concatenate([np.full(len(p), sl, dtype=np.int32) for sl, p in self._admit_prompts])
        ids = np.concatenate([np.asarray(p, dtype=np.int32) for _, p in self._admit_prompts])
        rows_t = torch.from_numpy(rows).pin_memory().to(self.device, non_blocking=True)
        ids_t = torch.from_numpy(ids).pin_memory().to(self.device, non_blocking=True)
        self.stats["h2d_bytes"] += rows.nbytes + ids.nbytes
        self._count(rows_t, ids_t)
        self._pending_admit = 0
        self._admit_prompts = []

    # ------------------------------------------------------------ execute
    def execute(self, batch: ScheduledBatch) -> tuple[list, np.ndarray]:
        """Run one step to completion; returns (sequences that sampled, their new tokens)."""
        return self.collect(self.launch(batch))

    def launch(self, batch: ScheduledBatch) -> "Inflight":
        """Fill and copy the step's inputs, launch its kernels and the read-back of
        its sampled tokens; returns without waiting for the GPU."""
        decode_only = not batch.prefill and len(batch.decode) > 0
        pad_to = 0
        gsize = 0
        bucket = 0
        if decode_only:
            k = bisect.bisect_left(self.graph_sizes, len(batch.decode))
            if k < len(self.graph_sizes):
                bucket = self.graph_sizes[k]
                if self.use_graph:
                    gsize = pad_to = bucket
        full = self._needs_full(batch.decode) or self._needs_full(
            s for s, n in batch.prefill if s.num_computed + n >= s.length)
        tp0 = time.perf_counter()
        c0 = launch_count()
        self._select(self._buf ^ 1)  # the set used two steps ago: its copies have completed
        T, S, R, Rpad, Bd, Bpad, nwork, sample_seqs = self._fill(batch, pad_to)
        self._write_admissions()
        self._h2d()
        self._apply_admissions()
        tl0 = time.perf_counter()
        self.last_prepare_s = tl0 - tp0
        prof = self.prof
        ev0 = None
        if prof is not None:
            ev0 = torch.cuda.Event(enable_timing=True)
            ev0.record()
        if gsize:
            key = (gsize, full)
            g = self.graphs.get(key)
            if g is None:
                g = self._capture(gsize, full)
            g.replay()
            self.launches += launch_count() - c0 + self.graph_launches[key]
            self.stats["graph_steps"] += 1
        else:
            max_ctx = int(self.n32[self.L.ctx:self.L.ctx + Bd].max()) if Bd else 0
            nsplit = 0
            if bucket:  # same split-KV policy as the captured graphs, so both paths agree bitwise
                nsplit = self._graph_splits(bucket)
            fb = self._forward_batch(T, S, R, Bd, max_ctx, nwork, nsplit, nsrc=Bpad)
            logits = self.model.forward(fb, self.pool.k, self.pool.v, full_vocab=full)
            if logits is not None:  # None: an earlier pipeline stage (the last stage samples)
                self._sample(logits, R, full)
            self.launches += launch_count() - c0
        self.h_out[:R].copy_(self.out_tokens[:R], non_blocking=True)
        self.h_err.copy_(ops.error_buffer(self.device), non_blocking=True)
        done = torch.cuda.Event(enable_timing=prof is not None)
        done.record()
        self._step_id += 1
        self.stats["d2h_bytes"] += R * 4
        self.stats["steps"] += 1
        inf = Inflight(self._step_id, sample_seqs, R, self.h_out, done, ev0, "graph" if gsize else "eager", T)
        inf.h_err = self.h_err
        if prof is not None:
            inf.launch_s = time.perf_counter() - tl0
            self._tally(f"{inf.kind}_launch_s", inf.launch_s)
        return inf

    def collect(self, inf: "Inflight") -> tuple[list, np.ndarray]:
        """Wait for step ``inf`` and return (its sampling sequences, their tokens)."""
        t0 = time.perf_counter()
        inf.done.synchronize()
        if self.prof is not None:
            dev_s = inf.start.elapsed_time(inf.done) / 1e3
            self._tally("sync_s", time.perf_counter() - t0)
            self._tally(f"{inf.kind}_steps", 1)
            self._tally(f"{inf.kind}_tokens", inf.num_tokens)
            self._tally(f"{inf.kind}_device_s", dev_s)
            trace = self.prof.get("trace")
            if trace is not None:  # per step: kind, tokens, sampling rows, host launch s, device s
                trace.append((inf.kind, inf.num_tokens, inf.R, round(inf.launch_s, 6), round(dev_s, 6)))
        if inf.h_err is not None:
            codes = inf.h_err.numpy()
            if codes.any():
                code = int(codes[codes != 0][0])
                ops.error_buffer(self.device).zero_()
                raise DeviceError(code)
        return inf.seqs, inf.h_out[:inf.R].numpy().copy()

    def _tally(self, key: str, v) -> None:
        self.prof[key] = self.prof.get(key, 0) + v

    def logits(self, batch: ScheduledBatch) -> torch.Tensor:
        """Eager forward of ``batch`` returning the fp32 logits of its sampling
        rows (decode rows, then prompt-completing chunks); nothing is sampled."""
        T, S, R, Rpad, Bd, Bpad, nwork, _ = self._fill(batch, 0)
        self._h2d()
        max_ctx = int(self.n32[self.L.ctx:self.L.ctx + Bd].max()) if Bd else 0
        fb = self._forward_batch(T, S, R, Bd, max_ctx, nwork, 0, nsrc=Bpad)
        out = self.model.forward(fb, self.pool.k, self.pool.v)
        torch.cuda.current_stream(self.device).synchronize()
        return out

    def capture_all(self) -> int:
        """Capture the decode graph of every batch bucket now (engine start-up), so
        no capture (a synchronize, a warm-up pass and a graph build, ~0.1 s each)
        lands in the middle of serving.  Inputs are padding rows (no KV write,
        a 1-token context on block 0).  Every rank of a tensor-parallel group
        runs this at the same point (the warm-up passes hold collectives)."""
        if not self.use_graph:
            return 0
        L, n32, n64, f32 = self.L, self.n32, self.n64, self.f32view
        MB = self.max_blocks
        n = 0
        for B in self.graph_sizes:
            if (B, False) in self.graphs:
                continue
            n32[L.ids:L.ids + B] = 0
            n32[L.src:L.src + B] = -1
            n32[L.pos:L.pos + B] = 0
            n64[L.slots:L.slots + B] = -1
            n32[L.ctx:L.ctx + B] = 1
            n32[L.bt + np.arange(B, dtype=np.int64) * MB] = 0
            n64[L.lidx:L.lidx + B] = np.arange(B, dtype=np.int64)
            n32[L.sslot:L.sslot + B] = self.pad_slot
            f32[L.temp:L.temp + B] = 0.0
            n32[L.topk:L.topk + B] = 0
            f32[L.topp:L.topp + B] = 1.0
            f32[L.pen:L.pen + B] = 1.0
            self._h2d()
            self._capture(B, False)
            n += 1
        torch.cuda.synchronize(self.device)
        return n

    def _graph_splits(self, B: int) -> int:
        return int(ops.cuda_ops().decode_num_splits(B, self.model.hkv, self.max_blocks * self.bs))

    def _capture(self, B: int, full: bool = False) -> torch.cuda.CUDAGraph:
        """Capture forward+sample for a decode batch of ``B`` rows (inputs are the
        staging views, already filled for this step); ``full``: the variant whose
        rows may sample over the whole vocabulary."""
        max_ctx = self.max_blocks * self.bs
        nsplit = self._graph_splits(B)
        fb = self._forward_batch(B, B, B, B, max_ctx, 0, nsplit, nsrc=B)
        if full and self.full_scratch is None:
            self.full_scratch = ops.sample_full_scratch(self.vocab, self.device, self.FULL_CTAS)
        # warm up once outside capture (allocator, function attributes)
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            logits = self.model.forward(fb, self.pool.k, self.pool.v, full_vocab=full)
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        # the warm-up wrote KV for real rows at their slots (same values as the replay will); fine.
        g = torch.cuda.CUDAGraph()
        c0 = launch_count()
        with torch.cuda.graph(g, pool=self.graph_pool):
            logits = self.model.forward(fb, self.pool.k, self.pool.v, full_vocab=full)
            self._sample(logits, B, full)
        key = (B, full)
        self.graph_launches[key] = launch_count() - c0
        if self.graph_pool is None:
            self.graph_pool = g.pool()
        self.graphs[key] = g
        return g

    def release_graphs(self) -> None:
        self.graphs.clear()
        self.graph_pool = None
