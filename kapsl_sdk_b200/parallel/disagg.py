"""Disaggregated prefill / decode with a KV connector.

The world is split in two tensor-parallel groups of equal size: ranks
``[0, P)`` run the prefill engine, ranks ``[P, 2P)`` the decode engine.
Prefill rank ``i`` is paired with decode rank ``P + i``: both hold the same
KV-head shard, so the KV pages computed by the one are exactly the pages the
other needs.

Life of a request (``DecodeWorker.submit``)::

    decode ranks   allocate the prompt's KV blocks (identical ids on every rank:
                   the ranks apply the same events in the same order)
    decode leader  posts  job/<k> = (request, prompt, block ids)    [control store]
    prefill ranks  run the prompt as a one-token request (chunked prefill, TP)
                   on finish: KVConnector.push copies the prompt's blocks of
                   every layer into the paired decode rank's pool, at the
                   job's block ids, on the compute stream; when that copy has
                   completed each rank posts done/<k>/<rank> (first token, RNG)
    decode ranks   once all prefill ranks have posted: adopt the sequence
                   (LLMEngine.add_prefilled) and decode it

Transfer modes (``KVConnector``):
  * ``"p2p"`` (default): the decode pool is allocated with cudaMalloc, exported
    with CUDA IPC and mapped by the paired prefill rank; one kernel
    (``kv_push``, csrc/cuda/kv_connector.cu) moves every layer's K and V page
    of the request over NVLink with peer stores straight into the decode pool.
  * ``"copy"``: baseline — gather the pages into a staging buffer, then one
    copy-engine ``cudaMemcpyAsync`` per layer plane and contiguous run.
  * ``"host"``: pages travel through the control store (CPU engines, tests).

Control messages go through the ``torch.distributed`` key-value store; each
group's leader reads them and broadcasts them to its group (gloo) at a step
boundary, so every rank of a group applies the same events at the same step.

Reference counterpart: none — the reference has no disaggregated serving or
KV transfer (its KV cache lives in host memory per engine,
crates/kapsl-llm/src/kv_cache.rs:640-1796).
"""
from __future__ import annotations

import os
import pickle
import time
from dataclasses import dataclass, field
from typing import Optional

import torch

from ..llm.sequence import SamplingParams

LCG_A = 6364136223846793005
MASK64 = (1 << 64) - 1


def _groups(world: int):
    """Creates (prefill ranks, decode ranks, gloo prefill group, gloo decode group,
    nccl prefill group, nccl decode group); every rank must call this."""
    import torch.distributed as dist

    if world % 2:
        raise ValueError("disaggregated serving needs an even number of ranks (prefill group + decode group)")
    P = world // 2
    pr, dr = list(range(P)), list(range(P, world))
    gp, gd = dist.new_group(pr, backend="gloo"), dist.new_group(dr, backend="gloo")
    nb = dist.get_backend()
    np_, nd = dist.new_group(pr, backend=nb), dist.new_group(dr, backend=nb)
    return pr, dr, gp, gd, np_, nd


class KVConnector:
    """Moves finished prompt KV blocks from a prefill rank's pool into its paired
    decode rank's pool."""

    def __init__(self, pool, role: str, pair_index: int, store, ns: str, mode: str = "p2p"):
        assert role in ("prefill", "decode") and mode in ("p2p", "copy", "host")
        self.pool, self.role, self.pair, self.store, self.ns, self.mode = pool, role, pair_index, store, ns, mode
        self.peer_base = 0
        self.peer_blocks = 0
        key = f"{ns}/pool/{pair_index}"
        if mode == "host":
            return
        if role == "decode":
            store.set(key, pickle.dumps((pool.ipc_handle(), pool.num_blocks)))
        else:
            from .._ext import cuda_ops

            handle, nblocks = pickle.loads(store.get(key))
            self.peer_base = cuda_ops().symm_open(handle)
            self.peer_blocks = nblocks

    def close(self) -> None:
        if self.peer_base:
            from .._ext import cuda_ops

            torch.cuda.synchronize(self.pool.device)
            cuda_ops().symm_close(self.peer_base)
            self.peer_base = 0

    # ------------------------------------------------------------- prefill side
    def push(self, src_blocks: list, dst_blocks: list, job: int) -> Optional[torch.cuda.Event]:
        """Copy ``src_blocks`` (all layers, K and V) into the peer's ``dst_blocks``.
        Returns an event that completes with the copy (None for host mode)."""
        pool = self.pool
        n = len(src_blocks)
        planes = pool.storage.shape[0] * pool.storage.shape[1]
        if self.mode == "host":
            pages = pool.storage[:, :, torch.as_tensor(src_blocks, dtype=torch.long)].contiguous().cpu()
            self.store.set(f"{self.ns}/pages/{job}/{self.pair}", pickle.dumps(pages.numpy()))
            return None
        from .._ext import cuda_ops

        c = cuda_ops()
        dev = pool.device
        if self.mode == "p2p":
            s = torch.tensor(src_blocks, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
            d = torch.tensor(dst_blocks, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
            c.kv_push(pool.storage, self.peer_base, s, d, planes, self.peer_blocks)
        else:
            staged = pool.storage.index_select(2, torch.as_tensor(src_blocks, dtype=torch.long, device=dev))
            blk = pool.layout.bytes_per_block() // planes
            runs = _runs(dst_blocks)
            for p in range(planes):
                src_plane = staged.data_ptr() + p * n * blk
                dst_plane = self.peer_base + p * self.peer_blocks * blk
                for i0, b0, cnt in runs:
                    c.copy_async(dst_plane + b0 * blk, src_plane + i0 * blk, cnt * blk)
            # `staged` may be freed now: the caching allocator hands its memory
            # only to work queued later on this stream, i.e. after the copies
        ev = torch.cuda.Event()
        ev.record()
        return ev

    # -------------------------------------------------------------- decode side
    def receive(self, job: int, dst_blocks: list) -> None:
        """Host mode: write the pages posted by the paired prefill rank."""
        if self.mode != "host":
            return
        import numpy as np

        pages = torch.from_numpy(np.asarray(pickle.loads(self.store.get(f"{self.ns}/pages/{job}/{self.pair}"))))
        idx = torch.as_tensor(dst_blocks, dtype=torch.long, device=self.pool.device)
        self.pool.storage.index_copy_(2, idx, pages.to(self.pool.device, self.pool.storage.dtype))
        self.store.delete_key(f"{self.ns}/pages/{job}/{self.pair}")


def _runs(ids: list) -> list:
    """[(index of first, first id, count)] of maximal runs of consecutive ids."""
    out = []
    i = 0
    while i < len(ids):
        j = i
        while j + 1 < len(ids) and ids[j + 1] == ids[j] + 1:
            j += 1
        out.append((i, ids[i], j - i + 1))
        i = j + 1
    return out


def _advance_rng(state: int, params: SamplingParams) -> int:
    """Sampler state after one draw (the LCG advances once per sampled token when T > 0)."""
    return (state * LCG_A + 1) & MASK64 if params.temperature > 0 else state


@dataclass
class _Job:
    k: int
    request_id: str
    prompt: list
    blocks: list
    params: SamplingParams
    seq: Optional[object] = None
    t_submit: float = field(default_factory=time.perf_counter)
    pushed: int = 0  # prefill side: leading blocks already pushed to the decode pool


class _Worker:
    def __init__(self, engine, connector: KVConnector, store, ns: str, group, leader: int, is_leader: bool):
        self.engine, self.conn, self.store, self.ns = engine, connector, store, ns
        self.group, self.leader, self.is_leader = group, leader, is_leader

    def _bcast(self, obj):
        import torch.distributed as dist

        box = [obj]
        dist.broadcast_object_list(box, src=self.leader, group=self.group)
        return box[0]


class PrefillWorker(_Worker):
    """Runs on every prefill rank; ``poll_and_step`` once per loop iteration."""

    def __init__(self, engine, connector, store, ns, group, leader, is_leader, rank_in_group: int):
        super().__init__(engine, connector, store, ns, group, leader, is_leader)
        self.rank = rank_in_group
        self.next_job = 0
        self.total = -1  # number of jobs announced by the decode side's stop mark (-1: serve forever)
        self.jobs: dict[str, _Job] = {}
        self.pending: list = []  # (event, job, first token, rng)
        engine.kv_export = self._export

    def _export(self, seqs) -> None:
        """A prompt finished: push the blocks not streamed yet (the last, partial one
        at least); its completion post waits for that copy (same stream, so every
        earlier chunk's copy of the prompt has completed too)."""
        bs = self.engine.pool.layout.block_size
        for s in seqs:
            job = self.jobs.pop(s.request_id)
            nblk = (len(s.prompt_ids) + bs - 1) // bs
            ev = self.conn.push(s.block_ids[job.pushed:nblk], job.blocks[job.pushed:nblk], job.k)
            job.pushed = nblk
            self.pending.append((ev, job, s.output_ids[-1], _advance_rng(s.rng_state, s.params)))

    def _stream_chunks(self) -> None:
        """After a step: push every prompt's blocks that this step completed (full
        16-token blocks of every layer), so long prompts move to the decode pool
        chunk by chunk while their later chunks still prefill."""
        bs = self.engine.pool.layout.block_size
        for job in self.jobs.values():
            s = job.seq
            if s is None or s.status.finished:
                continue
            full = min(s.num_computed, len(s.prompt_ids)) // bs
            if full > job.pushed:
                self.conn.push(s.block_ids[job.pushed:full], job.blocks[job.pushed:full], job.k)
                job.pushed = full

    def progress(self) -> str:
        return (f"jobs seen {self.next_job}/{self.total}, prefilling {len(self.jobs)}, pushes in flight "
                f"{len(self.pending)}, engine busy {self.engine.has_unfinished()}, "
                f"free blocks {self.engine.allocator.num_free()}")

    def poll_and_step(self) -> bool:
        new = []
        total = self.total
        if self.is_leader:
            # read the stop mark (it carries the job count) before the jobs, so
            # every job posted before it is seen in this same poll
            if total < 0 and self.store.check([f"{self.ns}/stop"]):
                total = int(self.store.get(f"{self.ns}/stop"))
            while self.store.check([f"{self.ns}/job/{self.next_job + len(new)}"]):
                new.append(pickle.loads(self.store.get(f"{self.ns}/job/{self.next_job + len(new)}")))
        new, self.total = self._bcast((new, total))
        for j in new:
            self.next_job += 1
            self.jobs[j.request_id] = j
            p = SamplingParams(**{**j.params.__dict__, "max_new_tokens": 1})
            j.seq = self.engine.add_request(j.request_id, j.prompt, p)
        if self.engine.has_unfinished():
            self.engine.step()
            if self.conn.mode != "host":
                self._stream_chunks()
        more = (self.total < 0 or self.next_job < self.total or bool(self.jobs) or self.engine.has_unfinished())
        # The decision to go on must be the same on every rank of the group (each
        # poll holds a broadcast), so it never depends on this rank's copies in
        # flight: when the group is done, every rank waits for its own copies and
        # posts their completions before leaving the loop.
        still = []
        for ev, job, tok, rng in self.pending:
            if ev is not None and not ev.query() and not more:
                ev.synchronize()
            if ev is None or ev.query():
                self.store.set(f"{self.ns}/done/{job.k}/{self.rank}", pickle.dumps((tok, rng)))
            else:
                still.append((ev, job, tok, rng))
        self.pending = still
        return more


class DecodeWorker(_Worker):
    """Runs on every decode rank; requests enter through ``submit`` (all ranks,
    same order) and the loop calls ``poll_and_step``."""

    def __init__(self, engine, connector, store, ns, group, leader, is_leader, prefill_ranks: int):
        super().__init__(engine, connector, store, ns, group, leader, is_leader)
        self.prefill_ranks = prefill_ranks
        self.next_job = 0
        self.waiting: list[_Job] = []   # posted to the prefill side, KV not arrived yet
        self.submitted: list[_Job] = []

    def submit(self, request_id: str, prompt: list, params: SamplingParams) -> _Job:
        bs = self.engine.pool.layout.block_size
        nblk = (len(prompt) + bs - 1) // bs
        blocks = list(self.engine.allocator.allocate(nblk))
        job = _Job(self.next_job, request_id, [int(t) for t in prompt], blocks, params)
        self.next_job += 1
        if self.is_leader:
            self.store.set(f"{self.ns}/job/{job.k}", pickle.dumps(job))
        self.waiting.append(job)
        self.submitted.append(job)
        return job

    def poll_and_step(self) -> bool:
        ready = []
        if self.is_leader:
            for job in self.waiting:
                keys = [f"{self.ns}/done/{job.k}/{r}" for r in range(self.prefill_ranks)]
                if not self.store.check(keys):
                    break  # adopt in submission order
                tok, rng = pickle.loads(self.store.get(keys[0]))
                for k in keys:
                    self.store.delete_key(k)
                ready.append((job.k, tok, rng))
        ready = self._bcast(ready)
        for k, tok, rng in ready:
            job = self.waiting.pop(0)
            assert job.k == k
            self.conn.receive(job.k, job.blocks)
            job.seq = self.engine.add_prefilled(job.request_id, job.prompt, tok, job.blocks, job.params, rng)
            job.seq.arrival = job.t_submit  # TTFT counts from submission to the decode side
        if self.engine.has_unfinished():
            self.engine.step()
        return bool(self.waiting) or self.engine.has_unfinished()

    def progress(self) -> str:
        return (f"submitted {len(self.submitted)}, waiting for KV {len(self.waiting)}, "
                f"engine busy {self.engine.has_unfinished()}, free blocks {self.engine.allocator.num_free()}")

    def stop(self) -> None:
        """Tell the prefill side that no job beyond those submitted will come."""
        if self.is_leader:
            self.store.set(f"{self.ns}/stop", str(self.next_job).encode())


class Disaggregated:
    """One rank's part of a disaggregated deployment: builds the groups, the
    engine and the KV connector once; ``serve`` runs one batch of requests
    (every rank of the default process group calls each method)."""

    def __init__(self, make_engine, mode: str = "p2p", ns: str = "pd"):
        import torch.distributed as dist

        world, self.rank = dist.get_world_size(), dist.get_rank()
        self.pr, self.dr, self.gp, self.gd, np_, nd = _groups(world)
        self.P = len(self.pr)
        self.store = dist.distributed_c10d._get_default_store()
        self.role = "prefill" if self.rank < self.P else "decode"
        self.gi = self.rank if self.role == "prefill" else self.rank - self.P
        self.engine = make_engine(self.role, np_ if self.role == "prefill" else nd, self.gi, self.P)
        self.mode, self.ns, self.passes = mode, ns, 0
        # decode ranks publish their pools before the prefill ranks map them
        if self.role == "decode":
            self.conn = KVConnector(self.engine.pool, self.role, self.gi, self.store, ns, mode)
        dist.barrier()
        if self.role == "prefill":
            self.conn = KVConnector(self.engine.pool, self.role, self.gi, self.store, ns, mode)

    def serve(self, prompts: list, params: SamplingParams, timeout_s: float = 600.0, health=None):
        """Returns (outputs, sequences) in prompt order on decode ranks, (None, None) on prefill ranks.
        ``health``: a started :class:`~kapsl_sdk_b200.parallel.health.HeartbeatMonitor`; it is
        checked between steps, so a lost peer raises ``RankFailure`` here."""
        ns = f"{self.ns}/{self.passes}"
        self.passes += 1
        if self.role == "prefill":
            w = PrefillWorker(self.engine, self.conn, self.store, ns, self.gp, self.pr[0], self.gi == 0, self.gi)
        else:
            w = DecodeWorker(self.engine, self.conn, self.store, ns, self.gd, self.dr[0], self.gi == 0, self.P)
            for i, p in enumerate(prompts):
                w.submit(f"{ns}-{i}", p, params)
            w.stop()
        t0 = time.perf_counter()
        debug = os.environ.get("KAPSL_PD_DEBUG", "0") == "1"
        last_log = t0
        while w.poll_and_step():
            if health is not None:
                health.check()
            now = time.perf_counter()
            if debug and now - last_log > 5.0:
                print(f"[pd] {self.role} rank {self.rank} t={now - t0:.1f}s {w.progress()}", flush=True)
                last_log = now
            if now - t0 > timeout_s:
                raise TimeoutError(f"{self.role} rank {self.rank}: disaggregated serving did not finish "
                                   f"in {timeout_s} s ({w.progress()})")
        self.engine.kv_export = None
        if self.role == "prefill":
            return None, None
        return [j.seq.output_ids for j in w.submitted], [j.seq for j in w.submitted]

    def close(self) -> None:
        import torch.distributed as dist

        if self.engine.pool.device.type == "cuda":
            torch.cuda.synchronize(self.engine.pool.device)
        dist.barrier()
        self.conn.close()


def serve_disaggregated(make_engine, prompts: list, params: SamplingParams, mode: str = "p2p",
                        ns: str = "pd", timeout_s: float = 600.0):
    """One-shot helper: build a :class:`Disaggregated` deployment, serve
    ``prompts`` and close the connector.  Returns (engine, outputs, sequences);
    outputs and sequences are None on prefill ranks."""
    d = Disaggregated(make_engine, mode, ns)
    outs, seqs = d.serve(prompts, params, timeout_s)
    d.close()
    return d.engine, outs, seqs
