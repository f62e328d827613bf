"""Serving one model over a tensor- or expert-parallel group (one process per GPU).

Rank 0 of the group, the *leader*, owns the request stream: the socket / SHM
servers and :class:`~kapsl_sdk_b200.llm.backend.LLMBackend` run there, over a
:class:`GroupLeader` instead of a bare engine.  Every ``step()`` of the leader
first publishes the step's events (requests queued since the last step, with
the prompt after session history, the sequence id and the sampler seed the
leader resolved; aborts) and then steps its own engine.  The other ranks run
:func:`follow`: take the next event batch, apply it, step.  All ranks thus
queue identical sequences and take identical scheduling decisions; the
model's collectives keep their kernels in lock step, and the vocab-parallel
sampler hands every rank the same tokens, so followers send nothing back.

Events travel through :class:`StepChannel`, a single-producer ring of byte
messages in POSIX shared memory (every rank of a group is on one node): the
leader writes a slot and then its sequence number; a follower polls the
sequence number, copies the message and acknowledges it; the leader reuses a
slot only once every follower acknowledged its previous message.  Waits on
either side are bounded; a rank that stops consuming (or producing) turns
into a ``TimeoutError`` on its peers, next to the device-side wait limits of
the collectives.

Reference counterpart: the reference routes a tensor-parallel group's requests
to the group's first worker (crates/kapsl-scheduler/src/mesh_routing.rs:100-145)
but has no model that runs on a group.
"""
from __future__ import annotations

import pickle
import time
from multiprocessing import shared_memory
from typing import Optional

import numpy as np

_MAGIC = 0x4B50534C53544550  # "KPSLSTEP"
# header int64 words: magic, slots, slot_bytes, world, published seq, then one ack word per rank
_H_MAGIC, _H_SLOTS, _H_BYTES, _H_WORLD, _H_SEQ, _H_ACK = 0, 1, 2, 3, 4, 8


class StepChannel:
    """Ring of ``slots`` messages of at most ``slot_bytes`` each, one writer
    (rank 0) and ``world - 1`` readers, in shared memory ``name``."""

    def __init__(self, name: str, world: int, rank: int, slots: int = 8, slot_bytes: int = 8 << 20,
                 create: Optional[bool] = None, timeout_s: float = 60.0):
        self.name, self.world, self.rank = name, world, rank
        self.timeout_s = timeout_s
        create = rank == 0 if create is None else create
        hdr_words = _H_ACK + max(world, 1)
        self.hdr_bytes = (hdr_words * 8 + 4095) // 4096 * 4096
        if create:
            try:  # a ring left by a crashed run of the same name
                old = shared_memory.SharedMemory(name=name)
                old.close()
                old.unlink()
            except FileNotFoundError:
                pass
            size = self.hdr_bytes + slots * (16 + slot_bytes)
            self.shm = shared_memory.SharedMemory(name=name, create=True, size=size)
            self.hdr = np.ndarray((hdr_words,), dtype=np.int64, buffer=self.shm.buf)
            self.hdr[:] = 0
            self.hdr[_H_SLOTS], self.hdr[_H_BYTES], self.hdr[_H_WORLD] = slots, slot_bytes, world
            self.hdr[_H_MAGIC] = _MAGIC
        else:
            t0 = time.monotonic()
            while True:
                try:
                    self.shm = shared_memory.SharedMemory(name=name)
                    hdr = np.ndarray((hdr_words,), dtype=np.int64, buffer=self.shm.buf)
                    if hdr[_H_MAGIC] == _MAGIC:
                        self.hdr = hdr
                        break
                    del hdr
                    self.shm.close()
                except FileNotFoundError:
                    pass
                if time.monotonic() - t0 > timeout_s:
                    raise TimeoutError(f"step channel {name!r} did not appear within {timeout_s} s")
                time.sleep(0.01)
            slots, slot_bytes = int(self.hdr[_H_SLOTS]), int(self.hdr[_H_BYTES])
        self.slots, self.slot_bytes = slots, slot_bytes
        self.created = create
        self.seq = 0  # last published (leader) / received (follower)

    def _slot(self, seq: int):
        off = self.hdr_bytes + (seq % self.slots) * (16 + self.slot_bytes)
        meta = np.ndarray((2,), dtype=np.int64, buffer=self.shm.buf, offset=off)
        return meta, off + 16

    def _wait(self, cond, what: str, timeout_s: Optional[float]) -> None:
        t0 = time.monotonic()
        lim = self.timeout_s if timeout_s is None else timeout_s
        spins = 0
        while not cond():
            spins += 1
            if spins > 2000:  # back off after ~a few hundred microseconds of spinning
                time.sleep(0.0002 if spins < 20000 else 0.002)
            if time.monotonic() - t0 > lim:
                raise TimeoutError(f"step channel: {what} timed out after {lim} s")

    def publish(self, payload: bytes, timeout_s: Optional[float] = None) -> int:
        """Leader: append one message; returns its sequence number (1, 2, ...)."""
        if len(payload) > self.slot_bytes:
            raise ValueError(f"step message of {len(payload)} bytes exceeds the {self.slot_bytes}-byte slots")
        seq = self.seq + 1
        need = seq - self.slots  # the message this slot held last
        if need > 0 and self.world > 1:
            acks = self.hdr[_H_ACK + 1:_H_ACK + self.world]
            self._wait(lambda: int(acks.min()) >= need, f"followers acknowledging message {need}", timeout_s)
        meta, off = self._slot(seq)
        self.shm.buf[off:off + len(payload)] = payload
        meta[1] = len(payload)
        meta[0] = seq  # written last: a reader that sees seq sees the payload (x86-64 stores are ordered)
        self.hdr[_H_SEQ] = seq
        self.seq = seq
        return seq

    def receive(self, timeout_s: Optional[float] = None) -> bytes:
        """Follower: the next message (blocks, bounded)."""
        seq = self.seq + 1
        meta, off = self._slot(seq)
        self._wait(lambda: int(meta[0]) == seq, f"message {seq}", timeout_s)
        n = int(meta[1])
        data = bytes(self.shm.buf[off:off + n])
        self.seq = seq
        self.hdr[_H_ACK + self.rank] = seq
        return data

    def close(self) -> None:
        try:
            del self.hdr
        except AttributeError:
            pass
        self.shm.close()
        if self.created:
            try:
                self.shm.unlink()
            except FileNotFoundError:
                pass


class GroupLeader:
    """Engine facade for rank 0 of a serving group: the methods LLMBackend uses
    (``add_request``, ``abort``, ``step``, ``has_unfinished``, ``shutdown``) plus
    attribute pass-through to the wrapped engine."""

    def __init__(self, engine, channel: StepChannel):
        self.engine = engine
        self.channel = channel
        self._events: list = []
        self._stopped = False

    def __getattr__(self, name):
        return getattr(self.engine, name)

    def add_request(self, request_id: str, prompt_ids: list, params=None, session_id: Optional[str] = None,
                    on_token=None, admission_control: bool = False):
        seq = self.engine.add_request(request_id, prompt_ids, params, session_id=session_id, on_token=on_token,
                                      admission_control=admission_control)
        # the resolved sequence (after session history, with its id and seed) is what followers queue
        self._events.append(("add", request_id, np.asarray(seq.prompt_ids, dtype=np.int32), seq.params,
                             seq.seq_id, seq.rng_state, session_id))
        return seq

    def abort(self, request_id: str) -> None:
        self.engine.abort(request_id)
        self._events.append(("abort", request_id))

    def has_unfinished(self) -> bool:
        return self.engine.has_unfinished()

    def step(self):
        events, self._events = self._events, []
        self.channel.publish(pickle.dumps(events, protocol=pickle.HIGHEST_PROTOCOL))
        return self.engine.step()

    def generate(self, prompts: list, params=None) -> list:
        seqs = [self.add_request(f"gen-{i}-{time.monotonic_ns()}", p, params) for i, p in enumerate(prompts)]
        while self.has_unfinished():
            self.step()
        return [s.output_ids for s in seqs]

    def stop_followers(self) -> None:
        """Let the followers' :func:`follow` return (after the steps published so far)."""
        if not self._stopped:
            self._stopped = True
            self.channel.publish(pickle.dumps([("stop",)]))

    def shutdown(self) -> None:
        self.stop_followers()
        self.engine.shutdown()


def follow(engine, channel: StepChannel, idle_timeout_s: float = 3600.0, should_exit=None) -> int:
    """Follower loop: apply each published event batch to ``engine`` and step it,
    until the leader publishes a stop (the engine is left running for the
    caller).  ``should_exit()`` is polled while no message arrives (e.g. the
    leader was lost after a termination signal); a true value ends the loop.
    Returns the number of steps taken."""
    steps = 0
    idle_since = time.monotonic()
    while True:
        try:
            raw = channel.receive(timeout_s=1.0)
        except TimeoutError:
            if (should_exit is not None and should_exit()) or time.monotonic() - idle_since > idle_timeout_s:
                return steps
            continue
        idle_since = time.monotonic()
        events = pickle.loads(raw)
        stop = False
        for ev in events:
            kind = ev[0]
            if kind == "add":
                _, rid, prompt, params, seq_id, rng, session = ev
                engine.adopt_request(rid, prompt.tolist(), params, seq_id, rng, session)
            elif kind == "abort":
                engine.abort(ev[1])
            elif kind == "stop":
                stop = True
        if stop:
            return steps
        engine.step()
        steps += 1
