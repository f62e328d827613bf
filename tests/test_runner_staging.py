"""The GPU runner's host staging (ModelRunner._fill) writes every step's inputs
into pinned buffers with whole-array numpy assignments.  It must write exactly
what the element-by-element statement below writes: random decode / prefill /
padding mixes are filled by both and the buffers compared bit for bit (no GPU:
the staging buffers are host arrays)."""
import random

import numpy as np
import pytest

from kapsl_sdk_b200.llm.model_runner import ModelRunner, _Layout
from kapsl_sdk_b200.llm.scheduler import ScheduledBatch
from kapsl_sdk_b200.llm.sequence import SamplingParams, Sequence


class HostRunner(ModelRunner):
    """ModelRunner with plain host arrays in place of pinned and device buffers."""

    def __init__(self, max_seqs=16, max_tokens=256, max_len=1024, bs=16):
        self.bs, self.max_seqs = bs, max_seqs
        self.max_tokens = max_tokens + max_seqs
        self.max_blocks = (max_len + bs - 1) // bs
        S = max_seqs + 1
        self.pad_slot = max_seqs
        W = (max_tokens + 63) // 64 + max_seqs
        self.L = _Layout(self.max_tokens, S, self.max_blocks, W)
        rng = np.random.default_rng(0)
        self.n32 = rng.integers(-5, 5, self.L.n32).astype(np.int32)  # stale contents from "earlier steps"
        self.n64 = rng.integers(-5, 5, self.L.n64).astype(np.int64)
        self.f32view = self.n32.view(np.float32)


def reference_fill(self, batch, pad_to=0):
    L, n32, n64, f32 = self.L, self.n32, self.n64, self.f32view
    MB = self.max_blocks
    dec = batch.decode
    Bd = len(dec)
    for i, s in enumerate(dec):
        pos = s.length - 1
        if s.pending is not None:  # input token still on the device: its sampler row
            n32[L.src + i] = s.pending[1]
            n32[L.ids + i] = 0
        else:
            n32[L.src + i] = -1
            n32[L.ids + i] = s.output_ids[-1] if s.output_ids else s.prompt_ids[-1]
        n32[L.pos + i] = pos
        n64[L.slots + i] = s.block_ids[pos // self.bs] * self.bs + pos % self.bs
        n32[L.ctx + i] = s.length
        nb = len(s.block_ids)
        n32[L.bt + i * MB:L.bt + i * MB + nb] = s.block_ids
    Bpad = max(Bd, pad_to)
    for i in range(Bd, Bpad):
        n32[L.ids + i] = 0
        n32[L.src + i] = -1
        n32[L.pos + i] = 0
        n64[L.slots + i] = -1
        n32[L.ctx + i] = 1
        n32[L.bt + i * MB] = 0
    t = Bpad
    nwork = 0
    sample_seqs = list(dec)
    lrows = list(range(Bd))
    for j, (s, n) in enumerate(batch.prefill):
        row = Bpad + j
        p0 = s.num_computed
        npr = len(s.prompt_ids)
        toks = s.prompt_ids[p0:p0 + n] if p0 + n <= npr else (s.prompt_ids + s.output_ids)[p0:p0 + n]
        n32[L.ids + t:L.ids + t + n] = toks
        pos = np.arange(p0, p0 + n, dtype=np.int64)
        n32[L.pos + t:L.pos + t + n] = pos
        blk = np.asarray(s.block_ids, dtype=np.int64)
        n64[L.slots + t:L.slots + t + n] = blk[pos // self.bs] * self.bs + pos % self.bs
        n32[L.ctx + row] = p0 + n
        nb = len(s.block_ids)
        n32[L.bt + row * MB:L.bt + row * MB + nb] = s.block_ids
        si = L.sinfo + j * 4
        n32[si:si + 4] = (t, n, p0 + n, row)
        for t0 in range(0, n, 64):
            n32[L.work + nwork * 2] = j
            n32[L.work + nwork * 2 + 1] = t0
            nwork += 1
        if p0 + n >= s.length:
            sample_seqs.append(s)
            lrows.append(t + n - 1)
        t += n
    R = len(sample_seqs)
    Rpad = max(R, pad_to) if pad_to else R
    for r in range(Rpad):
        if r < R:
            s = sample_seqs[r]
            n64[L.lidx + r] = lrows[r]
            n32[L.sslot + r] = s.slot
            f32[L.temp + r] = s.params.temperature
            n32[L.topk + r] = s.params.top_k
            f32[L.topp + r] = s.params.top_p
            f32[L.pen + r] = s.params.repetition_penalty
        else:
            n64[L.lidx + r] = r
            n32[L.sslot + r] = self.pad_slot
            f32[L.temp + r] = 0.0
            n32[L.topk + r] = 0
            f32[L.topp + r] = 1.0
            f32[L.pen + r] = 1.0
    S = Bpad + len(batch.prefill)
    return t, S, R, Rpad, Bd, Bpad, nwork, sample_seqs


def _seq(rnd, i, bs=16):
    npr = rnd.randint(1, 300)
    nout = rnd.randint(0, 40)
    s = Sequence(seq_id=i, request_id=f"r{i}", prompt_ids=[rnd.randrange(1000) for _ in range(npr)],
                 params=SamplingParams(temperature=rnd.choice([0.0, 0.7, 1.3]), top_k=rnd.choice([0, 40]),
                                       top_p=rnd.choice([1.0, 0.9]), repetition_penalty=rnd.choice([1.0, 1.15])))
    s.output_ids = [rnd.randrange(1000) for _ in range(nout)]
    s.block_ids = rnd.sample(range(5000), (s.length + bs) // bs + rnd.randint(0, 2))
    s.slot = i
    return s


def _batch(rnd, seqs):
    b = ScheduledBatch()
    for s in seqs:
        s.pending = None
        if s.output_ids and rnd.random() < 0.6:
            s.num_computed = s.length - 1
            b.decode.append(s)
            if rnd.random() < 0.5:  # last token sampled by the step still in flight
                s.pending = (7, rnd.randrange(16))
        else:
            s.num_computed = rnd.randint(0, s.length - 1)
            b.prefill.append((s, rnd.randint(1, s.length - s.num_computed)))
    return b


@pytest.mark.parametrize("seed", range(40))
def test_fill_matches_elementwise_statement(seed):
    rnd = random.Random(seed)
    a, b = HostRunner(), HostRunner()
    for step in range(4):  # consecutive steps over the same (growing / replaced) block tables
        seqs = [_seq(rnd, i) for i in range(rnd.randint(0, 8))] if step == 0 or rnd.random() < 0.3 else seqs
        for s in seqs:
            if rnd.random() < 0.3:
                s.block_ids.extend(rnd.sample(range(5000, 6000), 2))  # grown in place
            elif rnd.random() < 0.1:
                s.block_ids = list(reversed(s.block_ids))  # replaced (same length)
        batch = _batch(rnd, seqs)
        if sum(n for _, n in batch.prefill) + len(batch.decode) > 250:
            continue
        pad = rnd.choice([0, 0, len(batch.decode) + rnd.randint(0, 4)]) if not batch.prefill else 0
        ra = ModelRunner._fill(a, batch, pad)
        rb = reference_fill(b, batch, pad)
        assert ra[:7] == rb[:7] and ra[7] == rb[7], (seed, step)
        assert np.array_equal(a.n32, b.n32), (seed, step, np.nonzero(a.n32 != b.n32)[0][:10])
        assert np.array_equal(a.n64, b.n64), (seed, step, np.nonzero(a.n64 != b.n64)[0][:10])


def test_block_table_cache_follows_the_list():
    s = Sequence(seq_id=0, request_id="r", prompt_ids=[1], params=SamplingParams())
    s.block_ids = [3, 4]
    assert s.block_table().tolist() == [3, 4]
    s.block_ids.extend([9])
    assert s.block_table().tolist() == [3, 4, 9]
    s.block_ids = [7, 8, 1]  # same length, new list
    assert s.block_table().tolist() == [7, 8, 1]
    assert s.block_table() is s.block_table()
