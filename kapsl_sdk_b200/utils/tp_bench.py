"""Row-parallel GEMM + all-reduce micro-benchmark: fused NVLink path vs NCCL.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m kapsl_sdk_b200.utils.tp_bench M N_OUT K_TOTAL

Modes (``TP_BENCH_MODES``, comma-separated): ``ll`` the model's layer boundary
(GEMM + reduction + residual + RMSNorm, the kernel picked by row count),
``ll1`` / ``ll2`` forced flag-carrying-line one-shot / two-shot, ``ll_only1``
/ ``ll_only2`` those kernels alone, ``norm`` / ``norm_only`` the barrier + pull kernel,
``pull_large`` the default selection but with the pull kernel instead of
the scatter GEMM above the line-kernel sizes, ``fused`` the pull reduction without the norm, ``nccl`` / ``nccl_norm`` GEMM +
NCCL all-reduce (+ add + RMSNorm), ``gemm_only``.  ``tp_bench ping`` measures
the NVLink flag round trip between ranks 0 and 1.

Each rank holds a [M, K_TOTAL/N] slice of the input and a [N_OUT, K_TOTAL/N]
slice of the weight; one call computes h += all_reduce(x @ w.T).  Times are
CUDA-event device times, 20 calls after 3 warm-ups, max over ranks.  The
roofline for the fused call is the slower of the GEMM FLOPs at the measured
bf16 peak and the NVLink bytes (reduce-scatter + all-gather: 2 * (N-1)/N *
M * N_OUT * 2 bytes sent per rank) at 770 GB/s per direction.
"""
from __future__ import annotations

import json
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist


def p2p_probe(dev, rank, world):
    """SM-driven NVLink bandwidth: rank 0 writes into / reads from rank 1's memory."""
    from .._ext import cuda_ops

    c = cuda_ops()
    nbytes = 256 << 20
    base = c.symm_alloc(2 * nbytes)
    handles = [None] * world
    dist.all_gather_object(handles, c.symm_handle(base))
    peer = c.symm_open(handles[1 - rank]) if world == 2 else None
    res = {}
    for ctas in (1, 2, 4, 8):
        for kind in ("write", "read", "local"):
            if kind == "write":
                dst, src = peer, base
            elif kind == "read":
                dst, src = base, peer
            else:
                dst, src = base + nbytes, base
            dist.barrier()
            if rank == 0:
                for _ in range(2):
                    c.p2p_copy(dst, src, nbytes, ctas)
                torch.cuda.synchronize()
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                for _ in range(5):
                    c.p2p_copy(dst, src, nbytes, ctas)
                e.record()
                torch.cuda.synchronize()
                res[f"{kind}_ctas{ctas}_GBps"] = round(5 * nbytes / (s.elapsed_time(e) / 1e3) / 1e9, 1)
            dist.barrier()
    if rank == 0:
        print(json.dumps(res), flush=True)
    torch.cuda.synchronize()
    dist.barrier()
    if peer:
        c.symm_close(peer)
    c.symm_free(base)


def ping_probe(dev, rank, world):
    """NVLink flag round trip between ranks 0 and 1 (one thread per GPU bouncing a
    counter): release/acquire, relaxed, and data-then-fence-then-flag."""
    from .. import ops
    from .._ext import cuda_ops

    c = cuda_ops()
    nbytes = 4 << 20
    base = c.symm_alloc(nbytes + 4096)
    handles = [None] * world
    dist.all_gather_object(handles, c.symm_handle(base))
    res = {}
    if rank < 2:
        peer = c.symm_open(handles[1 - rank])
        out = torch.zeros(1, dtype=torch.int64, device=dev)
        err = ops.error_buffer(dev)
        nxt = 0
        for mode, payload in ((0, 0), (1, 0), (2, 0), (2, 65536), (2, 1 << 20)):
            for it in (1, 200):
                torch.cuda.synchronize()
                dist.barrier(group=None)
                c.flag_pingpong(base, peer, peer + 4096, payload, rank, it, mode, nxt, int(2e9), out, err)
                torch.cuda.synchronize()
                nxt += it
                if it > 1:
                    res[f"mode{mode}_payload{payload}_rt_us"] = round(int(out.item()) / 1e3, 2)
        res["err"] = ops.check_errors(dev)
        torch.cuda.synchronize()
        dist.barrier()
        c.symm_close(peer)
    else:
        for _ in range(10):
            dist.barrier()
        dist.barrier()
    if rank == 0:
        print(json.dumps({"ping": res}), flush=True)
    torch.cuda.synchronize()
    dist.barrier()
    c.symm_free(base)


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    if sys.argv[1] in ("p2p", "ping"):
        (p2p_probe if sys.argv[1] == "p2p" else ping_probe)(dev, rank, world)
        dist.destroy_process_group()
        return
    M, NO, KT = (int(x) for x in sys.argv[1:4])
    from .. import ops
    from ..parallel.tp import TPComm

    K = KT // world
    x = torch.randn(M, K, device=dev, dtype=torch.bfloat16)
    w = torch.randn(NO, K, device=dev, dtype=torch.bfloat16) / 64
    res = {"M": M, "N": NO, "K_total": KT, "world": world}
    peak = 1666.7e12
    try:
        import json as _j

        peak = _j.load(open(os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")))[
            "bf16_tflops"] * 1e12
    except Exception:
        pass
    from .._ext import cuda_ops

    c = cuda_ops()
    nw = torch.ones(NO, device=dev, dtype=torch.bfloat16)
    modes = os.environ.get("TP_BENCH_MODES", "ll,ll1,ll2,ll_only1,ll_only2,pull_large,norm,norm_only,nccl,"
                                             "nccl_norm,gemm_only").split(",")
    for mode in modes:
        fusedbuf = mode not in ("nccl", "nccl_norm", "gemm_only")
        tp = TPComm(world, rank, dev, "fused" if fusedbuf else "nccl", max_tokens=M, hidden=NO)
        if mode in ("rows1", "rows_only1"):
            tp.oneshot_rows = 1 << 30
        elif mode in ("rows2", "rows_only2"):
            tp.oneshot_rows = 0
        if mode in ("ll1", "ll_only1"):
            tp.ll1_rows, tp.ll2_rows = M, 0
        elif mode in ("ll2", "ll_only2"):
            tp.ll1_rows, tp.ll2_rows = 0, M
        if mode in ("ll1", "ll_only1", "ll2", "ll_only2"):
            tp.close()  # re-size the slots
            tp._setup_symmetric(M, NO)
        if mode in ("norm", "norm_only"):
            tp.norm_kernel = "pull"
        if mode == "pull_large":  # the layer boundary with the pull kernel above the line-kernel sizes
            tp.large_kernel = "pull"
        h = tp.residual_stream(M) if fusedbuf else torch.zeros(M, NO, device=dev, dtype=torch.bfloat16)
        rpr = (M + world - 1) // world
        err = ops.error_buffer(dev)
        b = tp.bufs
        if mode in ("norm", "ll", "ll1", "ll2", "pull_large"):  # GEMM + reduce + residual + norm
            fn = lambda: tp.row_parallel_norm(x, w, h, nw, 1e-6)
        elif mode in ("ll_only1", "ll_only2"):
            two = mode == "ll_only2"
            own = tp.own_buf[:M]
            own.copy_(ops.linear(x, w))
            fn = lambda: c.tp_ll_norm(own, b["ll"], b["llg"], h, tp.xnorm_buf[:M], nw, 1e-6, rank, rpr, M, tp.ll_cap,
                                      two, tp.epoch, err, tp.timeout_ns, None, 1)
        elif mode == "norm_only":
            fn = lambda: c.tp_reduce_norm_ag(b["recv"], b["xnorm"], b["flags"], h, nw, 1e-6, rank, rpr, M, NO,
                                             tp.epoch, err, tp.timeout_ns)
        elif mode == "nccl_norm":  # the NCCL path's layer boundary: GEMM, all-reduce, residual add, RMSNorm
            xo = torch.empty_like(h)
            fn = lambda: (tp.row_parallel_residual(x, w, h), ops.rmsnorm(h, nw, 1e-6, out=xo))
        elif mode == "gemm_only":
            fn = lambda: ops.linear(x, w)
        else:
            fn = lambda: tp.row_parallel_residual(x, w, h)
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        if fusedbuf:
            tp.phase_times(reset=True)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(20):
            fn()
        e.record()
        torch.cuda.synchronize()
        ms = torch.tensor([s.elapsed_time(e) / 20], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        res[mode + "_ms"] = round(float(ms), 4)
        res[mode + "_err"] = ops.check_errors(dev)
        if fusedbuf:  # rank 0's mean phase times (us): first wait, data, second wait
            res[mode + "_phase_us"] = {k: round(v, 2) for k, v in tp.phase_times().items() if k != "calls"}
        tp.close()
    flops = 2 * M * NO * K
    nvl = 2 * (world - 1) / world * M * NO * 2
    roof = max(flops / peak, nvl / 770e9) * 1e3
    res["roofline_ms"] = round(roof, 4)
    for k in ("ll", "norm", "nccl"):
        if k + "_ms" in res:
            res[k + "_frac_of_roofline"] = round(roof / res[k + "_ms"], 3)
    if rank == 0:
        print(json.dumps(res), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
