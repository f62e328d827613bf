"""Row-parallel GEMM + all-reduce micro-benchmark: fused NVLink path vs NCCL.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m kapsl_sdk_b200.utils.tp_bench M N_OUT K_TOTAL

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


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    if sys.argv[1] == "p2p":
        p2p_probe(dev, rank, world)
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
    for mode in ("fused", "norm", "norm_only", "scatter", "nccl", "nccl_norm", "gemm_only", "scatter_only",
                 "reduce_only"):
        fusedbuf = mode in ("fused", "norm", "norm_only", "scatter", "scatter_only", "reduce_only")
        tp = TPComm(world, rank, dev, ("scatter" if mode == "scatter" else "fused") if fusedbuf else "nccl", max_tokens=M, hidden=NO)
        h = tp.residual_stream(M) if fusedbuf else torch.zeros(M, NO, device=dev, dtype=torch.bfloat16)
        rpr = (M + world - 1) // world
        err = ops.error_buffer(dev)
        b = tp.bufs
        if mode == "norm":  # the layer boundary of the fused path: GEMM + reduce + residual + RMSNorm + all-gather
            fn = lambda: tp.row_parallel_norm(x, w, h, nw, 1e-6)
        elif mode == "norm_only":
            fn = lambda: c.tp_reduce_norm_ag(b["recv"], b["xnorm"], b["flags"], h, nw, 1e-6, rank, rpr, M, NO,
                                             tp.epoch, err, tp.timeout_ns)
        elif mode == "nccl_norm":  # the NCCL path's layer boundary: GEMM, all-reduce, residual add, RMSNorm
            xo = torch.empty_like(h)
            fn = lambda: (tp.row_parallel_residual(x, w, h), ops.rmsnorm(h, nw, 1e-6, out=xo))
        elif mode == "gemm_only":
            fn = lambda: ops.linear(x, w)
        elif mode == "scatter_only":
            fn = lambda: c.gemm_scatter(x, w, tp.bufs["recv"], rank, rpr, NO, err)
        elif mode == "reduce_only":
            fn = lambda: c.tp_reduce_ag(tp.bufs["recv"], tp.bufs["hidden"], tp.bufs["flags"], rank, rpr, M, NO, NO,
                                        tp.epoch, err, tp.timeout_ns)
        else:
            fn = lambda: tp.row_parallel_residual(x, w, h)
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
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
        if mode in ("fused", "norm"):
            st = tp.epoch.tolist()  # start, after barrier 1, last CTA done, after barrier 2 (ns)
            res[mode + "_phase_us"] = {"barrier1": (st[3] - st[2]) / 1e3, "work": (st[4] - st[3]) / 1e3,
                                       "barrier2": (st[5] - st[4]) / 1e3}
        tp.close()
    flops = 2 * M * NO * K
    nvl = 2 * (world - 1) / world * M * NO * 2
    roof = max(flops / peak, nvl / 770e9) * 1e3
    res["roofline_ms"] = round(roof, 4)
    res["fused_frac_of_roofline"] = round(roof / res["fused_ms"], 3)
    res["nccl_frac_of_roofline"] = round(roof / res["nccl_ms"], 3)
    if rank == 0:
        print(json.dumps(res), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
