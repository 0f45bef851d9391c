"""Data-parallel collective micro-benchmark: native peer-memory kernels vs NCCL.

Launch one process per GPU, e.g.::

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        benchmarks/bench_collectives.py

For each message size it times, with CUDA events on the launching stream and
the maximum over ranks:

* ``native all-reduce``: :meth:`SymmetricWorkspace.all_reduce_mean` — the
  two-shot in-place fp32 mean over CUDA-IPC peer buffers (fixed rank order,
  scale fused, result written to every rank);
* ``nccl all-reduce``: ``dist.all_reduce`` (SUM) plus the scale, on a plain
  fp32 tensor;
* ``native reduce-scatter``: the same kernel writing only this rank's shard
  (the sharded optimizer's first half);
* ``native one-shot all-reduce``: every rank reads every rank's whole buffer
  and writes the mean locally (one phase; compare with the two-shot to place
  the crossover ``ONESHOT_MAX_ELEMS``).

Sizes are in KiB (``--sizes-kib``) so the latency-bound range is covered.

Each line reports milliseconds, bus bandwidth and the fraction of the NVLink
roofline (bus bandwidth ÷ the per-direction link bandwidth). For the two-shot
all-reduce the bytes leaving a rank on its link are the (n-1)/n of its buffer
that the peers read in the reduce phase plus the (n-1)/n it writes to the
peers in the gather phase, so the bus figure is ``2(n-1)/n · bytes / t``; the
reduce-scatter moves only the first half, ``(n-1)/n · bytes / t``.
"""

from __future__ import annotations

import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

from thundersync_b200.parallel.symm import SymmetricWorkspace


def _time(fn, iters: int, device) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize(device)
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize(device)
    ms = torch.tensor([a.elapsed_time(b) / iters], device=device, dtype=torch.float64)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return float(ms.item())


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--sizes-kib", default="16,64,256,1024,4096,16384,65536,262144,1048576,4194304")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--link-gbs", type=float, default=770.0, help="measured peer-copy GB/s per direction")
    args = ap.parse_args(argv)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=300))
    world, rank = dist.get_world_size(), dist.get_rank()
    ws = SymmetricWorkspace(device)
    rows = []
    for kib in (int(x) for x in args.sizes_kib.split(",")):
        n = (kib << 10) // 4
        buf, ptrs = ws.alloc(n, torch.float32)
        buf.normal_()
        plain = torch.randn(n, device=device)
        out = torch.empty(n, device=device)
        nbytes = n * 4
        t_native = _time(lambda: ws.all_reduce_mean(buf, ptrs), args.iters, device)
        ws.check()
        t_one = _time(lambda: ws.all_reduce_mean_oneshot(buf, ptrs, out), args.iters, device)
        ws.check()

        def nccl():
            dist.all_reduce(plain)
            plain.mul_(1.0 / world)

        t_nccl = _time(nccl, args.iters, device)
        t_rs = _time(lambda: ws.reduce_scatter(buf, ptrs), args.iters, device)
        ws.check()
        frac = (world - 1) / world
        for name, t in (("native all-reduce", t_native), ("native one-shot all-reduce", t_one),
                        ("nccl all-reduce", t_nccl), ("native reduce-scatter", t_rs)):
            # bus bandwidth in the usual all-reduce convention (2(n-1)/n of the buffer per rank), so the
            # one-shot and two-shot lines compare directly; the reduce-scatter moves (n-1)/n
            link_bytes = (2 if "all-reduce" in name else 1) * frac * nbytes
            bus = link_bytes / (t / 1e3) / 1e9
            roof = bus / args.link_gbs
            rows.append({"op": name, "kib": kib, "ms": round(t, 4), "bus_gbs": round(bus, 1),
                         "nvlink_roofline_fraction": round(roof, 3), "world": world})
        del buf, plain, out
    if rank == 0:
        for r in rows:
            print(json.dumps(r))
    ws.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
