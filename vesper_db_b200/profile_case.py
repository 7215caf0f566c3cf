"""A small, self-contained IVF-PQ search case for profiling the search kernels.

Builds an index from a seeded random model (no training) -- centroids drawn from a
Gaussian mixture, random PQ codebooks, optionally a random orthogonal OPQ rotation --
adds `n` vectors generated on the device, frees them, and runs `iters` device-resident
searches.  Sized so a profiler capture holds well under 1 GB of device memory while
the PQ codes still exceed L2 (n * m bytes; 2M x 96 = 192 MB by default).

    python -m vesper_db_b200.profile_case [--n 2000000 --dim 768 --nlist 16384 --m 96
                                            --nq 2000 --nprobe 32 --k 10 --iters 3 --opq]
"""
from __future__ import annotations

import argparse
import json


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--n", type=int, default=2_000_000)
    ap.add_argument("--dim", type=int, default=768)
    ap.add_argument("--nlist", type=int, default=16384)
    ap.add_argument("--m", type=int, default=96)
    ap.add_argument("--nq", type=int, default=2000)
    ap.add_argument("--nprobe", type=int, default=32)
    ap.add_argument("--k", type=int, default=10)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--opq", action="store_true")
    a = ap.parse_args()

    import numpy as np
    import torch

    from vesper_db_b200 import IvfPqIndex

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    centres = torch.rand(a.nlist, a.dim, generator=g, device=dev) * 2 - 1
    cb = 0.3 * torch.randn(a.m * 256, a.dim // a.m, generator=g, device=dev)
    R = torch.linalg.qr(torch.randn(a.dim, a.dim, generator=g, device=dev))[0] if a.opq else None
    idx = IvfPqIndex()
    idx.set_model(centres.cpu().numpy(), cb.cpu().numpy(), None if R is None else R.cpu().numpy())
    chunk = 250_000
    for c0 in range(0, a.n, chunk):
        n = min(chunk, a.n - c0)
        lab = torch.randint(0, a.nlist, (n,), generator=g, device=dev)
        x = centres[lab] + 0.15 * torch.randn(n, a.dim, generator=g, device=dev)
        ids = torch.arange(c0, c0 + n, device=dev, dtype=torch.int64)
        idx.add_device(ids.data_ptr(), x.data_ptr(), n)
        del x, ids, lab
    lab = torch.randint(0, a.nlist, (a.nq,), generator=g, device=dev)
    q = (centres[lab] + 0.15 * torch.randn(a.nq, a.dim, generator=g, device=dev)).contiguous()
    del centres
    torch.cuda.empty_cache()
    out_i = torch.empty((a.nq, a.k), dtype=torch.int64, device=dev)
    out_d = torch.empty((a.nq, a.k), dtype=torch.float32, device=dev)
    res = []
    for _ in range(a.iters):
        idx.search_batch_device(q.data_ptr(), a.nq, a.k, a.nprobe, out_i.data_ptr(), out_d.data_ptr())
        res.append(idx.last_timings())
    t = res[-1]
    t["scan_GBps_algorithmic"] = t["scanned_entries"] * a.m / (t["scan_ms"] / 1e3) / 1e9
    free, total = torch.cuda.mem_get_info()
    t["device_mem_in_use_GB"] = (total - free) / 1e9
    print(json.dumps({"case": vars(a), "last_timings": t, "stats": idx.get_stats()}))
    _ = np


if __name__ == "__main__":
    main()
