"""A self-contained IVF-PQ search case for profiling the search kernels.

--data uniform (default): a seeded random model (no training) -- centroids drawn
  uniformly, random PQ codebooks, optionally a random orthogonal OPQ rotation -- and
  `n` vectors generated on the device around the centroids (every list about n / nlist
  entries, each probed by about nq * nprobe / nlist queries).
--data bench: the benchmark's data distribution (vesper_db_b200.synth: 50,000
  anisotropic Gaussians) with the benchmark's training (131,072 rows, nlist 16,384,
  m 96, OPQ) and `n` base rows: lists as skewed as in the benchmark.
--save DIR writes the built index (reference v1.0 format) and exits; --load DIR reads
  it instead of building, so a profiler capture sees only the load and the searches.
--scan picks the FAST scan kernel (the engine's VGPU_SCAN switch).

    python -m vesper_db_b200.profile_case [--data uniform|bench] [--n 2000000 --dim 768
        --nlist 16384 --m 96 --nq 2000 --nprobe 32 --k 10 --iters 3 --opq]
        [--scan auto|tc|blocked] [--save DIR | --load DIR]
"""
from __future__ import annotations

import argparse
import json
import math
import os


def build_uniform(a, torch, dev, IvfPqIndex):
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
    return idx, q


def build_bench(a, torch, dev, IvfPqIndex):
    from . import synth
    n_centres, chunk, n_train = 50_000, 125_000, 131_072
    centres, sigmas = synth.gen_centres(torch, dev, n_centres, a.dim)
    q = synth.gen_queries(torch, dev, centres, sigmas, a.nq).contiguous()
    if a.load:
        return None, q
    train = torch.cat([synth.gen_base_chunk(torch, dev, centres, sigmas, c, chunk)
                       for c in range(math.ceil(n_train / chunk))])[:n_train].contiguous()
    idx = IvfPqIndex()
    idx.train_device(train.data_ptr(), n_train, a.dim, a.nlist, a.m, 8, use_opq=a.opq)
    del train
    buf = torch.empty((chunk, a.dim), device=dev)
    for c in range(math.ceil(a.n / chunk)):
        n = min(chunk, a.n - c * chunk)
        synth.gen_base_chunk(torch, dev, centres, sigmas, c, chunk, out=buf)
        ids = torch.arange(c * chunk, c * chunk + n, device=dev)
        idx.add_device(ids.data_ptr(), buf.data_ptr(), n)
    return idx, q


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--data", choices=["uniform", "bench"], default="uniform")
    ap.add_argument("--n", type=int, default=2_000_000)
    ap.add_argument("--dim", type=int, default=768)
    ap.add_argument("--nlist", type=int, default=16384)
    ap.add_argument("--m", type=int, default=96)
    ap.add_argument("--nq", type=int, default=2000)
    ap.add_argument("--nprobe", type=int, default=32)
    ap.add_argument("--k", type=int, default=10)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--opq", action="store_true")
    ap.add_argument("--scan", choices=["auto", "tc", "blocked"], default="auto")
    ap.add_argument("--save", default="")
    ap.add_argument("--load", default="")
    a = ap.parse_args()
    if a.scan != "auto":
        os.environ["VGPU_SCAN"] = a.scan

    import torch

    from vesper_db_b200 import IvfPqIndex

    dev = torch.device("cuda", 0)
    if a.data == "bench":
        idx, q = build_bench(a, torch, dev, IvfPqIndex)
    else:
        idx, q = build_uniform(a, torch, dev, IvfPqIndex)
    if a.load:
        idx = IvfPqIndex.from_file(a.load)
    if a.save:
        idx.save(a.save)
        print(json.dumps({"saved": a.save, "stats": idx.get_stats()}))
        return
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


if __name__ == "__main__":
    main()
