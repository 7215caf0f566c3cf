"""One exact flat top-k call on a seeded unit-vector case, for profiling.

    python -m vesper_db_b200.profile_flat --n 300000 --nq 2048 [--k 100] [--op ip|l2] [--iters 1]

Base and queries are N(0,1) rows normalised to unit length (torch generator seed 1, on the
device); each iteration is one vesper_flat_topk_device call; the stage times of the last
call are printed.
"""
from __future__ import annotations

import argparse


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--n", type=int, default=300_000)
    ap.add_argument("--nq", type=int, default=2048)
    ap.add_argument("--dim", type=int, default=768)
    ap.add_argument("--k", type=int, default=100)
    ap.add_argument("--op", default="ip", choices=["ip", "l2"])
    ap.add_argument("--iters", type=int, default=1)
    a = ap.parse_args()
    import torch

    from vesper_db_b200 import flat_topk_device
    from vesper_db_b200.flat import last_timings
    g = torch.Generator(device="cuda").manual_seed(1)
    base = torch.randn((a.n, a.dim), device="cuda", generator=g)
    base /= base.norm(dim=1, keepdim=True)
    q = torch.randn((a.nq, a.dim), device="cuda", generator=g)
    q /= q.norm(dim=1, keepdim=True)
    idx = torch.empty((a.nq, a.k), dtype=torch.int32, device="cuda")
    sc = torch.empty((a.nq, a.k), device="cuda")
    torch.cuda.synchronize()
    for _ in range(a.iters):
        flat_topk_device(1 if a.op == "ip" else 0, q.data_ptr(), a.nq, base.data_ptr(), a.n, a.dim, a.k,
                         idx.data_ptr(), sc.data_ptr())
    torch.cuda.synchronize()
    print(last_timings())


if __name__ == "__main__":
    main()
