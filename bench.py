"""Benchmark: IVF-PQ search QPS at matched recall@10, 10k-query batch (B200).

(`--workload flat` measures the exact flat top-k instead: 1M x 768 unit vectors, inner
product, k = 100, 10k queries; see main_flat.)

Workload (the IVF-PQ configuration with a 10k-query batch): N = 10,000,000 base vectors,
d = 768 fp32, from a seeded mixture of 50,000 anisotropic Gaussians (centres ~U[-1,1],
per-centre per-dim sigma ~U[0.01, 0.2]); OPQ rotation 768x768; nlist = 16,384;
m = 96 sub-quantizers x 8 bits; 10,000 queries from the same mixture; k = 10, L2;
nprobe 32 for the headline step, {8, 32, 128} in the sweep.

A step is one search of the 10k-query batch at nprobe = 32 through
vesper_ivfpq_search_batch_device (inputs resident in HBM).  `e2e` is the same
search through vesper_ivfpq_search_batch with host buffers (the reference's C call).
The index is trained (k-means++ -> k-means, OPQ, PQ) and filled on the GPU by this
library before timing; the training set is the first N_TRAIN base vectors.

--impl reference times the reference's own CPU search (oracle/_ref/libvesper_ref.so,
the reference IVF-PQ sources compiled with their own flags) on the host cores, on a
bounded sample of the same query batch, against the same index (built on the GPU by
this library and handed over through the reference's v1.0 file format, which the
reference's IvfPqIndex::load reads).

Multi-GPU (torchrun, one rank per GPU): the base set is sharded by vector (rank r
holds base chunks r, r+W, ...); every rank trains the same model on the same training
sample; each rank probes 1/W of the query batch (the coarse stage is identical on every
shard) and the probe lists are all-gathered over NCCL; every rank then searches all
queries over its shard, and the per-rank top-k are merged with an NCCL all_gather.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import shutil
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from vesper_db_b200 import synth  # noqa: E402  (data generator; imports no CUDA code)

N_BASE = 10_000_000
DIM = 768
N_CENTRES = 50_000
NLIST = 16_384
QUERY_CHUNK = (512 << 20) // (4 * NLIST)  # queries per engine pass: 512 MiB of coarse distances
M = 96
NBITS = 8
NQ = 10_000
K = 10
NPROBE = 32
SWEEP = (8, 32, 128)
N_TRAIN = 131_072
CHUNK = 125_000           # base rows per generator chunk (80 chunks; divisible by 1/2/4/8)
SCAN_KERNELS = {1: "scan_exact_kernel", 2: "scan_fast2_kernel", 3: "scan_blocked_kernel",
                4: "tc_list_scan_kernel"}
COARSE_KERNELS = {1: "l2_dist_kernel (CUDA cores)", 2: "tc_screen_kernel (tcgen05 tf32) + screen_select_kernel"}
METRIC = "QPS at matched recall@10 (IVF-PQ, 10k-query batch) at 1/2/4/8 B200 vs CPU ref"
LIST_SCAN_BYTES_PER_PAIR = (662.9e6 + 8.7e6) / 6.65e9   # ncu, main-pass launch on the 4M-vector case
WORKLOAD = ("IVF-PQ+OPQ search: N=10,000,000 x d=768 fp32 (mixture of 50,000 anisotropic Gaussians, "
            "sigma~U[0.01,0.2]), nlist=16384, m=96x8 bits, OPQ 768x768, 10,000 queries, k=10, L2, nprobe=32")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--workload", default="ivfpq", choices=["ivfpq", "flat"],
                    help="ivfpq: the IVF-PQ+OPQ search (default); flat: exact flat top-k, 1M x 768 IP, k=100")
    return ap.parse_args()


# ------------------------------------------------------------------------------- data
def gen_centres(torch, dev):
    return synth.gen_centres(torch, dev, N_CENTRES, DIM)


def gen_rows(torch, dev, centres, sigmas, n, seed, out=None):
    return synth.gen_rows(torch, dev, centres, sigmas, n, seed, out)


def gen_base_chunk(torch, dev, centres, sigmas, c, out=None):
    return synth.gen_base_chunk(torch, dev, centres, sigmas, c, CHUNK, out)


# ------------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.path = tempfile.mktemp(suffix=".csv")
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = []
        try:
            for line in open(self.path):
                p = [x.strip() for x in line.split(",")]
                if len(p) >= 9 and p[1].replace(".", "").isdigit():
                    rows.append(p)
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = sorted(float(r[1]) for r in rows)
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for nm, v in zip(names, r[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": max(float(r[2]) for r in rows),
                "reasons": sorted(reasons), "samples": len(rows),
                "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


# ------------------------------------------------------------------------------- helpers
def measured_peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))), "measured"
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def exact_topk_gt(torch, q, base_chunks, k):
    """Exact fp32 top-k (squared L2) of q over the base chunks (evaluation only)."""
    torch.backends.cuda.matmul.allow_tf32 = False
    qn = (q * q).sum(1, keepdim=True)
    best_d = torch.full((q.shape[0], k), float("inf"), device=q.device)
    best_i = torch.zeros((q.shape[0], k), dtype=torch.int64, device=q.device)
    for (x, id0) in base_chunks:
        d = qn - 2.0 * (q @ x.T) + (x * x).sum(1)[None, :]
        dd, ii = torch.topk(d, k, dim=1, largest=False)
        cat_d = torch.cat([best_d, dd], 1)
        cat_i = torch.cat([best_i, ii + id0], 1)
        sel_d, sel = torch.topk(cat_d, k, dim=1, largest=False)
        best_d, best_i = sel_d, torch.gather(cat_i, 1, sel)
    return best_d, best_i


def recall_at(ids, gt_ids, k):
    hits = 0
    for a, b in zip(ids[:, :k].tolist(), gt_ids[:, :k].tolist()):
        hits += len(set(a) & set(b))
    return hits / (ids.shape[0] * k)


def reference_cpu_search(index_dir, queries_np, nprobe, seconds):
    """Time the reference's own IvfPqIndex::search_batch (OpenMP over all host cores)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from oracle_lib import REF_SO, Reference
    ref = Reference(REF_SO)
    idx = ref.ivfpq()
    t0 = time.perf_counter()
    idx.load(index_dir)
    load_s = time.perf_counter() - t0
    idx.search(queries_np[:64], K, nprobe)  # warm-up
    done, elapsed, batch = 0, 0.0, 256
    ids_all = []
    while done < queries_np.shape[0] and elapsed < seconds:
        qb = queries_np[done:done + batch]
        t = time.perf_counter()
        ids, _, _ = idx.search(qb, K, nprobe)
        elapsed += time.perf_counter() - t
        ids_all.append(ids)
        done += qb.shape[0]
    import numpy as np
    return {"qps": done / elapsed, "queries": done, "seconds": elapsed, "load_s": load_s,
            "ids": np.concatenate(ids_all), "cores": os.cpu_count()}


# ------------------------------------------------------------------------------- flat top-k
FLAT_N, FLAT_NQ, FLAT_K, FLAT_CHUNK = 1_000_000, 10_000, 100, 125_000
FLAT_FILTER_BYTES_PER_ROW = (929.28e6 + 39.77e6) / 300_000   # ncu, filter launch over a 300k-row base
FLAT_METRIC = "QPS, exact flat top-k (inner product, k=100), 10k-query batch"
FLAT_WORKLOAD = ("Exact brute-force k-NN (flat index): N=1,000,000 x d=768 fp32 ~N(0,1) then L2-normalised, "
                 "10,000 queries from the same distribution, inner product, k=100")


def flat_rows(torch, dev, n, seed, out=None):
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn((n, DIM), device=dev, generator=g, out=out)
    x /= x.norm(dim=1, keepdim=True)
    return x


def reference_flat(base_np, q_np, seconds, batch=8):
    """Time the reference's find_nearest_centroids_batch_fused (OpenMP over all host
    threads) on query batches until `seconds` of search have run; the base sits in the
    reference's AlignedCentroidBuffer (filled once, untimed)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from oracle_lib import REF_SO, Reference
    fb = Reference(REF_SO).flat_buffer(base_np)
    fb.topk(1, q_np[:2], FLAT_K)  # warm-up
    done, el, ids, scores = 0, 0.0, [], []
    while done < q_np.shape[0] and (el < seconds or done == 0):
        qb = q_np[done:done + batch]
        t = time.perf_counter()
        i, sc = fb.topk(1, qb, FLAT_K)
        el += time.perf_counter() - t
        ids.append(i)
        scores.append(sc)
        done += qb.shape[0]
    import numpy as np
    return done / el, done, el, np.concatenate(ids), np.concatenate(scores)


def main_flat(args):
    import numpy as np
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference" and rank != 0:
        return 0
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1 and args.impl == "ours":
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)
    shard_world = world if args.impl == "ours" else 1
    from vesper_db_b200.shard import chunks_of, merge_topk
    my_chunks = chunks_of(rank if args.impl == "ours" else 0, shard_world, FLAT_N // FLAT_CHUNK)
    n_local = len(my_chunks) * FLAT_CHUNK
    base = torch.empty((n_local, DIM), device=dev)
    for j, c in enumerate(my_chunks):
        flat_rows(torch, dev, FLAT_CHUNK, 7000 + c, out=base[j * FLAT_CHUNK:(j + 1) * FLAT_CHUNK])
    queries = flat_rows(torch, dev, FLAT_NQ, 6999)
    torch.cuda.synchronize()
    q_np = queries.cpu().numpy()
    peaks, peak_kind = measured_peaks()
    cfg = {"workload": FLAT_WORKLOAD, "n_base": FLAT_N, "nq": FLAT_NQ, "k": FLAT_K, "op": "inner_product",
           "parallelism": f"vector-sharded x{world}" if world > 1 else "single GPU",
           "l2_policy": "inputs larger than L2 (3.07 GB base streamed per pass)"}
    if args.impl == "reference":
        per = max(1.0, args.cpu_seconds / max(1, args.steps))
        base_np = base.cpu().numpy()
        vals, nq_done = [], 0
        for s in range(args.warmup + args.steps):
            v, n, el, _, _ = reference_flat(base_np, q_np[(s * 64) % FLAT_NQ:], per)
            if s >= args.warmup:
                vals.append(v)
                nq_done += n
        v = sorted(vals)[len(vals) // 2]
        print(json.dumps({"impl": "reference", "metric": FLAT_METRIC, "value": v, "unit": "queries/s",
                          "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                          "ms_per_step": 1e3 * FLAT_NQ / v, "higher_is_better": True, "scaling": "strong",
                          "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1), normalised)",
                          "config": cfg,
                          "cpu_baseline": {"value": v, "unit": "queries/s", "cores": os.cpu_count(),
                                           "kind": "reference",
                                           "sample": f"{nq_done} queries over {args.steps} steps (~{per:.0f} s "
                                                     f"each), OpenMP over all host threads"},
                          "e2e": {"value": v, "unit": "queries/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}))
        return 0

    from vesper_db_b200 import flat_topk_device
    from vesper_db_b200.flat import last_timings
    import ctypes as C
    from vesper_db_b200 import _native as N
    out_i = torch.empty((FLAT_NQ, FLAT_K), dtype=torch.int32, device=dev)
    out_s = torch.empty((FLAT_NQ, FLAT_K), dtype=torch.float32, device=dev)
    chunk0 = torch.tensor([my_chunks[j] * FLAT_CHUNK for j in range(len(my_chunks))], device=dev)

    def one_step():
        flat_topk_device(1, queries.data_ptr(), FLAT_NQ, base.data_ptr(), n_local, DIM, FLAT_K, out_i.data_ptr(),
                         out_s.data_ptr())
        if world > 1:
            # local row -> global id, then the merge (scores negated: merge_topk keeps smallest)
            loc = out_i.long()
            gid = chunk0[loc // FLAT_CHUNK] + loc % FLAT_CHUNK
            d, i = merge_topk(-out_s, gid, FLAT_K)
            return -d, i
        return out_s, out_i.long()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        one_step()
    barrier()
    filt, stages, launches = [], [], 0
    with ClockSampler(local) as clk:
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        ev0.record()
        for _ in range(args.steps):
            res_s, res_i = one_step()
            t = last_timings()
            filt.append(t["filter_ms"])
            stages.append(t)
            launches += t["kernel_launches"]
        ev1.record()
        barrier()
    ms_total = ev0.elapsed_time(ev1)
    if world > 1:
        tt = torch.tensor([ms_total], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms_total = float(tt.item())
    qps = FLAT_NQ * args.steps / (ms_total / 1e3)

    # e2e: vesper_flat_topk with host buffers (queries and base copied in, results out)
    lib = N.load()
    base_h = torch.empty((n_local, DIM), dtype=torch.float32, pin_memory=True)
    base_h.copy_(base)
    q_h = torch.empty((FLAT_NQ, DIM), dtype=torch.float32, pin_memory=True)
    q_h.copy_(queries)
    i_h = torch.empty((FLAT_NQ, FLAT_K), dtype=torch.int32, pin_memory=True)
    s_h = torch.empty((FLAT_NQ, FLAT_K), dtype=torch.float32, pin_memory=True)
    f32p, u32p = C.POINTER(C.c_float), C.POINTER(C.c_uint32)
    e2e = []
    for s in range(args.warmup + args.steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        e0.record()
        st = lib.vesper_flat_topk(1, C.cast(q_h.data_ptr(), f32p), FLAT_NQ, C.cast(base_h.data_ptr(), f32p),
                                  n_local, DIM, FLAT_K, C.cast(i_h.data_ptr(), u32p), C.cast(s_h.data_ptr(), f32p))
        if st != 0:
            raise RuntimeError(lib.vesper_get_last_error().decode())
        e1.record()
        barrier()
        if s >= args.warmup:
            e2e.append(e0.elapsed_time(e1))
    e2e_ms = sum(e2e) / len(e2e)
    if world > 1:
        tt = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_ms = float(tt.item())

    fk = sum(filt) / len(filt)
    flop_launches = 2.0 * n_local * DIM * FLAT_NQ
    achieved = flop_launches / (fk / 1e3) / 1e12
    tf32_peak = peaks["bf16_tflops"] / 2.0
    avg = {k2: sum(t[k2] for t in stages) / len(stages) for k2 in stages[0] if k2.endswith("_ms")}
    out = {
        "metric": FLAT_METRIC, "value": qps, "unit": "queries/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_total / args.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1), L2-normalised, generated on device)",
        "config": cfg,
        "e2e": {"value": FLAT_NQ / (e2e_ms / 1e3), "unit": "queries/s",
                "h2d_bytes_per_step": (n_local + FLAT_NQ) * DIM * 4, "d2h_bytes_per_step": FLAT_NQ * FLAT_K * 8,
                "ms_per_step": e2e_ms},
        "gpu_launches": launches,
        "roofline": {"bound": "tensor", "kernel": "tc_screen_kernel filter mode (tcgen05 kind::tf32)",
                     "achieved": achieved, "peak": tf32_peak, "unit": "TFLOP/s", "frac": achieved / tf32_peak,
                     "peak_source": f"{peak_kind} bf16 dense burst / 2 (tf32 dense rate)",
                     # DRAM bytes of one filter launch, from the ncu capture in
                     # profiles/tc_screen_kernel_filter_300kx768_nq2048.md (969 MB for a 300,000-row
                     # base), scaled by base rows: the base is streamed once per launch.
                     "traffic": FLAT_FILTER_BYTES_PER_ROW * n_local,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, 300k-row case, "
                                       "scaled by base rows (one level-0 filter launch per step)",
                     "algorithmic_flop_per_step": flop_launches, "kernel_ms_per_step": fk},
        "stage_ms": avg,
        "candidates_per_query": stages[-1]["candidates"] / FLAT_NQ,
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            base_np = base.cpu().numpy()
            v, n, el, rid, rsc = reference_flat(base_np, q_np, args.cpu_seconds)
            gi = res_i[:n].cpu().numpy().astype(np.uint32)
            gs = res_s[:n].cpu().numpy()
            out["cpu_baseline"] = {"value": v, "unit": "queries/s", "cores": os.cpu_count(), "kind": "reference",
                                   "sample": f"first {n} queries of the batch ({el:.1f} s of search), "
                                             f"find_nearest_centroids_batch_fused, OpenMP over all host threads"}
            out["parity_vs_reference"] = {"queries": int(n), "indices_equal": bool(np.array_equal(gi, rid)),
                                          "scores_equal": bool(np.array_equal(gs, rsc))}
        except Exception as e:
            out["cpu_baseline"] = {"value": None, "unit": "queries/s", "cores": os.cpu_count(),
                                   "kind": "reference", "sample": f"unavailable: {e}"}
    if rank == 0:
        print(json.dumps(out))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# ------------------------------------------------------------------------------- main
def main():
    args = parse()
    if args.workload == "flat":
        return main_flat(args)
    import numpy as np
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference" and rank != 0:
        return 0
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1 and args.impl == "ours":
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)

    from vesper_db_b200 import IvfPqIndex
    from vesper_db_b200.shard import chunks_of, merge_topk, probed_search
    t_build0 = time.perf_counter()
    centres, sigmas = gen_centres(torch, dev)
    queries = synth.gen_queries(torch, dev, centres, sigmas, NQ)
    n_chunks = N_BASE // CHUNK
    shard_world = world if args.impl == "ours" else 1
    my_chunks = chunks_of(rank if args.impl == "ours" else 0, shard_world, n_chunks)
    n_local = len(my_chunks) * CHUNK
    base = torch.empty((n_local, DIM), device=dev)
    ids = torch.empty(n_local, dtype=torch.int64, device=dev)
    for j, c in enumerate(my_chunks):
        gen_base_chunk(torch, dev, centres, sigmas, c, out=base[j * CHUNK:(j + 1) * CHUNK])
        ids[j * CHUNK:(j + 1) * CHUNK] = torch.arange(c * CHUNK, (c + 1) * CHUNK, device=dev)
    # Training sample: the first N_TRAIN base vectors (chunks 0, 1, ...), identical on every rank.
    train_x = torch.cat([gen_base_chunk(torch, dev, centres, sigmas, c)
                         for c in range(math.ceil(N_TRAIN / CHUNK))])[:N_TRAIN].contiguous()
    del centres, sigmas
    torch.cuda.synchronize()
    t_data = time.perf_counter() - t_build0

    index = IvfPqIndex()
    t0 = time.perf_counter()
    rep = index.train_device(train_x.data_ptr(), N_TRAIN, DIM, NLIST, M, NBITS, use_opq=True)
    t_train = time.perf_counter() - t0
    del train_x
    t0 = time.perf_counter()
    index.add_device(ids.data_ptr(), base.data_ptr(), n_local)
    t_add = time.perf_counter() - t0

    # Ground truth for recall@10 (exact fp32 over every shard, merged across ranks).
    chunks = [(base[j * CHUNK:(j + 1) * CHUNK], my_chunks[j] * CHUNK) for j in range(len(my_chunks))]
    gt_d, gt_i = exact_topk_gt(torch, queries, chunks, K)
    if world > 1 and args.impl == "ours":
        gt_d, gt_i = merge_topk(gt_d, gt_i, K)
    del base, chunks
    torch.cuda.synchronize()
    gt_np = gt_i.cpu().numpy()
    q_np = queries.cpu().numpy()

    if args.impl == "reference":
        out = {"impl": "reference", "metric": METRIC, "unit": "queries/s", "higher_is_better": True,
               "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "scaling": "strong",
               "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded mixture)",
               "config": {"workload": WORKLOAD, "nprobe": NPROBE, "k": K, "nq": NQ, "n_train": N_TRAIN}}
        tmp = tempfile.mkdtemp(prefix="vesper_ref_")
        try:
            index.save(tmp)
            index.close()
            sys.path.insert(0, os.path.join(ROOT, "oracle"))
            from oracle_lib import REF_SO, Reference
            ridx = Reference(REF_SO).ivfpq()
            t0 = time.perf_counter()
            ridx.load(tmp)
            load_s = time.perf_counter() - t0
            # Each step searches a disjoint 128-query slice block for ~cpu_seconds/steps.
            per = max(1.0, args.cpu_seconds / max(1, args.steps))
            step_qps, hits, nq_done, qpos = [], 0, 0, 0
            for s in range(args.warmup + args.steps):
                done, el = 0, 0.0
                while (el < per or done == 0) and done < NQ:
                    lo = qpos % NQ
                    qb = q_np[lo:lo + 128]
                    t = time.perf_counter()
                    rid, _, _ = ridx.search(qb, K, NPROBE)
                    el += time.perf_counter() - t
                    if s >= args.warmup:
                        g = gt_np[lo:lo + qb.shape[0]]
                        hits += sum(len(set(a) & set(b)) for a, b in zip(rid.tolist(), g.tolist()))
                        nq_done += qb.shape[0]
                    done += qb.shape[0]
                    qpos += qb.shape[0]
                if s >= args.warmup:
                    step_qps.append(done / el)
            v = sorted(step_qps)[len(step_qps) // 2]
            out.update({"value": v, "ms_per_step": 1e3 * NQ / v,
                        "recall@10": hits / max(1, nq_done * K),
                        "cpu_baseline": {"value": v, "unit": "queries/s", "cores": os.cpu_count(),
                                         "kind": "reference",
                                         "sample": f"{nq_done} queries of the 10k batch over {args.steps} steps "
                                                   f"(~{per:.0f} s each), nprobe={NPROBE}, k={K}, OpenMP over all "
                                                   f"host threads; index load {load_s:.1f} s untimed"},
                        "e2e": {"value": v, "unit": "queries/s", "h2d_bytes_per_step": 0,
                                "d2h_bytes_per_step": 0},
                        "build": {"data_s": t_data, "train_s": t_train, "add_s": t_add}})
        finally:
            shutil.rmtree(tmp, ignore_errors=True)
        print(json.dumps(out))
        return 0

    # ------------------------------------------------------------------ our arm
    out_ids = torch.empty((NQ, K), dtype=torch.int64, device=dev)
    out_d = torch.empty((NQ, K), dtype=torch.float32, device=dev)
    out_n = torch.empty(NQ, dtype=torch.int32, device=dev)

    slot = torch.arange(K, device=dev)[None, :]

    # Multi-GPU: each rank probes 1/world of the batch (the coarse stage is the same on
    # every shard) and the probe lists are all-gathered before the shard searches.
    probe_bufs = {}

    def one_search(nprobe):
        if world > 1 and NQ % world == 0:
            probed_search(index, queries, K, nprobe, NLIST, out_ids, out_d, out_n, probe_bufs)
        else:
            index.search_batch_device(queries.data_ptr(), NQ, K, nprobe, out_ids.data_ptr(), out_d.data_ptr(),
                                      out_n.data_ptr())
        if world > 1:
            # padded slots (fewer than k results on this shard) must not win the merge
            d = torch.where(slot < out_n[:, None], out_d, torch.full_like(out_d, float("inf")))
            return merge_topk(d, out_ids, K)
        return out_d, out_ids

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        one_search(NPROBE)
    barrier()
    scan_ms, scanned, list_ms, launches = [], [], [], 0
    with ClockSampler(local) as clk:
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.nvtx.range_push("timed_search")
        ev0.record()
        for _ in range(args.steps):
            res_d, res_i = one_search(NPROBE)
            t = index.last_timings()
            scan_ms.append(t["scan_ms"])
            scanned.append(t["scanned_entries"])
            list_ms.append(t["list_kernel_ms"])
            launches += t["kernel_launches"]
        ev1.record()
        torch.cuda.nvtx.range_pop()
        barrier()
    ms_total = ev0.elapsed_time(ev1)
    if world > 1:
        tt = torch.tensor([ms_total], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms_total = float(tt.item())
    ms_step = ms_total / args.steps
    qps = NQ * args.steps / (ms_total / 1e3)
    timings = index.last_timings()
    recall = recall_at(res_i.cpu().numpy(), gt_np, K)

    # nprobe sweep (one timed pass each) with recall
    sweep = []
    for npb in SWEEP:
        one_search(npb)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        rd, ri = one_search(npb)
        e1.record()
        barrier()
        sweep.append({"nprobe": npb, "qps": NQ / (e0.elapsed_time(e1) / 1e3),
                      "recall@10": recall_at(ri.cpu().numpy(), gt_np, K)})

    # e2e: the reference's C call with host buffers (H2D of queries, D2H of results inside)
    q_host = torch.empty((NQ, DIM), dtype=torch.float32, pin_memory=True)
    q_host.copy_(queries)
    q_host_np = q_host.numpy()
    e2e_ms = []
    for s in range(args.warmup + args.steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        e0.record()
        if world == 1:
            index.search_batch_c(q_host_np, K, NPROBE)
        else:
            # per-shard search through the C ABI with host buffers (counts mark the
            # padding), then the merge across ranks and the merged result to the host
            hid, hd, hcnt = index.search_batch(q_host_np, K, NPROBE)
            hd = np.where(np.arange(K)[None, :] < hcnt[:, None], hd, np.inf).astype(np.float32)
            md, mi = merge_topk(torch.from_numpy(hd).to(dev), torch.from_numpy(hid.astype(np.int64)).to(dev), K)
            mi.cpu()
        e1.record()
        barrier()
        if s >= args.warmup:
            e2e_ms.append(e0.elapsed_time(e1))
    e2e_step = sum(e2e_ms) / len(e2e_ms)
    if world > 1:
        tt = torch.tensor([e2e_step], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_step = float(tt.item())

    peaks, peak_kind = measured_peaks()
    scan_avg = sum(scan_ms) / len(scan_ms)
    entries = sum(scanned) / len(scanned)
    code_bytes = entries * M
    if timings["scan_variant"] == 4:
        # Dominant kernel: the tcgen05 screen.  Algorithmic work = every (query, probed
        # entry) pair's dim-long product, 2 * dim FLOP each; one launch per query chunk.
        lk = sum(list_ms) / len(list_ms)
        flop = 2.0 * DIM * entries
        achieved = flop / (lk / 1e3) / 1e12
        roofline = {"bound": "tensor", "kernel": "tc_list_scan_kernel (tcgen05 kind::f16, bf16, A in TMEM)",
                    "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                    "frac": achieved / peaks["bf16_tflops"], "peak_source": f"{peak_kind} (bf16 dense, burst)",
                    # DRAM bytes per launch: profiles/tc_list_scan_kernel_4Mx768_nq8192.md measured
                    # 671.6 MB for 6.65e9 (query, entry) pairs on the 4M-vector case; scaled by the
                    # pairs of one launch here (codes of each probed tile are read once per batch).
                    "traffic": LIST_SCAN_BYTES_PER_PAIR * entries / -(-NQ // QUERY_CHUNK),
                    "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, 4M-vector case, "
                                      "scaled by (query, entry) pairs per launch",
                    "algorithmic_flop_per_search": flop, "kernel_ms_per_search": lk,
                    "launches_per_search": -(-NQ // QUERY_CHUNK),
                    "scan_stage_ms": scan_avg,
                    "scan_stage_code_GBps": code_bytes / (scan_avg / 1e3) / 1e9,
                    "candidates_refined": timings["list_candidates"],
                    "fallback_queries": timings["list_fallback_queries"]}
    else:
        achieved = code_bytes / (scan_avg / 1e3) / 1e9
        roofline = {"bound": "hbm", "kernel": SCAN_KERNELS.get(timings["scan_variant"], "?"), "achieved": achieved,
                    "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                    "peak_source": peak_kind, "traffic": None,
                    "algorithmic_bytes_per_search": code_bytes, "scan_ms": scan_avg}
    out = {
        "metric": METRIC, "value": qps, "unit": "queries/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded mixture generated on device)",
        "config": {"workload": WORKLOAD, "nlist": NLIST, "m": M, "nbits": NBITS, "nprobe": NPROBE, "k": K,
                   "nq": NQ, "n_base": N_BASE, "n_train": N_TRAIN, "search_mode": "fast",
                   "parallelism": f"vector-sharded x{world}" if world > 1 else "single GPU",
                   "l2_policy": "inputs larger than L2 (960 MB of PQ codes scanned per pass)"},
        "recall@10": recall,
        "sweep": sweep,
        "e2e": {"value": NQ / (e2e_step / 1e3), "unit": "queries/s", "h2d_bytes_per_step": NQ * DIM * 4,
                "d2h_bytes_per_step": NQ * K * 12, "ms_per_step": e2e_step},
        "gpu_launches": launches,
        "roofline": roofline,
        "stage_ms": {k2: v for k2, v in timings.items() if k2.endswith("_ms")},
        "coarse_kernel": COARSE_KERNELS.get(timings["coarse_variant"], "?"),
        "build": {"data_s": t_data, "train_s": t_train, "add_s": t_add, "opq_kept": rep.opq_kept,
                  "err_unrot": rep.err_unrot, "err_opq": rep.err_opq},
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tmp = tempfile.mkdtemp(prefix="vesper_cpu_")
        try:
            index.save(tmp)
            r = reference_cpu_search(tmp, q_np, NPROBE, args.cpu_seconds)
            out["cpu_baseline"] = {"value": r["qps"], "unit": "queries/s", "cores": r["cores"], "kind": "reference",
                                   "sample": f"first {r['queries']} queries of the 10k batch, nprobe={NPROBE}, "
                                             f"k={K} ({r['seconds']:.1f} s of search)",
                                   "recall@10": recall_at(r["ids"], gt_np[:r["queries"]], K)}
        except Exception as e:  # the reference oracle may be absent on a machine without it
            out["cpu_baseline"] = {"value": None, "unit": "queries/s", "cores": os.cpu_count(),
                                   "kind": "reference", "sample": f"unavailable: {e}"}
        finally:
            shutil.rmtree(tmp, ignore_errors=True)
    if rank == 0:
        print(json.dumps(out))
    index.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
