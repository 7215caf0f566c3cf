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
library before timing; the training set is the first N_TRAIN = 200,000 base vectors
(the reference IndexManager's subsample size).  The bench line states the shape of the
lists (`config.list_stats`: sizes, skew, entries probed per query).

One GPU, rank 0: the cpu_baseline leg runs the reference's search_batch on 256 queries
strided across the batch at nprobe 8/32/128; `recall_matched` gives its recall@10 beside
the GPU's on exactly those queries, and `parity_vs_reference` compares the GPU's ids and
distances with the reference's (ids equal outside 1e-4 ties, distance error).

--impl reference times the reference's own CPU search (oracle/_ref/libvesper_ref.so,
the reference IVF-PQ sources compiled with their own flags) on every host CPU (OpenMP
thread count set explicitly: torchrun exports OMP_NUM_THREADS=1), one query slice per
step, against the same index (built on the GPU by this library and handed over through
the reference's v1.0 file format, which the reference's IvfPqIndex::load reads).

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
SEARCH_QUERY_CHUNK = (1 << 30) // (4 * NLIST)  # queries per engine pass: 1 GiB of coarse distances
M = 96
NBITS = 8
NQ = 10_000
K = 10
NPROBE = 32
SWEEP = (8, 32, 128)
SWEEP_PASSES = 5
# Training sample: min(n, 200,000), the subsample the reference's IndexManager trains its
# IVF-PQ index on (src/index/index_manager.cpp:1712).
N_TRAIN = 200_000
CPU_SAMPLE = 256          # queries the reference searches per nprobe in the cpu_baseline leg
CHUNK = 125_000           # base rows per generator chunk (80 chunks; divisible by 1/2/4/8)
SCAN_KERNELS = {1: "scan_exact_kernel", 2: "scan_fast2_kernel", 3: "scan_blocked_kernel",
                4: "tc_list_scan_kernel"}
COARSE_KERNELS = {1: "l2_dist_kernel (CUDA cores)", 2: "tc_screen_kernel (tcgen05 tf32) + screen_select_kernel",
                  3: "sampled threshold + tc_screen_kernel filter (tcgen05 tf32) + flat_refine_kernel"}
METRIC = "QPS at matched recall@10 (IVF-PQ, 10k-query batch) at 1/2/4/8 B200 vs CPU ref"
LIST_SCAN_BYTES_PER_PAIR = (556.5e6 + 10.6e6) / 2.209e9   # ncu, main-pass launch on the 2M-vector case


def workload_name():
    return (f"IVF-PQ+OPQ search: N={N_BASE:,} x d=768 fp32 (mixture of 50,000 anisotropic Gaussians, "
            f"sigma~U[0.01,0.2]), nlist=16384, m=96x8 bits, OPQ 768x768, {NQ:,} queries, k=10, L2, nprobe=32")


WORKLOAD = workload_name()


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--workload", default="ivfpq", choices=["ivfpq", "flat", "kmeans", "c5"],
                    help="ivfpq: the IVF-PQ+OPQ search (default); flat: exact flat top-k, 1M x 768 IP, k=100; "
                         "kmeans: Lloyd iterations, 2M x 128 points, k=16,384; c5: sharded IVF-PQ search, "
                         "100M x 128, nlist 65,536, m 32, 100k queries, nprobe 64, k 100")
    # Smaller cases of the same workload, for profiler captures (the defaults are the
    # benchmark's sizes; a line measured with either flag names its sizes in config).
    ap.add_argument("--n-base", type=int, default=0,
                    help="base vectors (multiple of the generated chunk: 125,000 rows, c5 6,250,000); "
                         "k-means: points")
    ap.add_argument("--nq", type=int, default=0, help="queries in the batch")
    ap.add_argument("--no-tau-exchange", action="store_true",
                    help="several GPUs: each shard keeps its own k-th-distance bounds (no threshold exchange)")
    ap.add_argument("--scan", default="auto", choices=["auto", "tc", "blocked"],
                    help="FAST scan kernel: the engine's choice, the tensor-core list scan or the blocked scan")
    args = ap.parse_args()
    global N_BASE, NQ, WORKLOAD, FLAT_N, FLAT_NQ, KM_N, C5_N, C5_NQ
    if args.workload == "kmeans":
        KM_N = args.n_base or KM_N
    elif args.workload == "c5":
        C5_N = max(C5_CHUNK, args.n_base // C5_CHUNK * C5_CHUNK) if args.n_base else C5_N
        C5_NQ = args.nq or C5_NQ
    elif args.workload == "flat":
        FLAT_N = max(FLAT_CHUNK, args.n_base // FLAT_CHUNK * FLAT_CHUNK) if args.n_base else FLAT_N
        FLAT_NQ = args.nq or FLAT_NQ
    else:
        if args.n_base:
            N_BASE = max(CHUNK, args.n_base // CHUNK * CHUNK)
        NQ = args.nq or NQ
        WORKLOAD = workload_name()
    if args.scan != "auto":
        os.environ["VGPU_SCAN"] = args.scan
    return args


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

    def _lines(self):
        try:
            return [ln for ln in open(self.path) if ln.strip()]
        except OSError:
            return []

    def __enter__(self):
        self.skip = 0
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return self
        # nvidia-smi takes a moment to start: wait (bounded) for its first line so that
        # the sampling runs through the timed region, which starts after this returns
        t_end = time.time() + 5.0
        while time.time() < t_end and not self._lines():
            time.sleep(0.02)
        self.skip = len(self._lines())
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            # a region shorter than the sampling period: take the next sample, right
            # after it (the clocks have not moved yet)
            t_end = time.time() + 0.5
            while time.time() < t_end and len(self._lines()) <= self.skip:
                time.sleep(0.02)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        """The samples taken from the region's start to just after its end."""
        lines = self._lines()
        region = lines[self.skip:] or lines[-1:]
        rows = []
        for line in region:
            p = [x.strip() for x in line.split(",")]
            if len(p) >= 9 and p[1].replace(".", "").isdigit():
                rows.append(p)
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


def _oracle_lib():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle_lib
    return oracle_lib


def reference_threads():
    """Use every host CPU this process may run on for the reference's OpenMP regions
    (torchrun exports OMP_NUM_THREADS=1 to each rank) and describe the host."""
    ol = _oracle_lib()
    used = ol.set_omp_threads(ol.host_threads())
    return used, ol.host_cpu()


def topk_parity(ids, d, cnt, rids, rd, rcnt, rtol=1e-4):
    """Compare two top-k results query by query: distances within rtol (relative, floor
    1) position by position; an id that only one side returns must tie the reference's
    k-th distance within that band.  Returns counts, not assertions."""
    import numpy as np
    nq = ids.shape[0]
    bad_ids, bad_cnt, max_rel = 0, 0, 0.0
    for q in range(nq):
        n = int(rcnt[q])
        if int(cnt[q]) != n:
            bad_cnt += 1
            continue
        if n == 0:
            continue
        a, b = d[q, :n].astype(np.float64), rd[q, :n].astype(np.float64)
        max_rel = max(max_rel, float((np.abs(a - b) / np.maximum(1.0, np.abs(b))).max()))
        kth = b[n - 1]
        band = rtol * max(1.0, abs(kth))
        ia, ib = [int(i) for i in ids[q, :n]], [int(i) for i in rids[q, :n]]
        sa, sb = set(ia), set(ib)
        # an id only one side returns must tie the k-th distance within the band
        if any(i not in sb and abs(x - kth) > band for i, x in zip(ia, a)) or \
                any(i not in sa and abs(x - kth) > band for i, x in zip(ib, b)):
            bad_ids += 1
    return {"queries": int(nq), "count_mismatches": bad_cnt, "id_mismatches_outside_ties": bad_ids,
            "max_rel_dist_err": max_rel, "rtol": rtol}


def list_stats(index, n_queries, scanned_entries):
    """Shape of the inverted lists this rank holds and of the probe work per query."""
    import numpy as np
    sizes = np.diff(index.list_offsets().astype(np.int64))
    nz = sizes[sizes > 0]
    return {"lists": int(sizes.size), "entries": int(sizes.sum()), "mean": float(sizes.mean()),
            "max": int(sizes.max()), "p50": float(np.percentile(sizes, 50)), "p99": float(np.percentile(sizes, 99)),
            "empty": int((sizes == 0).sum()), "max_over_mean": float(sizes.max() / max(sizes.mean(), 1e-9)),
            "nonempty_min": int(nz.min()) if nz.size else 0,
            "probed_entries_per_query": float(scanned_entries) / max(1, n_queries)}


def list_scan_tiles(index, probe_np, tile=128, qchunk=128):
    """Work the tensor-core list scan does for one batch: it pairs each probed list's
    128-entry tiles with 128-query chunks of the queries that probe it, so partial tiles
    and partial chunks are padded.  Returns the (query, entry) pairs of the batch and the
    pairs its MMAs compute."""
    import numpy as np
    sizes = np.diff(index.list_offsets().astype(np.int64))
    q_per_list = np.bincount(probe_np.reshape(-1).astype(np.int64), minlength=sizes.size)
    pairs = float((sizes * q_per_list).sum())
    padded = float(((-(-sizes // tile)) * tile * (-(-q_per_list // qchunk)) * qchunk).sum())
    hot = q_per_list > 0
    return {"pairs": pairs, "mma_pairs": padded, "mma_over_pairs": padded / max(pairs, 1.0),
            "queries_per_probed_list_mean": float(q_per_list[hot].mean()) if hot.any() else 0.0,
            "pairs_in_chunks_under_half_full": float((sizes * q_per_list)[(q_per_list % qchunk > 0) &
                                                                         (q_per_list % qchunk < qchunk // 2)].sum())
            / max(pairs, 1.0)}


# ------------------------------------------------------------------------------- flat top-k
FLAT_N, FLAT_NQ, FLAT_K, FLAT_CHUNK = 1_000_000, 10_000, 100, 125_000
FLAT_FILTER_BYTES_PER_ROW = (839.23e6 + 36.71e6) / 250_000   # ncu, filter launch over a 250k-row base
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
    reference_threads()
    ol = _oracle_lib()
    fb = ol.Reference(ol.REF_SO).flat_buffer(base_np)
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
    workload = FLAT_WORKLOAD.replace("N=1,000,000", f"N={FLAT_N:,}").replace("10,000 queries", f"{FLAT_NQ:,} queries")
    cfg = {"workload": workload, "n_base": FLAT_N, "nq": FLAT_NQ, "k": FLAT_K, "op": "inner_product",
           "parallelism": f"vector-sharded x{world}" if world > 1 else "single GPU",
           "l2_policy": "inputs larger than L2 (3.07 GB base streamed per pass)"}
    if args.impl == "reference":
        per = max(1.0, args.cpu_seconds / max(1, args.steps))
        base_np = base.cpu().numpy()
        els, nq_done = [], 0
        for s in range(args.warmup + args.steps):
            v, n, el, _, _ = reference_flat(base_np, q_np[(s * 64) % FLAT_NQ:], per)
            if s >= args.warmup:
                els.append(el)
                nq_done += n
        v = nq_done / sum(els)
        print(json.dumps({"impl": "reference", "metric": FLAT_METRIC, "value": v, "unit": "queries/s",
                          "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                          "ms_per_step": 1e3 * sum(els) / len(els), "higher_is_better": True, "scaling": "strong",
                          "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1), normalised)",
                          "config": cfg,
                          "cpu_baseline": {"value": v, "unit": "queries/s", "cores": reference_threads()[0],
                                           "host_cpu": reference_threads()[1], "kind": "reference",
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
                     # DRAM bytes of one filter launch, from an ncu capture of the filter
                     # over a smaller base, scaled by base rows: the base is streamed once
                     # per launch.
                     "traffic": FLAT_FILTER_BYTES_PER_ROW * n_local,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, 250k-row case, "
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
            threads, cpu = reference_threads()
            out["cpu_baseline"] = {"value": v, "unit": "queries/s", "cores": threads, "kind": "reference",
                                   "host_cpu": cpu,
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


# ------------------------------------------------------------------------------- k-means training
KM_N, KM_DIM, KM_K, KM_CENTRES, KM_SIGMA, KM_ITERS = 2_000_000, 128, 16_384, 20_000, 0.05, 20
KM_SEED = 42
KM_PARITY_N, KM_PARITY_K = 200_000, 2_048     # the scaled run checked against the reference
KM_CPU_SAMPLE = 100_000                        # points of the reference's timed Lloyd iteration
KM_METRIC = "k-means Lloyd iterations/s (2,000,000 x 128 points, k=16,384)"
KM_WORKLOAD = ("k-means training for the coarse quantizer: 2,000,000 x 128 fp32 from a seeded mixture of "
               "20,000 isotropic Gaussians (sigma 0.05, centres ~U[-1,1]), k=16,384, Lloyd iterations from "
               "k-means++ (seed 42)")


def kmeans_launches_per_iteration():
    """This library's kernels in one Lloyd iteration: the E-step's point norms, centroid
    norms, their square roots, the column maxima and the fused tcgen05 arg-min; the
    M-step's iota, segment boundaries, segmented sums and means (the grouping sort
    between them is CUB's).  Rows left by a candidate-list overflow would add the filter
    path's launches; none are expected on this data."""
    return 5 + 4


def main_kmeans(args):
    """One step = one Lloyd iteration over the 2M points (src/index/kmeans.cpp:137-252):
    E-step (tcgen05 tf32 screen + exact arg-min in the reference's lane order, lowest
    index wins a tie), the convergence test's inertia (per-point minima summed in fp64
    in point order on the host, as the engine's fit does), and the M-step (points
    grouped by cluster, fp64 sums in point order / count).  The centroids come from the
    library's k-means++ (the reference's draws); the whole 20-iteration fit through
    vesper_kmeans_fit_device is timed once beside it."""
    import numpy as np
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if rank != 0:
        return 0   # k-means training runs on one GPU here (its sharded form is tested, not benched)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from vesper_db_b200 import _native as N
    from vesper_db_b200.kmeans import kmeans_fit_device
    from vesper_db_b200.shard import GpuKmeansOps
    x = synth.gen_isotropic_mixture(torch, dev, KM_CENTRES, KM_DIM, KM_SIGMA, KM_N, 4242)
    torch.cuda.synchronize()
    cfg = {"workload": KM_WORKLOAD.replace("2,000,000", f"{KM_N:,}"), "n": KM_N, "dim": KM_DIM, "k": KM_K,
           "algorithm": "lloyd",
           "parallelism": "single GPU", "l2_policy": "inputs larger than L2 (1.02 GB of points per iteration)"}
    out_common = {"unit": "iterations/s", "higher_is_better": True, "n_gpus": 1, "steps": args.steps,
                  "warmup": args.warmup, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
                  "data": "synthetic (seeded isotropic mixture generated on device)", "config": cfg}
    if args.impl == "reference":
        threads, cpu = reference_threads()
        ol = _oracle_lib()
        ref = ol.Reference(ol.REF_SO)
        xs = x[:KM_CPU_SAMPLE].cpu().numpy()
        c0 = x[torch.randperm(KM_N, device=dev, generator=torch.Generator(device=dev).manual_seed(7))[:KM_K]]
        c0 = c0.cpu().numpy()
        step_s = []
        for s in range(args.warmup + args.steps):
            t = time.perf_counter()
            a, _ = ref.kmeans_assign(xs, c0)
            ref.kmeans_update(xs, a, c0)
            el = time.perf_counter() - t
            if s >= args.warmup:
                step_s.append(el * KM_N / KM_CPU_SAMPLE)
        v = len(step_s) / sum(step_s)
        print(json.dumps({"impl": "reference", "metric": KM_METRIC, "value": v, **out_common,
                          "ms_per_step": 1e3 * sum(step_s) / len(step_s) * KM_CPU_SAMPLE / KM_N,
                          "cpu_baseline": {"value": v, "unit": "iterations/s", "cores": threads, "kind": "reference",
                                           "host_cpu": cpu,
                                           "sample": f"kmeans_assign + kmeans_update (src/index/kmeans.cpp:91-135) "
                                                     f"on {KM_CPU_SAMPLE:,} of the {KM_N:,} points per step, time "
                                                     f"scaled by n (work is linear in n); OpenMP on {threads} threads"},
                          "e2e": {"value": v, "unit": "iterations/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}))
        return 0

    ops = GpuKmeansOps()
    c = torch.empty((KM_K, KM_DIM), device=dev)
    a = torch.empty(KM_N, dtype=torch.int32, device=dev)
    mind = torch.empty(KM_N, device=dev)
    s_sum = torch.empty((KM_K, KM_DIM), dtype=torch.float64, device=dev)
    s_comp = torch.empty_like(s_sum)
    s_cnt = torch.empty(KM_K, dtype=torch.int64, device=dev)

    # The whole fit once: k-means++ + 20 Lloyd iterations (+ the final update and the
    # reference's running-total inertia), through the library's device entry point.
    t0 = time.perf_counter()
    it, inertia = kmeans_fit_device(x.data_ptr(), KM_N, KM_DIM, KM_K, c.data_ptr(), a.data_ptr(), max_iter=KM_ITERS,
                                    epsilon=0.0, seed=KM_SEED, algorithm=N.KMEANS_LLOYD)
    fit_s = time.perf_counter() - t0
    # Steps continue from the fitted centroids (the same work per iteration as any other).
    host_mind = torch.empty(KM_N, dtype=torch.float32, pin_memory=True)

    def one_iteration(xx):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        ev[0].record()
        ops.assign(xx, c, False, a, mind)
        ev[1].record()
        host_mind.copy_(mind)
        np.add.accumulate(host_mind.numpy().astype(np.float64))[-1]   # inertia in point order
        ev[2].record()
        s_sum.zero_(), s_comp.zero_(), s_cnt.zero_()
        ops.accumulate(xx, a, KM_K, N.KMEANS_LLOYD, s_sum, s_comp, s_cnt)
        ops.finish(s_sum, s_cnt, N.KMEANS_LLOYD, c)
        ev[3].record()
        return ev

    for _ in range(args.warmup):
        one_iteration(x)
    torch.cuda.synchronize()
    evs = []
    with ClockSampler(local) as clk:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(args.steps):
            evs.append(one_iteration(x))
        e1.record()
        torch.cuda.synchronize()
    ms_total = e0.elapsed_time(e1)
    e_ms = sum(e[0].elapsed_time(e[1]) for e in evs) / len(evs)
    inert_ms = sum(e[1].elapsed_time(e[2]) for e in evs) / len(evs)
    m_ms = sum(e[2].elapsed_time(e[3]) for e in evs) / len(evs)

    # e2e: the points copied from pinned host memory every step, the centroids read back.
    x_host = torch.empty((KM_N, KM_DIM), dtype=torch.float32, pin_memory=True)
    x_host.copy_(x)
    x_dev = torch.empty_like(x)
    c_host = torch.empty((KM_K, KM_DIM), dtype=torch.float32, pin_memory=True)
    e2e = []
    for s in range(args.warmup + args.steps):
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        x_dev.copy_(x_host, non_blocking=True)
        one_iteration(x_dev)
        c_host.copy_(c)
        f1.record()
        torch.cuda.synchronize()
        if s >= args.warmup:
            e2e.append(f0.elapsed_time(f1))
    e2e_ms = sum(e2e) / len(e2e)

    peaks, peak_kind = measured_peaks()
    tf32 = peaks["bf16_tflops"] / 2.0
    flop = 2.0 * KM_N * KM_K * KM_DIM
    achieved = flop / (e_ms / 1e3) / 1e12
    m_bytes = KM_N * KM_DIM * 4 + KM_N * 4
    out = {"metric": KM_METRIC, "value": args.steps / (ms_total / 1e3), **out_common,
           "ms_per_step": ms_total / args.steps,
           "e2e": {"value": 1e3 / e2e_ms, "unit": "iterations/s", "h2d_bytes_per_step": KM_N * KM_DIM * 4,
                   "d2h_bytes_per_step": KM_K * KM_DIM * 4 + KM_N * 4, "ms_per_step": e2e_ms},
           "gpu_launches": args.steps * kmeans_launches_per_iteration(),
           "roofline": {"bound": "tensor", "kernel": "E-step: tc_argmin_kernel (tcgen05 kind::tf32 screen fused "
                                                     "with the arg-min and its exact refine)",
                        "achieved": achieved, "peak": tf32, "unit": "TFLOP/s", "frac": achieved / tf32,
                        "peak_source": f"{peak_kind} bf16 dense burst / 2 (tf32 dense rate)",
                        "traffic": None, "algorithmic_flop_per_step": flop, "estep_ms": e_ms},
           "stage_ms": {"estep_ms": e_ms, "inertia_ms": inert_ms, "mstep_ms": m_ms},
           "mstep": {"algorithmic_bytes": m_bytes, "GBps": m_bytes / (m_ms / 1e3) / 1e9,
                     "hbm_frac": m_bytes / (m_ms / 1e3) / 1e9 / peaks["hbm_gbs"]},
           "fit": {"seconds": fit_s, "iterations": it, "inertia": inertia,
                   "what": "vesper_kmeans_fit_device: k-means++ (16,384 host draws on GPU D^2) + 20 Lloyd "
                           "iterations + final update and running-total inertia"},
           "clocks": clk.summary()}
    if not args.no_cpu_baseline:
        out.update(kmeans_cpu_leg(torch, dev, x, c))
    print(json.dumps(out))
    ops.close()
    return 0


def kmeans_cpu_leg(torch, dev, x, c):
    """The reference's Lloyd iteration (kmeans_assign + kmeans_update) on a sample of the
    points with the GPU's current centroids, and the scaled fit (200,000 points, k=2,048,
    20 iterations from k-means++) run by the library and by the reference, compared bit
    for bit."""
    import numpy as np
    from vesper_db_b200.kmeans import kmeans_cluster
    threads, cpu = reference_threads()
    ol = _oracle_lib()
    ref = ol.Reference(ol.REF_SO)
    n_s = min(KM_CPU_SAMPLE, KM_N)
    xs = x[:n_s].cpu().numpy()
    cs = c.cpu().numpy()
    t = time.perf_counter()
    a_ref, _ = ref.kmeans_assign(xs, cs)
    c_ref = ref.kmeans_update(xs, a_ref, cs)
    el = time.perf_counter() - t
    ops = __import__("vesper_db_b200.shard", fromlist=["GpuKmeansOps"]).GpuKmeansOps()
    xs_d = x[:KM_CPU_SAMPLE].contiguous()
    a_d = torch.empty(KM_CPU_SAMPLE, dtype=torch.int32, device=dev)
    m_d = torch.empty(KM_CPU_SAMPLE, device=dev)
    c_d = c.clone()
    ops.assign(xs_d, c_d, False, a_d, m_d)
    ss = torch.zeros((KM_K, KM_DIM), dtype=torch.float64, device=dev)
    sc, sn = torch.zeros_like(ss), torch.zeros(KM_K, dtype=torch.int64, device=dev)
    from vesper_db_b200 import _native as N
    ops.accumulate(xs_d, a_d, KM_K, N.KMEANS_LLOYD, ss, sc, sn)
    ops.finish(ss, sn, N.KMEANS_LLOYD, c_d)
    ops.close()
    same_step = {"points": KM_CPU_SAMPLE,
                 "assignments_equal": bool(np.array_equal(a_d.cpu().numpy().view(np.uint32), a_ref)),
                 "centroids_equal": bool(np.array_equal(c_d.cpu().numpy(), c_ref))}
    # scaled fit, both sides from k-means++ with seed 42
    xp = x[:KM_PARITY_N].cpu().numpy()
    t = time.perf_counter()
    g = kmeans_cluster(xp, KM_PARITY_K, max_iter=KM_ITERS, epsilon=0.0, seed=KM_SEED)
    g_s = time.perf_counter() - t
    t = time.perf_counter()
    rc, ra, rit, rin = ref.kmeans_lloyd(xp, KM_PARITY_K, max_iter=KM_ITERS, eps=0.0, seed=KM_SEED)
    r_s = time.perf_counter() - t
    fit_parity = {"n": KM_PARITY_N, "k": KM_PARITY_K, "iterations": [g.iterations, rit],
                  "assignments_equal": bool(np.array_equal(g.assignments, ra)),
                  "centroids_equal": bool(np.array_equal(g.centroids, rc)),
                  "inertia": [g.inertia, rin], "inertia_equal": g.inertia == rin,
                  "gpu_fit_s_host_api": g_s, "reference_fit_s": r_s}
    v = 1.0 / (el * KM_N / KM_CPU_SAMPLE)
    return {"cpu_baseline": {"value": v, "unit": "iterations/s", "cores": threads, "kind": "reference",
                             "host_cpu": cpu,
                             "sample": f"one Lloyd iteration (kmeans_assign + kmeans_update, src/index/kmeans.cpp:"
                                       f"91-135) on {KM_CPU_SAMPLE:,} points with the GPU's centroids, {el:.2f} s, "
                                       f"scaled by n to the {KM_N:,} points"},
            "parity_vs_reference": {"lloyd_iteration": same_step, "fit": fit_parity}}


# ------------------------------------------------------------------------------- sharded 100M-vector search
C5_N, C5_DIM, C5_CENTRES, C5_SIGMA = 100_000_000, 128, 200_000, 0.1
C5_NLIST, C5_M, C5_NQ, C5_NPROBE, C5_K = 65_536, 32, 100_000, 64, 100
C5_CHUNK = 6_250_000          # rows per generated chunk (16 chunks; divisible by 1/2/4/8)
C5_TRAIN = 2_000_000          # training rows: the first rows of chunk 0, about 30 per list
C5_GT_Q = 1_000               # queries with exact ground truth (strided across the batch)
C5_CPU_Q = 128                # queries the reference searches in the cpu_baseline leg
C5_METRIC = "QPS at recall@100 (IVF-PQ, 100M x 128, 100k-query batch) at 1/2/4/8 B200 vs CPU ref"
C5_BASE_SEED, C5_QUERY_SEED = 9000, 5678


def c5_workload():
    return (f"Sharded IVF-PQ: N={C5_N:,} x d=128 fp32 from a seeded mixture of 200,000 isotropic Gaussians "
            f"(sigma=0.1, centres ~U[-1,1]), nlist=65,536, m=32x8 bits (no OPQ), {C5_NQ:,} queries, nprobe=64, "
            f"k=100, L2; database sharded by vector across the GPUs")


def greedy_bins(sizes, bins):
    """Greedy size-balanced bin packing of lists (largest first onto the lightest GPU):
    the max/mean load a partition by list would have."""
    import heapq
    loads = [(0, b) for b in range(bins)]
    heapq.heapify(loads)
    for s in sorted((int(x) for x in sizes), reverse=True):
        load, b = heapq.heappop(loads)
        heapq.heappush(loads, (load + s, b))
    mx = max(l for l, _ in loads)
    return mx / (sum(int(x) for x in sizes) / bins)


def main_c5(args):
    """A step is one search of the 100k-query batch (nprobe 64, k 100) over the whole
    100M-vector database: on one GPU the full index, on W GPUs a 1/W vector shard per
    rank with the probe lists computed once per query across ranks and the per-rank
    top-100 merged over NCCL.  The index is trained on the GPU (k-means++ and Elkan
    k-means on 2,000,000 rows, PQ sub-quantizers) and filled chunk by chunk; nothing of
    that is timed."""
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
    ours = args.impl == "ours"
    if world > 1 and ours:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=900), device_id=dev)
    from vesper_db_b200 import IvfPqIndex
    from vesper_db_b200.shard import ShardResults, ThresholdExchange, chunks_of, merge_topk, probed_search
    shard_world = world if ours else 1
    n_chunks = C5_N // C5_CHUNK
    my_chunks = chunks_of(rank if ours else 0, shard_world, n_chunks)

    def chunk_rows(c, out=None):
        return synth.gen_isotropic_mixture(torch, dev, C5_CENTRES, C5_DIM, C5_SIGMA, C5_CHUNK, C5_BASE_SEED + c, out)

    t0 = time.perf_counter()
    queries = synth.gen_isotropic_mixture(torch, dev, C5_CENTRES, C5_DIM, C5_SIGMA, C5_NQ, C5_QUERY_SEED)
    gt_rows = np.linspace(0, C5_NQ - 1, C5_GT_Q).round().astype(np.int64)
    q_gt = queries[torch.from_numpy(gt_rows).to(dev)].contiguous()
    index = IvfPqIndex()
    train = chunk_rows(0)[:C5_TRAIN].contiguous()
    torch.cuda.synchronize()
    t_train0 = time.perf_counter()
    index.train_device(train.data_ptr(), C5_TRAIN, C5_DIM, C5_NLIST, C5_M, 8, use_opq=False)
    t_train = time.perf_counter() - t_train0
    del train
    buf = torch.empty((C5_CHUNK, C5_DIM), device=dev)
    ids = torch.empty(C5_CHUNK, dtype=torch.int64, device=dev)
    gt_d = torch.full((C5_GT_Q, C5_K), float("inf"), device=dev)
    gt_i = torch.zeros((C5_GT_Q, C5_K), dtype=torch.int64, device=dev)
    torch.backends.cuda.matmul.allow_tf32 = False
    qn = (q_gt * q_gt).sum(1, keepdim=True)
    t_add = 0.0
    for c in my_chunks:
        chunk_rows(c, out=buf)
        torch.arange(c * C5_CHUNK, (c + 1) * C5_CHUNK, out=ids)
        torch.cuda.synchronize()
        ta = time.perf_counter()
        index.add_device(ids.data_ptr(), buf.data_ptr(), C5_CHUNK)
        t_add += time.perf_counter() - ta
        for s0 in range(0, C5_CHUNK, 500_000):   # exact fp32 ground truth of the sampled queries
            x = buf[s0:s0 + 500_000]
            dd = qn - 2.0 * (q_gt @ x.T) + (x * x).sum(1)[None, :]
            v, i = torch.topk(dd, C5_K, dim=1, largest=False)
            cd, ci = torch.cat([gt_d, v], 1), torch.cat([gt_i, i + c * C5_CHUNK + s0], 1)
            gt_d, sel = torch.topk(cd, C5_K, dim=1, largest=False)
            gt_i = torch.gather(ci, 1, sel)
    del buf, ids
    torch.cuda.empty_cache()   # the search holds only the index and the queries
    if world > 1 and ours:
        gt_d, gt_i = merge_topk(gt_d, gt_i, C5_K)
    gt_np = gt_i.cpu().numpy()
    torch.cuda.synchronize()
    build = {"setup_s": time.perf_counter() - t0, "train_s": t_train, "add_s": t_add}

    # list shape: this rank's lists, and the global list sizes (summed over the shards)
    local_sizes = np.diff(index.list_offsets().astype(np.int64))
    sizes_t = torch.from_numpy(local_sizes).to(dev)
    if world > 1 and ours:
        dist.all_reduce(sizes_t)
    sizes = sizes_t.cpu().numpy()
    list_stats_c5 = {"lists": int(sizes.size), "mean": float(sizes.mean()), "max": int(sizes.max()),
                     "p99": float(np.percentile(sizes, 99)), "empty": int((sizes == 0).sum()),
                     "max_over_mean": float(sizes.max() / sizes.mean()),
                     "list_partition_max_over_mean": {str(b): greedy_bins(sizes, b) for b in (2, 4, 8)}}

    if args.impl == "reference":
        return c5_reference_arm(args, index, queries.cpu().numpy(), gt_rows, gt_np, build, list_stats_c5)

    probe_bufs, phase, tau_x = {}, {}, None
    if world > 1:
        shard_res = ShardResults(C5_NQ, C5_K, dev)
        out_ids, out_d, out_n = shard_res.ids, shard_res.dist, shard_res.counts
        if not args.no_tau_exchange:
            tau_x = ThresholdExchange().install(index)
    else:
        out_ids = torch.empty((C5_NQ, C5_K), dtype=torch.int64, device=dev)
        out_d = torch.empty((C5_NQ, C5_K), dtype=torch.float32, device=dev)
        out_n = torch.empty(C5_NQ, dtype=torch.int32, device=dev)

    def one_search(q, local=None):
        if world > 1:
            probed_search(index, q, C5_K, C5_NPROBE, C5_NLIST, out_ids, out_d, out_n, probe_bufs, local=local,
                          times=phase)
            t0 = time.perf_counter()
            md, mi, mn = shard_res.merge()
            phase["merge_ms"] = phase.get("merge_ms", 0.0) + (time.perf_counter() - t0) * 1e3
            return md, mi, mn
        index.search_batch_device(q.data_ptr(), C5_NQ, C5_K, C5_NPROBE, out_ids.data_ptr(), out_d.data_ptr(),
                                  out_n.data_ptr())
        return out_d, out_ids, out_n

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        one_search(queries)
    barrier()
    steps_t, launches = [], 0
    phase.clear()
    with ClockSampler(local) as clk:
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.nvtx.range_push("timed_search")
        ev0.record()
        for _ in range(args.steps):
            res_d, res_i, res_n = one_search(queries)
            t = index.last_timings()
            steps_t.append(t)
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
    gi_all, gd_all, gn_all = res_i.cpu().numpy(), res_d.cpu().numpy(), res_n.cpu().numpy()
    recall = recall_at(gi_all[gt_rows], gt_np, C5_K)
    stage_ms = {k2: sum(t[k2] for t in steps_t) / len(steps_t) for k2 in steps_t[0] if k2.endswith("_ms")}
    timings = steps_t[-1]
    shard_phase = None
    if world > 1:
        shard_phase = {k2: v / args.steps for k2, v in phase.items()}
        names = sorted(stage_ms)
        tt = torch.tensor([stage_ms[n] for n in names], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        shard_phase["stage_ms_max_over_ranks"] = dict(zip(names, tt.tolist()))
        shard_phase["threshold_exchange"] = tau_x is not None

    # e2e: pinned host queries in (one GPU: the whole batch; several: each rank its
    # slice, all-gathered with the probe lists), merged results to the host, every step
    q_host = torch.empty((C5_NQ, C5_DIM), dtype=torch.float32, pin_memory=True)
    q_host.copy_(queries)
    q_dev = torch.empty_like(queries)
    per = C5_NQ // world
    q_local = torch.empty((per, C5_DIM), dtype=torch.float32, device=dev) if world > 1 else None
    # the result (120 MB per 100k batch) lands in pinned host buffers
    h_ids = torch.empty((C5_NQ, C5_K), dtype=torch.int64, pin_memory=True)
    h_d = torch.empty((C5_NQ, C5_K), dtype=torch.float32, pin_memory=True)
    e2e_ms = []
    for s in range(args.warmup + args.steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        e0.record()
        if world > 1:
            q_local.copy_(q_host[rank * per:(rank + 1) * per], non_blocking=True)
        else:
            q_dev.copy_(q_host, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        md, mi, _ = one_search(q_dev, local=q_local)
        if rank == 0:
            h_ids.copy_(mi, non_blocking=True)
            h_d.copy_(md, non_blocking=True)
            torch.cuda.current_stream().synchronize()
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
    entries = sum(t["scanned_entries"] for t in steps_t) / len(steps_t)
    if timings["scan_variant"] == 4:
        lk = stage_ms["list_kernel_ms"]
        flop = 2.0 * C5_DIM * entries
        achieved = flop / (lk / 1e3) / 1e12
        roofline = {"bound": "tensor", "kernel": "tc_list_scan_kernel (tcgen05 kind::f16, bf16, A in TMEM)",
                    "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                    "frac": achieved / peaks["bf16_tflops"], "peak_source": f"{peak_kind} (bf16 dense, burst)",
                    "traffic": None, "algorithmic_flop_per_search": flop, "kernel_ms_per_search": lk,
                    "scan_stage_code_GBps": entries * C5_M / (stage_ms["scan_ms"] / 1e3) / 1e9,
                    "scan_stage_code_hbm_frac": entries * C5_M / (stage_ms["scan_ms"] / 1e3) / 1e9 / peaks["hbm_gbs"],
                    "candidates_refined": timings["list_candidates"],
                    "fallback_queries": timings["list_fallback_queries"]}
    else:
        achieved = entries * C5_M / (stage_ms["scan_ms"] / 1e3) / 1e9
        roofline = {"bound": "hbm", "kernel": SCAN_KERNELS.get(timings["scan_variant"], "?"), "achieved": achieved,
                    "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                    "peak_source": peak_kind, "traffic": None}
    out = {"metric": C5_METRIC, "value": C5_NQ * args.steps / (ms_total / 1e3), "unit": "queries/s",
           "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
           "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
           "data": "synthetic (seeded isotropic mixture generated on device)",
           "config": {"workload": c5_workload(), "nlist": C5_NLIST, "m": C5_M, "nprobe": C5_NPROBE, "k": C5_K,
                      "nq": C5_NQ, "n_base": C5_N, "n_train": C5_TRAIN,
                      "parallelism": f"vector-sharded x{world}" if world > 1 else "single GPU",
                      "l2_policy": "inputs larger than L2 (3.2 GB of PQ codes)", "list_stats": list_stats_c5,
                      "probed_entries_per_query_per_rank": entries / C5_NQ},
           "recall@100": recall, "recall_queries": C5_GT_Q,
           "e2e": {"value": C5_NQ / (e2e_step / 1e3), "unit": "queries/s", "h2d_bytes_per_step": C5_NQ * C5_DIM * 4,
                   "d2h_bytes_per_step": C5_NQ * C5_K * 12, "ms_per_step": e2e_step,
                   "path": "pinned H2D of the batch (N>1: each rank its slice, all-gathered with the probe "
                           "lists), search (N>1: threshold exchange, packed result all-gather, device merge), "
                           "rank 0 copies the merged result into pinned host memory"},
           "gpu_launches": launches, "roofline": roofline, "stage_ms": stage_ms,
           "outside_engine_ms": ms_step - stage_ms["total_ms"], "shard_phase_ms": shard_phase,
           "coarse_kernel": COARSE_KERNELS.get(timings["coarse_variant"], "?"), "build": build,
           "clocks": clk.summary()}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            out.update(c5_cpu_leg(index, queries.cpu().numpy(), gt_rows, gt_np, gi_all, gd_all, gn_all))
        except Exception as e:
            out["cpu_baseline"] = {"value": None, "unit": "queries/s", "cores": os.cpu_count(), "kind": "reference",
                                   "sample": f"unavailable: {e}"}
    if rank == 0:
        print(json.dumps(out))
    if world > 1:
        index.set_threshold_exchange(None)
    index.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def c5_reference_search(index):
    """Save the GPU-built index as the reference's v1.0 file and load it into the
    reference's IvfPqIndex (untimed); returns (reference index, load seconds, threads,
    host description)."""
    threads, cpu = reference_threads()
    ol = _oracle_lib()
    tmp = tempfile.mkdtemp(prefix="vesper_c5_")
    try:
        index.save(tmp)
        ridx = ol.Reference(ol.REF_SO).ivfpq()
        t0 = time.perf_counter()
        ridx.load(tmp)
        load_s = time.perf_counter() - t0
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    return ridx, load_s, threads, cpu


def c5_cpu_leg(index, q_np, gt_rows, gt_np, gi_all, gd_all, gn_all):
    """The reference's search_batch on C5_CPU_Q of the ground-truth queries: its QPS,
    its recall@100 beside the GPU's on the same queries, and the GPU results compared
    with the reference's ids and distances (the heap branch of its top-k, pool > 64)."""
    import numpy as np
    ridx, load_s, threads, cpu = c5_reference_search(index)
    pick = np.linspace(0, C5_GT_Q - 1, C5_CPU_Q).round().astype(np.int64)
    rows = gt_rows[pick]
    qs = np.ascontiguousarray(q_np[rows])
    ridx.search(qs[:4], C5_K, C5_NPROBE)
    t = time.perf_counter()
    rid, rd, rcnt = ridx.search(qs, C5_K, C5_NPROBE)
    el = time.perf_counter() - t
    par = topk_parity(gi_all[rows], gd_all[rows], gn_all[rows], rid, rd, rcnt)
    return {"cpu_baseline": {"value": C5_CPU_Q / el, "unit": "queries/s", "cores": threads, "kind": "reference",
                             "host_cpu": cpu,
                             "sample": f"{C5_CPU_Q} queries of the batch, nprobe={C5_NPROBE}, k={C5_K}, reference "
                                       f"IvfPqIndex::search_batch with OpenMP on {threads} threads, {el:.1f} s; "
                                       f"v1.0 file load {load_s:.0f} s untimed"},
            "recall_matched": [{"nprobe": C5_NPROBE, "queries": C5_CPU_Q, "gpu": recall_at(gi_all[rows], gt_np[pick], C5_K),
                                "cpu": recall_at(rid, gt_np[pick], C5_K)}],
            "parity_vs_reference": par}


def c5_reference_arm(args, index, q_np, gt_rows, gt_np, build, list_stats_c5):
    import numpy as np
    ridx, load_s, threads, cpu = c5_reference_search(index)
    index.close()
    per_step = max(16, 2 * threads)
    step_s, hits, done, qpos = [], 0, 0, 0
    for s in range(args.warmup + args.steps):
        rows = gt_rows[(np.arange(per_step) + qpos) % C5_GT_Q]
        qpos += per_step
        t = time.perf_counter()
        rid, _, _ = ridx.search(np.ascontiguousarray(q_np[rows]), C5_K, C5_NPROBE)
        el = time.perf_counter() - t
        if s >= args.warmup:
            step_s.append(el)
            g = gt_np[(np.arange(per_step) + qpos - per_step) % C5_GT_Q]
            hits += sum(len(set(a) & set(b)) for a, b in zip(rid.tolist(), g.tolist()))
            done += per_step
    v = done / sum(step_s)
    print(json.dumps({"impl": "reference", "metric": C5_METRIC, "value": v, "unit": "queries/s",
                      "higher_is_better": True, "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                      "ms_per_step": 1e3 * sum(step_s) / len(step_s), "queries_per_step": per_step,
                      "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded mixture)",
                      "config": {"workload": c5_workload(), "nprobe": C5_NPROBE, "k": C5_K, "nq": C5_NQ,
                                 "list_stats": list_stats_c5},
                      "recall@100": hits / max(1, done * C5_K),
                      "cpu_baseline": {"value": v, "unit": "queries/s", "cores": threads, "kind": "reference",
                                       "host_cpu": cpu,
                                       "sample": f"{done} queries ({per_step} per step) of the batch, OpenMP on "
                                                 f"{threads} threads; v1.0 file load {load_s:.0f} s untimed"},
                      "e2e": {"value": v, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                      "build": build}))
    return 0


# ------------------------------------------------------------------------------- main
def build_ivfpq_workload(args, torch, dev, world, rank):
    """Data, training and add of the IVF-PQ+OPQ workload on this rank's GPU (untimed),
    plus the exact ground truth of the query batch."""
    from vesper_db_b200 import IvfPqIndex
    from vesper_db_b200.shard import chunks_of, merge_topk
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
    torch.cuda.empty_cache()   # the search holds only the index and the queries
    build = {"data_s": t_data, "train_s": t_train, "add_s": t_add, "opq_kept": rep.opq_kept,
             "err_unrot": rep.err_unrot, "err_opq": rep.err_opq}
    return index, queries, gt_i.cpu().numpy(), build


def reference_arm(args, index, q_np, gt_np, build):
    """--impl reference: the reference's own IvfPqIndex::search_batch (AVX2 build, OpenMP
    over every host CPU) on the same index, handed over through its v1.0 file.  Each
    step searches the next slice of the query batch; the value is the queries searched
    over the summed step times."""
    threads, cpu = reference_threads()
    ol = _oracle_lib()
    out = {"impl": "reference", "metric": METRIC, "unit": "queries/s", "higher_is_better": True,
           "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "scaling": "strong",
           "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded mixture)",
           "config": {"workload": WORKLOAD, "nlist": NLIST, "m": M, "nbits": NBITS, "nprobe": NPROBE, "k": K,
                      "nq": NQ, "n_base": N_BASE, "n_train": N_TRAIN, "search_mode": "reference search_batch",
                      "parallelism": "host CPU (OpenMP)"}}
    tmp = tempfile.mkdtemp(prefix="vesper_ref_")
    try:
        index.save(tmp)
        index.close()
        ridx = ol.Reference(ol.REF_SO).ivfpq()
        t0 = time.perf_counter()
        ridx.load(tmp)
        load_s = time.perf_counter() - t0
        per_step = max(16, 4 * threads)   # one query slice per step, a few queries per thread
        step_s, hits, nq_done, qpos = [], 0, 0, 0
        for s in range(args.warmup + args.steps):
            lo = qpos % NQ
            qb = q_np[lo:lo + per_step]
            t = time.perf_counter()
            rid, _, _ = ridx.search(qb, K, NPROBE)
            el = time.perf_counter() - t
            qpos += qb.shape[0]
            if s >= args.warmup:
                step_s.append(el)
                g = gt_np[lo:lo + qb.shape[0]]
                hits += sum(len(set(a) & set(b)) for a, b in zip(rid.tolist(), g.tolist()))
                nq_done += qb.shape[0]
        v = nq_done / sum(step_s)
        out.update({"value": v, "ms_per_step": 1e3 * sum(step_s) / len(step_s), "queries_per_step": per_step,
                    "recall@10": hits / max(1, nq_done * K),
                    "cpu_baseline": {"value": v, "unit": "queries/s", "cores": threads, "kind": "reference",
                                     "host_cpu": cpu,
                                     "sample": f"{nq_done} queries of the 10k batch, {per_step} per step over "
                                               f"{args.steps} steps, nprobe={NPROBE}, k={K}, OpenMP on {threads} "
                                               f"threads; index load {load_s:.1f} s untimed"},
                    "e2e": {"value": v, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                    "build": build})
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    print(json.dumps(out))
    return 0


def cpu_leg(index, q_np, gt_np, gpu_results, seconds_hint):
    """Rank 0 at N=1: the reference's search_batch on a strided sample of the batch at
    every swept nprobe -- its QPS (the cpu_baseline at the headline nprobe), its recall
    beside the GPU's on exactly the same queries, and the GPU results compared with the
    reference's ids and distances."""
    import numpy as np
    threads, cpu = reference_threads()
    ol = _oracle_lib()
    sample = np.linspace(0, NQ - 1, CPU_SAMPLE).round().astype(np.int64)
    qs = np.ascontiguousarray(q_np[sample])
    tmp = tempfile.mkdtemp(prefix="vesper_cpu_")
    try:
        index.save(tmp)
        ridx = ol.Reference(ol.REF_SO).ivfpq()
        t0 = time.perf_counter()
        ridx.load(tmp)
        load_s = time.perf_counter() - t0
        ridx.search(qs[:8], K, NPROBE)  # warm-up
        matched, parity, qps = [], {}, {}
        for npb in SWEEP:
            t = time.perf_counter()
            rid, rd, rcnt = ridx.search(qs, K, npb)
            el = time.perf_counter() - t
            qps[npb] = CPU_SAMPLE / el
            gi, gd, gn = gpu_results[npb]
            gi, gd, gn = gi[sample], gd[sample], gn[sample]
            matched.append({"nprobe": npb, "queries": CPU_SAMPLE,
                            "gpu": recall_at(gi, gt_np[sample], K), "cpu": recall_at(rid, gt_np[sample], K),
                            "cpu_qps": qps[npb]})
            parity[npb] = topk_parity(gi, gd, gn, rid, rd, rcnt)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    base = {"value": qps[NPROBE], "unit": "queries/s", "cores": threads, "kind": "reference", "host_cpu": cpu,
            "sample": f"{CPU_SAMPLE} queries strided across the 10k batch, nprobe={NPROBE}, k={K}, reference "
                      f"IvfPqIndex::search_batch with OpenMP on {threads} threads; index load {load_s:.1f} s untimed",
            "recall@10": matched[SWEEP.index(NPROBE)]["cpu"]}
    par = dict(parity[NPROBE])
    par["by_nprobe"] = {str(k2): v for k2, v in parity.items()}
    return base, matched, par


def main():
    args = parse()
    if args.workload == "flat":
        return main_flat(args)
    if args.workload == "kmeans":
        return main_kmeans(args)
    if args.workload == "c5":
        return main_c5(args)
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

    from vesper_db_b200.shard import ShardResults, ThresholdExchange, probed_search
    index, queries, gt_np, build = build_ivfpq_workload(args, torch, dev, world, rank)
    q_np = queries.cpu().numpy()
    if args.impl == "reference":
        return reference_arm(args, index, q_np, gt_np, build)

    # ------------------------------------------------------------------ our arm
    # Multi-GPU: each rank probes 1/world of the batch (the coarse stage is the same on
    # every shard) and the probe lists are all-gathered before the shard searches; the
    # shards share their per-query k-th-distance bounds (threshold exchange, an
    # all-reduce MIN inside the search) and their packed results are all-gathered and
    # merged on the device.
    probe_bufs, phase, tau_x = {}, {}, None
    if world > 1:
        shard_res = ShardResults(NQ, K, dev)
        out_ids, out_d, out_n = shard_res.ids, shard_res.dist, shard_res.counts
        if not args.no_tau_exchange:
            tau_x = ThresholdExchange().install(index)
    else:
        out_ids = torch.empty((NQ, K), dtype=torch.int64, device=dev)
        out_d = torch.empty((NQ, K), dtype=torch.float32, device=dev)
        out_n = torch.empty(NQ, dtype=torch.int32, device=dev)

    def one_search(q, nprobe, local=None):
        if world > 1:
            probed_search(index, q, K, nprobe, NLIST, out_ids, out_d, out_n, probe_bufs, local=local, times=phase)
            t0 = time.perf_counter()
            md, mi, mn = shard_res.merge()
            phase["merge_ms"] = phase.get("merge_ms", 0.0) + (time.perf_counter() - t0) * 1e3
            return md, mi, mn
        index.search_batch_device(q.data_ptr(), NQ, K, nprobe, out_ids.data_ptr(), out_d.data_ptr(),
                                  out_n.data_ptr())
        return out_d, out_ids, out_n

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        one_search(queries, NPROBE)
    barrier()
    steps_t, launches = [], 0
    phase.clear()
    with ClockSampler(local) as clk:
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.nvtx.range_push("timed_search")
        ev0.record()
        for _ in range(args.steps):
            res_d, res_i, res_n = one_search(queries, NPROBE)
            t = index.last_timings()
            steps_t.append(t)
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
    recall = recall_at(res_i.cpu().numpy(), gt_np, K)
    stage_ms = {k2: sum(t[k2] for t in steps_t) / len(steps_t) for k2 in steps_t[0] if k2.endswith("_ms")}
    timings = steps_t[-1]
    shard_phase = None
    if world > 1:
        # host-side time per step of the sharded search's phases (rank 0; the library's
        # calls are synchronous, the merge is only queued), and the slowest rank's stages
        shard_phase = {k2: v / args.steps for k2, v in phase.items()}
        names = sorted(stage_ms)
        tt = torch.tensor([stage_ms[n] for n in names], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        shard_phase["stage_ms_max_over_ranks"] = dict(zip(names, tt.tolist()))
        shard_phase["threshold_exchange"] = tau_x is not None

    # nprobe sweep: SWEEP_PASSES timed passes per nprobe, recall of the last pass
    sweep, gpu_results = [], {}
    for npb in SWEEP:
        one_search(queries, npb)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(SWEEP_PASSES):
            rd, ri, rn = one_search(queries, npb)
        e1.record()
        barrier()
        ms = e0.elapsed_time(e1) / SWEEP_PASSES
        if world > 1:
            tt = torch.tensor([ms], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            ms = float(tt.item())
        ri_np = ri.cpu().numpy()
        gpu_results[npb] = (ri_np, rd.cpu().numpy(), rn.cpu().numpy())
        sweep.append({"nprobe": npb, "qps": NQ / (ms / 1e3), "passes": SWEEP_PASSES,
                      "recall@10": recall_at(ri_np, gt_np, K),
                      "stage_ms": {k2: v for k2, v in index.last_timings().items() if k2.endswith("_ms")}})

    # e2e: host query buffer in, host result out, every step.  One GPU: the reference's
    # C call vesper_ivfpq_search_batch with host buffers (copies inside the library).
    # Several GPUs: each rank copies its 1/world slice of the batch from pinned host
    # memory, the slices travel with the probe exchange (NVLink), the sharded search
    # runs, and rank 0 reads the merged result.
    q_host = torch.empty((NQ, DIM), dtype=torch.float32, pin_memory=True)
    q_host.copy_(queries)
    q_host_np = q_host.numpy()
    q_dev = torch.empty_like(queries)
    per = NQ // world
    q_local = torch.empty((per, DIM), dtype=torch.float32, device=dev)
    h_ids = torch.empty((NQ, K), dtype=torch.int64, pin_memory=True)
    h_d = torch.empty((NQ, K), dtype=torch.float32, pin_memory=True)
    e2e_ms = []
    for s in range(args.warmup + args.steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        e0.record()
        if world == 1:
            index.search_batch_c(q_host_np, K, NPROBE)
        else:
            q_local.copy_(q_host[rank * per:(rank + 1) * per], non_blocking=True)
            torch.cuda.current_stream().synchronize()   # the library's stream does not wait on torch's
            md, mi, _ = one_search(q_dev, NPROBE, local=q_local)
            if rank == 0:
                h_ids.copy_(mi, non_blocking=True)
                h_d.copy_(md, non_blocking=True)
                torch.cuda.current_stream().synchronize()
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
    entries = sum(t["scanned_entries"] for t in steps_t) / len(steps_t)
    code_bytes = entries * M
    launches_per_search = -(-NQ // SEARCH_QUERY_CHUNK)
    if timings["scan_variant"] == 4:
        # Dominant kernel: the tcgen05 screen.  Algorithmic work = every (query, probed
        # entry) pair's dim-long product, 2 * dim FLOP each.
        lk = stage_ms["list_kernel_ms"]
        flop = 2.0 * DIM * entries
        achieved = flop / (lk / 1e3) / 1e12
        roofline = {"bound": "tensor", "kernel": "tc_list_scan_kernel (tcgen05 kind::f16, bf16, A in TMEM)",
                    "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                    "frac": achieved / peaks["bf16_tflops"], "peak_source": f"{peak_kind} (bf16 dense, burst)",
                    # DRAM bytes per launch: the ncu capture of one main-pass launch on the
                    # 2M-vector case (567.1 MB for 2.209e9 (query, entry) pairs), scaled by
                    # the pairs of one launch here (codes of each probed tile are read once
                    # per batch).
                    "traffic": LIST_SCAN_BYTES_PER_PAIR * entries / launches_per_search,
                    "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, 2M-vector case "
                                      "(--n-base 2000000 --nq 8192), scaled by (query, entry) pairs per launch",
                    "algorithmic_flop_per_search": flop, "kernel_ms_per_search": lk,
                    "launches_per_search": launches_per_search,
                    "scan_stage_ms": stage_ms["scan_ms"],
                    "scan_stage_code_GBps": code_bytes / (stage_ms["scan_ms"] / 1e3) / 1e9,
                    "candidates_refined": timings["list_candidates"],
                    "fallback_queries": timings["list_fallback_queries"]}
    else:
        achieved = code_bytes / (stage_ms["scan_ms"] / 1e3) / 1e9
        roofline = {"bound": "hbm", "kernel": SCAN_KERNELS.get(timings["scan_variant"], "?"), "achieved": achieved,
                    "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                    "peak_source": peak_kind, "traffic": None,
                    "algorithmic_bytes_per_search": code_bytes, "scan_ms": stage_ms["scan_ms"]}
    ls = list_stats(index, NQ, entries)
    ls["probed_entries_per_query_at_mean_list_size"] = NPROBE * ls["mean"]
    if world == 1:
        # padding of the list scan's (tile, query chunk) pairs, from this batch's probe lists
        pr = torch.empty((NQ, min(NPROBE, NLIST)), dtype=torch.int32, device=dev)
        prd = torch.empty((NQ, min(NPROBE, NLIST)), dtype=torch.float32, device=dev)
        index.probe_device(queries.data_ptr(), NQ, NPROBE, pr.data_ptr(), prd.data_ptr())
        ls["list_scan_tiles"] = list_scan_tiles(index, pr.cpu().numpy())
    out = {
        "metric": METRIC, "value": qps, "unit": "queries/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded mixture generated on device)",
        "config": {"workload": WORKLOAD, "nlist": NLIST, "m": M, "nbits": NBITS, "nprobe": NPROBE, "k": K,
                   "nq": NQ, "n_base": N_BASE, "n_train": N_TRAIN, "search_mode": "fast",
                   "parallelism": f"vector-sharded x{world}" if world > 1 else "single GPU",
                   "l2_policy": "inputs larger than L2 (960 MB of PQ codes scanned per pass)",
                   "list_stats": ls},
        "recall@10": recall,
        "sweep": sweep,
        "e2e": {"value": NQ / (e2e_step / 1e3), "unit": "queries/s", "h2d_bytes_per_step": NQ * DIM * 4,
                "d2h_bytes_per_step": NQ * K * 12, "ms_per_step": e2e_step,
                "path": "vesper_ivfpq_search_batch (host buffers)" if world == 1 else
                        "per rank: pinned H2D of its 1/world slice of the batch, probe of the slice, NCCL "
                        "all-gather of the slices and probe lists, shard search with the threshold exchange, "
                        "NCCL all-gather of the packed results and the device merge; rank 0 copies the merged "
                        "result to the host (h2d bytes summed over the ranks)"},
        "gpu_launches": launches,
        "gpu_launches_counted": "the library's own kernels in the search calls, from its launch counter; CUB scan "
                                "kernels excluded" + ("; at N>1 the probe call and the merge kernel not included"
                                                      if world > 1 else ""),
        "roofline": roofline,
        "stage_ms": stage_ms,
        "outside_engine_ms": ms_step - stage_ms["total_ms"],
        "shard_phase_ms": shard_phase,
        "coarse_kernel": COARSE_KERNELS.get(timings["coarse_variant"], "?"),
        "build": build,
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            base, matched, par = cpu_leg(index, q_np, gt_np, gpu_results, args.cpu_seconds)
            out["cpu_baseline"] = base
            out["recall_matched"] = matched
            out["parity_vs_reference"] = par
        except Exception as e:  # the reference oracle may be absent on a machine without it
            out["cpu_baseline"] = {"value": None, "unit": "queries/s", "cores": os.cpu_count(),
                                   "kind": "reference", "sample": f"unavailable: {e}"}
    if rank == 0:
        print(json.dumps(out))
    if world > 1:
        index.set_threshold_exchange(None)
    index.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
