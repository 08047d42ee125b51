"""Benchmark of the exact flat search hot path (config C2: 1M x 128 euclidean, 10k queries, k=10).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python bench.py --workload kmeans [...]   # config C3: k-means 1M x 96, k=4096, 20 iterations
    python bench.py --workload ivfpq [...]    # config C4: IVF-PQ 20M x 128, nlist 16384, m=16, recall@10 >= 0.9
    python bench.py --workload sq [...]       # config C5: SQ int8 filtered scan, 6.25M x 768 per GPU, 4,096 queries

One step = one exact top-k search of all queries over the whole database
(sharded by rows across N GPUs, one process per GPU under torchrun; local
top-k, NCCL allgather of k candidates per query, device merge). Prints one
JSON line on rank 0. Data are synthetic (csrc/fixtures.cpp) with the
configuration's shapes; nothing reads the reference tree at run time.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "queries/s: exact 1M×128 k=10 (FlatIndex batched search, euclidean)"
CONFIG = {"workload": "C2 exact flat search: 1,000,000 x 128 f32 (integers in [0,255], 1,024 blobs, sigma 20), "
                      "10,000 queries, k=10, euclidean",
          "n": 1_000_000, "dim": 128, "queries": 10_000, "k": 10}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--n", type=int, default=1_000_000)
    p.add_argument("--nq", type=int, default=10_000)
    p.add_argument("--k", type=int, default=10)
    p.add_argument("--dim", type=int, default=128)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--cpu-seconds", type=float, default=12.0)
    p.add_argument("--workload", choices=["flat", "kmeans", "ivfpq", "sq", "snapshot"], default="flat")
    p.add_argument("--flat-scaling", choices=["weak", "strong"], default="weak",
                   help="flat at N>1: weak = N x --nq queries per step over the row-sharded database (each GPU "
                        "scans the equivalent of --nq queries x --n rows); strong = --nq queries split N ways")
    p.add_argument("--data", choices=["u8", "real"], default="u8",
                   help="flat: C2's integer rows (u8, the exact u8 tensor-core scan) or the same blobs unrounded "
                        "(real, the f16 tensor-core screen + exact re-rank)")
    p.add_argument("--metric", choices=["euclidean", "cosine"], default="euclidean")
    p.add_argument("--no-extras", action="store_true",
                   help="flat at N=1: skip the sub-records of the other configurations (C2 k=100, real-valued "
                        "C2, C3, C4, C5), each measured by its own bench.py run")
    p.add_argument("--extras-steps", type=int, default=5)
    p.add_argument("--parity-queries", type=int, default=96, help="N>1: queries checked against the oracle")
    p.add_argument("--sq-n", type=int, default=6_250_000, help="rows per GPU (C5: 50M over 8 GPUs)")
    p.add_argument("--ivf-n", type=int, default=20_000_000)
    p.add_argument("--ivf-nlist", type=int, default=16384)
    return p.parse_args()


def k1_source_hash() -> str:
    """SHA-256 of the sources that decide K1's memory traffic (the kernel and its launch), comments
    removed, so that a DRAM-traffic figure captured by ncu is reported only for the code it was
    measured on."""
    import hashlib
    import re

    h = hashlib.sha256()
    for name in ("flat_tc.cuh", "flat.cu", "sm100.cuh"):
        text = (ROOT / "proxima_b200" / "csrc" / name).read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)  # block comments
        text = re.sub(r"//[^\n]*", "", text)  # line comments
        h.update(text.encode())
    return h.hexdigest()


def peaks():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured (MEASURED_PEAKS.json)"
    return 6650.0, 1590.0, "fallback (profiling recipe)"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str | None):
        self.uuid = uuid
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        rows = []
        for line in Path(self.file.name).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 10:
                continue
            if self.uuid and self.uuid not in parts[1]:
                continue
            rows.append(parts)
        os.unlink(self.file.name)
        if not rows:
            return None
        sm = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        mx = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for name, v in zip(names, r[6:10]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(rows)}


def cpu_baseline(db: np.ndarray, queries: np.ndarray, k: int, seconds: float, gpu_ids=None, gpu_dist=None,
                 metric: int = 0) -> dict:
    """The oracle port of FlatIndex::search on all host cores, on a bounded query sample; its answers for
    the sample are also compared with the GPU's, ids and f32 distance bits (gpu_ids / gpu_dist: the GPU's
    answer for every query). `db` and `queries` are prepared (cosine: normalised)."""
    from oracle import pxo

    threads = os.cpu_count() or 1
    batch = max(threads, 8)
    pxo.flat_search(db, queries[:batch], k, metric, nthreads=threads)  # warm
    done, t0, same = 0, time.perf_counter(), 0
    while time.perf_counter() - t0 < seconds and done + batch <= len(queries):
        ref_ids, ref_d, ref_len = pxo.flat_search(db, queries[done:done + batch], k, metric, nthreads=threads)
        if gpu_ids is not None:
            for i in range(batch):
                n_ = ref_len[i]
                same += int(np.array_equal(gpu_ids[done + i, :n_], ref_ids[i, :n_]) and
                            np.array_equal(gpu_dist[done + i, :n_].view(np.uint32), ref_d[i, :n_].view(np.uint32)))
        done += batch
    el = time.perf_counter() - t0
    out = {"value": done / el, "unit": "queries/s", "cores": threads, "kind": "port",
           "sample": f"{done} of the {len(queries)} queries against the full {db.shape[0]:,}-row database "
                     f"({el:.1f} s, C++ oracle restating FlatIndex::search, one query per thread at a time)"}
    if gpu_ids is not None:
        out["parity"] = {"queries": done, "identical_ids_and_distance_bits": same}
    return out


def run_reference(args):
    """--impl reference: the reference algorithm on the host cores (the oracle port; no Rust toolchain here)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from proxima_b200 import fixtures
    from oracle import pxo

    db = fixtures.c2_database(args.n, args.dim)
    queries = fixtures.c2_queries(args.nq, args.dim)
    threads = os.cpu_count() or 1
    per_step = max(threads, 16)
    for w in range(args.warmup):
        pxo.flat_search(db, queries[w * per_step % args.nq:][:per_step], args.k, pxo.EUCLIDEAN, nthreads=threads)
    t0 = time.perf_counter()
    off = 0
    for _ in range(args.steps):
        q = queries[off:off + per_step]
        if len(q) < per_step:
            off, q = 0, queries[:per_step]
        pxo.flat_search(db, q, args.k, pxo.EUCLIDEAN, nthreads=threads)
        off += per_step
    el = time.perf_counter() - t0
    qps = args.steps * per_step / el
    line = {"metric": METRIC, "value": qps, "unit": "queries/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": el * 1000 / args.steps, "higher_is_better": True,
            "scaling": "weak" if args.gpus > 1 and args.flat_scaling == "weak" else "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": dict(CONFIG, parallelism=f"host threads {threads}"), "impl": "reference",
            "cpu_baseline": {"value": qps, "unit": "queries/s", "cores": threads, "kind": "port",
                             "sample": f"each step = {per_step} queries over the full {args.n:,}-row database "
                                       "(C++ restatement of FlatIndex::search; the Rust reference cannot be built here)"},
            "e2e": {"value": qps, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)

KM_METRIC = "Lloyd iterations/s: k-means 1M×96 k=4096 (proxima_quantize::kmeans, 20 iterations from a seeded sample)"
KM_CONFIG = {"workload": "C3 k-means: 1,000,000 x 96 f32 (L2-normalised, 4,096 unit-sphere blobs, sigma 0.05), "
                         "k=4096, 20 Lloyd iterations from 4,096 seeded sample points",
             "n": 1_000_000, "dim": 96, "k": 4096, "iterations": 20}


def kmeans_cpu_baseline(pts: np.ndarray, k: int, seconds: float) -> dict:
    """One Lloyd iteration of the oracle port on a point sample, on all host cores, scaled to the full set.

    The sample's own first k points are the initial centroids, so no cluster
    starts empty and the iteration is the assignment plus the update that
    dominate the reference's cost at full size."""
    from oracle import pxo

    threads = os.cpu_count() or 1
    n = len(pts)
    ns = 4 * k
    while True:
        t0 = time.perf_counter()
        pxo.kmeans(pts[:ns], k, 1, init=pts[:k], nthreads=threads)
        el = time.perf_counter() - t0
        if el > seconds / 3 or ns * 2 > n:
            break
        ns *= 2
    per_iter_full = el * n / ns
    return {"value": 1.0 / per_iter_full, "unit": "iterations/s", "cores": threads, "kind": "port",
            "sample": f"one Lloyd iteration (assignment + update) of the C++ oracle on the first {ns:,} points, "
                      f"the first {k:,} of them as the centroids ({el:.2f} s), scaled linearly to {n:,} points"}


def run_kmeans(args):
    """--workload kmeans: one step = one 20-iteration k-means training of C3 with inputs resident on the GPU."""
    import torch

    from proxima_b200 import _native as N
    from proxima_b200 import fixtures
    from proxima_b200.index import Context
    from proxima_b200.quantize import kmeans

    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    n, dim, k, iters = 1_000_000, 96, 4096, 20
    pts = fixtures.c3_points(n, dim)
    init = fixtures.c3_init(pts, k)
    if args.impl == "reference":
        if rank != 0:
            return
        cb = kmeans_cpu_baseline(pts, k, args.cpu_seconds)
        line = {"metric": KM_METRIC, "value": cb["value"], "unit": "iterations/s", "n_gpus": args.gpus,
                "steps": 1, "warmup": 0, "ms_per_step": 1000.0 / cb["value"] * iters, "higher_is_better": True,
                "scaling": "replicas", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": dict(KM_CONFIG, parallelism=f"host threads {cb['cores']}"), "impl": "reference",
                "cpu_baseline": cb,
                "e2e": {"value": cb["value"], "unit": "iterations/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta

        from proxima_b200.quantize import kmeans_sharded
        from proxima_b200.sharded import init_comm

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    ctx = Context(local)
    lib = N.load()
    lo, hi = rank * n // world, (rank + 1) * n // world
    if world > 1:
        init_comm(ctx, timeout_ms=120_000)

        def kmeans(points, dim_, k_, iters_, init, context, want_assignment=False):  # noqa: F811
            return kmeans_sharded(points, dim_, k_, iters_, init, context)
    N.call("pxc_ctx_set_profiling", ctx.handle, 1)
    dp = torch.from_numpy(pts[lo:hi]).to(dev)
    di = torch.from_numpy(init).to(dev)
    stream = torch.cuda.current_stream(dev)
    for _ in range(max(3, args.warmup)):
        kmeans(dp, dim, k, iters, init=di, context=ctx)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        pass
    sampler = ClockSampler(uuid)
    sampler.start()
    launches0 = lib.pxc_ctx_launch_count(ctx.handle)
    ms, screen_ms, screen_passes, res = [], 0.0, 0, None
    for _ in range(args.steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        res = kmeans(dp, dim, k, iters, init=di, context=ctx)
        b.record(stream)
        torch.cuda.synchronize(dev)
        ms.append(a.elapsed_time(b))
        screen_ms += res.screen_ms
        screen_passes += res.screen_passes
    launches = lib.pxc_ctx_launch_count(ctx.handle) - launches0
    clocks = sampler.stop()
    ms_per_step = sum(ms) / len(ms)
    # e2e: points copied in and centroids + assignments copied out each step
    e2e_steps = max(2, min(args.steps, 3))
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        if world > 1:
            dq = torch.from_numpy(pts[lo:hi]).to(dev)
            kmeans(dq, dim, k, iters, init=init, context=ctx)
        else:
            kmeans(pts, dim, k, iters, init=init, context=ctx, want_assignment=True)
    e2e_s = (time.perf_counter() - t0) / e2e_steps
    if world > 1:
        t = torch.tensor([ms_per_step, e2e_s], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_per_step, e2e_s = t[0].item(), t[1].item()
    if rank == 0:
        hbm, bf16, src = peaks()
        tf32 = bf16 / 2.0  # B200 dense TF32 runs at half its dense BF16 rate
        flops = 2.0 * (hi - lo) * k * dim  # one screening launch on this rank's points
        per_pass = screen_ms / max(1, screen_passes)
        achieved = flops / (per_pass / 1e3) / 1e12 if per_pass > 0 else None
        line = {"metric": KM_METRIC, "value": iters / (ms_per_step / 1e3), "unit": "iterations/s",
                "n_gpus": world, "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": ms_per_step,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "tf32+f32",
                "data": "synthetic",
                "config": dict(KM_CONFIG, step="one 20-iteration training from the same seeded init",
                               l2="inputs (384 MB) larger than L2", iterations_run=res.iterations,
                               reseeded=res.reseeded, rescanned=res.rescanned,
                               parallelism="single GPU" if world == 1 else
                               f"points sharded x{world}; per iteration the inertia, changed flag and per-cluster "
                               "f64 sums + counts exchanged over the library's communicator (rank-order fold)"),
                "clocks": clocks, "gpu_launches": int(launches),
                "e2e": {"value": iters / e2e_s, "unit": "iterations/s", "h2d_bytes_per_step": n * dim * 4 + k * dim * 4,
                        "d2h_bytes_per_step": k * dim * 4 + n * 4},
                "roofline": {"bound": "tensor", "achieved": achieved, "peak": tf32, "unit": "TFLOP/s",
                             "frac": achieved / tf32 if achieved else None, "traffic": None,
                             "kernel": "km_tc::screen_kernel (K7a, CAND pass: the assignment screen of every iteration)",
                             "kernel_ms": per_pass,
                             "peak_source": f"dense bf16 {src} / 2 = dense tf32 rate",
                             "algorithmic_flops_per_launch": flops}}
        if not args.no_cpu_baseline and world == 1:
            line["cpu_baseline"] = kmeans_cpu_baseline(pts, k, args.cpu_seconds)
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


IVF_METRIC = "queries/s: IVF-PQ 20M×128 nlist=16384 m=16 k=10 @recall@10≥0.9 (IvfPqIndex::search_with_nprobe)"
# the operating points swept; the line reports the fastest with recall@10 >= 0.9
IVF_NPROBES = (16, 32, 48, 64, 96)
IVF_RERANKS = (0, 300, 1000, 2000, 3000, 4000)


def run_ivfpq(args):
    """--workload ivfpq: C4 built on the GPU (untimed), then one step = the 10k-query batch search at the
    fastest (nprobe, rerank) whose recall@10 against exact search is >= 0.9."""
    import torch

    from proxima_b200 import _native as N
    from proxima_b200 import fixtures
    from proxima_b200.index import Context
    from proxima_b200.ivfpq import IvfPqIndex

    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    n, dim, nlist, m, nq, k = args.ivf_n, 128, args.ivf_nlist, 16, 10_000, 10
    sample = min(500_000, n)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ctx = Context(local)
    lib = N.load()
    t0 = time.perf_counter()
    chunk = 2_000_000
    d_vec = torch.empty((n, dim), dtype=torch.float32, device=dev)
    for b in range(0, n, chunk):
        e = min(n, b + chunk)
        d_vec[b:e].copy_(torch.from_numpy(fixtures.blobs_u8(e - b, dim, 4096, fixtures.C4_CENTRES, fixtures.C4_BASE,
                                                            row_begin=b)))
    queries = fixtures.blobs_u8(nq, dim, 4096, fixtures.C4_CENTRES, fixtures.C4_QUERIES)
    t_gen = time.perf_counter() - t0
    t0 = time.perf_counter()
    idx = IvfPqIndex(dim, nlist, m, context=ctx)
    idx.set_store_device(d_vec)
    report = idx.train(training_sample=sample, max_iterations=25, seed=0x1FF9C0D)
    torch.cuda.synchronize(dev)
    t_build = time.perf_counter() - t0
    # exact ground truth: the flat index over the same rows (integers: the tensor-core exact path)
    t0 = time.perf_counter()
    h = N.vp()
    N.call("pxc_flat_create", ctx.handle, dim, 0, C.byref(h))
    for b in range(0, n, chunk):
        e = min(n, b + chunk)
        rows = d_vec[b:e].cpu().numpy()
        N.call("pxc_flat_sync", h, N.ptr(rows), None, None, b, e - b)
    truth = np.zeros((nq, k), dtype=np.uint64)
    td = np.zeros((nq, k), dtype=np.float32)
    tl = np.zeros(nq, dtype=np.uint32)
    N.call("pxc_flat_search", h, N.ptr(queries), nq, k, None, N.ptr(truth), N.ptr(td), N.ptr(tl))
    lib.pxc_flat_destroy(h)
    t_truth = time.perf_counter() - t0

    stream = torch.cuda.Stream(dev)  # an explicit stream: the library's work and the events share it
    torch.cuda.set_stream(stream)
    sp = stream.cuda_stream
    q_host = torch.from_numpy(queries).pin_memory()
    q_dev = q_host.to(dev)
    ids = torch.empty((nq, k), dtype=torch.int64, device=dev)
    dist = torch.empty((nq, k), dtype=torch.float32, device=dev)
    lens = torch.empty(nq, dtype=torch.int32, device=dev)

    def recall(got):
        hits = 0
        for q in range(nq):
            hits += len(set(truth[q].tolist()) & set(got[q].tolist()))
        return hits / (nq * k)

    def timed(nprobe, rerank, steps):
        for _ in range(2):
            idx.search_device(q_dev, k, nprobe, rerank, ids, dist, lens, sp)
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(steps):
            idx.search_device(q_dev, k, nprobe, rerank, ids, dist, lens, sp)
        b.record(stream)
        torch.cuda.synchronize(dev)
        return a.elapsed_time(b) / steps

    # diagnostics: the exact truth against a brute-force torch check, and the share of true
    # neighbours that lie in the probed lists at all (an upper bound on recall at any rerank)
    cent_t = torch.from_numpy(idx.parts()[0]).to(dev)
    list_of_t = torch.from_numpy(idx.parts()[2].astype(np.int64)).to(dev)
    qd = torch.from_numpy(queries).to(dev)
    chk = []
    for q in range(4):
        dq = ((d_vec - qd[q]) ** 2).sum(1)
        top = torch.topk(dq, k, largest=False).values.cpu().numpy()
        chk.append(bool(np.allclose(np.sort(top), np.sort(td[q]))))
    cd = torch.cdist(qd, cent_t) ** 2
    truth_t = torch.from_numpy(truth.astype(np.int64)).to(dev)
    truth_lists = list_of_t[truth_t]
    list_recall = {}
    for nprobe in (16, 32, 64, 256):
        probes = torch.topk(cd, nprobe, dim=1, largest=False).indices
        hit = (truth_lists.unsqueeze(2) == probes.unsqueeze(1)).any(2)
        list_recall[nprobe] = round(hit.float().mean().item(), 4)
    del cd, cent_t, list_of_t
    sweep = []
    for nprobe in IVF_NPROBES:
        for rerank in IVF_RERANKS:
            ms = timed(nprobe, rerank, 3)
            rc = recall(ids.cpu().numpy().view(np.uint64))
            sweep.append({"nprobe": nprobe, "rerank": rerank, "recall@10": round(rc, 4), "ms": round(ms, 3),
                          "qps": round(nq / (ms / 1e3))})
    ok = [c for c in sweep if c["recall@10"] >= 0.9]
    best = max(ok, key=lambda c: c["qps"]) if ok else max(sweep, key=lambda c: c["recall@10"])
    nprobe, rerank = best["nprobe"], best["rerank"]

    N.call("pxc_ctx_set_profiling", ctx.handle, 1)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)
    for _ in range(max(3, args.warmup)):
        idx.search_device(q_dev, k, nprobe, rerank, ids, dist, lens, sp)
    torch.cuda.synchronize(dev)
    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        pass
    sampler = ClockSampler(uuid)
    sampler.start()
    launches0 = lib.pxc_ctx_launch_count(ctx.handle)
    step_ms, scan_ms, scanned = [], [], 0
    for _ in range(args.steps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        idx.search_device(q_dev, k, nprobe, rerank, ids, dist, lens, sp)
        b.record(stream)
        torch.cuda.synchronize(dev)
        step_ms.append(a.elapsed_time(b))
        scan_ms.append(idx.last_scan_ms())
        scanned = idx.last_scanned()
    launches = lib.pxc_ctx_launch_count(ctx.handle) - launches0
    clocks = sampler.stop()
    rc = recall(ids.cpu().numpy().view(np.uint64))
    ms_per_step = sum(step_ms) / len(step_ms)
    # e2e: host queries in, host results out (the host entry point)
    e2e_steps = 5
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        idx.search_batch(queries, k, nprobe, rerank)
    e2e_s = (time.perf_counter() - t0) / e2e_steps
    if rank == 0:
        hbm, bf16, src = peaks()
        # algorithmic bytes of the scan launch: every probed code (16 B) and its id rank (4 B), plus the
        # shortlist's rows for the rerank. C4's rows and queries are integers in [0,255], so the library
        # re-ranks on its u8 copy of the rows (dim bytes per row, exact for dim <= 256).
        row_bytes = dim if dim <= 256 and dim % 16 == 0 else dim * 4
        bytes_launch = scanned * (m + 4) + (nq * max(rerank, k) * row_bytes if rerank else 0)
        bytes_q = bytes_launch / nq
        scan_mean = sum(scan_ms) / len(scan_ms)
        achieved = bytes_launch / (scan_mean / 1e3) / 1e9 if scan_mean > 0 else None
        line = {"metric": IVF_METRIC, "value": nq / (ms_per_step / 1e3), "unit": "queries/s", "n_gpus": world,
                "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": ms_per_step,
                "higher_is_better": True, "scaling": "replicas", "vs_baseline": None,
                "dtype": "u8 codes, u8 re-rank rows (exact integer distances)",
                "data": "synthetic",
                "config": {"workload": f"C4 IVF-PQ: {n:,} x 128 f32 (integers in [0,255], 4,096 blobs, sigma 20), "
                                       f"nlist {nlist}, m=16 x 8 bit, trained on the GPU from a {sample:,}-vector "
                                       "stride sample (25 iterations, k-means++), 10,000 queries, k=10",
                           "nprobe": nprobe, "rerank": rerank, "recall@10": round(rc, 4), "sweep": sweep,
                           "l2": "flushed (256 MiB write) between timed steps", "build_s": round(t_build, 2),
                           "generate_s": round(t_gen, 2), "truth_s": round(t_truth, 2),
                           "training": {k2: v for k2, v in report.items()},
                           "parallelism": "single GPU" if world == 1 else f"{world} independent replicas",
                           "truth_check": chk, "list_recall": list_recall},
                "clocks": clocks, "gpu_launches": int(launches),
                "e2e": {"value": nq / e2e_s, "unit": "queries/s", "h2d_bytes_per_step": nq * dim * 4,
                        "d2h_bytes_per_step": nq * k * 12 + nq * 4},
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                             "frac": achieved / hbm if achieved else None, "traffic": None,
                             "kernel": "ivf::scan_kernel (K5 + K6)", "kernel_ms": scan_mean,
                             "peak_source": src,
                             "algorithmic_bytes_per_query": bytes_q, "codes_scanned_per_query": scanned / nq}}
        line["config"]["parity_sample"] = ivfpq_parity_sample(idx, d_vec, queries, ids, nprobe, rerank, k)
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = ivfpq_cpu_baseline(idx, d_vec, queries, nprobe, rerank, args.cpu_seconds)
        print(json.dumps(line), flush=True)
    idx.close()
    ctx.close()


def run_ivfpq_sharded(args):
    """--workload ivfpq at N > 1: C4 with its lists split by rows across the ranks. Every rank trains the same
    parts from the index's stride sample (rows 0, 40, 80, ... of the 20M: IvfPqIndex::train's sample), holds
    its 20M/N rows and their lists, and one step is pxc_ivfpq_search_sharded: the same nprobe lists probed on
    every shard, each shard's own re-rank, one packed allgather, merge. Exact truth: the sharded flat search."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from proxima_b200 import _native as N
    from proxima_b200 import fixtures
    from proxima_b200.index import Context
    from proxima_b200.ivfpq import IvfPqIndex
    from proxima_b200.sharded import init_comm

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)
    n, dim, nlist, m, nq, k = args.ivf_n, 128, args.ivf_nlist, 16, 10_000, 10
    sample_n = min(500_000, n)
    stride = (n + sample_n - 1) // sample_n
    lo, hi = rank * n // world, (rank + 1) * n // world
    ctx = Context(local)
    lib = N.load()
    init_comm(ctx, timeout_ms=300_000)
    t0 = time.perf_counter()
    d_vec = torch.empty((hi - lo, dim), dtype=torch.float32, device=dev)
    chunk = 2_000_000
    for b in range(lo, hi, chunk):
        e = min(hi, b + chunk)
        d_vec[b - lo:e - lo].copy_(torch.from_numpy(fixtures.blobs_u8(e - b, dim, 4096, fixtures.C4_CENTRES,
                                                                      fixtures.C4_BASE, row_begin=b)))
    queries = fixtures.blobs_u8(nq, dim, 4096, fixtures.C4_CENTRES, fixtures.C4_QUERIES)
    sample = fixtures.blobs_u8_strided((n + stride - 1) // stride, stride, dim, 4096, fixtures.C4_CENTRES,
                                       fixtures.C4_BASE)
    t_gen = time.perf_counter() - t0
    t0 = time.perf_counter()
    trainer = IvfPqIndex(dim, nlist, m, context=ctx)
    trainer.set_store(sample)
    report = trainer.train(training_sample=len(sample), max_iterations=25, seed=0x1FF9C0D)
    cent, books, _, _ = trainer.parts()
    trainer.close()
    idx = IvfPqIndex(dim, len(cent), m, context=ctx)
    idx.from_parts(cent, books)
    idx.set_store_device(d_vec, ids=np.arange(lo, hi, dtype=np.uint64))
    idx.encode_all()
    torch.cuda.synchronize(dev)
    t_build = time.perf_counter() - t0
    # exact truth: the sharded flat search over the same rows
    t0 = time.perf_counter()
    fh = N.vp()
    N.call("pxc_flat_create", ctx.handle, dim, 0, C.byref(fh))
    for b in range(0, hi - lo, chunk):
        e = min(hi - lo, b + chunk)
        rows = d_vec[b:e].cpu().numpy()
        row_ids = np.arange(lo + b, lo + e, dtype=np.uint64)  # kept alive across the call
        N.call("pxc_flat_sync", fh, N.ptr(rows), N.ptr(row_ids), None, b, e - b)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    sp = stream.cuda_stream
    q_host = torch.from_numpy(queries).pin_memory()
    q_dev = q_host.to(dev)
    ids = torch.empty((nq, k), dtype=torch.int64, device=dev)
    dists = torch.empty((nq, k), dtype=torch.float32, device=dev)
    lens = torch.empty(nq, dtype=torch.int32, device=dev)
    N.call("pxc_flat_search_sharded", fh, q_dev.data_ptr(), nq, k, None, ids.data_ptr(), dists.data_ptr(),
           lens.data_ptr(), sp)
    truth = ids.cpu().numpy().view(np.uint64).copy()
    lib.pxc_flat_destroy(fh)
    t_truth = time.perf_counter() - t0

    def recall(got):
        return sum(len(set(truth[q].tolist()) & set(got[q].tolist())) for q in range(nq)) / (nq * k)

    def search(nprobe, rerank, q=q_dev):
        idx.search_sharded_device(q, k, nprobe, rerank, ids, dists, lens, sp)

    def timed(nprobe, rerank, steps):
        for _ in range(2):
            search(nprobe, rerank)
        dist.barrier()
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(steps):
            search(nprobe, rerank)
        b.record(stream)
        torch.cuda.synchronize(dev)
        t = torch.tensor([a.elapsed_time(b) / steps], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    sweep = []
    for nprobe in IVF_NPROBES:
        for rerank in IVF_RERANKS:
            ms = timed(nprobe, rerank, 3)
            rc = recall(ids.cpu().numpy().view(np.uint64))
            sweep.append({"nprobe": nprobe, "rerank": rerank, "recall@10": round(rc, 4), "ms": round(ms, 3),
                          "qps": round(nq / (ms / 1e3))})
    ok = [c for c in sweep if c["recall@10"] >= 0.9]
    best = max(ok, key=lambda c: c["qps"]) if ok else max(sweep, key=lambda c: c["recall@10"])
    nprobe, rerank = best["nprobe"], best["rerank"]
    N.call("pxc_ctx_set_profiling", ctx.handle, 1)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)
    for _ in range(max(3, args.warmup)):
        search(nprobe, rerank)
    torch.cuda.synchronize(dev)
    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        pass
    sampler = ClockSampler(uuid)
    sampler.start()
    launches0 = lib.pxc_ctx_launch_count(ctx.handle)
    dist.barrier()
    torch.cuda.synchronize(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for i in range(args.steps):
        flush.zero_()
        ev[i][0].record(stream)
        search(nprobe, rerank)
        ev[i][1].record(stream)
    torch.cuda.synchronize(dev)
    dist.barrier()
    launches = lib.pxc_ctx_launch_count(ctx.handle) - launches0
    total = torch.tensor([sum(a.elapsed_time(b) for a, b in ev)], dtype=torch.float64, device=dev)
    dist.all_reduce(total, op=dist.ReduceOp.MAX)
    ms_per_step = total.item() / args.steps
    clocks = sampler.stop()
    got_ids = ids.cpu().numpy().view(np.uint64).copy()
    got_d = dists.cpu().numpy().copy()
    rc = recall(got_ids)
    # e2e: host queries in, host results out
    out_ids = torch.empty((nq, k), dtype=torch.int64).pin_memory()
    out_d = torch.empty((nq, k), dtype=torch.float32).pin_memory()
    out_l = torch.empty(nq, dtype=torch.int32).pin_memory()
    dist.barrier()
    t0 = time.perf_counter()
    e2e_steps = 5
    for _ in range(e2e_steps):
        qd = q_host.to(dev, non_blocking=True)
        search(nprobe, rerank, qd)
        out_ids.copy_(ids, non_blocking=True)
        out_d.copy_(dists, non_blocking=True)
        out_l.copy_(lens, non_blocking=True)
        torch.cuda.synchronize(dev)
    e2e_s = torch.tensor([(time.perf_counter() - t0) / e2e_steps], dtype=torch.float64, device=dev)
    dist.all_reduce(e2e_s, op=dist.ReduceOp.MAX)
    # parity: every rank answers the sampled queries on its shard with the oracle; rank 0 merges them by
    # (total_cmp, id) and compares with the GPU's merged answer
    from oracle import pxo

    samp = np.arange(0, nq, nq // 32)[:32]
    _, _, list_of, codes = idx.parts()
    vec = d_vec.cpu().numpy() if rerank else None
    ri, rd, rl = pxo.ivfpq_search(vec, cent, books, m, list_of, codes, queries[samp], k, nprobe, rerank,
                                  ids=np.arange(lo, hi, dtype=np.uint64))
    g = [torch.empty((len(samp), k), dtype=torch.int64, device=dev) for _ in range(world)]
    gd = [torch.empty((len(samp), k), dtype=torch.float32, device=dev) for _ in range(world)]
    gl = [torch.empty(len(samp), dtype=torch.int32, device=dev) for _ in range(world)]
    dist.all_gather(g, torch.from_numpy(ri.view(np.int64)).to(dev))
    dist.all_gather(gd, torch.from_numpy(rd).to(dev))
    dist.all_gather(gl, torch.from_numpy(rl.view(np.int32)).to(dev))
    idx.close()
    ctx.close()
    if rank == 0:
        same = 0
        parts = [(g[r].cpu().numpy().view(np.uint64), gd[r].cpu().numpy(), gl[r].cpu().numpy()) for r in range(world)]
        for i, q in enumerate(samp):
            cand = []
            for pi, pd, pl in parts:
                for j in range(int(pl[i])):
                    bb = int(pd[i, j:j + 1].view(np.int32)[0])
                    cand.append((bb ^ 0x7FFFFFFF if bb < 0 else bb, int(pi[i, j]), pd[i, j]))
            cand.sort(key=lambda c: (c[0], c[1]))
            want_i = [c[1] for c in cand[:k]]
            want_d = np.array([c[2] for c in cand[:k]], np.float32)
            same += int(want_i == [int(x) for x in got_ids[q, :len(want_i)]] and
                        np.array_equal(want_d.view(np.uint32), got_d[q, :len(want_i)].view(np.uint32)))
        line = {"metric": IVF_METRIC, "value": nq / (ms_per_step / 1e3), "unit": "queries/s", "n_gpus": world,
                "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": ms_per_step,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "u8 codes, u8 re-rank rows (exact integer distances)", "data": "synthetic",
                "config": {"workload": f"C4 IVF-PQ: {n:,} x 128 f32 (integers in [0,255], 4,096 blobs, sigma 20), "
                                       f"nlist {nlist}, m=16 x 8 bit, lists split by rows over {world} GPUs, "
                                       "10,000 queries, k=10", "nprobe": nprobe, "rerank": rerank,
                           "recall@10": round(rc, 4), "sweep": sweep, "build_s": round(t_build, 2),
                           "generate_s": round(t_gen, 2), "truth_s": round(t_truth, 2),
                           "training": report, "rows_per_gpu": hi - lo,
                           "parallelism": f"row shards x{world}; every shard probes the same lists and re-ranks "
                                          "its own shortlist; one packed allgather + merge (library communicator)",
                           "parity_sample": {"queries": len(samp), "identical_ids_and_distance_bits": same,
                                             "against": "oracle search_prepared per shard, merged by (total_cmp, id)"}},
                "clocks": clocks, "gpu_launches": int(launches),
                "e2e": {"value": nq / e2e_s.item(), "unit": "queries/s", "h2d_bytes_per_step": nq * dim * 4,
                        "d2h_bytes_per_step": nq * k * 12 + nq * 4}}
        print(json.dumps(line), flush=True)
    dist.barrier()
    dist.destroy_process_group()


def _csr(list_of, nlist):
    order = np.argsort(list_of, kind="stable").astype(np.uint32)
    order = order[list_of[order] != 0xFFFFFFFF]
    off = np.zeros(nlist + 1, dtype=np.uint64)
    np.cumsum(np.bincount(list_of[order], minlength=nlist), out=off[1:])
    return off.astype(np.uint32), order


def ivfpq_parity_sample(idx, d_vec, queries, d_ids, nprobe, rerank, k, count=64):
    """The GPU's answers for the first queries against the oracle port on the same full-size parts."""
    from oracle import pxo

    cent, books, list_of, codes = idx.parts()
    off, order = _csr(list_of, len(cent))
    vec = d_vec.cpu().numpy() if rerank else None
    ref_ids, _, ref_len = pxo.ivfpq_search_csr(vec, cent, books, idx.m, off, order, codes, queries[:count], k,
                                               nprobe, rerank=rerank)
    got = d_ids[:count].cpu().numpy().view(np.uint64)
    same = sum(int(np.array_equal(got[q, :ref_len[q]], ref_ids[q, :ref_len[q]])) for q in range(count))
    return {"queries": count, "identical_ids": same}


def ivfpq_cpu_baseline(idx, d_vec, queries, nprobe, rerank, seconds):
    """The oracle port of search_prepared on all host cores, on a query sample, against the same parts
    (lists built once, as the index holds them)."""
    from oracle import pxo

    threads = os.cpu_count() or 1
    cent, books, list_of, codes = idx.parts()
    off, order = _csr(list_of, len(cent))
    vec = d_vec.cpu().numpy() if rerank else None
    batch = max(threads, 16)
    pxo.ivfpq_search_csr(vec, cent, books, idx.m, off, order, codes, queries[:batch], 10, nprobe,
                         rerank=rerank, nthreads=threads)
    done, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds and done + batch <= len(queries):
        pxo.ivfpq_search_csr(vec, cent, books, idx.m, off, order, codes,
                             queries[done:done + batch], 10, nprobe, rerank=rerank, nthreads=threads)
        done += batch
    el = time.perf_counter() - t0
    return {"value": done / el, "unit": "queries/s", "cores": threads, "kind": "port",
            "sample": f"{done} of the 10,000 queries (nprobe {nprobe}, rerank {rerank}) against the same trained "
                      f"index ({el:.1f} s; C++ restatement of search_prepared over the index's lists, one query "
                      "per thread)"}


SQ_METRIC = "queries/s: SQ int8 filtered scan (768-d cosine, year >= 2027, over-fetch 100 on int8, exact top-10)"


def run_sq(args):
    """--workload sq: C5 per GPU. Each GPU holds one 6.25M-row shard of the 50M x 768 corpus (the 8-way
    split of C5), its I8 codes under a per-dimension quantizer trained over every shard, and the year
    column. One step = the 4,096-query batch: filter compaction, int8 over-fetch of 100 on the tensor cores,
    exact fp32 re-rank to 10 on the shard; with N GPUs an NCCL allgather of the 10 per query and the
    (total_cmp, id) merge."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    from proxima_b200 import _native as N
    from proxima_b200 import fixtures
    from proxima_b200.core import Metric
    from proxima_b200.index import Context
    from proxima_b200.sq import CodeType, IntRange, RangeMode, ScalarQuantizer, SqIndex, combine_ranges, ranges_device

    per, dim, nq, k, F = args.sq_n, 768, 4096, 10, 100
    lo = rank * per
    ctx = Context(local)
    lib = N.load()
    keep_host = world == 1 and rank == 0
    t0 = time.perf_counter()
    d_vec = torch.empty((per, dim), dtype=torch.float32, device=dev)
    host = np.empty((per, dim), dtype=np.float32) if keep_host else None
    chunk = 500_000
    for b in range(0, per, chunk):
        e = min(per, b + chunk)
        part = fixtures.sphere_blobs(e - b, dim, 10_000, fixtures.C5_CENTRES, fixtures.C5_BASE, 0.03, row_begin=lo + b)
        d_vec[b:e].copy_(torch.from_numpy(part))
        if host is not None:
            host[b:e] = part
    years = fixtures.uniform_int(per, fixtures.C5_YEARS, 2000, 30, row_begin=lo)
    queries = fixtures.sphere_blobs(nq, dim, 10_000, fixtures.C5_CENTRES, fixtures.C5_QUERIES, 0.03)
    t_gen = time.perf_counter() - t0

    t0 = time.perf_counter()
    # quantizer over all shards: per-shard ranges folded in rank order (== one pass over the corpus)
    rlo, rhi = ranges_device(d_vec, dim, RangeMode.PER_DIMENSION, ctx)
    if world > 1:
        t = torch.from_numpy(np.stack([rlo, rhi])).to(dev)
        g = torch.empty((world, 2, dim), dtype=torch.float32, device=dev)
        dist.all_gather_into_tensor(g, t)
        g = g.cpu().numpy()
        lows, highs = [g[r, 0] for r in range(world)], [g[r, 1] for r in range(world)]
    else:
        lows, highs = [rlo], [rhi]
    mn, sc, inv = combine_ranges(lows, highs)
    idx = SqIndex(dim, Metric.COSINE, ctx)
    idx.set_store(d_vec, ids=np.arange(lo, lo + per, dtype=np.uint64))
    idx.set_quantizer(ScalarQuantizer(dim, RangeMode.PER_DIMENSION, CodeType.I8, mn, sc, inv, ctx))
    idx.set_column(0, years)
    del d_vec
    torch.cuda.empty_cache()
    torch.cuda.synchronize(dev)
    t_build = time.perf_counter() - t0
    flt = [IntRange(0, lo=2027)]

    stream = torch.cuda.Stream(dev)  # an explicit stream: the library's work and the events share it
    torch.cuda.set_stream(stream)
    sp = stream.cuda_stream
    q_host = torch.from_numpy(queries).pin_memory()
    q_dev = q_host.to(dev)
    ids = torch.empty((nq, k), dtype=torch.int64, device=dev)
    dists = torch.empty((nq, k), dtype=torch.float32, device=dev)
    lens = torch.empty(nq, dtype=torch.int32, device=dev)
    if world > 1:
        from proxima_b200.sharded import init_comm

        init_comm(ctx, timeout_ms=120_000)
        m_ids = torch.empty((nq, k), dtype=torch.int64, device=dev)
        m_d = torch.empty((nq, k), dtype=torch.float32, device=dev)
        m_l = torch.empty(nq, dtype=torch.int32, device=dev)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)  # 256 MiB > 126 MB L2

    def step(q_ptr):
        N.call("pxc_sq_search_device", idx.handle, q_ptr, nq, k, F, None, *idx._ranges(flt), ids.data_ptr(),
               dists.data_ptr(), lens.data_ptr(), sp)
        if world > 1:  # one packed allgather over the library's communicator, then the merge
            N.call("pxc_topk_exchange", ctx.handle, ids.data_ptr(), dists.data_ptr(), lens.data_ptr(), nq, k, k,
                   m_ids.data_ptr(), m_d.data_ptr(), m_l.data_ptr(), sp)

    N.call("pxc_ctx_set_profiling", ctx.handle, 1)
    for _ in range(max(3, args.warmup)):
        step(q_dev.data_ptr())
    torch.cuda.synchronize(dev)
    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        pass
    sampler = ClockSampler(uuid)
    sampler.start()
    launches0 = lib.pxc_ctx_launch_count(ctx.handle)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    scan_ms = []
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    for i in range(args.steps):
        flush.zero_()  # evict L2 between timed steps (not timed)
        ev[i][0].record(stream)
        step(q_dev.data_ptr())
        ev[i][1].record(stream)
        scan_ms.append(idx.last_scan_ms())
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    launches = lib.pxc_ctx_launch_count(ctx.handle) - launches0
    step_ms = [a.elapsed_time(b) for a, b in ev]
    total_ms = torch.tensor([sum(step_ms)], dtype=torch.float64, device=dev)
    scan_mean = torch.tensor([sum(scan_ms) / len(scan_ms)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(total_ms, op=dist.ReduceOp.MAX)
        dist.all_reduce(scan_mean, op=dist.ReduceOp.MAX)
    ms_per_step = total_ms.item() / args.steps
    clocks = sampler.stop()
    accepted = idx.last_accepted()
    fallback = idx.last_fallback()
    retried = idx.last_retried()
    res_ids = (m_ids if world > 1 else ids).cpu().numpy().view(np.uint64)

    # ---- e2e: host queries in, host results out, every step ----
    out_ids = torch.empty((nq, k), dtype=torch.int64).pin_memory()
    out_d = torch.empty((nq, k), dtype=torch.float32).pin_memory()
    out_l = torch.empty(nq, dtype=torch.int32).pin_memory()
    e2e_steps = max(3, min(args.steps, 20))

    def e2e_step():
        if world == 1:
            rr, nr = idx._ranges(flt)
            N.call("pxc_sq_search", idx.handle, q_host.data_ptr(), nq, k, F, None, rr, nr, out_ids.data_ptr(),
                   out_d.data_ptr(), out_l.data_ptr())
        else:
            qd = q_host.to(dev, non_blocking=True)
            step(qd.data_ptr())
            out_ids.copy_(m_ids, non_blocking=True)
            out_d.copy_(m_d, non_blocking=True)
            out_l.copy_(m_l, non_blocking=True)
            torch.cuda.synchronize(dev)

    for _ in range(2):
        e2e_step()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    torch.cuda.synchronize(dev)
    e2e_s = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(e2e_s, op=dist.ReduceOp.MAX)
    e2e_qps = nq * e2e_steps / e2e_s.item()

    if rank == 0:
        hbm, bf16, src = peaks()
        peak_tops = 2.0 * bf16
        ops = 2.0 * accepted * dim * nq  # int8 multiply-adds of one step on the accepted rows of this shard
        achieved = ops / (scan_mean.item() / 1e3) / 1e12 if scan_mean.item() > 0 else None
        line = {"metric": SQ_METRIC, "value": nq / (ms_per_step / 1e3), "unit": "queries/s", "n_gpus": world,
                "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": ms_per_step,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "s8 x s8 -> s32, f32 re-rank",
                "data": "synthetic",
                "config": {"workload": f"C5 per GPU: {per:,} x 768 f32 rows of the 50M-row corpus (10,000 unit-sphere "
                                       "blobs, sigma 0.03, L2-normalised), per-dimension I8 SQ trained over all "
                                       "shards, year uniform in [2000, 2029], filter year >= 2027, 4,096 queries, "
                                       "over-fetch 100 on int8, exact cosine re-rank to k=10",
                           "rows_per_gpu": per, "accepted_rows_per_gpu": accepted, "retried_queries": retried,
                           "fallback_queries": fallback,
                           "l2": "flushed (256 MiB write) between timed steps; codes 4.8 GB per GPU",
                           "generate_s": round(t_gen, 2), "build_s": round(t_build, 2),
                           "parallelism": "single GPU" if world == 1 else
                           f"row shards x{world}; the library's NCCL communicator: one packed allgather, merge"},
                "clocks": clocks, "gpu_launches": int(launches),
                "e2e": {"value": e2e_qps, "unit": "queries/s", "h2d_bytes_per_step": nq * dim * 4,
                        "d2h_bytes_per_step": nq * k * 12 + nq * 4},
                "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_tops, "unit": "TOPS",
                             "frac": achieved / peak_tops if achieved else None, "traffic": None,
                             "kernel": "sq_scan_kernel (K12, DENSE prefix + THRESH) with the over-fetch selection",
                             "kernel_ms": scan_mean.item(), "peak_source": f"2 x dense bf16 {src} = dense int8 rate",
                             "algorithmic_ops_per_launch": ops}}
        if keep_host and not args.no_cpu_baseline:
            line["cpu_baseline"] = sq_cpu_baseline(host, years, queries, res_ids, k, args.cpu_seconds)
        print(json.dumps(line), flush=True)
    idx.close()
    ctx.close()
    if world > 1:
        dist.destroy_process_group()


def sq_cpu_baseline(host, years, queries, gpu_ids, k, seconds):
    """The reference's CPU answer to the same query: FlatIndex::search with the filter (the oracle port,
    one query per thread), on a bounded query sample over the full shard; its ids are compared with the
    GPU's, which must be identical (the re-rank is exact)."""
    from oracle import pxo

    threads = os.cpu_count() or 1
    acc = years >= 2027
    words = np.zeros((len(acc) + 63) // 64, dtype=np.uint64)
    idx = np.nonzero(acc)[0].astype(np.uint64)
    np.bitwise_or.at(words, (idx >> np.uint64(6)).astype(np.int64), np.left_shift(np.uint64(1), idx & np.uint64(63)))
    batch = max(threads, 8)
    done, same, t0 = 0, 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds and done + batch <= len(queries):
        ref_ids, _, ref_len = pxo.flat_search(host, queries[done:done + batch], k, pxo.COSINE, bitmap=words,
                                              nthreads=threads)
        for i in range(batch):
            same += int(np.array_equal(gpu_ids[done + i, :ref_len[i]], ref_ids[i, :ref_len[i]]))
        done += batch
    el = time.perf_counter() - t0
    return {"value": done / el if el > 0 else None, "unit": "queries/s", "cores": threads, "kind": "port",
            "sample": f"{done} of the 4,096 queries, exact filtered FlatIndex::search (cosine, year >= 2027) over the "
                      f"full {host.shape[0]:,}-row shard ({el:.1f} s, C++ oracle, one query per thread)",
            "parity": {"queries": done, "identical_ids": same}}


def flat_rows(args, lo: int, hi: int) -> np.ndarray:
    from proxima_b200 import fixtures

    gen = fixtures.blobs_u8 if args.data == "u8" else fixtures.blobs_f32
    return gen(hi - lo, args.dim, 1024, fixtures.C2_CENTRES, fixtures.C2_BASE, row_begin=lo)


def flat_queries(args, nq: int) -> np.ndarray:
    from proxima_b200 import fixtures

    gen = fixtures.blobs_u8 if args.data == "u8" else fixtures.blobs_f32
    return gen(nq, args.dim, 1024, fixtures.C2_CENTRES, fixtures.C2_QUERIES)


SNAP_METRIC = "GB/s: IVF-PQ snapshot load (decode, snapshot.rs) of a 1M x 128, nlist 4096, m=16 index, host image -> device index"


def run_snapshot(args):
    """--workload snapshot: an IVF-PQ index (1M x 128 f32 integer rows, nlist 4096, m=16) trained on the GPU
    (untimed) and saved once; one step = pxc_ivfpq_snapshot_load of the host image into a new device index
    (header, checksum, sections, arrays to HBM, id ranks, inverted lists), timed on the host around the call.
    Also reported: the save (device index -> host image) and the device CRC-32C kernel on the vectors."""
    import torch

    from oracle import pxo
    from proxima_b200 import _native as N
    from proxima_b200 import fixtures
    from proxima_b200 import snapshot as S
    from proxima_b200.index import Context
    from proxima_b200.ivfpq import IvfPqIndex

    local = int(os.environ.get("LOCAL_RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    n, dim, nlist, m = 1_000_000, 128, 4096, 16
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ctx = Context(local)
    lib = N.load()
    d_vec = torch.from_numpy(fixtures.blobs_u8(n, dim, 4096, fixtures.C4_CENTRES, fixtures.C4_BASE)).to(dev)
    idx = IvfPqIndex(dim, nlist, m, context=ctx)
    ids = np.arange(n, dtype=np.uint64) * 2 + 1
    live = np.ones(n, np.uint8)
    live[::97] = 0  # some removed slots
    idx.set_store_device(d_vec, ids=ids, live=live)
    idx.train(training_sample=200_000, max_iterations=10, seed=0x1FF9C0D)
    cfg = S.IvfPqConfig(idx.nlist, m, nprobe=32, rerank=100)
    image = np.frombuffer(S.save_ivfpq(idx, cfg), dtype=np.uint8)
    nbytes = len(image)

    def load_once(img):
        h = N.vp()
        info = N.PxcSnapshotInfo()
        N.call("pxc_ivfpq_snapshot_load", ctx.handle, img.ctypes.data, len(img), C.byref(h), C.byref(info))
        return h

    for _ in range(max(3, args.warmup)):
        lib.pxc_ivfpq_destroy(load_once(image))
    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        pass
    sampler = ClockSampler(uuid)
    sampler.start()
    launches0 = lib.pxc_ctx_launch_count(ctx.handle)
    load_s = []
    for _ in range(args.steps):
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        h = load_once(image)
        load_s.append(time.perf_counter() - t0)
        lib.pxc_ivfpq_destroy(h)
    launches = (lib.pxc_ctx_launch_count(ctx.handle) - launches0) // max(1, args.steps)
    clocks = sampler.stop()
    # the same load from a pinned copy of the image
    pinned = torch.from_numpy(image.copy()).pin_memory().numpy()
    lib.pxc_ivfpq_destroy(load_once(pinned))
    pin_s = []
    for _ in range(max(3, args.steps // 2)):
        t0 = time.perf_counter()
        h = load_once(pinned)
        pin_s.append(time.perf_counter() - t0)
        lib.pxc_ivfpq_destroy(h)
    # save
    save_s = []
    for _ in range(3):
        t0 = time.perf_counter()
        again = S.save_ivfpq(idx, cfg)
        save_s.append(time.perf_counter() - t0)
    # the device CRC kernel on the vectors (CUDA events on the launching stream)
    stream = torch.cuda.Stream(dev)
    out = C.c_uint32()
    vec_bytes = d_vec.numel() * 4
    for _ in range(3):
        N.call("pxc_crc32c_device", ctx.handle, d_vec.data_ptr(), vec_bytes, C.byref(out), stream.cuda_stream)
    crc_ms = []
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)
    for _ in range(5):
        flush.zero_()
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        N.call("pxc_crc32c_device", ctx.handle, d_vec.data_ptr(), vec_bytes, C.byref(out), stream.cuda_stream)
        b.record(stream)
        torch.cuda.synchronize(dev)
        crc_ms.append(a.elapsed_time(b))
    crc_host = pxo.crc32c(d_vec.cpu().numpy().tobytes())
    # parity: the loaded index re-saves to the same bytes, answers as the saved one, and the image's
    # checksum (device-computed) verifies on the host
    idx2, info = S.load_ivfpq(image, ctx, with_metadata=False)
    resaved = np.frombuffer(S.save_ivfpq(idx2, cfg), dtype=np.uint8)
    qs = fixtures.blobs_u8(200, dim, 4096, fixtures.C4_CENTRES, fixtures.C4_QUERIES)
    r1, r2 = idx.search_batch(qs, 10, 32, 100), idx2.search_batch(qs, 10, 32, 100)
    same_search = all(np.array_equal(x.view(np.uint8), y.view(np.uint8)) for x, y in zip(r1, r2))
    peek_ok = S.peek(image).len == int(live.sum())
    parity = {"resave_identical": bool(np.array_equal(resaved, image)), "search_identical_200q": bool(same_search),
              "host_checksum_verifies": bool(peek_ok), "device_crc_equals_oracle": bool(out.value == crc_host),
              "save_deterministic": again == image.tobytes()}
    idx2.close()
    mean_load = sum(load_s) / len(load_s)
    hbm, bf16, src = peaks()
    crc_mean = sum(crc_ms) / len(crc_ms)
    achieved = vec_bytes / (crc_mean / 1e3) / 1e9
    line = {"metric": SNAP_METRIC, "value": nbytes / mean_load / 1e9, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": mean_load * 1e3,
            "higher_is_better": True, "scaling": "replicas", "vs_baseline": None, "dtype": "u8 (bytes)",
            "data": "synthetic",
            "config": {"workload": f"IVF-PQ snapshot of {n:,} x {dim} f32 rows (C4 blobs, integers), "
                                   f"{int(live.sum()):,} live, nlist {idx.nlist}, m={m}, metadata empty; "
                                   f"image {nbytes:,} bytes in pageable host memory",
                       "image_bytes": nbytes, "pinned_image_gb_s": nbytes / (sum(pin_s) / len(pin_s)) / 1e9,
                       "save_gb_s": nbytes / (sum(save_s) / len(save_s)) / 1e9,
                       "l2": "inputs (the host image) larger than L2; the CRC kernel's vectors flushed between runs",
                       "parity": parity, "parallelism": "single GPU"},
            "clocks": clocks, "gpu_launches": int(launches),
            "e2e": {"value": nbytes / mean_load / 1e9, "unit": "GB/s", "h2d_bytes_per_step": nbytes,
                    "d2h_bytes_per_step": 32},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                         "traffic": None, "kernel": "crc::crc_step_kernel + crc_finish_kernel (device CRC-32C)",
                         "kernel_ms": crc_mean, "peak_source": src, "algorithmic_bytes_per_launch": vec_bytes}}
    if not args.no_cpu_baseline:
        t0 = time.perf_counter()
        dec = pxo.snapshot_decode_ivfpq(image.tobytes())
        cpu_s = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": nbytes / cpu_s / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
                                "sample": "the whole image: the oracle's decode (byte-at-a-time CRC-32C as crc.rs, "
                                          "sections, from_parts checks), one pass",
                                "parts_equal": bool(np.array_equal(dec["codes"].reshape(-1, m), idx.parts()[3]))}
    print(json.dumps(line), flush=True)
    idx.close()
    ctx.close()


def run_extras(args) -> dict:
    """Sub-records of the other configurations, each from its own bench.py run (fresh process, the same GPU):
    C2 at k=100, real-valued C2 (euclidean and cosine: the f16 tensor-core screen), C3, C4 and C5."""
    runs = {
        "c2_k100": ["--workload", "flat", "--k", "100"],
        "c2_real_euclidean": ["--workload", "flat", "--data", "real"],
        "c2_real_cosine": ["--workload", "flat", "--data", "real", "--metric", "cosine"],
        "c3_kmeans": ["--workload", "kmeans"],
        "c4_ivfpq": ["--workload", "ivfpq"],
        "c5_sq": ["--workload", "sq"],
        "c4_snapshot": ["--workload", "snapshot"],
    }
    out = {}
    for name, extra in runs.items():
        cmd = [sys.executable, str(ROOT / "bench.py"), "--gpus", "1", "--steps", str(args.extras_steps),
               "--warmup", "3", "--no-extras", "--cpu-seconds", "6", *extra]
        t0 = time.perf_counter()
        try:
            proc = subprocess.run(cmd, capture_output=True, text=True, timeout=900,
                                  env=dict(os.environ, RANK="0", LOCAL_RANK=os.environ.get("LOCAL_RANK", "0"),
                                           WORLD_SIZE="1"))
            line = None
            for ln in proc.stdout.splitlines():
                if ln.startswith("{"):
                    line = json.loads(ln)
            if line is None:
                line = {"error": f"exit {proc.returncode}: {proc.stderr.strip().splitlines()[-1:]}"}
        except subprocess.TimeoutExpired:
            line = {"error": "timed out after 900 s"}
        line["wall_s"] = round(time.perf_counter() - t0, 1)
        out[name] = line
    return out


def main():
    args = parse()
    if args.workload == "sq":
        run_sq(args)
        return
    if args.workload == "ivfpq":
        if int(os.environ.get("WORLD_SIZE", "1")) > 1 and args.impl != "reference":
            run_ivfpq_sharded(args)
        else:
            run_ivfpq(args)
        return
    if args.workload == "kmeans":
        run_kmeans(args)
        return
    if args.workload == "snapshot":
        run_snapshot(args)
        return
    if args.impl == "reference":
        run_reference(args)
        return
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)

    from proxima_b200 import _native as N
    from proxima_b200.core import Metric, VectorSpace
    from proxima_b200.index import Context
    from proxima_b200.sharded import init_comm

    n, dim, k = args.n, args.dim, args.k
    metric = Metric.COSINE if args.metric == "cosine" else Metric.EUCLIDEAN
    space = VectorSpace(dim, metric)
    # Weak scaling keeps each GPU's scan at (--nq queries x --n rows): the rows are split N ways and the
    # query batch grows N-fold (the first N x --nq queries of the same seeded stream).
    weak = world > 1 and args.flat_scaling == "weak"
    nq = args.nq * world if weak else args.nq
    lo, hi = rank * n // world, (rank + 1) * n // world
    shard = space.prepare_batch(flat_rows(args, lo, hi))
    queries = space.prepare_batch(flat_queries(args, nq))

    ctx = Context(local)
    lib = N.load()
    if world > 1:
        init_comm(ctx, timeout_ms=120_000)  # the library's NCCL communicator over the ranks
    h = N.vp()
    N.call("pxc_flat_create", ctx.handle, dim, int(metric), C.byref(h))
    gids = np.arange(lo, hi, dtype=np.uint64)
    N.call("pxc_flat_sync", h, N.ptr(shard), N.ptr(gids), None, 0, hi - lo)
    path = lib.pxc_flat_path(h)

    stream = torch.cuda.Stream(dev)  # an explicit stream: the library's work and the events share it
    torch.cuda.set_stream(stream)
    sp = stream.cuda_stream
    q_host = torch.from_numpy(queries).pin_memory()
    q_dev = q_host.to(dev)
    # weak scaling: each rank owns its slice of the batch and receives only that slice's candidates
    own_b, own_n = C.c_uint32(0), C.c_uint32(nq)
    if weak:
        lib.pxc_ctx_owned_range(ctx.handle, nq, C.byref(own_b), C.byref(own_n))
    own_b, own_n = own_b.value, own_n.value
    ids = torch.empty((own_n, k), dtype=torch.int64, device=dev)
    dists = torch.empty((own_n, k), dtype=torch.float32, device=dev)
    lens = torch.empty(own_n, dtype=torch.int32, device=dev)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)  # 256 MiB > 126 MB L2
    entry = ("pxc_flat_search_sharded_owned" if weak else "pxc_flat_search_sharded") if world > 1 \
        else "pxc_flat_search_device"

    def step(q_ptr):
        # N > 1: local search, then the candidate exchange and merge inside the library (weak: to each query's
        # owner, grouped NCCL sends; strong: one packed allgather to every rank)
        N.call(entry, h, q_ptr, nq, k, None, ids.data_ptr(), dists.data_ptr(), lens.data_ptr(), sp)

    N.call("pxc_ctx_set_profiling", ctx.handle, 1)
    for _ in range(max(3, args.warmup)):
        step(q_dev.data_ptr())
    torch.cuda.synchronize(dev)

    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        pass
    sampler = ClockSampler(uuid)
    sampler.start()
    launches0 = lib.pxc_ctx_launch_count(ctx.handle)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    scan_ms, redone = [], 0
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    for i in range(args.steps):
        flush.zero_()  # evict L2 between timed steps (not timed)
        ev[i][0].record(stream)
        step(q_dev.data_ptr())
        ev[i][1].record(stream)
        scan_ms.append(lib.pxc_flat_last_scan_ms(h))
        redone += lib.pxc_flat_last_redone(h)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    launches = lib.pxc_ctx_launch_count(ctx.handle) - launches0
    step_ms = [a.elapsed_time(b) for a, b in ev]
    total_ms = torch.tensor([sum(step_ms)], dtype=torch.float64, device=dev)
    scan_mean = torch.tensor([sum(scan_ms) / len(scan_ms)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(total_ms, op=dist.ReduceOp.MAX)
        dist.all_reduce(scan_mean, op=dist.ReduceOp.MAX)
    ms_per_step = total_ms.item() / args.steps
    clocks = sampler.stop()
    res_ids = ids.cpu().numpy().view(np.uint64)
    res_d = dists.cpu().numpy()

    # ---- e2e: host buffers in, host results out, every step ----
    out_ids = torch.empty((own_n, k), dtype=torch.int64).pin_memory()
    out_d = torch.empty((own_n, k), dtype=torch.float32).pin_memory()
    out_l = torch.empty(own_n, dtype=torch.int32).pin_memory()
    h2d = nq * dim * 4
    d2h = own_n * k * 12 + own_n * 4
    e2e_steps = max(3, min(args.steps, 50))

    def e2e_step():
        if world == 1:
            N.call("pxc_flat_search", h, q_host.data_ptr(), nq, k, None, out_ids.data_ptr(), out_d.data_ptr(),
                   out_l.data_ptr())
        else:
            qd = q_host.to(dev, non_blocking=True)
            step(qd.data_ptr())
            out_ids.copy_(ids, non_blocking=True)
            out_d.copy_(dists, non_blocking=True)
            out_l.copy_(lens, non_blocking=True)
            torch.cuda.synchronize(dev)

    for _ in range(2):
        e2e_step()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    torch.cuda.synchronize(dev)
    e2e_s = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(e2e_s, op=dist.ReduceOp.MAX)
    e2e_qps = nq * e2e_steps / e2e_s.item()
    lib.pxc_flat_destroy(h)
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()

    if rank != 0:
        return
    hbm, bf16, src = peaks()
    # K1 is u8 x u8 -> s32 on tcgen05 (kind::i8): dense int8 = 2 x dense bf16. K2's screen is
    # f16 x f16 -> f32 (kind::f16): the dense bf16/f16 rate.
    peak = 2.0 * bf16 if path == 1 else bf16 if path == 2 else None
    ops = 2.0 * (hi - lo) * dim * nq  # per launch of the scan kernel on this rank
    achieved = ops / (scan_mean.item() / 1e3) / 1e12 if scan_mean.item() > 0 else None
    traffic, traffic_src = None, None
    tf = ROOT / "profiles" / "traffic.json"
    if tf.exists() and world == 1 and path == 1 and k <= 32 and n == 1_000_000 and nq == 10_000:
        rec = json.loads(tf.read_text())
        t = rec.get("flat_u8_kernel_c2_bytes_per_launch")
        if t and rec.get("kernel_source_sha256") == k1_source_hash():
            traffic, traffic_src = t, "ncu dram__bytes_read.sum + dram__bytes_write.sum of this launch shape " \
                                      "and this kernel source (profiles/flat_u8_kernel_c2.md)"
        elif t:
            traffic_src = "not reported: the K1 source changed since the ncu capture in profiles/traffic.json"
    kernel = {1: ("flat_scan_kernel<KT, U8Scan> (K1)" if k <= 32 else
                  "K1 sample pass (flat_scan_kernel<16, U8Scan>, own lists) + K1 collect launch "
                  "(flat_scan_kernel<1, U8Scan, collect>) + candidate merge, timed together"),
              2: "flat_scan_kernel<32, F16Scan> (K2 screen)"}.get(path, "dist_chunk_kernel + select (K1g)")
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak,
                "unit": "TOPS" if path == 1 else "TFLOP/s",
                "frac": (achieved / peak) if (achieved and peak) else None, "traffic": traffic,
                "traffic_source": traffic_src, "kernel": kernel, "kernel_ms": scan_mean.item(),
                "peak_source": (f"2 x dense bf16 {src} = dense int8 rate" if path == 1 else
                                f"dense bf16 {src} = dense f16 rate"),
                "algorithmic_ops_per_launch": ops}
    data_desc = ("integers in [0,255], 1,024 blobs, sigma 20" if args.data == "u8"
                 else "real-valued: the same 1,024 blobs, sigma 20, unrounded")
    workload = (f"C2 exact flat search: {n:,} x {dim} f32 ({data_desc}), {nq:,} queries, k={k}, {args.metric}")
    scan_path = {1: ("tensor-core u8 (exact)" if k <= 32 else
                     "tensor-core u8: a sample pass bounds each query's k-th distance, one collect launch keeps "
                     "every row within the bound, exact top k of those (queries whose candidates overflow: "
                     "row groups, merged and proven exact)"),
                 2: "tensor-core f16 screen of 32 per query, exact f32 re-rank, proven per query"}.get(
        path, "fp32 reference order")
    line = {"metric": METRIC.replace("k=10", f"k={k}").replace("euclidean", args.metric) +
            ("" if args.data == "u8" else ", real-valued rows"),
            "value": nq / (ms_per_step / 1e3), "unit": "queries/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "weak" if weak else "strong", "vs_baseline": None,
            "dtype": {1: "u8", 2: "f16 screen + f32 re-rank"}.get(path, "f32"),
            "data": "synthetic",
            "config": dict(CONFIG, workload=workload, n=n, queries=nq, k=k, metric=args.metric, rows=args.data,
                           l2="flushed (256 MiB write) between timed steps",
                           parallelism=(f"row shards x{world}; the library's NCCL communicator: "
                                        + (f"each rank owns {args.nq:,} queries of the batch and receives only "
                                           f"their k candidates from every rank (grouped sends), device merge; "
                                           f"each GPU scans {nq:,} queries x {n // world:,} rows = "
                                           f"{args.nq:,} x {n:,} query-row pairs as on one GPU" if weak else
                                           "one packed allgather of k candidates per query, device merge"))
                           if world > 1 else "single GPU",
                           scan_path=scan_path, unproven_queries_rescanned=redone),
            "clocks": clocks, "gpu_launches": int(launches),
            "e2e": {"value": e2e_qps, "unit": "queries/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "roofline": roofline}
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(shard, queries, k, args.cpu_seconds, res_ids, res_d, int(metric))
    elif world > 1:
        # the merged answer of the sampled queries against the oracle over the whole database
        from oracle import pxo

        full = space.prepare_batch(flat_rows(args, 0, n))
        samp = np.linspace(0, own_n - 1, num=min(args.parity_queries, own_n)).astype(np.int64)  # rank 0's slice
        ri, rd, rl = pxo.flat_search(full, queries[own_b + samp], k, int(metric))
        same = sum(int(np.array_equal(res_ids[q, :rl[i]], ri[i, :rl[i]]) and
                       np.array_equal(res_d[q, :rl[i]].view(np.uint32), rd[i, :rl[i]].view(np.uint32)))
                   for i, q in enumerate(samp))
        line["config"]["parity_sample"] = {"queries": len(samp), "identical_ids_and_distance_bits": same,
                                           "against": f"oracle FlatIndex::search over all {n:,} rows"}
    if world == 1 and not args.no_extras:
        line["extras"] = run_extras(args)
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
