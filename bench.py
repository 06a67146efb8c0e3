"""LEMA prefill match on B200 -- the benchmark line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload ("kernel-level prefill on 1 B200"): B=8 x H=64 = 512 streams of
T=16384 positions, 32-bit codes (per-stream pool of 8192 codes, Zipf 1.1, 10% fresh), value
rows of 24 bf16 (48 bytes). One step = the exact op over the whole batch: for every position,
the latest earlier position whose key code equals its query code, and its value row gathered
(zeros on a miss) -- code/lema/attention.py:100-158 -- through lema_prefill_match (K2).

Metric: Mpos/s of the whole job. Inputs are resident in HBM when the timed region starts;
codes + values + outputs (~0.9 GB) exceed the 126 MB L2, so no flush is needed between
steps. `e2e` is the same metric through the public host-buffer call (attention.HostPrefill)
with host buffers: every step copies its codes and values host->device from pinned memory
and its outputs back.

Multi-GPU (torchrun, one process per GPU): the 512 streams are independent, so they are split
by head over the ranks (512 / N streams each, "scaling": "strong") with no collective on the
data path; the time is the max over ranks of CUDA-event time. The line also carries a small
batched-decode record (config 4's model, batch split over the ranks, short prefix).

--impl reference: the reference's own CPU implementation of the path -- its C++ store
(code/lema/csrc/store.cpp, built from source into oracle/_ref) exchanging all 512 streams'
positions in one call on all host cores, as code/lema/cache.py:184-201 does. Rank 0 alone
runs it.
"""
from __future__ import annotations

import argparse
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

B, H, T, D_V = 8, 64, 16384, 24
N_STREAMS = B * H          # --streams overrides (smaller cases for profiling)
VBYTES = D_V * 2
METRIC = "LEMA prefill Mpos/s/GPU & batched decode tok/s; % of HBM roofline"
UNIT = "Mpos/s"
WORKLOAD = "cfg2: kernel-level prefill, B=8 H=64 T=16384, 32-bit codes, d_v 24 bf16"


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        self.file.flush()
        rows = [r.split(",") for r in Path(self.file.name).read_text().splitlines() if r.strip()]
        os.unlink(self.file.name)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [x.strip() for x in r]
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except (ValueError, IndexError):
                continue
            for name, val in zip(names, r[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(n_gpus: int):
    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}: launch N>1 with torchrun")
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    return rank, world


def make_inputs(device, n_total: int, lo: int, hi: int):
    """Streams [lo, hi) of the config-2 workload (all n_total streams drawn with one seed, so
    every GPU count sees the same data)."""
    import torch

    from latest_exact_match_attention_b200 import synth
    qc, kc = synth.code_streams(n_total, T, synth.CONFIG2, seed=0, config_id=2)
    qc, kc = np.ascontiguousarray(qc[lo:hi]), np.ascontiguousarray(kc[lo:hi])
    q = torch.from_numpy(qc.view(np.int32)).to(device)
    k = torch.from_numpy(kc.view(np.int32)).to(device)
    v = synth.values_torch(n_total, T, D_V, torch.bfloat16, device, seed=0, config_id=2)[lo:hi].contiguous()
    return qc, kc, q, k, v


def cpu_reference_sample(qc: np.ndarray, kc: np.ndarray, n_streams: int, reps: int = 1):
    """The reference's C++ store exchange (oracle/_ref) over `n_streams` full streams in one
    call on all host cores: returns (Mpos/s, cores, kind, sample description). With reps = 0
    the one timed call is also the warm-up (the caller has warmed up already)."""
    import torch

    import oracle
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    ref = oracle.ref_store()
    qs, ks = qc[:n_streams].astype(np.int64), kc[:n_streams].astype(np.int64)
    n = n_streams * T
    vals = torch.from_numpy(np.random.default_rng(0).integers(0, 1 << 16, size=(n, D_V), dtype=np.uint16))
    out = torch.empty_like(vals)
    q64, k64 = torch.from_numpy(qs.reshape(-1)), torch.from_numpy(ks.reshape(-1))
    if ref is not None:
        cap = int(n * 1.6)
        times = []
        for _ in range(reps + 1):          # one warm-up: OpenMP team, page touch
            table = torch.zeros((cap, 16 + VBYTES), dtype=torch.uint8)
            t0 = time.perf_counter()
            ref.exchange(table, q64, k64, vals, out, T, 0, cap, VBYTES)
            times.append(time.perf_counter() - t0)
        dt = min(times[1:] or times)
        return n / dt / 1e6, cores, "reference", (
            f"code/lema/csrc/store.cpp exchange, {n_streams} streams x {T} positions in one call "
            f"(P={n_streams}, T={T}), {cores} OpenMP threads, table load {n / cap:.2f}")
    # no reference build: the oracle port (single-threaded dictionary sweep + gather)
    t0 = time.perf_counter()
    src = oracle.latest_prev_match(qs, ks)
    oracle.gather(src, vals.numpy().reshape(n_streams, T, D_V))
    dt = time.perf_counter() - t0
    return n / dt / 1e6, 1, "port", f"oracle latest_prev_match + gather, {n_streams} streams x {T}"


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from latest_exact_match_attention_b200 import synth
    n = args.streams                              # the whole workload: 512 streams
    qc, kc = synth.code_streams(n, T, synth.CONFIG2, seed=0, config_id=2)
    vals = []
    for _ in range(args.warmup):
        cpu_reference_sample(qc, kc, n, reps=0)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        v, cores, kind, desc = cpu_reference_sample(qc, kc, n, reps=0)
        vals.append(v)
    wall = time.perf_counter() - t0
    value = statistics.median(vals)
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * wall / max(1, args.steps), 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "u32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "streams": n, "global_batch": N_STREAMS,
                   "seq_len": T, "parallelism": "cpu", "same_config": n == N_STREAMS},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": cores, "kind": kind,
                         "sample": desc},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_b200(args):
    import torch

    from latest_exact_match_attention_b200 import _lib
    from latest_exact_match_attention_b200._lib import call, ptr

    rank, world = dist_setup(args.gpus)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    n_total = args.streams
    if n_total % world:
        raise SystemExit(f"{n_total} streams do not split over {world} GPUs")
    n_rank = n_total // world                 # heads split over the ranks: strong scaling
    lo, hi = rank * n_rank, (rank + 1) * n_rank
    qc, kc, q, k, v = make_inputs(dev, n_total, lo, hi)
    n_pos = n_rank * T
    src = torch.empty((n_rank, T), dtype=torch.int32, device=dev)
    out = torch.empty_like(v)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ws_bytes = int(_lib.lib().lema_prefill_workspace_bytes(n_rank, T, 4))
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        call("lema_prefill_match", ptr(q), ptr(k), 4, n_rank, T, ptr(src), ptr(v), VBYTES,
             ptr(out), ptr(ws), ws_bytes, ptr(status), stream.cuda_stream)

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        import torch.distributed as dist
        t = torch.tensor([x], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    assert int(status.item()) == 0, "device status raised during warm-up"

    # algorithmic bytes per step: codes in, index + row out, each distinct source row read once
    s = src.to(torch.int64)
    hit = s >= 0
    ids = (torch.arange(n_rank, device=dev, dtype=torch.int64)[:, None] * T + s)[hit]
    U = int(torch.unique(ids).numel())
    alg_bytes = n_pos * (4 + 4 + VBYTES + 4) + U * VBYTES
    hit_rate = float(hit.float().mean())
    del s, hit, ids

    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        # the sampler's start-up pause leaves the GPU idle: warm it up again, untimed, right
        # before the barrier and synchronisation that open the timed region
        for _ in range(max(3, args.warmup)):
            step()
        barrier()
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for i in range(args.steps):
            ev[i][0].record(stream)
            step()
            ev[i][1].record(stream)
        t1.record(stream)
        torch.cuda.synchronize()
        barrier()
        # sustained: repeats of >= 0.1 s each (>= 0.5 s in all), median per step, under the
        # same clock sampling -- the K-step region above is only a few milliseconds
        per_step = max(1e-3, t0.elapsed_time(t1) / args.steps)
        reps_steps = max(1, int(100.0 / per_step))
        sustained = []
        for _ in range(5):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(reps_steps):
                step()
            b.record(stream)
            torch.cuda.synchronize()
            sustained.append(a.elapsed_time(b) / reps_steps)
    barrier()
    clocks = clk.summary()
    total_ms = max_over_ranks(t0.elapsed_time(t1))
    per_launch_ms = statistics.mean(a.elapsed_time(b) for a, b in ev)
    sustained_ms = max_over_ranks(statistics.median(sustained))
    assert int(status.item()) == 0, "device status raised during the timed region"
    ms_per_step = total_ms / args.steps
    value = n_total * T * args.steps / (total_ms / 1e3) / 1e6

    # end to end through the public host-buffer call, copies inside the timed region
    e2e_steps = 0 if args.no_e2e else max(1, min(args.steps, 5))
    hq = torch.from_numpy(qc.view(np.int32)).pin_memory()
    hk = torch.from_numpy(kc.view(np.int32)).pin_memory()
    hv = v.cpu().pin_memory()
    ho = torch.empty_like(hv).pin_memory()
    hs = torch.empty((n_rank, T), dtype=torch.int32).pin_memory()
    h2d = hq.numel() * 4 + hk.numel() * 4 + hv.numel() * 2
    d2h = ho.numel() * 2 + hs.numel() * 4
    # the public host-buffer call: batches of --e2e-batch streams, copies both ways overlapped
    # with the kernels (attention.HostPrefill); one untimed call first
    from latest_exact_match_attention_b200.attention import HostPrefill
    hp = HostPrefill(dev, T, torch.int32, (D_V,), torch.bfloat16, batch=min(args.e2e_batch, n_rank),
                     slots=args.e2e_slots)
    if e2e_steps:
        hp(hq, hk, hv, hs, ho)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    if e2e_steps == 0:
        step()
    for _ in range(e2e_steps):
        hp(hq, hk, hv, hs, ho)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    e2e_value = n_total * T * e2e_steps / (e2e_ms / 1e3) / 1e6 if e2e_steps else None
    _lib.check_status(dev, "bench e2e")

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cv, cores, kind, desc = cpu_reference_sample(qc, kc, n_rank, reps=1)
        cpu = {"value": round(cv, 3), "unit": UNIT, "cores": cores, "kind": kind, "sample": desc}

    decode = None
    if not args.no_decode:
        try:
            decode = decode_record(args, rank, world, dev, small=True)
        except Exception as e:      # the headline line is printed whatever happens here
            decode = {"error": f"{type(e).__name__}: {e}"[:300]}

    peak, peak_src = peaks()
    achieved = alg_bytes / (per_launch_ms / 1e3) / 1e9
    # K2 runs pipelined (one launch matches and copies rows) from one full wave of matchers
    # (2 per SM) on, unless LEMA_K2_PIPELINE=0; the rows here are 48 bytes (16-byte aligned)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    pipelined = (os.environ.get("LEMA_K2_PIPELINE", "")[:1] != "0" and n_rank >= 2 * sms
                 and T <= (1 << 22))
    # DRAM bytes per call: not observable without a profiler, so taken from the ncu capture
    # of this workload summarised in profiles/ (full 512-stream calls only), and labelled
    traffic = None
    tf = ROOT / "profiles" / "prefill_match_cfg2.md"
    if tf.exists() and n_rank == 512:
        import re
        key = "traffic_bytes_per_call_pipelined" if pipelined else "traffic_bytes_per_call"
        m = re.search(key + r":\s*(\d+)", tf.read_text())
        traffic = int(m.group(1)) if m else None
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u32",
        "data": "synthetic (seeded Zipf-pool codes, N(0,1) bf16 values)",
        "value_scope": "whole job: all streams' positions / max-over-ranks time",
        "value_per_gpu": round(value / world, 2),
        "config": {"workload": WORKLOAD, "streams_total": n_total, "streams_per_gpu": n_rank,
                   "positions_per_gpu": n_pos, "seq_len": T, "value_bytes": VBYTES,
                   "parallelism": f"heads split over {world} GPU(s), no collective",
                   "l2": "inputs+outputs 0.9 GB > 126 MB L2 (no flush)", "hit_rate": round(hit_rate, 4),
                   "distinct_sources": U,
                   "k2_mode": "pipelined" if pipelined else "two-kernel"},
        "sustained": {"ms_per_step_median": round(sustained_ms, 4), "repeats": 5,
                      "steps_per_repeat": reps_steps,
                      "value": round(n_total * T / (sustained_ms / 1e3) / 1e6, 2)},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "traffic_source": "ncu capture of this workload (profiles/prefill_match_cfg2.md)"
                     if traffic else None,
                     "peak_source": peak_src, "alg_bytes_per_launch": alg_bytes,
                     "launch_ms": round(per_launch_ms, 4)},
        "e2e": {"value": e2e_value and round(e2e_value, 2), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                "batch_streams": min(args.e2e_batch, n_rank), "device_slots": args.e2e_slots},
        "cpu_baseline": cpu,
        "decode": decode,
        # per step: the shared-memory match kernel (pipelined: it also copies the rows), the
        # overflow-path kernel (launched whenever a stream could outgrow the shared table,
        # T > 6144; it exits at once when none did) and, two-kernel path only, the row gather
        "gpu_launches": args.steps * ((1 if pipelined else 2) + (1 if T > 6144 else 0)),
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)


def run_match(args):
    """Config 2's streams without value rows: the index half of the op (what
    `latest_prev_match` computes, code/lema/attention.py:100-132), through lema_prefill_match
    with src only, on the default matcher for such calls (the dictionary + sweep matcher from
    one wave of streams) and on the chunked matcher (LEMA_K2_SWEEP=0). Algorithmic bytes: two
    codes in and one index out per position."""
    import torch

    from latest_exact_match_attention_b200 import _lib
    from latest_exact_match_attention_b200._lib import call, ptr
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    n = args.streams
    qc, kc, q, k, _ = make_inputs(dev, n, 0, n)
    src = torch.empty((n, T), dtype=torch.int32, device=dev)
    nb = int(_lib.lib().lema_prefill_workspace_bytes(n, T, 4))
    ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=dev)
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    peak, peak_src = peaks()
    res = {}
    for name, env in (("sweep", None), ("chunked", "0")):
        if env is None:
            os.environ.pop("LEMA_K2_SWEEP", None)
        else:
            os.environ["LEMA_K2_SWEEP"] = env

        def step():
            call("lema_prefill_match", ptr(q), ptr(k), 4, n, T, ptr(src), None, 0, None, ptr(ws), nb,
                 ptr(st), stream.cuda_stream)
        with ClockSampler(dev.index) as clk:
            for _ in range(max(3, args.warmup)):     # after the sampler's start-up pause
                step()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(args.steps):
                step()
            b.record(stream)
            torch.cuda.synchronize()
        ms = a.elapsed_time(b) / args.steps
        assert int(st.item()) == 0
        alg = n * T * 12
        res[name] = {"ms": round(ms, 4), "mpos_s": round(n * T / ms / 1e3, 1),
                     "roofline_frac": round(alg / (ms / 1e3) / 1e9 / peak, 4), "clocks": clk.summary()}
    os.environ.pop("LEMA_K2_SWEEP", None)
    print(json.dumps({
        "metric": "latest_prev_match Mpos/s (config 2 streams, indices only)", "value": res["sweep"]["mpos_s"],
        "unit": "Mpos/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "dtype": "u32", "data": "synthetic (seeded Zipf-pool codes)",
        "config": {"workload": f"cfg2 streams without value rows: {n} x {T}", "alg_bytes_per_call": n * T * 12,
                   "peak_gbs": peak, "peak_source": peak_src},
        "matchers": res, "gpu_launches": args.steps * (1 + (1 if T > 6144 else 0)),
    }), flush=True)


def run_proj(args):
    """K1 alone at config 3's projection shapes: B=32 x T=16384 rows of dim 1024, d_qk 32,
    hq = hk = H for H in --heads. One JSON line per H (TFLOP/s against the measured bf16 GEMM
    peak), with the reference's own GPU recipe -- a bf16 GEMM to z in HBM, then pack_codes as
    code/lema/attention.py:94-97 writes it -- timed beside it on the same inputs."""
    import torch

    from latest_exact_match_attention_b200 import proj_codes
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    Bp, Tp, dim = args.proj_batch, 16384, 1024
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn((Bp, Tp, dim), generator=g, device=dev).to(torch.bfloat16)
    pk = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak, peak_src = (float(pk["bf16_tflops"]), "measured (burst)") if "bf16_tflops" in pk else (1590.0, "fallback")
    stream = torch.cuda.current_stream(dev)

    def timed(fn, steps):
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(steps):
            fn()
        b.record(stream)
        torch.cuda.synchronize()
        return a.elapsed_time(b) / steps

    for H in args.heads:
        w = (0.02 * torch.randn((2 * H * 32, dim), generator=g, device=dev)).to(torch.bfloat16)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        with ClockSampler(dev.index) as clk:
            ms = timed(lambda: proj_codes(x, w, H, H, status=status), args.steps)
        assert int(status.item()) == 0
        pw = torch.ones((), dtype=torch.int64, device=dev) << torch.arange(32, device=dev)

        def reference_recipe():
            z = (x @ w.T).view(Bp, Tp, 2 * H, 32)
            return ((z >= 0).to(torch.int64) * pw).sum(-1)
        ref_ms = None if args.no_recipe else timed(reference_recipe, max(2, args.steps // 4))
        # code flips against an fp64 z (the benchmark's rule: a bit may differ from the exact
        # sign only where |z_d| < 1e-3 ||z_row||), on the first 65536 rows
        qc, kc = proj_codes(x, w, H, H, status=status)
        rows = min(65536, Tp)
        z = (x[0, :rows].double() @ w.double().T).view(rows, 2 * H, 32)
        codes = torch.cat([qc[0, :, :rows], kc[0, :, :rows]], 0).transpose(0, 1).to(torch.int64) & 0xFFFFFFFF
        bits = ((codes[..., None] >> torch.arange(32, device=dev)) & 1).bool()
        diff = bits != (z >= 0)
        band = z.abs() < 1e-3 * z.norm(dim=-1, keepdim=True)
        flips = {"rows": rows, "bits": int(z.numel()), "code_flips": int(diff.sum()),
                 "code_flips_outside_band": int((diff & ~band).sum())}
        del z, codes, bits, diff, band
        flops = 2.0 * Bp * Tp * dim * (2 * H * 32)
        tf = flops / (ms / 1e3) / 1e12
        print(json.dumps({
            "metric": "K1 code projection TFLOP/s", "value": round(tf, 1), "unit": "TFLOP/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "dtype": "bf16", "data": "synthetic N(0,1) x, N(0,0.02) w",
            "config": {"workload": f"cfg3 K1: B={Bp} T={Tp} dim={dim} hq=hk={H} d_qk=32",
                       "rows": Bp * Tp, "cols": 2 * H * 32, "l2": "x 1 GiB > L2"},
            "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(tf / peak, 4), "peak_source": peak_src},
            "reference_recipe_ms": ref_ms and round(ref_ms, 4), "codes_vs_fp64": flips,
            "speedup_vs_reference_recipe": ref_ms and round(ref_ms / ms, 2),
            "gpu_launches": args.steps, "clocks": clk.summary(),
        }), flush=True)
        del w


def _model_cfg(which: int, H: int = 64):
    from latest_exact_match_attention_b200.model import ModelConfig
    if which == 3:   # 309M-shaped: d_model 1024, 24 blocks, SwiGLU 4x, heads swept, 32-bit codes
        return ModelConfig(vocab_size=50304, depth=24, dim=1024, num_heads=H, d_qk=32,
                           d_v=1024 // H, dim_ff=4096)
    # 834M-shaped: d_model 1536, 24 blocks, 64 heads, d_v 24, 32-bit codes
    return ModelConfig(vocab_size=50304, depth=24, dim=1536, num_heads=64, d_qk=32, d_v=24)


def run_model_prefill(args):
    """Config 3: full prefill of a random-init 309M-shaped LEMA LM (bf16), B=32 x T=16384
    synthetic tokens, heads swept; every layer runs K1 (codes) and K2 (exact op). One JSON
    line per head count, in tokens (= positions) per second."""
    import torch

    from latest_exact_match_attention_b200 import synth
    from latest_exact_match_attention_b200.model import Transformer
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    Bm, Tm = args.proj_batch, 16384
    idx = torch.from_numpy(synth.token_stream(Bm, Tm, 50304, seed=0, config_id=3)).to(dev)
    stream = torch.cuda.current_stream(dev)
    for H in args.heads:
        torch.manual_seed(0)
        cfg = _model_cfg(3, H)
        model = Transformer(cfg).to(dev).to(torch.bfloat16).eval()
        for _ in range(max(3, args.warmup)):
            model(idx, return_logits=False)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(dev.index) as clk:
            a.record(stream)
            for _ in range(args.steps):
                model(idx, return_logits=False)
            b.record(stream)
            torch.cuda.synchronize()
        ms = a.elapsed_time(b) / args.steps
        print(json.dumps({
            "metric": "LEMA full prefill tokens/s (config 3)", "value": round(Bm * Tm / ms / 1e3, 3),
            "unit": "Mtok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 3), "higher_is_better": True, "dtype": "bf16",
            "data": "synthetic Zipf(1.1) tokens, 20% bigram copies; random-init weights",
            "config": {"workload": f"cfg3: {cfg.summary()}, B={Bm} T={Tm}", "params": model.n_params()},
            "clocks": clk.summary(),
        }), flush=True)
        del model
        torch.cuda.empty_cache()


def decode_record(args, rank: int, world: int, dev, small: bool = False, worst_load: float | None = None):
    """Config 4: batched greedy decode of a random-init 834M-shaped LEMA LM (bf16), the batch
    split over the ranks (each its own store and graph, no collective). Each sequence's store
    is pre-filled from a bigram-structured prefix (chunked prefill through the store), then
    every step is one CUDA-graph replay (all 24 layers' store exchanges inside). `small`: the
    sub-record of the headline line (prefix 512, 32 steps). `worst_load`: the stress mode --
    every layer's codes replaced by fresh random codes (cache.worst_case_codes, the reference's
    worst-case hook), the store sized so that it ends at that load. Returns the record (rank 0)
    with tokens/s of the whole job = all ranks' tokens / max-over-ranks time."""
    import math

    import torch

    from latest_exact_match_attention_b200 import synth
    from latest_exact_match_attention_b200.cache import worst_case_codes
    from latest_exact_match_attention_b200.decode import decoder
    from latest_exact_match_attention_b200.model import Transformer
    cfg = _model_cfg(4)
    B_all = args.decode_batch if worst_load is None else args.worst_batch
    prefix = 512 if small else args.prefix
    steps = 32 if small else args.steps
    warm = 3 if small else max(3, args.warmup)
    if B_all % world:
        raise SystemExit(f"decode batch {B_all} does not split over {world} GPUs")
    Bd = B_all // world
    torch.manual_seed(0)
    model = Transformer(cfg).to(dev).to(torch.bfloat16).eval()
    toks = synth.token_stream(B_all, prefix + 1, 50304, seed=0, config_id=4)
    idx = torch.from_numpy(toks[rank * Bd:(rank + 1) * Bd]).to(dev)
    P = Bd * cfg.num_heads
    # the decoder's warm-up runs on a scratch store; the real store takes the prefix, the
    # warm-up-free timed steps and the first replays
    tokens = prefix + warm + steps + 8
    if worst_load is not None:
        per_part, load = tokens, worst_load          # one new entry per token per partition
    else:
        per_part = (min(args.entries_per_partition, tokens) if args.entries_per_partition else tokens)
        load = args.max_load
    cap = math.ceil(cfg.depth * P * per_part / load)
    from latest_exact_match_attention_b200 import _lib
    need = cap * int(_lib.lib().lema_store_slot_bytes(cfg.d_v * 2))
    free = torch.cuda.mem_get_info(dev)[0]
    if need > 0.9 * free - (4 << 30):
        raise SystemExit(f"decode store of {cap} slots ({need / 2**30:.1f} GiB) does not fit the "
                         f"{free / 2**30:.1f} GiB free; lower --entries-per-partition or --decode-batch")
    hook = worst_case_codes(cfg.depth) if worst_load is not None else None
    cache = model.new_cache("hbm", capacity=cap, batch=Bd, codes_hook=hook)
    stream = torch.cuda.current_stream(dev)

    def maxr(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for s0 in range(0, prefix, args.chunk):
        model(idx[:, s0:min(prefix, s0 + args.chunk)], cache=cache, return_logits=False)
    b.record(stream)
    torch.cuda.synchronize()
    prefill_ms = maxr(a.elapsed_time(b))
    cache.check()
    counts = cache.counts().float()            # [depth, batch, heads]
    d = decoder(model, cache, tok=idx[:, prefix:prefix + 1])
    with ClockSampler(dev.index) as clk:
        for _ in range(warm):            # after the sampler's start-up pause, untimed
            d.step()
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        a.record(stream)
        for _ in range(steps):
            d.step()
        b.record(stream)
        torch.cuda.synchronize()
    cache.check()
    ms = maxr(a.elapsed_time(b)) / steps
    weights = sum(p.numel() * p.element_size() for p in model.parameters())
    store_bytes = cfg.depth * P * 216          # per (layer, seq, head) op: codes, row, slots
    rec = {
        "metric": "LEMA batched decode tok/s (config 4)" + (" worst-case codes" if hook else ""),
        "value": round(B_all * 1e3 / ms, 1), "unit": "tok/s", "n_gpus": world, "steps": steps,
        "warmup": warm, "ms_per_step": round(ms, 4), "higher_is_better": True, "dtype": "bf16",
        "scaling": "strong" if world > 1 else None,
        "data": "synthetic Zipf(1.1) tokens, 20% bigram copies; random-init weights",
        "config": {"workload": f"cfg4: {cfg.summary()}, B={B_all} ({Bd} per GPU), prefix {prefix}",
                   "parallelism": f"batch split over {world} GPU(s), own store and graph each",
                   "store_slots_per_gpu": cap, "store_gb_per_gpu": round(cache.nbytes() / 1e9, 2),
                   "store_load": round(cache.load(), 4),
                   "entries_per_partition_mean": round(float(counts.mean()), 1),
                   "entries_per_partition_max": int(counts.max())},
        "roofline": {"bound": "hbm", "bytes_per_step_per_gpu": weights + store_bytes,
                     "achieved": round((weights + store_bytes) / (ms / 1e3) / 1e9, 1),
                     "peak": peaks()[0], "unit": "GB/s",
                     "frac": round((weights + store_bytes) / (ms / 1e3) / 1e9 / peaks()[0], 4)},
        "prefill": {"tokens": B_all * prefix, "ms": round(prefill_ms, 1),
                    "tok_s": round(B_all * prefix / prefill_ms * 1e3, 1), "chunk": args.chunk},
        "clocks": clk.summary(),
    }
    del d, cache, model
    torch.cuda.empty_cache()
    return rec


def run_decode(args):
    """Config 4 (see decode_record); --worst-case: the stress mode at store loads 0.5 / 0.9 /
    0.95 at the end of the run, batch --worst-batch, against context --prefix."""
    import torch
    rank, world = dist_setup(args.gpus)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    loads = [None] if not args.worst_case else [0.5, 0.9, 0.95]
    for ld in loads:
        rec = decode_record(args, rank, world, dev, worst_load=ld)
        if rank == 0:
            if ld is not None:
                rec["worst_case"] = {"store_load_target": ld,
                                     "ms_per_token": rec["ms_per_step"],
                                     "reference_published": "RTX 3090 + host store, 834M (24 heads), B=1: "
                                     "3.045 ms/tok @1.4k ctx ... 4.059 @573k (load 0.95), "
                                     "code/experiments/main_inference/out/gen_08B_ram.jsonl"}
            print(json.dumps(rec), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def check_longctx_heads(args, rank, world, dev, src, out, v, H, T, L):
    """Config 5 parity at full length: for heads 0 .. args.check_heads - 1 the indices of the
    whole sequence (every rank's shard, gathered on rank 0) equal the oracle's
    latest_prev_match over the single unsharded sequence (code/lema/attention.py:100-132),
    regenerated on rank 0; each rank checks the value rows of 2^16 sampled positions whose
    source lies in its own shard (and zeros where there is none)."""
    import torch

    import oracle
    from latest_exact_match_attention_b200 import synth
    base = rank * L
    res = {"heads": [], "rows_checked": 0, "rows_equal": True}
    g = torch.Generator(device=dev).manual_seed(rank)
    for h in range(min(args.check_heads, H)):
        idx = torch.randint(0, L, (1 << 16,), generator=g, device=dev)
        s = src[h, idx].long()
        local = s >= base
        ok = torch.equal(out[h, idx[local]], v[h, s[local] - base])
        ok = ok and bool((out[h, idx[s < 0]] == 0).all())
        res["rows_checked"] += int(local.sum()) + int((s < 0).sum())
        res["rows_equal"] = res["rows_equal"] and ok
        mine = src[h].contiguous()
        if world > 1:
            parts = [torch.empty_like(mine) for _ in range(world)]
            torch.distributed.all_gather(parts, mine)
            full = torch.cat(parts)
        else:
            full = mine
        if rank == 0:
            q1, k1, _ = synth.long_code_shard(H, 0, T, synth.CONFIG5, seed=0, device=dev, heads=[h],
                                              values=False)
            qn, kn = q1.cpu().numpy().view(np.uint32), k1.cpu().numpy().view(np.uint32)
            del q1, k1
            t0 = time.perf_counter()
            want = oracle.latest_prev_match(qn, kn)[0]
            cpu_s = time.perf_counter() - t0
            got = full.cpu().numpy().astype(np.int64)
            res["heads"].append({"head": h, "positions": T, "indices_equal": bool(np.array_equal(got, want)),
                                 "mismatches": int((got != want).sum()),
                                 "oracle_cpu_s": round(cpu_s, 2)})
            del qn, kn, want, got
        del full
    return res


def run_longctx(args):
    """Config 5: the exact op over ONE sequence of --long-t positions (default 2^26), 16 heads,
    32-bit codes (pool 2^20, Zipf 1.05, 5% fresh), 128-byte bf16 value rows, sharded by
    sequence over the torchrun ranks (one per GPU): each rank owns a contiguous slice of every
    head and the ranks exchange last-occurrence tables and value rows over NCCL
    (latest_exact_match_attention_b200.longctx; value rows read in place from the earlier
    ranks' memory, or with LEMA_SHARD_PEER=0 requested and exchanged by all-to-all). Value:
    positions per second of the whole sequence; time = max over ranks of CUDA-event time."""
    import torch

    from latest_exact_match_attention_b200 import synth
    from latest_exact_match_attention_b200.longctx import CudaOps, SingleComm, TorchComm, sharded_prefill
    rank, world = dist_setup(args.gpus)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    H, T = 16, args.long_t
    L = T // world
    qc, kc, v = synth.long_code_shard(H, rank * L, L, synth.CONFIG5, seed=0, device=dev)
    comm = TorchComm() if world > 1 else SingleComm()
    ops = CudaOps(dev, rows_per_head=args.sweep_rows or None)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    for _ in range(max(1, args.warmup)):
        src, out = sharded_prefill(qc, kc, v, comm, ops, seg_len=args.seg_len)
        del src, out
    torch.cuda.synchronize()
    hit = 0.0
    times, phases = [], {}
    with ClockSampler(local) as clk:
        for it in range(args.steps):
            barrier()
            torch.cuda.synchronize()
            marks = []
            a = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            src, out = sharded_prefill(qc, kc, v, comm, ops, seg_len=args.seg_len, marks=marks)
            torch.cuda.synchronize()
            times.append(a.elapsed_time(marks[-1][1]))
            prev = a
            for name, e in marks:
                phases[name] = phases.get(name, 0.0) + prev.elapsed_time(e) / args.steps
                prev = e
            hit = float((src >= 0).float().mean())
            if it < args.steps - 1 or not args.check_heads:
                del src, out           # the last step's results are checked below
    barrier()
    check = None
    if args.check_heads:
        check = check_longctx_heads(args, rank, world, dev, src, out, v, H, T, L)
        del src, out
    ms = statistics.mean(times)
    names = list(phases)
    pmax = dict(phases)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
        pt = torch.tensor([phases[k] for k in names], device=dev)
        torch.distributed.all_reduce(pt, op=torch.distributed.ReduceOp.MAX)
        pmax = dict(zip(names, pt.tolist()))
    if world > 1:
        torch.distributed.destroy_process_group()
    if rank != 0:
        return
    n = H * T
    alg = n * (4 + 4 + 128 + 4)            # codes, index, row out per position (+ rows read)
    print(json.dumps({
        "metric": "LEMA sequence-sharded prefill Mpos/s (config 5)", "value": round(n / ms / 1e3, 2),
        "unit": "Mpos/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong",
        "dtype": "u32", "data": "synthetic (device-generated, chunk-seeded)",
        "config": {"workload": f"cfg5: T={T} H={H} 32-bit codes pool 2^20 Zipf 1.05 5% fresh, d_v 64 bf16",
                   "positions_per_gpu": n // world, "seg_len": args.seg_len, "hit_rate": round(hit, 4),
                   "parallelism": "one GPU, no collective" if world == 1 else
                   f"sequence x{world}, NCCL all-gather + " + (
                       "all-to-all of rows" if "row_all_to_all" in phases else
                       "rows read from peer GPUs' memory (CUDA IPC, NVLink)")},
        "parity_check": check,
        "phases_ms_rank0": {k: round(x, 3) for k, x in phases.items()},
        "phases_ms_max_over_ranks": {k: round(x, 3) for k, x in pmax.items()},
        "roofline": {"bound": "hbm", "alg_bytes_per_gpu_lower": alg // world,
                     "achieved": round(alg / world / (ms / 1e3) / 1e9, 1), "peak": peaks()[0],
                     "unit": "GB/s", "frac": round(alg / world / (ms / 1e3) / 1e9 / peaks()[0], 4)},
        "clocks": clk.summary(),
    }), flush=True)


def run_cpu_baselines(args):
    """The CPU timings the benchmark plan asks for beside the GPU (rank 0, host cores of the
    box), each next to the same work on the GPU through this library:
      config 1  the reference's C++ store (oracle/_ref): one prefill exchange of 8 partitions x
                4096 positions, then 512 single-position exchanges (16-bit codes, fp32 d_v 64);
      config 4  store work of one decode step: 24 single-position exchanges of P = 256 x 64
                partitions against a table holding a 3050-entry prefix state per partition;
      config 5  the index oracle (C restatement of code/lema/attention.py:100-132, one thread)
                over one full head of 2^26 positions.
    One JSON line each."""
    import torch

    import oracle
    from latest_exact_match_attention_b200 import synth
    from latest_exact_match_attention_b200.cache import HashStore
    dev = torch.device("cuda", 0)
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    ref = oracle.ref_store()
    kind = "reference" if ref is not None else "port"

    def cpu_exchange(table, q, k, vals, out, Tx, cap, vb):
        if ref is not None:
            ref.exchange(table, q, k, vals, out, Tx, 0, cap, vb)
        else:
            oracle.store_exchange(table.numpy(), q.numpy(), k.numpy(), vals.numpy(), Tx, 0)

    def gpu_time(fn, reps=3):
        fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps

    # ---------------------------------------------------------------- config 1
    P1, T1, S1, dv1 = 8, 4096, 512, 64
    qc, kc = synth.code_streams(P1, T1 + S1, synth.CONFIG1, seed=0, config_id=1)
    q64, k64 = qc.astype(np.int64), kc.astype(np.int64)
    vals = torch.from_numpy(synth.values_np(P1, T1 + S1, dv1, seed=0, config_id=1))
    cap1, vb1 = 4 * P1 * (T1 + S1), dv1 * 4
    times = []
    for _ in range(2):
        table = torch.zeros((cap1, 16 + vb1), dtype=torch.uint8)
        out = torch.empty((P1 * T1, dv1), dtype=torch.float32)
        t0 = time.perf_counter()
        cpu_exchange(table, torch.from_numpy(q64[:, :T1].reshape(-1).copy()),
                     torch.from_numpy(k64[:, :T1].reshape(-1).copy()),
                     vals[:, :T1].reshape(-1, dv1).contiguous(), out, T1, cap1, vb1)
        t1 = time.perf_counter()
        o1 = torch.empty((P1, dv1), dtype=torch.float32)
        for t in range(T1, T1 + S1):
            cpu_exchange(table, torch.from_numpy(q64[:, t].copy()), torch.from_numpy(k64[:, t].copy()),
                         vals[:, t].contiguous(), o1, 1, cap1, vb1)
        times.append((t1 - t0, time.perf_counter() - t1))
    cpu_pre, cpu_dec = times[-1]
    # the same on the GPU: the HBM store (K3), codes and values resident
    qd = torch.from_numpy(qc.astype(np.uint32).view(np.int32)).to(dev)
    kd = torch.from_numpy(kc.astype(np.uint32).view(np.int32)).to(dev)
    vd = vals.to(dev)

    def gpu_run():
        st = HashStore(dv1, groups=P1, dtype=torch.float32, capacity=cap1, device=dev)
        o = torch.empty((P1 * T1, dv1), dtype=torch.float32, device=dev)
        o1 = torch.empty((P1, dv1), dtype=torch.float32, device=dev)
        st.exchange(qd[:, :T1].reshape(-1), kd[:, :T1].reshape(-1), vd[:, :T1].reshape(-1, dv1), o, T1, 0,
                    check=False)
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        for t in range(T1, T1 + S1):
            st.exchange(qd[:, t].contiguous(), kd[:, t].contiguous(), vd[:, t].contiguous(), o1, 1, 0,
                        check=False)
        return e
    gpu_run()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    a.record()
    e = gpu_run()
    b = torch.cuda.Event(enable_timing=True)
    b.record()
    torch.cuda.synchronize()
    print(json.dumps({
        "metric": "config 1 store: prefill Mpos/s and decode us/step", "n_gpus": 1,
        "config": {"workload": "cfg1: B=1 H=8, 16-bit codes, fp32 d_v 64, prefill 4096 + 512 decode steps"},
        "cpu_baseline": {"kind": kind, "cores": cores, "prefill_mpos_s": round(P1 * T1 / cpu_pre / 1e6, 3),
                         "decode_us_per_step": round(cpu_dec / S1 * 1e6, 2),
                         "sample": "code/lema/csrc/store.cpp exchange: one call of 8 x 4096, then 512 calls of 8 x 1"},
        "gpu": {"prefill_plus_setup_ms": round(a.elapsed_time(e), 3),
                "decode_us_per_step": round(e.elapsed_time(b) / S1 * 1e3, 2),
                "note": "HBM store, one exchange launch per step (not graph-captured here)"},
    }), flush=True)
    del table

    # ---------------------------------------------------------------- config 4 (store only)
    P4, E4, dv4, L4 = 256 * 64, 3050, 24, 24
    rng = np.random.default_rng(4)
    cap4 = int(P4 * (E4 + 64) / 0.65)
    kpre = rng.integers(0, 1 << 62, size=(P4, E4), dtype=np.int64)
    vpre = torch.from_numpy(rng.integers(0, 1 << 16, size=(P4 * E4, dv4), dtype=np.uint16).view(np.int16))
    qstep = [rng.integers(0, 1 << 62, size=P4, dtype=np.int64) for _ in range(L4)]
    for i, qs in enumerate(qstep):                 # half of the lookups hit the prefix state
        hit = rng.random(P4) < 0.5
        qs[hit] = kpre[np.nonzero(hit)[0], rng.integers(0, E4, size=int(hit.sum()))]
    kstep = [rng.integers(0, 1 << 62, size=P4, dtype=np.int64) for _ in range(L4)]
    vstep = torch.from_numpy(rng.integers(0, 1 << 16, size=(P4, dv4), dtype=np.uint16).view(np.int16))
    vb4 = dv4 * 2
    table = torch.zeros((cap4, 16 + vb4), dtype=torch.uint8)
    outp = torch.empty((P4 * E4, dv4), dtype=torch.int16)
    t0 = time.perf_counter()
    cpu_exchange(table, torch.from_numpy(kpre.reshape(-1)), torch.from_numpy(kpre.reshape(-1)), vpre, outp, E4,
                 cap4, vb4)
    fill_s = time.perf_counter() - t0
    o4 = torch.empty((P4, dv4), dtype=torch.int16)
    t0 = time.perf_counter()
    for i in range(L4):
        cpu_exchange(table, torch.from_numpy(qstep[i]), torch.from_numpy(kstep[i]), vstep, o4, 1, cap4, vb4)
    cpu_step = time.perf_counter() - t0
    del table, outp
    st = HashStore(dv4, groups=P4, dtype=torch.bfloat16, capacity=cap4, device=dev)
    st.exchange(torch.from_numpy(kpre.reshape(-1)).to(dev), torch.from_numpy(kpre.reshape(-1)).to(dev),
                vpre.to(dev).view(torch.bfloat16), torch.empty((P4 * E4, dv4), dtype=torch.bfloat16, device=dev),
                E4, 0, check=False)
    qd4 = [torch.from_numpy(x).to(dev) for x in qstep]
    kd4 = [torch.from_numpy(x).to(dev) for x in kstep]
    vd4 = vstep.to(dev).view(torch.bfloat16)
    od4 = torch.empty((P4, dv4), dtype=torch.bfloat16, device=dev)

    def step4():
        for i in range(L4):
            st.exchange(qd4[i], kd4[i], vd4, od4, 1, 0, check=False)
    g_ms = gpu_time(step4)
    print(json.dumps({
        "metric": "config 4 store work per decode step (24 layers x P = 256 x 64, T = 1)", "n_gpus": 1,
        "config": {"workload": "cfg4 store only: 3050-entry prefix state per partition (64-bit codes), "
                               "half the lookups hit, d_v 24 bf16",
                   "table_load": round(P4 * (E4 + 2 * L4) / cap4, 3)},
        "cpu_baseline": {"kind": kind, "cores": cores, "ms_per_step": round(cpu_step * 1e3, 3),
                         "prefix_fill_s": round(fill_s, 2),
                         "sample": "code/lema/csrc/store.cpp exchange, 24 calls of 16384 x 1"},
        "gpu": {"ms_per_step": round(g_ms, 4)},
    }), flush=True)
    del st

    # ---------------------------------------------------------------- config 5 (index oracle)
    q5, k5, _ = synth.long_code_shard(16, 0, 1 << 26, synth.CONFIG5, seed=0, device=dev, heads=[0], values=False)
    qn, kn = q5.cpu().numpy().view(np.uint32), k5.cpu().numpy().view(np.uint32)
    t0 = time.perf_counter()
    oracle.latest_prev_match(qn, kn)
    o_s = time.perf_counter() - t0
    print(json.dumps({
        "metric": "config 5 index oracle, one head (Mpos/s)", "n_gpus": 0,
        "config": {"workload": "cfg5 head 0: 2^26 positions, 32-bit codes"},
        "cpu_baseline": {"kind": "port", "cores": 1, "value": round((1 << 26) / o_s / 1e6, 2), "unit": "Mpos/s",
                         "seconds": round(o_s, 2),
                         "sample": "oracle/lema_oracle.c latest_prev_match (dictionary sweep) over one full head"},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-slots", type=int, default=3,
                    help="batches in flight on the device in the host-buffer call (e2e)")
    ap.add_argument("--e2e-batch", type=int, default=64,
                    help="streams per batch of the host-buffer call (e2e): smaller batches shorten "
                         "the copy pipeline's fill and drain")
    ap.add_argument("--streams", type=int, default=N_STREAMS,
                    help="streams per GPU (default: the workload's 512); smaller for profiling")
    ap.add_argument("--long-t", type=int, default=1 << 26, help="--workload longctx: positions")
    ap.add_argument("--seg-len", type=int, default=8192, help="--workload longctx: segment")
    ap.add_argument("--check-heads", type=int, default=0,
                    help="--workload longctx: compare this many full-length heads with the oracle")
    ap.add_argument("--sweep-rows", type=int, default=0,
                    help="--workload longctx: sweep rows per head (0 = chosen automatically)")
    ap.add_argument("--workload", choices=["prefill", "match", "proj", "model-prefill", "decode", "longctx",
                                           "cpu-baselines"],
                    default="prefill",
                    help="prefill: the headline config-2 line; proj: K1 at config 3's shapes; "
                         "model-prefill: config 3; decode: config 4")
    ap.add_argument("--decode-batch", type=int, default=256, help="--workload decode: batch")
    ap.add_argument("--prefix", type=int, default=16384, help="--workload decode: prefix tokens")
    ap.add_argument("--chunk", type=int, default=1024, help="--workload decode: prefill chunk")
    ap.add_argument("--entries-per-partition", type=int, default=4300,
                    help="--workload decode: store sizing, entries per (layer, sequence, head) "
                         "(the Zipf prefix of 16384 tokens leaves <= 3200; 0 = one per token)")
    ap.add_argument("--max-load", type=float, default=0.9,
                    help="--workload decode: table load at --entries-per-partition entries")
    ap.add_argument("--worst-case", action="store_true",
                    help="--workload decode: worst-case codes at store loads 0.5 / 0.9 / 0.95")
    ap.add_argument("--worst-batch", type=int, default=1, help="--workload decode --worst-case: batch")
    ap.add_argument("--no-decode", action="store_true",
                    help="headline line: skip its small batched-decode record")
    ap.add_argument("--heads", type=int, nargs="+", default=[8, 16, 32, 64],
                    help="--workload proj: query (= key) heads per layer")
    ap.add_argument("--proj-batch", type=int, default=32, help="--workload proj: sequences")
    ap.add_argument("--no-recipe", action="store_true",
                    help="--workload proj: skip timing the bf16 GEMM + pack recipe")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "b200":
        args.warmup = 3
    if args.workload == "proj":
        run_proj(args)
    elif args.workload == "match":
        run_match(args)
    elif args.workload == "model-prefill":
        run_model_prefill(args)
    elif args.workload == "decode":
        run_decode(args)
    elif args.workload == "longctx":
        run_longctx(args)
    elif args.workload == "cpu-baselines":
        run_cpu_baselines(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
