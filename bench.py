#!/usr/bin/env python3
"""Benchmark of the B200 packed-Q6 routed-expert FFN.

Workload (per GPU, weak scaling): 128 experts, each a SwiGLU FFN with gate/up
2048 -> 512 and down 512 -> 2048, weights N(0, 0.02) (seed 1) encoded to Q6_K (or
Q4_K) by this repository's encoder; 128 * M activation rows N(0, 1) (seed 0) assigned
uniformly at random to the experts (seed 10), route weight 1. A step is one pass of
the routed FFN (route metadata, gate/up + SwiGLU, down, combine) over all rows.

value: algorithmic HBM bytes of the step (packed bytes of every routed expert + the
activation rows read + the output rows written) / device time, summed over ranks.
e2e:   the same bytes / time of the user-facing call with host (pinned) buffers:
       H2D of x, ids and weights, the forward, D2H of the output, every step.
The weights (331 MB of Q6_K at 128 experts) exceed the 126 MB L2, so no flush is
needed between steps.

The line also carries the Q8 KV decode-attention sweep of configs[2] (B in {1, 8, 32},
context 4096 and 32768, 16 q / 2 kv heads, head dim 256, page-table indices) as GB/s of
codes + scales per call, unless --no-attention.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--m 16] [--qtype Q6_K]
    python bench.py --impl reference ...   # the reference's CPU path (NumPy port)
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "data-synth-tpu_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

METRIC = "MoE decode tokens/s (B=1..64, 1/2/4/8 GPU); Q6 expert GEMM HBM GB/s"
HIDDEN, INTER, EXPERTS = 2048, 512, 128
SWEEP_M = (1, 4, 16, 64, 256)
FALLBACK_HBM_GBS = 6650.0


# ---------------------------------------------------------------------------------------
# synthetic weights (NumPy encoder, one process per expert chunk; cached per node in /tmp)
# ---------------------------------------------------------------------------------------


def _encode_chunk(args):
    qtype, seed, first, count = args
    import numpy as np

    from oracle import gguf

    out = {"gate": [], "up": [], "down": []}
    for e in range(first, first + count):
        rng = np.random.default_rng([seed, e])
        for kind, shape in (("gate", (INTER, HIDDEN)), ("up", (INTER, HIDDEN)), ("down", (HIDDEN, INTER))):
            w = rng.normal(0, 0.02, shape).astype(np.float32)
            out[kind].append(gguf.encode(w, qtype).reshape(-1))
    return {k: np.stack(v) for k, v in out.items()}


def synth_experts(qtype, count, seed=1):
    """Raw GGUF bytes ``{gate, up, down: uint8[count, bytes]}``; one generator per node."""
    import numpy as np

    path = Path(tempfile.gettempdir()) / f"qk_bench_{qtype}_{count}_{seed}.npz"
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if not path.exists() and local_rank == 0:
        import multiprocessing as mp

        workers = max(1, min(os.cpu_count() or 1, 16))
        chunk = (count + workers - 1) // workers
        jobs = [(qtype, seed, f, min(chunk, count - f)) for f in range(0, count, chunk)]
        with mp.get_context("spawn").Pool(len(jobs)) as pool:
            parts = pool.map(_encode_chunk, jobs)
        data = {k: np.concatenate([p[k] for p in parts]) for k in ("gate", "up", "down")}
        tmp = path.with_suffix(".tmp.npz")
        np.savez(tmp, **data)
        os.replace(tmp, path)
    deadline = time.time() + 600
    while not path.exists():
        if time.time() > deadline:
            raise TimeoutError(f"{path} was not written by local rank 0")
        time.sleep(0.5)
    with np.load(path) as f:
        return {k: f[k] for k in ("gate", "up", "down")}


def workload_ids(m, rank=0, world=1):
    """Expert of each of rank `rank`'s 128 * M rows: uniform over the 128 * world experts of
    all ranks (seed [10, rank]); with one rank, uniform over its 128."""
    import numpy as np

    return np.random.default_rng([10, rank]).integers(0, EXPERTS * world, (EXPERTS * m, 1)).astype(np.int32)


def workload(m, rank=0, world=1):
    """Activation rows (N(0, 1), seed [0, rank]), expert assignment and route weights (1) of
    rank `rank`'s 128 * M rows."""
    import numpy as np

    rows = EXPERTS * m
    x = np.random.default_rng([0, rank]).normal(size=(rows, HIDDEN)).astype(np.float32)
    weights = np.ones((rows, 1), np.float32)
    return x, workload_ids(m, rank, world), weights


def ep_step_bytes(qtype, m, world):
    """Algorithmic bytes of one expert-parallel step summed over ranks: every rank's routed
    experts (those any rank's rows name) x packed bytes, plus every rank's x rows read and
    output rows written."""
    import numpy as np

    every = np.concatenate([workload_ids(m, r, world)[:, 0] for r in range(world)])
    active = len(np.unique(every))
    return active * packed_bytes_per_expert(qtype) + world * EXPERTS * m * HIDDEN * 2 * 2, active


def packed_bytes_per_expert(qtype):
    per_block = {"Q6_K": 210, "Q4_K": 144}[qtype]
    return (2 * INTER * HIDDEN + HIDDEN * INTER) // 256 * per_block


def step_bytes(qtype, ids):
    """Algorithmic bytes of one step: routed experts' packed bytes + x read + out written."""
    import numpy as np

    active = len(np.unique(ids))
    rows = ids.shape[0]
    return active * packed_bytes_per_expert(qtype) + rows * HIDDEN * 2 * 2, active


PARITY_TOL = 1e-2  # north-star layer tolerance: max relative error (BF16, FP32 accumulation)
PARITY_ROWS = 64


def moe_parity(raw, qtype, res):
    """Max relative error of a seeded sample of the timed step's output rows against the
    oracle's routed FFN (experts.py:61-131 restated); only the sampled rows' experts are
    decoded, so this costs seconds. Runs after the timed region."""
    import numpy as np
    import torch

    from oracle import moe

    x, ids, weights = res["x"], res["ids"], res["weights"]
    rows = np.sort(np.random.default_rng(1000 + res["m"]).choice(x.shape[0], PARITY_ROWS, replace=False))
    expected = moe.expert_ffn(raw["gate"], raw["up"], raw["down"], x[rows], ids[rows], weights[rows],
                              gate_type=qtype, up_type=qtype, down_type=qtype, hidden=HIDDEN,
                              intermediate=INTER)
    got = res["out"].to(torch.float32).cpu().numpy()[rows]
    err = float(np.max(np.abs(got - expected)) / max(np.max(np.abs(expected)), 1e-30))
    return {"moe_rows": PARITY_ROWS, "moe_max_rel_err": err, "tolerance": PARITY_TOL,
            "ok": bool(np.all(np.isfinite(got)) and err < PARITY_TOL)}


def sweep_row(qtype, r, peak):
    gbs = r["bytes"] / (r["ms"] * 1e-3) / 1e9
    gu = r["gate_up_bytes"] / (r["stage_ms"][1] * 1e-3) / 1e9
    return {"qtype": qtype, "m": r["m"], "ms_per_step": r["ms"], "gbs": gbs, "frac": gbs / peak,
            "gate_up_gbs": gu, "gate_up_frac": gu / peak,
            "tflops": r["rows"] * FLOPS_PER_ROW / (r["ms"] * 1e-3) / 1e12,
            "rows_per_s": r["rows"] / (r["ms"] * 1e-3), "active_experts": r["active"],
            "stage_ms": dict(zip(("route_dispatch", "gate_up", "down", "combine"), r["stage_ms"]))}


FLOPS_PER_ROW = 2 * (2 * INTER * HIDDEN + HIDDEN * INTER)


def kernel_bytes(qtype, ids):
    """Algorithmic bytes of the gate/up (dominant) launch: gate+up packed bytes of the routed
    experts + x rows read + h rows written."""
    import numpy as np

    active = len(np.unique(ids))
    rows = ids.shape[0]
    per_block = {"Q6_K": 210, "Q4_K": 144}[qtype]
    return active * 2 * INTER * HIDDEN // 256 * per_block + rows * (HIDDEN + INTER) * 2


# ---------------------------------------------------------------------------------------
# measurement helpers
# ---------------------------------------------------------------------------------------


class ClockSampler:
    """nvidia-smi clocks / throttle reasons of one GPU, sampled every 100 ms."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def hbm_peak():
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic(qtype, m):
    """DRAM bytes per gate/up launch from the committed ncu summary, if one matches."""
    path = ROOT / "profiles" / f"moe_gateup_{qtype.lower()}_m{m}.md"
    try:
        for line in path.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


def cpu_port_gbs(raw, qtype, x, ids, weights, budget_s=10.0):
    """Reference CPU path (NumPy port of experts.py:82-110): decode each routed expert and
    run its SwiGLU with FP32 BLAS, on all host threads, over a bounded sample of experts."""
    import numpy as np

    from oracle import moe
    from oracle.precision import bf16_round

    xb = bf16_round(x)
    order = np.unique(ids)
    done_bytes, elapsed, experts = 0, 0.0, 0
    start = time.perf_counter()
    for e in order:
        rows = np.nonzero(ids[:, 0] == e)[0]
        t0 = time.perf_counter()
        wg = moe.expert_weights(raw["gate"][e], qtype, INTER, HIDDEN)
        wu = moe.expert_weights(raw["up"][e], qtype, INTER, HIDDEN)
        wd = moe.expert_weights(raw["down"][e], qtype, HIDDEN, INTER)
        y = moe.expert_forward(xb[rows], wg, wu, wd, accumulate="f32")
        _ = (y * weights[rows]).astype(np.float32)
        elapsed += time.perf_counter() - t0
        done_bytes += packed_bytes_per_expert(qtype) + rows.size * HIDDEN * 4
        experts += 1
        if time.perf_counter() - start > budget_s:
            break
    return done_bytes / elapsed / 1e9, experts


# ---------------------------------------------------------------------------------------
# arms
# ---------------------------------------------------------------------------------------


def init_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def reference_arm(args):
    import numpy as np

    world, rank, _ = init_dist()
    if rank != 0:
        return 0
    raw = synth_experts(args.qtype, EXPERTS)
    x, ids, weights = workload(args.m)
    cores = os.cpu_count() or 1
    for _ in range(args.warmup):
        cpu_port_gbs(raw, args.qtype, x, ids, weights, budget_s=0.5)
    samples, experts = [], 0
    for _ in range(args.steps):
        gbs, n = cpu_port_gbs(raw, args.qtype, x, ids, weights, budget_s=args.ref_budget)
        samples.append(gbs)
        experts = n
    value = statistics.median(samples)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": config_dict(args, world),
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": f"{experts} of {EXPERTS} routed experts per step, M={args.m} rows/expert"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def config_dict(args, world):
    return {
        "workload": f"expert_gemm_{args.qtype.lower()}_m{args.m}",
        "experts_per_gpu": EXPERTS, "hidden": HIDDEN, "intermediate": INTER, "qtype": args.qtype,
        "tokens_per_expert": args.m, "rows_per_gpu": EXPERTS * args.m, "top_k": 1,
        "parallelism": (f"ep{world}: each rank's rows routed uniformly over all {EXPERTS * world} experts of "
                        "the ranks, dispatched and combined through peer memory (ExpertAllToAll)")
        if world > 1 else "ep1",
        "l2": "inputs larger than L2 (331 MB packed weights per GPU)",
    }


def b200_arm(args):
    import numpy as np
    import torch

    import qk_b200
    from qk_b200 import _lib
    from qk_b200.experts import expert_parallel
    from qk_b200.parallel import put_expert_bytes

    world, rank, local = init_dist()
    raw = synth_experts(args.qtype, EXPERTS)  # before CUDA init: the encoder pool is spawned
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=device)
    tensors = {k: put_expert_bytes(v, k, args.qtype, HIDDEN, INTER, device=device)
               for k, v in raw.items()}
    fn = expert_parallel(gate_type=args.qtype, up_type=args.qtype, down_type=args.qtype,
                         hidden=HIDDEN, intermediate=INTER)
    stream = torch.cuda.current_stream(device)

    def run_m(m, steps, warmup, profile, sync=True, qtype=None):
        qtype = qtype or args.qtype
        x, ids, weights = workload(m, rank)
        xd = torch.from_numpy(x).to(device).to(torch.bfloat16)
        idd = torch.from_numpy(ids).to(device)
        wd = torch.from_numpy(weights).to(device).to(torch.bfloat16)
        rows = x.shape[0]
        desc = fn.desc(EXPERTS, 0, 1)
        ws = fn.workspace(desc, rows, device)
        out = torch.empty((rows, HIDDEN), dtype=torch.bfloat16, device=device)
        events = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
        for e in events:  # torch creates the CUDA event on its first record
            e.record(stream)
        torch.cuda.synchronize(device)
        ev_ptrs = (ctypes_void_p * 5)(*[e.cuda_event for e in events]) if profile else None

        def step(profiled=False):
            lib = _lib.load()
            if profiled:
                rc = lib.qk_moe_forward_profiled(desc, _lib.ptr(tensors["gate"]), _lib.ptr(tensors["up"]),
                                                 _lib.ptr(tensors["down"]), _lib.ptr(xd), _lib.ptr(idd),
                                                 _lib.ptr(wd), rows, _lib.QK_OUT_BF16, _lib.ptr(out),
                                                 _lib.ptr(ws), ws.numel(), _lib.stream_handle(device),
                                                 ev_ptrs)
            else:
                rc = lib.qk_moe_forward(desc, _lib.ptr(tensors["gate"]), _lib.ptr(tensors["up"]),
                                        _lib.ptr(tensors["down"]), _lib.ptr(xd), _lib.ptr(idd),
                                        _lib.ptr(wd), rows, _lib.QK_OUT_BF16, _lib.ptr(out),
                                        _lib.ptr(ws), ws.numel(), _lib.stream_handle(device))
            _lib.check(rc)

        for _ in range(warmup):
            step()
        torch.cuda.synchronize(device)
        launched = qk_b200.launch_count()
        step()  # one more eager step, counting this library's kernel launches
        launches = qk_b200.launch_count() - launched
        torch.cuda.synchronize(device)
        # capture one step in a CUDA graph so the timed loop is free of host launch gaps
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        graph.replay()
        torch.cuda.synchronize(device)
        if dist and sync:
            dist.barrier()
        torch.cuda.synchronize(device)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(steps):
            graph.replay()
        t1.record(stream)
        torch.cuda.synchronize(device)
        if dist and sync:
            dist.barrier()
        ms = t0.elapsed_time(t1) / steps
        fn.check_status()  # every bounded wait of the last timed call completed
        stage_ms = None
        if profile:  # per-kernel times from events recorded between the launches
            acc = [0.0] * 4
            reps = max(10, min(steps, 200))
            for _ in range(reps):
                step(profiled=True)
                torch.cuda.synchronize(device)
                for i in range(4):
                    acc[i] += events[i].elapsed_time(events[i + 1])
            stage_ms = [a / reps for a in acc]
        fn.check_status()
        nbytes, active = step_bytes(qtype, ids)
        return dict(m=m, ms=ms, bytes=nbytes, active=active, rows=rows, stage_ms=stage_ms, launches=launches,
                    gate_up_bytes=kernel_bytes(qtype, ids), x=x, ids=ids, weights=weights,
                    out=out)

    def run_ep(m, steps, warmup):
        """The expert-parallel step over all ranks (ExpertAllToAll, peer memory): this rank's
        rows routed uniformly over every rank's experts, dispatched, computed by their
        owners and combined back."""
        from qk_b200.ep import ExpertAllToAll

        x, ids, weights = workload(m, rank, world)
        xd = torch.from_numpy(x).to(device).to(torch.bfloat16)
        idd = torch.from_numpy(ids).to(device)
        wd = torch.from_numpy(weights).to(device).to(torch.bfloat16)
        rows = x.shape[0]
        layer = ExpertAllToAll(dist.group.WORLD, gate_type=args.qtype, up_type=args.qtype,
                               down_type=args.qtype, hidden=HIDDEN, intermediate=INTER,
                               experts_per_rank=EXPERTS, top_k=1, max_tokens=rows, device=device)

        def step():
            return layer(tensors["gate"], tensors["up"], tensors["down"], xd, idd, wd)

        for _ in range(warmup):
            step()
        torch.cuda.synchronize(device)
        launched = qk_b200.launch_count()
        step()
        launches = qk_b200.launch_count() - launched
        torch.cuda.synchronize(device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        graph.replay()
        torch.cuda.synchronize(device)
        dist.barrier()
        torch.cuda.synchronize(device)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(steps):
            graph.replay()
        t1.record(stream)
        torch.cuda.synchronize(device)
        dist.barrier()
        ms = t0.elapsed_time(t1) / steps
        layer.check_status()
        return dict(m=m, ms=ms, rows=rows, x=x, ids=ids, weights=weights, out=layer.out[:rows], layer=layer,
                    launches=launches,
                    graph=graph)

    peak, peak_kind = hbm_peak()
    with ClockSampler(local) as clocks:
        # untimed soak so clocks settle before the measured region; no collectives inside,
        # since each rank runs as many soak passes as fit in its own wall time
        soak_end = time.time() + args.soak
        while time.time() < soak_end:
            run_m(args.m, 20, 1, False, sync=False)
        res = run_m(args.m, args.steps, args.warmup, True)
        ep = run_ep(args.m, args.steps, args.warmup) if world > 1 else None
    ms = res["ms"] if ep is None else ep["ms"]
    if dist:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    if ep is None:
        step_total = res["bytes"]
    else:
        step_total, _ = ep_step_bytes(args.qtype, args.m, world)
    value = step_total / (ms * 1e-3) / 1e9

    # launches per step, counted by the library around one eager step: route, dispatch,
    # gate/up, down (and the combine unless the routes are top-1); the expert-parallel step
    # adds the dispatch, the wait for the sources and the final combine
    launches_per_step = res["launches"] if ep is None else ep["launches"]

    # e2e through the public call with host buffers
    if ep is None:
        def call(xs, ids_s, ws_s, out_s):
            return fn(tensors["gate"], tensors["up"], tensors["down"], xs, ids_s, ws_s)
    else:
        def call(xs, ids_s, ws_s, out_s):
            return ep["layer"](tensors["gate"], tensors["up"], tensors["down"], xs, ids_s, ws_s, out=out_s)
    e2e = e2e_measure(call, device, args, res if ep is None else ep, step_total // world if ep else res["bytes"])

    sweep = []
    if not args.no_sweep and rank == 0 and world == 1:
        for m in SWEEP_M:
            r = run_m(m, max(5, args.steps // 4), 3, True)
            sweep.append(sweep_row(args.qtype, r, peak))
        other = "Q4_K" if args.qtype == "Q6_K" else "Q6_K"
        raw_o = synth_experts(other, EXPERTS)
        tensors_o = {k: put_expert_bytes(v, k, other, HIDDEN, INTER, device=device) for k, v in raw_o.items()}
        fn_o = expert_parallel(gate_type=other, up_type=other, down_type=other, hidden=HIDDEN, intermediate=INTER)
        saved = (tensors, fn)
        tensors, fn = tensors_o, fn_o
        for m in SWEEP_M:
            r = run_m(m, max(5, args.steps // 4), 3, True, qtype=other)
            sweep.append(sweep_row(other, r, peak))
        tensors, fn = saved
        del tensors_o, raw_o

    # parity of the timed step: a seeded sample of output rows against the oracle (with
    # several ranks, of the expert-parallel step: every rank holds the same 128 experts'
    # bytes, so global expert g computes with the bytes of expert g % 128)
    parity = None
    if rank == 0:
        if ep is None:
            parity = moe_parity(raw, args.qtype, res)
        else:
            parity = moe_parity(raw, args.qtype, dict(ep, ids=ep["ids"] % EXPERTS))
    layer_ep = ep_layer_report(device, dist, world, rank, args) if not args.no_ep_layer else None

    gate_up_ms = res["stage_ms"][1]
    achieved = res["gate_up_bytes"] / (gate_up_ms * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": config_dict(args, world),
        "rows_per_s": res["rows"] * world / (ms * 1e-3),
        "stage_ms": {"route_dispatch": res["stage_ms"][0], "gate_up": res["stage_ms"][1],
                     "down": res["stage_ms"][2], "combine": res["stage_ms"][3]},
        "roofline": {"kernel": f"umma_proj_kernel<{args.qtype}, gate/up>",
                     "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": peak_kind,
                     "traffic": ncu_traffic(args.qtype, args.m)},
        "e2e": e2e,
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks.summary(),
    }
    if ep is not None:
        t = torch.tensor([res["ms"]], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        local_ms = float(t.item())
        line["expert_parallel"] = {
            "step_ms": ms, "local_only_ms": local_ms, "exchange_overhead_ms": ms - local_ms,
            "exchange_share": (ms - local_ms) / ms,
            "exchange": "peer-memory stores over NVLink (dispatch of x rows, return of FP32 partials)",
            "bytes_over_nvlink_per_rank": int(ep["rows"] * (world - 1) / world * HIDDEN * (2 + 4)),
            "local_only": "the same rows and kernels on this rank's own 128 experts, no exchange"}
    if layer_ep is not None:
        line["ep_layer"] = layer_ep
    if sweep:
        line["sweep"] = sweep
    if parity is not None:
        line["parity"] = parity
    if rank == 0 and not args.no_attention:
        line["attention"] = attention_report(device, args)
        line["qsa_select"] = qsa_report(device, args)
        errs = [r["parity_max_rel_err"] for r in line["attention"]["configs"]]
        line["parity"]["attention_rows"] = len(errs)
        line["parity"]["attention_max_rel_err"] = max(errs)
        line["parity"]["ok"] = line["parity"]["ok"] and max(errs) < PARITY_TOL
    if parity is not None:
        line["parity_checked"] = bool(line["parity"]["ok"])
    if rank == 0 and world == 1:
        line["layer"] = layer_report(raw, device, args)
    if not args.no_stack:
        stack = stack_report(device, args, dist)
        if rank == 0:
            line["stack"] = stack
    if not args.no_generation:
        gen = generation_report(device, dist, args)
        if rank == 0 and gen is not None:
            line["generation"] = gen
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gbs, experts = cpu_port_gbs(raw, args.qtype, res["x"], res["ids"], res["weights"],
                                    budget_s=args.ref_budget)
        line["cpu_baseline"] = {"value": gbs, "unit": "GB/s", "cores": os.cpu_count() or 1,
                                "kind": "port",
                                "sample": f"{experts} of {res['active']} routed experts, M={args.m} rows/expert"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


ATTN_CONFIGS = ((1, 4096), (8, 4096), (32, 4096), (1, 32768), (8, 32768), (32, 32768))
ATTN_SLOT_BYTES = 2 * 512 + 2 * 16 * 2  # K + V codes (2 kv heads x 256) + BF16 scales (16 groups)


EP_LAYER_EXPERTS, EP_LAYER_TOPK, EP_LAYER_TOKENS = 512, 10, 512


def ep_layer_report(device, dist, world, rank, args):
    """The routed-expert layer of BASELINE.json configs[3] across the ranks: 512 Q6_K experts
    (hidden 2048, intermediate 512), top-10 routes, a global batch of 512 decode tokens
    (strong scaling: 512 / world tokens and 512 / world experts per rank). Tokens go to the
    experts' owners and back through peer memory (ExpertAllToAll; with one rank the same
    layer exchanges with itself). Experts are random code bytes with fixed block scales (the
    kernels' cost does not depend on the values); routes are 10 distinct experts per token
    (seed [4, rank]) with softmax-like BF16 weights. One step is one CUDA-graph replay.
    Bytes = the distinct experts all ranks' routes name x packed bytes + every rank's x rows
    read and output rows written."""
    import numpy as np
    import torch

    from qk_b200.decoder import synthetic_expert_bytes
    from qk_b200.ep import ExpertAllToAll
    from qk_b200.parallel import expert_shape, put_expert_bytes

    E, k, T = EP_LAYER_EXPERTS, EP_LAYER_TOPK, EP_LAYER_TOKENS
    if E % world or T % world:
        return None
    per, tokens = E // world, T // world
    g = torch.Generator(device=device).manual_seed(100 + rank)
    tensors = {}
    for kind in ("gate", "up", "down"):
        rows, width = expert_shape(kind, HIDDEN, INTER)
        raw = synthetic_expert_bytes(args.qtype, per, rows, width, g, device)
        tensors[kind] = put_expert_bytes(raw, kind, args.qtype, HIDDEN, INTER, device=device)
        del raw

    def routes(r):
        rng = np.random.default_rng([4, r])
        ids = np.argsort(rng.random((tokens, E)), axis=1)[:, :k].astype(np.int32)
        w = rng.random((tokens, k)).astype(np.float32)
        return ids, w / w.sum(axis=1, keepdims=True)

    ids, w = routes(rank)
    x = torch.randn((tokens, HIDDEN), device=device, generator=g).to(torch.bfloat16)
    idd = torch.from_numpy(ids).to(device)
    wd = torch.from_numpy(w).to(device).to(torch.bfloat16)
    layer = ExpertAllToAll(dist.group.WORLD if dist else None, gate_type=args.qtype, up_type=args.qtype,
                           down_type=args.qtype, hidden=HIDDEN, intermediate=INTER, experts_per_rank=per, top_k=k,
                           max_tokens=tokens, device=device)
    stream = torch.cuda.current_stream(device)

    def step():
        layer(tensors["gate"], tensors["up"], tensors["down"], x, idd, wd)

    for _ in range(3):
        step()
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    graph.replay()
    torch.cuda.synchronize(device)
    if dist:
        dist.barrier()
    steps = max(10, args.steps // 2)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(steps):
        graph.replay()
    t1.record(stream)
    torch.cuda.synchronize(device)
    ms = t0.elapsed_time(t1) / steps
    if dist:
        dist.barrier()
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    layer.check_status()
    del graph
    torch.cuda.synchronize(device)
    if dist:
        dist.barrier()
    layer.close()
    every = np.concatenate([routes(r)[0].reshape(-1) for r in range(world)])
    active = len(np.unique(every))
    nbytes = active * packed_bytes_per_expert(args.qtype) + T * HIDDEN * 2 * 2
    peak, _ = hbm_peak()
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"workload": "configs[3] routed-expert layer: 512 Q6_K experts, top-10, global batch 512, "
                        "strong scaling over the ranks", "experts_per_rank": per, "tokens_per_rank": tokens,
            "qtype": args.qtype, "ms_per_step": ms, "tokens_per_s": T / (ms * 1e-3), "gbs": gbs,
            "frac_of_aggregate_hbm": gbs / (peak * world), "active_experts": active,
            "exchange": "peer memory (ExpertAllToAll)" if world > 1 else "one rank (the exchange writes to itself)"}


def generation_report(device, dist, args):
    """the 48-layer synthetic MoE model with every expert Q4_K (512
    routed, top-10, + 1 shared), batched static generation of 64 sequences: a prefill of 2048
    random prompt ids (uniform over a vocabulary of 151936, embedding N(0, 0.02), tied output
    head) and 512 greedy decode steps (checked_argmax), end to end on the device. With N
    ranks the 64 sequences are split 64 / N per rank (strong scaling): attention data
    parallel, experts sharded with the exchange through peer memory. Also the prefill-regime
    grouped GEMM of the last layer (1 GPU: 131072 tokens x 11 routes, ~2560 tokens per routed
    expert): its gate/up and down passes' TFLOP/s against the measured sustained BF16 peak."""
    import ctypes

    import torch

    from qk_b200.decoder import StackConfig, SyntheticDecoder
    from qk_b200.generate import StaticGeneration

    world = dist.get_world_size() if dist else 1
    seqs, prompt, new = args.gen_batch, args.gen_prompt, args.gen_new
    if seqs % world:
        return None
    cfg = StackConfig(layers=args.stack_layers, qtype="Q4_K", context=prompt + new)
    t_build = time.time()
    model = SyntheticDecoder(cfg, device, seed=11, group=dist.group.WORLD if dist else None)
    gen = StaticGeneration(model, seqs // world, prompt, new, seed=0)
    torch.cuda.synchronize(device)
    build_s = time.time() - t_build
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
    if world == 1:
        for e in ev:
            e.record()
        torch.cuda.synchronize(device)
        gen.moe_events = (ctypes.c_void_p * 5)(*[e.cuda_event for e in ev])
    gen.capture()  # the decode step's graph (its warm-up step is undone)
    torch.cuda.synchronize(device)
    if dist:
        dist.barrier()
    stream = torch.cuda.current_stream(device)
    t = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    t[0].record(stream)
    gen.prefill()
    t[1].record(stream)
    gen.decode()
    t[2].record(stream)
    torch.cuda.synchronize(device)
    prefill_ms, decode_ms = t[0].elapsed_time(t[1]), t[1].elapsed_time(t[2])
    nonfinite = int(gen.nonfinite.item())
    if dist:
        tt = torch.tensor([prefill_ms, decode_ms], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        prefill_ms, decode_ms = float(tt[0]), float(tt[1])
        dist.barrier()
    total_ms = prefill_ms + decode_ms
    out = {"workload": "configs[4]: 48-layer MoE model, Q4_K experts (512 top-10 + shared), static generation",
           "sequences": seqs, "prompt_tokens": prompt, "new_tokens": new, "vocab": 151936,
           "sequences_per_gpu": seqs // world, "build_s": build_s,
           "prefill_ms": prefill_ms, "decode_ms": decode_ms, "end_to_end_ms": total_ms,
           "generated_tokens_per_s": seqs * new / (total_ms * 1e-3),
           "prefill_tokens_per_s": seqs * prompt / (prefill_ms * 1e-3),
           "decode_tokens_per_s": seqs * (new - 1) / (decode_ms * 1e-3),
           "nonfinite_logits": nonfinite,
           "parallelism": "1 GPU" if world == 1 else f"ep{world}: attention data parallel, experts sharded"}
    if world == 1:
        st = [ev[i].elapsed_time(ev[i + 1]) for i in range(4)]
        routes = seqs * prompt * (cfg.top_k + 1)
        sustained = peak_tflops("bf16_tflops_sustained")
        gu = routes * 2 * (2 * cfg.intermediate * cfg.hidden) / (st[1] * 1e-3) / 1e12
        dn = routes * 2 * (cfg.intermediate * cfg.hidden) / (st[2] * 1e-3) / 1e12
        out["prefill_grouped_gemm"] = {
            "layer": "last", "tokens": seqs * prompt, "routes": routes,
            "stage_ms": dict(zip(("route_dispatch", "gate_up", "down", "combine"), st)),
            "gate_up_tflops": gu, "down_tflops": dn, "peak_tflops": sustained,
            "gate_up_frac": gu / sustained, "down_frac": dn / sustained,
            "kernel": "umma_prefill_kernel (256-token chunks, tcgen05 kind::f16, A and B in shared memory)"}
    gen.close()
    del gen, model
    torch.cuda.synchronize(device)
    return out


def peak_tflops(key="bf16_tflops"):
    try:
        return float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())[key])
    except (OSError, KeyError, ValueError):
        return 1400.0 if "sustained" in key else 1590.0


def flushed_graph_times(call, device, reps, flush):
    """Device times (ms) of `reps` replays of `call` captured in a CUDA graph, each after an
    L2 flush (`flush`, a buffer larger than L2, zeroed). The graph keeps the host's per-call
    work (argument checks, tensor map encoding, launches) out of the timed region: issued
    eagerly, it can reach the GPU after the flush has drained and leave an idle gap between
    the events."""
    import torch

    stream = torch.cuda.current_stream(device)
    for _ in range(3):
        call()
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        call()
    graph.replay()
    torch.cuda.synchronize(device)
    times = []
    for _ in range(reps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        graph.replay()
        e1.record(stream)
        torch.cuda.synchronize(device)
        times.append(e0.elapsed_time(e1))
    del graph
    return times


def attention_inputs(device, batch, ctx):
    """Inputs of one configs[2] call: 16 q / 2 kv heads, head dim 256, one query token per
    sequence, every slot of the context attended through a page table that is a random
    permutation (seed 0) of 256-token pages. K/V codes and BF16 scales are synthetic
    (uniform codes, scales in [0.001, 0.021)); the kernel's cost does not depend on their
    values. The same tensors feed the timed sweep and the parity tests."""
    import numpy as np
    import torch

    from qk_b200 import _lib

    lib = _lib.load()
    g = torch.Generator(device=device).manual_seed(batch * 7 + ctx)
    k = torch.randint(-127, 128, (batch, ctx, 512), dtype=torch.int8, device=device, generator=g)
    v = torch.randint(-127, 128, (batch, ctx, 512), dtype=torch.int8, device=device, generator=g)
    ks = (torch.rand((batch * 16, ctx), device=device, generator=g) * 0.02 + 0.001).to(torch.bfloat16)
    vs = (torch.rand((batch * 16, ctx), device=device, generator=g) * 0.02 + 0.001).to(torch.bfloat16)
    rng = np.random.default_rng(0)
    pages = ctx // 256
    table = np.stack([rng.permutation(pages) for _ in range(batch)])
    slots = np.arange(ctx)
    idx = torch.from_numpy(np.ascontiguousarray((table[:, slots // 256] * 256 + slots % 256).astype(np.int32))).to(device)
    lengths = torch.full((batch,), ctx - 1, dtype=torch.int32, device=device)
    q = torch.randn((batch, 16, 256), device=device, generator=g).to(torch.bfloat16)
    out = torch.empty((batch, 16, 256), dtype=torch.bfloat16, device=device)
    need = int(lib.qk_kv_q8_attention_workspace_bytes(batch, ctx, 16, 2, 256))
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device=device)
    return dict(batch=batch, ctx=ctx, device=device, k=k, v=v, ks=ks, vs=vs, idx=idx, lengths=lengths, q=q,
                out=out, ws=ws, need=need)


def attention_call(inp):
    """One decode attention call through the C ABI on `inp` (attention_inputs); returns out."""
    from qk_b200 import _lib

    lib = _lib.load()
    batch, ctx, need = inp["batch"], inp["ctx"], inp["need"]
    _lib.check(lib.qk_kv_q8_decode_attention(
        _lib.ptr(inp["q"]), _lib.ptr(inp["k"]), _lib.ptr(inp["v"]), _lib.ptr(inp["ks"]), _lib.ptr(inp["vs"]),
        _lib.ptr(inp["idx"]), None, _lib.ptr(inp["lengths"]), None, batch, ctx, ctx, 16, 2, 256,
        _lib.ptr(inp["out"]), _lib.ptr(inp["ws"]) if need else None, need, _lib.stream_handle(inp["device"])))
    return inp["out"]


def attention_parity(inp, row):
    """Max relative error of row `row` of the last call's output against the oracle
    (attention_cache.py:152-170 restated)."""
    import numpy as np
    import torch

    from oracle import kv

    def f32(t):
        return t.detach().to(torch.float32).cpu().numpy()

    ctx = inp["ctx"]
    sel = inp["idx"][row : row + 1].cpu().numpy()
    codes = {n: inp[n][row : row + 1].cpu().numpy() for n in ("k", "v")}
    planes = {n: f32(inp[n + "s"][row * 16 : (row + 1) * 16]) for n in ("k", "v")}
    keys = kv.read_quantized(codes["k"], planes["k"], sel, 2, 256)
    values = kv.read_quantized(codes["v"], planes["v"], sel, 2, 256)
    mask = np.arange(ctx)[None, :] <= int(inp["lengths"][row])
    expected = kv.attention(f32(inp["q"][row : row + 1]), keys, values, mask)
    got = f32(inp["out"][row : row + 1])
    return float(np.max(np.abs(got - expected)) / max(np.max(np.abs(expected)), 1e-30))


def attention_sweep(device, reps=20, configs=ATTN_CONFIGS, parity=False):
    """Q8 KV decode attention over `configs`, inputs from
    attention_inputs. Bytes per step = B * ctx * 1088 (codes + scales); each timed call
    follows an L2 flush. With `parity`, one row of each configuration's output is checked
    against the oracle after the timing."""
    import torch

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    results = []
    for batch, ctx in configs:
        inp = attention_inputs(device, batch, ctx)
        times = flushed_graph_times(lambda: attention_call(inp), device, reps, flush)
        ms = statistics.median(times)
        nbytes = batch * ctx * ATTN_SLOT_BYTES
        r = {"batch": batch, "ctx": ctx, "us": ms * 1e3, "gbs": nbytes / (ms * 1e-3) / 1e9,
             "tokens_per_s": batch / (ms * 1e-3)}
        if parity:
            r["parity_max_rel_err"] = attention_parity(inp, batch - 1)
        results.append(r)
        del inp
    return results


def attention_report(device, args):
    peak_gbs, _ = hbm_peak()
    attn = attention_sweep(device, args.attn_reps, parse_attn_configs(args.attn_configs), parity=True)
    for r in attn:
        r["frac"] = r["gbs"] / peak_gbs
    return {"kernel": "attn_stream_kernel + attn_merge_kernel (Q8 KV, 16q/2kv, hd 256)",
            "bytes_per_slot": ATTN_SLOT_BYTES, "l2": "flushed before every call", "configs": attn}


def layer_report(raw, device, args):
    """BASELINE.json configs[0] on one GPU: one routed-MoE layer call (router top-4 of 64 +
    expert SwiGLU + combine) on T = 8 tokens (N(0, 1), seed 0), router N(0, 0.02) FP32
    (seed 2), the first 64 of the bench's Q6_K experts (N(0, 0.02), seed 1). The layer touches
    at most 32 experts (82 MB, less than L2), so L2 is flushed before every timed call."""
    import numpy as np
    import torch

    from qk_b200.experts import expert_parallel
    from qk_b200.parallel import put_expert_bytes
    from qk_b200.routing import routes

    count, T, k = 64, 8, 4
    tensors = {n: put_expert_bytes(raw[n][:count], n, args.qtype, HIDDEN, INTER, device=device) for n in raw}
    x = torch.from_numpy(np.random.default_rng(0).normal(size=(T, HIDDEN)).astype(np.float32)).to(device).bfloat16()
    router = torch.from_numpy(np.random.default_rng(2).normal(0, 0.02, (count, HIDDEN)).astype(np.float32)).to(device)
    fn = expert_parallel(gate_type=args.qtype, up_type=args.qtype, down_type=args.qtype, hidden=HIDDEN,
                         intermediate=INTER)
    stream = torch.cuda.current_stream(device)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)

    def call():
        ids, w = routes(x, router, k)
        return fn(tensors["gate"], tensors["up"], tensors["down"], x, ids, w), ids

    times = flushed_graph_times(call, device, args.attn_reps, flush)
    _, ids = call()
    ms = statistics.median(times)
    active = int(torch.unique(ids).numel())
    nbytes = active * packed_bytes_per_expert(args.qtype) + count * HIDDEN * 4 + T * HIDDEN * 4
    peak, _ = hbm_peak()
    return {"workload": "configs[0]: one routed-MoE layer, T=8, top-4 of 64 experts, 1 GPU", "qtype": args.qtype,
            "us": ms * 1e3, "tokens_per_s": T / (ms * 1e-3), "active_experts": active,
            "gbs": nbytes / (ms * 1e-3) / 1e9, "frac": nbytes / (ms * 1e-3) / 1e9 / peak,
            "l2": "flushed before every call", "launches_per_call": 6}


def stack_report(device, args, dist=None):
    """Decode steps of the synthetic 48-layer MoE decoder stack (
    hidden 2048, Q8-cache GQA 16 q / 2 kv heads of 256 at context 8192 through a random page
    table of 256-slot pages, 512 routed experts top-10 + 1 shared expert, intermediate 512,
    Q6_K) on one GPU, one CUDA-graph replay per step. tokens/s = B / step time; GB/s = the
    step's algorithmic bytes (distinct routed experts per layer x packed bytes, the dense
    weights, the K/V codes and scales of every attended slot) / step time."""
    import torch

    from qk_b200.decoder import StackConfig, SyntheticDecoder

    cfg = StackConfig(layers=args.stack_layers, qtype=args.qtype, down_qtype=args.stack_down_qtype)
    peak, _ = hbm_peak()
    world = dist.get_world_size() if dist else 1
    t_build = time.time()
    model = SyntheticDecoder(cfg, device, seed=1, group=dist.group.WORLD if dist else None)
    torch.cuda.synchronize(device)
    build_s = time.time() - t_build
    stream = torch.cuda.current_stream(device)
    rows = []
    for batch in args.stack_batches:
        state = model.state(batch, seed=2)
        for _ in range(2):
            state.step()
        torch.cuda.synchronize(device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            state.step()
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize(device)
        if dist:
            dist.barrier()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        steps = args.stack_steps
        t0.record(stream)
        for _ in range(steps):
            graph.replay()
        t1.record(stream)
        torch.cuda.synchronize(device)
        ms = t0.elapsed_time(t1) / steps
        nbytes, distinct = state.step_bytes()
        if dist:
            t = torch.tensor([ms, float(nbytes)], device=device, dtype=torch.float64)
            dist.all_reduce(t[:1], op=dist.ReduceOp.MAX)
            dist.all_reduce(t[1:], op=dist.ReduceOp.SUM)
            ms, nbytes = float(t[0]), int(t[1])
        kernels, gemms = state.launches_per_step()
        tokens = batch * world
        rows.append({"batch": tokens, "batch_per_gpu": batch, "ms_per_step": ms, "tokens_per_s": tokens / (ms * 1e-3),
                     "gbs": nbytes / (ms * 1e-3) / 1e9, "frac": nbytes / (ms * 1e-3) / 1e9 / (peak * world),
                     "bytes_per_step": nbytes, "distinct_experts_per_layer": statistics.mean(distinct),
                     "launches_per_step": {"library": kernels, "cublas_gemm": gemms}})
        del graph
        torch.cuda.synchronize(device)
        if dist:
            dist.barrier()
        state.close()
        del state
        torch.cuda.synchronize(device)
    return {"workload": ("synthetic 48-layer MoE decoder stack (configs[3]), 1 GPU" if world == 1 else
                         f"synthetic 48-layer MoE decoder stack (configs[3]), expert parallel over {world} GPUs: "
                         "each rank decodes batch_per_gpu sequences (attention data parallel) and holds "
                         f"{cfg.experts // world} routed experts + the shared expert per layer; tokens cross "
                         "ranks through peer memory (ExpertAllToAll)"),
            "layers": cfg.layers, "context": cfg.context, "experts": cfg.experts, "top_k": cfg.top_k,
            "shared_experts": 1, "qtype": cfg.qtype, "down_qtype": cfg.down_qtype or cfg.qtype,
            "weights": "synthetic (random code bytes, fixed block scales)",
            "l2": "inputs larger than L2 (packed experts of 48 layers)", "build_s": build_s, "batches": rows}


def qsa_report(device, args):
    """Sparse token selection (attention_cache.py:84-125) at the attention sweep's long
    context: B in {1, 8, 32} rows, context 32768 -> 8192 index blocks of 128 BF16 values
    (ratio 4), 4 indexer heads, budget 2048 tokens (K = 512 blocks). Bytes per call = the
    index keys read (B x 8192 x 256 B) + the scores written and read back; L2 is flushed
    before every call."""
    import torch

    from qk_b200 import _lib

    stream = torch.cuda.current_stream(device)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    peak, _ = hbm_peak()
    rows = []
    for batch in (1, 8, 32):
        blocks, heads, dim, ratio, budget = 8192, 4, 128, 4, 2048
        g = torch.Generator(device=device).manual_seed(batch)
        q = torch.randn((batch, heads, dim), device=device, generator=g).to(torch.bfloat16)
        k = torch.randn((batch, blocks, dim), device=device, generator=g).to(torch.bfloat16)
        lengths = torch.full((batch,), blocks * ratio - 1, dtype=torch.int32, device=device)
        scores = torch.empty((batch, blocks), dtype=torch.float32, device=device)
        K = budget // ratio
        idx = torch.empty((batch, K * ratio + ratio - 1), dtype=torch.int32, device=device)
        val = torch.empty(idx.shape, dtype=torch.uint8, device=device)
        def call():
            st = _lib.stream_handle(device)  # the current stream: the capture stream under a graph
            _lib.call("qk_qsa_block_scores", _lib.ptr(q), _lib.ptr(k), _lib.ptr(lengths), batch, heads, dim, blocks,
                      ratio, _lib.ptr(scores), st)
            _lib.call("qk_qsa_select", _lib.ptr(scores), _lib.ptr(lengths), batch, blocks, ratio, budget,
                      _lib.ptr(idx), _lib.ptr(val), st)

        times = flushed_graph_times(call, device, args.attn_reps, flush)
        ms = statistics.median(times)
        nbytes = batch * blocks * (dim * 2 + 8)
        rows.append({"batch": batch, "us": ms * 1e3, "gbs": nbytes / (ms * 1e-3) / 1e9,
                     "frac": nbytes / (ms * 1e-3) / 1e9 / peak})
    return {"kernel": "qsa_scores_kernel + qsa_select_kernel (8192 blocks x 128, 4 heads, K = 512)",
            "l2": "flushed before every call", "configs": rows}


def parse_attn_configs(text):
    if not text:
        return ATTN_CONFIGS
    return tuple(tuple(int(v) for v in item.split("x")) for item in text.split(","))


def attention_only(args):
    """Only the Q8 KV decode attention sweep (one GPU), as one JSON line."""
    import torch

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    print(json.dumps({"attention": attention_report(device, args)}), flush=True)
    return 0


def e2e_measure(call, device, args, res, step_bytes_rank):
    """Public-call throughput with pinned host inputs/outputs copied every step.

    Each step copies its x, ids and weights host -> device, runs the public ``fn`` and
    copies its output device -> host. The three run on their own streams with two buffer
    slots, so step i's compute overlaps step i+1's input copy and step i-1's output copy,
    as a serving loop would pipeline them; events order each slot's reuse."""
    import torch

    x, ids, weights = res["x"], res["ids"], res["weights"]
    rows = x.shape[0]
    x_h = torch.from_numpy(x).to(torch.bfloat16).pin_memory()
    ids_h = torch.from_numpy(ids).pin_memory()
    w_h = torch.from_numpy(weights).to(torch.bfloat16).pin_memory()
    slots = 2
    out_h = [torch.empty((rows, HIDDEN), dtype=torch.bfloat16).pin_memory() for _ in range(slots)]
    out_d = [torch.empty((rows, HIDDEN), dtype=torch.bfloat16, device=device) for _ in range(slots)]
    x_d = [torch.empty_like(x_h, device=device) for _ in range(slots)]
    ids_d = [torch.empty_like(ids_h, device=device) for _ in range(slots)]
    w_d = [torch.empty_like(w_h, device=device) for _ in range(slots)]
    h2d, comp, d2h = (torch.cuda.Stream(device) for _ in range(3))
    copied = [torch.cuda.Event() for _ in range(slots)]
    computed = [torch.cuda.Event() for _ in range(slots)]
    read = [torch.cuda.Event() for _ in range(slots)]

    def step(i):
        s = i % slots
        with torch.cuda.stream(h2d):
            if i >= slots:
                h2d.wait_event(computed[s])  # slot s inputs free once step i - 2 computed
            x_d[s].copy_(x_h, non_blocking=True)
            ids_d[s].copy_(ids_h, non_blocking=True)
            w_d[s].copy_(w_h, non_blocking=True)
            copied[s].record(h2d)
        with torch.cuda.stream(comp):
            comp.wait_event(copied[s])
            out = call(x_d[s], ids_d[s], w_d[s], out_d[s])
            computed[s].record(comp)
        with torch.cuda.stream(d2h):
            d2h.wait_event(computed[s])
            if i >= slots:
                d2h.wait_event(read[s])
            out_h[s].copy_(out, non_blocking=True)
            out.record_stream(d2h)
            read[s].record(d2h)

    for i in range(max(args.warmup, slots)):
        step(i)
    torch.cuda.synchronize(device)
    steps = max(3, args.steps // 2)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(h2d)
    for i in range(steps):
        step(i)
    t1.record(d2h)
    torch.cuda.synchronize(device)
    ms = t0.elapsed_time(t1) / steps
    h2d_bytes = x_h.numel() * 2 + ids_h.numel() * 4 + w_h.numel() * 2
    d2h_bytes = out_h[0].numel() * 2
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return {"value": step_bytes_rank * world / (ms * 1e-3) / 1e9, "unit": "GB/s",
            "ms_per_step": ms, "h2d_bytes_per_step": h2d_bytes, "d2h_bytes_per_step": d2h_bytes,
            "pipeline": "H2D, compute and D2H on separate streams, 2 buffer slots"}


import ctypes  # noqa: E402

ctypes_void_p = ctypes.c_void_p


def main():
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=200)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=("b200", "reference"), default="b200")
    parser.add_argument("--m", type=int, default=16, help="tokens per expert")
    parser.add_argument("--qtype", choices=("Q6_K", "Q4_K"), default="Q6_K")
    parser.add_argument("--soak", type=float, default=1.0, help="untimed seconds before timing")
    parser.add_argument("--no-sweep", action="store_true",
                        help="skip the M in {1,4,16,64,256} sweep over Q6_K and Q4_K")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-attention", action="store_true", help="skip the Q8 KV attention sweep")
    parser.add_argument("--attention-only", action="store_true",
                        help="only the Q8 KV attention sweep (no MoE step, no contract line)")
    parser.add_argument("--attn-configs", default="",
                        help="attention configs as BxCTX[,BxCTX...] (default: the six of the sweep)")
    parser.add_argument("--attn-reps", type=int, default=20)
    parser.add_argument("--no-stack", action="store_true", help="skip the 48-layer decoder stack")
    parser.add_argument("--no-ep-layer", action="store_true", help="skip the configs[3] expert-parallel layer")
    parser.add_argument("--no-generation", action="store_true", help="skip the configs[4] static generation")
    parser.add_argument("--generation-only", action="store_true", help="only the configs[4] static generation (one GPU)")
    parser.add_argument("--gen-batch", type=int, default=64)
    parser.add_argument("--gen-prompt", type=int, default=2048)
    parser.add_argument("--gen-new", type=int, default=512)
    parser.add_argument("--qsa-only", action="store_true", help="only the sparse token selection (one GPU)")
    parser.add_argument("--stack-only", action="store_true", help="only the decoder stack (one GPU)")
    parser.add_argument("--stack-batches", type=lambda t: [int(v) for v in t.split(",")], default=[1, 8, 64])
    parser.add_argument("--stack-layers", type=int, default=48)
    parser.add_argument("--stack-down-qtype", choices=("Q6_K", "Q4_K", "Q8_0"), default=None,
                        help="down projection type of the stack's experts (default: --qtype)")
    parser.add_argument("--stack-steps", type=int, default=10)
    parser.add_argument("--ref-budget", type=float, default=10.0,
                        help="seconds of CPU work per reference sample")
    args = parser.parse_args()
    if args.warmup < 3:
        parser.error("--warmup must be >= 3")
    if args.impl == "reference":
        return reference_arm(args)
    if args.attention_only:
        return attention_only(args)
    if args.qsa_only:
        import torch

        device = torch.device("cuda", 0)
        torch.cuda.set_device(device)
        print(json.dumps({"qsa_select": qsa_report(device, args)}), flush=True)
        return 0
    if args.generation_only:
        import torch

        device = torch.device("cuda", 0)
        torch.cuda.set_device(device)
        print(json.dumps({"generation": generation_report(device, None, args)}), flush=True)
        return 0
    if args.stack_only:
        import torch

        device = torch.device("cuda", 0)
        torch.cuda.set_device(device)
        print(json.dumps({"stack": stack_report(device, args)}), flush=True)
        return 0
    return b200_arm(args)


if __name__ == "__main__":
    sys.exit(main())
