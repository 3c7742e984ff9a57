"""Benchmark: RecoverSSM verify + commit seq-steps/sec on B200.

One step = one speculative verify over a batch (gdn_recoverssm_verify) plus the
commit of the accepted prefixes (GDNRecoverSSMCommitContext.commit: plan +
fold; `--conv-dim D` adds the conv compaction of D channels) on one GDN layer
of the named configuration (default: config 2, B=512, H=16, HV=32, K=V=128,
Q=4, prefix-cache align mode with 64-token blocks, bf16 q/k/v, fp32 state pool
of 4096 pages, packed fp32 records).  Synthetic, seeded inputs of those
shapes.  `--gated` verifies through the fused-gating entry point.

The headline loop replays the steps back to back from a CUDA graph of whole
steps (`--launch eager` issues each step from Python instead), nothing between
the launches; a second pass with CUDA events between the launches gives the
per-kernel split.  `e2e` repeats the step through the public API with the
inputs copied from pinned host memory and the output copied back, every step.
`--impl reference` times the CPU restatement of the reference's path
(oracle/cpu_executors.py) on the host cores instead.

Multi-GPU (torchrun, one process per GPU): value heads (and their key heads)
are sharded across ranks, each rank owning the state pool of its heads; the
launches are independent, with no collective in the path (host barrier and a
MAX reduction of the timings only, outside the timed region).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl b200|reference]
                    [--gated] [--conv-dim D] [--no-cpu-baseline]
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

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "gdn-recoverssm-ascend_b200"))
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

METRIC = "verify+commit seq-steps/sec"
UNIT = "seq-steps/s"


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _traffic_profile(key, reduced):
    """Per-launch DRAM traffic (bytes) of the named kernel at a config's full
    size (``key`` = "<kernel>_config<N>"), from the committed ncu summaries;
    None for reduced workloads or when no capture exists."""
    p = ROOT / "profiles" / "traffic.json"
    if reduced or not p.exists():
        return None
    entry = json.loads(p.read_text()).get(key)
    return int(entry) if entry is not None else None


class ClockSampler:
    """SM clock and clock-event reasons of one GPU, sampled every millisecond
    through NVML on a background thread while the timed passes run (falls
    back to ``nvidia-smi -lms 200`` without NVML)."""

    REASONS = (("hw_slowdown", 0x8), ("sw_thermal_slowdown", 0x20), ("hw_thermal_slowdown", 0x40),
               ("sw_power_cap", 0x4))

    def __init__(self, device):
        self.device = device
        self.rows = []  # (sm MHz, power W, reason bits)
        self.max_mhz = None
        self.source = "nvml"
        self._stop = None
        self._thread = None
        self._smi = None

    def _handle(self):
        import pynvml

        pynvml.nvmlInit()
        try:
            p = torch.cuda.get_device_properties(self.device)
            bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.device.index or 0)

    def __enter__(self):
        import threading

        try:
            nv, h = self._handle()
        except Exception:
            self.source = "nvidia-smi"
            self._smi = _SmiSampler(self.device.index or 0).__enter__()
            return self
        self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        self._stop = threading.Event()

        def run():
            while not self._stop.is_set():
                try:
                    self.rows.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                                      nv.nvmlDeviceGetPowerUsage(h) / 1000.0, int(reasons(h))))
                except Exception:
                    pass
                self._stop.wait(0.001)

        self._thread = threading.Thread(target=run, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._smi is not None:
            self._smi.__exit__(*exc)
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)

    def summary(self):
        if self._smi is not None:
            return self._smi.summary()
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["no samples"], "source": self.source}
        active = sorted({name for _, _, bits in self.rows for name, bit in self.REASONS if bits & bit})
        return {"sm_mhz": statistics.median(r[0] for r in self.rows), "sm_max_mhz": self.max_mhz,
                "reasons": active, "samples": len(self.rows), "sm_mhz_min": min(r[0] for r in self.rows),
                "power_w_max": max(r[1] for r in self.rows), "source": "nvml, every 1 ms over the timed passes"}


class _SmiSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu_index = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or not self.path:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "source": "nvidia-smi, every 200 ms",
                "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def cpu_baseline(cfg, *, rows_sample, seed=0, repeats=1, gated=False):
    """Time the oracle's torch CPU executors (all host threads) on a bounded
    sample of the workload: `rows_sample` sequence rows with every head
    (with ``gated``, the gates are computed from raw a, b inside the timed
    region, as the fused-gating verify does)."""
    from gdn_recoverssm_b200 import synthetic
    from oracle import cpu_executors as X

    spec = dict(synthetic.CONFIGS[cfg])
    B, H, HV, D, Q = rows_sample, spec["H"], spec["HV"], spec["D"], spec["Q"]
    gen = torch.Generator().manual_seed(seed)
    T = B * Q
    act = spec["act"]
    unit = lambda x: x / x.norm(dim=-1, keepdim=True)  # noqa: E731
    q = unit(torch.randn(T, H, D, generator=gen)).to(act)
    k = unit(torch.randn(T, H, D, generator=gen)).to(act)
    v = torch.randn(T, HV, D, generator=gen).to(act)
    g = -torch.nn.functional.softplus(torch.randn(T, HV, generator=gen))
    beta = torch.sigmoid(torch.randn(T, HV, generator=gen))
    a_raw = torch.randn(T, HV, generator=gen).to(act)
    b_raw = torch.randn(T, HV, generator=gen).to(act)
    A_log = torch.log(torch.rand(HV, generator=gen) * 15.0 + 1.0)
    dt_bias = torch.full((HV,), -4.0)
    pool = 2 * B + 1
    state = torch.randn(pool, HV, D, D, generator=gen) * 0.1
    src = torch.arange(1, B + 1, dtype=torch.int32)
    fin = torch.arange(B + 1, 2 * B + 1, dtype=torch.int32)
    qsl = torch.arange(B + 1, dtype=torch.int32) * Q
    acc = torch.randint(1, Q + 1, (B,), generator=gen, dtype=torch.int32)
    records = torch.zeros(B, HV, Q, 2 * D + 1)
    out = torch.zeros(T, HV, D, dtype=act)
    zeros = torch.zeros(B, dtype=torch.int32)
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        if gated:
            g = -torch.exp(A_log) * torch.nn.functional.softplus(a_raw.float() + dt_bias)
            beta = torch.sigmoid(b_raw.float())
        X.verify_packed(q, k, v, g, beta, state, qsl, src, records, out, spec_query_len=Q, scale=D**-0.5)
        X.fold_packed(state, records, src, acc, fin, zeros, zeros, rows=B)
        times.append(time.perf_counter() - t0)
    t = min(times)
    return {"value": B / t, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"config {cfg}: {B} of {spec['B']} rows x {HV} value heads, verify + fold, best of {repeats}",
            "seconds_per_sample": t}


def numpy_oracle_baseline(cfg, *, units_sample=1024, seed=0):
    """Time the float64 NumPy restatement of the reference's math oracle --
    ``verify_records`` + ``commit`` of plugin/tests/test_math_oracle.py:56-92,
    as oracle/gdn_oracle.py restates them -- looped over a seeded sample of
    (row, value head) units of the configuration in one process, and
    extrapolate to the whole batch (every unit costs the same)."""
    import numpy as np

    from gdn_recoverssm_b200 import synthetic
    from oracle import gdn_oracle as O

    spec = synthetic.CONFIGS[cfg]
    B, HV, D, Q = spec["B"], spec["HV"], spec["D"], spec["Q"]
    rng = np.random.default_rng(seed)
    n = min(units_sample, B * HV)
    unit = lambda x: x / np.linalg.norm(x, axis=-1, keepdims=True)  # noqa: E731
    cases = [(rng.standard_normal((D, D)) * 0.1, unit(rng.standard_normal((Q, D))), unit(rng.standard_normal((Q, D))),
              rng.standard_normal((Q, D)), -np.log1p(np.exp(rng.standard_normal(Q))),
              1.0 / (1.0 + np.exp(-rng.standard_normal(Q))), int(rng.integers(1, Q + 1))) for _ in range(n)]
    t0 = time.perf_counter()
    for state, q, k, v, g, beta, acc in cases:
        _, recs = O.verify_records(state, q, k, v, g, beta, D**-0.5)
        O.commit(state, recs, acc)
    per_unit = (time.perf_counter() - t0) / n
    try:
        from threadpoolctl import threadpool_info

        blas = max((i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"), default=1)
    except Exception:  # pragma: no cover
        blas = None
    return {"value": 1.0 / (per_unit * HV), "unit": UNIT, "cores": 1, "blas_threads": blas, "kind": "port",
            "sample": f"config {cfg}: {n} of {B * HV} (row, value head) units, float64 verify_records + commit "
                      f"per unit in one process, extrapolated to the batch",
            "seconds_per_unit": per_unit}


def run_reference(args):
    world, rank, _ = _dist()
    if rank != 0:
        return 0
    from gdn_recoverssm_b200 import synthetic

    # torchrun sets OMP_NUM_THREADS=1 for multi-process launches; rank 0 runs
    # alone here (the other ranks have exited), so it takes every host core
    torch.set_num_threads(len(os.sched_getaffinity(0)))
    spec = synthetic.CONFIGS[args.config]
    # size each step's sample so that warm-up + K steps fit the time budget
    probe = cpu_baseline(args.config, rows_sample=4, gated=args.gated)
    per_row = probe["seconds_per_sample"] / 4
    budget = args.reference_budget_s / max(1, args.steps + min(args.warmup, 1))
    rows = int(max(1, min(spec["B"], budget / per_row)))
    if args.warmup > 0:
        cpu_baseline(args.config, rows_sample=rows, gated=args.gated)
    vals = []
    for _ in range(args.steps):
        vals.append(cpu_baseline(args.config, rows_sample=rows, gated=args.gated)["value"])
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1000.0 * spec["B"] / value, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": _config_dict(args.config, world, args.gated),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                         "sample": f"each step: {rows} of {spec['B']} rows x all heads (verify + fold), torch CPU "
                                   f"executors restating the reference's CPU path"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


def _config_dict(cfg, world, gated=False):
    from gdn_recoverssm_b200 import synthetic

    s = synthetic.CONFIGS[cfg]
    mode = "align (block %d)" % s["block"] if s["align"] else "none"
    return {
        "workload": f"config{cfg}: B={s['B']} H={s['H']} HV={s['HV']} K=V={s['D']} Q={s['Q']} {mode}, "
                    f"{str(s['act']).split('.')[-1]} q/k/v, fp32 state pool {s['pool']} pages, packed fp32 records",
        "global_batch": s["B"],
        "spec_query_len": s["Q"],
        "parallelism": f"v-head shards x{world} (no collective)",
        "l2": "inputs larger than L2: every step reads all B x HV state tiles (64 KiB each)",
        "gates": ("fused in the verify prologue from raw a, b (activation dtype) and per-head A_log, dt_bias"
                  if gated else "precomputed: g (fp32 log-space decay), beta (fp32)"),
    }


def run_b200(args):
    import torch.distributed as dist

    world, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", init_method="env://", device_id=dev,
                                timeout=__import__("datetime").timedelta(seconds=120))
    import gdn_recoverssm_b200 as g
    from gdn_recoverssm_b200 import _native, synthetic

    _native.ops()
    conv = args.conv_dim > 0
    shard_world, shard_rank = (args.shard_of, 0) if args.shard_of else (world, rank)
    wl = synthetic.make(args.config, dev, seed=0, world=shard_world, rank=shard_rank,
                        conv_dim=args.conv_dim if conv else 16,
                        rows=args.rows, pool=args.pool,
                        gated=args.gated)
    stream = torch.cuda.current_stream(dev)
    ctx = g.GDNRecoverSSMCommitContext.from_tensors([wl.conv], [wl.state], [wl.records], spec_query_len=wl.Q,
                                                    max_num_reqs=wl.B)
    align_kw = {}
    if wl.block_table is not None:
        align_kw = dict(block_table=wl.block_table, num_computed_tokens=wl.num_computed,
                        mamba_block_size=wl.block_size)

    # --grouped-layers L: L GDN layers (each its own state pool, conv pool and
    # records; the same inputs and metadata), L verifies and ONE grouped commit
    # of the L groups in one bucket -- the serving commit of a KV-cache group
    # set (grouped plan, conv compaction and fold over every layer at once)
    layers = [(wl, ctx)]
    for _ in range(1, args.grouped_layers):
        w2 = synthetic.make(args.config, dev, seed=0, world=shard_world, rank=shard_rank,
                            conv_dim=args.conv_dim if conv else 16, rows=args.rows, pool=args.pool, gated=args.gated)
        layers.append((w2, g.GDNRecoverSSMCommitContext.from_tensors([w2.conv], [w2.state], [w2.records],
                                                                      spec_query_len=w2.Q, max_num_reqs=w2.B)))

    def verify():
        for lw, _ in layers:
            if args.gated:
                g.gdn_recoverssm_verify_gated(lw.A_log, lw.a, lw.b, lw.dt_bias, lw.q, lw.k, lw.v,
                                              checkpoint_state=lw.state, replay_cache=lw.records,
                                              query_start_loc=lw.qsl, state_indices=lw.state_indices,
                                              spec_query_len=lw.Q, use_qk_l2norm_in_kernel=False, out=lw.out)
            else:
                g.gdn_recoverssm_verify(lw.g, lw.beta, lw.q, lw.k, lw.v, checkpoint_state=lw.state,
                                        replay_cache=lw.records, query_start_loc=lw.qsl,
                                        state_indices=lw.state_indices, spec_query_len=lw.Q, out=lw.out)

    if args.grouped_layers:
        from types import SimpleNamespace

        rows_host = tuple(range(wl.B))
        qlens = tuple(int(x) for x in (wl.qsl[1:] - wl.qsl[:-1]).cpu())
        entries = []
        for lw, lctx in layers:
            payload = SimpleNamespace(
                state_indices=lw.state_indices, query_start_loc=lw.qsl,
                request_indices=torch.arange(wl.B, dtype=torch.int32, device=dev),
                block_table=lw.block_table, num_computed_tokens=lw.num_computed, block_size=lw.block_size,
                request_rows=rows_host, query_lens=qlens)
            entries.append(g.CommitEntry(SimpleNamespace(recoverssm_commit=payload), payload, lctx))
        bucket = g.GroupedCommitBucket(tuple(lctx for _, lctx in layers))
        persistent = [torch.zeros(wl.B, dtype=torch.int32, device=dev) for _ in range(2)]
        specs = bucket.make_specs(entries, wl.accepted, torch.arange(wl.B, dtype=torch.int32, device=dev),
                                  *persistent, publish_align=True)
        conv = True  # the grouped commit always compacts the conv history
    else:
        specs = ctx.make_commit_specs(wl.accepted, wl.state_indices, wl.qsl, commit_conv=conv, **align_kw)
    names = [sp.name for sp in specs]  # (grouped_)plan, (compact_conv,) fold

    def barrier():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()

    def step():
        verify()
        for sp in specs:
            sp.launch()

    for _ in range(args.warmup):
        step()
    barrier()
    graph, gsteps = None, 1
    if args.launch == "graph":
        # the headline steps replayed from a CUDA graph of `gsteps` whole steps
        # (verify + every commit launch, programmatic dependencies kept), as a
        # serving loop replays its decode step: no host work per step
        gsteps = next(d for d in (10, 5, 4, 2, 1) if args.steps % d == 0)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(gsteps):
                step()
        graph.replay()
        barrier()
    # plan outputs are identical every step (same metadata): byte model inputs
    if args.grouped_layers:  # group 0's rows of the bucket's plan
        plan_len, plan_final = bucket.length[: wl.B], bucket.final[: wl.B]
        plan_boundary, plan_blen = bucket.boundary[: wl.B], bucket.boundary_len[: wl.B]
    else:
        plan_len, plan_final = ctx.commit_lens[: wl.B], ctx.final_state_indices[: wl.B]
        plan_boundary, plan_blen = ctx.boundary_state_indices[: wl.B], ctx.boundary_recovery_lens[: wl.B]
    lens = plan_len.cpu()
    bnd = ((plan_boundary > 0) & (plan_blen > 0) & (plan_boundary != plan_final)).cpu()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2 + len(specs))] for _ in range(args.steps)]
    with ClockSampler(dev) as clocks:
        barrier()
        # the step as a serving loop issues it: nothing between the launches
        # (each commit launch is a programmatic dependent of the kernel before it)
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        host_t0 = time.perf_counter()
        t_start.record(stream)
        if graph is not None:
            for _ in range(args.steps // gsteps):
                graph.replay()
        else:
            for i in range(args.steps):
                step()
        t_end.record(stream)
        host_issue_ms = (time.perf_counter() - host_t0) * 1e3 / args.steps
        barrier()
        # the same steps again with an event between launches: per-kernel times
        for i in range(args.steps):
            e = ev[i]
            e[0].record(stream)
            verify()
            e[1].record(stream)
            for j, sp in enumerate(specs):
                sp.launch()
                e[2 + j].record(stream)
        barrier()
        # end to end through the public API with host buffers
        e2e = _e2e(g, wl, ctx, align_kw, args, dev, stream, barrier, nbuf=args.e2e_buffers)
    total_ms = t_start.elapsed_time(t_end)
    split = [sum(e[k].elapsed_time(e[k + 1]) for e in ev) / args.steps for k in range(1 + len(specs))]
    step_ms = total_ms / args.steps
    from gdn_recoverssm_b200.sharding import max_over_ranks

    timings = max_over_ranks([step_ms, e2e["ms"], *split], device=dev)
    step_ms, e2e_ms, verify_ms, spec_ms = timings[0], timings[1], timings[2], dict(zip(names, timings[3:]))
    clk = clocks.summary()
    status = int(torch.ops.gdn_recoverssm_ac.device_status())
    graphed, graph = graph is not None, None  # released before the process group
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    peak, peak_kind = _peaks()
    L = len(layers)  # every layer moves the same bytes (same inputs and metadata)
    vbytes = L * synthetic.verify_bytes(wl)
    fbytes = L * synthetic.commit_bytes(wl, lens, int(bnd.sum()))
    cbytes = L * synthetic.conv_bytes(wl, lens, int(bnd.sum()), ctx.conv_history_len) if conv else 0
    cfloor = L * synthetic.conv_floor_bytes(wl, lens, wl.state_indices[: wl.B].cpu(),
                                            plan_final[: wl.B].cpu(), plan_boundary[: wl.B].cpu(), bnd) if conv else 0
    verify_gbs = vbytes / (verify_ms * 1e-3) / 1e9
    step_gbs = (vbytes + fbytes + cbytes) / (step_ms * 1e-3) / 1e9
    kernels = {"verify": {"ms": verify_ms, "bytes": vbytes, "GB/s": verify_gbs, "frac": verify_gbs / peak}}
    bytes_of = {"fold": fbytes, "compact_conv": cbytes}
    for name, ms in spec_ms.items():
        kernels[name] = {"ms": ms}
        if name in bytes_of:
            gbs = bytes_of[name] / (ms * 1e-3) / 1e9
            kernels[name].update({"bytes": bytes_of[name], "GB/s": gbs, "frac": gbs / peak})
    if conv:
        # the sector floor of the dim-first conv pool: what the layout makes any kernel move
        gbs = cfloor / (spec_ms["compact_conv"] * 1e-3) / 1e9
        kernels["compact_conv"].update({"sector_floor_bytes": cfloor, "floor_GB/s": gbs, "floor_frac": gbs / peak})
    kernels["step"] = {"GB/s": step_gbs, "frac": step_gbs / peak, "per_rank_bytes": vbytes + fbytes + cbytes}
    top = "fold"  # the largest byte mover
    reduced = args.rows is not None or args.pool is not None or bool(args.shard_of) or conv
    traffic = _traffic_profile(f"{top}_config{args.config}", reduced)
    if traffic is not None:
        traffic = int(traffic * wl.units / (synthetic.CONFIGS[args.config]["B"] * synthetic.CONFIGS[args.config]["HV"]))
    value = wl.B / (step_ms * 1e-3)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": step_ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": _config_dict(args.config, world, args.gated),
        "e2e": {"value": wl.B / (e2e_ms * 1e-3), "unit": UNIT, "h2d_bytes_per_step": e2e["h2d"],
                "d2h_bytes_per_step": e2e["d2h"], "ms_per_step": e2e_ms},
        "roofline": {"bound": "hbm", "kernel": "fold (grouped commit)",
                     "achieved": kernels[top]["GB/s"], "peak": peak, "unit": "GB/s", "frac": kernels[top]["frac"],
                     "peak_kind": peak_kind, "traffic": traffic, "algorithmic_bytes_per_launch": bytes_of[top]},
        "kernels": kernels,
        "gpu_launches": (L + len(specs)) * args.steps * world,  # the verifies + the commit launches, per step and rank
        "clocks": clk,
        "device_status": status,
    }
    line["config"]["commit_launches"] = names
    if args.grouped_layers:
        line["config"]["grouped_commit"] = (f"{L} GDN layers: {L} verifies and one grouped commit of one bucket "
                                            f"of {L} groups per step (bytes counted for every layer); e2e is the "
                                            f"single-layer public-API step")
    line["config"]["launch"] = (f"CUDA graph of {gsteps} steps, replayed" if graphed
                                else "eager: each step issued from Python")
    line["host_issue_ms_per_step"] = host_issue_ms
    if args.shard_of:
        line["config"]["parallelism"] = f"rank 0 of a {args.shard_of}-way v-head split, on one GPU (profiling only)"
    if conv:
        line["config"]["commit_conv"] = f"conv history compacted in the commit: {int(wl.conv.shape[1])} channels"
    if not args.no_cpu_baseline and world == 1:
        line["cpu_baseline"] = cpu_baseline(args.config, rows_sample=args.cpu_rows, gated=args.gated)
        line["cpu_baseline"]["nproc"] = os.cpu_count()
        line["cpu_baseline"]["numpy_oracle"] = numpy_oracle_baseline(args.config)
    print(json.dumps(line))
    return 0


def _arena_views(buf, layout):
    """Typed views of one flat uint8 buffer, ``layout`` = [(name, offset, dtype, shape)]."""
    views = {}
    for name, off, dtype, shape in layout:
        n = int(torch.Size(shape).numel()) * torch.empty((), dtype=dtype).element_size()
        views[name] = buf.narrow(0, off, n).view(dtype).view(shape)
    return views


def _e2e(g, wl, ctx, align_kw, args, dev, stream, barrier, nbuf=3):
    """Same step through the public API from pinned host memory, as a serving
    loop runs it: every step copies its inputs (q, k, v, g, beta and the row
    metadata, packed in one pinned staging buffer) host -> device in one copy,
    runs verify + commit, and copies the attention output device -> host.
    Copies go on their own streams into ``nbuf`` device buffers, so the H2D of
    step i + 1 and the D2H of step i - 1 overlap the compute of step i; all of
    it is inside the timed region (from the first H2D to the last D2H)."""
    gated = wl.a is not None
    names = ["q", "k", "v"] + (["a", "b"] if gated else ["g", "beta"]) + ["qsl", "state_indices", "accepted"]
    if align_kw:
        names += ["block_table", "num_computed"]
    layout, off = [], 0
    for n in names:
        t = getattr(wl, n)
        layout.append((n, off, t.dtype, tuple(t.shape)))
        off += (t.numel() * t.element_size() + 255) // 256 * 256
    h2d = off
    host_buf = torch.empty(h2d, dtype=torch.uint8).pin_memory()
    host = _arena_views(host_buf, layout)
    for n in names:
        host[n].copy_(getattr(wl, n).cpu())
    dev_buf = [torch.empty(h2d, dtype=torch.uint8, device=dev) for _ in range(nbuf)]
    dev_in = [_arena_views(b, layout) for b in dev_buf]
    out_dev = [torch.empty_like(wl.out) for _ in range(nbuf)]
    out_host = [torch.empty(wl.out.shape, dtype=wl.out.dtype).pin_memory() for _ in range(nbuf)]
    d2h = out_host[0].numel() * out_host[0].element_size()
    steps = max(args.e2e_steps, args.steps)
    h2d_stream = torch.cuda.Stream(dev)
    d2h_stream = torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(nbuf)]    # inputs of buffer b on the device
    ev_done = [torch.cuda.Event() for _ in range(nbuf)]  # the step using buffer b has computed
    ev_out = [torch.cuda.Event() for _ in range(nbuf)]   # its output is on the host

    def step(i):
        b = i % nbuf
        d = dev_in[b]
        h2d_stream.wait_event(ev_done[b])  # the step that last read buffer b is done
        with torch.cuda.stream(h2d_stream):
            dev_buf[b].copy_(host_buf, non_blocking=True)
            ev_in[b].record(h2d_stream)
        stream.wait_event(ev_in[b])
        stream.wait_event(ev_out[b])  # out_dev[b] has been copied out
        kw = {}
        if align_kw:
            kw = dict(block_table=d["block_table"], num_computed_tokens=d["num_computed"],
                      mamba_block_size=wl.block_size)
        common = dict(checkpoint_state=wl.state, replay_cache=wl.records, query_start_loc=d["qsl"],
                      state_indices=d["state_indices"], spec_query_len=wl.Q, out=out_dev[b])
        if gated:  # A_log / dt_bias are layer weights: resident, not copied per step
            g.gdn_recoverssm_verify_gated(wl.A_log, d["a"], d["b"], wl.dt_bias, d["q"], d["k"], d["v"],
                                          use_qk_l2norm_in_kernel=False, **common)
        else:
            g.gdn_recoverssm_verify(d["g"], d["beta"], d["q"], d["k"], d["v"], **common)
        ctx.commit(d["accepted"], d["state_indices"], d["qsl"], commit_conv=args.conv_dim > 0, **kw)
        ev_done[b].record(stream)
        d2h_stream.wait_event(ev_done[b])
        with torch.cuda.stream(d2h_stream):
            out_host[b].copy_(out_dev[b], non_blocking=True)
            ev_out[b].record(d2h_stream)

    for i in range(nbuf + 1):
        step(i)
    torch.cuda.synchronize(dev)
    barrier()
    a = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    a.record(h2d_stream)  # the first copy of the timed steps starts after this
    stream.wait_event(a)
    for i in range(steps):
        step(i)
    for ev in ev_out:  # the timed region ends with the last output on the host
        d2h_stream.wait_event(ev)
    e.record(d2h_stream)
    torch.cuda.synchronize(dev)
    barrier()
    return {"ms": a.elapsed_time(e) / steps, "h2d": h2d, "d2h": d2h}


def main(argv=None):
    ap = argparse.ArgumentParser(description="RecoverSSM verify+commit benchmark")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--config", type=int, default=2, choices=[1, 2, 3, 4])
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--cpu-rows", type=int, default=512, help="rows in the CPU baseline's bounded sample")
    ap.add_argument("--reference-budget-s", type=float, default=60.0,
                    help="CPU seconds the --impl reference run may spend over all its steps")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--conv-dim", type=int, default=0,
                    help="also compact the conv history in the commit (channels; 0 = the metric's verify + fold)")
    ap.add_argument("--gated", action="store_true",
                    help="verify through the fused-gating entry point (raw a, b, A_log, dt_bias)")
    ap.add_argument("--e2e-buffers", type=int, default=3, help="device input/output buffers of the end-to-end loop")
    ap.add_argument("--e2e-steps", type=int, default=50, help="fewest steps the end-to-end pass times")
    ap.add_argument("--grouped-layers", type=int, default=0, choices=[0, 1, 2, 3],
                    help="L GDN layers committed by one grouped-commit bucket per step (0: the per-context commit)")
    ap.add_argument("--launch", default="graph", choices=["graph", "eager"],
                    help="headline steps replayed from a CUDA graph, or issued one by one from Python")
    ap.add_argument("--rows", type=int, default=None, help="reduced batch (profiling cases only)")
    ap.add_argument("--shard-of", type=int, default=0,
                    help="one GPU runs rank 0's head shard of an N-way split (profiling the per-rank step only)")
    ap.add_argument("--pool", type=int, default=None, help="reduced state pool (profiling cases only)")
    args = ap.parse_args(argv)
    if args.warmup < 3 and args.impl == "b200":
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
