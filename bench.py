"""Benchmark of the paged decode-attention hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c3|c0|c1|c2|c4] [--exchange nccl|peer]

Under torchrun (N > 1) there is one process per GPU.

A step is one decode-attention pass over one synthetic batch (see
vllm_fastdecoder_b200/workloads.py):
  c3 (default)  8 rows x 131072 tokens, GQA 32/8 bf16, each row's KV split
                contiguously over the N GPUs; every rank decodes its shard
                and the partials are exchanged and LSE-merged (strong
                scaling); after the timed region the merged output of three
                (row, kv head) pairs is checked against the C oracle over the
                whole context (`parity`)
  c0            16 rows, one 4096-block HBM pool (the reference's CPU case)
  c1            GPU/host split: 64 rows of U[256,4096] tokens, 32/32 heads,
                fp16, HBM tier of 2048 blocks, the rest in pinned host memory;
                N > 1 runs N independent replicas (weak scaling)
  c2            GQA 32/8 bf16, 256 rows, lognormal lengths, all HBM
  c4            a continuous-batching decode trace over 32 layers (about 128
                running requests, most of their KV in the host tier); a step
                is one decode step of every running request through all 32
                layers (KV write + decode per layer); N > 1: replicas

Reported: `value` = rows/s with inputs resident (device-timed, CUDA events,
max over ranks); `e2e` = the same through the public API with the step's q /
block table / lengths copied in from pinned host memory and o / lse copied
back every step; `roofline` = algorithmic bytes of the decode kernel per
launch / its event-timed duration, against the measured HBM copy peak (and,
for the host tier, the pinned host->device copy rate measured in the same
run); `cpu_baseline` = the reference's own AVX2 kernel (compiled from its
source into oracle/_ref) on this host's cores, on the same values.
`--impl reference` times only that reference CPU kernel on the same workload,
by the same method (3 warm-ups, median of at least 10 calls).
"""

from __future__ import annotations

import argparse
import dataclasses
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

METRIC = "decode-attn seqs/s"
UNIT = "seqs/s"


def _peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured (MEASURED_PEAKS.json)"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


def _traffic(kernel: str, workload: str):
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    return json.loads(p.read_text()).get(f"{kernel}/{workload}")


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# ---------------------------------------------------------------- clocks


class ClockSampler:
    """nvidia-smi samples of this GPU during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: torch.device):
        pr = torch.cuda.get_device_properties(device)
        self.bus = f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.bus, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self._t is not None:
            self._t.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for nm, val in zip(names, parts[4:8]):
                if val.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- helpers


def pcie_h2d_gbs(device: torch.device, nbytes: int = 1 << 30) -> float:
    """Pinned host -> device copy rate (the PCIe roofline of the host tier)."""
    h = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    d = torch.empty(nbytes, dtype=torch.uint8, device=device)
    d.copy_(h, non_blocking=True)
    torch.cuda.synchronize(device)
    best = 0.0
    for _ in range(3):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        d.copy_(h, non_blocking=True)
        e.record()
        e.synchronize()
        best = max(best, nbytes / (s.elapsed_time(e) * 1e-3) / 1e9)
    del h, d
    return best


def host_part(batch):
    """The reference's CPU leg of a step: host-tier rows of the batch with
    host-relative, compacted block ids (what its planner feeds decode_attn,
    fastdecode/plan.py:157-160)."""
    n, BS, G = batch.n, batch.BS, batch.G
    rows, lens = [], []
    for i in range(n):
        L = int(batch.lens[i])
        nb = (L + BS - 1) // BS
        ids, toks = [], 0
        for j in range(nb):
            b = int(batch.block_table[i, j])
            if b >= G:
                ids.append(b - G)
                toks += BS if j < nb - 1 else L - (nb - 1) * BS
        rows.append(ids)
        lens.append(toks)
    W = max(1, max(len(r) for r in rows))
    bt = torch.zeros(n, W, dtype=torch.int32)
    for i, r in enumerate(rows):
        if r:
            bt[i, :len(r)] = torch.tensor(r, dtype=torch.int32)
    return bt, torch.tensor(lens, dtype=torch.int32)


def reference_inputs(batch, resident, rows: int | None = None):
    """CPU tensors in the reference layout for its decode_attn, holding the
    same values the GPU arm decodes: q [n,H,D], caches [C,KVH,BS,D], table,
    lens.  With a host tier (c1) the caches are the pinned host tier itself
    and the table covers its host blocks only (the reference's CPU leg);
    otherwise the HBM pool is copied to the host in the reference layout and
    the table is the batch's own."""
    n = batch.n if rows is None else rows
    if batch.num_host_blocks > 0:
        hk, hv = resident.tiers[1].k, resident.tiers[1].v
        bt, lens = host_part(batch)
        return resident.q[:n].cpu(), hk, hv, bt[:n].contiguous(), lens[:n].contiguous()
    t = resident.tiers[0]
    kc = t.k.contiguous().cpu()
    vc = t.v.contiguous().cpu()
    return (resident.q[:n].cpu(), kc, vc, batch.block_table[:n].contiguous(), batch.lens[:n].contiguous())


def time_reference(inputs, scale: float, steps: int, warmup: int) -> dict:
    """The reference AVX2 decode_attn (oracle/_ref, all host threads) on
    `inputs` = (q, k_cache, v_cache, block_table, lens): `warmup` untimed
    calls, then `steps` timed calls (at least 10).  Falls back to the C
    restatement, single-threaded, when the reference was not built.
    Returns the median / min / max seconds per call, the thread count, the
    kind ("reference" or "port") and the outputs of the last call."""
    from oracle import oracle as O

    q, kc, vc, bt, lens = inputs
    ext = O.load_reference_ext()
    H, n = q.shape[1], q.shape[0]
    out = torch.empty_like(q)
    lse = torch.empty(H, n, dtype=torch.float32)
    threads = os.cpu_count() or 1
    if ext is not None:
        kind = "reference"
        ext.set_num_threads(threads)
        fn = lambda: ext.decode_attn(q, kc, vc, bt, lens, scale, out, lse)  # noqa: E731
    else:
        kind, threads = "port", 1
        fn = lambda: O.decode_attn(q, kc, vc, bt, lens, scale, out, lse)  # noqa: E731
    for _ in range(max(3, warmup)):
        fn()
    times = []
    for _ in range(max(10, steps)):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
    return {"median": statistics.median(times), "min": min(times), "max": max(times), "calls": len(times),
            "threads": threads, "kind": kind, "rows": n, "out": out, "lse": lse,
            "build": O.reference_ext_variant() if ext is not None else "oracle/libfd_oracle.so"}


def _cpu_baseline_entry(r: dict, batch, unit_factor: float = 1.0, sample: str | None = None) -> dict:
    """The cpu_baseline object of a timed reference leg: value from the
    median, with the spread of the calls."""
    per = lambda t: round(r["rows"] / (t * unit_factor), 2)  # noqa: E731
    return {"value": per(r["median"]), "unit": UNIT, "cores": r["threads"], "kind": r["kind"],
            "sample": sample or _sample_text(batch, r["rows"], r["calls"]),
            "min_value": per(r["max"]), "max_value": per(r["min"]), "calls": r["calls"],
            "method": "3 warm-up calls, then the median of the timed calls (min/max value from the slowest/fastest)",
            "build": r["build"], "cpu": _cpu_model()}


# ---------------------------------------------------------------- parity in the run


def c3_slices(batch) -> list[tuple[int, int]]:
    """(row, kv head) pairs whose full-context output the bench checks: the
    first and the last, and one in between."""
    return [(0, 0), (batch.n // 2, batch.KVH // 2), (batch.n - 1, batch.KVH - 1)]


def c3_parity(batch, res, final: torch.Tensor, lse_out: torch.Tensor, ws: int, rank: int,
              device: torch.device) -> dict | None:
    """Check the sharded step's merged output against the C oracle over the
    whole context.  For each checked (row, kv head) every rank gathers that
    head's K and V over its shard in table order; an all-gather (every rank
    takes part) brings the shards to rank 0 in rank order, i.e. sequence
    order, and rank 0 runs the oracle's decode over the concatenated
    131072 tokens (and a float64 evaluation) and compares the GPU's merged
    o (bf16) and lse.  Returns the parity entry on rank 0, None elsewhere."""
    import numpy as np

    BS, D, G = batch.BS, batch.D, batch.H // batch.KVH
    kt, vt = res.tiers[0].k, res.tiers[0].v  # [B, KVH, BS, D] views
    worst = {"max_abs_o": 0.0, "max_abs_lse": 0.0, "max_abs_o_f64": 0.0, "max_abs_lse_f64": 0.0, "max_o": 0.0}
    for (r, h) in c3_slices(batch):
        L = int(batch.lens[r])
        nb = (L + BS - 1) // BS
        ids = res.block_table[r, :nb].long()
        k = kt[ids, h].reshape(nb * BS, D)[:L].contiguous()
        v = vt[ids, h].reshape(nb * BS, D)[:L].contiguous()
        if ws > 1:
            kk = torch.empty(ws * L, D, dtype=k.dtype, device=device)
            vv = torch.empty(ws * L, D, dtype=v.dtype, device=device)
            torch.distributed.all_gather_into_tensor(kk, k)
            torch.distributed.all_gather_into_tensor(vv, v)
            k, v = kk, vv
        if rank != 0:
            continue
        from oracle import oracle as O

        Lt = k.shape[0]
        kc = k.cpu().view(Lt // BS, 1, BS, D)
        vc = v.cpu().view(Lt // BS, 1, BS, D)
        q = res.q[r, h * G:(h + 1) * G].cpu().view(1, G, D).contiguous()
        bt = torch.arange(Lt // BS, dtype=torch.int32).view(1, -1)
        ln = torch.tensor([Lt], dtype=torch.int32)
        o_ref = torch.empty(1, G, D, dtype=batch.dtype)
        lse_ref = torch.empty(G, 1, dtype=torch.float32)
        O.decode_attn(q, kc, vc, bt, ln, batch.scale, o_ref, lse_ref)
        o_gpu = final[r, h * G:(h + 1) * G].float().cpu()
        l_gpu = lse_out[h * G:(h + 1) * G, r].cpu()
        # float64 evaluation of the same head
        kd = k.double().cpu().numpy()
        vd = v.double().cpu().numpy()
        qd = q[0].double().numpy()
        sc = (qd @ kd.T) * batch.scale
        m = sc.max(axis=1, keepdims=True)
        e = np.exp(sc - m)
        ssum = e.sum(axis=1, keepdims=True)
        o64 = (e @ vd) / ssum
        l64 = (m + np.log(ssum))[:, 0]
        worst["max_abs_o"] = max(worst["max_abs_o"], float((o_gpu - o_ref[0].float()).abs().max()))
        worst["max_abs_lse"] = max(worst["max_abs_lse"], float((l_gpu - lse_ref[:, 0]).abs().max()))
        worst["max_abs_o_f64"] = max(worst["max_abs_o_f64"], float(np.abs(o_gpu.double().numpy() - o64).max()))
        worst["max_abs_lse_f64"] = max(worst["max_abs_lse_f64"], float(np.abs(l_gpu.double().numpy() - l64).max()))
        worst["max_o"] = max(worst["max_o"], float(np.abs(o64).max()))
    if rank != 0:
        return None
    tol_o, tol_lse = 1.6e-2, 1e-4
    return {k2: float(f"{v2:.3e}") for k2, v2 in worst.items()} | {
        "checked": [f"row {r} kv-head {h}: {G} heads x {int(batch.lens[r]) * ws} tokens" for r, h in c3_slices(batch)],
        "against": "C oracle (restatement of the reference decode_attn) over the whole context, and float64",
        "tol": {"o_bf16": tol_o, "lse": tol_lse},
        "ok": bool(worst["max_abs_o"] <= tol_o and worst["max_abs_lse"] <= tol_lse),
    }


def reference_parity(r: dict, out: torch.Tensor, lse: torch.Tensor, tol_o: float) -> dict:
    """Our output against the reference kernel's on the same inputs (all rows)."""
    o_gpu = out.float().cpu()
    l_gpu = lse.cpu()
    fin = torch.isfinite(r["lse"])
    d_lse = float((l_gpu[fin] - r["lse"][fin]).abs().max()) if bool(fin.any()) else 0.0
    d_o = float((o_gpu - r["out"].float()).abs().max())
    return {"max_abs_o": float(f"{d_o:.3e}"), "max_abs_lse": float(f"{d_lse:.3e}"),
            "against": f"the reference AVX2 decode_attn on the same inputs, all {r['rows']} rows",
            "tol": {"o": tol_o, "lse": 1e-4}, "ok": bool(d_o <= tol_o and d_lse <= 1e-4)}


# ---------------------------------------------------------------- our arm


def run_ours(args, ws, rank, device):
    from vllm_fastdecoder_b200 import gpu_ops, workloads

    dist = ws > 1
    if args.workload == "c3":
        batch = workloads.config3(world=ws, rank=rank, ctx=args.ctx)
    else:
        batch = workloads.CONFIGS[args.workload]()
    if args.layout and batch.num_hbm_blocks > 0:
        batch = dataclasses.replace(batch, hbm_layout=args.layout)
    res = workloads.materialize(batch, device)
    n, H, D = batch.n, batch.H, batch.D
    sharded = args.workload == "c3" and ws > 1
    gather = None
    if sharded:
        from vllm_fastdecoder_b200 import sharded as sh

        gather = (sh.PeerExchange(n, H, D, ws, device) if args.exchange in ("peer", "peer-split")
                  else sh.PartialExchange(n, H, D, ws, device))
        final = torch.empty(n, H, D, dtype=batch.dtype, device=device)
        out, lse = gather.o_view, gather.lse_view
    else:
        out = torch.empty(n, H, D, dtype=batch.dtype, device=device)
        lse = torch.empty(H, n, dtype=torch.float32, device=device)
    # 0: the persistent, length-balanced schedule; --split-grid: fixed splits
    tps = gpu_ops.choose_tiles_per_split(int(batch.lens.sum()), batch.KVH, batch.BS) if args.split_grid else 0
    max_len = int(batch.lens.max())
    # host tier: read in place over PCIe (mapped), or staged into HBM by the
    # copy engine each step and read at HBM rate
    staged = args.host_read == "staged" and res.tiers[1] is not None
    host_range = gpu_ops.host_block_range(batch.block_table, batch.lens, batch.BS, batch.G) if staged else None
    # chunked: host blocks staged in chunks on a side stream, each chunk
    # decoded into partials once it has landed, then one P-way merge
    chunked = args.host_read == "chunked" and res.tiers[1] is not None
    cplan = (gpu_ops.plan_chunked_staging(batch.block_table, batch.lens, batch.BS, batch.G, args.stage_chunks)
             if chunked else None)
    dec_tiers, dec_split = res.tiers, batch.G
    if staged:
        dec_tiers = (res.tiers[0], gpu_ops.stage_host_blocks(res.tiers[1], *host_range, device))
        dec_split = batch.G + host_range[0]
    a = gpu_ops.decode_args(res.q, dec_tiers, dec_split, res.block_table, res.lens, batch.scale, out, lse,
                            max_len=max_len, tiles_per_split=tps)
    has_combine = a.workspace_bytes > 0
    # the peer exchange does the decode's combine itself (fd_decode_exchange_merge)
    fused = gather is not None and args.exchange == "peer"  # "peer-split": decode + combine + fd_exchange_merge
    if fused:
        has_combine = False

    def exchange(args_):
        if fused:
            gather.decode_exchange_merge(args_, final, decode=False)  # after the caller's decode launch
        else:
            gather.exchange_and_merge(out, lse, final)
    copy_evs = []

    def stage(ev=None):
        if staged:
            if ev is not None:
                ev[0].record()
            gpu_ops.stage_host_blocks(res.tiers[1], *host_range, device)  # same buffer: `a` stays valid
            if ev is not None:
                ev[1].record()

    def step(ev=None, cev=None):
        if chunked:  # the whole overlapped step (copies, decodes, merge) is the timed unit
            if ev is not None:
                ev[0].record()
            gpu_ops.decode_staged_chunks(res.q, res.tiers, batch.scale, out, lse, cplan)
            if ev is not None:
                ev[1].record()
            return
        stage(cev)
        if ev is not None:
            ev[0].record()
        gpu_ops.launch_decode(a, device, "partials")
        if ev is not None:
            ev[1].record()
        if has_combine:
            gpu_ops.launch_decode(a, device, "combine")
        if gather is not None:
            exchange(a)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)
    gpu_ops.check_device_errors(device)

    # the step as one CUDA graph (decode and combine launches, and on N > 1
    # GPUs of config 3 the exchange: the NCCL all-gather and merge, or the
    # peer-memory kernel, whose step counter lives on the device), with its
    # own workspace so no later call can move it
    graph = None
    # steps per graph: consecutive steps in one graph, so that each decode
    # is a programmatic dependent of the previous step's last kernel (its
    # combine or exchange, which write none of the decode's inputs) and its
    # set-up overlaps that kernel, as consecutive layers' decodes do in a
    # model; K must be a multiple
    gsteps = next(c for c in (args.graph_steps, 4, 2, 1) if c >= 1 and args.steps % c == 0)
    if not args.no_graph:
        ws_g = torch.empty(max(256, a.workspace_bytes), dtype=torch.uint8, device=device)
        a_g = gpu_ops.decode_args(res.q, dec_tiers, dec_split, res.block_table, res.lens, batch.scale, out, lse,
                                  max_len=max_len, tiles_per_split=tps, workspace_buf=ws_g, pdl=not args.no_pdl)

        parts_g = (torch.empty((1 + len(cplan.chunks)) * (n * H * D + H * n), dtype=torch.float32, device=device)
                   if chunked else None)

        def gstep():
            if chunked:
                gpu_ops.decode_staged_chunks(res.q, res.tiers, batch.scale, out, lse, cplan, parts_buf=parts_g)
                return
            stage()
            if fused:
                gather.decode_exchange_merge(a_g, final)  # decode, then the exchange with the combine in it
                return
            gpu_ops.launch_decode(a_g, device, "partials")
            if has_combine:
                gpu_ops.launch_decode(a_g, device, "combine")
            if gather is not None:
                gather.exchange_and_merge(out, lse, final)

        gstep()
        torch.cuda.synchronize(device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(gsteps):
                gstep()
        for _ in range(args.warmup):
            graph.replay()
        torch.cuda.synchronize(device)
        gpu_ops.check_device_errors(device)

    # kernel time of the decode launch: eager steps with events around it
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    cevs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(device)
    if dist:
        torch.distributed.barrier()
    torch.cuda.synchronize(device)
    if graph is None:
        clocks.start()
        time.sleep(0.25)  # let nvidia-smi take its first sample before the region
    t_start.record()
    for k in range(args.steps):
        step(evs[k], cevs[k])
    t_end.record()
    torch.cuda.synchronize(device)
    elapsed_eager = t_start.elapsed_time(t_end) * 1e-3
    copy_t = (sum(c0.elapsed_time(c1) for c0, c1 in cevs) * 1e-3 / args.steps) if staged else 0.0
    phases = None
    if gather is not None:
        # per-phase device time of eager sharded steps (outside the timed
        # regions): decode kernel, its combine, the exchange + merge (which
        # includes waiting for the slowest rank)
        pev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
        for k in range(args.steps):
            e = pev[k]
            e[0].record()
            gpu_ops.launch_decode(a, device, "partials")
            e[1].record()
            if has_combine:
                gpu_ops.launch_decode(a, device, "combine")
            e[2].record()
            exchange(a)
            e[3].record()
        torch.cuda.synchronize(device)
        ph = torch.tensor([sum(e[j].elapsed_time(e[j + 1]) for e in pev) / args.steps for j in range(3)],
                          dtype=torch.float64, device=device)
        lo, hi = ph.clone(), ph.clone()
        torch.distributed.all_reduce(lo, op=torch.distributed.ReduceOp.MIN)
        torch.distributed.all_reduce(hi, op=torch.distributed.ReduceOp.MAX)
        phases = {nm: {"min_ms": round(float(lo[j]), 4), "max_ms": round(float(hi[j]), 4)}
                  for j, nm in enumerate(("decode", "combine", "exchange_merge"))}
        phases["note"] = ("eager steps, CUDA events per rank; min / max over ranks; exchange_merge includes the "
                          "wait for the slowest rank" + (" and the decode's combine (done by the exchange kernel)"
                                                         if fused else ""))
    # the timed region of `value`: K graph replays (or the eager steps above).
    # A short step makes K steps shorter than nvidia-smi's sampling period,
    # so the sampler starts under an untimed pre-roll of replays (~0.3 s of
    # the same work) and its samples see the GPU under load.
    if graph is not None:
        if dist:
            torch.distributed.barrier()
        torch.cuda.synchronize(device)
        clocks.start()
        time.sleep(0.1)
        # every rank replays the same number of graphs (they hold collectives):
        # the pre-roll count comes from the slowest rank's eager step
        step_est = torch.tensor([elapsed_eager / args.steps], dtype=torch.float64, device=device)
        if dist:
            torch.distributed.all_reduce(step_est, op=torch.distributed.ReduceOp.MAX)
        pre = max(1, int(0.3 / max(float(step_est) * gsteps, 1e-5)))
        for _ in range(pre):
            graph.replay()
        if dist:
            torch.distributed.barrier()  # NCCL barrier on the stream: after the pre-roll everywhere
        t_start.record()
        for _ in range(args.steps // gsteps):
            graph.replay()
        t_end.record()
        torch.cuda.synchronize(device)
    clk = clocks.stop()
    if dist:
        torch.distributed.barrier()
    gpu_ops.check_device_errors(device)
    elapsed = t_start.elapsed_time(t_end) * 1e-3
    kern = sorted(e0.elapsed_time(e1) * 1e-3 for e0, e1 in evs)
    kern_t = sum(kern) / len(kern)
    if dist:
        t = torch.tensor([elapsed, kern_t], dtype=torch.float64, device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        elapsed, kern_t = float(t[0]), float(t[1])

    rows_per_step = n if args.workload == "c3" else n * ws
    value = rows_per_step * args.steps / elapsed

    # ---- end to end through the public API: inputs from pinned host memory
    h_q = res.q.cpu().pin_memory()
    h_bt = batch.block_table.pin_memory()
    h_lens = batch.lens.pin_memory()
    h_out = torch.empty(out.shape, dtype=batch.dtype, pin_memory=True)
    h_lse = torch.empty(H, n, dtype=torch.float32, pin_memory=True)
    d_q = torch.empty_like(res.q)
    d_bt = torch.empty_like(res.block_table)
    d_lens = torch.empty_like(res.lens)
    e_out = out if not sharded else final

    def e2e_step():
        d_q.copy_(h_q, non_blocking=True)
        d_bt.copy_(h_bt, non_blocking=True)
        d_lens.copy_(h_lens, non_blocking=True)
        # the staged range comes from the step's host-side table, as a caller
        # holding the plan on the host would compute it
        hr = gpu_ops.host_block_range(h_bt, h_lens, batch.BS, batch.G) if staged else None
        if chunked:
            cp = gpu_ops.plan_chunked_staging(h_bt, h_lens, batch.BS, batch.G, args.stage_chunks)
            gpu_ops.decode_staged_chunks(d_q, res.tiers, batch.scale, out, lse, cp)
        elif fused:
            from vllm_fastdecoder_b200 import sharded as sh

            sh.sharded_decode(d_q, res.tiers, batch.G, d_bt, d_lens, batch.scale, gather, final, max_len=max_len,
                              tiles_per_split=tps)
        else:
            gpu_ops.decode_tiered(d_q, res.tiers, batch.G, d_bt, d_lens, batch.scale, out, lse,
                                  max_len=max_len, tiles_per_split=tps, host_range=hr)
            if gather is not None:
                gather.exchange_and_merge(out, lse, final)
        h_out.copy_(e_out, non_blocking=True)
        h_lse.copy_(lse if gather is None else gather.lse_out, non_blocking=True)
        torch.cuda.current_stream(device).synchronize()

    for _ in range(max(3, args.warmup)):
        e2e_step()
    if dist:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize(device)
    e2e_t = e0.elapsed_time(e1) * 1e-3
    if dist:
        t = torch.tensor([e2e_t], dtype=torch.float64, device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_t = float(t[0])
    gpu_ops.check_device_errors(device)
    h2d = h_q.numel() * h_q.element_size() + h_bt.numel() * 4 + h_lens.numel() * 4
    if chunked:  # the per-part tables and lengths, copied to the device by each step's call
        h2d += 4 * sum(t.numel() for t in cplan.tables) + 4 * sum(ln.numel() for ln in cplan.lens)
    d2h = h_out.numel() * h_out.element_size() + h_lse.numel() * 4

    # ---- roofline of the decode kernel (per launch, this rank's batch)
    peaks = _peaks()
    hbm_b, host_b = batch.kv_bytes()
    step_b = batch.step_bytes()
    achieved = step_b / kern_t / 1e9
    kname = gpu_ops.decode_kernel_name(batch.dtype, batch.D, batch.H, batch.KVH, batch.BS, batch.n, tps)
    # the captured traffic of the host-tier workloads is the staged path's
    # (every byte from HBM); the mapped path reads the host tier over PCIe
    traffic = _traffic(kname, args.workload) if staged or host_b == 0 else None
    if traffic is not None and args.workload == "c3":
        traffic = int(traffic * (args.ctx / ws) / 131072)  # the table holds one GPU's full-context launch
    roof = {"unit": "GB/s", "achieved": round(achieved, 1), "traffic": traffic,
            "kernel": kname, "algorithmic_bytes_per_launch": step_b,
            "kernel_ms": round(kern_t * 1e3, 4)}
    if host_b > 0:
        pcie = pcie_h2d_gbs(device)
        t_ideal = (step_b - host_b) / (peaks["hbm_gbs"] * 1e9) + host_b / (pcie * 1e9)
        t_step = kern_t + copy_t  # staged: the host-tier copy, then the decode at HBM rate
        if chunked:
            # overlapped: the copies bound the step (the HBM-tier bytes and the
            # decode of landed chunks run under them)
            t_ideal = max(host_b / (pcie * 1e9), step_b / (peaks["hbm_gbs"] * 1e9))
            roof.update({"achieved": round(step_b / t_step / 1e9, 1),
                         "host_read": f"chunked: host blocks staged in {len(cplan.chunks)} chunks on a side stream, "
                                      "each decoded into partials once landed (HBM blocks first), then one P-way "
                                      "merge; achieved and frac over the whole step (kernel_ms), ideal = the "
                                      "host-tier copy at the pinned-copy rate"})
        elif staged:
            roof.update({"achieved": round(step_b / t_step / 1e9, 1), "copy_ms": round(copy_t * 1e3, 4),
                         "host_read": "staged: host blocks copied to HBM by the copy engine (cudaMemcpyAsync), "
                                      "then decoded at HBM rate; achieved and frac over copy + kernel"})
        else:
            roof["host_read"] = "mapped: the kernel reads pinned host memory over PCIe"
        roof.update({"bound": "hbm+pcie", "peak": round(step_b / t_ideal / 1e9, 1),
                     "frac": round(t_ideal / t_step, 4),
                     "peak_note": f"bytes at their tier's rate: HBM {peaks['hbm_gbs']} GB/s "
                                  f"({peaks['source']}), host tier {pcie:.1f} GB/s (pinned H2D copy "
                                  "measured in this run)",
                     "hbm_bytes": step_b - host_b, "host_bytes": host_b})
    else:
        roof.update({"bound": "hbm", "peak": peaks["hbm_gbs"], "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "peak_note": f"HBM copy bandwidth, {peaks['source']} (burst figure)"})

    # ---- parity of this run's output (after the timed regions, outside them)
    parity = None
    if args.workload == "c3" and not args.no_parity:
        parity = c3_parity(batch, res, final if sharded else out, gather.lse_out if sharded else lse, ws, rank,
                           device)

    run = {
        "schedule": "split grid" if tps else "persistent (all CTAs resident, equal ranges of tiles plus "
                                             "per-segment weight positions)",
        "tiles_per_split": tps, "split_combine": has_combine, "kernel": kname,
        "host_read": (args.host_read if res.tiers[1] is not None else "none (all HBM)"),
        "timing": (f"value: one CUDA graph of {gsteps} consecutive steps (each: the decode launch"
                   + (" + its combine" if has_combine else "")
                   + (", exchange and merge" if gather is not None else "") + "; decodes launched as programmatic "
                   "dependents of the kernel ahead" + (", off" if args.no_pdl else "") + f") replayed K/{gsteps} "
                   "times after an untimed pre-roll; roofline: eager steps with CUDA events around the decode launch "
                   "(eager step "
                   f"{elapsed_eager / args.steps * 1e3:.4f} ms)" if graph is not None
                   else "value and roofline: eager steps, CUDA events"),
    }
    if gather is not None:
        run["exchange"] = {
            "peer": "peer memory: fd_decode_exchange_merge (the decode, then one exchange launch that also does the "
                    "decode's combine; CUDA IPC buffers, NVLink stores)",
            "peer-split": "peer memory: the decode, its combine, then one fd_exchange_merge launch (CUDA IPC "
                          "buffers, NVLink stores)",
            "nccl": "NCCL all_gather_into_tensor + fd_merge_partials"}[args.exchange]
    full = workloads.config3(world=1, rank=0, ctx=args.ctx) if args.workload == "c3" else batch
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(elapsed / args.steps * 1e3, 4), "higher_is_better": True,
        "scaling": "strong" if args.workload == "c3" else "weak", "vs_baseline": None, "dtype": _dtype_name(batch.dtype),
        "data": "synthetic (seeded N(0,1) q/K/V, configuration shapes)",
        "config": _config(full, args, ws),
        "run": run,
        "kv_gbs": round((hbm_b + host_b) * ws * args.steps / elapsed / 1e9, 1),
        "e2e": {"value": round(rows_per_step * args.steps / e2e_t, 2), "unit": UNIT,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "api": ("vllm_fastdecoder_b200.sharded.sharded_decode (C ABI fd_decode_exchange_merge)" if fused else
                        "vllm_fastdecoder_b200.gpu_ops.decode_tiered (C ABI fd_decode_attn)"
                        + (" + the exchange and merge" if gather is not None else ""))},
        "roofline": roof,
        "clocks": clk,
        "gpu_launches": args.steps * ((1 + len(cplan.chunks)) * (1 + int(has_combine)) + 1 if chunked else
                                      1 + int(has_combine) + (1 if gather is not None else 0)),
    }
    if parity is not None:
        line["parity"] = parity
    if phases is not None:
        line["run"]["phases"] = phases
    if graph is not None:
        graph.reset()  # a graph holding NCCL calls goes before the process group does
    if gather is not None and hasattr(gather, "close"):
        gather.close()  # collective: every rank reaches it
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        inputs = reference_inputs(batch, res)
        r = time_reference(inputs, batch.scale, steps=10, warmup=3)
        line["cpu_baseline"] = _cpu_baseline_entry(r, batch)
        if batch.num_host_blocks == 0:
            line["parity_vs_reference"] = reference_parity(
                r, out, lse, 1.6e-2 if batch.dtype == torch.bfloat16 else 2e-3)
    return line


# ---------------------------------------------------------------- config 4: the trace


def _trace_caches(tr, device):
    """The trace's KV tiers: vLLM's NHD HBM cache [G, BS, KVH, 2D] (logical
    [G, KVH, BS, 2D]) and the pinned host tier [blocks, KVH, BS, D] x 2,
    filled with N(0,1).  One physical cache serves every layer: a layer reads
    the same bytes as with per-layer caches, and each tier is larger than L2,
    so nothing is reused across layers."""
    from vllm_fastdecoder_b200.gpu_ops import KVTier

    dt, KVH, BS, D = tr.dtype, tr.KVH, tr.BS, tr.D
    gen = torch.Generator(device=device).manual_seed(tr.seed + 1)
    phys = torch.empty(tr.G, BS, KVH, 2 * D, dtype=dt, device=device)
    phys.normal_(generator=gen)
    kv_cache = phys.permute(0, 2, 1, 3)
    shape = (tr.host_blocks, KVH, BS, D)
    hk = torch.empty(shape, dtype=dt, pin_memory=True)
    hv = torch.empty(shape, dtype=dt, pin_memory=True)
    chunk = max(1, (256 << 20) // (KVH * BS * D * hk.element_size()))
    tmp = torch.empty((chunk,) + shape[1:], dtype=dt, device=device)
    for dst in (hk, hv):
        for s0 in range(0, shape[0], chunk):
            e = min(shape[0], s0 + chunk)
            tmp[:e - s0].normal_(generator=gen)
            dst[s0:e].copy_(tmp[:e - s0])
    del tmp
    torch.cuda.synchronize(device)
    return kv_cache, (KVTier(kv_cache[..., :D], kv_cache[..., D:]), KVTier(hk, hv))


def run_trace(args, ws, rank, device):
    """Config 4 on this GPU (replicas for N > 1): per step, for each of the 32
    layers, the tier-aware KV write of every running request's new token and
    the decode over both tiers.  `value` is device time with the step's tables
    resident; `e2e` runs the plugin's own path per step (host planner,
    to_device, q/k/v for every layer copied in from pinned memory, 32 x
    FastDecodeImpl._forward_split, the last layer's output read back)."""
    from types import SimpleNamespace

    from vllm_fastdecoder_b200 import backend, gpu_ops, plan, state, workloads

    dist = ws > 1
    W0, K = args.warmup, args.steps
    tr = workloads.trace4(seed=rank, steps=2 * (W0 + K))
    L, H, KVH, D, BS, G, dt = tr.layers, tr.H, tr.KVH, tr.D, tr.BS, tr.G, tr.dtype
    kv_cache, tiers = _trace_caches(tr, device)
    Rmax = max(st.rows for st in tr.steps)
    gen = torch.Generator(device=device).manual_seed(tr.seed + 2)
    q_all = torch.empty(L, Rmax, H, D, dtype=dt, device=device).normal_(generator=gen)
    k_all = torch.empty(L, Rmax, KVH, D, dtype=dt, device=device).normal_(generator=gen)
    v_all = torch.empty(L, Rmax, KVH, D, dtype=dt, device=device).normal_(generator=gen)
    out = torch.empty(Rmax, H, D, dtype=dt, device=device)
    lse = torch.empty(H, Rmax, dtype=torch.float32, device=device)
    staged = args.host_read == "staged"
    dev_steps = [(st.block_table.to(device), st.lens.to(device), st.slots.to(device), st.rows,
                  int(st.lens.max()), gpu_ops.host_block_range(st.block_table, st.lens, BS, G) if staged else None)
                 for st in tr.steps[:W0 + K]]

    def dev_step(k, evs=None):
        bt, lens, slots, R, mx, hr = dev_steps[k]
        for l in range(L):
            gpu_ops.store_kv_tiered(k_all[l, :R], v_all[l, :R], slots, tiers, G)
            if evs is not None:
                evs[l][0].record()
            # staged: this layer's host blocks copied to HBM (after its KV
            # write), then the decode; the events cover both
            gpu_ops.decode_tiered(q_all[l, :R], tiers, G, bt, lens, tr.scale, out[:R], lse[:, :R], max_len=mx,
                                  host_range=hr)
            if evs is not None:
                evs[l][1].record()

    for k in range(W0):
        dev_step(k)
    torch.cuda.synchronize(device)
    gpu_ops.check_device_errors(device)
    evs = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(L)]
           for _ in range(K)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(device)
    if dist:
        torch.distributed.barrier()
    torch.cuda.synchronize(device)
    clocks.start()
    time.sleep(0.25)
    t0.record()
    for k in range(K):
        dev_step(W0 + k, evs[k])
    t1.record()
    torch.cuda.synchronize(device)
    clk = clocks.stop()
    gpu_ops.check_device_errors(device)
    elapsed = t0.elapsed_time(t1) * 1e-3
    kern = [sum(a.elapsed_time(b) for a, b in evs[k]) * 1e-3 / L for k in range(K)]  # per decode launch
    kern_t = sum(kern) / len(kern)
    rows = sum(dev_steps[W0 + k][3] for k in range(K))
    if dist:
        t = torch.tensor([elapsed, kern_t], dtype=torch.float64, device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        elapsed, kern_t = float(t[0]), float(t[1])
    value = rows * ws / elapsed

    # ---- end to end through the plugin's split path
    names = [f"model.layers.{l}.self_attn.attn" for l in range(L)]
    hk, hv = tiers[1].k, tiers[1].v
    state.STORE = state.CpuKVStore(num_gpu_blocks=G, num_cpu_blocks=tr.host_blocks, block_size=BS,
                                   num_kv_heads=KVH, head_size=D, dtype=dt, k={nm: hk for nm in names},
                                   v={nm: hv for nm in names})
    impl = backend.FastDecodeImpl.__new__(backend.FastDecodeImpl)
    impl.num_heads, impl.num_kv_heads, impl.head_size = H, KVH, D
    impl.scale, impl.logits_soft_cap = tr.scale, 0.0
    impl.vllm_flash_attn_version = 2
    impl.kv_cache_dtype = "auto"
    impl.kv_sharing_target_layer_name = None
    layers = [SimpleNamespace(layer_name=nm, _k_scale=None, _v_scale=None) for nm in names]
    h_qkv = torch.empty(L, Rmax, H + 2 * KVH, D, dtype=dt, pin_memory=True)
    h_qkv.normal_()
    d_qkv = torch.empty(L, Rmax, H + 2 * KVH, D, dtype=dt, device=device)
    h_out = torch.empty(Rmax, H, D, dtype=dt, pin_memory=True)
    e_out = torch.empty(Rmax, H, D, dtype=dt, device=device)
    h2d_bytes = []

    def e2e_step(k):
        st = tr.steps[W0 + K + k]
        R = st.rows
        qsl = torch.arange(R + 1, dtype=torch.int32)
        width = int(st.block_table.shape[1])
        hp = plan.build_host_plan(qsl, st.lens, st.block_table, st.slots, G, tr.host_blocks, BS)
        bt_d = st.block_table.to(device)
        dp = plan.to_device(hp, bt_d, device)
        d_qkv[:, :R].copy_(h_qkv[:, :R], non_blocking=True)
        for l in range(L):
            q, kk, vv = d_qkv[l, :R].split([H, KVH, KVH], dim=1)
            impl._forward_split(layers[l], q, kk, vv, kv_cache, dp, e_out[:R])
        h_out[:R].copy_(e_out[:R], non_blocking=True)
        torch.cuda.current_stream(device).synchronize()
        h2d_bytes.append(R * width * 4 + (2 * R + 1) * 4 + R * 8 + L * R * (H + 2 * KVH) * D * 2)

    for k in range(W0):
        e2e_step(k)
    h2d_bytes.clear()
    if dist:
        torch.distributed.barrier()
    e2e_rows = 0
    tt = time.perf_counter()
    for k in range(K):
        e2e_step(W0 + k)
        e2e_rows += tr.steps[W0 + K + W0 + k].rows
    e2e_t = time.perf_counter() - tt
    gpu_ops.check_device_errors(device)
    if dist:
        t = torch.tensor([e2e_t], dtype=torch.float64, device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_t = float(t[0])

    # ---- roofline of the decode launches (per launch, averaged over the timed steps)
    peaks = _peaks()
    pcie = pcie_h2d_gbs(device)
    step_b = hbm_b = host_b = 0
    for k in range(K):
        b = tr.batch(W0 + k)
        step_b += b.step_bytes()
        hb, xb = b.kv_bytes()
        hbm_b += hb
        host_b += xb
    step_b, hbm_b, host_b = step_b / K, hbm_b / K, host_b / K  # one layer's decode launch
    t_ideal = (step_b - host_b) / (peaks["hbm_gbs"] * 1e9) + host_b / (pcie * 1e9)
    kname = gpu_ops.decode_kernel_name(dt, D, H, KVH, BS, Rmax)
    roof = {"unit": "GB/s", "achieved": round(step_b / kern_t / 1e9, 1), "traffic": _traffic(kname, "c4") if staged else None,
            "kernel": kname, "algorithmic_bytes_per_launch": int(step_b), "kernel_ms": round(kern_t * 1e3, 4),
            "bound": "hbm+pcie", "peak": round(step_b / t_ideal / 1e9, 1), "frac": round(t_ideal / kern_t, 4),
            "peak_note": f"bytes at their tier's rate: HBM {peaks['hbm_gbs']} GB/s ({peaks['source']}), host tier "
                         f"{pcie:.1f} GB/s (pinned H2D copy measured in this run)",
            "hbm_bytes": int(step_b - host_b), "host_bytes": int(host_b),
            "host_read": ("staged: each layer's host blocks copied to HBM by the copy engine, then decoded; "
                          "kernel_ms covers copy + decode" if staged
                          else "mapped: the kernel reads pinned host memory over PCIe")}
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": ws, "steps": K, "warmup": W0,
        "ms_per_step": round(elapsed / K * 1e3, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp16",
        "data": "synthetic (seeded N(0,1) q/K/V; simulated continuous-batching trace)",
        "config": {
            "workload": "continuous-batching decode trace (config 4): 32 layers, 32/32 heads, D128, fp16, BS16, "
                        "HBM tier 2048 blocks, host tier HBM-first up to 32768 blocks, <= 128 running, Poisson "
                        "arrivals, prompt U[128,1024], output U[64,1024], LIFO block reuse",
            "unit_note": "a seq is one running request advanced one token through all 32 layers",
            "rows_per_step": round(rows / K, 1), "layers": L, "host_blocks_touched": tr.host_blocks,
            "layer_storage": "one physical cache serves the 32 layers (same bytes per layer; each tier > L2)",
            "hbm_kv_bytes_per_layer": int(hbm_b), "host_kv_bytes_per_layer": int(host_b),
            "l2": "no flush: each layer streams more KV than the 126 MB L2",
            "parallelism": f"replicas x{ws}",
        },
        "kv_gbs": round((hbm_b + host_b) * L * K * ws / elapsed / 1e9, 1),
        "e2e": {"value": round(e2e_rows * ws / e2e_t, 2), "unit": UNIT,
                "h2d_bytes_per_step": int(sum(h2d_bytes) / max(1, len(h2d_bytes))),
                "d2h_bytes_per_step": Rmax * H * D * 2,
                "api": "FastDecodeImpl._forward_split x 32 layers per step (planner + C ABI fd_store_kv / "
                       "fd_decode_attn), wall clock with a host sync per step"},
        "roofline": roof,
        "clocks": clk,
        "gpu_launches": K * L * (2 + 1),
    }
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        b = tr.batch(W0)
        res = SimpleNamespace(tiers=tiers, q=q_all[0, :b.n])
        r = time_reference(reference_inputs(b, res), tr.scale, steps=10, warmup=3)
        line["cpu_baseline"] = _cpu_baseline_entry(
            r, b, unit_factor=L,
            sample=f"the reference's CPU leg of one layer of one step (decode_attn over the host-tier blocks of "
                   f"{r['rows']} rows, {host_b / 1e9:.3f} GB), median of {r['calls']} calls, times 32 layers")
    return line


def _dtype_name(dt) -> str:
    return {torch.float16: "fp16", torch.bfloat16: "bf16", torch.float32: "fp32"}[dt]


def _cpu_model() -> str:
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def _sample_text(batch, rows, calls: int) -> str:
    if batch.num_host_blocks > 0:
        _, host_b = batch.kv_bytes()
        return (f"the reference's CPU leg of one {batch.name} step: decode_attn over the host-tier blocks of "
                f"all {batch.n} rows ({host_b / 1e9:.3f} GB of host KV), median of {calls} calls")
    hbm_b, _ = batch.kv_bytes()
    return (f"decode_attn over all {rows} rows of one {batch.name} step ({hbm_b / 1e9:.3f} GB of KV, whole "
            f"contexts on one host), median of {calls} calls")


WORKLOADS = {
    "c1": "GPU/host split with LSE merge (config 1): 64 rows, ctx U[256,4096], 32/32 heads, D128, fp16, "
          "BS16, HBM tier 2048 blocks, per-row host fraction {0,.25,.5,.75,1}",
    "c0": "single-layer paged decode (config 0): 16 rows, ctx U[64,2048], 32/32 heads, D128, fp16, "
          "4096-block pool",
    "c2": "GQA decode (config 2): 256 rows, ctx lognormal(median 1024, sigma 0.75) clip [32,8192], "
          "32/8 heads, D128, bf16",
    "c3": "long-context sharded decode (config 3): 8 rows x 131072 ctx, 32/8 heads, D128, bf16, BS16, "
          "each row's blocks split contiguously over the GPUs, partials exchanged and LSE-merged",
}


def _config(batch, args, ws) -> dict:
    """The workload's identity, the same in both arms: `batch` is the whole
    workload (for c3 the unsharded batch, so byte counts are totals)."""
    hbm_b, host_b = batch.kv_bytes()
    return {
        "workload": WORKLOADS[args.workload],
        "rows": batch.n, "heads": batch.H, "kv_heads": batch.KVH, "head_size": batch.D, "block_size": batch.BS,
        "ctx_tokens": int(batch.lens.sum()),
        "hbm_kv_bytes": hbm_b, "host_kv_bytes": host_b, "hbm_layout": batch.hbm_layout,
        "l2": "no flush: each step streams more KV than the 126 MB L2" if hbm_b + host_b > (126 << 20)
              else "KV smaller than L2",
        "parallelism": f"replicas x{ws}" if args.workload != "c3" else f"kv-shard x{ws}",
    }


# ---------------------------------------------------------------- reference arm


def run_reference(args, ws, rank, device):
    """The reference arm: the reference's AVX2 decode_attn on this host's
    cores over the same workload and the same values as the GPU arm (inputs
    generated on the GPU with the same seeds, copied to the host in the
    reference layout).  For c3 that is the whole 131072-token context of
    every row on one host, whatever N is."""
    from vllm_fastdecoder_b200 import workloads

    if args.workload == "c4":
        return run_reference_trace(args, ws, device)
    if args.workload == "c3":
        batch = workloads.config3(world=1, rank=0, ctx=args.ctx)
    else:
        batch = workloads.CONFIGS[args.workload]()
    res = workloads.materialize(batch, device)
    inputs = reference_inputs(batch, res)
    del res
    torch.cuda.empty_cache()
    r = time_reference(inputs, batch.scale, steps=args.steps, warmup=args.warmup)
    entry = _cpu_baseline_entry(r, batch)
    v = entry["value"]
    return {
        "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(r["median"] * 1e3, 4), "higher_is_better": True, "impl": "reference",
        "scaling": "strong" if args.workload == "c3" else "weak", "vs_baseline": None,
        "dtype": _dtype_name(batch.dtype),
        "data": "synthetic (seeded N(0,1) q/K/V, configuration shapes)",
        "config": _config(batch, args, ws),
        "cpu_baseline": entry,
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference's AVX2 decode_attn (fastdecode/csrc/cpu_attn.cpp) compiled from its source, "
                "timed on this host with all its threads (rank 0 only; whole contexts, no sharding); for c1 "
                "only its CPU leg (host-tier blocks) is timed, its GPU FlashAttention leg would run concurrently",
    }


def run_reference_trace(args, ws, device):
    """Config 4 on the reference's CPU leg: its decode_attn over the host-tier
    blocks of one layer of each step (the layers are alike), times 32."""
    from types import SimpleNamespace

    from vllm_fastdecoder_b200 import workloads

    tr = workloads.trace4(seed=0, steps=args.warmup + args.steps)
    _, tiers = _trace_caches(tr, device)
    gen = torch.Generator(device=device).manual_seed(tr.seed + 2)
    q = torch.empty(max(st.rows for st in tr.steps), tr.H, tr.D, dtype=tr.dtype, device=device).normal_(
        generator=gen)
    per_layer, rows, th, kind = [], 0, 1, "reference"
    for k in range(args.warmup, args.warmup + args.steps):
        b = tr.batch(k)
        r = time_reference(reference_inputs(b, SimpleNamespace(tiers=tiers, q=q[:b.n])), tr.scale, steps=10,
                           warmup=3)
        th, kind = r["threads"], r["kind"]
        per_layer.append(r["median"])
        rows += r["rows"]
    t_step = statistics.mean(per_layer) * tr.layers
    v = round(rows / len(per_layer) / t_step, 2)
    return {
        "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(t_step * 1e3, 4), "higher_is_better": True, "impl": "reference",
        "scaling": "weak", "vs_baseline": None, "dtype": "fp16",
        "data": "synthetic (seeded N(0,1) q/K/V; simulated continuous-batching trace)",
        "config": {"workload": "continuous-batching decode trace (config 4), 32 layers; the reference's CPU leg"},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": th, "kind": kind,
                         "sample": "decode_attn over the host-tier blocks of one layer of each timed step "
                                   "(median of 10 calls after 3 warm-ups), times 32 layers", "cpu": _cpu_model()},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference's AVX2 decode_attn (fastdecode/csrc/cpu_attn.cpp) compiled from its source, "
                "timed on this host over the host-tier part of the trace; its GPU FlashAttention leg would "
                "run concurrently",
    }


def _emit(fd: int, line: dict) -> None:
    os.write(fd, (json.dumps(line) + "\n").encode())


def main() -> int:
    # Only the JSON line may reach stdout: libraries (NCCL's version banner,
    # warnings) write to fd 1 as well, so fd 1 points at stderr for the run
    # and the result goes to the saved original stdout.
    sys.stdout.flush()
    out_fd = os.dup(1)
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=0)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["c3", "c0", "c1", "c2", "c4"], default="c3")
    ap.add_argument("--no-parity", action="store_true", help="c3: skip the in-run oracle check of the output")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--split-grid", action="store_true", help="fixed split grid instead of the persistent schedule")
    ap.add_argument("--exchange", choices=["peer", "peer-split", "nccl"], default="peer",
                    help="c3 on N > 1 GPUs: partials exchanged over peer memory by the exchange kernel that also "
                         "does the decode's combine (peer), by the decode's combine and then the exchange kernel "
                         "(peer-split), or with an NCCL all-gather and a merge kernel (nccl)")
    ap.add_argument("--host-read", choices=["staged", "chunked", "mapped"], default="staged",
                    help="host tier: staged into HBM by the copy engine each step, staged in chunks on a side "
                         "stream with the decode of landed chunks overlapping the copies, or read in place over PCIe")
    ap.add_argument("--stage-chunks", type=int, default=8, help="--host-read chunked: chunks per step")
    ap.add_argument("--graph-steps", type=int, default=8,
                    help="consecutive steps captured in one CUDA graph (the largest of this, 4, 2, 1 dividing K)")
    ap.add_argument("--no-pdl", action="store_true",
                    help="launch the graph's decodes as ordinary launches, not programmatic dependents")
    ap.add_argument("--no-graph", action="store_true",
                    help="time eager launches instead of a captured CUDA graph of the step")
    ap.add_argument("--ctx", type=int, default=131072,
                    help="c3 context length per row (a smaller one for profiling captures)")
    ap.add_argument("--layout", choices=["nhd", "hnd"], default=None,
                    help="HBM-tier layout: nhd = vLLM [B, BS, KVH, 2D]; hnd = [2, B, KVH, BS, D] "
                         "(default: the workload's own)")
    args = ap.parse_args()
    if args.impl == "reference":
        args.split_grid = False
    if args.steps <= 0:
        args.steps = {"c1": 60, "c0": 400, "c2": 200, "c3": 100, "c4": 5}[args.workload]
    args.warmup = max(3, args.warmup)
    ws, rank, local = _dist()
    if args.impl == "reference":
        if rank != 0:
            return 0
        device = torch.device("cuda", local) if torch.cuda.is_available() else None
        if device is not None:
            torch.cuda.set_device(device)
        _emit(out_fd, run_reference(args, ws, rank, device))
        return 0
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if ws > 1:
        import datetime

        torch.distributed.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=120))
    try:
        line = run_trace(args, ws, rank, device) if args.workload == "c4" else run_ours(args, ws, rank, device)
        if rank == 0:
            _emit(out_fd, line)
    finally:
        if ws > 1:
            torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
