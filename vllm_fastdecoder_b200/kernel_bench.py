"""Per-kernel timings of the engine's smaller kernels (one JSON line per case).

    python -m vllm_fastdecoder_b200.kernel_bench [case ...] [--launches N]

The decode kernels and their combine are timed by bench.py on the benchmark
workloads; this covers the rest, each on inputs sized like the workload it
serves (and larger than the 126 MB L2 where the kernel streams data):

  store_kv_prefill  fd_store_kv_kernel: 16384 new tokens x 32 kv heads x D128
                    fp16 into the HBM tier (a prefill-sized write)
  store_kv_decode   fd_store_kv_kernel: 128 new tokens, half of them into the
                    mapped host tier (a decode step of config 4)
  merge2            fd_merge2_kernel: two fp16 partials of 4096 rows x 32
                    heads x D128 merged into one (the two-tier merge)
  merge_partials    fd_mergeP_kernel: 8 fp32 partials of 8 rows x 32 heads x
                    D128 (config 3's merge at 8 GPUs)
  split_merge       fd_split_merge_kernel: the split-grid combine of config 2
                    (tiles_per_split 16)
  combine           fd_persistent_combine_kernel: the persistent schedule's
                    merge of cut segments, config 2
  host_mapped       fd_decode_kernel reading only the host tier in place over
                    PCIe (pinned, device-mapped): 16 rows x 4096 tokens, 32/32
                    heads, D128, fp16 (1.07 GB in host memory)
  prefill           fd_prefill_kernel: 8 requests of 1024 new queries over
                    1024 cached + 1024 new keys (causal), 32/8 heads, D128,
                    bf16, paged HBM tier (achieved TFLOP/s against the
                    measured dense bf16 peak)
  prefill_fa        the same prefill through FlashAttention, the library the
                    reference calls for these rows: vLLM's
                    flash_attn_varlen_func over the paged cache when its
                    extension loads, else flash-attn 2.8 over the gathered
                    K/V (a baseline timing, not this engine's path)
  plan              fd_plan_kernel: the device planner on a 128-request
                    decode step of the config-4 trace
  exchange1         fd_exchange_merge_kernel with one rank (push, flags, merge
                    of config 3's partial)

Each line: the kernel, the mean device time per launch (CUDA events around
`--launches` back-to-back launches after warm-up), the algorithmic bytes per
launch, and achieved GB/s against the measured HBM copy rate (for
host_mapped: against a pinned host-to-device cudaMemcpyAsync of the same
bytes timed in the same run, and against PCIe Gen5 x16's nominal 63 GB/s).
"""

from __future__ import annotations

import argparse
import json
import math
from pathlib import Path

import torch

from vllm_fastdecoder_b200 import gpu_ops, workloads
from vllm_fastdecoder_b200.gpu_ops import KVTier

ROOT = Path(__file__).resolve().parents[1]
PCIE5_X16_GBS = 63.0  # PCIe Gen5 x16, per direction, nominal (32 GT/s x 16 lanes, 128b/130b)


def _hbm_peak() -> float:
    p = ROOT / "MEASURED_PEAKS.json"
    return float(json.loads(p.read_text())["hbm_gbs"]) if p.exists() else 6650.0


def _bf16_peak() -> float:
    p = ROOT / "MEASURED_PEAKS.json"
    return float(json.loads(p.read_text())["bf16_tflops"]) if p.exists() else 1590.0


def _time(fn, launches: int, warmup: int = 3) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(launches):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e-3 / launches


def case_store_kv(dev, host_half: bool):
    m, KVH, D, BS, dt = (16384, 32, 128, 16, torch.float16) if not host_half else (128, 32, 128, 16, torch.float16)
    G = 8192 if not host_half else 2048
    phys = torch.zeros(G, BS, KVH, 2 * D, dtype=dt, device=dev)  # vLLM NHD [B, BS, KVH, 2D]
    cache = phys.permute(0, 2, 1, 3)
    tiers = [KVTier(cache[..., :D], cache[..., D:]), None]
    C = 0
    if host_half:
        C = 512
        hk = torch.zeros(C, KVH, BS, D, dtype=dt, pin_memory=True)
        hv = torch.zeros(C, KVH, BS, D, dtype=dt, pin_memory=True)
        tiers[1] = KVTier(hk, hv)
    g = torch.Generator().manual_seed(0)
    slots = torch.randperm((G + C) * BS, generator=g)[:m].to(torch.int64)
    if host_half:  # half the rows to the host tier, half to HBM
        slots[: m // 2] = torch.randperm(C * BS, generator=g)[: m // 2] + G * BS
        slots[m // 2:] = torch.randperm(G * BS, generator=g)[: m - m // 2]
    slots = slots.to(dev)
    k = torch.randn(m, KVH, D, dtype=dt, device=dev)
    v = torch.randn(m, KVH, D, dtype=dt, device=dev)
    nbytes = 2 * m * KVH * D * 2 * 2 + m * 8  # K and V read and written, slots read
    return (lambda: gpu_ops.store_kv_tiered(k, v, slots, tuple(tiers), G)), nbytes, "fd_store_kv_kernel"


def case_merge2(dev):
    n, H, D, dt = 4096, 32, 128, torch.float16
    o_a = torch.randn(n, H, D, dtype=dt, device=dev)
    o_b = torch.randn(n, H, D, dtype=dt, device=dev)
    la = torch.randn(H, n, device=dev)
    lb = torch.randn(H, n, device=dev)
    out = torch.empty(n, H, D, dtype=dt, device=dev)
    out_lse = torch.empty(H, n, device=dev)
    nbytes = 3 * n * H * D * 2 + 3 * H * n * 4
    return (lambda: gpu_ops.merge_attn_states(out, o_a, la, o_b, lb, out_lse)), nbytes, "fd_merge2_kernel"


def case_merge_partials(dev):
    P, n, H, D = 8, 8, 32, 128
    stride = n * H * D + H * n
    parts = torch.randn(P, stride, device=dev)
    out = torch.empty(n, H, D, dtype=torch.bfloat16, device=dev)
    out_lse = torch.empty(H, n, device=dev)
    nbytes = P * stride * 4 + n * H * D * 2 + H * n * 4
    return (lambda: gpu_ops.merge_partials(parts, P, n, H, D, out, out_lse)), nbytes, "fd_mergeP_kernel"


def case_split_merge(dev):
    b = workloads.config2()
    res = workloads.materialize(b, dev)
    out = torch.empty(b.n, b.H, b.D, dtype=b.dtype, device=dev)
    lse = torch.empty(b.H, b.n, dtype=torch.float32, device=dev)
    a = gpu_ops.decode_args(res.q, res.tiers, b.G, res.block_table, res.lens, b.scale, out, lse,
                            max_len=int(b.lens.max()), tiles_per_split=16)
    gpu_ops.launch_decode(a, dev, "partials")
    torch.cuda.synchronize()
    # the merge reads every split's fp32 partial (o and lse) of every row-head
    tiles = [(int(L) + 15) // 16 for L in b.lens]
    splits = sum((t + 15) // 16 for t in tiles if (t + 15) // 16 > 1)
    rows_split = sum(1 for t in tiles if (t + 15) // 16 > 1)
    nbytes = splits * b.H * (b.D + 1) * 4 + rows_split * b.H * (b.D * 2 + 4)
    return (lambda: gpu_ops.launch_decode(a, dev, "combine")), nbytes, "fd_split_merge_kernel"


def case_combine(dev):
    b = workloads.config2()
    res = workloads.materialize(b, dev)
    out = torch.empty(b.n, b.H, b.D, dtype=b.dtype, device=dev)
    lse = torch.empty(b.H, b.n, dtype=torch.float32, device=dev)
    a = gpu_ops.decode_args(res.q, res.tiers, b.G, res.block_table, res.lens, b.scale, out, lse,
                            max_len=int(b.lens.max()))
    gpu_ops.launch_decode(a, dev, "partials")
    torch.cuda.synchronize()
    # every decode CTA's two fp32 partial slots (GQ heads of D + 1 floats)
    # are read at most once, and one merged segment (GQ heads of D outputs
    # and an lse) is written per CTA at most: an upper bound of the bytes the
    # kernel must move.  The tensor-core decode runs one CTA per SM.
    ctas = torch.cuda.get_device_properties(dev).multi_processor_count
    gq = b.H // b.KVH
    nbytes = ctas * 2 * gq * (b.D + 1) * 4 + ctas * gq * (b.D * 2 + 4)
    return (lambda: gpu_ops.launch_decode(a, dev, "combine")), nbytes, "fd_persistent_combine_kernel"


def case_host_mapped(dev):
    n, H, D, BS, L, dt = 16, 32, 128, 16, 4096, torch.float16
    nb = L // BS
    C = n * nb
    g = torch.Generator().manual_seed(3)
    hk = torch.empty(C, H, BS, D, dtype=dt, pin_memory=True)
    hv = torch.empty(C, H, BS, D, dtype=dt, pin_memory=True)
    tmp = torch.empty(nb, H, BS, D, dtype=dt, device=dev)
    for dst in (hk, hv):
        for r in range(n):
            tmp.normal_()
            dst[r * nb:(r + 1) * nb].copy_(tmp)
    del tmp
    bt = torch.randperm(C, generator=g).to(torch.int32).view(n, nb).to(dev)  # host ids from tier_split 0
    lens = torch.full((n,), L, dtype=torch.int32, device=dev)
    q = torch.randn(n, H, D, dtype=dt, device=dev)
    out = torch.empty(n, H, D, dtype=dt, device=dev)
    lse = torch.empty(H, n, dtype=torch.float32, device=dev)
    tiers = (None, KVTier(hk, hv))
    torch.cuda.synchronize()
    nbytes = 2 * n * L * H * D * 2 + n * H * (2 * D * 2 + 4) + n * nb * 4
    return (lambda: gpu_ops.decode_tiered(q, tiers, 0, bt, lens, 1.0 / math.sqrt(D), out, lse)), nbytes, \
        "fd_decode_kernel"


def pinned_copy_gbs(dev, nbytes: int = 1 << 30) -> float:
    """Pinned host-to-device cudaMemcpyAsync rate (GB/s), the PCIe reference."""
    src = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    dst = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    t = _time(lambda: dst.copy_(src, non_blocking=True), 5, warmup=2)
    return nbytes / t / 1e9


def case_prefill(dev):
    n, ql, kl, H, KVH, D, BS, dt = 8, 1024, 2048, 32, 8, 128, 16, torch.bfloat16
    nb = kl // BS
    g = torch.Generator().manual_seed(4)
    phys = torch.empty(n * nb + 8, BS, KVH, 2 * D, dtype=dt, device=dev).normal_()
    cache = phys.permute(0, 2, 1, 3)
    kv = KVTier(cache[..., :D], cache[..., D:])
    bt = torch.randperm(n * nb + 8, generator=g)[: n * nb].to(torch.int32).view(n, nb).to(dev)
    q = torch.randn(n * ql, H, D, dtype=dt, device=dev)
    out = torch.empty_like(q)
    i32 = lambda x: torch.tensor(x, dtype=torch.int32, device=dev)  # noqa: E731
    qs, qls, kls = i32([i * ql for i in range(n)]), i32([ql] * n), i32([kl] * n)
    # causal: query i sees kl - ql + i + 1 keys; 4 flops per (query, key, dim, head)
    keys_seen = sum(kl - ql + i + 1 for i in range(ql)) * n
    flops = 4 * keys_seen * H * D
    return (lambda: gpu_ops.prefill_attn(q, out, qs, qls, kls, 1.0 / math.sqrt(D), kv=kv, block_table=bt,
                                         total_q=n * ql)), flops, "fd_prefill_kernel"


def case_prefill_fa(dev):
    n, ql, kl, H, KVH, D, BS, dt = 8, 1024, 2048, 32, 8, 128, 16, torch.bfloat16
    nb = kl // BS
    g = torch.Generator().manual_seed(4)
    phys = torch.empty(n * nb + 8, BS, KVH, 2 * D, dtype=dt, device=dev).normal_()
    bt = torch.randperm(n * nb + 8, generator=g)[: n * nb].to(torch.int32).view(n, nb).to(dev)
    q = torch.randn(n * ql, H, D, dtype=dt, device=dev)
    cu_q = torch.arange(0, (n + 1) * ql, ql, dtype=torch.int32, device=dev)
    keys_seen = sum(kl - ql + i + 1 for i in range(ql)) * n
    flops = 4 * keys_seen * H * D
    scale = 1.0 / math.sqrt(D)
    try:  # the reference's own call (fastdecode/backend.py:317-329)
        from vllm.vllm_flash_attn import flash_attn_varlen_func as fa

        k_cache, v_cache = phys[..., :D], phys[..., D:]  # [B, BS, KVH, D] views
        seqused = torch.full((n,), kl, dtype=torch.int32, device=dev)
        fn = lambda: fa(q=q, k=k_cache, v=v_cache, cu_seqlens_q=cu_q, max_seqlen_q=ql, seqused_k=seqused,  # noqa: E731
                        max_seqlen_k=kl, softmax_scale=scale, causal=True, block_table=bt, fa_version=2)
        fn()
        return fn, flops, "vllm_flash_attn (fa2, paged)"
    except Exception:
        from flash_attn import flash_attn_varlen_func as fa

        k = phys[bt.long().flatten()].reshape(n * kl, KVH, 2 * D)
        kc, vc = k[..., :D].contiguous(), k[..., D:].contiguous()
        cu_k = torch.arange(0, (n + 1) * kl, kl, dtype=torch.int32, device=dev)
        fn = lambda: fa(q, kc, vc, cu_q, cu_k, ql, kl, softmax_scale=scale, causal=True)  # noqa: E731
        fn()
        return fn, flops, "flash_attn 2.8 (gathered K/V)"


def case_plan(dev):
    from vllm_fastdecoder_b200 import plan

    tr = workloads.trace4(seed=0, steps=1)
    st = tr.steps[0]
    R = st.rows
    qsl = torch.arange(R + 1, dtype=torch.int32, device=dev)
    lens, bt, slots = st.lens.to(dev), st.block_table.to(dev), st.slots.to(dev)
    out = plan.DeviceStepPlan(R, R, bt.shape[1], dev)

    def run():
        plan.plan_on_device(qsl, lens, bt, slots, tr.G, tr.host_blocks, tr.BS, out=out, max_tokens=R)

    nbytes = bt.numel() * 4 * 3 + R * (4 * 4 + 8 * 8)  # table read, two compacted tables written, lists
    return run, nbytes, "fd_plan_kernel"


def case_exchange1(dev):
    from vllm_fastdecoder_b200 import sharded

    n, H, D = 8, 32, 128
    ex = sharded.PeerExchange(n, H, D, 1, dev)
    ex.o_view.normal_()
    ex.lse_view.normal_()
    final = torch.empty(n, H, D, dtype=torch.bfloat16, device=dev)
    nbytes = 2 * ex.slot * 4 + ex.slot * 4 + n * H * D * 2  # read send, write + read the slot, write out
    return (lambda: ex.exchange_and_merge(None, None, final)), nbytes, "fd_exchange_merge_kernel"


CASES = {
    "store_kv_prefill": lambda dev: case_store_kv(dev, False),
    "store_kv_decode": lambda dev: case_store_kv(dev, True),
    "merge2": case_merge2,
    "merge_partials": case_merge_partials,
    "split_merge": case_split_merge,
    "combine": case_combine,
    "host_mapped": case_host_mapped,
    "prefill": case_prefill,
    "prefill_fa": case_prefill_fa,
    "plan": case_plan,
    "exchange1": case_exchange1,
}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("cases", nargs="*", default=list(CASES))
    ap.add_argument("--launches", type=int, default=20)
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peak = _hbm_peak()
    for name in args.cases:
        fn, nbytes, kernel = CASES[name](dev)
        t = _time(fn, args.launches)
        gpu_ops.check_device_errors(dev)
        gbs = nbytes / t / 1e9
        line = {"case": name, "kernel": kernel, "us_per_launch": round(t * 1e6, 2),
                "algorithmic_bytes": int(nbytes), "achieved_gbs": round(gbs, 1)}
        if name in ("prefill", "prefill_fa"):  # flops, not bytes
            tf = nbytes / t / 1e12
            peak_tf = _bf16_peak()
            line = {"case": name, "kernel": kernel, "us_per_launch": round(t * 1e6, 2), "flops": int(nbytes),
                    "achieved_tflops": round(tf, 1), "frac_of_bf16_peak": round(tf / peak_tf, 4),
                    "launches": args.launches}
            print(json.dumps(line), flush=True)
            del fn
            torch.cuda.empty_cache()
            continue
        if name == "host_mapped":
            pcie = pinned_copy_gbs(dev)
            line.update({"pinned_copy_gbs": round(pcie, 1), "frac_of_pinned_copy": round(gbs / pcie, 4),
                         "frac_of_pcie5_x16_nominal": round(gbs / PCIE5_X16_GBS, 4)})
        else:
            line["frac_of_hbm"] = round(gbs / peak, 4)
        line["launches"] = args.launches
        print(json.dumps(line), flush=True)
        del fn
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
