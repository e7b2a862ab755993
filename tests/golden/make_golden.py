"""Generate the golden fixtures in this directory from the reference itself.

Run where the reference checkout exists (FD_REFERENCE_DIR, else a directory
named `reference` beside this repository) after `make -C oracle` has compiled
the reference's CPU kernel into oracle/_ref:

    python tests/golden/make_golden.py

What is recorded (all from reference code, nothing from this engine):
  decode_avx2.npz      outputs of the reference's compiled AVX2 decode_attn
                       (fastdecode/csrc/cpu_attn.cpp) on the seeded cases of
                       its tests/test_cpu_kernel.py:38-72, plus input
                       checksums so the regenerated inputs are pinned too,
                       and float64 outputs of its ref_decode_attn
                       (fastdecode/cpu_ops.py:54-81) for a subset
  merge.npz            fastdecode/cpu_ops.py:93-113 merge_partials_torch on
                       random partials with +inf / -inf rows
  store_kv.npz         checksums of the caches after the reference store_kv
  plan.npz             every HostPlan / DevicePlan field of the reference
                       planner (fastdecode/plan.py:103-245) on its REQS
                       scenario and on a continuous-batching trace
  forward_split.npz    the reference FastDecodeImpl._forward_split run with
                       its own CPU stand-ins for the GPU ops
                       (tests/test_plan_and_forward.py:48-114) on REQS
"""

from __future__ import annotations

import hashlib
import math
import os
import random
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
REF = Path(os.environ.get("FD_REFERENCE_DIR") or Path(__file__).resolve().parents[3] / "reference")
if not (REF / "fastdecode").is_dir():
    sys.exit(f"reference checkout not found at {REF}: set FD_REFERENCE_DIR")
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(REF))

from oracle import oracle as O  # noqa: E402  (rand_case, reference module loader)


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def np_of(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().copy()  # raw bits
    return t.numpy().copy()


DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}
HKV = [(8, 8), (8, 2), (4, 1)]
DS = [64, 128, 72]


def decode_fixtures() -> None:
    from fastdecode import cpu_ops

    ext = O.load_reference_ext()
    assert ext is not None, "build the reference kernel first: make -C oracle"
    out = {}
    for dname, dt in DTYPES.items():
        for H, KVH in HKV:
            for D in DS:
                key = f"{dname}_H{H}_KVH{KVH}_D{D}"
                n, BS, C = 7, 16, 64
                q, kc, vc, bt, lens = O.rand_case(n, H, KVH, D, BS, C, dt, max_len=93, seed=D + H)
                lens[3] = 0
                scale = 1.0 / math.sqrt(D)
                o = torch.empty_like(q)
                lse = torch.empty(H, n, dtype=torch.float32)
                ext.decode_attn(q, kc, vc, bt, lens, scale, o, lse)
                out[key + "/out"] = np_of(o)
                out[key + "/lse"] = lse.numpy().copy()
                out[key + "/sha_inputs"] = np.array(
                    [sha(q), sha(kc), sha(vc), sha(bt), sha(lens)])
                if D == 128:
                    fo, fl = cpu_ops.ref_decode_attn(q, kc, vc, bt, lens, scale)
                    out[key + "/f64_out"] = fo.float().numpy()
                    out[key + "/f64_lse"] = fl.float().numpy()
    # large-score case (test_cpu_kernel.py:60-72)
    n, H, KVH, D, BS, C = 2, 4, 4, 64, 16, 8
    q, kc, vc, bt, lens = O.rand_case(n, H, KVH, D, BS, C, torch.float32, 40, 0)
    q = q * 300.0
    o = torch.empty_like(q)
    lse = torch.empty(H, n, dtype=torch.float32)
    ext.decode_attn(q, kc, vc, bt, lens, 1.0, o, lse)
    out["large/out"] = o.numpy().copy()
    out["large/lse"] = lse.numpy().copy()
    np.savez_compressed(HERE / "decode_avx2.npz", **out)


def merge_fixtures() -> None:
    from fastdecode import cpu_ops

    g = torch.Generator().manual_seed(17)
    out = {}
    for dname, dt in DTYPES.items():
        n, H, D = 6, 4, 32
        o_a = torch.randn(n, H, D, generator=g).to(dt)
        o_b = torch.randn(n, H, D, generator=g).to(dt)
        lse_a = torch.randn(H, n, generator=g) * 3
        lse_b = torch.randn(H, n, generator=g) * 3
        lse_a[0, 1] = float("inf")  # FlashAttention empty row
        lse_b[1, 2] = float("-inf")  # empty CPU partial
        lse_a[2, 3] = float("-inf")
        lse_b[2, 3] = float("inf")  # both empty
        lse_a[3, 4] = float("-inf")
        lse_b[3, 4] = float("-inf")  # both empty
        m = cpu_ops.merge_partials_torch(o_a, lse_a, o_b, lse_b)
        out[f"{dname}/o_a"] = np_of(o_a)
        out[f"{dname}/o_b"] = np_of(o_b)
        out[f"{dname}/lse_a"] = lse_a.numpy()
        out[f"{dname}/lse_b"] = lse_b.numpy()
        out[f"{dname}/merged"] = m.numpy()
    np.savez_compressed(HERE / "merge.npz", **out)


def store_kv_fixtures() -> None:
    from fastdecode import cpu_ops

    ext = O.load_reference_ext()
    out = {}
    for dname in ("float16", "bfloat16"):
        dt = DTYPES[dname]
        C, KVH, BS, D, m = 10, 4, 16, 128, 37
        g = torch.Generator().manual_seed(1)
        kc = torch.zeros(C, KVH, BS, D, dtype=dt)
        vc = torch.zeros_like(kc)
        kr, vr = kc.clone(), vc.clone()
        k = torch.randn(m, KVH, D, generator=g).to(dt)
        v = torch.randn(m, KVH, D, generator=g).to(dt)
        slots = torch.randperm(C * BS, generator=g)[:m].to(torch.int64)
        ext.store_kv(k, v, slots, kc, vc)
        cpu_ops.ref_store_kv(k, v, slots, kr, vr)
        assert torch.equal(kc, kr) and torch.equal(vc, vr)
        out[f"{dname}/slots"] = slots.numpy()
        out[f"{dname}/sha"] = np.array([sha(k), sha(v), sha(kc), sha(vc)])
    np.savez_compressed(HERE / "store_kv.npz", **out)


# the reference planner test scenario (tests/test_plan_and_forward.py:188-196)
BS_PLAN = 4
REQS = [
    (8, 1, [1, 2, 12]),
    (4, 1, [3, 4]),
    (0, 6, [13, 5]),
    (0, 3, [6]),
    (3, 1, [15]),
    (11, 1, [16, 7, 17]),
    (0, 1, [18]),
]


def plan_inputs(reqs, BS):
    qsl, seq, slots = [0], [], []
    W = max(len(r[2]) for r in reqs)
    bt = torch.zeros(len(reqs), W, dtype=torch.int32)
    for i, (ctx, ql, blocks) in enumerate(reqs):
        L = ctx + ql
        bt[i, :len(blocks)] = torch.tensor(blocks, dtype=torch.int32)
        for p in range(ctx, L):
            slots.append(blocks[p // BS] * BS + p % BS)
        qsl.append(qsl[-1] + ql)
        seq.append(L)
    return (torch.tensor(qsl, dtype=torch.int32), torch.tensor(seq, dtype=torch.int32), bt,
            torch.tensor(slots, dtype=torch.int64))


HP_FIELDS = ["gpu_slot_mapping", "cpu_w_tok", "cpu_w_slot", "p_tok", "p_cu", "p_seqlens", "p_req",
             "s_tok", "s_gpu_bt", "s_gpu_lens", "s_cpu_bt", "s_cpu_lens", "f_tok", "f_cu"]
HP_INTS = ["n_tok", "p_max_q", "p_max_k", "s_max_gpu_len", "f_max"]
DP_FIELDS = ["gpu_slot_mapping", "cpu_w_tok", "p_tok", "p_cu", "p_seqlens", "p_bt", "s_tok",
             "s_gpu_rows", "s_gpu_cu", "s_gpu_bt", "s_gpu_lens", "f_tok", "f_cu"]


def record_plan(out, key, qsl, seq, bt, slots, G, C, BS):
    from fastdecode import plan

    out[f"{key}/in_qsl"] = qsl.numpy()
    out[f"{key}/in_seq"] = seq.numpy()
    out[f"{key}/in_bt"] = bt.numpy()
    out[f"{key}/in_slots"] = slots.numpy()
    out[f"{key}/in_GCBS"] = np.array([G, C, BS])
    try:
        hp = plan.build_host_plan(qsl, seq, bt, slots, G, C, BS)
    except NotImplementedError:
        out[f"{key}/raises"] = np.array(["NotImplementedError"])
        return
    except RuntimeError:
        out[f"{key}/raises"] = np.array(["RuntimeError"])
        return
    if hp is None:
        out[f"{key}/none"] = np.array([1])
        return
    for f in HP_FIELDS:
        t = getattr(hp, f)
        out[f"{key}/hp/{f}"] = t.numpy()
        out[f"{key}/hp_dtype/{f}"] = np.array([str(t.dtype)])
    out[f"{key}/hp_ints"] = np.array([getattr(hp, f) for f in HP_INTS])
    dp = plan.to_device(hp, bt, "cpu")
    for f in DP_FIELDS:
        out[f"{key}/dp/{f}"] = getattr(dp, f).numpy()


def trace_steps(seed, G, C, BS, max_reqs, steps, max_prompt, max_new):
    """Continuous batching in the manner of the reference self-test
    (scripts/gpu_selftest.py:124-198): GPU-first allocation, LIFO reuse,
    junk past the end of each block-table row, shuffled rows."""
    rng = random.Random(seed)
    free_gpu = list(range(1, G))
    free_cpu = list(range(G, G + C))

    def alloc():
        if free_gpu:
            return free_gpu.pop(0)
        if free_cpu:
            return free_cpu.pop(0)
        return None

    def release(blocks):
        free_gpu[:0] = [b for b in blocks if b < G]
        free_cpu.extend(b for b in blocks if b >= G)

    running = []
    for _ in range(steps):
        rows = []
        for r in list(running):
            if r["L"] % BS == 0:
                b = alloc()
                if b is None:
                    running.remove(r)
                    release(r["blocks"])
                    continue
                r["blocks"].append(b)
            rows.append((r, r["L"], 1))
        while len(running) < max_reqs:
            P = 1 if rng.random() < 0.05 else rng.randint(2, max_prompt)
            need = (P + BS - 1) // BS
            if need > len(free_gpu) + len(free_cpu) - 8:
                break
            r = {"blocks": [alloc() for _ in range(need)], "L": 0, "left": rng.randint(1, max_new)}
            running.append(r)
            rows.append((r, 0, P))
        if not rows:
            continue
        rng.shuffle(rows)
        R = len(rows)
        W = max(len(r["blocks"]) for r, _, _ in rows) + 2
        bt = torch.zeros(R, W, dtype=torch.int32)
        slots, qlens, seqs = [], [], []
        for i, (r, ctx, ql) in enumerate(rows):
            bl = r["blocks"]
            bt[i, :len(bl)] = torch.tensor(bl, dtype=torch.int32)
            bt[i, len(bl):] = torch.tensor([rng.randrange(G + C) for _ in range(W - len(bl))], dtype=torch.int32)
            for p in range(ctx, ctx + ql):
                slots.append(bl[p // BS] * BS + p % BS)
            qlens.append(ql)
            seqs.append(ctx + ql)
        qsl = torch.zeros(R + 1, dtype=torch.int32)
        qsl[1:] = torch.cumsum(torch.tensor(qlens), 0)
        yield qsl, torch.tensor(seqs, dtype=torch.int32), bt, torch.tensor(slots, dtype=torch.int64)
        for r, ctx, ql in rows:
            r["L"] = ctx + ql
            r["left"] -= 1
            if r["left"] <= 0:
                running.remove(r)
                release(r["blocks"])


def plan_fixtures() -> None:
    out = {}
    G, C = 10, 20
    record_plan(out, "reqs", *plan_inputs(REQS, BS_PLAN), G, C, BS_PLAN)
    record_plan(out, "all_gpu", *plan_inputs([(4, 1, [1, 2]), (0, 3, [3])], BS_PLAN), 10, 5, BS_PLAN)
    record_plan(out, "chunked", *plan_inputs([(4, 3, [1, 12])], BS_PLAN), 10, 5, BS_PLAN)
    record_plan(out, "beyond", *plan_inputs([(4, 1, [1, 40])], BS_PLAN), 10, 5, BS_PLAN)
    k = 0
    for qsl, seq, bt, slots in trace_steps(0, G=12, C=80, BS=4, max_reqs=10, steps=60, max_prompt=30, max_new=20):
        record_plan(out, f"trace{k}", qsl, seq, bt, slots, 12, 80, 4)
        k += 1
    out["n_trace"] = np.array([k])
    np.savez_compressed(HERE / "plan.npz", **out)


def forward_split_fixture() -> None:
    sys.path.insert(0, str(REF / "tests"))
    import test_plan_and_forward as T  # the reference's own CPU stand-ins
    from fastdecode import backend, cpu_ops, plan, state

    # the reference's loader JIT-builds the same cpu_attn.cpp; hand it the copy
    # compiled from that source by oracle/Makefile instead
    cpu_ops._EXT = O.load_reference_ext()

    backend.OPS = T.CpuOps
    st = state.PinnedStaging.__new__(state.PinnedStaging)
    st._bufs, st._pin = {}, False
    state._STAGING = st
    out = {}
    for H, KVH in ((4, 4), (8, 2)):
        for dname in ("float32", "float16"):
            for seed in (0, 1):
                dt = DTYPES[dname]
                G, C, D = 10, 20, 64
                sc = T._scenario(T.REQS, G, C, H, KVH, D, dt, seed)
                key = f"H{H}_KVH{KVH}_{dname}_s{seed}"
                out[key + "/sha_inputs"] = np.array([sha(sc.query), sha(sc.key), sha(sc.value),
                                                     sha(sc.kv_cache), sha(sc.cpu_k), sha(sc.cpu_v)])
                hp = plan.build_host_plan(sc.qsl, sc.seq_lens, sc.bt, sc.slots, G, C, T.BS)
                dp = plan.to_device(hp, sc.bt, "cpu")
                state.STORE = state.CpuKVStore(num_gpu_blocks=G, num_cpu_blocks=C, block_size=T.BS,
                                               num_kv_heads=KVH, head_size=D, dtype=dt,
                                               k={"l0": sc.cpu_k}, v={"l0": sc.cpu_v})
                impl = T._impl(H, KVH, D, sc.scale)
                from types import SimpleNamespace

                layer = SimpleNamespace(layer_name="l0", _k_scale=None, _v_scale=None)
                output = torch.full_like(sc.query, float("nan"))
                impl._forward_split(layer, sc.query, sc.key, sc.value, sc.kv_cache, dp, output)
                out[key + "/output"] = np_of(output)
                out[key + "/ref_f64"] = sc.ref.numpy()
                out[key + "/sha_after"] = np.array([sha(sc.kv_cache), sha(sc.cpu_k), sha(sc.cpu_v)])
                state.STORE = None
    np.savez_compressed(HERE / "forward_split.npz", **out)


if __name__ == "__main__":
    decode_fixtures()
    merge_fixtures()
    store_kv_fixtures()
    plan_fixtures()
    forward_split_fixture()
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)
