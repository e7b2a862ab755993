"""Host-side logic of the benchmark workloads and the staging range (CPU only):
the config-4 trace generator keeps its invariants over many steps (every
running request's blocks are distinct from every other's, HBM ids are handed
out before host ids, each new token's slot is the position it decodes, the
host ids stay inside the tier), host_block_range returns the exact span of
the host blocks a step reads, and the planner's host_lo / host_hi / host_used
agree with it."""

from __future__ import annotations

import torch

from vllm_fastdecoder_b200 import gpu_ops, plan, workloads


def _used_ids(bt, lens, BS):
    out = []
    for i in range(bt.shape[0]):
        nb = (int(lens[i]) + BS - 1) // BS
        out.append([int(x) for x in bt[i, :nb]])
    return out


def test_trace4_invariants():
    tr = workloads.trace4(seed=5, steps=40)
    BS, G = tr.BS, tr.G
    assert tr.layers == 32 and (tr.H, tr.KVH, tr.D) == (32, 32, 128)
    for k, st in enumerate(tr.steps):
        R = st.rows
        assert 100 <= R <= 128, (k, R)
        rows = _used_ids(st.block_table, st.lens, BS)
        flat = [b for r in rows for b in r]
        assert len(flat) == len(set(flat)), k  # no block shared by two requests
        assert all(1 <= b < G + tr.host_blocks for b in flat), k  # id 0 is the null block
        for i, r in enumerate(rows):
            pos = int(st.lens[i]) - 1
            assert int(st.slots[i]) == r[pos // BS] * BS + pos % BS, (k, i)
        # HBM-first: a block taken this step (a row whose new token opens a
        # block) comes from the host tier only when every HBM block is in use
        # (nothing is freed within a step)
        new_host = any(int(st.lens[i]) % BS == 1 % BS and r[-1] >= G for i, r in enumerate(rows))
        if new_host:
            assert len({b for b in flat if b < G}) == G - 1, k
    # the warm start fills the HBM tier before the host tier
    first = [b for r in _used_ids(tr.steps[0].block_table, tr.steps[0].lens, BS) for b in r]
    assert any(b >= G for b in first) and len({b for b in first if b < G}) == G - 1
    # prompts U[128, 1024] + progress: every length within [129, 2048]
    assert all(129 <= int(x) <= 2048 for st in tr.steps for x in st.lens)


def test_host_block_range_is_exact():
    g = torch.Generator().manual_seed(1)
    BS, G, W = 16, 100, 12
    for _ in range(50):
        n = int(torch.randint(1, 9, (1,), generator=g))
        lens = torch.randint(0, W * BS + 1, (n,), generator=g).to(torch.int32)
        bt = torch.randint(0, G + 300, (n, W), generator=g).to(torch.int32)
        ids = [b for r in _used_ids(bt, lens, BS) for b in r if b >= G]
        want = (min(ids) - G, max(ids) - G + 1) if ids else (0, 0)
        assert gpu_ops.host_block_range(bt, lens, BS, G) == want


def test_plan_host_range_fields():
    tr = workloads.trace4(seed=2, steps=6)
    for st in tr.steps:
        R = st.rows
        qsl = torch.arange(R + 1, dtype=torch.int32)
        hp = plan.build_host_plan(qsl, st.lens, st.block_table, st.slots, tr.G, tr.host_blocks, tr.BS)
        lo, hi = gpu_ops.host_block_range(st.block_table, st.lens, tr.BS, tr.G)
        assert (hp.host_lo, hp.host_hi) == (lo, hi)
        used = sum(1 for r in _used_ids(st.block_table, st.lens, tr.BS) for b in r if b >= tr.G)
        assert hp.host_used == used
