"""Host-side plan of the chunked host-tier staging (gpu_ops.plan_chunked_staging):
every block a row reads lands in exactly one part (HBM part or one chunk),
each part's table lists the row's blocks with its last, partly filled block
at the end, and the parts' token counts add up to the row length.  Runs on
CPU (no kernel is launched)."""

from __future__ import annotations

import pytest
import torch

from vllm_fastdecoder_b200 import gpu_ops, workloads


def _check_plan(bt, lens, BS, G, plan):
    n = bt.shape[0]
    total = sum(ln.to(torch.int64) for ln in plan.lens)
    assert torch.equal(total, lens.to(torch.int64).clamp(min=0))
    assert plan.chunks == sorted(plan.chunks)
    if plan.chunks:
        assert plan.chunks[0][0] == plan.lo and plan.chunks[-1][1] == plan.hi
        assert all(a[1] == b[0] for a, b in zip(plan.chunks, plan.chunks[1:]))
    for i in range(n):
        L = int(lens[i])
        nb = (L + BS - 1) // BS
        want = sorted(bt[i, :nb].tolist())
        got = []
        for p, (t, ln) in enumerate(zip(plan.tables, plan.lens)):
            c = (int(ln[i]) + BS - 1) // BS
            ids = t[i, :c].tolist()
            if p > 0:
                lo, hi = plan.chunks[p - 1]
                assert all(lo <= x + plan.lo < hi for x in ids)
                ids = [x + plan.lo + G for x in ids]
            else:
                assert all(x < G for x in ids)
            got += ids
            if c and int(ln[i]) % BS:  # a part holding the partly filled block ends with it
                assert ids[-1] == int(bt[i, nb - 1])
        assert sorted(got) == want


@pytest.mark.parametrize("chunks", [1, 2, 8, 10000])
def test_chunked_staging_plan_config1(chunks):
    b = workloads.config1()
    plan = gpu_ops.plan_chunked_staging(b.block_table, b.lens, b.BS, b.G, chunks)
    assert len(plan.chunks) == min(chunks, plan.hi - plan.lo)
    assert (plan.lo, plan.hi) == gpu_ops.host_block_range(b.block_table, b.lens, b.BS, b.G)
    _check_plan(b.block_table, b.lens, b.BS, b.G, plan)


def test_chunked_staging_plan_edge_rows():
    BS, G = 16, 10
    lens = torch.tensor([0, 1, 16, 17, 40, 48], dtype=torch.int32)
    bt = torch.tensor([[0, 0, 0],
                       [12, 0, 0],   # one partly filled host block
                       [3, 0, 0],    # one full HBM block
                       [15, 4, 0],   # host then HBM (the partial block)
                       [11, 19, 2],  # host, host, HBM partial
                       [13, 5, 14]], dtype=torch.int32)  # host, HBM, host (all full)
    for chunks in (1, 3, 9):
        plan = gpu_ops.plan_chunked_staging(bt, lens, BS, G, chunks)
        assert (plan.lo, plan.hi) == (1, 10)
        _check_plan(bt, lens, BS, G, plan)
    none = gpu_ops.plan_chunked_staging(bt[:, :1] * 0, lens.clamp(max=16), BS, G, 4)
    assert none.chunks == [] and len(none.tables) == 1
