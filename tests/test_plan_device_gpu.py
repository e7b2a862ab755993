"""The device-side planner (fd_plan_step) against the host planner, which the
CPU tests pin bit-exactly to the reference (fastdecode/plan.py:103-245):
every HostPlan field (value, dtype, shape), the None case and both error
cases, on the reference's REQS scenario, its error cases and the recorded
continuous-batching trace (tests/golden/plan.npz), plus random steps of the
config-4 trace generator.  The decode list it emits drives fd_decode_attn
directly (bt_rows, q_rows = out_rows, padding rows untouched); outputs are
compared with a decode over gathered table rows (same kernel: 1e-2 on bf16
outputs, 1e-5 on lse) and with the oracle (bf16 1.6e-2, lse 1e-4)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from vllm_fastdecoder_b200 import plan

pytestmark = pytest.mark.gpu

GOLD = Path(__file__).resolve().parent / "golden"
FIELDS = ["gpu_slot_mapping", "cpu_w_tok", "cpu_w_slot", "p_tok", "p_cu", "p_seqlens", "p_req", "s_tok",
          "s_gpu_bt", "s_gpu_lens", "s_cpu_bt", "s_cpu_lens", "f_tok", "f_cu", "s_req", "s_seq_lens", "pd_req",
          "pd_tok", "pd_seq_lens", "pp_req", "pp_tok", "pp_cu", "pp_seqlens"]
INTS = ["n_tok", "p_max_q", "p_max_k", "s_max_gpu_len", "f_max", "s_max_len", "pd_max_len", "pp_max_q", "pp_max_k",
        "num_gpu_blocks", "block_size"]


def _same_plan(want, got, where):
    if want is None:
        assert got is None, where
        return
    assert got is not None, where
    for f in FIELDS:
        a, b = getattr(want, f), getattr(got, f)
        assert a.dtype == b.dtype and tuple(a.shape) == tuple(b.shape), (where, f, a.dtype, b.dtype, a.shape, b.shape)
        assert torch.equal(a, b), (where, f)
    for f in INTS:
        assert getattr(want, f) == getattr(got, f), (where, f)


def _check(qsl, seq, bt, slots, G, C, BS, where):
    dev = torch.device("cuda")
    try:
        want = plan.build_host_plan(qsl, seq, bt, slots, G, C, BS)
        err = None
    except (RuntimeError, NotImplementedError) as e:
        want, err = None, type(e)
    dp = plan.plan_on_device(qsl.to(dev, torch.int32), seq.to(dev, torch.int32), bt.to(dev, torch.int32).contiguous(),
                             slots.to(dev, torch.int64), G, C, BS)
    if err is not None:
        with pytest.raises(err):
            plan.device_plan_to_host(dp, C)
        return None
    got = plan.device_plan_to_host(dp, C)
    _same_plan(want, got, where)
    # the decode list: every live single-token request, in request order
    q_len = (qsl[1:] - qsl[:-1]).long()
    rows = torch.nonzero(q_len == 1).flatten()
    n = int(dp.header[21].item())
    assert n == rows.numel(), where
    assert torch.equal(dp.d_row[:n].cpu().long(), rows), where
    assert torch.equal(dp.d_tok[:n].cpu(), qsl.long()[rows]), where
    assert torch.equal(dp.d_lens[:n].cpu(), seq.to(torch.int32)[rows]), where
    R = qsl.numel() - 1
    assert torch.all(dp.d_tok[n:R].cpu() == -1) and torch.all(dp.d_lens[n:R].cpu() == 0), where
    # host-side checks: the device error word stays clean on valid steps
    from vllm_fastdecoder_b200 import gpu_ops

    gpu_ops.check_device_errors(dev)
    return dp


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD / "plan.npz")


def _inputs(gold, key):
    t = lambda k: torch.from_numpy(gold[f"{key}/{k}"])  # noqa: E731
    G, C, BS = (int(x) for x in gold[f"{key}/in_GCBS"])
    return t("in_qsl"), t("in_seq"), t("in_bt"), t("in_slots"), G, C, BS


@pytest.mark.parametrize("key", ["reqs", "all_gpu", "chunked", "beyond"])
def test_device_plan_cases(gold, key):
    from vllm_fastdecoder_b200 import gpu_ops

    _check(*_inputs(gold, key), where=key)
    gpu_ops.error_word(torch.device("cuda")).zero_()  # the error cases set it on purpose


def test_device_plan_trace(gold):
    for k in range(int(gold["n_trace"][0])):
        _check(*_inputs(gold, f"trace{k}"), where=f"trace{k}")


def test_device_plan_config4_trace():
    from vllm_fastdecoder_b200 import workloads

    tr = workloads.trace4(seed=3, steps=12)
    for k, st in enumerate(tr.steps):
        R = st.rows
        qsl = torch.arange(R + 1, dtype=torch.int32)
        _check(qsl, st.lens, st.block_table, st.slots, tr.G, tr.host_blocks, tr.BS, where=f"c4[{k}]")


def test_device_plan_many_rows_and_prefills():
    """More requests than the planner's 512 threads (chunked scans with a
    carry), prefills (P and F) among decodes, padding tokens (slot -1)."""
    g = torch.Generator().manual_seed(7)
    R, BS, G, C, W = 2500, 16, 3000, 9000, 40
    q_len = torch.where(torch.rand(R, generator=g) < 0.9, torch.ones(R, dtype=torch.int64),
                        torch.randint(2, 9, (R,), generator=g))
    prior = torch.randint(0, 300, (R,), generator=g)
    host = torch.rand(R, generator=g) < 0.5
    prior = torch.where((q_len > 1) & host, torch.zeros_like(prior), prior)  # fresh prefills only on the host
    seq = prior + q_len
    bt = torch.zeros(R, W, dtype=torch.int32)
    for i in range(R):
        nb = int((seq[i] + BS - 1) // BS)
        ids = torch.randint(1, G, (nb,), generator=g) if not host[i] else torch.randint(G, G + C, (nb,), generator=g)
        bt[i, :nb] = ids.to(torch.int32)
        bt[i, nb:] = torch.randint(0, G + C, (W - nb,), generator=g).to(torch.int32)
    qsl = torch.zeros(R + 1, dtype=torch.int32)
    qsl[1:] = torch.cumsum(q_len, 0).to(torch.int32)
    T = int(qsl[-1])
    slots = torch.randint(0, (G + C) * BS, (T + 5,), generator=g)
    slots[::17] = -1
    _check(qsl, seq.to(torch.int32), bt, slots, G, C, BS, where="many")


@pytest.mark.parametrize("mma", ["1", "0"])
def test_decode_list_drives_decode(monkeypatch, mma):
    """One launch over the planner's decode list equals the decode over
    gathered rows, and leaves the output rows of non-decode tokens untouched."""
    from oracle import oracle as O
    from vllm_fastdecoder_b200 import gpu_ops
    from vllm_fastdecoder_b200.gpu_ops import KVTier

    monkeypatch.setenv("FASTDECODE_B200_MMA", mma)
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(11)
    R, H, KVH, D, BS, G, C = 40, 16, 4, 128, 16, 1000, 1500
    q_len = torch.where(torch.rand(R, generator=g) < 0.8, torch.ones(R, dtype=torch.int64), torch.full((R,), 3))
    seq = torch.randint(1, 600, (R,), generator=g) + q_len
    seq = torch.where(q_len > 1, q_len, seq)  # prefills are fresh (prior context + host blocks is unsupported)
    W = int((seq.max() + BS - 1) // BS) + 2
    perm = torch.randperm(G + C - 1, generator=g) + 1
    bt = torch.zeros(R, W, dtype=torch.int32)
    pos = 0
    for i in range(R):
        nb = int((seq[i] + BS - 1) // BS)
        take = perm[pos:pos + nb] % (G + C)
        pos += nb
        bt[i, :nb] = take.to(torch.int32)
    qsl = torch.zeros(R + 1, dtype=torch.int32)
    qsl[1:] = torch.cumsum(q_len, 0).to(torch.int32)
    T = int(qsl[-1])
    slots = torch.full((T,), -1, dtype=torch.int64)
    dt = torch.bfloat16
    hk = torch.randn(G, KVH, BS, D, generator=g).to(dt)
    hv = torch.randn(G, KVH, BS, D, generator=g).to(dt)
    ck = torch.randn(C, KVH, BS, D, generator=g).to(dt)
    cv = torch.randn(C, KVH, BS, D, generator=g).to(dt)
    tiers = (KVTier(hk.to(dev), hv.to(dev)), KVTier(ck.pin_memory(), cv.pin_memory()))
    q = torch.randn(T, H, D, generator=g).to(dt).to(dev)
    dp = plan.plan_on_device(qsl.to(dev), seq.to(torch.int32).to(dev), bt.to(dev), slots.to(dev), G, C, BS)
    scale = D ** -0.5
    out = torch.full((T, H, D), float("nan"), dtype=dt, device=dev)
    lse = torch.empty(H, R, dtype=torch.float32, device=dev)
    gpu_ops.decode_tiered(q, tiers, G, dp.block_table, dp.d_lens, scale, out, lse, q_rows=dp.d_tok,
                          out_rows=dp.d_tok, bt_rows=dp.d_row, n=R, max_len=int(seq.max()))
    gpu_ops.check_device_errors(dev)
    rows = torch.nonzero(q_len == 1).flatten()
    toks = qsl.long()[rows]
    # the same rows through gathered tables
    ref = torch.full_like(out, float("nan"))
    lse2 = torch.empty(H, rows.numel(), dtype=torch.float32, device=dev)
    gpu_ops.decode_tiered(q, tiers, G, bt[rows].to(dev), seq.to(torch.int32)[rows].to(dev), scale, ref, lse2,
                          q_rows=toks.to(dev), out_rows=toks.to(dev), max_len=int(seq.max()))
    # same kernel, same rows: equal up to the split of the rows over CTAs
    torch.testing.assert_close(out.cpu()[toks].float(), ref.cpu()[toks].float(), atol=1e-2, rtol=1e-2)
    torch.testing.assert_close(lse.cpu()[:, :rows.numel()], lse2.cpu(), atol=1e-5, rtol=1e-5)
    others = torch.ones(T, dtype=torch.bool)
    others[toks] = False
    assert torch.all(torch.isnan(out.cpu()[others].float()))
    # and against the oracle over the unified pool
    kc = torch.cat([hk, ck])
    vc = torch.cat([hv, cv])
    o_or = torch.empty(rows.numel(), H, D, dtype=dt)
    l_or = torch.empty(H, rows.numel())
    O.decode_attn(q.cpu()[toks], kc, vc, bt[rows], seq.to(torch.int32)[rows], scale, o_or, l_or)
    torch.testing.assert_close(out.cpu()[toks].float(), o_or.float(), atol=1.6e-2, rtol=1.6e-2)
    assert (lse.cpu()[:, :rows.numel()] - l_or).abs().max().item() <= 1e-4
