"""The per-step planner is bit-exact against the reference planner: every
HostPlan / DevicePlan field (value, dtype, shape) recorded from the reference
(fastdecode/plan.py:103-245) on its REQS scenario, the error cases and a
continuous-batching trace (tests/golden/plan.npz).  CPU only."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from vllm_fastdecoder_b200 import plan

GOLD = Path(__file__).resolve().parent / "golden"
HP_FIELDS = ["gpu_slot_mapping", "cpu_w_tok", "cpu_w_slot", "p_tok", "p_cu", "p_seqlens", "p_req",
             "s_tok", "s_gpu_bt", "s_gpu_lens", "s_cpu_bt", "s_cpu_lens", "f_tok", "f_cu"]
HP_INTS = ["n_tok", "p_max_q", "p_max_k", "s_max_gpu_len", "f_max"]
DP_FIELDS = ["gpu_slot_mapping", "cpu_w_tok", "p_tok", "p_cu", "p_seqlens", "p_bt", "s_tok",
             "s_gpu_rows", "s_gpu_cu", "s_gpu_bt", "s_gpu_lens", "f_tok", "f_cu"]


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD / "plan.npz")


def _inputs(gold, key):
    qsl = torch.from_numpy(gold[f"{key}/in_qsl"])
    seq = torch.from_numpy(gold[f"{key}/in_seq"])
    bt = torch.from_numpy(gold[f"{key}/in_bt"])
    slots = torch.from_numpy(gold[f"{key}/in_slots"])
    G, C, BS = (int(x) for x in gold[f"{key}/in_GCBS"])
    return qsl, seq, bt, slots, G, C, BS


def _check_case(gold, key):
    qsl, seq, bt, slots, G, C, BS = _inputs(gold, key)
    if f"{key}/raises" in gold:
        exc = {"NotImplementedError": NotImplementedError, "RuntimeError": RuntimeError}[str(gold[f"{key}/raises"][0])]
        with pytest.raises(exc):
            plan.build_host_plan(qsl, seq, bt, slots, G, C, BS)
        return
    hp = plan.build_host_plan(qsl, seq, bt, slots, G, C, BS)
    if f"{key}/none" in gold:
        assert hp is None
        return
    assert hp is not None
    for f in HP_FIELDS:
        got = getattr(hp, f)
        want = gold[f"{key}/hp/{f}"]
        assert str(got.dtype) == str(gold[f"{key}/hp_dtype/{f}"][0]), (key, f, got.dtype)
        assert tuple(got.shape) == want.shape, (key, f, got.shape, want.shape)
        assert np.array_equal(got.numpy(), want), (key, f)
    assert [getattr(hp, f) for f in HP_INTS] == list(gold[f"{key}/hp_ints"]), key
    dp = plan.to_device(hp, bt, "cpu")
    for f in DP_FIELDS:
        got = getattr(dp, f)
        want = gold[f"{key}/dp/{f}"]
        assert tuple(got.shape) == want.shape and np.array_equal(got.numpy(), want), (key, f)
    # this engine's additions are consistent with the reference fields
    assert torch.equal(qsl.long()[hp.s_req], hp.s_tok)
    assert torch.equal(hp.s_seq_lens, hp.s_gpu_lens + hp.s_cpu_lens)
    host = dp.slot_mapping[hp.cpu_w_tok]
    assert torch.equal(host, slots[:hp.n_tok][hp.cpu_w_tok])
    keep = hp.gpu_slot_mapping >= 0
    assert torch.equal(dp.slot_mapping[keep], hp.gpu_slot_mapping[keep])


@pytest.mark.parametrize("key", ["reqs", "all_gpu", "chunked", "beyond"])
def test_plan_cases_bit_exact(gold, key):
    _check_case(gold, key)


def test_plan_trace_bit_exact(gold):
    n = int(gold["n_trace"][0])
    assert n >= 40
    for k in range(n):
        _check_case(gold, f"trace{k}")


def test_plan_classification_known_answers(gold):
    """The known-answer lists of the reference test (test_plan_and_forward.py:199-228)."""
    qsl, seq, bt, slots, G, C, BS = _inputs(gold, "reqs")
    hp = plan.build_host_plan(qsl, seq, bt, slots, G, C, BS)
    assert hp.p_req.tolist() == [1, 3]
    assert hp.s_tok.tolist() == [0, 11, 12, 13]
    assert hp.f_cu.tolist() == [0, 6]
    assert hp.s_gpu_lens.tolist() == [8, 0, 4, 0]
    assert hp.s_cpu_lens.tolist() == [1, 4, 8, 1]
    assert hp.s_gpu_bt[2, 0].item() == 7
    assert hp.s_cpu_bt[2, :2].tolist() == [16 - G, 17 - G]
    assert hp.pd_req.tolist() == [1]  # the all-HBM decode
    cpu_mask = slots >= G * BS
    assert torch.equal(hp.gpu_slot_mapping[cpu_mask], torch.full((int(cpu_mask.sum()),), -1))
    assert torch.equal(hp.cpu_w_slot, slots[cpu_mask] - G * BS)


def test_pack_rows_and_spans_edges():
    ids = torch.tensor([[5, 9, 2, 7], [1, 1, 1, 1]])
    keep = torch.tensor([[False, True, False, True], [False, False, False, False]])
    assert plan.pack_rows(ids, keep, 1).tolist() == [[8, 6], [0, 0]]
    assert plan.pack_rows(ids, keep, 0, multiple=16).shape == (2, 16)
    assert plan.pack_rows(torch.zeros(3, 0, dtype=torch.int64), torch.zeros(3, 0, dtype=torch.bool), 0,
                          multiple=16).shape == (3, 16)
    assert plan.spans(torch.tensor([3, 10, 0]), torch.tensor([2, 0, 3])).tolist() == [3, 4, 0, 1, 2]
    assert plan.spans(torch.tensor([], dtype=torch.int64), torch.tensor([], dtype=torch.int64)).numel() == 0
    assert plan.prefix_offsets(torch.tensor([2, 0, 3])).tolist() == [0, 2, 2, 5]
