"""Pin the CPU oracle to the reference: the C restatement and the float64
restatement must reproduce the outputs the reference itself produced
(tests/golden/*.npz, written by tests/golden/make_golden.py from the
reference's compiled AVX2 kernel, its ref_decode_attn, its merge rule and its
store_kv).  CPU only."""

from __future__ import annotations

import hashlib
import math
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle as O

GOLD = Path(__file__).resolve().parent / "golden"
DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def from_np(a: np.ndarray, dtype: torch.dtype) -> torch.Tensor:
    t = torch.from_numpy(a.copy())
    return t.view(torch.bfloat16) if dtype == torch.bfloat16 else t


@pytest.fixture(scope="module")
def dec():
    return np.load(GOLD / "decode_avx2.npz")


@pytest.mark.parametrize("dname", list(DTYPES))
@pytest.mark.parametrize("H,KVH", [(8, 8), (8, 2), (4, 1)])
@pytest.mark.parametrize("D", [64, 128, 72])
def test_oracle_matches_reference_avx2(dec, dname, H, KVH, D):
    dtype = DTYPES[dname]
    key = f"{dname}_H{H}_KVH{KVH}_D{D}"
    n, BS, C = 7, 16, 64
    q, kc, vc, bt, lens = O.rand_case(n, H, KVH, D, BS, C, dtype, max_len=93, seed=D + H)
    lens[3] = 0
    # the regenerated inputs are the reference test's inputs, byte for byte
    assert [sha(t) for t in (q, kc, vc, bt, lens)] == list(dec[key + "/sha_inputs"])
    scale = 1.0 / math.sqrt(D)
    out = torch.empty_like(q)
    lse = torch.empty(H, n)
    O.decode_attn(q, kc, vc, bt, lens, scale, out, lse)
    ref_out = from_np(dec[key + "/out"], dtype)
    ref_lse = torch.from_numpy(dec[key + "/lse"])
    nz = lens > 0
    # one rounding step of the output dtype apart at most (exp polynomial vs libm)
    ulp = {torch.float16: 2e-3, torch.bfloat16: 1.6e-2, torch.float32: 2e-6}[dtype]
    torch.testing.assert_close(out.float(), ref_out.float(), atol=ulp, rtol=ulp)
    torch.testing.assert_close(lse[:, nz], ref_lse[:, nz], atol=2e-6, rtol=0)
    assert torch.equal(out[~nz], ref_out[~nz]) and torch.all(out[~nz] == 0)
    assert torch.all(torch.isneginf(lse[:, ~nz]))
    if D == 128:
        f_out, f_lse = O.ref_decode_attn_f64(q, kc, vc, bt, lens, scale)
        torch.testing.assert_close(f_out.float(), torch.from_numpy(dec[key + "/f64_out"]), atol=1e-6, rtol=1e-6)
        torch.testing.assert_close(f_lse[:, nz].float(), torch.from_numpy(dec[key + "/f64_lse"])[:, nz],
                                   atol=1e-6, rtol=1e-7)


def test_oracle_large_scores_match_reference(dec):
    n, H, KVH, D, BS, C = 2, 4, 4, 64, 16, 8
    q, kc, vc, bt, lens = O.rand_case(n, H, KVH, D, BS, C, torch.float32, 40, 0)
    q = q * 300.0
    out = torch.empty_like(q)
    lse = torch.empty(H, n)
    O.decode_attn(q, kc, vc, bt, lens, 1.0, out, lse)
    torch.testing.assert_close(out, torch.from_numpy(dec["large/out"]), atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(lse, torch.from_numpy(dec["large/lse"]), atol=1e-3, rtol=1e-6)


@pytest.mark.parametrize("dname", list(DTYPES))
def test_oracle_merge_matches_reference(dname):
    m = np.load(GOLD / "merge.npz")
    dtype = DTYPES[dname]
    o_a = from_np(m[f"{dname}/o_a"], dtype)
    o_b = from_np(m[f"{dname}/o_b"], dtype)
    lse_a = torch.from_numpy(m[f"{dname}/lse_a"])
    lse_b = torch.from_numpy(m[f"{dname}/lse_b"])
    got = O.merge2(o_a, lse_a, o_b, lse_b)
    torch.testing.assert_close(got, torch.from_numpy(m[f"{dname}/merged"]), atol=1e-6, rtol=1e-6)
    # both-empty rows are exactly zero
    assert torch.all(got[3, 2] == 0) and torch.all(got[4, 3] == 0)


def test_oracle_merge_parts_reduces_to_merge2():
    g = torch.Generator().manual_seed(4)
    n, H, D, P = 5, 3, 16, 2
    o = torch.randn(P, n, H, D, generator=g)
    lse = torch.randn(P, H, n, generator=g)
    lse[0, 1, 2] = float("inf")
    lse[:, 2, 4] = float("-inf")
    packed = torch.cat([torch.cat([o[p].flatten(), lse[p].flatten()]) for p in range(P)]).view(P, -1)
    a = O.merge_parts(packed, P, n, H, D)
    b = O.merge2(o[0], lse[0], o[1], lse[1])
    torch.testing.assert_close(a, b, atol=1e-6, rtol=1e-6)


@pytest.mark.parametrize("dname", ["float16", "bfloat16"])
def test_oracle_store_kv_matches_reference(dname):
    st = np.load(GOLD / "store_kv.npz")
    dt = DTYPES[dname]
    C, KVH, BS, D, m = 10, 4, 16, 128, 37
    g = torch.Generator().manual_seed(1)
    kc = torch.zeros(C, KVH, BS, D, dtype=dt)
    vc = torch.zeros_like(kc)
    k = torch.randn(m, KVH, D, generator=g).to(dt)
    v = torch.randn(m, KVH, D, generator=g).to(dt)
    slots = torch.randperm(C * BS, generator=g)[:m].to(torch.int64)
    assert torch.equal(slots, torch.from_numpy(st[f"{dname}/slots"]))
    O.store_kv(k, v, slots, kc, vc)
    assert [sha(k), sha(v), sha(kc), sha(vc)] == list(st[f"{dname}/sha"])


def test_oracle_store_kv_rejects_out_of_range():
    kc = torch.zeros(2, 1, 16, 64, dtype=torch.float16)
    vc = kc.clone()
    k = torch.ones(1, 1, 64, dtype=torch.float16)
    with pytest.raises(RuntimeError):
        O.store_kv(k, k, torch.tensor([32], dtype=torch.int64), kc, vc)
    assert torch.all(kc == 0)


def test_oracle_split_merge_equals_full():
    """The LSE merge of any two-way partition equals full attention
    (reference test_cpu_kernel.py:99-138), on the oracle."""
    n, H, KVH, D, BS, C = 5, 8, 2, 128, 16, 64
    q, kc, vc, bt, lens = O.rand_case(n, H, KVH, D, BS, C, torch.float16, 80, 7)
    lens.clamp_(min=1)
    scale = D ** -0.5
    full, _ = O.ref_decode_attn_f64(q, kc, vc, bt, lens, scale)
    bt_a, bt_b = torch.zeros_like(bt), torch.zeros_like(bt)
    la, lb = torch.zeros_like(lens), torch.zeros_like(lens)
    for i in range(n):
        L = int(lens[i])
        nb = (L + BS - 1) // BS
        a, b = [], []
        for j in range(nb):
            ntok = BS if j < nb - 1 else L - (nb - 1) * BS
            (a if j % 2 == 0 else b).append((int(bt[i, j]), ntok))
        bt_a[i, :len(a)] = torch.tensor([x for x, _ in a], dtype=torch.int32)
        if b:
            bt_b[i, :len(b)] = torch.tensor([x for x, _ in b], dtype=torch.int32)
        la[i] = sum(t for _, t in a)
        lb[i] = sum(t for _, t in b)
    # the odd half may end in a partial block only if the row's last block is odd;
    # partial blocks in the middle are not expressible, so keep even-count rows
    o_a = torch.empty_like(q)
    l_a = torch.empty(H, n)
    o_b = torch.empty_like(q)
    l_b = torch.empty(H, n)
    O.decode_attn(q, kc, vc, bt_a, la, scale, o_a, l_a)
    O.decode_attn(q, kc, vc, bt_b, lb, scale, o_b, l_b)
    merged = O.merge2(o_a, l_a, o_b, l_b)
    torch.testing.assert_close(merged.double(), full, atol=2e-3, rtol=2e-3)


def test_half_conversion_round_trip():
    """The oracle's fp16/bf16 rounding equals torch's on edge values."""
    vals = torch.tensor([0.0, -0.0, 1.0, 65504.0, 65519.0, 65520.0, 1e-8, 5.96e-8, 2.98e-8, 6.1e-5,
                         3.0e-5, -2.5, 1 / 3, float("inf"), -float("inf"), 1.0009765625, 1.00048828125])
    L = O.lib()
    for v in vals.tolist():
        h = L.fdo_float_to_half(v)
        assert h == torch.tensor([v]).half().view(torch.int16).item() & 0xFFFF, v
        b = L.fdo_float_to_bf16(v)
        assert b == torch.tensor([v]).bfloat16().view(torch.int16).item() & 0xFFFF, v
    for bits in range(0, 1 << 16, 97):
        if (bits & 0x7C00) == 0x7C00:
            continue
        h = torch.tensor([bits], dtype=torch.int32).to(torch.int16).view(torch.float16)
        assert L.fdo_half_to_float(bits) == h.float().item()
