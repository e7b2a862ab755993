"""Kernel-level parity of the tier-aware KV write and the log-sum-exp merges
on the GPU, against the oracle (the reference's tests this mirrors:
fastdecode tests/test_cpu_kernel.py:75-96 store_kv bit-exact and its range
check, :99-147 the split/merge invariant and FlashAttention's +inf empty
convention; the merge rule is cpu_ops.py:93-113).

* fd_store_kv writes new K/V rows into both tiers at once (G+C numbering:
  slot s in block s // BS, ids >= G in the pinned host tier), skipping slot
  -1, from strided key/value views into a strided (vLLM NHD) HBM view and a
  [C, KVH, BS, D] host tier: both tiers bit-equal to the oracle's write into
  the unified pool.  An out-of-range slot writes nothing and is reported
  through the device error word.
* fd_merge_attn_states (2-way) and fd_merge_partials (P-way) against the
  oracle's merges, including +inf (empty, FlashAttention) and -inf partials
  and rows empty on every side (zeros, lse -inf): fp32 outputs within
  1e-6 relative, lse within 1e-5; 16-bit outputs within one rounding of the
  oracle's fp32 result.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from vllm_fastdecoder_b200 import gpu_ops

    return gpu_ops


def _tiers(G, C, KVH, BS, D, dtype, g):
    """HBM tier as vLLM's NHD cache viewed [B, KVH, BS, D] (strided), host
    tier [C, KVH, BS, D] pinned; both filled with garbage."""
    from vllm_fastdecoder_b200.gpu_ops import KVTier

    dev = torch.device("cuda")
    phys = (torch.randn(G, BS, KVH, 2 * D, generator=g) * 10).to(dtype).to(dev)
    hk = phys[..., :D].permute(0, 2, 1, 3)
    hv = phys[..., D:].permute(0, 2, 1, 3)
    ck = (torch.randn(C, KVH, BS, D, generator=g) * 10).to(dtype).pin_memory()
    cv = (torch.randn(C, KVH, BS, D, generator=g) * 10).to(dtype).pin_memory()
    return phys, (KVTier(hk, hv), KVTier(ck, cv))


def _unified(tiers):
    t0, t1 = tiers
    k = torch.cat([t0.k.cpu().contiguous(), t1.k.clone()])
    v = torch.cat([t0.v.cpu().contiguous(), t1.v.clone()])
    return k, v


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_store_kv_two_tiers_bit_exact(ops, dtype):
    from oracle import oracle as O

    g = torch.Generator().manual_seed(3)
    G, C, KVH, BS, D, m = 40, 60, 4, 16, 128, 300
    dev = torch.device("cuda")
    ops.error_word(dev).zero_()
    _, tiers = _tiers(G, C, KVH, BS, D, dtype, g)
    want_k, want_v = _unified(tiers)
    slots = torch.randperm((G + C) * BS, generator=g)[:m].to(torch.int64)
    slots[::13] = -1  # padding tokens
    # key/value as strided views of a fused qkv projection [m, H + 2 KVH, D]
    qkv = torch.randn(m, 8 + 2 * KVH, D, generator=g).to(dtype)
    key, value = qkv[:, 8:8 + KVH], qkv[:, 8 + KVH:]
    keep = slots >= 0
    O.store_kv(key[keep].contiguous(), value[keep].contiguous(), slots[keep].contiguous(), want_k, want_v)
    d_qkv = qkv.to(dev)
    ops.store_kv_tiered(d_qkv[:, 8:8 + KVH], d_qkv[:, 8 + KVH:], slots.to(dev), tiers, G)
    torch.cuda.synchronize()
    ops.check_device_errors(dev)
    got_k, got_v = _unified(tiers)
    assert torch.equal(got_k.view(torch.uint8), want_k.view(torch.uint8))
    assert torch.equal(got_v.view(torch.uint8), want_v.view(torch.uint8))


def test_store_kv_out_of_range_writes_nothing(ops):
    g = torch.Generator().manual_seed(4)
    G, C, KVH, BS, D, m = 8, 8, 2, 16, 64, 40
    dev = torch.device("cuda")
    ops.error_word(dev).zero_()
    _, tiers = _tiers(G, C, KVH, BS, D, torch.float16, g)
    before_k, before_v = _unified(tiers)
    slots = torch.randperm((G + C) * BS, generator=g)[:m].to(torch.int64)
    slots[17] = (G + C) * BS  # one past the last slot of the host tier
    k = torch.randn(m, KVH, D, generator=g).to(torch.float16).to(dev)
    v = torch.randn(m, KVH, D, generator=g).to(torch.float16).to(dev)
    ops.store_kv_tiered(k, v, slots.to(dev), tiers, G)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError):
        ops.check_device_errors(dev)
    ops.error_word(dev).zero_()
    after_k, after_v = _unified(tiers)
    assert torch.equal(after_k.view(torch.uint8), before_k.view(torch.uint8))
    assert torch.equal(after_v.view(torch.uint8), before_v.view(torch.uint8))
    # the reference signature with host-side slots raises before launching
    kc = torch.zeros(C, KVH, BS, D, dtype=torch.float16, device=dev)
    vc = torch.zeros_like(kc)
    with pytest.raises(RuntimeError):
        ops.store_kv(k.contiguous(), v.contiguous(), torch.full((m,), C * BS, dtype=torch.int64), kc, vc)
    assert not kc.any() and not vc.any()


def _large_case(g, m):
    """A prefill-sized write (more than 2048 rows: the check kernel, then the
    copy as its dependent launch), rows spread over both tiers."""
    G, C, KVH, BS, D = 1200, 400, 2, 16, 64
    _, tiers = _tiers(G, C, KVH, BS, D, torch.float16, g)
    slots = torch.randperm((G + C) * BS, generator=g)[:m].to(torch.int64)
    slots[::101] = -1
    k = torch.randn(m, KVH, D, generator=g).to(torch.float16)
    v = torch.randn(m, KVH, D, generator=g).to(torch.float16)
    return G, tiers, slots, k, v


def test_store_kv_two_launch_form_bit_exact(ops):
    """m = 20000 rows: twenty check CTAs (1024 slots each) folded into one
    flag, then the full-grid copy; repeated calls reuse the flag ring."""
    from oracle import oracle as O

    g = torch.Generator().manual_seed(21)
    dev = torch.device("cuda")
    ops.error_word(dev).zero_()
    G, tiers, slots, k, v = _large_case(g, 20000)
    want_k, want_v = _unified(tiers)
    keep = slots >= 0
    O.store_kv(k[keep].contiguous(), v[keep].contiguous(), slots[keep].contiguous(), want_k, want_v)
    dk, dv, ds = k.to(dev), v.to(dev), slots.to(dev)
    for _ in range(3):
        ops.store_kv_tiered(dk, dv, ds, tiers, G)
    torch.cuda.synchronize()
    ops.check_device_errors(dev)
    got_k, got_v = _unified(tiers)
    assert torch.equal(got_k.view(torch.uint8), want_k.view(torch.uint8))
    assert torch.equal(got_v.view(torch.uint8), want_v.view(torch.uint8))


def test_store_kv_two_launch_form_out_of_range_writes_nothing(ops):
    """One bad slot in the seventeenth check CTA's range: no row of the call is
    written and the error word says so; a good call afterwards (the flags
    reset by the last check CTA) writes everything, also from a CUDA graph."""
    from oracle import oracle as O

    g = torch.Generator().manual_seed(22)
    dev = torch.device("cuda")
    ops.error_word(dev).zero_()
    G, tiers, slots, k, v = _large_case(g, 20000)
    before_k, before_v = _unified(tiers)
    bad = slots.clone()
    bad[17000] = (G + 400) * 16  # one past the last slot of the host tier
    dk, dv = k.to(dev), v.to(dev)
    for _ in range(2):
        ops.store_kv_tiered(dk, dv, bad.to(dev), tiers, G)
        torch.cuda.synchronize()
        with pytest.raises(RuntimeError):
            ops.check_device_errors(dev)
        ops.error_word(dev).zero_()
        after_k, after_v = _unified(tiers)
        assert torch.equal(after_k.view(torch.uint8), before_k.view(torch.uint8))
        assert torch.equal(after_v.view(torch.uint8), before_v.view(torch.uint8))
    want_k, want_v = _unified(tiers)
    keep = slots >= 0
    O.store_kv(k[keep].contiguous(), v[keep].contiguous(), slots[keep].contiguous(), want_k, want_v)
    ds = slots.to(dev)
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s), torch.cuda.graph(graph, stream=s):
        ops.store_kv_tiered(dk, dv, ds, tiers, G)
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    ops.check_device_errors(dev)
    got_k, got_v = _unified(tiers)
    assert torch.equal(got_k.view(torch.uint8), want_k.view(torch.uint8))
    assert torch.equal(got_v.view(torch.uint8), want_v.view(torch.uint8))


def _lse(H, n, g, empty_frac=0.15):
    lse = torch.randn(H, n, generator=g) * 3
    r = torch.rand(H, n, generator=g)
    lse[r < empty_frac] = float("inf")  # FlashAttention's empty partial
    lse[(r >= empty_frac) & (r < 2 * empty_frac)] = float("-inf")
    return lse


@pytest.mark.parametrize("dtype,D", [(torch.float16, 128), (torch.bfloat16, 128), (torch.float32, 128),
                                     (torch.float16, 20), (torch.float32, 6)])
def test_merge_attn_states_matches_oracle(ops, dtype, D):
    """D = 128: the vectorized kernel (16-byte chunks); D = 20 fp16 / 6 fp32:
    rows that are not a whole number of 16-byte chunks (the general kernel)."""
    from oracle import oracle as O

    g = torch.Generator().manual_seed(5)
    n, H = 37, 8
    dev = torch.device("cuda")
    o_a = torch.randn(n, H, D, generator=g).to(dtype)
    o_b = torch.randn(n, H, D, generator=g).to(dtype)
    la, lb = _lse(H, n, g), _lse(H, n, g)
    la[:, 5] = float("inf")  # row 5: empty on both sides (+inf and -inf)
    lb[:, 5] = float("-inf")
    want_lse = torch.empty(H, n)
    want = O.merge2(o_a, la, o_b, lb, want_lse)
    assert torch.all(want[5] == 0)
    # fp32 output (the form the backend's merge of partials takes)
    out = torch.full((n, H, D), float("nan"), device=dev)
    out_lse = torch.empty(H, n, device=dev)
    ops.merge_attn_states(out, o_a.to(dev), la.to(dev), o_b.to(dev), lb.to(dev), out_lse)
    torch.cuda.synchronize()
    torch.testing.assert_close(out.cpu(), want, atol=1e-6, rtol=1e-6)
    torch.testing.assert_close(out_lse.cpu(), want_lse, atol=1e-5, rtol=1e-6)
    # output rows scattered through out_rows, in the partials' dtype
    rows = torch.randperm(2 * n, generator=g)[:n].to(torch.int64)
    out2 = torch.full((2 * n, H, D), float("nan"), dtype=dtype, device=dev)
    ops.merge_attn_states(out2, o_a.to(dev), la.to(dev), o_b.to(dev), lb.to(dev), None, out_rows=rows.to(dev))
    torch.cuda.synchronize()
    tol = {torch.float16: 1e-3, torch.bfloat16: 8e-3, torch.float32: 1e-6}[dtype]
    torch.testing.assert_close(out2.cpu()[rows].float(), want, atol=tol, rtol=tol)
    untouched = torch.ones(2 * n, dtype=torch.bool)
    untouched[rows] = False
    assert torch.all(torch.isnan(out2.cpu()[untouched].float()))


@pytest.mark.parametrize("P,D", [(2, 128), (3, 128), (8, 128), (16, 64), (17, 128), (4, 6)])
def test_merge_partials_matches_oracle(ops, P, D):
    """Up to 16 parts with D a multiple of 4: the vectorized kernel; 17 parts
    or D = 6: the general kernel."""
    from oracle import oracle as O

    g = torch.Generator().manual_seed(6 + P)
    n, H = 8, 32
    dev = torch.device("cuda")
    stride = n * H * D + H * n
    parts = torch.empty(P, stride)
    for p in range(P):
        parts[p, :n * H * D] = torch.randn(n * H * D, generator=g)
        parts[p, n * H * D:] = _lse(H, n, g, empty_frac=0.2).flatten()
    parts[:, n * H * D:].view(P, H, n)[:, 3, 2] = float("-inf")  # (row 2, head 3) empty in every part
    want_lse = torch.empty(H, n)
    want = O.merge_parts(parts, P, n, H, D, want_lse)
    out = torch.full((n, H, D), float("nan"), device=dev)
    out_lse = torch.empty(H, n, device=dev)
    ops.merge_partials(parts.to(dev), P, n, H, D, out, out_lse)
    torch.cuda.synchronize()
    assert torch.all(out.cpu()[2, 3] == 0) and out_lse.cpu()[3, 2] == float("-inf")
    torch.testing.assert_close(out.cpu(), want, atol=1e-6, rtol=1e-5)
    torch.testing.assert_close(out_lse.cpu(), want_lse, atol=1e-5, rtol=1e-6)
