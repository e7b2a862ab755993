"""GPU parity of the split-KV decode kernel (fd_decode_attn through the C ABI)
against the CPU oracle, on the reference's own test cases
(tests/test_cpu_kernel.py:38-72 of the reference) and on two-tier layouts.

Tolerances (written here, per dtype, on the attention output):
  vs the float64 reference: fp16 2e-3, bf16 1.6e-2, fp32 1e-5 (atol = rtol),
  the reference's own bounds (test_cpu_kernel.py:53); lse atol 1e-4.
  vs the fp32 oracle (same rounding of inputs, fp32 accumulation): output
  within 2 ulp of the output dtype at |x| <= 1 (fp16 2e-3, bf16 1.6e-2,
  fp32 2e-6) and lse within 1e-4 absolute.
"""

from __future__ import annotations

import math

import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL_F64 = {torch.float16: 2e-3, torch.bfloat16: 1.6e-2, torch.float32: 1e-5}
TOL_ORACLE = {torch.float16: 2e-3, torch.bfloat16: 1.6e-2, torch.float32: 2e-6}
LSE_TOL = 1e-4


@pytest.fixture(scope="module")
def ops():
    from vllm_fastdecoder_b200 import gpu_ops

    return gpu_ops


def _run_paged(ops, q, kc, vc, bt, lens, scale, host_cache=False, tiles_per_split=0):
    """Run the kernel through the C ABI; tiles_per_split 0 selects the
    persistent schedule (rows <= 1024), > 0 the fixed split grid."""
    dev = torch.device("cuda")
    n, H, D = q.shape
    if host_cache:
        kd, vd = kc.pin_memory(), vc.pin_memory()
    else:
        kd, vd = kc.to(dev), vc.to(dev)
    out = torch.full((n, H, D), float("nan"), dtype=q.dtype, device=dev)
    lse = torch.full((H, n), float("nan"), dtype=torch.float32, device=dev)
    if tiles_per_split:
        from vllm_fastdecoder_b200.gpu_ops import KVTier

        ops.decode_tiered(q.to(dev), (KVTier(kd, vd), None), 1 << 40, bt.to(dev), lens.to(dev), scale, out, lse,
                          tiles_per_split=tiles_per_split)
    else:
        ops.decode_attn(q.to(dev), kd, vd, bt.to(dev), lens.to(dev), scale, out, lse)
    ops.check_device_errors(dev)
    return out.cpu(), lse.cpu()


def _compare(q, kc, vc, bt, lens, scale, out, lse):
    dtype = q.dtype
    n, H, D = q.shape
    o_or = torch.empty_like(q)
    l_or = torch.empty(H, n)
    O.decode_attn(q, kc, vc, bt, lens, scale, o_or, l_or)
    f64_o, f64_l = O.ref_decode_attn_f64(q, kc, vc, bt, lens, scale)
    nz = lens > 0
    t = TOL_F64[dtype]
    torch.testing.assert_close(out[nz].double(), f64_o[nz], atol=t, rtol=t)
    torch.testing.assert_close(lse[:, nz].double(), f64_l[:, nz], atol=LSE_TOL, rtol=1e-5)
    t = TOL_ORACLE[dtype]
    torch.testing.assert_close(out[nz].float(), o_or[nz].float(), atol=t, rtol=t)
    assert (lse[:, nz] - l_or[:, nz]).abs().max().item() <= LSE_TOL
    assert torch.all(out[~nz] == 0)
    assert torch.all(torch.isneginf(lse[:, ~nz]))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("H,KVH", [(8, 8), (8, 2), (4, 1)])
@pytest.mark.parametrize("D", [64, 128, 72])
def test_decode_attn_matches_oracle(ops, dtype, H, KVH, D):
    n, BS, C = 7, 16, 64
    q, kc, vc, bt, lens = O.rand_case(n, H, KVH, D, BS, C, dtype, max_len=93, seed=D + H)
    lens[3] = 0
    scale = 1.0 / math.sqrt(D)
    out, lse = _run_paged(ops, q, kc, vc, bt, lens, scale)
    _compare(q, kc, vc, bt, lens, scale, out, lse)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_decode_attn_host_tier(ops, dtype):
    """Caches in pinned host memory: the kernel reads them over PCIe."""
    n, H, KVH, D, BS, C = 9, 8, 2, 128, 16, 96
    q, kc, vc, bt, lens = O.rand_case(n, H, KVH, D, BS, C, dtype, max_len=150, seed=11)
    lens[4] = 0
    scale = D ** -0.5
    out, lse = _run_paged(ops, q, kc, vc, bt, lens, scale, host_cache=True)
    _compare(q, kc, vc, bt, lens, scale, out, lse)


def test_decode_attn_large_scores(ops):
    """Large logits must not overflow (reference test_cpu_kernel.py:60-72)."""
    n, H, KVH, D, BS, C = 2, 4, 4, 64, 16, 8
    q, kc, vc, bt, lens = O.rand_case(n, H, KVH, D, BS, C, torch.float32, 40, 0)
    q = q * 300.0
    out, lse = _run_paged(ops, q, kc, vc, bt, lens, 1.0)
    ref_out, ref_lse = O.ref_decode_attn_f64(q, kc, vc, bt, lens, 1.0)
    assert torch.isfinite(out).all() and torch.isfinite(lse).all()
    torch.testing.assert_close(out.double(), ref_out, atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(lse.double(), ref_lse, atol=1e-3, rtol=1e-6)


@pytest.mark.parametrize("BS", [1, 4, 8, 32, 64])
def test_decode_attn_block_sizes(ops, BS):
    n, H, KVH, D = 5, 8, 2, 128
    C = max(8, 4096 // BS)
    q, kc, vc, bt, lens = O.rand_case(n, H, KVH, D, BS, C, torch.float16, max_len=700, seed=BS)
    scale = D ** -0.5
    out, lse = _run_paged(ops, q, kc, vc, bt, lens, scale)
    _compare(q, kc, vc, bt, lens, scale, out, lse)


@pytest.mark.parametrize("tiles_per_split", [0, 8, 36])
@pytest.mark.parametrize("dtype,H,KVH", [(torch.float16, 32, 32), (torch.bfloat16, 32, 8)])
def test_decode_attn_many_splits(ops, dtype, H, KVH, tiles_per_split):
    """Rows long enough to be cut across many CTAs: the persistent schedule
    (0) and the fixed split grid (8, 36 tiles per split), both through their
    combine kernels."""
    n, D, BS = 3, 128, 16
    L = 9000
    C = 3 * ((L + BS - 1) // BS) + 4
    q, kc, vc, bt, lens = O.rand_case(n, H, KVH, D, BS, C, dtype, max_len=L, seed=5)
    lens[1] = 17
    lens[2] = 4097
    scale = D ** -0.5
    out, lse = _run_paged(ops, q, kc, vc, bt, lens, scale, tiles_per_split=tiles_per_split)
    _compare(q, kc, vc, bt, lens, scale, out, lse)


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_decode_persistent_ragged_batch(ops, seed):
    """Many rows of very different lengths (empty, single-token, long) so CTA
    ranges start and end at every kind of boundary."""
    import random

    rng = random.Random(seed)
    n, H, KVH, D, BS = 37, 8, 2, 128, 16
    lens_l = [rng.choice([0, 1, 15, 16, 17, rng.randint(1, 3000)]) for _ in range(n)]
    C = sum((x + BS - 1) // BS for x in lens_l) + 8
    q, kc, vc, bt, lens = O.rand_case(n, H, KVH, D, BS, C, torch.bfloat16, max_len=max(lens_l), seed=seed)
    lens = torch.tensor(lens_l, dtype=torch.int32)
    W = bt.shape[1]
    perm = torch.randperm(C, generator=torch.Generator().manual_seed(seed)).tolist()
    bt = torch.zeros(n, W, dtype=torch.int32)
    for i, L in enumerate(lens_l):
        nb = (L + BS - 1) // BS
        bt[i, :nb] = torch.tensor([perm.pop() for _ in range(nb)], dtype=torch.int32)
    scale = D ** -0.5
    out, lse = _run_paged(ops, q, kc, vc, bt, lens, scale)
    _compare(q, kc, vc, bt, lens, scale, out, lse)


def _nhd_cache(C, BS, KVH, D, dtype, g):
    """vLLM's physical layout [B, BS, KVH, 2D] and its K/V views [B, KVH, BS, D]."""
    phys = torch.randn(C, BS, KVH, 2 * D, generator=g).to(dtype)
    k = phys[..., :D].permute(0, 2, 1, 3)
    v = phys[..., D:].permute(0, 2, 1, 3)
    return phys, k, v


@pytest.mark.parametrize("dtype,H,KVH", [(torch.float16, 8, 8), (torch.bfloat16, 16, 4)])
def test_decode_tiered_two_tiers(ops, dtype, H, KVH):
    """HBM tier in vLLM's NHD layout + pinned host tier [C,KVH,BS,D]; each row's
    block list mixes both tiers (prefix HBM, suffix host, and interleaved)."""
    from vllm_fastdecoder_b200.gpu_ops import KVTier

    g = torch.Generator().manual_seed(3)
    D, BS, G_blocks, C_blocks = 128, 16, 40, 60
    n = 6
    phys, k0, v0 = _nhd_cache(G_blocks, BS, KVH, D, dtype, g)
    k1 = torch.randn(C_blocks, KVH, BS, D, generator=g).to(dtype)
    v1 = torch.randn(C_blocks, KVH, BS, D, generator=g).to(dtype)
    lens = torch.tensor([1, 16, 17, 300, 0, 555], dtype=torch.int32)
    W = 40
    bt = torch.zeros(n, W, dtype=torch.int32)
    perm_g = torch.randperm(G_blocks, generator=g).tolist()
    perm_c = torch.randperm(C_blocks, generator=g).tolist()
    for i in range(n):
        nb = (int(lens[i]) + BS - 1) // BS
        ids = []
        for j in range(nb):
            use_host = (i % 2 == 0 and j >= nb // 2) or (i % 2 == 1 and j % 3 == 1)
            ids.append(G_blocks + perm_c.pop() if use_host and perm_c else perm_g.pop())
        bt[i, :nb] = torch.tensor(ids, dtype=torch.int32)
        bt[i, nb:] = torch.randint(0, G_blocks + C_blocks, (W - nb,), generator=g)  # junk past the end
    q = torch.randn(n, H, D, generator=g).to(dtype)
    scale = D ** -0.5

    dev = torch.device("cuda")
    phys_d = phys.to(dev)
    tiers = (KVTier(phys_d[..., :D].permute(0, 2, 1, 3), phys_d[..., D:].permute(0, 2, 1, 3)),
             KVTier(k1.pin_memory(), v1.pin_memory()))
    out = torch.full((n, H, D), float("nan"), dtype=dtype, device=dev)
    lse = torch.full((H, n), float("nan"), device=dev)
    ops.decode_tiered(q.to(dev), tiers, G_blocks, bt.to(dev), lens.to(dev), scale, out, lse)
    ops.check_device_errors(dev)

    o_or = torch.empty_like(q)
    l_or = torch.empty(H, n)
    O.decode_attn_tiered(q, (k0, v0), (k1, v1), G_blocks, bt, lens, scale, o_or, l_or)
    nz = lens > 0
    t = TOL_ORACLE[dtype]
    torch.testing.assert_close(out.cpu()[nz].float(), o_or[nz].float(), atol=t, rtol=t)
    assert (lse.cpu()[:, nz] - l_or[:, nz]).abs().max().item() <= LSE_TOL
    assert torch.all(out.cpu()[~nz] == 0) and torch.all(torch.isneginf(lse.cpu()[:, ~nz]))


def test_decode_fp32_partials_and_row_maps(ops):
    """fp32 output mode plus q_rows / out_rows gather-scatter."""
    from vllm_fastdecoder_b200.gpu_ops import KVTier

    dev = torch.device("cuda")
    n, H, KVH, D, BS, C = 4, 8, 2, 128, 16, 32
    q, kc, vc, bt, lens = O.rand_case(n, H, KVH, D, BS, C, torch.bfloat16, max_len=200, seed=9)
    T = 10
    q_rows = torch.tensor([7, 2, 9, 0], dtype=torch.int64)
    big_q = torch.randn(T, H, D).to(torch.bfloat16)
    big_q[q_rows] = q
    out_rows = torch.tensor([3, 8, 1, 5], dtype=torch.int64)
    out = torch.zeros(T, H, D, dtype=torch.float32, device=dev)
    ops.decode_tiered(big_q.to(dev), (KVTier(kc.to(dev), vc.to(dev)), None), 1 << 40, bt.to(dev),
                      lens.to(dev), D ** -0.5, out, None, q_rows=q_rows.to(dev), out_rows=out_rows.to(dev))
    ops.check_device_errors(dev)
    o_or = torch.empty(n, H, D, dtype=torch.float32)
    O.decode_attn_tiered(q, (kc, vc), None, 1 << 40, bt, lens, D ** -0.5, o_or, None)
    got = out.cpu()
    # fp32 output of 16-bit inputs: only the fp32 accumulation order differs
    torch.testing.assert_close(got[out_rows], o_or, atol=1e-5, rtol=1e-5)
    untouched = torch.ones(T, dtype=torch.bool)
    untouched[out_rows] = False
    assert torch.all(got[untouched] == 0)


def test_row_maps_must_be_int64(ops):
    """q_rows / out_rows are read as int64 by the kernels: any other dtype is
    refused on the host, before a launch."""
    from vllm_fastdecoder_b200.gpu_ops import KVTier

    dev = torch.device("cuda")
    n, H, KVH, D, BS, C = 2, 8, 2, 128, 16, 8
    q, kc, vc, bt, lens = O.rand_case(n, H, KVH, D, BS, C, torch.bfloat16, max_len=40, seed=4)
    out = torch.zeros(n, H, D, dtype=torch.bfloat16, device=dev)
    tiers = (KVTier(kc.to(dev), vc.to(dev)), None)
    rows32 = torch.arange(n, dtype=torch.int32, device=dev)
    for kw in ({"q_rows": rows32}, {"out_rows": rows32}, {"q_rows": torch.arange(n)}):
        with pytest.raises(RuntimeError, match="int64"):
            ops.decode_tiered(q.to(dev), tiers, 1 << 40, bt.to(dev), lens.to(dev), D ** -0.5, out, None, **kw)
    torch.cuda.synchronize()


def test_decode_bad_block_id_sets_error(ops):
    """An out-of-range block id is reported through the error word (no fault)."""
    dev = torch.device("cuda")
    n, H, KVH, D, BS, C = 2, 4, 4, 64, 16, 8
    q, kc, vc, bt, lens = O.rand_case(n, H, KVH, D, BS, C, torch.float16, 40, 0)
    bt[0, 1] = C + 5
    out = torch.empty(n, H, D, dtype=torch.float16, device=dev)
    lse = torch.empty(H, n, device=dev)
    ops.decode_attn(q.to(dev), kc.to(dev), vc.to(dev), bt.to(dev), lens.to(dev), 0.125, out, lse)
    with pytest.raises(RuntimeError, match="block id"):
        ops.check_device_errors(dev)
    ops.check_device_errors(dev)  # cleared


@pytest.mark.parametrize("H,KVH", [(8, 8), (16, 4)])
def test_staged_host_tier_equals_mapped(ops, H, KVH):
    """The host tier staged into device memory by the copy engine
    (host_range) gives the same result as reading it in place: same kernel,
    same data (CUDA-core kernel for MHA, tcgen05 kernel for the group of 4)."""
    from vllm_fastdecoder_b200.gpu_ops import KVTier

    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(H)
    D, BS, G, C, n = 128, 16, 30, 50, 7
    dt = torch.bfloat16
    hk = torch.randn(G, KVH, BS, D, generator=g).to(dt).to(dev)
    hv = torch.randn(G, KVH, BS, D, generator=g).to(dt).to(dev)
    ck = torch.randn(C, KVH, BS, D, generator=g).to(dt).pin_memory()
    cv = torch.randn(C, KVH, BS, D, generator=g).to(dt).pin_memory()
    lens = torch.tensor([1, 90, 0, 300, 17, 64, 200], dtype=torch.int32)
    W = 20
    bt = torch.zeros(n, W, dtype=torch.int32)
    ids = torch.randperm(G - 1, generator=g).tolist()
    host = (torch.randperm(C - 10, generator=g) + 5).tolist()  # host ids 5..44: the range starts above 0
    for i in range(n):
        nb = (int(lens[i]) + BS - 1) // BS
        for j in range(nb):
            bt[i, j] = (host.pop() + G) if j % 3 else ids.pop()
    q = torch.randn(n, H, D, generator=g).to(dt).to(dev)
    tiers = (KVTier(hk, hv), KVTier(ck, cv))
    outs = []
    for hr in (None, ops.host_block_range(bt, lens, BS, G)):
        out = torch.full((n, H, D), float("nan"), dtype=dt, device=dev)
        lse = torch.empty(H, n, dtype=torch.float32, device=dev)
        ops.decode_tiered(q, tiers, G, bt.to(dev), lens.to(dev), D ** -0.5, out, lse, host_range=hr)
        ops.check_device_errors(dev)
        outs.append((out.cpu(), lse.cpu()))
    assert ops.host_block_range(bt, lens, BS, G)[0] >= 5
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])


@pytest.mark.parametrize("H,KVH", [(8, 8), (16, 4)])
@pytest.mark.parametrize("chunks", [1, 3, 8])
def test_staged_chunks_match_oracle(ops, H, KVH, chunks):
    """Host tier staged in chunks on a side stream, each chunk's blocks
    decoded into fp32 partials once its copy has landed, the HBM blocks
    first, then one P-way merge (decode_staged_chunks): matches the oracle
    over the whole two-tier rows (row maps on q and out, an empty row, rows
    with no host block, rows whose last partly filled block sits in any
    chunk), over two calls in a row on the same staging buffer."""
    from vllm_fastdecoder_b200.gpu_ops import KVTier

    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(7 * H + chunks)
    D, BS, G, C, n = 128, 16, 40, 80, 8
    dt = torch.bfloat16
    hk = torch.randn(G, KVH, BS, D, generator=g).to(dt)
    hv = torch.randn(G, KVH, BS, D, generator=g).to(dt)
    ck = torch.randn(C, KVH, BS, D, generator=g).to(dt).pin_memory()
    cv = torch.randn(C, KVH, BS, D, generator=g).to(dt).pin_memory()
    lens = torch.tensor([1, 90, 0, 300, 17, 64, 200, 33], dtype=torch.int32)
    W = 20
    bt = torch.zeros(n, W, dtype=torch.int32)
    ids = torch.randperm(G - 1, generator=g).tolist()
    host = (torch.randperm(C - 10, generator=g) + 5).tolist()
    for i in range(n):
        nb = (int(lens[i]) + BS - 1) // BS
        for j in range(nb):
            bt[i, j] = (host.pop() + G) if (j % 3 and i != 5) else ids.pop()  # row 5: HBM only
    T = n + 3
    q_rows = torch.randperm(T, generator=g)[:n]  # int64, as fd_decode_args reads them
    out_rows = torch.randperm(T, generator=g)[:n]
    qa = torch.randn(T, H, D, generator=g).to(dt)
    tiers = (KVTier(hk.to(dev), hv.to(dev)), KVTier(ck, cv))
    plan = ops.plan_chunked_staging(bt, lens, BS, G, chunks)
    assert len(plan.chunks) == min(chunks, plan.hi - plan.lo)
    ref = torch.empty(n, H, D, dtype=dt)
    ref_l = torch.empty(H, n)
    O.decode_attn_tiered(qa[q_rows], (hk, hv), (ck, cv), G, bt, lens, D ** -0.5, ref, ref_l)
    nz = lens > 0
    for _ in range(2):
        out = torch.full((T, H, D), float("nan"), dtype=dt, device=dev)
        lse = torch.full((H, n), float("nan"), dtype=torch.float32, device=dev)
        ops.decode_staged_chunks(qa.to(dev), tiers, D ** -0.5, out, lse, plan, q_rows=q_rows.to(dev),
                                 out_rows=out_rows.to(dev))
        ops.check_device_errors(dev)
        o = out.cpu()[out_rows]
        assert (o[nz].float() - ref[nz].float()).abs().max().item() <= TOL_ORACLE[dt]
        assert (lse.cpu()[:, nz] - ref_l[:, nz]).abs().max().item() <= LSE_TOL
        assert torch.all(o[~nz] == 0) and torch.all(torch.isneginf(lse.cpu()[:, ~nz]))


@pytest.mark.parametrize("vtiles", ["0", "1", "12", "40"])
@pytest.mark.parametrize("H,KVH,mma", [(8, 2, "1"), (8, 2, "0"), (8, 8, "1")])
def test_decode_weighted_schedule(ops, monkeypatch, vtiles, H, KVH, mma):
    """The persistent schedule with any per-segment weight (weight positions
    carry no work; a CTA whose range opens or ends among them must still
    write, and the combine read, the right partial slots), on both kernels
    (query group 4 takes the tensor cores unless disabled; MHA the CUDA
    cores), with ragged rows so ranges cut segments everywhere."""
    import random

    monkeypatch.setenv("FASTDECODE_B200_VTILES", vtiles)
    monkeypatch.setenv("FASTDECODE_B200_MMA", mma)
    rng = random.Random(int(vtiles) * 7 + H + KVH)
    n, D, BS = 29, 128, 16
    lens_l = [rng.choice([0, 1, 16, 17, 130, rng.randint(1, 2500)]) for _ in range(n)]
    C = sum((x + BS - 1) // BS for x in lens_l) + 8
    q, kc, vc, bt, lens = O.rand_case(n, H, KVH, D, BS, C, torch.bfloat16, max_len=max(lens_l), seed=n)
    lens = torch.tensor(lens_l, dtype=torch.int32)
    perm = torch.randperm(C, generator=torch.Generator().manual_seed(int(vtiles))).tolist()
    bt = torch.zeros(n, bt.shape[1], dtype=torch.int32)
    for i, L in enumerate(lens_l):
        nb = (L + BS - 1) // BS
        bt[i, :nb] = torch.tensor([perm.pop() for _ in range(nb)], dtype=torch.int32)
    scale = D ** -0.5
    out, lse = _run_paged(ops, q, kc, vc, bt, lens, scale)
    _compare(q, kc, vc, bt, lens, scale, out, lse)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("H,KVH", [(32, 8), (16, 8), (64, 8)])
def test_decode_tensor_core_path_matches_cuda_core_path(ops, monkeypatch, dtype, H, KVH):
    """The tcgen05 GQA kernel (query groups 2, 4, 8; head size 128) and the
    CUDA-core kernel agree with each other and with the oracle, including rows
    whose last stage is partial and an empty row."""
    n, D, BS = 6, 128, 16
    lens_l = [1, 129, 0, 1000, 2049, 77]
    C = sum((x + BS - 1) // BS for x in lens_l) + 8
    q, kc, vc, bt, lens = O.rand_case(n, H, KVH, D, BS, C, dtype, max_len=max(lens_l), seed=H)
    lens = torch.tensor(lens_l, dtype=torch.int32)
    perm = torch.randperm(C, generator=torch.Generator().manual_seed(H + 1)).tolist()
    bt = torch.zeros(n, bt.shape[1], dtype=torch.int32)
    for i, L in enumerate(lens_l):
        nb = (L + BS - 1) // BS
        bt[i, :nb] = torch.tensor([perm.pop() for _ in range(nb)], dtype=torch.int32)
    scale = D ** -0.5
    out_tc, lse_tc = _run_paged(ops, q, kc, vc, bt, lens, scale)
    _compare(q, kc, vc, bt, lens, scale, out_tc, lse_tc)
    monkeypatch.setenv("FASTDECODE_B200_MMA", "0")
    out_cc, lse_cc = _run_paged(ops, q, kc, vc, bt, lens, scale)
    _compare(q, kc, vc, bt, lens, scale, out_cc, lse_cc)
    nz = lens > 0
    t = TOL_ORACLE[dtype]
    torch.testing.assert_close(out_tc[nz].float(), out_cc[nz].float(), atol=t, rtol=t)
    assert (lse_tc[:, nz] - lse_cc[:, nz]).abs().max().item() <= LSE_TOL
