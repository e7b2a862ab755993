"""GPU parity of the tensor-core prefill kernel (fd_prefill_attn through the C
ABI), the replacement of FlashAttention's causal varlen call for the P and F
classes (fastdecode/backend.py:317-340), against a float64 restatement of
causal attention with FlashAttention's bottom-right alignment: query i of a
request with q_len queries and k_len keys sees keys 0 .. k_len - q_len + i.

Tolerances (written here): output vs float64 fp16 2e-3, bf16 1.6e-2 (the
reference's own bounds for the decode, tests/test_cpu_kernel.py:53; P is
rounded to the input type before P.V, as in FlashAttention).  Rows of `out`
that belong to no request stay untouched."""

from __future__ import annotations

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 2e-3, torch.bfloat16: 1.6e-2}


def _ref(q, keys, vals, q_start, q_len, k_len, scale, G):
    """float64 causal attention per request; keys[r] / vals[r]: [k_len, KVH, D]."""
    out = {}
    for r in range(len(q_len)):
        qs, ql, kl = int(q_start[r]), int(q_len[r]), int(k_len[r])
        qr = q[qs:qs + ql].double()                      # [ql, H, D]
        K = keys[r].double().repeat_interleave(G, dim=1)  # [kl, H, D]
        V = vals[r].double().repeat_interleave(G, dim=1)
        s = torch.einsum("qhd,khd->hqk", qr, K) * scale
        i = torch.arange(ql).unsqueeze(1)
        j = torch.arange(kl).unsqueeze(0)
        s = s.masked_fill(~(j <= kl - ql + i), float("-inf"))
        out[r] = torch.einsum("hqk,khd->qhd", torch.softmax(s, dim=-1), V)
    return out


def _check(out, ref, q_start, q_len, dtype, T):
    covered = torch.zeros(T, dtype=torch.bool)
    for r, o in ref.items():
        qs, ql = int(q_start[r]), int(q_len[r])
        covered[qs:qs + ql] = True
        if ql == 0:
            continue
        err = (out[qs:qs + ql].double() - o).abs().max().item()
        assert err <= TOL[dtype], (r, err)
    assert torch.isnan(out[~covered].float()).all()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("H,KVH", [(8, 2), (4, 4), (16, 2)])
def test_prefill_paged_matches_reference(dtype, H, KVH):
    """P class: queries over a cached context in the paged HBM tier (vLLM's
    NHD layout), tiles cut across and inside requests, a one-token request,
    a request whose queries start mid-tile of the batch; query groups 4, 1
    and 8 (a tile holds 128 / G query tokens of all G heads of a kv head)."""
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(11 + H)
    D, BS = 128, 16
    q_len = [130, 1, 257, 64]
    k_len = [130 + 64, 40, 257 + 500, 64]
    W = max((k + BS - 1) // BS for k in k_len) + 2
    pool = sum((k + BS - 1) // BS for k in k_len) + 9
    phys = torch.randn(pool, BS, KVH, 2 * D, generator=g).to(dtype)  # [B, BS, KVH, 2D]
    perm = torch.randperm(pool, generator=g).tolist()
    bt = torch.zeros(len(q_len), W, dtype=torch.int32)
    for r, kl in enumerate(k_len):
        nb = (kl + BS - 1) // BS
        bt[r, :nb] = torch.tensor([perm.pop() for _ in range(nb)], dtype=torch.int32)
    q_start, pos = [], 3  # three leading rows belong to no request
    for ql in q_len:
        q_start.append(pos)
        pos += ql
    T = pos + 2
    q = torch.randn(T, H, D, generator=g).to(dtype)
    scale = 1.0 / math.sqrt(D)
    keys = [phys[bt[r, :(kl + BS - 1) // BS].long()].reshape(-1, KVH, 2 * D)[:kl, :, :D] for r, kl in enumerate(k_len)]
    vals = [phys[bt[r, :(kl + BS - 1) // BS].long()].reshape(-1, KVH, 2 * D)[:kl, :, D:] for r, kl in enumerate(k_len)]
    ref = _ref(q, keys, vals, q_start, q_len, k_len, scale, H // KVH)

    from vllm_fastdecoder_b200 import gpu_ops
    from vllm_fastdecoder_b200.gpu_ops import KVTier

    pd = phys.to(dev)
    cache = pd.permute(0, 2, 1, 3)  # logical [B, KVH, BS, 2D]
    kv = KVTier(cache[..., :D], cache[..., D:])
    i32 = lambda x: torch.tensor(x, dtype=torch.int32, device=dev)  # noqa: E731
    for _ in range(2):
        out = torch.full((T, H, D), float("nan"), dtype=dtype, device=dev)
        gpu_ops.prefill_attn(q.to(dev), out, i32(q_start), i32(q_len), i32(k_len), scale, kv=kv,
                             block_table=bt.to(dev))
        gpu_ops.check_device_errors(dev)
        _check(out.cpu(), ref, q_start, q_len, dtype, T)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_prefill_fresh_rows_match_reference(dtype):
    """F class: fresh prefills attend over the batch's own new K/V rows
    (k_len = q_len), as flash_attn_varlen_func(q, k, v, cu_seqlens, causal)."""
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(5)
    H, KVH, D = 8, 4, 128
    q_len = [200, 17, 128, 1]
    q_start, pos = [], 0
    for ql in q_len:
        q_start.append(pos)
        pos += ql
    T = pos
    q = torch.randn(T, H, D, generator=g).to(dtype)
    k = torch.randn(T, KVH, D, generator=g).to(dtype)
    v = torch.randn(T, KVH, D, generator=g).to(dtype)
    scale = 0.1
    keys = [k[s:s + ql] for s, ql in zip(q_start, q_len)]
    vals = [v[s:s + ql] for s, ql in zip(q_start, q_len)]
    ref = _ref(q, keys, vals, q_start, q_len, q_len, scale, H // KVH)

    from vllm_fastdecoder_b200 import gpu_ops

    i32 = lambda x: torch.tensor(x, dtype=torch.int32, device=dev)  # noqa: E731
    out = torch.full((T, H, D), float("nan"), dtype=dtype, device=dev)
    gpu_ops.prefill_attn(q.to(dev), out, i32(q_start), i32(q_len), i32(q_len), scale, k=k.to(dev), v=v.to(dev))
    gpu_ops.check_device_errors(dev)
    _check(out.cpu(), ref, q_start, q_len, dtype, T)


@pytest.mark.parametrize("n", [200, 300])
def test_prefill_many_requests(n):
    """Hundreds of ragged fresh prefills, some of them empty: the scan that
    maps a CTA to its request and tile pair must cover every query row
    exactly once, past the first 32-request chunk of the scan."""
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(40 + n)
    H, KVH, D = 8, 2, 128
    q_len = torch.randint(0, 70, (n,), generator=g).tolist()
    q_start, pos = [], 0
    for ql in q_len:
        q_start.append(pos)
        pos += ql
    T = pos
    dtype = torch.bfloat16
    q = torch.randn(T, H, D, generator=g).to(dtype)
    k = torch.randn(T, KVH, D, generator=g).to(dtype)
    v = torch.randn(T, KVH, D, generator=g).to(dtype)
    scale = 1.0 / math.sqrt(D)
    keys = [k[s:s + ql] for s, ql in zip(q_start, q_len)]
    vals = [v[s:s + ql] for s, ql in zip(q_start, q_len)]
    ref = _ref(q, keys, vals, q_start, q_len, q_len, scale, H // KVH)

    from vllm_fastdecoder_b200 import gpu_ops

    i32 = lambda x: torch.tensor(x, dtype=torch.int32, device=dev)  # noqa: E731
    out = torch.full((T, H, D), float("nan"), dtype=dtype, device=dev)
    gpu_ops.prefill_attn(q.to(dev), out, i32(q_start), i32(q_len), i32(q_len), scale, k=k.to(dev), v=v.to(dev))
    gpu_ops.check_device_errors(dev)
    _check(out.cpu(), ref, q_start, q_len, dtype, T)


def test_prefill_rejects_bad_arguments_before_launch():
    from vllm_fastdecoder_b200 import gpu_ops

    dev = torch.device("cuda")
    q = torch.zeros(4, 2, 64, dtype=torch.bfloat16, device=dev)  # head size 64: not covered
    one = torch.ones(1, dtype=torch.int32, device=dev)
    with pytest.raises(RuntimeError, match="head_size"):
        gpu_ops.prefill_attn(q, torch.empty_like(q), one * 0, one, one, 1.0, k=q, v=q)
    q = torch.zeros(4, 2, 128, dtype=torch.bfloat16, device=dev)
    with pytest.raises(RuntimeError, match="int32"):
        gpu_ops.prefill_attn(q, torch.empty_like(q), one.long(), one, one, 1.0, k=q, v=q)
