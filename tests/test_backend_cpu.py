"""FastDecodeImpl._forward_split on the CPU with the device primitives swapped
for oracle-backed stand-ins (the reference's own testing approach,
tests/test_plan_and_forward.py:48-114): block routing, the tier-aware KV write,
row gather/scatter, both split modes (one pass / two partials + merge) and the
prefill hand-off run exactly as on the GPU and are checked against
  * the reference's own _forward_split output on the same inputs
    (tests/golden/forward_split.npz), and
  * float64 attention over one unified KV cache,
and both tiers must afterwards hold exactly the reference's caches."""

from __future__ import annotations

import hashlib
import math
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import oracle as O
from vllm_fastdecoder_b200 import backend, config, plan, state

GOLD = Path(__file__).resolve().parent / "golden"
BS = 4


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def attend(q, k, v, scale, causal):
    """float64 attention; q [Lq,H,D], k/v [Lk,KVH,D] -> [Lq,H,D]."""
    H, KVH = q.shape[1], k.shape[1]
    G = H // KVH
    k = k.double().repeat_interleave(G, dim=1)
    v = v.double().repeat_interleave(G, dim=1)
    s = torch.einsum("qhd,khd->hqk", q.double(), k) * scale
    if causal:
        Lq, Lk = q.shape[0], k.shape[0]
        qi = torch.arange(Lq)[:, None] + (Lk - Lq)
        s = s.masked_fill((torch.arange(Lk)[None, :] > qi)[None], float("-inf"))
    return torch.einsum("hqk,khd->qhd", torch.softmax(s, dim=-1), v)


class OracleOps:
    """CPU stand-ins of the device primitives, computing with the oracle."""

    @staticmethod
    def tier(k, v):
        return (k, v)

    @staticmethod
    def store_kv(key, value, slots, tiers, tier_split):
        bs = tiers[0][0].shape[2]
        for j, s in enumerate(slots.tolist()):
            if s < 0:
                continue
            b, off = divmod(s, bs)
            t = 0 if b < tier_split else 1
            if t:
                b -= tier_split
            k, v = tiers[t]
            k[b, :, off] = key[j]
            v[b, :, off] = value[j]

    @staticmethod
    def decode(query, tiers, tier_split, block_table, lens, scale, out, lse=None, q_rows=None, out_rows=None,
               **_):
        n = block_table.shape[0]
        q = (query[q_rows] if q_rows is not None else query[:n]).contiguous()
        H, D = q.shape[1], q.shape[2]
        o = torch.empty(n, H, D, dtype=out.dtype)
        tmp_lse = torch.empty(H, n)
        O.decode_attn_tiered(q, tiers[0], tiers[1], tier_split, block_table.contiguous(), lens.contiguous(),
                             scale, o, tmp_lse)
        if out_rows is not None:
            out[out_rows] = o
        else:
            out[:n] = o
        if lse is not None:
            lse.copy_(tmp_lse)

    @staticmethod
    def merge(out, o_a, lse_a, o_b, lse_b, out_rows=None):
        m = O.merge2(o_a, lse_a, o_b, lse_b).to(out.dtype)
        if out_rows is not None:
            out[out_rows] = m
        else:
            out[: m.shape[0]] = m

    @staticmethod
    def fa(q, k, v, cu_seqlens_q, max_seqlen_q, max_seqlen_k, softmax_scale, causal, cu_seqlens_k=None,
           seqused_k=None, block_table=None, **_):
        outs = []
        for b in range(cu_seqlens_q.numel() - 1):
            q0, q1 = int(cu_seqlens_q[b]), int(cu_seqlens_q[b + 1])
            if block_table is not None:
                L = int(seqused_k[b])
                bs = k.shape[1]
                blks = block_table[b, : (L + bs - 1) // bs].long()
                kk = k[blks].reshape(-1, k.shape[2], k.shape[3])[:L]
                vv = v[blks].reshape(-1, v.shape[2], v.shape[3])[:L]
            else:
                k0, k1 = int(cu_seqlens_k[b]), int(cu_seqlens_k[b + 1])
                kk, vv = k[k0:k1], v[k0:k1]
            outs.append(attend(q[q0:q1], kk, vv, softmax_scale, causal))
        return torch.cat(outs).to(q.dtype)


    @staticmethod
    def prefill(query, out, q_start, q_len, k_len, scale, kv=None, block_table=None, k=None, v=None, total_q=None):
        """fd_prefill_attn's contract: request r's queries are rows q_start[r]
        .. + q_len[r] - 1, its k_len[r] keys from the paged tier (kv views
        [B, KVH, BS, D], table row r) or the batch rows q_start[r] + j."""
        assert total_q is None or total_q >= int(q_len.sum())
        for r in range(q_len.numel()):
            qs, ql, kl = int(q_start[r]), int(q_len[r]), int(k_len[r])
            if block_table is not None:
                bs = kv[0].shape[2]
                blks = block_table[r, : (kl + bs - 1) // bs].long()
                kk = kv[0][blks].transpose(1, 2).reshape(-1, kv[0].shape[1], kv[0].shape[3])[:kl]
                vv = kv[1][blks].transpose(1, 2).reshape(-1, kv[1].shape[1], kv[1].shape[3])[:kl]
            else:
                kk, vv = k[qs: qs + kl], v[qs: qs + kl]
            out[qs: qs + ql] = attend(query[qs: qs + ql], kk, vv, scale, causal=True).to(out.dtype)


@pytest.fixture(autouse=True)
def _cpu_ops(monkeypatch):
    monkeypatch.setattr(backend, "OPS", OracleOps)
    yield
    state.STORE = None


# the reference's planner/forward scenario (tests/test_plan_and_forward.py:123-196)
REQS = [
    (8, 1, [1, 2, 12]),
    (4, 1, [3, 4]),
    (0, 6, [13, 5]),
    (0, 3, [6]),
    (3, 1, [15]),
    (11, 1, [16, 7, 17]),
    (0, 1, [18]),
]


def scenario(reqs, G, C, H, KVH, D, dtype, seed):
    """Inputs built with the same generator calls as the reference scenario
    (pinned below by the input checksums the reference recorded)."""
    g = torch.Generator().manual_seed(seed)
    uk = torch.randn(G + C, BS, KVH, D, generator=g).to(dtype)
    uv = torch.randn(G + C, BS, KVH, D, generator=g).to(dtype)
    n_tok = sum(r[1] for r in reqs)
    query = torch.randn(n_tok, H, D, generator=g).to(dtype)
    key = torch.randn(n_tok, KVH, D, generator=g).to(dtype)
    value = torch.randn(n_tok, KVH, D, generator=g).to(dtype)
    qsl, seq, slots = [0], [], []
    W = max(len(r[2]) for r in reqs)
    bt = torch.zeros(len(reqs), W, dtype=torch.int32)
    for i, (ctx, ql, blocks) in enumerate(reqs):
        L = ctx + ql
        bt[i, : len(blocks)] = torch.tensor(blocks, dtype=torch.int32)
        slots += [blocks[p // BS] * BS + p % BS for p in range(ctx, L)]
        qsl.append(qsl[-1] + ql)
        seq.append(L)
    qsl = torch.tensor(qsl, dtype=torch.int32)
    seq = torch.tensor(seq, dtype=torch.int32)
    slots = torch.tensor(slots, dtype=torch.int64)
    rk, rv = uk.clone(), uv.clone()
    for t, s in enumerate(slots.tolist()):
        rk[s // BS, s % BS] = key[t]
        rv[s // BS, s % BS] = value[t]
    scale = 1.0 / math.sqrt(D)
    ref = torch.zeros(n_tok, H, D, dtype=torch.float64)
    for i, (ctx, ql, blocks) in enumerate(reqs):
        L = ctx + ql
        kk = rk[torch.tensor(blocks)].reshape(-1, KVH, D)[:L]
        vv = rv[torch.tensor(blocks)].reshape(-1, KVH, D)[:L]
        ref[qsl[i]: qsl[i + 1]] = attend(query[qsl[i]: qsl[i + 1]], kk, vv, scale, causal=True)
    kv_cache = torch.zeros(G, KVH, BS, 2 * D, dtype=dtype)  # vLLM logical [B, KVH, BS, 2D]
    kv_cache[..., :D] = uk[:G].transpose(1, 2)
    kv_cache[..., D:] = uv[:G].transpose(1, 2)
    cpu_k = uk[G:].transpose(1, 2).contiguous()
    cpu_v = uv[G:].transpose(1, 2).contiguous()
    return SimpleNamespace(query=query, key=key, value=value, qsl=qsl, seq_lens=seq, bt=bt, slots=slots,
                           kv_cache=kv_cache, cpu_k=cpu_k, cpu_v=cpu_v, ref=ref, ref_k=rk, ref_v=rv, scale=scale)


def make_impl(H, KVH, D, scale):
    impl = backend.FastDecodeImpl.__new__(backend.FastDecodeImpl)
    impl.num_heads, impl.num_kv_heads, impl.head_size = H, KVH, D
    impl.scale = scale
    impl.logits_soft_cap = 0
    impl.vllm_flash_attn_version = 2
    impl.kv_cache_dtype = "auto"
    impl.kv_sharing_target_layer_name = None
    return impl


def run_forward(sc, G, C, H, KVH, D, dtype):
    hp = plan.build_host_plan(sc.qsl, sc.seq_lens, sc.bt, sc.slots, G, C, BS)
    dp = plan.to_device(hp, sc.bt, "cpu")
    state.STORE = state.CpuKVStore(num_gpu_blocks=G, num_cpu_blocks=C, block_size=BS, num_kv_heads=KVH,
                                   head_size=D, dtype=dtype, k={"l0": sc.cpu_k}, v={"l0": sc.cpu_v})
    impl = make_impl(H, KVH, D, sc.scale)
    layer = SimpleNamespace(layer_name="l0", _k_scale=None, _v_scale=None)
    output = torch.full_like(sc.query, float("nan"))
    impl._forward_split(layer, sc.query, sc.key, sc.value, sc.kv_cache, dp, output)
    return output


@pytest.mark.parametrize("two_pass", [False, True])
@pytest.mark.parametrize("H,KVH", [(4, 4), (8, 2)])
@pytest.mark.parametrize("dname", ["float32", "float16"])
@pytest.mark.parametrize("seed", [0, 1])
def test_forward_split_matches_reference(monkeypatch, two_pass, H, KVH, dname, seed):
    if two_pass:
        monkeypatch.setenv(config.ENV_TWO_PASS, "1")
    gold = np.load(GOLD / "forward_split.npz")
    dtype = {"float32": torch.float32, "float16": torch.float16}[dname]
    G, C, D = 10, 20, 64
    sc = scenario(REQS, G, C, H, KVH, D, dtype, seed)
    key = f"H{H}_KVH{KVH}_{dname}_s{seed}"
    assert [sha(t) for t in (sc.query, sc.key, sc.value, sc.kv_cache, sc.cpu_k, sc.cpu_v)] == \
        list(gold[key + "/sha_inputs"])
    output = run_forward(sc, G, C, H, KVH, D, dtype)
    tol = 1e-5 if dtype == torch.float32 else 3e-3
    torch.testing.assert_close(output.double(), sc.ref, atol=tol, rtol=tol)
    ref_out = torch.from_numpy(gold[key + "/output"])
    torch.testing.assert_close(output.double(), ref_out.double(), atol=tol, rtol=tol)
    torch.testing.assert_close(torch.from_numpy(gold[key + "/ref_f64"]), sc.ref, atol=0, rtol=0)
    # both tiers hold exactly what the reference left in them
    assert [sha(sc.kv_cache), sha(sc.cpu_k), sha(sc.cpu_v)] == list(gold[key + "/sha_after"])


@pytest.mark.parametrize("H,KVH", [(4, 4), (8, 2)])
def test_forward_split_prefill_rows_on_the_b200_kernel(monkeypatch, H, KVH):
    """The P and F prefill rows routed to fd_prefill_attn (here its CPU
    stand-in) with the per-request query starts, query and key counts and
    table rows the backend derives from the plan: the output equals the
    reference's recorded forward (FlashAttention for those rows)."""
    monkeypatch.setattr(backend.FastDecodeImpl, "_prefill_on_b200", lambda self, q: True)
    gold = np.load(GOLD / "forward_split.npz")
    dtype, G, C, D, seed = torch.float16, 10, 20, 64, 0
    sc = scenario(REQS, G, C, H, KVH, D, dtype, seed)
    key = f"H{H}_KVH{KVH}_float16_s{seed}"
    output = run_forward(sc, G, C, H, KVH, D, dtype)
    torch.testing.assert_close(output.double(), sc.ref, atol=3e-3, rtol=3e-3)
    torch.testing.assert_close(output.double(), torch.from_numpy(gold[key + "/output"]).double(), atol=3e-3, rtol=3e-3)


def test_prefill_eligibility():
    impl = make_impl(8, 2, 128, 0.1)
    assert impl._prefill_on_b200(torch.empty(1, 8, 128, dtype=torch.bfloat16))
    assert not impl._prefill_on_b200(torch.empty(1, 8, 128, dtype=torch.float32))
    impl.head_size = 64
    assert not impl._prefill_on_b200(torch.empty(1, 8, 64, dtype=torch.float16))


def test_forward_none_metadata_zero_fills():
    impl = make_impl(4, 4, 16, 0.25)
    out = torch.ones(3, 4, 16)
    assert impl.forward(None, None, None, None, None, None, out) is out
    assert torch.all(out == 0)


def test_backend_class_surface():
    B = backend.FastDecodeBackend
    assert B.get_name() == "CUSTOM"
    assert B.forward_includes_kv_cache_update is True
    assert B.supported_kv_cache_dtypes == ["auto", "float16", "bfloat16"]
    assert B.get_impl_cls() is backend.FastDecodeImpl
    assert B.get_builder_cls() is backend.FastDecodeMetadataBuilder
    assert not B.supports_sliding_window() and not B.supports_sink()
    assert backend.FastDecodeMetadataBuilder._cudagraph_support == backend.AttentionCGSupport.NEVER
