"""GPU parity at the benchmark configurations' full sizes.

Each test decodes one configuration exactly as workloads.py builds it (the
shapes, lengths, tiers and seeds the bench times) through the C ABI and
compares every output row (or, for the 131072-token contexts, three whole
(row, kv head) slices) with the C oracle, the restatement of the reference
decode_attn (fastdecode/csrc/cpu_attn.cpp:298-411) that the golden vectors
pin; the oracle runs on all host cores, one row per call.  The reference's
own bounds (tests/test_cpu_kernel.py:53-55): fp16 output 2e-3, bf16 1.6e-2,
lse 1e-4 absolute; KV writes bit-exact.

  c0  16 rows, one 4096-block fp16 pool (CUDA-core kernel)
  c1  64 rows over the 2048-block HBM tier and the pinned host tier, read in
      place over PCIe, staged into HBM by the copy engine, and staged in
      chunks on a side stream with the decode overlapping the copies
  c2  256 GQA bf16 rows, lognormal lengths (tensor-core kernel)
  c3  8 rows x 131072 tokens on one GPU, and the same context cut into four
      shards (decoded separately on this GPU into fp32 partials and merged by
      fd_merge_partials, the sharded path's merge)
  c4  two continuous-batching trace steps through the plugin
      (FastDecodeImpl._forward_split over 32 layers, host planner)
"""

from __future__ import annotations

import math
from types import SimpleNamespace

import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL_O = {torch.float16: 2e-3, torch.bfloat16: 1.6e-2}
TOL_LSE = 1e-4


def _cpu_tier(t):
    return None if t is None else ((t.k.cpu(), t.v.cpu()) if not t.host else (t.k, t.v))


def _check(out, lse, ref, ref_l, lens, dtype):
    live = lens > 0
    err_o = (out.cpu().float() - ref.float()).abs().max().item()
    err_l = (lse.cpu()[:, live] - ref_l[:, live]).abs().max().item() if bool(live.any()) else 0.0
    assert err_o <= TOL_O[dtype], err_o
    assert err_l <= TOL_LSE, err_l
    assert torch.all(out.cpu()[~live] == 0)
    return err_o, err_l


def _decode_and_check(batch, res, dev, host_range=None, chunks=0):
    from vllm_fastdecoder_b200 import gpu_ops

    n, H, D = batch.n, batch.H, batch.D
    out = torch.full((n, H, D), float("nan"), dtype=batch.dtype, device=dev)
    lse = torch.full((H, n), float("nan"), dtype=torch.float32, device=dev)
    if chunks:
        plan = gpu_ops.plan_chunked_staging(batch.block_table, batch.lens, batch.BS, batch.G, chunks)
        gpu_ops.decode_staged_chunks(res.q, res.tiers, batch.scale, out, lse, plan)
    else:
        gpu_ops.decode_tiered(res.q, res.tiers, batch.G, res.block_table, res.lens, batch.scale, out, lse,
                              max_len=int(batch.lens.max()), host_range=host_range)
    gpu_ops.check_device_errors(dev)
    ref = torch.empty(n, H, D, dtype=batch.dtype)
    ref_l = torch.empty(H, n)
    O.decode_attn_tiered(res.q.cpu(), _cpu_tier(res.tiers[0]), _cpu_tier(res.tiers[1]), batch.G, batch.block_table,
                         batch.lens, batch.scale, ref, ref_l, threads=O.host_threads())
    return _check(out, lse, ref, ref_l, batch.lens, batch.dtype)


def test_config0_full_size():
    from vllm_fastdecoder_b200 import workloads

    dev = torch.device("cuda")
    b = workloads.config0()
    assert (b.n, b.H, b.KVH, b.num_hbm_blocks) == (16, 32, 32, 4096)
    _decode_and_check(b, workloads.materialize(b, dev), dev)


def test_config1_full_size_mapped_and_staged():
    from vllm_fastdecoder_b200 import gpu_ops, workloads

    dev = torch.device("cuda")
    b = workloads.config1()
    hbm_b, host_b = b.kv_bytes()
    assert b.n == 64 and b.G == 2048 and host_b > 1.5e9 and hbm_b > 0.5e9
    res = workloads.materialize(b, dev)
    _decode_and_check(b, res, dev)  # host tier read in place over PCIe
    hr = gpu_ops.host_block_range(b.block_table, b.lens, b.BS, b.G)
    _decode_and_check(b, res, dev, host_range=hr)  # staged by the copy engine
    _decode_and_check(b, res, dev, chunks=8)  # staged in 8 chunks on a side stream, overlapping the decode


def test_config2_full_size():
    from vllm_fastdecoder_b200 import gpu_ops, workloads

    dev = torch.device("cuda")
    b = workloads.config2()
    assert b.n == 256 and b.KVH == 8 and b.dtype == torch.bfloat16
    assert gpu_ops.decode_kernel_name(b.dtype, b.D, b.H, b.KVH, b.BS, b.n) == "fd_decode_mma_kernel"
    _decode_and_check(b, workloads.materialize(b, dev), dev)


def _slice_kv(res, batch, r, h):
    """K and V of row r, kv head h over the row's whole table, in order."""
    BS, D = batch.BS, batch.D
    L = int(batch.lens[r])
    nb = (L + BS - 1) // BS
    ids = res.block_table[r, :nb].long()
    k = res.tiers[0].k[ids, h].reshape(nb * BS, D)[:L]
    v = res.tiers[0].v[ids, h].reshape(nb * BS, D)[:L]
    return k, v


def _oracle_slice(q_heads, k, v, BS, scale, dtype):
    """The oracle over one kv head's whole context: q_heads [G, D] (CPU),
    k / v [L, D] (any device)."""
    L, D = k.shape
    G = q_heads.shape[0]
    kc = k.cpu().contiguous().view(L // BS, 1, BS, D)
    vc = v.cpu().contiguous().view(L // BS, 1, BS, D)
    o = torch.empty(1, G, D, dtype=dtype)
    lse = torch.empty(G, 1)
    O.decode_attn(q_heads.view(1, G, D).contiguous(), kc, vc, torch.arange(L // BS, dtype=torch.int32).view(1, -1),
                  torch.tensor([L], dtype=torch.int32), scale, o, lse)
    return o[0], lse[:, 0]


SLICES = [(0, 0), (3, 5), (7, 7)]


def test_config3_full_context_one_gpu():
    from vllm_fastdecoder_b200 import gpu_ops, workloads

    dev = torch.device("cuda")
    b = workloads.config3(world=1)
    assert b.n == 8 and int(b.lens[0]) == 131072
    res = workloads.materialize(b, dev)
    out = torch.empty(b.n, b.H, b.D, dtype=b.dtype, device=dev)
    lse = torch.empty(b.H, b.n, dtype=torch.float32, device=dev)
    gpu_ops.decode_tiered(res.q, res.tiers, b.G, res.block_table, res.lens, b.scale, out, lse)
    gpu_ops.check_device_errors(dev)
    G = b.H // b.KVH
    for r, h in SLICES:
        k, v = _slice_kv(res, b, r, h)
        o_ref, l_ref = _oracle_slice(res.q[r, h * G:(h + 1) * G].cpu(), k, v, b.BS, b.scale, b.dtype)
        assert (out[r, h * G:(h + 1) * G].cpu().float() - o_ref.float()).abs().max().item() <= TOL_O[b.dtype]
        assert (lse[h * G:(h + 1) * G, r].cpu() - l_ref).abs().max().item() <= TOL_LSE


def test_config3_four_shards_merged_on_one_gpu():
    """The sharded path's arithmetic at full size: each of four shards of
    every row decoded into packed fp32 partials [o | lse] (the layout the
    exchange moves), merged by fd_merge_partials, compared with the oracle
    over the concatenated 131072 tokens."""
    from vllm_fastdecoder_b200 import gpu_ops, workloads

    dev = torch.device("cuda")
    world = 4
    n, H, D = 8, 32, 128
    stride = n * H * D + H * n
    parts = torch.empty(world, stride, dtype=torch.float32, device=dev)
    shards = []
    for rank in range(world):
        b = workloads.config3(world=world, rank=rank)
        res = workloads.materialize(b, dev)
        o_view = parts[rank, : n * H * D].view(n, H, D)
        l_view = parts[rank, n * H * D:].view(H, n)
        gpu_ops.decode_tiered(res.q, res.tiers, b.G, res.block_table, res.lens, b.scale, o_view, l_view)
        shards.append((b, res))
    final = torch.empty(n, H, D, dtype=torch.bfloat16, device=dev)
    final_lse = torch.empty(H, n, dtype=torch.float32, device=dev)
    gpu_ops.merge_partials(parts, world, n, H, D, final, final_lse)
    gpu_ops.check_device_errors(dev)
    b0, res0 = shards[0]
    G = H // b0.KVH
    for r, h in SLICES:
        kv = [_slice_kv(res, b, r, h) for b, res in shards]
        k = torch.cat([x[0] for x in kv])
        v = torch.cat([x[1] for x in kv])
        assert k.shape[0] == 131072
        o_ref, l_ref = _oracle_slice(res0.q[r, h * G:(h + 1) * G].cpu(), k, v, b0.BS, b0.scale, b0.dtype)
        assert (final[r, h * G:(h + 1) * G].cpu().float() - o_ref.float()).abs().max().item() <= TOL_O[b0.dtype]
        assert (final_lse[h * G:(h + 1) * G, r].cpu() - l_ref).abs().max().item() <= TOL_LSE


def test_config4_trace_steps_through_the_plugin():
    """Two steps of the config-4 trace (32 layers, ~128 running requests,
    most KV in the host tier) through FastDecodeImpl._forward_split with the
    host planner, as the bench's end-to-end leg runs them.  One physical
    cache per tier serves all layers, so after a step the cache holds the
    last layer's new tokens: the last layer's output is checked against the
    oracle on that state, the first layer's after its new tokens are written
    back, and every new K/V row must sit bit-exactly at its slot."""
    from vllm_fastdecoder_b200 import backend, gpu_ops, plan, state, workloads
    from vllm_fastdecoder_b200.gpu_ops import KVTier

    dev = torch.device("cuda")
    tr = workloads.trace4(seed=0, steps=2)
    L, H, KVH, D, BS, G, dt = tr.layers, tr.H, tr.KVH, tr.D, tr.BS, tr.G, tr.dtype
    gen = torch.Generator(device=dev).manual_seed(5)
    phys = torch.empty(G, BS, KVH, 2 * D, dtype=dt, device=dev).normal_(generator=gen)
    kv_cache = phys.permute(0, 2, 1, 3)
    hk = torch.empty(tr.host_blocks, KVH, BS, D, dtype=dt, pin_memory=True)
    hv = torch.empty(tr.host_blocks, KVH, BS, D, dtype=dt, pin_memory=True)
    for t in (hk, hv):
        t.copy_(torch.empty(t.shape, dtype=dt, device=dev).normal_(generator=gen))
    names = [f"model.layers.{l}.self_attn.attn" for l in range(L)]
    state.STORE = state.CpuKVStore(num_gpu_blocks=G, num_cpu_blocks=tr.host_blocks, block_size=BS,
                                   num_kv_heads=KVH, head_size=D, dtype=dt, k={nm: hk for nm in names},
                                   v={nm: hv for nm in names})
    impl = backend.FastDecodeImpl.__new__(backend.FastDecodeImpl)
    impl.num_heads, impl.num_kv_heads, impl.head_size = H, KVH, D
    impl.scale, impl.logits_soft_cap = tr.scale, 0.0
    impl.vllm_flash_attn_version = 2
    impl.kv_cache_dtype = "auto"
    impl.kv_sharing_target_layer_name = None
    layers = [SimpleNamespace(layer_name=nm, _k_scale=None, _v_scale=None) for nm in names]
    tiers = (KVTier(kv_cache[..., :D], kv_cache[..., D:]), KVTier(hk, hv))
    try:
        for k_step, st in enumerate(tr.steps[:2]):
            R = st.rows
            _, host_b = tr.batch(k_step).kv_bytes()
            assert host_b > 0.5e9  # most of the step's KV is in the host tier
            qkv = torch.empty(L, R, H + 2 * KVH, D, dtype=dt, device=dev).normal_(generator=gen)
            outs = torch.full((L, R, H, D), float("nan"), dtype=dt, device=dev)
            qsl = torch.arange(R + 1, dtype=torch.int32)
            hp = plan.build_host_plan(qsl, st.lens, st.block_table, st.slots, G, tr.host_blocks, BS)
            dp = plan.to_device(hp, st.block_table.to(dev), dev)
            for l in range(L):
                q, kk, vv = qkv[l].split([H, KVH, KVH], dim=1)
                impl._forward_split(layers[l], q, kk, vv, kv_cache, dp, outs[l])
            gpu_ops.check_device_errors(dev)
            for l in (L - 1, 0):
                q, kk, vv = qkv[l].split([H, KVH, KVH], dim=1)
                if l != L - 1:  # the cache as it was when layer l decoded
                    gpu_ops.store_kv_tiered(kk, vv, st.slots.to(dev), tiers, G)
                # every new row at its slot, in the tier that owns it
                for i in range(R):
                    s = int(st.slots[i])
                    blk, off = s // BS, s % BS
                    got_k = kv_cache[blk, :, off, :D] if blk < G else hk[blk - G, :, off].to(dev)
                    got_v = kv_cache[blk, :, off, D:] if blk < G else hv[blk - G, :, off].to(dev)
                    assert torch.equal(got_k, kk[i]) and torch.equal(got_v, vv[i]), (l, i)
                ref = torch.empty(R, H, D, dtype=dt)
                ref_l = torch.empty(H, R)
                O.decode_attn_tiered(q.cpu(), (kv_cache[..., :D].cpu(), kv_cache[..., D:].cpu()), (hk, hv), G,
                                     st.block_table, st.lens, tr.scale, ref, ref_l, threads=O.host_threads())
                err = (outs[l].cpu().float() - ref.float()).abs().max().item()
                assert err <= TOL_O[dt], (k_step, l, err)
    finally:
        state.STORE = None
