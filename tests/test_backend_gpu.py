"""The backend's split path on the GPU with the real kernels, driven by a
continuous-batching trace in the manner of the reference's GPU self-test
(scripts/gpu_selftest.py): requests arrive with random prompts, decode for a
random number of steps and free their blocks; blocks are handed out HBM-first
and reused LIFO, so block tables mix both tiers in every pattern; caches start
filled with large garbage and table rows carry junk past their end, so any
read of an unwritten slot or a stray table entry shows up.

Every step runs FastDecodeImpl._forward_split (tier-aware KV write + split-KV
decode through the C ABI) and is compared with fp32 attention over one unified
cache holding the same data; the new K/V must land bit-exactly in the tier
that owns each slot.  Prefill rows (P and F classes) run on this engine's
tcgen05 prefill kernel (fd_prefill_attn); one case switches it off
(FASTDECODE_B200_PREFILL=0), which sends them to a torch stand-in for
FlashAttention as in the reference.  Tolerances: fp16 output 2e-3 absolute,
bf16 1.6e-2 (the decode tests' bounds), relative to outputs of magnitude <= 1.
"""

from __future__ import annotations

import math
import random
from types import SimpleNamespace

import pytest
import torch

from vllm_fastdecoder_b200 import backend, config, plan, state

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 2e-3, torch.bfloat16: 1.6e-2}


def attend_fp32(q, k, v, scale, causal):
    H, KVH = q.shape[1], k.shape[1]
    k = k.float().repeat_interleave(H // KVH, dim=1)
    v = v.float().repeat_interleave(H // KVH, dim=1)
    s = torch.einsum("qhd,khd->hqk", q.float(), k) * scale
    if causal:
        Lq, Lk = q.shape[0], k.shape[0]
        qi = torch.arange(Lq, device=q.device)[:, None] + (Lk - Lq)
        s = s.masked_fill((torch.arange(Lk, device=q.device)[None, :] > qi)[None], float("-inf"))
    return torch.einsum("hqk,khd->qhd", s.softmax(-1), v)


def torch_fa(q, k, v, cu_seqlens_q, max_seqlen_q, max_seqlen_k, softmax_scale, causal, cu_seqlens_k=None,
             seqused_k=None, block_table=None, **_):
    """Stand-in for FlashAttention on the prefill rows (fp32 math)."""
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
        outs.append(attend_fp32(q[q0:q1], kk, vv, softmax_scale, causal))
    return torch.cat(outs).to(q.dtype)


class GpuOpsTorchPrefill(backend._GpuOps):
    fa = staticmethod(torch_fa)


@pytest.mark.parametrize("dtype,H,KVH,two_pass,device_plan,b200_prefill", [
    (torch.float16, 8, 8, False, False, True),
    (torch.bfloat16, 16, 4, False, False, True),
    (torch.float16, 8, 2, True, False, True),
    (torch.float16, 8, 8, False, True, True),
    (torch.bfloat16, 16, 4, False, True, True),
    (torch.bfloat16, 16, 4, False, False, False),
])
def test_continuous_batching_trace(monkeypatch, dtype, H, KVH, two_pass, device_plan, b200_prefill):
    """device_plan: decode-only steps are planned on the GPU (fd_plan_step)
    and run through FastDecodeImpl._forward_device, as the metadata builder
    does for them; steps with prefills take the host planner."""
    if two_pass:
        monkeypatch.setenv(config.ENV_TWO_PASS, "1")
    monkeypatch.setenv(config.ENV_PREFILL, "1" if b200_prefill else "0")
    monkeypatch.setattr(backend, "OPS", GpuOpsTorchPrefill)
    from vllm_fastdecoder_b200 import gpu_ops

    dev = torch.device("cuda")
    rng = random.Random(0)
    torch.manual_seed(0)
    G, C, BS, D = 40, 500, 16, 128
    scale = 1.0 / math.sqrt(D)
    steps, max_reqs, max_prompt, max_new = 30, 24, 300, 80
    name = "l0"
    # physical NHD HBM cache viewed as vLLM's logical [B, KVH, BS, 2D]
    phys = (torch.randn(G, BS, KVH, 2 * D, device=dev) * 10).to(dtype)
    kv_cache = phys.permute(0, 2, 1, 3)
    host_k = (torch.randn(C, KVH, BS, D) * 10).to(dtype).pin_memory()
    host_v = (torch.randn(C, KVH, BS, D) * 10).to(dtype).pin_memory()
    state.STORE = state.CpuKVStore(num_gpu_blocks=G, num_cpu_blocks=C, block_size=BS, num_kv_heads=KVH,
                                   head_size=D, dtype=dtype, k={name: host_k}, v={name: host_v})
    # the unified pool the reference attention reads (same data, one tier)
    uk = (torch.randn(G + C, KVH, BS, D, device=dev) * 10).to(dtype)
    uv = (torch.randn(G + C, KVH, BS, D, device=dev) * 10).to(dtype)

    impl = backend.FastDecodeImpl.__new__(backend.FastDecodeImpl)
    impl.num_heads, impl.num_kv_heads, impl.head_size = H, KVH, D
    impl.scale, impl.logits_soft_cap = scale, 0.0
    impl.vllm_flash_attn_version = 2
    impl.kv_cache_dtype = "auto"
    impl.kv_sharing_target_layer_name = None
    layer = SimpleNamespace(layer_name=name, _k_scale=None, _v_scale=None)

    free_gpu, free_cpu = list(range(1, G)), list(range(G, G + C))

    def alloc():
        if free_gpu:
            return free_gpu.pop(0)
        return free_cpu.pop(0) if free_cpu else None

    def release(blocks):
        free_gpu[:0] = [b for b in blocks if b < G]
        free_cpu.extend(b for b in blocks if b >= G)

    running, n_split, n_rows, n_dev = [], 0, 0, 0
    for step in range(steps):
        rows = []
        for r in list(running):
            if r["L"] % BS == 0:
                b = alloc()
                if b is None:
                    running.remove(r)
                    release(r["blocks"])
                    continue
                r["blocks"].append(b)
            rows.append((r, r["L"], 1))
        while len(running) < max_reqs:
            P = 1 if rng.random() < 0.05 else rng.randint(2, max_prompt)
            need = (P + BS - 1) // BS
            if need > len(free_gpu) + len(free_cpu) - 8:
                break
            r = {"blocks": [alloc() for _ in range(need)], "L": 0, "left": rng.randint(1, max_new)}
            running.append(r)
            rows.append((r, 0, P))
        if not rows:
            continue
        rng.shuffle(rows)
        R = len(rows)
        qlens = [ql for _, _, ql in rows]
        seqs = [ctx + ql for _, ctx, ql in rows]
        T = sum(qlens)
        W = max(len(r["blocks"]) for r, _, _ in rows) + 2
        bt = torch.zeros(R, W, dtype=torch.int32)
        slots = []
        for i, (r, ctx, ql) in enumerate(rows):
            bl = r["blocks"]
            bt[i, : len(bl)] = torch.tensor(bl, dtype=torch.int32)
            bt[i, len(bl):] = torch.randint(0, G + C, (W - len(bl),), dtype=torch.int32)  # junk
            slots += [bl[p // BS] * BS + p % BS for p in range(ctx, ctx + ql)]
        qsl = torch.zeros(R + 1, dtype=torch.int32)
        qsl[1:] = torch.cumsum(torch.tensor(qlens), 0)
        seq = torch.tensor(seqs, dtype=torch.int32)
        slots = torch.tensor(slots, dtype=torch.int64)
        Tp = T + rng.randint(0, 5)  # padding rows like a cudagraph batch
        qkv = torch.randn(Tp, (H + 2 * KVH) * D, device=dev).to(dtype)
        q, k, v = qkv.split([H * D, KVH * D, KVH * D], dim=-1)
        q = q.reshape(Tp, H, D)
        k = k.reshape(Tp, KVH, D)
        v = v.reshape(Tp, KVH, D)

        width = max(1, min((max(seqs) + BS - 1) // BS, W))
        decode_only = all(ql == 1 for ql in qlens)
        hp = None if (device_plan and decode_only) else plan.build_host_plan(qsl, seq, bt[:, :width], slots, G, C, BS)
        # the unified pool gets this step's K/V (the reference cache)
        sl = slots.to(dev)
        uk[sl // BS, :, sl % BS] = k[:T]
        uv[sl // BS, :, sl % BS] = v[:T]
        out = torch.full((Tp, H, D), float("nan"), dtype=dtype, device=dev)
        if device_plan and decode_only:
            dp = plan.plan_on_device(qsl.to(dev), seq.to(dev), bt[:, :width].to(dev).contiguous(), sl, G, C, BS)
            ds = plan.DeviceDecodeStep(dp, R, T, max(seqs))
            impl._forward_device(layer, q, k, v, kv_cache, ds, sl, out)
            gpu_ops.check_device_errors(dev)
            n_dev += 1
            continue_check = True
        elif hp is None:
            # an all-HBM step takes vLLM's stock path; only mirror its KV write
            kv_cache[sl // BS, :, sl % BS, :D] = k[:T]
            kv_cache[sl // BS, :, sl % BS, D:] = v[:T]
            continue_check = False
        else:
            n_split += 1
            dp = plan.to_device(hp, bt[:, :width].to(dev), dev)
            impl._forward_split(layer, q, k, v, kv_cache, dp, out)
            gpu_ops.check_device_errors(dev)
            continue_check = True
        torch.cuda.synchronize()

        # KV of this step landed in the right tier and slot, bit-exactly
        sb, so = slots // BS, slots % BS
        on_hbm = sb < G
        if on_hbm.any():
            i = on_hbm.nonzero().flatten()
            bd, od = sb[i].to(dev), so[i].to(dev)
            assert torch.equal(kv_cache[bd, :, od, :D], uk[bd, :, od])
            assert torch.equal(kv_cache[bd, :, od, D:], uv[bd, :, od])
        if (~on_hbm).any():
            i = (~on_hbm).nonzero().flatten()
            hk = host_k[sb[i] - G, :, so[i]]
            hv = host_v[sb[i] - G, :, so[i]]
            assert torch.equal(hk.to(dev), uk[sb[i].to(dev), :, so[i].to(dev)])
            assert torch.equal(hv.to(dev), uv[sb[i].to(dev), :, so[i].to(dev)])

        if continue_check:
            assert bool(torch.isfinite(out[:T]).all()), f"step {step}: unwritten output rows"
            for i, (r, ctx, ql) in enumerate(rows):
                L = ctx + ql
                nb = (L + BS - 1) // BS
                ids = torch.tensor(r["blocks"][:nb], device=dev)
                kk = uk[ids].permute(0, 2, 1, 3).reshape(-1, KVH, D)[:L]
                vv = uv[ids].permute(0, 2, 1, 3).reshape(-1, KVH, D)[:L]
                r0, r1 = int(qsl[i]), int(qsl[i + 1])
                ref = attend_fp32(q[r0:r1], kk, vv, scale, causal=True)
                err = (out[r0:r1].float() - ref).abs().max().item()
                assert err <= TOL[dtype], (step, i, ctx, ql, err)
                n_rows += 1

        for r, ctx, ql in rows:
            r["L"] = ctx + ql
            r["left"] -= 1
            if r["left"] <= 0:
                running.remove(r)
                release(r["blocks"])
    if device_plan:
        assert n_dev >= 5 and n_split + n_dev >= steps // 2 and n_rows > 100, (n_dev, n_split, n_rows)
    else:
        assert n_split >= steps // 2 and n_rows > 100
    state.STORE = None
