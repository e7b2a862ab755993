"""CUDA-graph capture of a decode-only step (vllm_fastdecoder_b200.graph):
device planner + per layer KV write and decode, captured once and replayed on
new step data written into the same buffers.  Each replay must equal the
same launches run eagerly (same kernels and schedule: bit-identical) and the
oracle (bf16 output 1.6e-2, lse 1e-4); rows of idle requests (no query
token) are not written."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("H,KVH", [(16, 4), (8, 8)])
def test_captured_step_matches_eager_and_oracle(H, KVH):
    from oracle import oracle as O
    from vllm_fastdecoder_b200 import gpu_ops
    from vllm_fastdecoder_b200.graph import DecodeStepGraph
    from vllm_fastdecoder_b200.gpu_ops import KVTier

    dev = torch.device("cuda")
    dt = torch.bfloat16
    L, R, D, BS, G, C, W = 3, 24, 128, 16, 600, 800, 40
    scale = D ** -0.5
    g = torch.Generator().manual_seed(H)
    layers = []
    for _ in range(L):
        hk = torch.randn(G, KVH, BS, D, generator=g).to(dt)
        hv = torch.randn(G, KVH, BS, D, generator=g).to(dt)
        ck = torch.randn(C, KVH, BS, D, generator=g).to(dt).pin_memory()
        cv = torch.randn(C, KVH, BS, D, generator=g).to(dt).pin_memory()
        layers.append((hk.to(dev), hv.to(dev), ck, cv))
    tiers = [(KVTier(a, b), KVTier(c, d)) for a, b, c, d in layers]
    step = DecodeStepGraph(L, R, W, H, KVH, D, dt, tiers, G, C, BS, scale, max_len=W * BS, device=dev)

    def fill(seed):
        gs = torch.Generator().manual_seed(seed)
        active = torch.rand(R, generator=gs) < 0.85  # idle requests have no query token this step
        lens = torch.randint(1, W * BS + 1, (R,), generator=gs).to(torch.int32)
        perm = (torch.randperm(G + C - 1, generator=gs) + 1).tolist()
        bt = torch.randint(0, G + C, (R, W), generator=gs).to(torch.int32)  # junk past each row's end
        slots = []
        for i in range(R):
            nb = (int(lens[i]) + BS - 1) // BS
            bt[i, :nb] = torch.tensor([perm.pop() for _ in range(nb)], dtype=torch.int32)
            if active[i]:
                p = int(lens[i]) - 1
                slots.append(int(bt[i, p // BS]) * BS + p % BS)
        qsl = torch.zeros(R + 1, dtype=torch.int32)
        qsl[1:] = torch.cumsum(active.to(torch.int32), 0)
        T = int(qsl[-1])
        sm = torch.full((R,), -1, dtype=torch.int64)
        sm[:T] = torch.tensor(slots, dtype=torch.int64)
        step.query_start_loc.copy_(qsl)
        step.seq_lens.copy_(lens)
        step.block_table.copy_(bt)
        step.slot_mapping.copy_(sm)
        for t in (step.q, step.k, step.v):
            t.copy_(torch.randn(t.shape, generator=gs).to(dt))
        return active, lens, bt, qsl

    fill(0)
    step.capture()
    for seed in (1, 2, 3):
        active, lens, bt, qsl = fill(seed)
        step.out.fill_(float("nan"))
        step.replay()
        torch.cuda.synchronize()
        gpu_ops.check_device_errors(dev)
        out_g, lse_g = step.out.clone(), step.lse.clone()
        step.out.fill_(float("nan"))
        step.run_eager()
        torch.cuda.synchronize()
        gpu_ops.check_device_errors(dev)
        rows = active.nonzero().flatten()
        toks = qsl.long()[rows]
        n = rows.numel()
        assert torch.equal(out_g[:, toks], step.out[:, toks])
        assert torch.equal(lse_g[:, :, :n], step.lse[:, :, :n])
        idle = torch.ones(R, dtype=torch.bool)
        idle[toks] = False
        assert torch.all(torch.isnan(out_g[:, idle].float()))
        for l in range(L):
            hk, hv, ck, cv = layers[l]
            kc = torch.cat([hk.cpu(), ck])
            vc = torch.cat([hv.cpu(), cv])
            o = torch.empty(n, H, D, dtype=dt)
            lo = torch.empty(H, n)
            O.decode_attn(step.q[l].cpu()[toks], kc, vc, bt[rows], lens[rows], scale, o, lo)
            torch.testing.assert_close(out_g[l].cpu()[toks].float(), o.float(), atol=1.6e-2, rtol=1.6e-2)
            assert (lse_g[l].cpu()[:, :n] - lo).abs().max().item() <= 1e-4
