"""KV-sharded decode on 2, 4 and 8 GPUs: each rank decodes its contiguous shard of
every row with the split-KV kernel into the packed exchange buffer; the
partials are exchanged and merged either with NCCL (all-gather, then
fd_merge_partials) or over peer memory (fd_exchange_merge: one kernel,
CUDA-IPC buffers, no multicast; and fd_decode_exchange_merge, whose exchange
kernel also does the decode's combine).  All must match the oracle over the
unsharded rows (bf16 output 1.6e-2, lse 1e-4) and each other bit for bit,
over three consecutive steps (both parities of the peer buffers).  NVLS is
off.  Each world size is skipped on a box with fewer GPUs."""

from __future__ import annotations

import math
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case():
    n, H, KVH, D, BS = 4, 32, 8, 128, 16
    lens = [3000, 1, 0, 777]
    C = sum((L + BS - 1) // BS for L in lens) + 4
    q, kc, vc, bt, _ = O.rand_case(n, H, KVH, D, BS, C, torch.bfloat16, max_len=max(lens), seed=21)
    perm = torch.randperm(C, generator=torch.Generator().manual_seed(22)).tolist()
    bt = torch.zeros(n, bt.shape[1], dtype=torch.int32)
    for i, L in enumerate(lens):
        nb = (L + BS - 1) // BS
        bt[i, :nb] = torch.tensor([perm.pop() for _ in range(nb)], dtype=torch.int32)
    return q, kc, vc, bt, torch.tensor(lens, dtype=torch.int32)


def _rank(rank, world, port, path):
    import datetime

    import torch.distributed as dist

    from vllm_fastdecoder_b200 import gpu_ops, sharded
    from vllm_fastdecoder_b200.gpu_ops import KVTier

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        q, kc, vc, bt, lens = _case()
        n, H, D = q.shape
        BS = kc.shape[2]
        lbt, llens = sharded.shard_rows(bt, lens, BS, world, rank)
        tiers = (KVTier(kc.to(dev), vc.to(dev)), None)
        res = {}
        for name in ("nccl", "peer", "peer_fused"):
            ex = (sharded.PartialExchange(n, H, D, world, dev) if name == "nccl"
                  else sharded.PeerExchange(n, H, D, world, dev))
            outs = []
            for _ in range(3):
                final = torch.full((n, H, D), float("nan"), dtype=q.dtype, device=dev)
                if name == "peer":  # decode (with its combine), then fd_exchange_merge
                    gpu_ops.decode_tiered(q.to(dev), tiers, 1 << 40, lbt.to(dev), llens.to(dev), 1.0 / math.sqrt(D),
                                          ex.o_view, ex.lse_view)
                    ex.exchange_and_merge(None, None, final)
                else:  # nccl, and the fused step (fd_decode_exchange_merge)
                    sharded.sharded_decode(q.to(dev), tiers, 1 << 40, lbt.to(dev), llens.to(dev),
                                           1.0 / math.sqrt(D), ex, final)
                torch.cuda.synchronize(dev)
                gpu_ops.check_device_errors(dev)
                outs.append((final.cpu(), ex.lse_out.cpu()))
            res[name] = outs
            if isinstance(ex, sharded.PeerExchange):
                ex.close()
        if rank == 0:
            torch.save(res, path)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_decode_on_several_gpus(tmp_path, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    path = str(tmp_path / "res.pt")
    mp.start_processes(_rank, args=(world, _free_port(), path), nprocs=world, start_method="spawn")
    res = torch.load(path)
    q, kc, vc, bt, lens = _case()
    D = q.shape[2]
    ref_o, ref_l = O.ref_decode_attn_f64(q, kc, vc, bt, lens, 1.0 / math.sqrt(D))
    nz = lens > 0
    for k in range(3):
        for name in ("nccl", "peer", "peer_fused"):
            out, lse = res[name][k]
            torch.testing.assert_close(out[nz].double(), ref_o[nz], atol=1.6e-2, rtol=1.6e-2)
            torch.testing.assert_close(lse[:, nz].double(), ref_l[:, nz], atol=1e-4, rtol=1e-5)
            assert torch.all(out[~nz] == 0) and torch.all(torch.isneginf(lse[:, ~nz]))
        for name in ("peer", "peer_fused"):
            assert torch.equal(res["nccl"][k][0], res[name][k][0]) and torch.equal(res["nccl"][k][1], res[name][k][1])
