"""The KV-sharded long-context path with world_size 2 on CPU (gloo): block
sharding, the packed [o | lse] exchange buffer, the all-gather and the P-way
LSE merge, with the oracle standing in for the GPU kernels.  The merged
result must equal attention over the unsharded rows."""

from __future__ import annotations

import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O
from vllm_fastdecoder_b200 import sharded


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(seed=0):
    n, H, KVH, D, BS = 5, 8, 2, 64, 16
    lens = [1, 16, 17, 400, 0]
    C = sum((L + BS - 1) // BS for L in lens) + 4
    q, kc, vc, bt, _ = O.rand_case(n, H, KVH, D, BS, C, torch.float32, max_len=max(lens), seed=seed)
    lens_t = torch.tensor(lens, dtype=torch.int32)
    perm = torch.randperm(C, generator=torch.Generator().manual_seed(seed + 1)).tolist()
    bt = torch.zeros(n, bt.shape[1], dtype=torch.int32)
    for i, L in enumerate(lens):
        nb = (L + BS - 1) // BS
        bt[i, :nb] = torch.tensor([perm.pop() for _ in range(nb)], dtype=torch.int32)
    return q, kc, vc, bt, lens_t


def _merge_with_oracle(recv, world, n, H, D, final, lse_out):
    final.copy_(O.merge_parts(recv.view(world, -1), world, n, H, D, out_lse=lse_out))


def _rank(rank, world, port, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, kc, vc, bt, lens = _case()
        n, H, D = q.shape
        BS = kc.shape[2]
        lbt, llens = sharded.shard_rows(bt, lens, BS, world, rank)
        ex = sharded.PartialExchange(n, H, D, world, torch.device("cpu"), merge_fn=_merge_with_oracle)
        O.decode_attn_tiered(q, (kc, vc), None, 1 << 40, lbt, llens, 1.0 / math.sqrt(D), ex.o_view, ex.lse_view)
        final = torch.empty(n, H, D)
        ex.exchange_and_merge(None, None, final)
        if rank == 0:
            torch.save({"out": final, "lse": ex.lse_out}, result_path)
    finally:
        dist.destroy_process_group()


def test_shard_rows_partition_blocks_contiguously():
    q, kc, vc, bt, lens = _case()
    BS = kc.shape[2]
    for world in (1, 2, 3, 8):
        parts = [sharded.shard_rows(bt, lens, BS, world, r) for r in range(world)]
        for i in range(bt.shape[0]):
            L = int(lens[i])
            nb = (L + BS - 1) // BS
            ids = torch.cat([p[0][i, : (int(p[1][i]) + BS - 1) // BS] for p in parts])
            assert ids.tolist() == bt[i, :nb].tolist()
            assert sum(int(p[1][i]) for p in parts) == L


@pytest.mark.parametrize("world", [2])
def test_sharded_decode_gloo_matches_full(tmp_path, world):
    path = str(tmp_path / "result.pt")
    mp.start_processes(_rank, args=(world, _free_port(), path), nprocs=world, start_method="spawn")
    res = torch.load(path)
    q, kc, vc, bt, lens = _case()
    D = q.shape[2]
    ref_o, ref_l = O.ref_decode_attn_f64(q, kc, vc, bt, lens, 1.0 / math.sqrt(D))
    nz = lens > 0
    torch.testing.assert_close(res["out"][nz].double(), ref_o[nz], atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(res["lse"][:, nz].double(), ref_l[:, nz], atol=1e-4, rtol=1e-6)
    assert torch.all(res["out"][~nz] == 0) and torch.all(torch.isneginf(res["lse"][:, ~nz]))
