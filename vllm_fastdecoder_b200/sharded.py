"""KV-sharded long-context decode across the GPUs of one node.

Each sequence's blocks are cut into `world` contiguous shards; rank r holds
shard r in its own HBM, computes the fp32 partial (o, lse) of every row over
its shard with the split-KV kernel, the packed partials [o (n*H*D) | lse (H*n)]
of all ranks are all-gathered with NCCL over NVLink, and every rank merges the
`world` partials with the log-sum-exp kernel.  The merge rule is the
reference's two-tier rule (fastdecode/cpu_ops.py:93-113) applied to P parts;
the reference itself has no multi-GPU path.

One process per GPU (torchrun); the process group is the caller's.
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist


def shard_range(n_blocks: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous block range [lo, hi) of `rank` (earlier ranks take the
    remainder), so shards differ by at most one block."""
    base, extra = divmod(n_blocks, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def shard_rows(block_table: torch.Tensor, lens: torch.Tensor, block_size: int, world: int, rank: int):
    """This rank's slice of every row: (block_table [n, W'] int32, lens [n]
    int32).  The row's last, possibly partial block stays with the last shard
    that owns it, so every shard but the last holds whole blocks."""
    n = block_table.shape[0]
    parts, lengths = [], []
    for i in range(n):
        L = int(lens[i])
        nb = (L + block_size - 1) // block_size
        lo, hi = shard_range(nb, world, rank)
        ids = block_table[i, lo:hi]
        tok_hi = min(L, hi * block_size)
        tok_lo = lo * block_size
        parts.append(ids)
        lengths.append(max(0, tok_hi - tok_lo) if hi > lo else 0)
    W = max(1, max(int(p.numel()) for p in parts))
    out = torch.zeros(n, W, dtype=torch.int32)
    for i, p in enumerate(parts):
        out[i, :p.numel()] = p.to(torch.int32)
    return out, torch.tensor(lengths, dtype=torch.int32)


class PartialExchange:
    """Packed send/receive buffers for one all-gather of fp32 partials.

    The decode kernel writes straight into `o_view` [n, H, D] and `lse_view`
    [H, n] (both views of the send buffer), so the exchange needs no copy."""

    def __init__(self, n: int, H: int, D: int, world: int, device: torch.device, group=None,
                 merge_fn: Callable | None = None):
        self.n, self.H, self.D, self.world = n, H, D, world
        self.stride = n * H * D + H * n
        self.send = torch.zeros(self.stride, dtype=torch.float32, device=device)
        self.recv = torch.empty(world * self.stride, dtype=torch.float32, device=device)
        self.o_view = self.send[: n * H * D].view(n, H, D)
        self.lse_view = self.send[n * H * D:].view(H, n)
        self.lse_out = torch.empty(H, n, dtype=torch.float32, device=device)
        self.group = group
        if merge_fn is None:
            from vllm_fastdecoder_b200 import gpu_ops

            merge_fn = gpu_ops.merge_partials
        self.merge_fn = merge_fn

    def gather(self) -> None:
        if self.world == 1:
            self.recv.copy_(self.send)
        elif self.send.is_cuda:
            dist.all_gather_into_tensor(self.recv, self.send, group=self.group)
        else:  # gloo
            dist.all_gather(list(self.recv.view(self.world, self.stride).unbind(0)), self.send, group=self.group)

    def exchange_and_merge(self, o_local_unused, lse_local_unused, final: torch.Tensor) -> None:
        """All-gather the packed partials and merge them into `final` [n, H, D]
        (any output dtype) and `lse_out` [H, n]."""
        del o_local_unused, lse_local_unused
        self.gather()
        self.merge_fn(self.recv, self.world, self.n, self.H, self.D, final, self.lse_out)


def sharded_decode(q: torch.Tensor, tiers, tier_split: int, local_bt: torch.Tensor, local_lens: torch.Tensor,
                   scale: float, exchange: PartialExchange, final: torch.Tensor, **kw) -> None:
    """One decode step over the local shard followed by the exchange + merge."""
    from vllm_fastdecoder_b200 import gpu_ops

    gpu_ops.decode_tiered(q, tiers, tier_split, local_bt, local_lens, scale, exchange.o_view, exchange.lse_view,
                          **kw)
    exchange.exchange_and_merge(None, None, final)
