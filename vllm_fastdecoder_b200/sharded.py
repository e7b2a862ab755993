"""KV-sharded long-context decode across the GPUs of one node.

Each sequence's blocks are cut into `world` contiguous shards; rank r holds
shard r in its own HBM, computes the fp32 partial (o, lse) of every row over
its shard with the split-KV kernel, the packed partials [o (n*H*D) | lse (H*n)]
of all ranks are all-gathered with NCCL over NVLink, and every rank merges the
`world` partials with the log-sum-exp kernel.  The merge rule is the
reference's two-tier rule (fastdecode/cpu_ops.py:93-113) applied to P parts;
the reference itself has no multi-GPU path.

Two exchanges with the same interface: PartialExchange (NCCL all-gather,
then the merge kernel) and PeerExchange (fd_exchange_merge: one kernel per
step pushes the partial into every rank's buffer over NVLink, waits for
every rank's and merges; buffers shared with CUDA IPC, no multicast; with
decode_exchange_merge the same kernel also does the decode's combine).

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


class PeerExchange:
    """The exchange and merge over peer memory (C ABI fd_exchange_merge):
    o_view / lse_view are views of the packed send buffer the decode kernel
    writes; exchange_and_merge(final) runs one launch that needs every rank
    to call it for the same step.  Build it collectively (every rank of the
    group) after torch.cuda.set_device; close() collectively too.

    A step whose bounded wait ran out (a rank that never delivered) records
    FD_DEVERR_TIMEOUT in the device error word and leaves `final` unwritten;
    the launch itself reports nothing.  check() reads the word (a host
    synchronisation): after a timeout it marks the exchange unusable, so
    later steps raise until every rank closes it and builds a new one."""

    def __init__(self, n: int, H: int, D: int, world: int, device: torch.device, group=None, num_ctas: int = 64,
                 timeout_s: float = 2.0):
        import ctypes

        from vllm_fastdecoder_b200 import _native as nat

        self._nat, self._lib = nat, nat.load()
        self.n, self.H, self.D, self.world = n, H, D, world
        self.group, self.device = group, device
        self.rank = dist.get_rank(group) if world > 1 else 0
        self.num_ctas, self.timeout_ns = int(num_ctas), int(timeout_s * 1e9)
        self.slot = (n * H * D + H * n + 3) // 4 * 4
        self.send = torch.zeros(self.slot, dtype=torch.float32, device=device)
        self.o_view = self.send[: n * H * D].view(n, H, D)
        self.lse_view = self.send[n * H * D: n * H * D + H * n].view(H, n)
        self.lse_out = torch.empty(H, n, dtype=torch.float32, device=device)
        lib = self._lib
        nbytes = lib.fd_peer_buffer_bytes(world, self.slot)
        own = ctypes.c_void_p()
        handle = (ctypes.c_char * nat.IPC_HANDLE_BYTES)()
        nat.check(lib.fd_peer_alloc(nbytes, ctypes.byref(own), handle), "fd_peer_alloc")
        self._own, self._opened = own.value, []
        handles = [bytes(handle)]
        if world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, bytes(handle), group=group)
        x = nat.FdPeerExchange()
        x.rank, x.world, x.slot_floats = self.rank, world, self.slot
        for q in range(world):
            if q == self.rank:
                x.base[q] = self._own
                continue
            p = ctypes.c_void_p()
            buf = ctypes.create_string_buffer(handles[q], nat.IPC_HANDLE_BYTES)
            nat.check(lib.fd_peer_open(buf, ctypes.byref(p)), "fd_peer_open")
            x.base[q] = p.value
            self._opened.append(p.value)
        self.x = x
        self.failed: str | None = None
        if world > 1:
            dist.barrier(group=group)  # every rank mapped before the first step

    def gather(self) -> None:
        raise NotImplementedError("PeerExchange exchanges and merges in one launch: use exchange_and_merge")

    def exchange_and_merge(self, o_local_unused, lse_local_unused, final: torch.Tensor) -> None:
        import ctypes

        from vllm_fastdecoder_b200 import gpu_ops

        del o_local_unused, lse_local_unused
        nat = self._nat
        if self.failed is not None:
            raise RuntimeError(f"PeerExchange is unusable after a failed step ({self.failed}): close it on every "
                               "rank and build a new one")
        if not (final.is_contiguous() and tuple(final.shape) == (self.n, self.H, self.D)):
            raise RuntimeError("PeerExchange: final must be a contiguous [n, H, D] tensor")
        nat.check(self._lib.fd_exchange_merge(
            ctypes.byref(self.x), self.send.data_ptr(), self.n, self.H, self.D, final.data_ptr(),
            gpu_ops.dtype_code(final.dtype), self.lse_out.data_ptr(), self.num_ctas, self.timeout_ns,
            gpu_ops.error_word(self.device).data_ptr(), gpu_ops._stream(self.device)), "fd_exchange_merge")

    def check(self) -> None:
        """Synchronise and read the device error word of this rank's GPU;
        raise RuntimeError (and refuse every later step) if a kernel flagged
        an error, e.g. a step that timed out waiting for a rank."""
        from vllm_fastdecoder_b200 import gpu_ops

        try:
            gpu_ops.check_device_errors(self.device)
        except RuntimeError as e:
            self.failed = str(e)
            raise

    def decode_exchange_merge(self, args, final: torch.Tensor, decode: bool = True) -> None:
        """The whole sharded step (C ABI fd_decode_exchange_merge): the decode
        of `args` (gpu_ops.decode_args writing o_view / lse_view, fp32), then
        one exchange launch that also merges the segments the decode's CTAs
        cut, so no combine launch runs in between.  `final` [n, H, D].
        decode=False: only the exchange (fd_exchange_merge_decoded), after the
        caller's own gpu_ops.launch_decode(args, ..., "partials")."""
        import ctypes

        nat = self._nat
        if self.failed is not None:
            raise RuntimeError(f"PeerExchange is unusable after a failed step ({self.failed}): close it on every "
                               "rank and build a new one")
        if not (final.is_contiguous() and tuple(final.shape) == (self.n, self.H, self.D)):
            raise RuntimeError("PeerExchange: final must be a contiguous [n, H, D] tensor")
        if args.out != self.o_view.data_ptr() or args.lse != self.lse_view.data_ptr():
            raise RuntimeError("PeerExchange: the decode must write this exchange's o_view / lse_view")
        from vllm_fastdecoder_b200 import gpu_ops

        fn = self._lib.fd_decode_exchange_merge if decode else self._lib.fd_exchange_merge_decoded
        nat.check(fn(ctypes.byref(args), ctypes.byref(self.x), final.data_ptr(), gpu_ops.dtype_code(final.dtype),
                     self.lse_out.data_ptr(), self.num_ctas, self.timeout_ns, gpu_ops._stream(self.device)),
                  "fd_decode_exchange_merge" if decode else "fd_exchange_merge_decoded")

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (collective)."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            self._lib.fd_peer_close(p)
        self._opened = []
        if self.world > 1:
            dist.barrier(group=self.group)  # nobody maps this rank's buffer any more
        self._lib.fd_peer_free(self._own)
        self._own = None


def sharded_decode(q: torch.Tensor, tiers, tier_split: int, local_bt: torch.Tensor, local_lens: torch.Tensor,
                   scale: float, exchange: PartialExchange, final: torch.Tensor, **kw) -> None:
    """One decode step over the local shard followed by the exchange + merge
    (over peer memory: one decode launch and one exchange launch that also
    combines the decode's cut segments)."""
    from vllm_fastdecoder_b200 import gpu_ops

    if isinstance(exchange, PeerExchange) and kw.get("host_range") is None:
        kw.pop("host_range", None)
        a = gpu_ops.decode_args(q, tiers, tier_split, local_bt, local_lens, scale, exchange.o_view,
                                exchange.lse_view, **kw)
        exchange.decode_exchange_merge(a, final)
        return
    gpu_ops.decode_tiered(q, tiers, tier_split, local_bt, local_lens, scale, exchange.o_view, exchange.lse_view,
                          **kw)
    exchange.exchange_and_merge(None, None, final)
