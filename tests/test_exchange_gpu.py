"""The peer-memory exchange kernel (fd_exchange_merge) on one GPU.

world = 1: the rank merges its own partial, so over several consecutive
steps (both buffer parities, and replays of a captured CUDA graph) the
result must equal fd_merge_partials with one part, bit for bit.  A peer
that never signals (a second local buffer standing in for rank 1) must make
the bounded wait give up: FD_DEVERR_TIMEOUT in the error word, no fault, the
context still usable.  The two-rank exchange is tested on 2 GPUs in
test_sharded_gpu.py."""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _partials(n, H, D, seed, dev):
    g = torch.Generator().manual_seed(seed)
    o = torch.randn(n, H, D, generator=g)
    lse = torch.randn(H, n, generator=g) * 4
    lse[:, 1] = float("-inf")  # an empty row
    lse[2, 0] = float("inf")  # FlashAttention's empty convention counts as empty
    return o.to(dev), lse.to(dev)


def test_single_rank_exchange_equals_merge_partials():
    from vllm_fastdecoder_b200 import gpu_ops, sharded

    dev = torch.device("cuda")
    n, H, D = 5, 8, 128
    ex = sharded.PeerExchange(n, H, D, 1, dev)
    try:
        for step in range(4):
            o, lse = _partials(n, H, D, step, dev)
            ex.o_view.copy_(o)
            ex.lse_view.copy_(lse)
            final = torch.full((n, H, D), float("nan"), dtype=torch.bfloat16, device=dev)
            ex.exchange_and_merge(None, None, final)
            ref = torch.empty_like(final)
            ref_lse = torch.empty(H, n, dtype=torch.float32, device=dev)
            packed = torch.cat([o.flatten(), lse.flatten()])
            gpu_ops.merge_partials(packed, 1, n, H, D, ref, ref_lse)
            torch.cuda.synchronize()
            gpu_ops.check_device_errors(dev)
            assert torch.equal(final, ref), step
            assert torch.equal(ex.lse_out, ref_lse), step
        # the same launch captured in a graph keeps stepping through the parities
        g = torch.cuda.CUDAGraph()
        final = torch.empty(n, H, D, dtype=torch.bfloat16, device=dev)
        with torch.cuda.graph(g):
            ex.exchange_and_merge(None, None, final)
        for step in range(4, 7):
            o, lse = _partials(n, H, D, step, dev)
            ex.o_view.copy_(o)
            ex.lse_view.copy_(lse)
            g.replay()
            ref = torch.empty_like(final)
            ref_lse = torch.empty(H, n, dtype=torch.float32, device=dev)
            gpu_ops.merge_partials(torch.cat([o.flatten(), lse.flatten()]), 1, n, H, D, ref, ref_lse)
            torch.cuda.synchronize()
            gpu_ops.check_device_errors(dev)
            assert torch.equal(final, ref), step
            assert torch.equal(ex.lse_out, ref_lse), step
        del g
    finally:
        ex.close()


def test_silent_peer_times_out_without_fault():
    from vllm_fastdecoder_b200 import _native as nat
    from vllm_fastdecoder_b200 import gpu_ops

    dev = torch.device("cuda")
    lib = nat.load()
    n, H, D = 2, 4, 64
    slot = (n * H * D + H * n + 3) // 4 * 4
    nbytes = lib.fd_peer_buffer_bytes(2, slot)
    bufs = []
    for _ in range(2):
        p = ctypes.c_void_p()
        h = (ctypes.c_char * nat.IPC_HANDLE_BYTES)()
        nat.check(lib.fd_peer_alloc(nbytes, ctypes.byref(p), h), "fd_peer_alloc")
        bufs.append(p.value)
    try:
        x = nat.FdPeerExchange()
        x.rank, x.world, x.slot_floats = 0, 2, slot
        x.base[0], x.base[1] = bufs[0], bufs[1]  # "rank 1" is a buffer nobody signals from
        send = torch.zeros(slot, dtype=torch.float32, device=dev)
        out = torch.empty(n, H, D, dtype=torch.float16, device=dev)
        lse = torch.empty(H, n, dtype=torch.float32, device=dev)
        err = gpu_ops.error_word(dev)
        nat.check(lib.fd_exchange_merge(ctypes.byref(x), send.data_ptr(), n, H, D, out.data_ptr(),
                                        gpu_ops.dtype_code(out.dtype), lse.data_ptr(), 4, 50_000_000,
                                        err.data_ptr(), gpu_ops._stream(dev)), "fd_exchange_merge")
        with pytest.raises(RuntimeError, match="device error 3"):
            gpu_ops.check_device_errors(dev)
        # the context is still usable
        t = torch.ones(4, device=dev) * 2
        assert float(t.sum()) == 8.0
    finally:
        torch.cuda.synchronize()
        for p in bufs:
            lib.fd_peer_free(p)
