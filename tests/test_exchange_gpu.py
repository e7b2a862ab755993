"""The peer-memory exchange kernel (fd_exchange_merge, fd_decode_exchange_merge)
on one GPU.

world = 1: the rank merges its own partial, so over several consecutive
steps (both buffer parities, and replays of a captured CUDA graph) the
result must equal fd_merge_partials with one part, bit for bit; the fused
step (decode, then the exchange that also does the decode's combine) must
equal decode + combine + merge bit for bit, on both decode kernels, with
segments cut between CTAs and whole ones, and on the split grid.  A peer
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


def test_peer_a_step_ahead_does_not_complete_a_missing_rank():
    """World 3 on one GPU with two stand-in peer buffers: "rank 1" has already
    delivered the next step (every word of its slot carries step 2 where
    step 1 is due) and "rank 2" never delivers.  Neither may complete step 1:
    the merge waits for words carrying exactly this step, so the wait runs
    out (FD_DEVERR_TIMEOUT) and the outputs stay unwritten.  This rank's own
    words of step 1 reach every rank's buffer."""
    from vllm_fastdecoder_b200 import _native as nat
    from vllm_fastdecoder_b200 import gpu_ops

    dev = torch.device("cuda")
    lib = nat.load()
    n, H, D, world = 2, 4, 64, 3
    slot = (n * H * D + H * n + 3) // 4 * 4
    nbytes = lib.fd_peer_buffer_bytes(world, slot)
    assert nbytes == nat.PEER_RECV_OFFSET + 2 * world * slot * 8
    # plain device buffers stand in for the three ranks' allocations (zeroed:
    # counters and slots start at 0, as fd_peer_alloc leaves them); word i of
    # slot (parity, q) is the int64 at PEER_RECV_OFFSET / 8 + (parity * world + q) * slot + i,
    # its high 32 bits the step
    bufs = [torch.zeros(nbytes // 8 + 1, dtype=torch.int64, device=dev) for _ in range(world)]
    r0 = nat.PEER_RECV_OFFSET // 8
    par = 1  # step 1
    ahead = bufs[0][r0 + (par * world + 1) * slot: r0 + (par * world + 2) * slot]
    ahead.fill_((2 << 32) | 0x3F800000)  # rank 1's words: value 1.0, step 2
    x = nat.FdPeerExchange()
    x.rank, x.world, x.slot_floats = 0, world, slot
    for q in range(world):
        x.base[q] = bufs[q].data_ptr()
    send = torch.ones(slot, dtype=torch.float32, device=dev)
    out = torch.full((n, H, D), 7.0, dtype=torch.float16, device=dev)
    lse = torch.full((H, n), 7.0, dtype=torch.float32, device=dev)
    err = gpu_ops.error_word(dev)
    ctas = 4
    nat.check(lib.fd_exchange_merge(ctypes.byref(x), send.data_ptr(), n, H, D, out.data_ptr(),
                                    gpu_ops.dtype_code(out.dtype), lse.data_ptr(), ctas, 50_000_000,
                                    err.data_ptr(), gpu_ops._stream(dev)), "fd_exchange_merge")
    with pytest.raises(RuntimeError, match="device error 3"):
        gpu_ops.check_device_errors(dev)
    assert bool((out == 7.0).all()) and bool((lse == 7.0).all())
    # this rank did deliver: its slot of step 1 in every rank's buffer holds
    # send (1.0) tagged with step 1
    for q in range(world):
        own = bufs[q][r0 + (par * world + 0) * slot: r0 + (par * world + 1) * slot].cpu()
        assert bool(((own >> 32) == 1).all())
        assert bool(((own & 0xFFFFFFFF) == 0x3F800000).all())
    torch.cuda.synchronize()


def test_check_marks_a_timed_out_exchange_unusable():
    """PeerExchange.check() reads the error word after a step: a step that
    timed out (here: a stand-in rank 1 that never delivers) makes check()
    raise, and every later step is refused until the exchange is rebuilt."""
    from vllm_fastdecoder_b200 import _native as nat
    from vllm_fastdecoder_b200 import sharded

    dev = torch.device("cuda")
    n, H, D = 3, 8, 64
    ex = sharded.PeerExchange(n, H, D, 1, dev, num_ctas=4, timeout_s=0.05)
    fake = torch.zeros(ex._lib.fd_peer_buffer_bytes(2, ex.slot) // 8 + 1, dtype=torch.int64, device=dev)
    try:
        x = nat.FdPeerExchange()
        x.rank, x.world, x.slot_floats = 0, 2, ex.slot
        x.base[0], x.base[1] = ex.x.base[0], fake.data_ptr()
        ex.x = x  # as if rank 1 had mapped its buffer and then stopped
        final = torch.zeros(n, H, D, dtype=torch.bfloat16, device=dev)
        ex.exchange_and_merge(None, None, final)
        with pytest.raises(RuntimeError, match="device error 3"):
            ex.check()
        with pytest.raises(RuntimeError, match="unusable"):
            ex.exchange_and_merge(None, None, final)
    finally:
        torch.cuda.synchronize()
        ex.close()


@pytest.mark.parametrize("dtype,H,KVH,lens,tps", [
    (torch.bfloat16, 32, 8, [20000, 1, 0, 777, 9000], 0),  # tensor-core kernel, long rows cut between CTAs
    (torch.float16, 16, 16, [3000, 5, 0, 1200], 0),        # CUDA-core kernel
    (torch.float16, 8, 2, [40, 17, 0, 64], 0),             # short rows: segments whole within a CTA
    (torch.bfloat16, 32, 8, [9000, 3, 2500], 16),          # split grid: the decode's own combine runs
])
def test_fused_step_equals_decode_combine_merge(dtype, H, KVH, lens, tps):
    from oracle import oracle as O
    from vllm_fastdecoder_b200 import gpu_ops, sharded
    from vllm_fastdecoder_b200.gpu_ops import KVTier

    dev = torch.device("cuda")
    n, D, BS = len(lens), 128, 16
    C = sum((L + BS - 1) // BS for L in lens) + 4
    q, kc, vc, bt, _ = O.rand_case(n, H, KVH, D, BS, C, dtype, max_len=max(lens), seed=31)
    g = torch.Generator().manual_seed(32)
    perm = torch.randperm(C, generator=g).tolist()
    bt = torch.zeros(n, bt.shape[1], dtype=torch.int32)
    for i, L in enumerate(lens):
        nb = (L + BS - 1) // BS
        bt[i, :nb] = torch.tensor([perm.pop() for _ in range(nb)], dtype=torch.int32)
    lens_t = torch.tensor(lens, dtype=torch.int32, device=dev)
    tiers = (KVTier(kc.to(dev), vc.to(dev)), None)
    qd, btd = q.to(dev), bt.to(dev)
    scale = 1.0 / (D ** 0.5)
    ex = sharded.PeerExchange(n, H, D, 1, dev)
    try:
        for decode_in_call in (True, False, True):  # 3 steps: both parities, both entry points
            # reference: decode + combine into the send views, then the P = 1 merge
            ref = torch.empty(n, H, D, dtype=dtype, device=dev)
            ref_lse = torch.empty(H, n, dtype=torch.float32, device=dev)
            gpu_ops.decode_tiered(qd, tiers, 1 << 40, btd, lens_t, scale, ex.o_view, ex.lse_view, tiles_per_split=tps)
            gpu_ops.merge_partials(ex.send[: n * H * D + H * n], 1, n, H, D, ref, ref_lse)
            torch.cuda.synchronize()
            ex.o_view.fill_(float("nan"))  # the fused step must not lean on the reference's writes
            ex.lse_view.fill_(float("nan"))
            final = torch.full((n, H, D), float("nan"), dtype=dtype, device=dev)
            a = gpu_ops.decode_args(qd, tiers, 1 << 40, btd, lens_t, scale, ex.o_view, ex.lse_view,
                                    tiles_per_split=tps)
            if not decode_in_call:
                gpu_ops.launch_decode(a, dev, "partials")
            ex.decode_exchange_merge(a, final, decode=decode_in_call)
            torch.cuda.synchronize()
            gpu_ops.check_device_errors(dev)
            assert torch.equal(final, ref)
            assert torch.equal(ex.lse_out, ref_lse)
    finally:
        ex.close()
