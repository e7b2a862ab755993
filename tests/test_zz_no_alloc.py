"""fd_decode_attn_noalloc: the decode entry point for callers that cannot
allocate device memory (for example code that runs after vLLM has sized its
KV cache to fill the memory left free, or inside a framework that owns all
device memory through its own allocator).  It keeps its split partials in a
scratch array built into the library instead of a caller workspace.

The checks call both entry points through the C ABI on the same arguments and
require the same output, and the C oracle's (the restatement of the reference
decode_attn) within the decode tests' tolerances, on two calls in a row with
different batches (so a call cannot lean on what the previous one left in the
shared scratch).  Both schedules are covered: the split grid (fixed
tiles_per_split) and the default persistent schedule, on the CUDA-core kernel
(fp16 MHA) and the tensor-core kernel (bf16, 32 query heads over 8 kv heads).
Arguments needing more scratch than the array holds must be refused.  This
file is collected last so that a run stopping at the first failure has run
every other test first; it also passes alone in a fresh process.
"""

from __future__ import annotations

import ctypes
import math

import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

# the parity tolerance of the decode tests (output dtype fp16 / bf16; lse)
TOL = {torch.float16: 2e-3, torch.bfloat16: 1.6e-2}
LSE_TOL = 1e-4


def _batch(dtype, H, KVH, seed, max_len):
    n, D, BS = 5, 128, 16
    C = n * ((max_len + BS - 1) // BS) + 8
    q, kc, vc, bt, lens = O.rand_case(n, H, KVH, D, BS, C, dtype, max_len=max_len, seed=seed)
    lens[2] = 0
    return q, kc, vc, bt, lens


def _args(q, kc, vc, bt, lens, out, lse, tiles_per_split=8):
    from vllm_fastdecoder_b200 import gpu_ops
    from vllm_fastdecoder_b200.gpu_ops import KVTier

    D = q.shape[-1]
    return gpu_ops.decode_args(q, (KVTier(kc, vc), None), 1 << 40, bt, lens, 1.0 / math.sqrt(D), out, lse,
                               tiles_per_split=tiles_per_split)


@pytest.mark.parametrize("dtype,H,KVH,tps,kernel", [
    (torch.float16, 8, 8, 8, "fd_decode_kernel"),  # split grid
    (torch.bfloat16, 16, 4, 8, "fd_decode_kernel"),
    (torch.float16, 8, 8, 0, "fd_decode_kernel"),  # persistent schedule, CUDA cores
    (torch.bfloat16, 32, 8, 0, "fd_decode_mma_kernel"),  # persistent schedule, tensor cores
])
def test_noalloc_matches_workspace_entry_point_and_oracle_twice(dtype, H, KVH, tps, kernel):
    from vllm_fastdecoder_b200 import _native as nat
    from vllm_fastdecoder_b200 import gpu_ops

    lib = nat.load()
    dev = torch.device("cuda")
    stream = torch.cuda.current_stream(dev).cuda_stream
    for call, (seed, max_len) in enumerate([(1, 3000), (2, 1700)]):
        q_c, kc_c, vc_c, bt_c, lens_c = _batch(dtype, H, KVH, seed, max_len)
        q, kc, vc, bt, lens = (t.to(dev) for t in (q_c, kc_c, vc_c, bt_c, lens_c))
        n, _, D = q.shape
        assert gpu_ops.decode_kernel_name(dtype, D, H, KVH, kc.shape[2], n, tps) == kernel
        out_ws = torch.full((n, H, D), float("nan"), dtype=dtype, device=dev)
        lse_ws = torch.full((H, n), float("nan"), device=dev)
        a = _args(q, kc, vc, bt, lens, out_ws, lse_ws, tps)
        assert lib.fd_decode_workspace_size(ctypes.byref(a)) > 0, "case must use split scratch"
        nat.check(lib.fd_decode_attn(ctypes.byref(a), stream), "fd_decode_attn")

        out_na = torch.full((n, H, D), float("nan"), dtype=dtype, device=dev)
        lse_na = torch.full((H, n), float("nan"), device=dev)
        b = _args(q, kc, vc, bt, lens, out_na, lse_na, tps)
        b.workspace = None
        b.workspace_bytes = 0
        nat.check(lib.fd_decode_attn_noalloc(ctypes.byref(b), stream), f"fd_decode_attn_noalloc (call {call})")
        torch.cuda.synchronize(dev)
        gpu_ops.check_device_errors(dev)

        ref = torch.empty(n, H, D, dtype=dtype)
        ref_l = torch.empty(H, n)
        O.decode_attn(q_c, kc_c, vc_c, bt_c, lens_c, 1.0 / math.sqrt(D), ref, ref_l)
        nz = lens_c > 0
        for out, lse in ((out_na, lse_na), (out_ws, lse_ws)):
            assert (out.cpu().float() - ref.float()).abs().max().item() <= TOL[dtype]
            assert (lse.cpu()[:, nz] - ref_l[:, nz]).abs().max().item() <= LSE_TOL
        torch.testing.assert_close(out_na.cpu().float(), out_ws.cpu().float(), atol=TOL[dtype], rtol=TOL[dtype])
        assert (lse_na.cpu()[:, nz] - lse_ws.cpu()[:, nz]).abs().max().item() <= LSE_TOL
        assert torch.all(out_na.cpu()[~nz] == 0) and torch.all(torch.isneginf(lse_na.cpu()[:, ~nz]))


def test_noalloc_rejects_arguments_beyond_its_scratch():
    from vllm_fastdecoder_b200 import _native as nat

    lib = nat.load()
    dev = torch.device("cuda")
    n, H, KVH, D, BS, W = 4096, 32, 32, 128, 16, 256
    q = torch.zeros(n, H, D, dtype=torch.float16, device=dev)
    kc = torch.zeros(8, KVH, BS, D, dtype=torch.float16, device=dev)
    bt = torch.zeros(n, W, dtype=torch.int32, device=dev)
    lens = torch.zeros(n, dtype=torch.int32, device=dev)
    out = torch.zeros_like(q)
    lse = torch.zeros(H, n, device=dev)
    a = _args(q, kc, kc, bt, lens, out, lse)
    need = lib.fd_decode_workspace_size(ctypes.byref(a))
    assert need > nat.NOALLOC_SCRATCH_BYTES
    a.workspace = None
    a.workspace_bytes = 0
    rc = lib.fd_decode_attn_noalloc(ctypes.byref(a), torch.cuda.current_stream(dev).cuda_stream)
    assert rc == nat.FD_ERR_WORKSPACE
    assert b"FD_NOALLOC_SCRATCH_BYTES" in lib.fd_last_error_message()
