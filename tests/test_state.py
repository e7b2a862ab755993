"""The worker's host KV tier (state.ensure_store / HostArena).

CPU tests run with registration off (pin=False); the GPU test registers the
arena with CUDA and decodes from it over PCIe, checked against the oracle."""

from __future__ import annotations

import math
from types import SimpleNamespace

import pytest
import torch

from vllm_fastdecoder_b200 import state


def _spec(KVH=2, BS=16, D=64, dtype=torch.float16):
    elem = torch.empty((), dtype=dtype).element_size()
    return SimpleNamespace(num_kv_heads=KVH, block_size=BS, head_size=D, dtype=dtype,
                           page_size_bytes=2 * BS * KVH * D * elem, sliding_window=None)


def _vcfg(num_gpu_blocks):
    return SimpleNamespace(cache_config=SimpleNamespace(num_gpu_blocks=num_gpu_blocks))


@pytest.fixture(autouse=True)
def _clean(monkeypatch):
    monkeypatch.delenv("FASTDECODE_CPU_KV_GB", raising=False)
    monkeypatch.setenv("FASTDECODE_CPU_BLOCKS", "12")
    state.STORE = None
    yield
    state.STORE = None


def test_store_views_one_arena_in_the_reference_layout():
    names = ["l0", "l1", "l2"]
    state.ensure_store(_vcfg(40), _spec(), names, pin=False)
    st = state.STORE
    assert st is not None and st.num_gpu_blocks == 40 and st.num_cpu_blocks == 12
    assert st.arena is not None and st.arena.shape == (3, 2, 12, 2, 16, 64)
    for i, nm in enumerate(names):
        assert st.k[nm].shape == (12, 2, 16, 64) and st.k[nm].is_contiguous()
        assert st.k[nm].data_ptr() == st.arena.buf[i, 0].data_ptr()
        assert st.v[nm].data_ptr() == st.arena.buf[i, 1].data_ptr()
        assert float(st.k[nm].abs().sum()) == 0.0  # zero-filled
    # K and V of all layers are disjoint
    ptrs = sorted(t.data_ptr() for t in list(st.k.values()) + list(st.v.values()))
    step = 12 * 2 * 16 * 64 * 2
    assert all(b - a == step for a, b in zip(ptrs, ptrs[1:]))


def test_store_is_idempotent_and_replaced_on_new_sizes():
    names = ["a", "b"]
    state.ensure_store(_vcfg(None), _spec(), names, pin=False)  # memory profiling: no block count yet
    assert state.STORE is None
    state.ensure_store(_vcfg(40), _spec(), names, pin=False)
    first = state.STORE
    state.ensure_store(_vcfg(40), _spec(), names, pin=False)
    assert state.STORE is first  # same sizes and layers: kept
    state.ensure_store(_vcfg(41), _spec(), names, pin=False)
    assert state.STORE is not first and state.STORE.num_gpu_blocks == 41


def test_no_host_blocks_means_no_store(monkeypatch):
    state.ensure_store(_vcfg(40), _spec(), ["a"], pin=False)
    assert state.STORE is not None
    monkeypatch.setenv("FASTDECODE_CPU_BLOCKS", "0")
    state.ensure_store(_vcfg(40), _spec(), ["a"], pin=False)
    assert state.STORE is None
    monkeypatch.delenv("FASTDECODE_CPU_BLOCKS")
    state.ensure_store(_vcfg(40), _spec(), ["a"], pin=False)  # plugin off: nothing changes
    assert state.STORE is None


def test_size_from_gib(monkeypatch):
    monkeypatch.delenv("FASTDECODE_CPU_BLOCKS")
    spec = _spec()
    monkeypatch.setenv("FASTDECODE_CPU_KV_GB", str(10 * spec.page_size_bytes * 2 / 2**30))
    state.ensure_store(_vcfg(8), spec, ["a", "b"], pin=False)
    assert state.STORE.num_cpu_blocks == 10


def test_validate_spec_rejects_sliding_window():
    spec = _spec()
    spec.sliding_window = 128
    with pytest.raises(NotImplementedError):
        state.ensure_store(_vcfg(8), spec, ["a"], pin=False)


@pytest.mark.gpu
def test_registered_arena_is_read_by_the_decode_kernel():
    """The arena registered with CUDA is device-mapped: a decode over its
    host tier (read in place over PCIe) matches the oracle, and the
    registration ends with the store."""
    from oracle import oracle as O
    from vllm_fastdecoder_b200 import gpu_ops
    from vllm_fastdecoder_b200.gpu_ops import KVTier

    dev = torch.device("cuda")
    names = ["l0", "l1"]
    spec = _spec(KVH=2, BS=16, D=64)
    state.ensure_store(_vcfg(4), spec, names, pin=True)
    st = state.STORE
    g = torch.Generator().manual_seed(3)
    for nm in names:
        st.k[nm].copy_(torch.randn(st.k[nm].shape, generator=g).to(spec.dtype))
        st.v[nm].copy_(torch.randn(st.v[nm].shape, generator=g).to(spec.dtype))
    assert st.k["l1"].is_pinned()
    n, H = 3, 4
    lens = torch.tensor([37, 0, 150], dtype=torch.int32)
    bt = torch.zeros(n, 12, dtype=torch.int32)
    bt[0, :3] = torch.tensor([4, 9, 6])
    bt[2, :10] = torch.arange(1, 11) + 4  # host blocks 1..10 (ids G + 1 ..)
    q = torch.randn(n, H, 64, generator=g).to(spec.dtype)
    for nm in names:
        out = torch.empty(n, H, 64, dtype=spec.dtype, device=dev)
        lse = torch.empty(H, n, dtype=torch.float32, device=dev)
        tiers = (None, KVTier(st.k[nm], st.v[nm]))
        gpu_ops.decode_tiered(q.to(dev), tiers, 4, bt.to(dev), lens.to(dev), 1 / math.sqrt(64), out, lse)
        gpu_ops.check_device_errors(dev)
        ref = torch.empty(n, H, 64, dtype=spec.dtype)
        ref_l = torch.empty(H, n)
        O.decode_attn_tiered(q, None, (st.k[nm], st.v[nm]), 4, bt, lens, 1 / math.sqrt(64), ref, ref_l)
        assert (out.cpu().float() - ref.float()).abs().max().item() <= 2e-3
        live = lens > 0
        assert (lse.cpu()[:, live] - ref_l[:, live]).abs().max().item() <= 1e-4
    arena = st.arena
    state.STORE = None
    del st
    arena.release()  # explicit release is idempotent with the collector's
    assert not arena._registered
