"""Worker-process state: the host KV tier (the roles of the reference's
fastdecode/state.py:16-134, in this engine's own design).

The host tier of every layer lives in one host arena, a zero-filled tensor
[layers, 2, C, KVH, BS, D] (the zero fill commits its pages at start-up,
not mid-run) that is registered with CUDA as pinned, device-mapped memory
(fd_host_register: cudaHostRegister, Mapped | Portable).  Registering an
ordinary allocation keeps the tier at its exact size (a pinned-memory
allocator would round each allocation up) and gives one registration and one
device-address translation for all layers.  CpuKVStore.k / .v hold each
layer's K and V views [C, KVH, BS, D] of the arena (the reference's store
layout, fastdecode/state.py:66): the decode kernels read them over PCIe or
stage them into HBM with the copy engine, and the KV-write kernel writes new
rows into them directly.  No data moves through host staging buffers, so
the reference's PinnedStaging has no counterpart here.
"""

from __future__ import annotations

import logging
import time
from dataclasses import dataclass, field

import torch

from vllm_fastdecoder_b200 import config

logger = logging.getLogger("fastdecode")


class HostArena:
    """One host allocation holding the K and V tiers of `layers` layers,
    [layers, 2, C, KVH, BS, D], registered with CUDA (mapped) unless
    `register` is False (CPU-only use).  Every view it hands out keeps it
    alive; when the last one goes (or on release()) it is unregistered
    before the memory returns to the allocator."""

    def __init__(self, layers: int, shape: tuple[int, int, int, int], dtype: torch.dtype, register: bool = True):
        self.shape = (layers, 2) + tuple(shape)
        self.buf = torch.zeros(self.shape, dtype=dtype)
        self.nbytes = self.buf.numel() * self.buf.element_size()
        self._registered = False
        if register and self.nbytes > 0:
            from vllm_fastdecoder_b200 import _native as nat

            nat.check(nat.load().fd_host_register(self.buf.data_ptr(), self.nbytes), "fd_host_register")
            self._registered = True

    def _view(self, layer: int, which: int) -> torch.Tensor:
        t = self.buf[layer, which]
        t._fd_arena = self  # the registration lasts as long as any handed-out view
        return t

    def k(self, layer: int) -> torch.Tensor:
        return self._view(layer, 0)

    def v(self, layer: int) -> torch.Tensor:
        return self._view(layer, 1)

    def release(self) -> None:
        if self._registered:
            from vllm_fastdecoder_b200 import _native as nat
            from vllm_fastdecoder_b200 import gpu_ops

            self._registered = False
            gpu_ops.forget_host_pointer(self.buf)
            nat.check(nat.load().fd_host_unregister(self.buf.data_ptr()), "fd_host_unregister")

    def __del__(self) -> None:
        try:
            self.release()
        except Exception:  # interpreter shutdown: the library may be gone already
            pass


@dataclass
class CpuKVStore:
    num_gpu_blocks: int  # block ids [0, G) live in the HBM KV cache
    num_cpu_blocks: int  # block ids [G, G + C) live here
    block_size: int
    num_kv_heads: int
    head_size: int
    dtype: torch.dtype
    k: dict[str, torch.Tensor] = field(default_factory=dict)  # [C, KVH, BS, D] views, device-mapped
    v: dict[str, torch.Tensor] = field(default_factory=dict)
    steps: int = 0
    arena: HostArena | None = None  # owner of the k / v views (None: tensors the caller provided)

    def serves(self, num_gpu_blocks: int, num_cpu_blocks: int, layer_names: list[str]) -> bool:
        """Whether this store already is the tier these arguments ask for."""
        return (self.num_gpu_blocks == num_gpu_blocks and self.num_cpu_blocks == num_cpu_blocks
                and all(nm in self.k for nm in layer_names))


STORE: CpuKVStore | None = None


def allocate_host_tier(shape, dtype: torch.dtype, pin: bool = True) -> torch.Tensor:
    """A single zero-filled host tensor of `shape`, registered (device-mapped)
    unless `pin` is False; the arena that owns it stays alive with it."""
    return HostArena(1, tuple(shape), dtype, register=pin).k(0)


def _build_store(num_gpu: int, num_cpu: int, spec, layer_names: list[str], pin: bool) -> CpuKVStore:
    t0 = time.time()
    geom = (num_cpu, spec.num_kv_heads, spec.block_size, spec.head_size)
    arena = HostArena(len(layer_names), geom, spec.dtype, register=pin)
    store = CpuKVStore(num_gpu_blocks=int(num_gpu), num_cpu_blocks=int(num_cpu), block_size=spec.block_size,
                       num_kv_heads=spec.num_kv_heads, head_size=spec.head_size, dtype=spec.dtype,
                       k={nm: arena.k(i) for i, nm in enumerate(layer_names)},
                       v={nm: arena.v(i) for i, nm in enumerate(layer_names)}, arena=arena)
    if pin:
        from vllm_fastdecoder_b200 import gpu_ops

        gpu_ops.load_ext()  # a missing library fails here, at start-up
    logger.warning("FastDecode-B200: host KV tier of %d blocks beside %d HBM blocks, %d layers, %.2f GiB in one "
                   "%s host arena (%.1fs); the GPU reads it over PCIe", num_cpu, num_gpu, len(layer_names),
                   arena.nbytes / 2**30, "registered" if pin else "unregistered", time.time() - t0)
    return store


def ensure_store(vllm_config, spec, layer_names: list[str], pin: bool = True) -> None:
    """Create the worker's host tier once the real HBM block count is known
    (the metadata builder calls it on construction, as the reference does,
    fastdecode/backend.py:130-134): before that (vLLM's memory profiling)
    cache_config.num_gpu_blocks is None and nothing happens; a tier that
    already serves the same sizes and layers is kept; a plugin switched off
    or sized to no host blocks leaves no store."""
    global STORE
    if not config.enabled():
        return
    num_gpu = vllm_config.cache_config.num_gpu_blocks
    if num_gpu is None:
        return
    num_cpu = config.resolve_num_cpu_blocks_from_spec(spec, len(layer_names))
    if num_cpu <= 0:
        STORE = None
        return
    if STORE is not None and STORE.serves(num_gpu, num_cpu, layer_names):
        return
    config.validate_spec(spec)
    STORE = None  # the old tier's arena is unregistered once nothing holds its views
    STORE = _build_store(num_gpu, num_cpu, spec, layer_names, pin)
