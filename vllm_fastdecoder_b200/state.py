"""Worker-process state: the host KV tier (same roles as the reference's
fastdecode/state.py:16-134).

The host tier of every layer is a pair of K/V tensors [C, KVH, BS, D] in
pinned host memory, which CUDA maps into the device address space; the decode
kernel reads it over PCIe and the KV-write kernel writes new rows into it
directly, so no staging buffers or host-side kernels are involved.  The tensors
are zero-filled at creation so their pages are committed up front.
"""

from __future__ import annotations

import logging
import time
from dataclasses import dataclass, field

import torch

from vllm_fastdecoder_b200 import config

logger = logging.getLogger("fastdecode")


@dataclass
class CpuKVStore:
    num_gpu_blocks: int  # block ids [0, G) live in the HBM KV cache
    num_cpu_blocks: int  # block ids [G, G + C) live here
    block_size: int
    num_kv_heads: int
    head_size: int
    dtype: torch.dtype
    k: dict[str, torch.Tensor] = field(default_factory=dict)  # [C, KVH, BS, D], pinned
    v: dict[str, torch.Tensor] = field(default_factory=dict)
    steps: int = 0


STORE: CpuKVStore | None = None


def allocate_host_tier(shape, dtype: torch.dtype, pin: bool = True) -> torch.Tensor:
    """Zero-filled host tensor; pinned (and therefore device-mapped) unless
    `pin` is False (CPU-only unit tests)."""
    t = torch.zeros(shape, dtype=dtype, pin_memory=pin)
    return t


def ensure_store(vllm_config, spec, layer_names: list[str], pin: bool = True) -> None:
    """Create the host tier in the worker (idempotent), as the reference's
    ensure_store (state.py:32-90): builders created before the real GPU block
    count is known (memory profiling) see None and do nothing."""
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
    if (STORE is not None and STORE.num_gpu_blocks == num_gpu and STORE.num_cpu_blocks == num_cpu
            and all(n in STORE.k for n in layer_names)):
        return
    config.validate_spec(spec)
    store = CpuKVStore(num_gpu_blocks=int(num_gpu), num_cpu_blocks=num_cpu, block_size=spec.block_size,
                       num_kv_heads=spec.num_kv_heads, head_size=spec.head_size, dtype=spec.dtype)
    shape = (num_cpu, spec.num_kv_heads, spec.block_size, spec.head_size)
    t0 = time.time()
    for name in layer_names:
        store.k[name] = allocate_host_tier(shape, spec.dtype, pin)
        store.v[name] = allocate_host_tier(shape, spec.dtype, pin)
    elem = torch.empty((), dtype=spec.dtype).element_size()
    gib = 2 * len(layer_names) * torch.Size(shape).numel() * elem / (1 << 30)
    if pin:
        from vllm_fastdecoder_b200 import gpu_ops

        gpu_ops.load_ext()  # fail at startup, not mid-run, if the library is missing
    logger.warning(
        "FastDecode-B200: %d HBM blocks + %d host blocks (block_size=%d, %.1f GiB pinned host KV for %d "
        "layers, allocated in %.1fs); host tier read by the GPU over PCIe",
        store.num_gpu_blocks, num_cpu, spec.block_size, gib, len(layer_names), time.time() - t0,
    )
    STORE = store


class PinnedStaging:
    """Grow-only pinned buffers (the reference's PinnedStaging,
    state.py:93-124).  Kept for API compatibility; this engine's split path
    moves no data through the host."""

    def __init__(self, pin: bool = True) -> None:
        self._bufs: dict[str, torch.Tensor] = {}
        self._pin = pin

    def get(self, name: str, shape: tuple[int, ...], dtype: torch.dtype) -> torch.Tensor:
        numel = 1
        for s in shape:
            numel *= s
        buf = self._bufs.get(name)
        if buf is None or buf.dtype != dtype or buf.numel() < numel:
            cap = max(numel, 1, 2 * (buf.numel() if buf is not None else 0))
            buf = torch.empty(cap, dtype=dtype, pin_memory=self._pin)
            self._bufs[name] = buf
        return buf[:numel].view(shape)


_STAGING: PinnedStaging | None = None


def staging() -> PinnedStaging:
    global _STAGING
    if _STAGING is None:
        _STAGING = PinnedStaging()
    return _STAGING
