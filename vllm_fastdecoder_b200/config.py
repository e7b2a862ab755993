"""Environment-driven configuration (same variables as the reference,
fastdecode/config.py:1-81).

FASTDECODE_CPU_BLOCKS   number of KV blocks held in the host tier, or
FASTDECODE_CPU_KV_GB    the same as GiB of host memory (ignored if
                        FASTDECODE_CPU_BLOCKS is set)
FASTDECODE_STATS        "1" logs the per-step class mix every 50 steps
FASTDECODE_CPU_THREADS  accepted for compatibility; no host kernel runs here
FASTDECODE_B200_TWO_PASS "1" computes split decodes as two partials (HBM tier,
                        host tier) merged by the LSE kernel, the reference's
                        structure; default is one pass over both tiers
"""

from __future__ import annotations

import os

ENV_CPU_BLOCKS = "FASTDECODE_CPU_BLOCKS"
ENV_CPU_KV_GB = "FASTDECODE_CPU_KV_GB"
ENV_STATS = "FASTDECODE_STATS"
ENV_TWO_PASS = "FASTDECODE_B200_TWO_PASS"
# decode-only steps are planned on the GPU (fd_plan_step) unless set to 0
ENV_DEVICE_PLAN = "FASTDECODE_B200_DEVICE_PLAN"
# host-planned steps copy their host-tier blocks to HBM with the copy engine
# (when the range they span is dense) unless set to 0
ENV_STAGE_HOST = "FASTDECODE_B200_STAGE_HOST"
# prefill rows (P and F classes) on this engine's tcgen05 kernel instead of
# vLLM's FlashAttention (the reference's choice)
ENV_PREFILL = "FASTDECODE_B200_PREFILL"


def enabled() -> bool:
    return bool(os.environ.get(ENV_CPU_BLOCKS) or os.environ.get(ENV_CPU_KV_GB))


def _flag(name: str) -> bool:
    return os.environ.get(name, "0") not in ("", "0", "false", "False")


def stats_enabled() -> bool:
    return _flag(ENV_STATS)


def two_pass() -> bool:
    return _flag(ENV_TWO_PASS)


def stage_host() -> bool:
    return os.environ.get(ENV_STAGE_HOST, "1") not in ("", "0", "false", "False")


def b200_prefill() -> bool:
    return os.environ.get(ENV_PREFILL, "1") not in ("", "0", "false", "False")


def device_plan() -> bool:
    return os.environ.get(ENV_DEVICE_PLAN, "1") not in ("", "0", "false", "False") and not two_pass()


def kv_bytes_per_block(kv_cache_config) -> int:
    """Bytes one KV block occupies across all layers (K and V)."""
    return sum(g.kv_cache_spec.page_size_bytes * len(g.layer_names) for g in kv_cache_config.kv_cache_groups)


def _resolve(per_block_bytes: int) -> int:
    blocks = os.environ.get(ENV_CPU_BLOCKS)
    if blocks:
        return max(0, int(blocks))
    gb = os.environ.get(ENV_CPU_KV_GB)
    if gb:
        return max(0, int(float(gb) * (1 << 30)) // per_block_bytes)
    return 0


def resolve_num_cpu_blocks(kv_cache_config) -> int:
    """Engine-core side (sees the whole KV-cache config)."""
    return _resolve(kv_bytes_per_block(kv_cache_config))


def resolve_num_cpu_blocks_from_spec(spec, num_layers: int) -> int:
    """Worker side (one group's spec and its layer count); agrees with
    resolve_num_cpu_blocks for single-group models."""
    return _resolve(spec.page_size_bytes * num_layers)


def validate_kv_cache_config(kv_cache_config) -> None:
    groups = kv_cache_config.kv_cache_groups
    if len(groups) != 1:
        raise NotImplementedError(
            f"FastDecode supports models with a single KV cache group, got {len(groups)} "
            "(hybrid / sliding-window / MLA models are out of scope)."
        )
    validate_spec(groups[0].kv_cache_spec)


def validate_spec(spec) -> None:
    """Full attention, unquantised KV, head_size_v == head_size."""
    if getattr(spec, "sliding_window", None) is not None:
        raise NotImplementedError(f"FastDecode needs full attention, got {type(spec).__name__}")
    mode = getattr(spec, "kv_quant_mode", None)
    if mode is not None and getattr(mode, "name", str(mode)) not in ("NONE", "None"):
        raise NotImplementedError("FastDecode does not support quantized KV cache")
    if getattr(spec, "head_size_v", spec.head_size) != spec.head_size:
        raise NotImplementedError("FastDecode needs head_size_v == head_size")
