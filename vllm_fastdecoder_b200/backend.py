"""vLLM attention backend "CUSTOM" with an HBM + host KV tier, B200 kernels.

Same classes, class attributes and method signatures as the reference
plugin's backend (fastdecode/backend.py:67-357):

  FastDecodeBackend          get_name() == "CUSTOM", forward_includes_kv_cache_update
  FastDecodeMetadataBuilder  build() attaches fd_plan / fd_num_reqs / fd_seq_cpu
  FastDecodeImpl             forward(layer, query, key, value, kv_cache,
                             attn_metadata, output, ...) -> output

and the same OPS indirection that tests swap for CPU stand-ins.  A step in
which no request touches the host tier runs the stock FlashAttention path,
like the reference.  Otherwise every layer does, all on the GPU's stream:

  1. one tier-aware KV write: each new K/V row goes to its HBM slot or, over
     PCIe, to its slot in the pinned host tier (fd_store_kv)
  2. split decodes (S) in one pass of the split-KV kernel over each row's
     whole block table, HBM blocks via TMA and host blocks over PCIe, written
     straight into their output rows (fd_decode_attn); with
     FASTDECODE_B200_TWO_PASS=1 the reference's structure instead: an HBM
     partial, a host partial and the LSE merge (fd_merge_attn_states)
  3. all-HBM decodes (P rows with one query token) through the same kernel
  4. prefills (P rows with several query tokens, fresh F prefills) through
     vLLM's FlashAttention, as in the reference (outside the decode engine)

vLLM is optional at import time: without it the classes still import (for the
planner and the kernels' own tests) but cannot be instantiated by an engine.
"""

from __future__ import annotations

import logging
import os

import torch

from vllm_fastdecoder_b200 import config, state
from vllm_fastdecoder_b200.plan import DeviceDecodeStep, DevicePlan, build_host_plan, plan_on_device, to_device

logger = logging.getLogger("fastdecode")

_HAVE_VLLM = False
if os.environ.get("FASTDECODE_B200_NO_VLLM", "0") in ("", "0"):
    try:
        from vllm.v1.attention.backend import AttentionCGSupport, AttentionType
        from vllm.v1.attention.backends import flash_attn as _fa
        from vllm.v1.attention.backends.flash_attn import (
            FlashAttentionBackend,
            FlashAttentionImpl,
            FlashAttentionMetadataBuilder,
        )

        _HAVE_VLLM = True
    except Exception:  # pragma: no cover - depends on the installed vLLM
        _HAVE_VLLM = False

if not _HAVE_VLLM:
    import enum

    class AttentionCGSupport(enum.Enum):  # type: ignore[no-redef]
        NEVER = 0

    class AttentionType:  # type: ignore[no-redef]
        DECODER = "decoder"

    class FlashAttentionBackend:  # type: ignore[no-redef]
        pass

    class FlashAttentionImpl:  # type: ignore[no-redef]
        def __init__(self, *args, **kwargs):
            raise RuntimeError("FastDecode-B200: vLLM is not importable; the backend needs it")

    class FlashAttentionMetadataBuilder:  # type: ignore[no-redef]
        def __init__(self, *args, **kwargs):
            raise RuntimeError("FastDecode-B200: vLLM is not importable; the backend needs it")

    _fa = None


class _GpuOps:
    """Device primitives of the split path (tests swap in CPU stand-ins)."""

    @staticmethod
    def tier(k: torch.Tensor, v: torch.Tensor):
        from vllm_fastdecoder_b200.gpu_ops import KVTier

        return KVTier(k, v)

    @staticmethod
    def store_kv(key, value, slots, tiers, tier_split):
        from vllm_fastdecoder_b200 import gpu_ops

        gpu_ops.store_kv_tiered(key, value, slots, tiers, tier_split)

    @staticmethod
    def decode(query, tiers, tier_split, block_table, lens, scale, out, lse=None, **kw):
        from vllm_fastdecoder_b200 import gpu_ops

        gpu_ops.decode_tiered(query, tiers, tier_split, block_table, lens, scale, out, lse, **kw)

    @staticmethod
    def merge(out, o_a, lse_a, o_b, lse_b, out_rows=None):
        from vllm_fastdecoder_b200 import gpu_ops

        gpu_ops.merge_attn_states(out, o_a, lse_a, o_b, lse_b, out_rows=out_rows)

    @staticmethod
    def prefill(query, out, q_start, q_len, k_len, scale, kv=None, block_table=None, k=None, v=None, total_q=None):
        from vllm_fastdecoder_b200 import gpu_ops

        gpu_ops.prefill_attn(query, out, q_start, q_len, k_len, scale, kv=kv, block_table=block_table, k=k, v=v,
                             total_q=total_q)

    @staticmethod
    def fa(**kw):
        return _fa.flash_attn_varlen_func(**kw)


OPS = _GpuOps


class FastDecodeBackend(FlashAttentionBackend):
    supported_kv_cache_dtypes = ["auto", "float16", "bfloat16"]
    # host-tier K/V are written from inside forward(), which runs eagerly
    forward_includes_kv_cache_update: bool = True

    @staticmethod
    def get_name() -> str:
        return "CUSTOM"

    @staticmethod
    def get_impl_cls() -> type["FastDecodeImpl"]:
        return FastDecodeImpl

    @staticmethod
    def get_builder_cls() -> type["FastDecodeMetadataBuilder"]:
        return FastDecodeMetadataBuilder

    @classmethod
    def supports_attn_type(cls, attn_type: str) -> bool:
        return attn_type == AttentionType.DECODER

    @classmethod
    def supports_sliding_window(cls) -> bool:
        return False

    @classmethod
    def supports_rswa(cls) -> bool:
        return False

    @classmethod
    def supports_mm_prefix(cls) -> bool:
        return False

    @classmethod
    def supports_sink(cls) -> bool:
        return False

    @classmethod
    def supports_non_causal(cls) -> bool:
        return False

    @classmethod
    def supports_batch_invariance(cls) -> bool:
        return False

    @classmethod
    def supports_kv_connector(cls) -> bool:
        return False


class FastDecodeMetadataBuilder(FlashAttentionMetadataBuilder):
    # the per-step plan needs the block table on the host (one D2H copy per
    # step), so the attention step is not captured in a CUDA graph
    _cudagraph_support = AttentionCGSupport.NEVER
    supports_update_block_table: bool = False
    supports_draft_decode_metadata_update: bool = False

    @classmethod
    def get_cudagraph_support(cls, vllm_config, kv_cache_spec):
        return AttentionCGSupport.NEVER

    def __init__(self, kv_cache_spec, layer_names, vllm_config, device):
        super().__init__(kv_cache_spec, layer_names, vllm_config, device)
        self.supports_draft_decode_metadata_update = False
        state.ensure_store(vllm_config, kv_cache_spec, layer_names)
        self._acc = [0, 0, 0, 0, 0]  # steps, P reqs, S reqs, F reqs, host tokens

    def use_cascade_attention(self, *args, **kwargs) -> bool:
        return False

    def build(self, common_prefix_len, common_attn_metadata, fast_build: bool = False):
        cm = common_attn_metadata
        md = super().build(0, cm, fast_build)
        md.fd_plan = None
        md.fd_dplan = None
        md.fd_num_reqs = cm.num_reqs
        md.fd_seq_cpu = None
        store = state.STORE
        if store is None:
            return md
        if getattr(self, "kernel_block_size", None) not in (None, store.block_size):
            raise NotImplementedError(
                "FastDecode needs kernel block size == KV block size "
                f"({self.kernel_block_size} vs {store.block_size})")
        bs = store.block_size
        R = cm.num_reqs
        if R == 0:
            return md
        qsl = cm.query_start_loc_cpu[: R + 1]
        upper = getattr(cm, "seq_lens_cpu_upper_bound", None)
        if (config.device_plan() and upper is not None and cm.block_table_tensor.is_cuda
                and bool(((qsl[1:] - qsl[:-1]) <= 1).all())):
            # a decode-only step: planned on the GPU from the device tensors,
            # no block-table or slot copy to the host (fd_plan_step)
            md.fd_dplan = self._device_plan(cm, R, int(qsl[-1]), int(upper[:R].max()), store)
            return md
        seq = upper[:R] if upper is not None else cm.seq_lens[:R].cpu()
        width = max(1, min(int((int(seq.max()) + bs - 1) // bs), cm.block_table_tensor.shape[1]))
        bt_dev = cm.block_table_tensor[:R]
        n_tok = int(qsl[-1])
        bt = bt_dev[:, :width].cpu()  # the step's one device-to-host copy
        slots = cm.slot_mapping[:n_tok].cpu()
        md.fd_seq_cpu = seq
        hp = build_host_plan(qsl, seq, bt, slots, store.num_gpu_blocks, store.num_cpu_blocks, bs)
        if hp is not None:
            md.fd_plan = to_device(hp, bt_dev[:, :width], self.device)
        if config.stats_enabled():
            self._log_stats(hp, R)
        return md

    def _device_plan(self, cm, R: int, n_tok: int, max_seq: int, store):
        """fd_plan_step over the step's device tensors; the plan buffers are
        kept and reused while they fit."""
        bt = cm.block_table_tensor[:R]
        if bt.stride(1) != 1:
            bt = bt.contiguous()
        qsl = cm.query_start_loc[: R + 1]
        seq = cm.seq_lens[:R]
        if qsl.dtype != torch.int32:
            qsl = qsl.to(torch.int32)
        if seq.dtype != torch.int32:
            seq = seq.to(torch.int32)
        buf = getattr(self, "_dplan_buf", None)
        dp = plan_on_device(qsl, seq, bt, cm.slot_mapping, store.num_gpu_blocks, store.num_cpu_blocks,
                            store.block_size, out=buf, max_tokens=n_tok)
        self._dplan_buf = dp
        return DeviceDecodeStep(dp, R, n_tok, max_seq)

    def _log_stats(self, hp, num_reqs) -> None:
        a = self._acc
        a[0] += 1
        if hp is None:
            a[1] += num_reqs
        else:
            a[1] += int(hp.p_req.numel())
            a[2] += hp.n_s
            a[3] += int(hp.f_cu.numel()) - 1
            a[4] += int(hp.s_cpu_lens.sum())
        if a[0] % 50 == 0:
            logger.warning(
                "FastDecode stats (last 50 steps): avg reqs/step all-GPU=%.1f split-decode=%.1f "
                "fresh-prefill-on-CPU=%.1f, avg host KV tokens read per layer per step=%.0f",
                a[1] / 50, a[2] / 50, a[3] / 50, a[4] / 50)
            self._acc = [a[0], 0, 0, 0, 0]


class FastDecodeImpl(FlashAttentionImpl):
    supports_dcp: bool = False

    def __init__(self, *args, **kwargs) -> None:
        super().__init__(*args, **kwargs)
        if self.alibi_slopes is not None:
            raise NotImplementedError("FastDecode: ALiBi is not supported")
        if tuple(self.sliding_window) != (-1, -1):
            raise NotImplementedError("FastDecode: sliding window is not supported")
        if getattr(self, "sinks", None) is not None:
            raise NotImplementedError("FastDecode: attention sinks are not supported")
        if str(self.kv_cache_dtype).startswith("fp8"):
            raise NotImplementedError("FastDecode: quantized KV cache is not supported")
        if getattr(self, "dcp_world_size", 1) > 1:
            raise NotImplementedError("FastDecode: DCP is not supported")
        if self.logits_soft_cap:
            raise NotImplementedError("FastDecode: logits soft-capping is not supported")

    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output, output_scale=None,
                output_block_scale=None):
        if output_scale is not None or output_block_scale is not None:
            raise NotImplementedError("FastDecode: fused output quantization")
        if attn_metadata is None:  # profiling run
            return output.fill_(0)
        dstep = getattr(attn_metadata, "fd_dplan", None)
        if dstep is not None:
            return self._forward_device(layer, query, key, value, kv_cache, dstep, attn_metadata.slot_mapping, output)
        plan = getattr(attn_metadata, "fd_plan", None)
        if plan is None:
            if self.kv_sharing_target_layer_name is None and key is not None:
                FlashAttentionImpl.do_kv_cache_update(self, layer, key, value, kv_cache,
                                                      attn_metadata.slot_mapping)
            return super().forward(layer, query, key, value, kv_cache, attn_metadata, output)
        return self._forward_split(layer, query, key, value, kv_cache, plan, output)

    def _forward_device(self, layer, query, key, value, kv_cache, ds: "DeviceDecodeStep", slot_mapping, output):
        """A decode-only step planned on the GPU: one tier-aware KV write of
        the step's tokens and one decode launch over the planner's decode
        list (every request, whichever tiers its blocks are in), all inputs
        on the device.  Replaces the reference's split path for such steps
        (fastdecode/backend.py:257-357)."""
        store = state.STORE
        assert store is not None
        D = self.head_size
        G = store.num_gpu_blocks
        hbm = OPS.tier(kv_cache[..., :D], kv_cache[..., D:])
        host = OPS.tier(store.k[layer.layer_name], store.v[layer.layer_name])
        tiers = (hbm, host)
        if self.kv_sharing_target_layer_name is None and ds.n_tok:
            OPS.store_kv(key[: ds.n_tok], value[: ds.n_tok], slot_mapping[: ds.n_tok], tiers, G)
        dp = ds.plan
        OPS.decode(query, tiers, G, dp.block_table, dp.d_lens, self.scale, output, q_rows=dp.d_tok,
                   out_rows=dp.d_tok, bt_rows=dp.d_row, n=ds.num_reqs, max_len=ds.max_seq)
        return output

    def _forward_split(self, layer, query, key, value, kv_cache, dp: DevicePlan, output):
        hp = dp.host
        store = state.STORE
        assert store is not None
        H, D = self.num_heads, self.head_size
        G = store.num_gpu_blocks
        # vLLM's logical cache is [B, KVH, BS, 2D] (K then V per head row)
        hbm = OPS.tier(kv_cache[..., :D], kv_cache[..., D:])  # [B, KVH, BS, D] views
        key_cache, value_cache = kv_cache.transpose(1, 2).split(D, dim=-1)  # FlashAttention's [B, BS, KVH, D]
        host = OPS.tier(store.k[layer.layer_name], store.v[layer.layer_name])
        tiers = (hbm, host)

        # 1) new K/V into whichever tier owns each slot
        if self.kv_sharing_target_layer_name is None and hp.n_tok:
            OPS.store_kv(key[: hp.n_tok], value[: hp.n_tok], dp.slot_mapping, tiers, G)

        # 2) split decodes
        if hp.n_s:
            if config.two_pass():
                self._split_two_pass(query, tiers, G, dp, output)
            else:
                # a dense range of host blocks is staged into HBM by the copy
                # engine (faster than SM loads over PCIe), a sparse one read in place
                span = hp.host_hi - hp.host_lo
                hr = ((hp.host_lo, hp.host_hi)
                      if config.stage_host() and span > 0 and hp.host_used >= 0.6 * span else None)
                OPS.decode(query, tiers, G, dp.s_bt, dp.s_seq_lens, self.scale, output,
                           q_rows=dp.s_tok, out_rows=dp.s_tok, max_len=hp.s_max_len, host_range=hr)

        # 3) all-HBM decodes
        if hp.pd_req.numel():
            OPS.decode(query, (hbm, None), G, dp.pd_bt, dp.pd_seq_lens, self.scale, output,
                       q_rows=dp.pd_tok, out_rows=dp.pd_tok, max_len=hp.pd_max_len)

        # 4) prefills: this engine's tcgen05 kernel, written straight into the
        # requests' output rows (FASTDECODE_B200_PREFILL=0: FlashAttention,
        # as in the reference)
        if self._prefill_on_b200(query):
            if hp.pp_req.numel():
                cu = dp.pp_cu
                OPS.prefill(query, output, dp.pp_tok.index_select(0, cu[:-1].long()).to(torch.int32),
                            (cu[1:] - cu[:-1]).to(torch.int32), dp.pp_seqlens, self.scale, kv=hbm,
                            block_table=dp.pp_bt, total_q=int(hp.pp_tok.numel()))
            if hp.n_f_tok:
                cu = dp.f_cu
                q_len = (cu[1:] - cu[:-1]).to(torch.int32)
                OPS.prefill(query, output, dp.f_tok.index_select(0, cu[:-1].long()).to(torch.int32), q_len, q_len,
                            self.scale, k=key, v=value, total_q=int(hp.n_f_tok))
            return output
        if hp.pp_req.numel():
            q_p = query.index_select(0, dp.pp_tok)
            o_p = OPS.fa(q=q_p, k=key_cache, v=value_cache, cu_seqlens_q=dp.pp_cu, max_seqlen_q=hp.pp_max_q,
                         seqused_k=dp.pp_seqlens, max_seqlen_k=hp.pp_max_k, softmax_scale=self.scale,
                         causal=True, block_table=dp.pp_bt, softcap=self.logits_soft_cap,
                         fa_version=self.vllm_flash_attn_version)
            output.index_copy_(0, dp.pp_tok, o_p)
        if hp.n_f_tok:
            q_f = query.index_select(0, dp.f_tok)
            k_f = key.index_select(0, dp.f_tok)
            v_f = value.index_select(0, dp.f_tok)
            o_f = OPS.fa(q=q_f, k=k_f, v=v_f, cu_seqlens_q=dp.f_cu, cu_seqlens_k=dp.f_cu, max_seqlen_q=hp.f_max,
                         max_seqlen_k=hp.f_max, softmax_scale=self.scale, causal=True,
                         softcap=self.logits_soft_cap, fa_version=self.vllm_flash_attn_version)
            output.index_copy_(0, dp.f_tok, o_f)
        return output

    def _prefill_on_b200(self, query) -> bool:
        """Whether this layer's prefill rows run on fd_prefill_attn: enabled
        (FASTDECODE_B200_PREFILL), fp16 / bf16, head size 128, a query group
        dividing 128, no soft cap; otherwise FlashAttention, as in the
        reference."""
        G = self.num_heads // max(1, self.num_kv_heads)
        return (config.b200_prefill() and query.dtype in (torch.float16, torch.bfloat16) and self.head_size == 128
                and not self.logits_soft_cap and G <= 16 and 128 % G == 0)

    def _split_two_pass(self, query, tiers, G, dp: DevicePlan, output):
        """The reference's structure (backend.py:293-356): an HBM partial over
        the compacted HBM table, a host partial over the compacted host table,
        merged by log-sum-exp into the output rows."""
        hp = dp.host
        ns, H, D = hp.n_s, self.num_heads, self.head_size
        dev = query.device
        o_gpu = torch.zeros(ns, H, D, dtype=query.dtype, device=dev)
        lse_gpu = torch.full((H, ns), float("-inf"), dtype=torch.float32, device=dev)
        lse_g = torch.empty(H, ns, dtype=torch.float32, device=dev)
        # rows without HBM tokens get len 0 -> (o = 0, lse = -inf)
        gpu_lens = torch.zeros(ns, dtype=torch.int32, device=dev)
        gpu_lens.index_copy_(0, dp.s_gpu_rows, dp.s_gpu_lens)
        gpu_bt = torch.zeros(ns, dp.s_gpu_bt.shape[1], dtype=torch.int32, device=dev)
        gpu_bt.index_copy_(0, dp.s_gpu_rows, dp.s_gpu_bt)
        OPS.decode(query, (tiers[0], None), G, gpu_bt, gpu_lens, self.scale, o_gpu, lse_g, q_rows=dp.s_tok,
                   max_len=hp.s_max_gpu_len)
        lse_gpu.copy_(lse_g)
        o_cpu = torch.empty(ns, H, D, dtype=query.dtype, device=dev)
        lse_cpu = torch.empty(H, ns, dtype=torch.float32, device=dev)
        # host-relative ids: everything >= tier_split 0 resolves to the host tier
        OPS.decode(query, (None, tiers[1]), 0, dp.s_cpu_bt, dp.s_cpu_lens, self.scale, o_cpu, lse_cpu,
                   q_rows=dp.s_tok, max_len=int(hp.s_cpu_lens.max()) if ns else 0)
        OPS.merge(output, o_gpu, lse_gpu, o_cpu, lse_cpu, out_rows=dp.s_tok)
