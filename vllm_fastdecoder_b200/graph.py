"""CUDA-graph capture of a decode-only step.

A decode-only step needs nothing from the host once the device planner has
run (fd_plan_step: plan and decode list on the GPU), so the whole step over
L layers — the planner, then per layer the tier-aware KV write and one
decode launch over the decode list — is captured once into a CUDA graph and
replayed every step: the step's inputs are written into persistent device
buffers, and replaying costs one graph launch instead of ~3·L + 1 kernel
launches with their host work (argument packing, tensor-map encoding).

The host tier is read in place over PCIe by the decode kernels, alongside
the HBM tiles of the same launch, so there is no staging copy to overlap.
"""

from __future__ import annotations

import torch

from vllm_fastdecoder_b200 import gpu_ops, plan
from vllm_fastdecoder_b200.gpu_ops import KVTier


class DecodeStepGraph:
    """A captured decode step of `layers` layers for up to R requests (one
    query token each, so T = R tokens) and block tables of width W.

    Inputs (write the step's values, then replay()): query_start_loc [R+1],
    seq_lens [R], block_table [R, W] (int32), slot_mapping [R] (int64,
    unified slots, -1 to skip), q [L, R, H, D], k / v [L, R, KVH, D].
    Output: out [L, R, H, D] (rows of requests without a query token are
    left as they were).  tiers[l] = (HBM tier, host tier) of layer l;
    tier_split = G; max_len bounds every sequence length of the steps the
    graph will replay (it sizes the persistent schedule)."""

    def __init__(self, layers: int, R: int, W: int, H: int, KVH: int, D: int, dtype: torch.dtype,
                 tiers: list[tuple[KVTier | None, KVTier | None]], tier_split: int, num_cpu_blocks: int,
                 block_size: int, scale: float, max_len: int, device: torch.device):
        self.L, self.R, self.W = layers, R, W
        self.tiers, self.G, self.C, self.BS = tiers, int(tier_split), int(num_cpu_blocks), int(block_size)
        self.scale, self.max_len, self.device = float(scale), int(max_len), device
        i32 = dict(dtype=torch.int32, device=device)
        self.query_start_loc = torch.arange(R + 1, **i32)
        self.seq_lens = torch.zeros(R, **i32)
        self.block_table = torch.zeros(R, W, **i32)
        self.slot_mapping = torch.full((R,), -1, dtype=torch.int64, device=device)
        self.q = torch.zeros(layers, R, H, D, dtype=dtype, device=device)
        self.k = torch.zeros(layers, R, KVH, D, dtype=dtype, device=device)
        self.v = torch.zeros(layers, R, KVH, D, dtype=dtype, device=device)
        self.out = torch.zeros(layers, R, H, D, dtype=dtype, device=device)
        self.lse = torch.zeros(layers, H, R, dtype=torch.float32, device=device)
        self.plan = plan.DeviceStepPlan(R, R, W, device)
        self.workspace: torch.Tensor | None = None
        self.graph: torch.cuda.CUDAGraph | None = None

    def _launch(self) -> None:
        dp = plan.plan_on_device(self.query_start_loc, self.seq_lens, self.block_table, self.slot_mapping,
                                 self.G, self.C, self.BS, out=self.plan, max_tokens=self.R)
        for l in range(self.L):
            gpu_ops.store_kv_tiered(self.k[l], self.v[l], self.slot_mapping, self.tiers[l], self.G)
            a = gpu_ops.decode_args(self.q[l], self.tiers[l], self.G, self.block_table, dp.d_lens, self.scale,
                                    self.out[l], self.lse[l], q_rows=dp.d_tok, out_rows=dp.d_tok,
                                    bt_rows=dp.d_row, n=self.R, max_len=self.max_len,
                                    workspace_buf=self.workspace)
            gpu_ops.launch_decode(a, self.device)

    def _size_workspace(self) -> None:
        import ctypes

        from vllm_fastdecoder_b200 import _native as nat

        a = gpu_ops.decode_args(self.q[0], self.tiers[0], self.G, self.block_table, self.plan.d_lens, self.scale,
                                self.out[0], self.lse[0], q_rows=self.plan.d_tok, out_rows=self.plan.d_tok,
                                bt_rows=self.plan.d_row, n=self.R, max_len=self.max_len,
                                workspace_buf=None)
        need = int(nat.load().fd_decode_workspace_size(ctypes.byref(a)))
        self.workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=self.device)

    def run_eager(self) -> None:
        """The same launches without a graph (on the current stream)."""
        if self.workspace is None:
            self._size_workspace()
        self._launch()

    def capture(self) -> None:
        """Capture the step (after one eager run that loads the library,
        sets kernel attributes and sizes the dedicated workspace)."""
        self.run_eager()
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._launch()

    def replay(self) -> None:
        assert self.graph is not None, "capture() first"
        self.graph.replay()
