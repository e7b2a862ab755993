"""B200-native paged decode attention behind the vLLM fastdecode plugin API.

Block ids below G live in HBM, ids at or above G in pinned, device-mapped
host memory; one split-KV sm_100a kernel walks each row's block table across
both tiers.  See gpu_ops (operator front end), plan (per-step plan), state
(tier storage), backend (Backend / MetadataBuilder / Impl) and sharded
(KV-sharded long context over NCCL).
"""

__version__ = "0.1.0"

BACKEND_CLASS = "vllm_fastdecoder_b200.backend.FastDecodeBackend"
