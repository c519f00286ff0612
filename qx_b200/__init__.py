"""qx_b200 — B200 (sm_100a) implementation of qx's grouped-query-attention
hot path behind a C ABI (include/qxcuda.h, libqxcuda.so).

The host API mirrors blasrodri/qx's KvCache / granite_attention_decode /
ExecutionPlan interfaces; all computation runs in hand-written CUDA kernels.
"""
from .runtime import (  # noqa: F401
    BF16, F16, F32, HASH_AUTO, HASH_PER_CHUNK, HASH_PER_SLOT, MODEL_GRANITE, MODEL_QWEN3, Context, PeerGroup, ExecutionPlan, KvArena, KvCache, KvPrecision, Q4Weights,
    QxError, apply_granite_rope, default_context, granite_attention_decode, q4_mat_vec,
)
