"""dcc_kv_b200 -- B200-native (sm_100a) DCC-KV compact-KV path.

Drop-in for the reference package ``src.dcc_kv_ref`` (lfei7199-star/dcc-kv)
plus its distributed layer: the same public names, arguments and errors,
computed by hand-written CUDA kernels in ``libdcckv.so`` (C ABI in
``include/dcc_kv.h``).  There is no CPU fallback: CUDA tensors in, CUDA
tensors out.
"""
from .online_softmax import (
    OnlineSoftmaxState,
    attention_output_from_state,
    merge_lse,
    merge_softmax_states,
    merge_softmax_states_list,
    online_softmax_from_attention,
    verify_order_invariance,
)
from .representative_query import (
    farthest_point_sampling,
    rademacher_projection,
    select_representative_queries,
)
from .key_selection import rms_per_token_score, select_topk_keys
from .calibration import fit_logit_bias, nonneg_least_squares
from .value_regression import fit_compact_value, ridge_regression_value
from .compact_kv import CompactKV, build_compact_kv, build_compact_kv_batched
from .attention import attention
from .layer import DccKvSyncLayer

__all__ = [
    "OnlineSoftmaxState", "online_softmax_from_attention", "merge_softmax_states",
    "merge_softmax_states_list", "verify_order_invariance", "attention_output_from_state", "merge_lse",
    "farthest_point_sampling", "rademacher_projection", "select_representative_queries",
    "rms_per_token_score", "select_topk_keys",
    "nonneg_least_squares", "fit_logit_bias",
    "ridge_regression_value", "fit_compact_value",
    "CompactKV", "build_compact_kv", "build_compact_kv_batched",
    "attention", "DccKvSyncLayer",
]
