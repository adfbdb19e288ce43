"""B200 (sm_100a) gated-delta-rule library for the linear-attention layers of a Qwen3.5-style hybrid model.

Drop-in replacements for the gated-delta hot path of PostHog/jeeves: the chunked
prefill, the recurrent decode and block-K verify steps with snapshot rollback, the
causal conv1d + SiLU and the output-gated RMSNorm around them. All compute runs in
hand-written CUDA kernels of ``_lib/libgdn_b200.so`` through its C ABI
(``include/gdn_b200.h``); ``install`` routes the reference's dispatchers to them.
"""

from .gated_delta import (  # noqa: F401
    gated_delta_rule_advance_inplace,
    gated_delta_rule_chunk,
    gated_delta_rule_chunk_gated_norm,
    gated_delta_rule_delta_commit,
    gated_delta_rule_delta_commit_layers,
    gated_delta_rule_rollback,
    gated_delta_rule_step,
    gated_delta_rule_verify,
    gated_delta_rule_verify_deltas,
    gated_delta_rule_verify_deltas_gated_norm,
)
from .conv import causal_conv1d, causal_conv1d_step, conv_state_commit, conv_step, eager_conv_step  # noqa: F401
from .norm import GatedRMSNorm, gated_rms_norm  # noqa: F401
from .gates import delta_gates, gated_delta_rule_chunk_gates, gated_delta_rule_step_gates  # noqa: F401
from .layer import (decode_layer_step, fp8_linear, in_proj_conv, prefill_layer, verify_layer_commit,  # noqa: F401
                    verify_layer_step, verify_layers_commit)
from .attention import decode_attention, rotary, rotate_into_cache  # noqa: F401
from . import fla_inplace  # noqa: F401
from ._lib import load as load_library  # noqa: F401
from .integration import install  # noqa: F401
