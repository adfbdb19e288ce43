"""CPU oracle for the gated-delta-rule hot path.

TEST INFRASTRUCTURE ONLY. This package is the checker that the CUDA kernels of
``jeeves_b200`` are compared against; nothing in the product imports it. Only
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py``
may use it.

Every function restates, in plain fp32 PyTorch on the CPU, one operation of the
reference's eager (non-Triton) path in ``model/model.py`` of PostHog/jeeves; each
docstring cites the reference lines it follows. The restatement is pinned against
golden vectors produced by the reference's own functions (see
``tests/golden/make_golden.py`` and ``tests/test_oracle.py``).
"""

from .gdn import (  # noqa: F401
    l2norm,
    recurrent_gated_delta_rule,
    chunk_gated_delta_rule,
    chunk_gated_delta_rule_varlen,
    advance_gated_delta_rule,
    verify_with_snapshots,
    exact_recurrence_f64,
)
from .wrappers import (  # noqa: F401
    causal_conv1d,
    causal_conv1d_step,
    conv_step,
    gated_rms_norm,
    delta_gates,
    apply_rotary,
    rotate_into_cache,
    decode_attention_f32,
)
