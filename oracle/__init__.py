"""CPU oracle for the GDN linear-attention and normalisation hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product (``torch_npu_ops_b200``)
imports this package.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may call it, and
there only as the checker or the timed CPU baseline, never as the thing that
is measured or shipped.

Every function is a plain fp32 torch-on-CPU restatement of the reference's
own torch-native implementation of the op (the functions the reference's
pytest files compare their NPU kernels against), written out again from the
maths and citing the reference file:line it follows.  Paths in the citations
are relative to the reference project root (``triton_npu/...``,
``ascendc_npu/...``).

Pinning: ``tests/golden/make_golden.py`` imports the reference's own torch
references (in the build container only) and writes seeded input/output
fixtures to ``tests/golden/*.pt``; ``tests/test_oracle_golden.py`` checks this
oracle against every fixture.  Two ops have no reference implementation to
pin against and are marked "parity unpinned" in their docstrings:
``gemma_rms_norm`` (a closed CANN op) and the partial (rotary_dim < head_dim)
NeoX RoPE of ``split_rmsnorm_rope``.
"""

from ._out import fp32_outputs  # noqa: F401
from .norms import layer_norm_fwd, gemma_rms_norm, l2norm_last_dim  # noqa: F401
from .rope import split_rmsnorm_rope, rope_inplace  # noqa: F401
from .conv1d import (  # noqa: F401
    causal_conv1d_update, causal_conv1d_varlen, causal_conv1d_update_v2_slots)
from .gdn import (  # noqa: F401
    chunk_local_cumsum,
    chunk_scaled_dot_kkt_fwd,
    solve_tril,
    recompute_w_u_fwd,
    chunk_gated_delta_rule_fwd_h,
    chunk_fwd_o,
    chunk_gated_delta_rule,
    fused_recurrent_gated_delta_rule,
    fused_gdn_gating,
    fused_sigmoid_gating_delta_rule_update,
    fused_qkvzba_split_reshape_cat,
    prepare_chunk_offsets,
)
