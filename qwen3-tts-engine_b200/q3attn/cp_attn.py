"""Drop-in for engine/cp_attn.py: ``cp_attn(q, K, V, n_live, scale) -> o [B, 2048]`` (engine/cp_attn.py:33-39).

Same contract as the reference wrapper: q [B,16,128] (or [B,2048]); K/V [B,8,16,128] whose batch stride may exceed the
live batch; n_live = p + 1 slots attended; fp32 scores/softmax, probabilities rounded to bf16, fp32 P.V, bf16 output.
``cp_step`` additionally writes the step's K/V into slot p first (engine/code_predictor.py:58) in the same launch.
"""
from . import ops


def cp_attn(q, K, V, n_live, scale):
    return ops.cp_attn_op(q, K, V, int(n_live), float(scale))


def cp_step(q, k, v, K, V, p, scale):
    return ops.cp_step(q, k, v, K, V, int(p), float(scale))
