"""CPU oracle for the Drama-3 MoE / block-FP8 GEMV hot path.

TEST INFRASTRUCTURE ONLY. Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU
baseline leg may import this package, and only as the checker (or, in bench.py, as the timed
CPU restatement). The product path (`drama3_b200`) never imports it.

Parity status: pinned. `tests/golden/make_golden.py` runs the reference's own code on this
CPU to produce the committed fixtures. The code it runs is `engine.fp8_block`, `engine.Speaker`
and `engine.speaker_forward`, imported with `fish_speech` stubbed, plus `fp8_linear.quantize` /
`dequantize` and the Triton `_gemv` kernel under the Triton interpreter. `tests/test_oracle.py`
checks this oracle against those fixtures. One gap remains: the grouped product inside
fish-speech's `fp8_moe_forward` is a third-party function absent from the reference. It is
restated here after the reference's own pure-torch MoE (`exp3_distill.SpeakerMoE.forward`,
exp3_distill.py:34-48).
"""

from .moe_oracle import (  # noqa: F401
    BLOCK,
    audio_head,
    direction_score,
    FP8_MAX,
    dequant,
    fp8_block,
    gemv,
    linear_dequant,
    moe_forward,
    moe_layer,
    permutation,
    quantize_rows,
    route,
    router_logits,
    shared_expert,
    shared_gate,
    speaker,
    speaker_forward,
)
