"""drama3_b200: the Drama-3 per-frame MoE feed-forward and block-FP8 GEMV, hand-written for B200.

Python host code over a C ABI (include/dm3.h, libdm3.so built for sm_100a) with the call
signatures of the reference engine: `fp8_moe_forward`, `Speaker`, `speaker_forward`,
`FP8Linear` / `convert` / `quantize` / `dequantize`, `fp8_block`; plus the HBM-resident expert
table read from the checkpoint (`ExpertTable`) and the speaker file reader. Import name `drama3_b200`
(see drama3_b200.py at the repository root; the directory name has hyphens).
"""

from . import _lib, ep, ops  # noqa: F401
from .audio_head import AudioHead  # noqa: F401
from .fp8_linear import BLOCK, FP8Linear, convert, dequantize, quantize  # noqa: F401
from .fp8_moe import fp8_moe_forward  # noqa: F401
from .experts import ExpertTable, ResidentExperts, attach_expert_table, read_expert_checkpoint  # noqa: F401
from .speaker import (  # noqa: F401
    SharedExpert,
    Speaker,
    fp8_block,
    install,
    make_speaker_forward,
    read_speaker_file,
    speakers_from_file,
)

__version__ = "0.1.0"
