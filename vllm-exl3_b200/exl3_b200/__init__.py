"""B200-native (sm_100a) EXL3 routed-expert MoE path.

``vllm_exl3_c`` (next to this package) is the drop-in for the reference's
native module; :mod:`exl3_b200.moe` mirrors the reference's dispatch layer;
:mod:`exl3_b200.ep` adds expert-parallel dispatch/combine over NCCL;
:mod:`exl3_b200.synthetic` builds the seeded benchmark packs.
"""

from . import _native  # noqa: F401

__all__ = ["_native"]
