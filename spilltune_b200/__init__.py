"""B200-native frozen-linear hot path of the SpillTune layer-streaming LoRA trainer.

* ``spilltune_b200.codec``  – packed group-128 weight records (unchanged format).
* ``spilltune_b200.ops``    – fused dequant-GEMM + LoRA forward/backward over the C ABI.
* ``spilltune_b200.build``  – builds libspilltune_b200.so (nvcc, sm_100a).
"""
from .codec import PackedWeight, encode, encode_int4_sym, encode_nf4, from_record, INT4_SYM, NF4  # noqa: F401

__all__ = ["PackedWeight", "encode", "encode_int4_sym", "encode_nf4", "from_record", "INT4_SYM", "NF4"]
