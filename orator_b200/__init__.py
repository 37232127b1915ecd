"""B200-native Qwen3-ASR streaming text decoder (sm_100a CUDA behind a C ABI).

``AsrTextDecoder`` mirrors the reference class of the same name
(thomas-hiddenpeak/Orator include/model/asr_text_decoder.h); the compute runs
in ``liborator_b200.so`` built from ``orator_b200/csrc``.
"""
from ._lib import OrxError, LIB_PATH  # noqa: F401
from .decoder import AsrTextConfig, AsrTextDecoder, synth_f32  # noqa: F401
from .batch import BatchDecoder  # noqa: F401
from .layer32 import Layer32  # noqa: F401
