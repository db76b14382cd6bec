"""B200-native decode engine for the Qwen2.5-1.5B architecture with Q4 block-32
weights: hand-written sm_100a CUDA kernels behind a C ABI (include/qwen_b200.h,
libqwen_b200.so), with the reference's QwenEngine surface on top.

    from qweninferenceengine_b200 import QwenEngine, QwenConfig
    eng = QwenEngine("weights/")                # reference weight directory
    ids = eng.generate(prompt_ids, max_tokens=96)
"""
from ._lib import LIB_PATH, QwenError, lib  # noqa: F401
from .engine import STOP_TOKENS, QwenConfig, QwenEngine  # noqa: F401

__all__ = ["QwenEngine", "QwenConfig", "QwenError", "STOP_TOKENS", "lib", "LIB_PATH"]
