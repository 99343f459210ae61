"""B200-native (sm_100a) CuteChronos2 encoder forward: drop-in for the
``cutechronos`` model / pipeline API of lee101/cutedsl, computed by the
hand-written CUDA kernels of ``_lib/libcc2_b200.so``."""

from .model import CuteChronos2Config, CuteChronos2Model  # noqa: F401
from .pipeline import CuteChronos2Pipeline  # noqa: F401

__all__ = ["CuteChronos2Config", "CuteChronos2Model", "CuteChronos2Pipeline"]
