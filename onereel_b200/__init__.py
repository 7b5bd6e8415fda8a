"""onereel_b200: a B200-native (sm_100a) implementation of OneReel's scene-structured attention hot path.

Drop-in modules, same names and behaviour as the reference package `onereel`:
  onereel_b200.layout      SceneLayout (src/onereel/layout.py)
  onereel_b200.attention   cu_seqlens / varlen / varlen_lse / packed / packed_lse / overlapping_ranges / dense on the
                           sm_100a kernel (src/onereel/attention.py)
The device work runs in libonereel_b200.so (C ABI: include/onereel_b200.h), built by onereel_b200/csrc/build.py.
"""
from onereel_b200.layout import SceneLayout

__all__ = ['SceneLayout']
__version__ = '0.1.0'
