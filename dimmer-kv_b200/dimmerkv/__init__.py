"""DimmerKV for B200: attention directly over a compressed KV cache (sm_100a kernels).

Host package mirroring the reference's Python API for the hot path (scripts/compressed_attention.py,
scripts/progressive.py, scripts/kvtc.py, scripts/dimmer.py, scripts/methods.py). The kernels live in
libdimmerkv.so (built from ../csrc by ../build_lib.py) and are bound with ctypes (``_lib``).
"""

__version__ = "0.1.0"
