"""turbopress_b200: B200-native (sm_100a) packed-TCQ decode path.

A drop-in for the packed runtime of TurboPress (godsonj64/turbopress):
``PackedTCQLinear`` with the reference constructor / forward / decode_rows /
packed_bytes API, the format-v2 bit-stream helpers and the artifact loader,
backed by hand-written CUDA kernels behind a C ABI
(``include/turbopress_b200.h``).
"""

from .runtime import (  # noqa: F401
    MODES,
    PackedTCQLinear,
    Trellis,
    load_packed_model,
    pack_le,
    rotate,
    subset_lut,
    unpack_le,
    v1_payload_to_packed,
    window_decode_levels,
)

__version__ = "0.1.0"
