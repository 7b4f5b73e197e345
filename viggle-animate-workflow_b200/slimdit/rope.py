"""Rotary frequency table ``rope.inv_freq`` (derived, not in the official checkpoint).

ComfyUI's MiniMax-H3 model registers the buffer uninitialised and expects the checkpoint to
carry it. Values: ``1 / 10000 ** (k / 16)`` for k in [0, 16), evaluated entirely in float32
(the reference's slimdit/rope.py:23-27; other spellings round differently in the last ulp).
"""

from __future__ import annotations

import numpy as np

INV_FREQ_LEN = 16
THETA = 10000.0


def rope_inv_freq(length: int = INV_FREQ_LEN, theta: float = THETA) -> np.ndarray:
    """float32 [length]; index 0 is 1.0."""
    k = np.arange(length, dtype=np.float32)
    return np.float32(1.0) / (np.float32(theta) ** (k / np.float32(length)))
