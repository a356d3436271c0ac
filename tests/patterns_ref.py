"""Independent Python restatement of the reference input generator — test infrastructure.

host/src/lib.rs:218-256 (make_input): an xorshift32 state seeded with `seed`,
advanced (<<13, >>17, <<5) once per element in row-major order, feeding seven
patterns; values are rounded to half with reference/src/lib.rs:48-83. Used to
check the product's C++ generator (cs_make_input) bit for bit.
"""
import numpy as np

import oracle_ctypes as O

PATTERNS = ["zeros", "ramp", "alternating", "spikes", "extreme", "tiny", "random"]


def make_input(rows: int, cols: int, pattern: str, seed: int) -> np.ndarray:
    f32 = np.float32
    state = seed & 0xFFFFFFFF
    out = np.zeros(rows * cols, dtype=np.uint16)
    for i in range(rows * cols):
        r, c = divmod(i, cols)
        state ^= (state << 13) & 0xFFFFFFFF
        state ^= state >> 17
        state ^= (state << 5) & 0xFFFFFFFF
        if pattern == "zeros":
            v = f32(0.0)
        elif pattern == "ramp":
            v = (f32(c) - f32(r)) * f32(0.125)
        elif pattern == "alternating":
            v = f32(-11.0) if c % 2 == 0 else f32(11.0)
        elif pattern == "spikes":
            v = f32(28.0) if c == min(r, cols - 1) else f32(-23.0)
        elif pattern == "extreme":
            v = f32(65000.0) if c % 5 == 0 else f32(-65000.0)
        elif pattern == "tiny":
            v = f32(c % 11) * f32(0.00005) - f32(0.00025)
        else:
            v = (f32(state >> 16) / f32(65536.0) - f32(0.5)) * f32(32.0)
        out[i] = O.h(float(v))
    return out
