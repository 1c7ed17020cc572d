"""The reference test's input generator, restated: XorShift32 and its
uniform [-2, 2] floats (Singularity/tests/test_and_bench_a5.cpp:362-379)."""
import numpy as np


class XorShift32:
    def __init__(self, seed: int = 0xC0FFEE05):
        self.state = seed & 0xFFFFFFFF

    def next_u32(self) -> int:
        x = self.state
        x ^= (x << 13) & 0xFFFFFFFF
        x ^= x >> 17
        x ^= (x << 5) & 0xFFFFFFFF
        self.state = x
        return x

    def next_f32(self) -> np.float32:
        s = (self.next_u32() & 0xFFFF) - 32768
        return np.float32(s) * np.float32(1.0 / 16384.0)


def rel_error(a, b) -> float:
    """rel_error, Singularity/tests/test_and_bench_a5.cpp:381-388."""
    a = np.float32(a)
    b = np.float32(b)
    diff = abs(a - b)
    denom = max(abs(a), abs(b), np.float32(1e-2))
    return float(diff / denom)
