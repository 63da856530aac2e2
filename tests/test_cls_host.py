"""Host parts of the angle classifier: the seeded synthetic-weight generator
(tocr_synth_weights) against a numpy restatement of its formula, bit for bit,
and its argument checks."""
import numpy as np

M64 = (1 << 64) - 1


def restated(seed, scale, n):
    out = np.empty(n, np.float32)
    for i in range(n):
        z = (seed + (i + 1) * 0x9E3779B97F4A7C15) & M64
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
        z ^= z >> 31
        u = np.float32(z >> 40) * np.float32(1.0 / 16777216.0)
        out[i] = np.float32(scale) * (np.float32(2.0) * u - np.float32(1.0))
    return out


def test_synth_weights_formula(tocr):
    L = tocr.lib()
    for seed, scale, n in [(0x7EC0C150, 0.35, 864), (0x7EC0C150 + 18, 0.22, 4096), (7, 1.0, 33)]:
        got = np.empty(n, np.float32)
        assert L.tocr_synth_weights(seed, scale, got.ctypes.data, n) == 0
        assert np.array_equal(got, restated(seed, scale, n))
        assert np.abs(got).max() <= np.float32(scale) and got.std() > 0.4 * scale


def test_synth_weights_arguments(tocr):
    L = tocr.lib()
    assert L.tocr_synth_weights(1, 1.0, None, 0) == 0
    assert L.tocr_synth_weights(1, 1.0, None, 5) == 1
