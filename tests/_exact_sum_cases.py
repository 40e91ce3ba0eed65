"""Term vectors for the exact left-to-right sum tests: squares of normal
activations (the RMSNorm case), wide dynamic range, exact halfway ties,
subnormals, a single dominant term, zeros, and overflow to inf."""
import numpy as np


def cases(seed: int, count: int, nmax: int = 3000):
    rng = np.random.default_rng(seed)
    out = []
    for t in range(count):
        n = int(rng.integers(1, nmax))
        kind = t % 7
        if kind == 0:
            v = rng.standard_normal(n).astype(np.float32)
            a = v * v
        elif kind == 1:
            a = np.exp(rng.uniform(-80, 80, n)).astype(np.float32)
        elif kind == 2:  # few mantissa bits: many exact halfway cases
            a = (rng.integers(0, 16, n) * 2.0 ** rng.integers(-5, 5, n)).astype(np.float32)
        elif kind == 3:
            a = rng.integers(0, 4, n).astype(np.float32) * np.float32(2.0 ** -140)
        elif kind == 4:
            a = np.full(n, rng.uniform(0, 1), np.float32)
            a[rng.integers(0, n)] = 1e30
        elif kind == 5:
            a = np.zeros(n, np.float32)
            a[rng.integers(0, n, size=min(n, 5))] = rng.random(min(n, 5)).astype(np.float32)
        else:
            with np.errstate(over="ignore"):
                a = (rng.standard_normal(n) * 1e18).astype(np.float32) ** 2
        out.append((kind, np.ascontiguousarray(a, np.float32)))
    return out


def serial(a: np.ndarray) -> np.float32:
    """s = 0; s = fl(s + a_j) in order (np.cumsum over float32 is sequential)."""
    if a.size == 0:
        return np.float32(0)
    with np.errstate(over="ignore", invalid="ignore"):
        return np.cumsum(a, dtype=np.float32)[-1]
