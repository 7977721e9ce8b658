"""Helpers for the GPU parity tests: synthetic inputs of the BASELINE
configurations (seeded numpy, N(0, 0.02) weights, N(0, 1) activations) and
bit comparison."""
import numpy as np

F = np.float32


def bits_equal(a, b) -> bool:
    a = np.ascontiguousarray(np.asarray(a, F))
    b = np.ascontiguousarray(np.asarray(b, F))
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def mismatch_report(got, want, k=5) -> str:
    g = np.asarray(got, F).view(np.uint32)
    w = np.asarray(want, F).view(np.uint32)
    bad = np.nonzero(g != w)[0]
    return f"{bad.size} mismatches; first {bad[:k].tolist()}: got {np.asarray(got)[bad[:k]]} want {np.asarray(want)[bad[:k]]}"


def weights(seed, n):
    return (np.random.default_rng(seed).standard_normal(n, dtype=F) * F(0.02)).astype(F)


def acts(seed, n):
    return np.random.default_rng(seed + 1_000_000).standard_normal(n, dtype=F)


def to_dev(*arrs):
    import torch
    return [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in arrs]


def to_host(t):
    return t.cpu().numpy()
