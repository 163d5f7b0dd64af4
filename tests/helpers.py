"""Shared helpers for the parity tests: host <-> device tensors and tolerances."""

from __future__ import annotations

import numpy as np

# Attention tolerances (|got - want| <= ATOL + RTOL * |want|), per element type.
TOL = {"f32": (1e-5, 1e-5), "f16": (2e-3, 1e-3), "bf16": (2e-3, 1e-3)}
CODE = {"f32": 0, "f16": 1, "bf16": 2}


def torch_dtype(dtype: str):
    import torch

    return {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[dtype]


def to_dev(a: np.ndarray, dtype: str | None = None, device="cuda"):
    import torch

    a = np.ascontiguousarray(a)
    if dtype == "bf16":
        return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).to(device)
    return torch.from_numpy(a).to(device)


def to_host(t, dtype: str | None = None) -> np.ndarray:
    import torch

    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def as_f64(t) -> np.ndarray:
    return t.detach().float().cpu().numpy().astype(np.float64)


# Significand bits of each output type: the result is stored in that type, so
# on top of TOL the comparison allows half a unit in its last place at the
# expected value (bf16: 2^-9 relative, f16: 2^-11, f32: 2^-24) -- a correctly
# computed bf16 output near 1.06 can only be 1.0547 or 1.0625.
MANTISSA = {"f32": 23, "f16": 10, "bf16": 7}


def half_ulp(want: np.ndarray, dtype: str) -> np.ndarray:
    e = np.floor(np.log2(np.maximum(np.abs(want), 1e-30)))
    return np.exp2(e - MANTISSA[dtype] - 1)


def assert_close(got: np.ndarray, want: np.ndarray, dtype: str, what: str = "") -> None:
    atol, rtol = TOL[dtype]
    err = np.abs(got - want)
    lim = atol + rtol * np.abs(want) + half_ulp(want, dtype)
    bad = ~(err <= lim)
    if bad.any():
        i = np.unravel_index(np.argmax(err - lim), err.shape)
        raise AssertionError(
            f"{what}: {bad.sum()} of {bad.size} elements out of tolerance ({dtype}: atol={atol}, "
            f"rtol={rtol}); worst at {i}: got {got[i]!r} want {want[i]!r} (max abs err {err.max():.3e})"
        )


def random_tables(rng, ctx, pool):
    """Block tables with physical ids drawn without replacement from a shuffled pool."""
    bs = 16
    nblk = [(int(c) + bs - 1) // bs for c in ctx]
    assert sum(nblk) <= pool
    ids = rng.permutation(pool)
    mbps = max(1, max(nblk))
    t = np.zeros((len(ctx), mbps), np.int32)
    o = 0
    for s, n in enumerate(nblk):
        t[s, :n] = ids[o:o + n]
        o += n
    return t
