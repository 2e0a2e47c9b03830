"""Helpers shared by the GPU parity tests."""
import numpy as np
import torch

RTOL = 1e-5
ATOL = 1e-5  # |got - ref| <= 1e-5 + 1e-5 * |ref|, the reference's criterion (benchmark/q4_compare.c:139)


def dev(array, dtype=None) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(array))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def dev_bytes(payload) -> torch.Tensor:
    return dev(np.frombuffer(bytes(payload), dtype=np.uint8).copy())


def assert_within_tolerance(got, ref, what=""):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    err = np.abs(got - ref)
    bound = ATOL + RTOL * np.abs(ref)
    bad = np.nonzero(err > bound)[0]
    assert bad.size == 0, (f"{what}: {bad.size} outside 1e-5+1e-5|ref|; first index {bad[0]} "
                           f"got {got[bad[0]]!r} ref {ref[bad[0]]!r}")
    return float((err / bound).max()) if err.size else 0.0


def with_canaries(n, dtype=torch.float32, guard=8, fill=123456.0):
    """An output buffer with red zones on both sides (benchmark/q4_compare.c:359-361)."""
    buf = torch.full((n + 2 * guard,), fill, dtype=dtype, device="cuda")
    return buf, buf[guard:guard + n]


def canaries_intact(buf, guard=8, fill=123456.0):
    host = buf.cpu()
    return bool((host[:guard] == fill).all() and (host[-guard:] == fill).all())
