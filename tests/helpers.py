"""Input generation and comparison shared by the parity tests."""
import numpy as np

import oracle

ATOL = 2e-3          # max |gpu - oracle| on outputs
MIN_COSINE = 0.9999  # cosine similarity floor on outputs

TORCH_DTYPE_NAMES = {oracle.F32: "float32", oracle.F16: "float16", oracle.BF16: "bfloat16"}


def normal(seed: int, shape, dtype: int, offset: int = 0) -> np.ndarray:
    """Seeded N(0,1) (splitmix64 + Box-Muller) rounded to `dtype`, as float32."""
    n = int(np.prod(shape))
    return oracle.round_to(oracle.splitmix_normal(seed, n, offset), dtype).reshape(shape)


def to_dev(a: np.ndarray, dtype: int):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
    return t.to(device="cuda", dtype=getattr(torch, TORCH_DTYPE_NAMES[dtype])).contiguous()


def to_np(t) -> np.ndarray:
    import torch
    return t.detach().to(device="cpu", dtype=torch.float32).numpy()


def cosine(a: np.ndarray, b: np.ndarray) -> float:
    a = a.astype(np.float64).ravel()
    b = b.astype(np.float64).ravel()
    na, nb = np.linalg.norm(a), np.linalg.norm(b)
    if na == 0 and nb == 0:
        return 1.0
    return float(a @ b / (na * nb))


def assert_close(got: np.ndarray, want: np.ndarray, atol: float = ATOL, min_cos: float = MIN_COSINE, what=""):
    assert got.shape == want.shape, (got.shape, want.shape)
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    i = int(np.argmax(err))
    assert err.flat[i] <= atol, f"{what}: max abs err {err.flat[i]:.3e} at {np.unravel_index(i, got.shape)} " \
                                f"(got {got.flat[i]}, want {want.flat[i]})"
    c = cosine(got, want)
    assert c >= min_cos, f"{what}: cosine {c:.6f} < {min_cos}"
    return float(err.max()), c


def ulp_error(got: np.ndarray, want: np.ndarray, dtype: int) -> float:
    """Largest error in units of the output dtype's spacing at the reference value."""
    w = np.abs(want.astype(np.float64))
    mant = {oracle.F16: 10, oracle.BF16: 7, oracle.F32: 23}[dtype]
    spacing = np.maximum(2.0 ** (np.floor(np.log2(np.maximum(w, 1e-30))) - mant), 2.0 ** -24)
    return float(np.max(np.abs(got.astype(np.float64) - want) / spacing))
