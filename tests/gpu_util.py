"""Helpers shared by the GPU parity tests (seeded data, host/device conversion)."""
import numpy as np

UT = {32: np.uint32, 64: np.uint64}
FT = {32: np.float32, 64: np.float64}


def from_hex(width, hexes, shape=None):
    a = np.array([int(h, 16) for h in hexes], dtype=UT[width]).view(FT[width])
    return a.reshape(shape) if shape is not None else a


def bits(array):
    array = np.ascontiguousarray(array)
    return array.view(np.uint32 if array.dtype == np.float32 else np.uint64)


def to_device(array):
    import torch

    return torch.from_numpy(np.ascontiguousarray(array)).cuda()


def to_host(tensor):
    return tensor.detach().cpu().numpy()


def status_word(status_tensor):
    return int(status_tensor.cpu().numpy().view(np.uint64)[0])


def dyadic_uniform(rng, shape, width, low=-1.0):
    """Exact dyadic U[low, 1): k * 2^-23 (binary32) or k * 2^-52 (binary64), SplitMix-style seeded."""
    frac = 23 if width == 32 else 52
    if low < 0:
        k = rng.integers(-(1 << frac), 1 << frac, size=shape, dtype=np.int64)
        return (k.astype(np.float64) * 2.0 ** -frac).astype(FT[width])
    k = rng.integers(0, 1 << (frac + 1), size=shape, dtype=np.int64)
    return (k.astype(np.float64) * 2.0 ** -(frac + 1)).astype(FT[width])


def specials(width):
    fi = np.finfo(FT[width])
    return [0.0, -0.0, fi.tiny, -fi.tiny, fi.tiny / 4, fi.max, -fi.max, np.nan, np.inf, -np.inf,
            fi.smallest_subnormal, 1.0, -1.0]


def sprinkle(rng, array, values, count):
    flat = array.reshape(-1)
    idx = rng.choice(flat.size, size=min(count, flat.size), replace=False)
    for j, i in enumerate(idx):
        flat[i] = values[j % len(values)]
    return array
