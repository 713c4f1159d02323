"""Seeded synthetic GGUF weights and activations.

The reference publishes no dataset for this path; the benchmark configurations
define value distributions instead, and these generators draw them:

* Q4_0: fp16 d ~ U[0.005, 0.02], 16 bytes of uniform random nibbles.
* Q8_0: fp16 d ~ U[0.002, 0.01], 32 int8 ~ U{-127..127}.
* Q5_K: fp16 d ~ U[0.001, 0.01], fp16 dmin ~ U[0, 0.005], scales[12], qh[32]
  and qs[128] uniform random bytes.
* Q6_K: ql[128], qh[64] uniform random bytes, int8 scales[16] uniform over
  the full int8 range, fp16 d ~ U[0.001, 0.01].
* FP16: weights ~ N(0, 0.02) rounded to fp16.
* Activations x: fp32 ~ N(0, 1).

Scales are drawn in fp32 and rounded to fp16 with round-to-nearest-even,
then stored as raw little-endian bits in the block layout of
include/quantization.hpp:8-47.

Two back ends produce the same layouts and distributions:
``numpy`` (``Generator(PCG64(seed))``, used for fixtures and parity tests)
and ``torch`` on a CUDA device (used to fill multi-GB benchmark stacks
without a host round trip).  The two do not produce identical bytes for the
same seed.  By convention ``seed = 1000 * config + matrix_index``.
"""
from __future__ import annotations

import numpy as np

from .formats import BLOCK, DataType, parse

_D_RANGE = {
    DataType.GGUF_Q4_0: (0.005, 0.02),
    DataType.GGUF_Q8_0: (0.002, 0.01),
    DataType.GGUF_Q5_K: (0.001, 0.01),
    DataType.GGUF_Q6_K: (0.001, 0.01),
}
_DMIN_RANGE = (0.0, 0.005)
FP16_STD = 0.02


def _f16_bits_np(a: np.ndarray) -> np.ndarray:
    return a.astype(np.float32).astype(np.float16).view(np.uint8).reshape(-1, 2)


def blocks_numpy(dtype, rows: int, cols: int, seed: int) -> np.ndarray:
    """Weight matrix [rows, cols] as a flat uint8 array of GGUF blocks
    (FP16: a flat uint16 array of rows*cols halves)."""
    dt = parse(dtype)
    rng = np.random.Generator(np.random.PCG64(seed))
    per, nbytes = BLOCK[dt]
    if dt == DataType.FP16:
        w = rng.normal(0.0, FP16_STD, rows * cols).astype(np.float32)
        return w.astype(np.float16).view(np.uint16)
    nb = rows * cols // per
    lo, hi = _D_RANGE[dt]
    d = _f16_bits_np(rng.uniform(lo, hi, nb))
    if dt == DataType.GGUF_Q4_0:
        a = np.empty((nb, nbytes), np.uint8)
        a[:, 0:2] = d
        a[:, 2:] = rng.integers(0, 256, (nb, 16), dtype=np.uint8)
    elif dt == DataType.GGUF_Q8_0:
        a = np.empty((nb, nbytes), np.uint8)
        a[:, 0:2] = d
        a[:, 2:] = rng.integers(-127, 128, (nb, 32), dtype=np.int16).astype(np.int8).view(np.uint8)
    elif dt == DataType.GGUF_Q5_K:
        a = rng.integers(0, 256, (nb, nbytes), dtype=np.uint8)
        a[:, 0:2] = d
        a[:, 2:4] = _f16_bits_np(rng.uniform(*_DMIN_RANGE, nb))
    else:  # Q6_K
        a = rng.integers(0, 256, (nb, nbytes), dtype=np.uint8)
        a[:, 208:210] = d
    return a.reshape(-1)


def activations_numpy(m: int, k: int, seed: int) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(seed))
    return rng.normal(0.0, 1.0, (m, k)).astype(np.float32)


def blocks_torch(dtype, rows: int, cols: int, seed: int, device="cuda"):
    """Device-side generator with the same layout and distributions as
    `blocks_numpy` (different bytes).  Returns a flat uint8 tensor."""
    import torch

    dt = parse(dtype)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    per, nbytes = BLOCK[dt]
    if dt == DataType.FP16:
        w = torch.empty(rows * cols, dtype=torch.float32, device=device).normal_(0.0, FP16_STD, generator=g)
        return w.to(torch.float16).view(torch.uint8)
    nb = rows * cols // per

    def f16bits(lo, hi):
        v = torch.empty(nb, dtype=torch.float32, device=device).uniform_(lo, hi, generator=g)
        return v.to(torch.float16).view(torch.uint8).view(nb, 2)

    out = torch.empty((nb, nbytes), dtype=torch.uint8, device=device)
    # torch.randint's upper bound is exclusive and must fit int64; 256 is fine for uint8
    out.random_(0, 256, generator=g)
    if dt == DataType.GGUF_Q4_0:
        out[:, 0:2] = f16bits(*_D_RANGE[dt])
    elif dt == DataType.GGUF_Q8_0:
        out[:, 0:2] = f16bits(*_D_RANGE[dt])
        q = torch.randint(-127, 128, (nb, 32), dtype=torch.int16, device=device, generator=g)
        out[:, 2:] = q.to(torch.int8).view(torch.uint8)
    elif dt == DataType.GGUF_Q5_K:
        out[:, 0:2] = f16bits(*_D_RANGE[dt])
        out[:, 2:4] = f16bits(*_DMIN_RANGE)
    else:
        out[:, 208:210] = f16bits(*_D_RANGE[dt])
    return out.view(-1)
