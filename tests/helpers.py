"""Helpers shared by the tests (not part of the product)."""
from __future__ import annotations

import glob
import os

import numpy as np

from oracle import gguf_oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
QTYPES = [O.Q8_0, O.Q4_0, O.Q4_K, O.Q6_K]
QNAMES = {qt: O.QTYPES[qt][0] for qt in QTYPES}
TOL = 2e-3  # max|y - y_ref| / rms(y_ref), the north-star gate


def golden(qt: int) -> dict:
    with np.load(os.path.join(GOLDEN, f"golden_{QNAMES[qt].lower()}.npz")) as z:
        return {k: z[k] for k in z.files}


def same_bits(a: np.ndarray, b: np.ndarray) -> bool:
    """Bitwise equality of fp32 arrays, with any NaN matching any NaN."""
    a = np.asarray(a, np.float32).reshape(-1)
    b = np.asarray(b, np.float32).reshape(-1)
    if a.shape != b.shape:
        return False
    na, nb = np.isnan(a), np.isnan(b)
    if not np.array_equal(na, nb):
        return False
    return np.array_equal(a[~na].view(np.uint32), b[~nb].view(np.uint32))


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 to the nearest bf16 value (RNE), returned as fp32."""
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return u.astype(np.uint32).view(np.float32)


def header_functions() -> list[str]:
    """Every function name declared in include/*.h."""
    import re
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    names = []
    for h in glob.glob(os.path.join(root, "include", "*.h")):
        txt = open(h).read()
        txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
        names += re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(ggufmm_[a-z_0-9]+)\s*\(", txt, flags=re.M)
    return sorted(set(names))
