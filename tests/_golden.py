"""Loader for the committed golden fixtures (tests/golden/*.npz)."""
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    with np.load(os.path.join(GOLDEN, name + ".npz")) as z:
        return {k: z[k] for k in z.files}


def e4m3_to_float(u8):
    """Decode float8_e4m3fn bytes (uint8 array) to float64 (1-4-3, bias 7, no inf, 0x7f/0xff NaN)."""
    u = np.asarray(u8, dtype=np.uint8).astype(np.int64)
    s = np.where(u & 0x80, -1.0, 1.0)
    e = (u >> 3) & 0xF
    m = u & 0x7
    val = np.where(e == 0, m / 8.0 * 2.0 ** -6, (1 + m / 8.0) * 2.0 ** (e - 7))
    val = np.where((e == 0xF) & (m == 0x7), np.nan, val)
    return s * val


def varlen_cases():
    return ["varlen_g4_nosink", "varlen_g4_sink", "varlen_g4_sink01", "varlen_g8_sink", "varlen_edge_sink",
            "varlen_g16_nosink", "varlen_g8_d64_nosink", "varlen_g4_d64_sink"]


def paged_cases():
    return ["paged_g4", "paged_g4_d64"]
