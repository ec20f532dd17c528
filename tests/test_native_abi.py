"""The C-ABI library loads on a machine without a GPU and exports every entry
point include/*.h declares; argument validation needs no device."""
import ctypes
import glob
import os
import re

import pytest

from fasterkernels_b200 import _native as N
from fasterkernels_b200.build import LIB_PATH, build_library

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names |= set(re.findall(r"\b(fk_[a-z0-9_]+)\s*\(", src))
    return names


def test_library_builds_and_loads():
    build_library()
    assert os.path.exists(LIB_PATH)
    assert N.lib().fk_version() == 100


def test_every_declared_symbol_is_exported():
    syms = declared_symbols()
    assert {"fk_flash_decode_gqa_varlen", "fk_flash_decode_gqa_hf_dense", "fk_paged_flash_decode",
            "fk_decode_workspace_bytes", "fk_last_error", "fk_version"} <= syms
    L = ctypes.CDLL(LIB_PATH)
    for s in sorted(syms):
        assert hasattr(L, s), s


def test_invalid_arguments_are_rejected_without_touching_the_device():
    L = N.lib()
    rc = L.fk_flash_decode_gqa_varlen(None, None, None, None, None, None, 1, 32, 8, 128, 16, 0,
                                      0, 0, 0, 0, 0, 0, 0, 0, None, 0, None)
    assert rc == 1 and "non-null" in N.last_error()
    fake = ctypes.c_void_p(16)
    rc = L.fk_flash_decode_gqa_varlen(fake, fake, fake, fake, None, fake, 1, 32, 8, 96, 16, 0,
                                      0, 0, 0, 0, 0, 0, 0, 0, fake, 0, None)
    assert rc == 2 and "head_dim" in N.last_error()
    rc = L.fk_flash_decode_gqa_varlen(fake, fake, fake, fake, None, fake, 1, 36, 8, 128, 16, 0,
                                      0, 0, 0, 0, 0, 0, 0, 0, fake, 0, None)
    assert rc == 1 and "multiple" in N.last_error()
    assert L.fk_decode_workspace_bytes_gqa(0, 4, 36, 8, 0) == 0 and "bad sizes" in N.last_error()
    rc = L.fk_paged_flash_decode(fake, fake, fake, fake, fake, None, fake, 1, 32, 8, 128, 10, 32, 4, 0, 0, 0,
                                 None, None, None, *([0] * 11), fake, 0, None)
    assert rc in (1, 2)


def test_entry_points_reject_cpu_tensors():
    import torch
    import fasterkernels_b200 as fk
    q = torch.zeros(1, 32, 128, dtype=torch.float16)
    k = torch.zeros(4, 8, 128, dtype=torch.float16)
    with pytest.raises(ValueError, match="CUDA"):
        fk.flash_decode_gqa_varlen(q, k, k, torch.tensor([0, 4], dtype=torch.int32))


def test_debug_hook_validates_its_arguments():
    L = N.lib()
    assert L.fk_debug_configure(10, 0) == 1 and "wait_ns" in N.last_error()
    assert L.fk_debug_configure(4_000_000_000, 2) == 1 and "inject" in N.last_error()
    assert L.fk_debug_configure(4_000_000_000, 0) == 0  # the default: 4 s bound, no injection


def test_custom_ops_are_registered_with_mutation_schemas():
    # torch.compile traces the entry points through these ops; each declares
    # the tensors it writes
    import torch
    import fasterkernels_b200  # noqa: F401  (registers the ops)
    ns = torch.ops.fasterkernels_b200
    for name, mutated in (("varlen_decode", {"out"}), ("dense_decode", {"out"}), ("paged_decode", {"out"}),
                          ("paged_kv_append", {"k_pool", "v_pool", "positions", "status"})):
        schema = getattr(ns, name).default._schema
        written = {a.name for a in schema.arguments if a.alias_info is not None and a.alias_info.is_write}
        assert written == mutated, (name, written)
