"""The C-ABI launches of the decode entry points, and their registration as
``torch.library`` custom ops so that ``torch.compile`` traces a model through
them without a graph break.

The reference's entry points are user Triton kernels, which ``torch.compile``
traces (fskernels/triton/triton_gqa_decode.py:126-155); a ``ctypes`` call is
opaque to it.  Each launcher below takes checked, laid-out tensors and writes
``out`` (declared as mutated; the fake implementation does nothing, since the
output is preallocated by the caller).  Eager calls go straight to the
launcher (no dispatcher overhead on the hot path); calls made while
``torch.compile`` is tracing go through ``torch.ops.fasterkernels_b200.*``.
Both run the same kernel with the same arguments, so the results are
bit-identical.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _native as N


def _scale(x):
    return N.ptr(x) if x is not None else None


# ---------------------------------------------------------------- launchers
def varlen_launch(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu: torch.Tensor, s_aux: Optional[torch.Tensor],
                  out: torch.Tensor) -> None:
    dev = q.device
    B, QH, D = q.shape
    T, KVH, _ = k.shape
    code = N.dtype_code(q.dtype)
    ws = N.workspace(dev, B, QH, KVH, code)
    rc = N.lib().fk_flash_decode_gqa_varlen(
        N.ptr(q), N.ptr(k), N.ptr(v), N.ptr(cu), N.ptr(s_aux), N.ptr(out),
        B, QH, KVH, D, T, code,
        q.stride(0), q.stride(1), k.stride(0), k.stride(1), v.stride(0), v.stride(1), out.stride(0), out.stride(1),
        N.ptr(ws), ws.numel(), N.stream_of(dev))
    N.check(rc, "fk_flash_decode_gqa_varlen")


def dense_launch(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, lens: torch.Tensor,
                 starts: Optional[torch.Tensor], s_aux: Optional[torch.Tensor], scale_q: Optional[torch.Tensor],
                 scale_k: Optional[torch.Tensor], scale_v: Optional[torch.Tensor], out: torch.Tensor) -> None:
    dev = q.device
    B, QH, D = q.shape
    _, KVH, S, _ = k_cache.shape
    kv_code = N.dtype_code(k_cache.dtype)
    ws = N.workspace(dev, B, QH, KVH, kv_code)
    rc = N.lib().fk_flash_decode_gqa_hf_dense(
        N.ptr(q), N.ptr(k_cache), N.ptr(v_cache), N.ptr(lens), N.ptr(starts), N.ptr(s_aux), N.ptr(out),
        B, QH, KVH, D, S, N.dtype_code(q.dtype), kv_code, N.dtype_code(out.dtype),
        _scale(scale_q), _scale(scale_k), _scale(scale_v),
        q.stride(0), q.stride(1), k_cache.stride(0), k_cache.stride(1), k_cache.stride(2),
        v_cache.stride(0), v_cache.stride(1), v_cache.stride(2), out.stride(0), out.stride(1),
        N.ptr(ws), ws.numel(), N.stream_of(dev))
    N.check(rc, "fk_flash_decode_gqa_hf_dense")


def paged_launch(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor, bt: torch.Tensor, lens: torch.Tensor,
                 s_aux: Optional[torch.Tensor], scale_q: Optional[torch.Tensor], scale_k: Optional[torch.Tensor],
                 scale_v: Optional[torch.Tensor], out: torch.Tensor) -> None:
    dev = q.device
    B, QH, D = q.shape
    P, KVH, PS, _ = k_pool.shape
    kv_code = N.dtype_code(k_pool.dtype)
    ws = N.workspace(dev, B, QH, KVH, kv_code)
    rc = N.lib().fk_paged_flash_decode(
        N.ptr(q), N.ptr(k_pool), N.ptr(v_pool), N.ptr(bt), N.ptr(lens), N.ptr(s_aux), N.ptr(out),
        B, QH, KVH, D, P, PS, bt.shape[1], N.dtype_code(q.dtype), kv_code, N.dtype_code(out.dtype),
        _scale(scale_q), _scale(scale_k), _scale(scale_v),
        q.stride(0), q.stride(1), k_pool.stride(0), k_pool.stride(1), k_pool.stride(2),
        v_pool.stride(0), v_pool.stride(1), v_pool.stride(2), bt.stride(0), out.stride(0), out.stride(1),
        N.ptr(ws), ws.numel(), N.stream_of(dev))
    N.check(rc, "fk_paged_flash_decode")


def append_launch(k_new: torch.Tensor, v_new: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                  bt: torch.Tensor, positions: torch.Tensor, increment: bool, scale_k: Optional[torch.Tensor],
                  scale_v: Optional[torch.Tensor], status: Optional[torch.Tensor]) -> None:
    B, KVH, D = k_new.shape
    rc = N.lib().fk_paged_kv_append(
        N.ptr(k_new), N.ptr(v_new), N.dtype_code(k_new.dtype), N.ptr(k_pool), N.ptr(v_pool),
        N.dtype_code(k_pool.dtype), N.ptr(bt), N.ptr(positions), 1 if increment else 0, _scale(scale_k),
        _scale(scale_v), N.ptr(status), B, KVH, D, k_pool.shape[0], bt.shape[1], k_new.stride(0), k_new.stride(1),
        v_new.stride(0), v_new.stride(1), k_pool.stride(0), k_pool.stride(1), k_pool.stride(2), v_pool.stride(0),
        v_pool.stride(1), v_pool.stride(2), bt.stride(0), N.stream_of(k_new.device))
    N.check(rc, "fk_paged_kv_append")


# ---------------------------------------------------------------- custom ops
_LIB = "fasterkernels_b200"


@torch.library.custom_op(f"{_LIB}::varlen_decode", mutates_args=("out",), device_types="cuda")
def _varlen_op(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu: torch.Tensor, s_aux: Optional[torch.Tensor],
               out: torch.Tensor) -> None:
    varlen_launch(q, k, v, cu, s_aux, out)


@torch.library.custom_op(f"{_LIB}::dense_decode", mutates_args=("out",), device_types="cuda")
def _dense_op(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, lens: torch.Tensor,
              starts: Optional[torch.Tensor], s_aux: Optional[torch.Tensor], scale_q: Optional[torch.Tensor],
              scale_k: Optional[torch.Tensor], scale_v: Optional[torch.Tensor], out: torch.Tensor) -> None:
    dense_launch(q, k_cache, v_cache, lens, starts, s_aux, scale_q, scale_k, scale_v, out)


@torch.library.custom_op(f"{_LIB}::paged_decode", mutates_args=("out",), device_types="cuda")
def _paged_op(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor, bt: torch.Tensor, lens: torch.Tensor,
              s_aux: Optional[torch.Tensor], scale_q: Optional[torch.Tensor], scale_k: Optional[torch.Tensor],
              scale_v: Optional[torch.Tensor], out: torch.Tensor) -> None:
    paged_launch(q, k_pool, v_pool, bt, lens, s_aux, scale_q, scale_k, scale_v, out)


@torch.library.custom_op(f"{_LIB}::paged_kv_append", mutates_args=("k_pool", "v_pool", "positions", "status"),
                         device_types="cuda")
def _append_op(k_new: torch.Tensor, v_new: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
               bt: torch.Tensor, positions: torch.Tensor, increment: bool, scale_k: Optional[torch.Tensor],
               scale_v: Optional[torch.Tensor], status: Optional[torch.Tensor]) -> None:
    append_launch(k_new, v_new, k_pool, v_pool, bt, positions, increment, scale_k, scale_v, status)


# The outputs are preallocated by the callers, so the fake (meta)
# implementations have nothing to compute.
for _op in (_varlen_op, _dense_op, _paged_op, _append_op):
    _op.register_fake(lambda *args, **kwargs: None)


def _dispatch(op, launch):
    def call(*args):
        if torch.compiler.is_compiling():
            return op(*args)
        return launch(*args)
    return call


varlen = _dispatch(_varlen_op, varlen_launch)
dense = _dispatch(_dense_op, dense_launch)
paged = _dispatch(_paged_op, paged_launch)
append = _dispatch(_append_op, append_launch)
