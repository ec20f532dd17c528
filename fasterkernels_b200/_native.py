"""ctypes binding of the C-ABI in include/fk_decode.h, plus the per-stream
workspace and the torch-tensor -> C-argument plumbing shared by the entry
points.  torch supplies device memory and the current stream only; every
decode runs in the sm_100a kernels of ``_lib/libfk_decode.so``.  There is no
fallback: if the library is missing or fails, the call raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

from .build import LIB_PATH

FK_DTYPE_F16 = 0
FK_DTYPE_BF16 = 1
FK_DTYPE_E4M3 = 2

FK_STATUS_BAD_PAGE = 1
FK_STATUS_TIMEOUT = 2

_DTYPE_CODES = {
    torch.float16: FK_DTYPE_F16,
    torch.bfloat16: FK_DTYPE_BF16,
    torch.float8_e4m3fn: FK_DTYPE_E4M3,
}

_lib = None
_lib_lock = threading.Lock()

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64
_Z = ctypes.c_size_t


def lib() -> ctypes.CDLL:
    """Load the native library (once).  Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lib_lock:
        if _lib is not None:
            return _lib
        path = os.environ.get("FK_DECODE_LIB", LIB_PATH)  # alternate build, e.g. for A/B timing
        if not os.path.exists(path):
            raise RuntimeError(
                f"fasterkernels_b200 native library not found at {path}; build it with "
                "`python -m fasterkernels_b200.build` (needs nvcc with sm_100a support)")
        L = ctypes.CDLL(path)
        L.fk_version.restype = _I
        L.fk_version.argtypes = []
        L.fk_last_error.restype = ctypes.c_char_p
        L.fk_last_error.argtypes = []
        L.fk_decode_workspace_bytes.restype = _Z
        L.fk_decode_workspace_bytes.argtypes = [_I, _I, _I, _I]
        L.fk_decode_workspace_bytes_gqa.restype = _Z
        L.fk_decode_workspace_bytes_gqa.argtypes = [_I, _I, _I, _I, _I]
        L.fk_flash_decode_gqa_varlen.restype = _I
        L.fk_flash_decode_gqa_varlen.argtypes = [
            _P, _P, _P, _P, _P, _P,          # q k v cu s_aux out
            _I, _I, _I, _I, _L, _I,          # batch q_heads kv_heads head_dim total_tokens dtype
            _L, _L, _L, _L, _L, _L, _L, _L,  # strides
            _P, _Z, _P]
        L.fk_flash_decode_gqa_hf_dense.restype = _I
        L.fk_flash_decode_gqa_hf_dense.argtypes = [
            _P, _P, _P, _P, _P, _P, _P,      # q k v cache_lens starts s_aux out
            _I, _I, _I, _I, _L,              # batch q_heads kv_heads head_dim max_seqlen
            _I, _I, _I,                      # q_dtype kv_dtype out_dtype
            _P, _P, _P,                      # scales
            _L, _L, _L, _L, _L, _L, _L, _L, _L, _L,
            _P, _Z, _P]
        L.fk_paged_flash_decode.restype = _I
        L.fk_paged_flash_decode.argtypes = [
            _P, _P, _P, _P, _P, _P, _P,      # q k v bt seq_lens s_aux out
            _I, _I, _I, _I, _L, _I, _I,      # batch q_heads kv_heads head_dim num_pages page_size max_blocks
            _I, _I, _I,                      # dtypes
            _P, _P, _P,                      # scales
            _L, _L, _L, _L, _L, _L, _L, _L, _L, _L, _L,
            _P, _Z, _P]
        L.fk_paged_kv_append.restype = _I
        L.fk_paged_kv_append.argtypes = [
            _P, _P, _I, _P, _P, _I, _P, _P, _I,  # k_new v_new in_dtype k_pool v_pool pool_dtype bt positions increment
            _P, _P, _P,                          # scale_k scale_v status
            _I, _I, _I, _L, _I,                  # batch kv_heads head_dim num_pages max_blocks
            _L, _L, _L, _L, _L, _L, _L, _L, _L, _L, _L,
            _P]
        L.fk_profile_begin.restype = _I
        L.fk_profile_begin.argtypes = [_I]
        L.fk_profile_end.restype = _I
        L.fk_profile_end.argtypes = [ctypes.POINTER(ctypes.c_float), ctypes.POINTER(_I)]
        L.fk_decode_num_ctas.restype = _I
        L.fk_decode_num_ctas.argtypes = [_I, _I, _I]
        L.fk_debug_configure.restype = _I
        L.fk_debug_configure.argtypes = [ctypes.c_ulonglong, _I]
        _lib = L
        return L


def last_error() -> str:
    msg = lib().fk_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed (code {rc}): {last_error()}")


def dtype_code(t: torch.dtype) -> int:
    try:
        return _DTYPE_CODES[t]
    except KeyError:
        raise TypeError(f"unsupported dtype {t}; expected float16, bfloat16 or float8_e4m3fn") from None


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


# ---------------------------------------------------------------- workspace
_ws = {}
_ws_retired = []
_ws_lock = threading.Lock()


def workspace(device: torch.device, batch: int, q_heads: int, kv_heads: int, kv_dtype_code: int) -> torch.Tensor:
    """The cached workspace of (device, current stream), grown to fit
    (batch, q_heads, kv_heads).

    One workspace per stream: eager decode calls on different streams of a
    device may run concurrently (their arrival counters and partials never
    meet); calls on one stream are ordered by it.  Never allocated during
    CUDA-graph capture: a graph replays the pointer it captured, so run one
    eager call with the largest batch before capturing; a capture stream
    without its own workspace adopts the device's largest one, so replay such
    graphs in order with the eager calls of the warm-up stream.
    """
    idx = device.index if device.index is not None else torch.cuda.current_device()
    need = int(lib().fk_decode_workspace_bytes_gqa(idx, batch, q_heads, kv_heads, kv_dtype_code))
    if need == 0:
        raise RuntimeError(f"fk_decode_workspace_bytes_gqa failed: {last_error()}")
    key = (idx, torch.cuda.current_stream(torch.device("cuda", idx)).cuda_stream)
    with _ws_lock:
        ws = _ws.get(key)
        if ws is None or ws.numel() < need:
            if torch.cuda.is_current_stream_capturing():
                # torch.cuda.graph captures on a side stream: adopt the largest
                # workspace the eager warm-up calls left on this device
                fits = [w for (i, _), w in _ws.items() if i == idx and w.numel() >= need]
                if not fits:
                    raise RuntimeError(
                        "decode workspace must be allocated before CUDA graph capture: run one eager "
                        "decode call with the captured batch size first")
                ws = max(fits, key=lambda w: w.numel())
                _ws[key] = ws
                return ws
            if ws is not None:
                _ws_retired.append(ws)  # a captured graph may still point at it
            size = max(need, 0 if ws is None else ws.numel() * 2)
            ws = torch.zeros(size, dtype=torch.uint8, device=torch.device("cuda", idx))
            _ws[key] = ws
        return ws


def device_workspaces(device=None):
    """The cached workspaces of a device (one per stream that decoded on it)."""
    idx = torch.cuda.current_device() if device is None else torch.device(device).index
    with _ws_lock:
        return [w for (i, _), w in _ws.items() if i == idx]


def read_status(device=None, clear: bool = True) -> int:
    """Read (and by default clear) the sticky FK_STATUS_* word of a device's
    workspaces (OR over its streams).  Synchronises with the device; keep it
    off the hot path.  After FK_STATUS_TIMEOUT the whole workspace is cleared
    when clearing: a kernel that gave up may leave arrival counters mid-count."""
    st = 0
    for ws in device_workspaces(device):
        w = int(ws[:4].view(torch.int32).item())
        st |= w
        if clear:
            if w & FK_STATUS_TIMEOUT:
                ws.zero_()
            else:
                ws[:4].zero_()
    return st


def profile_begin(max_launches: int) -> None:
    """Record CUDA events around the decode kernel of the next
    ``max_launches`` decode calls (on their launching streams)."""
    check(lib().fk_profile_begin(int(max_launches)), "fk_profile_begin")


def profile_end():
    """Stop recording; returns (kernel_ms_total, calls)."""
    a, n = ctypes.c_float(), ctypes.c_int()
    check(lib().fk_profile_end(ctypes.byref(a), ctypes.byref(n)), "fk_profile_end")
    return a.value, n.value
