"""Loader for the gsplat_b200 C ABI (libgsplat_b200.so, include/gsplat_b200.h).

The shared library is built in-tree by ``python -m gsplat_b200.csrc.build``. There
is no fallback: every op raises ``RuntimeError`` when the library is missing or a
tensor is not on a CUDA device, so a silent CPU or library path can never stand in
for the kernels.
"""

import ctypes
import os
import threading
import time
from typing import Optional

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "libgsplat_b200.so")

_lib = None
_lock = threading.Lock()

P = ctypes.c_void_p
I32 = ctypes.c_int
I64 = ctypes.c_longlong
F32 = ctypes.c_float
SZ = ctypes.c_size_t


class GsbPeerGroup(ctypes.Structure):
    """Mirror of ``GsbPeerGroup`` in include/gsplat_b200.h."""

    _fields_ = [
        ("arena", P * 8),
        ("recv_offset", I64),
        ("recv_stride", I64),
        ("grad_offset", I64),
        ("rank", I32),
        ("world", I32),
        ("error", P),
    ]


class GsbAdamGroup(ctypes.Structure):
    """Mirror of ``GsbAdamGroup`` in include/gsplat_b200.h."""

    _fields_ = [
        ("param", P),
        ("grad", P),
        ("exp_avg", P),
        ("exp_avg_sq", P),
        ("numel", I64),
        ("D", I32),
        ("lr", F32),
        ("eps", F32),
    ]


# name -> (restype, argtypes); must match include/gsplat_b200.h.
_PROJ_COMMON = [I32, I32, I32, P, P, P, P, P, P, P, I32, I32, F32, F32, F32, F32, I32, I32]
SIGNATURES = {
    "gsb_last_error": (ctypes.c_char_p, []),
    "gsb_version": (I32, []),
    "gsb_projection_fused_fwd": (I32, _PROJ_COMMON + [P, P, P, P, P, P]),
    "gsb_projection_fused_bwd": (
        I32,
        [I32, I32, I32, P, P, P, P, P, P, I32, I32, F32, I32, P, P, P, P, P, P, P, P, P, P, P, P, P],
    ),
    "gsb_projection_packed_blocks": (I32, [I32]),
    "gsb_projection_packed_count": (I32, _PROJ_COMMON + [P, P, P]),
    "gsb_projection_packed_write": (I32, _PROJ_COMMON + [P, P, I64, P, P, P, P, P, P, P, P, P, P]),
    "gsb_projection_packed_bwd": (
        I32,
        [I32, I32, I32, I32, P, P, P, P, P, P, I32, I32, F32, I32, P, P, P, P, P, P, P, P, P, I32,
         P, P, P, P, P, P],
    ),
    "gsb_projection_sh_dense_fwd": (
        I32,
        [I32, I32, I32, P, P, P, P, P, I32, I32, P, P, I32, I32, F32, F32, F32, F32, I32, I32,
         P, P, P, P, P, P, P, P],
    ),
    "gsb_projection_sh_packed_write": (
        I32,
        [I32, I32, I32, P, P, P, P, P, I32, I32, P, P, I32, I32, F32, F32, F32, F32, I32, I32,
         P, P, I64, P, P, P, P, P, P, P, P, P, P, P, P, P],
    ),
    "gsb_projection_sh_bwd": (
        I32,
        [I32, I32, I32, I32, P, P, P, P, P, I32, I32, P, P, I32, I32, F32, I32, I32,
         P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P],
    ),
    "gsb_quat_scale_to_covar_preci_fwd": (I32, [I64, P, P, I32, P, P, P]),
    "gsb_quat_scale_to_covar_preci_bwd": (I32, [I64, P, P, I32, P, P, P, P, P]),
    "gsb_proj_fwd": (I32, [I32, I32, I32, P, P, P, I32, I32, I32, P, P, P]),
    "gsb_proj_bwd": (I32, [I32, I32, I32, P, P, P, I32, I32, I32, P, P, P, P, P]),
    "gsb_rasterize_to_indices": (I32, [I32, I32, I32, I32, I64, P, P, P, I32, I32, I32, I32, I32, P, P, P, P, P, P,
                                       P, P]),
    "gsb_densify_accumulate": (I32, [I64, I32, P, P, P, I32, I32, I32, P, P, P, P]),
    "gsb_spherical_harmonics_fwd": (I32, [I32, I64, I32, P, P, P, P, P]),
    "gsb_spherical_harmonics_bwd": (I32, [I32, I64, I32, P, P, P, P, P, P, P]),
    "gsb_scan_scratch_bytes": (SZ, [I64]),
    "gsb_inclusive_scan_i32": (I32, [P, P, I64, P, SZ, P]),
    "gsb_inclusive_scan_i32_noalloc": (I32, [P, P, I64, P]),
    "gsb_isect_key_bits": (I32, [I32, I32, I32]),
    "gsb_isect_count": (I32, [I32, I32, I32, I32, P, P, P, P, P, P, I32, I32, I32, P, P]),
    "gsb_isect_emit": (I32, [I32, I32, I32, I32, P, P, P, P, P, P, I32, I32, I32, P, P, P, P]),
    "gsb_radix_sort_scratch_bytes": (SZ, [I64]),
    "gsb_radix_sort_pairs": (I32, [P, P, P, P, I64, I32, P, SZ, P]),
    "gsb_isect_offset_encode": (I32, [P, I64, I32, I32, I32, P, P]),
    "gsb_isect_count_tiles": (I32, [I32, I32, I32, I32, P, P, P, P, P, P, I32, I32, I32, P, P, P, P]),
    "gsb_isect_bucket_shards": (I32, [I32, I32, I32]),
    "gsb_isect_bucket_offsets_scratch_bytes": (SZ, [I64, I32]),
    "gsb_isect_bucket_offsets": (I32, [P, I64, I32, P, P, P, P, P, P, P, SZ, P]),
    "gsb_isect_bucket_emit": (I32, [I32, I32, I32, I32, P, P, P, P, P, P, I32, I32, I32, I64, P, P, P]),
    "gsb_isect_bucket_sort_max": (I32, []),
    "gsb_pack_rows": (I32, [I64, P, I32, P, P, P, P]),
    "gsb_unpack_rows": (I32, [I64, P, I32, P, I32, P, P, P]),
    "gsb_peer_mailbox_bytes": (ctypes.c_size_t, []),
    "gsb_peer_alloc": (I32, [ctypes.c_size_t, P, P]),
    "gsb_peer_open": (I32, [P, P]),
    "gsb_peer_close": (I32, [P]),
    "gsb_peer_free": (I32, [P]),
    "gsb_peer_set_wait_limit": (I64, [I64]),
    "gsb_peer_error_alloc": (I32, [P, P]),
    "gsb_peer_error_free": (I32, [P]),
    "gsb_peer_send_rows": (I32, [P, ctypes.c_ulonglong, I64, P, P, P, I32, I64, I32, P, P, P]),
    "gsb_peer_recv_rows": (I32, [P, ctypes.c_ulonglong, I64, P, P, P, I32, I64, I32, P, P, P]),
    "gsb_peer_send_grads": (I32, [P, ctypes.c_ulonglong, I64, P, P, I64, I32, P, P, P]),
    "gsb_peer_recv_grads": (I32, [P, ctypes.c_ulonglong, I64, P, I32, P, P, P]),
    "gsb_exchange_ids": (I32, [I64, P, P, P, I32, P, P, P, P]),
    "gsb_isect_bucket_sort": (I32, [I32, I32, I32, P, P, I32, I32, I32, P, P, P, P, P]),
    "gsb_isect_bucket_sort_scratch_bytes": (SZ, [I64]),
    "gsb_isect_bucket_sort_ex": (I32, [I32, I32, I32, P, P, I32, I32, I32, P, P, I64, P, SZ, P, P, P, P]),
    "gsb_rasterize_fwd": (
        I32,
        [I32, I32, P, P, P, P, P, P, I32, I32, I32, I32, I32, P, P, I64, P, P, P, P],
    ),
    "gsb_rasterize_fwd_counted": (
        I32,
        [I32, I32, P, P, P, P, P, P, I32, I32, I32, I32, I32, P, P, I64, P, P, P, P, P],
    ),
    "gsb_rasterize_fwd_ex": (
        I32,
        [I32, I32, P, P, P, P, P, P, I32, I32, I32, I32, I32, P, P, I64, P, P, P, P, P, P],
    ),
    "gsb_rasterize_bwd_ex": (
        I32,
        [I32, I32, P, P, P, P, P, P, I32, I32, I32, I32, I32, P, P, I64, P, P, P, P, P, P, P, P,
         P, P, P],
    ),
    "gsb_fp32_fma_probe": (I32, [P, I32, I32, I32, P]),
    "gsb_rasterize_bwd": (
        I32,
        [I32, I32, P, P, P, P, P, P, I32, I32, I32, I32, I32, P, P, I64, P, P, P, P, P, P, P, P,
         P, P],
    ),
    "gsb_adam": (I32, [P, P, P, P, P, I64, I64, F32, F32, F32, F32, P]),
    "gsb_adam_multi": (I32, [I32, ctypes.POINTER(GsbAdamGroup), P, F32, F32, P]),
}


def _load():
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                "gsplat_b200 CUDA library is not built (expected "
                f"{LIB_PATH}); run `python -m gsplat_b200.csrc.build`."
            )
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def lib():
    return _lib if _lib is not None else _load()


def is_available() -> bool:
    try:
        lib()
        return True
    except (RuntimeError, OSError):
        return False


# Optional per-entry-point timing: when a dict is installed here (bench.py does
# this), every call (or, with ``timing_names`` a set, every call of those entry
# points) records a pair of CUDA events on the current stream of the current
# device around the launch, keyed by entry-point name. ``calls``, when a dict,
# counts the calls by entry point (no events).
timing = None
timing_names = None
calls = None


def call(name: str, *args) -> int:
    """Calls a C-ABI function and raises RuntimeError on a negative status."""
    fn = getattr(lib(), name)
    if calls is not None:
        calls[name] = calls.get(name, 0) + 1
    if timing is not None and (timing_names is None or name in timing_names):
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        rc = fn(*args)
        end.record()
        timing.setdefault(name, []).append((start, end))
    else:
        rc = fn(*args)
    if isinstance(rc, int) and rc < 0:
        msg = lib().gsb_last_error()
        raise RuntimeError(msg.decode() if msg else f"{name} failed with status {rc}")
    return rc


# Optional accounting of the host time spent blocked in device-to-host reads of
# sizes (the wrapper's only synchronising calls): when a two-element list
# [seconds, reads] is installed here, read_back() adds to it.
host_wait = None


def read_back(t: torch.Tensor) -> list:
    """``t.tolist()``: a blocking device-to-host read of a few values."""
    if host_wait is None:
        return t.tolist()
    t0 = time.perf_counter()
    out = t.tolist()
    host_wait[0] += time.perf_counter() - t0
    host_wait[1] += 1
    return out


def wait_event(ev) -> None:
    """``ev.synchronize()``, accounted like read_back()."""
    if host_wait is None:
        ev.synchronize()
        return
    t0 = time.perf_counter()
    ev.synchronize()
    host_wait[0] += time.perf_counter() - t0
    host_wait[1] += 1


def ptr(t: Optional[torch.Tensor]):
    """Device pointer of a CUDA tensor (None -> NULL)."""
    if t is None:
        return None
    return t.data_ptr()


def check_cuda(name: str, t: Optional[torch.Tensor]) -> None:
    if t is None:
        return
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def stream_of(t: torch.Tensor) -> int:
    """Raw handle of the current CUDA stream of t's device."""
    return torch._C._cuda_getCurrentRawStream(t.device.index)


class _NoGuard:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


_NO_GUARD = _NoGuard()


def device_guard(device: torch.device):
    """torch.cuda.device(device), skipped when that device is already current
    (the common case: it saves a device switch and restore per call)."""
    if device.type == "cuda" and device.index == torch.cuda.current_device():
        return _NO_GUARD
    return torch.cuda.device(device)
