"""ctypes binding of liblizard_cuda.so (the C ABI in include/lizard_cuda.h).

The shared library is built in-tree by lizard-reproduction_b200/csrc/build.py.
There is no fallback: if the library is missing or its ABI revision differs,
every call raises.
"""
import contextlib
import ctypes
import threading
from pathlib import Path

import torch

ABI_VERSION = 3
LIB_PATH = Path(__file__).resolve().with_name("liblizard_cuda.so")
HEADER = Path(__file__).resolve().parents[2] / "include" / "lizard_cuda.h"

LZ_DTYPE_F32 = 0
LZ_DTYPE_BF16 = 1
LZ_ERR_UNSUPPORTED = 2

_c_int, _c_size, _vp = ctypes.c_int, ctypes.c_size_t, ctypes.c_void_p
_SIGNATURES = {
    "lz_abi_version": (_c_int, []),
    "lz_last_error_string": (ctypes.c_char_p, []),
    "lz_launch_count": (ctypes.c_uint64, []),
    "lz_device_timeout_flag": (_c_int, [ctypes.POINTER(ctypes.c_uint)]),
    "lz_device_timeout_clear": (_c_int, []),
    "lz_test_withhold_decode_ring_copy": (_c_int, [_c_int]),
    "lz_gla_saved_bytes": (_c_size, [_c_int] * 6),
    "lz_gla_bwd_workspace_bytes": (_c_size, [_c_int] * 6),
    "lz_gla_fwd_workspace_bytes": (_c_size, [_c_int] * 6),
    "lz_gla_set_schedule": (_c_int, [_c_int]),
    "lz_gla_set_split_out_tc": (_c_int, [_c_int]),
    "lz_gla_set_fwd_tc64": (_c_int, [_c_int]),
    "lz_gla_set_bwd_prefetch": (_c_int, [_c_int]),
    "lz_gla_fwd": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _vp, _vp, _c_size, _vp, _c_size]
                   + [_c_int] * 6 + [_vp]),
    "lz_gla_bwd": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _vp, _c_size, _vp, _vp, _vp, _vp, _c_int,
                            _vp, _vp, _c_size] + [_c_int] * 6 + [_vp]),
    "lz_gla_bwd_gqa_workspace_bytes": (_c_size, [_c_int] * 7),
    "lz_gla_fwd_gqa_workspace_bytes": (_c_size, [_c_int] * 9),
    "lz_gla_fwd_gqa": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _vp, _vp, _c_size, _vp, _c_size]
                       + [_c_int] * 7 + [_vp]),
    "lz_gla_bwd_gqa": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _vp, _c_size, _vp, _vp, _vp, _vp,
                                _c_int, _vp, _vp, _c_size] + [_c_int] * 7 + [_vp]),
    "lz_gla_seg_workspace_bytes": (_c_size, [_c_int] * 5),
    "lz_gla_seg_summary_floats": (_c_size, [_c_int] * 4),
    "lz_gla_seg_fwd_begin": (_c_int, [_vp, _vp, _vp, _c_int, _vp, _vp, _c_size] + [_c_int] * 5
                             + [_vp]),
    "lz_gla_seg_fwd_end": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _vp, _vp, _vp, _c_size, _vp,
                                    _c_size] + [_c_int] * 5 + [_vp]),
    "lz_gla_seg_bwd_begin": (_c_int, [_vp, _vp, _c_size, _vp, _vp, _vp, _c_size] + [_c_int] * 5
                             + [_vp]),
    "lz_gla_seg_bwd_end": (_c_int, [_vp, _vp, _vp, _c_int, _vp, _c_size, _vp, _vp, _c_int, _vp,
                                    _vp, _vp, _c_int, _vp, _vp, _c_size] + [_c_int] * 5 + [_vp]),
    "lz_gla_seg_combine": (_c_int, [_vp, _c_int, _c_int, _c_int, _vp] + [_c_int] * 4 + [_vp]),
    "lz_gla_seg_gate_offset": (_c_int, [_vp, _vp] + [_c_int] * 4 + [_vp]),
    "lz_hedgehog_fwd": (_c_int, [_vp, _c_int, _vp, _vp, _c_int, _c_int, _c_int, _vp]),
    "lz_hedgehog_bwd": (_c_int, [_vp, _c_int, _vp, _vp, _c_int, _vp, _vp, _vp, _c_size, _c_int,
                                 _c_int, _c_int, _vp]),
    "lz_hedgehog_bwd_workspace_bytes": (_c_size, [_c_int] * 3),
    "lz_hedgehog_set_tc": (_c_int, [_c_int]),
    "lz_hedgehog_set_rows_max": (ctypes.c_longlong, [ctypes.c_longlong]),
    "lz_swa_set_tc": (_c_int, [_c_int]),
    "lz_hedgehog_fwd_strided": (_c_int, [_vp, _c_int, ctypes.c_longlong, ctypes.c_longlong, ctypes.c_longlong, _c_int, _c_int, _c_int,
                                         _vp, _vp, _c_int, _c_int, _vp]),
    "lz_hedgehog_bwd_strided": (_c_int, [_vp, _c_int, ctypes.c_longlong, ctypes.c_longlong, ctypes.c_longlong, _c_int, _c_int, _c_int,
                                         _vp, _vp, _c_int, _vp, _vp, _vp, _c_size, _c_int,
                                         _c_int, _vp]),
    "lz_rope_split": (_c_int, [_vp, _c_int, ctypes.c_longlong, ctypes.c_longlong,
                               ctypes.c_longlong, _vp, _vp, _c_int, ctypes.c_longlong,
                               ctypes.c_longlong, _vp, _vp] + [_c_int] * 4 + [_vp]),
    "lz_rope_bwd": (_c_int, [_vp, _vp, _vp, _c_int, ctypes.c_longlong, ctypes.c_longlong, _vp,
                             _c_int] + [_c_int] * 4 + [_vp]),
    "lz_blend_fwd": (_c_int, [_vp, _vp, _vp, _vp] + [_c_int] * 5 + [_vp]),
    "lz_blend_bwd_workspace_bytes": (_c_size, [_c_int] * 4),
    "lz_blend_bwd": (_c_int, [_vp, _c_int, _vp, _vp, _vp, _vp, _vp, _vp, _c_size] + [_c_int] * 4
                     + [_vp]),
    "lz_gla_decode": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _vp, _vp, _vp] + [_c_int] * 6 + [_vp]),
    "lz_swa_decode": (_c_int, [_vp, _vp, _vp, _c_int] + [ctypes.c_longlong] * 6 + [_vp, _vp, _c_int, ctypes.c_longlong,
                                                                     _vp, _vp, _vp, _vp, _c_int,
                                                                     _vp] + [_c_int] * 5 + [_vp]),
    "lz_swa_rope_fwd": (_c_int, [_vp, _vp, _vp, _c_int] + [ctypes.c_longlong] * 9 + [_vp, _vp, _c_int, ctypes.c_longlong,
                                                                     ctypes.c_longlong, _vp, _c_int, _c_int,
                                                                     _vp, _vp, _c_size, _vp, _vp,
                                                                     _vp, _vp] + [_c_int] * 5
                        + [_vp]),
    "lz_swa_saved_bytes": (_c_size, [_c_int] * 4),
    "lz_swa_bwd_workspace_bytes": (_c_size, [_c_int] * 5),
    "lz_swa_fwd": (_c_int, [_vp] * 6 + [_c_int, _c_int, _vp, _vp, _c_size] + [_c_int] * 4
                   + [_vp]),
    "lz_swa_bwd": (_c_int, [_vp] * 6 + [_c_int, _c_int, _vp, _c_size, _vp, _vp, _vp, _vp,
                                        _c_int, _vp, _vp, _c_size] + [_c_int] * 4 + [_vp]),
    "lz_swa_fwd_gqa": (_c_int, [_vp] * 6 + [_c_int, _c_int, _vp, _vp, _c_size] + [_c_int] * 5
                       + [_vp]),
    "lz_swa_bwd_gqa": (_c_int, [_vp] * 6 + [_c_int, _c_int, _vp, _c_size, _vp, _vp, _vp, _vp,
                                            _c_int, _vp, _vp, _c_size] + [_c_int] * 5 + [_vp]),
    "lz_swa_bwd_noalloc": (_c_int, [_vp] * 6 + [_c_int, _c_int, _vp, _c_size, _vp, _vp, _vp,
                                                _vp, _c_int, _vp] + [_c_int] * 4 + [_vp]),
}

_lock = threading.Lock()
_lib = None


def load():
    """Load and type the library once per process."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH.name} is not built; run "
                    "`python lizard-reproduction_b200/csrc/build.py` first")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype, fn.argtypes = res, args
            if lib.lz_abi_version() != ABI_VERSION:
                raise RuntimeError(f"{LIB_PATH.name} has ABI {lib.lz_abi_version()}, "
                                   f"this module expects {ABI_VERSION}")
            _lib = lib
    return _lib


def check(rc, what):
    if rc != 0:
        msg = load().lz_last_error_string().decode(errors="replace")
        raise RuntimeError(f"lizard_cuda {what} failed (code {rc}): {msg}")


def launch_count():
    return int(load().lz_launch_count())


def device_timeout_flag():
    """Site of the first bounded wait that gave up on the current device (0 = none)."""
    out = ctypes.c_uint(0)
    check(load().lz_device_timeout_flag(ctypes.byref(out)), "timeout flag query")
    return int(out.value)


_size_cache = {}


def size_query(name, *args):
    """The library's buffer-size query `name`(*args), remembered per argument
    tuple: the sizes depend only on the shape and the GLA schedule switch, and
    set_schedule clears what is remembered. (Every call still checks the sizes
    it is given, so a wrong size raises instead of corrupting memory.)"""
    key = (name,) + args
    hit = _size_cache.get(key)
    if hit is None:
        hit = int(getattr(load(), name)(*args))
        _size_cache[key] = hit
    return hit


def clear_device_timeout_flag():
    """Clear the current device's timeout flag once a timeout has been handled."""
    check(load().lz_device_timeout_clear(), "timeout flag clear")


SCHEDULES = {"auto": 0, "walk": 1, "split": 2}


def set_schedule(name):
    """Process-wide GLA schedule ("auto", "walk" or "split"); returns the previous name."""
    _size_cache.clear()
    prev = load().lz_gla_set_schedule(SCHEDULES[name])
    if prev < 0:
        check(-prev, "set schedule")
    return {v: k for k, v in SCHEDULES.items()}[prev]


def ptr(t):
    """Device address of a tensor as a plain int (ctypes passes it as void*)."""
    return None if t is None else t.data_ptr()


def stream_of(t):
    return torch.cuda.current_stream(t.device).cuda_stream


def on_device(device):
    """Make `device` current for a library call; a no-op when it already is,
    which saves the device switch on every call of the common single-GPU case."""
    if device.index is None or device.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(device)


def require_cuda(*tensors):
    for t in tensors:
        if not (isinstance(t, torch.Tensor) and t.is_cuda):
            raise RuntimeError("lizard_cuda runs on CUDA tensors only (no CPU path); "
                               f"got {type(t).__name__} on "
                               f"{getattr(t, 'device', 'n/a')}")
    dev = tensors[0].device
    for t in tensors[1:]:
        if t.device != dev:
            raise RuntimeError(f"lizard_cuda: tensors on different devices ({dev}, {t.device})")
