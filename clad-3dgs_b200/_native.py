"""ctypes binding of libclad3dgs_b200.so, the C ABI declared in include/clad3dgs_b200.h.

There is no fallback: if the library is missing or cannot be loaded, every op
raises. Tensors are passed as raw device pointers; launches go to the given
stream (torch's current stream by default) except the reference drop-in SH
entries, which, like the reference, use the legacy default stream.
"""

from __future__ import annotations

import ctypes
import threading
from ctypes import POINTER, c_bool, c_double, c_float, c_int, c_int64, c_size_t, c_uint, c_void_p
from pathlib import Path

LIBRARY = Path(__file__).resolve().with_name("libclad3dgs_b200.so")

OK, INVALID_ARGUMENT, CUDA_ERROR, DEVICE_FAULT = 0, 1, 2, 3


class AdamConfig(ctypes.Structure):
    _fields_ = [("inv_bias1", c_float), ("inv_bias2", c_float)]


class TorchAdamConfig(ctypes.Structure):
    _fields_ = [("bias1", c_float), ("bias2_sqrt", c_float)]


MAX_RANKS, SHARD_GROUPS, IPC_HANDLE_BYTES = 8, 5, 64


class ShardUpdateArgs(ctypes.Structure):
    """clad3dgs_shard_update_args."""
    _fields_ = [("begin", c_int64), ("end", c_int64), ("grad_origin", c_int64),
                ("ranks", c_int), ("local", c_int),
                ("grads", (c_void_p * SHARD_GROUPS) * MAX_RANKS),
                ("params", (c_void_p * SHARD_GROUPS) * MAX_RANKS),
                ("first", c_void_p * SHARD_GROUPS), ("second", c_void_p * SHARD_GROUPS),
                ("saved_scaling", c_void_p), ("saved_opacity", c_void_p),
                ("saved_norm", c_void_p), ("rates", c_double * (SHARD_GROUPS + 1)),
                ("bias1", c_float), ("bias2_sqrt", c_float),
                ("seeds", c_void_p * MAX_RANKS), ("cameras", c_void_p * MAX_RANKS),
                ("degree", c_int), ("colours", c_void_p * MAX_RANKS),
                ("next_cameras", c_void_p * MAX_RANKS), ("clamp_bits", c_void_p)]


_P = c_void_p
_PP = POINTER(c_void_p)
# char* (*)(void* ctx, int which, size_t bytes): device buffer for the rasterizer.
ALLOC_FN = ctypes.CFUNCTYPE(c_void_p, c_void_p, c_int, c_size_t)
_SIGNATURES = {
    "sh_consumer_sgd": (None, [c_int, c_int, _P, _P, _P, _P, _P, _P, _P]),
    "sh_consumer_adam": (None, [c_int, c_int, _P, _P, _P, _P, _P, _P, _P, _P, _P, AdamConfig]),
    "sh_consumer_split_adam": (None, [c_int, c_int] + [_P] * 13 + [AdamConfig]),
    "sh_consumer_split_torch_adam": (None, [c_int, c_int] + [_P] * 13 + [TorchAdamConfig]),
    "launch_activation_consume": (None, [c_int, _PP, _PP, _PP, _PP, _PP, POINTER(c_double),
                                         POINTER(c_float), POINTER(c_float), _P]),
    "launch_quaternion_backward": (None, [c_int, _P, _P, _P, _P, _P]),
    "clad3dgs_last_error": (ctypes.c_char_p, []),
    "clad3dgs_describe": (c_int, [POINTER(c_int)] * 4),
    "clad3dgs_fault_status": (c_int, [c_int, POINTER(c_uint)]),
    "clad3dgs_sh_consume_split_torch_adam": (c_int, [c_int64, c_int] + [_P] * 13
                                             + [TorchAdamConfig, _P]),
    "clad3dgs_sh_consume_variant": (c_int, [c_int, c_int64, c_int] + [_P] * 16
                                    + [AdamConfig, _P]),
    "clad3dgs_activation_consume": (c_int, [c_int64, _PP, _PP, _PP, _PP, _PP, POINTER(c_double),
                                            POINTER(c_float), POINTER(c_float), _P]),
    "clad3dgs_quaternion_backward": (c_int, [c_int64, _P, _P, _P, _P, _P]),
    "clad3dgs_gaussian_step": (c_int, [c_int64, c_int] + [_P] * 13 + [TorchAdamConfig]
                               + [_PP] * 5 + [POINTER(c_double), POINTER(c_float),
                                              POINTER(c_float), _P]),
    "clad3dgs_host_step_workspace": (c_size_t, [c_int64]),
    "clad3dgs_gaussian_step_host": (c_int, [c_int64, c_int] + [_P] * 12 + [TorchAdamConfig]
                                    + [_PP] * 5 + [POINTER(c_double), POINTER(c_float),
                                                   POINTER(c_float), _P, c_size_t, c_int64,
                                                   _P]),
    "clad3dgs_raster_geom_bytes": (c_size_t, [c_int]),
    "clad3dgs_raster_image_bytes": (c_size_t, [c_int, c_int]),
    "clad3dgs_raster_binning_bytes": (c_size_t, [c_int] * 4),
    "clad3dgs_raster_forward": (c_int, [c_int, c_int] + [_P] * 5 + [c_float] + [_P] * 4
                                + [c_float, c_float, c_int, c_int] + [_P] * 4
                                + [c_int, _P, _P, _P, _P, _P, POINTER(c_int), _P]),
    "clad3dgs_raster_render_backward": (c_int, [c_int, c_int, c_int] + [_P] * 3 + [c_int]
                                        + [_P] * 8 + [c_int, _P]),
    "clad3dgs_raster_count_accumulation": (c_int, [c_int] * 3 + [_P] * 2 + [c_int] + [_P] * 3),
    "clad3dgs_warp_accumulate_probe": (c_int, [c_int] * 3 + [_P] * 4 + [c_int, _P]
                                       + [c_int] * 3 + [_P]),
    "clad3dgs_raster_backward": (c_int, [c_int, c_int] + [_P] * 6 + [c_float] + [_P] * 4
                                 + [c_float, c_float, c_int, c_int] + [_P] * 7 + [c_int]
                                 + [_P] * 2 + [c_int] + [_P] * 10 + [c_int, c_int]
                                 + [_P] * 6 + [TorchAdamConfig, _P, _P, c_double,
                                               TorchAdamConfig, _P]),
    "clad3dgs_raster_sh_backward": (c_int, [c_int, c_int] + [_P] * 11),
    "clad3dgs_raster_sh_seeds": (c_int, [c_int] + [_P] * 5),
    "clad3dgs_raster_forward_2d": (c_int, [c_int] + [_P] * 5 + [c_int, c_int, _P, _P, _P,
                                                               _P, _P, POINTER(c_int), _P]),
    "clad3dgs_gaussian_step_host_static": (c_int, [c_int64, c_int] + [_P] * 12
                                           + [TorchAdamConfig] + [_PP] * 5
                                           + [POINTER(c_double), POINTER(c_float),
                                              POINTER(c_float), c_int64, _P]),
    "clad3dgs_sh_consume_xyz": (c_int, [c_int64, c_int] + [_P] * 13 + [TorchAdamConfig]
                                + [_P, _P, c_double, TorchAdamConfig, _P]),
    "clad3dgs_gaussian_step_xyz": (c_int, [c_int64, c_int] + [_P] * 13 + [TorchAdamConfig]
                                   + [_PP] * 5 + [POINTER(c_double), POINTER(c_float),
                                                  POINTER(c_float)]
                                   + [_P, _P, c_double, TorchAdamConfig, _P]),
    "clad3dgs_activate": (c_int, [c_int64] + [_P] * 7 + [_P]),
    "clad3dgs_l1_loss": (c_int, [c_int64, _P, _P, _P, _P, _P]),
    "clad3dgs_shard_update": (c_int, [POINTER(ShardUpdateArgs), _P]),
    "clad3dgs_shard_colours": (c_int, [POINTER(ShardUpdateArgs), _P]),
    "clad3dgs_ipc_alloc": (c_int, [c_size_t, POINTER(c_void_p), POINTER(ctypes.c_ubyte)]),
    "clad3dgs_ipc_free": (c_int, [_P]),
    "clad3dgs_ipc_open": (c_int, [POINTER(ctypes.c_ubyte), POINTER(c_void_p)]),
    "clad3dgs_ipc_close": (c_int, [_P]),
}

_lock = threading.Lock()
_lib = None


def library() -> ctypes.CDLL:
    """Loads the C-ABI library once; raises if it is not built."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIBRARY.exists():
                raise RuntimeError(
                    f"{LIBRARY.name} is not built; run clad-3dgs_b200/build_native.py "
                    "(or __graft_entry__.build()) first")
            lib = ctypes.CDLL(str(LIBRARY))
            for name, (restype, argtypes) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = lib
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def check(status: int, what: str) -> None:
    if status != OK:
        message = library().clad3dgs_last_error().decode(errors="replace")
        kind = ValueError if status == INVALID_ARGUMENT else RuntimeError
        raise kind(f"{what}: {message or 'status ' + str(status)}")


def pointer_array(values) -> ctypes.Array:
    return (c_void_p * len(values))(*[int(v) for v in values])


def doubles(values) -> ctypes.Array:
    return (c_double * len(values))(*[float(v) for v in values])


def floats(values) -> ctypes.Array:
    return (c_float * len(values))(*[float(v) for v in values])


def ptr(tensor) -> int | None:
    """Raw data pointer of a tensor (None for None or an empty tensor)."""
    if tensor is None or tensor.numel() == 0:
        return None
    return tensor.data_ptr()


def stream_handle(stream=None) -> int:
    import torch

    s = torch.cuda.current_stream() if stream is None else stream
    return s.cuda_stream


def fault_status(clear: bool = True) -> int:
    word = c_uint(0)
    library().clad3dgs_fault_status(int(clear), ctypes.byref(word))
    return int(word.value)


def describe() -> dict:
    vals = [c_int(0) for _ in range(4)]
    library().clad3dgs_describe(*[ctypes.byref(v) for v in vals])
    return dict(sm_count=vals[0].value, tile_gaussians=vals[1].value,
                sh_stages=vals[2].value, fused_stages=vals[3].value)
