"""ctypes binding of libmpo_b200.so (the C ABI declared in include/mpo_b200.h).

This is the reference's kernel-dispatch layer re-targeted at B200: where the
reference compiles Metal sources with ``torch.mps.compile_shader`` and calls
``library.<kernel>(...)`` (mps_pointops/ops.py:33-37), this module loads the
prebuilt sm_100a library once and calls its ``extern "C"`` entry points with
raw device pointers and the current CUDA stream.

There is no fallback: if the library is missing, does not load, or the device
is not an sm_100 part, every call raises ``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

LIB_NAME = "libmpo_b200.so"
ABI_VERSION = 9
_lib = None
_lock = threading.Lock()
_checked_devices: set[int] = set()

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_f32 = ctypes.c_float
_i32 = ctypes.c_int32
_sz = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/mpo_b200.h one to one.
SIGNATURES = {
    "mpo_abi_version": (ctypes.c_int32, []),
    "mpo_last_error": (ctypes.c_char_p, []),
    "mpo_device_supported": (_int, [_int]),
    "mpo_launch_count": (ctypes.c_uint64, []),
    "mpo_fps_workspace_bytes": (_sz, [_i64, _i64, _i64, _int]),
    "mpo_fps": (_int, [_vp, _i64, _i64, _i64, _i64, _int, _int, _int, _vp, _vp, _vp, _sz, _vp]),
    "mpo_fps_gather": (_int, [_vp, _i64, _i64, _i64, _i64, _int, _int, _int, _vp, _vp, _vp, _vp,
                              _sz, _vp]),
    "mpo_gather_points_backward": (_int, [_vp, _vp, _i64, _i64, _i64, _vp, _vp]),
    "mpo_fps_noalloc": (_int, [_vp, _i64, _i64, _i64, _i64, _int, _int, _int, _vp, _vp, _vp]),
    "mpo_knn_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64, _i64]),
    "mpo_index_check": (_int, [_vp, _int, _i64, _i64, _vp, _vp]),
    "mpo_knn": (_int, [_vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _sz, _vp]),
    "mpo_ball_query": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _f32, _vp, _vp, _vp]),
    "mpo_ball_query_pointnet2": (_int, [_vp, _vp, _i64, _i64, _i64, _i64, _f32, _vp, _vp]),
    "mpo_ball_query_backward": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp,
                                       _vp]),
    "mpo_three_nn": (_int, [_vp, _vp, _i64, _i64, _i64, _vp, _vp, _vp]),
    "mpo_three_interpolate": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp]),
    "mpo_three_interpolate_backward": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp]),
    "mpo_chamfer_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64, _int]),
    "mpo_chamfer_loss_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64, _int]),
    "mpo_chamfer_loss": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _int, _int,
                                _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "mpo_chamfer_loss_backward": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _int,
                                         _int, _vp, _vp, _vp, _vp, _vp, _vp]),
    "mpo_chamfer_nearest": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _vp, _vp,
                                   _vp, _vp, _vp, _sz, _vp]),
    "mpo_chamfer_backward": (_int, [_vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp,
                                    _vp, _vp]),
    "mpo_chamfer_nearest_l1": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _vp,
                                      _vp, _vp, _vp, _vp]),
    "mpo_chamfer_l1_backward": (_int, [_vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _vp,
                                       _vp, _vp, _vp]),
    "mpo_chamfer_check_inputs": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp]),
    "mpo_gather_rows": (_int, [_vp, _i64, _i64, _i64, _vp, _int, _i64, _vp, _i64, _vp, _i64,
                                _i64, _vp]),
    "mpo_gather_rows_backward": (_int, [_vp, _i64, _i64, _i64, _i64, _i64, _vp, _int, _i64,
                                         _i64, _vp, _vp, _vp]),
    "mpo_flat_interpolate": (_int, [_vp, _i64, _i64, _vp, _vp, _i64, _i64, _vp, _vp]),
    "mpo_flat_interpolate_backward": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp]),
    "mpo_chamfer_nearest_f64": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _int,
                                       _vp, _vp, _vp, _vp, _vp]),
    "mpo_chamfer_backward_f64": (_int, [_vp, _vp, _i64, _i64, _i64, _i64, _int, _vp, _vp, _vp,
                                        _vp, _vp, _vp, _vp]),
    "mpo_flat_knn": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _vp,
                            _vp]),
    "mpo_flat_radius": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _f32, _i64, _int, _vp, _vp,
                               _vp]),
    "mpo_group_points_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64, _i64]),
    "mpo_group_points": (_int, [_vp, _vp, _int, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _sz,
                                _vp]),
    "mpo_query_and_group_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64, _i64]),
    "mpo_group_points_backward": (_int, [_vp, _vp, _int, _i64, _i64, _i64, _i64, _i64, _vp,
                                         _vp, _sz, _vp]),
    "mpo_query_and_group": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _f32, _int,
                                   _vp, _vp, _vp, _sz, _vp]),
    "mpo_query_and_group_backward": (_int, [_vp, _vp, _i64, _i64, _i64, _i64, _i64, _int, _vp,
                                            _vp, _vp, _vp, _sz, _vp]),
    "mpo_grid_workspace_bytes": (_sz, [_i64, _i64]),
    "mpo_grid_build": (_int, [_vp, _i64, _vp, _f32, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "mpo_grid_knn": (_int, [_vp, _i64, _vp, _f32, _vp, _vp, _vp, _vp, _i32, _i64, _vp, _vp, _vp]),
    "mpo_grid_ball_query": (_int, [_vp, _i64, _vp, _f32, _vp, _vp, _vp, _f32, _f32, _i64, _vp,
                                   _vp, _vp]),
    "mpo_flat_fps_workspace_bytes": (_sz, [_i64, _i64]),
    "mpo_flat_fps": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _sz,
                            _vp]),
    "mpo_p2p_slots_bytes": (_sz, []),
    "mpo_p2p_slots_create": (_int, [_vp, _vp]),
    "mpo_p2p_slots_open": (_int, [_vp, _vp]),
    "mpo_p2p_slots_close": (_int, [_vp]),
    "mpo_p2p_slots_destroy": (_int, [_vp]),
    "mpo_allreduce_sum_f32_p2p": (_int, [_vp, _f32, _vp, _vp, _i64, _i64, ctypes.c_uint32, _i64,
                                         _vp, _vp]),
}


def library_path() -> Path:
    env = os.environ.get("MPO_B200_LIB")
    if env:
        return Path(env)
    return Path(__file__).resolve().parent / "_lib" / LIB_NAME


def lib():
    """The loaded library (loaded on first use)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = library_path()
        if not path.exists():
            raise RuntimeError(
                f"mps_pointops: native library {path} is missing; build it with "
                "`python mps-pointops_b200/build.py` (there is no fallback path)")
        handle = ctypes.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        got = handle.mpo_abi_version()
        if got != ABI_VERSION:
            raise RuntimeError(f"mps_pointops: {path} has ABI {got}, expected {ABI_VERSION}")
        _lib = handle
    return _lib


def launch_count() -> int:
    """Kernels launched by libmpo_b200.so so far in this process."""
    return int(lib().mpo_launch_count())


def last_error() -> str:
    return lib().mpo_last_error().decode("utf-8", "replace")


def check(status: int, what: str) -> None:
    if status != 0:
        raise RuntimeError(f"mps_pointops: {what} failed (status {status}): {last_error()}")


def require_cuda(t: torch.Tensor, what: str) -> None:
    """Raise unless ``t`` is a CUDA tensor on a device this build supports."""
    if t.device.type != "cuda":
        raise RuntimeError(
            f"mps_pointops (B200 build): {what} computes on CUDA tensors only, got a "
            f"{t.device.type} tensor; move the inputs to the GPU")
    dev = t.device.index if t.device.index is not None else torch.cuda.current_device()
    if dev not in _checked_devices:
        check(lib().mpo_device_supported(dev), "device check")
        _checked_devices.add(dev)


def ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


_side_streams: dict[int, torch.cuda.Stream] = {}


def side_stream(device: torch.device) -> torch.cuda.Stream:
    """A second stream per device for the input checks: a check and the copy
    of its flags to the host run there (after waiting for the caller's
    stream), so neither sits in the caller's stream ahead of the compute."""
    key = device.index if device.index is not None else torch.cuda.current_device()
    st = _side_streams.get(key)
    if st is None:
        st = _side_streams[key] = torch.cuda.Stream(torch.device("cuda", key))
    return st


class on_device:
    """Make ``device`` current for the duration of a native call."""

    __slots__ = ("dev", "prev")

    def __init__(self, device: torch.device):
        self.dev = device.index if device.index is not None else torch.cuda.current_device()
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.dev:
            self.prev = cur
            torch.cuda.set_device(self.dev)
        return self

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)
        return False


class KernelTimer:
    """Records CUDA events around the native calls tagged ``tag`` while
    active (used by the benchmark to time one kernel inside a timed region,
    on the stream the kernel runs on)."""

    active: "KernelTimer | None" = None

    def __init__(self, tag: str):
        self.tag = tag
        self.pairs: list[tuple[torch.cuda.Event, torch.cuda.Event]] = []

    def __enter__(self):
        KernelTimer.active = self
        return self

    def __exit__(self, *exc):
        KernelTimer.active = None
        return False

    def mean_ms(self) -> float:
        if not self.pairs:
            return float("nan")
        return sum(a.elapsed_time(b) for a, b in self.pairs) / len(self.pairs)


def timed(tag: str, device: torch.device, fn, *args) -> int:
    """Call ``fn(*args)``; if a KernelTimer for ``tag`` is active, bracket the
    call with CUDA events on the current stream of ``device``."""
    timer = KernelTimer.active
    if timer is None or timer.tag != tag:
        return fn(*args)
    s = torch.cuda.current_stream(device)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(s)
    status = fn(*args)
    b.record(s)
    timer.pairs.append((a, b))
    return status


def workspace(nbytes: int, device: torch.device) -> torch.Tensor | None:
    if nbytes <= 0:
        return None
    return torch.empty(int(nbytes), dtype=torch.uint8, device=device)
