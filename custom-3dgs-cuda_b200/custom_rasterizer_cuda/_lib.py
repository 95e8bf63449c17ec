"""ctypes binding of libgs3d_b200.so, the C ABI declared in include/gs3d_b200.h.

The library is loaded from this package directory. Loading never falls back to anything:
if the shared library is missing or lacks a symbol, importing the package raises.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import c_double, c_float, c_int, c_longlong, c_size_t, c_uint, c_void_p, POINTER
from pathlib import Path

# The library built in-tree by build.py; GS3D_B200_LIB may point at another build of it.
LIB_PATH = Path(os.environ.get("GS3D_B200_LIB",
                               Path(__file__).resolve().parent / "libgs3d_b200.so"))

GS_OK = 0
GS_ERR_INVALID_ARG = 1
GS_ERR_CUDA = 2
GS_ERR_CAPACITY = 3
GS_ERR_DEVICE = 4

P = c_void_p  # every pointer crosses the boundary as an integer address

# name -> (restype, argtypes), one entry per declaration in include/gs3d_b200.h
SIGNATURES = {
    "gs_last_error": (ctypes.c_char_p, []),
    "gs_version": (ctypes.c_char_p, []),
    "gs_project": (c_int, [c_int, P, P, P, P, P, c_float, c_float, c_float, c_float, P, P, P,
                           P]),
    "gs_sh_forward": (c_int, [c_int, P, P, P, P, P, P]),
    "gs_rasterize_workspace_size": (c_size_t, [c_int, c_int, c_int, c_longlong]),
    "gs_rasterize": (c_int, [c_int, c_int, c_int, P, P, P, P, P, P, c_size_t, c_longlong, P,
                             P, P, P, P, P, P, P, P]),
    "gs_rasterize_noalloc": (c_int, [c_int, c_int, c_int, P, P, P, P, P, c_longlong, P, P, P,
                                     P, P, P, P]),
    "gs_rasterize_backward_workspace_size": (c_size_t, [c_int]),
    "gs_rasterize_backward": (c_int, [c_int, c_int, c_int, P, P, P, P, P, P, P, P, P, P,
                                      c_size_t, P, P, P, P, P]),
    "gs_sh_backward": (c_int, [c_int, P, P, P, P, P, P, P, P, P]),
    "gs_project_backward": (c_int, [c_int, P, P, P, P, P, P, P, c_float, c_float, c_float,
                                    c_float, P, P, P, P]),
    "gs_render_workspace_size": (c_size_t, [c_int, c_int, c_int, c_longlong]),
    "gs_render_forward": (c_int, [c_int, c_int, c_int, P, P, P, P, P, P, P, P, P, c_float,
                                  c_float, c_float, c_float, P, c_size_t, c_longlong, P, P, P,
                                  P, P, P, P, P, c_uint, P]),
    "gs_render_backward_workspace_size": (c_size_t, [c_int]),
    "gs_render_backward": (c_int, [c_int, c_int, c_int, P, P, P, P, P, P, P, P, P, c_float,
                                   c_float, c_float, c_float, P, c_longlong, P, P, P, P, P,
                                   c_size_t, P, P, P, P, P, P, P, c_int, P, P, P, c_float,
                                   c_float, P, P, c_uint, P]),
    "gs_render_backward_blend": (c_int, [c_int, c_int, c_int, P, P, c_longlong, P, P, P, P, P,
                                         c_size_t, c_uint, P]),
    "gs_render_backward_gaussians": (c_int, [c_int, c_int, P, P, P, P, P, P, P, P, P, P, P, P,
                                             c_int, P, P, P, P]),
    "gs_l1_ssim_workspace_size": (c_size_t, [c_int, c_int]),
    "gs_l1_ssim_forward": (c_int, [c_int, c_int, P, P, c_float, P, c_size_t, P, P, P]),
    "gs_l1_ssim_backward": (c_int, [c_int, c_int, P, P, c_float, P, c_size_t, P, P, P]),
    "gs_adam_step": (c_int, [c_int, P, P, P, P, P, P, c_double, c_double, c_double, c_longlong,
                             P, P, P]),
    "gs_sharded_adam_step": (c_int, [P, P, P, c_int, P, P, c_double, c_double, c_double,
                                     c_longlong, c_float, P, P, P]),
    "gs_adc_workspace_size": (c_size_t, [c_int]),
    "gs_adc_plan": (c_int, [c_int, P, P, P, P, P, c_float, c_float, c_float, c_float, c_float,
                            c_int, c_int, P, c_size_t, P, P, P]),
    "gs_adc_apply": (c_int, [c_int, P, c_size_t, P, P, P, P, P, c_int, P, P, P, P]),
    "gs_densify_stats": (c_int, [c_int, P, c_int, c_float, c_float, P, P, P, P]),
    "gs_event_create": (c_int, [POINTER(c_void_p)]),
    "gs_event_synchronize": (c_int, [P]),
    "gs_event_destroy": (c_int, [P]),
    "gs_set_stage_events": (c_int, [P, c_int]),
    "gs_event_create_timed": (c_int, [POINTER(c_void_p)]),
    "gs_event_elapsed_ms": (c_int, [P, P, POINTER(c_float)]),
    "gs_kernel_launches": (ctypes.c_ulonglong, []),
    "gs_device_error_bits": (c_int, [POINTER(c_uint)]),
    "gs_clear_device_errors": (c_int, []),
}


GS_MAX_VIEWS_PER_CALL = 16


class ViewSums(ctypes.Structure):
    """Mirror of gs_view_sums (include/gs3d_b200.h): one view's blend-backward workspace and
    camera for gs_render_backward_gaussians."""

    _fields_ = [("workspace", c_void_p), ("workspace_bytes", c_size_t), ("R", c_void_p),
                ("t", c_void_p), ("cam_pos", c_void_p),
                ("fx", c_float), ("fy", c_float), ("cx", c_float), ("cy", c_float),
                ("stat_scale_x", c_float), ("stat_scale_y", c_float)]


def load(path: Path = LIB_PATH) -> ctypes.CDLL:
    if not path.exists():
        raise ImportError(
            f"{path.name} is not built; run `python custom-3dgs-cuda_b200/build.py` "
            "(or __graft_entry__.build()) first"
        )
    lib = ctypes.CDLL(str(path))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)  # AttributeError if the symbol is missing
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


lib = load()


def check(status: int) -> None:
    """Raises RuntimeError with the library's message when a call did not return GS_OK."""
    if status != GS_OK:
        msg = lib.gs_last_error().decode(errors="replace")
        raise RuntimeError(f"gs3d_b200 error {status}: {msg}")


def device_error_bits() -> int:
    bits = c_uint(0)
    check(lib.gs_device_error_bits(ctypes.byref(bits)))
    return int(bits.value)


def kernel_launches() -> int:
    """Kernels launched by libgs3d_b200 in this process so far."""
    return int(lib.gs_kernel_launches())


def clear_device_errors() -> None:
    check(lib.gs_clear_device_errors())


class Event:
    """A CUDA event owned by the library (timing disabled unless `timed`)."""

    def __init__(self, timed: bool = False) -> None:
        h = c_void_p(0)
        if timed:
            check(lib.gs_event_create_timed(ctypes.byref(h)))
        else:
            check(lib.gs_event_create(ctypes.byref(h)))
        self.handle = h.value

    def elapsed_ms(self, end: "Event") -> float:
        ms = c_float(0.0)
        check(lib.gs_event_elapsed_ms(self.handle, end.handle, ctypes.byref(ms)))
        return float(ms.value)

    def synchronize(self) -> None:
        check(lib.gs_event_synchronize(self.handle))

    def __del__(self) -> None:
        try:
            if self.handle:
                lib.gs_event_destroy(self.handle)
        except Exception:
            pass


def set_stage_events(events: list["Event | None"] | None) -> None:
    """Installs (or, with None, removes) the process-wide stage events of the render path."""
    if not events:
        check(lib.gs_set_stage_events(None, 0))
        return
    arr = (c_void_p * len(events))(*[e.handle if e is not None else None for e in events])
    check(lib.gs_set_stage_events(arr, len(events)))
