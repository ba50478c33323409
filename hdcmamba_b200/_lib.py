"""ctypes binding of ``libhdcmamba_b200.so`` (the C ABI declared in include/hdcmamba_b200.h).

There is no fallback: if the library is missing or was built for another
architecture, importing the ops raises.  Build it with
``python -m hdcmamba_b200.build``.
"""
import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libhdcmamba_b200.so")

HDC_F32, HDC_BF16 = 0, 1
HDC_ACT_NONE, HDC_ACT_SILU = 0, 1

c_i64 = ctypes.c_int64
c_vp = ctypes.c_void_p
c_int = ctypes.c_int
c_float = ctypes.c_float
c_size = ctypes.c_size_t

# name -> (restype, argtypes); the single source of truth for the Python side.
SIGNATURES = {
    "hdc_version": (c_int, []),
    "hdc_built_arch": (c_int, []),
    "hdc_error_string": (ctypes.c_char_p, []),
    "hdc_launch_count": (ctypes.c_longlong, []),
    "hdc_ln_conv_fwd": (c_int, [c_int, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                                c_i64, c_i64, c_i64, c_float, c_int, c_vp]),
    "hdc_ln_conv_fwd_halo_flag": (c_int, [c_int, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                                          c_i64, c_i64, c_i64, c_float, c_int, c_vp, c_vp, c_vp]),
    "hdc_ln_conv_bwd_workspace_bytes": (c_size, [c_i64, c_i64, c_i64]),
    "hdc_ln_conv_bwd": (c_int, [c_int, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_size,
                                c_i64, c_i64, c_i64, c_vp]),
    "hdc_ssm_chunk_stats": (c_int, [c_int, c_vp, c_i64, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp]),
    "hdc_ssm_scan_fwd": (c_int, [c_int, c_vp, c_i64, c_i64, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64,
                                 c_i64, c_vp]),
    "hdc_ssm_scan_out": (c_int, [c_int, c_vp, c_i64, c_i64, c_vp, c_vp, c_i64, c_i64, c_vp, c_i64, c_i64,
                                 c_i64, c_i64, c_i64, c_i64, c_vp]),
    "hdc_ssm_scan_out_blocked": (c_int, [c_int, c_vp, c_i64, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp,
                                         c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, ctypes.c_uint32, c_vp,
                                         c_vp]),
    "hdc_ssm_scan_fwd_noalloc": (c_int, [c_int, c_vp, c_i64, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64,
                                         c_i64, c_vp]),
    "hdc_ssm_noalloc_capacity": (c_i64, []),
    "hdc_slot_workspace_bytes": (c_size, [c_i64, c_i64, c_i64, c_i64, c_i64]),
    "hdc_slot_scan_fwd": (c_int, [c_int, c_vp, c_vp, c_vp, c_i64, c_i64, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64,
                                  c_vp, c_vp, c_vp, c_size, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp]),
    "hdc_slot_gate_fwd": (c_int, [c_int, c_vp, c_vp, c_vp, c_i64, c_i64, c_vp, c_vp, c_vp, c_i64, c_i64, c_vp, c_vp,
                                  c_vp, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_size, c_i64, c_i64, c_i64, c_i64,
                                  c_i64, c_vp]),
    "hdc_slot_state_fwd": (c_int, [c_int, c_vp, c_vp, c_i64, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp, c_size, c_i64,
                                   c_i64, c_i64, c_i64, c_i64, c_vp]),
    "hdc_slot_gate_carry_fwd": (c_int, [c_int, c_vp, c_vp, c_vp, c_i64, c_i64, c_vp, c_vp, c_vp, c_i64, c_i64, c_vp,
                                        c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_vp, c_i64, c_i64, c_vp, c_vp, c_size,
                                        c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, ctypes.c_uint32, c_vp, c_vp]),
    "hdc_slot_scan_fwd_path": (c_int, [c_int, c_vp, c_vp, c_vp, c_i64, c_i64, c_vp, c_vp, c_vp, c_i64, c_i64,
                                       c_i64, c_vp, c_vp, c_vp, c_size, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64,
                                       c_int, ctypes.POINTER(c_int), c_vp]),
    "hdc_device_error": (c_int, [c_int]),
    "hdc_gate_cat_fwd": (c_int, [c_int, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_i64,
                                 c_i64, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp]),
    "hdc_row_layernorm": (c_int, [c_int, c_vp, c_vp, c_i64, c_i64, c_float, c_vp]),
    "hdc_row_layernorm_affine": (c_int, [c_int, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_float, c_vp]),
    "hdc_ln_conv_step": (c_int, [c_int, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_float, c_vp]),
    "hdc_ssm_step": (c_int, [c_int, c_vp, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp]),
    "hdc_ssm_carry_fwd": (c_int, [c_int, c_vp, c_i64, c_i64, c_i64, c_vp, c_vp]),
    "hdc_slot_step": (c_int, [c_int, c_vp, c_vp, c_vp, c_vp, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                              c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp]),
    "hdc_peer_alloc": (c_int, [c_size, ctypes.POINTER(c_vp)]),
    "hdc_peer_free": (c_int, [c_vp]),
    "hdc_ipc_handle_bytes": (c_int, []),
    "hdc_ipc_handle": (c_int, [c_vp, c_vp]),
    "hdc_ipc_open": (c_int, [c_vp, ctypes.POINTER(c_vp)]),
    "hdc_ipc_close": (c_int, [c_vp]),
    "hdc_peer_put": (c_int, [c_vp, c_size, c_vp, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint32, c_int, c_vp,
                             c_vp, c_vp]),
    "hdc_peer_wait": (c_int, [c_vp, ctypes.c_uint32, c_vp, c_vp]),
    "hdc_peer_wait_for": (c_int, [c_vp, ctypes.c_uint32, c_vp, ctypes.c_uint64, c_vp]),
    "hdc_peer_gen_bump": (c_int, [c_vp, c_vp]),
    "hdc_peer_barrier": (c_int, [c_vp, ctypes.c_uint64, c_int, c_int, c_vp, c_vp, c_vp]),
    "hdc_trace_stamp": (c_int, [c_vp, ctypes.c_longlong, c_vp]),
}

_lib = None
_lock = threading.Lock()


class HdcError(RuntimeError):
    """A rejected argument or a CUDA launch error reported by libhdcmamba_b200."""


def load():
    """Load the shared library once (raises OSError if it is absent)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise OSError(f"{LIB_PATH} is missing: build it with `python -m hdcmamba_b200.build`")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def call(name, *args):
    """Call an entry point; raise HdcError on a non-zero status."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != 0:
        msg = lib.hdc_error_string().decode(errors="replace")
        raise HdcError(f"{name} failed ({rc}): {msg}")
    return rc


def launch_count():
    """Kernel launches issued by the library so far (counted in the library)."""
    return int(load().hdc_launch_count())
