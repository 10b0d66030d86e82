"""ctypes binding of libtao_b200.so (C ABI declared in include/tao_b200.h).

The library is built in-tree by ``tao_memory_b200.build``.  There is no CPU or
eager fallback: if the shared object is missing, every entry point raises.
"""

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libtao_b200.so")

TAO_OK, TAO_ERR_ARG, TAO_ERR_POSITION, TAO_ERR_SEAL = 0, 1, 2, 3
TAO_ERR_CAPACITY, TAO_ERR_CUDA, TAO_ERR_DEVICE, TAO_ERR_TIMEOUT = 4, 5, 6, 7


class TaoPolicy(ctypes.Structure):
    _fields_ = [("fine_tokens", ctypes.c_int32), ("local_keep", ctypes.c_int32),
                ("coarse_group", ctypes.c_int32), ("route_period", ctypes.c_int32),
                ("layer_stagger", ctypes.c_int32), ("budget_root_scale", ctypes.c_int32),
                ("budget_offset", ctypes.c_int32), ("route_cap", ctypes.c_int32),
                ("fine_read", ctypes.c_int32), ("coarse", ctypes.c_int32)]


class TaoState(ctypes.Structure):
    _fields_ = [("k_ring", ctypes.c_void_p), ("v_ring", ctypes.c_void_p),
                ("rk_ring", ctypes.c_void_p), ("fine_c", ctypes.c_void_p),
                ("fine_z", ctypes.c_void_p), ("page_z", ctypes.c_void_p),
                ("page_w", ctypes.c_void_p), ("route_ids", ctypes.c_void_p),
                ("route_pages", ctypes.c_void_p), ("counters", ctypes.c_void_p),
                ("position", ctypes.c_int64),
                ("n_route", ctypes.c_int32), ("n_chosen", ctypes.c_int32),
                ("cap_fines", ctypes.c_int32), ("route_cap", ctypes.c_int32),
                ("layer_index", ctypes.c_int32), ("heads", ctypes.c_int32),
                ("width", ctypes.c_int32), ("arrive", ctypes.c_int32),
                ("route_refreshes", ctypes.c_int32), ("seal_events", ctypes.c_int32),
                ("page_c", ctypes.c_void_p), ("coarse_w", ctypes.c_void_p)]


class TaoError(RuntimeError):
    """A CUDA or device-side failure reported by the library."""


_VP, _I, _I64, _SZ, _F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t, ctypes.c_float

_SIGNATURES = {
    "tao_last_error": (ctypes.c_char_p, []),
    "tao_version": (_I, []),
    "tao_state_sizeof": (_SZ, []),
    "tao_stream_workspace_bytes": (_SZ, [_I, _I, _I, _I, _I, ctypes.POINTER(TaoPolicy)]),
    "tao_stream_step": (_I, [_VP, _I, ctypes.POINTER(_I64), ctypes.POINTER(ctypes.c_int32),
                             ctypes.POINTER(TaoPolicy), _I, _I, _I, _VP, _VP, _VP, _VP, _VP,
                             _VP, _VP, _F, _VP, _VP, _SZ, _VP]),
    "tao_stream_check": (_I, [_VP, ctypes.POINTER(_I), _VP]),
    "tao_decode_variant": (_I, [_I]),
    "tao_attention_variant": (_I, [_I]),
    "tao_decode_graph_mode": (_I, [_I]),
    "tao_writer_stats": (_I, [_VP, _VP, _I64, _I64, _I64, _I, _I, _I, _VP, _VP, _VP, _VP]),
    "tao_decode_step": (_I, [_VP, _I, ctypes.POINTER(_I64), ctypes.POINTER(ctypes.c_int32),
                             ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(TaoPolicy), _I, _I,
                             _VP, _VP, _VP, _VP, _VP, _VP, _VP, _F, _VP, _VP, _SZ, _VP]),
    "tao_stream_decode_noalloc": (_I, [_VP, _I, ctypes.POINTER(_I64), ctypes.POINTER(ctypes.c_int32),
                                       ctypes.POINTER(TaoPolicy), _I, _I, _VP, _VP, _VP, _VP, _VP,
                                       _VP, _VP, _F, _VP, _VP]),
    "tao_stream_decode_noalloc_check": (_I, [ctypes.POINTER(_I), _VP]),
    "tao_ring_gather": (_I, [_VP, _I, _I, _I64, _I, _VP, _VP]),
    "tao_ring_scatter": (_I, [_VP, _I, _I, _I64, _I, _VP, _VP]),
    "tao_state_rebuild_memo": (_I, [_VP, _I, _I, _I, _VP]),
    "tao_state_refresh_page_weights": (_I, [_VP, _I, _I, _I, _VP]),
    "tao_decode_step_host": (_I, [_VP, _I, ctypes.POINTER(_I64), ctypes.POINTER(ctypes.c_int32),
                                  ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(TaoPolicy), _I, _I,
                                  _VP, _VP, _VP, _VP, _VP, _VP, _F, _VP, _SZ, _VP]),
    "tao_host_device_pointer": (_I, [_VP, ctypes.POINTER(_VP)]),
    "tao_host_wait": (_I, [_VP, _I, ctypes.c_longlong]),
    "tao_graph_launch": (_I, [_VP, _VP]),
    "tao_copy_host_to_device": (_I, [_VP, _VP, _SZ, _VP]),
    "tao_copy_device_to_host": (_I, [_VP, _VP, _SZ, _VP]),
    "tao_copy_host_to_device_many": (_I, [ctypes.POINTER(_VP), ctypes.POINTER(_VP), ctypes.POINTER(_SZ), _I,
                                          _VP]),
    "tao_window_attention": (_I, [_VP, _VP, _VP, _VP, _VP, _I, _I, _I, _I, _VP]),
    "tao_train_geometry": (_I, [_I, ctypes.POINTER(_I), ctypes.POINTER(_I), ctypes.POINTER(_I)]),
    "tao_train_forward": (_I, [_VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _I, _I, _I, _I, _VP, _VP, _VP]),
    "tao_train_backward": (_I, [_VP] * 9 + [_I, _I, _I, _I, _VP, _VP, _VP, _VP]),
    "tao_qkv_split_norm": (_I, [_VP, _I64, _I, _I, _F, _VP, _VP, _VP, _VP, _VP, _VP]),
    "tao_qkv_split_norm_backward": (_I, [_VP] * 7 + [_I64, _I, _I, _F, _VP, _VP]),
    "tao_feature_read_forward": (_I, [_VP, _VP, _VP, _VP, _I, _I, _I, _I, _I, _VP, _VP, _VP]),
    "tao_feature_read_backward": (_I, [_VP, _VP, _VP, _VP, _VP, _I, _I, _I, _I, _I, _VP, _VP, _VP, _VP, _VP]),
    "tao_train_pairs": (_I, [_I]),
    "tao_event_create": (_I, [ctypes.POINTER(_VP)]),
    "tao_event_destroy": (_I, [_VP]),
    "tao_event_record": (_I, [_VP, _VP]),
    "tao_event_elapsed": (_I, [_VP, _VP, ctypes.POINTER(_F)]),
    "tao_stream_profile_next": (_I, [_VP, _VP]),
}

_lib = None


def lib():
    """Load the shared object once; raise if it is missing (no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError("libtao_b200.so is not built: run `python -m tao_memory_b200.build`; "
                               "this package has no CPU or eager fallback")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        if handle.tao_state_sizeof() != ctypes.sizeof(TaoState):
            raise RuntimeError("TaoState layout mismatch between Python and libtao_b200.so")
        _lib = handle
    return _lib


def check(rc):
    """Map a status code to the reference's exception types."""
    if rc == TAO_OK:
        return
    msg = lib().tao_last_error().decode()
    if rc in (TAO_ERR_ARG, TAO_ERR_POSITION, TAO_ERR_SEAL, TAO_ERR_CAPACITY):
        raise ValueError(msg)
    raise TaoError(msg)


def exported_symbols():
    return tuple(_SIGNATURES)
