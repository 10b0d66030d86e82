"""CPU-side checks of the C ABI: the library loads, exports every symbol the
header declares, and its host-side validation and schedule agree with the
reference's integer policy (no kernel is launched)."""
import ctypes
import os
import re

import pytest

from tao_memory_b200 import _lib
from tao_memory_b200.config import TaoConfig, index_only_page_memo, routed_counts
from tao_memory_b200.stream import sealed_at, window_start, is_refresh
from oracle import tao_oracle as o

HEADER = os.path.join(os.path.dirname(os.path.dirname(__file__)), "include", "tao_b200.h")


def declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|const char\*)\s+(tao_\w+)\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    names = declared()
    assert len(names) >= 9
    for name in names:
        assert hasattr(lib, name), name
    assert set(_lib.exported_symbols()) <= set(names)


def test_state_layout_matches_header():
    assert _lib.lib().tao_state_sizeof() == ctypes.sizeof(_lib.TaoState)


def test_host_validation_errors_without_gpu():
    lib = _lib.lib()
    pol = _lib.TaoPolicy(256, 512, 8, 24, 2, 2, 2, 256)
    pos = (ctypes.c_int64 * 1)(0)
    cap = (ctypes.c_int32 * 1)(64)
    # width 96 is rejected before any launch
    rc = lib.tao_stream_step(1, 1, pos, cap, ctypes.byref(pol), 1, 2, 96, *([16] * 7), 0.5, 16, 256, 1 << 20, None)
    assert rc == _lib.TAO_ERR_ARG
    with pytest.raises(ValueError):
        _lib.check(rc)
    # a chunk that crosses the 768 seal boundary
    pos[0] = 700
    rc = lib.tao_stream_step(1, 1, pos, cap, ctypes.byref(pol), 100, 2, 64, *([16] * 7), 0.5, 16, 256, 1 << 20, None)
    assert rc == _lib.TAO_ERR_SEAL
    # geometry other than the preset
    bad = _lib.TaoPolicy(128, 512, 8, 24, 2, 2, 2, 256)
    pos[0] = 0
    rc = lib.tao_stream_step(1, 1, pos, cap, ctypes.byref(bad), 1, 2, 64, *([16] * 7), 0.5, 16, 256, 1 << 20, None)
    assert rc == _lib.TAO_ERR_ARG
    assert lib.tao_stream_workspace_bytes(8, 1, 12, 64, 256, ctypes.byref(pol)) > 0
    assert lib.tao_stream_workspace_bytes(8, 1, 12, 96, 256, ctypes.byref(pol)) == 0
    # the feature-mass read (fine_read = 1): the no-alloc decode refuses it, the
    # other decode kernel variants refuse it, and unknown read modes are refused
    feat = _lib.TaoPolicy(256, 512, 8, 24, 2, 2, 2, 256, 1)
    layer = (ctypes.c_int32 * 1)(0)
    rc = lib.tao_stream_decode_noalloc(16, 1, pos, cap, ctypes.byref(feat), 2, 64, *([16] * 7), 0.5, 16, None)
    assert rc == _lib.TAO_ERR_ARG
    lib.tao_decode_variant(2)
    try:
        rc = lib.tao_decode_step(16, 1, pos, layer, cap, ctypes.byref(feat), 2, 64, *([16] * 7), 0.5, 16, 256,
                                 1 << 20, None)
    finally:
        lib.tao_decode_variant(1)
    assert rc == _lib.TAO_ERR_ARG and b"variant 1" in lib.tao_last_error()
    odd = _lib.TaoPolicy(256, 512, 8, 24, 2, 2, 2, 256, 2)
    rc = lib.tao_stream_step(1, 1, pos, cap, ctypes.byref(odd), 1, 2, 64, *([16] * 7), 0.5, 16, 256, 1 << 20, None)
    assert rc == _lib.TAO_ERR_ARG
    # w == 1 under the feature read: a window-attention output and one fine partial per query
    assert lib.tao_stream_workspace_bytes(8, 1, 12, 64, 256, ctypes.byref(feat)) > 0


def test_host_transfer_argument_checks_without_gpu():
    """Misaligned or ragged host transfers are refused before any CUDA call."""
    lib = _lib.lib()
    assert lib.tao_copy_host_to_device(16, 24, 64, None) == _lib.TAO_ERR_ARG
    assert lib.tao_copy_device_to_host(16, 32, 40, None) == _lib.TAO_ERR_ARG
    assert lib.tao_copy_host_to_device(None, 32, 64, None) == _lib.TAO_ERR_ARG
    assert b"16-byte" in lib.tao_last_error() or b"null" in lib.tao_last_error()
    # the host-staged decode step refuses missing buffers before any CUDA call
    pos = (ctypes.c_int64 * 1)(1000)
    one = (ctypes.c_int32 * 1)(64)
    pol = _lib.TaoPolicy()
    assert lib.tao_decode_step_host(None, 1, pos, one, one, ctypes.byref(pol), 2, 64, None, None, None,
                                    None, None, None, 0.5, None, 0, None) == _lib.TAO_ERR_ARG
    assert b"null" in lib.tao_last_error()
    dev = ctypes.c_void_p()
    assert lib.tao_host_device_pointer(None, ctypes.byref(dev)) == _lib.TAO_ERR_ARG


def test_host_wait_on_a_completion_word():
    """tao_host_wait returns once the word has reached the value (wrap-around order)
    and reports a timeout otherwise."""
    lib = _lib.lib()
    word = ctypes.c_int32(7)
    assert lib.tao_host_wait(ctypes.addressof(word), 7, 0) == _lib.TAO_OK
    assert lib.tao_host_wait(ctypes.addressof(word), 5, 0) == _lib.TAO_OK
    assert lib.tao_host_wait(ctypes.addressof(word), 8, 2000) == _lib.TAO_ERR_TIMEOUT
    word.value = -2147483648          # one past INT_MAX: later than it in wrap-around order
    assert lib.tao_host_wait(ctypes.addressof(word), 2147483647, 0) == _lib.TAO_OK
    assert lib.tao_host_wait(None, 1, 0) == _lib.TAO_ERR_ARG
    assert lib.tao_graph_launch(None, None) == _lib.TAO_ERR_ARG


def test_schedule_matches_reference_policy():
    cfg = index_only_page_memo()
    for completed in range(0, 80):
        for pending in range(0, 8):
            assert routed_counts(completed, pending, cfg) == o.routed_counts(completed, pending)
    for c in range(0, 5000):
        assert cfg.budget(c) == o.budget(c)
    # cursor helpers follow the reference's seal/refresh schedule (tao_stream.py:196-227, 959-967)
    assert [sealed_at(p) for p in (0, 767, 768, 1023, 1024, 1280)] == [0, 0, 1, 1, 2, 3]
    assert [p for p in range(700, 900) if is_refresh(p, 3, cfg)] == [768, 774, 798, 822, 846, 870, 894]
    assert window_start(767) == 0 and window_start(768) == 256 and window_start(1023) == 256


def test_config_validation_matches_reference():
    with pytest.raises(ValueError):
        TaoConfig(fine_writer="nope")
    with pytest.raises(TypeError):
        TaoConfig(fine_tokens=256.0)
    with pytest.raises(ValueError):
        TaoConfig(local_keep=300)
    assert TaoConfig(**index_only_page_memo().export()) == index_only_page_memo()


@pytest.mark.parametrize("writer", ["feature_mass_association", "structured_gram_association"])
def test_feature_read_writers_policy(writer):
    """The feature-mass and structured-Gram writers run in streaming and in training
    on the index-only preset with the feature-mass read; with the coarse value branch
    they are refused loudly rather than computed with another read."""
    from tao_memory_b200.stream import check_config, policy_for
    cfg = TaoConfig(**{**index_only_page_memo().export(), "fine_writer": writer})
    check_config(cfg)
    check_config(cfg, training=True)
    assert policy_for(cfg).fine_read == 1 and policy_for(index_only_page_memo()).fine_read == 0
    with pytest.raises(NotImplementedError):
        check_config(TaoConfig(fine_writer=writer), training=True)


def test_batch_argument_cache_keys_on_layer_and_policy():
    """A descriptor address reused by a new state with another layer index must
    not return cached per-state arrays of the old state."""
    import torch
    from tao_memory_b200.stream import _BatchArgs
    from tao_memory_b200.config import TaoConfig

    class _Desc:
        def __init__(self, p):
            self.p = p

        def data_ptr(self):
            return self.p

    class _State:
        def __init__(self, layer, cfg=TaoConfig()):
            self._desc, self.cap_fines, self.layer_index, self.config = _Desc(4096), 64, layer, cfg

    dev = torch.device("cpu")
    a = _BatchArgs.get([_State(0)], 1, 2, 64, dev)
    b = _BatchArgs.get([_State(3)], 1, 2, 64, dev)
    assert a is not b and list(a.layers) == [0] and list(b.layers) == [3]
    c = _BatchArgs.get([_State(3, TaoConfig(route_period=12))], 1, 2, 64, dev)
    assert c is not b and c.policy.route_period == 12
