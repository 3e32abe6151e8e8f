"""The C-ABI library loads, exports every declared symbol, and its host-only
logic (plan sizing, binding, argument validation) behaves -- no GPU needed."""
import ctypes
import os
import re

import pytest

from conftest import REPO
from tributary_b200 import _lib, build


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def declared_functions():
    text = open(os.path.join(REPO, "include", "rt_attention.h")).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(rt_\w+)\s*\(", text, re.M)))


def test_header_and_binding_agree():
    assert sorted(_lib.EXPORTED) == declared_functions()


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert lib.rt_version() == 100


def test_status_strings(lib):
    assert lib.rt_status_string(0) == b"ok"
    assert b"wait" in lib.rt_status_string(_lib.RT_ERR_TIMEOUT)
    assert lib.rt_status_string(99) == b"unknown status"


def test_plan_bytes_and_bind(lib):
    b, s, r = 4, 1000, 77
    n = lib.rt_tile_plan_bytes(b, s, r)
    t = (s + 127) // 128
    assert n >= 2 * b * t * t * 2048  # element bits in both orientations
    plan = _lib.RtTilePlan()
    base = 1 << 20  # host-only carve of a fake, 256-aligned address
    assert lib.rt_tile_plan_bind(ctypes.c_void_p(base), n, b, s, r, ctypes.byref(plan)) == 0
    assert plan.tiles == t and plan.words == 1 and plan.batch == b
    fields = ["live_bits", "full_bits", "q2k_ptr", "q2k_idx", "k2q_ptr", "k2q_idx",
              "tile_masks", "tile_masks_t", "fk_bits", "nnz"]
    addrs = [getattr(plan, f) for f in fields]
    assert addrs == sorted(addrs) and all(a % 256 == 0 for a in addrs)
    assert addrs[-1] + 4 <= base + n
    assert lib.rt_tile_plan_bind(ctypes.c_void_p(base), n - 1, b, s, r,
                                 ctypes.byref(plan)) == _lib.RT_ERR_WORKSPACE
    assert lib.rt_tile_plan_bind(ctypes.c_void_p(base + 16), n, b, s, r,
                                 ctypes.byref(plan)) == _lib.RT_ERR_INVALID_ARGUMENT
    assert lib.rt_tile_plan_bind(ctypes.c_void_p(base), n, b, 70000, r,
                                 ctypes.byref(plan)) == _lib.RT_ERR_INVALID_ARGUMENT


def test_argument_validation_before_device_work(lib):
    plan = _lib.RtTilePlan()
    n = lib.rt_tile_plan_bytes(1, 128, 4)
    assert lib.rt_tile_plan_bind(ctypes.c_void_p(1 << 20), n, 1, 128, 4, ctypes.byref(plan)) == 0
    fake = ctypes.c_void_p(1 << 21)
    # bad kind
    assert lib.rt_build_tile_plan(fake, fake, fake, fake, fake, 1, 128, 4, 7,
                                  ctypes.byref(plan), None) == _lib.RT_ERR_INVALID_ARGUMENT
    # plan built for another shape
    assert lib.rt_build_tile_plan(fake, fake, fake, fake, fake, 2, 128, 4, 0,
                                  ctypes.byref(plan), None) == _lib.RT_ERR_INVALID_ARGUMENT
    # unsupported head_dim is reported as such
    assert lib.rt_attention_fwd(fake, fake, fake, 1, 1, 128, 48, 1.0, ctypes.byref(plan),
                                fake, fake, None) == _lib.RT_ERR_UNSUPPORTED
    # a scale that is not positive and finite
    for bad in (0.0, -0.125, float("nan"), float("inf")):
        assert lib.rt_attention_fwd(fake, fake, fake, 1, 1, 128, 64, bad, ctypes.byref(plan),
                                    fake, fake, None) == _lib.RT_ERR_INVALID_ARGUMENT
        assert lib.rt_attention_bwd(fake, fake, fake, fake, fake, fake, 1, 1, 128, 64, bad,
                                    ctypes.byref(plan), fake, fake, fake, fake, 1 << 20,
                                    None) == _lib.RT_ERR_INVALID_ARGUMENT
        assert lib.rt_attention_bwd_noalloc(fake, fake, fake, fake, fake, fake, 1, 1, 128, 64, bad,
                                            ctypes.byref(plan), fake, fake, fake,
                                            None) == _lib.RT_ERR_INVALID_ARGUMENT
    # misaligned tensor
    odd = ctypes.c_void_p((1 << 21) + 2)
    assert lib.rt_attention_fwd(odd, fake, fake, 1, 1, 128, 64, 1.0, ctypes.byref(plan),
                                fake, fake, None) == _lib.RT_ERR_INVALID_ARGUMENT
    # empty problems are a no-op
    empty = _lib.RtTilePlan()
    assert lib.rt_tile_plan_bind(None, 0, 0, 0, 0, ctypes.byref(empty)) == 0
    assert lib.rt_build_tile_plan(None, None, None, None, None, 0, 0, 0, 0,
                                  ctypes.byref(empty), None) == 0
    assert lib.rt_attention_fwd(None, None, None, 0, 4, 0, 64, 1.0, ctypes.byref(empty),
                                None, None, None) == 0
    # workspace too small for the backward
    ws = lib.rt_attention_bwd_workspace_bytes(1, 1, 128)
    assert ws >= 512
    assert lib.rt_attention_bwd(fake, fake, fake, fake, fake, fake, 1, 1, 128, 64, 1.0,
                                ctypes.byref(plan), fake, fake, fake, fake, ws - 256,
                                None) == _lib.RT_ERR_WORKSPACE
    # the sublayer backward (token-order outputs): same checks, plus its own pointers
    def bwd_qkv(scale=1.0, head_dim=64, perm=fake, dtau=fake, ws_bytes=ws):
        return lib.rt_attention_bwd_qkv(fake, fake, fake, fake, fake, fake, 1, 1, 128, head_dim, scale,
                                        ctypes.byref(plan), perm, fake, fake, fake, fake, dtau, fake,
                                        ws_bytes, None)
    assert bwd_qkv(head_dim=48) == _lib.RT_ERR_UNSUPPORTED
    assert bwd_qkv(scale=0.0) == _lib.RT_ERR_INVALID_ARGUMENT
    assert bwd_qkv(perm=None) == _lib.RT_ERR_INVALID_ARGUMENT
    assert bwd_qkv(dtau=odd) == _lib.RT_ERR_INVALID_ARGUMENT
    assert bwd_qkv(ws_bytes=ws - 256) == _lib.RT_ERR_WORKSPACE
    assert lib.rt_attention_bwd_qkv(None, None, None, None, None, None, 0, 1, 128, 64, 1.0, ctypes.byref(empty),
                                    None, None, None, None, None, None, None, 0, None) == 0


def test_xla_ffi_handlers_need_jax():
    """The XLA FFI adapter builds only against jax's FFI headers; without jax
    the build says so and returns None instead of failing."""
    import importlib.util
    from tributary_b200.ffi import build_ffi
    assert os.path.exists(os.path.join(REPO, "tributary_b200", "ffi", "rt_xla_ffi.cc"))
    if importlib.util.find_spec("jax") is None:
        assert build_ffi.build() is None
