"""CPU checks of the C-ABI library: it builds, loads, exports every symbol
include/hba_b200.h declares, and rejects bad arguments with the documented
status codes before touching a device (no compute calls here)."""

import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "hba_b200.h")


@pytest.fixture(scope="module")
def lib():
    from hba_b200 import _build, _lib
    if not os.path.exists(_lib.LIB_PATH):
        _build.build()
    return _lib.load()


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(hba_b200_\w+)\s*\(", src)))


def test_header_declares_the_expected_entry_points():
    names = declared_functions()
    for n in ("hba_b200_decode", "hba_b200_prefill", "hba_b200_summarize", "hba_b200_build_supers",
              "hba_b200_qknorm", "hba_b200_append_kv", "hba_b200_decode_workspace_size",
              "hba_b200_prefill_workspace_size"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    from hba_b200 import _lib
    for name in declared_functions():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\b(hba_b200_\w+)\b", out))
    assert exported == set(declared_functions())


def test_config_struct_matches_header(lib):
    from hba_b200 import _lib
    assert ctypes.sizeof(_lib.Config) == 13 * 4


def cfg(**kw):
    from hba_b200 import _lib
    base = dict(n_heads=14, n_kv=2, head_dim=64, block=64, window=1024, sinks=4, k_blocks=16, slots=4, fanout=16,
                beam=4, hier=0, qknorm=1, eps=1e-6)
    base.update(kw)
    return _lib.Config(**base)


def test_status_strings_and_version(lib):
    assert lib.hba_b200_version() >= 100
    assert lib.hba_b200_status_string(0) == b"ok"
    assert b"block" in lib.hba_b200_status_string(2)


def test_workspace_queries_validate_config(lib):
    c = cfg()
    assert lib.hba_b200_prefill_workspace_size(ctypes.byref(c), 1, 4096) > 0
    assert lib.hba_b200_prefill_workspace_size(ctypes.byref(c), 1, 4000) == 0          # n % block
    assert lib.hba_b200_decode_workspace_size(ctypes.byref(c), 64, 32768) > 0
    for bad in (cfg(head_dim=96), cfg(n_heads=15), cfg(k_blocks=64), cfg(slots=9), cfg(block=128),
                cfg(sinks=65), cfg(n_heads=34, n_kv=2), cfg(hier=1, beam=0), cfg(hier=1, beam=33)):
        assert lib.hba_b200_prefill_workspace_size(ctypes.byref(bad), 1, 4096) == 0
    # workspace grows with the batch and the context
    a = lib.hba_b200_decode_workspace_size(ctypes.byref(c), 8, 32768)
    b = lib.hba_b200_decode_workspace_size(ctypes.byref(c), 16, 32768)
    assert b > a


def test_entry_points_reject_bad_arguments_without_a_device(lib):
    from hba_b200 import _lib
    c = cfg()
    P = ctypes.c_void_p
    one = P(16)   # never dereferenced: validation fails first
    z = P(0)
    st = lib.hba_b200_prefill(ctypes.byref(c), 1, 100, ctypes.c_float(0.1), one, one, one, one, one, one, one, one,
                              one, one, z, z, z, one, 1 << 30, z)
    assert st == _lib.ERR_NOT_BLOCK_MULTIPLE
    st = lib.hba_b200_prefill(ctypes.byref(c), 1, 128, ctypes.c_float(0.1), z, one, one, one, one, one, one, one,
                              one, one, z, z, z, one, 1 << 30, z)
    assert st == _lib.ERR_INVALID_ARGUMENT
    st = lib.hba_b200_prefill(ctypes.byref(c), 1, 128, ctypes.c_float(0.1), one, one, one, one, one, one, one, one,
                              one, one, z, z, z, one, 16, z)
    assert st == _lib.ERR_WORKSPACE
    bad = cfg(head_dim=80)
    st = lib.hba_b200_decode(ctypes.byref(bad), 1, 128, one, one, one, one, one, one, one, one, one, z, one, one,
                             one, z, z, z, one, 1 << 20, z)
    assert st == _lib.ERR_UNSUPPORTED
    st = lib.hba_b200_decode(ctypes.byref(cfg(hier=1)), 1, 128, one, one, one, one, one, one, one, one, one, z,
                             one, one, one, z, z, z, one, 1 << 20, z)
    assert st == _lib.ERR_INVALID_ARGUMENT                                             # hier needs supers
    st = lib.hba_b200_decode(ctypes.byref(c), 1, 128, one, one, one, one, one, one, z, one, one, z, one, one,
                             one, z, z, z, one, 1 << 20, z)
    assert st == _lib.ERR_INVALID_ARGUMENT                                             # needs the RoPE'd keys
    st = lib.hba_b200_qknorm(z, one, one, 4, 2, 64, ctypes.c_float(1e-6), z)
    assert st == _lib.ERR_INVALID_ARGUMENT


def test_status_maps_to_reference_style_exceptions():
    from hba_b200 import _lib
    with pytest.raises(AssertionError):
        _lib.check(_lib.ERR_NOT_BLOCK_MULTIPLE, "x")
    with pytest.raises(ValueError):
        _lib.check(_lib.ERR_INVALID_ARGUMENT, "x")
    with pytest.raises(NotImplementedError):
        _lib.check(_lib.ERR_UNSUPPORTED, "x")
    with pytest.raises(_lib.HBAError):
        _lib.check(_lib.ERR_CUDA, "x")


def test_backward_and_teacher_workspace_queries(lib):
    """hba_b200_prefill_backward / hba_b200_aux_teacher: sizes for the
    configurations their kernels take (flat, block 64, dh 64 / 128; the
    backward also G >= 4), 0 otherwise; the teacher's one-pass scratch is
    capped at 1 GiB whatever the batch and length."""
    c = cfg(n_heads=8, n_kv=2, block=64)
    ok_b = lib.hba_b200_prefill_backward_workspace_size(ctypes.byref(c), 1, 4096)
    ok_t = lib.hba_b200_aux_teacher_workspace_size(ctypes.byref(c), 1, 4096)
    assert ok_b > 0 and ok_t > 0
    for bad in (cfg(n_heads=8, n_kv=2, hier=1), cfg(n_heads=8, n_kv=2, block=32)):
        assert lib.hba_b200_prefill_backward_workspace_size(ctypes.byref(bad), 1, 4096) == 0
        assert lib.hba_b200_aux_teacher_workspace_size(ctypes.byref(bad), 1, 4096) == 0
    assert lib.hba_b200_prefill_backward_workspace_size(ctypes.byref(c), 1, 4000) == 0    # n % block
    # G = 2: outside the backward's tile shape, inside the teacher's
    g2 = cfg(n_heads=4, n_kv=2)
    assert lib.hba_b200_prefill_backward_workspace_size(ctypes.byref(g2), 1, 4096) == 0
    assert lib.hba_b200_aux_teacher_workspace_size(ctypes.byref(g2), 1, 4096) > 0
    # the teacher's scratch: all queries' masses when small, at most 1 GiB beyond
    big = cfg(n_heads=32, n_kv=8, head_dim=128)
    n = 131072
    kv = 4 * n * 8 * 128
    qv = 4 * n * 32 * 128
    base = 256 + 3 * kv * 2 + qv * 2
    t = lib.hba_b200_aux_teacher_workspace_size(ctypes.byref(big), 4, n)
    assert base < t <= base + (1 << 30) + 4096


def test_backward_and_teacher_reject_bad_arguments_without_a_device(lib):
    from hba_b200 import _lib
    c = cfg(n_heads=8, n_kv=2)
    P = ctypes.c_void_p
    one = P(16)
    z = P(0)
    args = [one] * 16  # q k v cos sin q_gain k_gain out lse sel dout dq dk dv dq_gain dk_gain
    st = lib.hba_b200_prefill_backward(ctypes.byref(c), 1, 100, ctypes.c_float(0.1), *args, one, 1 << 40, z)
    assert st == _lib.ERR_NOT_BLOCK_MULTIPLE
    st = lib.hba_b200_prefill_backward(ctypes.byref(c), 1, 128, ctypes.c_float(0.1), z, *args[1:], one, 1 << 40, z)
    assert st == _lib.ERR_INVALID_ARGUMENT
    st = lib.hba_b200_prefill_backward(ctypes.byref(cfg(n_heads=8, n_kv=2, hier=1)), 1, 128, ctypes.c_float(0.1),
                                       *args, one, 1 << 40, z)
    assert st == _lib.ERR_UNSUPPORTED
    st = lib.hba_b200_prefill_backward(ctypes.byref(c), 1, 128, ctypes.c_float(0.1), *args, one, 16, z)
    assert st == _lib.ERR_WORKSPACE
    targs = [one] * 7  # q k cos sin q_gain k_gain pstar
    st = lib.hba_b200_aux_teacher(ctypes.byref(c), 1, 100, ctypes.c_float(0.1), *targs, one, 1 << 40, z)
    assert st == _lib.ERR_NOT_BLOCK_MULTIPLE
    st = lib.hba_b200_aux_teacher(ctypes.byref(c), 1, 128, ctypes.c_float(0.1), *targs[:6], z, one, 1 << 40, z)
    assert st == _lib.ERR_INVALID_ARGUMENT
    st = lib.hba_b200_aux_teacher(ctypes.byref(c), 1, 128, ctypes.c_float(0.1), *targs, one, 16, z)
    assert st == _lib.ERR_WORKSPACE
