"""ctypes binding of ``libhba_b200.so`` (the C ABI declared in
``include/hba_b200.h``).  There is no fallback: if the library is missing or
no CUDA device is present, every entry point raises."""

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libhba_b200.so")

OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_NOT_BLOCK_MULTIPLE = 2
ERR_WORKSPACE = 3
ERR_UNSUPPORTED = 4
ERR_CUDA = 5
ERR_DEVICE_TIMEOUT = 6


class HBAError(RuntimeError):
    """A non-OK status from the CUDA library."""

    def __init__(self, status, what):
        self.status = status
        super().__init__(f"{what}: {status_string(status)} (status {status})")


class Config(ctypes.Structure):
    """Mirror of `hba_b200_config` (include/hba_b200.h)."""
    _fields_ = [("n_heads", ctypes.c_int32), ("n_kv", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("block", ctypes.c_int32), ("window", ctypes.c_int32), ("sinks", ctypes.c_int32),
                ("k_blocks", ctypes.c_int32), ("slots", ctypes.c_int32), ("fanout", ctypes.c_int32),
                ("beam", ctypes.c_int32), ("hier", ctypes.c_int32), ("qknorm", ctypes.c_int32),
                ("eps", ctypes.c_float)]


# Every exported symbol with its (restype, argtypes); the CPU test suite checks
# that the library exports exactly what include/hba_b200.h declares.
_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_F = ctypes.c_float
_SZ = ctypes.c_size_t
_CFG = ctypes.POINTER(Config)
SIGNATURES = {
    "hba_b200_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "hba_b200_version": (ctypes.c_int, []),
    "hba_b200_last_kernels": (ctypes.c_char_p, []),
    "hba_b200_qknorm": (ctypes.c_int, [_P, _P, _P, _I64, _I32, _I32, _F, _P]),
    "hba_b200_summarize": (ctypes.c_int, [_CFG, _I32, _I32, _P, _P, _P, _P, _I32, _I32, _P]),
    "hba_b200_build_supers": (ctypes.c_int, [_CFG, _I32, _I32, _I32, _P, _P, _I32, _I32, _P]),
    "hba_b200_append_kv": (ctypes.c_int, [_CFG, _I32, _I32, _I32, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                          _P, _P, _P]),
    "hba_b200_decode_workspace_size": (_SZ, [_CFG, _I32, _I32]),
    "hba_b200_decode": (ctypes.c_int, [_CFG, _I32, _I32, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                       _P, _P, _P, _P, _SZ, _P]),
    "hba_b200_decode_noalloc": (ctypes.c_int, [_CFG, _I32, _I32, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                               _P, _P, _P, _P, _P]),
    "hba_b200_decode_noalloc_status": (ctypes.c_int, [_I32, _P]),
    "hba_b200_device_status": (ctypes.c_int, [_P, _I32, _P]),
    "hba_b200_prefill_workspace_size": (_SZ, [_CFG, _I32, _I32]),
    "hba_b200_set_profile_events": (ctypes.c_int, [ctypes.POINTER(ctypes.c_void_p), _I32]),
    "hba_b200_profile_events_recorded": (ctypes.c_int, []),
    "hba_b200_set_debug_trace": (ctypes.c_int, [_P, _I64]),
    # cfg, batch, n_cap_local, tok_lo, level, seq_lens, scales, q, q_gain, summ, supers, in_idx, in_score,
    # n_in_lists, out_idx, out_score, stream
    "hba_b200_decode_shard_select": (ctypes.c_int, [_CFG, _I32, _I32, _I32, _I32, _P, _P, _P, _P, _P, _P, _P, _P,
                                                    _I32, _P, _P, _P]),
    # cfg, batch, n_cap_local, tok_lo, seq_lens, scales, q, q_gain, k_gain, k, kr, v, cos, sin, in_idx, in_score,
    # n_in, part_o, part_l, part_m2, sel_idx, sel_score, dev_status, stream
    "hba_b200_decode_shard_attend": (ctypes.c_int, [_CFG, _I32, _I32, _I32, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                                    _P, _P, _P, _I32, _P, _P, _P, _P, _P, _P, _P]),
    # cfg, batch, world, parts, out, lse, stream
    "hba_b200_decode_shard_finish": (ctypes.c_int, [_CFG, _I32, _I32, _P, _P, _P, _P]),
    "hba_b200_shard_xbuf_bytes": (_I64, [_CFG, _I32, _I32]),
    "hba_b200_host_alloc": (ctypes.c_int, [_I64, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p)]),
    "hba_b200_host_free": (ctypes.c_int, [_P]),
    "hba_b200_peer_alloc": (ctypes.c_int, [_I64, ctypes.POINTER(ctypes.c_void_p), _P]),
    "hba_b200_peer_open": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_void_p)]),
    "hba_b200_peer_close": (ctypes.c_int, [_P]),
    "hba_b200_peer_free": (ctypes.c_int, [_P]),
    # cfg, batch, n_cap_local, tok_lo, world, rank, xbufs, epoch, seq_lens, scales, q, q_gain, k_gain, summ,
    # supers, k, kr, v, cos, sin, out, lse, sel_idx, sel_score, dev_status, stream
    "hba_b200_decode_shard_fused": (ctypes.c_int, [_CFG, _I32, _I32, _I32, _I32, _I32, _P, _P, _P, _P, _P, _P,
                                                   _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "hba_b200_prefill": (ctypes.c_int, [_CFG, _I32, _I32, _F, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                        _P, _P, _SZ, _P]),
    "hba_b200_prefill_range_workspace_size": (_SZ, [_CFG, _I32, _I32, _I32]),
    # cfg, batch, n, q_lo, n_q, scale, q, k, v, cos, sin, q_gain, k_gain, probes, proj, out, lse, sel_idx,
    # sel_score, workspace, workspace_bytes, stream
    "hba_b200_prefill_range": (ctypes.c_int, [_CFG, _I32, _I32, _I32, _I32, _F, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                              _P, _P, _P, _P, _P, _SZ, _P]),
    "hba_b200_aux_teacher_workspace_size": (_SZ, [_CFG, _I32, _I32]),
    # cfg, batch, n, scale, q, k, cos, sin, q_gain, k_gain, pstar, workspace, workspace_bytes, stream
    "hba_b200_aux_teacher": (ctypes.c_int, [_CFG, _I32, _I32, _F, _P, _P, _P, _P, _P, _P, _P, _P, _SZ, _P]),
    "hba_b200_prefill_backward_workspace_size": (_SZ, [_CFG, _I32, _I32]),
    # cfg, batch, n, scale, q, k, v, cos, sin, q_gain, k_gain, out, lse, sel_idx, dout, dq, dk, dv, dq_gain,
    # dk_gain, workspace, workspace_bytes, stream
    "hba_b200_prefill_backward": (ctypes.c_int, [_CFG, _I32, _I32, _F, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                                 _P, _P, _P, _P, _P, _P, _SZ, _P]),
}

_lib = None


def load():
    """Load the library once (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is not built; run `python -m hba_b200._build` from hierarchical-block-attention_b200/ "
                "(the HBA B200 path has no CPU fallback)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def status_string(status):
    try:
        return load().hba_b200_status_string(int(status)).decode()
    except Exception:
        return "unknown"


def check_device(status_word_ptr, stream, what, clear=False):
    """Wait for `stream`, read a kernel status word (a workspace's first 4
    bytes, or a shard call's dev_status) and raise HBAError
    (ERR_DEVICE_TIMEOUT: a bounded device-side wait expired) unless it is 0."""
    check(load().hba_b200_device_status(status_word_ptr, 1 if clear else 0, stream), what)


def check(status, what):
    if status == OK:
        return
    if status == ERR_NOT_BLOCK_MULTIPLE:
        # the reference asserts n % Bk == 0 (src/hba/attention.py:339,581,650)
        raise AssertionError(f"{what}: sequence length is not a multiple of the block size")
    if status == ERR_INVALID_ARGUMENT:
        raise ValueError(f"{what}: {status_string(status)}")
    if status == ERR_UNSUPPORTED:
        raise NotImplementedError(f"{what}: {status_string(status)}")
    raise HBAError(status, what)
