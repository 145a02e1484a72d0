"""ctypes binding of libfast_trimul_b200.so (the C ABI in include/fast_trimul_b200.h).

The library is built in-tree (`python fast_trimul_b200/csrc/build.py`). Loading is
lazy; `load()` raises `NativeLibraryMissing` when the .so is absent or lacks a
symbol, and the CUDA backend lets that error propagate instead of silently
falling back.
"""

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
# FTM_LIBRARY names another build of the same library (A/B measurements of two builds)
LIB_PATH = os.environ.get("FTM_LIBRARY") or os.path.join(HERE, "libfast_trimul_b200.so")

# status codes (ftm_status)
OK, BAD_SHAPE, BAD_DTYPE, BAD_ALIGN, UNSUPPORTED_ARCH, LAUNCH_FAILED, TIMEOUT, BAD_WORKSPACE, \
    BAD_ARGUMENT = range(9)
# dtypes (ftm_dtype) and modes (ftm_mode)
F32, F16, BF16 = 0, 1, 2
OUTGOING, INCOMING = 0, 1

# every symbol the header declares, with (restype, argtypes)
_vp, _i32, _sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_size_t


class Problem(ctypes.Structure):
    """Mirror of ftm_problem."""
    _fields_ = [("batch", _i32), ("rows", _i32), ("cols", _i32), ("c_z", _i32), ("c_h", _i32),
                ("mode", _i32), ("residual", _i32), ("z_dtype", _i32), ("out_dtype", _i32),
                ("eps_in", ctypes.c_float), ("eps_out", ctypes.c_float)]


MAX_RANKS = 8


class PeerPlanes(ctypes.Structure):
    """Mirror of ftm_peer_planes: rank q's receive plane as mapped in this process."""
    _fields_ = [("world", _i32), ("rank", _i32), ("base", _vp * MAX_RANKS)]

    @classmethod
    def make(cls, world, rank, ptrs):
        pp = cls()
        pp.world, pp.rank = world, rank
        for q, ptr in enumerate(ptrs):
            pp.base[q] = ptr
        return pp


SHARD_ALLTOALL, SHARD_ALLGATHER = 0, 1
SHARD_MAX_ROW_CHUNKS = 8
SHARD_FLAG_WORDS = 256
SHARD_BUF_LOCAL, SHARD_BUF_ZSTATS, SHARD_BUF_XBLOCKS, SHARD_BUF_RECV, SHARD_BUF_XPLANE, \
    SHARD_BUF_FLAGS = range(6)


class ShardConfig(ctypes.Structure):
    """Mirror of ftm_shard_config."""
    _fields_ = [("world", _i32), ("rank", _i32), ("scheme", _i32), ("row_chunks", _i32),
                ("shard", Problem), ("packed", _vp), ("a_local", _vp),
                ("zstats", _vp), ("x_blocks", _vp), ("err_word", _vp),
                ("recv_a", _vp * MAX_RANKS), ("recv_b", _vp * MAX_RANKS),
                ("x_plane", _vp * MAX_RANKS), ("flags", _vp * MAX_RANKS)]


class ContractionLayout(ctypes.Structure):
    """Mirror of ftm_contraction_layout."""
    _i64 = ctypes.c_int64
    _fields_ = [("L", _i32), ("m", _i32), ("n", _i32), ("k", _i32), ("k_per_block", _i32),
                ("a", _vp), ("a_rows_per_block", _i32), ("a_block_stride", _i64),
                ("a_l_stride", _i64), ("a_row_stride", _i64), ("a_kblock_stride", _i64),
                ("b", _vp), ("b_rows_per_block", _i32), ("b_block_stride", _i64),
                ("b_l_stride", _i64), ("b_row_stride", _i64), ("b_kblock_stride", _i64),
                ("x", _vp), ("x_rows_per_block", _i32), ("x_block_stride", _i64),
                ("x_l_stride", _i64), ("x_row_stride", _i64),
                ("a_mn_major", _i32), ("b_mn_major", _i32)]


_PP = ctypes.POINTER(Problem)
_IP = ctypes.POINTER(ctypes.c_int)
_PPL = ctypes.POINTER(PeerPlanes)

SIGNATURES = {
    "ftm_packed_params_bytes": (_sz, [_i32, _i32]),
    "ftm_pack_params": (ctypes.c_int, [ctypes.POINTER(_vp), _i32, _i32, _i32, _vp, _vp]),
    "ftm_workspace_bytes": (_sz, [_PP]),
    "ftm_trimul_fwd": (ctypes.c_int, [_PP, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "ftm_input_stage": (ctypes.c_int, [_PP, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "ftm_contraction": (ctypes.c_int, [_vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _vp, _vp]),
    "ftm_contraction_blocked": (ctypes.c_int, [_vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32,
                                               _vp, _vp]),
    "ftm_output_stage": (ctypes.c_int, [_PP, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "ftm_input_stage_scatter": (ctypes.c_int, [_PP, _vp, _vp, _vp, _PPL, _PPL, _vp, _vp, _vp]),
    "ftm_contraction_scatter": (ctypes.c_int, [_vp, _vp, _PPL, _i32, _i32, _i32, _i32, _i32, _vp,
                                               _vp]),
    "ftm_contraction_kblocked": (ctypes.c_int, [_vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32,
                                                _vp, _vp]),
    "ftm_check_error": (ctypes.c_int, [_vp, _IP, _vp]),
    "ftm_workspace_error_word": (_vp, [_PP, _vp]),
    "ftm_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "ftm_device_supported": (ctypes.c_int, [ctypes.c_int]),
    "ftm_last_launch_count": (ctypes.c_int, []),
    "ftm_trimul_fwd_static_scratch": (ctypes.c_int, [_PP, _vp, _vp, _vp, _vp, _vp]),
    "ftm_contraction_general": (ctypes.c_int, [ctypes.POINTER(ContractionLayout), _vp, _vp]),
    "ftm_shard_buffer_bytes": (_sz, [ctypes.POINTER(ShardConfig), ctypes.c_int]),
    "ftm_shard_plan_create": (ctypes.c_int, [ctypes.POINTER(ShardConfig), ctypes.POINTER(_vp)]),
    "ftm_shard_forward": (ctypes.c_int, [_vp, _vp, _vp, _vp, _i32, _vp]),
    "ftm_shard_plan_destroy": (None, [_vp]),
    "ftm_shard_set_trace": (ctypes.c_int, [_vp, _vp]),
    "ftm_bwd_partial_blocks": (ctypes.c_int, []),
    "ftm_bwd_ln_in": (ctypes.c_int, [_vp, _i32, _vp, _vp, _vp, ctypes.c_float, _vp, _vp,
                                     ctypes.c_int64, _vp]),
    "ftm_bwd_x_ln": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_float, _vp, _vp, _i32, _i32, _vp]),
    "ftm_bwd_gate": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _i32, _vp, _vp, _vp, _vp,
                                    _vp, ctypes.c_int64, _vp]),
    "ftm_bwd_x_ln_bwd": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _vp]),
    "ftm_bwd_gates_in": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32,
                                        _vp]),
    "ftm_bwd_ln_in_bwd": (ctypes.c_int, [_vp, _i32, _vp, _vp, _vp, _vp, _vp, _i32, _vp,
                                         _i32, _vp, _i32, _vp, ctypes.c_int64, _vp]),
    "ftm_static_scratch_error_word": (_vp, []),
}


class NativeLibraryMissing(RuntimeError):
    """The CUDA library is not built / not loadable: a hard error, never a fallback."""


class NativeKernelError(RuntimeError):
    """A launch failed or a device-side bounded wait expired."""


class NativeDeclined(RuntimeError):
    """The kernels do not support this input (shape / dtype / device); callers may
    route it to another backend, exactly as the reference's guard does."""


_lock = threading.Lock()
_lib = None

# counters the tests use to prove the native path ran
stats = {"calls": 0, "kernel_launches": 0}


def load():
    """Load the shared library (once) and bind every declared symbol."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise NativeLibraryMissing(
                f"{LIB_PATH} not found: build it with `python fast_trimul_b200/csrc/build.py`")
        try:
            lib = ctypes.CDLL(LIB_PATH)
        except OSError as e:
            raise NativeLibraryMissing(f"cannot load {LIB_PATH}: {e}") from e
        for name, (res, args) in SIGNATURES.items():
            try:
                fn = getattr(lib, name)
            except AttributeError as e:
                raise NativeLibraryMissing(f"{LIB_PATH} lacks symbol {name}") from e
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def available():
    try:
        load()
        return True
    except NativeLibraryMissing:
        return False


def status_string(code):
    return load().ftm_status_string(int(code)).decode()


def check(code, what):
    """Map an ftm_status to the exception the dispatcher understands."""
    if code == OK:
        return
    msg = f"{what}: {status_string(code)} (status {code})"
    if code in (BAD_SHAPE, BAD_DTYPE, BAD_ALIGN, UNSUPPORTED_ARCH):
        raise NativeDeclined(msg)
    raise NativeKernelError(msg)


def record_launches():
    n = load().ftm_last_launch_count()
    stats["calls"] += 1
    stats["kernel_launches"] += n
    return n
