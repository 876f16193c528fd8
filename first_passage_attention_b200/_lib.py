"""ctypes binding of libfpa_b200.so (the C ABI declared in include/fpa.h).

The library is loaded lazily on first use; a missing or stale library raises immediately. There is no fallback:
the CUDA path either runs the native kernels or fails with the reason.
"""
import ctypes
import os
import struct
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("FPA_B200_LIB", os.path.join(HERE, "libfpa_b200.so"))

ABI_VERSION = 1
DTYPE_F16, DTYPE_F32 = 0, 1
PATH_AUTO, PATH_SIMT, PATH_TENSOR = 0, 1, 2
OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA, ERR_TIMEOUT, ERR_WORKSPACE = range(6)

# Exported symbols, in the order include/fpa.h declares them.
EXPORTS = ("fpa_abi_version", "fpa_struct_size", "fpa_fwd_workspace_bytes", "fpa_bwd_workspace_bytes", "fpa_fwd",
           "fpa_bwd", "fpa_field_fwd", "fpa_field_bwd", "fpa_workspace_status", "fpa_status_string", "fpa_last_error", "fpa_profile",
           "fpa_profile_report", "fpa_selftest_wait_timeout", "fpa_fwd_noalloc")
NOALLOC_SCRATCH_BYTES = 8 << 20

_c_i64x4 = ctypes.c_int64 * 4


class FpaFwdArgs(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int32), ("path", ctypes.c_int32),
                ("B", ctypes.c_int32), ("H", ctypes.c_int32), ("T", ctypes.c_int32), ("D", ctypes.c_int32),
                ("tau", ctypes.c_float),
                ("q", ctypes.c_void_p), ("q_stride", _c_i64x4),
                ("k", ctypes.c_void_p), ("k_stride", _c_i64x4),
                ("v", ctypes.c_void_p), ("v_stride", _c_i64x4),
                ("phi", ctypes.c_void_p), ("psi", ctypes.c_void_p), ("beta", ctypes.c_void_p),
                ("o", ctypes.c_void_p), ("o_stride", _c_i64x4),
                ("lse", ctypes.c_void_p),
                ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
                ("kernels_launched", ctypes.c_int32), ("path_taken", ctypes.c_int32)]


class FpaBwdArgs(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int32), ("path", ctypes.c_int32),
                ("B", ctypes.c_int32), ("H", ctypes.c_int32), ("T", ctypes.c_int32), ("D", ctypes.c_int32),
                ("tau", ctypes.c_float),
                ("q", ctypes.c_void_p), ("q_stride", _c_i64x4),
                ("k", ctypes.c_void_p), ("k_stride", _c_i64x4),
                ("v", ctypes.c_void_p), ("v_stride", _c_i64x4),
                ("o", ctypes.c_void_p), ("o_stride", _c_i64x4),
                ("dout", ctypes.c_void_p), ("dout_stride", _c_i64x4),
                ("lse", ctypes.c_void_p), ("phi", ctypes.c_void_p), ("psi", ctypes.c_void_p),
                ("beta", ctypes.c_void_p),
                ("dq", ctypes.c_void_p), ("dq_stride", _c_i64x4),
                ("dk", ctypes.c_void_p), ("dk_stride", _c_i64x4),
                ("dv", ctypes.c_void_p), ("dv_stride", _c_i64x4),
                ("dphi", ctypes.c_void_p), ("dpsi", ctypes.c_void_p), ("dbeta", ctypes.c_void_p),
                ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
                ("kernels_launched", ctypes.c_int32), ("path_taken", ctypes.c_int32)]


class FpaFieldArgs(ctypes.Structure):
    _fields_ = [("B", ctypes.c_int32), ("T", ctypes.c_int32), ("H", ctypes.c_int32),
                ("proj", ctypes.c_void_p), ("proj_stride", ctypes.c_int64 * 3),
                ("phi", ctypes.c_void_p), ("psi", ctypes.c_void_p),
                ("dphi", ctypes.c_void_p), ("dpsi", ctypes.c_void_p),
                ("dproj", ctypes.c_void_p), ("dproj_stride", ctypes.c_int64 * 3)]


def _packer(cls):
    """A struct.Struct with the byte layout of the ctypes Structure `cls` (the compiler's padding included), so that
    one pack_into call fills an argument block: much cheaper per call than the keyword constructor."""
    codes = {ctypes.c_int32: "i", ctypes.c_float: "f", ctypes.c_void_p: "Q", ctypes.c_size_t: "Q"}
    fmt, pos = "<", 0
    for name, ct in cls._fields_:
        f = getattr(cls, name)
        if f.offset > pos:
            fmt += f"{f.offset - pos}x"
        fmt += codes.get(ct) or f"{ct._length_}q"
        pos = f.offset + f.size
    if ctypes.sizeof(cls) > pos:
        fmt += f"{ctypes.sizeof(cls) - pos}x"
    packer = struct.Struct(fmt)
    assert packer.size == ctypes.sizeof(cls), (cls.__name__, packer.size, ctypes.sizeof(cls))
    return packer


# Field order of the packers = the order of _fields_ (pointers as integers, each stride array as four integers).
FWD_PACKER = _packer(FpaFwdArgs)
BWD_PACKER = _packer(FpaBwdArgs)

_lock = threading.Lock()
_lib = None


def load():
    """Load and check the native library (once per process)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"the FPA CUDA library is not built ({LIB_PATH} is missing); "
                               "run `python -m first_passage_attention_b200.build`")
        lib = ctypes.CDLL(LIB_PATH)
        lib.fpa_abi_version.restype = ctypes.c_int
        lib.fpa_struct_size.restype = ctypes.c_size_t
        lib.fpa_struct_size.argtypes = [ctypes.c_int]
        for n in ("fpa_fwd_workspace_bytes", "fpa_bwd_workspace_bytes"):
            f = getattr(lib, n)
            f.restype = ctypes.c_size_t
            f.argtypes = [ctypes.c_int] * 6
        lib.fpa_fwd.restype = ctypes.c_int
        lib.fpa_fwd.argtypes = [ctypes.POINTER(FpaFwdArgs), ctypes.c_void_p]
        lib.fpa_bwd.restype = ctypes.c_int
        lib.fpa_bwd.argtypes = [ctypes.POINTER(FpaBwdArgs), ctypes.c_void_p]
        for n in ("fpa_field_fwd", "fpa_field_bwd"):
            f = getattr(lib, n)
            f.restype = ctypes.c_int
            f.argtypes = [ctypes.POINTER(FpaFieldArgs), ctypes.c_void_p]
        lib.fpa_workspace_status.restype = ctypes.c_int
        lib.fpa_workspace_status.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        lib.fpa_status_string.restype = ctypes.c_char_p
        lib.fpa_status_string.argtypes = [ctypes.c_int]
        lib.fpa_last_error.restype = ctypes.c_char_p
        lib.fpa_profile.restype = ctypes.c_int
        lib.fpa_profile.argtypes = [ctypes.c_int]
        lib.fpa_profile_report.restype = ctypes.c_int
        lib.fpa_profile_report.argtypes = [ctypes.c_char_p, ctypes.c_size_t]
        lib.fpa_selftest_wait_timeout.restype = ctypes.c_int
        lib.fpa_selftest_wait_timeout.argtypes = [ctypes.c_void_p, ctypes.c_ulonglong, ctypes.c_void_p]
        lib.fpa_fwd_noalloc.restype = ctypes.c_int
        lib.fpa_fwd_noalloc.argtypes = [ctypes.POINTER(FpaFwdArgs), ctypes.c_void_p]
        if lib.fpa_abi_version() != ABI_VERSION:
            raise RuntimeError(f"libfpa_b200 ABI version {lib.fpa_abi_version()} != {ABI_VERSION}; rebuild it")
        if lib.fpa_struct_size(0) != ctypes.sizeof(FpaFwdArgs) or lib.fpa_struct_size(1) != ctypes.sizeof(FpaBwdArgs) \
                or lib.fpa_struct_size(2) != ctypes.sizeof(FpaFieldArgs):
            raise RuntimeError("libfpa_b200 argument structs do not match the Python mirror; rebuild it")
        _lib = lib
        return lib


def profile_report():
    """{kernel: (launches, total ms)} of the launches recorded since profiling was enabled (clears them)."""
    lib = load()
    buf = ctypes.create_string_buffer(1 << 16)
    n = lib.fpa_profile_report(buf, len(buf))
    if n < 0:
        raise RuntimeError("fpa_profile_report failed")
    out = {}
    for line in buf.value.decode().splitlines():
        name, cnt, ms = line.split()
        out[name] = (int(cnt), float(ms))
    return out


def check(rc):
    """Turn a non-zero FpaStatus into an exception carrying the library's message."""
    if rc == OK:
        return
    lib = load()
    msg = lib.fpa_last_error().decode() or lib.fpa_status_string(rc).decode()
    if rc == ERR_INVALID:
        raise ValueError(msg)
    raise RuntimeError(f"libfpa_b200: {lib.fpa_status_string(rc).decode()}: {msg}")
