"""ctypes binding of libternocl.so (the C ABI declared in include/ternocl.h).

The shared library is built in-tree (``ternocl_b200/lib/libternocl.so``) by
``python -m ternocl_b200.build`` / ``make -C ternocl_b200/csrc``.  There is no
fallback: if the library is missing or cannot be loaded, every call raises.
"""
import ctypes as C
import os
import re

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libternocl.so")
HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "ternocl.h")

TERNOCL_OK = 0
STATUS_NAMES = {0: "OK", 1: "ERR_SHAPE", 2: "ERR_ARG", 3: "ERR_CUDA", 4: "ERR_TIMEOUT",
                5: "ERR_COMM", 6: "ERR_UNSUPPORTED", 7: "ERR_WORKSPACE"}

vp, i32, sz, u64, f64 = C.c_void_p, C.c_int, C.c_size_t, C.c_uint64, C.c_double

# name -> (restype, argtypes); must match include/ternocl.h
SIGNATURES = {
    "ternocl_version": (C.c_char_p, []),
    "ternocl_status_string": (C.c_char_p, [i32]),
    "ternocl_last_error": (C.c_char_p, []),
    "ternocl_set_option": (i32, [i32, i32]),
    "ternocl_device_error": (i32, [i32]),
    "ternocl_gemv_workspace_size": (sz, [i32, i32, i32]),
    "ternocl_int2_upcvt": (i32, [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, vp, sz, vp]),
    "ternocl_int2_upcvt_noalloc": (i32, [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, vp]),
    "ternocl_gemv_allgather_workspace_size": (sz, [i32, i32, i32]),
    "ternocl_ipc_handle": (i32, [vp, vp, vp]),
    "ternocl_ipc_open": (i32, [vp, sz, vp]),
    "ternocl_ipc_close": (i32, [vp, sz]),
    "ternocl_int2_upcvt_allgather": (i32, [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, i32, i32,
                                           i32, vp, C.c_uint, vp, sz, vp]),
    "ternocl_int1_upcvt": (i32, [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, vp, sz, vp]),
    "ternocl_int8_ldsa": (i32, [i32]),
    "ternocl_int8_quant_a": (i32, [vp, vp, vp, i32, i32, i32, vp]),
    "ternocl_int2_int8": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, i32, vp]),
    "ternocl_int2_int8_group_dots": (i32, [vp, vp, vp, i32, i32, i32, vp]),
    "ternocl_bitcos_upcvt": (i32, [vp, vp, vp, vp, i32, vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, vp]),
    "ternocl_hadamard_fwht": (i32, [vp, vp, vp, i32, i32, i32, i32, i32, vp]),
    "ternocl_bitcos_upcvt_hadamard": (i32, [vp, vp, i32, i32, vp, vp, vp, i32, vp, vp, vp, i32, i32, i32, i32, i32,
                                            i32, vp]),
    "ternocl_moe_rows_per_tile": (i32, []),
    "ternocl_moe_route": (i32, [vp, vp, vp, vp, i32, i32, i32, vp]),
    "ternocl_moe_gather": (i32, [vp, vp, vp, i32, i32, i32, vp]),
    "ternocl_moe_gemm": (i32, [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, vp]),
    "ternocl_moe_gather_q": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, i32, vp]),
    "ternocl_moe_gemm_i8": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, i32, vp]),
    "ternocl_moe_combine": (i32, [vp, vp, vp, vp, i32, i32, i32, i32, vp]),
    "ternocl_moe_decode_gate_up": (i32, [vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, vp]),
    "ternocl_moe_decode_down": (i32, [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, vp]),
    "ternocl_moe_decode_reduce": (i32, [vp, vp, i32, i32, i32, i32, vp]),
    "ternocl_moe_decode_down_sum": (i32, [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, vp]),
    "ternocl_bitcos_random": (sz, [i32, i32, f64, u64, vp, sz]),
    "ternocl_bitcos_pack": (sz, [vp, i32, i32, vp, sz]),
    "ternocl_bitcos_slice_ranks": (i32, [vp, i32, i32, i32, vp]),
    "ternocl_int1_to_sel": (i32, [vp, vp, i32, i32]),
}

_lib = None


class TernoclError(RuntimeError):
    def __init__(self, fn, status):
        self.status = status
        msg = "%s failed: %s (%s)" % (fn, STATUS_NAMES.get(status, status),
                                     lib().ternocl_status_string(status).decode())
        err = lib().ternocl_last_error().decode()
        if err:
            msg += " [" + err + "]"
        super().__init__(msg)


def header_functions():
    """Names of the functions declared in include/ternocl.h."""
    with open(HEADER) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ternocl_[a-z0-9_]+)\s*\(", text)))


def lib():
    """Load libternocl.so (raises OSError if it is absent: no fallback exists)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError("libternocl.so not built: %s (run python -m ternocl_b200.build)" % LIB_PATH)
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def call(name, *args):
    """Call a status-returning entry point; raise TernoclError unless it returns OK."""
    st = getattr(lib(), name)(*args)
    if st != TERNOCL_OK:
        raise TernoclError(name, st)
    return st
