"""ctypes binding of liblssab8_b200.so (the C ABI declared in include/lssab8.h).

There is no fallback: if the library is missing or fails to load, importing the product
modules raises, so no caller can silently run a non-native path.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIBPATH = os.path.join(_HERE, "liblssab8_b200.so")

DT_F32, DT_F16, DT_BF16 = 0, 1, 2
DEV_EV_RANGE, DEV_TIMEOUT, DEV_BAD_PAGE, DEV_ALIGN = 1, 2, 4, 8

# every symbol include/lssab8.h declares (tests check the library exports each one)
SYMBOLS = (
    "lssab8_version", "lssab8_strerror", "lssab8_device_errors",
    "lssab8_quant_rows", "lssab8_quant_heads", "lssab8_quant_blocks", "lssab8_quant_keys_offset",
    "lssab8_quant_values_keyshift",
    "lssab8_prefill_lattice", "lssab8_prefill_lattice_general", "lssab8_prefill_lattice_keyshift",
    "lssab8_prefill_chunk_lattice", "lssab8_prefill_workspace_size", "lssab8_prefill",
    "lssab8_prefill_peers", "lssab8_peer_export", "lssab8_peer_import", "lssab8_peer_close", "lssab8_peer_copy2d",
    "lssab8_decode_prep_kv", "lssab8_kv_append", "lssab8_decode_workspace_size", "lssab8_decode",
    "lssab8_decode_noalloc", "lssab8_selftest_div", "lssab8_selftest_rescale", "lssab8_selftest_timeout",
)

_lib = None


class Lssab8Error(RuntimeError):
    def __init__(self, code, what):
        self.code = code
        super().__init__("%s: %s (status %d)" % (what, strerror(code) if _lib else "?", code))


def load():
    """Load (once) and return the library; raises OSError if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIBPATH):
        raise OSError("liblssab8_b200.so is not built (run lockstep_b200/build.py or __graft_entry__.build())")
    L = ctypes.CDLL(LIBPATH)
    P, I, I64, SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t
    PI64 = ctypes.POINTER(ctypes.c_int64)
    L.lssab8_version.argtypes = [ctypes.c_char_p, I]
    L.lssab8_strerror.argtypes = [I]
    L.lssab8_strerror.restype = ctypes.c_char_p
    L.lssab8_device_errors.argtypes = [I, P, ctypes.POINTER(I)]
    L.lssab8_quant_rows.argtypes = [P, I, I, I, I, I, PI64, I, P, P, P]
    L.lssab8_quant_heads.argtypes = [P, I, I, I, I, I, PI64, I, P, P, P]
    L.lssab8_quant_blocks.argtypes = [P, I, I, I, I, I, PI64, I, I, P, P, P, P]
    L.lssab8_prefill_lattice_general.argtypes = [P] * 7 + [I] * 7 + [P, P, PI64, P]
    L.lssab8_quant_values_keyshift.argtypes = [P, I, I, I, I, I, PI64, I, I, I, P, P, P, P, P]
    L.lssab8_prefill_lattice_keyshift.argtypes = [P] * 8 + [I] * 6 + [P, I, PI64, P]
    L.lssab8_quant_keys_offset.argtypes = [P, I, I, I, I, I, PI64, I, P, P, P, P]
    L.lssab8_prefill_lattice.argtypes = [P] * 7 + [I] * 6 + [P, P, I, PI64, P]
    L.lssab8_prefill_chunk_lattice.argtypes = [P] * 7 + [I] * 6 + [P, P, I, PI64, P]
    L.lssab8_prefill_workspace_size.argtypes = [I] * 5
    L.lssab8_prefill_workspace_size.restype = SZ
    L.lssab8_prefill.argtypes = [P, P, P, I, I, I, I, I, I, PI64, PI64, PI64, I, P, I, PI64, P, SZ, P]
    L.lssab8_prefill_peers.argtypes = [P, P, P, I, I, I, I, I, I, PI64, PI64, PI64, I, P, I, PI64, P, I, P, SZ, P]
    L.lssab8_peer_export.argtypes = [P, P, ctypes.POINTER(ctypes.c_uint64)]
    L.lssab8_peer_import.argtypes = [P, ctypes.c_uint64, I, ctypes.POINTER(P)]
    L.lssab8_peer_close.argtypes = [P, ctypes.c_uint64]
    L.lssab8_peer_copy2d.argtypes = [P, SZ, P, SZ, SZ, SZ, P]
    L.lssab8_decode_prep_kv.argtypes = [P, P, I, I, I, I, P, P, I64, I64, I64, P, I, I, I, I, P, P, P, P, P, P]
    L.lssab8_kv_append.argtypes = [P, P, I, I, I, I, P, P, P, I64, I64, P, I64, P, I, I, I, I, P, P, P, P, P, P]
    L.lssab8_decode_workspace_size.argtypes = [I] * 5
    L.lssab8_decode_workspace_size.restype = SZ
    L.lssab8_decode.argtypes = [P, I, PI64, I, I, I, I, P, P, I, I, P, P, P, P, P, I, I, I, P, I, PI64, P, SZ, P]
    L.lssab8_decode_noalloc.argtypes = [P, I, PI64, I, I, I, I, P, P, I, I, P, P, P, P, P, I, I, I, P, I, PI64, P]
    L.lssab8_selftest_div.argtypes = [P, P, I64, P, P]
    L.lssab8_selftest_rescale.argtypes = [P, P, I64, P, P]
    L.lssab8_selftest_timeout.argtypes = [P] * 6 + [I] * 7 + [P, PI64, P]
    for name in SYMBOLS:
        getattr(L, name).restype = getattr(L, name).restype or I
    _lib = L
    return L


def strerror(code):
    return load().lssab8_strerror(int(code)).decode()


def check(rc, what):
    if rc != 0:
        raise Lssab8Error(rc, what)


def version():
    buf = ctypes.create_string_buffer(160)
    check(load().lssab8_version(buf, len(buf)), "lssab8_version")
    return buf.value.decode()


def i64x(vals):
    arr = (ctypes.c_int64 * len(vals))(*[int(v) for v in vals])
    return arr


def device_errors(stream=None, clear=True):
    bits = ctypes.c_int(0)
    check(load().lssab8_device_errors(int(clear), stream, ctypes.byref(bits)), "lssab8_device_errors")
    return bits.value
