"""The C-ABI library: it loads, exports every symbol include/lssab8.h declares, reports the
contract's T2 digest, and rejects bad arguments with status codes (no GPU needed: argument
validation happens before any CUDA call)."""
import ctypes
import os
import re

import pytest

from lockstep_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    src = open(os.path.join(ROOT, "include", "lssab8.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(lssab8_\w+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    L = _lib.load()
    names = header_symbols()
    assert len(names) >= 10
    for n in names:
        assert hasattr(L, n), n
    assert sorted(_lib.SYMBOLS) == names


def test_version_reports_contract_t2_digest():
    v = _lib.version()
    assert v.startswith("lssab8-b200 ")
    assert v.endswith("T2=7a42a785940f557d5d5a4188fa5683ea00cf8b29e8d5213c75c581a5a0d92fbb")


def test_strerror():
    assert _lib.strerror(0) == "ok"
    assert "workspace" in _lib.strerror(4)


def test_workspace_sizes():
    L = _lib.load()
    n = L.lssab8_prefill_workspace_size(4, 32, 8, 2048, 128)
    # q8 + k8 + v8 + exponents, 256-byte aligned pieces
    assert n >= 4 * 32 * 2048 * 128 + 2 * 4 * 8 * 2048 * 128
    assert L.lssab8_prefill_workspace_size(1, 3, 2, 128, 128) == 0      # H % KVH != 0
    assert L.lssab8_decode_workspace_size(32, 32, 8, 128, 64) >= 32 * 8 * 64 * 4 * 128 * 4


def test_bad_arguments_return_status_codes():
    L = _lib.load()
    s4 = _lib.i64x([0, 0, 0, 0])
    # null pointers -> EARG, before any CUDA call
    rc = L.lssab8_prefill(None, None, None, 2, 1, 8, 8, 128, 64, s4, s4, s4, 0, None, 2, s4, None, 0, None)
    assert rc == 1
    buf = ctypes.create_string_buffer(8)
    assert L.lssab8_version(buf, 8) == 1
    # unsupported head dim on an otherwise valid call -> EUNSUPPORTED before touching memory
    fake = ctypes.c_void_p(256)
    rc = L.lssab8_prefill(fake, fake, fake, 2, 1, 8, 8, 128, 96, s4, s4, s4, 0, fake, 2, s4, fake, 1 << 30, None)
    assert rc == 2
    # the key-offset quantiser needs its offset
    ks = _lib.i64x([2 * 300 * 64, 300 * 64, 64, 1])
    rc = L.lssab8_quant_keys_offset(fake, 2, 1, 2, 300, 64, ks, 384, None, fake, fake, None)
    assert rc == 1
    # a chunk must start on a 128-key block boundary, below the sequence length
    for T0, T in ((100, 300), (256, 256), (-128, 300)):
        rc = L.lssab8_prefill_chunk_lattice(fake, fake, fake, fake, fake, fake, None, 1, 8, 8, T0, T, 128, None,
                                            fake, 2, s4, None)
        assert rc == 1, (T0, T)
