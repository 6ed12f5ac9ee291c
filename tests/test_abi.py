"""The C-ABI library loads on a host without a GPU and exports every symbol include/ktmoe.h declares."""

import ctypes
import os
import re

import pytest

import tritify_b200 as tb
from tritify_b200 import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "ktmoe.h")).read()
    return sorted(set(re.findall(r"\b(ktmoe_[a-z0-9_]+)\s*\(", text)))


def test_every_declared_symbol_is_exported_and_bound():
    lib = ctypes.CDLL(_native.LIB_PATH)
    names = declared_symbols()
    assert len(names) >= 25
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/ktmoe.h but not exported"
    assert set(names) == set(_native.SIGNATURES), "the ctypes binding and the header disagree"


def test_error_strings_and_argument_checks():
    L = tb.lib()
    for st in range(0, 8):
        assert L.ktmoe_error_string(st)
    assert L.ktmoe_device_count(None) == _native.ERR_ARG
    assert L.ktmoe_open(0, None) == _native.ERR_ARG


def test_no_device_here_is_reported_not_crashed():
    if tb.device_count() > 0:
        pytest.skip("a GPU is present")
    h = ctypes.c_void_p()
    assert tb.lib().ktmoe_open(0, ctypes.byref(h)) == _native.ERR_NO_DEVICE


def declared_arities():
    """name -> number of parameters, from each `ret ktmoe_name(params);` declaration of the header."""
    text = open(os.path.join(ROOT, "include", "ktmoe.h")).read()
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    out = {}
    for m in re.finditer(r"\b(ktmoe_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", text):
        params = " ".join(m.group(2).split())
        out[m.group(1)] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_the_binding_passes_as_many_arguments_as_the_header_declares():
    arity = declared_arities()
    assert len(arity) >= 25
    for name, (argtypes, _) in _native.SIGNATURES.items():
        assert name in arity, name
        assert len(argtypes) == arity[name], f"{name}: header {arity[name]} parameters, binding {len(argtypes)}"


# Entry points whose all-zero call is empty work, not an error (nothing to generate, no rows); the string and handle
# getters return a string or NULL; every other entry point must refuse null handles and buffers with KTMOE_ERR_ARG.
EMPTY_OK = {"ktmoe_lcg_uniform", "ktmoe_linear_noalloc", "ktmoe_synth_normal", "ktmoe_synth_normal_portable"}
NOT_STATUS = {"ktmoe_error_string", "ktmoe_last_error", "ktmoe_stream"}

_NULL_SWEEP = r"""
import ctypes, sys
sys.path.insert(0, sys.argv[1])
import tritify_b200 as tb
from tritify_b200 import _native
L = tb.lib()
ints = (ctypes.c_int, ctypes.c_int32, ctypes.c_int64, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_size_t,
        ctypes.c_uint8, ctypes.c_int8, ctypes.c_long, ctypes.c_ulong, ctypes.c_longlong, ctypes.c_ulonglong)
for name in sorted(_native.SIGNATURES):
    argtypes, _ = _native.SIGNATURES[name]
    args = []
    for t in argtypes:
        if t in (ctypes.c_double, ctypes.c_float):
            args.append(0.0)
        elif isinstance(t, type) and issubclass(t, ctypes.Structure):
            args.append(t())
        elif t in ints:
            args.append(0)
        else:
            args.append(None)
    print("CALL", name, flush=True)
    print("RESULT", name, repr(getattr(L, name)(*args)), flush=True)
"""


def test_every_entry_point_refuses_null_handles_without_crashing():
    """Each exported function, called with null pointers and zero sizes (in a child process, so that a crash names
    the function it happened in), returns KTMOE_ERR_ARG, or OK where the call is empty work; none touches the
    missing objects. The C ABI never aborts its host (the reference's Rust contract turns statuses into panics)."""
    import subprocess
    import sys

    r = subprocess.run([sys.executable, "-c", _NULL_SWEEP, ROOT], capture_output=True, text=True, timeout=600)
    calls = [ln.split()[1] for ln in r.stdout.splitlines() if ln.startswith("CALL")]
    assert r.returncode == 0, f"crashed in {calls[-1] if calls else '?'}: {r.stderr[-2000:]}"
    results = {}
    for ln in r.stdout.splitlines():
        if ln.startswith("RESULT"):
            _, name, val = ln.split(" ", 2)
            results[name] = val
    assert set(results) == set(_native.SIGNATURES)
    for name, val in results.items():
        if name in NOT_STATUS:
            continue
        want = str(_native.OK) if name in EMPTY_OK else str(_native.ERR_ARG)
        assert val == want, f"{name}: status {val}, expected {want}"


def test_noalloc_argument_and_size_checks_come_before_any_device_call():
    """ktmoe_linear_noalloc validates its arguments and its scratch limit on the host first, so these answers hold
    on any machine: bad device or sizes -> KTMOE_ERR_ARG, missing buffers -> KTMOE_ERR_ARG, planes beyond the 64 MiB
    array -> KTMOE_ERR_UNSUPPORTED, no rows -> OK."""
    f = tb.lib().ktmoe_linear_noalloc
    one = ctypes.c_void_p(16)  # never dereferenced: every case below returns before touching memory
    assert f(-1, one, one, 4, 4, 4, one, None) == _native.ERR_ARG
    assert f(64, one, one, 4, 4, 4, one, None) == _native.ERR_ARG
    assert f(0, one, one, -1, 4, 4, one, None) == _native.ERR_ARG
    assert f(0, one, one, 4, -1, 4, one, None) == _native.ERR_ARG
    assert f(0, one, one, 4, 4, -1, one, None) == _native.ERR_ARG
    assert f(0, one, one, 4, 4, 4, None, None) == _native.ERR_ARG
    assert f(0, None, one, 4, 4, 4, one, None) == _native.ERR_ARG
    assert f(0, one, None, 4, 4, 4, one, None) == _native.ERR_ARG
    assert f(0, one, one, 0, 4, 4, one, None) == _native.OK
    # 3*4096*4096 + 3*4096*4096 bytes of planes: far above the array
    assert f(0, one, one, 4096, 4096, 4096, one, None) == _native.ERR_UNSUPPORTED
    # just above the limit: rows_pad 64, out_pad 128, k_pad = k rounded to 128; 3*k_pad*(64+128) + 256 > 64 MiB
    k = 116608
    assert 3 * k * (64 + 128) + 256 > (64 << 20)
    assert f(0, one, one, 1, 1, k, one, None) == _native.ERR_UNSUPPORTED
