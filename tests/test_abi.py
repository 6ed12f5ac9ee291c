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
