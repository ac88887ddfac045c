"""The C-ABI library loads and exports every symbol the public header declares
(no compute calls: this runs without a GPU)."""

import os
import re

from tabpack_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    text = open(os.path.join(ROOT, 'include', 'tabpack_b200.h')).read()
    text = re.sub(r'/\*.*?\*/', '', text, flags=re.S)
    return sorted(set(re.findall(r'\b(tp_\w+)\s*\(', text)))


def test_header_symbols_exported_and_bound():
    lib = _lib.load()
    names = declared_functions()
    assert names, 'no declarations found'
    for n in names:
        assert hasattr(lib, n), f'{n} is declared but not exported'
        assert n in _lib.SIGNATURES, f'{n} has no ctypes binding'
    assert set(_lib.SIGNATURES) == set(names)


def test_version_without_gpu():
    assert _lib.load().tp_version().decode().startswith('tabpack_b200')
