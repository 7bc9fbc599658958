"""CPU tests of the C ABI: the library loads and exports every declared symbol.

No compute call is made here (there may be no GPU); the GPU tests exercise
the same entry points.
"""
import ctypes
import subprocess

import numpy as np
import pytest

from localai_b200 import _lib, native_quant


def test_library_exports_every_header_symbol():
    names = _lib.header_functions()
    assert len(names) >= 20
    lib = _lib.load()
    for n in names:
        assert hasattr(lib, n), n
        assert n in _lib.SIGNATURES, f'{n} declared in the header but not bound'
    # and nothing bound that the header does not declare
    assert set(_lib.SIGNATURES) == set(names)


def test_reference_symbol_set_is_complete():
    """The ten symbols the reference ctypes loader binds (engine/native_quant.py:80-94)."""
    ref = {f'localai_{t}_{k}' for t in ('q8_0', 'q4_0', 'q4k', 'q5k', 'q6k') for k in ('matvec', 'matmul')}
    out = subprocess.run(['nm', '-D', '--defined-only', str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if ' T ' in line}
    assert ref <= exported
    assert all(n.startswith(('localai_', 'b200q_')) for n in exported if n.startswith(('localai', 'b200q')))


def test_status_query_without_compute():
    lib = _lib.load()
    assert lib.b200q_last_status() == 0
    assert isinstance(lib.b200q_last_error(), bytes)


def test_python_wrapper_shape_contract_needs_no_gpu():
    """Reference conventions (engine/native_quant.py:104-116): None for
    unsupported types/shapes, ValueError for byte-size mismatches -- both
    decided before any device work."""
    raw = bytes(144)
    assert native_quant.matvec(raw, np.zeros(256, np.float32), 1, 256, 99) is None
    assert native_quant.matvec(raw, np.zeros(256, np.float32), 0, 256, 12) is None
    assert native_quant.matvec(raw, np.zeros(128, np.float32), 1, 128, 12) is None
    assert native_quant.matvec(raw, np.zeros(300, np.float32), 1, 300, 12) is None
    with pytest.raises(ValueError):
        native_quant.matvec(raw + b'\0', np.zeros(256, np.float32), 1, 256, 12)
    with pytest.raises(ValueError):
        native_quant.matvec(raw, np.zeros(255, np.float32), 1, 256, 12)
    with pytest.raises(ValueError):
        native_quant.matmul(raw, np.zeros((2, 128), np.float32), 1, 256, 12)
    assert native_quant.matmul(raw, np.zeros((2, 256), np.float32), 1, 256, 5) is None
