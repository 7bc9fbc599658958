"""Generate the golden dequantization fixtures from the reference engine itself.

Run once in a container that has the reference checkout:

    python tests/golden/make_golden.py --reference <path of the reference checkout>

The reference engine package is copied to a temporary directory first (its
numba kernels are ``cache=True`` and write ``__pycache__`` next to the
sources), then ``engine.dequant.dequantize`` is called on seeded block bytes:

* once with numba importable (the branch the reference takes for Q4_K/Q6_K,
  engine/dequant.py:48-60), and
* once with ``engine.numba_kernels`` made unimportable (the NumPy branch,
  engine/dequant.py:62-167).

Both outputs must agree bit-for-bit; the script asserts that and stores one.
The fixtures land in ``tests/golden/dequant_golden.npz``; the GPU box never
needs the reference checkout.
"""
from __future__ import annotations

import argparse
import importlib
import shutil
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))
from localai_b200 import synth  # noqa: E402

# (name, ggml_type, rows, cols, generator)
CASES = [
    ('q4k_bench', 12, 8, 512, 'bench'),
    ('q4k_rand', 12, 6, 768, 'rand'),
    ('q6k_bench', 14, 8, 512, 'bench'),
    ('q6k_rand', 14, 6, 768, 'rand'),
    ('q8_0_bench', 8, 8, 256, 'bench'),
    ('q8_0_rand', 8, 6, 96, 'rand'),
    ('q4_0_rand', 2, 6, 96, 'rand'),
    ('q5k_rand', 13, 6, 512, 'rand'),
    ('q4_1_rand', 3, 4, 64, 'rand'),
    ('q5_0_rand', 6, 4, 64, 'rand'),
    ('q5_1_rand', 7, 4, 64, 'rand'),
]
BYTES = {2: 18, 3: 20, 6: 22, 7: 24, 8: 34, 12: 144, 13: 176, 14: 210}
VALS = {2: 32, 3: 32, 6: 32, 7: 32, 8: 32, 12: 256, 13: 256, 14: 256}
SCALE_OFFSETS = {2: (0,), 3: (0, 2), 6: (0,), 7: (0, 2), 8: (0,), 12: (0, 2), 13: (0, 2), 14: (208,)}


def _raw(rng, t, rows, cols, style):
    if style == 'bench':
        return synth.make(rng, t, rows, cols)
    nb = (rows * cols) // VALS[t]
    blocks = rng.integers(0, 256, size=(nb, BYTES[t]), dtype=np.uint8)
    # Random fp16 scale fields, but finite: a mix of normal, subnormal, zero
    # and negative values (the bytes of an fp16 NaN/inf would make the
    # bitwise comparison depend on NaN payload propagation).
    pool = np.array([0.0, -0.0, 6e-8, 3e-5, 0.0005, 0.03125, -0.02, 1.0, 0.75], np.float16)
    for off in SCALE_OFFSETS[t]:
        vals = pool[rng.integers(0, len(pool), size=nb)]
        blocks[:, off:off + 2] = vals.view(np.uint8).reshape(nb, 2)
    return blocks.reshape(-1).tobytes()


def _load_engine(ref_root: Path, tmp: Path, with_numba: bool):
    for name in [m for m in sys.modules if m == 'engine' or m.startswith('engine.')]:
        del sys.modules[name]
    pkg = tmp / ('with_numba' if with_numba else 'numpy_only')
    if not pkg.exists():
        (pkg / 'engine').mkdir(parents=True)
        for f in ('__init__.py', 'dequant.py', 'numba_kernels.py'):
            shutil.copy(ref_root / 'engine' / f, pkg / 'engine' / f)
        if not with_numba:
            (pkg / 'engine' / 'numba_kernels.py').write_text(
                "raise ImportError('numba branch disabled for the NumPy fixture pass')\n")
    sys.path.insert(0, str(pkg))
    try:
        return importlib.import_module('engine.dequant')
    finally:
        sys.path.remove(str(pkg))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--reference', required=True, help='path of the reference checkout')
    ap.add_argument('--out', default=str(HERE / 'dequant_golden.npz'))
    args = ap.parse_args()
    rng = np.random.default_rng(20260101)
    raws = {name: _raw(rng, t, rows, cols, style) for name, t, rows, cols, style in CASES}
    store = {}
    with tempfile.TemporaryDirectory() as tmp:
        outs = {}
        for with_numba in (True, False):
            dq = _load_engine(Path(args.reference), Path(tmp), with_numba)
            for name, t, rows, cols, _ in CASES:
                outs[(name, with_numba)] = dq.dequantize(raws[name], t, (rows, cols))
    for name, t, rows, cols, _ in CASES:
        a, b = outs[(name, True)], outs[(name, False)]
        assert a.dtype == np.float32 and b.dtype == np.float32
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), f'{name}: numba != numpy branch'
        store[f'{name}__raw'] = np.frombuffer(raws[name], np.uint8)
        store[f'{name}__out'] = a
        store[f'{name}__meta'] = np.array([t, rows, cols], np.int64)
    np.savez_compressed(args.out, **store)
    print(f'wrote {args.out}: {len(CASES)} cases')


if __name__ == '__main__':
    main()
