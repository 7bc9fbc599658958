import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / 'tests' / 'golden' / 'dequant_golden.npz'


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA GPU (B200); run with -m gpu')


def golden_cases():
    z = np.load(GOLDEN)
    names = sorted({k.split('__')[0] for k in z.files})
    out = []
    for n in names:
        t, rows, cols = (int(v) for v in z[n + '__meta'])
        out.append((n, t, rows, cols, z[n + '__raw'].tobytes(), z[n + '__out']))
    return out


@pytest.fixture(scope='session')
def golden():
    return golden_cases()
