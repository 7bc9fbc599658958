"""The library GEMV on unquantised GGML rows (F32 = 0, F16 = 1), which GGUF
files use for some matrices (often the output head) and the reference takes
through NumPy (engine/gguf_parser.py:180-288): y = x @ W^T with f32
accumulation, against float64, for decode-sized token counts."""
import numpy as np
import pytest
import torch

from localai_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize('t,rows,cols,tokens', [(1, 300, 4096, 1), (1, 1000, 512, 3), (0, 257, 1024, 9),
                                                 (0, 64, 8, 1), (1, 128256 // 64, 4096, 2)])
def test_dense_gemv_matches_f64(t, rows, cols, tokens):
    rng = np.random.default_rng(rows + cols + tokens)
    dt = np.float16 if t == 1 else np.float32
    W = rng.normal(0, 1, size=(rows, cols)).astype(dt)
    x = rng.normal(size=(tokens, cols)).astype(np.float32)
    w = torch.frombuffer(bytearray(W.tobytes()), dtype=torch.uint8).cuda()
    y = ops.gemv(w, torch.from_numpy(x).cuda(), t, rows, cols).cpu().numpy()
    ref = x.astype(np.float64) @ W.astype(np.float64).T
    err = np.linalg.norm(y - ref) / np.linalg.norm(ref)
    assert err < 1e-6, err
    ops.check_device_error()
