"""DeviceGGUF: the tensors of a GGUF file resident on the device, serving the
reference's GGUFFile surface (engine/gguf_parser.py:47-367)."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import quant_oracle as o
from localai_b200.gguf import DeviceGGUF, parse_gguf

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / 'golden'


def test_upload_is_byte_exact_and_dequant_bit_exact():
    buf = (GOLD / 'tiny.gguf').read_bytes()
    _, _, tensors, _ = parse_gguf(buf)
    g = DeviceGGUF(GOLD / 'tiny.gguf', chunk_bytes=1024)          # several staging chunks per tensor
    for name, x in tensors.items():
        dev = g.raw(name).cpu().numpy().tobytes()
        assert dev == buf[x.offset:x.offset + x.nbytes], name
        if x.ggml_type in (8, 12, 14):
            np.testing.assert_array_equal(g.tensor(name), o.dequantize(dev, x.ggml_type, x.shape))
    assert g.find('nope', 'token_embd.weight') == 'token_embd.weight'
    np.testing.assert_array_equal(g.tensor_row('token_embd.weight', 4),
                                  o.dequantize(buf[tensors['token_embd.weight'].offset:
                                                   tensors['token_embd.weight'].offset + tensors['token_embd.weight'].nbytes],
                                               8, (6, 64))[4])
    np.testing.assert_array_equal(g.tensor('output_norm.weight'),
                                  np.frombuffer(buf[tensors['output_norm.weight'].offset:][:256], np.float32))


def test_matvec_matmul_match_oracle():
    buf = (GOLD / 'tiny.gguf').read_bytes()
    _, _, tensors, _ = parse_gguf(buf)
    g = DeviceGGUF(GOLD / 'tiny.gguf')
    rng = np.random.default_rng(0)
    for name in ('blk.0.ffn_gate.weight', 'blk.0.ffn_down.weight', 'token_embd.weight'):
        x = tensors[name]
        raw = buf[x.offset:x.offset + x.nbytes]
        v = rng.normal(size=x.shape[1]).astype(np.float32)
        y = g.matvec(name, v)
        assert isinstance(y, np.ndarray) and y.shape == (x.shape[0],)
        assert o.normwise_rel_err(y, o.matvec_f64(raw, x.ggml_type, x.shape[0], x.shape[1], v)) < 1e-3
        X = rng.normal(size=(5, x.shape[1])).astype(np.float32)
        Y = g.matmul(name, torch.from_numpy(X).cuda())
        assert Y.shape == (5, x.shape[0])
        assert o.normwise_rel_err(Y.cpu().numpy(), o.matmul_f64(raw, x.ggml_type, x.shape[0], x.shape[1], X)) < 1e-3


def test_gguffile_surface_details():
    """Context manager, raw_tensor (host bytes), tensor_bytes, row_chunk,
    and the reference's argument errors (engine/gguf_parser.py:147-156,
    187-197,297-307,368-378)."""
    buf = (GOLD / 'tiny.gguf').read_bytes()
    _, _, tensors, _ = parse_gguf(buf)
    name = 'blk.0.ffn_gate.weight'
    x = tensors[name]
    with DeviceGGUF(GOLD / 'tiny.gguf') as g:
        assert bytes(g.raw_tensor(name)) == buf[x.offset:x.offset + x.nbytes]
        assert g.tensor_bytes(x) == x.nbytes
        v = np.random.default_rng(1).normal(size=x.shape[1]).astype(np.float32)
        np.testing.assert_array_equal(g.matvec(name, v, row_chunk=7), g.matvec(name, v))
        with pytest.raises(ValueError, match='expected vector shape'):
            g.matvec(name, v.reshape(1, -1))
        with pytest.raises(ValueError, match='expected batch shape'):
            g.matmul(name, v)
        with pytest.raises(ValueError, match='row_chunk must be positive'):
            g.matvec(name, v, row_chunk=0)
        with pytest.raises(ValueError, match='requires a 2-D tensor'):
            g.matvec('output_norm.weight', v)
        assert g.device_tensors
    assert not g.device_tensors                        # closed on leaving the block
