"""GGUF parsing and writing (CPU).  The parser is pinned to the reference's
own parser (engine/gguf_parser.py:47-178) through the committed fixture
tests/golden/tiny.gguf and what that parser read from it
(tests/golden/tiny_gguf_reference.json)."""
import json
import struct
from pathlib import Path

import numpy as np
import pytest

from oracle import quant_oracle as o
from localai_b200.gguf import parse_gguf, write_gguf

GOLD = Path(__file__).resolve().parent / 'golden'


def test_parse_matches_reference_parser():
    buf = (GOLD / 'tiny.gguf').read_bytes()
    ref = json.loads((GOLD / 'tiny_gguf_reference.json').read_text())
    version, meta, tensors, align = parse_gguf(buf)
    assert version == ref['version'] and align == ref['alignment']
    assert meta == ref['metadata']
    assert set(tensors) == set(ref['tensors'])
    for name, r in ref['tensors'].items():
        x = tensors[name]
        assert list(x.shape) == r['shape'] and x.ggml_type == r['type'] and x.offset == r['offset']
        raw = buf[x.offset:x.offset + x.nbytes]
        if x.ggml_type == 0:
            vals = np.frombuffer(raw, np.float32)
        elif x.ggml_type == 1:
            vals = np.frombuffer(raw, np.float16).astype(np.float32)
        else:
            vals = o.dequantize(raw, x.ggml_type, x.shape)
        assert np.isclose(np.asarray(vals, np.float64).sum(), r['sum'], rtol=1e-6, atol=1e-6)


def test_write_parse_round_trip(tmp_path):
    rng = np.random.default_rng(1)
    raw = rng.integers(0, 256, size=34 * 8, dtype=np.uint8).tobytes()
    meta = {'a.u': 7, 'a.neg': -3, 'a.f': 0.5, 'a.s': 'héllo', 'a.b': False, 'a.list': [1.0, 2.0], 'a.big': -2 ** 40}
    p = tmp_path / 'x.gguf'
    write_gguf(p, meta, {'w': (raw, 8, (2, 128)), 'v': (np.ones(5, np.float32).tobytes(), 0, (5,))})
    version, m, t, align = parse_gguf(p.read_bytes())
    assert version == 3 and align == 32 and m == meta
    assert t['w'].shape == (2, 128) and t['w'].ggml_type == 8 and t['w'].nbytes == len(raw)
    b = p.read_bytes()
    assert b[t['w'].offset:t['w'].offset + len(raw)] == raw
    assert t['w'].offset % 32 == 0 and t['v'].offset % 32 == 0


@pytest.mark.parametrize('mutate,msg', [
    (lambda b: b'GGUX' + b[4:], 'not a GGUF'),
    (lambda b: b[:4] + struct.pack('<I', 7) + b[8:], 'version'),
    (lambda b: b[:40], 'truncated'),
])
def test_rejects_malformed(mutate, msg):
    buf = (GOLD / 'tiny.gguf').read_bytes()
    with pytest.raises(ValueError, match=msg):
        parse_gguf(mutate(buf))


def test_rejects_tensor_past_end():
    buf = (GOLD / 'tiny.gguf').read_bytes()
    with pytest.raises(ValueError, match='past the end'):
        parse_gguf(buf[:-100])


def test_find_exact_names_before_suffix_matches():
    """DeviceGGUF.find follows engine/gguf_parser.py:368-376: every exact name
    first, then suffix matches on '.' + name in the order the names are given;
    'output.weight' never picks 'blk.N.attn_output.weight'."""
    from localai_b200.gguf import DeviceGGUF, tensor_nbytes
    g = DeviceGGUF.__new__(DeviceGGUF)          # the lookup needs only the tensor table
    g.tensors = dict.fromkeys(['blk.0.attn_output.weight', 'model.norm.weight', 'token_embd.weight',
                               'model.embed.output.weight'])
    assert g.find('output.weight') == 'model.embed.output.weight'
    assert g.find('output_norm.weight', 'norm.weight') == 'model.norm.weight'
    assert g.find('tok_embeddings.weight', 'token_embd.weight') == 'token_embd.weight'
    assert g.find('missing.weight') is None
    g.tensors = dict.fromkeys(['blk.0.attn_output.weight'])
    assert g.find('output.weight') is None

    class Info:
        ggml_type, shape = 12, (16, 512)
    assert DeviceGGUF.tensor_bytes(g, Info) == tensor_nbytes(12, (16, 512)) == 16 * 2 * 144
