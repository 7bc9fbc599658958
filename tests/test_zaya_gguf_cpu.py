"""CPU checks of the ZAYA GGUF fixture (tests/golden/zaya_gguf_golden.npz,
made by running the reference's ZayaModel._moe through its own GGUFFile on a
seeded one-layer file): the file rebuilds byte for byte, and the oracle's
router chain and expert FFN, given the file's tensors, reproduce the
reference's routes, router states and outputs."""
import hashlib
import importlib.util
from pathlib import Path

import numpy as np

from oracle import quant_oracle as o
from localai_b200.gguf import parse_gguf

GOLD = Path(__file__).resolve().parent / 'golden'


def fixture_module():
    spec = importlib.util.spec_from_file_location('make_zaya_gguf_golden', GOLD / 'make_zaya_gguf_golden.py')
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_zaya_fixture_rebuilds_and_oracle_matches_reference(tmp_path):
    mod = fixture_module()
    gold = np.load(GOLD / 'zaya_gguf_golden.npz')
    path = tmp_path / 'zaya.gguf'
    mod.build_file(path)
    buf = path.read_bytes()
    assert hashlib.sha256(buf).hexdigest() == str(gold['sha256'])
    _, _, tensors, _ = parse_gguf(buf)
    p = f'blk.{mod.LAYER}.'

    def raw(name):
        x = tensors[p + name]
        return buf[x.offset:x.offset + x.nbytes]

    def f32(name):
        return np.frombuffer(raw(name), np.float32).reshape(tensors[p + name].shape)

    H, P = gold['H'], gold['P'].copy()
    P[::3] = 0.0                               # tokens the reference ran without a previous router state
    e, w, _, state = o.zaya_router_f32(
        H, f32('ffn_gate_inp.weight'), f32('ffn_gate.weight'), f32('zaya_router_mlp2.weight'),
        f32('zaya_router_mlp4.weight'), f32('ffn_norm.weight'), f32('zaya_router_biases.weight'), 1e-5, prev=P,
        w_eda=f32('zaya_router_eda.weight'), b_in=f32('ffn_gate_inp.bias'), b_gate=f32('ffn_gate.bias'),
        b_mlp2=f32('zaya_router_mlp2.bias'))
    assert np.array_equal(e, gold['route'])
    assert o.normwise_rel_err(state, gold['S']) < 1e-6
    gu, dn = raw('ffn_gate_up_exps.weight'), raw('ffn_down_exps.weight')
    n_gu, n_dn = len(gu) // mod.E, len(dn) // mod.E
    experts = [(gu[i * n_gu:(i + 1) * n_gu], dn[i * n_dn:(i + 1) * n_dn]) for i in range(mod.E)]
    y = o.zaya_moe_f64(H, e, w, experts, 12, 14, mod.D, mod.F, mod.F)
    assert o.normwise_rel_err(y, gold['Y']) < 1e-5
