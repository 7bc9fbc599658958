"""Generate tests/golden/tiny.gguf (with localai_b200.gguf.write_gguf) and
tests/golden/tiny_gguf_reference.json: what the reference's own parser
(engine/gguf_parser.py:47-178, GGUFFile) reads from that file -- version,
alignment, metadata and tensor infos (shape, type, absolute offset) -- plus
its dequantised values of every tensor (sums, as a fingerprint).

    python tests/golden/make_gguf_golden.py <reference checkout>
"""
import json
import shutil
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))


def build_file(path):
    from localai_b200 import synth
    from localai_b200.gguf import write_gguf
    rng = np.random.default_rng(9)
    meta = {'general.architecture': 'llama', 'llama.block_count': 1, 'llama.embedding_length': 256,
            'llama.rope.freq_base': 500000.0, 'general.flag': True, 'tokenizer.ggml.tokens': ['a', 'bb', 'ccc'],
            'test.ints': [1, -2, 3], 'test.big': 2 ** 40}
    tensors = {'blk.0.ffn_gate.weight': (synth.q4_k(rng, 8, 512), 12, (8, 512)),
               'blk.0.ffn_down.weight': (synth.q6_k(rng, 4, 256), 14, (4, 256)),
               'token_embd.weight': (synth.q8_0(rng, 6, 64), 8, (6, 64)),
               'output_norm.weight': (rng.normal(size=64).astype(np.float32).tobytes(), 0, (64,)),
               'half.weight': (rng.normal(size=(3, 16)).astype(np.float16).tobytes(), 1, (3, 16))}
    write_gguf(path, meta, tensors, alignment=64)


def main(ref_root):
    gg = HERE / 'tiny.gguf'
    build_file(gg)
    tmp = Path(tempfile.mkdtemp())
    shutil.copytree(Path(ref_root) / 'engine', tmp / 'engine')
    sys.path.insert(0, str(tmp))
    from engine.gguf_parser import GGUFFile                           # noqa: E402
    f = GGUFFile(gg)
    out = {'version': f.version, 'alignment': f.alignment, 'metadata': f.metadata,
           'tensors': {n: {'shape': list(x.shape), 'type': x.ggml_type, 'offset': x.offset,
                           'sum': float(np.asarray(f.tensor(n), np.float64).sum())} for n, x in f.tensors.items()}}
    f.close()
    (HERE / 'tiny_gguf_reference.json').write_text(json.dumps(out, indent=1, sort_keys=True))
    print('wrote', gg, 'and tiny_gguf_reference.json')


if __name__ == '__main__':
    if len(sys.argv) != 2:
        sys.exit('usage: make_gguf_golden.py <reference checkout>')
    main(sys.argv[1])
