"""Build libb200quant.so (CUDA, sm_100a) in-tree with nvcc.

    python -m localai_b200.build [--verbose] [--ptxas]

Every ``csrc/*.cu`` is compiled to ``_build/<name>.o`` (in parallel, only when
the source or a header is newer) and linked into
``localai_b200/libb200quant.so``.  The CUDA runtime is linked statically, so
the library does not depend on the runtime version that PyTorch ships.
nvcc cross-compiles, so this works on a machine without a GPU.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / 'csrc'
BUILD = PKG / '_build'
LIB = PKG / 'libb200quant.so'
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
FLAGS = ['-O3', '-std=c++17', '-lineinfo', '--expt-relaxed-constexpr',
         '-Xcompiler', '-fPIC', '-Xcompiler', '-fvisibility=hidden',
         '-I', str(ROOT / 'include'), '-I', str(CSRC)]


def nvcc() -> str:
    exe = shutil.which('nvcc') or '/usr/local/cuda/bin/nvcc'
    if not Path(exe).exists():
        raise RuntimeError('nvcc not found; the CUDA toolkit is required to build libb200quant.so')
    return exe


def _headers():
    return list(CSRC.glob('*.cuh')) + list((ROOT / 'include').glob('*.h'))


def _stale(src: Path, obj: Path) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *_headers(), Path(__file__)])


def _compile(src: Path, ptxas: bool) -> tuple[Path, str]:
    obj = BUILD / (src.stem + '.o')
    cmd = [nvcc(), *ARCH, *FLAGS, '-c', str(src), '-o', str(obj)]
    if ptxas:
        cmd.insert(1, '-Xptxas=-v')
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f'nvcc failed for {src.name}:\n{res.stderr[-6000:]}')
    return obj, res.stderr


def build(verbose: bool = False, ptxas: bool = False, force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob('*.cu'))
    todo = [s for s in sources if force or ptxas or _stale(s, BUILD / (s.stem + '.o'))]
    logs = []
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(len(todo), os.cpu_count() or 4)) as ex:
            for obj, log in ex.map(lambda s: _compile(s, ptxas), todo):
                logs.append((obj.name, log))
                if verbose:
                    print(f'compiled {obj.name}', file=sys.stderr)
    objs = [BUILD / (s.stem + '.o') for s in sources]
    if todo or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cmd = [nvcc(), *ARCH, '-shared', '-o', str(LIB), *map(str, objs), '-lcuda']
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f'link failed:\n{res.stderr[-4000:]}')
        if verbose:
            print(f'linked {LIB}', file=sys.stderr)
    if ptxas:
        (BUILD / 'ptxas.log').write_text('\n'.join(f'== {n}\n{l}' for n, l in logs))
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--verbose', action='store_true')
    ap.add_argument('--ptxas', action='store_true', help='rebuild with -Xptxas=-v, log to _build/ptxas.log')
    ap.add_argument('--force', action='store_true')
    a = ap.parse_args()
    print(build(verbose=a.verbose, ptxas=a.ptxas, force=a.force))


if __name__ == '__main__':
    main()
