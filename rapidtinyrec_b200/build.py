"""Build the native engine: ``csrc/*.cu`` -> ``librtr_b200.so`` for sm_100a.

``python -m rapidtinyrec_b200.build`` (or ``__graft_entry__.build()``) compiles
each translation unit with nvcc in parallel and links one shared library next
to this file.  nvcc cross-compiles, so no GPU is needed.  Objects are rebuilt
only when a source or header is newer than the library.
"""
from __future__ import annotations

import concurrent.futures
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / 'csrc'
INCLUDE = HERE.parent / 'include'
LIB = HERE / 'librtr_b200.so'
BUILD_DIR = HERE.parent / '_build'

ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
NVCC_FLAGS = ['-O3', '-lineinfo', '-std=c++17', '-Xcompiler', '-fPIC', '--expt-relaxed-constexpr',
              '-Xptxas', '-warn-spills', f'-I{INCLUDE}', f'-I{CSRC}']


def nvcc() -> str:
    for cand in (os.environ.get('NVCC'), '/usr/local/cuda/bin/nvcc', 'nvcc'):
        if cand and (Path(cand).exists() or cand == 'nvcc'):
            return cand
    raise RuntimeError('nvcc not found')


def sources():
    return sorted(CSRC.glob('*.cu'))


def _stale() -> bool:
    if not LIB.exists():
        return True
    newest = max(p.stat().st_mtime for p in list(CSRC.iterdir()) + list(INCLUDE.iterdir()) + [Path(__file__)])
    return newest > LIB.stat().st_mtime


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        return LIB
    BUILD_DIR.mkdir(exist_ok=True)
    cc = nvcc()

    def compile_one(src: Path) -> Path:
        obj = BUILD_DIR / (src.stem + '.o')
        cmd = [cc, *ARCH, *NVCC_FLAGS, '-c', str(src), '-o', str(obj)]
        if verbose:
            print(' '.join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f'nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}')
        if verbose and (res.stdout or res.stderr):
            print(res.stdout + res.stderr, flush=True)
        return obj

    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as pool:
        objs = list(pool.map(compile_one, sources()))
    tmp = LIB.with_suffix('.so.tmp')
    cmd = [cc, *ARCH, '-shared', '-o', str(tmp), *map(str, objs), '-lcudart']
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f'link failed:\n{res.stdout}\n{res.stderr}')
    tmp.replace(LIB)
    return LIB


if __name__ == '__main__':
    print(build(force='--force' in sys.argv, verbose='-v' in sys.argv))
