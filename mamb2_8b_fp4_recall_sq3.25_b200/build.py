"""Build recipe for the in-tree C-ABI library libsq325.so (sm_100a only).

    python mamb2_8b_fp4_recall_sq3.25_b200/build.py [--force] [--verbose]

Compiles every csrc/*.cu with nvcc for `-gencode arch=compute_100a,code=sm_100a`
and links them into sq325/libsq325.so next to the Python host package, so the
shared object travels with the source tree.  Rebuilds only when a source or
header is newer than the library.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / 'csrc'
INCLUDE = HERE.parent / 'include'
OUT = HERE / 'sq325' / 'libsq325.so'
SOURCES = ['scan.cu', 'codec.cu', 'fp4.cu', 'gemm.cu', 'layer.cu', 'decode.cu', 's16.cu', 'ste.cu', 'fp4mma.cu', 'abi.cu',
           'noalloc.cu']
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']


def nvcc():
    for cand in (os.environ.get('NVCC'), shutil.which('nvcc'), '/usr/local/cuda/bin/nvcc'):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError('nvcc not found (set NVCC)')


def stale():
    if not OUT.exists():
        return True
    t = OUT.stat().st_mtime
    deps = list(CSRC.glob('*.cu')) + list(CSRC.glob('*.cuh')) + list(INCLUDE.glob('*.h')) + [Path(__file__)]
    return any(p.stat().st_mtime > t for p in deps)


def build(force=False, verbose=False, ptxas_info=False):
    if not force and not stale():
        return OUT
    objdir = HERE / '_build'
    objdir.mkdir(exist_ok=True)
    cc = nvcc()
    flags = ARCH + ['-O3', '-lineinfo', '-std=c++17', '-Xcompiler', '-fPIC', '-I', str(CSRC), '-I', str(INCLUDE),
                    '--expt-relaxed-constexpr']
    if ptxas_info:
        flags += ['-Xptxas', '-v']
    def compile_one(src):
        obj = objdir / (src + '.o')
        cmd = [cc, '-c', str(CSRC / src), '-o', str(obj)] + flags
        if verbose:
            print(' '.join(cmd), flush=True)
        return src, obj, subprocess.run(cmd, capture_output=True, text=True)

    # translation units compile independently: one nvcc process per source
    from concurrent.futures import ThreadPoolExecutor
    with ThreadPoolExecutor(max_workers=max(1, min(len(SOURCES), os.cpu_count() or 1))) as pool:
        results = list(pool.map(compile_one, SOURCES))
    objs = []
    for src, obj, r in results:
        if r.returncode != 0:
            raise RuntimeError(f'nvcc failed for {src}:\n{r.stdout}\n{r.stderr}')
        if ptxas_info and r.stderr:
            print(f'== {src}\n{r.stderr}', file=sys.stderr)
        objs.append(str(obj))
    tmp = OUT.with_suffix('.so.tmp')
    cmd = [cc, '-shared', '-o', str(tmp)] + objs + ARCH + ['-lcudart']
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f'link failed:\n{r.stdout}\n{r.stderr}')
    os.replace(tmp, OUT)
    return OUT


if __name__ == '__main__':
    ap = argparse.ArgumentParser()
    ap.add_argument('--force', action='store_true')
    ap.add_argument('--verbose', action='store_true')
    ap.add_argument('--ptxas-info', action='store_true')
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, ptxas_info=a.ptxas_info))
