"""Build the native library in-tree: nvcc -> marearts_tinydeform_b200/_tinydeform.so (sm_100a only).

The library is a plain C-ABI shared object (include/tinydeform.h) with no torch headers; Python reaches it through
ctypes (``_native.py``). It is rebuilt when any source under csrc/ or the public header is newer than the .so.

    python -m marearts_tinydeform_b200.build [--force]
"""

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, 'csrc')
HEADER = os.path.join(ROOT, 'include', 'tinydeform.h')
LIB = os.path.join(HERE, '_tinydeform.so')
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']


def _nvcc():
    for cand in (os.environ.get('NVCC'), '/usr/local/cuda/bin/nvcc'):
        if cand and os.path.exists(cand):
            return cand
    return 'nvcc'


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(('.cu', '.cuh')))


def stale():
    if not os.path.exists(LIB):
        return True
    built = os.path.getmtime(LIB)
    return any(os.path.getmtime(p) > built for p in sources() + [HEADER, __file__])


def build(force=False, verbose=False):
    """Compile csrc/tinydeform.cu into _tinydeform.so if it is missing or stale; return the library path."""
    if not force and not stale():
        return LIB
    tmp = LIB + '.tmp'
    cmd = [_nvcc(), *ARCH, '-O3', '-lineinfo', '-std=c++17', '--expt-relaxed-constexpr',
           '-Xcompiler', '-fPIC,-O3,-fvisibility=hidden', '-shared',
           '-I' + os.path.join(ROOT, 'include'), os.path.join(CSRC, 'tinydeform.cu'), '-o', tmp]
    if verbose:
        cmd.insert(1, '-Xptxas=-v')
    print(' '.join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == '__main__':
    build(force='--force' in sys.argv, verbose='-v' in sys.argv)
