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
# the checked build: every corner token re-tested against [0, N) where a kernel reads or writes its row (tests only)
DEBUG_LIB = os.path.join(HERE, '_tinydeform_debug.so')
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']


def _nvcc():
    for cand in (os.environ.get('NVCC'), '/usr/local/cuda/bin/nvcc'):
        if cand and os.path.exists(cand):
            return cand
    return 'nvcc'


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(('.cu', '.cuh')))


def stale(lib=LIB):
    if not os.path.exists(lib):
        return True
    built = os.path.getmtime(lib)
    return any(os.path.getmtime(p) > built for p in sources() + [HEADER, __file__])


def build(force=False, verbose=False, debug=False):
    """Compile csrc/tinydeform.cu into _tinydeform.so (debug: the checked _tinydeform_debug.so, -DTD_DEBUG_BOUNDS) if
    it is missing or stale; return the library path."""
    lib = DEBUG_LIB if debug else LIB
    if not force and not stale(lib):
        return lib
    tmp = lib + '.tmp'
    cmd = [_nvcc(), *ARCH, '-O3', '-lineinfo', '-std=c++17', '--expt-relaxed-constexpr',
           '-Xcompiler', '-fPIC,-O3,-fvisibility=hidden', '-shared',
           '-I' + os.path.join(ROOT, 'include'), os.path.join(CSRC, 'tinydeform.cu'), '-o', tmp]
    if debug:
        cmd.insert(1, '-DTD_DEBUG_BOUNDS')
    if verbose:
        cmd.insert(1, '-Xptxas=-v')
    print(' '.join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, lib)
    return lib


if __name__ == '__main__':
    build(force='--force' in sys.argv, verbose='-v' in sys.argv)
    if '--debug' in sys.argv:
        build(force='--force' in sys.argv, verbose='-v' in sys.argv, debug=True)
