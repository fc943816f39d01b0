import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, 'tests')):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA GPU (B200, sm_100a) and the built native library')


@pytest.fixture(scope='session')
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip('no CUDA device')
    from marearts_tinydeform_b200 import _native
    _native.load()  # a GPU run must have the native library: fail loudly, never fall back
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    return torch.device('cuda')


@pytest.fixture(params=['tensor-cores', 'cuda-cores'])
def policy(request, cuda):
    """Run a test once with the default kernels (tcgen05 where shapes allow) and once on CUDA cores only."""
    from marearts_tinydeform_b200 import _native
    code = _native.POLICY_BEST if request.param == 'tensor-cores' else _native.POLICY_CUDA_CORES
    prev = _native.set_kernel_policy(code)
    yield request.param
    _native.set_kernel_policy(prev)
