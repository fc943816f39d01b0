"""The drop-in API on CPU: names, the CPU route to the reference, the auto picker and its per-GPU tables."""

import pytest
import torch

import marearts_tinydeform
import marearts_tinydeform_b200 as td
from cases import make
from marearts_tinydeform_b200 import choose_mode, ma_deform_attn, ma_deform_attn_reference


def test_upstream_import_name_serves_this_package():
    for name in ('ma_deform_attn_reference', 'choose_mode', 'FUSED_LIMIT', 'FUSED_LIMIT_SM75', '_limits', 'MODES',
                 '__version__'):
        assert getattr(marearts_tinydeform, name) is getattr(td, name)
    assert td.MODES == ('auto', 'fused', 'project')
    assert marearts_tinydeform.__all__ == ['ma_deform_attn', 'ma_deform_attn_reference', 'choose_mode']
    # upstream's signature exactly (the B200 package's own ma_deform_attn adds keyword arguments)
    import inspect
    assert list(inspect.signature(marearts_tinydeform.ma_deform_attn).parameters) == [
        'memory', 'value_weight', 'value_bias', 'spatial_shapes', 'level_start_index', 'sampling_locations',
        'attention_weights', 'mode']


def test_upstream_import_name_keeps_the_cpu_route_and_mode_check():
    """Upstream order: the mode is checked first, then CPU tensors go to the reference -- with grad too, since the
    inference-only rule guards the CUDA path only."""
    args = make(1, 10, 2, 8, 16, [(6, 7), (3, 4)], 2)
    with pytest.raises(ValueError):
        marearts_tinydeform.ma_deform_attn(*args, mode='nope')
    with torch.inference_mode():
        assert torch.equal(marearts_tinydeform.ma_deform_attn(*args), ma_deform_attn_reference(*args))
    grad = [t.clone().requires_grad_(True) if i == 0 else t for i, t in enumerate(args)]
    marearts_tinydeform.ma_deform_attn(*grad).sum().backward()
    assert grad[0].grad is not None


def test_cpu_path_is_reference():
    args = make(1, 10, 2, 8, 16, [(6, 7), (3, 4)], 2)
    with torch.inference_mode():
        assert torch.equal(ma_deform_attn(*args), ma_deform_attn_reference(*args))
        for mode in td.MODES:
            assert torch.equal(ma_deform_attn(*args, mode=mode), ma_deform_attn_reference(*args))


def test_value_padding_mask_on_the_cpu_route():
    """The mask zeroes padded tokens' projected value (Deformable-DETR's input_padding_mask): on CPU the reference
    applies it; with no bias that equals zeroing those memory rows; an all-False mask changes nothing."""
    args = make(2, 9, 2, 8, 16, [(6, 7), (3, 4)], 2, bias=False, seed=4)
    N = args[0].shape[1]
    mask = torch.rand(2, N, generator=torch.Generator().manual_seed(1)) < 0.4
    zeroed = list(args)
    zeroed[0] = args[0].masked_fill(mask[..., None], 0)
    with torch.inference_mode():
        got = ma_deform_attn(*args, value_padding_mask=mask)
        torch.testing.assert_close(got, ma_deform_attn_reference(*zeroed), atol=1e-6, rtol=1e-5)
        none = torch.zeros_like(mask)
        assert torch.equal(ma_deform_attn(*args, value_padding_mask=none), ma_deform_attn(*args))
        full = torch.ones_like(mask)
        assert ma_deform_attn(*args, value_padding_mask=full).abs().max().item() == 0.0


def test_output_proj_on_the_cpu_route():
    args = make(1, 10, 2, 8, 16, [(6, 7), (3, 4)], 2)
    wo = torch.randn(12, 16, generator=torch.Generator().manual_seed(2)) * 0.1
    bo = torch.randn(12, generator=torch.Generator().manual_seed(3)) * 0.1
    with torch.inference_mode():
        got = ma_deform_attn(*args, output_weight=wo, output_bias=bo)
        assert torch.equal(got, torch.nn.functional.linear(ma_deform_attn_reference(*args), wo, bo))
    with pytest.raises(ValueError):
        ma_deform_attn(*args, output_bias=bo)


def test_bad_mode_is_a_value_error():
    args = make(1, 4, 2, 8, 16, [(6, 7)], 2)
    with pytest.raises(ValueError):
        ma_deform_attn(*args, mode='nope')


def test_reference_supports_autograd():
    args = make(1, 6, 2, 8, 16, [(6, 7), (3, 4)], 2)
    args[0].requires_grad_(True)
    args[1].requires_grad_(True)
    ma_deform_attn_reference(*args).square().sum().backward()
    assert args[0].grad is not None and args[1].grad is not None


def test_auto_picks_fused_for_few_queries():
    few = make(1, 50, 8, 32, 256, [(80, 80), (40, 40), (20, 20)], 4)
    many = make(8, 900, 8, 32, 256, [(80, 80), (40, 40), (20, 20)], 4)
    assert choose_mode(few[0], few[1], few[5]) == 'fused'
    assert choose_mode(many[0], many[1], many[5]) == 'project'


def test_auto_limits_follow_the_gpu_generation():
    get = torch.cuda.get_device_capability
    try:
        for cap, table in (((8, 9), td.FUSED_LIMIT), ((7, 5), td.FUSED_LIMIT_SM75), ((10, 0), td.FUSED_LIMIT_SM100),
                           ((9, 0), td.FUSED_LIMIT)):
            torch.cuda.get_device_capability = lambda device=None, cap=cap: cap
            assert td._limits.__wrapped__(0) is table
    finally:
        torch.cuda.get_device_capability = get


def test_auto_tables_cover_every_dtype():
    for table in (td.FUSED_LIMIT, td.FUSED_LIMIT_SM75, td.FUSED_LIMIT_SM100):
        for dtype in (torch.float32, torch.float16, torch.bfloat16):
            a, b = table[dtype]
            assert a > 0 and a + b > -0.1  # b may be negative on B200: the limit grows with the batch


def test_tensor_contract_rejects_cpu_tensors_in_the_native_path():
    from marearts_tinydeform_b200 import _native
    args = make(1, 4, 2, 8, 16, [(6, 7)], 2)
    with pytest.raises(RuntimeError, match='CUDA'):
        _native.check_geometry(args[0], args[3], args[4], args[5], args[6])


def test_b200_table_picks_the_measured_faster_order(monkeypatch):
    """The sm_100 table on the BASELINE shapes and the sweep's crossovers: 16-bit types take the fused order at 50-100
    queries (c2: RT-DETR, batch 1, 100 queries) and the project order from 200 queries on (c1h, c3, c4); float32
    takes the fused order up to 300 queries at every batch and the project order from 600."""
    from marearts_tinydeform_b200 import workloads
    monkeypatch.setattr(td, '_limits', lambda device_index: td.FUSED_LIMIT_SM100)

    class FakeCuda:  # choose_mode only reads .is_cuda, .get_device(), .shape and .dtype
        def __init__(self, t):
            self.shape, self.dtype, self.is_cuda = t.shape, t.dtype, True

        def get_device(self):
            return 0

    def pick(name, **kw):
        a = workloads.make_inputs(name, seed=0, **kw)
        return choose_mode(FakeCuda(a[0]), a[1], a[5])

    assert pick('c1h') == 'project'
    assert pick('c2') == 'fused'
    assert pick('c3') == 'project'
    assert pick('c4') == 'project'
    assert pick('c1h', B=8, Q=50) == 'fused'
    assert pick('c1h', Q=200) == 'project'
    assert pick('c3', Q=50) == 'fused'
    assert pick('c5', B=4, Q=50) == 'project'
    assert pick('c5', B=64, Q=50) == 'fused'
    assert pick('c1', Q=300) == 'fused'
    assert pick('c1', Q=600) == 'project'
    assert pick('c1', B=8, Q=100) == 'fused'
    assert pick('c1', B=4, Q=300) == 'fused'
    assert pick('c5', dtype=torch.float32, B=1, Q=300) == 'project'
