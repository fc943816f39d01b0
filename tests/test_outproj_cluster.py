"""output_proj inside the sampler's kernel (sample_outproj_kernel: thread-block clusters of 8 CTAs that share their
queries' attention rows over distributed shared memory and split Wo's output columns), selected through
td_set_output_proj_plan. Checked against the float64 oracle projected in float64 (upstream has no output_proj; the
oracle is the reference operator's result followed by nn.Linear, the decoder's definition) and against the chained
tensor-core GEMM, over the kernel's shape conditions: 1, 2, 4 and 8 heads (8, 4, 2 and 1 queries per CTA), head rows
of 64 to 512 bytes, H * D rows of 512 bytes (wider ones chain), output widths that do not fill a CTA's columns,
query counts that leave the last cluster partly empty, bias or none, a value padding mask, and the whole layer."""

import numpy as np
import pytest
import torch

from cases import LAYER_CASES, make, make_layer, to, upcast
from marearts_tinydeform_b200 import _native, deform_attn_layer, ma_deform_attn
from oracle import deform_oracle as O

pytestmark = pytest.mark.gpu

TOL = {torch.float32: (2e-5, 1e-4), torch.float16: (3e-3, 3e-3), torch.bfloat16: (2e-2, 2e-2)}

# (name, B, Q, H, D, C, levels, P, C_out)
CASES = [
    ('rtdetr-640', 1, 300, 8, 32, 256, [(80, 80), (40, 40), (20, 20)], 4, 256),
    ('ragged last cluster', 2, 33, 8, 32, 256, [(12, 13), (6, 7)], 4, 256),
    ('4 heads, 2 queries a CTA', 3, 7, 4, 64, 128, [(10, 12), (5, 6)], 4, 96),
    ('2 heads, 256-byte rows', 2, 19, 2, 128, 64, [(9, 11)], 4, 200),
    ('1 head, 8 queries a CTA', 1, 50, 1, 256, 128, [(16, 16), (8, 8)], 2, 20),
    ('H*D = 512', 1, 40, 8, 64, 256, [(20, 20)], 4, 256),
]


def _cluster_applies(dtype, H, D, c_out):
    e = torch.tensor([], dtype=dtype).element_size()
    row = D * e
    return (8 % H == 0 and H * D * e == 512 and c_out <= 256 and row % 16 == 0 and row <= 512
            and (row // 16) & (row // 16 - 1) == 0)


def _with_plan(plan, fn):
    prev = _native.set_output_proj_plan(plan)
    try:
        return fn()
    finally:
        _native.set_output_proj_plan(prev)


def _weights(c_out, HD, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    wo = ((torch.rand(c_out, HD, generator=g) * 2 - 1) / HD ** 0.5).to(dtype)
    bo = ((torch.rand(c_out, generator=g) * 2 - 1) * 0.05).to(dtype)
    return wo, bo


@pytest.mark.parametrize('dtype', [torch.float32, torch.float16, torch.bfloat16])
def test_cluster_output_proj_against_oracle_and_chained(cuda, dtype):
    for i, (name, B, Q, H, D, C, levels, P, c_out) in enumerate(CASES):
        args = make(B, Q, H, D, C, levels, P, dtype=dtype, seed=200 + i)
        wo, bo = _weights(c_out, H * D, dtype, 300 + i)
        attn = O.ma_deform_attn_oracle(*upcast(args))
        dev = to(args, 'cuda')
        atol, rtol = TOL[dtype]
        for bias in (bo, None):
            want = torch.from_numpy(attn @ wo.double().numpy().T + (0 if bias is None else bias.double().numpy()))
            outs = {}
            for plan in (_native.OUTPROJ_CLUSTER, _native.OUTPROJ_CHAINED):
                def run():
                    with torch.inference_mode():
                        n0 = _native.launch_count()
                        y = ma_deform_attn(*dev, mode='project', output_weight=wo.cuda(),
                                           output_bias=None if bias is None else bias.cuda())
                        torch.cuda.synchronize()
                        return y, _native.launch_count() - n0
                y, launches = _with_plan(plan, run)
                # the projection and one sampler kernel with output_proj in it, or the chain of three
                cluster = plan == _native.OUTPROJ_CLUSTER and _cluster_applies(dtype, H, D, c_out)
                assert launches == (2 if cluster else 3), f'{name} {dtype} plan {plan}: {launches} launches'
                got = y.double().cpu()
                assert got.shape == (B, Q, c_out)
                err = (got - want).abs().max().item()
                assert torch.allclose(got, want, atol=atol, rtol=rtol), \
                    f'{name} {dtype} plan {plan} bias={bias is not None}: max |diff| {err:.3g}'
                outs[plan] = got
            # the two plans differ only in the order of the output projection's float32 sums
            assert torch.allclose(outs[_native.OUTPROJ_CLUSTER], outs[_native.OUTPROJ_CHAINED], atol=atol,
                                  rtol=rtol), f'{name} {dtype}: plans disagree'


def test_cluster_output_proj_with_padding_mask(cuda):
    name, B, Q, H, D, C, levels, P, c_out = CASES[1]
    N = sum(h * w for h, w in levels)
    g = torch.Generator().manual_seed(7)
    mask = torch.rand(B, N, generator=g) < 0.3
    for dtype in (torch.float32, torch.float16):
        args = make(B, Q, H, D, C, levels, P, dtype=dtype, seed=17)
        wo, bo = _weights(c_out, H * D, dtype, 18)
        up = upcast(args)
        attn = O.ma_deform_attn_oracle(*up, mask)
        want = torch.from_numpy(attn @ wo.double().numpy().T + bo.double().numpy())
        dev = to(args, 'cuda')

        def run():
            with torch.inference_mode():
                return ma_deform_attn(*dev, mode='project', value_padding_mask=mask.cuda(), output_weight=wo.cuda(),
                                      output_bias=bo.cuda()).double().cpu()
        got = _with_plan(_native.OUTPROJ_CLUSTER, run)
        atol, rtol = TOL[dtype]
        assert torch.allclose(got, want, atol=atol, rtol=rtol), f'{dtype}: {(got - want).abs().max().item():.3g}'


def test_cluster_output_proj_in_the_layer(cuda):
    """deform_attn_layer in the project order: the sampler computes the producer in its prologue and output_proj in
    its epilogue (three launches: query projection paired with the value projection where both fit one launch)."""
    for i, (name, B, Q, Cq, H, D, C, levels, P) in enumerate(LAYER_CASES[:2]):
        for dtype in (torch.float32, torch.float16, torch.bfloat16):
            args = [t.cuda() for t in make_layer(B, Q, Cq, H, D, C, levels, P, ref_dim=4, dtype=dtype, seed=400 + i)]
            wo, bo = [t.cuda() for t in _weights(256, H * D, dtype, 500 + i)]

            def run():
                with torch.inference_mode():
                    return deform_attn_layer(*args[:5], H, P, *args[5:], output_weight=wo, output_bias=bo,
                                             mode='project').double()
            a = _with_plan(_native.OUTPROJ_CLUSTER, run)
            b = _with_plan(_native.OUTPROJ_CHAINED, run)
            atol, rtol = TOL[dtype]
            assert torch.allclose(a, b, atol=atol, rtol=rtol), f'{name} {dtype}: {(a - b).abs().max().item():.3g}'


def test_cluster_output_proj_is_deterministic_and_graph_capturable(cuda):
    name, B, Q, H, D, C, levels, P, c_out = CASES[0]
    dev = to(make(B, Q, H, D, C, levels, P, dtype=torch.float16, seed=600), 'cuda')
    wo, bo = [t.cuda() for t in _weights(c_out, H * D, torch.float16, 601)]
    prev = _native.set_output_proj_plan(_native.OUTPROJ_CLUSTER)
    try:
        with torch.inference_mode():
            eager = ma_deform_attn(*dev, mode='project', output_weight=wo, output_bias=bo)
            again = ma_deform_attn(*dev, mode='project', output_weight=wo, output_bias=bo)
            assert torch.equal(eager, again)
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                ma_deform_attn(*dev, mode='project', output_weight=wo, output_bias=bo)
            torch.cuda.current_stream().wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                out = ma_deform_attn(*dev, mode='project', output_weight=wo, output_bias=bo)
            for _ in range(3):
                graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(out, eager)
    finally:
        _native.set_output_proj_plan(prev)
    assert _native.device_error() == 0


def test_output_proj_plan_rejects_unknown_codes(cuda):
    with pytest.raises(ValueError):
        _native.set_output_proj_plan(7)
    assert _native.set_output_proj_plan(_native.OUTPROJ_AUTO) in (0, 1, 2)


def test_auto_with_output_proj_prefers_the_epilogue_at_batch_one(cuda):
    """'auto' with output_proj: at batch 1, where the project order folds output_proj into the sampler's epilogue,
    it runs the project order (bit for bit); at batch 2 it keeps the operator's own pick."""
    from marearts_tinydeform_b200 import choose_mode
    for B, expect_project in ((1, True), (2, False)):
        dev = to(make(B, 100, 8, 32, 256, [(20, 20), (10, 10)], 4, dtype=torch.float16, seed=70 + B), 'cuda')
        wo, bo = [t.cuda() for t in _weights(256, 256, torch.float16, 71)]
        with torch.inference_mode():
            auto = ma_deform_attn(*dev, mode='auto', output_weight=wo, output_bias=bo)
            want_mode = 'project' if expect_project else choose_mode(dev[0], dev[1], dev[5])
            want = ma_deform_attn(*dev, mode=want_mode, output_weight=wo, output_bias=bo)
        assert torch.equal(auto, want), f'B={B}: auto is not {want_mode}'
