"""Parity of the backward pass on the GPU (td_sample_backward through the C ABI, and ma_deform_attn under
autograd): the golden gradients written by autograd through upstream's own reference, the float64 oracle at full
BASELINE-config size, torch.autograd.gradcheck in float64, torch's own grid_sample backward on the GPU, the value
padding mask, output_proj and the whole layer under autograd, and the inputs' gradient flags."""

import numpy as np
import pytest
import torch

from cases import LAYER_CASES, make, make_layer, to
from marearts_tinydeform_b200 import (_native, deform_attn_layer, deform_attn_layer_reference, ma_deform_attn,
                                      ma_deform_attn_reference)
from oracle import deform_oracle as O
from test_backward_cpu import GRAD_CASES

pytestmark = pytest.mark.gpu

# relative to the largest magnitude of each gradient: fp32 / fp64 accumulate in float32 / float64 (atomics), fp16 and
# bf16 recompute value in the dtype and round the small gradients to it once
GRAD_TOL = {torch.float32: 1e-4, torch.float16: 6e-3, torch.bfloat16: 4e-2, torch.float64: 1e-10}
ORDER = ('memory', 'value_weight', 'value_bias', None, None, 'sampling_locations', 'attention_weights')


def run_grads(inputs, grad_out, mask=None, mode='project'):
    """Gradients of ma_deform_attn on CUDA for the float inputs (all of them require grad)."""
    x = [t if t is None or t.dtype == torch.long else t.detach().cuda().requires_grad_(True) for t in inputs]
    x = [t.cuda() if t is not None and t.dtype == torch.long else t for t in x]
    out = ma_deform_attn(*x, mode=mode, value_padding_mask=None if mask is None else mask.cuda())
    out.backward(grad_out.to(out.dtype).cuda())
    return {name: x[i].grad.double().cpu().numpy() for i, name in enumerate(ORDER)
            if name is not None and x[i] is not None}


def kinks(loc, shapes):
    """bool [B, Q, H, L, P, 2]: points whose pixel coordinate x = loc * w - 0.5 (or y) is within 1e-4 of an integer.
    The location gradient jumps there (the bilinear weights are piecewise linear), so arithmetic in another precision
    or order may take the other side; the boundary-location case puts points exactly on pixel centres on purpose,
    and random float32 locations land that close now and then. Location gradients are compared off these points."""
    loc = loc.double().numpy()
    out = np.zeros(loc.shape, dtype=bool)
    for lvl, (h, w) in enumerate(shapes.tolist()):
        for k, size in ((0, w), (1, h)):
            x = loc[:, :, :, lvl, :, k] * size - 0.5
            near = np.abs(x - np.round(x)) < 1e-4
            out[:, :, :, lvl, :, 0] |= near
            out[:, :, :, lvl, :, 1] |= near
    return out


def close(got, want, tol, what):
    scale = max(1.0, float(np.abs(want).max()))
    err = float(np.abs(got - want).max())
    assert err <= tol * scale, f'{what}: max |diff| {err:.3g} (max |want| {scale:.3g})'


@pytest.mark.parametrize('case', GRAD_CASES, ids=[c[0] for c in GRAD_CASES])
def test_golden_gradients(cuda, case):
    key, dtype, inputs, mask, grad_out, want = case
    kink = kinks(inputs[5], inputs[3])
    for mode in ('project', 'fused'):
        got = run_grads(inputs, grad_out, mask, mode)
        for name, w in want.items():
            g = got[name]
            if name == 'sampling_locations':  # compared off the kinks only
                g, w = np.where(kink, 0.0, g), np.where(kink, 0.0, w)
            close(g, w, GRAD_TOL[dtype], f'{key} [{mode}] grad {name}')


@pytest.mark.parametrize('dtype', [torch.float32, torch.float16, torch.bfloat16])
def test_full_size_against_oracle(cuda, dtype):
    """BASELINE c1h geometry (B=1, Q=300, 80x80 + 40x40 + 20x20, H=8, D=32, C=256) against the float64 oracle on
    the upcast inputs, plus a value padding mask."""
    args = make(1, 300, 8, 32, 256, [(80, 80), (40, 40), (20, 20)], 4, dtype=dtype, seed=5)
    g = torch.randn(1, 300, 256, generator=torch.Generator().manual_seed(6), dtype=torch.float64)
    mask = torch.rand(1, args[0].shape[1], generator=torch.Generator().manual_seed(7)) < 0.2
    up = [t if t is None or t.dtype == torch.long else t.double() for t in args]
    kink = kinks(args[5], args[3])
    for m in (None, mask):
        want = O.ma_deform_attn_backward_oracle(*up, g, m)
        got = run_grads(args, g, m)
        want['sampling_locations'] = np.where(kink, 0.0, want['sampling_locations'])
        got['sampling_locations'] = np.where(kink, 0.0, got['sampling_locations'])
        for name in ('memory', 'value_weight', 'value_bias', 'sampling_locations', 'attention_weights'):
            close(got[name], want[name], GRAD_TOL[dtype], f'c1h {dtype} mask={m is not None} grad {name}')


def test_gradcheck_float64(cuda):
    args = to(make(1, 5, 2, 4, 8, [(5, 6), (3, 3)], 3, dtype=torch.float64, seed=11), cuda)
    x = [t.clone().requires_grad_(True) if t is not None and t.dtype == torch.float64 else t for t in args]
    for mode in ('project', 'fused'):
        assert torch.autograd.gradcheck(lambda *a: ma_deform_attn(*a, mode=mode), tuple(x), eps=1e-6, atol=1e-7,
                                        rtol=1e-5, nondet_tol=1e-10)


def test_matches_torch_grid_sample_backward(cuda):
    """float32 on the GPU: our gradients against autograd through ma_deform_attn_reference (grid_sample) on the same
    device (TF32 off for torch's GEMMs)."""
    for B, Q, H, D, C, levels, P in ((2, 100, 8, 32, 256, [(50, 76), (25, 38), (13, 19), (7, 10)], 4),
                                     (1, 64, 2, 64, 128, [(20, 30)], 16),
                                     (2, 33, 3, 10, 30, [(13, 17), (7, 9)], 4)):
        args = to(make(B, Q, H, D, C, levels, P, seed=Q), cuda)
        g = torch.randn(B, Q, H * D, device=cuda)
        xs, xr = [], []
        for t in args:
            if t is not None and t.dtype == torch.float32:
                xs.append(t.clone().requires_grad_(True))
                xr.append(t.clone().requires_grad_(True))
            else:
                xs.append(t)
                xr.append(t)
        ma_deform_attn(*xs).backward(g)
        ma_deform_attn_reference(*xr).backward(g)
        kink = kinks(args[5].cpu(), args[3].cpu())
        for i, name in enumerate(ORDER):
            if name is None or xs[i] is None:
                continue
            a, b = xs[i].grad.double().cpu().numpy(), xr[i].grad.double().cpu().numpy()
            if name == 'sampling_locations':
                a, b = np.where(kink, 0.0, a), np.where(kink, 0.0, b)
            close(a, b, 1e-4, f'{Q} {name}')


def test_backward_kernel_alone_and_mask(cuda):
    """td_sample_backward on a head-major value: grad_value zero on padded tokens, and the vector and generic
    kernels (D * 2 bytes not a power-of-two number of 16-byte words takes the generic one) against the oracle."""
    for D, dtype in ((32, torch.float16), (24, torch.float16), (12, torch.float32), (10, torch.float64)):
        B, Q, H, levels, P = 2, 9, 3, [(7, 8), (4, 4)], 4
        args = make(B, Q, H, D, 4 * D, levels, P, dtype=dtype, seed=D)
        N = args[0].shape[1]
        mask = torch.rand(B, N, generator=torch.Generator().manual_seed(D)) < 0.3
        value = torch.randn(B, N, H * D, dtype=torch.float64)
        g = torch.randn(B, Q, H * D, dtype=torch.float64)
        v_hm = value.view(B, N, H, D).permute(0, 2, 1, 3).contiguous().to(dtype)
        with torch.inference_mode():
            gv, gl, ga = _native.sample_backward(v_hm.cuda(), args[3].cuda(), args[4].cuda(), args[5].cuda(),
                                                 args[6].cuda(), g.to(dtype).cuda(), mask.cuda())
        vz = np.where(mask.numpy()[..., None], 0.0, v_hm.double().permute(0, 2, 1, 3).reshape(B, N, H * D).numpy())
        want_v, want_l, want_a = O.sample_backward(vz, H, args[3], args[4], args[5].double(), args[6].double(),
                                                   g.to(dtype).double())
        want_v = np.where(mask.numpy()[..., None], 0.0, want_v)
        tol = GRAD_TOL[dtype]
        kink = kinks(args[5], args[3])
        close(gv.double().cpu().numpy(), want_v, tol, f'D={D} {dtype} grad_value')
        close(np.where(kink, 0.0, gl.double().cpu().numpy()), np.where(kink, 0.0, want_l), tol,
              f'D={D} {dtype} grad_loc')
        close(ga.double().cpu().numpy(), want_a, tol, f'D={D} {dtype} grad_attn')
        assert float(gv[mask.cuda()].abs().max()) == 0.0


def test_output_proj_and_layer_under_autograd(cuda):
    """output_proj (torch nn.Linear behind the differentiable operator) and the whole layer (producer in torch
    operators, then the operator) against the all-torch layer's autograd on the GPU, float32."""
    name, B, Q, Cq, H, D, C, levels, P = LAYER_CASES[2]
    args = make_layer(B, Q, Cq, H, D, C, levels, P, ref_dim=4, dtype=torch.float32, seed=81)
    wo = torch.randn(48, H * D) / (H * D) ** 0.5
    bo = torch.randn(48) * 0.1
    mask = torch.rand(B, args[2].shape[1], generator=torch.Generator().manual_seed(3)) < 0.25
    grads = []
    for fn in (deform_attn_layer, deform_attn_layer_reference):
        x = [t.cuda().requires_grad_(True) if t is not None and t.is_floating_point() else
             (t.cuda() if t is not None else None) for t in args]
        o_w, o_b = wo.cuda().requires_grad_(True), bo.cuda().requires_grad_(True)
        out = fn(*x[:5], H, P, *x[5:], output_weight=o_w, output_bias=o_b, value_padding_mask=mask.cuda())
        out.square().sum().backward()
        grads.append([t.grad.double().cpu().numpy() for t in x + [o_w, o_b] if t is not None and t.requires_grad])
    for k, (a, b) in enumerate(zip(*grads)):
        close(a, b, 2e-4, f'layer input {k}')


def test_only_requested_gradients_and_no_grad_path(cuda):
    args = to(make(1, 12, 2, 8, 16, [(6, 7), (3, 4)], 2, seed=2), cuda)
    loc = args[5].clone().requires_grad_(True)
    out = ma_deform_attn(*args[:5], loc, args[6])
    assert out.requires_grad
    out.sum().backward()
    assert loc.grad is not None and loc.grad.shape == loc.shape
    with torch.no_grad():
        assert not ma_deform_attn(*args[:5], loc, args[6]).requires_grad


def test_grad_value_finish(cuda):
    """td_grad_value_finish: the rounding to the dtype and the column sums of a float32 accumulator, for widths that
    fill the 256-thread CTA exactly (HD = 256) and not (HD = 80, 1024), against torch."""
    g = torch.Generator(device=cuda).manual_seed(4)
    for rows, HD in ((67200, 256), (999, 80), (130, 1024), (0, 256)):
        acc = torch.randn(rows, HD, generator=g, device=cuda)
        for dtype in (torch.float16, torch.bfloat16, torch.float32):
            out, bias = _native.grad_value_finish(acc, dtype, True)
            assert torch.equal(out, acc.to(dtype)), f'{rows}x{HD} {dtype}'
            want = acc.double().sum(0)
            assert torch.allclose(bias.double(), want, atol=1e-3 * max(1.0, rows ** 0.5), rtol=1e-5), \
                f'{rows}x{HD} {dtype}: bias'
    assert _native.grad_value_finish(torch.zeros(4, 6, device=cuda), torch.float16, True) is None


LINEAR_GRAD_TOL = {torch.float16: 2e-3, torch.bfloat16: 1e-2, torch.float32: 2e-5, torch.float64: 1e-12}


@pytest.mark.parametrize('dtype', [torch.float16, torch.bfloat16, torch.float32, torch.float64])
def test_linear_gradients(policy, dtype):
    """td_linear_grad_input and td_linear_grad_weight (+ the bias column sums) against float64 torch on the same
    rounded inputs: the operator backward's shapes (c1h: 8400 tokens; c3: 67200 tokens, many K splits), output_proj
    (300 x 256), and ragged shapes (Nout, K not multiples of the 128-wide tiles or the 64-deep K blocks, token counts
    not multiples of 64), on tensor cores (16-bit types) and on CUDA cores."""
    g = torch.Generator(device='cuda').manual_seed(17)
    for M, Nout, K in ((8400, 256, 256), (67200, 256, 256), (300, 256, 256), (1000, 200, 136), (130, 48, 32),
                       (37, 8, 24)):
        if dtype == torch.float64 and M > 10000:
            continue
        go = torch.randn(M, Nout, generator=g, device='cuda').to(dtype)
        x = torch.randn(M, K, generator=g, device='cuda').to(dtype)
        w = (torch.randn(Nout, K, generator=g, device='cuda') / K ** 0.5).to(dtype)
        with torch.inference_mode():
            gi = _native.linear_grad_input(go, w)
            gw, gb = _native.linear_grad_weight(go, x, with_bias=True)
        want_i = go.double() @ w.double()
        want_w = go.double().t() @ x.double()
        want_b = go.double().sum(0)
        tol = LINEAR_GRAD_TOL[dtype]
        tag = f'{dtype} {policy} M{M} Nout{Nout} K{K}'
        for got, want, what in ((gi, want_i, 'grad_input'), (gw, want_w, 'grad_weight'), (gb, want_b, 'grad_bias')):
            assert got.dtype == dtype and got.shape == want.shape, f'{tag} {what}'
            err = (got.double() - want).abs().max().item()
            assert err <= tol * max(1.0, want.abs().max().item()), f'{tag} {what}: max |diff| {err:.3g}'
    torch.cuda.synchronize()
    assert _native.device_error(clear=True) == 0


def test_backward_runs_only_library_kernels(cuda):
    """One training step of the operator (project and fused order, with output_proj) through the profiler: every
    GPU kernel of the backward is this library's (no cuBLAS / cuDNN GEMM), besides torch's own elementwise work."""
    args = make(1, 300, 8, 32, 256, [(80, 80), (40, 40), (20, 20)], 4, dtype=torch.float16, seed=9)
    x = [t.cuda().requires_grad_(True) if t is not None and t.is_floating_point() else
         (t.cuda() if t is not None else None) for t in args]
    wo = (torch.randn(256, 256, device='cuda') / 16).half().requires_grad_(True)
    for mode in ('project', 'fused'):
        out = ma_deform_attn(*x, mode=mode, output_weight=wo)
        g = torch.randn_like(out)
        with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
            out.backward(g)
            torch.cuda.synchronize()
        names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
        gemm_like = [n for n in names if any(k in n.lower() for k in ('gemm', 'cublas', 'cutlass', 'sm90_', 'sm100_',
                                                                      'nvjet', 'xmma'))
                     and 'grad_gemm' not in n]
        assert not gemm_like, f'{mode}: library GEMMs in the backward: {sorted(set(gemm_like))}'
        assert any('grad_gemm_tc_kernel' in n for n in names), f'{mode}: {sorted(set(names))}'
        for t in x + [wo]:
            if t is not None and t.grad is not None:
                t.grad = None


def test_a_starved_pipeline_ends_in_an_error_status(cuda):
    """The bounded waits of a tensor-core kernel, run out on purpose: with td_test_starve_next_grad_gemm the next
    gradient GEMM's producers issue nothing (no copy, no MMA in flight), every wait gives up after ~1 ms, the kernel
    records the wait's code, frees its tensor memory and exits. The context stays usable: the error word reads the
    code, and the next launches of the same kernel and of the projection kernel (which allocate tensor memory on the
    same SMs) are correct."""
    lib = _native.load()
    assert lib.td_test_starve_next_grad_gemm(0) == 1 and lib.td_test_starve_next_grad_gemm(-5) == 1
    g = torch.Generator(device='cuda').manual_seed(23)
    go = torch.randn(2048, 256, generator=g, device='cuda').half()
    x = torch.randn(2048, 192, generator=g, device='cuda').half()
    torch.cuda.synchronize()
    assert _native.device_error(clear=True) == 0
    assert lib.td_test_starve_next_grad_gemm(2_000_000) == 0
    with torch.inference_mode():
        _native.linear_grad_weight(go, x)  # starved: its output is not written
    torch.cuda.synchronize()
    code = _native.device_error(clear=True)
    assert code in (1, 2), code  # a TMA wait (kErrTmaWait) or the accumulator wait (kErrMmaWait) ran out first
    with torch.inference_mode():
        gw, _ = _native.linear_grad_weight(go, x)
        w = (torch.randn(256, 192, generator=g, device='cuda') / 16).half()
        y = _native.linear(x, w, None)
    torch.cuda.synchronize()
    assert _native.device_error(clear=True) == 0
    want = go.double().t() @ x.double()
    assert (gw.double() - want).abs().max().item() <= 2e-3 * want.abs().max().item()
    assert torch.allclose(y.double(), x.double() @ w.double().t(), atol=3e-3, rtol=3e-3)
