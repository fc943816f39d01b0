"""Parity of the CUDA path (through the C ABI) with the oracle, following upstream's test strategy
(tests/test_correctness.py): every mode on every shape case, float32 with TF32 off against atol 2e-5 / rtol 1e-4,
float16 / bfloat16 against the float64 oracle on upcast inputs with atol = rtol = 3e-3 / 2e-2, misaligned memory,
far-outside and empty inputs, rejected inputs; plus the golden vectors, the BASELINE configs at full size, and
size-independent properties (order agreement, linearity, batch independence, graph capture)."""

import numpy as np
import pytest
import torch

from cases import CASES, boundary_case, make, to, upcast
from marearts_tinydeform_b200 import _native, choose_mode, ma_deform_attn, workloads
from oracle import deform_oracle as O

pytestmark = pytest.mark.gpu

TOL = {torch.float32: (2e-5, 1e-4), torch.float16: (3e-3, 3e-3), torch.bfloat16: (2e-2, 2e-2),
       torch.float64: (1e-12, 1e-10)}
MODES = ('fused', 'project', 'auto')


def oracle(args):
    return torch.from_numpy(O.ma_deform_attn_oracle(*[t if t is None else t.cpu() for t in args]))


def check(name, args, ref, atol, rtol, modes=MODES, mask=None):
    with torch.inference_mode():
        for mode in modes:
            got = ma_deform_attn(*args, mode=mode, value_padding_mask=mask).double().cpu()
            assert got.shape == ref.shape, f'{name} [{mode}]'
            err = (got - ref).abs().max().item() if got.numel() else 0.0
            assert torch.allclose(got, ref, atol=atol, rtol=rtol), \
                f'{name} [{mode}]: max |diff| {err:.3g} (max |ref| {ref.abs().max().item():.3g})'


def test_cuda_float32(cuda):
    for name, *shape in CASES:
        for bias in (True, False):
            args = make(*shape, bias=bias)
            check(f'{name} fp32 bias={bias}', to(args, cuda), oracle(args), *TOL[torch.float32])


@pytest.mark.parametrize('dtype', [torch.float16, torch.bfloat16])
def test_cuda_half_and_bfloat16(policy, dtype):
    for name, *shape in CASES:
        for bias in (True, False):
            args = make(*shape, dtype=dtype, bias=bias, seed=1)
            check(f'{name} {dtype} bias={bias} {policy}', to(args, 'cuda'), oracle(upcast(args)), *TOL[dtype])


def test_cuda_float64(cuda):
    for name, *shape in CASES[:3] + CASES[6:]:
        args = make(*shape, dtype=torch.float64)
        check(f'{name} fp64', to(args, cuda), oracle(args), *TOL[torch.float64])


def test_head_rows_that_are_not_a_power_of_two_vectors(cuda):
    """D * element size a multiple of 16 bytes but not a power-of-two number of 16-byte vectors (D=48 half,
    D=10 double, D=12 float) take the generic sampler."""
    for dtype, D in ((torch.float16, 48), (torch.float64, 10), (torch.float32, 12), (torch.bfloat16, 24)):
        args = make(2, 21, 4, D, 4 * D, [(9, 10), (5, 5)], 4, dtype=dtype, seed=D)
        check(f'D={D} {dtype}', to(args, cuda), oracle(upcast(args)), *TOL[dtype])


def test_golden_vectors_through_cuda(policy):
    from test_oracle_golden import CASES as GOLDEN, MASKS
    for key, dtype, inputs, expected, _ in GOLDEN:
        atol, rtol = TOL[dtype]
        mask = MASKS.get(key)
        check(f'golden {key} {policy}', to(inputs, 'cuda'), expected.double(), atol, rtol,
              mask=None if mask is None else mask.cuda())


@pytest.mark.parametrize('dtype', [torch.float32, torch.float16, torch.bfloat16])
def test_value_padding_mask(policy, dtype):
    """The value padding mask in both orders and every kernel family: random masks (some images fully padded)
    against the oracle with the mask; an all-False mask gives the unmasked result bit for bit."""
    for i, (B, Q, H, D, C, levels, P) in enumerate((
            (2, 33, 8, 32, 256, [(12, 13), (6, 7), (3, 4)], 4),   # tensor-core shapes
            (3, 17, 4, 16, 64, [(9, 11), (5, 6)], 4),
            (2, 9, 3, 10, 30, [(5, 7), (3, 4)], 4))):             # odd channels: CUDA-core kernels
        args = make(B, Q, H, D, C, levels, P, dtype=dtype, seed=40 + i)
        N = args[0].shape[1]
        mask = torch.rand(B, N, generator=torch.Generator().manual_seed(i)) < 0.35
        if i == 1:
            mask[-1] = True  # the last image fully padded
        ref = torch.from_numpy(O.ma_deform_attn_oracle(*upcast(args), value_padding_mask=mask))
        dev = to(args, 'cuda')
        check(f'mask case {i} {dtype} {policy}', dev, ref, *TOL[dtype], mask=mask.cuda())
        with torch.inference_mode():
            for mode in ('fused', 'project'):
                none = torch.zeros(B, N, dtype=torch.bool, device='cuda')
                assert torch.equal(ma_deform_attn(*dev, mode=mode, value_padding_mask=none),
                                   ma_deform_attn(*dev, mode=mode)), f'all-False mask {mode} {dtype}'


@pytest.mark.parametrize('dtype', [torch.float32, torch.float16, torch.bfloat16])
def test_output_proj(policy, dtype):
    """The decoder's output_proj chained behind the attention (output_weight / output_bias): against the oracle's
    result projected in float64, both orders, with and without bias; odd widths take the CUDA-core GEMM."""
    g = torch.Generator().manual_seed(9)
    # the last case takes the CUDA-core paths
    for B, Q, H, D, C, levels, P, c_out in ((2, 33, 8, 32, 256, [(12, 13), (6, 7)], 4, 256),
                                            (1, 150, 4, 16, 64, [(9, 11), (5, 6)], 4, 96),
                                            (8, 300, 8, 32, 256, [(10, 12), (5, 6)], 4, 256),
                                            (2, 9, 3, 10, 30, [(5, 7), (3, 4)], 4, 20)):
        args = make(B, Q, H, D, C, levels, P, dtype=dtype, seed=Q)
        HD = H * D
        wo = ((torch.rand(c_out, HD, generator=g) * 2 - 1) / HD ** 0.5).to(dtype)
        for bo in (((torch.rand(c_out, generator=g) * 2 - 1) * 0.05).to(dtype), None):
            attn = O.ma_deform_attn_oracle(*upcast(args))
            want = attn @ wo.double().numpy().T + (0 if bo is None else bo.double().numpy())
            dev = to(args, 'cuda')
            atol, rtol = TOL[dtype]
            with torch.inference_mode():
                for mode in MODES:
                    got = ma_deform_attn(*dev, mode=mode, output_weight=wo.cuda(),
                                         output_bias=None if bo is None else bo.cuda()).double().cpu()
                    assert got.shape == (B, Q, c_out)
                    err = (got - torch.from_numpy(want)).abs().max().item()
                    assert torch.allclose(got, torch.from_numpy(want), atol=atol, rtol=rtol), \
                        f'output_proj {dtype} {mode} c_out={c_out} bias={bo is not None}: {err:.3g}'


def test_linear_matches_torch(cuda):
    """td_linear alone on assorted shapes (tensor-core and CUDA-core paths), against float64."""
    g = torch.Generator().manual_seed(3)
    for dtype in (torch.float32, torch.float16, torch.bfloat16, torch.float64):
        for M, K, N in ((300, 256, 256), (1000, 64, 128), (7, 30, 20), (129, 96, 48)):
            x = (torch.rand(M, K, generator=g) * 2 - 1).to(dtype)
            w = ((torch.rand(N, K, generator=g) * 2 - 1) / K ** 0.5).to(dtype)
            b = ((torch.rand(N, generator=g) * 2 - 1) * 0.1).to(dtype)
            want = x.double() @ w.double().T + b.double()
            with torch.inference_mode():
                got = _native.linear(x.cuda(), w.cuda(), b.cuda()).double().cpu()
            atol, rtol = TOL[dtype]
            assert torch.allclose(got, want, atol=atol, rtol=rtol), f'{dtype} {M}x{K}x{N}'


def test_value_padding_mask_is_checked(cuda):
    args = to(make(2, 8, 2, 8, 16, [(6, 7), (3, 4)], 2), cuda)
    N = args[0].shape[1]
    for bad in (torch.zeros(2, N, device=cuda),                       # not bool
                torch.zeros(2, N - 1, dtype=torch.bool, device=cuda),  # wrong shape
                torch.zeros(2, N, dtype=torch.bool)):                  # wrong device
        for mode in ('fused', 'project'):
            with pytest.raises(RuntimeError):
                with torch.inference_mode():
                    ma_deform_attn(*args, mode=mode, value_padding_mask=bad)


def test_unaligned_memory(cuda):
    for dtype in (torch.float32, torch.float16, torch.bfloat16):
        args = make(1, 40, 8, 32, 256, [(20, 20), (10, 10)], 4, dtype=dtype)
        mem = args[0].to(cuda)
        buf = torch.empty(mem.numel() + 1, dtype=dtype, device=cuda)
        shifted = buf[1:].view(mem.shape)  # contiguous, but 2 or 4 bytes off a 16-byte boundary
        shifted.copy_(mem)
        assert shifted.is_contiguous() and shifted.data_ptr() % 16 != 0
        dev = to(args, cuda)
        check(f'unaligned {dtype}', [shifted] + dev[1:], oracle(upcast(args)), *TOL[dtype])


def test_non_contiguous_inputs(cuda):
    args = make(2, 30, 4, 16, 64, [(12, 10), (6, 5)], 4)
    dev = to(args, cuda)
    mem_t = dev[0].transpose(1, 2).contiguous().transpose(1, 2)     # same values, strided
    w_t = dev[1].t().contiguous().t()
    loc_nc = dev[5].permute(0, 2, 1, 3, 4, 5).contiguous().permute(0, 2, 1, 3, 4, 5)
    assert not mem_t.is_contiguous() and not w_t.is_contiguous() and not loc_nc.is_contiguous()
    check('non-contiguous', [mem_t, w_t, dev[2], dev[3], dev[4], loc_nc, dev[6]], oracle(args),
          *TOL[torch.float32])


def test_far_outside_and_empty(cuda):
    args = make(2, 20, 4, 8, 32, [(9, 11), (5, 6)], 4, spread=200.0)
    check('far outside', to(args, cuda), oracle(args), 1e-5, 1e-4)
    empty = to(make(1, 0, 4, 8, 32, [(9, 11)], 4), cuda)
    with torch.inference_mode():
        for mode in MODES:
            assert ma_deform_attn(*empty, mode=mode).shape == (1, 0, 32)
    nobatch = to(make(0, 5, 4, 8, 32, [(9, 11)], 4), cuda)
    with torch.inference_mode():
        for mode in MODES:
            assert ma_deform_attn(*nobatch, mode=mode).shape == (0, 5, 32)


def test_boundary_locations(cuda):
    for dtype in (torch.float32, torch.float16):
        args = boundary_case(dtype)
        check(f'boundary {dtype}', to(args, cuda), oracle(upcast(args)), *TOL[dtype])


def test_nan_and_inf_locations_sample_nothing(cuda):
    """Upstream's CUDA rule (csrc/ma_deform_fused.cu:87-89): such points contribute zero instead of poisoning the
    output (grid_sample itself would return NaN)."""
    args = make(1, 6, 2, 8, 16, [(6, 7), (3, 4)], 2)
    loc = args[5].clone()
    loc[0, 0, :, :, 0, 0] = float('nan')
    loc[0, 1, :, :, 1, 1] = float('inf')
    loc[0, 2, :, :, 0, 0] = -float('inf')
    loc[0, 3] = float('nan')
    clean = list(args)
    clean_loc = args[5].clone()
    clean_loc[0, 0, :, :, 0] = 5.0   # far outside: samples nothing either
    clean_loc[0, 1, :, :, 1] = 5.0
    clean_loc[0, 2, :, :, 0] = 5.0
    clean_loc[0, 3] = 5.0
    clean[5] = clean_loc
    ref = oracle(clean)
    check('nan/inf locations', to(args[:5] + [loc, args[6]], cuda), ref, *TOL[torch.float32])


def test_rejects_bad_input(cuda):
    args = to(make(1, 8, 2, 8, 16, [(6, 7), (3, 4)], 2), cuda)
    bad = [
        ('weight cols', 1, args[1][:, :8].contiguous()),
        ('dtype', 1, args[1].half()),
        ('bias size', 2, args[2][:4]),
        ('shapes dtype', 3, args[3].int()),
        ('starts dtype', 4, args[4].int()),
        ('loc dtype', 5, args[5].double()),
        ('attn shape', 6, args[6][:, :, :, :1]),
        ('batch', 5, args[5].expand(2, -1, -1, -1, -1, -1)),
        ('shapes on cpu', 3, args[3].cpu()),
        ('too many points', 6, torch.ones(1, 8, 2, 2, 40, device=cuda) / 80),
    ]
    for what, i, value in bad:
        a = list(args)
        a[i] = value
        if what == 'too many points':
            a[5] = torch.rand(1, 8, 2, 2, 40, 2, device=cuda)
        if what == 'batch':
            a[6] = args[6].expand(2, -1, -1, -1, -1)
        for mode in ('fused', 'project'):
            with pytest.raises(RuntimeError):
                with torch.inference_mode():
                    ma_deform_attn(*a, mode=mode)
    with pytest.raises(ValueError):
        ma_deform_attn(*args, mode='nope')


def test_sample_forward_and_value_proj(policy):
    cuda = 'cuda'
    """The two halves of the project order through their own entry points (td_value_proj, td_sample_forward)."""
    for dtype in (torch.float32, torch.float16, torch.bfloat16):
        args = make(2, 37, 8, 32, 256, [(12, 13), (6, 7), (3, 4)], 4, dtype=dtype, seed=3)
        dev = to(args, cuda)
        atol, rtol = TOL[dtype]
        with torch.inference_mode():
            value = _native.value_proj(dev[0], dev[1], dev[2], 8)
            vref = torch.from_numpy(O.project(*[t.cpu() for t in args[:3]]))
            assert torch.allclose(value.double().cpu(), vref, atol=atol, rtol=rtol), dtype
            hm = _native.value_proj(dev[0], dev[1], dev[2], 8, head_major=True)
            assert torch.equal(hm.permute(0, 2, 1, 3).reshape(value.shape), value)
            out = _native.sample_forward(value, 8, *dev[3:])
            sref = torch.from_numpy(O.sample(value.double().cpu(), 8, *args[3:5], *upcast(args[5:])))
            assert torch.allclose(out.double().cpu(), sref, atol=atol, rtol=rtol), dtype


def test_cuda_graph_capture(cuda):
    args = to(make(2, 50, 8, 32, 256, [(20, 20), (10, 10)], 4, dtype=torch.float16), cuda)
    with torch.inference_mode():
        for mode in ('fused', 'project'):
            eager = ma_deform_attn(*args, mode=mode)
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                ma_deform_attn(*args, mode=mode)
            torch.cuda.current_stream().wait_stream(s)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                out = ma_deform_attn(*args, mode=mode)
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(out, eager), mode


def test_modes_agree_and_are_linear_in_attention(cuda):
    """Size-independent properties: fused and project orders agree; without bias the output is linear in the
    attention weights; images are independent (a batch equals its images run one at a time)."""
    args = to(make(3, 64, 8, 32, 256, [(30, 30), (15, 15), (8, 8)], 4, bias=False, seed=5), cuda)
    with torch.inference_mode():
        f = ma_deform_attn(*args, mode='fused')
        p = ma_deform_attn(*args, mode='project')
        torch.testing.assert_close(f, p, atol=2e-5, rtol=1e-4)
        a2 = list(args)
        a2[6] = args[6] * 2
        torch.testing.assert_close(ma_deform_attn(*a2, mode='fused'), 2 * f, atol=4e-5, rtol=1e-4)
        for b in range(3):
            one = [args[0][b:b + 1], args[1], args[2], args[3], args[4], args[5][b:b + 1], args[6][b:b + 1]]
            for mode, whole in (('fused', f), ('project', p)):
                torch.testing.assert_close(ma_deform_attn(*one, mode=mode), whole[b:b + 1], atol=1e-6, rtol=1e-6)


@pytest.mark.parametrize('name', ['c1', 'c1h', 'c2', 'c3'])
def test_baseline_configs_full_size(policy, name):
    """BASELINE configs c1-c3 at full size against the full oracle."""
    for seed in (0, 1):
        args = workloads.make_inputs(name, seed=seed)
        dtype = args[0].dtype
        check(f'{name} seed {seed} {policy}', to(args, 'cuda'), oracle(upcast(args)), *TOL[dtype])


def _rows_oracle(args, picks):
    """oracle_rows for the (b, q) picks, given only the picked images (so that a B=64 batch is never upcast whole)."""
    images = sorted({b for b, _ in picks})
    slot = {b: i for i, b in enumerate(images)}
    idx = torch.tensor(images)
    sub = [None if t is None else (t.index_select(0, idx) if i in (0, 5, 6) else t) for i, t in enumerate(args)]
    return torch.from_numpy(O.oracle_rows(*[t if t is None else t.cpu() for t in upcast(sub)],
                                          [(slot[b], q) for b, q in picks]))


def _spot_check(name, args, dtype, n=24, seed=0):
    """Full-size config: all modes agree with each other, and sampled (b, q) rows match the row oracle."""
    rng = np.random.default_rng(seed)
    B, Q = args[5].shape[:2]
    picks = sorted({(int(rng.integers(B)), int(rng.integers(Q))) for _ in range(n)})
    ref = _rows_oracle(args, picks)
    dev = to(args, 'cuda')
    atol, rtol = TOL[dtype]
    with torch.inference_mode():
        outs = {m: ma_deform_attn(*dev, mode=m) for m in ('fused', 'project')}
    for mode, out in outs.items():
        got = torch.stack([out[b, q] for b, q in picks]).double().cpu()
        err = (got - ref).abs().max().item()
        assert torch.allclose(got, ref, atol=atol, rtol=rtol), f'{name} [{mode}] max |diff| {err:.3g}'
    diff = (outs['fused'].double() - outs['project'].double()).abs()
    assert diff.max().item() <= 2 * atol + 2 * rtol * outs['project'].double().abs().max().item(), name


def test_c4_dino_full_size(cuda):
    args = workloads.make_inputs('c4', seed=0)
    _spot_check('c4', args, torch.float16)
    with torch.inference_mode():
        assert choose_mode(args[0].cuda(), args[1].cuda(), args[5].cuda()) in ('fused', 'project')


def test_c4_dino_full_tensor(cuda):
    """c4 (fp16, B=8, Q=900, DINO 4-level shapes) in full: every output element of both orders against the
    float64 oracle, one seed."""
    args = workloads.make_inputs('c4', seed=1)
    check('c4 full tensor', to(args, cuda), oracle(upcast(args)), *TOL[torch.float16], modes=('fused', 'project'))


def _c5_cases():
    return [(B, Q) for B in workloads.C5_BATCHES for Q in workloads.C5_QUERIES]


@pytest.mark.parametrize('dtype', [torch.float32, torch.float16, torch.bfloat16])
def test_c5_stress_sweep(policy, dtype):
    """The stress config at the operator limits (L*P = 64, C = 512, D = 64) at four points of its batch/query grid,
    under both kernel policies."""
    for B, Q in ((1, 50), (4, 300), (8, 900), (64, 100)):
        args = workloads.make_inputs('c5', seed=B + Q, B=B, Q=Q, dtype=dtype)
        _spot_check(f'c5 B{B} Q{Q} {dtype}', args, dtype, n=12, seed=B)


@pytest.mark.parametrize('B,Q', _c5_cases())
def test_c5_full_grid(cuda, B, Q):
    """Every (B, Q) pair of the stress grid (B in 1, 4, 8, 64; Q in 50, 100, 300, 900 -- B=64 at Q=900 is the
    8-GPU split's whole batch) in all three dtypes with the default kernels: sampled rows of both orders against the
    row oracle, and the two orders against each other over the whole output."""
    base = workloads.make_inputs('c5', seed=1000 + B * 7 + Q, B=B, Q=Q, dtype=torch.float32)
    for dtype in (torch.float32, torch.float16, torch.bfloat16):
        args = [t if t is None or t.dtype == torch.long else t.to(dtype) for t in base]
        _spot_check(f'c5 grid B{B} Q{Q} {dtype}', args, dtype, n=8, seed=B * Q)
        del args
    torch.cuda.empty_cache()


def test_tensor_core_shapes(policy):
    """Shapes at the edges of the tcgen05 paths: D = 16 / 48 / 64 / 128, C = 64 .. 768, query tiles with a ragged
    last tile, token counts that are not a multiple of the 128-row GEMM tile."""
    for dtype in (torch.float16, torch.bfloat16):
        for B, Q, H, D, C, levels, P in ((1, 7, 4, 16, 64, [(5, 7)], 4), (2, 33, 2, 48, 96 * 2, [(9, 9), (4, 5)], 4),
                                         (1, 129, 4, 64, 256, [(11, 13), (6, 6)], 2),
                                         (1, 40, 2, 128, 256, [(12, 12)], 8), (3, 17, 6, 64, 768, [(7, 9)], 4)):
            args = make(B, Q, H, D, C, levels, P, dtype=dtype, seed=D + C)
            check(f'tc shapes B{B} Q{Q} H{H} D{D} C{C} {dtype} {policy}', to(args, 'cuda'), oracle(upcast(args)),
                  *TOL[dtype])


def test_value_proj_tile_widths(cuda):
    """The persistent tcgen05 projection at every tile plan it picks: 64 / 128 / 256 columns reloading the weights
    with every tile (with a staging tile for TMA stores, or storing straight from registers), 256 columns with a
    resident weight slice (16-bit types, C <= 256, at least three tiles per CTA), float32 on the three-product TF32
    path; more tiles than SMs so every CTA walks several, ragged last row and column tiles and a K that is not a
    multiple of the 128-byte block; plain and head-major layouts (head-major D = 24 / 36 cannot store directly)."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    g = torch.Generator().manual_seed(11)
    shapes = ((256, 8, 256), (192, 4, 200), (128, 4, 96), (96, 2, 64), (64, 8, 72), (256, 8, 320), (128, 2, 512),
              (192, 8, 256), (144, 4, 128))
    for dtype in (torch.float32, torch.float16, torch.bfloat16):
        # more 128-row tiles than SMs; 16-bit types also with three 256-wide tiles per SM (resident weights)
        for M in ((128 * (sms + 1) + 37,) if dtype == torch.float32 else (128 * (sms + 1) + 37, 128 * 3 * sms + 101)):
            for HD, H, C in shapes:
                if dtype == torch.float32 and C % 4:
                    continue
                mem = (torch.rand(1, M, C, generator=g) * 2 - 1).to(dtype).cuda()
                w = ((torch.rand(HD, C, generator=g) * 2 - 1) * 0.1).to(dtype).cuda()
                b = ((torch.rand(HD, generator=g) * 2 - 1) * 0.05).to(dtype).cuda()
                ref = mem[0].double() @ w.double().T + b.double()
                with torch.inference_mode():
                    got = _native.value_proj(mem, w, b, H)
                    hm = _native.value_proj(mem, w, b, H, head_major=True)
                atol, rtol = TOL[dtype]
                err = (got[0].double() - ref).abs().max().item()
                tag = f'{dtype} M{M} HD{HD} C{C}'
                assert torch.allclose(got[0].double(), ref, atol=atol, rtol=rtol), f'{tag}: {err:.3g}'
                assert torch.equal(hm.permute(0, 2, 1, 3).reshape(got.shape), got), f'{tag} head-major'
    torch.cuda.synchronize()
    assert _native.device_error(clear=True) == 0


def test_device_error_word_is_clear(cuda):
    """No bounded wait in any tensor-core kernel gave up during the tests above."""
    torch.cuda.synchronize()
    assert _native.device_error(clear=True) == 0
