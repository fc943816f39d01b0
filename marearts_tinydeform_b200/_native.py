"""ctypes binding of the C ABI in include/tinydeform.h, plus the tensor-level argument contract.

The checks here raise ``RuntimeError`` under the same conditions as upstream's TORCH_CHECKs
(``csrc/ma_deform_fused.cu:236-266, :298-308, :333``); the library repeats the size checks and returns a status
that is turned into ``RuntimeError`` as well. Tensors are made contiguous (a device copy only when they are not),
the output is allocated from torch's caching allocator, and kernels run on torch's current stream of the memory's
device, so calls are stream-ordered and can be captured in CUDA graphs.
"""

import ctypes
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, '_tinydeform.so')

TD_F32, TD_F16, TD_BF16, TD_F64 = 0, 1, 2, 3
DTYPE_CODE = {torch.float32: TD_F32, torch.float16: TD_F16, torch.bfloat16: TD_BF16, torch.float64: TD_F64}
MAX_LEVEL_POINTS = 64
MAX_CHANNELS = 8192
INT32_MAX = 2 ** 31 - 1

# exported symbol -> (restype, argtypes); the list is also what tests check the .so against
_i64, _vp, _ip, _sz, _cp = ctypes.c_int64, ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t, ctypes.c_char_p
SIGNATURES = {
    'td_fused_forward': (_ip, [_ip, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                               _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _cp, _sz]),
    'td_sample_forward': (_ip, [_ip, _vp, _i64, _vp, _vp, _vp, _vp, _vp,
                                _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _cp, _sz]),
    'td_sample_strided': (_ip, [_ip, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp,
                                _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _cp, _sz]),
    'td_value_proj': (_ip, [_ip, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _ip, _vp, _cp, _sz]),
    'td_project_workspace_bytes': (_sz, [_ip, _i64, _i64, _i64]),
    'td_peer_buffer_alloc': (_ip, [_sz, ctypes.POINTER(ctypes.c_void_p), _vp, _cp, _sz]),
    'td_peer_buffer_open': (_ip, [_vp, ctypes.POINTER(ctypes.c_void_p), _cp, _sz]),
    'td_peer_buffer_close': (_ip, [_vp, ctypes.c_int, _cp, _sz]),
    'td_project_forward_peer': (_ip, [_ip, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64,
                                      _i64, _i64, _i64, _i64, ctypes.c_int, ctypes.c_int,
                                      ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p), _vp, _sz,
                                      _vp, _cp, _sz]),
    'td_test_peer_wait': (_ip, [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_longlong, _vp, _cp, _sz]),
    'td_project_forward': (_ip, [_ip, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                 _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _sz, _vp, _cp, _sz]),
    'td_linear': (_ip, [_ip, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _cp, _sz]),
    'td_sampling_producer': (_ip, [_ip, _vp, _vp, ctypes.c_int, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp,
                                   _cp, _sz]),
    'td_sampling_producer_backward': (_ip, [_ip, _vp, _vp, ctypes.c_int, _vp, _vp, _vp, _vp, _vp, _i64, _i64,
                                            _i64, _i64, _i64, _vp, _cp, _sz]),
    'td_sample_backward': (_ip, [_ip, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                 _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _cp, _sz]),
    'td_project_ex_workspace_bytes': (_sz, [_ip, _i64, _i64, _i64, _i64, _ip]),
    'td_project_forward_ex': (_ip, [_ip, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _vp,
                                    _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _sz, _vp, _cp, _sz]),
    'td_grad_value_finish': (_ip, [_ip, _vp, _vp, _vp, _i64, _i64, _vp, _cp, _sz]),
    'td_layer_workspace_bytes': (_sz, [_ip, _ip, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _ip]),
    'td_layer_forward': (_ip, [_ip, _ip, _vp, _i64, _vp, _ip, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64,
                               _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _sz, _vp, _cp, _sz]),
    'td_fused_forward_masked': (_ip, [_ip, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                      _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _cp, _sz]),
    'td_project_forward_masked': (_ip, [_ip, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                        _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _sz, _vp, _cp, _sz]),
    'td_project_forward_noalloc': (_ip, [_ip, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                         _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _cp, _sz]),
    'td_linear_grad_workspace_bytes': (_sz, [_ip, _i64, _i64]),
    'td_linear_grad_input': (_ip, [_ip, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _cp, _sz]),
    'td_linear_grad_weight': (_ip, [_ip, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _sz, _vp, _cp, _sz]),
    'td_test_starve_next_grad_gemm': (_ip, [ctypes.c_longlong]),
    'td_probe_row_gather': (_ip, [_vp, _i64, _ip, _ip, _i64, ctypes.c_uint, _vp, _sz, _ip, _vp, _cp, _sz]),
    'td_set_kernel_policy': (_ip, [_ip]),
    'td_set_output_proj_plan': (_ip, [_ip]),
    'td_device_error': (_ip, [_ip, ctypes.POINTER(ctypes.c_uint), _cp, _sz]),
    'td_device_info': (_ip, [_ip, ctypes.POINTER(_ip), ctypes.POINTER(_ip), ctypes.POINTER(_ip), _cp, _sz]),
    'td_launch_count': (ctypes.c_uint64, []),
    'td_version': (ctypes.c_char_p, []),
}

_lib = None
_load_error = None


def load(path=LIB_PATH):
    """Load the library (once) and declare every signature. Raises RuntimeError when it is missing."""
    global _lib, _load_error
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        _load_error = f'{path} is not built (run python -m marearts_tinydeform_b200.build)'
        raise RuntimeError('marearts-tinydeform-b200 was installed without its CUDA library: ' + _load_error)
    try:
        lib = ctypes.CDLL(path)
    except OSError as exc:
        _load_error = str(exc)
        raise RuntimeError('marearts-tinydeform-b200 could not load its CUDA library: ' + _load_error) from exc
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def available():
    try:
        load()
        return True
    except RuntimeError:
        return False


def _call(fn, *args):
    err = ctypes.create_string_buffer(512)
    rc = fn(*args, err, ctypes.sizeof(err))
    if rc != 0:
        raise RuntimeError(f'{fn.__name__} failed ({rc}): {err.value.decode(errors="replace")}')


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def check_geometry(ref, spatial_shapes, level_start_index, sampling_locations, attention_weights):
    """Upstream check_geometry (csrc/ma_deform_fused.cu:236-266); returns B, Q, H, L, P."""
    if not ref.is_cuda:
        raise RuntimeError('inputs must be CUDA tensors')
    if ref.dim() != 3:
        raise RuntimeError('memory / value must be [B, N, C]')
    if ref.size(1) > INT32_MAX:
        raise RuntimeError('too many memory tokens')
    if sampling_locations.dim() != 6 or sampling_locations.size(5) != 2:
        raise RuntimeError('sampling_locations must be [B, Q, H, L, P, 2]')
    if attention_weights.dim() != 5:
        raise RuntimeError('attention_weights must be [B, Q, H, L, P]')
    if tuple(attention_weights.shape) != tuple(sampling_locations.shape[:5]):
        raise RuntimeError('attention_weights must be [B, Q, H, L, P] like sampling_locations')
    B, Q, H, L, P = sampling_locations.shape[:5]
    if ref.size(0) != B:
        raise RuntimeError('batch size mismatch')
    if H <= 0:
        raise RuntimeError('need at least one head')
    if L * P > MAX_LEVEL_POINTS:
        raise RuntimeError(f'levels x points must be <= {MAX_LEVEL_POINTS}')
    if spatial_shapes.dtype != torch.long or spatial_shapes.dim() != 2 or spatial_shapes.size(0) != L \
            or spatial_shapes.size(1) != 2:
        raise RuntimeError('spatial_shapes must be int64 [L, 2]')
    if level_start_index.dtype != torch.long or level_start_index.dim() != 1 or level_start_index.size(0) != L:
        raise RuntimeError('level_start_index must be int64 [L]')
    for t in (sampling_locations, attention_weights, spatial_shapes, level_start_index):
        if t.device != ref.device:
            raise RuntimeError('all tensors must be on the same device')
    for t in (sampling_locations, attention_weights):
        if t.dtype != ref.dtype:
            raise RuntimeError('all float tensors must have the same dtype')
    if ref.dtype not in DTYPE_CODE:
        raise RuntimeError(f'unsupported dtype {ref.dtype}')
    if B * Q * H > INT32_MAX:
        raise RuntimeError('too many (batch, query, head) rows')
    return B, Q, H, L, P


def check_projection(memory, value_weight, value_bias, heads):
    """Upstream weight / bias checks (csrc/ma_deform_fused.cu:297-308); returns HD."""
    C = memory.size(2)
    if value_weight.dim() != 2 or value_weight.size(1) != C:
        raise RuntimeError('value_weight must be [H * D, C] with C = memory.size(2)')
    HD = value_weight.size(0)
    if HD % heads != 0:
        raise RuntimeError('value_weight rows must be a multiple of the head count')
    if value_weight.device != memory.device or value_weight.dtype != memory.dtype:
        raise RuntimeError('value_weight must have the device and dtype of memory')
    if value_bias is not None and (value_bias.device != memory.device or value_bias.dtype != memory.dtype
                                   or value_bias.dim() != 1 or value_bias.size(0) != HD):
        raise RuntimeError('value_bias must be [H * D] like value_weight, same device and dtype')
    return HD


def _dense(*ts):
    return [None if t is None else t.contiguous() for t in ts]


def check_mask(value_padding_mask, memory):
    """The value padding mask: bool (or uint8) [B, N] on memory's device, nonzero = padded token. Returns it as a
    contiguous one-byte tensor (or None)."""
    if value_padding_mask is None:
        return None
    m = value_padding_mask
    if m.dtype not in (torch.bool, torch.uint8):
        raise RuntimeError('value_padding_mask must be a bool (or uint8) tensor')
    if m.dim() != 2 or m.size(0) != memory.size(0) or m.size(1) != memory.size(1):
        raise RuntimeError('value_padding_mask must be [B, N] like memory')
    if m.device != memory.device:
        raise RuntimeError('value_padding_mask must be on the device of memory')
    return m.contiguous()


def fused_forward(memory, value_weight, value_bias, spatial_shapes, level_start_index,
                  sampling_locations, attention_weights, value_padding_mask=None):
    """Fused order (upstream _C.fused_forward, csrc/ma_deform_fused.cu:291-325) through td_fused_forward (with a
    value padding mask: td_fused_forward_masked)."""
    lib = load()
    B, Q, H, L, P = check_geometry(memory, spatial_shapes, level_start_index, sampling_locations, attention_weights)
    HD = check_projection(memory, value_weight, value_bias, H)
    mask = check_mask(value_padding_mask, memory)
    N, C = memory.size(1), memory.size(2)
    if C > MAX_CHANNELS:
        raise RuntimeError(f'channels must be <= {MAX_CHANNELS}')
    mem, w, b, shp, st, loc, att = _dense(memory, value_weight, value_bias, spatial_shapes, level_start_index,
                                          sampling_locations, attention_weights)
    out = torch.empty((B, Q, HD), dtype=memory.dtype, device=memory.device)
    if B * Q == 0:
        return out
    with torch.cuda.device(memory.device):
        if mask is None:
            _call(lib.td_fused_forward, DTYPE_CODE[memory.dtype], _ptr(mem), _ptr(w), _ptr(b), _ptr(shp), _ptr(st),
                  _ptr(loc), _ptr(att), _ptr(out), B, Q, N, C, H, HD, L, P, _stream(memory.device))
        else:
            _call(lib.td_fused_forward_masked, DTYPE_CODE[memory.dtype], _ptr(mem), _ptr(w), _ptr(b), _ptr(shp),
                  _ptr(st), _ptr(loc), _ptr(att), _ptr(mask), _ptr(out), B, Q, N, C, H, HD, L, P,
                  _stream(memory.device))
    return out


def check_output_proj(output_weight, output_bias, HD, ref):
    """output_weight [C_out, HD] / output_bias [C_out] or None on ref's device and dtype; returns C_out (0: none)."""
    if output_weight is None:
        if output_bias is not None:
            raise RuntimeError('output_bias needs output_weight')
        return 0
    if output_weight.dim() != 2 or output_weight.size(1) != HD:
        raise RuntimeError('output_weight must be [C_out, H * D]')
    C_out = output_weight.size(0)
    if output_bias is not None and output_bias.shape != (C_out,):
        raise RuntimeError('output_bias must be [C_out] like output_weight')
    for t in (output_weight, output_bias):
        if t is not None and (t.device != ref.device or t.dtype != ref.dtype):
            raise RuntimeError('output_weight / output_bias must have the device and dtype of memory')
    return C_out


def project_forward(memory, value_weight, value_bias, spatial_shapes, level_start_index,
                    sampling_locations, attention_weights, value_padding_mask=None, output_weight=None,
                    output_bias=None, return_value=False):
    """Project order (upstream __init__.py:77-79: F.linear + _C.sample_forward) through td_project_forward (with a
    value padding mask: td_project_forward_masked; with output_proj: td_project_forward_ex). return_value (no
    output_proj): also return the projected value the call computed, head-major [B, H, N, D] (a view of its
    workspace), for a backward pass."""
    lib = load()
    B, Q, H, L, P = check_geometry(memory, spatial_shapes, level_start_index, sampling_locations, attention_weights)
    HD = check_projection(memory, value_weight, value_bias, H)
    mask = check_mask(value_padding_mask, memory)
    C_out = check_output_proj(output_weight, output_bias, HD, memory)
    N, C = memory.size(1), memory.size(2)
    mem, w, b, shp, st, loc, att = _dense(memory, value_weight, value_bias, spatial_shapes, level_start_index,
                                          sampling_locations, attention_weights)
    code = DTYPE_CODE[memory.dtype]
    if C_out:
        out = torch.empty((B, Q, C_out), dtype=memory.dtype, device=memory.device)
        if B * Q == 0:
            return out
        ow, ob = _dense(output_weight, output_bias)
        ws_bytes = lib.td_project_ex_workspace_bytes(code, B, Q, N, HD, 1)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=memory.device)
        with torch.cuda.device(memory.device):
            _call(lib.td_project_forward_ex, code, _ptr(mem), _ptr(w), _ptr(b), _ptr(shp), _ptr(st), _ptr(loc),
                  _ptr(att), _ptr(mask), _ptr(ow), _ptr(ob), C_out, _ptr(out), B, Q, N, C, H, HD, L, P, _ptr(ws),
                  ws_bytes, _stream(memory.device))
        return out
    out = torch.empty((B, Q, HD), dtype=memory.dtype, device=memory.device)
    if B * Q == 0:
        return (out, None) if return_value else out
    ws_bytes = lib.td_project_workspace_bytes(code, B, N, HD)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=memory.device)
    with torch.cuda.device(memory.device):
        if mask is None:
            _call(lib.td_project_forward, code, _ptr(mem), _ptr(w), _ptr(b), _ptr(shp), _ptr(st), _ptr(loc),
                  _ptr(att), _ptr(out), B, Q, N, C, H, HD, L, P, _ptr(ws), ws_bytes, _stream(memory.device))
        else:
            _call(lib.td_project_forward_masked, code, _ptr(mem), _ptr(w), _ptr(b), _ptr(shp), _ptr(st), _ptr(loc),
                  _ptr(att), _ptr(mask), _ptr(out), B, Q, N, C, H, HD, L, P, _ptr(ws), ws_bytes,
                  _stream(memory.device))
    if not return_value:
        return out
    # the library puts the value at the workspace's first 256-byte boundary
    skip = (-ws.data_ptr()) % 256
    e = memory.element_size()
    value = ws[skip:skip + B * N * HD * e].view(memory.dtype).view(B, H, N, HD // H)
    return out, value


IPC_HANDLE_BYTES, PEER_CTRL_BYTES, DEVERR_PEER_WAIT = 64, 64, 5


def peer_buffer_alloc(nbytes):
    """(device pointer, IPC handle bytes) of a new zeroed device buffer that other processes can map."""
    ptr = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    _call(load().td_peer_buffer_alloc, nbytes, ctypes.byref(ptr), ctypes.cast(handle, ctypes.c_void_p))
    return ptr.value, handle.raw


def peer_buffer_open(handle):
    """Device pointer of another process's buffer, mapped into this one from its IPC handle."""
    ptr = ctypes.c_void_p()
    buf = ctypes.create_string_buffer(bytes(handle), IPC_HANDLE_BYTES)
    _call(load().td_peer_buffer_open, ctypes.cast(buf, ctypes.c_void_p), ctypes.byref(ptr))
    return ptr.value


def peer_buffer_close(ptr, opened):
    _call(load().td_peer_buffer_close, ctypes.c_void_p(ptr), 1 if opened else 0)


def project_forward_peer(memory, value_weight, value_bias, spatial_shapes, level_start_index, sampling_locations,
                         attention_weights, first_image, rank, outputs, controls, value_padding_mask=None):
    """This rank's images in the project order, every output row stored into every rank's gathered buffer
    (outputs / controls: device pointers in rank order, as mapped in this process), through td_project_forward_peer;
    returns nothing (the rows land in the buffers)."""
    lib = load()
    B, Q, H, L, P = check_geometry(memory, spatial_shapes, level_start_index, sampling_locations, attention_weights)
    HD = check_projection(memory, value_weight, value_bias, H)
    mask = check_mask(value_padding_mask, memory)
    N, C = memory.size(1), memory.size(2)
    mem, w, b, shp, st, loc, att = _dense(memory, value_weight, value_bias, spatial_shapes, level_start_index,
                                          sampling_locations, attention_weights)
    code = DTYPE_CODE[memory.dtype]
    ws_bytes = lib.td_project_workspace_bytes(code, B, N, HD)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=memory.device)
    world = len(outputs)
    outs = (ctypes.c_void_p * world)(*outputs)
    ctrls = (ctypes.c_void_p * world)(*controls)
    with torch.cuda.device(memory.device):
        _call(lib.td_project_forward_peer, code, _ptr(mem), _ptr(w), _ptr(b), _ptr(shp), _ptr(st), _ptr(loc),
              _ptr(att), _ptr(mask), B, Q, N, C, H, HD, L, P, first_image, world, rank, outs, ctrls, _ptr(ws),
              ws_bytes, _stream(memory.device))


def test_peer_wait(control_ptr, world, rank, limit_cycles, device):
    """Test hook: the peer wait alone on one control block with a short limit (td_test_peer_wait)."""
    with torch.cuda.device(device):
        _call(load().td_test_peer_wait, ctypes.c_void_p(control_ptr), world, rank, limit_cycles, _stream(device))


def linear(x, weight, bias):
    """y = x @ weight.T + bias over the last dimension of x, through td_linear (the tensor-core projection kernel,
    launched to overlap the kernel before it): the decoder's output_proj after ma_deform_attn."""
    lib = load()
    if not x.is_cuda:
        raise RuntimeError('inputs must be CUDA tensors')
    if x.dtype not in DTYPE_CODE:
        raise RuntimeError(f'unsupported dtype {x.dtype}')
    K = x.size(-1)
    if weight.dim() != 2 or weight.size(1) != K:
        raise RuntimeError('output_weight must be [C_out, K] with K = the last dimension of the input')
    if weight.device != x.device or weight.dtype != x.dtype:
        raise RuntimeError('output_weight must have the device and dtype of the input')
    Nout = weight.size(0)
    if bias is not None and (bias.device != x.device or bias.dtype != x.dtype or bias.dim() != 1
                             or bias.size(0) != Nout):
        raise RuntimeError('output_bias must be [C_out] like output_weight, same device and dtype')
    xs, w, b = _dense(x, weight, bias)
    y = torch.empty(tuple(x.shape[:-1]) + (Nout,), dtype=x.dtype, device=x.device)
    M = xs.numel() // K if K else 0
    if M == 0:
        return y
    with torch.cuda.device(x.device):
        _call(lib.td_linear, DTYPE_CODE[x.dtype], _ptr(xs), _ptr(w), _ptr(b), _ptr(y), M, K, Nout,
              _stream(x.device))
    return y


def sampling_producer(proj, reference_points, spatial_shapes, heads, points):
    """sampling_locations [B, Q, H, L, P, 2] and attention_weights [B, Q, H, L, P] from the query projection
    proj [B, Q, 3 * H * L * P] (offsets, then logits) and reference points [B, Q, L, 2 | 4], through
    td_sampling_producer."""
    lib = load()
    if not proj.is_cuda or not reference_points.is_cuda or not spatial_shapes.is_cuda:
        raise RuntimeError('inputs must be CUDA tensors')
    if proj.dtype not in DTYPE_CODE or reference_points.dtype != proj.dtype:
        raise RuntimeError('proj and reference_points must share a supported float dtype')
    if spatial_shapes.dtype != torch.long or spatial_shapes.dim() != 2 or spatial_shapes.size(1) != 2:
        raise RuntimeError('spatial_shapes must be int64 [L, 2]')
    L = spatial_shapes.size(0)
    if reference_points.dim() != 4 or reference_points.size(2) != L or reference_points.size(3) not in (2, 4):
        raise RuntimeError('reference_points must be [B, Q, L, 2] or [B, Q, L, 4]')
    B, Q = reference_points.shape[:2]
    H, P = heads, points
    if proj.shape != (B, Q, 3 * H * L * P):
        raise RuntimeError('the query projection must be [B, Q, 3 * H * L * P]')
    if L * P > MAX_LEVEL_POINTS:
        raise RuntimeError(f'levels x points must be <= {MAX_LEVEL_POINTS}')
    pr, ref, shp = _dense(proj, reference_points, spatial_shapes)
    loc = torch.empty((B, Q, H, L, P, 2), dtype=proj.dtype, device=proj.device)
    attn = torch.empty((B, Q, H, L, P), dtype=proj.dtype, device=proj.device)
    if B * Q == 0:
        return loc, attn
    with torch.cuda.device(proj.device):
        _call(lib.td_sampling_producer, DTYPE_CODE[proj.dtype], _ptr(pr), _ptr(ref), ref.size(3), _ptr(shp),
              _ptr(loc), _ptr(attn), B, Q, H, L, P, _stream(proj.device))
    return loc, attn


def sampling_producer_backward(proj, reference_points, spatial_shapes, heads, points, grad_loc, grad_attn,
                               want_ref=True):
    """(grad_proj [B, Q, 3 * H * L * P], grad_reference_points or None) of the producer through
    td_sampling_producer_backward; grad_loc / grad_attn may be None (zero)."""
    lib = load()
    B, Q = reference_points.shape[:2]
    L = spatial_shapes.size(0)
    pr, ref, shp = _dense(proj, reference_points, spatial_shapes)
    gl = None if grad_loc is None else _dense(grad_loc.to(proj.dtype))[0]
    ga = None if grad_attn is None else _dense(grad_attn.to(proj.dtype))[0]
    grad_proj = torch.empty_like(pr)
    grad_ref = torch.empty_like(ref) if want_ref else None
    if B * Q == 0:
        return grad_proj, None if grad_ref is None else grad_ref.zero_()
    with torch.cuda.device(proj.device):
        _call(lib.td_sampling_producer_backward, DTYPE_CODE[proj.dtype], _ptr(pr), _ptr(ref), ref.size(3),
              _ptr(shp), None if gl is None else _ptr(gl), None if ga is None else _ptr(ga), _ptr(grad_proj),
              None if grad_ref is None else _ptr(grad_ref), B, Q, heads, L, points, _stream(proj.device))
    return grad_proj, grad_ref


ORDER_CODE = {'project': 0, 'fused': 1}


def layer_forward(query, reference_points, memory, spatial_shapes, level_start_index, heads, points,
                  sampling_weight, sampling_bias, value_weight, value_bias, output_weight=None, output_bias=None,
                  value_padding_mask=None, order='project'):
    """One deformable attention layer through td_layer_forward: query projection -> producer -> attention
    (-> output projection). Returns [B, Q, H * D], or [B, Q, C_out] with output_weight."""
    lib = load()
    if order not in ORDER_CODE:
        raise RuntimeError(f'order must be one of {tuple(ORDER_CODE)}')
    for t in (query, reference_points, memory, spatial_shapes, level_start_index):
        if not t.is_cuda:
            raise RuntimeError('inputs must be CUDA tensors')
    if memory.dim() != 3 or query.dim() != 3:
        raise RuntimeError('memory must be [B, N, C] and query [B, Q, Cq]')
    dt, dev = memory.dtype, memory.device
    if dt not in DTYPE_CODE:
        raise RuntimeError(f'unsupported dtype {dt}')
    B, N, C = memory.shape
    Q, Cq = query.size(1), query.size(2)
    if query.size(0) != B:
        raise RuntimeError('batch size mismatch')
    if spatial_shapes.dtype != torch.long or spatial_shapes.dim() != 2 or spatial_shapes.size(1) != 2:
        raise RuntimeError('spatial_shapes must be int64 [L, 2]')
    L = spatial_shapes.size(0)
    if level_start_index.dtype != torch.long or level_start_index.shape != (L,):
        raise RuntimeError('level_start_index must be int64 [L]')
    if reference_points.dim() != 4 or reference_points.shape[:3] != (B, Q, L) or reference_points.size(3) not in (2, 4):
        raise RuntimeError('reference_points must be [B, Q, L, 2] or [B, Q, L, 4]')
    H, P = heads, points
    if H <= 0 or P <= 0 or L <= 0:
        raise RuntimeError('heads, points and levels must be positive')
    if L * P > MAX_LEVEL_POINTS:
        raise RuntimeError(f'levels x points must be <= {MAX_LEVEL_POINTS}')
    if B * Q * H > INT32_MAX:
        raise RuntimeError('too many (batch, query, head) rows')
    if sampling_weight.shape != (3 * H * L * P, Cq):
        raise RuntimeError('sampling_weight must be [3 * H * L * P, Cq]: the offset rows, then the attention rows')
    if sampling_bias is not None and sampling_bias.shape != (3 * H * L * P,):
        raise RuntimeError('sampling_bias must be [3 * H * L * P]')
    HD = check_projection(memory, value_weight, value_bias, H)
    C_out = 0
    if output_weight is not None:
        if output_weight.dim() != 2 or output_weight.size(1) != HD:
            raise RuntimeError('output_weight must be [C_out, H * D]')
        C_out = output_weight.size(0)
        if output_bias is not None and output_bias.shape != (C_out,):
            raise RuntimeError('output_bias must be [C_out] like output_weight')
    elif output_bias is not None:
        raise RuntimeError('output_bias needs output_weight')
    if order == 'fused' and C > MAX_CHANNELS:
        raise RuntimeError(f'channels must be <= {MAX_CHANNELS}')
    floats = (query, reference_points, sampling_weight, sampling_bias, value_weight, value_bias, output_weight,
              output_bias)
    for t in floats:
        if t is not None and (t.device != dev or t.dtype != dt):
            raise RuntimeError('all float tensors must have the dtype and device of memory')
    for t in (spatial_shapes, level_start_index):
        if t.device != dev:
            raise RuntimeError('all tensors must be on the same device')
    mask = check_mask(value_padding_mask, memory)
    q, ref, sw, sb, mem, vw, vb, ow, ob, shp, st = _dense(query, reference_points, sampling_weight, sampling_bias,
                                                          memory, value_weight, value_bias, output_weight,
                                                          output_bias, spatial_shapes, level_start_index)
    out = torch.empty((B, Q, C_out if output_weight is not None else HD), dtype=dt, device=dev)
    if B * Q == 0:
        return out
    code, oc = DTYPE_CODE[dt], ORDER_CODE[order]
    ws_bytes = lib.td_layer_workspace_bytes(code, oc, B, Q, N, H, HD, L, P, int(output_weight is not None))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _call(lib.td_layer_forward, code, oc, _ptr(q), Cq, _ptr(ref), ref.size(3), _ptr(sw), _ptr(sb), _ptr(mem),
              _ptr(vw), _ptr(vb), _ptr(mask), _ptr(shp), _ptr(st), _ptr(ow), _ptr(ob), C_out, _ptr(out),
              B, Q, N, C, H, HD, L, P, _ptr(ws), ws_bytes, _stream(dev))
    return out


def sample_forward(value, heads, spatial_shapes, level_start_index, sampling_locations, attention_weights):
    """Sampling of a projected value [B, N, H*D] (upstream _C.sample_forward, csrc/ma_deform_fused.cu:327-350)."""
    lib = load()
    B, Q, H, L, P = check_geometry(value, spatial_shapes, level_start_index, sampling_locations, attention_weights)
    N, HD = value.size(1), value.size(2)
    if heads != H or HD % H != 0:
        raise RuntimeError('value must be [B, N, H * D] with H = sampling_locations.size(2)')
    v, shp, st, loc, att = _dense(value, spatial_shapes, level_start_index, sampling_locations, attention_weights)
    out = torch.empty((B, Q, HD), dtype=value.dtype, device=value.device)
    if B * Q == 0:
        return out
    with torch.cuda.device(value.device):
        _call(lib.td_sample_forward, DTYPE_CODE[value.dtype], _ptr(v), heads, _ptr(shp), _ptr(st), _ptr(loc),
              _ptr(att), _ptr(out), B, Q, N, HD, H, L, P, _stream(value.device))
    return out


def sample_backward(value, spatial_shapes, level_start_index, sampling_locations, attention_weights,
                    grad_out, value_padding_mask=None, heads=None):
    """Gradients of the sampling half through td_sample_backward, for value in the nn.Linear layout [B, N, H * D]
    (heads given) or head-major [B, H, N, D] (heads=None), and grad_out [B, Q, H * D]: (grad_value [B, N, H * D]
    in float32 -- float64 for float64 --, grad_sampling_locations, grad_attention_weights in the input dtype)."""
    lib = load()
    if heads is None:
        B, H, N, D = value.shape
        strides = (H * N * D, D, N * D)
    else:
        B, N, HD = value.shape
        H = heads
        if HD % H != 0:
            raise RuntimeError('value must be [B, N, H * D]')
        D = HD // H
        strides = (N * HD, HD, D)
    check_geometry(value.reshape(B, -1, D), spatial_shapes, level_start_index, sampling_locations,
                   attention_weights)
    Q = sampling_locations.size(1)
    L, P = sampling_locations.shape[3:5]
    if grad_out.shape != (B, Q, H * D) or grad_out.dtype != value.dtype or grad_out.device != value.device:
        raise RuntimeError('grad_out must be [B, Q, H * D] with the dtype and device of value')
    mask = value_padding_mask
    if mask is not None:
        if mask.dtype not in (torch.bool, torch.uint8) or mask.shape != (B, N) or mask.device != value.device:
            raise RuntimeError('value_padding_mask must be a bool (or uint8) [B, N] tensor on the device of value')
        mask = mask.contiguous()
    v, shp, st, loc, att, g = _dense(value, spatial_shapes, level_start_index, sampling_locations,
                                     attention_weights, grad_out)
    acc = torch.float64 if value.dtype == torch.float64 else torch.float32
    grad_value = torch.empty((B, N, H * D), dtype=acc, device=v.device)
    grad_loc = torch.empty_like(loc)
    grad_attn = torch.empty_like(att)
    with torch.cuda.device(v.device):
        _call(lib.td_sample_backward, DTYPE_CODE[v.dtype], _ptr(v), *strides, _ptr(shp), _ptr(st),
              _ptr(loc), _ptr(att), _ptr(mask), _ptr(g), _ptr(grad_value), _ptr(grad_loc), _ptr(grad_attn),
              B, Q, N, H, D, L, P, _stream(v.device))
    return grad_value, grad_loc, grad_attn


def grad_value_finish(grad_value, dtype, with_bias):
    """(grad_value rounded to dtype -- the float32 accumulator itself for float32 --, its column sums in float32 or
    None) through td_grad_value_finish; grad_value is the float32 [B, N, HD] of sample_backward. Returns None when
    the shape does not fit the kernel (HD % 4 != 0 or HD > 1024)."""
    lib = load()
    HD = grad_value.size(-1)
    if dtype not in (torch.float32, torch.float16, torch.bfloat16) or grad_value.dtype != torch.float32 \
            or HD % 4 != 0 or HD > 1024 or not grad_value.is_contiguous():
        return None
    rows = grad_value.numel() // HD
    out = grad_value if dtype == torch.float32 else torch.empty(grad_value.shape, dtype=dtype,
                                                                device=grad_value.device)
    bias = torch.empty(HD, dtype=torch.float32, device=grad_value.device) if with_bias else None
    with torch.cuda.device(grad_value.device):
        _call(lib.td_grad_value_finish, DTYPE_CODE[dtype], _ptr(grad_value),
              None if dtype == torch.float32 else _ptr(out), _ptr(bias), rows, HD, _stream(grad_value.device))
    return out, bias


def sample_head_major(value_hm, spatial_shapes, level_start_index, sampling_locations, attention_weights):
    """Sampling of a head-major value [B, H, N, D] (the layout td_project_forward uses) via td_sample_strided."""
    lib = load()
    B, H, N, D = value_hm.shape
    check_geometry(value_hm.view(B, H * N, D), spatial_shapes, level_start_index, sampling_locations,
                   attention_weights)
    Q = sampling_locations.size(1)
    L, P = sampling_locations.shape[3:5]
    v, shp, st, loc, att = _dense(value_hm, spatial_shapes, level_start_index, sampling_locations, attention_weights)
    out = torch.empty((B, Q, H * D), dtype=value_hm.dtype, device=value_hm.device)
    if B * Q == 0:
        return out
    with torch.cuda.device(value_hm.device):
        _call(lib.td_sample_strided, DTYPE_CODE[v.dtype], _ptr(v), H * N * D, D, N * D, _ptr(shp), _ptr(st),
              _ptr(loc), _ptr(att), _ptr(out), B, Q, N, H, D, L, P, _stream(v.device))
    return out


def value_proj(memory, value_weight, value_bias, heads, head_major=False):
    """value = memory @ value_weight.T + value_bias as [B, N, HD], or head-major [B, H, N, D], via td_value_proj."""
    lib = load()
    if not memory.is_cuda or memory.dim() != 3:
        raise RuntimeError('memory must be a CUDA [B, N, C] tensor')
    HD = check_projection(memory, value_weight, value_bias, heads)
    B, N, C = memory.shape
    mem, w, b = _dense(memory, value_weight, value_bias)
    shape = (B, heads, N, HD // heads) if head_major else (B, N, HD)
    value = torch.empty(shape, dtype=memory.dtype, device=memory.device)
    if B * N == 0:
        return value
    with torch.cuda.device(memory.device):
        _call(lib.td_value_proj, DTYPE_CODE[memory.dtype], _ptr(mem), _ptr(w), _ptr(b), _ptr(value), B, N, C,
              heads, HD, 1 if head_major else 0, _stream(memory.device))
    return value


POLICY_BEST, POLICY_CUDA_CORES = 0, 1


def set_kernel_policy(policy):
    """POLICY_BEST (tcgen05 where the shapes allow, the default) or POLICY_CUDA_CORES; returns the previous one."""
    prev = load().td_set_kernel_policy(policy)
    if prev < 0:
        raise ValueError(f'unknown kernel policy {policy}')
    return prev


OUTPROJ_AUTO, OUTPROJ_CHAINED, OUTPROJ_CLUSTER = 0, 1, 2


_outproj_plan = 0  # the plan last set through set_output_proj_plan (the library's default is automatic)


def output_proj_plan():
    return _outproj_plan


def set_output_proj_plan(plan):
    """How the project order applies output_proj: OUTPROJ_AUTO (in the sampler's cluster kernel while its grid is one
    wave, B * Q * H / 8 <= 3 CTAs per SM; the default), OUTPROJ_CHAINED (a separate GEMM) or OUTPROJ_CLUSTER (the
    cluster kernel wherever its shape conditions hold); returns the previous plan."""
    global _outproj_plan
    prev = load().td_set_output_proj_plan(plan)
    if prev < 0:
        raise ValueError(f'unknown output_proj plan {plan}')
    _outproj_plan = plan
    return prev


def device_error(clear=True):
    """The library's device error word on the current device (0 = fine); synchronises."""
    code = ctypes.c_uint(0)
    _call(load().td_device_error, 1 if clear else 0, ctypes.byref(code))
    return code.value


def launch_count():
    return int(load().td_launch_count())


def version():
    return load().td_version().decode()


def probe_row_gather(buf, row_bytes, visits, wide=False, seed=12345, grid=None, sink=None):
    """One launch of the L2 random-row gather probe over buf (a CUDA tensor, bytes viewed as [rows, row_bytes]):
    `visits` rows rounded up to the kernel's multiple. Returns the number of rows actually read (queued on the
    current stream, not synchronised). sink: int32 [grid * 1024] scratch (allocated when None)."""
    lib = load()
    dev = buf.device
    if grid is None:
        grid = torch.cuda.get_device_properties(dev).multi_processor_count * 8
    word = 32 if wide else 16
    chunk = grid * 8 * (32 // (row_bytes // word)) * (4 if wide else 8)
    visits = -(-visits // chunk) * chunk
    if sink is None:
        sink = torch.empty(grid * 256 * 4, dtype=torch.int32, device=dev)
    rows = buf.numel() * buf.element_size() // row_bytes
    with torch.cuda.device(dev):
        _call(lib.td_probe_row_gather, _ptr(buf), rows, row_bytes, 1 if wide else 0, visits, seed, _ptr(sink),
              sink.numel() * 4, grid, _stream(dev))
    return visits


def linear_grad_input(grad_out, weight):
    """grad_out [..., Nout] @ weight [Nout, K] -> [..., K] through td_linear_grad_input: the input gradient of
    y = x @ weight.T (+ b)."""
    lib = load()
    Nout, K = weight.shape
    if grad_out.size(-1) != Nout or grad_out.dtype != weight.dtype or grad_out.device != weight.device:
        raise RuntimeError('grad_out must be [..., Nout] with the dtype and device of weight [Nout, K]')
    if grad_out.dtype not in DTYPE_CODE:
        raise RuntimeError(f'unsupported dtype {grad_out.dtype}')
    g, w = _dense(grad_out, weight)
    out = torch.empty(tuple(grad_out.shape[:-1]) + (K,), dtype=weight.dtype, device=weight.device)
    M = g.numel() // Nout
    if M == 0:
        return out
    with torch.cuda.device(weight.device):
        _call(lib.td_linear_grad_input, DTYPE_CODE[weight.dtype], _ptr(g), _ptr(w), _ptr(out), M, Nout, K,
              _stream(weight.device))
    return out


def linear_grad_weight(grad_out, x, with_bias=False):
    """(grad_out^T @ x [Nout, K], the column sums of grad_out [Nout] or None) over every row of grad_out [..., Nout]
    and x [..., K], through td_linear_grad_weight: the weight and bias gradients of y = x @ weight.T + b."""
    lib = load()
    Nout, K = grad_out.size(-1), x.size(-1)
    if grad_out.dtype != x.dtype or grad_out.device != x.device or grad_out.numel() // max(Nout, 1) != \
            x.numel() // max(K, 1):
        raise RuntimeError('grad_out and x must have the same rows, dtype and device')
    if x.dtype not in DTYPE_CODE:
        raise RuntimeError(f'unsupported dtype {x.dtype}')
    g, xs = _dense(grad_out, x)
    M = g.numel() // Nout
    code = DTYPE_CODE[x.dtype]
    grad_w = torch.empty((Nout, K), dtype=x.dtype, device=x.device)
    grad_b = torch.empty((Nout,), dtype=x.dtype, device=x.device) if with_bias else None
    ws_bytes = lib.td_linear_grad_workspace_bytes(code, Nout, K)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device)
    with torch.cuda.device(x.device):
        _call(lib.td_linear_grad_weight, code, _ptr(g), _ptr(xs), _ptr(grad_w), _ptr(grad_b), M, Nout, K, _ptr(ws),
              ws_bytes, _stream(x.device))
    return grad_w, grad_b
