"""CPU oracle for ma_deform_attn -- TEST INFRASTRUCTURE ONLY.

Nothing in the product imports this module. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline and
reference legs use it, and only as the checker or as the timed CPU baseline, never as the thing measured or shipped.

It restates upstream's definition of the operator, ``ma_deform_attn_reference`` (marearts_tinydeform/reference.py
:13-40 of MareArts/marearts-tinydeform v0.1.1):
  * value = memory @ W^T + b                                             (reference.py:28)
  * per level, grid_sample(value, 2 * loc - 1, bilinear, zeros, align_corners=False)  (reference.py:29-37)
  * the attention-weighted sum over levels x points                      (reference.py:38-40)

Two forms:
  ``ma_deform_attn_oracle``  numpy, float64, explicit bilinear corners: the parity checker.
  ``torch_port``             the same steps on torch's CPU operators (F.linear + F.grid_sample) in the input dtype:
                             the timed CPU baseline (it runs the exact operators upstream's CPU path runs).
Both are pinned against golden vectors written by upstream's own ma_deform_attn_reference
(tests/golden/make_golden.py, checked by tests/test_oracle_golden.py).

Value padding mask (an addition to upstream's operator, which has none): Deformable-DETR's input_padding_mask,
value = value.masked_fill(mask[..., None], 0) right after the projection (models/ops/modules/ms_deform_attn.py of
fundamentalvision/Deformable-DETR, not vendored here); a padded token then contributes nothing, its bias included.
With bias=None this equals zeroing the padded memory rows before upstream's own reference, which is how the golden
vectors pin it.

Sampling producer (``sampling_producer_oracle``; an addition: upstream takes sampling_locations and
attention_weights as inputs, already normalised, reference.py:22-23, and has no producer): the published
MSDeformAttn forward of Deformable-DETR (offsets and logits as linear maps of the query, softmax over L * P,
ref + off / (w, h) or ref.xy + off / P * ref.wh * 0.5). Parity of this part is unpinned against upstream, which has
no implementation of it; it is checked against the same steps written with torch's operators.

Sampling rule: grid_sample with align_corners=False maps g = 2 * loc - 1 to pixel x = ((g + 1) * w - 1) / 2 =
loc * w - 0.5; corner (x0 + dx, y0 + dy) of x0 = floor(x) has weight (dx ? fx : 1 - fx) * (dy ? fy : 1 - fy) and
contributes only inside the map (zero padding). For finite locations, clamping x to [-2, w + 1] first changes
nothing; for NaN / +-inf it makes the oracle follow upstream's CUDA kernel (csrc/ma_deform_fused.cu:87-89: such
points sample nothing), where grid_sample itself returns NaN.
"""

import numpy as np


def _np(t):
    """torch tensor / numpy array / None -> float64 or int64 numpy array."""
    if t is None:
        return None
    if hasattr(t, 'detach'):
        t = t.detach().cpu()
        if t.dtype.is_floating_point:
            t = t.double()
        t = t.numpy()
    t = np.asarray(t)
    return t.astype(np.float64) if t.dtype.kind == 'f' else t.astype(np.int64)


def _mask(m):
    """value padding mask (torch / numpy, bool or 0/1) -> numpy bool [B, N]."""
    if hasattr(m, 'detach'):
        m = m.detach().cpu().numpy()
    return np.asarray(m).astype(bool)


def project(memory, weight, bias):
    """value = memory @ weight.T + bias in float64 (reference.py:28, F.linear)."""
    value = _np(memory) @ _np(weight).T
    if bias is not None:
        value = value + _np(bias)
    return value


def level_corners(loc_xy, attn, height, width, start, n_tok):
    """Corner tokens and weights of every point of one level (reference.py:30-37 restated).

    loc_xy [..., 2] (x, y in [0, 1]); attn [...] -> tok [..., 4] int64 (-1 = outside), wt [..., 4] float64.
    """
    def pixel(v, size):
        p = v * size - 0.5
        p = np.where(np.isnan(p), -2.0, p)
        return np.clip(p, -2.0, size + 1.0)

    x = pixel(loc_xy[..., 0], width)
    y = pixel(loc_xy[..., 1], height)
    x0, y0 = np.floor(x), np.floor(y)
    fx, fy = x - x0, y - y0
    x0, y0 = x0.astype(np.int64), y0.astype(np.int64)
    toks, wts = [], []
    for dy in (0, 1):
        for dx in (0, 1):
            xi, yi = x0 + dx, y0 + dy
            tok = start + yi * width + xi
            inside = (xi >= 0) & (xi < width) & (yi >= 0) & (yi < height) & (tok >= 0) & (tok < n_tok)
            w = attn * (fx if dx else 1.0 - fx) * (fy if dy else 1.0 - fy)
            toks.append(np.where(inside, tok, -1))
            wts.append(np.where(inside, w, 0.0))
    return np.stack(toks, -1), np.stack(wts, -1)


def sample(value, n_head, spatial_shapes, level_start_index, sampling_locations, attention_weights):
    """Multi-scale deformable sampling of value [B, N, H*D] -> [B, Q, H*D] in float64 (reference.py:29-40)."""
    value = _np(value)
    shapes, starts = _np(spatial_shapes), _np(level_start_index)
    loc, attn = _np(sampling_locations), _np(attention_weights)
    B, N, HD = value.shape
    _, Q, H, L, P, _ = loc.shape
    assert H == n_head
    D = HD // H
    v = value.reshape(B, N, H, D)
    out = np.zeros((B, Q, H, D))
    bi = np.arange(B).reshape(B, 1, 1, 1)
    hi = np.arange(H).reshape(1, 1, H, 1)
    for lvl in range(L):
        tok, wt = level_corners(loc[:, :, :, lvl], attn[:, :, :, lvl], int(shapes[lvl, 0]), int(shapes[lvl, 1]),
                                int(starts[lvl]), N)                      # [B, Q, H, P, 4]
        for k in range(4):
            t = tok[..., k]
            rows = v[bi, np.maximum(t, 0), hi]                         # [B, Q, H, P, D]
            out += np.einsum('bqhp,bqhpd->bqhd', wt[..., k], np.where((t >= 0)[..., None], rows, 0.0))
    return out.reshape(B, Q, HD)


def ma_deform_attn_oracle(memory, value_weight, value_bias, spatial_shapes, level_start_index,
                          sampling_locations, attention_weights, value_padding_mask=None):
    """Upstream ma_deform_attn_reference (reference.py:13-40) in float64 numpy: [B, Q, H*D]; padded tokens' value
    rows zeroed after the projection."""
    H = sampling_locations.shape[2]
    value = project(memory, value_weight, value_bias)
    if value_padding_mask is not None:
        value = np.where(_mask(value_padding_mask)[..., None], 0.0, value)
    return sample(value, H, spatial_shapes, level_start_index, sampling_locations, attention_weights)


def sample_backward(value, n_head, spatial_shapes, level_start_index, sampling_locations, attention_weights,
                    grad_out):
    """Gradients of sample() with respect to value [B, N, H*D], sampling_locations and attention_weights, given
    grad_out [B, Q, H*D], in float64: the derivative of grid_sample's bilinear rule (x = loc * w - 0.5, corners
    weighted (dx ? fx : 1 - fx) * (dy ? fy : 1 - fy), zero outside the map), which is what autograd computes
    through reference.py:29-40. d x / d loc = w, so d out / d loc_x = attn * w * sum over corners of
    (dx ? 1 : -1) * (dy ? fy : 1 - fy) * <grad_out, value[corner]>, and likewise for y."""
    value = _np(value)
    shapes, starts = _np(spatial_shapes), _np(level_start_index)
    loc, attn, g = _np(sampling_locations), _np(attention_weights), _np(grad_out)
    B, N, HD = value.shape
    _, Q, H, L, P, _ = loc.shape
    D = HD // H
    v = value.reshape(B, N, H, D)
    g = g.reshape(B, Q, H, D)
    grad_value = np.zeros((B, N, H, D))
    grad_loc = np.zeros(loc.shape)
    grad_attn = np.zeros(attn.shape)
    bi = np.broadcast_to(np.arange(B).reshape(B, 1, 1, 1), (B, Q, H, P))
    hi = np.broadcast_to(np.arange(H).reshape(1, 1, H, 1), (B, Q, H, P))
    for lvl in range(L):
        h_l, w_l = int(shapes[lvl, 0]), int(shapes[lvl, 1])
        ones = np.ones(attn[:, :, :, lvl].shape)
        tok, wt = level_corners(loc[:, :, :, lvl], ones, h_l, w_l, int(starts[lvl]), N)   # [B, Q, H, P, 4]
        def pixel(u, size):
            p = u * size - 0.5
            p = np.where(np.isnan(p), -2.0, p)
            return np.clip(p, -2.0, size + 1.0)
        x = pixel(loc[:, :, :, lvl, :, 0], w_l)
        y = pixel(loc[:, :, :, lvl, :, 1], h_l)
        fx, fy = x - np.floor(x), y - np.floor(y)
        a = attn[:, :, :, lvl]                                                             # [B, Q, H, P]
        for k in range(4):
            dx, dy = k & 1, k >> 1
            t = tok[..., k]
            inside = t >= 0
            rows = np.where(inside[..., None], v[bi, np.maximum(t, 0), hi], 0.0)           # [B, Q, H, P, D]
            dot = np.einsum('bqhd,bqhpd->bqhp', g, rows)
            grad_attn[:, :, :, lvl] += wt[..., k] * dot
            grad_loc[:, :, :, lvl, :, 0] += a * w_l * (1.0 if dx else -1.0) * (fy if dy else 1.0 - fy) * dot
            grad_loc[:, :, :, lvl, :, 1] += a * h_l * (1.0 if dy else -1.0) * (fx if dx else 1.0 - fx) * dot
            contrib = (a * wt[..., k])[..., None] * g[:, :, :, None, :]                    # [B, Q, H, P, D]
            sel = np.nonzero(inside)
            np.add.at(grad_value, (bi[sel], t[sel], hi[sel]), contrib[sel])
    return grad_value.reshape(B, N, HD), grad_loc, grad_attn


def ma_deform_attn_backward_oracle(memory, value_weight, value_bias, spatial_shapes, level_start_index,
                                   sampling_locations, attention_weights, grad_out, value_padding_mask=None):
    """float64 gradients of ma_deform_attn_oracle for grad_out [B, Q, H*D]: a dict with 'memory', 'value_weight',
    'value_bias' (None without bias), 'sampling_locations', 'attention_weights' -- what torch autograd gives through
    upstream's reference (nn.Linear, masked_fill, grid_sample)."""
    H = sampling_locations.shape[2]
    mem, W = _np(memory), _np(value_weight)
    value = project(mem, W, value_bias)
    mask = None if value_padding_mask is None else _mask(value_padding_mask)
    if mask is not None:
        value = np.where(mask[..., None], 0.0, value)
    grad_value, grad_loc, grad_attn = sample_backward(value, H, spatial_shapes, level_start_index,
                                                      sampling_locations, attention_weights, grad_out)
    if mask is not None:
        grad_value = np.where(mask[..., None], 0.0, grad_value)
    B, N, HD = grad_value.shape
    gv = grad_value.reshape(B * N, HD)
    return {'memory': grad_value @ W, 'value_weight': gv.T @ mem.reshape(B * N, -1),
            'value_bias': None if value_bias is None else gv.sum(0),
            'sampling_locations': grad_loc, 'attention_weights': grad_attn}


def fused_order(memory, value_weight, value_bias, spatial_shapes, level_start_index,
                sampling_locations, attention_weights, value_padding_mask=None):
    """The same result in the fused order (upstream csrc/ma_deform_fused.cu:6-14):
    out[d] = W[hD + d] . (sum_s w_s memory[t_s]) + b[hD + d] * sum_s w_s, the sums over corners on unpadded tokens.
    Used as an independent property check."""
    mem, W = _np(memory), _np(value_weight)
    b = None if value_bias is None else _np(value_bias)
    shapes, starts = _np(spatial_shapes), _np(level_start_index)
    loc, attn = _np(sampling_locations), _np(attention_weights)
    B, N, C = mem.shape
    _, Q, H, L, P, _ = loc.shape
    D = W.shape[0] // H
    m = np.zeros((B, Q, H, C))
    wsum = np.zeros((B, Q, H))
    bi = np.arange(B).reshape(B, 1, 1, 1)
    pad = None if value_padding_mask is None else _mask(value_padding_mask)
    for lvl in range(L):
        tok, wt = level_corners(loc[:, :, :, lvl], attn[:, :, :, lvl], int(shapes[lvl, 0]), int(shapes[lvl, 1]),
                                int(starts[lvl]), N)
        if pad is not None:  # a corner on a padded token counts as outside
            hit = pad[bi[..., None], np.maximum(tok, 0)] & (tok >= 0)
            tok, wt = np.where(hit, -1, tok), np.where(hit, 0.0, wt)
        for k in range(4):
            t = tok[..., k]
            rows = np.where((t >= 0)[..., None], mem[bi, np.maximum(t, 0)], 0.0)   # [B, Q, H, P, C]
            m += np.einsum('bqhp,bqhpc->bqhc', wt[..., k], rows)
            wsum += wt[..., k].sum(-1)
    Wh = W.reshape(H, D, C)
    out = np.einsum('bqhc,hdc->bqhd', m, Wh)
    if b is not None:
        out += wsum[..., None] * b.reshape(H, D)
    return out.reshape(B, Q, H * D)


def oracle_rows(memory, value_weight, value_bias, spatial_shapes, level_start_index, sampling_locations,
                attention_weights, queries, value_padding_mask=None):
    """Oracle output for selected (b, q) pairs only: [len(queries), H*D] float64.

    Projects only the memory rows those queries touch, so full-size configs can be spot-checked in seconds.
    """
    mem, W = _np(memory), _np(value_weight)
    b = None if value_bias is None else _np(value_bias)
    shapes, starts = _np(spatial_shapes), _np(level_start_index)
    loc, attn = _np(sampling_locations), _np(attention_weights)
    B, N, C = mem.shape
    _, Q, H, L, P, _ = loc.shape
    D = W.shape[0] // H
    out = np.zeros((len(queries), H * D))
    pad = None if value_padding_mask is None else _mask(value_padding_mask)
    for i, (bb, qq) in enumerate(queries):
        acc = np.zeros((H, D))
        for lvl in range(L):
            tok, wt = level_corners(loc[bb, qq, :, lvl], attn[bb, qq, :, lvl], int(shapes[lvl, 0]),
                                    int(shapes[lvl, 1]), int(starts[lvl]), N)   # [H, P, 4]
            for h in range(H):
                t, w = tok[h].ravel(), wt[h].ravel()
                keep = t >= 0
                if pad is not None:
                    keep &= ~pad[bb, np.maximum(t, 0)]
                if not keep.any():
                    continue
                rows = mem[bb, t[keep]] @ W[h * D:(h + 1) * D].T                 # [k, D]
                if b is not None:
                    rows = rows + b[h * D:(h + 1) * D]
                acc[h] += w[keep] @ rows
        out[i] = acc.reshape(-1)
    return out


def torch_port(memory, value_weight, value_bias, spatial_shapes, level_start_index,
               sampling_locations, attention_weights, value_padding_mask=None):
    """reference.py:13-40 on torch's CPU operators, in the inputs' dtype (the timed CPU baseline)."""
    import torch
    import torch.nn.functional as F

    B, N, _ = memory.shape
    _, Q, H, L, P, _ = sampling_locations.shape
    value = F.linear(memory, value_weight, value_bias)
    if value_padding_mask is not None:
        value = value.masked_fill(value_padding_mask.to(torch.bool)[..., None], 0)
    D = value.shape[-1] // H
    grid = (2 * sampling_locations - 1).transpose(1, 2).reshape(B * H, Q, L, P, 2)
    heads = value.view(B, N, H, D).permute(0, 2, 3, 1).reshape(B * H, D, N)
    parts = []
    for lvl in range(L):
        h, w, s = int(spatial_shapes[lvl, 0]), int(spatial_shapes[lvl, 1]), int(level_start_index[lvl])
        img = heads[:, :, s:s + h * w].reshape(B * H, D, h, w)
        parts.append(F.grid_sample(img, grid[:, :, lvl], mode='bilinear', padding_mode='zeros', align_corners=False))
    a = attention_weights.transpose(1, 2).reshape(B * H, 1, Q, L * P)
    out = (torch.cat(parts, -1) * a).sum(-1)
    return out.view(B, H * D, Q).transpose(1, 2).contiguous()


def producer_from_proj(proj, reference_points, spatial_shapes, n_heads, n_points):
    """float64 sampling_locations and attention_weights from the query projection proj [B, Q, 3 * H * L * P]
    (the 2 * H * L * P offsets, then the H * L * P logits) and the reference points / boxes."""
    proj = _np(proj)
    ref = _np(reference_points)
    shapes = _np(spatial_shapes)
    B, Q, _ = proj.shape
    L = shapes.shape[0]
    H, P = n_heads, n_points
    off = proj[..., :2 * H * L * P].reshape(B, Q, H, L, P, 2)
    logit = proj[..., 2 * H * L * P:].reshape(B, Q, H, L * P)
    e = np.exp(logit - logit.max(-1, keepdims=True))
    attn = (e / e.sum(-1, keepdims=True)).reshape(B, Q, H, L, P)
    loc = np.empty((B, Q, H, L, P, 2))
    for l in range(L):
        h_l, w_l = float(shapes[l, 0]), float(shapes[l, 1])
        r = ref[:, :, None, l, None, :]                                  # [B, Q, 1, 1, ref_dim]
        o = off[:, :, :, l]                                              # [B, Q, H, P, 2]
        if ref.shape[-1] == 2:
            loc[:, :, :, l, :, 0] = r[..., 0] + o[..., 0] / w_l
            loc[:, :, :, l, :, 1] = r[..., 1] + o[..., 1] / h_l
        else:
            loc[:, :, :, l, :, 0] = r[..., 0] + o[..., 0] / P * r[..., 2] * 0.5
            loc[:, :, :, l, :, 1] = r[..., 1] + o[..., 1] / P * r[..., 3] * 0.5
    return loc, attn


def sampling_producer_oracle(query, reference_points, spatial_shapes, n_heads, n_points, sampling_weight,
                             sampling_bias):
    """float64 sampling_locations [B, Q, H, L, P, 2] and attention_weights [B, Q, H, L, P] of the MSDeformAttn
    layer, from the query [B, Q, Cq], reference points [B, Q, L, 2] (x, y) or [B, Q, L, 4] (cx, cy, w, h) and the
    packed sampling weight [W_offsets; W_attention] ([3 * H * L * P, Cq]) and bias."""
    proj = project(query, sampling_weight, sampling_bias)
    return producer_from_proj(proj, reference_points, spatial_shapes, n_heads, n_points)


def deform_attn_layer_oracle(query, reference_points, memory, spatial_shapes, level_start_index, n_heads, n_points,
                             sampling_weight, sampling_bias, value_weight, value_bias, output_weight=None,
                             output_bias=None, value_padding_mask=None):
    """float64 layer: sampling_producer_oracle, then ma_deform_attn_oracle on its float64 locations and weights,
    then the optional output projection."""
    loc, attn = sampling_producer_oracle(query, reference_points, spatial_shapes, n_heads, n_points,
                                         sampling_weight, sampling_bias)
    out = ma_deform_attn_oracle(memory, value_weight, value_bias, spatial_shapes, level_start_index, loc, attn,
                                value_padding_mask)
    return out if output_weight is None else project(out, output_weight, output_bias)
