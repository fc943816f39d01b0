"""Closed-form golden cases of the sampling producer and the whole layer: producer_closed_form.npz.

The producer has no counterpart in upstream (its operator takes sampling_locations and attention_weights as inputs),
so its parity cannot be pinned to upstream's code. These cases pin it to the published definition of Deformable-DETR's
MSDeformAttn instead, by construction rather than by any implementation of it:

  * the query projection's weights are zero, so the offsets and the attention logits are its bias;
  * each query's reference point of level l sits on the centre of pixel (xq, yq) of that level, and every offset is a
    whole number of pixels (dx, dy) -- in pixels for reference points (loc = ref + off / (w_l, h_l)), and scaled by the
    box for reference boxes (loc = ref.xy + off / P * ref.wh * 0.5, boxes of P / (2 w_l) x P / (2 h_l), offsets 4 dx,
    4 dy) -- so every sampling location is the centre of pixel (xq + dx, yq + dy), where bilinear sampling returns
    that pixel's value row and nothing else;
  * the attention weights are the softmax of the logits over each head's L * P points.

The expected output is then plain indexing and a weighted sum -- value = memory @ Wv^T + bv; out[q, h] = sum over
(l, p) of softmax(logits)[h, l, p] * value[start_l + (yq + dy) w_l + (xq + dx), h] (zero for a pixel outside the map)
-- with no bilinear or grid_sample arithmetic anywhere in this script.

    python tests/golden/make_producer_golden.py     # rewrites producer_closed_form.npz beside this file
"""

import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def make(seed=2026):
    rng = np.random.default_rng(seed)
    B, Q, H, P, C, D, Cq = 2, 5, 3, 2, 16, 8, 12
    levels = [(4, 5), (3, 3), (2, 4)]                     # (h, w)
    L = len(levels)
    shapes = np.array(levels, dtype=np.int64)
    starts = np.concatenate([[0], np.cumsum(shapes[:, 0] * shapes[:, 1])[:-1]]).astype(np.int64)
    N = int((shapes[:, 0] * shapes[:, 1]).sum())
    # reference pixels per (b, q, l) and whole-pixel steps per (h, l, p); some steps leave the map on purpose
    ref_px = np.stack([rng.integers(0, shapes[:, 1], size=(B, Q, L)),   # x in [0, w_l)
                       rng.integers(0, shapes[:, 0], size=(B, Q, L))], -1)  # y in [0, h_l)
    step = rng.integers(-2, 3, size=(H, L, P, 2))
    step[0, 0, 0] = (7, 0)                                                # always outside every level's map
    logits = rng.normal(size=(H, L * P))
    w_l = shapes[:, 1].astype(np.float64)
    h_l = shapes[:, 0].astype(np.float64)
    ref2 = np.stack([(ref_px[..., 0] + 0.5) / w_l, (ref_px[..., 1] + 0.5) / h_l], -1)      # [B, Q, L, 2]
    box = np.stack([P / (2 * w_l), P / (2 * h_l)], -1)                                     # [L, 2]
    ref4 = np.concatenate([ref2, np.broadcast_to(box, (B, Q, L, 2))], -1)                  # [B, Q, L, 4]
    # the query projection: zero weights; bias = offsets (head, level, point, xy), then logits (head, level*point)
    off2 = step.astype(np.float64)                  # pixels: loc = ref + off / (w, h)
    off4 = 4.0 * step                               # box form: off / P * wh * 0.5 = 4 dx * (1 / (4 w)) = dx / w
    bias2 = np.concatenate([off2.reshape(-1), logits.reshape(-1)])
    bias4 = np.concatenate([off4.reshape(-1), logits.reshape(-1)])
    sampling_weight = np.zeros((3 * H * L * P, Cq))
    query = rng.normal(size=(B, Q, Cq))
    memory = rng.normal(size=(B, N, C))
    value_weight = rng.normal(size=(H * D, C)) / np.sqrt(C)
    value_bias = rng.normal(size=H * D) * 0.1
    # expected: locations on pixel centres, softmaxed weights, and the output by indexing
    tx = ref_px[:, :, None, :, None, 0] + step[None, None, :, :, :, 0]          # [B, Q, H, L, P]
    ty = ref_px[:, :, None, :, None, 1] + step[None, None, :, :, :, 1]
    locations = np.stack([(tx + 0.5) / w_l[None, None, None, :, None], (ty + 0.5) / h_l[None, None, None, :, None]], -1)
    e = np.exp(logits - logits.max(-1, keepdims=True))
    attn = (e / e.sum(-1, keepdims=True)).reshape(H, L, P)
    weights = np.broadcast_to(attn, (B, Q, H, L, P)).copy()
    value = memory @ value_weight.T + value_bias                                # [B, N, H * D]
    out = np.zeros((B, Q, H * D))
    for b in range(B):
        for q in range(Q):
            for h in range(H):
                for l in range(L):
                    for p in range(P):
                        x, y = tx[b, q, h, l, p], ty[b, q, h, l, p]
                        if 0 <= x < shapes[l, 1] and 0 <= y < shapes[l, 0]:
                            t = starts[l] + y * shapes[l, 1] + x
                            out[b, q, h * D:(h + 1) * D] += attn[h, l, p] * value[b, t, h * D:(h + 1) * D]
    return dict(query=query, ref2=ref2, ref4=ref4, memory=memory, spatial_shapes=shapes, level_start_index=starts,
                sampling_weight=sampling_weight, sampling_bias2=bias2, sampling_bias4=bias4,
                value_weight=value_weight, value_bias=value_bias, locations=locations, weights=weights, out=out,
                n_heads=np.int64(H), n_points=np.int64(P))


if __name__ == '__main__':
    path = os.path.join(HERE, 'producer_closed_form.npz')
    np.savez(path, **make())
    print('wrote', path)
