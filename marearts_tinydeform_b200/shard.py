"""Batch sharding of ma_deform_attn over torch.distributed ranks (one process per GPU).

Images are independent in the operator: every input except value_weight, value_bias, spatial_shapes and
level_start_index has a leading batch dimension, and output image b depends only on input image b. So a batch is
split into contiguous per-rank shards with no communication in the data path; the only collective is an optional
all-gather of the outputs (NCCL over NVLink on GPUs, gloo on CPU), for callers that need the whole batch on every
rank. Upstream has no distributed code; this module is the B200 build's multi-GPU layer.
"""

import torch
import torch.distributed as dist

from . import ma_deform_attn

BATCHED = (0, 5, 6)  # memory, sampling_locations, attention_weights


def batch_range(batch, world, rank):
    """[start, stop) of `rank`'s images when `batch` images are split over `world` ranks: contiguous, and the first
    batch % world ranks take one image more. A rank may get an empty shard when batch < world."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f'rank {rank} is outside a world of {world}')
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_inputs(inputs, rank, world):
    """This rank's slice of full-batch inputs (memory, value_weight, value_bias, spatial_shapes, level_start_index,
    sampling_locations, attention_weights[, value_padding_mask]); the weights and level metadata are shared, not
    sliced; the padding mask, like memory, is sliced along the batch."""
    start, stop = batch_range(inputs[0].shape[0], world, rank)
    return [t[start:stop] if (i in BATCHED or i == 7) and t is not None else t for i, t in enumerate(inputs)]


def ma_deform_attn_sharded(memory, value_weight, value_bias, spatial_shapes, level_start_index,
                           sampling_locations, attention_weights, mode='auto', group=None, gather=False,
                           value_padding_mask=None, global_batch=None):
    """ma_deform_attn on this rank's images; with gather=True, the outputs of every rank concatenated in rank order.

    Each rank passes its own shard (possibly empty). Without gather there is no collective at all. With gather, the
    shard sizes are exchanged first (one small all-gather and a host read), shards are padded to the largest one for
    a single all_gather_into_tensor, and the padding is dropped; every rank must call it, in the same order.
    global_batch: the whole batch's size, when the shards are batch_range's split of it (as shard_inputs makes
    them). The sizes are then known without the exchange, nothing reads device memory on the host, and the call can
    be captured in a CUDA graph; with equal shards the gathered tensor is the result itself, with no copy.
    """
    out = ma_deform_attn(memory, value_weight, value_bias, spatial_shapes, level_start_index,
                         sampling_locations, attention_weights, mode=mode, value_padding_mask=value_padding_mask)
    if not gather:
        return out
    world = dist.get_world_size(group)
    if global_batch is None:
        sizes = torch.zeros(world, dtype=torch.long, device=out.device)
        mine = torch.tensor([out.shape[0]], dtype=torch.long, device=out.device)
        dist.all_gather_into_tensor(sizes, mine, group=group)
        sizes = sizes.tolist()
    else:
        sizes = [stop - start for start, stop in (batch_range(global_batch, world, r) for r in range(world))]
        if sizes[dist.get_rank(group)] != out.shape[0]:
            raise ValueError(f'this rank holds {out.shape[0]} images, but batch_range gives it '
                             f'{sizes[dist.get_rank(group)]} of {global_batch}')
    widest = max(sizes)
    if all(n == widest for n in sizes):
        everything = out.new_empty((world * widest,) + tuple(out.shape[1:]))
        dist.all_gather_into_tensor(everything, out.contiguous(), group=group)
        return everything
    padded = out.new_zeros((widest,) + tuple(out.shape[1:]))
    padded[:out.shape[0]] = out
    everything = out.new_empty((world * widest,) + tuple(out.shape[1:]))
    dist.all_gather_into_tensor(everything, padded, group=group)
    return torch.cat([everything[r * widest:r * widest + n] for r, n in enumerate(sizes)])
