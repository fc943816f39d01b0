"""Batch sharding of ma_deform_attn over torch.distributed ranks (one process per GPU).

Images are independent in the operator: every input except value_weight, value_bias, spatial_shapes and
level_start_index has a leading batch dimension, and output image b depends only on input image b. So a batch is
split into contiguous per-rank shards with no communication in the data path; the only collective is an optional
all-gather of the outputs, for callers that need the whole batch on every rank: NCCL (or gloo on CPU) after the
operator, or -- PeerGather -- fused into the sampler, which stores every finished row into every rank's output
buffer over NVLink (CUDA IPC peer mappings) and signals its peers when its last row is stored. Upstream has no
distributed code; this module is the B200 build's multi-GPU layer.
"""

import torch
import torch.distributed as dist

from . import _native, ma_deform_attn

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
                           value_padding_mask=None, global_batch=None, peer=None):
    """ma_deform_attn on this rank's images; with gather=True, the outputs of every rank concatenated in rank order.

    Each rank passes its own shard (possibly empty). Without gather there is no collective at all. With gather, the
    shard sizes are exchanged first (one small all-gather and a host read), shards are padded to the largest one for
    a single all_gather_into_tensor, and the padding is dropped; every rank must call it, in the same order.
    global_batch: the whole batch's size, when the shards are batch_range's split of it (as shard_inputs makes
    them). The sizes are then known without the exchange, nothing reads device memory on the host, and the call can
    be captured in a CUDA graph; with equal shards the gathered tensor is the result itself, with no copy.
    peer: a PeerGather (implies gather): the all-gather is fused into the sampler, which stores every row into every
    rank's output over NVLink (project order; `mode` and `group` are the PeerGather's).
    """
    if peer is not None:
        return peer(memory, value_weight, value_bias, spatial_shapes, level_start_index, sampling_locations,
                    attention_weights, value_padding_mask)
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


class _DeviceBuffer:
    """A torch view of a device buffer this module does not allocate through torch (__cuda_array_interface__)."""

    def __init__(self, ptr, shape, typestr, device):
        self.__cuda_array_interface__ = {'shape': tuple(shape), 'typestr': typestr, 'data': (ptr, False),
                                         'version': 3, 'strides': None}
        self.device = device


_TYPESTR = {torch.float16: '<i2', torch.bfloat16: '<i2', torch.float32: '<f4', torch.float64: '<f8'}


def _on(device):
    """The CUDA device context for `device` (a no-op context for other devices)."""
    import contextlib
    return torch.cuda.device(device) if device.type == 'cuda' else contextlib.nullcontext()


def _device_view(ptr, shape, dtype, device):
    """A tensor of `dtype` and `shape` over the device memory at ptr (not owned by the tensor)."""
    return torch.as_tensor(_DeviceBuffer(ptr, shape, _TYPESTR[dtype], device), device=device).view(dtype)


class PeerGather:
    """ma_deform_attn_sharded's all-gather fused into the sampler (td_project_forward_peer): every rank's rows are
    stored straight into every rank's gathered output [global_batch, Q, H * D] over NVLink while the sampler runs,
    and no collective runs afterwards.

    Setup (collective: every rank of `group` constructs it with the same arguments, in the same order): each rank
    allocates `buffers` gathered outputs and one control block through the library, the IPC handles are exchanged
    with all_gather_object, and every rank maps its peers' buffers. Calls (every rank, same order; a rank whose shard
    is empty still calls) return the gathered output of that call; the `buffers` outputs are used in turn, so a
    result stays valid until `buffers` more calls have been made, whatever the peers do (a peer can be at most one
    call ahead, since each call waits for every peer's rows). Under CUDA graph capture keep the number of captured
    calls a multiple of `buffers`. close() (collective) unmaps and frees.

    Without an initialised process group (and group None) it is one rank holding the whole batch: the sampler stores
    its rows into the one output and nothing is exchanged (the same kernels, for single-GPU use and profiling).

    Requirements: CUDA tensors, one GPU per rank, 1-8 ranks, the project order's vector sampler shapes (D * element
    size of 16 * 2^k bytes up to 512); the shards are batch_range's split of global_batch (shard_inputs)."""

    def __init__(self, global_batch, queries, heads, head_dim, dtype, group=None, device=None, buffers=2):
        if buffers < 1:
            raise ValueError('buffers must be >= 1')
        self.group = group
        self._dist = group is not None or (dist.is_available() and dist.is_initialized())
        self.world = dist.get_world_size(group) if self._dist else 1
        self.rank = dist.get_rank(group) if self._dist else 0
        if self.world > 8:
            raise ValueError('PeerGather takes at most 8 ranks')
        if device is None:
            device = torch.device('cuda', torch.cuda.current_device())
        self.device = torch.device(device)
        self.global_batch, self.queries, self.heads, self.head_dim = global_batch, queries, heads, head_dim
        self.dtype = dtype
        self.shape = (global_batch, queries, heads * head_dim)
        e = torch.tensor([], dtype=dtype).element_size()
        nbytes = max(256, -(-global_batch * queries * heads * head_dim * e // 256) * 256)
        self._own, self._opened = [], []
        with _on(self.device):
            mine = []
            for _ in range(buffers):
                ptr, handle = _native.peer_buffer_alloc(nbytes)
                self._own.append(ptr)
                mine.append(handle)
            ctrl, handle = _native.peer_buffer_alloc(_native.PEER_CTRL_BYTES)
            self._own.append(ctrl)
            mine.append(handle)
            everyone = [None] * self.world
            if self._dist:
                dist.all_gather_object(everyone, mine, group=group)
            else:
                everyone[0] = mine
            # table[k][r]: buffer k (the last one is the control block) of rank r, as mapped in this process
            self._table = [[None] * self.world for _ in range(buffers + 1)]
            for r in range(self.world):
                for k in range(buffers + 1):
                    if r == self.rank:
                        self._table[k][r] = self._own[k]
                    else:
                        ptr = _native.peer_buffer_open(everyone[r][k])
                        self._opened.append(ptr)
                        self._table[k][r] = ptr
        self.outputs = [_device_view(self._own[k], self.shape, dtype, self.device) for k in range(buffers)]
        self.calls = 0
        self.first_image = batch_range(global_batch, self.world, self.rank)[0]

    def __call__(self, memory, value_weight, value_bias, spatial_shapes, level_start_index, sampling_locations,
                 attention_weights, value_padding_mask=None):
        """This rank's shard in; the gathered output [global_batch, Q, H * D] (every rank's rows) out."""
        start, stop = batch_range(self.global_batch, self.world, self.rank)
        if memory.shape[0] != stop - start:
            raise ValueError(f'this rank holds {memory.shape[0]} images, but batch_range gives it {stop - start} of '
                             f'{self.global_batch}')
        if memory.dtype != self.dtype or sampling_locations.shape[1] != self.queries:
            raise ValueError('the shard does not match the PeerGather (dtype or query count)')
        k = self.calls % len(self.outputs)
        self.calls += 1
        _native.project_forward_peer(memory, value_weight, value_bias, spatial_shapes, level_start_index,
                                     sampling_locations, attention_weights, self.first_image, self.rank,
                                     self._table[k], self._table[-1], value_padding_mask)
        return self.outputs[k]

    def close(self):
        """Unmap the peers' buffers, wait for every rank to have done so, then free this rank's (collective)."""
        if self._own is None:
            return
        if self.device.type == 'cuda':
            torch.cuda.synchronize(self.device)
        with _on(self.device):
            for ptr in self._opened:
                _native.peer_buffer_close(ptr, True)
            if self._dist:
                dist.barrier(group=self.group)
            for ptr in self._own:
                _native.peer_buffer_close(ptr, False)
        self._own, self._opened, self.outputs = None, [], []
