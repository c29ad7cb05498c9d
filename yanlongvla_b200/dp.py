"""Data-parallel replicas of the quantized policy over the observation batch (benchmark config 5).

The policy shards only over independent observations: rank r of W runs observations [r*B/W, (r+1)*B/W) on its own
GPU with its own copy of the weights, and the only communication is one gather of the action chunks to rank 0
(NCCL over NVLink on GPUs, gloo in the CPU tests). There is no collective inside the kernels. Ranks with an empty
slice (B < W) still take part in the gather with a zero-filled slice, so every rank takes the same collective steps.
"""
import datetime
import os

import torch
import torch.distributed as dist


def shard(B, world, rank):
    """[begin, end) of rank's observations: contiguous, sizes differ by at most one, empty when B < world."""
    base, extra = divmod(B, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def max_shard(B, world):
    return (B + world - 1) // world


def gather_actions(actions, B, group=None):
    """All ranks pass their (b_r, chunk, dim) actions; rank 0 gets the (B, chunk, dim) batch in observation order, the
    other ranks None. One padded all_gather_into_tensor (NCCL's fastest gather form; equal sizes on every rank)."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    cap = max_shard(B, world)
    pad = torch.zeros((cap,) + tuple(actions.shape[1:]), dtype=actions.dtype, device=actions.device)
    pad[:actions.shape[0]] = actions
    out = torch.empty((world * cap,) + tuple(actions.shape[1:]), dtype=actions.dtype, device=actions.device)
    dist.all_gather_into_tensor(out, pad, group=group)
    if rank != 0:
        return None
    parts = []
    for r in range(world):
        b, e = shard(B, world, r)
        parts.append(out[r * cap:r * cap + (e - b)])
    return torch.cat(parts, 0)


def init(backend='nccl', timeout_s=120):
    """Process group from the torchrun environment (RANK / WORLD_SIZE / MASTER_ADDR / MASTER_PORT), short timeout so
    that ranks waiting for a dead peer end with an error instead of hanging."""
    if dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    rank, world = int(os.environ.get('RANK', 0)), int(os.environ.get('WORLD_SIZE', 1))
    kw = {}
    if backend == 'nccl':
        local = int(os.environ.get('LOCAL_RANK', 0))
        torch.cuda.set_device(local)
        kw['device_id'] = torch.device('cuda', local)
    dist.init_process_group(backend, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return rank, world
