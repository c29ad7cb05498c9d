"""Host logic of the data-parallel policy replicas (config 5) on CPU: observation sharding and the action gather over
gloo ranks (world size 2 and 3), including a batch smaller than the world and a rank that fails."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from yanlongvla_b200 import dp


@pytest.mark.parametrize('B,W', [(1, 1), (1, 2), (8, 2), (7, 3), (512, 8), (3, 8)])
def test_shard_covers_batch(B, W):
    spans = [dp.shard(B, W, r) for r in range(W)]
    assert spans[0][0] == 0 and spans[-1][1] == B
    for (b0, e0), (b1, e1) in zip(spans, spans[1:]):
        assert e0 == b1
    sizes = [e - b for b, e in spans]
    assert max(sizes) - min(sizes) <= 1 and max(sizes) == dp.max_shard(B, W) or B == 0


def _port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _worker(rank, world, port, B, q, fail_rank):
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    try:
        dp.init('gloo', timeout_s=20)
        b, e = dp.shard(B, world, rank)
        if rank == fail_rank:
            raise RuntimeError('injected failure before the gather')
        # every observation's actions are a function of its global index, so rank 0 can check order and content
        acts = torch.arange(b, e, dtype=torch.float32)[:, None, None].expand(e - b, 16, 32).contiguous()
        out = dp.gather_actions(acts, B)
        if rank == 0:
            want = torch.arange(B, dtype=torch.float32)[:, None, None].expand(B, 16, 32)
            q.put(('ok', bool(torch.equal(out, want))))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:                       # noqa: BLE001  (reported to the parent)
        q.put(('error', rank, type(exc).__name__))


def _run(world, B, fail_rank=-1):
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, B, q, fail_rank)) for r in range(world)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(60)
    out = []
    while not q.empty():
        out.append(q.get())
    for p in ps:
        if p.is_alive():
            p.kill()
    return out


@pytest.mark.parametrize('world,B', [(2, 8), (2, 1), (3, 7)])
def test_gather_actions_gloo(world, B):
    res = _run(world, B)
    assert ('ok', True) in res, res


def test_failed_rank_is_reported_not_hung():
    """A rank that dies before the gather: the others end with an error from the short process-group timeout."""
    res = _run(2, 4, fail_rank=1)
    kinds = {r[0] for r in res}
    assert 'error' in kinds and ('ok', True) not in res, res
