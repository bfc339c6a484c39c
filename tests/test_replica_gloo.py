"""Multi-rank host logic of the data-parallel replicas, on CPU gloo ranks (world size 2 and 3).

Covers the batch sharding, the MAX-over-ranks timing reduction, the single final logits gather
(uneven shards included), and failure behaviour: a rank that dies before the gather makes the
surviving rank's collective fail within the process-group timeout instead of hanging.
"""
import os
import socket
import sys
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import PKG_DIR


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, batch, mode, q):
    try:
        sys.path.insert(0, PKG_DIR)
        os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        from vitfp4 import replica
        replica.init_from_env("gloo", timeout_s=5.0 if mode == "die" else 30.0)
        torch.manual_seed(0)
        model = torch.nn.Linear(12, 5)                      # identical replica on every rank
        images = torch.randn(batch, 12, generator=torch.Generator().manual_seed(1))
        start, count = replica.shard_range(batch, rank, world)
        local = model(images[start:start + count])
        t = replica.max_over_ranks([float(rank + 1), 10.0 - rank])
        if mode == "die" and rank == 1:
            os._exit(3)                                     # leaves between steps, before the gather
        full = replica.gather_logits(local, batch)
        ok = torch.allclose(full, model(images), atol=1e-6) and t == [float(world), 10.0]
        q.put((rank, "ok" if ok else f"mismatch {t}"))
        dist.destroy_process_group()
    except Exception as e:  # the surviving rank of the failure test ends here
        q.put((rank, f"error: {type(e).__name__}: {str(e)[:200]}"))
        traceback.print_exc()


def _run(world, batch, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, batch, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung"
    out = {}
    while not q.empty():
        r, msg = q.get()
        out[r] = msg
    return out, [p.exitcode for p in procs]


def test_shard_range_covers_batch_exactly():
    sys.path.insert(0, PKG_DIR)
    from vitfp4.replica import shard_range
    for batch in (0, 1, 7, 1024, 1025):
        for world in (1, 2, 3, 8):
            spans = [shard_range(batch, r, world) for r in range(world)]
            assert spans[0][0] == 0 and sum(c for _, c in spans) == batch
            assert all(spans[i][0] + spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            assert max(c for _, c in spans) - min(c for _, c in spans) <= 1
    with pytest.raises(ValueError):
        shard_range(8, 2, 2)


@pytest.mark.parametrize("world,batch", [(2, 16), (3, 10)])
def test_replicas_gather_matches_single_process(world, batch):
    out, codes = _run(world, batch, "ok")
    assert out == {r: "ok" for r in range(world)}, out
    assert codes == [0] * world


def test_dead_rank_fails_the_gather_instead_of_hanging():
    out, codes = _run(2, 16, "die")
    assert codes[1] == 3
    assert 0 in out and out[0].startswith("error"), out
