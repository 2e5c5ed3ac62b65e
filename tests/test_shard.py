"""Multi-rank host logic of the batch sharding (cross_b200/shard.py) on CPU:
world size 2 over gloo on 127.0.0.1, one spawned process per rank, including a
batch-sharded HE-Mult (the oracle's) that must equal the one-rank bytes."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from cross_b200 import shard


def test_shard_bounds_cover_the_batch():
    for total in (0, 1, 5, 64, 65):
        for world in (1, 2, 3, 8):
            spans = [shard.shard_bounds(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard.shard_bounds(4, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    try:
        w, r, lr = shard.rank_env()
        assert (w, r, lr) == (world, rank, rank)
        # slowest rank sets the job time
        assert shard.max_over_ranks(10.0 + rank) == 10.0 + world - 1
        # apply-and-gather over an odd batch returns the 1-rank result on every rank
        batch = torch.arange(5 * 3, dtype=torch.int64).reshape(5, 3)
        out = shard.apply_sharded(lambda x: x * 7 + 1, batch, world, rank)
        assert torch.equal(out, batch * 7 + 1)
        # a batch-sharded HE operator (the oracle's HEMul.mul, hemul.py:153-217)
        # assembled on every rank equals the one-rank result byte for byte
        import numpy as np
        from oracle import cross_oracle as O
        from tests.conftest import rng_residues
        n, r, c, L, K, dnum, B = 1024, 32, 32, 4, 2, 2, 3
        ov = O.find_moduli_ntt(L + K, 28, 2 * n)
        rng = np.random.default_rng(9)
        ct = rng_residues(rng, (B, 4, r, c, L), ov[:L])
        he = O.HEMul(B, r, c, dnum, 1, ov[:L], ov[L:])
        he.setup_relinearization(rng_residues(rng, (dnum, n, L + K), ov), rng_residues(rng, (dnum, n, L + K), ov))
        mul = lambda x: torch.from_numpy(he.mul(x.numpy().view(np.uint32)).view(np.int32))  # noqa: E731
        got = shard.apply_sharded(mul, torch.from_numpy(ct.view(np.int32)), world, rank)
        assert np.array_equal(got.numpy().view(np.uint32), he.mul(ct))
        q.put((rank, "ok"))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_two_ranks_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    results = dict(q.get(timeout=5) for _ in procs)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert results == {0: "ok", 1: "ok"}, results
    assert all(p.exitcode == 0 for p in procs)
