"""Limb-sharded HE-Mult on the GPU (cross_hemul_shard_*): every shard's output
limbs equal the same limbs of the one-GPU cross_hemul result, bit for bit.

test_limb_shards_match_one_gpu runs all shards of a split on one GPU, one
after another per phase, with the two exchanges done by copying into the
shared limb-outer buffers (what the all-gathers would deliver).  With two or
more GPUs, test_limb_shards_over_nccl runs one process per GPU with the
all-gathers over NCCL."""
import os
import socket

import numpy as np
import pytest

from oracle import cross_oracle as O
from tests.conftest import rng_residues

pytestmark = pytest.mark.gpu


def _setup(n, L, K, dnum, B, seed):
    import torch
    from cross_b200 import hemul, util
    r, c = util.default_rc(n)
    ov = O.find_moduli_ntt(L + K, 28, 2 * n)
    Q, P = ov[:L], ov[L:]
    rng = np.random.default_rng(seed)
    ct = rng_residues(rng, (B, 4, r, c, L), Q)
    ea = rng_residues(rng, (dnum, n, L + K), ov)
    eb = rng_residues(rng, (dnum, n, L + K), ov)
    he = hemul.HEMul(B, r, c, dnum, 1, Q, P)
    he.control_gen(degree_layout=(r, c))
    he.setup_relinearization(ea, eb)
    x_lm = torch.from_numpy(np.ascontiguousarray(ct.reshape(B, 4, n, L).transpose(0, 1, 3, 2))).cuda()
    return he, x_lm


@pytest.mark.parametrize("n,L,K,dnum,world,B", [(65536, 24, 8, 3, 2, 3), (65536, 35, 7, 5, 3, 2),
                                                (65536, 35, 7, 5, 8, 1), (4096, 8, 3, 3, 3, 4)])
def test_limb_shards_match_one_gpu(n, L, K, dnum, world, B):
    import torch
    from cross_b200 import _lib, limb_shard
    he, x_lm = _setup(n, L, K, dnum, B, seed=n + L + world)
    want = he.mul(x_lm, layout=_lib.LAYOUT_LIMB_MAJOR)                          # (B, 2, L - 1, N)
    shards = [limb_shard.LimbShard(he, g, world) for g in range(world)]
    s0 = shards[0]
    cc_all = s0.empty((world * s0.cq, B, n))
    kp_all = s0.empty((world * s0.cp, 2 * B, n))
    for g, s in enumerate(shards):
        s.modup_input(s.own_input(x_lm), cc_all[g * s.cq:(g + 1) * s.cq])
    for g, s in enumerate(shards):
        s.keyswitch(cc_all, kp_all[g * s.cp:(g + 1) * s.cp])
    covered = 0
    for s in shards:
        out = s.empty((B, 2, s.nq, n))
        s.moddown(kp_all, out)
        # integer operator: the tolerance is exact equality
        assert torch.equal(out.view(torch.int32), want[:, :, s.q0:s.q1].contiguous().view(torch.int32)), \
            (world, s.rank, s.q0, s.q1)
        covered += s.nq
    assert covered == L - 1
    he.check_device()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, q):
    import datetime
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))
    try:
        from cross_b200 import _lib, limb_shard
        he, x_lm = _setup(65536, 35, 7, 5, 3, seed=77)
        want = he.mul(x_lm, layout=_lib.LAYOUT_LIMB_MAJOR)
        s = limb_shard.LimbShard(he, rank, world)
        mine = want[:, :, s.q0:s.q1].contiguous().view(torch.int32)
        x_own = s.own_input(x_lm)
        out = s.mul(x_own)
        # the pipelined form, one ciphertext per call (three calls in flight:
        # every workspace slot, gathers overlapping the other calls' kernels)
        many = s.mul_many([x_own[i:i + 1] for i in range(x_own.shape[0])])
        torch.cuda.synchronize()
        bad = [] if torch.equal(out.view(torch.int32), mine) else ["one call"]
        bad += [f"pipelined call {i}" for i, g in enumerate(many) if not torch.equal(g.view(torch.int32), mine[i:i + 1])]
        q.put((rank, "ok" if not bad else f"limbs [{s.q0}, {s.q1}) differ: {bad}"))
        del s, he
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, repr(e)))
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_limb_shards_over_nccl():
    import torch
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("one GPU: the NCCL exchange needs two or more")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    results = dict(q.get(timeout=5) for _ in procs)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert results == {r: "ok" for r in range(world)}, results
