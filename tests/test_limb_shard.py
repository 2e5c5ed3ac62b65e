"""Limb-sharded HE-Mult (cross_b200/limb_shard.py) on CPU: the ownership ranges,
and the phase driver with its two all-gathers over gloo ranks on 127.0.0.1.

The driver is backend-generic; here each rank runs a numpy backend that
restates the oracle's HE-Mult (hemul.py:153-217) restricted to the rank's own
limbs, with every table taken from the full modulus set (the rescale's
gamma_i depends on all of Q').  Each rank's output limbs must equal the same
limbs of the one-rank oracle result, bit for bit, for 2 ranks and for 3 (an
uneven split: the last rank owns no Q' limb and no P limb)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from cross_b200 import limb_shard

U32, U64 = np.uint32, np.uint64


def test_limb_ranges_cover_the_limbs():
    for n in (0, 1, 4, 7, 23, 34):
        for world in (1, 2, 3, 4, 8):
            rs, ch = limb_shard.limb_ranges(n, world)
            assert len(rs) == world and rs[0][0] == 0 and rs[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(rs, rs[1:]))
            assert all(a == min(n, r * ch) for r, (a, _) in enumerate(rs))    # limb l at gathered index l
            assert max(b - a for a, b in rs) == ch
    with pytest.raises(ValueError):
        limb_shard.limb_ranges(4, 0)


class OracleShard:
    """Numpy backend of limb_sharded_mul: the oracle's HEMul.mul restricted to
    this rank's limbs (test infrastructure)."""

    def __init__(self, he, rank, world):
        from oracle import cross_oracle as O
        self.O, self.he = O, he
        self.r, self.c = he.r, he.c
        self.L1, self.K = len(he.Qd), len(he.P)
        self.q_ranges, self.cq = limb_shard.limb_ranges(self.L1, world)
        self.p_ranges, self.cp = limb_shard.limb_ranges(self.K, world)
        (self.q0, self.q1), (self.p0, self.p1) = self.q_ranges[rank], self.p_ranges[rank]
        self.nq, self.np = self.q1 - self.q0, self.p1 - self.p0
        self.dle = he.Qd + he.P
        self.own = list(range(self.q0, self.q1)) + [self.L1 + k for k in range(self.p0, self.p1)]
        self.qown = he.Qd[self.q0:self.q1]
        self.ff_q = O.Barrett(self.qown) if self.nq else None
        self.ntt_q = O.NTTBarrett(self.qown, self.r, self.c) if self.nq else None
        self.st = {}                       # per-slot state between the phases (the workspace)

    def empty(self, shape):
        return torch.zeros(tuple(shape), dtype=torch.int32)

    def _ref(self, x_lm, E):
        """(B, E, M, N) limb-major -> (B, E, r, c, M)."""
        B, _, M, _ = x_lm.shape
        return np.ascontiguousarray(x_lm.transpose(0, 1, 3, 2)).reshape(B, E, self.r, self.c, M)

    def modup_input(self, x_own, cc_rows, slot=0):
        O, he, own = self.O, self.he, slice(self.q0, self.q1)
        st = self.st.setdefault(slot, {})
        if not self.nq:
            return
        x = self._ref(x_own.numpy().view(U32), 4)
        rp = he.rescale_plan
        last = O._ntt_flat(rp.ntt_last, x[..., -1:].astype(U32), inverse=True)
        last = O._modmul(rp.ff_last, last, rp.power_of_last_tower_inv_psi)
        ge = rp.drop_last[own] - U64(rp.q_last) + last.astype(U64)
        coef = np.where(last < rp.threshold, last.astype(U64), ge)
        red = self.ff_q.reduce(coef.astype(U64) * rp.gammas_power_of_psi_no_last[..., own].astype(U64))
        nt = O._ntt_flat(self.ntt_q, red, inverse=False)
        xr = self.ff_q.reduce(x[..., :self.nq].astype(U64) * rp.betas[own] + nt.astype(U64))
        st["post"], st["d2"] = O.ciphertext_mult(xr, self.ff_q)
        cf = O._ntt_flat(self.ntt_q, st["d2"], inverse=True)
        cf = O._modmul(self.ff_q, cf, he.ks.inv_psi[..., own])                  # (B, 1, r, c, nq)
        B = cf.shape[0]
        cc_rows[:self.nq] = torch.from_numpy(np.ascontiguousarray(
            cf.reshape(B, -1, self.nq).transpose(2, 0, 1)).view(np.int32))

    def keyswitch(self, cc_all, kp_rows, slot=0):
        O, he, ks = self.O, self.he, self.he.ks
        st = self.st.setdefault(slot, {})
        cc = cc_all.numpy().view(U32)[:self.L1]                                 # (L', B, N)
        B = cc.shape[1]
        coef = np.ascontiguousarray(cc.transpose(1, 2, 0)).reshape(B, 1, self.r, self.c, self.L1)
        lt = len(self.own)
        if not lt:
            return
        t0 = t1 = None
        for j, sel in enumerate(ks.sel):
            tg = [l for l in self.own if l not in sel]
            ev = None
            if tg:
                bc = O.BConvBarrett(self.dle)
                bc.control_gen([(list(sel), tg)])
                ev = bc.basis_change_bat(coef[..., list(sel)], 0)
                ev = O._modmul(O.Barrett([self.dle[l] for l in tg]), ev, ks.dl_power_of_psi[..., tg])
                ev = O._ntt_flat(O.NTTBarrett([self.dle[l] for l in tg], self.r, self.c), ev, inverse=False)
            cols = [st["d2"][..., l - self.q0] if l in sel else ev[..., tg.index(l)] for l in self.own]
            ext = np.stack(cols, -1).astype(U64)
            a = ext * ks.evk_b[j][..., self.own][None, None]
            b = ext * ks.evk_a[j][..., self.own][None, None]
            t0 = a if t0 is None else t0 + a
            t1 = b if t1 is None else t1 + b
        st["ks_out"] = O.Barrett([self.dle[l] for l in self.own]).reduce(np.concatenate([t0, t1], axis=1))
        if self.np:
            pm = he.P[self.p0:self.p1]
            ntt_p = O.NTTBarrett(pm, he.ntt_ext.r, he.ntt_ext.c)
            kp = O._ntt_flat(ntt_p, st["ks_out"][..., self.nq:], inverse=True)
            kp = O._modmul(O.Barrett(pm), kp, he.power_of_inv_psi_approx_down[..., self.p0:self.p1])
            kp_rows[:self.np] = torch.from_numpy(np.ascontiguousarray(
                kp.reshape(2 * B, -1, self.np).transpose(2, 0, 1)).view(np.int32))

    def moddown(self, kp_all, out, slot=0):
        O, he, own = self.O, self.he, slice(self.q0, self.q1)
        st = self.st.setdefault(slot, {})
        if not self.nq:
            return
        kp = kp_all.numpy().view(U32)[:self.K]                                  # (K, 2B, N)
        B = kp.shape[1] // 2
        kref = np.ascontiguousarray(kp.transpose(1, 2, 0)).reshape(B, 2, self.r, self.c, self.K)
        bc = O.BConvBarrett(self.dle)
        bc.control_gen([(list(range(self.L1, self.L1 + self.K)), list(range(self.q0, self.q1)))])
        nb = bc.basis_change_bat(kref, 0)
        q = np.array(self.qown, U32)
        outs = []
        for e in range(2):
            t = O._modmul(self.ff_q, nb[:, e:e + 1], he.power_of_psi[..., own])
            t = O._ntt_flat(self.ntt_q, t, inverse=False)
            a = st["ks_out"][:, e:e + 1, ..., :self.nq]
            sub = np.where(a < t, a + q - t, a - t)
            outs.append(O._modmul(self.ff_q, sub, he.PInvModq[own]))
        res = st["post"] + np.concatenate(outs, axis=1)
        res = np.where(res >= q, res - q, res)
        out.copy_(torch.from_numpy(np.ascontiguousarray(
            res.reshape(B, 2, -1, self.nq).transpose(0, 1, 3, 2)).view(np.int32)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    from oracle import cross_oracle as O
    from tests.conftest import rng_residues
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    try:
        n, r, c, L, K, dnum, B = 1024, 32, 32, 5, 2, 2, 3
        ov = O.find_moduli_ntt(L + K, 28, 2 * n)
        Q, P = ov[:L], ov[L:]
        rng = np.random.default_rng(5)
        ct = rng_residues(rng, (B, 4, r, c, L), Q)
        ea = rng_residues(rng, (dnum, n, L + K), ov)
        eb = rng_residues(rng, (dnum, n, L + K), ov)
        he = O.HEMul(B, r, c, dnum, 1, Q, P)
        he.setup_relinearization(ea, eb)
        want = he.mul(ct)                                                       # (B, 2, r, c, L - 1)
        sh = OracleShard(he, rank, world)
        x_lm = ct.reshape(B, 4, n, L).transpose(0, 1, 3, 2)                     # (B, 4, L, N)
        x_own = np.ascontiguousarray(np.concatenate([x_lm[:, :, sh.q0:sh.q1], x_lm[:, :, -1:]], 2))
        got = limb_shard.limb_sharded_mul(sh, torch.from_numpy(x_own.view(np.int32)), rank, world)
        got = got.numpy().view(U32)                                             # (B, 2, nq, N)
        ref = np.ascontiguousarray(want.reshape(B, 2, n, L - 1).transpose(0, 1, 3, 2))[:, :, sh.q0:sh.q1]
        assert np.array_equal(got, ref), f"rank {rank}: limbs [{sh.q0}, {sh.q1}) differ from one rank"
        # the pipelined form, one ciphertext per call: three calls in flight
        # use every workspace slot, and the gathers complete out of call order
        calls = [torch.from_numpy(np.ascontiguousarray(x_own[i:i + 1]).view(np.int32)) for i in range(B)]
        many = limb_shard.limb_sharded_mul_many(sh, calls, rank, world)
        for i, g in enumerate(many):
            assert np.array_equal(g.numpy().view(U32), ref[i:i + 1]), f"rank {rank}: pipelined call {i} differs"
        q.put((rank, "ok"))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_limb_sharded_hemul_gloo_matches_one_rank(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    results = dict(q.get(timeout=5) for _ in procs)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert results == {r: "ok" for r in range(world)}, results
    assert all(p.exitcode == 0 for p in procs)


class _RecordingShard:
    """Backend that records the phases limb_sharded_mul_many runs."""
    cq, cp, nq = 2, 1, 2

    def __init__(self):
        self.log = []

    def empty(self, shape):
        return torch.zeros(tuple(shape), dtype=torch.int32)

    def modup_input(self, x, cc_rows, slot=0):
        self.log.append(("modup", int(x[0, 0, 0, 0]), slot))

    def keyswitch(self, cc_all, kp_rows, slot=0):
        self.log.append(("keyswitch", slot))

    def moddown(self, kp_all, out, slot=0):
        self.log.append(("moddown", slot))
        out.fill_(len(self.log))


def test_pipelined_schedule_order_and_slots():
    """limb_sharded_mul_many's schedule on one rank: step i runs phase 1 of
    call i, phase 2 of call i - 1 and phase 3 of call i - 2, each call keeping
    the workspace slot call % PIPELINE_DEPTH for all three phases, and the
    outputs come back in call order (the order every rank follows, so the
    collectives between the phases match across ranks)."""
    sh = _RecordingShard()
    xs = [torch.full((1, 4, 3, 8), k, dtype=torch.int32) for k in range(5)]
    outs = limb_shard.limb_sharded_mul_many(sh, xs, 0, 1)
    D = limb_shard.PIPELINE_DEPTH
    want = []
    for i in range(len(xs) + 2):
        if i < len(xs):
            want.append(("modup", i, i % D))
        if 0 <= i - 1 < len(xs):
            want.append(("keyswitch", (i - 1) % D))
        if 0 <= i - 2 < len(xs):
            want.append(("moddown", (i - 2) % D))
    assert sh.log == want
    moddown_pos = [j + 1 for j, e in enumerate(want) if e[0] == "moddown"]
    assert [int(o[0, 0, 0, 0]) for o in outs] == moddown_pos
    assert [tuple(o.shape) for o in outs] == [(1, 2, 2, 8)] * len(xs)
