"""HE-Mult sharded by RNS limb across ranks (one process per GPU).

The reference parallelises only over the ciphertext batch (util.py:40-58).
For large parameter sets or small batches the limbs of every ciphertext can
be split across GPUs instead: rank g owns a contiguous range of the Q' limbs
(Q without its last modulus) and of the P limbs, and computes exactly the
per-limb operations of HEMul.mul (hemul.py:153-217) for them -- the output
limbs are bit-identical to one GPU's.  Only the key switch's two basis
conversions read limbs of other ranks (ciphertext.py:486-498 needs every
digit's limbs, hemul.py:179-186 every P limb), so one HE-Mult takes two
all-gathers of coefficient-form limbs:

    phase 1  rescale, tensor product, INTT(d2) psi^-i    (owned Q' limbs)
             all-gather cc: L' limbs x B ciphertexts
    phase 2  ModUp BConv into the owned limbs, NTTs, inner product with the
             evaluation key, INTT(KS) psi^-i of the owned P limbs
             all-gather kp: K limbs x 2 B elements
    phase 3  ModDown BConv into the owned Q' limbs, NTT with the ModDown
             tail and the add of (d0, d1)

Exchange buffers are limb-outer ([limb][ciphertext][N]) so that each rank's
slice is contiguous and an all-gather of equal chunks places limb l at index
l; ranges are chunks of ceil(limbs / world) (the last ranks may own fewer
limbs, or none).  `limb_sharded_mul` runs the phases of any backend with
that interface for one call; `limb_sharded_mul_many` runs a sequence of calls
three deep, so that each all-gather overlaps the neighbouring calls' compute;
`LimbShard` is the CUDA backend (the C ABI's cross_hemul_shard_* phases).
"""
from __future__ import annotations

from typing import List, Tuple

from . import _lib, _tensor
from .bconv import BConvBarrett


def limb_ranges(n: int, world: int) -> Tuple[List[Tuple[int, int]], int]:
    """Contiguous [start, stop) ranges of n limbs over `world` ranks, each a
    chunk of ceil(n / world) limbs (trailing ranks may get fewer or none),
    and the chunk size."""
    if world < 1 or n < 0:
        raise ValueError(f"bad limb split n={n} world={world}")
    ch = -(-n // world) if n else 0
    return [(min(n, r * ch), min(n, (r + 1) * ch)) for r in range(world)], ch


def gather_start(buf, chunk: int, rank: int, world: int, group=None):
    """Start filling buf (world * chunk rows on axis 0) with every rank's rows
    [rank * chunk, (rank + 1) * chunk) and return the function that completes
    it.  CUDA tensors: an in-place NCCL all-gather on the process group's
    stream, which starts once the current stream's earlier work is done;
    completing it makes the current stream wait for it (the host does not
    block).  CPU tensors: a gloo all-gather through a list, waited for and
    copied in on completion.  The rows travel as int32 words."""
    if world == 1 or chunk == 0:
        return lambda: None
    import torch
    import torch.distributed as dist
    flat = buf.view(torch.int32) if buf.dtype == torch.uint32 else buf
    mine = flat[rank * chunk:(rank + 1) * chunk]
    if flat.is_cuda:
        return dist.all_gather_into_tensor(flat, mine, group=group, async_op=True).wait
    parts = [torch.empty_like(mine) for _ in range(world)]
    work = dist.all_gather(parts, mine.contiguous(), group=group, async_op=True)

    def finish():
        work.wait()
        flat.copy_(torch.cat(parts, 0))
    return finish


def all_gather_chunks(buf, chunk: int, rank: int, world: int, group=None) -> None:
    """gather_start, completed at once."""
    gather_start(buf, chunk, rank, world, group)()


def limb_sharded_mul(backend, x_own, rank: int, world: int, group=None):
    """One rank's HE-Mult of a batch split by limb.  x_own: (B, 4, nq + 1, N),
    the owned Q' limbs then the last limb of Q, limb-major; returns (B, 2, nq,
    N), the owned limbs of HEMul.mul.  backend: modup_input(x, cc_rows),
    keyswitch(cc_all, kp_rows), moddown(kp_all, out), with attributes nq,
    cq, cp (owned Q' limbs, exchange chunks) and empty(shape)."""
    B, N = x_own.shape[0], x_own.shape[-1]
    cc_all = backend.empty((world * backend.cq, B, N))
    backend.modup_input(x_own, cc_all[rank * backend.cq:(rank + 1) * backend.cq])
    all_gather_chunks(cc_all, backend.cq, rank, world, group)
    kp_all = backend.empty((world * backend.cp, 2 * B, N))
    backend.keyswitch(cc_all, kp_all[rank * backend.cp:(rank + 1) * backend.cp])
    all_gather_chunks(kp_all, backend.cp, rank, world, group)
    out = backend.empty((B, 2, backend.nq, N))
    backend.moddown(kp_all, out)
    return out


# calls in flight in limb_sharded_mul_many: phase 1 of call k, phase 2 of
# call k - 1 and phase 3 of call k - 2
PIPELINE_DEPTH = 3


def limb_sharded_mul_many(backend, xs, rank: int, world: int, group=None):
    """limb_sharded_mul over a sequence of calls, software-pipelined so that
    every all-gather overlaps other calls' compute: in step i the rank runs
    phase 1 of call i (whose ModUp gather then starts), phase 2 of call i - 1
    (after its ModUp gather; its ModDown gather then starts) and phase 3 of
    call i - 2 (after its ModDown gather).  Every rank issues the same
    collectives in the same order.  The backend keeps one workspace per call
    in flight: its phase methods take `slot` (call index mod PIPELINE_DEPTH).
    Returns the outputs of the calls in order."""
    n = len(xs)
    outs = [None] * n
    cc, kp, fin1, fin2 = {}, {}, {}, {}
    for i in range(n + 2):
        k = i
        if k < n:
            B, N = xs[k].shape[0], xs[k].shape[-1]
            cc[k] = backend.empty((world * backend.cq, B, N))
            backend.modup_input(xs[k], cc[k][rank * backend.cq:(rank + 1) * backend.cq], slot=k % PIPELINE_DEPTH)
            fin1[k] = gather_start(cc[k], backend.cq, rank, world, group)
        k = i - 1
        if 0 <= k < n:
            fin1.pop(k)()
            B, N = xs[k].shape[0], xs[k].shape[-1]
            kp[k] = backend.empty((world * backend.cp, 2 * B, N))
            backend.keyswitch(cc[k], kp[k][rank * backend.cp:(rank + 1) * backend.cp], slot=k % PIPELINE_DEPTH)
            fin2[k] = gather_start(kp[k], backend.cp, rank, world, group)
        k = i - 2
        if 0 <= k < n:
            fin2.pop(k)()
            B, N = xs[k].shape[0], xs[k].shape[-1]
            outs[k] = backend.empty((B, 2, backend.nq, N))
            backend.moddown(kp.pop(k), outs[k], slot=k % PIPELINE_DEPTH)
            del cc[k]
    return outs


class LimbShard:
    """Rank `rank` of `world`'s share of an HEMul (after control_gen and
    setup_relinearization) on the current CUDA device: owned limb ranges,
    its basis-conversion controls and the cross_hemul_shard plan."""

    def __init__(self, hemul, rank: int, world: int):
        if hemul._plan is None:
            raise RuntimeError("call HEMul.control_gen() and setup_relinearization() first")
        if not 0 <= rank < world:
            raise ValueError(f"rank {rank} out of range for world {world}")
        self.hemul, self.rank, self.world = hemul, rank, world
        L1, K = len(hemul.drop_last_moduli), len(hemul.extend_moduli)
        self.q_ranges, self.cq = limb_ranges(L1, world)
        self.p_ranges, self.cp = limb_ranges(K, world)
        (self.q0, self.q1), (self.p0, self.p1) = self.q_ranges[rank], self.p_ranges[rank]
        self.nq, self.np = self.q1 - self.q0, self.p1 - self.p0
        dle = hemul.drop_last_extend_moduli
        own = list(range(self.q0, self.q1)) + [L1 + k for k in range(self.p0, self.p1)]
        ctl, self._ctl_index = [], []
        for g in hemul.digit_groups:
            tg = [l for l in own if l not in g]
            self._ctl_index.append(len(ctl) if tg else None)
            if tg:
                ctl.append((g, tg))
        self.ks_bconv = BConvBarrett(dle)
        if ctl:
            self.ks_bconv.control_gen(ctl)
        self.down_bconv = None
        if self.nq:
            self.down_bconv = BConvBarrett(dle)
            self.down_bconv.control_gen([(list(range(L1, L1 + K)), list(range(self.q0, self.q1)))])
        ks = [self.ks_bconv.plan(i) if i is not None else None for i in self._ctl_index]
        self._ks_arr = (_lib.vp * len(ks))(*ks)
        desc = _lib.HemulShardDesc(hemul._plan, self.q0, self.q1, self.p0, self.p1, self._ks_arr,
                                   self.down_bconv.plan(0) if self.down_bconv else None)
        out = _lib.vp()
        _lib.check(_lib.lib().cross_hemul_shard_create(_lib.C.byref(desc), _lib.C.byref(out)),
                   "cross_hemul_shard_create")
        self._shard = out
        self._ws = [None] * PIPELINE_DEPTH

    def __del__(self):
        if getattr(self, "_shard", None) is not None and getattr(_lib, "_lib", None) is not None:
            _lib._lib.cross_hemul_shard_destroy(self._shard)
            self._shard = None

    def empty(self, shape):
        return _tensor.empty_u32(tuple(shape))

    def _workspace(self, batch, slot=0):
        need = int(_lib.lib().cross_hemul_shard_workspace_size(self._shard, batch))
        if self._ws[slot] is None or self._ws[slot].numel() < need:
            self._ws[slot] = _tensor.workspace(need)
        return self._ws[slot]

    def own_input(self, x_lm):
        """The rank's input (B, 4, nq + 1, N) from a full limb-major batch
        (B, 4, L, N): the owned Q' limbs and the last limb of Q."""
        t = _tensor.torch()
        xi = x_lm.view(t.int32)
        return t.cat([xi[:, :, self.q0:self.q1], xi[:, :, -1:]], 2).contiguous().view(t.uint32)

    def modup_input(self, x_own, cc_rows, slot=0):
        B = x_own.shape[0]
        ws = self._workspace(B, slot)
        _tensor.call("cross_hemul_shard_modup_input", self._shard, x_own.data_ptr(), B, cc_rows.data_ptr(),
                     ws.data_ptr(), ws.numel(), _lib.cuda_stream())

    def keyswitch(self, cc_all, kp_rows, slot=0):
        B = cc_all.shape[1]
        ws = self._workspace(B, slot)
        _tensor.call("cross_hemul_shard_keyswitch", self._shard, cc_all.data_ptr(), B, kp_rows.data_ptr(),
                     ws.data_ptr(), ws.numel(), _lib.cuda_stream())

    def moddown(self, kp_all, out, slot=0):
        B = out.shape[0]
        ws = self._workspace(B, slot)
        _tensor.call("cross_hemul_shard_moddown", self._shard, kp_all.data_ptr(), B, out.data_ptr(),
                     ws.data_ptr(), ws.numel(), _lib.cuda_stream())

    def mul(self, x_own, group=None):
        """limb_sharded_mul on this shard (collectives in `group`)."""
        return limb_sharded_mul(self, x_own, self.rank, self.world, group)

    def mul_many(self, xs, group=None):
        """limb_sharded_mul_many on this shard: the calls' exchanges overlap
        the neighbouring calls' compute."""
        return limb_sharded_mul_many(self, xs, self.rank, self.world, group)
