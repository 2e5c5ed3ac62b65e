"""The bootstrapping kernel mix on the GPU (tabIX.py): each kind of kernel at a
size of the schedule, through the C ABI in the reference's layouts, bit-exact
against the oracle; then a timed pass over those rows whose log the
reference's accumulation reads back."""
import functools

import numpy as np
import pytest

from oracle import cross_oracle as O
from oracle import variants as V

pytestmark = pytest.mark.gpu
N = 65536
ROWS = [("add", (18, N)), ("mult", (19, N)), ("automorph", (19, N)), ("ntt_common", (1, N)),
        ("ntt_common", (7, N)), ("basis_convert", (7, 20, N))]


@pytest.fixture(scope="module")
def mixes():
    import torch
    from cross_b200 import bts_mix
    torch.cuda.set_device(0)
    return {lay: bts_mix.KernelMix(batch=2, layout=lay) for lay in ("native", "reference")}


def _np(t):
    return t.cpu().numpy()


@functools.lru_cache(maxsize=None)
def _oracle_ntt(q):
    return V.NTTVariant(list(q), 256, 256, "montgomery")


@pytest.mark.parametrize("layout", ["native", "reference"])
@pytest.mark.parametrize("kernel,dims", ROWS)
def test_kernel_bit_exact(mixes, kernel, dims, layout):
    import torch
    mix = mixes[layout]
    cs = mix.case(kernel, dims, sets=2)
    for i in range(cs.sets):
        cs.call(i)
    torch.cuda.synchronize()
    q = mix.q
    for i in range(cs.sets):
        got = cs.to_reference(_np(cs.outputs[i]))
        ins = [cs.to_reference(_np(t[i])) for t in cs.inputs]
        if kernel == "add":
            want = O.jax_add(ins[0], ins[1], q[:dims[0]])
        elif kernel == "mult":
            want = O.Barrett(q[:dims[0]]).reduce(ins[0].astype(np.uint64) * ins[1])
        elif kernel == "automorph":
            want = ins[0][:, _np(cs.coef_map).astype(np.int64), :]
        elif kernel == "ntt_common":
            want = _oracle_ntt(tuple(q[:dims[0]])).ntt(ins[0])
        else:
            a, b = dims[0], dims[1]
            ob = O.BConvBarrett(q[:a + b])
            ob.control_gen([(list(range(a)), list(range(a, a + b)))])
            want = ob.basis_change_bat(ins[0])
        assert got.dtype == np.uint32 and got.shape == want.shape
        assert np.array_equal(got, want), f"{kernel}{dims} copy {i}"
    if kernel == "ntt_common":
        cs.ctx.check_device()


def test_measure_and_accumulate(mixes):
    from cross_b200 import bts_mix
    mix = mixes["native"]
    table = bts_mix.invocations()
    rows = [r for r in table if (r[0], r[1]) in set(ROWS)]
    assert len(rows) == len(ROWS)
    log = mix.measure(rows, reps=3)
    lat = bts_mix.parse_latency_log(log)
    assert len(lat) == len(ROWS) and all(v > 0 for v in lat.values())
    want = sum(lat[(k, ",".join(map(str, d)))] * (1 if (k, d) == ("ntt_common", (1, N)) else n)
               for k, d, n in rows)
    assert bts_mix.accumulate_latency_from_log(log, table) == pytest.approx(want)
