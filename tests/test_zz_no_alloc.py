"""cross_ntt_noalloc: the allocation-free NTT entry point.

Callers that cannot allocate device memory on their call path (a plugin
inside a framework that has already reserved the GPU's memory, a loop that
cannot afford cudaFree's synchronisation) use cross_ntt_noalloc, which keeps
the NTT's intermediate in a static device array instead of a workspace.  This
file checks, through the C ABI, that it returns exactly what cross_ntt
returns on two calls in a row (the array keeps the previous call's contents,
so the second call must not depend on them), that the largest batch the
array holds matches as well, and that the first batch beyond it is refused.  It is collected last so a failure here leaves the rest of
the suite already run.
"""
import numpy as np
import pytest

from oracle import cross_oracle as O
from tests.conftest import rng_residues

pytestmark = pytest.mark.gpu


def _lm_input(rng, batch, r, c, moduli):
    x = rng_residues(rng, (batch, r, c, len(moduli)), moduli)
    return np.ascontiguousarray(x.transpose(0, 3, 1, 2))   # (batch, M, r, c) limb-major


@pytest.mark.parametrize("n,r,c,limbs,batch", [(4096, 64, 64, 8, 4), (65536, 256, 256, 6, 2)])
def test_noalloc_matches_workspace_entry_point(n, r, c, limbs, batch):
    import torch
    from cross_b200 import _lib, ntt_mm
    lib = _lib.lib()
    q = O.find_moduli_ntt(limbs, 28, 2 * n)
    ctx = ntt_mm.NTTCiphertextBarrettContext(q, {"r": r, "c": c})
    plan = ctx.plan()
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(n + batch)
    ws = torch.empty(lib.cross_ntt_workspace_size(plan, batch, _lib.LAYOUT_LIMB_MAJOR), dtype=torch.uint8,
                     device="cuda")
    for call in range(2):                       # two calls in a row, fresh inputs each time
        for inverse in (0, 1):
            x = torch.from_numpy(_lm_input(rng, batch, r, c, q)).cuda()
            want = torch.empty_like(x)
            got = torch.empty_like(x)
            _lib.check(lib.cross_ntt(plan, inverse, x.data_ptr(), want.data_ptr(), batch, _lib.LAYOUT_LIMB_MAJOR,
                                     ws.data_ptr(), ws.numel(), stream), "cross_ntt")
            _lib.check(lib.cross_ntt_noalloc(plan, inverse, x.data_ptr(), got.data_ptr(), batch, stream),
                       "cross_ntt_noalloc")
            torch.cuda.synchronize()
            # integer transform: the tolerance is exact equality
            assert torch.equal(got.view(torch.int32), want.view(torch.int32)), (call, inverse)


def test_noalloc_boundary_of_the_static_array():
    """The intermediate takes two words per input word (CROSS_NTT_NOALLOC_MAX_WORDS
    = 16 MiB / 8): with 8 limbs at N = 2^16 batch 4 fits exactly and matches
    cross_ntt, batch 5 is refused before any launch.  Both calls get in/out
    buffers sized for their request, so even a regressed size guard could
    not touch memory outside them."""
    import torch
    from cross_b200 import _lib, ntt_mm
    lib = _lib.lib()
    n, limbs = 65536, 8
    q = O.find_moduli_ntt(limbs, 28, 2 * n)
    ctx = ntt_mm.NTTCiphertextBarrettContext(q, {"r": 256, "c": 256})
    plan = ctx.plan()
    stream = torch.cuda.current_stream().cuda_stream
    max_words = (16 << 20) // 8
    fits = max_words // (limbs * n)              # largest batch whose 2 x batch x M x N scratch words fit
    assert fits == 4
    rng = np.random.default_rng(99)
    x = torch.from_numpy(_lm_input(rng, fits, 256, 256, q)).cuda()
    want, got = torch.empty_like(x), torch.empty_like(x)
    ws = torch.empty(lib.cross_ntt_workspace_size(plan, fits, _lib.LAYOUT_LIMB_MAJOR), dtype=torch.uint8,
                     device="cuda")
    _lib.check(lib.cross_ntt(plan, 0, x.data_ptr(), want.data_ptr(), fits, _lib.LAYOUT_LIMB_MAJOR, ws.data_ptr(),
                             ws.numel(), stream), "cross_ntt")
    _lib.check(lib.cross_ntt_noalloc(plan, 0, x.data_ptr(), got.data_ptr(), fits, stream), "cross_ntt_noalloc")
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int32), want.view(torch.int32))
    over = fits + 1                              # the first batch that does not fit
    xo = torch.zeros((over, limbs, n), dtype=torch.int32, device="cuda")
    yo = torch.zeros_like(xo)
    rc = lib.cross_ntt_noalloc(plan, 0, xo.data_ptr(), yo.data_ptr(), over, stream)
    assert rc == -4                              # CROSS_ERR_WORKSPACE, before any launch
    assert b"exceeds" in lib.cross_last_error()
    torch.cuda.synchronize()
    assert int(yo.abs().sum()) == 0              # nothing was written
