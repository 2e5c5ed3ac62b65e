"""Host-buffer operator calls with the PCIe copies overlapped with compute.

An operator called on CPU tensors (pinned for asynchronous copies) runs
over the batch in chunks: chunk k's host-to-device copy, chunk k-1's
compute and chunk k-2's device-to-host copy proceed together on three
streams, cycling through three sets of device buffers.  The caller's current
stream waits for the last copy, so events or a synchronize on it cover the
whole call; with sync (the default) the host also waits, so the returned
CPU tensor is ready to read.
"""
from __future__ import annotations

from . import _tensor


class HostPipeline:
    NBUF = 3

    def __init__(self):
        self._streams = None
        self._bufs = {}

    def _init(self, t):
        if self._streams is None:
            self._streams = [t.cuda.Stream() for _ in range(3)]

    def _buffers(self, t, cb, in_shape, out_shape):
        key = (cb, tuple(in_shape), tuple(out_shape))
        if key not in self._bufs:
            self._bufs = {key: [(_tensor.empty_u32((cb, *in_shape)), _tensor.empty_u32((cb, *out_shape)))
                                for _ in range(self.NBUF)]}
        return self._bufs[key]

    def run(self, x_host, out_host, chunk, compute, sync=True):
        """compute(x_dev, out_dev, nb, stream) runs the operator on nb
        ciphertexts on `stream`.  x_host / out_host: CPU tensors with the batch
        on axis 0."""
        t = _tensor.torch()
        self._init(t)
        s_in, s_cmp, s_out = self._streams
        cur = t.cuda.current_stream()
        for s in self._streams:
            s.wait_stream(cur)
        B = x_host.shape[0]
        cb = max(1, min(chunk, B))
        bufs = self._buffers(t, cb, x_host.shape[1:], out_host.shape[1:])
        ev = [[t.cuda.Event() for _ in range(3)] for _ in range(self.NBUF)]   # copied in, computed, copied out
        # full chunks, then the last chunk one ciphertext at a time so that little
        # compute and copy-out remains after the final copy-in
        bounds = [(lo, min(B, lo + cb)) for lo in range(0, B, cb)]
        if len(bounds) > 1:
            lo, hi = bounds.pop()
            bounds += [(i, i + 1) for i in range(lo, hi)]
        for k, (lo, hi) in enumerate(bounds):
            nb = hi - lo
            i = k % self.NBUF
            xd, od = bufs[i]
            e_in, e_cmp, e_out = ev[i]
            if k >= self.NBUF:
                s_in.wait_event(e_cmp)        # the compute that read this input buffer is done
            with t.cuda.stream(s_in):
                xd[:nb].copy_(x_host[lo:hi], non_blocking=True)
                e_in.record(s_in)
            s_cmp.wait_event(e_in)
            if k >= self.NBUF:
                s_cmp.wait_event(e_out)       # the output buffer has been copied out
            compute(xd[:nb], od[:nb], nb, s_cmp)
            e_cmp.record(s_cmp)
            s_out.wait_event(e_cmp)
            with t.cuda.stream(s_out):
                out_host[lo:hi].copy_(od[:nb], non_blocking=True)
                e_out.record(s_out)
        cur.wait_stream(s_out)
        if sync:
            s_out.synchronize()
        return out_host
