"""The CKKS bootstrapping kernel mix (tabIX.py).

A bootstrapping at N = 2^16 calls five kinds of evaluation kernel, each at many
limb counts; ``data/bts_invocations.csv`` (the reference's
BTS_KERNEL_INVOCATION_CSV, tabIX.py:399-580) says how often.  The mix times
each kernel once per size and weights the latencies by those counts
(tabIX.py:582-617).  The kernels, at 256 x 256 and one polynomial per GPU by
default (the reference runs one per device, tabIX.py:47-53):

  add(L)              element-wise modular add over L limbs (tabIX.py:208-245)
  mult(L)             element-wise modular multiply over L limbs (tabIX.py:247-284)
  automorph(L)        the coefficient permutation of HE-Rotate (tabIX.py:286-316)
  ntt_common(L)       the Montgomery NTT over L limbs; L = 1 is the
                      single-modulus context (tabIX.py:131-206)
  basis_convert(a, b) BConvBarrett.basis_change_bat from a to b limbs (tabIX.py:319-354)

Each measurement prints a line in the reference's format (``add(L,N) -
latency:X``, ...); :func:`parse_latency_log`, :func:`accumulate_latency_from_log`
and :func:`print_latency_ratios` read such a log as the reference's functions
of the same names do.  Latencies are microseconds per polynomial.

The operands are device-resident, in the library's limb-major layout by
default (the layout its HE chains keep between kernels) or in the reference's;
the element-wise kernels have one layout for both.
"""
from __future__ import annotations

import csv
import math
import os
import re
import zlib
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import numpy as np

KERNELS = ("mult", "ntt_common", "basis_convert", "automorph", "add")
DEGREE = 65536
R = C = 256
TABLE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "data", "bts_invocations.csv")
# L2 of a B200 is 126 MB: every row cycles through enough copies of its
# operands that consecutive calls never find their inputs in L2.
L2_BYTES = 126 * 1024 * 1024

Row = Tuple[str, Tuple[int, ...], int]


def invocations(path: str = TABLE) -> List[Row]:
    """(kernel, dims, count) rows of the bootstrapping schedule, dims as in the
    reference's table: (L, N) for add / mult / automorph / ntt_common and
    (a, b, N) for basis_convert."""
    with open(path, newline="") as f:
        return [(r["kernel"], tuple(int(v) for v in r["dims"].split()), int(r["count"]))
                for r in csv.DictReader(f)]


def _normalize_dims(dim: str) -> str:
    """tabIX.py:357-359: a dims key without spaces or parentheses."""
    return dim.strip().lstrip("(").rstrip(")").replace(" ", "")


def _dims_key(*numbers) -> str:
    return ",".join(str(n) for n in numbers)


# tabIX.py:367-393: how each latency line is recognised and keyed.  ntt_common
# lines print the degree first, the table keys them limbs first; the
# basis_convert key carries the degree, which its line omits.
_PATTERNS: Sequence[Tuple[str, Callable]] = (
    (r"add\((\d+),\s*(\d+)\)\s*-\s*latency:([0-9.]+)",
     lambda m: ("add", _dims_key(m.group(1), m.group(2)), float(m.group(3)))),
    (r"mult\((\d+),\s*(\d+)\)\s*-\s*latency:([0-9.]+)",
     lambda m: ("mult", _dims_key(m.group(1), m.group(2)), float(m.group(3)))),
    (r"automorph\((\d+),\s*(\d+)\)\s*-\s*latency:([0-9.]+)",
     lambda m: ("automorph", _dims_key(m.group(1), m.group(2)), float(m.group(3)))),
    (r"ntt_common\((\d+),\s*(\d+)\)\s*b\d+\s*-\s*latency:([0-9.]+)",
     lambda m: ("ntt_common", _dims_key(m.group(2), m.group(1)), float(m.group(3)))),
    (r"ntt_common\((\d+),\s*(\d+)\)\s*-\s*latency:([0-9.]+)",
     lambda m: ("ntt_common", _dims_key(m.group(2), m.group(1)), float(m.group(3)))),
    (r"basis_convert\((\d+),\s*(\d+)\)\s*-\s*latency:([0-9.]+)",
     lambda m: ("basis_convert", _dims_key(m.group(1), m.group(2), DEGREE), float(m.group(3)))),
)


def parse_latency_log(log_text: str) -> Dict[Tuple[str, str], float]:
    """tabIX.py:362-396: {(kernel, dims key): latency} from the latency lines
    of a log; a later line for the same key wins."""
    latencies: Dict[Tuple[str, str], float] = {}
    for pattern, build in _PATTERNS:
        for m in re.finditer(pattern, log_text):
            kernel, key, latency = build(m)
            latencies[(kernel, _normalize_dims(f"({key})"))] = latency
    return latencies


def latency_line(kernel: str, dims: Tuple[int, ...], latency_us: float) -> str:
    """One latency line in the reference's print format (tabIX.py:205,244,283,
    315,354), the latency in fixed-point microseconds (the log parser reads no
    exponents)."""
    lat = f"{latency_us:.4f}"
    if kernel == "ntt_common":
        return f"ntt_common({dims[1]},{dims[0]}) - latency:{lat}"
    if kernel == "basis_convert":
        return f"basis_convert({dims[0]},{dims[1]}) - latency:{lat}"
    return f"{kernel}({dims[0]},{dims[1]}) - latency:{lat}"


def _weighted(log_text: str, rows: Optional[List[Row]] = None) -> Tuple[Dict[str, float], float]:
    latencies = parse_latency_log(log_text)
    totals: Dict[str, float] = {}
    overall = 0.0
    for kernel, dims, count in (rows if rows is not None else invocations()):
        key = _normalize_dims(_dims_key(*dims))
        latency = latencies.get((kernel, key))
        if latency is None:
            continue
        # tabIX.py:612-615: the single-modulus NTT row is counted once
        part = latency if (kernel == "ntt_common" and key == f"1,{DEGREE}") else latency * count
        totals[kernel] = totals.get(kernel, 0.0) + part
        overall += part
    return totals, overall


def accumulate_latency_from_log(log_text: str, rows: Optional[List[Row]] = None) -> float:
    """tabIX.py:582-617: sum over the schedule of latency x invocation count
    (rows without a latency line are skipped)."""
    return _weighted(log_text, rows)[1]


def latency_ratios(log_text: str, rows: Optional[List[Row]] = None) -> Dict[str, float]:
    """tabIX.py:620-649: the share (percent) of each kernel type in the
    accumulated latency."""
    totals, overall = _weighted(log_text, rows)
    return {k: 100.0 * totals[k] / overall for k in KERNELS if k in totals and overall > 0}


def print_latency_ratios(log_text: str) -> None:
    """tabIX.py:620-649."""
    ratios = latency_ratios(log_text)
    print("\nLatency Ratios by Kernel Type:")
    print("-" * 30)
    for k in KERNELS:
        if k in ratios:
            print(f"{k:<15}: {ratios[k]:6.2f}%")
    print("-" * 30)


def default_moduli(count: int = 53) -> List[int]:
    """28-bit NTT primes for N = 2^16 (util.find_moduli_ntt), enough for the
    largest row of the schedule (53 limbs)."""
    from . import util
    return list(util.find_moduli_ntt(count, 28, 2 * DEGREE))


def schedule_order(rows: List[Row]) -> List[Tuple[str, Tuple[int, ...]]]:
    """The distinct (kernel, dims) of ``rows`` in measuring order: the NTT rows
    first in decreasing L (one context serves them all, shortened limb by
    limb), then the others in table order."""
    order = list(dict.fromkeys((k, d) for k, d, _ in rows))
    order.sort(key=lambda kd: (kd[0] != "ntt_common", -kd[1][0] if kd[0] == "ntt_common" else 0))
    return order


class Case:
    """One row's operands on the device: ``sets`` copies of the inputs and
    outputs, ``call(i)`` launching the kernel on copy i, and
    ``to_reference`` mapping a host copy of an operand to the reference's
    layout."""

    def __init__(self, inputs: List, outputs: List, call: Callable[[int], None],
                 to_reference: Callable[[np.ndarray], np.ndarray]):
        self.inputs, self.outputs, self.call, self.to_reference = inputs, outputs, call, to_reference
        self.sets = len(outputs)


class KernelMix:
    """The kernels of the schedule on the current CUDA device, through the
    library's C ABI on device-resident operands.

    moduli: the basis (at least 53 primes for the full schedule);
    batch: polynomials per call (latencies are reported per polynomial);
    layout: "native", the library's limb-major layout that its HE chains keep
    on the device, or "reference", the reference's limbs-last layout
    (the NTT and the basis conversion then transpose on the way in and out)."""

    def __init__(self, moduli: Optional[Sequence[int]] = None, batch: int = 1, seed: int = 0,
                 layout: str = "native"):
        if layout not in ("native", "reference"):
            raise ValueError(f"layout must be 'native' or 'reference', got {layout!r}")
        self.layout = layout
        import torch
        from . import _lib
        if not torch.cuda.is_available():
            raise RuntimeError("KernelMix needs a CUDA device")
        self.torch, self._lib = torch, _lib
        self.lib = _lib.lib()
        self.q = list(moduli) if moduli is not None else default_moduli()
        self.batch = batch
        self.seed = seed
        self.dev = torch.device("cuda", torch.cuda.current_device())
        self._ntt = None            # Montgomery context, dropped limb by limb
        self._ntt_sm = None
        self._auto_map = None
        self._ws = None

    # -- operands ---------------------------------------------------------
    def _residues(self, shape: Tuple[int, ...], q: Sequence[int], limb_axis: int, salt: int):
        rng = np.random.default_rng([self.seed, salt])
        qa = np.array(q, np.uint64).reshape([-1 if a == limb_axis % len(shape) else 1 for a in range(len(shape))])
        return (rng.integers(0, 2 ** 62, size=shape, dtype=np.uint64) % qa).astype(np.uint32)

    def _sets(self, per_set_bytes: int, sets: Optional[int]) -> int:
        if sets is not None:
            return sets
        return max(1, math.ceil(1.25 * L2_BYTES / max(per_set_bytes, 1)))

    def _copies(self, host: np.ndarray, sets: int) -> List:
        t = self.torch.from_numpy(host).to(self.dev)
        return [t] + [t.clone() for _ in range(sets - 1)]

    def _workspace(self, nbytes: int):
        if self._ws is None or self._ws.numel() < nbytes:
            self._ws = self.torch.empty(max(nbytes, 1), dtype=self.torch.uint8, device=self.dev)
        return self._ws

    def case(self, kernel: str, dims: Tuple[int, ...], sets: Optional[int] = None) -> Case:
        """The operands and the launch of one row.  ``Case.to_reference``
        maps an operand or result of this layout to the reference's
        (limbs last; add.jax_add's (elements, limbs, N) for add)."""
        torch, L_, lib, B, N = self.torch, self._lib, self.lib, self.batch, DEGREE
        stream = lambda: torch.cuda.current_stream().cuda_stream  # noqa: E731
        salt = zlib.crc32(f"{kernel}{tuple(dims)}".encode())
        native = self.layout == "native"
        empty = lambda shape, n: [torch.empty(shape, dtype=torch.uint32, device=self.dev) for _ in range(n)]  # noqa: E731
        ident = lambda a: a  # noqa: E731
        if kernel in ("add", "mult"):
            # element-wise: one layout serves both (add.jax_add's (elements,
            # limbs, N); the modular multiply's (rows, limbs))
            from . import finite_field
            L = dims[0]
            ff = finite_field.BarrettContext(self.q[:L])
            h = ff.handle()
            shape = (B, L, N) if kernel == "add" else (B * N, L)
            n = self._sets(3 * 4 * B * N * L, sets)
            a = self._copies(self._residues(shape, self.q[:L], 1, salt), n)
            b = self._copies(self._residues(shape, self.q[:L], 1, salt + 1), n)
            out = empty(shape, n)
            if kernel == "add":
                def call(i):
                    L_.check(lib.cross_add_mod(h, a[i].data_ptr(), b[i].data_ptr(), out[i].data_ptr(), B, N,
                                               stream()), "cross_add_mod")
            else:
                def call(i):
                    L_.check(lib.cross_modmul(h, a[i].data_ptr(), 0, b[i].data_ptr(), 0, B * N, out[i].data_ptr(),
                                              B * N, stream()), "cross_modmul")
            cs = Case([a, b], out, call, ident)
            cs.ctx = ff
            return cs
        if kernel == "automorph":
            from . import util
            L = dims[0]
            if self._auto_map is None:
                # tabIX.py:126: the map of automorphism index
                # find_automorphism_index_2n_complex(1, 65536) over N = 2^16
                k = util.find_automorphism_index_2n_complex(1, DEGREE)
                m = np.asarray(util.precompute_auto_map(DEGREE, k), np.int32)
                self._auto_map = torch.from_numpy(m).to(self.dev)
            cmap = self._auto_map
            n = self._sets(2 * 4 * B * N * L, sets)
            # native: every limb row (B, L, N) permuted as a one-limb polynomial
            shape, axis, polys, limbs = ((B, L, N), 1, B * L, 1) if native else ((B, N, L), 2, B, L)
            x = self._copies(self._residues(shape, self.q[:L], axis, salt), n)
            out = empty(shape, n)

            def call(i):
                L_.check(lib.cross_automorphism(x[i].data_ptr(), cmap.data_ptr(), out[i].data_ptr(), polys, N,
                                                limbs, stream()), "cross_automorphism")
            cs = Case([x], out, call, (lambda a: np.moveaxis(a, 1, 2)) if native else ident)
            cs.coef_map = cmap
            return cs
        if kernel == "ntt_common":
            L = dims[0]
            plan = self._ntt_plan(L)
            n = self._sets(2 * 4 * B * N * L, sets)
            lay = L_.LAYOUT_LIMB_MAJOR if native else L_.LAYOUT_REFERENCE
            shape, axis = ((B, L, R, C), 1) if native else ((B, R, C, L), 3)
            x = self._copies(self._residues(shape, self.q[:L], axis, salt), n)
            out = empty(shape, n)
            ws = self._workspace(lib.cross_ntt_workspace_size(plan, B, lay))

            def call(i):
                L_.check(lib.cross_ntt(plan, 0, x[i].data_ptr(), out[i].data_ptr(), B, lay, ws.data_ptr(),
                                       ws.numel(), stream()), "cross_ntt")
            cs = Case([x], out, call, (lambda a: np.moveaxis(a, 1, 3)) if native else ident)
            cs.ctx = self._ntt_sm if L == 1 else self._ntt
            return cs
        if kernel == "basis_convert":
            from . import bconv
            a, b_ = dims[0], dims[1]
            bc = bconv.BConvBarrett(self.q[:a + b_])
            bc.control_gen([(list(range(a)), list(range(a, a + b_)))])
            plan = bc.plan(0)
            n = self._sets(4 * B * N * (a + b_), sets)
            lay = L_.LAYOUT_LIMB_MAJOR if native else L_.LAYOUT_REFERENCE
            (si, so), axis = (((B, a, N), (B, b_, N)), 1) if native else (((B, N, a), (B, N, b_)), 2)
            x = self._copies(self._residues(si, self.q[:a], axis, salt), n)
            out = empty(so, n)

            def call(i):
                L_.check(lib.cross_bconv(plan, 1, x[i].data_ptr(), out[i].data_ptr(), B, N, lay, stream()),
                         "cross_bconv")
            cs = Case([x], out, call, (lambda t: np.moveaxis(t, 1, 2)) if native else ident)
            cs.ctx = bc
            return cs
        raise ValueError(f"unknown kernel {kernel!r}")

    def _ntt_plan(self, L: int):
        """The Montgomery NTT plan over the first L moduli.  One context is
        built at the largest L asked for and shortened with drop_last_modulus
        (ntt_mm.py:412-419), so rows are cheapest in decreasing L."""
        from . import finite_field, ntt_mm, ntt_sm
        if L == 1:
            if self._ntt_sm is None:
                q0 = int(self.q[0])
                self._ntt_sm = ntt_sm.NTTMontgomeryContext(
                    q0, {"r": R, "c": C, "finite_field_context": finite_field.MontgomeryContext(q0)})
            return self._ntt_sm._mm.plan()
        if self._ntt is None or self._ntt.ntt_tf_step2.shape[-1] < L:
            q = self.q[:L]
            self._ntt = ntt_mm.NTTCiphertextMontgomeryContext(
                q, {"r": R, "c": C, "finite_field_context": finite_field.MontgomeryContext(q)})
        while self._ntt.ntt_tf_step2.shape[-1] > L:
            self._ntt.drop_last_modulus()
        return self._ntt.plan()

    # -- timing -----------------------------------------------------------
    # queued timing: calls per chunk, and the spin that holds the stream while
    # a chunk is issued (about 8 ms at 2 GHz; the host issues 128 calls in a
    # few ms)
    CHUNK = 128
    HOLD_CYCLES = 16_000_000

    def time_case(self, cs: Case, reps: int = 20, warmup: int = 2, queued: bool = True) -> float:
        """Microseconds per polynomial over ``max(reps, cs.sets)`` calls that
        cycle through the case's operand copies (at least one pass over all),
        from CUDA events on the current stream.

        queued: the device time of the calls run back to back -- every chunk of
        calls is issued while a spin kernel holds the stream, so the events
        bracket the kernels alone, not the host's issue rate (the quantity
        tabIX.py reads from the device trace).  Otherwise the calls are timed
        as the host issues them, one after another."""
        torch = self.torch
        for i in range(warmup):
            cs.call(i % cs.sets)
        reps = max(reps, cs.sets)
        st = torch.cuda.current_stream()
        torch.cuda.synchronize()
        pairs = []
        step = self.CHUNK if queued else reps
        for c0 in range(0, reps, step):
            if queued:
                torch.cuda._sleep(self.HOLD_CYCLES)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            for i in range(c0, min(c0 + step, reps)):
                cs.call(i % cs.sets)
            e1.record(st)
            pairs.append((e0, e1))
        torch.cuda.synchronize()
        return 1000.0 * sum(a.elapsed_time(b) for a, b in pairs) / reps / self.batch

    def measure(self, rows: Optional[List[Row]] = None, reps: int = 20,
                log: Optional[Callable[[str], None]] = None) -> str:
        """Time every distinct (kernel, dims) of ``rows`` (the whole schedule by
        default) and return the latency log in the reference's format."""
        lines = []
        for kernel, dims in schedule_order(rows if rows is not None else invocations()):
            cs = self.case(kernel, dims)
            us = self.time_case(cs, reps)
            line = latency_line(kernel, dims, us)
            lines.append(line)
            if log:
                log(line)
            del cs
        for ctx in (self._ntt, self._ntt_sm):
            if ctx is not None:
                ctx.check_device()
        return "\n".join(lines) + "\n"


def summary(log_text: str, rows: Optional[List[Row]] = None) -> Dict[str, object]:
    """Accumulated latency (us) and per-kernel totals and shares of a log."""
    totals, overall = _weighted(log_text, rows)
    return {"total_us": overall, "by_kernel_us": totals,
            "ratios_pct": {k: 100.0 * v / overall for k, v in totals.items()} if overall else {}}
