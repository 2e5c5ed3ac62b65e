"""Benchmark: CKKS HE-Mult (with its input rescale) and relinearisation at N = 2^16.

Workload (one step): HEMul.mul (hemul.py:153-217: rescale of the inputs,
tensor product, hybrid key switch, ModDown) over the box-scale batch of 512
ciphertexts with N = 2^16 (256 x 256), L = 35 limbs of 28-bit NTT primes,
K = 7 special limbs, dnum = 5; seeded uniform residues; evaluation keys
seeded uniform.  The 512 ciphertexts are split across the ranks (512 / N per
GPU, strong scaling); ciphertexts are independent, so ranks exchange nothing
on the data path (the reference shards the batch axis only, util.py:40-58).
Each rank runs its share in calls of 64 ciphertexts.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Prints one JSON line on rank 0.  On one GPU the line also carries the other
configurations of the scope (key "configs"): the N = 2^12 NTT + INTT, the
24 -> 25 limb BConv, HE-Mult and HE-Rotate at L = 24, K = 8, dnum = 3 with 64
ciphertexts, each with its own roofline.  Other workloads of the same line
format:
  --workload herot              HE-Rotate (B, 2, r, c, L) -> (B, 2, N, L)
  --limbs L --special K --dnum D --global-batch B
                                another HE-Mult / HE-Rotate point (24, 8, 3, 64: one GPU's
                                L = 24 benchmark point)
  --workload ntt / bconv        the transform or the basis conversion alone for one reduction
                                (--reduction barrett | montgomery | shoup | bat_lazy): NTT + INTT
                                over --ntt-limbs limbs x --ntt-polys polys of N = --ntt-degree
                                (default 2^16, 24, 16); BConv 24 -> 25 limbs, 32 polys of N = 2^16
  --workload i8peak             the int8 tensor-core probe alone (burst and sustained)
  --workload ckks               a CKKS encode -> encrypt -> decrypt -> decode round trip
  --workload bts                the bootstrapping kernel mix: every (kernel, size) of a CKKS
                                bootstrapping's schedule timed, latencies weighted by invocation
                                counts (us per polynomial, lower is better)
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from dataclasses import dataclass

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

N_DEG, R, C = 65536, 256, 256
# DRAM bytes (read + write) of one k_bat_tc2 launch of the roofline NTT per
# limb-polynomial it processes, from an ncu capture of the same launches at
# 64 polys x 34 limbs (1222.7 MB and 1195.4 MB for the two stages; traffic
# grows with the limb-polynomials processed).
TRAFFIC_PER_LP = (1222.7e6 + 1195.4e6) / 2 / (64 * 34)
L2_BYTES = 126 * 2 ** 20                # B200 L2


@dataclass
class Point:
    """An HE operator configuration: operator, limbs, special limbs, digits,
    ciphertexts per step over all ranks, ciphertexts per call."""
    workload: str = "hemul"
    L: int = 35
    K: int = 7
    dnum: int = 5
    global_batch: int = 512
    call_batch: int = 64

    @property
    def metric(self):
        op = "HE-Rotate/s" if self.workload == "herot" else "HE-Mult/s"
        return f"{op} (N=2^16, L={self.L}, K={self.K}, dnum={self.dnum})"

    @property
    def unit(self):
        return "HE-Rot/s" if self.workload == "herot" else "HE-Mult/s"

    def describe(self, per_gpu):
        op = ("CKKS HE-Rotate (hybrid key switch)" if self.workload == "herot" else
              "CKKS HE-Mult with input rescale + relinearisation")
        return (f"{op}, N=2^16 (256x256), L={self.L} x 28-bit, K={self.K}, dnum={self.dnum}, "
                f"{self.global_batch} ciphertexts per step ({per_gpu} per GPU, calls of {self.call_batch})")

    def transforms_per_ct(self):
        """Limb-transforms of one ciphertext (rescale, key switch, ModDown)."""
        L, K, d = self.L, self.K, self.dnum
        if self.workload == "herot":
            alpha = -(-L // d)
            parts = [min(alpha, L - j * alpha) for j in range(d)]
            return L + sum(L + K - a for a in parts) + 2 * K + 2 * L
        L1 = L - 1
        alpha = -(-L1 // d)
        parts = [min(alpha, L1 - j * alpha) for j in range(-(-L1 // alpha))]
        return 4 + 4 * L1 + L1 + sum(L1 + K - a for a in parts) + 2 * K + 2 * L1

    def int8_ops_per_ct(self):
        """Algorithmic int8 operations of one ciphertext: 32 N (R + C) per
        limb-transform plus 2 N (4 sq)(4 sp) per basis conversion."""
        L, K, d, n = self.L, self.K, self.dnum, N_DEG
        ops = self.transforms_per_ct() * 32.0 * n * (R + C)
        if self.workload == "herot":
            alpha = -(-L // d)
            parts = [min(alpha, L - j * alpha) for j in range(d)]
            bc = sum(a * (L + K - a) for a in parts) + 2 * K * L
        else:
            L1 = L - 1
            alpha = -(-L1 // d)
            parts = [min(alpha, L1 - j * alpha) for j in range(-(-L1 // alpha))]
            bc = sum(a * (L1 + K - a) for a in parts) + 2 * K * L1
        return ops + 2.0 * n * 16 * bc


BOX = Point()
L24 = Point(L=24, K=8, dnum=3, global_batch=64)


def rotation_map(seed: int = 0):
    """A seeded rotation index k in [1, N/2) and its coefficient map
    (util.py:652-693)."""
    import numpy as np
    from cross_b200 import util
    k = int(np.random.default_rng(seed).integers(1, N_DEG // 2))
    return k, util.precompute_auto_map(N_DEG, util.find_automorphism_index_2n_complex(k, 2 * N_DEG))


def moduli(pt):
    from cross_b200 import util
    ov = util.find_moduli_ntt(pt.L + pt.K, 28, 2 * N_DEG)
    return ov[:pt.L], ov[pt.L:]


def keys(pt):
    """Seeded uniform evaluation keys (dnum, N, L + K)."""
    import numpy as np
    Q, P = moduli(pt)
    krng = np.random.default_rng(1)
    ov = np.array(Q + P, np.uint64)
    ea = (krng.integers(0, 2 ** 62, size=(pt.dnum, N_DEG, pt.L + pt.K), dtype=np.uint64) % ov).astype(np.uint32)
    eb = (krng.integers(0, 2 ** 62, size=(pt.dnum, N_DEG, pt.L + pt.K), dtype=np.uint64) % ov).astype(np.uint32)
    return ea, eb


def device_residues(torch, shape, mods, seed, dev, axis=-1):
    """Seeded uniform residues below mods[i] along `axis`, drawn on the device."""
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    view = [1] * len(shape)
    view[axis] = len(mods)
    q = torch.tensor(mods, dtype=torch.int64, device=dev).reshape(view)
    out = torch.empty(shape, dtype=torch.int32, device=dev)
    flat = out.view(shape[0], -1)
    for i in range(shape[0]):           # one leading slice at a time bounds the int64 temporary
        x = torch.randint(0, 2 ** 62, (1, *shape[1:]), generator=g, device=dev, dtype=torch.int64)
        flat[i] = (x % q).to(torch.int32).reshape(-1)
    return out.view(torch.uint32)


def host_residues(shape, mods, seed):
    import numpy as np
    rng = np.random.default_rng(seed)
    return (rng.integers(0, 2 ** 62, size=shape, dtype=np.uint64) % np.array(mods, np.uint64)).astype(np.uint32)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons, sampled every 50 ms; summary() keeps
    the samples received inside a host-time window (the timed region)."""
    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.time()
            while not self.rows and time.time() - t0 < 3.0:    # wait for the first sample
                time.sleep(0.02)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append((time.time(), [x.strip() for x in line.split(",")]))

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, t0=None, t1=None):
        sm, mx, pw, reasons = [], None, [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        rows = [r for t, r in self.rows if (t0 is None or t >= t0) and (t1 is None or t <= t1 + 0.06)]
        for r in rows:
            try:
                sm.append(float(r[0]))
                mx = float(r[1])
                pw.append(float(r[2]))
                for n, v in zip(names, r[3:7]):
                    if "Active" in v and "Not" not in v:
                        reasons.add(n)
            except (ValueError, IndexError):
                pass
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "power_w_max": max(pw) if pw else None, "reasons": sorted(reasons), "samples": len(sm)}



def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


_I8 = {}


def i8_probe(torch, dev, sustained_s=3.0, kchunks=8192):
    """The int8 tensor-core peak of this GPU, measured: cross_tc_i8_probe
    launches on every SM, operands resident in shared memory, timed with CUDA
    events on the launching stream.  burst = best of five launches after
    warm-up (the denominator for a kernel timed alone); sustained = launches
    back to back for `sustained_s` seconds (for kernels timed inside a long
    step).  pair = the two-SM cta_group::2 form of the NTT contraction."""
    key = (str(dev), sustained_s)
    if key in _I8:
        return _I8[key]
    from cross_b200 import _lib
    lib = _lib.lib()
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ctas = ctypes.c_int(0)
    st = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def go(pair):
        _lib.check(lib.cross_tc_i8_probe(pair, kchunks, ctypes.c_void_p(err.data_ptr()), ctypes.byref(ctas),
                                         ctypes.c_void_p(st.cuda_stream)), "cross_tc_i8_probe")

    res = {}
    for pair in (1, 0):
        for _ in range(3):
            go(pair)
        torch.cuda.synchronize(dev)
        best = float("inf")
        for _ in range(5):
            e0.record(st)
            go(pair)
            e1.record(st)
            torch.cuda.synchronize(dev)
            best = min(best, e0.elapsed_time(e1))
        ops = ctas.value * kchunks * 2.0 * 128 * 256 * 128
        res[pair] = (ops / (best * 1e-3) / 1e12, best, ops)
    reps = max(3, int(sustained_s * 1e3 / res[1][1]))
    with ClockSampler(dev.index if dev.index is not None else 0) as clk:
        torch.cuda.synchronize(dev)
        h0 = time.time()
        e0.record(st)
        for _ in range(reps):
            go(1)
        e1.record(st)
        torch.cuda.synchronize(dev)
        h1 = time.time()
    sustained = reps * res[1][2] / (e0.elapsed_time(e1) * 1e-3) / 1e12
    if int(err.item()) != 0:
        raise TimeoutError(f"cross_tc_i8_probe: a bounded wait expired (code {int(err.item())})")
    out = {"burst_tops": res[1][0], "sustained_tops": sustained, "burst_tops_1sm": res[0][0],
           "ms_per_launch": res[1][1], "kchunks": kchunks, "sustained_launches": reps,
           "sustained_seconds": e0.elapsed_time(e1) / 1e3, "clocks_sustained": clk.summary(h0, h1),
           "how": "cross_tc_i8_probe: tcgen05.mma kind::i8 M=256 N=256 K=32 (cta_group::2) on shared-memory "
                  "operands on every SM, CUDA events; burst = best of 5 launches, sustained = back to back"}
    _I8[key] = out
    return out


def int8_peak(torch, dev, sustained=False):
    """(TOPS, source) of the int8 roofline denominator: the probe measured in
    this process (burst for a kernel timed alone, sustained for a long step)."""
    p = i8_probe(torch, dev)
    v = p["sustained_tops"] if sustained else p["burst_tops"]
    return v, (f"int8 tensor-core peak measured in this run ({'sustained' if sustained else 'burst'}): "
               f"{p['how']}")


def _oracle_op(pt):
    """The oracle's operator for one ciphertext of the workload and its input."""
    from oracle import cross_oracle as O
    Q, P = moduli(pt)
    ea, eb = keys(pt)
    ct = host_residues((1, 4 if pt.workload == "hemul" else 2, R, C, pt.L), Q, seed=0)
    if pt.workload == "herot":
        op = O.HERot(R, C, pt.dnum, Q, P)
        op.control_gen(1)
        op.setup_rotate(ea.reshape(pt.dnum, R, C, -1), eb.reshape(pt.dnum, R, C, -1), rotation_map()[1])
        return op.rotate, ct, "HERot.rotate"
    he = O.HEMul(1, R, C, pt.dnum, 1, Q, P)
    he.setup_relinearization(ea, eb)
    return he.mul, ct, "HEMul.mul"


def cpu_baseline(pt, steps=2):
    """The oracle (numpy restatement of jaxite_word) on the host cores: one
    ciphertext per step, the median of `steps`."""
    fn, ct, name = _oracle_op(pt)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        fn(ct)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": 1.0 / t, "unit": pt.unit, "cores": os.cpu_count(), "kind": "port",
            "sample": f"{steps} x 1 ciphertext of the workload (oracle/cross_oracle.py {name}, numpy BLAS threads; "
                      f"median {t:.2f} s per ciphertext)"}


def run_reference(args, pt):
    """--impl reference: the oracle port of jaxite_word's operator on the host
    cores (all BLAS threads), W warm-up and K timed steps of one ciphertext."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if args.workload == "bts":
        t0 = time.perf_counter()
        for _ in range(args.warmup + args.steps):
            total, per, sample = bts_oracle_estimate()
        dt = (time.perf_counter() - t0) / max(args.warmup + args.steps, 1)
        print(json.dumps({"impl": "reference", "metric": "CKKS bootstrapping kernel-mix latency (us per polynomial, N=2^16)",
                          "value": total, "unit": "us", "n_gpus": args.gpus, "steps": args.steps,
                          "warmup": args.warmup, "ms_per_step": 1000.0 * dt, "higher_is_better": False,
                          "scaling": "weak", "vs_baseline": None, "dtype": "u32 residues, u64 intermediates",
                          "data": "synthetic seeded", "config": {"workload": "tabIX bootstrapping schedule"},
                          "by_kernel_us": per,
                          "cpu_baseline": {"value": total, "unit": "us", "cores": os.cpu_count(), "kind": "port",
                                           "sample": sample},
                          "e2e": {"value": total, "unit": "us", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
              flush=True)
        return
    fn, ct, name = _oracle_op(pt)
    for _ in range(args.warmup):
        fn(ct)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fn(ct)
    dt = (time.perf_counter() - t0) / max(args.steps, 1)
    v = 1.0 / dt
    sample = f"1 ciphertext of the workload per step (oracle/cross_oracle.py {name}, numpy BLAS threads)"
    print(json.dumps({"impl": "reference", "metric": pt.metric, "value": v, "unit": pt.unit, "n_gpus": args.gpus,
                      "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * dt,
                      "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                      "dtype": "u32 residues, u64 intermediates, u8 BAT contractions", "data": "synthetic seeded",
                      "config": {"workload": pt.describe(pt.global_batch // max(args.gpus, 1)),
                                 "sample": "1 ciphertext per step"},
                      "cpu_baseline": {"value": v, "unit": pt.unit, "cores": os.cpu_count(), "kind": "port",
                                       "sample": sample},
                      "e2e": {"value": v, "unit": pt.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
          flush=True)


class _Timer:
    """CUDA-event timing of `steps` calls on the current stream, max over ranks."""

    def __init__(self, torch, dist, dev):
        self.torch, self.dist, self.dev = torch, dist, dev

    def __call__(self, fn, steps):
        from cross_b200 import shard
        t = self.torch
        t.cuda.synchronize()
        if self.dist:
            self.dist.barrier()
        e0, e1 = t.cuda.Event(enable_timing=True), t.cuda.Event(enable_timing=True)
        st = t.cuda.current_stream()
        e0.record(st)
        for _ in range(steps):
            fn()
        e1.record(st)
        t.cuda.synchronize()
        return shard.max_over_ranks(e0.elapsed_time(e1), device=self.dev)


def measure_component(workload, torch, dist, world, rank, local, steps, warmup, reduction="barrett",
                      ntt_limbs=24, ntt_polys=16, ntt_degree=N_DEG, cpu=True, e2e=True):
    """--workload ntt | bconv for one reduction: device throughput, end-to-end
    throughput through the operator API with host buffers, the kernel's
    roofline and the oracle on the host cores.  Returns the JSON line."""
    import numpy as np
    from cross_b200 import _lib, bconv, ntt_mm, util
    from oracle import cross_oracle as O
    from oracle import variants as V
    dev = torch.device("cuda", local)
    timer = _Timer(torch, dist, dev)
    lib = _lib.lib()
    red = reduction
    pk, src = peaks()
    rng = np.random.default_rng(200 + rank)
    if workload == "ntt":
        Lw, B, nd = ntt_limbs, ntt_polys, ntt_degree
        rr, cc = util.default_rc(nd)
        q = O.find_moduli_ntt(Lw, 28, 2 * nd)
        cls = {"barrett": ntt_mm.NTTCiphertextBarrettContext, "montgomery": ntt_mm.NTTCiphertextMontgomeryContext,
               "shoup": ntt_mm.NTTCiphertextShoupContext, "bat_lazy": ntt_mm.NTTCiphertextBATLazyContext}[red]
        ctx = cls(q, {"r": rr, "c": cc})
        xh = (rng.integers(0, 2 ** 62, size=(B, Lw, rr, cc), dtype=np.uint64) %
              np.array(q, np.uint64)[:, None, None]).astype(np.uint32)
        x = torch.from_numpy(xh).to(dev)
        # a configuration smaller than L2 cycles through enough copies of its
        # input (> 1.25 x L2 in all) that every timed step reads cold data
        nsets = max(1, -(-int(1.25 * L2_BYTES) // (2 * x.numel() * 4))) if x.numel() * 4 < L2_BYTES else 1
        xs = [x] + [x.clone() for _ in range(nsets - 1)]
        ys = [torch.empty_like(x) for _ in range(nsets)]
        y = ys[0]
        ws = torch.empty(lib.cross_ntt_workspace_size(ctx.plan(), B, _lib.LAYOUT_LIMB_MAJOR), dtype=torch.uint8,
                         device=dev)
        ctr = [0]

        def step():
            cs = torch.cuda.current_stream().cuda_stream
            k = ctr[0] % nsets
            ctr[0] += 1
            for inv, a, b in ((0, xs[k], ys[k]), (1, ys[k], ys[k])):
                _lib.check(lib.cross_ntt(ctx.plan(), inv, a.data_ptr(), b.data_ptr(), B, _lib.LAYOUT_LIMB_MAJOR,
                                         ws.data_ptr(), ws.numel(), cs), "cross_ntt")
        units = 2 * B * Lw                                   # limb-transforms per step
        metric, unit = f"NTT+INTT limb-transforms/s (N={nd}, {red})", "limb-transform/s"
        wl = f"BAT NTT then INTT, {red} reduction, N={nd} ({rr}x{cc}), {Lw} limbs x {B} polys per GPU"
        hin = torch.from_numpy(np.ascontiguousarray(xh.transpose(0, 2, 3, 1))).pin_memory()   # (B, R, C, L)

        def e2e_step():
            out = ctx.intt(ctx.ntt(hin))
            return out.cpu()
        sample_x = np.ascontiguousarray(xh[:1].transpose(0, 2, 3, 1))

        def cpu_once():
            ref = O.NTTBarrett(q, rr, cc) if red == "barrett" else V.NTTVariant(q, rr, cc, red)
            t0 = time.perf_counter()
            ref.intt(ref.ntt(sample_x))
            return time.perf_counter() - t0
        cpu_units = 2 * Lw
        if red == "shoup":
            # CUDA cores: per limb-transform 2 N (R + C) multiply-adds (the sum and
            # its Shoup companion over both stages)
            ops = units * 2.0 * nd * (rr + cc)
            nominal = 148 * 128 * 1.965e9 / 1e12
            roof = {"bound": "cuda-core int32 issue", "unit": "TMAC/s", "peak": nominal,
                    "peak_source": "nominal 148 SMs x 128 int32 lanes x 1965 MHz (no measured figure on this pool)"}
        else:
            ops = units * 32.0 * nd * (rr + cc)
            # HBM bound as well: 8 N bytes per limb-transform (read + write)
            hbm_s = units * 8.0 * nd / (pk["hbm_gbs"] * 1e9)
            pv, ps = int8_peak(torch, dev)
            roof = {"bound": "tensor", "unit": "TOPS (int8)", "peak": pv, "peak_source": ps,
                    "hbm_bound_ms_per_step": 1e3 * hbm_s, "hbm_peak_source": f"hbm_gbs of MEASURED_PEAKS.json ({src})"}
        roof["kernel"] = "all launches of one NTT + INTT"
    else:
        sq, sp, B = 24, 25, 32
        ov = O.find_moduli_ntt(sq + sp, 28, 2 * N_DEG)
        cls = {"barrett": bconv.BConvBarrett, "montgomery": bconv.BConvMontgomery, "shoup": bconv.BConvShoup,
               "bat_lazy": bconv.BConvBATLazy}[red]
        bc = cls(ov)
        bc.control_gen([(list(range(sq)), list(range(sq, sq + sp)))])
        bat = red != "shoup"
        xh = (rng.integers(0, 2 ** 62, size=(B, sq, N_DEG), dtype=np.uint64) %
              np.array(ov[:sq], np.uint64)[:, None]).astype(np.uint32)
        x = torch.from_numpy(xh).to(dev)
        ob = lib.cross_bconv_output_bytes(bc.plan(0))
        y = torch.empty((B, sp, N_DEG), dtype=torch.uint64 if ob == 8 else torch.uint32, device=dev)

        def step():
            cs = torch.cuda.current_stream().cuda_stream
            _lib.check(lib.cross_bconv_ex(bc.plan(0), int(bat), x.data_ptr(), y.data_ptr(), B, N_DEG,
                                          _lib.LAYOUT_LIMB_MAJOR, cs), "cross_bconv_ex")
        units = B
        metric, unit = f"BConv polys/s (N=2^16, 24->25 limbs, {red})", "poly/s"
        wl = (f"basis conversion {'basis_change_bat' if bat else 'basis_change'}, {red}, 24 -> 25 limbs, "
              f"N=2^16, 32 polys per GPU")
        hin = torch.from_numpy(np.ascontiguousarray(xh.transpose(0, 2, 1))).pin_memory()      # (B, N, sq)

        def e2e_step():
            out = bc.basis_change_bat(hin) if bat else bc.basis_change(hin)
            return out.cpu()
        sample_x = np.ascontiguousarray(xh[:1].transpose(0, 2, 1))

        def cpu_once():
            ref = O.BConvBarrett(ov) if red == "barrett" else V.BConvVariant(ov, red)
            ref.control_gen([(list(range(sq)), list(range(sq, sq + sp)))])
            t0 = time.perf_counter()
            ref.basis_change_bat(sample_x) if bat else ref.basis_change(sample_x)
            return time.perf_counter() - t0
        cpu_units = 1
        ops = units * (sq * 4 + sp * ob) * N_DEG
        roof = {"bound": "hbm", "unit": "GB/s", "peak": pk["hbm_gbs"],
                "peak_source": f"hbm_gbs of MEASURED_PEAKS.json ({src})",
                "kernel": "k_bconv_tc (Barrett) / k_bconv_var (variants), one launch per step"}
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    l0 = lib.cross_launch_count()
    step()
    torch.cuda.synchronize()
    launches = (lib.cross_launch_count() - l0) * steps
    # the K timed steps captured once in a CUDA graph and replayed: device time
    # without the host's per-call issue cost (one step of the N = 2^12
    # transform is a few microseconds)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, capture_error_mode="relaxed"):
        for _ in range(steps):
            step()
    graph.replay()
    flush = torch.empty(int(2 * L2_BYTES) // 4, dtype=torch.int32, device=dev)
    flush.fill_(1)                       # evict L2 before the timed replay
    ms = timer(graph.replay, 1)
    del flush
    value = world * units * steps / (ms / 1000.0)
    line = {"metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": ms / steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u32 residues, u64 intermediates",
            "data": "synthetic seeded uniform residues",
            "config": {"workload": wl, "reduction": red,
                       "l2": "inputs larger than L2" if x.numel() * 4 > L2_BYTES else
                             "each timed step on its own copy of the input (copies > 1.25 x L2 in all; L2 "
                             "flushed before the timed replay)",
                       "timing": "K steps captured in one CUDA graph, replayed once between CUDA events"},
            "gpu_launches": int(launches)}
    if e2e:
        e2e_step()
        ems = timer(e2e_step, steps)
        line["e2e"] = {"value": world * units * steps / (ems / 1000.0), "unit": unit,
                       "h2d_bytes_per_step": int(hin.numel() * 4),
                       "d2h_bytes_per_step": int(y.numel() * y.element_size())}
    per = ms / steps / 1000.0
    achieved = ops / per / (1e12 if roof["unit"] != "GB/s" else 1e9)
    roof.update({"achieved": achieved, "frac": achieved / roof["peak"], "traffic": None,
                 "ms_per_step": ms / steps})
    if "hbm_bound_ms_per_step" in roof:
        roof["frac_of_hbm_bound"] = roof["hbm_bound_ms_per_step"] / (ms / steps)
    line["roofline"] = roof
    if cpu and rank == 0 and world == 1:
        dt = cpu_once()
        line["cpu_baseline"] = {"value": cpu_units / dt, "unit": unit, "cores": os.cpu_count(), "kind": "port",
                                "sample": f"{cpu_units} units of the workload (oracle, numpy BLAS threads)"}
    return line


def run_component(args, torch, dist, world, rank, local):
    line = measure_component(args.workload, torch, dist, world, rank, local, args.steps, args.warmup,
                             args.reduction, args.ntt_limbs, args.ntt_polys, args.ntt_degree,
                             cpu=not args.no_cpu_baseline)
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_i8peak(args, torch, dist, world, rank, local):
    dev = torch.device("cuda", local)
    p = i8_probe(torch, dev, sustained_s=4.0)
    if rank == 0:
        print(json.dumps({"metric": "int8 tensor-core peak (TOPS)", "value": p["burst_tops"], "unit": "TOPS",
                          "n_gpus": world, "higher_is_better": True, "probe": p}), flush=True)

# Algorithmic work per polynomial of each kernel of the bootstrapping mix:
# HBM bytes for the element-wise kernels and the permutation, int8 tensor
# operations for the transform and the basis conversion (the same per-limb
# counts as the NTT and BConv configurations).
def _bts_work(kernel, dims):
    n = N_DEG
    if kernel in ("add", "mult"):
        return "hbm", 3 * 4 * n * dims[0]
    if kernel == "automorph":
        return "hbm", 2 * 4 * n * dims[0]
    if kernel == "ntt_common":
        return "tensor", 32.0 * n * (R + C) * dims[0]
    return "tensor", 2.0 * n * (4 * dims[0]) * (4 * dims[1])


def bts_oracle_estimate():
    """The oracle's latency for the bootstrapping mix on the host cores, from a
    bounded sample: one row of each kernel type timed (add 30, mult 30,
    automorph 30 limbs, ntt_common 10 limbs, basis_convert 10 -> 30), every
    row of the schedule scaled from its type's sample by limbs (a x b for the
    basis conversion).  Returns (total us, per-type us, sample text)."""
    import numpy as np
    from cross_b200 import bts_mix, util
    from oracle import cross_oracle as O
    from oracle import variants as V
    q = bts_mix.default_moduli()
    rng = np.random.default_rng(7)

    def res(shape, mods, axis):
        qa = np.array(mods, np.uint64).reshape([-1 if a == axis else 1 for a in range(len(shape))])
        return (rng.integers(0, 2 ** 62, size=shape, dtype=np.uint64) % qa).astype(np.uint32)
    cmap = np.asarray(util.precompute_auto_map(N_DEG, util.find_automorphism_index_2n_complex(1, N_DEG)), np.int64)
    ntt = V.NTTVariant(q[:10], R, C, "montgomery")
    bc = O.BConvBarrett(q[:40])
    bc.control_gen([(list(range(10)), list(range(10, 40)))])
    a30, b30 = res((1, 30, N_DEG), q[:30], 1), res((1, 30, N_DEG), q[:30], 1)
    m30, n30 = res((N_DEG, 30), q[:30], 1), res((N_DEG, 30), q[:30], 1)
    x10, xb = res((1, R, C, 10), q[:10], 3), res((1, N_DEG, 10), q[:10], 2)
    bar = O.Barrett(q[:30])
    samples = {
        "add": (30, lambda: O.jax_add(a30, b30, q[:30])),
        "mult": (30, lambda: bar.reduce(m30.astype(np.uint64) * n30)),
        "automorph": (30, lambda: m30[None][:, cmap, :]),
        "ntt_common": (10, lambda: ntt.ntt(x10)),
        "basis_convert": (300, lambda: bc.basis_change_bat(xb)),
    }
    per_unit = {}
    for k, (units, fn) in samples.items():
        fn()
        t0 = time.perf_counter()
        fn()
        per_unit[k] = (time.perf_counter() - t0) * 1e6 / units
    totals, total = {}, 0.0
    for kernel, dims, count in bts_mix.invocations():
        units = dims[0] * dims[1] if kernel == "basis_convert" else dims[0]
        lat = per_unit[kernel] * units
        part = lat if (kernel == "ntt_common" and dims[0] == 1) else lat * count
        totals[kernel] = totals.get(kernel, 0.0) + part
        total += part
    return total, totals, ("one row of each kernel type on the oracle (add/mult/automorph 30 limbs, "
                           "Montgomery NTT 10 limbs, BConv 10->30), every schedule row scaled from it by limbs")


def run_bts(args, torch, dist, world, rank, local):
    """--workload bts: the CKKS bootstrapping kernel mix (tabIX.py).  Every
    (kernel, size) of the schedule is timed on device-resident operands with
    CUDA events (W warm-up and max(K, copies) timed calls cycling through
    enough operand copies to defeat L2, run back to back on the device); the
    value is the schedule's accumulated latency per polynomial, max over ranks
    divided by the ranks (each GPU runs its own polynomials, as the
    reference's one per device).  host_issued_total_us is the same sum with
    the calls timed as Python issues them one by one."""
    from cross_b200 import _lib, bts_mix, shard
    dev = torch.device("cuda", local)
    lib = _lib.lib()
    rows = bts_mix.invocations()
    mix = bts_mix.KernelMix(batch=args.bts_batch, seed=rank, layout=args.bts_layout)
    lines, host_lines = [], []
    launches = 0
    logf = open(args.bts_log, "w") if (args.bts_log and rank == 0) else None
    order = bts_mix.schedule_order(rows)
    with ClockSampler(local) as clk:
        h0 = time.time()
        for i, (kernel, dims) in enumerate(order):
            cs = mix.case(kernel, dims)
            l0 = lib.cross_launch_count()
            us = mix.time_case(cs, reps=args.steps, warmup=args.warmup, queued=True)
            timed = max(args.steps, cs.sets)          # time_case's timed calls
            launches += (lib.cross_launch_count() - l0) * timed // (timed + args.warmup)
            host_us = mix.time_case(cs, reps=args.steps, warmup=0, queued=False)
            lines.append(bts_mix.latency_line(kernel, dims, us))
            host_lines.append(bts_mix.latency_line(kernel, dims, host_us))
            if logf:
                logf.write(lines[-1] + "\n")
                logf.flush()
            if rank == 0 and (i + 1) % 40 == 0:
                print(f"bts: {i + 1}/{len(order)} rows, {time.time() - h0:.1f} s", file=sys.stderr, flush=True)
            del cs
        h1 = time.time()
    if logf:
        logf.close()
    for ctx in (mix._ntt, mix._ntt_sm):
        if ctx is not None:
            ctx.check_device()
    log = "\n".join(lines) + "\n"
    summ = bts_mix.summary(log)
    host_total = bts_mix.accumulate_latency_from_log("\n".join(host_lines) + "\n")
    total = shard.max_over_ranks(summ["total_us"], device=dev)
    value = total / world
    lat = bts_mix.parse_latency_log(log)
    pk, src = peaks()
    by_kernel = {}
    for kernel in bts_mix.KERNELS:
        work = t_us = 0.0
        bound = None
        for k, dims, count in rows:
            if k != kernel:
                continue
            bound, w = _bts_work(k, dims)
            c = 1 if (k == "ntt_common" and dims[0] == 1) else count
            work += w * c
            t_us += lat[(k, ",".join(map(str, dims)))] * c
        if bound == "hbm":
            a = work / (t_us * 1e-6) / 1e9
            by_kernel[kernel] = {"bound": "hbm", "achieved": a, "unit": "GB/s", "peak": pk["hbm_gbs"],
                                 "frac": a / pk["hbm_gbs"], "share_pct": summ["ratios_pct"].get(kernel)}
        else:
            a = work / (t_us * 1e-6) / 1e12
            i8, _ = int8_peak(torch, dev)
            by_kernel[kernel] = {"bound": "tensor", "achieved": a, "unit": "TOPS (int8)",
                                 "peak": i8, "frac": a / i8, "share_pct": summ["ratios_pct"].get(kernel)}
    top = max(summ["ratios_pct"], key=summ["ratios_pct"].get)
    roof = dict(by_kernel[top])
    roof.update({"kernel": f"{top} rows of the schedule (count-weighted)", "traffic": None,
                 "peak_source": f"hbm_gbs of MEASURED_PEAKS.json ({src}); {int8_peak(torch, dev)[1]}"})
    line = {"metric": "CKKS bootstrapping kernel-mix latency (us per polynomial, N=2^16)", "value": value,
            "unit": "us", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": value / 1000.0, "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
            "dtype": "u32 residues, u64 intermediates, u8 BAT contractions",
            "data": "synthetic seeded uniform residues",
            "config": {"workload": f"tabIX bootstrapping schedule: {len(rows)} (kernel, size) rows, N=2^16 "
                                   f"(256x256), {args.bts_batch} polynomial(s) per call per GPU",
                       "layout": {"native": "limb-major (the library's on-device layout)",
                                  "reference": "limbs last (the reference's)"}[args.bts_layout],
                       "l2": "each row cycles through operand copies totalling > 1.25 x L2"},
            "by_kernel_us": summ["by_kernel_us"], "ratios_pct": summ["ratios_pct"],
            "timing": "device time of each row's calls run back to back (issued while a spin kernel holds the "
                      "stream), as tabIX.py reads kernel durations from the device trace",
            "host_issued_total_us": host_total,
            "e2e": None,
            "e2e_note": "the mix is defined on device-resident operands (tabIX.py times jitted kernels on device arrays)",
            "gpu_launches": int(launches), "clocks": clk.summary(h0, h1), "roofline": roof,
            "by_kernel_roofline": by_kernel}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        t, per, sample = bts_oracle_estimate()
        line["cpu_baseline"] = {"value": t, "unit": "us", "cores": os.cpu_count(), "kind": "port",
                                "sample": sample, "by_kernel_us": per}
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_ckks(args, torch, dist, world, rank, local):
    """--workload ckks: one CKKS round trip per step at N = 2^16 with 24 towers
    (ckks_ctx.py: encode -> encrypt with fresh noise -> decrypt -> decode of
    N/2 real slots), through the operator API (host slot values in, host
    complex values out)."""
    import math
    import numpy as np
    from cross_b200 import _lib, ckks_ctx, key_gen, util
    dev = torch.device("cuda", local)
    timer = _Timer(torch, dist, dev)
    lib = _lib.lib()
    deg, towers = N_DEG, 24
    mods = util.find_moduli_ntt(32, 28, 2 * deg)
    qt, pt = mods[:towers], mods[towers:]
    kp = key_gen.gen_pke_pair(qt, pt, deg)
    ctx = ckks_ctx.CKKSContext({"degree": deg, "num_slots": deg // 2, "scalingFactor": 2.0 ** 40,
                                "output_scale": 2.0 ** 40, "q_towers": qt, "p_towers": pt, "p": 40,
                                "public_key": kp["public_key"], "secret_key": kp["secret_key"]})
    rng = np.random.default_rng(300 + rank)
    x = [complex(v, 0.0) for v in rng.uniform(-1.0, 1.0, deg // 2)]
    xd = torch.from_numpy(np.array(x, np.complex128)).to(dev)
    res = {}

    def step_dev():
        res["out"] = ctx.decode(ctx.decrypt(ctx.encrypt(ctx.encode(xd))))

    def step_host():
        res["out"] = ctx.decode(ctx.decrypt(ctx.encrypt(ctx.encode(x))))
    for _ in range(args.warmup):
        step_dev()
    err = float(np.max(np.abs(res["out"].real - np.array([v.real for v in x]))))
    if err > 1e-3:
        raise RuntimeError(f"CKKS round trip error {err}")
    ms = timer(step_dev, args.steps)
    l0 = lib.cross_launch_count()
    step_dev()
    torch.cuda.synchronize()
    launches = (lib.cross_launch_count() - l0) * args.steps
    step_host()
    ems = timer(step_host, args.steps)
    value = world * args.steps / (ms / 1000.0)
    e2e = world * args.steps / (ems / 1000.0)
    # forward / inverse negacyclic transforms per step: encode 1, encrypt 3 (v, e0, e1), decrypt 1
    transforms = 5 * towers
    ops = transforms * 32.0 * deg * (R + C)
    i8, i8_src = int8_peak(torch, dev)
    achieved = ops / (ms / args.steps / 1000.0) / 1e12
    line = {"metric": "CKKS encode+encrypt+decrypt+decode round trips/s (N=2^16, 24 towers)", "value": value,
            "unit": "round-trip/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "u32 residues, f64 slot values", "data": "synthetic seeded uniform slot values",
            "config": {"workload": "CKKSContext encode -> encrypt (sampled noise) -> decrypt -> decode, N=2^16, "
                                   "24 x 28-bit towers, scale 2^40, N/2 real slots", "round_trip_max_error": err},
            "e2e": {"value": e2e, "unit": "round-trip/s", "h2d_bytes_per_step": int(deg // 2 * 16),
                    "d2h_bytes_per_step": int(deg // 2 * 16)},
            "gpu_launches": int(launches),
            "roofline": {"bound": "latency (launch- and host-bound chain of small kernels)",
                         "kernel": "the 5 x 24 negacyclic transforms of a step on the tensor cores",
                         "achieved": achieved, "peak": i8, "unit": "TOPS (int8)",
                         "frac": achieved / i8, "traffic": None, "peak_source": i8_src}}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import ckks as K
        from oracle import cross_oracle as O
        d2 = 8192
        m2 = O.find_moduli_ntt(32, 28, 2 * d2)
        q2, p2 = m2[:towers], m2[towers:]
        r2 = np.random.default_rng(1)
        xs = [complex(v, 0.0) for v in r2.uniform(-1.0, 1.0, d2 // 2)]
        s2 = [int(v) for v in r2.integers(0, 2, d2)]
        e2 = [int(v) for v in np.rint(r2.normal(0, 3.19, d2))]
        a2 = [[int(v) for v in r2.integers(0, q, d2)] for q in m2]
        kp2 = K.gen_pke_pair(q2, p2, d2, s2, a2, e2)
        ev = lambda co, q: O.bit_reverse_array(K.ntt_negacyclic([c % q for c in co], q, O.root_of_unity(2 * d2, q)))  # noqa: E731
        t0 = time.perf_counter()
        enc = K.ckks_encode(xs, 2 * d2, q2, 2.0 ** 40)
        v2 = [ev(s2, q) for q in q2]
        ct2 = K.ckks_encrypt(enc, kp2["public_key"], q2, v2, (v2, v2))
        K.decode_rns(O.ckks_decrypt(ct2, kp2["secret_key"], q2), q2, 2.0 ** 40, d2 // 2, 40)
        dt = time.perf_counter() - t0
        scale_n = (deg * math.log2(deg)) / (d2 * math.log2(d2))
        line["cpu_baseline"] = {"value": 1.0 / (dt * scale_n), "unit": "round-trip/s", "cores": 1, "kind": "port",
                                "sample": f"one round trip at N=2^13 with 24 towers on the oracle (pure Python, "
                                          f"{dt:.1f} s), scaled to N=2^16 by N log N (x{scale_n:.2f})"}
    if rank == 0:
        print(json.dumps(line), flush=True)



def copies_alone(torch, dev, hin, hout, units, unit, world):
    """The operator rate that the end-to-end path's host<->device copies alone
    would allow: one call's pinned inputs copied in and outputs copied out,
    H2D alone, D2H alone and both at once on two streams, every rank at the
    same time (CUDA events around each, best of 3 after a warm-up, max over
    ranks).  On one GPU the e2e pipeline approaches it when the compute hides
    under the copies; with several ranks sharing the host's memory and PCIe
    links, whole-call copies contend more than the pipeline's chunks do, so
    the e2e value can exceed it."""
    from cross_b200 import shard
    din = torch.empty(hin.shape, dtype=hin.dtype, device=dev)
    dout = torch.empty(hout.shape, dtype=hout.dtype, device=dev)
    cur = torch.cuda.current_stream(dev)
    s1, s2 = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)

    def best(h2d, d2h):
        times = []
        for _ in range(4):
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(cur)
            s1.wait_stream(cur)
            s2.wait_stream(cur)
            if h2d:
                with torch.cuda.stream(s1):
                    din.copy_(hin, non_blocking=True)
            if d2h:
                with torch.cuda.stream(s2):
                    hout.copy_(dout, non_blocking=True)
            cur.wait_stream(s1)
            cur.wait_stream(s2)
            e1.record(cur)
            torch.cuda.synchronize(dev)
            times.append(e0.elapsed_time(e1))
        return shard.max_over_ranks(min(times[1:]), device=dev)

    h2d_ms, d2h_ms, both_ms = best(True, False), best(False, True), best(True, True)
    bi, bo = hin.numel() * hin.element_size(), hout.numel() * hout.element_size()
    del din, dout
    torch.cuda.empty_cache()
    return {"value": world * units / (both_ms / 1000.0), "unit": unit, "call_units": units,
            "h2d_gbs": bi / h2d_ms / 1e6, "d2h_gbs": bo / d2h_ms / 1e6, "both_ms_per_call": both_ms,
            "note": "pinned host memory, one call's bytes per rank, all ranks at once"}


def measure_he(pt, torch, dist, world, rank, local, steps, warmup, e2e=True, cpu=True, roofline=True, probe=True):
    """One HE operator point: each rank runs its share of pt.global_batch
    ciphertexts (inputs resident in HBM) in calls of pt.call_batch; CUDA events
    around the timed steps, max over ranks.  Returns the JSON line."""
    from cross_b200 import _lib, hemul, herot, ntt_mm, shard
    dev = torch.device("cuda", local)
    lib = _lib.lib()
    lo, hi = shard.shard_bounds(pt.global_batch, world, rank)
    nb = hi - lo
    cb = max(1, min(pt.call_batch, nb))
    Q, P = moduli(pt)
    ea, eb = keys(pt)
    if pt.workload == "herot":
        he = herot.HERot(R, C, pt.dnum, Q, P)
        he.control_gen(batch=cb, degree_layout=(R, C))
        he.setup_rotate(ea, eb, rotation_map()[1])
        E, op, out_shape, tag = 2, he.rotate, (nb, 2, N_DEG, pt.L), "herot"
    else:
        he = hemul.HEMul(cb, R, C, pt.dnum, 1, Q, P)
        he.control_gen(degree_layout=(R, C))
        he.setup_relinearization(ea, eb)
        E, op, out_shape, tag = 4, he.mul, (nb, 2, R, C, pt.L - 1), "hemul"
    del ea, eb
    x = device_residues(torch, (nb, E, R, C, pt.L), Q, 100 + lo, dev)
    out = torch.empty(out_shape, dtype=torch.uint32, device=dev)
    ws = torch.empty(he.workspace_size(cb), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()

    def step():
        torch.cuda.nvtx.range_push(tag)
        for a in range(0, nb, cb):
            b = min(nb, a + cb)
            op(x[a:b], out=out[a:b], workspace=ws)
        torch.cuda.nvtx.range_pop()

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        l0 = lib.cross_launch_count()
        h0 = time.time()
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        h1 = time.time()
        launches = lib.cross_launch_count() - l0
    ms = shard.max_over_ranks(e0.elapsed_time(e1), device=dev)
    he.check_device()
    value = pt.global_batch * steps / (ms / 1000.0)
    if probe:
        sus, sus_src = int8_peak(torch, dev, sustained=True)
    else:
        sus, sus_src = 4500.0, "nominal B200 dense int8 (probe skipped)"
    ops_ct = pt.int8_ops_per_ct()
    per_gpu = value / world
    line = {
        "metric": pt.metric, "value": value, "unit": pt.unit, "n_gpus": world, "steps": steps,
        "warmup": warmup, "ms_per_step": ms / steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "u32 residues, u64 intermediates, u8 BAT contractions",
        "data": "synthetic seeded uniform residues (no dataset in the reference)",
        "config": {"workload": pt.describe(nb), "global_batch": pt.global_batch, "batch_per_gpu": nb,
                   "call_batch": cb, "N": N_DEG, "r": R, "c": C, "L": pt.L, "K": pt.K, "dnum": pt.dnum,
                   "parallelism": f"batch-sharded x{world} (ciphertexts independent, no data-path collective)",
                   "l2": f"inputs {x.numel() * 4 / 1e9:.2f} GB per GPU, larger than L2 (no flush needed)"},
        "gpu_launches": int(launches),
        "clocks": clk.summary(h0, h1),
        "operator_roofline": {"bound": "tensor", "unit": "TOPS (int8)", "int8_ops_per_ct": ops_ct,
                              "limb_transforms_per_ct": pt.transforms_per_ct(),
                              "achieved": per_gpu * ops_ct / 1e12, "peak": sus,
                              "frac": per_gpu * ops_ct / 1e12 / sus, "peak_source": sus_src,
                              "roofline_ct_per_s_per_gpu": sus * 1e12 / ops_ct},
    }
    if e2e:
        # through the public API with pinned host buffers: the operator on CPU
        # tensors copies every input word in and every output word out inside
        # the timed region (chunks of 4 ciphertexts, copies overlapped with compute)
        hin = torch.empty(x.shape, dtype=torch.uint32, pin_memory=True)
        hin.copy_(x)
        hout = torch.empty(out.shape, dtype=torch.uint32, pin_memory=True)
        del x, out, ws
        torch.cuda.empty_cache()

        def e2e_step():
            torch.cuda.nvtx.range_push("e2e")
            op(hin, out=hout)
            torch.cuda.nvtx.range_pop()

        e2e_step()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        e0.record(stream)
        for _ in range(steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        ems = shard.max_over_ranks(e0.elapsed_time(e1), device=dev)
        line["e2e"] = {"value": pt.global_batch * steps / (ems / 1000.0), "unit": pt.unit,
                       "h2d_bytes_per_step": int(hin.numel() * 4), "d2h_bytes_per_step": int(hout.numel() * 4)}
        line["e2e"]["copies_alone"] = copies_alone(torch, dev, hin[:cb], hout[:cb], cb, pt.unit, world)
        del hin, hout
    else:
        del x, out, ws
    torch.cuda.empty_cache()
    if roofline:
        line["roofline"] = ntt_roofline(torch, dev, lib, Q[:pt.L - 1])
    if cpu and rank == 0 and world == 1:
        try:
            line["cpu_baseline"] = cpu_baseline(pt)
        except Exception as exc:  # noqa: BLE001
            line["cpu_baseline"] = {"error": str(exc)}
    del he
    torch.cuda.empty_cache()
    return line


def measure_he_limb(pt, torch, dist, world, rank, local, steps, warmup):
    """HE-Mult with the limbs of every ciphertext split across the ranks
    (cross_b200.limb_shard): each rank holds its Q' limbs (and the last limb
    of Q) of all pt.global_batch ciphertexts and runs the three phases per
    call of pt.call_batch ciphertexts, with the ModUp and ModDown limb
    all-gathers over NCCL in between.  Returns the JSON line."""
    from cross_b200 import _lib, hemul, limb_shard, shard
    dev = torch.device("cuda", local)
    lib = _lib.lib()
    B, cb = pt.global_batch, max(1, min(pt.call_batch, pt.global_batch))
    Q, P = moduli(pt)
    ea, eb = keys(pt)
    he = hemul.HEMul(cb, R, C, pt.dnum, 1, Q, P)
    he.control_gen(degree_layout=(R, C))
    he.setup_relinearization(ea, eb)
    del ea, eb
    sh = limb_shard.LimbShard(he, rank, world)
    own_mods = Q[sh.q0:sh.q1] + [Q[-1]]
    x = device_residues(torch, (B, 4, sh.nq + 1, N_DEG), own_mods, 100 + rank, dev, axis=2)
    outs = [None] * (-(-B // cb))

    def step():
        # the calls pipelined: each call's all-gathers overlap the others' kernels
        torch.cuda.nvtx.range_push("hemul_limb")
        outs[:] = sh.mul_many([x[a:a + cb] for a in range(0, B, cb)])
        torch.cuda.nvtx.range_pop()

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        l0 = lib.cross_launch_count()
        h0 = time.time()
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        h1 = time.time()
        launches = lib.cross_launch_count() - l0
    ms = shard.max_over_ranks(e0.elapsed_time(e1), device=dev)
    he.check_device()
    value = B * steps / (ms / 1000.0)
    cc_bytes = (world * sh.cq) * B * N_DEG * 4
    kp_bytes = (world * sh.cp) * 2 * B * N_DEG * 4
    line = {"metric": pt.metric + " limb-sharded", "value": value, "unit": pt.unit, "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": ms / steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "u32 residues, u64 intermediates, u8 BAT contractions",
            "data": "synthetic seeded uniform residues",
            "config": {"workload": pt.describe(B) + ", limbs split across the GPUs", "global_batch": B,
                       "call_batch": cb, "L": pt.L, "K": pt.K, "dnum": pt.dnum,
                       "parallelism": f"limb-sharded x{world}: Q' limbs [{sh.q0}, {sh.q1}), P limbs [{sh.p0}, "
                                      f"{sh.p1}) on rank {rank}; ModUp and ModDown all-gathers over NCCL, overlapping the "
                                      f"neighbouring calls' kernels (calls pipelined {limb_shard.PIPELINE_DEPTH} deep)",
                       "allgather_bytes_per_step": cc_bytes + kp_bytes},
            "gpu_launches": int(launches), "clocks": clk.summary(h0, h1),
            "e2e": None, "e2e_note": "inputs are resident per rank by limb (no host-buffer API for a limb split)"}
    del x, outs, sh, he
    torch.cuda.empty_cache()
    return line


def ntt_roofline(torch, dev, lib, mods, polys=256):
    """The dominant kernel, the two-SM tensor-core BAT contraction k_bat_tc2:
    one forward NTT of `polys` x len(mods) limb-polynomials in the kernels'
    native coefficient order is exactly two launches (the column stage with its
    twiddle epilogue, the row stage), timed alone with CUDA events on the
    launching stream; inputs are residues below each limb's modulus."""
    from cross_b200 import _lib, ntt_mm
    stream = torch.cuda.current_stream()
    M = len(mods)
    ctx = ntt_mm.NTTCiphertextBarrettContext(list(mods), {"r": R, "c": C})
    xin = device_residues(torch, (polys, M, R, C), list(mods), 17, dev, axis=1)
    xo = torch.empty_like(xin)
    nws = torch.empty(lib.cross_ntt_workspace_size(ctx.plan(), polys, _lib.LAYOUT_LIMB_MAJOR_TRANSPOSED),
                      dtype=torch.uint8, device=dev)

    def ntt_once():
        # NVTX range "roofline": profilers select these launches with
        # --nvtx --nvtx-include "roofline/"
        torch.cuda.nvtx.range_push("roofline")
        _lib.check(lib.cross_ntt(ctx.plan(), 0, xin.data_ptr(), xo.data_ptr(), polys,
                                 _lib.LAYOUT_LIMB_MAJOR_TRANSPOSED, nws.data_ptr(), nws.numel(),
                                 stream.cuda_stream), "cross_ntt")
        torch.cuda.nvtx.range_pop()

    for _ in range(2):
        ntt_once()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3
    e0.record(stream)
    for _ in range(reps):
        ntt_once()
    e1.record(stream)
    torch.cuda.synchronize()
    ntt_ms = e0.elapsed_time(e1) / reps
    ctx.check_device()
    l0 = lib.cross_launch_count()
    ntt_once()
    torch.cuda.synchronize()
    launches = lib.cross_launch_count() - l0              # 2: column + row contraction
    lps = polys * M
    ops = lps * 32.0 * N_DEG * (R + C)                    # int8 MAC x2 per limb-transform
    peak, src = int8_peak(torch, dev)
    achieved = ops / (ntt_ms / 1000.0) / 1e12
    del xin, xo, nws, ctx
    return {"kernel": f"k_bat_tc2 tensor-core BAT contraction (NTT column + row stage launches), {M} limbs x "
                      f"{polys} polys, N=2^16",
            "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TOPS (int8)", "frac": achieved / peak,
            "traffic": TRAFFIC_PER_LP * lps, "traffic_unit": "bytes per launch (ncu dram read + write, scaled by "
                                                             "limb-polynomials from the profiled launch)",
            "peak_source": src, "launches": launches, "ms_per_launch": ntt_ms / max(launches, 1),
            "algorithmic_ops_per_launch": ops / max(launches, 1)}


def _summary(line):
    keep = ("metric", "value", "unit", "ms_per_step", "gpu_launches")
    s = {k: line[k] for k in keep if k in line}
    s["workload"] = line["config"]["workload"]
    for k in ("roofline", "operator_roofline"):
        if k in line:
            s[k] = {kk: line[k][kk] for kk in ("bound", "achieved", "peak", "unit", "frac", "frac_of_hbm_bound",
                                               "hbm_bound_ms_per_step") if kk in line[k]}
    return s


def other_configs(torch, local, steps=10, warmup=3):
    """The scope's other configurations on this GPU (device-resident inputs)."""
    out = {}
    c = measure_component("ntt", torch, None, 1, 0, local, steps, warmup, ntt_limbs=8, ntt_polys=16,
                          ntt_degree=4096, cpu=False, e2e=False)
    out["1_ntt_intt_n4096_64x64_8limbs_16polys"] = _summary(c)
    c = measure_component("bconv", torch, None, 1, 0, local, steps, warmup, cpu=False, e2e=False)
    out["2_bconv_modup_n65536_24to25_32polys"] = _summary(c)
    c = measure_he(L24, torch, None, 1, 0, local, steps, warmup, e2e=False, cpu=False, roofline=False)
    out["3_hemul_n65536_l24_k8_dnum3_64ct"] = _summary(c)
    c = measure_he(Point("herot", 24, 8, 3, 64, 64), torch, None, 1, 0, local, steps, warmup, e2e=False, cpu=False,
                   roofline=False)
    out["4_herot_n65536_l24_k8_dnum3_64ct"] = _summary(c)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="cross_b200")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="skip the other configurations on one GPU")
    ap.add_argument("--lean", action="store_true",
                    help="time the HE step only: no end-to-end pass, roofline NTT, tensor-core probe, CPU baseline "
                         "or other configurations (small profiler captures)")
    ap.add_argument("--workload", choices=["hemul", "herot", "ntt", "bconv", "ckks", "bts", "i8peak"], default="hemul")
    ap.add_argument("--limbs", type=int, default=BOX.L, help="L of the HE-Mult / HE-Rotate point")
    ap.add_argument("--special", type=int, default=BOX.K, help="K of the HE-Mult / HE-Rotate point")
    ap.add_argument("--dnum", type=int, default=BOX.dnum, help="key-switch digits of the HE-Mult / HE-Rotate point")
    ap.add_argument("--global-batch", type=int, default=BOX.global_batch, help="ciphertexts per step over all GPUs")
    ap.add_argument("--call-batch", type=int, default=BOX.call_batch, help="ciphertexts per operator call")
    ap.add_argument("--shard", choices=["batch", "limb"], default="batch",
                    help="split the ciphertexts (batch) or the limbs of every ciphertext (limb) across GPUs")
    ap.add_argument("--bts-batch", type=int, default=1, help="polynomials per call of the bootstrapping mix")
    ap.add_argument("--bts-log", default=None, help="write the mix's latency lines (tabIX.py format) here")
    ap.add_argument("--bts-layout", choices=["native", "reference"], default="native")
    ap.add_argument("--reduction", choices=["barrett", "montgomery", "shoup", "bat_lazy"], default="barrett")
    ap.add_argument("--ntt-degree", type=int, default=N_DEG)
    ap.add_argument("--ntt-limbs", type=int, default=24)
    ap.add_argument("--ntt-polys", type=int, default=16)
    args = ap.parse_args()
    pt = Point("herot" if args.workload == "herot" else "hemul", args.limbs, args.special, args.dnum,
               args.global_batch, args.call_batch)
    if args.impl == "reference":
        return run_reference(args, pt)

    import torch
    from cross_b200 import shard
    world, rank, local = shard.rank_env()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=torch.device("cuda", local))
    if args.workload not in ("hemul", "herot"):
        {"ckks": run_ckks, "bts": run_bts, "i8peak": run_i8peak}.get(args.workload, run_component)(
            args, torch, dist, world, rank, local)
    elif args.shard == "limb":
        if pt.workload != "hemul":
            raise SystemExit("--shard limb is implemented for HE-Mult")
        line = measure_he_limb(pt, torch, dist, world, rank, local, args.steps, args.warmup)
        if rank == 0:
            print(json.dumps(line), flush=True)
    else:
        lean = args.lean
        line = measure_he(pt, torch, dist, world, rank, local, args.steps, args.warmup, e2e=not lean,
                          cpu=not (args.no_cpu_baseline or lean), roofline=not lean, probe=not lean)
        if world == 1 and not (args.no_configs or lean) and pt == BOX:
            line["configs"] = other_configs(torch, local)
        if rank == 0:
            print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
