"""Benchmark: CKKS HE-Mult with relinearisation at N = 2^16.

Workload (one step): HEMul.mul over a batch of 64 ciphertexts with N = 2^16
(256 x 256), L = 24 limbs of 28-bit NTT primes, K = 8 special limbs, dnum = 3;
seeded uniform residues; evaluation keys seeded uniform.  Weak scaling: every
rank processes its own batch of 64 (the reference shards the batch axis only).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Prints one JSON line on rank 0.  Other workloads of the same line format:
  --workload herot              HE-Rotate at the same point (B, 2, r, c, L) -> (B, 2, N, L)
  --limbs L --special K --dnum D  another HE-Mult / HE-Rotate point (35, 7, 5: the 8-GPU point)
  --workload ntt / bconv        the transform or the basis conversion alone for one reduction
                                (--reduction barrett | montgomery | shoup | bat_lazy): NTT + INTT
                                over --ntt-limbs limbs x --ntt-polys polys of N = --ntt-degree
                                (default 2^16, 24, 16); BConv 24 -> 25 limbs, 32 polys of N = 2^16
  --workload ckks               a CKKS encode -> encrypt -> decrypt -> decode round trip
  --workload bts                the bootstrapping kernel mix: every (kernel, size) of a CKKS
                                bootstrapping's schedule timed, latencies weighted by invocation
                                counts (us per polynomial, lower is better)
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

N_DEG, R, C, L, K, DNUM, BATCH = 65536, 256, 256, 24, 8, 3, 64
# DRAM bytes (read + write) per k_bat_tc2 launch of the roofline NTT at batch 64,
# from profiles/k_bat_tc2_ntt_n65536.md (batch-16 ncu capture scaled by 4).
TRAFFIC_PER_LAUNCH = 3.148e9
METRIC = "HE-Mult/s (N=2^16, L=24, dnum=3)"
WORKLOAD = "CKKS HE-Mult + relinearisation, N=2^16 (256x256), L=24 x 28-bit, K=8, dnum=3, batch 64 per GPU"


def set_point(workload: str, limbs: int, special: int, dnum: int, batch: int) -> None:
    """Select the HE operator point (module constants used by the helpers)."""
    global L, K, DNUM, METRIC, WORKLOAD
    L, K, DNUM = limbs, special, dnum
    if workload == "herot":
        METRIC = f"HE-Rotate/s (N=2^16, L={L}, dnum={DNUM})"
        WORKLOAD = (f"CKKS HE-Rotate (hybrid key switch), N=2^16 (256x256), L={L} x 28-bit, K={K}, dnum={DNUM}, "
                    f"batch {batch} per GPU")
    else:
        METRIC = f"HE-Mult/s (N=2^16, L={L}, dnum={DNUM})"
        WORKLOAD = (f"CKKS HE-Mult + relinearisation, N=2^16 (256x256), L={L} x 28-bit, K={K}, dnum={DNUM}, "
                    f"batch {batch} per GPU")


def rotation_map(seed: int = 0):
    """A seeded rotation index k in [1, N/2) and its coefficient map
    (util.py:652-693)."""
    import numpy as np
    from cross_b200 import util
    k = int(np.random.default_rng(seed).integers(1, N_DEG // 2))
    return k, util.precompute_auto_map(N_DEG, util.find_automorphism_index_2n_complex(k, 2 * N_DEG))


def moduli():
    from cross_b200 import util
    ov = util.find_moduli_ntt(L + K, 28, 2 * N_DEG)
    return ov[:L], ov[L:]


def inputs(seed_ct: int, batch: int):
    import numpy as np
    Q, P = moduli()
    rng = np.random.default_rng(seed_ct)
    q = np.array(Q, np.uint64)
    ct = (rng.integers(0, 2 ** 62, size=(batch, 4, R, C, L), dtype=np.uint64) % q).astype(np.uint32)
    krng = np.random.default_rng(1)
    ov = np.array(Q + P, np.uint64)
    ea = (krng.integers(0, 2 ** 62, size=(DNUM, N_DEG, L + K), dtype=np.uint64) % ov).astype(np.uint32)
    eb = (krng.integers(0, 2 ** 62, size=(DNUM, N_DEG, L + K), dtype=np.uint64) % ov).astype(np.uint32)
    return ct, ea, eb


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


def _oracle_op(workload: str):
    """The oracle's operator for one ciphertext of the workload and its input."""
    from oracle import cross_oracle as O
    Q, P = moduli()
    ct, ea, eb = inputs(0, 1)
    if workload == "herot":
        op = O.HERot(R, C, DNUM, Q, P)
        op.control_gen(1)
        op.setup_rotate(ea.reshape(DNUM, R, C, -1), eb.reshape(DNUM, R, C, -1), rotation_map()[1])
        return op.rotate, ct[:, :2], "HE-Rot/s", "HERot.rotate"
    he = O.HEMul(1, R, C, DNUM, 1, Q, P)
    he.setup_relinearization(ea, eb)
    return he.mul, ct, "HE-Mult/s", "HEMul.mul"


def cpu_baseline(steps: int = 1, workload: str = "hemul"):
    """The oracle (numpy restatement of jaxite_word) on the host cores: one
    ciphertext per step."""
    fn, ct, unit, name = _oracle_op(workload)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        fn(ct)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": 1.0 / t, "unit": unit, "cores": os.cpu_count(), "kind": "port",
            "sample": f"{steps} x 1 ciphertext of the workload (oracle/cross_oracle.py {name}, numpy BLAS threads)",
            "seconds_per_ct": t}


def run_reference(args):
    """--impl reference: the oracle port of jaxite_word's HEMul.mul on the host
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
    fn, ct, unit, name = _oracle_op(args.workload)
    for _ in range(args.warmup):
        fn(ct)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fn(ct)
    dt = (time.perf_counter() - t0) / max(args.steps, 1)
    v = 1.0 / dt
    sample = f"1 ciphertext of the workload per step (oracle/cross_oracle.py {name}, numpy BLAS threads)"
    print(json.dumps({"impl": "reference", "metric": METRIC, "value": v, "unit": unit, "n_gpus": args.gpus,
                      "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * dt,
                      "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                      "dtype": "u32 residues, u64 intermediates, u8 BAT contractions", "data": "synthetic seeded",
                      "config": {"workload": WORKLOAD, "sample": "1 ciphertext per step"},
                      "cpu_baseline": {"value": v, "unit": unit, "cores": os.cpu_count(), "kind": "port",
                                       "sample": sample},
                      "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
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


def run_component(args, torch, dist, world, rank, local):
    """--workload ntt | bconv for one reduction: device throughput, end-to-end
    throughput through the operator API with host buffers, the kernel's
    roofline and the oracle on the host cores."""
    import numpy as np
    from cross_b200 import _lib, bconv, ntt_mm, util
    from oracle import cross_oracle as O
    from oracle import variants as V
    dev = torch.device("cuda", local)
    timer = _Timer(torch, dist, dev)
    lib = _lib.lib()
    red = args.reduction
    pk, src = peaks()
    rng = np.random.default_rng(200 + rank)
    if args.workload == "ntt":
        Lw, B, nd = args.ntt_limbs, args.ntt_polys, args.ntt_degree
        rr, cc = util.default_rc(nd)
        q = O.find_moduli_ntt(Lw, 28, 2 * nd)
        cls = {"barrett": ntt_mm.NTTCiphertextBarrettContext, "montgomery": ntt_mm.NTTCiphertextMontgomeryContext,
               "shoup": ntt_mm.NTTCiphertextShoupContext, "bat_lazy": ntt_mm.NTTCiphertextBATLazyContext}[red]
        ctx = cls(q, {"r": rr, "c": cc})
        xh = (rng.integers(0, 2 ** 62, size=(B, Lw, rr, cc), dtype=np.uint64) %
              np.array(q, np.uint64)[:, None, None]).astype(np.uint32)
        x = torch.from_numpy(xh).to(dev)
        y = torch.empty_like(x)
        ws = torch.empty(lib.cross_ntt_workspace_size(ctx.plan(), B, _lib.LAYOUT_LIMB_MAJOR), dtype=torch.uint8,
                         device=dev)
        cs = torch.cuda.current_stream().cuda_stream

        def step():
            for inv, a, b in ((0, x, y), (1, y, y)):
                _lib.check(lib.cross_ntt(ctx.plan(), inv, a.data_ptr(), b.data_ptr(), B, _lib.LAYOUT_LIMB_MAJOR,
                                         ws.data_ptr(), ws.numel(), cs), "cross_ntt")
        units = 2 * B * Lw                                   # limb-transforms per step
        metric, unit = f"NTT+INTT limb-transforms/s (N={nd}, {red})", "limb-transform/s"
        workload = f"BAT NTT then INTT, {red} reduction, N={nd} ({rr}x{cc}), {Lw} limbs x {B} polys per GPU"
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
            roof = {"bound": "tensor", "unit": "TOPS (int8)", "peak": 2.0 * pk["bf16_tflops"],
                    "peak_source": f"2 x bf16_tflops of MEASURED_PEAKS.json ({src})"}
        roof["kernel"] = "all launches of one NTT + INTT (2 contraction stages each)"
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
        cs = torch.cuda.current_stream().cuda_stream

        def step():
            _lib.check(lib.cross_bconv_ex(bc.plan(0), int(bat), x.data_ptr(), y.data_ptr(), B, N_DEG,
                                          _lib.LAYOUT_LIMB_MAJOR, cs), "cross_bconv_ex")
        units = B
        metric, unit = f"BConv polys/s (N=2^16, 24->25 limbs, {red})", "poly/s"
        workload = f"basis conversion {'basis_change_bat' if bat else 'basis_change'}, {red}, 24 -> 25 limbs, N=2^16, 32 polys per GPU"
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
    for _ in range(args.warmup):
        step()
    ms = timer(step, args.steps)
    l0 = lib.cross_launch_count()
    step()
    torch.cuda.synchronize()
    launches = (lib.cross_launch_count() - l0) * args.steps
    value = world * units * args.steps / (ms / 1000.0)
    e2e_step()
    ems = timer(e2e_step, args.steps)
    e2e = world * units * args.steps / (ems / 1000.0)
    per = ms / args.steps / 1000.0
    achieved = ops / per / (1e12 if roof["unit"] != "GB/s" else 1e9)
    roof.update({"achieved": achieved, "frac": achieved / roof["peak"], "traffic": None,
                 "ms_per_step": ms / args.steps})
    line = {"metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u32 residues, u64 intermediates",
            "data": "synthetic seeded uniform residues", "config": {"workload": workload, "reduction": red,
                                                                    "l2": "inputs larger than L2"},
            "e2e": {"value": e2e, "unit": unit, "h2d_bytes_per_step": int(hin.numel() * 4),
                    "d2h_bytes_per_step": int(y.numel() * y.element_size())},
            "gpu_launches": int(launches), "roofline": roof}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        dt = cpu_once()
        line["cpu_baseline"] = {"value": cpu_units / dt, "unit": unit, "cores": os.cpu_count(), "kind": "port",
                                "sample": f"{cpu_units} units of the workload (oracle, numpy BLAS threads)"}
    if rank == 0:
        print(json.dumps(line), flush=True)


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
            by_kernel[kernel] = {"bound": "tensor", "achieved": a, "unit": "TOPS (int8)",
                                 "peak": 2.0 * pk["bf16_tflops"], "frac": a / (2.0 * pk["bf16_tflops"]),
                                 "share_pct": summ["ratios_pct"].get(kernel)}
    top = max(summ["ratios_pct"], key=summ["ratios_pct"].get)
    roof = dict(by_kernel[top])
    roof.update({"kernel": f"{top} rows of the schedule (count-weighted)", "traffic": None,
                 "peak_source": f"MEASURED_PEAKS.json ({src}); int8 = 2 x bf16_tflops"})
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
    pk, src = peaks()
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
                         "achieved": achieved, "peak": 2.0 * pk["bf16_tflops"], "unit": "TOPS (int8)",
                         "frac": achieved / (2.0 * pk["bf16_tflops"]), "traffic": None,
                         "peak_source": f"2 x bf16_tflops of MEASURED_PEAKS.json ({src})"}}
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="cross_b200")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=BATCH, help="ciphertexts per GPU (profiling runs use a small case)")
    ap.add_argument("--workload", choices=["hemul", "herot", "ntt", "bconv", "ckks", "bts"], default="hemul")
    ap.add_argument("--bts-batch", type=int, default=1, help="polynomials per call of the bootstrapping mix")
    ap.add_argument("--bts-log", default=None, help="write the mix's latency lines (tabIX.py format) here")
    ap.add_argument("--bts-layout", choices=["native", "reference"], default="native")
    ap.add_argument("--reduction", choices=["barrett", "montgomery", "shoup", "bat_lazy"], default="barrett")
    ap.add_argument("--limbs", type=int, default=L, help="L of the HE-Mult / HE-Rotate point")
    ap.add_argument("--special", type=int, default=K, help="K of the HE-Mult / HE-Rotate point")
    ap.add_argument("--dnum", type=int, default=DNUM, help="key-switch digits of the HE-Mult / HE-Rotate point")
    ap.add_argument("--ntt-degree", type=int, default=N_DEG)
    ap.add_argument("--ntt-limbs", type=int, default=24)
    ap.add_argument("--ntt-polys", type=int, default=16)
    args = ap.parse_args()
    set_point(args.workload, args.limbs, args.special, args.dnum, args.batch)
    if args.impl == "reference":
        return run_reference(args)

    import numpy as np
    import torch
    from cross_b200 import shard
    world, rank, local = shard.rank_env()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    if args.workload not in ("hemul", "herot"):
        {"ckks": run_ckks, "bts": run_bts}.get(args.workload, run_component)(args, torch, dist, world, rank, local)
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return

    from cross_b200 import _lib, hemul, herot, ntt_mm
    batch = args.batch
    Q, P = moduli()
    ct, ea, eb = inputs(100 + rank, batch)
    dev = torch.device("cuda", local)
    if args.workload == "herot":
        he = herot.HERot(R, C, DNUM, Q, P)
        he.control_gen(batch=batch, degree_layout=(R, C))
        he.setup_rotate(ea, eb, rotation_map()[1])
        ct = ct[:, :2].copy()
        op, out_shape, unit, tag = he.rotate, (batch, 2, N_DEG, L), "HE-Rot/s", "herot"
    else:
        he = hemul.HEMul(batch, R, C, DNUM, 1, Q, P)
        he.control_gen(degree_layout=(R, C))
        he.setup_relinearization(ea, eb)
        op, out_shape, unit, tag = he.mul, (batch, 2, R, C, L - 1), "HE-Mult/s", "hemul"
    x = torch.from_numpy(ct).to(dev)
    out = torch.empty(out_shape, dtype=torch.uint32, device=dev)
    ws = torch.empty(he.workspace_size(batch), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()

    def step():
        torch.cuda.nvtx.range_push(tag)
        op(x, out=out, workspace=ws)
        torch.cuda.nvtx.range_pop()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    lib = _lib.lib()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        l0 = lib.cross_launch_count()
        h0 = time.time()
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        h1 = time.time()
        launches = lib.cross_launch_count() - l0
    ms = shard.max_over_ranks(e0.elapsed_time(e1), device=dev)
    value = world * batch * args.steps / (ms / 1000.0)

    # e2e through the public API with pinned host buffers: HEMul.mul on CPU
    # tensors copies every input word in and every output word out inside the
    # timed region (in chunks of 4 ciphertexts, copies overlapped with compute).
    hin = torch.from_numpy(ct).pin_memory()
    hout = torch.empty(out.shape, dtype=torch.uint32).pin_memory()

    def e2e_step():
        torch.cuda.nvtx.range_push("e2e")
        op(hin, out=hout)
        torch.cuda.nvtx.range_pop()

    e2e_step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    ems = shard.max_over_ranks(e0.elapsed_time(e1), device=dev)
    e2e = world * batch * args.steps / (ems / 1000.0)

    # Dominant kernel: the tensor-core BAT contraction.  One forward NTT in the
    # kernels' native coefficient order is exactly two contraction launches (the
    # column stage with its twiddle epilogue, the row stage); timed alone over
    # the polys x (L - 1) limb-polynomials of the input (for HE-Mult, those of
    # its rescale NTT).
    ctx = ntt_mm.NTTCiphertextBarrettContext(Q[:L - 1], {"r": R, "c": C})
    lps = x.numel() // (L * N_DEG)
    xin = x.reshape(-1)[: lps * (L - 1) * N_DEG].reshape(lps, L - 1, R, C)   # residues < q
    xo = torch.empty_like(xin)
    nws = torch.empty(lib.cross_ntt_workspace_size(ctx.plan(), lps, _lib.LAYOUT_LIMB_MAJOR_TRANSPOSED),
                      dtype=torch.uint8, device=dev)

    def ntt_once():
        # NVTX range "roofline": profilers select these launches with
        # --nvtx --nvtx-include "roofline/"
        torch.cuda.nvtx.range_push("roofline")
        _lib.check(lib.cross_ntt(ctx.plan(), 0, xin.data_ptr(), xo.data_ptr(), lps, _lib.LAYOUT_LIMB_MAJOR_TRANSPOSED,
                                 nws.data_ptr(), nws.numel(), stream.cuda_stream), "cross_ntt")
        torch.cuda.nvtx.range_pop()

    for _ in range(2):
        ntt_once()
    torch.cuda.synchronize()
    reps = 3
    e0.record(stream)
    for _ in range(reps):
        ntt_once()
    e1.record(stream)
    torch.cuda.synchronize()
    ntt_ms = e0.elapsed_time(e1) / reps
    # every tensor-core kernel of the timed work completed (no bounded wait expired)
    he.check_device()
    ctx.check_device()
    l0 = lib.cross_launch_count()
    ntt_once()
    torch.cuda.synchronize()
    ntt_launches = lib.cross_launch_count() - l0              # 2: column + row contraction
    transforms = lps * (L - 1)
    ops = transforms * 32.0 * N_DEG * (R + C)              # int8 MAC x2 per limb-transform
    pk, src = peaks()
    int8_peak = 2.0 * pk["bf16_tflops"]                     # TOPS: dense int8 = 2 x dense bf16 on B200
    achieved = ops / (ntt_ms / 1000.0) / 1e12

    line = {
        "metric": METRIC, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u32 residues, u64 intermediates, u8 BAT contractions",
        "data": "synthetic seeded uniform residues (no dataset in the reference)",
        "config": {"workload": WORKLOAD, "global_batch": world * batch, "batch_per_gpu": batch, "N": N_DEG, "r": R, "c": C, "L": L, "K": K,
                   "dnum": DNUM, "parallelism": f"batch-sharded x{world}",
                   "l2": f"inputs {x.numel() * 4 / 1e9:.2f} GB per GPU, larger than L2 (no flush needed)"},
        "e2e": {"value": e2e, "unit": unit, "h2d_bytes_per_step": int(hin.numel() * 4),
                "d2h_bytes_per_step": int(hout.numel() * 4)},
        "gpu_launches": int(launches),
        "clocks": clk.summary(h0, h1),
        "roofline": {"kernel": "k_bat_tc2 tensor-core BAT contraction (NTT column + row stage launches), "
                               f"{L - 1} limbs x {lps} polys, N=2^16",
                     "bound": "tensor", "achieved": achieved, "peak": int8_peak, "unit": "TOPS (int8)",
                     "frac": achieved / int8_peak,
                     # the captured launch processed 256 x 23 limb-polynomials; traffic scales with them
                     "traffic": TRAFFIC_PER_LAUNCH * transforms / (256 * 23),
                     "traffic_unit": "bytes per launch (ncu dram read + write)",
                     "peak_source": f"2 x bf16_tflops of MEASURED_PEAKS.json ({src}); no int8 measurement on this pool",
                     "launches": ntt_launches, "ms_per_launch": ntt_ms / max(ntt_launches, 1),
                     "algorithmic_ops_per_launch": ops / max(ntt_launches, 1)},
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            line["cpu_baseline"] = {k: v for k, v in cpu_baseline(1, args.workload).items() if k != "seconds_per_ct"}
        except Exception as exc:  # noqa: BLE001
            line["cpu_baseline"] = {"error": str(exc)}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    del np


if __name__ == "__main__":
    main()
