"""Benchmark of the FHE NTT hot path (negacyclic NTT + INTT at N = 2^16).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (benchmark config 3): N = 2^16, 48 RNS limbs (the 48 largest primes
below 2^31 with q = 1 mod 2N: the reference is exact only below 2^31),
128 ciphertexts x 2 polynomials per GPU, layout [ct][2][limb][N] (u64), seeded
uniform coefficients.  One step = one forward negacyclic NTT and one INTT of
every limb-polynomial (24,576 limb-transforms per GPU).  Each GPU owns its own
contiguous range of ciphertexts (no collective on the data path), so per-GPU
work is fixed as GPUs are added ("weak" scaling); --strong splits 128
ciphertexts over the GPUs instead.  Inputs (6.4 GB per GPU) are larger than
L2, so no flush is needed between steps.

Metric: limb-transforms/s for the whole job (all GPUs), device time from CUDA
events on the launching stream, max over ranks.  `e2e` repeats the step through
the public API with host buffers: pinned host -> device copy of the inputs,
forward + inverse, device -> host copy of the results, chunked over streams.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

N_LOG = 16
N = 1 << N_LOG
LIMBS = 48
CTS_PER_GPU = 128
BYTES_PER_TRANSFORM = 16 * N        # read N u64 + write N u64 (algorithmic)
METRIC = "negacyclic NTT limb-transforms/s at N=2^16 (fwd+inv, 48 limbs, 128 ct x 2 polys per GPU)"
UNIT = "limb-transforms/s"
# dram__bytes_read.sum + dram__bytes_write.sum of the dominant kernel per
# limb-transform, from an ncu capture of the forward kernel at 768 transforms
# per launch ((427.93 + 350.64) MB, `bench.py --cts 8`); DRAM traffic per
# transform does not depend on the batch, so it is scaled to a full launch.
NCU_TRAFFIC_PER_TRANSFORM = 1_013_763


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """SM clocks, power and throttle reasons sampled during the timed region:
    NVML polled every 10 ms from a thread (the timed region can be shorter
    than nvidia-smi's sampling period), nvidia-smi -lms 200 if NVML fails."""

    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.path = None
        self.thread = None
        self.rows = []
        self.done = False

    def _nvml_handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        try:
            pr = torch.cuda.get_device_properties(self.gpu)
            bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.gpu)

    def start(self):
        import threading
        import time
        try:
            nv, h = self._nvml_handle()
            bits = (nv.nvmlClocksEventReasonHwSlowdown, nv.nvmlClocksEventReasonHwThermalSlowdown,
                    nv.nvmlClocksEventReasonSwThermalSlowdown, nv.nvmlClocksEventReasonSwPowerCap)
            smax = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)

            def poll():
                while not self.done:
                    r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.rows.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM), smax,
                                      nv.nvmlDeviceGetPowerUsage(h) / 1000.0,
                                      [n for n, b in zip(self.NAMES, bits) if r & b]))
                    time.sleep(0.01)
            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.thread = None
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.thread is not None:
            self.done = True
            self.thread.join(timeout=5)
            rows, source = self.rows, "nvml, 10 ms"
        elif self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            rows, source = [], "nvidia-smi, 200 ms"
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9 and parts[1].isdigit():
                    pw = float(parts[3]) if parts[3].replace(".", "", 1).isdigit() else 0.0
                    rows.append((int(parts[1]), int(parts[2]), pw,
                                 [n for n, v in zip(self.NAMES, parts[5:9]) if v.lower().startswith("active")]))
            os.unlink(self.path)
        else:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no clock source"]}
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": rows[0][1],
                "power_w_max": max(r[2] for r in rows),
                "reasons": sorted({n for r in rows for n in r[3]}), "samples": len(rows),
                "source": source}


def numa_bind(local):
    """Binds this process's host threads to the CPUs of the NUMA node its GPU
    hangs off (from sysfs), so that pinned host buffers allocated afterwards
    are first touched there and host<->device copies do not cross the
    inter-socket link.  Returns (description for the bench line, previous
    affinity to restore)."""
    prev = os.sched_getaffinity(0)
    try:
        import torch
        pr = torch.cuda.get_device_properties(local)
        bus = f"{pr.pci_domain_id:04x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
        with open(f"/sys/bus/pci/devices/{bus}/numa_node") as f:
            node = int(f.read().strip())
        if node < 0:
            return {"gpu_pci": bus, "numa_node": None, "note": "the system reports no NUMA node"}, prev
        with open(f"/sys/devices/system/node/node{node}/cpulist") as f:
            spec = f.read().strip()
        cpus = set()
        for part in spec.split(","):
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
        cpus &= prev
        if not cpus:
            return {"gpu_pci": bus, "numa_node": node, "note": "no allowed CPU on that node"}, prev
        os.sched_setaffinity(0, cpus)
        return {"gpu_pci": bus, "numa_node": node, "cpus_bound": len(cpus),
                "pinned_buffers": "allocated after binding (first touch on the GPU's node)"}, prev
    except Exception as e:  # no sysfs entry (containers), or no properties
        return {"note": f"NUMA placement unavailable: {type(e).__name__}: {e}"}, prev


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# --------------------------------------------------------------- reference arm

def run_reference(args):
    """The reference's own algorithm on the host cores (oracle port of the WGSL
    path: bit-serial u64 emulation, radix-2 DIT passes, separate scale pass),
    negacyclic via the reference's own ops (pointwise twist + cyclic NTT)."""
    world, rank, _ = dist_setup()
    if rank != 0:
        return
    import numpy as np
    from oracle import oracle

    threads = os.cpu_count() or 1
    q = [oracle.ntt_prime(31, N, i) for i in range(LIMBS)]
    psi = [oracle.psi(x, N) for x in q]
    per_step = threads  # limb-polys per step: one per host thread (fwd + inv each)
    x = np.concatenate([oracle.seeded_fill(N, 0, p * N, q[p % LIMBS]) for p in range(per_step)])
    times = []
    for it in range(args.warmup + args.steps):
        t_f, X = oracle.baseline_run("negacyclic_ntt", x, N, q[:per_step], psi[:per_step], threads)
        t_i, y = oracle.baseline_run("negacyclic_intt", X, N, q[:per_step], psi[:per_step], threads)
        if it >= args.warmup:
            times.append(t_f + t_i)
        assert (y == x).all()
    total = sum(times)
    value = 2 * per_step * len(times) / total
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * total / len(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u32 (u64 storage)",
        "data": "synthetic",
        "config": {"workload": f"config3 sample: {per_step} limb-polys of N=2^16 per step (fwd+inv), "
                               "q < 2^31, reference algorithm restated in C (oracle/ref_wgsl.c)",
                   "N": N, "limbs": LIMBS},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{per_step} limb-polys x (fwd+inv) per step, {args.steps} steps"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline_sample(seconds_target=12.0):
    """Oracle (reference algorithm) timed on the host cores on a bounded sample."""
    import numpy as np
    from oracle import oracle
    threads = os.cpu_count() or 1
    q = [oracle.ntt_prime(31, N, i) for i in range(LIMBS)]
    psi = [oracle.psi(x, N) for x in q]
    # calibrate with one polynomial per thread, then scale to ~seconds_target
    count = threads
    x = np.concatenate([oracle.seeded_fill(N, 0, p * N, q[p % LIMBS]) for p in range(count)])
    t, _ = oracle.baseline_run("negacyclic_ntt", x, N, q[:count], psi[:count], threads)
    reps = max(1, int(seconds_target / max(t, 1e-3) / 2))
    count = min(threads * reps, 4 * LIMBS * 8)
    x = np.concatenate([oracle.seeded_fill(N, 0, p * N, q[p % LIMBS]) for p in range(count)])
    qq = [q[p % LIMBS] for p in range(count)]
    pp = [psi[p % LIMBS] for p in range(count)]
    t_f, X = oracle.baseline_run("negacyclic_ntt", x, N, qq, pp, threads)
    t_i, _ = oracle.baseline_run("negacyclic_intt", X, N, qq, pp, threads)
    return {"value": 2 * count / (t_f + t_i), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{count} limb-polys of N=2^16, fwd+inv, reference algorithm (oracle/ref_wgsl.c), "
                      f"{t_f + t_i:.1f} s"}


# --------------------------------------------------------------- our arm

def run_ours(args):
    import torch

    import barracuda_b200 as bc

    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    # one process per GPU; the only collectives are the timing max, the unit
    # count and the digest gather (NCCL), each preceded by a status check
    group = bc.ShardGroup("nccl", timeout=300.0, device=torch.device("cuda", local))
    try:
        _run_ours(args, torch, bc, group, world, rank, local)
    finally:
        group.close()


def _run_ours(args, torch, bc, group, world, rank, local):
    dev = bc.Device(local)
    cts_total = args.cts_total if args.strong else args.cts * world
    shard = bc.Shard.of(cts_total, world, rank)
    ct_begin, ct_count = shard.begin, shard.count
    polys = 2 * ct_count
    qs = bc.ntt_primes(31, N, LIMBS)
    psis = [bc.negacyclic_root(q, N) for q in qs]
    lay = bc.Layout(limb_stride=N, poly_stride=LIMBS * N)
    words = polys * LIMBS * N
    first_word = 2 * ct_begin * LIMBS * N  # global index of this shard's first coefficient
    # an explicit stream: handle 0 (torch's legacy default stream) would mean
    # "the context stream" to the C ABI, and the events must sit on the
    # stream the kernels run on
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    sh = stream.cuda_stream

    def setup():
        plan = bc.NttPlan(dev, N, qs, psis, mode=bc.NEGACYCLIC)
        x = torch.empty(words, dtype=torch.int64, device="cuda")
        X = torch.empty(words, dtype=torch.int64, device="cuda")
        plan.fill_uniform(x, polys, seed=0, first_poly=2 * ct_begin, total_polys=2 * cts_total,
                          layout=lay, stream=sh)
        return plan, x, X

    plan, x, X = group.step("setup", setup)
    dig = torch.zeros(3, dtype=torch.int64, device="cuda")
    bc.digest(dev, x, words, dig[0:1], stream=sh, first_index=first_word)

    def step(ev=None):
        if ev is not None:
            ev[0].record(stream)
        plan.forward(x, X, polys, layout=lay, stream=sh)
        if ev is not None:
            ev[1].record(stream)
        plan.inverse(X, x, polys, layout=lay, stream=sh)
        if ev is not None:
            ev[2].record(stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    group.step("warmup", lambda: None)
    group.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for k in range(args.steps):
        step(evs[k])
    t1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    group.step("timed", lambda: None)
    group.barrier()
    ms = t0.elapsed_time(t1)
    fwd_ms = [e[0].elapsed_time(e[1]) for e in evs]
    inv_ms = [e[1].elapsed_time(e[2]) for e in evs]
    ms_max = group.max_f64(ms)
    units = 2 * sum(r[0] for r in group.gather_u64([polys * LIMBS])) * args.steps
    value = units / (ms_max / 1000.0)

    # verification: forward output and round trip, digests with global
    # indices gathered to every rank (their sums do not depend on the split)
    bc.digest(dev, X, words, dig[1:2], stream=sh, first_index=first_word)
    bc.digest(dev, x, words, dig[2:3], stream=sh, first_index=first_word)
    torch.cuda.synchronize()
    rows = group.gather_u64([int(v) for v in dig.tolist()])
    verification = {
        "input_digest": f"{bc.job_digest(r[0] for r in rows):016x}",
        "forward_digest": f"{bc.job_digest(r[1] for r in rows):016x}",
        "roundtrip_identity": all(r[0] == r[2] for r in rows),
        "gathered": f"all_gather of per-rank digests over {world} rank(s)",
    }

    # ---- e2e through the public API with pinned host buffers
    placement, prev_affinity = numa_bind(local)
    try:
        e2e = (run_e2e(args, torch, plan, lay, polys, x, X, group) if args.e2e_steps > 0 else None)
    finally:
        os.sched_setaffinity(0, prev_affinity)  # the CPU baseline below uses every host core
    if e2e is not None:
        e2e["host_placement"] = placement

    info = plan.info
    launches_per_transform = {0: 1, 1: 1, 2: N_LOG + 2, 3: 1}[info["kernel_kind"]]
    hbm, peak_kind = peaks()
    per_launch_bytes = BYTES_PER_TRANSFORM * polys * LIMBS
    fwd_avg = statistics.mean(fwd_ms)
    inv_avg = statistics.mean(inv_ms)
    achieved = per_launch_bytes / (fwd_avg / 1000.0) / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": achieved / hbm, "peak_kind": peak_kind,
                "kernel": "negacyclic forward NTT (one launch over all limb-polys of the GPU)",
                "algorithmic_bytes_per_launch": per_launch_bytes,
                "avg_launch_ms": fwd_avg, "inverse_avg_launch_ms": inv_avg,
                "traffic": (NCU_TRAFFIC_PER_TRANSFORM * polys * LIMBS
                            if NCU_TRAFFIC_PER_TRANSFORM else None)}
    # The roofline's second term: (N/2) log2 N butterflies per transform at
    # the integer-pipe peak, measured live on this GPU with the plans' own
    # 32-bit arithmetic (after the timed region).
    bfly = bc.calibrate_butterflies(dev, 32)
    int_rate = bfly / ((N // 2) * N_LOG)
    hbm_rate = hbm * 1e9 / BYTES_PER_TRANSFORM
    launch_rate = polys * LIMBS / (fwd_avg / 1000.0)
    roofline["integer_peak"] = {"butterflies_per_s": bfly, "limb_transforms_per_s": int_rate,
                                "word_bits": 32, "measured": "bc_calibrate_butterflies, register-only"}
    roofline["hbm_limb_transforms_per_s"] = hbm_rate
    roofline["binding_term"] = "hbm" if hbm_rate <= int_rate else "integer"
    roofline["frac_of_binding_term"] = launch_rate / min(hbm_rate, int_rate)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_sample()

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "strong" if args.strong else "weak", "vs_baseline": None,
            "dtype": "u32 (u64 storage)", "data": "synthetic",
            "config": {"workload": "config3: N=2^16 negacyclic NTT+INTT, 48 limbs (largest primes "
                                   "< 2^31, q = 1 mod 2N), [ct][2][limb][N] u64 layout",
                       "cts_per_gpu": ct_count, "cts_total": cts_total, "limb_transforms_per_step":
                       int(units / args.steps), "l2": "inputs 6.4 GB/GPU > 126 MB L2, no flush",
                       "parallelism": f"shard by ciphertext x{world}",
                       "kernel_kind": info["kernel_kind"], "cluster": info["cluster_size"]},
            "gb_per_s": value * BYTES_PER_TRANSFORM / 1e9,
            "roofline": roofline,
            "clocks": clk,
            "gpu_launches": 2 * launches_per_transform * args.steps,
            "e2e": e2e,
            "cpu_baseline": cpu,
            "roundtrip_identity": verification["roundtrip_identity"],
            "verification": verification,
        }
        print(json.dumps(line), flush=True)
    plan.close()
    dev.close()


def run_e2e(args, torch, plan, lay, polys, x, X, group):
    """Host buffers in, host buffers out, through the same public calls."""
    steps = max(1, args.e2e_steps)
    words = polys * LIMBS * N
    host = torch.empty(words, dtype=torch.int64, pin_memory=True)
    # inputs for e2e: the seeded data, staged once to pinned host memory
    host.copy_(x, non_blocking=False)
    chunks = max(1, args.e2e_chunks)
    cts = polys // 2
    streams = [torch.cuda.Stream() for _ in range(max(1, args.e2e_streams))]
    per = [(c * cts) // chunks for c in range(chunks + 1)]
    elem_per_ct = 2 * LIMBS * N

    def one_step():
        cur = torch.cuda.current_stream()
        for s in streams:
            s.wait_stream(cur)
        for c in range(chunks):
            s = streams[c % len(streams)]
            lo, hi = per[c] * elem_per_ct, per[c + 1] * elem_per_ct
            if hi == lo:
                continue
            npol = 2 * (per[c + 1] - per[c])
            with torch.cuda.stream(s):
                x[lo:hi].copy_(host[lo:hi], non_blocking=True)
                plan.forward(x[lo:hi], X[lo:hi], npol, layout=lay, stream=s.cuda_stream)
                plan.inverse(X[lo:hi], x[lo:hi], npol, layout=lay, stream=s.cuda_stream)
                host[lo:hi].copy_(x[lo:hi], non_blocking=True)

    one_step()
    torch.cuda.synchronize()
    group.step("e2e warmup", lambda: None)
    group.barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(steps):
        one_step()
        for s in streams:
            torch.cuda.current_stream().wait_stream(s)
    ev1.record()
    torch.cuda.synchronize()
    secs = group.max_f64(ev0.elapsed_time(ev1) / 1000.0)
    limb_polys = sum(r[0] for r in group.gather_u64([polys * LIMBS]))  # whole job
    units = 2 * limb_polys * steps
    return {"value": units / secs, "unit": UNIT,
            "h2d_bytes_per_step": limb_polys * N * 8, "d2h_bytes_per_step": limb_polys * N * 8,
            "steps": steps, "chunks": chunks, "streams": len(streams),
            "timing": "CUDA events around the copy/compute streams, max over ranks"}


def run_sweep_large(args):
    """N = 2^18 .. 2^24 on one GPU, both prime families: forward and inverse
    of 4 limbs x a batch of about 1 GiB (u64) per buffer through the
    multi-pass kernels.  One JSON line per (bits, N): launch times, limb-
    transforms/s, and GB/s as 16N algorithmic bytes per limb-transform (the
    passes move 24N bytes at 2^18 with 32-bit words, 32N otherwise).  Not the
    headline bench line; --sweep-large selects it."""
    import torch

    import barracuda_b200 as bc

    torch.cuda.set_device(0)
    dev = bc.Device(0)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    sh = stream.cuda_stream
    hbm, peak_kind = peaks()
    for bits in (31, 60):
        for L in range(18, 25):
            n, limbs = 1 << L, 4
            batch = max(1, (1 << 27) // (n * limbs))
            qs = bc.ntt_primes(bits, n, limbs)
            plan = bc.NttPlan(dev, n, qs, [bc.negacyclic_root(q, n) for q in qs], mode=bc.NEGACYCLIC)
            x = torch.empty(limbs * batch * n, dtype=torch.int64, device="cuda")
            y, z = torch.empty_like(x), torch.empty_like(x)
            plan.fill_uniform(x, batch, seed=1, stream=sh)
            line = {"sweep": "large N, multi-pass kernels, 1 GPU", "N": n, "bits": bits, "limbs": limbs,
                    "batch": batch, "passes": 2 if (bits < 32 and L == 18) else 3,
                    "peak_gbs": hbm, "peak_kind": peak_kind}
            for name, fn, src, dst in (("forward", plan.forward, x, y), ("inverse", plan.inverse, y, z)):
                for _ in range(args.warmup):
                    fn(src, dst, batch, stream=sh)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                torch.cuda.synchronize()
                e0.record(stream)
                for _ in range(args.steps):
                    fn(src, dst, batch, stream=sh)
                e1.record(stream)
                torch.cuda.synchronize()
                ms = e0.elapsed_time(e1) / args.steps
                units = limbs * batch
                gbs = units * 16 * n / (ms / 1000.0) / 1e9
                line[name] = {"ms": ms, "limb_transforms_per_s": units / (ms / 1000.0), "gb_per_s": gbs,
                              "frac": gbs / hbm}
            line["round_trip_exact"] = bool(torch.equal(x, z))
            print(json.dumps(line), flush=True)
            del x, y, z
            plan.close()
    dev.close()


def run_sweep(args):
    """Config 4: for each N, forward and inverse of a [limb][poly][N] batch of
    about 2 GiB (u64) per GPU, sharded by limb across the ranks (each GPU
    owns a contiguous range of the limbs, 32 per GPU below N = 2^14, 16
    above).  One JSON line per N with the launch times (max over ranks) and
    the whole-job GB/s as a fraction of the measured HBM peak times the GPU
    count (16N bytes per limb-transform).  On one GPU it then adds lines
    for the coefficient-wise ops and the rotation / RNS ops.  Not the
    headline bench line; --sweep selects it."""
    import torch

    import barracuda_b200 as bc

    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    group = bc.ShardGroup("nccl", timeout=300.0, device=torch.device("cuda", local))
    try:
        _run_sweep(args, torch, bc, group, world, rank, local)
    finally:
        group.close()


def _run_sweep(args, torch, bc, group, world, rank, local):
    dev = bc.Device(local)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    sh = stream.cuda_stream
    hbm, peak_kind = peaks()
    for L in range(12, 18):
        n = 1 << L
        per_gpu = 32 if L < 14 else 16
        limbs_total = per_gpu * world
        begin, limbs = bc.partition(limbs_total, world, rank)
        batch = max(1, (1 << 28) // (n * per_gpu))
        qs = bc.ntt_primes(31, n, limbs_total)[begin:begin + limbs]
        plan = bc.NttPlan(dev, n, qs, [bc.negacyclic_root(q, n) for q in qs], mode=bc.NEGACYCLIC)
        lay = bc.Layout(limb_stride=batch * n, poly_stride=n)
        x = torch.empty(limbs * batch * n, dtype=torch.int64, device="cuda")
        y = torch.empty_like(x)
        plan.fill_uniform(x, batch, seed=1, layout=lay, stream=sh)
        line = {"sweep": f"config4 shape, {world} GPU(s), sharded by limb", "N": n, "n_gpus": world,
                "limbs_total": limbs_total, "limbs_per_gpu": per_gpu, "batch": batch,
                "peak_gbs": hbm, "peak_kind": peak_kind}
        for name, fn in (("forward", plan.forward), ("inverse", plan.inverse)):
            for _ in range(args.warmup):
                fn(x, y, batch, layout=lay, stream=sh)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            group.barrier()
            e0.record(stream)
            for _ in range(args.steps):
                fn(x, y, batch, layout=lay, stream=sh)
            e1.record(stream)
            torch.cuda.synchronize()
            ms = group.max_f64(e0.elapsed_time(e1)) / args.steps
            units = limbs_total * batch
            gbs = units * 16 * n / (ms / 1000.0) / 1e9
            line[name] = {"ms": ms, "limb_transforms_per_s": units / (ms / 1000.0),
                          "gb_per_s": gbs, "frac": gbs / (hbm * world)}
        if rank == 0:
            print(json.dumps(line), flush=True)
        del x, y
        plan.close()
    if world > 1:
        dev.close()
        return
    # coefficient-wise ops (FhePolyAdd / FhePolySub / FhePolyMul semantics), 24 bytes
    # per coefficient (read a, b; write c), both prime families
    for bits in (31, 60):
        n, limbs = 1 << 16, 16
        batch = (1 << 28) // (n * limbs)
        qs = bc.ntt_primes(bits, n, limbs)
        plan = bc.NttPlan(dev, n, qs, [bc.negacyclic_root(q, n) for q in qs], mode=bc.NEGACYCLIC)
        a = torch.empty(limbs * batch * n, dtype=torch.int64, device="cuda")
        b, c = torch.empty_like(a), torch.empty_like(a)
        plan.fill_uniform(a, batch, seed=1, stream=sh)
        plan.fill_uniform(b, batch, seed=2, stream=sh)
        line = {"sweep": "coefficient ops, 1 GPU", "N": n, "limbs": limbs, "batch": batch, "bits": bits,
                "peak_gbs": hbm, "peak_kind": peak_kind}
        for name in ("poly_add", "poly_sub", "poly_mul"):
            fn = getattr(plan, name)
            for _ in range(args.warmup):
                fn(a, b, c, batch, stream=sh)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record(stream)
            for _ in range(args.steps):
                fn(a, b, c, batch, stream=sh)
            e1.record(stream)
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / args.steps
            gbs = limbs * batch * 24 * n / (ms / 1000.0) / 1e9
            line[name] = {"ms": ms, "gb_per_s": gbs, "frac": gbs / hbm}
        print(json.dumps(line), flush=True)
        del a, b, c
        plan.close()
    # rotation (automorphism: 16 bytes per coefficient), modulus switch (16) and
    # base-2^16 decomposition into 3 digits (8 read + 24 written)
    for L in (12, 13, 14, 15, 16, 17):
        n, limbs = 1 << L, 16
        batch = (1 << 28) // (n * limbs)
        count = limbs * batch * n
        qs = bc.ntt_primes(31, n, limbs)
        plan = bc.NttPlan(dev, n, qs, [bc.negacyclic_root(q, n) for q in qs], mode=bc.NEGACYCLIC)
        a = torch.empty(count, dtype=torch.int64, device="cuda")
        b = torch.empty(count * (3 if L == 16 else 1), dtype=torch.int64, device="cuda")
        plan.fill_uniform(a, batch, seed=1, stream=sh)
        line = {"sweep": "rotation and rns ops, 1 GPU", "N": n, "limbs": limbs, "batch": batch,
                "peak_gbs": hbm, "peak_kind": peak_kind}
        ops = [("automorphism", lambda: plan.automorphism(a, b, batch, 2 * 1234 + 1, stream=sh), 16)]
        if L == 16:
            ops += [("modulus_switch", lambda: bc.modulus_switch(dev, a, b, count, qs[0], qs[1] >> 8,
                                                                 stream=sh), 16),
                    ("decompose_2^16_x3", lambda: bc.decompose(dev, a, b, count, 1 << 16, 3, stream=sh), 32)]
        for name, fn, bytes_per in ops:
            for _ in range(args.warmup):
                fn()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record(stream)
            for _ in range(args.steps):
                fn()
            e1.record(stream)
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / args.steps
            gbs = count * bytes_per / (ms / 1000.0) / 1e9
            line[name] = {"ms": ms, "gb_per_s": gbs, "frac": gbs / hbm}
        print(json.dumps(line), flush=True)
        del a, b
        plan.close()
    dev.close()


# --kernel-case: one kernel family alone on a small case (256 MiB per
# operand, larger than L2), for ncu captures of the kernels around the
# transform.  name -> (log2 N, limbs, kernel name, algorithmic bytes per word)
KERNEL_CASES = {
    "polymul": (15, 32, "k_polymul_fast", 40),       # NTT(B) into C, then the fused kernel
    "polymul_cyclic": (15, 32, "k_polymul_fast", 40),  # the same for a cyclic plan (primitive roots)
    "automorphism_smem": (13, 16, "k_automorph_smem", 16),
    "automorphism_cluster": (14, 16, "k_automorph_cluster", 16),
    "automorphism_gather": (16, 16, "k_automorph_gather", 16),
    "coeff_add": (16, 16, "k_coeff", 24),
    "coeff_mul": (16, 16, "k_coeff", 24),
    "pointwise": (16, 16, "k_pointwise", 24),
    "modulus_switch": (16, 16, "k_modulus_switch", 16),
    "decompose": (16, 16, "k_decompose", 32),            # base 2^16, 3 digits
    "forward": (16, 16, "k_ntt_fast", 16),               # the transform alone, for comparison
    "inverse": (16, 16, "k_ntt_fast", 16),
    "forward_mul": (16, 16, "k_ntt_mul_fast", 24),       # C = NTT(A) * B^
    "inverse_mul": (16, 16, "k_ntt_mul_fast", 24),       # C = INTT(A^ * B^)
    "forward_add": (16, 16, "k_ntt_mul_fast", 24),       # C = NTT(A) + B^, one launch
    "inverse_sub": (16, 16, "k_ntt_mul_fast", 24),       # C = INTT(A^ - B^), one launch
    "forward_then_add": (16, 16, "k_ntt_fast + k_coeff", 24),   # the same as two launches
    "sub_then_inverse": (16, 16, "k_coeff + k_ntt_fast", 24),
    "forward_large": (20, 4, "k_ntt_pass", 16),          # N = 2^20: three multi-pass launches
    "inverse_large": (20, 4, "k_ntt_pass", 16),
    "forward_13": (13, 32, "k_ntt_fast", 16),            # one CTA per polynomial (TMA staging with
                                                         # BARRACUDA_NTT_PERSISTENT=2)
    "inverse_13": (13, 32, "k_ntt_fast", 16),
    "forward_512": (9, 64, "k_ntt_smem", 16),            # below the cluster kernels: one CTA, stage per barrier
    "forward_unaligned": (16, 16, "k_glb_load + k_glb_stage + k_glb_store", 16),  # 8-byte aligned buffers
    "forward_w64": (16, 16, "k_ntt_fast", 16, 60),       # 64-bit words (primes below 2^60)
    "inverse_w64": (16, 16, "k_ntt_fast", 16, 60),
}


def run_kernel_case(args):
    """Warm-up + timed launches of one kernel family (KERNEL_CASES), one
    JSON line with the CUDA-event mean and the fraction of HBM peak."""
    import torch

    import barracuda_b200 as bc

    case = args.kernel_case
    logn, limbs, kernel, bytes_per_word = KERNEL_CASES[case][:4]
    bits = KERNEL_CASES[case][4] if len(KERNEL_CASES[case]) > 4 else 31
    torch.cuda.set_device(0)
    dev = bc.Device(0)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    sh = stream.cuda_stream
    hbm, peak_kind = peaks()
    n = 1 << logn
    words = 1 << 25
    batch = words // (n * limbs)
    qs = bc.ntt_primes(bits, n, limbs)
    psis = [bc.negacyclic_root(q, n) for q in qs]
    if case.endswith("_cyclic"):
        plan = bc.NttPlan(dev, n, qs, [p * p % q for p, q in zip(psis, qs)], mode=bc.CYCLIC)
    else:
        plan = bc.NttPlan(dev, n, qs, psis, mode=bc.NEGACYCLIC)
    # "_unaligned": operands start one word into their allocation (8-byte
    # aligned only), which the cluster kernels do not take
    off = 1 if case.endswith("_unaligned") else 0
    a = torch.empty(words + 2 * off, dtype=torch.int64, device="cuda")
    b = torch.empty_like(a)
    c = torch.empty(words * (3 if case == "decompose" else 1) + 2 * off, dtype=torch.int64, device="cuda")
    pa, pc = a.data_ptr() + 8 * off, c.data_ptr() + 8 * off
    plan.fill_uniform(pa, batch, seed=1, stream=sh)
    plan.fill_uniform(b, batch, seed=2, stream=sh)
    ops = {
        "polymul": lambda: plan.polymul(a, b, c, batch, stream=sh),
        "polymul_cyclic": lambda: plan.polymul(a, b, c, batch, stream=sh),
        "automorphism_smem": lambda: plan.automorphism(a, c, batch, 2469, stream=sh),
        "automorphism_cluster": lambda: plan.automorphism(a, c, batch, 2469, stream=sh),
        "automorphism_gather": lambda: plan.automorphism(a, c, batch, 2469, stream=sh),
        "coeff_add": lambda: plan.poly_add(a, b, c, batch, stream=sh),
        "coeff_mul": lambda: plan.poly_mul(a, b, c, batch, stream=sh),
        "pointwise": lambda: plan.pointwise_mul(a, b, c, batch, stream=sh),
        "modulus_switch": lambda: bc.modulus_switch(dev, a, c, words, qs[0], qs[1] >> 8, stream=sh),
        "decompose": lambda: bc.decompose(dev, a, c, words, 1 << 16, 3, stream=sh),
        "forward": lambda: plan.forward(a, c, batch, stream=sh),
        "inverse": lambda: plan.inverse(a, c, batch, stream=sh),
        "forward_large": lambda: plan.forward(a, c, batch, stream=sh),
        "inverse_large": lambda: plan.inverse(a, c, batch, stream=sh),
        "forward_13": lambda: plan.forward(a, c, batch, stream=sh),
        "inverse_13": lambda: plan.inverse(a, c, batch, stream=sh),
        "forward_512": lambda: plan.forward(a, c, batch, stream=sh),
        "forward_unaligned": lambda: plan.forward(pa, pc, batch, stream=sh),
        "forward_w64": lambda: plan.forward(a, c, batch, stream=sh),
        "inverse_w64": lambda: plan.inverse(a, c, batch, stream=sh),
        "forward_mul": lambda: plan.forward_mul(a, b, c, batch, stream=sh),
        "inverse_mul": lambda: plan.inverse_mul(a, b, c, batch, stream=sh),
        "forward_add": lambda: plan.forward_add(a, b, c, batch, stream=sh),
        "inverse_sub": lambda: plan.inverse_sub(a, b, c, batch, stream=sh),
        "forward_then_add": lambda: (plan.forward(a, c, batch, stream=sh),
                                     plan.poly_add(c, b, c, batch, stream=sh)),
        "sub_then_inverse": lambda: (plan.poly_sub(a, b, c, batch, stream=sh),
                                     plan.inverse(c, c, batch, stream=sh)),
    }
    fn = ops[case]
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    gbs = words * bytes_per_word / (ms / 1000.0) / 1e9
    print(json.dumps({"kernel_case": case, "kernel": kernel, "N": n, "bits": bits, "limbs": limbs, "batch": batch,
                      "words": words, "bytes_per_word": bytes_per_word, "ms": ms, "gb_per_s": gbs,
                      "frac": gbs / hbm, "peak_gbs": hbm, "peak_kind": peak_kind,
                      "launches_before_timed": args.warmup}), flush=True)
    plan.close()
    dev.close()


def run_op_latency(args):
    """Single synchronous calls of the reference op API at N = 4096 (q < 2^31),
    median over `--steps` calls after `--warmup`: (1) through the public op
    mirror (FheNtt.new(...).execute() and friends: output allocation, launch,
    wait), (2) through the C ABI into a preallocated output (launch and wait
    only).  One JSON line, microseconds per call."""
    import time

    import numpy as np

    import barracuda_b200 as bc
    from barracuda_b200 import _native as NN

    dev = bc.Device(0)
    n = 4096
    q = bc.ntt_prime(31, n, 0)
    w = pow(bc.negacyclic_root(q, n), 2, q)
    winv = pow(w, -1, q)
    rng = np.random.default_rng(1)
    a = bc.create_fhe_poly_tensor(rng.integers(0, q, n, dtype=np.uint64), dev)
    b = bc.create_fhe_poly_tensor(rng.integers(0, q, n, dtype=np.uint64), dev)
    out = bc.FheTensor(dev, 2 * n)
    lib = NN.lib()
    api = {
        "FheNtt": lambda: bc.FheNtt.new(a, n, q, w).execute(),
        "FheIntt": lambda: bc.FheIntt.new(a, n, q, winv).execute(),
        "FhePointwiseMul": lambda: bc.FhePointwiseMul.new(a, b, n, q).execute(),
        "FheFastPolyMul": lambda: bc.FheFastPolyMul.new(a, b, n, q, w).execute(),
    }
    cabi = {
        "FheNtt": lambda: lib.bc_fhe_ntt(dev.handle, a.ptr, 2 * n, n, q, w, out.ptr),
        "FheIntt": lambda: lib.bc_fhe_intt(dev.handle, a.ptr, 2 * n, n, q, winv, out.ptr),
        "FhePointwiseMul": lambda: lib.bc_fhe_pointwise_mul(dev.handle, a.ptr, 2 * n, b.ptr, 2 * n, n, q, out.ptr),
        "FheFastPolyMul": lambda: lib.bc_fhe_fast_poly_mul(dev.handle, a.ptr, 2 * n, b.ptr, 2 * n, n, q, w, out.ptr),
    }
    plan = bc.NttPlan(dev, n, [q], [w], mode=bc.CYCLIC)
    parts = {
        "ctx_sync_idle": lambda: lib.bc_ctx_sync(dev.handle),
        "plan_forward_and_sync": lambda: (lib.bc_ntt_forward(plan.handle, a.ptr, out.ptr, 1, None, None),
                                          lib.bc_ctx_sync(dev.handle))[1],
    }
    res = {"op_api_us": {}, "c_abi_us": {}, "parts_us": {}}
    steps = max(args.steps, 50)
    for key, table in (("op_api_us", api), ("c_abi_us", cabi), ("parts_us", parts)):
        for name, fn in table.items():
            for _ in range(max(args.warmup, 5)):
                r = fn()
                if key == "op_api_us":
                    r.free()
            ts = []
            for _ in range(steps):
                t0 = time.perf_counter()
                r = fn()
                ts.append((time.perf_counter() - t0) * 1e6)
                if key == "op_api_us":
                    r.free()
                else:
                    NN.check(r)
            res[key][name] = round(statistics.median(ts), 2)
    # the same calls from C (what a Rust or C caller sees, without Python's ctypes)
    probe = os.path.join(ROOT, "barracuda_b200", "lib", "bc_op_latency")
    c_level = None
    if os.path.exists(probe):
        r = subprocess.run([probe, str(max(steps, 200))], capture_output=True, text=True)
        if r.returncode == 0 and r.stdout.strip():
            c_level = json.loads(r.stdout.strip().splitlines()[-1])
    print(json.dumps({"op_latency": True, "N": n, "q_bits": 31, "calls": steps,
                      "timing": "host wall clock per synchronous call (perf_counter), median", **res,
                      "from_c": c_level}),
          flush=True)
    plan.close()
    dev.close()


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--strong", action="store_true", help="split 128 ciphertexts over the GPUs")
    ap.add_argument("--cts-total", type=int, default=CTS_PER_GPU)
    ap.add_argument("--cts", type=int, default=CTS_PER_GPU,
                    help="ciphertexts per GPU (weak scaling); smaller values make the profiling case")
    ap.add_argument("--e2e-steps", type=int, default=3, help="0 skips the end-to-end measurement")
    ap.add_argument("--e2e-chunks", type=int, default=32)
    ap.add_argument("--e2e-streams", type=int, default=2)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sweep", action="store_true",
                    help="per-N forward/inverse report (config 4 shape) instead of the bench line")
    ap.add_argument("--sweep-large", action="store_true",
                    help="per-N forward/inverse report for N = 2^18..2^24 (multi-pass kernels)")
    ap.add_argument("--op-latency", action="store_true",
                    help="single-call latency of the reference op API at N=4096 (not a bench line)")
    ap.add_argument("--kernel-case", choices=sorted(KERNEL_CASES),
                    help="time one kernel family on a small case (for ncu captures)")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        args.warmup = 3
    if args.kernel_case:
        run_kernel_case(args)
    elif args.op_latency:
        run_op_latency(args)
    elif args.sweep:
        run_sweep(args)
    elif args.sweep_large:
        run_sweep_large(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
