#!/usr/bin/env python
"""Key-switching throughput of the B200-native CKKS hybrid key switch.

Workload: N = 2^16, L = 35 ciphertext primes (one 58-bit
+ 34 x 42-bit), P = 5 x 60-bit special primes (alpha = 5, dnum = 7),
ternary secret of Hamming weight 192, Gaussian error sigma 3.2; a batch of 64
ciphertexts, ciphertext i rotated by step i+1 with its own Galois key (64 keys,
18.8 GB resident in HBM).  One step = the 64 rotations.  Inputs (2.3 GB of
ciphertexts + the keys) are far larger than the 126 MB L2, so no flush is
needed between steps.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0).  With N > 1 (torchrun), the ciphertext limbs
are sharded cyclically over the ranks (limb j on rank j % N) and the 64 key
switches are computed jointly: strong scaling, value = total key switches /
the slowest rank's time.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

LOG_N = 16
QBITS = [58] + [42] * 34
PBITS = [60] * 5
BATCH = 64
SCALE = 2.0 ** 40
METRIC = "key-switches/s at N=2^16,L=35 (rotation, hybrid KS dnum=7)"
# DRAM bytes (read + write) per key switch of each key-switch stage at config
# 3, from one ncu capture of a group of 4 key switches divided by 4
# (profiles/keyswitch_config3_kernels.md); a stage's launches summed.
PROFILED_TRAFFIC_SOURCE = ("constant from one ncu capture (profiles/keyswitch_config3_kernels.md), "
                           "not measured in this run")
# the kernels behind each stage of the serial profile (one stage timing per
# group of key switches brackets all of them)
STAGE_KERNELS = {
    "galois": "k_galois_ntt",
    "intt_input": "ntt_rows (inverse) + k_inv_cols_scaled",
    "modup_cols": "k_modup_cols",
    "modup_rows_ip": "k_modup_rows_ip: FP64 launch + integer launch on a side stream, concurrent",
    "intt_p": "k_inv_cols_scaled (the row pass is folded into k_modup_rows_ip)",
    "moddown_cols": "k_moddown_cols",
    "moddown_rows": "k_moddown_rows",
}
PROFILED_TRAFFIC = {
    "galois": 25.7e6, "intt_input": 55.3e6, "modup_cols": 133.5e6, "modup_rows_ip": 498.2e6,
    "intt_p": 5.3e6, "moddown_cols": 29.0e6, "moddown_rows": 160.7e6,
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=BATCH)
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--no-graph", action="store_true",
                    help="launch the batch directly instead of replaying its CUDA graph")
    ap.add_argument("--lanes", type=int, default=4,
                    help="execution lanes (streams + scratch) for the batched key switches")
    ap.add_argument("--group", type=int, default=8,
                    help="key switches each lane pushes through every launch together (1..8)")
    ap.add_argument("--mode", choices=["ib", "oa"], default="ib",
                    help="multi-GPU plan of the key-switch workload: input broadcast (limb-"
                         "sharded ciphertexts) or output aggregation (replicated ciphertexts, "
                         "digit-split inner product, all-reduce)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=["ks", "ntt", "hoisted", "matmul"], default="ks",
                    help="ks: config-3 rotations (default); ntt: config-2 batched NTT; "
                         "hoisted: config-4 hoisted linear transform; matmul: config-5 "
                         "BSGS matmul layer")
    ap.add_argument("--ntt-polys", type=int, default=128)
    ap.add_argument("--no-ntt", action="store_true",
                    help="leave the config-2 NTT record out of the default line")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# Config 2: standalone batched forward + inverse NTT
# ---------------------------------------------------------------------------
NTT_QBITS = [58] + [42] * 35  # config 2: one 58-bit + 35 x 42-bit primes, all 1 mod 2^17
NTT_METRIC = "NTT-coefficients/s (config 2, forward+inverse)"


def ntt_measure(polys, steps, warmup, rank, world, clocks=None):
    """Config 2 on this rank: 128 polynomials x 36 limbs (one 58-bit + 35 x
    42-bit primes, all 1 mod 2^17), N = 2^16, coefficients uniform in
    [0, q_i) from seed 1, batched forward then inverse transform, limbs
    sharded cyclically over the ranks (strong scaling).  Returns the timing
    record (max over ranks): NTT-coefficients/s of both directions over all
    ranks, and the forward transform's HBM roofline (each limb read and
    written once per direction: 16 N bytes)."""
    import torch
    import torch.distributed as dist
    from comp390project_b200 import KsContext, gen_primes

    dev = torch.cuda.current_device()
    q = gen_primes(LOG_N, NTT_QBITS)
    nl = len(range(rank, len(q), world))
    own = [q[j] for j in range(rank, len(q), world)]
    ctx = KsContext(LOG_N, own, [], device=dev)
    N = 1 << LOG_N
    P = polys
    g = torch.Generator(device="cuda")
    g.manual_seed(1 + rank)
    data = torch.empty((P, nl, N), dtype=torch.int64, device="cuda")
    for sl in range(nl):
        data[:, sl, :] = torch.randint(0, int(own[sl]), (P, N), generator=g, device="cuda",
                                       dtype=torch.int64)
    stream = torch.cuda.current_stream()
    for _ in range(warmup):
        ctx.ntt_forward(data, nl, 0, P)
        ctx.ntt_inverse(data, nl, 0, P)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    if clocks is not None:
        clocks.start()
        time.sleep(0.3)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(2 * steps + 1)]
    evs[0].record(stream)
    launches = 0
    for i in range(steps):
        ctx.ntt_forward(data, nl, 0, P)
        launches += ctx.last_launch_count()
        evs[2 * i + 1].record(stream)
        ctx.ntt_inverse(data, nl, 0, P)
        launches += ctx.last_launch_count()
        evs[2 * i + 2].record(stream)
    torch.cuda.synchronize()
    if clocks is not None:
        clocks.stop()
    fwd = sum(evs[2 * i].elapsed_time(evs[2 * i + 1]) for i in range(steps))
    inv = sum(evs[2 * i + 1].elapsed_time(evs[2 * i + 2]) for i in range(steps))
    ms = fwd + inv
    if world > 1:
        t = torch.tensor([ms, fwd, inv], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, fwd, inv = (float(x) for x in t.tolist())
    coeffs = 2 * P * len(q) * N * steps  # both directions, all ranks
    peak, peak_kind = measured_peaks()
    alg_per_launch = P * nl * 16 * N  # one direction on this rank
    f_ms, i_ms = fwd / steps, inv / steps
    achieved = alg_per_launch / (f_ms / 1000.0) / 1e9
    achieved_inv = alg_per_launch / (i_ms / 1000.0) / 1e9
    # pipe bound of the FP64 path: 8 FP64 instructions per butterfly, 64 FP64
    # lanes per SM (N/2 log N butterflies per limb transform)
    bfly = P * nl * (N // 2) * LOG_N
    ctx.close()
    del data
    return {
        "metric": NTT_METRIC, "value": coeffs / (ms / 1000), "unit": "coefficients/s",
        "ms_per_step": ms / steps, "steps": steps, "warmup": warmup, "launches": launches,
        "config": {"workload": "config2-ntt: %d polys x 36 limbs x 2^16" % P,
                   "parallelism": "limb-sharded x%d" % world,
                   "l2": "%.2f GB resident per rank, exceeds L2; no flush"
                         % (P * nl * N * 8 / 1e9)},
        "roofline": {"bound": "hbm", "kernel": "ntt_forward (column + row pass)",
                     "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": None, "peak_kind": peak_kind,
                     "launch_ms": f_ms, "inverse_ms": i_ms,
                     "inverse_achieved": achieved_inv, "inverse_frac": achieved_inv / peak,
                     "butterflies_per_launch": bfly,
                     "two_pass_cap": 0.5,
                     "note": "two HBM passes per direction: the algorithmic bytes count each "
                             "limb once, so a two-pass transform is capped at frac 0.5"},
    }


def run_ntt(args, rank, world):
    """--workload ntt: config 2 as its own bench line."""
    import torch
    dev = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(dev)
    clocks = ClockSampler(dev)
    rec = ntt_measure(args.ntt_polys, args.steps, args.warmup, rank, world, clocks)
    if rank == 0:
        line = {
            "metric": rec["metric"], "value": rec["value"], "unit": rec["unit"], "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": rec["ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u64",
            "data": "synthetic", "config": rec["config"], "roofline": rec["roofline"],
            "gpu_launches": rec["launches"], "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.rows = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.FIELDS,
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in self.rows:
            for i, n in enumerate(names):
                if r[5 + i].lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(self.rows)}


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def host_copy_probe(host_buf, dev_buf, rank, world, reps=2):
    """Host-side copy limit of this rank while every rank copies at once: the
    whole pinned host buffer to the device on one stream and the device
    buffer back to (the same) host memory on another, concurrently, as the
    end-to-end path's lanes do; GB/s per direction, max time over ranks."""
    import torch
    import torch.distributed as dist
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    nbytes = host_buf.numel() * host_buf.element_size()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e_in, e_out = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cur = torch.cuda.current_stream()
    e0.record(cur)
    s_in.wait_event(e0)
    s_out.wait_event(e0)
    scratch = torch.empty_like(dev_buf)
    for _ in range(reps):
        with torch.cuda.stream(s_in):
            scratch.copy_(host_buf, non_blocking=True)
        with torch.cuda.stream(s_out):
            host_buf.copy_(dev_buf, non_blocking=True)
    e_in.record(s_in)
    e_out.record(s_out)
    torch.cuda.synchronize()
    t_in, t_out = e0.elapsed_time(e_in), e0.elapsed_time(e_out)
    if world > 1:
        t = torch.tensor([t_in, t_out], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_in, t_out = (float(x) for x in t.tolist())
    del scratch
    return {"h2d_gbs": reps * nbytes / (t_in / 1000) / 1e9,
            "d2h_gbs": reps * nbytes / (t_out / 1000) / 1e9,
            "bytes_per_direction": reps * nbytes,
            "note": "pure pinned-memory copies, both directions at once on every rank, no "
                    "compute: the host-side limit of this rank's end-to-end path"}


# ---------------------------------------------------------------------------
# CPU baseline: the oracle port running the identical rotation key switch
# ---------------------------------------------------------------------------
CONFIG1 = (13, [60, 40, 40], [60])  # N=2^13, Q={60,40,40}, P={60}


def cpu_rotation_rate(n_rot: int, threads: int | None = None, cfg=None):
    """Rotation key switches per second of the oracle port on the host, over
    n_rot back-to-back rotations (key generation untimed).  threads=None: all
    host cores (OpenMP over limbs); cfg: (log_n, qbits, pbits), default
    config 3 (Hamming-weight-192 secret; config 1 uses a uniform ternary one)."""
    from oracle.oracle import Oracle, gen_primes, set_threads
    log_n, qbits, pbits = cfg or (LOG_N, QBITS, PBITS)
    threads = threads or os.cpu_count() or 1
    set_threads(threads)
    pr = gen_primes(log_n, list(qbits) + list(pbits))
    o = Oracle(log_n, pr[:len(qbits)], pr[len(qbits):])
    s = o.secret(0, 192 if cfg is None else 0)
    elt = o.galois_elt(1)
    key = o.keygen_galois(s, elt, 1001)
    rng = np.random.default_rng(5)
    z = rng.uniform(-1, 1, o.N // 2)
    ct = o.encrypt(s, o.encode(z, SCALE, len(qbits)), len(qbits), 7)
    t0 = time.perf_counter()
    for _ in range(n_rot):
        ct = o.apply_galois(ct, len(qbits), elt, key)
    dt = time.perf_counter() - t0
    set_threads(os.cpu_count() or 1)
    return n_rot / dt, threads, dt


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def cpu_baseline_config3():
    """The oracle port's rotation key switch on the host (about 15 s): config 3
    over 3 rotations on all cores (the reported value) and on one core, and
    config 1 over 20 rotations on all cores."""
    rate, cores, dt = cpu_rotation_rate(3)
    rate1, _, dt1 = cpu_rotation_rate(3, threads=1)
    rc1, _, dtc1 = cpu_rotation_rate(20, cfg=CONFIG1)
    return {"value": rate, "unit": "key-switches/s", "cores": cores, "kind": "port",
            "cpu_model": cpu_model(),
            "sample": "3 rotation key switches at config 3 on the host (%.1f s), oracle/ C++ "
                      "port with OpenMP over limbs" % dt,
            "single_thread": {"value": rate1, "cores": 1,
                              "sample": "3 rotations at config 3 on one core (%.1f s)" % dt1},
            "config1": {"value": rc1, "cores": cores,
                        "sample": "20 rotations at config 1 (N=2^13, Q={60,40,40}, P={60}) "
                                  "(%.2f s)" % dtc1}}


# Per-direction NVLink bandwidth of a peer copy measured on this pool's B200s
# (900 GB/s nominal per direction per GPU).
NVLINK_GBS = 770.0
NVLINK_NOMINAL_GBS = 900.0  # NVLink 5, per direction per GPU


def collective_roofline(prof, n_ks, L, alpha, world, N, oa=False, packed=False):
    """NVLink roofline of the collectives from the serial profile.  Input
    broadcast: per key switch a rank receives the other ranks' padded shares
    of the coefficient-form input ((G-1) ceil(L/G) limbs) and of the
    special-prime limbs of cx ((G-1) 2 max_r |P limbs of r| limbs); with
    42-bit packing (`packed`) a rank's share of the input is one whole limb
    plus ceil(L/G) - 1 limbs of 11/16 of the size.  Output aggregation: the
    all-reduce of cx (2 (L+alpha) limbs), which a ring all-reduce moves as
    2 (G-1)/G of the buffer into every rank."""
    ms, calls = prof.get("collective", (0.0, 0))
    if world <= 1 or ms <= 0 or n_ks <= 0:
        return None
    if oa:
        recv = 2 * (world - 1) * 2 * (L + alpha) * N * 8 // world
    else:
        coef_ml = -(-L // world)
        max_p_own = max(sum(1 for i in range(alpha) if (L + i) % world == r)
                        for r in range(world))
        share = (1 + (coef_ml - 1) * 11 / 16) if packed else coef_ml
        recv = int((world - 1) * (share + 2 * max_p_own) * N * 8)
    t = ms / n_ks / 1000.0
    ach = recv / t / 1e9
    return {"bound": "nvlink", "bytes_received_per_ks": recv, "ms_per_ks": ms / n_ks,
            "calls_per_ks": calls / n_ks, "achieved": ach, "peak": NVLINK_GBS, "unit": "GB/s",
            "frac": ach / NVLINK_GBS,
            "peak_kind": "this pool's measured peer copy per direction (serial collectives, "
                         "latency included)",
            "peak_nominal": NVLINK_NOMINAL_GBS, "frac_nominal": ach / NVLINK_NOMINAL_GBS}


# ---------------------------------------------------------------------------
# Config 4: hoisted rotations + plaintext diagonals (CoeffToSlot-style)
# ---------------------------------------------------------------------------
HOIST_QL = 25  # "level 24": 25 ciphertext limbs remain, 5 full digits
HOIST_STEPS = list(range(1, 33)) + [32 * k for k in range(1, 9)]


def run_hoisted(args, rank, world):
    """out = sum_i diag_i * rot_{s_i}(ct) over the 40 rotations of config 4 (baby
    steps 1..32, giant steps 32k, k = 1..8; the step-32 rotation is done twice
    with two diagonals), one ModUp and one ModDown shared by all 40 (double
    hoisting).  Diagonals: NTT-form plaintexts in the extended basis with
    uniform residues (the cost of an encoded complex diagonal)."""
    import torch
    import torch.distributed as dist
    from comp390project_b200 import KS_KEY_GALOIS, KsContext, gen_primes, secret_generate

    dev = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(dev)
    pr = gen_primes(LOG_N, QBITS + PBITS)
    q, p = pr[:len(QBITS)], pr[len(QBITS):]
    Ql = HOIST_QL
    if world > 1:
        ctx = KsContext.from_process_group(LOG_N, q, p, device=dev, max_batch=1)
    else:
        ctx = KsContext(LOG_N, q, p, device=dev, max_batch=1)
    N = 1 << LOG_N
    nloc = ctx.n_local_limbs(Ql)
    s = secret_generate(LOG_N, 0, 192)
    for st in sorted(set(HOIST_STEPS)):
        ctx.key_generate(KS_KEY_GALOIS, ctx.galois_elt(st), s, 3000 + st)
    g = torch.Generator(device="cuda")
    g.manual_seed(33 + rank)
    R = len(HOIST_STEPS)
    # this rank's output limbs: owned Q limbs, then owned P limbs (key index L + i)
    p_own = [i for i in range(len(p)) if (len(q) + i) % world == rank]
    n_out = nloc + len(p_own)
    ct = torch.empty((2, nloc, N), dtype=torch.int64, device="cuda")
    diags = torch.empty((R, n_out, N), dtype=torch.int64, device="cuda")
    for sl in range(nloc):
        j = rank + sl * world
        ct[:, sl] = torch.randint(0, int(q[j]), (2, N), generator=g, device="cuda",
                                  dtype=torch.int64)
        diags[:, sl] = torch.randint(0, int(q[j]), (R, N), generator=g, device="cuda",
                                     dtype=torch.int64)
    for k, i in enumerate(p_own):
        diags[:, nloc + k] = torch.randint(0, int(p[i]), (R, N), generator=g, device="cuda",
                                           dtype=torch.int64)
    out = torch.empty_like(ct)
    dl = [diags[i] for i in range(R)]
    stream = torch.cuda.current_stream()

    def step():
        ctx.linear_transform_hoisted(ct, Ql, HOIST_STEPS, dl, out, stream=stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(dev)
    clocks.start()
    time.sleep(0.3)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    launches = 0
    for _ in range(args.steps):
        step()
        launches += ctx.last_launch_count()
    ev1.record(stream)
    torch.cuda.synchronize()
    clocks.stop()
    ms = ev0.elapsed_time(ev1)
    # serial per-stage times of one transform
    ctx.profile_enable(True)
    step()
    torch.cuda.synchronize()
    ctx.profile_enable(False)
    prof = ctx.profile_read()
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = R * args.steps / (ms / 1000.0)
    # end to end: the input ciphertext up, the result down, every step
    host_in = torch.empty(ct.shape, dtype=torch.int64).pin_memory()
    host_in.copy_(ct)
    host_out = torch.empty_like(host_in).pin_memory()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(max(1, args.e2e_steps)):
        ct.copy_(host_in, non_blocking=True)
        step()
        host_out.copy_(out, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    ems = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ems], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ems = float(t.item())
    nbytes = host_in.numel() * 8
    e2e = {"value": R * max(1, args.e2e_steps) / (ems / 1000.0), "unit": "key-switches/s",
           "h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": nbytes}
    # roofline: the per-rotation inner product streams both key polys of every
    # digit (the shared extended digits stay in L2), the diagonal, and reads +
    # writes the two accumulators: (2 beta + 1 + 4) n_out limbs
    beta = (Ql + len(p) - 1) // len(p)
    U = 8 * N
    alg_ip = (2 * beta * n_out + n_out + 4 * n_out) * U
    ip_ms, n_ip = prof.get("inner_product", (0.0, 0))
    peak, peak_kind = measured_peaks()
    ach = alg_ip * n_ip / (ip_ms / 1000.0) / 1e9 if n_ip > 0 and ip_ms > 0 else None
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle.oracle import Oracle, set_threads
        threads = os.cpu_count() or 1
        set_threads(threads)
        o = Oracle(LOG_N, q, p)
        so = o.secret(0, 192)
        keys = [o.keygen_galois(so, o.galois_elt(st), 3000 + st) for st in (1, 2)]
        rng = np.random.default_rng(3)
        cth = np.stack([np.stack([rng.integers(0, int(q[j]), size=N, dtype=np.uint64)
                                  for j in range(Ql)]) for _ in range(2)])
        t0 = time.perf_counter()
        o.rotate_hoisted(cth, Ql, [o.galois_elt(1), o.galois_elt(2)], keys)
        dt = time.perf_counter() - t0
        cpu = {"value": 2 / dt, "unit": "key-switches/s", "cores": threads, "kind": "port",
               "sample": "2 hoisted rotations at config 4 on the host (%.1f s, one shared "
                         "ModUp), oracle/ C++ port with OpenMP over limbs" % dt}
    if rank == 0:
        line = {
            "metric": "key-switches/s (config 4: hoisted linear transform, 40 rotations)",
            "value": value, "unit": "key-switches/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "u64", "data": "synthetic",
            "config": {"workload": "config4-hoisted: 1 ciphertext at Ql=25, 40 rotations "
                                   "(steps 1..32, 32k k=1..8) x plaintext diagonals",
                       "N": N, "Ql": Ql, "alpha": len(p), "digits": beta,
                       "parallelism": "limb-sharded x%d" % world,
                       "l2": "keys (11.5 GB) stream from HBM every step; no flush"},
            "roofline": {"bound": "hbm", "kernel": "k_inner_product_acc (per rotation)",
                         "achieved": ach, "peak": peak, "unit": "GB/s",
                         "frac": (ach / peak) if ach else None, "traffic": None,
                         "peak_kind": peak_kind},
            "stages_ms_serial": {k: v[0] for k, v in prof.items()},
            "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches,
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    ctx.close()


# ---------------------------------------------------------------------------
# Config 5: BERT-base-shaped BSGS ciphertext x plaintext matmul
# ---------------------------------------------------------------------------
MM_TOKENS, MM_D = 128, 768


def mac_alg_bytes(lay, g_lo, g_hi, n_limbs, N):
    """Algorithmic DRAM bytes of the plaintext-product passes of one layer
    (k_mac_plain): per pass over <= 4 giant steps, every baby-step
    ciphertext (2 polys) and each giant step's diagonals are read once, and
    each giant step's partial sum (2 polys) is written; a pass over more than
    64 terms also re-reads its outputs."""
    terms = lay.n_in * lay.n_baby
    total = 0
    for _o in range(lay.n_out):
        for g0 in range(g_lo, g_hi, 4):
            ng = min(4, g_hi - g0)
            for m0 in range(0, terms, 64):
                nt = min(64, terms - m0)
                total += (2 * nt + ng * nt + 2 * ng + (2 * ng if m0 else 0)) * n_limbs * N * 8
    return total


def run_matmul(args, rank, world):
    """One BERT-base matmul layer per step: Y = X W, X 128 x 768 encrypted
    (3 ciphertexts, 256 features x 128 tokens each, column-major packing),
    W 768 x 768 as 2304 NTT-form diagonals (uniform residues: the cost of
    encoded diagonals), BSGS with B = G = 16 (45 hoisted baby-step and 45
    giant-step key switches).  Ring and primes of config 3 at Ql = 35.  With
    N > 1 ranks the giant steps and baby steps are split over the ranks
    (comp390project_b200.matmul.matmul_giant_parallel): strong scaling."""
    import torch
    import torch.distributed as dist
    from comp390project_b200 import KS_KEY_GALOIS, KsContext, gen_primes, matmul, secret_generate

    dev = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(dev)
    pr = gen_primes(LOG_N, QBITS + PBITS)
    q, p = pr[:len(QBITS)], pr[len(QBITS):]
    Ql = len(QBITS)
    N = 1 << LOG_N
    lay = matmul.layout(N // 2, MM_TOKENS, MM_D, MM_D)
    ctx = KsContext(LOG_N, q, p, device=dev, max_batch=args.lanes)
    s = secret_generate(LOG_N, 0, 192)
    g_lo, g_hi = matmul.giant_ranges(lay.n_giant, world)[rank]
    mine = matmul.baby_assignment(lay, world, rank)
    need = sorted({b * lay.unit for _, b in mine} |
                  {g * lay.n_baby * lay.unit for g in range(max(g_lo, 1), g_hi)})
    for st in need:
        ctx.key_generate(KS_KEY_GALOIS, ctx.galois_elt(st), s, 4000 + st)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(4 + rank)
    xs = torch.empty((lay.n_in, 2, Ql, N), dtype=torch.int64, device="cuda")
    # only this rank's giant steps' diagonals are resident; the others point
    # at one unread placeholder
    used = [((o * lay.n_in + i) * lay.n_giant + g) * lay.n_baby + b
            for o in range(lay.n_out) for i in range(lay.n_in)
            for g in range(g_lo, g_hi) for b in range(lay.n_baby)]
    diag = torch.empty((max(len(used), 1), Ql, N), dtype=torch.int64, device="cuda")
    for j in range(Ql):
        xs[:, :, j] = torch.randint(0, int(q[j]), (lay.n_in, 2, N), generator=gen, device="cuda",
                                    dtype=torch.int64)
        diag[:, j] = torch.randint(0, int(q[j]), (diag.shape[0], N), generator=gen,
                                   device="cuda", dtype=torch.int64)
    pts = [diag[0]] * lay.n_diagonals
    for k, idx in enumerate(used):
        pts[idx] = diag[k]
    ys = torch.empty((lay.n_out, 2, Ql, N), dtype=torch.int64, device="cuda")
    stream = torch.cuda.current_stream()
    if world == 1:
        work = torch.empty(ctx.bsgs_workspace_words(Ql, lay.n_in, lay.n_baby), dtype=torch.int64,
                           device="cuda")
        xl, yl = [xs[i] for i in range(lay.n_in)], [ys[o] for o in range(lay.n_out)]

        def step():
            ctx.bsgs_matmul(xl, Ql, lay.unit, lay.n_baby, lay.n_giant, pts, yl, work)
    else:
        def step():
            matmul.matmul_giant_parallel(ctx, [xs[i] for i in range(lay.n_in)], Ql, lay, pts, ys)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(dev)
    clocks.start()
    time.sleep(0.3)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    l0 = ctx.total_launch_count()
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    clocks.stop()
    launches = ctx.total_launch_count() - l0
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    n_ks = lay.n_in * (lay.n_baby - 1) + lay.n_out * (lay.n_giant - 1)
    value = n_ks * args.steps / (ms / 1000.0)
    # serial per-stage times of one layer (this rank)
    ctx.profile_enable(True)
    step()
    torch.cuda.synchronize()
    ctx.profile_enable(False)
    prof = ctx.profile_read()
    # end to end: the activations up, the product down, every step
    host_in = torch.empty(xs.shape, dtype=torch.int64).pin_memory()
    host_in.copy_(xs)
    host_out = torch.empty(ys.shape, dtype=torch.int64).pin_memory()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(max(1, args.e2e_steps)):
        xs.copy_(host_in, non_blocking=True)
        step()
        host_out.copy_(ys, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    ems = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ems], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ems = float(t.item())
    e2e = {"value": n_ks * max(1, args.e2e_steps) / (ems / 1000.0), "unit": "key-switches/s",
           "layer_ms": ems / max(1, args.e2e_steps),
           "h2d_bytes_per_step": host_in.numel() * 8, "d2h_bytes_per_step": host_out.numel() * 8}
    peak, peak_kind = measured_peaks()
    mac_ms, n_mac = prof.get("plain_mac", (0.0, 0))
    alg = mac_alg_bytes(lay, g_lo, g_hi, Ql, N)
    ach = alg / (mac_ms / 1000.0) / 1e9 if mac_ms > 0 else None
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = matmul_cpu_baseline(q, p, lay, n_ks)
    if rank == 0:
        line = {
            "metric": "key-switches/s (config 5: BERT-base 128x768x768 BSGS matmul layer)",
            "value": value, "unit": "key-switches/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "u64", "data": "synthetic",
            "config": {"workload": "config5-matmul: X 128x768 (3 ciphertexts) x W 768x768 "
                                   "(2304 diagonals), BSGS B=G=16, %d key switches" % n_ks,
                       "N": N, "Ql": Ql, "alpha": len(p),
                       "parallelism": "giant-step split x%d (all-gather of baby steps, "
                                      "all-reduce of partial products)" % world,
                       "l2": "diagonals (%.1f GB on this rank) stream from HBM every step; "
                             "no flush" % (diag.numel() * 8 / 1e9)},
            "roofline": {"bound": "hbm", "kernel": "k_mac_plain (plaintext products)",
                         "achieved": ach, "peak": peak, "unit": "GB/s",
                         "frac": (ach / peak) if ach else None, "traffic": None,
                         "alg_bytes_per_layer": alg, "launches_per_layer": n_mac,
                         "peak_kind": peak_kind},
            "stages_ms_serial": {k: v[0] for k, v in prof.items()},
            "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches,
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    ctx.close()


def matmul_cpu_baseline(q, p, lay, n_ks):
    """Bounded sample of the config-5 layer on the host cores (oracle/ C++
    port, OpenMP over limbs): 3 hoisted baby-step rotations of one input, one
    giant-step rotation and one plaintext-product term, scaled to a layer
    (n_in (B-1) / 3 hoisted groups, n_out (G-1) giant steps, n_diagonals
    terms)."""
    from oracle.oracle import Oracle, set_threads
    threads = os.cpu_count() or 1
    set_threads(threads)
    o = Oracle(LOG_N, q, p)
    Ql = len(q)
    N = 1 << LOG_N
    so = o.secret(0, 192)
    rng = np.random.default_rng(5)
    x = np.stack([np.stack([rng.integers(0, int(q[j]), size=N, dtype=np.uint64)
                            for j in range(Ql)]) for _ in range(2)])
    pt = np.stack([rng.integers(0, int(q[j]), size=N, dtype=np.uint64) for j in range(Ql)])
    bs = lay.baby_steps()[:3]
    keys = {st: o.keygen_galois(so, o.galois_elt(st), 4000 + st) for st in bs}
    gs = lay.giant_steps()[0]
    keys[gs] = o.keygen_galois(so, o.galois_elt(gs), 4000 + gs)
    t0 = time.perf_counter()
    o.rotate_hoisted(x, Ql, [o.galois_elt(st) for st in bs], [keys[st] for st in bs])
    t_h = time.perf_counter() - t0
    t0 = time.perf_counter()
    o.apply_galois(x, Ql, o.galois_elt(gs), keys[gs])
    t_g = time.perf_counter() - t0
    t0 = time.perf_counter()
    o.bsgs_matmul([x], Ql, lay.unit, 1, 1, [pt], {})
    t_m = time.perf_counter() - t0
    layer = (lay.n_in * (lay.n_baby - 1) / 3) * t_h + lay.n_out * (lay.n_giant - 1) * t_g + \
        lay.n_diagonals * t_m
    return {"value": n_ks / layer, "unit": "key-switches/s", "cores": threads, "kind": "port",
            "layer_s": layer,
            "sample": "3 hoisted rotations (%.2f s), 1 rotation (%.2f s) and 1 plaintext-product "
                      "term (%.3f s) of the layer on the host, scaled to %d hoisted groups, %d "
                      "giant steps and %d terms; oracle/ C++ port with OpenMP over limbs"
                      % (t_h, t_g, t_m, lay.n_in * (lay.n_baby - 1) // 3,
                         lay.n_out * (lay.n_giant - 1), lay.n_diagonals)}


def run_reference(args, rank, world):
    """--impl reference: the oracle port of the reference path on the host cores."""
    if rank != 0:
        return
    from oracle.oracle import Oracle, gen_primes, set_threads
    threads = os.cpu_count() or 1
    set_threads(threads)
    pr = gen_primes(LOG_N, QBITS + PBITS)
    o = Oracle(LOG_N, pr[:len(QBITS)], pr[len(QBITS):])
    s = o.secret(0, 192)
    rng = np.random.default_rng(5)
    z = rng.uniform(-1, 1, o.N // 2)
    ct = o.encrypt(s, o.encode(z, SCALE, len(QBITS)), len(QBITS), 7)
    keys = {}
    times = []
    for it in range(args.warmup + args.steps):
        step = (it % BATCH) + 1
        elt = o.galois_elt(step)
        if elt not in keys:
            keys = {elt: o.keygen_galois(s, elt, 1000 + step)}
        t0 = time.perf_counter()
        ct = o.apply_galois(ct, len(QBITS), elt, keys[elt])
        dt = time.perf_counter() - t0
        if it >= args.warmup:
            times.append(dt)
    total = sum(times)
    value = len(times) / total
    line = {
        "metric": METRIC, "value": value, "unit": "key-switches/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * total / len(times),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u64",
        "data": "synthetic", "impl": "reference",
        "config": {"workload": "config3-rotation", "N": 1 << LOG_N, "L": len(QBITS),
                   "alpha": len(PBITS), "dnum": 7, "sample": "one rotation key switch per step"},
        "cpu_baseline": {"value": value, "unit": "key-switches/s", "cores": threads,
                         "kind": "port",
                         "sample": "%d rotation key switches at config 3 (oracle/ C++ port, "
                                   "OpenMP over limbs)" % len(times)},
        "e2e": {"value": value, "unit": "key-switches/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# Our arm
# ---------------------------------------------------------------------------
def run_ours(args, rank, world):
    import torch
    import torch.distributed as dist
    from comp390project_b200 import (KS_KEY_GALOIS, KS_MODE_INPUT_BROADCAST,
                                     KS_MODE_OUTPUT_AGGREGATION, KsContext, gen_primes,
                                     secret_generate)

    dev = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(dev)
    pr = gen_primes(LOG_N, QBITS + PBITS)
    q, p = pr[:len(QBITS)], pr[len(QBITS):]
    L = len(q)
    oa = args.mode == "oa" and world > 1
    mode = KS_MODE_OUTPUT_AGGREGATION if oa else KS_MODE_INPUT_BROADCAST
    if world > 1:
        ctx = KsContext.from_process_group(LOG_N, q, p, device=dev, mode=mode,
                                           max_batch=args.lanes, batch_group=args.group)
    else:
        ctx = KsContext(LOG_N, q, p, device=dev, max_batch=args.lanes, batch_group=args.group)
    N = 1 << LOG_N
    # output aggregation: every rank holds the whole ciphertext
    nloc = L if oa else ctx.n_local_limbs(L)
    B = args.batch
    steps_of = [i + 1 for i in range(B)]
    # keys: one Galois key per rotation step, generated on the device
    s = secret_generate(LOG_N, 0, 192)
    for st in steps_of:
        ctx.key_generate(KS_KEY_GALOIS, ctx.galois_elt(st), s, 1000 + st)
    torch.cuda.synchronize()
    # ciphertexts: uniform residues per owned limb (a fresh encryption is
    # uniform in this distribution); [B][2][nloc][N]
    g = torch.Generator(device="cuda")
    g.manual_seed(1234 + rank)
    cts = torch.empty((B, 2, nloc, N), dtype=torch.int64, device="cuda")
    for sl in range(nloc):
        j = sl if oa else rank + sl * world
        cts[:, :, sl, :] = torch.randint(0, int(q[j]), (B, 2, N), generator=g, device="cuda",
                                         dtype=torch.int64)
    views = [cts[i] for i in range(B)]
    stream = torch.cuda.current_stream()

    def step():
        ctx.rotate_batch(views, steps_of, L, stream=stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # the batch as one CUDA graph (every kernel and NCCL call of the 64 key
    # switches over all lanes), replayed once per step
    graph, launches_per_step = None, ctx.last_launch_count()
    if not args.no_graph:
        stream = torch.cuda.Stream()
        torch.cuda.synchronize()
        ctx.graph_capture_begin(stream)
        ctx.rotate_batch(views, steps_of, L, stream=stream)
        launches_per_step = ctx.last_launch_count()
        graph = ctx.graph_capture_end(stream)
        graph.launch(stream, dev)  # one untimed replay
        torch.cuda.synchronize()

        def step():
            graph.launch(stream, dev)
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(dev)
    clocks.start()
    time.sleep(0.3)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ev0.record(stream)
    torch.cuda.nvtx.range_push("ks_timed")
    launches = 0
    for _ in range(args.steps):
        step()
        launches += launches_per_step
    ev1.record(stream)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    clocks.stop()
    ms = ev0.elapsed_time(ev1)
    # Per-kernel times come from a serial pass right after the timed region
    # (one group of key switches at a time on one stream, CUDA events around
    # every stage), because in the timed region the lanes overlap.  A batch
    # of exactly one group runs on lane 0 alone.
    gsz = max(1, args.group)
    n_prof = max(1, min(B, 8) // gsz) * gsz
    ctx.profile_enable(True)
    # NVTX range "ks_serial" lets a profiler select exactly these launches
    # (ncu --nvtx --nvtx-include "ks_serial/").
    torch.cuda.nvtx.range_push("ks_serial")
    for i0 in range(0, n_prof, gsz):
        ctx.rotate_batch(views[i0:i0 + gsz], steps_of[i0:i0 + gsz], L, stream=stream)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    ctx.profile_enable(False)
    prof = ctx.profile_read()
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    total_ks = B * args.steps
    value = total_ks / (ms / 1000.0)

    # dominant compute stage and its roofline (two-pass NTT counted as one
    # transform); the collectives have their own NVLink roofline below
    stages = {k: v for k, v in prof.items() if v[1] > 0}
    prof_ks = n_prof
    dom = max((k for k in stages if k != "collective"), key=lambda k: stages[k][0])
    per_launch_ms = stages[dom][0] / stages[dom][1]
    QlP = L + len(p)
    beta = 7
    U = 8 * N
    alpha = len(p)
    if oa:
        # every output limb on every rank, over this rank's digits d = rank mod G
        n_out, n_q = QlP, L
        my_digits = list(range(rank, beta, world))
        n_dig = len(my_digits)
        n_in = sum(min(alpha, L - d * alpha) for d in my_digits)  # limbs of those digits
        n_p_own = alpha
    else:
        n_out = len(range(rank, L, world)) + sum(1 for i in range(alpha)
                                                 if (L + i) % world == rank)
        n_q = nloc
        n_dig, n_in = beta, n_q
        n_p_own = n_out - n_q
    # Algorithmic bytes per key switch on this rank (U = one limb): compulsory
    # inputs once + outputs once of each stage (twiddle/constant tables excluded).
    n_jobs = n_dig * n_out - n_in  # extended limbs produced by ModUp (own digit limbs are copies)
    alg = {
        "galois": 2 * n_q * U,  # c0 -> g0 (c1 is read through the automorphism later)
        "intt_input": 2 * n_in * U,
        "modup_cols": ((n_in if oa else L) + n_jobs) * U,
        # extended limbs (column pass done) + own-digit input limbs, both key
        # polys of every digit, cx out
        "modup_rows_ip": (n_dig * n_out + 2 * n_dig * n_out + 2 * n_out) * U,
        "intt_p": 4 * n_p_own * U,
        "moddown_cols": (2 * alpha + 2 * n_q) * U,
        "moddown_rows": 7 * n_q * U,
    }
    peak, peak_kind = measured_peaks()
    # one launch of a stage serves a whole group of gsz key switches
    alg_launch = alg[dom] * gsz if dom in alg else None
    achieved = alg_launch / (per_launch_ms / 1000.0) / 1e9 if alg_launch else None
    # DRAM traffic per launch of the dominant kernel: not measurable without a
    # profiler, so it is the constant of one ncu capture of the same kernel at
    # the same workload (dram__bytes_read.sum + dram__bytes_write.sum, one key
    # switch) scaled to the group, named in traffic_source; one GPU only (the
    # capture is of the one-GPU launch)
    traffic = PROFILED_TRAFFIC.get(dom) * gsz if world == 1 and dom in PROFILED_TRAFFIC else None

    # end to end through the C ABI with host buffers: ks_rotate_batch_host on
    # pinned host ciphertexts (copy in, rotate, copy out, pipelined over the
    # lanes), every copy inside the timed region
    e2e = None
    if args.e2e_steps > 0:
        host_in = torch.empty_like(cts, device="cpu").pin_memory()
        host_in.copy_(cts)
        host_views = [host_in[i] for i in range(B)]
        ctx.rotate_batch_host(host_views, steps_of, L, stream=stream)  # warm-up
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.e2e_steps):
            ctx.rotate_batch_host(host_views, steps_of, L, stream=stream)
        e1.record(stream)
        torch.cuda.synchronize()
        ems = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ems], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ems = float(t.item())
        nbytes = host_in.numel() * 8
        e2e = {"value": B * args.e2e_steps / (ems / 1000.0), "unit": "key-switches/s",
               "h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": nbytes,
               "host_copy": host_copy_probe(host_in, cts, rank, world)}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_config3()
    # the context packs the input all-gather when every Q prime after q0 is below 2^42
    packed = not oa and world > 1 and all(int(x) < (1 << 42) for x in q[1:])
    nvlink = collective_roofline(prof, prof_ks, L, len(p), world, N, oa=oa, packed=packed)
    # the second half of the headline metric: config 2's NTT on the same GPUs
    # (every rank, after the key-switch measurements)
    ntt = None
    if not args.no_ntt:
        ntt = ntt_measure(args.ntt_polys, max(3, args.steps // 2), 3, rank, world)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "key-switches/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u64",
            "data": "synthetic",
            "config": {"workload": "config3-rotation: 64 ciphertexts, steps 1..64, 64 Galois keys",
                       "N": N, "L": L, "alpha": len(p), "dnum": beta, "batch": B,
                       "parallelism": "limb-sharded x%d (%s), %d lanes x groups of %d"
                                      % (world, "output aggregation" if oa else "input broadcast",
                                         args.lanes, args.group),
                       "cuda_graph": graph is not None,
                       "l2": "inputs (2.3 GB cts + 18.8 GB keys) exceed L2; no flush"},
            "roofline": {"bound": "hbm", "kernel": dom, "kernels": STAGE_KERNELS.get(dom),
                         "achieved": achieved, "peak": peak,
                         "unit": "GB/s", "frac": (achieved / peak) if achieved else None,
                         "traffic": traffic, "peak_kind": peak_kind,
                         "traffic_source": (PROFILED_TRAFFIC_SOURCE if traffic else None),
                         "alg_bytes": alg_launch, "ks_per_launch": gsz,
                         "launch_ms": per_launch_ms, "per_rank": world > 1},
            "collectives": nvlink,
            "ntt": ntt,
            "stages_ms_per_ks_serial": {k: v[0] / prof_ks for k, v in stages.items()},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches,
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    if graph is not None:
        graph.close()  # before the communicators go
    ctx.close()


def bind_to_gpu_numa(dev):
    """Restrict this process to the host cores NVML reports as closest to
    GPU `dev`, so that its pinned host buffers (first touched by this
    process) sit in that GPU's NUMA node and the end-to-end copies do not
    cross the socket interconnect.  Returns the number of cores kept, or None
    when NVML cannot say (the affinity is then left as it is)."""
    try:
        import pynvml
        pynvml.nvmlInit()
        try:
            h = pynvml.nvmlDeviceGetHandleByIndex(dev)
            n_words = (os.cpu_count() + 63) // 64
            mask = pynvml.nvmlDeviceGetCpuAffinity(h, n_words)
        finally:
            pynvml.nvmlShutdown()
        cpus = {w * 64 + b for w, m in enumerate(mask) for b in range(64) if (m >> b) & 1}
        cpus &= os.sched_getaffinity(0)
        if not cpus:
            return None
        os.sched_setaffinity(0, cpus)
        return len(cpus)
    except Exception:
        return None


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1 and args.impl == "ours":
        # one rank per GPU: keep each rank on its GPU's host cores (NUMA node)
        bind_to_gpu_numa(int(os.environ.get("LOCAL_RANK", 0)))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    if args.workload == "ntt":
        run_ntt(args, rank, world)
    elif args.workload == "hoisted":
        run_hoisted(args, rank, world)
    elif args.workload == "matmul":
        run_matmul(args, rank, world)
    else:
        run_ours(args, rank, world)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
