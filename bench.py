#!/usr/bin/env python3
"""bench.py -- device-timed throughput of the engine's hot path on 1..8 B200s.

    python bench.py --gpus N --steps K --warmup W [--workload hmult] [--impl reference]

One process per GPU (torchrun for N > 1); every rank owns its own batch (conversation
packs / ciphertext batches shard with no communication: weak scaling).  Rank 0 prints one
JSON line.  The timed region is bracketed by a barrier and a device synchronise on both
sides; device time comes from CUDA events recorded on the engine's own stream; the
reported time is the maximum over ranks.

Workload "hmult" (config 2 of the baseline, its HMult row): a batch of 64 ciphertext pairs
at N = 2^16, L = 20 (q0 60-bit + 19 x 45-bit), K = 4 x 60-bit special primes, dnum = 5;
one step = 64 x (EvalMult ct x ct + relinearise + RescaleInPlace).  The inputs (2.7 GB)
exceed the 126 MB L2, so no flush is needed between steps.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "fhe-ssm_b200"))
sys.path.insert(0, os.path.join(ROOT, "tests"))

CONF = dict(logN=16, L=20, K=4, alpha=4, hw=192)
BATCH = 64
METRIC = "HMult+relin+rescale ciphertexts/s aggregate (N=2^16, L=20, batch 64 per GPU)"


def peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        return {}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while active."""

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(args):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v, ws):
    if ws == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def rand_ct_words(rng, moduli, nl, N):
    return np.stack([np.stack([rng.integers(0, int(moduli[i]), N, dtype=np.uint64) for i in range(nl)])
                     for _ in range(2)])


# ------------------------------------------------------------------------ CPU oracle ----
def oracle_hmult_rate(moduli, key, nthreads, seconds, rng):
    """HMult+relin+rescale of the CPU oracle (single-threaded C) on `nthreads` host threads
    (ctypes releases the GIL), ciphertexts/s over a bounded sample."""
    from concurrent.futures import ThreadPoolExecutor

    from oracle_lib import Oracle, load
    L, K, N = CONF["L"], CONF["K"], 1 << CONF["logN"]
    o = Oracle(CONF["logN"], moduli[:L], moduli[L:], CONF["alpha"], load())
    a = rand_ct_words(rng, moduli, L, N)
    b = rand_ct_words(rng, moduli, L, N)

    def one(_):
        o.ct_rescale(o.ct_mul_relin(a, b, L, key), L)
        return 1

    done, t0 = 0, time.time()
    with ThreadPoolExecutor(nthreads) as ex:
        while time.time() - t0 < seconds or done == 0:
            done += sum(ex.map(one, range(nthreads)))
    return done / (time.time() - t0), done


# ------------------------------------------------------------------------------ main ----
def run_reference(args):
    ws, rank, local = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), 0
    if rank != 0:
        return 0
    rng = np.random.default_rng(7)
    # the chain and key words come from the same deterministic generator the engine uses;
    # generated on the CPU by the oracle so the reference arm needs no GPU
    from oracle_lib import Oracle, derive_seed, gen_chain, load
    lib = load()
    q, p = gen_chain(CONF["logN"], CONF["L"], 60, 45, CONF["K"], 60, lib)
    moduli = np.concatenate([q, p])
    o = Oracle(CONF["logN"], q, p, CONF["alpha"], lib)
    ms = (1).to_bytes(8, "little") + bytes(24)
    s = o.secret(derive_seed(lib, ms, 0xFFFFFFF1), CONF["hw"])
    se = o.secret_eval(s)
    s2 = np.stack([(se[m].astype(object) ** 2 % int(o.mods[m])).astype(np.uint64) for m in range(len(o.mods))])
    key = o.keygen_switch(s2, se, derive_seed(lib, ms, 2))
    nthreads = os.cpu_count() or 1
    rates = []
    for i in range(args.warmup + args.steps):
        r, n = oracle_hmult_rate(moduli, key, nthreads, 1.0, rng)
        if i >= args.warmup:
            rates.append(r)
    value = statistics.mean(rates)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "ciphertexts/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "ms_per_step": 1000.0 * BATCH * args.gpus / value, "dtype": "u64 (RNS residues)", "data": "synthetic",
        "config": {"workload": "config 2: HMult+relin+rescale, N=2^16, L=20, K=4, dnum=5", "batch": BATCH},
        "cpu_baseline": {"value": value, "unit": "ciphertexts/s", "cores": nthreads, "kind": "port",
                         "sample": f"{nthreads} ciphertexts per step on {nthreads} threads of the C oracle "
                                   "(OpenFHE, the reference's arithmetic library, is not installable here)"},
        "e2e": {"value": value, "unit": "ciphertexts/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="engine", choices=["engine", "reference"])
    ap.add_argument("--workload", default="hmult", choices=["hmult"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=64, help="ciphertexts per GPU per step (smaller for ncu captures)")
    args = ap.parse_args()
    global BATCH
    BATCH = args.batch
    if args.impl == "reference":
        return run_reference(args)
    ws, rank, local = dist_setup(args)
    import torch

    import fhessm
    torch.cuda.set_device(local)
    cx = fhessm.CryptoContext(device=local, **CONF)
    cx.KeyGen(seed=1 + rank)
    L, N = CONF["L"], 1 << CONF["logN"]
    rng = np.random.default_rng(100 + rank)
    host_a = [rand_ct_words(rng, cx.moduli, L, N) for _ in range(BATCH)]
    host_b = [rand_ct_words(rng, cx.moduli, L, N) for _ in range(BATCH)]
    A = [cx.ct_from_words(w, 0) for w in host_a]
    B = [cx.ct_from_words(w, 0) for w in host_b]
    stream = torch.cuda.ExternalStream(cx.stream_ptr(), device=local)

    def step():
        outs = []
        for a, b in zip(A, B):
            c = cx.EvalMult(a, b)
            cx.RescaleInPlace(c)
            outs.append(c)
        return outs

    for _ in range(args.warmup):
        step()
    cx.sync()
    barrier(ws)
    clk = ClockSampler(local)
    clk.start()
    l0 = cx.launches()
    cx.profile(True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cx.sync()
    barrier(ws)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    cx.sync()
    torch.cuda.synchronize()
    barrier(ws)
    clocks = clk.stop()
    ms = e0.elapsed_time(e1)
    prof = cx.profile_collect()
    cx.profile(False)
    launches = cx.launches() - l0
    ms_max = max_over_ranks(ms, ws)
    value = BATCH * ws * args.steps / (ms_max / 1000.0)

    # ---- end to end through the C-ABI with host buffers (import -> compute -> export)
    out_words = np.empty((2, L - 1, N), dtype=np.uint64)
    barrier(ws)
    t0 = time.time()
    for _ in range(max(1, args.steps // 2)):
        for wa, wb in zip(host_a, host_b):
            a, b = cx.ct_from_words(wa, 0), cx.ct_from_words(wb, 0)
            c = cx.EvalMult(a, b)
            cx.RescaleInPlace(c)
            out_words[...] = c.words()
    cx.sync()
    barrier(ws)
    e2e_s = max_over_ranks((time.time() - t0) / max(1, args.steps // 2), ws)
    e2e = {"value": BATCH * ws / e2e_s, "unit": "ciphertexts/s",
           "h2d_bytes_per_step": int(2 * BATCH * host_a[0].nbytes),
           "d2h_bytes_per_step": int(BATCH * out_words.nbytes)}

    # ---- roofline of the dominant kernel (by device time)
    pk = peaks()
    top = max(prof.items(), key=lambda kv: kv[1][1]) if prof else None
    roof = None
    if top:
        name, (nl_, tms, tbytes) = top
        achieved = tbytes / (tms / 1000.0) / 1e9
        peak = pk.get("hbm_gbs", 6650.0)
        traffic = None
        tf = os.path.join(ROOT, "profiles", "traffic.json")
        if os.path.exists(tf):
            traffic = json.load(open(tf)).get(name)
        roof = {"kernel": name, "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "traffic": traffic, "launches": nl_, "avg_launch_us": 1000.0 * tms / nl_,
                "peak_source": "MEASURED_PEAKS.json hbm_gbs (measured)" if "hbm_gbs" in pk else "fallback 6650"}
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        r, n = oracle_hmult_rate(cx.moduli, cx.key_words(0), 1, 10.0, rng)
        cpu = {"value": r, "unit": "ciphertexts/s", "cores": 1, "kind": "port",
               "sample": f"{n} HMult+relin+rescale of the C oracle, single thread, same shape"}
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "ciphertexts/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u64 (RNS residues)", "data": "synthetic",
            "config": {"workload": "config 2: HMult+relin+rescale, N=2^16, L=20 (q0 60b + 19x45b), K=4x60b, dnum=5",
                       "batch_per_gpu": BATCH, "parallelism": f"dp{ws} (independent batches)",
                       "l2": "inputs 2.7 GB per GPU > L2, no flush"},
            "gpu_launches": launches, "clocks": clocks, "e2e": e2e, "roofline": roof, "cpu_baseline": cpu,
            "kernels": {k: {"launches": v[0], "ms": v[1], "GB/s": v[2] / (v[1] / 1000.0) / 1e9 if v[1] else None}
                        for k, v in prof.items()},
        }
        print(json.dumps(line), flush=True)
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
