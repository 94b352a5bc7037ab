#!/usr/bin/env python3
"""bench.py -- device-timed throughput of the engine's hot path on 1..8 B200s.

    python bench.py --gpus N --steps K --warmup W [--workload 405m|hmult|rwkv7|...] [--impl reference]

One process per GPU (torchrun for N > 1); every rank owns its own pack of 64 conversations
(packs shard with no communication: weak scaling).  Rank 0 prints one JSON line.  The timed
region is bracketed by a barrier and a device synchronise on both sides; device time comes
from CUDA events recorded on the engine's own stream; the reported time is the max over ranks.

Workload "405m" (default; config 4 of the baseline): one encrypted decode pass of the 405M
polynomial SSM (24 layers, d 1024, dff 4096, 64 diagonal-decay channels per head x 16, tied
vocabulary 50,304) advancing 64 conversations by one token, with the recurrent state carried
encrypted and bootstrapped as needed.  Chain: N = 2^16, q0 60 bits, 13 x 45-bit user primes,
14 x 58-bit bootstrap primes, K = 4 x 60-bit special primes (logQP 1697), HW-192 secret.
Weights N(0, 0.02), polynomial coefficients U[-1, 1], seeded; tokens uniform, seeded.

Workload "hmult" (config 2, HMult row): 64 ciphertext pairs at N = 2^16, L = 20; one step =
64 x (EvalMult + relinearise + RescaleInPlace).

Workload "rwkv7" (config 5): one encrypted decode step of the RWKV-7 0.4B polynomial model (24
layers, d 1024, 16 heads of 64, d_ffn 4096, vocabulary 65,536) for 32 conversations (one
ciphertext in the contiguous channel layout), the wkv state carried encrypted as 64 row
ciphertexts per layer.  Sites: degree-7 Chebyshev series on intervals fitted to a calibration
run, Newton 1/sqrt from linear seeds.  Same chain as "405m".
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

METRIC_405M = "encrypted tokens/s aggregate, 405M poly-SSM, 64 conv/pass, 1/2/4/8 B200"
METRIC_HMULT = "HMult+relin+rescale ciphertexts/s aggregate (N=2^16, L=20, batch 64 per GPU)"
METRIC_RWKV7 = "encrypted tokens/s aggregate, RWKV-7 0.4B polynomial model, 32 conv/pass"
RWKV7_LANES = 32
# EvalMod of the model's bootstraps: degree-31 interpolant + 4 double angles.  Same 10 levels as
# config 3's degree 59 + 3, 8 fewer ciphertext products per bootstrap; bootstrap error 6.6e-5
# (vs 4.5e-5), 405M logits relErrRms 3-4e-4 either way.
BOOT_EVALMOD = (24.0, 31, 4)
MODEL_CTX = dict(logN=16, L=28, K=4, alpha=4, hw=192, boot_primes=14)
HMULT_CTX = dict(logN=16, L=20, K=4, alpha=4, hw=192)
METRIC_MATVEC = "1024x1024 encrypted BSGS matvecs/s (N=2^16, 64 conversations per ciphertext)"
MATVEC_CTX = dict(logN=16, L=8, K=4, alpha=4, hw=192)
LANES = 64
CAL_LANES = 512   # calibration conversations for the Newton seeds and bootstrap gains
E2E_PASSES = 4    # at most this many passes in the e2e leg (min with --steps)
CENSUS = os.path.join(ROOT, "profiles", "pass_census.json")


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


def host_threads():
    """torchrun sets OMP_NUM_THREADS=1 for every rank, which leaves the engine's host-side set-up
    (key, plan and table construction, OpenMP loops) on one core per rank.  Give each rank its
    share of the host's cores instead; must run before torch or the engine library is loaded.
    Set-up only: nothing in the timed region runs on these threads."""
    lws = int(os.environ.get("LOCAL_WORLD_SIZE", "1"))
    if lws > 1 and os.environ.get("OMP_NUM_THREADS") == "1":
        os.environ["OMP_NUM_THREADS"] = str(max(1, (os.cpu_count() or 1) // lws))


def dist_setup():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def broadcast_object(obj, ws):
    """rank 0's obj on every rank"""
    if ws == 1:
        return obj
    import torch.distributed as dist
    box = [obj]
    dist.broadcast_object_list(box, src=0)
    return box[0]


def max_over_ranks(v, ws):
    """The slowest rank's time: the whole job's step time for `value`."""
    if ws == 1:
        return v
    import torch
    import torch.distributed as dist
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def pack_seeds(rank):
    """Rank r owns its own pack of conversations: its own keys and token stream (no data
    crosses ranks; the packs are independent units of work)."""
    return 1 + rank, 100 + rank


def aggregate_tokens_per_s(lanes, ws, steps, ms_max):
    """Whole-job throughput: every rank advanced `lanes` conversations per step."""
    return lanes * ws * steps / (ms_max / 1000.0)


def rand_ct_words(rng, moduli, nl, N):
    return np.stack([np.stack([rng.integers(0, int(moduli[i]), N, dtype=np.uint64) for i in range(nl)])
                     for _ in range(2)])


def roofline(prof):
    """The dominant kernel (by device time) against the measured HBM copy bandwidth."""
    pk = peaks()
    if not prof:
        return None
    kern = {k: v for k, v in prof.items() if not k.startswith("op:")}
    if not kern:
        return None
    name, v = max(kern.items(), key=lambda kv: kv[1][1])
    n, tms, tbytes = v[:3]
    achieved = tbytes / (tms / 1000.0) / 1e9
    peak = pk.get("hbm_gbs", 6650.0)
    traffic = None
    tf = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tf):
        # DRAM bytes per limb-transform from an ncu capture, scaled to this run's average launch by its
        # limbs per launch (algorithmic bytes per launch / algorithmic bytes per limb)
        t = json.load(open(tf)).get(name)
        if isinstance(t, dict) and n:
            traffic = t["dram_bytes_per_limb"] * (tbytes / n) / t["algorithmic_bytes_per_limb"]
    return {"kernel": name, "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            "traffic": traffic, "launches": n, "avg_launch_us": 1000.0 * tms / n,
            "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)" if "hbm_gbs" in pk else "fallback 6650 GB/s"}


def tensor_pipe(prof):
    """The tcgen05 BSGS product against the dense int8 tensor peak: int8 multiply-accumulates the
    kernel issues (counted by the engine per launch) per second of its device time.  The int8 peak
    is taken as twice the measured bf16 rate (the nominal dense int8 : bf16 ratio), i.e. the
    measured bf16 TFLOP/s figure read as tera-MAC/s."""
    v = (prof or {}).get("bsgs_tc")
    if not v or len(v) < 4 or not v[1] or not v[3]:
        return None
    pk = peaks()
    peak = pk.get("bf16_tflops", 1590.0)
    achieved = v[3] / (v[1] / 1000.0) / 1e12
    return {"kernel": "k_bsgs_tc2", "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "int8 TMAC/s",
            "frac": achieved / peak, "launches": v[0], "ms": v[1],
            "peak_source": ("MEASURED_PEAKS.json bf16_tflops x 2 (int8 ops), as MAC/s (of measured)"
                            if "bf16_tflops" in pk else "fallback 1.59 PFLOP/s bf16 x 2 (of fallback)")}


def kernel_table(prof):
    """Per kernel class: launches, device ms, achieved GB/s of algorithmic bytes.  Entries
    named op:* are inclusive times of whole operations (bootstrap, matvec, ...)."""
    return {k: {"launches": v[0], "ms": round(v[1], 3),
                "GB/s": round(v[2] / (v[1] / 1000.0) / 1e9, 1) if v[1] and v[2] else None} for k, v in prof.items()}


def census():
    """The 405M pass's key-switch census, committed by hand from a bench line's "census" (the
    reference arm scales its timed key switches by it)."""
    try:
        return json.load(open(CENSUS))
    except Exception:
        return None


# ------------------------------------------------------------------------ CPU oracle ----
def oracle_keyswitch_seconds(nl_avg, nthreads, seconds):
    """Seconds per hybrid key switch of the C oracle at N = 2^16 and the pass's average limb
    count, on `nthreads` host threads in parallel (ctypes releases the GIL): returns
    (seconds per key switch per thread-parallel throughput, samples)."""
    from concurrent.futures import ThreadPoolExecutor

    from oracle_lib import Oracle, derive_seed, gen_chain, load
    lib = load()
    L, K, logN = 16, 4, 16
    q, p = gen_chain(logN, L, 60, 45, K, 60, lib)
    o = Oracle(logN, q, p, 4, lib)
    ms = (1).to_bytes(8, "little") + bytes(24)
    s = o.secret(derive_seed(lib, ms, 0xFFFFFFF1), 192)
    se = o.secret_eval(s)
    key = o.keygen_switch(se, se, derive_seed(lib, ms, 3))
    nl = max(2, min(L, int(round(nl_avg))))
    rng = np.random.default_rng(5)
    d = np.stack([rng.integers(0, int(o.mods[i]), o.N, dtype=np.uint64) for i in range(nl)])

    def one(_):
        o.keyswitch(d, nl, key)
        return 1

    done, t0 = 0, time.time()
    with ThreadPoolExecutor(nthreads) as ex:
        while time.time() - t0 < seconds or done == 0:
            done += sum(ex.map(one, range(nthreads)))
    return (time.time() - t0) / done, done, nl


# ------------------------------------------------------------------------ workloads ----
def oracle_hmult_setup(L=20, K=4, logN=16):
    """Config 2's HMult on the C oracle: a relinearisation key and one ciphertext pair at N = 2^16,
    L limbs (45-bit primes over a 60-bit q0, K x 60-bit special primes, dnum = ceil(L/4))."""
    from oracle_lib import Oracle, derive_seed, gen_chain, load
    lib = load()
    q, p = gen_chain(logN, L, 60, 45, K, 60, lib)
    o = Oracle(logN, q, p, 4, lib)
    ms = (1).to_bytes(8, "little") + bytes(24)
    se = o.secret_eval(o.secret(derive_seed(lib, ms, 0xFFFFFFF1), 192))
    # a switching key of the relinearisation key's shape (its words do not change the work)
    rlk = o.keygen_switch(se, se, derive_seed(lib, ms, 2))
    rng = np.random.default_rng(9)
    a = rand_ct_words(rng, o.mods, L, o.N)
    b = rand_ct_words(rng, o.mods, L, o.N)
    return o, rlk, a, b


def oracle_hmult_batch(o, rlk, a, b, L, nthreads):
    """nthreads HMult + relinearise + rescale of the oracle run concurrently (ctypes releases the
    GIL); returns the wall seconds of the batch."""
    from concurrent.futures import ThreadPoolExecutor

    def one(_):
        o.ct_rescale(o.ct_mul_relin(a, b, L, rlk), L)
        return 1

    t0 = time.time()
    with ThreadPoolExecutor(nthreads) as ex:
        assert sum(ex.map(one, range(nthreads))) == nthreads
    return time.time() - t0


def run_model(args, ws, rank, local):
    import torch

    import fhessm
    from fhessm.model import (CONFIG_405M, EncryptedModel, calibrate_seeds, pack_lanes, plain_step, rel_err_rms,
                              synthetic_weights)
    cfg = CONFIG_405M
    t_setup = time.time()
    w = synthetic_weights(cfg, seed=1234)
    # Newton seeds and bootstrap gains from 6 steps of 512 calibration conversations (not the
    # timed ones).  The Newton window reaches 3x above the largest mean square seen and 1.25x
    # below the smallest, at a tolerance of 3e-4: over 32 held-out packs of 64 conversations
    # (12 steps each) the worst Newton error is 9e-5, at two more iterations per pass than a
    # 64-conversation calibration whose window misses some of them
    # (rank 0 calibrates and sends the result: one host's cores are shared by all ranks)
    seeds = None
    if rank == 0:
        seeds = calibrate_seeds(cfg, w, steps=6, lanes=CAL_LANES, tol=3e-4, ms_margin=(1.25, 3.0))
    seeds = broadcast_object(seeds, ws)
    cx = fhessm.CryptoContext(device=local, **MODEL_CTX)
    key_seed, tok_seed = pack_seeds(rank)
    cx.KeyGen(seed=key_seed)
    cx.EvalBootstrapSetup(*BOOT_EVALMOD)
    m = EncryptedModel(cx, cfg, w, seeds)
    m.keygen()
    in_level = MODEL_CTX["boot_primes"]   # the top of the user region
    rng = np.random.default_rng(tok_seed)
    nsteps = args.warmup + args.steps
    # the e2e leg runs E more passes: the passes' cost follows the carried state's refresh
    # schedule, which repeats every few steps (103 to 130 bootstraps a pass), so one pass alone
    # is not representative
    n_e2e = max(1, min(args.steps, E2E_PASSES))
    toks = [rng.integers(0, cfg.vocab, LANES) for _ in range(nsteps + n_e2e)]
    cts = [cx.Encrypt(cx.MakeCKKSPackedPlaintext(pack_lanes(w["emb"][t], cfg.D, cx.slots), level=in_level))
           for t in toks]
    cx.sync()
    setup_s = time.time() - t_setup
    stream = torch.cuda.ExternalStream(cx.stream_ptr(), device=local)
    outs = []
    for i in range(args.warmup):
        outs.append(m.step(cts[i]))
        cx.sync()
        mem = cx.memory()
        print(f"warmup pass {i}: memory GiB " + ", ".join(f"{k} {v / 2**30:.1f}" for k, v in mem.items()),
              file=sys.stderr, flush=True)
    barrier(ws)
    clk = ClockSampler(local)
    clk.start()
    l0 = cx.launches()
    k0 = cx.counters()
    b0 = m.stats()["bootstraps"]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(ws)
    torch.cuda.nvtx.range_push("timed")   # ncu --nvtx --nvtx-include "timed/" selects these launches
    e0.record(stream)
    for i in range(args.warmup, nsteps):
        outs.append(m.step(cts[i]))
    e1.record(stream)
    torch.cuda.nvtx.range_pop()
    cx.sync()
    torch.cuda.synchronize()
    barrier(ws)
    clocks = clk.stop()
    ms = e0.elapsed_time(e1)
    launches = cx.launches() - l0
    k1 = cx.counters()
    boots = (m.stats()["bootstraps"] - b0) / args.steps
    ks_per_pass = (k1[0] - k0[0]) / args.steps
    ks_nl_avg = (k1[1] - k0[1]) / max(1, k1[0] - k0[0])
    ms_max = max_over_ranks(ms, ws)
    value = aggregate_tokens_per_s(LANES, ws, args.steps, ms_max)

    # end to end through the public API, right after the timed passes (the GPU still warm): per
    # pass, host words in (H2D), the pass, host words out (D2H); n_e2e passes
    words_in = [cts[nsteps + i].words() for i in range(n_e2e)]
    barrier(ws)
    t0 = time.time()
    for i in range(n_e2e):
        ct_in = cx.ct_from_words(words_in[i], in_level, cts[nsteps + i].scale)
        out = m.step(ct_in)
        words_out = out.words()
    cx.sync()
    e2e_s = max_over_ranks(time.time() - t0, ws) / n_e2e
    e2e = {"value": LANES * ws / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": int(words_in[0].nbytes),
           "d2h_bytes_per_step": int(words_out.nbytes), "passes": n_e2e}

    # the per-kernel table and the roofline come from two more passes, outside the timed region:
    # one call in 4 of every kernel kind bracketed by CUDA events on the engine's stream
    cx.set_option("profile_every", 4)
    cx.profile(True)
    for i in range(2):
        m.step(cts[i])
    prof = cx.profile_collect()
    cx.profile(False)
    prof = {k: (v[0] / 2, v[1] / 2, v[2] / 2, v[3] / 2) for k, v in prof.items()}   # per pass
    census = m.refresh_census()

    # fidelity against the float64 model (exact 1/sqrt), replaying every step from a cold state
    state, errs, top1 = None, [], []
    for i in range(nsteps):
        ref, state = plain_step(cfg, w, w["emb"][toks[i]], state)
        if i >= args.warmup:
            y = fhessm.model.unpack_lanes(cx.Decrypt(outs[i]), cfg.D, LANES, cfg.d)
            lg, lr = y @ w["emb"].T, ref @ w["emb"].T
            errs.append(rel_err_rms(lg, lr))
            top1.append(float(np.mean(lg.argmax(-1) == lr.argmax(-1))))
    fidelity = {"logits_relErrRms_max": max(errs), "top1_min": min(top1), "vs": "float64 model, exact 1/sqrt",
                "bar": "relErrRms <= 1e-3 and top-1 >= 0.98"}
    fidelity["ok"] = bool(fidelity["logits_relErrRms_max"] <= 1e-3 and fidelity["top1_min"] >= 0.98)

    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        t_ks, n, nl = oracle_keyswitch_seconds(ks_nl_avg, 1, 10.0)
        cpu = {"value": LANES / (ks_per_pass * t_ks), "unit": "tokens/s", "cores": 1, "kind": "port",
               "method": "estimate: timed key switches x the pass's key-switch census",
               "sample": f"{n} hybrid key switches of the C oracle at N=2^16, {nl} limbs (the pass's average), "
                         f"single thread, timed, then scaled by the pass's {ks_per_pass:.0f} key switches (a lower "
                         f"bound on the CPU pass time: all other work of the pass is excluded)"}
    if rank == 0:
        line = {
            "metric": METRIC_405M, "value": value, "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u64 (RNS residues, CKKS)", "data": "synthetic (seeded weights and tokens)",
            "config": {"workload": "config 4: 405M poly-SSM, one encrypted decode pass, 64 conversations per GPU",
                       "layers": cfg.n_layer, "d_model": cfg.d, "d_ffn": cfg.dff, "vocab": cfg.vocab,
                       "ring": "N=2^16, L=28 (60 + 13x45 + 14x58), K=4x60, HW 192", "global_batch": LANES * ws,
                       "parallelism": f"dp{ws} (independent packs)", "l2": "working set >> L2 (keys 39 GB)"},
            "kernels": kernel_table(prof),
            "memory_gib": {k: round(v / 2**30, 2) for k, v in cx.memory().items()},
            "census": {"keyswitches_per_pass": ks_per_pass, "ks_avg_limbs": ks_nl_avg, "bootstraps_per_pass": boots,
                       "kernel_launches_per_pass": launches / args.steps,
                       "bootstraps_by_site_all_passes": census},
            "setup_s": setup_s, "gpu_launches": launches, "clocks": clocks, "e2e": e2e, "cpu_baseline": cpu,
            "tensor_pipe": tensor_pipe(prof), "roofline": roofline(prof),
            "fidelity": fidelity,
        }
        print(json.dumps(line), flush=True)
        print(f"fidelity: logits relErrRms max {fidelity['logits_relErrRms_max']:.3e}, top-1 min "
              f"{fidelity['top1_min']:.4f} ({'ok' if fidelity['ok'] else 'FAILED'})", file=sys.stderr, flush=True)
    if not fidelity["ok"]:
        raise SystemExit(f"fidelity below the bar on rank {rank}: {fidelity}")


def run_rwkv7(args, ws, rank, local):
    """Config 5: decode steps of the RWKV-7 0.4B polynomial model for one pack of 32
    conversations per GPU, the state carried encrypted from a cold start (the warm-up steps are
    the first tokens).  Fidelity: the decrypted hidden state through the client's output norm and
    head against the float64 model with the same sites, every timed step."""
    import torch

    import fhessm
    from fhessm.model import rel_err_rms
    from fhessm.rwkv7 import RWKV7_04B, EncryptedRWKV7, Sites, fit_sites, new_state, synthetic_weights
    from fhessm.rwkv7 import step as plain_step
    sh = RWKV7_04B
    t_setup = time.time()
    w = synthetic_weights(sh, seed=2024)
    nsteps = args.warmup + args.steps
    key_seed, tok_seed = pack_seeds(rank)
    rng = np.random.default_rng(tok_seed)
    toks = [rng.integers(0, sh.vocab_size, RWKV7_LANES) for _ in range(nsteps + 1)]
    # the sites' intervals and Newton windows from a calibration run over every rank's tokens and
    # 96 more conversations, refitted twice on the polynomial model's own ranges (rank 0 fits
    # and sends the result)
    fits = None
    if rank == 0:
        crng = np.random.default_rng(4242)
        per_rank = []
        for r in range(ws):   # the same draws as each rank's own token generator
            g = np.random.default_rng(pack_seeds(r)[1])
            per_rank.append([g.integers(0, sh.vocab_size, RWKV7_LANES) for _ in range(nsteps + 1)])
        cal = [np.concatenate([pr[i] for pr in per_rank] + [crng.integers(0, sh.vocab_size, 96)])
               for i in range(nsteps + 1)]
        fits = fit_sites(sh, w, cal, degree=7, rounds=3)
    fits = broadcast_object(fits, ws)
    cx = fhessm.CryptoContext(device=local, **MODEL_CTX)
    cx.KeyGen(seed=key_seed)
    cx.EvalBootstrapSetup(*BOOT_EVALMOD)
    EncryptedRWKV7.keygen(cx, sh, b1=64)
    m = EncryptedRWKV7(cx, sh, w, fits, convs=RWKV7_LANES, b1=64)
    in_level = MODEL_CTX["boot_primes"]   # the top of the user region
    cts = [cx.Encrypt(cx.MakeCKKSPackedPlaintext(m.pack(m.client_input(t)), level=in_level)) for t in toks]
    cx.sync()
    setup_s = time.time() - t_setup
    stream = torch.cuda.ExternalStream(cx.stream_ptr(), device=local)
    outs = []
    for i in range(args.warmup):
        outs.append(m.step(cts[i]))
        cx.sync()
    barrier(ws)
    clk = ClockSampler(local)
    clk.start()
    l0, k0, b0 = cx.launches(), cx.counters(), m.bootstraps
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(ws)
    e0.record(stream)
    for i in range(args.warmup, nsteps):
        outs.append(m.step(cts[i]))
    e1.record(stream)
    cx.sync()
    torch.cuda.synchronize()
    barrier(ws)
    clocks = clk.stop()
    ms = e0.elapsed_time(e1)
    launches = cx.launches() - l0
    k1 = cx.counters()
    boots = (m.bootstraps - b0) / args.steps
    ms_max = max_over_ranks(ms, ws)
    value = aggregate_tokens_per_s(RWKV7_LANES, ws, args.steps, ms_max)
    # end to end through the public API: host words in, one step, host words out
    words_in = cts[nsteps].words()
    barrier(ws)
    t0 = time.time()
    out = m.step(cx.ct_from_words(words_in, in_level, cts[nsteps].scale))
    words_out = out.words()
    cx.sync()
    e2e_s = max_over_ranks(time.time() - t0, ws)
    e2e = {"value": RWKV7_LANES * ws / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": int(words_in.nbytes),
           "d2h_bytes_per_step": int(words_out.nbytes), "passes": 1}
    # fidelity: the float64 model with the same sites, replayed from the cold state
    sites = Sites(fits)
    st = new_state(sh, RWKV7_LANES)
    errs, top1 = [], []
    for i in range(nsteps):
        ref = plain_step(sh, w, toks[i], st, sites)
        if i >= args.warmup:
            lg = m.client_logits(m.unpack(cx.Decrypt(outs[i])))
            errs.append(rel_err_rms(lg, ref))
            top1.append(float(np.mean(lg.argmax(-1) == ref.argmax(-1))))
    fidelity = {"logits_relErrRms_max": max(errs), "top1_min": min(top1), "per_step": errs,
                "vs": "float64 model with the same polynomial sites", "bar": "relErrRms <= 1e-3 and top-1 >= 0.98"}
    fidelity["ok"] = bool(fidelity["logits_relErrRms_max"] <= 1e-3 and fidelity["top1_min"] >= 0.98)
    ks_step = (k1[0] - k0[0]) / args.steps
    ks_nl = (k1[1] - k0[1]) / max(1, k1[0] - k0[0])
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        t_ks, n, nl = oracle_keyswitch_seconds(ks_nl, 1, 10.0)
        cpu = {"value": RWKV7_LANES / (ks_step * t_ks), "unit": "tokens/s", "cores": 1, "kind": "port",
               "method": "estimate: timed key switches x the step's key-switch census",
               "sample": f"{n} hybrid key switches of the C oracle at N=2^16, {nl} limbs (the step's average), "
                         f"single thread, timed, then scaled by the step's {ks_step:.0f} key switches (a lower "
                         f"bound on the CPU step time: all other work of the step is excluded)"}
    if rank == 0:
        line = {
            "metric": METRIC_RWKV7, "value": value, "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u64 (RNS residues, CKKS)", "data": "synthetic (seeded weights and tokens)",
            "config": {"workload": "config 5: RWKV-7 0.4B polynomial model, one encrypted decode step, 32 "
                                   "conversations per GPU", "layers": sh.n_layer, "d_model": sh.n_embd,
                       "heads": sh.n_head, "head_size": sh.head_size, "d_ffn": sh.dim_ffn, "vocab": sh.vocab_size,
                       "sites": "degree-7 Chebyshev on fitted intervals, Newton 1/sqrt with tuned steps",
                       "ring": "N=2^16, L=28 (60 + 13x45 + 14x58), K=4x60, HW 192",
                       "global_batch": RWKV7_LANES * ws, "parallelism": f"dp{ws} (independent packs)",
                       "l2": "working set >> L2 (keys and the 64 state rows per layer)"},
            "memory_gib": {k: round(v / 2**30, 2) for k, v in cx.memory().items()},
            "census": {"keyswitches_per_step": ks_step, "ks_avg_limbs": ks_nl, "bootstraps_per_step": boots,
                       "kernel_launches_per_step": launches / args.steps},
            "setup_s": setup_s, "gpu_launches": launches, "clocks": clocks, "e2e": e2e,
            "cpu_baseline": cpu, "roofline": None, "fidelity": fidelity,
        }
        print(json.dumps(line), flush=True)
        print(f"fidelity: logits relErrRms max {fidelity['logits_relErrRms_max']:.3e}, top-1 min "
              f"{fidelity['top1_min']:.4f} ({'ok' if fidelity['ok'] else 'FAILED'})", file=sys.stderr, flush=True)
    if not fidelity["ok"]:
        raise SystemExit(f"fidelity below the bar on rank {rank}: {fidelity}")


def run_hmult(args, ws, rank, local):
    import torch

    import fhessm
    cx = fhessm.CryptoContext(device=local, **HMULT_CTX)
    cx.KeyGen(seed=1 + rank)
    L, N = HMULT_CTX["L"], 1 << HMULT_CTX["logN"]
    rng = np.random.default_rng(100 + rank)
    B = args.batch
    host_a = [rand_ct_words(rng, cx.moduli, L, N) for _ in range(B)]
    host_b = [rand_ct_words(rng, cx.moduli, L, N) for _ in range(B)]
    A = [cx.ct_from_words(x, 0) for x in host_a]
    Bc = [cx.ct_from_words(x, 0) for x in host_b]
    stream = torch.cuda.ExternalStream(cx.stream_ptr(), device=local)

    def step():
        for a, b in zip(A, Bc):
            c = cx.EvalMult(a, b)
            cx.RescaleInPlace(c)

    for _ in range(args.warmup):
        step()
    cx.sync()
    barrier(ws)
    clk = ClockSampler(local)
    clk.start()
    l0 = cx.launches()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
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
    launches = cx.launches() - l0
    ms_max = max_over_ranks(ms, ws)
    value = B * ws * args.steps / (ms_max / 1000.0)
    cx.profile(True)   # the kernel table: one more step, outside the timed region
    step()
    prof = cx.profile_collect()
    cx.profile(False)
    out_words = np.empty((2, L - 1, N), dtype=np.uint64)
    barrier(ws)
    t0 = time.time()
    for wa, wb in zip(host_a, host_b):
        a, b = cx.ct_from_words(wa, 0), cx.ct_from_words(wb, 0)
        c = cx.EvalMult(a, b)
        cx.RescaleInPlace(c)
        out_words[...] = c.words()
    cx.sync()
    e2e_s = max_over_ranks(time.time() - t0, ws)
    e2e = {"value": B * ws / e2e_s, "unit": "ciphertexts/s", "h2d_bytes_per_step": int(2 * B * host_a[0].nbytes),
           "d2h_bytes_per_step": int(B * out_words.nbytes)}
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        # the same operation on the C oracle, timed on this host: one thread, then every host thread
        o, rlk, ha, hb = oracle_hmult_setup(L)
        nth = os.cpu_count() or 1
        t1 = oracle_hmult_batch(o, rlk, ha, hb, L, 1)
        tn = min(oracle_hmult_batch(o, rlk, ha, hb, L, nth) for _ in range(2))
        cpu = {"value": nth / tn, "unit": "ciphertexts/s", "cores": nth, "kind": "port",
               "single_thread": 1.0 / t1,
               "sample": f"C oracle HMult+relin+rescale at N=2^16, L={L}, dnum=5: 1 on one thread ({t1:.2f} s), "
                         f"then {nth} at once on {nth} threads (best of 2 batches, {tn:.2f} s)"}
    if rank == 0:
        line = {
            "metric": METRIC_HMULT, "value": value, "unit": "ciphertexts/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u64 (RNS residues)", "data": "synthetic",
            "config": {"workload": "config 2: HMult+relin+rescale, N=2^16, L=20, K=4x60b, dnum=5",
                       "batch_per_gpu": B, "parallelism": f"dp{ws}", "l2": "inputs 2.7 GB per GPU > L2"},
            "gpu_launches": launches, "clocks": clocks, "e2e": e2e, "roofline": roofline(prof), "cpu_baseline": cpu,
            "kernels": kernel_table(prof),
        }
        print(json.dumps(line), flush=True)


def run_ntt(args, ws, rank, local):
    """Auxiliary kernel benchmark (not a bench line of the headline metric): batched forward and
    inverse NTTs over `--limbs` limb-polynomials of the 405M chain at N = 2^16 through the C-ABI
    (fhe_ntt_host: one batched transform per direction), timed by the per-kernel CUDA-event timer
    (device time of the transforms only, the host copies around them excluded)."""
    import fhessm
    cx = fhessm.CryptoContext(device=local, **MODEL_CTX)
    rng = np.random.default_rng(rank)
    n = args.limbs
    w = rng.integers(0, 1 << 44, (n, cx.N), dtype=np.uint64)   # below every modulus of the chain
    mi = [i % (cx.L + cx.K) for i in range(n)]
    for _ in range(args.warmup):
        cx.ntt(cx.ntt(w, mi), mi, inverse=True)
    cx.profile(True)
    for _ in range(args.steps):
        f = cx.ntt(w, mi)
        b = cx.ntt(f, mi, inverse=True)
    prof = cx.profile_collect()
    cx.profile(False)
    if not (b == w).all():
        raise RuntimeError("ntt workload: inverse(forward(x)) != x")
    if rank == 0:
        us = {k: 1000.0 * prof[name][1] / (prof[name][0] * n) for k, name in (("fwd", "ntt_fwd"), ("inv", "ntt_inv"))}
        print(json.dumps({"metric": "NTT limb-transforms/s (N=2^16, forward)", "value": 1e6 / us["fwd"],
                          "unit": "limbs/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
                          "higher_is_better": True, "dtype": "u64", "data": "synthetic",
                          "config": {"workload": f"{n} limb-polynomials, moduli of the 405M chain"},
                          "us_per_limb": us, "kernels": kernel_table(prof)}), flush=True)


def run_matvec(args, ws, rank, local):
    """One 1024 x 1024 block of the 405M model's linears (double-hoisted BSGS, b1 = 64): babies,
    tensor-core products, giants.  A step is one matvec on an input already on the device."""
    import torch

    import fhessm
    from fhessm.model import pack_lanes
    cx = fhessm.CryptoContext(device=local, **MATVEC_CTX)
    cx.KeyGen(seed=1 + rank)
    D, b1 = 1024, 64
    cx.matvec_keygen(D, b1)
    rng = np.random.default_rng(7 + rank)
    plan = cx.matvec_plan(rng.normal(0, 0.02, (D, D)), D, b1)
    U = rng.uniform(-1, 1, (LANES, D))
    ct = cx.Encrypt(cx.MakeCKKSPackedPlaintext(pack_lanes(U, D, cx.slots), level=2))
    stream = torch.cuda.ExternalStream(cx.stream_ptr(), device=local)
    for _ in range(args.warmup):
        cx.matvec(plan, [ct])
    cx.sync()
    barrier(ws)
    clk = ClockSampler(local)
    clk.start()
    l0 = cx.launches()
    cx.profile(True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(ws)
    e0.record(stream)
    for _ in range(args.steps):
        y = cx.matvec(plan, [ct])
    e1.record(stream)
    cx.sync()
    barrier(ws)
    clocks = clk.stop()
    ms = max_over_ranks(e0.elapsed_time(e1), ws)
    prof = cx.profile_collect()
    cx.profile(False)
    value = ws * args.steps / (ms / 1000.0)
    words = ct.words()
    t0 = time.time()
    out = cx.matvec(plan, [cx.ct_from_words(words, ct.level, ct.scale)]).words()
    e2e_s = max_over_ranks(time.time() - t0, ws)
    if rank == 0:
        print(json.dumps({
            "metric": METRIC_MATVEC, "value": value, "unit": "matvecs/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u64 (RNS residues, CKKS)", "data": "synthetic",
            "config": {"workload": "one 1024x1024 BSGS block of config 4 (b1 = 64, 6 limbs)", "parallelism": f"dp{ws}"},
            "gpu_launches": cx.launches() - l0, "clocks": clocks, "roofline": roofline(prof), "cpu_baseline": None,
            "e2e": {"value": ws / e2e_s, "unit": "matvecs/s", "h2d_bytes_per_step": int(words.nbytes),
                    "d2h_bytes_per_step": int(out.nbytes)},
            "kernels": kernel_table(prof)}), flush=True)


METRIC_KSDIST = "hybrid key switches/s of one ciphertext, limb-partitioned over N B200 (N=2^16, L=20)"


def run_ksdist(args, ws, rank, local):
    """Single-pack latency (config 5's multi-GPU case): one ciphertext's hybrid key switch at
    N = 2^16, L = 20 (dnum 5), its limbs split over the ranks (fhe_keyswitch_dist: NCCL all-gathers
    of d's coefficient limbs before ModUp and of the special limbs before ModDown).  Strong scaling:
    the same key switch on every N; a step is one key switch; the device time is the slowest rank's."""
    import torch

    import fhessm
    from fhessm import dist as fd
    import torch.distributed as tdist
    cx = fhessm.CryptoContext(device=local, logN=16, L=20, K=4, alpha=4, hw=192)
    cx.KeyGen(seed=1)                                   # the same keys on every rank
    if ws > 1:
        obj = [fd.unique_id() if rank == 0 else None]
        tdist.broadcast_object_list(obj, src=0)
        uid = obj[0]
    else:
        uid = fd.unique_id()
    fd.init(cx, ws, rank, uid)
    level, nl = 0, 20
    rng = np.random.default_rng(5)
    d = np.stack([rng.integers(0, int(cx.moduli[i]), cx.N, dtype=np.uint64) for i in range(nl)])
    lo, cnt, _ = fd.limb_block(nl, ws, rank)
    dev = torch.from_numpy(np.ascontiguousarray(d[lo:lo + cnt]).view(np.int64)).to(f"cuda:{local}")
    o0 = torch.zeros((max(cnt, 1), cx.N), dtype=torch.int64, device=f"cuda:{local}")
    o1 = torch.zeros_like(o0)
    stream = torch.cuda.ExternalStream(cx.stream_ptr(), device=local)

    def step():
        fd.keyswitch(cx, 0, dev.data_ptr(), level, o0.data_ptr(), o1.data_ptr())

    for _ in range(args.warmup):
        step()
    cx.sync()
    barrier(ws)
    clk = ClockSampler(local)
    clk.start()
    l0 = cx.launches()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(ws)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    cx.sync()
    torch.cuda.synchronize()
    barrier(ws)
    clocks = clk.stop()
    ms_max = max_over_ranks(e0.elapsed_time(e1), ws)
    value = args.steps / (ms_max / 1000.0)
    launches = cx.launches() - l0
    # correctness of the timed output against the single-GPU key switch of the whole ciphertext
    e_0, _ = cx.keyswitch_raw(d, level, cx.key_words(0))
    ok = bool((o0.cpu().numpy().view(np.uint64)[:cnt] == e_0[lo:lo + cnt]).all())
    # end to end: the rank's limbs from pinned host memory, the key switch, its result limbs back
    host_in = torch.from_numpy(np.ascontiguousarray(d[lo:lo + cnt]).view(np.int64)).pin_memory()
    host_out = torch.empty((2, max(cnt, 1), cx.N), dtype=torch.int64).pin_memory()
    barrier(ws)
    t0 = time.time()
    for _ in range(args.steps):
        dev.copy_(host_in, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        step()
        cx.sync()
        host_out[0].copy_(o0)
        host_out[1].copy_(o1)
    e2e_s = max_over_ranks(time.time() - t0, ws)
    if not ok:
        raise SystemExit(f"ksdist: rank {rank}'s limbs differ from the single-GPU key switch")
    if rank == 0:
        bytes_ks = 8.0 * cx.N * (2 * nl + 5 * 2 * (nl + 4) + 3 * 5 * (nl + 4) + 2 * nl)
        print(json.dumps({
            "metric": METRIC_KSDIST, "value": value, "unit": "key switches/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "u64 (RNS residues)", "data": "synthetic",
            "config": {"workload": "one ciphertext's hybrid key switch (relinearisation key), N=2^16, L=20, K=4, "
                                   "dnum=5, limbs split over the ranks", "parallelism": f"limb-partitioned x{ws}",
                       "l2": "key 120 MiB per rank > L2 share"},
            "gpu_launches": launches, "clocks": clocks, "bit_exact_vs_single_gpu": ok,
            "e2e": {"value": args.steps / e2e_s, "unit": "key switches/s",
                    "h2d_bytes_per_step": int(host_in.numel() * 8), "d2h_bytes_per_step": int(2 * cnt * cx.N * 8)},
            "algorithmic_bytes_per_ks": bytes_ks, "roofline": None, "cpu_baseline": None}), flush=True)


def run_reference(args):
    """The reference arm: the CPU path of the same workload on the host cores.  OpenFHE (the
    reference's arithmetic library) cannot be built here, so the C oracle (a restatement of the
    same RNS-CKKS algorithms, pinned to the reference's own expander and NTT) stands in.  Every step
    is a real, bounded sample timed on the host: one batch of oracle operations on all host
    threads.  hmult: the sample is config 2's operation itself, so `value` is measured directly.
    405m: the sample is a batch of key switches at the pass's average limb count, and `value`
    scales it by the pass's key-switch census (an estimate and a lower bound on the CPU pass: all
    other work of the pass is left out); ms_per_step is the sample's own time."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    nthreads = os.cpu_count() or 1
    base = {"impl": "reference", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "data": "synthetic"}
    if args.workload == "hmult":
        L = HMULT_CTX["L"]
        o, rlk, ha, hb = oracle_hmult_setup(L)
        times = []
        for i in range(args.warmup + args.steps):
            t = oracle_hmult_batch(o, rlk, ha, hb, L, nthreads)
            if i >= args.warmup:
                times.append(t)
        value = nthreads * len(times) / sum(times)
        line = dict(base, metric=METRIC_HMULT, value=value, unit="ciphertexts/s",
                    ms_per_step=1000.0 * statistics.mean(times), dtype="u64 (RNS residues)",
                    config={"workload": "config 2: HMult+relin+rescale, N=2^16, L=20, K=4x60b, dnum=5"},
                    cpu_baseline={"value": value, "unit": "ciphertexts/s", "cores": nthreads, "kind": "port",
                                  "sample": f"per step {nthreads} C-oracle HMult+relin+rescale, one per thread"},
                    e2e={"value": value, "unit": "ciphertexts/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0})
        print(json.dumps(line), flush=True)
        return 0
    if args.workload == "rwkv7":
        print(json.dumps({"impl": "reference", "unavailable": "the reference's encrypted RWKV-7 port is not in its "
                                                              "tree (README.md:156: an external fork); it holds only "
                                                              "the plaintext harness"}))
        return 0
    if args.workload != "405m":
        print(json.dumps({"impl": "reference", "unavailable": "reference arm implemented for the 405m and hmult "
                                                              "workloads"}))
        return 0
    cen = census()
    if not cen:
        print(json.dumps({"impl": "reference", "unavailable": "no key-switch census (profiles/pass_census.json)"}))
        return 0
    from concurrent.futures import ThreadPoolExecutor

    from oracle_lib import Oracle, derive_seed, gen_chain, load
    lib = load()
    q, p = gen_chain(16, 16, 60, 45, 4, 60, lib)
    o = Oracle(16, q, p, 4, lib)
    ms = (1).to_bytes(8, "little") + bytes(24)
    se = o.secret_eval(o.secret(derive_seed(lib, ms, 0xFFFFFFF1), 192))
    key = o.keygen_switch(se, se, derive_seed(lib, ms, 3))
    nl = max(2, min(16, int(round(cen["ks_avg_limbs"]))))
    rng = np.random.default_rng(5)
    d = np.stack([rng.integers(0, int(o.mods[i]), o.N, dtype=np.uint64) for i in range(nl)])
    times = []
    with ThreadPoolExecutor(nthreads) as ex:
        for i in range(args.warmup + args.steps):
            t0 = time.time()
            list(ex.map(lambda _: o.keyswitch(d, nl, key), range(nthreads)))
            if i >= args.warmup:
                times.append(time.time() - t0)
    t_ks = sum(times) / (nthreads * len(times))          # seconds per key switch at full concurrency
    value = LANES / (cen["keyswitches_per_pass"] * t_ks)
    line = dict(base, metric=METRIC_405M, value=value, unit="tokens/s", ms_per_step=1000.0 * statistics.mean(times),
                dtype="u64 (RNS residues, CKKS)",
                config={"workload": "config 4: 405M poly-SSM, one encrypted decode pass, 64 conversations"},
                cpu_baseline={"value": value, "unit": "tokens/s", "cores": nthreads, "kind": "port",
                              "method": "estimate: timed key switches x the pass's key-switch census",
                              "sample": f"per step {nthreads} C-oracle key switches at N=2^16, {nl} limbs, one per "
                                        f"thread (timed; ms_per_step is this sample), scaled by "
                                        f"{cen['keyswitches_per_pass']:.0f} key switches per pass"},
                e2e={"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0})
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="engine", choices=["engine", "reference"])
    ap.add_argument("--workload", default="405m", choices=["405m", "hmult", "matvec", "ntt", "ksdist", "rwkv7"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=64, help="hmult: ciphertext pairs per GPU per step")
    ap.add_argument("--limbs", type=int, default=1024, help="ntt: limb-polynomials per transform")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    host_threads()
    ws, rank, local = dist_setup()
    import torch
    torch.cuda.set_device(local)
    if args.workload == "405m":
        run_model(args, ws, rank, local)
    elif args.workload == "matvec":
        run_matvec(args, ws, rank, local)
    elif args.workload == "ntt":
        run_ntt(args, ws, rank, local)
    elif args.workload == "ksdist":
        run_ksdist(args, ws, rank, local)
    elif args.workload == "rwkv7":
        run_rwkv7(args, ws, rank, local)
    else:
        run_hmult(args, ws, rank, local)
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
