"""T3 decode benchmark.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (configs[0], the metric's batch-1 configuration): T3 Turbo GPT-2
Medium (24 layers, d 1024, 16 heads, FFN 4096, V 6563), random-init weights
quantized to Q4_0 (speech_head Q4_0 too, as convert --quant q4_0), batch 1,
no CFG, a 150-position prompt (1 speaker row + 62 cond speech tokens + 86
text ids + start token), temperature 0.8, top_k 1000, top_p 0.95,
repetition penalty 1.2, std::mt19937 seed 0.  One bench step = one decode
step (one speech token per stream): embedding, 24 layers, head, sampler.
K defaults to 256 (the config's decode length).  Under torchrun every rank
decodes its own utterance on its own GPU (independent utterances, no
collective: weak scaling); the job time is the max over ranks.

value: speech tokens/s with everything resident on the device (t3b_decode,
timed with CUDA events on the context's stream).  e2e: the same decode driven
through the per-step drop-in API (t3b_step -> logits to host -> t3b_sample
with host logits -> token to host), i.e. chatterbox.cpp's eval_step +
sample_next_token_ex call pattern, host copies included.
"""
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

PROMPT_TEXT = 86
PARAMS = dict(top_k=1000, top_p=0.95, temp=0.8, repeat_penalty=1.2)
METRIC = "T3 speech tokens/s (batch-1 Q4_0 decode, % HBM roofline)"
UNIT = "speech tokens/s"


def algorithmic_bytes_per_step(hp, L_mean, weight_bytes):
    """Bytes one decode step must move: every weight byte once plus the f16
    K and V of L positions for every layer (98 304 B per position for T3),
    plus the step's own K/V write and the logits."""
    kv = 2 * hp["n_layer"] * hp["n_embd"] * 2
    return weight_bytes + kv * (L_mean + 1) + hp["n_speech_vocab"] * 4


def model_weight_bytes(t):
    n = 0
    for name, (ty, arr) in t.items():
        if name in ("chatterbox/text_emb", "chatterbox/cond_spkr/w", "chatterbox/cond_spkr/b",
                    "chatterbox/builtin/speaker_emb", "chatterbox/builtin/cond_prompt_speech_tokens",
                    "model/wpe", "chatterbox/speech_emb"):
            continue
        n += np.asarray(arr).nbytes
    # one speech_emb row (f16) and one wpe row (f32) per step
    return n + 1024 * 2 + 1024 * 4


class Clocks:
    """nvidia-smi sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.p = None
        self.lines = []

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.p = None
        return self

    def _read(self):
        for line in self.p.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.p:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except Exception:
                self.p.kill()

    def summary(self):
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
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def cpu_reference(args, hp, t, text, label_impl):
    """The reference's CPU path for this workload: chatterbox.cpp cannot be
    built here (ggml absent), so the oracle's restatement of ggml's CPU
    arithmetic (oracle/t3_oracle.cpp, ggml-like mode) runs the same
    batch-1 decode on all host cores.  Bounded sample: as many decode steps
    as fit in ~12 s (at least 4), after an untimed prefill."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    oracle.set_threads(cores)
    m = oracle.Model(hp, t, max_ctx=150 + max(args.steps, 64) + 8, gemv_mode=1, gelu_f16=1, kv_f16=0)
    P, lg = m.prompt(text)
    words = oracle.mt19937_words(0, 0, 2 * (args.steps + 2))
    hist = []
    tok, _ = oracle.sample(lg, PARAMS, words[0], words[1])
    hist.append(tok)
    n, t0 = 0, time.perf_counter()
    budget = float(os.environ.get("T3B_CPU_SECONDS", "12"))
    while n < args.steps:
        lg = m.step(P + n, tok)
        tok, _ = oracle.sample(lg, PARAMS, words[2 * n + 2], words[2 * n + 3], hist=np.array(hist, np.int32))
        hist.append(tok)
        n += 1
        if n >= 4 and time.perf_counter() - t0 > budget:
            break
    dt = time.perf_counter() - t0
    return {"value": n / dt, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{n} decode steps of the batch-1 Q4_0 workload after a 150-position prefill "
                      f"(oracle restatement of ggml's CPU path, OpenMP x{cores}); {dt:.2f} s"}


def make_model(pkg, seed=0):
    hp = dict(pkg.t3_gguf.T3_TURBO)
    hp, t = pkg.t3_gguf.random_t3(hp, quant="q4_0", seed=seed)
    return hp, t


def run_reference(args):
    ws, rank, _ = dist_env()
    if rank != 0:
        return 0
    import __graft_entry__ as ge
    pkg = ge.load_package()
    hp, t = make_model(pkg)
    text = np.random.default_rng(0).integers(0, 50257, PROMPT_TEXT).astype(np.int32)
    cb = cpu_reference(args, hp, t, text, "reference")
    line = {"metric": METRIC, "value": cb["value"], "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 / cb["value"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "q4_0 x q8_0 (int dot, f32 accumulate)",
            "data": "synthetic (random-init T3 Q4_0 weights, seeded prompt)", "impl": "reference",
            "config": config_block(args), "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def config_block(args):
    return {"workload": "configs[0]: T3 Turbo batch-1 Q4_0 decode, 150-position prompt, "
                        f"{args.steps} decode steps per rank, temp 0.8 / top_k 1000 / top_p 0.95 / penalty 1.2, "
                        "mt19937 seed 0",
            "model": "T3 Turbo GPT-2 Medium 24x1024, 16 heads, FFN 4096, V 6563 (random init)",
            "global_batch": args.gpus, "seq_len": 150 + args.steps, "parallelism": f"replicas x{args.gpus}",
            "l2": "inputs larger than L2 (175 MB of weights streamed per step)"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-batched", action="store_true", help="leave out the batched CFG run (profiling commands)")
    ap.add_argument("--only", choices=["sampler", "gemv", "timeline", "batched", "kernels", "sweep", "serve3", "serve4",
                                       "refdefault"],
                    default=None,
                    help="run one kernel micro-benchmark alone (ncu captures), or the megakernel phase timeline")
    args = ap.parse_args()
    if args.only:
        import torch
        import __graft_entry__ as ge
        pkg = ge.load_package()
        peak, _ = peaks()
        if args.only == "timeline":
            r = phase_timeline(pkg)
        elif args.only == "batched":
            import torch
            r = batched_cfg(pkg, torch, peak)
        elif args.only == "kernels":
            import torch
            r = batched_kernels(pkg, torch, peak)
        elif args.only in ("serve3", "serve4"):
            # serve4 alone: rank 0's share of the 8-GPU configuration
            ws_ = 8 if args.only == "serve4" else 1
            r = serving(pkg, torch, peak, int(args.only[-1]), None, ws_, 0, 0, steps=args.steps if args.steps != 256 else None)
        elif args.only == "sweep":
            import torch
            r = gemv_sweep(pkg, torch, peak)
        elif args.only == "refdefault":
            hp, t = make_model(pkg, seed=0)
            r = reference_default_decode(pkg, hp, t, pkg.SampleParams.make(**PARAMS), model_weight_bytes(t), peak)
        else:
            r = sampler_microbench(pkg, torch, peak, reps=20) if args.only == "sampler" else gemv_roofline(pkg, torch, peak)
        print(json.dumps(r), flush=True)
        return 0
    if args.impl == "reference":
        return run_reference(args)
    args.warmup = max(args.warmup, 3)

    ws, rank, local = dist_env()
    import torch
    torch.cuda.set_device(local)
    dist = None
    if ws > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))

    import __graft_entry__ as ge
    pkg = ge.load_package()
    hp, t = make_model(pkg, seed=0)
    wbytes = model_weight_bytes(t)
    text = np.random.default_rng(rank).integers(0, 50257, PROMPT_TEXT).astype(np.int32)
    m = pkg.T3Model(hp, t, device=local)
    K, W = args.steps, args.warmup
    m.alloc_streams(1, 150 + max(K, W) + 8)
    params = pkg.SampleParams.make(**PARAMS)

    clk = Clocks(local).__enter__()   # sampling starts before the warm-up (nvidia-smi needs ~0.2 s)
    # warm-up: a W-step utterance
    m.prefill(0, text)
    m.set_rng(0, pkg.T3B_RNG_MT19937, 0, 0)
    m.decode([params], W, ignore_stop=True)
    # timed: K decode steps from the prompt end (positions 151 .. 150+K)
    P, _ = m.prefill(0, text)
    m.set_rng(0, pkg.T3B_RNG_MT19937, 0, 0)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    n_launch0 = m.launch_count()
    toks = m.decode([params], K, ignore_stop=True)[0]
    dev_ms = m.last_device_ms()
    n_launch = m.launch_count() - n_launch0
    torch.cuda.synchronize()
    time.sleep(0.25)
    clk.__exit__()
    if dist:
        dist.barrier()
    # every rank decoded K tokens of its own utterance; job time = slowest rank
    value, ms = pkg.sharding.job_throughput(dist, dev_ms, K, ws)
    ms_per_step = ms / K

    # e2e through the per-step drop-in API (host copies every step)
    m.prefill(0, text)
    m.set_rng(0, pkg.T3B_RNG_MT19937, 0, 0)
    m.set_history(0, np.zeros(0, np.int32))
    V = hp["n_speech_vocab"]
    e2e_steps = min(K, 64)
    tok = int(m.sample([params])[0])
    host_logits = np.zeros((1, 1, V), np.float32)
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        host_logits = m.step([tok])                         # eval_step: token H2D, logits D2H
        tok = int(m.sample([params], logits=host_logits)[0])  # sample_next_token_ex on host logits
    e2e_s = time.perf_counter() - t0
    e2e_value, _ = pkg.sharding.job_throughput(dist, e2e_s * 1000.0, e2e_steps, ws)
    e2e = {"value": e2e_value, "unit": UNIT,
           "h2d_bytes_per_step": 4 + 4 + V * 4 + 24 + 4, "d2h_bytes_per_step": V * 4 + 4,
           "steps": e2e_steps, "path": "t3b_step(host token) -> logits D2H -> t3b_sample(host logits) -> token D2H"}

    # roofline of the dominant kernel: the decode step itself is the unit
    # that streams every weight once; plus the GEMV alone (op-level)
    peak, peak_kind = peaks()
    L_mean = P + (K + 1) / 2.0
    step_bytes = algorithmic_bytes_per_step(hp, L_mean, wbytes)
    achieved = step_bytes / (ms_per_step / 1000.0) / 1e9
    gemv = gemv_roofline(pkg, torch, peak)

    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": K, "warmup": W,
            "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "q4_0 x q8_0 (int dot, f32 accumulate)",
            "data": "synthetic (random-init T3 Q4_0 weights, seeded prompt)",
            "config": config_block(args),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": measured_traffic(),
                         "peak_kind": peak_kind,
                         "kernel": "t3_decode_megakernel<Q4_0> (persistent; one launch decodes K steps); "
                                   "achieved/traffic per decode step",
                         "bytes_per_step": step_bytes, "mean_L": L_mean},
            "gemv_roofline": gemv,
            "sampler": sampler_microbench(pkg, torch, peak),
            "batch1_reference_default": reference_default_decode(pkg, hp, t, params, wbytes, peak, device=local),
            "serving_configs3": serving(pkg, torch, peak, 3, dist, ws, rank, local) if not args.no_batched else None,
            "serving_configs4": ({q: serving(pkg, torch, peak, 4, dist, ws, rank, local, quant=q) for q in ("q4_0", "f16")}
                                 if ws == 8 and not args.no_batched else None),
            "batched_kernels": batched_kernels(pkg, torch, peak),
            "gemv_sweep": gemv_sweep(pkg, torch, peak) if not args.no_batched else None,
            "e2e": e2e, "clocks": clk.summary(),
            "gpu_launches": n_launch,   # counted by the library (t3b_launch_count) over the timed decode
            "tokens_head": [int(x) for x in toks[:8]]}
    if ws == 1 and not args.no_cpu_baseline:   # the CPU baseline is measured at N = 1 only
        line["cpu_baseline"] = cpu_reference(args, hp, t, text, "port")
    if rank == 0:
        print(json.dumps(line), flush=True)
    m.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def serving(pkg, torch, peak, which, dist, ws, rank, local, quant=None, steps=None):
    """BASELINE configs[3] (which=3) or configs[4] (which=4) through the
    continuous-batching scheduler (t3b_serve_*), streams sharded over the
    ranks by expected KV cost (greedy LPT, sharding.assign_streams).

    64 utterances with CFG (128 rows), prompts U[100, 400],
    decode to 1024 tokens (or a stop token), Q8_0.  configs[4]: 512 with
    CFG (1024 rows over 8 GPUs), contexts U[50, 2048] (prompt U[50, 2048-K],
    then K decode steps), Q4_0 or F16, per-stream temperature U[0.6, 1.0],
    top_p U[0.8, 1.0] and penalty U[1.0, 1.5]; every stream draws from its
    own Philox stream.  Seeded synthetic prompts; random-init weights.

    value = decode tokens of all ranks / max over ranks of the device time
    of the batched steps (t3b_serve_stats); wall = the same tokens over the
    slowest rank's wall time of the whole serve loop (admission prefills,
    host bookkeeping and every step's token read-back included)."""
    rng = np.random.default_rng(1000 + which)
    if which == 3:
        n_total, quant, K = 64, quant or "q8_0", steps or 1024
        P = rng.integers(100, 401, n_total)
        prm = [pkg.SampleParams.make(**PARAMS, cfg_weight=0.5) for _ in range(n_total)]
    else:
        n_total, quant, K = 512, quant or "q4_0", steps or 128
        P = rng.integers(50, 2049 - K, n_total)
        temp, top_p, pen = rng.uniform(0.6, 1.0, n_total), rng.uniform(0.8, 1.0, n_total), rng.uniform(1.0, 1.5, n_total)
        prm = [pkg.SampleParams.make(top_k=1000, top_p=float(top_p[i]), temp=float(temp[i]),
                                     repeat_penalty=float(pen[i]), cfg_weight=0.5) for i in range(n_total)]
    costs = [pkg.sharding.stream_cost(int(p), K, cfg=True) for p in P]
    mine = pkg.sharding.assign_streams(costs, ws)[rank]
    hp = dict(pkg.t3_gguf.T3_TURBO)
    hp, t = pkg.t3_gguf.random_t3(hp, quant=quant, seed=3)
    m = pkg.T3Model(hp, t, device=local)
    m.alloc_streams(len(mine), int(max(P[i] for i in mine)) + K + 8, cfg=True)
    for i in mine:
        ri = np.random.default_rng(5000 + i)
        n_cond = min(hp["cond_prompt_len"], int(P[i]) - 3)     # short contexts use fewer conditioning tokens
        cond = ri.integers(0, hp["start_speech_token"], n_cond).astype(np.int32)
        text = ri.integers(0, 50257, int(P[i]) - 2 - n_cond).astype(np.int32)
        m.serve_submit(text, prm[i], seed=7000 + i, n_predict=K, rng_mode=pkg.T3B_RNG_PHILOX, cond=cond)
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    while True:
        act, q = m.serve_run(256)
        if act == 0 and q == 0:
            break
    wall = time.perf_counter() - t0
    tokens, step_ms = m.serve_stats()
    m.close()
    value, ms = pkg.sharding.job_throughput(dist, step_ms, tokens, ws)
    wall_value, wall_ms = pkg.sharding.job_throughput(dist, wall * 1000.0, tokens, ws)
    # algorithmic bytes of the decode steps: weights once per step plus every
    # row's K/V (98 304 B per cached position) and logits
    wbytes = model_weight_bytes(t)
    kvp = 2 * hp["n_layer"] * hp["n_embd"] * 2
    rows_pos = sum(2 * (int(P[i]) + (K + 1) / 2.0) for i in mine)    # mean context per row over the decode
    local_steps = max(1.0, tokens / max(1, len(mine)))
    step_bytes = wbytes + kvp * rows_pos + 2 * len(mine) * hp["n_speech_vocab"] * 4
    ach = step_bytes * local_steps / (step_ms / 1000.0) / 1e9 if step_ms > 0 else 0.0
    return {"config": f"configs[{which}]: {n_total} utterances x CFG, {quant.upper()}, "
                      + ("prompts U[100,400], decode to 1024 tokens or stop" if which == 3 else
                         f"contexts U[50,2048] (prompt U[50,{2048 - K}] + {K} decode steps), per-stream "
                         "temp U[0.6,1] / top_p U[0.8,1] / penalty U[1,1.5]")
                      + f"; streams sharded over {ws} GPU(s) by KV cost",
            "value": value, "unit": UNIT, "scaling": "strong", "n_gpus": ws, "decode_tokens": int(tokens),
            "device_ms": ms, "wall_tokens_per_s": wall_value, "wall_ms": wall_ms,
            "rank0_streams": len(mine), "rank0_achieved_gbs": ach, "rank0_frac": ach / peak, "peak": peak,
            "path": "t3b_serve_run: admit (prefill + first sample) into free slots, one batched step + sampler "
                    "per iteration over all admitted streams, retire at stop / n_predict"}


def reference_default_decode(pkg, hp, t, params, wbytes, peak, steps=1000, device=0):
    """Batch 1 at the reference's defaults: the builtin cond prompt of 375
    speech tokens (src/chatterbox_cli.cpp:707) + 86 text ids (prompt 463) and
    n_predict = 1000 (include/tts-cpp/chatterbox/engine.h:84), stop ignored:
    positions 463 .. 1462, past the 640 that fit the persistent kernel's
    K/V stage at once (the long-context instantiation streams K/V in tiles).
    Same weights as configs[0] with a 375-token cond prompt."""
    rng = np.random.default_rng(7)
    hp2 = dict(hp, cond_prompt_len=375)
    t2 = dict(t)
    ty, _ = t["chatterbox/builtin/cond_prompt_speech_tokens"]
    t2["chatterbox/builtin/cond_prompt_speech_tokens"] = (
        ty, rng.integers(0, hp["start_speech_token"], 375).astype(np.int32))
    m = pkg.T3Model(hp2, t2, device=device)
    try:
        m.alloc_streams(1, 1536)
        text = rng.integers(0, 50257, PROMPT_TEXT).astype(np.int32)
        m.prefill(0, text)
        m.set_rng(0, pkg.T3B_RNG_MT19937, 0, 0)
        m.decode([params], 8, ignore_stop=True)          # warm-up
        P, _ = m.prefill(0, text)
        m.set_rng(0, pkg.T3B_RNG_MT19937, 0, 0)
        n0 = m.launch_count()
        m.decode([params], steps, ignore_stop=True)
        ms = m.last_device_ms()
        launches = m.launch_count() - n0
    finally:
        m.close()
    L_mean = P + (steps + 1) / 2.0
    byts = algorithmic_bytes_per_step(hp, L_mean, wbytes)
    ach = byts / (ms / steps / 1000.0) / 1e9
    return {"config": "batch-1 Q4_0, builtin cond prompt 375 + 86 text ids, 1000 decode steps (stop ignored)",
            "positions": [int(P), int(P + steps - 1)], "value": steps / (ms / 1000.0), "unit": UNIT,
            "ms_per_step": ms / steps, "gpu_launches": launches,
            "roofline": {"achieved_gbs": ach, "peak": peak, "frac": ach / peak, "bytes_per_step": byts, "mean_L": L_mean}}


def sampler_microbench(pkg, torch, peak, reps=200):
    """128 rows x 6563, cond/uncond ~N(0, 3^2), CFG 0.5,
    256-token histories, penalty 1.2, temp 0.8, min_p 0.05, top_k 1000,
    top_p 0.95, one Philox stream per row.  Device time per call: `reps`
    calls captured in a CUDA graph and replayed (CUDA events on the replaying
    stream; host launch cost excluded), median over 5 replays."""
    import ctypes as C
    L = pkg.lib()
    rows, V, HL = 128, 6563, 256
    g = torch.Generator(device="cuda").manual_seed(0)
    cond = torch.randn(rows, V, device="cuda", generator=g) * 3
    unc = torch.randn(rows, V, device="cuda", generator=g) * 3
    hist = torch.randint(0, V, (rows, HL), device="cuda", dtype=torch.int32, generator=g)
    hlen = torch.full((rows,), HL, device="cuda", dtype=torch.int32)
    P = (pkg.SampleParams * rows)(*[pkg.SampleParams.make(1000, 0.95, 0.8, 1.2, 0.05, 0.5)] * rows)
    pd = torch.frombuffer(bytearray(bytes(P)), dtype=torch.uint8).cuda()
    seeds = torch.arange(rows, device="cuda", dtype=torch.int64)
    ctr = torch.zeros(rows, device="cuda", dtype=torch.int64)
    tok = torch.zeros(rows, device="cuda", dtype=torch.int32)
    s = torch.cuda.current_stream()
    a = [C.c_void_p(t.data_ptr()) for t in (cond, unc)]
    args = (a[0], a[1], rows, V, C.c_void_p(hist.data_ptr()), C.c_void_p(hlen.data_ptr()), HL,
            C.c_void_p(pd.data_ptr()), C.c_void_p(seeds.data_ptr()), C.c_void_p(ctr.data_ptr()),
            C.c_void_p(tok.data_ptr()), C.c_void_p(s.cuda_stream))
    for _ in range(5):
        pkg.check(L.t3b_op_sample_philox(*args))
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        gargs = args[:-1] + (C.c_void_p(torch.cuda.current_stream().cuda_stream),)
        for _ in range(reps):
            L.t3b_op_sample_philox(*gargs)
    g.replay()
    torch.cuda.synchronize()
    us = []
    for _ in range(5):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        g.replay()
        e1.record(s)
        torch.cuda.synchronize()
        us.append(e0.elapsed_time(e1) * 1000.0 / reps)
    del g
    us.sort()
    med = us[len(us) // 2]
    byts = 2 * rows * V * 4 + rows * HL * 4 + rows * 4
    return {"config": "configs[1]: 128x6563, CFG 0.5, min_p 0.05, top_k 1000, top_p 0.95, penalty 1.2, temp 0.8, "
                      "Philox", "us_per_step": med, "us_min": us[0], "target_us": 10.0,
            "achieved_gbs": byts / (med * 1e-6) / 1e9, "peak": peak}


def batched_cfg(pkg, torch, peak, steps=256, streams=64, seed=3):
    """BASELINE configs[3] on one GPU: 64 utterances with CFG (128 rows),
    random-init Q8_0 weights, prompts of U[100, 400] positions, `steps`
    decode steps of every stream (stop ignored) through t3b_decode (graph
    path: batched GEMVs, split-K attention, one sampler CTA per stream).
    Device time of the decode loop (library CUDA events); unit = one speech
    token per stream (a CFG pair counts once)."""
    hp = dict(pkg.t3_gguf.T3_TURBO)
    hp, t = pkg.t3_gguf.random_t3(hp, quant="q8_0", seed=seed)
    rng = np.random.default_rng(seed)
    p_target = rng.integers(100, 401, streams)
    warm = 4
    m = pkg.T3Model(hp, t)
    m.alloc_streams(streams, int(p_target.max()) + warm + steps + 8, cfg=True)
    lens = []
    for s in range(streams):
        n_text = int(p_target[s]) - (hp["cond_prompt_len"] + 2)
        P, _ = m.prefill(s, rng.integers(0, 50257, n_text).astype(np.int32))
        m.set_rng(s, pkg.T3B_RNG_PHILOX, seed * 1000 + s)
        lens.append(P)
    params = [pkg.SampleParams.make(**PARAMS, cfg_weight=0.5) for _ in range(streams)]
    m.decode(params, warm, ignore_stop=True)                      # graph capture + warm-up
    torch.cuda.synchronize()
    m.decode(params, steps, ignore_stop=True)
    ms = m.last_device_ms()
    m.close()
    wbytes = model_weight_bytes(t)
    L_mean = float(np.mean(lens)) + warm + (steps + 1) / 2.0
    kv = 2 * hp["n_layer"] * hp["n_embd"] * 2
    step_bytes = wbytes + 2 * streams * kv * (L_mean + 1) + 2 * streams * hp["n_speech_vocab"] * 4
    us = ms * 1000.0 / steps
    ach = step_bytes / (us * 1e-6) / 1e9
    return {"config": "configs[3]: 64 streams x CFG (128 rows), Q8_0, prompts U[100,400], "
                      f"{steps} decode steps per stream, temp 0.8 / top_k 1000 / top_p 0.95 / penalty 1.2 / cfg 0.5",
            "value": streams * steps / (ms / 1000.0), "unit": UNIT, "us_per_step": us,
            "mean_L": L_mean, "bytes_per_step": step_bytes, "achieved_gbs": ach, "peak": peak,
            "frac": ach / peak}


def batched_kernels(pkg, torch, peak, reps=50):
    """The batched decode step's kernels alone at 128 rows, device time per
    call from a CUDA-graph replay of `reps` back-to-back calls (no host
    launch overhead in the number): the fc (1024 -> 4096) and fc2 (4096 ->
    1024) GEMMs of T3 through t3b_op_gemv (activation prep + GEMM) with Q8_0
    weights (mma.sync int8 with the exact per-block rescale) and with F16
    weights (tcgen05 tensor cores, TMA-fed, split-K), and decode attention
    over 16 heads x 400 f16 positions per row through t3b_op_attention (one
    CTA per (row, head)); the attention's K/V (268 MB) exceed L2."""
    import ctypes as C
    import gguf
    L = pkg.lib()
    s = torch.cuda.current_stream()
    sp = C.c_void_p(s.cuda_stream)
    M = 128

    def timed(fn, make_args):
        for _ in range(5):
            pkg.check(fn(*make_args(sp)))                     # warm-up (scratch allocated here)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            cs = C.c_void_p(torch.cuda.current_stream().cuda_stream)
            for _ in range(reps):
                fn(*make_args(cs))
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        g.replay()
        e1.record(s)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1000.0 / reps

    res = {}
    for ty, tname in ((8, "q8_0"), (1, "f16")):
        for K, N in ((1024, 4096), (4096, 1024)):   # fc and fc2 of T3
            w = (np.random.default_rng(2).standard_normal((N, K)) * 0.02).astype(np.float32)
            if ty == 1:
                q = np.ascontiguousarray(w.astype(np.float16))
            else:
                q = np.ascontiguousarray(gguf.quants.quantize(w, gguf.GGMLQuantizationType.Q8_0))
            rb = L.t3b_op_row_bytes(ty, K)
            wd = torch.empty(N * rb, dtype=torch.uint8, device="cuda")
            pkg.check(L.t3b_op_repack(ty, q.ctypes.data, N, K, C.c_void_p(wd.data_ptr())))
            x = torch.randn(M, K, device="cuda")
            y = torch.empty(M, N, device="cuda")

            def args(stream, ty=ty, wd=wd, N=N, K=K, x=x, y=y):
                return (ty, C.c_void_p(wd.data_ptr()), N, K, C.c_void_p(x.data_ptr()), M, None, None, 1e-5, None, None,
                        0, C.c_void_p(y.data_ptr()), stream)
            us = timed(L.t3b_op_gemv, args)
            wbytes = N * rb
            res[f"gemm_{tname}_m128_{'fc' if N > K else 'fc2'}"] = {
                "shape": f"M={M} K={K} N={N}", "us_per_call": us, "tops": 2.0 * M * N * K / (us * 1e-6) / 1e12,
                "weight_gbs": wbytes / (us * 1e-6) / 1e9,
                "kernel": "prep_act + " + ("gemm_f16_tc_kernel (tcgen05)" if ty == 1 else "gemm_q_mma_kernel")}
            del wd
    # batch-1 / few-row decode attention (split-key kernel, M < 8): one row
    # over 1024 cached positions per head
    H1, T1, L1 = 16, 1024, 1024
    kv1 = torch.randn(2, 1, H1, T1, 64, device="cuda").half()
    q1 = torch.randn(1, H1 * 64, device="cuda")
    ln1 = torch.full((1,), L1, dtype=torch.int32, device="cuda")
    o1 = torch.empty(1, H1 * 64, device="cuda")

    def attn1_args(stream):
        return (C.c_void_p(q1.data_ptr()), C.c_void_p(kv1[0].data_ptr()), C.c_void_p(kv1[1].data_ptr()), 1, H1, T1,
                C.c_void_p(ln1.data_ptr()), C.c_void_p(o1.data_ptr()), stream)
    a1_us = timed(L.t3b_op_attention, attn1_args)
    a1_bytes = H1 * L1 * 64 * 2 * 2 + H1 * 64 * 8
    res["attn_decode_m1"] = {"shape": f"M=1 heads={H1} L={L1}", "us_per_call": a1_us, "bytes": a1_bytes,
                             "achieved_gbs": a1_bytes / (a1_us * 1e-6) / 1e9, "peak": peak,
                             "kernel": "attn_decode_kernel (split over 128-key chunks, last CTA merges)"}
    del kv1
    # prompt attention (eval_prompt's causal mask) over a 2048-position prompt
    P_, Hp = 2048, 16
    kvp = torch.randn(2, Hp, P_, 64, device="cuda").half()
    qp = torch.randn(P_, Hp * 64, device="cuda")
    posp = torch.arange(P_, dtype=torch.int32, device="cuda")
    op_ = torch.empty(P_, Hp * 64, device="cuda")

    def prompt_args(stream):
        return (C.c_void_p(qp.data_ptr()), C.c_void_p(kvp[0].data_ptr()), C.c_void_p(kvp[1].data_ptr()), P_, Hp, P_,
                C.c_void_p(posp.data_ptr()), C.c_void_p(op_.data_ptr()), stream)
    p_us = timed(L.t3b_op_attention_prompt, prompt_args)
    p_flops = 4.0 * Hp * 64 * (P_ * (P_ + 1) / 2)
    res["attn_prompt_p2048"] = {"shape": f"P={P_} heads={Hp} causal", "us_per_call": p_us,
                                "tflops": p_flops / (p_us * 1e-6) / 1e12,
                                "kernel": "attn_prefill_kernel (64 x 64 flash tiles, f32 on CUDA cores)"}
    del kvp
    H, T, Lk = 16, 512, 400
    kv = torch.randn(2, M, H, T, 64, device="cuda").half()
    qa = torch.randn(M, H * 64, device="cuda")
    ln = torch.full((M,), Lk, dtype=torch.int32, device="cuda")
    out = torch.empty(M, H * 64, device="cuda")

    def attn_args(stream):
        return (C.c_void_p(qa.data_ptr()), C.c_void_p(kv[0].data_ptr()), C.c_void_p(kv[1].data_ptr()), M, H, T,
                C.c_void_p(ln.data_ptr()), C.c_void_p(out.data_ptr()), stream)
    a_us = timed(L.t3b_op_attention, attn_args)
    a_bytes = M * H * Lk * 64 * 2 * 2 + M * H * 64 * 8
    res["attn_rows_m128"] = {"shape": f"M={M} heads={H} L={Lk}", "us_per_call": a_us, "bytes": a_bytes,
                             "achieved_gbs": a_bytes / (a_us * 1e-6) / 1e9, "peak": peak,
                             "frac": a_bytes / (a_us * 1e-6) / 1e9 / peak}
    return res


def gemv_sweep(pkg, torch, peak, reps=20):
    """the four T3 layer shapes x {Q4_0, Q8_0, F16} x
    M in {1, 2, 8, 32, 128} through t3b_op_gemv (M <= 4: one launch of the
    fused prep + GEMV kernel; 5 <= M < 16: activation prep + GEMV; M >= 16:
    int8 mma.sync (Q4_0/Q8_0) or tcgen05 (F16) GEMM).
    Device time per call: `reps` calls on weights cycled over enough copies
    to exceed L2 are captured into a CUDA graph and replayed, so host launch
    overhead is not in the number.  Algorithmic bytes
    N*K*{0.5625, 1.0625, 2} + M*K*4 + M*N*4."""
    import ctypes as C
    import gguf
    L = pkg.lib()
    s = torch.cuda.current_stream()
    sp = C.c_void_p(s.cuda_stream)
    out = []
    for ty, name in ((2, "q4_0"), (8, "q8_0"), (1, "f16")):
        for K, N in ((1024, 3072), (1024, 1024), (1024, 4096), (4096, 1024)):
            w = (np.random.default_rng(K + N).standard_normal((N, K)) * 0.02).astype(np.float32)
            if ty == 1:
                q = np.ascontiguousarray(w.astype(np.float16))
            else:
                qt = {2: gguf.GGMLQuantizationType.Q4_0, 8: gguf.GGMLQuantizationType.Q8_0}[ty]
                q = np.ascontiguousarray(gguf.quants.quantize(w, qt))
            rb = L.t3b_op_row_bytes(ty, K)
            copies = max(2, int(160e6 // (N * rb)) + 1)
            wd = torch.empty((copies, N * rb), dtype=torch.uint8, device="cuda")
            pkg.check(L.t3b_op_repack(ty, q.ctypes.data, N, K, C.c_void_p(wd[0].data_ptr())))
            wd[1:] = wd[0]
            for M in (1, 2, 8, 32, 128):
                x = torch.randn(M, K, device="cuda")
                y = torch.empty(M, N, device="cuda")

                def call(i, stream):
                    return L.t3b_op_gemv(ty, C.c_void_p(wd[i % copies].data_ptr()), N, K, C.c_void_p(x.data_ptr()),
                                         M, None, None, 1e-5, None, None, 0, C.c_void_p(y.data_ptr()), stream)
                for i in range(3):
                    pkg.check(call(i, sp))
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    cs = C.c_void_p(torch.cuda.current_stream().cuda_stream)
                    for i in range(reps):
                        call(i, cs)
                g.replay()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(s)
                g.replay()
                e1.record(s)
                torch.cuda.synchronize()
                us = e0.elapsed_time(e1) * 1000.0 / reps
                byts = N * rb + M * K * 4 + M * N * 4
                out.append([name, K, N, M, round(us, 2), round(byts / (us * 1e-6) / 1e9, 1),
                            round(2.0 * M * N * K / (us * 1e-6) / 1e12, 2)])
                del g
            del wd
    return {"columns": ["type", "K", "N", "M", "us_per_call", "GB/s", "TOP/s"], "rows": out, "peak": peak,
            "note": "t3b_op_gemv (LN off): M <= 4 gemv_prep_kernel (one launch); 5 <= M < 16 prep_act + GEMV; "
                    "M >= 16 int8 mma.sync GEMM (Q4_0/Q8_0), tcgen05 GEMM (F16); device time per call from "
                    "CUDA-graph replay"}


def phase_timeline(pkg, step=5):
    """Per-phase device timestamps (globaltimer) of one decode step of the
    persistent kernel, every CTA, via the library's T3B_MK_TIMELINE hook.
    Returns medians over CTAs (us from the step's first stamp) for layers 1
    and 12, the head, the sampler and its stages."""
    import tempfile
    tl_path = os.path.join(tempfile.mkdtemp(), "tl.bin")
    os.environ["T3B_MK_TIMELINE"] = tl_path
    os.environ["T3B_MK_TIMELINE_STEP"] = str(step)
    try:
        hp, t = make_model(pkg)
        m = pkg.T3Model(hp, t)
        m.alloc_streams(1, 512)
        m.prefill(0, np.random.default_rng(0).integers(0, 50257, PROMPT_TEXT).astype(np.int32))
        m.set_rng(0, pkg.T3B_RNG_MT19937, 0, 0)
        m.decode([pkg.SampleParams.make(**PARAMS)], 16, ignore_stop=True)
        ms = m.last_device_ms()
        m.close()
    finally:
        os.environ.pop("T3B_MK_TIMELINE", None)
        os.environ.pop("T3B_MK_TIMELINE_STEP", None)
    TL, TLL, TLH = 1024, 32, 800   # stamps per CTA, per layer, first head stamp (megakernel.cuh MK_TL*)
    tl = np.fromfile(tl_path, dtype=np.uint64).reshape(-1, TL).astype(np.int64)
    t0 = tl[tl > 0].min()
    rel = np.where(tl > 0, tl - t0, -1)

    def med(i):
        c = rel[:, i]
        c = c[c >= 0]
        return round(float(np.median(c)) / 1000.0, 2) if c.size else None

    # stamp indices of the Q4_0 kernel (attention CTAs compute their own q/k/v)
    names = {0: "P1 start", 1: "P1 x ready", 12: "P1 LN done", 14: "P1 K/W staged", 15: "P1 qkv dot done",
             16: "P1 V issued", 13: "P1 K/V appended", 9: "P2 softmax", 17: "P2 PV",
             18: "P2 head out Q8_0", 19: "P2 partials", 2: "P2 release barrier", 5: "P2 released",
             4: "P2 next K/W issued", 6: "P4 xm ready", 10: "P4 fc dot done", 20: "P4 h stored",
             21: "P4 done", 3: "P5 start", 7: "P5 h ready", 22: "P5 dot", 11: "P5 dot + next weights issued",
             8: "P5 released"}
    out = {"decode_16_steps_ms": ms, "step": step}
    for l in (1, 12):
        out[f"layer{l}"] = {nm: med(l * TLL + i) for i, nm in names.items() if med(l * TLL + i) is not None}
    out["head"] = {"start": med(TLH), "weights issued": med(TLH + 9), "x ready": med(TLH + 7),
                   "dot done": med(TLH + 8), "released": med(TLH + 1), "sampler logits ready": med(TLH + 2),
                   "sampled": med(TLH + 3), "token seen": med(TLH + 4)}
    st = tl[0, TLH + 10:TLH + 32]
    stages = ["start", "loaded", "min-p", "top-k", "top-p gathered", "sorted", "top-p exp", "top-p psum",
              "top-p cut", "penalty", "compacted", "final exp", "final psum", "rng", "dsum", "end",
              "k:hist", "k:scan", "k:scatter", "k:sort", "p:crossing", "p:fallback"]
    order = sorted([i for i in range(len(stages)) if st[i] > 0], key=lambda i: st[i])
    out["sampler_stages_us"] = {stages[i]: round((st[i] - st[0]) / 1000.0, 2) for i in order}
    return out


def measured_traffic():
    """DRAM bytes per decode step of the megakernel from the committed ncu
    summary (profiles/t3_decode_megakernel_q4_0.md), or None."""
    p = os.path.join(ROOT, "profiles", "t3_decode_megakernel_q4_0.md")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("traffic_bytes_per_step:"):
            return float(line.split(":")[1])
    return None


def gemv_roofline(pkg, torch, peak):
    """Average device time of the FC GEMV (1024 -> 4096, Q4_0, M = 1) through
    t3b_op_gemv (one launch of gemv_prep_kernel), weights > L2 by cycling 48
    distinct weight copies (113 MB); 192 calls captured in a CUDA graph and
    replayed, CUDA events on the replaying stream."""
    import ctypes as C
    import gguf
    L = pkg.lib()
    K, N, copies = 1024, 4096, 48
    w = (np.random.default_rng(1).standard_normal((N, K)) * 0.02).astype(np.float32)
    q = np.ascontiguousarray(gguf.quants.quantize(w, gguf.GGMLQuantizationType.Q4_0))
    rb = L.t3b_op_row_bytes(2, K)
    wd = torch.empty((copies, N * rb), dtype=torch.uint8, device="cuda")
    pkg.check(L.t3b_op_repack(2, q.ctypes.data, N, K, C.c_void_p(wd[0].data_ptr())))
    wd[1:] = wd[0]
    x = torch.randn(K, device="cuda")
    y = torch.empty(N, device="cuda")
    s = torch.cuda.current_stream()

    def call(i, stream):
        return L.t3b_op_gemv(2, C.c_void_p(wd[i % copies].data_ptr()), N, K, C.c_void_p(x.data_ptr()), 1, None, None,
                             1e-5, None, None, 0, C.c_void_p(y.data_ptr()), stream)
    for i in range(8):
        pkg.check(call(i, C.c_void_p(s.cuda_stream)))
    torch.cuda.synchronize()
    reps = copies * 4
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        cs = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        for i in range(reps):
            call(i, cs)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    g.replay()
    e1.record(s)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / reps
    del g
    byts = N * rb + K * 4 + N * 4
    ach = byts / (us * 1e-6) / 1e9
    return {"kernel": "gemv_prep_kernel<Q4_0, 1, 2> (1024x4096, M=1, one launch)", "us_per_launch": us,
            "bytes": byts, "achieved": ach, "peak": peak, "frac": ach / peak}


if __name__ == "__main__":
    sys.exit(main())
