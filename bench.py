#!/usr/bin/env python3
"""Decode throughput of the B200 GPT-2 engine -- BASELINE.json's metric.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c1|c3|c4|c5] [--impl ours|reference]

Workload (default ``c1``, BASELINE.json configs[0] -- the configuration the
north star's B=1 target is quoted on): GPT-2 small, fp32, random N(0, 0.02)
weights, batch 1, a 64-token seeded prompt, then 128 greedy decode steps.
One *step* is one such generation per GPU (prefill + 128 decode steps, all
on the device).  ``value`` is decode tokens per second over all GPUs:
sum(decode steps) / device time of the decode phases, timed with CUDA
events on the engine's stream and taken as the max over ranks; prefill time
is reported beside it.  N GPUs run N independent sequences (replicas of the
weights, no collective on the data path): weak scaling.

``e2e`` times the same workload through the C ABI as a host program drives
it -- g2_prefill, then per token g2_decode (token + position copied from
pinned host memory) and g2_argmax (the token read back) -- wall-clock.

``batched`` (on by default, ``--no-batched`` skips it) measures the two
batched configurations on the same GPUs in the same run, each with its own
tok/s, roofline, e2e and clocks: c5 (GPT-2 XL fp32, 32 sequences per GPU,
weak scaling) and c4 (GPT-2 medium fp16, 32 sequences in total split over
the GPUs, strong scaling); min(K, 5) timed steps each after W warm-up steps.

``--impl reference`` runs the reference's own prefill()/decode()/
sample_next_token() (main.c + math.cl compiled for the host CPU,
oracle/_ref) on this machine's cores, for a bounded sample of the workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "gpt2-opencl-1.1_b200")
for _p in (PKG, os.path.join(ROOT, "oracle")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

CONFIGS = {
    # name: shape, dtype, sequences per GPU, prompt, decode steps
    "c1": dict(shape="SMALL", dtype="f32", batch=1, prompt=64, steps=128, desc="GPT-2 small fp32 B=1 prompt 64 + 128 greedy decode steps"),
    "c3": dict(shape="SMALL", dtype="f32", batch=1, prompt=512, steps=511, desc="GPT-2 small fp32 B=1 prompt 512 + 511 greedy decode steps (fills ctx 1024)"),
    "c4": dict(shape="MEDIUM", dtype="f16", batch=32, prompt=256, steps=256, desc="GPT-2 medium fp16, 32 sequences, prompt 256 + 256 greedy steps"),
    "c5": dict(shape="XL", dtype="f32", batch=32, prompt=128, steps=384, desc="GPT-2 XL fp32, 32 sequences per GPU, prompt 128 + 384 greedy steps"),
}
README_DECODE_MS = 40.2   # reference, GT 730, GPT-2 small fp32 B=1 (README.md:59)
METRIC = "decode tok/s (B=1 ms/token; batched) + HBM GB/s % of peak"
DATA = "synthetic (seeded N(0,0.02) weights, seeded uniform prompt ids)"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    return ws, int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0"))


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, gpu: int):
        self.gpu = gpu
        import tempfile
        self.path = os.path.join(tempfile.gettempdir(), f"g2_clocks_{os.getpid()}.csv")
        self.p = None

    def start(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.f = open(self.path, "w")
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-lms", "20"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self):
        if not self.p:
            return None
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        self.f.close()
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            c = [x.strip() for x in line.split(",")]
            if len(c) < 9:
                continue
            try:
                sm.append(float(c[1]))
                mx = max(mx, float(c[2]))
            except ValueError:
                continue
            for n, v in zip(names, c[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def model_for(cfg):
    from gpt2b200 import synth
    shape = getattr(synth, cfg["shape"])
    name = f"{cfg['shape'].lower()}_{cfg['dtype']}_s0"
    return synth.ensure_model(os.path.join(synth.default_cache(), name), shape, seed=0, dtype=cfg["dtype"]), shape


def wait_for_model(cfg, timeout_s=1800.0):
    """The checkpoint model_for(cfg) names, once another process has finished writing it."""
    from gpt2b200 import synth
    shape = getattr(synth, cfg["shape"])
    d = os.path.join(synth.default_cache(), f"{cfg['shape'].lower()}_{cfg['dtype']}_s0")
    want = synth._tag(shape, 0, cfg["dtype"], False, "conv1d", False, None)
    t0 = time.time()
    while time.time() - t0 < timeout_s:
        try:
            with open(os.path.join(d, "synth.json")) as f:
                if json.load(f) == want:
                    return d, shape
        except (OSError, ValueError):
            pass
        time.sleep(1.0)
    raise RuntimeError(f"timed out waiting for {d}")


def kv_bytes(shape, elem, prompt, steps, batch):
    """KV read + write bytes of `steps` decode steps after a `prompt`-token prefill (per sequence x batch)."""
    L, E = shape.n_layer, shape.n_embd
    rd = sum(elem * L * 2 * E * (prompt + s + 1) for s in range(steps))
    wr = elem * L * 2 * E * steps
    return (rd + wr) * batch


def cpu_sample(cfg, seconds=12.0, force_reference=False):
    """The reference's own code (oracle/_ref) on this host's cores for a bounded sample:
    prefill of the prompt, then decode steps until ~`seconds` have passed."""
    import oracle
    d, shape = model_for(cfg)
    from gpt2b200 import synth
    prompt = synth.prompt_ids(0, cfg["prompt"])
    if (oracle.ref_available() and oracle.ref_fast()) or force_reference:
        ref, kind = oracle.RefMain(d), "reference"
        cores = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
    else:
        ref, kind = oracle.RefModel(d), "port"
        cores = oracle.cpu_lib().ref_num_threads()
    t0 = time.perf_counter()
    ref.prefill(prompt)
    t_pre = time.perf_counter() - t0
    ids = [int(t) for t in prompt]
    lg = ref.logits()
    tok = int(np.argmax(np.where(np.arange(len(lg)) == 50256, -np.inf, lg[:len(lg)])[:shape.vocab_size]))
    n, t0 = 0, time.perf_counter()
    while n < cfg["steps"] and (time.perf_counter() - t0 < seconds or n < 2):
        ids.append(tok)
        ref.decode(tok, len(ids) - 1)
        lg = ref.logits()[:shape.vocab_size]
        lg[50256] = -np.inf
        tok = int(np.argmax(lg))
        n += 1
    t_dec = time.perf_counter() - t0
    ref.close()
    return {"value": round(n / t_dec, 4), "unit": "tok/s", "cores": cores, "kind": kind,
            "sample": f"prefill {cfg['prompt']} tokens ({t_pre:.1f} s) + {n} greedy decode steps of the {cfg['shape']} "
                      f"workload, batch 1 (per-sequence rate)", "prefill_s": round(t_pre, 3)}


def run_c2(args):
    """C2: per-kernel microbench on the device pointers entry points (g2k_*), weights rotating
    over a pool larger than L2 so HBM is what is measured; one JSON line with every case."""
    import torch
    import gpt2b200 as g2
    peak_gbs, _ = peaks()
    try:
        bf16 = float(json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["bf16_tflops"])
    except Exception:
        bf16 = 1590.0
    gen = torch.Generator(device="cuda").manual_seed(0)
    dev = torch.device("cuda")
    L2 = 126 * 2**20
    cases = []

    stream = torch.cuda.Stream()

    def timed(fn, reps):
        """Device time per call: `reps` calls captured in a CUDA graph (no host launch
        overhead in the timed region), replayed between events."""
        with torch.cuda.stream(stream):
            for i in range(3):
                fn(i, stream.cuda_stream)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(reps):
                fn(i, stream.cuda_stream)
        g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            a.record()
            g.replay()
            b.record()
        torch.cuda.synchronize()
        del g
        return a.elapsed_time(b) * 1000.0 / reps   # us per call

    shapes = [("qkv", 2304, 768), ("attn_proj", 768, 768), ("ffn1", 3072, 768), ("ffn2", 768, 3072),
              ("lm_head", 50260, 768)]
    for name, N, K in shapes:
        wbytes = 4 * N * K
        pool = max(2, -(-3 * L2 // wbytes))
        W = torch.randn(pool, K, N, generator=gen, device=dev) * 0.02
        x = torch.randn(K, generator=gen, device=dev)
        y = torch.zeros(N, device=dev)
        wsb = g2.matvec_workspace(N, K)
        ws = torch.zeros(wsb // 4 + 64, device=dev)
        us = timed(lambda i, st: g2.matvec(x, W[i % pool], y, N, K, workspace=ws, workspace_bytes=wsb, stream=st),
                   4 * pool)
        gbs = (wbytes + 4 * (N + K)) / us / 1e3
        cases.append({"kernel": "gemv_kernel (g2k_matvec)", "case": f"{name} {K}->{N}, B=1 fp32", "us": round(us, 2),
                      "GB/s": round(gbs, 1), "frac_hbm": round(gbs / peak_gbs, 3)})
        del W
    for M in (64, 256, 1024):
        for name, N, K in shapes[:4]:
            for prec, pname in ((g2.G2_F32, "3xTF32"), (g2.G2_F16, "fp16")):
                pool = max(2, -(-3 * L2 // (4 * N * K)))
                W = torch.randn(pool, K, N, generator=gen, device=dev) * 0.02
                A = torch.randn(M, K, generator=gen, device=dev)
                Cm = torch.zeros(M, N, device=dev)
                wsb = g2.matmul_tc_workspace(M, N, K, prec)
                ws = torch.zeros(wsb // 4 + 64, device=dev)
                us = timed(lambda i, st: g2.matmul_tc(A, W[i % pool], Cm, M, N, K, precision=prec, workspace=ws,
                                                      workspace_bytes=wsb, stream=st), 2 * pool)
                tf = 2.0 * M * N * K / us / 1e6
                cases.append({"kernel": "tc_gemm_kernel (g2k_matmul_tc, incl. operand split + reduce)",
                              "case": f"{name} M={M} {K}->{N} {pname}", "us": round(us, 2), "TFLOP/s": round(tf, 2),
                              "frac_bf16": round(tf / bf16, 4)})
                del W
            if M == 64:
                W = torch.randn(K, N, generator=gen, device=dev) * 0.02
                A = torch.randn(M, K, generator=gen, device=dev)
                Cm = torch.zeros(M, N, device=dev)
                us = timed(lambda i, st: g2.matmul(A, W, Cm, M, N, K, stream=st), 10)
                cases.append({"kernel": "gemm_kernel (g2k_matmul, SIMT fp32)", "case": f"{name} M={M} {K}->{N}",
                              "us": round(us, 2), "TFLOP/s": round(2.0 * M * N * K / us / 1e6, 2)})
    H, S = 12, 1024
    for T in (64, 128, 256, 512, 1024):
        pool = 8
        Kc = torch.randn(pool, H, S, 64, generator=gen, device=dev)
        Vc = torch.randn(pool, H, S, 64, generator=gen, device=dev)
        q = torch.randn(H * 64, generator=gen, device=dev)
        out = torch.zeros(H * 64, device=dev)
        wsb = g2.attention_workspace(H, S)
        ws = torch.zeros(wsb // 4 + 64, device=dev)
        us = timed(lambda i, st: g2.attention(q, Kc[i % pool], Vc[i % pool], out, H, S, T, ws, wsb, stream=st),
                   4 * pool)
        by = 2 * H * T * 64 * 4
        cases.append({"kernel": "attn_kernel (g2k_attention)", "case": f"12 heads x 64, T_kv={T}", "us": round(us, 2),
                      "GB/s": round(by / us / 1e3, 1), "frac_hbm": round(by / us / 1e3 / peak_gbs, 3)})
        del Kc, Vc
    line = {"metric": "C2 kernel microbench (device us per call from CUDA-graph replay; GB/s or TFLOP/s)", "value": None, "unit": "per case",
            "n_gpus": 1, "higher_is_better": True, "config": {"workload": "c2", "pool": "weights rotate over > 3x L2"},
            "peaks": {"hbm_gbs": peak_gbs, "bf16_tflops": bf16}, "cases": cases}
    print(json.dumps(line), flush=True)


def weight_bytes(shape, elem):
    """Weights, biases and LayerNorm parameters streamed per decode step (the engine's
    g2_config.weight_bytes): elem * [L (4E^2 + 2EF) + E V_pad] + elem * [L (9E + F) + 2E]."""
    L, E, F = shape.n_layer, shape.n_embd, shape.ffn
    return elem * (L * (4 * E * E + 2 * E * F) + E * shape.padded_vocab) + elem * (L * (9 * E + F) + 2 * E)


def workload_config(name, cfg, ws, rank=0):
    """The `config` object of a line for workload `name` on `ws` GPUs (the same in both arms)."""
    from gpt2b200 import replicas, synth
    shape = getattr(synth, cfg["shape"])
    scaling = "strong" if name == "c4" else "weak"
    B = len(replicas.shard(cfg["batch"], ws, rank, scaling))
    wb = weight_bytes(shape, 2 if cfg["dtype"] == "f16" else 4)
    return {"workload": name, "description": cfg["desc"], "sequences_per_gpu": B,
            "sequences_total": cfg["batch"] * (ws if scaling == "weak" else 1), "decode_steps_per_step": cfg["steps"],
            "parallelism": f"replicas x{ws} (independent sequences)",
            "l2": f"weights {wb / 1e6:.0f} MB per decode step > 126 MB L2 (no flush needed)"}


def run_reference(args, cfg):
    """The reference's own code (oracle/_ref: main.c + math.cl compiled for the host
    CPU) on this machine's cores.  Under torchrun only rank 0 runs; it takes every
    host core (OMP_NUM_THREADS is set before the library loads, overriding
    torchrun's 1).  N GPUs' worth of sequences would run one after another on
    those cores, so the job's rate equals the single-sequence rate measured here."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    os.environ["OMP_NUM_THREADS"] = str(os.cpu_count() or 1)
    try:
        import oracle
        if not oracle.ref_available():
            raise RuntimeError("oracle/_ref not built")
    except Exception as ex:
        print(json.dumps({"impl": "reference", "unavailable": f"reference CPU build missing: {ex}"}))
        return
    per = []
    total_steps = args.warmup + args.steps
    budget = max(4.0, 150.0 / max(total_steps, 1))
    for i in range(total_steps):
        r = cpu_sample(cfg, seconds=budget)
        if i >= args.warmup:
            per.append(r)
    val = statistics.mean(p["value"] for p in per)
    line = {"metric": METRIC, "value": round(val, 4),
            "unit": "tok/s", "impl": "reference", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1000.0 / val, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": DATA,
            "config": workload_config(args.config, cfg, ws),
            "cpu_baseline": {k: per[-1][k] for k in ("kind", "cores", "sample")} | {"value": round(val, 4), "unit": "tok/s"},
            "e2e": {"value": round(val, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": (f"{ws} GPU(s)' worth of sequences run one after another on all {os.cpu_count()} host threads: "
                     "the job's rate is the single-sequence rate" if ws > 1 else None)}
    print(json.dumps(line))


class Measured(dict):
    pass


def measure(name, cfg, args, steps, warmup, ws, rank, local, dist, torch, g2, synth, replicas, loaded):
    """One workload on this rank's engine: `warmup` untimed generations, then `steps`
    timed ones (device time of the decode phases, CUDA events on the engine's
    stream), then the e2e runs through the C ABI with host buffers.  Returns the
    line's fields (on every rank; timings are max over ranks)."""
    d, shape = loaded[name]
    scaling = "strong" if name == "c4" else "weak"
    mine = replicas.shard(cfg["batch"], ws, rank, scaling)
    B = len(mine)
    dtype = g2.G2_F16 if cfg["dtype"] == "f16" else g2.G2_F32
    eng = g2.Engine(d, device=local if ws > 1 else 0, max_batch=max(B, 1), dtype=dtype)
    n_new = cfg["steps"] + 1
    prompts = [synth.prompt_ids(i, cfg["prompt"]) for i in mine]

    def one_step():
        if B == 1:
            eng.generate(prompts[0], n_new)
        else:
            eng.generate_batch(prompts, n_new)
        return eng.last_timing()

    for _ in range(warmup):
        one_step()
    barrier = (lambda: (dist.barrier(), torch.cuda.synchronize())) if ws > 1 else torch.cuda.synchronize
    clocks = Clocks(local)
    barrier()
    clocks.start()
    l0 = eng.launch_count()
    t0 = time.perf_counter()
    pre_ms = dec_ms = 0.0
    dec_steps = 0
    for _ in range(steps):
        p, dm, nd = one_step()
        pre_ms += p
        dec_ms += dm
        dec_steps += nd
    eng.synchronize()
    wall = time.perf_counter() - t0
    barrier()
    clk = clocks.stop()
    launches = eng.launch_count() - l0
    # e2e: the same workload through the C ABI with host buffers, wall-clock: g2_generate(_batch)
    # (prompt ids copied from host memory, generated ids copied back), and for B = 1 also
    # the reference's host loop (g2_prefill, then per token g2_decode + g2_argmax).
    e2e_t, loop_t, loop_tokens = 0.0, 0.0, 0
    reps = max(1, min(steps, 3))
    for _ in range(reps):
        t1 = time.perf_counter()
        if B == 1:
            eng.generate(prompts[0], n_new)
        else:
            eng.generate_batch(prompts, n_new)
        e2e_t += time.perf_counter() - t1
    if B == 1:
        for _ in range(reps):
            t1 = time.perf_counter()
            eng.prefill(prompts[0])
            tok, _ = eng.argmax(forbid_eos=True)
            pos = cfg["prompt"]
            for s_ in range(cfg["steps"]):
                eng.decode(tok, pos + s_)
                tok, _ = eng.argmax(forbid_eos=True)
            loop_t += time.perf_counter() - t1
            loop_tokens += cfg["steps"]
    # --lm-shard (c5 only): the same generation with the LM head split over the ranks by
    # vocabulary rows (gpt2b200.lmshard), wall-clock with prefill, beside g2_generate_batch's
    shard_t = 0.0
    if getattr(args, "lm_shard", False) and name == "c5" and B > 1:
        from gpt2b200 import lmshard
        dev = torch.device("cuda", local if ws > 1 else 0)
        lmshard.generate_batch_sharded(eng, prompts, n_new, dev)   # warm-up
        for _ in range(reps):
            t1 = time.perf_counter()
            lmshard.generate_batch_sharded(eng, prompts, n_new, dev)
            shard_t += time.perf_counter() - t1
    cfgd = eng.cfg
    elem = 2 if cfg["dtype"] == "f16" else 4
    per_seq_kv = kv_bytes(shape, elem, cfg["prompt"], cfg["steps"], 1)
    bytes_per_step = cfgd.weight_bytes + per_seq_kv * B / cfg["steps"] + B * (2 * shape.n_embd * elem + 4 * shape.padded_vocab)
    persistent = bool(cfgd.persistent) and B == 1
    eng.close()
    dec_max, pre_max, wall_max, e2e_max, loop_max, shard_max = replicas.max_over_ranks(
        [dec_ms, pre_ms, wall, e2e_t, loop_t, shard_t], device="cuda")
    n_total = cfg["batch"] * (ws if scaling == "weak" else 1)    # sequences over all ranks
    total_tokens = dec_steps * n_total
    value = total_tokens / (dec_max / 1000.0)
    step_s = dec_max / 1000.0 / max(dec_steps, 1)            # seconds per decode step (all B rows of a rank)
    achieved = bytes_per_step / step_s / 1e9
    peak, peak_kind = peaks()
    traffic = None
    tp = os.path.join(ROOT, "profiles", f"traffic_{name}.json")
    if os.path.exists(tp):
        traffic = json.load(open(tp)).get("bytes_per_decode_step")
    kernel = ("mega_decode_kernel (persistent: every layer, LM head and greedy argmax of all decode steps "
              "in one launch)" if persistent else
              "decode step kernels (embed, 5-7 per layer on the tensor cores, LM head + argmax) in a CUDA graph")
    h2d = 4 * B * cfg["prompt"] + 12 * B
    d2h = 4 * B * n_new
    m = Measured(
        value=round(value, 3), unit="tok/s", steps=steps, warmup=warmup, scaling=scaling,
        ms_per_step=round((dec_max + pre_max) / max(steps, 1), 4),
        ms_per_token=round(1000.0 * step_s, 5) if B == 1 else None,
        ms_per_decode_step=round(1000.0 * step_s, 5),
        prefill_ms=round(pre_max / max(steps, 1), 4),
        dtype=cfg["dtype"],
        config=workload_config(name, cfg, ws),
        roofline={"bound": "hbm", "kernel": kernel, "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                  "frac": round(achieved / peak, 4), "peak_source": peak_kind, "bytes_per_step": int(bytes_per_step),
                  "traffic": traffic},
        e2e={"value": round(cfg["steps"] * n_total / e2e_max * reps, 3) if e2e_max > 0 else None, "unit": "tok/s",
             "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
             "path": ("g2_generate" if B == 1 else "g2_generate_batch") + " (C ABI, host buffers, wall-clock, "
                     "prefill included)",
             "host_loop": ({"value": round(loop_tokens * ws / loop_max, 3), "unit": "tok/s",
                            "path": "g2_prefill + per-token g2_decode/g2_argmax (the reference's host loop)"}
                           if loop_max > 0 else None)},
        gpu_launches=int(launches) * ws, wall_s=round(wall_max, 4))
    if shard_max > 0:
        m["lm_shard"] = {"e2e": round(cfg["steps"] * n_total / shard_max * reps, 3), "unit": "tok/s",
                         "unsplit_e2e": m["e2e"]["value"],
                         "path": f"LM head split by vocabulary rows over {ws} GPU(s) (gpt2b200.lmshard: NCCL "
                                 "all-gather of rows and of per-row bests), wall-clock, prefill included"}
    if clk:
        m["clocks"] = clk
    return m


def run_ours(args, cfg):
    import torch
    ws, rank, local = dist_env()
    dist = None
    if ws > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    import gpt2b200 as g2
    from gpt2b200 import replicas, synth
    names = [args.config] + ([b for b in ("c4", "c5") if b != args.config] if args.batched else [])
    # The synthetic checkpoints are written once per node, by local rank 0; the other
    # ranks wait for each one's completion tag (written last) outside any collective.
    loaded = {}
    for n in names:
        c = dict(CONFIGS[n])
        if local == 0:
            loaded[n] = model_for(c)
    for n in names:
        if local != 0:
            loaded[n] = wait_for_model(dict(CONFIGS[n]))
    main = measure(args.config, cfg, args, args.steps, args.warmup, ws, rank, local, dist, torch, g2, synth,
                   replicas, loaded)
    batched = {}
    for n in names[1:]:
        c = dict(CONFIGS[n])
        k = min(args.steps, 5)
        batched[n] = measure(n, c, args, k, args.warmup, ws, rank, local, dist, torch, g2, synth, replicas, loaded)
    if rank == 0:
        line = {"metric": METRIC, "value": main["value"], "unit": "tok/s", "n_gpus": ws, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": main["ms_per_step"], "ms_per_token": main["ms_per_token"],
                "prefill_ms": main["prefill_ms"], "higher_is_better": True, "scaling": main["scaling"],
                "vs_baseline": (round((main["value"] / ws) / (1000.0 / README_DECODE_MS), 2)
                                if args.config in ("c1", "c3") else None),
                "dtype": cfg["dtype"], "data": DATA, "config": main["config"],
                "roofline": main["roofline"], "e2e": main["e2e"], "gpu_launches": main["gpu_launches"],
                "wall_s": main["wall_s"]}
        if "clocks" in main:
            line["clocks"] = main["clocks"]
        if "lm_shard" in main:
            line["lm_shard"] = main["lm_shard"]
        if batched:
            line["batched"] = {n: dict(b) for n, b in batched.items()}
            line["gpu_launches"] += sum(b["gpu_launches"] for b in batched.values())
        if ws == 1 and not args.no_cpu_baseline:
            try:
                line["cpu_baseline"] = cpu_sample(cfg)
            except Exception as ex:   # reported, never fatal
                line["cpu_baseline"] = {"error": str(ex)}
        print(json.dumps(line), flush=True)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="c1", choices=sorted(CONFIGS) + ["c2"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--lm-shard", action="store_true",
                    help="also time c5 with the LM head split over the GPUs by vocabulary rows")
    ap.add_argument("--no-batched", dest="batched", action="store_false",
                    help="skip the batched sub-object (c4 and c5 on the same GPUs)")
    ap.add_argument("--decode-steps", type=int, default=0,
                    help="override the workload's decode steps (short runs for profiler captures; not a bench number)")
    args = ap.parse_args()
    if args.config == "c2":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "c2 is a per-kernel device microbench"}))
        else:
            run_c2(args)
        return
    cfg = dict(CONFIGS[args.config])
    if args.decode_steps > 0:
        cfg["steps"] = args.decode_steps
    ws, _, _ = dist_env()
    if args.impl == "reference":
        run_reference(args, cfg)
    else:
        run_ours(args, cfg)


if __name__ == "__main__":
    main()
