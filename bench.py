#!/usr/bin/env python
"""Batch-1 greedy decode benchmark of the token loop (one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: the 4B-shape Llama model with TQ1_0
linear weights and a Q8_0 embedding/head (seeded random-init, synthetic), a
512-id random prompt, greedy decoding (`fox run --temp 0`: repeat penalty 1.1
over the last 64 tokens), fp16 KV cache, context 4096. A step is one decode
token. The weights (1.18 GB) are far larger than the 126 MB L2, so every step
streams them from HBM; no L2 flush is needed.

  value  tokens/s of K decode steps run on the device with the picked token fed
         back on the device (CUDA graphs; CUDA-event time, max over ranks)
  e2e    tokens/s of K decode steps through the C ABI (foxcuda_decode): each
         step copies the input token from pinned host memory and reads the
         picked token back
  roofline  the dominant kernel (the fused gate|up TQ1_0 GEMV), timed live
         with CUDA events on its launching stream over successive layers

Under torchrun (`--gpus N`, any N) the workload is config 4 instead: the 27B
TQ2_0 model, one sequence split over the N ranks (tensor parallel, strong
scaling; run_tp). N = 1 there is the single-GPU decode of the 27B model, the
baseline of the speed-up. A plain `python bench.py` times config 2 on one GPU.

--impl reference times upstream RustFox's own CPU implementation (the library
built from the upstream sources, oracle/_ref) on this host's cores for the
same metric and config.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = ("batch-1 decode tok/s and achieved HBM GB/s (% of 8 TB/s) per model, 1/2/4/8 B200")
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default=None,
                    help="model config (default: 4b; 27b under torchrun or with --tp)")
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--ctx", type=int, default=4096)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--tp", action="store_true",
                    help="one sequence split over the GPUs (tensor parallel, strong scaling) "
                         "instead of one replica per GPU")
    ap.add_argument("--gemm", default=None, metavar="M[,M...]",
                    help="time the M-token tensor-core pass over one layer's matrices "
                         "(prefill / verification) instead of decoding")
    ap.add_argument("--exchange", default="sums", choices=["nccl", "p2p", "sums"],
                    help="tensor parallel: collectives through NCCL, the library's bit-exact "
                         "term exchange over peer memory, or its partial-sum exchange")
    ap.add_argument("--split", action="store_true",
                    help="with --gemm: also time the split form of the pass")
    ap.add_argument("--prefill", action="store_true",
                    help="time fox_eval of a --prompt long prompt (chunks through the tensor "
                         "cores, and token by token) next to upstream's CPU fox_eval")
    ap.add_argument("--batch", type=int, default=0, metavar="N",
                    help="decode N sequences together at a --ctx long synthetic context "
                         "(config 5: --config 8b-tq2 --batch 16 --ctx 32768)")
    ap.add_argument("--contiguous", action="store_true",
                    help="with --batch: one contiguous cache per sequence instead of pages "
                         "from one shared pool")
    ap.add_argument("--attention", action="store_true",
                    help="time the tile attention on its own (foxcuda_attention, one sequence, fp16 "
                         "caches) at 32768 positions and at the 4B and 27B decode shapes")
    ap.add_argument("--image", action="store_true",
                    help="time the model load: tensors uploaded and packed on the device, "
                         "against a device image opened from a file")
    args = ap.parse_args()
    if args.config is None:
        args.config = "27b" if (args.tp or under_torchrun()) else "4b"
    return args


def under_torchrun() -> bool:
    """Launched by torch.distributed.run (any number of ranks)."""
    return "TORCHELASTIC_RUN_ID" in os.environ or "WORLD_SIZE" in os.environ


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


TYPE_NAMES = {0: "F32", 1: "F16", 8: "Q8_0", 12: "Q4_K", 14: "Q6_K", 34: "TQ1_0", 35: "TQ2_0"}


def workload(cfg, args) -> dict:
    lin = TYPE_NAMES[cfg.linear_type]
    if cfg.attn_v_type and cfg.attn_v_type != cfg.linear_type:
        lin += f" (attn_v {TYPE_NAMES[cfg.attn_v_type]})"
    wb = cfg.weight_bytes()
    gb = (wb["layers"] + wb["output"]) / 1e9
    return {"workload": f"{cfg.name} {cfg.n_layer}L/{cfg.n_embd} {lin} linear + "
                        f"{TYPE_NAMES[cfg.output_type]} head, batch-1 greedy decode after a "
                        f"{args.prompt}-id prompt",
            "prompt": args.prompt, "n_ctx": args.ctx, "kv_cache": "f16",
            "sampler": "greedy, repeat penalty 1.1 over 64",
            "l2": f"weights {gb:.2f} GB per step > 126 MB L2: streamed from HBM, no flush"}


def measured_hbm_gbs():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class Clocks:
    """nvidia-smi samples every 200 ms while the timed regions run."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.device)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---- CPU side: upstream's own implementation ------------------------------
def reference_decode(model, cfg, warmup: int, steps: int, budget_s: float = 60.0, n_prompt: int = 512):
    """Upstream fox_eval greedy decode on this host (oracle/_ref, the upstream
    sources built with their default -O3 and AVX2/FMA code generation), the
    loop of `fox run --temp 0` (src/cli.c:333-361) on token ids, after the
    same n_prompt-id prompt as the device's decode (so both read a cache of
    the same length; the prompt itself is not timed). Returns (tok/s, cores,
    sample description, kind)."""
    from oracle import oracle as O
    from rustfox_b200 import synth
    prompt = synth.random_prompt(cfg, n_prompt, seed=1)
    with tempfile.TemporaryDirectory() as d:
        path = synth.write_gguf(model, os.path.join(d, "model.gguf"), tokenizer=False)
        if os.path.exists(O.REF_FAST_SO):
            ref = O.RefLib(fast=True)
            kind = "reference"
            cores = int(ref.L.fox_cpu_count_online())
            m = ref.open_model(path)
            n_ctx = n_prompt + max(1, warmup) + steps + 8
            ctx = ref.context(m, n_ctx, 32, 0)
            smp_cfg = O.SamplerConfig(0.0, 40, 0.95, 1.1, 64, 0)
            smp = ref.L.fox_sampler_create(O.C.byref(smp_cfg), cfg.n_vocab)
            logits = ref.eval(ctx, prompt, cfg.n_vocab)
            for t in prompt:
                ref.L.fox_sampler_accept(smp, int(t))

            def pick(lg):
                o = np.zeros(1, np.uint32)
                lg = np.ascontiguousarray(lg, np.float32)
                ref.L.fox_sampler_pick(smp, O._ptr(lg), O._ptr(o))
                ref.L.fox_sampler_accept(smp, int(o[0]))
                return int(o[0])

            tok = pick(logits)
            t_tok = None
            for _ in range(max(1, warmup)):
                logits = ref.eval(ctx, [tok], cfg.n_vocab)
                t_tok = ref.L.fox_context_last_eval_seconds(ctx)
                tok = pick(logits)
            n = max(2, min(steps, int(budget_s / max(t_tok, 1e-6))))
            total = 0.0
            for _ in range(n):
                logits = ref.eval(ctx, [tok], cfg.n_vocab)
                total += ref.L.fox_context_last_eval_seconds(ctx)
                tok = pick(logits)
            ref.L.fox_sampler_destroy(smp)
            ref.L.fox_context_destroy(ctx)
            ref.L.fox_model_close(m)
        else:  # the upstream sources were not available where this was built
            kind = "port"
            cores = os.cpu_count() or 1
            om = O.OracleModel(model)
            octx = om.context(n_prompt + max(1, warmup) + steps + 8)
            octx.eval(prompt)
            n = max(2, min(steps, 8))
            t0 = time.perf_counter()
            for i in range(n):
                octx.eval([int(prompt[i % len(prompt)])])
            total = time.perf_counter() - t0
    sample = (f"{n} greedy decode tokens after a {n_prompt}-id prompt and {max(1, warmup)} warm-up "
              f"tokens (fox_eval time per token, as `fox run` reports gen tok/s)")
    return n / total, cores, sample, kind


def reference_cli(model, n_gen: int = 8):
    """Upstream's own `fox run` binary (oracle/_ref/fox, built from the upstream
    sources) on the same model with its byte-level vocabulary: --temp 0 (the
    CLI's greedy with its default repeat penalty), all cores, the gen tok/s it
    prints (src/cli.c:364-369). The prompt has no spaces: the CLI sizes its id
    buffer from the prompt's length, and each space costs three byte ids.
    Returns a dict for the record, or None when the binary is absent."""
    from oracle import oracle as O
    from rustfox_b200 import synth
    fox = os.path.join(os.path.dirname(O.REF_FAST_SO), "fox")
    if not os.path.exists(fox):
        return None
    prompt = "thequickbrownfox"
    with tempfile.TemporaryDirectory() as d:
        path = synth.write_gguf(model, os.path.join(d, "model.gguf"), tokenizer=True)
        cmd = [fox, "run", path, "-p", prompt, "-n", str(n_gen), "--temp", "0", "--ctx", "64"]
        res = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    out = {"command": "fox run model.gguf -p " + prompt + f" -n {n_gen} --temp 0 --ctx 64",
           "exit": res.returncode}
    for line in res.stderr.splitlines():
        parts = line.split()
        if parts and parts[0] in ("prompt", "gen") and "tok/s)" in line:
            out[f"{parts[0]}_tok_s"] = float(line.rsplit("(", 1)[1].split()[0])
    return out


def cpu_model() -> str:
    """The host CPU's model name (/proc/cpuinfo), for the CPU-baseline record."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def reference_decode_sampled(cfg, warmup: int, steps: int, n_prompt: int, budget_s: float = 40.0):
    """Upstream's decode of a model too large to generate here in minutes
    (config 4: 62 layers of 27B shape): the same decode timed on 1-layer and
    2-layer models with the config's shapes, types, embedding and head
    (bytes drawn uniformly, synth.timing_sample), the per-token time taken
    as t1 + (n_layer - 1) * (t2 - t1). Returns (tok/s, cores, sample, kind)."""
    from rustfox_b200 import synth
    shared = {}
    per = []
    for n in (1, 2):
        m = synth.timing_sample(cfg, n, shared=shared)
        v, cores, _, kind = reference_decode(m, m.cfg, warmup, steps, budget_s=budget_s / 2,
                                             n_prompt=n_prompt)
        per.append(1.0 / v)
    t = per[0] + (cfg.n_layer - 1) * max(per[1] - per[0], 0.0)
    sample = (f"fox_eval per-token time of 1- and 2-layer models with {cfg.name}'s shapes, types, "
              f"embedding and head ({per[0] * 1e3:.1f} and {per[1] * 1e3:.1f} ms after a "
              f"{n_prompt}-id prompt), extended to {cfg.n_layer} layers as t1 + "
              f"{cfg.n_layer - 1} x (t2 - t1)")
    return 1.0 / t, cores, sample, kind


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from rustfox_b200 import synth
    cfg = synth.CONFIGS[args.config]
    if args.config == "27b":  # the torchrun workload (run_tp)
        cli = None
        v, cores, sample, kind = reference_decode_sampled(cfg, args.warmup, args.steps, args.prompt)
        work = {"workload": f"{cfg.name} {cfg.n_layer}L/{cfg.n_embd} TQ2_0 linear + Q8_0 head, "
                            f"batch-1 greedy decode after a {args.prompt}-id prompt",
                "prompt": args.prompt, "sampler": "greedy, repeat penalty 1.1 over 64",
                "parallelism": f"the upstream CPU decode (one process) against tp{world}"}
    else:
        model = synth.generate(cfg)
        cli = reference_cli(model)
        v, cores, sample, kind = reference_decode(model, cfg, args.warmup, args.steps,
                                                  n_prompt=args.prompt)
        work = workload(cfg, args)
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 / v,
            "higher_is_better": True, "scaling": "strong" if args.config == "27b" else "weak",
            "vs_baseline": None,
            "dtype": "i8 x ternary -> i32, f32", "data": "synthetic (seeded random-init weights, "
            "uniform random prompt ids)",
            "config": {**work, "kv_cache": "f32 (upstream's cache)"},
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": kind,
                             "sample": sample, "cpu": cpu_model()},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "fox_run_cli": cli}
    print(json.dumps(line), flush=True)


# ---- GPU side ----------------------------------------------------------------
def run_ours(args):
    import torch
    import rustfox_b200 as rf
    from rustfox_b200 import synth

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(minutes=10))

    def barrier_max(x: float) -> float:
        torch.cuda.synchronize()
        if dist is None:
            return x
        t = torch.tensor([x], device=f"cuda:{local}", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    cfg = synth.CONFIGS[args.config]
    host_model = synth.generate(cfg)
    model = rf.Model.from_synthetic(host_model, device=local)
    ctx = model.context(args.ctx, kv="f16")
    smp = rf.Sampler(ctx, temperature=0.0)  # `fox run --temp 0` defaults otherwise
    prompt = synth.random_prompt(cfg, args.prompt, seed=1)
    need = args.prompt + 2 * (args.warmup + args.steps) + 2
    if need > args.ctx:
        raise SystemExit(f"context {args.ctx} too small for {need} positions")
    ctx.eval(prompt, want_logits=False)
    for t in prompt:
        smp.accept(int(t))
    tok = smp.pick()
    smp.accept(tok)

    clocks = Clocks(local)
    # device-resident decode: K graph launches, token fed back on the device
    tok = int(smp.generate(tok, max(3, args.warmup))[-1])
    pos0 = ctx.pos
    barrier()
    clocks.start()
    toks = smp.generate(tok, args.steps)
    dev_s = barrier_max(ctx.last_eval_seconds)
    tok = int(toks[-1])

    # end to end through the C ABI: H2D token, one-graph step, D2H pick
    for _ in range(max(3, args.warmup)):
        tok = smp.decode(tok)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        tok = smp.decode(tok)
    e2e_s = barrier_max(time.perf_counter() - t0)
    clk = clocks.stop()

    # the dominant kernel, timed live on its stream over successive layers
    kern_us, w_bytes = ctx.bench_kernel("gate_up", reps=2 * cfg.n_layer)
    algo_bytes = w_bytes + cfg.n_embd * 4 + cfg.n_ff * 4
    peak, peak_kind = measured_hbm_gbs()
    achieved = algo_bytes / (kern_us * 1e-6) / 1e9
    traffic = None
    tp = os.path.join(ROOT, "profiles", "roofline_traffic.json")
    if os.path.exists(tp):
        with open(tp) as f:
            traffic = json.load(f).get(args.config, {}).get("gate_up_dram_bytes_per_launch")

    wb = cfg.weight_bytes()
    mean_pos = pos0 + args.steps / 2
    bytes_tok = wb["layers"] + wb["output"] + wb["embd_row"] + wb["norms"] + \
        cfg.kv_bytes_per_token(int(mean_pos))
    value = world * args.steps / dev_s
    per_gpu = args.steps / dev_s
    launches_per_tok = 1 + cfg.n_layer * 5 + 1 + 1 + 2

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            v, cores, sample, kind = reference_decode(host_model, cfg, 2, 8, budget_s=25.0, n_prompt=args.prompt)
            cpu = {"value": v, "unit": "tok/s", "cores": cores, "kind": kind, "sample": sample,
                   "cpu": cpu_model()}
        except Exception as e:  # the baseline is reported, never required
            cpu = {"value": None, "unit": "tok/s", "cores": None, "kind": "reference",
                   "sample": f"failed: {e}"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * dev_s / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "i8 x ternary -> i32, f32", "data": "synthetic (seeded random-init weights, "
            "uniform random prompt ids)",
            "config": {**workload(cfg, args), "parallelism": f"{world} replica(s)"},
            "hbm_bytes_per_token": bytes_tok,
            "hbm_gbs_per_gpu": bytes_tok * per_gpu / 1e9,
            "hbm_frac_of_8tbs": bytes_tok * per_gpu / 1e9 / NOMINAL_HBM_GBS,
            "roofline": {"bound": "hbm",
                         "kernel": f"fused gate|up {TYPE_NAMES[cfg.linear_type]} GEMV (+RMSNorm, SwiGLU)",
                         "achieved": achieved, "peak": peak, "peak_kind": peak_kind,
                         "unit": "GB/s", "frac": achieved / peak, "traffic": traffic,
                         "algorithmic_bytes_per_launch": algo_bytes,
                         "us_per_launch": kern_us},
            "cpu_baseline": cpu,
            "e2e": {"value": world * args.steps / e2e_s, "unit": "tok/s",
                    "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 8},
            "gpu_launches": launches_per_tok * args.steps,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    smp.close()
    ctx.close()
    model.close()
    if dist is not None:
        dist.destroy_process_group()


def run_tp(args):
    """One sequence of config 4 (27B TQ2_0 by default) decoded over the ranks
    of a torchrun launch (strong scaling: the work per token is fixed, each
    rank holds 1/N of it). N > 1: the shards of rustfox_b200/tp.py with the
    sums exchange over peer memory by default (--exchange), the whole step
    captured as one CUDA graph per rank; time per token is the max over
    ranks of the CUDA-event time on each rank's context stream. N = 1: the
    single-GPU decode step of the same model (the fastest one-GPU path, the
    baseline the speed-up is read against). Greedy with upstream's repeat
    penalty (1.1 over 64), as `fox run --temp 0`."""
    import datetime
    import torch
    import rustfox_b200 as rf
    from rustfox_b200 import synth
    from rustfox_b200.tp import TPContext
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(minutes=5))
    cfg = synth.CONFIGS[args.config]
    # weights generated on the device: the 27B shape is 7.7 GB, minutes of
    # host-side generation while every GPU of the run is held
    model = rf.Model.from_synthetic_device(cfg, device=local, tp_rank=rank, tp_size=world)
    warm = max(3, args.warmup)
    n_ctx = args.prompt + 2 * (warm + args.steps) + 8
    prompt = synth.random_prompt(cfg, args.prompt, seed=1)
    clocks = Clocks(local)

    def max_over_ranks(x: float) -> float:
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()

    if world == 1:
        ctx = model.context(n_ctx, kv="f16")
        smp = rf.Sampler(ctx, temperature=0.0)
        ctx.eval(prompt, want_logits=False)
        for t in prompt:
            smp.accept(int(t))
        tok = smp.pick()
        smp.accept(tok)
        tok = int(smp.generate(tok, warm)[-1])
        barrier()
        clocks.start()
        toks = smp.generate(tok, args.steps)
        dev_s = ctx.last_eval_seconds
        tok = int(toks[-1])
        for _ in range(warm):
            tok = smp.decode(tok)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            tok = smp.decode(tok)
        e2e_s = time.perf_counter() - t0
        clk = clocks.stop()
        prof = {}
        for kind, us in ctx.profile_step(tok):
            prof[kind] = prof.get(kind, 0.0) + us
        phases = {"qkv+attention": prof.get("qkv", 0) + prof.get("attention", 0),
                  "o": prof.get("o", 0), "gate_up": prof.get("gate_up", 0),
                  "down": prof.get("down", 0), "head+pick": prof.get("head", 0)}
        d2h, exchange = 8, "none (one GPU: the single-GPU decode step)"
        launches = 1 + 5 * cfg.n_layer + 2 + 2
        smp.close()
        ctx.close()
    else:
        ctx = TPContext(model, n_ctx, kv="f16", exchange=args.exchange, repeat_penalty=1.1,
                        repeat_last_n=64)
        toks = ctx.generate(prompt, warm, graphs=True)  # captures the step graph
        barrier()
        clocks.start()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(ctx.stream)
        ctx.replay(args.steps)
        e1.record(ctx.stream)
        torch.cuda.synchronize()
        dev_s = e0.elapsed_time(e1) / 1e3
        # end to end: the token from pinned host memory, the captured step,
        # the pick (and position) read back, every step on every rank
        tok = int(ctx.decode(0 if toks is None else int(toks[-1])))
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            tok = ctx.decode(tok)
        e2e_s = time.perf_counter() - t0
        clk = clocks.stop()
        barrier()
        phases = ctx.profile_step()
        d2h = 12
        exchange = {
            "nccl": "torch.distributed NCCL per row-parallel GEMV (max-allreduce of the absmax, "
                    "all-gather of the block terms), bit-identical to one GPU",
            "p2p": "the library's exchanges over peer memory (CUDA IPC): per row-parallel GEMV "
                   "the block terms of every rank folded in upstream's order, bit-identical to "
                   "one GPU",
            "sums": "the library's exchanges over peer memory (CUDA IPC): per row-parallel GEMV "
                    "the absmax traded in its prologue and n_embd row sums pushed to every rank, "
                    "added in rank order by the next GEMV's prologue (within 1e-3 of one GPU)"}[
            args.exchange]
        launches = 1 + 5 * cfg.n_layer + 3 + 4
        ctx.close()
    dev_s = max_over_ranks(dev_s)
    e2e_s = max_over_ranks(e2e_s)
    if rank == 0:
        # the whole model's bytes per token (weights once, K/V at the mean
        # position of the timed steps), against every rank's HBM together
        wb = cfg.weight_bytes()
        pos = args.prompt + warm + args.steps // 2
        tok_bytes = (wb["layers"] + wb["output"] + wb["embd_row"] + wb["norms"]
                     + cfg.kv_bytes_per_token(pos))
        hbm, src = measured_hbm_gbs()
        achieved = tok_bytes * args.steps / dev_s / 1e9
        print(json.dumps({
            "metric": METRIC, "value": args.steps / dev_s, "unit": "tok/s", "n_gpus": world,
            "roofline": {"bound": "hbm", "kernel": "the whole decode step (weights and K/V read "
                                                   "once per token over all ranks)",
                         "achieved": achieved, "peak": hbm * world, "unit": "GB/s",
                         "frac": achieved / (hbm * world), "traffic": None,
                         "peak_kind": f"{src} {hbm:.0f} GB/s per GPU x {world}",
                         "bytes_per_token": tok_bytes},
            "steps": args.steps, "warmup": warm, "ms_per_step": 1e3 * dev_s / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "i8 x ternary -> i32, f32",
            "data": "synthetic (seeded random-init weights generated on the device, uniform "
                    "random prompt ids)",
            "config": {"workload": f"{cfg.name} {cfg.n_layer}L/{cfg.n_embd} "
                                   f"{TYPE_NAMES[cfg.linear_type]} linear + "
                                   f"{TYPE_NAMES[cfg.output_type]} head, batch-1 greedy decode "
                                   f"of one sequence over {world} GPU(s) after a "
                                   f"{args.prompt}-id prompt",
                       "prompt": args.prompt, "n_ctx": n_ctx, "kv_cache": "f16",
                       "sampler": "greedy, repeat penalty 1.1 over 64",
                       "parallelism": f"tp{world}", "exchange": exchange,
                       "l2": f"weights {(wb['layers'] + wb['output']) / 1e9:.2f} GB per token "
                             f"({(wb['layers'] + wb['output']) / 1e9 / world:.2f} GB per rank) "
                             "> 126 MB L2: streamed from HBM, no flush",
                       "why_not_config_2": "a torchrun launch times config 4 (27B TQ2_0) split "
                                           "over the ranks, north_star's multi-GPU deliverable "
                                           "(strong scaling); a plain `python bench.py` times "
                                           "config 2 (4B TQ1_0) on one GPU"},
            "phases_us_per_token": {k: round(v, 1) for k, v in phases.items()},
            "limiting_phase": max(phases, key=phases.get) if phases else None,
            "e2e": {"value": args.steps / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 4,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": launches * args.steps,
            "clocks": clk}), flush=True)
    barrier()  # no rank unmaps a peer arena another may still read
    model.close()
    if dist is not None:
        dist.destroy_process_group()


def run_gemm(args):
    """The M-token tensor-core pass (tcgen05 kind::i8) over the seven matrices
    of one layer of the config (q, k, v, o, gate, up, down), against M
    single-token decode GEMVs (foxcuda_gemv_packed) of the same matrices:
    foxcuda_gemm_tq2_i8_packed for ternary configs (TQ1_0 is held as TQ2_0),
    foxcuda_gemm_kq_i8_packed for K-quant ones (Q4_K, with the config's v
    type). Enough packed copies of the layer are cycled that the weights read
    per timed region exceed the L2 three times over. CUDA-event time on the
    current stream, one GPU."""
    import torch
    import rustfox_b200 as rf
    from rustfox_b200 import formats as F, synth
    cfg = synth.CONFIGS[args.config]
    torch.cuda.set_device(0)
    e, f = cfg.n_embd, cfg.n_ff
    nq, nkv = cfg.n_head * cfg.head_dim, cfg.n_head_kv * cfg.head_dim
    shapes = [(nq, e), (nkv, e), (nkv, e), (e, nq), (f, e), (f, e), (e, f)]
    kq = cfg.linear_type in (F.Q4_K, F.Q6_K)
    lin = cfg.linear_type if kq else F.TQ2_0
    types = [lin, lin, (cfg.attn_v_type or cfg.linear_type) if kq else lin, lin, lin, lin, lin]
    layer_bytes = sum(F.row_bytes(t, k) * r for t, (r, k) in zip(types, shapes))
    params = sum(r * k for r, k in shapes)
    rng = np.random.default_rng(0)
    one = [rf.pack(t, torch.from_numpy(F.random_blocks(rng, t, r, k, 0.01)).cuda(), r, k)
           for t, (r, k) in zip(types, shapes)]
    copies = [one] + [[p.clone() for p in one]
                      for _ in range(max(1, int(np.ceil(3 * 126e6 / layer_bytes))) - 1)]
    kmax = max(k for _, k in shapes)
    rows = []
    for m in [int(v) for v in args.gemm.split(",")]:
        ks = {k for _, k in shapes}
        qs = {k: torch.randint(-127, 128, (m, k), dtype=torch.int8, device="cuda") for k in ks}
        s = torch.full((m,), 1e-3, dtype=torch.float32, device="cuda")
        sk = {k: torch.full((m, k // 256), 1e-3, dtype=torch.float32, device="cuda") for k in ks}
        x = torch.randn(kmax, dtype=torch.float32, device="cuda")
        outs = [torch.empty(m, r, dtype=torch.float32, device="cuda") for r, _ in shapes]

        def tc_pass(layer):
            for t, (r, k), pk, o in zip(types, shapes, layer, outs):
                if kq:
                    rf.gemm_kq_i8_packed(t, qs[k], sk[k], pk, r, k, out=o)
                else:
                    rf.gemm_tq2_i8_packed(qs[k], s, pk, r, k, out=o)

        def gemv_pass(layer):
            for _ in range(m):
                for t, (r, k), pk, o in zip(types, shapes, layer, outs):
                    rf.gemv_packed(t, x[:k], pk, r, k, out=o[0])

        split = args.split and not kq
        terms = (torch.empty(m * max(r * (k // 256) for r, k in shapes), dtype=torch.float32,
                             device="cuda") if split else None)

        def split_pass(layer):
            for (r, k), pk, o in zip(shapes, layer, outs):
                rf.gemm_tq2_i8_split(qs[k], s, pk, r, k, terms=terms, out=o)

        res = {"M": m}
        kinds = [("tc", tc_pass), ("gemv", gemv_pass)] + ([("split", split_pass)] if split else [])
        for name, fn in kinds:
            for i in range(max(3, args.warmup)):
                fn(copies[i % len(copies)])
            n = max(len(copies), args.steps)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record()
            for i in range(n):
                fn(copies[i % len(copies)])
            e1.record()
            torch.cuda.synchronize()
            res[f"{name}_us_per_layer"] = 1e3 * e0.elapsed_time(e1) / n
        t = res["tc_us_per_layer"] * 1e-6
        res["tc_weight_gbs"] = layer_bytes / t / 1e9
        res["tc_int8_tops"] = 2.0 * m * params / t / 1e12
        res["speedup_vs_gemv"] = res["gemv_us_per_layer"] / res["tc_us_per_layer"]
        rows.append(res)
    hbm, src = measured_hbm_gbs()
    names = "/".join(sorted({TYPE_NAMES[t] for t in types}))
    print(json.dumps({
        "metric": "M-token pass, one layer (q k v o gate up down)", "unit": "us",
        "higher_is_better": False, "dtype": "i8 x quantised weights -> i32 (tcgen05 kind::i8), f32 terms",
        "data": f"synthetic (seeded random {names} weights, random int8 activations)",
        "config": {"workload": f"{cfg.name} layer matrices, {names} packed",
                   "layer_weight_bytes": layer_bytes, "l2": f"{len(copies)} layer copies cycled",
                   "hbm_peak_gbs": hbm, "hbm_peak_source": src},
        "results": rows}), flush=True)


def reference_prompt(model, cfg, n_prompt: int):
    """Upstream fox_eval of one prompt on this host's cores (oracle/_ref, the
    upstream sources with their default -O3 and AVX2/FMA code generation,
    n_batch 32 as `fox run` uses it). Returns (prompt tok/s, cores)."""
    from oracle import oracle as O
    from rustfox_b200 import synth
    prompt = synth.random_prompt(cfg, n_prompt, seed=1)
    with tempfile.TemporaryDirectory() as d:
        path = synth.write_gguf(model, os.path.join(d, "model.gguf"), tokenizer=False)
        ref = O.RefLib(fast=True)
        cores = int(ref.L.fox_cpu_count_online())
        m = ref.open_model(path)
        ctx = ref.context(m, n_prompt + 8, 32, 0)
        ref.eval(ctx, prompt, cfg.n_vocab)
        secs = ref.L.fox_context_last_eval_seconds(ctx)
        ref.L.fox_context_destroy(ctx)
        ref.L.fox_model_close(m)
    return n_prompt / secs, cores


def run_prefill(args):
    """Prompt evaluation: foxcuda_eval of an --prompt long prompt with the
    chunk mode (tensor-core passes) and token by token (decode steps), CUDA
    event time of the eval (median of up to 5 runs, after warm-up), next to
    upstream's CPU fox_eval of a bounded prompt (32 ids, one n_batch chunk)."""
    import torch
    import rustfox_b200 as rf
    from oracle import oracle as O
    from rustfox_b200 import synth
    cfg = synth.CONFIGS[args.config]
    torch.cuda.set_device(0)
    host = synth.generate(cfg)
    model = rf.Model.from_synthetic(host)
    prompt = synth.random_prompt(cfg, args.prompt, seed=1)
    res = {}
    for name, chunks in (("chunks", True), ("steps", False)):
        ctx = rf.Context(model, args.prompt + 8, kv="f16")
        ctx.set_prefill(chunks)
        times = []
        for i in range(max(1, args.warmup) + min(max(1, args.steps), 5)):
            ctx.reset()
            ctx.eval(prompt, want_logits=False)
            if i >= max(1, args.warmup):
                times.append(ctx.last_eval_seconds)
        ctx.close()
        res[f"{name}_tok_s"] = args.prompt / statistics.median(times)
    res["chunks_vs_steps"] = res["chunks_tok_s"] / res["steps_tok_s"]
    model.close()
    cpu = None
    if not args.no_cpu_baseline and os.path.exists(O.REF_FAST_SO):
        n_ref = min(args.prompt, 32)
        v, cores = reference_prompt(host, cfg, n_ref)
        cpu = {"value": v, "unit": "tok/s", "cores": cores, "kind": "reference",
               "sample": f"upstream fox_eval of a {n_ref}-id prompt (n_batch 32)"}
    print(json.dumps({
        "metric": "prompt tok/s (fox_eval of one prompt)", "unit": "tok/s", "higher_is_better": True,
        "dtype": "i8 x ternary -> i32 (tcgen05 kind::i8 in chunks), f32",
        "data": "synthetic (seeded random-init weights, uniform random prompt ids)",
        "config": {"workload": f"{cfg.name} {cfg.n_layer}L/{cfg.n_embd}, a {args.prompt}-id prompt",
                   "kv_cache": "f16", "chunk": 64},
        "results": res, "cpu_baseline": cpu}), flush=True)


def run_batch(args):
    """Config 5: --batch sequences of the --config model decoded together
    (foxcuda_batch_generate: one pass per step, one CUDA graph per step) at a
    --ctx long context. The K/V of every sequence is seeded N(0, 1) fp16
    (foxcuda_context_fill_kv), a stand-in for the long prompts; sampling is
    top-k 40 at temperature 0.8, top-p and repeat penalty off, seed 1 + i.
    The caches are pages of one shared pool (foxcuda_kv_pool_create), as a
    server holds them; --contiguous gives each sequence its own cache.
    CUDA-event time of the timed steps on the batch's stream."""
    import torch
    import rustfox_b200 as rf
    from rustfox_b200 import synth
    cfg = synth.CONFIGS[args.config]
    torch.cuda.set_device(0)
    wb = cfg.weight_bytes()
    model = rf.Model.from_synthetic_device(cfg)  # no CPU baseline here: no host copy needed
    n, warm = args.batch, max(3, args.warmup)
    n_ctx = args.ctx + warm + args.steps + 8
    pages = (n_ctx + rf.api.KV_PAGE - 1) // rf.api.KV_PAGE
    pool = None if args.contiguous else model.kv_pool(n * pages)
    ctxs = [rf.Context(model, n_ctx, kv="f16", pool=pool) for _ in range(n)]
    for i, c in enumerate(ctxs):
        c.fill_kv(args.ctx, seed=1 + i)
    smp = [rf.Sampler(c, temperature=0.8, top_k=40, top_p=1.0, repeat_penalty=1.0, seed=1 + i)
           for i, c in enumerate(ctxs)]
    batch = rf.Batch(ctxs)
    batch.generate(smp, warm, first=synth.random_prompt(cfg, n, seed=2))
    clocks = Clocks(0)
    clocks.start()
    batch.generate(smp, args.steps)
    secs = batch.last_seconds
    ck = clocks.stop()
    # the attention launches on their own: one profiled step (events after
    # each phase on the batch's stream), its position at the end of the run
    prof = batch.profile_step(synth.random_prompt(cfg, n, seed=3))
    phase_us = {}
    for kind, us in prof:
        phase_us[kind] = phase_us.get(kind, 0.0) + us
    attn_us = phase_us.get("attention", 0.0) / cfg.n_layer
    p_prof = args.ctx + warm + args.steps + 1  # positions each sequence reads in that step
    # algorithmic bytes of a step: the layer and head GGUF bytes once, the
    # K/V every sequence reads (mean position of the timed steps) and writes
    pos = args.ctx + warm + args.steps / 2.0
    kv_row = cfg.n_head_kv * cfg.head_dim * 2
    step_bytes = (wb["layers"] + wb["output"] + 2 * cfg.n_layer * pos * kv_row * n
                  + 2 * cfg.n_layer * kv_row * n)
    achieved = step_bytes / (secs / args.steps) / 1e9
    attn_bytes = 2 * p_prof * kv_row * n  # one layer's K and V of every sequence
    attn_gbs = attn_bytes / (attn_us * 1e-6) / 1e9 if attn_us > 0 else None
    hbm, src = measured_hbm_gbs()
    print(json.dumps({
        "metric": f"batch-{n} decode tok/s at {args.ctx} context", "value": n * args.steps / secs,
        "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": warm,
        "ms_per_step": 1e3 * secs / args.steps, "higher_is_better": True, "scaling": None,
        "vs_baseline": None, "dtype": "i8 x ternary -> i32 (tcgen05 kind::i8), f32",
        "data": "synthetic (seeded random-init weights generated on the device; seeded N(0,1) fp16 "
                "K/V in place of prompts)",
        "config": {"workload": f"{cfg.name} {cfg.n_layer}L/{cfg.n_embd}, {n} sequences at position "
                               f"{args.ctx}, top-k 40 T 0.8", "batch": n, "ctx": args.ctx,
                   "kv_cache": "f16, " + ("one contiguous cache per sequence" if pool is None else
                                          f"paged: {rf.api.KV_PAGE}-position pages of one shared pool"),
                   "l2": f"{step_bytes / 1e9:.1f} GB per step > 126 MB L2"},
        "roofline": {"bound": "hbm", "kernel": "attention_tile_kernel (one launch per layer, all sequences)",
                     "achieved": attn_gbs, "peak": hbm, "unit": "GB/s",
                     "frac": attn_gbs / hbm if attn_gbs else None, "traffic": None, "peak_source": src,
                     "algorithmic_bytes_per_launch": attn_bytes, "us_per_launch": attn_us},
        "step_roofline": {"achieved": achieved, "frac": achieved / hbm, "bytes_per_step": step_bytes},
        "phases_us_per_step": {k: round(v, 1) for k, v in phase_us.items()},
        "cpu_baseline": None,
        "cpu_baseline_note": "upstream has no way to set its cache (or to decode several sequences "
                             "in one pass), so a 32k-position upstream decode would need the 32k-token "
                             "prompt evaluated on the CPU first; not timed",
        "clocks": ck}), flush=True)
    batch.close()
    for s in smp:
        s.close()
    for c in ctxs:
        c.close()
    if pool is not None:
        pool.close()
    model.close()


def run_image(args):
    """Model load, two ways, wall time of the (synchronous) model calls:
    every tensor uploaded from host memory and packed on the device
    (foxcuda_model_upload + finalize), and a device image of the same model
    opened from a file (foxcuda_model_open_image; median of up to 3 opens,
    the file in the page cache after it was written). Both models then
    decode the same tokens."""
    import shutil
    import torch
    import rustfox_b200 as rf
    from rustfox_b200 import synth
    cfg = synth.CONFIGS[args.config]
    torch.cuda.set_device(0)
    host = synth.generate(cfg)
    t0 = time.perf_counter()
    a = rf.Model.from_synthetic(host)
    upload_s = time.perf_counter() - t0
    d = tempfile.mkdtemp(prefix="foximg")
    try:
        path = os.path.join(d, "model.fdi")
        t0 = time.perf_counter()
        a.save_image(path)
        save_s = time.perf_counter() - t0
        size = os.path.getsize(path)
        opens = []
        b = None
        for _ in range(max(1, min(args.steps, 3))):
            if b is not None:
                b.close()
            t0 = time.perf_counter()
            b = rf.Model.open_image(path)
            opens.append(time.perf_counter() - t0)
        prompt = synth.random_prompt(cfg, 16, seed=1)
        same = bool(np.array_equal(rf.greedy_generate(a, prompt, 8, 64, repeat_penalty=1.0),
                                   rf.greedy_generate(b, prompt, 8, 64, repeat_penalty=1.0)))
        b.close()
    finally:
        shutil.rmtree(d, ignore_errors=True)
    a.close()
    open_s = statistics.median(opens)
    print(json.dumps({
        "metric": "model load seconds", "value": open_s, "unit": "s", "higher_is_better": False,
        "dtype": "bytes", "data": "synthetic (seeded random-init weights)",
        "config": {"workload": f"{cfg.name} {cfg.n_layer}L/{cfg.n_embd}: upload + pack vs device image"},
        "results": {"upload_and_pack_s": upload_s, "image_open_s": open_s, "image_save_s": save_s,
                    "image_bytes": size, "image_open_gbs": size / open_s / 1e9,
                    "speedup": upload_s / open_s, "tokens_identical": same},
        "cpu_baseline": None,
        "note": "upstream loads through its own GGUF/foxpack reader on the host; no device "
                "counterpart to time"}), flush=True)


def run_attention(args):
    """The tile attention on its own through the C ABI (foxcuda_attention):
    one sequence, fp16 K/V caches of N(0, 1) values, 32 query heads, head_dim
    128, at (positions, KV heads) = (32768, 8), (576, 8) and (576, 16). Each
    call cycles to another copy of the caches (together larger than L2).
    CUDA-event time per call includes the call's own position copy and stream
    synchronisation; the kernel alone is the ncu launch list of this command."""
    import ctypes as C
    import torch
    import rustfox_b200 as rf
    torch.cuda.set_device(0)
    L = rf.lib()
    p = C.c_void_p
    gen = torch.Generator(device="cuda").manual_seed(1)
    hbm, src = measured_hbm_gbs()
    res = []
    for n_ctx, pos, nkv in [(32768, 32767, 8), (4096, 575, 8), (4096, 575, 16)]:
        nh, hd = 32, 128
        copies = 4 if n_ctx > 8192 else 16
        ks = [torch.randn(nkv, n_ctx, hd, device="cuda", generator=gen).half() for _ in range(copies)]
        vs = [torch.randn(nkv, n_ctx, hd, device="cuda", generator=gen).half() for _ in range(copies)]
        q = torch.randn(nh * hd, device="cuda", generator=gen)
        out = torch.empty(nh * hd, device="cuda")
        stream = torch.cuda.current_stream().cuda_stream

        def call(i):
            st = L.foxcuda_attention(p(q.data_ptr()), p(ks[i % copies].data_ptr()), p(vs[i % copies].data_ptr()),
                                     0, nh, nkv, hd, n_ctx, pos, 0, p(out.data_ptr()), p(stream))
            if st != 0:
                raise rf.FoxError(st, rf.api.last_error())
        for i in range(max(3, args.warmup)):
            call(i)
        torch.cuda.synchronize()
        ts = []
        for i in range(args.steps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            call(i)
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b) * 1e3)
        us = statistics.median(ts)
        kv_bytes = 2 * nkv * (pos + 1) * hd * 2
        res.append({"positions": pos + 1, "kv_heads": nkv, "us_per_call": us, "kv_bytes": kv_bytes,
                    "gbs_per_call": kv_bytes / us / 1e3})
        del ks, vs
        torch.cuda.empty_cache()
    print(json.dumps({
        "metric": "tile attention per call", "unit": "us", "higher_is_better": False, "steps": args.steps,
        "dtype": "f16 K/V, f32 arithmetic", "data": "synthetic (seeded N(0,1) caches and queries)",
        "config": {"workload": "foxcuda_attention, one sequence, 32 query heads, head_dim 128",
                   "l2": "caches cycled over copies larger than L2 together"},
        "hbm_peak_gbs": hbm, "hbm_peak_source": src,
        "note": "per-call event time includes the call's position copy and synchronisation; "
                "kernel durations: ncu --metrics gpu__time_duration.sum on this command",
        "results": res}), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.attention:
        run_attention(args)
    elif args.image:
        run_image(args)
    elif args.gemm:
        run_gemm(args)
    elif args.prefill:
        run_prefill(args)
    elif args.batch:
        run_batch(args)
    elif args.tp or under_torchrun():
        run_tp(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
