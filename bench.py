"""Benchmark: decode tok/s of the Llama-3-8B-shaped Q4_K_M model at batch 1
on one B200, as a fraction of the HBM roofline; prefill tok/s alongside.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One "step" is one batch-1 greedy decode step (all 32 layers + logits +
argmax) over a context that starts after a 1024-token prompt prefill. The
weights (4.6 GB of quantised bytes per step) are far larger than L2, so no
flush is needed between steps. `value` is device-timed with CUDA events over
K persistent-kernel launches whose inputs are already in HBM; `e2e` is the
same metric through the C ABI's ifx_decode_step with host buffers (token H2D,
logits D2H every step). With --gpus N > 1 (under torchrun) each rank decodes
an independent sequence (replicas, weak scaling, value = N / the slowest
rank's step time) and a tensor-parallel leg decodes one sequence over all N
GPUs (`tensor_parallel` in the line); --tp makes tensor parallelism the
headline instead (strong scaling). `batched_decode` times 16 sequences per
GPU decoded together.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s @8B Q4_K_M batch 1 as % of HBM roofline; prefill tok/s"
# The workloads of BASELINE's configs 2-4 (--config): model shape, prompt
# length, the smallest KV capacity the config names, and the batch of the
# batched-decode leg (0: none). The default, 8b, is the headline metric's.
WORKLOADS = {
    "8b": dict(name="llama3-8b-shaped Q4_K_M", prompt=1024, min_ctx=0, batch=16),
    "70b": dict(name="llama2-70b-shaped Q4_K_M", prompt=2048, min_ctx=4096, batch=32),
    "1b": dict(name="llama3.2-1b-shaped Q4_K_M (tied embedding)", prompt=512, min_ctx=2048, batch=0),
}
# a faithful single-thread CPU step of these shapes takes minutes: their CPU
# figures come from 1- and 2-layer cuts of the same width (see cpu_step_time)
CPU_CUT = {"70b"}
# DRAM bytes (read + write) per algorithmic byte of decode_mega_kernel, from
# an ncu capture of the 4-layer 8B-shaped case (974.5 MB + 11.8 MB over
# 973.3 MB); traffic scales with the weight bytes.
TRAFFIC_PER_ALGO_BYTE = 1.013


def bf16_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return float(json.load(open(p))["bf16_tflops"])
    return 1590.0


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Clocks:
    """nvidia-smi sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = []
        try:
            for line in open(self.path):
                f = [x.strip() for x in line.split(",")]
                if len(f) >= 9 and f[1].isdigit():
                    rows.append(f)
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        mhz = [int(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": int(rows[0][2]), "reasons": reasons,
                "samples": len(rows)}


def prompt_ids(vocab: int, n: int, seq_index: int = 0, seed: int = 42):
    """Seeded uniform prompt ids in [3, vocab): the benchmark's prompts (the
    same rule as inferox_b200.synth.prompt_ids, restated here so the reference
    arm needs nothing from the product package)."""
    import numpy as np
    return np.random.default_rng(seed + seq_index).integers(3, vocab, size=n, dtype=np.uint32)


def shape_overrides(args) -> dict:
    """Profiling / testing cuts of the configured shape (--layers, --vocab)."""
    o = {}
    if args.layers:
        o["n_layers"] = args.layers
    if args.vocab:
        o["vocab"] = args.vocab
    return o


def bench_config(args) -> dict:
    """The workload both arms run (identical dicts, so the driver can compare
    them): decode contexts start after the prompt and the warm-up steps."""
    wl = WORKLOADS[args.config]
    ctx0 = wl["prompt"] + args.warmup
    return {"workload": f"{wl['name']}: {wl['prompt']}-token prompt prefill, then batch-1 greedy decode"
                        + (f" (profiling case: {args.layers} layers)" if args.layers else "")
                        + (f" (test case: vocabulary {args.vocab})" if args.vocab else ""),
            "batch": 1, "prompt_tokens": wl["prompt"], "decode_context": [ctx0, ctx0 + args.steps],
            "l2": "no flush needed: the weights of one step are far larger than the 126 MB L2"}


def cpu_step_time(make_gguf, n_layers: int, prompt: int, warmup: int, steps: int, threads: int):
    """Seconds per faithful decode step of the oracle port (per-call
    whole-tensor dequant + AVX2-order matmul_t, as the reference runs) at the
    benchmark's context: the cache is first filled by an untimed prefill of
    the same prompt (per-row dequant fused into the dots: the same bits, far
    faster) and `warmup` faithful steps. make_gguf(n_layers) builds the model;
    with n_layers = 0 the full model is timed, otherwise 1- and 2-layer cuts of
    the same width, and the step time is extrapolated linearly to n_layers
    (every layer costs the same; the embedding and output projection are the
    fixed part)."""
    from oracle import refcpu as R

    cores = len(os.sched_getaffinity(0))

    def one(gguf):
        m = R.Model(gguf)
        kv = m.kv_cache(int(m.config.n_layers), prompt + warmup + steps + 8)
        R.set_threads(cores)
        R.set_faithful(False)
        tok = R.argmax(m.prefill(prompt_ids(m.vocab, prompt), kv, True)[0])
        R.set_threads(threads)
        R.set_faithful(True)
        for _ in range(warmup):
            tok = R.argmax(m.decode_step(tok, kv))
        t0 = time.perf_counter()
        for _ in range(steps):
            tok = R.argmax(m.decode_step(tok, kv))
        dt = (time.perf_counter() - t0) / steps
        R.set_faithful(False)
        R.set_threads(cores)
        return dt

    if not n_layers:
        return one(make_gguf(0)), "the full model"
    t1, t2 = one(make_gguf(1)), one(make_gguf(2))
    return t1 + (n_layers - 1) * (t2 - t1), f"1- and 2-layer cuts extrapolated to {n_layers} layers"


def cpu_baseline(args, make_gguf, n_layers: int):
    """The reference's CPU path, single thread as the reference runs, on a
    bounded sample of the workload: one faithful decode step at the
    benchmark's context (the full model, or layer cuts for shapes whose full
    step takes minutes)."""
    wl = WORKLOADS[args.config]
    cut = n_layers if args.config in CPU_CUT and not args.layers else 0
    dt, what = cpu_step_time(make_gguf, cut, wl["prompt"], 0, 1, 1)
    return {"value": 1.0 / dt, "unit": "tok/s", "cores": 1, "kind": "port",
            "sample": f"1 faithful decode step of the {wl['name']} model at context {wl['prompt']} "
                      f"({what}; per-call whole-tensor dequant + AVX2 matmul_t, as the reference does), "
                      "1 host thread, as the reference runs"}


def run_reference(args):
    """The reference's CPU implementation of the decode step (the oracle port:
    src/model/forward.rs:543-586 with per-call whole-tensor dequantisation,
    src/gguf/weights.rs:66-74, and the AVX2-order matmul_t, src/ops.rs:106-149)
    on the same model, prompt and decode contexts as the GPU arm. It loads only
    the oracle library: the model comes from the oracle's own generator. The
    dequantisation and the matmuls run on every host thread (bit-identical to
    one thread); the reference itself is single-threaded, so this is an upper
    bound on its speed. Under torchrun only rank 0 runs."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import refcpu as R

    cores = len(os.sched_getaffinity(0))
    R.set_threads(cores)
    wl = WORKLOADS[args.config]
    full_layers = int(R.BENCH_CONFIGS[args.config]["n_layers"])
    cut = full_layers if args.config in CPU_CUT and not args.layers else 0
    t0 = time.time()

    def make(n):
        o = shape_overrides(args)
        if n:
            o["n_layers"] = n
        return R.synth_gguf(args.config, threads=cores, **o)

    dt, what = cpu_step_time(make, cut, wl["prompt"], args.warmup, args.steps, cores)
    setup_s = time.time() - t0
    ctx0 = wl["prompt"] + args.warmup
    value = 1.0 / dt
    sample = (f"{args.steps} decode steps (after {args.warmup} warm-up steps) of the {wl['name']} model "
              f"at context {ctx0}-{ctx0 + args.steps} ({what}), faithful mode (per-call whole-tensor "
              f"dequant + AVX2-order matmul_t), {cores} host threads")
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * dt,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,0.02) weights quantised Q4_K_M; seeded uniform prompt ids)",
            "impl": "reference", "config": bench_config(args),
            "placement": f"host CPU, {cores} threads (oracle port of the reference's CPU path)",
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "setup_s": setup_s}
    print(json.dumps(line), flush=True)


def run_70b_leg(args, dist, rank, world, local, hbm):
    """The 70B-shaped workload (2048-token prompt, then greedy decode) on all
    `world` GPUs: tensor parallel with one rank per GPU, or one GPU alone.
    Device-timed like the main line (max over ranks). A failure on any rank is
    reported in the result, never fatal: each rank catches its own error and
    the ranks agree through one all-reduce."""
    import numpy as np
    import torch
    from inferox_b200 import Model, synth, tp

    wl = WORKLOADS["70b"]
    steps, warm = min(args.steps, 32), 3
    err, ms, pf_s, kernels, wbytes = "", 0.0, 0.0, 0, 0
    m = kv = tcomm = None
    gpath = None
    t0 = time.time()
    try:
        if world > 1:
            gpath = os.path.join("/dev/shm" if os.path.isdir("/dev/shm") else tempfile.gettempdir(),
                                 f"ifx_bench_70b_scale_{os.getppid()}.gguf")
            if rank == 0:
                synth.build("70b").tofile(gpath + ".part")
                os.replace(gpath + ".part", gpath)
    except Exception as e:  # noqa: BLE001
        err = repr(e)[:300]
    if dist:
        dist.barrier()
    t_gen = time.time() - t0
    try:
        if not err:
            if world > 1:
                uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
                if rank == 0:
                    uid.copy_(torch.frombuffer(bytearray(tp.unique_id()), dtype=torch.uint8))
                dist.broadcast(uid, 0)
                tcomm = tp.Comm(bytes(uid.cpu().numpy()), world, rank, local)
                m = Model.open(gpath, device=local, tp_size=world, tp_rank=rank,
                               nccl_comm=tcomm.handle, tp_timeout_ms=120000)
            else:
                m = Model.from_bytes(synth.build("70b"), device=local)
            V = int(m.config.vocab_size)
            kv = m.kv_cache(wl["min_ctx"])
            prompt = synth.prompt_ids(V, wl["prompt"], seq_index=0)
            m.prefill(prompt[:64], kv, last_row_only=True)  # first-call costs out of the timing
            kv.clear()
            torch.cuda.synchronize()
            tpf = time.perf_counter()
            f0 = int(np.argmax(m.prefill(prompt, kv, last_row_only=True)[0]))
            pf_s = time.perf_counter() - tpf
            m.decode_greedy(f0, warm, kv)
            kernels = kv.decode_kernels()
            wbytes = m.decode_weight_bytes()
    except Exception as e:  # noqa: BLE001
        err = repr(e)[:300]

    def all_ok(e: str) -> bool:
        if not dist:
            return not e
        f = torch.tensor([0.0 if e else 1.0], device="cuda")
        dist.all_reduce(f, op=dist.ReduceOp.MIN)
        return f.item() > 0

    ctx0 = 0
    if all_ok(err):
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        try:
            ctx0 = len(kv)
            _, t = m.decode_greedy(f0, steps, kv, timed=True)
            ms = t / steps
        except Exception as e:  # noqa: BLE001
            err = repr(e)[:300]
    elif not err:
        err = "failed on another rank"
    ok = torch.tensor([0.0 if err else 1.0, ms, pf_s], device="cuda")
    if dist:
        okmin = ok.clone()
        dist.all_reduce(okmin, op=dist.ReduceOp.MIN)
        dist.all_reduce(ok, op=dist.ReduceOp.MAX)
        good = okmin[0].item() > 0
    else:
        good = not err
    del kv, m  # before the communicator
    if tcomm is not None:
        tcomm.close()
    if gpath and rank == 0 and os.path.exists(gpath):
        os.remove(gpath)
    if not good:
        return {"n_gpus": world, "error": err or "failed on another rank"}
    ms, pf_s = float(ok[1].item()), float(ok[2].item())
    c = synth.CONFIGS["70b"]
    kvh = c["n_kv_heads"] // world
    hd = c["dim"] // c["n_heads"]
    kv_bytes = 2 * c["n_layers"] * kvh * hd * 2 * (ctx0 + steps / 2)
    per_gpu = wbytes + kv_bytes
    gbs = per_gpu / (ms * 1e-3) / 1e9
    return {"workload": f"{wl['name']}: {wl['prompt']}-token prompt prefill, then batch-1 greedy decode",
            "n_gpus": world, "tok_s": 1000.0 / ms, "tok_s_per_gpu": 1000.0 / ms / world,
            "ms_per_step": ms, "steps": steps, "warmup": warm, "decode_context": [ctx0, ctx0 + steps],
            "scaling": "strong",
            "parallelism": ("single GPU" if world == 1 else f"tp{world}: " + (
                "persistent kernel, all-reduces over NVLink peer memory inside the step"
                if kernels == 1 else "per-op kernels, NCCL all-reduce after Wo and W2")),
            "hbm_roofline": {"bytes_per_step_per_gpu": per_gpu, "achieved_gbs_per_gpu": gbs,
                             "peak_gbs": hbm, "frac": gbs / hbm,
                             "roofline_tok_s": hbm * 1e9 / per_gpu},
            "prefill": {"tokens": wl["prompt"], "s": pf_s, "tok_s": wl["prompt"] / pf_s},
            "gpu_launches": steps * kernels, "setup_s": {"synth": t_gen}}


def run_ours(args):
    import numpy as np
    import torch

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        from datetime import timedelta

        import torch.distributed as dist_

        dist_.init_process_group("nccl", timeout=timedelta(seconds=600),
                                 device_id=torch.device("cuda", local))
        dist = dist_

    from inferox_b200 import Model, synth, tp

    # several GPUs: tensor parallelism over all of them (one sequence, the
    # weights split N ways) with --tp; by default one independent sequence per
    # GPU (replicas: weak scaling, no collective on the data path), with a
    # tensor-parallel leg measured afterwards
    tp_mode = world > 1 and args.tp
    comm = None
    t0 = time.time()
    wl = WORKLOADS[args.config]
    PROMPT = wl["prompt"]
    # one GPU: the model in host memory; several: rank 0 writes the GGUF once
    # to shared memory and every rank maps it (the library mmaps a path), so
    # N ranks do not each build the whole model
    gpath = None
    if world > 1:
        tag = "_".join(f"{k}{v}" for k, v in sorted(shape_overrides(args).items()))
        gpath = os.path.join("/dev/shm" if os.path.isdir("/dev/shm") else tempfile.gettempdir(),
                             f"ifx_bench_{args.config}{'_' + tag if tag else ''}_{os.getpid() if rank == 0 else 0}.gguf")
        name = torch.zeros(256, dtype=torch.uint8, device="cuda")
        if rank == 0:
            synth.build(args.config, **shape_overrides(args)).tofile(gpath)
            enc = gpath.encode()
            name[:len(enc)] = torch.frombuffer(bytearray(enc), dtype=torch.uint8)
        dist.broadcast(name, 0)
        gpath = bytes(name.cpu().numpy()).rstrip(b"\0").decode()
        g = None
    else:
        g = synth.build(args.config, **shape_overrides(args))

    def load(**kw):
        return Model.open(gpath, device=local, **kw) if gpath else Model.from_bytes(g, device=local, **kw)

    t_gen = time.time() - t0
    t0 = time.time()
    if tp_mode:
        uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
        if rank == 0:
            uid.copy_(torch.frombuffer(bytearray(tp.unique_id()), dtype=torch.uint8))
        dist.broadcast(uid, 0)
        comm = tp.Comm(bytes(uid.cpu().numpy()), world, rank, local)
        m = load(tp_size=world, tp_rank=rank, nccl_comm=comm.handle)
    else:
        m = load()
    t_load = time.time() - t0
    cfg = m.config
    L, G, hd, V = int(cfg.n_layers), int(cfg.n_kv_heads), int(cfg.head_dim), int(cfg.vocab_size)
    max_seq = max(wl["min_ctx"], PROMPT + 2 * (args.warmup + args.steps) + 16)
    kv = m.kv_cache(max_seq)
    prompt = synth.prompt_ids(V, PROMPT, seq_index=0 if tp_mode else rank)

    # prefill: one untimed pass, then a timed one (wall clock around a
    # synchronous call; the prefill is a single device-bound call)
    m.prefill(prompt, kv, last_row_only=True)
    kv.clear()
    torch.cuda.synchronize()
    t_pf = time.perf_counter()
    lg = m.prefill(prompt, kv, last_row_only=True)
    prefill_s = time.perf_counter() - t_pf
    first = int(np.argmax(lg[0]))

    # decode: W untimed steps, then K device-fed steps timed with CUDA events
    m.decode_greedy(first, args.warmup, kv)
    ctx0 = len(kv)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        toks, dev_ms = m.decode_greedy(first, args.steps, kv, timed=True)
    clocks = clk.summary()
    ms_step = dev_ms / args.steps
    if dist:
        t = torch.tensor([ms_step], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_step = float(t.item())
    seqs = 1 if tp_mode else world  # sequences decoded per step by the whole job
    value = seqs * 1000.0 / ms_step

    # end to end through the reference-facing call: ifx_decode_step with the
    # token from host memory and the logits copied back to host every step
    e2e_steps = max(8, min(args.steps, 64))
    m.decode_step(first, kv, want_logits=True)
    torch.cuda.synchronize()
    te = time.perf_counter()
    tok = first
    for _ in range(e2e_steps):
        lg = m.decode_step(tok, kv, want_logits=True)
        tok = int(lg.argmax())
    e2e_s = time.perf_counter() - te
    e2e = {"value": seqs * e2e_steps / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 4,
           "d2h_bytes_per_step": V * 4}

    # per-kernel figures of the per-op path (each fused kernel timed alone,
    # cycling through the layers so every launch streams from HBM)
    hbm, peak_kind = peaks()
    kernels_per_step = kv.decode_kernels()
    kern = {}
    for which in ("w13", "w2", "qkv", "wo", "logits", "attn"):
        ms, b = m.bench_kernel(kv, which, 2 * L if which != "logits" else 8)
        kern[which] = {"ms": ms, "bytes": b, "gbs": b / (ms * 1e-3) / 1e9}
    # batched decode (the config's batch-16 workload: independent seeded
    # prompts, each prefilled, then all 16 decoded together; one weight read
    # per step for the 16 tokens), single GPU only
    batch = None
    B = wl["batch"] if args.batch < 0 else args.batch
    if not tp_mode and B > 1:
        kb = m.kv_batch(B, PROMPT + args.batch_steps + 16)
        firsts = [int(np.argmax(kb.prefill(b, synth.prompt_ids(V, PROMPT, seq_index=b), True)[0]))
                  for b in range(B)]
        kb.decode_greedy(firsts, 3)
        torch.cuda.synchronize()
        _, bms = kb.decode_greedy(firsts, args.batch_steps, timed=True)
        if dist:
            t = torch.tensor([bms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            bms = float(t.item())
        batch = {"batch": B * world, "per_gpu_batch": B, "steps": args.batch_steps,
                 "ms_per_step": bms / args.batch_steps,
                 "tok_s": world * B * args.batch_steps / (bms * 1e-3),
                 "context": f"{PROMPT}-token prompts, {args.batch_steps} timed steps after 3"}
        del kb

    # tensor-parallel leg (several GPUs, replicas mode): one sequence over all
    # of them, Megatron split with NCCL all-reduces, device-timed like `value`.
    # A failure here (on any rank) must not cost the replicas' line: the
    # library's collectives are bounded (tp_timeout_ms: a stalled peer turns
    # into an error on every rank), each rank catches its own error, and the
    # ranks then agree through one all-reduce whether the leg succeeded.
    tpleg = None
    if world > 1 and not tp_mode and not args.no_tp_leg:
        uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
        if rank == 0:
            uid.copy_(torch.frombuffer(bytearray(tp.unique_id()), dtype=torch.uint8))
        dist.broadcast(uid, 0)
        tp_err, tp_ms, tp_prefill_s, tp_kernels = "", 0.0, 0.0, 0
        tcomm = mt = kvt = None

        def all_ok(err: str) -> bool:
            f = torch.tensor([0.0 if err else 1.0], device="cuda")
            dist.all_reduce(f, op=dist.ReduceOp.MIN)
            return f.item() > 0

        f0 = 0
        try:
            tcomm = tp.Comm(bytes(uid.cpu().numpy()), world, rank, local)
            mt = load(tp_size=world, tp_rank=rank, nccl_comm=tcomm.handle, tp_timeout_ms=120000)
            kvt = mt.kv_cache(max_seq)
            p0 = synth.prompt_ids(V, PROMPT, seq_index=0)
            tpf = time.perf_counter()
            f0 = int(np.argmax(mt.prefill(p0, kvt, last_row_only=True)[0]))
            tp_prefill_s = time.perf_counter() - tpf
            mt.decode_greedy(f0, args.warmup, kvt)
            tp_kernels = kvt.decode_kernels()
        except Exception as e:  # noqa: BLE001 (reported in the line, never fatal)
            tp_err = repr(e)[:300]
        if all_ok(tp_err):
            dist.barrier()
            torch.cuda.synchronize()
            try:
                _, tms = mt.decode_greedy(f0, args.steps, kvt, timed=True)
                tp_ms = tms / args.steps
            except Exception as e:  # noqa: BLE001
                tp_err = repr(e)[:300]
        elif not tp_err:
            tp_err = "failed on another rank"
        ok = torch.tensor([0.0 if tp_err else 1.0, tp_ms], device="cuda")
        okmin = ok.clone()
        dist.all_reduce(okmin, op=dist.ReduceOp.MIN)
        dist.all_reduce(ok, op=dist.ReduceOp.MAX)
        if okmin[0].item() > 0:
            t_ms = float(ok[1].item())
            tpleg = {"n_gpus": world, "tok_s": 1000.0 / t_ms, "ms_per_step": t_ms,
                     "prefill_tok_s": PROMPT / tp_prefill_s, "scaling": "strong",
                     "parallelism": f"tp{world}: " + (
                         "persistent kernel, all-reduces over NVLink peer memory inside the step"
                         if tp_kernels == 1 else "per-op kernels, NCCL all-reduce after Wo and W2")}
        else:
            tpleg = {"n_gpus": world, "error": tp_err or "failed on another rank"}
        del kvt, mt  # the cache's CUDA graph holds NCCL work: release it before the comm
        if tcomm is not None:
            tcomm.close()

    # the dequant-fused matmul microbench at the 8B W1 shape (every type and
    # batch; the full table is `--microbench`)
    micro = None
    if not args.no_microbench and rank == 0 and not tp_mode:
        micro = run_microbench([(14336, 4096)], reps=3) if args.config == "8b" else None

    # whole-step algorithmic bytes: every weight once + K/V at the mean context
    ctx_mean = ctx0 + args.steps / 2
    # per GPU: under tensor parallelism each rank reads its shard of the
    # weights (decode_weight_bytes is this rank's) and its kv heads
    kv_bytes = 2 * L * (G // world if tp_mode else G) * hd * 2 * ctx_mean
    step_bytes = m.decode_weight_bytes() + kv_bytes
    step_gbs = step_bytes / (ms_step * 1e-3) / 1e9
    tp_placement = (f"tp{world}: " + ("persistent kernel, all-reduces over NVLink peer memory inside the step"
                                      if kernels_per_step == 1 else "per-op kernels, NCCL all-reduce after Wo and W2"))

    # the 70B-shaped config at this GPU count: one
    # sequence, tensor parallel over all N GPUs (a single GPU at N = 1)
    scale70 = None
    if args.config == "8b" and not args.no_70b and not args.layers:
        del kv, m  # room for the 70B weights
        kv = m = None
        torch.cuda.synchronize()
        scale70 = run_70b_leg(args, dist, rank, world, local, hbm)

    def finish():
        nonlocal m, kv
        del kv, m  # the cache's CUDA graph holds NCCL work: release it first
        if comm:
            comm.close()
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        if gpath and rank == 0 and os.path.exists(gpath):
            os.remove(gpath)

    if rank != 0:
        finish()
        return
    base = None
    if world == 1 and not args.no_cpu_baseline:
        def make(n):
            if not n:
                return g
            return synth.build(args.config, **{**shape_overrides(args), "n_layers": n})
        base = cpu_baseline(args, make, L)
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong" if tp_mode else "weak", "vs_baseline": None,
        "dtype": "f16 tensor-core operands (exact small-integer weights; activations as hi + lo f16 planes, ~22 bits), f32 accumulate; f16 KV cache",
        "data": "synthetic (seeded N(0,0.02) weights quantised Q4_K_M; seeded uniform prompt ids)",
        "config": bench_config(args),
        "placement": (tp_placement if tp_mode
                      else f"replicas x{world}, one sequence per GPU" if world > 1 else "single GPU"),
        "global_batch": seqs,
        "hbm_roofline": {"bytes_per_step": step_bytes, "achieved_gbs": step_gbs, "peak_gbs": hbm,
                         "frac": step_gbs / hbm, "peak": peak_kind,
                         "roofline_tok_s": hbm * 1e9 / step_bytes},
        "prefill": {"tokens": PROMPT, "s": prefill_s, "tok_s": PROMPT / prefill_s},
        "batched_decode": batch,
        "matmul_microbench": micro,
        "tensor_parallel": tpleg,
        "scale_70b": scale70,
        # the dominant kernel is the decode step itself: with the persistent
        # path one launch per token, so achieved = algorithmic step bytes over
        # the device time of one step
        "roofline": {"bound": "hbm",
                     "kernel": "decode_mega_kernel" if kernels_per_step == 1 else "per-op step",
                     "achieved": step_gbs, "peak": hbm, "unit": "GB/s", "frac": step_gbs / hbm,
                     "traffic": TRAFFIC_PER_ALGO_BYTE * step_bytes if kernels_per_step == 1 else None,
                     "traffic_unit": "bytes per launch", "peak_kind": peak_kind},
        "kernels": kern,
        "e2e": e2e,
        "gpu_launches": args.steps * kernels_per_step,
        "clocks": clocks,
        "cpu_baseline": base,
        "setup_s": {"synth": t_gen, "load": t_load},
    }
    print(json.dumps(line), flush=True)
    finish()


MB_TYPES = {"Q4_0": (2, 4.5), "Q8_0": (7, 8.5), "Q4_K": (12, 4.5), "Q6_K": (14, 6.5625)}
MB_SHAPES = [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]
MB_BATCHES = [1, 8, 64, 512]


def _quantize_parallel(ttype: int, x, block: int):
    """Host quantisation of a large matrix in block-aligned chunks on every
    core (the library's quantiser releases the GIL through ctypes)."""
    from concurrent.futures import ThreadPoolExecutor

    import numpy as np
    from inferox_b200 import synth
    nblk = x.size // block
    cores = len(os.sched_getaffinity(0))
    parts = max(1, min(cores * 2, nblk // 4096))
    cuts = [x.size * i // parts // block * block for i in range(parts)] + [x.size]
    with ThreadPoolExecutor(max_workers=cores) as ex:
        out = list(ex.map(lambda i: synth.quantize(ttype, x[cuts[i]:cuts[i + 1]]), range(parts)))
    return np.frombuffer(b"".join(out), np.uint8)


def run_microbench(shapes, reps: int = 5):
    """the dequant-fused matmul (what replaces tensor_f32_by_index
    + matmul_t, src/gguf/dequant.rs:62-199 + src/ops.rs:33-44) for Q4_0, Q8_0,
    Q4_K and Q6_K weights drawn N(0, 0.02), activations N(0, 1), at batch 1,
    8, 64 and 512: ms per call (input staging included, weights from HBM),
    algorithmic GB/s (weights + activations + outputs) against the measured
    HBM peak and useful TFLOP/s against the measured bf16 peak."""
    import numpy as np
    import torch
    from inferox_b200 import ops
    hbm, _ = peaks()
    tflops_peak = bf16_peak()
    rng = np.random.default_rng(0)
    rows_out = []
    for rows, cols in shapes:
        w = (rng.standard_normal(rows * cols, dtype=np.float32) * np.float32(0.02))
        for tname, (ttype, bpw) in MB_TYPES.items():
            blk = 256 if ttype in (12, 14) else 32
            W = ops.QMatrix(ttype, _quantize_parallel(ttype, w, blk), rows, cols)
            for B in MB_BATCHES:
                x = torch.from_numpy(rng.standard_normal(B * cols, dtype=np.float32)).cuda()
                ms = ops.bench_matmul_t_q(x, W, B, reps)
                nbytes = rows * cols * bpw / 8 + 4 * B * (rows + cols)
                fl = 2.0 * B * rows * cols
                kernel = ("gemv_b1_kernel" if B == 1 else "gemm_kernel (small batch)" if B <= 32
                          else "tc_gemm_kernel (tcgen05)")
                rows_out.append({"type": tname, "shape": [rows, cols], "batch": B, "kernel": kernel,
                                 "ms": ms, "gbs": nbytes / (ms * 1e-3) / 1e9,
                                 "hbm_frac": nbytes / (ms * 1e-3) / 1e9 / hbm,
                                 "tflops": fl / (ms * 1e-3) / 1e12,
                                 "tensor_frac": fl / (ms * 1e-3) / 1e12 / tflops_peak})
            del W
        del w
    return rows_out


def run_gemm_case(spec: str):
    """Profiling case for one fused dequant matmul (prefill-sized m goes to the
    tcgen05 GEMM): four calls on a seeded matrix; prints the CUDA-event time."""
    import numpy as np
    import torch
    from inferox_b200 import ops, synth
    rows, cols, m, ttype = (int(v) for v in spec.split(","))
    rng = np.random.default_rng(0)
    w = (rng.standard_normal(rows * cols) * 0.02).astype(np.float32)
    W = ops.QMatrix(ttype, synth.quantize(ttype, w), rows, cols)
    x = torch.from_numpy(rng.standard_normal((m, cols)).astype(np.float32)).cuda()
    ops.matmul_t_q(x, W, m)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(3):
        ops.matmul_t_q(x, W, m)
    e1.record()
    torch.cuda.synchronize()
    print(json.dumps({"gemm": spec, "ms_per_call_incl_staging_and_alloc": e0.elapsed_time(e1) / 3}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--gemm", default="",
                    help="profiling only: ROWS,COLS,M,TYPE — four calls of the fused dequant "
                         "matmul (ifx_op_matmul_t_q) on a seeded matrix, then exit")
    ap.add_argument("--batch", type=int, default=-1,
                    help="also time batched decode of this many sequences (0/1: skip; default: "
                         "the config's, 16 for 8b and 32 for 70b)")
    ap.add_argument("--config", default="8b", choices=sorted(WORKLOADS),
                    help="the workload: 8b (the headline metric's, default), 70b or 1b")
    ap.add_argument("--batch-steps", type=int, default=32)
    ap.add_argument("--tp", action="store_true",
                    help="with several GPUs: decode one sequence with tensor parallelism over "
                         "all of them (strong scaling) instead of one sequence per GPU")
    ap.add_argument("--replicas", action="store_true",
                    help="one independent sequence per GPU (the default with several GPUs)")
    ap.add_argument("--no-tp-leg", action="store_true",
                    help="with several GPUs: skip the tensor-parallel leg")
    ap.add_argument("--microbench", action="store_true",
                    help="only the dequant-fused matmul microbench: 4 types x 4 shapes x batch "
                         "1/8/64/512, one JSON line")
    ap.add_argument("--no-70b", action="store_true",
                    help="skip the 70B-shaped leg of the default run (tensor parallel over all "
                         "GPUs; one GPU at N = 1)")
    ap.add_argument("--no-microbench", action="store_true",
                    help="skip the one-shape microbench leg of the default run")
    ap.add_argument("--vocab", type=int, default=0,
                    help="testing only: an 8B-shaped model with this vocabulary size (0 = 128256)")
    ap.add_argument("--layers", type=int, default=0,
                    help="profiling only: an 8B-shaped model with this many layers "
                         "(0 = the full 32); the line's config names it")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.gemm:
        run_gemm_case(args.gemm)
    elif args.microbench:
        rows = run_microbench(MB_SHAPES)
        print(json.dumps({"metric": "dequant-fused matmul microbench (configs[1])", "unit": "GB/s | TFLOP/s",
                          "peaks": {"hbm_gbs": peaks()[0], "bf16_tflops": bf16_peak()},
                          "rows": rows}), flush=True)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
