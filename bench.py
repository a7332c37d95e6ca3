"""Decode benchmark: Llama-3-8B-shape Q4_0 greedy decode on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 8b|8b-q4km|tiny|70b]

A step is one greedy decode token at batch 1 (the reference's per-token decode loop,
reference src/engine.cpp:684-804), after a 512-token prompt: positions 512+W .. 512+W+K-1.
  value  tokens/s with everything resident in HBM: K decode steps back to back (one
         persistent kernel per token on one GPU; the captured kernel-per-operation graph
         under tensor parallelism), the argmax token fed back on the device (CUDA events on
         the engine stream, max over ranks).
  e2e    the same K tokens through jinf_engine_generate with host buffers: per token a
         4-byte H2D of the fed-back id from pinned memory and a 4-byte D2H of the argmax.
  roofline  the dominant kernel against the measured HBM copy bandwidth: on one GPU the
         persistent step kernel itself (algorithmic bytes per launch = quantized weights +
         KV rows read per token, timed by the same CUDA events as `value`); under tensor
         parallelism the costliest per-operation GEMV timed alone.
  cpu_baseline  the CPU oracle (restated reference math, reference dequant conventions)
         on the host cores timing whole decode tokens (every layer and the LM head), a
         bounded sample of the same decode, rank 0 at N=1 only; --impl reference runs the
         same function over --steps tokens. Its weights come from the oracle's own copy of
         the seeded generator, so that arm loads no B200 code.
Under torchrun (N > 1) the model is tensor parallel over the ranks (NCCL allreduce inside
the captured step). --impl reference times the CPU implementation of the path.
--batch B (config C5's batch 8) decodes B sequences per step (jinf_engine_decode_batch: every
projection's weights streamed once for all B, each sequence with its own KV cache, filled with
seeded values to the first decode position); value and e2e count the tokens of all B.
Weights are synthetic N(0, 0.02) Q4_0 from seed 0 (no checkpoints): data "synthetic".
"""
from __future__ import annotations

import argparse
import contextlib
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "jetson-inference_b200"))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s Llama-3-8B-shape Q4_0 @1/2/4/8 B200; GEMV HBM GB/s vs peak"
PROMPT = 512


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d.get("hbm_gbs", 6650.0)), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines = []
        self.n0 = 0

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.idx), "-lms", "20"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            # nvidia-smi takes a while to start: wait for its first sample, so that it samples
            # while the timed region runs; samples taken before the region are not counted
            t0 = time.time()
            while not self.lines and time.time() - t0 < 3.0:
                time.sleep(0.005)
            self.n0 = len(self.lines)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def __exit__(self, *a):
        if self.proc:
            # a region shorter than the sampling period: the first sample after it ends
            t0 = time.time()
            while len(self.lines) <= self.n0 and time.time() - t0 < 0.2:
                time.sleep(0.002)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines[self.n0:]:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


@contextlib.contextmanager
def stdout_to_stderr():
    """File descriptor 1 points at stderr meanwhile: NCCL prints its version banner on stdout
    when the engine creates its communicator, and rank 0's JSON line must be the only output."""
    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(2, 1)
    try:
        yield
    finally:
        sys.stdout.flush()
        os.dup2(saved, 1)
        os.close(saved)


def init_dist(world):
    if world == 1:
        return None
    import datetime
    import torch.distributed as dist
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
    return dist


def all_max(dist, v: float) -> float:
    if dist is None:
        return v
    import torch
    t = torch.tensor([v], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class Shape:
    """A Llama-architecture shape (the BASELINE configurations; the same fields as the
    package's LlamaShape, kept here so the CPU arm never loads the B200 library)."""

    def __init__(self, n_layers, n_embd, n_heads, n_heads_kv, n_ff, n_vocab, rope_freq_base, rms_norm_eps=1e-5):
        self.n_layers, self.n_embd, self.n_heads, self.n_heads_kv = n_layers, n_embd, n_heads, n_heads_kv
        self.n_ff, self.n_vocab, self.rope_freq_base, self.rms_norm_eps = n_ff, n_vocab, rope_freq_base, rms_norm_eps
        self.n_ctx_train = 8192
        self.head_dim = n_embd // n_heads

    def llama(self):
        import jinf
        return jinf.LlamaShape(self.n_layers, self.n_embd, self.n_heads, self.n_heads_kv, self.n_ff, self.n_vocab,
                               self.rope_freq_base, self.rms_norm_eps)


SHAPES = {"8b": Shape(32, 4096, 32, 8, 14336, 128256, 500000.0), "8b-q4km": Shape(32, 4096, 32, 8, 14336, 128256, 500000.0),
          "tiny": Shape(4, 512, 8, 2, 1408, 4096, 10000.0), "70b": Shape(80, 8192, 64, 8, 28672, 128256, 500000.0)}
Q4_0, Q4_K, Q6_K = 2, 12, 14  # the reference's jinf_qtype values


def shape_for(name):
    return SHAPES[name]


def wtype_for(name):
    """Weight quantisation of a config: Q4_K for the 70B shape (config C5) and for the
    Q4_K_M-like 8B file, else Q4_0."""
    return Q4_K if name in ("70b", "8b-q4km") else Q4_0


def mix_for(name):
    """Second weight type of a config: Q6_K for attn_v and ffn_down of the even layers and for
    the output head in the Q4_K_M-like 8B file (8b-q4km), else none."""
    return Q6_K if name == "8b-q4km" else 0


def wname_for(name):
    return {"70b": "q4_k", "8b-q4km": "q4_k+q6_k"}.get(name, "q4_0")


def prompt_ids(n_vocab, n=PROMPT):
    import numpy as np
    return [int(t) for t in np.random.default_rng(0).integers(0, n_vocab, size=n)]


# ------------------------------------------------------------------------- CPU decode

def start_pos(args):
    """Position of the first decode step: the prompt length, or --ctx (the KV cache filled with
    seeded values up to it after the prompt: config C5's 8192-position cache)."""
    return max(PROMPT, args.ctx)


def bench_config(args, world):
    """The workload description both arms print (the same dict on both)."""
    shape = shape_for(args.config)
    wbytes = weight_bytes(shape, args.config)
    p0 = start_pos(args)
    if args.batch > 1:
        kv = f", {args.batch} sequences, each KV cache filled with seeded values to {p0} positions"
    else:
        kv = "" if p0 == PROMPT else f", KV cache filled to {p0} positions"
    return {"workload": f"{args.config} greedy decode batch {args.batch}, prompt {PROMPT}{kv}, positions "
                        f"{p0 + args.warmup}..{p0 + args.warmup + args.steps - 1}",
            "model": f"llama3-{args.config}-shape", "global_batch": args.batch, "seq_len": p0 + args.steps,
            "parallelism": f"tp{world}",
            "ffn": ["dense", "sparse: device predictor top-k 15%", "sparse: fixed mask 15% (runs of 8)"][args.sparse],
            "l2": f"{wbytes / 1e9:.2f} GB of weights streamed per step >> 126 MB L2 (no flush needed)"}


def weight_bytes(shape, config):
    """Quantized weight bytes of one decode token (all projections and the LM head), in the
    reference's block sizes."""
    from oracle import oracle
    src = oracle.SynthSource(shape, seed=0, weight_type=wtype_for(config), mix_type=mix_for(config))
    tot = 0
    for n in src.tensor_names():
        t, _, nb = src.tensor_info(n)
        if t != 0 and n != "token_embd.weight":
            tot += nb
    src.close()
    return tot


def cpu_decode(shape, config, warmup: int, steps: int, max_seconds: float | None = None, p0: int = PROMPT):
    """The CPU implementation of the decode path (the oracle: the reference's dequant
    conventions and its kernels' math restated on the host, OpenMP over rows) timing WHOLE
    decode tokens: every layer and the LM head, positions PROMPT + warmup onwards over a KV
    cache filled with seeded values for the prompt. Weights come from the oracle's own copy of
    the seeded generator (oracle/libsynth.so), so nothing of the B200 library is loaded.
    With max_seconds, stops early once that much timed work is done (at least 2 tokens).
    Returns (tok/s, threads, tokens timed, seconds timed)."""
    from oracle import oracle
    src = oracle.SynthSource(shape, seed=0, weight_type=wtype_for(config), mix_type=mix_for(config))
    om = oracle.OracleModel(src, max_ctx=p0 + warmup + steps + 8, kv_f16=True)
    om.fill_kv_random(p0, seed=1)
    tok = 1
    for _ in range(warmup):
        tok = oracle.argmax(om.forward(tok))
    n, t = 0, 0.0
    while n < steps:
        a = time.perf_counter()
        logits = om.forward(tok)
        t += time.perf_counter() - a
        tok = oracle.argmax(logits)
        n += 1
        if max_seconds is not None and n >= 2 and t >= max_seconds:
            break
    om.close()
    src.close()
    return n / t, oracle.num_threads(), n, t


# ------------------------------------------------------------------------- reference arm

def run_reference(args, rank, world):
    """The reference's decode path on the host cores. The reference has no CPU forward pass
    (its math exists only as CUDA kernels), so this is the oracle restatement of it
    (cpu_decode), timing --steps whole tokens after --warmup untimed ones."""
    if rank != 0:
        return
    shape = shape_for(args.config)
    p0 = start_pos(args)
    value, cores, n, secs = cpu_decode(shape, args.config, args.warmup, args.steps, p0=p0)
    sample = (f"{n} whole decode tokens (all {shape.n_layers} layers + LM head, greedy argmax) at positions "
              f"{p0 + args.warmup}..{p0 + args.warmup + n - 1} after {args.warmup} untimed, "
              f"{secs:.1f} s timed")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * secs / n,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": f"{wname_for(args.config)} weights, f32 activations, f16 KV",
            "data": f"synthetic (seeded N(0,0.02) {wname_for(args.config).upper()} weights, uniform prompt ids)",
            "config": bench_config(args, world),
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------- our arm

def gemv_microbench(dev, peak):
    """C2: Q4_0 GEMV on the 8B projection shapes, batch 1 / 4 / 8, fp16 x, rotating weight copies
    so every launch streams from HBM (>= 4x L2 of weights per shape); the launches are
    captured in a CUDA graph so the host launch rate does not cap small shapes."""
    import numpy as np
    import torch
    from jinf import kernels as K
    import jinf
    shapes = [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]
    out = {}
    for rows, cols in shapes:
        wbytes = rows * cols // 32 * 18
        copies = max(2, int(4 * 126e6 // wbytes) + 1)
        nq = K.q4m_bytes(rows, cols)
        syn = jinf.SynthModel(jinf.LlamaShape(1, cols, 32, 8, 4096, rows), seed=rows)
        aos = torch.empty(wbytes, dtype=torch.uint8, device=dev)
        syn.read_rows_device("output.weight", aos)
        qs = []
        for c in range(copies):
            q = torch.empty(nq, dtype=torch.uint8, device=dev)
            K.q4m_pack(aos, q, rows, cols)
            qs.append(q)
        del aos
        out[f"{rows}x{cols}"] = {}
        for batch in (1, 4, 8):
            if batch == 1:
                ws = torch.zeros(K.gemv_q4m_workspace_bytes(rows, cols), dtype=torch.uint8, device=dev)
            else:
                ws = torch.zeros(K.gemv_q4m_batch_workspace_bytes(rows, cols, batch), dtype=torch.uint8, device=dev)
            x = torch.from_numpy(np.random.default_rng(0).standard_normal((batch, cols)).astype(np.float16)).to(dev)
            y = torch.empty((batch, rows), dtype=torch.float32, device=dev)

            def launch(q):
                if batch == 1:
                    K.gemv_q4m(q, x, y, rows, cols, workspace=ws)
                else:
                    K.gemv_q4m_batch(q, x, y, rows, cols, batch, workspace=ws)

            for i in range(3):
                launch(qs[i % copies])
            torch.cuda.synchronize()
            n = copies * max(1, 60 // copies)
            s = torch.cuda.Stream()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(s):
                with torch.cuda.graph(g, stream=s):
                    for i in range(n):
                        launch(qs[i % copies])
            g.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            del g
            us = e0.elapsed_time(e1) * 1000.0 / n
            gbs = (wbytes + batch * (2 * cols + 4 * rows)) / (us * 1e-6) / 1e9
            out[f"{rows}x{cols}"][f"b{batch}"] = {"us": round(us, 2), "GB/s": round(gbs, 1), "frac": round(gbs / peak, 3)}
        del qs
        torch.cuda.empty_cache()
    return out


def cpu_gemv_c2(reps: int = 5):
    """C2 on the host cores: the oracle's dequant-matvec (reference Q4_0 conventions, OpenMP
    over rows) on the same shapes at batch 1, GB/s of weight + x + y bytes, median of reps."""
    import numpy as np
    from oracle import oracle
    out = {}
    for rows, cols in [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]:
        src = oracle.SynthSource(Shape(1, cols, 32, 8, 4096, rows, 10000.0), seed=rows)
        w = np.ascontiguousarray(src.read_rows("output.weight"))
        x = np.random.default_rng(0).standard_normal(cols).astype(np.float16).astype(np.float32)
        oracle.matvec(w, Q4_0, x, rows, cols)
        ts = []
        for _ in range(reps):
            a = time.perf_counter()
            oracle.matvec(w, Q4_0, x, rows, cols)
            ts.append(time.perf_counter() - a)
        t = sorted(ts)[len(ts) // 2]
        out[f"{rows}x{cols}"] = {"us": round(1e6 * t, 1), "GB/s": round((w.nbytes + 4 * cols + 4 * rows) / t / 1e9, 2)}
        src.close()
    out["cores"] = oracle.num_threads()
    return out


def run_ours(args, rank, world, local):
    import numpy as np
    import torch
    import jinf

    dist = init_dist(world)
    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    shape = shape_for(args.config)
    peak, peak_kind = peaks()

    nccl_id = None
    if world > 1:
        buf = [jinf.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(buf, src=0)
        nccl_id = buf[0]
    t_load = time.perf_counter()
    syn = jinf.SynthModel(shape.llama(), seed=0, weight_type=wtype_for(args.config), mix_type=mix_for(args.config))
    p0 = start_pos(args)
    max_ctx = p0 + args.warmup + args.steps + 8
    opts = jinf.b200_options(device=local, tp_rank=rank, tp_size=world, nccl_id=nccl_id, eos_token=-1,
                             sparse_mode=args.sparse)
    with stdout_to_stderr():
        eng = jinf.Engine.from_synth(syn, max_context=max_ctx, options=opts)
    t_load = time.perf_counter() - t_load
    stream = torch.cuda.ExternalStream(eng.h.contents.compute_stream, device=dev)
    prompt = prompt_ids(shape.n_vocab)

    # ---- time to first token: the prompt through forward() (batched tensor-core prefill of all
    # but its last token where the model allows it, then one decode step), and the same prompt
    # one token per forward() as the reference runs it (src/engine.cpp:690-751)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    eng.forward(prompt)
    torch.cuda.synchronize()
    prompt_s = time.perf_counter() - t0
    eng.reset()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for t in prompt:
        eng.forward([t])
    torch.cuda.synchronize()
    tokenwise_s = time.perf_counter() - t0
    eng.reset()
    eng.forward(prompt)
    if p0 > PROMPT:
        eng.fill_kv_random(p0, seed=1)

    # ---- value: resident decode, K steps timed on the device
    eng.decode_resident(args.warmup)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(stream)
        eng.decode_resident(args.steps)
        e1.record(stream)
        torch.cuda.synchronize()
    if dist:
        dist.barrier()
    dev_s = all_max(dist, e0.elapsed_time(e1) / 1000.0)
    value = args.steps / dev_s

    # ---- e2e: the same window through jinf_engine_generate (host buffers)
    eng.reset()
    eng.forward(prompt)
    if p0 > PROMPT:
        eng.fill_kv_random(p0, seed=1)
    eng.generate([], args.warmup)  # emits W tokens, forwards them
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    out = eng.generate([], args.steps)
    t1 = time.perf_counter()
    if dist:
        dist.barrier()
    e2e_s = all_max(dist, t1 - t0)
    e2e = len(out) / e2e_s

    # ---- roofline of the dominant kernel, per-launch algorithmic bytes / CUDA-event time
    persistent = eng.persistent
    prof = eng.profile_kernels(reps=max(32, shape.n_layers))  # kernel-per-operation form, each timed alone
    wbytes = eng.weight_bytes_per_token()
    kv_bytes = 2 * 2 * shape.n_layers * (shape.n_heads_kv // world) * shape.head_dim * (p0 + args.warmup + args.steps / 2)
    step_gbs = (wbytes + kv_bytes) / (dev_s / args.steps) / 1e9
    if persistent:
        roof = {"bound": "hbm", "kernel": "k_step (persistent decode step, one launch per token)",
                "achieved": round(step_gbs, 1), "peak": peak, "unit": "GB/s", "frac": round(step_gbs / peak, 4),
                "peak_kind": peak_kind, "traffic": None,
                "traffic_note": "not measured by this run (no profiler in the timed process); DRAM bytes of the "
                                "same kernel come from separate ncu captures",
                "bytes_per_launch": int(wbytes + kv_bytes), "us_per_launch": round(1e6 * dev_s / args.steps, 2)}
    else:
        top = max(("qkv", "o_proj", "gate_up", "down", "lm_head", "sparse_ffn"),
                  key=lambda k: prof[k]["us"] * (shape.n_layers if k != "lm_head" else 1))
        achieved = prof[top]["bytes"] / (prof[top]["us"] * 1e-6) / 1e9
        kname = "sparse FFN (predictor + bundles)" if top == "sparse_ffn" else f"k_gemv_q4m ({top})"
        roof = {"bound": "hbm", "kernel": kname, "achieved": round(achieved, 1), "peak": peak,
                "unit": "GB/s", "frac": round(achieved / peak, 4), "peak_kind": peak_kind, "traffic": None,
                "bytes_per_launch": prof[top]["bytes"], "us_per_launch": round(prof[top]["us"], 2)}

    gemv = gemv_microbench(dev, peak) if (world == 1 and args.config == "8b" and not args.no_gemv) else None
    launches_per_step = 1 if persistent else shape.n_layers * 5 + 2
    line = None
    if rank == 0:
        cpu, cpu_gemv = None, None
        if world == 1 and not args.no_cpu:
            cv, cores, n, secs = cpu_decode(shape, args.config, 1, 64, max_seconds=args.cpu_seconds, p0=p0)
            desc = (f"{n} whole decode tokens (all {shape.n_layers} layers + LM head, greedy argmax) at positions "
                    f"{p0 + 1}..{p0 + n} after 1 untimed, {secs:.1f} s timed; the same method as "
                    f"--impl reference")
            cpu = {"value": cv, "unit": "tok/s", "cores": cores, "kind": "port", "sample": desc}
            if gemv:
                cpu_gemv = cpu_gemv_c2()
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 * dev_s / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": f"{wname_for(args.config)} weights, f32 activations, f16 KV",
            "data": f"synthetic (seeded N(0,0.02) {wname_for(args.config).upper()} weights, uniform prompt ids)",
            "config": bench_config(args, world),
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4},
            "gpu_launches": launches_per_step * args.steps,
            "roofline": roof,
            "decode_roofline": {"weights_bytes_per_token": wbytes, "kv_bytes_per_token_avg": int(kv_bytes),
                                "achieved_GBs": round(step_gbs, 1), "frac": round(step_gbs / peak, 4),
                                "roofline_tok_s": round(peak * 1e9 / (wbytes + kv_bytes), 1)},
            "per_op_kernels_us": {k: round(v["us"], 2) for k, v in prof.items()},
            "prompt": {"tokens": len(prompt), "forward_ms": round(1e3 * prompt_s, 2),
                       "tok_s": round(len(prompt) / prompt_s, 1), "one_token_per_forward_ms": round(1e3 * tokenwise_s, 2),
                       "note": "host wall time of forward(prompt) (batched tensor-core prefill of all but the last "
                               "token where the model allows it, then one decode step) and of one forward() per "
                               "prompt token"},
            "clocks": clk.summary(),
            "load_s": round(t_load, 1),
        }
        if cpu:
            line["cpu_baseline"] = cpu
        if gemv:
            line["gemv_c2"] = gemv
        if cpu_gemv:
            line["gemv_c2_cpu"] = cpu_gemv
        print(json.dumps(line), flush=True)
    eng.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def run_ours_batch(args, rank, world, local):
    """--batch B: B sequences per step through the multi-sequence decode."""
    import torch
    import jinf

    dist = init_dist(world)
    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    shape = shape_for(args.config)
    peak, peak_kind = peaks()
    B = args.batch
    nccl_id = None
    if world > 1:
        buf = [jinf.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(buf, src=0)
        nccl_id = buf[0]
    t_load = time.perf_counter()
    syn = jinf.SynthModel(shape.llama(), seed=0, weight_type=wtype_for(args.config), mix_type=mix_for(args.config))
    p0 = start_pos(args)
    max_ctx = p0 + args.warmup + args.steps + 8
    opts = jinf.b200_options(device=local, tp_rank=rank, tp_size=world, nccl_id=nccl_id, eos_token=-1,
                             max_seqs=B)
    with stdout_to_stderr():
        eng = jinf.Engine.from_synth(syn, max_context=max_ctx, options=opts)
    t_load = time.perf_counter() - t_load
    stream = torch.cuda.ExternalStream(eng.h.contents.compute_stream, device=dev)
    seqs = list(range(B))
    first = prompt_ids(shape.n_vocab, n=B)

    def fill():
        for s in seqs:
            eng.seq_fill_kv_random(s, p0, seed=1 + s)

    # ---- value: resident steps (argmax fed back on the device), K steps timed on the device
    fill()
    eng.decode_batch_resident(seqs, first, args.warmup)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(stream)
        eng.decode_batch_resident(seqs, first, args.steps)
        e1.record(stream)
        torch.cuda.synchronize()
    if dist:
        dist.barrier()
    dev_s = all_max(dist, e0.elapsed_time(e1) / 1000.0)
    value = B * args.steps / dev_s

    # ---- e2e: the same window through jinf_engine_decode_batch, host buffers every step
    fill()
    toks = first
    for _ in range(args.warmup):
        toks = eng.decode_batch(seqs, toks)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        toks = eng.decode_batch(seqs, toks)
    t1 = time.perf_counter()
    if dist:
        dist.barrier()
    e2e = B * args.steps / all_max(dist, t1 - t0)
    # per-kernel times of the step (each kind back to back over the layers, after the timed runs)
    prof = eng.profile_multi(B, reps=2 * shape.n_layers)

    wbytes = eng.weight_bytes_per_token()
    kv_seq = 2 * 2 * shape.n_layers * (shape.n_heads_kv // world) * shape.head_dim * (p0 + args.warmup + args.steps / 2)
    step_bytes = wbytes + B * kv_seq
    step_gbs = step_bytes / (dev_s / args.steps) / 1e9
    launches = 1 + 5 * shape.n_layers + 2 + (2 * shape.n_layers if world > 1 else 0)
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 * dev_s / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": f"{wname_for(args.config)} weights, f32 activations, f16 KV",
            "data": f"synthetic (seeded N(0,0.02) {wname_for(args.config).upper()} weights, seeded N(0,1) KV)",
            "config": bench_config(args, world),
            # per step: the 8-slot token / position / sequence arrays and sequence 0's position in,
            # one argmax id per sequence out
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 3 * 8 * 4 + 4,
                    "d2h_bytes_per_step": 4 * B},
            "gpu_launches": launches * args.steps,
            "roofline": {"bound": "hbm", "kernel": "multi-sequence step (k_gemv_multi + k_attn_multi graph)",
                         "achieved": round(step_gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(step_gbs / peak, 4), "peak_kind": peak_kind, "traffic": None,
                         "bytes_per_step": int(step_bytes), "us_per_step": round(1e6 * dev_s / args.steps, 2),
                         "note": "weights once per step + every sequence's KV rows"},
            "per_op_kernels_us": {k: round(v["us"], 2) for k, v in prof.items()},
            "clocks": clk.summary(),
            "load_s": round(t_load, 1),
        }
        print(json.dumps(line), flush=True)
    eng.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def profile_case(steps: int, batch: int = 1) -> None:
    """The small case of the persistent step for ncu captures: ~0.6 GB of weights plus a
    0.5 GB embedding table; with a 3-token prompt the captured launch `-s 3 -c 1` is the
    first decode step at position 513. With batch > 1: the same model's multi-sequence step,
    `batch` sequences each with its KV cache filled to 512 positions, `steps` resident steps
    (per step one k_multi_rows, per layer QKV, attention, o, gate|up, down, then the LM head
    and the finaliser: 4 x 4 + 1 k_gemv_multi launches)."""
    import torch
    import jinf
    shape = jinf.LlamaShape(4, 4096, 32, 8, 14336, 32000, 5e5)
    if batch > 1:
        eng = jinf.Engine.from_synth(jinf.SynthModel(shape, seed=0), max_context=600,
                                     options=jinf.b200_options(eos_token=-1, max_seqs=batch))
        seqs = list(range(batch))
        for s in seqs:
            eng.seq_fill_kv_random(s, 512, seed=1 + s)
        eng.decode_batch_resident(seqs, [1 + s for s in seqs], steps)
        torch.cuda.synchronize()
        eng.close()
        print("profile case ok")
        return
    eng = jinf.Engine.from_synth(jinf.SynthModel(shape, seed=0), max_context=600,
                                 options=jinf.b200_options(eos_token=-1))
    eng.forward([1, 2, 3])
    eng.fill_kv_random(512, seed=1)
    eng.forward([5])
    eng.decode_resident(steps)
    torch.cuda.synchronize()
    eng.close()
    print("profile case ok")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="8b", choices=["8b", "8b-q4km", "tiny", "70b"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--no-gemv", action="store_true", help="skip the C2 GEMV shape sweep")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--ctx", type=int, default=PROMPT,
                    help="first decode position: the KV cache is filled with seeded values up to it after the prompt "
                         "(config C5: 8192)")
    ap.add_argument("--batch", type=int, default=1, choices=range(1, 9), metavar="B",
                    help="sequences decoded per step (1..8; config C5: 8)")
    ap.add_argument("--sparse", type=int, default=0, choices=[0, 1, 2],
                    help="FFN: 0 dense, 1 device predictor top-k, 2 fixed mask (BASELINE config C4)")
    ap.add_argument("--profile-case", type=int, default=0, metavar="STEPS",
                    help="run only the small case used for ncu captures of the step kernel and exit: a 4-layer "
                         "8B-shaped model (vocabulary 32000), KV filled to position 512, one forwarded token, "
                         "then STEPS resident decode steps (with --batch B: B sequences through the "
                         "multi-sequence step)")
    args = ap.parse_args()
    if args.profile_case:
        profile_case(args.profile_case, args.batch)
        return
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.batch > 1:
        if args.sparse:
            ap.error("--batch needs the dense FFN")
        run_ours_batch(args, rank, world, local)
        return
    run_ours(args, rank, world, local)


if __name__ == "__main__":
    main()
