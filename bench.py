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
         on the host cores, a bounded sample of the same decode, rank 0 at N=1 only.
Under torchrun (N > 1) the model is tensor parallel over the ranks (NCCL allreduce inside
the captured step). --impl reference times the CPU implementation of the path.
Weights are synthetic N(0, 0.02) Q4_0 from seed 0 (no checkpoints): data "synthetic".
"""
from __future__ import annotations

import argparse
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


def traffic_ratio():
    """DRAM bytes / algorithmic bytes of the step kernel from the committed ncu summary
    (profiles/k_step_4layer_8bshape_full.md, captured on a 4-layer case of the same kernel
    and scaled per launch by the bytes processed), or None."""
    p = os.path.join(ROOT, "profiles", "k_step_4layer_8bshape_full.md")
    try:
        for ln in open(p):
            if ln.startswith("traffic_ratio:"):
                return float(ln.split(":", 1)[1])
    except OSError:
        pass
    return None


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

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.idx), "-lms", "20"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            time.sleep(0.05)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.03)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

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


def shape_for(name):
    import jinf
    return {"8b": jinf.LLAMA3_8B, "8b-q4km": jinf.LLAMA3_8B, "tiny": jinf.TINY, "70b": jinf.LLAMA3_70B}[name]


def wtype_for(name):
    """Weight quantisation of a config: Q4_K for the 70B shape and for the
    Q4_K_M-like 8B file, else Q4_0."""
    from jinf import _lib as L
    return L.Q4_K if name in ("70b", "8b-q4km") else L.Q4_0


def mix_for(name):
    """Second weight type of a config: Q6_K for attn_v and ffn_down of the even layers and for
    the output head in the Q4_K_M-like 8B file (8b-q4km), else none."""
    from jinf import _lib as L
    return L.Q6_K if name == "8b-q4km" else 0


def wname_for(name):
    return {"70b": "q4_k", "8b-q4km": "q4_k+q6_k"}.get(name, "q4_0")


def prompt_ids(n_vocab, n=PROMPT):
    import numpy as np
    return [int(t) for t in np.random.default_rng(0).integers(0, n_vocab, size=n)]


# ------------------------------------------------------------------------- CPU oracle

def cpu_decode_sample(shape, layers: int, target_s: float, min_reps: int = 2, wtype=None, mix=0):
    """Time the CPU oracle on `layers` layers (+ LM head) of a decode token at position PROMPT,
    extrapolate the per-token time to all layers. Returns (tok/s, threads, description)."""
    from oracle import oracle
    import jinf
    syn = (jinf.SynthModel(shape, seed=0, weight_type=wtype, mix_type=mix) if wtype is not None
           else jinf.SynthModel(shape, seed=0))
    om = oracle.OracleModel(syn, max_ctx=PROMPT + 512, kv_f16=True, layers=layers)
    om.fill_kv_random(PROMPT, seed=1)
    tok = 1
    om.forward(tok, want_logits=False)  # warm caches / threads
    t_layers, t_full = [], []
    t0 = time.perf_counter()
    while (len(t_layers) < min_reps or time.perf_counter() - t0 < target_s) and om.pos < PROMPT + 500:
        a = time.perf_counter()
        om.forward(tok, want_logits=False)
        b = time.perf_counter()
        om.forward(tok, want_logits=True)
        c = time.perf_counter()
        t_layers.append(b - a)
        t_full.append(c - b)
    t_l = sorted(t_layers)[len(t_layers) // 2] / layers
    t_head = max(0.0, sorted(t_full)[len(t_full) // 2] - t_l * layers)
    per_tok = t_l * shape.n_layers + t_head
    desc = (f"{len(t_layers)}x2 decode tokens at position {PROMPT}..{om.pos} over {layers}/{shape.n_layers} "
            f"layers + LM head, per-token time = {shape.n_layers}*layer + head (extrapolated); "
            f"{time.perf_counter() - t0:.1f} s of CPU work")
    om.close()
    return 1.0 / per_tok, oracle.num_threads(), desc, per_tok


# ------------------------------------------------------------------------- reference arm

def run_reference(args, rank, world):
    """CPU implementation of the decode path on the host cores (the reference has no CPU
    forward pass: the oracle restatement of its math, with its dequant conventions)."""
    if rank != 0:
        return
    shape = shape_for(args.config)
    from oracle import oracle
    import jinf
    layers = 1
    syn = jinf.SynthModel(shape, seed=0, weight_type=wtype_for(args.config), mix_type=mix_for(args.config))
    om = oracle.OracleModel(syn, max_ctx=PROMPT + args.warmup + args.steps + 8, kv_f16=True, layers=layers)
    om.fill_kv_random(PROMPT, seed=1)
    for _ in range(args.warmup):
        om.forward(1, want_logits=False)
    times = []
    for _ in range(args.steps):
        a = time.perf_counter()
        om.forward(1, want_logits=False)
        times.append(time.perf_counter() - a)
    a = time.perf_counter()
    om.forward(1, want_logits=True)
    t_head = max(0.0, time.perf_counter() - a - sorted(times)[len(times) // 2])
    t_layer = sum(times) / len(times) / layers
    per_tok = t_layer * shape.n_layers + t_head
    value = 1.0 / per_tok
    cores = oracle.num_threads()
    sample = (f"each step = 1 of {shape.n_layers} layers of one decode token (positions {PROMPT}+), "
              f"tok/s = 1/({shape.n_layers}*mean step + LM head)")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * per_tok,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": f"{wname_for(args.config)} weights, f32",
            "data": f"synthetic (seeded N(0,0.02) {wname_for(args.config).upper()} weights)",
            "config": {"workload": f"{args.config} decode batch 1, prompt {PROMPT}", "model": args.config,
                       "global_batch": 1, "seq_len": PROMPT + args.steps, "parallelism": "cpu"},
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
    syn = jinf.SynthModel(shape, seed=0, weight_type=wtype_for(args.config), mix_type=mix_for(args.config))
    max_ctx = PROMPT + args.warmup + args.steps + 8
    opts = jinf.b200_options(device=local, tp_rank=rank, tp_size=world, nccl_id=nccl_id, eos_token=-1,
                             sparse_mode=args.sparse)
    eng = jinf.Engine.from_synth(syn, max_context=max_ctx, options=opts)
    t_load = time.perf_counter() - t_load
    stream = torch.cuda.ExternalStream(eng.h.contents.compute_stream, device=dev)
    prompt = prompt_ids(shape.n_vocab)

    # ---- value: resident decode, K steps timed on the device
    eng.forward(prompt)
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
    kv_bytes = 2 * 2 * shape.n_layers * (shape.n_heads_kv // world) * shape.head_dim * (PROMPT + args.warmup + args.steps / 2)
    step_gbs = (wbytes + kv_bytes) / (dev_s / args.steps) / 1e9
    if persistent:
        ratio = traffic_ratio()
        roof = {"bound": "hbm", "kernel": "k_step (persistent decode step, one launch per token)",
                "achieved": round(step_gbs, 1), "peak": peak, "unit": "GB/s", "frac": round(step_gbs / peak, 4),
                "peak_kind": peak_kind,
                "traffic": int((wbytes + kv_bytes) * ratio) if ratio else None,
                "traffic_note": "ncu dram read+write bytes per launch, measured on a 4-layer case of the same "
                                "kernel and scaled by bytes processed (profiles/k_step_4layer_8bshape_full.md)",
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
        cpu = None
        if world == 1 and not args.no_cpu:
            cv, cores, desc, _ = cpu_decode_sample(
                shape, layers={"8b": 2, "8b-q4km": 2, "70b": 1}.get(args.config, shape.n_layers), target_s=args.cpu_seconds,
                wtype=wtype_for(args.config), mix=mix_for(args.config))
            cpu = {"value": cv, "unit": "tok/s", "cores": cores, "kind": "port", "sample": desc}
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 * dev_s / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": f"{wname_for(args.config)} weights, f32 activations, f16 KV",
            "data": f"synthetic (seeded N(0,0.02) {wname_for(args.config).upper()} weights, uniform prompt ids)",
            "config": {"workload": f"{args.config} greedy decode batch 1, prompt {PROMPT}, positions "
                                   f"{PROMPT + args.warmup}..{PROMPT + args.warmup + args.steps - 1}",
                       "model": f"llama3-{args.config}-shape", "global_batch": 1, "seq_len": PROMPT + args.steps,
                       "parallelism": f"tp{world}",
                       "ffn": ["dense", "sparse: device predictor top-k 15%", "sparse: fixed mask 15% (runs of 8)"][args.sparse],
                       "l2": f"{wbytes / 1e9:.2f} GB of weights streamed per step >> 126 MB L2 (no flush needed)"},
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4},
            "gpu_launches": launches_per_step * args.steps,
            "roofline": roof,
            "decode_roofline": {"weights_bytes_per_token": wbytes, "kv_bytes_per_token_avg": int(kv_bytes),
                                "achieved_GBs": round(step_gbs, 1), "frac": round(step_gbs / peak, 4),
                                "roofline_tok_s": round(peak * 1e9 / (wbytes + kv_bytes), 1)},
            "per_op_kernels_us": {k: round(v["us"], 2) for k, v in prof.items()},
            "clocks": clk.summary(),
            "load_s": round(t_load, 1),
        }
        if cpu:
            line["cpu_baseline"] = cpu
        if gemv:
            line["gemv_c2"] = gemv
        print(json.dumps(line), flush=True)
    eng.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


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
    ap.add_argument("--sparse", type=int, default=0, choices=[0, 1, 2],
                    help="FFN: 0 dense, 1 device predictor top-k, 2 fixed mask (BASELINE config C4)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    run_ours(args, rank, world, local)


if __name__ == "__main__":
    main()
