#!/usr/bin/env python3
"""Decode tokens/s at batch 1 for the B200 path of gollama.cu (one JSON line).

Default workload (1 GPU): a Llama-3.1-8B-shaped Q4_K_M model
with seeded random-init weights, the KV cache prefilled with seeded N(0,1)
fp16 values for positions 0..8191, then greedy decode steps at positions
8192..8319 (a 128-position window that repeats for longer runs). A step is one
decode token: embedding, 32 layers, lm_head and the argmax, as one CUDA graph
replay with the token and position resident on the device.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config 8b|1b|3b|70b]
  python -m torch.distributed.run --nproc-per-node N bench.py --gpus N ...   # tensor parallel
  python bench.py --impl reference ...   # the reference's CPU path (the C restatement of
                                         # backend/cpu + cpuForward), all host threads

`value` is device time (CUDA events on the model's stream, max over ranks);
`e2e` goes through the reference-facing call (gb_model_forward: token and
position copied in, the vocabulary logits copied out, host argmax) every step.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "gollama.cu_b200")
sys.path.insert(0, PKG)

CONFIGS = {
    # name: preset, KV setup, first decode position, window of positions, cache
    "8b": dict(preset=8, prefill=8192, prompt=0, window=128, kv_f16=1, max_len=8320,
               workload="llama-3.1-8b Q4_K_M decode, KV prefilled N(0,1) fp16 to 8192, positions 8192-8319"),
    "1b": dict(preset=1, prefill=0, prompt=16, window=64, kv_f16=0, max_len=512,
               workload="llama-3.2-1b Q4_0 decode after a 16-token prompt, f32 KV, positions 16-79"),
    "3b": dict(preset=3, prefill=0, prompt=32, window=256, kv_f16=1, max_len=4096,
               workload="llama-3.2-3b Q4_K_M decode after a 32-token prompt, fp16 KV, positions 32-287"),
    "70b": dict(preset=70, prefill=0, prompt=64, window=128, kv_f16=1, max_len=8192,
                workload="llama-3.1-70b Q4_K_M decode after a 64-token prompt, fp16 KV, positions 64-191"),
}
SEED = 0
KV_SEED = 1
METRIC = "decode tokens/s at batch 1"


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs, copy burst)"
    except Exception:
        return 6650.0, "fallback 6.65 TB/s (no MEASURED_PEAKS.json)"


def tensor_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured (MEASURED_PEAKS.json bf16_tflops, cuBLAS burst)"
    except Exception:
        return 1590.0, "fallback 1.59 PFLOP/s (no MEASURED_PEAKS.json)"


def prefill_flops(c, T):
    """Algorithmic FLOPs of gb_model_prefill over T tokens: the first T-1 through the
    batched layers (every GEMM 2*rows*cols per token; the last layer stops after its
    q|k|v; causal attention 4*head_dim per (query head, visible key)), the last token
    through one decode step (counted as its GEMV FLOPs)."""
    q, kv = c.heads * c.head_dim, c.kv_heads * c.head_dim
    qkv = 2 * c.dim * (q + 2 * kv)
    rest = 2 * q * c.dim + 2 * c.dim * 2 * c.ffn + 2 * c.ffn * c.dim
    n = T - 1
    gemm = n * (c.layers * qkv + (c.layers - 1) * rest)
    attn = (c.layers - 1) * 4 * c.heads * c.head_dim * (n * (n + 1) // 2)
    decode = c.layers * (qkv + rest) + 2 * c.dim * c.vocab
    return gemm + attn + decode


def ncu_traffic(config):
    """DRAM bytes per launch of the dominant kernel (gate/up + SwiGLU GEMV) from the
    ncu capture recorded in profiles/traffic.json (a static figure from an earlier
    capture, not measured in this run); None when no capture covers the config."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return int(json.load(f)[config]["dram_bytes_per_launch"])
    except (OSError, KeyError, ValueError):
        return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled while the timed region runs."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = gpus
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.out = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "--query-gpu=" + self.FIELDS,
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=self.out, stderr=subprocess.DEVNULL)
            time.sleep(0.2)
        except Exception:
            self.proc = None
        self.t0 = time.time()

    def mark(self):
        self.t0 = time.time()

    def stop(self):
        t1 = time.time()
        if not self.proc:
            return None
        time.sleep(0.1)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.out.close()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 10:
                    continue
                try:
                    ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                    rows.append((ts, int(parts[1]), float(parts[2]), float(parts[3]), parts[6:10]))
                except ValueError:
                    continue
        os.unlink(self.path)
        inside = [r for r in rows if self.t0 - 0.06 <= r[0] <= t1 + 0.06 and r[1] in self.gpus]
        if not inside:
            inside = [r for r in rows if r[1] in self.gpus][-3:]
        if not inside:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in inside for i, v in enumerate(r[4]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[2] for r in inside), "sm_max_mhz": max(r[3] for r in inside),
                "reasons": reasons, "samples": len(inside)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    # a CPU tensor under gloo (the CPU tests), a device tensor under NCCL
    dev = "cpu" if dist.get_backend() == "gloo" else "cuda"
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def build_image(gb, cfg, world, rank):
    """A synthetic GGUF image: in memory for one GPU, a shared file for several ranks."""
    spec = gb.synth_preset(cfg["preset"], seed=SEED)
    if cfg.get("layers"):
        spec.layers = cfg["layers"]  # profiling captures only: same shapes, fewer layers
    if world == 1:
        return gb.SynthImage(spec), spec
    path = os.path.join(tempfile.gettempdir(), f"gollama_b200_{cfg['preset']}_{SEED}.gguf")
    if rank == 0 and not os.path.exists(path):
        tmp = path + ".part"
        gb._check(gb.lib().gb_synth_model_file(gb.C.byref(spec), tmp.encode()))
        os.replace(tmp, path)
    barrier(world)
    return path, spec


def prompt_tokens(spec, n):
    rng = np.random.default_rng(SEED)
    return [int(t) for t in rng.integers(0, spec.vocab, n)]


SWEEP_TYPES = (("q4_0", 2), ("q4_k", 12), ("q6_k", 14))
SWEEP_SHAPES = ((4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096))
L2_BYTES = 126 * 1024 * 1024


def gemv_sweep(gb, torch, device, peak, launches=48, types=None, shapes=None):
    """the standalone batch-1 quantized GEMV (gb_linear_matvec,
    the kernel that replaces kernels/quantmv.go:18-136) for Q4_0 / Q4_K / Q6_K at
    four shapes. Weights follow the config's block recipe (seeds 0-3); enough
    device copies are rotated that every launch reads its weights from HBM (more
    than 3x the 126 MB L2 per pass). Launches go back to back on one stream
    (programmatic dependent launch, as in the decode step); CUDA events around
    `launches` of them give the time per launch. Algorithmic bytes per launch:
    rows*cols*(type bytes per weight) + 4*cols + 4*rows."""
    cases = []
    dev = torch.device("cuda", device)
    stream = torch.cuda.Stream(device=dev)
    for tname, typ in SWEEP_TYPES:
        if types and tname not in types:
            continue
        for rows, cols in SWEEP_SHAPES:
            if shapes and f"{rows}x{cols}" not in shapes:
                continue
            mats = [gb.synth_matrix(typ, rows, cols, seed=s) for s in range(4)]
            wbytes = mats[0].nbytes
            ncopy = max(4, -(-3 * L2_BYTES // wbytes))
            lins = [gb.Linear(typ, mats[i % 4], rows, cols, device=device) for i in range(ncopy)]
            xs = [torch.from_numpy(gb.synth_normal(s, 1, cols)).to(dev) for s in range(4)]
            ys = [torch.empty(rows, device=dev) for _ in range(4)]
            del mats
            with torch.cuda.stream(stream):
                for i in range(max(ncopy, 8)):  # warm-up: every copy once
                    lins[i % ncopy].matvec(xs[i % 4], ys[i % 4], stream=stream)
                ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                n = max(launches, ncopy)
                ev0.record(stream)
                for i in range(n):
                    lins[i % ncopy].matvec(xs[i % 4], ys[i % 4], stream=stream)
                ev1.record(stream)
            torch.cuda.synchronize(dev)
            us = ev0.elapsed_time(ev1) * 1e3 / n
            alg = wbytes + 4 * cols + 4 * rows
            cases.append({"type": tname, "rows": rows, "cols": cols, "bytes": alg, "us_per_launch": round(us, 3),
                          "gbs": round(alg / (us * 1e-6) / 1e9, 1), "frac": round(alg / (us * 1e-6) / 1e9 / peak, 4),
                          "copies": ncopy})
            for l in lins:
                l.close()
            del lins, xs, ys
            torch.cuda.empty_cache()
    big = [c for c in cases if c["rows"] * c["cols"] >= 14336 * 4096]
    return {"how": "gb_linear_matvec back to back over rotated weight copies (> 3x L2 per pass), CUDA events, "
                   "seeds 0-3 of the config-2 block recipe, x ~ N(0,1)",
            "peak_gbs": peak, "cases": cases,
            "min_frac_large_shapes": min(c["frac"] for c in big) if big else None}


def new_nccl_id(gb, world, rank):
    """A fresh NCCL unique id from rank 0 for one tensor-parallel model (None at one GPU)."""
    if world == 1:
        return None
    import torch.distributed as dist

    obj = [gb.tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    return obj[0]


def measure_config(gb, torch, name, world, rank, local, steps=64, warmup=4):
    """Decode tok/s of one more BASELINE configuration (1B, 3B, 70B) at the run's
    GPU count: its workload's prompt or KV prefill, then `steps` greedy graph steps
    timed with CUDA events on the model's stream (max over ranks), the
    bytes-per-token roofline, the first tokens, and one oracle step at the first
    decode position (rank 0)."""
    cfg = dict(CONFIGS[name])
    nccl_id = new_nccl_id(gb, world, rank)
    t_setup = time.perf_counter()
    src, spec = build_image(gb, cfg, world, rank)
    opts = dict(device=local, max_len=cfg["max_len"], kv_f16=cfg["kv_f16"], tp_rank=rank, tp_world=world)
    if nccl_id is not None:
        opts["nccl_id"] = nccl_id
    m = gb.Model(src, **opts)
    if cfg["prefill"]:
        m.fill_kv_normal(KV_SEED, cfg["prefill"])
    toks = prompt_tokens(spec, cfg["prompt"] + 1)
    for pos in range(cfg["prompt"]):
        m.forward_no_logits(toks[pos], pos)
    p0, t0 = cfg["prefill"] + cfg["prompt"], toks[-1]
    steps = min(steps, cfg["window"])
    stream = torch.cuda.ExternalStream(m.stream(), device=torch.device("cuda", local))
    m.start(t0, p0)
    m.decode_async(warmup)
    torch.cuda.synchronize()
    barrier(world)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    m.start(t0, p0)
    ev0.record(stream)
    m.decode_async(steps)
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(ev0.elapsed_time(ev1), world)
    first = [int(t) for t in m.read_tokens(p0, min(8, steps))]
    plog = m.forward(t0, p0).copy() if rank == 0 else m.forward_no_logits(t0, p0)
    # the prompt's K/V for the oracle (teacher-forced: running a 70B prompt through
    # the single-token CPU path would take minutes); one GPU only, since under
    # tensor parallelism each rank holds its own KV heads
    kv = [m.read_kv(layer, 0, p0) for layer in range(spec.layers)] if world == 1 and cfg["prompt"] else None
    m.close()
    setup_s = time.perf_counter() - t_setup
    peak = peaks()[0]
    tok_s = steps / (ms / 1e3)
    bytes_tok = model_bytes(spec, p0 + steps // 2, cfg["kv_f16"])
    out = {"workload": cfg["workload"], "model": bench_config(cfg, spec, world)["model"], "n_gpus": world,
           "value": round(tok_s, 2), "unit": "tok/s", "steps": steps, "ms_per_step": round(ms / steps, 5),
           "step_roofline": {"bytes_per_token": bytes_tok, "achieved_gbs": round(bytes_tok * tok_s / 1e9, 1),
                             "frac": round(bytes_tok * tok_s / 1e9 / (peak * world), 4),
                             "roofline_tok_s": round(peak * world * 1e9 / bytes_tok, 1),
                             "peak_gbs_per_gpu": peak},
           "first_tokens": first, "setup_s": round(setup_s, 1)}
    if rank == 0 and kv is not None:
        orc = _orc()
        om = orc.OracleModel(image_bytes(src), cfg["max_len"], bool(cfg["kv_f16"]))
        for layer, (k, v) in enumerate(kv):
            om.set_kv(layer, 0, k, v)
        out["parity"] = dict(parity_check(om, plog, t0, p0, spec.vocab),
                             how="one oracle step (C restatement of cpuForward) at the first decode position, "
                                 "the prompt's K/V copied from the device cache")
        om.close()
    elif rank == 0:
        out["parity"] = None if cfg["prompt"] else parity_check(oracle_model(image_bytes(src), spec, cfg), plog, t0,
                                                                p0, spec.vocab)
    if world == 1:
        src.close()
    barrier(world)
    if world > 1 and rank == 0 and isinstance(src, str):
        os.unlink(src)  # a 70B image is 42 GB of disk
    return out


def run_ours(args, cfg, world, rank, local):
    import torch

    import gollama_b200 as gb

    os.environ.setdefault("GB_HOST_THREADS", str(max(1, (os.cpu_count() or 8) // world)))
    nccl_id = None
    if world > 1:
        import torch.distributed as dist

        obj = [gb.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nccl_id = obj[0]
    src, spec = build_image(gb, cfg, world, rank)
    opts = dict(device=local, max_len=cfg["max_len"], kv_f16=cfg["kv_f16"], tp_rank=rank, tp_world=world)
    if nccl_id is not None:
        opts["nccl_id"] = nccl_id
    m = gb.Model(src, **opts)
    c = m.config
    if cfg["prefill"]:
        m.fill_kv_normal(KV_SEED, cfg["prefill"])
    toks = prompt_tokens(spec, cfg["prompt"] + 1)
    for pos in range(cfg["prompt"]):
        m.forward_no_logits(toks[pos], pos)
    p0 = cfg["prefill"] + cfg["prompt"]
    t0 = toks[-1]
    window = cfg["window"]
    stream = torch.cuda.ExternalStream(m.stream(), device=torch.device("cuda", local))

    def steps(n):
        # n greedy steps cycling over the window's positions
        done, off = 0, 0
        m.start(t0, p0)
        while done < n:
            k = min(n - done, window - off)
            m.decode_async(k)
            done += k
            off += k
            if off == window and done < n:
                m.start(t0, p0)
                off = 0

    # warm-up
    barrier(world)
    steps(args.warmup)
    torch.cuda.synchronize()
    barrier(world)
    clocks = ClockSampler(list(range(world))) if rank == 0 else None
    if clocks:
        clocks.start()
    barrier(world)
    torch.cuda.synchronize()
    if clocks:
        clocks.mark()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    steps(args.steps)
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop() if clocks else None
    ms = max_over_ranks(ev0.elapsed_time(ev1), world)
    toks_out = m.read_tokens(p0, min(args.steps, window))
    tok_s = args.steps / (ms / 1e3)

    # end to end through gb_model_forward: H2D token+position, D2H logits, host argmax
    barrier(world)
    n_e2e = max(8, min(args.steps, 2 * window))
    # the caller's logits buffer, page-locked: gb_model_forward copies into it directly
    logits = torch.empty(c.vocab, dtype=torch.float32, pin_memory=True).numpy()
    tok = t0
    m.forward(tok, p0) if rank == 0 else m.forward_no_logits(tok, p0)  # warm
    barrier(world)
    w0 = time.perf_counter()
    for i in range(n_e2e):
        pos = p0 + (i % window)
        if rank == 0:
            m.forward(tok, pos, out=logits)
            tok = gb.argmax(logits)
        else:
            m.forward_no_logits(tok, pos)
    wall = max_over_ranks(time.perf_counter() - w0, world)
    e2e = {"value": n_e2e / wall, "unit": "tok/s", "h2d_bytes_per_step": 8,
           "d2h_bytes_per_step": 4 * c.vocab + 4, "steps": n_e2e,
           "how": "wall clock around gb_model_forward into a page-locked host buffer + host model.Argmax per step"}

    # roofline of the dominant kernel (gate/up GEMV with the SwiGLU epilogue), device events
    prof = []
    for i in range(5):
        prof.append(m.profile_step(t0, p0 + i))
    gu_ms = statistics.median(p["gate_up"][0] / max(1, p["gate_up"][1]) for p in prof)
    bytes_tok, gu_bytes = m.step_bytes(p0 + window // 2)
    peak, peak_src = peaks()
    achieved = gu_bytes / (gu_ms / 1e3) / 1e9
    breakdown = {k: round(statistics.median(p[k][0] for p in prof), 4) for k in prof[0]}

    # batched prefill of a 512-token prompt (the timed decode above is done, so
    # overwriting cache positions 0..511 does not touch it) and continuous
    # batching (one GPU), first decoding the quantized weights in every GEMM,
    # then through the model's binary16 weight copy
    def time_prefill(weights):
        pt = prompt_tokens(spec, args.prefill_tokens)
        m.prefill(pt, 0)  # warm-up (allocates the workspace)
        torch.cuda.synchronize()
        barrier(world)
        reps = 3
        ev0.record(stream)
        for _ in range(reps):
            m.prefill(pt, 0)
        ev1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        pms = max_over_ranks(ev0.elapsed_time(ev1) / reps, world)
        tpk, tsrc = tensor_peak()
        fl = prefill_flops(c, len(pt))
        return {"tokens": len(pt), "value": round(len(pt) / (pms / 1e3), 1), "unit": "tok/s",
                "ms": round(pms, 3), "tflops": round(fl / (pms / 1e3) / 1e12, 1),
                "frac_of_tensor_peak": round(fl / (pms / 1e3) / 1e12 / tpk, 4), "peak_source": tsrc,
                "weights": weights,
                "how": "gb_model_prefill from host token ids: tcgen05 GEMMs (binary16 operands, f32 accumulate) "
                       "+ tensor-core causal attention, last token through the decode step; under tensor "
                       "parallelism the o/down partials summed by NCCL all-reduces; CUDA events, "
                       f"mean of {reps}, max over ranks"}

    def time_engine(weights, batch):
        e = gb.Engine(m, page_size=64, n_pages=batch * 4, max_batch=batch)
        ids = [e.add() for _ in range(batch)]
        btoks = prompt_tokens(spec, batch)
        for _ in range(4):  # warm-up: positions 0..3 of every sequence
            _, btoks = e.step(ids, btoks, logits=False)
        torch.cuda.synchronize()
        nsteps = 32
        w0 = time.perf_counter()
        ev0.record(stream)
        for _ in range(nsteps):
            _, btoks = e.step(ids, btoks, logits=False)
        ev1.record(stream)
        torch.cuda.synchronize()
        wall = time.perf_counter() - w0
        bms = ev0.elapsed_time(ev1) / nsteps
        e.close()
        return {"batch": batch, "value": round(batch * nsteps / (bms * nsteps / 1e3), 1), "unit": "tok/s",
                "ms_per_step": round(bms, 3), "e2e_tok_s": round(batch * nsteps / wall, 1),
                "positions": f"4..{4 + nsteps - 1}", "weights": weights,
                "how": "gb_engine_step: B sequences one token each per step through the tensor-core GEMMs and the "
                       "paged attention, replayed from a CUDA graph; value = CUDA events around 32 steps, each "
                       "synchronous (ids in, next tokens out, status check), e2e = wall clock of the same loop"}

    def time_engine_prompt(weights):
        # a prompt fed to the engine as the rows of one step (chunked prefill
        # into the paged cache), next to nothing else
        T = min(args.prefill_tokens, 512)
        e = gb.Engine(m, page_size=64, n_pages=(T + 63) // 64 + 1, max_batch=T)
        pt = prompt_tokens(spec, T)
        for _ in range(2):  # warm-up (captures the step's graph)
            sid = e.add()
            e.step([sid] * T, pt, logits=False)
            e.release(sid)
        torch.cuda.synchronize()
        reps, tot = 3, 0.0
        for _ in range(reps):
            sid = e.add()
            ev0.record(stream)
            e.step([sid] * T, pt, logits=False)
            ev1.record(stream)
            torch.cuda.synchronize()
            tot += ev0.elapsed_time(ev1)
            e.release(sid)
        e.close()
        pms = tot / reps
        return {"tokens": T, "value": round(T / (pms / 1e3), 1), "unit": "tok/s", "ms": round(pms, 3),
                "weights": weights,
                "how": "gb_engine_step with one sequence listed T times (its prompt at positions 0..T-1 in one "
                       "step: the batched GEMMs, paged RoPE/KV append, paged attention per row); CUDA events, "
                       f"mean of {reps}"}

    prefill = time_prefill("quantized, decoded per call") if args.prefill_tokens > 1 else None
    batched = time_engine("quantized, decoded per call", args.batch) if world == 1 and args.batch > 1 else None
    prefill16 = batched16 = prompt16 = None
    if args.prefill_tokens > 1 or (world == 1 and args.batch > 1):
        try:
            w16 = m.cache_f16_weights()
        except gb.GollamaError as exc:  # not enough device memory: reported, not measured
            w16 = str(exc)
        if isinstance(w16, int):
            what = f"binary16 copy ({w16 / 1e9:.2f} GB, gb_model_cache_f16_weights), read by TMA"
            prefill16 = time_prefill(what) if args.prefill_tokens > 1 else None
            batched16 = ([time_engine(what, b) for b in sorted({8, args.batch})]
                         if world == 1 and args.batch > 1 else None)
            prompt16 = time_engine_prompt(what) if world == 1 and args.prefill_tokens > 1 else None
        else:
            prefill16 = batched16 = prompt16 = {"unavailable": w16}

    sweep = gemv_sweep(gb, torch, local, peaks()[0]) if world == 1 and not args.no_sweep else None
    configs = {}
    for name in [n for n in args.configs.split(",") if n and n != args.config]:
        configs[name] = measure_config(gb, torch, name, world, rank, local)

    result = {
        "metric": METRIC, "value": round(tok_s, 2), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "q4_k/q6_k/q4_0 weights x int8-limb activations (dp4a), f32 accumulate",
        "data": "synthetic: seeded random-init weights" + (", KV prefilled with seeded N(0,1) fp16" if cfg["prefill"] else ""),
        "config": bench_config(cfg, spec, world),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": ncu_traffic(args.config) if world == 1 else None,
                     "traffic_source": "static: profiles/traffic.json (one earlier ncu capture), not this run",
                     "kernel": "gemv_kernel, gate/up + SwiGLU (one launch per layer)",
                     "bytes_per_launch": gu_bytes, "avg_launch_ms": round(gu_ms, 5), "peak_source": peak_src,
                     "timing": "CUDA events around each gate/up launch of an eager decode step (median of 5 steps); "
                               "in eager mode every launch runs alone, without the overlap of the graph's "
                               "programmatic dependent launches"},
        "step_roofline": {"bytes_per_token": bytes_tok, "achieved_gbs": round(bytes_tok * tok_s / 1e9, 1),
                          "frac": round(bytes_tok * tok_s / 1e9 / peak, 4),
                          "roofline_tok_s": round(peak * 1e9 / bytes_tok, 1)},
        "kernel_ms_per_step": dict(breakdown, how="CUDA events between the launches of one eager decode step: "
                                   "launches serialized (no PDL overlap), so the classes add up to more than "
                                   "ms_per_step"),
        "prefill": prefill, "prefill_f16w": prefill16,
        "batched_decode": batched, "batched_decode_f16w": batched16, "engine_prompt_f16w": prompt16,
        "gemv_sweep": sweep,
        "configs": configs or None,
        "e2e": e2e,
        "gpu_launches": m.launches_per_step() * args.steps,
        "clocks": clk,
        "first_tokens": [int(t) for t in toks_out[:8]],
    }
    # logits of the first timed position for the oracle check (every rank takes part)
    plog = m.forward(t0, p0).copy() if rank == 0 else m.forward_no_logits(t0, p0)
    m.close()
    if rank == 0:
        om = oracle_model(image_bytes(src), spec, cfg)
        result["parity"] = parity_check(om, plog, t0, p0, spec.vocab)
        if world == 1 and not args.no_cpu_baseline:
            result["cpu_baseline"] = cpu_baseline(om, spec, p0, t0)
        om.close()
        print(json.dumps(result), flush=True)


def model_bytes(spec, kv_len, kv_f16):
    """Algorithmic HBM bytes of one decode step of the whole (unsharded) model at
    kv_len cached positions: every weight matrix once, the norms, the K/V read
    and the new K/V row, the embedding row (the arithmetic of gb_model_step_bytes
    at one GPU)."""
    bs = {2: (32, 18), 8: (32, 34), 12: (256, 144), 13: (256, 176), 14: (256, 210), 1: (1, 2), 0: (1, 4)}

    def rb(t, n):
        return n // bs[t][0] * bs[t][1]

    def qt(six):
        m = spec.mix
        return {0: 2, 2: 12, 3: 14, 4: 8, 5: 1}.get(m, (14 if six else (13 if m == 6 else 12)))

    q, kv = spec.heads * spec.head_dim, spec.kv_heads * spec.head_dim
    w = 0
    for i in range(spec.layers):
        w += (q + kv) * rb(qt(False), spec.dim) + kv * rb(qt(True), spec.dim) + spec.dim * rb(qt(False), q)
        w += 2 * spec.ffn * rb(qt(False), spec.dim) + spec.dim * rb(qt(i % 2 == 0), spec.ffn)
    w += spec.vocab * rb(qt(spec.mix != 0), spec.dim)
    norms = 4 * spec.dim * (2 * spec.layers + 1)
    esz = 2 if kv_f16 else 4
    kvb = spec.layers * kv_len * 2 * kv * esz + spec.layers * 2 * kv * esz
    return w + norms + kvb + rb(qt(False), spec.dim)


def bench_config(cfg, spec, world):
    """The `config` object of the JSON line (the same for both arms)."""
    kv_len = cfg["prefill"] + cfg["prompt"] + cfg["window"] // 2
    gb_tok = model_bytes(spec, kv_len, cfg["kv_f16"]) / 1e9
    return {"workload": cfg["workload"],
            "model": f"preset {cfg['preset']} (dim {spec.dim}, {spec.layers} layers, {spec.heads}/{spec.kv_heads} "
                     f"heads, ffn {spec.ffn}, vocab {spec.vocab})",
            "global_batch": 1, "seq_len": cfg["max_len"], "parallelism": f"tp{world}",
            "l2": f"inputs larger than L2: {gb_tok:.2f} GB of weights and KV read per token vs 126 MB L2"}


def _orc():
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_lib as orc

    return orc


def oracle_model(raw, spec, cfg):
    """The C restatement of the reference's backend/cpu forward over the bench's
    image, with the same KV prefill and prompt (oracle library only)."""
    orc = _orc()
    om = orc.OracleModel(raw, cfg["max_len"], bool(cfg["kv_f16"]))
    kv_dim = spec.kv_heads * spec.head_dim
    if cfg["prefill"]:
        for layer in range(spec.layers):
            k, v = orc.synth_kv_normal(KV_SEED, layer, 0, cfg["prefill"], kv_dim, bool(cfg["kv_f16"]))
            om.set_kv(layer, 0, k, v)
    toks = prompt_tokens(spec, cfg["prompt"] + 1)
    for pos in range(cfg["prompt"]):
        om.forward(toks[pos], pos, spec.vocab)
    return om


def image_bytes(src):
    """The GGUF bytes of the bench's model: an in-memory image or a file."""
    if isinstance(src, str):
        return np.fromfile(src, np.uint8)
    return src.view()


def parity_check(om, logits, t0, p0, vocab):
    """One decode step of the oracle against the device step's logits, with the
    bars of the parity tests: |got - want| <= 1e-3 + 1e-4 |want|, greedy token
    equal unless the oracle's top two logits are within 1e-3."""
    orc = _orc()
    want = om.forward(t0, p0, vocab).astype(np.float64)
    got = np.asarray(logits, np.float64)
    err = np.abs(got - want)
    top2 = np.sort(want)[-2:]
    tok_ref, tok = orc.argmax(want.astype(np.float32)), orc.argmax(np.asarray(logits, np.float32))
    return {"position": p0, "max_abs": float(err.max()), "max_rel": float((err / np.maximum(np.abs(want), 1e-30)).max()),
            "max_excess_over_bar": float((err - 1e-4 * np.abs(want)).max()),
            "within_1e-3_abs_1e-4_rel": bool((err <= 1e-3 + 1e-4 * np.abs(want)).all()),
            "token": int(tok), "token_oracle": int(tok_ref), "token_match": bool(tok == tok_ref),
            "near_tie": bool(top2[1] - top2[0] < 1e-3),
            "how": "one oracle step (C restatement of cpuForward) on the bench's image, KV and prompt"}


def cpu_baseline(om, spec, p0, t0):
    cores = os.cpu_count() or 1
    t = time.perf_counter()
    om.forward(t0, p0, spec.vocab, threads=1)
    t1 = time.perf_counter() - t
    t = time.perf_counter()
    om.forward(t0, p0, spec.vocab, threads=cores)
    tn = time.perf_counter() - t
    return {"value": round(1 / t1, 4), "unit": "tok/s", "cores": 1, "kind": "port",
            "sample": f"1 decode token at position {p0} of the bench workload, C restatement of backend/cpu "
                      "+ cpuForward, single thread (the reference's Go path is single-threaded)",
            "all_cores": {"value": round(1 / tn, 3), "cores": cores}}


def run_reference(args, cfg, world, rank):
    """The reference's CPU path (backend/cpu + cpuForward restated in C: Go is not on
    this image), all host threads, rank 0 only. Each step is one decode token of the
    same workload. Only the oracle library is loaded: it builds the same synthetic
    image (oracle/synth.c) and picks tokens with model.Argmax's rule."""
    if rank != 0:
        return
    orc = _orc()
    spec = orc.synth_preset(cfg["preset"], seed=SEED)
    if cfg.get("layers"):
        spec.layers = cfg["layers"]
    raw = orc.synth_model(spec)
    p0 = cfg["prefill"] + cfg["prompt"]
    toks = prompt_tokens(spec, cfg["prompt"] + 1)
    om = oracle_model(raw, spec, cfg)
    cores = os.cpu_count() or 1
    window = cfg["window"]
    tok = toks[-1]
    for i in range(args.warmup):
        tok = orc.argmax(om.forward(tok, p0 + i % window, spec.vocab, threads=cores))
    t = time.perf_counter()
    tok = toks[-1]
    for i in range(args.steps):
        logits = om.forward(tok, p0 + i % window, spec.vocab, threads=cores)
        tok = orc.argmax(logits)
    wall = time.perf_counter() - t
    om.close()
    v = args.steps / wall
    sample = (f"{args.steps} decode tokens of the bench workload ({cfg['workload']}), C restatement of "
              f"backend/cpu + cpuForward, {cores} host threads")
    print(json.dumps({"metric": METRIC, "value": round(v, 4), "unit": "tok/s", "n_gpus": world,
                      "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(wall / args.steps * 1e3, 3),
                      "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "impl": "reference",
                      "dtype": "f32 weights dequantized per token, f64 accumulate",
                      "data": "synthetic: seeded random-init weights" + (", KV prefilled with seeded N(0,1) fp16" if cfg["prefill"] else ""),
                      "config": bench_config(cfg, spec, world), "host_threads": cores,
                      "cpu_baseline": {"value": round(v, 4), "unit": "tok/s", "cores": cores, "kind": "port",
                                       "sample": sample},
                      "e2e": {"value": round(v, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
          flush=True)


def profile_batched(args, cfg):
    """One engine step (or prefill) of the config's model, with its binary16
    weight copy, after warm-up, between cudaProfilerStart/Stop: the launch list
    and kernel captures of the batched paths. The engine runs without its
    CUDA graphs (use_graph=0), so that ncu sees plain kernel launches. Prints
    the wall time of the warm steps (not a bench line)."""
    import torch

    import gollama_b200 as gb

    src, spec = build_image(gb, cfg, 1, 0)
    m = gb.Model(src, device=0, max_len=max(1024, args.profile_prefill + 1), kv_f16=1, use_graph=0)
    m.cache_f16_weights()
    if args.profile_engine:
        B = args.profile_engine
        e = gb.Engine(m, page_size=64, n_pages=B * 4, max_batch=B)
        ids = [e.add() for _ in range(B)]
        toks = prompt_tokens(spec, B)
        for _ in range(4):
            _, toks = e.step(ids, toks, logits=False)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(8):
            _, toks = e.step(ids, toks, logits=False)
        ms = (time.perf_counter() - t0) / 8 * 1e3
        torch.cuda.profiler.start()
        e.step(ids, toks, logits=False)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        e.close()
        print(json.dumps({"profile": "engine step", "batch": B, "layers": spec.layers, "ms_per_step_wall": round(ms, 3)}))
    else:
        pt = prompt_tokens(spec, args.profile_prefill)
        for _ in range(2):
            m.prefill(pt, 0)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        m.prefill(pt, 0)
        ms = (time.perf_counter() - t0) * 1e3
        torch.cuda.profiler.start()
        m.prefill(pt, 0)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        print(json.dumps({"profile": "prefill", "tokens": len(pt), "layers": spec.layers, "ms_wall": round(ms, 3)}))
    m.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--config", default="8b", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=64,
                    help="sequences per step of the continuous-batching measurement (0 = skip)")
    ap.add_argument("--prefill-tokens", type=int, default=512,
                    help="prompt length of the batched-prefill measurement (0 = skip)")
    ap.add_argument("--no-sweep", action="store_true", help="skip the standalone GEMV sweep (config 2)")
    ap.add_argument("--configs", default="1b,3b,70b",
                    help="more decode configurations measured after the main one ('' = none)")
    ap.add_argument("--sweep-only", default=None, metavar="TYPES:SHAPES",
                    help="run only the GEMV sweep, e.g. q4_k:14336x4096 or all:all (profiling captures)")
    ap.add_argument("--layers", type=int, default=0,
                    help="truncate the model to this many layers (small ncu captures only; not a bench line)")
    ap.add_argument("--profile-engine", type=int, default=0, metavar="B",
                    help="one engine step of B sequences through the binary16 weight copy between "
                         "cudaProfilerStart/Stop (ncu --profile-from-start off); not a bench line")
    ap.add_argument("--profile-prefill", type=int, default=0, metavar="T",
                    help="one T-token prefill through the binary16 weight copy between cudaProfilerStart/Stop")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    cfg = dict(CONFIGS[args.config])
    if args.layers:
        cfg["layers"] = args.layers
        cfg["workload"] += f" [truncated to {args.layers} layers for profiling]"
    if args.profile_engine or args.profile_prefill:
        profile_batched(args, cfg)
        return
    if args.sweep_only:
        import torch

        import gollama_b200 as gb

        t, _, sh = args.sweep_only.partition(":")
        sweep = gemv_sweep(gb, torch, 0, peaks()[0], types=None if t == "all" else t.split(","),
                           shapes=None if sh in ("", "all") else sh.split(","))
        print(json.dumps({"gemv_sweep": sweep}), flush=True)
        return
    world, rank, local = dist_setup()
    try:
        if args.impl == "reference":
            run_reference(args, cfg, world, rank)
        else:
            run_ours(args, cfg, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
