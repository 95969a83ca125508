"""Benchmark of the quantized-weight hot path on B200.

Headline (`value`): fused Q4_0 dequant+GEMV, batch-1 decode shape 4096x4096
(W ~ N(0,0.02) seed 2, x ~ N(0,1) seed 3), in HBM GB/s of algorithmic bytes
(W blocks 9,437,184 B + x 16,384 B + y 16,384 B per GEMV).  One step = one
sweep of batch-1 GEMVs over a rotating set of 64 distinct weight copies
(606 MB, > 4x L2), so every GEMV streams its weights from HBM.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference] [--quick]

Under torchrun each rank runs the same per-GPU work on its own GPU (replicas:
the 4096x4096 GEMV does not shard) and rank 0 prints one JSON line with the
whole-job value over the max-over-ranks device time.  `--impl reference`
times the reference's own CPU implementation (its AVX-512 gemv_4bit_into,
restated in C) on the host cores instead.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "fused Q4 GEMV & dequant HBM GB/s (% of 8 TB/s); 8B-shape decode tokens/s"
ROWS = COLS = 4096
N_COPIES = 64
GEMV_BYTES = ROWS * (COLS // 32) * 18 + COLS * 4 + ROWS * 4  # 9,469,952
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0
PROFILE_GEMV = os.path.join(ROOT, "profiles", "gemv_q4_0_4096x4096_batch1.md")


def ncu_traffic_per_launch():
    """dram__bytes_read.sum + dram__bytes_write.sum of one headline GEMV launch,
    as the ncu summary of this kernel records it ("traffic_bytes_per_launch:"),
    or None when no capture is recorded."""
    import re
    try:
        m = re.search(r"traffic_bytes_per_launch:\s*([0-9,]+)", open(PROFILE_GEMV).read())
        return int(m.group(1).replace(",", "")) if m else None
    except OSError:
        return None


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self._t.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU legs (the reference's own algorithm, restated in C under oracle/)
# ---------------------------------------------------------------------------

def cpu_gemv_setup(n_copies: int):
    """Engine-format copies of the benchmark weight (same values as the Q4_0
    blocks: f32 scale = f16 d, identical nibbles), for the reference's
    gemv_4bit_into (f32 scales, linear nibbles)."""
    from oracle import oracle as O
    rng = np.random.default_rng(2)
    w = (rng.standard_normal(ROWS * COLS) * 0.02).astype(np.float32)
    blocks = O.quantize_q4_0(w).reshape(-1, 18)
    scales = blocks[:, :2].copy().view(np.float16).astype(np.float32).ravel()
    packed = np.ascontiguousarray(blocks[:, 2:]).ravel()
    x = np.random.default_rng(3).standard_normal(COLS).astype(np.float32)
    copies = [(scales.copy(), packed.copy()) for _ in range(n_copies)]
    return O, copies, x


def cpu_threads():
    return max(1, min(os.cpu_count() or 1, 32))  # inference/math.rs:275 caps at 32


def time_cpu_gemv(seconds: float = 8.0, n_copies: int = 32):
    O, copies, x = cpu_gemv_setup(n_copies)
    out = np.empty(ROWS, np.float32)
    nt = cpu_threads()
    for s, p in copies[:2]:
        O.avx_gemv_4bit_into(out, s, p, x, ROWS, COLS, nt)
    n = 0
    t0 = time.perf_counter()
    while True:
        s, p = copies[n % n_copies]
        O.avx_gemv_4bit_into(out, s, p, x, ROWS, COLS, nt)
        n += 1
        if n % n_copies == 0 and time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    # single-thread scalar worker, as benches/dequant_bench.rs also times
    t1 = time.perf_counter()
    s, p = copies[0]
    O.lib().or_gemv_4bit_worker_scalar(out, s, p, x, 0, ROWS, COLS, 32)
    dt1 = time.perf_counter() - t1
    return {"value": n * GEMV_BYTES / dt / 1e9, "unit": "GB/s", "cores": nt, "kind": "port",
            "sample": f"{n} AVX-512 gemv_4bit_into calls (math.rs:255-380 restated) over {n_copies} rotating "
                      f"4096x4096 copies, {dt:.1f} s; GB/s counts the same {GEMV_BYTES} algorithmic bytes per GEMV",
            "scalar_1thread_gbs": GEMV_BYTES / dt1 / 1e9}


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    O, copies, x = cpu_gemv_setup(N_COPIES if args.steps >= N_COPIES else max(2, args.steps))
    nc = len(copies)
    out = np.empty(ROWS, np.float32)
    nt = cpu_threads()
    for i in range(args.warmup):
        s, p = copies[i % nc]
        O.avx_gemv_4bit_into(out, s, p, x, ROWS, COLS, nt)
    t0 = time.perf_counter()
    for i in range(args.steps):
        s, p = copies[i % nc]
        O.avx_gemv_4bit_into(out, s, p, x, ROWS, COLS, nt)
    dt = time.perf_counter() - t0
    v = args.steps * GEMV_BYTES / dt / 1e9
    line = {"metric": METRIC, "value": round(v, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": "Q4_0 fused dequant+GEMV 4096x4096 batch 1 (one GEMV per step on CPU)",
                       "rows": ROWS, "cols": COLS, "batch": 1, "rotating_copies": nc},
            "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": nt, "kind": "port",
                             "sample": f"{args.steps} AVX-512 gemv_4bit_into calls (inference/math.rs:255-380 "
                                       f"restated in C, thread spawn per call as in the reference)"},
            "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# GPU leg
# ---------------------------------------------------------------------------

def run_gpu(args):
    import torch
    rank, world, local = dist_env()
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=__import__("datetime").timedelta(seconds=120))
    else:
        torch.cuda.set_device(0)
    dev = torch.device("cuda", torch.cuda.current_device())
    from agent_harness_b200 import _lib
    from agent_harness_b200 import kernels as K
    _lib.check(_lib.lib().ah_device_init(dev.index))

    # --- inputs (resident in HBM before timing) ---
    blocks = K.synth_q4_0(ROWS, COLS, 0.02, 2, device=dev)
    Ws = [K.Q4Weight.from_q4_0(blocks, ROWS, COLS) for _ in range(N_COPIES)]
    del blocks
    x = K.fill_normal(COLS, 0.0, 1.0, 3, device=dev)
    y = torch.empty(ROWS, dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def sweep():
        for W in Ws:
            W.gemv(x, out=y)

    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            sweep()
    torch.cuda.synchronize()
    # capture `chunk` steps per graph (the weights do not change between steps)
    chunk = next(c for c in (16, 10, 8, 5, 4, 2, 1) if args.steps % c == 0)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for _ in range(chunk):
            sweep()
    with torch.cuda.stream(stream):
        g.replay()
    torch.cuda.synchronize()

    sampler = ClockSampler(dev.index)
    sampler.start()
    time.sleep(0.3)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(args.steps // chunk):
            g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    launches = args.steps * N_COPIES
    per_launch_s = ms / 1e3 / launches
    value = world * args.steps * N_COPIES * GEMV_BYTES / (ms / 1e3) / 1e9
    achieved = GEMV_BYTES / per_launch_s / 1e9
    peak, peak_kind = peaks()

    # correctness spot check of the timed kernel's output (cheap, outside timing)
    ok = bool(torch.isfinite(y).all().item())

    # --- end to end through the C-ABI with host buffers, per GEMV: the
    # gemv_4bit_into calling convention (host x in, host y out, synchronous)
    # on resident weights: ah_q4w_gemv_host copies x in, runs the GEMV, copies
    # y out and waits, all inside the timed region ---
    x_host = torch.empty(COLS, dtype=torch.float32).pin_memory()
    x_host.copy_(x.cpu())
    y_host = torch.empty(ROWS, dtype=torch.float32).pin_memory()
    e2e_steps = max(1, min(args.steps, 200))
    gemv_host = _lib.lib().ah_q4w_gemv_host
    xp, yp, sp = C.c_void_p(x_host.data_ptr()), C.c_void_p(y_host.data_ptr()), C.c_void_p(stream.cuda_stream)
    handles = [W.handle for W in Ws]
    for h in handles:  # first call per weight allocates its staging: keep it untimed
        _lib.check(gemv_host(h, xp, yp, 1, sp))
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        for h in handles:
            rc = gemv_host(h, xp, yp, 1, sp)
            if rc != 0:
                _lib.check(rc)
    e2e_dt = time.perf_counter() - t0
    e2e_ok = bool(np.isfinite(y_host.numpy()).all())
    e2e_val = world * e2e_steps * N_COPIES * GEMV_BYTES / e2e_dt / 1e9
    if world > 1:
        t = torch.tensor([e2e_dt], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_val = world * e2e_steps * N_COPIES * GEMV_BYTES / float(t.item()) / 1e9

    for W in Ws:
        W.close()
    Ws = []
    extra = {}
    if rank == 0 and not args.quick:
        extra = secondary_measurements(K, dev, stream, peak, no_cpu=args.no_cpu)
        extra["prefill_gemm"] = prefill_gemm(K, dev, cpu_tokens=0 if args.no_cpu else 8)
    if not args.quick and not args.no_decode:
        dec = decode_8b(dev, args.decode_prompt, args.decode_new)
        if world > 1:
            t = torch.tensor([dec["ms_per_token"]], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            dec["tokens_per_s_all_replicas"] = round(world * 1e3 / float(t.item()), 2)
        extra["decode_8b"] = dec
    if not args.quick and not args.no_tp:
        extra["decode_70b_tp"] = decode_70b_tp(dev, rank, world, args.tp_prompt, args.tp_new,
                                               allreduce=args.tp_allreduce)
    if rank == 0 and not args.no_cpu and not args.quick:
        if "decode_8b" in extra:
            sh8 = [(4096, 4096), (1024, 4096), (1024, 4096), (4096, 4096), (14336, 4096), (14336, 4096),
                   (4096, 14336)]
            step, nt, layer = cpu_decode_baseline(sh8, 32, (128256, 4096), 1)
            extra["decode_8b"]["cpu_baseline"] = {
                "value": round(1.0 / step, 3), "unit": "tokens/s", "cores": nt, "kind": "port",
                "sample": f"extrapolated: one layer's 7 projection GEMVs ({layer * 1e3:.1f} ms) x 32 + the LM head "
                          "through the AVX-512 gemv_4bit_into restatement (the engine forward's weight streaming, "
                          "inference/mod.rs:411-538); attention and norms not included"}
        if "decode_70b_tp" in extra:
            sh70 = [(8192, 8192), (1024, 8192), (1024, 8192), (8192, 8192), (28672, 8192), (28672, 8192),
                    (8192, 28672)]
            step, nt, layer = cpu_decode_baseline(sh70, 80, (128256, 8192), TP_BATCH)
            extra["decode_70b_tp"]["cpu_baseline"] = {
                "value": round(TP_BATCH / step, 4), "unit": "tokens/s", "cores": nt, "kind": "port",
                "sample": f"extrapolated: one layer's 7 projection GEMVs ({layer * 1e3:.1f} ms per token) x 80 + "
                          f"the LM head, x {TP_BATCH} sequences, through the AVX-512 gemv_4bit_into restatement "
                          "(the reference decodes one token per forward); attention and norms not included"}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = time_cpu_gemv(seconds=args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "q4_0 x f32 (f16-split tensor-core, f32 accumulate)",
            "data": "synthetic (seeded counter-based N(0,1) generator; weights N(0,0.02) seed 2, x seed 3)",
            "config": {"workload": "Q4_0 fused dequant+GEMV 4096x4096 batch 1", "rows": ROWS, "cols": COLS,
                       "batch": 1, "rotating_copies": N_COPIES, "gemvs_per_step": N_COPIES,
                       "l2": "inputs larger than L2: each step streams 64 distinct weight copies (606 MB)",
                       "bytes_per_gemv": GEMV_BYTES, "graph_steps_per_replay": chunk,
                       "parallelism": f"replicas x{world}"},
            "pct_of_8tbs": round(100.0 * achieved / NOMINAL_HBM_GBS, 2),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                         "traffic": ncu_traffic_per_launch(),
                         "traffic_source": "profiles/gemv_q4_0_4096x4096_batch1.md (ncu, this kernel)",
                         "kernel": "k_gemv_q4<1,false,0,0>", "bytes_per_launch": GEMV_BYTES,
                         "avg_launch_us": round(per_launch_s * 1e6, 4)},
            "e2e": {"value": round(e2e_val, 3), "unit": "GB/s", "h2d_bytes_per_step": N_COPIES * COLS * 4,
                    "d2h_bytes_per_step": N_COPIES * ROWS * 4,
                    "path": "ah_q4w_gemv_host per GEMV: pinned x H2D, GEMV, y D2H, stream sync in one C-ABI call; weights "
                            "resident from load"},
            "gpu_launches": launches,
            "clocks": clocks,
            "output_finite": ok and e2e_ok,
        }
        if cpu is not None:
            line["cpu_baseline"] = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
            line["cpu_baseline"]["value"] = round(cpu["value"], 3)
            line["cpu_scalar_1thread_gbs"] = round(cpu["scalar_1thread_gbs"], 3)
        line.update(extra)
        print(json.dumps(line), flush=True)
    for W in Ws:
        W.close()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


DECODE_PROMPT, DECODE_NEW = 2048, 256
DECODE_BYTES_PER_TOKEN_WEIGHTS = 4221370368  # all Q4_0 projections + LM head of the 8B shape
DECODE_PROJ_WEIGHTS = 32 * (4096 * 6144 + 4096 * 4096 + 3 * 14336 * 4096)  # per token, without the LM head


TP_PROMPT, TP_NEW, TP_BATCH = 2048, 128, 16
# all Q4_0 projections + LM head of the 70B shape (80 x (q 8192^2 + k,v 1024x8192
# + o 8192^2 + gate,up,down 3 x 28672x8192) + 128256x8192) x 18/32 bytes
DECODE70_WEIGHT_BYTES = 39094714368


def decode70_weight_bytes(n_layer):
    """Q4_0 bytes (18 per 32 weights) one 70B-shape decode step streams: the
    q|k|v, o, gate|up and down projections of n_layer layers plus the LM head."""
    d, ff, kv, vocab = 8192, 28672, 1024, 128256
    per_layer = d * (d + 2 * kv) + d * d + 2 * ff * d + d * ff
    return (per_layer * n_layer + vocab * d) * 18 // 32


def cpu_decode_baseline(layer_shapes, n_layer, head_shape, tokens, min_s=0.3):
    """The reference's decode on the host cores: its engine forward spends its
    time in gemv_4bit_into (the AVX-512 worker, inference/math.rs:255-380) once
    per projection, layer and token.  Each projection shape of one layer and the
    LM head is timed on engine-format weights (random bytes: the timing does
    not depend on the values); the step is layer x n_layer + head, times the
    tokens of a step.  Attention, norms and sampling are left out (they are a
    few per cent of the weight streaming at these shapes), so this is an
    extrapolated lower bound on the reference's step time."""
    from oracle import oracle as O
    rng = np.random.default_rng(0)
    nt = cpu_threads()
    per = {}
    for rows, cols in list(layer_shapes) + [head_shape]:
        if (rows, cols) in per:
            continue
        sc = (rng.random(rows * cols // 32) * 0.004).astype(np.float32)
        pk = rng.integers(0, 256, rows * cols // 2, dtype=np.uint8)
        x = rng.standard_normal(cols).astype(np.float32)
        y = np.empty(rows, np.float32)
        per[(rows, cols)] = _cpu_seconds(lambda: O.avx_gemv_4bit_into(y, sc, pk, x, rows, cols, nt), min_s=min_s,
                                         max_calls=10)
    layer = sum(per[sh] for sh in layer_shapes)
    step = (layer * n_layer + per[head_shape]) * tokens
    return step, nt, layer


def decode_70b_tp(dev, rank, world, n_prompt=TP_PROMPT, n_new=TP_NEW, batch=TP_BATCH, allreduce="peer", n_layer=None):
    """70B-shape greedy decode, batch 16, tensor-parallel over the job's ranks
    (80 layers, d 8192, FFN 28672, 64/8 heads x 128, vocab 128256; Q4_0
    N(0,0.02) seed 8; prompts of uniform ids seed 9).  Decode steps are timed
    with CUDA events on every rank; the max over ranks is reported."""
    import torch
    from agent_harness_b200.model import LLAMA_70B, Model, ModelConfig, nccl_unique_id
    cfg = ModelConfig(**{**LLAMA_70B.__dict__, "max_seq": n_prompt + n_new + 8, "max_batch": batch,
                         "n_layer": n_layer or LLAMA_70B.n_layer})
    nid = None
    if world > 1:
        import torch.distributed as dist
        obj = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nid = obj[0]
    m = Model(cfg, device=dev, tp_rank=rank, tp_world=world, nccl_id=nid)
    m.init_random(8, w_std=0.02, emb_std=1.0, norm_std=0.02)
    if world > 1 and allreduce == "peer":
        import torch.distributed as dist

        def allgather(blob):
            out = [None] * world
            dist.all_gather_object(out, blob)
            return out
        m.enable_peer_allreduce(allgather)
    prompt = np.random.default_rng(9).integers(0, cfg.vocab_size, (batch, n_prompt)).astype(np.int32)
    t0 = time.perf_counter()
    m.generate(prompt, 1)  # prompt through the prefill GEMMs + first token
    prefill_s = time.perf_counter() - t0
    st = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    toks = m.decode(n_new + 1, batch)
    e1.record(st)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms, prefill_s * 1e3], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms, prefill_s = float(t[0].item()), float(t[1].item()) / 1e3
    first = toks[1, :4].cpu().numpy().tolist()
    m.close()
    per_step = ms / 1e3 / n_new
    split = {}
    if world > 1:
        # the step's collective alone: 2 all-reduces per layer of the block
        # output [batch, d_model] f32 (NCCL), timed on the device, max over ranks
        import torch.distributed as dist
        buf = torch.zeros(batch, cfg.n_embd, device=dev)
        for _ in range(20):
            dist.all_reduce(buf)
        torch.cuda.synchronize(dev)
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(st)
        for _ in range(2 * cfg.n_layer):
            dist.all_reduce(buf)
        c1.record(st)
        torch.cuda.synchronize(dev)
        t = torch.tensor([c0.elapsed_time(c1)], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        split = {"allreduce_alone_ms_per_step": round(float(t.item()), 3),
                 "allreduce_note": f"{2 * cfg.n_layer} ncclAllReduce of [{batch}, {cfg.n_embd}] f32 timed alone; "
                                   "the rest of the step streams weights"}
    return {"tokens_per_s": round(batch * n_new / (ms / 1e3), 1), "ms_per_step": round(per_step * 1e3, 3),
            "batch": batch, "n_prompt": n_prompt, "n_new": n_new, "tp": world, "n_layer": cfg.n_layer,
            "block_allreduce": (allreduce if world > 1 else "none"),
            "weight_gbs_per_gpu": round(decode70_weight_bytes(cfg.n_layer) / world / per_step / 1e9, 1),
            "prefill_tokens_per_s": round(batch * (n_prompt - 1) / prefill_s, 1),
            "prefill_s": round(prefill_s, 2),
            "first_tokens_seq0_3": first, **split,
            "note": "tensor parallel over the job's ranks: row/column-sharded projections, one all-reduce per "
                    "attention/MLP block (peer: GEMV epilogue stores into every rank's slots over NVLink + flag; "
                    "nccl: ncclAllReduce), argmax-candidate all-gather; steps replayed as CUDA graphs"}


def decode_8b(dev, n_prompt=DECODE_PROMPT, n_new=DECODE_NEW, n_layer=None):
    """8B-shape greedy decode, batch 1: 32 layers, d 4096, FFN 14336, 32/8 heads
    x 128, vocab 128256, theta 5e5; Q4_0 projections N(0,0.02) seed 6, f16
    embeddings/norms, f16 KV; prompt of uniform token ids (seed 7)."""
    import torch
    from agent_harness_b200.model import LLAMA_8B, Model
    from agent_harness_b200.model import ModelConfig
    cfg = ModelConfig(**{**LLAMA_8B.__dict__, "max_seq": max(n_prompt, 256) + n_new + 16,
                         "n_layer": n_layer or LLAMA_8B.n_layer})
    m = Model(cfg, device=dev)
    m.init_random(6, w_std=0.02, emb_std=1.0, norm_std=0.02)
    prompt = np.random.default_rng(7).integers(0, cfg.vocab_size, (1, n_prompt)).astype(np.int32)
    first = m.generate(prompt[:, :64], 1)  # warm-up: buffers, graphs
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    first = m.generate(prompt, 1)  # prompt through the prefill GEMMs + first token
    prefill_s = time.perf_counter() - t0
    st = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    toks = m.decode(n_new + 1, 1)  # n_new full decode steps after the first token
    e1.record(st)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1)
    tk = toks.cpu().numpy().ravel()
    # replay check: the same prompt decodes to the same tokens; and the GEMM
    # prefill agrees with the reference's token-by-token prefill on a prefix
    again = m.generate(prompt[:, :256], 8)
    again2 = m.generate(prompt[:, :256], 8)
    m.set_prefill(0)
    t1 = time.perf_counter()
    tokwise = m.generate(prompt[:, :256], 8)
    tok_s = time.perf_counter() - t1
    m.set_prefill(1)
    # the same decode with temperature 0.8 + top-k 40 sampling in place of the argmax
    m.set_sampling(0.8, 40, 1)
    m.generate(prompt, 1)
    e0.record(st)
    m.decode(n_new + 1, 1)
    e1.record(st)
    torch.cuda.synchronize(dev)
    ms_sampled = e0.elapsed_time(e1)
    m.set_sampling(0.0)
    m.close()
    per_tok = ms / 1e3 / n_new
    gemm_flop = 2.0 * (n_prompt - 1) * DECODE_PROJ_WEIGHTS
    peak_tf, _ = tensor_peak()
    return {"tokens_per_s": round(n_new / (ms / 1e3), 2), "ms_per_token": round(per_tok * 1e3, 4),
            "prefill_tokens_per_s": round((n_prompt - 1) / prefill_s, 1),
            "prefill": {"path": "tcgen05 GEMM prefill (projections) + causal attention over the f16 KV cache, "
                                "chunks of 2048 rows; wall clock incl. the first decode step",
                        "ms": round(prefill_s * 1e3, 2),
                        "projection_tflops": round(gemm_flop / prefill_s / 1e12, 1),
                        "projection_frac_of_peak": round(gemm_flop / prefill_s / 1e12 / peak_tf, 4),
                        "token_by_token_tokens_per_s": round(255 / tok_s, 1),
                        "agrees_with_token_by_token": bool(np.array_equal(tokwise, again))},
            "weight_gbs": round(DECODE_BYTES_PER_TOKEN_WEIGHTS / per_tok / 1e9, 1),
            "n_prompt": n_prompt, "n_new": n_new, "n_layer": cfg.n_layer, "first_tokens": [int(first[0, 0])] + [int(v) for v in tk[1:6]],
            "deterministic": bool(np.array_equal(again, again2)),
            "sampled_tokens_per_s": round(n_new / (ms_sampled / 1e3), 2),
            "note": "decode steps replayed as one CUDA graph each (5 fused kernels per layer + head + argmax)"}


GEMM_M, GEMM_N, GEMM_K = 512, 14336, 4096
GEMM_FLOP = 2 * GEMM_M * GEMM_N * GEMM_K  # 6.013e10


def tensor_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured (bf16 cuBLAS burst)"
    except Exception:
        return 1590.0, "fallback"


def prefill_gemm(K, dev, iters=20, cpu_tokens=0):
    """Q4_0 prefill GEMM, M 512 x N 14336 x K 4096 (MLP up-projection shape):
    W ~ N(0,0.02) seed 4, A ~ N(0,1) seed 5, C f32.  Each timed launch (the
    activation conversion + the tcgen05 GEMM, CUDA events on the launching
    stream) follows a 256 MB write that flushes L2."""
    import torch
    blocks = K.synth_q4_0(GEMM_N, GEMM_K, 0.02, 4, device=dev)
    W = K.Q4Weight.from_q4_0(blocks, GEMM_N, GEMM_K)
    a = K.fill_normal(GEMM_M * GEMM_K, 0.0, 1.0, 5, device=dev).reshape(GEMM_M, GEMM_K)
    c = torch.empty(GEMM_M, GEMM_N, dtype=torch.float32, device=dev)
    ws = torch.empty(W.gemm_workspace_bytes(GEMM_M) + 1024, dtype=torch.uint8, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream(dev)
    for _ in range(3):
        W.gemm(a, c, ws)
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        flush.fill_(1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        W.gemm(a, c, ws)
        e1.record(st)
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    times.sort()
    ms = times[len(times) // 2]
    peak, kind = tensor_peak()
    tf = GEMM_FLOP / (ms / 1e3) / 1e12
    out = {"tflops": round(tf, 1), "us_per_call": round(ms * 1e3, 2), "frac_of_peak": round(tf / peak, 4),
           "peak_tflops": peak, "peak_source": kind, "flop_per_call": GEMM_FLOP,
           "shape": f"M{GEMM_M} N{GEMM_N} K{GEMM_K}", "l2": "flushed (256 MB write) before each timed launch",
           "kernels": "k_gemm_prep + k_gemm_q4_tc<2,false>", "finite": bool(torch.isfinite(c).all().item())}
    if cpu_tokens:
        # the reference's prefill path: one AVX-512 gemv_4bit_into per token row
        from oracle import oracle as O
        rng = np.random.default_rng(4)
        nb = GEMM_N * GEMM_K // 32
        scales = (rng.random(nb) * 0.004).astype(np.float32)
        packed = rng.integers(0, 256, GEMM_N * GEMM_K // 2, dtype=np.uint8)
        ah = a[:cpu_tokens].cpu().numpy()
        ch = np.empty((cpu_tokens, GEMM_N), np.float32)
        nt = cpu_threads()
        t0 = time.perf_counter()
        O.lib().or_avx_gemm_rows(ch, scales, packed, np.ascontiguousarray(ah), cpu_tokens, GEMM_N, GEMM_K, nt)
        dt = time.perf_counter() - t0
        out["cpu_baseline"] = {"value": round(2.0 * cpu_tokens * GEMM_N * GEMM_K / dt / 1e12, 5),
                               "unit": "TFLOP/s", "cores": nt, "kind": "port",
                               "sample": f"{cpu_tokens} token rows through the AVX-512 gemv_4bit_into restatement "
                                         f"(token-by-token prefill, inference/mod.rs:550), {dt:.2f} s"}
    W.close()
    return out


def _gpu_seconds(fn, stream, iters=20):
    """Device time per call (CUDA events on `stream`, after 3 warm-up calls)."""
    import torch
    with torch.cuda.stream(stream):
        for _ in range(3):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(iters):
            fn()
        e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / 1e3 / iters


def _cpu_seconds(fn, min_s=0.5, max_calls=20):
    fn()  # first touch of the output pages
    n, t0 = 0, time.perf_counter()
    while n < max_calls:
        fn()
        n += 1
        if time.perf_counter() - t0 >= min_s:
            break
    return (time.perf_counter() - t0) / n


def secondary_measurements(K, dev, stream, peak, no_cpu=False):
    """Config-1 conversions and dequantisation (every launch > L2: 206-271 MB
    moved), each with the reference's CPU implementation of the same call timed
    on the host beside it, and the DedupCount load path and SSM step."""
    import torch
    from agent_harness_b200 import _lib
    out = {}
    n = 4096 * 11008
    w = K.fill_normal(n, 0.0, 0.02, 0, device=dev)
    q8 = K.quantize_q8_0(w)
    q4 = K.quantize_q4_0(w)
    sc, pk = K.quantize_q4(w, 32)
    del w
    f = torch.empty(n, dtype=torch.float32, device=dev)
    h = K.f32_to_f16(K.fill_normal(n, 0.0, 1.0, 1, device=dev))
    st = C.c_void_p(stream.cuda_stream)
    L = _lib.lib()
    rows = (
        ("dequant_q8_0", lambda: K.dequant_q8_0(q8, n, out=f), q8.numel() + 4 * n,
         "Q8_0 blocks {f16 d; i8 q[32]} (gguf.rs:459-479)"),
        ("dequant_q4_0", lambda: K.dequant_q4_0(q4, n, out=f), q4.numel() + 4 * n,
         "Q4_0 blocks {f16 d; u8 q[16]} (gguf.rs:480-502)"),
        ("dequant_layer", lambda: L.ah_dequant_layer(C.c_void_p(sc.data_ptr()), C.c_void_p(pk.data_ptr()),
                                                     C.c_void_p(f.data_ptr()), n, 32, st),
         pk.numel() + 4 * sc.numel() + 4 * n, "engine format, f32 group-32 scales (quantization.rs:439-454)"),
        ("f16_to_f32", lambda: L.ah_f16_to_f32(C.c_void_p(h.data_ptr()), C.c_void_p(f.data_ptr()), n, st),
         2 * n + 4 * n, "f16 bits N(0,1) seed 1 (gguf.rs:93-120)"),
    )
    for name, fn, nbytes, what in rows:
        s = _gpu_seconds(fn, stream)
        gbs = nbytes / s / 1e9
        out[name] = {"gbs": round(gbs, 2), "pct_of_8tbs": round(100 * gbs / NOMINAL_HBM_GBS, 2),
                     "frac_of_measured_peak": round(gbs / peak, 4), "bytes_per_call": nbytes,
                     "us_per_call": round(s * 1e6, 2), "shape": "4096x11008", "input": what}
    if not no_cpu:
        from oracle import oracle as O
        OL = O.lib()
        q8h, q4h, sch, pkh, hh = (t.cpu().numpy() for t in (q8, q4, sc, pk, h))
        # the AVX-512 restatement keeps the reference's read of 4 halves past the
        # end (avx512_kernel.rs:147): give it a padded copy
        hu8 = np.zeros(2 * n + 64, np.uint8)
        hu8[: 2 * n] = hh.view(np.uint8)
        dst = np.empty(n, np.float32)
        cpu = {
            "dequant_q8_0": [("scalar gguf.rs:459-479 restated", 1,
                              lambda: OL.or_dequantize_to_f32(q8h, q8h.size, 8, n, dst))],
            "dequant_q4_0": [("scalar gguf.rs:480-502 restated", 1,
                              lambda: OL.or_dequantize_to_f32(q4h, q4h.size, 2, n, dst))],
            "dequant_layer": [("dequant_layer_avx512 as-is (quantization.rs:456-530)", 1,
                               lambda: OL.or_avx_dequant_layer(sch, pkh, dst, n)),
                              ("scalar branch quantization.rs:444-452", 1,
                               lambda: OL.or_dequant_layer(sch, pkh, dst, n, 32))],
            "f16_to_f32": [("f16_bytes_to_f32 AVX-512 as-is (avx512_kernel.rs:212-232)", 1,
                            lambda: OL.or_avx_f16_bytes_to_f32(hu8, 2 * n, dst)),
                           ("scalar gguf::f16_to_f32 per element (gguf.rs:93-120)", 1,
                            lambda: OL.or_f16_array_to_f32(hh.view(np.uint16), dst, n))],
        }
        for name, legs in cpu.items():
            nbytes = out[name]["bytes_per_call"]
            res = []
            for what, cores, fn in legs:
                sec = _cpu_seconds(fn)
                res.append({"value": round(nbytes / sec / 1e9, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                            "sample": f"the whole 4096x11008 call, {what}, {sec * 1e3:.1f} ms per call"})
            out[name]["cpu_baseline"] = res[0]
            if len(res) > 1:
                out[name]["cpu_baseline_alt"] = res[1]
    del q8, q4, sc, pk, f, h
    out["dedup_load"] = dedup_load(K, dev, stream, peak, cpu=not no_cpu)
    out["ssm_step"] = ssm_step(dev, stream, peak, cpu=not no_cpu)
    return out


SSM_CFG = dict(n_embd=2048, d_state=128, n_group=16, dt_rank=32, d_inner=4096, d_conv=4, eps=1e-6)


def ssm_step(dev, stream, peak, cpu=True, steps=200):
    """One token through the gated delta-net SSM block (inference/ssm.rs:171-296)
    at a Qwen3.5-like width: f32 weights (128 MB), the per-head state read and
    written (2 x 2 MB) and the conv window per step.  Three weight copies
    rotate (384 MB, larger than L2)."""
    import torch
    from agent_harness_b200.ssm import SsmBlock
    cfg = SSM_CFG
    rng = np.random.default_rng(13)
    D, nv, ng, d = cfg["d_state"], cfg["dt_rank"], cfg["n_group"], cfg["n_embd"]
    vd = cfg["d_inner"]
    cd = 2 * ng * D + vd
    shapes = {"wqkv": (cd, d), "wqkv_gate": (vd, d), "conv1d": (cd, cfg["d_conv"]), "dt_bias": (nv,), "a": (nv,),
              "alpha": (nv, d), "beta": (nv, d), "norm": (D,), "out": (d, vd)}
    blocks = []
    for c in range(3):
        w = {k: (rng.standard_normal(sh) * (0.02 if len(sh) == 2 and sh[1] == d or k == "out" else 0.5))
             .astype(np.float32) for k, sh in shapes.items()}
        w["a"] = -np.abs(w["a"])
        blocks.append(SsmBlock(cfg, w, device=dev))
    states = [b.new_state() for b in blocks]
    x = torch.randn(d, device=dev)
    out = torch.empty(d, device=dev)
    with torch.cuda.stream(stream):
        for i in range(6):
            blocks[i % 3].forward(x, states[i % 3], out=out)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(steps):
            blocks[i % 3].forward(x, states[i % 3], out=out)
        e1.record(stream)
    torch.cuda.synchronize()
    sec = e0.elapsed_time(e1) / 1e3 / steps
    wbytes = sum(int(np.prod(sh)) * 4 for sh in shapes.values())
    sbytes = 2 * nv * D * D * 4 + 2 * (cfg["d_conv"] - 1) * cd * 4
    nbytes = wbytes + sbytes
    res = {"config": "n_embd 2048, d_state 128, 16 k heads, 32 v heads, d_inner 4096, d_conv 4 (f32 weights)",
           "us_per_token": round(sec * 1e6, 2), "gbs": round(nbytes / sec / 1e9, 1),
           "frac_of_measured_peak": round(nbytes / sec / 1e9 / peak, 4), "bytes_per_token": nbytes,
           "launches_per_token": 3, "finite": bool(torch.isfinite(out).all().item())}
    if cpu:
        from oracle import oracle as O
        wc = {k: blocks[0].w[k].cpu().numpy() for k in O.SSM_WEIGHTS}
        cs = np.zeros(((cfg["d_conv"] - 1), cd), np.float32)
        ss = np.zeros((nv, D, D), np.float32)
        xn = x.cpu().numpy()
        t0 = time.perf_counter()
        n = 3
        for _ in range(n):
            O.ssm_forward(cfg, wc, cs, ss, xn)
        dt = (time.perf_counter() - t0) / n
        res["cpu_baseline"] = {"us_per_token": round(dt * 1e6, 1), "cores": 1, "kind": "port",
                               "sample": f"{n} tokens through the oracle restatement of ssm.rs:171-296"}
    return res


DEDUP_ROWS, DEDUP_COLS = 14336, 4096  # an 8B FFN gate/up matrix


def dedup_load(K, dev, stream, peak, cpu=True):
    """DedupCount load path on one FFN matrix: the fused decode + quantize +
    tiled repack (inference/mod.rs:255-271) and the decode alone
    (decompressor.rs:7-27).  Synthetic sandbag: 12 prefixes, 900 unique tails,
    uniform indices and signs (inputs 242 MB, larger than L2)."""
    import torch
    from agent_harness_b200 import dedup as D
    rows, cols = DEDUP_ROWS, DEDUP_COLS
    n = rows * cols
    g = torch.Generator(device=dev).manual_seed(11)
    rng = np.random.default_rng(11)
    t = D.DedupCountTensor(np.arange(12, dtype=np.uint16) * 3, np.sort(rng.choice(60000, 900, replace=False)), n, 2, 3,
                           2e-6)
    s = D.Sandbag(torch.randint(0, 12, (n,), dtype=torch.int16, device=dev, generator=g),
                  torch.randint(0, 900, (n,), dtype=torch.int16, device=dev, generator=g),
                  torch.randint(0, 256, ((n + 7) // 8,), dtype=torch.uint8, device=dev, generator=g), n)
    p_idx, t_idx, signs = s.on(dev)
    table = t._table_local()
    w = t.to_q4weight(s, rows, cols)
    f = torch.empty(n, dtype=torch.float32, device=dev)
    st = C.c_void_p(stream.cuda_stream)
    args = (table, C.c_void_p(p_idx.data_ptr()), n, C.c_void_p(t_idx.data_ptr()), n, C.c_void_p(signs.data_ptr()),
            signs.numel())
    from agent_harness_b200 import _lib
    fused = lambda: _lib.call("ah_dedup_into_q4w", *args, w.handle, st)                       # noqa: E731
    decode = lambda: _lib.call("ah_dedup_decompress_f32", *args, n, C.c_void_p(f.data_ptr()), st)  # noqa: E731
    res = {"shape": f"{rows}x{cols}", "table": "local (12 prefixes, 900 tails)"}
    for name, fn, per in (("fused_decode_quantize_repack", fused, 2 + 2 + 0.125 + 0.5 + 0.125),
                          ("decode_f32", decode, 2 + 2 + 0.125 + 4)):
        with torch.cuda.stream(stream):
            for _ in range(3):
                fn()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            iters = 20
            e0.record(stream)
            for _ in range(iters):
                fn()
            e1.record(stream)
        torch.cuda.synchronize()
        sec = e0.elapsed_time(e1) / 1e3 / iters
        nbytes = int(per * n)
        res[name] = {"gbs": round(nbytes / sec / 1e9, 2), "frac_of_measured_peak": round(nbytes / sec / 1e9 / peak, 4),
                     "us_per_call": round(sec * 1e6, 2), "bytes_per_call": nbytes,
                     "bytes_per_element": per, "gelem_per_s": round(n / sec / 1e9, 3)}
    _lib.call("ah_dedup_table_destroy", table)
    w.close()
    if cpu:
        res["cpu_baseline"] = dedup_cpu_baseline()
    return res


def dedup_cpu_baseline(n=1 << 21):
    """The oracle's decompress_all + quantize (scalar restatements of
    decompressor.rs:7-27 and quantization.rs:369-404), one thread, on a
    2M-element sample compressed by the oracle's compress."""
    from oracle import oracle as O
    w = (np.random.default_rng(12).standard_normal(n) * 0.02).astype(np.float32)
    t, s = O.dedup_compress(w, 2, 2)
    scales = np.empty(n // 32, np.float32)
    packed = np.empty(n // 2, np.uint8)
    t0 = time.perf_counter()
    dec = O.dedup_decompress_all(t, s)
    O.lib().or_quantize_q4(dec, n, 32, scales, packed)
    dt = time.perf_counter() - t0
    per = 2 + 2 + 0.125 + 0.5 + 0.125
    return {"gbs": round(per * n / dt / 1e9, 3), "gelem_per_s": round(n / dt / 1e9, 4), "cores": 1, "kind": "port",
            "sample": f"{n} elements: oracle compress(pd 2, 2 rounds), then decompress_all + quantize timed"}


def mma_rate():
    """Cost of one tcgen05.mma (kind::f16, K = 16) by N and form, from 256
    back-to-back MMAs on one SM (ah_debug_tc_mma_rate)."""
    import ctypes as C
    from agent_harness_b200 import _lib
    rows = []
    names = {0: "1-CTA, A in shared memory, M=64", 1: "1-CTA, A in tensor memory, M=128",
             2: "CTA pair, A in tensor memory, M=256"}
    for mode, ns in ((1, (16, 32, 64, 128, 256)), (0, (16, 64, 256)), (2, (32, 64, 128, 256))):
        for n in ns:
            out = (C.c_longlong * 3)()
            for _ in range(3):
                _lib.call("ah_debug_tc_mma_rate", mode, n, C.cast(out, C.c_void_p))
            rows.append({"form": names[mode], "n": n, "issue_cycles": round(out[0] / 256, 1),
                         "complete_cycles": round(out[1] / 256, 1), "ns_per_mma": round(out[2] / 256, 1),
                         "sm_mhz": round(1e3 * out[1] / max(out[2], 1))})
    return rows


def sample_rate(dev):
    """Temperature + top-k sampling (ah_sample_logits, T 0.8, top-k 40) per
    call over [batch][vocab] f32 logits: device time of back-to-back calls
    captured in one CUDA graph (no host launch cost), rows split over slice
    CTAs and walked by one CTA each."""
    import torch
    from agent_harness_b200 import kernels as K
    rows = []
    reps = 100
    for vocab in (128256, 32000):
        for batch in (1, 16, 64):
            lg = K.fill_normal(batch * vocab, 0.0, 2.0, 3, device=dev).reshape(batch, vocab)
            out = torch.empty(batch, dtype=torch.int32, device=dev)
            ws = torch.empty(max(K.sample_workspace_bytes(batch, vocab), 16), dtype=torch.uint8, device=dev)
            row = {"vocab": vocab, "batch": batch, "top_k": 40}
            for split in (True, False):
                st = torch.cuda.Stream(device=dev)
                with torch.cuda.stream(st):
                    for s in range(3):
                        K.sample_logits(lg, 0.8, 40, seed=1, step=s, out=out, workspace=ws, split=split)
                st.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=st):
                    for s in range(reps):
                        K.sample_logits(lg, 0.8, 40, seed=1, step=s, out=out, workspace=ws, split=split)
                g.replay()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                with torch.cuda.stream(st):
                    e0.record(st)
                    g.replay()
                    e1.record(st)
                torch.cuda.synchronize()
                us = e0.elapsed_time(e1) * 1e3 / reps
                row["split_us" if split else "one_cta_per_row_us"] = round(us, 2)
                del g
            rows.append(row)
    return rows


def bgemv_shapes(dev):
    """The batched tcgen05 GEMV (ah_q4w_gemv_tc) against the mma.sync GEMV
    (ah_q4w_gemv) on the 70B projections and their tensor-parallel slices at
    batches 9, 12 and 16: per-call device time over back-to-back calls on
    rotating weight copies (>= 600 MB streamed per pass, larger than L2)."""
    import torch
    from agent_harness_b200 import kernels as K
    shapes = []
    for tp in (1, 2, 4, 8):
        shapes += [(tp, "qkv", 10240 // tp, 8192), (tp, "o", 8192, 8192 // tp), (tp, "gate_up", 57344 // tp, 8192),
                   (tp, "down", 8192, 28672 // tp), (tp, "lm_head", 128256 // tp, 8192)]
    rows = []
    for tp, name, r, c in shapes:
        blocks = K.synth_q4_0(r, c, 0.02, 1, device=dev)
        ncopy = max(1, 600_000_000 // (r * c * 9 // 16))
        Ws = [K.Q4Weight.from_q4_0(blocks, r, c) for _ in range(ncopy)]
        del blocks
        wb = Ws[0].weight_bytes
        ws = torch.empty(Ws[0].gemv_tc_workspace_bytes() + 1024, dtype=torch.uint8, device=dev)
        for B in (16, 12, 9):
            x = K.fill_normal(B * c, 0.0, 1.0, 2, device=dev).reshape(B, c)
            y = torch.empty(B, r, device=dev)
            t = {}
            for impl in ("tc", "mma"):
                def run(W):
                    if impl == "tc":
                        W.gemv_tc(x, out=y, workspace=ws)
                    else:
                        W.gemv(x, out=y)
                for W in Ws:
                    run(W)
                torch.cuda.synchronize()
                reps = max(1, 40 // ncopy)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(reps):
                    for W in Ws:
                        run(W)
                e1.record()
                torch.cuda.synchronize()
                t[impl] = e0.elapsed_time(e1) * 1e3 / (reps * ncopy)
            rows.append({"tp": tp, "weight": name, "rows": r, "cols": c, "batch": B, "tc_us": round(t["tc"], 1),
                         "mma_us": round(t["mma"], 1), "tc_gbs": round(wb / t["tc"] / 1e3),
                         "mma_gbs": round(wb / t["mma"] / 1e3)})
        for W in Ws:
            W.close()
    return rows


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=4000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--quick", action="store_true", help="headline only")
    ap.add_argument("--workload", default="gemv",
                    choices=["gemv", "decode", "gemm", "tp", "load", "ssm", "bgemv", "mma-rate", "sample"],
                    help="decode / gemm / tp / load: only the 8B decode, the prefill GEMM, the 70B tensor-parallel "
                         "decode or the DedupCount load-path measurement (for profiling); bgemv: the batched "
                         "decode GEMVs on the 70B shapes; mma-rate: the tcgen05.mma cost table; sample: "
                         "temperature + top-k sampling per call")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--cpu-seconds", type=float, default=8.0)
    ap.add_argument("--no-decode", action="store_true", help="skip the 8B decode measurement")
    ap.add_argument("--decode-prompt", type=int, default=DECODE_PROMPT)
    ap.add_argument("--decode-new", type=int, default=DECODE_NEW)
    ap.add_argument("--decode-layers", type=int, default=None, help="fewer 8B-shape layers (profiling only)")
    ap.add_argument("--no-tp", action="store_true", help="skip the 70B tensor-parallel decode measurement")
    ap.add_argument("--tp-prompt", type=int, default=TP_PROMPT)
    ap.add_argument("--tp-new", type=int, default=TP_NEW)
    ap.add_argument("--tp-layers", type=int, default=None, help="fewer 70B-shape layers (profiling only)")
    ap.add_argument("--tp-allreduce", default="peer", choices=["peer", "nccl"],
                    help="block all-reduce of the tensor-parallel decoder")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload in ("bgemv", "mma-rate", "sample"):
        import torch
        torch.cuda.set_device(0)
        from agent_harness_b200 import _lib
        _lib.check(_lib.lib().ah_device_init(0))
        dev = torch.device("cuda", 0)
        rows = (mma_rate() if args.workload == "mma-rate" else
                sample_rate(dev) if args.workload == "sample" else bgemv_shapes(dev))
        for r in rows:
            print(json.dumps({"workload": args.workload, **r}), flush=True)
        return 0
    if args.workload == "ssm":
        import torch
        torch.cuda.set_device(0)
        from agent_harness_b200 import _lib
        _lib.check(_lib.lib().ah_device_init(0))
        dev = torch.device("cuda", 0)
        print(json.dumps({"workload": "ssm_step", **ssm_step(dev, torch.cuda.Stream(device=dev), peaks()[0],
                                                             cpu=not args.no_cpu)}), flush=True)
        return 0
    if args.workload == "load":
        import torch
        torch.cuda.set_device(0)
        from agent_harness_b200 import _lib
        from agent_harness_b200 import kernels as K
        _lib.check(_lib.lib().ah_device_init(0))
        dev = torch.device("cuda", 0)
        print(json.dumps({"workload": "dedup_load", **dedup_load(K, dev, torch.cuda.Stream(device=dev), peaks()[0],
                                                                 cpu=not args.no_cpu)}), flush=True)
        return 0
    if args.workload == "decode":
        import torch
        torch.cuda.set_device(0)
        from agent_harness_b200 import _lib
        _lib.check(_lib.lib().ah_device_init(0))
        print(json.dumps({"workload": "decode_8b", **decode_8b(torch.device("cuda", 0), args.decode_prompt,
                                                               args.decode_new, args.decode_layers)}), flush=True)
        return 0
    if args.workload == "tp":
        import torch
        rank, world, local = dist_env()
        torch.cuda.set_device(local)
        if world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                    timeout=datetime.timedelta(seconds=300))
        from agent_harness_b200 import _lib
        _lib.check(_lib.lib().ah_device_init(local))
        r = decode_70b_tp(torch.device("cuda", local), rank, world, args.tp_prompt, args.tp_new,
                          allreduce=args.tp_allreduce, n_layer=args.tp_layers)
        if rank == 0:
            print(json.dumps({"workload": "decode_70b_tp", **r}), flush=True)
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
        return 0
    if args.workload == "gemm":
        import torch
        torch.cuda.set_device(0)
        from agent_harness_b200 import _lib
        from agent_harness_b200 import kernels as K
        _lib.check(_lib.lib().ah_device_init(0))
        print(json.dumps({"workload": "prefill_gemm", **prefill_gemm(K, torch.device("cuda", 0),
                                                                      iters=max(args.steps, 1))}), flush=True)
        return 0
    return run_gpu(args)


if __name__ == "__main__":
    sys.exit(main())
