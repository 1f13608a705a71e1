#!/usr/bin/env python
"""Benchmark of the decode hot path on B200: INT4 g128 dequant-GEMV HBM throughput.

Workload (default): W is 4096x14336 f32 ~ N(0, 0.02) (seed 0) with 72 = 0.5% of the input
channels scaled x20, 3.5-sigma outlier extraction, INT4 g128 quantization of the rest (the
reference's `pox quantize` pipeline); x is 1x14336 f16 ~ N(0,1) promoted to f32. One step =
one GEMV y = W x with the fused outlier correction. Inputs are synthetic (no dataset exists).

Timing: W warm-up steps, then exactly K steps captured in CUDA graphs and timed with CUDA
events on the launching stream, bracketed by barrier + synchronize; eight resident weight
copies (8 x 32.6 MB > 2 x the 126 MB L2) are rotated so every step reads its weights from HBM.
Multi-GPU: each rank runs its own GEMV stream on its own weights (the path has no exchange
step: weak scaling, no data-path collective); the time is the max over ranks.

`--impl reference` times the reference's CPU path for the same workload (the oracle's C
restatement of quant::gemv_int4, single-threaded per call as the reference is) on every host
thread this process may use, one row slice per thread.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import re
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

ROWS, COLS, GS, HOT_COLS = 4096, 14336, 128, 72
NCOPY = 8
METRIC = "INT4 dequant-GEMV HBM GB/s (% of peak); decode tokens/s at 1/2/4/8 B200"
WORKLOAD = "int4_g128_gemv_4096x14336_b1_outliers3.5sigma"
FALLBACK_HBM_GBS = 6650.0


def make_workload(seed: int = 0):
    from paraoxidizer_b200 import quant as Q

    rng = np.random.default_rng(seed)
    w = rng.standard_normal(ROWS * COLS, dtype=np.float32) * np.float32(0.02)
    hot = rng.choice(COLS, HOT_COLS, replace=False)
    w.reshape(ROWS, COLS)[:, hot] *= np.float32(20.0)
    tab = Q.extract_and_zero_outliers(w, "automatic")
    packed, scales = Q.quantize_int4_group(w, GS)
    ob = Q.outliers_to_bytes(*tab)
    xr = np.random.default_rng(seed + 1)
    x = xr.standard_normal(COLS, dtype=np.float32).astype(np.float16).astype(np.float32)
    return packed, scales, tab, ob, x


def algorithmic_bytes(nnz: int) -> int:
    """Bytes one GEMV must move: packed nibbles + f16 scale/min pairs + the .pox outlier table
    (4 + 6 nnz) + x (f16 input, 2 B/elem) + y (f32 output)."""
    return ROWS * COLS // 2 + ROWS * (COLS // GS) * 4 + 4 + 6 * nnz + COLS * 2 + ROWS * 4


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic():
    """dram read+write bytes per launch of the GEMV kernel from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "gemv_int4_4096x14336_b1.md")
    try:
        with open(p) as f:
            m = re.search(r"traffic_bytes_per_launch:\s*([0-9]+)", f.read())
        return int(m.group(1)) if m else None
    except OSError:
        return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "50"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self):
        rows = []
        for line in (self.out or "").strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[4:8]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i in range(4) if r[i].lower().startswith("active")})
        sm = sorted(r[0] for r in rows)
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": max(r[1] for r in rows), "reasons": reasons,
                "samples": len(rows)}


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def _slice_tables(tab, rows_per_call):
    """Outlier tables re-based to each row slice (built outside any timed region). Entries
    outside the slice stay in the table: the reference scans the whole table for every row."""
    out = {}
    for r0 in range(0, ROWS, rows_per_call):
        out[r0] = ((tab[0].astype(np.int64) - r0 * COLS).astype(np.uint32), tab[1])
    return out


def cpu_baseline_sample(packed, scales, tab, budget_s: float = 12.0, rows_per_call: int = 256):
    """Times the oracle (C restatement of quant::gemv_int4, single-threaded like the reference)
    on row slices of the same workload until the budget is spent. Returns GB/s and details."""
    from oracle import oracle as O

    x = np.random.default_rng(1).standard_normal(COLS, dtype=np.float32).astype(np.float16).astype(np.float32)
    rb, sb = COLS // 2, (COLS // GS) * 4
    tables = _slice_tables(tab, rows_per_call)
    rows_done, t_total = 0, 0.0
    r0 = 0
    while t_total < budget_s:
        t0 = time.perf_counter()
        O.gemv_int4(packed[r0 * rb:(r0 + rows_per_call) * rb], scales[r0 * sb:(r0 + rows_per_call) * sb], GS,
                    rows_per_call, COLS, tables[r0], x)
        t_total += time.perf_counter() - t0
        rows_done += rows_per_call
        r0 = (r0 + rows_per_call) % ROWS
    full = algorithmic_bytes(len(tab[0]))
    gbs = full * rows_done / ROWS / t_total / 1e9
    return gbs, rows_done, t_total


def host_cpu():
    """The host CPU model and the number of cores this process may use."""
    model = "unknown"
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:
        n = os.cpu_count() or 1
    return model, n


def cpu_decode_baseline(be, cfg=None, positions=3):
    """The reference's forward_token (the oracle's C restatement, single-threaded like the reference)
    timed at the Llama-3-8B widths on a reduced schedule: a 1-layer and a 2-layer model share the
    first layer's weights (INT4 g128 from the GPU quantizer, f16 embedding / lm_head), each decodes
    `positions` tokens; the difference gives one layer's time and the rest the embedding / norm /
    lm_head, so tokens/s of the full model = 1 / (rest + layers x layer). Random-init weights."""
    import torch

    from oracle import oracle as O
    from paraoxidizer_b200 import _lib as L

    cfg = dict(cfg or LLAMA_8B)
    H, I, V = cfg["hidden"], cfg["inter"], cfg["vocab"]
    hd = H // cfg["n_heads"]
    qd, kvd = cfg["n_heads"] * hd, cfg["n_kv_heads"] * hd
    gen = torch.Generator(device="cuda")
    gen.manual_seed(4)
    shapes = {"q": (qd, H), "k": (kvd, H), "v": (kvd, H), "o": (H, qd), "gate": (I, H), "up": (I, H), "down": (H, I)}
    layer = {}
    for name, (r, c) in shapes.items():
        w = torch.randn(r * c, device="cuda", generator=gen).mul_(0.02)
        p = torch.empty(r * c // 2, dtype=torch.uint8, device="cuda")
        sc = torch.empty(r * c // 128 * 4, dtype=torch.uint8, device="cuda")
        torch.cuda.synchronize()
        L.check(L.lib().pox_cuda_quantize_int4(be.ctx, w.data_ptr(), r * c, 128, p.data_ptr(), sc.data_ptr(), None))
        be.synchronize()
        layer[name] = {"packed": p.cpu().numpy(), "scales": sc.cpu().numpy(), "rows": r, "cols": c, "group_size": 128,
                       "outliers": None}
        del w, p, sc
    ones = np.ones(H, np.float32).astype(np.float16).view(np.uint16)
    layer["attn_norm"] = layer["mlp_norm"] = ones
    emb = torch.randn(V * H, device="cuda", generator=gen).mul_(0.02).half().cpu().numpy().view(np.uint16)
    head = torch.randn(V * H, device="cuda", generator=gen).mul_(0.02).half().cpu().numpy().view(np.uint16)
    times = {}
    for nl in (1, 2):
        c = dict(cfg, layers=nl)
        m = O.OracleModel(c, {"embed": emb, "lm_head": head, "final_norm": ones, "layers": [layer] * nl},
                          max_seq=positions + 1, kv_f16=False)
        t0 = time.perf_counter()
        for pos in range(positions):
            m.forward_token(7 + pos, pos)
        times[nl] = (time.perf_counter() - t0) / positions
    t_layer = max(times[2] - times[1], 1e-9)
    t_rest = max(times[1] - t_layer, 0.0)
    per_token = t_rest + cfg["layers"] * t_layer
    model, n = host_cpu()
    return {"tokens_per_s": round(1.0 / per_token, 4), "s_per_token": round(per_token, 3), "cores": 1,
            "kind": "port", "cpu_model": model, "host_cores": n,
            "sample": f"forward_token (oracle C restatement, single-threaded like the reference) at the Llama-3-8B "
                      f"widths: {positions} tokens through a 1-layer and a 2-layer model ({times[1]:.3f} / "
                      f"{times[2]:.3f} s per token), extrapolated to {cfg['layers']} layers "
                      f"(one layer {t_layer:.3f} s, embedding + norm + lm_head {t_rest:.3f} s)"}


def run_reference(args):
    world, rank, _ = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), 0
    if rank != 0:
        return 0
    packed, scales, tab, ob, x = make_workload()
    nnz = len(tab[0])
    full = algorithmic_bytes(nnz)
    from oracle import oracle as O

    import concurrent.futures as cf

    rows_per_slice = 64
    rb, sb = COLS // 2, (COLS // GS) * 4
    tables = _slice_tables(tab, rows_per_slice)
    # every host thread this process may use runs its own row slice through the reference's
    # single-threaded loop (the oracle's C calls release the GIL): one step = one slice per thread
    threads = host_cpu()[1]
    pool = cf.ThreadPoolExecutor(threads)

    def one(r0):
        O.gemv_int4(packed[r0 * rb:(r0 + rows_per_slice) * rb], scales[r0 * sb:(r0 + rows_per_slice) * sb], GS,
                    rows_per_slice, COLS, tables[r0], x)

    def step(i):
        list(pool.map(one, [((i * threads + j) * rows_per_slice) % ROWS for j in range(threads)]))

    # bound the run: at most ~90 s of timed CPU work whatever K is
    t0 = time.perf_counter()
    step(0)
    per_step = time.perf_counter() - t0
    steps = max(1, min(args.steps, int(90.0 / max(per_step, 1e-6))))
    for i in range(min(args.warmup, 3)):
        step(i + 1)
    t0 = time.perf_counter()
    for i in range(steps):
        step(i)
    dt = time.perf_counter() - t0
    pool.shutdown()
    bytes_per_step = full * rows_per_slice * threads / ROWS
    gbs = bytes_per_step * steps / dt / 1e9
    sample = (f"{steps} steps, each {threads} concurrent slices (one per host thread) of quant::gemv_int4 (oracle "
              f"C restatement, single-threaded per call as the reference) over {rows_per_slice} rows x {COLS} cols, "
              f"with the full {nnz}-entry outlier table scanned per row as the reference does; bytes counted pro "
              f"rata of one {ROWS}x{COLS} GEMV")
    line = {"metric": METRIC, "value": round(gbs, 4), "unit": "GB/s", "impl": "reference", "n_gpus": world,
            "steps": steps, "warmup": min(args.warmup, 3), "ms_per_step": dt / steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,0.02) weights, N(0,1) f16 x)",
            "config": {"workload": WORKLOAD, "rows": ROWS, "cols": COLS, "group_size": GS, "batch": 1,
                       "outliers": nnz},
            "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                             "cpu_model": host_cpu()[0], "sample": sample},
            "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def batched_gemv_bench(be, batches=(1, 4, 16, 64), reps=400):
    """The batched configurations: INT8 14336x4096 (per-tensor scale, the parity path) and INT4 g128
    4096x14336 without and with 3.5-sigma outliers, at B rows of x (each line names the kernel the
    library chose: the mma.sync GEMV at small B, a tcgen05 small-M kernel above). Copies rotated past L2, CUDA graph of `reps` launches, CUDA events.
    Algorithmic bytes: weights + scales (+ outlier table) + x as f16 (2 K B) + y as f32 (4 N B)."""
    import torch

    from paraoxidizer_b200 import quant as Q

    out = {}
    peak, _ = measured_peak()
    rng = np.random.default_rng(11)
    stream = torch.cuda.Stream()
    cases = []
    w8 = rng.standard_normal(14336 * 4096, dtype=np.float32) * np.float32(0.02)
    q8, s8 = Q.quantize_int8_symmetric(w8)
    cases.append(("int8_14336x4096", 14336, 4096, [be.upload_int8(q8, s8, 14336, 4096) for _ in range(6)],
                  14336 * 4096 + 4))
    # the configuration as worded: one f16 scale per output row (the per-channel extension)
    q8r, s8r = Q.quantize_int8_rows(w8, 14336, 4096)
    cases.append(("int8_rowscale_14336x4096", 14336, 4096,
                  [be.upload_int8_rows(q8r, s8r, 14336, 4096) for _ in range(6)], 14336 * 4096 + 2 * 14336))
    del w8, q8, q8r
    packed, scales, tab, ob, _ = make_workload(seed=3)
    cases.append(("int4_g128_4096x14336", ROWS, COLS,  # the decode weights' format: no outlier table
                  [be.upload_int4(packed, scales, ROWS, COLS, GS) for _ in range(8)],
                  ROWS * COLS // 2 + ROWS * (COLS // GS) * 4))
    cases.append(("int4_g128_4096x14336_outliers", ROWS, COLS,
                  [be.upload_int4(packed, scales, ROWS, COLS, GS, ob) for _ in range(8)],
                  ROWS * COLS // 2 + ROWS * (COLS // GS) * 4 + 4 + 6 * len(tab[0])))
    for name, N, K, ts, wbytes in cases:
        res = {}
        for B in batches:
            x = torch.randn(B * K, device="cuda")
            y = torch.zeros(B * N, device="cuda")
            with torch.cuda.stream(stream):
                for i in range(3 * len(ts)):
                    ts[i % len(ts)].gemv_device(x.data_ptr(), B, y.data_ptr(), stream.cuda_stream)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(stream):
                with torch.cuda.graph(g, stream=stream):
                    for i in range(reps):
                        ts[i % len(ts)].gemv_device(x.data_ptr(), B, y.data_ptr(),
                                                    torch.cuda.current_stream().cuda_stream)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                g.replay()
                e0.record(stream)
                g.replay()
                e1.record(stream)
            torch.cuda.synchronize()
            sec = e0.elapsed_time(e1) * 1e-3 / reps
            nbytes = wbytes + 2 * K * B + 4 * N * B
            res[str(B)] = {"us": round(sec * 1e6, 2), "gbs": round(nbytes / sec / 1e9, 1),
                           "frac_of_hbm_peak": round(nbytes / sec / 1e9 / peak, 4),
                           "tflops": round(2.0 * N * K * B / sec / 1e12, 2),
                           "kernel": ts[0].gemv_kernel(B)}
            del g
        out[name] = res
        for t in ts:
            t.free()
    return out


LLAMA_8B = {"hidden": 4096, "inter": 14336, "layers": 32, "n_heads": 32, "n_kv_heads": 8, "vocab": 128256,
            "rms_eps": 1e-5, "rope_theta": 500000.0}
LLAMA_70B = {"hidden": 8192, "inter": 28672, "layers": 80, "n_heads": 64, "n_kv_heads": 8, "vocab": 128256,
             "rms_eps": 1e-5, "rope_theta": 500000.0}
# decode workloads: (config, default batches, context before the timed steps, how it is reached,
# outlier sigma of the projections)
DECODE_MODELS = {
    "llama8b": (LLAMA_8B, "1,8,32", 512, "tokens", None),
    # context 4096 reached by reserving the pages (token-by-token prefill of 4096 x 80 layers would
    # dominate the run); the pages hold whatever the allocation held, which only changes values
    "llama70b": (LLAMA_70B, "1,16,64", 4096, "reserve", 3.5),
}


def decode_bench(be, cfg=LLAMA_8B, batches=(1, 8, 32), prefill=512, steps=256, warm=3, seed=0, world=1, rank=0,
                 modes=("peer", "nccl"), prefill_mode="tokens", outlier_sigma=None, name="llama-3-8b"):
    """Llama-3-8B-architecture INT4 g128 decode (random-init weights): prefill of `prefill` random
    token ids per sequence in passes of up to 256 rows (pox_cuda_model_prefill; the reference feeds
    them token by token through forward_token, engine.rs:760-762), then `steps` greedy decode steps
    timed as CUDA-graph replays of one step on the device. With
    world > 1 every rank holds a tensor-parallel shard and the step time is the max over ranks;
    each exchange implementation in `modes` is timed (the first is the default)."""
    import torch

    from paraoxidizer_b200.synth import build_llama_on_device

    max_b = max(batches)
    runs = len(modes) if world > 1 else 1
    bps = (prefill + steps * runs + warm + 15) // 16
    t0 = time.perf_counter()
    # prefill passes take up to 256 rows (the KV cache is sized for the decode batches only)
    model = build_llama_on_device(be, cfg, max(max_b, 256) if prefill_mode == "tokens" else max_b, max_b * bps, bps,
                                  seed=seed, tp_rank=rank, tp_size=world, outlier_sigma=outlier_sigma)
    if world > 1:
        model.init_comm(modes=modes)
    build_s = time.perf_counter() - t0
    H, L_, nkv = cfg["hidden"], cfg["layers"], cfg["n_kv_heads"] // world
    hd = H // cfg["n_heads"]
    rng = np.random.default_rng(2)
    out = {}
    stream = torch.cuda.Stream()
    for B in batches:
        seqs = [model.new_sequence() for _ in range(B)]
        prompts = rng.integers(0, cfg["vocab"], (B, prefill))
        t0 = time.perf_counter()
        nxt = None
        if prefill_mode == "reserve":
            for sq in seqs:
                sq.reserve(model.blocks, prefill)
                sq.sequence_len = prefill
            nxt = prompts[:, -1].astype(np.uint32)
        else:
            # the prompts through pox_cuda_model_prefill (tensor-core GEMMs over passes of 256 rows)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            _, nxt = model.prefill([list(r) for r in prompts], seqs, want_logits=False)
        prefill_s = time.perf_counter() - t0
        for sq in seqs:
            sq.reserve(model.blocks, steps * runs + warm)
        model.set_state(nxt, seqs)
        with torch.cuda.stream(stream):
            for _ in range(warm):
                model.decode_device(B, True, stream.cuda_stream)
        torch.cuda.synchronize()
        n = steps - 1
        per_mode = {}
        for mode in (modes if world > 1 else ("single",)):
            if world > 1:
                model.set_comm_mode(mode)
            g = torch.cuda.CUDAGraph()  # with tp, the exchange kernels / NCCL calls are part of the graph
            with torch.cuda.stream(stream):
                with torch.cuda.graph(g, stream=stream):
                    model.decode_device(B, True, torch.cuda.current_stream().cuda_stream)
            torch.cuda.synchronize()
            if world > 1:
                torch.distributed.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                e0.record(stream)
                for _ in range(n):
                    g.replay()
                e1.record(stream)
            torch.cuda.synchronize()
            t = torch.tensor([e0.elapsed_time(e1) * 1e-3 / n], dtype=torch.float64, device="cuda")
            if world > 1:
                torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            per_mode[mode] = float(t.item())
            del g
        sec = per_mode[modes[0] if world > 1 else "single"]
        ctx_avg = prefill + warm + 1 + n / 2.0
        kv_bytes = B * ctx_avg * L_ * nkv * hd * 2 * 2
        bytes_step = model.weight_bytes + kv_bytes
        peak, _ = measured_peak()
        out[str(B)] = {"tokens_per_s": round(B / sec, 1), "ms_per_step": round(sec * 1e3, 4),
                       "bytes_per_step": int(bytes_step), "achieved_gbs": round(bytes_step / sec / 1e9, 1),
                       "roofline_frac": round(bytes_step / sec / 1e9 / peak, 4),
                       "roofline_tokens_per_s": round(B * peak * 1e9 / bytes_step, 1),
                       "prefill_tokens_per_s": round(B * prefill / prefill_s, 1) if prefill_mode == "tokens" else None}
        if world > 1:
            out[str(B)]["exchange"] = modes[0]
            out[str(B)]["tokens_per_s_by_exchange"] = {k: round(B / v, 1) for k, v in per_mode.items()}
        for sq in seqs:
            sq.free(model.blocks)
    model.close()
    torch.cuda.empty_cache()
    return {"model": f"{name} architecture, INT4 g128 projections (GPU quantizer"
                     + (f", {outlier_sigma}-sigma outliers" if outlier_sigma else "") + "), f16 embed/lm_head, "
                     "random-init N(0,0.02)", "kv": "fp16 pages of 16 tokens", "prefill": prefill,
            "context": "prompt through pox_cuda_model_prefill (passes of up to 256 rows)" if prefill_mode == "tokens" else
                       "pages reserved for the prefill length (no prefill compute)",
            "parallelism": f"tp{world}" if world > 1 else "single GPU",
            "bytes_per_step": "per GPU: its weight shard + its kv heads' pages (roofline = that / measured HBM peak)",
            "decode_steps_timed": steps - 1, "build_s": round(build_s, 1), "per_batch": out}


# Small models of the tensor-parallel check, grown with the rank count so that every rank holds a kv
# head and 128-column slices of o_proj and down_proj (the shapes the multi-GPU parity tests use).
TP_CHECK_CFGS = {
    2: {"hidden": 512, "inter": 1024, "layers": 2, "n_heads": 4, "n_kv_heads": 2, "vocab": 1000,
        "rms_eps": 1e-5, "rope_theta": 500000.0},
    4: {"hidden": 512, "inter": 1024, "layers": 2, "n_heads": 8, "n_kv_heads": 4, "vocab": 1000,
        "rms_eps": 1e-5, "rope_theta": 500000.0},
    8: {"hidden": 1024, "inter": 2048, "layers": 2, "n_heads": 16, "n_kv_heads": 8, "vocab": 1000,
        "rms_eps": 1e-5, "rope_theta": 500000.0},
}


def tp_check(be, world, rank, modes=("peer", "nccl")):
    """Correctness of tensor-parallel decode in the benchmark run itself: a small random model
    (INT4 g128 with 3.5-sigma outliers) decoded tensor-parallel over `world` ranks, once per exchange,
    against the same model decoded on this rank's GPU alone -- the single-GPU path the parity tests
    check against the oracle. Three sequences (prompts of 5, 40 and 19 tokens, then 8 greedy steps),
    teacher-forced on the single-GPU greedy tokens. Returns the max |logit difference| over every
    rank's vocab slice and whether the greedy tokens agree (max / all over ranks)."""
    import torch
    import torch.distributed as dist

    from paraoxidizer_b200 import tp as TP
    from paraoxidizer_b200.model import CudaModel
    from paraoxidizer_b200.synth import load_into, make_llama

    cfg = TP_CHECK_CFGS[world]
    w = make_llama(cfg, seed=21, outlier_policy="automatic", norm_jitter=0.1)
    rng = np.random.default_rng(8)
    prompts = [list(int(t) for t in rng.integers(0, cfg["vocab"], n)) for n in (5, 40, 19)]
    steps = 8
    ref = CudaModel(be, cfg, max_batch=3, kv_blocks=24, max_blocks_per_seq=8)
    load_into(ref, w)
    feeds = [list(p) for p in prompts]
    horizon = max(len(p) for p in prompts) + steps
    ref_logits = {i: [] for i in range(3)}
    ref_next = {i: [] for i in range(3)}
    seqs = [ref.new_sequence() for _ in prompts]
    for t in range(horizon):
        act = [i for i in range(3) if t < len(prompts[i]) + steps]
        lg, nx = ref.decode([feeds[i][t] for i in act], [seqs[i] for i in act])
        for j, i in enumerate(act):
            ref_logits[i].append(lg[j])
            ref_next[i].append(int(nx[j]))
            if t + 1 >= len(prompts[i]):
                feeds[i].append(int(nx[j]))
    ref.close()
    Vl = cfg["vocab"] // world
    m = CudaModel(be, cfg, max_batch=3, kv_blocks=24 * len(modes), max_blocks_per_seq=8, tp_rank=rank, tp_size=world)
    load_into(m, TP.shard_llama(w, cfg, world, rank))
    m.init_comm(modes=modes)
    worst, agree = 0.0, 1
    for mode in modes:
        m.set_comm_mode(mode)
        seqs = [m.new_sequence() for _ in prompts]
        for t in range(horizon):
            act = [i for i in range(3) if t < len(prompts[i]) + steps]
            lg, nx = m.decode([feeds[i][t] for i in act], [seqs[i] for i in act])
            for j, i in enumerate(act):
                worst = max(worst, float(np.max(np.abs(lg[j] - ref_logits[i][t][rank * Vl:(rank + 1) * Vl]))))
                agree &= int(nx[j]) == ref_next[i][t]
    m.close()
    v = torch.tensor([worst, 1.0 - agree], dtype=torch.float64, device="cuda")
    dist.all_reduce(v, op=dist.ReduceOp.MAX)
    return {"max_abs_logit_diff": float(v[0]), "greedy_tokens_agree": bool(v[1] == 0.0), "exchanges": list(modes),
            "against": "the same model decoded on one GPU (the path the parity tests pin to the oracle)",
            "model": f"hidden {cfg['hidden']}, {cfg['layers']} layers, {cfg['n_heads']}/{cfg['n_kv_heads']} heads, "
                     f"vocab {cfg['vocab']}, INT4 g128 + 3.5-sigma outliers", "sequences": "prompts 5/40/19 + 8 steps"}


def decode_batches(args):
    spec = args.decode_batches if args.decode_batches is not None else DECODE_MODELS[args.decode_model][1]
    if spec in ("", "none"):
        return ()
    return tuple(int(b) for b in spec.split(","))


def decode_kwargs(args):
    cfg, _, ctx, mode, osig = DECODE_MODELS[args.decode_model]
    return dict(cfg=cfg, prefill=args.decode_prefill if args.decode_prefill is not None else ctx,
                prefill_mode=mode, outlier_sigma=osig, name={"llama8b": "llama-3-8b", "llama70b": "llama-3-70b"}[
                    args.decode_model])


def run_decode_only(args):
    import torch

    world, rank, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    from paraoxidizer_b200.backend import CudaBackend

    be = CudaBackend.create(local)
    bg = None
    if world == 1 and args.with_batched:
        bg = batched_gemv_bench(be, batches=tuple(int(b) for b in args.batched_sizes.split(",")))
    d = None
    if decode_batches(args):
        d = decode_bench(be, batches=decode_batches(args), steps=args.decode_steps, world=world, rank=rank,
                         **decode_kwargs(args))
    if rank == 0:
        print(json.dumps({"batched_gemv": bg, "decode": d}), flush=True)
    be.close()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


def _section(name, fn):
    """Runs one optional part of the benchmark line (batched GEMV, decode, the checks, the CPU
    baseline). A failure there is recorded in the line and on stderr, and the GEMV measurement
    already taken is still printed."""
    try:
        return fn()
    except Exception as e:  # noqa: BLE001 -- any failure of an optional part
        print(f"bench: {name} failed: {e!r}", file=sys.stderr, flush=True)
        return {"error": f"{type(e).__name__}: {e}"[:400]}


def run_ours(args):
    import torch

    world, rank, local = dist_setup(args.gpus)
    if world == 1:
        torch.cuda.set_device(0)
    dev = torch.cuda.current_device()
    from paraoxidizer_b200 import _lib as L
    from paraoxidizer_b200.backend import CudaBackend

    be = CudaBackend.create(dev)
    packed, scales, tab, ob, x = make_workload(seed=rank)
    nnz = len(tab[0])
    copies = [(packed.copy(), scales.copy(), ob.copy()) for _ in range(NCOPY)]
    tensors = [be.upload_int4(p, s, ROWS, COLS, GS, o) for p, s, o in copies]
    xd = torch.from_numpy(x).cuda()
    yd = torch.zeros(ROWS, dtype=torch.float32, device="cuda")

    stream = torch.cuda.Stream()
    G = 1000

    def capture(n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(g, stream=stream):
                s = torch.cuda.current_stream().cuda_stream
                for i in range(n):
                    tensors[i % NCOPY].gemv_device(xd.data_ptr(), 1, yd.data_ptr(), s)
        return g

    # warm-up: eager launches first (sets kernel attributes), then one graph
    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            tensors[i % NCOPY].gemv_device(xd.data_ptr(), 1, yd.data_ptr(), stream.cuda_stream)
    torch.cuda.synchronize()
    full_graphs, rem = divmod(args.steps, G)
    g_full = capture(G) if full_graphs else None
    g_rem = capture(rem) if rem else None
    g_lead = capture(64)  # replayed untimed right before the timed graphs (see below)
    with torch.cuda.stream(stream):  # CUDAGraph.replay() launches on the current stream
        for g in (g_full, g_rem, g_lead):  # first replays upload the graphs: untimed
            if g is not None:
                g.replay()
    torch.cuda.synchronize()

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    with ClockSampler(dev if world == 1 else local) as cs, torch.cuda.stream(stream):
        # 64 untimed GEMVs keep the GPU busy while the host enqueues the event and the timed graphs,
        # so the timed region holds exactly `steps` GEMVs and no host launch latency
        g_lead.replay()
        ev0.record(stream)
        for _ in range(full_graphs):
            g_full.replay()
        if g_rem is not None:
            g_rem.replay()
        ev1.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    ms = ev0.elapsed_time(ev1)
    t = torch.tensor([ms], dtype=torch.float64, device="cuda")
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = float(t.item())
    clocks = cs.summary()

    kname = tensors[0].gemv_kernel(1)
    launches_per_step = 2  # x preparation + GEMV
    bytes_per = algorithmic_bytes(nnz)
    total_bytes = bytes_per * args.steps * world
    gbs = total_bytes / (ms * 1e-3) / 1e9
    per_launch_s = ms * 1e-3 / args.steps
    peak, peak_kind = measured_peak()
    achieved = bytes_per / per_launch_s / 1e9
    traffic = profiled_traffic()

    # correctness spot-check of the timed configuration (cheap: device GEMV vs device dequant)
    ref_w = torch.empty(ROWS * COLS, dtype=torch.float32, device="cuda")
    tensors[0].dequant_device(ref_w.data_ptr(), stream.cuda_stream)
    tensors[0].gemv_device(xd.data_ptr(), 1, yd.data_ptr(), stream.cuda_stream)
    torch.cuda.synchronize()
    ref_y = ref_w.view(ROWS, COLS).double() @ xd.double()
    rel = float((yd.double() - ref_y).abs().max() / ref_y.abs().max())
    del ref_w

    # e2e: the reference-facing host-slice call (registered weights, host x in, host y out), called
    # through the C ABI with the slices' addresses taken once, as a compiled caller passes them (the
    # numpy checks of the Python wrapper are not part of the call)
    yh = np.zeros(ROWS, np.float32)
    xh = np.ascontiguousarray(x, dtype=np.float32)
    # 2000 calls whatever --steps (about 60 ms): the per-call cost in steady state; the first calls
    # of a run are about 2 us slower, which a 20-call average would carry
    e2e_steps = 2000
    fn = L.lib().pox_cuda_gemv_int4_outliers
    vp, sz = ctypes.c_void_p, ctypes.c_size_t  # converted once, as a compiled caller holds them
    call_args = [(vp(be.ctx), vp(p.ctypes.data), sz(p.size), vp(s.ctypes.data), sz(s.size), sz(GS), sz(ROWS),
                  sz(COLS), vp(o.ctypes.data), sz(o.size), vp(xh.ctypes.data), sz(xh.size), vp(yh.ctypes.data),
                  sz(yh.size)) for p, s, o in copies]
    for i in range(10):
        p, s, o = copies[i % NCOPY]
        be.gemv_int4_outliers(p, s, GS, ROWS, COLS, o, x, yh)  # the wrapper's checks, once per copy
    if world > 1:
        torch.distributed.barrier()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        rc = fn(*call_args[i % NCOPY])
        if rc:
            L.check(rc)
    e2e_s = time.perf_counter() - t0
    t = torch.tensor([e2e_s], dtype=torch.float64, device="cuda")
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    e2e_s = float(t.item())
    e2e_gbs = bytes_per * e2e_steps * world / e2e_s / 1e9

    batched = None
    if world == 1 and not args.no_decode:
        batched = _section("batched_gemv", lambda: batched_gemv_bench(be))

    decode = None
    if not args.no_decode:
        decode = _section("decode", lambda: decode_bench(be, batches=decode_batches(args), steps=args.decode_steps,
                                                         world=world, rank=rank, **decode_kwargs(args)))

    tpc = None
    decode70 = None
    if world > 1 and not args.no_decode:
        tpc = _section("tp_check", lambda: tp_check(be, world, rank))
        if not args.no_decode_70b and args.decode_model != "llama70b":
            # the Llama-3-70B configuration is quoted tensor-parallel on 2 / 4 / 8 GPUs
            a70 = argparse.Namespace(**vars(args))
            a70.decode_model, a70.decode_prefill = "llama70b", None
            decode70 = _section("decode_70b", lambda: decode_bench(be, batches=(1, 16, 64), steps=args.decode_steps_70b,
                                                                   world=world, rank=rank, **decode_kwargs(a70)))

    def cpu_leg():
        cgbs, crows, ct = cpu_baseline_sample(packed, scales, tab)
        cmodel, ncores = host_cpu()
        c = {"value": round(cgbs, 4), "unit": "GB/s", "cores": 1, "kind": "port",
             "cpu_model": cmodel, "host_cores": ncores,
             "sample": f"{crows} rows ({crows / ROWS:.2f} GEMVs) of the same workload in {ct:.1f} s through the "
                       f"oracle's quant::gemv_int4 (single-threaded, as the reference)"}
        if not args.no_decode:
            c["decode"] = _section("cpu decode", lambda: cpu_decode_baseline(be))
        return c

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = _section("cpu_baseline", cpu_leg)

    if rank == 0:
        line = {"metric": METRIC, "value": round(gbs, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None,
                "dtype": "int4 weights (g128 f16 scale/min) x activations as a 15-bit fixed point per 128-k "
                         "block (two exact int8 limbs, from f32), s32 block sums, f32 accumulate",
                "data": "synthetic (seeded N(0,0.02) weights, N(0,1) f16 x)",
                "config": {"workload": WORKLOAD, "rows": ROWS, "cols": COLS, "group_size": GS, "batch": 1,
                           "outliers": nnz, "bytes_per_step": bytes_per, "parallelism": f"replicas x{world}",
                           "l2": f"inputs larger than L2: {NCOPY} resident weight copies rotated "
                                 f"({NCOPY * bytes_per / 1e6:.0f} MB)"},
                "pct_of_peak": round(100.0 * achieved / peak, 2),
                "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                             "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                             "kernel": f"{kname}<INT4,1> with its x preparation (one step = both launches, "
                                       "PDL-overlapped, timed together with CUDA events)",
                             "traffic": traffic},
                "e2e": {"value": round(e2e_gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": COLS * 4,
                        "d2h_bytes_per_step": ROWS * 4, "steps": e2e_steps,
                        "us_per_call": e2e_s / e2e_steps * 1e6},
                "gpu_launches": launches_per_step * args.steps, "clocks": clocks, "check_max_rel": rel,
                "cpu_baseline": cpu, "batched_gemv": batched, "decode": decode}
        if tpc is not None:
            line["tp_check_max_abs"] = tpc.get("max_abs_logit_diff")
            line["tp_check"] = tpc
        if decode70 is not None:
            line["decode_70b"] = decode70
        print(json.dumps(line), flush=True)
    for tt in tensors:
        tt.free()
    be.close()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200000)
    ap.add_argument("--warmup", type=int, default=200)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true", help="skip the Llama-8B-architecture decode benchmark")
    ap.add_argument("--decode-only", action="store_true",
                    help="run only the decode benchmark (one JSON object; for launch lists and captures)")
    ap.add_argument("--with-batched", action="store_true", help="--decode-only: also run the batched GEMV bench")
    ap.add_argument("--batched-sizes", default="1,4,16,64", help="--with-batched: rows of x per call")
    ap.add_argument("--decode-model", default="llama8b", choices=sorted(DECODE_MODELS),
                    help="decode workload (the default run uses llama8b)")
    ap.add_argument("--decode-batches", default=None, help="comma list, or 'none' (default: the model's)")
    ap.add_argument("--decode-prefill", type=int, default=None, help="context before the timed steps")
    ap.add_argument("--decode-steps", type=int, default=256)
    ap.add_argument("--decode-steps-70b", type=int, default=32,
                    help="timed steps of the 70B-architecture decode that runs with --gpus >= 2")
    ap.add_argument("--no-decode-70b", action="store_true", help="with --gpus >= 2: skip the 70B decode")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.decode_only:
        return run_decode_only(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
