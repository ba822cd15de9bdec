"""Decode throughput of the 32-layer Llama-shaped f32 model
on B200, through the planned launch sequence captured as one CUDA graph.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl ours|reference]

One step is one greedy decode step of the whole model at batch B (default
1): the embedding gather, 32 planned layers (6 launches each at batch 1:
q/k/v, the fused KV store + attention, its combine, o, [gate; up], down),
the head's norm + tied LM head + argmax, and the feedback of the ids.
Weights are seeded N(0, 0.02) on the device; the KV cache holds a
512-position prompt's keys and values (seeded N(0, 1)) and decode continues
from position 512. Every step streams the 26.4 GB of weights, far more than
L2.

--impl reference times the reference's CPU path instead: the C
restatement of the FuryKernel.Cpu target's arithmetic (oracle/), whole
32-layer greedy decode steps on one thread as the CPU target runs (the 32
layer passes read one full-size layer's weights, far past any host cache),
then one step on all host threads reported beside it.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tokens/s, 32-layer Llama-shaped f32 (BASELINE config 5)"
PROMPT = 512


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--config", default="5", choices=["5", "1", "2", "3a", "3b", "3c", "4", "5g", "5h"],
                    help="5: the 32-layer decode step (default); 1, 2, 3a, 3b, 3c, 4: BASELINE's other configs; "
                         "5g, 5h: config 5's [gate;up] GEMV and its LM head alone, batch 1 (for kernel profiles)")
    ap.add_argument("--weights", default="f32", choices=["f32", "bf16", "f16"],
                    help="config 5: the model's weights (f32, the BASELINE configuration; bf16, the reference's "
                         "own element type; f16)")
    ap.add_argument("--cache", default="f32", choices=["f32", "bf16", "f16"],
                    help="config 5: the KV caches' element type")
    ap.add_argument("--block-size", type=int, default=0,
                    help="config 5: a paged KV cache of blocks of this many positions, each row's blocks its own "
                         "(0, the default: Ring caches)")
    return ap.parse_args()


def model_types(args) -> tuple:
    """Config 5's metric and dtype for the element types asked for."""
    if args.weights == "f32" and args.cache == "f32":
        return METRIC, "f32"
    kind = f"{args.weights} weights, {args.cache} KV caches, f32 activations"
    return f"decode tokens/s, 32-layer Llama-shaped, {kind} (config 5's shape)", kind


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


class Clocks:
    """nvidia-smi samples of the SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.path = tempfile.mktemp(suffix=".csv")

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.device)], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            self.proc.wait()
            self.f.close()

    def summary(self):
        rows = []
        try:
            for line in open(self.path):
                w = [x.strip() for x in line.split(",")]
                if len(w) >= 9 and w[1].replace(".", "").isdigit():
                    rows.append(w)
        except OSError:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no nvidia-smi samples"]}
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no nvidia-smi samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(float(r[1]) for r in rows), "sm_max_mhz": float(rows[0][2]),
                "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit()) if rows else None,
                "samples": len(rows), "reasons": reasons}


# ---------------------------------------------------------------------------
# The CPU path: the reference's CPU target restated (oracle/), timed


def cpu_model(batch: int, positions: int):
    """Host copies of config 5's model for the CPU path: one full-size
    layer's weights (q/k/v, o, gate/up, down, the two norm gains), the tied
    embedding and the final norm, and a Ring KV cache of `positions` for each
    of the 32 layers (keys and values N(0, 1), batch rows in their own
    slots). The 32 layer passes of a step all read the one layer's 809 MB of
    weights: far past any host cache, so a pass costs what a distinct
    layer's would. The caches are distinct a layer, as a model's are."""
    from oracle import oracle as O

    d, h, hd, f, V = 4096, 32, 128, 11008, 32000
    w = {
        "qkv": O.normal(11, 3 * d * d, 0.0, 0.02).reshape(3 * d, d),
        "o": O.normal(12, d * d, 0.0, 0.02).reshape(d, d),
        "gu": O.normal(13, 2 * f * d, 0.0, 0.02).reshape(2 * f, d),
        "down": O.normal(14, d * f, 0.0, 0.02).reshape(d, f),
        "embed": O.normal(15, V * d, 0.0, 0.02).reshape(V, d),
        "g1": O.normal(16, d, 0.0, 0.02), "g2": O.normal(17, d, 0.0, 0.02), "gf": O.normal(18, d, 0.0, 0.02),
        "kc": [O.normal(1000 + 2 * i, batch * h * positions * hd).reshape(batch, h, positions, hd)
               for i in range(32)],
        "vc": [O.normal(1001 + 2 * i, batch * h * positions * hd).reshape(batch, h, positions, hd)
               for i in range(32)],
        "positions": positions,
    }
    w["cos"], w["sin"] = O.rope_tables(10000.0, hd, hd // 2, positions)
    w["tok"] = O.ints(22, batch, V)
    return w


def cpu_step(threads: int, w: dict, tokens, pos):
    """One greedy decode step of the 32-layer model on the host, in the CPU
    target's arithmetic (oracle/): the embedding gather; each of the 32
    layers' RMSNorm + q/k/v GEMV, RoPE, the KV store at `pos`, the split
    attention over positions 0..pos, the o GEMV + residual, RMSNorm +
    gate/up GEMV, SiLU-gate, the down GEMV + residual; then the final norm,
    the tied LM head and the argmax. Returns the ids."""
    import math

    import numpy as np

    from oracle import oracle as O

    d, h, hd, f = 4096, 32, 128, 11008
    L = w["positions"]
    b = len(tokens)
    slot = np.arange(b, dtype=np.uint32)
    eps, scale = np.float32(1e-5), np.float32(1.0 / math.sqrt(hd))
    x = O.gather(w["embed"], tokens)
    for layer in range(32):
        kc, vc = w["kc"][layer], w["vc"][layer]
        qkv = O.gemv(w["qkv"], O.rmsnorm_rows(x, w["g1"], eps, 1.0, threads), 1, threads)
        kr = O.rope(qkv[:, d:2 * d], h, hd, hd // 2, pos, w["cos"], w["sin"])
        O.kv_store_ring(kr, h, hd, L, pos, slot, kc)
        O.kv_store_ring(np.ascontiguousarray(qkv[:, 2 * d:]), h, hd, L, pos, slot, vc)
        qr = O.rope(qkv[:, :d], h, hd, hd // 2, pos, w["cos"], w["sin"])
        att, _ = O.attend(qr, h, h, hd, L, pos, slot, kc, vc, scale, 128, 4, (L + 127) // 128, threads)
        x = O.add(x, O.gemv(w["o"], att, 2, threads))
        gu = O.gemv(w["gu"], O.rmsnorm_rows(x, w["g2"], eps, 1.0, threads), 1, threads)
        x = O.add(x, O.gemv(w["down"], O.silu_mul(gu[:, :f], gu[:, f:]), 2, threads))
    return O.argmax(O.gemv(w["embed"], O.rmsnorm_rows(x, w["gf"], eps, 1.0, threads), 1, threads))


def cpu_decode(threads: int, w: dict, steps: int, warmup: int):
    """Greedy decode on the host from position PROMPT: `warmup` steps, then
    the positions reset to PROMPT (as the GPU arm's are) and `steps` timed
    steps, each step's ids fed to the next. Returns the seconds a step."""
    import numpy as np

    b = len(w["tok"])
    tokens = w["tok"].astype(np.uint32)
    for i in range(warmup):
        tokens = cpu_step(threads, w, tokens, np.full(b, PROMPT + i, np.uint32))
    tokens = w["tok"].astype(np.uint32)
    t0 = time.perf_counter()
    for i in range(steps):
        tokens = cpu_step(threads, w, tokens, np.full(b, PROMPT + i, np.uint32))
    return (time.perf_counter() - t0) / steps


def cpu_step_text(b: int, steps: int, threads: int) -> str:
    return (f"{steps} whole greedy decode step(s) of the 32-layer model at batch {b} from context {PROMPT}, in "
            "the CPU target's arithmetic (oracle/, C): every layer's GEMVs, RoPE, KV store and attention and the "
            "LM head; the 32 layer passes read one full-size layer's weights (809 MB, far past any host cache), "
            f"each layer its own KV cache; {threads} thread(s)"
            + ("" if threads > 1 else ", as the CPU target runs"))


def config5(b: int, steps: int, world: int, length: int, bs: int = 0, weights: str = "f32") -> dict:
    """Config 5's workload description, the same for both arms."""
    gb = 26.4 if weights == "f32" else 13.2
    return {"workload": f"config 5 decode, batch {b}, context {PROMPT}..{PROMPT + steps}",
            "model": "llama-shaped 32 layers, d 4096, 32 heads x 128, ffn 11008, vocab 32000, tied head",
            "global_batch": b, "seq_len": PROMPT, "parallelism": f"tp{world}", "kv_length": length,
            "kv_layout": f"paged, blocks of {bs} positions" if bs else "ring",
            "l2": f"no flush: each step streams {gb} GB of weights, > 126 MB L2"}


def kv_length(b: int) -> int:
    """Config 5's KV positions: the 512-position prompt and 128 decode steps
    (640) for large batches; 4096 up to batch 4, config 5's longest."""
    return 4096 if b <= 4 else PROMPT + 128


# DRAM bytes (read + write) of one launch, from ncu captures of the same
# kernel and shape (dram__bytes_read.sum + dram__bytes_write.sum, one
# capture each; the summaries under profiles/ give the commands).
NCU_TRAFFIC = {
    ("gemv_rmsnorm_silu", 22016, 4096, 1): (360.78e6 + 3.81e6, "profiles/gemv_stream_gateup_b1.md"),
    ("gemv_rmsnorm", 32000, 4096, 1): (524.35e6 + 3.51e6, "profiles/gemv_stream_lm_head_b1.md"),
    ("gemv", 11008, 4096, 16): (180.90e6 + 3.87e6, "profiles/gemv_batch_b16.md"),
    ("gemm_tf32x3w", 512, 11008, 4096): (285.73e6 + 22.33e6, "profiles/gemm_tf32x3w_3c.md"),
}


def kernel_roofline(ctx, eng, L, local: int, peak: float, peak_kind: str, b: int, share: float) -> dict:
    """One GEMV launch of the step timed alone (20 launches after 3, CUDA
    events on the context's stream), against the measured HBM peak: its
    algorithmic bytes (the weights once, x and y) over its mean duration."""
    import torch

    for _ in range(3):
        L.run(ctx)
    ctx.sync()
    stream = torch.cuda.ExternalStream(ctx.stream())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 20
    e0.record(stream)
    for _ in range(reps):
        L.run(ctx)
    e1.record(stream)
    e1.synchronize()
    k_ms = e0.elapsed_time(e1) / reps
    p = L.params
    outs = p["n"] // 2 if "_silu" in L.kernel and "rmsnorm" in L.kernel else p["n"]  # a row pair, one output
    k_bytes = eng.wb * (p["n"] * p["k"] + p["k"]) + 4 * (p["m"] * p["k"] + p["m"] * outs)
    k_gbs = k_bytes / (k_ms / 1e3) / 1e9
    traffic = NCU_TRAFFIC.get((L.kernel, p["n"], p["k"], p["m"]), (None, None))
    return {"kernel": "%s %d x %d, batch %d" % (L.kernel, p["n"], p["k"], b), "bound": "hbm",
            "achieved": k_gbs, "peak": peak, "unit": "GB/s", "frac": k_gbs / peak, "traffic": traffic[0],
            "traffic_source": traffic[1], "algorithmic_bytes": k_bytes, "launch_ms": k_ms, "peak_kind": peak_kind,
            "weight_share_of_step": share}


GEN_STEPS = 128


def generation_run(eng, graph, tokens, seqs, prefill: dict) -> dict:
    """Config 5's whole request after its prompt: GEN_STEPS greedy decode
    steps from position PROMPT (the captured step replayed, each feeding
    its ids to the next, device-timed), and with the prompt's prefill time
    the request's generated tokens a second."""
    import numpy as np

    b = len(tokens)
    eng.set_rows(tokens, np.full(b, PROMPT, np.uint32), seqs)
    ms = graph.time(0, GEN_STEPS)
    return {"prompt": PROMPT, "decode_steps": GEN_STEPS, "contexts": f"{PROMPT}..{PROMPT + GEN_STEPS}",
            "decode_ms": ms, "decode_tokens_per_s": b * GEN_STEPS / (ms / 1e3),
            "prefill_ms": prefill["ms"],
            "request_tokens_per_s": b * GEN_STEPS / ((ms + prefill["ms"]) / 1e3),
            "note": "generated tokens over the prompt's prefill plus the decode steps, device time"}


def prompt_prefill(ctx, eng, b: int, local: int, tables=None):
    """Config 5's prompt: b prompts of PROMPT ids U[0, vocab) (numpy PCG64,
    seed 512, the same on every rank), every row but the last prefilled
    through the layers with the 3xTF32 GEMMs, then one decode step from the
    last ids. With a paged cache, `tables` holds each prompt's block table.
    Returns (the first generated ids, the prefill's line)."""
    import numpy as np
    import torch

    from furykernel_b200.prefill import Prefill, prompt_chunks, prompt_rows

    prompts = np.random.default_rng(512).integers(0, eng.full.vocab, size=(b, PROMPT), dtype=np.uint32)
    slots = np.arange(b, dtype=np.uint32)
    toks, poss, sl = prompt_rows(prompts, slots)
    R = PROMPT - 1  # one prompt a run: the query-tiled prompt attention
    pre = Prefill(eng, rows=R, positions=PROMPT, one_slot=True)
    chunks = prompt_chunks(pre, toks, poss, sl)
    # Capture, then one untimed pass (a graph's first replay uploads it, and
    # NCCL's first captured collectives set up): prefill writes the same
    # keys and values again in the timed pass.
    seq = sl if tables is None else tables[sl]  # each row's slot, or its block table
    for i, m in chunks:
        pre.run(toks[i:i + m], poss[i:i + m], seq[i:i + m])
    ctx.sync()
    torch.cuda.set_device(local)
    stream = torch.cuda.ExternalStream(ctx.stream())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i, m in chunks:
        pre.run(toks[i:i + m], poss[i:i + m], seq[i:i + m])
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1)
    rows = len(toks)
    flops = pre.gemm_flops(rows)
    pre.close()
    eng.set_rows(prompts[:, -1], np.full(b, PROMPT - 1, np.uint32), slots if tables is None else tables)
    ids = eng.step()
    info = {"prompts": b, "prompt_len": PROMPT, "rows": rows, "launch_rows": R, "ms": ms,
            "tokens_per_s": rows / (ms / 1e3), "gemm_flops_per_gpu": flops,
            "gemm_tflops_per_gpu": flops / (ms / 1e3) / 1e12,
            "note": "every prompt row but the last through the layers (tcgen05 3xTF32 GEMMs); the last row is the "
                    "first decode step; row uploads (synchronous) between launch groups are inside the time"}
    return ids, info


def cpu_positions(args) -> int:
    """The host caches' ring length: the prompt, the decode steps and one,
    rounded up to the attention's chunk of 128."""
    need = PROMPT + max(args.steps, args.warmup) + 1
    return (need + 127) // 128 * 128


def run_reference(args):
    """The reference's CPU path on the host: the CPU target's arithmetic
    (oracle/, the C restatement of FuryKernel.Cpu: no GHC or rustc on this
    image), whole 32-layer greedy decode steps, one thread as the CPU target
    runs (src/FuryKernel/Cpu.hs:259-266). Rank 0 alone runs; the other ranks
    exit. After the timed steps, one step on all host threads (OpenMP over
    rows and heads, a variant of ours) is reported beside it."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle as O

    O.build()
    b = args.batch
    w = cpu_model(b, cpu_positions(args))
    per_step = cpu_decode(1, w, args.steps, args.warmup)
    value = b / per_step
    threads = os.cpu_count() or 1
    omp = cpu_decode(threads, w, 1, 0)
    metric, dtype = model_types(args)
    line = {
        "impl": "reference", "metric": metric, "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_step * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": dtype,
        "data": "synthetic: seeded N(0,0.02) weights, N(0,1) KV caches of the 512-position prompt, seeded ids",
        "config": config5(b, args.steps, args.gpus, kv_length(b), args.block_size, args.weights),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": 1, "kind": "port",
                         "sample": cpu_step_text(b, args.steps, 1)
                                   + ("" if dtype == "f32" else
                                      "; 16-bit weights and caches are the same arithmetic over widened values")},
        "cpu_openmp": {"value": b / omp, "unit": "tokens/s", "cores": threads, "kind": "port (ours: OpenMP)",
                       "sample": cpu_step_text(b, 1, threads)},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# Ours


def run_ours(args):
    import ctypes

    import numpy as np

    from furykernel_b200 import _native as N
    from furykernel_b200.engine import Llama
    from furykernel_b200.shape import LlamaShape

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        from furykernel_b200 import tp

        if args.block_size:
            raise SystemExit("bench: --block-size is for one GPU; the tensor-parallel bench runs Ring caches.")
        length = kv_length(args.batch)
        return tp.bench_main(args, model_types(args)[0], PROMPT, prompt_prefill,
                             lambda world, n: config5(args.batch, args.steps, world, n, 0, args.weights), length,
                             Clocks, generation_run)

    metric, dtype = model_types(args)
    b = args.batch
    length = kv_length(b)
    bs = args.block_size
    paged = {}
    if bs:  # a pool of blocks, each row's table its own blocks (distinct entries)
        table_len = (length + bs - 1) // bs
        paged = {"blocks": b * table_len, "block_size": bs}
    shape = LlamaShape(layers=args.layers, slots=b, length=length, positions=length, weights=args.weights,
                       cache=args.cache, **paged)
    ctx = N.Context(local)
    eng = Llama(ctx, shape, b, seed=2026, chunk=32)
    tables = np.arange(b * table_len, dtype=np.uint32).reshape(b, table_len) if bs else None
    tokens, prefill = prompt_prefill(ctx, eng, b, local, tables)
    slots = np.arange(b, dtype=np.uint32)
    seqs = slots if tables is None else tables
    eng.set_rows(tokens, np.full(b, PROMPT, np.uint32), seqs)
    graph = eng.capture()
    for _ in range(args.warmup):
        graph.launch()
    ctx.sync()
    eng.set_rows(tokens, np.full(b, PROMPT, np.uint32), seqs)
    with Clocks(local) as clk:
        ms = graph.time(0, args.steps)
    clocks = clk.summary()
    ms_step = ms / args.steps
    value = b * args.steps / (ms / 1e3)
    hbm_peak, peak_kind = peaks()
    contexts = [PROMPT + args.steps / 2] * b
    step_bytes = eng.algorithmic_bytes(contexts)
    step_gbs = step_bytes / (ms_step / 1e3) / 1e9

    # The dominant kernel: the GEMV shape that streams the most weight bytes
    # a step (the [gate; up] GEMV, 32 launches), timed alone by CUDA events
    # on the context's stream; the LM head (the largest single launch)
    # beside it.
    import torch

    torch.cuda.set_device(local)
    gemvs = [L for L in eng.launches if L.kernel.startswith("gemv")]
    per_shape = {}
    for L in gemvs:
        key = (L.kernel, L.params["n"], L.params["k"])
        per_shape[key] = per_shape.get(key, 0) + L.params["n"] * L.params["k"]
    dominant = max(per_shape, key=per_shape.get)
    L_dom = next(L for L in gemvs if (L.kernel, L.params["n"], L.params["k"]) == dominant)
    L_head = max(gemvs, key=lambda L: L.params["n"] * L.params["k"])
    roof = {}
    for name, L in (("dominant", L_dom), ("lm_head", L_head)):
        roof[name] = kernel_roofline(ctx, eng, L, local, hbm_peak, peak_kind, b,
                                     share=per_shape[(L.kernel, L.params["n"], L.params["k"])] /
                                     sum(per_shape.values()))

    # End to end through the C ABI: host token ids and positions in (pinned),
    # the graph replayed, the greedy ids back, every step.
    rs = eng.row_stride
    host_in = N.pinned((eng.rows_words,), np.uint32)
    host_out = N.pinned((b,), np.uint32)
    host_in[:] = 0
    host_in[:b] = tokens
    host_in[rs:rs + b] = PROMPT
    host_in[2 * rs:2 * rs + seqs.size] = seqs.reshape(-1)
    rows_ptr = eng.rows.ptr
    for _ in range(3):
        N.check(N.lib().fkc_step(ctx.handle, graph.handle, host_in.ctypes.data, rows_ptr, host_in.nbytes,
                                 host_out.ctypes.data, eng.out_ids.ptr, host_out.nbytes))
    host_in[rs:rs + b] = PROMPT
    t0 = time.perf_counter()
    for _ in range(args.steps):
        N.check(N.lib().fkc_step(ctx.handle, graph.handle, host_in.ctypes.data, rows_ptr, host_in.nbytes,
                                 host_out.ctypes.data, eng.out_ids.ptr, host_out.nbytes))
        host_in[:b] = host_out
        host_in[rs:rs + b] += 1
    e2e_s = time.perf_counter() - t0
    e2e = b * args.steps / e2e_s
    generation = generation_run(eng, graph, tokens, seqs, prefill)

    line = {
        "metric": metric, "value": value, "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": dtype,
        "data": "synthetic: seeded N(0,0.02) weights made on the device; prompts of 512 ids U[0,32000) (numpy "
                "PCG64 seed 512) prefilled through the model",
        "config": config5(b, args.steps, 1, length, bs, args.weights),
        "hbm": {"step_algorithmic_bytes": step_bytes, "achieved_gbs": step_gbs,
                "frac_of_8tbs": step_gbs / 8000.0, "frac_of_peak": step_gbs / hbm_peak, "peak": hbm_peak,
                "peak_kind": peak_kind},
        "roofline": roof["dominant"],
        "roofline_lm_head": roof["lm_head"],
        "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": int(host_in.nbytes),
                "d2h_bytes_per_step": int(host_out.nbytes)},
        "gpu_launches": eng.launch_count() * args.steps,
        "clocks": clocks,
        "prefill": prefill,
        "generation": generation,
    }
    if not args.no_cpu_baseline and rank == 0:
        steps = 2
        t = cpu_decode(1, cpu_model(b, (PROMPT + steps + 127) // 128 * 128), steps, 0)
        line["cpu_baseline"] = {"value": b / t, "unit": "tokens/s", "cores": 1, "kind": "port",
                                "sample": cpu_step_text(b, steps, 1)}
    print(json.dumps(line), flush=True)
    graph.destroy()
    ctx.close()


def run_gemm(args):
    """Config 3c: C[512, 11008] = A[512, 4096] W^T on tcgen05 (3xTF32),
    gemm_tf32x3w: W read as f32 and split into TF32 halves inside the
    kernel, A split in every call. With N ranks, each computes 11008 / N
    columns (no collective); the time is the max over ranks."""
    import numpy as np
    import torch

    from furykernel_b200 import _native as N

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    M, K, NN = 512, 4096, 11008
    n = NN // world
    ctx = N.Context(local)
    a, w = ctx.empty((M, K)), ctx.empty((n, K))
    ctx.fill_normal(a, 31, 0.0, 1.0)
    ctx.fill_normal(w, 32 + rank, 0.0, 0.02)
    ahi, alo, c = ctx.empty((M, K)), ctx.empty((M, K)), ctx.empty((M, n))
    params = {"M": M, "N": n, "K": K, "ldc": n}
    bufs = [a, ahi, alo, w, c]
    kernel = "gemm_tf32x3w"
    # One call (the split of A, C zeroed where the GEMM splits K, the GEMM)
    # captured once and replayed: the device time of the launches, without
    # the host's tensor-map encoding between calls.
    ctx.capture_begin()
    ctx.launch(kernel, params, bufs)
    graph = ctx.capture_end()
    for _ in range(args.warmup):
        graph.launch()
    assert ctx.status() == 0
    torch.cuda.set_device(local)
    stream = torch.cuda.ExternalStream(ctx.stream())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    ctx.sync()
    with Clocks(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            graph.launch()
        e1.record(stream)
        e1.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    status = ctx.status()
    graph.destroy()
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    useful = 2.0 * M * K * NN
    tflops = useful / (ms / 1e3) / 1e12
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            bf16 = float(json.load(f)["bf16_tflops"])
        kind = "measured bf16 / 2"
    except (OSError, KeyError, ValueError):
        bf16, kind = 1590.0, "fallback bf16 / 2"
    tf32_peak = bf16 / 2
    if rank == 0:
        line = {
            "metric": "GEMM TFLOP/s (useful 2MNK), f32 as 3xTF32 on tcgen05 (BASELINE config 3c)", "value": tflops,
            "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32 (3xTF32)",
            "data": "synthetic: A N(0,1), W N(0,0.02), seeded on the device",
            "config": {"workload": "config 3c prefill GEMM [512 x 4096] x [4096 x 11008]", "M": M, "K": K, "N": NN,
                       "parallelism": f"column split over {world}", "status": status, "kernel": kernel,
                       "tile": "%d rows of A x 128 rows of W on %d CTAs" % gemm_tile(M, n, K, ctx.sms),
                       "l2": "inputs 8 + 180 MB per call (> L2 for the weights)"},
            "roofline": {"bound": "tensor", "achieved": 3 * tflops, "peak": tf32_peak, "unit": "TFLOP/s",
                         "frac": 3 * tflops / tf32_peak,
                         "traffic": NCU_TRAFFIC[("gemm_tf32x3w", M, NN, K)][0] if world == 1 else None,
                         "traffic_source": NCU_TRAFFIC[("gemm_tf32x3w", M, NN, K)][1], "peak_kind": kind,
                         "note": "achieved counts the 3 TF32 products the tensor pipe runs"},
            "gpu_launches": 2 * args.steps, "clocks": clk.summary(),  # split_tf32 of A, then the GEMM (+ a memset node)
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = gemm_cpu_baseline(M, K, NN)
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        dist.destroy_process_group()


def gemm_tile(M: int, N: int, K: int, sms: int) -> tuple:
    """gemm_tf32x3w's tile for M x N x K (the launcher's rule, restated):
    (tm A rows against 128 W rows, G CTAs), G = tiles, 2 tiles or (more
    tiles than SMs) sms, the least modelled time: a CTA's slabs of 16 x
    6 (138 + 0.117 tm) + its pieces x (500 + 8 tm)."""
    wt, S = (N + 127) // 128, K // 16
    best, best_cost = (256, 1), float("inf")
    for tm in range(256, 15, -16):
        tiles = wt * -(-M // tm)
        slab, epi = 6 * (138.0 + 0.117 * tm), 500.0 + 8.0 * tm
        for g, G in enumerate((tiles, 2 * tiles, sms)):
            if G > sms or (g == 1 and S < 2) or (g == 2 and tiles <= sms):
                continue
            per = -(-tiles * S // G)
            pieces = 1.0 if g < 2 else -(-per // S) + 1.0
            cost = per * slab + pieces * epi
            if cost < best_cost:
                best, best_cost = (tm, G), cost
    return best


def gemm_cpu_baseline(M: int, K: int, N: int, rows: int = 4) -> dict:
    """Config 3c on the host as the CPU target computes it (gemmTile: each
    element a sequential binary32 sum over k, oracle/fko_gemm_tile), one
    thread, on `rows` of A's M rows, scaled to the whole product."""
    from oracle import oracle as O

    a = O.normal(31, rows * K).reshape(rows, K)
    w = O.normal(32, N * K, 0.0, 0.02).reshape(N, K)
    t0 = time.perf_counter()
    O.gemm_tile(a, w, 1)
    s = (time.perf_counter() - t0) * M / rows
    return {"value": 2.0 * M * N * K / s / 1e12, "unit": "TFLOP/s", "cores": 1, "kind": "port",
            "sample": f"{rows} of the {M} rows of A against all of W, gemmTile's order (k in order), 1 thread, "
                      "scaled to all rows", "ms": s * 1e3}


def time_graph(ctx, launches, steps, warmup, rotate=None):
    """Device time (ms) of one replay of the launches captured as a graph,
    averaged over `steps` replays after `warmup`. With `rotate`, a list of
    launch lists over distinct input copies, each replay takes the next
    (inputs then come from HBM, not L2)."""
    graphs = []
    for ls in rotate or [launches]:
        ctx.capture_begin()
        for L in ls:
            L.run(ctx)
        graphs.append(ctx.capture_end())
    import torch

    stream = torch.cuda.ExternalStream(ctx.stream())
    for i in range(warmup):
        graphs[i % len(graphs)].launch()
    ctx.sync()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        graphs[i % len(graphs)].launch()
    e1.record(stream)
    e1.synchronize()
    for g in graphs:
        g.destroy()
    return e0.elapsed_time(e1) / steps


def run_kernel_config(args):
    """Configs 1, 2, 3a, 3b and 4, one GPU: device time a launch sequence,
    HBM bytes against the measured peak, and the CPU target's arithmetic
    (oracle) timed on one core over the same input."""
    import numpy as np
    import torch

    from furykernel_b200 import _native as N
    from furykernel_b200.engine import Launch, Llama
    from furykernel_b200.shape import LlamaShape
    from oracle import oracle as O

    torch.cuda.set_device(0)
    ctx = N.Context(0)
    peak, kind = peaks()
    cfg = args.config
    cpu_ms, cpu_sample_text = None, ""
    if cfg == "1":
        n = 16_777_216
        xs = [ctx.empty(n) for _ in range(4)]
        for i, x in enumerate(xs):
            ctx.fill_uniform(x, 100 + i, -1.0, 1.0)
        part, y = ctx.empty(n // 256), ctx.empty(1)
        rot = [[Launch("reduce_groups", {"n": n}, [x.ptr, part.ptr]),
                Launch("reduce_final", {"count": n // 256}, [part.ptr, y.ptr])] for x in xs]
        ms = time_graph(ctx, None, args.steps, args.warmup, rotate=rot)
        nbytes, workload, unit_label = 4 * n, "config 1: tree reduction of 16,777,216 f32 (4 rotating copies)", "sums/s"
        host = O.uniform(100, n, -1.0, 1.0)
        t0 = time.perf_counter()
        O.reduce_sum(host, 1)
        cpu_ms = (time.perf_counter() - t0) * 1e3
        cpu_sample_text = "one whole sum, fko_reduce_sum, 1 thread"
    elif cfg == "2":
        rows = h = 4096
        x, g, y, z = ctx.empty((rows, h)), ctx.empty(h), ctx.empty((rows, h)), ctx.empty((rows, h))
        ctx.fill_normal(x, 11, 0.0, 1.0)
        ctx.fill_uniform(g, 12, 0.5, 1.5)
        ls = [Launch("rmsnorm_rows", {"rows": rows, "h": h, "eps": 1e-5, "factor": 1.0}, [x.ptr, g.ptr, y.ptr]),
              Launch("softmax_rows", {"rows": rows, "h": h}, [y.ptr, z.ptr])]
        ms = time_graph(ctx, ls, args.steps, args.warmup)
        nbytes, workload, unit_label = 2 * 2 * 4 * rows * h + 4 * h, "config 2: RMSNorm then softmax, 4096 x 4096 f32", "passes/s"
        hx = O.normal(11, rows * h).reshape(rows, h)
        hg = O.uniform(12, h, 0.5, 1.5)
        t0 = time.perf_counter()
        O.softmax_rows(O.rmsnorm_rows(hx, hg, 1e-5, 1.0, 1), 1)
        cpu_ms = (time.perf_counter() - t0) * 1e3
        cpu_sample_text = "the whole pass, fko_rmsnorm_rows + fko_softmax_rows, 1 thread"
    elif cfg in ("5g", "5h"):
        # One layer's [gate; up] GEMV (rows interleaved, the RMSNorm prologue,
        # the SiLU-pair epilogue) or the LM head (the RMSNorm prologue), as
        # the config-5 step launches them at batch 1: 4 copies of the weights
        # in rotation, so that each launch streams its weights from HBM.
        n, kern = (22016, "gemv_rmsnorm_silu") if cfg == "5g" else (32000, "gemv_rmsnorm")
        k = 4096
        # --weights bf16 / f16: the 16-bit form of the launch (weights and
        # gain in that type, x and y f32), as the config-5 step with those
        # weights launches it.
        wt = args.weights
        eb = 4 if wt == "f32" else 2
        kern += {"f32": "", "bf16": "_wbf16", "f16": "_wf16"}[wt]
        x, y = ctx.empty((1, k)), ctx.empty((1, n))
        ctx.fill_normal(x, 2, 0.0, 1.0)
        if wt == "f32":
            g = ctx.empty(k)
            ctx.fill_uniform(g, 3, 0.5, 1.5)
        else:
            g = ctx.empty(k, np.uint16)
            (ctx.fill_normal_bf16 if wt == "bf16" else ctx.fill_normal_f16)(g, 3, 1.0, 0.25)
        ws = [ctx.empty((n, k), np.float32 if wt == "f32" else np.uint16) for _ in range(4)]
        for i, w in enumerate(ws):
            if wt == "f32":
                ctx.fill_normal(w, 10 + i, 0.0, 0.02)
            else:
                (ctx.fill_normal_bf16 if wt == "bf16" else ctx.fill_normal_f16)(w, 10 + i, 0.0, 0.02)
        p = {"n": n, "k": k, "m": 1, "split": 1, "ldx": k, "ldy": n // 2 if cfg == "5g" else n, "eps": 1e-5,
             "factor": 1.0}
        rot = [[Launch(kern, p, [w.ptr, x.ptr, g.ptr, y.ptr])] for w in ws]
        ms = time_graph(ctx, None, args.steps, args.warmup, rotate=rot)
        outs = n // 2 if cfg == "5g" else n
        nbytes = eb * (n * k + k) + 4 * (k + outs)
        workload = f"config 5's {'[gate; up] GEMV' if cfg == '5g' else 'LM head'} {n} x {k}, batch 1 ({kern})"
        unit_label = "GEMVs/s"
    elif cfg in ("3a", "3b"):
        m = 1 if cfg == "3a" else 16
        n, k = 11008, 4096
        w, x, y = ctx.empty((n, k)), ctx.empty((m, k)), ctx.empty((m, n))
        ctx.fill_normal(w, 21, 0.0, 0.02)
        ctx.fill_normal(x, 22, 0.0, 1.0)
        split = 1  # the streaming (m <= 4) and batched (m <= 64) kernels keep one
        ls = [Launch("gemv", {"n": n, "k": k, "m": m, "split": split, "ldx": k, "ldy": n}, [w.ptr, x.ptr, y.ptr])]
        ms = time_graph(ctx, ls, args.steps, args.warmup)
        nbytes = 4 * (n * k + m * k + m * n)
        workload, unit_label = f"config 3{'a' if m == 1 else 'b'}: GEMV 11008 x 4096 f32, batch {m}", "GEMVs/s"
        hw = O.normal(21, n * k, 0.0, 0.02).reshape(n, k)
        hx = O.normal(22, m * k).reshape(m, k)
        rows = 1024 if m > 1 else n
        t0 = time.perf_counter()
        O.gemv(hw[:rows], hx, split, 1)
        cpu_ms = (time.perf_counter() - t0) * 1e3 * n / rows
        cpu_sample_text = f"fko_gemv over {rows} of the 11008 rows, 1 thread, scaled to all rows"
    else:  # config 4: one layer, context 2048
        b = args.batch
        s = LlamaShape(layers=1, slots=b, length=2304, positions=2304)
        eng = Llama(ctx, s, b, seed=2026, chunk=32, prefill_kv=1.0)
        eng.set_rows(np.arange(b, dtype=np.uint32) + 1, np.full(b, 2048, np.uint32), np.arange(b, dtype=np.uint32))
        eng.run_eager()
        ctx.sync()
        per_layer = (len(eng.launches) - 4) // s.layers  # gather | layers | head, argmax, advance
        layer = eng.launches[1:1 + per_layer]
        assert "attend_decode" in [L.kernel for L in layer] or "attend_split" in [L.kernel for L in layer], \
            [L.kernel for L in layer]
        ctx.set_pdl(True)
        ms = time_graph(ctx, layer, args.steps, args.warmup)
        ctx.set_pdl(False)
        nbytes = eng.weight_bytes() - 4 * (eng.vocab_local * s.d_model + s.d_model) + \
            b * 2 * s.kv_heads * s.head_dim * 4 * 2049
        workload, unit_label = f"config 4: one Llama-shaped layer, decode at context 2048, batch {b}", "tokens/s"
    gbs = nbytes / (ms / 1e3) / 1e9
    value = (args.batch if cfg == "4" else 1) / (ms / 1e3)
    line = {"metric": workload, "value": value, "unit": unit_label, "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None,
            "dtype": f"{args.weights} weights, f32 arithmetic" if cfg in ("5g", "5h") and args.weights != "f32" else "f32",
            "data": "synthetic, seeded on the device",
            "config": {"workload": workload},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                         "traffic": NCU_TRAFFIC[("gemv", 11008, 4096, 16)][0] if cfg == "3b" else None,
                         "algorithmic_bytes": nbytes, "peak_kind": kind}}
    if cpu_ms is not None:
        line["cpu_baseline"] = {"value": 1e3 / cpu_ms, "unit": unit_label, "cores": 1, "kind": "port",
                                "sample": cpu_sample_text, "ms": cpu_ms}
    print(json.dumps(line), flush=True)
    ctx.close()


def main():
    args = parse()
    if args.config == "3c":
        return run_gemm(args)
    if args.config in ("1", "2", "3a", "3b", "4", "5g", "5h"):
        return run_kernel_config(args)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
