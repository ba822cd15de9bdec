"""Tensor parallelism across the GPUs of one box: one process per GPU.

torch.distributed (NCCL) is the plumbing: the group's rendezvous, barriers,
the exchange of the shim's NCCL unique id and of the peer regions' IPC
handles, and the max over ranks of a timing. The data path -- the sum after
each row-parallel projection and the gather of the greedy candidates -- runs
inside the captured decode graph on the context's stream: over NVLink peer
memory for decode batches of up to 4 rows (the row-parallel GEMV writes its
partial rows into every rank's region and the next GEMV's prologue sums
them, fk_peers.cuh), and on the shim's own NCCL communicator for larger
batches, the prompt prefill and routed-expert models.
"""

from __future__ import annotations

import datetime
import json
import os
import time

import numpy as np

from . import _native as N


def init(timeout_s: int = 120):
    """(ctx, rank, world, local): the context of this rank's GPU with an NCCL
    communicator over all ranks."""
    import torch
    import torch.distributed as dist

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    if not dist.is_initialized():
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=timeout_s),
                                device_id=torch.device("cuda", local))
    ctx = N.Context(local)
    uid = [N.Context.comm_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    ctx.comm_init(world, rank, uid[0])
    peer_set(ctx, rank, world)
    return ctx, rank, world, local


def peer_set(ctx, rank: int, world: int) -> None:
    """Every rank's exchange region mapped into this process (IPC handles
    gathered over the process group), registered with the context."""
    import ctypes

    import torch.distributed as dist

    L = N.lib()
    local = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(64)
    N.check(L.fkc_peer_alloc(ctx.handle, L.fkc_peer_region_bytes(), ctypes.byref(local), handle))
    handles = [None] * world
    dist.all_gather_object(handles, handle.raw)
    regions = (ctypes.c_void_p * world)()
    for q in range(world):
        if q == rank:
            regions[q] = local.value
        else:
            p = ctypes.c_void_p()
            N.check(L.fkc_peer_open(ctx.handle, ctypes.create_string_buffer(handles[q], 64), ctypes.byref(p)))
            regions[q] = p.value
    N.check(L.fkc_peer_set(ctx.handle, world, rank, regions))
    dist.barrier()


def finish(ctx, graphs=()) -> None:
    """Graphs holding NCCL calls go first, then the communicator, then the group."""
    import torch.distributed as dist

    for g in graphs:
        if g is not None:
            g.destroy()
    ctx.comm_destroy()
    ctx.close()
    if dist.is_initialized():
        dist.destroy_process_group()


def max_over_ranks(v: float) -> float:
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def peer_wait_profile(ctx, eng, steps: int) -> dict:
    """How long the peer exchanges of a step wait, after the timed run: the
    step captured again with wait statistics on (each waiting block adds its
    wait, fkc_set_wait_stats) and replayed `steps` times on every rank.
    Reports, over ranks, the mean time a block waited at one exchange and
    the exchanges of a step; their product is the time a rank's blocks
    spend waiting for their peers in a step."""
    import torch.distributed as dist

    exchanges = sum(1 for L in eng.launches if L.kernel.startswith(("gemv_reduce_rmsnorm", "argmax_gather_pick")))
    ctx.set_wait_stats(True)
    eng.graph = None
    g = eng.capture()
    ctx.set_wait_stats(False)
    dist.barrier()
    ctx.sync()
    ms = g.time(1, steps)
    ns, n = ctx.read_wait_stats()
    g.destroy()
    eng.graph = None
    per_wait_us = ns / max(n, 1) / 1e3
    import torch

    t = torch.tensor([per_wait_us, ms / steps], dtype=torch.float64, device="cuda")
    got = [torch.zeros_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(got, t)
    per_rank = [float(x[0]) for x in got]
    return {"us_per_block_wait_by_rank": per_rank, "exchanges_per_step": exchanges,
            "us_waited_per_step_max_rank": max(per_rank) * exchanges,
            "ms_per_step_with_stats_max_rank": max(float(x[1]) for x in got),
            "note": "mean over the waiting blocks of one exchange's wait (device clock), from a separate capture "
                    "with wait statistics on; not inside the timed region"}


def bench_main(args, metric: str, prompt: int, prefill_fn, config_fn, length: int, clocks_cls=None,
               generation_fn=None) -> None:
    """The decode bench at N ranks: each rank replays its shard's captured
    step; the step time is the max over ranks of the device-timed replays.
    `config_fn(world, length)` describes the workload; `clocks_cls(device)`,
    when given, samples the SM clocks of rank 0's GPU over the timed
    replays."""
    import contextlib

    import torch.distributed as dist

    from .engine import Llama
    from .shape import LlamaShape

    ctx, rank, world, local = init()
    b = args.batch
    wt, ct = getattr(args, "weights", "f32"), getattr(args, "cache", "f32")
    shape = LlamaShape(layers=args.layers, slots=b, length=length, positions=length, weights=wt, cache=ct)
    eng = Llama(ctx, shape, b, seed=2026, chunk=32, rank=rank, world=world)
    tokens, prefill = prefill_fn(ctx, eng, b, local)
    prefill["ms"] = max_over_ranks(prefill["ms"])
    prefill["tokens_per_s"] = prefill["rows"] / (prefill["ms"] / 1e3)
    prefill["gemm_tflops_per_gpu"] = prefill["gemm_flops_per_gpu"] / (prefill["ms"] / 1e3) / 1e12
    slots = np.arange(b, dtype=np.uint32)
    eng.set_rows(tokens, np.full(b, prompt, np.uint32), slots)
    graph = eng.capture()
    for _ in range(args.warmup):
        graph.launch()
    ctx.sync()
    eng.set_rows(tokens, np.full(b, prompt, np.uint32), slots)
    # Rank 0's clock sampler starts (and settles) before the barrier, so
    # that every rank's timed replays start together: a rank that starts
    # late holds the others in their peer exchanges.
    clk = clocks_cls(local) if (clocks_cls is not None and rank == 0) else contextlib.nullcontext()
    with clk:
        dist.barrier()
        ctx.sync()
        ms = graph.time(0, args.steps)
    dist.barrier()
    ms = max_over_ranks(ms)
    ms_step = ms / args.steps
    value = b * args.steps / (ms / 1e3)

    # End to end through the C ABI on every rank: the same host inputs in,
    # the ids out, each step; the max over ranks of the wall time.
    rs = eng.row_stride
    host_in = N.pinned((3 * rs,), np.uint32)
    host_out = N.pinned((b,), np.uint32)
    host_in[:] = 0
    host_in[:b] = tokens
    host_in[rs:rs + b] = prompt
    host_in[2 * rs:2 * rs + b] = slots
    dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        N.check(N.lib().fkc_step(ctx.handle, graph.handle, host_in.ctypes.data, eng.rows.ptr, host_in.nbytes,
                                 host_out.ctypes.data, eng.out_ids.ptr, host_out.nbytes))
        host_in[:b] = host_out
        host_in[rs:rs + b] += 1
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    per_rank = eng.algorithmic_bytes([prompt + args.steps / 2] * b)
    waits = peer_wait_profile(ctx, eng, args.steps) if eng.peer_exchange else None
    generation = None
    if generation_fn is not None:
        dist.barrier()
        generation = generation_fn(eng, graph, tokens, slots, prefill)
        generation["decode_ms"] = max_over_ranks(generation["decode_ms"])
    if rank == 0:
        line = {
            "metric": metric, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None,
            "dtype": "f32" if (wt, ct) == ("f32", "f32") else f"{wt} weights, {ct} KV caches, f32 activations",
            "data": "synthetic: seeded N(0,0.02) weights made on the device; prompts of 512 ids U[0,32000) (numpy "
                    "PCG64 seed 512) prefilled through the model",
            "config": config_fn(world, length),
            "hbm": {"per_gpu_step_bytes": per_rank, "per_gpu_achieved_gbs": per_rank / (ms_step / 1e3) / 1e9},
            "e2e": {"value": b * args.steps / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": int(host_in.nbytes),
                    "d2h_bytes_per_step": int(host_out.nbytes)},
            "gpu_launches": eng.launch_count() * args.steps,
            "prefill": prefill,
        }
        if clocks_cls is not None:
            line["clocks"] = clk.summary()
        if waits is not None:
            line["peer_waits"] = waits
        if generation is not None:
            g = generation
            g["decode_tokens_per_s"] = b * g["decode_steps"] / (g["decode_ms"] / 1e3)
            g["request_tokens_per_s"] = b * g["decode_steps"] / ((g["decode_ms"] + g["prefill_ms"]) / 1e3)
            line["generation"] = g
        print(json.dumps(line), flush=True)
    finish(ctx, [graph])
