"""Selections of this target's GEMV variants (src/FuryKernel/Selection.hs):
which split-K each GEMV shape runs, as tuning chose and a repository
commits, validated by the C++ host library (libfurykernel_host.so).

The family is `gemv` on target `Cuda`; a class is n_k_m (m the batch), and
its one axis, the split-K `s`, decides the order of the reduction, so the
classes of one (n, k) must agree on it: a row's bits do not depend on the
batch it ran in. `tune` measures every variant pruning keeps and picks, per
(n, k), the split whose summed time over the batches is least."""

from __future__ import annotations

import os

from . import _host as H
from . import _native as N

SPLITS = (1, 2, 4, 8)


def gemv_classes(eng) -> list:
    """The engine's GEMV classes (n, k, m), m its batch, in launch order,
    each once (from the host library's launch list); the routed GEMV is no
    member (its split is the lowering's)."""
    out = []
    for L in getattr(eng, "launches", None) or eng._launches():
        if L.kernel.startswith("gemv") and not L.kernel.startswith("gemv_routed"):
            c = (L.params["n"], L.params["k"], eng.m)
            if c not in out:
                out.append(c)
    return out


def read(selection: str) -> str:
    """A selection's text: the argument itself when it is JSON, else the
    file it names."""
    if selection.lstrip().startswith("{"):
        return selection
    with open(selection) as f:
        return f.read()


def splits_for(eng, selection: str) -> dict:
    """Each of the engine's GEMV shapes (n, k) and its selected split, or
    Refused with every problem of the selection for these classes."""
    saved, eng.splits = getattr(eng, "splits", {}), {}
    try:
        classes = gemv_classes(eng)
    finally:
        eng.splits = saved
    picks = H.gemv_selection_validate(read(selection), classes, eng.ctx.sms)
    return {(n, k): s for (n, k, _), s in zip(classes, picks)}


def choose(classes, times) -> list:
    """Per (n, k), the split whose summed time over its batches is least,
    among the splits every batch keeps; `times[(n, k, m)]` maps each kept
    split to its milliseconds. The splits in class order."""
    best = {}
    for n, k in dict.fromkeys((n, k) for n, k, _ in classes):
        ms = [m for nn, kk, m in classes if (nn, kk) == (n, k)]
        common = set.intersection(*(set(times[(n, k, m)]) for m in ms))
        if not common:
            raise N.Refused(N.FKC_ERR_ARGUMENT, f"no split is kept at every batch of n {n}, k {k}.")
        best[(n, k)] = min(sorted(common), key=lambda s: sum(times[(n, k, m)][s] for m in ms))
    return [best[(n, k)] for n, k, _ in classes]


def tune(ctx, classes, reps: int = 20, warmup: int = 3, path: str | None = None) -> str:
    """Times every kept variant of each class on the context's GPU (CUDA
    events around `reps` launches of the `gemv` entry, inputs seeded on the
    device) and returns, or writes to `path`, the selection of the fastest
    split per (n, k)."""
    import torch

    times = {}
    torch.cuda.set_device(ctx.device)
    stream = torch.cuda.ExternalStream(ctx.stream())
    for n, k, m in classes:
        kept = [s for s in SPLITS if H.gemv_consider(n, k, m, s, ctx.sms)[0] == "kept"]
        w, x, y = ctx.alloc(4 * n * k), ctx.alloc(4 * m * k), ctx.alloc(4 * m * n)
        ctx.fill_normal(w, 1, 0.0, 0.02)
        ctx.fill_normal(x, 2)
        times[(n, k, m)] = {}
        for s in kept:
            p = {"n": n, "k": k, "m": m, "split": s, "ldx": k, "ldy": n}
            for _ in range(warmup):
                ctx.launch("gemv", p, [w, x, y])
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                ctx.launch("gemv", p, [w, x, y])
            e1.record(stream)
            e1.synchronize()
            times[(n, k, m)][s] = e0.elapsed_time(e1) / reps
        for b in (w, x, y):
            b.free()
    text = H.gemv_selection_render(classes, choose(classes, times), ctx.sms)
    if path:
        os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
        with open(path, "w") as f:
            f.write(text)
    return text


def classes_for(shape, batch: int, sms: int, chunk: int = 32) -> list:
    """The GEMV classes (n, k, batch) of a one-GPU decode step of `shape`
    at `batch`, from the host library's launch list at stand-in addresses
    (no device memory): the engine's own choices of forms."""
    addrs = {n: (i + 1) << 32 for i, n in enumerate(H.DESC_ADDRS + H.MOE_ADDRS)}
    addrs["part"] = [(64 + i) << 32 for i in range(3)]
    out = []
    for kernel, params, _ in H.llama_launches(shape, batch, 0, 1, sms, chunk, batch <= 64, False, batch <= 4,
                                              addrs):
        if kernel.startswith("gemv") and not kernel.startswith("gemv_routed"):
            c = (params["n"], params["k"], batch)
            if c not in out:
                out.append(c)
    return out


def main(argv=None) -> None:
    """python -m furykernel_b200.select tune [--batches 1,4,16,64] [--layers L] [--out FILE]: times the
    GEMV variants of config 5's decode step on GPU 0 and writes the selection."""
    import argparse

    from .shape import LlamaShape

    ap = argparse.ArgumentParser(prog="python -m furykernel_b200.select")
    ap.add_argument("command", choices=["tune", "classes"])
    ap.add_argument("--batches", default="1,4,16,64")
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--sms", type=int, default=148, help="classes: the multiprocessors to prune for")
    ap.add_argument("--out", default=None)
    args = ap.parse_args(argv)
    batches = [int(b) for b in args.batches.split(",")]

    def shape(b):  # config 5's model at batch b: a slot a row
        length = 4096 if b <= 4 else 640  # config 5: a 512-position prompt and 128 steps
        return LlamaShape(layers=args.layers, slots=b, length=length, positions=length)

    if args.command == "classes":
        for b in batches:
            print(b, classes_for(shape(b), b, args.sms))
        return
    ctx = N.Context(0)
    try:
        classes = [c for b in batches for c in classes_for(shape(b), b, ctx.sms)]
        print(tune(ctx, classes, path=args.out))
    finally:
        ctx.close()


if __name__ == "__main__":
    main()
