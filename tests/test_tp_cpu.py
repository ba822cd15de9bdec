"""The tensor-parallel host logic on the CPU, as 2 gloo ranks: each rank's
shard of the weight arena (shard_weights, in the engine's layout) computes
its column- and row-parallel parts of a layer in f64; the allreduce of the
row-parallel partial sums and the gather of the vocabulary shards' greedy
candidates give the whole model's results. No GPU is touched."""

import dataclasses
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from furykernel_b200.engine import shard_weights
from furykernel_b200.shape import LlamaShape

S = LlamaShape(d_model=64, heads=4, kv_heads=2, head_dim=8, ffn=48, vocab=40, layers=2, slots=1, length=16,
               positions=16)


def full_model(seed=3):
    rng = np.random.default_rng(seed)
    d, hd = S.d_model, S.head_dim
    layers = [{"q": rng.standard_normal((S.heads * hd, d)), "k": rng.standard_normal((S.kv_heads * hd, d)),
               "v": rng.standard_normal((S.kv_heads * hd, d)), "o": rng.standard_normal((d, S.heads * hd)),
               "gate": rng.standard_normal((S.ffn, d)), "up": rng.standard_normal((S.ffn, d)),
               "down": rng.standard_normal((d, S.ffn)), "attn_norm": rng.standard_normal(d),
               "mlp_norm": rng.standard_normal(d)} for _ in range(S.layers)]
    return layers, rng.standard_normal((S.vocab, d)), rng.standard_normal(d)


def unpack(arena, rank, world, interleave):
    """Reads a rank's arena back with the engine's layout (Llama.layer_sizes)."""
    loc = dataclasses.replace(S, heads=S.heads // world, kv_heads=S.kv_heads // world, ffn=S.ffn // world)
    d, qw, kvw, f = loc.d_model, loc.q_width, loc.kv_width, loc.ffn
    sizes = [("q", qw, d), ("k", kvw, d), ("v", kvw, d), ("o", d, qw), ("gate", f, d), ("up", f, d), ("down", d, f),
             ("attn_norm", 1, d), ("mlp_norm", 1, d)]
    at, out = 0, []
    for _ in range(S.layers):
        w = {}
        for name, r, c in sizes:
            w[name] = arena[at:at + r * c].reshape(r, c)
            at += r * c
        if interleave:
            gu = np.concatenate([w["gate"], w["up"]]).reshape(f, 2, d)
            w["gate"], w["up"] = gu[:, 0], gu[:, 1]
        out.append(w)
    embed = arena[at:at + S.vocab * d].reshape(S.vocab, d)
    return out, embed


def rank_main(rank, world, port, interleave, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import torch

    layers, embed, final_norm = full_model()
    arena = shard_weights(S, layers, embed.astype(np.float32), final_norm.astype(np.float32), rank, world, interleave)
    mine, emb = unpack(arena.astype(np.float64), rank, world, interleave)
    x = np.linspace(-1, 1, S.d_model)
    ok = True
    for l, w in enumerate(mine):
        whole = layers[l]
        # Column parallel: this rank's q/k/v rows and gate/up rows.
        hq = S.heads // world * S.head_dim
        ok &= np.allclose(w["q"], np.float32(whole["q"][rank * hq:(rank + 1) * hq]))
        # Row parallel: the partial sums of o and down over the rank's columns, allreduced.
        att = np.cos(np.arange(S.heads * S.head_dim))[rank * hq:(rank + 1) * hq]
        part = torch.tensor(w["o"] @ att)
        dist.all_reduce(part)
        ok &= np.allclose(part.numpy(), np.float32(whole["o"]).astype(np.float64) @ np.cos(np.arange(S.heads * S.head_dim)))
        g, u = w["gate"] @ x, w["up"] @ x
        act = g / (1 + np.exp(-g)) * u
        part = torch.tensor(w["down"] @ act)
        dist.all_reduce(part)
        gw, uw = np.float32(whole["gate"]).astype(np.float64) @ x, np.float32(whole["up"]).astype(np.float64) @ x
        want = np.float32(whole["down"]).astype(np.float64) @ (gw / (1 + np.exp(-gw)) * uw)
        ok &= np.allclose(part.numpy(), want)
    # Vocabulary-parallel head: each rank's (max, index) over its rows, gathered; ties to the lower index.
    vl = S.vocab // world
    logits = emb[rank * vl:(rank + 1) * vl] @ x
    logits[3] = logits.max()  # a tie within and across shards
    j = int(np.argmax(logits))
    cand = torch.tensor([logits[j], float(j + rank * vl)])
    got = [torch.zeros(2, dtype=cand.dtype) for _ in range(world)]
    dist.all_gather(got, cand)
    best = got[0]
    for c in got[1:]:
        if c[0] > best[0] or (c[0] == best[0] and c[1] < best[1]):
            best = c
    full = np.float32(embed).astype(np.float64) @ x
    for r in range(world):
        full[r * vl + 3] = full[r * vl:(r + 1) * vl].max()
    ok &= int(best[1]) == int(np.argmax(full))  # the first index of the maximum
    q.put((rank, bool(ok)))
    dist.destroy_process_group()


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("interleave", [False, True])
def test_tp2_sharding_on_gloo(interleave):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=rank_main, args=(r, 2, port, interleave, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs)
    results = dict(q.get(timeout=10) for _ in range(2))
    assert results == {0: True, 1: True}


SM = dataclasses.replace(S, ffn=16, experts=4, top_k=2)


def moe_model(seed=5):
    rng = np.random.default_rng(seed)
    d, hd, e, f = SM.d_model, SM.head_dim, SM.experts, SM.ffn
    layers = [{"q": rng.standard_normal((SM.heads * hd, d)), "k": rng.standard_normal((SM.kv_heads * hd, d)),
               "v": rng.standard_normal((SM.kv_heads * hd, d)), "o": rng.standard_normal((d, SM.heads * hd)),
               "router": rng.standard_normal((e, d)), "egu": rng.standard_normal((e, 2 * f, d)),
               "edn": rng.standard_normal((e, d, f)), "attn_norm": rng.standard_normal(d),
               "mlp_norm": rng.standard_normal(d)} for _ in range(SM.layers)]
    return layers, rng.standard_normal((SM.vocab, d)), rng.standard_normal(d)


def gelu(v):
    return 0.5 * v * (1 + np.tanh(np.sqrt(2 / np.pi) * (v + 0.044715 * v ** 3)))


def moe_rank_main(rank, world, port, q):
    """Each rank reads its arena back in the engine's MoE layout (the whole
    router, its ffn slice of every expert) and runs its slice of the chosen
    experts; the allreduce of the slices is the whole experts' output."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import torch

    layers, embed, final_norm = moe_model()
    arena = shard_weights(SM, layers, embed.astype(np.float32), final_norm.astype(np.float32), rank, world)
    arena = arena.astype(np.float64)
    d, qw, kvw, e, k = SM.d_model, SM.q_width // world, SM.kv_width // world, SM.experts, SM.top_k
    fl, f = SM.ffn // world, SM.ffn
    sizes = [("q", qw * d), ("k", kvw * d), ("v", kvw * d), ("o", d * qw), ("router", e * d),
             ("egu", e * 2 * fl * d), ("edn", e * d * fl), ("attn_norm", d), ("mlp_norm", d)]
    x = np.linspace(-1, 1, d)
    ok, at = True, 0
    for whole in layers:
        w = {}
        for name, n in sizes:
            w[name] = arena[at:at + n]
            at += n
        router, egu, edn = w["router"].reshape(e, d), w["egu"].reshape(e, 2 * fl, d), w["edn"].reshape(e, d, fl)
        ok &= np.array_equal(router, np.float32(whole["router"]).astype(np.float64))
        logits = router @ x
        top = np.argsort(-logits, kind="stable")[:k]
        part = np.concatenate([edn[j] @ (gelu(egu[j, :fl] @ x) * (egu[j, fl:] @ x)) for j in top])
        t = torch.tensor(part)
        dist.all_reduce(t)
        w32 = {n: np.float32(whole[n]).astype(np.float64) for n in ("egu", "edn")}
        want = np.concatenate([w32["edn"][j] @ (gelu(w32["egu"][j, :f] @ x) * (w32["egu"][j, f:] @ x)) for j in top])
        ok &= np.allclose(t.numpy(), want)
    ok &= at + SM.vocab * d + d == arena.size
    q.put((rank, bool(ok)))
    dist.destroy_process_group()


def test_tp2_moe_sharding_on_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=moe_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs)
    results = dict(q.get(timeout=10) for _ in range(2))
    assert results == {0: True, 1: True}
