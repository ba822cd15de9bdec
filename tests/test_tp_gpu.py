"""Tensor parallelism on 2, 4 and 8 GPUs: a small model's decode step sharded
over the ranks (torchrun, one process a GPU), checked bit for bit against the
CPU restatement of the tensor-parallel arithmetic (each shard's sums, the
row-parallel partials added in rank order) and, over the whole model, within
the f64 evaluator's bounds; the ranks' hidden rows bit-identical, greedy ids
equal to the referee's where its bounds decide them."""

import math
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

from oracle import oracle as O
from tests import model_check as MC

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def gpus() -> int:
    try:
        import torch

        return torch.cuda.device_count()
    except Exception:
        return 0


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_decode_step_within_bounds(tmp_path, world):
    if gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT)
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", str(world), "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
           os.path.join(ROOT, "tests", "tp_worker.py"), str(tmp_path)]
    r = subprocess.run(cmd, env=env, cwd=ROOT, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import tp_worker as W
    s = W.shape()
    layers, embed, final_norm = W.model(s)
    ids = [np.load(tmp_path / f"ids_{r}.npy") for r in range(world)]
    xs = [np.load(tmp_path / f"x_{r}.npy") for r in range(world)]
    logits = np.concatenate([np.load(tmp_path / f"logits_{r}.npy") for r in range(world)], axis=1)
    kc = np.concatenate([np.load(tmp_path / f"kc_{r}.npy") for r in range(world)], axis=2)
    vc = np.concatenate([np.load(tmp_path / f"vc_{r}.npy") for r in range(world)], axis=2)
    for r in range(1, world):
        assert np.array_equal(ids[0], ids[r])
        assert np.array_equal(xs[0].view(np.uint32), xs[r].view(np.uint32))
    # Bit for bit with the CPU restatement of the tensor-parallel arithmetic
    # (shard GEMVs, partials added in rank order, then the residual).
    tokens = np.array([5, 2999], np.uint32)
    pos = np.array([3, 7], np.uint32)
    slot = np.arange(2, dtype=np.uint32)
    kc0 = np.zeros_like(kc)
    vc0 = np.zeros_like(vc)
    want_ids, want_logits, want_x = MC.oracle_decode_tp(s, world, layers, embed, final_norm, kc0, vc0, tokens, pos,
                                                        slot, 16, 4)
    assert np.array_equal(kc0.view(np.uint32), kc.view(np.uint32))
    assert np.array_equal(vc0.view(np.uint32), vc.view(np.uint32))
    assert np.array_equal(xs[0].view(np.uint32), want_x.view(np.uint32))
    assert np.array_equal(logits.view(np.uint32), want_logits.view(np.uint32))
    assert np.array_equal(ids[0], want_ids)

    class Full:  # the referee reads only the whole model's shape
        pass

    full = Full()
    full.s = s
    lw = [{"qkv": np.concatenate([w["q"], w["k"], w["v"]]), "o": w["o"],
           "gu": np.concatenate([w["gate"], w["up"]]), "down": w["down"], "attn_norm": w["attn_norm"],
           "mlp_norm": w["mlp_norm"]} for w in layers]
    tokens = np.array([5, 2999], np.uint32)
    pos = np.array([3, 7], np.uint32)
    slot = np.arange(2, dtype=np.uint32)
    ref, (ref_ids, decided), stored_ok = MC.referee_decode(full, lw, embed, final_norm, kc, vc, tokens, pos, slot)
    assert stored_ok
    assert O.within(logits, ref).all()
    rel = float(np.max(np.abs(logits - ref[0])) / np.max(np.abs(ref[0])))
    assert rel <= 1e-4, rel
    assert np.array_equal(ids[0][decided], ref_ids[decided])


def test_tp_moe_decode_step(tmp_path):
    """Routed experts over 2 ranks: the router whole on each, each rank's ffn
    slice of every expert, the experts' outputs and the attention's partials
    summed by NCCL (two addends: the same bits in either order), then the
    combine; bit for bit with the CPU restatement."""
    world = 2
    if gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT)
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", str(world), "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
           os.path.join(ROOT, "tests", "tp_worker.py"), str(tmp_path), "moe"]
    r = subprocess.run(cmd, env=env, cwd=ROOT, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import tp_worker as W
    s = W.shape(moe=True)
    layers, embed, final_norm = W.model(s)
    ids = [np.load(tmp_path / f"ids_{r}.npy") for r in range(world)]
    xs = [np.load(tmp_path / f"x_{r}.npy") for r in range(world)]
    logits = np.concatenate([np.load(tmp_path / f"logits_{r}.npy") for r in range(world)], axis=1)
    kc = np.concatenate([np.load(tmp_path / f"kc_{r}.npy") for r in range(world)], axis=2)
    vc = np.concatenate([np.load(tmp_path / f"vc_{r}.npy") for r in range(world)], axis=2)
    assert np.array_equal(ids[0], ids[1]) and np.array_equal(xs[0].view(np.uint32), xs[1].view(np.uint32))
    tokens = np.array([5, 2999], np.uint32)
    pos = np.array([3, 7], np.uint32)
    slot = np.arange(2, dtype=np.uint32)
    kc0, vc0 = np.zeros_like(kc), np.zeros_like(vc)
    want_ids, want_logits, want_x = MC.oracle_decode_tp(s, world, layers, embed, final_norm, kc0, vc0, tokens, pos,
                                                        slot, 16, 4)
    assert np.array_equal(kc0.view(np.uint32), kc.view(np.uint32))
    assert np.array_equal(vc0.view(np.uint32), vc.view(np.uint32))
    assert np.array_equal(xs[0].view(np.uint32), want_x.view(np.uint32))
    assert np.array_equal(logits.view(np.uint32), want_logits.view(np.uint32))
    assert np.array_equal(ids[0], want_ids)
