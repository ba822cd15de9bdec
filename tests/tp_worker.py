"""One rank of the tensor-parallel GPU test (launched by torchrun from
tests/test_tp_gpu.py): a small model's whole weights made on the host from
seeds, this rank's shard uploaded, one greedy decode step; the rank's
logits shard, ids and final hidden row written to the output directory."""

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402


def model(s):
    d, hd, f, e = s.d_model, s.head_dim, s.ffn, s.experts
    layers = []
    for l in range(s.layers):
        seed = 1000 + 10 * l
        layers.append({
            "q": O.normal(seed, s.heads * hd * d, 0, 0.02).reshape(s.heads * hd, d),
            "k": O.normal(seed + 1, s.kv_heads * hd * d, 0, 0.02).reshape(s.kv_heads * hd, d),
            "v": O.normal(seed + 2, s.kv_heads * hd * d, 0, 0.02).reshape(s.kv_heads * hd, d),
            "o": O.normal(seed + 3, d * s.heads * hd, 0, 0.02).reshape(d, s.heads * hd),
            "attn_norm": O.uniform(seed + 7, d, 0.5, 1.5),
            "mlp_norm": O.uniform(seed + 8, d, 0.5, 1.5),
        })
        if e:  # routed experts: the router, each expert's [gate; up] rows and down
            layers[-1].update(router=O.normal(seed + 4, e * d, 0, 0.02).reshape(e, d),
                              egu=O.normal(seed + 5, e * 2 * f * d, 0, 0.02).reshape(e, 2 * f, d),
                              edn=O.normal(seed + 6, e * d * f, 0, 0.02).reshape(e, d, f))
        else:
            layers[-1].update(gate=O.normal(seed + 4, f * d, 0, 0.02).reshape(f, d),
                              up=O.normal(seed + 5, f * d, 0, 0.02).reshape(f, d),
                              down=O.normal(seed + 6, d * f, 0, 0.02).reshape(d, f))
    embed = O.normal(77, s.vocab * d, 0, 0.02).reshape(s.vocab, d)
    final_norm = O.uniform(78, d, 0.5, 1.5)
    return layers, embed, final_norm


def shape(batch=2, moe=False):
    """The test model: 8 heads, so that it shards over 2, 4 or 8 ranks; with
    `moe`, its FFN routed experts (the top 2 of 8, ffn 256 each)."""
    from furykernel_b200.shape import LlamaShape

    if moe:
        return LlamaShape(d_model=512, heads=8, kv_heads=8, head_dim=128, ffn=256, vocab=3000, layers=2,
                          slots=batch, length=64, positions=64, experts=8, top_k=2)
    return LlamaShape(d_model=512, heads=8, kv_heads=8, head_dim=128, ffn=1024, vocab=3000, layers=2, slots=batch,
                      length=64, positions=64)


def main():
    out_dir = sys.argv[1]
    from furykernel_b200 import tp
    from furykernel_b200.engine import Llama, shard_weights

    ctx, rank, world, local = tp.init()
    batch = 2
    s = shape(batch, moe=len(sys.argv) > 2 and sys.argv[2] == "moe")
    layers, embed, final_norm = model(s)
    arena = shard_weights(s, layers, embed, final_norm, rank, world, interleave=batch <= 4)
    eng = Llama(ctx, s, batch, chunk=16, rank=rank, world=world, host_weights=arena)
    tokens = np.array([5, 2999], np.uint32)
    pos = np.array([3, 7], np.uint32)
    eng.set_rows(tokens, pos, np.arange(batch, dtype=np.uint32))
    ids = eng.step()
    np.save(os.path.join(out_dir, f"ids_{rank}.npy"), ids)
    np.save(os.path.join(out_dir, f"logits_{rank}.npy"), eng.logits.download())
    np.save(os.path.join(out_dir, f"x_{rank}.npy"), eng.x.download())
    from tests import model_check as MC

    kc, vc = MC.host_caches(eng)
    np.save(os.path.join(out_dir, f"kc_{rank}.npy"), kc)
    np.save(os.path.join(out_dir, f"vc_{rank}.npy"), vc)
    tp.finish(ctx, [eng.graph])


if __name__ == "__main__":
    main()
