"""The tensor-parallel decode step on CPU: two gloo ranks, no GPU.

The GPU path (gollama.cu_b200/csrc/gb_model.cu load_model / enqueue_step)
shards one decode step Megatron-style: q|k|v and gate/up split by output
rows (whole heads, whole FFN rows), attention and its KV cache local, o and
down split by input columns with every rank's partial summed in rank order,
the lm_head split by vocabulary rows with a (max value, lowest index) key
reduced across ranks (model.Argmax, model/model.go:376). Here each rank runs
that decomposition on its shard of a small seeded float64 model, the
exchanges go through torch.distributed (gloo), and the result must match the
unsharded step. Also: the library rejects shapes that do not split before it
touches CUDA, and the bench's max-over-ranks helper works under gloo.
"""
import importlib.util
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

CFG = dict(dim=64, ffn=128, heads=4, kv_heads=2, head_dim=16, vocab=96, ctx=8, eps=1e-5, base=10000.0)


def make_model(seed=7):
    c = CFG
    rng = np.random.default_rng(seed)
    qd, kvd = c["heads"] * c["head_dim"], c["kv_heads"] * c["head_dim"]
    w = lambda r, k: rng.standard_normal((r, k)) / np.sqrt(k)
    return dict(
        embd=rng.standard_normal((c["vocab"], c["dim"])),
        attn_norm=1 + 0.1 * rng.standard_normal(c["dim"]), ffn_norm=1 + 0.1 * rng.standard_normal(c["dim"]),
        out_norm=1 + 0.1 * rng.standard_normal(c["dim"]),
        wq=w(qd, c["dim"]), wk=w(kvd, c["dim"]), wv=w(kvd, c["dim"]), wo=w(c["dim"], qd),
        wg=w(c["ffn"], c["dim"]), wu=w(c["ffn"], c["dim"]), wd=w(c["dim"], c["ffn"]),
        head=w(c["vocab"], c["dim"]),
        # KV cache of the earlier positions (one layer)
        kc=rng.standard_normal((c["ctx"], kvd)), vc=rng.standard_normal((c["ctx"], kvd)))


def rmsnorm(x, w, eps):
    return x / np.sqrt(np.mean(x * x) + eps) * w


def rope(v, pos, hd, base):
    out = v.copy()
    for h in range(len(v) // hd):
        for j in range(hd // 2):
            th = pos * base ** (-2 * j / hd)
            a, b = v[h * hd + 2 * j], v[h * hd + 2 * j + 1]
            out[h * hd + 2 * j] = a * np.cos(th) - b * np.sin(th)
            out[h * hd + 2 * j + 1] = a * np.sin(th) + b * np.cos(th)
    return out


def argmax_key(v, idx):
    # larger value first, then the lower index (model.Argmax)
    return (v, -idx)


def step(m, token, pos, rank=0, world=1, allsum=None, allkeys=None):
    """One decode step on shard `rank` of `world`; allsum/allkeys exchange across ranks."""
    c = CFG
    hd, H, KV = c["head_dim"], c["heads"] // world, c["kv_heads"] // world
    F, V = c["ffn"] // world, c["vocab"] // world
    qs = slice(rank * H * hd, (rank + 1) * H * hd)          # this rank's q rows (o input columns)
    ks = slice(rank * KV * hd, (rank + 1) * KV * hd)        # its k/v rows
    fs = slice(rank * F, (rank + 1) * F)                    # its FFN rows (down input columns)
    vs = slice(rank * V, (rank + 1) * V)                    # its vocabulary rows
    x = m["embd"][token].copy()
    # attention block: column-parallel q|k|v, local attention, row-parallel o
    xn = rmsnorm(x, m["attn_norm"], c["eps"])
    q = rope(m["wq"][qs] @ xn, pos, hd, c["base"])
    k = rope(m["wk"][ks] @ xn, pos, hd, c["base"])
    v = m["wv"][ks] @ xn
    kc = np.vstack([m["kc"][:pos, ks], k[None]])
    vc = np.vstack([m["vc"][:pos, ks], v[None]])
    attn = np.zeros(H * hd)
    g = H // KV
    for h in range(H):
        kvh = h // g
        sc = kc[:, kvh * hd:(kvh + 1) * hd] @ q[h * hd:(h + 1) * hd] / np.sqrt(hd)
        p = np.exp(sc - sc.max())
        p /= p.sum()
        attn[h * hd:(h + 1) * hd] = p @ vc[:, kvh * hd:(kvh + 1) * hd]
    part = m["wo"][:, qs] @ attn
    x = x + (allsum(part) if allsum else part)
    # FFN block: column-parallel gate/up, row-parallel down
    xn = rmsnorm(x, m["ffn_norm"], c["eps"])
    gt, up = m["wg"][fs] @ xn, m["wu"][fs] @ xn
    act = gt / (1 + np.exp(-gt)) * up
    part = m["wd"][:, fs] @ act
    x = x + (allsum(part) if allsum else part)
    # vocabulary-parallel lm_head and the argmax key
    logits = m["head"][vs] @ rmsnorm(x, m["out_norm"], c["eps"])
    i = int(np.argmax(logits))  # first maximum: the lowest index of the shard
    key = argmax_key(float(logits[i]), rank * V + i)
    best = max(allkeys(key)) if allkeys else key
    return logits, -best[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, token, pos, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        def allsum(part):
            # every rank's partial, added in rank order: the same bits on every rank
            got = [torch.zeros(len(part), dtype=torch.float64) for _ in range(world)]
            dist.all_gather(got, torch.from_numpy(np.ascontiguousarray(part)))
            acc = np.zeros(len(part))
            for t in got:
                acc = acc + t.numpy()
            return acc

        def allkeys(key):
            got = [None] * world
            dist.all_gather_object(got, key)
            return got

        logits, tok = step(make_model(), token, pos, rank, world, allsum, allkeys)
        np.save(os.path.join(out_dir, f"logits{rank}.npy"), logits)
        np.save(os.path.join(out_dir, f"token{rank}.npy"), np.array([tok]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("token,pos", [(5, 0), (17, 3), (95, 7)])
def test_two_rank_step_matches_unsharded(tmp_path, token, pos):
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), token, pos, str(tmp_path)), nprocs=world,
                       start_method="spawn")
    want, want_tok = step(make_model(), token, pos)
    got = np.concatenate([np.load(tmp_path / f"logits{r}.npy") for r in range(world)])
    np.testing.assert_allclose(got, want, rtol=1e-12, atol=1e-12)
    for r in range(world):
        assert int(np.load(tmp_path / f"token{r}.npy")[0]) == want_tok == int(np.argmax(want))


def test_argmax_key_rule_across_shards():
    # equal maxima in two shards: the lower global index wins, as in model.Argmax
    keys = [argmax_key(3.0, 40), argmax_key(3.0, 7), argmax_key(2.5, 1)]
    assert -max(keys)[1] == 7


def _max_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        spec = importlib.util.spec_from_file_location(
            "bench", os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "bench.py"))
        bench = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(bench)
        bench.barrier(world)
        v = bench.max_over_ranks(1.5 + rank, world)  # each rank's time; the job's is the slowest
        np.save(os.path.join(out_dir, f"max{rank}.npy"), np.array([v]))
    finally:
        dist.destroy_process_group()


def test_bench_max_over_ranks_gloo(tmp_path):
    world = 2
    mp.start_processes(_max_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    for r in range(world):
        assert float(np.load(tmp_path / f"max{r}.npy")[0]) == 2.5


def test_library_rejects_unsplittable_shapes(gb):
    # load_model checks the tensor-parallel shard shapes before any CUDA call
    spec = gb.synth_spec(layers=1, dim=256, ffn=512, heads=4, kv_heads=2, head_dim=64, vocab=512, ctx_len=16,
                         mix=0, seed=3)
    img = gb.SynthImage(spec)
    for world, rank in ((3, 0), (4, 1)):
        with pytest.raises(gb.GollamaError) as e:
            gb.Model(img, tp_world=world, tp_rank=rank)
        assert f"shape does not split over {world} GPUs" in str(e.value)
    with pytest.raises(gb.GollamaError) as e:
        gb.Model(img, tp_world=2, tp_rank=2)
    assert "rank 2 outside world 2" in str(e.value)
