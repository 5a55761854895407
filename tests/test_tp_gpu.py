"""Tensor parallelism on two GPUs: the sharded decode step against the one-GPU
step and against cpuForward on the same seeded model (skipped with fewer than
two GPUs). Each rank is its own process and device, as bench.py runs them;
the NCCL id goes from rank 0 to rank 1 over a gloo group on the host."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

# a shape that splits over 2 GPUs: heads, KV heads, FFN rows (in 256-multiples
# per rank), vocabulary rows and the per-rank q width (a 256 multiple)
CFG = dict(layers=2, dim=512, ffn=1024, heads=8, kv_heads=2, head_dim=64, vocab=1024, ctx_len=96, mix=1, seed=21)
TOKENS = [7, 300, 1023, 0]
PREFILL = [int(t) for t in np.random.default_rng(5).integers(0, 1024, 40)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out_dir):
    import sys

    import torch.distributed as dist

    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(os.path.dirname(here), "gollama.cu_b200"))
    import gollama_b200 as gb

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.cuda.set_device(rank)
        obj = [gb.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        img = gb.SynthImage(gb.synth_spec(**CFG))
        m = gb.Model(img, max_len=64, device=rank, tp_rank=rank, tp_world=world, nccl_id=obj[0])
        logits = [m.forward(t, p).copy() for p, t in enumerate(TOKENS)]
        toks = m.generate(int(np.argmax(logits[-1])), len(TOKENS), 6)
        # batched prefill over both ranks (all-reduced o/down partials)
        pre = m.prefill(PREFILL, 0).copy()
        # and through each rank's binary16 weight copy (the few-token GEMM)
        m.cache_f16_weights()
        pre16 = m.prefill(PREFILL, 0).copy()
        m.close()
        if rank == 0:
            np.save(os.path.join(out_dir, "tp_logits.npy"), np.stack(logits))
            np.save(os.path.join(out_dir, "tp_tokens.npy"), toks)
            np.save(os.path.join(out_dir, "tp_prefill.npy"), pre)
            np.save(os.path.join(out_dir, "tp_prefill16.npy"), pre16)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_step_matches_one_gpu_and_cpu(gb, orc, cuda, tmp_path):
    import torch.multiprocessing as mp

    mp.start_processes(_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn")
    tp = np.load(tmp_path / "tp_logits.npy")
    tp_toks = np.load(tmp_path / "tp_tokens.npy")
    img = gb.SynthImage(gb.synth_spec(**CFG))
    raw = np.array(img.view(), copy=True)
    m = gb.Model(img, max_len=64)
    om = orc.OracleModel(raw, 64, True)
    for p, t in enumerate(TOKENS):
        one = m.forward(t, p).copy()
        want = om.forward(t, p, CFG["vocab"])
        # the sharded sums differ from the one-GPU ones only in float rounding
        np.testing.assert_allclose(tp[p], one, atol=1e-3, rtol=1e-4)
        d = np.abs(tp[p].astype(np.float64) - want)
        assert (d <= 1e-3 + 1e-4 * np.abs(want)).all(), f"pos {p}: max abs diff {d.max():.3g}"
    one_toks = m.generate(int(np.argmax(tp[-1])), len(TOKENS), 6)
    assert list(tp_toks) == list(one_toks)
    # the two-GPU prefill against the one-GPU prefill (binary16 GEMMs on both;
    # the sharded sums differ in rounding) and against 40 one-GPU decode steps
    one_pre = m.prefill(PREFILL, 0).copy()
    tp_pre = np.load(tmp_path / "tp_prefill.npy")
    rel = lambda a, b: float(np.abs(a.astype(np.float64) - b).max() / np.abs(b).max())
    assert rel(tp_pre, one_pre) < 5e-3, rel(tp_pre, one_pre)
    tp_pre16 = np.load(tmp_path / "tp_prefill16.npy")
    assert rel(tp_pre16, one_pre) < 5e-3, rel(tp_pre16, one_pre)
    d = gb.Model(img, max_len=64)
    for p, t in enumerate(PREFILL):
        dec = d.forward(t, p).copy()
    d.close()
    assert rel(tp_pre, dec) < 5e-3, rel(tp_pre, dec)
    m.close()
    om.close()
