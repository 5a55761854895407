"""Decode attention over a paged KV cache for a batch of sequences
(gb_gpu_attn_decode_paged; the reference's roadmap "Paged KV cache plus
continuous batching", ROADMAP.md:197-202): every sequence's output against
the oracle's AttnDecode (backend/cpu/cpu.go:140-168) over that sequence's
pages gathered into the reference's contiguous [position][kv_dim] cache."""
import math

import numpy as np
import pytest
import torch

from test_kernels_gpu import assert_close

pytestmark = pytest.mark.gpu

CASES = [  # n_heads, n_kv, head_dim, page_size, seq_lens
    (8, 2, 64, 16, [1, 17, 100, 5]),
    (32, 8, 128, 64, [300, 1, 64, 129, 1000, 2]),
    (24, 8, 128, 256, [33, 4100]),
    (64, 8, 128, 32, [777, 8, 2049]),
    (6, 6, 64, 128, [513]),
]


def run_case(kernels, orc, nh, nkv, hd, page, lens, kv_f16, seed):
    rng = np.random.default_rng(seed)
    B = len(lens)
    max_pages = max((L + page - 1) // page for L in lens) + 1
    n_pages = sum((L + page - 1) // page for L in lens) + 3
    pool_shape = (n_pages, nkv, page, hd)
    kp = rng.standard_normal(pool_shape).astype(np.float32)
    vp = rng.standard_normal(pool_shape).astype(np.float32)
    if kv_f16:
        kp, vp = kp.astype(np.float16), vp.astype(np.float16)
    # each sequence takes a random set of physical pages, in random order
    perm = rng.permutation(n_pages)
    table = np.full((B, max_pages), -1, np.int32)
    used = 0
    for b, L in enumerate(lens):
        n = (L + page - 1) // page
        table[b, :n] = perm[used:used + n]
        used += n
    q = rng.standard_normal((B, nh, hd)).astype(np.float32)
    scale = float(np.float32(1 / math.sqrt(hd)))
    out = torch.full((B, nh, hd), float("nan"), device="cuda")
    dq = torch.from_numpy(q).cuda()
    dk = torch.from_numpy(kp.view(np.uint16) if kv_f16 else kp).cuda()
    dv = torch.from_numpy(vp.view(np.uint16) if kv_f16 else vp).cuda()
    dt = torch.from_numpy(table).cuda()
    dl = torch.from_numpy(np.array(lens, np.int32)).cuda()
    for _ in range(2):  # the second call reuses the split counters
        kernels.attn_decode_paged(dq, dk, dv, kv_f16, dt, dl, B, max_pages, n_pages, page, nh, nkv, hd, scale, out)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        for b, L in enumerate(lens):
            pos = np.arange(L)
            phys = table[b, pos // page]
            kc = kp[phys, :, pos % page, :].astype(np.float32).reshape(L, nkv * hd)
            vc = vp[phys, :, pos % page, :].astype(np.float32).reshape(L, nkv * hd)
            want = orc.attn_decode(q[b].reshape(-1), kc.reshape(-1), vc.reshape(-1), L, nh, nkv, hd, scale)
            assert_close(f"paged b={b} L={L}", got[b].reshape(-1), want, 1e-5, 1e-4)


@pytest.mark.parametrize("kv_f16", [1, 0])
@pytest.mark.parametrize("ci", range(len(CASES)))
def test_paged_attention_vs_oracle(kernels, orc, cuda, ci, kv_f16):
    nh, nkv, hd, page, lens = CASES[ci]
    run_case(kernels, orc, nh, nkv, hd, page, lens, kv_f16, 100 + ci)


def test_paged_attention_empty_batch_and_errors(kernels, gb, cuda):
    out = torch.zeros(1, device="cuda")
    z = torch.zeros(16, device="cuda")
    zi = torch.zeros(4, dtype=torch.int32, device="cuda")
    kernels.attn_decode_paged(z, z, z, 0, zi, zi, 0, 1, 1, 16, 8, 2, 64, 0.1, out)  # no sequences: nothing to do
    with pytest.raises(gb.GollamaError):
        kernels.attn_decode_paged(z, z, z, 0, zi, zi, 1, 1, 1, 16, 8, 3, 64, 0.1, out)  # 8 heads over 3 KV heads
    with pytest.raises(gb.GollamaError):
        kernels.attn_decode_paged(z, z, z, 0, zi, zi, 1, 1, 1, 16, 8, 2, 256, 0.1, out)  # head_dim above 128
