"""gb_gpu_attn_decode_noalloc (fixed device scratch, no allocation) against
gb_gpu_attn_decode and against the CPU oracle's AttnDecode (cpu.AttnDecode,
backend/cpu/cpu.go:143) on the same seeded inputs, through the C ABI: they
must agree within the AttnDecode tolerance of backend/gpu/gpu_test.go:265 on
two calls in a row (the second call reuses the shared scratch after the first
left its counters at zero). Requests beyond the fixed scratch are refused
before any launch."""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-5, 1e-4  # the AttnDecode tolerance of the per-op tests

SHAPES = [(6, 2, 64, 7), (32, 8, 128, 300), (24, 8, 128, 33), (64, 8, 128, 4100), (32, 8, 128, 8193)]


def _close(name, got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    d = np.abs(got - want)
    bad = (d > ATOL + RTOL * np.abs(want)) | np.isnan(got)
    assert not bad.any(), f"{name}[{int(np.argmax(bad))}] = {got[np.argmax(bad)]}, want {want[np.argmax(bad)]}"


@pytest.mark.parametrize("nh,nkv,hd,kv_len", SHAPES)
def test_noalloc_matches_allocating_entry_point(gb, orc, cuda, nh, nkv, hd, kv_len):
    rng = np.random.default_rng(100 + kv_len)
    q = torch.from_numpy((rng.random(nh * hd, dtype=np.float32) * 2 - 1)).cuda()
    kc = torch.from_numpy((rng.random(kv_len * nkv * hd, dtype=np.float32) * 2 - 1)).cuda()
    vc = torch.from_numpy((rng.random(kv_len * nkv * hd, dtype=np.float32) * 2 - 1)).cuda()
    scale = float(np.float32(1 / math.sqrt(hd)))
    k = gb.Kernels(0)
    try:
        want = torch.zeros(nh * hd, device="cuda")
        k.attn_decode(q, kc, vc, want, kv_len, nh, nkv, hd, scale)
        torch.cuda.synchronize()
        want_h = want.cpu().numpy()
        oracle = orc.attn_decode(q.cpu().numpy(), kc.cpu().numpy(), vc.cpu().numpy(), kv_len, nh, nkv, hd, scale)
        for call in range(2):
            got = torch.full((nh * hd,), float("nan"), device="cuda")
            rc = gb.lib().gb_gpu_attn_decode_noalloc(k.h, None, q.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                                      got.data_ptr(), kv_len, nh, nkv, hd, scale)
            assert rc == gb.OK, gb.lib().gb_last_error().decode()
            torch.cuda.synchronize()
            _close(f"call {call + 1}", got.cpu().numpy(), want_h)
            _close(f"call {call + 1} vs oracle", got.cpu().numpy(), oracle)
    finally:
        k.close()


def test_noalloc_rejects_sizes_beyond_its_scratch(gb, cuda):
    # 300 KV heads exceed the 256 counters of the static scratch: refused
    # before any launch, with a message that names the limit
    t = torch.zeros(300 * 64, device="cuda")
    k = gb.Kernels(0)
    try:
        rc = gb.lib().gb_gpu_attn_decode_noalloc(k.h, None, t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(),
                                                  1, 300, 300, 64, 0.125)
        assert rc == gb.ERR_UNSUPPORTED
        assert "at most 256" in gb.lib().gb_last_error().decode()
    finally:
        k.close()


def test_noalloc_rejects_partials_beyond_its_scratch(gb, cuda):
    # 128 KV heads, 8 query heads each, head_dim 128 and 16384 positions need
    # 8 slices per KV head: 128 * 8 * 8 * 132 floats of partials, more than the
    # 2^20 the static scratch holds. Refused before any launch (so the cache
    # pointers are never read), with a message that names the limit.
    t = torch.zeros(1024 * 128, device="cuda")
    k = gb.Kernels(0)
    try:
        rc = gb.lib().gb_gpu_attn_decode_noalloc(k.h, None, t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(),
                                                  16384, 1024, 128, 128, 0.0884)
        assert rc == gb.ERR_UNSUPPORTED
        msg = gb.lib().gb_last_error().decode()
        assert "slice partials" in msg and str(1 << 20) in msg
        # the scratch is still usable afterwards
        y = torch.ones(64, device="cuda")
        k.add(y, y, y, 64)
        assert float(y.sum().item()) == 128.0
    finally:
        k.close()
