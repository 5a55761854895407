"""The bounded waits of the tensor-parallel exchanges, on one GPU and with no
fault. The flag form (gb_gpu_peer_resid): a two-rank exchange whose second
rank's flag is a local word that nothing writes must give up after its poll
limit, report GB_ERR_TIMEOUT (and GB_DEVERR_TIMEOUT in a caller's status
word), skip the sum, and leave the device usable; with both flags set it sums
the partials in rank order. The tagged form the model runs
(gb_gpu_peer_resid_tagged): a rank whose words still carry the previous
step's tag makes every element's wait run out the same way, and once its
words of this step land the sum completes."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

GB_ERR_TIMEOUT, GB_DEVERR_TIMEOUT = 6, 4


def setup(dim, slots=3):
    bufs = [torch.randn(slots * dim, device="cuda") for _ in range(2)]
    flags = [torch.zeros(slots, dtype=torch.int32, device="cuda") for _ in range(2)]
    tb = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device="cuda")
    tf = torch.tensor([f.data_ptr() for f in flags], dtype=torch.int64, device="cuda")
    step = torch.tensor([6], dtype=torch.int32, device="cuda")  # flags must read 7
    return bufs, flags, tb, tf, step


def test_exchange_sums_in_rank_order(gb, kernels):
    dim, slot, n = 512, 1, 512
    bufs, flags, tb, tf, step = setup(dim)
    for f in flags:
        f[slot] = 7
    x = torch.randn(n, device="cuda")
    x0 = x.cpu().numpy().copy()
    ssq = torch.zeros(n // 32, device="cuda")
    kernels.peer_resid(2, tb, tf, step, slot, dim, x, n, ssq)
    torch.cuda.synchronize()
    parts = [b.cpu().numpy()[slot * dim:slot * dim + n] for b in bufs]
    want = x0 + (np.float32(0) + parts[0] + parts[1])
    got = x.cpu().numpy()
    assert np.array_equal(got, want.astype(np.float32))
    np.testing.assert_allclose(ssq.cpu().numpy(), (got.reshape(-1, 32).astype(np.float64) ** 2).sum(1), rtol=1e-5)


def test_missing_flag_times_out_and_device_stays_usable(gb, kernels):
    dim, slot, n = 256, 2, 256
    bufs, flags, tb, tf, step = setup(dim)
    flags[0][slot] = 7  # rank 0 has published; rank 1's flag is never written
    x = torch.randn(n, device="cuda")
    x0 = x.cpu().numpy().copy()
    ssq = torch.zeros(n // 32, device="cuda")
    # synchronous form: the call reports the timeout
    with pytest.raises(gb.GollamaError) as e:
        kernels.peer_resid(2, tb, tf, step, slot, dim, x, n, ssq, wait_limit=2000)
    assert e.value.code == GB_ERR_TIMEOUT
    assert "did not arrive" in str(e.value)
    assert np.array_equal(x.cpu().numpy(), x0)  # the sum was skipped
    # asynchronous form: the caller's status word carries the device error bit
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    kernels.peer_resid(2, tb, tf, step, slot, dim, x, n, ssq, wait_limit=2000, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & GB_DEVERR_TIMEOUT
    # the device and the library still work: the flag arrives, the exchange completes
    flags[1][slot] = 7
    kernels.peer_resid(2, tb, tf, step, slot, dim, x, n, ssq, wait_limit=2000)
    torch.cuda.synchronize()
    parts = [b.cpu().numpy()[slot * dim:slot * dim + n] for b in bufs]
    assert np.array_equal(x.cpu().numpy(), (x0 + (np.float32(0) + parts[0] + parts[1])).astype(np.float32))
    y = torch.ones(64, device="cuda")
    kernels.add(y, y, y, 64)
    assert float(y.sum().item()) == 128.0


# ---- the tagged exchange the model runs (gb_gpu_peer_resid_tagged) ----------

def tagged(values, tag):
    """64-bit words (tag << 32 | float bits) of float32 values, as an int64 tensor."""
    bits = torch.from_numpy(np.asarray(values, dtype=np.float32).view(np.uint32).astype(np.int64))
    return (bits | (int(tag) << 32)).cuda()


def tagged_setup(dim, slots=3, seed=0):
    rng = np.random.default_rng(seed)
    parts = [rng.standard_normal(slots * dim).astype(np.float32) for _ in range(2)]
    step = torch.tensor([6], dtype=torch.int32, device="cuda")  # words must carry tag 7
    return parts, step


def test_tagged_exchange_sums_in_rank_order(gb, kernels):
    dim, slot, n = 512, 1, 512
    parts, step = tagged_setup(dim)
    bufs = [tagged(p, 7) for p in parts]
    x = torch.randn(n, device="cuda")
    x0 = x.cpu().numpy().copy()
    ssq = torch.zeros(n // 32, device="cuda")
    kernels.peer_resid_tagged(2, [b.data_ptr() for b in bufs], step, slot, dim, x, n, ssq)
    torch.cuda.synchronize()
    want = x0 + (np.float32(0) + parts[0][slot * dim:slot * dim + n] + parts[1][slot * dim:slot * dim + n])
    got = x.cpu().numpy()
    assert np.array_equal(got, want.astype(np.float32))
    np.testing.assert_allclose(ssq.cpu().numpy(), (got.reshape(-1, 32).astype(np.float64) ** 2).sum(1), rtol=1e-5)


def test_tagged_stale_word_times_out_and_device_stays_usable(gb, kernels):
    dim, slot, n = 256, 2, 256
    parts, step = tagged_setup(dim, seed=1)
    # rank 0 has written this step's words; rank 1's words still carry the previous step's tag
    bufs = [tagged(parts[0], 7), tagged(parts[1], 6)]
    x = torch.randn(n, device="cuda")
    x0 = x.cpu().numpy().copy()
    ssq = torch.zeros(n // 32, device="cuda")
    with pytest.raises(gb.GollamaError) as e:
        kernels.peer_resid_tagged(2, [b.data_ptr() for b in bufs], step, slot, dim, x, n, ssq, wait_limit=2000)
    assert e.value.code == GB_ERR_TIMEOUT
    assert "did not arrive" in str(e.value)
    assert np.array_equal(x.cpu().numpy(), x0)  # every element kept its x
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    kernels.peer_resid_tagged(2, [b.data_ptr() for b in bufs], step, slot, dim, x, n, ssq, wait_limit=2000,
                              status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & GB_DEVERR_TIMEOUT
    # rank 1's words of this step land: the exchange completes on the same device
    bufs[1].copy_(tagged(parts[1], 7))
    kernels.peer_resid_tagged(2, [b.data_ptr() for b in bufs], step, slot, dim, x, n, ssq, wait_limit=2000)
    torch.cuda.synchronize()
    want = x0 + (np.float32(0) + parts[0][slot * dim:slot * dim + n] + parts[1][slot * dim:slot * dim + n])
    assert np.array_equal(x.cpu().numpy(), want.astype(np.float32))


def test_tagged_exchange_ten_ranks_ragged(gb, kernels):
    """Ten ranks (two batches of eight words per element) and n not a multiple of
    the 256-thread CTA: the sum is the rank-order float32 sum, elements past n
    are untouched."""
    world, dim, slot, n, slots = 10, 800, 2, 672, 4
    rng = np.random.default_rng(7)
    parts = [rng.standard_normal(slots * dim).astype(np.float32) for _ in range(world)]
    step = torch.tensor([41], dtype=torch.int32, device="cuda")
    bufs = [tagged(p, 42) for p in parts]
    x = torch.randn(dim, device="cuda")
    x0 = x.cpu().numpy().copy()
    ssq = torch.zeros(dim // 32, device="cuda")
    kernels.peer_resid_tagged(world, [b.data_ptr() for b in bufs], step, slot, dim, x, n, ssq)
    torch.cuda.synchronize()
    acc = np.zeros(n, dtype=np.float32)
    for p in parts:
        acc = (acc + p[slot * dim:slot * dim + n]).astype(np.float32)
    got = x.cpu().numpy()
    assert np.array_equal(got[:n], (x0[:n] + acc).astype(np.float32))
    assert np.array_equal(got[n:], x0[n:])
