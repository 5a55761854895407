"""The bounded peer-flag wait of the tensor-parallel exchange, on one GPU and
with no fault: a two-rank exchange whose second rank's flag is a local word
that nothing writes must give up after its poll limit, report
GB_ERR_TIMEOUT (and GB_DEVERR_TIMEOUT in a caller's status word), skip the
sum, and leave the device usable. The same exchange with both flags set sums
the partials in rank order."""
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
