"""Kernels behind the drop-in utilities: elementwise multiply (Multiply's
forward and backward, mulKernel), the NaN count behind isNan, the arg-max
behind ArgMaxToCPU and the noise fill behind Noise."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _k():
    from ml_engine_b200._lib import kernels
    return kernels()


def _s():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("n", [1, 1000, 4096 * 33 + 3])
def test_mul_and_mul_accumulate(cuda, rng, n):
    x = torch.from_numpy(rng.standard_normal(n).astype(np.float32)).to(cuda)
    y = torch.from_numpy(rng.standard_normal(n).astype(np.float32)).to(cuda)
    z0 = torch.from_numpy(rng.standard_normal(n).astype(np.float32)).to(cuda)
    z = torch.empty_like(x)
    _k().call("mle_mul", x.data_ptr(), y.data_ptr(), z.data_ptr(), n, 0, _s())
    za = z0.clone()
    _k().call("mle_mul", x.data_ptr(), y.data_ptr(), za.data_ptr(), n, 1, _s())
    torch.cuda.synchronize()
    xn, yn, z0n = x.cpu().numpy(), y.cpu().numpy(), z0.cpu().numpy()
    assert np.array_equal(z.cpu().numpy(), xn * yn)
    want = (z0n.astype(np.float64) + xn.astype(np.float64) * yn.astype(np.float64)).astype(np.float32)
    assert np.max(np.abs(za.cpu().numpy() - want)) <= 1e-6 * np.max(np.abs(want))   # one fused multiply-add


def test_count_nan_and_argmax(cuda, rng):
    n = 100_003
    a = rng.standard_normal(n).astype(np.float32)
    a[[5, 777, n - 1]] = np.nan
    x = torch.from_numpy(a).to(cuda)
    cnt = torch.zeros(1, dtype=torch.int64, device=cuda)
    _k().call("mle_count_nan", x.data_ptr(), n, cnt.data_ptr(), _s())
    torch.cuda.synchronize()
    assert int(cnt.item()) == 3
    b = rng.standard_normal(5000).astype(np.float32)
    b[[1234, 4000]] = 9.0                         # a tie: the first index wins
    out = torch.zeros(1, dtype=torch.int32, device=cuda)
    xb = torch.from_numpy(b).to(cuda)
    _k().call("mle_argmax", xb.data_ptr(), b.size, out.data_ptr(), _s())
    torch.cuda.synchronize()
    assert int(out.item()) == 1234 == int(np.argmax(b))


def test_noise_moments(cuda):
    n = 1 << 22
    x = torch.empty(n, device=cuda)
    _k().call("mle_fill_noise", x.data_ptr(), n, 0.5, 2.0, 0, 1234, _s())
    torch.cuda.synchronize()
    g = x.cpu().numpy().astype(np.float64)
    assert abs(g.mean() - 0.5) < 0.01 and abs(g.std() - 2.0) < 0.01
    _k().call("mle_fill_noise", x.data_ptr(), n, -1.0, 3.0, 1, 99, _s())
    torch.cuda.synchronize()
    u = x.cpu().numpy().astype(np.float64)
    assert u.min() >= -1.0 and u.max() < 2.0 and abs(u.mean() - 0.5) < 0.01
