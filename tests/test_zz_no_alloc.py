"""mle_clip_grad_norm_static (no caller workspace) against the workspace
entry points mle_grad_sumsq + mle_clip_finalize + mle_clip_apply, called
twice in a row through the C ABI with different tensor sets, so state left
in the static scratch by the first call would show in the second.  Named to
run last; it also passes alone in a fresh process."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _grads(rng, sizes, scale, dev):
    return [torch.from_numpy((rng.standard_normal(n) * scale).astype(np.float32)).to(dev) for n in sizes]


def _views(ops, grads):
    return ops.param_views([dict(w=g, g=g, m=g, v=g, t=torch.ones(1, dtype=torch.int32, device=g.device))
                            for g in grads])


def _call(name, *args):
    from ml_engine_b200._lib import kernels
    kernels().call(name, *args)


@pytest.mark.parametrize("max_norm", [1.0, 0.25])
def test_static_clip_matches_workspace_clip_twice(cuda, rng, max_norm):
    from ml_engine_b200 import ops
    stream = torch.cuda.current_stream().cuda_stream
    # first call: many tensors (more than one 96-tensor launch round), one
    # empty; second call: fewer, larger tensors (fewer partial slots)
    cases = [[4097, 1, 0, 300000] + [777] * 120, [1 << 20, 12345]]
    for sizes in cases:
        g_static = _grads(rng, sizes, 0.05, cuda)
        g_ws = [g.clone() for g in g_static]
        coef = torch.full((1,), -1.0, dtype=torch.float64, device=cuda)
        vs = _views(ops, g_static)
        _call("mle_clip_grad_norm_static", ctypes.cast(vs, ctypes.c_void_p), len(sizes), max_norm,
              coef.data_ptr(), stream)
        ws = torch.zeros(1, dtype=torch.float64, device=cuda)
        vw = _views(ops, g_ws)
        _call("mle_grad_sumsq", ctypes.cast(vw, ctypes.c_void_p), len(sizes), ws.data_ptr(), 1.0, stream)
        _call("mle_clip_finalize", ws.data_ptr(), max_norm, stream)
        _call("mle_clip_apply", ctypes.cast(vw, ctypes.c_void_p), len(sizes), ws.data_ptr(), stream)
        torch.cuda.synchronize()
        c_static, c_ws = float(coef.item()), float(ws.item())
        assert c_ws > 1.0  # the sets are large enough to be clipped
        assert abs(c_static - c_ws) <= 1e-12 * c_ws, (c_static, c_ws)
        for a, b in zip(g_static, g_ws):
            if a.numel():
                np.testing.assert_allclose(a.cpu().numpy(), b.cpu().numpy(), rtol=1e-6, atol=0)


def test_static_clip_rejects_oversized_set(cuda):
    from ml_engine_b200 import ops
    from ml_engine_b200._lib import MLEError, kernels
    max_blocks = 8192  # MLE_CLIP_STATIC_MAX_BLOCKS
    g = torch.zeros(4096, device=cuda)
    vs = _views(ops, [g] * (max_blocks + 1))
    with pytest.raises(MLEError):
        kernels().call("mle_clip_grad_norm_static", ctypes.cast(vs, ctypes.c_void_p), max_blocks + 1, 1.0, None,
                       torch.cuda.current_stream().cuda_stream)
