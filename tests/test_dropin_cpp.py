"""The drop-in C++ surface: a program written against the reference's
engine.h / transformer.h API (tests/cpp/usecase_train.cu: use_cases/mnist.cu's
convolutional classifier without its OpenCV loader, Multi_Linear_Residual_Block,
TimeMLPBlock, MultiHeadAttention self and cross attention, operators + - *,
Noise, isNan, printHeadGPU, ArgMaxToCPU, TopKSampleToCPU, SafeCudaMalloc,
fillKernel, CheckError) compiles and links against this repository's
headers and libmle_engine.so unchanged (CPU), and trains (GPU)."""
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
SRC = ROOT / "tests" / "cpp" / "usecase_train.cu"


def _build(tmp_path):
    sys.path.insert(0, str(ROOT / "tests" / "cpp"))
    import build as cppbuild
    out = tmp_path / "usecase_train"
    cppbuild.build(SRC, out)
    return out


def test_reference_style_program_compiles_and_links(tmp_path):
    out = _build(tmp_path)
    assert out.exists() and out.stat().st_size > 0


@pytest.mark.gpu
def test_reference_style_program_trains(tmp_path):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    out = _build(tmp_path)
    r = subprocess.run([str(out)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "usecase ok" in r.stdout


TWO = ROOT / "tests" / "cpp" / "two_graphs.cu"


def test_two_graph_program_compiles_and_links(tmp_path):
    sys.path.insert(0, str(ROOT / "tests" / "cpp"))
    import build as cppbuild
    out = tmp_path / "two_graphs"
    cppbuild.build(TWO, out)
    assert out.exists()


@pytest.mark.gpu
def test_shared_node_gradient_is_cleared_and_accumulated_across_graphs(tmp_path):
    """Two GraphOperations share a node; graph A's first writer of its
    gradient is an activation (which may assign), graph B's a Scale (which
    adds).  Both zero_grads run, then B's backward, then A's: the node's
    gradient must be the sum of both contributions (tests/cpp/two_graphs.cu),
    so neither graph may leave a gradient uncleared that another graph's
    backward writes."""
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    sys.path.insert(0, str(ROOT / "tests" / "cpp"))
    import build as cppbuild
    out = tmp_path / "two_graphs"
    cppbuild.build(TWO, out)
    r = subprocess.run([str(out)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "two graphs ok" in r.stdout
