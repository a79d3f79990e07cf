"""Embedding-table SGD update (KeyUpdate / TextualEmbedding::EmbeddingUpdate,
Engine/kernels.cu:1536-1549, Engine/transformer.cu:233-245) and the token
gather, against the reference's compiled kernel and the C oracle.

The reference's KeyUpdate adds -lr * grad into the table without atomics, so
two tokens with the same key race; its result is defined only for distinct
keys, where ours must equal it bit for bit (one fused multiply-add per
element).  With repeated keys ours sums the rows' gradients first and is
compared with the exact scatter-add at the fp32 elementwise bound."""
import numpy as np
import pytest

from conftest import RTOL_EXACT, rel_err

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def T(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def H(t):
    return t.detach().cpu().numpy()


@pytest.fixture
def ops():
    from ml_engine_b200 import ops as o
    return o


@pytest.fixture
def orc():
    from oracle import ops as o
    return o


@pytest.mark.parametrize("dim", [256, 512, 30])
def test_embedding_update_equals_reference_kernel_on_distinct_keys(cuda, ops, orc, rng, dim):
    from oracle import ref
    if not ref.available():
        pytest.skip("reference kernels not built")
    batch, clen, max_clen, vocab = 4, 50, 64, 1000
    keys = np.full((batch, max_clen), -1, np.int32)
    perm = rng.permutation(vocab)[: batch * clen].reshape(batch, clen).astype(np.int32)
    keys[:, :clen] = perm
    keys[1, 7] = -1                      # a masked token
    grad = rng.standard_normal((batch * clen, dim)).astype(np.float32)
    table = (rng.standard_normal((vocab, dim)) * 0.02).astype(np.float32)
    lr = 1e-4
    r_tab, k_dev = T(table, cuda), T(keys, cuda)
    ref.call("ref_key_update", ref.ptr(r_tab), ref.ptr(T(grad, cuda)), ref.ptr(k_dev), clen, max_clen, dim, lr,
             grad.size)
    o_tab = T(table, cuda)
    ops.embedding_update(k_dev, T(grad, cuda), o_tab, clen, lr, key_stride=max_clen)
    torch.cuda.synchronize()
    assert np.array_equal(H(o_tab), H(r_tab))
    c_tab = orc.key_update(table.copy(), grad, keys, clen, max_clen, lr)
    assert np.array_equal(c_tab, H(r_tab))


def test_embedding_update_sums_repeated_keys(cuda, ops, orc, rng):
    """Zipf-like ids over a small vocabulary: most rows share their key."""
    rows, dim, vocab, lr = 4096, 256, 64, 1e-3
    keys = np.minimum(rng.zipf(1.3, rows) - 1, vocab - 1).astype(np.int32)
    keys[::97] = -1
    grad = rng.standard_normal((rows, dim)).astype(np.float32)
    table = (rng.standard_normal((vocab, dim)) * 0.02).astype(np.float32)
    o_tab = T(table, cuda)
    ops.embedding_update(T(keys, cuda), T(grad, cuda), o_tab, rows, lr)
    torch.cuda.synchronize()
    exact = table.astype(np.float64).copy()
    np.add.at(exact, keys[keys >= 0], -lr * grad[keys >= 0].astype(np.float64))
    # the update itself (table - table0) to the fp32 reduction bound: the
    # rows of a key are summed, then applied with one fused multiply-add
    assert rel_err(H(o_tab).astype(np.float64) - table, exact - table) <= RTOL_EXACT
    # the oracle restates the reference's per-row chain (what it computes
    # when its threads do not race): one rounding per row
    c_tab = orc.key_update(table.copy(), grad, keys, rows, rows, lr)
    assert rel_err(c_tab.astype(np.float64) - table, exact - table) <= 1e-4


def test_embedding_gather_masked_rows_are_zero(cuda, ops, orc, rng):
    keys = rng.integers(0, 100, 300).astype(np.int32)
    keys[[3, 50, 299]] = -1
    table = rng.standard_normal((100, 64)).astype(np.float32)
    out = torch.full((300, 64), 7.0, device=cuda)
    ops.embedding_gather(T(keys, cuda), T(table, cuda), out)
    torch.cuda.synchronize()
    assert np.array_equal(H(out), orc.embedding_gather(keys, table))
    assert not H(out)[[3, 50, 299]].any()


@pytest.mark.parametrize("batch,seq,dim", [(32, 128, 256), (3, 37, 64), (2, 256, 512)])
def test_gather_with_positional_add_matches_two_launches(cuda, ops, rng, batch, seq, dim):
    """The gather and the positional table's add in one pass (what the
    sessions run for token inputs) against mle_embedding_gather followed by
    mle_rows_add_table: bit for bit, masked keys included."""
    from ml_engine_b200._lib import kernels
    keys = rng.integers(0, 500, batch * seq).astype(np.int32)
    keys[::17] = -1
    table = T(rng.standard_normal((500, dim)).astype(np.float32), cuda)
    pe = torch.empty(seq * dim, device=cuda)
    ops.matpe_table(pe, seq, dim)
    k = T(keys, cuda)
    out = torch.full((batch * seq, dim), 7.0, device=cuda)
    kernels().call("mle_embedding_gather_add", k.data_ptr(), table.data_ptr(), pe.data_ptr(), out.data_ptr(),
                   batch * seq, dim, seq, torch.cuda.current_stream().cuda_stream)
    g = torch.empty(batch * seq, dim, device=cuda)
    ops.embedding_gather(k, table, g)
    ref = torch.empty_like(g)
    ops.rows_add_table(g, pe, ref, batch)
    assert torch.equal(out, ref)
