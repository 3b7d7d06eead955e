"""Variable-length attention on the GPU (``sc_attention_varlen``).

Bound: relative L2 < 5e-3 against the float64 oracle on the same
bf16/f16-rounded inputs (the kernel rounds P to the input type for the second
product and the output once), per sequence, over every head.  Larger cases
are checked against torch's fp32 SDPA on the GPU with the same bound.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 5e-3


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _qkv(cuda, nq, nkv, heads, dtype, seed, spread=1.0):
    rng = np.random.default_rng(seed)
    mk = lambda n: torch.from_numpy((spread * rng.standard_normal((n, heads, 64))).astype(np.float32)).to(cuda, dtype)
    return mk(nq), mk(nkv), mk(nkv)


def _f64(t):
    return t.float().cpu().numpy().astype(np.float64)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("lens", [[300], [1], [128], [129, 1, 257, 64], [500, 3]])
def test_self_attention_matches_oracle(pkg, oracle, cuda, dtype, lens):
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    q, k, v = _qkv(cuda, int(cu[-1]), int(cu[-1]), 4, dtype, sum(lens))
    out = pkg.sparse_attention(q, k, v, cu)
    ref = oracle.attention_varlen(_f64(q), _f64(k), _f64(v), cu)
    for b in range(len(lens)):
        s = slice(int(cu[b]), int(cu[b + 1]))
        assert rel_l2(_f64(out[s]), ref[s]) < TOL, (b, lens[b])


def test_cross_attention_ragged_and_empty(pkg, oracle, cuda):
    """Different query and key lengths per item, including an item with no
    key rows (its queries stay zero) and one with no query rows."""
    lq, lk = [70, 0, 200, 33, 5], [130, 9, 1, 0, 300]
    cq = np.concatenate([[0], np.cumsum(lq)]).astype(np.int32)
    ck = np.concatenate([[0], np.cumsum(lk)]).astype(np.int32)
    q, k, v = _qkv(cuda, int(cq[-1]), int(ck[-1]), 2, torch.bfloat16, 7, spread=2.0)
    out = pkg.sparse_attention(q, k, v, cq, ck)
    ref = oracle.attention_varlen(_f64(q), _f64(k), _f64(v), cq, ck)
    for b in range(len(lq)):
        s = slice(int(cq[b]), int(cq[b + 1]))
        if lq[b] == 0:
            continue
        if lk[b] == 0:
            assert torch.count_nonzero(out[s]).item() == 0
        else:
            assert rel_l2(_f64(out[s]), ref[s]) < TOL, b


def test_custom_scale(pkg, oracle, cuda):
    q, k, v = _qkv(cuda, 200, 200, 3, torch.bfloat16, 8)
    out = pkg.sparse_attention(q, k, v, [0, 200], scale=0.3)
    ref = oracle.attention_varlen(_f64(q), _f64(k), _f64(v), [0, 200], scale=0.3)
    assert rel_l2(_f64(out), ref) < TOL


def test_large_matches_torch_sdpa(pkg, cuda):
    """Two sequences of 4,000 and 2,500 tokens, 16 heads, against torch's fp32
    SDPA per sequence on the GPU."""
    lens = [4000, 2500]
    cu = [0, 4000, 6500]
    q, k, v = _qkv(cuda, 6500, 6500, 16, torch.bfloat16, 9)
    out = pkg.sparse_attention(q, k, v, cu)
    for b in range(2):
        s = slice(cu[b], cu[b + 1])
        t = lambda x: x[s].float().transpose(0, 1)
        ref = torch.nn.functional.scaled_dot_product_attention(t(q), t(k), t(v)).transpose(0, 1)
        assert rel_l2(_f64(out[s]), _f64(ref)) < TOL, lens[b]


def test_deterministic(pkg, cuda):
    q, k, v = _qkv(cuda, 700, 700, 4, torch.bfloat16, 10)
    a = pkg.sparse_attention(q, k, v, [0, 300, 700])
    b = pkg.sparse_attention(q, k, v, [0, 300, 700])
    assert torch.equal(a, b)


def test_refuses_bad_arguments(pkg, cuda):
    q, k, v = _qkv(cuda, 10, 10, 2, torch.bfloat16, 11)
    with pytest.raises(ValueError):
        pkg.sparse_attention(q, k, v, [0, 9])              # does not end at the token count
    with pytest.raises(pkg.SparseConvError, match="non-decreasing"):
        pkg.sparse_attention(q, k, v, [0, 6, 4, 10], [0, 3, 7, 10])
    q32 = torch.zeros((10, 2, 32), device=cuda, dtype=torch.bfloat16)
    with pytest.raises(pkg.SparseConvError, match="head_dim"):
        pkg.sparse_attention(q32, q32, q32, [0, 10])
    with pytest.raises(TypeError):
        pkg.sparse_attention(q.float(), k.float(), v.float(), [0, 10])


def test_sequences_stay_isolated(pkg, oracle, cuda):
    """The last key tile of a sequence also covers rows of the next one; a
    NaN in the next sequence's K or V must not reach this sequence's output."""
    cu = np.array([0, 200, 500], np.int32)
    q, k, v = _qkv(cuda, 500, 500, 2, torch.bfloat16, 12)
    k[250] = float("nan")  # rows 200..255 share sequence 0's second key tile
    v[230] = float("nan")
    out = pkg.sparse_attention(q, k, v, cu)
    ref = oracle.attention_varlen(_f64(q[:200]), _f64(k[:200]), _f64(v[:200]), [0, 200])
    assert torch.isfinite(out[:200]).all()
    assert rel_l2(_f64(out[:200]), ref) < TOL
