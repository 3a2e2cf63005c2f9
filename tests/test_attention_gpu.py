"""Fused decode attention (C ABI dial_b200_attention_decode) against the
oracle's q/k RMSNorm + RoPE + KV append + grouped attention
(text.rs:1466-1536, cache.rs:169-237, text.rs:1258-1281) on paged KV."""

import numpy as np
import pytest

from attn_case import PagedCase, assert_attn_close, run, ulp

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("qh,kvh", [(32, 8), (8, 8), (10, 2), (16, 4), (8, 1)])
@pytest.mark.parametrize("splits", [1, 4])
def test_attention_decode_matches_oracle(cuda, qh, kvh, splits):
    import dial_b200

    case = PagedCase(qh, kvh, [0, 1, 15, 16, 200, 777], seed=qh * 10 + kvh)
    (got,), dev, _ = run(case, cuda, splits)
    assert dial_b200.device_status() == 0
    ref, kref, vref = case.oracle()
    assert_attn_close(got, ref, "bf16")
    k, v = case.new_kv(dev["k_pages"], dev["v_pages"])
    np.testing.assert_array_equal(v, vref)
    dk = np.abs(k - kref)
    assert np.all(dk <= ulp(kref, "bf16")), "appended K more than 1 ulp from the oracle"
    assert np.mean(dk == 0) >= 0.999


def test_attention_decode_f16_long_context(cuda):
    case = PagedCase(32, 8, [1000, 513, 64], seed=5, max_pos=1024, dtype="f16")
    (got,), _, _ = run(case, cuda, 16)
    ref, _, _ = case.oracle()
    assert_attn_close(got, ref, "f16")


def test_attention_decode_many_rows_f16_long_context(cuda):
    """More than 4 rows with groups of 4 query heads take the token-split
    form (each warp scores a quarter of every page for the whole group):
    long and one-token contexts, 16 splits, and a second call that
    reproduces the first bit for bit."""
    import dial_b200

    case = PagedCase(32, 8, [1000, 513, 64, 0, 250, 1023, 31, 600], seed=6, dtype="f16")
    (a, b), _, _ = run(case, cuda, 16, calls=2)
    assert dial_b200.device_status() == 0
    ref, _, _ = case.oracle()
    assert_attn_close(a, ref, "f16")
    np.testing.assert_array_equal(a, b)


@pytest.mark.parametrize("qh,kvh,dtype", [(32, 8, "bf16"), (40, 8, "bf16"), (8, 8, "bf16"),
                                          (16, 8, "f16"), (8, 1, "f16")])
@pytest.mark.parametrize("splits", [1, 4, 16])
def test_attention_decode_tensor_core_form(cuda, qh, kvh, dtype, splits):
    """More than 4 rows with the pool size given take the tensor-core form
    (attn_decode_mma.cu: TMA-staged pages, mma.sync scores and P.V with the
    probabilities split into two act terms): group sizes 1, 2, 4, 5 and 8,
    one-token, page-edge and long contexts, the new token's row patched into
    its landed page, the appended K/V, and a repeat call bit for bit."""
    import dial_b200

    case = PagedCase(qh, kvh, [0, 1, 15, 16, 17, 200, 777, 1023], seed=qh + 7 * kvh + splits,
                     dtype=dtype)
    (a, b), dev, _ = run(case, cuda, splits, calls=2, num_blocks=case.rows * case.max_blocks)
    assert dial_b200.device_status() == 0
    ref, kref, vref = case.oracle()
    assert_attn_close(a, ref, dtype)
    np.testing.assert_array_equal(a, b)
    k, v = case.new_kv(dev["k_pages"], dev["v_pages"])
    np.testing.assert_array_equal(v, vref)
    assert np.all(np.abs(k - kref) <= ulp(kref, dtype))


def test_attention_decode_tensor_core_form_matches_cuda_core_form(cuda):
    """Both many-row forms against each other on one long-context case: the
    tensor-core form's two-term probabilities keep it as close to the
    CUDA-core form's f32 probabilities as either is to the oracle."""
    case = PagedCase(32, 8, [1000, 513, 64, 0, 250, 1023, 31, 600], seed=21)
    (tc,), _, _ = run(case, cuda, 16, num_blocks=case.rows * case.max_blocks)
    (cc,), _, _ = run(case, cuda, 16)
    ref, _, _ = case.oracle()
    assert_attn_close(tc, ref, "bf16")
    d = np.abs(tc - cc)
    assert np.mean(d <= ulp(np.maximum(np.abs(cc), 1e-3), "bf16")) >= 0.99


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("splits", [8, 16])
def test_attention_decode_cluster_token_split(cuda, monkeypatch, dtype, splits):
    """The opt-in token split inside the cluster-merge form
    (DIAL_B200_ATTN_TOKSPLIT=2: steps of up to 4 rows, groups of 4 query
    heads, splits a multiple of the cluster) against the oracle, the appended
    V, and a repeat call bit for bit."""
    import dial_b200

    monkeypatch.setenv("DIAL_B200_ATTN_TOKSPLIT", "2")
    case = PagedCase(32, 8, [0, 200, 777, 1023], seed=40 + splits, dtype=dtype)
    (a, b), dev, _ = run(case, cuda, splits, calls=2)
    assert dial_b200.device_status() == 0
    ref, _, vref = case.oracle()
    assert_attn_close(a, ref, dtype)
    np.testing.assert_array_equal(a, b)
    _, v = case.new_kv(dev["k_pages"], dev["v_pages"])
    np.testing.assert_array_equal(v, vref)


@pytest.mark.parametrize("rows", [2, 8])
def test_attention_decode_block_id_outside_pool(cuda, rows):
    """With the pool size given, a block id outside [0, num_blocks) in the
    caller's table records the bad-argument device status and reads page 0
    instead (the page-ring form for 2 rows, the tensor-core form for 8); the
    status clears."""
    import dial_b200
    import torch
    from dial_b200 import attention as A

    dial_b200.device_status(clear=True)
    case = PagedCase(32, 8, [100, 300, 5, 64, 200, 17, 900, 40][:rows], seed=70 + rows)
    nb = case.rows * case.max_blocks
    sh = A.make_shape(case.QH, case.KVH, case.max_blocks, case.max_pos, case.eps, num_blocks=nb)
    dev = case.device(cuda)
    dev["block_table"][0, 3] = nb + 5  # a page row 0 reads (position 100)
    dev["block_table"][1, 0] = -1
    scratch = torch.zeros(max(A.scratch_bytes(sh, case.rows, 4), 16), dtype=torch.uint8, device=cuda)
    A.attention_decode(sh, splits=4, scratch=scratch, **dev)
    torch.cuda.synchronize()
    assert dial_b200.device_status(clear=True) == 0x104  # bad arguments
    assert dial_b200.device_status() == 0


def test_attention_decode_repeat_calls_agree(cuda):
    """Scratch counters reset themselves: a second call (which re-appends the
    same K/V) reproduces the first bit for bit."""
    case = PagedCase(32, 8, [300, 40, 900, 5], seed=11)
    (a, b), _, _ = run(case, cuda, 8, calls=2)
    np.testing.assert_array_equal(a, b)


def test_attention_decode_rejects_bad_args(cuda):
    import dial_b200
    from dial_b200 import attention as A

    case = PagedCase(8, 2, [3], seed=1)
    dev = case.device(cuda)
    sh = A.make_shape(8, 2, case.max_blocks, case.max_pos)
    with pytest.raises(dial_b200.DialError, match="splits > 1 needs scratch"):
        A.attention_decode(sh, splits=2, scratch=None, **dev)
    bad = A.make_shape(8, 3, case.max_blocks, case.max_pos)
    with pytest.raises(dial_b200.DialError, match="multiple of kv_heads"):
        A.attention_decode(bad, **dev)
