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
