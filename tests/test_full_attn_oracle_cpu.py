"""The Qwen3.8 gated full-attention oracle (oracle/dial_oracle.py,
qwen3_8/text.rs:82-226) on its own: the partial RoPE reduces to the full one
when it covers every dim; the session cache makes a prefill of S tokens equal
to a shorter prefill followed by single-token calls, bit for bit
(llama3/cache.rs:117-160); and each head's gate sits next to its own query
(text.rs:155-166), so closing one head's gate silences that head only."""

import numpy as np

import dial_oracle as O

HEADS, KVH, D, ROT = 4, 2, 256, 64


def _inputs(rng, S):
    r = lambda *s: O.bf16_round(rng.standard_normal(s).astype(np.float32))  # noqa: E731
    return r(S, HEADS * 2 * D), r(S, KVH * D), r(S, KVH * D)


def _norms(rng):
    w = lambda: O.bf16_round(0.1 * rng.standard_normal(D).astype(np.float32))  # noqa: E731
    return w(), w()


def _tables(n):
    cos, sin = O.rope_tables(ROT, n, 1e7)
    return cos, sin


def test_rope_partial_over_every_dim_is_rope():
    rng = np.random.default_rng(1)
    x = O.bf16_round(rng.standard_normal((3, 5, 64)).astype(np.float32))
    cos, sin = O.rope_tables(64, 5, 1e6)
    np.testing.assert_array_equal(O.rope_partial(x, cos, sin, 64), O.rope(x, cos, sin))
    # a quarter of the dims rotated: the rest is passed through
    cos4, sin4 = O.rope_tables(16, 5, 1e6)
    y = O.rope_partial(x, cos4, sin4, 16)
    np.testing.assert_array_equal(y[..., 16:], x[..., 16:])
    np.testing.assert_array_equal(y[..., :16], O.rope(x[..., :16], cos4, sin4))


def test_chunked_calls_equal_one_prefill():
    rng = np.random.default_rng(2)
    S = 9
    qg, k, v = _inputs(rng, S)
    qn, kn = _norms(rng)
    cos, sin = _tables(S)
    args = (qn, kn, HEADS, KVH, D, ROT)
    whole, st_whole = O.gated_full_attention(qg, k, v, *args, cos, sin, 1e-6, 0, None)
    parts, st = [], None
    for lo, hi in ((0, S - 3), (S - 3, S - 2), (S - 2, S - 1), (S - 1, S)):
        out, st = O.gated_full_attention(qg[lo:hi], k[lo:hi], v[lo:hi], *args, cos[lo:hi],
                                         sin[lo:hi], 1e-6, lo, st)
        parts.append(out)
    np.testing.assert_array_equal(np.concatenate(parts), whole)
    np.testing.assert_array_equal(st.k, st_whole.k)
    np.testing.assert_array_equal(st.v, st_whole.v)


def test_each_head_reads_its_own_gate():
    rng = np.random.default_rng(3)
    S = 5
    qg, k, v = _inputs(rng, S)
    qn, kn = _norms(rng)
    cos, sin = _tables(S)
    args = (qn, kn, HEADS, KVH, D, ROT, cos, sin, 1e-6, 0, None)
    open_all = qg.reshape(S, HEADS, 2 * D).copy()
    open_all[:, :, D:] = 30.0  # sigmoid -> 1
    half = open_all.copy()
    half[:, 1::2, D:] = -30.0  # odd heads closed
    ref, _ = O.gated_full_attention(open_all.reshape(S, -1), k, v, *args)
    got, _ = O.gated_full_attention(half.reshape(S, -1), k, v, *args)
    ref = ref.reshape(S, HEADS, D)
    got = got.reshape(S, HEADS, D)
    np.testing.assert_array_equal(got[:, 0::2], ref[:, 0::2])
    assert np.max(np.abs(got[:, 1::2])) < 1e-9 * max(1.0, float(np.max(np.abs(ref))))


def test_f32_attention_close_to_bf16():
    rng = np.random.default_rng(4)
    S = 7
    qg, k, v = _inputs(rng, S)
    qn, kn = _norms(rng)
    cos, sin = _tables(S)
    args = (qn, kn, HEADS, KVH, D, ROT, cos, sin, 1e-6, 0, None)
    a, _ = O.gated_full_attention(qg, k, v, *args)
    b, _ = O.gated_full_attention(qg, k, v, *args, attn_f32=True)
    np.testing.assert_allclose(a, b, rtol=0.05, atol=0.02)
