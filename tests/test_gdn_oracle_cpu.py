"""The Gated-DeltaNet oracle (oracle/dial_oracle.py, qwen3_8/text.rs:233-481)
on its own: the state carried between calls makes a prefill of S tokens equal
to a prefill of S-3 tokens followed by three single-token calls, bit for bit
(the reference's cache contract, llama3/cache.rs:267-290); a zero decay and
beta of one reduce the recurrence to the delta rule's exact key recall."""

import numpy as np

import dial_oracle as O


def _params(rng, C, K, hv, act="bf16"):
    return dict(conv_w=O.act_round(rng.standard_normal((C, K)).astype(np.float32) * 0.5, act),
                dt_bias=O.bf16_round(rng.standard_normal(hv).astype(np.float32) * 0.5),
                a_log=O.bf16_round(rng.uniform(-1, 1, hv).astype(np.float32)),
                norm_w=O.bf16_round(1 + 0.1 * rng.standard_normal(128).astype(np.float32)))


def test_chunked_calls_equal_one_prefill():
    rng = np.random.default_rng(3)
    hk, hv, K, S = 2, 4, 4, 9
    C = 2 * hk * 128 + hv * 128
    p = _params(rng, C, K, hv)
    r = lambda *s: O.bf16_round(rng.standard_normal(s).astype(np.float32))  # noqa: E731
    mixed, z, b, a = r(S, C), r(S, hv * 128), r(S, hv), r(S, hv)
    args = (p["conv_w"], p["dt_bias"], p["a_log"], p["norm_w"], hk, hv, 128, 128, 1e-6)
    whole, st_whole = O.gdn_mixer(mixed, z, b, a, *args, None)
    parts, st = [], None
    for lo, hi in ((0, S - 3), (S - 3, S - 2), (S - 2, S - 1), (S - 1, S)):
        out, st = O.gdn_mixer(mixed[lo:hi], z[lo:hi], b[lo:hi], a[lo:hi], *args, st)
        parts.append(out)
    np.testing.assert_array_equal(np.concatenate(parts), whole)
    np.testing.assert_array_equal(st.recurrent, st_whole.recurrent)
    np.testing.assert_array_equal(st.conv, st_whole.conv)


def test_delta_rule_recall():
    """With g = 0 (no decay) and beta = 1, writing value v under unit key k
    and then reading with q = k returns v exactly for an orthogonal key set."""
    H, dk, dv = 1, 128, 128
    keys = np.eye(dk, dtype=np.float32)[:3][None]  # [1, 3, dk] orthonormal
    vals = np.arange(3 * dv, dtype=np.float32).reshape(1, 3, dv) / 64
    g = np.zeros((H, 3), np.float32)
    beta = np.ones((H, 3), np.float32)
    _, st = O.gdn_recurrent_scan(keys, keys, vals, g, beta, np.zeros((H, dk, dv), np.float32))
    out, _ = O.gdn_recurrent_scan(keys, keys, np.zeros_like(vals), g, np.zeros((H, 3), np.float32),
                                  st)
    np.testing.assert_array_equal(out, vals)


def test_conv_state_is_the_last_inputs():
    rng = np.random.default_rng(1)
    x = O.bf16_round(rng.standard_normal((2, 5)).astype(np.float32))
    w = O.bf16_round(rng.standard_normal((5, 4)).astype(np.float32))
    _, st = O.gdn_causal_conv(x, w, None)
    assert st.shape == (5, 3)
    np.testing.assert_array_equal(st[:, 1:], x.T)  # zero-padded history, then the 2 inputs
    np.testing.assert_array_equal(st[:, 0], np.zeros(5, np.float32))
