"""Gated-DeltaNet mixer (dial_b200_gdn_forward) against the oracle restatement
of GatedDeltaNet::forward (qwen3_8/text.rs:390-481) at the official Qwen3.8
linear-attention shape (16 key heads, 48 value heads, head dims 128, conv
kernel 4): a prefill at index_pos 0, then decode tokens that carry the conv
and recurrent state on the device, in bf16 and f16.

Tolerance: the kernel sums in f32 in another order than the oracle's f64
sums, and the recurrence feeds rounding differences forward, so the gated
output is held to max |d| <= 2^-5 max|ref| + 1e-3 and 99 % of elements within
4 ulp of max(|ref|, rms); the f32 recurrent state to a relative L2 error of
2^-10."""

import numpy as np
import pytest
import torch

import dial_oracle as O

pytestmark = pytest.mark.gpu


def _case(rng, S, hk, hv, act):
    C = 2 * hk * 128 + hv * 128
    r = lambda *s, sc=1.0: O.act_round(rng.standard_normal(s).astype(np.float32) * sc, act)  # noqa: E731
    return dict(mixed=r(S, C), z=r(S, hv * 128), b=r(S, hv), a=r(S, hv))


@pytest.mark.parametrize("act", ["bf16", "f16"])
def test_gdn_prefill_then_decode_matches_oracle(cuda, act):
    from dial_b200 import gdn

    hk, hv, K, eps = 16, 48, 4, 1e-6
    dt = torch.bfloat16 if act == "bf16" else torch.float16
    rng = np.random.default_rng(12)
    C = 2 * hk * 128 + hv * 128
    conv_w = O.act_round(rng.standard_normal((C, K)).astype(np.float32) * 0.5, act)
    dt_bias = O.bf16_round(rng.standard_normal(hv).astype(np.float32) * 0.5)
    a_log = O.bf16_round(rng.uniform(-1.0, 1.0, hv).astype(np.float32))
    norm_w = O.bf16_round(1.0 + 0.1 * rng.standard_normal(128).astype(np.float32))
    sh = gdn.make_shape(hk, hv, K, eps, dt)
    state = gdn.GdnState.empty(sh, cuda, dt)
    ref_state = None
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(cuda).to(dt)  # noqa: E731
    pos = 0
    for S in (21, 1, 1, 3):
        c = _case(rng, S, hk, hv, act)
        ref, ref_state = O.gdn_mixer(c["mixed"], c["z"], c["b"], c["a"], conv_w, dt_bias, a_log,
                                     norm_w, hk, hv, 128, 128, eps, ref_state, act)
        got = gdn.gdn_forward(sh, t(c["mixed"]), t(c["z"]), t(c["b"]), t(c["a"]), t(conv_w),
                              torch.from_numpy(dt_bias), torch.from_numpy(a_log),
                              torch.from_numpy(norm_w), state, pos)
        torch.cuda.synchronize()
        g = got.float().cpu().numpy()
        d = np.abs(g - ref)
        rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
        assert float(d.max()) <= 2 ** -5 * float(np.abs(ref).max()) + 1e-3, (S, pos, d.max())
        mant = 7 if act == "bf16" else 10
        ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(ref), rms))) - mant)
        assert np.mean(d <= 4 * ulp) >= 0.99, (S, pos, np.mean(d <= 4 * ulp))
        rec = state.recurrent.cpu().numpy()
        rel = np.linalg.norm(rec - ref_state.recurrent) / np.linalg.norm(ref_state.recurrent)
        assert rel <= 2 ** -10, (S, pos, rel)
        np.testing.assert_array_equal(state.conv.float().cpu().numpy(), ref_state.conv)
        pos += S


def test_gdn_rejects_bad_shapes(cuda):
    import dial_b200
    from dial_b200 import gdn

    sh = gdn.make_shape(16, 40, 4)  # 40 % 16 != 0
    z = torch.zeros(1, 40 * 128, dtype=torch.bfloat16, device=cuda)
    st = gdn.GdnState(torch.zeros(1, 3, dtype=torch.bfloat16, device=cuda),
                      torch.zeros(1, dtype=torch.float32, device=cuda))
    x = torch.zeros(1, 8, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(dial_b200.DialError, match="not a multiple"):
        gdn.gdn_forward(sh, x, z, x, x, x, torch.zeros(40), torch.zeros(40), torch.zeros(128),
                        st, 0)
