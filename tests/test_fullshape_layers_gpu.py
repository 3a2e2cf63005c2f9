"""Decoder layers at the benchmark shapes against the C++ oracle
(oracle/dial_oracle_c.cpp, equal to oracle/dial_oracle.py).

* one decode step of 32 ragged sessions (KV lengths
  uniform in [128, 8192], seed 2, the bench's draw) through two Qwen3-8B-shape
  W8A16 layers (hidden 4096, 32 q / 8 kv heads, FFN 12288) in one
  dial_b200_batch_decode_forward call: the 32-row split-K GEMMs and the
  token-split decode attention over 16-token pages filled by
  dial_b200_session_fill_random, which the oracle's cache mirrors.
* one 27B-class layer (hidden 5120, 40 q / 8 kv heads, FFN
  21504) with FP8 e4m3 128 x 128 block-scaled or NVFP4 (e2m1, e4m3 group of
  16, f32 global) linears quantised on the device: a 40-token prefill (split-K
  GEMMs, prefill attention) then one decode token (GEMV, decode attention).

Both use the single-layer hidden-state tolerance of tests/test_layer_gpu.py
against the oracle with either softmax-probability rounding; the ragged case
(two W8A16 layers) also holds mean |d| <= 2^-8 rms against the oracle with f32
probabilities (the kernels' choice).  The FP8 block-128 GEMM rounds each
e4m3 x block-scale weight to f16 for its MMA operand, which keeps the 27B
layer inside the single-layer tolerance but above that tighter mean."""

import numpy as np
import pytest
import torch

import dial_oracle as O
import dial_oracle_fast as F
from test_layer_gpu import assert_hidden_close

pytestmark = pytest.mark.gpu


def test_ragged32_sessions_qwen3_8b_two_layers(cuda):
    import dial_b200

    n_sess, layers = 32, 2
    lengths = np.random.default_rng(2).integers(128, 8193, size=n_sess).astype(np.int32)
    cap = 8192 + 16
    cfg = dial_b200.Config(num_hidden_layers=layers, max_seq_len=cap, max_sessions=n_sess,
                           max_tokens=64)
    eng = dial_b200.Engine(cfg, has_embed=False, has_head=False)
    eng.load_synthetic(seed=0)
    fm = F.FastModel(O.ModelConfig(layers=layers, max_seq_len=cap), seed=0, has_embed=False,
                     has_head=False)
    rows = O.bf16_round(np.random.default_rng(3).standard_normal((n_sess, cfg.hidden_size),
                                                                  dtype=np.float32))
    ref, tight = [], []
    for s, L in enumerate(lengths.tolist()):
        eng.session_fill_random(s, L, seed=2 + s)
        for rp, out in ((True, ref), (False, tight)):
            c = fm.new_cache()
            c.fill_random(s, L, seed=2 + s)
            y = rows[s:s + 1].copy()
            fm.forward(y, c, L, round_probs=rp)
            out.append(y[0])
            del c
    xt = torch.from_numpy(rows).to(cuda).to(torch.bfloat16)
    eng.batch_decode(xt, list(range(n_sess)), lengths)
    torch.cuda.synchronize()
    assert dial_b200.device_status() == 0
    got = xt.float().cpu().numpy()
    assert_hidden_close(got, np.stack(ref))
    # same probability rounding as the kernels; two full-size layers: 2^-8 mean
    assert_hidden_close(got, np.stack(tight), mean_rel=2 ** -8, ulps=4, frac=0.99)
    eng.close()


@pytest.mark.parametrize("fmt_name", ["FMT_FP8_BLOCK128", "FMT_NVFP4_G16"])
def test_27b_layer_prefill_then_decode(cuda, fmt_name):
    import dial_b200

    fmt = getattr(dial_b200, fmt_name)
    ofmt = F.FMT_FP8_BLOCK128 if fmt == dial_b200.FMT_FP8_BLOCK128 else F.FMT_NVFP4
    cfg = dial_b200.Config.dense_27b(num_hidden_layers=1, max_seq_len=256, max_sessions=1,
                                     max_tokens=64, linear_fmt=fmt)
    eng = dial_b200.Engine(cfg, has_embed=False, has_head=False)
    eng.load_synthetic(seed=0)
    ocfg = O.ModelConfig(hidden=5120, inter=21504, heads=40, kv_heads=8, layers=1,
                         max_seq_len=256)
    fm = F.FastModel(ocfg, seed=0, fmt=ofmt, has_embed=False, has_head=False)
    rng = np.random.default_rng(11)
    S = 40
    x = O.bf16_round(rng.standard_normal((S + 1, ocfg.hidden), dtype=np.float32))
    for rp in (True, False):
        c = fm.new_cache()
        y = x[:S].copy()
        fm.forward(y, c, 0, round_probs=rp)
        y1 = x[S:].copy()
        fm.forward(y1, c, S, round_probs=rp)
        if rp:
            ref, ref1 = y, y1
        else:
            tight, tight1 = y, y1
    xt = torch.from_numpy(x[:S]).to(cuda).to(torch.bfloat16).contiguous()
    eng.forward(xt, 0, 0)
    x1 = torch.from_numpy(x[S:]).to(cuda).to(torch.bfloat16).contiguous()
    eng.forward(x1, S, 0)
    torch.cuda.synchronize()
    assert dial_b200.device_status() == 0
    got, got1 = xt.float().cpu().numpy(), x1.float().cpu().numpy()
    assert_hidden_close(got, ref)
    assert_hidden_close(got1, ref1)
    assert_hidden_close(got, tight)
    assert_hidden_close(got1, tight1)
    eng.close()
