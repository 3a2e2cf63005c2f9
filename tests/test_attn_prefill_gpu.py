"""Prefill attention on the tensor cores (tcgen05 flash pass over paged KV,
prompts of >= 64 tokens) against the oracle's causal grouped attention
(text.rs:1283-1327, cache.rs:102-160) and against the CUDA-core path."""

import os

import numpy as np
import pytest
import torch

import dial_oracle as O
from test_layer_gpu import assert_hidden_close, engine_for, random_layer, small_cfg

pytestmark = pytest.mark.gpu


def _run(cfg, lw, chunks, cuda, tc: bool):
    import dial_b200

    old = os.environ.get("DIAL_B200_ATTN_TC")
    os.environ["DIAL_B200_ATTN_TC"] = "1" if tc else "0"
    try:
        eng = engine_for(cfg, dial_b200, max_tokens=320)
        eng.set_layer_w8a16(0, lw)
        outs, pos = [], 0
        for x in chunks:
            xt = torch.from_numpy(x).to(cuda).to(torch.bfloat16)
            eng.forward(xt, pos, 0)
            torch.cuda.synchronize()
            outs.append(xt.float().cpu().numpy())
            pos += x.shape[0]
        assert dial_b200.device_status() == 0
        return outs
    finally:
        if old is None:
            os.environ.pop("DIAL_B200_ATTN_TC", None)
        else:
            os.environ["DIAL_B200_ATTN_TC"] = old


@pytest.mark.parametrize("heads,kv,lens", [(8, 2, [64]), (8, 2, [200]), (4, 1, [300]),
                                           (8, 8, [130]), (10, 2, [96, 160])])
def test_prefill_attention_tensor_cores(cuda, heads, kv, lens):
    cfg = small_cfg(heads=heads, kv_heads=kv, hidden=128 * heads, inter=512, layers=1,
                    max_seq_len=512)
    lw = random_layer(cfg, 4)
    rng = np.random.default_rng(12)
    chunks = [O.bf16_round(rng.standard_normal((n, cfg.hidden)).astype(np.float32)) for n in lens]
    cos, sin = O.rope_tables(cfg.head_dim, cfg.max_seq_len, cfg.rope_theta)
    cache = O.Cache(1, cfg.max_seq_len)
    refs, pos = [], 0
    for x in chunks:
        refs.append(O.layer_forward(x, lw, cfg, pos, 0, cache, cos, sin))
        pos += x.shape[0]
    tc = _run(cfg, lw, chunks, cuda, tc=True)
    cc = _run(cfg, lw, chunks, cuda, tc=False)
    for got, alt, ref in zip(tc, cc, refs):
        assert_hidden_close(got, ref)
        assert_hidden_close(alt, ref)
        assert_hidden_close(got, alt)
