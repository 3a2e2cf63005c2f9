"""27B-class formats end to end (at test size): engines
whose linears are FP8 e4m3 with 128x128 block scales or NVFP4 (e2m1 + e4m3
group scale + f32 global), synthesised and quantised on the device, against
the oracle model whose linears are the same weights quantised by the CPU
quantisers (quantize_fp8_block128 / quantize_nvfp4, cuda_quant.rs:11-65
decode) and applied densely."""

import numpy as np
import pytest
import torch

import dial_oracle as O
from test_layer_gpu import assert_hidden_close, small_cfg

pytestmark = pytest.mark.gpu


def _oracle_model(cfg, seed, fmt):
    """synth_model with every layer linear replaced by its FP8/NVFP4 dequant."""
    import dial_b200

    table = O.normal_table(0.02)
    H, I, D, QH, KVH = cfg.hidden, cfg.inter, cfg.head_dim, cfg.heads, cfg.kv_heads
    st = lambda l, p: ((l + 1) << 8) + p  # noqa: E731

    def quant(w):
        n, k = w.shape
        if fmt == dial_b200.FMT_FP8_BLOCK128:
            codes, sc = O.quantize_fp8_block128(w)
            return O.fp8_block_dense_weight(codes, sc, k, n)
        packed, sc, gs = O.quantize_nvfp4(w)
        return O.nvfp4_dense_weight(packed, sc, gs, k, n)

    base = O.synth_model(cfg, seed)
    one = lambda n: np.ones(n, np.float32)  # noqa: E731
    layers = []
    for l in range(cfg.layers):
        nrm = lambda s_, n, k: O.synth_normal(seed, st(l, s_), n * k, table).reshape(n, k)  # noqa: E731
        qkv = quant(np.concatenate([nrm(0, QH * D, H), nrm(1, KVH * D, H), nrm(2, KVH * D, H)]))
        o = quant(nrm(3, H, QH * D))
        gu = quant(np.concatenate([nrm(4, I, H), nrm(5, I, H)]))
        dn = quant(nrm(6, H, I))
        layers.append(O.LayerWeights(qkv, one(qkv.shape[0]), o, one(H), gu, one(2 * I), dn, one(H),
                                     one(H), one(H), one(D), one(D)))
    return O.Model(cfg, base.embed, layers, base.final_norm, base.lm_head, "bf16")


@pytest.mark.parametrize("fmt_name", ["FMT_FP8_BLOCK128", "FMT_NVFP4_G16"])
@pytest.mark.parametrize("n_prompt,wide", [(9, False), (80, False), (40, True)])
def test_synthetic_quantised_model_matches_oracle(cuda, fmt_name, n_prompt, wide):
    """The wide case (hidden 1024, FFN 2048, 40 rows) runs its projections as
    split-K tensor-core GEMMs (few 128-row tiles, K long enough to cut)."""
    import dial_b200

    fmt = getattr(dial_b200, fmt_name)
    if wide:
        cfg = small_cfg(hidden=1024, inter=2048, heads=8, kv_heads=2, layers=1, vocab=1000)
    else:
        cfg = small_cfg(hidden=256, inter=512, heads=2, kv_heads=1, layers=2, vocab=1000)
    dcfg = dial_b200.Config(hidden_size=cfg.hidden, intermediate_size=cfg.inter,
                            vocab_size=cfg.vocab, num_hidden_layers=cfg.layers,
                            num_attention_heads=cfg.heads, num_key_value_heads=cfg.kv_heads,
                            rms_norm_eps=cfg.eps, rope_theta=cfg.rope_theta,
                            max_seq_len=cfg.max_seq_len, max_tokens=128, linear_fmt=fmt)
    eng = dial_b200.Engine(dcfg)
    eng.load_synthetic(seed=5)
    model = _oracle_model(cfg, 5, fmt)
    prompt = O.synth_tokens(1, n_prompt, cfg.vocab)
    # hidden state after the layers, through the Forwarder API
    x = model.embed[prompt.astype(np.int64)]
    ref = x.copy()
    cache = O.Cache(cfg.layers, cfg.max_seq_len)
    for l, lw in enumerate(model.layers):
        ref = O.layer_forward(ref, lw, cfg, 0, l, cache, model.cos, model.sin)
    xt = torch.from_numpy(x).to(cuda).to(torch.bfloat16)
    eng.forward_local_batch(xt, [(f"model.layers.{i}", 0, i) for i in range(cfg.layers)])
    torch.cuda.synchronize()
    assert dial_b200.device_status() == 0
    assert_hidden_close(xt.float().cpu().numpy(), ref)
