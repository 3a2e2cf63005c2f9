"""A dense bf16 Qwen3 checkpoint written to safetensors and loaded with
load_checkpoint (dense linears quantised to W8A16 on the device,
worker_w8a16.rs:302-366) decodes like the oracle model built from the same
weights: hidden states after the layers, and greedy tokens."""

import numpy as np
import pytest
import torch
from safetensors.torch import save_file

import dial_oracle as O
from test_layer_gpu import assert_hidden_close, engine_for, small_cfg

pytestmark = pytest.mark.gpu


def _checkpoint(tmp_path, cfg, seed):
    rng = np.random.default_rng(seed)
    H, I, D = cfg.hidden, cfg.inter, cfg.head_dim
    w = lambda n, k: O.bf16_round(rng.standard_normal((n, k)).astype(np.float32) * 0.02)  # noqa: E731
    nw = lambda n: O.bf16_round(1.0 + 0.1 * rng.standard_normal(n).astype(np.float32))  # noqa: E731
    bf = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(torch.bfloat16)  # noqa: E731
    t, layers = {}, []
    for l in range(cfg.layers):
        p = f"model.layers.{l}."
        q, k, v = w(cfg.heads * D, H), w(cfg.kv_heads * D, H), w(cfg.kv_heads * D, H)
        o, g, u, d = w(H, cfg.heads * D), w(I, H), w(I, H), w(H, I)
        norms = [nw(H), nw(H), nw(D), nw(D)]
        for name, a in (("self_attn.q_proj", q), ("self_attn.k_proj", k), ("self_attn.v_proj", v),
                        ("self_attn.o_proj", o), ("mlp.gate_proj", g), ("mlp.up_proj", u),
                        ("mlp.down_proj", d)):
            t[p + name + ".weight"] = bf(a)
        for name, a in zip(("input_layernorm", "post_attention_layernorm", "self_attn.q_norm",
                            "self_attn.k_norm"), norms):
            t[p + name + ".weight"] = bf(a)
        layers.append(O.LayerWeights(*O.quantize_w8a16_rows(np.concatenate([q, k, v])),
                                     *O.quantize_w8a16_rows(o),
                                     *O.quantize_w8a16_rows(np.concatenate([g, u])),
                                     *O.quantize_w8a16_rows(d), *norms))
    embed, final, head = w(cfg.vocab, H), nw(H), w(cfg.vocab, H)
    t["model.embed_tokens.weight"], t["model.norm.weight"], t["lm_head.weight"] = \
        bf(embed), bf(final), bf(head)
    save_file(t, str(tmp_path / "model.safetensors"))
    return O.Model(cfg, embed, layers, final, head, "bf16")


def test_dense_checkpoint_matches_oracle(cuda, tmp_path):
    import dial_b200

    cfg = small_cfg(hidden=512, inter=1024, heads=4, kv_heads=1, layers=2, vocab=1000)
    model = _checkpoint(tmp_path, cfg, 21)
    eng = engine_for(cfg, dial_b200)
    dial_b200.load_checkpoint(eng, tmp_path)
    # hidden states after the layers (Forwarder API), 40-row prefill
    prompt = O.synth_tokens(1, 40, cfg.vocab)
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
    # greedy decode from a fresh session, teacher-forced against the oracle
    eng.session_reset(0)
    prompt = prompt[:12].tolist()
    toks, _, _ = eng.generate(prompt, 6)
    ref_toks, ref_logits = O.greedy_generate(model, prompt, 6, forced=toks)
    for i, (a, b) in enumerate(zip(toks.tolist(), ref_toks)):
        if a != b:  # a disagreement must be a near tie under the oracle
            lg = ref_logits[i]
            assert lg[b] - lg[a] <= 2 * 2.0 ** (np.floor(np.log2(abs(lg[b]))) - 7) + 1e-6
    assert dial_b200.device_status() == 0
