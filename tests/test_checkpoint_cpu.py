"""Safetensors loading on the host: format detection in the reference's order
(qwen3_8/quant.rs:448-501), NVFP4 global-scale conventions (compressed-tensors
divisor vs ModelOpt multiplier, quant.rs:304-311, 376-399), FP8 scale shapes
(quant.rs:316-345, 406-429), q|k|v and gate|up fusion (qwen3_vl/text.rs:
1428-1431, 634-636), and lm_head lookup with tied embeddings
(qwen3_vl.rs:3099-3127).  The engine is a recorder, so no GPU is needed; dense
weights go through the oracle's W8A16 quantizer (worker_w8a16.rs:330-341)."""

import json

import numpy as np
import pytest
import torch
from safetensors.torch import save_file

import dial_oracle as O

H, I, QH, KVH, D, V, LAYERS = 256, 512, 2, 1, 128, 64, 2


class Recorder:
    """Engine stand-in: records set_linear / set_tensor calls."""

    def __init__(self, first_layer=0, num_layers=LAYERS, has_embed=True, has_head=True):
        from dial_b200 import Config

        self.cfg = Config(hidden_size=H, intermediate_size=I, vocab_size=V,
                          num_hidden_layers=LAYERS, num_attention_heads=QH,
                          num_key_value_heads=KVH)
        self.first_layer, self.num_layers = first_layer, num_layers
        self.has_embed, self.has_head = has_embed, has_head
        self.linears, self.tensors = {}, {}

    def set_linear(self, layer, which, fmt, codes, scales=None, global_scale=0.0):
        self.linears[(layer, which)] = (fmt, np.asarray(codes), None if scales is None
                                        else np.asarray(scales), float(global_scale))

    def set_tensor(self, layer, which, values):
        self.tensors[(layer, which)] = np.asarray(values)


def _shapes():
    return {"self_attn.q_proj": (QH * D, H), "self_attn.k_proj": (KVH * D, H),
            "self_attn.v_proj": (KVH * D, H), "self_attn.o_proj": (H, QH * D),
            "mlp.gate_proj": (I, H), "mlp.up_proj": (I, H), "mlp.down_proj": (H, I)}


def _dense(rng, shape):
    return torch.from_numpy((rng.standard_normal(shape) * 0.02).astype(np.float32)).to(torch.bfloat16)


def _write(tmp_path, tensors, config=None, name="model.safetensors"):
    save_file({k: v.contiguous() for k, v in tensors.items()}, str(tmp_path / name))
    if config is not None:
        (tmp_path / "config.json").write_text(json.dumps(config))
    return tmp_path


def _base(rng, pre, form, head=True):
    """A 2-layer checkpoint whose projections are stored as `form`."""
    t = {}
    for l in range(LAYERS):
        lp = f"{pre}layers.{l}."
        for nm, shp in _shapes().items():
            w = _dense(rng, shp)
            p = lp + nm + "."
            if form == "dense":
                t[p + "weight"] = w
            elif form == "fp8_tensor" or form == "fp8_row":
                wf = w.float().numpy()
                s = (np.abs(wf).max() if form == "fp8_tensor" else np.abs(wf).max(axis=1)) / 448.0
                s = np.asarray(s, np.float32)
                codes = O.f32_to_e4m3(wf / (s if s.ndim == 0 else s[:, None]))
                t[p + "weight"] = torch.from_numpy(codes).view(torch.float8_e4m3fn)
                t[p + "weight_scale"] = torch.from_numpy(s.reshape(-1) if s.ndim else s.reshape(()))
            elif form == "fp8_block":
                codes, sc = O.quantize_fp8_block128(w.float().numpy())
                t[p + "weight"] = torch.from_numpy(codes).view(torch.float8_e4m3fn)
                t[p + "weight_scale"] = torch.from_numpy(sc.astype(np.float32))
            elif form in ("nvfp4_ct", "nvfp4_mo"):
                packed, sc, gs = O.quantize_nvfp4(w.float().numpy(), global_scale=1e-3)
                sct = torch.from_numpy(sc).view(torch.float8_e4m3fn)
                if form == "nvfp4_ct":
                    t[p + "weight_packed"] = torch.from_numpy(packed)
                    t[p + "weight_scale"] = sct
                    t[p + "weight_global_scale"] = torch.tensor([1.0 / gs], dtype=torch.float32)
                else:
                    t[p + "weight"] = torch.from_numpy(packed)
                    t[p + "weight_scale"] = sct
                    t[p + "weight_scale_2"] = torch.tensor(gs, dtype=torch.float32)
        for nm in ("input_layernorm", "post_attention_layernorm"):
            t[lp + nm + ".weight"] = _dense(rng, (H,)) + 1
        t[lp + "self_attn.q_norm.weight"] = _dense(rng, (D,)) + 1
        t[lp + "self_attn.k_norm.weight"] = _dense(rng, (D,)) + 1
    t[pre + "embed_tokens.weight"] = _dense(rng, (V, H))
    t[pre + "norm.weight"] = _dense(rng, (H,)) + 1
    if head:
        t["lm_head.weight"] = _dense(rng, (V, H))
    return t


def _bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _load(path, **kw):
    from dial_b200 import load_checkpoint

    eng = Recorder(**kw)
    load_checkpoint(eng, path, quantize=lambda w: O.quantize_w8a16_rows(w.float().numpy()))
    return eng


def test_dense_checkpoint_quantises_and_fuses(tmp_path):
    import dial_b200

    t = _base(np.random.default_rng(0), "model.", "dense")
    eng = _load(_write(tmp_path, t))
    for l in range(LAYERS):
        fmt, codes, scales, _ = eng.linears[(l, 0)]
        assert fmt == dial_b200.FMT_W8A16_ROW
        w = torch.cat([t[f"model.layers.{l}.self_attn.{p}.weight"] for p in ("q_proj", "k_proj",
                                                                              "v_proj")])
        q, s = O.quantize_w8a16_rows(w.float().numpy())
        np.testing.assert_array_equal(codes, q)
        np.testing.assert_array_equal(scales, s)
        fmt, codes, _, _ = eng.linears[(l, 2)]
        w = torch.cat([t[f"model.layers.{l}.mlp.{p}.weight"] for p in ("gate_proj", "up_proj")])
        np.testing.assert_array_equal(codes, O.quantize_w8a16_rows(w.float().numpy())[0])
        assert eng.linears[(l, 3)][1].shape == (H, I)
        np.testing.assert_array_equal(eng.tensors[(l, 2)],
                                      _bits(t[f"model.layers.{l}.self_attn.q_norm.weight"]))
    np.testing.assert_array_equal(eng.tensors[(0, 5)].reshape(V, H),
                                  _bits(t["model.embed_tokens.weight"]))
    fmt, codes, _, _ = eng.linears[(0, 4)]
    assert fmt == dial_b200.FMT_DENSE
    np.testing.assert_array_equal(codes, _bits(t["lm_head.weight"]))


def test_qwen3_vl_prefix_and_tied_head(tmp_path):
    t = _base(np.random.default_rng(1), "model.language_model.", "dense", head=False)
    path = _write(tmp_path, t, {"text_config": {"tie_word_embeddings": True}})
    eng = _load(path)
    np.testing.assert_array_equal(eng.linears[(0, 4)][1],
                                  _bits(t["model.language_model.embed_tokens.weight"]))
    (tmp_path / "config.json").write_text(json.dumps({"tie_word_embeddings": False}))
    from dial_b200 import DialError
    with pytest.raises(DialError, match="cannot find lm_head.weight"):
        _load(path)


@pytest.mark.parametrize("form", ["fp8_tensor", "fp8_row"])
def test_fp8_scales_expand_to_rows(tmp_path, form):
    import dial_b200

    t = _base(np.random.default_rng(2), "model.", form)
    eng = _load(_write(tmp_path, t))
    fmt, codes, scales, _ = eng.linears[(1, 0)]
    assert fmt == dial_b200.FMT_FP8_ROW and codes.shape == ((QH + 2 * KVH) * D, H)
    parts = [t[f"model.layers.1.self_attn.{p}.weight_scale"].numpy().reshape(-1)
             for p in ("q_proj", "k_proj", "v_proj")]
    rows = [np.full(n, p[0], np.float32) if p.size == 1 else p
            for p, n in zip(parts, (QH * D, KVH * D, KVH * D))]
    np.testing.assert_array_equal(scales, np.concatenate(rows))
    np.testing.assert_array_equal(
        codes[:QH * D], t["model.layers.1.self_attn.q_proj.weight"].view(torch.uint8).numpy())


def test_fp8_block_scales_stack_by_block_rows(tmp_path):
    import dial_b200

    t = _base(np.random.default_rng(3), "model.", "fp8_block")
    eng = _load(_write(tmp_path, t))
    fmt, codes, scales, _ = eng.linears[(0, 2)]
    assert fmt == dial_b200.FMT_FP8_BLOCK128
    assert scales.shape == (2 * I // 128, H // 128)
    np.testing.assert_array_equal(scales[:I // 128],
                                  t["model.layers.0.mlp.gate_proj.weight_scale"].numpy())


@pytest.mark.parametrize("form", ["nvfp4_ct", "nvfp4_mo"])
def test_nvfp4_global_scale_conventions(tmp_path, form):
    import dial_b200

    t = _base(np.random.default_rng(4), "model.", form)
    eng = _load(_write(tmp_path, t))
    fmt, codes, scales, glob = eng.linears[(0, 3)]
    assert fmt == dial_b200.FMT_NVFP4_G16
    assert codes.shape == (H, I // 2) and scales.shape == (H, I // 16)
    # compressed-tensors stores the divisor, ModelOpt the multiplier: both load as 1e-3
    assert glob == pytest.approx(1e-3, rel=1e-6)
    key = "weight_packed" if form == "nvfp4_ct" else "weight"
    np.testing.assert_array_equal(codes, t[f"model.layers.0.mlp.down_proj.{key}"].numpy()
                                  .reshape(H, I // 2))


def test_detection_order_and_errors(tmp_path):
    from dial_b200 import DialError
    from dial_b200.checkpoint import Checkpoint, read_linear

    rng = np.random.default_rng(5)
    packed, sc, gs = O.quantize_nvfp4((rng.standard_normal((128, 64)) * 0.02).astype(np.float32))
    t = {"a.weight_packed": torch.from_numpy(packed),
         "a.weight_scale": torch.from_numpy(sc).view(torch.float8_e4m3fn),
         "a.weight_global_scale": torch.tensor([1.0 / gs]),
         "b.weight": torch.zeros(128, 64, dtype=torch.uint8).view(torch.float8_e4m3fn),
         "b.weight_scale": torch.ones(3),
         "c.weight_packed": torch.from_numpy(packed.copy()),
         "c.weight_scale": torch.from_numpy(sc.copy()).view(torch.float8_e4m3fn),
         "c.weight_global_scale": torch.tensor([0.0])}
    ck = Checkpoint(_write(tmp_path, t))
    q = lambda w: (np.zeros(w.shape, np.int8), np.ones(w.shape[0], np.float32))  # noqa: E731
    # NVFP4 (compressed-tensors) wins although weight_scale is present too
    import dial_b200
    assert read_linear(ck, "a", 64, 128, q).fmt == dial_b200.FMT_NVFP4_G16
    with pytest.raises(DialError, match="contains 3 values"):
        read_linear(ck, "b", 64, 128, q)
    with pytest.raises(DialError, match="one non-zero value"):
        read_linear(ck, "c", 64, 128, q)


def test_mixed_formats_cannot_fuse(tmp_path):
    from dial_b200 import DialError

    rng = np.random.default_rng(6)
    t = _base(rng, "model.", "dense")
    wf = t["model.layers.0.self_attn.k_proj.weight"].float().numpy()
    s = np.float32(np.abs(wf).max() / 448.0)
    t["model.layers.0.self_attn.k_proj.weight"] = torch.from_numpy(
        O.f32_to_e4m3(wf / s)).view(torch.float8_e4m3fn)
    t["model.layers.0.self_attn.k_proj.weight_scale"] = torch.tensor(s)
    with pytest.raises(DialError, match="different formats"):
        _load(_write(tmp_path, t))


def test_stage_engine_loads_only_its_layers(tmp_path):
    t = _base(np.random.default_rng(7), "model.", "dense")
    eng = _load(_write(tmp_path, t), first_layer=1, num_layers=1, has_embed=False, has_head=True)
    assert sorted({k[0] for k in eng.linears if k[1] != 4}) == [1]
    assert (0, 5) not in eng.tensors and (0, 4) in eng.tensors


def test_sharded_directory_and_config(tmp_path):
    from dial_b200 import config_from_checkpoint

    t = _base(np.random.default_rng(8), "model.", "dense")
    keys = sorted(t)
    half = len(keys) // 2
    save_file({k: t[k].contiguous() for k in keys[:half]}, str(tmp_path / "a.safetensors"))
    save_file({k: t[k].contiguous() for k in keys[half:]}, str(tmp_path / "b.safetensors"))
    index = {"weight_map": {k: ("a.safetensors" if i < half else "b.safetensors")
                            for i, k in enumerate(keys)}}
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps(index))
    (tmp_path / "config.json").write_text(json.dumps({
        "model_type": "qwen3_vl", "text_config": {
            "hidden_size": H, "intermediate_size": I, "vocab_size": V, "num_hidden_layers": LAYERS,
            "num_attention_heads": QH, "num_key_value_heads": KVH, "head_dim": D,
            "rms_norm_eps": 1e-6, "rope_theta": 1e6}}))
    cfg = config_from_checkpoint(tmp_path, max_seq_len=256)
    assert (cfg.hidden_size, cfg.num_key_value_heads, cfg.rope_theta, cfg.max_seq_len) == \
        (H, KVH, 1e6, 256)
    eng = _load(tmp_path)
    assert len([k for k in eng.linears if k[1] != 4]) == 4 * LAYERS


def test_reference_loader_known_answers(tmp_path):
    """The reference's own loader tests (qwen3_8/quant.rs:528-662), each as a
    tiny safetensors file read by dial_b200.checkpoint.read_linear and
    dequantised by the oracle: raw e4m3 bit patterns survive (528-544);
    ModelOpt NVFP4 with weight_scale_2 (547-576); FP8 with a per-output f32
    scale, also at the f16 runtime dtype (579-630); compressed-tensors NVFP4
    whose weight_global_scale is a divisor (633-662).  As in those tests, the
    e4m3 fields of 547-662 are stored as f32 values."""
    from dial_b200 import FMT_FP8_ROW, FMT_NVFP4_G16
    from dial_b200.checkpoint import Checkpoint, read_linear

    def no_dense(_):
        raise AssertionError("a quantised layer must not reach the dense path")

    # 528-544: raw e4m3 codes, one scale
    raw = torch.tensor([0x00, 0x38, 0xB8, 0x7E], dtype=torch.uint8).view(torch.float8_e4m3fn)
    _write(tmp_path, {"a.weight": raw.reshape(2, 2), "a.weight_scale": torch.tensor([1.0])},
           name="a.safetensors")
    spec = read_linear(Checkpoint(tmp_path / "a.safetensors"), "a", 2, 2, no_dense)
    assert spec.fmt == FMT_FP8_ROW
    assert spec.codes.reshape(-1).tolist() == [0x00, 0x38, 0xB8, 0x7E]

    # 547-576: ModelOpt NVFP4
    _write(tmp_path, {"b.weight": torch.full((1, 8), 0x92, dtype=torch.uint8),
                      "b.weight_scale": torch.tensor([[2.0]]),
                      "b.weight_scale_2": torch.tensor([4.0])}, name="b.safetensors")
    spec = read_linear(Checkpoint(tmp_path / "b.safetensors"), "b", 16, 1, no_dense)
    assert spec.fmt == FMT_NVFP4_G16 and spec.global_scale == 4.0
    w = O.nvfp4_dense_weight(spec.codes, spec.scales, spec.global_scale, 16, 1)
    assert w.reshape(-1).tolist() == [8.0, -4.0] * 8

    # 579-630: FP8 values [[1,2],[3,4]] with per-output scale [2, 0.5]
    _write(tmp_path, {"c.weight": torch.tensor([[1.0, 2.0], [3.0, 4.0]]),
                      "c.weight_scale": torch.tensor([2.0, 0.5])}, name="c.safetensors")
    spec = read_linear(Checkpoint(tmp_path / "c.safetensors"), "c", 2, 2, no_dense)
    assert spec.fmt == FMT_FP8_ROW
    w = O.fp8_row_dense_weight(spec.codes, spec.scales, 2, 2)
    assert w.reshape(-1).tolist() == [2.0, 4.0, 1.5, 2.0]
    assert O.f16_round(w).reshape(-1).tolist() == [2.0, 4.0, 1.5, 2.0]

    # 633-662: compressed-tensors NVFP4, global scale 4.0 is a divisor
    _write(tmp_path, {"d.weight_packed": torch.full((1, 8), 0x92, dtype=torch.uint8),
                      "d.weight_scale": torch.tensor([[2.0]]),
                      "d.weight_global_scale": torch.tensor([4.0])}, name="d.safetensors")
    spec = read_linear(Checkpoint(tmp_path / "d.safetensors"), "d", 16, 1, no_dense)
    assert spec.global_scale == 0.25
    w = O.nvfp4_dense_weight(spec.codes, spec.scales, spec.global_scale, 16, 1)
    assert w.reshape(-1).tolist() == [0.5, -0.25] * 8


def test_e4m3_fields_must_hold_e4m3_values(tmp_path):
    from dial_b200 import DialError
    from dial_b200.checkpoint import Checkpoint, read_linear

    _write(tmp_path, {"e.weight": torch.tensor([[1.0, 2.0], [3.0, 4.1]]),
                      "e.weight_scale": torch.tensor([1.0])}, name="e.safetensors")
    with pytest.raises(DialError, match="not an e4m3 value"):
        read_linear(Checkpoint(tmp_path / "e.safetensors"), "e", 2, 2, lambda w: None)
