"""Pins the CPU oracle against every known answer the reference's own tests
hold for this path (CPU only).

Sources (lisa301/DIAL-27B):
  dial-core/src/models/qwen3_8/quant.rs:509-662      NVFP4/FP8 dequant known answers
  dial-core/src/models/llama3/cache.rs:349-415       KV cache index semantics
  dial-core/src/models/qwen3_vl/worker_w8a16.rs:483-516   W8A16 vs dense (max_abs < 0.04)
  dial-core/src/models/qwen3_8/cuda_quant.rs:507-552 NVFP4/FP8 vs dense (max_abs < 0.02)
  dial-core/examples/qwen38_quant_smoke.rs:11-95     patterned codes (max_abs < 0.06)
"""

import numpy as np
import pytest

import dial_oracle as O


# -------------------------------------------------- quant.rs known answers
def test_nvfp4_low_nibble_first_and_group_scales():
    # quant.rs:510-519
    packed = np.zeros(16, dtype=np.uint8)
    packed[0] = 0x92
    packed[8] = 0x65
    d = O.decode_nvfp4_values(packed, [2.0, 0.5], 4.0, 32, 1)
    assert d[0, 0] == 8.0
    assert d[0, 1] == -4.0
    assert d[0, 16] == 6.0
    assert d[0, 17] == 8.0


def test_nvfp4_rejects_invalid_shapes():
    # quant.rs:522-525
    with pytest.raises(O.QuantError, match="expected 8"):
        O.decode_nvfp4_values(np.zeros(7, np.uint8), [1.0], 1.0, 16, 1)


def test_e4m3_decode_of_the_raw_codes():
    # the codes of quant.rs:528-544 and their decode (cuda_quant.rs:27-41); the
    # loading half of that test runs through the checkpoint reader in
    # tests/test_checkpoint_cpu.py::test_reference_loader_known_answers
    codes = np.array([0x00, 0x38, 0xB8, 0x7E], dtype=np.uint8)
    assert O.e4m3_to_f32(codes).tolist() == [0.0, 1.0, -1.0, 448.0]


def test_modelopt_nvfp4_linear():
    # quant.rs:547-576: packed 0x92 x8, weight_scale 2.0, weight_scale_2 4.0
    d = O.decode_nvfp4_values(np.full(8, 0x92, np.uint8), [2.0], 4.0, 16, 1)
    assert d.reshape(-1).tolist() == [8.0, -4.0] * 8


def test_fp8_per_output_scale():
    # quant.rs:579-601 (weight codes of [[1,2],[3,4]], scale [2, 0.5]) through
    # the oracle's FP8 row dequant (quant.rs:408-429); the checkpoint reader
    # half is tests/test_checkpoint_cpu.py::test_reference_loader_known_answers
    codes = O.f32_to_e4m3(np.array([[1.0, 2.0], [3.0, 4.0]], np.float32))
    w = O.fp8_row_dense_weight(codes, [2.0, 0.5], 2, 2)
    assert w.reshape(-1).tolist() == [2.0, 4.0, 1.5, 2.0]
    # quant.rs:604-630: the same values survive the f16 runtime dtype exactly
    assert O.f16_round(w).reshape(-1).tolist() == [2.0, 4.0, 1.5, 2.0]


def test_compressed_tensors_reciprocal_global():
    # quant.rs:633-662: weight_global_scale 4.0 is a divisor -> multiplier 0.25
    d = O.decode_nvfp4_values(np.full(8, 0x92, np.uint8), [2.0], 1.0 / 4.0, 16, 1)
    assert d.reshape(-1).tolist() == [0.5, -0.25] * 8


def test_e4m3_decoder_table_edges():
    # cuda_quant.rs:27-41: subnormal m*2^-9, max 448, NaN codes -> 0
    assert O.e4m3_to_f32(np.array([0x01, 0x07, 0x08, 0x7E, 0x7F, 0xFF, 0x80], np.uint8)).tolist() == [
        2.0 ** -9, 7 * 2.0 ** -9, 2.0 ** -6, 448.0, 0.0, 0.0, 0.0]
    # every code equals the IEEE-style decode of e4m3fn except the NaN codes
    import torch

    codes = np.arange(256, dtype=np.uint8)
    ref = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    mine = O.e4m3_to_f32(codes)
    ok = ~np.isnan(ref)
    assert np.array_equal(mine[ok], ref[ok])
    assert np.all(mine[~ok] == 0.0)


def test_e2m1_table():
    assert O.e2m1_to_f32(np.arange(16, dtype=np.uint8)).tolist() == [
        0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, 0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0]


# ------------------------------------------------ cache.rs known answers
def test_process_kv_replaces_on_index_pos_zero():
    # cache.rs:349-373
    c = O.Cache(2, 64)
    k, _ = c.process_kv(0, 1, np.zeros((1, 4, 10, 8), np.float32), np.zeros((1, 4, 10, 8), np.float32))
    assert k.shape[2] == 10
    k, _ = c.process_kv(0, 0, np.zeros((1, 4, 7, 8), np.float32), np.zeros((1, 4, 7, 8), np.float32))
    assert k.shape[2] == 7


def test_decode_cache_preallocated_and_indexed():
    # cache.rs:375-410
    c = O.Cache(1, 8)
    pk = np.arange(16, dtype=np.float32).reshape(1, 1, 2, 8)
    c.process_kv(0, 0, pk, pk + 100)
    for pos in range(2, 5):
        ak, av = c.process_kv_decode_in_place(0, pos, np.full((1, 1, 1, 8), pos, np.float32),
                                              np.full((1, 1, 1, 8), pos + 100, np.float32))
        assert ak.shape == (1, 1, pos + 1, 8) and av.shape == (1, 1, pos + 1, 8)
        assert c.kvs[0][0].shape == (1, 1, 8, 8)
    ak, av = c.process_kv_decode_in_place(0, 5, np.full((1, 1, 1, 8), 5, np.float32),
                                          np.full((1, 1, 1, 8), 105, np.float32))
    assert ak.reshape(-1)[16] == 2.0
    assert ak.reshape(-1)[40] == 5.0
    assert av.reshape(-1)[40] == 105.0


def test_mask_upper_triangular():
    # cache.rs:102-113
    m = O.Cache(1, 8).mask(3)
    assert m.tolist() == [[0, 1, 1], [0, 0, 1], [0, 0, 0]]


def test_process_kv_slides_past_capacity():
    # cache.rs:144-154
    c = O.Cache(1, 4)
    c.process_kv(0, 0, np.zeros((1, 1, 3, 2), np.float32), np.zeros((1, 1, 3, 2), np.float32))
    k, _ = c.process_kv(0, 3, np.ones((1, 1, 2, 2), np.float32), np.ones((1, 1, 2, 2), np.float32))
    assert k.shape[2] == 4 and k[0, 0, -1, 0] == 1.0


# ----------------------------------------- linear known-answer test vectors
def _w8a16_reference_case():
    # worker_w8a16.rs:483-516
    in_dim, out_dim = 64, 37
    i = np.arange(out_dim * in_dim, dtype=np.float32)
    w = (np.sin(i * np.float32(0.037)) * 0.25 + ((i % 11) - 5.0) * 0.002).astype(np.float32)
    w = O.f16_round(w.reshape(out_dim, in_dim))
    return w


@pytest.mark.parametrize("rows", [1, 9])
def test_w8a16_oracle_matches_dense_within_reference_tolerance(rows):
    w = _w8a16_reference_case()
    q, s = O.quantize_w8a16_rows(w)
    x = O.f16_round(np.cos(np.arange(rows * 64, dtype=np.float32) * 0.071) * 0.5).reshape(rows, 64)
    dense = O.dense_linear(x, w, "f16")
    mine = O.w8a16_linear(x, q, s, "f16")
    assert np.max(np.abs(dense - mine)) < 0.04


def test_w8a16_quantization_rules():
    w = np.array([[0.0, 0.0, 0.0], [1.0, -0.5, 0.25], [127.0, 63.5, -63.5]], dtype=np.float32)
    q, s = O.quantize_w8a16_rows(w)
    assert s[0] == 1.0 and q[0].tolist() == [0, 0, 0]
    assert s[1] == np.float32(1.0) / np.float32(127.0)
    assert q[1].tolist() == [127, -64, 32]  # -63.5 rounds away from zero
    assert q[2].tolist() == [127, 64, -64]


def test_quant_linears_match_dense_reference_case():
    # cuda_quant.rs:507-552: codes 0x22 (e2m1 1.0, 1.0) scale 0x38 (1.0) global 0.5 ; fp8 0x38 * 0.5
    in_dim, out_dim = 32, 3
    packed = np.full(out_dim * in_dim // 2, 0x22, np.uint8)
    scales = np.full(out_dim * in_dim // 16, 0x38, np.uint8)
    dense = np.full((out_dim, in_dim), 0.5, np.float32)
    for rows in (1, 7):
        x = O.f16_round(np.sin(np.arange(rows * in_dim, dtype=np.float32) * 0.07)).reshape(rows, in_dim)
        exp = O.dense_linear(x, dense, "f16")
        a = O.nvfp4_linear(x, packed, scales, 0.5, in_dim, out_dim, "f16")
        b = O.fp8_linear(x, np.full(out_dim * in_dim, 0x38, np.uint8), np.full(out_dim, 0.5, np.float32),
                         in_dim, out_dim, "f16")
        assert np.max(np.abs(exp - a)) < 0.02
        assert np.max(np.abs(exp - b)) < 0.02


def smoke_case():
    """examples/qwen38_quant_smoke.rs:11-58 patterned codes."""
    in_dim, out_dim = 32, 3
    pp = [0x92, 0x65, 0x38, 0x07, 0xAB, 0xCD, 0xEF, 0x14]
    sp = [0x38, 0x30, 0x40, 0x28, 0x3C, 0x34]
    packed = np.array([pp[i % len(pp)] for i in range(out_dim * in_dim // 2)], np.uint8)
    scales = np.array([sp[i % len(sp)] for i in range(out_dim * in_dim // 16)], np.uint8)
    fp = [0x38, 0xB8, 0x30, 0x40, 0x01, 0x48, 0x34, 0xBC]
    fp8 = np.array([fp[i % len(fp)] for i in range(out_dim * in_dim)], np.uint8)
    fp8_s = np.array([0.5, 0.25, 0.75], np.float32)
    return in_dim, out_dim, packed, scales, 0.5, fp8, fp8_s


def test_quant_smoke_patterns_within_tolerance():
    in_dim, out_dim, packed, scales, g, fp8, fp8_s = smoke_case()
    nv_dense = O.nvfp4_dense_weight(packed, scales, g, in_dim, out_dim)
    f8_dense = O.fp8_row_dense_weight(fp8, fp8_s, in_dim, out_dim)
    for rows in (1, 7):
        x = O.f16_round(np.sin(np.arange(rows * in_dim, dtype=np.float32) * 0.07)).reshape(rows, in_dim)
        for dw, y in ((nv_dense, O.nvfp4_linear(x, packed, scales, g, in_dim, out_dim, "f16")),
                      (f8_dense, O.fp8_linear(x, fp8, fp8_s, in_dim, out_dim, "f16"))):
            exp = O.dense_linear(x, O.f16_round(dw), "f16")
            assert np.max(np.abs(exp - y)) < 0.06


def test_lcg_fixture_generator():
    # qwen3_8/ggml_tests.rs:36-47 deterministic fixture values
    def random(n, seed, scale):
        out = []
        for i in range(n):
            v = ((i + seed * 97) * 6364136223846793005 + 1442695040888963407) & ((1 << 64) - 1)
            out.append((((v >> 32) % 10000) / 5000.0 - 1.0) * scale)
        return np.array(out, np.float32)

    a = random(4, 0, 1.0)
    b = random(4, 0, 1.0)
    assert np.array_equal(a, b) and np.all(np.abs(a) <= 1.0)


# ----------------------------------------------------- restatement sanity
def test_bf16_round_ties_to_even_matches_torch():
    import torch

    x = np.random.default_rng(0).standard_normal(100000).astype(np.float32) * 10
    x = np.concatenate([x, np.array([1.00390625, 1.01171875, -3.0e38, 1e-40], np.float32)])
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(O.bf16_round(x), ref)


def test_rms_norm_and_rope_shapes():
    x = O.bf16_round(np.random.default_rng(1).standard_normal((3, 128)).astype(np.float32))
    y = O.rms_norm(x, np.ones(128, np.float32), 1e-6)
    assert y.shape == x.shape
    cos, sin = O.rope_tables(128, 16, 1e6)
    assert cos.shape == (16, 64) and cos[0, 0] == 1.0 and sin[0, 5] == 0.0
    r = O.rope(y[None], cos[:3], sin[:3])
    assert np.allclose(r[0, 0], y[0])  # position 0 is the identity


def test_attention_decode_equals_last_row_of_prefill():
    rng = np.random.default_rng(2)
    q = O.bf16_round(rng.standard_normal((4, 5, 128)).astype(np.float32))
    k = O.bf16_round(rng.standard_normal((2, 5, 128)).astype(np.float32))
    v = O.bf16_round(rng.standard_normal((2, 5, 128)).astype(np.float32))
    full = O.attention(q, k, v, causal=True)
    last = O.attention(q[:, -1:], k, v, causal=False)
    assert np.array_equal(full[:, -1:], last)


def test_synth_hash_is_stable():
    idx = np.arange(4, dtype=np.uint64)
    h = O.synth_hash(0, 0, idx)
    # SplitMix64 finalizer of consecutive integers (independent re-derivation)
    def mix(z):
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9 & ((1 << 64) - 1)
        z = (z ^ (z >> 27)) * 0x94D049BB133111EB & ((1 << 64) - 1)
        return z ^ (z >> 31)
    assert [int(v) for v in h] == [mix(i) for i in range(4)]
