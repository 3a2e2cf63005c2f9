"""Linear-op parity on the GPU through the C ABI (CudaW8A16Linear /
CudaQuantLinear counterparts) against the CPU oracle and the reference's own
test cases."""

import numpy as np
import pytest
import torch

import dial_oracle as O

pytestmark = pytest.mark.gpu


def _bf16(a: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev).to(torch.bfloat16)


def _f16(a: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev).to(torch.float16)


def _ulp_bf16(v: np.ndarray) -> np.ndarray:
    a = np.abs(v).astype(np.float32)
    e = np.floor(np.log2(np.maximum(a, 1e-30)))
    return np.exp2(e - 7).astype(np.float32)


def assert_bf16_close(got: np.ndarray, ref: np.ndarray, frac_ulp=0.999):
    """Config-2 tolerance: |d| <= 2^-7 max|ref| + 1e-3 everywhere and within
    one bf16 ulp of the reference for >= 99.9% of the elements."""
    d = np.abs(got.astype(np.float32) - ref.astype(np.float32))
    bound = 2.0 ** -7 * float(np.max(np.abs(ref))) + 1e-3
    assert float(d.max()) <= bound, f"max |d| {d.max()} > {bound}"
    within = np.mean(d <= _ulp_bf16(ref) * 1.0001)
    assert within >= frac_ulp, f"only {within:.5f} within 1 ulp"


# ------------------------------------------------------------- a1 quantize
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_w8a16_quantization_bit_exact(cuda, dtype):
    from dial_b200 import w8a16_quantize

    rng = np.random.default_rng(3)
    w = (rng.standard_normal((300, 520)) * 0.02).astype(np.float32)
    w[7] = 0.0                          # all-zero row -> scale 1.0
    w[9, :4] = [0.5, -0.5, 0.25, 0.0]    # exact halves after scaling
    t = torch.from_numpy(w).to(dtype)
    q, s = w8a16_quantize(t)
    ref_q, ref_s = O.quantize_w8a16_rows(t.float().numpy())
    assert np.array_equal(s, ref_s)
    assert np.array_equal(q, ref_q)


# ------------------------------------------------ reference W8A16 test case
@pytest.mark.parametrize("rows", [1, 9])
def test_w8a16_reference_case_f16(cuda, rows):
    """worker_w8a16.rs:483-516: in 64, out 37, rows {1, 9}, max_abs < 0.04 vs dense."""
    from dial_b200 import CudaW8A16Linear

    in_dim, out_dim = 64, 37
    i = np.arange(out_dim * in_dim, dtype=np.float32)
    w = (np.sin(i * np.float32(0.037)) * 0.25 + ((i % 11) - 5.0) * 0.002).reshape(out_dim, in_dim)
    wt = torch.from_numpy(w.astype(np.float32)).to(torch.float16)
    lin = CudaW8A16Linear.from_linear("test.linear", wt, act=torch.float16)
    x = torch.from_numpy((np.cos(np.arange(rows * in_dim, dtype=np.float32) * 0.071) * 0.5)
                         .reshape(1, rows, in_dim)).to(torch.float16).to(cuda)
    got = lin.forward(x).float().cpu().numpy().reshape(rows, out_dim)
    dense = (x.float() @ wt.to(cuda).float().T).to(torch.float16).float().cpu().numpy().reshape(rows, out_dim)
    assert np.max(np.abs(got - dense)) < 0.04
    q, s = O.quantize_w8a16_rows(wt.float().numpy())
    ref = O.w8a16_linear(x.float().cpu().numpy().reshape(rows, in_dim), q, s, "f16")
    assert np.max(np.abs(got - ref)) <= np.max(np.abs(ref)) * 2 ** -10 + 1e-6
    assert lin.resident_bytes() == out_dim * in_dim + out_dim * 4


# ------------------------------------- config-2 microbench shapes (parity)
SHAPES = [(4096, 4096), (4096, 1024), (4096, 12288), (12288, 4096), (4096, 6144), (4096, 24576)]


@pytest.mark.parametrize("K,N", SHAPES)
@pytest.mark.parametrize("M", [1, 4, 16])
def test_w8a16_config2_shapes(cuda, K, N, M):
    from dial_b200 import CudaW8A16Linear

    idx = SHAPES.index((K, N))
    w = O.bf16_round(np.random.default_rng(10 + idx).standard_normal((N, K)).astype(np.float32) * 0.02)
    x = O.bf16_round(np.random.default_rng(20 + idx).standard_normal((M, K)).astype(np.float32))
    q, s = O.quantize_w8a16_rows(w)
    lin = CudaW8A16Linear.from_quantized(q, s, act=torch.bfloat16)
    got = lin.forward(_bf16(x, cuda)).float().cpu().numpy()
    ref = O.w8a16_linear(x, q, s, "bf16")
    assert_bf16_close(got, ref)


@pytest.mark.parametrize("K,N,M", [(96, 37, 3), (64, 16, 8), (128, 100, 17), (32, 5, 1), (1024, 40, 9)])
def test_w8a16_ragged_shapes(cuda, K, N, M):
    from dial_b200 import CudaW8A16Linear

    rng = np.random.default_rng(K * 7 + N)
    w = O.bf16_round(rng.standard_normal((N, K)).astype(np.float32) * 0.05)
    x = O.bf16_round(rng.standard_normal((M, K)).astype(np.float32))
    q, s = O.quantize_w8a16_rows(w)
    lin = CudaW8A16Linear.from_quantized(q, s, act=torch.bfloat16)
    got = lin.forward(_bf16(x, cuda)).float().cpu().numpy()
    assert_bf16_close(got, O.w8a16_linear(x, q, s, "bf16"), frac_ulp=0.99)


def test_w8a16_large_activations_keep_range(cuda):
    """bf16 activations beyond the f16 range are pre-scaled by a power of two."""
    from dial_b200 import CudaW8A16Linear

    rng = np.random.default_rng(5)
    w = O.bf16_round(rng.standard_normal((64, 256)).astype(np.float32) * 0.02)
    x = O.bf16_round(rng.standard_normal((2, 256)).astype(np.float32) * 3e5)
    q, s = O.quantize_w8a16_rows(w)
    lin = CudaW8A16Linear.from_quantized(q, s, act=torch.bfloat16)
    got = lin.forward(_bf16(x, cuda)).float().cpu().numpy()
    assert np.all(np.isfinite(got))
    assert_bf16_close(got, O.w8a16_linear(x, q, s, "bf16"), frac_ulp=0.99)


def test_w8a16_input_errors(cuda):
    from dial_b200 import CudaW8A16Linear, DialError

    lin = CudaW8A16Linear.from_linear("x", torch.ones(16, 64, dtype=torch.float16), act=torch.float16)
    with pytest.raises(DialError, match="expects F16 activation"):
        lin.forward(torch.ones(1, 64, dtype=torch.bfloat16, device=cuda))
    with pytest.raises(DialError, match="input mismatch: expected last dim 64"):
        lin.forward(torch.ones(1, 63, dtype=torch.float16, device=cuda))


# ------------------------------------------------------- FP8 / NVFP4 cases
def _x_f16(rows, in_dim, dev):
    return _f16(np.sin(np.arange(rows * in_dim, dtype=np.float32) * 0.07).reshape(rows, in_dim), dev)


@pytest.mark.parametrize("rows", [1, 7])
def test_quant_linears_reference_case(cuda, rows):
    """cuda_quant.rs:507-552: NVFP4 0x22/0x38/0.5 and FP8 0x38*0.5 vs dense 0.5, < 0.02."""
    from dial_b200 import CudaQuantLinear

    in_dim, out_dim = 32, 3
    nv = CudaQuantLinear.nvfp4(np.full(out_dim * in_dim // 2, 0x22, np.uint8),
                               np.full(out_dim * in_dim // 16, 0x38, np.uint8), 0.5, in_dim, out_dim)
    f8 = CudaQuantLinear.fp8(np.full(out_dim * in_dim, 0x38, np.uint8), [0.5] * out_dim, in_dim, out_dim)
    x = _x_f16(rows, in_dim, cuda)
    dense = (x.float() @ torch.full((out_dim, in_dim), 0.5, device=cuda).T).half().float()
    for lin in (nv, f8):
        got = lin.forward(x).float()
        assert float((got - dense).abs().max()) < 0.02


@pytest.mark.parametrize("rows", [1, 7])
def test_quant_smoke_patterns(cuda, rows):
    """examples/qwen38_quant_smoke.rs: patterned codes vs dense decode, < 0.06,
    and the oracle's exact linears within one f16 ulp."""
    from dial_b200 import CudaQuantLinear
    from test_oracle_golden import smoke_case

    in_dim, out_dim, packed, scales, g, fp8, fp8_s = smoke_case()
    nv = CudaQuantLinear.nvfp4(packed, scales, g, in_dim, out_dim)
    f8 = CudaQuantLinear.fp8(fp8, fp8_s, in_dim, out_dim)
    x = _x_f16(rows, in_dim, cuda)
    xn = x.float().cpu().numpy()
    for lin, dw, ref in (
            (nv, O.nvfp4_dense_weight(packed, scales, g, in_dim, out_dim),
             O.nvfp4_linear(xn, packed, scales, g, in_dim, out_dim, "f16")),
            (f8, O.fp8_row_dense_weight(fp8, fp8_s, in_dim, out_dim),
             O.fp8_linear(xn, fp8, fp8_s, in_dim, out_dim, "f16"))):
        got = lin.forward(x).float().cpu().numpy()
        dense = O.dense_linear(xn, O.f16_round(dw), "f16")
        assert np.max(np.abs(got - dense)) < 0.06
        assert np.max(np.abs(got - ref)) <= np.max(np.abs(ref)) * 2 ** -10 + 1e-6


def test_fp8_nan_codes_decode_to_zero(cuda):
    from dial_b200 import CudaQuantLinear

    in_dim, out_dim = 64, 16
    codes = np.full(out_dim * in_dim, 0x38, np.uint8)
    codes[::3] = 0x7F
    codes[1::5] = 0xFF
    lin = CudaQuantLinear.fp8(codes, [1.0], in_dim, out_dim)
    x = _x_f16(2, in_dim, cuda)
    got = lin.forward(x).float().cpu().numpy()
    ref = O.fp8_linear(x.float().cpu().numpy(), codes, [1.0], in_dim, out_dim, "f16")
    assert np.all(np.isfinite(got))
    assert np.max(np.abs(got - ref)) <= np.max(np.abs(ref)) * 2 ** -10 + 1e-6


@pytest.mark.parametrize("K,N,M", [(5120, 1024, 1), (5120, 640, 4), (1024, 5120, 3), (384, 200, 9)])
def test_fp8_block128_bf16(cuda, K, N, M):
    from dial_b200 import CudaQuantLinear

    rng = np.random.default_rng(K + N + M)
    w = rng.standard_normal((N, K)).astype(np.float32) * 0.02
    codes, scales = O.quantize_fp8_block128(w)
    x = O.bf16_round(rng.standard_normal((M, K)).astype(np.float32))
    lin = CudaQuantLinear.fp8_block128(codes, scales, K, N)
    got = lin.forward(_bf16(x, cuda)).float().cpu().numpy()
    assert_bf16_close(got, O.fp8_block_linear(x, codes, scales, K, N, "bf16"), frac_ulp=0.99)


@pytest.mark.parametrize("K,N,M", [(5120, 1024, 1), (5120, 640, 4), (256, 48, 9)])
def test_nvfp4_bf16(cuda, K, N, M):
    from dial_b200 import CudaQuantLinear

    rng = np.random.default_rng(K * 3 + N + M)
    w = rng.standard_normal((N, K)).astype(np.float32) * 0.02
    packed, sc, g = O.quantize_nvfp4(w)
    x = O.bf16_round(rng.standard_normal((M, K)).astype(np.float32))
    lin = CudaQuantLinear.nvfp4(packed, sc, g, K, N, act=torch.bfloat16)
    got = lin.forward(_bf16(x, cuda)).float().cpu().numpy()
    assert_bf16_close(got, O.nvfp4_linear(x, packed, sc, g, K, N, "bf16"), frac_ulp=0.99)


@pytest.mark.parametrize("M", [1, 3])
def test_dense_bf16_linear(cuda, M):
    from dial_b200 import DenseLinear

    rng = np.random.default_rng(M)
    w = O.bf16_round(rng.standard_normal((1000, 512)).astype(np.float32) * 0.02)
    x = O.bf16_round(rng.standard_normal((M, 512)).astype(np.float32))
    lin = DenseLinear.from_weight(_bf16(w, "cpu"))
    got = lin.forward(_bf16(x, cuda)).float().cpu().numpy()
    assert_bf16_close(got, O.dense_linear(x, w, "bf16"))
