"""Prefill W8A16 linear on the tensor cores (tcgen05 GEMM, M >= 16 rows)
against the oracle's dequant + matmul (worker_w8a16.rs:186-224 semantics:
y = act(s[n] * sum_k q[n, k] x[m, k])) and against the decode GEMV path."""

import os

import numpy as np
import pytest
import torch

import dial_oracle as O
from test_linear_gpu import SHAPES, _bf16, _f16, assert_bf16_close

pytestmark = pytest.mark.gpu


@pytest.fixture
def gemv_only():
    """Route every linear through the decode GEMV for the duration of a block."""
    class _Switch:
        def __enter__(self):
            os.environ["DIAL_B200_GEMM_MIN_ROWS"] = "0"

        def __exit__(self, *exc):
            os.environ.pop("DIAL_B200_GEMM_MIN_ROWS", None)
    return _Switch()


def _case(K, N, M, seed):
    rng = np.random.default_rng(seed)
    w = O.bf16_round(rng.standard_normal((N, K)).astype(np.float32) * 0.02)
    x = O.bf16_round(rng.standard_normal((M, K)).astype(np.float32))
    q, s = O.quantize_w8a16_rows(w)
    return x, q, s


@pytest.mark.parametrize("K,N", SHAPES)
@pytest.mark.parametrize("M", [64, 200])
def test_gemm_config2_shapes_vs_oracle(cuda, K, N, M):
    from dial_b200 import CudaW8A16Linear

    x, q, s = _case(K, N, M, 30 + SHAPES.index((K, N)))
    lin = CudaW8A16Linear.from_quantized(q, s, act=torch.bfloat16)
    got = lin.forward(_bf16(x, cuda)).float().cpu().numpy()
    assert_bf16_close(got, O.w8a16_linear(x, q, s, "bf16"))


@pytest.mark.parametrize("M", [128, 2048])
def test_gemm_large_m_vs_torch_fp32(cuda, M):
    """Config-2 M = 2048 on the q/o shape against a torch fp32 dequant+matmul
    (the oracle's f64 loop is too slow at this size)."""
    from dial_b200 import CudaW8A16Linear

    K, N = 4096, 4096
    x, q, s = _case(K, N, M, 7)
    lin = CudaW8A16Linear.from_quantized(q, s, act=torch.bfloat16)
    xt = _bf16(x, cuda)
    got = lin.forward(xt).float()
    wf = torch.from_numpy(q.astype(np.float32)).to(cuda) * torch.from_numpy(s).to(cuda)[:, None]
    ref = (xt.float() @ wf.T).to(torch.bfloat16).float()
    assert_bf16_close(got.cpu().numpy(), ref.cpu().numpy(), frac_ulp=0.995)


def test_gemm_matches_gemv_path(cuda, gemv_only):
    from dial_b200 import CudaW8A16Linear

    x, q, s = _case(4096, 6144, 96, 11)
    lin = CudaW8A16Linear.from_quantized(q, s, act=torch.bfloat16)
    xt = _bf16(x, cuda)
    tc = lin.forward(xt).float().cpu().numpy()
    with gemv_only:
        gv = lin.forward(xt).float().cpu().numpy()
    assert_bf16_close(tc, gv)


def test_gemm_f16_and_large_activations(cuda):
    """f16 activations, and bf16 activations beyond the f16 range (the
    per-row power-of-two pre-scale keeps them finite)."""
    from dial_b200 import CudaW8A16Linear

    x, q, s = _case(1024, 256, 130, 5)
    lin16 = CudaW8A16Linear.from_quantized(q, s, act=torch.float16)
    got = lin16.forward(_f16(x, cuda)).float().cpu().numpy()
    ref = O.w8a16_linear(x, q, s, "f16")
    assert np.max(np.abs(got - ref)) <= 2 ** -9 * np.max(np.abs(ref)) + 1e-3

    big = x * np.float32(4.0e5)
    big[3] *= np.float32(100.0)
    big = O.bf16_round(big)
    lin = CudaW8A16Linear.from_quantized(q, s, act=torch.bfloat16)
    got = lin.forward(_bf16(big, cuda)).float().cpu().numpy()
    assert np.all(np.isfinite(got))
    assert_bf16_close(got, O.w8a16_linear(big, q, s, "bf16"), frac_ulp=0.99)


def test_layer_prefill_on_tensor_cores(cuda, gemv_only):
    """A 100-token prefill takes the GEMM for QKV (RMSNorm fused), o_proj
    (residual), gate/up (SwiGLU) and down (residual): hidden states match the
    oracle and the GEMV path."""
    import dial_b200
    from test_layer_gpu import assert_hidden_close, engine_for, random_layer, small_cfg

    cfg = small_cfg(heads=8, kv_heads=2, hidden=1024, inter=1024, layers=1)
    lw = random_layer(cfg, 3)
    cos, sin = O.rope_tables(cfg.head_dim, cfg.max_seq_len, cfg.rope_theta)
    x = O.bf16_round(np.random.default_rng(8).standard_normal((100, cfg.hidden)).astype(np.float32))
    ref = O.layer_forward(x, lw, cfg, 0, 0, O.Cache(1, cfg.max_seq_len), cos, sin)
    outs = []
    for path in ("tensor", "gemv"):
        eng = engine_for(cfg, dial_b200, max_tokens=128)
        eng.set_layer_w8a16(0, lw)
        xt = torch.from_numpy(x).to(cuda).to(torch.bfloat16)
        if path == "gemv":
            with gemv_only:
                eng.forward(xt, 0, 0)
        else:
            eng.forward(xt, 0, 0)
        torch.cuda.synchronize()
        assert dial_b200.device_status() == 0
        outs.append(xt.float().cpu().numpy())
    assert_hidden_close(outs[0], ref)
    assert_hidden_close(outs[1], ref)
    # the two paths sum in different orders; each is held to the oracle's bound
    assert_hidden_close(outs[0], outs[1])


@pytest.mark.parametrize("K,N,M", [(5120, 1024, 64), (1024, 384, 200), (4096, 6144, 96)])
def test_gemm_fp8_block128_vs_oracle(cuda, K, N, M):
    """FP8 e4m3 with 128x128 block scales (the 27B-class format) on the tensor
    cores: the block scale is folded into the f16 operand (relative error
    <= 2^-11 per weight), so the bound is max |d| <= 2^-7 max|y| + 1e-3 and
    98% of outputs within 1 bf16 ulp (measured 98.3% at K=5120)."""
    from dial_b200 import CudaQuantLinear

    rng = np.random.default_rng(K + N + M)
    w = rng.standard_normal((N, K)).astype(np.float32) * 0.02
    codes, scales = O.quantize_fp8_block128(w)
    x = O.bf16_round(rng.standard_normal((M, K)).astype(np.float32))
    lin = CudaQuantLinear.fp8_block128(codes, scales, K, N)
    got = lin.forward(_bf16(x, cuda)).float().cpu().numpy()
    assert_bf16_close(got, O.fp8_block_linear(x, codes, scales, K, N, "bf16"), frac_ulp=0.98)


@pytest.mark.parametrize("M", [64, 150])
def test_gemm_fp8_row_vs_oracle(cuda, M):
    """FP8 e4m3 with per-row scales (cuda_quant.rs:58-65), f16 activations as
    the reference's FP8 path: exact f16 operands, row scale in the epilogue."""
    from dial_b200 import CudaQuantLinear

    K, N = 1024, 512
    rng = np.random.default_rng(M)
    w = rng.standard_normal((N, K)).astype(np.float32) * 0.02
    row_scale = (np.abs(w).max(axis=1) / 448.0).astype(np.float32)
    codes = O.f32_to_e4m3(w / row_scale[:, None])
    x = O.f16_round(rng.standard_normal((M, K)).astype(np.float32))
    lin = CudaQuantLinear.fp8(codes, row_scale, K, N)
    got = lin.forward(_f16(x, cuda)).float().cpu().numpy()
    ref = O.fp8_linear(x, codes, row_scale, K, N, "f16")
    assert np.max(np.abs(got - ref)) <= 2 ** -9 * np.max(np.abs(ref)) + 1e-3


@pytest.mark.parametrize("K,N,M", [(1024, 512, 64), (4096, 1024, 200), (5120, 256, 130)])
def test_gemm_nvfp4_vs_oracle(cuda, K, N, M):
    """NVFP4 (e2m1 codes, e4m3 scale per 16 inputs, f32 global scale;
    cuda_quant.rs:67-100) on the tensor cores: e2m1 x e4m3 is exact in f16,
    the global scale is applied in the f32 epilogue, so the bound is the
    W8A16 one (f32 accumulation order only)."""
    from dial_b200 import CudaQuantLinear

    rng = np.random.default_rng(K + 3 * N + M)
    w = rng.standard_normal((N, K)).astype(np.float32) * 0.02
    packed, sc, gs = O.quantize_nvfp4(w)
    x = O.bf16_round(rng.standard_normal((M, K)).astype(np.float32))
    lin = CudaQuantLinear.nvfp4(packed, sc, gs, K, N, act=torch.bfloat16)
    got = lin.forward(_bf16(x, cuda)).float().cpu().numpy()
    assert_bf16_close(got, O.nvfp4_linear(x, packed, sc, gs, K, N, "bf16"))


def test_gemm_nvfp4_matches_gemv(cuda, gemv_only):
    from dial_b200 import CudaQuantLinear

    rng = np.random.default_rng(4)
    K, N, M = 2048, 768, 96
    w = rng.standard_normal((N, K)).astype(np.float32) * 0.05
    packed, sc, gs = O.quantize_nvfp4(w)
    lin = CudaQuantLinear.nvfp4(packed, sc, gs, K, N, act=torch.bfloat16)
    xt = _bf16(O.bf16_round(rng.standard_normal((M, K)).astype(np.float32)), cuda)
    tc = lin.forward(xt).float().cpu().numpy()
    with gemv_only:
        gv = lin.forward(xt).float().cpu().numpy()
    assert_bf16_close(tc, gv)
