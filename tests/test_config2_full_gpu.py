"""BASELINE config 2 in full: the W8A16 linear over every Qwen3-8B projection
shape (K x N = 4096x4096, 4096x1024, 4096x12288, 12288x4096 and the fused
4096x6144 / 4096x24576) at the row counts the small-M tests leave out,
M in {32, 128, 2048}, through the C ABI (dial_b200_qlinear_forward) against
the oracle's dequant + matmul (worker_w8a16.rs:146-224 semantics,
y = bf16(s[n] * sum_k q[n,k] x[m,k])), computed by the C++ oracle with f64
accumulation (equal to oracle/dial_oracle.py).

M = 32 runs the split-K tcgen05 GEMM with 128 x 64 tiles (the many-row decode
path), M = 128 the split-K 128 x 128 tiles, M = 2048 the 256 x 256 tiles.
Seeds follow the config: W = 10 + shape index, x = 20 + shape index; W is
N(0, 0.02) in bf16, quantised per row (worker_w8a16.rs:330-341); x is bf16
N(0, 1).  Tolerance (config 2): |d| <= 2^-7 max|y| + 1e-3 and >= 99.9 % of
the elements within one bf16 ulp."""

import numpy as np
import pytest
import torch

import dial_oracle as O
import dial_oracle_fast as F
from test_linear_gpu import SHAPES, _bf16, assert_bf16_close

pytestmark = pytest.mark.gpu

_CACHE = {}


def _weights(idx):
    if idx not in _CACHE:
        K, N = SHAPES[idx]
        rng = np.random.default_rng(10 + idx)
        w = O.bf16_round((rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)))
        _CACHE.clear()
        _CACHE[idx] = F.quantize_w8a16_rows(w)
    return _CACHE[idx]


@pytest.mark.parametrize("M", [32, 128, 2048])  # varies fastest: one weight set per shape
@pytest.mark.parametrize("idx", range(len(SHAPES)))
def test_config2_shape_vs_oracle(cuda, idx, M):
    from dial_b200 import CudaW8A16Linear

    K, N = SHAPES[idx]
    q, s = _weights(idx)
    x = O.bf16_round(np.random.default_rng(20 + idx).standard_normal((M, K), dtype=np.float32))
    lin = CudaW8A16Linear.from_quantized(q, s, act=torch.bfloat16)
    got = lin.forward(_bf16(x, cuda)).float().cpu().numpy()
    del lin
    ref = F.w8a16_linear(x, q, s)
    assert_bf16_close(got, ref)
