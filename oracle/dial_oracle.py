"""CPU restatement of DIAL's decoder-layer path -- TEST INFRASTRUCTURE ONLY.

This module is the parity oracle.  Only ``tests/``, ``__graft_entry__.smoke()``
and the CPU-baseline leg of ``bench.py`` may import it; the product path
(``dial-27b_b200``) never does and has no CPU fallback.

Everything here restates the reference's semantics in NumPy, one function per
reference item, citing the reference file and lines it follows (paths are
relative to the reference project root, lisa301/DIAL-27B):

* W8A16 row quantization .......... dial-core/src/models/qwen3_vl/worker_w8a16.rs:330-341
* W8A16 linear (decode/prefill) ... dial-core/src/models/qwen3_vl/worker_w8a16.rs:146-224
* e2m1 / e4m3 decoders ............ dial-core/src/models/qwen3_8/cuda_quant.rs:11-41
* NVFP4 host dequant .............. dial-core/src/models/qwen3_8/quant.rs:142-190
* NVFP4 / FP8 linears ............. dial-core/src/models/qwen3_8/cuda_quant.rs:43-206
* FP8 per-row scale load .......... dial-core/src/models/qwen3_8/quant.rs:316-345
* RoPE tables ..................... dial-core/src/models/llama3/cache.rs:37-67
* KV cache semantics .............. dial-core/src/models/llama3/cache.rs:102-237
* q/k norm, RoPE, grouped attention dial-core/src/models/qwen3_vl/text.rs:1143-1153,1258-1358,1478-1596
* SwiGLU MLP ...................... dial-core/src/models/qwen3_vl/text.rs:816-820
* pre-norm residual block ......... dial-core/src/models/qwen3_vl/text.rs:1636-1688
* head + greedy argmax ............ dial-core/src/models/qwen3_vl/qwen3_vl.rs:138-143,2459-2498
* Gated-DeltaNet mixer ............ dial-core/src/models/qwen3_8/text.rs:233-481
* Qwen3.8 gated full attention .... dial-core/src/models/qwen3_8/text.rs:14-39,82-226

Ops whose arithmetic lives in the third-party ``candle`` 0.11.0 crates
(RMSNorm, RoPE, softmax, SiLU, matmul) are NOT pinned by any reference test.
The rounding points chosen here (and mirrored by the CUDA kernels) are:

* every op output is rounded to the activation dtype (bf16 or f16);
* RMSNorm: ``m = act(sqrt(sum(x^2)/n + eps))``, ``y = act(act(x / m) * w)``
  with the sum in f32 (candle's CPU ``rms_norm`` form);
* RoPE: ``act(act(x1*c) - act(x2*s))`` / ``act(act(x1*s) + act(x2*c))``
  (element ops in the activation type, candle CPU form);
* SiLU: ``act(v / act(1 + act(exp(-v))))``, then ``act(silu * up)``;
* attention: scores ``act(act(q.k) * act(1/sqrt(d)))``, softmax in f32,
  probabilities rounded to ``act``, ``act(sum p*v)`` with f32 accumulation;
* matmuls accumulate in f64 here (the GPU accumulates in f32 in another
  order); this is the reference's "f32 accumulate" up to summation order.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from functools import lru_cache

import numpy as np

# ---------------------------------------------------------------------------
# dtype helpers
# ---------------------------------------------------------------------------


def bf16_round(x) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even); returns f32."""
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    b = x.view(np.uint32).astype(np.uint64)
    bias = ((b >> np.uint64(16)) & np.uint64(1)) + np.uint64(0x7FFF)
    r = ((b + bias) & np.uint64(0xFFFF0000)).astype(np.uint32)
    out = r.view(np.float32).copy()
    nan = np.isnan(x)
    if nan.any():
        out[nan] = np.float32("nan")
    return out.reshape(x.shape)


def f16_round(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def act_round(x, act: str) -> np.ndarray:
    if act == "bf16":
        return bf16_round(x)
    if act == "f16":
        return f16_round(x)
    if act == "f32":
        return np.asarray(x, dtype=np.float32)
    raise ValueError(f"unknown activation dtype {act!r}")


def bf16_bits(x) -> np.ndarray:
    """float32 values (already bf16-representable) -> uint16 bit patterns."""
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(bits) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint32) << 16).view(np.float32)


def _round_half_away(x: np.ndarray) -> np.ndarray:
    """Rust ``f32::round``: half away from zero (exact via f64)."""
    a = np.floor(np.abs(x.astype(np.float64)) + 0.5)
    return np.copysign(a, x).astype(np.float32)


# ---------------------------------------------------------------------------
# a1: W8A16 row-wise symmetric int8 quantization
# ---------------------------------------------------------------------------


def quantize_w8a16_rows(w) -> tuple[np.ndarray, np.ndarray]:
    """Row-wise symmetric int8 (worker_w8a16.rs:330-341).

    ``scale = max|w_row| / 127`` (1.0 for an all-zero row), ``inv = 1/scale``
    in f32, ``q = clamp(round(w * inv), -127, 127)`` with Rust's
    half-away-from-zero ``round``.
    """
    w = np.asarray(w, dtype=np.float32)
    if w.ndim != 2:
        raise ValueError("expected a 2-D [out, in] weight")
    max_abs = np.max(np.abs(w), axis=1).astype(np.float32)
    scale = np.where(max_abs > 0, max_abs / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    inv = (np.float32(1.0) / scale).astype(np.float32)
    v = (w * inv[:, None]).astype(np.float32)
    q = np.clip(_round_half_away(v), -127, 127).astype(np.int8)
    return q, scale


# ---------------------------------------------------------------------------
# a2/a3: W8A16 linear
# ---------------------------------------------------------------------------


def w8a16_linear(x, q, scale, act: str = "bf16") -> np.ndarray:
    """``y[r,n] = act(scale[n] * sum_k q[n,k] * x[r,k])`` (worker_w8a16.rs:146-184,186-224).

    The sum is formed before the scale is applied, as in both reference
    kernels; ``x`` holds activation-dtype values.
    """
    x = np.asarray(x, dtype=np.float32)
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1]).astype(np.float64)
    acc = (x2 @ np.asarray(q, dtype=np.float64).T).astype(np.float32)
    y = act_round(acc * np.asarray(scale, dtype=np.float32)[None, :], act)
    return y.reshape(*lead, q.shape[0])


def dense_linear(x, w, act: str = "bf16") -> np.ndarray:
    """candle ``Linear`` without bias: ``act(x @ w.T)`` with wide accumulation."""
    x = np.asarray(x, dtype=np.float32)
    lead = x.shape[:-1]
    acc = (x.reshape(-1, x.shape[-1]).astype(np.float64) @ np.asarray(w, dtype=np.float64).T)
    return act_round(acc.astype(np.float32), act).reshape(*lead, w.shape[0])


# ---------------------------------------------------------------------------
# a5/a6: FP8 (e4m3) and NVFP4 (e2m1 + e4m3 group scale) decoders and linears
# ---------------------------------------------------------------------------

E2M1_VALUES = np.array(
    [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, 0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0],
    dtype=np.float32,
)  # quant.rs:16-18 / cuda_quant.rs:11-25


def e2m1_to_f32(code) -> np.ndarray:
    return E2M1_VALUES[np.asarray(code, dtype=np.uint8) & 0xF]


def e4m3_to_f32(code) -> np.ndarray:
    """Software e4m3 decode (cuda_quant.rs:27-41): subnormals ``m*2^-9``,
    the NaN codes 0x7F/0xFF decode to 0."""
    c = np.asarray(code, dtype=np.uint8).astype(np.uint32)
    sign = c >> 7
    exp = (c >> 3) & 15
    man = c & 7
    sub = man.astype(np.float32) * np.float32(0.001953125)
    norm = np.ldexp(np.float32(1.0) + man.astype(np.float32) * np.float32(0.125),
                    exp.astype(np.int32) - 7).astype(np.float32)
    v = np.where(exp == 0, sub, norm)
    v = np.where((exp == 15) & (man == 7), np.float32(0.0), v).astype(np.float32)
    return np.where(sign == 1, -v, v).astype(np.float32)


NVFP4_GROUP_SIZE = 16


class QuantError(ValueError):
    """Shape/format errors raised with the reference's wording."""


def decode_nvfp4_values(packed, scales, global_scale, input_size: int, output_size: int) -> np.ndarray:
    """Host NVFP4 dequant (quant.rs:142-190): low nibble holds the even column."""
    if input_size % NVFP4_GROUP_SIZE != 0:
        raise QuantError(
            f"NVFP4 input dimension {input_size} is not divisible by group size {NVFP4_GROUP_SIZE}")
    packed = np.asarray(packed, dtype=np.uint8).reshape(-1)
    expected_packed = output_size * input_size // 2
    if packed.size != expected_packed:
        raise QuantError(f"NVFP4 packed weight has {packed.size} bytes, expected {expected_packed}")
    groups = input_size // NVFP4_GROUP_SIZE
    scales = np.asarray(scales, dtype=np.float32).reshape(-1)
    if scales.size != output_size * groups:
        raise QuantError(
            f"NVFP4 weight scale has {scales.size} values, expected {output_size * groups}")
    p = packed.reshape(output_size, input_size // 2)
    codes = np.empty((output_size, input_size), dtype=np.uint8)
    codes[:, 0::2] = p & 0x0F
    codes[:, 1::2] = p >> 4
    s = np.repeat(scales.reshape(output_size, groups), NVFP4_GROUP_SIZE, axis=1)
    return (E2M1_VALUES[codes] * s * np.float32(global_scale)).astype(np.float32)


def nvfp4_dense_weight(packed, scale_codes, global_scale, in_dim: int, out_dim: int) -> np.ndarray:
    """Per-element weight of the NVFP4 kernel (cuda_quant.rs:43-56), scale as e4m3 codes."""
    return decode_nvfp4_values(packed, e4m3_to_f32(scale_codes), global_scale, in_dim, out_dim)


def nvfp4_linear(x, packed, scale_codes, global_scale, in_dim, out_dim, act="f16") -> np.ndarray:
    """NVFP4 linear (cuda_quant.rs:67-100,135-170): ``act(sum_k x*w)``."""
    w = nvfp4_dense_weight(packed, scale_codes, global_scale, in_dim, out_dim)
    x = np.asarray(x, dtype=np.float32)
    acc = x.reshape(-1, in_dim).astype(np.float64) @ w.astype(np.float64).T
    return act_round(acc.astype(np.float32), act).reshape(*x.shape[:-1], out_dim)


def fp8_row_dense_weight(codes, row_scales, in_dim: int, out_dim: int) -> np.ndarray:
    """FP8 weight with one f32 scale per output row (cuda_quant.rs:58-65; quant.rs:408-429)."""
    w = e4m3_to_f32(np.asarray(codes, dtype=np.uint8).reshape(out_dim, in_dim))
    s = np.asarray(row_scales, dtype=np.float32).reshape(-1)
    if s.size == 1:
        s = np.full(out_dim, s[0], dtype=np.float32)
    if s.size != out_dim:
        raise QuantError(f"FP8 weight_scale contains {s.size} values, expected 1 or {out_dim}")
    return (w * s[:, None]).astype(np.float32)


def fp8_block_dense_weight(codes, block_scales, in_dim: int, out_dim: int, block: int = 128) -> np.ndarray:
    """FP8 e4m3 with one f32 scale per ``block x block`` tile (the 27B-class format)."""
    w = e4m3_to_f32(np.asarray(codes, dtype=np.uint8).reshape(out_dim, in_dim))
    nb_r, nb_c = -(-out_dim // block), -(-in_dim // block)
    s = np.asarray(block_scales, dtype=np.float32).reshape(nb_r, nb_c)
    s_full = np.repeat(np.repeat(s, block, axis=0), block, axis=1)[:out_dim, :in_dim]
    return (w * s_full).astype(np.float32)


def fp8_linear(x, codes, row_scales, in_dim, out_dim, act="f16") -> np.ndarray:
    """FP8 per-row linear (cuda_quant.rs:102-133,172-206): scale applied per element."""
    w = fp8_row_dense_weight(codes, row_scales, in_dim, out_dim)
    x = np.asarray(x, dtype=np.float32)
    acc = x.reshape(-1, in_dim).astype(np.float64) @ w.astype(np.float64).T
    return act_round(acc.astype(np.float32), act).reshape(*x.shape[:-1], out_dim)


def fp8_block_linear(x, codes, block_scales, in_dim, out_dim, act="bf16") -> np.ndarray:
    w = fp8_block_dense_weight(codes, block_scales, in_dim, out_dim)
    x = np.asarray(x, dtype=np.float32)
    acc = x.reshape(-1, in_dim).astype(np.float64) @ w.astype(np.float64).T
    return act_round(acc.astype(np.float32), act).reshape(*x.shape[:-1], out_dim)


# e4m3 encoder (round to nearest even, saturating) used to build FP8/NVFP4
# test weights from dense values; it mirrors no reference function (the
# reference loads pre-quantized checkpoints) but produces valid codes.
_E4M3_TABLE = e4m3_to_f32(np.arange(256, dtype=np.uint8))


def f32_to_e4m3(v) -> np.ndarray:
    v = np.asarray(v, dtype=np.float32)
    pos = _E4M3_TABLE[:127]  # codes 0..126 (0x7F is NaN)
    mag = np.minimum(np.abs(v), np.float32(448.0))
    idx = np.searchsorted(pos, mag)  # first code >= mag
    idx = np.clip(idx, 1, 126)
    lo, hi = pos[idx - 1], pos[idx]
    pick_hi = (mag - lo > hi - mag) | ((mag - lo == hi - mag) & ((idx & 1) == 0))
    code = np.where(pick_hi, idx, idx - 1).astype(np.uint8)
    code = np.where(mag == 0, 0, code).astype(np.uint8)
    return np.where((v < 0) & (code != 0), code | 0x80, code).astype(np.uint8)


def f32_to_e2m1(v) -> np.ndarray:
    vals = E2M1_VALUES[:8]
    v = np.asarray(v, dtype=np.float32)
    mag = np.minimum(np.abs(v), np.float32(6.0))
    d = np.abs(mag[..., None] - vals)
    code = np.argmin(d, axis=-1).astype(np.uint8)
    return np.where((v < 0) & (code != 0), code | 0x8, code).astype(np.uint8)


def quantize_fp8_block128(w, block: int = 128) -> tuple[np.ndarray, np.ndarray]:
    """Dense -> FP8 e4m3 codes + f32 per-block scale ``blockmax/448`` (RN, saturating)."""
    w = np.asarray(w, dtype=np.float32)
    n, k = w.shape
    nb_r, nb_c = -(-n // block), -(-k // block)
    scales = np.ones((nb_r, nb_c), dtype=np.float32)
    codes = np.zeros((n, k), dtype=np.uint8)
    for i in range(nb_r):
        for j in range(nb_c):
            blk = w[i * block:(i + 1) * block, j * block:(j + 1) * block]
            amax = np.float32(np.max(np.abs(blk))) if blk.size else np.float32(0)
            s = np.float32(amax / np.float32(448.0)) if amax > 0 else np.float32(1.0)
            scales[i, j] = s
            codes[i * block:(i + 1) * block, j * block:(j + 1) * block] = f32_to_e4m3(blk / s)
    return codes, scales


def quantize_nvfp4(w, global_scale: float | None = None) -> tuple[np.ndarray, np.ndarray, float]:
    """Dense -> NVFP4: e2m1 codes in 16-element groups, e4m3 group scale ``groupmax/6``."""
    w = np.asarray(w, dtype=np.float32)
    n, k = w.shape
    if k % 16:
        raise QuantError("NVFP4 needs in_dim % 16 == 0")
    g = w.reshape(n, k // 16, 16)
    gmax = np.max(np.abs(g), axis=2)
    if global_scale is None:
        amax = float(np.max(gmax)) if gmax.size else 0.0
        global_scale = (amax / 6.0 / 448.0) if amax > 0 else 1.0
    gs = np.float32(global_scale)
    sc = f32_to_e4m3(gmax / np.float32(6.0) / gs)
    sdec = e4m3_to_f32(sc) * gs
    sdec = np.where(sdec == 0, np.float32(1.0), sdec)
    codes = f32_to_e2m1(g / sdec[..., None]).reshape(n, k)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    return packed.reshape(-1), sc.reshape(-1), float(gs)


# ---------------------------------------------------------------------------
# a8/a9: RMSNorm
# ---------------------------------------------------------------------------


def rms_norm(x, w, eps: float, act: str = "bf16") -> np.ndarray:
    """candle ``rms_norm`` over the last dim (text.rs:1466,1620-1626).

    ``sum2`` in f32, ``m = act(sqrt(sum2/n + eps))``, ``y = act(act(x/m) * w)``.
    """
    x = np.asarray(x, dtype=np.float32)
    n = x.shape[-1]
    sum2 = np.sum(x.astype(np.float64) ** 2, axis=-1, keepdims=True).astype(np.float32)
    m = act_round(np.sqrt(sum2 / np.float32(n) + np.float32(eps)).astype(np.float32), act)
    return act_round(act_round(x / m, act) * np.asarray(w, dtype=np.float32), act)


# ---------------------------------------------------------------------------
# a10: RoPE tables and rotation
# ---------------------------------------------------------------------------


def rope_tables(head_dim: int, max_seq_len: int, theta: float, act: str = "bf16"):
    """cos/sin tables (cache.rs:37-67), f32 then rounded to the model dtype.

    ``inv_freq[i] = 1 / theta^(2i/d)`` in f32, ``angle = pos * inv_freq`` in
    f32, cos/sin evaluated on that f32 angle.
    """
    i = np.arange(0, head_dim, 2, dtype=np.float32)
    inv = (np.float32(1.0) / np.power(np.float32(theta), i / np.float32(head_dim))).astype(np.float32)
    pos = np.arange(max_seq_len, dtype=np.float32)[:, None]
    ang = (pos * inv[None, :]).astype(np.float32)
    cos = np.cos(ang.astype(np.float64)).astype(np.float32)
    sin = np.sin(ang.astype(np.float64)).astype(np.float32)
    return act_round(cos, act), act_round(sin, act)


def rope(x, cos, sin, act: str = "bf16") -> np.ndarray:
    """Non-interleaved half-split rotation (text.rs:1143-1153).

    x: [..., T, D]; cos/sin: [T, D/2].
    """
    x = np.asarray(x, dtype=np.float32)
    d = x.shape[-1]
    x1, x2 = x[..., : d // 2], x[..., d // 2:]
    r = lambda v: act_round(v, act)  # noqa: E731
    o1 = r(r(x1 * cos) - r(x2 * sin))
    o2 = r(r(x1 * sin) + r(x2 * cos))
    return np.concatenate([o1, o2], axis=-1)


# ---------------------------------------------------------------------------
# a11: KV cache (llama3::Cache semantics)
# ---------------------------------------------------------------------------


class Cache:
    """Per-connection KV cache (cache.rs:9-265): replace at ``index_pos==0``,
    append + sliding truncation otherwise, preallocated decode storage."""

    def __init__(self, num_layers: int, max_seq_len: int):
        self.max_seq_len = max_seq_len
        self.kvs: list = [None] * num_layers
        self.masks: dict = {}

    def mask(self, seq_len: int) -> np.ndarray:
        """u8 upper-triangular mask, 1 where ``j > i`` (cache.rs:102-113)."""
        if seq_len not in self.masks:
            i = np.arange(seq_len)[:, None]
            j = np.arange(seq_len)[None, :]
            self.masks[seq_len] = (j > i).astype(np.uint8)
        return self.masks[seq_len]

    def process_kv(self, block_idx: int, index_pos: int, k, v):
        """cache.rs:117-160. k, v: [b, kv_heads, seq, d]."""
        if index_pos == 0:
            self.kvs[block_idx] = (k.copy(), v.copy())
            return k, v
        if self.kvs[block_idx] is not None:
            ck, cv = self.kvs[block_idx]
            k = np.concatenate([ck, k], axis=2)
            v = np.concatenate([cv, v], axis=2)
            if k.shape[2] > self.max_seq_len:
                k = k[:, :, k.shape[2] - self.max_seq_len:]
            if v.shape[2] > self.max_seq_len:
                v = v[:, :, v.shape[2] - self.max_seq_len:]
        self.kvs[block_idx] = (k, v)
        return k, v

    def process_kv_decode_in_place(self, block_idx: int, index_pos: int, k, v):
        """cache.rs:169-237: single-token decode into preallocated storage."""
        if index_pos == 0 or index_pos >= self.max_seq_len or k.ndim != 4 or k.shape[2] != 1:
            return self.process_kv(block_idx, index_pos, k, v)
        b, kvh, _, d = k.shape
        dst = min(index_pos, self.max_seq_len - 1)
        active = min(index_pos + 1, self.max_seq_len)
        cur = self.kvs[block_idx]
        if cur is None or cur[0].shape != (b, kvh, self.max_seq_len, d):
            ck = np.zeros((b, kvh, self.max_seq_len, d), dtype=k.dtype)
            cv = np.zeros_like(ck)
            if cur is not None:
                old_len = min(cur[0].shape[2], dst)
                if old_len > 0:
                    ck[:, :, :old_len] = cur[0][:, :, :old_len]
                    cv[:, :, :old_len] = cur[1][:, :, :old_len]
            self.kvs[block_idx] = (ck, cv)
        ck, cv = self.kvs[block_idx]
        ck[:, :, dst] = k[:, :, 0]
        cv[:, :, dst] = v[:, :, 0]
        start = max(index_pos + 1 - self.max_seq_len, 0)
        return ck[:, :, start:start + active], cv[:, :, start:start + active]

    def clear(self):
        self.masks.clear()
        self.kvs = [None] * len(self.kvs)


# ---------------------------------------------------------------------------
# a12/a13: grouped GQA attention
# ---------------------------------------------------------------------------


def _softmax_rows(s: np.ndarray, act: str) -> np.ndarray:
    s32 = s.astype(np.float32)
    m = np.max(s32, axis=-1, keepdims=True)
    e = np.exp((s32 - m).astype(np.float64)).astype(np.float32)
    return act_round(e / np.sum(e.astype(np.float64), axis=-1, keepdims=True).astype(np.float32), act)


def attention(q, k, v, causal: bool, act: str = "bf16", round_probs: bool = True) -> np.ndarray:
    """Grouped attention (text.rs:1258-1327): q [qh, S, d], k/v [kvh, L, d].

    Query head ``h`` reads kv head ``h // (qh/kvh)``.  With ``causal`` the
    last ``S`` keys align with the queries (prefill: S == L).
    ``round_probs=False`` keeps the softmax probabilities in f32 (the GPU's
    online-softmax semantics) instead of rounding them to ``act``.
    """
    qh, S, d = q.shape
    kvh, L, _ = k.shape
    rep = qh // kvh
    scale = act_round(np.float32(1.0 / math.sqrt(d)), act)
    out = np.empty((qh, S, d), dtype=np.float32)
    for h in range(qh):
        kh = k[h // rep].astype(np.float64)
        vh = v[h // rep]
        s = act_round((q[h].astype(np.float64) @ kh.T).astype(np.float32), act)
        s = act_round(s * scale, act)
        if causal and S > 1:
            qpos = np.arange(L - S, L)[:, None]
            kpos = np.arange(L)[None, :]
            s = np.where(kpos > qpos, np.float32(-np.inf), s)
        p = _softmax_rows(s, act if round_probs else "f32")
        out[h] = act_round((p.astype(np.float64) @ vh.astype(np.float64)).astype(np.float32), act)
    return out


# ---------------------------------------------------------------------------
# a14-a17: layer and model
# ---------------------------------------------------------------------------


@dataclass
class ModelConfig:
    hidden: int = 4096
    inter: int = 12288
    vocab: int = 151936
    layers: int = 36
    heads: int = 32
    kv_heads: int = 8
    eps: float = 1e-6
    rope_theta: float = 1e6
    max_seq_len: int = 4096

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads


@dataclass
class LayerWeights:
    """One decoder layer; linear weights are W8A16 (q int8 [N,K], scale f32 [N])
    with QKV and gate/up fused as in text.rs:1428-1432 and text.rs:634-637."""
    qkv_q: np.ndarray
    qkv_s: np.ndarray
    o_q: np.ndarray
    o_s: np.ndarray
    gate_up_q: np.ndarray
    gate_up_s: np.ndarray
    down_q: np.ndarray
    down_s: np.ndarray
    input_norm: np.ndarray
    post_norm: np.ndarray
    q_norm: np.ndarray
    k_norm: np.ndarray


def silu_mul(gate_up, inter: int, act: str = "bf16") -> np.ndarray:
    """``silu(gate) * up`` over the fused gate_up output (text.rs:816-820)."""
    g = gate_up[..., :inter]
    u = gate_up[..., inter:]
    r = lambda t: act_round(t, act)  # noqa: E731
    e = r(np.exp((-g).astype(np.float64)).astype(np.float32))
    s = r(g / r(np.float32(1.0) + e))
    return r(s * u)


def layer_forward(x, lw: LayerWeights, cfg: ModelConfig, index_pos: int, block_idx: int,
                  cache: Cache, cos, sin, act: str = "bf16", round_probs: bool = True) -> np.ndarray:
    """``Transformer::forward`` (text.rs:1636-1688) for batch 1, x [S, H]."""
    S, H = x.shape
    d, qh, kvh = cfg.head_dim, cfg.heads, cfg.kv_heads
    h = rms_norm(x, lw.input_norm, cfg.eps, act)
    qkv = w8a16_linear(h, lw.qkv_q, lw.qkv_s, act)
    q = qkv[:, : qh * d].reshape(S, qh, d).transpose(1, 0, 2)
    k = qkv[:, qh * d: (qh + kvh) * d].reshape(S, kvh, d).transpose(1, 0, 2)
    v = qkv[:, (qh + kvh) * d:].reshape(S, kvh, d).transpose(1, 0, 2)
    q = rms_norm(q, lw.q_norm, cfg.eps, act)
    k = rms_norm(k, lw.k_norm, cfg.eps, act)
    c, s_ = cos[index_pos:index_pos + S], sin[index_pos:index_pos + S]
    q = rope(q, c, s_, act)
    k = rope(k, c, s_, act)
    if S == 1 and index_pos > 0:
        kc, vc = cache.process_kv_decode_in_place(block_idx, index_pos, k[None], v[None])
    else:
        kc, vc = cache.process_kv(block_idx, index_pos, k[None], v[None])
    y = attention(q, kc[0], vc[0], causal=S > 1, act=act, round_probs=round_probs)
    y = y.transpose(1, 0, 2).reshape(S, qh * d)
    x = act_round(w8a16_linear(y, lw.o_q, lw.o_s, act) + x, act)
    h = rms_norm(x, lw.post_norm, cfg.eps, act)
    gu = w8a16_linear(h, lw.gate_up_q, lw.gate_up_s, act)
    m = silu_mul(gu, cfg.inter, act)
    return act_round(w8a16_linear(m, lw.down_q, lw.down_s, act) + x, act)


def argmax_first(v) -> int:
    """Greedy argmax; among equal maxima the lowest index wins."""
    v = np.asarray(v, dtype=np.float32)
    return int(np.argmax(v))


@dataclass
class Model:
    """Whole text stack: embedding, layers, ln_f, dense lm_head."""
    cfg: ModelConfig
    embed: np.ndarray            # [vocab, hidden] activation values
    layers: list                 # LayerWeights
    final_norm: np.ndarray
    lm_head: np.ndarray          # [vocab, hidden] activation values
    act: str = "bf16"
    cos: np.ndarray = field(default=None)
    sin: np.ndarray = field(default=None)

    def __post_init__(self):
        if self.cos is None:
            self.cos, self.sin = rope_tables(self.cfg.head_dim, self.cfg.max_seq_len,
                                             self.cfg.rope_theta, self.act)


def model_hidden(model: Model, tokens, index_pos: int, cache: Cache) -> np.ndarray:
    """Embedding (qwen3_vl.rs:3302) then every layer (forward_blocks_from)."""
    x = model.embed[np.asarray(tokens, dtype=np.int64)]
    for l, lw in enumerate(model.layers):
        x = layer_forward(x, lw, model.cfg, index_pos, l, cache, model.cos, model.sin, model.act)
    return x


def model_logits(model: Model, hidden_last) -> np.ndarray:
    """ln_f + last-token slice + dense lm_head (qwen3_vl.rs:2462-2487)."""
    h = rms_norm(np.asarray(hidden_last)[None, :], model.final_norm, model.cfg.eps, model.act)
    return dense_linear(h, model.lm_head, model.act)[0]


def greedy_generate(model: Model, prompt, n_gen: int, cache: Cache | None = None,
                    forced=None):
    """Master::generate with temperature 0 (device argmax, qwen3_vl.rs:138-143).

    Returns (tokens, logits per step).  With ``forced`` (teacher forcing) the
    next input token is ``forced[i]`` instead of the argmax.
    """
    cache = cache or Cache(len(model.layers), model.cfg.max_seq_len)
    prompt = list(prompt)
    h = model_hidden(model, prompt, 0, cache)
    logits = model_logits(model, h[-1])
    toks, all_logits = [argmax_first(logits)], [logits]
    pos = len(prompt)
    for i in range(1, n_gen):
        inp = toks[-1] if forced is None else int(forced[i - 1])
        h = model_hidden(model, [inp], pos, cache)
        logits = model_logits(model, h[-1])
        toks.append(argmax_first(logits))
        all_logits.append(logits)
        pos += 1
    return toks, all_logits


def synth_model(cfg: ModelConfig, seed: int, std: float = 0.02) -> Model:
    """Random-init model from the seeded generator: bf16 N(0, std) weights
    drawn per tensor stream, norms 1.0, layer linears quantized by a1.

    Stream ids: layer l part p -> ((l + 1) << 8) + p with parts q, k, v, o,
    gate, up, down = 0..6; embedding 0xE0000, lm_head 0xE0002.
    """
    table = normal_table(std)
    H, I, D = cfg.hidden, cfg.inter, cfg.head_dim
    QH, KVH = cfg.heads, cfg.kv_heads
    st = lambda l, p: ((l + 1) << 8) + p  # noqa: E731
    layers = []
    one = lambda n: np.ones(n, dtype=np.float32)  # noqa: E731
    for l in range(cfg.layers):
        q = synth_normal(seed, st(l, 0), QH * D * H, table).reshape(QH * D, H)
        k = synth_normal(seed, st(l, 1), KVH * D * H, table).reshape(KVH * D, H)
        v = synth_normal(seed, st(l, 2), KVH * D * H, table).reshape(KVH * D, H)
        qkv_q, qkv_s = quantize_w8a16_rows(np.concatenate([q, k, v], axis=0))
        o_q, o_s = quantize_w8a16_rows(synth_normal(seed, st(l, 3), H * QH * D, table).reshape(H, QH * D))
        g = synth_normal(seed, st(l, 4), I * H, table).reshape(I, H)
        u = synth_normal(seed, st(l, 5), I * H, table).reshape(I, H)
        gu_q, gu_s = quantize_w8a16_rows(np.concatenate([g, u], axis=0))
        d_q, d_s = quantize_w8a16_rows(synth_normal(seed, st(l, 6), H * I, table).reshape(H, I))
        layers.append(LayerWeights(qkv_q, qkv_s, o_q, o_s, gu_q, gu_s, d_q, d_s,
                                   one(H), one(H), one(D), one(D)))
    embed = synth_normal(seed, 0xE0000, cfg.vocab * H, table).reshape(cfg.vocab, H)
    lm_head = synth_normal(seed, 0xE0002, cfg.vocab * H, table).reshape(cfg.vocab, H)
    return Model(cfg, embed, layers, one(H), lm_head, "bf16")


# ---------------------------------------------------------------------------
# Seeded synthetic inputs (shared definition with the product's generator)
# ---------------------------------------------------------------------------

MASK64 = (1 << 64) - 1


def mix64(z: np.ndarray) -> np.ndarray:
    """SplitMix64 finalizer (Steele, Lea & Flood 2014) on uint64 arrays."""
    z = z.astype(np.uint64)
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    return z


def synth_hash(seed: int, stream: int, idx: np.ndarray) -> np.ndarray:
    """64-bit hash of (seed, stream, element index)."""
    base = np.uint64(((seed * 0x9E3779B97F4A7C15) ^ (stream * 0xD1B54A32D192ED03)) & MASK64)
    with np.errstate(over="ignore"):
        return mix64(idx.astype(np.uint64) + base)


@lru_cache(maxsize=8)
def normal_table(std: float) -> np.ndarray:
    """65536 bf16 quantiles of N(0, std) at (u + 0.5) / 65536, as f32 values."""
    from statistics import NormalDist

    nd = NormalDist(0.0, 1.0)
    q = np.array([nd.inv_cdf((u + 0.5) / 65536.0) for u in range(65536)], dtype=np.float64)
    return bf16_round((q * std).astype(np.float32))


def synth_normal(seed: int, stream: int, n: int, table: np.ndarray, offset: int = 0) -> np.ndarray:
    idx = np.arange(offset, offset + n, dtype=np.uint64)
    return table[(synth_hash(seed, stream, idx) & np.uint64(0xFFFF)).astype(np.int64)]


def synth_tokens(seed: int, n: int, vocab: int) -> np.ndarray:
    idx = np.arange(n, dtype=np.uint64)
    return (synth_hash(seed, 0x70CE, idx) % np.uint64(vocab)).astype(np.int64)


# ---------------------------------------------------------------------------
# f4: Gated-DeltaNet token mixer of the Qwen3.8 hybrid (qwen3_8/text.rs:233-481)
# ---------------------------------------------------------------------------
#
# Rounding points (candle-owned, unpinned by any reference test): the causal
# depthwise conv sums its K products in f32 and rounds once to the activation
# dtype; SiLU and sigmoid round each elementary step to the activation dtype
# (SiLU as silu_mul above, sigmoid act(1 / act(1 + act(exp(-x))))); everything
# from the l2 normalisation on (q, k, v, beta, g, the recurrence) is f32 as
# the reference states (text.rs:393-459); the scan output is rounded to the
# activation dtype before the gated RMSNorm (text.rs:460-466), which is f32
# with one rounding at its end (text.rs:240-250).


def silu_act(v, act: str = "bf16") -> np.ndarray:
    """candle SiLU on activation-dtype values: act(v / act(1 + act(exp(-v))))."""
    r = lambda t: act_round(t, act)  # noqa: E731
    v = np.asarray(v, dtype=np.float32)
    e = r(np.exp((-v).astype(np.float64)).astype(np.float32))
    return r(v / r(np.float32(1.0) + e))


def sigmoid_act(v, act: str = "bf16") -> np.ndarray:
    """candle sigmoid on activation-dtype values: act(1 / act(1 + act(exp(-v))))."""
    r = lambda t: act_round(t, act)  # noqa: E731
    v = np.asarray(v, dtype=np.float32)
    e = r(np.exp((-v).astype(np.float64)).astype(np.float32))
    return r(np.float32(1.0) / r(np.float32(1.0) + e))


def gdn_causal_conv(mixed, weight, prev, act: str = "bf16"):
    """GatedDeltaNet::causal_conv (text.rs:301-337): depthwise causal conv1d of
    kernel K over time, then SiLU.  mixed [S, C]; weight [C, K]; prev [C, K-1]
    (the carried conv state) or None (zeros: a sequence start).  Returns
    (silu(conv) [S, C], new state [C, K-1] = the last K-1 inputs)."""
    mixed = np.asarray(mixed, dtype=np.float32)
    S, C = mixed.shape
    K = weight.shape[1]
    hist = np.zeros((C, K - 1), np.float32) if prev is None else np.asarray(prev, np.float32)
    inp = np.concatenate([hist, mixed.T], axis=1)  # [C, K-1+S]
    out = np.empty((S, C), np.float32)
    w = np.asarray(weight, dtype=np.float32)
    for t in range(S):
        out[t] = act_round(np.sum(inp[:, t:t + K].astype(np.float64) * w, axis=1)
                           .astype(np.float32), act)
    state = inp[:, -(K - 1):].copy() if K > 1 else np.zeros((C, 0), np.float32)
    return silu_act(out, act), state


def gdn_l2_normalize(x) -> np.ndarray:
    """GatedDeltaNet::l2_normalize (text.rs:339-342): x / sqrt(sum x^2 + 1e-6), f32."""
    x = np.asarray(x, dtype=np.float32)
    ss = np.sum(x.astype(np.float64) ** 2, axis=-1, keepdims=True).astype(np.float32)
    return (x / np.sqrt(ss + np.float32(1e-6))).astype(np.float32)


def gdn_recurrent_scan(q, k, v, g, beta, state):
    """GatedDeltaNet::recurrent_scan (text.rs:344-388), f32: per token
    state *= exp(g); pred = k . state; delta = (v - pred) * beta;
    state += k (x) delta; out = q . state.  q, k [H, S, dk]; v [H, S, dv];
    g, beta [H, S]; state [H, dk, dv].  Returns (out [H, S, dv], state)."""
    q, k, v = (np.asarray(t, np.float32) for t in (q, k, v))
    st = np.array(state, dtype=np.float32, copy=True)
    H, S, _ = q.shape
    out = np.empty((H, S, v.shape[2]), np.float32)
    for t in range(S):
        st = (st * np.exp(g[:, t].astype(np.float32))[:, None, None]).astype(np.float32)
        pred = np.einsum("hi,hij->hj", k[:, t].astype(np.float64), st.astype(np.float64))
        delta = ((v[:, t] - pred.astype(np.float32)) * beta[:, t][:, None]).astype(np.float32)
        st = (st + k[:, t][:, :, None] * delta[:, None, :]).astype(np.float32)
        out[:, t] = np.einsum("hi,hij->hj", q[:, t].astype(np.float64),
                              st.astype(np.float64)).astype(np.float32)
    return out, st


def gdn_gated_rms_norm(x, gate, weight, eps: float, act: str = "bf16") -> np.ndarray:
    """GatedRmsNorm::forward (text.rs:240-250): f32 x / sqrt(mean x^2 + eps) *
    w * silu(gate), rounded once to the activation dtype."""
    x = np.asarray(x, dtype=np.float32)
    ms = (np.sum(x.astype(np.float64) ** 2, axis=-1, keepdims=True) / x.shape[-1]).astype(np.float32)
    y = x / np.sqrt(ms + np.float32(eps))
    gate = np.asarray(gate, dtype=np.float32)
    silu = gate / (np.float32(1.0) + np.exp(-gate.astype(np.float64)).astype(np.float32))
    return act_round(y * np.asarray(weight, np.float32) * silu, act)


def zero_centered_rms_norm(x, weight, eps: float, act: str = "bf16") -> np.ndarray:
    """ZeroCenteredRmsNorm::forward (text.rs:26-38): f32 x / sqrt(mean x^2 + eps)
    * (w + 1), rounded once to the activation dtype."""
    x = np.asarray(x, dtype=np.float32)
    ms = (np.sum(x.astype(np.float64) ** 2, axis=-1, keepdims=True) / x.shape[-1]).astype(np.float32)
    y = x / np.sqrt(ms + np.float32(eps))
    return act_round(y * (np.asarray(weight, np.float32) + np.float32(1.0)), act)


@dataclass
class GdnState:
    """Per-session linear-attention state of one layer (cache.rs:267-290):
    conv [C, K-1] (activation values) and recurrent [Hv, dk, dv] f32."""
    conv: np.ndarray
    recurrent: np.ndarray


def gdn_mixer(mixed, z, b, a, conv_w, dt_bias, a_log, norm_w, hk: int, hv: int, dk: int,
              dv: int, eps: float, state: GdnState | None, act: str = "bf16"):
    """GatedDeltaNet::forward (text.rs:390-481) from the outputs of its input
    projections to the input of out_proj: mixed [S, 2*hk*dk + hv*dv] (q | k |
    v), z [S, hv*dv], b and a [S, hv]; conv_w [C, K]; dt_bias, a_log [hv];
    norm_w [dv]; state None at a sequence start (index_pos 0).  Returns
    (core [S, hv*dv] in the activation dtype, the new GdnState)."""
    mixed = np.asarray(mixed, np.float32)
    S = mixed.shape[0]
    conv_out, conv_state = gdn_causal_conv(mixed, conv_w, None if state is None else state.conv,
                                           act)
    ks = hk * dk
    q = conv_out[:, :ks].reshape(S, hk, dk).transpose(1, 0, 2)
    k = conv_out[:, ks:2 * ks].reshape(S, hk, dk).transpose(1, 0, 2)
    v = conv_out[:, 2 * ks:].reshape(S, hv, dv).transpose(1, 0, 2)
    rep = hv // hk
    q = np.repeat(q, rep, axis=0)  # repeat_kv: v head h reads key head h // rep
    k = np.repeat(k, rep, axis=0)
    q = (gdn_l2_normalize(q) / np.float32(math.sqrt(dk))).astype(np.float32)
    k = gdn_l2_normalize(k)
    beta = sigmoid_act(b, act).T.astype(np.float32)  # [hv, S]
    af = np.asarray(a, np.float32)
    sp = np.log(np.exp((af + np.asarray(dt_bias, np.float32)).astype(np.float64)) + 1.0) \
        .astype(np.float32)
    g = (-(sp * np.exp(np.asarray(a_log, np.float32).astype(np.float64)).astype(np.float32))) \
        .T.astype(np.float32)  # [hv, S]
    rec = np.zeros((hv, dk, dv), np.float32) if state is None else state.recurrent
    core, rec = gdn_recurrent_scan(q, k, v, g, beta, rec)
    core = act_round(core.transpose(1, 0, 2), act)  # [S, hv, dv]
    zz = np.asarray(z, np.float32).reshape(S, hv, dv)
    out = gdn_gated_rms_norm(core, zz, norm_w, eps, act).reshape(S, hv * dv)
    return out, GdnState(conv_state, rec)


# ---------------------------------------------------------------------------
# f4: the Qwen3.8 full-attention layers (qwen3_8/text.rs:82-226)
# ---------------------------------------------------------------------------


def rope_partial(x, cos, sin, rotary_dim: int, act: str = "bf16") -> np.ndarray:
    """rotate_partial (qwen3_8/text.rs:83-110): the half-split rotation on the
    first ``rotary_dim`` dims of x [..., T, D] with tables [T, rotary_dim/2];
    the remaining dims pass through unchanged."""
    x = np.asarray(x, dtype=np.float32)
    d = x.shape[-1]
    rot = rope(x[..., :rotary_dim], cos, sin, act)
    if rotary_dim == d:
        return rot
    return np.concatenate([rot, x[..., rotary_dim:]], axis=-1)


@dataclass
class FullAttnState:
    """Per-session KV of one full-attention layer (llama3/cache.rs:117-160):
    k, v [kv_heads, L, head_dim] in the activation dtype."""
    k: np.ndarray
    v: np.ndarray


def gated_full_attention(q_gate, k, v, q_norm_w, k_norm_w, heads: int, kv_heads: int,
                         head_dim: int, rotary_dim: int, cos, sin, eps: float, index_pos: int,
                         state: FullAttnState | None, act: str = "bf16", attn_f32: bool = False):
    """FullAttention::forward (qwen3_8/text.rs:146-226) between its input
    projections and o_proj, for one session.

    q_gate [S, heads * 2 * head_dim] holds [q | gate] per head (text.rs:155-166:
    head h is columns [2 h d, 2 h d + d) for q and the next d for its gate);
    k, v [S, kv_heads * head_dim]; cos / sin the tables' rows from index_pos
    ([S, rotary_dim / 2]).  q and k take the zero-centred RMSNorm per head
    (text.rs:26-38), the partial RoPE, the session's cache, grouped causal
    attention in the activation dtype (f32 with ``attn_f32``) with the softmax
    in f32, and the output is multiplied by sigmoid(gate) (text.rs:223).
    Returns (out [S, heads * head_dim], the new FullAttnState)."""
    S = np.asarray(q_gate).shape[0]
    qg = np.asarray(q_gate, np.float32).reshape(S, heads, 2 * head_dim)
    q = qg[:, :, :head_dim]
    gate = qg[:, :, head_dim:].reshape(S, heads * head_dim)
    q = zero_centered_rms_norm(q, q_norm_w, eps, act).transpose(1, 0, 2)  # [heads, S, d]
    kk = zero_centered_rms_norm(np.asarray(k, np.float32).reshape(S, kv_heads, head_dim),
                                k_norm_w, eps, act).transpose(1, 0, 2)
    vv = act_round(np.asarray(v, np.float32).reshape(S, kv_heads, head_dim).transpose(1, 0, 2),
                   act)
    q = rope_partial(q, cos, sin, rotary_dim, act)
    kk = rope_partial(kk, cos, sin, rotary_dim, act)
    if state is not None and index_pos > 0:  # index_pos 0 starts the session over
        kk = np.concatenate([state.k, kk], axis=1)
        vv = np.concatenate([state.v, vv], axis=1)
    cdt = "f32" if attn_f32 else act
    out = attention(act_round(q, cdt), act_round(kk, cdt), act_round(vv, cdt), causal=True,
                    act=cdt)
    out = act_round(out, act).transpose(1, 0, 2).reshape(S, heads * head_dim)
    out = act_round(out * sigmoid_act(gate, act), act)
    return out, FullAttnState(kk, vv)
