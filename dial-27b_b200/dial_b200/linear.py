"""Linear custom ops: the B200 counterparts of the reference's candle
``CustomOp1`` implementations.

* ``CudaW8A16Linear`` -- dial-core/src/models/qwen3_vl/worker_w8a16.rs:295-476
* ``CudaQuantLinear`` -- dial-core/src/models/qwen3_8/cuda_quant.rs:256-500

Both keep their weights device resident for the object's lifetime and run
``forward`` on the current torch CUDA stream through the C ABI; outputs are
newly allocated tensors, like the reference's ``cuda_fwd``.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _abi
from ._abi import ACT_BF16, ACT_F16, ACT_F32, DialError, call, lib

_ACT = {torch.bfloat16: ACT_BF16, torch.float16: ACT_F16}
_SRC = {torch.bfloat16: ACT_BF16, torch.float16: ACT_F16, torch.float32: ACT_F32}
_NAME = {torch.bfloat16: "BF16", torch.float16: "F16", torch.float32: "F32"}


def _host_bytes(a) -> np.ndarray:
    if isinstance(a, torch.Tensor):
        a = a.detach().cpu()
        if a.dtype == torch.bfloat16:
            a = a.view(torch.int16)
        a = a.numpy()
    elif isinstance(a, (bytes, bytearray)):
        a = np.frombuffer(a, dtype=np.uint8)
    return np.ascontiguousarray(a)


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


class _QLinearBase:
    _handle: C.c_void_p
    in_dim: int
    out_dim: int
    act: torch.dtype
    op_name = "linear"

    def __del__(self):
        h = getattr(self, "_handle", None)
        if h:
            lib.dial_b200_qlinear_destroy(h)
            self._handle = None

    def resident_bytes(self) -> int:
        return int(lib.dial_b200_qlinear_resident_bytes(self._handle))

    def _check_input(self, x: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = self._check_input(x)
        rows = x.numel() // self.in_dim
        y = torch.empty(*x.shape[:-1], self.out_dim, dtype=x.dtype, device=x.device)
        stream = torch.cuda.current_stream(x.device).cuda_stream
        with torch.cuda.device(x.device):
            call("dial_b200_qlinear_forward", self._handle, C.c_void_p(x.data_ptr()),
                 C.c_void_p(y.data_ptr()), rows, C.c_void_p(stream))
        return y

    __call__ = forward


class CudaW8A16Linear(_QLinearBase):
    """Row-wise int8 weight, activation-dtype input/output, f32 row scales."""

    op_name = "dial-w8a16-linear"

    @classmethod
    def from_linear(cls, name: str, weight: torch.Tensor, act: torch.dtype = torch.float16,
                    bias: torch.Tensor | None = None) -> "CudaW8A16Linear":
        """Quantize a dense ``[out, in]`` weight (worker_w8a16.rs:302-366)."""
        if bias is not None:
            raise DialError(_abi.DIAL_ERR_INVALID, "W8A16 only supports bias-free linear layers")
        if weight.dim() != 2:
            raise DialError(_abi.DIAL_ERR_INVALID, f"expected a 2-D weight, got {tuple(weight.shape)}")
        if weight.dtype not in _SRC:
            raise DialError(_abi.DIAL_ERR_INVALID, f"unsupported weight dtype {weight.dtype}")
        if act not in _ACT:
            raise DialError(_abi.DIAL_ERR_INVALID, f"W8A16 activations must be F16 or BF16, got {act}")
        self = cls.__new__(cls)
        self.name = name
        self.out_dim, self.in_dim = (int(s) for s in weight.shape)
        self.act = act
        w = _host_bytes(weight.contiguous())
        h = C.c_void_p()
        call("dial_b200_w8a16_from_dense", _ptr(w), _SRC[weight.dtype], self.out_dim, self.in_dim,
             _ACT[act], C.byref(h))
        self._handle = h
        return self

    @classmethod
    def from_quantized(cls, q: np.ndarray, scale: np.ndarray, act: torch.dtype = torch.bfloat16
                       ) -> "CudaW8A16Linear":
        q = np.ascontiguousarray(q, dtype=np.int8)
        s = np.ascontiguousarray(scale, dtype=np.float32)
        self = cls.__new__(cls)
        self.name = "w8a16"
        self.out_dim, self.in_dim = q.shape
        self.act = act
        h = C.c_void_p()
        call("dial_b200_qlinear_create", _abi.FMT_W8A16_ROW, _ACT[act], _ptr(q), _ptr(s), 0.0,
             self.in_dim, self.out_dim, C.byref(h))
        self._handle = h
        return self

    def _check_input(self, x: torch.Tensor) -> torch.Tensor:
        # worker_w8a16.rs:368-387
        if x.dtype != self.act:
            raise DialError(_abi.DIAL_ERR_INVALID,
                            f"W8A16 expects {_NAME.get(self.act)} activation, got {_NAME.get(x.dtype, x.dtype)}")
        if x.dim() == 0 or x.shape[-1] != self.in_dim:
            raise DialError(_abi.DIAL_ERR_INVALID,
                            f"W8A16 input mismatch: expected last dim {self.in_dim}, got {list(x.shape)}")
        if not x.is_cuda:
            raise DialError(_abi.DIAL_ERR_INVALID, "W8A16 linear is only available on CUDA")
        return x.contiguous()


class CudaQuantLinear(_QLinearBase):
    """FP8 (e4m3) and NVFP4 (e2m1 + e4m3 group scale) weight-only linears."""

    op_name = "dial-qwen38-quant-linear"

    @classmethod
    def _make(cls, fmt, act, codes, scales, global_scale, in_dim, out_dim):
        self = cls.__new__(cls)
        self.in_dim, self.out_dim, self.act, self.fmt = in_dim, out_dim, act, fmt
        h = C.c_void_p()
        call("dial_b200_qlinear_create", fmt, _ACT[act], _ptr(codes), _ptr(scales),
             float(global_scale), in_dim, out_dim, C.byref(h))
        self._handle = h
        return self

    @classmethod
    def nvfp4(cls, packed, scales, global_scale: float, in_dim: int, out_dim: int,
              act: torch.dtype = torch.float16) -> "CudaQuantLinear":
        """CudaQuantLinear::nvfp4 (cuda_quant.rs:270-303)."""
        if in_dim % 16 != 0:
            raise DialError(_abi.DIAL_ERR_INVALID,
                            f"NVFP4 QuantLinear input dimension {in_dim} is not divisible by 16")
        p = _host_bytes(packed).astype(np.uint8, copy=False).reshape(-1)
        s = _host_bytes(scales).astype(np.uint8, copy=False).reshape(-1)
        if p.size != out_dim * in_dim // 2:
            raise DialError(_abi.DIAL_ERR_INVALID, f"invalid NVFP4 packed weight length {p.size}")
        if s.size != out_dim * in_dim // 16:
            raise DialError(_abi.DIAL_ERR_INVALID, f"invalid NVFP4 scale length {s.size}")
        return cls._make(_abi.FMT_NVFP4_G16, act, p, s, global_scale, in_dim, out_dim)

    @classmethod
    def fp8(cls, weight, scales, in_dim: int, out_dim: int,
            act: torch.dtype = torch.float16) -> "CudaQuantLinear":
        """CudaQuantLinear::fp8 (cuda_quant.rs:305-334); a single per-tensor
        scale is expanded to every row as try_cuda_fp8 does (quant.rs:416-427)."""
        w = _host_bytes(weight).astype(np.uint8, copy=False).reshape(-1)
        s = np.ascontiguousarray(np.asarray(scales, dtype=np.float32).reshape(-1))
        if w.size != out_dim * in_dim:
            raise DialError(_abi.DIAL_ERR_INVALID, f"invalid FP8 weight length {w.size}")
        if s.size == 1:
            s = np.full(out_dim, s[0], dtype=np.float32)
        if s.size != out_dim:
            raise DialError(_abi.DIAL_ERR_INVALID, f"invalid FP8 scale length {s.size}")
        return cls._make(_abi.FMT_FP8_ROW, act, w, s, 0.0, in_dim, out_dim)

    @classmethod
    def fp8_block128(cls, weight, block_scales, in_dim: int, out_dim: int,
                     act: torch.dtype = torch.bfloat16) -> "CudaQuantLinear":
        """e4m3 weight with one f32 scale per 128x128 block."""
        w = _host_bytes(weight).astype(np.uint8, copy=False).reshape(-1)
        nbr, nbc = -(-out_dim // 128), -(-in_dim // 128)
        s = np.ascontiguousarray(np.asarray(block_scales, dtype=np.float32).reshape(-1))
        if w.size != out_dim * in_dim:
            raise DialError(_abi.DIAL_ERR_INVALID, f"invalid FP8 weight length {w.size}")
        if s.size != nbr * nbc:
            raise DialError(_abi.DIAL_ERR_INVALID, f"invalid FP8 block scale length {s.size}")
        return cls._make(_abi.FMT_FP8_BLOCK128, act, w, s, 0.0, in_dim, out_dim)

    def _check_input(self, x: torch.Tensor) -> torch.Tensor:
        # cuda_quant.rs:373-391
        if x.dtype != self.act:
            raise DialError(_abi.DIAL_ERR_INVALID,
                            f"Qwen3.8 QuantLinear expects {_NAME.get(self.act)} input, got {_NAME.get(x.dtype, x.dtype)}")
        if x.dim() == 0 or x.shape[-1] != self.in_dim:
            raise DialError(_abi.DIAL_ERR_INVALID,
                            f"Qwen3.8 QuantLinear expected last dim {self.in_dim}, got {list(x.shape)}")
        if not x.is_cuda:
            raise DialError(_abi.DIAL_ERR_INVALID, "Qwen3.8 QuantLinear is only available on CUDA")
        return x.contiguous()


class DenseLinear(_QLinearBase):
    """Activation-dtype dense weight through the same GEMV (the lm_head path)."""

    @classmethod
    def from_weight(cls, weight: torch.Tensor) -> "DenseLinear":
        if weight.dtype not in _ACT:
            raise DialError(_abi.DIAL_ERR_INVALID, "dense weight must be F16 or BF16")
        self = cls.__new__(cls)
        self.out_dim, self.in_dim = (int(s) for s in weight.shape)
        self.act = weight.dtype
        w = _host_bytes(weight.contiguous())
        h = C.c_void_p()
        call("dial_b200_qlinear_create", _abi.FMT_DENSE, _ACT[weight.dtype], _ptr(w), None, 0.0,
             self.in_dim, self.out_dim, C.byref(h))
        self._handle = h
        return self

    def _check_input(self, x):
        if x.dtype != self.act or x.shape[-1] != self.in_dim or not x.is_cuda:
            raise DialError(_abi.DIAL_ERR_INVALID, "dense linear input mismatch")
        return x.contiguous()


def w8a16_quantize(weight: torch.Tensor | np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """a1 on the GPU: row-wise int8 codes and f32 scales (worker_w8a16.rs:330-341)."""
    if isinstance(weight, np.ndarray):
        weight = torch.from_numpy(np.ascontiguousarray(weight, dtype=np.float32))
    out_dim, in_dim = weight.shape
    w = _host_bytes(weight.contiguous())
    q = np.empty((out_dim, in_dim), dtype=np.int8)
    s = np.empty(out_dim, dtype=np.float32)
    call("dial_b200_w8a16_quantize", _ptr(w), _SRC[weight.dtype], out_dim, in_dim, _ptr(q), _ptr(s))
    return q, s
