"""Gated-DeltaNet token mixer of the Qwen3.8 hybrid (C ABI dial_b200_gdn_forward).

The B200 counterpart of GatedDeltaNet::forward
(dial-core/src/models/qwen3_8/text.rs:390-481) between its input projections
and out_proj: causal depthwise conv + SiLU over q | k | v, L2-normalised q and
k, the gated delta-rule recurrence in f32, and the gated RMSNorm.  The
per-session linear-attention cache (llama3/cache.rs:267-290) is a
``GdnState`` of device tensors.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from ._abi import ACT_BF16, ACT_F16, GdnShape, call, lib

_ACT = {torch.bfloat16: ACT_BF16, torch.float16: ACT_F16}
HEAD_DIM = 128


def _p(t: torch.Tensor | None):
    return C.c_void_p(t.data_ptr() if t is not None else 0)


def make_shape(k_heads: int, v_heads: int, conv_kernel: int = 4, eps: float = 1e-6,
               dtype: torch.dtype = torch.bfloat16) -> GdnShape:
    return GdnShape(k_heads, v_heads, HEAD_DIM, HEAD_DIM, conv_kernel, eps, _ACT[dtype])


def channels(sh: GdnShape) -> int:
    return 2 * sh.k_heads * sh.k_head_dim + sh.v_heads * sh.v_head_dim


@dataclass
class GdnState:
    """conv [channels, K-1] (activation dtype) and recurrent [v_heads, 128, 128] f32."""
    conv: torch.Tensor
    recurrent: torch.Tensor

    @classmethod
    def empty(cls, sh: GdnShape, device, dtype=torch.bfloat16) -> "GdnState":
        return cls(torch.zeros(channels(sh), sh.conv_kernel - 1, dtype=dtype, device=device),
                   torch.zeros(sh.v_heads, sh.k_head_dim, sh.v_head_dim, dtype=torch.float32,
                               device=device))


def gdn_forward(sh: GdnShape, mixed: torch.Tensor, z: torch.Tensor, b: torch.Tensor,
                a: torch.Tensor, conv_weight: torch.Tensor, dt_bias: torch.Tensor,
                a_log: torch.Tensor, norm_weight: torch.Tensor, state: GdnState,
                index_pos: int) -> torch.Tensor:
    """One call for seq_len = mixed.shape[0] tokens starting at index_pos
    (0 restarts the state); returns core [seq_len, v_heads * 128] on the current
    stream and leaves the state after the call in ``state``."""
    S = mixed.shape[0]
    dev = mixed.device
    scratch = torch.empty(int(lib.dial_b200_gdn_scratch_bytes(C.byref(sh), S)), dtype=torch.uint8,
                          device=dev)
    out = torch.empty(S, sh.v_heads * sh.v_head_dim, dtype=mixed.dtype, device=dev)
    f32 = lambda t: t.to(device=dev, dtype=torch.float32).contiguous()  # noqa: E731
    dt, al, nw = f32(dt_bias), f32(a_log), f32(norm_weight)
    stream = torch.cuda.current_stream(dev).cuda_stream
    call("dial_b200_gdn_forward", C.byref(sh), _p(mixed.contiguous()), _p(z.contiguous()),
         _p(b.contiguous()), _p(a.contiguous()), _p(conv_weight.contiguous()), _p(dt), _p(al),
         _p(nw), _p(state.conv), _p(state.recurrent), S, index_pos, _p(scratch), _p(out),
         C.c_void_p(stream))
    return out
