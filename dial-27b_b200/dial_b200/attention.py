"""Fused decode attention op over paged KV (C ABI dial_b200_attention_decode).

The B200 counterpart of QwenAttention::forward's per-token middle section
(dial-core/src/models/qwen3_vl/text.rs:1466-1536 and 1258-1281): q/k RMSNorm,
RoPE, KV append and grouped attention, for many decode rows at once.
"""

from __future__ import annotations

import ctypes as C

import torch

from ._abi import ACT_BF16, ACT_F16, AttnShape, DialError, call, lib

_ACT = {torch.bfloat16: ACT_BF16, torch.float16: ACT_F16}


def _p(t: torch.Tensor):
    return C.c_void_p(t.data_ptr())


def make_shape(q_heads: int, kv_heads: int, max_blocks: int, max_pos: int, eps: float = 1e-6,
               dtype: torch.dtype = torch.bfloat16, num_blocks: int = 0) -> AttnShape:
    """num_blocks: pages in each KV pool; > 0 lets steps of more than 4 rows
    take the tensor-core form."""
    return AttnShape(q_heads, kv_heads, 128, max_blocks, max_pos, eps, _ACT[dtype], num_blocks)


def scratch_bytes(sh: AttnShape, rows: int, splits: int) -> int:
    return int(lib.dial_b200_attention_scratch_bytes(C.byref(sh), rows, splits))


def attention_decode(sh: AttnShape, qkv, q_norm_w, k_norm_w, cos, sin, k_pages, v_pages,
                     block_table, sids, positions, out, splits: int = 1, scratch=None):
    """Run the fused op on the current CUDA stream; `out` receives the result."""
    rows = qkv.shape[0]
    stream = torch.cuda.current_stream(qkv.device).cuda_stream
    call("dial_b200_attention_decode", C.byref(sh), _p(qkv), qkv.shape[1], _p(q_norm_w),
         _p(k_norm_w), _p(cos), _p(sin), _p(k_pages), _p(v_pages), _p(block_table), _p(sids),
         _p(positions), _p(out), out.shape[1], rows, splits,
         C.c_void_p(scratch.data_ptr() if scratch is not None else 0), C.c_void_p(stream))
    return out


NOALLOC_MAX_PART_ROWS = 2048
NOALLOC_MAX_COUNTERS = 1024


def attention_decode_noalloc(sh: AttnShape, qkv, q_norm_w, k_norm_w, cos, sin, k_pages, v_pages,
                             block_table, sids, positions, out, splits: int = 1):
    """attention_decode with the split-KV scratch in the library's static
    device array: allocates nothing.  Limits: rows * q_heads * splits <=
    2048 and rows * kv_heads <= 1024 when splits > 1.  Calls that overlap on
    one device race on that scratch."""
    rows = qkv.shape[0]
    stream = torch.cuda.current_stream(qkv.device).cuda_stream
    call("dial_b200_attention_decode_noalloc", C.byref(sh), _p(qkv), qkv.shape[1], _p(q_norm_w),
         _p(k_norm_w), _p(cos), _p(sin), _p(k_pages), _p(v_pages), _p(block_table), _p(sids),
         _p(positions), _p(out), out.shape[1], rows, splits, C.c_void_p(stream))
    return out
