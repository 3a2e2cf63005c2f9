"""ctypes binding of libdial_b200.so (the C ABI in include/dial_b200.h).

There is no CPU fallback: importing this module without the built library
raises, and every entry point reports CUDA or argument errors as DialError.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

_HERE = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("DIAL_B200_LIB", _HERE / "libdial_b200.so"))

ABI_VERSION = 2  # DIAL_B200_ABI_VERSION of the structs below
DIAL_OK, DIAL_ERR_INVALID, DIAL_ERR_CUDA, DIAL_ERR_DEVICE = 0, 1, 2, 3
FMT_W8A16_ROW, FMT_FP8_BLOCK128, FMT_FP8_ROW, FMT_NVFP4_G16, FMT_DENSE = 0, 1, 2, 3, 4
ACT_BF16, ACT_F16, ACT_F32 = 0, 1, 2


class DialError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


if not LIB_PATH.exists():
    raise ImportError(
        f"{LIB_PATH} is missing: build it with `python dial-27b_b200/build.py` "
        "(the DIAL B200 path has no CPU fallback)")

lib = C.CDLL(str(LIB_PATH))


class AttnShape(C.Structure):
    _fields_ = [
        ("q_heads", C.c_int32),
        ("kv_heads", C.c_int32),
        ("head_dim", C.c_int32),
        ("max_blocks", C.c_int32),
        ("max_pos", C.c_int32),
        ("eps", C.c_float),
        ("act", C.c_int32),
        ("num_blocks", C.c_int32),
    ]


class GdnShape(C.Structure):
    _fields_ = [
        ("k_heads", C.c_int32),
        ("v_heads", C.c_int32),
        ("k_head_dim", C.c_int32),
        ("v_head_dim", C.c_int32),
        ("conv_kernel", C.c_int32),
        ("eps", C.c_float),
        ("act", C.c_int32),
    ]


class ModelConfig(C.Structure):
    _fields_ = [
        ("hidden_size", C.c_int32),
        ("intermediate_size", C.c_int32),
        ("vocab_size", C.c_int32),
        ("num_hidden_layers", C.c_int32),
        ("num_attention_heads", C.c_int32),
        ("num_key_value_heads", C.c_int32),
        ("rms_norm_eps", C.c_float),
        ("rope_theta", C.c_float),
        ("max_seq_len", C.c_int32),
        ("max_sessions", C.c_int32),
        ("max_tokens", C.c_int32),
        ("act", C.c_int32),
        ("linear_fmt", C.c_int32),
        ("first_layer", C.c_int32),
        ("num_layers", C.c_int32),
        ("has_embed", C.c_int32),
        ("has_head", C.c_int32),
    ]


_vp, _i64, _i32, _u64 = C.c_void_p, C.c_int64, C.c_int32, C.c_uint64
_err = [C.c_char_p, C.c_size_t]

_SIGS = {
    "dial_b200_abi_version": (C.c_uint32, []),
    "dial_b200_device_status": (C.c_int, [C.POINTER(C.c_int), C.c_int, *_err]),
    "dial_b200_w8a16_quantize": (C.c_int, [_vp, C.c_int, _i64, _i64, _vp, _vp, *_err]),
    "dial_b200_w8a16_from_dense": (C.c_int, [_vp, C.c_int, _i64, _i64, C.c_int, C.POINTER(_vp), *_err]),
    "dial_b200_qlinear_create": (C.c_int, [C.c_int, C.c_int, _vp, _vp, C.c_float, _i64, _i64,
                                           C.POINTER(_vp), *_err]),
    "dial_b200_qlinear_destroy": (None, [_vp]),
    "dial_b200_qlinear_forward": (C.c_int, [_vp, _vp, _vp, _i64, _vp, *_err]),
    "dial_b200_qlinear_in_dim": (_i64, [_vp]),
    "dial_b200_qlinear_out_dim": (_i64, [_vp]),
    "dial_b200_qlinear_resident_bytes": (_i64, [_vp]),
    "dial_b200_attention_scratch_bytes": (_i64, [C.POINTER(AttnShape), _i64, _i32]),
    "dial_b200_attention_decode": (C.c_int, [C.POINTER(AttnShape), _vp, _i64, _vp, _vp, _vp, _vp, _vp,
                                             _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i32, _vp, _vp,
                                             *_err]),
    "dial_b200_attention_decode_noalloc": (C.c_int, [C.POINTER(AttnShape), _vp, _i64, _vp, _vp, _vp, _vp,
                                                     _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i32,
                                                     _vp, *_err]),
    "dial_b200_stage_prepare": (C.c_int, [_vp, _i64, _vp, _vp, *_err]),
    "dial_b200_stage_step": (C.c_int, [_vp, _i64, _vp, _vp, _vp, _vp, *_err]),
    "dial_b200_stage_step_rows": (C.c_int, [_vp, _i64, _i64, _vp, _vp, _vp, _vp, *_err]),
    "dial_b200_gdn_scratch_bytes": (_i64, [C.POINTER(GdnShape), _i64]),
    "dial_b200_stage_link_handle": (C.c_int, [_vp, _vp, *_err]),
    "dial_b200_stage_link_open": (C.c_int, [_vp, _vp, _vp, *_err]),
    "dial_b200_stage_link_step": (C.c_int, [_vp, _i64, _vp, _vp, *_err]),
    "dial_b200_stage_link_finish": (C.c_int, [_vp, _i64, _vp, _vp, *_err]),
    "dial_b200_gdn_forward": (C.c_int, [C.POINTER(GdnShape), _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                        _vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp, *_err]),
    "dial_b200_engine_create": (C.c_int, [C.POINTER(ModelConfig), C.c_int, C.POINTER(_vp), *_err]),
    "dial_b200_engine_destroy": (None, [_vp]),
    "dial_b200_engine_load_synthetic": (C.c_int, [_vp, _u64, _vp, *_err]),
    "dial_b200_engine_set_linear": (C.c_int, [_vp, C.c_int, C.c_int, C.c_int, _vp, _vp, C.c_float,
                                              _i64, _i64, *_err]),
    "dial_b200_engine_set_tensor": (C.c_int, [_vp, C.c_int, C.c_int, _vp, _i64, *_err]),
    "dial_b200_layer_forward": (C.c_int, [_vp, C.c_int, _vp, _i64, _i32, _i64, _vp, *_err]),
    "dial_b200_range_forward": (C.c_int, [_vp, C.c_int, C.c_int, _vp, _i64, _i32, _i64, _vp, *_err]),
    "dial_b200_batch_decode_forward": (C.c_int, [_vp, C.c_int, C.c_int, _vp, _i64, _vp, _vp, _vp,
                                                 *_err]),
    "dial_b200_session_reset": (C.c_int, [_vp, _i32, *_err]),
    "dial_b200_embed": (C.c_int, [_vp, _vp, _i64, _vp, _vp, *_err]),
    "dial_b200_head": (C.c_int, [_vp, _vp, _i64, _vp, _vp, _vp, *_err]),
    "dial_b200_decode_step": (C.c_int, [_vp, _i64, _vp, _vp, _vp, _vp, *_err]),
    "dial_b200_generate": (C.c_int, [_vp, _i32, _vp, _i64, _i64, _vp, C.POINTER(C.c_double),
                                     C.POINTER(C.c_double), *_err]),
    "dial_b200_decode_loop_prepare": (C.c_int, [_vp, _i64, _vp, _vp, _vp, *_err]),
    "dial_b200_decode_loop_run": (C.c_int, [_vp, _i64, _i64, *_err]),
    "dial_b200_decode_loop_state": (C.c_int, [_vp, _i64, _vp, _vp, *_err]),
    "dial_b200_engine_stream": (_vp, [_vp]),
    "dial_b200_session_fill_random": (C.c_int, [_vp, _i32, _i64, _u64, _vp, *_err]),
    "dial_b200_step_kernel_count": (_i64, [_vp, _i64]),
    "dial_b200_prefill_kernel_count": (_i64, [_vp, _i64]),
    "dial_b200_engine_linear_replay": (C.c_int, [_vp, C.c_int, C.c_int, _i64, _i64, *_err]),
    "dial_b200_engine_linear_bytes": (_i64, [_vp, C.c_int, C.c_int, _i64]),
}

for _name, (_res, _args) in _SIGS.items():
    _f = getattr(lib, _name)
    _f.restype = _res
    _f.argtypes = _args

if lib.dial_b200_abi_version() != ABI_VERSION:
    raise ImportError(f"{LIB_PATH} has ABI version {lib.dial_b200_abi_version()}, this binding "
                      f"expects {ABI_VERSION}: rebuild it with `python dial-27b_b200/build.py`")


def call(name: str, *args):
    """Call an int-status entry point, raising DialError on failure."""
    buf = C.create_string_buffer(1024)
    rc = getattr(lib, name)(*args, buf, C.sizeof(buf))
    if rc != DIAL_OK:
        raise DialError(rc, buf.value.decode(errors="replace") or f"{name} failed ({rc})")
    return rc


def exported_symbols() -> list[str]:
    return list(_SIGS)
