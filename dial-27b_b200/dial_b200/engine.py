"""Layer engine: the B200 counterpart of the reference's ``Forwarder`` layer
API, per-connection KV ``Cache`` and ``Worker`` layer ownership.

* ``Engine.forward`` .............. Forwarder::forward (dial-core/src/spm/mod.rs:236-242;
                                     Transformer::forward, qwen3_vl/text.rs:1636-1688)
* ``Engine.forward_local_batch`` .. Forwarder::forward_local_batch (spm/mod.rs:268-277)
* ``Engine.batch_decode`` ......... one decode token for many sessions (paged KV)
* ``Engine.session_reset`` ........ Cache::clear / as_new (llama3/cache.rs:240-265)
* ``Engine.generate`` ............. Master::generate greedy loop (spm/master.rs:56-103)

An engine owns a contiguous layer range (one topology node / pipeline
stage); ``has_embed``/``has_head`` mark the first and last stages.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _abi
from ._abi import ACT_BF16, ACT_F16, DialError, ModelConfig, call, lib
from .synth import normal_table_bits

_TORCH_ACT = {ACT_BF16: torch.bfloat16, ACT_F16: torch.float16}


@dataclass
class Config:
    """llama3::Config shape contract (llama3/config.rs:68-85), Qwen3-8B defaults."""
    hidden_size: int = 4096
    intermediate_size: int = 12288
    vocab_size: int = 151936
    num_hidden_layers: int = 36
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    max_seq_len: int = 4096
    max_sessions: int = 1
    max_tokens: int = 2048
    act: int = ACT_BF16
    linear_fmt: int = _abi.FMT_W8A16_ROW

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    @property
    def qkv_dim(self) -> int:
        return (self.num_attention_heads + 2 * self.num_key_value_heads) * self.head_dim

    @classmethod
    def qwen3_8b(cls, **kw) -> "Config":
        return cls(**kw)

    @classmethod
    def dense_27b(cls, **kw) -> "Config":
        base = dict(hidden_size=5120, intermediate_size=21504, num_hidden_layers=64,
                    num_attention_heads=40, num_key_value_heads=8)
        base.update(kw)
        return cls(**base)


def _np_ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def _host(a, dtype=None) -> np.ndarray:
    if isinstance(a, torch.Tensor):
        a = a.detach().cpu()
        if a.dtype == torch.bfloat16:
            a = a.view(torch.int16)
        a = a.numpy()
    a = np.ascontiguousarray(a if dtype is None else a.astype(dtype))
    return a


def _act_bits(x: np.ndarray, act: int) -> np.ndarray:
    """float32 values -> uint16 bit patterns of the activation dtype."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if act == ACT_F16:
        return x.astype(np.float16).view(np.uint16)
    b = x.view(np.uint32).astype(np.uint64)
    bias = ((b >> np.uint64(16)) & np.uint64(1)) + np.uint64(0x7FFF)
    return ((b + bias) >> np.uint64(16)).astype(np.uint16)


class Engine:
    LINEAR_QKV, LINEAR_O, LINEAR_GATE_UP, LINEAR_DOWN, LINEAR_LM_HEAD = range(5)
    T_INPUT_NORM, T_POST_NORM, T_Q_NORM, T_K_NORM, T_FINAL_NORM, T_EMBED = range(6)

    def __init__(self, cfg: Config, first_layer: int = 0, num_layers: int | None = None,
                 has_embed: bool | None = None, has_head: bool | None = None, device: int = 0):
        if num_layers is None:
            num_layers = cfg.num_hidden_layers - first_layer
        if has_embed is None:
            has_embed = first_layer == 0
        if has_head is None:
            has_head = first_layer + num_layers == cfg.num_hidden_layers
        self.cfg = cfg
        self.first_layer, self.num_layers = first_layer, num_layers
        self.has_embed, self.has_head = has_embed, has_head
        self.device = device
        self.dtype = _TORCH_ACT[cfg.act]
        c = ModelConfig(cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size,
                        cfg.num_hidden_layers, cfg.num_attention_heads, cfg.num_key_value_heads,
                        cfg.rms_norm_eps, cfg.rope_theta, cfg.max_seq_len, cfg.max_sessions,
                        cfg.max_tokens, cfg.act, cfg.linear_fmt, first_layer, num_layers,
                        int(has_embed), int(has_head))
        h = C.c_void_p()
        call("dial_b200_engine_create", C.byref(c), device, C.byref(h))
        self._h = h
        self.stream = torch.cuda.ExternalStream(lib.dial_b200_engine_stream(h), device=device)

    def close(self):
        if getattr(self, "_h", None):
            lib.dial_b200_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    # ------------------------------------------------------------- weights
    def load_synthetic(self, seed: int = 0, std: float = 0.02):
        """Random-init bf16 weights N(0, std), norms 1.0, quantized at load."""
        table = normal_table_bits(std)
        call("dial_b200_engine_load_synthetic", self._h, seed, _np_ptr(table))

    def set_linear(self, layer: int, which: int, fmt: int, codes, scales=None,
                   global_scale: float = 0.0):
        codes = _host(codes)
        out_dim, in_dim = codes.shape[0], codes.shape[1]
        if fmt == _abi.FMT_NVFP4_G16:
            in_dim *= 2
        sc = None if scales is None else _host(scales)
        call("dial_b200_engine_set_linear", self._h, layer, which, fmt, _np_ptr(codes),
             None if sc is None else _np_ptr(sc), float(global_scale), out_dim, in_dim)

    def set_tensor(self, layer: int, which: int, values):
        bits = values if (isinstance(values, np.ndarray) and values.dtype == np.uint16) \
            else _act_bits(np.asarray(values, dtype=np.float32), self.cfg.act)
        bits = np.ascontiguousarray(bits.reshape(-1))
        call("dial_b200_engine_set_tensor", self._h, layer, which, _np_ptr(bits), bits.size)

    def set_layer_w8a16(self, layer: int, lw):
        """Install an oracle-style LayerWeights (int8 codes + f32 scales)."""
        f = _abi.FMT_W8A16_ROW
        self.set_linear(layer, self.LINEAR_QKV, f, lw.qkv_q, lw.qkv_s)
        self.set_linear(layer, self.LINEAR_O, f, lw.o_q, lw.o_s)
        self.set_linear(layer, self.LINEAR_GATE_UP, f, lw.gate_up_q, lw.gate_up_s)
        self.set_linear(layer, self.LINEAR_DOWN, f, lw.down_q, lw.down_s)
        self.set_tensor(layer, self.T_INPUT_NORM, lw.input_norm)
        self.set_tensor(layer, self.T_POST_NORM, lw.post_norm)
        self.set_tensor(layer, self.T_Q_NORM, lw.q_norm)
        self.set_tensor(layer, self.T_K_NORM, lw.k_norm)

    # ------------------------------------------------------------- forward
    def _stream_ptr(self):
        return C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    def forward(self, x: torch.Tensor, index_pos: int, block_idx: int, session: int = 0
                ) -> torch.Tensor:
        """Forwarder::forward for one layer; x [seq, H] or [1, seq, H] (device)."""
        return self.forward_local_batch(x, [(f"model.layers.{block_idx}", index_pos, block_idx)],
                                        session)

    def forward_local_batch(self, x: torch.Tensor, batch, session: int = 0) -> torch.Tensor:
        """Forwarder::forward_local_batch: (layer_name, index_pos, block_idx) entries that
        must form one contiguous range sharing index_pos; validated before any
        cache update."""
        if not batch:
            return x
        idx = [b[2] for b in batch]
        pos = {b[1] for b in batch}
        if len(pos) != 1 or idx != list(range(idx[0], idx[0] + len(idx))):
            raise DialError(_abi.DIAL_ERR_INVALID, "batch must be one contiguous layer range")
        self._check_hidden(x)
        seq = x.numel() // self.cfg.hidden_size
        call("dial_b200_range_forward", self._h, idx[0], len(idx), C.c_void_p(x.data_ptr()), seq,
             session, pos.pop(), self._stream_ptr())
        return x

    def batch_decode(self, x: torch.Tensor, sids, positions, first: int | None = None,
                     count: int | None = None) -> torch.Tensor:
        self._check_hidden(x)
        first = self.first_layer if first is None else first
        count = self.num_layers if count is None else count
        s = np.ascontiguousarray(np.asarray(sids, dtype=np.int32))
        p = np.ascontiguousarray(np.asarray(positions, dtype=np.int32))
        call("dial_b200_batch_decode_forward", self._h, first, count, C.c_void_p(x.data_ptr()),
             s.size, _np_ptr(s), _np_ptr(p), self._stream_ptr())
        return x

    def session_reset(self, session: int):
        call("dial_b200_session_reset", self._h, session)

    def _check_hidden(self, x: torch.Tensor):
        if x.dtype != self.dtype or not x.is_cuda or not x.is_contiguous() or \
                x.shape[-1] != self.cfg.hidden_size:
            raise DialError(_abi.DIAL_ERR_INVALID,
                            f"hidden state must be a contiguous CUDA {self.dtype} [.., "
                            f"{self.cfg.hidden_size}] tensor, got {x.dtype} {list(x.shape)}")

    def embed(self, tokens: torch.Tensor) -> torch.Tensor:
        tokens = tokens.to(device=f"cuda:{self.device}", dtype=torch.int32).contiguous()
        out = torch.empty(tokens.numel(), self.cfg.hidden_size, dtype=self.dtype,
                          device=tokens.device)
        call("dial_b200_embed", self._h, C.c_void_p(tokens.data_ptr()), tokens.numel(),
             C.c_void_p(out.data_ptr()), self._stream_ptr())
        return out

    def head(self, hidden: torch.Tensor, return_logits: bool = False):
        self._check_hidden(hidden)
        rows = hidden.numel() // self.cfg.hidden_size
        toks = torch.empty(rows, dtype=torch.int32, device=hidden.device)
        logits = torch.empty(rows, self.cfg.vocab_size, dtype=self.dtype, device=hidden.device) \
            if return_logits else None
        call("dial_b200_head", self._h, C.c_void_p(hidden.data_ptr()), rows,
             C.c_void_p(logits.data_ptr() if logits is not None else 0),
             C.c_void_p(toks.data_ptr()), self._stream_ptr())
        return (toks, logits) if return_logits else toks

    # ---------------------------------------------------------- end to end
    def decode_step(self, tokens, sids, positions) -> np.ndarray:
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        s = np.ascontiguousarray(np.asarray(sids, dtype=np.int32))
        p = np.ascontiguousarray(np.asarray(positions, dtype=np.int32))
        out = np.empty_like(t)
        call("dial_b200_decode_step", self._h, t.size, _np_ptr(t), _np_ptr(s), _np_ptr(p),
             _np_ptr(out))
        return out

    def generate(self, prompt, n_gen: int, session: int = 0):
        pr = np.ascontiguousarray(np.asarray(prompt, dtype=np.int32))
        out = np.empty(n_gen, dtype=np.int32)
        ttft, dec = C.c_double(), C.c_double()
        call("dial_b200_generate", self._h, session, _np_ptr(pr), pr.size, n_gen, _np_ptr(out),
             C.byref(ttft), C.byref(dec))
        return out, ttft.value, dec.value

    def loop_prepare(self, tokens, sids, positions):
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        s = np.ascontiguousarray(np.asarray(sids, dtype=np.int32))
        p = np.ascontiguousarray(np.asarray(positions, dtype=np.int32))
        call("dial_b200_decode_loop_prepare", self._h, t.size, _np_ptr(t), _np_ptr(s), _np_ptr(p))
        return t.size

    def loop_run(self, rows: int, n_steps: int):
        call("dial_b200_decode_loop_run", self._h, rows, n_steps)

    def loop_state(self, rows: int):
        t = np.empty(rows, dtype=np.int32)
        p = np.empty(rows, dtype=np.int32)
        call("dial_b200_decode_loop_state", self._h, rows, _np_ptr(t), _np_ptr(p))
        return t, p

    def stage_prepare(self, sids, positions):
        """Set the decode rows' sessions/positions on the device for stage_step."""
        s = np.ascontiguousarray(np.asarray(sids, dtype=np.int32))
        p = np.ascontiguousarray(np.asarray(positions, dtype=np.int32))
        call("dial_b200_stage_prepare", self._h, s.size, _np_ptr(s), _np_ptr(p))

    def stage_step(self, rows: int, tokens: torch.Tensor | None, hidden: torch.Tensor,
                   tokens_out: torch.Tensor | None = None):
        """One graph-captured decode step of this engine's stage on the current
        stream (embed if it owns the embedding, head + argmax if it owns the
        head); positions advance on the device."""
        self._check_hidden(hidden)
        ptr = lambda t: C.c_void_p(t.data_ptr() if t is not None else 0)  # noqa: E731
        call("dial_b200_stage_step", self._h, rows, ptr(tokens), ptr(hidden), ptr(tokens_out),
             self._stream_ptr())

    def stage_step_rows(self, row_offset: int, rows: int, tokens: torch.Tensor | None,
                        hidden: torch.Tensor, tokens_out: torch.Tensor | None = None):
        """stage_step for the prepared rows [row_offset, row_offset + rows) (one
        micro-batch of the sessions given to stage_prepare)."""
        self._check_hidden(hidden)
        ptr = lambda t: C.c_void_p(t.data_ptr() if t is not None else 0)  # noqa: E731
        call("dial_b200_stage_step_rows", self._h, row_offset, rows, ptr(tokens), ptr(hidden),
             ptr(tokens_out), self._stream_ptr())

    # ------------------------------------------------------ stage link (peer memory)
    def stage_link_handle(self) -> bytes:
        """64-byte CUDA IPC handle of this stage's inbox (allocated on first use)."""
        buf = (C.c_char * 64)()
        call("dial_b200_stage_link_handle", self._h, C.cast(buf, C.c_void_p))
        return bytes(buf)

    def stage_link_open(self, next_handle: bytes | None, first_handle: bytes | None):
        """Map the next stage's inbox (all but the last stage) and the first
        stage's inbox (the last stage)."""
        nb = C.create_string_buffer(next_handle, 64) if next_handle else None
        fb = C.create_string_buffer(first_handle, 64) if first_handle else None
        call("dial_b200_stage_link_open", self._h, C.cast(nb, C.c_void_p) if nb else None,
             C.cast(fb, C.c_void_p) if fb else None)

    def stage_link_step(self, rows: int, tokens: torch.Tensor | None = None):
        """One linked decode step of this stage on the current stream; the first
        stage passes the tokens on the first step of a run, None after it."""
        call("dial_b200_stage_link_step", self._h, rows,
             C.c_void_p(tokens.data_ptr() if tokens is not None else 0), self._stream_ptr())

    def stage_link_finish(self, rows: int) -> np.ndarray:
        """First stage: receive the last step's tokens (synchronizes)."""
        out = np.empty(rows, dtype=np.int32)
        call("dial_b200_stage_link_finish", self._h, rows, _np_ptr(out), self._stream_ptr())
        return out

    def session_fill_random(self, session: int, length: int, seed: int, std: float = 1.0):
        call("dial_b200_session_fill_random", self._h, session, length, seed,
             _np_ptr(normal_table_bits(std)))

    def step_kernel_count(self, rows: int) -> int:
        return int(lib.dial_b200_step_kernel_count(self._h, rows))

    def prefill_kernel_count(self, n_prompt: int) -> int:
        return int(lib.dial_b200_prefill_kernel_count(self._h, n_prompt))

    def linear_replay(self, layer: int, which: int, rows: int, iters: int):
        call("dial_b200_engine_linear_replay", self._h, layer, which, rows, iters)

    def linear_bytes(self, layer: int, which: int, rows: int) -> int:
        return int(lib.dial_b200_engine_linear_bytes(self._h, layer, which, rows))


def device_status(clear: bool = False) -> int:
    v = C.c_int()
    call("dial_b200_device_status", C.byref(v), int(clear))
    return v.value
