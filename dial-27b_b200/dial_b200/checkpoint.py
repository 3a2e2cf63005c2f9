"""Safetensors checkpoints into an :class:`Engine`.

Covers the text decoder of Qwen3 (``model.layers.*``) and Qwen3-VL
(``model.language_model.layers.*``, qwen3_vl/qwen3_vl.rs:3089-3172), with each
projection stored as one of the forms the reference loads
(qwen3_8/quant.rs:448-501, checked in this order):

* compressed-tensors NVFP4: ``weight_packed`` (u8 [out, in/2], even k in the
  low nibble), ``weight_scale`` (e4m3 [out, in/16]) and ``weight_global_scale``
  (one f32 quantisation divisor; the dequant multiplier is its reciprocal,
  quant.rs:304-311, 376-399);
* ModelOpt NVFP4: ``weight`` packed as above, ``weight_scale``, and
  ``weight_scale_2`` (one f32 multiplier);
* FP8 e4m3: ``weight`` + ``weight_scale`` with one value or one per output row
  (quant.rs:316-345, 406-429); a [ceil(out/128), ceil(in/128)] scale is taken
  as 128 x 128 block scales (the 27B-class format of this build);
* dense ``weight``: quantised to W8A16 at load, as the reference's W8A16
  worker does (worker_w8a16.rs:302-366).

The engine's linears are fused (q|k|v rows, gate|up rows,
qwen3_vl/text.rs:1428-1431, 634-636), so the projections of one fused linear
must share a form (and NVFP4 one global scale).  The embedding, the final
norm and the lm_head (``lm_head.weight``, then
``model.language_model.lm_head.weight``, then the tied embedding when the
config says so, qwen3_vl.rs:3099-3127) load on the engines that own them.
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path
from typing import Callable

import numpy as np
import torch

from . import _abi
from ._abi import DialError
from .engine import Config, Engine

_BLOCK = 128


def _err(msg: str) -> DialError:
    return DialError(_abi.DIAL_ERR_INVALID, msg)


class Checkpoint:
    """Tensors of one ``.safetensors`` file, or of every shard of a directory
    (``model.safetensors.index.json`` when present), read lazily on the host."""

    def __init__(self, path: str | Path):
        from safetensors import safe_open

        path = Path(path)
        self.dir = path if path.is_dir() else path.parent
        if path.is_dir():
            index = path / "model.safetensors.index.json"
            if index.exists():
                shards = sorted(set(json.loads(index.read_text())["weight_map"].values()))
                files = [path / f for f in shards]
            else:
                files = sorted(path.glob("*.safetensors"))
        else:
            files = [path]
        if not files:
            raise _err(f"no safetensors file under {path}")
        self._where: dict[str, object] = {}
        self._handles = []
        for f in files:
            h = safe_open(str(f), framework="pt")
            self._handles.append(h)
            for k in h.keys():
                self._where[k] = h

    def has(self, name: str) -> bool:
        return name in self._where

    def get(self, name: str) -> torch.Tensor:
        if name not in self._where:
            raise _err(f"tensor {name} not found in the checkpoint")
        return self._where[name].get_tensor(name)

    def names(self) -> list[str]:
        return sorted(self._where)

    def config(self) -> dict:
        """config.json beside the tensors (text_config of a Qwen3-VL config)."""
        p = self.dir / "config.json"
        if not p.exists():
            return {}
        cfg = json.loads(p.read_text())
        text = dict(cfg.get("text_config", {}))
        for k, v in cfg.items():
            text.setdefault(k, v)
        return text


@dataclass
class LinearSpec:
    """One projection in an engine weight format (see Engine.set_linear)."""
    fmt: int
    codes: np.ndarray            # int8 / u8 codes ([out, in] or NVFP4 [out, in/2])
    scales: np.ndarray | None    # f32 rows / blocks, or e4m3 group codes (NVFP4)
    global_scale: float = 0.0
    out_dim: int = 0
    in_dim: int = 0


def _u8(t: torch.Tensor) -> np.ndarray:
    """Packed bytes (NVFP4 ``weight_packed``): one-byte tensors are viewed as
    u8; a wider integer tensor holding byte values is narrowed."""
    t = t.detach().cpu().contiguous()
    if t.dtype != torch.uint8:
        t = t.view(torch.uint8) if t.element_size() == 1 else t.to(torch.uint8)
    return t.numpy()


def _e4m3_codes(t: torch.Tensor, name: str) -> np.ndarray:
    """e4m3 codes of an FP8 weight or NVFP4 group-scale tensor.  One-byte
    tensors (float8_e4m3fn or u8) are the codes themselves, bit for bit
    (quant.rs:528-544); a wider float tensor holds e4m3 values, as in the
    reference's loader tests (quant.rs:547-601, where f32 tensors carry them),
    and is converted to the code of each value, which must be exact."""
    t = t.detach().cpu().contiguous()
    if t.element_size() == 1:
        return t.view(torch.uint8).numpy()
    if not t.dtype.is_floating_point:
        raise _err(f"{name}: expected e4m3 codes or values, got {t.dtype}")
    v = t.to(torch.float32)
    codes = v.to(torch.float8_e4m3fn)
    back = codes.to(torch.float32)
    if not torch.equal(back, v):
        bad = int(torch.nonzero(back != v)[0, 0]) if v.ndim == 1 else int(
            torch.nonzero((back != v).reshape(-1))[0, 0])
        raise _err(f"{name}: value {float(v.reshape(-1)[bad])} is not an e4m3 value")
    return codes.view(torch.uint8).numpy()


def _f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().to(torch.float32).contiguous().numpy()


def _global(ck: Checkpoint, name: str, invert: bool) -> float:
    g = _f32(ck.get(name)).reshape(-1)
    if g.size != 1 or g[0] == 0.0:
        raise _err(f"{name} must contain one non-zero value, got {g.tolist()}")
    return float(1.0 / g[0]) if invert else float(g[0])


def read_linear(ck: Checkpoint, prefix: str, in_dim: int, out_dim: int,
                quantize: Callable[[torch.Tensor], tuple[np.ndarray, np.ndarray]]) -> LinearSpec:
    """The projection ``prefix`` in the form the reference would load it."""
    p = prefix + "."
    if ck.has(p + "weight_packed") and ck.has(p + "weight_global_scale"):
        packed, glob = p + "weight_packed", _global(ck, p + "weight_global_scale", True)
    elif ck.has(p + "weight_scale_2"):
        packed, glob = p + "weight", _global(ck, p + "weight_scale_2", False)
    else:
        packed = None
    if packed is not None:
        if in_dim % 16:
            raise _err(f"{prefix}: NVFP4 needs in_dim % 16 == 0, got {in_dim}")
        codes = _u8(ck.get(packed)).reshape(-1)
        sc = _e4m3_codes(ck.get(p + "weight_scale"), p + "weight_scale").reshape(-1)
        if codes.size != out_dim * in_dim // 2 or sc.size != out_dim * in_dim // 16:
            raise _err(f"{prefix}: NVFP4 tensors do not match [{out_dim}, {in_dim}]")
        return LinearSpec(_abi.FMT_NVFP4_G16, codes.reshape(out_dim, in_dim // 2),
                          sc.reshape(out_dim, in_dim // 16), glob, out_dim, in_dim)
    if ck.has(p + "weight_scale"):
        codes = _e4m3_codes(ck.get(p + "weight"), p + "weight").reshape(-1)
        if codes.size != out_dim * in_dim:
            raise _err(f"{prefix}: FP8 weight does not match [{out_dim}, {in_dim}]")
        sc = _f32(ck.get(p + "weight_scale"))
        nbr, nbc = -(-out_dim // _BLOCK), -(-in_dim // _BLOCK)
        if sc.size == 1 or (sc.size == out_dim and sc.shape != (nbr, nbc)):
            rows = np.full(out_dim, sc.reshape(-1)[0], np.float32) if sc.size == 1 \
                else sc.reshape(-1).astype(np.float32)
            return LinearSpec(_abi.FMT_FP8_ROW, codes.reshape(out_dim, in_dim), rows, 0.0,
                              out_dim, in_dim)
        if sc.size == nbr * nbc:
            return LinearSpec(_abi.FMT_FP8_BLOCK128, codes.reshape(out_dim, in_dim),
                              sc.reshape(nbr, nbc).astype(np.float32), 0.0, out_dim, in_dim)
        raise _err(f"FP8 weight_scale for {prefix} contains {sc.size} values, "
                   f"expected 1, {out_dim} or {nbr}x{nbc}")
    w = ck.get(p + "weight")
    if tuple(w.shape) != (out_dim, in_dim):
        raise _err(f"{prefix}.weight has shape {tuple(w.shape)}, expected [{out_dim}, {in_dim}]")
    q, s = quantize(w)
    return LinearSpec(_abi.FMT_W8A16_ROW, np.asarray(q, np.int8), np.asarray(s, np.float32),
                      0.0, out_dim, in_dim)


def fuse_rows(name: str, parts: list[LinearSpec]) -> LinearSpec:
    """Stack projections along the output rows (one engine linear)."""
    fmt = parts[0].fmt
    if any(p.fmt != fmt for p in parts):
        raise _err(f"{name}: the fused projections are stored in different formats")
    out_dim = sum(p.out_dim for p in parts)
    in_dim = parts[0].in_dim
    codes = np.concatenate([p.codes for p in parts], axis=0)
    glob = parts[0].global_scale
    if fmt == _abi.FMT_NVFP4_G16:
        if any(p.global_scale != glob for p in parts):
            raise _err(f"{name}: NVFP4 projections with different global scales cannot share "
                       f"one linear")
    if fmt == _abi.FMT_FP8_BLOCK128 and any(p.out_dim % _BLOCK for p in parts[:-1]):
        raise _err(f"{name}: block-scaled rows must split at multiples of {_BLOCK}")
    scales = np.concatenate([p.scales for p in parts], axis=0)
    return LinearSpec(fmt, codes, scales, glob, out_dim, in_dim)


def _prefix(ck: Checkpoint) -> str:
    for p in ("model.language_model.", "model."):
        if ck.has(p + "embed_tokens.weight") or ck.has(p + "layers.0.input_layernorm.weight") \
                or any(n.startswith(p + "layers.") for n in ck.names()):
            return p
    raise _err("no Qwen3 text-decoder tensors (model.layers.* or model.language_model.layers.*)")


def config_from_checkpoint(path: str | Path, **overrides) -> Config:
    """Engine Config from config.json (Qwen3 or the text_config of Qwen3-VL)."""
    c = Checkpoint(path).config()
    if not c:
        raise _err(f"no config.json beside {path}")
    kw = dict(hidden_size=c["hidden_size"], intermediate_size=c["intermediate_size"],
              vocab_size=c["vocab_size"], num_hidden_layers=c["num_hidden_layers"],
              num_attention_heads=c["num_attention_heads"],
              num_key_value_heads=c.get("num_key_value_heads", c["num_attention_heads"]),
              rms_norm_eps=c.get("rms_norm_eps", 1e-6), rope_theta=c.get("rope_theta", 10000.0))
    head_dim = c.get("head_dim", kw["hidden_size"] // kw["num_attention_heads"])
    if head_dim * kw["num_attention_heads"] != kw["hidden_size"] or head_dim != 128:
        raise _err(f"head_dim {head_dim} with {kw['num_attention_heads']} heads and hidden "
                   f"{kw['hidden_size']} is not supported (128 and heads x 128 == hidden)")
    kw.update(overrides)
    return Config(**kw)


def _act_values(t: torch.Tensor, act: int) -> np.ndarray:
    """Activation-dtype bit patterns of a tensor (exact when the dtypes agree)."""
    want = torch.bfloat16 if act == _abi.ACT_BF16 else torch.float16
    t = t.detach().cpu().contiguous()
    if t.dtype != want:
        t = t.to(torch.float32).to(want)
    return t.view(torch.int16).numpy().view(np.uint16)


def load_checkpoint(engine: Engine, path: str | Path,
                    quantize: Callable | None = None) -> None:
    """Install the layers, norms, embedding and head this engine owns.

    ``quantize`` turns a dense [out, in] weight into (int8 codes, f32 row
    scales); by default the device quantizer of this library
    (:func:`dial_b200.w8a16_quantize`, worker_w8a16.rs:330-341)."""
    if quantize is None:
        from .linear import w8a16_quantize
        quantize = w8a16_quantize
    ck = Checkpoint(path)
    cfg = engine.cfg
    pre = _prefix(ck)
    H, I, D = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    QH, KVH = cfg.num_attention_heads, cfg.num_key_value_heads
    act = cfg.act

    def put_linear(layer: int, which: int, spec: LinearSpec):
        engine.set_linear(layer, which, spec.fmt, spec.codes, spec.scales, spec.global_scale)

    for layer in range(engine.first_layer, engine.first_layer + engine.num_layers):
        lp = f"{pre}layers.{layer}."
        att, mlp = lp + "self_attn.", lp + "mlp."
        qkv = fuse_rows(att + "qkv", [read_linear(ck, att + "q_proj", H, QH * D, quantize),
                                      read_linear(ck, att + "k_proj", H, KVH * D, quantize),
                                      read_linear(ck, att + "v_proj", H, KVH * D, quantize)])
        put_linear(layer, Engine.LINEAR_QKV, qkv)
        put_linear(layer, Engine.LINEAR_O, read_linear(ck, att + "o_proj", QH * D, H, quantize))
        gu = fuse_rows(mlp + "gate_up", [read_linear(ck, mlp + "gate_proj", H, I, quantize),
                                         read_linear(ck, mlp + "up_proj", H, I, quantize)])
        put_linear(layer, Engine.LINEAR_GATE_UP, gu)
        put_linear(layer, Engine.LINEAR_DOWN, read_linear(ck, mlp + "down_proj", I, H, quantize))
        engine.set_tensor(layer, Engine.T_INPUT_NORM,
                          _act_values(ck.get(lp + "input_layernorm.weight"), act))
        engine.set_tensor(layer, Engine.T_POST_NORM,
                          _act_values(ck.get(lp + "post_attention_layernorm.weight"), act))
        engine.set_tensor(layer, Engine.T_Q_NORM, _act_values(ck.get(att + "q_norm.weight"), act))
        engine.set_tensor(layer, Engine.T_K_NORM, _act_values(ck.get(att + "k_norm.weight"), act))
    if engine.has_embed:
        engine.set_tensor(0, Engine.T_EMBED, _act_values(ck.get(pre + "embed_tokens.weight"), act))
    if engine.has_head:
        engine.set_tensor(0, Engine.T_FINAL_NORM, _act_values(ck.get(pre + "norm.weight"), act))
        for name in ("lm_head", pre + "lm_head"):
            if ck.has(name + ".weight"):
                head = ck.get(name + ".weight")
                if any(ck.has(name + "." + s) for s in ("weight_scale", "weight_packed")):
                    spec = read_linear(ck, name, H, cfg.vocab_size, quantize)
                    put_linear(0, Engine.LINEAR_LM_HEAD, spec)
                else:
                    engine.set_linear(0, Engine.LINEAR_LM_HEAD, _abi.FMT_DENSE,
                                      _act_values(head, act).reshape(cfg.vocab_size, H))
                break
        else:
            if not ck.config().get("tie_word_embeddings", False):
                raise _err("cannot find lm_head.weight (tried lm_head.weight and "
                           f"{pre}lm_head.weight) and the embeddings are not tied")
            engine.set_linear(0, Engine.LINEAR_LM_HEAD, _abi.FMT_DENSE,
                              _act_values(ck.get(pre + "embed_tokens.weight"), act)
                              .reshape(cfg.vocab_size, H))
