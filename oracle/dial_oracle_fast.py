"""ctypes binding of the C++/OpenMP oracle (oracle/dial_oracle_c.cpp) --
TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py``
use this module; the product path never does.  It runs the same algorithm as
``dial_oracle.py`` (same synthetic weights, same rounding points, see the C++
file's header for the reference file:line of every function) fast enough for
the full Qwen3-8B-shape model: 36 layers, hidden 4096, vocab 151936.

``accum=64`` sums the matmuls in f64 (order-independent for bf16 x int8 / bf16
products, so results equal ``dial_oracle.py``'s); ``accum=32`` sums in f32
(the reference kernels' accumulation), used when the library is timed as the
CPU baseline.
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

import dial_oracle as O

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libdial_oracle_c.so"

FMT_W8A16, FMT_FP8_BLOCK128, FMT_NVFP4, FMT_DENSE = 0, 1, 3, 4


class _Cfg(C.Structure):
    _fields_ = [("hidden", C.c_int32), ("inter", C.c_int32), ("vocab", C.c_int32),
                ("layers", C.c_int32), ("heads", C.c_int32), ("kv_heads", C.c_int32),
                ("eps", C.c_float), ("rope_theta", C.c_float), ("max_seq_len", C.c_int32),
                ("fmt", C.c_int32)]


_lib = None


def lib() -> C.CDLL:
    """Load (building with ``make -C oracle`` when missing) the oracle library."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        subprocess.run(["make", "-C", str(HERE)], check=True, capture_output=True)
    L = C.CDLL(str(LIB_PATH))
    P, I32, I64, F, U64 = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_uint64
    sig = {
        "orc_last_error": (C.c_char_p, []),
        "orc_set_threads": (None, [I32]),
        "orc_get_threads": (I32, []),
        "orc_model_new": (P, [C.POINTER(_Cfg), I32, I32, I32, I32]),
        "orc_model_free": (None, [P]),
        "orc_model_synth": (I32, [P, U64, P]),
        "orc_set_w8a16": (I32, [P, I32, I32, P, P, I64, I64]),
        "orc_set_norm": (I32, [P, I32, I32, P, I64]),
        "orc_cache_new": (P, [P]),
        "orc_cache_free": (None, [P]),
        "orc_cache_fill_random": (I32, [P, P, I32, I32, U64, P]),
        "orc_cache_len": (I32, [P, I32]),
        "orc_cache_read": (I32, [P, I32, I32, I32, P]),
        "orc_embed": (I32, [P, P, I32, P]),
        "orc_forward": (I32, [P, P, P, I32, I32, I32, I32, I32, I32, P]),
        "orc_logits": (I32, [P, P, I32, P, I32]),
        "orc_linear": (I32, [I32, P, P, F, I64, I64, P, I64, P, I32]),
        "orc_quantize_w8a16": (I32, [P, I64, I64, P, P]),
        "orc_synth_normal": (I32, [U64, U64, I64, P, P]),
        "orc_quantize_fp8_block128": (I32, [P, I64, I64, P, P]),
        "orc_quantize_nvfp4": (I32, [P, I64, I64, P, P, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    threads = int(os.environ.get("DIAL_ORACLE_THREADS", "0"))
    if threads > 0:
        L.orc_set_threads(threads)
    _lib = L
    return L


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def _check(rc: int) -> None:
    if rc != 0:
        raise RuntimeError(lib().orc_last_error().decode())


def threads() -> int:
    return lib().orc_get_threads()


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def _table(std: float = 0.02) -> np.ndarray:
    return np.ascontiguousarray(O.normal_table(std), dtype=np.float32)


def linear(fmt: int, codes, scales, x, out_dim: int, in_dim: int, global_scale: float = 1.0,
           accum: int = 64) -> np.ndarray:
    """y [M, out] = act(...) of one linear in the given format (see orc_linear)."""
    x = np.ascontiguousarray(np.asarray(x, np.float32).reshape(-1, in_dim))
    y = np.empty((x.shape[0], out_dim), np.float32)
    codes = np.ascontiguousarray(codes)
    scales = np.ascontiguousarray(scales)
    _check(lib().orc_linear(fmt, _ptr(codes), _ptr(scales), float(global_scale), out_dim, in_dim,
                            _ptr(x), x.shape[0], _ptr(y), accum))
    return y


def w8a16_linear(x, q, scale, accum: int = 64) -> np.ndarray:
    """dial_oracle.w8a16_linear (bf16 activations) for large shapes."""
    q = np.ascontiguousarray(q, dtype=np.int8)
    return linear(FMT_W8A16, q, np.asarray(scale, np.float32), x, q.shape[0], q.shape[1],
                  accum=accum)


def quantize_w8a16_rows(w) -> tuple[np.ndarray, np.ndarray]:
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    q = np.empty((n, k), np.int8)
    s = np.empty(n, np.float32)
    _check(lib().orc_quantize_w8a16(_ptr(w), n, k, _ptr(q), _ptr(s)))
    return q, s


def synth_normal(seed: int, stream: int, n: int, std: float = 0.02) -> np.ndarray:
    out = np.empty(n, np.float32)
    t = _table(std)
    _check(lib().orc_synth_normal(seed, stream, n, _ptr(t), _ptr(out)))
    return out


def quantize_fp8_block128(w):
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    codes = np.empty((n, k), np.uint8)
    sc = np.empty((-(-n // 128), -(-k // 128)), np.float32)
    _check(lib().orc_quantize_fp8_block128(_ptr(w), n, k, _ptr(codes), _ptr(sc)))
    return codes, sc


def quantize_nvfp4(w):
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    packed = np.empty(n * k // 2, np.uint8)
    sc = np.empty(n * k // 16, np.uint8)
    gs = np.zeros(1, np.float32)
    _check(lib().orc_quantize_nvfp4(_ptr(w), n, k, _ptr(packed), _ptr(sc), _ptr(gs)))
    return packed, sc, float(gs[0])


class Cache:
    """One session's KV cache for the model's layers (cache.rs:117-237)."""

    def __init__(self, model: "FastModel"):
        self.model = model
        self.h = lib().orc_cache_new(model.h)

    def fill_random(self, session: int, length: int, seed: int, std: float = 1.0) -> None:
        """Mirror of dial_b200_session_fill_random's values for this session."""
        t = _table(std)
        _check(lib().orc_cache_fill_random(self.model.h, self.h, session, length, seed, _ptr(t)))

    def length(self, layer: int) -> int:
        return lib().orc_cache_len(self.h, layer)

    def read(self, layer: int, which: int, n: int) -> np.ndarray:
        cfg = self.model.cfg
        out = np.empty((cfg.kv_heads, n, cfg.head_dim), np.float32)
        _check(lib().orc_cache_read(self.h, layer, which, n, _ptr(out)))
        return out

    def __del__(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.orc_cache_free(self.h)
            self.h = None


class FastModel:
    """Decoder stack (or a layer range of it) with seeded synthetic weights.

    ``cfg`` is a ``dial_oracle.ModelConfig``; ``fmt`` the layer-linear format
    (FMT_W8A16, FMT_FP8_BLOCK128, FMT_NVFP4 or FMT_DENSE).  The weights are the
    ones ``dial_oracle.synth_model`` and the engine's
    ``dial_b200_engine_load_synthetic`` generate for the same seed.
    """

    def __init__(self, cfg: O.ModelConfig, seed: int | None = 0, fmt: int = FMT_W8A16,
                 first_layer: int = 0, num_layers: int | None = None, has_embed: bool = True,
                 has_head: bool = True, std: float = 0.02):
        self.cfg = cfg
        self.first = first_layer
        self.count = cfg.layers - first_layer if num_layers is None else num_layers
        c = _Cfg(cfg.hidden, cfg.inter, cfg.vocab, cfg.layers, cfg.heads, cfg.kv_heads, cfg.eps,
                 cfg.rope_theta, cfg.max_seq_len, fmt)
        self.h = lib().orc_model_new(C.byref(c), first_layer, self.count, int(has_embed),
                                     int(has_head))
        if seed is not None:
            t = _table(std)
            _check(lib().orc_model_synth(self.h, seed, _ptr(t)))

    def set_layer_w8a16(self, layer: int, lw: O.LayerWeights) -> None:
        """Explicit W8A16 weights of one layer (a dial_oracle.LayerWeights)."""
        for which, (q, s) in enumerate([(lw.qkv_q, lw.qkv_s), (lw.o_q, lw.o_s),
                                        (lw.gate_up_q, lw.gate_up_s), (lw.down_q, lw.down_s)]):
            q = np.ascontiguousarray(q, np.int8)
            s = np.ascontiguousarray(s, np.float32)
            _check(lib().orc_set_w8a16(self.h, layer, which, _ptr(q), _ptr(s), q.shape[0],
                                       q.shape[1]))
        for which, w in enumerate([lw.input_norm, lw.post_norm, lw.q_norm, lw.k_norm]):
            w = np.ascontiguousarray(w, np.float32)
            _check(lib().orc_set_norm(self.h, layer, which, _ptr(w), w.size))

    def new_cache(self) -> Cache:
        return Cache(self)

    def embed(self, tokens) -> np.ndarray:
        t = np.ascontiguousarray(np.asarray(tokens, np.int32).reshape(-1))
        out = np.empty((t.size, self.cfg.hidden), np.float32)
        _check(lib().orc_embed(self.h, _ptr(t), t.size, _ptr(out)))
        return out

    def forward(self, hidden: np.ndarray, cache: Cache, index_pos: int, first: int | None = None,
                count: int | None = None, capture: bool = False, accum: int = 64,
                round_probs: bool = True):
        """Layers [first, first+count) on hidden [S, H] (updated in place).
        With ``capture`` returns the hidden state after each layer [count, S, H]."""
        assert hidden.dtype == np.float32 and hidden.flags.c_contiguous
        first = self.first if first is None else first
        count = self.first + self.count - first if count is None else count
        S = hidden.shape[0]
        cap = np.empty((count, S, self.cfg.hidden), np.float32) if capture else None
        _check(lib().orc_forward(self.h, cache.h, _ptr(hidden), S, index_pos, first, count, accum,
                                 int(round_probs), _ptr(cap) if capture else None))
        return cap

    def logits(self, hidden_rows, accum: int = 64) -> np.ndarray:
        h = np.ascontiguousarray(np.asarray(hidden_rows, np.float32).reshape(-1, self.cfg.hidden))
        out = np.empty((h.shape[0], self.cfg.vocab), np.float32)
        _check(lib().orc_logits(self.h, _ptr(h), h.shape[0], _ptr(out), accum))
        return out

    def generate(self, prompt, n_gen: int, forced=None, capture_layers=(), capture_steps=(0,),
                 accum: int = 64, round_probs: bool = True, topk: int = 8):
        """Greedy generation (Master::generate, qwen3_vl.rs:3276-3331 with the
        device argmax of qwen3_vl.rs:138-143, first index among ties).

        Returns a dict: ``tokens`` [n_gen]; ``top_ids`` / ``top_logits``
        [n_gen, topk] (descending, ties by index); ``margin`` [n_gen] (top-1
        minus top-2 logit); ``hidden`` {(step, layer): rows} for the steps in
        ``capture_steps`` (0 = the prefill, all prompt rows) and the layers in
        ``capture_layers``.  With ``forced`` the input of step i >= 1 is
        ``forced[i-1]`` (teacher forcing).
        """
        cache = self.new_cache()
        caps = {}
        toks, top_ids, top_lg, margins = [], [], [], []
        inp = list(np.asarray(prompt).tolist())
        pos = 0
        for step in range(n_gen):
            x = self.embed(inp)
            want = bool(capture_layers) and step in capture_steps
            cap = self.forward(x, cache, pos, capture=want, accum=accum, round_probs=round_probs)
            if want:
                for l in capture_layers:
                    caps[(step, l)] = cap[l - self.first].copy()
            lg = self.logits(x[-1], accum=accum)[0]
            order = np.lexsort((np.arange(lg.size), -lg))[:topk]
            top_ids.append(order)
            top_lg.append(lg[order])
            margins.append(float(lg[order[0]] - lg[order[1]]))
            toks.append(int(order[0]))
            pos += len(inp)
            nxt = toks[-1] if forced is None else int(forced[step])
            inp = [nxt]
        return {"tokens": np.array(toks, np.int64), "top_ids": np.array(top_ids),
                "top_logits": np.array(top_lg, np.float32), "margin": np.array(margins),
                "hidden": caps}

    def __del__(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.orc_model_free(self.h)
            self.h = None
