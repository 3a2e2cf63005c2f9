"""W8A16 linear microbenchmark over the Qwen3-8B projection shapes.

    PYTHONPATH=dial-27b_b200 python -m dial_b200.microbench [--shapes q,gate_up] [--M 1,4,16]
        [--iters 20] [--min-footprint-mb 512]
    PYTHONPATH=dial-27b_b200 python -m dial_b200.microbench --replay gate_up --layers 4 --M 1 \
        [--model 27b --fmt nvfp4]

Each case builds enough copies of the quantized weight that one rotation
through them streams more than the L2 cache (126 MB) from HBM, captures the
rotation of dial_b200_qlinear_forward calls in a CUDA graph, replays it and
times the replays with CUDA events on the launching stream.  One JSON line per
case: microseconds per forward, algorithmic bytes (int8 weights + f32 row
scales + bf16 activations in and out) and FLOPs (2*M*N*K), GB/s and TFLOP/s,
and the fraction of the measured HBM copy bandwidth.

Shapes follow the W8A16 linear microbench of the baseline: K x N =
4096x4096 (q/o), 4096x1024 (k/v), 4096x12288 (gate/up), 12288x4096 (down)
plus the fused 4096x6144 (QKV) and 4096x24576 (gate+up) layouts the decoder
uses (text.rs:1428-1432, 634-637).  Weights are int8 codes with per-row
scales drawn from a seeded generator: the kernel's speed does not depend on
the values.
"""

from __future__ import annotations

import argparse
import json
import math
from pathlib import Path

import numpy as np
import torch

from .linear import CudaW8A16Linear

SHAPES = {  # name: (K, N)
    "q": (4096, 4096),
    "kv": (4096, 1024),
    "gate": (4096, 12288),
    "down": (12288, 4096),
    "qkv": (4096, 6144),
    "gate_up": (4096, 24576),
}


def measured_hbm_gbs() -> tuple[float, str]:
    p = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def run_case(name: str, M: int, iters: int, min_footprint: int, device: int = 0) -> dict:
    K, N = SHAPES[name]
    rng = np.random.default_rng(10 + list(SHAPES).index(name))
    q = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    s = (rng.random(N, dtype=np.float32) * 1e-3 + 1e-4).astype(np.float32)
    wbytes = N * K + 4 * N
    copies = max(2, math.ceil(min_footprint / wbytes))
    lins = [CudaW8A16Linear.from_quantized(q, s, act=torch.bfloat16) for _ in range(copies)]
    dev = torch.device("cuda", device)
    x = torch.randn(M, K, generator=torch.Generator().manual_seed(20), dtype=torch.float32)
    x = x.to(dev, torch.bfloat16)
    for lin in lins:  # warm-up outside capture (first call per device sets up status memory)
        lin(x)
    torch.cuda.synchronize(dev)

    g = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        for lin in lins:
            lin(x)
        stream.synchronize()
        with torch.cuda.graph(g, stream=stream, capture_error_mode="thread_local"):
            outs = [lin(x) for lin in lins]
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize(dev)
    cur = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    for _ in range(iters):
        g.replay()
    e1.record(cur)
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / (iters * copies)
    del outs
    nbytes = lins[0].resident_bytes() + 2 * M * K + 2 * M * N
    flops = 2.0 * M * N * K
    peak, src = measured_hbm_gbs()
    gbs = nbytes / (us * 1e-6) / 1e9
    return {"shape": name, "K": K, "N": N, "M": M, "us": us, "bytes": nbytes, "GB_s": gbs,
            "frac_hbm": gbs / peak, "TFLOP_s": flops / (us * 1e-6) / 1e12, "copies": copies,
            "peak_gbs": peak, "peak_source": src,
            "l2": f"rotation over {copies} weight copies ({copies * wbytes / 2**20:.0f} MiB)"}


def run_prefill(n_prompt: int) -> dict:
    """Two prefills of n_prompt seeded tokens on the synthetic Qwen3-8B W8A16
    engine (the first loads kernels lazily); reports the second's TTFT and
    how many kernels one prefill launches (the tail of a profiler's launch
    list)."""
    from .engine import Config, Engine

    cfg = Config(max_seq_len=n_prompt + 64, max_sessions=1, max_tokens=n_prompt)
    eng = Engine(cfg, device=0)
    eng.load_synthetic(seed=0)
    prompt = np.random.default_rng(1).integers(0, cfg.vocab_size, n_prompt).astype(np.int32)
    eng.generate(prompt, 1)
    _, ttft, _ = eng.generate(prompt, 1)
    return {"prefill_tokens": n_prompt, "ttft_ms": ttft * 1e3,
            "launches_per_prefill": eng.prefill_kernel_count(n_prompt)}


LINEARS = {"qkv": 0, "o": 1, "gate_up": 2, "down": 3}


def run_replay(name: str, layers: int, rows: int, iters: int, model: str = "8b",
               fmt: str = "w8a16") -> dict:
    """One decode-step linear of the synthetic Qwen3-8B W8A16 engine (the
    epilogue the decode step uses: fused RMSNorm + SwiGLU for gate_up, RMSNorm
    for qkv, residual add for o and down) replayed `iters` times, rotating over
    `layers` layers so that no launch finds its weights in L2
    (dial_b200_engine_linear_replay).  A small device footprint for profiler
    captures of the exact kernel variant the decode step runs."""
    from . import _abi
    from .engine import Config, Engine

    fmts = {"w8a16": _abi.FMT_W8A16_ROW, "fp8": _abi.FMT_FP8_BLOCK128, "nvfp4": _abi.FMT_NVFP4_G16}
    base = Config.dense_27b if model == "27b" else Config
    cfg = base(num_hidden_layers=layers, max_seq_len=64, max_sessions=1,
               max_tokens=max(rows, 16), linear_fmt=fmts[fmt])
    eng = Engine(cfg, device=0, has_embed=False, has_head=False)
    eng.load_synthetic(seed=0)
    which = LINEARS[name]
    eng.linear_replay(-1, which, rows, 200)  # clocks up before timing
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(eng.stream)
    eng.linear_replay(-1, which, rows, iters)
    e1.record(eng.stream)
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / iters
    nbytes = eng.linear_bytes(0, which, rows)
    peak, src = measured_hbm_gbs()
    gbs = nbytes / (us * 1e-6) / 1e9
    return {"linear": name, "model": model, "fmt": fmt, "rows": rows, "layers": layers, "us": us,
            "bytes": nbytes,
            "GB_s": gbs, "frac_hbm": gbs / peak, "peak_gbs": peak, "peak_source": src}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", default=",".join(SHAPES))
    ap.add_argument("--M", default="1,4,16,128,2048")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--min-footprint-mb", type=int, default=512)
    ap.add_argument("--prefill", type=int, default=0,
                    help="instead: time a warmed prefill of this many tokens on the synthetic model")
    ap.add_argument("--replay", default="",
                    help="instead: replay one decode-step linear (qkv, o, gate_up, down) of a "
                         "--layers-layer synthetic engine, --M rows (first value)")
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--model", default="8b", choices=["8b", "27b"],
                    help="--replay: Qwen3-8B shapes or the 27B-class decoder's")
    ap.add_argument("--fmt", default="w8a16", choices=["w8a16", "fp8", "nvfp4"],
                    help="--replay: weight format of the engine's layer linears")
    args = ap.parse_args(argv)
    torch.cuda.set_device(0)
    if args.replay:
        rows = int(args.M.split(",")[0])
        print(json.dumps(run_replay(args.replay, args.layers, rows, args.iters, args.model,
                                    args.fmt)), flush=True)
        return
    if args.prefill > 0:
        print(json.dumps(run_prefill(args.prefill)), flush=True)
        return
    for name in args.shapes.split(","):
        for M in (int(m) for m in args.M.split(",")):
            r = run_case(name, M, args.iters, args.min_footprint_mb << 20)
            print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
