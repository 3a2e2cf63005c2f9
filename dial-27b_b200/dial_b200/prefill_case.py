"""A small prefill case for profiler captures of BASELINE config 3's prompt
pass: one `length`-token prompt (default 2048) through `layers` Qwen3-8B-shape
W8A16 decoder layers (the tcgen05 GEMMs and the tensor-core prefill
attention), `iters` times, with no embedding or head.

    PYTHONPATH=dial-27b_b200 python -m dial_b200.prefill_case [--layers 2] [--length 2048] [--iters 3]
"""

from __future__ import annotations

import argparse
import json
import time

import torch

from .engine import Config, Engine, device_status


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=2)
    ap.add_argument("--length", type=int, default=2048)
    ap.add_argument("--iters", type=int, default=3)
    args = ap.parse_args(argv)
    torch.cuda.set_device(0)
    cfg = Config(num_hidden_layers=args.layers, max_seq_len=args.length + 16, max_sessions=1,
                 max_tokens=args.length)
    eng = Engine(cfg, has_embed=False, has_head=False)
    eng.load_synthetic(seed=0)
    x0 = torch.randn(args.length, cfg.hidden_size, generator=torch.Generator().manual_seed(3)).to(
        "cuda", torch.bfloat16)
    times = []
    for _ in range(args.iters):
        x = x0.clone()
        eng.session_reset(0)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        eng.forward_local_batch(x, [(f"model.layers.{i}", 0, i) for i in range(args.layers)])
        torch.cuda.synchronize()
        times.append((time.perf_counter() - t0) * 1e3)
    print(json.dumps({"layers": args.layers, "tokens": args.length, "iters": args.iters,
                      "ms_last": times[-1], "device_status": device_status()}), flush=True)


if __name__ == "__main__":
    main()
