"""A small many-row decode case for profiler captures of the decode attention
of BASELINE config 4: 32 sessions with KV lengths uniform in [128, 8192]
(seed 2, the bench's draw) in 16-token pages, `layers` Qwen3-8B-shape W8A16
layers, `iters` batched decode steps (dial_b200_batch_decode_forward).

    PYTHONPATH=dial-27b_b200 python -m dial_b200.ragged_case [--layers 2] [--iters 4]
"""

from __future__ import annotations

import argparse
import json
import time

import numpy as np
import torch

from .engine import Config, Engine, device_status


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=2)
    ap.add_argument("--iters", type=int, default=4)
    args = ap.parse_args(argv)
    torch.cuda.set_device(0)
    n = 32
    lengths = np.random.default_rng(2).integers(128, 8193, size=n).astype(np.int32)
    cfg = Config(num_hidden_layers=args.layers, max_seq_len=8192 + args.iters + 16,
                 max_sessions=n, max_tokens=64)
    eng = Engine(cfg, has_embed=False, has_head=False)
    eng.load_synthetic(seed=0)
    for s in range(n):
        eng.session_fill_random(s, int(lengths[s]), seed=2 + s)
    x = torch.randn(n, cfg.hidden_size, generator=torch.Generator().manual_seed(3)).to(
        "cuda", torch.bfloat16)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(args.iters):
        eng.batch_decode(x, np.arange(n), lengths + i)
    torch.cuda.synchronize()
    print(json.dumps({"sessions": n, "layers": args.layers, "iters": args.iters,
                      "kv_tokens": int(lengths.sum()),
                      "ms_per_iter": (time.perf_counter() - t0) * 1e3 / args.iters,
                      "device_status": device_status()}), flush=True)


if __name__ == "__main__":
    main()
