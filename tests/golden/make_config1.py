"""Writes tests/golden/config1_qwen3_8b_w8a16.npz: the oracle's greedy decode of
the headline workload, used by the full-size parity test
and by bench.py's token check.

    python tests/golden/make_config1.py        (about 3 minutes on 8 cores)

Model: Qwen3-8B architecture (36 layers, hidden 4096, 32 q / 8 kv heads,
head_dim 128, FFN 12288, vocab 151936, RMSNorm eps 1e-6, RoPE theta 1e6),
bf16 weights N(0, 0.02) from seed 0 (the engine's synthetic generator), every
layer linear quantised to W8A16 by the reference's row quantiser
(worker_w8a16.rs:330-341), bf16 lm_head.  Prompt: 128 token ids uniform over
the vocabulary from seed 1.  Greedy decode of 32 tokens, argmax first index
among ties (qwen3_vl.rs:138-143, 3276-3331).

Computed by the C++ oracle (oracle/dial_oracle_c.cpp, f64 accumulation, which
equals oracle/dial_oracle.py bit for bit) twice: with the reference's
bf16-rounded softmax probabilities (``*``) and with f32 probabilities
(``*_f32p``, the GPU kernels' online softmax).  Hidden states are stored as
bf16 bit patterns of the prefill rows ``prefill_rows`` (0..32 and five later
rows) after the layers in ``layers`` (``layers_ref`` for the reference-rounding
run), and of the first decode step (position 128).  Rows 0..32 after layers 16
and 34 let a test run layer 17 or 35 alone from the oracle's input: a 32-token
prefill (rows 0..31) then one decode token (row 32 at position 32), which by
causality must reproduce rows 0..32 after that layer.

A third, teacher-forced run (inputs = the ``_f32p`` tokens) with f32
accumulation records ``top_logits_acc32`` for the same ids as
``top_ids_f32p``: how far two correct summation orders move the logits
(``logit_spread``, the largest difference per step), which sets the token
test's bound.
"""

from __future__ import annotations

import hashlib
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "oracle"))

import dial_oracle as O  # noqa: E402
import dial_oracle_fast as F  # noqa: E402

OUT = Path(__file__).resolve().parent / "config1_qwen3_8b_w8a16.npz"
N_PROMPT, N_GEN, SEED_W, SEED_PROMPT = 128, 32, 0, 1
LAYERS = (0, 16, 17, 34, 35)
LAYERS_REF = (0, 17, 35)
ROWS = np.array(list(range(33)) + [63, 64, 95, 126, 127])
TOPK = 16


def tokens_sha(tokens) -> str:
    """sha256 of the token ids as little-endian int32 (bench.py prints the same)."""
    return hashlib.sha256(np.asarray(tokens, dtype="<i4").tobytes()).hexdigest()


def main() -> None:
    cfg = O.ModelConfig(max_seq_len=256)
    prompt = O.synth_tokens(SEED_PROMPT, N_PROMPT, cfg.vocab)
    t0 = time.time()
    model = F.FastModel(cfg, seed=SEED_W)
    print(f"model synthesised in {time.time() - t0:.1f} s", flush=True)
    out = {"prompt": prompt.astype(np.int32), "layers": np.array(LAYERS),
           "layers_ref": np.array(LAYERS_REF), "prefill_rows": ROWS, "n_gen": np.array(N_GEN)}
    for suffix, rp, layers in (("", True, LAYERS_REF), ("_f32p", False, LAYERS)):
        t0 = time.time()
        r = model.generate(prompt, N_GEN, capture_layers=layers, capture_steps=(0, 1),
                           round_probs=rp, topk=TOPK)
        print(f"round_probs={rp}: {time.time() - t0:.1f} s, tokens {r['tokens'].tolist()}",
              flush=True)
        out["tokens" + suffix] = r["tokens"].astype(np.int32)
        out["top_ids" + suffix] = r["top_ids"].astype(np.int32)
        out["top_logits" + suffix] = r["top_logits"]
        out["margin" + suffix] = r["margin"].astype(np.float32)
        for l in layers:
            out[f"prefill_l{l}{suffix}"] = O.bf16_bits(r["hidden"][(0, l)][ROWS])
            out[f"step1_l{l}{suffix}"] = O.bf16_bits(r["hidden"][(1, l)])
    t0 = time.time()
    # logits of the f32-accumulation run at the f32p run's top ids
    cache = model.new_cache()
    inp, pos, acc32 = list(prompt), 0, []
    for step in range(N_GEN):
        x = model.embed(inp)
        model.forward(x, cache, pos, accum=32, round_probs=False)
        lg = model.logits(x[-1], accum=32)[0]
        acc32.append(lg[out["top_ids_f32p"][step]])
        pos += len(inp)
        inp = [int(out["tokens_f32p"][step])]
    out["top_logits_acc32"] = np.array(acc32, np.float32)
    out["logit_spread"] = np.max(np.abs(out["top_logits_acc32"] - out["top_logits_f32p"]), axis=1)
    print(f"f32-accumulation run: {time.time() - t0:.1f} s, logit spread "
          f"{out['logit_spread'].tolist()}", flush=True)
    out["tokens_sha"] = np.array(tokens_sha(out["tokens"]))
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes), sha {out['tokens_sha']}")


if __name__ == "__main__":
    main()
