"""Benchmark: bs1 greedy decode of the Qwen3-8B-architecture W8A16 model.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = the greedy decode of BASELINE config 1: 128 tokens (positions
128..255) after the 128-token seed-1 prompt, each token through embed -> 36
W8A16 decoder layers (RMSNorm + fused QKV GEMV + q/k-norm + RoPE + paged
split-KV attention + o_proj + fused gate/up SwiGLU + down) -> ln_f -> bf16
lm_head -> argmax.  Weights are seeded random-init N(0, 0.02) bf16 quantized
to int8 at load (8.2 GB streamed per token, far larger than L2); the prompt is
prefilled before timing and every step restarts from its first token.

``value`` is tok/s of the device-resident decode loop (CUDA-graph replays,
CUDA events on the engine stream around each step's 128 tokens).  ``e2e`` is
the same metric through the public C ABI call dial_b200_decode_step with host
token buffers (H2D of the token/session/position, D2H of the next token +
status inside the timed region), 128 calls per step.  ``tokens`` carries the
sha256 of the first 32 greedy tokens and how many of them equal the oracle's
(tests/golden/config1_qwen3_8b_w8a16.npz).  ``roofline`` reports the dominant kernel (the fused gate/up W8A16
GEMV) timed live with CUDA events on the engine stream.  With --gpus N > 1
(torchrun) the 36 layers are split into N pipeline stages that hand the
hidden state to the next GPU with NCCL send/recv.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "dial-27b_b200"))

PROMPT_LEN = 128
GEN_TOKENS = 128      # config 1: greedy decode of 128 tokens per step
CHECK_TOKENS = 32     # north_star: the first 32 greedy tokens are checked
WORKLOAD = "qwen3-8b-w8a16-bs1-decode"
METRIC = "decode tok/s (bs1, Qwen3-8B W8A16)"
GOLDEN = ROOT / "tests" / "golden" / "config1_qwen3_8b_w8a16.npz"
# DRAM bytes (read + write) of one launch of the W8A16 GEMV on the fused gate/up weight
# (N=24576, K=4096, M=1) with the decode step's fused RMSNorm + SwiGLU epilogue, from an ncu
# capture of that kernel variant (profiles/gemv_w8a16_gate_up_m1_swiglu_norm.md).
GATE_UP_TRAFFIC_BYTES = 100_844_544 + 588_032
GATE_UP_TRAFFIC_SOURCE = ("ncu dram__bytes_read+write, gemv_kernel<bf16,W8A16,SwiGLU,norm> "
                          "N=24576 K=4096 M=1 (decode-step variant, replayed over 4 layers)")


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


def _smi_index(local: int) -> str:
    """nvidia-smi id of CUDA device `local` (CUDA_VISIBLE_DEVICES may remap)."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    ids = [v.strip() for v in vis.split(",") if v.strip()]
    return ids[local] if local < len(ids) else str(local)


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={_smi_index(self.gpu)}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------- CPU leg
def headline_config(parallelism: str, world: int = 1) -> dict:
    """The `config` of the headline line; both arms print the same dict."""
    cfg = {"workload": WORKLOAD, "prompt_len": PROMPT_LEN, "gen_tokens_per_step": GEN_TOKENS,
           "batch": 1, "layers": 36, "hidden": 4096, "linear": "W8A16 row int8 + f32 scale",
           "lm_head": "bf16 dense", "parallelism": parallelism,
           "l2": "inputs larger than L2 (8.2 GB weights streamed per token)"}
    if world > 1:
        from dial_b200.pipeline import plan_stages

        cfg["stages"] = [p.num_layers for p in plan_stages(36, world)]
    return cfg


def tokens_report(tokens) -> dict:
    """sha256 of the first CHECK_TOKENS greedy tokens (int32 little endian) and
    the length of their common prefix with the oracle's greedy tokens."""
    import hashlib

    import numpy as np

    t = np.asarray(tokens[:CHECK_TOKENS], dtype="<i4")
    rep = {"sha256": hashlib.sha256(t.tobytes()).hexdigest(), "n": int(t.size)}
    if GOLDEN.exists():
        g = np.load(GOLDEN)["tokens_f32p"][:CHECK_TOKENS]
        same = np.nonzero(t != g[:t.size])[0]
        rep["oracle_prefix"] = int(same[0]) if same.size else int(t.size)
    return rep


class CpuDecoder:
    """The C++/OpenMP oracle (oracle/dial_oracle_c.cpp, f32 accumulation as in
    the reference kernels) on the host cores: the first `layers` layers of the
    headline model plus its full embedding and lm_head, the prompt prefilled,
    then greedy decode.  One token's time is scaled to the 36-layer model as
    36 / layers x (layer stack) + head."""

    def __init__(self, layers: int = 4):
        sys.path.insert(0, str(ROOT / "oracle"))
        import dial_oracle as O
        import dial_oracle_fast as F

        self.F, self.layers = F, layers
        self.cfg = O.ModelConfig(max_seq_len=PROMPT_LEN + 2048)
        self.m = F.FastModel(self.cfg, seed=0, num_layers=layers)
        self._prefill()

    def _prefill(self):
        self.cache = self.m.new_cache()
        x = self.m.embed(_prompt_tokens(self.cfg.vocab))
        self.m.forward(x, self.cache, 0, accum=32, round_probs=False)
        self.tok = int(self.m.logits(x[-1], accum=32)[0].argmax())
        self.pos = PROMPT_LEN

    def token_seconds(self) -> tuple[float, float]:
        """Decode one token; returns (layer-stack seconds, head seconds)."""
        if self.pos >= self.cfg.max_seq_len:
            self._prefill()
        x = self.m.embed([self.tok])
        a = time.perf_counter()
        self.m.forward(x, self.cache, self.pos, accum=32, round_probs=False)
        b = time.perf_counter()
        self.tok = int(self.m.logits(x, accum=32)[0].argmax())
        c = time.perf_counter()
        self.pos += 1
        return b - a, c - b

    def sample(self, n_tokens: int) -> float:
        """tok/s of the 36-layer model estimated from n_tokens decode tokens."""
        ls, hs = zip(*(self.token_seconds() for _ in range(n_tokens)))
        return 1.0 / (36 / self.layers * statistics.median(ls) + statistics.median(hs))

    def describe(self, n_tokens: int) -> dict:
        import platform

        cpu = platform.processor() or ""
        try:
            for ln in open("/proc/cpuinfo"):
                if ln.startswith("model name"):
                    cpu = ln.split(":", 1)[1].strip()
                    break
        except OSError:
            pass
        return {"unit": "tok/s", "cores": self.F.threads(), "kind": "port", "cpu_model": cpu,
                "sample": f"{n_tokens} greedy decode tokens at context {PROMPT_LEN}+ of the "
                          f"first {self.layers} W8A16 layers + full bf16 lm_head of the same "
                          f"synthetic model, C++/OpenMP CPU restatement of the reference "
                          f"(oracle/dial_oracle_c.cpp, f32 accumulation; not the reference "
                          f"binary), scaled to 36 layers"}


def cpu_decode_sample(n_tokens: int = 24) -> dict:
    d = CpuDecoder()
    d.sample(2)
    return {"value": d.sample(n_tokens), **d.describe(n_tokens)}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    d = CpuDecoder()
    per_step = 6
    vals = []
    for i in range(args.warmup + args.steps):
        v = d.sample(per_step)
        if i >= args.warmup:
            vals.append(v)
    v = statistics.median(vals)
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    par = "single GPU" if world <= 1 else f"pp{world}"
    line = {"impl": "reference", "metric": METRIC, "value": v,
            "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": GEN_TOKENS * 1000.0 / v, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": headline_config(par, world),
            "cpu_baseline": {"value": v, **d.describe(per_step * args.steps)},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------- GPU leg
def run_single(args) -> dict:
    import numpy as np
    import torch

    import dial_b200

    dev = 0
    torch.cuda.set_device(dev)
    cfg = dial_b200.Config(max_seq_len=4096, max_sessions=1, max_tokens=PROMPT_LEN)
    eng = dial_b200.Engine(cfg, device=dev)
    eng.load_synthetic(seed=0)
    prompt = _prompt_tokens(cfg.vocab_size)
    eng.generate(prompt, 2)  # first call: lazy kernel loading, tensor maps, graphs
    first, ttft, _ = eng.generate(prompt, 1)
    check, _, _ = eng.generate(prompt, CHECK_TOKENS)
    stream = eng.stream
    tok0 = int(first[0])

    # ---- e2e through the public C ABI (host buffers, synchronous per token)
    def e2e_step():
        tok = tok0
        for i in range(GEN_TOKENS):
            tok = int(eng.decode_step([tok], [0], [PROMPT_LEN + i])[0])
        return tok

    for _ in range(args.warmup):
        e2e_step()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        last_e2e = e2e_step()
    e2e_s = time.perf_counter() - t0

    # ---- device-resident loop: each step decodes positions 128..255 from the
    # prompt's first token (graph replays, tokens fed back on the device)
    def loop_step(ev_a=None, ev_b=None):
        eng.loop_prepare([tok0], [0], [PROMPT_LEN])
        if ev_a is not None:
            ev_a.record(stream)
        eng.loop_run(1, GEN_TOKENS)
        if ev_b is not None:
            ev_b.record(stream)

    for _ in range(args.warmup):
        loop_step()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    with ClockSampler(dev) as clk:
        time.sleep(0.3)
        for a, b in evs:
            loop_step(a, b)
        torch.cuda.synchronize()
    step_ms = sum(a.elapsed_time(b) for a, b in evs) / args.steps
    toks, positions = eng.loop_state(1)

    # ---- dominant kernel live: fused gate/up GEMV, same launch config, rotating
    # over the 36 layers' weights (3.6 GB) so every launch streams from HBM
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    iters = 72
    eng.linear_replay(-1, 2, 1, 3)
    torch.cuda.synchronize()
    ev0.record(stream)
    eng.linear_replay(-1, 2, 1, iters)
    ev1.record(stream)
    ev1.synchronize()
    k_us = ev0.elapsed_time(ev1) * 1000.0 / iters
    k_bytes = eng.linear_bytes(0, 2, 1)
    mean_ctx = PROMPT_LEN + GEN_TOKENS / 2
    token_bytes = sum(eng.linear_bytes(0, w, 1) for w in range(4)) * cfg.num_hidden_layers + \
        eng.linear_bytes(0, 4, 1) + 36 * 2 * 8 * 128 * 2 * mean_ctx
    peaks = load_peaks()
    achieved = k_bytes / (k_us * 1e-6) / 1e9
    status = dial_b200.device_status()
    tok_ms = step_ms / GEN_TOKENS
    return {
        "value": 1000.0 / tok_ms, "ms_per_step": step_ms,
        "e2e_tok_s": args.steps * GEN_TOKENS / e2e_s,
        "ttft_s": ttft, "clocks": clk.summary(), "status": status,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "traffic": GATE_UP_TRAFFIC_BYTES,
                     "traffic_source": GATE_UP_TRAFFIC_SOURCE,
                     "kernel": "gemv_kernel<bf16,W8A16,SwiGLU,norm> (fused gate/up, N=24576 K=4096 M=1)",
                     "launch_us": k_us, "bytes_per_launch": k_bytes, "peak_source": peaks["source"],
                     "token_bytes": token_bytes,
                     "token_frac": token_bytes / (tok_ms * 1e-3) / 1e9 / peaks["hbm_gbs"]},
        "gpu_launches": eng.step_kernel_count(1) * GEN_TOKENS * args.steps,
        "tokens": tokens_report(check),
        "loop_consistent": bool(int(positions[0]) == PROMPT_LEN + GEN_TOKENS and
                                int(toks[0]) == last_e2e),
    }


def run_pipeline(args) -> None:
    """N > 1: one process per GPU (torchrun), the 36 layers split evenly into N
    pipeline stages, the hidden state handed stage to stage and the token
    returned to stage 0 (dial_b200.pipeline).  Same step as N = 1: 128 greedy
    tokens from the prompt's first token, positions 128..255."""
    import datetime

    import numpy as np
    import torch
    import torch.distributed as dist

    import dial_b200
    from dial_b200.pipeline import StageRunner, plan_stages

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    try:
        cfg = dial_b200.Config(max_seq_len=4096, max_sessions=1, max_tokens=PROMPT_LEN)
        plan = plan_stages(cfg.num_hidden_layers, world)[rank]
        eng = dial_b200.Engine(cfg, first_layer=plan.first_layer, num_layers=plan.num_layers,
                               device=local)
        eng.load_synthetic(seed=0)
        runner = StageRunner(eng, plan, cfg.hidden_size)
        stream = torch.cuda.Stream(dev)

        def max_over_ranks(v: float) -> float:
            t = torch.tensor([v], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item())

        def sync_all():
            torch.cuda.synchronize()
            dist.barrier()
            torch.cuda.synchronize()

        prompt_np = _prompt_tokens(cfg.vocab_size)
        with torch.cuda.stream(stream):
            prompt = torch.as_tensor(prompt_np, device=dev) if plan.is_first else None
            # warm-up: communicators, kernel loading, the stage graph
            runner.generate(prompt_np, 4)
            sync_all()
            ttfts = []
            for _ in range(3):
                sync_all()
                t0 = time.perf_counter()
                runner.step(prompt, PROMPT_LEN, 0)
                torch.cuda.synchronize()
                ttfts.append(max_over_ranks(time.perf_counter() - t0))
            ttft = statistics.median(ttfts)
            check = runner.generate(prompt_np, CHECK_TOKENS)
            first = torch.zeros(1, dtype=torch.int32, device=dev)
            if plan.is_first:
                first.fill_(int(check[0]))

            # ---- the stage hop: the peer-memory link (default), or NCCL
            # send/recv (DIAL_B200_PEER_LINK=0, or when the link cannot open on
            # every rank)
            transport = "nccl"
            if os.environ.get("DIAL_B200_PEER_LINK", "1") == "1":
                transport = "peer"
                try:
                    runner.link()
                except Exception as e:  # noqa: BLE001  (reported, the NCCL path still runs)
                    transport = f"nccl ({type(e).__name__}: {e})"
            peer = transport == "peer"
            ok = torch.tensor([1 if peer else 0], dtype=torch.int32, device=dev)
            dist.all_reduce(ok, op=dist.ReduceOp.MIN)
            if peer and int(ok.item()) == 0:
                peer, transport = False, "nccl (the link did not open on every rank)"

            # ---- device-resident decode: tokens stay on the GPUs
            def loop_step(ev_a=None, ev_b=None):
                stream.synchronize()  # the previous step's graphs read the positions
                runner.decode_prepare(PROMPT_LEN)
                tok = first.clone() if plan.is_first else None
                if ev_a is not None:
                    ev_a.record(stream)
                if peer:
                    last = runner.decode_linked(tok, GEN_TOKENS)
                else:
                    for _ in range(GEN_TOKENS):
                        tok = runner.decode_step(tok)
                    last = int(tok.item()) if plan.is_first else None
                if ev_b is not None:
                    ev_b.record(stream)
                return last

            for _ in range(args.warmup):
                loop_step()
            sync_all()
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in range(args.steps)]
            with ClockSampler(local) as clk:
                time.sleep(0.2)
                for a, b in evs:
                    last_loop = loop_step(a, b)
                torch.cuda.synchronize()
            sync_all()
            step_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in evs) / args.steps)
            last_loop = last_loop if plan.is_first else -1

            # ---- end to end: each token goes host -> stage 0 and back to the host
            pin_in = torch.zeros(1, dtype=torch.int32).pin_memory()
            pin_out = torch.zeros(1, dtype=torch.int32).pin_memory()
            tok_dev = torch.zeros(1, dtype=torch.int32, device=dev)

            def e2e_step():
                stream.synchronize()
                runner.decode_prepare(PROMPT_LEN)
                tok_host = int(check[0]) if plan.is_first else 0
                for _ in range(GEN_TOKENS):
                    if plan.is_first:
                        pin_in.fill_(tok_host)
                        tok_dev.copy_(pin_in, non_blocking=True)
                        if peer:
                            eng.stage_link_step(1, tok_dev)
                            tok_host = int(eng.stage_link_finish(1)[0])
                        else:
                            out = runner.decode_step(tok_dev)
                            pin_out.copy_(out, non_blocking=True)
                            stream.synchronize()
                            tok_host = int(pin_out.item())
                    elif peer:
                        eng.stage_link_step(1, None)
                    else:
                        runner.decode_step(None)
                return tok_host

            for _ in range(args.warmup):
                e2e_step()
            sync_all()
            t0 = time.perf_counter()
            for _ in range(args.steps):
                last_e2e = e2e_step()
            torch.cuda.synchronize()
            e2e_s = max_over_ranks(time.perf_counter() - t0)

            # ---- each stage's own compute per token (its stage graph, no hop), summed
            # over the stages: the rest of the pipelined per-token time is the hops
            h_loc = torch.zeros(1, cfg.hidden_size, dtype=torch.bfloat16, device=dev)
            t_in = torch.zeros(1, dtype=torch.int32, device=dev)
            t_out = torch.zeros(1, dtype=torch.int32, device=dev)
            eng.stage_prepare([0], [PROMPT_LEN])
            for _ in range(4):
                eng.stage_step(1, t_in if plan.is_first else None, h_loc,
                               t_out if plan.is_last else None)
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            ev0.record(stream)
            for _ in range(64):
                eng.stage_step(1, t_in if plan.is_first else None, h_loc,
                               t_out if plan.is_last else None)
            ev1.record(stream)
            ev1.synchronize()
            stage_us = torch.tensor([ev0.elapsed_time(ev1) * 1000.0 / 64], dtype=torch.float64,
                                    device=dev)
            dist.all_reduce(stage_us)
            compute_us = float(stage_us.item())
            hop_us = max(0.0, (step_ms * 1000.0 / GEN_TOKENS - compute_us) / world)

            # ---- dominant kernel live on this rank: fused gate/up GEMV, rotating layers
            layers = list(range(plan.first_layer, plan.first_layer + plan.num_layers))
            eng.linear_replay(-1, 2, 1, 2)
            torch.cuda.synchronize()
            iters = 8 * len(layers)
            ev0.record(eng.stream)
            eng.linear_replay(-1, 2, 1, iters)
            ev1.record(eng.stream)
            ev1.synchronize()
            k_us = ev0.elapsed_time(ev1) * 1000.0 / iters
            k_bytes = eng.linear_bytes(layers[0], 2, 1)
        # per stage and token: 5 per layer, embed (first), head (last), position advance,
        # and with the link a receive and a send kernel
        per_stage = plan.num_layers * 5 + int(plan.is_first) + 2 * int(plan.is_last) + 1 + \
            (2 if peer else 0)
        launches = torch.tensor([per_stage * GEN_TOKENS * args.steps], dtype=torch.int64,
                                device=dev)
        dist.all_reduce(launches)
        status = dial_b200.device_status()
        peaks = load_peaks()
        achieved = k_bytes / (k_us * 1e-6) / 1e9
        if rank == 0:
            line = {
                "metric": METRIC, "value": GEN_TOKENS * 1000.0 / step_ms,
                "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": step_ms, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": headline_config(f"pp{world}", world),
                "e2e": {"value": GEN_TOKENS * args.steps / e2e_s, "unit": "tok/s",
                        "h2d_bytes_per_step": 4 * GEN_TOKENS, "d2h_bytes_per_step": 4 * GEN_TOKENS},
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                             "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                             "traffic": GATE_UP_TRAFFIC_BYTES,
                             "traffic_source": GATE_UP_TRAFFIC_SOURCE,
                             "kernel": "gemv_kernel<bf16,W8A16,SwiGLU,norm> (fused gate/up, "
                                       "N=24576 K=4096 M=1), stage 0",
                             "launch_us": k_us, "bytes_per_launch": k_bytes,
                             "peak_source": peaks["source"]},
                "cpu_baseline": None, "clocks": clk.summary(),
                "gpu_launches": int(launches.item()), "ttft_s": ttft,
                "transport": transport, "handoff_us": hop_us,
                "handoff_note": "per hop: (pipelined ms per token - sum of the stages' own "
                                "compute per token) / stages",
                "stage_compute_us_sum": compute_us, "device_status": status,
                "tokens": tokens_report(check),
                "loop_consistent": bool(last_loop == last_e2e),
            }
            print(json.dumps(line), flush=True)
        sync_all()
    finally:
        dist.destroy_process_group()


def _relaunch_with_torchrun(args) -> None:
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={args.gpus}", "--master-addr", "127.0.0.1", "--master-port",
           str(port), str(Path(__file__).resolve()), "--gpus", str(args.gpus), "--steps",
           str(args.steps), "--warmup", str(args.warmup), "--impl", args.impl,
           "--workload", args.workload]
    raise SystemExit(subprocess.call(cmd))


def _pipeline_init():
    """torchrun rank, world, local GPU and the NCCL process group (short timeout)."""
    import datetime

    import torch
    import torch.distributed as dist

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    return rank, world, local, dev


def _max_over_ranks(v: float, dev) -> float:
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _sync_all():
    import torch
    import torch.distributed as dist

    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()


def run_pipeline_long(args) -> None:
    """N > 1, BASELINE configs 3 and 5: the decoder split evenly into N
    pipeline stages (dial_b200.pipeline.StageRunner), a long prompt prefilled
    through the stages (TTFT, warmed, median of the timed steps) and bs1
    greedy decode of 256 tokens after it (device-side stage graphs, CUDA
    events, max over ranks).  prefill2048: Qwen3-8B W8A16, 2048-token prompt;
    fp8_27b / nvfp4_27b: the 27B-class decoder (64 layers) with FP8 block-128
    or NVFP4 linears, 4096-token prompt."""
    import numpy as np
    import torch
    import torch.distributed as dist

    import dial_b200
    from dial_b200.pipeline import StageRunner, plan_stages

    rank, world, local, dev = _pipeline_init()
    try:
        n_gen = 256
        if args.workload == "prefill2048":
            n_prompt = 2048
            cfg = dial_b200.Config(max_seq_len=n_prompt + n_gen + 64, max_sessions=1,
                                   max_tokens=n_prompt)
            tag, metric_model = "qwen3-8b-w8a16-prefill2048-decode256", "Qwen3-8B W8A16"
        else:
            n_prompt = 4096
            fmt = dial_b200.FMT_FP8_BLOCK128 if args.workload == "fp8_27b" \
                else dial_b200.FMT_NVFP4_G16
            cfg = dial_b200.Config.dense_27b(max_seq_len=n_prompt + n_gen + 64, max_sessions=1,
                                             max_tokens=n_prompt, linear_fmt=fmt)
            ftag = "fp8-block128" if args.workload == "fp8_27b" else "nvfp4"
            tag, metric_model = f"dense27b-{ftag}-prefill4096-decode256", f"27B-class {ftag}"
        plan = plan_stages(cfg.num_hidden_layers, world)[rank]
        eng = dial_b200.Engine(cfg, first_layer=plan.first_layer, num_layers=plan.num_layers,
                               device=local)
        eng.load_synthetic(seed=0)
        runner = StageRunner(eng, plan, cfg.hidden_size)
        stream = torch.cuda.Stream(dev)
        prompt_np = _prompt_tokens(cfg.vocab_size, n_prompt)
        with torch.cuda.stream(stream):
            prompt = torch.as_tensor(prompt_np, device=dev) if plan.is_first else None
            runner.generate(prompt_np[:64], 2)  # communicators, kernels, stage graph
            ttfts = []
            for i in range(args.warmup + args.steps):
                _sync_all()
                t0 = time.perf_counter()
                tok = runner.step(prompt, n_prompt, 0)
                torch.cuda.synchronize()
                if i >= args.warmup:
                    ttfts.append(_max_over_ranks(time.perf_counter() - t0, dev))
            ttft = statistics.median(ttfts)
            runner.decode_prepare(n_prompt)
            for _ in range(8):
                tok = runner.decode_step(tok)
            _sync_all()
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with ClockSampler(local) as clk:
                ev0.record(stream)
                for _ in range(n_gen - 8):
                    tok = runner.decode_step(tok)
                ev1.record(stream)
                ev1.synchronize()
            _sync_all()
            dec_ms = _max_over_ranks(ev0.elapsed_time(ev1) / (n_gen - 8), dev)
            last = int(tok.item()) if plan.is_first else -1
        w_bytes = torch.tensor([sum(eng.linear_bytes(plan.first_layer, w, 1) for w in range(4)) *
                                plan.num_layers + (eng.linear_bytes(0, 4, 1) if plan.is_last
                                                   else 0)], dtype=torch.float64, device=dev)
        dist.all_reduce(w_bytes)
        status = dial_b200.device_status()
        peaks = load_peaks()
        gbs = float(w_bytes.item()) / (dec_ms * 1e-3) / 1e9
        if rank == 0:
            line = {"metric": f"decode tok/s (bs1, {metric_model}, after a {n_prompt}-token "
                              f"prefill, pipelined)", "value": 1000.0 / dec_ms, "unit": "tok/s",
                    "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                    "ms_per_step": dec_ms, "higher_is_better": True, "scaling": "strong",
                    "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                    "config": {"workload": tag, "prompt_len": n_prompt, "gen_tokens": n_gen,
                               "parallelism": f"pp{world}",
                               "stages": [p.num_layers for p in
                                          plan_stages(cfg.num_hidden_layers, world)],
                               "l2": "inputs larger than L2"},
                    "ttft_ms": ttft * 1e3, "prefill_tok_s": n_prompt / ttft,
                    "hbm": {"weight_bytes_per_token": float(w_bytes.item()),
                            "aggregate_gbs": gbs, "frac_of_one_gpu": gbs / peaks["hbm_gbs"],
                            "peak": peaks["hbm_gbs"]},
                    "clocks": clk.summary(), "device_status": status, "last_token": last}
            print(json.dumps(line), flush=True)
        _sync_all()
    finally:
        dist.destroy_process_group()


def run_pipeline_ragged(args) -> None:
    """N > 1: 32 sessions with KV lengths uniform in
    [128, 8192] (seed 2), the decoder split evenly into N stages, the
    sessions cut into N micro-batches that are in flight on different stages
    at once (dial_b200.pipeline.MicroBatchRunner); one decode token per
    session per iteration, CUDA events on every rank, max over ranks."""
    import hashlib

    import numpy as np
    import torch

    import dial_b200
    from dial_b200.pipeline import MicroBatchRunner, plan_stages

    rank, world, local, dev = _pipeline_init()
    try:
        n_sess = 32
        n_micro = world
        lengths = np.random.default_rng(2).integers(128, 8193, size=n_sess).astype(np.int32)
        cfg = dial_b200.Config(max_seq_len=8192 + args.steps + args.warmup + 16,
                               max_sessions=n_sess, max_tokens=64)
        plan = plan_stages(cfg.num_hidden_layers, world)[rank]
        eng = dial_b200.Engine(cfg, first_layer=plan.first_layer, num_layers=plan.num_layers,
                               device=local)
        eng.load_synthetic(seed=0)
        for sidx in range(n_sess):
            eng.session_fill_random(sidx, int(lengths[sidx]), seed=2 + sidx)
        runner = MicroBatchRunner(eng, plan, cfg.hidden_size, n_sess, n_micro)
        stream = torch.cuda.Stream(dev)
        with torch.cuda.stream(stream):
            runner.prepare(np.arange(n_sess), lengths, _prompt_tokens(cfg.vocab_size, n_sess))
            for _ in range(args.warmup):
                runner.iteration()
            runner.finish()
            _sync_all()
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with ClockSampler(local) as clk:
                ev0.record(stream)
                for _ in range(args.steps):
                    runner.iteration()
                runner.finish()
                ev1.record(stream)
                ev1.synchronize()
            _sync_all()
            it_ms = _max_over_ranks(ev0.elapsed_time(ev1) / args.steps, dev)
            toks = runner.tokens()
        status = dial_b200.device_status()
        if rank == 0:
            line = {"metric": "decode tok/s (32 ragged sessions, KV 128-8192, Qwen3-8B W8A16, "
                              "pipelined)", "value": n_sess * 1000.0 / it_ms, "unit": "tok/s",
                    "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                    "ms_per_step": it_ms, "higher_is_better": True, "scaling": "strong",
                    "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                    "config": {"workload": "qwen3-8b-w8a16-ragged32", "sessions": n_sess,
                               "kv_lengths": "U[128, 8192] seed 2",
                               "kv_tokens": int(lengths.sum()), "page_tokens": 16,
                               "parallelism": f"pp{world}", "micro_batches": n_micro,
                               "stages": [p.num_layers for p in plan_stages(36, world)],
                               "l2": "inputs larger than L2"},
                    "clocks": clk.summary(), "device_status": status,
                    "tokens_sha256": hashlib.sha256(toks.astype("<i4").tobytes()).hexdigest()}
            print(json.dumps(line), flush=True)
        _sync_all()
    finally:
        import torch.distributed as dist

        dist.destroy_process_group()


def run_prefill2048(args) -> dict:
    """Long-prompt workload on one GPU: prefill of 2048 seeded token ids (TTFT,
    first token on the host), then bs1 greedy decode of 256 tokens."""
    import torch

    import dial_b200

    torch.cuda.set_device(0)
    n_prompt, n_gen = 2048, 256
    cfg = dial_b200.Config(max_seq_len=n_prompt + n_gen + 64, max_sessions=1, max_tokens=n_prompt)
    eng = dial_b200.Engine(cfg, device=0)
    eng.load_synthetic(seed=0)
    prompt = _prompt_tokens(cfg.vocab_size, n_prompt)
    ttfts = []
    for i in range(args.warmup + args.steps):
        _, ttft, _ = eng.generate(prompt, 1)
        if i >= args.warmup:
            ttfts.append(ttft)
    ttft = statistics.median(ttfts)
    first, _, _ = eng.generate(prompt, 1)
    stream = eng.stream
    eng.loop_prepare([int(first[0])], [0], [n_prompt])
    eng.loop_run(1, 8)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        ev0.record(stream)
        eng.loop_run(1, n_gen - 8)
        ev1.record(stream)
        ev1.synchronize()
    dec_ms = ev0.elapsed_time(ev1) / (n_gen - 8)
    status = dial_b200.device_status()
    H, I, QKV = cfg.hidden_size, cfg.intermediate_size, cfg.qkv_dim
    flops = 2.0 * n_prompt * cfg.num_hidden_layers * (QKV * H + H * H + 2 * I * H + H * I)
    return {"metric": "TTFT ms (prefill 2048 tokens, Qwen3-8B W8A16)", "value": ttft * 1e3,
            "unit": "ms", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ttft * 1e3, "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "qwen3-8b-w8a16-prefill2048-decode256", "prompt_len": n_prompt,
                       "gen_tokens": n_gen, "batch": 1, "parallelism": "single GPU",
                       "l2": "inputs larger than L2"},
            "prefill_tok_s": n_prompt / ttft, "decode_tok_s": 1000.0 / dec_ms,
            "decode_ms_per_token": dec_ms, "clocks": clk.summary(), "device_status": status,
            "linear_tflop_per_prefill_approx": flops / 1e12,
            "gpu_launches": eng.prefill_kernel_count(n_prompt) * args.steps,
            "decode_gpu_launches_per_token": eng.step_kernel_count(1),
            "e2e": {"value": ttft * 1e3, "unit": "ms", "h2d_bytes_per_step": 4 * n_prompt,
                    "d2h_bytes_per_step": 4}}


def run_ragged32(args) -> dict:
    """Ragged multi-session workload on one GPU: 32 sessions with KV lengths uniform in
    [128, 8192] (seed 2) in 16-token pages, one decode token per session per
    iteration (device loop)."""
    import numpy as np
    import torch

    import dial_b200

    torch.cuda.set_device(0)
    n_sess = 32
    lengths = np.random.default_rng(2).integers(128, 8193, size=n_sess).astype(np.int32)
    cfg = dial_b200.Config(max_seq_len=8192 + args.steps + args.warmup + 16, max_sessions=n_sess,
                           max_tokens=64)
    eng = dial_b200.Engine(cfg, device=0)
    eng.load_synthetic(seed=0)
    for sidx in range(n_sess):
        eng.session_fill_random(sidx, int(lengths[sidx]), seed=2 + sidx)
    toks = _prompt_tokens(cfg.vocab_size, n_sess)
    sids = np.arange(n_sess, dtype=np.int32)
    eng.loop_prepare(toks, sids, lengths)
    eng.loop_run(n_sess, args.warmup)
    torch.cuda.synchronize()
    stream = eng.stream
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        ev0.record(stream)
        eng.loop_run(n_sess, args.steps)
        ev1.record(stream)
        ev1.synchronize()
    it_ms = ev0.elapsed_time(ev1) / args.steps
    _, pos = eng.loop_state(n_sess)
    status = dial_b200.device_status()
    kv_bytes = float(np.sum(lengths + args.warmup + args.steps / 2)) * 36 * 2 * 8 * 128 * 2
    w_bytes = sum(eng.linear_bytes(0, w, n_sess) for w in range(4)) * 36 + eng.linear_bytes(0, 4, n_sess)
    gbs = (kv_bytes + w_bytes) / (it_ms * 1e-3) / 1e9
    peaks = load_peaks()
    return {"metric": "decode tok/s (32 ragged sessions, KV 128-8192, Qwen3-8B W8A16)",
            "value": n_sess * 1000.0 / it_ms, "unit": "tok/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": it_ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "qwen3-8b-w8a16-ragged32", "sessions": n_sess,
                       "kv_lengths": "U[128, 8192] seed 2", "kv_tokens": int(lengths.sum()),
                       "page_tokens": 16, "parallelism": "single GPU",
                       "l2": "inputs larger than L2"},
            "hbm": {"bytes_per_iteration": kv_bytes + w_bytes, "achieved_gbs": gbs,
                    "frac": gbs / peaks["hbm_gbs"], "peak": peaks["hbm_gbs"]},
            "clocks": clk.summary(), "device_status": status,
            "gpu_launches": eng.step_kernel_count(n_sess) * args.steps,
            "positions_advanced": bool(np.all(pos == lengths + args.warmup + args.steps))}


def run_quant27b(args, fmt_name: str) -> dict:
    """27B-class workload on one GPU: the dense decoder (64 layers,
    hidden 5120, 40 q / 8 kv heads, FFN 21504) with FP8 block-128 or NVFP4
    linears, prefill of 4096 seeded tokens (TTFT) then bs1 greedy decode."""
    import torch

    import dial_b200

    torch.cuda.set_device(0)
    fmt = getattr(dial_b200, fmt_name)
    n_prompt, n_gen = 4096, 256
    cfg = dial_b200.Config.dense_27b(max_seq_len=n_prompt + n_gen + 64, max_sessions=1,
                                     max_tokens=n_prompt, linear_fmt=fmt)
    eng = dial_b200.Engine(cfg, device=0)
    eng.load_synthetic(seed=0)
    prompt = _prompt_tokens(cfg.vocab_size, n_prompt)
    ttfts = []
    for i in range(args.warmup + args.steps):
        first, ttft, _ = eng.generate(prompt, 1)
        if i >= args.warmup:
            ttfts.append(ttft)
    ttft = statistics.median(ttfts)
    eng.loop_prepare([int(first[0])], [0], [n_prompt])
    eng.loop_run(1, 8)
    torch.cuda.synchronize()
    stream = eng.stream
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        ev0.record(stream)
        eng.loop_run(1, n_gen - 8)
        ev1.record(stream)
        ev1.synchronize()
    dec_ms = ev0.elapsed_time(ev1) / (n_gen - 8)
    status = dial_b200.device_status()
    w_bytes = sum(eng.linear_bytes(0, w, 1) for w in range(4)) * cfg.num_hidden_layers + \
        eng.linear_bytes(0, 4, 1)
    peaks = load_peaks()
    gbs = w_bytes / (dec_ms * 1e-3) / 1e9
    tag = "fp8-block128" if fmt == dial_b200.FMT_FP8_BLOCK128 else "nvfp4"
    return {"metric": f"decode tok/s (bs1, 27B-class dense, {tag})", "value": 1000.0 / dec_ms,
            "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dec_ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"dense27b-{tag}-prefill4096-decode256", "layers": 64,
                       "hidden": 5120, "heads": "40q/8kv", "ffn": 21504, "prompt_len": n_prompt,
                       "gen_tokens": n_gen, "parallelism": "single GPU",
                       "l2": "inputs larger than L2"},
            "ttft_ms": ttft * 1e3, "prefill_tok_s": n_prompt / ttft,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": gbs / peaks["hbm_gbs"], "bytes_per_token": w_bytes,
                         "traffic": None, "kernel": "whole decode step (weights only)"},
            "clocks": clk.summary(), "device_status": status,
            "gpu_launches": eng.step_kernel_count(1) * (n_gen - 8),
            "prefill_gpu_launches": eng.prefill_kernel_count(n_prompt)}


def _prompt_tokens(vocab: int, n: int = PROMPT_LEN):
    import numpy as np

    from dial_b200.synth import STREAM_TOKENS

    # seed-1 uniform ids; same hash as the device generator (layout.cu)
    def mix64(z):
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))

    seed = 1
    base = np.uint64(((seed * 0x9E3779B97F4A7C15) ^ (STREAM_TOKENS * 0xD1B54A32D192ED03)) & ((1 << 64) - 1))
    with np.errstate(over="ignore"):
        h = mix64(np.arange(n, dtype=np.uint64) + base)
    return (h % np.uint64(vocab)).astype(np.int32)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="decode",
                    choices=["decode", "prefill2048", "ragged32", "fp8_27b", "nvfp4_27b"],
                    help="decode (bs1 Qwen3-8B W8A16 decode, the headline metric), prefill2048 "
                         "(2048-token prefill then decode), ragged32 (32 ragged sessions), "
                         "fp8_27b / nvfp4_27b (27B-class decoder with FP8 block-128 or NVFP4 "
                         "linears); with --gpus N > 1 each runs as N pipeline stages "
                         "(ragged32 with N micro-batches in flight)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world == 1 and args.gpus > 1:
        _relaunch_with_torchrun(args)
    if world > 1 and args.workload != "decode":
        if args.workload == "ragged32":
            run_pipeline_ragged(args)
        else:
            run_pipeline_long(args)
        return
    if args.workload != "decode":
        if args.workload == "prefill2048":
            r = run_prefill2048(args)
        elif args.workload == "ragged32":
            r = run_ragged32(args)
        else:
            r = run_quant27b(args, "FMT_FP8_BLOCK128" if args.workload == "fp8_27b"
                             else "FMT_NVFP4_G16")
        print(json.dumps(r), flush=True)
        return
    if world > 1:
        run_pipeline(args)
        return
    r = run_single(args)
    cpu = None if args.no_cpu_baseline else cpu_decode_sample()
    line = {
        "metric": METRIC, "value": r["value"], "unit": "tok/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "config": headline_config("single GPU"),
        "e2e": {"value": r["e2e_tok_s"], "unit": "tok/s", "h2d_bytes_per_step": 12 * GEN_TOKENS,
                "d2h_bytes_per_step": 8 * GEN_TOKENS},
        "roofline": r["roofline"], "cpu_baseline": cpu, "clocks": r["clocks"],
        "gpu_launches": r["gpu_launches"], "ttft_s": r["ttft_s"], "device_status": r["status"],
        "tokens": r["tokens"], "loop_consistent": r["loop_consistent"],
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
