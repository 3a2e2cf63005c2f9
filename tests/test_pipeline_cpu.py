"""Pipeline stage logic (dial_b200.pipeline) on CPU with gloo ranks.

Each rank owns a contiguous layer range of a small oracle model and runs the
same StageRunner the GPU path uses, with an oracle-backed stand-in engine; the
tokens stage 0 collects must equal the single-process greedy decode
(qwen3_vl.rs:138-143 over forward_blocks_from, qwen3_vl.rs:2018-2177)."""

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _cfg():
    import dial_oracle as O

    return O.ModelConfig(hidden=256, inter=512, vocab=500, layers=5, heads=2, kv_heads=1,
                         max_seq_len=64)


class OracleStage:
    """Stand-in engine for one stage: embed / forward_local_batch / head on
    CPU float32 tensors through the oracle."""

    dtype = torch.float32
    torch_device = torch.device("cpu")

    def __init__(self, model):
        import dial_oracle as O

        self.O = O
        self.model = model
        self.cache = O.Cache(model.cfg.layers, model.cfg.max_seq_len)

    def embed(self, tokens):
        return torch.from_numpy(self.model.embed[tokens.numpy().astype(np.int64)].copy())

    def forward_local_batch(self, x, batch, session=0):
        O, m = self.O, self.model
        h = x.numpy()
        for _, pos, idx in batch:
            h = O.layer_forward(h, m.layers[idx], m.cfg, pos, idx, self.cache, m.cos, m.sin)
        return torch.from_numpy(np.ascontiguousarray(h, dtype=np.float32))

    def head(self, x):
        O = self.O
        logits = O.model_logits(self.model, x.numpy()[-1])
        return torch.tensor([O.argmax_first(logits)], dtype=torch.int32)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, prompt, n_gen, out_path, topo_text):
    sys.path[:0] = [str(ROOT / "dial-27b_b200"), str(ROOT / "oracle"), str(ROOT / "tests")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import dial_oracle as O
    from dial_b200.pipeline import StageRunner, plan_stages
    from dial_b200.topology import Topology

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        cfg = _cfg()
        model = O.synth_model(cfg, seed=3, std=0.05)
        topo = Topology.from_yaml(topo_text) if topo_text else None
        plan = plan_stages(cfg.layers, world, topo)[rank]
        runner = StageRunner(OracleStage(model), plan, cfg.hidden)
        toks = runner.generate(prompt, n_gen)
        if rank == 0:
            np.save(out_path, toks)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _run(world, tmp_path, topo_text=None, n_gen=5):
    import dial_oracle as O

    prompt = list(np.random.default_rng(4).integers(0, 500, size=7))
    out = tmp_path / "toks.npy"
    mp.start_processes(_worker, args=(world, _free_port(), prompt, n_gen, str(out), topo_text),
                       nprocs=world, start_method="spawn", join=True)
    got = np.load(out)
    cfg = _cfg()
    want, _ = O.greedy_generate(O.synth_model(cfg, seed=3, std=0.05), prompt, n_gen)
    np.testing.assert_array_equal(got, np.asarray(want, dtype=np.int32))


@pytest.mark.parametrize("world", [1, 2, 3])
def test_pipeline_tokens_match_single_process(tmp_path, world):
    _run(world, tmp_path)


def test_pipeline_follows_topology_ranges(tmp_path):
    topo = """
tail:
  host: gpu1
  layers: ["model.layers.1-4"]
head:
  host: gpu0
  layers: ["model.layers.0"]
"""
    _run(2, tmp_path, topo)


def test_plan_rejects_mismatched_world():
    from dial_b200.pipeline import plan_stages

    with pytest.raises(ValueError, match="3 stages but the job has 2 ranks"):
        plan_stages(36, 2, __import__("dial_b200").Topology.even_split(36, 3))
    plans = plan_stages(36, 8)
    assert [p.num_layers for p in plans] == [5, 5, 5, 5, 4, 4, 4, 4]
    assert plans[0].is_first and plans[-1].is_last


class OracleRowsStage:
    """Stand-in engine for the micro-batch runner: stage_prepare /
    stage_step_rows over per-session oracle caches for this stage's layers."""

    dtype = torch.float32
    torch_device = torch.device("cpu")

    def __init__(self, model, plan, caches):
        import dial_oracle as O

        self.O, self.model, self.plan, self.caches = O, model, plan, caches

    def stage_prepare(self, sids, positions):
        self.sids = list(np.asarray(sids))
        self.pos = list(np.asarray(positions))

    def stage_step_rows(self, off, rows, tokens, hidden, tokens_out=None):
        O, m, p = self.O, self.model, self.plan
        for r in range(off, off + rows):
            sid, pos = int(self.sids[r]), int(self.pos[r])
            if p.is_first:
                x = m.embed[[int(tokens[r - off])]]
            else:
                x = hidden[r - off:r - off + 1].numpy()
            for l in range(p.first_layer, p.first_layer + p.num_layers):
                x = O.layer_forward(x, m.layers[l], m.cfg, pos, l, self.caches[sid], m.cos, m.sin)
            hidden[r - off] = torch.from_numpy(np.ascontiguousarray(x[0], dtype=np.float32))
            if p.is_last:
                tokens_out[r - off] = O.argmax_first(O.model_logits(m, x[0]))
            self.pos[r] += 1


def _sessions(cfg, model, n):
    """Prompts of different lengths, their prefilled caches and first tokens
    (the single-process oracle)."""
    import dial_oracle as O

    rng = np.random.default_rng(8)
    prompts = [list(rng.integers(0, cfg.vocab, size=int(rng.integers(2, 9)))) for _ in range(n)]
    caches, first = [], []
    for pr in prompts:
        c = O.Cache(cfg.layers, cfg.max_seq_len)
        h = O.model_hidden(model, pr, 0, c)
        caches.append(c)
        first.append(O.argmax_first(O.model_logits(model, h[-1])))
    return prompts, caches, first


def _mb_worker(rank, world, port, n_sess, n_micro, n_iter, out_path):
    sys.path[:0] = [str(ROOT / "dial-27b_b200"), str(ROOT / "oracle"), str(ROOT / "tests")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import dial_oracle as O
    from dial_b200.pipeline import MicroBatchRunner, plan_stages

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        cfg = _cfg()
        model = O.synth_model(cfg, seed=3, std=0.05)
        prompts, caches, first = _sessions(cfg, model, n_sess)
        plan = plan_stages(cfg.layers, world)[rank]
        runner = MicroBatchRunner(OracleRowsStage(model, plan, caches), plan, cfg.hidden, n_sess,
                                  n_micro)
        runner.prepare(np.arange(n_sess), [len(p) for p in prompts], first)
        seen = []
        for _ in range(n_iter):
            runner.iteration()
            toks = runner.tokens()
            if rank == 0:
                seen.append(toks.copy())
        if rank == 0:
            np.save(out_path, np.stack(seen))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n_micro", [(1, 2), (2, 2), (3, 4), (2, 5)])
def test_micro_batched_ragged_sessions_match_single_process(tmp_path, world, n_micro):
    """5 sessions with prompts of different lengths, cut into micro-batches
    that are in flight on different stages: the tokens of every iteration
    equal each session's own greedy decode."""
    import dial_oracle as O

    n_sess, n_iter = 5, 3
    out = tmp_path / "mb.npy"
    mp.start_processes(_mb_worker, args=(world, _free_port(), n_sess, n_micro, n_iter, str(out)),
                       nprocs=world, start_method="spawn", join=True)
    got = np.load(out)
    cfg = _cfg()
    model = O.synth_model(cfg, seed=3, std=0.05)
    prompts, _, _ = _sessions(cfg, model, n_sess)
    for s, pr in enumerate(prompts):
        want, _ = O.greedy_generate(model, pr, n_iter + 1)
        np.testing.assert_array_equal(got[:, s], np.asarray(want[1:], dtype=np.int32))
