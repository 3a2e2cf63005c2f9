"""Pipeline-stage decode (dial_b200_stage_prepare / dial_b200_stage_step) on
one GPU: two engines that each own half of the layers, chained on one stream,
must produce the same greedy tokens as one engine that owns the whole model
(the Master -> Worker hop of spm/client.rs:391-453 replaced by a device
copy), and a 2-GPU NCCL run of dial_b200.pipeline must do the same."""

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def _cfg(dial_b200, **kw):
    base = dict(hidden_size=512, intermediate_size=1024, vocab_size=2000, num_hidden_layers=4,
                num_attention_heads=4, num_key_value_heads=1, max_seq_len=256, max_sessions=1,
                max_tokens=64)
    base.update(kw)
    return dial_b200.Config(**base)


def test_two_stage_engines_match_whole_model(cuda):
    import dial_b200

    cfg = _cfg(dial_b200)
    prompt = np.random.default_rng(5).integers(0, cfg.vocab_size, size=9).astype(np.int32)
    n_gen = 12
    full = dial_b200.Engine(cfg)
    full.load_synthetic(seed=7)
    want, _, _ = full.generate(prompt, n_gen)

    a = dial_b200.Engine(cfg, first_layer=0, num_layers=2)
    b = dial_b200.Engine(cfg, first_layer=2, num_layers=2)
    a.load_synthetic(seed=7)
    b.load_synthetic(seed=7)
    n = len(prompt)
    x = a.embed(torch.as_tensor(prompt, device=cuda))
    a.forward_local_batch(x, [(f"model.layers.{i}", 0, i) for i in range(2)])
    b.forward_local_batch(x, [(f"model.layers.{i}", 0, i) for i in range(2, 4)])
    tok_in = b.head(x[n - 1:n].contiguous())
    got = [int(tok_in.item())]
    a.stage_prepare([0], [n])
    b.stage_prepare([0], [n])
    h = torch.empty(1, cfg.hidden_size, dtype=torch.bfloat16, device=cuda)
    tok_out = torch.zeros(1, dtype=torch.int32, device=cuda)
    seq = []
    for _ in range(n_gen - 1):
        a.stage_step(1, tok_in, h)
        b.stage_step(1, None, h, tok_out)
        tok_in.copy_(tok_out)
        seq.append(tok_in.clone())
    torch.cuda.synchronize()
    got += [int(t.item()) for t in seq]
    assert dial_b200.device_status() == 0
    np.testing.assert_array_equal(np.asarray(got, np.int32), want)


def test_stage_step_argument_checks(cuda):
    import dial_b200

    cfg = _cfg(dial_b200)
    a = dial_b200.Engine(cfg, first_layer=0, num_layers=2)
    a.load_synthetic(seed=1)
    h = torch.empty(1, cfg.hidden_size, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(dial_b200.DialError, match="first stage needs device token ids"):
        a.stage_step(1, None, h)
    with pytest.raises(dial_b200.DialError, match="outside the KV capacity"):
        a.stage_prepare([0], [cfg.max_seq_len])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, prompt, n_gen, out_path):
    sys.path[:0] = [str(ROOT / "dial-27b_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch.distributed as dist

    import dial_b200
    from dial_b200.pipeline import StageRunner, plan_stages

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        cfg = _cfg(dial_b200)
        plan = plan_stages(cfg.num_hidden_layers, world)[rank]
        eng = dial_b200.Engine(cfg, first_layer=plan.first_layer, num_layers=plan.num_layers,
                               device=rank)
        eng.load_synthetic(seed=7)
        runner = StageRunner(eng, plan, cfg.hidden_size)
        toks = runner.generate(prompt, n_gen)
        torch.cuda.synchronize()
        if rank == 0:
            np.save(out_path, toks)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_nccl_pipeline_two_gpus_matches_whole_model(cuda, tmp_path):
    import torch.multiprocessing as mp

    import dial_b200

    cfg = _cfg(dial_b200)
    prompt = np.random.default_rng(5).integers(0, cfg.vocab_size, size=9).astype(np.int32)
    full = dial_b200.Engine(cfg)
    full.load_synthetic(seed=7)
    want, _, _ = full.generate(prompt, 12)
    out = tmp_path / "toks.npy"
    mp.start_processes(_nccl_worker, args=(2, _free_port(), prompt, 12, str(out)), nprocs=2,
                       start_method="spawn", join=True)
    np.testing.assert_array_equal(np.load(out), want)


def _link_worker(rank, world, port, prompt, n_gen, out_path):
    sys.path[:0] = [str(ROOT / "dial-27b_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch.distributed as dist

    import dial_b200
    from dial_b200.pipeline import StageRunner, plan_stages

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        cfg = _cfg(dial_b200)
        plan = plan_stages(cfg.num_hidden_layers, world)[rank]
        eng = dial_b200.Engine(cfg, first_layer=plan.first_layer, num_layers=plan.num_layers,
                               device=rank)
        eng.load_synthetic(seed=7)
        runner = StageRunner(eng, plan, cfg.hidden_size)
        runner.link()
        n = len(prompt)
        toks = torch.as_tensor(prompt, device=f"cuda:{rank}") if plan.is_first else None
        first = runner.step(toks, n, 0)  # prefill through the NCCL path
        first_dev = first.clone() if plan.is_first else None
        # one linked run of n_gen - 1 steps: the tokens stay on the devices
        runner.decode_prepare(n)
        last = runner.decode_linked(first_dev, n_gen - 1)
        # token by token (a run of one step each): every sampled id reaches the host
        runner.decode_prepare(n)
        seq, tok = [], first_dev
        for _ in range(n_gen - 1):
            t = runner.decode_linked(tok, 1)
            if plan.is_first:
                seq.append(t)
                tok = torch.tensor([t], dtype=torch.int32, device=f"cuda:{rank}")
        torch.cuda.synchronize()
        assert dial_b200.device_status() == 0
        if rank == 0:
            np.save(out_path, np.asarray([int(first.item())] + seq + [last], np.int32))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_link_pipeline_two_gpus_matches_whole_model(cuda, tmp_path):
    """The peer-memory stage link (dial_b200_stage_link_*): a linked run keeps
    the tokens on the devices and its last token, and a run of one-step runs
    returns every token, both equal to the whole-model engine's greedy decode."""
    import torch.multiprocessing as mp

    import dial_b200

    cfg = _cfg(dial_b200)
    prompt = np.random.default_rng(6).integers(0, cfg.vocab_size, size=9).astype(np.int32)
    n_gen = 12
    full = dial_b200.Engine(cfg)
    full.load_synthetic(seed=7)
    want, _, _ = full.generate(prompt, n_gen)
    out = tmp_path / "link.npy"
    mp.start_processes(_link_worker, args=(2, _free_port(), prompt, n_gen, str(out)), nprocs=2,
                       start_method="spawn", join=True)
    got = np.load(out)
    np.testing.assert_array_equal(got[:n_gen], want)
    assert got[n_gen] == want[-1]
