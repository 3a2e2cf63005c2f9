"""Full-size parity of the headline model on the GPU.

Qwen3-8B architecture (36 layers, hidden 4096, 32 q / 8 kv heads, FFN 12288,
vocab 151936), bf16 weights N(0, 0.02) from seed 0 generated on the device,
every layer linear W8A16 (worker_w8a16.rs:330-341), bf16 lm_head; prompt of
128 seed-1 token ids; greedy decode (qwen3_vl.rs:138-143, 2018-2177,
3276-3331).  The expected values are tests/golden/config1_qwen3_8b_w8a16.npz,
written by tests/golden/make_config1.py from the C++ oracle.

What the fixture shows about this synthetic model: it is chaotic.  Two
correct CPU evaluations that differ only in summation order (f64 vs f32
accumulation) move the top logits by up to 0.156 (``logit_spread``) and pick
different argmaxes at 2 of 32 teacher-forced steps; bf16 logits near 5.4 are
spaced 2^-5 apart, and exact top-2 ties occur (margin 0 at steps 4 and 13 of
the f32-probability run).  So the checks are:

* each layer alone, from the oracle's input (layers 17 and 35: a 32-token
  prefill then one decode token), within the single-layer tolerance of the
  small-shape tests;
* the free-running hidden state after layers 0, 17 and 35 (prefill and the
  first decode step) within twice the drift between the two oracle runs
  (bf16 vs f32 softmax probabilities) at that depth;
* teacher-forced greedy tokens: identical wherever the oracle's top-1 minus
  top-2 margin exceeds TOKEN_BOUND = 0.25 logit (8 bf16 ulps at |logit| in
  [4, 8), above twice the largest f32-vs-f64 accumulation spread); at the
  other steps the GPU's token must be within TOKEN_BOUND of the oracle's best
  logit;
* free-running generation through the public API (dial_b200_generate)
  repeats the teacher-forced GPU tokens up to and including the first step
  where those differ from the oracle's (until then both runs have the same
  inputs).
"""

from pathlib import Path

import numpy as np
import pytest
import torch

import dial_oracle as O
from test_layer_gpu import assert_hidden_close

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden" / "config1_qwen3_8b_w8a16.npz"
TOKEN_BOUND = 0.25
N_ISO = 32  # rows of the isolated-layer prefill; row N_ISO is the decode token


@pytest.fixture(scope="module")
def fix():
    return dict(np.load(GOLDEN))


@pytest.fixture(scope="module")
def engine(cuda):
    import dial_b200

    cfg = dial_b200.Config(max_seq_len=256, max_sessions=1, max_tokens=128)
    eng = dial_b200.Engine(cfg)
    eng.load_synthetic(seed=0)
    yield eng
    eng.close()


def _h(bits) -> np.ndarray:
    return O.bf16_from_bits(bits)


def _drift_close(got, ref, alt, what):
    """|got - ref| within twice the oracle's own drift |alt - ref| (mean and
    max), with the single-layer tolerance as the floor."""
    d = np.abs(got - ref)
    drift = np.abs(alt - ref)
    rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
    mean_bound = max(2 * float(drift.mean()), 2 ** -7 * rms)
    max_bound = max(2 * float(drift.max()), 2 ** -5 * float(np.abs(ref).max()) + 1e-3)
    assert float(d.mean()) <= mean_bound, f"{what}: mean |d| {d.mean():.4g} > {mean_bound:.4g}"
    assert float(d.max()) <= max_bound, f"{what}: max |d| {d.max():.4g} > {max_bound:.4g}"
    return float(d.mean()) / rms


def _token_ok(fix, step, tok):
    ids, lg, margin = fix["top_ids_f32p"][step], fix["top_logits_f32p"][step], \
        float(fix["margin_f32p"][step])
    if tok == int(ids[0]):
        return True
    if margin > TOKEN_BOUND:
        return False
    hit = np.nonzero(ids == tok)[0]
    return hit.size > 0 and float(lg[0] - lg[hit[0]]) <= TOKEN_BOUND


def test_config1_free_running_hidden_and_teacher_forced_tokens(cuda, engine, fix):
    import dial_b200

    eng = engine
    rows = fix["prefill_rows"]
    prompt = torch.as_tensor(fix["prompt"], dtype=torch.int32, device=cuda)
    # prefill through the Forwarder API one layer at a time (index_pos 0)
    x = eng.embed(prompt)
    caps = {}
    for l in range(36):
        eng.forward(x, 0, l)
        if l in (0, 17, 35):
            caps[l] = x[torch.as_tensor(rows, device=cuda)].float().cpu().numpy()
    tok0, logits0 = eng.head(x[-1:].contiguous(), return_logits=True)
    # first decode step (position 128) from the oracle's first token
    y = eng.embed(torch.as_tensor(fix["tokens_f32p"][:1], dtype=torch.int32, device=cuda))
    caps1 = {}
    for l in range(36):
        eng.forward(y, 128, l)
        if l in (0, 17, 35):
            caps1[l] = y.float().cpu().numpy()
    tok1 = eng.head(y)
    torch.cuda.synchronize()
    assert dial_b200.device_status() == 0

    # layer 0 has no accumulated drift: the single-layer tolerance holds
    assert_hidden_close(caps[0], _h(fix["prefill_l0_f32p"]))
    assert_hidden_close(caps1[0], _h(fix["step1_l0_f32p"]))
    rel = {}
    for l in (17, 35):
        rel[l] = _drift_close(caps[l], _h(fix[f"prefill_l{l}_f32p"]), _h(fix[f"prefill_l{l}"]),
                              f"prefill after layer {l}")
        _drift_close(caps1[l], _h(fix[f"step1_l{l}_f32p"]), _h(fix[f"step1_l{l}"]),
                     f"decode step 1 after layer {l}")

    # logits of the prefill's last row at the oracle's top ids
    got_lg = logits0.float().cpu().numpy()[0][fix["top_ids_f32p"][0]]
    assert np.max(np.abs(got_lg - fix["top_logits_f32p"][0])) <= TOKEN_BOUND

    # teacher-forced greedy tokens through dial_b200_decode_step
    toks = [int(tok0.cpu()[0]), int(tok1.cpu()[0])]
    forced = fix["tokens_f32p"]
    for s in range(2, int(fix["n_gen"])):
        toks.append(int(eng.decode_step([int(forced[s - 1])], [0], [128 + s - 1])[0]))
    assert dial_b200.device_status() == 0
    bad = [s for s, t in enumerate(toks) if not _token_ok(fix, s, t)]
    exact = sum(int(t == int(forced[s])) for s, t in enumerate(toks))
    assert not bad, (f"steps {bad} disagree beyond the bound; gpu {toks}, oracle "
                     f"{forced.tolist()}, margins {fix['margin_f32p'].tolist()}")
    print(f"config1 tokens: {exact}/32 identical to the oracle (teacher-forced); "
          f"hidden drift after layer 17 / 35: {rel[17]:.4f} / {rel[35]:.4f} of rms")

    # free-running generation through the public API
    eng.session_reset(0)
    out, _, _ = eng.generate(fix["prompt"], int(fix["n_gen"]))
    first_div = next((s for s, t in enumerate(toks) if t != int(forced[s])), len(toks) - 1)
    assert out[:first_div + 1].tolist() == toks[:first_div + 1]
    assert dial_b200.device_status() == 0


def test_config1_isolated_layers(cuda, engine, fix):
    """Layers 17 and 35 from the oracle's own inputs: prefill of rows 0..31
    (index_pos 0 replaces that layer's cache), then row 32 as a decode token
    at position 32; by causality the outputs equal the oracle's rows 0..32
    after that layer."""
    import dial_b200

    eng = engine
    rows = list(fix["prefill_rows"])
    sel = [rows.index(i) for i in range(N_ISO + 1)]
    for l in (17, 35):
        inp = _h(fix[f"prefill_l{l - 1}_f32p"])[sel]
        want = _h(fix[f"prefill_l{l}_f32p"])[sel]
        x = torch.from_numpy(inp[:N_ISO]).to(cuda).to(torch.bfloat16).contiguous()
        eng.forward(x, 0, l)
        y = torch.from_numpy(inp[N_ISO:]).to(cuda).to(torch.bfloat16).contiguous()
        eng.forward(y, N_ISO, l)
        torch.cuda.synchronize()
        assert dial_b200.device_status() == 0
        assert_hidden_close(x.float().cpu().numpy(), want[:N_ISO])
        assert_hidden_close(y.float().cpu().numpy(), want[N_ISO:])
