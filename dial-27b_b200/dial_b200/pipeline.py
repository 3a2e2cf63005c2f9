"""Pipeline stages over NCCL: the in-box replacement of DIAL's Master/Worker
layer handoff.

In the reference the Master ships the hidden state of a token to each remote
Worker that owns the next contiguous layer range and waits for it to come back
(spm/client.rs:391-453 `Client::forward_batch`, spm/worker.rs:670-893
`Worker::handle_master_client`), one TCP round trip per remote segment per
token.  Inside one box the topology's layer ranges become one process per GPU
(launched by torchrun) and the hidden state moves stage to stage with NCCL
send/recv over NVLink; the last stage runs the head and returns the sampled
token id to stage 0, which embeds it for the next step.  Everything is
stream-ordered: no host synchronisation happens inside a step, so the host of
every rank runs ahead and a stage's kernels start as soon as its input lands.

`StageRunner` drives one rank.  It only needs an engine with `embed`,
`forward_local_batch`, `head`, `dtype` and a torch device, so the same stage
logic runs on CPU with `gloo` ranks in the tests.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
import torch.distributed as dist

from .topology import Topology


@dataclass
class StagePlan:
    rank: int
    world: int
    first_layer: int
    num_layers: int

    @property
    def is_first(self) -> bool:
        return self.rank == 0

    @property
    def is_last(self) -> bool:
        return self.rank == self.world - 1


def plan_stages(num_layers: int, world: int, topology: Topology | None = None) -> list[StagePlan]:
    """Stage s owns one contiguous layer range: the topology's node ranges
    ordered by first layer (spm/topology.rs), or an even split."""
    topo = topology if topology is not None else Topology.even_split(num_layers, world)
    stages = topo.stages(num_layers)
    if len(stages) != world:
        raise ValueError(f"topology has {len(stages)} stages but the job has {world} ranks")
    return [StagePlan(r, world, first, count) for r, (_, first, count) in enumerate(stages)]


class StageRunner:
    """One pipeline stage on one rank (one GPU)."""

    def __init__(self, engine, plan: StagePlan, hidden_size: int, session: int = 0,
                 group=None):
        self.eng = engine
        self.plan = plan
        self.H = hidden_size
        self.session = session
        self.group = group
        self.device = getattr(engine, "torch_device", None) or torch.device("cuda", engine.device)
        self.dtype = engine.dtype
        self._batch_names = [f"model.layers.{i}" for i in
                             range(plan.first_layer, plan.first_layer + plan.num_layers)]

    def _batch(self, index_pos: int):
        first = self.plan.first_layer
        return [(n, index_pos, first + i) for i, n in enumerate(self._batch_names)]

    def _send(self, t: torch.Tensor, dst: int):
        dist.send(t, dst, group=self.group)

    def _recv(self, t: torch.Tensor, src: int):
        dist.recv(t, src, group=self.group)

    def step(self, tokens: torch.Tensor | None, rows: int, index_pos: int) -> torch.Tensor | None:
        """Run `rows` tokens starting at `index_pos` through this stage with the
        engine's layer-range call (prefill, or decode without graphs).

        Stage 0 takes the token ids (device int32 [rows]) and returns the next
        token id (device int32 [1]) once the last stage sends it back; the
        other stages return None (the last stage returns its token too)."""
        p = self.plan
        if p.is_first:
            x = self.eng.embed(tokens)
        else:
            x = torch.empty(rows, self.H, dtype=self.dtype, device=self.device)
            self._recv(x, p.rank - 1)
        x = self.eng.forward_local_batch(x, self._batch(index_pos), self.session)
        tok = None
        if not p.is_last:
            self._send(x, p.rank + 1)
        else:
            tok = self.eng.head(x[rows - 1:rows].contiguous())
            if p.world > 1:
                self._send(tok, 0)
        if p.is_first and p.world > 1:
            tok = torch.empty(1, dtype=torch.int32, device=self.device)
            self._recv(tok, p.world - 1)
        return tok

    # ------------------------------------------------------- graph decode
    @property
    def graphs(self) -> bool:
        return hasattr(self.eng, "stage_step")

    def decode_prepare(self, index_pos: int):
        """Fix the decode buffers and put the position on the device (engines
        with stage_step: every later decode_step is one graph launch with no
        host synchronisation)."""
        self.pos = index_pos
        if self.graphs:
            self.eng.stage_prepare([self.session], [index_pos])
            if not hasattr(self, "_x"):  # fixed buffers: the stage graph is captured once
                self._x = torch.empty(1, self.H, dtype=self.dtype, device=self.device)
                self._tok_in = torch.zeros(1, dtype=torch.int32, device=self.device)
                self._tok_out = torch.zeros(1, dtype=torch.int32, device=self.device)

    def decode_step(self, token: torch.Tensor | None) -> torch.Tensor | None:
        """One bs1 decode token through this stage; stage 0 passes the current
        token (device int32 [1]) and gets the next one back."""
        if not self.graphs:
            tok = self.step(token, 1, self.pos)
            self.pos += 1
            return tok
        p, x = self.plan, self._x
        if p.is_first:
            if token is not None and token.data_ptr() != self._tok_in.data_ptr():
                self._tok_in.copy_(token)
        else:
            self._recv(x, p.rank - 1)
        self.eng.stage_step(1, self._tok_in if p.is_first else None, x,
                            self._tok_out if p.is_last else None)
        self.pos += 1
        tok = None
        if not p.is_last:
            self._send(x, p.rank + 1)
        else:
            tok = self._tok_out
            if p.world > 1:
                self._send(tok, 0)
        if p.is_first:
            if p.world > 1:
                self._recv(self._tok_in, p.world - 1)
            else:
                self._tok_in.copy_(self._tok_out)
            tok = self._tok_in
        return tok

    # ------------------------------------------------ peer-memory stage link
    def link(self):
        """Open the peer-memory stage link (collective over the group): every
        rank publishes its inbox's IPC handle, stage s maps stage s + 1's and
        the last stage maps stage 0's.  Afterwards decode_linked runs the
        decode loop with no NCCL call and no host synchronisation per token."""
        p = self.plan
        try:
            mine = self.eng.stage_link_handle()
        except Exception:  # noqa: BLE001  (every rank still joins the exchange below)
            mine = None
        handles = [None] * p.world
        dist.all_gather_object(handles, mine, group=self.group)
        if any(h is None for h in handles):
            raise RuntimeError("a stage could not export its link inbox")
        self.eng.stage_link_open(None if p.is_last else handles[p.rank + 1],
                                 handles[0] if p.is_last else None)
        self.linked = True

    def decode_linked(self, token: torch.Tensor | None, n_steps: int) -> int | None:
        """`n_steps` bs1 decode tokens over the stage link from position
        decode_prepare set; stage 0 passes the first token (device int32 [1])
        and gets the last sampled token id back (host int), others None."""
        p = self.plan
        for i in range(n_steps):
            self.eng.stage_link_step(1, token if (p.is_first and i == 0) else None)
        self.pos += n_steps
        if p.is_first:
            return int(self.eng.stage_link_finish(1)[0])
        return None

    def generate(self, prompt, n_gen: int) -> np.ndarray | None:
        """Greedy generation of `n_gen` tokens after `prompt` (host ids on
        stage 0; ignored elsewhere).  Returns the ids on stage 0, else None."""
        n = len(prompt)
        toks = None
        if self.plan.is_first:
            toks = torch.as_tensor(np.asarray(prompt, dtype=np.int32), device=self.device)
        tok = self.step(toks, n, 0)
        out = [tok.clone() if tok is not None else None]
        self.decode_prepare(n)
        for _ in range(1, n_gen):
            tok = self.decode_step(tok if self.plan.is_first else None)
            out.append(tok.clone() if tok is not None else None)
        if self.plan.is_first:
            return torch.cat(out).cpu().numpy()
        return None


class MicroBatchRunner:
    """Ragged multi-session decode pipelined over the stages.

    The decode rows (one per session) are cut into ``n_micro`` contiguous
    micro-batches; on every rank an iteration runs the micro-batches in order,
    each as one graph-captured stage step (``Engine.stage_step_rows``), with
    the hidden state of micro-batch j handed to the next stage while this
    stage already works on j + 1.  The last stage returns each micro-batch's
    sampled tokens to stage 0, which embeds them in the next iteration.  With
    ``n_micro`` >= the number of stages every stage is busy in the steady
    state.  This is the in-box form of the reference Worker serving one
    layer range for many Master connections at once (spm/worker.rs:316-325,
    899-912), each connection's hop replaced by a send/recv between GPUs.

    The engine needs ``stage_prepare``, ``stage_step_rows``, ``dtype`` and a
    device; the same logic runs on CPU with ``gloo`` ranks in the tests.
    """

    def __init__(self, engine, plan: StagePlan, hidden_size: int, n_rows: int, n_micro: int,
                 group=None):
        if not 1 <= n_micro <= n_rows:
            raise ValueError(f"n_micro must be in [1, {n_rows}], got {n_micro}")
        self.eng, self.plan, self.H, self.group = engine, plan, hidden_size, group
        self.device = getattr(engine, "torch_device", None) or torch.device("cuda", engine.device)
        self.dtype = engine.dtype
        bounds = [n_rows * j // n_micro for j in range(n_micro + 1)]
        self.micro = [(bounds[j], bounds[j + 1] - bounds[j]) for j in range(n_micro)]
        mk = lambda rows, **kw: torch.zeros(rows, **kw, device=self.device)  # noqa: E731
        self._h = [mk(r, dtype=self.dtype).reshape(r, 1).expand(r, hidden_size).contiguous()
                   for _, r in self.micro]
        self._tok_in = [mk(r, dtype=torch.int32) for _, r in self.micro]
        self._tok_out = [mk(r, dtype=torch.int32) for _, r in self.micro]
        self._pending = False  # stage 0 owes receives of the last iteration's tokens
        # sends are asynchronous (only receives block, so no two ranks can wait
        # on each other's sends); a buffer is rewritten only after its send
        self._sent = [None] * n_micro

    def prepare(self, sids, positions, tokens=None):
        """Sessions and positions of all rows (host arrays); stage 0 also takes
        the rows' current token ids."""
        self.finish()
        self.eng.stage_prepare(sids, positions)
        if self.plan.is_first:
            t = torch.as_tensor(np.asarray(tokens, dtype=np.int32))
            for (off, rows), buf in zip(self.micro, self._tok_in):
                buf.copy_(t[off:off + rows])

    def _recv(self, t, src):
        dist.recv(t, src, group=self.group)

    def _sent_wait(self, j):
        if self._sent[j] is not None:
            self._sent[j].wait()
            self._sent[j] = None

    def iteration(self):
        """One decode token for every row, micro-batch by micro-batch."""
        p = self.plan
        for j, (off, rows) in enumerate(self.micro):
            h = self._h[j]
            self._sent_wait(j)  # h (or the last stage's tokens) is rewritten below
            if p.is_first:
                if self._pending:
                    self._recv(self._tok_in[j], p.world - 1)
            else:
                self._recv(h, p.rank - 1)
            self.eng.stage_step_rows(off, rows, self._tok_in[j] if p.is_first else None, h,
                                     self._tok_out[j] if p.is_last else None)
            if not p.is_last:
                self._sent[j] = dist.isend(h, p.rank + 1, group=self.group)
            elif p.world > 1:
                self._sent[j] = dist.isend(self._tok_out[j], 0, group=self.group)
            else:
                self._tok_in[j].copy_(self._tok_out[j])
        self._pending = p.is_first and p.world > 1

    def finish(self):
        """Complete every send and, on stage 0, receive the tokens of the last
        iteration (before the next prepare or the end of the run)."""
        if self._pending:
            for j in range(len(self.micro)):
                self._recv(self._tok_in[j], self.plan.world - 1)
            self._pending = False
        for j in range(len(self.micro)):
            self._sent_wait(j)

    def tokens(self) -> np.ndarray | None:
        """Stage 0: the rows' current token ids (after finish())."""
        if not self.plan.is_first:
            return None
        self.finish()
        return torch.cat(self._tok_in).cpu().numpy()
