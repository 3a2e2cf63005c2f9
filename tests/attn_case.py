"""Shared paged-KV decode attention cases for the GPU tests: a random
problem, its oracle answer (text.rs:1466-1536, cache.rs:169-237,
text.rs:1258-1281) and the tolerance the fused op is held to."""

import numpy as np
import torch

import dial_oracle as O


class PagedCase:
    """Random paged-KV problem: `rows` decode tokens, one per session, at the
    given positions; pages hold random (already normed/rotated) history."""

    def __init__(self, q_heads, kv_heads, positions, seed=0, max_pos=1024, dtype="bf16"):
        rng = np.random.default_rng(seed)
        self.act = dtype
        self.QH, self.KVH, self.D = q_heads, kv_heads, 128
        self.positions = np.asarray(positions, np.int32)
        self.rows = len(positions)
        self.max_pos = max_pos
        self.max_blocks = (max_pos + 15) // 16
        nb = self.rows * self.max_blocks
        self.block_table = rng.permutation(nb).astype(np.int32).reshape(self.rows, self.max_blocks)
        r = lambda *s: O.act_round(rng.standard_normal(s).astype(np.float32), dtype)  # noqa: E731
        self.k_pages = r(nb, kv_heads, 16, 128)
        self.v_pages = r(nb, kv_heads, 16, 128)
        self.qkv = r(self.rows, (q_heads + 2 * kv_heads) * 128)
        self.q_norm = O.act_round(1.0 + 0.1 * rng.standard_normal(128).astype(np.float32), dtype)
        self.k_norm = O.act_round(1.0 + 0.1 * rng.standard_normal(128).astype(np.float32), dtype)
        self.eps = 1e-6
        self.cos, self.sin = O.rope_tables(128, max_pos, 1e6, dtype)

    def session_kv(self, pages, m, length):
        bt = self.block_table[m]
        toks = [pages[bt[p // 16], :, p % 16] for p in range(length)]
        return np.stack(toks, axis=1) if toks else np.zeros((self.KVH, 0, 128), np.float32)

    def oracle(self, round_probs=False):
        """Expected (out [rows, QH*128], new k [rows, KVH, 128], new v)."""
        QH, KVH, D, act = self.QH, self.KVH, self.D, self.act
        outs, ks, vs = [], [], []
        for m, pos in enumerate(self.positions):
            row = self.qkv[m]
            q = row[: QH * D].reshape(QH, 1, D)
            k = row[QH * D:(QH + KVH) * D].reshape(KVH, 1, D)
            v = row[(QH + KVH) * D:].reshape(KVH, 1, D)
            c, s = self.cos[pos:pos + 1], self.sin[pos:pos + 1]
            qn = O.rope(O.rms_norm(q, self.q_norm, self.eps, act), c, s, act)
            kn = O.rope(O.rms_norm(k, self.k_norm, self.eps, act), c, s, act)
            K = np.concatenate([self.session_kv(self.k_pages, m, pos), kn], axis=1)
            V = np.concatenate([self.session_kv(self.v_pages, m, pos), v], axis=1)
            o = O.attention(qn, K, V, causal=False, act=act, round_probs=round_probs)
            outs.append(o.reshape(QH * D))
            ks.append(kn[:, 0])
            vs.append(v[:, 0])
        return np.stack(outs), np.stack(ks), np.stack(vs)

    def device(self, cuda):
        dt = torch.bfloat16 if self.act == "bf16" else torch.float16
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda).to(dt)  # noqa: E731
        i = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
        return dict(qkv=t(self.qkv), q_norm_w=t(self.q_norm), k_norm_w=t(self.k_norm),
                    cos=t(self.cos), sin=t(self.sin), k_pages=t(self.k_pages),
                    v_pages=t(self.v_pages), block_table=i(self.block_table),
                    sids=i(np.arange(self.rows, dtype=np.int32)), positions=i(self.positions),
                    out=torch.zeros(self.rows, self.QH * 128, dtype=dt, device=cuda))

    def new_kv(self, k_pages, v_pages):
        k = k_pages.float().cpu().numpy()
        v = v_pages.float().cpu().numpy()
        ks, vs = [], []
        for m, pos in enumerate(self.positions):
            b = self.block_table[m, pos // 16]
            ks.append(k[b, :, pos % 16])
            vs.append(v[b, :, pos % 16])
        return np.stack(ks), np.stack(vs)


def ulp(x, act):
    mant = 7 if act == "bf16" else 10
    mag = np.maximum(np.abs(x), 2.0 ** -14)
    return np.exp2(np.floor(np.log2(mag)) - mant)


def assert_attn_close(got, ref, act):
    """Attention output against the f32-probability oracle: the GPU rounds
    once per output element like the oracle but sums in another order, so
    max |d| <= 2^-6 max|ref| and >= 99% of elements within 2 ulp of
    max(|ref|, rms(ref))."""
    d = np.abs(got - ref)
    scale = float(np.max(np.abs(ref)))
    rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
    assert float(d.max()) <= 2 ** -6 * scale + 1e-3, f"max |d| {d.max()} vs {scale}"
    assert np.mean(d <= 2 * ulp(np.maximum(np.abs(ref), rms), act)) >= 0.99


def run(case, cuda, splits, calls=1, num_blocks=0):
    """num_blocks > 0 passes the pool size (the tensor-core form for more
    than 4 rows)."""
    from dial_b200 import attention as A

    dt = torch.bfloat16 if case.act == "bf16" else torch.float16
    sh = A.make_shape(case.QH, case.KVH, case.max_blocks, case.max_pos, case.eps, dt,
                      num_blocks=num_blocks)
    dev = case.device(cuda)
    nbytes = A.scratch_bytes(sh, case.rows, splits)
    scratch = torch.zeros(max(nbytes, 16), dtype=torch.uint8, device=cuda) if splits > 1 else None
    outs = []
    for _ in range(calls):
        A.attention_decode(sh, splits=splits, scratch=scratch, **dev)
        torch.cuda.synchronize()
        outs.append(dev["out"].float().cpu().numpy())
    return outs, dev, sh
