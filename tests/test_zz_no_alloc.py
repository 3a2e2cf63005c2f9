"""dial_b200_attention_decode_noalloc (static device scratch, no allocation)
against dial_b200_attention_decode (caller scratch) and the oracle.

Named to be collected last so it also runs after every other GPU test; it
sets up nothing that other tests share and passes alone."""

import numpy as np
import pytest
import torch

from attn_case import PagedCase, assert_attn_close

pytestmark = pytest.mark.gpu


def _both(case, cuda, splits):
    from dial_b200 import attention as A

    sh = A.make_shape(case.QH, case.KVH, case.max_blocks, case.max_pos, case.eps)
    dev = case.device(cuda)
    scratch = torch.zeros(max(A.scratch_bytes(sh, case.rows, splits), 16), dtype=torch.uint8,
                          device=cuda)
    A.attention_decode(sh, splits=splits, scratch=scratch, **dev)
    torch.cuda.synchronize()
    want = dev["out"].float().cpu().numpy()

    dev2 = case.device(cuda)
    got = []
    for _ in range(2):
        dev2["out"].zero_()
        A.attention_decode_noalloc(sh, splits=splits, **dev2)
        torch.cuda.synchronize()
        got.append(dev2["out"].float().cpu().numpy())
    return want, got, dev, dev2


@pytest.mark.parametrize("splits", [1, 8])
def test_noalloc_matches_scratch_entry_point_twice(cuda, splits):
    case = PagedCase(32, 8, [700, 3, 150, 64], seed=21)
    want, got, dev, dev2 = _both(case, cuda, splits)
    ref, _, _ = case.oracle()
    for g in got:
        np.testing.assert_allclose(g, want, rtol=2 ** -7, atol=1e-3)
        assert_attn_close(g, ref, "bf16")
    # the pages the two entry points appended to agree as well
    assert torch.equal(dev["k_pages"], dev2["k_pages"])
    assert torch.equal(dev["v_pages"], dev2["v_pages"])


def test_noalloc_at_the_limit_and_beyond(cuda):
    import dial_b200
    from dial_b200 import attention as A

    # 4 rows x 32 q heads x 16 splits = 2048 partial rows: exactly the limit
    case = PagedCase(32, 8, [1000, 900, 800, 700], seed=3)
    want, got, _, _ = _both(case, cuda, 16)
    for g in got:
        np.testing.assert_allclose(g, want, rtol=2 ** -7, atol=1e-3)

    dev = case.device(cuda)
    sh = A.make_shape(32, 8, case.max_blocks, case.max_pos)
    with pytest.raises(dial_b200.DialError, match="static scratch limit of 2048"):
        A.attention_decode_noalloc(sh, splits=17, **dev)
