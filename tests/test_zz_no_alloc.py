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


STATUS_BAD_ARGS = 0x104  # kStatusBadArgs (csrc/common.cuh)


def test_noalloc_host_rejection_leaves_device_status_clear(cuda):
    """An argument the host side rejects never reaches the GPU: the call
    raises, writes nothing and leaves the device status at zero."""
    import dial_b200
    from dial_b200 import attention as A

    dial_b200.device_status(clear=True)
    case = PagedCase(32, 8, [100, 5], seed=5)
    dev = case.device(cuda)
    sh = A.make_shape(32, 8, case.max_blocks, case.max_pos)
    with pytest.raises(dial_b200.DialError, match="splits 0 outside"):
        A.attention_decode_noalloc(sh, splits=0, **dev)
    bad_shape = A.make_shape(32, 6, case.max_blocks, case.max_pos)
    with pytest.raises(dial_b200.DialError, match="multiple of kv_heads"):
        A.attention_decode_noalloc(bad_shape, splits=4, **dev)
    torch.cuda.synchronize()
    assert dial_b200.device_status() == 0
    assert not bool(torch.any(dev["out"] != 0))


def test_noalloc_position_beyond_capacity_reports_status(cuda):
    """A row at a position outside max_pos: the kernel records the bad-argument
    status and skips that row's KV append (the other row appends normally);
    dial_b200_device_status reports the status of this entry point, clearing
    it resets the static split counters, and the next calls match the scratch
    entry point again."""
    import dial_b200
    from dial_b200 import attention as A

    dial_b200.device_status(clear=True)
    case = PagedCase(32, 8, [200, 40], seed=6, max_pos=512)
    dev = case.device(cuda)
    sh = A.make_shape(32, 8, case.max_blocks, case.max_pos)
    k0, v0 = dev["k_pages"].clone(), dev["v_pages"].clone()
    bad = dev["positions"].clone()
    bad[1] = case.max_pos
    A.attention_decode_noalloc(sh, splits=8, **{**dev, "positions": bad})
    torch.cuda.synchronize()
    assert dial_b200.device_status() == STATUS_BAD_ARGS
    # only row 0's slot (position 200 of session 0) changed in the pages
    b0, t0 = int(case.block_table[0, 200 // 16]), 200 % 16
    for new, old in ((dev["k_pages"], k0), (dev["v_pages"], v0)):
        changed = (new != old).any(dim=3).any(dim=1)  # [blocks, 16 tokens]
        assert bool(changed[b0, t0])
        changed[b0, t0] = False
        assert not bool(changed.any())
    assert dial_b200.device_status(clear=True) == STATUS_BAD_ARGS
    assert dial_b200.device_status() == 0
    want, got, _, _ = _both(case, cuda, 8)
    for g in got:
        np.testing.assert_allclose(g, want, rtol=2 ** -7, atol=1e-3)
    assert dial_b200.device_status() == 0
