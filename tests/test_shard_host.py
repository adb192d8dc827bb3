"""Host-side sequence sharding (dgx_monarch_b200/shard.py) against the oracle:
the zero pad and the per-rank chunk of adapters/base.py:48-123, and the typed
refusal of an indivisible stream that must not pad."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import usp


@pytest.mark.parametrize("length,world", [(7, 2), (9, 3), (8, 4), (1, 8), (1216, 8)])
def test_shard_seq_matches_the_oracle(length, world):
    from dgx_monarch_b200.shard import shard_seq

    x = torch.randn(2, length, 3, dtype=torch.float64)
    for rank in range(world):
        local, orig = shard_seq(x, world, rank)
        want, want_orig = usp.shard_seq(x.numpy(), world, rank)
        assert orig == want_orig == length
        np.testing.assert_array_equal(local.numpy(), want)


def test_shard_then_oracle_gather_round_trips():
    from dgx_monarch_b200.shard import shard_seq

    x = torch.randn(1, 13, 4, dtype=torch.float64)
    chunks = [shard_seq(x, 4, r)[0].numpy() for r in range(4)]
    np.testing.assert_array_equal(usp.sp_gather(chunks, 13), x.numpy())


def test_indivisible_stream_that_must_not_pad_is_refused():
    from dgx_monarch_b200.shard import ShardRefusal, pad_seq_to_multiple, shard_seq

    x = torch.zeros(1, 10, 2)
    with pytest.raises(ShardRefusal, match="text stream length 10"):
        shard_seq(x, 4, 0, allow_padding=False, name="text")
    assert shard_seq(None, 4, 0) == (None, 0)
    padded, orig = pad_seq_to_multiple(x, 4)
    assert padded.shape == (1, 12, 2) and orig == 10


def test_dual_model_cfg_refuses_a_guidance_scale_of_one():
    """actor/dual_model_cfg.py:122-130: at cfg 1.0 the unconditional rank would
    skip the exchange, so the split is refused before any window exists."""
    from dgx_monarch_b200.cfg import DualModelCfg, UnsupportedModelError

    with pytest.raises(UnsupportedModelError, match="cfg above 1"):
        DualModelCfg(1024, 1.0, device=torch.device("cpu"))


def test_oracle_cfg_combine_rounds_each_operation():
    """The oracle's combine against torch's unfused expression on the CPU for
    fp32 (each operation rounded to fp32)."""
    g = torch.Generator().manual_seed(3)
    c, u = torch.randn(1000, generator=g), torch.randn(1000, generator=g)
    want = (u + (c - u) * 4.5).numpy()
    np.testing.assert_array_equal(usp.cfg_combine(c.numpy(), u.numpy(), 4.5, "float32"), want)
