"""Pins the oracle's mask semantics to xgrammar's CPU apply_token_bitmask_inplace,
the mask kernel of the reference's dense route (gsp/triton_runtime.py:305-307).
xgrammar is pinned at 0.2.8 by the reference; the installed version is used."""
import numpy as np
import pytest
import torch

from oracle import gsp_oracle as O

xgr = pytest.importorskip("xgrammar")


@pytest.mark.parametrize("vocab,batch,extra", [(1000, 3, 0), (4096, 2, 0), (777, 4, 3), (32, 1, 0), (33, 2, 1)])
def test_unpack_matches_xgrammar_cpu(vocab, batch, extra):
    rng = np.random.default_rng(vocab + batch)
    mask = rng.integers(-2**31, 2**31 - 1, size=(batch, O.mask_words(vocab) + extra), dtype=np.int64).astype(np.int32)
    mask[0, :] = -1
    logits = torch.randn(batch, vocab)
    ref = logits.clone()
    xgr.apply_token_bitmask_inplace(ref, torch.from_numpy(mask), vocab_size=vocab, backend="cpu")
    legal = O.unpack_bitmask(mask, vocab)
    assert np.array_equal(torch.isfinite(ref).numpy(), legal)
    assert torch.equal(ref[torch.from_numpy(legal)], logits[torch.from_numpy(legal)])
