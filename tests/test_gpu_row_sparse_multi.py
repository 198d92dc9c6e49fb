"""GPU parity of the multi-request row-sparse path: masks of more than 16,384
flat (request, word) entries go through the cooperative kernel, which splits
the mask into one word slice per CTA and balances legal rows across CTAs
from the published slice counts.

Cases: legal rows packed into one request (rank ranges far from the slices),
all-legal masks (several list rounds per CTA), no legal token anywhere,
slices longer than one chunk scan (V = 1,000,000), compact output with request
offsets, a broadcast mask (row stride 0), bf16, ragged V. Same tolerance as
test_gpu_row_sparse.py (oracle.value_bound); fused top-1 equal to
torch.argmax of the kernel's own logits.
"""
import numpy as np
import pytest
import torch

from gsp import _native
from gsp import triton_runtime as tr
from oracle import gsp_oracle as O

pytestmark = pytest.mark.gpu


def _inputs(rng, vocab, hidden, batch, dtype, scale=1.0):
    w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32) * scale).to(dtype)
    h = torch.from_numpy(rng.standard_normal((batch, hidden), dtype=np.float32)).to(dtype)
    return w, h


def _run_and_check(dev, h, w, mask, dtype, label):
    b, v = h.shape[0], w.shape[0]
    md = torch.from_numpy(mask).to(dev)
    logits = torch.empty(b, v, device=dev, dtype=dtype)
    tv = torch.empty(b, device=dev, dtype=torch.float32)
    ti = torch.empty(b, device=dev, dtype=torch.int64)
    _native.row_sparse(h.to(dev), w.to(dev), md, logits=logits, top_value=tv, top_index=ti)
    exact = O.masked_logits_exact(h, w, mask)
    rep = O.compare_logits(exact, logits.cpu(), dtype=dtype)
    assert rep["support"] and rep["values"], (label, rep)
    assert torch.equal(ti, logits.argmax(-1)), label
    assert torch.equal(tv, logits.float().gather(1, ti[:, None])[:, 0]), label
    _, idx = O.top1(logits.cpu())
    assert O.top1_agrees(exact, idx, dtype=dtype), label
    return logits, tv, ti


def test_rows_packed_into_one_request(cuda_device):
    """Request 3 all legal, the others 0-3 tokens: nearly every CTA's rank
    range lies inside the slices of one request."""
    rng = np.random.default_rng(31)
    vocab, hidden, batch = 50000, 256, 16
    w, h = _inputs(rng, vocab, hidden, batch, torch.float16)
    ks = [i % 4 for i in range(batch)]
    ks[3] = vocab
    mask = O.make_batch_mask(rng, batch, vocab, ks)
    _run_and_check(cuda_device, h, w, mask, torch.float16, "packed")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_all_legal_several_rounds(cuda_device, dtype):
    """400,000 units: about 2,700 per CTA, more than one list round each."""
    rng = np.random.default_rng(32)
    vocab, hidden, batch = 100000, 64, 6
    w, h = _inputs(rng, vocab, hidden, batch, dtype)
    mask = O.make_batch_mask(rng, batch, vocab, [vocab] * batch)
    logits, _, _ = _run_and_check(cuda_device, h, w, mask, dtype, "all legal")
    assert bool(torch.isfinite(logits).all())


def test_no_legal_token_anywhere(cuda_device):
    rng = np.random.default_rng(33)
    vocab, hidden, batch = 40000, 64, 16
    w, h = _inputs(rng, vocab, hidden, batch, torch.float16)
    mask = np.zeros((batch, O.mask_words(vocab)), dtype=np.int32)
    dev = cuda_device
    logits = torch.empty(batch, vocab, device=dev, dtype=torch.float16)
    tv = torch.empty(batch, device=dev, dtype=torch.float32)
    ti = torch.empty(batch, device=dev, dtype=torch.int64)
    _native.row_sparse(h.to(dev), w.to(dev), torch.from_numpy(mask).to(dev), logits=logits, top_value=tv,
                       top_index=ti)
    assert not torch.isfinite(logits).any()
    assert ti.tolist() == [0] * batch and all(v == float("-inf") for v in tv.tolist())


@pytest.mark.parametrize("clustered", [False, True])
def test_slices_longer_than_one_chunk(cuda_device, clustered):
    """V = 1,000,000, B = 20: 625,000 mask words, more than 4,096 per slice."""
    rng = np.random.default_rng(34 + clustered)
    vocab, hidden, batch = 1000000, 16, 20
    w, h = _inputs(rng, vocab, hidden, batch, torch.float16)
    ks = [int(k) for k in rng.integers(0, 3000, size=batch)]
    ks[7] = 0
    mask = O.make_batch_mask(rng, batch, vocab, ks, clustered=clustered, max_runs=8)
    logits, _, _ = _run_and_check(cuda_device, h, w, mask, torch.float16, f"long slices clustered={clustered}")
    assert int(torch.isfinite(logits).sum()) == sum(ks)


def test_compact_output_and_offsets(cuda_device):
    rng = np.random.default_rng(35)
    vocab, hidden, batch = 60001, 128, 10
    w, h = _inputs(rng, vocab, hidden, batch, torch.bfloat16)
    ks = [5, 0, 7000, 60001, 1, 300, 12, 0, 2500, 60001]
    mask = O.make_batch_mask(rng, batch, vocab, ks, clustered=True, max_runs=8)
    ids, lg, off = tr.bitmask_compact_logits(h.to(cuda_device), w.to(cuda_device), torch.from_numpy(mask).to(cuda_device))
    assert off.tolist() == list(np.concatenate([[0], np.cumsum(ks)]))
    legal = O.unpack_bitmask(mask, vocab)
    exact = O.masked_logits_exact(h, w, mask)
    for b in range(batch):
        s, e = off[b].item(), off[b + 1].item()
        assert np.array_equal(ids[s:e].cpu().numpy(), np.flatnonzero(legal[b])), b
        rep = O.compare_logits(exact[b, np.flatnonzero(legal[b])], lg[s:e].cpu(), dtype=torch.bfloat16)
        assert rep["support"] and rep["values"], (b, rep)


def test_broadcast_mask_and_ragged_vocab(cuda_device):
    """One mask row for every request (row stride 0), V % 32 != 0."""
    rng = np.random.default_rng(36)
    vocab, hidden, batch = 40007, 96, 14
    w, h = _inputs(rng, vocab, hidden, batch, torch.float16)
    row = O.recipe_mask("c900", rng, 1, vocab)
    mask_full = np.repeat(row, batch, axis=0)
    dev = cuda_device
    logits = torch.empty(batch, vocab, device=dev, dtype=torch.float16)
    md = torch.from_numpy(row).to(dev).expand(batch, -1)
    _native.row_sparse(h.to(dev), w.to(dev), md, logits=logits)
    rep = O.compare_logits(O.masked_logits_exact(h, w, mask_full), logits.cpu(), dtype=torch.float16)
    assert rep["support"] and rep["values"], rep


def test_repeated_calls_are_identical(cuda_device):
    """Slice counts, flags and the unit list are re-zeroed by the kernel itself."""
    rng = np.random.default_rng(37)
    vocab, hidden, batch = 70000, 64, 8
    w, h = _inputs(rng, vocab, hidden, batch, torch.float16)
    mask = O.make_batch_mask(rng, batch, vocab, [10, 2000, 0, 70000, 333], clustered=True, max_runs=4)
    first = _run_and_check(cuda_device, h, w, mask, torch.float16, "call 0")
    for i in range(1, 4):
        again = _run_and_check(cuda_device, h, w, mask, torch.float16, f"call {i}")
        assert all(torch.equal(a, b) for a, b in zip(first, again))


def test_workspace_left_zero_across_sizes(cuda_device):
    """Calls of different sizes carve one workspace differently, so every
    kernel must leave it all zero (error word aside): slice counts, flags,
    tickets, keys, tile lists and the unit list."""
    rng = np.random.default_rng(38)
    dev = cuda_device
    hidden = 64
    w = torch.from_numpy(rng.standard_normal((250000, hidden), dtype=np.float32)).half().to(dev)
    for batch, vocab in ((5, 70000), (2, 248320), (64, 30000), (3, 250000), (300, 3000), (16, 50000)):
        h = torch.from_numpy(rng.standard_normal((batch, hidden), dtype=np.float32)).half().to(dev)
        mask = torch.from_numpy(O.make_batch_mask(rng, batch, vocab, [int(k) for k in rng.integers(0, 3000, batch)],
                                                  clustered=True, max_runs=8)).to(dev)
        for fn in (_native.row_sparse, _native.block_gemm, _native.dense_masked):
            logits = torch.empty(batch, vocab, device=dev, dtype=torch.float16)
            ti = torch.empty(batch, device=dev, dtype=torch.int64)
            fn(h, w[:vocab], mask, logits=logits, top_index=ti)
            assert torch.equal(ti, logits.argmax(-1)), (batch, vocab, fn.__name__)
            ws = _native.workspace(dev, batch, vocab)
            torch.cuda.synchronize()
            assert int(ws[:4].count_nonzero()) == 0 and int(ws[8:].count_nonzero()) == 0, (batch, vocab, fn.__name__)


def test_no_bounded_wait_gave_up_multi(cuda_device):
    assert _native.workspace_error(cuda_device) == 0
