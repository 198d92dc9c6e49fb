"""GPU parity of the fused grammar-conditioned sampler (gsp_row_sparse_sample)
against the oracle's restatement of its contract, on every row-sparse kernel
(batch 1 staged, multi-request cooperative, unaligned direct).

Checks: the sampled token equals the oracle's Gumbel-max pick except where
the oracle's best and the kernel's pick score within the logit tolerance of
each other; logsumexp within that tolerance; greedy top-1 unchanged by
sampling; the same (seeds, step) reproduce the same tokens bit for bit (the
log-sum-exp to fp32 rounding) and a new step draws new ones; over many seeds the draws follow softmax(logits / T) over the
legal tokens (chi-square); requests without a legal token; the workspace is
left all zero.
"""
import numpy as np
import pytest
import torch

from gsp import _native
from gsp import triton_runtime as tr
from oracle import gsp_oracle as O

pytestmark = pytest.mark.gpu


def _seeds(dev, n, base=1000):
    """Distinct 64-bit seeds (high and low words both vary)."""
    i = torch.arange(n, dtype=torch.int64, device=dev)
    return (i + base) * 2654435761 + ((i * 40503 + base) << 32)


def _check_against_oracle(res, ref, temperature, dtype_label):
    inv_t = 1.0 / temperature
    for b, (pick, lse, scores, ids) in enumerate(ref):
        got = int(res.token_ids[b])
        if ids.size == 0:
            assert got == 0 and res.logsumexp[b].item() == float("-inf"), (dtype_label, b)
            continue
        best = float(scores.max())
        x_best = abs(best)
        tol = (2e-3 + 2e-3 * x_best) * inv_t * 2 + 1e-5 * (1 + x_best)
        if got != pick:
            assert got in set(ids.tolist()), (dtype_label, b, "not a legal token")
            assert best - float(scores[list(ids).index(got)]) <= tol, (dtype_label, b, got, pick)
        lse_tol = (2e-3 + 2e-3 * np.abs(scores).max()) * inv_t + 1e-4 * (1 + abs(lse))
        assert abs(res.logsumexp[b].item() - lse) <= lse_tol, (dtype_label, b, res.logsumexp[b].item(), lse)


@pytest.mark.parametrize("case", [
    # vocab, hidden, batch, dtype, temperature, clustered, misaligned  (kernel)
    (50000, 256, 1, torch.float16, 1.0, False, False),     # staged
    (40000, 128, 16, torch.bfloat16, 0.7, True, False),    # cooperative (20,000 flat words)
    (3000, 96, 3, torch.float16, 1.5, False, True),        # direct (unaligned hidden)
])
def test_sample_matches_oracle(cuda_device, case):
    vocab, hidden, batch, dtype, temperature, clustered, misaligned = case
    rng = np.random.default_rng(vocab + batch)
    w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32) * 0.3).to(dtype)
    h = torch.from_numpy(rng.standard_normal((batch, hidden), dtype=np.float32)).to(dtype)
    ks = [max(1, vocab // 100)] * batch
    mask = O.make_batch_mask(rng, batch, vocab, ks, clustered=clustered, max_runs=8)
    dev = cuda_device
    hd = h.to(dev)
    if misaligned:
        buf = torch.empty(batch * hidden + 1, dtype=dtype, device=dev)
        buf[1:] = hd.reshape(-1)
        hd = buf[1:].view(batch, hidden)
    seeds = _seeds(dev, batch)
    for step in (0, 1, 12345):
        res = tr.grammar_sample(hd, w.to(dev), torch.from_numpy(mask).to(dev), seeds=seeds, step=step,
                                temperature=temperature, return_logits=True)
        ref = O.sample_reference(h, w, mask, dtype, temperature, seeds.cpu().numpy(), step)
        _check_against_oracle(res, ref, temperature, f"{case} step {step}")
        # greedy top-1 is that of the materialised logits
        assert torch.equal(res.top_index, res.logits.argmax(-1))
        assert O.top1_agrees(O.masked_logits_exact(h, w, mask), res.top_index.cpu(), dtype=dtype)
    assert _native.workspace_error(dev) == 0


def test_sample_is_reproducible_and_steps_differ(cuda_device):
    dev = cuda_device
    rng = np.random.default_rng(4)
    vocab, hidden, batch = 20000, 64, 16
    w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32) * 0.05).half().to(dev)
    h = torch.from_numpy(rng.standard_normal((batch, hidden), dtype=np.float32)).half().to(dev)
    mask = torch.from_numpy(O.make_batch_mask(rng, batch, vocab, [2000] * batch)).to(dev)
    seeds = _seeds(dev, batch, 7)
    a = tr.grammar_sample(h, w, mask, seeds=seeds, step=5, temperature=2.0)
    b = tr.grammar_sample(h, w, mask, seeds=seeds, step=5, temperature=2.0)
    c = tr.grammar_sample(h, w, mask, seeds=seeds, step=6, temperature=2.0)
    # the draws are exact integer maxima: bit-identical; the log-sum-exp merges
    # (max, sum) pairs in arrival order: identical to fp32 rounding
    assert torch.equal(a.token_ids, b.token_ids)
    assert torch.allclose(a.logsumexp, b.logsumexp, rtol=1e-6, atol=1e-6)
    assert (a.token_ids != c.token_ids).sum().item() >= batch // 2  # near-flat logits: new draws
    assert torch.allclose(a.logsumexp, c.logsumexp, rtol=1e-6, atol=1e-6)  # no dependence on the noise
    # with logits materialised or not, the draw is the same
    d = tr.grammar_sample(h, w, mask, seeds=seeds, step=5, temperature=2.0, return_logits=True)
    assert torch.equal(a.token_ids, d.token_ids)


def test_sample_distribution_follows_softmax(cuda_device):
    """512 requests x 16 steps with one mask of 12 legal tokens and one hidden
    state: 8,192 draws against softmax(logits / T) of the kernel's own rounded
    logits (chi-square, 11 degrees of freedom)."""
    from scipy.stats import chi2
    dev = cuda_device
    rng = np.random.default_rng(11)
    vocab, hidden, batch, temperature = 2048, 64, 512, 0.8
    w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32) * 0.08).half().to(dev)
    h1 = torch.from_numpy(rng.standard_normal((1, hidden), dtype=np.float32)).half().to(dev)
    h = h1.expand(batch, hidden).contiguous()
    legal_ids = np.sort(rng.choice(vocab, size=12, replace=False))
    mask = torch.from_numpy(np.repeat(O.ids_to_bitmask(legal_ids, vocab), batch, axis=0)).to(dev)
    counts = np.zeros(vocab, dtype=np.int64)
    logits = None
    for step in range(16):
        res = tr.grammar_sample(h, w, mask, seeds=_seeds(dev, batch, 31 + step * batch), step=step,
                                temperature=temperature, return_logits=(step == 0))
        if logits is None:
            logits = res.logits[0].float().cpu().numpy()
        np.add.at(counts, res.token_ids.cpu().numpy(), 1)
    assert counts.sum() == 16 * batch and counts[legal_ids].sum() == counts.sum()
    y = logits[legal_ids].astype(np.float64) / temperature
    p = np.exp(y - y.max())
    p /= p.sum()
    expected = p * counts.sum()
    stat = float(((counts[legal_ids] - expected) ** 2 / expected).sum())
    assert chi2.sf(stat, df=len(legal_ids) - 1) > 1e-4, (stat, counts[legal_ids], expected.round(1))
    # the reported logsumexp is that of the same logits
    lse = y.max() + np.log(np.exp(y - y.max()).sum())
    assert abs(res.logsumexp[0].item() - lse) < 1e-3


def test_sample_without_legal_tokens_and_workspace_left_zero(cuda_device):
    dev = cuda_device
    rng = np.random.default_rng(12)
    hidden = 64
    w = torch.from_numpy(rng.standard_normal((30000, hidden), dtype=np.float32)).half().to(dev)
    for batch, vocab in ((1, 30000), (5, 20000), (40, 30000), (2, 1000)):
        h = torch.from_numpy(rng.standard_normal((batch, hidden), dtype=np.float32)).half().to(dev)
        ks = [0 if b % 2 == 0 else 77 for b in range(batch)]
        mask = torch.from_numpy(O.make_batch_mask(rng, batch, vocab, ks, clustered=True, max_runs=4)).to(dev)
        res = tr.grammar_sample(h, w[:vocab], mask, seeds=_seeds(dev, batch), step=3)
        for b in range(batch):
            if ks[b] == 0:
                assert res.token_ids[b].item() == 0 and res.logsumexp[b].item() == float("-inf")
            else:
                assert bool(mask[b, res.token_ids[b].item() // 32].item() >> (res.token_ids[b].item() % 32) & 1)
        ws = _native.workspace(dev, batch, vocab)
        torch.cuda.synchronize()
        assert int(ws[:4].count_nonzero()) == 0 and int(ws[8:].count_nonzero()) == 0, (batch, vocab)


@pytest.mark.parametrize("shards", [2, 3])
def test_sharded_sampling_equals_whole_vocabulary(cuda_device, shards):
    """The sampler on row shards of one vocabulary (vocab_offset = the shard's
    first id, as each rank of a vocabulary-parallel head runs it): the integer
    MAX of the shards' sample keys is the unsharded draw bit for bit, their
    log-sum-exps merged by gsp_merge_logsumexp agree to fp32 rounding, and the
    greedy keys give the unsharded top-1."""
    from gsp import vocab_parallel as vp
    dev = cuda_device
    rng = np.random.default_rng(60 + shards)
    vocab, hidden, batch, temperature = 30017, 128, 6, 0.9
    w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32) * 0.2).half().to(dev)
    h = torch.from_numpy(rng.standard_normal((batch, hidden), dtype=np.float32)).half().to(dev)
    ks = [int(k) for k in rng.integers(0, vocab // 20, size=batch)]
    ks[0] = 0  # a request without a legal token
    mask = torch.from_numpy(O.make_batch_mask(rng, batch, vocab, ks, clustered=True, max_runs=8)).to(dev)
    seeds = _seeds(dev, batch, 77)
    for step in (0, 9):
        full = tr.grammar_sample(h, w, mask, seeds=seeds, step=step, temperature=temperature)
        skeys, tkeys, lses = [], [], []
        for r in range(shards):
            lo, hi = vp.shard_bounds(vocab, shards, r)
            sk = torch.empty(batch, dtype=torch.int64, device=dev)
            tk = torch.empty(batch, dtype=torch.int64, device=dev)
            ls = torch.empty(batch, device=dev)
            si = torch.empty(batch, dtype=torch.int64, device=dev)
            _native.row_sparse_sample(h, w[lo:hi], mask[:, lo // 32:(hi + 31) // 32].contiguous(), seeds, step,
                                      temperature, si, sample_logsumexp=ls, vocab_offset=lo, sample_key=sk,
                                      top_key=tk)
            skeys.append(sk)
            tkeys.append(tk)
            lses.append(ls)
        ids = torch.empty(batch, dtype=torch.int64, device=dev)
        _native.top1_from_keys(torch.stack(skeys).max(dim=0).values, None, ids)
        assert torch.equal(ids, full.token_ids), (shards, step)
        lse = torch.empty(batch, device=dev)
        _native.merge_logsumexp(torch.stack(lses).contiguous(), lse)
        assert lse[0].item() == float("-inf") and full.logsumexp[0].item() == float("-inf")
        assert torch.allclose(lse[1:], full.logsumexp[1:], rtol=1e-5, atol=1e-5), (lse, full.logsumexp)
        tv = torch.empty(batch, device=dev)
        ti = torch.empty(batch, dtype=torch.int64, device=dev)
        _native.top1_from_keys(torch.stack(tkeys).max(dim=0).values, tv, ti)
        assert torch.equal(ti, full.top_index) and torch.equal(tv, full.top_value)


@pytest.mark.parametrize("route", ["block-sparse", "dense-mask"])
@pytest.mark.parametrize("case", [
    # vocab, hidden, batch, dtype, temperature, clustered
    (50000, 256, 8, torch.float16, 1.0, True),      # narrow epilogue (batch pads to 32)
    (20011, 192, 40, torch.bfloat16, 0.7, False),   # wide epilogue, ragged vocabulary and hidden size
    (3000, 128, 300, torch.float16, 1.3, True),     # two batch chunks (256 + 44)
])
def test_tensor_core_sample_matches_oracle(cuda_device, route, case):
    """The sampler in the tensor-core epilogue (gsp_sample, block-sparse and
    dense-mask routes) draws under the same contract: the oracle's Gumbel-max
    pick except within the tie tolerance, its log-sum-exp, the greedy top-1 of
    the materialised logits, and the same tokens on a repeated call; the
    workspace is left all zero."""
    vocab, hidden, batch, dtype, temperature, clustered = case
    rng = np.random.default_rng(vocab + batch + hidden)
    w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32) * 0.3).to(dtype)
    h = torch.from_numpy(rng.standard_normal((batch, hidden), dtype=np.float32)).to(dtype)
    ks = [int(x) for x in rng.integers(1, max(2, vocab // 50), size=batch)]
    ks[0] = 0  # a request with no legal token
    mask = O.make_batch_mask(rng, batch, vocab, ks, clustered=clustered, max_runs=8)
    dev = cuda_device
    hd, wd, md = h.to(dev), w.to(dev), torch.from_numpy(mask).to(dev)
    seeds = _seeds(dev, batch, base=77)
    for step in (0, 9):
        res = tr.grammar_sample(hd, wd, md, seeds=seeds, step=step, temperature=temperature, return_logits=True,
                                route=route)
        ref = O.sample_reference(h, w, mask, dtype, temperature, seeds.cpu().numpy(), step)
        _check_against_oracle(res, ref, temperature, f"{route} {case} step {step}")
        assert torch.equal(res.top_index, res.logits.argmax(-1))
        again = tr.grammar_sample(hd, wd, md, seeds=seeds, step=step, temperature=temperature, route=route)
        assert torch.equal(again.token_ids, res.token_ids)
        assert torch.allclose(again.logsumexp, res.logsumexp, rtol=1e-5, atol=1e-5, equal_nan=True)
    torch.cuda.synchronize()
    assert _native.workspace_error(dev) == 0
    ws = _native.workspace(dev, batch, vocab)
    assert int(ws[:4].count_nonzero()) == 0 and int(ws[8:].count_nonzero()) == 0


def test_tensor_core_sample_batched_workload(cuda_device):
    """The batched workload's shape (V=248,320, H=2,048 fp16, batch 32, each
    request 0.5% legal in <= 16 runs) on the block-sparse route: every draw
    against the oracle, and the same draws as the row-sparse sampler except
    within the tie tolerance."""
    dev = cuda_device
    vocab, hidden, batch = 248_320, 2048, 32
    g = torch.Generator(device=dev).manual_seed(7)
    wd = (torch.randn(vocab, hidden, device=dev, generator=g) * 0.02).half()
    hd = torch.randn(batch, hidden, device=dev, generator=g).half()
    rng = np.random.default_rng(32)
    mask = O.make_batch_mask(rng, batch, vocab, [1242] * batch, clustered=True, max_runs=16)
    md = torch.from_numpy(mask).to(dev)
    seeds = _seeds(dev, batch, base=5)
    res = tr.grammar_sample(hd, wd, md, seeds=seeds, step=3, temperature=0.8, route="block-sparse")
    ref = O.sample_reference(hd.cpu(), wd.cpu(), mask, torch.float16, 0.8, seeds.cpu().numpy(), 3)
    _check_against_oracle(res, ref, 0.8, "block-sparse batched")
    rs = tr.grammar_sample(hd, wd, md, seeds=seeds, step=3, temperature=0.8, route="row-sparse")
    _check_against_oracle(rs, ref, 0.8, "row-sparse batched")
    assert _native.workspace_error(dev) == 0
