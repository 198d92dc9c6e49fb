"""GPU parity at the full sizes of the mixed-density dispatcher sweep and of the
vocabulary-parallel head, each compared with exact float64 logits:

* mixed sweep: V=151,936, H=1,024, bf16, batch 64; a seeded mix of
  near-unconstrained requests (95% legal, uniform) and constrained ones (0.2%
  legal in <= 16 clustered runs) at constrained fractions 0 / 25 / 50 / 75 /
  100%; every route, and the routes each dispatcher policy picks (the
  reference rule's pick equal to the oracle's restatement of it,
  gsp/triton_runtime.py:341-353);
* vocabulary-parallel head on one GPU: V=262,144, H=8,192, bf16,
  W ~ N(0, 0.01), batch 1 / 32 / 128, 1% legal per request in <= 16 clustered
  runs; every route; and the head cut into 2 and 8 contiguous row shards run
  through vocab_offset, whose logits and top-1 keys merged must equal the
  unsharded call's bit for bit.

The exact reference for the whole batch is a float64 torch product on the GPU
(tests/conftest.py exact_logits_gpu); it is itself checked against the CPU
oracle on sampled requests. Tolerances are the oracle's: legal support
bit-exact, legal logits within atol 2e-3 + max(rtol 2e-3 |x|, half a bf16 ulp),
top-1 equal to the exact argmax except within the near-tie window.
"""
import numpy as np
import pytest
import torch

from conftest import exact_logits_gpu
from gsp import _native, triton_runtime as tr, vocab_parallel as vp
from gsp import workloads as wl
from oracle import gsp_oracle as O

pytestmark = pytest.mark.gpu

ROUTES = {"row-sparse": _native.row_sparse, "block-sparse": _native.block_gemm, "dense-mask": _native.dense_masked}


def _run(fn, h, w, m, *, vocab_offset=0, with_logits=True):
    b, v = h.shape[0], w.shape[0]
    logits = torch.empty(b, v, device=h.device, dtype=h.dtype) if with_logits else None
    tv = torch.empty(b, device=h.device, dtype=torch.float32)
    ti = torch.empty(b, device=h.device, dtype=torch.int64)
    tk = torch.empty(b, device=h.device, dtype=torch.int64)
    fn(h, w, m, logits=logits, top_value=tv, top_index=ti, top_key=tk, vocab_offset=vocab_offset)
    return logits, tv, ti, tk


def _check(exact, logits, ti, dtype, what):
    rep = O.compare_logits(exact.cpu(), logits.cpu(), dtype=dtype)
    assert rep["support"] and rep["values"], (what, rep)
    assert torch.equal(ti, logits.argmax(-1)), what
    assert O.top1_agrees(exact.cpu(), ti.cpu(), dtype=dtype), what


def _oracle_tie_in(h, w, mask, exact, rows):
    """The GPU float64 reference equals the CPU oracle on sampled requests."""
    ref = O.masked_logits_exact(h[rows].cpu(), w.cpu(), mask[rows])
    got = exact[rows].cpu()
    assert torch.equal(torch.isfinite(ref), torch.isfinite(got))
    fin = torch.isfinite(ref)
    assert torch.allclose(ref[fin], got[fin], rtol=1e-12, atol=1e-12)


@pytest.fixture(scope="module")
def mixed_head(cuda_device):
    vocab, hidden, batch = 151_936, 1024, 64
    g = torch.Generator(device=cuda_device).manual_seed(5)
    w = (torch.randn(vocab, hidden, device=cuda_device, generator=g) * 0.02).bfloat16()
    h = torch.randn(batch, hidden, device=cuda_device, generator=g).bfloat16()
    return w, h


@pytest.mark.parametrize("frac", [0.0, 0.25, 0.5, 0.75, 1.0])
def test_mixed_density_sweep_full_size(cuda_device, mixed_head, frac):
    w, h = mixed_head
    batch, vocab = h.shape[0], w.shape[0]
    rng = np.random.default_rng(int(frac * 100))
    mask = wl.mixed_batch_mask(rng, batch, vocab, frac)
    md = torch.from_numpy(mask).to(cuda_device)
    exact = exact_logits_gpu(h, w, md)
    legal = wl.unpack_bitmask(mask, vocab).sum(axis=1)
    constrained = int(np.argmin(legal))
    _oracle_tie_in(h, w, mask, exact, [constrained, int(np.argmax(legal))])
    for name, fn in ROUTES.items():
        logits, tv, ti, _ = _run(fn, h, w, md)
        _check(exact, logits, ti, torch.bfloat16, (frac, name))
        assert torch.equal(tv, logits.float().gather(1, ti[:, None])[:, 0]), (frac, name)
    fwf = O.full_word_fraction(mask)
    got, route = tr.adaptive_grammar_logits(h, w, md, full_word_fraction=fwf)
    assert route == O.adaptive_route(batch, fwf), frac
    rep = O.compare_logits(exact.cpu(), got.cpu(), dtype=torch.bfloat16)
    assert rep["support"] and rep["values"], (frac, "reference policy", rep)
    for policy in ("b200", "device"):
        got, route = tr.adaptive_grammar_logits(h, w, md, policy=policy)
        assert route in ROUTES, (policy, route)
        rep = O.compare_logits(exact.cpu(), got.cpu(), dtype=torch.bfloat16)
        assert rep["support"] and rep["values"], (frac, policy, rep)
    assert _native.workspace_error(cuda_device) == 0


@pytest.fixture(scope="module")
def vp_head(cuda_device):
    vocab, hidden = 262_144, 8192
    g = torch.Generator(device=cuda_device).manual_seed(4321)
    w = (torch.randn(vocab, hidden, device=cuda_device, generator=g) * 0.01).bfloat16()
    return w


@pytest.mark.parametrize("batch", [1, 32, 128])
def test_vocab_parallel_config_full_size_one_gpu(cuda_device, vp_head, batch):
    w = vp_head
    vocab, hidden = w.shape
    rng = np.random.default_rng(500 + batch)
    mask = wl.make_batch_mask(rng, batch, vocab, [vocab // 100] * batch, clustered=True, max_runs=16)
    md = torch.from_numpy(mask).to(cuda_device)
    h = torch.randn(batch, hidden, device=cuda_device,
                    generator=torch.Generator(device=cuda_device).manual_seed(600 + batch)).bfloat16()
    exact = exact_logits_gpu(h, w, md)
    _oracle_tie_in(h, w, mask, exact, [0])
    full = {}
    for name, fn in ROUTES.items():
        if name == "block-sparse" and batch == 1:
            logits, tv, ti, tk = _run(_native.block_gemm, h, w, md)
        else:
            logits, tv, ti, tk = _run(fn, h, w, md)
        _check(exact, logits, ti, torch.bfloat16, (batch, name))
        full[name] = (logits, tv, ti, tk)
    # 2 and 8 contiguous row shards, each run with its vocab_offset: merged
    # logits and integer-MAX-merged keys equal the unsharded call bit for bit
    for ranks in (2, 8):
        for name, fn in ROUTES.items():
            parts, keys = [], []
            for r in range(ranks):
                lo, hi = vp.shard_bounds(vocab, ranks, r)
                m = md[:, lo // 32:(hi + 31) // 32].contiguous()
                logits, _, _, tk = _run(fn, h, w[lo:hi], m, vocab_offset=lo)
                parts.append(logits)
                keys.append(tk)
            merged = torch.cat(parts, dim=1)
            assert torch.equal(merged.view(torch.int16), full[name][0].view(torch.int16)), (batch, ranks, name)
            key = torch.stack(keys).max(dim=0).values
            assert torch.equal(key, full[name][3]), (batch, ranks, name)
            tv, ti = vp.decode_keys(key)
            assert torch.equal(ti, full[name][2]) and torch.equal(tv, full[name][1]), (batch, ranks, name)
    assert _native.workspace_error(cuda_device) == 0
