"""fp32 heads on the GPU: the reference's wrappers take any floating dtype (the
output dtype is the hidden dtype, gsp/triton_runtime.py:111) and
constrained_projection is a plain F.linear (gsp/runtime.py:46-51), and the CPU
plumbing configuration is fp32: V=32,768, H=1,024, batch 1, W ~ N(0, 0.02),
h ~ N(0, 1), 1% of the tokens legal, drawn uniformly with seed 0.

fp32 runs on the row-sparse kernels (fp32 products accumulated in fp32, no
rounding step); the block and dense entry points run the same kernel.

Tolerance, written here because the stated rtol/atol 2e-3 is for half-precision
weights: fp32 logits agree with the reference's fp32 outputs and with the exact
float64 values within atol 1e-5 + rtol 1e-5 (the difference is summation order
over 1,024 products of magnitude ~0.02, about 1e-6). Legal support is bit-exact
and top-1 equals the exact argmax except within that window.
"""
import json

import numpy as np
import pytest
import torch

from conftest import load_npz
from gsp import _native, runtime as rt, triton_runtime as tr
from oracle import gsp_oracle as O

pytestmark = pytest.mark.gpu

RTOL32 = 1e-5
ATOL32 = 1e-5


def _config0():
    data, meta = load_npz("projection_ref.npz")
    case = [c for c in meta if c["name"] == "config0_fp32_1pct"][0]
    w, h, ids = O.config0_inputs(seed=case["seed"])
    assert O.tensor_sha256(w) == case["weight_sha256"] and O.tensor_sha256(h) == case["hidden_sha256"]
    assert np.array_equal(ids, data[case["name"] + "/ids"])
    return data, case, w, h, ids


def test_config0_constrained_projection_fp32_matches_reference(cuda_device):
    data, case, w, h, ids = _config0()
    res = rt.constrained_projection(h.to(cuda_device), w.to(cuda_device), torch.from_numpy(ids).to(cuda_device),
                                    dense_threshold=case["threshold"])
    assert res.logits.dtype == torch.float32
    assert res.mode == case["mode"] == "sparse-gather"
    assert np.array_equal(res.token_ids.cpu().numpy(), data[case["name"] + "/token_ids"])
    ref = torch.from_numpy(data[case["name"] + "/logits"]).double()  # the reference's own fp32 output
    rep = O.compare_logits(ref, res.logits.cpu(), rtol=RTOL32, atol=ATOL32)
    assert rep["support"] and rep["values"], rep
    exact = h.double() @ w[torch.from_numpy(ids)].double().T
    rep = O.compare_logits(exact, res.logits.cpu(), rtol=RTOL32, atol=ATOL32)
    assert rep["support"] and rep["values"], rep


def test_config0_vocab_shaped_routes_fp32(cuda_device):
    data, case, w, h, ids = _config0()
    vocab = w.shape[0]
    mask = O.ids_to_bitmask(ids, vocab)[0]
    exact = O.masked_logits_exact(h[0], w, mask)  # [V]
    wd, hd, md = w.to(cuda_device), h[0].to(cuda_device), torch.from_numpy(mask).to(cuda_device)
    outs = {
        "row-sparse": tr.bitmask_sparse_logits(hd, wd, md),
        "dense-mask": tr.dense_masked_logits(hd, wd, md),
    }
    got, route = tr.adaptive_grammar_logits(hd, wd, md)
    assert route == "row-sparse"
    outs["adaptive"] = got
    for name, out in outs.items():
        assert out.dtype == torch.float32 and out.shape == (vocab,), name
        rep = O.compare_logits(exact, out.cpu(), rtol=RTOL32, atol=ATOL32)
        assert rep["support"] and rep["values"], (name, rep)
        # the compact reference logits sit at the legal ids
        ref = torch.from_numpy(data[case["name"] + "/logits"][0]).double()
        assert torch.allclose(out.cpu()[torch.from_numpy(ids)].double(), ref, rtol=RTOL32, atol=ATOL32), name
    logits, top_value, top_index = tr.grammar_logits_with_top1(hd, wd, md)  # [1, V]
    assert torch.equal(top_index.cpu(), logits.argmax(-1).cpu())
    assert O.top1_agrees(exact[None], top_index.cpu(), rtol=RTOL32, atol=ATOL32)
    assert top_value.item() == logits.max().item()


@pytest.mark.parametrize("batch", [2, 5])
def test_fp32_batches_every_route(cuda_device, batch):
    """Batched fp32 heads: block-sparse and dense-mask names run the row-sparse
    kernel; all three agree with the oracle; fused top-1 = argmax."""
    rng = np.random.default_rng(300 + batch)
    vocab, hidden = 20_011, 192
    w = torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32) * np.float32(0.02))
    h = torch.from_numpy(rng.standard_normal((batch, hidden), dtype=np.float32))
    ks = [int(x) for x in rng.integers(0, 400, size=batch)]
    ks[-1] = vocab  # one request with every token legal
    mask = O.make_batch_mask(rng, batch, vocab, ks, clustered=True, max_runs=8)
    exact = O.masked_logits_exact(h, w, mask)
    wd, hd, md = w.to(cuda_device), h.to(cuda_device), torch.from_numpy(mask).to(cuda_device)
    for name, fn in (("row-sparse", tr.bitmask_sparse_logits), ("block-sparse", tr.bitmask_block_gemm_logits),
                     ("dense-mask", tr.dense_masked_logits)):
        out = fn(hd, wd, md)
        assert out.dtype == torch.float32
        rep = O.compare_logits(exact, out.cpu(), rtol=RTOL32, atol=ATOL32)
        assert rep["support"] and rep["values"], (name, rep)
    for route in ("row-sparse", "block-sparse", "dense-mask"):
        logits, tv, ti = tr.grammar_logits_with_top1(hd, wd, md, route=route)
        assert torch.equal(ti.cpu(), logits.argmax(-1).cpu()), route
        assert O.top1_agrees(exact, ti.cpu(), rtol=RTOL32, atol=ATOL32), route
    got, route = tr.adaptive_grammar_logits(hd, wd, md, full_word_fraction=O.full_word_fraction(mask))
    assert route == O.adaptive_route(batch, O.full_word_fraction(mask))
    rep = O.compare_logits(exact, got.cpu(), rtol=RTOL32, atol=ATOL32)
    assert rep["support"] and rep["values"], rep
    assert _native.workspace_error(cuda_device) == 0


def test_fp32_unconstrained_projection_and_half_only_extensions(cuda_device):
    rng = np.random.default_rng(5)
    w = torch.from_numpy(rng.standard_normal((3000, 64), dtype=np.float32) * np.float32(0.02)).to(cuda_device)
    h = torch.from_numpy(rng.standard_normal((2, 64), dtype=np.float32)).to(cuda_device)
    res = rt.constrained_projection(h, w, None)
    assert res.mode == "dense-unconstrained" and res.logits.dtype == torch.float32
    exact = h.cpu().double() @ w.cpu().double().T
    rep = O.compare_logits(exact, res.logits.cpu(), rtol=RTOL32, atol=ATOL32)
    assert rep["values"], rep
    mask = torch.full((2, (3000 + 31) // 32), -1, dtype=torch.int32, device=cuda_device)
    for fn in (lambda: tr.grammar_head(h, w, mask),
               lambda: tr.grouped_grammar_logits(h, w, mask),
               lambda: tr.grammar_sample(h, w, mask, seeds=torch.zeros(2, dtype=torch.int64, device=cuda_device),
                                         step=0),
               lambda: tr.adaptive_grammar_logits(h, w, mask, policy="device")):
        with pytest.raises(ValueError, match="float16 or bfloat16"):
            fn()
