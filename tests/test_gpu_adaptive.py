"""Device-side route choice (gsp_adaptive_logits, grammar_head,
GraphedGrammarHead): the selector kernel picks the route the host cost model
picks for the same mask, and the chosen route's outputs are bit-identical to
calling that route directly: eagerly, inside a torch CUDA graph whose replays
switch routes as the mask changes, and in the graphed head (pinned mask staged by
a copy stream, head replayed after it). Batch 1 is always row-sparse; the
workspace is left zero.
"""
import numpy as np
import pytest
import torch

from gsp import _native
from gsp import triton_runtime as tr
from gsp import workloads as wl
from gsp.graphed import GraphedGrammarHead

pytestmark = pytest.mark.gpu

# Small head with the cost model steered so that all three routes occur:
# sparse uniform masks -> row-sparse (the multi-request cooperative kernel at
# 24 x 1,024 mask words), one shared 10% run -> block-sparse, 95% uniform ->
# dense-mask.
V, H, B = 32768, 512, 24
COST = {"row_sparse_fixed_us": 0.5, "block_floor_us": 0.0, "block_fixed_us": 1.0, "dense_fixed_us": 0.0}
EXPECTED = {"sparse": "row-sparse", "shared": "block-sparse", "wide": "dense-mask"}
DIRECT = {"row-sparse": _native.row_sparse, "block-sparse": _native.block_gemm, "dense-mask": _native.dense_masked}


def _mask(kind, rng, batch=B):
    if kind == "sparse":
        return wl.make_batch_mask(rng, batch, V, [10] * batch)
    if kind == "shared":
        row = wl.make_batch_mask(rng, 1, V, [V // 10], clustered=True, max_runs=1)
        return np.repeat(row, batch, axis=0)
    return wl.make_batch_mask(rng, batch, V, [int(0.95 * V)] * batch)


def _host_route(mask_np, cost=COST):
    legal = wl.unpack_bitmask(mask_np, V).sum(axis=1).tolist()
    return tr.choose_route(mask_np.shape[0], V, H, 2, legal, wl.active_tiles(mask_np, V), cost)


@pytest.fixture(scope="module")
def head(cuda_device):
    rng = np.random.default_rng(42)
    w = (torch.from_numpy(rng.standard_normal((V, H), dtype=np.float32)) * 0.05).half().to(cuda_device)
    h = torch.from_numpy(rng.standard_normal((B, H), dtype=np.float32)).half().to(cuda_device)
    masks = {k: _mask(k, rng) for k in EXPECTED}
    for k, m in masks.items():
        assert _host_route(m) == EXPECTED[k], k  # the case design itself
    return w, h, masks


def _direct(route, h, w, mask_dev):
    lg = torch.empty(h.shape[0], V, dtype=h.dtype, device=h.device)
    tv = torch.empty(h.shape[0], device=h.device)
    ti = torch.empty(h.shape[0], dtype=torch.int64, device=h.device)
    DIRECT[route](h, w, mask_dev, logits=lg, top_value=tv, top_index=ti)
    return lg, tv, ti


def _same(res, ref, what):
    lg, tv, ti = ref
    assert torch.equal(res.logits, lg), what
    assert torch.equal(res.top_value, tv) and torch.equal(res.top_index, ti), what


def test_eager_selector_matches_host_model_and_route(cuda_device, head):
    w, h, masks = head
    for kind, m in masks.items():
        md = torch.from_numpy(m).to(cuda_device)
        res = tr.grammar_head(h, w, md, cost=COST)
        route = tr.ROUTES[int(res.route.item())]
        assert route == EXPECTED[kind], kind
        _same(res, _direct(route, h, w, md), kind)
        # default cost model: same choice as the host-side b200 policy
        lg_dev, r_dev = tr.adaptive_grammar_logits(h, w, md, policy="device")
        lg_b200, r_b200 = tr.adaptive_grammar_logits(h, w, md, policy="b200")
        assert r_dev == r_b200 and torch.equal(lg_dev, lg_b200), kind
    assert _native.workspace_error(cuda_device) == 0


def test_captured_head_switches_route_per_replay(cuda_device, head):
    w, h, masks = head
    dev = cuda_device
    static_mask = torch.from_numpy(masks["sparse"]).to(dev)
    out = tr.HeadResult(torch.empty(B, V, dtype=h.dtype, device=dev), torch.empty(B, device=dev),
                        torch.empty(B, dtype=torch.int64, device=dev), torch.zeros(1, dtype=torch.int32, device=dev))
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for fn in DIRECT.values():  # warm-up on the capturing stream
            fn(h, w, static_mask, logits=out.logits, top_value=out.top_value, top_index=out.top_index)
        tr.grammar_head(h, w, static_mask, cost=COST, out=out)
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        tr.grammar_head(h, w, static_mask, cost=COST, out=out)
    for kind in ("sparse", "shared", "wide", "sparse", "wide", "shared", "shared"):
        static_mask.copy_(torch.from_numpy(masks[kind]))
        out.logits.fill_(0)
        g.replay()
        torch.cuda.synchronize()
        route = tr.ROUTES[int(out.route.item())]
        assert route == EXPECTED[kind], kind
        _same(out, _direct(route, h, w, static_mask), f"replay {kind}")
    with torch.cuda.stream(s):
        ws = _native.workspace(dev, B, V)
        torch.cuda.synchronize()
        assert int(ws[:4].count_nonzero()) == 0 and int(ws[8:].count_nonzero()) == 0
    del g


def test_graphed_head_with_staged_pinned_mask(cuda_device, head):
    w, h, masks = head
    gh = GraphedGrammarHead(w, B, cost=COST)
    rng = np.random.default_rng(7)
    for step, kind in enumerate(("wide", "sparse", "shared", "sparse")):
        gh.wait_mask_copied()
        gh.mask_host.copy_(torch.from_numpy(masks[kind]))
        gh.stage_mask()
        hid = h if step % 2 == 0 else torch.from_numpy(rng.standard_normal((B, H), dtype=np.float32)).half().to(h.device)
        res = gh.step(hid)
        torch.cuda.synchronize()
        assert gh.route_names() == [EXPECTED[kind]], (step, kind)
        _same(res, _direct(EXPECTED[kind], hid, w, torch.from_numpy(masks[kind]).to(h.device)), f"step {step}")


def test_batch_one_is_row_sparse_captured(cuda_device, head):
    w, h, masks = head
    dev = cuda_device
    gh = GraphedGrammarHead(w, 1, cost={"row_sparse_fixed_us": 1e6})  # row-sparse regardless of cost
    for kind in ("wide", "sparse"):
        gh.wait_mask_copied()
        gh.mask_host.copy_(torch.from_numpy(masks[kind][:1]))
        gh.stage_mask()
        res = gh.step(h[:1])
        torch.cuda.synchronize()
        assert gh.route_names() == ["row-sparse"]
        _same(res, _direct("row-sparse", h[:1], w, torch.from_numpy(masks[kind][:1]).to(dev)), kind)


@pytest.mark.parametrize("vocab, hidden, batch, dtype", [(30001, 96, 5, torch.float16), (4099, 256, 2, torch.bfloat16)])
def test_selector_on_ragged_sizes(cuda_device, vocab, hidden, batch, dtype):
    """Vocabularies that are not multiples of 32 or 128 (tail bits of the last
    mask word set on purpose): the device's statistics give the host model's
    route for each cost model, and the outputs equal that route's."""
    dev = cuda_device
    rng = np.random.default_rng(vocab)
    w = (torch.from_numpy(rng.standard_normal((vocab, hidden), dtype=np.float32)) * 0.05).to(dtype).to(dev)
    h = torch.from_numpy(rng.standard_normal((batch, hidden), dtype=np.float32)).to(dtype).to(dev)
    fns = {"row-sparse": _native.row_sparse, "block-sparse": _native.block_gemm, "dense-mask": _native.dense_masked}
    for ks, cost in (([vocab // 200] * batch, COST), ([int(0.9 * vocab)] * batch, COST),
                     ([vocab // 50] * batch, {"row_sparse_fixed_us": 50.0, "block_floor_us": 0.0, "dense_fixed_us": 50.0})):
        mask_np = wl.make_batch_mask(rng, batch, vocab, ks, clustered=True, max_runs=4)
        mask_np[:, -1] |= np.int32(-1)  # bits past the vocabulary in the last word: ignored
        legal = wl.unpack_bitmask(mask_np, vocab).sum(axis=1).tolist()
        want = tr.choose_route(batch, vocab, hidden, 2, legal, wl.active_tiles(mask_np, vocab), cost)
        md = torch.from_numpy(mask_np).to(dev)
        res = tr.grammar_head(h, w, md, cost=cost)
        got = tr.ROUTES[int(res.route.item())]
        assert got == want, (ks[0], cost, got, want)
        lg = torch.empty(batch, vocab, dtype=dtype, device=dev)
        ti = torch.empty(batch, dtype=torch.int64, device=dev)
        fns[got](h, w, md, logits=lg, top_index=ti)
        assert torch.equal(res.logits, lg) and torch.equal(res.top_index, ti), (ks[0], got)
